"""The Python surface (F.scaled_dot_product_attention, FlashAttentionFn, MultiheadAttention) on
CPU: argument checks and error messages that fire before any kernel, as the reference's tests
exercise them (tests/test_pooling_and_attention.py:303-319, :375-386)."""

from __future__ import annotations

import pytest
import torch


def test_sdpa_mask_shape_errors_before_any_device_work():
    import gguf_train_b200 as gtb

    q, k, v = torch.randn(2, 3, 4, 6), torch.randn(2, 3, 5, 6), torch.randn(2, 3, 5, 6)
    for shape in ((2, 3), (4, 6), (7, 4, 5), (2, 3, 4, 5, 1)):
        with pytest.raises(RuntimeError, match="cannot be broadcast"):
            gtb.scaled_dot_product_attention(q, k, v, attn_mask=torch.ones(*shape, dtype=torch.bool))


def test_sdpa_refuses_cpu_tensors():
    import gguf_train_b200 as gtb

    q = torch.randn(1, 2, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        gtb.scaled_dot_product_attention(q, q, q)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        gtb.FlashAttentionFn.apply(q, q, q, None, 0.4, False)


def test_mha_argument_checks():
    import gguf_train_b200 as gtb

    m = gtb.MultiheadAttention(8, 2, batch_first=True).eval()
    x = torch.randn(3, 4, 8)
    cases = {
        "2D attn_mask": dict(attn_mask=torch.zeros(4, 5)),
        "3D attn_mask": dict(attn_mask=torch.zeros(3, 4, 4)),
        "4D attn_mask": dict(attn_mask=torch.zeros(3, 2, 4, 4)),
        "key_padding_mask": dict(key_padding_mask=torch.zeros(3, 5, dtype=torch.bool)),
        "integer mask": dict(attn_mask=torch.zeros(4, 4, dtype=torch.int64)),
    }
    for name, kwargs in cases.items():
        with pytest.raises(RuntimeError, match="MultiheadAttention"):
            m(x, x, x, **kwargs)
    with pytest.raises(RuntimeError):
        m(x[0], x, x)


def test_mha_parameters_follow_the_reference():
    import gguf_train_b200 as gtb

    m = gtb.MultiheadAttention(512, 8, batch_first=True)
    assert tuple(m.in_proj_weight.shape) == (1536, 512)
    assert float(m.in_proj_bias.detach().abs().max()) == 0.0
    bound = (6.0 / (512 + 1536)) ** 0.5  # Xavier-uniform over the (3E, E) matrix (init.py:105-109)
    assert float(m.in_proj_weight.detach().abs().max()) <= bound
    assert m.head_dim == 64


def test_mha_need_weights_path_refuses_cpu_tensors():
    """need_weights=True runs on the engine's kernels too (the output from the fused forward, the
    weights from its lse), so a CPU input is refused like every other attention call."""
    import gguf_train_b200 as gtb

    torch.manual_seed(0)
    m = gtb.MultiheadAttention(8, 2, batch_first=True).eval()
    x = torch.randn(2, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        m(x, x, x)


def test_q8_0_python_checks():
    import gguf_train_b200 as gtb

    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        gtb.quantize_q8_0(torch.zeros(4, 64))


def test_sdpa_from_host_argument_checks():
    """sdpa_from_host takes host tensors, no mask, and a host `out` of the result's shape; the checks
    fire before any device work."""
    import gguf_train_b200 as gtb

    q = torch.randn(2, 2, 4, 8)
    with pytest.raises(RuntimeError, match="attn_mask is not supported"):
        gtb.sdpa_from_host(q, q, q, attn_mask=torch.ones(4, 4, dtype=torch.bool))
    with pytest.raises(RuntimeError, match="expects 4D"):
        gtb.sdpa_from_host(q[0], q[0], q[0])
    with pytest.raises(RuntimeError, match="out must be"):
        gtb.sdpa_from_host(q, q, q, out=torch.empty(2, 2, 4, 4))
    with pytest.raises(RuntimeError, match="same batch size"):
        gtb.sdpa_from_host(q, q[:1], q[:1])
