"""gtb_decode_q8_0_noalloc, the decode entry point for callers that cannot let a library allocate
device memory (a runtime whose own allocator owns the GPU, or a loop that must not reach cudaMalloc),
checked through the C ABI against the allocating gtb_decode_q8_0 on two calls in a row.

Inputs and outputs are the caller's (torch allocates them here); the entry point itself keeps its
split-KV partials in a fixed device array shared by every call. The second call uses other
sequence lengths and queries, so a result that leaned on the first call's scratch contents would
show up. The file is collected last so that a stop-at-first-failure run has run everything else."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close

pytestmark = pytest.mark.gpu

# Smax spans 3 chunks of GTB_DECODE_CHUNK = 2048 rows, so the split-KV partials in the fixed array
# are used; the lengths below sit on and beside the chunk edges (2047, 2048, 2049, 4096, 4097)
B, H, Hkv, D, SMAX = 3, 8, 2, 128, 4100


def _cache(seed):
    import torch

    O.manual_seed(seed)
    row = D // 32 * 34
    kq = O.q8_0_quantize(O.randn(B, Hkv, SMAX, D).astype(np.float32)).reshape(B, Hkv, SMAX, row)
    vq = O.q8_0_quantize(O.randn(B, Hkv, SMAX, D).astype(np.float32)).reshape(B, Hkv, SMAX, row)
    return torch.tensor(kq).cuda(), torch.tensor(vq).cuda()


def _call(fn, q, kq, vq, lens, out):
    import torch

    from gguf_train_b200 import _C

    rc = fn(q.data_ptr(), _C.GT_F16, kq.data_ptr(), vq.data_ptr(), lens.data_ptr(), B, H, Hkv, SMAX, D, 0.0,
            out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _C.check_rc(rc, "decode")


def test_noalloc_decode_matches_the_allocating_entry_point_twice():
    import torch

    from gguf_train_b200 import _C

    kq, vq = _cache(31)
    for call, (seed, lens) in enumerate(((41, [4100, 2049, 7]), (42, [2047, 2048, 4097]))):
        O.manual_seed(seed)
        q = torch.tensor(O.randn(B, H, 1, D), dtype=torch.float16).cuda()
        lt = torch.tensor(lens, dtype=torch.int32).cuda()
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        _call(_C.lib.gtb_decode_q8_0, q, kq, vq, lt, want)
        _call(_C.lib.gtb_decode_q8_0_noalloc, q, kq, vq, lt, got)
        torch.cuda.synchronize()
        # gtb_device_status reads and clears this entry point's own status word too: 0 means none of
        # its bounded waits ran out and none of its copies was refused
        assert _C.device_status() == 0
        assert_close(got, want.double().cpu().numpy(), 2e-2, 1e-2, f"no-alloc decode, call {call + 1}")


def test_noalloc_decode_rejects_calls_beyond_its_scratch():
    import torch

    from gguf_train_b200 import _C

    q = torch.zeros((1, 8, 1, D), dtype=torch.float16, device="cuda")
    lens = torch.zeros((1,), dtype=torch.int32, device="cuda")
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    # 512 sequences x 8 kv heads x 32 chunks x 4 heads x 130 floats = 272 MB of partials: refused
    # before any kernel runs (the buffers are never read)
    rc = _C.lib.gtb_decode_q8_0_noalloc(q.data_ptr(), _C.GT_F16, dummy.data_ptr(), dummy.data_ptr(),
                                        lens.data_ptr(), 512, 32, 8, 32768, D, 0.0, q.data_ptr(),
                                        ctypes.c_void_p(0))
    assert rc != 0
    assert "bytes of scratch" in _C.lib.gtb_last_error().decode()
