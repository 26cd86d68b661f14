"""Multi-GPU placement on CPU: the unit partitioning and the decode balancing, and a world-size-2
gloo run in which each rank computes its own (batch, kv head) units (the CPU oracle stands in for
the kernels) and the gathered shards equal the unsharded result -- no data-path collective is needed
because the units are independent."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from gguf_train_b200 import sharding


def test_unit_ranges_cover_every_unit_once():
    for n in (0, 1, 7, 64):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                a, b = sharding.unit_range(n, world, r)
                assert 0 <= a <= b <= n
                seen.extend(range(a, b))
            assert seen == list(range(n))
            sizes = [np.subtract(*sharding.unit_range(n, world, r)[::-1]) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_batch_head_units():
    assert sharding.batch_head_units(2, 2, 3, 0) == [(0, 0), (0, 1)]
    assert sharding.batch_head_units(2, 2, 3, 2) == [(1, 1)]


def test_decode_balance_by_length():
    lens = [32768, 1024, 1024, 16000, 16000, 1024, 1024, 30000]
    owned = sharding.balance_sequences(lens, 2)
    assert sorted(owned[0] + owned[1]) == list(range(len(lens)))
    loads = [sum(lens[i] for i in o) for o in owned]
    assert abs(loads[0] - loads[1]) <= max(lens)
    with pytest.raises(ValueError):
        sharding.balance_sequences(lens, 0)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, k, v, ret):
    import torch.distributed as dist

    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    B, H, L, D = q.shape
    Hkv = k.shape[1]
    g = H // Hkv
    local = np.zeros_like(q)
    for b, hk in sharding.batch_head_units(B, Hkv, world, rank):
        sl = slice(hk * g, (hk + 1) * g)
        local[b:b + 1, sl] = O.sdpa_fwd(q[b:b + 1, sl], k[b:b + 1, hk:hk + 1], v[b:b + 1, hk:hk + 1], is_causal=True)
    parts = [torch.zeros(q.shape, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(parts, torch.tensor(local))  # result gathering for the check, not the data path
    if rank == 0:
        ret.put(sum(p.numpy() for p in parts))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_reassemble_the_full_result():
    import torch.multiprocessing as mp

    from oracle import oracle as O

    O.manual_seed(5)
    q, k, v = O.randn(2, 4, 24, 8), O.randn(2, 2, 24, 8), O.randn(2, 2, 24, 8)
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.abs(got - O.sdpa_fwd(q, k, v, is_causal=True)).max() < 1e-12


def test_segments_cover_the_units_in_at_most_three_rectangles():
    for B, Hkv in ((8, 8), (4, 8), (3, 5), (1, 8), (2, 1)):
        for world in (1, 2, 3, 4, 5, 8):
            seen = []
            for r in range(world):
                segs = sharding.segments(B, Hkv, world, r)
                assert len(segs) <= 3
                for s in segs:
                    assert 0 <= s.b0 < s.b1 <= B and 0 <= s.hk0 < s.hk1 <= Hkv
                    assert s.b1 - s.b0 == 1 or (s.hk0, s.hk1) == (0, Hkv)
                    seen += [(b, hk) for b in range(s.b0, s.b1) for hk in range(s.hk0, s.hk1)]
                assert sum(s.units for s in segs) == len(sharding.batch_head_units(B, Hkv, world, r))
            assert sorted(seen) == [(b, hk) for b in range(B) for hk in range(Hkv)]


def _stand_ins():
    """CPU stand-ins for the native forward / backward, with the engine's call shapes (results
    written into the given views)."""
    import torch

    from oracle import oracle as O

    def fwd(q, k, v, scale, causal, out):
        out.copy_(torch.tensor(O.sdpa_fwd(q.numpy(), k.numpy(), v.numpy(), scale=scale, is_causal=causal)))
        return out, None

    def bwd(g, q, k, v, o, lse, scale, causal, grads):
        res = O.sdpa_bwd(q.numpy(), k.numpy(), v.numpy(), g.numpy(), scale=scale, is_causal=causal)
        for dst, src in zip(grads, res):
            dst.copy_(torch.tensor(src))
        return grads

    return fwd, bwd


def _sharded_worker(rank, world, port, q, k, v, g, ret):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, H = q.shape[:2]
    Hkv = k.shape[1]
    fwd, bwd = _stand_ins()
    sa = sharding.ShardedAttention(B, H, Hkv, world, rank, forward_fn=fwd, backward_fn=bwd)
    tq, tk, tv, tg = (torch.tensor(x) for x in (q, k, v, g))
    out = torch.zeros_like(tq)
    lses = sa.forward(tq, tk, tv, out, 0.35, True)
    dq, dk, dv = torch.zeros_like(tq), torch.zeros_like(tk), torch.zeros_like(tv)
    sa.backward(tg, tq, tk, tv, out, lses, dq, dk, dv, 0.35, True)
    full = [sa.gather_to(out), sa.gather_to(dq), sa.gather_to(dk, kv=True), sa.gather_to(dv, kv=True)]
    if rank == 0:
        ret.put([t.numpy() for t in full])
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_attention_reassembles_forward_and_gradients(world):
    """ShardedAttention on gloo ranks: each rank computes only its (batch, kv head) segments (no
    collective while computing), gather_to collects them on rank 0 afterwards, and the result equals
    the unsharded forward and backward."""
    import torch.multiprocessing as mp

    from oracle import oracle as O

    O.manual_seed(17)
    B, H, Hkv, L, D = 3, 4, 2, 20, 8  # 6 units: with 2 ranks each holds one whole and one partial batch
    q, k, v, g = O.randn(B, H, L, D), O.randn(B, Hkv, L, D), O.randn(B, Hkv, L, D), O.randn(B, H, L, D)
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, q, k, v, g, ret)) for r in range(world)]
    for p in procs:
        p.start()
    got = ret.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [O.sdpa_fwd(q, k, v, scale=0.35, is_causal=True)] + list(O.sdpa_bwd(q, k, v, g, scale=0.35, is_causal=True))
    for a, b in zip(got, want):
        assert np.abs(a - b).max() < 1e-12
