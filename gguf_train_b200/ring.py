"""Causal attention over one long sequence split across the GPUs of a box: a ring of K/V shards.

The reference has no multi-device path (its attention runs on the host, csrc/gt_ops_nn.cpp:2423-2525).
For a sequence too long for one GPU's time budget (config 5b: B=1, 32 query heads, 8 kv heads,
L=131072, D=128, causal), the sequence is cut into 2N chunks and rank i of N keeps chunks i and
2N-1-i of q, k and v ("zig-zag"), so that every rank has the same causal work. In N steps every
rank sees every K/V shard: at step s it attends its q chunks to the shard of rank (i - s) mod N
while that shard travels on to rank i + 1 and the next one arrives from rank i - 1 (NCCL
send/receive over NVLink on a side stream, overlapped with the attention). Per (q chunk, kv chunk)
pair the attention is full (kv chunk before the q chunk), causal (the same chunk: top-left causal
with equal lengths), or skipped (kv chunk after). Partial results are merged by log-sum-exp
(gtb_attn_merge) into f32 accumulators.

`ring_step` is the per-rank work of one step; `ring_attention` drives it over a process group and
`ring_attention_emulated` runs all ranks' steps on one GPU (the same arithmetic, no exchange), which
is how a single-GPU test checks the schedule and the merge.
"""

from __future__ import annotations

import ctypes

import torch

from . import _C
from . import functional as Fn


def zigzag_chunks(world: int, rank: int) -> tuple[int, int]:
    """The two chunk indices (of 2 * world) rank `rank` holds."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    return rank, 2 * world - 1 - rank


def shard_zigzag(x: torch.Tensor, world: int, rank: int, dim: int = 2) -> torch.Tensor:
    """This rank's shard of x along `dim`: chunks (rank, 2*world-1-rank) of 2*world equal chunks,
    concatenated (contiguous)."""
    n = x.shape[dim]
    if n % (2 * world):
        raise ValueError(f"sequence length {n} is not a multiple of 2 * world = {2 * world}")
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunks(world, rank)
    return torch.cat([chunks[a], chunks[b]], dim=dim).contiguous()


def unshard_zigzag(shards, dim: int = 2) -> torch.Tensor:
    """Inverse of shard_zigzag over all ranks' shards (in rank order)."""
    world = len(shards)
    chunks = [None] * (2 * world)
    for r, s in enumerate(shards):
        a, b = zigzag_chunks(world, r)
        chunks[a], chunks[b] = s.chunk(2, dim=dim)
    return torch.cat(chunks, dim=dim)


def attend(q, k, v, scale: float, causal: bool):
    """One native forward call: (out, lse) with lse the natural-log sum per query row."""
    return Fn.sdpa_forward(q, k, v, None, scale, causal, need_lse=True)


def merge_(o_acc: torch.Tensor, lse_acc: torch.Tensor, o_part: torch.Tensor, lse_part: torch.Tensor) -> None:
    """o_acc, lse_acc (B, H, R, D) / (B, H, R) f32 contiguous <- merged with a partial result over
    other keys; o_part (B, H, R, D) and lse_part (B, H, R) may be row-range views with unit inner
    strides (e.g. half of a wider result)."""
    B, H, R, D = o_acc.shape
    if o_part.stride(3) != 1 or o_part.stride(2) != D or lse_part.stride(2) != 1:
        raise RuntimeError("attn_merge: partial rows must be contiguous")
    if o_part.stride(0) != H * o_part.stride(1) or lse_part.stride(0) != H * lse_part.stride(1):
        raise RuntimeError("attn_merge: partial batch and head strides must nest")
    rc = _C.lib.gtb_attn_merge(o_acc.data_ptr(), lse_acc.data_ptr(), o_part.data_ptr(), lse_part.data_ptr(),
                               Fn._code(o_part), B * H, R, D, o_part.stride(1), lse_part.stride(1),
                               Fn._stream(o_acc.device))
    _C.check_rc(rc, "attn_merge")


class RingAccumulator:
    """f32 output and log-sum-exp of a rank's two q chunks."""

    def __init__(self, q_shard: torch.Tensor, dv: int):
        B, H, L2, _ = q_shard.shape
        c = L2 // 2
        self.o = torch.zeros((2, B, H, c, dv), dtype=torch.float32, device=q_shard.device)
        self.lse = torch.full((2, B, H, c), float("-inf"), dtype=torch.float32, device=q_shard.device)

    def result(self, dtype) -> torch.Tensor:
        return torch.cat([self.o[0], self.o[1]], dim=2).to(dtype)


def ring_pairs(world: int, rank: int, src: int):
    """(q chunk 0/1, kv chunk 0/1, causal) pairs rank `rank` computes against the shard of `src`."""
    qi = zigzag_chunks(world, rank)
    kj = zigzag_chunks(world, src)
    out = []
    for a in range(2):
        for b in range(2):
            if kj[b] < qi[a]:
                out.append((a, b, False))
            elif kj[b] == qi[a]:
                out.append((a, b, True))
    return out


def ring_step(q_shard, k_shard, v_shard, src: int, rank: int, world: int, acc: RingAccumulator, scale: float,
              attend_fn=attend, merge_fn=merge_) -> int:
    """Attend this rank's q chunks to the K/V shard of rank `src` and merge into `acc`. Returns the
    number of attention calls. Two full pairs that share a q chunk (or a kv chunk) run as one call on
    the whole shard (both shards are chunk a then chunk b, contiguous)."""
    c = q_shard.shape[2] // 2
    ck = k_shard.shape[2] // 2
    qc = (q_shard[:, :, :c], q_shard[:, :, c:])
    kc = (k_shard[:, :, :ck], k_shard[:, :, ck:])
    vc = (v_shard[:, :, :ck], v_shard[:, :, ck:])
    pairs = ring_pairs(world, rank, src)
    full = {(a, b) for a, b, causal in pairs if not causal}
    calls = 0
    done = set()
    # both q chunks against the same kv chunk: one call with the whole q shard
    for b in range(2):
        if (0, b) in full and (1, b) in full:
            o, lse = attend_fn(q_shard, kc[b], vc[b], scale, False)
            for a in range(2):
                merge_fn(acc.o[a], acc.lse[a], o[:, :, a * c:(a + 1) * c], lse[:, :, a * c:(a + 1) * c])
            done |= {(0, b), (1, b)}
            calls += 1
    # one q chunk against both kv chunks: one call with the whole kv shard
    for a in range(2):
        if (a, 0) in full and (a, 1) in full and (a, 0) not in done and (a, 1) not in done:
            o, lse = attend_fn(qc[a], k_shard, v_shard, scale, False)
            merge_fn(acc.o[a], acc.lse[a], o, lse)
            done |= {(a, 0), (a, 1)}
            calls += 1
    for a, b, causal in pairs:
        if (a, b) in done:
            continue
        o, lse = attend_fn(qc[a], kc[b], vc[b], scale, causal)
        merge_fn(acc.o[a], acc.lse[a], o, lse)
        calls += 1
    return calls


def ring_attention(q_shard, k_shard, v_shard, scale: float | None = None, group=None, attend_fn=attend,
                   merge_fn=merge_) -> torch.Tensor:
    """Causal attention of this rank's zig-zag shards (B, H, 2c, D) / (B, Hkv, 2c, D) over the whole
    sequence held by the ranks of `group`. Returns this rank's output shard (B, H, 2c, Dv)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sc = (q_shard.shape[-1] ** -0.5) if scale is None else float(scale)
    acc = RingAccumulator(q_shard, v_shard.shape[-1])
    nxt = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
    prv = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world
    cur_k, cur_v = k_shard.contiguous(), v_shard.contiguous()
    buf_k, buf_v = torch.empty_like(cur_k), torch.empty_like(cur_v)
    on_gpu = cur_k.is_cuda
    comm = torch.cuda.Stream(device=cur_k.device) if on_gpu else None
    for s in range(world):
        src = (rank - s) % world
        reqs = []
        if s < world - 1:
            ops = [dist.P2POp(dist.isend, cur_k, nxt, group), dist.P2POp(dist.isend, cur_v, nxt, group),
                   dist.P2POp(dist.irecv, buf_k, prv, group), dist.P2POp(dist.irecv, buf_v, prv, group)]
            if on_gpu:
                # the exchange waits for the shard to be ready, then runs beside the attention
                comm.wait_stream(torch.cuda.current_stream(cur_k.device))
                with torch.cuda.stream(comm):
                    reqs = dist.batch_isend_irecv(ops)
            else:
                reqs = dist.batch_isend_irecv(ops)
        ring_step(q_shard, cur_k, cur_v, src, rank, world, acc, sc, attend_fn, merge_fn)
        if s < world - 1:
            for r in reqs:
                r.wait()
            if on_gpu:
                torch.cuda.current_stream(cur_k.device).wait_stream(comm)
            cur_k, buf_k = buf_k, cur_k
            cur_v, buf_v = buf_v, cur_v
    return acc.result(q_shard.dtype)


def ring_attention_emulated(q, k, v, world: int, scale: float | None = None) -> torch.Tensor:
    """All ranks of a `world`-rank ring run on q's device, one after the other: the arithmetic of
    ring_attention without the exchange. q (B, H, L, D), k, v (B, Hkv, L, D) are whole sequences;
    returns the whole (B, H, L, Dv) output."""
    sc = (q.shape[-1] ** -0.5) if scale is None else float(scale)
    qs = [shard_zigzag(q, world, r) for r in range(world)]
    ks = [shard_zigzag(k, world, r) for r in range(world)]
    vs = [shard_zigzag(v, world, r) for r in range(world)]
    outs = []
    for r in range(world):
        acc = RingAccumulator(qs[r], v.shape[-1])
        for s in range(world):
            src = (r - s) % world
            ring_step(qs[r], ks[src], vs[src], src, r, world, acc, sc)
        outs.append(acc.result(q.dtype))
    return unshard_zigzag(outs)
