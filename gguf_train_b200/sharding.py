"""Placement of attention work on the GPUs of one box (one process per GPU).

The reference runs attention on the host with OpenMP over (batch, head) pairs
(csrc/gt_ops_nn.cpp:2468) and has no multi-device path. Here the independent units are
(batch, kv head) pairs: a kv head carries its H/Hkv query heads, so dK/dV of a unit never need a
cross-GPU reduction and the forward, backward and decode shard with no collective on the data path.

* prefill / training: contiguous ranges of the B*Hkv units, sizes differing by at most one;
* decode: whole sequences, balanced by cached length (the work is proportional to it) with a
  longest-first greedy assignment.
"""

from __future__ import annotations


def unit_range(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the units rank `rank` of `world` owns: contiguous, sizes differ by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_head_units(B: int, Hkv: int, world: int, rank: int) -> list[tuple[int, int]]:
    """The (batch, kv head) pairs of one rank, in row-major order of (b, hk)."""
    start, stop = unit_range(B * Hkv, world, rank)
    return [(u // Hkv, u % Hkv) for u in range(start, stop)]


def balance_sequences(lengths, world: int) -> list[list[int]]:
    """Assign sequences to ranks so the summed lengths are balanced (longest first, each to the
    currently lightest rank; ties go to the lower rank). Returns per-rank sorted index lists."""
    if world <= 0:
        raise ValueError("world must be positive")
    load = [0] * world
    owned = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owned[r].append(i)
        load[r] += max(int(lengths[i]), 0)
    return [sorted(o) for o in owned]


# ------------------------------------------------------------------ running a rank's share

class Segment(tuple):
    """A rectangle of (batch, kv head) units: batches [b0, b1) x kv heads [hk0, hk1). A rank's
    contiguous unit range is at most three of them (a partial batch, whole batches, a partial batch),
    so it runs as at most three calls of the 4-D kernels, each on views of the global tensors."""

    __slots__ = ()

    def __new__(cls, b0: int, b1: int, hk0: int, hk1: int):
        return super().__new__(cls, (b0, b1, hk0, hk1))

    b0 = property(lambda s: s[0])
    b1 = property(lambda s: s[1])
    hk0 = property(lambda s: s[2])
    hk1 = property(lambda s: s[3])

    @property
    def units(self) -> int:
        return (self.b1 - self.b0) * (self.hk1 - self.hk0)


def segments(B: int, Hkv: int, world: int, rank: int) -> list[Segment]:
    """The rank's unit range (unit_range over the B*Hkv (batch, kv head) units, row-major) as
    rectangles."""
    start, stop = unit_range(B * Hkv, world, rank)
    out, u = [], start
    while u < stop:
        b, hk = divmod(u, Hkv)
        if hk == 0 and stop - u >= Hkv:
            nb = (stop - u) // Hkv
            out.append(Segment(b, b + nb, 0, Hkv))
            u += nb * Hkv
        else:
            hk1 = min(Hkv, hk + (stop - u))
            out.append(Segment(b, b + 1, hk, hk1))
            u += hk1 - hk
    return out


def segment_views(seg: Segment, group: int, *tensors, kv=(False,), base: int = 0):
    """Views of (B, heads, ...) tensors restricted to a segment: query-head tensors (q, out, dO) take
    heads [hk0*group, hk1*group), kv-head tensors (k, v) heads [hk0, hk1). `kv` flags each tensor.
    The tensors' batch index 0 is global batch `base` (a rank may hold only the batches it needs)."""
    flags = list(kv) + [False] * (len(tensors) - len(kv))
    res = []
    for t, is_kv in zip(tensors, flags):
        h0, h1 = (seg.hk0, seg.hk1) if is_kv else (seg.hk0 * group, seg.hk1 * group)
        res.append(t[seg.b0 - base:seg.b1 - base, h0:h1])
    return res


class ShardedAttention:
    """One rank's share of a batched attention over the GPUs of one box.

    The B*Hkv (batch, kv head) units are split into contiguous ranges (unit_range); a kv head carries
    its H/Hkv query heads, so each rank's forward and backward are complete on their own: no
    collective on the data path. The rank is handed global-shaped tensors (only its units need to
    hold data); `forward` / `backward` call the engine once per segment on views and write the
    results straight into views of global-shaped outputs. `gather_to` collects an output on one
    rank afterwards (outside any timed region).

    forward_fn(q, k, v, scale, is_causal, out) -> (out, lse) and backward_fn(dout, q, k, v, out, lse,
    scale, is_causal, grads) -> grads default to the native kernels (gguf_train_b200.functional);
    CPU tests pass stand-ins."""

    def __init__(self, B: int, H: int, Hkv: int, world: int, rank: int, forward_fn=None, backward_fn=None):
        if Hkv <= 0 or H % Hkv:
            raise ValueError("num_heads must be divisible by num_kv_heads")
        self.B, self.H, self.Hkv, self.world, self.rank = B, H, Hkv, world, rank
        self.group = H // Hkv
        self.segs = segments(B, Hkv, world, rank)
        if forward_fn is None or backward_fn is None:
            from . import functional as Fn

            forward_fn = forward_fn or (lambda q, k, v, sc, c, out: Fn.sdpa_forward(q, k, v, None, sc, c, out=out))
            backward_fn = backward_fn or (lambda g, q, k, v, o, l, sc, c, grads:
                                          Fn.sdpa_backward(g, q, k, v, None, o, l, sc, c, grads=grads))
        self._fwd, self._bwd = forward_fn, backward_fn

    @property
    def units(self) -> int:
        return sum(s.units for s in self.segs)

    def batch_span(self) -> tuple[int, int]:
        """[first, last + 1) of the global batches this rank's units touch: the batches a rank has to
        hold (pass tensors covering just these with base = first)."""
        if not self.segs:
            return 0, 0
        return self.segs[0].b0, self.segs[-1].b1

    def forward(self, q, k, v, out, scale: float, is_causal: bool, base: int = 0):
        """Attention of this rank's units: results into the matching views of `out`; returns the
        per-segment log-sum-exp tensors (what backward needs). The tensors cover global batches
        base .. (global shapes with base 0, or batch_span() with base = its first batch)."""
        lses = []
        for seg in self.segs:
            qs, ks, vs, os_ = segment_views(seg, self.group, q, k, v, out, kv=(False, True, True, False), base=base)
            lses.append(self._fwd(qs, ks, vs, scale, is_causal, os_)[1])
        return lses

    def backward(self, dout, q, k, v, out, lses, dq, dk, dv, scale: float, is_causal: bool, base: int = 0):
        """Gradients of this rank's units into the matching views of dq, dk, dv."""
        for seg, lse in zip(self.segs, lses):
            views = segment_views(seg, self.group, dout, q, k, v, out, dq, dk, dv,
                                  kv=(False, False, True, True, False, False, True, True), base=base)
            self._bwd(*views[:5], lse, scale, is_causal, tuple(views[5:]))

    def gather_to(self, t, dst: int = 0, kv: bool = False, group=None):
        """This rank's units of the global-shaped tensor `t` sent to rank `dst`, which fills in every
        other rank's units and gets `t` back (other ranks get None). One send/recv per segment,
        after the computation."""
        import torch.distributed as dist

        if self.world == 1:
            return t
        if self.rank != dst:
            for seg in self.segs:
                (part,) = segment_views(seg, self.group, t, kv=(kv,))
                dist.send(part.contiguous(), dst, group=group)
            return None
        for r in range(self.world):
            if r == dst:
                continue
            for seg in segments(self.B, self.Hkv, self.world, r):
                (part,) = segment_views(seg, self.group, t, kv=(kv,))
                buf = part.contiguous().clone()
                dist.recv(buf, r, group=group)
                part.copy_(buf)
        return t
