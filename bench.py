"""Benchmark of the B200 attention engine: causal GQA prefill.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (one "step"): one causal GQA attention forward over a batch of B=8 sequences,
Hq=32, Hkv=8, L=S=4096, D=128, bf16, inputs N(0,1)*0.5 (seeded, generated on the device),
scale 1/sqrt(128). Work per step: 4*B*Hq*(L(L+1)/2)*D = 1.0998e12 FLOP.

Multi-GPU: one process per GPU (torchrun). The (batch, kv head) units are independent, so a global
batch is partitioned over the ranks by gguf_train_b200.sharding.ShardedAttention (contiguous unit
ranges, no collective on the data path). The default line is weak scaling: a global batch of
N x 8 sequences, each rank getting config 3's 64 units. `extra` adds strong-scaling lines (the fixed
config-3 / config-4 batches and config 5a's 64 sequences split over the N ranks). The process
group is used only for barriers and the max-over-ranks of the timed regions.

Reported on one JSON line by rank 0:
  value        whole-job TFLOP/s with inputs resident in HBM (CUDA events on the launching
               stream, K steps between barriers + synchronize, max over ranks);
  e2e          the same through the public API (gguf_train_b200.sdpa_from_host, i.e. the C ABI's
               gtb_sdpa_fwd_host) with the inputs copied from pinned host memory and the output
               copied back inside every timed step (pieces of the batch, the copies overlapped with
               the kernels);
  roofline     the tcgen05 forward kernel against the measured bf16 dense peak;
  cpu_baseline the reference's CPU forward (restated loop, float64, OpenMP on every host
               core) on a bounded sample of the same workload, rank 0 at N=1 only;
  clocks       SM clocks and throttle reasons sampled through NVML during the timed region.
`--impl reference` times that CPU forward alone (rank 0; other ranks exit at once).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "SDPA TFLOP/s (fwd, fwd+bwd) & decode KV GB/s, % of B200 peak, 1/2/4/8 GPUs"
CFG = dict(B=8, H=32, Hkv=8, L=4096, D=128)
WORKLOAD = "config 3: causal GQA prefill forward, bf16, B=8 Hq=32 Hkv=8 L=S=4096 D=128"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "bf16_tflops_sustained": 1400.0}


def fwd_flops(B, H, L, D, causal=True):
    pairs = L * (L + 1) / 2 if causal else L * L
    return 4.0 * B * H * pairs * D


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": float(p["bf16_tflops"]), "hbm_gbs": float(p["hbm_gbs"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "source": "measured"}
    except Exception:
        return dict(FALLBACK_PEAKS, source="fallback")


def profile_traffic(name: str, kernel: str = ""):
    """DRAM bytes per launch recorded in the committed ncu summary profiles/<name>.md
    (a line 'traffic_bytes_per_launch: N', or 'traffic_bytes_per_launch (kernel): N'), or None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    tag = r"\s*\(" + re.escape(kernel) + r"\)" if kernel else ""
    try:
        with open(path) as f:
            m = re.search(r"traffic_bytes_per_launch" + tag + r":\s*([0-9.eE+]+)", f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


# ------------------------------------------------------------------ CPU baseline (reference arm)

def _host_threads() -> int:
    """Every host core this process may run on (torchrun sets OMP_NUM_THREADS=1 for its ranks, so the
    thread counts below are set explicitly)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def cpu_sample_reference(reps: int = 1, rows: int = 256):
    """The reference's own gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525, compiled from its source
    into oracle/_ref with its OpenMP loop over (batch, head)) on a bounded sample of the workload: one
    (batch, head) unit per host thread, a unit being `rows` query rows against all L keys of a GQA
    kv head, bf16 storage as in the workload. The reference aligns causal masking top-left, so the
    sample runs unmasked: the last query rows of the causal workload see all but a few of their keys,
    so this is their work. Returns (TFLOP/s, threads, description), or None when oracle/_ref is absent."""
    import ctypes

    import numpy as np

    from oracle import oracle as O
    from oracle import ref as R

    if not R.available():
        return None
    lib = R.lib()
    threads = _host_threads()
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(threads)
    except OSError:
        pass
    L, D, H = CFG["L"], CFG["D"], threads
    rng = np.random.default_rng(0)
    q = np.ascontiguousarray(O.to_bits(rng.standard_normal((1, H, rows, D)) * 0.5, O.BF16))
    k = np.ascontiguousarray(O.to_bits(rng.standard_normal((1, 1, L, D)) * 0.5, O.BF16))
    v = np.ascontiguousarray(O.to_bits(rng.standard_normal((1, 1, L, D)) * 0.5, O.BF16))
    out = np.zeros((1, H, rows, D), dtype=np.uint16)
    scale = 1.0 / math.sqrt(D)

    def call(nh):
        rc = lib.ref_flash_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, int(O.BF16), 1, nh, rows, D, 1, L, D,
                                     None, 0, 0, None, scale, 0, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(lib.ref_last_error().decode())

    call(1)  # warm the pages and the OpenMP pool
    t0 = time.perf_counter()
    for _ in range(reps):
        call(H)
    dt = (time.perf_counter() - t0) / reps
    flops = 4.0 * H * rows * L * D
    desc = (f"the reference's gt_flash_attention (oracle/_ref, compiled from its source): {threads} (batch, head) "
            f"units per step, each {rows} query rows against all {L} keys (D={D}, bf16 storage, double "
            f"arithmetic), one unit per OpenMP thread")
    return flops / dt / 1e12, threads, desc


def cpu_sample_port(reps: int = 1, rows: int = 256):
    """The reference's CPU forward restated in oracle/ (gt_flash_attention's loop in float64 with
    OpenMP over heads) on a bounded sample of the workload: one unit per host thread, a unit being
    the last `rows` query rows of one (batch, head) against all their keys (causal).
    Returns (TFLOP/s, threads, description)."""
    import numpy as np

    from oracle import oracle as O

    threads = _host_threads()
    L, D, H = CFG["L"], CFG["D"], threads
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, H, rows, D)) * 0.5
    k = rng.standard_normal((1, 1, L, D)) * 0.5
    v = rng.standard_normal((1, 1, L, D)) * 0.5
    out = np.zeros((1, H, rows, D))
    off = L - rows
    flops = 4.0 * H * D * sum(l + 1 for l in range(off, L))
    O.sdpa_fwd_reforder(q[:, :1, :8], k, v, 1.0 / math.sqrt(D), True, threads, off + rows - 8)  # warm the pages
    t0 = time.perf_counter()
    for _ in range(reps):
        O.sdpa_fwd_reforder(q, k, v, 1.0 / math.sqrt(D), True, threads, off, out)
    dt = (time.perf_counter() - t0) / reps
    desc = (f"{threads} units per step, each the last {rows} query rows of one (batch, head) of the workload "
            f"against all their keys (L=4096, D=128, causal), float64, one unit per OpenMP thread")
    return flops / dt / 1e12, threads, desc


def cpu_sample(reps: int = 1):
    """The CPU baseline: the reference's own loop from oracle/_ref where it was built (kind
    "reference"), else the restatement (kind "port"). Returns (TFLOP/s, threads, description, kind)."""
    r = cpu_sample_reference(reps)
    if r is not None:
        return (*r, "reference")
    return (*cpu_sample_port(reps), "port")


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    vals, times = [], []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        v, threads, desc, kind = cpu_sample(1)
        if i >= args.warmup:
            vals.append(v)
            times.append((time.perf_counter() - t0) * 1e3)
    value = statistics.mean(vals)
    cfg = {"workload": WORKLOAD, "global_batch": CFG["B"] * args.gpus, "seq_len": CFG["L"],
           "parallelism": f"replicas x{args.gpus}",
           "kernel": ("the reference's gt_flash_attention loop (compiled from its source)" if kind == "reference"
                      else "reference CPU loop (restated)")}
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded normal)",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons of one GPU through NVML (read-only)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self._stop = [], 0, threading.Event()
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                self.reasons |= self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._nv:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self._nv or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ------------------------------------------------------------------ decode workload (config 5a)

DEC = dict(B=64, H=32, Hkv=8, D=128, Smax=32768, Lmin=1024)


def run_decode(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 5a: one decode step of B=64 sequences (Hq=32, Hkv=8, D=128) against Q8_0 K/V caches
    with lengths uniform in [1024, 32768]; q fp16. Metric: cache bytes read per second (HBM-bound)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    B, H, Hkv, D, Smax = DEC["B"], DEC["H"], DEC["Hkv"], DEC["D"], DEC["Smax"]
    if getattr(args, "decode_batch", None):
        B = args.decode_batch  # smaller case of the same kernel (profiling); the workload line says so
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    lens = torch.randint(DEC["Lmin"], Smax + 1, (B,), generator=g, device=dev).to(torch.int32)
    row = D // 32 * 34
    kq = torch.empty((B, Hkv, Smax, row), dtype=torch.uint8, device=dev)
    vq = torch.empty_like(kq)
    for b in range(B):  # N(0,1) values quantised to Q8_0 by the engine's own quantiser
        kq[b] = gtb.quantize_q8_0(torch.randn((Hkv, Smax, D), generator=g, device=dev))
        vq[b] = gtb.quantize_q8_0(torch.randn((Hkv, Smax, D), generator=g, device=dev))
    q = torch.randn((B, H, 1, D), generator=g, device=dev).to(torch.float16)
    tokens = int(lens.sum().item())
    nbytes = tokens * Hkv * 2 * row + q.numel() * 2 * 2
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > L2: every step reads from HBM
    for _ in range(max(args.warmup, 3)):
        gtb.decode_q8_0(q, kq, vq, lens)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    times = []
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler:
        for _ in range(args.steps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            gtb.decode_q8_0(q, kq, vq, lens)
            e.record(stream)
            torch.cuda.synchronize(dev)
            times.append(s.elapsed_time(e))
    ms = max_over_ranks(statistics.mean(times))
    peaks = load_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": gbs * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q8_0 K/V, f16 q", "data": "synthetic: N(0,1) K/V quantised to Q8_0",
        "config": {"workload": f"config 5a: Q8_0-KV decode, B={B} Hq=32 Hkv=8 D=128, L_b ~ U[1024, 32768]",
                   "tokens": tokens, "bytes_per_step": nbytes, "l2": "256 MB flush before every step"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": profile_traffic("decode_q8_0_config5a"),
                     "peak_source": peaks["source"] + " HBM copy"},
        # per step: decode_mma_kernel and the split-KV combine (after a 4-byte memset of the claim
        # counter); above 256 sequences a plan kernel runs first
        "gpu_launches": (2 if B <= 256 else 3) * args.steps,
        "clocks": sampler.summary(), "status": _C.device_status(),
    }
    del kq, vq, flush
    torch.cuda.empty_cache()
    return line


# ------------------------------------------------------------------ training workload (config 4)

TRAIN = dict(B=4, H=32, Hkv=8, L=8192, D=128)


def run_train(args, rank: int, world: int, dev, max_over_ranks=lambda x: x, strong: bool = False) -> dict:
    """Config 4: causal GQA attention forward + backward, bf16, B=4 Hq=32 Hkv=8 L=S=8192 D=128,
    q/k/v N(0,1)*0.5 and upstream gradient N(0,1). Work per step: forward 4*B*Hq*L(L+1)/2*D FLOP and
    backward twice that (the 4-GEMM convention; the kernels recompute S and dP, which is not credited).
    The (batch, kv head) units are partitioned by sharding.ShardedAttention: weak scaling (a global
    batch of N x 4, each rank config 4's 32 units) or, with `strong`, config 4's batch of 4 split over
    the N ranks."""
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200.sharding import ShardedAttention

    B, H, Hkv, L, D = TRAIN["B"], TRAIN["H"], TRAIN["Hkv"], TRAIN["L"], TRAIN["D"]
    B_glob = B if strong else B * world
    sa = ShardedAttention(B_glob, H, Hkv, world, rank)
    b_lo, b_hi = sa.batch_span()
    nb = b_hi - b_lo
    g = torch.Generator(device=dev)
    g.manual_seed(4321 if strong else 4321 + rank)
    if strong:  # the same global batch on every rank; each keeps the batches its units touch
        sl = lambda t: t[b_lo:b_hi].contiguous()  # noqa: E731
    else:
        sl = lambda t: t  # noqa: E731
    nq = B if strong else nb
    q = sl((torch.randn((nq, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16))
    k = sl((torch.randn((nq, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16))
    v = sl((torch.randn((nq, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16))
    gd = sl(torch.randn((nq, H, L, D), generator=g, device=dev).to(torch.bfloat16))
    out = torch.empty_like(q)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    scale = 1.0 / math.sqrt(D)
    fwd = fwd_flops(B, H, L, D)  # config 4's batch: one rank's share (weak) or the whole split batch (strong)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        lse = sa.forward(q, k, v, out, scale, True, base=b_lo)
        sa.backward(gd, q, k, v, out, lse, dq, dk, dv, scale, True, base=b_lo)
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 20))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        ev[i][0].record(stream)
        lse = sa.forward(q, k, v, out, scale, True, base=b_lo)
        ev[i][1].record(stream)
        sa.backward(gd, q, k, v, out, lse, dq, dk, dv, scale, True, base=b_lo)
        ev[i][2].record(stream)
    torch.cuda.synchronize(dev)
    f_ms = max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in ev))
    b_ms = max_over_ranks(statistics.mean(e[1].elapsed_time(e[2]) for e in ev))
    peaks = load_peaks()
    tf = 3 * fwd / ((f_ms + b_ms) * 1e-3) / 1e12  # strong: the whole batch's rate; weak: one rank's
    per_gpu = tf / world if strong else tf
    line = {
        "workload": ("config 4 fixed batch (B=4, 32 units) split over the ranks" if strong else
                     "config 4: causal GQA forward+backward, bf16, B=4 Hq=32 Hkv=8 L=S=8192 D=128"),
        "value": tf if strong else tf * world, "unit": "TFLOP/s", "ms_per_step": f_ms + b_ms, "fwd_ms": f_ms,
        "bwd_ms": b_ms, "scaling": "strong" if strong else "weak", "units_this_rank": sa.units,
        "flops_per_step": 3 * fwd,
        # the timed region is `steps` forward+backward pairs of a few ms each (well under a second of
        # back-to-back work), so the burst peak is the denominator
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s per GPU",
                     "frac": per_gpu / peaks["bf16_tflops"],
                     "peak_source": peaks["source"] + " bf16 dense (burst)",
                     "timed_ms": steps * (f_ms + b_ms),
                     # per GPU: a strong-scaling rank ran 1/N of the batch's FLOPs in these times
                     "backward_tflops": 2 * fwd / (b_ms * 1e-3) / 1e12 / (world if strong else 1),
                     "forward_tflops": fwd / (f_ms * 1e-3) / 1e12 / (world if strong else 1),
                     "backward_frac": 2 * fwd / (b_ms * 1e-3) / 1e12 / (world if strong else 1) / peaks["bf16_tflops"]},
        "launches_per_step": "forward 1, backward 3 (preprocess, dK/dV with the dQ sums, dQ conversion)",
        "gpu_launches": 4 * steps, "status": _C.device_status(),
    }
    line["roofline"]["traffic_bwd_dkdv"] = profile_traffic("bwd_sm100_config4", "dkdv")
    line["roofline"]["traffic_bwd_dq_convert"] = profile_traffic("bwd_sm100_config4", "dq_convert")
    del q, k, v, gd, out, lse, dq, dk, dv
    torch.cuda.empty_cache()
    return line


# ------------------------------------------------------------------ strong scaling and masked workloads

def _time_events(stream, fn, steps: int) -> float:
    """Mean ms of fn() over `steps` launches, CUDA events on `stream` around each."""
    import torch

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s, e in ev:
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    return statistics.mean(s.elapsed_time(e) for s, e in ev)


def run_prefill_strong(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 3's fixed batch (B=8, 64 (batch, kv head) units) split over the ranks by
    sharding.ShardedAttention: each rank runs 64/N units; TFLOP/s of the whole batch over the
    slowest rank's time (strong scaling)."""
    import torch

    from gguf_train_b200.sharding import ShardedAttention

    B, H, Hkv, L, D = CFG["B"], CFG["H"], CFG["Hkv"], CFG["L"], CFG["D"]
    sa = ShardedAttention(B, H, Hkv, world, rank)
    b_lo, b_hi = sa.batch_span()
    g = torch.Generator(device=dev)
    g.manual_seed(555)  # the same global batch on every rank; each keeps the batches its units touch
    q = (torch.randn((B, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)[b_lo:b_hi].contiguous()
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)[b_lo:b_hi].contiguous()
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)[b_lo:b_hi].contiguous()
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)
    step = lambda: sa.forward(q, k, v, out, scale, True, base=b_lo)  # noqa: E731
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 20))
    ms = max_over_ranks(_time_events(torch.cuda.current_stream(dev), step, steps))
    flops = fwd_flops(B, H, L, D)
    return {"workload": "config 3 fixed batch (B=8, 64 units) split over the ranks", "value": flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps, "scaling": "strong",
            "units_this_rank": sa.units, "segments_rank0": [list(x) for x in sa.segs] if rank == 0 else None}


def run_prefill_key_padding(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 3 with a key-padding mask, the mask nn.TransformerEncoderLayer passes for padded batches:
    a bool (B, 1, 1, S) mask in which sequence b may not attend its last n_b ~ U{0..64} keys, on the
    tcgen05 kernel (the mask's 128 x 128 blocks classified first; only blocks holding padded keys
    are read entry by entry). Reported against the unmasked forward on the same inputs."""
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    B, H, Hkv, L, D = CFG["B"], CFG["H"], CFG["Hkv"], CFG["L"], CFG["D"]
    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)
    q = (torch.randn((B, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    pad = torch.randint(0, 65, (B,), generator=g, device=dev)
    mask = (torch.arange(L, device=dev)[None, :] < (L - pad)[:, None]).view(B, 1, 1, L)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)
    masked = lambda: Fn.sdpa_forward(q, k, v, mask, scale, True, need_lse=False, out=out)  # noqa: E731
    plain = lambda: Fn.sdpa_forward(q, k, v, None, scale, True, need_lse=False, out=out)  # noqa: E731
    for _ in range(max(args.warmup, 3)):
        masked()
        plain()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 20))
    stream = torch.cuda.current_stream(dev)
    ms_m = max_over_ranks(_time_events(stream, masked, steps))
    path = _C.last_path()
    ms_p = max_over_ranks(_time_events(stream, plain, steps))
    flops = fwd_flops(B, H, L, D)
    peaks = load_peaks()
    tf = flops / (ms_m * 1e-3) / 1e12
    return {"workload": "config 3 + key-padding mask (B,1,1,S) bool, last U{0..64} keys of each sequence masked",
            "value": tf * world, "unit": "TFLOP/s", "ms_per_step": ms_m, "steps": steps, "kernel": path,
            "unmasked_ms": ms_p, "fraction_of_unmasked": ms_p / ms_m,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "peak_source": peaks["source"] + " bf16 dense (burst)"},
            "status": _C.device_status()}


MHA = dict(B=16, E=512, H=8, L=512)


def run_mha(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 2: nn.MultiheadAttention, fp32, E=512, 8 heads, batch_first, B=16, L=512, an additive
    float attn_mask with -inf at ~10% of the positions plus a key_padding_mask of the last U{0..64}
    tokens, need_weights=False; forward + backward of the module (projections and attention) per
    step. The attention itself (the engine's fp32 path: the SIMT kernels; a single-pass tf32
    tensor-core product misses the 1e-3 tolerance) is also timed alone on the module's q, k, v and
    merged mask. FLOPs: attention 4*B*H*L*S*D forward, twice that backward; projections 2*B*L*E*E per
    linear, 4 linears forward, twice that backward."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    B, E, H, L = MHA["B"], MHA["E"], MHA["H"], MHA["L"]
    D = E // H
    torch.manual_seed(2 + rank)
    m = gtb.MultiheadAttention(E, H, batch_first=True, device=dev)
    x = torch.randn((B, L, E), device=dev, requires_grad=True)
    am = torch.where(torch.rand((L, L), device=dev) < 0.1, float("-inf"), 0.0)
    am[:, 0] = 0.0
    n_pad = torch.randint(0, 65, (B,), device=dev)
    kpm = torch.arange(L, device=dev)[None, :] >= (L - n_pad)[:, None]
    gy = torch.randn((B, L, E), device=dev)

    def module_step():
        y, _ = m(x, x, x, key_padding_mask=kpm, need_weights=False, attn_mask=am)
        y.backward(gy)

    with torch.no_grad():
        qkv = torch.nn.functional.linear(x, m.in_proj_weight, m.in_proj_bias)
        q, k, v = qkv.view(B, L, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
        bias = m._score_bias(am, kpm, B, L, L, q.dtype)
    go = torch.randn_like(q)

    def attention_step():
        o, lse = Fn.sdpa_forward(q, k, v, bias, D ** -0.5, False)
        Fn.sdpa_backward(go, q, k, v, bias, o, lse, D ** -0.5, False)

    for _ in range(max(args.warmup, 3)):
        module_step()
        attention_step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 20))
    stream = torch.cuda.current_stream(dev)
    ms_mod = max_over_ranks(_time_events(stream, module_step, steps))
    ms_att = max_over_ranks(_time_events(stream, attention_step, steps))
    path = _C.last_path()
    att_flops = 3 * 4.0 * B * H * L * L * D
    proj_flops = 3 * 4 * 2.0 * B * L * E * E
    return {"workload": "config 2: nn.MultiheadAttention fp32 E=512 H=8 B=16 L=512, float mask (-inf ~10%) + "
                        "key_padding_mask, forward + backward",
            "value": (att_flops + proj_flops) * world / (ms_mod * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms_mod, "steps": steps,
            "attention_ms": ms_att, "attention_tflops": att_flops / (ms_att * 1e-3) / 1e12, "attention_kernel": path,
            "flops_per_step": {"attention": att_flops, "projections": proj_flops}, "dtype": "f32",
            "status": _C.device_status()}


def run_linear(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """The tensor-core linear layer (gtb_linear: c = a b^T + bias, bf16, f32 accumulation) on
    MultiheadAttention's bf16 in-projection at config 2's token count (M = 16 x 512 tokens, N = 3 x 512,
    K = 512) and on a large square product (8192^3); torch.matmul (cuBLAS) on the same operands is timed
    beside it for reference. FLOPs 2 M N K per call."""
    import torch

    from gguf_train_b200 import functional as Fn

    peaks = load_peaks()
    res = {"workload": "tcgen05 linear (gtb_linear), bf16", "unit": "TFLOP/s", "shapes": []}
    g = torch.Generator(device=dev)
    g.manual_seed(5 + rank)
    for M, N, K in ((8192, 1536, 512), (8192, 8192, 8192)):
        a = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        b = (torch.randn((N, K), generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
        bias = torch.randn((N,), generator=g, device=dev).to(torch.bfloat16)
        ours = lambda: Fn._linear_2d(a, b, bias)  # noqa: E731
        lib = lambda: torch.addmm(bias, a, b.t())  # noqa: E731
        for _ in range(max(args.warmup, 3)):
            ours()
            lib()
        torch.cuda.synchronize(dev)
        steps = max(3, min(args.steps, 20))
        stream = torch.cuda.current_stream(dev)
        ms = max_over_ranks(_time_events(stream, ours, steps))
        ms_lib = max_over_ranks(_time_events(stream, lib, steps))
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        res["shapes"].append({"M": M, "N": N, "K": K, "ms": ms, "tflops": tf, "frac": tf / peaks["bf16_tflops"],
                              "cublas_ms": ms_lib, "cublas_tflops": 2.0 * M * N * K / (ms_lib * 1e-3) / 1e12})
        del a, b, bias
    res["value"] = res["shapes"][-1]["tflops"] * world
    res["roofline"] = {"bound": "tensor", "achieved": res["shapes"][-1]["tflops"], "peak": peaks["bf16_tflops"],
                       "unit": "TFLOP/s", "frac": res["shapes"][-1]["frac"],
                       "peak_source": peaks["source"] + " bf16 dense (burst)"}
    torch.cuda.empty_cache()
    return res


def run_weights(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """MultiheadAttention's need_weights output at config 3's shape (bf16, B=8, Hq=32, Hkv=8, L=4096,
    D=128, causal): the head-averaged weights (B, L, S) formed by the tcgen05 weights kernel from the
    forward's lse (functional.attention_weights). Per (head, query, key) of the causal triangle the
    kernel does a 2*D-FLOP product on the tensor cores and one exponential on the MUFU unit (16 a clock
    per SM); both rates are reported, the exponentials against the MUFU's nominal rate at the sampled
    clock. The forward that produces lse runs once, outside the timed region; the output (268 MB) is
    larger than L2 and rewritten by every launch."""
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    H, Hkv, L, D = CFG["H"], CFG["Hkv"], CFG["L"], CFG["D"]
    B = args.weights_batch or CFG["B"]
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    q = (torch.randn((B, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    _, lse = Fn.sdpa_forward(q, k, v, None, scale, True)
    step = lambda: Fn.attention_weights(q, k, lse, None, scale, True, True)  # noqa: E731
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(10, min(args.steps, 50))
    with ClockSampler(torch.cuda.current_device()) as sampler:
        ms = max_over_ranks(_time_events(torch.cuda.current_stream(dev), step, steps))
    clocks = sampler.summary()
    pairs = B * H * L * (L + 1) / 2  # (head, query, key) triples of the causal triangle
    tf = 2.0 * D * pairs / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    mhz = clocks.get("sm_mhz") or 1965.0
    mufu_peak = 16 * 148 * mhz * 1e6  # exponentials a second
    exps = pairs / (ms * 1e-3)
    del q, k, v, lse
    torch.cuda.empty_cache()
    return {"workload": f"need_weights at config 3's shape (B={B}): head-averaged attention weights (B, L, S) "
                        "from the forward's lse, bf16, causal", "value": tf * world, "unit": "TFLOP/s", "ms_per_step": ms,
            "steps": steps, "scaling": "weak",
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "peak_source": peaks["source"] + " bf16 dense (burst)"},
            "mufu": {"exps_per_s": exps, "nominal_per_s": mufu_peak, "frac": exps / mufu_peak,
                     "note": "16 exponentials a clock per SM x 148 SMs at the median sampled SM clock"},
            "clocks": clocks, "status": _C.device_status()}


def run_rope_prefill(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 3 preceded by RoPE on q and k (n_dims = 128, normal pairs, freq_base 10^4, positions
    0..L-1), the llama-style prefill: gtb_sdpa_fwd_rope (q rotated inside the tcgen05 kernel, k once
    into k_rot) against rope() on q and k followed by the forward, on the same inputs. FLOPs: the
    attention's (4 D per causal pair)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    B, H, Hkv, L, D = CFG["B"], CFG["H"], CFG["Hkv"], CFG["L"], CFG["D"]
    g = torch.Generator(device=dev)
    g.manual_seed(31 + rank)
    q = (torch.randn((B, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    pos = torch.arange(L, dtype=torch.int32, device=dev)
    scale = 1.0 / math.sqrt(D)
    fused = lambda: Fn.sdpa_forward_rope(q, k, v, pos, D, 0, 10000.0, 1.0, scale=scale, is_causal=True,  # noqa: E731
                                         need_lse=False)
    in_kernel = lambda: Fn.sdpa_forward_rope(q, k, v, pos, D, 0, 10000.0, 1.0, scale=scale,  # noqa: E731
                                             is_causal=True, need_lse=False, q_in_kernel=True)

    def unfused():
        qr = gtb.rope(q, pos, D, 0, 0, 10000.0, 1.0)
        kr = gtb.rope(k, pos, D, 0, 0, 10000.0, 1.0)
        return Fn.sdpa_forward(qr, kr, v, None, scale, True, need_lse=False)

    for _ in range(max(args.warmup, 3)):
        fused()
        in_kernel()
        unfused()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 20))
    stream = torch.cuda.current_stream(dev)
    ms_f = max_over_ranks(_time_events(stream, fused, steps))
    path = _C.last_path()
    ms_k = max_over_ranks(_time_events(stream, in_kernel, steps))
    ms_u = max_over_ranks(_time_events(stream, unfused, steps))
    flops = fwd_flops(B, H, L, D)
    peaks = load_peaks()
    tf = flops / (ms_f * 1e-3) / 1e12
    del q, k, v
    torch.cuda.empty_cache()
    return {"workload": "config 3 with RoPE on q and k first (n_dims 128, normal pairs, positions 0..L-1): "
                        "gtb_sdpa_fwd_rope", "value": tf * world, "unit": "TFLOP/s", "ms_per_step": ms_f,
            "steps": steps, "kernel": path, "unfused_ms": ms_u, "speedup_over_unfused": ms_u / ms_f,
            "q_in_kernel_ms": ms_k,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "peak_source": peaks["source"] + " bf16 dense (burst)"},
            "status": _C.device_status()}


def run_decode_strong(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 5a's 64 sequences split over the ranks by sharding.balance_sequences (by cached length,
    longest first); GB/s of the whole step's cache bytes over the slowest rank (strong scaling)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200.sharding import balance_sequences

    B, H, Hkv, D, Smax = DEC["B"], DEC["H"], DEC["Hkv"], DEC["D"], DEC["Smax"]
    g = torch.Generator(device=dev)
    g.manual_seed(77)  # the same lengths on every rank
    lens_all = torch.randint(DEC["Lmin"], Smax + 1, (B,), generator=g, device=dev).to(torch.int32)
    mine = balance_sequences(lens_all.cpu().tolist(), world)[rank]
    lens = lens_all[mine].contiguous()
    Smax_r = int(lens.max().item()) if mine else 1
    Smax_r += Smax_r % 2  # even cache length: the tensor-core path's 16-byte row pairs
    row = D // 32 * 34
    n = len(mine)
    kq = torch.empty((n, Hkv, Smax_r, row), dtype=torch.uint8, device=dev)
    vq = torch.empty_like(kq)
    gr = torch.Generator(device=dev)
    gr.manual_seed(1000 + rank)
    for i in range(n):
        kq[i] = gtb.quantize_q8_0(torch.randn((Hkv, Smax_r, D), generator=gr, device=dev))
        vq[i] = gtb.quantize_q8_0(torch.randn((Hkv, Smax_r, D), generator=gr, device=dev))
    q = torch.randn((n, H, 1, D), generator=gr, device=dev).to(torch.float16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        gtb.decode_q8_0(q, kq, vq, lens)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    times = []
    for _ in range(max(3, min(args.steps, 20))):
        flush.zero_()
        times.append(_time_events(stream, lambda: gtb.decode_q8_0(q, kq, vq, lens), 1))
    ms = max_over_ranks(statistics.mean(times))
    total = int(lens_all.sum().item()) * Hkv * 2 * row + B * H * D * 2 * 2
    del kq, vq, flush
    torch.cuda.empty_cache()
    return {"workload": "config 5a's 64 sequences split over the ranks by cached length", "value": total / (ms * 1e-3) / 1e9,
            "unit": "GB/s", "ms_per_step": ms, "scaling": "strong", "sequences_this_rank": n,
            "tokens_this_rank": int(lens.sum().item())}


# ------------------------------------------------------------------ long-context workload (config 5b)

RING = dict(B=1, H=32, Hkv=8, L=131072, D=128)


def run_ring(args, rank: int, world: int, dev, max_over_ranks=lambda x: x) -> dict:
    """Config 5b: causal GQA forward of one 131072-token sequence, bf16, Hq=32 Hkv=8 D=128. One GPU
    runs the whole sequence in one launch; N GPUs hold zig-zag shards and run the K/V ring
    (gguf_train_b200.ring: N steps of native forwards on chunk pairs, log-sum-exp merges, K/V shards
    passed on over NVLink with NCCL send/receive beside the compute). FLOPs: 4*Hq*D*L(L+1)/2."""
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn
    from gguf_train_b200 import ring

    B, H, Hkv, L, D = RING["B"], RING["H"], RING["Hkv"], RING["L"], RING["D"]
    g = torch.Generator(device=dev)
    g.manual_seed(2024)  # the same sequence on every rank; each keeps its shard
    q = (torch.randn((B, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    if world > 1:
        qs, ks, vs = (ring.shard_zigzag(t, world, rank) for t in (q, k, v))
        del q, k, v

        def step():
            return ring.ring_attention(qs, ks, vs, scale)
    else:
        def step():
            return Fn.sdpa_forward(q, k, v, None, scale, True, need_lse=False)[0]
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    flops = fwd_flops(B, H, L, D)
    tf = flops / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    kv_bytes = 2 * B * Hkv * L * D * 2
    line = {
        "workload": "config 5b: causal GQA prefill of one long sequence, bf16, B=1 Hq=32 Hkv=8 L=131072 D=128",
        "value": tf, "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps, "flops_per_step": flops,
        "parallelism": (f"zig-zag sequence shards, K/V ring over {world} GPUs (NCCL send/recv beside the compute)"
                        if world > 1 else "one GPU, one launch"),
        "scaling": "strong",
        "nvlink_bytes_per_rank_per_step": kv_bytes // world * (world - 1),
        # `steps` ring steps of ~0.1 s each: under a second of back-to-back work, so the burst peak
        "roofline": {"bound": "tensor", "achieved": tf / world, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s per GPU", "frac": tf / world / peaks["bf16_tflops"],
                     "peak_source": peaks["source"] + " bf16 dense (burst)", "timed_ms": steps * ms},
        "status": _C.device_status(),
    }
    torch.cuda.empty_cache()
    return line


# ------------------------------------------------------------------ GPU arm

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-batch", type=int, default=None,
                    help="sequences of the decode workload (default: config 5a's 64; smaller for profiling)")
    ap.add_argument("--weights-batch", type=int, default=None,
                    help="sequences of the weights workload (default: config 3's 8; smaller for profiling)")
    ap.add_argument("--workload", default="prefill",
                    choices=["prefill", "decode", "train", "ring", "key_padding", "mha", "linear", "prefill_strong",
                             "train_strong", "decode_strong", "weights", "rope_prefill"],
                    help="prefill: config 3 (the default line); train: config 4 fwd+bwd; decode: config 5a; "
                         "ring: config 5b (one long sequence, K/V ring over the GPUs); key_padding: config 3 with a "
                         "key-padding mask; mha: config 2 (nn.MultiheadAttention fp32 fwd+bwd); *_strong: the fixed "
                         "config-3 / config-4 / config-5a work split over the GPUs; weights: MHA's need_weights output at "
                         "config 3's shape; rope_prefill: config 3 with RoPE fused into the forward")
    ap.add_argument("--no-extra", action="store_true",
                    help="default line without the fwd+bwd (config 4) and decode (config 5a) measurements")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.workload != "prefill":
        barrier()
        runner = {"decode": run_decode, "train": run_train, "ring": run_ring, "key_padding": run_prefill_key_padding,
                  "mha": run_mha, "linear": run_linear, "prefill_strong": run_prefill_strong, "decode_strong": run_decode_strong,
                  "train_strong": lambda *a: run_train(*a, strong=True), "weights": run_weights, "rope_prefill": run_rope_prefill}[args.workload]
        res = runner(args, rank, world, dev, max_over_ranks)
        if args.workload != "decode":
            scaling = res.pop("scaling", "weak")
            res = dict(metric=METRIC, n_gpus=world, steps=res.pop("steps", max(3, min(args.steps, 20))),
                       warmup=max(args.warmup, 3), higher_is_better=True, scaling=scaling, vs_baseline=None,
                       dtype=res.pop("dtype", "bf16"),
                       data="synthetic: seeded normal inputs generated on the device",
                       config={"workload": res.pop("workload")}, **res)
        if world > 1:
            barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(res), flush=True)
        return

    from gguf_train_b200.sharding import ShardedAttention

    B, H, Hkv, L, D = CFG["B"], CFG["H"], CFG["Hkv"], CFG["L"], CFG["D"]
    # weak scaling: a global batch of world x B sequences; this rank's share of its units is config 3
    sa = ShardedAttention(B * world, H, Hkv, world, rank)
    b_lo, b_hi = sa.batch_span()
    assert sa.units == B * Hkv and b_hi - b_lo == B
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    q = (torch.randn((B, H, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)
    flops = fwd_flops(B, H, L, D)
    stream = torch.cuda.current_stream(dev)

    def step():
        sa.forward(q, k, v, out, scale, True, base=b_lo)  # one native call per segment (here one)
        return out

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    assert _C.device_status() == 0, "a kernel reported a wait timeout during warm-up"

    # ---- kernel-resident timing: K launches, one event pair per launch
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(torch.cuda.current_device())
    barrier()
    torch.cuda.synchronize(dev)
    with sampler:
        t_all0 = torch.cuda.Event(enable_timing=True)
        t_all1 = torch.cuda.Event(enable_timing=True)
        t_all0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        t_all1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    total_ms = max_over_ranks(t_all0.elapsed_time(t_all1))
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    launch_ms = max_over_ranks(launch_ms)
    status = _C.device_status()
    ms_per_step = total_ms / args.steps
    value = flops * world / (ms_per_step * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 10))
    qh = q.cpu().pin_memory()
    kh = k.cpu().pin_memory()
    vh = v.cpu().pin_memory()
    oh = torch.empty((B, H, L, D), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        # host q, k, v in, host out: the batch in chunks, copies in both directions overlapped with
        # the kernels (every byte of q, k, v and out crosses PCIe each step)
        gtb.sdpa_from_host(qh, kh, vh, out=oh, is_causal=True, scale=scale)

    for _ in range(2):
        e2e_step()
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    h2d = qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2
    d2h = oh.numel() * 2
    status |= _C.device_status()

    peaks = load_peaks()
    achieved = flops / (launch_ms * 1e-3) / 1e12
    traffic = profile_traffic("fwd_sm100_config3")
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)*0.5 generated on the device (the configuration's shapes and distribution)",
        "config": {"workload": WORKLOAD, "global_batch": B * world, "seq_len": L, "heads": H, "kv_heads": Hkv,
                   "head_dim": D,
                   "parallelism": f"sharding.ShardedAttention: {B * Hkv} (batch, kv head) units per rank of a "
                                  f"global batch of {B * world}, no collective",
                   "l2": "inputs larger than L2 (q+k+v = 402 MB per GPU)", "kernel": "fwd_sm100 (tcgen05/TMA)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"],
                     "traffic": traffic, "peak_source": peaks["source"] + " bf16 dense (burst)",
                     "flops_per_launch": flops, "launch_ms": launch_ms},
        "e2e": {"value": flops * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "gguf_train_b200.sdpa_from_host -> C ABI gtb_sdpa_fwd_host (pinned host q, k, v, out; "
                       "8 pieces of one sequence, copies in both directions overlapped with the tcgen05 forward "
                       "on three streams)"},
        "gpu_launches": args.steps,
        "clocks": sampler.summary(),
        "status": status,
    }
    if not args.no_extra:
        del q, k, v, qh, kh, vh, oh
        torch.cuda.empty_cache()
        barrier()
        line["extra"] = {"fwd_bwd": run_train(args, rank, world, dev, max_over_ranks)}
        barrier()
        line["extra"]["decode_q8_0"] = run_decode(args, rank, world, dev, max_over_ranks)
        barrier()
        line["extra"]["long_context_ring"] = run_ring(args, rank, world, dev, max_over_ranks)
        barrier()
        line["extra"]["prefill_key_padding"] = run_prefill_key_padding(args, rank, world, dev, max_over_ranks)
        barrier()
        line["extra"]["mha_config2"] = run_mha(args, rank, world, dev, max_over_ranks)
        barrier()
        line["extra"]["linear_bf16"] = run_linear(args, rank, world, dev, max_over_ranks)
        barrier()
        line["extra"]["need_weights"] = run_weights(args, rank, world, dev, max_over_ranks)
        barrier()
        line["extra"]["prefill_rope"] = run_rope_prefill(args, rank, world, dev, max_over_ranks)
        if world > 1:  # strong scaling: the fixed batches split over the ranks
            barrier()
            line["extra"]["prefill_strong"] = run_prefill_strong(args, rank, world, dev, max_over_ranks)
            barrier()
            line["extra"]["fwd_bwd_strong"] = run_train(args, rank, world, dev, max_over_ranks, strong=True)
            barrier()
            line["extra"]["decode_strong"] = run_decode_strong(args, rank, world, dev, max_over_ranks)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cv, threads, desc, kind = cpu_sample(2)
        line["cpu_baseline"] = {"value": cv, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": desc}
    if world > 1:
        barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
