"""Attention forward throughput on B200 — the headline metric of BASELINE.json.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one forward pass of the configured workload through the public API
(mlx_primitives.*) on each rank's GPU.  Default workload (config "c2", the one BASELINE's
metric is quoted on): flash_attention bf16, BHSD, causal, batch 4 x 32 heads x 4096 tokens x
head_dim 128.  Multi-GPU runs (torchrun, one process per GPU) split the fixed workload's
(batch, head) units across the ranks (mlx_primitives.attention.partition: contiguous unit
ranges, each rank computes its own in place, no collective on the data path), so the total
work is fixed ("strong"); config 5 is one 128K-token sequence run as a zig-zag ring.

Printed by rank 0, one JSON line: value = whole-job TFLOPS (algorithmic FLOPs: 4*D per
admissible (query, key) pair, masked pairs not counted) over the max-over-ranks device time;
e2e = the same through the public API with pinned host tensors, H2D/D2H inside the timed
region; roofline = the attention kernel against MEASURED_PEAKS.json; cpu_baseline = the CPU
oracle (test infrastructure, the reference's algorithm restated) on a bounded sample.
`--impl reference` times that CPU path alone on rank 0 (the reference's own MLX code cannot
run on Linux without Apple hardware).  Other workloads: --config c1 c3 c4 c5 (the other
BASELINE configs), g2 (grouped-query), r2 (RoPE + attention), p4 (paged-KV decode, HBM
roofline), b2 / b4 (backward).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "mlx-primitives_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "attention fwd TFLOPS/GPU and % of BF16 tensor peak at 1/2/4/8 B200"

# DRAM bytes (read + write) of one launch of the dominant kernel at N=1 (attn_fwd_sm100_kernel
# for c2, c3, c4 and c5s, attn_fwd_fp32_kernel for c1, paged_attn_tma_kernel for p4,
# attn_bwd_sm100_kernel for b2), from one ncu capture of the same command; null where no
# capture of that configuration was taken.
NCU_TRAFFIC_BYTES = {"c1": 18.94e6, "c2": 546.2e6, "c3": 1.0947e9, "c4": 2.2867e9,
                     "c5s": 351.6e6, "p4": 541.18e6, "b2": 1.3016e9}

CONFIGS = {
    "c1": dict(workload="flash_attention fp32 BSHD causal (config 1)", api="flash", dtype="fp32",
               layout="BSHD", B=2, H=12, S=1024, Skv=1024, D=64, causal=True, window=-1, std=1.0),
    "c2": dict(workload="flash_attention bf16 BHSD causal (config 2)", api="flash", dtype="bf16",
               layout="BHSD", B=4, H=32, S=4096, Skv=4096, D=128, causal=True, window=-1, std=1.0),
    "c3": dict(workload="SlidingWindowAttention bf16 BSHD causal W4096 (config 3)", api="swa",
               dtype="bf16", layout="BSHD", B=2, H=32, S=16384, Skv=16384, D=128, causal=True,
               window=4096, std=1.0),
    "c4": dict(workload="ChunkedCrossAttention bf16 BSHD chunk4096 (config 4)", api="chunked",
               dtype="bf16", layout="BSHD", B=8, H=16, S=512, Skv=65536, D=64, causal=False,
               window=-1, std=0.5),
    # grouped-query variant of config 2 (32 query heads sharing 8 K/V heads), not a BASELINE
    # config: the measurement of the gqa_attention entry point
    "g2": dict(workload="gqa_attention bf16 BSHD causal, 32 query / 8 K/V heads", api="gqa",
               dtype="bf16", layout="BSHD", B=4, H=32, Hkv=8, S=4096, Skv=4096, D=128,
               causal=True, window=-1, std=1.0),
    # RoPE + attention (kernels.fused_rope_attention) on the config-2 shape, BSHD: the RoPE
    # launch for Q and K is inside the timed step; not a BASELINE config
    "r2": dict(workload="fused_rope_attention bf16 BSHD causal (config-2 shape)", api="frope",
               dtype="bf16", layout="BSHD", B=4, H=32, S=4096, Skv=4096, D=128, causal=True,
               window=-1, std=1.0),
    # backward pass (dQ, dK, dV) of config 2 through torch autograd's entry point
    # (attention_backward); algorithmic FLOPs = 2.5 x the forward's (five matmuls per pair)
    "b2": dict(workload="attention backward bf16 BHSD causal (config-2 shape)", api="bwd",
               dtype="bf16", layout="BHSD", B=4, H=32, S=4096, Skv=4096, D=128, causal=True,
               window=-1, std=1.0),
    # backward of the config-4 shape's head_dim (64), causal self-attention, BSHD
    "b4": dict(workload="attention backward bf16 BHSD causal, head_dim 64", api="bwd",
               dtype="bf16", layout="BHSD", B=8, H=16, S=4096, Skv=4096, D=64, causal=True,
               window=-1, std=1.0),
    # paged-KV decode (cache.paged_attention): the reference cache benchmark's largest shape
    # (benchmarks/suites/cache.py:64-80, 204-234: batch 8, 4096 cached tokens, 32 heads,
    # head_dim 128, block 16, sequential block tables); HBM-bound, not a BASELINE config
    "p4": dict(workload="paged_attention decode bf16, 8 sequences x 4096 cached tokens, block 16",
               api="paged", dtype="bf16", layout="BSHD", B=8, H=32, S=1, Skv=4096, D=128,
               block=16, causal=True, window=-1, std=1.0),
    # config 5's kernel on a profilable slice (2 of its 32 heads, the full 128K sequence): the
    # case ncu summaries of the long-context kernel are taken on; not a BASELINE config
    "c5s": dict(workload="flash_attention bf16 BHSD causal, 2 heads x 131072 tokens (config-5 slice)",
                api="flash", dtype="bf16", layout="BHSD", B=1, H=2, S=131072, Skv=131072, D=128,
                causal=True, window=-1, std=1.0),
    # total work fixed: one 128K-token sequence, sequence-parallel ring over the N GPUs
    "c5": dict(workload="long-context flash_attention bf16 BHSD causal, zig-zag ring (config 5)",
               api="ring", dtype="bf16", layout="BHSD", B=1, H=32, S=131072, Skv=131072,
               D=128, causal=True, window=-1, std=1.0),
}

L2_BYTES = 126 * 1024 * 1024
# configs whose (batch, head) units are split across the GPUs of a multi-GPU run
SPLIT_APIS = ("flash", "swa", "chunked", "gqa")
FP32_LANES_PER_SM = 128  # FP32 FMA lanes per SM (4 sub-partitions x 32)


def admissible_pairs(Sq, Skv, causal, wl=-1, wr=-1, qoff=0, kvoff=0) -> int:
    """Number of (query, key) pairs the mask admits for one (batch, head)."""
    qpos = np.arange(Sq, dtype=np.int64) + qoff
    lo = np.zeros(Sq, np.int64)
    hi = np.full(Sq, Skv, np.int64)
    if wl >= 0:
        lo = np.maximum(lo, qpos - wl - kvoff)
    if causal:
        hi = np.minimum(hi, qpos - kvoff + 1)
    if wr >= 0:
        hi = np.minimum(hi, qpos + wr - kvoff + 1)
    return int(np.clip(hi - lo, 0, None).sum())


def config_flops(c) -> float:
    """Algorithmic FLOPs of one forward of config c on one GPU."""
    wr = -1 if c["causal"] else c["window"]
    pairs = admissible_pairs(c["S"], c["Skv"], c["causal"], c["window"], wr,
                             (c["Skv"] - c["S"]) if (c["api"] == "flash" and c["causal"]) else 0)
    return 4.0 * c["D"] * pairs * c["B"] * c["H"]


def config_bytes(c) -> float:
    es = 4 if c["dtype"] == "fp32" else 2
    return es * c["B"] * c["D"] * (2 * c["H"] * c["S"] + 2 * c.get("Hkv", c["H"]) * c["Skv"])


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d.get("bf16_tflops_sustained"), d["hbm_gbs"], "MEASURED_PEAKS.json (measured)"
    return 1590.0, 1400.0, 6650.0, "profiling-recipe fallback"


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(self.period)

    def sample(self):
        if self.nv is None:
            return
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for name, bit in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:  # noqa: BLE001
            pass

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()
        self.sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------ CPU side
def blas_threads() -> int:
    """Threads of the BLAS pool the numpy oracle runs on (the cores the CPU baseline uses)."""
    try:
        from threadpoolctl import threadpool_info
        return max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
    except Exception:  # noqa: BLE001
        return os.cpu_count()


def host_cores() -> dict:
    """The GPU box's host: logical CPUs and torch's intra-op thread count."""
    try:
        import torch
        torch_threads = torch.get_num_threads()
    except Exception:  # noqa: BLE001
        torch_threads = None
    return {"os_cpu_count": os.cpu_count(), "torch_num_threads": torch_threads}


def cpu_oracle_tflops(c, budget_s: float, max_units: int | None = None):
    """Time the CPU oracle (dense fp32 restatement of the reference's CPU path, numpy + BLAS)
    on whole (batch, head) units of config c until budget_s is used.  Returns (TFLOPS, units,
    seconds, threads)."""
    from oracle import attention_oracle as O

    threads = blas_threads()
    D, S, Skv = c["D"], c["S"], c["Skv"]
    wr = -1 if c["causal"] else c["window"]
    qoff = (Skv - S) if (c["api"] == "flash" and c["causal"]) else 0
    pairs = admissible_pairs(S, Skv, c["causal"], c["window"], wr, qoff)
    rng = np.random.RandomState(1234)
    q = (rng.standard_normal((1, 1, S, D)) * c["std"]).astype(np.float32)
    k = (rng.standard_normal((1, 1, Skv, D)) * c["std"]).astype(np.float32)
    v = (rng.standard_normal((1, 1, Skv, D)) * c["std"]).astype(np.float32)
    if c["dtype"] != "fp32":
        q, k, v = (O.round_bf16(a) for a in (q, k, v))
    units, t_total = 0, 0.0
    cap = max_units or c["B"] * c["H"]
    if S * Skv > (1 << 26):
        # a dense score matrix of this unit would not fit in host memory (config 5: 128K x 128K):
        # time exact rows (each against its whole admissible key range) on an even sample of
        # query rows and count only their pairs
        rows = np.linspace(0, S - 1, 64).astype(np.int64)
        kpos = np.arange(Skv)[None, :]
        qpos = rows[:, None] + qoff
        ok = np.ones((len(rows), Skv), dtype=bool)
        if c["causal"]:
            ok &= kpos <= qpos
        if c["window"] >= 0:
            ok &= (qpos - kpos) <= c["window"]
        if wr >= 0:
            ok &= (kpos - qpos) <= wr
        row_pairs = int(ok.sum())
        while units < cap and (units == 0 or t_total < budget_s):
            t0 = time.perf_counter()
            O.attention_rows_bhsd(q, k, v, rows, 1.0 / math.sqrt(D), causal=c["causal"],
                                  window_left=c["window"], window_right=wr, q_offset=qoff)
            t_total += time.perf_counter() - t0
            units += 1
        return 4.0 * D * row_pairs * units / t_total / 1e12, units, t_total, threads
    while units < cap and (units == 0 or t_total < budget_s):
        t0 = time.perf_counter()
        O.attention_bhsd(q, k, v, 1.0 / math.sqrt(D), causal=c["causal"], window_left=c["window"],
                         window_right=wr, q_offset=qoff, dtype=np.float32)
        t_total += time.perf_counter() - t0
        units += 1
    return 4.0 * D * pairs * units / t_total / 1e12, units, t_total, threads


def run_reference_arm(args, c, rank):
    """--impl reference: the CPU path (oracle port) on rank 0's host cores."""
    if rank != 0:
        return
    split = args.gpus > 1 and c["api"] in SPLIT_APIS
    units_per_gpu = -(-c["B"] * c["H"] // args.gpus) if split else None
    per_step = []
    total_units = 0
    total_flops = 0.0
    threads = None
    for i in range(args.warmup + args.steps):
        tf, units, secs, threads = cpu_oracle_tflops(c, budget_s=0.0, max_units=1)
        if i >= args.warmup:
            per_step.append(secs)
            total_units += units
            total_flops += tf * 1e12 * secs  # the sample's own algorithmic FLOPs
    secs = sum(per_step)
    value = total_flops / secs / 1e12
    sample = (f"{total_units} x 64 evenly spaced query rows of one (batch, head) unit of "
              f"{c['workload']}, exact fp64 rows, one per step" if c["S"] * c["Skv"] > (1 << 26)
              else f"{total_units} (batch, head) units of {c['workload']}, one per step, fp32 numpy")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * secs / max(len(per_step), 1), "higher_is_better": True,
        "scaling": "strong" if split or c["api"] == "ring" else "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config_json(c, args.gpus, units_per_gpu),
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, **host_cores(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's runtime) cannot run on this Linux/NVIDIA box; this arm times "
                "the oracle's restatement of the reference's CPU algorithm (dense fp32 SDPA path)",
    }
    print(json.dumps(line), flush=True)


def l2_note(per_gpu_bytes):
    if per_gpu_bytes > L2_BYTES:
        return "inputs larger than L2"
    rot = math.ceil(3 * L2_BYTES / per_gpu_bytes)
    return (f"inputs rotated over {rot} copies ({rot * per_gpu_bytes / 2**20:.0f} MiB per GPU, "
            f"more than 3x the 126 MiB L2): each step reads inputs evicted since their last use")


def config_json(c, n, units_per_gpu=None):
    if c["api"] == "ring":
        par = (f"sequence-parallel zig-zag ring over {n} GPUs (NCCL send/recv of K/V, LSE merge)"
               if n > 1 else "single GPU")
        return {"workload": c["workload"], "global_batch": c["B"], "heads": c["H"],
                "seq_len": c["S"], "head_dim": c["D"], "layout": c["layout"], "causal": True,
                "parallelism": par, "l2": "inputs larger than L2"}
    split = units_per_gpu is not None
    per_gpu_bytes = config_bytes(c) * (units_per_gpu / (c["B"] * c["H"]) if split else 1)
    return {"workload": c["workload"], "global_batch": c["B"] if split else c["B"] * n,
            "batch_per_gpu": None if split else c["B"],
            "heads": c["H"], "kv_heads": c.get("Hkv", c["H"]), "seq_len": c["S"],
            "kv_len": c["Skv"], "head_dim": c["D"],
            "layout": c["layout"], "causal": c["causal"], "window": c["window"],
            "parallelism": (f"the fixed workload's {c['B'] * c['H']} (batch, head) units split "
                            f"over {n} GPUs (up to {units_per_gpu} per GPU), no collective"
                            if split else f"dp{n} over (batch, head) units, no collective"),
            "l2": l2_note(per_gpu_bytes)}


# ------------------------------------------------------------------------------ paged decode
def paged_tables(c):
    """Sequential block tables of the reference cache benchmark (create_block_table_from_lengths
    over equal lengths): sequence b owns blocks b * n .. b * n + n - 1."""
    n = (c["Skv"] + c["block"] - 1) // c["block"]
    bt = np.arange(c["B"] * n, dtype=np.int32).reshape(c["B"], n)
    return bt, np.full(c["B"], c["Skv"], dtype=np.int32), c["B"] * n


def paged_flops_bytes(c, seqs=None):
    """Algorithmic FLOPs (4 * D per admissible (query, key) pair per head) and minimum HBM bytes
    (every K/V row of the contexts read once, q read and o written once) of a decode step."""
    seqs = c["B"] if seqs is None else seqs
    es = 4 if c["dtype"] == "fp32" else 2
    pairs = seqs * c["Skv"] * c["H"]
    return 4.0 * c["D"] * pairs, es * c["D"] * (2 * pairs + 2 * seqs * c["H"])


def cpu_paged_sample(c, budget_s, max_seqs=None):
    """The oracle's paged_attention (fp32 numpy) on whole sequences of config c until budget_s
    is used.  Returns (TFLOPS, sequences, seconds, threads)."""
    from oracle import attention_oracle as O
    threads = blas_threads()
    n = (c["Skv"] + c["block"] - 1) // c["block"]
    q, kp, vp = O.make_qkv((1, 1, c["H"], c["D"]), (n, c["block"], c["H"], c["D"]), seed=7)
    if c["dtype"] != "fp32":
        q, kp, vp = (O.round_bf16(a) for a in (q, kp, vp))
    bt = np.arange(n, dtype=np.int32)[None]
    ctx = np.array([c["Skv"]], dtype=np.int32)
    seqs, t_total = 0, 0.0
    cap = max_seqs or c["B"]
    while seqs < cap and (seqs == 0 or t_total < budget_s):
        t0 = time.perf_counter()
        O.paged_attention(q, kp, vp, bt, ctx, block_size=c["block"], dtype=np.float32)
        t_total += time.perf_counter() - t0
        seqs += 1
    flops, _ = paged_flops_bytes(c, seqs)
    return flops / t_total / 1e12, seqs, t_total, threads


def bench_paged(args, c, world, rank, local):
    """Decode step of paged attention: q (B, 1, H, D) over the block pools through
    mlx_primitives.cache.paged_attention.  value = algorithmic TFLOPS of the whole job; the
    roofline is HBM (K/V bytes of the contexts / launch time, against MEASURED_PEAKS hbm_gbs)."""
    if args.impl == "reference":
        if rank != 0:
            return
        per, seqs_total, threads = [], 0, None
        for i in range(args.warmup + args.steps):
            _, seqs, secs, threads = cpu_paged_sample(c, 0.0, max_seqs=1)
            if i >= args.warmup:
                per.append(secs)
                seqs_total += seqs
        flops, _ = paged_flops_bytes(c, seqs_total)
        value = flops / sum(per) / 1e12
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * sum(per) / len(per), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": paged_config_json(c, args.gpus),
            "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, **host_cores(), "kind": "port",
                             "sample": f"{seqs_total} sequences of {c['workload']}, one per step, "
                                       "fp32 numpy (gather + dense masked softmax, as the reference)"},
            "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "MLX cannot run on this Linux/NVIDIA box; this arm times the oracle's "
                    "restatement of the reference's paged_attention"}), flush=True)
        return

    import ctypes

    import torch
    import torch.distributed as dist

    from mlx_primitives import _lib
    from mlx_primitives.cache import paged_attention

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    dtype = torch.float32 if c["dtype"] == "fp32" else torch.bfloat16
    B, H, D, bs = c["B"], c["H"], c["D"], c["block"]
    bt_np, ctx_np, nblk = paged_tables(c)
    g = torch.Generator(device=dev)
    g.manual_seed(42 + rank)
    q = torch.randn((B, 1, H, D), generator=g, device=dev).to(dtype)
    kp = torch.randn((nblk, bs, H, D), generator=g, device=dev).to(dtype)
    vp = torch.randn((nblk, bs, H, D), generator=g, device=dev).to(dtype)
    bt = torch.from_numpy(bt_np).to(dev)
    ctx = torch.from_numpy(ctx_np).to(dev)

    def step(qq, btt, cc):
        return paged_attention(qq, kp, vp, btt, cc, block_size=bs)

    # the same launch straight through the C-ABI (arguments built once): the kernel timing
    L = _lib.lib()
    dt = _lib.DTYPE_CODES[dtype]
    o = torch.empty_like(q)
    ws_bytes = L.mlxp_paged_attn_workspace_size(dt, B, H, 1, D, H, nblk, bs, bt.shape[1], 0)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    cargs = (q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), ctx.data_ptr(), None,
             o.data_ptr(), dt, B, H, 1, D, H, nblk, bs, bt.shape[1], _lib.strides4(q, "BSHD"),
             (ctypes.c_int64 * 4)(*kp.stride()), bt.stride(0), _lib.strides4(o, "BSHD"),
             ctypes.c_float(D ** -0.5), 1, 0, ws.data_ptr(), ws_bytes, stream.cuda_stream)
    launches = 1  # one paged-attention kernel per call (shares merged inside it)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, n):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(n)]
        barrier()
        torch.cuda.synchronize(dev)
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return sum(a.elapsed_time(b) for a, b in ev) / n

    for _ in range(args.warmup):
        step(q, bt, ctx)
        _lib.check(L.mlxp_paged_attn(*cargs), "mlxp_paged_attn")
    with ClockSampler(local) as clocks:
        ms_local = timed(lambda: step(q, bt, ctx), args.steps)
        ms_kernel = timed(lambda: L.mlxp_paged_attn(*cargs), args.steps)
    torch.cuda.synchronize(dev)
    assert torch.equal(o, step(q, bt, ctx)), "C-ABI launch and public API disagree"
    ms = max_over_ranks(ms_local)
    flops, min_bytes = paged_flops_bytes(c)
    value = world * flops / (ms * 1e-3) / 1e12
    _, _, hbm, peak_src = load_peaks()
    achieved_gbs = min_bytes / (ms_kernel * 1e-3) / 1e9

    # e2e: q, block tables and lengths from pinned host memory, output back to pinned memory;
    # the pools are the cache's state and stay resident in HBM between decode steps
    hq, hbt, hctx = q.cpu().pin_memory(), bt.cpu().pin_memory(), ctx.cpu().pin_memory()
    oh = torch.empty(q.shape, dtype=dtype, pin_memory=True)

    def e2e_step():
        o_ = step(hq.to(dev, non_blocking=True), hbt.to(dev, non_blocking=True),
                  hctx.to(dev, non_blocking=True))
        oh.copy_(o_, non_blocking=True)

    for _ in range(3):
        e2e_step()
    e2e_ms = max_over_ranks(timed(e2e_step, max(args.e2e_steps, 1)))
    e2e = {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
           "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (hq, hbt, hctx)),
           "d2h_bytes_per_step": oh.numel() * oh.element_size(), "ms_per_step": e2e_ms,
           "note": "per decode step: q, block tables and context lengths copied in, the output "
                   "copied out; the K/V pools are the cache state, resident in HBM"}

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0, 1) q and pools generated on device (seed 42 + rank)",
            "config": paged_config_json(c, world),
            "kv_gbs": min_bytes / (ms * 1e-3) / 1e9,
            "roofline": {
                "bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s",
                "frac": achieved_gbs / hbm, "traffic": NCU_TRAFFIC_BYTES.get(args.config),
                "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum)",
                "kernel": "paged_attn_tma_kernel (one C-ABI call: counter reset + kernel)",
                "kernel_ms": ms_kernel,
                "peak_source": f"{peak_src}: hbm_gbs",
                "algorithmic_bytes_per_launch": min_bytes,
            },
            "e2e": e2e,
            "gpu_launches": args.steps * launches * 2,
            "clocks": clocks.summary(),
        }
        if world == 1 and args.cpu_budget > 0:
            tf, seqs, secs, threads = cpu_paged_sample(c, args.cpu_budget)
            line["cpu_baseline"] = {
                "value": tf, "unit": "TFLOPS", "cores": threads, **host_cores(), "kind": "port",
                "sample": f"{seqs} of {B} sequences, oracle paged_attention fp32 numpy, "
                          f"{secs:.1f} s"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def bench_backward(args, c, world, rank, local):
    """Backward of attention on config c: the forward's O and log-sum-exp are computed once,
    each step runs attention_backward (the autograd backward of every attention entry point)
    on a fresh dO.  value = algorithmic TFLOPS (2.5 x the forward's FLOPs)."""
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference's gradients "
                              "come from MLX autodiff, which cannot run on this Linux/NVIDIA box"}),
                  flush=True)
        return
    import torch
    import torch.distributed as dist

    from mlx_primitives.attention._core import _forward_impl, attention_backward

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    B, H, S, D = c["B"], c["H"], c["S"], c["D"]
    g = torch.Generator(device=dev)
    g.manual_seed(42 + rank)
    q, k, v, do = (torch.randn((B, H, S, D), generator=g, device=dev).bfloat16() for _ in range(4))
    kw = dict(layout=c["layout"], scale=D ** -0.5, causal=c["causal"])
    out, lse = _forward_impl(q, k, v, return_lse=True, **kw)

    def step():
        return attention_backward(q, k, v, out, lse, do, **kw)

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        for a, b in ev:
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize(dev)
    ms_local = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    ms = ms_local
    if world > 1:
        t = torch.tensor([ms_local], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = 2.5 * config_flops(c)
    peak, _, _, peak_src = load_peaks()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC + " (backward)", "value": world * flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: seeded N(0, 1) q, k, v, dO on device",
            "config": config_json(c, world),
            "roofline": {"bound": "tensor", "achieved": flops / (ms_local * 1e-3) / 1e12,
                         "peak": peak, "unit": "TFLOP/s",
                         "frac": flops / (ms_local * 1e-3) / 1e12 / peak,
                         "traffic": NCU_TRAFFIC_BYTES.get(args.config),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum)",
                         "kernel": "attn_bwd_sm100_kernel (+ prep, dQ convert)",
                         "peak_source": f"{peak_src}: bf16_tflops (the tensor-core target)",
                         "algorithmic_flops_per_launch": flops},
            "gpu_launches": 3 * args.steps, "clocks": clocks.summary()}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def paged_config_json(c, n):
    return {"workload": c["workload"], "global_batch": c["B"] * n, "batch_per_gpu": c["B"],
            "heads": c["H"], "head_dim": c["D"], "context_len": c["Skv"],
            "block_size": c["block"], "block_tables": "sequential (reference benchmark)",
            "parallelism": f"dp{n} over sequences, no collective",
            "l2": "inputs larger than L2"}


# ------------------------------------------------------------------------------ GPU side
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    c = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if c["api"] == "paged":
        bench_paged(args, c, world, rank, local)
        return
    if c["api"] == "bwd":
        bench_backward(args, c, world, rank, local)
        return
    if args.impl == "reference":
        run_reference_arm(args, c, rank)
        return

    import torch
    import torch.distributed as dist

    import mlx_primitives as mp
    import mlx_primitives.kernels  # noqa: F401  (RoPE entry points, config r2)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    dtype = torch.float32 if c["dtype"] == "fp32" else torch.bfloat16
    B, H, S, Skv, D = c["B"], c["H"], c["S"], c["Skv"], c["D"]
    shape_q = (B, H, S, D) if c["layout"] == "BHSD" else (B, S, H, D)
    Hkv = c.get("Hkv", H)
    shape_kv = (B, Hkv, Skv, D) if c["layout"] == "BHSD" else (B, Skv, Hkv, D)
    ring = c["api"] == "ring" and world > 1
    # configs 1-4 and g2 on N > 1 GPUs: the fixed workload's (batch, head) units are split
    # across the ranks (strong scaling, no collective); every rank builds the same tensors
    part = world > 1 and c["api"] in SPLIT_APIS
    g = torch.Generator(device=dev)
    g.manual_seed(42 + (0 if c["api"] == "ring" or part else rank))
    q = (torch.randn(shape_q, generator=g, device=dev) * c["std"]).to(dtype)
    k = (torch.randn(shape_kv, generator=g, device=dev) * c["std"]).to(dtype)
    v = (torch.randn(shape_kv, generator=g, device=dev) * c["std"]).to(dtype)
    if ring:
        from mlx_primitives.attention.ring import ring_flash_attention, zigzag_shard
        q, k, v = (zigzag_shard(t, world, rank).contiguous() for t in (q, k, v))
        torch.cuda.empty_cache()

    def api_call(qq, kk, vv):
        """The config's public entry point on a whole call (or on one rank's piece)."""
        if c["api"] in ("flash", "ring"):
            return mp.flash_attention(qq, kk, vv, causal=c["causal"], layout=c["layout"])
        if c["api"] == "swa":
            return mp.sliding_window_attention(qq, kk, vv, window_size=c["window"], causal=c["causal"])
        if c["api"] == "frope":
            return mp.kernels.fused_rope_attention(qq, kk, vv, causal=c["causal"])
        if c["api"] == "gqa":
            return mp.attention.gqa_attention(qq, kk, vv, num_kv_groups=qq.shape[2] // kk.shape[2],
                                              causal=c["causal"])
        return mp.chunked_cross_attention(qq, kk, vv, chunk_size=4096, causal=c["causal"])

    units = range(B * H)
    if part:
        from mlx_primitives.attention import partition as P
        units = P.shard_units(B, H, world, rank)
        pieces = P.rank_pieces(q, k, v, units, c["layout"])
        out_full = torch.empty(q.shape, dtype=dtype, device=dev)

        def part_step(qq, kk, vv):
            """This rank's units of the fixed workload, written in place into out_full."""
            if c["api"] == "flash":
                return P.flash_attention_shard(qq, kk, vv, world, rank, causal=c["causal"],
                                               layout=c["layout"], out=out_full)
            if c["api"] == "swa":
                return P.sliding_window_attention_shard(qq, kk, vv, c["window"], world, rank,
                                                        causal=c["causal"], out=out_full)
            if c["api"] == "chunked":
                return P.chunked_cross_attention_shard(qq, kk, vv, world, rank,
                                                       causal=c["causal"], out=out_full)
            return P.attention_units(qq, kk, vv, units, layout=c["layout"], scale=D ** -0.5,
                                     causal=c["causal"], q_offset=Skv - S if c["causal"] else 0,
                                     out=out_full)

    def step(qq, kk, vv):
        if part:
            return part_step(qq, kk, vv)
        if ring:
            host = qq.device.type == "cpu"
            if host:
                qq, kk, vv = (t.to(dev, non_blocking=True) for t in (qq, kk, vv))
            o = ring_flash_attention(qq, kk, vv)
            if host:
                h = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
                h.copy_(o, non_blocking=True)
                torch.cuda.current_stream(dev).synchronize()
                return h
            return o
        return api_call(qq, kk, vv)

    if ring:  # per ring call and rank: one accumulate per admissible chunk pair (2P + 1), 2 casts
        launches_per_step = (2 * world + 1) + 2
    else:
        launches_per_step = 1  # splits and RoPE run inside the one attention launch
        if part:
            launches_per_step *= len(pieces)
    unit_frac = len(units) / (B * H)  # share of the workload this rank computes
    # Inputs of one step that fit in L2 are rotated over `rot` copies holding together more than
    # 3x L2: every step reads inputs that the other copies' traffic has evicted since their last
    # use, and the steps run back to back (no flush kernel between them, so no launch gap after
    # one either).
    rank_bytes = config_bytes(c) * unit_frac
    rot = 1 if rank_bytes > L2_BYTES else math.ceil(3 * L2_BYTES / rank_bytes)
    inputs = [(q, k, v)] + [tuple(t.clone() for t in (q, k, v)) for _ in range(rot - 1)]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(max(args.warmup, rot)):
        step(*inputs[i % rot])
    stream = torch.cuda.current_stream(dev)
    # The timed steps replay a CUDA graph of the same public-API call (one graph per input
    # copy): the device runs exactly the eager step's kernels, without the Python call path in
    # between (at 8 GPUs one rank's step is ~80 us, about the host time of an eager call).
    # The ring's steps are NCCL-bound and long; they run eagerly.
    graphs = None
    if not ring:
        torch.cuda.synchronize(dev)
        graphs = []
        for i in range(rot):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step(*inputs[i])
            graphs.append(gr)
        for i in range(rot):
            graphs[i].replay()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            starts[i].record(stream)
            if graphs is not None:
                graphs[i % rot].replay()
            else:
                step(*inputs[i % rot])
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms_local = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    ms = max_over_ranks(ms_local)

    # this rank's algorithmic FLOPs per step, and the whole job's
    flops = config_flops(c)
    if c["api"] == "ring":
        flops = flops / world
        job_flops = config_flops(c)
    elif part:
        flops = flops * unit_frac
        job_flops = config_flops(c)
    else:  # every rank runs the whole config (weak scaling)
        job_flops = world * flops
    value = job_flops / (ms * 1e-3) / 1e12
    peak, peak_sus, hbm, peak_src = load_peaks()
    achieved = flops / (ms_local * 1e-3) / 1e12  # this rank's work per step / its step time

    # ---- e2e: public API with pinned host tensors (H2D and D2H inside the timed region)
    e2e = None
    if args.e2e_steps > 0:
        # pinned host inputs: the whole call, or with the split this rank's pieces only (the
        # shard a data loader would hand the rank), each a public-API call on host tensors
        if part:
            host_in = [tuple(t.contiguous().cpu().pin_memory() for t in pc[:3]) for pc in pieces]
        else:
            host_in = [tuple(t.cpu().pin_memory() for t in (q, k, v))]
        call = api_call if part else step

        def e2e_step():
            return [call(*hin) for hin in host_in]

        # warm-up in the timed loop's own pattern (the previous result is still held while
        # the next call runs), so the pinned-memory cache holds both result buffers
        for _ in range(3):
            out_host = e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            out_host = e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.e2e_steps)
        e2e = {"value": job_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "h2d_bytes_per_step": sum(t.numel() * t.element_size() for hin in host_in
                                         for t in hin),
               "d2h_bytes_per_step": sum(o.numel() * o.element_size() for o in out_host),
               "ms_per_step": e2e_ms}
        if part:
            e2e["note"] = "bytes per rank: its own (batch, head) pieces copied in and out"

    # config 1 is fp32 on CUDA cores: its roofline is the FP32 pipe, not the tensor cores
    fp32 = c["dtype"] == "fp32"
    roof_peak = peak
    if fp32:
        props = torch.cuda.get_device_properties(dev)
        max_mhz = clocks.max_mhz or 1965.0
        roof_peak = FP32_LANES_PER_SM * 2 * props.multi_processor_count * max_mhz * 1e6 / 1e12
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong" if c["api"] == "ring" or part else "weak", "vs_baseline": None,
            "dtype": "f32" if c["dtype"] == "fp32" else "bf16",
            "data": ("synthetic: seeded N(0, std^2) tensors generated on device (seed 42; every "
                     "rank builds the same tensors of the split workload)" if (part or ring) else
                     "synthetic: seeded N(0, std^2) tensors generated on device (seed 42 + rank)"),
            "config": config_json(c, world, len(units) if part else None),
            "tflops_per_gpu": value / world,
            "pct_of_bf16_peak": 100.0 * (value / world) / peak,
            "pct_of_bf16_sustained": (100.0 * (value / world) / peak_sus
                                      if peak_sus else None),
            "roofline": {
                "bound": "fp32" if fp32 else "tensor", "achieved": achieved,
                "peak": roof_peak, "unit": "TFLOP/s", "frac": achieved / roof_peak,
                # the N=1 launch's capture; a split rank's launch covers unit_frac of its units
                # (traffic in proportion: every unit's Q, K, V and O once); none for the ring
                "traffic": (NCU_TRAFFIC_BYTES[args.config] * unit_frac
                            if c["api"] != "ring" and args.config in NCU_TRAFFIC_BYTES else None),
                "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum)",
                "kernel": ("attn_fwd_fp32_kernel" if c["dtype"] == "fp32" else
                           "attn_fwd_sm100_kernel"),
                "peak_source": (f"nominal FP32 CUDA-core peak: {FP32_LANES_PER_SM} FMA lanes x 2 x "
                                f"SMs x max SM clock (no measured fp32 figure); "
                                f"{100.0 * achieved / peak:.1f} % of the bf16 tensor peak"
                                if fp32 else
                                f"{peak_src}: bf16_tflops (burst); sustained {peak_sus}"),
                "algorithmic_flops_per_launch": flops,
                "hbm_gbs_at_min_bytes": config_bytes(c) / (ms_local * 1e-3) / 1e9,
            },
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "launch": ("CUDA graph replay of the public-API step" if graphs is not None
                       else "eager public-API calls"),
            "clocks": clocks.summary(),
        }
        if world == 1 and args.cpu_budget > 0:
            tf, units, secs, threads = cpu_oracle_tflops(c, budget_s=args.cpu_budget)
            line["cpu_baseline"] = {
                "value": tf, "unit": "TFLOPS", "cores": threads, **host_cores(), "kind": "port",
                "sample": (f"{units} x 64 evenly spaced query rows of one (batch, head) unit "
                           f"(exact fp64 rows; a dense unit does not fit in host memory), "
                           f"{secs:.1f} s" if c["S"] * c["Skv"] > (1 << 26) else
                           f"{units} of {c['B'] * c['H']} (batch, head) units, dense fp32 numpy, "
                           f"{secs:.1f} s")}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
