#!/usr/bin/env python3
"""NVFP4 QSA benchmark: sparse-decode KV read GB/s (headline) and KV-write tokens/s on B200.

Workload (per GPU, weak scaling): the scale-out decode configuration -- 96
independent sequences of 131,072 tokens, 12 full-attention layers, 2 KV heads
x d=256 in an NVFP4 paged cache (page 3,136, random block tables), one query
row per sequence with 2,048 sorted selected tokens.  Each rank owns its own
96 sequences; there is no data-path collective.  One step = one decode step
(12 layers) = 12 reader launches, replayed from a CUDA graph.  The 12 layers'
selected records (1.36 GB) exceed L2 (126 MB), so every step streams from HBM.

Reported: value (GB/s of algorithmic bytes, all ranks) with the reader's
roofline against the measured HBM copy bandwidth; e2e (same metric through the
public API with pinned host inputs/outputs copied inside the timed region);
the writer on the prefill configuration (8,192 tokens into 64 x 3,136);
cpu_baseline (the C oracle on a bounded sample, rank 0, N=1).
`--impl reference` times the reference algorithm's CPU restatement (oracle/)
on this host -- the reference itself is Python+Triton with no compiled CPU path.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "nvfp4-qsa_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

HEAD_DIM, KV_HEADS, QUERY_HEADS, RECORD = 256, 2, 24, 288
METRIC = "NVFP4 sparse-decode KV read GB/s"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seqs", type=int, default=96)
    ap.add_argument("--context", type=int, default=131072)
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--topk", type=int, default=2048)
    ap.add_argument("--page", type=int, default=3136)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--split-context", type=int, default=169984, help="split-KV section: one sequence of this length")
    ap.add_argument("--split-topk", type=int, default=8192, help="split-KV section: selected tokens per row")
    ap.add_argument("--skip-split", action="store_true", help="skip the split-KV section")
    ap.add_argument("--skip-mtp", action="store_true", help="skip the MTP (config 4) section")
    ap.add_argument("--skip-fp8", action="store_true", help="skip the FP8 sibling-reader section")
    ap.add_argument("--skip-bf16", action="store_true", help="skip the BF16 sibling-reader section")
    ap.add_argument("--skip-proj", action="store_true", help="skip the fused K/V projection section")
    return ap.parse_args()


def read_bytes(rows, topk, layers):
    """Algorithmic bytes of one reader step: unique records + indices + q + out."""
    return layers * (rows * KV_HEADS * topk * RECORD + rows * topk * 4 + rows * QUERY_HEADS * HEAD_DIM * 2 * 2)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 TFLOP/s: the measured burst figure (a kernel timed in isolation), else the fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of each timed kernel, from one ncu
# capture of that kernel on its bench workload shape; the command of each capture is given in the ncu
# summary of that kernel.  Reported as roofline.traffic beside the algorithmic bytes.
NCU_TRAFFIC = {
    "read": 157334784,         # sparse_attention_kernel<0>, 96 rows x 2 KV heads x top-2048 (one layer)
    "mtp": 19777280,           # sparse_attention_mtp_kernel, config 4 (12 x 4 rows, top-2048)
    "fp8": 210388736,          # sparse_attention_kernel<3>, 96 rows x top-2048, FP8 K/V
    "write": 16863744,         # write_cache_group_kernel, 8,192 tokens into 64 x 3,136
    "fused_write": 18579712,   # write_cache_kernel<256,...,FUSE>, 8,192 tokens
    "bf16": 413479424,         # sparse_attention_bf16_kernel, 96 rows x top-2048 (48-row capture x 2)
    "topk": 50476800,          # topk_indices_kernel, 96 rows x 131,072 scores, k = 2048
    "kv_proj": 79862272,       # kv_proj_write_kernel<2>, 8,192 tokens x hidden 4,096 -> 1,024 K|V columns
}


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, read-only)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x1: "gpu_idle"}

    def __init__(self, torch_device):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            props = torch.cuda.get_device_properties(torch_device)
            self._nvml = pynvml
            try:
                uuid = str(props.uuid)
                self._handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # clocks are reported as unavailable, never fatal
            self.error = f"{type(exc).__name__}: {exc}"

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                for bit, name in self.REASONS.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._handle is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._handle is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if self._handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "error", "")}
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2] if s else None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(s)}


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
def build_workload(args, device, seed):
    """Per-rank NVFP4 caches (written by our writer), block tables, selections, queries."""
    import torch
    from nvfp4_qsa import kernels

    seqs, ctx, page, layers, topk = args.seqs, args.context, args.page, args.layers, args.topk
    width = (ctx + page - 1) // page
    blocks = seqs * width
    gen = torch.Generator(device=device).manual_seed(seed)
    L = []
    chunk = 1 << 20
    for layer in range(layers):
        storage = torch.empty(blocks, KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        parts = storage.transpose(1, 2).split(HEAD_DIM // 2 + HEAD_DIM // 16, dim=-1)
        kd, ks = parts[0].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        vd, vs = parts[1].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        total = blocks * page
        for s0 in range(0, total, chunk):
            n = min(chunk, total - s0)
            kv = torch.randn(2, n, KV_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=gen)
            slots = torch.arange(s0, s0 + n, device=device, dtype=torch.int64)
            kernels.qsa_write_cache_nvfp4(kv[0], kv[1], kd, ks, vd, vs, slots, 1.0, 1.0)
        table = torch.randperm(blocks, device=device, generator=gen).to(torch.int32).view(seqs, width).contiguous()
        idx = torch.rand(seqs, ctx, device=device, generator=gen).topk(topk, dim=1).indices
        idx = idx.sort(dim=1).values.to(torch.int32).contiguous()
        q = torch.randn(seqs, QUERY_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=gen)
        L.append(dict(storage=storage, kd=kd, ks=ks, vd=vd, vs=vs, table=table, idx=idx, q=q,
                      out=torch.empty_like(q)))
    t2r = torch.arange(seqs, device=device, dtype=torch.int32)
    torch.cuda.synchronize(device)
    return L, t2r


def run_step(L, t2r, q_override=None, idx_override=None):
    from nvfp4_qsa import kernels
    for i, d in enumerate(L):
        q = d["q"] if q_override is None else q_override[i]
        idx = d["idx"] if idx_override is None else idx_override[i]
        kernels.qsa_sparse_paged_attention_nvfp4(q, d["kd"], d["ks"], d["vd"], d["vs"], 1.0, 1.0, idx, d["table"],
                                                 t2r, d["out"])


def timed(fn, steps, device):
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / 1e3


def bench_write(device, steps):
    """Writer on the prefill configuration: 8,192 tokens x (K+V) into a 64 x 3,136 cache."""
    import torch
    from nvfp4_qsa import kernels
    from nvfp4_qsa import workloads as W

    tokens, blocks, page, sets = 8192, 64, 3136, 8  # 8 input sets: 134 MB of inputs > L2
    gen = torch.Generator(device=device).manual_seed(99)
    bufs = []
    for i in range(sets):
        kv = torch.randn(2, tokens, KV_HEADS, HEAD_DIM, device=device, generator=gen)
        kv = torch.where(torch.rand(kv.shape, device=device, generator=gen) < 0.02, kv * 32, kv).to(torch.bfloat16)
        storage = torch.zeros(blocks, KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        parts = storage.transpose(1, 2).split(HEAD_DIM // 2 + HEAD_DIM // 16, dim=-1)
        kd, ks = parts[0].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        vd, vs = parts[1].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        slots = torch.randperm(blocks * page, device=device, generator=gen)[:tokens].contiguous()
        bufs.append((kv[0], kv[1], kd, ks, vd, vs, slots))

    def one_round():
        for b in bufs:
            kernels.qsa_write_cache_nvfp4(*b, 1.0, 1.0)

    one_round()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        one_round()
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        one_round()
    for _ in range(3):
        graph.replay()
    rounds = max(20, steps)
    secs = timed(graph.replay, rounds, device)
    launches = rounds * sets
    per_launch = secs / launches
    algo = tokens * (KV_HEADS * HEAD_DIM * 2 * 2 + 8 + KV_HEADS * RECORD)
    peak, kind = measured_peaks()
    # CPU baseline for the writer: the oracle restatement on one prefill batch (port).
    del W
    return {
        "config": {"workload": "prefill: 8192 tokens bf16 K/V [8192,2,256], 2% x32 outliers, into a 64 x 3136 "
                               "NVFP4 cache at random free slots; 8 rotating buffer sets (inputs > L2)",
                   "launches": launches},
        "tokens_per_s": tokens / per_launch,
        "gb_per_s": algo / per_launch / 1e9,
        "us_per_launch": per_launch * 1e6,
        "roofline": {"bound": "hbm", "achieved": algo / per_launch / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": algo / per_launch / 1e9 / peak, "peak_kind": kind,
                     "algorithmic_bytes_per_launch": algo,
                     "traffic": NCU_TRAFFIC["write"]},
        "gpu_launches": launches,
    }


def bench_fused_write(device, steps):
    """Fused k-norm -> RoPE -> NVFP4 writer on the prefill configuration (8,192 projection rows).

    K and V as they leave the QKV projection (before GemmaRMSNorm and a 64-dim NeoX rotary of Qwen3-Next's
    shape) are normed, rotated, quantised and scattered by nvqsa_norm_rope_write_cache into a 64 x 3,136 cache;
    once without and once with the rotated bf16 K written back (key_out).  8 rotating input sets (> L2)
    per CUDA-graph round, like the plain writer's section.
    """
    import torch
    from nvfp4_qsa import kernels
    from nvfp4_qsa import workloads as W

    tokens, blocks, page, sets, rot, max_pos = 8192, 64, 3136, 8, 64, 262144
    gen = torch.Generator(device=device).manual_seed(98)
    cos_sin = torch.from_numpy(W.rope_cos_sin(max_pos, rot)).to(device=device, dtype=torch.bfloat16)
    weight = (torch.randn(HEAD_DIM, device=device, generator=gen) * 0.1).to(torch.bfloat16).float()
    bufs = []
    for i in range(sets):
        kv = torch.randn(2, tokens, KV_HEADS, HEAD_DIM, device=device, generator=gen)
        kv[0] *= torch.exp2(torch.rand(tokens, KV_HEADS, 1, device=device, generator=gen) * 4 - 1)
        kv = torch.where(torch.rand(kv.shape, device=device, generator=gen) < 0.02, kv * 32, kv).to(torch.bfloat16)
        storage = torch.zeros(blocks, KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        parts = storage.transpose(1, 2).split(HEAD_DIM // 2 + HEAD_DIM // 16, dim=-1)
        kd, ks = parts[0].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        vd, vs = parts[1].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        slots = torch.randperm(blocks * page, device=device, generator=gen)[:tokens].contiguous()
        pos = torch.randint(0, max_pos, (tokens,), device=device, generator=gen)
        bufs.append((kv[0], kv[1], kd, ks, vd, vs, slots, pos, torch.empty_like(kv[0])))

    def measure(with_key_out):
        def one_round():
            for k, v, kd, ks, vd, vs, slots, pos, ko in bufs:
                kernels.qsa_norm_rope_write_cache_nvfp4(k, v, kd, ks, vd, vs, slots, 1.0, 1.0, positions=pos,
                                                        cos_sin_cache=cos_sin, k_norm_weight=weight, eps=1e-6,
                                                        key_out=ko if with_key_out else None)

        one_round()
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            one_round()
        torch.cuda.current_stream(device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_round()
        for _ in range(3):
            graph.replay()
        rounds = max(20, steps)
        secs = timed(graph.replay, rounds, device)
        del graph
        return secs / (rounds * sets), rounds * sets

    per_launch, launches = measure(False)
    per_launch_ko, launches_ko = measure(True)
    # per token: K and V bf16 in (2,048 B), slot + position (16 B), the position's cos/sin row (128 B),
    # two 288-byte records out; key_out adds the rotated K (1,024 B)
    algo = tokens * (KV_HEADS * HEAD_DIM * 2 * 2 + 16 + rot * 2 + KV_HEADS * RECORD)
    algo_ko = algo + tokens * KV_HEADS * HEAD_DIM * 2
    peak, kind = measured_peaks()
    return {
        "config": {"workload": "prefill projection rows: 8192 tokens bf16 K/V [8192,2,256] before k_norm and RoPE "
                               "(GemmaRMSNorm, NeoX rotary 64 of 256, positions U[0, 262144)), into a 64 x 3136 "
                               "NVFP4 cache at random free slots; 8 rotating buffer sets (inputs > L2)",
                   "launches": launches + launches_ko},
        "us_per_launch": per_launch * 1e6,
        "gb_per_s": algo / per_launch / 1e9,
        "us_per_launch_key_out": per_launch_ko * 1e6,
        "gb_per_s_key_out": algo_ko / per_launch_ko / 1e9,
        "roofline": {"bound": "hbm", "achieved": algo / per_launch / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": algo / per_launch / 1e9 / peak, "peak_kind": kind,
                     "kernel": "write_cache_kernel<256, true, true, true> (fused k-norm + RoPE, no key_out)",
                     "algorithmic_bytes_per_launch": algo,
                     "traffic": NCU_TRAFFIC["fused_write"]},
        "gpu_launches": launches + launches_ko,
    }


def bench_kv_proj_write(device, steps):
    """K/V projection GEMM fused with k-norm, RoPE, NVFP4 quantisation and the scatter, against the chain it
    replaces (cuBLAS projection into bf16 K|V, then the fused norm/RoPE writer), on the prefill configuration.

    8,192 tokens, hidden size 4,096 (the reference's architecture file gives no hidden size; 4,096 is assumed),
    2 KV heads x 256 for K and for V (1,024 output columns), GemmaRMSNorm and a 64-dim NeoX rotary, into a
    64 x 3,136 cache.  3 rotating sets of hidden states and weights (216 MB > L2) per CUDA-graph round.
    """
    import torch
    from nvfp4_qsa import kernels
    from nvfp4_qsa import workloads as W

    tokens, hidden, blocks, page, sets, rot, max_pos = 8192, 4096, 64, 3136, 3, 64, 262144
    cols = 2 * KV_HEADS * HEAD_DIM
    gen = torch.Generator(device=device).manual_seed(77)
    cos_sin = torch.from_numpy(W.rope_cos_sin(max_pos, rot)).to(device=device, dtype=torch.bfloat16)
    weight = (torch.randn(HEAD_DIM, device=device, generator=gen) * 0.1).to(torch.bfloat16).float()
    bufs = []
    for i in range(sets):
        x = torch.randn(tokens, hidden, device=device, generator=gen).to(torch.bfloat16)
        wkv = (torch.randn(cols, hidden, device=device, generator=gen) * hidden ** -0.5).to(torch.bfloat16)
        storage = torch.zeros(blocks, KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        parts = storage.transpose(1, 2).split(HEAD_DIM // 2 + HEAD_DIM // 16, dim=-1)
        kd, ks = parts[0].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        vd, vs = parts[1].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        slots = torch.randperm(blocks * page, device=device, generator=gen)[:tokens].contiguous()
        pos = torch.randint(0, max_pos, (tokens,), device=device, generator=gen)
        kv = torch.empty(tokens, cols, device=device, dtype=torch.bfloat16)
        bufs.append((x, wkv, (kd, ks, vd, vs), slots, pos, kv))

    def fused_round():
        for x, wkv, regs, slots, pos, _ in bufs:
            kernels.qsa_kv_proj_write_cache_nvfp4(x, wkv[:cols // 2], wkv[cols // 2:], *regs, slots, 1.0, 1.0,
                                                  positions=pos, cos_sin_cache=cos_sin, k_norm_weight=weight,
                                                  eps=1e-6)

    def chain_round():
        for x, wkv, regs, slots, pos, kv in bufs:
            torch.mm(x, wkv.t(), out=kv)
            k = kv[:, :cols // 2].view(-1, KV_HEADS, HEAD_DIM)
            v = kv[:, cols // 2:].view(-1, KV_HEADS, HEAD_DIM)
            kernels.qsa_norm_rope_write_cache_nvfp4(k, v, *regs, slots, 1.0, 1.0, positions=pos,
                                                    cos_sin_cache=cos_sin, k_norm_weight=weight, eps=1e-6)

    def gemm_round():
        for x, wkv, _, _, _, kv in bufs:
            torch.mm(x, wkv.t(), out=kv)

    def measure(body):
        body()
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            body()
        torch.cuda.current_stream(device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            body()
        for _ in range(3):
            graph.replay()
        rounds = max(10, steps // 4)
        secs = timed(graph.replay, rounds, device)
        del graph
        return secs / (rounds * sets), rounds * sets

    fused, launches = measure(fused_round)
    chain, _ = measure(chain_round)
    gemm, _ = measure(gemm_round)
    # a decode-size batch (96 tokens, the config-5a row count) through both paths, same buffers
    full = bufs
    bufs = [(x[:96], wkv, regs, slots[:96], pos[:96], kv[:96]) for x, wkv, regs, slots, pos, kv in full]
    fused96, launches96 = measure(fused_round)
    chain96, _ = measure(chain_round)
    bufs = full
    flops = 2.0 * tokens * hidden * cols
    peak, kind = measured_tensor_peak()
    achieved = flops / fused / 1e12
    return {
        "config": {"workload": "prefill: hidden [8192, 4096] bf16 x K|V weight [1024, 4096] bf16 (2 KV heads x 256 "
                               "each), GemmaRMSNorm + NeoX rotary 64 of 256 on K, NVFP4 into a 64 x 3136 cache at "
                               "random free slots; 3 rotating sets of hidden states and weights (inputs > L2)",
                   "hidden_size_assumed": hidden, "launches": launches},
        "us_per_launch": fused * 1e6,
        "tflops": achieved,
        "unfused_us": chain * 1e6,
        "unfused": "torch.mm (cuBLAS) into bf16 K|V [8192, 1024], then nvqsa_norm_rope_write_cache",
        "cublas_gemm_only_us": gemm * 1e6,
        "speedup_vs_unfused": chain / fused,
        "decode_96_tokens": {"us_per_launch": fused96 * 1e6, "unfused_us": chain96 * 1e6,
                             "what": "the same call on the first 96 tokens: 4 tiles, each k-loop split over a cluster of 8 CTAs"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_kind": kind, "kernel": "kv_proj_write_kernel",
                     "algorithmic_flops_per_launch": flops, "traffic": NCU_TRAFFIC["kv_proj"],
                     "algorithmic_bytes_per_launch": tokens * hidden * 2 + cols * hidden * 2 + tokens * (
                         16 + rot * 2 + KV_HEADS * RECORD)},
        "gpu_launches": launches + launches96,
    }


def bench_mtp(args, device, steps):
    """Config 4: MTP=3 decode batch, 12 sequences x 4 rows sharing each sequence's 2,048 selections.

    Contexts U[8,192, 169,984] (seeded), page 3,136, random block tables, 12 layers (one cache each) replayed
    from one CUDA graph per step.  The grouped reader (rows_per_group=4: one gather and dequantisation per record
    for the four rows) and the per-row reader run on the same inputs; bytes are the unique records of the step.
    """
    import numpy as np
    import torch
    from nvfp4_qsa import kernels

    seqs, rows_per_seq, topk, page, layers = 12, 4, 2048, args.page, args.layers
    rng = np.random.default_rng(2024)
    contexts = rng.integers(8192, 169984 + 1, size=seqs)
    widths = [(int(cx) + page - 1) // page for cx in contexts]
    width = max(widths)
    blocks = sum(widths)
    gen = torch.Generator(device=device).manual_seed(4)
    rows = seqs * rows_per_seq
    L = []
    for layer in range(layers):
        storage = torch.empty(blocks, KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        parts = storage.transpose(1, 2).split(HEAD_DIM // 2 + HEAD_DIM // 16, dim=-1)
        kd, ks = parts[0].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        vd, vs = parts[1].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        total, chunk = blocks * page, 1 << 20
        for s0 in range(0, total, chunk):
            n = min(chunk, total - s0)
            kv = torch.randn(2, n, KV_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=gen)
            kernels.qsa_write_cache_nvfp4(kv[0], kv[1], kd, ks, vd, vs,
                                          torch.arange(s0, s0 + n, device=device, dtype=torch.int64), 1.0, 1.0)
        perm = torch.randperm(blocks, device=device, generator=gen).to(torch.int32)
        table = torch.full((seqs, width), -1, dtype=torch.int32, device=device)
        b0 = 0
        for i, w in enumerate(widths):
            table[i, :w] = perm[b0:b0 + w]
            b0 += w
        sel = []
        for cx in contexts:
            sel.append(torch.rand(int(cx), device=device, generator=gen).topk(topk).indices.sort().values)
        idx = torch.stack(sel).to(torch.int32).repeat_interleave(rows_per_seq, dim=0).contiguous()
        q = torch.randn(rows, QUERY_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=gen)
        L.append(dict(regions=(kd, ks, vd, vs), table=table, idx=idx, q=q, out=torch.empty_like(q)))
    t2r = torch.arange(seqs, device=device, dtype=torch.int32).repeat_interleave(rows_per_seq).contiguous()
    torch.cuda.synchronize(device)

    def step(group):
        for d in L:
            kernels.qsa_sparse_paged_attention_nvfp4(d["q"], *d["regions"], 1.0, 1.0, d["idx"], d["table"], t2r,
                                                     d["out"], rows_per_group=group)

    times = {}
    for group in (4, 1):
        step(group)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            step(group)
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(group)
        for _ in range(3):
            graph.replay()
        reps = max(20, steps)
        times[group] = timed(graph.replay, reps, device) / reps / layers
        del graph
    # where a grouped layer's time goes: %globaltimer stamps per (group, kv head), one graph-replayed step
    units = seqs * KV_HEADS
    stamps = torch.zeros(layers, units, kernels.STAMP_SLOTS, dtype=torch.int64, device=device)

    def stamped():
        for li, d in enumerate(L):
            kernels.reset_stamps(stamps[li])
            kernels.set_stamp_buffer(stamps[li])
            kernels.qsa_sparse_paged_attention_nvfp4(d["q"], *d["regions"], 1.0, 1.0, d["idx"], d["table"], t2r,
                                                     d["out"], rows_per_group=4)
        kernels.set_stamp_buffer(None)

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        stamped()
    torch.cuda.current_stream(device).wait_stream(side)
    sgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(sgraph):
        stamped()
    for _ in range(4):
        sgraph.replay()
    torch.cuda.synchronize(device)
    del sgraph
    st = stamps.double()
    layer_start = st[..., 0].min(dim=1).values  # first CTA of the launch
    phases = {"prologue": ((st[..., 2] - st[..., 0]).mean() / 1e3).item(),
              "tiles": ((st[..., 1] - st[..., 2]).mean() / 1e3).item(),
              "cluster_merge_store": ((st[..., 6] - st[..., 1]).mean() / 1e3).item(),
              "launch_span": ((st[..., 6].max(dim=1).values - layer_start).mean() / 1e3).item()}
    records = seqs * KV_HEADS * topk * RECORD
    algo = records + rows * topk * 4 + 2 * rows * QUERY_HEADS * HEAD_DIM * 2
    peak, kind = measured_peaks()
    g4, g1 = times[4], times[1]
    return {
        "config": {"workload": "MTP=3 decode (config 4): 12 sequences x 4 rows sharing 2048 sorted selections per "
                               "sequence, contexts U[8192, 169984], page 3136, 24 query heads over 2 KV heads, "
                               f"{layers} layers (one cache each) in one CUDA graph per step",
                   "l2": f"inputs larger than L2 over a step: {layers} layers x {records / 1e6:.1f} MB of records"},
        "us_per_layer": g4 * 1e6,
        "gb_per_s": algo / g4 / 1e9,
        "per_row_us_per_layer": g1 * 1e6,
        "per_row_gb_per_s": algo / g1 / 1e9,
        "speedup_vs_per_row": g1 / g4,
        "phases_us": {"what": "grouped reader, graph-replayed step with %globaltimer stamps per (group, kv head): "
                              "first CTA entry -> last CTA past its prologue -> last CTA done with its tiles -> "
                              "last CTA stored; mean over layers and units; launch_span = first entry to last store",
                      **{k: round(v, 2) for k, v in phases.items()}},
        "roofline": {"bound": "hbm", "achieved": algo / g4 / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": algo / g4 / 1e9 / peak, "peak_kind": kind,
                     "kernel": "sparse_attention_mtp_kernel (one layer, splits merged in a cluster)",
                     "algorithmic_bytes_per_launch": algo,
                     "traffic": NCU_TRAFFIC["mtp"]},
        "gpu_launches": 2 * (max(20, steps) + 5) * layers,
    }


def bench_fp8(args, device, steps):
    """FP8 sibling reader (src/qsa_fp8_harness.py:42-208) on the config-5a row shape.

    96 rows x 2 KV heads x top-2,048 over float8_e4m3 K and V caches [blocks, page, 2, 256] (one per layer,
    context 32,768 so that 12 layers fit beside the NVFP4 workload: 201 MB of selected rows per layer, more
    than L2), 12 layers replayed from one CUDA graph per step.  Bytes: the selected K and V rows (512 B per
    row and KV head), indices, q and out.
    """
    import torch
    from nvfp4_qsa import kernels

    seqs, ctx, page, layers, topk = args.seqs, 32768, args.page, args.layers, args.topk
    width = (ctx + page - 1) // page
    blocks = seqs * width
    gen = torch.Generator(device=device).manual_seed(8)
    L = []
    for layer in range(layers):
        kc = torch.empty(blocks, page, KV_HEADS, HEAD_DIM, dtype=torch.float8_e4m3fn, device=device)
        vc = torch.empty_like(kc)
        for b0 in range(0, blocks, 64):
            b1 = min(blocks, b0 + 64)
            kc[b0:b1] = torch.randn(b1 - b0, page, KV_HEADS, HEAD_DIM, device=device, generator=gen).to(kc.dtype)
            vc[b0:b1] = torch.randn(b1 - b0, page, KV_HEADS, HEAD_DIM, device=device, generator=gen).to(vc.dtype)
        table = torch.randperm(blocks, device=device, generator=gen).to(torch.int32).view(seqs, width).contiguous()
        idx = torch.rand(seqs, ctx, device=device, generator=gen).topk(topk, dim=1).indices
        idx = idx.sort(dim=1).values.to(torch.int32).contiguous()
        q = torch.randn(seqs, QUERY_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=gen)
        L.append(dict(kc=kc, vc=vc, table=table, idx=idx, q=q, out=torch.empty_like(q)))
    t2r = torch.arange(seqs, device=device, dtype=torch.int32)
    torch.cuda.synchronize(device)

    def step():
        for d in L:
            kernels.qsa_sparse_paged_attention_fp8(d["q"], d["kc"], d["vc"], 1.0, 1.0, d["idx"], d["table"], t2r,
                                                   d["out"])

    step()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    reps = max(20, steps)
    per_layer = timed(graph.replay, reps, device) / reps / layers
    del graph
    algo = seqs * KV_HEADS * topk * 2 * HEAD_DIM + seqs * topk * 4 + 2 * seqs * QUERY_HEADS * HEAD_DIM * 2
    peak, kind = measured_peaks()
    return {
        "config": {"workload": f"FP8 sibling reader on the config-5a row shape: {seqs} rows x 2 KV heads x top-{topk} "
                               f"of {ctx} tokens, float8_e4m3 K and V caches, page {page}, {layers} layers (one "
                               "cache each) in one CUDA graph per step",
                   "l2": f"inputs larger than L2: {seqs * KV_HEADS * topk * 512 / 1e6:.0f} MB of selected rows per layer"},
        "us_per_layer": per_layer * 1e6,
        "gb_per_s": algo / per_layer / 1e9,
        "roofline": {"bound": "hbm", "achieved": algo / per_layer / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": algo / per_layer / 1e9 / peak, "peak_kind": kind,
                     "kernel": "sparse_attention_kernel<3> (one layer, FP8 rows)",
                     "algorithmic_bytes_per_launch": algo,
                     "traffic": NCU_TRAFFIC["fp8"]},
        "gpu_launches": (reps + 5) * layers,
    }


def bench_bf16(args, device, steps):
    """BF16 sibling reader (integration/snapshot/qsa.py:352-366) on the config-5a row shape.

    96 rows x 2 KV heads x top-2,048 over bf16 caches laid out as vLLM allocates them, [blocks, 2, page, 512]
    split into K and V views (context 16,384 per layer so that 12 layers fit beside the NVFP4 workload:
    403 MB of selected rows per layer, more than L2), 12 layers replayed from one CUDA graph per step.  Bytes:
    the selected K and V rows (1,024 B per row and KV head), indices, q and out.
    """
    import torch
    from nvfp4_qsa import kernels

    seqs, ctx, page, layers, topk = args.seqs, 16384, args.page, args.layers, args.topk
    width = (ctx + page - 1) // page
    blocks = seqs * width
    gen = torch.Generator(device=device).manual_seed(9)
    L = []
    for layer in range(layers):
        storage = torch.randn(blocks, KV_HEADS, page, 2 * HEAD_DIM, device=device, dtype=torch.bfloat16,
                              generator=gen)
        cache = storage.transpose(1, 2)
        table = torch.randperm(blocks, device=device, generator=gen).to(torch.int32).view(seqs, width).contiguous()
        idx = torch.rand(seqs, ctx, device=device, generator=gen).topk(topk, dim=1).indices
        idx = idx.sort(dim=1).values.to(torch.int32).contiguous()
        q = torch.randn(seqs, QUERY_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=gen)
        L.append(dict(storage=storage, kc=cache[..., :HEAD_DIM], vc=cache[..., HEAD_DIM:], table=table, idx=idx,
                      q=q, out=torch.empty_like(q)))
    t2r = torch.arange(seqs, device=device, dtype=torch.int32)
    torch.cuda.synchronize(device)

    def step():
        for d in L:
            kernels.qsa_sparse_paged_attention(d["q"], d["kc"], d["vc"], d["idx"], d["table"], t2r, d["out"])

    step()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    reps = max(20, steps)
    per_layer = timed(graph.replay, reps, device) / reps / layers
    del graph
    algo = seqs * KV_HEADS * topk * 4 * HEAD_DIM + seqs * topk * 4 + 2 * seqs * QUERY_HEADS * HEAD_DIM * 2
    peak, kind = measured_peaks()
    return {
        "config": {"workload": f"BF16 sibling reader on the config-5a row shape: {seqs} rows x 2 KV heads x "
                               f"top-{topk} of {ctx} tokens, bf16 caches [blocks, 2, page, 512] (K and V views), "
                               f"page {page}, {layers} layers (one cache each) in one CUDA graph per step",
                   "l2": f"inputs larger than L2: {seqs * KV_HEADS * topk * 1024 / 1e6:.0f} MB of selected rows per layer"},
        "us_per_layer": per_layer * 1e6,
        "gb_per_s": algo / per_layer / 1e9,
        "roofline": {"bound": "hbm", "achieved": algo / per_layer / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": algo / per_layer / 1e9 / peak, "peak_kind": kind,
                     "kernel": "sparse_attention_bf16_kernel (one layer)",
                     "algorithmic_bytes_per_launch": algo,
                     "traffic": NCU_TRAFFIC.get("bf16")},
        "gpu_launches": (reps + 5) * layers,
    }


def bench_topk(device, steps):
    """Indexer top-k (nvqsa_topk_indices): the decode selection of config 5a (96 rows x 131,072 scores) and of
    config 5b (1 row x 169,984), k = 2,048, eight rotating score buffers (more than L2 for 5a).  Algorithmic bytes:
    the scores (4 B each) read once and the indices (4 B each) written."""
    import torch
    from nvfp4_qsa import indexer

    res = {}
    for name, rows, ctx in (("5a", 96, 131072), ("5b", 1, 169984)):
        gen = torch.Generator(device=device).manual_seed(11)
        bufs = [torch.randn(rows, ctx, device=device, generator=gen) for _ in range(8)]
        out = torch.empty(rows, 2048, dtype=torch.int32, device=device)
        for b in bufs:
            indexer.qsa_select_topk(b, out)
        torch.cuda.synchronize(device)
        reps = max(40, steps)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(reps):
            indexer.qsa_select_topk(bufs[i % 8], out)
        end.record()
        end.synchronize()
        per = start.elapsed_time(end) / 1e3 / reps
        algo = rows * ctx * 4 + rows * 2048 * 4
        res[name] = {"rows": rows, "context": ctx, "k": 2048, "us_per_call": per * 1e6, "gb_per_s": algo / per / 1e9}
    peak, kind = measured_peaks()
    a = res["5a"]
    res["roofline"] = {"bound": "hbm", "achieved": a["gb_per_s"], "peak": peak, "unit": "GB/s",
                       "frac": a["gb_per_s"] / peak, "peak_kind": kind, "kernel": "topk_indices_kernel (96 rows)",
                       "algorithmic_bytes_per_launch": 96 * 131072 * 4 + 96 * 2048 * 4, "traffic": NCU_TRAFFIC["topk"]}
    res["gpu_launches"] = 2 * (max(40, steps) + 8)
    return res


def bench_split_kv(args, device, world, rank, steps):
    """Config 5b: one 169,984-token sequence, 8,192 selected per row, 12 layers, split-KV over the ranks.

    Every rank draws the same bf16 K/V and selections per layer (shared seeds) and writes only its contiguous
    share of the sequence's pages (nvfp4_qsa.distributed.SplitKV).  Per layer, one reader launch computes the
    rank's partial, pushes it into every rank's exchange buffer over NVLink and merges (``attend_fused``); the
    NCCL variant (``attend``: partial kernel, all_gather of the packed partials, merge kernel) is timed beside
    it.  At N=1 the step is the plain single-GPU reader.  Both the fused step and the N=1 reader are timed the
    same two ways at every N: eager launches, and the 12 layers replayed from one CUDA graph.  Device time with
    CUDA events, max over ranks.  Correctness: every rank's merged outputs of the last timed step are compared
    with the single-GPU reader over the whole sequence (max-abs and mean-abs over all layers and ranks).
    """
    import torch
    import torch.distributed as dist
    from nvfp4_qsa import distributed as D
    from nvfp4_qsa import kernels

    ctx, topk, page, layers = args.split_context, args.split_topk, args.page, args.layers
    pages = (ctx + page - 1) // page
    sk = D.SplitKV(pages, page, world, rank)
    shared = torch.Generator(device=device).manual_seed(777)  # K/V, indices and queries identical on every rank
    L = []
    positions = torch.arange(ctx, device=device)
    slots = sk.slot_mapping(positions) if world > 1 else positions
    t2r = torch.zeros(1, device=device, dtype=torch.int32)
    full_table = torch.arange(pages, device=device, dtype=torch.int32).view(1, -1)

    def regions_of(storage):
        parts = storage.transpose(1, 2).split(HEAD_DIM // 2 + HEAD_DIM // 16, dim=-1)
        kd, ks = parts[0].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        vd, vs = parts[1].split((HEAD_DIM // 2, HEAD_DIM // 16), dim=-1)
        return kd, ks, vd, vs

    for layer in range(layers):
        kv = torch.randn(2, ctx, KV_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=shared)
        idx = torch.rand(1, ctx, device=device, generator=shared).topk(topk, dim=1).indices
        idx = idx.sort(dim=1).values.to(torch.int32).contiguous()
        q = torch.randn(1, QUERY_HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16, generator=shared)
        # the single-GPU answer over the whole sequence, for the correctness check
        whole = torch.zeros(pages, KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        kernels.qsa_write_cache_nvfp4(kv[0], kv[1], *regions_of(whole), positions, 1.0, 1.0)
        ref = torch.empty_like(q)
        kernels.qsa_sparse_paged_attention_nvfp4(q, *regions_of(whole), 1.0, 1.0, idx, full_table, t2r, ref)
        del whole
        nblk = sk.local_blocks if world > 1 else pages
        storage = torch.zeros(max(nblk, 1), KV_HEADS, page, RECORD, dtype=torch.uint8, device=device)
        regs = regions_of(storage)
        kernels.qsa_write_cache_nvfp4(kv[0], kv[1], *regs, slots, 1.0, 1.0)
        del kv
        table = sk.block_table(device) if world > 1 else full_table
        L.append(dict(regions=regs, idx=idx, q=q, table=table, out=torch.empty_like(q), ref=ref,
                      buf=sk.partial_buffer(1, QUERY_HEADS, HEAD_DIM, device)))
    exchange = D.PeerExchange(1, QUERY_HEADS, KV_HEADS) if world > 1 else None
    assert exchange is None or layers % 2 == 0  # a graph replays the exchange parities of an even layer count

    def step():  # fused: the exchange over NVLink peer memory inside the reader kernel
        for d in L:
            if world > 1:
                sk.attend_fused(d["q"], *d["regions"], 1.0, 1.0, d["idx"], t2r, d["out"], exchange,
                                block_table=d["table"])
            else:
                kernels.qsa_sparse_paged_attention_nvfp4(d["q"], *d["regions"], 1.0, 1.0, d["idx"], d["table"], t2r,
                                                         d["out"])

    def step_nccl():  # partial kernel, NCCL all_gather of the packed partials, merge kernel
        for d in L:
            sk.attend(d["q"], *d["regions"], 1.0, 1.0, d["idx"], t2r, d["out"], block_table=d["table"],
                      buffer=d["buf"])

    def check():
        err = torch.zeros(2, device=device, dtype=torch.float64)
        for d in L:
            diff = (d["out"].float() - d["ref"].float()).abs()
            err[0] = torch.maximum(err[0], diff.max().double())
            err[1] += diff.mean().double() / len(L)
        if world > 1:
            dist.all_reduce(err, op=dist.ReduceOp.MAX)
        return {"max_abs": float(err[0].item()), "mean_abs": float(err[1].item()), "vs": "single-GPU reader"}

    def sync_all():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    n = max(10, steps // 4)
    for _ in range(3):
        step()
    sync_all()
    eager_secs = max_over_ranks(timed(step, n, device))
    sync_all()
    # the same step captured once and replayed (no NCCL call inside: only the fused reader launches)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream(device).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    sync_all()
    secs = max_over_ranks(timed(graph.replay, n, device))
    sync_all()
    del graph
    fused_check = check()

    # Where a layer's time goes (the same eager step, once, with the readers' %globaltimer stamps on):
    # per (row, kv head) unit, averaged over layers and units, max over ranks.
    units = KV_HEADS  # one row
    stamps = torch.zeros(layers, units, kernels.STAMP_SLOTS, dtype=torch.int64, device=device)

    def stamped_step():  # each layer's launch carries its own stamp buffer (read at launch / capture time)
        for li, d in enumerate(L):
            kernels.reset_stamps(stamps[li])
            kernels.set_stamp_buffer(stamps[li])
            if world > 1:
                sk.attend_fused(d["q"], *d["regions"], 1.0, 1.0, d["idx"], t2r, d["out"], exchange,
                                block_table=d["table"])
            else:
                kernels.qsa_sparse_paged_attention_nvfp4(d["q"], *d["regions"], 1.0, 1.0, d["idx"], d["table"],
                                                         t2r, d["out"])
        kernels.set_stamp_buffer(None)

    # steady state: the stamped step captured once and replayed like the timed graph
    s2 = torch.cuda.Stream(device)
    s2.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s2):
        stamped_step()
    torch.cuda.current_stream(device).wait_stream(s2)
    sgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(sgraph):
        stamped_step()
    for _ in range(5):
        sgraph.replay()
    sync_all()
    for _ in range(3):
        sgraph.replay()
    torch.cuda.synchronize(device)
    del sgraph
    st = stamps.double()

    def span(a, b):
        return ((st[..., b] - st[..., a]).mean() / 1e3).item()

    phases = torch.tensor([span(0, 1), span(1, 2), span(2, 3), span(3, 4) if world > 1 else 0.0,
                           span(4, 5) if world > 1 else 0.0, span(5 if world > 1 else 3, 6), span(0, 6)],
                          device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(phases, op=dist.ReduceOp.MAX)
    stamp_us = dict(zip(["tiles", "parts_in", "local_merge", "push_to_peers", "peer_wait", "final_merge_store",
                         "kernel"], [round(x, 2) for x in phases.tolist()]))
    nccl_secs, nccl_check = None, None
    if world > 1:
        for _ in range(3):
            step_nccl()
        sync_all()
        nccl_secs = max_over_ranks(timed(step_nccl, n, device))
        sync_all()
        nccl_check = check()
        exchange.close()
    per_layer_bytes = KV_HEADS * topk * RECORD + topk * 4 + 2 * QUERY_HEADS * HEAD_DIM * 2
    return {
        "config": {"workload": f"split-KV decode (config 5b): one sequence of {ctx} tokens, {topk} selected per row, "
                               f"{layers} layers, page {page}, pages split contiguously over {world} GPU(s); "
                               "per layer one reader launch whose last CTA per (row, kv head) pushes its partial "
                               "into every rank's exchange buffer over NVLink and merges; one GPU: the plain "
                               "reader. Timed as a CUDA graph of the 12 layers and as eager launches.",
                   "scaling": "strong"},
        "ms_per_step": secs / n * 1e3,
        "us_per_layer": secs / n / layers * 1e6,
        "us_per_layer_eager": eager_secs / n / layers * 1e6,
        "gb_per_s": per_layer_bytes * layers * n / secs / 1e9,
        "exchange_bytes_per_rank_per_layer": L[0]["buf"].numel() * 4 if world > 1 else 0,
        "nccl_us_per_layer": nccl_secs / n / layers * 1e6 if nccl_secs is not None else None,
        "check": fused_check,
        "nccl_check": nccl_check,
        "phases_us": {"what": "graph-replayed step with the readers' %globaltimer stamps: first CTA entry -> last CTA done "
                              "with its tiles -> last split part in -> local merge -> partial pushed to the peers -> "
                              "every peer's partial seen -> stored; mean over layers and (row, kv head), max over "
                              "ranks", **stamp_us},
    }


def cpu_baseline_read(args, budget_s):
    """C oracle (float64) over a bounded sample of the decode workload; rank 0 only."""
    import numpy as np
    import torch
    import oracle

    page, ctx, topk = args.page, args.context, args.topk
    width = (ctx + page - 1) // page
    nseq = 4  # distinct sequences in the host-side sample cache
    blocks = nseq * width
    gen = torch.Generator().manual_seed(7)
    storage = np.zeros((blocks, KV_HEADS, page, RECORD), np.uint8)
    total = blocks * page
    chunk = 1 << 18
    rng = np.random.default_rng(7)
    for s0 in range(0, total, chunk):
        n = min(chunk, total - s0)
        kv = torch.randn(2, n, KV_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16).view(torch.int16).numpy()
        oracle.write_cache(kv[0].view(np.uint16), kv[1].view(np.uint16), storage,
                           np.arange(s0, s0 + n, dtype=np.int64))
    table = rng.permutation(blocks).astype(np.int32).reshape(nseq, width)
    threads = oracle.get_threads()
    rows_done, secs = 0, 0.0
    batch = max(threads, 8)
    while secs < budget_s:
        q = torch.randn(batch, QUERY_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16).view(torch.int16).numpy()
        idx = np.stack([np.sort(rng.choice(ctx, topk, replace=False)) for _ in range(batch)]).astype(np.int32)
        t2r = (np.arange(batch) % nseq).astype(np.int32)
        t0 = time.perf_counter()
        oracle.sparse_attention(q.view(np.uint16), storage, idx, table, t2r)
        secs += time.perf_counter() - t0
        rows_done += batch
    per_row_bytes = read_bytes(1, topk, 1)
    return {"value": rows_done * per_row_bytes / secs / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle/nvfp4_oracle.c float64 reader over {rows_done} decode rows (2 KV heads x {topk} "
                      f"selected of {ctx} tokens, page {page}) in {secs:.1f} s on {threads} OpenMP threads"}


def cpu_baseline_write(fused, budget_s):
    """C oracle restatement of the writer (fused: k-norm + rotation first) on prefill batches; rank 0 only."""
    import numpy as np
    import oracle
    from nvfp4_qsa import workloads as W

    tokens, blocks, page, rot = 8192, 64, 3136, 64
    kb, vb, slots, pos, cs, w = W.projection_config(seed=21, tokens=tokens, blocks=blocks, page=page,
                                                    max_position=65536, rotary_dim=rot)
    csb = W.f32_to_bf16_bits(cs)
    storage = np.zeros((blocks, KV_HEADS, page, RECORD), np.uint8)
    threads = oracle.get_threads()
    done, secs = 0, 0.0
    while secs < budget_s or done == 0:
        t0 = time.perf_counter()
        k = oracle.norm_rope(kb, pos, csb, w)[0] if fused else kb
        oracle.write_cache(k, vb, storage, slots)
        secs += time.perf_counter() - t0
        done += tokens
    per_token = KV_HEADS * HEAD_DIM * 2 * 2 + 8 + KV_HEADS * RECORD + ((8 + rot * 2) if fused else 0)
    what = "k-norm + rotation + writer" if fused else "writer"
    return {"value": done * per_token / secs / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle/nvfp4_oracle.c {what} over {done} tokens (8,192-token prefill batches into a "
                      f"64 x 3,136 cache) in {secs:.1f} s on {threads} OpenMP threads"}


def main_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    from nvfp4_qsa import kernels

    L, t2r = build_workload(args, device, seed=1000 + rank)
    # warm-up eager, then capture one decode step (12 layers) into a CUDA graph
    run_step(L, t2r)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        run_step(L, t2r)
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run_step(L, t2r)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    with ClockSampler(device) as clocks:
        secs = timed(graph.replay, args.steps, device)
    if world > 1:
        t = torch.tensor([secs], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    step_bytes = read_bytes(args.seqs, args.topk, args.layers)
    value = world * step_bytes * args.steps / secs / 1e9
    launches_per_layer = 1  # sparse_attention_kernel (split-KV merge fused; plus a counter memset when split)
    per_layer = secs / args.steps / args.layers
    peak, kind = measured_peaks()
    achieved = step_bytes / args.layers / per_layer / 1e9

    # e2e: every step copies each layer's queries and selections from pinned host memory, runs the public
    # API call on them and copies the layer's output back to pinned host memory.  The copies of layer i+1
    # in and of layer i-1 out run on two copy streams while layer i computes (full-duplex PCIe).
    qh = torch.stack([d["q"] for d in L]).cpu().pin_memory()
    ih = torch.stack([d["idx"] for d in L]).cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    qd, idd = torch.empty_like(qh, device=device), torch.empty_like(ih, device=device)
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in L]
    ev_done = [torch.cuda.Event() for _ in L]
    ev_back = [torch.cuda.Event() for _ in L]

    def e2e_step():
        comp = torch.cuda.current_stream(device)
        for i, d in enumerate(L):
            with torch.cuda.stream(copy_in):
                copy_in.wait_event(ev_done[i])  # the previous step's layer i has consumed qd[i], idd[i]
                qd[i].copy_(qh[i], non_blocking=True)
                idd[i].copy_(ih[i], non_blocking=True)
                ev_in[i].record(copy_in)
            comp.wait_event(ev_in[i])
            comp.wait_event(ev_back[i])  # the previous step's output i is back on the host
            kernels.qsa_sparse_paged_attention_nvfp4(qd[i], d["kd"], d["ks"], d["vd"], d["vs"], 1.0, 1.0, idd[i],
                                                     d["table"], t2r, d["out"])
            ev_done[i].record(comp)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_done[i])
                oh[i].copy_(d["out"], non_blocking=True)
                ev_back[i].record(copy_out)
        comp.wait_event(ev_back[-1])  # the step ends when its last output is on the host

    def e2e_graph_body():
        # The same step as one CUDA graph (what a serving loop replays): copy streams fork from and join
        # the capturing stream; replays of consecutive steps are ordered by the stream.
        comp = torch.cuda.current_stream(device)
        copy_in.wait_stream(comp)
        copy_out.wait_stream(comp)
        for i, d in enumerate(L):
            with torch.cuda.stream(copy_in):
                qd[i].copy_(qh[i], non_blocking=True)
                idd[i].copy_(ih[i], non_blocking=True)
                ev_in[i].record(copy_in)
            comp.wait_event(ev_in[i])
            kernels.qsa_sparse_paged_attention_nvfp4(qd[i], d["kd"], d["ks"], d["vd"], d["vs"], 1.0, 1.0, idd[i],
                                                     d["table"], t2r, d["out"])
            ev_done[i].record(comp)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_done[i])
                oh[i].copy_(d["out"], non_blocking=True)
        comp.wait_stream(copy_in)
        comp.wait_stream(copy_out)

    for _ in range(max(3, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e2e_steps = max(10, args.steps // 4)
    eager_secs = timed(e2e_step, e2e_steps, device)
    e2e_graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        e2e_graph_body()
    torch.cuda.current_stream(device).wait_stream(side)
    with torch.cuda.graph(e2e_graph):
        e2e_graph_body()
    for _ in range(3):
        e2e_graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e2e_secs = timed(e2e_graph.replay, e2e_steps, device)
    del e2e_graph

    # Copy-only leg: the same per-layer host<->device copies on the same streams, without the reader: the
    # ceiling the host copy path alone puts on e2e at this N (all ranks copy at once through host memory).
    def copy_graph_body():
        comp = torch.cuda.current_stream(device)
        copy_in.wait_stream(comp)
        copy_out.wait_stream(comp)
        for i, d in enumerate(L):
            with torch.cuda.stream(copy_in):
                qd[i].copy_(qh[i], non_blocking=True)
                idd[i].copy_(ih[i], non_blocking=True)
            with torch.cuda.stream(copy_out):
                oh[i].copy_(d["out"], non_blocking=True)
        comp.wait_stream(copy_in)
        comp.wait_stream(copy_out)

    copy_graph = torch.cuda.CUDAGraph()
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        copy_graph_body()
    torch.cuda.current_stream(device).wait_stream(side)
    with torch.cuda.graph(copy_graph):
        copy_graph_body()
    for _ in range(3):
        copy_graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    copy_secs = timed(copy_graph.replay, e2e_steps, device)
    del copy_graph
    if world > 1:
        t = torch.tensor([e2e_secs, eager_secs, copy_secs], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_secs, eager_secs, copy_secs = float(t[0].item()), float(t[1].item()), float(t[2].item())
    e2e_value = world * step_bytes * e2e_steps / e2e_secs / 1e9
    e2e_eager_value = world * step_bytes * e2e_steps / eager_secs / 1e9

    split = None if args.skip_split else bench_split_kv(args, device, world, rank, args.steps)
    write = bench_write(device, args.steps) if rank == 0 else None
    fused_write = bench_fused_write(device, args.steps) if rank == 0 else None
    kv_proj = bench_kv_proj_write(device, args.steps) if rank == 0 and not args.skip_proj else None
    # config 4 and the FP8 sibling reader are single-GPU side measurements: one GPU runs only
    mtp = bench_mtp(args, device, args.steps) if world == 1 and not args.skip_mtp else None
    fp8 = bench_fp8(args, device, args.steps) if world == 1 and not args.skip_fp8 else None
    bf16 = bench_bf16(args, device, args.steps) if world == 1 and not args.skip_bf16 else None
    topk = bench_topk(device, args.steps) if world == 1 else None
    del graph
    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 storage, f16 mma, fp32 softmax+acc",
            "data": "synthetic (seeded torch.randn K/V written by our writer; uniform sorted selections)",
            "config": {
                "workload": f"scale-out decode (config 5a per GPU): {args.seqs} sequences x {args.context} tokens x "
                            f"{args.layers} layers per GPU, 2 KV heads x 256, 24 query heads, top-{args.topk} "
                            f"selected, page {args.page}, random block tables",
                "rows_per_layer": args.seqs, "layers": args.layers, "topk": args.topk, "context": args.context,
                "page": args.page, "cache_gb_per_gpu": sum(d["storage"].numel() for d in L) / 1e9,
                "step_bytes_per_gpu": step_bytes, "l2": "inputs larger than L2: 12 layers x 113 MB of records",
                "launch": "one CUDA graph per step (12 layers)", "parallelism": f"dp{world} (sequence-sharded)"},
            "clocks": clocks.summary(),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": kind, "kernel": "sparse_attention_kernel (one layer, split-KV merge fused)",
                         "algorithmic_bytes_per_launch": step_bytes / args.layers,
                         "us_per_launch": per_layer * 1e6,
                         "traffic": NCU_TRAFFIC["read"]},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": qh.numel() * 2 + ih.numel() * 4,
                    "d2h_bytes_per_step": oh.numel() * 2, "ms_per_step": e2e_secs / e2e_steps * 1e3,
                    "api": "nvfp4_qsa.kernels.qsa_sparse_paged_attention_nvfp4 x12 with per-layer pinned copies in "
                           "and out on two copy streams overlapping the other layers' compute, captured from "
                           "those public calls into one CUDA graph replayed per step",
                    "eager_value": e2e_eager_value,
                    "eager_ms_per_step": eager_secs / e2e_steps * 1e3,
                    "copy_only": {
                        "ms_per_step": copy_secs / e2e_steps * 1e3,
                        "h2d_gb_per_s_per_gpu": (qh.numel() * 2 + ih.numel() * 4) * e2e_steps / copy_secs / 1e9,
                        "d2h_gb_per_s_per_gpu": oh.numel() * 2 * e2e_steps / copy_secs / 1e9,
                        "value_ceiling": world * step_bytes * e2e_steps / copy_secs / 1e9,
                        "what": "the same pinned copies on the same streams without the reader, graph-replayed, "
                                "max over ranks: the e2e ceiling of the host copy path at this N"}},
            "gpu_launches": args.steps * args.layers * launches_per_layer,
            "write": write,
            "fused_write": fused_write,
            "kv_proj_write": kv_proj,
        }
        if split is not None:
            result["split_kv"] = split
        if mtp is not None:
            result["mtp"] = mtp
        if fp8 is not None:
            result["fp8"] = fp8
        if bf16 is not None:
            result["bf16"] = bf16
        if topk is not None:
            result["topk"] = topk
        if world == 1 and not args.skip_cpu:
            result["cpu_baseline"] = cpu_baseline_read(args, args.cpu_seconds)
            write["cpu_baseline"] = cpu_baseline_write(False, 3.0)
            fused_write["cpu_baseline"] = cpu_baseline_write(True, 3.0)
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main_reference(args):
    """Reference arm: the reference algorithm's CPU restatement (oracle/) on this host, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import torch
    import oracle

    world = int(os.environ.get("WORLD_SIZE", "1"))
    page, ctx, topk = args.page, args.context, args.topk
    width = (ctx + page - 1) // page
    nseq = 4
    blocks = nseq * width
    gen = torch.Generator().manual_seed(7)
    rng = np.random.default_rng(7)
    storage = np.zeros((blocks, KV_HEADS, page, RECORD), np.uint8)
    total = blocks * page
    for s0 in range(0, total, 1 << 18):
        n = min(1 << 18, total - s0)
        kv = torch.randn(2, n, KV_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16).view(torch.int16).numpy()
        oracle.write_cache(kv[0].view(np.uint16), kv[1].view(np.uint16), storage,
                           np.arange(s0, s0 + n, dtype=np.int64))
    table = rng.permutation(blocks).astype(np.int32).reshape(nseq, width)
    # All of the host's cores, whatever OMP_NUM_THREADS the launcher set (torch.distributed.run sets 1).
    oracle.set_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count())
    threads = oracle.get_threads()

    def sample(rows):
        q = torch.randn(rows, QUERY_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16).view(torch.int16).numpy()
        idx = np.stack([np.sort(rng.choice(ctx, topk, replace=False)) for _ in range(rows)]).astype(np.int32)
        return q.view(np.uint16), idx, (np.arange(rows) % nseq).astype(np.int32)

    # One step = a bounded sample of the workload's rows (one layer), sized from a calibration call so that
    # the --warmup W + --steps K steps together take about two minutes of CPU time.
    cq, cidx, ct2r = sample(threads)
    t0 = time.perf_counter()
    oracle.sparse_attention(cq, storage, cidx, table, ct2r)
    per_row = (time.perf_counter() - t0) / threads
    budget = min(10.0, 120.0 / max(1, args.steps + args.warmup))
    rows = max(1, min(4 * threads, int(budget / per_row)))
    q, idx, t2r = sample(rows)
    steps, warmup = args.steps, args.warmup
    for _ in range(warmup):
        oracle.sparse_attention(q, storage, idx, table, t2r)
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.sparse_attention(q, storage, idx, table, t2r)
    secs = time.perf_counter() - t0
    value = rows * steps * read_bytes(1, topk, 1) / secs / 1e9
    sample = (f"oracle/nvfp4_oracle.c float64 reader: {rows} decode rows of one layer per step (2 KV heads x {topk} "
              f"selected of {ctx} tokens, page {page}), {threads} OpenMP threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": secs / steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"scale-out decode (config 5a), bounded CPU sample: {sample}", "topk": topk,
                   "context": ctx, "page": page},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        main_reference(args)
    else:
        main_ours(args)


if __name__ == "__main__":
    main()
