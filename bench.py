#!/usr/bin/env python3
"""Attention-forward benchmark on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Headline (`value`): prefill, non-causal, H_q=32, H_kv=8 (GQA 4:1), D=128,
S_q=S_kv=4096, fp16 in / fp32 out, one sequence per GPU (global batch = N,
batch-sharded, no communication): whole-job TFLOP/s with
FLOPs = 4*B*H_q*S_q*S_kv*D (the reference benchmark's formula,
tests/bench_flash_attn.cu:125-127).  A step is one attention forward of the
rank's batch; inputs are resident in HBM and rotate over 4 buffer sets
(448 MiB > 2x the 126 MB L2).  `e2e` is the same metric through the public
API (flash_attn_fwd) with the step's Q/K/V copied from pinned host memory and
O copied back inside the timed region.  `extra` holds the decode configs
(HBM GB/s with bytes = 2*B*H_kv*S_kv*D*2 + 2*B*H_q*D + 4*B*H_q*D; device time
from CUDA-graph replay, the host-call time beside it), MQA D=64,
prefill S=512, RMSNorm / RoPE / SwiGLU (HBM GB/s of their algorithmic bytes)
and, for N > 1, the KV-split long decode across the N GPUs.

--impl reference times the reference's CPU path for the same workload: the
NumPy reference_attn of kernel_models/flash_attn.py (restated in oracle/, the
reference tree does not travel), fp32, BLAS threads = host cores, each step a
bounded sample of query heads; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "prefill TFLOP/s & decode HBM GB/s (H_q32/H_kv8/D128) at 1/2/4/8 B200"
H_Q, H_KV, D, S = 32, 8, 128, 4096
ROTATE = 4
MIB = 1 << 20


def prefill_flops(B, H_q, S_q, S_kv, D_):
    return 4.0 * B * H_q * S_q * S_kv * D_


def causal_flops(B, H_q, S_q, S_kv, D_):
    """4*D per visible (query, key) pair under the bottom-right causal mask."""
    off = S_kv - S_q
    pairs = sum(min(S_kv, off + i + 1) for i in range(S_q))
    return 4.0 * B * H_q * pairs * D_


def decode_bytes(B, H_q, H_kv, S_kv, D_):
    return 2.0 * B * H_kv * S_kv * D_ * 2 + 2.0 * B * H_q * D_ + 4.0 * B * H_q * D_


def workload_config(world):
    return {
        "workload": "prefill non-causal H_q=32 H_kv=8 D=128 S_q=S_kv=4096, fp16 in / fp32 out, "
                    "1 sequence per GPU (batch-sharded)",
        "global_batch": world,
        "seq_len": S,
        "heads_q": H_Q,
        "heads_kv": H_KV,
        "head_dim": D,
        "parallelism": f"batch-shard x{world} (no collective)",
        "l2": f"inputs rotate over {ROTATE} HBM-resident sets ({ROTATE * 112} MiB > 2x L2)",
    }


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def profile_traffic(name):
    """dram bytes per launch from a committed ncu summary line 'traffic_bytes_per_launch: N'."""
    path = os.path.join(REPO, "profiles", name)
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- clocks
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}
BAD_REASONS = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


class ClockSampler:
    """Polls this rank's GPU (NVML) every few ms while the timed region runs."""

    def __init__(self, cuda_index, period_s=0.005):
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nv = pynvml
            uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
            try:
                self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        names = sorted(n for bit, n in _REASONS.items() if self.reasons & bit and n != "gpu_idle")
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------- helpers
def rand_f16(shape, gen, device):
    """The next prod(shape) N(0,1) fp16 values of the seeded stream ``gen`` (a
    kernelfoundry_b200.NormalStream), generated on the device by kf_fill_normal_f16.
    oracle/synth_oracle.normal_f16 rebuilds any slice of them on the host."""
    return gen.f16(shape, device)


# Long-context decode: one full-length K then V [1, H_KV, S_kv, D] of this seed; each rank
# generates only its KV range.
LONG_KV_SEED = 6006


def long_kv_offsets(h, lo, s_kv):
    """Stream offsets of row `lo` of KV head `h` in the full-length K and in V."""
    return (h * s_kv + lo) * D, (H_KV * s_kv + h * s_kv + lo) * D


# Seed of the headline's inputs on rank r: Q sets, then K sets, then V sets, drawn in that order.
def headline_seed(rank):
    return 1002 + 7919 * rank


def headline_host_qkv(heads):
    """Rank 0's first headline input set rebuilt on the host (float32 of the fp16 values):
    query heads [0, heads) and the KV head they share (GQA group 0)."""
    import numpy as np

    from oracle.synth_oracle import normal_f16

    nq, nkv, hd = H_Q * S * D, H_KV * S * D, S * D
    seed = headline_seed(0)
    Q = normal_f16(heads * hd, seed, 0).astype(np.float32).reshape(1, heads, S, D)
    K = normal_f16(hd, seed, ROTATE * nq).astype(np.float32).reshape(1, 1, S, D)
    V = normal_f16(hd, seed, ROTATE * nq + ROTATE * nkv).astype(np.float32).reshape(1, 1, S, D)
    return Q, K, V


def time_loop(fn, iters, warmup, stream):
    """Mean ms per call over `iters` back-to-back calls (CUDA events on `stream`)."""
    import torch

    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(iters):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def time_graph(fn, n_calls, reps, stream):
    """Mean ms per call with the n_calls calls captured once in a CUDA graph and
    replayed `reps` times (device time without Python/launch overhead)."""
    import torch

    for i in range(n_calls):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n_calls):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * n_calls)
    del g
    return ms


def max_over_ranks(vals, world, device):
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


# ---------------------------------------------------------------- our arm
def run_prefill_headline(args, rank, world, dev):
    import torch
    import torch.distributed as dist

    from kernelfoundry_b200 import NormalStream, flash_attn_fwd, plan

    stream = torch.cuda.current_stream(dev)
    gen = NormalStream(headline_seed(rank))
    qs = [rand_f16((1, H_Q, S, D), gen, dev) for _ in range(ROTATE)]
    ks = [rand_f16((1, H_KV, S, D), gen, dev) for _ in range(ROTATE)]
    vs = [rand_f16((1, H_KV, S, D), gen, dev) for _ in range(ROTATE)]
    os_ = [torch.empty((1, H_Q, S, D), dtype=torch.float32, device=dev) for _ in range(ROTATE)]
    assert plan(1, H_Q, H_KV, S, S, D)["path"] == "prefill"

    def step(i):
        j = i % ROTATE
        flash_attn_fwd(qs[j], ks[j], vs[j], out=os_[j])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    def timed():
        # Events only around the K steps: an event pair per step costs ~1.7 % here.
        # The per-launch duration for the roofline is total / K, which also counts
        # the gaps between back-to-back launches (an upper bound on the kernel time).
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize()
        with ClockSampler(dev.index) as cs:
            t0.record(stream)
            for i in range(args.steps):
                step(i)
            t1.record(stream)
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        total_ms = t0.elapsed_time(t1)
        return total_ms, total_ms / args.steps, cs.summary()

    total_ms, kern_ms, clocks = timed()
    if set(clocks["reasons"]) & BAD_REASONS:           # rejected clocks: measure once more
        total_ms, kern_ms, clocks = timed()
    total_ms, kern_ms = max_over_ranks([total_ms, kern_ms], world, dev)
    if world > 1:
        all_clocks = [None] * world
        dist.all_gather_object(all_clocks, clocks)
    else:
        all_clocks = [clocks]
    ms_per_step = total_ms / args.steps
    del qs, ks, vs, os_
    torch.cuda.empty_cache()
    return ms_per_step, kern_ms, all_clocks


def run_prefill_e2e(args, rank, world, dev, out_dtype=None):
    """Same workload through the public API with host buffers, pipelined as a serving
    loop runs it: every step copies its Q/K/V from pinned host memory and its O back,
    on their own streams, so step i+1's upload and step i-1's download overlap step i's
    kernel (two device buffer sets).  Time per step = (last download's end - first
    upload's start) / steps; every byte of every step is inside that window."""
    import torch
    import torch.distributed as dist

    from kernelfoundry_b200 import NormalStream, flash_attn_fwd

    out_dtype = out_dtype or torch.float32
    g = NormalStream(2002 + rank)
    hq = [rand_f16((1, H_Q, S, D), g, dev).cpu().pin_memory() for _ in range(2)]
    hk = [rand_f16((1, H_KV, S, D), g, dev).cpu().pin_memory() for _ in range(2)]
    hv = [rand_f16((1, H_KV, S, D), g, dev).cpu().pin_memory() for _ in range(2)]
    ho = [torch.empty((1, H_Q, S, D), dtype=out_dtype).pin_memory() for _ in range(2)]
    dq = [torch.empty_like(x, device=dev) for x in hq]
    dk = [torch.empty_like(x, device=dev) for x in hk]
    dv = [torch.empty_like(x, device=dev) for x in hv]
    do = [torch.empty((1, H_Q, S, D), dtype=out_dtype, device=dev) for _ in range(2)]
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(2)]      # set b uploaded
    ev_cmp = [torch.cuda.Event() for _ in range(2)]     # set b computed (its inputs free)
    ev_out = [torch.cuda.Event() for _ in range(2)]     # set b downloaded (its output free)
    used = [False, False]

    def step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(ev_cmp[b])
            dq[b].copy_(hq[b], non_blocking=True)
            dk[b].copy_(hk[b], non_blocking=True)
            dv[b].copy_(hv[b], non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in[b])
            if used[b]:
                s_cmp.wait_event(ev_out[b])
            flash_attn_fwd(dq[b], dk[b], dv[b], out=do[b])
            ev_cmp[b].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp[b])
            ho[b].copy_(do[b], non_blocking=True)
            ev_out[b].record(s_out)
        used[b] = True

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(args.steps):
        step(args.warmup + i)
    t1.record(s_out)
    t1.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    (ms,) = max_over_ranks([ms], world, dev)
    h2d = sum(x.numel() * x.element_size() for x in (hq[0], hk[0], hv[0]))
    d2h = ho[0].numel() * ho[0].element_size()
    return ms, h2d, d2h


def run_extras(args, rank, world, dev, peaks):
    """Decode (C3), long decode (C5), MQA (C4), short prefill (C1) on this rank's GPU."""
    import torch

    from kernelfoundry_b200 import NormalStream, flash_attn_fwd, plan

    stream = torch.cuda.current_stream(dev)
    gen = NormalStream(4242)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    iters = max(10, min(args.steps, 50))
    out = {}

    def bench_cfg(B, Hq, Hkv, Sq, Skv, Dh, causal=False):
        one = (B * Hq * Sq * Dh * 2 + 2 * B * Hkv * Skv * Dh * 2 + B * Hq * Sq * Dh * 4)
        # Enough input sets that consecutive calls never find their inputs in L2: the
        # sets together exceed 2x L2, and there are always at least two.
        rot = max(2, min(16, -(-2 * l2 // one) + 1))
        qs = [rand_f16((B, Hq, Sq, Dh), gen, dev) for _ in range(rot)]
        ks = [rand_f16((B, Hkv, Skv, Dh), gen, dev) for _ in range(rot)]
        vs = [rand_f16((B, Hkv, Skv, Dh), gen, dev) for _ in range(rot)]
        os_ = [torch.empty((B, Hq, Sq, Dh), dtype=torch.float32, device=dev) for _ in range(rot)]

        def f(i):
            j = i % rot
            flash_attn_fwd(qs[j], ks[j], vs[j], out=os_[j], causal=causal)

        host_ms = time_loop(f, iters, 3, stream)
        n_calls = rot * max(1, 8 // rot)
        ms = time_graph(f, n_calls, max(2, iters // n_calls), stream)
        pl = plan(B, Hq, Hkv, Sq, Skv, Dh)
        pl["host_call_us"] = round(host_ms * 1e3, 2)
        del qs, ks, vs, os_
        return ms, rot, pl

    for B in (1, 16, 64):
        ms, rot, pl = bench_cfg(B, H_Q, H_KV, 1, 4096, D)
        gbs = decode_bytes(B, H_Q, H_KV, 4096, D) / (ms * 1e-3) / 1e9
        out[f"decode_kv4096_B{B}"] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                                      "frac_hbm": round(gbs / peaks["hbm_gbs"], 3), "n_split": pl["n_split"],
                                      "rotated_sets": rot, "host_call_us": pl["host_call_us"]}
    ms, rot, pl = bench_cfg(1, H_Q, H_KV, 1, 131072, D)
    gbs = decode_bytes(1, H_Q, H_KV, 131072, D) / (ms * 1e-3) / 1e9
    out["long_decode_kv131072_1gpu"] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                                        "frac_hbm": round(gbs / peaks["hbm_gbs"], 3), "n_split": pl["n_split"],
                                        "host_call_us": pl["host_call_us"]}
    ms, rot, pl = bench_cfg(4, 32, 1, 2048, 2048, 64)
    tf = prefill_flops(4, 32, 2048, 2048, 64) / (ms * 1e-3) / 1e12
    out["mqa_d64_B4_S2048"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1),
                               "frac_tensor": round(tf / peaks["bf16_tflops"], 3)}
    ms, rot, pl = bench_cfg(1, H_Q, H_KV, 512, 512, D)
    tf = prefill_flops(1, H_Q, 512, 512, D) / (ms * 1e-3) / 1e12
    out["prefill_S512_B1"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1)}
    out.update(bench_paged(stream, gen, dev, peaks, l2, iters))
    ms, rot, pl = bench_cfg(1, H_Q, H_KV, S, S, D, causal=True)
    tf = causal_flops(1, H_Q, S, S, D) / (ms * 1e-3) / 1e12
    out["prefill_causal_S4096_B1"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1),
                                      "frac_tensor": round(tf / peaks["bf16_tflops"], 3),
                                      "flops": "4*D per visible (query, key) pair"}
    # Chunked prefill: a 512-token chunk over a 4096-key cache, causal (bottom-right mask).
    ms, rot, pl = bench_cfg(1, H_Q, H_KV, 512, S, D, causal=True)
    tf = causal_flops(1, H_Q, 512, S, D) / (ms * 1e-3) / 1e12
    out["prefill_causal_chunk_Sq512_Skv4096_B1"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1),
                                                    "frac_tensor": round(tf / peaks["bf16_tflops"], 3),
                                                    "flops": "4*D per visible (query, key) pair"}
    torch.cuda.empty_cache()
    out.update(bench_pointwise(stream, gen, dev, peaks, iters))
    out["reference_bench_sweep"] = run_ref_sweep(stream, gen, dev, peaks, l2)
    return out


def bench_paged(stream, gen, dev, peaks, l2, iters):
    """Decode B=16 KV=4096 over a paged cache (block 16, randomly permuted pages), as
    the reference's paged benchmark lays it out; same bytes formula as contiguous decode."""
    import torch

    from kernelfoundry_b200 import flash_attn_paged

    B, bs = 16, 16
    nb = S // bs
    one = 2 * B * nb * H_KV * bs * D * 2
    rot = max(1, min(8, -(-2 * l2 // one) + 1))
    sets = []
    for r in range(rot):
        pk = rand_f16((B * nb + 7, H_KV, bs, D), gen, dev)
        pv = rand_f16((B * nb + 7, H_KV, bs, D), gen, dev)
        perm = torch.randperm(B * nb + 7, generator=torch.Generator().manual_seed(r))[:B * nb]
        table = perm.to(torch.int32).reshape(B, nb).to(dev)
        seq = torch.full((B,), S, dtype=torch.int32, device=dev)
        q = rand_f16((B, H_Q, 1, D), gen, dev)
        o = torch.empty((B, H_Q, 1, D), dtype=torch.float32, device=dev)
        sets.append((q, pk, pv, table, seq, o))

    def f(i):
        q, pk, pv, table, seq, o = sets[i % rot]
        flash_attn_paged(q, pk, pv, table, seq, out=o)

    host_ms = time_loop(f, iters, 3, stream)
    n_calls = rot * max(1, 8 // rot)
    ms = time_graph(f, n_calls, max(2, iters // n_calls), stream)
    gbs = decode_bytes(B, H_Q, H_KV, S, D) / (ms * 1e-3) / 1e9
    del sets
    return {"paged_decode_kv4096_B16_bs16": {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                                             "frac_hbm": round(gbs / peaks["hbm_gbs"], 3),
                                             "host_call_us": round(host_ms * 1e3, 2), "rotated_sets": rot}}


# RMSNorm / RoPE / SwiGLU on decoder-layer shapes of the same model family
# (hidden = H_q * D = 4096; MLP width 14336; RoPE on the C2 batch-8 Q/K).
# Every working set is above 2x L2, so each call streams from HBM.
POINTWISE = {
    # name: (description, algorithmic bytes per call)
    "rmsnorm_add_T16384_H4096": ("fused residual add + RMSNorm, fp16 [16384, 4096]: read x and residual, "
                                 "write residual and out", 4 * 16384 * 4096 * 2),
    "rmsnorm_T16384_H4096": ("RMSNorm, fp16 [16384, 4096]: read x, write out", 2 * 16384 * 4096 * 2),
    "rope_B8_S4096": ("NeoX RoPE in place on Q [8, 32, 4096, 128] and K [8, 8, 4096, 128] fp16, theta 5e5: "
                      "read + write both", 2 * 8 * (H_Q + H_KV) * S * D * 2),
    "swiglu_T8192_I14336": ("SwiGLU, fp16 gate_up [8192, 28672] -> out [8192, 14336]",
                            8192 * 14336 * 3 * 2),
}


def pointwise_setup(name, gen, dev):
    """Inputs for one POINTWISE entry; returns the call f(i)."""
    import torch

    from kernelfoundry_b200 import fused_add_rms_norm, rms_norm, rope_, swiglu

    if name.startswith("rmsnorm"):
        x = rand_f16((16384, 4096), gen, dev)
        w = rand_f16((4096,), gen, dev)
        o = torch.empty_like(x)
        if name.startswith("rmsnorm_add"):
            res = rand_f16((16384, 4096), gen, dev)
            return lambda i: fused_add_rms_norm(x, res, w, 1e-5, out=o)
        return lambda i: rms_norm(x, w, 1e-5, out=o)
    if name.startswith("rope"):
        q = rand_f16((8, H_Q, S, D), gen, dev)
        k = rand_f16((8, H_KV, S, D), gen, dev)
        return lambda i: rope_(q, k, theta=500000.0)
    gu = rand_f16((8192, 2 * 14336), gen, dev)
    o = torch.empty((8192, 14336), dtype=torch.float16, device=dev)
    return lambda i: swiglu(gu, out=o)


def bench_pointwise(stream, gen, dev, peaks, iters):
    import torch

    out = {}
    for name, (desc, nbytes) in POINTWISE.items():
        f = pointwise_setup(name, gen, dev)
        ms = time_loop(f, iters, 3, stream)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 3),
                     "bytes": nbytes, "what": desc}
        del f
        torch.cuda.empty_cache()
    return out


def run_prefill_b8_strong(args, rank, world, dev, peaks):
    """BASELINE configs[1] at its own shape: one global batch of 8 sequences (S=4096,
    H_q=32, H_kv=8, D=128) split over the N GPUs, 8/N sequences per rank, no
    communication.  Whole-job time = max over ranks of the K timed calls (barrier and
    synchronize on both sides); one input set per rank already exceeds 2x L2."""
    import torch
    import torch.distributed as dist

    from kernelfoundry_b200 import NormalStream, flash_attn_fwd

    if 8 % world:
        return {"unavailable": f"8 sequences do not divide over {world} GPUs"}
    b = 8 // world
    gen = NormalStream(3003 + 7919 * rank)
    q = rand_f16((b, H_Q, S, D), gen, dev)
    k = rand_f16((b, H_KV, S, D), gen, dev)
    v = rand_f16((b, H_KV, S, D), gen, dev)
    o = torch.empty((b, H_Q, S, D), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        flash_attn_fwd(q, k, v, out=o)
    steps = max(5, min(args.steps, 20))
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        flash_attn_fwd(q, k, v, out=o)
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    (ms,) = max_over_ranks([t0.elapsed_time(t1) / steps], world, dev)
    del q, k, v, o
    torch.cuda.empty_cache()
    tf = prefill_flops(8, H_Q, S, S, D) / (ms * 1e-3) / 1e12
    return {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "TFLOP/s_per_gpu": round(tf / world, 1),
            "frac_tensor_per_gpu": round(tf / world / peaks["bf16_tflops"], 3), "n_gpus": world,
            "seqs_per_gpu": b, "scaling": "strong (global batch 8 fixed)", "steps": steps}


# The reference benchmark's sweep (tests/bench_flash_attn.cu:148-185), as
# (B, S_kv, H_q, H_kv, D, q_len); q_len None = prefill with S_q = S_kv.
REF_SWEEP = [
    (1, 512, 32, 8, 128, 1), (1, 1024, 32, 8, 128, 1), (1, 2048, 32, 8, 128, 1), (1, 4096, 32, 8, 128, 1),
    (8, 512, 32, 8, 128, 1), (8, 1024, 32, 8, 128, 1),
    (1, 64, 32, 8, 128, None), (1, 128, 32, 8, 128, None), (1, 256, 32, 8, 128, None), (8, 64, 32, 8, 128, None),
    (1, 512, 32, 8, 128, None), (1, 1024, 32, 8, 128, None), (1, 2048, 32, 8, 128, None),
    (1, 4096, 32, 8, 128, None),
    (1, 1024, 32, 8, 64, None), (1, 1024, 32, 8, 128, None), (1, 1024, 32, 8, 256, None),
    (1, 512, 32, 1, 128, None), (1, 1024, 32, 1, 128, None), (1, 512, 32, 1, 128, 1), (1, 1024, 32, 1, 128, 1),
]


def ref_sweep_bytes(B, H_q, H_kv, S_q, S_kv, D_):
    """The reference benchmark's byte count: fp16 Q, K, V read, fp32 O written
    (tests/bench_flash_attn.cu:129-131)."""
    q_n, kv_n = B * H_q * S_q * D_, B * H_kv * S_kv * D_
    return 2.0 * q_n + 2.0 * kv_n + 2.0 * kv_n + 4.0 * q_n


def run_ref_sweep(stream, gen, dev, peaks, l2):
    """Our kernels on every row of the reference benchmark's sweep: device time per call
    from CUDA-graph replay over enough input sets that they exceed 2x L2."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd

    rows = []
    for (B, S_kv, Hq, Hkv, Dh, ql) in REF_SWEEP:
        S_q = ql or S_kv
        one = B * Hq * S_q * Dh * 2 + 2 * B * Hkv * S_kv * Dh * 2 + B * Hq * S_q * Dh * 4
        rot = max(2, min(64, -(-2 * l2 // one) + 1))
        sets = [(rand_f16((B, Hq, S_q, Dh), gen, dev), rand_f16((B, Hkv, S_kv, Dh), gen, dev),
                 rand_f16((B, Hkv, S_kv, Dh), gen, dev),
                 torch.empty((B, Hq, S_q, Dh), dtype=torch.float32, device=dev)) for _ in range(rot)]

        def f(i):
            q, k, v, o = sets[i % rot]
            flash_attn_fwd(q, k, v, out=o)

        n_calls = rot * max(1, 16 // rot)
        ms = time_graph(f, n_calls, 4, stream)
        fl = prefill_flops(B, Hq, S_q, S_kv, Dh)
        by = ref_sweep_bytes(B, Hq, Hkv, S_q, S_kv, Dh)
        row = {"shape": {"B": B, "S_q": S_q, "S_kv": S_kv, "H_q": Hq, "H_kv": Hkv, "D": Dh},
               "us": round(ms * 1e3, 2), "TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 2),
               "GB/s": round(by / (ms * 1e-3) / 1e9, 1)}
        if ql == 1:
            row["frac_hbm"] = round(row["GB/s"] / peaks["hbm_gbs"], 3)
        else:
            row["frac_tensor"] = round(row["TFLOP/s"] / peaks["bf16_tflops"], 3)
        rows.append(row)
        del sets
    torch.cuda.empty_cache()
    return rows


def run_long_decode_split(args, rank, world, dev, peaks):
    """C5 across the N GPUs: KV split by ranges, partials + one all-gather + LSE merge.

    Timed two ways, max over ranks: host-driven calls, and the same step (partial
    kernel, NCCL all-gather, combine kernel) captured once in a CUDA graph and
    replayed (device time, the number a decode loop that replays graphs sees)."""
    import torch
    import torch.distributed as dist

    from kernelfoundry_b200 import NormalStream, fill_normal_f16
    from kernelfoundry_b200.multi_gpu import kv_shard, long_decode_forward

    S_kv = 131072
    lo, hi = kv_shard(S_kv, world, rank)
    q = rand_f16((1, H_Q, 1, D), NormalStream(5005), dev)
    # This rank's KV range [lo, hi) of the one full-length K and V of LONG_KV_SEED (K first,
    # then V), so every world size sees the same cache as one GPU does.
    k = torch.empty((1, H_KV, hi - lo, D), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    for h in range(H_KV):
        k_off, v_off = long_kv_offsets(h, lo, S_kv)
        fill_normal_f16(k[0, h], LONG_KV_SEED, k_off)
        fill_normal_f16(v[0, h], LONG_KV_SEED, v_off)
    n = (H_Q * (D + 2) + 3) // 4 * 4
    buf = torch.empty(world * n, dtype=torch.float32, device=dev)
    out = torch.empty((1, H_Q, 1, D), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    iters = max(10, min(args.steps, 50))

    def step(_):
        long_decode_forward(q, k, v, gather_buf=buf, out=out)

    dist.barrier(device_ids=[dev.index])
    host_ms = time_loop(step, iters, 3, stream)
    # CUDA graph: warm-up outside capture (NCCL communicator, workspace), then capture.
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for i in range(3):
            step(i)
    stream.wait_stream(side)
    torch.cuda.synchronize()
    dist.barrier(device_ids=[dev.index])
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(0)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[dev.index])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        g.replay()
    e1.record(stream)
    e1.synchronize()
    graph_ms = e0.elapsed_time(e1) / iters
    del g                                   # graphs holding NCCL work go before the process group
    torch.cuda.synchronize()
    # The same step with the NVLink peer exchange (no NCCL): partial kernel + one
    # exchange-and-merge kernel, host-driven and as a CUDA graph.
    from kernelfoundry_b200 import device_error
    from kernelfoundry_b200.multi_gpu import PeerExchange

    # Every rank agrees that the windows were set up before any rank times them.
    ex, why = None, ""
    try:
        ex = PeerExchange(tuple(q.shape), device=dev)
    except Exception as e:  # noqa: BLE001 -- reported in the JSON line, the NCCL numbers stand
        why = f"{type(e).__name__}: {e}"[:200]
    agree = torch.tensor([1 if ex is not None else 0], device=dev)
    dist.all_reduce(agree, op=dist.ReduceOp.MIN)
    host_ms, graph_ms = max_over_ranks([host_ms, graph_ms], world, dev)
    gbs = decode_bytes(1, H_Q, H_KV, S_kv, D) / (graph_ms * 1e-3) / 1e9
    res = {"us": round(graph_ms * 1e3, 2), "host_call_us": round(host_ms * 1e3, 2), "GB/s_total": round(gbs, 1),
           "GB/s_per_gpu": round(gbs / world, 1), "frac_hbm_per_gpu": round(gbs / world / peaks["hbm_gbs"], 3),
           "collective": "1x all_gather (NCCL), in place; us = CUDA-graph replay"}
    if int(agree.item()) == 0:
        if ex is not None:
            ex.close()
        res["p2p"] = {"unavailable": why or "peer window setup failed on another rank"}
        return res

    fused_ok = torch.tensor([1 if ex.attend(q, k, v, out=out) is not None else 0], device=dev)
    dist.all_reduce(fused_ok, op=dist.ReduceOp.MIN)

    def time_p2p(fused):
        def step_p2p(_):
            long_decode_forward(q, k, v, exchange=ex, out=out, fused=fused)

        dist.barrier(device_ids=[dev.index])
        host = time_loop(step_p2p, iters, 3, stream)
        with torch.cuda.stream(side):
            for i in range(3):
                step_p2p(i)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        dist.barrier(device_ids=[dev.index])
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step_p2p(0)
        g.replay()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[dev.index])
        e0.record(stream)
        for _ in range(iters):
            g.replay()
        e1.record(stream)
        e1.synchronize()
        graph = e0.elapsed_time(e1) / iters
        del g
        torch.cuda.synchronize()
        return host, graph

    timings = {"two_launch": time_p2p(False)}
    if int(fused_ok.item()):
        timings["fused"] = time_p2p(True)
    rc, raw = device_error()                # an expired peer wait would void the timing
    ex.close()
    flat = [x for k in ("two_launch", "fused") if k in timings for x in timings[k]]
    vals = max_over_ranks(flat + [float(rc != 0)], world, dev)
    if vals[-1]:
        res["p2p"] = {"unavailable": f"a peer wait expired during timing (device error word {raw:#x})"}
        return res
    what = {"two_launch": "kf_attn_fwd_partial, then kf_attn_exchange_combine: {value, sequence} words written into "
                          "the peers' windows over NVLink (CUDA IPC), polled and merged in a second kernel",
            "fused": "kf_attn_fwd_exchange: the decode kernel's merging CTA of each (b, h_kv) writes its partial into "
                     "the peers' windows and merges theirs; one launch"}
    i = 0
    for key in ("two_launch", "fused"):
        if key not in timings:
            continue
        host_ms, graph_ms = vals[i], vals[i + 1]
        i += 2
        gbs_p = decode_bytes(1, H_Q, H_KV, S_kv, D) / (graph_ms * 1e-3) / 1e9
        res["p2p_fused" if key == "fused" else "p2p_two_launch"] = {
            "us": round(graph_ms * 1e3, 2), "host_call_us": round(host_ms * 1e3, 2), "GB/s_total": round(gbs_p, 1),
            "frac_hbm_per_gpu": round(gbs_p / world / peaks["hbm_gbs"], 3),
            "exchange": what[key] + "; no NCCL; us = CUDA-graph replay, max over ranks"}
    # The path long_decode_forward takes by default (fused for two ranks, else two launches).
    default = "p2p_fused" if (world <= 2 and "p2p_fused" in res) else "p2p_two_launch"
    res["p2p"] = dict(res[default], path=default)
    return res


def cpu_baseline_sample(budget_s=12.0):
    """The reference's NumPy path (reference_attn restated), fp32, on a bounded sample of the
    query heads of rank 0's first headline input set (rebuilt on the host from its seed: the
    same fp16 values the GPU arm reads).  Only the attention calls are timed."""
    import numpy as np

    from oracle.attn_oracle import reference_attn
    from oracle.synth_oracle import normal_f16

    try:
        from threadpoolctl import threadpool_info

        threads = max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"), default=1)
    except Exception:
        threads = os.cpu_count() or 1
    seed, nq, nkv, hd = headline_seed(0), H_Q * S * D, H_KV * S * D, S * D

    def head(off):
        return normal_f16(hd, seed, off).astype(np.float32).reshape(1, 1, S, D)

    kv = {}
    done, dt = 0, 0.0
    while done < H_Q and dt < budget_s:
        g = done // (H_Q // H_KV)                     # GQA: query head -> its KV head
        if g not in kv:
            kv = {g: (head(ROTATE * nq + g * hd), head(ROTATE * nq + ROTATE * nkv + g * hd))}
        Qh = head(done * hd)
        t0 = time.perf_counter()
        reference_attn(Qh, *kv[g])
        dt += time.perf_counter() - t0
        done += 1
    tf = prefill_flops(1, done, S, S, D) / dt / 1e12
    return {"value": round(tf, 5), "unit": "TFLOP/s", "cores": int(threads), "kind": "port",
            "sample": f"{done} of {H_Q} query heads of the first headline input set (S=4096, D=128, the GPU "
                      f"arm's own fp16 values rebuilt from its seed), fp32 NumPy reference_attn (oracle "
                      f"restatement), {dt:.1f} s of attention"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and "RANK" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks = load_peaks()

    ms_step, kern_ms, clocks = run_prefill_headline(args, rank, world, dev)
    flops_rank = prefill_flops(1, H_Q, S, S, D)
    value = world * flops_rank / (ms_step * 1e-3) / 1e12
    e2e_ms, h2d, d2h = run_prefill_e2e(args, rank, world, dev)
    e2e_value = world * flops_rank / (e2e_ms * 1e-3) / 1e12
    # The same serving loop with fp16 O (KF_FLAG_OUT_F16): the fp32 O download of the
    # reference's contract is what bounds e2e; this shows the loop with half of it.
    e2e16_ms, h2d16, d2h16 = run_prefill_e2e(args, rank, world, dev, out_dtype=torch.float16)

    achieved = flops_rank / (kern_ms * 1e-3) / 1e12
    traffic = profile_traffic("prefill_sm100_C2.md")
    from kernelfoundry_b200 import plan
    unsplit_ctas = plan(1, H_Q, H_KV, S, S, D, workspace_bytes=0)["ctas"]
    split = plan(1, H_Q, H_KV, S, S, D)["ctas"] > unsplit_ctas
    # One-tile units with an even count of 128-key tiles run as key-half units (KVH).
    kvh = unsplit_ctas == H_Q * ((S + 127) // 128) and ((S + 127) // 128) % 2 == 0
    tf = lambda x: "true" if x else "false"  # noqa: E731
    kernel_name = f"kf::prefill_fwd_kernel<128, false, {tf(split)}, {tf(kvh)}>"

    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": traffic,
                "kernel": kernel_name, "kernel_ms": round(kern_ms, 5),
                "kernel_ms_src": "CUDA events around the K timed launches / K (launch gaps included)",
                "flops_per_launch": flops_rank, "peak_src": f"{peaks['src']} bf16 dense (burst)"}

    extra = {}
    if not args.no_extras:
        if rank == 0:
            extra = run_extras(args, rank, world, dev, peaks)
        b8 = run_prefill_b8_strong(args, rank, world, dev, peaks)
        if rank == 0:
            extra["prefill_B8_S4096_strong"] = b8
            extra["e2e_out_f16"] = {"value": round(world * flops_rank / (e2e16_ms * 1e-3) / 1e12, 2),
                                    "unit": "TFLOP/s", "ms_per_step": round(e2e16_ms, 4),
                                    "h2d_bytes_per_step": h2d16, "d2h_bytes_per_step": d2h16,
                                    "what": "e2e pipeline with fp16 O (KF_FLAG_OUT_F16) instead of fp32"}
        if world > 1:
            ld = run_long_decode_split(args, rank, world, dev, peaks)
            if rank == 0:
                extra[f"long_decode_kv131072_split_{world}gpu"] = ld

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded N(0,1) fp16 from the counter-based generator of include/kf_synth.h, made on the device)",
        "config": workload_config(world),
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "pipeline": "pinned host buffers; per step H2D of Q/K/V, flash_attn_fwd, D2H of O on 3 streams "
                            "with 2 device buffer sets (step i+1 upload and i-1 download overlap step i)"},
        "gpu_launches": args.steps,
        "roofline": roofline,
        "clocks": {"sm_mhz": clocks[0]["sm_mhz"], "sm_max_mhz": clocks[0]["sm_max_mhz"],
                   "reasons": sorted({r for c in clocks for r in c["reasons"]}),
                   "per_gpu_median_mhz": [c["sm_mhz"] for c in clocks]},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample()
    if extra:
        line["extra"] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
        dist.destroy_process_group()


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import numpy as np

    from oracle.attn_oracle import reference_attn

    try:
        from threadpoolctl import threadpool_info

        threads = max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"), default=1)
    except Exception:
        threads = os.cpu_count() or 1
    heads = 2     # bounded sample per step: 2 of the 32 query heads (1/16 of the per-GPU work)
    Q, K, V = headline_host_qkv(heads)     # the GPU arm's first input set, rebuilt from its seed
    for _ in range(args.warmup):
        reference_attn(Q, K, V)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reference_attn(Q, K, V)
    dt = (time.perf_counter() - t0) / args.steps
    value = prefill_flops(1, heads, S, S, D) / dt / 1e12
    sample = (f"{heads} of {H_Q} query heads (GQA group of one KV head) of the first headline input set "
              f"(S=4096, D=128, the GPU arm's own fp16 values rebuilt from its seed) per step, "
              f"fp32 NumPy reference_attn (restated from kernel_models/flash_attn.py:250-265)")
    line = {
        "metric": METRIC, "value": round(value, 5), "unit": "TFLOP/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (the GPU arm's seeded N(0,1) fp16 inputs, rebuilt on the host by oracle/synth_oracle.py)",
        "config": workload_config(world),
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": int(threads), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- single-case mode (profiling)
CASES = {
    # name: (B, H_q, H_kv, S_q, S_kv, D)
    "prefill_C2": (1, H_Q, H_KV, S, S, D),
    "prefill_C2_B8": (8, H_Q, H_KV, S, S, D),
    "prefill_C1": (1, H_Q, H_KV, 512, 512, D),
    "prefill_chunk_q128": (1, H_Q, H_KV, 128, S, D),
    "mqa_C4": (4, 32, 1, 2048, 2048, 64),
    "decode_B1": (1, H_Q, H_KV, 1, 4096, D),
    "decode_B16": (16, H_Q, H_KV, 1, 4096, D),
    "decode_B64": (64, H_Q, H_KV, 1, 4096, D),
    "long_decode_C5": (1, H_Q, H_KV, 1, 131072, D),
    "prefill_C2_causal": (1, H_Q, H_KV, S, S, D),
    "prefill_C2_B8_causal": (8, H_Q, H_KV, S, S, D),
}


def run_case(args):
    """One configuration, `--warmup` then `--steps` back-to-back launches on one input set.

    Small and deterministic so that a profiler can capture one launch (-s warmup -c 1);
    prints one JSON line with the mean device time of the timed launches."""
    import torch

    from kernelfoundry_b200 import NormalStream, flash_attn_fwd, plan

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = NormalStream(77)
    if args.case in POINTWISE:
        desc, nbytes = POINTWISE[args.case]
        ms = time_loop(pointwise_setup(args.case, gen, dev), args.steps, args.warmup, torch.cuda.current_stream(dev))
        print(json.dumps({"case": args.case, "ms": round(ms, 5), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                          "bytes": nbytes, "what": desc}), flush=True)
        return
    B, Hq, Hkv, Sq, Skv, Dh = CASES[args.case]
    q = rand_f16((B, Hq, Sq, Dh), gen, dev)
    k = rand_f16((B, Hkv, Skv, Dh), gen, dev)
    v = rand_f16((B, Hkv, Skv, Dh), gen, dev)
    o = torch.empty((B, Hq, Sq, Dh), dtype=torch.float32, device=dev)
    causal = args.case.endswith("_causal")
    ms = time_loop(lambda i: flash_attn_fwd(q, k, v, out=o, causal=causal), args.steps, args.warmup,
                   torch.cuda.current_stream(dev))
    line = {"case": args.case, "shape": [B, Hq, Hkv, Sq, Skv, Dh], "ms": round(ms, 5), "plan": plan(B, Hq, Hkv, Sq, Skv, Dh)}
    if Sq > 1:
        fl = (causal_flops if causal else prefill_flops)(B, Hq, Sq, Skv, Dh)
        line["TFLOP/s"] = round(fl / (ms * 1e-3) / 1e12, 1)
    else:
        line["GB/s"] = round(decode_bytes(B, Hq, Hkv, Skv, Dh) / (ms * 1e-3) / 1e9, 1)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="headline only (skip decode/MQA/long-decode lines)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", choices=sorted(CASES) + sorted(POINTWISE),
                    help="time one configuration only (for profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
