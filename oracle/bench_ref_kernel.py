#!/usr/bin/env python3
"""Times the reference's own CUDA kernel on a B200 -- TEST INFRASTRUCTURE ONLY.

    python oracle/bench_ref_kernel.py [--iters 50] [--warmup 5] [--only NAME]

The kernel is flash_attn_kernel<D> (kernels/flash_attn.cu:384-585) compiled
unmodified from the reference sources into oracle/_ref/libkfref.so
(oracle/Makefile), launched as the reference benchmark launches it
(launch_once, tests/bench_flash_attn.cu:39-54, through kfref_launch_general).
Method as the reference benchmark (tests/bench_flash_attn.cu:57-146): warm-up
launches, then back-to-back launches between two CUDA events on one stream,
FLOPs 4*B*H_q*S_q*S_kv*D and bytes 2Q + 2K + 2V + 4O.  Unlike the reference,
inputs rotate over enough sets to exceed 2x L2, as bench.py does for our
kernels, so both are timed from HBM.

Rows: the BASELINE configurations (C1-C5) and every row of the reference
benchmark's sweep (tests/bench_flash_attn.cu:148-185).  One JSON line per row.
This measures the reference, it is never the product: nothing under
kernelfoundry_b200/ loads this library.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)

from bench import REF_SWEEP, decode_bytes, prefill_flops, ref_sweep_bytes  # noqa: E402

CONFIGS = {
    # name: (B, H_q, H_kv, S_q, S_kv, D)
    "C1_prefill_S512": (1, 32, 8, 512, 512, 128),
    "C2_prefill_S4096_B1": (1, 32, 8, 4096, 4096, 128),
    "C2_prefill_S4096_B8": (8, 32, 8, 4096, 4096, 128),
    "C3_decode_kv4096_B1": (1, 32, 8, 1, 4096, 128),
    "C3_decode_kv4096_B16": (16, 32, 8, 1, 4096, 128),
    "C3_decode_kv4096_B64": (64, 32, 8, 1, 4096, 128),
    "C4_mqa_D64_B4_S2048": (4, 32, 1, 2048, 2048, 64),
    "C5_long_decode_kv131072": (1, 32, 8, 1, 131072, 128),
}


def rows():
    out = list(CONFIGS.items())
    for (B, S_kv, Hq, Hkv, Dh, ql) in REF_SWEEP:
        S_q = ql or S_kv
        out.append((f"sweep_B{B}_Sq{S_q}_Skv{S_kv}_Hq{Hq}_Hkv{Hkv}_D{Dh}", (B, Hq, Hkv, S_q, S_kv, Dh)))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--only", default=None, help="run the rows whose name contains this text")
    args = ap.parse_args()

    import torch

    lib_path = os.path.join(HERE, "_ref", "libkfref.so")
    if not os.path.exists(lib_path):
        print(json.dumps({"unavailable": "oracle/_ref/libkfref.so not built (make -C oracle ref)"}))
        return
    lib = ctypes.CDLL(lib_path)
    P = ctypes.c_void_p
    lib.kfref_launch_general.argtypes = [P] * 6 + [ctypes.c_int] * 6 + [P]
    lib.kfref_launch_general.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    stream = torch.cuda.current_stream(dev)
    gen = torch.Generator(device=dev).manual_seed(1234)
    for name, (B, Hq, Hkv, Sq, Skv, Dh) in rows():
        if args.only and args.only not in name:
            continue
        one = B * Hq * Sq * Dh * 2 + 2 * B * Hkv * Skv * Dh * 2 + B * Hq * Sq * Dh * 4
        rot = max(2, min(64, -(-2 * l2 // one) + 1))

        def randn(shape):
            return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).to(torch.float16)

        sets = [(randn((B, Hq, Sq, Dh)), randn((B, Hkv, Skv, Dh)), randn((B, Hkv, Skv, Dh)),
                 torch.empty((B, Hq, Sq, Dh), dtype=torch.float32, device=dev),
                 torch.empty((B, Hq, Sq), dtype=torch.float32, device=dev),
                 torch.empty((B, Hq, Sq), dtype=torch.float32, device=dev)) for _ in range(rot)]

        def launch(i):
            q, k, v, o, mi, li = sets[i % rot]
            rc = lib.kfref_launch_general(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(o.data_ptr()),
                                          P(mi.data_ptr()), P(li.data_ptr()), B, Sq, Skv, Hq, Hkv, Dh,
                                          P(stream.cuda_stream))
            if rc != 0:
                raise RuntimeError(f"reference launch failed: cudaError {rc}")

        for i in range(args.warmup):
            launch(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.iters):
            launch(i)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        line = {"row": name, "impl": "reference CUDA kernel (oracle/_ref/libkfref.so)",
                "shape": {"B": B, "H_q": Hq, "H_kv": Hkv, "S_q": Sq, "S_kv": Skv, "D": Dh},
                "ms": round(ms, 5), "TFLOP/s": round(prefill_flops(B, Hq, Sq, Skv, Dh) / (ms * 1e-3) / 1e12, 3),
                "GB/s_ref_formula": round(ref_sweep_bytes(B, Hq, Hkv, Sq, Skv, Dh) / (ms * 1e-3) / 1e9, 1),
                "rotated_sets": rot, "iters": args.iters}
        if Sq == 1:
            line["GB/s_decode_formula"] = round(decode_bytes(B, Hq, Hkv, Skv, Dh) / (ms * 1e-3) / 1e9, 1)
        print(json.dumps(line), flush=True)
        del sets
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
