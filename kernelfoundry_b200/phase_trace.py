"""Where a prefill launch's time goes, per phase and CTA (developer tool).

    python -m kernelfoundry_b200.phase_trace [CASE ...]      # on a B200; CASE as in CASES

Builds a separate library with ``-DKF_PREFILL_TRACE`` (``lib/libkf_attn_trace.so``; the
shipped ``libkf_attn.so`` has no trace code) in which every prefill CTA writes one
global-timer stamp per phase of its last work item: set-up, the producer's first Q load, Q and
the first K landing at the MMA warp, each softmax tile's first S and last O, the key-half
merge, the split owner's wait, a donor's partial and ticket, the staged store's passes, exit.
Each case runs its call through the C ABI (``kf_attn_fwd_ex``) after warm-up calls on other
inputs, seven times, and prints per phase the number of CTAs that reached it and the min /
median / max over CTAs of the time since the first CTA started (median over the seven launches).
The stamps themselves cost a few tens of ns per phase.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np

from . import build as _build

CASES = {  # B, H_q, H_kv, S_q, S_kv, D, causal
    "C1": (1, 32, 8, 512, 512, 128, 0),
    "C2": (1, 32, 8, 4096, 4096, 128, 0),
    "chunk_q128": (1, 32, 8, 128, 4096, 128, 0),
    "chunk_q256": (1, 32, 8, 256, 4096, 128, 0),
    "causal_chunk512": (1, 32, 8, 512, 4096, 128, 1),
}

# Slot order of kf::PrefillTracePoint (prefill_sm100.cuh).
PHASES = ["entry", "setup (MMA warp past the set-up barrier)", "producer: first Q load issued",
          "MMA: Q landed", "MMA: first K landed", "tile 0: first S", "tile 1: first S", "tile 0: last O",
          "tile 1: last O", "key halves met", "key halves merged in TMEM", "split owner: partials ready",
          "split donor: partial written", "split donor: ticket taken", "tile 0: item done", "tile 1: item done",
          "exit", "producer: registers set", "producer: item decoded", "staged store: pass 0 built",
          "staged store: pass 0 stored", "staged store: pass 1 built", "staged store: pass 1 stored"]
SLOTS, MAX_CTAS, SMID = 32, 1024, 23
TRACE_LIB = os.path.join(_build.LIB_DIR, "libkf_attn_trace.so")


def build_traced() -> str:
    deps = [os.path.join(_build.CSRC, f) for f in _build.SOURCES + _build.HEADERS]
    if os.path.exists(TRACE_LIB) and all(os.path.getmtime(d) <= os.path.getmtime(TRACE_LIB) for d in deps):
        return TRACE_LIB
    os.makedirs(_build.LIB_DIR, exist_ok=True)
    cmd = [_build._nvcc(), *_build.NVCC_FLAGS, "-DKF_PREFILL_TRACE", "-o", TRACE_LIB + ".tmp",
           os.path.join(_build.CSRC, "kf_api.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(res.stdout + res.stderr)
    os.replace(TRACE_LIB + ".tmp", TRACE_LIB)
    return TRACE_LIB


def trace_case(L, name: str, reps: int = 7) -> None:
    import torch

    B, H_q, H_kv, S_q, S_kv, D, causal = CASES[name]
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(1234)
    set_bytes = 2 * B * (H_q * S_q + 2 * H_kv * S_kv) * D
    n_sets = max(3, int(3 * 126e6 // set_bytes) + 1)          # warm-up sets evict the traced one from L2
    sets = [[torch.randn(s, device=dev, generator=g).half() for s in
             ((B, H_q, S_q, D), (B, H_kv, S_kv, D), (B, H_kv, S_kv, D))] for _ in range(n_sets)]
    out = torch.empty((B, H_q, S_q, D), device=dev)
    ws_bytes = int(L.kf_attn_workspace_bytes(B, H_q, H_kv, S_q, S_kv, D))
    ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=dev)

    def call(i):
        q, k, v = sets[i]
        rc = L.kf_attn_fwd_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), None, None, B, H_q, H_kv,
                              S_q, S_kv, D, causal, ws.data_ptr(), ws_bytes, ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"kf_attn_fwd_ex: {rc}")

    per_phase: dict[int, list] = {}
    n_ctas = sms = 0
    for _ in range(reps):
        for i in range(n_sets - 1):
            call(i)
        torch.cuda.synchronize()
        if L.kf_prefill_trace_clear() != 0:
            raise RuntimeError("kf_prefill_trace_clear")
        call(n_sets - 1)
        torch.cuda.synchronize()
        buf = np.zeros(MAX_CTAS * SLOTS, dtype=np.uint64)
        if L.kf_prefill_trace_read(buf.ctypes.data, MAX_CTAS) != 0:
            raise RuntimeError("kf_prefill_trace_read")
        tr = buf.reshape(MAX_CTAS, SLOTS).astype(np.int64)
        ctas = np.nonzero(tr[:, 0])[0]
        n_ctas, sms = len(ctas), len(set(tr[ctas, SMID].tolist()))
        t0 = tr[ctas, 0].min()
        for k in range(len(PHASES)):
            v = tr[ctas, k]
            v = v[v > 0] - t0
            if len(v):
                per_phase.setdefault(k, []).append((len(v), v.min(), np.median(v), v.max()))
    print(f"{name}: B={B} H_q={H_q} H_kv={H_kv} S_q={S_q} S_kv={S_kv} D={D} causal={causal}: "
          f"{n_ctas} CTAs on {sms} SMs")
    print(f"  {'phase':44s} {'CTAs':>5s} {'min':>7s} {'median':>7s} {'max':>7s}  us since the first CTA's entry")
    order = [0, 1, 17, 18, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 19, 20, 21, 22, 14, 15, 16]
    for k in order:
        if k not in per_phase:
            continue
        a = np.median(np.array(per_phase[k], dtype=np.float64), axis=0)
        print(f"  {PHASES[k]:44s} {int(a[0]):5d} {a[1] / 1e3:7.2f} {a[2] / 1e3:7.2f} {a[3] / 1e3:7.2f}")


def main(argv: list[str]) -> None:
    import torch

    if not torch.cuda.is_available():
        raise SystemExit("phase_trace needs a B200")
    names = argv or ["C1", "chunk_q128"]
    L = ctypes.CDLL(build_traced(), mode=ctypes.RTLD_LOCAL)
    L.kf_attn_fwd_ex.restype = ctypes.c_int
    L.kf_attn_fwd_ex.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_uint, ctypes.c_void_p,
                                                                              ctypes.c_size_t, ctypes.c_void_p]
    L.kf_attn_workspace_bytes.restype = ctypes.c_size_t
    L.kf_attn_workspace_bytes.argtypes = [ctypes.c_int] * 6
    L.kf_prefill_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.kf_prefill_trace_read.restype = ctypes.c_int
    L.kf_prefill_trace_clear.restype = ctypes.c_int
    torch.cuda.set_device(0)
    for n in names:
        trace_case(L, n)


if __name__ == "__main__":
    main(sys.argv[1:])
