"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference tree (its root given by --ref-root):

    make -C oracle ref            # builds oracle/_ref/libkfref.so from the reference sources
    python tests/golden/make_golden.py [--ref-root REFERENCE_TREE]

Writes (small, committed):
  tests/golden/sdpa_golden.npz      outputs of the reference's own
      kernel_models/flash_attn.py:reference_attn (fp64, on fp16-rounded seeded
      N(0,1) inputs) for prefill / decode / GQA / MQA / D=16 / D=256 / ragged
      shapes, of its tile model flash_attn_kernel for prefill shapes, and of its
      __main__ smoke test (np.random.seed(42), D = 16/64/128).
  tests/golden/legacy18_golden.npz  for the 18 cases of
      tests/test_flash_attn.cu:295-318: SHA-256 digests (and leading values) of
      the fp32 inputs made by the reference's fill_random_f32 and of the
      outputs of its fp32 cpu_attn, both run from oracle/_ref/libkfref.so.

The reference itself only runs here; on the GPU box the tests read these files.
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import LEGACY_CASES, load_ref_lib  # noqa: E402
from oracle.attn_oracle import normal_qkv  # noqa: E402

# (name, B, H_q, H_kv, S_q, S_kv, D, seed)
SDPA_CASES = [
    ("prefill_gqa", 1, 4, 2, 48, 48, 64, 1),
    ("decode_gqa", 2, 8, 2, 1, 300, 128, 2),
    ("mqa_ragged", 1, 8, 1, 17, 40, 64, 3),
    ("d16", 1, 2, 1, 16, 16, 16, 4),
    ("d256_ragged", 1, 2, 2, 5, 33, 256, 5),
    ("decode_long", 1, 4, 1, 1, 1024, 128, 6),
    ("prefill_ratio5", 1, 10, 2, 33, 33, 128, 7),
]
TILE_MODEL_CASES = ["prefill_gqa", "d16", "prefill_ratio5"]


def load_reference_model(ref_root):
    path = os.path.join(ref_root, "kernel_models", "flash_attn.py")
    spec = importlib.util.spec_from_file_location("kf_reference_model", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_sdpa(ref_model, out_path):
    data = {}
    for name, B, Hq, Hkv, Sq, Skv, D, seed in SDPA_CASES:
        Q, K, V = normal_qkv(B, Hq, Hkv, Sq, Skv, D, seed)
        O64 = ref_model.reference_attn(Q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))
        data[f"{name}/shape"] = np.array([B, Hq, Hkv, Sq, Skv, D, seed], dtype=np.int64)
        data[f"{name}/Q"] = Q.view(np.uint16)
        data[f"{name}/K"] = K.view(np.uint16)
        data[f"{name}/V"] = V.view(np.uint16)
        data[f"{name}/O_ref64"] = O64
        if name in TILE_MODEL_CASES:
            assert Sq == Skv
            O_tile = ref_model.flash_attn_kernel(Q.astype(np.float32), K.astype(np.float32),
                                                 V.astype(np.float32), kv_block_rows=16)
            data[f"{name}/O_tile32"] = O_tile
    # The reference model's own smoke test (kernel_models/flash_attn.py:269-281).
    np.random.seed(42)
    for D in (16, 64, 128):
        B, S, Hq, Hkv = 1, 16, 2, 1
        Q = np.random.randn(B, Hq, S, D).astype(np.float32)
        K = np.random.randn(B, Hkv, S, D).astype(np.float32)
        V = np.random.randn(B, Hkv, S, D).astype(np.float32)
        data[f"smoke{D}/tile"] = ref_model.flash_attn_kernel(Q, K, V, kv_block_rows=S)
        data[f"smoke{D}/ref"] = ref_model.reference_attn(Q, K, V)
    np.savez_compressed(out_path, **data)


def make_legacy(out_path):
    lib = load_ref_lib()
    P = ctypes.c_void_p
    rows = []
    heads = []
    for (B, S, Hq, Hkv, D, seed) in LEGACY_CASES:
        qn, kn = B * Hq * S * D, B * Hkv * S * D
        arrs = []
        for n, s in ((qn, seed), (kn, seed + 1), (kn, seed + 2)):
            a = np.empty(n, np.float32)
            lib.kfref_fill_random_f32(a.ctypes.data_as(P), n, -1.0, 1.0, s)
            arrs.append(a)
        q, k, v = arrs
        o = np.empty(qn, np.float32)
        lib.kfref_cpu_attn(q.ctypes.data_as(P), k.ctypes.data_as(P), v.ctypes.data_as(P),
                           o.ctypes.data_as(P), B, S, Hq, Hkv, D)
        rows.append([sha(q), sha(k), sha(v), sha(o)])
        heads.append(np.concatenate([q[:8], k[:8], v[:8], o[:8]]))
    np.savez_compressed(out_path, cases=np.array(LEGACY_CASES, dtype=np.int64),
                        digests=np.array(rows), heads=np.stack(heads))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))),
                                                         "reference"),
                    help="reference checkout (default: the directory `reference` beside this repository)")
    args = ap.parse_args()
    ref_model = load_reference_model(args.ref_root)
    make_sdpa(ref_model, os.path.join(HERE, "sdpa_golden.npz"))
    make_legacy(os.path.join(HERE, "legacy18_golden.npz"))
    for f in ("sdpa_golden.npz", "legacy18_golden.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
