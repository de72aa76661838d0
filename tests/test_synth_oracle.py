"""The NumPy restatement of the counter-based input generator (oracle/synth_oracle.py).

splitmix64 is pinned by the published test vector of Vigna's splitmix64.c
(seed 1234567); Box-Muller and the fp16 rounding by direct evaluation of the
definition in include/kf_synth.h for single elements; the stream by its
offset/slice identity and its moments.
"""
from __future__ import annotations

import math

import numpy as np

from oracle.synth_oracle import normal_f16, splitmix64


def test_splitmix64_known_answer():
    assert splitmix64(1234567, np.arange(5)).tolist() == [
        6457827717110365317, 3203168211198807973, 9817491932198370423, 4593380528125082431,
        16408922859458223821]


def _element(seed, i):
    """One element straight from the definition, with Python integers and math."""
    m = (1 << 64) - 1

    def w(c):
        z = (seed + (c + 1) * 0x9E3779B97F4A7C15) & m
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
        return z ^ (z >> 31)

    k = i // 2
    u1 = ((w(2 * k) >> 11) + 1) * 2.0 ** -53
    u2 = (w(2 * k + 1) >> 11) * 2.0 ** -53
    r = math.sqrt(-2.0 * math.log(u1))
    t = 6.283185307179586 * u2
    return np.float16(r * (math.cos(t) if i % 2 == 0 else math.sin(t)))


def test_elements_follow_the_definition():
    for seed in (0, 1, 2**64 - 1, 0x1234ABCD):
        got = normal_f16(64, seed, 1000)
        want = np.array([_element(seed, 1000 + j) for j in range(64)], dtype=np.float16)
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), seed


def test_offsets_slice_one_stream():
    full = normal_f16(4099, 77)
    for off in (0, 1, 2, 3, 1024, 4098):
        part = normal_f16(4099 - off, 77, off)
        assert np.array_equal(part.view(np.uint16), full[off:].view(np.uint16)), off
    # chunking inside the generator does not change the values
    assert np.array_equal(normal_f16(4096, 77, 3, chunk=33).view(np.uint16), full[3:4099].view(np.uint16))
    assert normal_f16(0, 77, 5).size == 0


def test_moments_and_seeds():
    x = normal_f16(1 << 20, 2024).astype(np.float64)
    assert abs(x.mean()) < 5e-3 and abs(x.std() - 1.0) < 5e-3
    assert np.abs(x).max() < 8.6                     # sqrt(-2 ln 2^-53)
    y = normal_f16(1 << 12, 2025).astype(np.float64)
    assert abs(np.corrcoef(x[:1 << 12], y)[0, 1]) < 0.06


def test_long_decode_rank_slices_rebuild_one_cache():
    """bench.py's per-rank KV ranges of the long-context decode are slices of one cache."""
    import bench
    from kernelfoundry_b200.multi_gpu import kv_shard

    s_kv, H, D = 96, bench.H_KV, bench.D
    n = H * s_kv * D
    full_k = normal_f16(n, bench.LONG_KV_SEED, 0).reshape(H, s_kv, D)
    full_v = normal_f16(n, bench.LONG_KV_SEED, n).reshape(H, s_kv, D)
    for world in (1, 2, 4, 8):
        ks, vs = [], []
        for rank in range(world):
            lo, hi = kv_shard(s_kv, world, rank)
            k = np.empty((H, hi - lo, D), np.float16)
            v = np.empty_like(k)
            for h in range(H):
                k_off, v_off = bench.long_kv_offsets(h, lo, s_kv)
                k[h] = normal_f16((hi - lo) * D, bench.LONG_KV_SEED, k_off).reshape(hi - lo, D)
                v[h] = normal_f16((hi - lo) * D, bench.LONG_KV_SEED, v_off).reshape(hi - lo, D)
            ks.append(k)
            vs.append(v)
        assert np.array_equal(np.concatenate(ks, 1).view(np.uint16), full_k.view(np.uint16)), world
        assert np.array_equal(np.concatenate(vs, 1).view(np.uint16), full_v.view(np.uint16)), world
