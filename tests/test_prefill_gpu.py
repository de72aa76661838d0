"""Parity of the attention forward (prefill shapes) on a B200, through the C ABI.

Oracles: the fp64 NumPy restatement of kernel_models/flash_attn.py:
reference_attn (pinned to the reference's own outputs by test_oracle.py and
tests/golden/), the fp32 C restatement of the reference harness's cpu_attn,
and the reference CUDA kernel itself (oracle/_ref/libkfref.so, built from the
reference sources).  Tolerances: max-abs 2e-3 and rel-L2 1e-3 vs fp64
(north star); max-abs 5e-2 vs fp32 cpu_attn on the 18 harness cases
(tests/test_flash_attn.cu:22).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from oracle.attn_oracle import error_stats, normal_qkv

from conftest import golden_case, golden_names
from gpu_util import assert_close, oracle64, run_fwd, to_dev

pytestmark = pytest.mark.gpu


def test_golden_vectors(cuda, sdpa_golden):
    """Every golden case (prefill, decode, GQA, MQA, D=16/256, ragged) vs the reference's own fp64 output."""
    for name in golden_names(sdpa_golden):
        _, Q, K, V = golden_case(sdpa_golden, name)
        got = run_fwd(Q, K, V, cuda)
        assert_close(got, sdpa_golden[f"{name}/O_ref64"], name)


@pytest.mark.parametrize("case", oracle.LEGACY_CASES, ids=lambda c: "B{}_S{}_Hq{}_Hkv{}_D{}_s{}".format(*c))
def test_legacy_harness_case(cuda, case):
    """The reference harness's 18 cases through the reference-compatible launcher."""
    import torch

    from kernelfoundry_b200 import launch_flash_attn

    B, S, Hq, Hkv, D, seed = case
    (q32, k32, v32), (q16, k16, v16) = oracle.legacy_case_inputs(*case)
    q, k, v = (to_dev(x, cuda) for x in (q16, k16, v16))
    o = torch.full((B, Hq, S, D), float("nan"), dtype=torch.float32, device=cuda)
    rc = launch_flash_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, S, Hq, Hkv, D, 0)
    assert rc == 0
    got = o.cpu().numpy()
    ref32 = oracle.cpu_attn_f32(q32, k32, v32)          # the reference harness's check
    assert np.abs(got - ref32).max() <= oracle.LEGACY_TOL
    ref64 = oracle64(q16, k16, v16)[0]                  # north-star check on the same fp16 inputs
    assert_close(got, ref64, f"legacy {case}")


BASELINE = {
    "C1_prefill_S512": (1, 32, 8, 512, 512, 128, 1001),
    "C2_prefill_S4096": (1, 32, 8, 4096, 4096, 128, 1002),
    "C4_mqa_D64": (4, 32, 1, 2048, 2048, 64, 1004),
}


@pytest.mark.parametrize("name", list(BASELINE))
def test_baseline_configs_full_size(cuda, name):
    B, Hq, Hkv, Sq, Skv, D, seed = BASELINE[name]
    Q, K, V = normal_qkv(B, Hq, Hkv, Sq, Skv, D, seed)
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, name)
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


def test_baseline_prefill_batch8_sampled(cuda):
    """C2 at B=8 (the batch-sharded configuration): full run, oracle on b = 0 and 7."""
    Q, K, V = normal_qkv(8, 32, 8, 4096, 4096, 128, 1012)
    got = run_fwd(Q, K, V, cuda)
    for b in (0, 7):
        ref = oracle64(Q[b:b + 1], K[b:b + 1], V[b:b + 1])[0]
        assert_close(got[b:b + 1], ref, f"b={b}")


RAGGED = [
    (2, 8, 2, 300, 1000, 128),
    (1, 4, 4, 129, 17, 64),
    (1, 2, 1, 257, 300, 256),
    (1, 2, 2, 1000, 129, 16),
    (3, 6, 3, 200, 64, 128),
    (1, 2, 2, 33, 4096, 128),
    (1, 1, 1, 256, 1, 64),
]


@pytest.mark.parametrize("shape", RAGGED, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_ragged_shapes(cuda, shape):
    Q, K, V = normal_qkv(*shape, seed=sum(shape))
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, str(shape))
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


_SPLIT_SHAPES = [(1, 32, 8, 4096, 4096, 128), (3, 8, 2, 700, 1500, 64), (1, 4, 1, 129, 4097, 256),
                 (1, 8, 2, 600, 2048, 128)]     # the last: 4 chunks per split unit (3 donors)


@pytest.mark.parametrize("merge", ["owner", "ticket"])
@pytest.mark.parametrize("shape", _SPLIT_SHAPES, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_tail_split_matches_unsplit(cuda, shape, merge, monkeypatch):
    """A partial last wave split along KV (needs a workspace) gives the unsplit result.

    ``owner``: chunk 0 waits for the other chunks' partials and merges them with its
    own O from TMEM (the default); ``ticket``: the owner's wait is zero, so every chunk
    writes a partial and the last to take a ticket merges (the fallback path)."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd, plan
    from kernelfoundry_b200.attention import new_workspace, workspace_bytes

    if merge == "ticket":
        monkeypatch.setenv("KF_PREFILL_TICKET_MERGE", "1")
    need = workspace_bytes(*shape)
    assert need > 0, "expected a split plan for this shape"
    assert plan(*shape)["ctas"] > plan(*shape, workspace_bytes=0)["ctas"]
    Q, K, V = normal_qkv(*shape, seed=5 * sum(shape))
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    ws = new_workspace(need, cuda)
    split_o, split_mi, split_li = (x.cpu().numpy() for x in flash_attn_fwd(q, k, v, workspace=ws, return_lse=True))
    none = torch.empty(0, dtype=torch.uint8, device=cuda)
    plain_o = flash_attn_fwd(q, k, v, workspace=none).cpu().numpy()
    ma, rl = error_stats(split_o, plain_o)
    assert ma <= 2e-3 and rl <= 1e-3, (ma, rl)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(split_o, O, "split")
    assert np.abs(split_mi - rMi).max() < 1e-3
    assert np.abs(split_li / rLi - 1).max() < 1e-3
    assert int(ws[:65536].view(torch.int32).abs().sum()) == 0     # tickets reset
    half = flash_attn_fwd(q, k, v, workspace=ws, out_dtype=torch.float16).float().cpu().numpy()
    assert_close(half, O, "split fp16 out", max_abs=4e-3)
    assert int(ws[:65536].view(torch.int32).abs().sum()) == 0


@pytest.mark.parametrize("merge", ["owner", "ticket"])
def test_partial_form_split(cuda, merge, monkeypatch):
    """Unnormalized partials (O_u, m, l) of a split plan: O_u / l is the softmax output."""
    from kernelfoundry_b200 import flash_attn_partial
    from kernelfoundry_b200.attention import new_workspace, workspace_bytes

    if merge == "ticket":
        monkeypatch.setenv("KF_PREFILL_TICKET_MERGE", "1")
    shape = (1, 8, 2, 600, 2048, 128)
    need = workspace_bytes(*shape)
    assert need > 0
    Q, K, V = normal_qkv(*shape, seed=91)
    ws = new_workspace(need, cuda)
    O_u, m, l = (t.cpu().numpy() for t in flash_attn_partial(*(to_dev(x, cuda) for x in (Q, K, V)), workspace=ws))
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(O_u / l[..., None], O, "split partial O_u/l")
    assert np.abs(m - rMi).max() < 1e-3
    assert np.abs(l / rLi - 1).max() < 1e-3


def test_partial_form_prefill(cuda):
    from kernelfoundry_b200 import flash_attn_partial

    Q, K, V = normal_qkv(1, 8, 2, 384, 700, 128, seed=77)
    O_u, m, l = (t.cpu().numpy() for t in flash_attn_partial(*(to_dev(x, cuda) for x in (Q, K, V))))
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(O_u / l[..., None], O, "partial O_u/l")
    assert np.abs(m - rMi).max() < 1e-3
    assert np.abs(l / rLi - 1).max() < 1e-3


def _ref_kernel(Q, K, V, device):
    """Run the reference CUDA kernel (compiled from its sources) on the same fp16 inputs."""
    import torch

    ref = oracle.load_ref_lib()
    B, Hq, Sq, D = Q.shape
    Hkv, Skv = K.shape[1], K.shape[2]
    q, k, v = (to_dev(x, device) for x in (Q, K, V))
    o = torch.empty((B, Hq, Sq, D), dtype=torch.float32, device=device)
    mi = torch.empty((B, Hq, Sq), dtype=torch.float32, device=device)
    li = torch.empty_like(mi)
    P = ctypes.c_void_p
    rc = ref.kfref_launch_general(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(o.data_ptr()),
                                  P(mi.data_ptr()), P(li.data_ptr()), B, Sq, Skv, Hq, Hkv, D,
                                  P(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    return o.cpu().numpy(), mi.cpu().numpy(), li.cpu().numpy()


@pytest.mark.parametrize("shape", [(1, 32, 8, 512, 512, 128), (2, 8, 2, 129, 129, 64), (1, 4, 1, 1, 4096, 128),
                                   (3, 8, 8, 1, 777, 256), (1, 2, 1, 16, 16, 16)])
def test_matches_reference_cuda_kernel(cuda, shape):
    """Same fp16 inputs through the reference's own kernel: outputs and Mi/Li agree."""
    Q, K, V = normal_qkv(*shape, seed=3 * sum(shape))
    ref_o, ref_mi, ref_li = _ref_kernel(Q, K, V, cuda)
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    ma, rl = error_stats(got, ref_o)
    assert ma <= 2e-3 and rl <= 1e-3, (ma, rl)
    assert np.abs(Mi - ref_mi).max() < 1e-3
    assert np.abs(Li / ref_li - 1).max() < 1e-3


CAUSAL = [
    (1, 32, 8, 4096, 4096, 128),      # C2 with the mask
    (2, 8, 2, 300, 1000, 128),        # chunk of 300 queries at the end of a 1000-key cache
    (1, 4, 1, 129, 129, 64),
    (1, 2, 1, 257, 300, 256),
    (1, 2, 2, 1000, 1000, 16),
    (1, 32, 8, 7, 2048, 128),         # few queries: decode-sized, but the mask needs the prefill kernel
    (3, 8, 8, 1, 777, 128),           # one query sees every key: decode kernel, same as unmasked
]


@pytest.mark.parametrize("shape", CAUSAL, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_causal_matches_oracle(cuda, shape):
    from oracle.attn_oracle import causal_attn_lse

    from kernelfoundry_b200 import flash_attn_fwd

    Q, K, V = normal_qkv(*shape, seed=11 * sum(shape))
    got, Mi, Li = (t.cpu().numpy() for t in flash_attn_fwd(*(to_dev(x, cuda) for x in (Q, K, V)),
                                                            causal=True, return_lse=True))
    O, rMi, rLi = causal_attn_lse(*(x.astype(np.float64) for x in (Q, K, V)))
    assert_close(got, O, f"causal {shape}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


def test_causal_rejects_more_queries_than_keys(cuda):
    from kernelfoundry_b200 import KFError, flash_attn_fwd

    Q, K, V = normal_qkv(1, 2, 1, 65, 64, 64, seed=1)
    with pytest.raises(KFError):
        flash_attn_fwd(*(to_dev(x, cuda) for x in (Q, K, V)), causal=True)


OUT16 = [
    (1, 32, 8, 4096, 4096, 128, False),     # C2, tail split: partials fp32, merged O 16-bit
    (2, 8, 2, 300, 1000, 128, True),
    (1, 4, 1, 129, 129, 64, False),
    (1, 2, 1, 257, 300, 256, False),
    (1, 2, 2, 1000, 1000, 16, True),        # D=16: direct row stores
    (4, 32, 8, 1, 4096, 128, False),        # decode, one split
    (1, 32, 8, 1, 131072, 128, False),      # decode with KV split and merge
]


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("shape", OUT16, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}_c{}".format(*s))
def test_half_precision_output(cuda, shape, dtype):
    """O written as fp16 / bf16: the fp32 result rounded to nearest, within one output ulp
    of the oracle plus the north-star bar."""
    import torch

    from oracle.attn_oracle import causal_attn_lse

    from kernelfoundry_b200 import flash_attn_fwd

    *dims, causal = shape
    Q, K, V = normal_qkv(*dims, seed=7 * sum(dims))
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    tdt = getattr(torch, dtype)
    got, Mi, Li = flash_attn_fwd(q, k, v, causal=causal, out_dtype=tdt, return_lse=True)
    assert got.dtype == tdt
    f32 = flash_attn_fwd(q, k, v, causal=causal)
    # Same arithmetic, then one rounding: equals the fp32 output rounded to the type.
    assert torch.equal(got, f32.to(tdt))
    ref = (causal_attn_lse if causal else oracle64)(*(x.astype(np.float64) for x in (Q, K, V)))[0]
    ulp = 2.0 ** -8 if dtype == "bfloat16" else 2.0 ** -11
    g = got.float().cpu().numpy()
    assert np.abs(g - ref).max() <= 2e-3 + ulp * np.abs(ref).max()
    assert np.linalg.norm(g - ref) / np.linalg.norm(ref) <= 1e-3 + ulp


@pytest.mark.parametrize("D,causal", [(128, False), (128, True), (64, False), (256, False)])
def test_lazy_rescale_paths(cuda, D, causal):
    """Scores that jump by more than 2^8 between KV tiles and between the two
    halves of a tile, on some rows only: drives the O rescale, the reload of
    the first half of S, and the warp-uniform decision with rows that do not
    need it.  Random N(0,1) data almost never reaches these paths."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd

    B, Hq, Hkv, S = 1, 4, 2, 1024
    bc = 128 if D <= 128 else 64
    rng = np.random.default_rng(D + causal)
    Q = rng.standard_normal((B, Hq, S, D)).astype(np.float16)
    K = rng.standard_normal((B, Hkv, S, D)).astype(np.float16)
    V = rng.standard_normal((B, Hkv, S, D)).astype(np.float16)
    s = np.arange(S)
    # Feature 0 carries a bias: +8 per KV tile and +4 in the second half of each
    # tile; query rows alternate between feeling it (q0 = 16) and not (q0 = 0).
    K[..., 0] = (8 * (s // bc) + 4 * ((s % bc) >= bc // 2)).astype(np.float16)
    Q[..., 0] = np.where((np.arange(S) // 3) % 2 == 0, 16.0, 0.0).astype(np.float16)
    q, k, v = (torch.from_numpy(x).to(cuda) for x in (Q, K, V))
    got = flash_attn_fwd(q, k, v, causal=causal).cpu().numpy()
    if causal:
        from oracle.attn_oracle import causal_attn_lse
        ref = causal_attn_lse(Q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))[0]
    else:
        ref = oracle64(Q, K, V)[0]
    assert_close(got, ref, f"rescale D={D} causal={causal}")


@pytest.mark.parametrize("kvh", ["1", "0"])
@pytest.mark.parametrize("shape", [(1, 32, 8, 512, 512, 128), (1, 32, 8, 300, 300, 64), (1, 16, 4, 384, 500, 16),
                                   (2, 8, 8, 129, 700, 128), (1, 32, 8, 256, 256, 128), (1, 32, 8, 512, 500, 128),
                                   (1, 16, 4, 300, 512, 64), (2, 8, 8, 200, 256, 16), (1, 8, 2, 64, 512, 128),
                                   (2, 4, 4, 100, 256, 64)],
                         ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_single_tile_units(cuda, shape, kvh, monkeypatch):
    """Short sequences run one 128-row query tile per CTA (twice the CTAs of two-tile units).
    With an even count of 128-key tiles the CTA's two softmax warpgroups take the keys' two
    halves and the halves are merged in TMEM (KF_PREFILL_KVH=0: one warpgroup over all keys).
    Results and softmax state match the fp64 oracle."""
    from kernelfoundry_b200 import plan

    monkeypatch.setenv("KF_PREFILL_KVH", kvh)
    B, H_q, H_kv, S_q, S_kv, D = shape
    assert plan(*shape)["ctas"] == B * H_q * ((S_q + 127) // 128)
    Q, K, V = normal_qkv(*shape, seed=sum(shape) + 9)
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, str(shape))
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


def test_key_half_units_outputs(cuda):
    """Key-half units (C1's shape): fp16 output and the unnormalized partial form."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd, flash_attn_partial

    Q, K, V = normal_qkv(1, 32, 8, 512, 512, 128, seed=4242)
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    O, rMi, rLi = oracle64(Q, K, V)
    half = flash_attn_fwd(q, k, v, out_dtype=torch.float16).float().cpu().numpy()
    assert_close(half, O, "key halves, fp16 out", max_abs=4e-3)
    O_u, m, l = (t.cpu().numpy() for t in flash_attn_partial(q, k, v))
    assert_close(O_u / l[..., None], O, "key halves, partial O_u/l")
    assert np.abs(m - rMi).max() < 1e-3
    assert np.abs(l / rLi - 1).max() < 1e-3


@pytest.mark.parametrize("shape", [(1, 32, 8, 512, 512, 128), (1, 8, 2, 1, 4096, 128), (1, 4, 1, 4096, 4096, 128)],
                         ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_back_to_back_dependent_calls(cuda, shape):
    """Launch overlap (programmatic dependent launch) must not let a call read inputs before the
    previous call on the stream has written them: call i+1 takes call i's fp16 output as its Q,
    with no host synchronisation between the calls, eagerly and replayed in a CUDA graph."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd
    from kernelfoundry_b200.attention import new_workspace, workspace_bytes

    B, H_q, H_kv, S_q, S_kv, D = shape
    Q, K, V = normal_qkv(*shape, seed=sum(shape) + 3)
    k, v = to_dev(K, cuda), to_dev(V, cuda)
    ws = new_workspace(max(workspace_bytes(*shape), 16), cuda)
    n = 4
    outs = [torch.empty((B, H_q, S_q, D), dtype=torch.float16, device=cuda) for _ in range(n)]
    q0 = to_dev(Q, cuda)

    def chain():
        q = q0
        for i in range(n):
            flash_attn_fwd(q, k, v, out=outs[i], workspace=ws)
            q = outs[i]

    # Reference: the same chain on the host, each step's fp16 output as the next Q.
    ref_q = Q
    refs = []
    for i in range(n):
        o = oracle64(ref_q, K, V)[0]
        refs.append(o)
        ref_q = o.astype(np.float16)
    chain()
    for i in range(n):
        assert_close(outs[i].float().cpu().numpy(), refs[i], f"eager step {i}", max_abs=4e-3)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    for o in outs:
        o.zero_()
    g.replay()
    torch.cuda.synchronize()
    for i in range(n):
        assert_close(outs[i].float().cpu().numpy(), refs[i], f"graph step {i}", max_abs=4e-3)
    del g


CAUSAL_SPLIT = [(1, 32, 8, 512, 4096, 128), (1, 16, 4, 256, 2048, 64), (2, 8, 2, 300, 1500, 128),
                (1, 8, 8, 128, 1024, 256), (1, 8, 2, 1024, 2048, 128)]


@pytest.mark.parametrize("merge", ["owner", "ticket"])
@pytest.mark.parametrize("shape", CAUSAL_SPLIT, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_causal_chunked_prefill_split(cuda, shape, merge, monkeypatch):
    """Causal chunked prefill over a long cache (S_kv >= 2 S_q) with few units: the last wave's
    units are split along their own keys (evenly, every row seeing keys in every chunk) and
    merged; results, softmax state and the zeroed counters against the causal oracle."""
    import torch

    from oracle.attn_oracle import causal_attn_lse

    from kernelfoundry_b200 import flash_attn_fwd
    from kernelfoundry_b200.attention import new_workspace, workspace_bytes

    if merge == "ticket":
        monkeypatch.setenv("KF_PREFILL_TICKET_MERGE", "1")
    need = workspace_bytes(*shape)
    Q, K, V = normal_qkv(*shape, seed=13 * sum(shape))
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    ws = new_workspace(max(need, 16), cuda)
    got, Mi, Li = (t.cpu().numpy() for t in flash_attn_fwd(q, k, v, causal=True, return_lse=True, workspace=ws))
    O, rMi, rLi = causal_attn_lse(*(x.astype(np.float64) for x in (Q, K, V)))
    assert np.isfinite(got).all()
    assert_close(got, O, f"causal split {shape}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3
    assert int(ws[:65536].view(torch.int32).abs().sum()) == 0
    plain = flash_attn_fwd(q, k, v, causal=True, workspace=torch.empty(0, dtype=torch.uint8, device=cuda))
    ma, rl = error_stats(got, plain.cpu().numpy())
    assert ma <= 2e-3 and rl <= 1e-3, (ma, rl)


# (8, 32, 8, 128, 512, 16): D = 16 (no staged store) with two items on most CTAs;
# (8, 32, 8, 128, 1024, 64): the eight-slot ring of D = 64 over several items.
SHORT_CHUNKS = [(1, 32, 8, 128, 4096, 128), (2, 8, 2, 100, 2048, 64), (1, 16, 4, 128, 3000, 128),
                (1, 8, 8, 64, 1024, 16), (8, 32, 8, 128, 1024, 128), (3, 8, 2, 128, 512, 128),
                (8, 32, 8, 128, 512, 16), (8, 32, 8, 128, 1024, 64)]


@pytest.mark.parametrize("merge", ["owner", "ticket"])
@pytest.mark.parametrize("shape", SHORT_CHUNKS, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_short_query_chunks(cuda, shape, merge, monkeypatch):
    """Up to 128 queries over a longer cache: one-tile units whose two chains take the keys'
    halves (merged in TMEM), split along KV when the units are few (each chunk's halves merged
    in TMEM, then the chunks by the owner or by ticket), and over several rounds when many.
    Results, softmax state and zeroed counters against the fp64 oracle and the one-chain form."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd
    from kernelfoundry_b200.attention import new_workspace, workspace_bytes

    if merge == "ticket":
        monkeypatch.setenv("KF_PREFILL_TICKET_MERGE", "1")
    Q, K, V = normal_qkv(*shape, seed=17 * sum(shape))
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    ws = new_workspace(max(workspace_bytes(*shape), 16), cuda)
    got, Mi, Li = (t.cpu().numpy() for t in flash_attn_fwd(q, k, v, return_lse=True, workspace=ws))
    O, rMi, rLi = oracle64(Q, K, V)
    assert np.isfinite(got).all()
    assert_close(got, O, f"short chunk {shape}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3
    assert int(ws[:65536].view(torch.int32).abs().sum()) == 0
    half = flash_attn_fwd(q, k, v, out_dtype=torch.float16, workspace=ws).float().cpu().numpy()
    assert_close(half, O, "short chunk fp16 out", max_abs=4e-3)
    monkeypatch.setenv("KF_PREFILL_KVH", "0")
    one_chain = flash_attn_fwd(q, k, v, workspace=ws).cpu().numpy()
    ma, rl = error_stats(got, one_chain)
    assert ma <= 2e-3 and rl <= 1e-3, (ma, rl)
