"""Parity of the short-query (decode) split-KV path on a B200, through the C ABI.

The reference's own harness never checks decode (all 18 cases have
S_q = S_kv); these cases are pinned by the fp64 oracle (reference_attn, which
handles S_q != S_kv) and by the reference CUDA kernel in test_prefill_gpu.py.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.attn_oracle import normal_qkv

from gpu_util import assert_close, oracle64, run_fwd, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B", [1, 16, 64])
def test_c3_decode_kv4096(cuda, B):
    from kernelfoundry_b200 import plan

    Q, K, V = normal_qkv(B, 32, 8, 1, 4096, 128, seed=3000 + B)
    assert plan(B, 32, 8, 1, 4096, 128)["path"] == "decode"
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, f"decode B={B}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


def test_c5_long_decode(cuda):
    from kernelfoundry_b200 import plan

    Q, K, V = normal_qkv(1, 32, 8, 1, 131072, 128, seed=5005)
    pl = plan(1, 32, 8, 1, 131072, 128)
    assert pl["path"] == "decode" and pl["n_split"] > 1
    got = run_fwd(Q, K, V, cuda)
    assert_close(got, oracle64(Q, K, V)[0], "long decode")


SHAPES = [
    (4, 32, 1, 1, 2048, 64),     # MQA, D=64 (two 16-row tiles)
    (2, 32, 1, 1, 1000, 128),    # MQA, D=128
    (3, 8, 8, 1, 777, 256),      # D=256
    (2, 4, 1, 1, 300, 16),       # D=16
    (1, 40, 8, 1, 513, 128),     # GQA ratio 5
    (2, 32, 8, 2, 1024, 128),    # S_q = 2 (speculative-style short query)
    (1, 32, 8, 8, 700, 128),     # R = 32
    (1, 32, 1, 2, 4096, 64),     # R = 64 -> two row groups
    (1, 8, 2, 1, 1, 128),        # single key
    (2, 8, 2, 1, 63, 128),
    (2, 8, 2, 1, 65, 128),
    (1, 8, 2, 1, 4097, 128),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_decode_shapes(cuda, shape):
    from kernelfoundry_b200 import plan

    assert plan(*shape)["path"] == "decode"
    Q, K, V = normal_qkv(*shape, seed=7 * sum(shape))
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, str(shape))
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


def test_workspace_optional_and_reusable(cuda, monkeypatch):
    """Split merges through the workspace (the cluster merge off): no workspace (single
    split) and a shared workspace reused across shapes give correct results."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd, plan
    from kernelfoundry_b200.attention import new_workspace, workspace_bytes

    monkeypatch.setenv("KF_DECODE_CLUSTER", "0")
    assert plan(1, 32, 8, 1, 4096, 128, workspace_bytes=0)["n_split"] == 1
    ws = new_workspace(max(workspace_bytes(1, 32, 8, 1, 8192, 128), workspace_bytes(4, 32, 8, 1, 3000, 128)), cuda)
    for shape in [(1, 32, 8, 1, 8192, 128), (4, 32, 8, 1, 3000, 128), (1, 32, 8, 1, 8192, 128), (2, 8, 2, 1, 999, 128)]:
        Q, K, V = normal_qkv(*shape, seed=sum(shape))
        q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
        ref = oracle64(Q, K, V)[0]
        out_ws = flash_attn_fwd(q, k, v, workspace=ws).cpu().numpy()
        out_none = flash_attn_fwd(q, k, v, workspace=torch.empty(0, dtype=torch.uint8, device=cuda)).cpu().numpy()
        assert_close(out_ws, ref, f"ws {shape}")
        assert_close(out_none, ref, f"no-ws {shape}")
    # The ticket counters at the head of the workspace are back to zero.
    assert int(ws[:65536].view(torch.int32).abs().sum()) == 0


def test_partials_and_combine_match_full(cuda):
    """Per-slice partials (as on G GPUs) merged by kf_attn_combine == attention over the whole cache."""
    import torch

    from kernelfoundry_b200 import combine_partials, flash_attn_partial

    Q, K, V = normal_qkv(1, 32, 8, 1, 16384, 128, seed=99)
    q = to_dev(Q, cuda)
    cuts = [0, 4096, 4097, 10000, 16384]
    parts = [flash_attn_partial(q, to_dev(K[:, :, lo:hi].copy(), cuda), to_dev(V[:, :, lo:hi].copy(), cuda))
             for lo, hi in zip(cuts[:-1], cuts[1:])]
    O_p = torch.stack([p[0] for p in parts])
    m_p = torch.stack([p[1] for p in parts])
    l_p = torch.stack([p[2] for p in parts])
    out, Mi, Li = combine_partials(O_p, m_p, l_p, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(out.cpu().numpy(), O, "combined")
    assert np.abs(Mi.cpu().numpy() - rMi).max() < 1e-3
    assert np.abs(Li.cpu().numpy() / rLi - 1).max() < 1e-3


def test_combine_packed_matches_combine(cuda):
    """Partials written into the slots of one packed buffer ([O_u | m | l] per part, as an
    all-gather leaves them) merge to the same result as the stacked form."""
    import torch

    from kernelfoundry_b200 import combine_packed, combine_partials, flash_attn_partial

    Q, K, V = normal_qkv(2, 16, 4, 1, 9000, 128, seed=123)
    q = to_dev(Q, cuda)
    B, H_q, S_q, D = Q.shape
    rows = B * H_q * S_q
    n = (rows * (D + 2) + 3) // 4 * 4
    cuts = [0, 3000, 3001, 9000]
    G = len(cuts) - 1
    buf = torch.full((G * n,), float("nan"), dtype=torch.float32, device=cuda)
    stacked = []
    for g, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:])):
        k = to_dev(K[:, :, lo:hi].copy(), cuda)
        v = to_dev(V[:, :, lo:hi].copy(), cuda)
        slot = buf[g * n:(g + 1) * n]
        views = (slot[:rows * D].view(B, H_q, S_q, D), slot[rows * D:rows * D + rows].view(B, H_q, S_q),
                 slot[rows * D + rows:rows * (D + 2)].view(B, H_q, S_q))
        flash_attn_partial(q, k, v, out=views)
        stacked.append(flash_attn_partial(q, k, v))
    got, Mi, Li = combine_packed(buf, G, n, (B, H_q, S_q, D), return_lse=True)
    ref = combine_partials(torch.stack([s[0] for s in stacked]), torch.stack([s[1] for s in stacked]),
                           torch.stack([s[2] for s in stacked]))
    assert torch.equal(got, ref)                       # same arithmetic, same order: bit-exact
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got.cpu().numpy(), O, "packed")
    assert np.abs(Mi.cpu().numpy() - rMi).max() < 1e-3
    assert np.abs(Li.cpu().numpy() / rLi - 1).max() < 1e-3


def test_long_decode_forward_single_process(cuda):
    """The in-place (partial -> slot -> packed combine) path with one rank == full attention."""
    import torch

    from kernelfoundry_b200.multi_gpu import long_decode_forward

    Q, K, V = normal_qkv(1, 32, 8, 1, 20000, 128, seed=321)
    out = torch.empty((1, 32, 1, 128), dtype=torch.float32, device=cuda)
    got = long_decode_forward(*(to_dev(x, cuda) for x in (Q, K, V)), out=out)
    assert got.data_ptr() == out.data_ptr()
    assert_close(out.cpu().numpy(), oracle64(Q, K, V)[0], "long decode, one rank")


@pytest.mark.parametrize("cluster", ["0", "1"])
@pytest.mark.parametrize("nsplit", ["8", "16", "32"])
def test_split_merge_paths(cuda, nsplit, cluster, monkeypatch):
    """Forced split counts (KF_DECODE_NSPLIT): the merge of 8, 16 and 32 partials -- the
    cluster merge in distributed shared memory (up to 16 splits) or the last CTA's ticket
    merge through the workspace (KF_DECODE_CLUSTER=0, and 32 splits) -- gives the oracle's
    result."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd, plan

    monkeypatch.setenv("KF_DECODE_NSPLIT", nsplit)
    monkeypatch.setenv("KF_DECODE_CLUSTER", cluster)
    Q, K, V = normal_qkv(2, 32, 8, 1, 40000, 128, seed=int(nsplit))
    assert plan(2, 32, 8, 1, 40000, 128)["n_split"] == int(nsplit)
    got, Mi, Li = (t.cpu().numpy() for t in flash_attn_fwd(*(to_dev(x, cuda) for x in (Q, K, V)), return_lse=True))
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, f"nsplit {nsplit}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


DEEP_SHAPES = [
    (1, 32, 8, 1, 4096, 128),    # the C3 B=1 shape
    (3, 32, 8, 1, 1000, 128),    # ragged last stage
    (2, 8, 2, 1, 777, 64),       # D=64
    (1, 40, 8, 1, 2049, 128),    # GQA ratio 5, one key past a stage
    (2, 16, 8, 2, 513, 16),      # D=16, S_q=2
]


@pytest.mark.parametrize("deep", [0, 1])
@pytest.mark.parametrize("n_split", [1, 3, 16])
@pytest.mark.parametrize("shape", DEEP_SHAPES, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_decode_ring_variants(cuda, shape, n_split, deep, monkeypatch):
    """Both decode kernels -- one consumer group with the 3-stage ring, and the deep ring
    with two consumer groups taking alternate stages -- at forced split counts agree with
    the fp64 oracle (the planner normally chooses between them; the overrides are its
    benchmark sweep switches)."""
    B, H_q, H_kv, S_q, S_kv, D = shape
    monkeypatch.setenv("KF_DECODE_DEEP", str(deep))
    monkeypatch.setenv("KF_DECODE_NSPLIT", str(n_split))
    Q, K, V = normal_qkv(*shape, seed=sum(shape) + 31 * n_split + deep)
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, f"deep={deep} n_split={n_split} {shape}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3


CLUSTER_SHAPES = [
    (1, 32, 8, 1, 4096, 128),    # the C3 B=1 shape
    (3, 32, 8, 1, 1000, 128),    # ragged last stage
    (1, 32, 1, 1, 4096, 128),    # MQA: 32 packed rows (two 16-row MMA tiles per CTA)
    (2, 32, 1, 2, 1500, 128),    # 64 packed rows: two row groups per KV head (grid y = 2)
    (2, 8, 2, 1, 1100, 64),      # D=64
    (2, 16, 8, 2, 1090, 16),     # D=16, S_q=2
    (1, 8, 8, 1, 3000, 256),     # D=256
]


# Every shape has more 64-key stages than the largest forced split count (the override
# applies only up to one stage per split).
@pytest.mark.parametrize("n_split", [2, 5, 16])
@pytest.mark.parametrize("shape", CLUSTER_SHAPES, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_cluster_merge(cuda, shape, n_split, monkeypatch):
    """Split decode merged inside a thread-block cluster (the unit's splits read each other's
    partials from distributed shared memory; no workspace): O, Mi, Li against the fp64
    oracle, the fp16 output, and the unnormalized partial form."""
    import torch

    from kernelfoundry_b200 import flash_attn_fwd, flash_attn_partial, plan
    from kernelfoundry_b200.attention import workspace_bytes

    monkeypatch.setenv("KF_DECODE_NSPLIT", str(n_split))
    monkeypatch.setenv("KF_DECODE_DEEP", "0")
    stages = (shape[4] + 63) // 64
    per = (stages + n_split - 1) // n_split
    want = (stages + per - 1) // per
    assert plan(*shape)["n_split"] == want
    assert workspace_bytes(*shape) == 0          # the cluster plan needs no workspace
    Q, K, V = normal_qkv(*shape, seed=sum(shape) + 7 * n_split)
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    got, Mi, Li = (t.cpu().numpy() for t in flash_attn_fwd(q, k, v, return_lse=True))
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, f"cluster n_split={n_split} {shape}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3
    half = flash_attn_fwd(q, k, v, out_dtype=torch.float16).float().cpu().numpy()
    assert_close(half, O, "cluster fp16 out", max_abs=4e-3)
    O_u, m, l = (t.cpu().numpy() for t in flash_attn_partial(q, k, v))
    assert_close(O_u / l[..., None], O, "cluster partial O_u/l")


@pytest.mark.parametrize("shape", [(1, 32, 8, 1, 4096, 128), (2, 8, 2, 1, 1100, 64), (1, 16, 4, 1, 9000, 128)],
                         ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_cluster_merge_deep_ring(cuda, shape, monkeypatch):
    """The deep-ring kernel (two consumer groups, one CTA per SM) with its splits merged in a
    thread-block cluster, where every cluster of the launch fits on the GPU at once."""
    from kernelfoundry_b200 import plan
    from kernelfoundry_b200.attention import workspace_bytes

    monkeypatch.setenv("KF_DECODE_DEEP", "1")
    monkeypatch.setenv("KF_DECODE_NSPLIT", "16")
    stages = (shape[4] + 63) // 64
    per = (stages + 15) // 16
    assert plan(*shape)["n_split"] == (stages + per - 1) // per
    Q, K, V = normal_qkv(*shape, seed=sum(shape) + 77)
    got, Mi, Li = run_fwd(Q, K, V, cuda, return_lse=True)
    O, rMi, rLi = oracle64(Q, K, V)
    assert_close(got, O, f"deep cluster {shape}")
    assert np.abs(Mi - rMi).max() < 1e-3
    assert np.abs(Li / rLi - 1).max() < 1e-3
    # Whether the cluster merge or the workspace merge ran depends on how many 16-CTA
    # clusters of one-CTA-per-SM blocks this GPU can hold; both must agree with the oracle.
    assert workspace_bytes(*shape) >= 0

