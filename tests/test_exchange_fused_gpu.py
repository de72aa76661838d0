"""The decode kernel with the cross-GPU exchange fused in (kf_attn_fwd_exchange), on one GPU.

With a world of one rank the kernel still runs its whole exchange: the CTA that
merges a (b, h_kv) unit's KV splits writes the unit's partial as {value,
sequence} words into the (own) window, polls them back and merges.  Checked
against the fp64 oracle over several calls (both parities of the double-buffered
slots), CUDA-graph replays (sequence numbers kept on the device) and the shapes
the fused kernel declines.  The two-rank exchange is in test_multi_gpu_p2p.py.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.attn_oracle import normal_qkv

from gpu_util import assert_close, oracle64, to_dev

pytestmark = pytest.mark.gpu

SHAPES = [
    (1, 32, 8, 1, 16384, 128),    # the 8-GPU slice of the long-context config
    (2, 8, 2, 1, 20001, 128),     # ragged
    (1, 40, 8, 1, 4097, 128),     # GQA ratio 5
    (2, 16, 8, 2, 3000, 128),     # two query positions
    (1, 32, 8, 1, 300, 128),      # short: one split
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}_Hq{}_Hkv{}_Sq{}_Skv{}_D{}".format(*s))
def test_fused_exchange_world1(cuda, shape):
    import torch

    from kernelfoundry_b200 import device_error
    from kernelfoundry_b200.multi_gpu import PeerExchange

    B, H_q, H_kv, S_q, S_kv, D = shape
    Q, K, V = normal_qkv(*shape, seed=sum(shape) + 17)
    O, rMi, rLi = oracle64(Q, K, V)
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    ex = PeerExchange(tuple(q.shape), device=cuda)
    try:
        for call in range(3):
            Mi = torch.empty((B, H_q, S_q), dtype=torch.float32, device=cuda)
            Li = torch.empty_like(Mi)
            out = ex.attend(q, k, v, Mi=Mi, Li=Li)
            assert out is not None
            torch.cuda.synchronize()
            assert_close(out.cpu().numpy(), O, f"call {call}")
            assert np.abs(Mi.cpu().numpy() - rMi).max() < 1e-3
            assert np.abs(Li.cpu().numpy() / rLi - 1).max() < 1e-3
        out = torch.empty((B, H_q, S_q, D), dtype=torch.float32, device=cuda)
        stream = torch.cuda.current_stream(cuda)
        side = torch.cuda.Stream(cuda)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            ex.attend(q, k, v, out=out)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ex.attend(q, k, v, out=out)
        for _ in range(3):
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert_close(out.cpu().numpy(), O, "graph replay")
        del g
        rc, raw = device_error()
        assert rc == 0 and raw == 0, (rc, raw)
    finally:
        ex.close()


def test_fused_exchange_declines_unsupported_shapes(cuda):
    import torch

    from kernelfoundry_b200.multi_gpu import PeerExchange, long_decode_forward

    Q, K, V = normal_qkv(1, 8, 2, 1, 1000, 64, seed=3)     # D = 64: two-launch path
    q, k, v = (to_dev(x, cuda) for x in (Q, K, V))
    ex = PeerExchange(tuple(q.shape), device=cuda)
    try:
        assert ex.attend(q, k, v) is None
        out = long_decode_forward(q, k, v, exchange=ex)     # falls back to partial + exchange kernel
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), oracle64(Q, K, V)[0], "two-launch path")
    finally:
        ex.close()
