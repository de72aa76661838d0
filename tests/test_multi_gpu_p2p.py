"""KV-split long decode over 2 GPUs with the NVLink peer exchange (no NCCL).

Each rank holds a contiguous KV range; its partials go into the peer's window as
{value, sequence} words, it polls the peer's words in its own window and merges:
either inside the decode kernel (kf_attn_fwd_exchange, one launch) or in a
second kernel after the partial (kf_attn_exchange_combine).  Both paths share
the windows: the fused calls alternate with two-launch calls.
Checked against the fp64 oracle over the whole cache, over several calls
(both parities of the double-buffered slots) and over CUDA-graph replays
(sequence numbers kept on the device).  The failure path: one rank calls
alone with a 50 ms wait limit and must get KF_ERR_DEVICE_TIMEOUT with the
peer bit set, not a hang.  The process group is gloo (it only carries the
IPC handles and barriers).  Needs two visible GPUs; skipped otherwise.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir, mode):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from kernelfoundry_b200 import device_error
    from kernelfoundry_b200._lib import lib
    from kernelfoundry_b200.multi_gpu import PeerExchange, kv_shard, long_decode_forward
    from oracle.attn_oracle import normal_qkv, reference_attn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    ex = None
    try:
        Q, K, V = normal_qkv(2, 8, 2, 1, 20001, 128, seed=5)
        lo, hi = kv_shard(K.shape[2], world, rank)
        q = torch.from_numpy(Q).to(dev)
        k = torch.from_numpy(np.ascontiguousarray(K[:, :, lo:hi])).to(dev)
        v = torch.from_numpy(np.ascontiguousarray(V[:, :, lo:hi])).to(dev)
        ex = PeerExchange(tuple(q.shape), device=dev)
        result = {}
        if mode == "ok":
            assert ex.attend(q, k, v) is not None            # the fused kernel supports this shape
            outs = [long_decode_forward(q, k, v, exchange=ex, fused=(i % 2 == 0)).cpu().numpy() for i in range(6)]
            out = torch.empty(tuple(q.shape), dtype=torch.float32, device=dev)
            stream = torch.cuda.current_stream(dev)
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                long_decode_forward(q, k, v, exchange=ex, out=out)
            stream.wait_stream(side)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                long_decode_forward(q, k, v, exchange=ex, out=out)
            for _ in range(3):
                out.zero_()
                g.replay()
                torch.cuda.synchronize(dev)
                outs.append(out.cpu().numpy())
            del g
            ref = reference_attn(Q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))
            result["err"] = max(float(np.abs(o - ref).max()) for o in outs)
            result["rc"], raw = device_error()
            result["raw"] = raw
        else:
            lib().kf_set_wait_timeout_ns(50_000_000)
            if rank == 0:
                long_decode_forward(q, k, v, exchange=ex)
                result["rc"], result["raw"] = device_error()
            dist.barrier()
            lib().kf_set_wait_timeout_ns(0)
        np.save(os.path.join(result_dir, f"{mode}{rank}.npy"), np.array([result.get("err", 0.0), result.get("rc", -1),
                                                                         result.get("raw", 0)], dtype=np.float64))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


def _run(tmp_path, mode):
    import multiprocessing as mp

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [np.load(tmp_path / f"{mode}{r}.npy") for r in range(2)]


def test_long_decode_peer_exchange_world2(tmp_path):
    for err, rc, raw in _run(tmp_path, "ok"):
        assert err < 2e-3, err
        assert rc == 0 and raw == 0, (rc, raw)


def test_peer_exchange_missing_peer_times_out(tmp_path):
    from kernelfoundry_b200 import _lib

    res = _run(tmp_path, "timeout")
    _, rc, raw = res[0]
    assert int(rc) == _lib.KF_ERR_DEVICE_TIMEOUT
    assert int(raw) & (1 << 4)          # KF_DEVERR_TIMEOUT_PEER
