"""Host API of the attention forward (torch tensors in, CUDA kernels underneath).

Mirrors the reference's launcher interface (sviraaj/kernelfoundry,
tests/test_flash_attn.cu:52-113 and tests/bench_flash_attn.cu:39-54):

* :func:`launch_flash_attn` -- same name, arguments and meaning as the
  reference's C++ launcher (raw device pointers, B, S, H_q, H_kv, D, stream),
  blocking, returning a status code (0 = success) instead of raising, like the
  reference's ``cudaError_t`` return.
* :func:`flash_attn_fwd` -- the general q_len/kv_len form on torch tensors
  ``[B, H, S, D]`` fp16 -> fp32, asynchronous on the current stream, with the
  reference kernel's optional softmax state (Mi, Li).
* :func:`flash_attn_partial` / :func:`combine_partials` -- (m, l, O_u) partials
  over a KV slice and their log-sum-exp merge (cross-GPU split decode).

torch only supplies device memory and the current stream; the arithmetic runs
in libkf_attn.so (sm_100a).  Nothing here falls back to a CPU path.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from ._lib import KF_FLAG_CAUSAL, KF_FLAG_OUT_BF16, KF_FLAG_OUT_F16, KFError, check, lib

__all__ = [
    "launch_flash_attn",
    "flash_attn_fwd",
    "flash_attn_partial",
    "combine_partials",
    "combine_packed",
    "flash_attn_paged",
    "plan",
    "workspace_bytes",
    "device_error",
    "KFError",
]

_ws_lock = threading.Lock()
_ws_cache: dict[int, torch.Tensor] = {}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream_handle(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check_qkv(q, k, v):
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (no CPU path)")
        if t.dtype != torch.float16:
            raise ValueError(f"{name} must be float16")
        if t.dim() != 4 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous [B, H, S, D] tensor")
    B, H_q, S_q, D = q.shape
    Bk, H_kv, S_kv, Dk = k.shape
    if v.shape != k.shape or Bk != B or Dk != D:
        raise ValueError("k/v shape mismatch with q")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on one device")
    return B, H_q, H_kv, S_q, S_kv, D


def workspace_bytes(B, H_q, H_kv, S_q, S_kv, D) -> int:
    return int(lib().kf_attn_workspace_bytes(B, H_q, H_kv, S_q, S_kv, D))


def _workspace(device: torch.device, nbytes: int):
    """Per-device zero-initialised workspace, grown on demand.

    Calls that overlap on the GPU (different streams) must not share it; use
    the ``workspace=`` argument to give each stream its own.
    """
    if nbytes == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _ws_cache.get(idx)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            _ws_cache[idx] = ws
        return ws


def new_workspace(nbytes: int, device=None) -> torch.Tensor:
    """A private zero-filled workspace (for concurrent streams)."""
    return torch.zeros(max(int(nbytes), 16), dtype=torch.uint8, device=device or torch.device("cuda"))


def plan(B, H_q, H_kv, S_q, S_kv, D, workspace_bytes=2**62):
    """Kernel selection for a call: {'path': 'prefill'|'decode', 'n_split', 'ctas'}.

    'ctas' counts work items (kf_attn_plan's grid_ctas): a prefill with full-size
    tiles runs them on min(items, SM count) persistent CTAs.
    """
    path, ns, ctas = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    check(lib().kf_attn_plan(B, H_q, H_kv, S_q, S_kv, D, workspace_bytes,
                             ctypes.byref(path), ctypes.byref(ns), ctypes.byref(ctas)), "kf_attn_plan")
    return {"path": "prefill" if path.value == 0 else "decode", "n_split": ns.value, "ctas": ctas.value}


_OUT_FLAGS = {torch.float32: 0, torch.float16: KF_FLAG_OUT_F16, torch.bfloat16: KF_FLAG_OUT_BF16}


def flash_attn_fwd(q, k, v, *, out=None, return_lse=False, workspace=None, causal=False, out_dtype=None):
    """O = softmax(Q K^T / sqrt(D)) V per head; GQA head map h_kv = h_q // (H_q // H_kv).

    q [B,H_q,S_q,D] fp16, k/v [B,H_kv,S_kv,D] fp16 (CUDA, contiguous) ->
    O [B,H_q,S_q,D] fp32.  With ``return_lse`` also returns (Mi, Li), the
    reference kernel's row max of the scaled scores and sum of exp(s - Mi).
    ``causal``: bottom-right causal mask, query i attends keys j <= S_kv - S_q + i
    (needs S_q <= S_kv); an extension, the reference has no mask.  ``out_dtype``
    (or the dtype of ``out``): torch.float32 (the reference's), float16 or bfloat16.
    """
    B, H_q, H_kv, S_q, S_kv, D = _check_qkv(q, k, v)
    dev = q.device
    if out is None:
        out = torch.empty((B, H_q, S_q, D), dtype=out_dtype or torch.float32, device=dev)
    elif out_dtype is not None and out.dtype != out_dtype:
        raise ValueError("out and out_dtype disagree")
    if out.dtype not in _OUT_FLAGS:
        raise ValueError("output dtype must be float32, float16 or bfloat16")
    if tuple(out.shape) != (B, H_q, S_q, D) or not out.is_contiguous() or out.device != dev:
        raise ValueError(f"out must be a contiguous [{B}, {H_q}, {S_q}, {D}] tensor on {dev}")
    Mi = Li = None
    if return_lse:
        Mi = torch.empty((B, H_q, S_q), dtype=torch.float32, device=dev)
        Li = torch.empty_like(Mi)
    flags = (KF_FLAG_CAUSAL if causal else 0) | _OUT_FLAGS[out.dtype]
    with torch.cuda.device(dev):
        if workspace is None:
            workspace = _workspace(dev, workspace_bytes(B, H_q, H_kv, S_q, S_kv, D))
        wsb = workspace.numel() if workspace is not None else 0
        rc = lib().kf_attn_fwd_ex(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(Mi), _ptr(Li),
                                  B, H_q, H_kv, S_q, S_kv, D, flags, _ptr(workspace), wsb, _stream_handle(dev))
    check(rc, "kf_attn_fwd_ex")
    return (out, Mi, Li) if return_lse else out


def flash_attn_partial(q, k, v, *, workspace=None, out=None):
    """(O_u, m, l) over the given K/V: O_u = sum exp(s - m) v, m = max s, l = sum exp(s - m).

    `out` = (O_u [B,H_q,S_q,D], m [B,H_q,S_q], l [B,H_q,S_q]) contiguous fp32 views to
    write into (e.g. this rank's slot of an all-gather buffer)."""
    B, H_q, H_kv, S_q, S_kv, D = _check_qkv(q, k, v)
    dev = q.device
    if out is None:
        O_u = torch.empty((B, H_q, S_q, D), dtype=torch.float32, device=dev)
        m = torch.empty((B, H_q, S_q), dtype=torch.float32, device=dev)
        l = torch.empty_like(m)
    else:
        O_u, m, l = out
        for t, shp in ((O_u, (B, H_q, S_q, D)), (m, (B, H_q, S_q)), (l, (B, H_q, S_q))):
            if tuple(t.shape) != shp or t.dtype != torch.float32 or not t.is_contiguous() or t.device != dev:
                raise ValueError(f"out tensors must be contiguous fp32 {shp} on {dev}")
    with torch.cuda.device(dev):
        if workspace is None:
            workspace = _workspace(dev, workspace_bytes(B, H_q, H_kv, S_q, S_kv, D))
        wsb = workspace.numel() if workspace is not None else 0
        rc = lib().kf_attn_fwd_partial(_ptr(q), _ptr(k), _ptr(v), _ptr(O_u), _ptr(m), _ptr(l),
                                       B, H_q, H_kv, S_q, S_kv, D, _ptr(workspace), wsb, _stream_handle(dev))
    check(rc, "kf_attn_fwd_partial")
    return O_u, m, l


def flash_attn_paged(q, k_pool, v_pool, block_table, seq_lens, *, out=None, return_lse=False, workspace=None):
    """Decode attention over a paged KV cache.

    q [B,H_q,S_q,D] fp16; k_pool/v_pool [n_blocks,H_kv,block_size,D] fp16;
    block_table [B,max_blocks] int32 (pool block of each logical block);
    seq_lens [B] int32 (keys per sequence).  Every query row sees its sequence's
    keys (decode shapes: H_q/H_kv * S_q small).  -> O [B,H_q,S_q,D] fp32."""
    for t, name in ((q, "q"), (k_pool, "k_pool"), (v_pool, "v_pool")):
        if not t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous() or t.dim() != 4:
            raise ValueError(f"{name} must be a contiguous 4-D fp16 CUDA tensor (no CPU path)")
    for t, name, nd in ((block_table, "block_table", 2), (seq_lens, "seq_lens", 1)):
        if not t.is_cuda or t.dtype != torch.int32 or not t.is_contiguous() or t.dim() != nd:
            raise ValueError(f"{name} must be a contiguous {nd}-D int32 CUDA tensor")
    B, H_q, S_q, D = q.shape
    n_blocks, H_kv, block_size, D2 = k_pool.shape
    if tuple(v_pool.shape) != tuple(k_pool.shape) or D2 != D:
        raise ValueError("pool shapes must match [n_blocks, H_kv, block_size, D]")
    if block_table.shape[0] != B or seq_lens.shape[0] != B:
        raise ValueError("block_table / seq_lens must have B rows")
    max_blocks = block_table.shape[1]
    dev = q.device
    if out is None:
        out = torch.empty((B, H_q, S_q, D), dtype=torch.float32, device=dev)
    Mi = Li = None
    if return_lse:
        Mi = torch.empty((B, H_q, S_q), dtype=torch.float32, device=dev)
        Li = torch.empty_like(Mi)
    with torch.cuda.device(dev):
        if workspace is None:
            workspace = _workspace(dev, int(lib().kf_attn_paged_workspace_bytes(B, H_q, H_kv, S_q, D, block_size,
                                                                                max_blocks)))
        wsb = workspace.numel() if workspace is not None else 0
        rc = lib().kf_attn_fwd_paged(_ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(block_table), _ptr(seq_lens),
                                     _ptr(out), _ptr(Mi), _ptr(Li), B, H_q, H_kv, S_q, D, n_blocks, block_size,
                                     max_blocks, _ptr(workspace), wsb, _stream_handle(dev))
    check(rc, "kf_attn_fwd_paged")
    return (out, Mi, Li) if return_lse else out


def combine_packed(parts, n_parts, part_stride, shape, *, out=None, return_lse=False):
    """Merge n_parts partials packed back to back in the fp32 buffer `parts`
    (part g at g*part_stride: [O_u rows*D][m rows][l rows]) into O of `shape` (B,H_q,S_q,D)."""
    if not parts.is_cuda or parts.dtype != torch.float32 or not parts.is_contiguous():
        raise ValueError("parts must be a contiguous fp32 CUDA tensor (no CPU path)")
    B, H_q, S_q, D = shape
    if parts.numel() < (n_parts - 1) * part_stride + B * H_q * S_q * (D + 2):
        raise ValueError("parts buffer too small")
    dev = parts.device
    if out is None:
        out = torch.empty((B, H_q, S_q, D), dtype=torch.float32, device=dev)
    Mi = Li = None
    if return_lse:
        Mi = torch.empty((B, H_q, S_q), dtype=torch.float32, device=dev)
        Li = torch.empty_like(Mi)
    with torch.cuda.device(dev):
        rc = lib().kf_attn_combine_packed(_ptr(parts), part_stride, n_parts, _ptr(out), _ptr(Mi), _ptr(Li),
                                          B, H_q, S_q, D, _stream_handle(dev))
    check(rc, "kf_attn_combine_packed")
    return (out, Mi, Li) if return_lse else out


def combine_partials(O_parts, m_parts, l_parts, *, out=None, return_lse=False):
    """Merge stacked partials O_parts [G,B,H,S,D], m/l_parts [G,B,H,S] by log-sum-exp."""
    if not (O_parts.is_cuda and m_parts.is_cuda and l_parts.is_cuda):
        raise ValueError("partials must be CUDA tensors (no CPU path)")
    G, B, H_q, S_q, D = O_parts.shape
    O_parts = O_parts.contiguous()
    m_parts = m_parts.contiguous()
    l_parts = l_parts.contiguous()
    dev = O_parts.device
    if out is None:
        out = torch.empty((B, H_q, S_q, D), dtype=torch.float32, device=dev)
    Mi = Li = None
    if return_lse:
        Mi = torch.empty((B, H_q, S_q), dtype=torch.float32, device=dev)
        Li = torch.empty_like(Mi)
    with torch.cuda.device(dev):
        rc = lib().kf_attn_combine(_ptr(O_parts), _ptr(m_parts), _ptr(l_parts), G, _ptr(out), _ptr(Mi), _ptr(Li),
                                   B, H_q, S_q, D, _stream_handle(dev))
    check(rc, "kf_attn_combine")
    return (out, Mi, Li) if return_lse else out


def launch_flash_attn(Q, K, V, O, B, S, H_q, H_kv, D, stream=0) -> int:
    """Reference-compatible blocking launcher on raw device pointers (ints).

    Same arguments as tests/test_flash_attn.cu:52-58; returns 0 on success or a
    KF_* status (the reference returns cudaError_t; kf_attn_compat.h maps ours
    onto it).  Prefill only: S_q = S_kv = S.
    """
    return int(lib().kf_launch_flash_attn(ctypes.c_void_p(Q), ctypes.c_void_p(K), ctypes.c_void_p(V),
                                          ctypes.c_void_p(O), B, S, H_q, H_kv, D, ctypes.c_void_p(stream)))


def device_error(clear: bool = True):
    """(status, raw bits) of the device error word; synchronizes the device."""
    raw = ctypes.c_uint(0)
    rc = lib().kf_device_error(1 if clear else 0, ctypes.byref(raw))
    return rc, raw.value


def selftest_wait_timeout(timeout_ns: int = 20_000_000) -> int:
    """Run the bounded-wait self-test kernel; returns KF_ERR_DEVICE_TIMEOUT when the wait expired as designed."""
    return int(lib().kf_selftest_wait_timeout(timeout_ns, _stream_handle(torch.device("cuda"))))


def set_wait_timeout_ns(ns: int) -> None:
    lib().kf_set_wait_timeout_ns(int(ns))
