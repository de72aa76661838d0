"""Multi-GPU partitioning of the attention forward (one process per GPU).

The reference is single-GPU; the path shards naturally:

* **batch / KV-head sharding** (prefill, batched decode): each rank owns
  ``B/world`` sequences, or, when there are fewer sequences than ranks, a
  contiguous group of KV heads together with their ``H_q/H_kv`` query heads.
  No communication: every rank runs :func:`flash_attn_fwd` on its own shard.
* **KV-sequence sharding** (single-sequence long-context decode): the KV
  cache is cut into ``world`` contiguous ranges, each rank computes the
  softmax partials (m, l, O_u) of its range ([rows*(D+2)] fp32; 16.6 KB at
  H_q=32, D=128) and they are merged by log-sum-exp on every rank.  Two
  exchanges: one NCCL all-gather followed by the library's combine kernel,
  or (:class:`PeerExchange`) one kernel that writes the partials into every
  peer's window over NVLink, waits for the peers' flags and merges.

The compute callables default to the CUDA kernels; tests on CPU ranks (gloo)
inject stand-ins to check the partitioning and the exchange.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

__all__ = ["shard_range", "batch_shard", "head_shard", "kv_shard", "long_decode_forward", "pack_partials",
           "unpack_partials", "PeerExchange"]


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of n items for `rank`; the first n % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def batch_shard(B: int, world: int, rank: int) -> tuple[int, int]:
    """Sequences [lo, hi) of rank `rank` (no exchange)."""
    return shard_range(B, world, rank)


def head_shard(H_q: int, H_kv: int, world: int, rank: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """(query-head range, KV-head range) of `rank` when sharding by KV-head group.

    KV heads are split contiguously; each rank takes the query heads
    h_kv*G .. (h_kv+1)*G-1 of its KV heads (the reference's GQA grouping,
    kernels/flash_attn.cu:406), so no KV head is needed on two ranks.
    """
    if H_q % H_kv:
        raise ValueError("H_q must be a multiple of H_kv")
    G = H_q // H_kv
    lo, hi = shard_range(H_kv, world, rank)
    return (lo * G, hi * G), (lo, hi)


def kv_shard(S_kv: int, world: int, rank: int) -> tuple[int, int]:
    """KV positions [lo, hi) held by `rank` in the long-context split."""
    return shard_range(S_kv, world, rank)


def pack_partials(O_u: torch.Tensor, m: torch.Tensor, l: torch.Tensor) -> torch.Tensor:
    """[rows*D + 2*rows] fp32 buffer: O_u, then m, then l."""
    return torch.cat([O_u.reshape(-1), m.reshape(-1), l.reshape(-1)])


def unpack_partials(buf: torch.Tensor, world: int, shape_o, shape_m):
    """Inverse of pack_partials on the gathered [world, n] buffer -> stacked (O, m, l)."""
    rows = 1
    for s in shape_m:
        rows *= s
    n_o = buf.shape[1] - 2 * rows
    O = buf[:, :n_o].reshape(world, *shape_o)
    m = buf[:, n_o:n_o + rows].reshape(world, *shape_m)
    l = buf[:, n_o + rows:].reshape(world, *shape_m)
    return O, m, l


def _cuda_partial(q, k, v):
    from .attention import flash_attn_partial

    return flash_attn_partial(q, k, v)


def _cuda_combine(O_p, m_p, l_p):
    from .attention import combine_partials

    return combine_partials(O_p, m_p, l_p)


class _DevArray:
    """A raw device range as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape, device: torch.device):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device = device


class PeerExchange:
    """NVLink peer windows for the long-context decode exchange (one per rank).

    Collective constructor: every rank of ``group`` allocates a window
    (``kf_peer_window_alloc``), the CUDA IPC handles are all-gathered over
    ``group`` (any backend; only host objects travel) and every peer window is
    mapped into this process.  ``staging(shape)`` returns (O_u, m, l) tensors
    over the own window's staging part, where :func:`flash_attn_partial`
    writes; ``combine(out)`` launches the exchange-and-merge kernel.  Both are
    stream-ordered and allocation-free (CUDA-graph capturable).  Every rank
    must make the same sequence of calls.  ``close()`` (collective) unmaps.
    """

    def __init__(self, shape, group: Optional[dist.ProcessGroup] = None, n_chunks: Optional[int] = None,
                 device: Optional[torch.device] = None):
        import ctypes

        from ._lib import KF_PEER_HANDLE_BYTES, check, lib

        B, H_q, S_q, D = shape
        self.shape = (B, H_q, S_q, D)
        self.rows = B * H_q * S_q
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.part_stride = (self.rows * (D + 2) + 3) // 4 * 4
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.n_chunks = int(n_chunks or max(1, min(sms, self.rows)))   # up to one row per CTA
        L = lib()
        nbytes = L.kf_peer_window_bytes(self.world, self.part_stride, self.n_chunks)
        if nbytes == 0:
            raise ValueError("unsupported exchange shape or world size")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * KF_PEER_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            check(L.kf_peer_window_alloc(nbytes, ctypes.byref(own), handle), "kf_peer_window_alloc")
        self._own = own.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs = []
        self._opened = []
        with torch.cuda.device(self.device):
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                buf = (ctypes.c_ubyte * KF_PEER_HANDLE_BYTES).from_buffer_copy(handles[r])
                peer = ctypes.c_void_p()
                check(L.kf_peer_window_open(buf, ctypes.byref(peer)), "kf_peer_window_open")
                ptrs.append(peer.value)
                self._opened.append(peer.value)
        self._windows = (ctypes.c_void_p * self.world)(*ptrs)
        self._xws = None                       # split workspace of the fused path (attend)
        self._xws_shape = None
        rows, dev = self.rows, self.device
        self._stage = (torch.as_tensor(_DevArray(self._own, (B, H_q, S_q, D), dev), device=dev),
                       torch.as_tensor(_DevArray(self._own + rows * D * 4, (B, H_q, S_q), dev), device=dev),
                       torch.as_tensor(_DevArray(self._own + rows * (D + 1) * 4, (B, H_q, S_q), dev), device=dev))

    def staging(self):
        """(O_u [B,H_q,S_q,D], m [B,H_q,S_q], l [B,H_q,S_q]) over the own staging part."""
        return self._stage

    def combine(self, out: Optional[torch.Tensor] = None, Mi: Optional[torch.Tensor] = None,
                Li: Optional[torch.Tensor] = None) -> torch.Tensor:
        import ctypes

        from ._lib import check, lib

        B, H_q, S_q, D = self.shape
        if out is None:
            out = torch.empty(self.shape, dtype=torch.float32, device=self.device)
        if out.shape != self.shape or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError("out must be a contiguous float32 tensor of the exchange shape")
        p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        check(lib().kf_attn_exchange_combine(self._windows, self.world, self.rank, self.part_stride, self.n_chunks,
                                             p(out), p(Mi), p(Li), B, H_q, S_q, D, stream),
              "kf_attn_exchange_combine")
        return out

    def attend(self, q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
               out: Optional[torch.Tensor] = None, Mi: Optional[torch.Tensor] = None,
               Li: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """One launch for the whole decode step (kf_attn_fwd_exchange): attention of q over
        this rank's KV range, with each (b, h_kv) unit's partial sent to every rank's
        window and merged with the other ranks' partials inside the same kernel.  Returns
        the full O, or None when the shape is outside what the fused kernel supports
        (D = 128, world 1/2/4/8, one wave): the caller then uses the two-launch path.
        Every rank must make the same calls (the same choice follows from the same
        shapes)."""
        import ctypes

        from ._lib import KF_ERR_INVALID_ARG, check, lib

        if tuple(q.shape) != self.shape:
            raise ValueError("exchange was built for another shape")
        B, H_q, S_q, D = self.shape
        H_kv, S_kv = k_shard.shape[1], k_shard.shape[2]
        L = lib()
        if self._xws is None or self._xws_shape != (H_kv, S_kv):
            nbytes = int(L.kf_attn_exchange_workspace_bytes(B, H_q, H_kv, S_q, S_kv, D))
            self._xws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=self.device)
            self._xws_shape = (H_kv, S_kv)
        if out is None:
            out = torch.empty(self.shape, dtype=torch.float32, device=self.device)
        if out.shape != self.shape or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError("out must be a contiguous float32 tensor of the exchange shape")
        for t, name in ((q, "q"), (k_shard, "k"), (v_shard, "v")):
            if not t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"{name} must be a contiguous fp16 tensor on {self.device}")
        p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        rc = L.kf_attn_fwd_exchange(p(q), p(k_shard), p(v_shard), self._windows, self.world, self.rank,
                                    self.part_stride, p(out), p(Mi), p(Li), B, H_q, H_kv, S_q, S_kv, D,
                                    p(self._xws), self._xws.numel(), stream)
        if rc == KF_ERR_INVALID_ARG:
            return None
        check(rc, "kf_attn_fwd_exchange")
        return out

    def close(self) -> None:
        """Collective: unmap the peers' windows, then free the own one."""
        from ._lib import check, lib

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)       # no peer still writes into the own window
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                check(lib().kf_peer_window_close(ptr), "kf_peer_window_close")
            if self.world > 1:
                dist.barrier(group=self.group)   # every mapping of the own window is gone
            check(lib().kf_peer_window_free(self._own), "kf_peer_window_free")
        self._own = None
        self._opened = []
        self._stage = None


def long_decode_forward(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                        group: Optional[dist.ProcessGroup] = None,
                        partial_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None,
                        gather_buf: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None,
                        exchange: Optional[PeerExchange] = None, fused: Optional[bool] = None) -> torch.Tensor:
    """Attention of q over a KV cache split across the ranks of `group`.

    q [B,H_q,S_q,D] is replicated; k_shard/v_shard [B,H_kv,S_r,D] hold this
    rank's contiguous KV range (kv_shard()).  Returns the full O on every rank.
    Every rank makes the same single collective call (all_gather_into_tensor).

    With the CUDA kernels (the default) the partials are written straight into
    this rank's slot of `gather_buf` ([world * B*H_q*S_q*(D+2)] fp32, reusable
    across calls), gathered in place and merged from the packed layout: one
    partial launch, one all-gather, one combine launch and no host-side copies,
    so a decode step can be captured in a CUDA graph.  `partial_fn` /
    `combine_fn` substitute the compute (tests on CPU ranks).

    With ``exchange`` (a :class:`PeerExchange` of q's shape) and ``fused``, one decode
    kernel computes this rank's partials, sends them over NVLink and merges
    (:meth:`PeerExchange.attend`); shapes it does not support, or ``fused=False``, take
    two launches: the partials go to the exchange's staging part and one kernel
    exchanges them and merges.  Neither calls NCCL.  ``fused=None`` picks the fused
    kernel for two ranks only: measured on B200 (KV=131072, B=1) it takes 53.7 us
    against 54.9 us at 2 GPUs, but 38.2 / 31.6 us against 37.5 / 25.1 us at 4 / 8 GPUs,
    where one CTA per (b, h_kv) pushing the unit to every peer is slower than the
    exchange kernel's 32 CTAs.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if exchange is not None:
        from .attention import flash_attn_partial

        if tuple(q.shape) != exchange.shape:
            raise ValueError("exchange was built for another shape")
        if fused is None:
            fused = exchange.world <= 2
        if fused:
            res = exchange.attend(q, k_shard, v_shard, out=out)
            if res is not None:
                return res
        flash_attn_partial(q, k_shard, v_shard, out=exchange.staging())
        return exchange.combine(out=out)
    if partial_fn is None and combine_fn is None:
        from .attention import combine_packed, flash_attn_partial

        B, H_q, S_q, D = q.shape
        rows = B * H_q * S_q
        n = rows * (D + 2)
        n = (n + 3) // 4 * 4                      # 16-byte aligned slots
        rank = dist.get_rank(group) if world > 1 else 0
        if gather_buf is None or gather_buf.numel() != world * n or gather_buf.device != q.device:
            gather_buf = torch.empty(world * n, dtype=torch.float32, device=q.device)
        slot = gather_buf[rank * n:(rank + 1) * n]
        O_u = slot[:rows * D].view(B, H_q, S_q, D)
        m = slot[rows * D:rows * D + rows].view(B, H_q, S_q)
        l = slot[rows * D + rows:rows * (D + 2)].view(B, H_q, S_q)
        flash_attn_partial(q, k_shard, v_shard, out=(O_u, m, l))
        if world > 1:
            dist.all_gather_into_tensor(gather_buf, slot, group=group)   # in place: slot is this rank's part
        return combine_packed(gather_buf, world, n, (B, H_q, S_q, D), out=out)
    partial_fn = partial_fn or _cuda_partial
    combine_fn = combine_fn or _cuda_combine
    O_u, m, l = partial_fn(q, k_shard, v_shard)
    if world == 1:
        return combine_fn(O_u.unsqueeze(0), m.unsqueeze(0), l.unsqueeze(0))
    local = pack_partials(O_u, m, l)
    if gather_buf is None or gather_buf.numel() != world * local.numel():
        gather_buf = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(gather_buf, local, group=group)   # concatenation form (NCCL and gloo)
    O_p, m_p, l_p = unpack_partials(gather_buf.view(world, -1), world, tuple(O_u.shape), tuple(m.shape))
    return combine_fn(O_p, m_p, l_p)
