"""Multi-GPU partitioning of the attention forward (one process per GPU).

The reference is single-GPU; the path shards naturally:

* **batch / KV-head sharding** (prefill, batched decode): each rank owns
  ``B/world`` sequences, or, when there are fewer sequences than ranks, a
  contiguous group of KV heads together with their ``H_q/H_kv`` query heads.
  No communication: every rank runs :func:`flash_attn_fwd` on its own shard.
* **KV-sequence sharding** (single-sequence long-context decode): the KV
  cache is cut into ``world`` contiguous ranges, each rank computes the
  softmax partials (m, l, O_u) of its range, one NCCL all-gather exchanges
  them ([rows*(D+2)] fp32 per rank; 16.6 KB at H_q=32, D=128), and every rank
  merges them by log-sum-exp with the library's combine kernel.

The compute callables default to the CUDA kernels; tests on CPU ranks (gloo)
inject stand-ins to check the partitioning and the exchange.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

__all__ = ["shard_range", "batch_shard", "head_shard", "kv_shard", "long_decode_forward", "pack_partials",
           "unpack_partials"]


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


def long_decode_forward(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                        group: Optional[dist.ProcessGroup] = None,
                        partial_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None,
                        gather_buf: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
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
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
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
