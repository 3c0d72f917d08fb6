"""Multi-GPU sharding of the attention forward: one process per GPU, no collective in the hot loop.

The reference is single-GPU (Tiny-transformer README.md:48). The work partitions without any
exchange: prefill by (batch x head) pairs, decode by batch rows (balanced by the visible key
count when per-sequence lengths are given). Each rank computes its slice on its own GPU; NCCL
(torch.distributed over NVLink) is used only by :func:`gather_outputs`, when the caller asks
for the full O / LSE on every rank.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch


@dataclass(frozen=True)
class Shard:
    """A contiguous range [start, stop) of the partitioned axis owned by one rank."""
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def even_shards(n_units: int, world: int) -> list[Shard]:
    """Split n_units into `world` contiguous ranges whose sizes differ by at most one."""
    if world <= 0:
        raise ValueError("world size must be positive")
    base, extra = divmod(n_units, world)
    out, start = [], 0
    for r in range(world):
        stop = start + base + (1 if r < extra else 0)
        out.append(Shard(start, stop))
        start = stop
    return out


def balanced_batch_shards(lengths: Sequence[int], world: int) -> list[Shard]:
    """Contiguous batch ranges whose visible-key totals are as even as a prefix split allows:
    rank r's range ends where the running total first reaches (r + 1) / world of the whole."""
    if world <= 0:
        raise ValueError("world size must be positive")
    n = len(lengths)
    total = float(sum(max(0, int(x)) for x in lengths))
    bounds, acc, b = [0], 0.0, 0
    for r in range(1, world):
        target = total * r / world
        while b < n and acc + max(0, int(lengths[b])) <= target:
            acc += max(0, int(lengths[b]))
            b += 1
        # Leave at least one row for every remaining rank when possible.
        b = max(b, bounds[-1])
        b = min(b, n - (world - r)) if n >= world else b
        bounds.append(max(b, bounds[-1]))
    bounds.append(n)
    return [Shard(bounds[i], bounds[i + 1]) for i in range(world)]


def prefill_slice(x: torch.Tensor, shard: Shard) -> torch.Tensor:
    """Rows [start, stop) of the flattened (batch x head) axis of a [B, H, T, D] tensor, as a
    [n, 1, T, D] view (a copy only when B and H cannot be flattened as a view)."""
    B, H, T, D = x.shape
    return x.reshape(B * H, 1, T, D)[shard.start:shard.stop]


def run_sharded(compute: Callable, q, k, v, past_len: int, rank: int, world: int,
                kv_lens: torch.Tensor | None = None):
    """Compute this rank's slice with ``compute(q, k, v, past_len, kv_lens) -> (O, LSE)``.

    Returns (O_local, LSE_local, shard, axis) where axis is "bh" (prefill: O_local is
    [n, 1, Tq, D] over flattened batch x head) or "batch" (decode: O_local is [n, H, 1, D]).
    """
    if q.shape[2] == 1:
        lens = kv_lens.tolist() if kv_lens is not None else [k.shape[2]] * q.shape[0]
        shard = balanced_batch_shards(lens, world)[rank]
        sl = slice(shard.start, shard.stop)
        local_lens = kv_lens[sl] if kv_lens is not None else None
        o, lse = compute(q[sl], k[sl], v[sl], past_len, local_lens)
        return o, lse, shard, "batch"
    shard = even_shards(q.shape[0] * q.shape[1], world)[rank]
    o, lse = compute(prefill_slice(q, shard), prefill_slice(k, shard), prefill_slice(v, shard),
                     past_len, None)
    return o, lse, shard, "bh"


def gather_outputs(o_local: torch.Tensor, lse_local: torch.Tensor, shard_sizes: Sequence[int],
                   full_shape: Sequence[int], axis: str, group=None):
    """All-gather every rank's O / LSE slice into the full [B, H, Tq, D] / [B, H, Tq] tensors
    on every rank (NCCL on GPUs, gloo on CPU). Slices may differ in size: each is padded to
    the largest before the collective and trimmed after."""
    import torch.distributed as dist

    B, H, Tq, D = full_shape
    world = len(shard_sizes)
    n_max = max(shard_sizes)

    def pad(x):
        if x.shape[0] == n_max:
            return x.contiguous()
        fill = torch.zeros((n_max - x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                           device=x.device)
        return torch.cat([x, fill]).contiguous()

    outs = [torch.empty((n_max,) + tuple(o_local.shape[1:]), dtype=o_local.dtype,
                        device=o_local.device) for _ in range(world)]
    lses = [torch.empty((n_max,) + tuple(lse_local.shape[1:]), dtype=lse_local.dtype,
                        device=lse_local.device) for _ in range(world)]
    dist.all_gather(outs, pad(o_local), group=group)
    dist.all_gather(lses, pad(lse_local), group=group)
    o = torch.cat([t[:n] for t, n in zip(outs, shard_sizes)])
    lse = torch.cat([t[:n] for t, n in zip(lses, shard_sizes)])
    if axis == "bh":
        return o.reshape(B, H, Tq, D), lse.reshape(B, H, Tq)
    return o, lse


def sharded_attention(q, k, v, past_len: int = 0, kv_lens: torch.Tensor | None = None,
                      gather: bool = False, group=None):
    """This rank's share of the attention forward on its current CUDA device.

    Without ``gather`` returns (O_local, LSE_local, shard, axis) (see :func:`run_sharded`); with
    it, the full (O, LSE) on every rank, gathered once after the local kernels finish.
    """
    import torch.distributed as dist

    from .operators import student

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0

    def compute(qs, ks, vs, pl, lens):
        return student.attention_with_lse(qs, ks, vs, pl, None, lens)

    o, lse, shard, axis = run_sharded(compute, q, k, v, past_len, rank, world, kv_lens)
    if not gather:
        return o, lse, shard, axis
    if world == 1:
        # The one shard is the whole problem: no collective.
        if axis == "bh":
            B, H, Tq, D = q.shape
            return o.reshape(B, H, Tq, D), lse.reshape(B, H, Tq)
        return o, lse
    if axis == "batch":
        lens = kv_lens.tolist() if kv_lens is not None else [k.shape[2]] * q.shape[0]
        sizes = [s.size for s in balanced_batch_shards(lens, world)]
    else:
        sizes = [s.size for s in even_shards(q.shape[0] * q.shape[1], world)]
    return gather_outputs(o, lse, sizes, tuple(q.shape), axis, group)
