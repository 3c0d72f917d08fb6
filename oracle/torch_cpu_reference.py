"""The reference's own arithmetic path on the host CPU, for the timed CPU baseline.

TEST / MEASUREMENT INFRASTRUCTURE ONLY. ``bench.py`` times this module as the CPU baseline
(``cpu_baseline`` and ``--impl reference``); nothing in the shipped package imports it.

Tiny-transformer's ``reference`` backend is PyTorch code (tiny_transformer/operators/reference.py),
which does not exist on the machine that runs the benchmark. This module issues the same ATen
operations in the same order on CPU tensors, so the timed work is the reference's own CPU path:

* ``causal_mask``            -> :func:`causal_allowed`   (reference.py:37-46, no segment ids)
* ``attention``              -> :func:`attention`        (reference.py:12-13, 49-53): bf16
  ``matmul(q, k^T)``, division by ``sqrt(D)``, ``.float()``, ``masked_fill(-inf)``, FP32
  ``softmax``, ``.to(v.dtype)``, bf16 ``matmul(P, v)``.

:func:`attention_lse` adds the FP32 logsumexp of the same masked scores (the LSE the native
operator returns alongside O). The bit-level checker of the GPU kernels stays the numpy
restatement in ``attention_oracle.py``; this file exists to time the ATen path.
"""
from __future__ import annotations

import math
import os

import torch


def host_threads() -> int:
    """Host cores available to this process (the thread count the baseline runs with)."""
    if hasattr(os, "sched_getaffinity"):
        return max(1, len(os.sched_getaffinity(0)))
    return max(1, os.cpu_count() or 1)


def causal_allowed(tq: int, tk: int, past_len: int = 0) -> torch.Tensor:
    """[1, 1, tq, tk] bool: key j visible to query i iff j <= i + past_len (reference.py:37-41)."""
    q_pos = torch.arange(tq) + past_len
    k_pos = torch.arange(tk)
    return (k_pos[None, :] <= q_pos[:, None])[None, None]


def _masked_scores(q, k, past_len):
    scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    allowed = causal_allowed(q.shape[-2], k.shape[-2], past_len)
    return scores.float().masked_fill(~allowed, float("-inf"))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, past_len: int = 0) -> torch.Tensor:
    """``reference.attention`` on CPU tensors (bf16 in, bf16 out)."""
    scores = _masked_scores(q, k, past_len)
    probability = torch.softmax(scores, dim=-1).to(v.dtype)
    return torch.matmul(probability, v)


def attention_lse(q, k, v, past_len: int = 0):
    """(O, LSE): ``reference.attention`` plus the FP32 logsumexp of its masked scores."""
    scores = _masked_scores(q, k, past_len)
    lse = torch.logsumexp(scores, dim=-1)
    probability = torch.softmax(scores, dim=-1).to(v.dtype)
    return torch.matmul(probability, v), lse


def prefill_rows(q, k, v, past_len: int = 0, rows_per_call: int = 4):
    """The reference operator over every (batch, head) row of [B, H, T, 64] inputs, called on
    groups of ``rows_per_call`` rows so the FP32 score matrices stay bounded in host memory.
    Returns O [B, H, Tq, 64]."""
    B, H, Tq, D = q.shape
    rows = B * H
    qf, kf, vf = (x.reshape(1, rows, x.shape[2], D) for x in (q, k, v))
    out = torch.empty((1, rows, Tq, D), dtype=v.dtype)
    for r0 in range(0, rows, rows_per_call):
        r1 = min(rows, r0 + rows_per_call)
        out[:, r0:r1] = attention(qf[:, r0:r1], kf[:, r0:r1], vf[:, r0:r1], past_len)
    return out.reshape(B, H, Tq, D)


def decode_rows(q, k, v, kv_lens):
    """Single-token decode with per-sequence lengths: row b is ``reference.attention`` on its
    valid prefix with ``past_len = L_b - 1``. Returns O [B, H, 1, 64]."""
    out = torch.zeros(q.shape, dtype=v.dtype)
    for b in range(q.shape[0]):
        L = int(kv_lens[b])
        if L <= 0:
            continue
        out[b:b + 1] = attention(q[b:b + 1], k[b:b + 1, :, :L], v[b:b + 1, :, :L], L - 1)
    return out
