"""CPU oracle for Tiny-transformer's BF16 causal attention forward.

TEST INFRASTRUCTURE ONLY. This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` / ``--impl reference`` leg may
import it. The shipped path (``tiny-transformer_b200``) never calls it and raises when its CUDA
extension is missing.

It restates, in numpy, the arithmetic of the reference's executable specification
(Tiny-transformer ``tiny_transformer/operators/reference.py``):

* ``causal_mask``            -> :func:`causal_allowed`            (reference.py:37-46)
* ``attention`` (bf16 path)  -> :func:`reference_attention_bf16`  (reference.py:12-13, 49-53)
* the FP64 oracle of the reference's CUDA tests -> :func:`attention_fp64`
  (tests/test_student_attention.py:104-117)
* per-sequence valid lengths -> :func:`decode_with_kv_lens`: the reference API has no such
  argument; each batch row is the reference operator on its valid prefix with
  ``past_len = L_b - 1`` (pure reference semantics).

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
``reference.attention`` (PyTorch, CPU) and stored inputs and outputs in
``tests/golden/attention_golden.npz``; ``tests/test_oracle_golden.py`` checks this module
against them.

BF16 tensors are carried as float32 numpy arrays whose values are exactly representable in
bf16 (or as raw uint16 bit patterns, see :func:`bf16_bits_to_f32`).
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634
SCALE = 0.125  # 1/sqrt(64), exact in binary


# ----------------------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN stays NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), rounded)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32/float64 values to the nearest bf16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


# ----------------------------------------------------------------------------- masks
def causal_allowed(tq: int, tk: int, past_len: int = 0) -> np.ndarray:
    """[tq, tk] bool: key j visible to query i iff j <= i + past_len (reference.py:37-41)."""
    q_pos = np.arange(tq, dtype=np.int64) + past_len
    k_pos = np.arange(tk, dtype=np.int64)
    return k_pos[None, :] <= q_pos[:, None]


def _check(q, k, v, past_len):
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4, "q, k, v must be 4D"
    assert q.shape[-1] == 64 and k.shape[-1] == 64 and v.shape[-1] == 64, "head_dim=64"
    assert k.shape[2] == v.shape[2] and k.shape[2] == past_len + q.shape[2], \
        "expected Tk == past_len + Tq"


# ----------------------------------------------------------------------------- reference.py
def reference_attention_bf16(q: np.ndarray, k: np.ndarray, v: np.ndarray, past_len: int = 0,
                             return_lse: bool = False):
    """``reference.attention`` (reference.py:49-53) on BF16 inputs, step by step:

    1. ``torch.matmul(q, k^T)`` in bf16: exact products, FP32 accumulation, one rounding to bf16;
    2. ``/ sqrt(64)``: division by 8, exact in bf16;
    3. ``accumulation(scores)``: cast to FP32; masked positions set to -inf;
    4. FP32 softmax over keys, then ``.to(v.dtype)``: rounded to bf16;
    5. ``torch.matmul(P, v)`` in bf16: FP32 accumulation, rounded to bf16.

    Returns O (float32 holding bf16 values), and with ``return_lse`` also the FP32 logsumexp of
    the step-3 scores (the LSE companion the native operator returns).
    """
    _check(q, k, v, past_len)
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    tq, tk = q.shape[2], k.shape[2]
    allowed = causal_allowed(tq, tk, past_len)
    scores = round_bf16(np.matmul(q, np.swapaxes(k, -1, -2), dtype=np.float32))
    scores = scores * np.float32(SCALE)
    scores = np.where(allowed, scores, np.float32(-np.inf)).astype(np.float32)
    row_max = scores.max(axis=-1, keepdims=True)
    safe_max = np.where(np.isfinite(row_max), row_max, np.float32(0))
    e = np.exp(scores - safe_max, dtype=np.float32)
    denom = e.sum(axis=-1, keepdims=True, dtype=np.float32)
    prob = round_bf16(e / denom)
    out = round_bf16(np.matmul(prob, v, dtype=np.float32))
    if not return_lse:
        return out
    lse = (np.log(denom[..., 0]) + safe_max[..., 0]).astype(np.float32)
    lse = np.where(np.isfinite(row_max[..., 0]), lse, np.float32(-np.inf))
    return out, lse


def attention_fp64(q: np.ndarray, k: np.ndarray, v: np.ndarray, past_len: int = 0):
    """FP64 oracle of the reference's CUDA tests (tests/test_student_attention.py:108-117):
    scores = q.k^T / sqrt(64) in FP64, causal mask, softmax, P.v. Returns (O, LSE), FP64."""
    _check(q, k, v, past_len)
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    tq, tk = q.shape[2], k.shape[2]
    allowed = causal_allowed(tq, tk, past_len)
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) / 8.0
    scores = np.where(allowed, scores, -np.inf)
    row_max = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - row_max)
    denom = e.sum(axis=-1, keepdims=True)
    out = np.matmul(e / denom, v)
    lse = np.log(denom[..., 0]) + row_max[..., 0]
    return out, lse


def attention_backward_fp64(q: np.ndarray, k: np.ndarray, v: np.ndarray, dout: np.ndarray,
                            past_len: int = 0):
    """FP64 gradients of attention_fp64 with respect to q, k, v for upstream ``dout``, in the
    form of the reference's BF16 backward (csrc/attention/attention.cu:161-234 with
    attention_backward_preprocess_kernel.cuh, attention_backward_dKdV_kernel.cu:232-309 and
    attention_backward_dQ_kernel.cu): D = rowsum(dO * O), P = exp(S / 8 - LSE) on visible
    pairs, dS = P * (dO.V^T - D), dQ = dS.K / 8, dK = dS^T.Q / 8, dV = P^T.dO. Returns
    (dQ, dK, dV), FP64."""
    _check(q, k, v, past_len)
    q, k, v, dout = (np.asarray(x, dtype=np.float64) for x in (q, k, v, dout))
    out, lse = attention_fp64(q, k, v, past_len)
    allowed = causal_allowed(q.shape[2], k.shape[2], past_len)
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) / 8.0
    p = np.where(allowed, np.exp(scores - lse[..., None]), 0.0)
    d = (dout * out).sum(axis=-1, keepdims=True)
    ds = p * (np.matmul(dout, np.swapaxes(v, -1, -2)) - d)
    dq = np.matmul(ds, k) / 8.0
    dk = np.matmul(np.swapaxes(ds, -1, -2), q) / 8.0
    dv = np.matmul(np.swapaxes(p, -1, -2), dout)
    return dq, dk, dv


def decode_with_kv_lens(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_lens, fn=attention_fp64):
    """Single-token decode where key j is visible to batch row b iff j < kv_lens[b].

    Each row is the reference operator on its valid prefix with past_len = L_b - 1
    (reference.py:37-53 semantics; the reference API has no per-sequence length). Lengths are
    clamped to [0, Tk]; a row with no visible key gets O = 0 and LSE = -inf, the reference
    kernel's convention for rows without visible keys
    (csrc/attention/attention_forward_BF16_kernel.cuh:367-386).
    ``fn`` is :func:`attention_fp64` or ``reference_attention_bf16(..., return_lse=True)``.
    """
    assert q.shape[2] == 1, "kv_lens requires Tq == 1"
    B, H, _, D = q.shape
    tk = k.shape[2]
    outs = np.zeros((B, H, 1, D), dtype=np.float64)
    lses = np.full((B, H, 1), -np.inf, dtype=np.float64)
    for b in range(B):
        L = int(min(max(int(kv_lens[b]), 0), tk))
        if L == 0:
            continue
        o, lse = fn(q[b:b + 1], k[b:b + 1, :, :L], v[b:b + 1, :, :L], L - 1)
        outs[b] = o[0]
        lses[b] = lse[0]
    return outs, lses


def reference_bf16_with_lse(q, k, v, past_len=0):
    """Convenience: (O, LSE) from :func:`reference_attention_bf16`."""
    return reference_attention_bf16(q, k, v, past_len, return_lse=True)


# ----------------------------------------------------------------------------- counts
def visible_pairs(tq: int, tk: int, past_len: int) -> int:
    """Number of (query, key) pairs with j <= i + past_len, keys < tk."""
    i = np.arange(tq, dtype=np.int64)
    return int(np.minimum(i + past_len + 1, tk).sum())


def prefill_flops(b: int, h: int, tq: int, tk: int, past_len: int) -> int:
    """Algorithmic FLOPs: 2 GEMMs x 2 FLOP x D per visible pair (softmax excluded)."""
    return 4 * b * h * 64 * visible_pairs(tq, tk, past_len)


def decode_bytes(b: int, h: int, lens) -> int:
    """Algorithmic HBM bytes of single-token decode: the visible K and V rows, q, O (bf16)
    and LSE (fp32)."""
    total_keys = int(np.sum(lens)) * h
    return total_keys * 64 * 2 * 2 + b * h * (64 * 2 * 2 + 4)
