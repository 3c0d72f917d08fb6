"""``student`` attention operator on the sm_100a kernels.

Same signature, guards and error behaviour as Tiny-transformer's
``tiny_transformer/operators/student.py:214-232`` for the BF16 forward path, plus one optional,
additive argument ``kv_lens``. Selected in the reference with ``--op attention=student`` once its
``load_attention_extension`` returns this package's native module.

Differences from the reference operator, all deliberate:
* FP32 inputs raise (the reference ran an FP32 SIMT kernel; this path is BF16 only);
* autograd (the reference's BF16 backward) is not provided: inputs that require grad under
  grad mode raise ``NotImplementedError`` mentioning ``backward``;
* ``kv_lens`` (int32/int64 CUDA ``[B]``, Tq must be 1): key j is visible to batch row b iff
  ``j < kv_lens[b]``; ``past_len`` must still equal ``Tk - 1``.
"""
from __future__ import annotations

import torch

from ._extension import load_attention_extension


def _guard(q, k, v):
    if not all(x.is_cuda for x in (q, k, v)):
        raise RuntimeError("student attention requires q, k, v to be CUDA tensors")
    if torch.is_autocast_enabled("cuda"):
        raise RuntimeError("student attention does not support AMP/autocast yet")
    if torch.is_grad_enabled() and any(x.requires_grad for x in (q, k, v)):
        raise NotImplementedError(
            "student attention backward is not provided by the sm_100a forward path; "
            "run under torch.no_grad() or select --op attention=reference for training")


def attention(q, k, v, past_len=0, segment_ids=None, kv_lens=None):
    """BF16 CUDA causal attention forward, head_dim=64; returns O (B,H,Tq,64) BF16, contiguous.

    Key j is visible to query row i iff ``j <= i + past_len`` with ``Tk == past_len + Tq``
    (reference.py:37-53). Strided views are read in place when their last stride is 1, other
    strides are multiples of 8 elements and the base is 16-byte aligned (KV-cache prefixes);
    other views are copied first, as the reference does. Runs on the current CUDA stream.
    """
    _guard(q, k, v)
    output, _ = load_attention_extension().attention_forward(q, k, v, past_len, segment_ids,
                                                             kv_lens)
    return output


def attention_with_lse(q, k, v, past_len=0, segment_ids=None, kv_lens=None):
    """Like :func:`attention` but returns ``(O, LSE)``; LSE is FP32 (B,H,Tq), natural log, the
    format the reference's BF16 backward consumes (attention.cu:161-234)."""
    _guard(q, k, v)
    return load_attention_extension().attention_forward(q, k, v, past_len, segment_ids, kv_lens)
