"""``student`` attention operator on the sm_100a kernels.

Same signature, guards and error behaviour as Tiny-transformer's
``tiny_transformer/operators/student.py:190-232`` (the ``_Attention`` autograd bridge and the
``attention`` operator), plus one optional, additive argument ``kv_lens``. Selected in the
reference with ``--op attention=student`` once its ``load_attention_extension`` returns this
package's native module (``tt_attention_C``, loaded by ``_extension.load_attention_extension``).

Differences from the reference operator, all deliberate:
* FP32 inputs raise (the reference ran an FP32 SIMT kernel; this path is BF16 only);
* ``kv_lens`` (int32/int64 CUDA ``[B]``, Tq must be 1): key j is visible to batch row b iff
  ``j < kv_lens[b]``; ``past_len`` must still equal ``Tk - 1``. It is a decode-time argument:
  combined with inputs that require grad it raises ``NotImplementedError``.
"""
from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from ._extension import load_attention_extension


def _guard(q, k, v):
    if not all(x.is_cuda for x in (q, k, v)):
        raise RuntimeError("student attention requires q, k, v to be CUDA tensors")
    if torch.is_autocast_enabled("cuda"):
        raise RuntimeError("student attention does not support AMP/autocast yet")


def _needs_grad(q, k, v):
    return torch.is_grad_enabled() and any(x.requires_grad for x in (q, k, v))


class _Attention(torch.autograd.Function):
    """BF16 forward + backward through the native module (student.py:190-211): the forward
    saves q, k, v (the original views, so autograd checks their versions and maps gradients to
    their bases), O and the FP32 LSE; the backward runs the sm_100a dQ / dK / dV kernels."""

    @staticmethod
    def forward(ctx, q, k, v, past_len, segment_ids):
        output, lse = load_attention_extension().attention_forward(q, k, v, past_len, segment_ids)
        ctx.save_for_backward(q, k, v, output, lse)
        ctx.past_len = past_len
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        q, k, v, output, lse = ctx.saved_tensors
        dq, dk, dv = load_attention_extension().attention_backward(
            q, k, v, grad_output, output, lse, ctx.past_len, None)
        return (dq if ctx.needs_input_grad[0] else None,
                dk if ctx.needs_input_grad[1] else None,
                dv if ctx.needs_input_grad[2] else None, None, None)


def attention(q, k, v, past_len=0, segment_ids=None, kv_lens=None):
    """BF16 CUDA causal attention forward, head_dim=64; returns O (B,H,Tq,64) BF16, contiguous.

    Key j is visible to query row i iff ``j <= i + past_len`` with ``Tk == past_len + Tq``
    (reference.py:37-53). Strided views are read in place when their last stride is 1, other
    strides are multiples of 8 elements and the base is 16-byte aligned (KV-cache prefixes);
    other views are copied first, as the reference does. Runs on the current CUDA stream.
    """
    _guard(q, k, v)
    if _needs_grad(q, k, v):
        if any(x.dtype != torch.bfloat16 for x in (q, k, v)):
            raise NotImplementedError(
                "student attention backward supports only bf16; FP32 backward is not implemented")
        if kv_lens is not None:
            raise NotImplementedError("student attention backward does not take kv_lens")
        return _Attention.apply(q, k, v, past_len, segment_ids)
    output, _ = load_attention_extension().attention_forward(q, k, v, past_len, segment_ids,
                                                             kv_lens)
    return output


def attention_with_lse(q, k, v, past_len=0, segment_ids=None, kv_lens=None):
    """Like :func:`attention` but returns ``(O, LSE)``; LSE is FP32 (B,H,Tq), natural log, the
    format the reference's BF16 backward consumes (attention.cu:161-234)."""
    _guard(q, k, v)
    if _needs_grad(q, k, v):
        raise NotImplementedError(
            "attention_with_lse records no autograd graph (no backward); use attention() for "
            "training or call it under torch.no_grad()")
    return load_attention_extension().attention_forward(q, k, v, past_len, segment_ids, kv_lens)
