"""Fused operators around the attention call (the caller side of the hot path)."""
from ._extension import load_attention_extension


def rope_append(qkv, cos, sin, position, cache_k, cache_v):
    """RoPE on q and k of a fused QKV projection plus the KV-cache append, in one kernel.

    ``qkv`` is the contiguous ``[B, T, 3, H, 64]`` BF16 output of the QKV linear (the
    reference reshapes it the same way, model.py:60); ``cos`` / ``sin`` are FP32 ``[L, 32]``
    tables indexed by position; ``position`` is the first position (an int, or a one-element
    int64 CUDA tensor read on the device). Writes rope(k) and v into rows ``position + t`` of
    the ``[B, H, C, 64]`` caches and returns rope(q) as ``[B, H, T, 64]``. Bit-exact with the
    reference's bf16 ``rope`` (reference.py:30-34) followed by ``KVCache.update``
    (model.py:29-41).
    """
    return load_attention_extension().rope_append(qkv, cos, sin, position, cache_k, cache_v)


def qkv_rope_append(hidden, w_qkv, cos, sin, position, cache_k, cache_v):
    """The QKV projection of a decoder layer with RoPE and the KV-cache append in its epilogue.

    ``hidden`` is the normalised hidden state ``[B, T, dim]`` (BF16, contiguous), ``w_qkv`` the
    layer's ``[3 * H * 64, dim]`` weight (the reference's ``Block.qkv``). Equivalent to
    ``rope_append(F.linear(hidden, w_qkv).view(B, T, 3, H, 64), ...)`` with the projection
    accumulated in FP32 inside the kernel and never written to memory (model.py:59-67); returns
    rope(q) as ``[B, H, T, 64]``.
    """
    return load_attention_extension().qkv_rope_append(hidden, w_qkv, cos, sin, position,
                                                      cache_k, cache_v)
