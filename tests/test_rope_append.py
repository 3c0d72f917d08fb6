"""Fused RoPE + KV-cache append (tt_rope_append_bf16): argument validation through the C ABI on
CPU, and on the GPU bit-exactness against the reference's bf16 rope expression
(reference.py:30-34) followed by the cache write of KVCache.update (model.py:29-41)."""
import ctypes

import pytest
import torch

from tiny_transformer_b200.generation import Decoder, DecoderConfig, rope

OK, BAD_ARG = 0, 1


@pytest.fixture(scope="module")
def lib():
    from tiny_transformer_b200.operators._extension import load_c_abi
    return load_c_abi()


def _call(lib, *, qkv=256, B=2, T=3, H=2, cos=512, sin=768, L=16, pos=0, pos_dev=None,
          q_out=1024, ck=2048, cv=4096, cks=None, cvs=None, cap=8):
    i64 = ctypes.c_int64 * 4
    cks = cks or i64(H * cap * 64, cap * 64, 64, 1)
    cvs = cvs or i64(H * cap * 64, cap * 64, 64, 1)
    return lib.tt_rope_append_bf16(qkv, B, T, H, cos, sin, L, pos, pos_dev, q_out, ck, cks, cv,
                                   cvs, cap, None)


@pytest.mark.parametrize("kwargs,fragment", [
    (dict(qkv=None), "NULL"),
    (dict(B=0), "positive"),
    (dict(cap=0), "positive"),
    (dict(pos=6), "capacity"),          # 6 + 3 > 8
    (dict(pos=-1), "capacity"),
    (dict(L=4, pos=2), "capacity"),     # table shorter than position + T
    (dict(cks=(ctypes.c_int64 * 4)(2 * 8 * 64, 8 * 64, 64, 2)), "contiguous"),
    (dict(cvs=(ctypes.c_int64 * 4)(2 * 8 * 64, 8 * 64, 65, 1)), "even"),
    (dict(qkv=258), "aligned"),
    (dict(B=1 << 31), "grid"),
])
def test_rope_append_rejects_bad_arguments(lib, kwargs, fragment):
    assert _call(lib, **kwargs) == BAD_ARG
    assert fragment in lib.tt_attn_last_error().decode()


def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")


def _tables(n, d=64, theta=10000.0):
    freq = 1.0 / theta ** (torch.arange(0, d, 2).float() / d)
    ang = torch.arange(n).float()[:, None] * freq
    return ang.cos().contiguous(), ang.sin().contiguous()


def _expected(qkv, cos, sin, position):
    """q, k rotated with the reference expression, v as is; all [B, H, T, 64]."""
    T = qkv.shape[1]
    c = cos[position:position + T][None, None]
    s = sin[position:position + T][None, None]
    q, k, v = (t.transpose(1, 2) for t in qkv.unbind(dim=2))
    return rope(q, c, s), rope(k, c, s), v


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,position,cap", [(2, 37, 3, 5, 64), (4, 1, 12, 100, 101),
                                                (1, 128, 12, 0, 384), (3, 9, 5, 0, 9)])
def test_rope_append_bit_exact(B, T, H, position, cap):
    _gpu()
    from tiny_transformer_b200.operators import fused
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T)
    qkv = (torch.randn(B, T, 3, H, 64, device="cuda", generator=g) * 3).bfloat16()
    cos, sin = (t.cuda() for t in _tables(cap + 3))
    sentinel = torch.tensor(-7.0, dtype=torch.bfloat16)
    ck = torch.full((B, H, cap, 64), sentinel.item(), dtype=torch.bfloat16, device="cuda")
    cv = ck.clone()
    q_out = fused.rope_append(qkv, cos, sin, position, ck, cv)
    eq, ek, ev = _expected(qkv, cos, sin, position)
    assert q_out.shape == (B, H, T, 64) and q_out.is_contiguous()
    assert torch.equal(q_out, eq)
    assert torch.equal(ck[:, :, position:position + T], ek)
    assert torch.equal(cv[:, :, position:position + T], ev)
    rest = torch.ones(cap, dtype=torch.bool)
    rest[position:position + T] = False
    assert bool((ck[:, :, rest] == sentinel).all()) and bool((cv[:, :, rest] == sentinel).all())


@pytest.mark.gpu
def test_rope_append_device_position_and_range_flag():
    _gpu()
    from tiny_transformer_b200.operators import fused
    from tiny_transformer_b200.operators._extension import load_c_abi
    lib = load_c_abi()
    flags = ctypes.c_uint(0)
    lib.tt_attn_device_status(ctypes.byref(flags), 1)
    B, H, cap = 3, 4, 16
    qkv = torch.randn(B, 1, 3, H, 64, device="cuda").bfloat16()
    cos, sin = (t.cuda() for t in _tables(cap))
    ck = torch.zeros(B, H, cap, 64, dtype=torch.bfloat16, device="cuda")
    cv = torch.zeros_like(ck)
    pos = torch.tensor([7], dtype=torch.long, device="cuda")
    q_out = fused.rope_append(qkv, cos, sin, pos, ck, cv)
    eq, ek, ev = _expected(qkv, cos, sin, 7)
    assert torch.equal(q_out, eq) and torch.equal(ck[:, :, 7:8], ek) and torch.equal(cv[:, :, 7:8], ev)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 0) == OK
    # A device-held position past the cache: rows are skipped, bit 1 is set, nothing faults.
    before_k, before_v = ck.clone(), cv.clone()
    pos.fill_(cap)
    fused.rope_append(qkv, cos, sin, pos, ck, cv)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 1) == BAD_ARG
    assert flags.value & 2
    assert torch.equal(ck, before_k) and torch.equal(cv, before_v)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 0) == OK


@pytest.mark.gpu
@torch.inference_mode()
def test_fused_decoder_matches_unfused():
    _gpu()
    cfg = DecoderConfig(vocab_size=512, dim=192, n_layers=2, n_heads=3, hidden_dim=256,
                        max_seq_len=256)
    torch.manual_seed(4)
    model = Decoder(cfg, "student").to(device="cuda", dtype=torch.bfloat16).eval()
    assert model.rope_cos.dtype == torch.float32
    ids = torch.randint(0, cfg.vocab_size, (2, 30), device="cuda")
    model.fused_qkv = False  # the cuBLAS projection in both runs: bit-exact comparison
    outs = []
    for fused_flag in (False, True):
        model.fused_rope = fused_flag
        cache = model.new_cache(2, 30)
        steps = [model(ids[:, :20], cache=cache)]
        for t in range(20, 30):
            steps.append(model(ids[:, t:t + 1], cache=cache))
        outs.append(torch.cat(steps, dim=1))
    assert torch.equal(outs[0], outs[1])
