"""QKV projection with RoPE and the KV-cache append in its epilogue (tt_qkv_rope_append_bf16).

CPU: argument validation through the C ABI before any CUDA call. GPU (B200): against the
unfused steps of the reference's Block.forward (model.py:59-67) - the QKV projection computed
in FP32 by torch and rounded to bf16, then rope_append (itself bit-exact with the reference's
bf16 rope expression and KVCache.update) - and against today's cuBLAS projection + rope_append.
The fused projection is an FP32 sum in another order, so single elements may round to the
neighbouring bf16 value: the bar is one bf16 ulp of the projection for v, and for the rotated q
and k the error that one ulp in each input of the pair carries through the rotation (e*c - o*s
can cancel, so that bound is relative to |e| + |o|, not to the result), with at least 99 % of
the elements identical; cache rows outside the written positions must stay untouched, and the
decoder's greedy tokens must match the unfused path.
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

OK, BAD_ARG, UNSUPPORTED = 0, 1, 2


@pytest.fixture(scope="module")
def lib():
    from tiny_transformer_b200.operators._extension import load_c_abi
    return load_c_abi()


def _call(lib, *, h=256, B=2, T=3, dim=128, w=512, H=2, cos=768, sin=1024, L=16, pos=0,
          pos_dev=None, q_out=1280, ck=2048, cv=4096, cks=None, cvs=None, cap=8):
    i64 = ctypes.c_int64 * 4
    cks = cks or i64(H * cap * 64, cap * 64, 64, 1)
    cvs = cvs or i64(H * cap * 64, cap * 64, 64, 1)
    return lib.tt_qkv_rope_append_bf16(h, B, T, dim, w, H, cos, sin, L, pos, pos_dev, q_out, ck,
                                       cks, cv, cvs, cap, None)


@pytest.mark.parametrize("kwargs,status,fragment", [
    (dict(h=None), BAD_ARG, "NULL"),
    (dict(B=0), BAD_ARG, "positive"),
    (dict(dim=96), UNSUPPORTED, "multiple of 64"),
    (dict(pos=6), BAD_ARG, "capacity"),
    (dict(L=4, pos=2), BAD_ARG, "capacity"),
    (dict(cks=(ctypes.c_int64 * 4)(2 * 8 * 64, 8 * 64, 64, 2)), BAD_ARG, "contiguous"),
    (dict(cvs=(ctypes.c_int64 * 4)(2 * 8 * 64, 8 * 64, 68, 1)), BAD_ARG, "multiples of 8"),
    (dict(w=520), BAD_ARG, "aligned"),
])
def test_qkv_rope_rejects_bad_arguments(lib, kwargs, status, fragment):
    assert _call(lib, **kwargs) == status
    assert fragment in lib.tt_attn_last_error().decode()


def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")


def _tables(n, d=64, theta=10000.0):
    freq = 1.0 / theta ** (torch.arange(0, d, 2).float() / d)
    ang = torch.arange(n).float()[:, None] * freq
    return ang.cos().contiguous(), ang.sin().contiguous()


def _ulps(a, b):
    """Distance in bf16 units in the last place (same sign assumed for the bulk)."""
    ai = a.contiguous().view(torch.int16).int()
    bi = b.contiguous().view(torch.int16).int()
    return (ai - bi).abs()


def _close(got, want, ulps):
    d = _ulps(got, want)
    same = (d == 0).float().mean().item()
    assert same >= 0.99, f"only {same:.4f} identical"
    # Near zero the integer distance is meaningless; compare those by value.
    tiny = want.float().abs() < 1e-3
    assert int(d[~tiny].max()) <= ulps if (~tiny).any() else True
    assert (got.float() - want.float())[tiny].abs().max().item() < 1e-3 if tiny.any() else True


def _close_rotated(got, want, pre):
    """``got``/``want`` rotated by (e, o) -> (e*c - o*s, e*s + o*c) from projections that may
    differ by one bf16 ulp; ``pre`` is the unrotated projection in the same layout. One ulp of
    e and o (<= 2^-8 of their magnitude), carried through the products and their bf16
    roundings, moves a result by at most about 2^-7 * (|e| + |o|) plus its own rounding."""
    same = (_ulps(got, want) == 0).float().mean().item()
    assert same >= 0.99, f"only {same:.4f} identical"
    mag = pre.float().abs().unflatten(-1, (32, 2)).sum(-1).repeat_interleave(2, dim=-1)
    bound = mag * 2.0 ** -7 + want.float().abs() * 2.0 ** -7 + 1e-6
    err = (got.float() - want.float()).abs()
    worst = (err / bound).max().item()
    assert worst <= 1.0, f"error {worst:.3f} x the two-ulp bound"


# Kernels and tiles the host picks on 148 SMs. One row tile (B * T <= 128), split-K clusters:
# (2, 37, 2, 128) 16-feature tiles x 2 parts, (32, 1, 12, 768) 64 x 3, (2, 50, 3, 192) 16 x 3,
# (3, 5, 2, 64) a single K slice (a cluster of one); the identity-rotation test below, 16 x 2. More rows, persistent: 128-feature tiles
# for (1, 129, 4, 256), (3, 200, 12, 768), (4, 100, 6, 384), (4, 256, 12, 768); 64-feature
# tiles for the odd head count of (5, 220, 5, 128).
@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,dim,position,cap", [
    (2, 37, 2, 128, 5, 64), (32, 1, 12, 768, 100, 384), (2, 50, 3, 192, 1, 64),
    (3, 5, 2, 64, 2, 16), (1, 129, 4, 256, 3, 140), (3, 200, 12, 768, 0, 256),
    (4, 100, 6, 384, 7, 128), (4, 256, 12, 768, 0, 256), (5, 220, 5, 128, 0, 256)])
@torch.no_grad()
def test_qkv_rope_matches_unfused(B, T, H, dim, position, cap):
    _gpu()
    from tiny_transformer_b200.operators import fused
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(B * 100 + T)
    hidden = torch.randn(B, T, dim, device="cuda", generator=g).bfloat16()
    w = (torch.randn(3 * H * 64, dim, device="cuda", generator=g) * 0.05).bfloat16()
    cos, sin = (t.cuda() for t in _tables(cap + 2))
    sentinel = -7.0
    caches = [torch.full((B, H, cap, 64), sentinel, dtype=torch.bfloat16, device="cuda")
              for _ in range(4)]
    q = fused.qkv_rope_append(hidden, w, cos, sin, position, caches[0], caches[1])
    # Unfused, with the projection accumulated in FP32 by torch.
    qkv32 = (hidden.float() @ w.float().t()).bfloat16().view(B, T, 3, H, 64).contiguous()
    q_ref = fused.rope_append(qkv32, cos, sin, position, caches[2], caches[3])
    assert q.shape == (B, H, T, 64) and q.is_contiguous()
    pre_q, pre_k = qkv32[:, :, 0].transpose(1, 2), qkv32[:, :, 1].transpose(1, 2)
    _close_rotated(q, q_ref, pre_q)
    sl = slice(position, position + T)
    _close_rotated(caches[0][:, :, sl], caches[2][:, :, sl], pre_k)
    _close(caches[1][:, :, sl], caches[3][:, :, sl], 1)
    rest = torch.ones(cap, dtype=torch.bool)
    rest[sl] = False
    assert bool((caches[0][:, :, rest] == sentinel).all()) and bool((caches[1][:, :, rest] == sentinel).all())
    # Today's path: cuBLAS projection (bf16 out) + rope_append.
    qkv_cublas = F.linear(hidden, w).view(B, T, 3, H, 64).contiguous()
    ck, cv = (torch.full_like(caches[0], sentinel) for _ in range(2))
    q_today = fused.rope_append(qkv_cublas, cos, sin, position, ck, cv)
    _close_rotated(q, q_today, pre_q)
    _close_rotated(caches[0][:, :, sl], ck[:, :, sl], pre_k)
    _close(caches[1][:, :, sl], cv[:, :, sl], 1)


@pytest.mark.gpu
@torch.no_grad()
def test_qkv_rope_device_position_and_identity_rotation():
    """With cos = 1 and sin = 0 the rotation is the identity (bf16(e * 1) - bf16(o * 0) = e), so
    q is the projection itself: within one ulp of the FP32 product. The position is read on the
    device; one past the cache skips the rows and flags TT_ERR_RANGE."""
    _gpu()
    from tiny_transformer_b200.operators import fused
    from tiny_transformer_b200.operators._extension import load_c_abi
    lib = load_c_abi()
    flags = ctypes.c_uint(0)
    lib.tt_attn_device_status(ctypes.byref(flags), 1)
    B, H, dim, cap = 8, 4, 512, 16
    hidden = torch.randn(B, 1, dim, device="cuda").bfloat16()
    w = (torch.randn(3 * H * 64, dim, device="cuda") * 0.05).bfloat16()
    cos = torch.ones(cap, 32, device="cuda")
    sin = torch.zeros(cap, 32, device="cuda")
    ck = torch.zeros(B, H, cap, 64, dtype=torch.bfloat16, device="cuda")
    cv = torch.zeros_like(ck)
    pos = torch.tensor([9], dtype=torch.long, device="cuda")
    q = fused.qkv_rope_append(hidden, w, cos, sin, pos, ck, cv)
    proj = (hidden.float() @ w.float().t()).bfloat16().view(B, 1, 3, H, 64)
    _close(q, proj[:, :, 0].transpose(1, 2), 1)
    _close(ck[:, :, 9:10], proj[:, :, 1].transpose(1, 2), 1)
    _close(cv[:, :, 9:10], proj[:, :, 2].transpose(1, 2), 1)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 0) == OK
    before = ck.clone()
    pos.fill_(cap)
    fused.qkv_rope_append(hidden, w, cos, sin, pos, ck, cv)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 1) == BAD_ARG and flags.value & 2
    assert torch.equal(ck, before)


@pytest.mark.gpu
@torch.inference_mode()
def test_decoder_with_fused_projection_matches_unfused():
    """The model_60m-shaped decoder (reduced depth) greedy-decodes the same tokens with the
    projection fused into the RoPE/append kernel as with cuBLAS + rope_append, eager and
    graphed; the logits agree to bf16 rounding."""
    _gpu()
    from tiny_transformer_b200.generation import Decoder, DecoderConfig, generate
    cfg = DecoderConfig(n_layers=2, max_seq_len=256)
    torch.manual_seed(11)
    model = Decoder(cfg, "student").to(device="cuda", dtype=torch.bfloat16).eval()
    assert model.fused_qkv
    prompt = torch.randint(0, cfg.vocab_size, (4, 32), device="cuda",
                           generator=torch.Generator("cuda").manual_seed(5))
    runs = {}
    for flag in (False, True):
        model.fused_qkv = flag
        cache = model.new_cache(4, 48)
        runs[flag] = (model(prompt, cache=cache).float(), generate(model, prompt, 16),
                      generate(model, prompt, 16, graphed=True))
    assert (runs[True][0] - runs[False][0]).abs().max().item() < 5e-2
    agree = (runs[True][1] == runs[False][1]).float().mean().item()
    assert agree >= 0.9, agree
    assert torch.equal(runs[True][1], runs[True][2])  # graphed == eager with the fused kernel
