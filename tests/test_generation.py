"""End-to-end generation around the attention path: the decoder and KV cache restated from the
reference (tiny_transformer/model.py), eager and CUDA-graph decode, and the zero-copy hand-off
of cache prefix views to the kernels."""
import ctypes

import pytest
import torch

from tiny_transformer_b200.generation import (Decoder, DecoderConfig, GraphedDecode, KVCache,
                                              attention_operator, generate, request)

SMALL = DecoderConfig(vocab_size=512, dim=128, n_layers=2, n_heads=2, hidden_dim=256,
                      max_seq_len=256)


def _model(backend="reference", dtype=torch.float32, device="cpu", seed=3):
    torch.manual_seed(seed)
    return Decoder(SMALL, backend).to(device=device, dtype=dtype).eval()


def test_kv_cache_semantics():
    cache = KVCache(SMALL, batch_size=2, capacity=8)
    k = torch.randn(2, 2, 3, 64)
    v = torch.randn(2, 2, 3, 64)
    kp, vp = cache.update(0, k, v)
    assert kp.shape == (2, 2, 3, 64) and cache.length == 0  # length advances per model call
    assert kp.data_ptr() == cache.keys[0].data_ptr()  # a view of the storage, not a copy
    assert torch.equal(kp, k) and torch.equal(vp, v)
    cache.length = 3
    kp, _ = cache.update(0, k[:, :, :1], v[:, :, :1])
    assert kp.shape[2] == 4 and kp.stride() == (2 * 8 * 64, 8 * 64, 64, 1)
    with pytest.raises(ValueError, match="capacity"):
        cache.update(0, torch.randn(2, 2, 6, 64), torch.randn(2, 2, 6, 64))
    with pytest.raises(ValueError, match="batch"):
        cache.update(0, torch.randn(1, 2, 1, 64), torch.randn(1, 2, 1, 64))
    with pytest.raises(ValueError):
        KVCache(SMALL, batch_size=1, capacity=SMALL.max_seq_len + 1)
    assert cache.allocated_bytes() == 2 * 2 * 2 * 8 * 64 * 4


def test_unknown_backend_rejected():
    with pytest.raises(ValueError, match="Unsupported backend"):
        attention_operator("flash")


@torch.inference_mode()
def test_cached_decode_matches_full_forward_cpu():
    """Prefill + one-token steps through the cache give the logits of a full forward."""
    model = _model("reference")
    ids = torch.randint(0, SMALL.vocab_size, (2, 12), generator=torch.Generator().manual_seed(5))
    full = model(ids)
    cache = model.new_cache(2, 12)
    steps = [model(ids[:, :8], cache=cache)]
    for t in range(8, 12):
        steps.append(model(ids[:, t:t + 1], cache=cache))
    inc = torch.cat(steps, dim=1)
    assert cache.length == 12
    assert torch.allclose(inc, full, atol=1e-5, rtol=1e-4)
    # sdpa and the reference specification agree as well.
    model.set_attention("sdpa")
    assert torch.allclose(model(ids), full, atol=1e-5, rtol=1e-4)


@torch.inference_mode()
def test_generate_eager_cpu_is_greedy():
    model = _model("reference")
    prompt = torch.randint(0, SMALL.vocab_size, (2, 6), generator=torch.Generator().manual_seed(9))
    out = generate(model, prompt, 5)
    assert out.shape == (2, 5)
    seq = prompt
    for i in range(5):
        nxt = model(seq)[:, -1].argmax(-1, keepdim=True)
        assert torch.equal(nxt, out[:, i:i + 1])
        seq = torch.cat([seq, nxt], dim=1)


def test_cache_prefix_views_are_read_in_place():
    """The C ABI accepts a cache prefix view [B, H, :end, 64] of BF16 storage as it is, so the
    student path hands it to the kernels without the reference's aligned_contiguous copy."""
    from tiny_transformer_b200.operators._extension import load_c_abi
    lib = load_c_abi()
    cap, heads = 384, 12
    strides = (ctypes.c_int64 * 4)(heads * cap * 64, cap * 64, 64, 1)
    assert lib.tt_attn_layout_supported(ctypes.c_void_p(1 << 20), strides) == 1
    # q/k/v split out of the fused QKV projection: row stride 3 * dim elements.
    strides = (ctypes.c_int64 * 4)(40 * 3 * 768, 64, 3 * 768, 1)
    assert lib.tt_attn_layout_supported(ctypes.c_void_p((1 << 20) + 1536), strides) == 1


def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")


@pytest.mark.gpu
@torch.inference_mode()
def test_student_decoder_matches_reference_attention_gpu():
    _gpu()
    model = _model("student", torch.bfloat16, "cuda")
    ids = torch.randint(0, SMALL.vocab_size, (3, 40), device="cuda",
                        generator=torch.Generator("cuda").manual_seed(1))
    model.set_attention("reference")
    want = model(ids).float()
    model.set_attention("student")
    got = model(ids).float()
    assert (got - want).abs().max().item() < 3e-2
    # Incremental decode through the cache (prefix views) matches the full forward.
    cache = model.new_cache(3, 40)
    inc = [model(ids[:, :24], cache=cache)]
    for t in range(24, 40):
        inc.append(model(ids[:, t:t + 1], cache=cache))
    inc = torch.cat(inc, dim=1).float()
    assert (inc - want).abs().max().item() < 3e-2


@pytest.mark.gpu
@torch.inference_mode()
def test_graphed_decode_matches_eager_gpu():
    _gpu()
    model = _model("student", torch.bfloat16, "cuda")
    prompt = torch.randint(0, SMALL.vocab_size, (4, 20), device="cuda",
                           generator=torch.Generator("cuda").manual_seed(2))
    eager = generate(model, prompt, 12)
    graphed = generate(model, prompt, 12, graphed=True)
    assert graphed.shape == eager.shape == (4, 12)
    assert torch.equal(graphed, eager)
    r = request(model, prompt, 12, graphed=True)
    assert torch.equal(r["last_tokens"], eager)
    assert r["tpot_ms"] > 0 and r["ttft_ms"] > 0


@pytest.mark.gpu
@torch.inference_mode()
def test_graphed_decode_refuses_steps_beyond_capacity_gpu():
    _gpu()
    model = _model("student", torch.bfloat16, "cuda")
    prompt = torch.randint(0, SMALL.vocab_size, (2, 8), device="cuda")
    cache = model.new_cache(2, 8 + 4)
    first = model(prompt, cache=cache, last_only=True)[:, -1].argmax(-1, keepdim=True)
    g = GraphedDecode(model, cache, 4)
    g.prepare(first)
    g.capture()
    g.replay(3)
    with pytest.raises(ValueError, match="output buffer|capacity"):
        g.replay(8)
    torch.cuda.synchronize()
