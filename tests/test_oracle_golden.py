"""Pin the CPU oracle against the reference's own outputs and known answers (no GPU).

tests/golden/attention_golden.npz holds outputs of Tiny-transformer's reference.attention
(reference.py:49-53) computed by tests/golden/make_golden.py; the known-answer tests restate
the analytic cases of tests/test_student_attention.py in the reference.
"""
import numpy as np
import pytest

from oracle import attention_oracle as oracle


def _inputs(case):
    return [oracle.bf16_bits_to_f32(case[x]) for x in ("q", "k", "v")]


def test_golden_cases_present(golden):
    kinds = {name.split("_")[0] for name in golden}
    assert {"prefill", "chunk", "decode", "kvlens", "large"} <= kinds
    assert len(golden) >= 20


def test_bf16_restatement_matches_reference_outputs(golden):
    """The numpy restatement reproduces reference.attention's BF16 output: every element within
    one bf16 ulp, and at least 99% bit-identical (accumulation order is the only difference)."""
    for name, case in golden.items():
        q, k, v = _inputs(case)
        past = int(case["past_len"])
        if "kv_lens" in case:
            out, _ = oracle.decode_with_kv_lens(q, k, v, case["kv_lens"], oracle.reference_bf16_with_lse)
            out = out.astype(np.float32)
        else:
            out = oracle.reference_attention_bf16(q, k, v, past)
        ref = oracle.bf16_bits_to_f32(case["o"])
        mine = oracle.f32_to_bf16_bits(out).astype(np.int32)
        theirs = case["o"].astype(np.int32)
        ulps = np.abs(mine - theirs)
        same = np.mean(mine == theirs)
        assert same >= 0.99, f"{name}: only {same:.4f} bit-identical"
        assert ulps.max() <= 1 or np.abs(out - ref).max() <= 1e-6, f"{name}: {ulps.max()} ulp"


def test_fp64_oracle_matches_reference_lse_and_output(golden):
    for name, case in golden.items():
        q, k, v = _inputs(case)
        past = int(case["past_len"])
        if "kv_lens" in case:
            out, lse = oracle.decode_with_kv_lens(q, k, v, case["kv_lens"])
        else:
            out, lse = oracle.attention_fp64(q, k, v, past)
        np.testing.assert_allclose(lse, case["lse64"], rtol=1e-12, atol=1e-12, err_msg=name)
        ref = oracle.bf16_bits_to_f32(case["o"])
        # Reference BF16 output vs exact FP64: within the reference tests' O tolerance.
        np.testing.assert_allclose(ref, out, atol=2e-2, rtol=3e-2, err_msg=name)


def test_known_answers():
    # Uniform attention returns V exactly (test_student_attention.py:244-257, 312-317).
    v = oracle.round_bf16(np.random.default_rng(0).normal(size=(1, 2, 9, 64)))
    z = np.zeros_like(v)
    out = oracle.reference_attention_bf16(z, z, v)
    # Row i averages v[0..i]; row 0 is v[0] exactly.
    np.testing.assert_array_equal(out[:, :, 0], v[:, :, 0])
    # LSE = 2 * key_value + ln(n) for q = 0.25, constant k (test_student_attention.py:349-368).
    for key_value in (-10.0, -0.5, 0.5, 10.0):
        tq, tk = 65, 193
        q = np.full((1, 1, tq, 64), 0.25, np.float32)
        k = np.full((1, 1, tk, 64), key_value, np.float32)
        ones = np.ones_like(k)
        out, lse = oracle.attention_fp64(q, k, ones, tk - tq)
        expected = 2 * key_value + np.log(np.arange(tk - tq + 1, tk + 1))
        np.testing.assert_allclose(lse[0, 0], expected, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(out, 1.0, atol=1e-12)
    # Decode with q = 0, v = 1 gives exactly 1 (test_student_attention.py:307-310).
    q = np.zeros((2, 3, 1, 64), np.float32)
    k = oracle.round_bf16(np.random.default_rng(1).normal(size=(2, 3, 257, 64)))
    out = oracle.reference_attention_bf16(q, k, np.ones_like(k), 256)
    np.testing.assert_array_equal(out, 1.0)


def test_causal_mask_semantics():
    allowed = oracle.causal_allowed(3, 7, 4)
    assert allowed.tolist() == [[j <= i + 4 for j in range(7)] for i in range(3)]
    assert oracle.visible_pairs(512, 512, 0) == 512 * 513 // 2
    assert oracle.prefill_flops(8, 12, 512, 512, 0) == 3_227_516_928  # 3.2275 GFLOP
    assert oracle.prefill_flops(4, 12, 4096, 4096, 0) == 4 * 4 * 12 * 64 * 4096 * 4097 // 2


def test_kv_lens_zero_and_clamp():
    rng = np.random.default_rng(3)
    q = oracle.round_bf16(rng.normal(size=(3, 1, 1, 64)))
    k = oracle.round_bf16(rng.normal(size=(3, 1, 10, 64)))
    v = oracle.round_bf16(rng.normal(size=(3, 1, 10, 64)))
    out, lse = oracle.decode_with_kv_lens(q, k, v, [0, 10, 99])
    assert (out[0] == 0).all() and np.isneginf(lse[0]).all()
    np.testing.assert_allclose(out[1], out[2] * 0 + oracle.attention_fp64(q[1:2], k[1:2], v[1:2], 9)[0][0])
    np.testing.assert_allclose(out[2], oracle.attention_fp64(q[2:3], k[2:3], v[2:3], 9)[0][0])


def test_planted_mistake_is_caught(golden):
    """A checker that cannot fail proves nothing: an oracle with an off-by-one causal mask
    (keys j < i + past_len) must disagree with the reference outputs."""
    case = golden["prefill_t65"]
    q, k, v = _inputs(case)
    tq = q.shape[2]
    allowed = oracle.causal_allowed(tq, tq, 0) & ~np.eye(tq, dtype=bool)
    allowed[0, 0] = True
    scores = np.matmul(q.astype(np.float64), np.swapaxes(k, -1, -2).astype(np.float64)) / 8
    scores = np.where(allowed, scores, -np.inf)
    e = np.exp(scores - scores.max(-1, keepdims=True))
    wrong = np.matmul(e / e.sum(-1, keepdims=True), v)
    ref = oracle.bf16_bits_to_f32(case["o"])
    assert np.abs(wrong - ref).max() > 2e-2


@pytest.mark.parametrize("x", [0.0, 1.0, -1.5, 3.0e38, 1e-40, np.inf, -np.inf])
def test_bf16_rounding(x):
    r = oracle.round_bf16(np.array([x], np.float32))[0]
    if np.isfinite(x) and abs(x) < 3.3e38:
        assert abs(r - x) <= max(abs(x) * 2 ** -8, 2.0 ** -133)  # subnormals: absolute
    else:
        assert r == x or np.isinf(r)


def test_oracle_backward_matches_fp64_autograd():
    """The FP64 backward restatement equals torch autograd of the FP64 forward, including a
    chunked-prefill (past_len > 0) case and rows whose keys are partly masked."""
    import torch
    from oracle import attention_oracle as oracle
    g = torch.Generator().manual_seed(21)
    for tq, tk in ((9, 9), (5, 12), (1, 7)):
        q, k, v, dout = (torch.randn(2, 3, t, 64, generator=g, dtype=torch.float64)
                         for t in (tq, tk, tk, tq))
        past = tk - tq
        qq, kk, vv = (x.clone().requires_grad_() for x in (q, k, v))
        mask = torch.arange(tk)[None, :] <= torch.arange(tq)[:, None] + past
        scores = (qq @ kk.transpose(-1, -2) / 8).masked_fill(~mask, float("-inf"))
        out = scores.softmax(-1) @ vv
        want = torch.autograd.grad(out, (qq, kk, vv), dout)
        got = oracle.attention_backward_fp64(q.numpy(), k.numpy(), v.numpy(), dout.numpy(), past)
        for a, b in zip(got, want):
            np.testing.assert_allclose(a, b.numpy(), rtol=1e-10, atol=1e-12)
