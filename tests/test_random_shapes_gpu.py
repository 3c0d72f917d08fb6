"""Seeded random-shape sweep on the GPU: prefill, chunked prefill and decode forward against the
FP64 oracle at the reference tests' tolerances (O atol 2e-2 / rtol 3e-2, LSE atol 2e-4 /
rtol 2e-5), and the backward against FP64 gradients (atol 1e-2 / rtol 3e-2). Shapes are drawn to
hit tile tails (multiples of 128 +- small offsets), past_len offsets and odd batch x head counts.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")


def _shapes(seed, n):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        b, h = int(rng.integers(1, 4)), int(rng.integers(1, 6))
        tq = int(rng.choice([1, 2, 63, 127, 128, 129, 255, 256, 257, 384, 511, 700]))
        past = int(rng.choice([0, 0, 1, 64, 127, 200])) if tq > 1 else int(rng.integers(0, 900))
        out.append((b, h, tq, tq + past, past))
    return out


@pytest.mark.parametrize("shape", _shapes(2027, 24))
def test_forward_random_shapes_match_fp64(shape):
    _gpu()
    from oracle import attention_oracle as oracle
    from tiny_transformer_b200.operators import student
    b, h, tq, tk, past = shape
    g = torch.Generator().manual_seed(b * 100000 + h * 10000 + tq * 10 + past)
    q = torch.randn(b, h, tq, 64, generator=g).bfloat16()
    k = torch.randn(b, h, tk, 64, generator=g).bfloat16()
    v = torch.randn(b, h, tk, 64, generator=g).bfloat16()
    with torch.no_grad():
        o, lse = student.attention_with_lse(q.cuda(), k.cuda(), v.cuda(), past)
    ro, rlse = oracle.attention_fp64(q.float().numpy(), k.float().numpy(), v.float().numpy(), past)
    torch.testing.assert_close(o.double().cpu(), torch.from_numpy(ro), atol=2e-2, rtol=3e-2)
    torch.testing.assert_close(lse.double().cpu(), torch.from_numpy(rlse), atol=2e-4, rtol=2e-5)


@pytest.mark.parametrize("shape", [s for s in _shapes(2028, 16) if s[2] > 1][:10])
def test_backward_random_shapes_match_fp64(shape):
    _gpu()
    from oracle import attention_oracle as oracle
    from tiny_transformer_b200.operators import student
    b, h, tq, tk, past = shape
    g = torch.Generator().manual_seed(b * 7 + h * 131 + tq * 17 + past)
    q, k, v = (torch.randn(b, h, t, 64, generator=g).bfloat16() for t in (tq, tk, tk))
    dout = (torch.randn(b, h, tq, 64, generator=g) * 0.25).bfloat16()
    qg, kg, vg = (x.cuda().requires_grad_() for x in (q, k, v))
    o = student.attention(qg, kg, vg, past)
    grads = torch.autograd.grad(o, (qg, kg, vg), dout.cuda())
    want = oracle.attention_backward_fp64(*(x.float().numpy() for x in (q, k, v, dout)), past)
    for got, ref in zip(grads, want):
        torch.testing.assert_close(got.double().cpu(), torch.from_numpy(ref), atol=1e-2, rtol=3e-2)
