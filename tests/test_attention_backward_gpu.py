"""BF16 attention backward on the GPU: the reference's backward test catalogue
(Tiny-transformer tests/test_student_attention.py:449-607) ported to this package, through
``student.attention`` (autograd) and the native ``attention_backward`` (C ABI underneath).

Gradients are compared with FP64 autograd of the reference expression at the reference's
tolerances (atol 1e-2, rtol 3e-2); shapes are widened around this kernel's 128-row / 128-key
tiles.
"""
import pytest
import torch

from tiny_transformer_b200.generation import reference_attention

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")
    from tiny_transformer_b200.operators._extension import load_attention_extension
    return load_attention_extension()


def check_bf16_backward(inputs, upstream=None):
    from tiny_transformer_b200.operators import student
    q, k, v = [x.detach().requires_grad_() for x in inputs]
    past_len = k.size(2) - q.size(2)
    originals = [x.detach().clone() for x in (q, k, v)]
    actual = student.attention(q, k, v, past_len)
    saved = actual.grad_fn.saved_tensors
    assert saved[4].dtype == torch.float32
    expected_inputs = [x.detach().double().requires_grad_() for x in (q, k, v)]
    expected = reference_attention(*expected_inputs, past_len=past_len)
    if upstream is None:
        upstream = (torch.randn(*q.shape[:-1], 128, device="cuda") * 0.25).bfloat16()[..., ::2]
    actual_grads = torch.autograd.grad(actual, (q, k, v), upstream)
    expected_grads = torch.autograd.grad(expected, expected_inputs, upstream.double())
    torch.testing.assert_close(actual.double(), expected, atol=2e-2, rtol=3e-2)
    for gradient, expected_gradient, original in zip(actual_grads, expected_grads, originals):
        assert gradient.shape == original.shape
        assert gradient.dtype == torch.bfloat16
        assert gradient.is_contiguous()
        assert torch.isfinite(gradient).all().item()
        torch.testing.assert_close(gradient.double(), expected_gradient, atol=1e-2, rtol=3e-2)
    for x, original in zip((q, k, v), originals):
        torch.testing.assert_close(x, original, atol=0, rtol=0)
    return actual_grads


@pytest.mark.parametrize("tq,tk", [(1, 1), (63, 63), (64, 64), (65, 65), (128, 128), (129, 129),
                                   (1, 257), (17, 64), (64, 129), (65, 193), (257, 321),
                                   (255, 255), (300, 700), (640, 640)])
def test_bf16_backward_tiles_tails_and_cached_queries(ext, tq, tk):
    torch.manual_seed(tq * 1000 + tk)
    inputs = [torch.randn(2, 3, t, 64, device="cuda", dtype=torch.bfloat16) for t in (tq, tk, tk)]
    check_bf16_backward(inputs)


@pytest.mark.parametrize("layout", ["unaligned", "feature_stride", "cache_prefix", "expanded"])
def test_bf16_backward_strides_offsets_and_expanded_upstream(ext, layout):
    torch.manual_seed(3)
    if layout == "unaligned":
        inputs = [torch.randn(2 * 3 * t * 64 + 1, device="cuda", dtype=torch.bfloat16)[1:]
                  .view(2, 3, t, 64) for t in (65, 129, 129)]
    elif layout == "feature_stride":
        inputs = [torch.randn(2, 3, t, 128, device="cuda", dtype=torch.bfloat16)[..., ::2]
                  for t in (65, 129, 129)]
    elif layout == "cache_prefix":
        inputs = [torch.randn(2, 3, t + 64, 64, device="cuda", dtype=torch.bfloat16)[:, :, :t]
                  for t in (65, 129, 129)]
    else:
        inputs = [torch.randn(1, 1, t, 64, device="cuda", dtype=torch.bfloat16).expand(2, 3, -1, -1)
                  for t in (65, 129, 129)]
    # Like backward of sum(): broadcast gradient with zero strides.
    upstream = torch.full((), 0.125, device="cuda", dtype=torch.bfloat16).expand_as(inputs[0])
    check_bf16_backward(inputs, upstream=upstream)


def test_bf16_backward_shared_qkv_base_and_partial_requires_grad(ext):
    from tiny_transformer_b200.operators import student
    torch.manual_seed(4)
    base = torch.randn(2, 65, 3, 2, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    expected_base = base.detach().double().requires_grad_()
    inputs = [x.transpose(1, 2) for x in base.unbind(2)]
    expected_inputs = [x.transpose(1, 2) for x in expected_base.unbind(2)]
    actual = student.attention(*inputs)
    expected = reference_attention(*expected_inputs)
    upstream = (torch.randn_like(actual.float()) * 0.25).bfloat16()
    actual.backward(upstream)
    expected.backward(upstream.double())
    torch.testing.assert_close(base.grad.double(), expected_base.grad, atol=1e-2, rtol=3e-2)
    for index in range(3):
        leaves = [x.detach().requires_grad_(i == index) for i, x in enumerate(inputs)]
        student.attention(*leaves).backward(torch.zeros_like(upstream))
        for i, x in enumerate(leaves):
            if i == index:
                assert torch.count_nonzero(x.grad).item() == 0
            else:
                assert x.grad is None


def test_bf16_backward_on_current_stream(ext):
    torch.manual_seed(5)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        torch.cuda._sleep(10_000_000)
        inputs = [torch.randn(2 * 3 * t * 64 + 1, device="cuda", dtype=torch.bfloat16)[1:]
                  .view(2, 3, t, 64) for t in (129, 193, 193)]
        upstream = torch.zeros_like(inputs[0])
        upstream[:, :, 64:].normal_(std=0.25)
        check_bf16_backward(inputs, upstream=upstream)
    stream.synchronize()


@torch.no_grad()
def test_bf16_native_backward_strided_saved_state(ext):
    torch.manual_seed(6)
    q, k, v = [torch.randn(2, 3, t, 64, device="cuda", dtype=torch.bfloat16) for t in (65, 129, 129)]
    out, lse = ext.attention_forward(q, k, v, 64)
    dout = torch.randn(out.numel() + 1, device="cuda", dtype=torch.bfloat16)[1:].view_as(out)
    saved_out = torch.empty(*out.shape[:-1], 128, device="cuda", dtype=out.dtype)[..., ::2]
    saved_out.copy_(out)
    saved_lse = torch.empty(2, 3, 130, device="cuda")[:, :, ::2]
    saved_lse.copy_(lse)
    actual = ext.attention_backward(q, k, v, dout, saved_out, saved_lse, 64)
    expected = ext.attention_backward(q, k, v, dout.contiguous(), out, lse, 64)
    for left, right in zip(actual, expected):
        torch.testing.assert_close(left, right, atol=0, rtol=0)


class deterministic_algorithms:
    """torch.use_deterministic_algorithms(True) for a block, restoring the previous mode."""

    def __enter__(self):
        self.mode = (torch.are_deterministic_algorithms_enabled(),
                     torch.is_deterministic_algorithms_warn_only_enabled())
        torch.use_deterministic_algorithms(True)

    def __exit__(self, *exc):
        torch.use_deterministic_algorithms(self.mode[0], warn_only=self.mode[1])


@torch.no_grad()
def test_bf16_native_backward_is_deterministic_and_leaves_inputs(ext):
    """Deterministic mode (like the reference's atomic-free kernels): bit-identical repeats. The
    default path adds dQ contributions in timing-dependent order: dK and dV (each key tile's
    from one CTA, in a fixed order) still repeat exactly, dQ within one bf16 ulp."""
    torch.manual_seed(7)
    q, k, v = [torch.randn(3, 4, t, 64, device="cuda", dtype=torch.bfloat16) for t in (300, 300, 300)]
    out, lse = ext.attention_forward(q, k, v)
    dout = torch.randn_like(out)
    before = [x.clone() for x in (q, k, v, dout, out, lse)]
    with deterministic_algorithms():
        first = ext.attention_backward(q, k, v, dout, out, lse)
        second = ext.attention_backward(q, k, v, dout, out, lse)
    for left, right in zip(first, second):
        assert torch.equal(left, right)
    fused = [ext.attention_backward(q, k, v, dout, out, lse) for _ in range(2)]
    assert torch.equal(fused[0][1], fused[1][1]) and torch.equal(fused[0][2], fused[1][2])
    torch.testing.assert_close(fused[0][0], fused[1][0], atol=0, rtol=2 ** -7)
    for a, b in zip(fused[0], first):  # the two paths agree to bf16 rounding of the same sums
        torch.testing.assert_close(a.float(), b.float(), atol=2e-3, rtol=2 ** -7)
    for x, y in zip((q, k, v, dout, out, lse), before):
        assert torch.equal(x, y)


@pytest.mark.parametrize("tq,tk", [(1, 1), (65, 65), (129, 129), (17, 64), (65, 193), (300, 700)])
def test_bf16_backward_deterministic_mode_matches_fp64(ext, tq, tk):
    """student.attention's backward under torch.use_deterministic_algorithms(True) (the FP64
    reference is computed outside that mode: its cuBLAS calls would need a workspace config)."""
    from tiny_transformer_b200.operators import student
    torch.manual_seed(tq * 31 + tk)
    q, k, v = [torch.randn(2, 3, t, 64, device="cuda", dtype=torch.bfloat16).requires_grad_()
               for t in (tq, tk, tk)]
    upstream = (torch.randn(2, 3, tq, 64, device="cuda") * 0.25).bfloat16()
    with deterministic_algorithms():
        actual = student.attention(q, k, v, tk - tq)
        grads = torch.autograd.grad(actual, (q, k, v), upstream)
    expected_inputs = [x.detach().double().requires_grad_() for x in (q, k, v)]
    expected = reference_attention(*expected_inputs, past_len=tk - tq)
    expected_grads = torch.autograd.grad(expected, expected_inputs, upstream.double())
    for gradient, expected_gradient in zip(grads, expected_grads):
        torch.testing.assert_close(gradient.double(), expected_gradient, atol=1e-2, rtol=3e-2)


@torch.no_grad()
def test_bf16_native_backward_validation(ext):
    q, k, v = [torch.randn(2, 3, 7, 64, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    out, lse = ext.attention_forward(q, k, v)
    dout = torch.randn_like(out)
    valid = [q, k, v, dout, out, lse]
    cases = [
        (0, q.cpu(), "CUDA"),
        (2, v[:, :, :6], "sequence length"),
        (3, dout.cpu(), "same device"),
        (4, out.cpu(), "same device"),
        (5, lse.cpu(), "same device"),
        (3, dout.float(), "same dtype"),
        (4, out.float(), "same dtype"),
        (3, dout[:, :, :6], "same shape"),
        (4, out[..., :32], "same shape"),
        (5, lse.bfloat16(), "float32"),
        (5, lse[..., None], "shape"),
        (5, lse[:, :, :6], "shape"),
        (3, dout.to_sparse(), "strided"),
    ]
    for index, replacement, message in cases:
        args = valid.copy()
        args[index] = replacement
        with pytest.raises(RuntimeError, match=message):
            ext.attention_backward(*args)
    ids = torch.zeros(2, 7, device="cuda", dtype=torch.long)
    with pytest.raises(RuntimeError, match="segment_ids is not supported"):
        ext.attention_backward(*valid, 0, ids)
    with pytest.raises(RuntimeError, match="only bf16"):
        ext.attention_backward(q.float(), k.float(), v.float(), dout.float(), out.float(), lse)
    for past_len in (-1, 1):
        with pytest.raises(RuntimeError, match="past_len"):
            ext.attention_backward(*valid, past_len)
    # Validate before copying enormous zero-stride views or allocating outputs. The flattened
    # grid is B * H * tiles (int32), so the grid case needs B * H above 2^31.
    seed = q[:1, :1, :1]
    for shape, message in (((1, 1, 2**31, 64), "int32"),
                           ((65536, 65536, 1, 64), "grid limits")):
        big = seed.expand(shape)
        big_lse = lse[:1, :1, :1].expand(shape[:3])
        with pytest.raises(RuntimeError, match=message):
            ext.attention_backward(big, big, big, big, big, big_lse)


@torch.no_grad()
def test_bf16_native_calls_from_a_fresh_thread(ext):
    """A thread that has made no CUDA runtime call (like autograd's worker) has no current
    context; the entry points must bind one before encoding their tensor maps."""
    import threading
    torch.manual_seed(8)
    q, k, v = [torch.randn(2, 3, t, 64, device="cuda", dtype=torch.bfloat16) for t in (192, 192, 192)]
    out, lse = ext.attention_forward(q, k, v)
    dout = torch.randn_like(out)
    expected = ext.attention_backward(q, k, v, dout, out, lse)
    result = {}

    def run():
        try:
            result["forward"] = ext.attention_forward(q, k, v)
            result["backward"] = ext.attention_backward(q, k, v, dout, out, lse)
            torch.cuda.current_stream().synchronize()
        except Exception as exc:  # re-raised on the main thread
            result["error"] = exc

    worker = threading.Thread(target=run)
    worker.start()
    worker.join()
    if "error" in result:
        raise result["error"]
    for left, right in zip(result["forward"], (out, lse)):
        assert torch.equal(left, right)
    for left, right in zip(result["backward"], expected):
        assert torch.equal(left, right)
