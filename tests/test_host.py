"""Host-side wiring of the student operator and the native extension, without a GPU.

Mirrors StudentAttentionHostTests (Tiny-transformer tests/test_student_attention.py:12-87): the
extension is replaced by a test double to check argument forwarding and guards.
"""
from unittest.mock import Mock, patch

import pytest
import torch


def test_extension_loads_and_exposes_operator():
    from tiny_transformer_b200.operators._extension import load_attention_extension
    ext = load_attention_extension()
    assert hasattr(ext, "attention_forward")
    assert ext.HEAD_DIM == 64 and ext.ABI_VERSION == 1


def test_native_rejects_cpu_tensors_before_any_cuda_call():
    from tiny_transformer_b200.operators._extension import load_attention_extension
    ext = load_attention_extension()
    x = torch.zeros(1, 1, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.attention_forward(x, x, x)


def test_student_forwards_arguments_and_guards():
    from tiny_transformer_b200.operators import student
    q, k, v = [Mock(is_cuda=True, requires_grad=False, dtype=torch.float32) for _ in range(3)]
    output, lse, segments, lens = object(), object(), object(), object()
    extension = Mock()
    extension.attention_forward.return_value = (output, lse)
    with patch.object(student, "load_attention_extension", return_value=extension) as load:
        assert student.attention(q, k, v, 0, segments) is output
        extension.attention_forward.assert_called_once_with(q, k, v, 0, segments, None)
        assert student.attention(q, k, v, 5, None, lens) is output
        extension.attention_forward.assert_called_with(q, k, v, 5, None, lens)
        assert student.attention_with_lse(q, k, v, 7) == (output, lse)
        for tensor in (q, k, v):
            # FP32 inputs that need grad: no backward (reference student.py:223-226).
            tensor.requires_grad = True
            load.reset_mock()
            with pytest.raises(NotImplementedError, match="backward"):
                student.attention(q, k, v)
            with pytest.raises(NotImplementedError, match="backward"):
                student.attention_with_lse(q, k, v)
            load.assert_not_called()
            with torch.no_grad():
                assert student.attention(q, k, v, 9) is output
            extension.attention_forward.assert_called_with(q, k, v, 9, None, None)
            tensor.requires_grad = False
        # The BF16 training path reaches the autograd bridge (reference student.py:227-228).
        for tensor in (q, k, v):
            tensor.dtype = torch.bfloat16
        q.requires_grad = True
        with patch.object(student._Attention, "apply", return_value=output) as apply:
            assert student.attention(q, k, v, 2) is output
            apply.assert_called_once_with(q, k, v, 2, None)
            with pytest.raises(NotImplementedError, match="kv_lens"):
                student.attention(q, k, v, 2, None, lens)
        q.requires_grad = False
        q.is_cuda = False
        with pytest.raises(RuntimeError, match="CUDA"):
            student.attention(q, k, v)


def test_autograd_bridge_saved_state_and_gradients_with_cpu_double():
    """The real _Attention autograd function, with the native module replaced by FP64 CPU
    doubles (as in the reference's host test): saved O / LSE reach the native backward, past_len
    is carried, gradients map back through strided views and match autograd of the reference
    expression."""
    from tiny_transformer_b200.generation import reference_attention
    from tiny_transformer_b200.operators import student

    def forward(q, k, v, past_len, segments):
        assert not torch.is_grad_enabled() and segments is None
        mask = torch.arange(k.size(2))[None, :] <= torch.arange(q.size(2))[:, None] + past_len
        scores = (q @ k.transpose(-1, -2) / 8).masked_fill(~mask, -torch.inf)
        return scores.softmax(-1) @ v, scores.logsumexp(-1)

    def backward(q, k, v, dout, out, lse, past_len, segments):
        assert segments is None
        mask = torch.arange(k.size(2))[None, :] <= torch.arange(q.size(2))[:, None] + past_len
        p = torch.exp(q @ k.transpose(-1, -2) / 8 - lse[..., None]).masked_fill(~mask, 0)
        ds = p * (dout @ v.transpose(-1, -2) - (dout * out).sum(-1, keepdim=True))
        return ds @ k / 8, ds.transpose(-1, -2) @ q / 8, p.transpose(-1, -2) @ dout

    extension = Mock(attention_forward=Mock(side_effect=forward),
                     attention_backward=Mock(side_effect=backward))
    torch.manual_seed(42)
    bases = [torch.randn(2, 2, t, 128, dtype=torch.float64, requires_grad=True) for t in (5, 7, 7)]
    expected_bases = [x.detach().clone().requires_grad_() for x in bases]
    with patch.object(student, "load_attention_extension", return_value=extension):
        actual, expected = [], []
        for tk in (7, 6):
            q, k, v = (x[..., ::2] for x in bases)
            rq, rk, rv = (x[..., ::2] for x in expected_bases)
            actual.append(student._Attention.apply(q, k[:, :, :tk], v[:, :, :tk], tk - 5, None))
            expected.append(reference_attention(rq, rk[:, :, :tk], rv[:, :, :tk], tk - 5))
        saved = [value.grad_fn.saved_tensors for value in actual]
        assert saved[0][4].data_ptr() != saved[1][4].data_ptr()
        for index in (1, 0):
            if index:
                actual[index].sum().backward()
                expected[index].sum().backward()
            else:
                upstream = torch.randn(2, 2, 5, 128, dtype=torch.float64)[..., ::2]
                actual[index].backward(upstream)
                expected[index].backward(upstream)
            args = extension.attention_backward.call_args.args
            assert args[4].data_ptr() == saved[index][3].data_ptr()
            assert args[5] is saved[index][4]
            assert args[6] == (2, 1)[index]
        for x, expected_x in zip(bases, expected_bases):
            torch.testing.assert_close(x.grad, expected_x.grad)
        assert extension.attention_forward.call_count == 2


def test_student_rejects_autocast():
    from tiny_transformer_b200.operators import student
    q = Mock(is_cuda=True, requires_grad=False, dtype=torch.bfloat16)
    with patch.object(torch, "is_autocast_enabled", return_value=True):
        with pytest.raises(RuntimeError, match="autocast"):
            student.attention(q, q, q)


def test_missing_build_fails_loudly(tmp_path, monkeypatch):
    from tiny_transformer_b200.operators import _extension
    monkeypatch.setattr(_extension, "BUILD_DIR", str(tmp_path))
    monkeypatch.setattr(_extension, "LIB_PATH", str(tmp_path / "libtt_attention.so"))
    _extension.load_c_abi.cache_clear()
    _extension.load_attention_extension.cache_clear()
    try:
        with pytest.raises(_extension.ExtensionMissingError, match="no non-CUDA fallback"):
            _extension.load_c_abi()
        with pytest.raises(_extension.ExtensionMissingError):
            _extension.load_attention_extension()
    finally:
        _extension.load_c_abi.cache_clear()
        _extension.load_attention_extension.cache_clear()
