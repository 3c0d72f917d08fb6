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
    q, k, v = [Mock(is_cuda=True, requires_grad=False, dtype=torch.bfloat16) for _ in range(3)]
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
            tensor.requires_grad = True
            load.reset_mock()
            with pytest.raises(NotImplementedError, match="backward"):
                student.attention(q, k, v)
            load.assert_not_called()
            with torch.no_grad():
                assert student.attention(q, k, v, 9) is output
            extension.attention_forward.assert_called_with(q, k, v, 9, None, None)
            tensor.requires_grad = False
        q.is_cuda = False
        with pytest.raises(RuntimeError, match="CUDA"):
            student.attention(q, k, v)


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
