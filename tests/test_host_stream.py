"""attention_from_host: causal attention of pinned host tensors with the copies overlapped with
the kernels. Every (batch, head) row runs the same kernel as one call over device copies of the
whole batch, so its O and LSE must match that call bit for bit, whatever the slicing."""
import pytest
import torch

import __graft_entry__

__graft_entry__.import_package()

from tiny_transformer_b200.operators import student  # noqa: E402
from tiny_transformer_b200.operators.host_stream import attention_from_host  # noqa: E402


def test_rejects_unpinned_and_device_inputs():
    x = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="pinned"):
        attention_from_host(x, x, x)


def test_rejects_bad_arguments_before_any_copy():
    # Checked before the pinned-memory check, i.e. before anything is allocated or queued.
    q = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 10, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="Tk == past_len"):
        attention_from_host(q, k, k, 0)
    with pytest.raises(RuntimeError, match="non-negative"):
        attention_from_host(q, q, q, -1)
    w = torch.zeros(1, 2, 8, 32, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="head_dim=64"):
        attention_from_host(w, w, w, 0)


gpu = pytest.mark.gpu


def _host(*shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(torch.bfloat16).pin_memory()


def _reference(q, k, v, past_len):
    with torch.no_grad():
        o, lse = student.attention_with_lse(q.cuda(), k.cuda(), v.cuda(), past_len)
    return o.cpu(), lse.cpu()


@gpu
@pytest.mark.parametrize("B,H,Tq,Tk,slices", [
    (2, 3, 300, 300, 4),      # ragged tiles, slices of uneven row counts
    (2, 3, 200, 456, 5),      # chunked prefill (past_len = 256)
    (4, 12, 1, 2000, 3),      # single-token decode
    (1, 2, 130, 130, 8),      # more slices than rows
])
def test_matches_device_call_bitwise(B, H, Tq, Tk, slices):
    q = _host(B, H, Tq, 64, seed=1)
    k = _host(B, H, Tk, 64, seed=2)
    v = _host(B, H, Tk, 64, seed=3)
    past = Tk - Tq
    out, lse = attention_from_host(q, k, v, past, slices=slices)
    torch.cuda.current_stream().synchronize()
    ro, rl = _reference(q, k, v, past)
    assert out.is_pinned() and lse.is_pinned()
    assert torch.equal(out, ro)
    assert torch.equal(lse, rl)


@gpu
def test_fills_given_buffers_twice_in_a_row():
    B, H, T = 2, 4, 512
    q, k, v = (_host(B, H, T, 64, seed=s) for s in (4, 5, 6))
    out = torch.full((B, H, T, 64), float("nan"), dtype=torch.bfloat16).pin_memory()
    lse = torch.full((B, H, T), float("nan"), dtype=torch.float32).pin_memory()
    ro, rl = _reference(q, k, v, 0)
    for _ in range(2):
        o2, l2 = attention_from_host(q, k, v, 0, out=out, lse=lse)
        torch.cuda.current_stream().synchronize()
        assert o2 is out and l2 is lse
        assert torch.equal(out, ro) and torch.equal(lse, rl)


@gpu
def test_rejects_device_tensors_and_bad_buffers():
    x = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="host tensor"):
        attention_from_host(x, x, x)
    h = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16).pin_memory()
    bad = torch.zeros(1, 2, 8, 64, dtype=torch.float32).pin_memory()
    with pytest.raises(RuntimeError, match="out must be"):
        attention_from_host(h, h, h, out=bad)
