"""Failure path of the bounded kernel waits, exercised without faulting, trapping or hanging a
GPU: a diagnostic kernel waits on a barrier phase that nothing completes, with a budget of a
few million cycles. The wait has to end by itself, the host has to read TT_ERR_TIMEOUT through
tt_attn_device_status, clearing it has to work, and the same context has to compute attention
correctly afterwards."""
import ctypes

import pytest
import torch

OK, BAD_ARG, TIMEOUT = 0, 1, 4


@pytest.fixture(scope="module")
def lib():
    from tiny_transformer_b200.operators._extension import load_c_abi
    return load_c_abi()


def test_selftest_budget_validated_before_cuda(lib):
    for budget in (0, -5, 10**9 + 1):
        assert lib.tt_attn_selftest_wait_timeout(budget, None) == BAD_ARG
        assert "budget_cycles" in lib.tt_attn_last_error().decode()


@pytest.mark.gpu
def test_wait_runs_out_and_reports_timeout(lib):
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")
    from oracle import attention_oracle as oracle
    from tiny_transformer_b200.operators import student

    flags = ctypes.c_uint(0)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 1) == OK  # start clean

    budget = 4_000_000  # ~2 ms at 1.9 GHz
    stream = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    assert lib.tt_attn_selftest_wait_timeout(budget, ctypes.c_void_p(stream.cuda_stream)) == OK
    stop.record(stream)
    stop.synchronize()
    ms = start.elapsed_time(stop)
    # The wait gave up on its own: not before its budget (>= budget at <= 2.1 GHz), and long
    # before anything that would look like a hang.
    assert budget / 2.1e6 <= ms < 1000.0, ms

    assert lib.tt_attn_device_status(ctypes.byref(flags), 1) == TIMEOUT
    assert flags.value & 1
    assert lib.tt_attn_device_status(ctypes.byref(flags), 0) == OK
    assert flags.value == 0

    # The context is still usable: a prefill and a decode on the same device are correct.
    g = torch.Generator().manual_seed(11)
    for tq, tk, past in ((96, 96, 0), (1, 300, 299)):
        q = torch.randn(2, 3, tq, 64, generator=g).bfloat16()
        k = torch.randn(2, 3, tk, 64, generator=g).bfloat16()
        v = torch.randn(2, 3, tk, 64, generator=g).bfloat16()
        o, lse = student.attention_with_lse(q.cuda(), k.cuda(), v.cuda(), past)
        ro, rlse = oracle.attention_fp64(q.float().numpy(), k.float().numpy(),
                                         v.float().numpy(), past)
        assert torch.allclose(o.float().cpu(), torch.from_numpy(ro).float(), atol=2e-2, rtol=3e-2)
        assert torch.allclose(lse.cpu(), torch.from_numpy(rlse).float(), atol=2e-4, rtol=2e-5)
    assert lib.tt_attn_device_status(ctypes.byref(flags), 0) == OK
