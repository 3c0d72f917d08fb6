"""Prefill with the KV range of long query blocks split over several CTAs (needs a B200).

When a call has few 256-row query blocks for the 148 SMs (a (batch x head) shard of a long
sequence on one of several GPUs, or a single long sequence), query blocks longer than the
average KV tiles per SM run as several CTAs over consecutive parts of their KV range; the parts
write FP32 partial records (unnormalised O, running max, row sum) that a combine kernel
merges. These tests check the split path against the oracle, against the unsplit path (the
same rows inside a batch large enough not to split), and the workspace it asks for.
"""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS, LSE_REL = 2e-2, 2e-3, 1e-3
O_ATOL, O_RTOL = 2e-2, 3e-2
LSE_ATOL, LSE_RTOL = 2e-4, 2e-5


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")
    from tiny_transformer_b200.operators._extension import load_attention_extension
    return load_attention_extension()


def _np(x):
    return x.detach().float().cpu().numpy()


def _check(out, lse, q, k, v, past_len):
    ref_bf16 = oracle.reference_attention_bf16(q, k, v, past_len)
    ref64, lse64 = oracle.attention_fp64(q, k, v, past_len)
    diff = np.abs(out - ref_bf16)
    assert diff.max() <= MAX_ABS and diff.mean() <= MEAN_ABS, (diff.max(), diff.mean())
    rel = np.abs(lse - lse64) / np.maximum(np.abs(lse64), 1.0)
    assert rel.max() <= LSE_REL
    np.testing.assert_allclose(out, ref64, atol=O_ATOL, rtol=O_RTOL)
    np.testing.assert_allclose(lse, lse64, atol=LSE_ATOL, rtol=LSE_RTOL)


def _workspace(B, H, tq, tk):
    from tiny_transformer_b200.operators._extension import load_c_abi
    return load_c_abi().tt_attn_forward_workspace_size(B, H, tq, tk)


@pytest.mark.parametrize("B,H,tq,tk", [
    (1, 1, 4096, 4096),   # one sequence: every block past the first 4 KV tiles is split
    (1, 6, 4096, 4096),   # an 8-way shard of config 3
    (2, 3, 1000, 1000),   # ragged last block
    (1, 2, 1500, 2000),   # chunked prefill (past_len = 500): the diagonal moves inside parts
    (1, 1, 300, 4096),    # short query over a long cache
])
@torch.no_grad()
def test_split_prefill_matches_oracle(ext, B, H, tq, tk):
    assert _workspace(B, H, tq, tk) > 0, "shape expected to take the split path"
    g = torch.Generator(device="cuda").manual_seed(tq + 7 * tk + B * H)
    q = torch.randn(B, H, tq, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, H, tk, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, H, tk, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    past = tk - tq
    out, lse = ext.attention_forward(q, k, v, past)
    assert torch.isfinite(out).all() and torch.isfinite(lse).all()
    for b in range(B):
        for h in sorted({0, H - 1}):
            _check(_np(out[b:b + 1, h:h + 1]), _np(lse[b:b + 1, h:h + 1]), _np(q[b:b + 1, h:h + 1]),
                   _np(k[b:b + 1, h:h + 1]), _np(v[b:b + 1, h:h + 1]), past)


@torch.no_grad()
def test_split_rows_equal_unsplit_rows(ext):
    """The same (batch, head) rows computed split (6 rows) and unsplit (inside 300 rows, enough
    CTAs to fill the SMs): equal to within the FP32 merge order."""
    T, H = 4096, 300
    assert _workspace(1, H, T, T) == 0 and _workspace(1, 6, T, T) > 0
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(1, H, T, 64, generator=g, device="cuda", dtype=torch.bfloat16)
               for _ in range(3))
    whole_o, whole_l = ext.attention_forward(q, k, v, 0)
    part_o, part_l = ext.attention_forward(q[:, :6], k[:, :6], v[:, :6], 0)
    torch.testing.assert_close(part_o, whole_o[:, :6], atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(part_l, whole_l[:, :6], atol=1e-5, rtol=1e-6)
    # bf16 outputs differ at most by one rounding step of the merge.
    assert (part_o.float() - whole_o[:, :6].float()).abs().mean() < 1e-4


@torch.no_grad()
def test_split_prefill_poisoned_workspace_and_repeat(ext):
    """Every partial record is written before it is read: a workspace full of NaN (through the
    C ABI) gives the same result as a fresh one, twice in a row."""
    import ctypes
    from tiny_transformer_b200.operators._extension import load_c_abi
    lib = load_c_abi()
    B, H, T = 1, 2, 3000
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(B, H, T, 64, generator=g, device="cuda", dtype=torch.bfloat16)
               for _ in range(3))
    ref_o, ref_l = ext.attention_forward(q, k, v, 0)
    n = lib.tt_attn_forward_workspace_size(B, H, T, T)
    assert n > 0
    ws = torch.full((n // 4,), float("nan"), device="cuda", dtype=torch.float32)
    st = (ctypes.c_int64 * 4)(*q.stride())
    for _ in range(2):
        out = torch.empty_like(q)
        lse = torch.empty(B, H, T, device="cuda", dtype=torch.float32)
        rc = lib.tt_attn_forward_bf16(q.data_ptr(), st, k.data_ptr(), st, v.data_ptr(), st, B, H,
                                      T, T, 64, 0, None, out.data_ptr(), lse.data_ptr(),
                                      ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.tt_attn_last_error()
        torch.cuda.synchronize()
        assert torch.equal(out, ref_o) and torch.equal(lse, ref_l)
