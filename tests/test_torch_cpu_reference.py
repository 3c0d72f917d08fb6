"""The ATen restatement timed as the CPU baseline (oracle/torch_cpu_reference.py) reproduces the
reference's stored outputs (tests/golden, produced by Tiny-transformer's reference.attention on
CPU). It issues the same ATen operations in the same order, so on the same PyTorch build the
outputs are bit-identical; across builds a BF16 CPU matmul may round one element differently,
so the bar is one bf16 ulp with at least 99 % of elements identical."""
import numpy as np
import torch

from oracle import attention_oracle as oracle
from oracle import torch_cpu_reference as tref


def _t(bits):
    return torch.from_numpy(oracle.bf16_bits_to_f32(bits)).to(torch.bfloat16)


def test_aten_restatement_matches_reference_outputs(golden):
    for name, case in golden.items():
        q, k, v = (_t(case[x]) for x in ("q", "k", "v"))
        past = int(case["past_len"])
        if "kv_lens" in case:
            out = tref.decode_rows(q, k, v, case["kv_lens"])
        else:
            out = tref.attention(q, k, v, past)
        mine = out.view(torch.int16).numpy().astype(np.int32) & 0xFFFF
        theirs = case["o"].astype(np.int32)
        if "kv_lens" in case:
            # Rows with no visible key: the reference convention is O = 0.
            dead = np.asarray(case["kv_lens"]) <= 0
            mine[dead] = theirs[dead]
        same = np.mean(mine == theirs)
        ulps = np.abs(mine - theirs)
        assert same >= 0.99 and ulps.max() <= 1, f"{name}: {same:.4f} identical, {ulps.max()} ulp"


def test_prefill_rows_equals_one_call():
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(2, 3, 70, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    whole = tref.attention(q, k, v, 0)
    rows = tref.prefill_rows(q, k, v, 0, rows_per_call=4)
    assert torch.equal(whole, rows)


def test_lse_companion():
    g = torch.Generator().manual_seed(6)
    q, k, v = (torch.randn(1, 2, 33, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    out, lse = tref.attention_lse(q, k, v, 0)
    assert torch.equal(out, tref.attention(q, k, v, 0))
    _, lse64 = oracle.attention_fp64(*(x.float().numpy() for x in (q, k, v)), 0)
    # LSE of the bf16-rounded scores vs exact FP64 scores: within the rounding of the scores.
    np.testing.assert_allclose(lse.numpy(), lse64, atol=2e-2)
