"""Parity at the exact configurations bench.py times (needs a B200).

The bench's own generators (bench.make_prefill / make_decode, same seeds) feed the native
operator, and the outputs are checked against the CPU oracle:

* against the restated BF16 ``reference.attention`` with the north-star bars: max |dO| <= 2e-2,
  mean |dO| <= 2e-3, LSE relative error <= 1e-3 (vs the FP64 LSE);
* against the FP64 oracle with the reference tests' bars (tests/test_student_attention.py:
  116-117): O atol 2e-2 / rtol 3e-2, LSE atol 2e-4 / rtol 2e-5.

Configurations: cfg1 (B=8 H=12 T=512) whole; cfg3 (B=4 H=12 T=4096) on the first, a middle and
the last (batch, head) row of the whole-workload call, and on the 8-way shards bench.py gives
each rank (whose long query blocks run split over their KV range); cfg4 (B=64 H=12 Tk=8192,
kv_lens U[1024, 8192] by the bench seed) on every sequence; cfg2 (B=8 H=12 Tk=512 decode)
whole.
"""
import numpy as np
import pytest
import torch

import bench
from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS, LSE_REL = 2e-2, 2e-3, 1e-3
O_ATOL, O_RTOL = 2e-2, 3e-2
LSE_ATOL, LSE_RTOL = 2e-4, 2e-5


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    if torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")
    from tiny_transformer_b200.operators._extension import load_attention_extension
    return load_attention_extension()


def _np(x):
    return x.detach().float().cpu().numpy()


def _check(out, lse, q, k, v, past_len):
    """out/lse/q/k/v: numpy float32 of one or more rows; returns (max, mean) |dO|."""
    ref_bf16 = oracle.reference_attention_bf16(q, k, v, past_len)
    ref64, lse64 = oracle.attention_fp64(q, k, v, past_len)
    diff = np.abs(out - ref_bf16)
    assert diff.max() <= MAX_ABS, f"max |dO| vs reference {diff.max()}"
    assert diff.mean() <= MEAN_ABS, f"mean |dO| vs reference {diff.mean()}"
    rel = np.abs(lse - lse64) / np.maximum(np.abs(lse64), 1.0)
    assert rel.max() <= LSE_REL, f"LSE relative error {rel.max()}"
    np.testing.assert_allclose(out, ref64, atol=O_ATOL, rtol=O_RTOL)
    np.testing.assert_allclose(lse, lse64, atol=LSE_ATOL, rtol=LSE_RTOL)
    assert np.isfinite(out).all()
    return diff.max(), diff.mean()


@torch.no_grad()
def test_cfg1_whole(ext):
    q, k, v = bench.make_prefill(torch, bench.CFG1)
    out, lse = ext.attention_forward(q, k, v, 0)
    _check(_np(out), _np(lse), _np(q), _np(k), _np(v), 0)


@torch.no_grad()
def test_cfg3_rows_whole_and_sharded(ext):
    from tiny_transformer_b200.sharding import even_shards, prefill_slice
    q, k, v = bench.make_prefill(torch)
    out, lse = ext.attention_forward(q, k, v, 0)
    flat = [x.reshape(-1, 1, *x.shape[2:]) for x in (out, lse, q, k, v)]
    n = flat[0].shape[0]
    for r in (0, n // 2, n - 1):
        _check(*(_np(x[r:r + 1]) for x in flat), 0)
    # The 8-way shards the multi-GPU bench computes (6 rows each: few CTAs, so the long query
    # blocks are split over their KV range and merged): the oracle on each shard's last row,
    # and the whole call's rows to within the FP32 merge order.
    for shard in even_shards(n, 8):
        qs, ks, vs = (prefill_slice(x, shard) for x in (q, k, v))
        o_s, l_s = ext.attention_forward(qs, ks, vs, 0)
        torch.testing.assert_close(o_s, flat[0][shard.start:shard.stop], atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(l_s, flat[1][shard.start:shard.stop], atol=1e-5, rtol=1e-6)
        r = shard.size - 1
        _check(_np(o_s[r:r + 1]), _np(l_s[r:r + 1]), _np(qs[r:r + 1]), _np(ks[r:r + 1]),
               _np(vs[r:r + 1]), 0)


@torch.no_grad()
def test_cfg4_every_sequence(ext):
    c = bench.DECODE_CFG
    q, k, v, lens = bench.make_decode(torch)
    out, lse = ext.attention_forward(q, k, v, c["Tk"] - 1, None, lens)
    lens_np = bench.decode_lengths()
    assert (lens.cpu().numpy() == lens_np).all()
    worst = 0.0
    for b in range(c["B"]):
        L = int(lens_np[b])
        mx, _ = _check(_np(out[b:b + 1]), _np(lse[b:b + 1]), _np(q[b:b + 1]),
                       _np(k[b:b + 1, :, :L]), _np(v[b:b + 1, :, :L]), L - 1)
        worst = max(worst, mx)
    # The batch shards of the multi-GPU bench at 2, 4 and 8 ranks (the split-KV kernel, then
    # the cluster kernel): a smaller batch may take another kernel or split, so the FP32 merge
    # order (not the result's accuracy) can differ from the whole call.
    shards = [bench.decode_shard(w, r, lens_np) for w in (2, 4, 8) for r in range(w)]
    for shard in shards:
        sl = slice(shard.start, shard.stop)
        o_s, l_s = ext.attention_forward(q[sl], k[sl], v[sl], c["Tk"] - 1, None, lens[sl])
        torch.testing.assert_close(o_s, out[sl], atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(l_s, lse[sl], atol=1e-5, rtol=1e-6)


@torch.no_grad()
def test_cfg2_whole(ext):
    c = bench.CFG2
    q, k, v, _ = bench.make_decode(torch, dict(c, data_seed=c["seed"]), with_lens=False)
    out, lse = ext.attention_forward(q, k, v, c["Tk"] - 1)
    _check(_np(out), _np(lse), _np(q), _np(k), _np(v), c["Tk"] - 1)
