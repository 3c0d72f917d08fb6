"""tiny_transformer_b200.metrics: the work counts agree with the oracle's and bench.py's, and the
fields a benchmark entry gets are consistent (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as oracle
from tiny_transformer_b200 import metrics


@pytest.mark.parametrize("tq,tk", [(1, 1), (7, 7), (512, 512), (300, 1000), (129, 4096),
                                   (4096, 4096), (3, 2)])
def test_visible_pairs_match_oracle(tq, tk):
    if tk < tq:
        pytest.skip("Tk >= Tq by construction")
    past = tk - tq
    assert metrics.visible_pairs(tq, tk, past) == oracle.visible_pairs(tq, tk, past)


def test_work_matches_bench_counts():
    assert metrics.attention_work((4, 12, 4096, 64), 4096, 0)["flops"] == \
        oracle.prefill_flops(4, 12, 4096, 4096, 0) == 103104380928
    lens = np.random.default_rng(2026).integers(1024, 8193, size=64)
    assert metrics.attention_work((64, 12, 1, 64), 8192, 8191, lens.tolist())["bytes"] == \
        oracle.decode_bytes(64, 12, lens)
    assert metrics.attention_work((8, 12, 1, 64), 512, 511)["bytes"] == 12607872


def test_benchmark_entry_fields():
    q = torch.zeros(8, 12, 512, 64)
    k = torch.zeros(8, 12, 512, 64)
    fields = metrics.attention_metrics((q, k, k, 0, None), 39.78, peak_tflops=312.0)
    assert fields["kind"] == "prefill" and fields["bound"] == "tensor"
    assert abs(fields["tflops"] - 3227516928 / 39.78e-6 / 1e12) < 1e-9
    assert abs(fields["roofline_fraction"] - fields["tflops"] / 312.0) < 1e-12
    qd = torch.zeros(8, 12, 1, 64)
    fields = metrics.attention_metrics((qd, k, k, 511, None), 12.73, peak_gbs=1935.0)
    assert fields["kind"] == "decode" and "gbs" in fields and "roofline_fraction" in fields
    with pytest.raises(ValueError):
        metrics.attention_rates(0.0, {"kind": "prefill", "flops": 1})
