"""Throughput fields for the attention entries of Tiny-transformer's operator benchmark.

The reference's ``python -m tiny_transformer.benchmarks --operator attention`` (benchmarks/
operators.py:124-167, ``run_case``) records ``reference_us`` / ``candidate_us`` per phase. These
helpers turn a measured time and the case's inputs into the algorithmic work and rates this
library reports in its own bench: TFLOP/s over the visible (query, key) pairs for prefill
(4 * D FLOP per pair: the two products, softmax excluded), GB/s of the K/V rows a decode step
must read plus q, O and LSE, and the fraction of a roofline peak when one is given.

The counts are those of bench.py and oracle/attention_oracle.py (visible_pairs, prefill_flops,
decode_bytes), restated here so that the shipped package does not import the oracle.
"""
from __future__ import annotations

from typing import Sequence


def visible_pairs(q_len: int, kv_len: int, past_len: int) -> int:
    """(query, key) pairs with key <= query + past_len and key < kv_len (inclusive causal)."""
    if q_len <= 0 or kv_len <= 0:
        return 0
    # Query i sees min(i + past_len + 1, kv_len) keys.
    full_from = max(0, min(q_len, kv_len - past_len))  # queries whose row is not capped
    rows = full_from * (past_len + 1) + full_from * (full_from - 1) // 2
    return rows + (q_len - full_from) * kv_len


def attention_work(q_shape: Sequence[int], kv_len: int, past_len: int,
                   kv_lens: Sequence[int] | None = None) -> dict:
    """Algorithmic work of one BF16 attention forward call on [B, H, Tq, 64] queries.

    Prefill (Tq > 1): ``{"kind": "prefill", "flops": 4 * B * H * 64 * visible_pairs}``.
    Decode (Tq == 1): ``{"kind": "decode", "bytes": K/V rows read (all Tk, or sum(kv_lens)
    per head) * 128 bytes * 2 + q and O (128 bytes each) and LSE (4 bytes) per (b, h)}``.
    """
    B, H, Tq, D = (int(x) for x in q_shape)
    if Tq == 1:
        keys = (sum(max(0, min(int(L), kv_len)) for L in kv_lens) if kv_lens is not None
                else B * kv_len)
        return {"kind": "decode",
                "bytes": keys * H * D * 2 * 2 + B * H * (D * 2 * 2 + 4)}
    return {"kind": "prefill", "flops": 4 * B * H * D * visible_pairs(Tq, kv_len, past_len)}


def attention_rates(microseconds: float, work: dict, peak_tflops: float | None = None,
                    peak_gbs: float | None = None) -> dict:
    """TFLOP/s (prefill) or GB/s (decode) for a call that took ``microseconds``, and the
    fraction of the given peak (dense BF16 TFLOP/s or HBM GB/s) when one is given."""
    if not microseconds > 0:
        raise ValueError("time must be positive")
    if work["kind"] == "prefill":
        rate = work["flops"] / (microseconds * 1e-6) / 1e12
        out = {"tflops": rate, "bound": "tensor"}
        if peak_tflops:
            out["roofline_fraction"] = rate / peak_tflops
    else:
        rate = work["bytes"] / (microseconds * 1e-6) / 1e9
        out = {"gbs": rate, "bound": "hbm"}
        if peak_gbs:
            out["roofline_fraction"] = rate / peak_gbs
    return out


def attention_metrics(inputs: Sequence, microseconds: float, peak_tflops: float | None = None,
                      peak_gbs: float | None = None) -> dict:
    """Fields for a ``run_case`` phase result from the case's ``inputs`` (q, k, v, past_len,
    segment_ids, as benchmarks/cases.py builds them) and the candidate's time."""
    q, k = inputs[0], inputs[1]
    past_len = int(inputs[3]) if len(inputs) > 3 else 0
    work = attention_work(tuple(q.shape), int(k.shape[-2]), past_len)
    return {**work, **attention_rates(microseconds, work, peak_tflops, peak_gbs)}
