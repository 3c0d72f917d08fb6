"""Generate tests/golden/attention_golden.npz from the reference's own operator.

Runs Tiny-transformer's executable specification ``tiny_transformer.operators.reference.attention``
(reference.py:49-53) on CPU with PyTorch, on seeded BF16 inputs, and stores inputs and outputs as
raw bf16 bit patterns. The oracle (oracle/attention_oracle.py) is pinned against this file by
tests/test_oracle_golden.py; the CUDA path is checked against both.

The reference checkout is only available in the build container, so this script is run there
once and its output committed:

    python tests/golden/make_golden.py /path/to/Tiny-transformer

Cases (all seeded, N(0,1) unless noted):
  prefill_*    square causal prefill (past_len = 0), tile tails around 64/128
  chunk_*      chunked prefill with a KV cache (past_len > 0)
  decode_*     single-token decode (Tq = 1), split boundaries around 128/256
  kvlens_*     decode with per-sequence valid lengths: the reference has no such argument, so
               each row is reference.attention on its prefix with past_len = L_b - 1
  large_logit  q = k = 10 everywhere (large equal logits), V random
"""
from __future__ import annotations

import os
import sys

import numpy as np


def main(ref_root: str, out_path: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    from tiny_transformer.operators import reference

    def bits(t: torch.Tensor) -> np.ndarray:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def lse64(q, k, v, past_len):
        # FP64 logsumexp of the scaled, causally masked scores (test_student_attention.py:108-117).
        scores = q.double() @ k.double().transpose(-1, -2) / 8.0
        allowed = reference.causal_mask(q, k, past_len)
        return scores.masked_fill(~allowed, -float("inf")).logsumexp(-1).numpy()

    cases = {}

    def add(name, q, k, v, past_len, kv_lens=None):
        if kv_lens is None:
            o = reference.attention(q, k, v, past_len)
            lse = lse64(q, k, v, past_len)
        else:
            o = torch.zeros_like(q)
            lse = np.full(q.shape[:-1], -np.inf)
            for b, L in enumerate(kv_lens):
                if L == 0:
                    continue
                sl = slice(b, b + 1)
                o[sl] = reference.attention(q[sl], k[sl, :, :L], v[sl, :, :L], L - 1)
                lse[sl] = lse64(q[sl], k[sl, :, :L], v[sl, :, :L], L - 1)
            cases[f"{name}/kv_lens"] = np.asarray(kv_lens, dtype=np.int32)
        cases[f"{name}/q"] = bits(q)
        cases[f"{name}/k"] = bits(k)
        cases[f"{name}/v"] = bits(v)
        cases[f"{name}/o"] = bits(o)
        cases[f"{name}/lse64"] = lse.astype(np.float64)
        cases[f"{name}/past_len"] = np.asarray(past_len, dtype=np.int64)

    gen = torch.Generator().manual_seed(20261201)

    def randn(*shape):
        return torch.randn(*shape, generator=gen).to(torch.bfloat16)

    for t in (1, 17):
        add(f"prefill_t{t}", randn(2, 3, t, 64), randn(2, 3, t, 64), randn(2, 3, t, 64), 0)
    for t in (64, 65, 129, 200):
        add(f"prefill_t{t}", randn(1, 2, t, 64), randn(1, 2, t, 64), randn(1, 2, t, 64), 0)
    for tq, tk in ((7, 129), (63, 193), (65, 257), (2, 64), (128, 300)):
        add(f"chunk_q{tq}_k{tk}", randn(1, 1, tq, 64), randn(1, 1, tk, 64), randn(1, 1, tk, 64),
            tk - tq)
    for tk in (1, 2, 127, 128, 129, 257):
        add(f"decode_k{tk}", randn(1, 2, 1, 64), randn(1, 2, tk, 64), randn(1, 2, tk, 64), tk - 1)
    add("decode_k600", randn(1, 1, 1, 64), randn(1, 1, 600, 64), randn(1, 1, 600, 64), 599)
    add("kvlens_a", randn(4, 1, 1, 64), randn(4, 1, 200, 64), randn(4, 1, 200, 64), 199,
        kv_lens=[1, 77, 200, 130])
    add("kvlens_b", randn(3, 1, 1, 64), randn(3, 1, 260, 64), randn(3, 1, 260, 64), 259,
        kv_lens=[129, 0, 260])
    big = torch.full((1, 2, 96, 64), 10.0).to(torch.bfloat16)
    add("large_logit", big, big.clone(), randn(1, 2, 96, 64), 0)

    np.savez_compressed(out_path, **cases)
    print(f"wrote {out_path}: {len([c for c in cases if c.endswith('/q')])} cases, "
          f"{os.path.getsize(out_path)} bytes")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TT_REFERENCE_ROOT", "")
    if not root or not os.path.isdir(root):
        raise SystemExit("usage: make_golden.py <Tiny-transformer checkout>")
    main(root, os.path.join(os.path.dirname(os.path.abspath(__file__)), "attention_golden.npz"))
