"""B200 (sm_100a) BF16 causal attention forward for Tiny-transformer.

A drop-in for the ``student`` attention operator of Tiny-transformer
(tiny_transformer/operators/student.py:214-232): prefill runs a tcgen05/TMEM/TMA kernel,
single-token decode a split-KV bulk-copy kernel, both behind the C ABI in
``include/tt_attention.h``. The directory name carries a hyphen, so the package is imported
under the name ``tiny_transformer_b200`` (see ``__graft_entry__.import_package``).

Public API:
    operators.student.attention(q, k, v, past_len=0, segment_ids=None, kv_lens=None) -> O
    operators.student.attention_with_lse(...) -> (O, LSE)
    operators._extension.load_attention_extension() -> the native module
    sharding: per-rank slices of the (batch x head) / batch work and the optional NCCL gather
"""

__version__ = "0.1.0"
