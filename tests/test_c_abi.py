"""The C ABI library loads, exports every declared symbol, and validates arguments before any
CUDA call (runs without a GPU: no kernel is launched here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tt_attention.h")


@pytest.fixture(scope="module")
def lib():
    from tiny_transformer_b200.operators._extension import load_c_abi
    return load_c_abi()


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"TT_ATTN_API\s+[\w\s\*]+?\b(tt_attn_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "tt_attn_forward_bf16" in names
    assert len(names) == len(set(names)) >= 8


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} missing from libtt_attention.so"


def test_status_strings_and_version(lib):
    assert lib.tt_attn_abi_version() == 1
    for code, name in enumerate(["TT_ATTN_OK", "TT_ATTN_BAD_ARG", "TT_ATTN_UNSUPPORTED",
                                 "TT_ATTN_LAUNCH_FAIL", "TT_ATTN_TIMEOUT"]):
        assert lib.tt_attn_status_string(code).decode() == name


def _strides(*s):
    return (ctypes.c_int64 * 4)(*s)


def _call(lib, *, q=16, k=16, v=16, out=16, lse=16, B=1, H=1, tq=4, tk=4, d=64, past=0,
          lens=None, qs=None, ks=None, vs=None, ws=None, ws_bytes=0):
    qs = qs or _strides(tq * 64 * H, tq * 64, 64, 1)
    ks = ks or _strides(tk * 64 * H, tk * 64, 64, 1)
    vs = vs or ks
    return lib.tt_attn_forward_bf16(q, qs, k, ks, v, vs, B, H, tq, tk, d, past, lens, out, lse,
                                    ws, ws_bytes, None)


def _err(lib):
    return lib.tt_attn_last_error().decode()


@pytest.mark.parametrize("kwargs,fragment", [
    (dict(q=None), "must not be NULL"),
    (dict(out=None), "must not be NULL"),
    (dict(d=32), "head_dim=64"),
    (dict(B=0), "positive"),
    (dict(tk=0), "positive"),
    (dict(past=-1), "non-negative"),
    (dict(past=1), "Tk == past_len"),
    (dict(tq=5, tk=4, past=0), "Tk == past_len"),
    (dict(tq=2**31, tk=2**31), "fit int32"),
    (dict(tq=2, tk=2, lens=16), "kv_lens requires"),
    (dict(B=2**31 - 1, H=2), "grid limits"),
])
def test_bad_arguments_rejected_before_cuda(lib, kwargs, fragment):
    assert _call(lib, **kwargs) == 1  # TT_ATTN_BAD_ARG
    assert fragment in _err(lib)


def test_unsupported_layouts(lib):
    # Unaligned base, non-unit inner stride, stride not a multiple of 8 elements.
    assert _call(lib, q=18) == 2
    assert "aligned" in _err(lib)
    assert _call(lib, ks=_strides(512, 256, 128, 2)) == 2
    assert _call(lib, ks=_strides(4 * 66, 4 * 66, 66, 1), H=1, B=2, tk=4, tq=4) == 2


def test_workspace_and_layout_queries(lib):
    # Decode of a large cache (the persistent split-KV kernel) splits into several chunks and
    # needs partials.
    n = lib.tt_attn_forward_workspace_size(64, 12, 1, 4096)
    arrivals = -(-64 * 12 * 4 // 256) * 256       # one counter per (batch, head), 256-B rounded
    assert n > 256 + arrivals and (n - 256 - arrivals) % (68 * 4) == 0  # counters + partials
    # Caches of at most 2^20 (batch * head * key) rows, or of at most 2^21 rows in at most 640
    # sequences, take the cluster kernel: no workspace.
    assert lib.tt_attn_forward_workspace_size(8, 12, 1, 16) == 0
    assert lib.tt_attn_forward_workspace_size(8, 12, 1, 4096) == 0
    assert lib.tt_attn_forward_workspace_size(8, 12, 1, 8192) == 0
    assert lib.tt_attn_forward_workspace_size(16, 12, 1, 8192) == 0
    assert lib.tt_attn_forward_workspace_size(1, 1, 1, 1 << 21) == 0
    assert lib.tt_attn_forward_workspace_size(640, 1, 1, 2048) == 0
    assert lib.tt_attn_forward_workspace_size(641, 1, 1, 2048) > 0
    assert lib.tt_attn_forward_workspace_size(1, 1, 1, (1 << 21) + 1) > 0
    assert lib.tt_attn_forward_workspace_size(32, 12, 1, 8192) > 0
    # Enough sequences that each takes one 1536-key item: the work counter only.
    assert lib.tt_attn_forward_workspace_size(100, 12, 1, 1500) == 256
    assert lib.tt_attn_forward_workspace_size(8, 12, 512, 512) == 0  # enough CTAs: no split
    assert lib.tt_attn_forward_workspace_size(4, 12, 4096, 4096) == 0
    # Fewer query blocks than SMs (an 8-way shard of B=4 H=12 T=4096: 6 rows, 96 blocks): the
    # long blocks are split into parts of at most 16 KV tiles, the smallest size whose CTAs
    # (8 + 8 x 2 per row = 144) fit one wave of 148; the longest block (32 tiles) has 2 parts,
    # and each row, block and part has a 272-byte record.
    assert lib.tt_attn_forward_workspace_size(1, 6, 4096, 4096) == 6 * 16 * 2 * 256 * 272
    # One sequence: parts of 4 tiles (72 CTAs), the longest block in 8.
    assert lib.tt_attn_forward_workspace_size(1, 1, 4096, 4096) == 16 * 8 * 256 * 272
    # 12 rows (192 blocks) already exceed one wave: no split.
    assert lib.tt_attn_forward_workspace_size(1, 12, 4096, 4096) == 0
    assert lib.tt_attn_forward_workspace_size(1, 1, 513, 512) == 0  # q_len > kv_len: invalid
    assert lib.tt_attn_forward_workspace_size(0, 12, 1, 512) == 0
    # Missing workspace for a split decode is rejected.
    assert _call(lib, B=64, H=12, tq=1, tk=4096, past=4095) == 1
    assert "workspace" in _err(lib)
    assert lib.tt_attn_layout_supported(16, _strides(4096, 4096, 64, 1)) == 1
    assert lib.tt_attn_layout_supported(17, _strides(4096, 4096, 64, 1)) == 0
    assert lib.tt_attn_layout_supported(16, _strides(4096, 4096, 64, 2)) == 0
    assert lib.tt_attn_layout_supported(16, _strides(0, 4096, 64, 1)) == 0
    assert lib.tt_attn_layout_supported(None, _strides(4096, 4096, 64, 1)) == 0


def _bwd(lib, *, q=16, k=16, v=16, do=16, o=16, lse=16, dq=16, dk=16, dv=16, B=1, H=1, tq=4,
         tk=4, d=64, past=0, ws=256, ws_bytes=1 << 20, entry="tt_attn_backward_bf16"):
    qs = _strides(tq * 64 * H, tq * 64, 64, 1)
    ks = _strides(tk * 64 * H, tk * 64, 64, 1)
    return getattr(lib, entry)(q, qs, k, ks, v, ks, do, o, lse, B, H, tq, tk, d, past,
                               dq, dk, dv, ws, ws_bytes, None)


@pytest.mark.parametrize("kwargs,fragment", [
    (dict(do=None), "must not"),
    (dict(d=32), "head_dim=64"),
    (dict(B=0), "positive"),
    (dict(past=-1), "non-negative"),
    (dict(tk=5), "Tk == past_len + Tq"),
    (dict(tq=2**31, tk=2**31), "int32"),
    (dict(B=2**20, H=2**12), "grid limits"),
    (dict(tq=2**31 - 64, tk=2**31 - 64), "grid limits"),  # rows padded to 128 exceed int32
    (dict(dq=24), "16-byte"),
    (dict(lse=18), "4-byte"),
    (dict(ws_bytes=4), "workspace"),
])
@pytest.mark.parametrize("entry", ["tt_attn_backward_bf16", "tt_attn_backward_bf16_deterministic"])
def test_backward_rejects_bad_arguments_before_cuda(lib, kwargs, fragment, entry):
    assert _bwd(lib, entry=entry, **kwargs) == 1  # TT_ATTN_BAD_ARG
    assert fragment in _err(lib)


def test_backward_unsupported_layout_and_workspace_size(lib):
    # q with a feature stride of 2 cannot be read in place.
    qs = _strides(4 * 128, 128, 128, 2)
    ks = _strides(4 * 64, 64, 64, 1)
    assert lib.tt_attn_backward_bf16(16, qs, 16, ks, 16, ks, 16, 16, 16, 1, 1, 4, 4, 64, 0,
                                     16, 16, 16, 256, 1 << 20, None) == 2  # UNSUPPORTED
    # -LSE * log2(e) and -D for 6 heads x 128 padded rows, then the 30 x 64 FP32 dQ accumulator.
    assert lib.tt_attn_backward_workspace_size(2, 3, 5) == 2 * 6 * 128 * 4 + 2 * 3 * 5 * 64 * 4 + 16
    assert lib.tt_attn_backward_workspace_size(0, 3, 5) == 0


def test_no_alloc_argument_checks_before_any_cuda_call(lib):
    """The no-allocation decode rejects non-positive sizes and shapes whose partials exceed its
    8 MiB scratch before touching CUDA (no GPU in this process)."""
    fn = lib.tt_attn_decode_bf16_noalloc
    i64p = ctypes.POINTER(ctypes.c_int64)
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, i64p, ctypes.c_void_p, i64p, ctypes.c_void_p, i64p,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    st = _strides(64, 64, 64, 1)
    assert fn(16, st, 16, st, 16, st, 0, 12, 100, None, 16, 16, None) == 1
    assert "positive" in _err(lib)
    assert fn(16, st, 16, st, 16, st, 64, 12, 1 << 20, None, 16, 16, None) == 1
    assert "at most 8388608 bytes" in _err(lib)
