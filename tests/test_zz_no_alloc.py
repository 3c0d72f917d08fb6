"""GPU test of tt_attn_decode_bf16_noalloc, the decode entry point that allocates nothing.

It serves callers that cannot allocate device memory while they decode (a server whose GPU
memory is all reserved by its own pools, a Go/Java/Rust host using this library only through its
C ABI, a loop that must stay out of the driver's allocator): the split-KV partials live in an
8 MiB static device array inside libtt_attention.so instead of a caller workspace.

The test calls it through the C ABI twice in a row, on different inputs, and compares each
result with the workspace-taking entry point tt_attn_forward_bf16 on the same inputs. The
file name makes pytest collect it last; it needs no state from other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 8 << 20


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")
    from tiny_transformer_b200.operators._extension import load_c_abi
    lib = load_c_abi()
    i64p = ctypes.POINTER(ctypes.c_int64)
    fn = lib.tt_attn_decode_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, i64p, ctypes.c_void_p, i64p, ctypes.c_void_p, i64p,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _strides(x):
    return (ctypes.c_int64 * 4)(*x.stride())


def _inputs(seed, B, H, Tk, with_lens):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, H, 1, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, H, Tk, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, H, Tk, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    lens = None
    if with_lens:
        lens = torch.randint(1, Tk + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    return q, k, v, lens


def _with_workspace(lib, q, k, v, lens):
    B, H, _, _ = q.shape
    Tk = k.shape[2]
    out = torch.empty_like(q)
    lse = torch.empty(B, H, 1, device="cuda", dtype=torch.float32)
    n = lib.tt_attn_forward_workspace_size(B, H, 1, Tk)
    assert 0 < n <= NOALLOC_SCRATCH_BYTES  # the shapes below do use the scratch
    ws = torch.empty(n, device="cuda", dtype=torch.uint8)
    st = lib.tt_attn_forward_bf16(
        q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
        B, H, 1, Tk, 64, Tk - 1, None if lens is None else lens.data_ptr(), out.data_ptr(),
        lse.data_ptr(), ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.tt_attn_last_error()
    return out, lse


def _no_alloc(lib, q, k, v, lens):
    B, H, _, _ = q.shape
    Tk = k.shape[2]
    out = torch.full_like(q, float("nan"))
    lse = torch.full((B, H, 1), float("nan"), device="cuda", dtype=torch.float32)
    st = lib.tt_attn_decode_bf16_noalloc(
        q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
        B, H, Tk, None if lens is None else lens.data_ptr(), out.data_ptr(), lse.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.tt_attn_last_error()
    return out, lse


@torch.no_grad()
def test_no_alloc_decode_matches_workspace_entry_point_twice(lib):
    # Two calls in a row, with caches large enough (over 2^20 batch * head * key rows in more
    # than 640 sequences) for the split-KV kernel that uses the scratch.
    cases = [(11, 64, 12, 2048, False), (12, 56, 12, 2100, True)]
    for seed, B, H, Tk, with_lens in cases:
        q, k, v, lens = _inputs(seed, B, H, Tk, with_lens)
        ref_o, ref_lse = _with_workspace(lib, q, k, v, lens)
        o, lse = _no_alloc(lib, q, k, v, lens)
        torch.cuda.synchronize()
        # Same kernels on the same inputs: the tolerance of the parity suite, met exactly here.
        torch.testing.assert_close(o, ref_o, atol=2e-2, rtol=3e-2)
        torch.testing.assert_close(lse, ref_lse, atol=2e-4, rtol=2e-5)
        assert torch.equal(o, ref_o) and torch.equal(lse, ref_lse)


def test_no_alloc_rejects_shapes_beyond_its_scratch(lib):
    # 64 x 12 heads x 1M keys needs far more than 8 MiB of partials: rejected before any launch.
    B, H, Tk = 64, 12, 1 << 20
    assert lib.tt_attn_forward_workspace_size(B, H, 1, Tk) > NOALLOC_SCRATCH_BYTES
    seed = torch.zeros(1, 1, 1, 64, device="cuda", dtype=torch.bfloat16)
    q = seed.expand(B, H, 1, 64)
    kv = seed.expand(B, H, Tk, 64)
    out = torch.empty(B, H, 1, 64, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, H, 1, device="cuda", dtype=torch.float32)
    st = lib.tt_attn_decode_bf16_noalloc(
        q.data_ptr(), _strides(q), kv.data_ptr(), _strides(kv), kv.data_ptr(), _strides(kv),
        B, H, Tk, None, out.data_ptr(), lse.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 1  # TT_ATTN_BAD_ARG
    assert "at most 8388608 bytes" in lib.tt_attn_last_error().decode()
