"""Loaders for the prebuilt in-tree sm_100a libraries.

Mirrors ``load_attention_extension`` of Tiny-transformer (tiny_transformer/operators/_extension.py:9-46),
but does not JIT-compile: the libraries are built ahead of time by ``build.py`` into ``_build/``
(``__graft_entry__.build()``) and travel with the checkout. A missing library is an error; there is
no fallback implementation.
"""
from __future__ import annotations

import ctypes
import glob
import importlib.machinery
import importlib.util
import os
import sys
from functools import lru_cache

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD_DIR = os.path.join(_PKG_DIR, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libtt_attention.so")
EXT_NAME = "tt_attention_C"


class ExtensionMissingError(RuntimeError):
    """The sm_100a libraries have not been built in this checkout."""


def _missing(what: str) -> ExtensionMissingError:
    return ExtensionMissingError(
        f"{what} is not built under {BUILD_DIR}; run `python tiny-transformer_b200/build.py` "
        "(or __graft_entry__.build()). The attention operator has no non-CUDA fallback.")


@lru_cache(maxsize=1)
def load_c_abi() -> ctypes.CDLL:
    """Load libtt_attention.so (the C ABI of include/tt_attention.h) with typed prototypes."""
    if not os.path.exists(LIB_PATH):
        raise _missing("libtt_attention.so")
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    i64p = ctypes.POINTER(ctypes.c_int64)
    lib.tt_attn_forward_bf16.restype = ctypes.c_int
    lib.tt_attn_forward_bf16.argtypes = [
        ctypes.c_void_p, i64p, ctypes.c_void_p, i64p, ctypes.c_void_p, i64p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.tt_attn_forward_workspace_size.restype = ctypes.c_size_t
    lib.tt_attn_forward_workspace_size.argtypes = [ctypes.c_int64] * 4
    lib.tt_attn_layout_supported.restype = ctypes.c_int
    lib.tt_attn_layout_supported.argtypes = [ctypes.c_void_p, i64p]
    lib.tt_attn_device_supported.restype = ctypes.c_int
    lib.tt_attn_device_supported.argtypes = []
    lib.tt_attn_device_status.restype = ctypes.c_int
    lib.tt_attn_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
    lib.tt_attn_backward_bf16.restype = ctypes.c_int
    lib.tt_attn_backward_bf16.argtypes = [
        ctypes.c_void_p, i64p, ctypes.c_void_p, i64p, ctypes.c_void_p, i64p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_void_p]
    lib.tt_attn_backward_bf16_deterministic.restype = ctypes.c_int
    lib.tt_attn_backward_bf16_deterministic.argtypes = lib.tt_attn_backward_bf16.argtypes
    lib.tt_attn_backward_workspace_size.restype = ctypes.c_size_t
    lib.tt_attn_backward_workspace_size.argtypes = [ctypes.c_int64] * 3
    lib.tt_rope_append_bf16.restype = ctypes.c_int
    lib.tt_rope_append_bf16.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, i64p, ctypes.c_void_p, i64p, ctypes.c_int64, ctypes.c_void_p]
    lib.tt_qkv_rope_append_bf16.restype = ctypes.c_int
    lib.tt_qkv_rope_append_bf16.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, i64p, ctypes.c_void_p, i64p,
        ctypes.c_int64, ctypes.c_void_p]
    lib.tt_attn_selftest_wait_timeout.restype = ctypes.c_int
    lib.tt_attn_selftest_wait_timeout.argtypes = [ctypes.c_int64, ctypes.c_void_p]
    lib.tt_attn_status_string.restype = ctypes.c_char_p
    lib.tt_attn_status_string.argtypes = [ctypes.c_int]
    lib.tt_attn_last_error.restype = ctypes.c_char_p
    lib.tt_attn_last_error.argtypes = []
    lib.tt_attn_abi_version.restype = ctypes.c_int
    lib.tt_attn_abi_version.argtypes = []
    return lib


@lru_cache(maxsize=1)
def load_attention_extension():
    """Import the PyTorch extension ``tt_attention_C`` (attention_forward -> (O, LSE))."""
    import torch  # noqa: F401  (loads libc10/libtorch before the extension)

    matches = sorted(glob.glob(os.path.join(BUILD_DIR, EXT_NAME + "*.so")))
    if not matches:
        raise _missing(EXT_NAME)
    load_c_abi()  # resolve libtt_attention.so by SONAME from the process
    loader = importlib.machinery.ExtensionFileLoader(EXT_NAME, matches[0])
    spec = importlib.util.spec_from_file_location(EXT_NAME, matches[0], loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    sys.modules[EXT_NAME] = module
    return module
