"""In-tree build of the sm_100a attention libraries.

Produces, under ``_build/`` next to this file:

* ``libtt_attention.so`` - the C ABI (``include/tt_attention.h``) with the sm_100a
  kernels, compiled by nvcc for ``-gencode arch=compute_100a,code=sm_100a``. The CUDA
  runtime is linked statically, so the library loads without a GPU or a driver.
* ``tt_attention_C<EXT_SUFFIX>`` - the PyTorch extension exposing
  ``attention_forward(q, k, v, past_len=0, segment_ids=None, kv_lens=None)``; it links
  ``libtt_attention.so`` through an ``$ORIGIN`` rpath.

Run ``python tiny-transformer_b200/build.py`` (or ``__graft_entry__.build()``). Targets are
rebuilt only when a source is newer than the output.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
import sysconfig

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")

LIB_NAME = "libtt_attention.so"
EXT_NAME = "tt_attention_C"
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]

KERNEL_SOURCES = ["tt_attention_abi.cu"]
KERNEL_HEADERS = ["sm100_ptx.cuh", "prefill_sm100.cuh", "decode_sm100.cuh",
                  "decode_direct_sm100.cuh",
                  "rope_append_sm100.cuh", "qkv_rope_sm100.cuh", "selftest_sm100.cuh", "backward_sm100.cuh",
                  "backward_det_sm100.cuh"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def lib_path() -> str:
    return os.path.join(BUILD_DIR, LIB_NAME)


def ext_path() -> str:
    return os.path.join(BUILD_DIR, EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, check=True, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                         text=True)
    if verbose and res.stdout.strip():
        print(res.stdout, flush=True)
    return res.stdout


# The prefill kernel re-allocates registers between warpgroups (setmaxnreg); its launch register
# count must equal the value that hand-over was sized for (prefill_sm100.cuh: LAUNCH_REGS).
def _prefill_launch_regs() -> int:
    text = open(os.path.join(CSRC, "prefill_sm100.cuh")).read()
    return int(re.search(r"constexpr uint32_t LAUNCH_REGS = (\d+);", text).group(1))


def _check_ptxas(report: str) -> None:
    lines = report.splitlines()
    found = 0
    for i, line in enumerate(lines):
        if "Compiling entry function" in line and "attention_prefill_kernel" in line:
            for follow in lines[i + 1:i + 4]:
                m = re.search(r"Used (\d+) registers", follow)
                if m:
                    regs = int(m.group(1))
                    want = _prefill_launch_regs()
                    if regs != want:
                        raise RuntimeError(
                            f"attention_prefill_kernel compiled with {regs} registers, expected "
                            f"{want}: the setmaxnreg hand-over would not be sound")
                    found += 1
                    break
    if found == 0:
        raise RuntimeError("ptxas report for attention_prefill_kernel not found")


def build_library(verbose: bool = False, force: bool = False) -> str:
    """Compile the C ABI and kernels into _build/libtt_attention.so."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in KERNEL_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in KERNEL_HEADERS] + [
        os.path.join(INCLUDE, "tt_attention.h")]
    out = lib_path()
    if force or _stale(out, deps):
        cmd = [_nvcc(), *GENCODE, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xptxas=-v",
               "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I" + INCLUDE, "-I" + CSRC,
               *srcs, "-o", out, "-Xlinker", "-soname=" + LIB_NAME]
        try:
            _check_ptxas(_run(cmd, verbose))
        except Exception:
            if os.path.exists(out):
                os.remove(out)
            raise
    return out


def build_extension(verbose: bool = False, force: bool = False) -> str:
    """Compile the PyTorch binding against libtt_attention.so."""
    import torch
    from torch.utils import cpp_extension

    lib = build_library(verbose=verbose, force=force)
    src = os.path.join(CSRC, "torch_binding.cpp")
    out = ext_path()
    if force or _stale(out, [src, lib, os.path.join(INCLUDE, "tt_attention.h")]):
        cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        includes = cpp_extension.include_paths() + [
            sysconfig.get_paths()["include"], os.path.join(cuda_home, "include"), INCLUDE]
        libdirs = cpp_extension.library_paths()
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
               "-DTORCH_API_INCLUDE_EXTENSION_H", src, "-o", out]
        cmd += ["-I" + p for p in includes]
        cmd += ["-L" + p for p in libdirs]
        cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
                "-L" + BUILD_DIR, "-ltt_attention", "-Wl,-rpath,$ORIGIN"]
        _run(cmd, verbose)
    return out


def build(verbose: bool = False, force: bool = False) -> None:
    build_extension(verbose=verbose, force=force)


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
