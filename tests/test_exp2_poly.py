"""The FMA-pipe exp2 of the prefill softmax: coefficients match their derivation and the FP32
evaluation meets its error bound (no GPU; the kernel's outputs are covered by the GPU suite)."""
import importlib.util
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "tiny-transformer_b200", "csrc")


def _fit_module():
    spec = importlib.util.spec_from_file_location("fit_exp2_poly", os.path.join(CSRC, "fit_exp2_poly.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _kernel_coeffs():
    text = open(os.path.join(CSRC, "prefill_sm100.cuh")).read()
    return np.array([float(re.search(rf"kPolyC{k} = ([0-9.eE+-]+)f;", text).group(1))
                     for k in (1, 2, 3)], dtype=np.float32)


def test_kernel_coefficients_match_fit():
    fitted = _fit_module().fit()
    np.testing.assert_array_equal(_kernel_coeffs(), fitted)


def test_error_bound_and_exact_points():
    mod = _fit_module()
    c = _kernel_coeffs()
    x = np.linspace(-60.0, 8.0, 200001, dtype=np.float32)
    rel = np.abs(mod.eval_fp32(c, x).astype(np.float64) / np.exp2(x.astype(np.float64)) - 1)
    assert rel.max() <= 1.05e-4
    # Masked scores and the clamp give exact zeros; 2^0 and integer powers are exact.
    assert (mod.eval_fp32(c, np.array([-np.inf, -1e30, -127.0, -200.0], np.float32)) == 0).all()
    ints = np.arange(-20, 9, dtype=np.float32)
    np.testing.assert_array_equal(mod.eval_fp32(c, ints), np.exp2(ints))
