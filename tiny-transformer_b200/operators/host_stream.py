"""Causal attention over host-resident inputs, with the PCIe copies overlapped with the kernels.

``student.attention`` takes CUDA tensors: a caller whose q, k, v sit in host memory (offline
scoring, a CPU-side data pipeline) would copy all of them in, run the kernel, and copy O and LSE
out, one after the other. Every (batch, head) row of causal attention is independent of the
others, so this entry point streams the rows in slices instead: slice i + 1 is copied in on one
stream while slice i runs on the caller's current stream and slice i - 1 is copied out on a third
stream (PCIe is full duplex, so input and output copies overlap each other too). The kernel is
the same prefill / decode path as ``student.attention_with_lse``, called per slice through it,
so each row's O and LSE are bitwise those of one call over device copies of the whole batch.

No reference counterpart: the reference operator (tiny_transformer/operators/student.py:213-232)
accepts CUDA tensors only.
"""
from __future__ import annotations

import threading

import torch

from . import student

_streams = {}
_streams_lock = threading.Lock()


def _side_streams(device):
    """Two non-default streams per device (input copies, output copies), created once.
    ``device`` carries an explicit index (the caller normalises "cuda" to the current one)."""
    key = device.index
    with _streams_lock:
        if key not in _streams:
            _streams[key] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
        return _streams[key]


def _check_host(name, x, shape=None, dtype=torch.bfloat16):
    if x.is_cuda:
        raise RuntimeError(f"attention_from_host: {name} must be a host tensor")
    if not x.is_pinned():
        raise RuntimeError(f"attention_from_host: {name} must be in pinned host memory "
                           "(tensor.pin_memory()), so its copies run asynchronously")
    if not x.is_contiguous():
        raise RuntimeError(f"attention_from_host: {name} must be contiguous")
    if x.dtype != dtype:
        raise RuntimeError(f"attention_from_host: {name} must be {dtype}, got {x.dtype}")
    if shape is not None and tuple(x.shape) != tuple(shape):
        raise RuntimeError(f"attention_from_host: {name} must have shape {tuple(shape)}, "
                           f"got {tuple(x.shape)}")


def attention_from_host(q, k, v, past_len=0, out=None, lse=None, slices=8, device=None):
    """Causal BF16 attention of pinned host tensors q (B,H,Tq,64), k and v (B,H,Tk,64), with
    ``Tk == past_len + Tq`` as in :func:`student.attention`; returns host ``(O, LSE)``: O bf16
    (B,H,Tq,64), LSE fp32 (B,H,Tq), natural log, written into ``out`` / ``lse`` when given
    (pinned, contiguous, of those shapes and dtypes) or into new pinned tensors.

    The (batch, head) rows are processed in ``slices`` groups on ``device`` (default: the
    current CUDA device). The call returns once all work is queued; the caller's current stream
    is ordered after the last output copy, so O and LSE are complete once that stream has
    reached this point (``torch.cuda.current_stream().synchronize()``). Device memory: one
    device copy of q, k and v, plus O and LSE of one slice at a time per slice in flight.
    """
    # Shapes and the operator's own checks first: nothing is allocated or queued for a call
    # that the operator would reject.
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("attention_from_host: q, k, v must be 4-D (B, H, T, 64)")
    B, H, Tq, D = q.shape
    if tuple(k.shape[:2]) != (B, H) or k.shape != v.shape or k.shape[3] != D:
        raise RuntimeError("attention_from_host: k and v must be (B, H, Tk, D) with q's B, H, D")
    Tk = k.shape[2]
    if D != 64:
        raise RuntimeError("attention_from_host: attention currently supports only head_dim=64")
    if int(past_len) < 0:
        raise RuntimeError("attention_from_host: past_len must be non-negative")
    if Tk < Tq or int(past_len) != Tk - Tq:
        raise RuntimeError("attention_from_host: expected Tk == past_len + Tq")
    for name, x in (("q", q), ("k", k), ("v", v)):
        _check_host(name, x)
    if out is None:
        out = torch.empty((B, H, Tq, D), dtype=torch.bfloat16, pin_memory=True)
    else:
        _check_host("out", out, (B, H, Tq, D))
    if lse is None:
        lse = torch.empty((B, H, Tq), dtype=torch.float32, pin_memory=True)
    else:
        _check_host("lse", lse, (B, H, Tq), torch.float32)
    if int(slices) < 1:
        raise RuntimeError("attention_from_host: slices must be at least 1")
    device = torch.device("cuda" if device is None else device)
    if device.type != "cuda":
        raise RuntimeError("attention_from_host: device must be a CUDA device")
    if device.index is None:
        # "cuda" without an index means the current device; the side streams are per index.
        device = torch.device("cuda", torch.cuda.current_device())

    rows = B * H
    n_slices = min(int(slices), rows)
    bounds = [rows * i // n_slices for i in range(n_slices + 1)]
    # (B, H) flattened to one batch row of B*H heads: the same attention per row.
    hq, hk, hv = (x.view(1, rows, x.shape[2], D) for x in (q, k, v))
    ho, hl = out.view(1, rows, Tq, D), lse.view(1, rows, Tq)
    with torch.cuda.device(device), torch.no_grad():
        cur = torch.cuda.current_stream(device)
        h2d, d2h = _side_streams(device)
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        dq, dk, dv = (torch.empty(x.shape, dtype=torch.bfloat16, device=device)
                      for x in (hq, hk, hv))
        for i in range(n_slices):
            r0, r1 = bounds[i], bounds[i + 1]
            with torch.cuda.stream(h2d):
                for d, h in ((dq, hq), (dk, hk), (dv, hv)):
                    d[:, r0:r1].copy_(h[:, r0:r1], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(h2d)
            cur.wait_event(landed)
            o, l = student.attention_with_lse(dq[:, r0:r1], dk[:, r0:r1], dv[:, r0:r1], past_len)
            computed = torch.cuda.Event()
            computed.record(cur)
            d2h.wait_event(computed)
            with torch.cuda.stream(d2h):
                ho[:, r0:r1].copy_(o, non_blocking=True)
                hl[:, r0:r1].copy_(l, non_blocking=True)
            # o and l were allocated on the current stream and are read on d2h.
            o.record_stream(d2h)
            l.record_stream(d2h)
        done = torch.cuda.Event()
        done.record(d2h)
        cur.wait_event(done)
    return out, lse
