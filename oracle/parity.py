"""Parity arithmetic for GPU-vs-reference attention outputs.

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's parity check,
always as the checker of the GPU path, never on it.

The tolerance (per output element):

    |gpu - ref| <= ATOL_REL * sqrt(max(1, seq / 64)) * scale + RTOL * |ref|

scale = the p-weighted mean |v| of the element's column (attn_scale), the natural size of an
attention output.  The two sides differ in expf implementations (glibc on the CPU, the SFU's
exp2 on the GPU), in accumulation order (the reference's sequential online softmax with 8-lane
FMA chains, against tensor-core tiles and a split-K fold) -- the P weights themselves enter the
GPU's tensor cores exactly (three bf16 terms carry all 24 bits of the fp32 weight).  The
reference's own fp32 error against a float64 softmax grows with the sequence like sqrt(seq)
(tests/test_oracle.py::test_reference_error_grows_with_length measures it), which is what the
length factor covers.
"""
from __future__ import annotations

import numpy as np

ATOL_REL = 2e-5
RTOL = 1e-4


def bf16_to_f64(x):
    return (np.asarray(x, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _softmax_weights(q, k, chunk=1 << 16):
    """exp(s - max s) for s = q K^T (float64), [n_q, seq]; K is bf16 bits [seq, dim]."""
    qf = bf16_to_f64(q)
    seq = k.shape[0]
    s = np.empty((qf.shape[0], seq), dtype=np.float64)
    for t0 in range(0, seq, chunk):
        s[:, t0:t0 + chunk] = qf @ bf16_to_f64(k[t0:t0 + chunk]).T
    s -= s.max(axis=1, keepdims=True)
    return np.exp(s)


def attention_f64(q, k, v, chunk=1 << 16):
    """Float64 softmax(q K^T) V over all tokens (no scaling), q [G,D], k/v [S,D] bf16 bits."""
    p = _softmax_weights(q, k, chunk)
    acc = np.zeros((p.shape[0], v.shape[1]), dtype=np.float64)
    for t0 in range(0, v.shape[0], chunk):
        acc += p[:, t0:t0 + chunk] @ bf16_to_f64(v[t0:t0 + chunk])
    return acc / p.sum(axis=1, keepdims=True)


def attn_scale(q, k, v, chunk=1 << 16):
    """Per query and column: the p-weighted mean of |v| -- the natural scale of an output."""
    p = _softmax_weights(q, k, chunk)
    acc = np.zeros((p.shape[0], v.shape[1]), dtype=np.float64)
    for t0 in range(0, v.shape[0], chunk):
        acc += p[:, t0:t0 + chunk] @ np.abs(bf16_to_f64(v[t0:t0 + chunk]))
    return acc / p.sum(axis=1, keepdims=True)


def tolerance(ref, scale, seq):
    return ATOL_REL * np.sqrt(max(1.0, seq / 64.0)) * scale + RTOL * np.abs(ref)


def err_over_tol(got, ref, scale, seq) -> float:
    """max |got - ref| / tolerance: <= 1 passes.  Non-finite outputs count as infinite error."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if not np.all(np.isfinite(got)):
        return float("inf")
    return float(np.max(np.abs(got - ref) / tolerance(ref, scale, seq)))


def err_over_scale(got, ref, scale) -> float:
    """max |got - ref| / scale (the error in units of the output's natural size)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref) / np.maximum(scale, 1e-300)))
