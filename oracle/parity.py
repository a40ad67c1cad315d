"""Parity arithmetic for GPU-vs-reference attention outputs.

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's parity check,
always as the checker of the GPU path, never on it.

Both sides are measured against the exact result: softmax(q K^T) V in float64 over the same BF16
inputs ("truth").  The reference's own FP32 error against it grows with the sequence (its
sequential online softmax adds 32768 terms one at a time into fp32 running sums: about
5e-4 of the output scale at 32K tokens with a flat softmax,
tests/test_oracle.py::test_reference_error_grows_with_length), so a fixed tolerance around the
reference's output either fails a correct GPU result or lets a wrong one through.  The checks
per output element are therefore:

    accuracy:  |gpu - truth| <= tol
    parity:    |gpu - ref|   <= |ref - truth| + tol
    tol = ATOL * scale + RTOL * |truth| + sqrt(D) * u * cond        (u = 2^-24)

scale = the p-weighted mean |v| of the element's column (the natural size of an attention
output).  cond = the p-weighted mean over tokens of S_t * (|v_t| + |truth|), S_t = sum_d |q_d k_td|:
any fp32 evaluation of a score q . k_t is off by about sqrt(D) u S_t (the probabilistic bound of a
D-term dot product), which moves the token's weight by that fraction -- large only when a few
outlier elements make S_t large (unsoftened queries against K with 2^9 outliers).  (Parity
follows from accuracy by the triangle inequality; it is checked anyway, against the reference's
actual output.)  The GPU's own error is about 1e-6 of the scale at 32K tokens with softened
queries: the P weights enter its tensor cores exactly (three bf16 terms carry all 24 bits of the
fp32 weight) and each warp's running sums cover only its share of the tiles.
"""
from __future__ import annotations

import numpy as np

ATOL = 2e-5
RTOL = 2e-5


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


class Exact:
    """The float64 result of one attention output block and what its tolerance needs."""

    def __init__(self, truth, scale, cond, dim):
        self.truth, self.scale, self.cond, self.dim = truth, scale, cond, dim

    def __iter__(self):  # (truth, scale), for callers that only need those
        return iter((self.truth, self.scale))


def exact(q, k, v, chunk=1 << 16) -> Exact:
    """softmax(q K^T) V in float64 over all tokens (no scaling), with its scale and cond (see the
    module docstring); q [G, D], k / v [S, D] as bf16 bits."""
    qf = bf16_to_f64(q)
    qa = np.abs(qf)
    p = _softmax_weights(q, k, chunk)
    g, d = p.shape[0], v.shape[1]
    acc = np.zeros((g, d))
    mag = np.zeros((g, d))
    cv = np.zeros((g, d))
    cs = np.zeros((g, 1))
    for t0 in range(0, v.shape[0], chunk):
        vf = bf16_to_f64(v[t0:t0 + chunk])
        pc = p[:, t0:t0 + chunk]
        ps = pc * (qa @ np.abs(bf16_to_f64(k[t0:t0 + chunk])).T)  # p_t S_t
        acc += pc @ vf
        mag += pc @ np.abs(vf)
        cv += ps @ np.abs(vf)
        cs += ps.sum(axis=1, keepdims=True)
    den = p.sum(axis=1, keepdims=True)
    truth = acc / den
    return Exact(truth, mag / den, (cv + cs * np.abs(truth)) / den, d)


def truth_and_scale(q, k, v, chunk=1 << 16) -> Exact:
    return exact(q, k, v, chunk)


def attention_f64(q, k, v, chunk=1 << 16):
    return exact(q, k, v, chunk).truth


def attn_scale(q, k, v, chunk=1 << 16):
    return exact(q, k, v, chunk).scale


def tolerance(ex: Exact):
    return (ATOL * ex.scale + RTOL * np.abs(ex.truth)
            + np.sqrt(ex.dim) * 2.0 ** -24 * ex.cond)


def measure(gpu, ref, ex: Exact) -> dict:
    """The parity figures of one output block: max over its elements of
    |gpu - truth| / tol (accuracy, <= 1 passes), |gpu - ref| / (|ref - truth| + tol) (parity,
    <= 1 passes), and the errors in units of the scale.  Non-finite GPU outputs count as infinite
    error."""
    g = np.asarray(gpu, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    t = ex.truth
    tol = tolerance(ex)
    sc = np.maximum(ex.scale, 1e-300)
    if not np.all(np.isfinite(g)):
        inf = float("inf")
        return {"accuracy": inf, "parity": inf, "gpu_err_over_scale": inf,
                "ref_err_over_scale": float(np.max(np.abs(r - t) / sc))}
    return {
        "accuracy": float(np.max(np.abs(g - t) / tol)),
        "parity": float(np.max(np.abs(g - r) / (np.abs(r - t) + tol))),
        "gpu_err_over_scale": float(np.max(np.abs(g - t) / sc)),
        "ref_err_over_scale": float(np.max(np.abs(r - t) / sc)),
    }
