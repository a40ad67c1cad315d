"""Test data generators and numeric references (test infrastructure only)."""
import numpy as np

from parity import (ATOL, RTOL, attention_f64, attn_scale, bf16_to_f64, exact,  # noqa: F401
                    measure, tolerance, truth_and_scale)


class XorShift32:
    """The reference tests' RNG (tests/test_main.cpp:26-32), seeded 0x12345678."""

    def __init__(self, seed=0x12345678):
        self.s = seed & 0xFFFFFFFF

    def __call__(self):
        s = self.s
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        self.s = s
        return s


def make_bf16(exp, mant, sign):
    return ((0x8000 if sign else 0) | ((exp & 0xFF) << 7) | (mant & 0x7F)) & 0xFFFF


def clustered(rng, n, base, spread):
    """Exponents base + U[0, spread), 1 in 200 at base + 80 (tests/test_main.cpp:38-48)."""
    out = np.zeros(n, dtype=np.uint16)
    for i in range(n):
        e = base + rng() % spread
        if rng() % 200 == 0:
            e = (base + 80) & 0xFF
        mant = rng() & 0x7F
        sign = rng() & 1
        out[i] = make_bf16(e, mant, sign)
    return out


def mixed_modes(seq, dim, block, seed=7):
    """BF16 bits whose blocks favour every mode of the {raw, 2, 3, 4}-bit policy in turn: block b
    draws its exponents per channel from a window of 3, 7, 15 or 64 values (2-bit, 3-bit, 4-bit,
    raw), with a few outliers and the special classes (+-0, subnormals, +-inf, NaN)."""
    rng = np.random.default_rng(seed)
    spreads = (3, 7, 15, 64)
    x = np.empty((seq, dim), dtype=np.uint16)
    for b0 in range(0, seq, block):
        n = min(block, seq - b0)
        spread = spreads[(b0 // block) % len(spreads)]
        base = rng.integers(100, 130, size=dim)
        e = base[None, :] + rng.integers(0, spread, size=(n, dim))
        out = rng.random((n, dim)) < 0.01
        e[out] = rng.integers(1, 255, size=int(out.sum()))
        x[b0:b0 + n] = ((rng.integers(0, 2, size=(n, dim)) << 15) | ((e & 0xFF) << 7) |
                        rng.integers(0, 128, size=(n, dim))).astype(np.uint16)
    specials = np.array([0x0000, 0x8000, 0x0001, 0x807F, 0x7F80, 0xFF80, 0x7FC0, 0xFFC1],
                        dtype=np.uint16)
    flat = x.reshape(-1)
    flat[::211] = specials[np.arange(flat[::211].size) % specials.size]
    return x


def assert_attention_close(gpu, ref, q=None, k=None, v=None, what="", truth=None):
    """The GPU output against the float64 truth and the reference's output (oracle/parity.py):
    per element |gpu - truth| <= tol and |gpu - ref| <= |ref - truth| + tol.  `truth` = the
    parity.Exact of the block when already computed, else computed from q, k, v (BF16 bits)."""
    ex = truth if truth is not None else exact(q, k, v)
    t, sc = ex.truth, ex.scale
    g = np.asarray(gpu, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    tol = tolerance(ex)
    bad = ~(np.abs(g - t) <= tol) | ~(np.abs(g - r) <= np.abs(r - t) + tol)
    if bad.any():
        i = tuple(np.argwhere(bad)[0])
        with np.errstate(invalid="ignore"):
            gerr = np.max(np.abs(g - t) / np.maximum(sc, 1e-300))
            rerr = np.max(np.abs(r - t) / np.maximum(sc, 1e-300))
        raise AssertionError(
            f"{what}: {bad.sum()} of {bad.size} elements out of tolerance; first {i}: "
            f"gpu={g[i]!r} ref={r[i]!r} truth={t[i]!r} tol={tol[i]!r}; "
            f"max |gpu-truth|/scale={gerr:.3e}, max |ref-truth|/scale={rerr:.3e}")


def soften(q, shift=4):
    """Scale bf16 queries by 2**-shift (exponent arithmetic) for a flatter softmax."""
    q = np.asarray(q, dtype=np.uint16)
    e = (q >> 7) & 0xFF
    e2 = np.where(e > shift, e - shift, e)
    return ((q & 0x807F) | (e2 << 7)).astype(np.uint16)
