"""ctypes loader for the CPU checkers.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs import this module, and only to check or time against the GPU path.

Two libraries:
  * oracle/_build/libxkv_oracle.so -- C restatement of the reference (xkv_oracle.c), always built.
  * oracle/_ref/libkvexp_ref.so    -- the reference's own sources compiled in place by
    `make -C oracle ref` (only where the reference checkout exists; the built .so travels).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libxkv_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkvexp_ref.so")

SCALAR, AVX2, AVX512BF16 = 0, 1, 2

_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_f32p = C.POINTER(C.c_float)


class OracleError(Exception):
    """A failure reported by a checker; `code` says which C++ exception the reference threw
    (1 std::invalid_argument, 2 std::runtime_error, 3 std::logic_error)."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def default_ref_root() -> str:
    """The reference checkout: $KVX_REFERENCE_ROOT, else a `reference` directory beside the
    repository."""
    return os.environ.get("KVX_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def build(ref_root: str | None = None) -> None:
    ref_root = ref_root or default_ref_root()
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if os.path.isdir(ref_root):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_ROOT={ref_root}"], check=True)
        # the reference's own test program over the GPU library (needs the library built first)
        subprocess.run(["make", "-s", "-C", HERE, "shimtest", f"REF_ROOT={ref_root}"], check=True)


def _ptr(a, t):
    return None if a is None else a.ctypes.data_as(t)


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.lib = C.CDLL(path)
        self.prefix = prefix
        err = getattr(self.lib, prefix + "last_error")
        err.restype = C.c_char_p
        self._err = err

    def check(self, rc: int) -> None:
        if rc != 0:
            raise OracleError(rc, self._err().decode())


class Oracle(_Lib):
    """The C restatement (xkv_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path, "ox_")
        L = self.lib
        L.ox_encode_bound.restype = C.c_size_t
        L.ox_encode_bound.argtypes = [C.c_int, C.c_int, C.c_int]
        L.ox_encode_bf16.argtypes = [_u16p, C.c_int, C.c_int, C.c_int, _u8p, C.c_size_t,
                                     C.POINTER(C.c_size_t), _u8p]
        L.ox_encode_bf16_modes.argtypes = [_u16p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p,
                                           C.c_size_t, C.POINTER(C.c_size_t), _u8p]
        L.ox_decode_bf16.argtypes = [_u8p, C.c_size_t, C.c_int, C.c_int, _u16p]
        L.ox_attention_decode.argtypes = [_u16p, _u16p, _u16p, _u8p, C.c_size_t, _u8p,
                                          C.c_size_t, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_int]

    def encode(self, kv: np.ndarray, block: int = 128, with_modes: bool = False,
               code_bits=(2, 4)):
        """Encode like kvexp::encode_bf16; code_bits=(2, 3, 4) also allows the 3-bit extension."""
        kv = np.ascontiguousarray(kv, dtype=np.uint16)
        seq, dim = kv.shape
        cap = max(1, self.lib.ox_encode_bound(seq, dim, block))
        out = np.zeros(cap, dtype=np.uint8)
        nb = C.c_size_t(0)
        modes = np.zeros(max(1, (seq + block - 1) // block), dtype=np.uint8)
        mask = sum(1 << b for b in set(code_bits))
        self.check(self.lib.ox_encode_bf16_modes(_ptr(kv, _u16p), seq, dim, block, mask,
                                                 _ptr(out, _u8p), cap, C.byref(nb),
                                                 _ptr(modes, _u8p)))
        blob = out[: nb.value].copy()
        return (blob, modes) if with_modes else blob

    def encode_raw_args(self, kv_ptr, seq, dim, block):
        """Call the encoder with possibly invalid arguments (for error-path parity tests)."""
        out = np.zeros(16, dtype=np.uint8)
        nb = C.c_size_t(0)
        self.check(self.lib.ox_encode_bf16(kv_ptr, seq, dim, block, _ptr(out, _u8p), 16,
                                           C.byref(nb), None))

    def decode(self, blob: np.ndarray, seq: int, dim: int) -> np.ndarray:
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        out = np.zeros((seq, dim), dtype=np.uint16)
        self.check(self.lib.ox_decode_bf16(_ptr(blob, _u8p), blob.size, seq, dim,
                                           _ptr(out, _u16p)))
        return out

    def attention(self, q, k=None, v=None, kx=None, vx=None, *, seq, threads=1, split=128):
        q = np.ascontiguousarray(q, dtype=np.uint16)
        n_q, dim = q.shape
        out = np.zeros((n_q, dim), dtype=np.float32)
        k = None if k is None else np.ascontiguousarray(k, dtype=np.uint16)
        v = None if v is None else np.ascontiguousarray(v, dtype=np.uint16)
        kx = None if kx is None else np.ascontiguousarray(kx, dtype=np.uint8)
        vx = None if vx is None else np.ascontiguousarray(vx, dtype=np.uint8)
        self.check(self.lib.ox_attention_decode(
            _ptr(q, _u16p), _ptr(k, _u16p), _ptr(v, _u16p), _ptr(kx, _u8p),
            0 if kx is None else kx.size, _ptr(vx, _u8p), 0 if vx is None else vx.size,
            _ptr(out, _f32p), n_q, dim, seq, threads, split))
        return out


class Reference(_Lib):
    """The reference library itself (oracle/_ref/libkvexp_ref.so)."""

    def __init__(self, path: str = REF_SO):
        super().__init__(path, "ref_")
        L = self.lib
        L.ref_encode.argtypes = [_u16p, C.c_int, C.c_int, C.c_int, C.POINTER(_u8p),
                                 C.POINTER(C.c_size_t)]
        L.ref_free.argtypes = [C.c_void_p]
        L.ref_decode.argtypes = [_u8p, C.c_size_t, C.c_int, C.c_int, _u16p]
        L.ref_attention.argtypes = [C.c_int, _u16p, _u16p, _u16p, _u8p, C.c_size_t, _u8p,
                                    C.c_size_t, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int]
        L.ref_model_heads.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_int]
        a, b = C.c_int(0), C.c_int(0)
        L.ref_detect(C.byref(a), C.byref(b))
        self.avx2, self.avx512_bf16 = bool(a.value), bool(b.value)

    def backends(self):
        out = [SCALAR]
        if self.avx2:
            out.append(AVX2)
        if self.avx512_bf16:
            out.append(AVX512BF16)
        return out

    def encode(self, kv: np.ndarray, block: int = 128) -> np.ndarray:
        kv = np.ascontiguousarray(kv, dtype=np.uint16)
        seq, dim = kv.shape
        p = _u8p()
        nb = C.c_size_t(0)
        self.check(self.lib.ref_encode(_ptr(kv, _u16p), seq, dim, block, C.byref(p),
                                       C.byref(nb)))
        try:
            return np.ctypeslib.as_array(p, shape=(nb.value,)).copy() if nb.value else \
                np.zeros(0, dtype=np.uint8)
        finally:
            self.lib.ref_free(p)

    def decode(self, blob: np.ndarray, seq: int, dim: int) -> np.ndarray:
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        out = np.zeros((seq, dim), dtype=np.uint16)
        self.check(self.lib.ref_decode(_ptr(blob, _u8p), blob.size, seq, dim, _ptr(out, _u16p)))
        return out

    def attention(self, q, k=None, v=None, kx=None, vx=None, *, seq, backend=SCALAR, threads=1,
                  split=128):
        q = np.ascontiguousarray(q, dtype=np.uint16)
        n_q, dim = q.shape
        out = np.zeros((n_q, dim), dtype=np.float32)
        k = None if k is None else np.ascontiguousarray(k, dtype=np.uint16)
        v = None if v is None else np.ascontiguousarray(v, dtype=np.uint16)
        kx = None if kx is None else np.ascontiguousarray(kx, dtype=np.uint8)
        vx = None if vx is None else np.ascontiguousarray(vx, dtype=np.uint8)
        self.check(self.lib.ref_attention(
            backend, _ptr(q, _u16p), _ptr(k, _u16p), _ptr(v, _u16p), _ptr(kx, _u8p),
            0 if kx is None else kx.size, _ptr(vx, _u8p), 0 if vx is None else vx.size,
            _ptr(out, _f32p), n_q, dim, seq, threads, split))
        return out

    def model_heads(self, backend, qs, kxs, vxs, outs, n_q, dim, seq, threads, block=128):
        """One OpenMP model_heads pass over units (lists of numpy arrays, outs filled)."""
        n = len(qs)
        arr = lambda xs: (C.c_void_p * n)(*[x.ctypes.data for x in xs])
        kb = (C.c_size_t * n)(*[x.size for x in kxs])
        vb = (C.c_size_t * n)(*[x.size for x in vxs])
        self.check(self.lib.ref_model_heads(backend, n, arr(qs), arr(kxs), kb, arr(vxs), vb,
                                            arr(outs), n_q, dim, seq, threads, block))


_oracle = None
_ref = None


def oracle() -> Oracle:
    global _oracle
    if _oracle is None:
        _oracle = Oracle()
    return _oracle


def reference():
    """The compiled reference, or None when oracle/_ref was never built."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        _ref = Reference()
    return _ref
