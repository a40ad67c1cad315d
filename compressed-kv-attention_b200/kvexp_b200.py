"""Python binding of libkvexp_b200.so (the C ABI in include/kvexp_b200.h).

Mirrors the reference library's public API (namespace kvexp, include/kvexp/*.hpp of
cvs0/compressed-kv-attention): attention_decode, encode_bf16 / decode_bf16 / EncodedTensor,
Backend, plus the GPU-native batched plan.  Arguments may be numpy arrays (host memory), torch
tensors (host or CUDA), raw integer addresses or None.  Errors raise the Python counterpart of the
reference's exception type:

    std::invalid_argument -> ValueError
    std::runtime_error    -> RuntimeError
    std::logic_error      -> LogicError

There is no CPU fallback: importing this module fails when the shared library is missing.
"""
from __future__ import annotations

import ctypes as C
import enum
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libkvexp_b200.so")

KVX_OK = 0
KVX_ERR_INVALID_ARGUMENT = 1
KVX_ERR_RUNTIME = 2
KVX_ERR_LOGIC = 3
KVX_ERR_CUDA = 4
KVX_ERR_TIMEOUT = 5
KVX_ERR_UNSUPPORTED = 6

K_ENCODE_BLOCK = 128   # kEncodeBlock, include/kvexp/bf16.hpp:12
K_MAX_HEAD_DIM = 256   # kMaxHeadDim, include/kvexp/bf16.hpp:13


class Backend(enum.IntEnum):
    """kvexp::Backend (include/kvexp/attention.hpp:10-14).  All values run the GPU kernels; the
    value selects the reference's shape rule and error text."""
    Scalar = 0
    Avx2 = 1
    Avx512Bf16 = 2


class LogicError(Exception):
    """std::logic_error of the reference (encoder size-model drift)."""


class CudaError(RuntimeError):
    """A CUDA runtime call inside the library failed."""


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait expired (the kernel returned instead of hanging)."""


if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with "
                      "`python compressed-kv-attention_b200/build.py` (there is no CPU fallback)")

_lib = C.CDLL(LIB_PATH)

_vp = C.c_void_p
_sz = C.c_size_t


class kvx_block(C.Structure):
    _fields_ = [("offset", C.c_uint32), ("n_escape", C.c_uint16), ("mode", C.c_uint8),
                ("n_tokens", C.c_uint8)]


class kvx_unit(C.Structure):
    _fields_ = [("k", _vp), ("v", _vp), ("k_index", _vp), ("v_index", _vp), ("q", _vp),
                ("out", _vp), ("k_bytes", C.c_uint64), ("v_bytes", C.c_uint64),
                ("n_blocks", C.c_int32), ("seq", C.c_int32), ("lse", _vp)]


def _sig(name, res, args):
    f = getattr(_lib, name)
    f.restype = res
    f.argtypes = args
    return f


_last_error = _sig("kvx_last_error", C.c_char_p, [])
_version = _sig("kvx_version", C.c_char_p, [])
_device_info = _sig("kvx_device_info", C.c_int, [C.POINTER(C.c_int)] * 3 + [C.POINTER(_sz)])
_attention = _sig("kvx_attention_decode", C.c_int,
                  [C.c_int, _vp, _vp, _vp, _vp, _sz, _vp, _sz, _vp, C.c_int, C.c_int, C.c_int,
                   C.c_int, C.c_int])
_attention_units = _sig("kvx_attention_decode_units", C.c_int,
                        [C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int,
                         C.c_int, C.c_int])
_encode_bound = _sig("kvx_encode_bound", _sz, [C.c_int, C.c_int, C.c_int])
_encode = _sig("kvx_encode_bf16", C.c_int,
               [_vp, C.c_int, C.c_int, C.c_int, _vp, _sz, C.POINTER(_sz)])
_encode_bits = _sig("kvx_encode_bf16_bits", C.c_int,
                    [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _sz, C.POINTER(_sz)])
_decode = _sig("kvx_decode_bf16", C.c_int, [_vp, _sz, C.c_int, C.c_int, _vp])
_xkv_index = _sig("kvx_xkv_index", C.c_int,
                  [_vp, _sz, C.c_int, _vp, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_longlong)])
_plan_create = _sig("kvx_plan_create", C.c_int,
                    [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)])
_plan_run = _sig("kvx_plan_run", C.c_int, [_vp, _vp])
_plan_run_part = _sig("kvx_plan_run_part", C.c_int, [_vp, C.c_int, _vp])
_plan_check = _sig("kvx_plan_check", C.c_int, [_vp])
_plan_launches = _sig("kvx_plan_launches", C.c_int, [_vp])
_plan_split = _sig("kvx_plan_split_units", C.c_int, [_vp])
_plan_destroy = _sig("kvx_plan_destroy", None, [_vp])
_enc_bounds = _sig("kvx_encode_batch_bounds", C.c_int,
                   [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_sz), C.POINTER(_sz)])
_enc_batch = _sig("kvx_encode_batch", C.c_int,
                  [C.c_int, _vp, C.c_int, C.c_int, C.c_int, _vp, _sz, _vp, _vp, _vp, _vp])
_enc_batch_bits = _sig("kvx_encode_batch_bits", C.c_int,
                       [C.c_int, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _sz, _vp, _vp,
                        _vp, _vp])
_append_bits = _sig("kvx_cache_append_bits", C.c_int,
                    [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _sz, _sz, _vp,
                     C.POINTER(_sz), C.POINTER(C.c_int), _vp])
_append = _sig("kvx_cache_append", C.c_int,
               [_vp, C.c_int, C.c_int, C.c_int, _vp, _sz, _sz, _vp, C.POINTER(_sz),
                C.POINTER(C.c_int), _vp])
_synth = _sig("kvx_synth_bf16", C.c_int,
              [_vp, C.c_int, C.c_int, C.c_uint64, C.c_uint64, C.c_int, C.c_uint32, _vp])
_probe = _sig("kvx_hbm_read_probe", C.c_int, [_vp, _sz, C.c_int, C.POINTER(C.c_double)])
_noalloc = _sig("kvx_attention_decode_noalloc", C.c_int,
                [_vp, _vp, _sz, _vp, _vp, _sz, _vp, C.c_int, _vp, C.c_int, C.c_int, C.c_int, _vp])
_fold = _sig("kvx_fold_shards", C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp])
_expstats = _sig("kvx_exponent_stats", C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp])

# Every symbol the C header declares, for load/export checks.
EXPORTED = [
    "kvx_last_error", "kvx_version", "kvx_device_info", "kvx_attention_decode",
    "kvx_attention_decode_units", "kvx_encode_bound", "kvx_encode_bf16", "kvx_decode_bf16",
    "kvx_xkv_index", "kvx_plan_create", "kvx_plan_run", "kvx_plan_run_part", "kvx_plan_check", "kvx_plan_launches", "kvx_plan_split_units",
    "kvx_plan_destroy", "kvx_encode_batch_bounds", "kvx_encode_batch", "kvx_cache_append",
    "kvx_synth_bf16", "kvx_hbm_read_probe", "kvx_attention_decode_noalloc", "kvx_fold_shards",
    "kvx_exponent_stats", "kvx_encode_bf16_bits", "kvx_encode_batch_bits", "kvx_cache_append_bits",
]

# Residual code widths the encoder may use (include/kvexp_b200.h KVX_CODE_BITS_*): the reference's
# {2, 4}, or with the library's 3-bit extension.
CODE_BITS_REFERENCE = 0x14
CODE_BITS_ALL = 0x1C


def _check(rc: int) -> None:
    if rc == KVX_OK:
        return
    msg = (_last_error() or b"").decode()
    if rc == KVX_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == KVX_ERR_LOGIC:
        raise LogicError(msg)
    if rc == KVX_ERR_CUDA:
        raise CudaError(msg)
    if rc == KVX_ERR_TIMEOUT:
        raise DeviceTimeout(msg)
    if rc == KVX_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def _addr(x):
    """Address of a numpy array / torch tensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays must be C-contiguous")
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return x.data_ptr()
    raise TypeError(f"unsupported buffer type {type(x)!r}")


def _nbytes(x):
    if isinstance(x, np.ndarray):
        return x.nbytes
    if hasattr(x, "data_ptr"):
        return x.numel() * x.element_size()
    raise TypeError("size unknown for raw addresses; pass the byte count")


def version() -> str:
    return _version().decode()


def device_info() -> dict:
    a, b, n = C.c_int(0), C.c_int(0), C.c_int(0)
    mem = _sz(0)
    _check(_device_info(C.byref(a), C.byref(b), C.byref(n), C.byref(mem)))
    return {"sm": (a.value, b.value), "sm_count": n.value, "hbm_bytes": mem.value}


def attention_decode(backend, q, k_raw, v_raw, k_xkv, k_bytes, v_xkv, v_bytes, out, n_q, dim,
                     seq, n_threads, split_tokens=K_ENCODE_BLOCK):
    """kvexp::attention_decode (include/kvexp/attention.hpp:58-61), run on the GPU."""
    _check(_attention(int(backend), _addr(q), _addr(k_raw), _addr(v_raw), _addr(k_xkv),
                      int(k_bytes), _addr(v_xkv), int(v_bytes), _addr(out), int(n_q), int(dim),
                      int(seq), int(n_threads), int(split_tokens)))


def attention_decode_units(backend, qs, kxs, k_bytes, vxs, v_bytes, outs, n_q, dim, seq,
                           split_tokens=K_ENCODE_BLOCK):
    """All (layer, KV head) units of a step in one GPU job (the reference's model_heads loop)."""
    n = len(qs)
    arr = lambda xs: (C.c_void_p * n)(*[_addr(x) for x in xs])
    kb = (_sz * n)(*[int(b) for b in k_bytes])
    vb = (_sz * n)(*[int(b) for b in v_bytes])
    _check(_attention_units(int(backend), n, arr(qs), arr(kxs), kb, arr(vxs), vb, arr(outs),
                            int(n_q), int(dim), int(seq), int(split_tokens)))


class EncodedTensor:
    """kvexp::EncodedTensor (include/kvexp/codec.hpp:38-43): bytes (numpy uint8) + shape."""

    def __init__(self, data, seq_len, head_dim, block_tokens):
        self.bytes = data
        self.seq_len = seq_len
        self.head_dim = head_dim
        self.block_tokens = block_tokens


def encode_bound(seq_len, head_dim, block_tokens=K_ENCODE_BLOCK) -> int:
    return int(_encode_bound(int(seq_len), int(head_dim), int(block_tokens)))


def encode_bf16(kv, seq_len, head_dim, block_tokens=K_ENCODE_BLOCK,
                code_bits=CODE_BITS_REFERENCE) -> EncodedTensor:
    """kvexp::encode_bf16 (include/kvexp/codec.hpp:45-46) on the GPU; byte-identical output.
    code_bits=CODE_BITS_ALL also allows 3-bit blocks (the library's extension)."""
    cap = max(16, encode_bound(seq_len, head_dim, block_tokens))
    out = np.zeros(cap, dtype=np.uint8)
    nb = _sz(0)
    if code_bits == CODE_BITS_REFERENCE:
        _check(_encode(_addr(kv), int(seq_len), int(head_dim), int(block_tokens), out.ctypes.data,
                       cap, C.byref(nb)))
    else:
        _check(_encode_bits(_addr(kv), int(seq_len), int(head_dim), int(block_tokens),
                            int(code_bits), out.ctypes.data, cap, C.byref(nb)))
    return EncodedTensor(out[: nb.value].copy(), seq_len, head_dim, block_tokens)


def decode_bf16(blob, nbytes, seq_len, head_dim, out):
    """kvexp::decode_bf16 (include/kvexp/codec.hpp:48) on the GPU."""
    _check(_decode(_addr(blob), int(nbytes), int(seq_len), int(head_dim), _addr(out)))


def xkv_index(blob, nbytes, head_dim, index, max_blocks):
    """Block index of a device blob into device memory `index`; returns (n_blocks, n_tokens)."""
    nb, nt = C.c_int(0), C.c_longlong(0)
    _check(_xkv_index(_addr(blob), int(nbytes), int(head_dim), _addr(index), int(max_blocks),
                      C.byref(nb), C.byref(nt)))
    return nb.value, nt.value


def attention_decode_noalloc(q, k_xkv, k_bytes, k_index, v_xkv, v_bytes, v_index, n_blocks, out,
                             n_q, dim, seq, stream=None):
    """One decode step over device-resident XKV K/V that allocates no GPU memory (for callers
    whose device memory is all reserved up front; see kvx_attention_decode_noalloc).  Every
    argument is device memory; the indexes come from xkv_index or the GPU encoder."""
    _check(_noalloc(_addr(q), _addr(k_xkv), int(k_bytes), _addr(k_index), _addr(v_xkv),
                    int(v_bytes), _addr(v_index), int(n_blocks), _addr(out), int(n_q), int(dim),
                    int(seq), _addr(stream)))


def fold_shards(parts, n_parts, n_rows, dim, out, lse_out=None, stream=None):
    """Rank-ordered fold of sequence-shard results on the GPU (kvx_fold_shards): parts holds
    n_parts blocks of [n_rows * dim outputs, n_rows lse] FP32; asynchronous on `stream`."""
    _check(_fold(_addr(parts), int(n_parts), int(n_rows), int(dim), _addr(out), _addr(lse_out),
                 stream))


class Plan:
    """A reusable batched decode step (kvx_plan): fixed units, one launch (+ combine) per run."""

    def __init__(self, units, n_q, dim, block_tokens=K_ENCODE_BLOCK):
        arr = (kvx_unit * len(units))(*units)
        h = _vp()
        _check(_plan_create(C.cast(arr, _vp), len(units), int(n_q), int(dim), int(block_tokens),
                            C.byref(h)))
        self._h = h

    def run(self, stream=None):
        _check(_plan_run(self._h, stream))

    def run_part(self, part, stream=None):
        _check(_plan_run_part(self._h, int(part), stream))

    @property
    def n_split(self) -> int:
        return int(_plan_split(self._h))

    def check(self):
        _check(_plan_check(self._h))

    @property
    def launches(self) -> int:
        return int(_plan_launches(self._h))

    def close(self):
        if self._h:
            _plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def make_unit(k, v, q, out, *, k_index=None, v_index=None, k_bytes=0, v_bytes=0, n_blocks=0,
              seq, lse=None) -> kvx_unit:
    return kvx_unit(_addr(k), _addr(v), _addr(k_index), _addr(v_index), _addr(q), _addr(out),
                    int(k_bytes), int(v_bytes), int(n_blocks), int(seq), _addr(lse))


def encode_batch_bounds(n_tensors, seq, head_dim, block_tokens=K_ENCODE_BLOCK):
    a, b = _sz(0), _sz(0)
    _check(_enc_bounds(int(n_tensors), int(seq), int(head_dim), int(block_tokens), C.byref(a),
                       C.byref(b)))
    return a.value, b.value


def encode_batch(tensors, seq, head_dim, arena, index, block_tokens=K_ENCODE_BLOCK,
                 stream=None, code_bits=CODE_BITS_REFERENCE):
    """GPU-encode device tensors into `arena`; returns (blob_offsets, blob_bytes) numpy arrays."""
    n = len(tensors)
    ptrs = (C.c_void_p * n)(*[_addr(t) for t in tensors])
    off = np.zeros(n, dtype=np.uint64)
    nb = np.zeros(n, dtype=np.uint64)
    if code_bits == CODE_BITS_REFERENCE:
        _check(_enc_batch(n, C.cast(ptrs, _vp), int(seq), int(head_dim), int(block_tokens),
                          _addr(arena), _nbytes(arena), _addr(index), off.ctypes.data,
                          nb.ctypes.data, stream))
    else:
        _check(_enc_batch_bits(n, C.cast(ptrs, _vp), int(seq), int(head_dim), int(block_tokens),
                               int(code_bits), _addr(arena), _nbytes(arena), _addr(index),
                               off.ctypes.data, nb.ctypes.data, stream))
    return off, nb


def cache_append(kv_new, n_new, head_dim, blob, at, capacity, index,
                 block_tokens=K_ENCODE_BLOCK, stream=None, code_bits=CODE_BITS_REFERENCE):
    """Encode n_new tokens and append them at byte `at` of a device blob; returns
    (bytes_written, blocks_written)."""
    bw, kw = _sz(0), C.c_int(0)
    if code_bits == CODE_BITS_REFERENCE:
        _check(_append(_addr(kv_new), int(n_new), int(head_dim), int(block_tokens), _addr(blob),
                       int(at), int(capacity), _addr(index), C.byref(bw), C.byref(kw), stream))
    else:
        _check(_append_bits(_addr(kv_new), int(n_new), int(head_dim), int(block_tokens),
                            int(code_bits), _addr(blob), int(at), int(capacity), _addr(index),
                            C.byref(bw), C.byref(kw), stream))
    return bw.value, kw.value


def synth_bf16(out, seq, dim, seed, stream_id, profile, rate, stream=None):
    _check(_synth(_addr(out), int(seq), int(dim), int(seed), int(stream_id), int(profile),
                  int(rate), stream))


def hbm_read_probe(buf, nbytes=None, reps=10) -> float:
    g = C.c_double(0)
    _check(_probe(_addr(buf), int(nbytes if nbytes is not None else _nbytes(buf)), int(reps),
                  C.byref(g)))
    return g.value


def exponent_stats(kv, seq_len, head_dim, block_tokens=K_ENCODE_BLOCK):
    """kvx_exponent_stats on a [seq_len, head_dim] BF16 tensor (host numpy or a device tensor):
    returns (best [3, n_blocks, head_dim] int32 for windows of 3 / 7 / 15 exponents,
    entropy [n_blocks, head_dim] float32)."""
    nb = (int(seq_len) + int(block_tokens) - 1) // int(block_tokens)
    best = np.zeros((3, nb, int(head_dim)), dtype=np.int32)
    ent = np.zeros((nb, int(head_dim)), dtype=np.float32)
    _check(_expstats(_addr(kv), int(seq_len), int(head_dim), int(block_tokens), best.ctypes.data,
                     ent.ctypes.data))
    return best, ent


def exponent_report(kv, seq_len, head_dim, block_tokens=K_ENCODE_BLOCK, bit_widths=(2, 3, 4)):
    """The reference analyser's per-tensor report from the GPU statistics: the size policy
    (python/analyze_exponents.py:117-156 `policy_size`: per block the smallest of the raw
    container and each residual width, ties to raw, then fewer escapes, then narrower codes) and
    the mean entropy of the exponent in each (full block, dim) (`block_conditional_entropy`,
    :57-72; nan when there is no full block)."""
    seq, dim, bt = int(seq_len), int(head_dim), int(block_tokens)
    best, ent = exponent_stats(kv, seq, dim, bt)
    col = {2: 0, 3: 1, 4: 2}
    total = 0
    esc_total = 0
    coded = 0
    modes = {}
    for b in range(best.shape[1]):
        n = min(bt, seq - b * bt)
        options = [(0, 8 + 2 * n * dim, 0)]
        for bits in bit_widths:
            n_esc = n * dim - int(best[col[bits], b].sum())
            options.append((bits, 8 + dim + n * dim + (n * dim * bits + 7) // 8 + 2 * n_esc, n_esc))
        mode, size, n_esc = min(options, key=lambda t: (t[1], 0 if t[0] == 0 else 1, t[2], t[0]))
        total += size
        esc_total += n_esc
        modes[mode] = modes.get(mode, 0) + 1
        if mode != 0:
            coded += n * dim
    full = seq // bt
    tight = 2 * seq * dim
    return {
        "container_bytes": total, "tight_bytes": tight, "ratio": total / tight,
        "escape_rate": esc_total / (seq * dim), "coded_element_fraction": coded / (seq * dim),
        "mode_blocks": {str(k): v for k, v in sorted(modes.items())},
        "block_conditional_entropy": float(ent[:full].astype(np.float64).mean()) if full else float("nan"),
    }
