"""CPU checks of the C ABI (include/kvexp_b200.h) -- no GPU needed.

The library must load, export every entry point the header declares (the Python binding lists
the same set), and mirror the reference's argument errors (same exception kind and message)
before it touches a device: these checks run ahead of any CUDA call.
"""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kvexp_b200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"KVX_API\s+[\w\s\*]+?\b(kvx_\w+)\s*\(", text)))


def test_header_lists_the_drop_in_entry_points():
    syms = header_symbols()
    for s in ("kvx_attention_decode", "kvx_encode_bf16", "kvx_decode_bf16", "kvx_device_info",
              "kvx_plan_create", "kvx_plan_run", "kvx_attention_decode_noalloc"):
        assert s in syms


def test_library_exports_every_header_symbol(kvx):
    lib = C.CDLL(kvx.LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", kvx.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (kvx_\w+)", out))
    assert set(header_symbols()) <= exported
    assert sorted(kvx.EXPORTED) == header_symbols()


@pytest.mark.parametrize("seq,dim,block", [(1, 64, 128), (1000, 64, 128), (219, 128, 32),
                                           (5, 256, 1), (300, 8, 255)])
def test_encode_bound_matches_oracle(kvx, oracle, seq, dim, block):
    assert kvx.encode_bound(seq, dim, block) == oracle.lib.ox_encode_bound(seq, dim, block)


def _ref_error(fn):
    with pytest.raises(Exception) as e:
        fn()
    return e.value


@pytest.mark.parametrize("case", ["null_q", "both", "neither", "backend", "scalar_dim",
                                  "avx512_dim", "seq0", "split0"])
def test_attention_argument_errors_mirror_the_reference(kvx, reference_or_none, case):
    dim, n_q, seq = 64, 2, 16
    q = np.zeros((n_q, dim), dtype=np.uint16)
    k = np.zeros((seq, dim), dtype=np.uint16)
    kx = np.zeros(64, dtype=np.uint8)
    out = np.zeros((n_q, dim), dtype=np.float32)
    args = dict(backend=0, q=q, k=k, v=k, kx=None, vx=None, n_q=n_q, dim=dim, seq=seq, split=128)
    if case == "null_q":
        args["q"] = None
    elif case == "both":
        args.update(kx=kx, vx=kx)
    elif case == "neither":
        args.update(k=None, v=None)
    elif case == "backend":
        args["backend"] = 7
    elif case == "scalar_dim":
        args.update(dim=12)
    elif case == "avx512_dim":
        args.update(backend=2, dim=48)
    elif case == "seq0":
        args["seq"] = 0
    elif case == "split0":
        args["split"] = 0
    a = args
    err = _ref_error(lambda: kvx.attention_decode(
        a["backend"], a["q"], a["k"], a["v"], a["kx"], 0 if a["kx"] is None else a["kx"].size,
        a["vx"], 0 if a["vx"] is None else a["vx"].size, out, a["n_q"], a["dim"], a["seq"], 1,
        a["split"]))
    assert isinstance(err, ValueError), err  # std::invalid_argument in the reference
    if reference_or_none is not None and case not in ("null_q", "backend"):
        qq = np.zeros((n_q, a["dim"]), dtype=np.uint16)
        kk = None if a["k"] is None else np.zeros((seq, a["dim"]), dtype=np.uint16)
        with pytest.raises(O.OracleError) as r:
            reference_or_none.attention(qq, k=kk, v=kk, kx=a["kx"], vx=a["vx"], seq=a["seq"],
                                        backend=a["backend"], threads=1, split=a["split"])
        assert r.value.code == 1
        assert str(r.value) == str(err)


@pytest.mark.parametrize("seq,dim,block", [(0, 64, 128), (16, 6, 128), (16, 260, 128),
                                           (16, 64, 256), (16, 64, 0)])
def test_encode_argument_errors_mirror_the_reference(kvx, oracle, seq, dim, block):
    x = np.zeros((max(seq, 1), dim), dtype=np.uint16)
    with pytest.raises(ValueError) as e:
        kvx.encode_bf16(x, seq, dim, block)
    with pytest.raises(O.OracleError) as r:
        oracle.encode_raw_args(x.ctypes.data_as(O._u16p), seq, dim, block)
    assert r.value.code == 1
    assert str(e.value) == str(r.value)


def test_shim_compiles_against_reference_headers():
    """The drop-in shim (the reference's kvexp:: API over the C ABI) compiles against the
    reference's own public headers, where a reference checkout is present."""
    import subprocess
    import oracle as O
    ref = O.default_ref_root()
    if not os.path.isdir(os.path.join(ref, "include", "kvexp")):
        pytest.skip("no reference checkout on this host")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    shim = os.path.join(root, "compressed-kv-attention_b200", "shim", "kvexp_gpu_shim.cpp")
    subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-Wall", "-Werror",
                    "-I" + os.path.join(ref, "include"), "-I" + os.path.join(root, "include"), shim],
                   check=True)
