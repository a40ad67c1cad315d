"""The reference's own test program, unmodified, on the GPU library.

oracle/_ref/kvexp_tests_gpu is the reference's tests/test_main.cpp compiled from its source and
linked, through the drop-in shim (compressed-kv-attention_b200/shim/kvexp_gpu_shim.cpp), against
libkvexp_b200.so instead of the reference's dispatch.cpp / codec.cpp / cpu.cpp (built by
`make -C oracle shimtest` where the reference checkout exists; the binary travels with the
repository).  Its checks: lossless round trip with signed zeros, subnormals, infinities and NaN;
container sizes; the identity token (out == v exactly) at head_dim 8; raw and XKV outputs
bit-identical per backend over the reference's shape matrix (head_dim 16 to 64, 1 to 300 tokens,
blocks of 16 to 128, 1 and 4 threads), and Scalar == AVX2 at one thread.  It prints "ok".
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "kvexp_tests_gpu")


def test_reference_test_program_passes(kvx, cuda):
    if not os.path.exists(BIN):
        pytest.skip("oracle/_ref/kvexp_tests_gpu was not built (no reference checkout at build time)")
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout, r.stderr)
