#!/usr/bin/env python
"""Write tests/golden/golden.json from the reference library itself.

The reference (kvexp) is compiled from its own sources into oracle/_ref/libkvexp_ref.so by
`make -C oracle ref` (oracle/Makefile).  For every case below this script regenerates the seeded
inputs with synth.py, encodes them with the reference encoder (`kvexp::encode_bf16`) and runs the
reference attention (`kvexp::attention_decode`, scalar backend and, where the host has it, AVX2),
then stores the blob hashes and sizes, the block-mode histograms and the output bits.  The tests
in tests/test_oracle.py check the C restatement in oracle/ against these fixtures, so the oracle
stays pinned to the reference on machines where the reference cannot be built.

    python tests/golden/make_golden.py
"""
import base64
import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "compressed-kv-attention_b200"),
                os.path.join(ROOT, "tests")]
import oracle as O  # noqa: E402
import synth as S  # noqa: E402
from golden_cases import CASES, inputs  # noqa: E402


def modes(blob):
    """Block modes of a blob by walking its headers (include/kvexp/codec.hpp:18-31)."""
    out, off = [], 0
    while off < blob.size:
        mode, nt, ne, hd, _ = struct.unpack_from("<BBHHH", blob, off)
        out.append(int(mode))
        off += 8 + (2 * nt * hd if mode == 0 else hd + nt * hd + (nt * hd * mode + 7) // 8 + 2 * ne)
    return {str(m): out.count(m) for m in (0, 2, 4)}


def b64(a):
    return base64.b64encode(np.ascontiguousarray(a).tobytes()).decode()


def main():
    ref = O.reference()
    if ref is None:
        sys.exit("oracle/_ref/libkvexp_ref.so is missing: run `make -C oracle ref` first")
    out = {"generator": "tests/golden/make_golden.py", "reference": "kvexp built from its sources",
           "cases": {}}
    exact = elems = 0
    for name, c in CASES.items():
        q, k, v = inputs(c)
        kx = ref.encode(k, c["block"])
        vx = ref.encode(v, c["block"])
        assert np.array_equal(ref.decode(kx, c["seq"], c["dim"]), k)
        assert np.array_equal(ref.decode(vx, c["seq"], c["dim"]), v)
        e = {"k_bytes": int(kx.size), "v_bytes": int(vx.size),
             "k_sha256": hashlib.sha256(kx.tobytes()).hexdigest(),
             "v_sha256": hashlib.sha256(vx.tobytes()).hexdigest(),
             "k_modes": modes(kx), "v_modes": modes(vx)}
        runs = [("scalar_t1", O.SCALAR, 1)]
        if ref.avx2:
            runs.append(("avx2_t1", O.AVX2, 1))
        if c["seq"] >= 4 * c["block"]:
            runs.append(("scalar_t3", O.SCALAR, 3))
        for tag, backend, threads in runs:
            o = ref.attention(q, kx=kx, vx=vx, seq=c["seq"], backend=backend, threads=threads,
                              split=c["block"])
            e["out_" + tag] = b64(o.astype(np.float32))
        o1 = np.frombuffer(base64.b64decode(e["out_scalar_t1"]), dtype=np.uint32)
        exact += int(np.count_nonzero((o1 & 0xFFFF) == 0))
        elems += o1.size
        out["cases"][name] = e
        print(name, e["k_bytes"], e["v_bytes"], e["k_modes"], e["v_modes"])
    # share of output elements that are exact BF16 values (a one-hot softmax copies a V row)
    out["exact_bf16_fraction"] = exact / elems
    print(f"exact-BF16 output elements: {exact} of {elems} ({100 * exact / elems:.2f} %)")
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
