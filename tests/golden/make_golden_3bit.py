#!/usr/bin/env python
"""Write tests/golden/golden_3bit.json: container sizes of the 3-bit extension, from the reference.

The reference implements 2- and 4-bit residual blocks only; its exponent analyser
(python/analyze_exponents.py, `policy_size`) also prices a per-block policy over {raw, 2, 3, 4}
bits, which is how its README quotes the 3-bit figure (ratio 0.712120 at block 128).  This script
imports that analyser from the reference checkout ($KVX_REFERENCE_ROOT, else a `reference`
directory beside the repository) and records, for the K and V tensors of every case in
tests/golden_cases.py (plus two longer config[1]-shaped tensors), the container bytes, escape
count and per-mode block counts of the {raw, 2, 3, 4} policy.  The per-block minimum size does
not depend on how ties are broken, so the encoder's container size must equal these figures
exactly; the mode counts also match because the analyser's tie order (smaller, then raw, then
fewer escapes, then narrower) is the encoder's.

    python tests/golden/make_golden_3bit.py
"""
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "compressed-kv-attention_b200"),
                os.path.join(ROOT, "tests")]
import oracle as O  # noqa: E402
import synth as S  # noqa: E402
from golden_cases import CASES, inputs  # noqa: E402

# longer tensors with the config[1] distributions (K with outliers, V, the 2-bit layer-0 K)
EXTRA = {
    "c1_k_s16384": dict(seed=31, stream=0, seq=16384, dim=64, block=128, profile=S.PROFILE_K),
    "c1_v_s16384": dict(seed=31, stream=1, seq=16384, dim=64, block=128, profile=S.PROFILE_V),
    "c1_narrow_s4096": dict(seed=32, stream=0, seq=4096, dim=64, block=128,
                            profile=S.PROFILE_NARROW),
}


def analyser():
    path = os.path.join(O.default_ref_root(), "python", "analyze_exponents.py")
    spec = importlib.util.spec_from_file_location("ref_analyze_exponents", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def policy(A, bits, block):
    exp = ((bits.astype(np.uint16) >> 7) & 0xFF).astype(np.uint8)
    r = A.policy_size(exp, block, (2, 3, 4))
    n_el = bits.shape[0] * bits.shape[1]
    return {"container_bytes": r["container_bytes"],
            "escapes": int(round(r["escape_rate"] * n_el)),
            "mode_blocks": {m: int(r["mode_blocks"].get(m, 0)) for m in ("0", "2", "3", "4")}}


def main():
    A = analyser()
    out = {"generator": "tests/golden/make_golden_3bit.py",
           "source": "the reference's python/analyze_exponents.py policy_size(exp, block, (2, 3, 4))",
           "cases": {}}
    for name, c in CASES.items():
        _, k, v = inputs(c)
        out["cases"][name] = {"kind": "case", "block": c["block"],
                              "k": policy(A, k, c["block"]), "v": policy(A, v, c["block"])}
    for name, c in EXTRA.items():
        t = S.synth_bf16(c["seed"], c["stream"], c["seq"], c["dim"], c["profile"])
        out["cases"][name] = {"kind": "tensor", **{k: c[k] for k in c if k != "profile"},
                              "profile": int(c["profile"]), "t": policy(A, t, c["block"])}
    with open(os.path.join(HERE, "golden_3bit.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", len(out["cases"]), "cases")


if __name__ == "__main__":
    main()
