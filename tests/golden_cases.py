"""Seeded cases behind tests/golden/golden.json (inputs are regenerated, not stored)."""
import numpy as np

import synth as S

# name -> shape and data profile.  Small enough for the scalar CPU code to finish in seconds.
CASES = {
    "c0_d64_s1000": dict(seed=11, seq=1000, dim=64, n_q=7, block=128, kp=S.PROFILE_K, vp=S.PROFILE_V),
    "tail_d64_s219": dict(seed=12, seq=219, dim=64, n_q=7, block=128, kp=S.PROFILE_K, vp=S.PROFILE_V),
    "narrow_2bit": dict(seed=13, seq=512, dim=64, n_q=7, block=128, kp=S.PROFILE_NARROW, vp=S.PROFILE_V),
    "wide_raw_d256": dict(seed=14, seq=384, dim=256, n_q=4, block=128, kp=S.PROFILE_WIDE_K,
                          vp=S.PROFILE_WIDE_V),
    "d128_s300": dict(seed=15, seq=300, dim=128, n_q=4, block=128, kp=S.PROFILE_K, vp=S.PROFILE_V),
    "d32_block32": dict(seed=16, seq=90, dim=32, n_q=2, block=32, kp=S.PROFILE_K, vp=S.PROFILE_V),
    "d8_block64": dict(seed=17, seq=200, dim=8, n_q=3, block=64, kp=S.PROFILE_K, vp=S.PROFILE_V),
}


def inputs(c):
    q = S.synth_bf16(c["seed"], 2, c["n_q"], c["dim"], S.PROFILE_Q)
    k = S.synth_bf16(c["seed"], 0, c["seq"], c["dim"], c["kp"])
    v = S.synth_bf16(c["seed"], 1, c["seq"], c["dim"], c["vp"])
    return q, k, v
