"""Seeded cases behind tests/golden/golden.json (inputs are regenerated, not stored).

Queries are softened (bf16 exponent lowered by `soft`, i.e. scaled by 2**-soft) so that every
case's softmax spreads its weight over many tokens: the fixtures then pin the exp / running-sum /
P.V accumulation of the reference, not only which token wins.  (Unsoftened BASELINE queries
against the synthetic K, whose 0.3 % outliers are scaled by 2**9, give a one-hot softmax, and the
output is a V row copied through.)
"""
import numpy as np

import synth as S
from helpers import soften

# name -> shape and data profile.  Small enough for the scalar CPU code to finish in seconds.
CASES = {
    "c0_d64_s1000": dict(seed=11, seq=1000, dim=64, n_q=7, block=128, kp=S.PROFILE_K,
                         vp=S.PROFILE_V, soft=8),
    "tail_d64_s219": dict(seed=12, seq=219, dim=64, n_q=7, block=128, kp=S.PROFILE_K,
                          vp=S.PROFILE_V, soft=8),
    "narrow_2bit": dict(seed=13, seq=512, dim=64, n_q=7, block=128, kp=S.PROFILE_NARROW,
                        vp=S.PROFILE_V, soft=6),
    "wide_raw_d256": dict(seed=14, seq=384, dim=256, n_q=4, block=128, kp=S.PROFILE_WIDE_K,
                          vp=S.PROFILE_WIDE_V, soft=32),
    "d128_s300": dict(seed=15, seq=300, dim=128, n_q=4, block=128, kp=S.PROFILE_K,
                      vp=S.PROFILE_V, soft=8),
    "d32_block32": dict(seed=16, seq=90, dim=32, n_q=2, block=32, kp=S.PROFILE_K, vp=S.PROFILE_V,
                        soft=6),
    "d8_block64": dict(seed=17, seq=200, dim=8, n_q=3, block=64, kp=S.PROFILE_K, vp=S.PROFILE_V,
                       soft=0),
    # one (layer, KV head) unit of config[1] at full length, and its 2-bit layer-0 K
    "c1_unit_d64_s32768": dict(seed=18, seq=32768, dim=64, n_q=7, block=128, kp=S.PROFILE_K,
                               vp=S.PROFILE_V, soft=8),
    "c1_layer0_2bit_s8192": dict(seed=19, seq=8192, dim=64, n_q=7, block=128,
                                 kp=S.PROFILE_NARROW, vp=S.PROFILE_V, soft=6),
    # config[4]'s distribution (5 % raw blocks, 2 % escapes) at D=256
    "c4_raw_d256_s2048": dict(seed=20, seq=2048, dim=256, n_q=4, block=128,
                              kp=S.PROFILE_WIDE_K, vp=S.PROFILE_WIDE_V, soft=32),
    # config[3]'s shape (D=128, GQA 4)
    "c3_d128_s4096": dict(seed=22, seq=4096, dim=128, n_q=4, block=128, kp=S.PROFILE_K,
                          vp=S.PROFILE_V, soft=8),
}


def inputs(c):
    q = S.synth_bf16(c["seed"], 2, c["n_q"], c["dim"], S.PROFILE_Q)
    if c.get("soft", 0):
        q = soften(q, c["soft"])
    k = S.synth_bf16(c["seed"], 0, c["seq"], c["dim"], c["kp"])
    v = S.synth_bf16(c["seed"], 1, c["seq"], c["dim"], c["vp"])
    return np.ascontiguousarray(q), k, v
