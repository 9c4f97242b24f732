"""Parity cases shared by the golden-fixture generator and the tests.

Each case names its geometry, RocketConfig fields and input recipe; inputs
are rebuilt from the seed with tests/rkvgen.py, so the fixture file only
stores the reference's outputs.
"""
from __future__ import annotations

import numpy as np

import rkvgen

# ---- stage 1: (name, dict) -------------------------------------------------
STAGE1 = [
    ("s1_basic", dict(H=24, HK=8, D=128, len_q=1024, len_k=1024, window=32, ks=63, budget=256, seed=11, kind="normal")),
    ("s1_needle", dict(H=24, HK=8, D=128, len_q=2048, len_k=2048, window=32, ks=63, budget=512, seed=12, kind="needle")),
    ("s1_shortq", dict(H=8, HK=2, D=64, len_q=20, len_k=700, window=32, ks=7, budget=100, seed=13, kind="normal")),
    ("s1_mha_ks1", dict(H=4, HK=4, D=128, len_q=600, len_k=600, window=32, ks=1, budget=64, seed=14, kind="normal")),
    ("s1_q8", dict(H=24, HK=8, D=128, len_q=1024, len_k=1024, window=32, ks=63, budget=256, seed=15, kind="q8_0")),
    ("s1_bf16", dict(H=24, HK=8, D=128, len_q=1000, len_k=1000, window=32, ks=63, budget=300, seed=16, kind="bf16")),
    ("s1_evenks", dict(H=12, HK=4, D=96, len_q=777, len_k=777, window=16, ks=10, budget=200, seed=17, kind="normal")),
    # the single-layer fp32 configuration: K [8, 8192, 128], window queries Q [24, 32, 128], budget 1024
    ("s1_config0", dict(H=24, HK=8, D=128, len_q=32, len_k=8192, window=32, ks=63, budget=1024, seed=42, kind="normal")),
]

# ---- stage 2 ------------------------------------------------------------------
STAGE2 = [
    ("s2_cfg1", dict(H=24, HK=8, D=128, L=2048, C=16, r=32, k=256, cr=4.0, seed=21, bf16=True, outl=0.01)),
    ("s2_headline", dict(H=24, HK=8, D=128, L=3717, C=2, r=71, k=512, cr=3.6298828125, seed=22, bf16=True, outl=0.01)),
    ("s2_rfull", dict(H=24, HK=8, D=128, L=300, C=4, r=128, k=64, cr=4.0, seed=23, bf16=False, outl=0.0)),
    ("s2_fallback", dict(H=24, HK=8, D=128, L=1024, C=0, r=0, k=256, cr=4.0, seed=24, bf16=False, outl=0.0)),
    ("s2_bigchunk", dict(H=24, HK=8, D=128, L=1000, C=100, r=16, k=300, cr=4.0, seed=25, bf16=True, outl=0.01)),
    ("s2_mha_d64", dict(H=8, HK=8, D=64, L=500, C=3, r=20, k=50, cr=4.0, seed=26, bf16=True, outl=0.02)),
    ("s2_d256", dict(H=16, HK=2, D=256, L=400, C=8, r=100, k=96, cr=4.0, seed=27, bf16=False, outl=0.01)),
    ("s2_keepall", dict(H=24, HK=8, D=128, L=200, C=16, r=32, k=500, cr=4.0, seed=28, bf16=True, outl=0.0)),
    ("s2_gqa4", dict(H=32, HK=8, D=128, L=777, C=5, r=40, k=111, cr=4.0, seed=29, bf16=True, outl=0.01)),
]


def stage1_config(p):
    from oracle import Config
    return Config(num_heads=p["H"], num_heads_kv=p["HK"], dim_head=p["D"], window_size=p["window"],
                  kernel_size=p["ks"], prompt_budget=p["budget"], topk_decode=0, chunk_size=0, r_dim=0,
                  compression_ratio=1.0)


def stage1_build(p):
    """Returns (Q, K) float32 as the oracle sees them, plus the device form:
    (dtype name, Q_dev, K_dev) where *_dev are float32, uint16 bf16 bits or
    uint8 q8_0 rows."""
    H, HK, D, lq, lk, seed = p["H"], p["HK"], p["D"], p["len_q"], p["len_k"], p["seed"]
    kind = p["kind"]
    if kind == "q8_0":
        qp, Q = rkvgen.q8_0_inputs(seed, (H, lq), D)
        kp, K = rkvgen.q8_0_inputs(seed + 1, (HK, lk), D)
        return Q, K, ("q8_0", qp, kp)
    Q, K = rkvgen.stage1_inputs(seed, H, HK, D, lq, lk)
    if kind == "needle":  # the planted-needle layout of the reference's stage-1 test
        Q *= np.float32(0.1)
        K *= np.float32(0.1)
        for pos in (120, 450, 980, 1420):
            K[:, pos, :] = 5.0
        Q[:, lq - p["window"]:, :] = 2.0
    if kind == "bf16":
        Q, K = rkvgen.bf16_round(Q), rkvgen.bf16_round(K)
        return Q, K, ("bf16", rkvgen.bf16_bits(Q), rkvgen.bf16_bits(K))
    return Q, K, ("f32", Q, K)


def stage2_config(p):
    from oracle import Config
    return Config(num_heads=p["H"], num_heads_kv=p["HK"], dim_head=p["D"], window_size=32, kernel_size=63,
                  prompt_budget=0, topk_decode=p["k"], chunk_size=p["C"], r_dim=p["r"],
                  compression_ratio=p["cr"])


def stage2_build(p):
    q, K, V = rkvgen.stage2_inputs(p["seed"], p["H"], p["HK"], p["D"], p["L"], p["outl"], 8.0, p["bf16"])
    return q, K, V


PARAM_GRID = [(b, s, t, d, w) for b in (64, 128, 512, 1024, 2048, 4096)
              for s in (100, 1000, 2048, 8192, 16384, 131072)
              for t in (0, 16, 32, 128) for d in (64, 128) for w in (16, 32)]
