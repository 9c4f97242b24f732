"""The oracle is pinned before it is trusted (CPU only).

* known-answer values of the reference's own test (test_rocket.cpp:184-209);
* golden outputs of the reference rocket.cpp (tests/golden/golden.npz,
  written by tests/golden/gen_golden.py from oracle/_ref);
* live comparisons with oracle/_ref where it was built;
* the deterministic exp against float64 exp.
"""
import math

import numpy as np
import pytest

import cases
import oracle as O
import rkvgen

GOLD = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "golden.npz"))


# test_rocket.cpp:184-209
@pytest.mark.parametrize("S,cap,prompt,k,chunk,r", [(8192, 3717, 3685, 512, 2, 71), (16384, 4837, 4805, 512, 3, 81)])
def test_params_known_answers(S, cap, prompt, k, chunk, r):
    p = O.compute_params(1024, S, 32, 128)
    assert (p["capacity_budget"], p["prompt_budget"], p["k"], p["chunk_size"], p["r"]) == (cap, prompt, k, chunk, r)


def test_params_golden_grid():
    inp, out = GOLD["params/in"], GOLD["params/out"]
    for g, want in zip(inp, out):
        p = O.compute_params(*[int(x) for x in g])
        got = [p["token_budget"], p["sequence_length"], p["max_new_tokens"], p["capacity_budget"],
               p["prompt_budget"], p["chunk_size"], p["r"], p["k"],
               int(np.float32(p["compression_ratio"]).view(np.int32))]
        assert got == [int(x) for x in want], g


def test_expf_accuracy():
    xs = np.concatenate([np.linspace(-103.9, 0.0, 20001, dtype=np.float32),
                         -np.abs(rkvgen.normalish(5, (5000,), 8.0))]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = O.expf(float(x))
        ref = math.exp(float(x))
        if ref < 1.2e-38:
            continue
        ulp = float(np.spacing(np.float32(ref)))
        worst = max(worst, abs(got - ref) / ulp)
    assert worst <= 1.0, worst
    assert O.expf(0.0) == 1.0 and O.expf(-200.0) == 0.0


def _tie_equivalent(a, b, total):
    """Same size, and any difference lies inside one exact-tie score group."""
    if len(a) != len(b):
        return False
    da, db = sorted(set(a) - set(b)), sorted(set(b) - set(a))
    if not da:
        return True
    vals = {float(total[i]) for i in da + db}
    return len(vals) == 1


@pytest.mark.parametrize("name", [n for n, _ in cases.STAGE1])
def test_stage1_oracle_vs_reference_golden(name):
    p = dict(cases.STAGE1)[name]
    Q, K, _ = cases.stage1_build(p)
    cfg = cases.stage1_config(p)
    kept, total = O.prefill_eviction(Q, K, p["len_q"], p["len_k"], cfg, want_total=True)
    ref = GOLD[f"{name}/kept"]
    assert np.all(np.diff(kept) > 0)
    assert _tie_equivalent(list(kept), list(ref), total), name
    # the window is always kept (rocket.cpp:163-165)
    ow = min(p["window"], p["len_q"])
    assert set(range(p["len_k"] - ow, p["len_k"])) <= set(kept.tolist())


def test_stage1_needles_kept():
    """test_rocket.cpp:114-134: size, window and planted needles."""
    p = dict(cases.STAGE1)["s1_needle"]
    Q, K, _ = cases.stage1_build(p)
    kept = O.prefill_eviction(Q, K, p["len_q"], p["len_k"], cases.stage1_config(p))
    assert len(kept) == p["budget"]
    assert {120, 450, 980, 1420} <= set(kept.tolist())


def topr_tie_groups(q, cfg, L):
    """KV groups whose sum_h |q| has an exact tie across the top-r boundary.
    There rocket.cpp's std::nth_element (score-only comparator,
    rocket.cpp:232-235) keeps an unspecified member; the oracle keeps the
    lower dimension."""
    G = max(1, cfg.num_heads // cfg.num_heads_kv)
    C = cfg.chunk_size if cfg.chunk_size > 0 else max(1, min(int(np.floor(cfg.compression_ratio)),
                                                               int(np.ceil(np.sqrt(cfg.compression_ratio)))))
    r = cfg.r_dim if cfg.r_dim > 0 else min(cfg.dim_head, max(1, int(round(cfg.dim_head * C / cfg.compression_ratio))))
    out = set()
    if r >= cfg.dim_head or cfg.topk_decode >= L:
        return out
    for g in range(cfg.num_heads_kv):
        sabs = np.zeros(cfg.dim_head, np.float32)
        for h in range(G):
            sabs = (sabs + np.abs(q[g * G + h])).astype(np.float32)
        srt = np.sort(sabs)[::-1]
        if srt[r - 1] == srt[r]:
            out.add(g)
    return out


def assert_matches_reference(Oo, Oref, q, cfg, L):
    """Bit-identical per query head, except in KV groups with a top-r tie,
    which must still agree within the attention tolerance."""
    G = max(1, cfg.num_heads // cfg.num_heads_kv)
    ties = topr_tie_groups(q, cfg, L)
    for g in range(cfg.num_heads_kv):
        a, b = Oo[g * G:(g + 1) * G], Oref[g * G:(g + 1) * G]
        if g in ties:
            np.testing.assert_allclose(a, b, rtol=1e-3, atol=1e-4)
        else:
            np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("name", [n for n, _ in cases.STAGE2])
def test_stage2_oracle_vs_reference_golden(name):
    """Selection identical => the attention half repeats rocket.cpp's float
    operations one for one, so O is bit-identical to the reference's."""
    p = dict(cases.STAGE2)[name]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    Oo, sel = O.hsa_decode(q, K, V, p["L"], cfg)
    assert_matches_reference(Oo, GOLD[f"{name}/O"], q, cfg, p["L"])
    k = min(p["k"], p["L"])
    assert all(len(s) == k and np.all(np.diff(s) > 0) for s in sel)


def test_stage2_dense_cosine():
    """test_rocket.cpp:140-178: sparse vs dense attention cosine on noise."""
    p = dict(cases.STAGE2)["s2_fallback"]
    q, K, V = cases.stage2_build(p)
    Oo, _ = O.hsa_decode(q, K, V, p["L"], cases.stage2_config(p))
    G = p["H"] // p["HK"]
    dense = np.zeros_like(Oo)
    for h in range(p["H"]):
        s = K[h // G] @ q[h] / np.sqrt(p["D"])
        e = np.exp(s - s.max())
        dense[h] = (e / e.sum()) @ V[h // G]
    cos = float((Oo * dense).sum() / np.sqrt((Oo ** 2).sum() * (dense ** 2).sum()))
    assert cos > 0.70


def test_stage2_recent_window_semantics():
    """recent_window = w: the reference selection over the first len_k - w
    tokens, plus the last w tokens."""
    p = dict(cases.STAGE2)["s2_cfg1"]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    w = 32
    L = p["L"]
    _, sel_w = O.hsa_decode(q, K, V, L, cfg, recent_window=w)
    _, sel_0 = O.hsa_decode(q, np.ascontiguousarray(K[:, :L - w]), np.ascontiguousarray(V[:, :L - w]), L - w, cfg)
    for a, b in zip(sel_w, sel_0):
        np.testing.assert_array_equal(a, np.concatenate([b, np.arange(L - w, L)]))


def test_head_sharded_stage1_matches():
    p = dict(cases.STAGE1)["s1_basic"]
    Q, K, _ = cases.stage1_build(p)
    cfg = cases.stage1_config(p)
    parts = [O.evict_pool_heads(Q, K, p["len_q"], p["len_k"], cfg, h, 1) for h in range(p["HK"])]
    kept = O.evict_select_pooled(np.concatenate(parts, 0), p["len_q"], p["len_k"], cfg)
    np.testing.assert_array_equal(kept, O.prefill_eviction(Q, K, p["len_q"], p["len_k"], cfg))


@pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built (no reference sources)")
@pytest.mark.parametrize("seed", [101, 102, 103])
def test_stage1_oracle_vs_reference_live(seed):
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=400)
    Q, K = rkvgen.stage1_inputs(seed, 24, 8, 128, 1536, 1536)
    kept, total = O.prefill_eviction(Q, K, 1536, 1536, cfg, want_total=True)
    ref = O.ref_prefill_eviction(Q, K, 1536, 1536, cfg)
    assert _tie_equivalent(list(kept), list(ref), total)


@pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built (no reference sources)")
@pytest.mark.parametrize("seed", [201, 202])
def test_stage2_oracle_vs_reference_live(seed):
    cfg = O.Config(topk_decode=200, chunk_size=8, r_dim=48)
    q, K, V = rkvgen.stage2_inputs(seed, 24, 8, 128, 1500)
    Oo, _ = O.hsa_decode(q, K, V, 1500, cfg)
    assert_matches_reference(Oo, O.ref_hsa_decode(q, K, V, 1500, cfg), q, cfg, 1500)


@pytest.mark.parametrize("lk,budget", [(100, 100), (100, 500), (50, 40)])
def test_stage1_keep_all_paths(lk, budget):
    """rocket.cpp:67-71 and :134-138."""
    cfg = O.Config(num_heads=4, num_heads_kv=2, dim_head=32, prompt_budget=budget)
    Q, K = rkvgen.stage1_inputs(7, 4, 2, 32, lk, lk)
    kept = O.prefill_eviction(Q, K, lk, lk, cfg)
    if lk <= budget or budget - 32 >= lk - 32:
        np.testing.assert_array_equal(kept, np.arange(lk))
