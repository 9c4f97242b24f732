"""Stage-1 eviction on the GPU against the oracle (bit-exact kept indices,
ties to the lower index) and against the reference's own outputs."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import cases
import oracle as O
import rkvgen
import rocketkv_b200 as rkv
from gpuutil import boundary_report, dev

pytestmark = pytest.mark.gpu
GOLD = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "golden.npz"))
KIND = {"f32": rkv.F32, "bf16": rkv.BF16, "q8_0": rkv.Q8_0}


def to_rkv(cfg):
    return rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__})


def run_gpu(Qd, Kd, kind, len_q, len_k, cfg, device):
    import torch
    Qt = dev(Qd, kind, device).unsqueeze(0).contiguous()
    Kt = dev(Kd, kind, device).unsqueeze(0).contiguous()
    ev = rkv.Evictor(to_rkv(cfg), len_q, len_k, 1, KIND[kind], device)
    kept, n = ev(Qt, Kt)
    torch.cuda.synchronize()
    return kept[0, : int(n[0])].cpu().numpy()


@pytest.mark.parametrize("name", [n for n, _ in cases.STAGE1])
def test_stage1_cases(name, cuda):
    p = dict(cases.STAGE1)[name]
    Q, K, (kind, Qd, Kd) = cases.stage1_build(p)
    cfg = cases.stage1_config(p)
    want, total = O.prefill_eviction(Q, K, p["len_q"], p["len_k"], cfg, want_total=True)
    got = run_gpu(Qd, Kd, kind, p["len_q"], p["len_k"], cfg, cuda)
    assert np.array_equal(got, want), boundary_report(total, got, want)
    # and the reference's own output, up to its unspecified tie members
    ref = GOLD[f"{name}/kept"]
    diff = set(got.tolist()) ^ set(ref.tolist())
    assert len(got) == len(ref) and len({float(total[i]) for i in diff}) <= 1


@pytest.mark.parametrize("name", ["s1_basic", "s1_bf16", "s1_shortq", "s1_mha_ks1", "s1_evenks", "s1_q8", "s1_needle"])
def test_stage1_tensor_engines_match_cuda_cores(name, cuda):
    """The tcgen05 scorers (the persistent kernel, and for fp32/bf16 the
    per-tile kernel; fp32 and q8_0 as three TF32 products per step, bf16
    direct) against the fp32 CUDA-core engine on the same inputs: pooled rows
    within 1e-4 relative, kept indices identical."""
    import torch
    p = dict(cases.STAGE1)[name]
    Q, K, (kind, Qd, Kd) = cases.stage1_build(p)
    cfg = to_rkv(cases.stage1_config(p))
    Qt = dev(Qd, kind, cuda).unsqueeze(0).contiguous()
    Kt = dev(Kd, kind, cuda).unsqueeze(0).contiguous()
    ev = rkv.Evictor(cfg, p["len_q"], p["len_k"], 1, KIND[kind], cuda)
    nk = p["len_k"] - min(p["window"], p["len_q"])
    engines = [rkv.ENGINE_TENSOR, rkv.ENGINE_SIMT] + ([rkv.ENGINE_TENSOR_TILES] if kind != "q8_0" else [])
    pooled = {}
    for eng in engines:
        out = torch.empty((1, p["HK"], nk), dtype=torch.float32, device=cuda)
        ev.pool_heads(Qt, Kt, 0, p["HK"], out, engine=eng)
        torch.cuda.synchronize()
        pooled[eng] = out[0].cpu().numpy()
    kept = {}
    for eng in engines:
        k, n = ev(Qt, Kt, engine=eng)
        kept[eng] = k[0, : int(n[0])].cpu().numpy().copy()
    for eng in engines:
        np.testing.assert_allclose(pooled[eng], pooled[rkv.ENGINE_SIMT], rtol=1e-4, atol=1e-7, err_msg=str(eng))
        np.testing.assert_array_equal(kept[eng], kept[rkv.ENGINE_SIMT], err_msg=str(eng))
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ev.ws), 0) == 0


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_stage1_long_prefix_select(kind, cuda):
    """nk > 16384 takes the selection that keeps its keys in global memory
    (and the tensor scorer with many tiles per head): kept indices equal the
    oracle's and every engine's."""
    import torch
    cfg = O.Config(num_heads=6, num_heads_kv=2, dim_head=64, prompt_budget=3000)
    len_k = 20000
    Q, K = rkvgen.stage1_inputs(91, 6, 2, 64, 32, len_k)
    if kind == "bf16":
        Q, K = rkvgen.bf16_round(Q), rkvgen.bf16_round(K)
        Qd, Kd = rkvgen.bf16_bits(Q), rkvgen.bf16_bits(K)
    else:
        Qd, Kd = Q, K
    want, total = O.prefill_eviction(Q, K, 32, len_k, cfg, want_total=True)
    Qt = dev(Qd, kind, cuda).unsqueeze(0).contiguous()
    Kt = dev(Kd, kind, cuda).unsqueeze(0).contiguous()
    ev = rkv.Evictor(to_rkv(cfg), 32, len_k, 1, KIND[kind], cuda)
    for eng in (rkv.ENGINE_AUTO, rkv.ENGINE_TENSOR_TILES, rkv.ENGINE_SIMT):
        k, n = ev(Qt, Kt, engine=eng)
        torch.cuda.synchronize()
        got = k[0, : int(n[0])].cpu().numpy()
        assert len(got) == 3000
        assert np.array_equal(got, want), (eng, boundary_report(total, got, want))


@pytest.mark.parametrize("H,HK,window,kind", [
    (32, 8, 32, "bf16"),  # 128 window rows: every lane quarter full
    (16, 8, 24, "bf16"),  # 48 rows: the second quarter partly padding
    (24, 8, 40, "f32"),   # 120 rows: the fourth quarter partly padding
    (8, 8, 8, "f32"),     # 8 rows: most of the first quarter padding
])
def test_stage1_window_row_counts(H, HK, window, kind, cuda):
    """The persistent scorer holds the window rows on the tensor-memory lanes,
    32 per warp: row counts that fill every lane quarter, or leave one partly
    or mostly padding, keep the oracle's indices."""
    cfg = O.Config(num_heads=H, num_heads_kv=HK, dim_head=128, window_size=window, prompt_budget=700)
    len_k = 3000
    Q, K = rkvgen.stage1_inputs(400 + H + window, H, HK, 128, window, len_k)
    if kind == "bf16":
        Q, K = rkvgen.bf16_round(Q), rkvgen.bf16_round(K)
        Qd, Kd = rkvgen.bf16_bits(Q), rkvgen.bf16_bits(K)
    else:
        Qd, Kd = Q, K
    want, total = O.prefill_eviction(Q, K, window, len_k, cfg, want_total=True)
    got = run_gpu(Qd, Kd, kind, window, len_k, cfg, cuda)
    assert np.array_equal(got, want), boundary_report(total, got, want)


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_stage1_recompute_form(kind, cuda):
    """Kept exp values of 8 heads x 96 rows x 20000 keys (61 MB) exceed what
    the persistent scorer keeps for pass 1, so pass 1 recomputes the logits
    through the copy / MMA pipeline (in reverse tile order): kept indices equal
    the oracle's and the other engines'."""
    import torch
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=2500)
    len_k = 20000
    Q, K = rkvgen.stage1_inputs(97, 24, 8, 128, 32, len_k)
    if kind == "bf16":
        Q, K = rkvgen.bf16_round(Q), rkvgen.bf16_round(K)
        Qd, Kd = rkvgen.bf16_bits(Q), rkvgen.bf16_bits(K)
    else:
        Qd, Kd = Q, K
    want, total = O.prefill_eviction(Q, K, 32, len_k, cfg, want_total=True)
    Qt = dev(Qd, kind, cuda).unsqueeze(0).contiguous()
    Kt = dev(Kd, kind, cuda).unsqueeze(0).contiguous()
    ev = rkv.Evictor(to_rkv(cfg), 32, len_k, 1, KIND[kind], cuda)
    for eng in (rkv.ENGINE_TENSOR, rkv.ENGINE_SIMT):
        k, n = ev(Qt, Kt, engine=eng)
        torch.cuda.synchronize()
        got = k[0, : int(n[0])].cpu().numpy()
        assert len(got) == 2500
        assert np.array_equal(got, want), (eng, boundary_report(total, got, want))
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ev.ws), 0) == 0


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_stage1_even_split_crosses_heads(kind, cuda):
    """8 sequences x 8 KV heads of 20 key tiles: the head-aligned split would
    give some CTAs 10 tiles, so the persistent scorer splits all 1280 tiles
    evenly (at most 9 per CTA) and CTAs cross from one KV head (and sequence)
    to the next, reloading the window queries and the row statistics: kept
    indices equal the oracle's for every sequence, on both engines."""
    import torch
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=300)
    nb, len_k = 8, 2560
    Qs, Ks, wants = [], [], []
    for b in range(nb):
        Q, K = rkvgen.stage1_inputs(300 + b, 24, 8, 128, 32, len_k)
        if kind == "bf16":
            Q, K = rkvgen.bf16_round(Q), rkvgen.bf16_round(K)
        wants.append(O.prefill_eviction(Q, K, 32, len_k, cfg, want_total=True))
        Qs.append(rkvgen.bf16_bits(Q) if kind == "bf16" else Q)
        Ks.append(rkvgen.bf16_bits(K) if kind == "bf16" else K)
    Qt = torch.stack([dev(q, kind, cuda) for q in Qs]).contiguous()
    Kt = torch.stack([dev(k, kind, cuda) for k in Ks]).contiguous()
    ev = rkv.Evictor(to_rkv(cfg), 32, len_k, nb, KIND[kind], cuda)
    for eng in (rkv.ENGINE_TENSOR, rkv.ENGINE_SIMT):
        k, n = ev(Qt, Kt, engine=eng)
        torch.cuda.synchronize()
        for b in range(nb):
            want, total = wants[b]
            got = k[b, : int(n[b])].cpu().numpy()
            assert len(got) == 300
            assert np.array_equal(got, want), (eng, b, boundary_report(total, got, want))
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ev.ws), 0) == 0


def test_stage1_config0_full_size(cuda):
    """K [8, 8192, 128] fp32, Q [24, 32, 128] window, budget 1024, ks 63."""
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=1024)
    Q, K = rkvgen.stage1_inputs(42, 24, 8, 128, 32, 8192)
    want, total = O.prefill_eviction(Q, K, 32, 8192, cfg, want_total=True)
    got = run_gpu(Q, K, "f32", 32, 8192, cfg, cuda)
    assert len(got) == 1024
    assert np.array_equal(got, want), boundary_report(total, got, want)
    if O.have_ref():
        ref = O.ref_prefill_eviction(Q, K, 32, 8192, cfg)
        diff = set(got.tolist()) ^ set(ref.tolist())
        assert len({float(total[i]) for i in diff}) <= 1


def test_stage1_batched_q8_layers(cuda):
    """Several q8_0 layers in one launch (the 28-layer configuration's shape,
    fewer layers and a shorter prefix); every layer against the oracle."""
    import torch
    L, S, budget = 6, 4096, 1024
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=budget)
    items = [(rkvgen.q8_0_inputs(900 + 2 * l, (24, 32), 128), rkvgen.q8_0_inputs(901 + 2 * l, (8, S), 128))
             for l in range(L)]
    Qt = torch.stack([torch.from_numpy(q[0]) for q, _ in items]).to(cuda)
    Kt = torch.stack([torch.from_numpy(k[0]) for _, k in items]).to(cuda)
    ev = rkv.Evictor(to_rkv(cfg), 32, S, L, rkv.Q8_0, cuda)
    kept, n = ev(Qt, Kt)
    kept, n = kept.cpu().numpy(), n.cpu().numpy()
    with ThreadPoolExecutor(8) as ex:
        wants = list(ex.map(lambda it: O.prefill_eviction(it[0][1], it[1][1], 32, S, cfg, want_total=True), items))
    for l, (want, total) in enumerate(wants):
        got = kept[l, : n[l]]
        assert np.array_equal(got, want), (l, boundary_report(total, got, want))


def test_stage1_head_sharded_equals_fused(cuda):
    import torch
    p = dict(cases.STAGE1)["s1_basic"]
    Q, K, _ = cases.stage1_build(p)
    cfg = cases.stage1_config(p)
    Qt, Kt = dev(Q, "f32", cuda)[None], dev(K, "f32", cuda)[None]
    ev = rkv.Evictor(to_rkv(cfg), p["len_q"], p["len_k"], 1, rkv.F32, cuda)
    nk = p["len_k"] - min(p["window"], p["len_q"])
    pooled = torch.empty((1, p["HK"], nk), dtype=torch.float32, device=cuda)
    for h in range(p["HK"]):  # one head at a time, as one rank each would
        part = torch.empty((1, 1, nk), dtype=torch.float32, device=cuda)
        ev.pool_heads(Qt, Kt, h, 1, part)
        pooled[:, h] = part[:, 0]
    # pooled scores: float sums in another order than the oracle's, and (tensor
    # engine) logits from three TF32 products per step, about 1e-6 relative
    np.testing.assert_allclose(pooled[0].cpu().numpy(), O.evict_pool_heads(Q, K, p["len_q"], p["len_k"], cfg, 0, p["HK"]),
                               rtol=1e-4, atol=1e-9)
    k1, n1 = ev.select_pooled(pooled)
    a = k1[0, : int(n1[0])].cpu().numpy().copy()
    k2, n2 = ev(Qt, Kt)
    np.testing.assert_array_equal(a, k2[0, : int(n2[0])].cpu().numpy())


def test_stage1_host_dropin(cuda):
    """rocket.h path: host fp32 buffers, copies inside the call."""
    p = dict(cases.STAGE1)["s1_needle"]
    Q, K, _ = cases.stage1_build(p)
    cfg = cases.stage1_config(p)
    got = rkv.compute_prefill_eviction(Q, K, p["len_q"], p["len_k"], to_rkv(cfg))
    np.testing.assert_array_equal(got, O.prefill_eviction(Q, K, p["len_q"], p["len_k"], cfg))
    assert {120, 450, 980, 1420} <= set(got.tolist()) and len(got) == 512


@pytest.mark.parametrize("len_q,len_k,budget,ks,window", [
    (300, 300, 300, 63, 32),    # len_k <= budget: keep all
    (300, 300, 290, 63, 32),    # target_keep >= nk: keep all
    (300, 300, 10, 63, 32),     # budget < window: only the window
    (16, 300, 100, 63, 32),     # len_q < window
    (300, 300, 100, 0, 32),     # kernel 0: no pooling
    (300, 300, 100, 2, 32),     # even kernel
    (300, 300, 100, -3, 32),    # negative kernel: empty windows, -FLT_MAX scores
    (300, 300, 100, 4095, 32),  # window wider than the sequence
    (300, 300, 100, 63, 0),     # no observation window: nothing scored
    (129, 129, 40, 63, 1),      # one window row, odd tile edge
])
def test_stage1_edges(len_q, len_k, budget, ks, window, cuda):
    cfg = O.Config(num_heads=6, num_heads_kv=2, dim_head=64, window_size=window, kernel_size=ks, prompt_budget=budget)
    Q, K = rkvgen.stage1_inputs(77, 6, 2, 64, len_q, len_k)
    want, total = O.prefill_eviction(Q, K, len_q, len_k, cfg, want_total=True)
    got = run_gpu(Q, K, "f32", len_q, len_k, cfg, cuda)
    assert np.array_equal(got, want), boundary_report(total, got, want)


def test_stage1_invalid_sizes(cuda):
    cfg = rkv.RocketConfig(num_heads=6, num_heads_kv=2, dim_head=64, prompt_budget=5)
    with pytest.raises(rkv.RkvError) as e:  # len_k < window rows: rocket.cpp cannot size its buffer
        rkv.compute_prefill_eviction(np.zeros((6, 64, 64), np.float32), np.zeros((2, 10, 64), np.float32), 64, 10, cfg)
    assert e.value.status == rkv.RKV_ERR_INVALID_ARG


def test_stage1_config2_full_size_q8(cuda):
    """The 28-layer q8_0 configuration at full size: K [28][8, 8192, 128] and
    window queries Q [28][24, 32, 128] stored q8_0 (int8 uniform in
    [-127, 127], fp16 scales |N(0, 0.02)|), all layers in one call, budgets
    512, 1024 and 2048.  Every layer's kept set equals the oracle's (pooled
    rows per layer from the oracle's scoring, its own selection per budget)."""
    import torch
    layers, S = 28, 8192
    base = O.Config(num_heads=24, num_heads_kv=8, dim_head=128)

    def oracle_layer(l):
        qp, Qf = rkvgen.q8_0_inputs(3000 + 2 * l, (24, 32), 128)
        kp, Kf = rkvgen.q8_0_inputs(3001 + 2 * l, (8, S), 128)
        return qp, kp, O.evict_pool_heads(Qf, Kf, 32, S, base, 0, 8)

    with ThreadPoolExecutor(8) as ex:
        per_layer = list(ex.map(oracle_layer, range(layers)))
    Qt = torch.stack([torch.from_numpy(q) for q, _, _ in per_layer]).to(cuda)
    Kt = torch.stack([torch.from_numpy(k) for _, k, _ in per_layer]).to(cuda)
    for budget in (512, 1024, 2048):
        cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=budget)
        ev = rkv.Evictor(to_rkv(cfg), 32, S, layers, rkv.Q8_0, cuda)
        kept, n = ev(Qt, Kt)
        kept, n = kept.cpu().numpy(), n.cpu().numpy()
        assert rkv.lib().rkv_workspace_status(rkv._ptr(ev.ws), 0) == 0
        for l, (_, _, pooled) in enumerate(per_layer):
            want = O.evict_select_pooled(pooled, 32, S, cfg)
            got = kept[l, : n[l]]
            assert len(want) == budget
            assert np.array_equal(got, want), (budget, l, boundary_report(pooled.sum(0), got, want))


def test_long_context_pipeline(cuda):
    """The long-context configuration on one GPU, end to end for two sequences:
    S = 131072 bf16 K/V/Q (N(0,1), 0.5 % of K rows x8), stage 1 at budget 4096
    (window 32, kernel 63), the KV cache compacted to the kept rows, then one
    stage-2 decode step over the 4096-row cache (page 16, r 32, top-k 256, the
    last 32 rows as the recent window).  Kept indices equal the oracle's per
    sequence (oracle pooling per KV head in host threads); the decode's
    selections equal the oracle's on the compacted cache and O is within
    1e-3 / 1e-4."""
    import torch
    B, S, H, HK, D, budget = 2, 131072, 24, 8, 128, 4096
    g = torch.Generator(device=cuda).manual_seed(4444)
    K = torch.randn((B, HK, S, D), generator=g, device=cuda)
    rows = torch.rand((B, HK, S, 1), generator=g, device=cuda) < 0.005
    K = torch.where(rows, K * 8, K).to(torch.bfloat16).contiguous()
    V = torch.randn((B, HK, S, D), generator=g, device=cuda).to(torch.bfloat16)
    Qw = torch.randn((B, H, 32, D), generator=g, device=cuda).to(torch.bfloat16)  # the window rows
    q = torch.randn((B, H, D), generator=g, device=cuda).to(torch.bfloat16)        # the decode query
    cfg = O.Config(num_heads=H, num_heads_kv=HK, dim_head=D, prompt_budget=budget)
    ev = rkv.Evictor(to_rkv(cfg), 32, S, B, rkv.BF16, cuda)
    kept, n = ev(Qw, K)
    torch.cuda.synchronize()
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ev.ws), 0) == 0
    kept_h, n_h = kept.cpu().numpy(), n.cpu().numpy()
    assert np.all(n_h == budget)
    for b in range(B):
        Qf, Kf = Qw[b].float().cpu().numpy(), K[b].float().cpu().numpy()
        with ThreadPoolExecutor(8) as ex:
            pooled = np.concatenate(list(ex.map(lambda h: O.evict_pool_heads(Qf, Kf, 32, S, cfg, h, 1), range(HK))))
        want = O.evict_select_pooled(pooled, 32, S, cfg)
        got = kept_h[b, : n_h[b]]
        assert np.array_equal(got, want), (b, boundary_report(pooled.sum(0), got, want))
    del Kf
    # the cache left by eviction: the kept rows of every KV head, in order
    Kc = torch.empty((B, HK, budget, D), dtype=torch.bfloat16, device=cuda)
    Vc = torch.empty_like(Kc)
    rkv.compact_kv(K, V, kept, n, D, K_out=Kc, V_out=Vc)
    cfg2 = O.Config(num_heads=H, num_heads_kv=HK, dim_head=D, topk_decode=256, chunk_size=16, r_dim=32,
                    compression_ratio=4.0)
    dec = rkv.HsaDecoder(to_rkv(cfg2), budget, B, cuda, recent_window=32)
    dec(q, Kc, Vc)
    torch.cuda.synchronize()
    assert dec.status() == 0
    for b in range(B):
        idx = kept_h[b, :budget]
        Kb, Vb = K[b].float().cpu().numpy()[:, idx], V[b].float().cpu().numpy()[:, idx]
        assert np.array_equal(Kc[b].float().cpu().numpy(), Kb)
        Oo, so = O.hsa_decode(q[b].float().cpu().numpy(), Kb, Vb, budget, cfg2, recent_window=32)
        for h in range(HK):
            assert np.array_equal(dec.sel[b, h, : int(dec.n_sel[b, h])].cpu().numpy(), so[h]), (b, h)
        np.testing.assert_allclose(dec.O[b].cpu().numpy(), Oo, rtol=1e-3, atol=1e-4)
