"""KV-cache compaction on the GPU (rkv_compact_kv): the kept rows of every
(item, KV head) moved to the front, bit for bit, against numpy indexing --
the device analogue of the reference runner removing the evicted ranges from
its KV cache after stage 1 (runner.cpp:246-269)."""
import numpy as np
import pytest

import cases
import oracle as O
import rkvgen
import rocketkv_b200 as rkv

pytestmark = pytest.mark.gpu


def _kept_lists(rng, batch, len_k, counts):
    kept = np.zeros((batch, max(max(counts), 1)), np.int32)
    for b, n in enumerate(counts):
        kept[b, :n] = np.sort(rng.choice(len_k, n, replace=False))
    return kept


def _expect(K, kept, counts, out_len, base):
    out = base.copy()
    for b, n in enumerate(counts):
        n = min(n, out_len)
        out[b, :, :n] = K[b][:, kept[b, :n]]
    return out


@pytest.mark.parametrize("kind,D", [("bf16", 128), ("f32", 64), ("q8_0", 128)])
@pytest.mark.parametrize("inplace", [False, True])
def test_compact_matches_indexing(kind, D, inplace, cuda):
    import torch
    rng = np.random.default_rng(5)
    B, HK, L = 3, 8, 1500
    counts = [700, 0, 1500 if inplace else 1100]
    if kind == "q8_0":
        rows = [rkvgen.q8_0_inputs(40 + b, (HK, L), D)[0] for b in range(B)]
        Kh = np.stack(rows)
        Vh = np.stack([rkvgen.q8_0_inputs(60 + b, (HK, L), D)[0] for b in range(B)])
        to = lambda a: torch.from_numpy(a).to(cuda)
    else:
        Kh = rng.standard_normal((B, HK, L, D)).astype(np.float32)
        Vh = rng.standard_normal((B, HK, L, D)).astype(np.float32)
        if kind == "bf16":
            Kh, Vh = rkvgen.bf16_bits(Kh), rkvgen.bf16_bits(Vh)
            to = lambda a: torch.from_numpy(a).view(torch.bfloat16).to(cuda)
        else:
            to = lambda a: torch.from_numpy(a).to(cuda)
    kept = _kept_lists(rng, B, L, counts)
    kt = torch.from_numpy(kept).to(cuda)
    nt = torch.tensor(counts, dtype=torch.int32, device=cuda)
    K, V = to(Kh), to(Vh)
    if inplace:
        rkv.compact_kv(K, V, kt, nt, D)
        out_len, baseK, baseV = L, Kh, Vh
        gotK, gotV = K, V
    else:
        out_len = 1200
        sentinel = np.full(Kh.shape[:2] + (out_len,) + Kh.shape[3:], 0x7F, Kh.dtype)
        gotK, gotV = to(sentinel), to(sentinel)
        rkv.compact_kv(K, V, kt, nt, D, K_out=gotK, V_out=gotV)
        baseK = baseV = sentinel
    torch.cuda.synchronize()
    back = (lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)) if kind == "bf16" else (lambda t: t.cpu().numpy())
    np.testing.assert_array_equal(back(gotK), _expect(Kh, kept, counts, out_len, baseK))
    np.testing.assert_array_equal(back(gotV), _expect(Vh, kept, counts, out_len, baseV))
    if not inplace:  # the inputs are untouched
        np.testing.assert_array_equal(back(K), Kh)


def test_compact_skips_indices_outside_the_cache(cuda):
    import torch
    B, HK, L, D = 1, 2, 64, 64
    Kh = np.arange(B * HK * L * D, dtype=np.float32).reshape(B, HK, L, D)
    kept = np.array([[1, -1, 5, 64, 70, 9]], np.int32)
    out = torch.full((B, HK, 6, D), -7.0, device=cuda)
    rkv.compact_kv(torch.from_numpy(Kh).to(cuda), None, torch.from_numpy(kept).to(cuda),
                   torch.tensor([6], dtype=torch.int32, device=cuda), D, K_out=out)
    got = out.cpu().numpy()
    for i, s in enumerate(kept[0]):
        want = Kh[0, :, s] if 0 <= s < L else np.full((HK, D), -7.0, np.float32)
        np.testing.assert_array_equal(got[0, :, i], want)


def test_compact_rejects_bad_arguments(cuda):
    import torch
    L_ = rkv.lib()
    K = torch.zeros((1, 2, 16, 64), device=cuda)
    kept = torch.zeros((1, 4), dtype=torch.int32, device=cuda)
    n = torch.ones(1, dtype=torch.int32, device=cuda)
    out = torch.zeros((1, 2, 8, 64), device=cuda)
    # in place needs out_len == len_k
    assert L_.rkv_compact_kv(K.data_ptr(), None, rkv.F32, 64, 2, 16, 1, K[0].nbytes, kept.data_ptr(), n.data_ptr(),
                             4, K.data_ptr(), None, 8, K[0].nbytes, None) == rkv.RKV_ERR_INVALID_ARG
    # V without V_out, and an unknown dtype
    assert L_.rkv_compact_kv(K.data_ptr(), K.data_ptr(), rkv.F32, 64, 2, 16, 1, K[0].nbytes, kept.data_ptr(),
                             n.data_ptr(), 4, out.data_ptr(), None, 8, out[0].nbytes, None) == rkv.RKV_ERR_INVALID_ARG
    assert L_.rkv_compact_kv(K.data_ptr(), None, 7, 64, 2, 16, 1, K[0].nbytes, kept.data_ptr(), n.data_ptr(), 4,
                             out.data_ptr(), None, 8, out[0].nbytes, None) == rkv.RKV_ERR_INVALID_ARG


def test_evict_then_compact(cuda):
    """Stage 1 on the device, then its kept indices applied to K and V in
    place: the compacted cache equals K[kept] of the oracle's selection."""
    import torch
    p = dict(cases.STAGE1)["s1_basic"]
    Q, K, _ = cases.stage1_build(p)
    cfg = cases.stage1_config(p)
    want = O.prefill_eviction(Q, K, p["len_q"], p["len_k"], cfg)
    V = np.random.default_rng(3).standard_normal(K.shape).astype(np.float32)
    ev = rkv.Evictor(rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}), p["len_q"],
                     p["len_k"], 1, rkv.F32, cuda)
    Kt, Vt = torch.from_numpy(K)[None].to(cuda), torch.from_numpy(V)[None].to(cuda)
    kept, n = ev(torch.from_numpy(Q)[None].to(cuda), Kt)
    rkv.compact_kv(Kt, Vt, kept, n, p["D"])
    torch.cuda.synchronize()
    m = len(want)
    assert int(n[0]) == m
    np.testing.assert_array_equal(Kt[0, :, :m].cpu().numpy(), K[:, want])
    np.testing.assert_array_equal(Vt[0, :, :m].cpu().numpy(), V[:, want])


@pytest.mark.parametrize("kind", ["f32", "bf16", "q8_0"])
@pytest.mark.parametrize("inplace", [False, True])
def test_evict_compact_equals_evict_then_compact(kind, inplace, cuda):
    """rkv_evict_compact (stage 1, then the compaction launched as a dependent
    of the selection) leaves the same kept lists and the same cache, bit for
    bit, as rkv_evict followed by rkv_compact_kv."""
    import torch
    B, H, HK, D, L, w = 3, 24, 8, 128, 2000, 32
    cfg = O.Config(num_heads=H, num_heads_kv=HK, dim_head=D, prompt_budget=500)
    rcfg = rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__})
    if kind == "q8_0":
        Qh = np.stack([rkvgen.q8_0_inputs(80 + b, (H, w), D)[0] for b in range(B)])
        Kh = np.stack([rkvgen.q8_0_inputs(90 + b, (HK, L), D)[0] for b in range(B)])
        Vh = np.stack([rkvgen.q8_0_inputs(95 + b, (HK, L), D)[0] for b in range(B)])
        to = lambda a: torch.from_numpy(a).to(cuda)
        dt = rkv.Q8_0
    else:
        Qh = np.stack([rkvgen.stage1_inputs(80 + b, H, HK, D, w, L)[0] for b in range(B)])
        Kh = np.stack([rkvgen.stage1_inputs(80 + b, H, HK, D, w, L)[1] for b in range(B)])
        Vh = rkvgen.normalish(97, (B, HK, L, D))
        if kind == "bf16":
            Qh, Kh, Vh = rkvgen.bf16_bits(rkvgen.bf16_round(Qh)), rkvgen.bf16_bits(rkvgen.bf16_round(Kh)), rkvgen.bf16_bits(rkvgen.bf16_round(Vh))
            to = lambda a: torch.from_numpy(a).view(torch.bfloat16).to(cuda)
            dt = rkv.BF16
        else:
            to = lambda a: torch.from_numpy(a).to(cuda)
            dt = rkv.F32
    Q = to(Qh)
    # reference: the two calls
    ev = rkv.Evictor(rcfg, w, L, B, dt, cuda)
    K1, V1 = to(Kh), to(Vh)
    kept1, n1 = ev(Q, K1)
    kept1, n1 = kept1.clone(), n1.clone()
    out_len = L if inplace else int(cfg.prompt_budget)
    if inplace:
        rkv.compact_kv(K1, V1, kept1, n1, D)
        refK, refV = K1, V1
    else:
        refK = torch.zeros((B, HK, out_len) + tuple(K1.shape[3:]), dtype=K1.dtype, device=cuda)
        refV = torch.zeros_like(refK)
        rkv.compact_kv(K1, V1, kept1, n1, D, K_out=refK, V_out=refV)
    # the fused call
    ev2 = rkv.Evictor(rcfg, w, L, B, dt, cuda)
    K2, V2 = to(Kh), to(Vh)
    if inplace:
        kept2, n2 = ev2.evict_compact(Q, K2, V2)
        gotK, gotV = K2, V2
    else:
        gotK, gotV = torch.zeros_like(refK), torch.zeros_like(refV)
        kept2, n2 = ev2.evict_compact(Q, K2, V2, K_out=gotK, V_out=gotV)
    torch.cuda.synchronize()
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ev2.ws), 0) == 0
    assert torch.equal(n2, n1) and torch.equal(kept2, kept1)
    assert torch.equal(gotK.view(torch.uint8), refK.view(torch.uint8))
    assert torch.equal(gotV.view(torch.uint8), refV.view(torch.uint8))
