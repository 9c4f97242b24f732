"""Stage-2 hybrid sparse decode on the GPU: selected indices bit-identical to
the oracle, O within 1e-3 relative / 1e-4 absolute of it and of the
reference's own output."""
import numpy as np
import pytest

import cases
import oracle as O
import rkvgen
import rocketkv_b200 as rkv
from gpuutil import dev, stage2_boundary_gap

pytestmark = pytest.mark.gpu
GOLD = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "golden.npz"))
RTOL, ATOL = 1e-3, 1e-4


def to_rkv(cfg):
    return rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__})


def run_gpu(qs, Ks, Vs, L, cfg, device, bf16=True, w=0, head_begin=0, head_count=None):
    """qs [B, H, D], Ks/Vs [B, HK, L, D] float32 (exact bf16 values when bf16)."""
    import torch
    kind = "bf16" if bf16 else "f32"
    conv = (lambda a: rkvgen.bf16_bits(a)) if bf16 else (lambda a: a)
    Q = dev(conv(qs), kind, device)
    K = dev(conv(Ks), kind, device)
    V = dev(conv(Vs), kind, device)
    d = rkv.HsaDecoder(to_rkv(cfg), L, qs.shape[0], device, recent_window=w, head_begin=head_begin,
                       head_count=head_count)
    d(Q, K, V)
    torch.cuda.synchronize()
    assert d.status() == 0
    return d.O.cpu().numpy(), d.sel.cpu().numpy(), d.n_sel.cpu().numpy()


def check_against_oracle(q, K, V, L, cfg, Og, sel, nsel, w=0, heads=None, bf16=True):
    Oo, so = O.hsa_decode(q, K, V, L, cfg, recent_window=w, kv_bytes=2 if bf16 else 4)
    G = max(1, cfg.num_heads // cfg.num_heads_kv)
    heads = range(cfg.num_heads_kv) if heads is None else heads
    for i, h in enumerate(heads):
        got = sel[i, : nsel[i]]
        if not np.array_equal(got, so[h]):
            gap = stage2_boundary_gap(q, K, cfg, L, w, h)
            raise AssertionError(f"KV head {h}: selection differs from the oracle; only GPU "
                                 f"{np.setdiff1d(got, so[h])[:5]}, only oracle {np.setdiff1d(so[h], got)[:5]}; "
                                 f"float64 boundary gap {gap:.3e}")
        np.testing.assert_allclose(Og[h * G:(h + 1) * G], Oo[h * G:(h + 1) * G], rtol=RTOL, atol=ATOL)
    return Oo


@pytest.mark.parametrize("name", [n for n, _ in cases.STAGE2])
def test_stage2_cases(name, cuda):
    p = dict(cases.STAGE2)[name]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    Og, sel, nsel = run_gpu(q[None], K[None], V[None], p["L"], cfg, cuda, bf16=p["bf16"])
    check_against_oracle(q, K, V, p["L"], cfg, Og[0], sel[0], nsel[0], bf16=p["bf16"])
    np.testing.assert_allclose(Og[0], GOLD[f"{name}/O"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name,w", [("s2_cfg1", 32), ("s2_headline", 32), ("s2_bigchunk", 7), ("s2_keepall", 50)])
def test_stage2_recent_window(name, w, cuda):
    p = dict(cases.STAGE2)[name]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    Og, sel, nsel = run_gpu(q[None], K[None], V[None], p["L"], cfg, cuda, bf16=p["bf16"], w=w)
    check_against_oracle(q, K, V, p["L"], cfg, Og[0], sel[0], nsel[0], w=w, bf16=p["bf16"])
    for h in range(cfg.num_heads_kv):
        assert set(range(p["L"] - w, p["L"])) <= set(sel[0, h, : nsel[0, h]].tolist())


def test_stage2_batched_head_subset(cuda):
    p = dict(cases.STAGE2)["s2_cfg1"]
    cfg = cases.stage2_config(p)
    items = [rkvgen.stage2_inputs(500 + i, 24, 8, 128, 1111) for i in range(3)]
    qs = np.stack([it[0] for it in items])
    Ks = np.stack([it[1] for it in items])
    Vs = np.stack([it[2] for it in items])
    Og, sel, nsel = run_gpu(qs, Ks, Vs, 1111, cfg, cuda, head_begin=2, head_count=5)
    for b in range(3):
        check_against_oracle(qs[b], Ks[b], Vs[b], 1111, cfg, Og[b], sel[b], nsel[b], heads=range(2, 7))


def test_stage2_host_dropin_matches_reference(cuda):
    """rocket.h compute_hybrid_sparse_decode: fp32 host buffers, reference semantics."""
    for name in ("s2_fallback", "s2_rfull", "s2_cfg1"):
        p = dict(cases.STAGE2)[name]
        q, K, V = cases.stage2_build(p)
        cfg = cases.stage2_config(p)
        out = rkv.compute_hybrid_sparse_decode(q, K, V, p["L"], to_rkv(cfg)).reshape(p["H"], p["D"])
        np.testing.assert_allclose(out, GOLD[f"{name}/O"], rtol=RTOL, atol=ATOL)


def test_stage2_host_ex_bf16_with_selection(cuda):
    p = dict(cases.STAGE2)["s2_headline"]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    Og, sel, nsel = rkv.hsa_decode_host(rkvgen.bf16_bits(q)[None], rkvgen.bf16_bits(K)[None],
                                        rkvgen.bf16_bits(V)[None], rkv.BF16, p["L"], to_rkv(cfg),
                                        recent_window=32, with_sel=True)
    check_against_oracle(q, K, V, p["L"], cfg, Og[0], sel[0], nsel[0], w=32)


def test_stage2_host_ex_pinned_v_read_in_place(cuda):
    """Host path with V in pinned host memory: the attention reads the selected
    V rows in place (no copy of V); same selection and O as the oracle."""
    import torch
    p = dict(cases.STAGE2)["s2_headline"]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    Vp = torch.from_numpy(rkvgen.bf16_bits(V)[None].view(np.int16)).pin_memory()
    Og, sel, nsel = rkv.hsa_decode_host(rkvgen.bf16_bits(q)[None], rkvgen.bf16_bits(K)[None],
                                        Vp.numpy().view(np.uint16), rkv.BF16, p["L"], to_rkv(cfg),
                                        recent_window=32, with_sel=True)
    check_against_oracle(q, K, V, p["L"], cfg, Og[0], sel[0], nsel[0], w=32)


@pytest.mark.parametrize("L,k,C,r", [(1, 1, 1, 1), (5, 0, 2, 8), (33, 32, 2, 8), (64, 1, 64, 128), (130, 17, 65, 3)])
def test_stage2_edges(L, k, C, r, cuda):
    cfg = O.Config(num_heads=6, num_heads_kv=2, dim_head=128, topk_decode=k, chunk_size=C, r_dim=r)
    q, K, V = rkvgen.stage2_inputs(31 + L, 6, 2, 128, L)
    for w in (0, 3):
        Og, sel, nsel = run_gpu(q[None], K[None], V[None], L, cfg, cuda, w=w)
        check_against_oracle(q, K, V, L, cfg, Og[0], sel[0], nsel[0], w=w)


@pytest.mark.parametrize("bf16,C", [(True, 2), (True, 3), (False, 2), (True, 65)])
def test_stage2_nonfinite_keys(bf16, C, cuda):
    """Pages whose representative the reference clamps (rocket.cpp:261-278:
    the max starts at -FLT_MAX, the min at +FLT_MAX, NaN never wins): all rows
    NaN or all rows infinite on a selected dimension, a single NaN row, and
    NaN / inf on dimensions outside the top r.  Selected indices must equal the
    oracle's; O is compared with NaN == NaN."""
    L, r = 601, 40
    cfg = O.Config(num_heads=6, num_heads_kv=2, dim_head=128, topk_decode=64, chunk_size=C, r_dim=r)
    q, K, V = rkvgen.stage2_inputs(4242 + C, 6, 2, 128, L)
    q = rkvgen.bf16_round(q * np.float32(0.05))  # keeps q * FLT_MAX finite
    K = K.copy()
    for hk in range(2):
        qg = q[hk * 3:(hk + 1) * 3]
        sabs = np.abs(qg).sum(0)
        top = sorted(range(128), key=lambda d: (-sabs[d], d))
        sd, ud = top[:r], top[r:]
        pos = qg.sum(0) >= 0
        rows = lambda p: slice(p * C, min(p * C + C, L))
        K[hk, rows(2), sd[0]] = np.nan                                  # all NaN
        K[hk, rows(4), sd[1]] = -np.inf if pos[sd[1]] else np.inf       # clamped to -/+FLT_MAX
        K[hk, 6 * C, sd[2]] = np.nan                                    # one NaN row
        K[hk, rows(7), ud[0]] = np.nan                                  # outside the top r
        K[hk, 8 * C, ud[1]] = np.inf
        K[hk, 8 * C, ud[2]] = -np.inf
    Og, sel, nsel = run_gpu(q[None], K[None], V[None], L, cfg, cuda, bf16=bf16)
    check_against_oracle(q, K, V, L, cfg, Og[0], sel[0], nsel[0], bf16=bf16)


def test_stage2_headline_batch_properties(cuda):
    """Headline geometry (3685 + 32 tokens, k 512, page 2, r 71) on a batch of
    items: structural properties on every unit, the oracle on a sample."""
    import torch
    B, L, w = 24, 3717, 32
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=512, chunk_size=2, r_dim=71,
                   compression_ratio=3.6298828125)
    g = torch.Generator(device=cuda).manual_seed(7)
    Q = torch.randn((B, 24, 128), generator=g, device=cuda).to(torch.bfloat16)
    K = torch.randn((B, 8, L, 128), generator=g, device=cuda).to(torch.bfloat16)
    V = torch.randn((B, 8, L, 128), generator=g, device=cuda).to(torch.bfloat16)
    d = rkv.HsaDecoder(to_rkv(cfg), L, B, cuda, recent_window=w)
    d(Q, K, V)
    torch.cuda.synchronize()
    sel, nsel = d.sel.cpu().numpy(), d.n_sel.cpu().numpy()
    assert np.all(nsel == 512 + w)
    assert np.all(np.diff(sel, axis=2) > 0)
    assert np.all(sel[:, :, -w:] == np.arange(L - w, L))
    for b in (0, B // 2, B - 1):
        q = Q[b].float().cpu().numpy()
        Kb, Vb = K[b].float().cpu().numpy(), V[b].float().cpu().numpy()
        check_against_oracle(q, Kb, Vb, L, cfg, d.O[b].cpu().numpy(), sel[b], nsel[b], w=w)


def test_bounded_wait_runs_out_and_reports(cuda):
    """Failure path without a GPU fault: a kernel waits on a barrier nothing
    completes; the bounded wait gives up (about two seconds), the status is
    RKV_ERR_DEVICE_TIMEOUT, and the context still runs a decode correctly."""
    import torch
    ws = torch.zeros(64, dtype=torch.uint8, device=cuda)
    assert rkv.lib().rkv_selftest_wait_timeout(rkv._ptr(ws), 0) == 0
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ws), 0) == rkv.RKV_ERR_DEVICE_TIMEOUT
    assert rkv.lib().rkv_workspace_status(rkv._ptr(ws), 0) == 0  # reading the status clears it
    p = dict(cases.STAGE2)["s2_mha_d64"]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    Og, sel, nsel = run_gpu(q[None], K[None], V[None], p["L"], cfg, cuda, bf16=p["bf16"])
    check_against_oracle(q, K, V, p["L"], cfg, Og[0], sel[0], nsel[0], bf16=p["bf16"])


def test_stage2_headline_items_vs_reference(cuda):
    """The headline geometry (3685 tokens, k 512, page 2, r 71) with the
    reference's semantics (no recent window) on 8 items: GPU selections equal
    the oracle's, the oracle's O equals the reference rocket.cpp's bit for bit
    (outside groups with an exact top-r tie), so the GPU selections are the
    reference's own; GPU O within 1e-3 / 1e-4 of rocket.cpp.  The smallest
    float64 boundary gap over the units is printed."""
    from test_oracle import assert_matches_reference
    if not O.have_ref():
        pytest.skip("oracle/_ref not built (no reference sources)")
    L = 3685
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=512, chunk_size=2, r_dim=71,
                   compression_ratio=3.6298828125)
    items = [rkvgen.stage2_inputs(7000 + 3 * i, 24, 8, 128, L) for i in range(8)]
    qs, Ks, Vs = (np.stack([it[j] for it in items]) for j in range(3))
    Og, sel, nsel = run_gpu(qs, Ks, Vs, L, cfg, cuda)
    gaps = []
    for b in range(len(items)):
        Oo = check_against_oracle(qs[b], Ks[b], Vs[b], L, cfg, Og[b], sel[b], nsel[b])
        Oref = O.ref_hsa_decode(qs[b], Ks[b], Vs[b], L, cfg)
        assert_matches_reference(Oo, Oref, qs[b], cfg, L)
        np.testing.assert_allclose(Og[b], Oref, rtol=RTOL, atol=ATOL)
        gaps += [stage2_boundary_gap(qs[b], Ks[b], cfg, L, 0, h) for h in range(8)]
    print(f"smallest float64 boundary gap over {len(gaps)} units: {min(gaps):.3e}")


@pytest.mark.parametrize("C", [3, 4, 5, 8, 16])
def test_stage2_scan_ring_refill(C, cuda):
    """Enough units for one scan CTA per unit and a cache long enough that the
    K-row ring is refilled many times, at page sizes whose scan groups (one or
    two warps per stage) take stages in turn: every unit's selection equals
    the oracle's and O is within tolerance."""
    import torch
    B, L, w = 40, 1024, 8
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=160, chunk_size=C, r_dim=37)
    g = torch.Generator(device=cuda).manual_seed(300 + C)
    Q = torch.randn((B, 24, 128), generator=g, device=cuda).to(torch.bfloat16)
    K = torch.randn((B, 8, L, 128), generator=g, device=cuda).to(torch.bfloat16)
    V = torch.randn((B, 8, L, 128), generator=g, device=cuda).to(torch.bfloat16)
    d = rkv.HsaDecoder(to_rkv(cfg), L, B, cuda, recent_window=w)
    d(Q, K, V)
    torch.cuda.synchronize()
    assert d.status() == 0
    sel, nsel, Og = d.sel.cpu().numpy(), d.n_sel.cpu().numpy(), d.O.cpu().numpy()
    Qh, Kh, Vh = Q.float().cpu().numpy(), K.float().cpu().numpy(), V.float().cpu().numpy()
    for b in range(B):
        check_against_oracle(Qh[b], Kh[b], Vh[b], L, cfg, Og[b], sel[b], nsel[b], w=w)
