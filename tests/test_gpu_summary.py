"""Stage 2 with persistent page summaries (rkv_hsa_build_summary +
rkv_hsa_decode_summary): the page scoring reads the per-page extrema of K
instead of every K row; selected indices, their counts and O must equal the
stateless rkv_hsa_decode bit for bit, and the selection the oracle's."""
import numpy as np
import pytest

import cases
import oracle as O
import rkvgen
import rocketkv_b200 as rkv
from gpuutil import dev

pytestmark = pytest.mark.gpu


def to_rkv(cfg):
    return rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__})


def both_paths(Q, K, V, L, cfg, device, w=0, head_begin=0, head_count=None):
    import torch
    d = rkv.HsaDecoder(to_rkv(cfg), L, Q.shape[0], device, recent_window=w, head_begin=head_begin,
                       head_count=head_count)
    d(Q, K, V)
    torch.cuda.synchronize()
    ref = (d.O.cpu().numpy().copy(), d.sel.cpu().numpy().copy(), d.n_sel.cpu().numpy().copy())
    S = d.build_summary(K)
    d.O.zero_()
    d.sel.zero_()
    d.n_sel.zero_()
    d(Q, K, V, summary=S)
    torch.cuda.synchronize()
    assert d.status() == 0
    got = (d.O.cpu().numpy(), d.sel.cpu().numpy(), d.n_sel.cpu().numpy())
    np.testing.assert_array_equal(got[2], ref[2])
    np.testing.assert_array_equal(got[1], ref[1])
    np.testing.assert_array_equal(got[0], ref[0])
    return got


def _dev(a, bf16, device):
    return dev(rkvgen.bf16_bits(a) if bf16 else a, "bf16" if bf16 else "f32", device)


@pytest.mark.parametrize("name", [n for n, _ in cases.STAGE2])
@pytest.mark.parametrize("w", [0, 32])
def test_summary_matches_stateless_and_oracle(name, w, cuda):
    p = dict(cases.STAGE2)[name]
    q, K, V = cases.stage2_build(p)
    cfg = cases.stage2_config(p)
    bf = p["bf16"]
    Og, sel, nsel = both_paths(_dev(q[None], bf, cuda), _dev(K[None], bf, cuda), _dev(V[None], bf, cuda), p["L"],
                               cfg, cuda, w=w)
    _, so = O.hsa_decode(q, K, V, p["L"], cfg, recent_window=w, kv_bytes=2 if bf else 4)
    for h in range(cfg.num_heads_kv):
        np.testing.assert_array_equal(sel[0, h, : nsel[0, h]], so[h])


@pytest.mark.parametrize("L,k,C,r", [(1, 1, 1, 1), (5, 0, 2, 8), (33, 32, 2, 8), (64, 1, 64, 128), (130, 17, 65, 3),
                                     (1001, 100, 7, 50)])
@pytest.mark.parametrize("bf16", [True, False])
def test_summary_edges(L, k, C, r, bf16, cuda):
    cfg = O.Config(num_heads=6, num_heads_kv=2, dim_head=128, topk_decode=k, chunk_size=C, r_dim=r)
    q, K, V = rkvgen.stage2_inputs(31 + L, 6, 2, 128, L)
    for w in (0, 3):
        both_paths(_dev(q[None], bf16, cuda), _dev(K[None], bf16, cuda), _dev(V[None], bf16, cuda), L, cfg, cuda, w=w)


@pytest.mark.parametrize("bf16,C", [(True, 2), (True, 3), (False, 2), (True, 65)])
def test_summary_nonfinite_keys(bf16, C, cuda):
    """All rows NaN or infinite on a selected dimension, one NaN row, NaN / inf
    outside the top r: the clamped representatives of the reference
    (rocket.cpp:261-278) from the summaries."""
    L, r = 601, 40
    cfg = O.Config(num_heads=6, num_heads_kv=2, dim_head=128, topk_decode=64, chunk_size=C, r_dim=r)
    q, K, V = rkvgen.stage2_inputs(4242 + C, 6, 2, 128, L)
    q = rkvgen.bf16_round(q * np.float32(0.05))
    K = K.copy()
    for hk in range(2):
        qg = q[hk * 3:(hk + 1) * 3]
        sabs = np.abs(qg).sum(0)
        top = sorted(range(128), key=lambda d: (-sabs[d], d))
        sd, ud = top[:r], top[r:]
        pos = qg.sum(0) >= 0
        rows = lambda p: slice(p * C, min(p * C + C, L))
        K[hk, rows(2), sd[0]] = np.nan
        K[hk, rows(4), sd[1]] = -np.inf if pos[sd[1]] else np.inf
        K[hk, 6 * C, sd[2]] = np.nan
        K[hk, rows(7), ud[0]] = np.nan
        K[hk, 8 * C, ud[1]] = np.inf
        K[hk, 8 * C, ud[2]] = -np.inf
    Og, sel, nsel = both_paths(_dev(q[None], bf16, cuda), _dev(K[None], bf16, cuda), _dev(V[None], bf16, cuda), L,
                               cfg, cuda)
    _, so = O.hsa_decode(q, K, V, L, cfg, kv_bytes=2 if bf16 else 4)
    for h in range(2):
        np.testing.assert_array_equal(sel[0, h, : nsel[0, h]], so[h])


def test_summary_headline_batch_head_subset(cuda):
    """Headline geometry (3685 + 32 tokens, k 512, page 2, r 71), a batch of
    items, and a KV-head subset (the head-sharded form): the summaries cover
    every head of an item, the decode reads its heads' part."""
    import torch
    B, L, w = 16, 3717, 32
    cfg = O.Config(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=512, chunk_size=2, r_dim=71,
                   compression_ratio=3.6298828125)
    g = torch.Generator(device=cuda).manual_seed(11)
    Q = torch.randn((B, 24, 128), generator=g, device=cuda).to(torch.bfloat16)
    K = torch.randn((B, 8, L, 128), generator=g, device=cuda).to(torch.bfloat16)
    V = torch.randn((B, 8, L, 128), generator=g, device=cuda).to(torch.bfloat16)
    both_paths(Q, K, V, L, cfg, cuda, w=w)
    both_paths(Q, K, V, L, cfg, cuda, w=w, head_begin=3, head_count=4)
    n = __import__("ctypes").c_size_t(0)
    assert rkv.lib().rkv_hsa_summary_size(__import__("ctypes").byref(to_rkv(cfg).c()), rkv.BF16, L, w, B,
                                          __import__("ctypes").byref(n)) == 0
    pages = (L - w + 1) // 2
    # per item: the extrema [KV head][2][D][pages rounded to 8] in bf16, then a mask word per 32 dimensions
    # and KV head (dimensions with an extremum of -inf or NaN), rounded to 16 bytes
    assert n.value == B * (8 * 2 * 128 * ((pages + 7) // 8 * 8) * 2 + 8 * 128 // 8)


def test_summary_survives_window_growth(cuda):
    """Summaries built for (len_k, window) serve later steps whose appended
    tokens joined the window (len_k + n, window + n): the compressed part, and
    so the summaries, are unchanged.  Same selections and O as the stateless
    call on the grown cache."""
    import torch
    B, L, w, n = 4, 1200, 8, 5
    cfg = to_rkv(O.Config(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=128, chunk_size=2, r_dim=40))
    g = torch.Generator(device=cuda).manual_seed(9)
    Q = torch.randn((B, 24, 128), generator=g, device=cuda).to(torch.bfloat16)
    K = torch.randn((B, 8, L + n, 128), generator=g, device=cuda).to(torch.bfloat16)
    V = torch.randn((B, 8, L + n, 128), generator=g, device=cuda).to(torch.bfloat16)
    S = rkv.HsaDecoder(cfg, L, B, cuda, recent_window=w).build_summary(K[:, :, :L].contiguous())
    d = rkv.HsaDecoder(cfg, L + n, B, cuda, recent_window=w + n)
    d(Q, K, V)
    torch.cuda.synchronize()
    ref = (d.O.cpu().numpy().copy(), d.sel.cpu().numpy().copy(), d.n_sel.cpu().numpy().copy())
    d.O.zero_()
    d.sel.zero_()
    d.n_sel.zero_()
    d(Q, K, V, summary=S)
    torch.cuda.synchronize()
    assert d.status() == 0
    np.testing.assert_array_equal(d.n_sel.cpu().numpy(), ref[2])
    np.testing.assert_array_equal(d.sel.cpu().numpy(), ref[1])
    np.testing.assert_array_equal(d.O.cpu().numpy(), ref[0])


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("G", [1, 2, 3, 4, 6])
@pytest.mark.parametrize("bf16", [True, False])
def test_summary_every_instantiation(D, G, bf16, cuda):
    """Every head size, group size (kernel templates 1, 2, 3, 4, 8) and element
    type of the summary scan, including fp32 at D 256 (two pages per lane):
    the same selections and O as the stateless call."""
    HK, L = 2, 333
    cfg = O.Config(num_heads=G * HK, num_heads_kv=HK, dim_head=D, topk_decode=40, chunk_size=3, r_dim=D // 3)
    q, K, V = rkvgen.stage2_inputs(100 + D + G, G * HK, HK, D, L)
    for w in (0, 5):
        both_paths(_dev(q[None], bf16, cuda), _dev(K[None], bf16, cuda), _dev(V[None], bf16, cuda), L, cfg, cuda, w=w)
