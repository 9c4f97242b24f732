"""rkv_hsa_decode_noalloc: stage-2 decode without any device allocation.

Callers that cannot allocate device memory -- an inference server or plugin
host whose allocator owns the whole device heap, or a hot loop that cannot
accept cudaMalloc's implicit synchronisation -- use this entry point instead
of rkv_hsa_decode.  Its scratch is a fixed 4 MiB array inside the library.
The tests call it twice in a row through the C ABI and compare each result
with the workspace entry point's on the same inputs, read its status call
after each, and check that warmed-up calls leave the device's free memory and
torch's allocator untouched.  This file sorts last so that a run stopping at
its first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import rocketkv_b200 as rkv

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4


def _inputs(torch, device, seed, B, H, HK, D, L, dtype):
    g = torch.Generator(device=device).manual_seed(seed)
    Q = torch.randn((B, H, D), generator=g, device=device).to(dtype)
    K = torch.randn((B, HK, L, D), generator=g, device=device).to(dtype)
    V = torch.randn((B, HK, L, D), generator=g, device=device).to(dtype)
    return Q, K, V


def _noalloc(torch, cfg, L, w, Q, K, V, O, sel, nsel, dt):
    B, HK = K.shape[0], K.shape[1]
    c = cfg.c()
    return rkv.lib().rkv_hsa_decode_noalloc(Q.data_ptr(), K.data_ptr(), V.data_ptr(), dt, L, w, B, Q[0].nbytes,
                                            K[0].nbytes, ctypes.byref(c), 0, HK, O.data_ptr(), sel.data_ptr(),
                                            sel.shape[2], nsel.data_ptr(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("kind", ["bf16", "f32"])
def test_noalloc_matches_workspace_entry_point(cuda, kind):
    import torch

    if kind == "bf16":
        B, H, HK, D, L, w = 4, 24, 8, 128, 2048, 32
        cfg = rkv.RocketConfig(num_heads=H, num_heads_kv=HK, dim_head=D, topk_decode=256, chunk_size=16,
                               r_dim=32, compression_ratio=4.0)
        dtype, dt = torch.bfloat16, rkv.BF16
    else:  # a small fp32 geometry
        B, H, HK, D, L, w = 2, 8, 2, 64, 700, 16
        cfg = rkv.RocketConfig(num_heads=H, num_heads_kv=HK, dim_head=D, topk_decode=96, chunk_size=8,
                               r_dim=20, compression_ratio=4.0)
        dtype, dt = torch.float32, rkv.F32
    assert rkv.hsa_workspace_size(cfg, L, w, B, HK) <= 4 << 20
    cap = rkv.hsa_sel_capacity(cfg, L, w)
    for call, seed in enumerate((11, 12)):  # two calls in a row share the scratch
        Q, K, V = _inputs(torch, cuda, seed + 10 * (kind == "f32"), B, H, HK, D, L, dtype)
        ref = rkv.HsaDecoder(cfg, L, B, cuda, recent_window=w)
        ref(Q, K, V)
        O = torch.zeros((B, H, D), dtype=torch.float32, device=cuda)
        sel = torch.zeros((B, HK, cap), dtype=torch.int32, device=cuda)
        nsel = torch.zeros((B, HK), dtype=torch.int32, device=cuda)
        st = _noalloc(torch, cfg, L, w, Q, K, V, O, sel, nsel, dt)
        assert st == rkv.RKV_OK, (call, rkv.status_string(st))
        st = rkv.lib().rkv_hsa_decode_noalloc_status(torch.cuda.current_stream().cuda_stream)
        assert st == rkv.RKV_OK, (call, rkv.status_string(st))
        np.testing.assert_array_equal(nsel.cpu().numpy(), ref.n_sel.cpu().numpy())
        np.testing.assert_array_equal(sel.cpu().numpy(), ref.sel.cpu().numpy())
        np.testing.assert_allclose(O.cpu().numpy(), ref.O.cpu().numpy(), rtol=RTOL, atol=ATOL)


def test_noalloc_calls_allocate_nothing(cuda):
    """Once the library's module is loaded (the first call), further calls
    change neither the device's free memory nor torch's allocator."""
    import torch

    B, H, HK, D, L, w = 4, 24, 8, 128, 2048, 32
    cfg = rkv.RocketConfig(num_heads=H, num_heads_kv=HK, dim_head=D, topk_decode=256, chunk_size=16, r_dim=32,
                           compression_ratio=4.0)
    cap = rkv.hsa_sel_capacity(cfg, L, w)
    Q, K, V = _inputs(torch, cuda, 21, B, H, HK, D, L, torch.bfloat16)
    O = torch.zeros((B, H, D), dtype=torch.float32, device=cuda)
    sel = torch.zeros((B, HK, cap), dtype=torch.int32, device=cuda)
    nsel = torch.zeros((B, HK), dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    assert _noalloc(torch, cfg, L, w, Q, K, V, O, sel, nsel, rkv.BF16) == rkv.RKV_OK  # warm-up
    assert rkv.lib().rkv_hsa_decode_noalloc_status(stream) == rkv.RKV_OK
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda)
    stats0 = torch.cuda.memory_stats(cuda).get("allocation.all.allocated", 0)
    for _ in range(3):
        assert _noalloc(torch, cfg, L, w, Q, K, V, O, sel, nsel, rkv.BF16) == rkv.RKV_OK
    assert rkv.lib().rkv_hsa_decode_noalloc_status(stream) == rkv.RKV_OK
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda)
    stats1 = torch.cuda.memory_stats(cuda).get("allocation.all.allocated", 0)
    assert free1 == free0, (free0, free1)
    assert stats1 == stats0, (stats0, stats1)


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    cfg = rkv.RocketConfig(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=512, chunk_size=2,
                           r_dim=71, compression_ratio=3.6298828125)
    B, L = 512, 3717  # about 120 MiB of scratch: over the fixed 4 MiB
    assert rkv.hsa_workspace_size(cfg, L, 32, B, 8) > 4 << 20
    c = cfg.c()
    st = rkv.lib().rkv_hsa_decode_noalloc(None, None, None, rkv.BF16, L, 32, B, 24 * 128 * 2,
                                          8 * L * 128 * 2, ctypes.byref(c), 0, 8, None, None, 0, None, None)
    # the size check comes first: nothing is read, written or launched
    assert st == rkv.RKV_ERR_WORKSPACE
