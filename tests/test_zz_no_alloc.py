"""rkv_hsa_decode_noalloc: stage-2 decode without any device allocation.

Callers that cannot allocate device memory -- an inference server or plugin
host whose allocator owns the whole device heap, or a hot loop that cannot
accept cudaMalloc's implicit synchronisation -- use this entry point instead
of rkv_hsa_decode.  Its scratch is a fixed 4 MiB array inside the library.
The test calls it twice in a row through the C ABI and compares each result
with the workspace entry point's on the same inputs.  This file sorts last so
that a run stopping at its first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import rocketkv_b200 as rkv

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4


def _inputs(torch, device, seed, B, H, HK, D, L):
    g = torch.Generator(device=device).manual_seed(seed)
    Q = torch.randn((B, H, D), generator=g, device=device).to(torch.bfloat16)
    K = torch.randn((B, HK, L, D), generator=g, device=device).to(torch.bfloat16)
    V = torch.randn((B, HK, L, D), generator=g, device=device).to(torch.bfloat16)
    return Q, K, V


def test_noalloc_matches_workspace_entry_point(cuda):
    import torch

    B, H, HK, D, L, w = 4, 24, 8, 128, 2048, 32
    cfg = rkv.RocketConfig(num_heads=H, num_heads_kv=HK, dim_head=D, topk_decode=256, chunk_size=16,
                           r_dim=32, compression_ratio=4.0)
    assert rkv.hsa_workspace_size(cfg, L, w, B, HK) <= 4 << 20
    c = cfg.c()
    cap = rkv.hsa_sel_capacity(cfg, L, w)
    L_ = rkv.lib()
    for call, seed in enumerate((11, 12)):  # two calls in a row share the scratch
        Q, K, V = _inputs(torch, cuda, seed, B, H, HK, D, L)
        ref = rkv.HsaDecoder(cfg, L, B, cuda, recent_window=w)
        ref(Q, K, V)
        O = torch.zeros((B, H, D), dtype=torch.float32, device=cuda)
        sel = torch.zeros((B, HK, cap), dtype=torch.int32, device=cuda)
        nsel = torch.zeros((B, HK), dtype=torch.int32, device=cuda)
        st = L_.rkv_hsa_decode_noalloc(Q.data_ptr(), K.data_ptr(), V.data_ptr(), rkv.BF16, L, w, B,
                                        Q[0].nbytes, K[0].nbytes, ctypes.byref(c), 0, HK, O.data_ptr(),
                                        sel.data_ptr(), cap, nsel.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
        assert st == rkv.RKV_OK, (call, rkv.status_string(st))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(nsel.cpu().numpy(), ref.n_sel.cpu().numpy())
        np.testing.assert_array_equal(sel.cpu().numpy(), ref.sel.cpu().numpy())
        np.testing.assert_allclose(O.cpu().numpy(), ref.O.cpu().numpy(), rtol=RTOL, atol=ATOL)


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
