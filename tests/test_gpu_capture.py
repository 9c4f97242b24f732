"""The capture side on the device (rkv_capture_rows): post-RoPE Q and K rows
taken from the producing attention's token-major buffers, micro-batch by
micro-batch and layer by layer, into stage 1's head-major layout with no host
copy -- the device analogue of the reference runner's eval callback
(runner.cpp:25-92) -- then every captured layer scored in one rkv_evict call.
Captured rows are bit-exact against a host transposition (fp16 and bf16
convert to fp32 exactly); kept indices equal the oracle's per layer."""
import numpy as np
import pytest

import oracle as O
import rkvgen
import rocketkv_b200 as rkv

pytestmark = pytest.mark.gpu


def _tokmajor(torch, device, seed, n, heads, D, dtype):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn((n, heads, D), generator=g, device=device).to(dtype)


@pytest.mark.parametrize("dtype_name", ["f16", "bf16", "f32"])
def test_capture_layers_then_evict(dtype_name, cuda):
    import torch
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dtype_name]
    H, HK, D, N, w, layers, ub = 24, 8, 128, 1536, 32, 2, 512
    cfg = O.Config(num_heads=H, num_heads_kv=HK, dim_head=D, prompt_budget=384)
    # the producer's Q, K and V rows of one layer share a fused buffer: token stride (H + 2 HK) D
    fused = [_tokmajor(torch, cuda, 70 + l, N, H + 2 * HK, D, dt) for l in range(layers)]
    Qsrc = [f[:, :H] for f in fused]
    Ksrc = [f[:, H:H + HK] for f in fused]
    out_dt = torch.bfloat16 if dt == torch.bfloat16 else torch.float32
    Qd = torch.zeros((layers, H, w, D), dtype=out_dt, device=cuda)  # only the window rows
    Kd = torch.zeros((layers, HK, N, D), dtype=out_dt, device=cuda)
    for l in range(layers):
        for t0 in range(0, N, ub):  # micro-batches, as llama_decode feeds the eval callback
            rkv.capture_rows(Ksrc[l][t0:t0 + ub], Kd, t0, dst_first=0, item=l)
            rkv.capture_rows(Qsrc[l][t0:t0 + ub], Qd, t0, dst_first=N - w, item=l)
    torch.cuda.synchronize()
    for l in range(layers):
        k_ref = Ksrc[l].float().permute(1, 0, 2).contiguous()
        q_ref = Qsrc[l][N - w:].float().permute(1, 0, 2).contiguous()
        assert torch.equal(Kd[l].float(), k_ref), l
        assert torch.equal(Qd[l].float(), q_ref), l
    ev = rkv.Evictor(rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}), w, N, layers,
                     rkv.BF16 if out_dt == torch.bfloat16 else rkv.F32, cuda)
    kept, n = ev(Qd, Kd)
    kept, n = kept.cpu().numpy(), n.cpu().numpy()
    for l in range(layers):
        want = O.prefill_eviction(Qd[l].float().cpu().numpy(), Kd[l].float().cpu().numpy(), w, N, cfg)
        assert np.array_equal(kept[l, : n[l]], want), l


def test_capture_skips_rows_outside_the_kept_range(cuda):
    import torch
    src = _tokmajor(torch, cuda, 5, 100, 4, 64, torch.float16)
    dst = torch.full((1, 4, 40, 64), -7.0, dtype=torch.float32, device=cuda)
    rkv.capture_rows(src, dst, token_offset=30, dst_first=50)  # tokens 30..129 -> rows of tokens 50..89
    torch.cuda.synchronize()
    ref = src.float().permute(1, 0, 2)[:, 20:60]
    assert torch.equal(dst[0], ref)


def test_capture_rejects_inexact_conversions(cuda):
    import torch
    src = _tokmajor(torch, cuda, 6, 8, 2, 64, torch.float16)
    dst = torch.zeros((1, 2, 8, 64), dtype=torch.bfloat16, device=cuda)  # fp16 -> bf16 would round
    with pytest.raises(rkv.RkvError) as e:
        rkv.capture_rows(src, dst, 0)
    assert e.value.status == rkv.RKV_ERR_UNSUPPORTED
