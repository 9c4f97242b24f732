"""Helpers shared by the GPU parity tests."""
import numpy as np


def dev(arr, kind, device):
    """numpy -> torch CUDA tensor.  kind: 'f32' (float32), 'bf16' (uint16 bit
    patterns viewed as bfloat16), 'q8_0' (uint8 rows)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if kind == "bf16":
        t = t.view(torch.bfloat16)
    return t.to(device)


def boundary_report(total, kept_a, kept_b):
    """Scores of the indices on which two kept lists disagree."""
    da = sorted(set(kept_a) - set(kept_b))
    db = sorted(set(kept_b) - set(kept_a))
    return {"only_a": [(i, float(total[i])) for i in da[:8]], "only_b": [(i, float(total[i])) for i in db[:8]]}


def stage2_boundary_gap(q, K, cfg, L, w, hk):
    """Relative gap, in float64, between the page score of the last selected
    token and the best page score left out, for KV head hk of one stage-2
    unit (the selection of rocket.cpp:197-340 over the first L - w tokens).
    A tiny gap marks a near-tie that another summation order could break the
    other way; inf when nothing is left out."""
    D = cfg.dim_head
    G = max(1, cfg.num_heads // cfg.num_heads_kv)
    C = cfg.chunk_size if cfg.chunk_size > 0 else max(1, min(int(np.floor(cfg.compression_ratio)),
                                                               int(np.ceil(np.sqrt(cfg.compression_ratio)))))
    r = cfg.r_dim if cfg.r_dim > 0 else min(D, max(1, int(round(D * C / cfg.compression_ratio))))
    Lc = L - w
    k = min(cfg.topk_decode, Lc)
    if k >= Lc or Lc <= 0:
        return float("inf")
    qg = q[hk * G:(hk + 1) * G].astype(np.float64)
    sabs = np.abs(qg).sum(0)
    dims = sorted(range(D), key=lambda d: (-sabs[d], d))[:r]
    pos = qg.sum(0) >= 0
    Kh = K[hk, :Lc].astype(np.float64)
    npg = (Lc + C - 1) // C
    rep = np.empty((npg, len(dims)))
    for i, d in enumerate(dims):
        col = Kh[:, d]
        pad = np.full(npg * C - Lc, -np.inf if pos[d] else np.inf)
        blk = np.concatenate([col, pad]).reshape(npg, C)
        rep[:, i] = blk.max(1) if pos[d] else blk.min(1)
    scale = np.sqrt(D * np.abs(qg[:, dims]).sum(1) / (np.abs(qg).sum(1) + 1e-9))
    logit = (qg[:, dims] @ rep.T) / scale[:, None]
    p = np.exp(logit - logit.max(1, keepdims=True))
    prob = (p / p.sum(1, keepdims=True)).sum(0)
    tok = np.repeat(prob, C)[:Lc]
    order = np.lexsort((np.arange(Lc), -tok))
    last, rest = tok[order[k - 1]], tok[order[k:]]
    below = rest[rest < last]
    if below.size == 0:
        return float("inf")
    return float((last - below.max()) / last)
