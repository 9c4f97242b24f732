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
