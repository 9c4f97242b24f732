"""Writes tests/golden/golden.npz: outputs of the REFERENCE rocket.cpp,
compiled unmodified into oracle/_ref/ by oracle/Makefile, on the cases of
cases.py.  Run from the repository root after `make -C oracle`:

    python tests/golden/gen_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden"), os.path.join(ROOT, "oracle")]

import cases  # noqa: E402
import oracle  # noqa: E402


def main():
    if not oracle.have_ref():
        sys.exit("oracle/_ref/librocket_ref.so not built (make -C oracle)")
    out = {}
    params = np.array([list(g) for g in cases.PARAM_GRID], np.int32)
    res = []
    for g in cases.PARAM_GRID:
        r = oracle.ref_compute_params(*g)
        res.append([r["token_budget"], r["sequence_length"], r["max_new_tokens"], r["capacity_budget"],
                    r["prompt_budget"], r["chunk_size"], r["r"], r["k"],
                    np.float32(r["compression_ratio"]).view(np.int32)])
    out["params/in"] = params
    out["params/out"] = np.array(res, np.int64)
    for name, p in cases.STAGE1:
        Q, K, _ = cases.stage1_build(p)
        kept = oracle.ref_prefill_eviction(Q, K, p["len_q"], p["len_k"], cases.stage1_config(p))
        out[f"{name}/kept"] = kept.astype(np.int32)
        print(name, len(kept))
    for name, p in cases.STAGE2:
        q, K, V = cases.stage2_build(p)
        O = oracle.ref_hsa_decode(q, K, V, p["L"], cases.stage2_config(p))
        out[f"{name}/O"] = O.astype(np.float32)
        print(name, float(np.abs(O).max()))
    np.savez_compressed(os.path.join(ROOT, "tests", "golden", "golden.npz"), **out)


if __name__ == "__main__":
    main()
