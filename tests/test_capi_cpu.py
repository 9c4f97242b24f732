"""The C-ABI library loads here (no GPU), exports every symbol include/rkv.h
declares, and its host-only entry points behave (no kernel is launched)."""
import ctypes
import os
import re

import numpy as np
import pytest

import rocketkv_b200 as rkv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "rkv.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(rkv_[a-z0-9_]+)\s*\(", txt)))


def test_library_loads_and_exports_header():
    L = rkv.lib()
    syms = header_symbols()
    assert len(syms) >= 16
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(rkv.EXPORTS) == syms


def test_rocket_h_symbols_exported():
    """The C++ drop-in (rocket.h:36-50) lives in the same library."""
    L = ctypes.CDLL(rkv.LIB_PATH)
    for mangled in ("_Z21compute_rocket_paramsiiiii",
                    "_Z24compute_prefill_evictionPKfS0_iiRK12RocketConfig",
                    "_Z28compute_hybrid_sparse_decodePKfS0_S0_iRK12RocketConfig"):
        assert hasattr(L, mangled), mangled


def test_abi_version_and_status_strings():
    assert rkv.lib().rkv_abi_version() == 1
    assert rkv.status_string(0) == "ok"
    assert "invalid" in rkv.status_string(1)


@pytest.mark.parametrize("S,cap,prompt,k,chunk,r", [(8192, 3717, 3685, 512, 2, 71), (16384, 4837, 4805, 512, 3, 81)])
def test_compute_params_known_answers(S, cap, prompt, k, chunk, r):
    p = rkv.compute_rocket_params(1024, S, 32, 128)
    assert (p.capacity_budget, p.prompt_budget, p.k, p.chunk_size, p.r) == (cap, prompt, k, chunk, r)


def test_compute_params_golden_grid():
    for g, want in zip(GOLD["params/in"], GOLD["params/out"]):
        p = rkv.compute_rocket_params(*[int(x) for x in g])
        got = [p.token_budget, p.sequence_length, p.max_new_tokens, p.capacity_budget, p.prompt_budget,
               p.chunk_size, p.r, p.k, int(np.float32(p.compression_ratio).view(np.int32))]
        assert got == [int(x) for x in want], g


def test_sizes_and_argument_errors():
    cfg = rkv.RocketConfig(num_heads=24, num_heads_kv=8, dim_head=128, prompt_budget=1024)
    assert rkv.evict_max_kept(cfg, 8192, 8192) == 1024
    assert rkv.evict_max_kept(cfg, 8192, 900) == 900          # len_k <= budget: keep all
    assert rkv.evict_max_kept(rkv.RocketConfig(24, 8, 128, prompt_budget=10), 64, 100) == 32
    assert rkv.evict_workspace_size(cfg, rkv.F32, 8192, 8192, 1) > 8 * 96 * 8160 * 4
    with pytest.raises(rkv.RkvError):
        rkv.evict_max_kept(rkv.RocketConfig(num_heads=24, num_heads_kv=0, dim_head=128), 10, 10)
    c2 = rkv.RocketConfig(num_heads=24, num_heads_kv=8, dim_head=128, topk_decode=512, chunk_size=2, r_dim=71)
    assert rkv.hsa_sel_capacity(c2, 3717, 32) == 544
    assert rkv.hsa_sel_capacity(c2, 100, 32) == 100
    assert rkv.hsa_workspace_size(c2, 3717, 32, 4, 8) > 4 * 8 * 3 * 1843 * 4


CHECK = os.path.join(ROOT, "tests", "_bin", "rocket_h_check")


def _check(mode, d):
    import subprocess
    assert os.path.exists(CHECK), f"{CHECK} missing: make -C tests"
    r = subprocess.run([CHECK, mode, str(d)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    return r.stdout


def test_rocket_h_cpp_params_golden_grid(tmp_path):
    """rocket.h's compute_rocket_params called from C++ (tests/rocket_h_check.cpp)
    on part of the golden grid of the reference's outputs."""
    for g, want in list(zip(GOLD["params/in"], GOLD["params/out"]))[::37]:
        (tmp_path / "args.txt").write_text(" ".join(str(int(x)) for x in g) + "\n")
        _check("params", tmp_path)
        f = (tmp_path / "params.txt").read_text().split()
        got = [int(x) for x in f[:8]] + [int(np.float32(float(f[8])).view(np.int32))]
        assert got == [int(x) for x in want], g


def test_rocket_h_cpp_invalid_config_throws(tmp_path):
    """A config the reference cannot size raises std::invalid_argument through
    rocket.h (its return type carries no status); no device is touched."""
    assert _check("bad", tmp_path).strip() == "invalid_argument"
