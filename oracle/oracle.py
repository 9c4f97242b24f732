"""ctypes front end of the oracle (TEST INFRASTRUCTURE).

Loads two CPU libraries built by oracle/Makefile:

* ``librkv_oracle.so`` -- the C restatement of RocketKV's kernels
  (rkv_oracle.c), with the deterministic tie rule and the exposed selections;
* ``_ref/librocket_ref[_omp].so`` -- the reference's own rocket.cpp, compiled
  unmodified from the reference sources (present only where they were built).

Only the tests, the smoke check and the benchmark's CPU-baseline leg import
this module.  The product library never does.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_F32P = ctypes.POINTER(ctypes.c_float)
_I32P = ctypes.POINTER(ctypes.c_int)


class RocketConfigC(ctypes.Structure):
    """Field-for-field image of RocketConfig (reference rocket.h:18-34)."""

    _fields_ = [
        ("num_heads", ctypes.c_int),
        ("num_heads_kv", ctypes.c_int),
        ("dim_head", ctypes.c_int),
        ("window_size", ctypes.c_int),
        ("kernel_size", ctypes.c_int),
        ("prompt_budget", ctypes.c_int),
        ("topk_decode", ctypes.c_int),
        ("chunk_size", ctypes.c_int),
        ("r_dim", ctypes.c_int),
        ("compression_ratio", ctypes.c_float),
    ]


class BudgetC(ctypes.Structure):
    """Image of RocketBudgetParams (reference rocket.h:5-15), field order kept."""

    _fields_ = [
        ("token_budget", ctypes.c_int),
        ("sequence_length", ctypes.c_int),
        ("max_new_tokens", ctypes.c_int),
        ("capacity_budget", ctypes.c_int),
        ("prompt_budget", ctypes.c_int),
        ("chunk_size", ctypes.c_int),
        ("r", ctypes.c_int),
        ("k", ctypes.c_int),
        ("compression_ratio", ctypes.c_float),
    ]


@dataclass
class Config:
    """Python mirror of RocketConfig; defaults follow rocket.h:25-26."""

    num_heads: int = 24
    num_heads_kv: int = 8
    dim_head: int = 128
    window_size: int = 32
    kernel_size: int = 63
    prompt_budget: int = 1024
    topk_decode: int = 256
    chunk_size: int = 16
    r_dim: int = 32
    compression_ratio: float = 4.0

    def c(self) -> RocketConfigC:
        return RocketConfigC(self.num_heads, self.num_heads_kv, self.dim_head,
                             self.window_size, self.kernel_size, self.prompt_budget,
                             self.topk_decode, self.chunk_size, self.r_dim,
                             ctypes.c_float(self.compression_ratio))


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F32P)


def _ip(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_I32P)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "librkv_oracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle`")
        L = ctypes.CDLL(path)
        L.rkvo_compute_params.argtypes = [ctypes.c_int] * 5 + [ctypes.POINTER(BudgetC)]
        L.rkvo_expf.argtypes = [ctypes.c_float]
        L.rkvo_expf.restype = ctypes.c_float
        L.rkvo_prefill_eviction.argtypes = [_F32P, _F32P, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(RocketConfigC), _I32P, _F32P]
        L.rkvo_evict_pool_heads.argtypes = [_F32P, _F32P, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(RocketConfigC), ctypes.c_int,
                                            ctypes.c_int, _F32P]
        L.rkvo_evict_select_pooled.argtypes = [_F32P, ctypes.c_int, ctypes.c_int,
                                               ctypes.POINTER(RocketConfigC), _I32P]
        L.rkvo_hsa_decode.argtypes = [_F32P, _F32P, _F32P, ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(RocketConfigC), _F32P, _I32P,
                                      ctypes.c_int, _I32P, ctypes.c_int]
        _lib = L
    return _lib


def compute_params(token_budget, seq_len, max_new, head_dim, window=32) -> dict:
    b = BudgetC()
    lib().rkvo_compute_params(token_budget, seq_len, max_new, head_dim, window, ctypes.byref(b))
    return {f: getattr(b, f) for f, _ in BudgetC._fields_}


def expf(x: float) -> float:
    return lib().rkvo_expf(x)


def max_kept(cfg: Config, len_q: int, len_k: int) -> int:
    return max(len_k, cfg.prompt_budget, min(cfg.window_size, len_q), 1)


def prefill_eviction(Q: np.ndarray, K: np.ndarray, len_q: int, len_k: int, cfg: Config,
                     want_total: bool = False):
    """Stage 1 restated (ties -> lower index). Returns kept indices (and totals)."""
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    out = np.zeros(max_kept(cfg, len_q, len_k), np.int32)
    nk = max(len_k - min(cfg.window_size, len_q), 0)
    tot = np.zeros(max(nk, 1), np.float32)
    c = cfg.c()
    n = lib().rkvo_prefill_eviction(_fp(Q), _fp(K), len_q, len_k, ctypes.byref(c), _ip(out),
                                    _fp(tot) if want_total else None)
    if n < 0:
        raise ValueError("invalid stage-1 sizes")
    kept = out[:n].copy()
    return (kept, tot[:nk]) if want_total else kept


def evict_pool_heads(Q, K, len_q, len_k, cfg: Config, h0: int, nh: int) -> np.ndarray:
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    nk = len_k - min(cfg.window_size, len_q)
    out = np.zeros((nh, max(nk, 1)), np.float32)
    c = cfg.c()
    lib().rkvo_evict_pool_heads(_fp(Q), _fp(K), len_q, len_k, ctypes.byref(c), h0, nh, _fp(out))
    return out[:, :nk]


def evict_select_pooled(pooled: np.ndarray, len_q: int, len_k: int, cfg: Config) -> np.ndarray:
    pooled = np.ascontiguousarray(pooled, np.float32)
    out = np.zeros(max_kept(cfg, len_q, len_k), np.int32)
    c = cfg.c()
    n = lib().rkvo_evict_select_pooled(_fp(pooled), len_q, len_k, ctypes.byref(c), _ip(out))
    return out[:n].copy()


def hsa_decode(Q, K, V, len_k: int, cfg: Config, recent_window: int = 0, kv_bytes: int = 2):
    """Stage 2 restated.  Returns (O [H, D], list of per-KV-head selected indices).
    kv_bytes: element size of K in the GPU run being checked (2 bf16, 4 fp32);
    it fixes the page-logit summation order."""
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    O = np.zeros((cfg.num_heads, cfg.dim_head), np.float32)
    stride = max(len_k, 1)
    sel = np.zeros((cfg.num_heads_kv, stride), np.int32)
    nsel = np.zeros(cfg.num_heads_kv, np.int32)
    c = cfg.c()
    rc = lib().rkvo_hsa_decode(_fp(Q), _fp(K), _fp(V), len_k, recent_window, ctypes.byref(c),
                               _fp(O), _ip(sel), stride, _ip(nsel), kv_bytes)
    if rc != 0:
        raise ValueError(f"unsupported stage-2 shape: dim_head {cfg.dim_head}, kv_bytes {kv_bytes}")
    return O, [sel[h, :nsel[h]].copy() for h in range(cfg.num_heads_kv)]


# ---------------------------------------------------------------------------
# The reference itself (oracle/_ref), where it was built.
# ---------------------------------------------------------------------------
_ref = {}


def ref_path(omp: bool = False) -> str:
    return os.path.join(HERE, "_ref", "librocket_ref_omp.so" if omp else "librocket_ref.so")


def have_ref(omp: bool = False) -> bool:
    return os.path.exists(ref_path(omp))


def ref(omp: bool = False) -> ctypes.CDLL:
    if omp not in _ref:
        L = ctypes.CDLL(ref_path(omp))
        L.rkvref_compute_params.argtypes = [ctypes.c_int] * 5 + [ctypes.c_void_p]
        L.rkvref_sizeof_budget_params.restype = ctypes.c_int
        L.rkvref_prefill_eviction.argtypes = [_F32P, _F32P, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p, _I32P]
        L.rkvref_prefill_eviction.restype = ctypes.c_int
        L.rkvref_hsa_decode.argtypes = [_F32P, _F32P, _F32P, ctypes.c_int, ctypes.c_void_p, _F32P]
        L.rkvref_hsa_decode.restype = ctypes.c_int
        L.rkvref_max_threads.restype = ctypes.c_int
        L.rkvref_set_threads.argtypes = [ctypes.c_int]
        _ref[omp] = L
    return _ref[omp]


def ref_compute_params(token_budget, seq_len, max_new, head_dim, window=32, omp=False) -> dict:
    L = ref(omp)
    assert L.rkvref_sizeof_budget_params() == ctypes.sizeof(BudgetC)
    b = BudgetC()
    L.rkvref_compute_params(token_budget, seq_len, max_new, head_dim, window, ctypes.byref(b))
    return {f: getattr(b, f) for f, _ in BudgetC._fields_}


def ref_prefill_eviction(Q, K, len_q, len_k, cfg: Config, omp=False) -> np.ndarray:
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    out = np.zeros(max_kept(cfg, len_q, len_k), np.int32)
    c = cfg.c()
    n = ref(omp).rkvref_prefill_eviction(_fp(Q), _fp(K), len_q, len_k, ctypes.byref(c), _ip(out))
    return out[:n].copy()


def ref_hsa_decode(Q, K, V, len_k, cfg: Config, omp=False) -> np.ndarray:
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    O = np.zeros((cfg.num_heads, cfg.dim_head), np.float32)
    c = cfg.c()
    ref(omp).rkvref_hsa_decode(_fp(Q), _fp(K), _fp(V), len_k, ctypes.byref(c), _fp(O))
    return O


# ---------------------------------------------------------------------------
# Input formats: the oracle always sees exact fp32 images of bf16 / q8_0 data.
# ---------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


Q8_BLOCK = 32
Q8_BYTES = 34  # {fp16 scale; int8 qs[32]}, the layout of ggml's block_q8_0


def q8_0_pack(scales: np.ndarray, qs: np.ndarray) -> np.ndarray:
    """scales [..., nb] float16, qs [..., nb, 32] int8 -> uint8 [..., nb*34]."""
    nb = scales.shape[-1]
    lead = scales.shape[:-1]
    out = np.zeros(lead + (nb, Q8_BYTES), np.uint8)
    out[..., 0:2] = np.ascontiguousarray(scales.astype(np.float16)).view(np.uint8).reshape(lead + (nb, 2))
    out[..., 2:] = qs.astype(np.int8).view(np.uint8)
    return out.reshape(lead + (nb * Q8_BYTES,))


def q8_0_dequant(packed: np.ndarray, dim: int) -> np.ndarray:
    """uint8 [..., dim/32*34] -> float32 [..., dim]; fp32(scale) * int8 is exact."""
    nb = dim // Q8_BLOCK
    lead = packed.shape[:-1]
    b = packed.reshape(lead + (nb, Q8_BYTES))
    d = np.ascontiguousarray(b[..., 0:2]).view(np.float16).reshape(lead + (nb, 1)).astype(np.float32)
    q = np.ascontiguousarray(b[..., 2:]).view(np.int8).astype(np.float32)
    return (d * q).reshape(lead + (dim,)).astype(np.float32)
