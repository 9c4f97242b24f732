"""Python front end of librkv_b200.so (the C ABI in include/rkv.h).

This module mirrors the reference's rocket.h interface for Python callers
(tests, benchmark, torch.distributed drivers): ``compute_rocket_params``,
``compute_prefill_eviction`` and ``compute_hybrid_sparse_decode`` with the
reference's argument meaning, plus the device-resident batched entry points
that take torch CUDA tensors.  Every call goes through the CUDA library; if
the library is missing, loading raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, fields

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librkv_b200.so")

RKV_OK = 0
RKV_ERR_INVALID_ARG = 1
RKV_ERR_UNSUPPORTED = 2
RKV_ERR_CUDA = 3
RKV_ERR_WORKSPACE = 4
RKV_ERR_DEVICE_TIMEOUT = 5
RKV_ERR_NO_DEVICE = 6

F32, BF16, Q8_0, F16 = 0, 1, 2, 3
ENGINE_AUTO, ENGINE_SIMT, ENGINE_TENSOR, ENGINE_TENSOR_TILES = 0, 1, 2, 3

# Every symbol include/rkv.h declares.
EXPORTS = [
    "rkv_abi_version", "rkv_status_string", "rkv_config_init", "rkv_compute_params",
    "rkv_evict_max_kept", "rkv_evict_workspace_size", "rkv_evict", "rkv_evict_pool_heads",
    "rkv_evict_select_pooled", "rkv_prefill_eviction_host", "rkv_hsa_sel_capacity",
    "rkv_hsa_workspace_size", "rkv_hsa_decode", "rkv_hybrid_sparse_decode_host",
    "rkv_hsa_decode_host_ex", "rkv_workspace_status", "rkv_hsa_decode_noalloc", "rkv_hsa_decode_noalloc_status",
    "rkv_selftest_wait_timeout", "rkv_compact_kv", "rkv_hsa_summary_size", "rkv_hsa_build_summary",
    "rkv_hsa_decode_summary", "rkv_capture_rows", "rkv_evict_compact",
]


class RkvError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "num_heads", "num_heads_kv", "dim_head", "window_size", "kernel_size",
        "prompt_budget", "topk_decode", "chunk_size", "r_dim")] + [("compression_ratio", ctypes.c_float)]


class _Budget(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "token_budget", "sequence_length", "max_new_tokens", "capacity_budget",
        "prompt_budget", "chunk_size", "r", "k")] + [("compression_ratio", ctypes.c_float)]


@dataclass
class RocketConfig:
    """Mirror of the reference RocketConfig (rocket.h:18-34); same defaults."""

    num_heads: int = 0
    num_heads_kv: int = 0
    dim_head: int = 0
    window_size: int = 32
    kernel_size: int = 63
    prompt_budget: int = 0
    topk_decode: int = 0
    chunk_size: int = 0
    r_dim: int = 0
    compression_ratio: float = 0.0

    def c(self) -> _Config:
        return _Config(*[getattr(self, f.name) for f in fields(self)])


@dataclass
class RocketBudgetParams:
    """Mirror of the reference RocketBudgetParams (rocket.h:5-15)."""

    token_budget: int
    sequence_length: int
    max_new_tokens: int
    capacity_budget: int
    prompt_budget: int
    chunk_size: int
    r: int
    k: int
    compression_ratio: float


_lib = None
_VP = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t
_CFGP = ctypes.POINTER(_Config)


def lib() -> ctypes.CDLL:
    """Loads librkv_b200.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(
            f"{LIB_PATH} is missing; build it with `make -C rocketkv-cpp_b200` "
            "(the CUDA library is required, there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    sig = {
        "rkv_abi_version": ([], _I),
        "rkv_status_string": ([_I], ctypes.c_char_p),
        "rkv_config_init": ([_CFGP], None),
        "rkv_compute_params": ([_I, _I, _I, _I, _I, ctypes.POINTER(_Budget)], _I),
        "rkv_evict_max_kept": ([_CFGP, _I, _I], _I),
        "rkv_evict_workspace_size": ([_CFGP, _I, _I, _I, _I, ctypes.POINTER(_SZ)], _I),
        "rkv_evict": ([_VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _VP, _I, _VP, _VP, _SZ, _I, _VP], _I),
        "rkv_evict_pool_heads": ([_VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _I, _I, _VP, _VP, _SZ, _I, _VP], _I),
        "rkv_evict_select_pooled": ([_VP, _I, _I, _I, _CFGP, _VP, _I, _VP, _VP, _SZ, _VP], _I),
        "rkv_prefill_eviction_host": ([_VP, _VP, _I, _I, _CFGP, _VP, _I, ctypes.POINTER(_I)], _I),
        "rkv_hsa_sel_capacity": ([_CFGP, _I, _I], _I),
        "rkv_hsa_workspace_size": ([_CFGP, _I, _I, _I, _I, ctypes.POINTER(_SZ)], _I),
        "rkv_hsa_decode": ([_VP, _VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _I, _I, _VP, _VP, _I, _VP,
                            _VP, _SZ, _VP], _I),
        "rkv_hybrid_sparse_decode_host": ([_VP, _VP, _VP, _I, _CFGP, _VP], _I),
        "rkv_hsa_decode_host_ex": ([_VP, _VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _VP, _VP, _I, _VP], _I),
        "rkv_workspace_status": ([_VP, _VP], _I),
        "rkv_selftest_wait_timeout": ([_VP, _VP], _I),
        "rkv_hsa_decode_noalloc": ([_VP, _VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _I, _I, _VP, _VP, _I, _VP,
                                    _VP], _I),
        "rkv_hsa_decode_noalloc_status": ([_VP], _I),
        "rkv_capture_rows": ([_VP, _I, _I, _I, _I, _LL, _LL, _I, _VP, _I, _I, _I, _LL, _I, _VP], _I),
        "rkv_evict_compact": ([_VP, _VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _VP, _I, _VP, _VP, _VP, _I, _LL,
                               _VP, _SZ, _I, _VP], _I),
        "rkv_compact_kv": ([_VP, _VP, _I, _I, _I, _I, _I, _LL, _VP, _VP, _I, _VP, _VP, _I, _LL, _VP], _I),
        "rkv_hsa_summary_size": ([_CFGP, _I, _I, _I, _I, ctypes.POINTER(_SZ)], _I),
        "rkv_hsa_build_summary": ([_VP, _I, _I, _I, _I, _LL, _CFGP, _VP, _VP], _I),
        "rkv_hsa_decode_summary": ([_VP, _VP, _VP, _VP, _I, _I, _I, _I, _LL, _LL, _CFGP, _I, _I, _VP, _VP, _I,
                                    _VP, _VP, _SZ, _VP], _I),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def status_string(st: int) -> str:
    return lib().rkv_status_string(st).decode()


def _check(st: int, what: str) -> None:
    if st != RKV_OK:
        raise RkvError(st, what)


def _ptr(a) -> int:
    """Address of a numpy array or torch tensor (0 for None)."""
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return int(stream)


# ---------------------------------------------------------------------------
# rocket.h mirror (host buffers, synchronous)
# ---------------------------------------------------------------------------
def compute_rocket_params(token_budget: int, sequence_length: int, max_new_tokens: int,
                          head_dim: int, window_size: int = 32) -> RocketBudgetParams:
    """rocket.h:36-41."""
    b = _Budget()
    _check(lib().rkv_compute_params(token_budget, sequence_length, max_new_tokens, head_dim,
                                    window_size, ctypes.byref(b)), "compute_rocket_params")
    return RocketBudgetParams(*[getattr(b, n) for n, _ in _Budget._fields_])


def compute_prefill_eviction(Q: np.ndarray, K: np.ndarray, len_q: int, len_k: int,
                             cfg: RocketConfig) -> np.ndarray:
    """rocket.h:43-46: fp32 host Q [H, len_q, D], K [HK, len_k, D] -> kept indices."""
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    c = cfg.c()
    cap = lib().rkv_evict_max_kept(ctypes.byref(c), len_q, len_k)
    if cap < 0:
        raise RkvError(-cap, "compute_prefill_eviction")
    out = np.zeros(cap, np.int32)
    n = _I(0)
    _check(lib().rkv_prefill_eviction_host(_ptr(Q), _ptr(K), len_q, len_k, ctypes.byref(c),
                                           _ptr(out), cap, ctypes.byref(n)),
           "compute_prefill_eviction")
    return out[: n.value].copy()


def compute_hybrid_sparse_decode(Q: np.ndarray, K: np.ndarray, V: np.ndarray, len_k: int,
                                 cfg: RocketConfig) -> np.ndarray:
    """rocket.h:48-50: fp32 host Q [H, D], K/V [HK, len_k, D] -> O [H * D]."""
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    O = np.zeros(cfg.num_heads * cfg.dim_head, np.float32)
    c = cfg.c()
    _check(lib().rkv_hybrid_sparse_decode_host(_ptr(Q), _ptr(K), _ptr(V), len_k, ctypes.byref(c),
                                               _ptr(O)), "compute_hybrid_sparse_decode")
    return O


def hsa_decode_host(Q: np.ndarray, K: np.ndarray, V: np.ndarray, dtype: int, len_k: int,
                    cfg: RocketConfig, recent_window: int = 0, with_sel: bool = False):
    """Host-buffer stage 2, any dtype and batch.  Q [B, H, D], K/V [B, HK, len_k, D]
    as float32 or uint16 (bf16 bits).  Returns O [B, H, D] (and sel, n_sel)."""
    B = Q.shape[0]
    c = cfg.c()
    O = np.zeros((B, cfg.num_heads, cfg.dim_head), np.float32)
    cap = lib().rkv_hsa_sel_capacity(ctypes.byref(c), len_k, recent_window)
    sel = np.zeros((B, cfg.num_heads_kv, cap), np.int32) if with_sel else None
    nsel = np.zeros((B, cfg.num_heads_kv), np.int32) if with_sel else None
    _check(lib().rkv_hsa_decode_host_ex(_ptr(Q), _ptr(K), _ptr(V), dtype, len_k, recent_window, B,
                                        Q[0].nbytes, K[0].nbytes, ctypes.byref(c), _ptr(O),
                                        _ptr(sel), cap, _ptr(nsel)), "hsa_decode_host")
    return (O, sel, nsel) if with_sel else O


# ---------------------------------------------------------------------------
# Device-resident batched entry points (torch CUDA tensors)
# ---------------------------------------------------------------------------
def evict_max_kept(cfg: RocketConfig, len_q: int, len_k: int) -> int:
    c = cfg.c()
    n = lib().rkv_evict_max_kept(ctypes.byref(c), len_q, len_k)
    if n < 0:
        raise RkvError(-n, "evict_max_kept")
    return n


def evict_workspace_size(cfg: RocketConfig, dtype: int, len_q: int, len_k: int, batch: int) -> int:
    c = cfg.c()
    b = _SZ(0)
    _check(lib().rkv_evict_workspace_size(ctypes.byref(c), dtype, len_q, len_k, batch, ctypes.byref(b)),
           "evict_workspace_size")
    return b.value


def hsa_sel_capacity(cfg: RocketConfig, len_k: int, recent_window: int = 0) -> int:
    c = cfg.c()
    n = lib().rkv_hsa_sel_capacity(ctypes.byref(c), len_k, recent_window)
    if n < 0:
        raise RkvError(-n, "hsa_sel_capacity")
    return n


def hsa_workspace_size(cfg: RocketConfig, len_k: int, recent_window: int, batch: int,
                       head_count: int) -> int:
    c = cfg.c()
    b = _SZ(0)
    _check(lib().rkv_hsa_workspace_size(ctypes.byref(c), len_k, recent_window, batch, head_count,
                                        ctypes.byref(b)), "hsa_workspace_size")
    return b.value


def _dtype_of(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.uint8:
        return Q8_0
    raise TypeError(f"unsupported tensor dtype {t.dtype}")


def _workspace(nbytes: int, device):
    import torch
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


class Evictor:
    """Stage 1 on device tensors.  Q [B, H, len_q, D*], K [B, HK, len_k, D*]
    (float32, bfloat16, or uint8 q8_0 rows), one workspace reused across calls."""

    def __init__(self, cfg: RocketConfig, len_q: int, len_k: int, batch: int, dtype: int, device):
        import torch
        self.cfg, self.len_q, self.len_k, self.batch, self.dtype = cfg, len_q, len_k, batch, dtype
        self.c = cfg.c()
        self.max_kept = evict_max_kept(cfg, len_q, len_k)
        self.ws_bytes = evict_workspace_size(cfg, dtype, len_q, len_k, batch)
        self.ws = _workspace(self.ws_bytes, device)
        self.kept = torch.zeros((batch, self.max_kept), dtype=torch.int32, device=device)
        self.n_kept = torch.zeros(batch, dtype=torch.int32, device=device)

    def __call__(self, Q, K, stream=None, engine: int = ENGINE_AUTO):
        assert Q.is_contiguous() and K.is_contiguous() and Q.shape[0] == K.shape[0] == self.batch
        _check(lib().rkv_evict(_ptr(Q), _ptr(K), self.dtype, self.len_q, self.len_k, self.batch,
                               Q[0].nbytes if self.batch else 0, K[0].nbytes if self.batch else 0,
                               ctypes.byref(self.c), _ptr(self.kept), self.max_kept, _ptr(self.n_kept),
                               _ptr(self.ws), self.ws_bytes, engine, _stream(stream)), "rkv_evict")
        return self.kept, self.n_kept

    def evict_compact(self, Q, K, V=None, K_out=None, V_out=None, stream=None, engine: int = ENGINE_AUTO):
        """Stage 1 on Q and the cache's K, then the cache compacted to the kept
        rows in the same call (rkv_evict_compact): in place without K_out /
        V_out, else into K_out / V_out [B, HK, out_len, D*].  Returns (kept, n_kept)."""
        assert Q.is_contiguous() and K.is_contiguous() and (V is None or V.is_contiguous())
        if K_out is None:
            K_out, V_out = K, V
        _check(lib().rkv_evict_compact(_ptr(Q), _ptr(K), _ptr(V) if V is not None else None, self.dtype, self.len_q,
                                       self.len_k, self.batch, Q[0].nbytes if self.batch else 0,
                                       K[0].nbytes if self.batch else 0, ctypes.byref(self.c), _ptr(self.kept),
                                       self.max_kept, _ptr(self.n_kept), _ptr(K_out),
                                       _ptr(V_out) if V_out is not None else None, K_out.shape[2],
                                       K_out[0].nbytes if self.batch else 0, _ptr(self.ws), self.ws_bytes, engine,
                                       _stream(stream)), "rkv_evict_compact")
        return self.kept, self.n_kept

    def pool_heads(self, Q, K, head_begin: int, head_count: int, pooled, stream=None, engine: int = ENGINE_AUTO):
        _check(lib().rkv_evict_pool_heads(_ptr(Q), _ptr(K), self.dtype, self.len_q, self.len_k,
                                          self.batch, Q[0].nbytes, K[0].nbytes, ctypes.byref(self.c),
                                          head_begin, head_count, _ptr(pooled), _ptr(self.ws),
                                          self.ws_bytes, engine, _stream(stream)),
               "rkv_evict_pool_heads")
        return pooled

    def select_pooled(self, pooled, stream=None):
        _check(lib().rkv_evict_select_pooled(_ptr(pooled), self.len_q, self.len_k, self.batch,
                                             ctypes.byref(self.c), _ptr(self.kept), self.max_kept,
                                             _ptr(self.n_kept), _ptr(self.ws), self.ws_bytes,
                                             _stream(stream)), "rkv_evict_select_pooled")
        return self.kept, self.n_kept


def compact_kv(K, V, kept, n_kept, dim_head: int, K_out=None, V_out=None, stream=None):
    """Applies kept token indices to a KV cache on the device (rkv_compact_kv).

    K, V: [B, HK, len_k, D*] (float32, bfloat16, or uint8 q8_0 rows of
    dim_head values); V may be None.  kept [B, >=n] int32 ascending, n_kept
    [B] int32 (an Evictor's outputs).  Without K_out / V_out the cache is
    compacted in place (row i of every head becomes row kept[i]); with them,
    K_out / V_out [B, HK, out_len, D*] receive the kept rows.  Returns the
    tensors written."""
    assert K.is_contiguous() and (V is None or V.is_contiguous())
    dtype = _dtype_of(K)
    B, HK, len_k = K.shape[0], K.shape[1], K.shape[2]
    if K_out is None:
        K_out, V_out = K, V
    assert K_out.is_contiguous() and (V_out is None or V_out.is_contiguous())
    _check(lib().rkv_compact_kv(_ptr(K), _ptr(V) if V is not None else None, dtype, dim_head, HK, len_k, B,
                                K[0].nbytes if B else 0, _ptr(kept), _ptr(n_kept), kept.shape[1], _ptr(K_out),
                                _ptr(V_out) if V_out is not None else None, K_out.shape[2],
                                K_out[0].nbytes if B else 0, _stream(stream)), "rkv_compact_kv")
    return K_out, V_out


def capture_rows(src, dst, token_offset: int, dst_first: int = 0, item: int = 0, stream=None):
    """The capture side on the device (rkv_capture_rows): one micro-batch of
    post-RoPE rows src [n_tokens, n_heads, dim_head] (float32, float16 or
    bfloat16, any strides along tokens and heads, unit stride along dim_head),
    global tokens token_offset .., scattered into item `item` of dst
    [items, n_heads, dst_tokens, dim_head] (float32, or bfloat16 from a
    bfloat16 source), row token - dst_first.  Returns dst."""
    assert src.dim() == 3 and src.stride(2) == 1 and dst.is_contiguous()
    n_tokens, n_heads, dim_head = src.shape
    es = src.element_size()
    _check(lib().rkv_capture_rows(_ptr(src), _dtype_of(src), n_tokens, n_heads, dim_head, src.stride(0) * es,
                                  src.stride(1) * es, token_offset, _ptr(dst), _dtype_of(dst), dst_first,
                                  dst.shape[2], dst[0].nbytes if dst.shape[0] else 0, item, _stream(stream)),
           "rkv_capture_rows")
    return dst


class HsaDecoder:
    """Stage 2 on device tensors.  Q [B, H, D], K/V [B, HK, len_k, D] (float32
    or bfloat16); KV heads [head_begin, head_begin + head_count)."""

    def __init__(self, cfg: RocketConfig, len_k: int, batch: int, device, recent_window: int = 0,
                 head_begin: int = 0, head_count: int | None = None):
        import torch
        self.cfg, self.len_k, self.batch, self.w = cfg, len_k, batch, recent_window
        self.head_begin = head_begin
        self.head_count = cfg.num_heads_kv if head_count is None else head_count
        self.c = cfg.c()
        self.sel_cap = hsa_sel_capacity(cfg, len_k, recent_window)
        self.ws_bytes = hsa_workspace_size(cfg, len_k, recent_window, batch, self.head_count)
        self.ws = _workspace(self.ws_bytes, device)
        self.O = torch.zeros((batch, cfg.num_heads, cfg.dim_head), dtype=torch.float32, device=device)
        self.sel = torch.zeros((batch, self.head_count, self.sel_cap), dtype=torch.int32, device=device)
        self.n_sel = torch.zeros((batch, self.head_count), dtype=torch.int32, device=device)

    def build_summary(self, K, stream=None, out=None):
        """Page summaries of K (every KV head) for this decoder's geometry:
        later calls with summary=... read them instead of scanning every K row.
        out: a buffer from an earlier call to rebuild into (no allocation)."""
        import torch
        dt = _dtype_of(K)
        n = ctypes.c_size_t(0)
        _check(lib().rkv_hsa_summary_size(ctypes.byref(self.c), dt, self.len_k, self.w, self.batch, ctypes.byref(n)),
               "rkv_hsa_summary_size")
        S = out if out is not None else torch.empty(max(n.value, 16), dtype=torch.uint8, device=K.device)
        assert S.numel() >= n.value
        _check(lib().rkv_hsa_build_summary(_ptr(K), dt, self.len_k, self.w, self.batch, K[0].nbytes if self.batch else 0,
                                           ctypes.byref(self.c), _ptr(S), _stream(stream)), "rkv_hsa_build_summary")
        return S

    def __call__(self, Q, K, V, stream=None, want_sel: bool = True, summary=None):
        assert Q.is_contiguous() and K.is_contiguous() and V.is_contiguous()
        assert K.shape == V.shape and Q.shape[0] == K.shape[0] == self.batch
        dt = _dtype_of(K)
        common = (dt, self.len_k, self.w, self.batch, Q[0].nbytes, K[0].nbytes, ctypes.byref(self.c), self.head_begin,
                  self.head_count, _ptr(self.O), _ptr(self.sel) if want_sel else 0, self.sel_cap,
                  _ptr(self.n_sel) if want_sel else 0, _ptr(self.ws), self.ws_bytes, _stream(stream))
        if summary is None:
            _check(lib().rkv_hsa_decode(_ptr(Q), _ptr(K), _ptr(V), *common), "rkv_hsa_decode")
        else:
            _check(lib().rkv_hsa_decode_summary(_ptr(Q), _ptr(K), _ptr(V), _ptr(summary), *common),
                   "rkv_hsa_decode_summary")
        return self.O

    def status(self, stream=None) -> int:
        return lib().rkv_workspace_status(_ptr(self.ws), _stream(stream))
