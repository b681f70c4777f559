"""TEST INFRASTRUCTURE ONLY: ctypes wrapper over the CPU oracle (libptts_oracle.so).

The oracle restates the reference's flow-LM attention path in C (see ptts_oracle.h for the
reference lines it follows and for what pins it: parity unpinned against `xn`, which the
reference delegates to and which cannot be built here). Only tests, `__graft_entry__.smoke()`
and the `cpu_baseline` / `--impl reference` legs of bench.py may import this module, and only as
the checker or the timed CPU baseline. The CUDA library never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libptts_oracle.so")

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float


class ModelDesc(ctypes.Structure):
    _fields_ = [
        ("d_model", I), ("num_heads", I), ("num_kv_heads", I), ("head_dim", I),
        ("num_layers", I), ("dim_feedforward", I), ("max_period", F), ("scale_group", I),
        ("gelu_tanh", I),
        ("w_qkv", P), ("s_qkv", P), ("w_out", P), ("s_out", P), ("w_ff1", P), ("s_ff1", P),
        ("w_ff2", P), ("s_ff2", P), ("ln1_g", P), ("ln1_b", P), ("ln2_g", P), ("ln2_b", P),
    ]


def _declare(L):
    L.oracle_rope_inv_freq.argtypes = [I, F, P]
    L.oracle_rope_table.argtypes = [I, P, I, F, P, P]
    L.oracle_attend.argtypes = [P, P, P, I, I, I, P, P, I, I, P, P, P, I, F, I, P, I]
    L.oracle_attend.restype = I
    L.oracle_linear_i8.argtypes = [P, P, P, I, I, I, I, P, I]
    L.oracle_layer_norm.argtypes = [P, P, P, I, I, F, P]
    L.oracle_gelu.argtypes = [F, I]
    L.oracle_gelu.restype = F
    L.oracle_model_create.argtypes = [ctypes.POINTER(ModelDesc)]
    L.oracle_model_create.restype = P
    L.oracle_model_free.argtypes = [P]
    L.oracle_model_forward.argtypes = [P, P, P, P, I, I, P, P, P, I, I, I]
    L.oracle_model_forward.restype = I


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


# Storage modes of the oracle (bit mask): which tensors are rounded to bf16 where they are stored.
ROUND_KV = 1        # the rotated k and the v rows entering the cache (the CUDA library's storage)
ROUND_OPERANDS = 2  # the GEMM inputs: normalised rows, attention output, GELU output


def threads() -> int:
    return len(os.sched_getaffinity(0))


# --- bf16 helpers (numpy, round to nearest even) -------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = _f32(x).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(_f32(x))
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --- ops -----------------------------------------------------------------------------------

def rope_inv_freq(head_dim: int, max_period: float = 10000.0) -> np.ndarray:
    out = np.zeros(head_dim // 2, np.float32)
    lib().oracle_rope_inv_freq(head_dim, max_period, _p(out))
    return out


def rope_table(head_dim: int, positions, max_period: float = 10000.0):
    pos = _f32(positions)
    c = np.zeros((len(pos), head_dim // 2), np.float32)
    s = np.zeros_like(c)
    lib().oracle_rope_table(head_dim, _p(pos), len(pos), max_period, _p(c), _p(s))
    return c, s


def attend(q, k, v, k_cache, v_cache, lengths, streams, row_offsets, *, max_period=10000.0,
           store=0, n_threads=None) -> np.ndarray:
    """Rope + append + causal attention for a ragged batch (caches updated in place).

    q [rows, H, D], k/v [rows, KVH, D], caches [S, cap, H, D] float32 (modified in place).
    Returns out [rows, H*D] f32. Raises ValueError when a sequence does not fit.
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    assert k_cache.dtype == np.float32 and k_cache.flags.c_contiguous
    assert v_cache.dtype == np.float32 and v_cache.flags.c_contiguous
    rows, H, D = q.shape
    KVH = k.shape[1]
    S, cap = k_cache.shape[:2]
    lengths, streams, row_offsets = _i32(lengths), _i32(streams), _i32(row_offsets)
    out = np.zeros((rows, H * D), np.float32)
    rc = lib().oracle_attend(_p(q), _p(k), _p(v), H, KVH, D, _p(k_cache), _p(v_cache), S, cap,
                             _p(lengths), _p(streams), _p(row_offsets), len(streams),
                             max_period, int(store), _p(out), n_threads or threads())
    if rc != 0:
        raise ValueError(f"oracle_attend failed with {rc}")
    return out


def linear_i8(x, w, scale, group=0, n_threads=None) -> np.ndarray:
    x = _f32(x)
    w = np.ascontiguousarray(w, dtype=np.int8)
    scale = _f32(scale)
    m, k = x.shape
    n = w.shape[0]
    y = np.zeros((m, n), np.float32)
    lib().oracle_linear_i8(_p(x), _p(w), _p(scale), m, n, k, group, _p(y), n_threads or threads())
    return y


def layer_norm(x, gamma, beta, eps=1e-5) -> np.ndarray:
    x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
    y = np.zeros_like(x)
    lib().oracle_layer_norm(_p(x), _p(gamma), _p(beta), x.shape[0], x.shape[1], eps, _p(y))
    return y


@dataclass
class Weights:
    """Per-layer weights concatenated over layers (numpy, host)."""
    w_qkv: np.ndarray  # int8 [L, (H+2KVH)D, d]
    s_qkv: np.ndarray  # f32 [L, rows] (group 0) or [L, rows, K/group]
    w_out: np.ndarray
    s_out: np.ndarray
    w_ff1: np.ndarray
    s_ff1: np.ndarray
    w_ff2: np.ndarray
    s_ff2: np.ndarray
    ln1_g: np.ndarray
    ln1_b: np.ndarray
    ln2_g: np.ndarray
    ln2_b: np.ndarray


class Model:
    """The oracle transformer: StreamingTransformer::forward restated in C."""

    def __init__(self, cfg, w: Weights):
        self.cfg = cfg
        self._keep = [np.ascontiguousarray(a) for a in (
            w.w_qkv, w.s_qkv, w.w_out, w.s_out, w.w_ff1, w.s_ff1, w.w_ff2, w.s_ff2,
            w.ln1_g, w.ln1_b, w.ln2_g, w.ln2_b)]
        ptrs = [_p(a) for a in self._keep]
        desc = ModelDesc(cfg.d_model, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                         cfg.num_layers, cfg.dim_feedforward, cfg.max_period, cfg.scale_group,
                         int(cfg.gelu == "tanh"), *ptrs)
        self._h = lib().oracle_model_create(ctypes.byref(desc))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().oracle_model_free(self._h)
            self._h = None

    def forward(self, x, k_cache, v_cache, lengths, streams, row_offsets, *, store=ROUND_KV,
                n_threads=None) -> np.ndarray:
        """x [rows, d] (layer-0 input) -> last layer's output [rows, d]; caches
        [L, S, cap, H, D] updated in place; lengths not advanced. `store`: ROUND_* bit mask."""
        x = _f32(x).copy()
        S, cap = k_cache.shape[1:3]
        lengths, streams, row_offsets = _i32(lengths), _i32(streams), _i32(row_offsets)
        rc = lib().oracle_model_forward(self._h, _p(x), _p(k_cache), _p(v_cache), S, cap,
                                        _p(lengths), _p(streams), _p(row_offsets), len(streams),
                                        int(store), n_threads or threads())
        if rc != 0:
            raise ValueError(f"oracle_model_forward failed with {rc}")
        return x
