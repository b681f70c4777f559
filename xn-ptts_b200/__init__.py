"""ptts_b200: the flow-LM attention path of Phonon TTS on B200, driven from Python.

A thin mirror, over the C ABI of ``include/ptts_b200.h`` (ctypes), of the reference's operator
surface for this path:

    KvState       StreamingTransformerState (ptts/src/transformer.rs:328-393)
    attend        StreamingMultiheadAttention::forward after in_proj (transformer.rs:197-248)
    linear_i8     Q::LinearQ::forward with int8 per-output-channel weights
    Transformer   StreamingTransformer::{forward, forward_step} (transformer.rs:742-838)

Device tensors are torch tensors (torch supplies memory, streams and torch.distributed; the
arithmetic runs in libptts_b200.so). There is no CPU fallback: without the built library or
without a CUDA device every call raises.

The package directory is ``xn-ptts_b200``; the hyphen keeps it out of ``import``, so load it by
path (``__graft_entry__.load_package()`` registers it as ``xn_ptts_b200``).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libptts_b200.so")

OK = 0
ERR_ARG, ERR_CAPACITY, ERR_CUDA, ERR_STATE, ERR_UNSUPPORTED, ERR_DEVICE = -1, -2, -3, -4, -5, -6
F32, BF16 = 0, 1
# Bits of a device-side error word (PTTS_B200_DEVERR_*).
DEVERR_BOUNDS, DEVERR_CAPACITY, DEVERR_TIMEOUT, DEVERR_DUPLICATE = 1, 2, 4, 8
_DTYPES = {"f32": F32, "float32": F32, "bf16": BF16, "bfloat16": BF16}

# Every symbol include/ptts_b200.h declares.
EXPORTS = (
    "ptts_b200_last_error", "ptts_b200_version",
    "ptts_b200_kv_create", "ptts_b200_kv_destroy", "ptts_b200_kv_lengths",
    "ptts_b200_kv_pointers", "ptts_b200_kv_advance", "ptts_b200_kv_reset",
    "ptts_b200_kv_set_lengths", "ptts_b200_set_tracing", "ptts_b200_trace_read",
    "ptts_b200_kv_load_prefix", "ptts_b200_kv_copy_stream", "ptts_b200_kv_check",
    "ptts_b200_attend", "ptts_b200_linear_i8",
    "ptts_b200_model_create", "ptts_b200_model_destroy", "ptts_b200_model_load_layer",
    "ptts_b200_forward", "ptts_b200_step", "ptts_b200_attend_decode_noalloc",
    "ptts_b200_flow_create", "ptts_b200_flow_destroy", "ptts_b200_flow_set_tensor",
    "ptts_b200_flow_finish", "ptts_b200_flow_sample", "ptts_b200_frame",
    "ptts_b200_kv_start_ring", "ptts_b200_kv_set_ring_slot", "ptts_b200_kv_set_ring_slots", "ptts_b200_kv_evict",
    "ptts_b200_model_config", "ptts_b200_model_load_layer_f32", "ptts_b200_model_load_layer_q8_0",
    "ptts_b200_load_gguf", "ptts_b200_gguf_remap_key", "ptts_b200_kv_set_window",
    "ptts_b200_model_stamps", "ptts_b200_model_stamps_read", "ptts_b200_model_set_layer_scale",
)


class PttsError(RuntimeError):
    """A failed ptts_b200 call: `code` is the PTTS_B200_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class CapacityError(PttsError):
    pass


P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
IP = ctypes.POINTER(ctypes.c_int32)


class Config(ctypes.Structure):
    """ptts_b200_config: FlowLMConfig's transformer shape (ptts/src/flow_lm.rs:114-146)."""
    _fields_ = [("d_model", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("num_layers", ctypes.c_int32), ("dim_feedforward", ctypes.c_int32),
                ("max_period", ctypes.c_float), ("gelu", ctypes.c_int32)]


class LayerWeightsF32(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "in_proj", "out_proj", "linear1", "linear2", "norm1_weight", "norm1_bias", "norm2_weight", "norm2_bias")]


class LayerWeightsQ8(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "in_proj", "out_proj", "linear1", "linear2", "norm1_weight", "norm1_bias", "norm2_weight", "norm2_bias")]


class FlowConfigC(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int), ("flow_dim", ctypes.c_int), ("flow_depth", ctypes.c_int),
                ("ldim", ctypes.c_int), ("freq_dim", ctypes.c_int), ("flow_type", ctypes.c_int),
                ("lsd_steps", ctypes.c_int), ("time_norm", ctypes.c_int)]


class Trace(ctypes.Structure):
    """ptts_b200_trace: counters of traced decode-attention launches (see set_tracing)."""
    _fields_ = [("steps", ctypes.c_int64), ("attn_launches", ctypes.c_int64),
                ("attn_ms", ctypes.c_double), ("attn_bytes", ctypes.c_double),
                ("step_ms", ctypes.c_double)]


class Stamp(ctypes.Structure):
    """ptts_b200_stamp: one launch of the kernel timeline (see Transformer.stamps)."""
    _fields_ = [("kernel", ctypes.c_char * 16), ("lane", ctypes.c_int), ("layer", ctypes.c_int),
                ("entry_us", ctypes.c_double), ("start_us", ctypes.c_double), ("end_us", ctypes.c_double),
                ("last_entry_us", ctypes.c_double)]


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, P) for n in (
        "in_proj_host", "in_proj_scale_host", "out_proj_host", "out_proj_scale_host",
        "linear1_host", "linear1_scale_host", "linear2_host", "linear2_scale_host",
        "norm1_weight_host", "norm1_bias_host", "norm2_weight_host", "norm2_bias_host")]


_lib = None


def build(verbose: bool = False) -> str:
    import importlib.util
    spec = importlib.util.spec_from_file_location("_ptts_b200_build", os.path.join(HERE, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(verbose=verbose)


def lib() -> ctypes.CDLL:
    """The loaded C library. Raises when it has not been built: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise PttsError(ERR_STATE, f"{LIB_PATH} is missing: build it (python xn-ptts_b200/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        L.ptts_b200_last_error.restype = ctypes.c_char_p
        L.ptts_b200_version.restype = ctypes.c_char_p
        L.ptts_b200_kv_create.argtypes = [I, I, I, I, I, I, I, ctypes.POINTER(P)]
        L.ptts_b200_kv_destroy.argtypes = [P]
        L.ptts_b200_kv_destroy.restype = None
        L.ptts_b200_kv_lengths.argtypes = [P, IP]
        L.ptts_b200_kv_pointers.argtypes = [P, I, ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(P)]
        L.ptts_b200_kv_advance.argtypes = [P, IP, IP, I, P]
        L.ptts_b200_kv_reset.argtypes = [P, IP, I, P]
        L.ptts_b200_kv_set_lengths.argtypes = [P, IP, IP, I, P]
        L.ptts_b200_set_tracing.argtypes = [I]
        L.ptts_b200_trace_read.argtypes = [ctypes.POINTER(Trace), I]
        L.ptts_b200_model_stamps.argtypes = [P, I]
        L.ptts_b200_model_stamps_read.argtypes = [P, ctypes.POINTER(Stamp), I, IP]
        L.ptts_b200_kv_load_prefix.argtypes = [P, I, I, P, P, I, I, P]
        L.ptts_b200_kv_copy_stream.argtypes = [P, I, P, I, P]
        L.ptts_b200_kv_check.argtypes = [P]
        L.ptts_b200_attend.argtypes = [P, I, P, P, P, I, I, IP, IP, I, F, P, I, P]
        L.ptts_b200_linear_i8.argtypes = [I, P, P, P, I, I, I, P, P]
        L.ptts_b200_model_create.argtypes = [I, ctypes.POINTER(Config), ctypes.POINTER(P)]
        L.ptts_b200_model_destroy.argtypes = [P]
        L.ptts_b200_model_destroy.restype = None
        L.ptts_b200_model_load_layer.argtypes = [P, I, ctypes.POINTER(LayerWeights)]
        L.ptts_b200_forward.argtypes = [P, P, P, IP, IP, I, P, P]
        L.ptts_b200_step.argtypes = [P, P, IP, I, P, P, P]
        L.ptts_b200_attend_decode_noalloc.argtypes = [P, P, I, I, I, P, P, I, P, P, P, I, I, F, P, I, P, P]
        L.ptts_b200_model_config.argtypes = [P, ctypes.POINTER(Config)]
        L.ptts_b200_model_load_layer_f32.argtypes = [P, I, ctypes.POINTER(LayerWeightsF32)]
        L.ptts_b200_model_load_layer_q8_0.argtypes = [P, I, ctypes.POINTER(LayerWeightsQ8)]
        L.ptts_b200_model_set_layer_scale.argtypes = [P, I, P, P]
        L.ptts_b200_load_gguf.argtypes = [P, P, ctypes.c_char_p]
        L.ptts_b200_gguf_remap_key.argtypes = [ctypes.c_char_p, ctypes.c_char_p, I]
        L.ptts_b200_kv_set_window.argtypes = [P, IP, I, I, P]
        L.ptts_b200_kv_start_ring.argtypes = [P, IP, I, P]
        L.ptts_b200_kv_set_ring_slot.argtypes = [P, I, I, P]
        L.ptts_b200_kv_set_ring_slots.argtypes = [P, IP, IP, I, P]
        L.ptts_b200_kv_evict.argtypes = [P, I, I, IP, I, F, P]
        L.ptts_b200_flow_create.argtypes = [I, ctypes.POINTER(FlowConfigC), ctypes.POINTER(P)]
        L.ptts_b200_flow_destroy.argtypes = [P]
        L.ptts_b200_flow_destroy.restype = None
        L.ptts_b200_flow_set_tensor.argtypes = [P, ctypes.c_char_p, P, ctypes.c_int64]
        L.ptts_b200_flow_finish.argtypes = [P]
        L.ptts_b200_flow_sample.argtypes = [P, P, I, P, P, P, P]
        L.ptts_b200_frame.argtypes = [P, P, P, IP, I, P, P, P, P, P]
        _lib = L
    return _lib


def version() -> str:
    return lib().ptts_b200_version().decode()


def _check(rc: int):
    if rc != OK:
        msg = lib().ptts_b200_last_error().decode(errors="replace")
        if rc == ERR_CAPACITY:
            raise CapacityError(rc, msg)
        raise PttsError(rc, msg)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _ip(a: np.ndarray):
    return a.ctypes.data_as(IP)


def _stream(stream=None) -> ctypes.c_void_p:
    """The CUDA stream handle for a call: `stream`'s, else torch's current stream on the current
    device (read through torch's raw-stream query, a few microseconds cheaper per call than
    building a torch.cuda.Stream object)."""
    import torch
    if stream is not None:
        return ctypes.c_void_p(stream.cuda_stream)
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return ctypes.c_void_p(raw(torch._C._cuda_getDevice()))
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dptr(t) -> ctypes.c_void_p:
    if not t.is_cuda:
        raise PttsError(ERR_ARG, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise PttsError(ERR_ARG, "expected a contiguous tensor")
    return ctypes.c_void_p(t.data_ptr())


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    raise PttsError(ERR_ARG, f"unsupported dtype {t.dtype}")


class _Cai:
    """A raw device buffer exposed through __cuda_array_interface__ (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


# --------------------------------------------------------------------------------------------
# KV state
# --------------------------------------------------------------------------------------------

class KvState:
    """Per-layer K/V caches of `num_streams` independent streams, `capacity` slots each, plus
    one filled length per stream: StreamingTransformerState (transformer.rs:328-393) for a
    whole batch. ``init_state`` there is this constructor (zero caches, lengths 0)."""

    def __init__(self, num_layers: int, num_streams: int, capacity: int, *, num_heads: int = 8,
                 head_dim: int = 64, dtype: str = "bf16", device: int = 0):
        self.num_layers, self.num_streams, self.capacity = num_layers, num_streams, capacity
        self.num_heads, self.head_dim, self.device = num_heads, head_dim, device
        self.dtype = dtype
        h = P()
        _check(lib().ptts_b200_kv_create(device, num_layers, num_streams, capacity, num_heads,
                                          head_dim, _DTYPES[dtype], ctypes.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().ptts_b200_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def lengths(self) -> np.ndarray:
        out = np.zeros(self.num_streams, np.int32)
        _check(lib().ptts_b200_kv_lengths(self._h, _ip(out)))
        return out

    def advance(self, streams: Sequence[int], rows: Sequence[int], stream=None):
        s, r = _i32(streams), _i32(rows)
        _check(lib().ptts_b200_kv_advance(self._h, _ip(s), _ip(r), len(s), _stream(stream)))

    def reset(self, streams: Sequence[int], stream=None):
        s = _i32(streams)
        _check(lib().ptts_b200_kv_reset(self._h, _ip(s), len(s), _stream(stream)))

    def set_window(self, streams: Sequence[int], context: int, stream=None):
        """Mimi's KvCache::new(context) for these (empty) streams (ptts_b200_kv_set_window)."""
        st = _i32(streams)
        _check(lib().ptts_b200_kv_set_window(self._h, _ip(st), len(st), context, _stream(stream)))

    def start_ring(self, streams: Sequence[int], stream=None):
        """StreamingTransformer::start_ring for these streams (ptts_b200_kv_start_ring)."""
        st = _i32(streams)
        _check(lib().ptts_b200_kv_start_ring(self._h, _ip(st), len(st), _stream(stream)))

    def set_ring_slot(self, stream_index: int, slot: int, stream=None):
        _check(lib().ptts_b200_kv_set_ring_slot(self._h, stream_index, slot, _stream(stream)))

    def set_ring_slots(self, streams: Sequence[int], slots: Sequence[int], stream=None):
        """set_ring_slot for many ring streams in one call (ptts_b200_kv_set_ring_slots)."""
        st, sl = _i32(streams), _i32(slots)
        if len(st) != len(sl):
            raise PttsError(ERR_ARG, "one slot per stream")
        _check(lib().ptts_b200_kv_set_ring_slots(self._h, _ip(st), _ip(sl), len(st), _stream(stream)))

    def evict(self, stream_index: int, prefix: int, slots: Sequence[int], max_period: float = 10000.0,
              stream=None):
        """StreamingTransformer::evict: hide `slots`, rotate kept keys past `prefix` back."""
        sl = _i32(slots)
        _check(lib().ptts_b200_kv_evict(self._h, stream_index, prefix, _ip(sl), len(sl), max_period,
                                        _stream(stream)))

    def set_lengths(self, streams: Sequence[int], lengths: Sequence[int], stream=None):
        """Lower (or raise, up to capacity) stream lengths, keeping the slots."""
        s, n = _i32(streams), _i32(lengths)
        _check(lib().ptts_b200_kv_set_lengths(self._h, _ip(s), _ip(n), len(s), _stream(stream)))

    def pointers(self, layer: int):
        k, v, ln = P(), P(), P()
        _check(lib().ptts_b200_kv_pointers(self._h, layer, ctypes.byref(k), ctypes.byref(v),
                                            ctypes.byref(ln)))
        return k.value, v.value, ln.value

    def tensors(self, layer: int):
        """Views (torch, no copy) of one layer's K and V caches and the device lengths [S]: the
        caches as [S, cap, H, D] with 8 heads, and as [S, cap, H / 8, 8, D] with more (each
        group of 8 heads is its own [S, cap, 8, D] block; `.reshape(S, cap, H, D)` copies)."""
        import torch
        k, v, ln = self.pointers(layer)
        G = self.num_heads // 8
        shape = (G, self.num_streams, self.capacity, 8, self.head_dim)
        if self.dtype == "bf16":
            kt = torch.as_tensor(_Cai(k, shape, "<i2"), device=f"cuda:{self.device}").view(torch.bfloat16)
            vt = torch.as_tensor(_Cai(v, shape, "<i2"), device=f"cuda:{self.device}").view(torch.bfloat16)
        else:
            kt = torch.as_tensor(_Cai(k, shape, "<f4"), device=f"cuda:{self.device}")
            vt = torch.as_tensor(_Cai(v, shape, "<f4"), device=f"cuda:{self.device}")
        kt, vt = (t[0] if G == 1 else t.permute(1, 2, 0, 3, 4) for t in (kt, vt))
        lt = torch.as_tensor(_Cai(ln, (self.num_streams,), "<i4"), device=f"cuda:{self.device}")
        return kt, vt, lt

    def load_prefix(self, layer: int, stream: int, k, v, set_length: bool = True, cuda_stream=None):
        """Rows [len, H, D] (device tensors of the cache dtype) into slots 0..len."""
        n = 0 if k is None else int(k.shape[0])
        kp = _dptr(k) if n else None
        vp = _dptr(v) if n else None
        _check(lib().ptts_b200_kv_load_prefix(self._h, layer, stream, kp, vp, n, int(set_length),
                                               _stream(cuda_stream)))

    def copy_stream(self, dst_stream: int, src: "KvState", src_stream: int, cuda_stream=None):
        _check(lib().ptts_b200_kv_copy_stream(self._h, dst_stream, src._h, src_stream,
                                               _stream(cuda_stream)))

    def with_seq_budget(self, seq_budget: int, streams: Optional[Sequence[int]] = None) -> "KvState":
        """A fresh state with room for `seq_budget` positions per stream, holding a copy of each
        stream's filled prefix (transformer.rs:350-392). Refused (CapacityError naming both
        numbers) when a prefix does not fit."""
        streams = range(self.num_streams) if streams is None else streams
        lens = self.lengths()
        for s in streams:
            if lens[s] > seq_budget:
                raise CapacityError(ERR_CAPACITY, f"cannot fit {lens[s]} filled KV positions into a budget of {seq_budget}")
        out = KvState(self.num_layers, self.num_streams, seq_budget, num_heads=self.num_heads,
                      head_dim=self.head_dim, dtype=self.dtype, device=self.device)
        for s in streams:
            out.copy_stream(s, self, s)
        return out

    def check(self):
        """Raise if a kernel's own bounds check or bounded wait tripped (synchronises)."""
        _check(lib().ptts_b200_kv_check(self._h))


# --------------------------------------------------------------------------------------------
# ops
# --------------------------------------------------------------------------------------------

def attend(kv: KvState, layer: int, q, k, v, streams: Sequence[int], rows: Sequence[int], *,
           max_period: float = 10000.0, out_dtype: str = "f32", out=None, stream=None):
    """RoPE + KV append + causal attention for a ragged batch of streams (see ptts_b200_attend).

    q [n_rows, H, D], k/v [n_rows, KVH, D] (CUDA, bf16 or f32, same dtype), rows grouped by
    sequence. Returns out [n_rows, H*D]. Lengths are not advanced (KvState.advance)."""
    import torch
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise PttsError(ERR_ARG, "q, k and v must share a dtype")
    s, r = _i32(streams), _i32(rows)
    n_rows = int(q.shape[0])
    if out is None:
        out = torch.empty((n_rows, q.shape[1] * q.shape[2]),
                          dtype=torch.bfloat16 if out_dtype == "bf16" else torch.float32,
                          device=q.device)
    _check(lib().ptts_b200_attend(kv.handle, layer, _dptr(q), _dptr(k), _dptr(v), _dtype_code(q),
                                  int(k.shape[1]), _ip(s), _ip(r), len(s), max_period, _dptr(out),
                                  _dtype_code(out), _stream(stream)))
    return out


def step_lanes(n: int) -> int:
    """How many lanes a decode step of n rows runs in (the library's rule: two from 128 rows,
    one with PTTS_B200_LANES=1)."""
    return 1 if os.environ.get("PTTS_B200_LANES", "").startswith("1") or n < 128 else 2


def set_tracing(on: bool):
    """Process-wide: while on, Transformer.step runs un-graphed and it and attend() time every
    decode-attention launch with CUDA events (one synchronisation per call)."""
    _check(lib().ptts_b200_set_tracing(int(on)))


def trace(reset: bool = False) -> dict:
    t = Trace()
    _check(lib().ptts_b200_trace_read(ctypes.byref(t), int(reset)))
    return {n: getattr(t, n) for n, _ in Trace._fields_}


def attend_decode_noalloc(k_cache, v_cache, lengths, streams, q, k, v, *, out, err=None,
                          max_period: float = 10000.0, stream=None):
    """ptts_b200_attend_decode_noalloc: one decode row per stream over a caller-owned cache,
    with no device allocation inside the call (for hosts that cannot allocate while running).

    k_cache/v_cache [S, cap, 8, 64] (CUDA, bf16 or f32), lengths [S] int32 (CUDA, not advanced),
    streams [n] int32 (CUDA), q [n, 8, 64], k/v [n, KVH, 64], out [n, 512] (all preallocated by
    the caller), err an optional CUDA uint32/int32 word for device-side range errors."""
    S, cap = int(k_cache.shape[0]), int(k_cache.shape[1])
    _check(lib().ptts_b200_attend_decode_noalloc(
        _dptr(k_cache), _dptr(v_cache), S, cap, _dtype_code(k_cache), _dptr(lengths),
        _dptr(streams), int(streams.shape[0]), _dptr(q), _dptr(k), _dptr(v), _dtype_code(q),
        int(k.shape[1]), max_period, _dptr(out), _dtype_code(out),
        _dptr(err) if err is not None else None, _stream(stream)))
    return out


def linear_i8(x, w, scale, stream=None):
    """y = x W^T with W = w * scale[:, None]: x [m, k] bf16, w [n, k] int8, scale [n] f32."""
    import torch
    m, k = x.shape
    n = w.shape[0]
    y = torch.empty((m, n), dtype=torch.float32, device=x.device)
    _check(lib().ptts_b200_linear_i8(x.device.index or 0, _dptr(x), _dptr(w), _dptr(scale), m, n,
                                     k, _dptr(y), _stream(stream)))
    return y


# --------------------------------------------------------------------------------------------
# transformer
# --------------------------------------------------------------------------------------------

@dataclass
class FlowLMConfig:
    """The flow LM's transformer shape (FlowLMConfig, ptts/src/flow_lm.rs:114-146)."""
    d_model: int = 512
    num_heads: int = 8
    num_kv_heads: int = 8
    head_dim: int = 64
    num_layers: int = 6
    dim_feedforward: int = 2048
    max_period: float = 10000.0
    gelu: str = "erf"
    scale_group: int = 0  # 0: one scale per output row (the only form the GPU path takes)

    def c_struct(self) -> Config:
        return Config(self.d_model, self.num_heads, self.num_kv_heads, self.head_dim,
                      self.num_layers, self.dim_feedforward, self.max_period,
                      1 if self.gelu == "tanh" else 0)


# The 31m and 40m flow LMs: 512 wide, 8 heads, ff 2048, theta 10000; 6 vs 9 layers.
PHONON_31M = FlowLMConfig(num_layers=6)
PHONON_40M = FlowLMConfig(num_layers=9)
# Mimi's transformers (encoder and decoder; MimiConfig, mimi.rs:34-40, with the values of
# ptts-wasm/js/gpu/support.js:13-14 and ptts/tests/fixtures/config.json:33-37): 512 wide, 8 heads,
# 2 layers, ff 2048, theta 10000, windowed attention over the last 250 positions, layer scale.
MIMI_TRANSFORMER = FlowLMConfig(num_layers=2)
MIMI_CONTEXT = 250


def random_mimi_tensors(cfg: FlowLMConfig, seed: int, *, layer_scale: float = 0.01) -> dict:
    """Random-init Mimi transformer tensors under the checkpoint's names: linears U(-1/sqrt(in),
    1/sqrt(in)) (torch's default), LayerNorm affine near (1, 0), layer scales near `layer_scale`."""
    rng = np.random.default_rng(seed)
    d, ff = cfg.d_model, cfg.dim_feedforward
    out = {}

    def lin(n, k):
        b = 1.0 / np.sqrt(k)
        return rng.uniform(-b, b, (n, k)).astype(np.float32)

    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        out[p + "self_attn.in_proj.weight"] = lin(3 * d, d)
        out[p + "self_attn.out_proj.weight"] = lin(d, d)
        out[p + "linear1.weight"] = lin(ff, d)
        out[p + "linear2.weight"] = lin(d, ff)
        for n in ("norm1", "norm2"):
            out[p + n + ".weight"] = rng.uniform(0.8, 1.2, d).astype(np.float32)
            out[p + n + ".bias"] = rng.normal(0.0, 0.05, d).astype(np.float32)
        for n in ("layer_scale_1", "layer_scale_2"):
            out[p + n + ".scale"] = (layer_scale * rng.uniform(0.5, 1.5, d)).astype(np.float32)
    return out


def quantize_q8_0(w) -> np.ndarray:
    """f32 weights [n][k] (k a multiple of 32) as GGUF q8_0 blocks, uint8 [n][k / 32 * 34]: per
    32 weights along k, d = max |w| / 127 stored as f16, then q = round(w / d) as int8 (the q8_0
    format of ggml, which Q8Linear::from_linear quantizes to, q8.rs:29-35). W = q * f16(d)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % 32:
        raise PttsError(ERR_ARG, f"q8_0 needs rows of a multiple of 32 weights, not {k}")
    b = w.reshape(n, k // 32, 32)
    d = np.abs(b).max(axis=2) / 127.0
    inv = np.divide(1.0, d, out=np.zeros_like(d), where=d > 0)
    q = np.clip(np.rint(b * inv[..., None]), -127, 127).astype(np.int8)
    out = np.empty((n, k // 32, 34), np.uint8)
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(n, k // 32 * 34)


class Transformer:
    """StreamingTransformer (transformer.rs:674-930) for the flow LM, int8 per-channel."""

    def __init__(self, cfg: FlowLMConfig, device: int = 0):
        self.cfg, self.device = cfg, device
        h = P()
        st = cfg.c_struct()
        _check(lib().ptts_b200_model_create(device, ctypes.byref(st), ctypes.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().ptts_b200_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_layer(self, layer: int, w: dict):
        """w: numpy arrays keyed like the checkpoint (in_proj, in_proj_scale, out_proj, ...,
        norm1_weight, norm1_bias, norm2_weight, norm2_bias)."""
        keep = {k: np.ascontiguousarray(v) for k, v in w.items()}
        lw = LayerWeights(*[keep[n].ctypes.data_as(P) for n in (
            "in_proj", "in_proj_scale", "out_proj", "out_proj_scale", "linear1", "linear1_scale",
            "linear2", "linear2_scale", "norm1_weight", "norm1_bias", "norm2_weight", "norm2_bias")])
        _check(lib().ptts_b200_model_load_layer(self._h, layer, ctypes.byref(lw)))

    def load(self, weights: "Weights"):
        for l in range(self.cfg.num_layers):
            self.load_layer(l, weights.layer(l))

    _DENSE = ("in_proj", "out_proj", "linear1", "linear2", "norm1_weight", "norm1_bias", "norm2_weight",
              "norm2_bias")

    def load_layer_f32(self, layer: int, w: dict):
        """Dense f32 linears [out][in] (ptts_b200_model_load_layer_f32); keys as load_layer's."""
        keep = {k: np.ascontiguousarray(w[k], dtype=np.float32) for k in self._DENSE}
        lw = LayerWeightsF32(*[keep[n].ctypes.data for n in self._DENSE])
        _check(lib().ptts_b200_model_load_layer_f32(self._h, layer, ctypes.byref(lw)))

    def set_layer_scale(self, layer: int, scale1=None, scale2=None):
        """LayerScale factors of one layer (ptts_b200_model_set_layer_scale): [d_model] each, or
        None for none."""
        keep = [None if v is None else np.ascontiguousarray(v, dtype=np.float32) for v in (scale1, scale2)]
        for v in keep:
            if v is not None and v.shape != (self.cfg.d_model,):
                raise PttsError(ERR_ARG, f"a layer scale has {self.cfg.d_model} entries, not {v.shape}")
        ptrs = [None if v is None else v.ctypes.data_as(P) for v in keep]
        _check(lib().ptts_b200_model_set_layer_scale(self._h, layer, *ptrs))

    def load_mimi(self, tensors: dict, q8_0: bool = False):
        """A Mimi transformer's layers under the checkpoint's names (mimi.rs:359-360 and
        transformer.rs:411-412, 549-563): layers.{i}.self_attn.in_proj.weight [3d, d],
        self_attn.out_proj.weight, linear1.weight, linear2.weight (f32, no biases), norm1/norm2
        weight and bias, layer_scale_1.scale and layer_scale_2.scale. With q8_0, the four
        linears are quantized to q8_0 first (prepare_q8 / apply_q8, transformer.rs:642-673)."""
        for i in range(self.cfg.num_layers):
            p = f"layers.{i}."
            w = {"in_proj": tensors[p + "self_attn.in_proj.weight"], "out_proj": tensors[p + "self_attn.out_proj.weight"],
                 "linear1": tensors[p + "linear1.weight"], "linear2": tensors[p + "linear2.weight"],
                 "norm1_weight": tensors[p + "norm1.weight"], "norm1_bias": tensors[p + "norm1.bias"],
                 "norm2_weight": tensors[p + "norm2.weight"], "norm2_bias": tensors[p + "norm2.bias"]}
            if q8_0:
                for k in ("in_proj", "out_proj", "linear1", "linear2"):
                    w[k] = quantize_q8_0(w[k])
                self.load_layer_q8_0(i, w)
            else:
                self.load_layer_f32(i, w)
            self.set_layer_scale(i, tensors.get(p + "layer_scale_1.scale"), tensors.get(p + "layer_scale_2.scale"))

    def load_layer_q8_0(self, layer: int, w: dict):
        """GGUF q8_0 block bytes for the four linears (uint8 arrays), f32 norms."""
        keep = {k: np.ascontiguousarray(w[k]) for k in self._DENSE}
        lw = LayerWeightsQ8(*[keep[n].ctypes.data for n in self._DENSE])
        _check(lib().ptts_b200_model_load_layer_q8_0(self._h, layer, ctypes.byref(lw)))

    def load_gguf(self, path: str, flow: "Flow" = None):
        """ptts_b200_load_gguf: every layer (and the flow head's tensors) from a GGUF file."""
        _check(lib().ptts_b200_load_gguf(self._h, flow._h if flow is not None else P(), path.encode()))

    def forward(self, kv: KvState, x, streams: Sequence[int], rows: Sequence[int], *, out=None,
                stream=None):
        """StreamingTransformer::forward: x [n_rows, d] bf16 -> [n_rows, d] f32; lengths advance."""
        import torch
        s, r = _i32(streams), _i32(rows)
        if out is None:
            out = torch.empty((x.shape[0], self.cfg.d_model), dtype=torch.float32, device=x.device)
        _check(lib().ptts_b200_forward(self._h, kv.handle, _dptr(x), _ip(s), _ip(r), len(s),
                                       _dptr(out), _stream(stream)))
        return out

    def step(self, kv: KvState, streams: Sequence[int], x, *, out=None, stream=None):
        """StreamingTransformer::forward_step: one row per stream, positions on the device, one
        CUDA graph per stream set. x [n, d] bf16 and out [n, d] f32 may be CUDA or pinned host."""
        import torch
        s = _i32(streams)
        if out is None:
            out = torch.empty((len(s), self.cfg.d_model), dtype=torch.float32, device=x.device)
        _check(lib().ptts_b200_step(self._h, kv.handle, _ip(s), len(s), ctypes.c_void_p(x.data_ptr()),
                                    ctypes.c_void_p(out.data_ptr()), _stream(stream)))
        return out

    def stamps(self, max_launches: int):
        """ptts_b200_model_stamps: kernel timeline of decode steps on (max_launches slots) or off (0)."""
        _check(lib().ptts_b200_model_stamps(self._h, int(max_launches)))

    def read_stamps(self) -> list:
        """The last step's launches: dicts of kernel, lane, layer and entry/start/end in µs."""
        buf = (Stamp * 4096)()
        n = ctypes.c_int(0)
        _check(lib().ptts_b200_model_stamps_read(self._h, buf, 4096, ctypes.byref(n)))
        return [{"kernel": b.kernel.decode(), "lane": b.lane, "layer": b.layer, "entry_us": b.entry_us,
                 "start_us": b.start_us, "end_us": b.end_us, "last_entry_us": b.last_entry_us}
                for b in buf[:n.value]]


# --------------------------------------------------------------------------------------------
# synthetic weights (random init in the checkpoint's layout)
# --------------------------------------------------------------------------------------------

@dataclass
class Weights:
    """All layers' weights, numpy, concatenated over layers (the oracle takes the same)."""
    w_qkv: np.ndarray
    s_qkv: np.ndarray
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

    def layer(self, l: int) -> dict:
        return dict(in_proj=self.w_qkv[l], in_proj_scale=self.s_qkv[l], out_proj=self.w_out[l],
                    out_proj_scale=self.s_out[l], linear1=self.w_ff1[l], linear1_scale=self.s_ff1[l],
                    linear2=self.w_ff2[l], linear2_scale=self.s_ff2[l], norm1_weight=self.ln1_g[l],
                    norm1_bias=self.ln1_b[l], norm2_weight=self.ln2_g[l], norm2_bias=self.ln2_b[l])


LN_GAIN = 1.0 / 16.0


def random_weights(cfg: FlowLMConfig, seed: int, *, ln_random: bool = False,
                   ln_gain: float = LN_GAIN) -> Weights:
    """int8 ~ U{-127..127}, scales ~ U(0.005, 0.02) per output row, LayerNorm gain `ln_gain`
    and bias 0 (or random affine parameters when ln_random, for tests).

    The gain is 1/16 rather than 1: with these int8 scales a unit gain gives q and k entries of
    std ~20 and attention logits of std ~430, an almost-argmax attention under which a one-ulp
    bf16 difference anywhere flips near-tied keys and the hidden states of two correct
    implementations part by O(1) within a few layers. Gain 1/16 gives logits of std ~1.7, the
    regime of a trained model. The byte and flop counts are the same either way."""
    rng = np.random.default_rng(seed)
    L, d, hd = cfg.num_layers, cfg.d_model, cfg.num_heads * cfg.head_dim
    nqkv = hd + 2 * cfg.num_kv_heads * cfg.head_dim
    ff = cfg.dim_feedforward

    def q(n, k):
        return rng.integers(-127, 128, size=(L, n, k), dtype=np.int8)

    def s(n):
        return rng.uniform(0.005, 0.02, size=(L, n)).astype(np.float32)

    w_qkv, s_qkv = q(nqkv, d), s(nqkv)
    w_out, s_out = q(d, hd), s(d)
    w_ff1, s_ff1 = q(ff, d), s(ff)
    w_ff2, s_ff2 = q(d, ff), s(d)
    if ln_random:
        ln = [rng.uniform(0.5, 1.5, (L, d)).astype(np.float32), rng.normal(0, 0.1, (L, d)).astype(np.float32),
              rng.uniform(0.5, 1.5, (L, d)).astype(np.float32), rng.normal(0, 0.1, (L, d)).astype(np.float32)]
    else:
        ln = [np.full((L, d), ln_gain, np.float32), np.zeros((L, d), np.float32),
              np.full((L, d), ln_gain, np.float32), np.zeros((L, d), np.float32)]
    return Weights(w_qkv, s_qkv, w_out, s_out, w_ff1, s_ff1, w_ff2, s_ff2, *ln)


# --------------------------------------------------------------------------------------------
# flow head (FlowLM's frame tail, flow_lm.rs:296-410; SimpleMLPAdaLN, mlp.rs)
# --------------------------------------------------------------------------------------------

FLOW_TYPES = {"lsd": 0, "drifting": 1, "pointwise": 2}
TIME_NORMS = {"rms": 0, "rms_var": 1}


@dataclass
class FlowConfig:
    """The flow head's shape (FlowLMConfig flow_* fields, flow_lm.rs:114-146). Phonon: flow_dim
    512, depth 6, ldim 32, one LSD step, the uncentred RMS time norm."""
    d_model: int = 512
    flow_dim: int = 512
    flow_depth: int = 6
    ldim: int = 32
    freq_dim: int = 256
    flow_type: str = "lsd"
    lsd_steps: int = 1
    time_norm: str = "rms"

    @property
    def time_conds(self) -> int:
        return 2 if self.flow_type == "lsd" else 0

    def c_struct(self) -> FlowConfigC:
        return FlowConfigC(self.d_model, self.flow_dim, self.flow_depth, self.ldim, self.freq_dim,
                           FLOW_TYPES[self.flow_type], self.lsd_steps, TIME_NORMS[self.time_norm])

    def shapes(self) -> dict:
        """Every tensor ptts_b200_flow_set_tensor takes, name -> shape (the checkpoint's keys)."""
        d, C, L, F = self.d_model, self.flow_dim, self.ldim, self.freq_dim
        sh = {"input_linear.weight": (d, L), "out_norm.weight": (d,), "out_norm.bias": (d,),
              "out_eos.weight": (1, d), "out_eos.bias": (1,), "bos_emb": (L,),
              "flow_net.input_proj.weight": (C, L), "flow_net.input_proj.bias": (C,),
              "flow_net.cond_embed.weight": (C, d), "flow_net.cond_embed.bias": (C,),
              "flow_net.final_layer.adaLN_modulation.1.weight": (2 * C, C),
              "flow_net.final_layer.adaLN_modulation.1.bias": (2 * C,),
              "flow_net.final_layer.linear.weight": (L, C), "flow_net.final_layer.linear.bias": (L,)}
        for i in range(self.time_conds):
            p = f"flow_net.time_embed.{i}."
            sh.update({p + "freqs": (F // 2,), p + "mlp.0.weight": (C, F), p + "mlp.0.bias": (C,),
                       p + "mlp.2.weight": (C, C), p + "mlp.2.bias": (C,), p + "mlp.3.alpha": (C,)})
        for b in range(self.flow_depth):
            p = f"flow_net.res_blocks.{b}."
            sh.update({p + "in_ln.weight": (C,), p + "in_ln.bias": (C,), p + "mlp.0.weight": (C, C),
                       p + "mlp.0.bias": (C,), p + "mlp.2.weight": (C, C), p + "mlp.2.bias": (C,),
                       p + "adaLN_modulation.1.weight": (3 * C, C), p + "adaLN_modulation.1.bias": (3 * C,)})
        return sh


PHONON_FLOW = FlowConfig()


def random_flow_weights(cfg: FlowConfig, seed: int, *, bf16_exact: bool = False,
                        condition: bool = False) -> dict:
    """Random-init flow-head tensors under the checkpoint's names: Linear weights and biases
    U(-1/sqrt(in), 1/sqrt(in)) (torch's default init), LayerNorm gains near 1, time-embedder
    frequencies exp(-ln(10^4) j / (F/2)) and alphas near 1. bf16_exact rounds the large linears'
    weights to bf16 (the form the reference's CUDA backend holds them in)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in cfg.shapes().items():
        if name.endswith(".freqs"):
            half = shape[0]
            v = np.exp(-np.log(10000.0) * np.arange(half) / half)
        elif name.endswith("alpha") or name.endswith("in_ln.weight") or name == "out_norm.weight":
            v = rng.uniform(0.8, 1.2, shape)
        elif name.endswith("in_ln.bias") or name == "out_norm.bias":
            v = rng.normal(0.0, 0.05, shape)
        elif name == "bos_emb":
            v = rng.normal(0.0, 1.0, shape)
        else:
            fan_in = shape[1] if len(shape) == 2 else cfg.shapes()[name[:-len("bias")] + "weight"][1]
            bound = 1.0 / np.sqrt(fan_in)
            v = rng.uniform(-bound, bound, shape)
        v = v.astype(np.float32)
        if bf16_exact and len(shape) == 2 and shape[0] >= 128 and shape[1] >= 128:
            v = round_bf16_np(v)
        out[name] = v
    if condition:
        out["condition"] = rng.normal(0.0, 0.5, (cfg.d_model,)).astype(np.float32)
    return out


def round_bf16_np(x: np.ndarray) -> np.ndarray:
    """f32 -> nearest-even bf16 -> f32 (finite values)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


class Flow:
    """The flow head on one device: ptts_b200_flow_* and ptts_b200_frame."""

    def __init__(self, cfg: FlowConfig, device: int = 0):
        self.cfg, self.device = cfg, device
        h = P()
        st = cfg.c_struct()
        _check(lib().ptts_b200_flow_create(device, ctypes.byref(st), ctypes.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().ptts_b200_flow_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set(self, name: str, value: np.ndarray):
        a = np.ascontiguousarray(value, dtype=np.float32)
        _check(lib().ptts_b200_flow_set_tensor(self._h, name.encode(), a.ctypes.data_as(P), a.size))

    def load(self, tensors: dict):
        for k, v in tensors.items():
            self.set(k, v)
        _check(lib().ptts_b200_flow_finish(self._h))

    def sample(self, t_out, noise, *, stream=None):
        """FlowLM::sample_from_noise: t_out [n, d] f32, noise [n, ldim] f32 (CUDA) -> (latent, eos)."""
        import torch
        n = t_out.shape[0]
        latent = torch.empty((n, self.cfg.ldim), dtype=torch.float32, device=t_out.device)
        eos = torch.empty((n,), dtype=torch.float32, device=t_out.device)
        _check(lib().ptts_b200_flow_sample(self._h, _dptr(t_out), n, _dptr(noise), _dptr(latent),
                                           _dptr(eos), _stream(stream)))
        return latent, eos

    def frame(self, model: Transformer, kv: KvState, streams: Sequence[int], latent, noise, *,
              stream=None):
        """One frame: latent [n, ldim] f32 (None: bos_emb) and noise [n, ldim] f32 on the device
        -> (next latent, eos logits). Lengths advance by one."""
        import torch
        s = _i32(streams)
        n = len(s)
        out = torch.empty((n, self.cfg.ldim), dtype=torch.float32, device=noise.device)
        eos = torch.empty((n,), dtype=torch.float32, device=noise.device)
        lat = _dptr(latent) if latent is not None else P()
        _check(lib().ptts_b200_frame(model._h, self._h, kv.handle, _ip(s), n, lat, _dptr(noise),
                                     _dptr(out), _dptr(eos), _stream(stream)))
        return out, eos


def gguf_remap_key(name: str):
    """loader.rs remap_key through the library: the new name, or None when dropped."""
    buf = ctypes.create_string_buffer(4096)
    rc = lib().ptts_b200_gguf_remap_key(name.encode(), buf, len(buf))
    if rc < 0:
        _check(rc)
    return buf.value.decode() if rc == 1 else None
