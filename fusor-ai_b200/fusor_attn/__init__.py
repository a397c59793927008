"""fusor_attn: the B200 attention hot path of fusor-ai behind its KvCache / Span / Mask API.

A thin ctypes binding of ``libfa_attn.so`` (include/fa_attn.h) whose names follow the
reference's ``blocks::transformer`` and ``blocks::attention`` (crates/blocks/src/transformer.rs,
attention.rs, rotary.rs). Device tensors are torch tensors (PyTorch is the plumbing for memory
and streams); every computation runs in this library's CUDA kernels. There is no CPU fallback:
without the built library, or without a CUDA device, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# FA_ATTN_LIB points at another build of the library (a tuning variant); default in-tree.
LIB_PATH = os.environ.get("FA_ATTN_LIB") or os.path.join(_HERE, "libfa_attn.so")

OK, ERR_ARG, ERR_SHAPE, ERR_CAPACITY, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED = range(7)
F32, BF16 = 0, 1
MASK_CAUSAL, MASK_WINDOW, MASK_FULL, MASK_GROUPS = range(4)
ROPE_NONE, ROPE_HALF, ROPE_INTERLEAVED = range(3)
NORM_NONE, NORM_ROW, NORM_HEAD = range(3)
GATE_NONE, GATE_ELEMENTWISE, GATE_HEADWISE = range(3)
(ROT_SEQUENCE, ROT_LINEAR, ROT_PARTIAL, ROT_MULTIMODAL, ROT_AXES, ROT_MULTIMODAL_INTERLEAVED,
 ROT_GRID) = range(7)


class FaError(RuntimeError):
    """A non-zero status of the C ABI; `code` is the FA_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class CapacityError(FaError):
    """The span does not fit the cache: the reference panics with "the cache holds every key
    the span sees" (transformer.rs:335-338)."""


class ShapeError(FaError):
    """heads % kv_heads != 0 and the like (transformer.rs:389-393)."""


# ---- C structures (include/fa_attn.h) --------------------------------------------------------

class _Mask(C.Structure):
    _fields_ = [("kind", C.c_int32), ("window", C.c_int32), ("state", C.c_int32),
                ("n_ends", C.c_int32), ("ends", C.POINTER(C.c_int32))]


class _Span(C.Structure):
    _fields_ = [("rows", C.c_int32), ("first", C.c_int32), ("mask", _Mask)]


class _Position(C.Structure):
    _fields_ = [("temporal", C.c_int32), ("height", C.c_int32), ("width", C.c_int32)]


class _Rotation(C.Structure):
    _fields_ = [("kind", C.c_int32), ("params", C.c_int32 * 3), ("base", C.c_float),
                ("spatial_scale", C.c_float)]


class _HeadNorm(C.Structure):
    _fields_ = [("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("eps", C.c_float)]


class _Linear(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("weight_stride", C.c_int64), ("bias", C.c_void_p),
                ("inputs", C.c_int32), ("outputs", C.c_int32)]


def _linear(weight, bias=None):
    """A device f32 weight matrix (outputs x inputs, rows weight.stride(0) apart) and bias."""
    return _Linear(_dptr(weight), weight.stride(0), _dptr(bias), weight.shape[1], weight.shape[0])


class _Operand(C.Structure):
    _fields_ = [("values", C.c_void_p), ("stride", C.c_int64), ("offset", C.c_int64)]


class _Call(C.Structure):
    _fields_ = [("heads", C.c_int32), ("kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("images", C.c_int32), ("queries", C.c_int32), ("keys", C.c_int32),
                ("query", _Operand), ("key", _Operand), ("value", _Operand),
                ("dtype", C.c_int32), ("out_dtype", C.c_int32)]


class _RelposCall(C.Structure):
    _fields_ = [("heads", C.c_int32), ("head_dim", C.c_int32), ("frames", C.c_int32),
                ("query", _Operand), ("key", _Operand), ("value", _Operand),
                ("positions", C.c_void_p), ("positions_stride", C.c_int64),
                ("bias_u", C.c_void_p), ("bias_v", C.c_void_p)]


class _Prologue(C.Structure):
    _fields_ = [("tokens", C.c_int32), ("heads", C.c_int32), ("head_dim", C.c_int32),
                ("norm", C.c_int32), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("eps", C.c_float), ("rope", C.c_int32), ("angles", C.c_void_p),
                ("rotated_rows", C.c_int32)]


_lib = None

# name -> (restype, argtypes) for every entry point of include/fa_attn.h
_P, _I32, _I64 = C.c_void_p, C.c_int32, C.c_int64
SIGNATURES = {
    "fa_last_error": (C.c_char_p, []),
    "fa_capabilities": (C.c_int, [_P, _P, _I32, _P]),
    "fa_kvcache_create": (C.c_int, [_I32, _I32, _I32, _I32, _I32, _I32, _I32, C.POINTER(_P)]),
    "fa_kvcache_destroy": (C.c_int, [_P]),
    "fa_kvcache_data": (C.c_int, [_P, C.POINTER(_P), C.POINTER(_P), _P, _P]),
    "fa_kvcache_reserve": (C.c_int, [_P, _I32]),
    "fa_kvcache_copy_rows": (C.c_int, [_P, _I32, _P, _P, _P]),
    "fa_kvcache_put_rows": (C.c_int, [_P, _I32, _P, _P, _P]),
    "fa_rotary_angles": (C.c_int, [_P, _I32, _P, _I32, _P]),
    "fa_attention_input": (C.c_int, [_P, _I32, _P, _I32, _P, _P, _P, _I64, _P, _P]),
    "fa_attend": (C.c_int, [_P, _I32, _P, _P, _I64, _P, _I64, _P]),
    "fa_rotate_queries": (C.c_int, [_I32, _I32, _I32, _I32, _P, _P, _P, _I64, _P, _I64, _P]),
    "fa_attention": (C.c_int, [_P, _I32, _P, _I32, _P, _P, _P, _I64, _P, _I64, _P]),
    "fa_attention_host": (C.c_int, [_P, _I32, _P, _I32, _P, _P, _P, _I64, _P, _I64, _P]),
    "fa_attention_batch": (C.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _I64, _P, _I64, _P]),
    "fa_attention_batch_host": (C.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _I64, _P, _I64,
                                          _P]),
    "fa_attention_input_batch": (C.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _I64, _P, _I64, _P]),
    "fa_peer_buffer_bytes": (C.c_int, [_I32, _I32, _I32, C.POINTER(C.c_uint64)]),
    "fa_peer_alloc": (C.c_int, [C.c_uint64, C.POINTER(_P), _P]),
    "fa_peer_open": (C.c_int, [_P, C.POINTER(_P)]),
    "fa_peer_close": (C.c_int, [_P]),
    "fa_peer_free": (C.c_int, [_P]),
    "fa_exchange_merge": (C.c_int, [_P, C.c_uint64, _I32, _I32, _I32, _I32, _P, _P, _P]),
    "fa_peer_reset": (C.c_int, [_P, C.c_uint64, _P]),
    "fa_attention_input_projected": (C.c_int, [_P, _I32, _P, _I32, _P, _P, _P, _P, _I64, _P, _P,
                                               _I64, _P]),
    "fa_attention_input_projected_batch": (C.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P,
                                                     _I64, _P, _I64, _P]),
    "fa_attend_batch": (C.c_int, [_P, _P, _I32, _I32, _P, _I64, _P, _I64, _P]),
    "fa_attend_partial": (C.c_int, [_P, _I32, _P, _I32, _I32, _P, _P]),
    "fa_attend_static": (C.c_int, [_P, _I32, _P, _P, _I64, _P, _I64, _P]),
    "fa_merge_partials": (C.c_int, [_P, _I32, _I32, _I32, _P, _P]),
    "fa_attend_full": (C.c_int, [_P, _P, _I64, _P]),
    "fa_attend_relpos": (C.c_int, [_P, _P, _I64, _P]),
    "fa_normalize_and_rotate": (C.c_int, [_P, _P, _I64, _P, _I64, _I32, _P]),
    "fa_gated_attention": (C.c_int, [_P, _I32, _P, _I32, _I32, _P, _P, _P, _I64, _P, _I64, _P]),
    "fa_device_status": (C.c_int, [_P]),
    "fa_rng_fill_normal": (C.c_int, [C.c_uint64, _P, _I64]),
}


def lib():
    """The loaded library (built first if it is missing or stale in a source checkout)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import _build
            _build.build()
        _lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _check(rc: int):
    if rc == OK:
        return
    msg = lib().fa_last_error().decode(errors="replace")
    cls = {ERR_CAPACITY: CapacityError, ERR_SHAPE: ShapeError}.get(rc, FaError)
    raise cls(rc, msg)


def _stream(stream=None):
    import torch
    if stream is None:
        # torch's current stream on the current device, as a raw handle: the Stream object
        # (torch.cuda.current_stream) costs several microseconds per call on a decode step
        raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
        if raw is not None:
            return C.c_void_p(raw(torch.cuda.current_device()))
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def _dptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


# ---- the reference's types -------------------------------------------------------------------

@dataclass(frozen=True)
class Mask:
    """transformer::Mask (transformer.rs:97-111)."""
    kind: int = MASK_CAUSAL
    window: int = 0
    state: int = 0
    ends: tuple = ()

    @staticmethod
    def causal() -> "Mask":
        return Mask(MASK_CAUSAL)

    @staticmethod
    def window_of(n: int) -> "Mask":
        return Mask(MASK_WINDOW, window=n)

    @staticmethod
    def full() -> "Mask":
        return Mask(MASK_FULL)

    @staticmethod
    def groups(state: int, ends: Sequence[int]) -> "Mask":
        return Mask(MASK_GROUPS, state=state, ends=tuple(int(e) for e in ends))


@dataclass(frozen=True)
class Span:
    """Span (transformer.rs:272-279): `rows` positions from `first` under `mask`."""
    rows: int
    first: int
    mask: Mask = field(default_factory=Mask.causal)

    def c(self) -> _Span:
        ends = (C.c_int32 * max(len(self.mask.ends), 1))(*self.mask.ends)
        s = _Span(self.rows, self.first,
                  _Mask(self.mask.kind, self.mask.window, self.mask.state, len(self.mask.ends),
                        C.cast(ends, C.POINTER(C.c_int32)) if self.mask.ends else None))
        s._keep = ends  # keep the ends array alive with the struct
        return s


@dataclass(frozen=True)
class Position:
    """rotary::Position (rotary.rs:27-33)."""
    temporal: int
    height: int
    width: int

    @staticmethod
    def uniform(index: int) -> "Position":
        return Position(index, index, index)


@dataclass(frozen=True)
class Rotation:
    """rotary::Rotation (rotary.rs:62-86) with the Rotary's base and spatial scale."""
    kind: int = ROT_SEQUENCE
    params: tuple = (0, 0, 0)
    base: float = 10000.0
    spatial_scale: float = 1.0

    def c(self) -> _Rotation:
        return _Rotation(self.kind, (C.c_int32 * 3)(*self.params), self.base, self.spatial_scale)


def rotary_angles(rotation: Rotation, head_dim: int, positions) -> np.ndarray:
    """Buffers.angles of rows at `positions` (ints or Position): per row the head_dim/2 cosines
    then sines, computed on the host bit for bit as Rotary::angles (rotary.rs:170-178)."""
    pos = [p if isinstance(p, Position) else Position.uniform(int(p)) for p in positions]
    arr = (_Position * max(len(pos), 1))(*[_Position(p.temporal, p.height, p.width) for p in pos])
    out = np.zeros((len(pos), head_dim), np.float32)
    r = rotation.c()
    _check(lib().fa_rotary_angles(C.byref(r), head_dim, arr, len(pos),
                                  out.ctypes.data_as(C.c_void_p)))
    return out


@dataclass(frozen=True)
class Shape:
    """The attention part of transformer::Shape (transformer.rs:54-67)."""
    layers: int
    heads: int
    kv_heads: int
    head_dim: int

    @property
    def qkv(self) -> int:
        """Heads::qkv (layer.rs:45-48): columns of the fused QKV projection."""
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def width(self) -> int:
        """Heads::width (layer.rs:50-53)."""
        return self.heads * self.head_dim


class KvCache:
    """transformer::KvCache (transformer.rs:131-270) in HBM: [layer][kv_head][slot][head_dim]."""

    def __init__(self, shape: Shape, capacity: int, dtype: int = F32, device: int | None = None):
        if device is None:  # the caller's current CUDA device, as torch tensors default to
            import torch
            device = torch.cuda.current_device() if torch.cuda.is_available() else 0
        self.shape, self.capacity, self.dtype, self.device = shape, capacity, dtype, device
        h = C.c_void_p()
        _check(lib().fa_kvcache_create(shape.layers, shape.heads, shape.kv_heads, shape.head_dim,
                                       capacity, dtype, device, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().fa_kvcache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def _torch_dtype(self):
        import torch
        return torch.float32 if self.dtype == F32 else torch.bfloat16

    def reserve(self, rows: int):
        _check(lib().fa_kvcache_reserve(self._h, rows))

    def copy_rows(self, rows: int | None = None, stream=None):
        """KvCache::copy_rows (transformer.rs:221-239) into new device tensors of
        [layers][kv_heads][rows][head_dim]."""
        import torch
        rows = self.capacity if rows is None else rows
        s = self.shape
        dims = (s.layers, s.kv_heads, rows, s.head_dim)
        dev = torch.device("cuda", self.device)
        k = torch.empty(dims, dtype=self._torch_dtype(), device=dev)
        v = torch.empty(dims, dtype=self._torch_dtype(), device=dev)
        _check(lib().fa_kvcache_copy_rows(self._h, rows, _dptr(k), _dptr(v), _stream(stream)))
        return k, v

    def put_rows(self, keys, values, stream=None):
        """KvCache::put_rows (transformer.rs:241-251): [layers][kv_heads][rows][head_dim]."""
        rows = keys.shape[2]
        keys = keys.contiguous()
        values = values.contiguous()
        _check(lib().fa_kvcache_put_rows(self._h, rows, _dptr(keys), _dptr(values),
                                         _stream(stream)))

    def attention_input(self, layer: int, span: Span, qkv, angles=None, rope: int = ROPE_HALF,
                        norm=None, q_out=None, stream=None):
        """RoPE (+ head norm) and keep of a span's rows (layer.rs:175-234)."""
        sp = span.c()
        nm = _norm(norm)
        _check(lib().fa_attention_input(self._h, layer, C.byref(sp), rope if angles is not None else ROPE_NONE,
                                        _dptr(angles), nm, _dptr(qkv), qkv.stride(0),
                                        _dptr(q_out), _stream(stream)))

    def attention_input_projected(self, layer: int, span: Span, x, weight, bias=None,
                                  angles=None, rope: int = ROPE_HALF, norm=None, q_out=None,
                                  qkv_out=None, stream=None):
        """Stack::attention_input (layer.rs:175-209) whole: the qkv projection of the span's
        input rows x (f32 weight: outputs x inputs, optional bias) fused with head norm, RoPE
        and keep; the rotated queries into q_out, the projected rows into qkv_out."""
        sp = span.c()
        lin = _linear(weight, bias)
        _check(lib().fa_attention_input_projected(
            self._h, layer, C.byref(sp), rope if angles is not None else ROPE_NONE,
            _dptr(angles), _norm(norm), C.byref(lin), _dptr(x), x.stride(0), _dptr(q_out),
            _dptr(qkv_out), 0 if qkv_out is None else qkv_out.stride(0), _stream(stream)))

    def attend(self, layer: int, span: Span, q, out, stream=None):
        """KvCache::attend (transformer.rs:182-219) of rotated queries."""
        sp = span.c()
        _check(lib().fa_attend(self._h, layer, C.byref(sp), _dptr(q), q.stride(0), _dptr(out),
                               out.stride(0), _stream(stream)))

    def attention(self, layer: int, span: Span, qkv, out, angles=None, rope: int = ROPE_HALF,
                  norm=None, stream=None):
        """The attention phase of one layer (Cached::keep + Cached::attend) on device tensors."""
        sp = span.c()
        nm = _norm(norm)
        _check(lib().fa_attention(self._h, layer, C.byref(sp),
                                  rope if angles is not None else ROPE_NONE, _dptr(angles), nm,
                                  _dptr(qkv), qkv.stride(0), _dptr(out), out.stride(0),
                                  _stream(stream)))

    def gated_attention(self, layer: int, span: Span, qkv, out, gate: int, rotary_dim: int,
                        angles, norm=None, stream=None):
        """The hybrid blocks' gated attention phase (hybrid/attention.rs:153-295): the heads of
        qkv's rows (query heads, gate heads for GATE_ELEMENTWISE, key heads, value heads, gates
        of whole heads for GATE_HEADWISE) normed and rotated by halves in their first
        rotary_dim elements, kept, attended, and the output times the sigmoid of its gates."""
        sp = span.c()
        _check(lib().fa_gated_attention(self._h, layer, C.byref(sp), gate, rotary_dim,
                                        _dptr(angles), _norm(norm), _dptr(qkv), qkv.stride(0),
                                        _dptr(out), out.stride(0), _stream(stream)))

    def attention_host(self, layer: int, span: Span, qkv: np.ndarray, angles=None,
                       rope: int = ROPE_HALF, norm=None, stream=None) -> np.ndarray:
        """The same on host (numpy) rows, as the reference's host Buffers hold them."""
        qkv = np.ascontiguousarray(qkv, np.float32)
        out = np.zeros((span.rows, self.shape.width), np.float32)
        ang = None if angles is None else np.ascontiguousarray(angles, np.float32)
        sp = span.c()
        nm = _norm(norm)
        _check(lib().fa_attention_host(self._h, layer, C.byref(sp),
                                       rope if ang is not None else ROPE_NONE,
                                       None if ang is None else ang.ctypes.data_as(C.c_void_p), nm,
                                       qkv.ctypes.data_as(C.c_void_p), qkv.shape[1],
                                       out.ctypes.data_as(C.c_void_p), out.shape[1],
                                       _stream(stream)))
        return out

    def attend_partial(self, layer: int, q, key_begin: int, key_end: int, partials, stream=None):
        """A KV-range shard's (max, sum, o) per head over positions [key_begin, key_end)."""
        _check(lib().fa_attend_partial(self._h, layer, _dptr(q), key_begin, key_end,
                                       _dptr(partials), _stream(stream)))


def _norm(norm):
    if norm is None:
        return None
    q, k, eps = norm
    return C.byref(_HeadNorm(_dptr(q), _dptr(k), eps))


def attention_batch(caches: Sequence[KvCache], spans: Sequence[Span], layer: int, qkv, out,
                    angles=None, rope: int = ROPE_HALF, norm=None, stream=None):
    """One decode row of each of `len(caches)` sequences in one launch."""
    n = len(caches)
    handles = (C.c_void_p * n)(*[c.handle.value for c in caches])
    cs = [s.c() for s in spans]
    arr = (_Span * n)(*cs)
    _check(lib().fa_attention_batch(handles, arr, n, layer,
                                    rope if angles is not None else ROPE_NONE, _dptr(angles),
                                    _norm(norm), _dptr(qkv), qkv.stride(0), _dptr(out),
                                    out.stride(0), _stream(stream)))


class Batch:
    """A batch of one-row spans over caches of one shape, its C arrays built once."""

    def __init__(self, caches: Sequence[KvCache], spans: Sequence[Span]):
        n = len(caches)
        self.n = n
        self.caches = list(caches)
        self.handles = (C.c_void_p * n)(*[c.handle.value for c in caches])
        self.spans = (_Span * n)(*[s.c() for s in spans])

    def attention_input(self, layer: int, qkv, q_out=None, angles=None, rope: int = ROPE_HALF,
                        norm=None, stream=None):
        _check(lib().fa_attention_input_batch(
            self.handles, self.spans, self.n, layer, rope if angles is not None else ROPE_NONE,
            _dptr(angles), _norm(norm), _dptr(qkv), qkv.stride(0), _dptr(q_out),
            0 if q_out is None else q_out.stride(0), _stream(stream)))

    def attention_input_projected(self, layer: int, x, weight, bias=None, q_out=None,
                                  angles=None, rope: int = ROPE_HALF, norm=None, stream=None):
        """The qkv projection of each sequence's input row (x row i) fused with head norm,
        RoPE and keep into its own cache; the rotated queries into q_out."""
        lin = _linear(weight, bias)
        _check(lib().fa_attention_input_projected_batch(
            self.handles, self.spans, self.n, layer, rope if angles is not None else ROPE_NONE,
            _dptr(angles), _norm(norm), C.byref(lin), _dptr(x), x.stride(0), _dptr(q_out),
            0 if q_out is None else q_out.stride(0), _stream(stream)))

    def attend(self, layer: int, q, out, stream=None):
        _check(lib().fa_attend_batch(self.handles, self.spans, self.n, layer, _dptr(q),
                                     q.stride(0), _dptr(out), out.stride(0), _stream(stream)))

    def attention(self, layer: int, qkv, out, angles=None, rope: int = ROPE_HALF, norm=None,
                  stream=None):
        _check(lib().fa_attention_batch(self.handles, self.spans, self.n, layer,
                                        rope if angles is not None else ROPE_NONE, _dptr(angles),
                                        _norm(norm), _dptr(qkv), qkv.stride(0), _dptr(out),
                                        out.stride(0), _stream(stream)))

    def attention_host(self, layer: int, qkv, out, angles=None, rope: int = ROPE_HALF, norm=None,
                       stream=None):
        """attention() over HOST tensors (qkv, angles and out in CPU memory, pinned for the
        copies to overlap the attention): returns when out holds every sequence's row."""
        for t in (qkv, out) + ((angles,) if angles is not None else ()):
            if not t.is_cpu or t.stride(-1) != 1:
                raise ValueError("host tensors with unit stride along a row")
        _check(lib().fa_attention_batch_host(self.handles, self.spans, self.n, layer,
                                             rope if angles is not None else ROPE_NONE,
                                             _dptr(angles), _norm(norm), _dptr(qkv),
                                             qkv.stride(0), _dptr(out), out.stride(0),
                                             _stream(stream)))


def rotate_queries(heads: int, head_dim: int, qkv, q_out, angles=None, rope: int = ROPE_HALF,
                   norm=None, stream=None):
    """RoPE (+ query head norm) of the query heads of qkv's rows into q_out, no cache."""
    _check(lib().fa_rotate_queries(heads, head_dim, qkv.shape[0],
                                   rope if angles is not None else ROPE_NONE, _dptr(angles),
                                   _norm(norm), _dptr(qkv), qkv.stride(0), _dptr(q_out),
                                   q_out.stride(0), _stream(stream)))


def merge_partials(partials, out, stream=None):
    """Log-sum-exp merge of shards' partials [shards][heads][head_dim + 2] into out."""
    shards, heads, width = partials.shape
    _check(lib().fa_merge_partials(_dptr(partials), shards, heads, width - 2, _dptr(out),
                                   _stream(stream)))


@dataclass
class Operand:
    """blocks::attention::Operand (attention.rs:24-31) over a device tensor."""
    values: object
    stride: int
    offset: int = 0


def attend_full(heads: int, kv_heads: int, head_dim: int, images: int, queries: int, keys: int,
                query: Operand, key: Operand, value: Operand, out, stream=None):
    """blocks::attention::attend / dit::Within: full-mask attention (attention.rs:79-95)."""
    import torch
    dt = {torch.float32: F32, torch.bfloat16: BF16}
    call = _Call(heads, kv_heads, head_dim, images, queries, keys,
                 _Operand(query.values.data_ptr(), query.stride, query.offset),
                 _Operand(key.values.data_ptr(), key.stride, key.offset),
                 _Operand(value.values.data_ptr(), value.stride, value.offset),
                 dt[query.values.dtype], dt[out.dtype])
    _check(lib().fa_attend_full(C.byref(call), _dptr(out), out.stride(0), _stream(stream)))


def attend_relpos(heads: int, head_dim: int, frames: int, query: Operand, key: Operand,
                  value: Operand, positions, bias_u, bias_v, out, stream=None):
    """conformer::attention::attend (conformer/attention.rs:25-159): full-mask attention with
    Transformer-XL relative-position scores over `positions` ((2 frames - 1) rows)."""
    call = _RelposCall(heads, head_dim, frames,
                       _Operand(query.values.data_ptr(), query.stride, query.offset),
                       _Operand(key.values.data_ptr(), key.stride, key.offset),
                       _Operand(value.values.data_ptr(), value.stride, value.offset),
                       positions.data_ptr(), positions.stride(0), bias_u.data_ptr(),
                       bias_v.data_ptr())
    _check(lib().fa_attend_relpos(C.byref(call), _dptr(out), out.stride(0), _stream(stream)))


def normalize_and_rotate(heads: int, head_dim: int, qkv, out, norm: int = NORM_ROW,
                         q_norm=None, k_norm=None, eps: float = 1e-6, angles=None,
                         rope: int = ROPE_INTERLEAVED, rotated_rows=None, stream=None):
    """The DiT blocks' query/key prologue (wan_dit/block.rs:109-140, pyramid_jit/block.rs:
    100-131 with NORM_ROW; mmdit/pass.rs:162-192 with NORM_HEAD): each token's query and key
    rows of qkv (tokens x stride f32) RMS-normalized and rotated by `angles` (tokens x head_dim),
    into out (f32 or bf16, queries/keys/values as in qkv; out may be qkv itself, f32)."""
    import torch
    tokens = qkv.shape[0]
    p = _Prologue(tokens, heads, head_dim, norm, _dptr(q_norm), _dptr(k_norm), eps,
                  rope if angles is not None else ROPE_NONE, _dptr(angles),
                  tokens if rotated_rows is None else rotated_rows)
    dt = F32 if out.dtype == torch.float32 else BF16
    _check(lib().fa_normalize_and_rotate(C.byref(p), _dptr(qkv), qkv.stride(0), _dptr(out),
                                         out.stride(0), dt, _stream(stream)))


class PeerExchange:
    """This rank's exchange buffer for fa_exchange_merge and the mappings of the other ranks'
    (CUDA IPC handles swapped over `group`, a torch.distributed process group of one process per
    GPU of a box). Every rank takes part in the swap even when its own allocation failed; `ok`
    says whether this rank has every buffer (the ranks agree on it before the first merge)."""

    def __init__(self, heads: int, head_dim: int, group=None):
        import torch.distributed as dist
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.heads, self.head_dim = heads, head_dim
        self.own, self.mapped, self.buffers, self.ok = None, [], None, False
        nbytes = C.c_uint64()
        _check(lib().fa_peer_buffer_bytes(self.world, heads, head_dim, C.byref(nbytes)))
        self.bytes = nbytes.value
        mine = None
        own = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        if lib().fa_peer_alloc(self.bytes, C.byref(own), handle) == OK:
            self.own, mine = own, bytes(handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)  # every rank, allocated or not
        if self.own is None or any(h is None for h in handles):
            return
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.own.value)
                continue
            p = C.c_void_p()
            if lib().fa_peer_open((C.c_ubyte * 64).from_buffer_copy(h), C.byref(p)) != OK:
                return
            self.mapped.append(p)
            ptrs.append(p.value)
        self.buffers = (C.c_void_p * self.world)(*ptrs)
        self.ok = True

    def merge(self, partials, out, stream=None):
        """This rank's (max, sum, o) partials (heads x (head_dim + 2) f32) exchanged with every
        rank's and merged into out (heads x head_dim f32)."""
        _check(lib().fa_exchange_merge(self.buffers, self.bytes, self.rank, self.world,
                                       self.heads, self.head_dim, _dptr(partials), _dptr(out),
                                       _stream(stream)))

    def recover(self, group=None):
        """Checks the exchanges so far on every rank and, if any rank's gave up waiting (its
        output was incomplete: FA_ERR_TIMEOUT), brings the ranks' step counters back in line:
        every rank clears its own buffer's header between two barriers. Collective: every rank
        of the group calls it at the same point. Returns whether any rank had timed out."""
        import torch
        import torch.distributed as dist
        timed_out = 0
        try:
            device_status()
        except FaError as e:
            if e.code != ERR_TIMEOUT:
                raise
            timed_out = 1
        device = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
        flag = torch.tensor([timed_out], device=device, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
        if int(flag.item()) == 0:
            return False
        dist.barrier(group=group)
        _check(lib().fa_peer_reset(self.own, self.bytes, _stream()))
        dist.barrier(group=group)
        return True

    def close(self):
        """Unmaps the other ranks' buffers and frees this one's (after every rank's last merge:
        a barrier of the group first)."""
        for p in self.mapped:
            lib().fa_peer_close(p)
        self.mapped = []
        if self.own:
            lib().fa_peer_free(self.own)
            self.own = None


def device_status(stream=None):
    """Raises FaError(ERR_TIMEOUT) if a kernel gave up a device-side wait."""
    _check(lib().fa_device_status(_stream(stream)))


def rng_normal(seed: int, n: int) -> np.ndarray:
    """kernels::rng::Rng::new(seed).fill_normal (rng.rs:5-52) of n values, on the host."""
    out = np.empty(n, np.float32)
    _check(lib().fa_rng_fill_normal(seed, out.ctypes.data_as(C.c_void_p), n))
    return out


def capabilities():
    flags = C.c_int32()
    dims = (C.c_int32 * 16)()
    n = C.c_int32()
    _check(lib().fa_capabilities(C.byref(flags), dims, 16, C.byref(n)))
    return flags.value, list(dims[: n.value])
