"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

A ctypes binding of ``oracle/oracle.cpp``, the C++ restatement of fusor-ai's f32 attention path
(crates/kernels/src/ops.rs, crates/blocks/src/transformer.rs, crates/blocks/src/rotary.rs).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this module, and only as the checker or the timed CPU baseline: the product library
(``fusor_attn`` / ``libfa_attn.so``) never calls it and has no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

MASK_CAUSAL, MASK_WINDOW, MASK_FULL, MASK_GROUPS, MASK_PREFIX = 0, 1, 2, 3, 4
ROT_SEQUENCE, ROT_LINEAR, ROT_PARTIAL, ROT_MULTIMODAL, ROT_AXES, ROT_MM_INTERLEAVED, ROT_GRID = range(7)


def build(force: bool = False) -> str:
    """Compiles the oracle with its Makefile (g++, -ffp-contract=off)."""
    src = os.path.join(HERE, "oracle.cpp")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class _Mask(C.Structure):
    _fields_ = [("kind", C.c_int), ("window", C.c_int64), ("state", C.c_int64),
                ("ends", C.POINTER(C.c_int64)), ("n_ends", C.c_int64)]


class _Cache(C.Structure):
    _fields_ = [("layers", C.c_int64), ("heads", C.c_int64), ("kv_heads", C.c_int64),
                ("head_dim", C.c_int64), ("capacity", C.c_int64),
                ("keys", C.POINTER(C.c_float)), ("values", C.POINTER(C.c_float))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        f, i, i64, p = C.c_float, C.c_int, C.c_int64, C.c_void_p
        sig = {
            "oracle_rope_inv_freq": (None, [f, i, p]),
            "oracle_rope_half": (None, [p, i, p, p]),
            "oracle_rope_interleaved": (None, [p, i, p, p]),
            "oracle_rotary_angles": (i, [i, p, f, i, f, p, p, p]),
            "oracle_exp": (f, [f]),
            "oracle_exp_fast": (f, [f]),
            "oracle_round_bf16": (f, [f]),
            "oracle_exponentials_apply": (f, [i, p, i]),
            "oracle_softmax": (None, [p, i]),
            "oracle_dot": (f, [p, p, i]),
            "oracle_rms_norm": (None, [p, p, f, i, p]),
            "oracle_mask_keys": (None, [p, i64, i64, p]),
            "oracle_cache_offset": (i64, [p, i64, i64, i64]),
            "oracle_cache_keep": (None, [p, i64, i64, i64, p]),
            "oracle_span_fits": (i, [p, i64, i64, p]),
            "oracle_attention_input": (None, [p, i64, i64, i64, i, p, p, p, f, p, i64]),
            "oracle_cache_attend": (None, [p, i64, i64, i64, p, p, i64, p]),
            "oracle_cache_attend_team": (None, [p, i64, i64, i64, p, p, i64, p, i]),
            "oracle_decode_batch_team": (None, [p, i64, i64, p, p, i64, p, i64, i]),
            "oracle_attend_call": (None, [i64] * 6 + [p, i64, i64] * 3 + [p, i64, i64, i64, i64, i]),
            "oracle_team_release": (None, []),
            "oracle_relpos_attend": (None, [i64, i64, i64, p, p, p, i64, p, i64, p, p, p]),
            "oracle_reference_attend_f64": (None, [p, i64, i64, i64, i64, p, p]),
            "oracle_qk_prologue": (None, [i64, i64, i64, i, i, i64, p, p, p, f, p, i64]),
            "oracle_gated_input": (None, [p, i64, i64, i64, i, i64, p, p, p, f, p, i64]),
            "oracle_gate": (None, [i64, i64, i64, i64, i, p, i64, p]),
            "oracle_attend_int8": (None, [i64] * 5 + [p, i64] * 3 + [i, p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Mask:
    """transformer::Mask (crates/blocks/src/transformer.rs:99-111), plus the tests' Prefix."""

    def __init__(self, kind: int, window: int = 0, state: int = 0, ends=()):
        self.kind, self.window, self.state = kind, window, state
        self.ends = np.ascontiguousarray(ends, dtype=np.int64)

    @staticmethod
    def causal():
        return Mask(MASK_CAUSAL)

    @staticmethod
    def window_of(n: int):
        return Mask(MASK_WINDOW, window=n)

    @staticmethod
    def full():
        return Mask(MASK_FULL)

    @staticmethod
    def groups(state: int, ends):
        return Mask(MASK_GROUPS, state=state, ends=ends)

    def c(self) -> _Mask:
        ends = self.ends.ctypes.data_as(C.POINTER(C.c_int64)) if len(self.ends) else None
        return _Mask(self.kind, self.window, self.state, ends, len(self.ends))


def mask_keys(mask: Mask, position: int, end: int):
    runs = np.zeros(4, dtype=np.int64)
    m = mask.c()
    lib().oracle_mask_keys(C.byref(m), position, end, _ptr(runs))
    return (int(runs[0]), int(runs[1])), (int(runs[2]), int(runs[3]))


def exp(x: float) -> float:
    return lib().oracle_exp(x)


def exp_fast(x: float) -> float:
    return lib().oracle_exp_fast(x)


def round_bf16(x: float) -> float:
    return lib().oracle_round_bf16(x)


def exponentials_apply(scores, fast: bool = False):
    s = _f32(scores).copy()
    total = lib().oracle_exponentials_apply(1 if fast else 0, _ptr(s), len(s))
    return s, total


def softmax(scores):
    s = _f32(scores).copy()
    lib().oracle_softmax(_ptr(s), len(s))
    return s


def rotary_angles(kind: int, base: float, head_dim: int, position, params=(0, 0, 0),
                  spatial_scale: float = 1.0):
    """Rotary::new(...).spatially_scaled(scale).angles(position) -> (cos, sin)."""
    half = head_dim // 2
    cos = np.zeros(half, np.float32)
    sin = np.zeros(half, np.float32)
    prm = np.ascontiguousarray(params, dtype=np.int64)
    pos = np.ascontiguousarray(position, dtype=np.int64)
    rc = lib().oracle_rotary_angles(kind, _ptr(prm), base, head_dim, spatial_scale, _ptr(pos),
                                    _ptr(cos), _ptr(sin))
    if rc != 0:
        raise ValueError("rotary sections do not cover half a head")
    return cos, sin


def angles_table(kind: int, base: float, head_dim: int, positions, params=(0, 0, 0)) -> np.ndarray:
    """Buffers.angles for rows at `positions` (Stack::turn, layer.rs:140-154): per row the
    head_dim/2 cosines then the head_dim/2 sines."""
    out = np.zeros((len(positions), head_dim), np.float32)
    for r, p in enumerate(positions):
        pos = p if isinstance(p, (tuple, list)) else (p, p, p)
        c, s = rotary_angles(kind, base, head_dim, pos, params)
        out[r, : head_dim // 2] = c
        out[r, head_dim // 2:] = s
    return out


class Cache:
    """An f32 KvCache (transformer.rs:134-162) in host memory for the oracle."""

    def __init__(self, layers, heads, kv_heads, head_dim, capacity):
        self.layers, self.heads, self.kv_heads = layers, heads, kv_heads
        self.head_dim, self.capacity = head_dim, capacity
        shape = (layers, kv_heads, capacity, head_dim)
        self.keys = np.zeros(shape, np.float32)
        self.values = np.zeros(shape, np.float32)

    def c(self) -> _Cache:
        fp = C.POINTER(C.c_float)
        return _Cache(self.layers, self.heads, self.kv_heads, self.head_dim, self.capacity,
                      self.keys.ctypes.data_as(fp), self.values.ctypes.data_as(fp))

    def fits(self, rows, first, mask: Mask) -> bool:
        c, m = self.c(), mask.c()
        return bool(lib().oracle_span_fits(C.byref(c), rows, first, C.byref(m)))

    def attention_input(self, layer, rows, first, rope, angles, qkv, stride,
                        q_norm=None, k_norm=None, eps=1e-6):
        """RoPE (+ head norm) and keep, in place on qkv (rows x stride f32)."""
        c = self.c()
        lib().oracle_attention_input(C.byref(c), layer, rows, first, rope,
                                     _ptr(None if angles is None else _f32(angles)),
                                     _ptr(None if q_norm is None else _f32(q_norm)),
                                     _ptr(None if k_norm is None else _f32(k_norm)),
                                     eps, _ptr(qkv), stride)

    def gated_input(self, layer, rows, first, gate, rotary_dim, angles, qkv, stride,
                    q_norm=None, k_norm=None, eps=1e-6):
        """The hybrid blocks' projected heads (hybrid/attention.rs:180-235), in place on qkv."""
        c = self.c()
        lib().oracle_gated_input(C.byref(c), layer, rows, first, gate, rotary_dim,
                                 _ptr(_f32(angles)),
                                 _ptr(None if q_norm is None else _f32(q_norm)),
                                 _ptr(None if k_norm is None else _f32(k_norm)),
                                 eps, _ptr(qkv), stride)

    def attend(self, layer, rows, first, mask: Mask, qkv, stride, threads: int = 1) -> np.ndarray:
        out = np.zeros((rows, self.heads * self.head_dim), np.float32)
        c, m = self.c(), mask.c()
        q = _f32(qkv)
        if threads <= 1:
            lib().oracle_cache_attend(C.byref(c), layer, rows, first, C.byref(m), _ptr(q), stride,
                                      _ptr(out))
        else:
            lib().oracle_cache_attend_team(C.byref(c), layer, rows, first, C.byref(m), _ptr(q),
                                           stride, _ptr(out), threads)
        return out


def attend_call(heads, kv_heads, head_dim, images, queries, keys, q, q_stride, q_offset,
                k, k_stride, k_offset, v, v_stride, v_offset, head_range=None,
                query_range=None, threads=1, out=None) -> np.ndarray:
    """f32 full-mask attention of a blocks::attention::Call with ops::attend arithmetic."""
    hb, he = head_range or (0, heads)
    qb, qe = query_range or (0, queries)
    if out is None:
        out = np.zeros((images * queries, heads * head_dim), np.float32)
    lib().oracle_attend_call(heads, kv_heads, head_dim, images, queries, keys,
                             _ptr(q), q_stride, q_offset, _ptr(k), k_stride, k_offset,
                             _ptr(v), v_stride, v_offset, _ptr(out), hb, he, qb, qe, threads)
    return out


def reference_attend_f64(qkv_heads: np.ndarray, rows, heads, kv_heads, head_dim,
                         mask: Mask) -> np.ndarray:
    """support::attend (crates/blocks/tests/support/mod.rs:471-512) in f64."""
    h = np.ascontiguousarray(qkv_heads, dtype=np.float64)
    out = np.zeros((rows, heads * head_dim), np.float64)
    m = mask.c()
    lib().oracle_reference_attend_f64(_ptr(h), rows, heads, kv_heads, head_dim, C.byref(m),
                                      _ptr(out))
    return out


def relpos_attend(heads, head_dim, frames, qkv, positions, bias_u, bias_v):
    """conformer::attention::attend (conformer/attention.rs:25-159) on rows of qkv (frames x
    3*heads*head_dim: queries, keys, values) and positions ((2 frames - 1) x heads*head_dim)."""
    qkv = _f32(qkv)
    hidden = heads * head_dim
    out = np.zeros((frames, hidden), np.float32)
    base = qkv.ctypes.data
    lib().oracle_relpos_attend(heads, head_dim, frames, C.c_void_p(base), C.c_void_p(base + 4 * hidden),
                               C.c_void_p(base + 8 * hidden), qkv.shape[1], _ptr(_f32(positions)),
                               hidden, _ptr(_f32(bias_u)), _ptr(_f32(bias_v)), _ptr(out))
    return out


def qk_prologue(tokens, heads, head_dim, norm, rope, rotated, angles, q_norm, k_norm, eps,
                qkv) -> np.ndarray:
    """The DiT blocks' query/key prologue (wan_dit/block.rs:109-140, mmdit/pass.rs:162-192) on a
    copy of qkv (tokens x stride f32); returns the copy."""
    out = _f32(qkv).copy()
    lib().oracle_qk_prologue(tokens, heads, head_dim, norm, rope, rotated,
                             _ptr(None if angles is None else _f32(angles)),
                             _ptr(None if q_norm is None else _f32(q_norm)),
                             _ptr(None if k_norm is None else _f32(k_norm)), eps, _ptr(out),
                             out.shape[1])
    return out


def gate(rows, heads, kv_heads, head_dim, gate_kind, qkv, attention) -> np.ndarray:
    """Weights::gate (hybrid/attention.rs:262-295) on a copy of attention."""
    out = _f32(attention).copy()
    q = _f32(qkv)
    lib().oracle_gate(rows, heads, kv_heads, head_dim, gate_kind, _ptr(q), q.shape[1], _ptr(out))
    return out


def attend_int8(heads, kv_heads, head_dim, q, k, v, fast=False) -> np.ndarray:
    """blocks::attention::attend's int8 approximation (attention.rs:79-214) of one image: q
    (queries x heads*head_dim), k and v (keys x kv_heads*head_dim)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.zeros((q.shape[0], heads * head_dim), np.float32)
    lib().oracle_attend_int8(heads, kv_heads, head_dim, q.shape[0], k.shape[0], _ptr(q), q.shape[1],
                             _ptr(k), k.shape[1], _ptr(v), v.shape[1], int(fast), _ptr(out))
    return out


def project(x: np.ndarray, weight: np.ndarray, bias=None) -> np.ndarray:
    """Linear::project_quads for f32 weights (crates/kernels/src/linear.rs:52-71, the matmul of
    crates/kernels/src/matmul.rs over an f32 matrix): out[r][c] = x[r] . weight[c] + bias[c],
    summed here in f64 and rounded once to f32 (the reference's f32 quad sums are within float
    rounding of it; the order of its additions is the backend's)."""
    out = np.asarray(x, np.float64) @ np.asarray(weight, np.float64).T
    if bias is not None:
        out += np.asarray(bias, np.float64)
    return out.astype(np.float32)


def release():
    lib().oracle_team_release()


class Lcg:
    """support::Weights::values (crates/blocks/tests/support/mod.rs:33-44): a 64-bit LCG with
    Knuth's constants, uniform in [-scale, scale]."""

    def __init__(self, seed: int):
        self.state = seed & 0xFFFFFFFFFFFFFFFF

    def floats(self, count: int, center: float = 0.0, scale: float = 1.0) -> np.ndarray:
        out = np.empty(count, np.float32)
        s = self.state
        for i in range(count):
            s = (s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
            unit = (s >> 11) / float(1 << 53)
            out[i] = np.float32(center + (2.0 * unit - 1.0) * scale)
        self.state = s
        return out
