"""The CPU oracle pinned against the reference's own known answers (tests/golden/), and against
the f64 reference attention of the reference's block tests at their tolerance.

These mirror crates/kernels/src/ops.rs's and crates/blocks/src/rotary.rs's unit tests and
crates/blocks/tests/stacks.rs's attention cases (transformer_attends_over_its_cache_like_the_
reference), restricted to the attention phase."""
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)


ROTATIONS = {"axes": oracle.ROT_AXES, "linear": oracle.ROT_LINEAR}


@pytest.mark.parametrize("case", kats()["rotary"], ids=lambda c: c["test"])
def test_rotary_angles_match_the_reference_literals(case):
    cos, sin = oracle.rotary_angles(ROTATIONS[case["rotation"]], case["base"], case["head_dim"],
                                    case["position"], case["params"], case["spatial_scale"])
    got = np.concatenate([cos, sin])
    want = np.array(case["want_cos"] + case["want_sin"], np.float32)
    assert np.abs(got - want).max() < case["tolerance"]


def test_round_bf16_ties_to_even():
    for value, rounded in kats()["round_bf16"]:
        assert oracle.round_bf16(value) == np.float32(rounded)


def test_exp_and_exp_fast_within_the_reference_bounds():
    bounds = kats()["exp"]
    lo, hi = bounds["range"]
    for i in range(lo, hi + 1):
        x = float(np.float32(i) / np.float32(bounds["divisor"]))
        want = math.exp(x)
        assert abs((oracle.exp(x) - want) / want) < bounds["exp_rel"], x
        if x <= 0.0:
            assert abs((oracle.exp_fast(x) - want) / want) < bounds["exp_fast_rel"], x


@pytest.mark.parametrize("fast", [False, True])
def test_exponentials_are_the_scalar_exp_of_every_score_less_their_maximum(fast):
    case = kats()["exponentials"]
    exponential = oracle.exp_fast if fast else oracle.exp
    tolerance = case["tolerance"]["fast" if fast else "exact"]
    for length in case["lengths"]:
        i = np.arange(length, dtype=np.float32)
        # (i as f32).mul_add(-0.37, -1.5): one rounding
        scores = (i.astype(np.float64) * np.float32(case["slope"]) + np.float32(case["intercept"])
                  ).astype(np.float32)
        swept, total = oracle.exponentials_apply(scores, fast)
        m = scores.max()
        for s, v in zip(scores, swept):
            assert np.float32(v).view(np.uint32) == np.float32(exponential(float(np.float32(s - m)))).view(np.uint32)
        want = np.exp((scores - m).astype(np.float64)).sum()
        assert abs(total - want) < tolerance * want


def test_softmax_sums_to_one_and_orders_like_the_scores():
    rng = np.random.default_rng(0)
    s = rng.standard_normal(1000).astype(np.float32)
    p = oracle.softmax(s)
    assert abs(p.sum() - 1.0) < 1e-5
    assert (np.argsort(p, kind="stable") == np.argsort(s, kind="stable")).all()


def test_mask_keys_follow_the_reference_runs():
    # transformer.rs:116-128
    assert oracle.mask_keys(oracle.Mask.causal(), 5, 9) == ((0, 6), (0, 0))
    assert oracle.mask_keys(oracle.Mask.window_of(4), 5, 9) == ((2, 6), (0, 0))
    assert oracle.mask_keys(oracle.Mask.window_of(4), 1, 9) == ((0, 2), (0, 0))
    assert oracle.mask_keys(oracle.Mask.full(), 5, 9) == ((0, 9), (0, 0))
    groups = oracle.Mask.groups(3, [5, 6, 8])
    assert oracle.mask_keys(groups, 1, 8) == ((0, 8), (0, 0))
    assert oracle.mask_keys(groups, 3, 8) == ((0, 3), (3, 5))
    assert oracle.mask_keys(groups, 5, 8) == ((0, 3), (5, 6))
    assert oracle.mask_keys(groups, 7, 8) == ((0, 3), (6, 8))


def test_capacity_rule():
    cache = oracle.Cache(1, 4, 2, 16, 7)
    assert cache.fits(3, 4, oracle.Mask.window_of(4))
    assert not cache.fits(4, 4, oracle.Mask.window_of(4))
    assert cache.fits(3, 4, oracle.Mask.causal())
    assert not cache.fits(3, 5, oracle.Mask.causal())


def _stream(name, masks):
    g = np.load(os.path.join(GOLDEN, "decoder_attention.npz"))
    heads, kv_heads, d, rows = (int(x) for x in g["dims"])
    capacity, call, rope, extra = (int(x) for x in g[f"{name}_meta"])
    mask = masks[name]
    units = heads + 2 * kv_heads
    qkv = g["qkv"].reshape(rows, units * d).copy()
    cache = oracle.Cache(1, heads, kv_heads, d, capacity)
    outs = []
    for first in range(0, rows, call):
        n = min(call, rows - first)
        part = qkv[first:first + n].copy()
        angles = None
        if rope > 0:
            angles = oracle.angles_table(oracle.ROT_SEQUENCE, 10000.0, d, list(range(first, first + n)))
        assert cache.fits(n, first, mask)
        cache.attention_input(0, n, first, max(rope, 0), angles, part, units * d)
        outs.append(cache.attend(0, n, first, mask, part, units * d))
    return np.concatenate(outs), g[f"{name}_want"]


MASKS = {
    "window": oracle.Mask.window_of(4),
    "causal": oracle.Mask.causal(),
    "full": oracle.Mask.full(),
    "groups": oracle.Mask.groups(3, [5, 6, 8]),
}


@pytest.mark.parametrize("name", list(MASKS))
def test_cached_attention_streams_like_the_f64_reference(name):
    got, want = _stream(name, MASKS)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    # stacks.rs:51-56: f32 agrees with the f64 reference within 1e-6 relative L2
    assert rel < 1e-6, rel


def test_oracle_f64_reference_matches_the_numpy_restatement():
    g = np.load(os.path.join(GOLDEN, "decoder_attention.npz"))
    heads, kv_heads, d, rows = (int(x) for x in g["dims"])
    qkv = g["qkv"].astype(np.float64)
    got = oracle.reference_attend_f64(qkv, rows, heads, kv_heads, d, oracle.Mask.causal())
    assert np.abs(got - g["causal_want"]).max() < 1e-12


def test_team_split_matches_one_thread():
    rng = np.random.default_rng(1)
    heads, kv, d, cap = 14, 2, 64, 300
    cache = oracle.Cache(1, heads, kv, d, cap)
    cache.keys[:] = rng.standard_normal(cache.keys.shape)
    cache.values[:] = rng.standard_normal(cache.values.shape)
    qkv = rng.standard_normal((3, (heads + 2 * kv) * d)).astype(np.float32)
    one = cache.attend(0, 3, 200, oracle.Mask.causal(), qkv, qkv.shape[1], threads=1)
    many = cache.attend(0, 3, 200, oracle.Mask.causal(), qkv, qkv.shape[1], threads=4)
    oracle.release()
    assert (one == many).all()


def test_attend_call_full_mask_matches_the_cache_path():
    rng = np.random.default_rng(2)
    heads, d, n = 3, 32, 40
    q = rng.standard_normal((n, heads * d)).astype(np.float32)
    k = rng.standard_normal((n, heads * d)).astype(np.float32)
    v = rng.standard_normal((n, heads * d)).astype(np.float32)
    got = oracle.attend_call(heads, heads, d, 1, n, n, q, heads * d, 0, k, heads * d, 0,
                             v, heads * d, 0)
    cache = oracle.Cache(1, heads, heads, d, n)
    cache.keys[0] = k.reshape(n, heads, d).transpose(1, 0, 2)
    cache.values[0] = v.reshape(n, heads, d).transpose(1, 0, 2)
    want = cache.attend(0, n, 0, oracle.Mask.full(), q, heads * d)
    assert (got == want).all()


# ---- the hybrid blocks' gated attention and the DiT query/key prologue ------------------------

def _rms_f64(x, w, eps):
    """support::rms_norm (crates/blocks/tests/support/mod.rs:301-311) over rows of len(w)."""
    x = x.reshape(-1, len(w))
    inverse = 1.0 / np.sqrt((x * x).sum(axis=1, keepdims=True) / len(w) + eps)
    return (x * inverse * w).reshape(-1)


def _rotate_f64(head, angles, half_pairs):
    """support::rotate (support/mod.rs:389-400) by halves or interleaved."""
    half = len(head) // 2
    out = head.copy()
    for i, a in enumerate(angles):
        f, s = (i, i + half) if half_pairs else (2 * i, 2 * i + 1)
        x, y = head[f], head[s]
        out[f] = x * np.cos(a) - y * np.sin(a)
        out[s] = y * np.cos(a) + x * np.sin(a)
    return out


def _attend_f64(q, k, v, visible):
    s = (q @ k.T) / np.sqrt(q.shape[-1])
    s = np.where(visible, s, -np.inf)
    p = np.exp(s - s.max(axis=1, keepdims=True))
    return (p / p.sum(axis=1, keepdims=True)) @ v


@pytest.mark.parametrize("gate", [0, 1, 2])
@pytest.mark.parametrize("mask_name,call", [("causal", 3), ("full", 8)])
def test_gated_attention_like_the_f64_reference(gate, mask_name, call):
    """The hybrid stack's attention (stacks.rs:669-757 HYBRID: DECODER dims, half of each head
    rotated; read in calls of 3 causal rows or one full call) against an f64 restatement of
    support::gated_attention (support/mod.rs:720-757), every gate kind, within the stack test's
    f32 tolerance (stacks.rs:51-56)."""
    heads, kv, d, rows, rotary_dim, eps, base = 4, 2, 16, 8, 8, 1e-5, 10000.0
    gate_heads = heads if gate == 1 else 0
    head_columns = (heads + gate_heads + 2 * kv) * d
    width = head_columns + (heads if gate == 2 else 0)
    lcg = oracle.Lcg(11)
    qkv = lcg.floats(rows * width, 0.0, 1.0).reshape(rows, width)
    qn = 1.0 + 0.1 * lcg.floats(d, 0.0, 1.0)
    kn = 1.0 + 0.1 * lcg.floats(d, 0.0, 1.0)
    positions = list(range(rows))
    inv = base ** (-np.arange(0, rotary_dim, 2) / rotary_dim)
    # f64: heads normed and rotated, gates through their sigmoid, attention, times the gates
    q64 = np.zeros((rows, heads, d)); k64 = np.zeros((rows, kv, d)); v64 = np.zeros((rows, kv, d))
    g64 = np.zeros((rows, heads, d))
    for r in range(rows):
        row = qkv[r].astype(np.float64)
        ang = positions[r] * inv
        for h in range(heads):
            x = _rms_f64(row[h * d:(h + 1) * d], qn, eps)
            x[:rotary_dim] = _rotate_f64(x[:rotary_dim], ang, True)
            q64[r, h] = x
            if gate == 1:
                g64[r, h] = 1.0 / (1.0 + np.exp(-row[(heads + h) * d:(heads + h + 1) * d]))
            elif gate == 2:
                g64[r, h] = 1.0 / (1.0 + np.exp(-row[head_columns + h]))
            else:
                g64[r, h] = 1.0
        for j in range(kv):
            at = (heads + gate_heads + j) * d
            x = _rms_f64(row[at:at + d], kn, eps)
            x[:rotary_dim] = _rotate_f64(x[:rotary_dim], ang, True)
            k64[r, j] = x
            v64[r, j] = row[(heads + gate_heads + kv + j) * d:(heads + gate_heads + kv + j + 1) * d]
    visible = np.tril(np.ones((rows, rows), bool)) if mask_name == "causal" else np.ones((rows, rows), bool)
    want = np.zeros((rows, heads, d))
    for h in range(heads):
        j = h // (heads // kv)
        want[:, h] = _attend_f64(q64[:, h], k64[:, j], v64[:, j], visible) * g64[:, h]
    # the oracle, in calls
    cache = oracle.Cache(1, heads, kv, d, rows)
    mask = oracle.Mask.causal() if mask_name == "causal" else oracle.Mask.full()
    got = []
    for first in range(0, rows, call):
        n = min(call, rows - first)
        part = qkv[first:first + n].copy()
        angles = oracle.angles_table(oracle.ROT_SEQUENCE, base, rotary_dim,
                                     list(range(first, first + n)))
        cache.gated_input(0, n, first, gate, rotary_dim, angles, part, width, qn, kn, eps)
        attended = cache.attend(0, n, first, mask, part, width)
        got.append(oracle.gate(n, heads, kv, d, gate, part, attended))
    got = np.concatenate(got).reshape(rows, heads, d)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel < 1e-6, rel


@pytest.mark.parametrize("norm,rope", [(1, 2), (2, 2), (2, 1), (0, 2)])
def test_qk_prologue_like_the_f64_reference(norm, rope):
    """Wan's normalize_and_rotate (wan_dit/block.rs:109-140: whole-row RMSNorm, interleaved 3-D
    RoPE by the token's frame, row and column, video.rs:48-55) and MMDiT's head norms
    (mmdit/pass.rs:162-192) against f64, within 1e-6 relative."""
    frames, grid_rows, cols, heads, d, eps, base = 2, 3, 4, 2, 16, 1e-6, 10000.0
    tokens, width = frames * grid_rows * cols, heads * d
    sections = (2, 3, 3)  # Rotation::Axes over d/2 = 8 pairs
    lcg = oracle.Lcg(12)
    qkv = lcg.floats(tokens * 3 * width, 0.0, 1.0).reshape(tokens, 3 * width)
    wq = 1.0 + 0.1 * lcg.floats(width if norm == 1 else d, 0.0, 1.0)
    wk = 1.0 + 0.1 * lcg.floats(width if norm == 1 else d, 0.0, 1.0)
    pos = [(t // (grid_rows * cols), t // cols % grid_rows, t % cols) for t in range(tokens)]
    angles = np.stack([np.concatenate(oracle.rotary_angles(oracle.ROT_AXES, base, d, p, sections))
                       for p in pos])
    got = oracle.qk_prologue(tokens, heads, d, norm, rope, tokens, angles, wq, wk, eps, qkv)
    # f64: the frequencies of each axis section over 2 * section dims (rotary.rs:117-156)
    inv = np.concatenate([base ** (-np.arange(0, 2 * s, 2) / (2 * s)) for s in sections])
    axis = np.repeat([0, 1, 2], sections)
    for t in range(tokens):
        ang = np.array([pos[t][axis[i]] for i in range(d // 2)]) * inv
        for part in range(2):
            x = qkv[t, part * width:(part + 1) * width].astype(np.float64)
            w = (wq if part == 0 else wk).astype(np.float64)
            if norm == 1:
                x = _rms_f64(x, w, eps)
            elif norm == 2:
                x = _rms_f64(x, w, eps)  # rows of len(w) = head_dim: each head on its own
            if rope:
                x = np.concatenate([_rotate_f64(x[h * d:(h + 1) * d], ang, rope == 1)
                                    for h in range(heads)])
            want = x
            g = got[t, part * width:(part + 1) * width]
            assert np.linalg.norm(g - want) / np.linalg.norm(want) < 1e-6
        assert (got[t, 2 * width:] == qkv[t, 2 * width:]).all()


def test_int8_approximation_of_blocks_attention():
    """blocks::attention::attend's int8 path (attention.rs:79-214: Q7b32 keys less their mean and
    values, int8 queries and exponentials) against the f32 attention on C5-like heads: within
    the reference's own bar for quantized paths (stacks.rs:51-56, 3e-2 relative), and the fast
    exponentials no worse than that either."""
    rng = np.random.default_rng(3)
    heads, d, n = 2, 128, 256
    q = rng.standard_normal((n, heads * d)).astype(np.float32)
    k = rng.standard_normal((n, heads * d)).astype(np.float32)
    v = rng.standard_normal((n, heads * d)).astype(np.float32)
    exact = oracle.attend_call(heads, heads, d, 1, n, n, q, heads * d, 0, k, heads * d, 0,
                               v, heads * d, 0)
    for fast in (False, True):
        approx = oracle.attend_int8(heads, heads, d, q, k, v, fast=fast)
        rel = np.linalg.norm(approx - exact) / np.linalg.norm(exact)
        print(f"int8 {'fast' if fast else 'exact'} exponentials: relative L2 {rel:.2e}")
        assert rel < 3e-2, rel
