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
