"""Generates the committed golden fixtures under tests/golden/ (run in the build container, where
the fusor-ai sources are mounted; the fixtures travel, this script's input does not).

1. ``reference_kats.json``: the known-answer literals of the reference's own unit tests, read out
   of its source text (each block is located by a snippet that must be present, so a changed
   reference fails loudly instead of silently producing other numbers):
   - crates/blocks/src/rotary.rs:185-229   rotary cos/sin literals (Axes, spatially scaled, Linear)
   - crates/kernels/src/ops.rs:512-523     round_bf16 ties-to-even cases
   - crates/kernels/src/ops.rs:352-361     exp / exp_fast relative bounds over [-20, 20]
   - crates/kernels/src/ops.rs:454-485     Exponentials::apply scores and sum tolerances
2. ``decoder_attention.npz``: the attention phase of crates/blocks/tests/stacks.rs's DECODER shapes
   (hidden 64, heads 4, kv_heads 2, head_dim 16, 8 rows) for each mask of its STREAMS (stacks.rs:
   222-278), with inputs from the tests' LCG (support/mod.rs:33-44, seed 2) and the output of the
   tests' f64 reference attention (support/mod.rs:471-512), restated here in numpy.

Usage: python tests/golden/make_golden.py <root of the fusor-ai source tree>
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _read(root: str, rel: str) -> str:
    with open(os.path.join(root, rel), encoding="utf-8") as f:
        return f.read()


def _floats(text: str) -> list[float]:
    return [float(x.replace("_", "")) for x in re.findall(r"-?\d[\d_]*\.?[\d_]*(?:e-?\d+)?", text)]


def _array_after(src: str, start: int, name: str) -> list[float]:
    m = re.compile(re.escape(name) + r"\s*=\s*\[([^\]]*)\]").search(src, start)
    if not m:
        raise SystemExit(f"literal {name} not found")
    return _floats(m.group(1))


def rotary_kats(root: str) -> list[dict]:
    src = _read(root, "crates/blocks/src/rotary.rs")
    cases = [
        # (test name, snippet that must follow it, config)
        ("axes_turn_each_section_by_its_own_frequencies",
         "Rotary::new(Rotation::Axes([2, 1, 1]), 10_000.0, 8);",
         {"rotation": "axes", "params": [2, 1, 1], "base": 10000.0, "head_dim": 8,
          "spatial_scale": 1.0, "position": [1, 2, 3]}),
        ("spatial_scale_turns_height_and_width_at_scaled_positions",
         "Rotary::new(Rotation::Axes([2, 1, 1]), 10_000.0, 8).spatially_scaled(0.5);",
         {"rotation": "axes", "params": [2, 1, 1], "base": 10000.0, "head_dim": 8,
          "spatial_scale": 0.5, "position": [1, 2, 3]}),
        ("linear_rotation_divides_every_frequency",
         "Rotary::new(Rotation::Linear(8), 10_000.0, 4);",
         {"rotation": "linear", "params": [8, 0, 0], "base": 10000.0, "head_dim": 4,
          "spatial_scale": 1.0, "position": [4, 4, 4]}),
    ]
    out = []
    for name, snippet, config in cases:
        at = src.index("fn " + name)
        if src.find(snippet, at) < 0:
            raise SystemExit(f"{name}: configuration changed in the reference")
        if "temporal: 1,\n            height: 2,\n            width: 3," not in src[at:at + 600] and \
                config["rotation"] == "axes":
            raise SystemExit(f"{name}: position changed in the reference")
        config = dict(config, test=name, source="crates/blocks/src/rotary.rs",
                      want_cos=_array_after(src, at, "want_cos"),
                      want_sin=_array_after(src, at, "want_sin"), tolerance=1e-6)
        out.append(config)
    return out


def bf16_kats(root: str) -> list[list[float]]:
    src = _read(root, "crates/kernels/src/ops.rs")
    at = src.index("fn round_bf16_rounds_to_nearest_ties_to_even")
    block = src[at:src.index("];", at)]
    pairs = re.findall(r"\(([^,()]+(?:\([^)]*\))?[^,()]*),\s*([^()]+?)\)", block)
    cases = []
    for value, rounded in pairs:
        # values are literal expressions such as `1.0 + 1.0 / 256.0`
        v = eval(value.replace("_", ""), {"__builtins__": {}})  # noqa: S307 - literal arithmetic
        cases.append([float(np.float32(v)), float(rounded.replace("_", ""))])
    if len(cases) != 4:
        raise SystemExit("round_bf16 cases changed in the reference")
    return cases


def exp_bounds(root: str) -> dict:
    src = _read(root, "crates/kernels/src/ops.rs")
    at = src.index("fn exp_and_activations_match_the_f64_reference")
    body = src[at:at + 800]
    for needle in ("for i in -2000..=2000", "let x = i as f32 / 100.0;", "< 4e-7", "< 6e-5"):
        if needle not in body:
            raise SystemExit(f"exp test changed: {needle}")
    return {"range": [-2000, 2000], "divisor": 100.0, "exp_rel": 4e-7, "exp_fast_rel": 6e-5,
            "source": "crates/kernels/src/ops.rs:352-361"}


def exponentials_kats(root: str) -> dict:
    src = _read(root, "crates/kernels/src/ops.rs")
    at = src.index("fn exponentials_are_the_scalar_exp_of_every_score_less_their_maximum")
    body = src[at:at + 1600]
    for needle in ("(Exponentials::Exact, exp as fn(f32) -> f32, 1e-6)",
                   "(Exponentials::Fast, exp_fast, 1e-4)", "for length in [37, 45]",
                   ".map(|i| (i as f32).mul_add(-0.37, -1.5))"):
        if needle not in body:
            raise SystemExit(f"exponentials test changed: {needle}")
    return {"lengths": [37, 45], "slope": -0.37, "intercept": -1.5,
            "tolerance": {"exact": 1e-6, "fast": 1e-4}, "source": "crates/kernels/src/ops.rs:454-485"}


# --- the stacks.rs attention phase -------------------------------------------------------------

def lcg_floats(state: int, count: int, center: float, scale: float):
    out = np.empty(count, np.float32)
    for i in range(count):
        state = (state * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        unit = (state >> 11) / float(1 << 53)
        out[i] = np.float32(center + (2.0 * unit - 1.0) * scale)
    return out, state


def f64_angles(position: int, base: float, head_dim: int) -> np.ndarray:
    """support::angles with every frequency turned by `position` (mod.rs:380-387)."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    return position * base ** (-(2 * i) / head_dim)


def f64_rotate(head: np.ndarray, angles: np.ndarray, interleaved: bool) -> np.ndarray:
    """support::rotate (mod.rs:389-400)."""
    head = head.copy()
    half = len(head) // 2
    for i, a in enumerate(angles):
        f, s = (2 * i, 2 * i + 1) if interleaved else (i, i + half)
        x, y = head[f], head[s]
        head[f] = x * np.cos(a) - y * np.sin(a)
        head[s] = y * np.cos(a) + x * np.sin(a)
    return head


def f64_attend(heads: np.ndarray, n_heads: int, kv_heads: int, d: int, mask) -> np.ndarray:
    """support::attend (mod.rs:471-512)."""
    rows = heads.shape[0]
    group = n_heads // kv_heads
    out = np.zeros((rows, n_heads * d))
    for row in range(rows):
        kind = mask[0]
        if kind == "causal":
            seen = list(range(row + 1))
        elif kind == "window":
            seen = list(range(max(row + 1 - mask[1], 0), row + 1))
        elif kind == "groups" and row >= mask[1]:
            state, ends = mask[1], mask[2]
            end = next(e for e in ends if e > row)
            first = next((e for e in reversed(ends) if e <= row), state)
            seen = list(range(state)) + list(range(first, end))
        else:
            seen = list(range(rows))
        for h in range(n_heads):
            q = heads[row, h]
            scores = np.array([q @ heads[j, n_heads + h // group] / np.sqrt(d) for j in seen])
            w = np.exp(scores - scores.max())
            total = w.sum()
            mixed = np.zeros(d)
            for j, wj in zip(seen, w):
                mixed += wj / total * heads[j, n_heads + kv_heads + h // group]
            out[row, h * d:(h + 1) * d] = mixed
    return out


def decoder_attention() -> dict:
    heads, kv_heads, d, rows, base = 4, 2, 16, 8, 10000.0
    units = heads + 2 * kv_heads
    streams = [
        # (name, mask, capacity, call, interleaved rotary or None) -- stacks.rs:222-278
        ("window", ("window", 4), 7, 3, True),
        ("causal", ("causal",), 8, 3, None),
        ("full", ("full",), 8, 8, None),
        ("groups", ("groups", 3, [5, 6, 8]), 8, 8, None),
    ]
    out = {}
    state = 2  # Weights::new("transformer", 2)
    qkv, state = lcg_floats(state, rows * units * d, 0.0, 1.0)
    qkv = qkv.reshape(rows, units, d)
    out["qkv"] = qkv
    for name, mask, capacity, call, interleaved in streams:
        heads64 = qkv.astype(np.float64)
        if interleaved is not None:
            heads64 = heads64.copy()
            for r in range(rows):
                a = f64_angles(r, base, d)
                for u in range(heads + kv_heads):
                    heads64[r, u] = f64_rotate(heads64[r, u], a, interleaved)
        out[f"{name}_want"] = f64_attend(heads64, heads, kv_heads, d, mask)
        out[f"{name}_meta"] = np.array([capacity, call, -1 if interleaved is None else 2,
                                        mask[1] if len(mask) > 1 else 0], np.int64)
    out["groups_ends"] = np.array([5, 6, 8], np.int64)
    out["dims"] = np.array([heads, kv_heads, d, rows], np.int64)
    return out


def main():
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <root of the fusor-ai source tree>")
    root = sys.argv[1]
    kats = {
        "rotary": rotary_kats(root),
        "round_bf16": bf16_kats(root),
        "exp": exp_bounds(root),
        "exponentials": exponentials_kats(root),
    }
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(kats, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "decoder_attention.npz"), **decoder_attention())
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
