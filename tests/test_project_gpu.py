"""The whole of Stack::attention_input on the device (crates/blocks/src/layer.rs:175-209): the
qkv projection (Linear::project_quads, crates/kernels/src/linear.rs:52-71, f32 weights) fused
with head norm, RoPE and keep. Checked three ways: the projected rows against the oracle's
projection (f64 sums rounded to f32); the kept keys/values and rotated queries bit for bit
against fa_attention_input run on those projected rows (the same epilogue code); and a decode
or prefill step's attention output against the oracle's whole phase."""
import numpy as np
import pytest

import fusor_attn as fa
import oracle
from gpu_util import TOL_F32, Pair, compare, max_abs, normal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def layer_weights(seed, shape, hidden, bias=True):
    """Weights scaled by 1/sqrt(hidden) so that the projected values are of magnitude 1."""
    w = normal(seed, (shape.qkv, hidden)) / np.float32(np.sqrt(hidden))
    b = 0.1 * normal(seed + 1, (shape.qkv,)) if bias else None
    return w.astype(np.float32), None if b is None else b.astype(np.float32)


# (name, heads, kv heads, head_dim, hidden, rows, first, rope, head norms, cache dtype)
CASES = [
    ("qwen2_decode", 14, 2, 64, 896, 1, 1024, fa.ROPE_HALF, False, fa.F32),
    ("qwen2_rows3", 14, 2, 64, 896, 3, 40, fa.ROPE_HALF, False, fa.F32),
    ("qwen2_prefill", 14, 2, 64, 896, 130, 0, fa.ROPE_HALF, False, fa.F32),
    ("qwen3_norms_interleaved", 8, 2, 128, 1024, 9, 17, fa.ROPE_INTERLEAVED, True, fa.F32),
    ("bf16_cache_no_rope", 4, 4, 32, 256, 2, 5, fa.ROPE_NONE, False, fa.BF16),
    ("llama_dims_decode", 32, 8, 128, 4096, 1, 300, fa.ROPE_HALF, False, fa.F32),
    # from 16 rows on the tensor cores (three tf32 products), the hidden dimension split over a
    # cluster: 16 rows (7 splits), a Llama-shaped batch of 64 (3 splits), a hidden dimension that
    # is not a whole number of 32-value blocks with 40 rows over a bf16 cache, and 300 rows
    # (three 128-row tiles, the last one ragged)
    ("qwen2_rows16", 14, 2, 64, 896, 16, 7, fa.ROPE_HALF, False, fa.F32),
    ("llama_dims_rows64", 32, 8, 128, 4096, 64, 300, fa.ROPE_HALF, False, fa.F32),
    ("ragged_hidden_rows40_bf16", 8, 2, 128, 900, 40, 3, fa.ROPE_INTERLEAVED, True, fa.BF16),
    ("rows300", 8, 2, 64, 512, 300, 0, fa.ROPE_HALF, False, fa.F32),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_projected_input_matches_projection_then_input(torch, case):
    name, heads, kv, d, hidden, rows, first, rope, norms, dtype = case
    shape = fa.Shape(1, heads, kv, d)
    cap = first + rows + 3
    w, b = layer_weights(70, shape, hidden)
    x = normal(72, (rows, hidden))
    angles = (fa.rotary_angles(fa.Rotation(base=1e6), d, range(first, first + rows))
              if rope != fa.ROPE_NONE else None)
    norm = None
    if norms:
        norm = (dev(torch, 1.0 + 0.2 * normal(73, (d,))), dev(torch, 1.0 + 0.2 * normal(74, (d,))), 1e-6)
    span = fa.Span(rows, first, fa.Mask.causal())
    fused = fa.KvCache(shape, cap, dtype)
    q_fused = torch.zeros((rows, shape.width), device="cuda")
    qkv_fused = torch.zeros((rows, shape.qkv), device="cuda")
    fused.attention_input_projected(0, span, dev(torch, x), dev(torch, w), dev(torch, b),
                                    angles=None if angles is None else dev(torch, angles),
                                    rope=rope, norm=norm, q_out=q_fused, qkv_out=qkv_fused)
    torch.cuda.synchronize()
    fa.device_status()
    # the projection against the oracle's
    want_qkv = oracle.project(x, w, b)
    got_qkv = qkv_fused.cpu().numpy()
    print(compare(f"{name} projection", got_qkv, want_qkv))
    assert max_abs(got_qkv, want_qkv) <= 2e-5 * max(1.0, np.abs(want_qkv).max())
    # the epilogue against fa_attention_input on the same projected rows: bit for bit
    plain = fa.KvCache(shape, cap, dtype)
    q_plain = torch.zeros((rows, shape.width), device="cuda")
    plain.attention_input(0, span, qkv_fused.clone(), None if angles is None else dev(torch, angles),
                          rope=rope, norm=norm, q_out=q_plain)
    torch.cuda.synchronize()
    kf, vf = fused.copy_rows()
    kp, vp = plain.copy_rows()
    assert torch.equal(kf, kp) and torch.equal(vf, vp)
    assert torch.equal(q_fused, q_plain)


def test_projected_decode_step_matches_the_oracle_phase(torch):
    """Qwen2-0.5B's layer shape (C1): project + keep + attend of one row over a 1024-row cache,
    against the oracle's projection then its attention phase."""
    shape = fa.Shape(1, 14, 2, 64)
    hidden, n = 896, 1024
    pair = Pair(shape, n + 1, filled=n, seed=81)
    w, b = layer_weights(82, shape, hidden)
    x = normal(84, (1, hidden))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 64, [n])
    span = fa.Span(1, n, fa.Mask.causal())
    q = torch.zeros((1, shape.width), device="cuda")
    out = torch.zeros((1, shape.width), device="cuda")
    pair.gpu.attention_input_projected(0, span, dev(torch, x), dev(torch, w), dev(torch, b),
                                       angles=dev(torch, angles), rope=fa.ROPE_HALF, q_out=q)
    pair.gpu.attend(0, span, q, out)
    torch.cuda.synchronize()
    fa.device_status()
    want = pair.oracle_attention(0, span, oracle.project(x, w, b), angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    print(compare("projected decode", got, want))
    assert max_abs(got, want) <= TOL_F32


@pytest.mark.parametrize("n", [12, 64])
def test_projected_batch_keeps_each_sequence_in_its_own_cache(torch, n):
    """A batch of sequences' rows in one projection (12 on the CUDA cores, 64 on the tensor
    cores): each keeps into its own cache at its own position, as single-sequence calls would
    (projected within float rounding)."""
    shape = fa.Shape(1, 8, 2, 64)
    hidden = 512
    w, b = layer_weights(90, shape, hidden)
    x = normal(92, (n, hidden))
    positions = [5 + 7 * i for i in range(n)]
    cap = positions[-1] + 1
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 64, positions)
    caches = [fa.KvCache(shape, cap) for _ in range(n)]
    spans = [fa.Span(1, p, fa.Mask.causal()) for p in positions]
    batch = fa.Batch(caches, spans)
    q = torch.zeros((n, shape.width), device="cuda")
    batch.attention_input_projected(0, dev(torch, x), dev(torch, w), dev(torch, b), q_out=q,
                                    angles=dev(torch, angles), rope=fa.ROPE_HALF)
    torch.cuda.synchronize()
    fa.device_status()
    qkv = oracle.project(x, w, b)
    for i, (c, p) in enumerate(zip(caches, positions)):
        cpu = oracle.Cache(1, shape.heads, shape.kv_heads, 64, cap)
        qi = qkv[i:i + 1].copy()
        cpu.attention_input(0, 1, p, fa.ROPE_HALF, angles[i:i + 1], qi, qi.shape[1])
        k, v = c.copy_rows()
        assert max_abs(k.cpu().numpy()[0, :, p], cpu.keys[0, :, p]) <= 1e-5
        assert max_abs(v.cpu().numpy()[0, :, p], cpu.values[0, :, p]) <= 1e-5
        assert max_abs(q.cpu().numpy()[i], qi[0, :shape.width]) <= 1e-5
        # nothing else of the cache was written
        others = np.delete(np.arange(cap), p)
        assert not k.cpu().numpy()[0][:, others].any()


def test_tensor_core_projection_without_bias(torch):
    """The tensor-core projection with no bias (32 rows, Qwen3's 16/8 x 128 heads over a 2048
    hidden dimension): the projected rows against the oracle's."""
    shape = fa.Shape(1, 16, 8, 128)
    hidden, rows = 2048, 32
    w, _ = layer_weights(95, shape, hidden, bias=False)
    x = normal(96, (rows, hidden))
    span = fa.Span(rows, 0, fa.Mask.causal())
    cache = fa.KvCache(shape, rows)
    qkv = torch.zeros((rows, shape.qkv), device="cuda")
    cache.attention_input_projected(0, span, dev(torch, x), dev(torch, w), None, rope=fa.ROPE_NONE,
                                    qkv_out=qkv)
    torch.cuda.synchronize()
    fa.device_status()
    want = oracle.project(x, w, None)
    got = qkv.cpu().numpy()
    print(compare("tensor-core projection, no bias", got, want))
    assert max_abs(got, want) <= 2e-5 * max(1.0, np.abs(want).max())


def test_projection_argument_errors(torch):
    shape = fa.Shape(1, 4, 2, 32)
    c = fa.KvCache(shape, 16)
    span = fa.Span(1, 0, fa.Mask.causal())
    x = torch.zeros((1, 64), device="cuda")
    q = torch.zeros((1, shape.width), device="cuda")
    with pytest.raises(fa.ShapeError):  # outputs must be (heads + 2 kv_heads) x head_dim
        c.attention_input_projected(0, span, x, torch.zeros((shape.qkv - 32, 64), device="cuda"),
                                    q_out=q)
    with pytest.raises(fa.FaError):  # inputs a multiple of 4
        c.attention_input_projected(0, span, torch.zeros((1, 66), device="cuda")[:, :62],
                                    torch.zeros((shape.qkv, 62), device="cuda"), q_out=q)
