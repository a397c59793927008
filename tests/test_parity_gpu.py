"""Parity of the CUDA path (through the C ABI) with the oracle, on the reference's own test
shapes and masks and on the north-star configurations (full size where the oracle finishes in
seconds, a bounded sample otherwise, with size-independent properties at full size).

Bar: max abs error <= 2e-3 on the attention output with f32 I/O; bf16-storage and bf16-compute
paths are held to the same bar against an oracle given the same bf16-rounded keys and values,
and their error against the unrounded f32 inputs is reported separately."""
import os

import numpy as np
import pytest

import fusor_attn as fa
import oracle
from gpu_util import (TOL_BF16, TOL_F32, Pair, compare, max_abs, normal, parity_ok, relative_l2,
                      round_bf16)

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


# ---- the reference's block tests: crates/blocks/tests/stacks.rs STREAMS ------------------------

STREAM_MASKS = {
    "window": fa.Mask.window_of(4),
    "causal": fa.Mask.causal(),
    "full": fa.Mask.full(),
    "groups": fa.Mask.groups(3, [5, 6, 8]),
}


@pytest.mark.parametrize("name", list(STREAM_MASKS))
@pytest.mark.parametrize("host", [False, True])
def test_decoder_streams_match_the_oracle_and_the_f64_reference(torch, name, host):
    g = np.load(os.path.join(GOLDEN, "decoder_attention.npz"))
    heads, kv_heads, d, rows = (int(x) for x in g["dims"])
    capacity, call, rope, _ = (int(x) for x in g[f"{name}_meta"])
    shape = fa.Shape(1, heads, kv_heads, d)
    pair = Pair(shape, capacity)
    qkv_all = g["qkv"].reshape(rows, shape.qkv)
    outs, wants = [], []
    for first in range(0, rows, call):
        n = min(call, rows - first)
        span = fa.Span(n, first, STREAM_MASKS[name])
        qkv = qkv_all[first:first + n]
        angles = None
        if rope > 0:
            angles = fa.rotary_angles(fa.Rotation(fa.ROT_SEQUENCE, base=10000.0), d,
                                      range(first, first + n))
        if host:
            got = pair.gpu.attention_host(0, span, qkv, angles, rope if rope > 0 else fa.ROPE_NONE)
        else:
            out = torch.zeros((n, shape.width), device="cuda")
            pair.gpu.attention(0, span, dev(torch, qkv), out,
                               None if angles is None else dev(torch, angles),
                               rope if rope > 0 else fa.ROPE_NONE)
            got = out.cpu().numpy()
        want = pair.oracle_attention(0, span, qkv, angles, max(rope, 0), threads=1)
        assert max_abs(got, want) <= 1e-5, compare(name, got, want)
        outs.append(got)
        wants.append(want)
    fa.device_status()
    got = np.concatenate(outs)
    # the reference's own bar for f32 against its f64 reference (stacks.rs:51-56)
    assert relative_l2(got, g[f"{name}_want"]) < 1e-6


def test_the_cache_holds_the_reference_keys_bit_for_bit(torch):
    """RoPE + keep on the device keeps exactly the rotated keys the CPU path keeps."""
    shape = fa.Shape(2, 14, 2, 64)
    pair = Pair(shape, 64)
    qkv = normal(11, (5, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 64, range(7, 12))
    span = fa.Span(5, 7, fa.Mask.causal())
    out = torch.zeros((5, shape.width), device="cuda")
    pair.gpu.attention(1, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    pair.oracle_attention(1, span, qkv, angles, fa.ROPE_HALF)
    k, v = pair.gpu.copy_rows()
    assert (k.cpu().numpy().view(np.uint32) == pair.cpu.keys.view(np.uint32)).all()
    assert (v.cpu().numpy().view(np.uint32) == pair.cpu.values.view(np.uint32)).all()


@pytest.mark.parametrize("rope", [fa.ROPE_HALF, fa.ROPE_INTERLEAVED])
@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
@pytest.mark.parametrize("rows", [3, 1100])
def test_head_dim_128_rotation_and_keep_bit_for_bit(torch, rope, dtype, rows):
    """RoPE + keep at head_dim 128 (a lane holds four consecutive elements; a warp takes four
    rows of a long span): the rotated queries and the kept keys and values equal the oracle's
    bit for bit (a bf16 cache holds them rounded to nearest)."""
    shape = fa.Shape(2, 8, 2, 128)
    pair = Pair(shape, rows, dtype)
    qkv = normal(61, (rows, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 128, range(rows))
    span = fa.Span(rows, 0, fa.Mask.causal())
    q = torch.zeros((rows, shape.width), device="cuda")
    pair.gpu.attention_input(1, span, dev(torch, qkv), dev(torch, angles), rope, q_out=q)
    fa.device_status()
    want_q = qkv.copy()
    pair.cpu.attention_input(1, rows, 0, rope, angles, want_q, want_q.shape[1])
    got_q = np.ascontiguousarray(q.cpu().numpy())
    want_q = np.ascontiguousarray(want_q[:, :shape.width])
    assert (got_q.view(np.uint32) == want_q.view(np.uint32)).all()
    k, v = pair.gpu.copy_rows()
    k, v = k.float().cpu().numpy(), v.float().cpu().numpy()
    wk, wv = pair.cpu.keys, pair.cpu.values
    if dtype == fa.BF16:
        wk, wv = round_bf16(wk), round_bf16(wv)
    assert (k.view(np.uint32) == np.ascontiguousarray(wk).view(np.uint32)).all()
    assert (v.view(np.uint32) == np.ascontiguousarray(wv).view(np.uint32)).all()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_head_norms_and_interleaved_rope(torch, head_dim):
    shape = fa.Shape(1, 8, 2, head_dim)
    pair = Pair(shape, 300, filled=200, seed=5)
    qkv = normal(12, (3, shape.qkv))
    qn = 1.0 + 0.2 * normal(13, (head_dim,))
    kn = 1.0 + 0.2 * normal(14, (head_dim,))
    angles = fa.rotary_angles(fa.Rotation(base=1e4), head_dim, range(200, 203))
    span = fa.Span(3, 200, fa.Mask.causal())
    out = torch.zeros((3, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_INTERLEAVED,
                       norm=(dev(torch, qn), dev(torch, kn), 1e-6))
    q = qkv.copy()
    pair.cpu.attention_input(0, 3, 200, fa.ROPE_INTERLEAVED, angles, q, q.shape[1], qn, kn, 1e-6)
    want = pair.cpu.attend(0, 3, 200, oracle.Mask.causal(), q, q.shape[1])
    got = out.cpu().numpy()
    assert max_abs(got, want) <= 1e-4, compare("head norm", got, want)


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
@pytest.mark.parametrize("head_dim", [16, 32, 64, 128, 256])
def test_every_head_dim_and_storage(torch, dtype, head_dim):
    shape = fa.Shape(1, 8, 2, head_dim)
    pair = Pair(shape, 700, dtype, filled=600, seed=3)
    qkv = normal(21, (2, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), head_dim, [600, 601])
    span = fa.Span(2, 600, fa.Mask.causal())
    out = torch.zeros((2, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    # a bf16 cache of head_dim 128 or 256 decodes on the tensor cores (bf16 queries and
    # probabilities)
    assert parity_ok(got, want, dtype == fa.BF16 and head_dim in (128, 256)), \
        compare(f"d{head_dim}", got, want)


def test_window_ring_wraps_and_groups(torch):
    """A sliding window over a ring smaller than the sequence, streamed for many calls."""
    shape = fa.Shape(1, 6, 3, 64)
    window, call = 50, 7
    pair = Pair(shape, window + call)
    for first in range(0, 300, call):
        span = fa.Span(call, first, fa.Mask.window_of(window))
        qkv = normal(1000 + first, (call, shape.qkv))
        angles = fa.rotary_angles(fa.Rotation(base=1e4), 64, range(first, first + call))
        out = torch.zeros((call, shape.width), device="cuda")
        pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
        want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
        assert max_abs(out.cpu().numpy(), want) <= TOL_F32
    # Groups over a longer call
    pair = Pair(shape, 400, filled=100, seed=9)
    span = fa.Span(120, 100, fa.Mask.groups(130, [150, 151, 190, 220]))
    qkv = normal(77, (120, shape.qkv))
    out = torch.zeros((120, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out)
    want = pair.oracle_attention(0, span, qkv, None, 0)
    assert max_abs(out.cpu().numpy(), want) <= TOL_F32


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
def test_batched_decode_under_groups_masks(torch, dtype):
    """One-row spans under Mask::Groups in one batch (Mask::keys, transformer.rs:119-126: the
    state's run and the row's own group, or every key before the state), beside causal and
    window rows; each against the oracle (two key runs decode on the CUDA cores, in f32)."""
    shape = fa.Shape(1, 8, 2, 128)
    cases = [(700, fa.Mask.groups(300, [650, 701])),   # the state, then its own group
             (90, fa.Mask.groups(91, [91])),           # before the state: every key
             (400, fa.Mask.groups(0, [380, 401])),     # no state: its own group alone
             (512, fa.Mask.causal()),
             (1000, fa.Mask.window_of(333))]
    pairs = [Pair(shape, n + 1, dtype, filled=n, seed=140 + i) for i, (n, _) in enumerate(cases)]
    qkv = normal(141, (len(cases), shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 128, [n for n, _ in cases])
    spans = [fa.Span(1, n, m) for n, m in cases]
    out = torch.zeros((len(cases), shape.width), device="cuda")
    fa.attention_batch([p.gpu for p in pairs], spans, 0, dev(torch, qkv), out, dev(torch, angles),
                       fa.ROPE_HALF)
    fa.device_status()
    got = out.cpu().numpy()
    for i, (p, span) in enumerate(zip(pairs, spans)):
        want = p.oracle_attention(0, span, qkv[i:i + 1], angles[i:i + 1], fa.ROPE_HALF)
        assert max_abs(got[i:i + 1], want) <= TOL_F32, compare(f"groups batch row {i}", got[i:i + 1], want)


def test_capacity_and_span_errors(torch):
    shape = fa.Shape(1, 4, 2, 16)
    cache = fa.KvCache(shape, 8)
    qkv = torch.zeros((4, shape.qkv), device="cuda")
    out = torch.zeros((4, shape.width), device="cuda")
    with pytest.raises(fa.CapacityError):
        cache.attention(0, fa.Span(4, 5, fa.Mask.causal()), qkv, out)
    with pytest.raises(fa.CapacityError):
        cache.attention(0, fa.Span(4, 100, fa.Mask.window_of(5)), qkv, out)
    with pytest.raises(fa.ShapeError):
        cache.attention(1, fa.Span(1, 0), qkv, out)
    with pytest.raises(fa.FaError):
        cache.attention(0, fa.Span(3, 0, fa.Mask.groups(1, [2, 4])), qkv, out)  # last end != 3
    cache.attention(0, fa.Span(0, 0), qkv, out)  # an empty span is a no-op
    # memory the kernels cannot address is refused before any launch, not faulted on
    import ctypes as C
    host = np.zeros((4, shape.width), np.float32)
    sp = fa.Span(1, 3).c()
    rc = fa.lib().fa_attend(cache.handle, 0, C.byref(sp), C.c_void_p(host.ctypes.data), shape.width,
                            C.c_void_p(out.data_ptr()), shape.width, fa._stream())
    assert rc == fa.ERR_ARG and b"pageable host memory" in fa.lib().fa_last_error()
    fa.device_status()


def test_copy_rows_put_rows_round_trip(torch):
    shape = fa.Shape(2, 4, 2, 32)
    pair = Pair(shape, 40, filled=40, seed=4)
    k, v = pair.gpu.copy_rows(17)
    pair.gpu.put_rows(torch.zeros_like(k), torch.zeros_like(v))
    k0, _ = pair.gpu.copy_rows(17)
    assert float(k0.abs().max()) == 0.0
    pair.gpu.put_rows(k, v)
    k2, v2 = pair.gpu.copy_rows()
    assert (k2.cpu().numpy() == pair.cpu.keys).all() and (v2.cpu().numpy() == pair.cpu.values).all()


# ---- north-star configurations ---------------------------------------------------------------

def test_config1_qwen2_decode_full_size(torch):
    """C1: 14 q / 2 kv heads, head_dim 64, decode at position 1024 over 1024 cached positions."""
    shape = fa.Shape(1, 14, 2, 64)
    pair = Pair(shape, 1025, filled=1024, seed=101)
    qkv = normal(102, (1, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 64, [1024])
    span = fa.Span(1, 1024, fa.Mask.causal())
    out = torch.zeros((1, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    print(compare("C1", got, want))
    assert max_abs(got, want) <= TOL_F32


def test_config2_qwen2_prefill_full_size(torch):
    """C2: 512 rows from position 0, causal, the cache written by the same pass."""
    shape = fa.Shape(1, 14, 2, 64)
    pair = Pair(shape, 512)
    qkv = normal(201, (512, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 64, range(512))
    span = fa.Span(512, 0, fa.Mask.causal())
    out = torch.zeros((512, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    print(compare("C2", got, want))
    assert max_abs(got, want) <= TOL_F32


def c3_lengths(seed=301, n=64):
    rng = np.random.default_rng(seed)
    return rng.integers(512, 8193, size=n)


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
def test_config3_batched_decode_sample(torch, dtype):
    """C3 on 8 of its sequences (32 q / 8 kv heads, head_dim 128), one launch."""
    shape = fa.Shape(1, 32, 8, 128)
    lengths = c3_lengths()[:8]
    pairs = [Pair(shape, int(n) + 1, dtype, filled=int(n), seed=310 + i) for i, n in enumerate(lengths)]
    qkv = normal(302, (len(pairs), shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 128, [int(n) for n in lengths])
    spans = [fa.Span(1, int(n), fa.Mask.causal()) for n in lengths]
    out = torch.zeros((len(pairs), shape.width), device="cuda")
    fa.attention_batch([p.gpu for p in pairs], spans, 0, dev(torch, qkv), out, dev(torch, angles),
                       fa.ROPE_HALF)
    fa.device_status()
    got = out.cpu().numpy()
    for i, (p, span) in enumerate(zip(pairs, spans)):
        want = p.oracle_attention(0, span, qkv[i:i + 1], angles[i:i + 1], fa.ROPE_HALF)
        # a bf16 cache decodes on the tensor cores (bf16 queries and probabilities)
        assert parity_ok(got[i:i + 1], want, dtype == fa.BF16), compare(f"C3 seq {i}", got[i:i + 1], want)


@pytest.mark.parametrize("batch,pinned,pad,dtype", [(40, True, 0, fa.F32), (5, False, 0, fa.F32),
                                                     (5, True, 64, fa.F32), (40, False, 64, fa.F32),
                                                     (40, True, 0, fa.BF16), (40, False, 0, fa.BF16)])
def test_config3_batch_from_host_memory(torch, batch, pinned, pad, dtype):
    """fa_attention_batch_host: the rows and angles in host memory (pinned, or pageable); 40
    sequences run as two groups (a quarter of the keys first), the second group's copy
    overlapping the first group's attention and its launch on a second stream, concurrent with
    the first; 5 run as one launch on the caller's stream. A
    pinned output takes the kernels' stores directly (mapped host memory), a pageable one a
    copy; `pad` columns past each output row stay untouched. Every sequence against the oracle
    (a bf16 cache: the tensor-core decode, at the bf16 bar), and against the device-memory batch
    call over the same caches (f32: within f32 rounding; bf16: its chunks differ from the
    groups', so the bf16 probabilities round differently, within the bf16 bar)."""
    shape = fa.Shape(1, 32, 8, 128)
    lengths = [int(n) // 8 for n in c3_lengths(seed=303, n=batch)]
    pairs = [Pair(shape, n + 1, dtype, filled=n, seed=330 + i) for i, n in enumerate(lengths)]
    qkv = normal(304, (batch, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 128, lengths)
    spans = [fa.Span(1, n, fa.Mask.causal()) for n in lengths]
    b = fa.Batch([p.gpu for p in pairs], spans)
    h_qkv, h_angles = torch.from_numpy(qkv), torch.from_numpy(angles)
    h_rows = torch.full((batch, shape.width + pad), 7.0)
    if pinned:
        h_qkv, h_angles, h_rows = h_qkv.pin_memory(), h_angles.pin_memory(), h_rows.pin_memory()
    h_out = h_rows[:, :shape.width]
    b.attention_host(0, h_qkv, h_out, h_angles, fa.ROPE_HALF)
    fa.device_status()
    got = h_out.numpy()
    assert bool((h_rows[:, shape.width:] == 7.0).all())
    bf16 = dtype == fa.BF16
    for i, (p, span) in enumerate(zip(pairs, spans)):
        want = p.oracle_attention(0, span, qkv[i:i + 1], angles[i:i + 1], fa.ROPE_HALF)
        assert parity_ok(got[i:i + 1], want, bf16), compare(f"host batch seq {i}", got[i:i + 1], want)
    # the same step from device memory (the kept rows are written again with the same values)
    out = torch.zeros((batch, shape.width), device="cuda")
    b.attention(0, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    assert float((out.cpu() - h_out).abs().max()) <= (TOL_BF16 if bf16 else 1e-5)


def test_config3_batch_equals_one_call_per_sequence(torch):
    """Batching is invisible: each sequence alone gives the same output (full C3 shape, a
    quarter of the sequences to keep host memory small). Over a bf16 cache the batch decodes on
    the tensor cores and a single span on the CUDA cores: they agree within the bf16 bar."""
    shape = fa.Shape(1, 32, 8, 128)
    lengths = c3_lengths()[:16]
    caches = []
    for i, n in enumerate(lengths):
        c = fa.KvCache(shape, int(n) + 1, fa.BF16)
        k = torch.randn((1, 8, int(n), 128), device="cuda", generator=torch.Generator("cuda").manual_seed(i))
        c.put_rows(k.to(torch.bfloat16), (-k).to(torch.bfloat16))
        caches.append(c)
    qkv = torch.randn((len(caches), shape.qkv), device="cuda")
    spans = [fa.Span(1, int(n), fa.Mask.causal()) for n in lengths]
    out = torch.zeros((len(caches), shape.width), device="cuda")
    fa.attention_batch(caches, spans, 0, qkv, out)
    for i, c in enumerate(caches):
        one = torch.zeros((1, shape.width), device="cuda")
        # the batch already kept row n; attend again over the same keys
        q = qkv[i:i + 1, : shape.width].contiguous()
        c.attend(0, spans[i], q, one)
        assert torch.allclose(one, out[i:i + 1], atol=TOL_BF16, rtol=0)


def test_config4_long_context_sharded_matches_unsharded(torch):
    """C4 at full size (131072 cached + 1 new, 16 q / 8 kv heads, head_dim 128): the KV range
    split into G shards whose partials merge by log-sum-exp equals the single-cache decode, for
    every G of the multi-GPU run; and the oracle agrees on a 16384-position prefix."""
    shape = fa.Shape(1, 16, 8, 128)
    total = 131072
    cache = fa.KvCache(shape, total + 1)
    gen = torch.Generator("cuda").manual_seed(401)
    k = torch.randn((1, 8, total, 128), device="cuda", generator=gen)
    v = torch.randn((1, 8, total, 128), device="cuda", generator=gen)
    cache.put_rows(k, v)
    qkv = torch.randn((1, shape.qkv), device="cuda", generator=gen)
    angles = dev(torch, fa.rotary_angles(fa.Rotation(base=1e6), 128, [total]))
    q = torch.zeros((1, shape.width), device="cuda")
    span = fa.Span(1, total, fa.Mask.causal())
    cache.attention_input(0, span, qkv, angles, fa.ROPE_HALF, q_out=q)
    whole = torch.zeros((1, shape.width), device="cuda")
    cache.attend(0, span, q, whole)
    for shards in (1, 2, 4, 8):
        bounds = np.linspace(0, total + 1, shards + 1).astype(int)
        parts = torch.zeros((shards, 16, 130), device="cuda")
        for s in range(shards):
            cache.attend_partial(0, q, int(bounds[s]), int(bounds[s + 1]), parts[s])
        merged = torch.zeros((16, 128), device="cuda")
        fa.merge_partials(parts, merged)
        assert torch.allclose(merged.reshape(1, -1), whole, atol=2e-5, rtol=0), shards
    fa.device_status()
    # oracle on a prefix
    n = 16384
    small = Pair(shape, n + 1, filled=n, seed=402)
    qkv_np = normal(403, (1, shape.qkv))
    ang = fa.rotary_angles(fa.Rotation(base=1e6), 128, [n])
    q2 = torch.zeros((1, shape.width), device="cuda")
    sp = fa.Span(1, n, fa.Mask.causal())
    small.gpu.attention_input(0, sp, dev(torch, qkv_np), dev(torch, ang), fa.ROPE_HALF, q_out=q2)
    parts = torch.zeros((3, 16, 130), device="cuda")
    for s, (a, b) in enumerate([(0, 5000), (5000, 12000), (12000, n + 1)]):
        small.gpu.attend_partial(0, q2, a, b, parts[s])
    merged = torch.zeros((16, 128), device="cuda")
    fa.merge_partials(parts, merged)
    want = small.oracle_attention(0, sp, qkv_np, ang, fa.ROPE_HALF)
    got = merged.reshape(1, -1).cpu().numpy()
    print(compare("C4 prefix", got, want))
    assert max_abs(got, want) <= TOL_F32


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_config5_full_mask_sample(torch, dtype):
    """C5's shape (12 heads x 128, MHA, full mask) on 2048 tokens, the output checked on the
    first and last 128 queries against the oracle (same bf16-rounded inputs for bf16)."""
    heads, d, n = 12, 128, 2048
    hidden = heads * d
    qkv = normal(501, (n, 3 * hidden))
    if dtype == "bf16":
        qkv = round_bf16(qkv)
    t = dev(torch, qkv)
    if dtype == "bf16":
        t = t.to(torch.bfloat16)
    out = torch.zeros((n, hidden), device="cuda")
    stride = 3 * hidden
    fa.attend_full(heads, heads, d, 1, n, n, fa.Operand(t, stride, 0), fa.Operand(t, stride, hidden),
                   fa.Operand(t, stride, 2 * hidden), out)
    fa.device_status()
    got = out.cpu().numpy()
    want = np.zeros_like(got)
    for qr in ((0, 128), (n - 128, n)):
        oracle.attend_call(heads, heads, d, 1, n, n, qkv, stride, 0, qkv, stride, hidden,
                           qkv, stride, 2 * hidden, query_range=qr, threads=8, out=want)
    rows = np.r_[0:128, n - 128:n]
    print(compare(f"C5 sample {dtype}", got[rows], want[rows]))
    assert parity_ok(got[rows], want[rows], dtype == "bf16")


def test_bf16_tensor_cores_beat_the_reference_int8_approximation(torch):
    """The full-mask attention the reference runs in int8 (attention.rs:79-214, restated in the
    oracle) against this build's bf16 tensor-core path on the same f32 inputs (rounded to bf16
    on the way in): both against the f32 attention, the bf16 path's error the smaller."""
    heads, d, n = 2, 128, 512
    q = normal(701, (n, heads * d))
    k = normal(702, (n, heads * d))
    v = normal(703, (n, heads * d))
    exact = oracle.attend_call(heads, heads, d, 1, n, n, q, heads * d, 0, k, heads * d, 0,
                               v, heads * d, 0)
    int8 = oracle.attend_int8(heads, heads, d, q, k, v)
    ops = [dev(torch, x).to(torch.bfloat16) for x in (q, k, v)]
    out = torch.zeros((n, heads * d), device="cuda")
    fa.attend_full(heads, heads, d, 1, n, n, fa.Operand(ops[0], heads * d),
                   fa.Operand(ops[1], heads * d), fa.Operand(ops[2], heads * d), out)
    fa.device_status()
    got = out.cpu().numpy()
    e_bf16, e_int8 = relative_l2(got, exact), relative_l2(int8, exact)
    print(f"relative L2 against f32: bf16 tensor cores {e_bf16:.2e}, reference int8 {e_int8:.2e}")
    assert e_bf16 < e_int8


def test_full_mask_images_and_gqa(torch):
    """blocks::attention::Call with several images and grouped KV heads."""
    heads, kv, d, images, queries, keys = 8, 2, 64, 3, 40, 56
    q = normal(601, (images * queries, heads * d))
    k = normal(602, (images * keys, kv * d))
    v = normal(603, (images * keys, kv * d))
    out = torch.zeros((images * queries, heads * d), device="cuda")
    fa.attend_full(heads, kv, d, images, queries, keys, fa.Operand(dev(torch, q), heads * d),
                   fa.Operand(dev(torch, k), kv * d), fa.Operand(dev(torch, v), kv * d), out)
    want = oracle.attend_call(heads, kv, d, images, queries, keys, q, heads * d, 0, k, kv * d, 0,
                              v, kv * d, 0)
    assert max_abs(out.cpu().numpy(), want) <= TOL_F32


@pytest.mark.parametrize("case", ["head_dim_32", "unaligned_queries"])
def test_full_mask_on_the_split_kv_kernel(torch, case):
    """f32 full-mask calls the tensor cores do not take (head_dim 32; a query stride of no
    16-byte rows) run on the split-KV kernel with its per-(device, stream) workspace: the oracle's
    output, and the same bits from a call on another stream."""
    d = 32 if case == "head_dim_32" else 64
    heads, kv, images, queries, keys = 6, 2, 2, 70, 90
    qs = heads * d + (1 if case == "unaligned_queries" else 0)
    q = normal(621, (images * queries, qs))
    k = normal(622, (images * keys, kv * d))
    v = normal(623, (images * keys, kv * d))
    tq, tk, tv = dev(torch, q), dev(torch, k), dev(torch, v)
    out = torch.zeros((images * queries, heads * d), device="cuda")
    fa.attend_full(heads, kv, d, images, queries, keys, fa.Operand(tq, qs), fa.Operand(tk, kv * d),
                   fa.Operand(tv, kv * d), out)
    side = torch.cuda.Stream()
    torch.cuda.synchronize()
    out2 = torch.zeros_like(out)
    fa.attend_full(heads, kv, d, images, queries, keys, fa.Operand(tq, qs), fa.Operand(tk, kv * d),
                   fa.Operand(tv, kv * d), out2, stream=side)
    torch.cuda.synchronize()
    fa.device_status()
    want = oracle.attend_call(heads, kv, d, images, queries, keys, q, qs, 0, k, kv * d, 0, v,
                              kv * d, 0)
    got = out.cpu().numpy()
    print(compare(f"split-KV full mask {case}", got, want))
    assert max_abs(got, want) <= TOL_F32
    assert torch.equal(out, out2)


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("mask_name", ["causal", "window", "full", "groups"])
def test_prefill_on_tensor_cores_every_mask(torch, dtype, head_dim, mask_name):
    """Spans of >= 64 rows run on the tcgen05 kernel: every mask, a cache already holding keys
    (first > 0), GQA 12/4, a row count that is not a multiple of the 128-row tile. head_dim 256
    runs on the tensor cores over a bf16 cache (one query tile per CTA, 64-key tiles), on the
    split-KV kernel over an f32 cache."""
    shape = fa.Shape(1, 12, 4, head_dim)
    first, rows = 150, 200
    mask = {"causal": fa.Mask.causal(), "window": fa.Mask.window_of(97), "full": fa.Mask.full(),
            "groups": fa.Mask.groups(180, [200, 260, 300, 350])}[mask_name]
    pair = Pair(shape, 400, dtype, filled=first, seed=7)
    qkv = normal(71, (rows, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), head_dim, range(first, first + rows))
    span = fa.Span(rows, first, mask)
    out = torch.zeros((rows, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    fa.device_status()
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    print(compare(f"tc d{head_dim} {mask_name} {'f32' if dtype == fa.F32 else 'bf16'}", got, want))
    tol = TOL_F32 if dtype == fa.F32 else TOL_BF16
    err = np.abs(got - want).reshape(rows, shape.heads, head_dim).max(axis=2)
    bad = np.argwhere(err > tol)
    assert len(bad) == 0, (f"{len(bad)} (row, head) pairs over {tol}: first {bad[:12].tolist()}, "
                           f"rows {sorted(set(bad[:, 0].tolist()))[:40]}, heads {sorted(set(bad[:, 1].tolist()))}")
    assert parity_ok(got, want, dtype == fa.BF16)


@pytest.mark.parametrize("first,rows", [(0, 1000), (37, 700)])
def test_causal_prefill_over_several_pairs(torch, first, rows):
    """A causal prefill of several 256-row pairs over a bf16 cache, GQA 8/2, ragged last tile:
    its units run heaviest pair first across the heads (the K/V fits in L2). Every row of
    every head against the oracle."""
    shape = fa.Shape(1, 8, 2, 128)
    pair = Pair(shape, first + rows + 8, fa.BF16, filled=first, seed=9)
    qkv = normal(91, (rows, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 128, range(first, first + rows))
    span = fa.Span(rows, first, fa.Mask.causal())
    out = torch.zeros((rows, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    fa.device_status()
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    print(compare(f"causal prefill {rows} rows from {first}, bf16", got, want))
    assert parity_ok(got, want, True)


@pytest.mark.parametrize("rows", [300, 1030])
def test_attend_over_f32_queries_equals_attention_on_a_bf16_cache(torch, rows):
    """The reference's plugin split (keep, then attend over f32 queries) on a bf16 cache: fa_attend
    converts the rotated f32 queries to bf16 operand rows before the tensor-core attention, and
    gives fa_attention's output bit for bit (there the RoPE kernel writes the bf16 queries):
    both round the same rotated values to nearest."""
    shape = fa.Shape(1, 8, 2, 128)
    cache = fa.KvCache(shape, rows, fa.BF16)
    qkv = dev(torch, normal(95, (rows, shape.qkv)))
    angles = dev(torch, fa.rotary_angles(fa.Rotation(base=1e6), 128, range(rows)))
    span = fa.Span(rows, 0, fa.Mask.causal())
    whole = torch.zeros((rows, shape.width), device="cuda")
    cache.attention(0, span, qkv, whole, angles, fa.ROPE_HALF)
    q = torch.zeros((rows, shape.width), device="cuda")
    cache.attention_input(0, span, qkv, angles, fa.ROPE_HALF, q_out=q)
    split = torch.zeros_like(whole)
    cache.attend(0, span, q, split)
    fa.device_status()
    assert torch.equal(whole, split)


def test_tensor_core_and_split_kv_paths_agree(torch):
    """The same rows through fa_attend on the tensor cores (64 rows) and through the split-KV
    kernel (one row at a time) give the same attention within the f32 bar."""
    shape = fa.Shape(1, 14, 2, 64)
    pair = Pair(shape, 4096, filled=4000, seed=8)
    q = torch.randn((64, shape.width), device="cuda")
    span = fa.Span(64, 3900, fa.Mask.causal())
    tc = torch.zeros((64, shape.width), device="cuda")
    pair.gpu.attend(0, span, q, tc)
    rows = torch.zeros_like(tc)
    for r in range(64):
        pair.gpu.attend(0, fa.Span(1, 3900 + r, fa.Mask.causal()), q[r:r + 1], rows[r:r + 1])
    err = float((tc - rows).abs().max())
    print(f"tensor cores vs split-KV: max abs {err:.2e}")
    assert err <= TOL_F32


@pytest.mark.parametrize("head_dim,frames", [(32, 7), (64, 150), (128, 257), (256, 33)])
def test_conformer_relative_position_attention(torch, head_dim, frames):
    """conformer::attention::attend: Transformer-XL scores over the projected relative-position
    table, on the conformer's packed qkv rows (queries, keys, values of `hidden` each)."""
    heads = 4
    hidden = heads * head_dim
    qkv = normal(801, (frames, 3 * hidden))
    positions = normal(802, (2 * frames - 1, hidden))
    bias_u = 0.1 * normal(803, (hidden,))
    bias_v = 0.1 * normal(804, (hidden,))
    t = dev(torch, qkv)
    out = torch.zeros((frames, hidden), device="cuda")
    fa.attend_relpos(heads, head_dim, frames, fa.Operand(t, 3 * hidden, 0),
                     fa.Operand(t, 3 * hidden, hidden), fa.Operand(t, 3 * hidden, 2 * hidden),
                     dev(torch, positions), dev(torch, bias_u), dev(torch, bias_v), out)
    fa.device_status()
    want = oracle.relpos_attend(heads, head_dim, frames, qkv, positions, bias_u, bias_v)
    got = out.cpu().numpy()
    print(compare(f"relpos d{head_dim} frames {frames}", got, want))
    assert max_abs(got, want) <= TOL_F32
