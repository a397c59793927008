"""Parity at the sizes `bench.py` times, on the bench's own seeded inputs.

The other parity tests check each configuration on its shapes at sizes the oracle finishes in a
moment; here the launches that set the measured numbers are checked as they run:

- C3: all 64 sequences of the batched decode (cache lengths U[512, 8192] seed 301, each
  sequence's keys and values from torch's generator seeded 1000 + its index, the qkv rows from
  seed 999), f32 and bf16 caches; and the batch split over 2, 4 and 8 ranks' shares
  (`shard_sequences`), each share one launch, against the whole batch.
- C4: the whole 131073-key decode (131072 cached positions and the new row from one generator
  seeded 7) against the oracle's decode of all of it.
- C5: the 32760-token full-mask call (bf16 qkv from seed 5): the first and last 256-row pair of
  every head, and rows of every unit the last wave splits into key pieces, against the oracle's
  f32 attention over the same bf16 inputs; and the row shards of 2, 4 and 8 ranks
  (`query_row_shards`), each its own call, against the whole call.

Bars: max abs 2e-3 with f32 I/O; the bf16-compute bar for bf16 caches and the bf16 full mask.
"""
import numpy as np
import pytest

import fusor_attn as fa
import oracle
from fusor_attn.shard import query_row_shards, shard_sequences
from gpu_util import TOL_F32, compare, max_abs, parity_ok, round_bf16

pytestmark = pytest.mark.gpu

HEADS, KV, D = 32, 8, 128


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def threads():
    import os
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return os.cpu_count() or 1


def c3_lengths():
    return [int(n) for n in np.random.default_rng(301).integers(512, 8193, size=64)]


def c3_batch(torch, dtype):
    """The bench's C3 batch: caches, spans and qkv rows."""
    shape = fa.Shape(1, HEADS, KV, D)
    tdt = torch.float32 if dtype == fa.F32 else torch.bfloat16
    caches = []
    for i, n in enumerate(c3_lengths()):
        gen = torch.Generator("cuda").manual_seed(1000 + i)
        c = fa.KvCache(shape, n + 1, dtype)
        k = torch.randn((1, KV, n, D), device="cuda", generator=gen).to(tdt)
        v = torch.randn((1, KV, n, D), device="cuda", generator=gen).to(tdt)
        c.put_rows(k, v)
        caches.append(c)
    gen = torch.Generator("cuda").manual_seed(999)
    qkv = torch.randn((64, shape.qkv), device="cuda", generator=gen)
    spans = [fa.Span(1, n, fa.Mask.causal()) for n in c3_lengths()]
    angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), D, c3_lengths())).cuda()
    return shape, caches, spans, qkv, angles


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
def test_c3_every_sequence_of_the_timed_batch(torch, dtype):
    shape, caches, spans, qkv, angles = c3_batch(torch, dtype)
    out = torch.zeros((64, shape.width), device="cuda")
    fa.Batch(caches, spans).attention(0, qkv, out, angles, fa.ROPE_HALF)
    fa.device_status()
    got = out.cpu().numpy()
    qkv_h, angles_h = qkv.cpu().numpy(), angles.cpu().numpy()
    worst = 0.0
    for i, (c, n) in enumerate(zip(caches, c3_lengths())):
        k, v = c.copy_rows(n)
        oc = oracle.Cache(1, HEADS, KV, D, n + 1)
        oc.keys[:, :, :n] = k.float().cpu().numpy()
        oc.values[:, :, :n] = v.float().cpu().numpy()
        q = qkv_h[i:i + 1].copy()
        oc.attention_input(0, 1, n, fa.ROPE_HALF, angles_h[i:i + 1], q, q.shape[1])
        if dtype == fa.BF16:
            oc.keys[0, :, n] = round_bf16(oc.keys[0, :, n])
            oc.values[0, :, n] = round_bf16(oc.values[0, :, n])
        want = oc.attend(0, 1, n, oracle.Mask.causal(), q, q.shape[1], threads=threads())
        assert parity_ok(got[i:i + 1], want, dtype == fa.BF16), compare(
            f"C3 sequence {i} ({n} keys)", got[i:i + 1], want)
        worst = max(worst, max_abs(got[i:i + 1], want))
    print(f"C3 {'f32' if dtype == fa.F32 else 'bf16'}: 64 sequences, max abs {worst:.2e}")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_c3_rank_shares_equal_the_whole_batch(torch, world):
    """Each rank's share of the sequences as its own launch (what a rank of the multi-GPU run
    computes) gives the whole batch's rows, within f32 rounding (the shares chunk the keys
    differently)."""
    shape, caches, spans, qkv, angles = c3_batch(torch, fa.F32)
    whole = torch.zeros((64, shape.width), device="cuda")
    fa.Batch(caches, spans).attention(0, qkv, whole, angles, fa.ROPE_HALF)
    parts = torch.zeros_like(whole)
    for mine in shard_sequences(c3_lengths(), world):
        idx = torch.tensor(mine, device="cuda")
        out = torch.zeros((len(mine), shape.width), device="cuda")
        fa.Batch([caches[i] for i in mine], [spans[i] for i in mine]).attention(
            0, qkv[idx].contiguous(), out, angles[idx].contiguous(), fa.ROPE_HALF)
        parts[idx] = out
    fa.device_status()
    err = float((parts - whole).abs().max())
    print(f"C3 over {world} shares: max abs {err:.2e} against the whole batch")
    assert err <= 1e-5


def test_c4_whole_context_against_the_oracle(torch):
    shape = fa.Shape(1, 16, 8, D)
    position = 131072
    gen = torch.Generator("cuda").manual_seed(7)
    k = torch.randn((1, 8, position, D), device="cuda", generator=gen)
    v = torch.randn((1, 8, position, D), device="cuda", generator=gen)
    qkv = torch.randn((1, shape.qkv), device="cuda", generator=gen)
    cache = fa.KvCache(shape, position + 1)
    cache.put_rows(k, v)
    angles = fa.rotary_angles(fa.Rotation(base=1e6), D, [position])
    out = torch.zeros((1, shape.width), device="cuda")
    cache.attention(0, fa.Span(1, position, fa.Mask.causal()), qkv, out,
                    torch.from_numpy(angles).cuda(), fa.ROPE_HALF)
    fa.device_status()
    oc = oracle.Cache(1, 16, 8, D, position + 1)
    oc.keys[:, :, :position] = k.cpu().numpy()
    oc.values[:, :, :position] = v.cpu().numpy()
    del k, v
    q = qkv.cpu().numpy().copy()
    oc.attention_input(0, 1, position, fa.ROPE_HALF, angles, q, q.shape[1])
    want = oc.attend(0, 1, position, oracle.Mask.causal(), q, q.shape[1], threads=threads())
    got = out.cpu().numpy()
    print(compare("C4 131073 keys", got, want))
    assert max_abs(got, want) <= TOL_F32
    # the kept row is the oracle's, bit for bit
    kk, vv = cache.copy_rows()
    assert (kk[0, :, position].cpu().numpy().view(np.uint32)
            == oc.keys[0, :, position].view(np.uint32)).all()
    assert (vv[0, :, position].cpu().numpy().view(np.uint32)
            == oc.values[0, :, position].view(np.uint32)).all()


C5_HEADS, C5_N = 12, 32760


def c5_inputs(torch):
    hidden = C5_HEADS * D
    gen = torch.Generator("cuda").manual_seed(5)
    qkv = torch.randn((C5_N, 3 * hidden), device="cuda", generator=gen).to(torch.bfloat16)
    return qkv, hidden, 3 * hidden


def c5_call(torch, qkv, hidden, stride, lo, hi, out):
    fa.attend_full(C5_HEADS, C5_HEADS, D, 1, hi - lo, C5_N, fa.Operand(qkv, stride, lo * stride),
                   fa.Operand(qkv, stride, hidden), fa.Operand(qkv, stride, 2 * hidden), out[lo:hi])


def test_c5_whole_call_against_the_oracle(torch):
    """The first and last 256-row pair of every head, and four rows (the first and last of each
    128-row tile) of every unit after the tenth wave of 148 units (the last 56 units of head 11,
    which the 1-GPU schedule cuts into key pieces), against the oracle."""
    qkv, hidden, stride = c5_inputs(torch)
    out = torch.zeros((C5_N, hidden), device="cuda", dtype=torch.bfloat16)
    c5_call(torch, qkv, hidden, stride, 0, C5_N, out)
    fa.device_status()
    host = qkv.float().cpu().numpy()
    got = out.float().cpu().numpy()
    want = np.zeros((C5_N, hidden), np.float32)
    edges = [(0, 256), (C5_N - 256, C5_N)]
    for qb, qe in edges:
        oracle.attend_call(C5_HEADS, C5_HEADS, D, 1, C5_N, C5_N, host, stride, 0, host, stride,
                           hidden, host, stride, 2 * hidden, query_range=(qb, qe),
                           threads=threads(), out=want)
    rows = np.r_[0:256, C5_N - 256:C5_N]
    print(compare("C5 edge pairs, every head", got[rows], want[rows]))
    assert parity_ok(got[rows], want[rows], True)
    pairs = (C5_N + 255) // 256
    units = C5_HEADS * pairs
    tail_units = range(units // 148 * 148, units)  # head-major: the last ones are head 11's
    split_rows = []
    for u in tail_units:
        head, pair = divmod(u, pairs)
        assert head == C5_HEADS - 1
        for r in (0, 127, 128, 255):
            row = pair * 256 + r
            if row < C5_N:
                split_rows.append(row)
    split_rows = sorted(set(split_rows))
    want11 = np.zeros((C5_N, hidden), np.float32)
    for row in split_rows:
        oracle.attend_call(C5_HEADS, C5_HEADS, D, 1, C5_N, C5_N, host, stride, 0, host, stride,
                           hidden, host, stride, 2 * hidden, head_range=(11, 12),
                           query_range=(row, row + 1), threads=threads(), out=want11)
    cols = slice(11 * D, 12 * D)
    print(compare(f"C5 head 11, {len(split_rows)} rows of the split units",
                  got[split_rows, cols], want11[split_rows, cols]))
    assert parity_ok(got[split_rows, cols], want11[split_rows, cols], True)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_c5_row_shares_equal_the_whole_call(torch, world):
    """Each rank's query rows as its own call (the multi-GPU run's per-rank call) give the whole
    call's rows within the bf16-compute bars: the shares' schedules cut other units into key
    pieces, whose probabilities are rounded to bf16 against their own running maxima, so the two
    differ at the level each differs from the f32 oracle (about 2e-4 here), not bit for bit."""
    qkv, hidden, stride = c5_inputs(torch)
    whole = torch.zeros((C5_N, hidden), device="cuda", dtype=torch.bfloat16)
    c5_call(torch, qkv, hidden, stride, 0, C5_N, whole)
    parts = torch.zeros_like(whole)
    for lo, hi in query_row_shards(C5_N, world):
        if hi > lo:
            c5_call(torch, qkv, hidden, stride, lo, hi, parts)
    fa.device_status()
    a, b = parts.float().cpu().numpy(), whole.float().cpu().numpy()
    print(compare(f"C5 over {world} shares against the whole call", a, b))
    assert parity_ok(a, b, True)


def test_f32_cache_long_prefill_on_tf32_against_f32_cores(torch):
    """The bench's f32-cache prefill (8192 rows from position 0, 32/8 heads x 128, causal) on the
    tf32 tensor-core kernel, every row against the same attention on the split-KV kernel's f32
    arithmetic (queries given with a row stride the tensor path's TMA cannot take), which the
    oracle matches within 1e-6; and sampled rows against the oracle itself."""
    rows, heads, kv = 8192, 32, 8
    shape = fa.Shape(1, heads, kv, D)
    cache = fa.KvCache(shape, rows)
    gen = torch.Generator("cuda").manual_seed(13)
    qkv = torch.randn((rows, shape.qkv), device="cuda", generator=gen)
    angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), D, range(rows))).cuda()
    span = fa.Span(rows, 0, fa.Mask.causal())
    q = torch.zeros((rows, shape.width), device="cuda")
    cache.attention_input(0, span, qkv, angles, fa.ROPE_HALF, q_out=q)
    tc = torch.zeros((rows, shape.width), device="cuda")
    cache.attend(0, span, q, tc)
    q_odd = torch.zeros((rows, shape.width + 1), device="cuda")
    q_odd[:, :shape.width] = q
    cores = torch.zeros_like(tc)
    cache.attend(0, span, q_odd[:, :shape.width], cores)
    fa.device_status()
    err = (tc - cores).abs()
    worst_rows = err.max(dim=1).values
    print(f"f32 prefill 8192 rows, tf32 tensor cores vs f32 cores: max abs {float(err.max()):.2e}, "
          f"rows over 1e-3: {int((worst_rows > 1e-3).sum())}, worst row {int(worst_rows.argmax())}")
    assert float(err.max()) <= TOL_F32
    # the f32 cores against the oracle on a few rows, the worst one among them
    k, v = cache.copy_rows(rows)
    oc = oracle.Cache(1, heads, kv, D, rows)
    oc.keys[:] = k.cpu().numpy()
    oc.values[:] = v.cpu().numpy()
    qh = q.cpu().numpy()
    for r in sorted({0, 1, 7, 100, rows - 1, int(worst_rows.argmax())}):
        want = oc.attend(0, 1, r, oracle.Mask.causal(), qh[r:r + 1], qh.shape[1], threads=threads())
        assert max_abs(cores.cpu().numpy()[r:r + 1], want) <= 1e-5
        assert max_abs(tc.cpu().numpy()[r:r + 1], want) <= TOL_F32
