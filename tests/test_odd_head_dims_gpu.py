"""Head dims between the powers of two: the reference's Kronos stack (Qwen2 layers of 16 heads of
52, models/kronos/model/src/model.rs:27-39) and Iris' DiT adapter (32 heads of 80,
models/iris/model/src/model.rs:46-54), and the other whole numbers of 16-byte vectors up to 256.
They run on the split-KV kernel of the next wider head_dim with the lanes past the head idle
(the rows stream and sit in shared memory head_dim apart); every output against the oracle at
the f32 bar (the split-KV kernel computes in f32 over f32 or bf16 rows)."""
import ctypes as C

import numpy as np
import pytest

import fusor_attn as fa
import oracle
from gpu_util import TOL_F32, Pair, compare, max_abs, normal, round_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


@pytest.mark.parametrize("rows,first", [(1, 900), (37, 0), (200, 300)])
def test_kronos_stack_attention(torch, rows, first):
    """Kronos' attention layer (16/16 heads of 52, RoPE base 1e4, f32): a decode, a prefill from
    the cache's start and a prefill over a filled cache."""
    shape = fa.Shape(1, 16, 16, 52)
    pair = Pair(shape, first + rows + 5, fa.F32, filled=first, seed=5201)
    qkv = normal(5202, (rows, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e4), 52, range(first, first + rows))
    span = fa.Span(rows, first, fa.Mask.causal())
    out = torch.zeros((rows, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    fa.device_status()
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    got = out.cpu().numpy()
    print(compare(f"kronos d52 rows {rows} from {first}", got, want))
    assert max_abs(got, want) <= TOL_F32


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
@pytest.mark.parametrize("head_dim", [40, 48, 80, 96, 112, 160, 200, 240])
def test_decode_batch_and_window(torch, dtype, head_dim):
    """A batch of decodes and a span under a window that wraps the ring, GQA 8/2."""
    if dtype == fa.BF16 and head_dim % 8:
        pytest.skip("bf16 rows need whole 8-element vectors")
    shape = fa.Shape(1, 8, 2, head_dim)
    lengths = [333, 1500, 70]
    pairs = [Pair(shape, n + 1, dtype, filled=n, seed=5210 + i) for i, n in enumerate(lengths)]
    qkv = normal(5214, (len(pairs), shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), head_dim, lengths)
    spans = [fa.Span(1, n, fa.Mask.causal()) for n in lengths]
    out = torch.zeros((len(pairs), shape.width), device="cuda")
    fa.attention_batch([p.gpu for p in pairs], spans, 0, dev(torch, qkv), out, dev(torch, angles),
                       fa.ROPE_HALF)
    fa.device_status()
    got = out.cpu().numpy()
    for i, (p, span) in enumerate(zip(pairs, spans)):
        want = p.oracle_attention(0, span, qkv[i:i + 1], angles[i:i + 1], fa.ROPE_HALF)
        assert max_abs(got[i:i + 1], want) <= TOL_F32, compare(f"d{head_dim} batch {i}", got[i:i + 1], want)
    # a window over a ring smaller than the sequence, several rows
    pair = Pair(shape, 900, dtype, filled=900, seed=5220)
    span = fa.Span(6, 2000, fa.Mask.window_of(700))
    qkv = normal(5221, (6, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), head_dim, range(2000, 2006))
    out = torch.zeros((6, shape.width), device="cuda")
    pair.gpu.attention(0, span, dev(torch, qkv), out, dev(torch, angles), fa.ROPE_HALF)
    fa.device_status()
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    assert max_abs(out.cpu().numpy(), want) <= TOL_F32, compare(f"d{head_dim} window", out.cpu().numpy(), want)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_iris_adapter_full_mask(torch, dtype):
    """Iris' DiT adapter attention (dit::Within, full mask): 32 heads of 80 over two images of
    300 tokens (the adapter's text rows), operands in one qkv row of stride 3 x hidden."""
    heads, d, images, n = 32, 80, 2, 300
    hidden = heads * d
    qkv = normal(5230, (images * n, 3 * hidden))
    if dtype == "bf16":
        qkv = round_bf16(qkv)
    t = dev(torch, qkv)
    if dtype == "bf16":
        t = t.to(torch.bfloat16)
    out = torch.zeros((images * n, hidden), device="cuda")
    stride = 3 * hidden
    fa.attend_full(heads, heads, d, images, n, n, fa.Operand(t, stride, 0),
                   fa.Operand(t, stride, hidden), fa.Operand(t, stride, 2 * hidden), out)
    fa.device_status()
    want = oracle.attend_call(heads, heads, d, images, n, n, qkv, stride, 0, qkv, stride, hidden,
                              qkv, stride, 2 * hidden, threads=8)
    got = out.cpu().numpy()
    print(compare(f"iris d80 full {dtype}", got, want))
    assert max_abs(got, want) <= TOL_F32


def test_key_range_partials_and_static_entry_at_head_dim_80(torch):
    """The KV-range shards' partials ([heads][80 + 2]) merged by log-sum-exp equal the whole
    decode, and fa_attend_static (its scratch sized by the wider kernel) agrees with fa_attend."""
    shape = fa.Shape(1, 8, 4, 80)
    n = 5000
    pair = Pair(shape, n + 1, fa.F32, filled=n, seed=5240)
    qkv = normal(5241, (1, shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), 80, [n])
    span = fa.Span(1, n, fa.Mask.causal())
    q = torch.zeros((1, shape.width), device="cuda")
    pair.gpu.attention_input(0, span, dev(torch, qkv), dev(torch, angles), fa.ROPE_HALF, q_out=q)
    whole = torch.zeros((1, shape.width), device="cuda")
    pair.gpu.attend(0, span, q, whole)
    bounds = [0, 1200, 3333, n + 1]
    parts = torch.zeros((3, 8, 82), device="cuda")
    for s in range(3):
        pair.gpu.attend_partial(0, q, bounds[s], bounds[s + 1], parts[s])
    merged = torch.zeros((8, 80), device="cuda")
    fa.merge_partials(parts, merged)
    static = torch.full((1, shape.width), float("nan"), device="cuda")
    sp = span.c()
    rc = fa.lib().fa_attend_static(pair.gpu.handle, 0, C.byref(sp), C.c_void_p(q.data_ptr()),
                                   q.stride(0), C.c_void_p(static.data_ptr()), static.stride(0),
                                   fa._stream())
    assert rc == fa.OK, fa.lib().fa_last_error()
    fa.device_status()
    want = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    for name, got in (("whole", whole), ("merged", merged.reshape(1, -1)), ("static", static)):
        g = got.cpu().numpy()
        assert max_abs(g, want) <= TOL_F32, compare(f"d80 {name}", g, want)
