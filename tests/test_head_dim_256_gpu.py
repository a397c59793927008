"""head_dim 256 on the tensor cores: the shape of the reference's flagship text model's attention
layers (Qwen3.5's LANGUAGE stack, models/qwen3-5/model/src/model.rs:60-75: 8 query heads over 2
key/value heads of 256, a quarter of each head rotated by interleaved multimodal RoPE of base
1e7 with sections [11, 11, 10], a head RMSNorm and an elementwise sigmoid gate), and of the DiT
and image models with 256-wide heads. A bf16 call or cache runs the one-query-tile tcgen05
kernel with 64-key tiles (two query tiles of 256 columns do not fit in TMEM); an f32 one the
split-KV kernel. Every output against the oracle."""
import numpy as np
import pytest

import fusor_attn as fa
import oracle
from gpu_util import Pair, compare, normal, parity_ok, round_bf16

pytestmark = pytest.mark.gpu

D = 256


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("heads,kv,images,queries,keys", [(4, 2, 2, 200, 300), (2, 2, 1, 128, 64),
                                                          (6, 3, 1, 1000, 777)])
def test_full_mask_bf16_head_dim_256(torch, out_dtype, heads, kv, images, queries, keys):
    """blocks::attention::attend at head_dim 256: GQA, several images, query counts off the
    128-row tile and key counts off the 64-key tile."""
    q = round_bf16(normal(2561, (images * queries, heads * D)))
    k = round_bf16(normal(2562, (images * keys, kv * D)))
    v = round_bf16(normal(2563, (images * keys, kv * D)))
    tq, tk, tv = (dev(torch, x).to(torch.bfloat16) for x in (q, k, v))
    odt = torch.float32 if out_dtype == "f32" else torch.bfloat16
    out = torch.zeros((images * queries, heads * D), device="cuda", dtype=odt)
    fa.attend_full(heads, kv, D, images, queries, keys, fa.Operand(tq, heads * D),
                   fa.Operand(tk, kv * D), fa.Operand(tv, kv * D), out)
    fa.device_status()
    want = oracle.attend_call(heads, kv, D, images, queries, keys, q, heads * D, 0, k, kv * D, 0,
                              v, kv * D, 0, threads=8)
    got = out.float().cpu().numpy()
    print(compare(f"full mask d256 {heads}/{kv} x{images} {queries}x{keys} {out_dtype}", got, want))
    assert parity_ok(got, want, True)


def qwen35_angles(positions):
    """Qwen3.5's rotary table over its 64 rotated dimensions, on both sides: the library's and
    the oracle's, which must agree bit for bit."""
    rot = fa.Rotation(fa.ROT_MULTIMODAL_INTERLEAVED, (11, 11, 10), 1e7)
    ours = fa.rotary_angles(rot, 64, positions)
    theirs = oracle.angles_table(oracle.ROT_MM_INTERLEAVED, 1e7, 64,
                                 [(p.temporal, p.height, p.width) for p in positions],
                                 params=(11, 11, 10))
    assert (ours.view(np.uint32) == theirs.view(np.uint32)).all()
    return ours


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
@pytest.mark.parametrize("rows,first", [(1, 5000), (200, 0), (300, 700), (7, 90)])
def test_qwen35_gated_attention(torch, dtype, rows, first):
    """The gated attention layer of Qwen3.5: decode (one row over 5000 keys), prefills from the
    cache's start and over a filled cache (the tensor cores over a bf16 cache), and a short span;
    text positions with a run of image tokens (their own height and width positions)."""
    shape = fa.Shape(1, 8, 2, D)
    pair = Pair(shape, first + rows + 4, dtype, filled=first, seed=2570)
    width = (2 * shape.heads + 2 * shape.kv_heads) * D  # query, gate, key and value heads
    qkv = normal(2571, (rows, width))
    qn = 1.0 + 0.2 * normal(2572, (D,))
    kn = 1.0 + 0.2 * normal(2573, (D,))
    positions = []
    for r in range(first, first + rows):
        if first <= r < first + 3 or r % 11 != 4:
            positions.append(fa.Position.uniform(r))
        else:  # an image token: its own row and column
            positions.append(fa.Position(r, r + (r % 5), r + (r % 7)))
    angles = qwen35_angles(positions)
    span = fa.Span(rows, first, fa.Mask.causal())
    out = torch.zeros((rows, shape.width), device="cuda")
    pair.gpu.gated_attention(0, span, dev(torch, qkv), out, fa.GATE_ELEMENTWISE, 64,
                             dev(torch, angles), norm=(dev(torch, qn), dev(torch, kn), 1e-6))
    fa.device_status()
    q = qkv.copy()
    pair.cpu.gated_input(0, rows, first, fa.GATE_ELEMENTWISE, 64, angles, q, width, qn, kn, 1e-6)
    pair.keep_rounding(0, first, rows)
    attended = pair.cpu.attend(0, rows, first, oracle.Mask.causal(), q, width, threads=8)
    want = oracle.gate(rows, shape.heads, shape.kv_heads, D, fa.GATE_ELEMENTWISE, q, attended)
    got = out.cpu().numpy()
    print(compare(f"qwen3.5 gated d256 rows {rows} from {first} "
                  f"{'f32' if dtype == fa.F32 else 'bf16'}", got, want))
    # a bf16 cache computes in bf16 on the tensor cores, prefill and decode rows alike
    assert parity_ok(got, want, dtype == fa.BF16)


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
def test_decode_batch_head_dim_256(torch, dtype):
    """A batch of one-row decodes at head_dim 256 against the oracle: over an f32 cache the
    split-KV kernel (f32 arithmetic), over a bf16 cache the tensor-core decode (bf16 operands)."""
    shape = fa.Shape(1, 8, 2, D)
    lengths = [700, 3000, 64, 5100]
    pairs = [Pair(shape, n + 1, dtype, filled=n, seed=2580 + i) for i, n in enumerate(lengths)]
    qkv = normal(2585, (len(pairs), shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), D, lengths)
    spans = [fa.Span(1, n, fa.Mask.causal()) for n in lengths]
    out = torch.zeros((len(pairs), shape.width), device="cuda")
    fa.attention_batch([p.gpu for p in pairs], spans, 0, dev(torch, qkv), out, dev(torch, angles),
                       fa.ROPE_HALF)
    fa.device_status()
    got = out.cpu().numpy()
    for i, (p, span) in enumerate(zip(pairs, spans)):
        want = p.oracle_attention(0, span, qkv[i:i + 1], angles[i:i + 1], fa.ROPE_HALF)
        assert parity_ok(got[i:i + 1], want, dtype == fa.BF16), \
            compare(f"d256 decode {i}", got[i:i + 1], want)
