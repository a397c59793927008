"""Parity of the steps either side of the attention that the DiT and hybrid blocks add, through
the C ABI, against the oracle: the DiT query/key prologue (whole-row or per-head RMSNorm, 3-D
RoPE; wan_dit/block.rs:109-140, mmdit/pass.rs:162-192) alone and chained into the full-mask
attention, and the hybrid blocks' gated attention (hybrid/attention.rs:153-295) on the decode
and the tensor-core prefill paths."""
import numpy as np
import pytest

import fusor_attn as fa
import oracle
from gpu_util import Pair, compare, max_abs, normal, parity_ok, round_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def video_positions(frames, rows, cols):
    """Patching::position (crates/blocks/src/video.rs:48-55) of every token."""
    return [fa.Position(t // (rows * cols), t // cols % rows, t % cols)
            for t in range(frames * rows * cols)]


def wan_sections(head_dim):
    """Wan's split of a head's d/2 rotary pairs over frames, rows and columns."""
    half = head_dim // 2
    hw = head_dim // 6
    return (half - 2 * hw, hw, hw)


def bf16_close(got, want):
    """got (bf16 values as f32) is want rounded to bf16, give or take one bf16 step where want
    lies within rounding noise of a rounding boundary."""
    return np.abs(got - round_bf16(want)) <= np.abs(want) * 2.0 ** -7 + 1e-30


# ---- the DiT query/key prologue ---------------------------------------------------------------

@pytest.mark.parametrize("case", ["wan_bf16", "wan_f32", "wan_in_place", "mmdit_head_half",
                                  "unaligned", "d128_head_half", "d128_20_heads"])
def test_prologue_matches_the_oracle(torch, case):
    """Head_dim 128 with at most 16 heads and aligned rows runs the register-resident kernel
    (the wan cases, d128_head_half); the rest the general one."""
    heads, d = {"d128_head_half": (5, 128), "d128_20_heads": (20, 128)}.get(
        case, (3, 128) if case.startswith("wan") else (4, 64))
    frames, rows, cols = 3, 5, 7
    positions = video_positions(frames, rows, cols)
    tokens, width = len(positions), heads * d
    head_half = case in ("mmdit_head_half", "d128_head_half")
    norm = fa.NORM_HEAD if head_half else fa.NORM_ROW
    rope = fa.ROPE_HALF if head_half else fa.ROPE_INTERLEAVED
    rotated = 70 if head_half else tokens
    stride = 3 * width + (1 if case == "unaligned" else 0)
    qkv = normal(901, (tokens, stride))
    wn = width if norm == fa.NORM_ROW else d
    qn = 1.0 + 0.2 * normal(902, (wn,))
    kn = 1.0 + 0.2 * normal(903, (wn,))
    angles = fa.rotary_angles(fa.Rotation(fa.ROT_AXES, wan_sections(d), 1e4), d, positions)
    t = dev(torch, qkv)
    if case == "wan_in_place":
        out = t
    elif case == "wan_bf16":
        out = torch.zeros((tokens, 3 * width), device="cuda", dtype=torch.bfloat16)
    else:
        out = torch.zeros((tokens, 3 * width + (3 if case == "unaligned" else 0)), device="cuda")
    fa.normalize_and_rotate(heads, d, t, out, norm, dev(torch, qn), dev(torch, kn), 1e-6,
                            dev(torch, angles), rope, rotated)
    fa.device_status()
    want = oracle.qk_prologue(tokens, heads, d, norm, rope, rotated, angles, qn, kn, 1e-6, qkv)
    got = out.float().cpu().numpy()[:, :3 * width]
    want = want[:, :3 * width]
    print(compare(f"prologue {case}", got, want))
    if case == "wan_bf16":
        assert bf16_close(got, want).all()
        assert (got[:, 2 * width:] == round_bf16(want[:, 2 * width:])).all()
    else:
        assert max_abs(got[:, :2 * width], want[:, :2 * width]) <= 1e-5
        assert (got[:, 2 * width:] == want[:, 2 * width:]).all()
    if case == "wan_in_place":
        # what is past the rows' queries, keys and values stays as it was
        assert (out.cpu().numpy()[:, 3 * width:] == qkv[:, 3 * width:]).all()


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_wan_self_attention_prologue_then_full_mask(torch, dtype):
    """Wan's self-attention phase (wan_dit/block.rs:63-107): the prologue into bf16 operand rows
    (or in place in f32), then the full-mask attention over them, against the oracle's f32
    prologue and attention (on the same bf16-rounded operands for bf16)."""
    heads, d = 2, 128
    positions = video_positions(2, 6, 10)
    tokens, width = len(positions), heads * d
    qkv = normal(911, (tokens, 3 * width))
    qn = 1.0 + 0.2 * normal(912, (width,))
    kn = 1.0 + 0.2 * normal(913, (width,))
    angles = fa.rotary_angles(fa.Rotation(fa.ROT_AXES, wan_sections(d), 1e4), d, positions)
    t = dev(torch, qkv)
    ops = t if dtype == "f32" else torch.zeros((tokens, 3 * width), device="cuda",
                                               dtype=torch.bfloat16)
    fa.normalize_and_rotate(heads, d, t, ops, fa.NORM_ROW, dev(torch, qn), dev(torch, kn), 1e-6,
                            dev(torch, angles), fa.ROPE_INTERLEAVED)
    out = torch.zeros((tokens, width), device="cuda")
    s = 3 * width
    fa.attend_full(heads, heads, d, 1, tokens, tokens, fa.Operand(ops, s, 0),
                   fa.Operand(ops, s, width), fa.Operand(ops, s, 2 * width), out)
    fa.device_status()
    prepared = oracle.qk_prologue(tokens, heads, d, fa.NORM_ROW, fa.ROPE_INTERLEAVED, tokens,
                                  angles, qn, kn, 1e-6, qkv)
    if dtype == "bf16":
        # the oracle attends over the operands the GPU attends over
        prepared = ops.float().cpu().numpy()
    want = oracle.attend_call(heads, heads, d, 1, tokens, tokens, prepared, s, 0, prepared, s,
                              width, prepared, s, 2 * width)
    got = out.cpu().numpy()
    print(compare(f"wan self-attention {dtype}", got, want))
    assert parity_ok(got, want, dtype == "bf16")


# ---- the hybrid blocks' gated attention -------------------------------------------------------

def gated_width(shape, gate):
    gate_heads = shape.heads if gate == fa.GATE_ELEMENTWISE else 0
    head_columns = (shape.heads + gate_heads + 2 * shape.kv_heads) * shape.head_dim
    return head_columns + (shape.heads if gate == fa.GATE_HEADWISE else 0)


@pytest.mark.parametrize("gate", [fa.GATE_NONE, fa.GATE_ELEMENTWISE, fa.GATE_HEADWISE])
@pytest.mark.parametrize("head_dim,rotary_dim", [(64, 32), (128, 64), (128, 128)])
@pytest.mark.parametrize("rows,first", [(1, 300), (96, 0), (5, 40)])
@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
def test_gated_attention_matches_the_oracle(torch, gate, head_dim, rotary_dim, rows, first, dtype):
    """Decode (1 row), tensor-core prefill (96 rows) and a short split-KV prefill, with head
    norms, a partial rotary width and every gate kind."""
    shape = fa.Shape(1, 8, 2, head_dim)
    pair = Pair(shape, 400, dtype, filled=first, seed=21)
    width = gated_width(shape, gate)
    qkv = normal(921, (rows, width))
    qn = 1.0 + 0.2 * normal(922, (head_dim,))
    kn = 1.0 + 0.2 * normal(923, (head_dim,))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), rotary_dim, range(first, first + rows))
    span = fa.Span(rows, first, fa.Mask.causal())
    out = torch.zeros((rows, shape.width), device="cuda")
    pair.gpu.gated_attention(0, span, dev(torch, qkv), out, gate, rotary_dim, dev(torch, angles),
                             norm=(dev(torch, qn), dev(torch, kn), 1e-6))
    fa.device_status()
    q = qkv.copy()
    pair.cpu.gated_input(0, rows, first, gate, rotary_dim, angles, q, width, qn, kn, 1e-6)
    pair.keep_rounding(0, first, rows)
    attended = pair.cpu.attend(0, rows, first, oracle.Mask.causal(), q, width, threads=8)
    want = oracle.gate(rows, shape.heads, shape.kv_heads, head_dim, gate, q, attended)
    got = out.cpu().numpy()
    print(compare(f"gated g{gate} d{head_dim}/{rotary_dim} rows {rows}", got, want))
    assert parity_ok(got, want, dtype == fa.BF16)


def test_gated_attention_argument_errors(torch):
    shape = fa.Shape(1, 8, 2, 64)
    cache = fa.KvCache(shape, 64)
    qkv = torch.zeros((1, gated_width(shape, fa.GATE_ELEMENTWISE)), device="cuda")
    out = torch.zeros((1, shape.width), device="cuda")
    angles = torch.zeros((1, 32), device="cuda")
    span = fa.Span(1, 0, fa.Mask.causal())
    for gate, rd in ((3, 32), (fa.GATE_NONE, 0), (fa.GATE_NONE, 66), (fa.GATE_NONE, 31)):
        with pytest.raises(fa.FaError) as e:
            cache.gated_attention(0, span, qkv, out, gate, rd, angles)
        assert e.value.code == fa.ERR_ARG
    narrow = torch.zeros((1, shape.qkv), device="cuda")
    with pytest.raises(fa.FaError) as e:
        cache.gated_attention(0, span, narrow, out, fa.GATE_ELEMENTWISE, 32, angles)
    assert e.value.code == fa.ERR_SHAPE
