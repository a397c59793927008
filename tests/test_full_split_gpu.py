"""The split schedule of bf16 full-mask calls (blocks::attention::Call, attention.rs:36-47): when a
call's (query head, 256-query pair) units do not fill the SMs evenly, the last waves' units run
as several CTAs over equal shares of the keys, and the last of them merges the partials. The
output must match the oracle as the unsplit schedule does, on every row (whole units and split
ones side by side), for GQA, several images, ragged query and key counts, f32 and bf16 output,
and again on a second call (the arrival counters reset themselves) and on another stream."""
import numpy as np
import pytest

import fusor_attn as fa
import oracle
from gpu_util import compare, normal, parity_ok, round_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def run_call(torch, heads, kv, d, images, queries, keys, out_dtype, seed, stream=None):
    q = round_bf16(normal(seed, (images * queries, heads * d)))
    k = round_bf16(normal(seed + 1, (images * keys, kv * d)))
    v = round_bf16(normal(seed + 2, (images * keys, kv * d)))
    tq, tk, tv = (torch.from_numpy(x).to("cuda").to(torch.bfloat16) for x in (q, k, v))
    out = torch.zeros((images * queries, heads * d), device="cuda", dtype=out_dtype)
    torch.cuda.synchronize()  # the operands are in place before a call on another stream
    fa.attend_full(heads, kv, d, images, queries, keys, fa.Operand(tq, heads * d),
                   fa.Operand(tk, kv * d), fa.Operand(tv, kv * d), out, stream=stream)
    torch.cuda.synchronize()
    fa.device_status()
    return (q, k, v), out


# (heads, kv heads, head_dim, images, queries, keys, output): on a 148-SM B200 the first splits
# its 4 units 8 ways, the second its 16 units 6 ways, the third runs 296 units whole and splits
# the other 24, the fourth splits its 12 units 6 ways.
CASES = {
    "eight_pieces": (2, 2, 128, 1, 300, 4100, "f32"),
    "gqa_images_bf16_out": (8, 2, 128, 2, 200, 3000, "bf16"),
    "whole_then_pieces": (20, 20, 128, 1, 4096, 4096, "bf16"),
    "head_dim_64": (4, 1, 64, 1, 520, 3000, "f32"),
}


@pytest.mark.parametrize("name", list(CASES))
def test_split_full_mask_matches_the_oracle(torch, name):
    heads, kv, d, images, queries, keys, out_name = CASES[name]
    out_dtype = torch.float32 if out_name == "f32" else torch.bfloat16
    (q, k, v), out = run_call(torch, heads, kv, d, images, queries, keys, out_dtype, 900)
    got = out.float().cpu().numpy()
    want = np.zeros_like(got)
    # rows of the first and the last pair of every head (whole and split units of the third
    # case), every row when the call is small
    ranges = [(0, queries)] if queries <= 600 else [(0, 64), (queries - 64, queries)]
    for qr in ranges:
        oracle.attend_call(heads, kv, d, images, queries, keys, q, heads * d, 0, k, kv * d, 0,
                           v, kv * d, 0, query_range=qr, threads=8, out=want)
    rows = np.concatenate([np.arange(i * queries + a, i * queries + b)
                           for i in range(images) for a, b in ranges])
    print(compare(f"split {name}", got[rows], want[rows]))
    assert parity_ok(got[rows], want[rows], True)


def test_split_calls_repeat_and_run_on_another_stream(torch):
    """Bit-identical output from a second call on the same stream (the counters were reset by
    the first) and from a call on another stream (its own partials)."""
    shape = CASES["eight_pieces"][:6]
    _, first = run_call(torch, *shape, torch.float32, 910)
    _, again = run_call(torch, *shape, torch.float32, 910)
    side = torch.cuda.Stream()
    _, other = run_call(torch, *shape, torch.float32, 910, stream=side)
    assert torch.equal(first, again)
    assert torch.equal(first, other)
