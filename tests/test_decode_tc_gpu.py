"""The tensor-core decode over bf16 caches (one-row spans of a batch, head_dim 128 and 256: the
latter's tiles in two 128-wide halves): every query head group up to 16, key counts around the
128-key tile and across chunks, the masks whose keys are one run of cache slots, and the cases
that stay on the CUDA cores (a window that wraps the ring), all against the oracle at the
bf16-compute bar."""
import numpy as np
import pytest

import fusor_attn as fa
from gpu_util import Pair, compare, max_abs, normal, parity_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def run_batch(torch, shape, positions, masks, capacity=None, seed=0):
    pairs = [Pair(shape, capacity or (p + 1), fa.BF16, filled=min(p, capacity or p), seed=seed + i)
             for i, p in enumerate(positions)]
    qkv = normal(seed + 100, (len(pairs), shape.qkv))
    angles = fa.rotary_angles(fa.Rotation(base=1e6), shape.head_dim, positions)
    spans = [fa.Span(1, p, m) for p, m in zip(positions, masks)]
    out = torch.zeros((len(pairs), shape.width), device="cuda")
    fa.attention_batch([p.gpu for p in pairs], spans, 0, dev(torch, qkv), out, dev(torch, angles),
                       fa.ROPE_HALF)
    fa.device_status()
    got = out.cpu().numpy()
    worst = 0.0
    for i, (p, span) in enumerate(zip(pairs, spans)):
        want = p.oracle_attention(0, span, qkv[i:i + 1], angles[i:i + 1], fa.ROPE_HALF, threads=4)
        err = max_abs(got[i:i + 1], want)
        worst = max(worst, err)
        assert parity_ok(got[i:i + 1], want, True), compare(f"row {i} position {positions[i]}",
                                                             got[i:i + 1], want)
    return worst


@pytest.mark.parametrize("head_dim", [128, 256])
@pytest.mark.parametrize("group", [1, 2, 4, 8, 16])
def test_every_group_size(torch, group, head_dim):
    kv = 2
    shape = fa.Shape(1, kv * group, kv, head_dim)
    positions = [0, 126, 127, 128, 300, 2047]
    worst = run_batch(torch, shape, positions, [fa.Mask.causal()] * len(positions),
                      seed=40 * group + head_dim)
    print(f"d{head_dim} group {group}: max abs {worst:.2e}")


@pytest.mark.parametrize("heads,kv,head_dim", [(32, 8, 128), (8, 2, 256), (16, 2, 256)])
def test_long_rows_across_chunks(torch, heads, kv, head_dim):
    """Rows of very different lengths in one batch: the long ones split into chunks merged by
    log-sum-exp, the short ones one chunk (head_dim 256: Qwen3.5's gated layers' 8/2 heads, and a
    group of 8)."""
    shape = fa.Shape(1, heads, kv, head_dim)
    positions = [9000, 17, 4500, 129, 12000, 1]
    worst = run_batch(torch, shape, positions, [fa.Mask.causal()] * len(positions), seed=900)
    print(f"long rows d{head_dim}: max abs {worst:.2e}")


@pytest.mark.parametrize("head_dim", [128, 256])
def test_window_and_full_masks(torch, head_dim):
    """A window inside the ring (one run of slots) and a full mask over the row's own keys; a
    window that wraps the ring decodes on the CUDA cores in the same batch call."""
    shape = fa.Shape(1, 8, 2, head_dim)
    positions = [700, 1500]
    worst = run_batch(torch, shape, positions, [fa.Mask.window_of(300), fa.Mask.full()],
                      capacity=2000, seed=77)
    print(f"window/full: max abs {worst:.2e}")
    wrapped = run_batch(torch, shape, [2500, 2600], [fa.Mask.window_of(400)] * 2, capacity=1000,
                        seed=78)
    print(f"wrapped window (CUDA cores): max abs {wrapped:.2e}")
