"""Caches past 2^31 elements: a decode row over every key of a 2-layer cache whose layers each
hold 8 x 2.1M x 128 = 2.15e9 elements, so the element offsets of a layer (and of layer 1's
base) exceed what 32 bits index. The attention at the last position, on the split-KV kernel (f32
cache) and on the tensor-core decode (bf16 cache), against plain PyTorch f32 attention over the
same keys and values (the oracle would take minutes over 2.1M keys; the cache's contents are
read back from the device for the reference)."""
import numpy as np
import pytest

import fusor_attn as fa
from gpu_util import compare, parity_ok

pytestmark = pytest.mark.gpu

CAPACITY = 2_100_000  # 8 kv heads x 128 x CAPACITY > 2^31


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    fa.lib()
    return t


def reference(torch, q, k, v, heads, kv_heads):
    """softmax(q k^T / sqrt(d)) v per query head over every key, f32 (TF32 off)."""
    d = q.shape[-1]
    group = heads // kv_heads
    out = torch.empty((heads, d), device="cuda", dtype=torch.float32)
    for h in range(heads):
        kk, vv = k[h // group].float(), v[h // group].float()
        s = (kk @ q[h]) / np.sqrt(d)
        p = torch.softmax(s, dim=0)
        out[h] = p @ vv
    return out


@pytest.mark.parametrize("dtype", [fa.F32, fa.BF16])
def test_decode_over_a_cache_past_two_billion_elements(torch, dtype):
    torch.backends.cuda.matmul.allow_tf32 = False
    heads, kv, d, layers = 16, 8, 128, 2
    shape = fa.Shape(layers, heads, kv, d)
    tdt = torch.float32 if dtype == fa.F32 else torch.bfloat16
    cache = fa.KvCache(shape, CAPACITY, dtype)
    gen = torch.Generator("cuda").manual_seed(77)
    # every row of both layers, filled on the device (put_rows copies [layers][kv][rows][d])
    k = torch.randn((layers, kv, CAPACITY, d), device="cuda", generator=gen).to(tdt)
    v = torch.randn((layers, kv, CAPACITY, d), device="cuda", generator=gen).to(tdt)
    cache.put_rows(k, v)
    q = torch.randn((1, heads * d), device="cuda", generator=gen)
    out = torch.zeros((1, heads * d), device="cuda")
    span = fa.Span(1, CAPACITY - 1, fa.Mask.causal())  # sees every slot of the cache
    cache.attend(1, span, q, out)
    torch.cuda.synchronize()
    fa.device_status()
    qq = q.view(heads, d)
    if dtype == fa.BF16:
        qq = qq.to(torch.bfloat16).float()  # the tensor-core decode's bf16 queries
    want = reference(torch, qq, k[1], v[1], heads, kv)
    got = out.view(heads, d)
    del k, v
    g, w = got.cpu().numpy(), want.cpu().numpy()
    print(compare(f"{CAPACITY}-row decode {'f32' if dtype == fa.F32 else 'bf16'}", g, w))
    rel = float(np.sqrt(((g - w) ** 2).sum() / (w ** 2).sum()))
    assert parity_ok(g, w, dtype == fa.BF16)
    assert rel <= (1e-4 if dtype == fa.F32 else 2e-2)
