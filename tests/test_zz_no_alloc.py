"""fa_attend_static, the decode entry point that allocates nothing, checked against fa_attend and
against the oracle.

Callers that cannot allocate device memory at call time (a host whose GPU memory is pre-reserved
by its own pool, or a decode loop that cannot take cudaMalloc's implicit synchronisation) use
this variant: its split-KV scratch is a fixed array inside the library. It runs the split-KV
kernel in f32 arithmetic over f32 or bf16 caches, so it is held to the f32 bar against the oracle
(given the bf16 cache's rounded keys and values) for every case; against fa_attend, which decodes
a bf16 cache of head_dim 128 on the tensor cores, to the bf16 bar there.

This file runs last (pytest collects it after the others) so that a failure here stops a `-x` run
only after every other test has run; it passes alone in a fresh process as well as after the
others.
"""
import ctypes as C

import pytest

import fusor_attn as fa
from gpu_util import TOL_BF16, TOL_F32, Pair, compare, max_abs, normal, to_oracle_mask

pytestmark = pytest.mark.gpu


def _static_attend(cache, span, q, out):
    sp = span.c()
    return fa.lib().fa_attend_static(cache.handle, 0, C.byref(sp), C.c_void_p(q.data_ptr()),
                                     q.stride(0), C.c_void_p(out.data_ptr()), out.stride(0),
                                     fa._stream())


# (name, cache dtype, shape (layers, heads, kv heads, head_dim), capacity, seeded rows, span)
CASES = [
    # one row over 20000 keys: the keys split into chunks whose partials merge through the array
    ("f32_split", fa.F32, (1, 16, 8, 128), 20001, 20000, fa.Span(1, 19999, fa.Mask.causal())),
    ("bf16_split", fa.BF16, (1, 16, 8, 128), 20001, 20000, fa.Span(1, 19999, fa.Mask.causal())),
    # head_dim 256 over a bf16 cache: the tensor-core decode's chunk partials in the array
    ("bf16_d256_split", fa.BF16, (1, 8, 2, 256), 12001, 12000, fa.Span(1, 11999, fa.Mask.causal())),
    # C1's shape: 1025 keys, whose chunks run as one thread-block cluster (merged in shared
    # memory: only the counters come from the array)
    ("f32_cluster", fa.F32, (1, 14, 2, 64), 1025, 1024, fa.Span(1, 1024, fa.Mask.causal())),
    ("bf16_cluster", fa.BF16, (1, 14, 2, 64), 1025, 1024, fa.Span(1, 1024, fa.Mask.causal())),
    # five rows under a window that wraps the cache's ring
    ("window_ring_rows", fa.F32, (1, 8, 2, 64), 3000, 3000,
     fa.Span(5, 10000, fa.Mask.window_of(2900))),
    # eight rows under Groups (the reference's stacks.rs mask), each row its own two key runs
    ("groups_rows", fa.F32, (1, 8, 2, 64), 64, 0, fa.Span(8, 0, fa.Mask.groups(3, [5, 6, 8]))),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_static_scratch_attend_matches_fa_attend_and_the_oracle_on_two_calls(case):
    import torch

    torch.cuda.set_device(0)
    name, dtype, dims, capacity, filled, span = case
    shape = fa.Shape(*dims)
    pair = Pair(shape, capacity, dtype, filled=filled, seed=1100)
    # the span's rows kept first (RoPE by halves), their rotated queries into q
    qkv = normal(1102, (span.rows, shape.qkv))
    positions = range(span.first, span.first + span.rows)
    angles = fa.rotary_angles(fa.Rotation(base=1e6), shape.head_dim, positions)
    q = torch.zeros((span.rows, shape.width), device="cuda")
    pair.gpu.attention_input(0, span, torch.from_numpy(qkv).cuda(), torch.from_numpy(angles).cuda(),
                             fa.ROPE_HALF, q_out=q)
    want_oracle = pair.oracle_attention(0, span, qkv, angles, fa.ROPE_HALF)
    # against fa_attend: the bf16 bar where fa_attend decodes on the tensor cores
    tc = dtype == fa.BF16 and shape.head_dim in (128, 256)
    tol_attend = TOL_BF16 if tc else TOL_F32
    for call in range(2):
        if call == 1:  # another query the second time: nothing carries over from the first call
            q = q.flip(0).contiguous() * 0.5
            qh = q.cpu().numpy()
            want_oracle = pair.cpu.attend(0, span.rows, span.first, to_oracle_mask(span.mask),
                                          qh, qh.shape[1], threads=8)
        want = torch.zeros((span.rows, shape.width), device="cuda")
        pair.gpu.attend(0, span, q, want)
        got = torch.full((span.rows, shape.width), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = _static_attend(pair.gpu, span, q, got)
        torch.cuda.synchronize()
        assert rc == fa.OK, fa.lib().fa_last_error()
        if call == 1:  # the first call on a device may load the library's device code
            assert torch.cuda.mem_get_info()[0] == free_before
        g = got.cpu().numpy()
        err = max_abs(g, want.cpu().numpy())
        print(f"{name} call {call}: fa_attend_static vs fa_attend max abs {err:.2e}; "
              + compare("vs the oracle", g, want_oracle))
        assert err <= tol_attend
        assert max_abs(g, want_oracle) <= TOL_F32
    fa.device_status()


def test_static_scratch_rejects_spans_beyond_its_size():
    import torch

    shape = fa.Shape(1, 32, 8, 256)
    cache = fa.KvCache(shape, 4096)
    q = torch.zeros((16, shape.width), device="cuda")
    out = torch.zeros_like(q)
    rc = _static_attend(cache, fa.Span(16, 4000, fa.Mask.causal()), q, out)
    assert rc == fa.ERR_ARG
    assert b"fa_attend_static holds" in fa.lib().fa_last_error()
    assert float(out.abs().max()) == 0.0  # nothing launched
