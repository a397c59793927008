"""fa_attend_static, the decode entry point that allocates nothing, checked against fa_attend.

Callers that cannot allocate device memory at call time (a host whose GPU memory is pre-reserved
by its own pool, or a decode loop that cannot take cudaMalloc's implicit synchronisation) use
this variant: its split-KV scratch is a fixed array inside the library. This file runs last
(pytest collects it after the others) so that a failure here stops a `-x` run only after every
other test has run; it passes alone in a fresh process as well as after the others.
"""
import ctypes as C

import pytest

import fusor_attn as fa
from gpu_util import TOL_F32

pytestmark = pytest.mark.gpu


def _static_attend(cache, span, q, out):
    sp = span.c()
    return fa.lib().fa_attend_static(cache.handle, 0, C.byref(sp), C.c_void_p(q.data_ptr()),
                                     q.stride(0), C.c_void_p(out.data_ptr()), out.stride(0),
                                     fa._stream())


def test_static_scratch_attend_matches_fa_attend_on_two_calls():
    import torch

    torch.cuda.set_device(0)
    shape = fa.Shape(1, 16, 8, 128)
    n = 20000  # long enough that the split-KV kernel splits the keys and merges partials
    cache = fa.KvCache(shape, n + 1)
    gen = torch.Generator("cuda").manual_seed(11)
    cache.put_rows(torch.randn((1, 8, n, 128), device="cuda", generator=gen),
                   torch.randn((1, 8, n, 128), device="cuda", generator=gen))
    span = fa.Span(1, n - 1, fa.Mask.causal())
    for call in range(2):
        q = torch.randn((1, shape.width), device="cuda", generator=gen)
        want = torch.zeros((1, shape.width), device="cuda")
        cache.attend(0, span, q, want)
        got = torch.full((1, shape.width), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = _static_attend(cache, span, q, got)
        torch.cuda.synchronize()
        assert rc == fa.OK, fa.lib().fa_last_error()
        if call == 1:  # the first call on a device may load the library's device code
            assert torch.cuda.mem_get_info()[0] == free_before
        err = float((got - want).abs().max())
        print(f"call {call}: fa_attend_static vs fa_attend max abs {err:.2e}")
        assert err <= TOL_F32
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
