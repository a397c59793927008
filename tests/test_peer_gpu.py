"""The exchange of a KV-range-sharded decode over NVLink peer memory (fa_exchange_merge) against
the NCCL all-gather + merge it replaces: one process per GPU (2 to 4 of them; skipped on a box
with fewer than 2), each rank holding a contiguous range of a 4097-position cache. Checked:
the same bits as the NCCL path over several steps (both halves of the double buffer), the same
bits again when the step is replayed as a CUDA graph (the step count lives on the device), and
the unsharded decode's output within the f32 bar."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HEADS, KV, D, TOTAL = 16, 8, 128, 4097


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port):
    import datetime

    import torch
    import torch.distributed as dist

    import fusor_attn as fa
    from fusor_attn.shard import ShardedDecode, kv_shards

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        position = TOTAL - 1
        rng = np.random.default_rng(17)
        keys = rng.standard_normal((KV, TOTAL, D), dtype=np.float32)
        values = rng.standard_normal((KV, TOTAL, D), dtype=np.float32)
        qkv = torch.from_numpy(rng.standard_normal((1, (HEADS + 2 * KV) * D), dtype=np.float32)).cuda()
        angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), D, [position])).cuda()
        lo, hi = kv_shards(TOTAL, world)[rank]
        cache = fa.KvCache(fa.Shape(1, HEADS, KV, D), hi - lo)
        filled = min(hi, position) - lo
        cache.put_rows(torch.from_numpy(keys[None, :, lo:lo + filled].copy()).cuda(),
                       torch.from_numpy(values[None, :, lo:lo + filled].copy()).cuda())
        nccl = ShardedDecode(cache, HEADS, D, lo, hi, position, world)
        peer = ShardedDecode(cache, HEADS, D, lo, hi, position, world, exchange="peer")
        want = nccl.step(qkv, angles, fa.ROPE_HALF, dist).clone()
        for _ in range(3):  # odd and even steps: both halves of the exchange buffers
            got = peer.step(qkv, angles, fa.ROPE_HALF, dist)
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"rank {rank}: peer exchange differs from NCCL"
        # the step replayed as a CUDA graph
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="relaxed"):
            peer.step(qkv, angles, fa.ROPE_HALF, dist)
        for _ in range(3):
            peer.out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(peer.out, want), f"rank {rank}: graph replay differs"
        del graph
        fa.device_status()
        if rank == 0:
            full = fa.KvCache(fa.Shape(1, HEADS, KV, D), TOTAL)
            full.put_rows(torch.from_numpy(keys[None, :, :position].copy()).cuda(),
                          torch.from_numpy(values[None, :, :position].copy()).cuda())
            out = torch.zeros((1, HEADS * D), device="cuda")
            full.attention(0, fa.Span(1, position, fa.Mask.causal()), qkv, out, angles,
                           fa.ROPE_HALF)
            err = float((out.view(HEADS, D) - want).abs().max())
            assert err <= 2e-3, f"sharded vs unsharded max abs {err:.3e}"
        peer.close(dist)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_matches_the_nccl_all_gather(world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_rank, args=(world, _free_port()), nprocs=world, join=True)


def test_exchange_wait_gives_up_on_a_rank_that_never_publishes():
    """One process, one GPU: rank 0 of a 2-rank exchange whose rank 1 never runs (its buffer is
    a second local allocation that nothing else writes). The kernel's wait on rank 1's flag runs
    out after about a second; the host reads ERR_TIMEOUT from fa_device_status, the rank's own
    partials are still merged, and the context stays usable (a 1-rank exchange right after it
    succeeds with a clean status)."""
    import ctypes as C
    import time

    import torch

    import fusor_attn as fa
    assert torch.cuda.is_available()
    lib = fa.lib()
    heads, d, world = 4, 64, 2
    nbytes = C.c_uint64()
    assert lib.fa_peer_buffer_bytes(world, heads, d, C.byref(nbytes)) == fa.OK
    owned = []
    for _ in range(world):
        p, handle = C.c_void_p(), (C.c_ubyte * 64)()
        assert lib.fa_peer_alloc(nbytes.value, C.byref(p), handle) == fa.OK
        owned.append(p)
    try:
        buffers = (C.c_void_p * world)(*(p.value for p in owned))
        gen = torch.Generator("cuda").manual_seed(5)
        partials = torch.empty((heads, d + 2), device="cuda")
        partials[:, 0] = torch.rand((heads,), device="cuda", generator=gen) * 4 - 2  # max (log2)
        partials[:, 1] = torch.rand((heads,), device="cuda", generator=gen) * 2 + 1  # sum
        partials[:, 2:] = torch.randn((heads, d), device="cuda", generator=gen)
        want = partials[:, 2:] / partials[:, 1:2]
        out = torch.zeros((heads, d), device="cuda")
        stream = fa._stream(None)
        start = time.monotonic()
        assert lib.fa_exchange_merge(buffers, nbytes.value, 0, world, heads, d,
                                     fa._dptr(partials), fa._dptr(out), stream) == fa.OK
        with pytest.raises(fa.FaError) as err:
            fa.device_status()
        waited = time.monotonic() - start
        assert err.value.code == fa.ERR_TIMEOUT
        assert 0.2 < waited < 30.0, f"the wait gave up after {waited:.2f} s"
        # rank 1's slot is still zero (max 0, sum 0): the merge is rank 0's partials alone
        assert torch.allclose(out, want, rtol=1e-6, atol=1e-6)
        # the context is usable and the error word was cleared: a 1-rank exchange on buffer 0
        out.zero_()
        assert lib.fa_exchange_merge(buffers, nbytes.value, 0, 1, heads, d, fa._dptr(partials),
                                     fa._dptr(out), stream) == fa.OK
        fa.device_status()
        assert torch.allclose(out, want, rtol=1e-6, atol=1e-6)
    finally:
        torch.cuda.synchronize()
        for p in owned:
            lib.fa_peer_free(p)


def test_exchange_leaves_out_a_late_rank_and_resumes_after_a_reset():
    """One process, one GPU, rank 0 of a 2-rank exchange. (1) Rank 1's slot holds words of an
    earlier step (planted, with a dominant max) that never carry this step's stamp: the wait gives
    up, and the merge leaves rank 1 out instead of merging the stale partials. (2) After
    fa_peer_reset the step counter starts again: with rank 1's words for step 1 in place
    beforehand (as rank 1's own kernel would have stored them), the next exchange waits for
    nothing and merges both ranks."""
    import ctypes as C

    import torch

    import fusor_attn as fa
    assert torch.cuda.is_available()
    lib = fa.lib()
    heads, d, world = 4, 64, 2
    pitch = heads * (d + 2)
    nbytes = C.c_uint64()
    assert lib.fa_peer_buffer_bytes(world, heads, d, C.byref(nbytes)) == fa.OK
    own, handle = C.c_void_p(), (C.c_ubyte * 64)()
    assert lib.fa_peer_alloc(nbytes.value, C.byref(own), handle) == fa.OK
    try:
        # the buffer as 64-bit words: the 256-byte header, then [half][rank][heads][d + 2]
        words = _view(torch, own.value, int(nbytes.value) // 8, "<i8")
        gen = torch.Generator("cuda").manual_seed(9)

        def partials_of(shift):
            p = torch.empty((heads, d + 2), device="cuda")
            p[:, 0] = torch.rand((heads,), device="cuda", generator=gen) * 4 - 2 + shift
            p[:, 1] = torch.rand((heads,), device="cuda", generator=gen) * 2 + 1
            p[:, 2:] = torch.randn((heads, d), device="cuda", generator=gen)
            return p

        def plant(half, rank, partials, step):
            bits = partials.reshape(-1).view(torch.int32).to(torch.int64) & 0xFFFFFFFF
            start = 32 + (half * world + rank) * pitch
            words[start:start + pitch] = (step << 32) | bits

        mine = partials_of(0.0)
        plant(1, 1, partials_of(20.0), 3)  # step 1 uses half 1; these words are of step 3
        out = torch.zeros((heads, d), device="cuda")
        bufs = (C.c_void_p * world)(own.value, own.value)  # rank 1's buffer: written, never read
        stream = fa._stream(None)
        torch.cuda.synchronize()
        assert lib.fa_exchange_merge(bufs, nbytes.value, 0, world, heads, d, fa._dptr(mine),
                                     fa._dptr(out), stream) == fa.OK
        with pytest.raises(fa.FaError) as err:
            fa.device_status()
        assert err.value.code == fa.ERR_TIMEOUT
        assert torch.allclose(out, mine[:, 2:] / mine[:, 1:2], rtol=1e-6, atol=1e-6)
        # the reset: the counter and every word cleared
        assert lib.fa_peer_reset(own, nbytes.value, stream) == fa.OK
        assert int(words.abs().max()) == 0
        # rank 1's step-1 words in place, then rank 0's step 1
        theirs = partials_of(0.5)
        plant(1, 1, theirs, 1)
        torch.cuda.synchronize()
        out.zero_()
        assert lib.fa_exchange_merge(bufs, nbytes.value, 0, world, heads, d, fa._dptr(mine),
                                     fa._dptr(out), stream) == fa.OK
        fa.device_status()
        both = torch.stack([mine, theirs])
        m = both[:, :, 0].max(0).values
        f = torch.exp2(both[:, :, 0] - m)
        want = (f[:, :, None] * both[:, :, 2:]).sum(0) / (f * both[:, :, 1]).sum(0)[:, None]
        assert torch.allclose(out, want, rtol=1e-5, atol=1e-6)
    finally:
        torch.cuda.synchronize()
        lib.fa_peer_free(own)


def _view(torch, address, count, typestr):
    """A tensor over `count` elements of device memory at `address` (not owned)."""
    class _Cuda:
        __cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (address, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(_Cuda(), device="cuda")
