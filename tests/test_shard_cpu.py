"""The multi-GPU partitioning on the CPU: the partition functions cover every unit exactly once,
and a KV-range split over world_size-2 gloo ranks, all-gathered and merged by log-sum-exp in the
partial format of fa_attend_partial (base-2 max, sum, unnormalised output), reproduces the
oracle's whole-context attention."""
import os
import socket
import types

import numpy as np
import pytest

from fusor_attn.shard import kv_shards, query_row_shards, shard_sequences

LOG2E = 1.4426950408889634


def test_shard_sequences_covers_and_balances():
    lengths = np.random.default_rng(301).integers(512, 8193, size=64)
    for world in (1, 2, 4, 8):
        parts = shard_sequences(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(int(lengths[i]) + 1 for i in p) for p in parts]
        assert max(loads) - min(loads) <= int(lengths.max()) + 1


def test_kv_shards_tile_the_range():
    for world in (1, 2, 4, 8):
        s = kv_shards(131073, world)
        assert s[0][0] == 0 and s[-1][1] == 131073
        assert all(a[1] == b[0] for a, b in zip(s, s[1:]))
        assert max(h - l for l, h in s) - min(h - l for l, h in s) <= 1


def test_query_row_shards_tile_the_rows_in_whole_pairs():
    for rows in (32760, 300, 129, 256, 5):
        for world in (1, 2, 3, 8):
            s = query_row_shards(rows, world)
            assert s[0][0] == 0 and s[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(s, s[1:]))
            # every boundary but the end falls on a 256-row pair
            assert all(a % 256 == 0 for a, _ in s if a < rows)
            pairs = [(-(-(hi - lo) // 256)) for lo, hi in s]
            assert max(pairs) - min(pairs) <= 1, (rows, world, s)


def partial_np(q, keys, values):
    """One shard's (max, sum, o) per head in fa_attend_partial's format, in float64."""
    d = q.shape[-1]
    s = np.einsum("hd,hkd->hk", q, keys) * (LOG2E / np.sqrt(d))
    m = s.max(axis=1) if s.shape[1] else np.full(q.shape[0], -np.inf)
    p = np.exp2(s - m[:, None]) if s.shape[1] else s
    return np.concatenate([m[:, None], p.sum(1)[:, None], np.einsum("hk,hkd->hd", p, values)], 1)


def merge_np(partials):
    m = partials[:, :, 0]
    mm = m.max(0)
    f = np.where(np.isinf(m), 0.0, np.exp2(m - mm))
    return (f[:, :, None] * partials[:, :, 2:]).sum(0) / (f * partials[:, :, 1]).sum(0)[:, None]


def _rank(rank, world, port, q, keys, values, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = kv_shards(keys.shape[1], world)[rank]
    mine = torch.from_numpy(partial_np(q, keys[:, lo:hi], values[:, lo:hi]))
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    result[rank] = merge_np(torch.stack(gathered).numpy())
    dist.barrier()
    dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_kv_range_split_over_gloo_ranks_matches_the_oracle(world):
    import torch.multiprocessing as mp

    import oracle

    rng = np.random.default_rng(4)
    heads, kv_heads, d, n = 4, 2, 32, 1001
    cache = oracle.Cache(1, heads, kv_heads, d, n)
    cache.keys[:] = rng.standard_normal(cache.keys.shape)
    cache.values[:] = rng.standard_normal(cache.values.shape)
    q = rng.standard_normal((heads, d)).astype(np.float32)
    qkv = np.zeros((1, (heads + 2 * kv_heads) * d), np.float32)
    qkv[0, : heads * d] = q.reshape(-1)
    want = cache.attend(0, 1, n - 1, oracle.Mask.causal(), qkv, qkv.shape[1]).reshape(heads, d)
    group = heads // kv_heads
    keys = np.repeat(cache.keys[0], group, axis=0).astype(np.float64)    # per query head
    values = np.repeat(cache.values[0], group, axis=0).astype(np.float64)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        port = free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, q.astype(np.float64), keys, values, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        for r in range(world):
            assert np.abs(result[r] - want).max() < 1e-5


class _FakeExchange:
    """Stands in for fa.PeerExchange: rank 1 cannot map the other ranks' buffers."""

    closed = False

    def __init__(self, heads, head_dim, group=None):
        import torch.distributed as dist
        self.ok = dist.get_rank(group) != 1

    def close(self):
        _FakeExchange.closed = True


def _agree_rank(rank, world, port, result):
    import torch.distributed as dist

    import fusor_attn as fa
    from fusor_attn.shard import ShardedDecode
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fa.PeerExchange = _FakeExchange
        decode = types.SimpleNamespace(heads=4, head_dim=32, group=None, exchange="peer")
        peers = ShardedDecode._open_peers(decode, dist)
        result[rank] = (peers is None, decode.exchange, _FakeExchange.closed)
    finally:
        dist.destroy_process_group()


def test_peer_exchange_falls_back_to_nccl_on_every_rank_when_one_cannot_map():
    """The set-up of the peer exchange is collective: when one rank could not map the others'
    buffers, every rank goes on with NCCL and releases what it had set up."""
    import torch.multiprocessing as mp
    world = 3
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        port = free_port()
        procs = [ctx.Process(target=_agree_rank, args=(r, world, port, result)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        for r in range(world):
            none, exchange, closed = result[r]
            assert none and exchange == "nccl"
            assert closed  # every rank releases what it holds (a failed rank its own buffer)


def _watchdog_rank(rank, world, port, mode, result):
    import datetime
    import time as _time

    import torch
    import torch.distributed as dist

    import fusor_attn as fa
    from fusor_attn.shard import wait_or_abort
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    mine = torch.full((3,), float(rank))
    out = torch.zeros(3 * world)
    wait_or_abort(dist.all_gather_into_tensor(out, mine, async_op=True), 5.0, "step 1")
    ok = out.tolist() == [float(r) for r in range(world) for _ in range(3)]
    if rank == world - 1:
        # this rank leaves between steps (none of its collectives in flight), at once or after
        # stalling longer than the others' watchdog
        if mode == "stalls":
            _time.sleep(4.0)
        result[rank] = ("left", ok)
        os._exit(0)
    start = _time.monotonic()
    try:
        wait_or_abort(dist.all_gather_into_tensor(out, mine, async_op=True), 1.5, "step 2")
        result[rank] = ("no error", ok, _time.monotonic() - start)
    except fa.FaError as e:
        result[rank] = (e.code, ok, _time.monotonic() - start)
    os._exit(0)


@pytest.mark.parametrize("mode", ["exits", "stalls"])
def test_exchange_watchdog_ends_a_step_whose_rank_left(mode):
    """The NCCL exchange's host-side watchdog (wait_or_abort), on gloo ranks: after a step every
    rank completes, the last rank leaves (at once, or after stalling past the others' 1.5 s
    limit); the other ranks' next collective ends with FaError(ERR_TIMEOUT) and an aborted group,
    within seconds instead of the process group's 60 s timeout."""
    import torch.multiprocessing as mp

    import fusor_attn as fa
    world = 3
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        port = free_port()
        procs = [ctx.Process(target=_watchdog_rank, args=(r, world, port, mode, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        assert result[world - 1] == ("left", True)
        for r in range(world - 1):
            code, ok, waited = result[r]
            assert ok and code == fa.ERR_TIMEOUT, result[r]
            assert waited < 30.0, result[r]
