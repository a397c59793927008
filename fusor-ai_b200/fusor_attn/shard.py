"""Multi-GPU partitioning of the attention path: one process per GPU, torch.distributed for the
plumbing, a collective only where the path has a real exchange step.

- Independent sequences (batched decode): whole sequences per rank, balanced by keys, no
  collective (`shard_sequences`).
- One long context (split-KV decode): each rank holds a contiguous range of key positions in
  its own KvCache (`kv_shards`); every rank attends its range and produces per-head
  (max, sum, partial output) triples, which reach every rank for the log-sum-exp merge
  (`ShardedDecode`): stored straight into every rank's buffer over NVLink peer memory by one
  small kernel that then merges (`exchange="peer"`), or by an NCCL all-gather and the merge
  kernel (`exchange="nccl"`).
- Full-mask attention: contiguous runs of 256-query pairs (all heads) split evenly over ranks,
  every rank reading the K/V locally and making one call (`query_row_shards`), no collective.

The reference has no multi-device path (one process, one thread team); these are the B200 forms
of its one-call semantics, checked against the single-GPU result by the tests.
"""
from __future__ import annotations

import time
from dataclasses import dataclass


def shard_sequences(lengths, world: int):
    """Sequence indices of each rank: longest first onto the least-loaded rank (keys + 1)."""
    order = sorted(range(len(lengths)), key=lambda i: -int(lengths[i]))
    loads = [0] * world
    parts = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: loads[k])
        parts[r].append(i)
        loads[r] += int(lengths[i]) + 1
    return [sorted(p) for p in parts]


def kv_shards(keys: int, world: int):
    """Contiguous key-position ranges [lo, hi) of each rank, as even as integers allow."""
    return [(keys * r // world, keys * (r + 1) // world) for r in range(world)]


def query_row_shards(rows: int, world: int, pair: int = 256):
    """Each rank's query rows [lo, hi) of a full-mask call: the ceil(rows / pair) pairs of query
    tiles (the two-tile kernel's unit, one per query head) in `world` contiguous, equal runs, so
    that every rank makes one call over all heads and ragged tiles occur only at the end."""
    pairs = (rows + pair - 1) // pair
    return [(min(rows, pairs * r // world * pair), min(rows, pairs * (r + 1) // world * pair))
            for r in range(world)]


def _abort(group=None):
    """Aborts the process group (its communicator released, every rank's pending collective on
    it ended with an error); best effort: the group may already be gone."""
    try:
        from torch.distributed import distributed_c10d as c10d
        c10d._abort_process_group(group)
    except Exception:  # noqa: BLE001 - the error raised to the caller is the exchange's
        pass


def wait_or_abort(work, timeout_s: float, what: str, group=None):
    """Waits on the host for this rank's asynchronous collective `work`, at most `timeout_s`, so
    that a rank that left or stalls cannot hold the others for the process group's own timeout
    (minutes). Past the limit the group is aborted and FaError(ERR_TIMEOUT) raised; a collective
    that ended with an error (a peer that exited) raises the same after the abort. The
    reference's analogue is a cancelled job (crates/bundle/src/engine.rs:13-14)."""
    import fusor_attn as fa
    deadline = time.monotonic() + timeout_s
    while not work.is_completed():
        if time.monotonic() > deadline:
            _abort(group)
            raise fa.FaError(fa.ERR_TIMEOUT, f"{what}: no progress in {timeout_s:g} s; the process "
                                             "group was aborted")
        time.sleep(50e-6)
    try:
        work.wait()
    except Exception as e:  # noqa: BLE001 - re-raised as the exchange's status
        _abort(group)
        raise fa.FaError(fa.ERR_TIMEOUT, f"{what} failed ({e}); the process group was aborted") from e


@dataclass
class ShardedDecode:
    """One decode row over a context split by key position across the ranks of `group`.

    Rank r's `cache` holds positions kv_shards(total, world)[r] at slots 0.. (its capacity is
    its range, plus one slot for the new row on the last rank). A step rotates the query on
    every rank, keeps the new row on the rank that holds its position, attends the local range
    into (max, sum, o) per head, all-gathers those over NCCL and merges them."""

    cache: object          # fusor_attn.KvCache of this rank's range
    heads: int
    head_dim: int
    lo: int
    hi: int                # this rank's key positions, hi exclusive (the new row included)
    position: int          # the new row's position
    world: int
    group: object = None   # torch.distributed process group (None: the default group)
    exchange: str = "nccl"  # "peer": fa_exchange_merge over NVLink peer memory
    timeout_s: float = 10.0  # the NCCL exchange's host-side watchdog (eager steps)

    def __post_init__(self):
        import torch
        self.q = torch.zeros((1, self.heads * self.head_dim), device="cuda")
        self.partials = torch.zeros((self.heads, self.head_dim + 2), device="cuda")
        self.gathered = torch.zeros((self.world, self.heads, self.head_dim + 2), device="cuda")
        self.out = torch.zeros((self.heads, self.head_dim), device="cuda")
        self.owner = self.lo <= self.position < self.hi
        self.peers = None  # the PeerExchange, made by the first exchange (a collective step)

    def rotate(self, qkv, angles, rope):
        """The query rotated on every rank; the new row kept on the rank holding its position."""
        import fusor_attn as fa
        if self.owner:
            # keep the new row at its slot in this shard; the rotated query comes back with it
            span = fa.Span(1, self.position - self.lo, fa.Mask.causal())
            self.cache.attention_input(0, span, qkv, angles, rope, q_out=self.q)
        else:
            fa.rotate_queries(self.heads, self.head_dim, qkv, self.q, angles, rope)

    def attend_local(self):
        """This rank's key range into per-head (max, sum, o)."""
        self.cache.attend_partial(0, self.q, 0, self.hi - self.lo, self.partials)

    def gather_merge(self, dist=None):
        """Every rank's partials merged into `out`: over peer memory, or over NCCL."""
        import fusor_attn as fa
        if dist is not None and self.world > 1 and self.exchange == "peer" and self.peers is None:
            self.peers = self._open_peers(dist)
        if self.peers is not None:
            self.peers.merge(self.partials, self.out)
            return self.out
        if dist is not None and self.world > 1:
            import torch
            # Eager steps wait for the all-gather on the host under the watchdog; a step being
            # captured into a CUDA graph cannot wait on the host (its replay is bounded by the
            # process group's own timeout).
            eager = not torch.cuda.is_current_stream_capturing()
            work = dist.all_gather_into_tensor(self.gathered, self.partials, group=self.group,
                                               async_op=eager)
            if eager:
                wait_or_abort(work, self.timeout_s, "the partials' all-gather", self.group)
        else:
            self.gathered[0].copy_(self.partials)
        fa.merge_partials(self.gathered, self.out)
        return self.out

    def _open_peers(self, dist):
        """The peer exchange, if every rank could map every other's buffer; otherwise (a box
        without peer access, say) every rank agrees to use NCCL instead."""
        import torch

        import fusor_attn as fa
        peers = fa.PeerExchange(self.heads, self.head_dim, self.group)
        device = "cuda" if dist.get_backend(self.group) == "nccl" else "cpu"
        flag = torch.tensor([1 if peers.ok else 0], device=device, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        if int(flag.item()) == 1:
            return peers
        peers.close()
        self.exchange = "nccl"
        return None

    def recover(self, dist=None):
        """After a run of steps, on every rank at the same point: whether any rank's peer
        exchange gave up waiting for another (its merged output was then incomplete), the
        exchange made ready again if so (every rank's step counter and flags cleared together).
        With the NCCL exchange a rank that fails raises from the collective itself."""
        if self.peers is None or dist is None:
            import fusor_attn as fa
            fa.device_status()
            return False
        return self.peers.recover(self.group)

    def close(self, dist=None):
        """Releases the peer buffers (every rank, after its last step)."""
        if self.peers is not None:
            import torch
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier(group=self.group)
            self.peers.close()
            self.peers = None

    def step(self, qkv, angles, rope, dist=None):
        self.rotate(qkv, angles, rope)
        self.attend_local()
        return self.gather_merge(dist)
