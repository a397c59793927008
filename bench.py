#!/usr/bin/env python
"""Benchmark of the attention hot path on B200 (one JSON line on rank 0).

Headline workload (`--config c3`, the default): BASELINE config 3, one batched GQA decode step of
64 independent sequences (32 query / 8 KV heads, head_dim 128, RoPE base 1e6, Mask::Causal,
cache lengths drawn uniform in [512, 8192] from a seed), f32 cache. A step is one pass of the
hot path over the batch: RoPE + keep of each sequence's new row, then attention of every row
over its cache. `value` is tokens/s of the whole job (64 tokens per step); with N GPUs the
sequences are split across ranks by total length with no collective (total work fixed).

Other configurations (`--config c1|c2|c3bf16|decode256|c4|c5|prefill|prefill_f32|qwen35|proj|
proj64|prologue`) run the same way; the
default run adds them under "configs" in the same line. `--cpu-baselines` (1 GPU) also times the
host restatement of the reference's CPU path for C1, C2, C4 and a slice of C5, beside each.

`--impl reference` times the reference's CPU path (the oracle's C++ restatement of fusor-ai's
f32 attention, split over the host's threads as its thread team splits heads) on the same
workload and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "fusor-ai_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

C3_SEQS, C3_HEADS, C3_KV, C3_D = 64, 32, 8, 128
L2_BYTES = 126 * 1024 * 1024
# Parity bars (the tests' own): max abs error on the attention output with f32 I/O; the
# bf16-compute paths (bf16 queries and probabilities on the tensor cores) are held to a max abs
# error and a relative L2 error.
TOL_F32, TOL_BF16, REL_BF16 = 2e-3, 1e-2, 5e-3


def c3_lengths():
    return np.random.default_rng(301).integers(512, 8193, size=C3_SEQS)


def measured_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, source, bf16 TFLOP/s sustained under the power cap)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured",
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])))
    except Exception:
        return 6650.0, 1590.0, "fallback", 1400.0


def profile_traffic(kernel_key: str):
    """DRAM bytes per launch of `kernel_key` from the committed ncu summaries (profiles/*.md,
    a line `traffic_bytes_per_launch[<config>] = <bytes>`), or None."""
    import glob
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        for line in open(path):
            if line.startswith(f"traffic_bytes_per_launch[{kernel_key}]"):
                return float(line.split("=")[1].split()[0])
    return None


class ClockSampler:
    """SM clocks and clock-event reasons of this rank's GPU, sampled by NVML while running."""

    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
    }

    def __init__(self, torch, device: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self._nv = None
            self.error = str(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if bits & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def report(self):
        if self._nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------

class Workload:
    """One configuration on this rank: `step()` enqueues one pass; `kernel()` the dominant
    kernel alone; `e2e_step()` a pass through the public API from pinned host memory."""

    name = ""
    tokens = 0             # tokens of one step on this rank's share (the whole job if sharded)
    sharded = False        # the job is split over the ranks (else every rank runs a replica)
    bound = "hbm"
    launches_per_step = 0
    flush_l2 = False
    graphs = False         # latency-bound steps: the step replayed as one captured CUDA graph
    e2e_ran = False        # time_e2e ran this workload's public-API step
    e2e_returns_synchronized = False  # e2e_step returns with its host output filled
    _step_graph = None
    _kernel_graph = None

    def parity(self, threads):
        """The timed launch's output against the oracle on this rank (after the timing)."""
        return None

    def phases(self):
        """The step's two calls (before and after the dominant kernel's event)."""
        raise NotImplementedError

    def capture(self):
        """Captures the step (both calls) into one CUDA graph, and the dominant kernel's call
        into another for its own timing (after warm-up: every buffer is sized, so a replay
        allocates nothing), as a serving loop replays a decode step."""
        torch = self.torch
        first, second = self.phases()
        self._step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._step_graph, capture_error_mode="relaxed"):
            first()
            second()
        self._kernel_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._kernel_graph, capture_error_mode="relaxed"):
            second()
        torch.cuda.synchronize()

    def step(self, mid=None):
        if self._step_graph is not None:
            self._step_graph.replay()
            return
        first, second = self.phases()
        first()
        if mid is not None:
            mid.record()
        second()

    def algorithmic(self) -> float:
        """Bytes (hbm) or FLOPs (tensor) of one launch of the dominant kernel on this rank."""
        raise NotImplementedError

    def close(self):
        """Releases what the workload holds beyond device tensors (every rank, in step)."""
        self._step_graph = self._kernel_graph = None


class C3Decode(Workload):
    """A batched decode: C3's 64 sequences (lengths U[512, 8192], seed 301) at C3's shape (32/8
    heads x 128) over an f32 or a bf16 cache; `decode256`: the same sequences at Qwen3.5's gated
    layers' shape (8/2 heads x 256) over a bf16 cache."""

    def __init__(self, torch, fa, rank, world, dtype, sequences=C3_SEQS, dims=None, name=None):
        self.torch, self.fa = torch, fa
        self.dtype = dtype
        self.name = name or ("c3" if dtype == fa.F32 else "c3bf16")
        heads, kv, d = dims or (C3_HEADS, C3_KV, C3_D)
        self.dims = (heads, kv, d)
        # f32 caches decode on the CUDA cores (split-KV), bf16 caches on the tensor cores
        self.kernel = "attend_kernel" if dtype == fa.F32 else "decode_tc_kernel"
        self.sharded = True
        from fusor_attn.shard import shard_sequences
        lengths = c3_lengths()[:sequences]
        mine = shard_sequences(lengths, world)[rank]
        self.tokens = len(lengths)
        self.lengths = [int(lengths[i]) for i in mine]
        shape = fa.Shape(1, heads, kv, d)
        self.shape = shape
        # every sequence's keys and values from its own seed, and the batch's qkv rows from one:
        # the job is the same whatever the number of GPUs it is split over
        tdt = torch.float32 if dtype == fa.F32 else torch.bfloat16
        self.caches = []
        for i, n in zip(mine, self.lengths):
            gen = torch.Generator("cuda").manual_seed(1000 + int(i))
            c = fa.KvCache(shape, n + 1, dtype)
            k = torch.randn((1, kv, n, d), device="cuda", generator=gen).to(tdt)
            v = torch.randn((1, kv, n, d), device="cuda", generator=gen).to(tdt)
            c.put_rows(k, v)
            del k, v
            self.caches.append(c)
        spans = [fa.Span(1, n, fa.Mask.causal()) for n in self.lengths]
        self.batch = fa.Batch(self.caches, spans)
        b = len(self.caches)
        gen = torch.Generator("cuda").manual_seed(999)
        qkv_all = torch.randn((len(lengths), shape.qkv), device="cuda", generator=gen)
        self.qkv = qkv_all[list(mine)].contiguous()
        del qkv_all
        self.angles = torch.from_numpy(
            fa.rotary_angles(fa.Rotation(base=1e6), d, self.lengths)).cuda()
        self.q = torch.zeros((b, shape.width), device="cuda")
        self.out = torch.zeros((b, shape.width), device="cuda")
        self.launches_per_step = 2 * ((b + 255) // 256)
        # a decode step as a serving loop runs it: replayed as a captured CUDA graph (a GPU's
        # share of C3 over 8 GPUs is tens of microseconds, less than the calls' host time)
        self.graphs = True
        # e2e: pinned host inputs and outputs
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_angles = self.angles.cpu().pin_memory()
        self.h_out = torch.zeros_like(self.out, device="cpu").pin_memory()
        self.h2d = self.h_qkv.numel() * 4 + self.h_angles.numel() * 4
        self.d2h = self.h_out.numel() * 4
        esize = 4 if dtype == fa.F32 else 2
        keys = sum(n + 1 for n in self.lengths)
        self.bytes = keys * kv * d * 2 * esize + 2 * b * shape.width * 4

    def phases(self):
        return (lambda: self.batch.attention_input(0, self.qkv, self.q, self.angles,
                                                   self.fa.ROPE_HALF),
                lambda: self.batch.attend(0, self.q, self.out))

    e2e_path = "pinned host rows -> fa_attention_batch_host -> pinned host output"

    e2e_returns_synchronized = True

    def e2e_step(self):
        # fa_attention_batch_host: the copy of the second group of sequences overlaps the first
        # group's attention; returns with h_out filled
        self.batch.attention_host(0, self.h_qkv, self.h_out, self.h_angles, self.fa.ROPE_HALF)

    def parity(self, threads):
        """Every sequence of this rank: the oracle's RoPE + keep of the row into a host copy of
        the sequence's cache, then its attend, against the timed launch's output row; and the
        end-to-end call's host output against the device output."""
        import oracle
        torch, fa = self.torch, self.fa
        out = self.out.cpu().numpy()
        qkv = self.qkv.cpu().numpy()
        angles = self.angles.cpu().numpy()
        bf16 = self.dtype == fa.BF16
        wants = []
        for j, (c, n) in enumerate(zip(self.caches, self.lengths)):
            k, v = c.copy_rows(n)
            oc = oracle.Cache(1, *self.dims, n + 1)
            oc.keys[:, :, :n] = k.float().cpu().numpy()
            oc.values[:, :, :n] = v.float().cpu().numpy()
            del k, v
            q = qkv[j:j + 1].copy()
            oc.attention_input(0, 1, n, fa.ROPE_HALF, angles[j:j + 1], q, q.shape[1])
            if bf16:  # a bf16 cache keeps the new row rounded to nearest
                oc.keys[0, :, n] = round_bf16(torch, oc.keys[0, :, n])
                oc.values[0, :, n] = round_bf16(torch, oc.values[0, :, n])
            wants.append(oc.attend(0, 1, n, oracle.Mask.causal(), q, q.shape[1], threads=threads))
        want = np.concatenate(wants) if wants else np.zeros_like(out)
        p = parity_result(out, want, TOL_BF16 if bf16 else TOL_F32,
                          f"{len(self.lengths)} sequences, every head",
                          REL_BF16 if bf16 else None)
        if self.e2e_ran and out.size:
            p["e2e_vs_device_max_abs"] = sci(np.abs(self.h_out.numpy() - out).max())
        return p

    def algorithmic(self):
        return float(self.bytes)


class SingleDecode(Workload):
    """C1 (14/2, d64, position 1024) and C4 (16/8, d128, position 131072) on one GPU."""

    def __init__(self, torch, fa, name, heads, kv, d, position):
        self.torch, self.fa, self.name = torch, fa, name
        shape = fa.Shape(1, heads, kv, d)
        self.shape = shape
        self.position = position
        self.cache = fa.KvCache(shape, position + 1)
        k, v, self.qkv = decode_inputs(torch, shape, position)
        self.cache.put_rows(k, v)
        del k, v
        self.span = fa.Span(1, position, fa.Mask.causal())
        self.angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), d, [position])).cuda()
        self.q = torch.zeros((1, shape.width), device="cuda")
        self.out = torch.zeros((1, shape.width), device="cuda")
        self.tokens = 1
        self.launches_per_step = 2
        self.flush_l2 = (position + 1) * kv * d * 8 < L2_BYTES
        self.graphs = name == "c1"  # microseconds per step: launch-bound
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_angles = self.angles.cpu().pin_memory()
        self.h_out = torch.zeros_like(self.out, device="cpu").pin_memory()
        self.d_qkv = torch.empty_like(self.qkv)
        self.d_angles = torch.empty_like(self.angles)
        self.h2d = (self.h_qkv.numel() + self.h_angles.numel()) * 4
        self.d2h = self.h_out.numel() * 4
        self.bytes = (position + 1) * kv * d * 2 * 4 + 2 * shape.width * 4

    def phases(self):
        return (lambda: self.cache.attention_input(0, self.span, self.qkv, self.angles,
                                                   self.fa.ROPE_HALF, q_out=self.q),
                lambda: self.cache.attend(0, self.span, self.q, self.out))

    def e2e_step(self):
        self.d_qkv.copy_(self.h_qkv, non_blocking=True)
        self.d_angles.copy_(self.h_angles, non_blocking=True)
        self.cache.attention(0, self.span, self.d_qkv, self.out, self.d_angles, self.fa.ROPE_HALF)
        self.h_out.copy_(self.out, non_blocking=True)

    def parity(self, threads):
        """The whole decode: the oracle's RoPE + keep and attend over a host copy of the cache's
        `position` seeded rows, against the timed output."""
        k, v = self.cache.copy_rows(self.position)
        want = oracle_decode(self.fa, self.shape, self.position, k.cpu().numpy(), v.cpu().numpy(),
                             self.qkv.cpu().numpy(), self.angles.cpu().numpy(), threads)
        p = parity_result(self.out.cpu().numpy(), want, TOL_F32,
                          f"the decode row, {self.position + 1} keys, every head")
        if self.e2e_ran:
            p["e2e_vs_device_max_abs"] = sci(np.abs(self.h_out.numpy() - self.out.cpu().numpy()).max())
        return p

    def algorithmic(self):
        return float(self.bytes)


def decode_inputs(torch, shape, position):
    """C1's and C4's seeded inputs: the cache's `position` keys and values, then the new row's
    qkv, from one generator (the same on every rank, whatever the number of GPUs)."""
    gen = torch.Generator("cuda").manual_seed(7)
    dims = (1, shape.kv_heads, position, shape.head_dim)
    k = torch.randn(dims, device="cuda", generator=gen)
    v = torch.randn(dims, device="cuda", generator=gen)
    qkv = torch.randn((1, shape.qkv), device="cuda", generator=gen)
    return k, v, qkv


def oracle_decode(fa, shape, position, keys, values, qkv, angles, threads):
    """The reference's attention phase of one decode row at `position` on the host: the
    oracle's RoPE + keep into a copy of the cache, then its team-split attend."""
    import oracle
    oc = oracle.Cache(1, shape.heads, shape.kv_heads, shape.head_dim, position + 1)
    oc.keys[:, :, :position] = keys
    oc.values[:, :, :position] = values
    q = np.ascontiguousarray(qkv, np.float32).copy()
    oc.attention_input(0, 1, position, fa.ROPE_HALF, angles, q, q.shape[1])
    return oc.attend(0, 1, position, oracle.Mask.causal(), q, q.shape[1], threads=threads)


class ProjectedInput(Workload):
    """Stack::attention_input with its qkv projection on the device
    (fa_attention_input_projected: projection, RoPE and keep), Llama-8B-shaped: 32/8 heads x
    128, hidden 4096, f32 weights (6144 x 4096, 100.7 MB) and bias, from position 4096. `proj`:
    one decode row (the fused CUDA-core kernel); `proj64`: 64 rows (a batched decode's or a
    prefill chunk's rows: the tensor-core projection in three tf32 products, then the RoPE +
    keep kernel). Roofline against the bytes (weights, input, kept rows, queries); L2 (126 MB)
    flushed between steps."""

    def __init__(self, torch, fa, rows=1):
        self.torch, self.fa = torch, fa
        self.name = "proj" if rows == 1 else f"proj{rows}"
        self.kernel = "project_keep_kernel" if rows < 16 else "project_tc_kernel"
        heads, kv, d, self.hidden, position = 32, 8, 128, 4096, 4096
        self.rows = rows
        shape = fa.Shape(1, heads, kv, d)
        self.cache = fa.KvCache(shape, position + rows)
        gen = torch.Generator("cuda").manual_seed(9)
        self.weight = torch.randn((shape.qkv, self.hidden), device="cuda", generator=gen) / 64.0
        self.bias = torch.randn((shape.qkv,), device="cuda", generator=gen)
        self.x = torch.randn((rows, self.hidden), device="cuda", generator=gen)
        self.span = fa.Span(rows, position, fa.Mask.causal())
        self.angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), d,
                                                        range(position, position + rows))).cuda()
        self.q = torch.zeros((rows, shape.width), device="cuda")
        self.tokens = rows
        self.launches_per_step = 1 if rows < 16 else 2
        self.flush_l2 = True
        self.graphs = True
        self.h_x = self.x.cpu().pin_memory()
        self.h_q = torch.zeros_like(self.q, device="cpu").pin_memory()
        self.h2d = self.h_x.numel() * 4
        self.d2h = self.h_q.numel() * 4
        self.bytes = (self.weight.numel() + self.bias.numel() + self.x.numel()
                      + rows * (2 * kv * d + shape.width)) * 4

    def phases(self):
        return (lambda: None,
                lambda: self.cache.attention_input_projected(
                    0, self.span, self.x, self.weight, self.bias, angles=self.angles,
                    rope=self.fa.ROPE_HALF, q_out=self.q))

    def e2e_step(self):
        self.x.copy_(self.h_x, non_blocking=True)
        self.phases()[1]()
        self.h_q.copy_(self.q, non_blocking=True)

    def parity(self, threads):
        """The rotated queries of the timed launch against the oracle's projection (f64 sums
        rounded to f32) followed by its RoPE + keep; and the kept key and value rows. The
        projection's sums run in another order than the host's, so the bar is relative to the
        magnitude of the projected values (2e-5, the projection tests' bar)."""
        import oracle
        fa = self.fa
        qkv = oracle.project(self.x.cpu().numpy(), self.weight.cpu().numpy(),
                             self.bias.cpu().numpy())
        scale = max(1.0, float(np.abs(qkv).max()))
        first, rows = self.span.first, self.rows
        shape = self.cache.shape
        oc = oracle.Cache(1, shape.heads, shape.kv_heads, shape.head_dim, first + rows)
        oc.attention_input(0, rows, first, fa.ROPE_HALF, self.angles.cpu().numpy(), qkv,
                           qkv.shape[1])
        k, v = self.cache.copy_rows(first + rows)
        kept = slice(first, first + rows)
        got = np.concatenate([self.q.cpu().numpy().ravel(), k[0, :, kept].cpu().numpy().ravel(),
                              v[0, :, kept].cpu().numpy().ravel()])
        want = np.concatenate([qkv[:, :shape.width].ravel(), oc.keys[0, :, kept].ravel(),
                               oc.values[0, :, kept].ravel()])
        return parity_result(got, want, 2e-5 * scale,
                             f"the rotated queries and the kept key and value rows of {rows} row(s)")

    def algorithmic(self):
        return float(self.bytes)


class DitPrologue(Workload):
    """The query/key prologue of C5's DiT block (Wan's normalize_and_rotate, wan_dit/block.rs:
    109-140): 32760 tokens of f32 qkv (12 heads x 128), whole-row RMSNorm of the query and key
    rows, interleaved RoPE by each token's angles, written as the bf16 operand rows the
    full-mask attention reads. HBM-bound: 604 MB read (+ 16.8 MB of angles), 302 MB written."""

    def __init__(self, torch, fa):
        self.torch, self.fa, self.name = torch, fa, "prologue"
        self.kernel = "prologue_kernel"
        self.heads, self.d, self.n = 12, 128, 32760
        hidden = self.heads * self.d
        gen = torch.Generator("cuda").manual_seed(11)
        self.qkv = torch.randn((self.n, 3 * hidden), device="cuda", generator=gen)
        self.out = torch.empty((self.n, 3 * hidden), device="cuda", dtype=torch.bfloat16)
        self.q_norm = 1.0 + 0.1 * torch.randn((hidden,), device="cuda", generator=gen)
        self.k_norm = 1.0 + 0.1 * torch.randn((hidden,), device="cuda", generator=gen)
        self.angles = torch.rand((self.n, self.d), device="cuda", generator=gen)
        self.tokens = self.n
        self.launches_per_step = 1
        self.graphs = True
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_out = torch.empty_like(self.out, device="cpu").pin_memory()
        self.h2d = self.h_qkv.numel() * 4
        self.d2h = self.h_out.numel() * 2
        self.bytes = self.qkv.numel() * 4 + self.out.numel() * 2 + self.angles.numel() * 4

    def phases(self):
        return (lambda: None,
                lambda: self.fa.normalize_and_rotate(self.heads, self.d, self.qkv, self.out,
                                                     self.fa.NORM_ROW, self.q_norm, self.k_norm,
                                                     1e-6, self.angles, self.fa.ROPE_INTERLEAVED))

    def e2e_step(self):
        self.qkv.copy_(self.h_qkv, non_blocking=True)
        self.phases()[1]()
        self.h_out.copy_(self.out, non_blocking=True)

    def parity(self, threads):
        """Every 32nd token (1024 of them) against the oracle's prologue (f32): each bf16 output
        within half a bf16 step of the oracle's f32 value (2^-8 of its magnitude: the output's
        own rounding) plus 1e-5 (the f32 arithmetic's difference, which decides the rounding of
        a value near a rounding boundary, and dominates for values near zero). `worst` is the
        largest ratio of an error to that bound."""
        import oracle
        torch, fa = self.torch, self.fa
        idx = np.arange(0, self.n, 32)
        qkv = self.qkv.cpu().numpy()[idx]
        angles = self.angles.cpu().numpy()[idx]
        want = oracle.qk_prologue(len(idx), self.heads, self.d, fa.NORM_ROW, fa.ROPE_INTERLEAVED,
                                  len(idx), angles, self.q_norm.cpu().numpy(),
                                  self.k_norm.cpu().numpy(), 1e-6, qkv)
        got = self.out.float().cpu().numpy()[idx]
        err = np.abs(got.astype(np.float64) - want)
        worst = float((err / (np.abs(want) * 2.0 ** -8 + 1e-5)).max())
        return {"max_abs": sci(err.max()), "worst": sci(worst), "tol": 1.0,
                "ok": bool(np.isfinite(worst) and worst <= 1.0),
                "checked": f"{len(idx)} of {self.n} tokens, queries, keys and values"}

    def algorithmic(self):
        return float(self.bytes)


class C2Prefill(Workload):
    """C2: 512 rows from position 0, causal, 14/2 heads, d64; the cache written by the pass."""

    def __init__(self, torch, fa):
        self.torch, self.fa, self.name = torch, fa, "c2"
        self.kernel = "fmha_kernel"
        shape = fa.Shape(1, 14, 2, 64)
        self.shape = shape
        self.cache = fa.KvCache(shape, 512)
        gen = torch.Generator("cuda").manual_seed(9)
        self.span = fa.Span(512, 0, fa.Mask.causal())
        self.qkv = torch.randn((512, shape.qkv), device="cuda", generator=gen)
        self.angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), 64, range(512))).cuda()
        self.q = torch.zeros((512, shape.width), device="cuda")
        self.out = torch.zeros((512, shape.width), device="cuda")
        self.tokens = 512
        self.bound = "tensor"
        self.launches_per_step = 2
        self.flush_l2 = True
        self.graphs = True  # tens of microseconds per step: launch-bound
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_angles = self.angles.cpu().pin_memory()
        self.h_out = torch.zeros_like(self.out, device="cpu").pin_memory()
        self.d_qkv = torch.empty_like(self.qkv)
        self.d_angles = torch.empty_like(self.angles)
        self.h2d = (self.h_qkv.numel() + self.h_angles.numel()) * 4
        self.d2h = self.h_out.numel() * 4
        self.flops = 4.0 * 14 * 64 * sum(i + 1 for i in range(512))

    def phases(self):
        return (lambda: self.cache.attention_input(0, self.span, self.qkv, self.angles,
                                                   self.fa.ROPE_HALF, q_out=self.q),
                lambda: self.cache.attend(0, self.span, self.q, self.out))

    def e2e_step(self):
        self.d_qkv.copy_(self.h_qkv, non_blocking=True)
        self.d_angles.copy_(self.h_angles, non_blocking=True)
        self.cache.attention(0, self.span, self.d_qkv, self.out, self.d_angles, self.fa.ROPE_HALF)
        self.h_out.copy_(self.out, non_blocking=True)

    def parity(self, threads):
        """All 512 rows: the oracle's RoPE + keep of the span into an empty cache, then its
        causal attend, against the timed output."""
        import oracle
        fa = self.fa
        oc = oracle.Cache(1, 14, 2, 64, 512)
        q = self.qkv.cpu().numpy().copy()
        oc.attention_input(0, 512, 0, fa.ROPE_HALF, self.angles.cpu().numpy(), q, q.shape[1])
        want = oc.attend(0, 512, 0, oracle.Mask.causal(), q, q.shape[1], threads=threads)
        out = self.out.cpu().numpy()
        p = parity_result(out, want, TOL_F32, "all 512 rows, every head")
        if self.e2e_ran:
            p["e2e_vs_device_max_abs"] = sci(np.abs(self.h_out.numpy() - out).max())
        return p

    def algorithmic(self):
        return self.flops


class LongPrefill(Workload):
    """A long causal prefill at C3's model shape (32/8 heads x 128, RoPE base 1e6): 8192 rows
    from position 0 over a bf16 cache: RoPE + keep (fa_attention_input), then the attention
    (fa_attend: the queries to bf16 operand rows and the tensor-core attention). FLOPs 4 x d x
    heads x the visible keys of every row (0.55 TFLOP) over the attend call's time.
    `prefill_f32`: the same over an f32 cache, the reference's own cache type (transformer.rs:
    134-162), on the tf32 tensor-core kernel (f32 queries, keys and values rounded to tf32 on the
    way in, f32 accumulation); its roofline is against half the bf16 peak, the tensor cores' tf32
    rate (1.1 of 2.25 PFLOP/s nominal, dense)."""

    def __init__(self, torch, fa, dtype=None):
        dtype = fa.BF16 if dtype is None else dtype
        self.torch, self.fa = torch, fa
        self.dtype = dtype
        self.name = "prefill" if dtype == fa.BF16 else "prefill_f32"
        self.kernel = "fmha2_kernel" if dtype == fa.BF16 else "fmha_kernel"
        if dtype == fa.F32:
            self.peak_scale = 0.5
        rows, heads, kv, d = 8192, 32, 8, 128
        shape = fa.Shape(1, heads, kv, d)
        self.cache = fa.KvCache(shape, rows, dtype)
        gen = torch.Generator("cuda").manual_seed(13)
        self.span = fa.Span(rows, 0, fa.Mask.causal())
        self.qkv = torch.randn((rows, shape.qkv), device="cuda", generator=gen)
        self.angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), d, range(rows))).cuda()
        self.q = torch.zeros((rows, shape.width), device="cuda")
        self.out = torch.zeros((rows, shape.width), device="cuda")
        self.tokens = rows
        self.bound = "tensor"
        self.launches_per_step = 3
        self.graphs = True
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_out = torch.zeros_like(self.out, device="cpu").pin_memory()
        self.h2d = self.h_qkv.numel() * 4
        self.d2h = self.h_out.numel() * 4
        self.flops = 4.0 * heads * d * rows * (rows + 1) / 2

    def phases(self):
        # the step as a user runs it: fa_attention (RoPE + keep writing bf16 operand queries,
        # then the tensor-core attention)
        return (lambda: None,
                lambda: self.cache.attention(0, self.span, self.qkv, self.out, self.angles,
                                             self.fa.ROPE_HALF))

    def capture(self):
        """The step graph (fa_attention), and for the roofline the attention alone: fa_attend
        over f32 queries that fa_attention_input rotated once beforehand (its own bf16
        conversion of the queries included)."""
        torch = self.torch
        self._step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._step_graph, capture_error_mode="relaxed"):
            self.phases()[1]()
        self.cache.attention_input(0, self.span, self.qkv, self.angles, self.fa.ROPE_HALF,
                                   q_out=self.q)
        self.cache.attend(0, self.span, self.q, self.out)  # sizes its workspace before capture
        torch.cuda.synchronize()
        self._kernel_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._kernel_graph, capture_error_mode="relaxed"):
            self.cache.attend(0, self.span, self.q, self.out)
        torch.cuda.synchronize()

    def e2e_step(self):
        self.qkv.copy_(self.h_qkv, non_blocking=True)
        self.phases()[1]()
        self.h_out.copy_(self.out, non_blocking=True)

    def parity(self, threads):
        """Sampled rows (the first and last 16, and 32 spread between) against the oracle: its
        RoPE + keep of all 8192 rows into a host cache (the kept rows rounded to bf16, as this
        cache holds them), then its causal attend of each sampled row. A bf16-compute path: the
        queries and probabilities are bf16 on the tensor cores."""
        import oracle
        torch, fa = self.torch, self.fa
        rows, heads, kv, d = 8192, 32, 8, 128
        oc = oracle.Cache(1, heads, kv, d, rows)
        q = self.qkv.cpu().numpy().copy()
        oc.attention_input(0, rows, 0, fa.ROPE_HALF, self.angles.cpu().numpy(), q, q.shape[1])
        bf16 = self.dtype == fa.BF16
        if bf16:
            oc.keys[:] = round_bf16(torch, oc.keys)
            oc.values[:] = round_bf16(torch, oc.values)
        sample = sorted(set(range(16)) | set(range(rows - 16, rows)) |
                        set(np.linspace(16, rows - 17, 32).astype(int).tolist()))
        out = self.out.cpu().numpy()
        want = np.concatenate([oc.attend(0, 1, r, oracle.Mask.causal(), q[r:r + 1], q.shape[1],
                                         threads=threads) for r in sample])
        return parity_result(out[sample], want, TOL_BF16 if bf16 else TOL_F32,
                             f"{len(sample)} of {rows} rows, every head",
                             REL_BF16 if bf16 else None)

    def algorithmic(self):
        return self.flops


class GatedPrefill256(Workload):
    """A long prefill of Qwen3.5's gated attention layer (models/qwen3-5/model/src/model.rs:
    60-75): 8 query heads over 2 KV heads of 256, 64 of each head's dimensions rotated by
    interleaved multimodal RoPE (base 1e7, sections [11, 11, 10]), head RMSNorm, an elementwise
    sigmoid gate; 8192 rows from position 0 over a bf16 cache. The step is fa_gated_attention
    (norm, RoPE and keep, the head_dim-256 tensor-core attention, the gate); the roofline times the
    attention alone (fa_attend over the rotated queries). FLOPs 4 x 256 x 8 x the visible keys of
    every row (0.275 TFLOP)."""

    def __init__(self, torch, fa):
        self.torch, self.fa, self.name = torch, fa, "qwen35"
        self.kernel = "fmha_kernel"
        rows, heads, kv, d = 8192, 8, 2, 256
        self.rows, self.heads, self.kv, self.d = rows, heads, kv, d
        shape = fa.Shape(1, heads, kv, d)
        self.shape = shape
        self.cache = fa.KvCache(shape, rows, fa.BF16)
        gen = torch.Generator("cuda").manual_seed(17)
        self.width = (2 * heads + 2 * kv) * d  # query, gate, key and value heads
        self.qkv = torch.randn((rows, self.width), device="cuda", generator=gen)
        self.q_norm = 1.0 + 0.1 * torch.randn((d,), device="cuda", generator=gen)
        self.k_norm = 1.0 + 0.1 * torch.randn((d,), device="cuda", generator=gen)
        rot = fa.Rotation(fa.ROT_MULTIMODAL_INTERLEAVED, (11, 11, 10), 1e7)
        self.angles = torch.from_numpy(fa.rotary_angles(rot, 64, range(rows))).cuda()
        self.span = fa.Span(rows, 0, fa.Mask.causal())
        self.out = torch.zeros((rows, shape.width), device="cuda")
        self.q = torch.zeros((rows, shape.width), device="cuda")
        self.tokens = rows
        self.bound = "tensor"
        self.launches_per_step = 4
        self.graphs = True
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_out = torch.zeros_like(self.out, device="cpu").pin_memory()
        self.h2d = self.h_qkv.numel() * 4
        self.d2h = self.h_out.numel() * 4
        self.flops = 4.0 * heads * d * rows * (rows + 1) / 2

    def gated(self):
        fa = self.fa
        self.cache.gated_attention(0, self.span, self.qkv, self.out, fa.GATE_ELEMENTWISE, 64,
                                   self.angles, norm=(self.q_norm, self.k_norm, 1e-6))

    def phases(self):
        return (lambda: None, self.gated)

    def capture(self):
        """The step graph (fa_gated_attention), and for the roofline the attention alone: fa_attend
        over the rows' query heads (f32, converted to bf16 operand rows by the call, as the
        step's own queries are; their values do not change the work)."""
        torch = self.torch
        self._step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._step_graph, capture_error_mode="relaxed"):
            self.gated()
        self.q.copy_(self.qkv[:, :self.shape.width])
        self.cache.attend(0, self.span, self.q, self.out)  # sizes its workspace before capture
        torch.cuda.synchronize()
        self._kernel_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._kernel_graph, capture_error_mode="relaxed"):
            self.cache.attend(0, self.span, self.q, self.out)
        torch.cuda.synchronize()

    def e2e_step(self):
        self.qkv.copy_(self.h_qkv, non_blocking=True)
        self.gated()
        self.h_out.copy_(self.out, non_blocking=True)

    def parity(self, threads):
        """Sampled rows of the gated layer's output (the first and last 16, 32 spread between)
        against the oracle: its norm, partial RoPE and keep of all 8192 rows into a host cache
        (the kept rows rounded to bf16, as this cache holds them), its causal attend of each
        sampled row, and the gate. A bf16-compute path."""
        import oracle
        torch, fa = self.torch, self.fa
        self.gated()  # the timed kernel graph overwrote the output with the attention alone
        torch.cuda.synchronize()
        rows, heads, kv, d = self.rows, self.heads, self.kv, self.d
        oc = oracle.Cache(1, heads, kv, d, rows)
        q = self.qkv.cpu().numpy().copy()
        angles = self.angles.cpu().numpy()
        oc.gated_input(0, rows, 0, fa.GATE_ELEMENTWISE, 64, angles, q, self.width,
                       self.q_norm.cpu().numpy(), self.k_norm.cpu().numpy(), 1e-6)
        oc.keys[:] = round_bf16(torch, oc.keys)
        oc.values[:] = round_bf16(torch, oc.values)
        sample = sorted(set(range(16)) | set(range(rows - 16, rows)) |
                        set(np.linspace(16, rows - 17, 32).astype(int).tolist()))
        got = self.out.cpu().numpy()[sample]
        want = []
        for r in sample:
            att = oc.attend(0, 1, r, oracle.Mask.causal(), q[r:r + 1], self.width, threads=threads)
            want.append(oracle.gate(1, heads, kv, d, fa.GATE_ELEMENTWISE, q[r:r + 1], att))
        return parity_result(got, np.concatenate(want), TOL_BF16,
                             f"{len(sample)} of {rows} rows, every head", REL_BF16)

    def algorithmic(self):
        return self.flops


class C4Sharded(Workload):
    """C4 over `world` GPUs: each rank holds a contiguous range of the 131073 key positions in
    its own cache; a step rotates the query everywhere, keeps the new row on its owner, attends
    the local range into per-head (max, sum, o), and one kernel stores those into every rank's
    exchange buffer over NVLink peer memory, waits for every rank's and merges them."""

    def __init__(self, torch, fa, rank, world, dist):
        from fusor_attn.shard import ShardedDecode, kv_shards
        self.torch, self.fa, self.dist, self.name = torch, fa, dist, "c4"
        self.sharded = True
        heads, kv, d, position = 16, 8, 128, 131072
        lo, hi = kv_shards(position + 1, world)[rank]
        shape = fa.Shape(1, heads, kv, d)
        self.shape, self.position, self.rank = shape, position, rank
        self.cache = fa.KvCache(shape, hi - lo)
        # the 1-GPU decode's inputs (one seeded stream), this rank's range of positions kept
        k, v, self.qkv = decode_inputs(torch, shape, position)
        filled = min(hi, position) - lo  # the new row's slot is kept by the step
        self.cache.put_rows(k[:, :, lo:lo + filled].contiguous(), v[:, :, lo:lo + filled].contiguous())
        del k, v
        self.angles = torch.from_numpy(fa.rotary_angles(fa.Rotation(base=1e6), d, [position])).cuda()
        self.decode = ShardedDecode(self.cache, heads, d, lo, hi, position, world,
                                    exchange="peer")
        self.tokens = 1
        self.launches_per_step = 3
        # a step is tens of microseconds on the GPU, less than its calls' host time: the whole
        # step (the exchange of the partials included) is replayed as one captured CUDA graph
        self.graphs = True
        self.bytes = (hi - lo) * kv * d * 2 * 4
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_angles = self.angles.cpu().pin_memory()
        self.h_out = torch.zeros((heads, d), device="cpu").pin_memory()
        self.h2d = (self.h_qkv.numel() + self.h_angles.numel()) * 4
        self.d2h = self.h_out.numel() * 4

    def capture(self):
        """The step (rotate, attend the local range, exchange and merge) as one CUDA graph, and
        the local attend alone as another (the dominant kernel's timing). Every rank captures
        the same collectives in the same order, after warm-up has created the communicator."""
        torch = self.torch
        self._step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._step_graph, capture_error_mode="relaxed"):
            self.decode.step(self.qkv, self.angles, self.fa.ROPE_HALF, self.dist)
        self._kernel_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._kernel_graph, capture_error_mode="relaxed"):
            self.decode.attend_local()
        torch.cuda.synchronize()

    def step(self, mid=None):
        if self._step_graph is not None:
            self._step_graph.replay()
            return
        if mid is not None:
            mid.record()
        self.decode.step(self.qkv, self.angles, self.fa.ROPE_HALF, self.dist)

    def e2e_step(self):
        self.qkv.copy_(self.h_qkv, non_blocking=True)
        self.angles.copy_(self.h_angles, non_blocking=True)
        out = self.decode.step(self.qkv, self.angles, self.fa.ROPE_HALF, self.dist)
        self.h_out.copy_(out, non_blocking=True)

    def phases_us(self, steps):
        """The step's three phases timed apart (each captured as its own CUDA graph and replayed
        `steps` times back to back between two events; the max over ranks, in microseconds): the
        query's RoPE (+ the keep on the owner), the local range's attention, and the exchange of
        the partials with the merge (which includes any wait for a slower rank)."""
        torch, fa, dist = self.torch, self.fa, self.dist
        calls = (("rotate_keep", lambda: self.decode.rotate(self.qkv, self.angles, fa.ROPE_HALF)),
                 ("attend_local", self.decode.attend_local),
                 ("exchange_merge", lambda: self.decode.gather_merge(dist)))
        out = {}
        for name, call in calls:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="relaxed"):
                call()
            g.replay()
            torch.cuda.synchronize()
            dist.barrier()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(steps):
                g.replay()
            end.record()
            torch.cuda.synchronize()
            t = torch.tensor([start.elapsed_time(end) * 1e3 / steps], device="cuda",
                             dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[name] = round(float(t[0]), 2)
            del g  # a graph holding the exchange goes before the peer buffers
        self.decode.recover(dist)
        return out

    def parity(self, threads):
        """The merged output of the timed steps: rank 0 against the oracle's decode of the whole
        131073-key context (the seeded inputs made again on its device), and every rank's merged
        output against rank 0's (they merge the same partials in the same order: equal bits)."""
        torch, dist = self.torch, self.dist
        out = self.decode.out.reshape(1, -1).clone()
        first = out.clone()
        dist.broadcast(first, 0)
        same = bool(torch.equal(out, first))
        p = {"checked": "the merged decode row on rank 0, every head; every rank's merged row "
                        "against rank 0's", "ok": same}
        if self.rank == 0:
            k, v, _ = decode_inputs(torch, self.shape, self.position)
            want = oracle_decode(self.fa, self.shape, self.position, k.cpu().numpy(),
                                 v.cpu().numpy(), self.qkv.cpu().numpy(),
                                 self.angles.cpu().numpy(), threads)
            del k, v
            p.update(parity_result(out.cpu().numpy(), want, TOL_F32, p["checked"]))
            p["ok"] = p["ok"] and same
        p["ranks_agree"] = same
        if self.e2e_ran:
            p["e2e_vs_device_max_abs"] = sci(np.abs(self.h_out.numpy().reshape(1, -1)
                                                    - out.cpu().numpy()).max())
        return p

    def algorithmic(self):
        return float(self.bytes)

    def close(self):
        super().close()  # the graphs that hold the exchange go first
        self.decode.close(self.dist)


class C5Full(Workload):
    """C5: DiT full-mask self-attention, 32760 tokens, 12 heads x 128, bf16 in / f32 accumulate,
    bf16 out; the query rows split over the ranks in whole 256-row pairs, one call per rank
    over all heads (the keys and values whole on every rank)."""

    def __init__(self, torch, fa, rank, world):
        from fusor_attn.shard import query_row_shards
        self.torch, self.fa, self.name = torch, fa, "c5"
        self.sharded = True
        self.kernel = "fmha2_kernel"  # bf16: two query tiles per CTA
        self.heads, self.d, self.n = 12, 128, 32760
        hidden = self.heads * self.d
        gen = torch.Generator("cuda").manual_seed(5)
        self.qkv = torch.randn((self.n, 3 * hidden), device="cuda", generator=gen).to(torch.bfloat16)
        self.out = torch.empty((self.n, hidden), device="cuda", dtype=torch.bfloat16)
        self.lo, self.hi = query_row_shards(self.n, world)[rank]
        self.tokens = self.n
        self.bound = "tensor"
        self.launches_per_step = 1 if self.hi > self.lo else 0
        self.flops = 4.0 * self.d * (self.hi - self.lo) * self.n * self.heads
        self.stride = 3 * hidden
        # e2e: the whole qkv from pinned host memory, this rank's output rows back
        self.h_qkv = self.qkv.cpu().pin_memory()
        self.h_out = torch.empty_like(self.out, device="cpu").pin_memory()
        self.h2d = self.h_qkv.numel() * 2
        self.d2h = (self.hi - self.lo) * hidden * 2

    def step(self, mid=None):
        fa, d, stride, lo, hi = self.fa, self.d, self.stride, self.lo, self.hi
        if mid is not None:
            mid.record()
        if hi > lo:
            fa.attend_full(self.heads, self.heads, d, 1, hi - lo, self.n,
                           fa.Operand(self.qkv, stride, lo * stride),
                           fa.Operand(self.qkv, stride, self.heads * d),
                           fa.Operand(self.qkv, stride, 2 * self.heads * d),
                           self.out[lo:hi])

    def e2e_step(self):
        self.qkv.copy_(self.h_qkv, non_blocking=True)
        self.step()
        self.h_out[self.lo:self.hi].copy_(self.out[self.lo:self.hi], non_blocking=True)

    def sample_rows(self):
        """This rank's checked query rows: its first and last 32 and 64 spread between (every
        head of each), so that whole units, the last wave's split units and the ragged last
        query tile are all sampled."""
        lo, hi = self.lo, self.hi
        if hi <= lo:
            return []
        spread = np.linspace(lo, hi - 1, 64).astype(int).tolist()
        return sorted(set(range(lo, min(lo + 32, hi))) | set(range(max(hi - 32, lo), hi)) | set(spread))

    def parity(self, threads):
        """Sampled query rows of this rank's share of the timed call (bf16 output) against the
        oracle's f32 full-mask attention over the same bf16 queries, keys and values (every one of
        the 32760 keys)."""
        import oracle
        rows = self.sample_rows()
        if not rows:
            return {"checked": "no rows on this rank", "ok": True}
        qkv = self.qkv.float().cpu().numpy()
        hidden = self.heads * self.d
        want = np.zeros((self.n, hidden), np.float32)
        runs, start = [], rows[0]
        for a, b in zip(rows, rows[1:] + [None]):
            if b != a + 1:
                runs.append((start, a + 1))
                start = b
        for qb, qe in runs:
            oracle.attend_call(self.heads, self.heads, self.d, 1, self.n, self.n, qkv, self.stride,
                               0, qkv, self.stride, hidden, qkv, self.stride, 2 * hidden,
                               query_range=(qb, qe), threads=threads, out=want)
        got = self.out.float().cpu().numpy()[rows]
        p = parity_result(got, want[rows], TOL_BF16,
                          f"{len(rows)} of this rank's {self.hi - self.lo} query rows, every head",
                          REL_BF16)
        if self.e2e_ran:
            p["e2e_vs_device_max_abs"] = sci(np.abs(self.h_out[self.lo:self.hi].float().numpy()
                                                    - self.out[self.lo:self.hi].float().cpu().numpy()).max())
        return p

    def algorithmic(self):
        return self.flops


class L2Flush:
    """Evicts L2 between timed steps, outside the timed events: a write of a buffer twice L2's
    size, then a read of another one as large, so that the lines left in L2 are clean and the
    timed step does not pay for writing the flush's own data back to HBM."""

    def __init__(self, torch):
        n = L2_BYTES * 2 // 4
        self.dirty = torch.empty(n, dtype=torch.float32, device="cuda")
        self.clean = torch.zeros(n, dtype=torch.float32, device="cuda")

    def __call__(self, i):
        self.dirty.fill_(float(i))
        self.clean.amax()


def time_workload(torch, dist, w: Workload, steps: int, warmup: int, sampler=None):
    """W untimed steps, then exactly K timed steps between barrier + synchronize, CUDA events
    per step around the pass and around the dominant kernel; the max over ranks."""
    flush = L2Flush(torch) if w.flush_l2 else None
    for _ in range(warmup):
        w.step()
    if w.graphs:
        w.capture()
        w.step()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ctx = sampler if sampler is not None else _null()
    with ctx:
        for i in range(steps):
            if flush is not None:
                flush(i)  # evicts L2 between steps, outside the timed events
            starts[i].record()
            w.step(mids[i])
            ends[i].record()
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if w._kernel_graph is not None:
        # the dominant kernel alone, replayed the same way (the step graph has no event inside)
        torch.cuda.synchronize()
        for i in range(steps):
            if flush is not None:
                flush(i)
            starts[i].record()
            w._kernel_graph.replay()
            ends[i].record()
        torch.cuda.synchronize()
        kern_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    else:
        kern_ms = sum(m.elapsed_time(e) for m, e in zip(mids, ends))
    t = torch.tensor([step_ms, kern_ms], device="cuda", dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]) / steps, float(t[1]) / steps


def time_e2e(torch, dist, w: Workload, steps: int, warmup: int):
    """Wall clock per step through the public API: H2D of the step's inputs from pinned host
    memory, the attention, D2H of the output, synchronized. Returns the mean over the steps
    (the reported value) and the median step, each the max over ranks. The warm-up is at least
    20 steps: the first host-memory calls of a process page in and grow their staging."""
    w.e2e_ran = True
    for _ in range(max(warmup, 20)):
        w.e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    times = []
    # a step whose call returns with the host output filled (it synchronizes its own streams)
    # needs no synchronize after it; every other step gets one
    sync_each = not w.e2e_returns_synchronized
    t0 = time.perf_counter()
    for _ in range(steps):
        a = time.perf_counter()
        w.e2e_step()
        if sync_each:
            torch.cuda.current_stream().synchronize()
        times.append(time.perf_counter() - a)
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3 / steps
    med = sorted(times)[len(times) // 2] * 1e3
    t = torch.tensor([ms, med], device="cuda", dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]), float(t[1])


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ---------------------------------------------------------------------------------------------
# parity of the timed outputs: the oracle (oracle/, test infrastructure) is the checker here,
# run after the timed region on the host; it is never what is timed
# ---------------------------------------------------------------------------------------------

def sci(x) -> float | str:
    """A JSON-safe figure with 3 significant digits ("non-finite" for NaN or infinity)."""
    x = float(x)
    return float(f"{x:.3e}") if np.isfinite(x) else "non-finite"


def round_bf16(torch, a):
    """f32 values rounded to the nearest bf16 (ties to even), as f32: ops::round_bf16."""
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def parity_result(got, want, tol, checked, rel_tol=None):
    """harness::parity's figures (max abs, relative L2) of `got` against the oracle's `want`,
    within the max abs bar `tol` (and the relative L2 bar `rel_tol` of a bf16-compute path)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if got.size == 0:
        return {"max_abs": 0.0, "rel_l2": 0.0, "tol": tol, "ok": True, "checked": checked}
    diff = got - want
    err = float(np.abs(diff).max())
    rel = float(np.sqrt((diff ** 2).sum() / max((want ** 2).sum(), 1e-300)))
    ok = bool(np.isfinite(err) and err <= tol and (rel_tol is None or rel <= rel_tol))
    out = {"max_abs": sci(err), "rel_l2": sci(rel), "tol": tol, "ok": ok, "checked": checked}
    if rel_tol is not None:
        out["rel_tol"] = rel_tol
    return out


def merge_parity(dist, p):
    """Every rank's parity of its share, gathered to one figure: the worst max abs and relative
    L2, the ranks' checked counts side by side, ok only if every rank's is."""
    if dist is None or p is None:
        return p
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, p)
    merged = {"ok": all(bool(q.get("ok", False)) for q in parts),
              "per_rank_checked": [q.get("checked") for q in parts]}
    for key in ("max_abs", "rel_l2", "worst", "e2e_vs_device_max_abs"):
        vals = [q[key] for q in parts if key in q]
        if vals:
            merged[key] = "non-finite" if any(isinstance(v, str) for v in vals) else max(vals)
    for key in ("tol", "rel_tol"):
        vals = [q[key] for q in parts if key in q]
        if vals:
            merged[key] = vals[0]
    vals = [q["ranks_agree"] for q in parts if "ranks_agree" in q]
    if vals:
        merged["ranks_agree"] = all(vals)
    return merged


def roofline(w: Workload, kern_ms: float, peaks, clocks=None):
    """The dominant kernel against the measured peak: the burst figure (`frac`); for a tensor
    kernel whose timed loop ran under the power cap (the clocks saw sw_power_cap), also against
    the sustained figure, measured the same way (`frac_sustained`)."""
    hbm, tflops, kind, sustained = peaks
    extra = {}
    if w.bound == "hbm":
        achieved = w.algorithmic() / (kern_ms * 1e-3) / 1e9
        peak, unit = hbm, "GB/s"
    else:
        achieved = w.algorithmic() / (kern_ms * 1e-3) / 1e12
        peak, unit = tflops, "TFLOP/s"
        scale = getattr(w, "peak_scale", 1.0)
        if scale != 1.0:  # tf32: half the bf16 rate
            peak, kind = peak * scale, f"{kind} bf16 x {scale} (tf32)"
            sustained *= scale
        if clocks is not None and "sw_power_cap" in clocks.get("reasons", []):
            extra = {"peak_sustained": round(sustained, 2),
                     "frac_sustained": round(achieved / sustained, 4)}
    return {"bound": w.bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "peak_source": kind, **extra,
            "traffic": profile_traffic(w.name), "kernel": getattr(w, "kernel", "attend_kernel"),
            "algorithmic_per_launch": w.algorithmic()}


def cpu_baseline_c3(threads: int, budget_s: float = 20.0):
    """The oracle's team-split decode of C3 sequences on the host (the reference's CPU path),
    on a bounded sample: 8 of the 64 sequences, evenly spaced by length."""
    import oracle
    lengths = c3_lengths()
    order = np.argsort(lengths)
    sample = [int(i) for i in order[4::8]]
    rng = np.random.default_rng(5)
    caches, firsts = [], []
    for i in sample:
        n = int(lengths[i])
        c = oracle.Cache(1, C3_HEADS, C3_KV, C3_D, n + 1)
        c.keys[:] = rng.standard_normal(c.keys.shape, dtype=np.float32)
        c.values[:] = rng.standard_normal(c.values.shape, dtype=np.float32)
        caches.append(c)
        firsts.append(n)
    qkv = rng.standard_normal((len(sample), (C3_HEADS + 2 * C3_KV) * C3_D), dtype=np.float32)
    mask = oracle.Mask.causal()

    def one_pass():
        for j, c in enumerate(caches):
            c.attend(0, 1, firsts[j], mask, qkv[j:j + 1], qkv.shape[1], threads=threads)

    one_pass()  # warm-up (harness::bench::time's one warm-up call)
    t0 = time.perf_counter()
    passes = 0
    while True:
        one_pass()
        passes += 1
        if time.perf_counter() - t0 > budget_s / 4 or passes >= 20:
            break
    dt = (time.perf_counter() - t0) / passes
    oracle.release()
    return len(sample) / dt, {
        "sample": f"{len(sample)} of the 64 C3 sequences (every 8th by length, mean "
                  f"{np.mean([lengths[i] for i in sample]):.0f} keys vs {np.mean(lengths):.0f}), "
                  f"one forward call each, heads split over the thread team; mean of {passes} passes"}


def _mean_seconds(call, budget_s):
    """One warm-up call, then the mean of up to 20 calls within about budget_s (the shape of
    harness::bench::time: a warm-up, then the mean of N calls)."""
    call()
    t0 = time.perf_counter()
    n = 0
    while True:
        call()
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 20:
            break
    return (time.perf_counter() - t0) / n, n


def cpu_baselines_other(threads: int, budget_s: float = 4.0):
    """The oracle's C++ restatement of the reference's CPU path timed on the host for C1, C2 and
    C4 (whole configs: RoPE and keep of the span, then the team-split attend) and for a slice of
    C5's f32 full-mask attention (12 heads x 16 query rows against all 32760 keys, scaled to the
    whole call by the query count), seeded N(0,1) inputs. Returns {config: cpu_baseline}."""
    import oracle
    rng = np.random.default_rng(11)
    out = {}

    def decode_or_prefill(name, heads, kv, d, first, rows):
        cache = oracle.Cache(1, heads, kv, d, first + rows)
        rng.standard_normal(cache.keys.shape, dtype=np.float32, out=cache.keys)
        rng.standard_normal(cache.values.shape, dtype=np.float32, out=cache.values)
        stride = (heads + 2 * kv) * d
        qkv0 = rng.standard_normal((rows, stride), dtype=np.float32)
        angles = oracle.angles_table(oracle.ROT_SEQUENCE, 1e6, d, range(first, first + rows))
        mask = oracle.Mask.causal()

        def call():
            qkv = qkv0.copy()
            cache.attention_input(0, rows, first, 1, angles, qkv, stride)
            cache.attend(0, rows, first, mask, qkv, stride, threads=threads)

        t, n = _mean_seconds(call, budget_s)
        out[name] = {"value": round(rows / t, 3), "unit": "tokens/s", "cores": threads,
                     "kind": "port", "ms_per_call": round(t * 1e3, 3),
                     "sample": f"the whole config: RoPE + keep of {rows} row(s) at position "
                               f"{first}, then the attend with heads split over the thread team; "
                               f"mean of {n} calls"}
        del cache

    decode_or_prefill("c1", 14, 2, 64, 1024, 1)
    decode_or_prefill("c2", 14, 2, 64, 0, 512)
    decode_or_prefill("c4", 16, 8, 128, 131072, 1)

    tokens, heads, d, sampled = 32760, 12, 128, 16
    width = heads * d
    k = rng.standard_normal((tokens, width), dtype=np.float32)
    v = rng.standard_normal((tokens, width), dtype=np.float32)
    q = rng.standard_normal((sampled, width), dtype=np.float32)
    res = np.zeros((sampled, width), np.float32)

    def slice_call():
        oracle.attend_call(heads, heads, d, 1, sampled, tokens, q, width, 0, k, width, 0,
                           v, width, 0, query_range=(0, sampled), threads=threads, out=res)

    t, n = _mean_seconds(slice_call, budget_s)
    whole = t * tokens / sampled
    out["c5"] = {"value": round(tokens / whole, 3), "unit": "tokens/s", "cores": threads,
                 "kind": "port", "tflops": round(6.594e12 / whole / 1e12, 5),
                 "ms_per_call": round(whole * 1e3, 1),
                 "sample": f"f32 full mask (dit::Within, ops::attend): {heads} heads x {sampled} "
                           f"query rows against all {tokens} keys, mean of {n} calls, scaled "
                           f"linearly by {tokens}/{sampled} to the whole call"}
    oracle.release()
    return out


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def harness_pool(cores: int) -> int:
    """harness::threads' default pool (crates/harness/src/lib.rs:35-43): min(8, cores - 2), at
    least 1 -- the thread team the reference's own benches run on."""
    return max(1, min(8, cores - 2))


def cpu_baseline_both():
    """C3's CPU baseline timed twice: at the reference harness's own pool size and at every host
    thread the team can use (its head split caps it at the 32 query heads); `value` is the
    latter, as the reference arm runs. The host is named, since the figure moves with it."""
    cores = host_threads()
    pool = harness_pool(cores)
    everything = min(cores, C3_HEADS)
    v_pool, meta = cpu_baseline_c3(pool)
    v_all, meta_all = cpu_baseline_c3(everything) if everything != pool else (v_pool, meta)
    return {"value": round(v_all, 3), "unit": "tokens/s", "cores": everything, "kind": "port",
            "sample": meta_all["sample"], "cpu_model": cpu_model(), "nproc": cores,
            "harness_pool": {"value": round(v_pool, 3), "cores": pool,
                             "rule": "min(8, cores - 2), harness::threads"}}


def summary_entry(ms, roof, parity):
    err = None
    if parity is not None:
        err = parity.get("max_abs")
    return [round(ms, 4), roof["frac"], err]


def run_ours(args):
    import torch
    import torch.distributed as distmod

    import fusor_attn as fa

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        distmod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                   device_id=torch.device("cuda", local))
        dist = distmod
    fa.lib()
    peaks = measured_peaks()
    steps, warmup = args.steps, max(args.warmup, 3)

    def build(name):
        if name in ("c3", "c3bf16"):
            return C3Decode(torch, fa, rank, world, fa.F32 if name == "c3" else fa.BF16,
                            args.sequences)
        if name == "decode256":
            return C3Decode(torch, fa, rank, world, fa.BF16, args.sequences, dims=(8, 2, 256),
                            name="decode256")
        if name == "c1":
            return SingleDecode(torch, fa, "c1", 14, 2, 64, 1024)
        if name == "c4":
            if world > 1:
                return C4Sharded(torch, fa, rank, world, dist)
            return SingleDecode(torch, fa, "c4", 16, 8, 128, 131072)
        if name == "c5":
            return C5Full(torch, fa, rank, world)
        if name == "c2":
            return C2Prefill(torch, fa)
        if name == "proj":
            return ProjectedInput(torch, fa)
        if name == "proj64":
            return ProjectedInput(torch, fa, rows=64)
        if name == "prologue":
            return DitPrologue(torch, fa)
        if name == "prefill":
            return LongPrefill(torch, fa)
        if name == "prefill_f32":
            return LongPrefill(torch, fa, fa.F32)
        if name == "qwen35":
            return GatedPrefill256(torch, fa)
        raise SystemExit(f"unknown config {name}")

    # the oracle's threads for the parity checks: the host's, shared by the ranks
    check_threads = max(1, min(host_threads() // world, C3_HEADS))

    def check(x):
        if args.no_parity:
            return None
        return merge_parity(dist, x.parity(check_threads))

    w = build(args.config)
    sampler = ClockSampler(torch, local)
    ms, kern_ms = time_workload(torch, dist, w, steps, warmup, sampler)
    clocks = sampler.report()
    fa.device_status()
    e2e_ms, e2e_median_ms = time_e2e(torch, dist, w, min(steps, 200), warmup)
    parity = check(w)
    job_tokens = w.tokens if w.sharded else w.tokens * world
    value = job_tokens / (ms * 1e-3)
    line = {
        "metric": f"{args.config} attention tokens/s (decode attn HBM GB/s & prefill TFLOP/s as roofline)",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if w.sharded else "weak", "vs_baseline": None,
        "dtype": {"c3bf16": "bf16-kv/f32", "decode256": "bf16-kv/f32", "c5": "bf16/f32-acc",
                  "prefill": "bf16-kv/f32",
                  "qwen35": "bf16-kv/f32", "prefill_f32": "f32 (tf32 tensor cores)",
                  "prologue": "f32-in/bf16-out"}.get(args.config, "f32"),
        "data": "synthetic N(0,1) (seeded), random keys/values of the config's shape",
        "config": config_of(args.config, world),
        "roofline": roofline(w, kern_ms, peaks, clocks),
        "e2e": {"value": round(job_tokens / (e2e_ms * 1e-3), 2),
                "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                "median_ms_per_step": round(e2e_median_ms, 4),
                "h2d_bytes_per_step": w.h2d, "d2h_bytes_per_step": w.d2h,
                "path": getattr(w, "e2e_path", "pinned host rows -> H2D copy, the step's calls, "
                                                "D2H copy -> pinned host output")},
        "gpu_launches": w.launches_per_step * steps,
        "clocks": clocks,
    }
    if parity is not None:
        line["parity"] = parity
    summary = {args.config: summary_entry(ms, line["roofline"], parity)}
    w.close()
    del w
    torch.cuda.empty_cache()
    if args.config == "c3" and not args.no_extras and args.sequences == C3_SEQS:
        extras = {}
        names = (("c1", "c2", "c3bf16", "decode256", "c4", "c5", "prefill", "prefill_f32", "qwen35",
                  "proj", "proj64", "prologue") if world == 1 else ("c4", "c5"))
        for name in names:
            x = build(name)
            xs = min(steps, 50 if name == "c5" else 200)
            sx = ClockSampler(torch, local)
            ms_x, kern_x = time_workload(torch, dist, x, xs, warmup, sx)
            clocks_x = sx.report()
            # replicas (c1, c2) run the whole config on every rank; the sharded ones split it
            tokens = x.tokens if x.sharded else x.tokens * world
            entry = {"tokens_per_s": round(tokens / (ms_x * 1e-3), 2),
                     "ms_per_step": round(ms_x, 5), "steps": xs,
                     "config": config_of(name, world),
                     "roofline": roofline(x, kern_x, peaks, clocks_x), "clocks": clocks_x,
                     "l2": "flushed between steps (clean lines left)" if x.flush_l2 else "inputs larger than L2"}
            if x.graphs:
                entry["launch"] = "each call of the step replayed as a captured CUDA graph"
            if name == "c5":
                entry["tflops"] = round(6.594e12 / (ms_x * 1e-3) / 1e12, 2)
            if hasattr(x, "phases_us"):
                entry["phases_us"] = x.phases_us(xs)
            px = check(x)
            if px is not None:
                entry["parity"] = px
            extras[name] = entry
            summary[name] = summary_entry(ms_x, entry["roofline"], px)
            x.close()  # graphs holding collectives and peer buffers go before the group
            del x
            torch.cuda.empty_cache()
        line["configs"] = extras
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config.startswith("c3") \
            and args.sequences == C3_SEQS:
        line["cpu_baseline"] = cpu_baseline_both()
        if args.cpu_baselines and "configs" in line:
            threads = min(host_threads(), C3_HEADS)
            for name, base in cpu_baselines_other(threads).items():
                if name in line["configs"]:
                    line["configs"][name]["cpu_baseline"] = base
    fa.device_status()
    # last, so that a reader of the line's tail sees every config: [ms per step, roofline
    # fraction, parity (max abs error against the oracle)]
    line["summary"] = summary
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def config_of(name, world):
    cfgs = {
        "c3": {"workload": "C3 batched GQA decode", "sequences": 64, "heads": 32, "kv_heads": 8,
               "head_dim": 128, "cache_lengths": "U[512, 8192] seed 301", "mask": "causal",
               "kv_dtype": "f32", "rope_base": 1e6},
        "c3bf16": {"workload": "C3 batched GQA decode, bf16 cache", "sequences": 64, "heads": 32,
                   "kv_heads": 8, "head_dim": 128, "kv_dtype": "bf16"},
        "decode256": {"workload": "C3's 64 sequences at Qwen3.5's gated layers' shape, bf16 cache "
                      "(tensor-core decode, head_dim 256 in two halves)", "sequences": 64,
                      "heads": 8, "kv_heads": 2, "head_dim": 256, "kv_dtype": "bf16",
                      "cache_lengths": "U[512, 8192] seed 301"},
        "c1": {"workload": "C1 Qwen2-0.5B decode", "heads": 14, "kv_heads": 2, "head_dim": 64,
               "position": 1024, "mask": "causal"},
        "c2": {"workload": "C2 Qwen2-0.5B prefill", "rows": 512, "heads": 14, "kv_heads": 2,
               "head_dim": 64, "mask": "causal"},
        "c4": {"workload": "C4 long-context decode", "keys": 131073, "heads": 16, "kv_heads": 8,
               "head_dim": 128},
        "c5": {"workload": "C5 DiT full-mask self-attention", "tokens": 32760, "heads": 12,
               "head_dim": 128, "dtype": "bf16 in, f32 accumulate, bf16 out", "mask": "full"},
        "prefill": {"workload": "long causal prefill at C3's model shape, bf16 cache",
                    "rows": 8192, "heads": 32, "kv_heads": 8, "head_dim": 128, "mask": "causal",
                    "path": "fa_attention (step); roofline over an fa_attend call alone"},
        "prefill_f32": {"workload": "long causal prefill at C3's model shape, f32 cache (tf32)",
                        "rows": 8192, "heads": 32, "kv_heads": 8, "head_dim": 128,
                        "mask": "causal",
                        "path": "fa_attention (step); roofline over an fa_attend call alone"},
        "qwen35": {"workload": "Qwen3.5 gated attention layer, long prefill, bf16 cache",
                   "rows": 8192, "heads": 8, "kv_heads": 2, "head_dim": 256, "rotary_dim": 64,
                   "rotation": "MultimodalInterleaved [11, 11, 10], base 1e7", "gate": "elementwise",
                   "head_norm": "rms", "mask": "causal",
                   "path": "fa_gated_attention (step); roofline over an fa_attend call alone"},
        "prologue": {"workload": "C5's DiT query/key prologue (RMSNorm + 3-D RoPE, bf16 out)",
                     "tokens": 32760, "heads": 12, "head_dim": 128, "norm": "whole row",
                     "rope": "interleaved"},
        "proj": {"workload": "attention input with its qkv projection (fused), one decode row",
                 "heads": 32, "kv_heads": 8, "head_dim": 128, "hidden": 4096,
                 "weights": "f32 6144 x 4096 + bias", "position": 4096},
        "proj64": {"workload": "attention input with its qkv projection, 64 rows (tensor cores, "
                   "three tf32 products, then RoPE + keep)",
                   "rows": 64, "heads": 32, "kv_heads": 8, "head_dim": 128, "hidden": 4096,
                   "weights": "f32 6144 x 4096 + bias", "first": 4096},
    }
    c = dict(cfgs[name])
    c["parallelism"] = {
        "c3": f"sequences over {world} GPU(s), no collective",
        "c3bf16": f"sequences over {world} GPU(s), no collective",
        "decode256": f"sequences over {world} GPU(s), no collective",
        "c4": (f"KV range over {world} GPU(s); (max, sum, o) exchanged over NVLink peer memory "
               "by one kernel (P2P stores of step-stamped words) that merges" if world > 1
               else "1 GPU"),
        "c5": f"query rows in whole 256-row pairs over {world} GPU(s), all heads, no collective",
    }.get(name, f"replicas x{world}")
    c["l2"] = ("inputs larger than L2" if name in ("c3", "c3bf16", "decode256", "c4", "c5",
                                                   "prologue", "prefill",
                                                   "prefill_f32", "qwen35")
               else "L2 flushed between steps (clean lines left)")
    if name in ("c1", "c2", "c3", "c3bf16", "decode256", "proj", "proj64", "prologue", "prefill",
                "prefill_f32",
                "qwen35") or \
            (name == "c4" and world > 1):
        c["launch"] = "the step's calls replayed as captured CUDA graphs"
    return c


# ---------------------------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------------------------

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    if not args.config.startswith("c3"):
        print(json.dumps({"impl": "reference", "unavailable": "reference arm implemented for c3"}))
        return
    import oracle
    threads = min(host_threads(), C3_HEADS)
    lengths = c3_lengths()
    order = np.argsort(lengths)
    sample = [int(i) for i in order[4::8]]
    rng = np.random.default_rng(5)
    caches = []
    for i in sample:
        n = int(lengths[i])
        c = oracle.Cache(1, C3_HEADS, C3_KV, C3_D, n + 1)
        c.keys[:] = rng.standard_normal(c.keys.shape, dtype=np.float32)
        c.values[:] = rng.standard_normal(c.values.shape, dtype=np.float32)
        caches.append((c, n))
    qkv = rng.standard_normal((len(sample), (C3_HEADS + 2 * C3_KV) * C3_D), dtype=np.float32)
    mask = oracle.Mask.causal()

    def step():
        for j, (c, n) in enumerate(caches):
            c.attend(0, 1, n, mask, qkv[j:j + 1], qkv.shape[1], threads=threads)

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    ms = (time.perf_counter() - t0) * 1e3 / args.steps
    oracle.release()
    value = len(sample) / (ms * 1e-3)
    sample_desc = (f"each step {len(sample)} of the 64 C3 sequences (every 8th by length), one "
                   f"forward call each, heads split over {threads} threads")
    config = config_of("c3", 1)
    config.pop("launch", None)
    config["parallelism"] = f"the host's thread team ({threads} threads), no GPU"

    print(json.dumps({
        "impl": "reference", "metric": "c3 attention tokens/s (decode attn HBM GB/s & prefill TFLOP/s as roofline)",
        "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)",
        "config": config,
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                         "kind": "port", "sample": sample_desc, "cpu_model": cpu_model(),
                         "nproc": host_threads()},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "fusor-ai is Rust and no Rust toolchain exists here: the oracle's C++ restatement "
                "of its Scalar-backend f32 attention is timed",
    }), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c3",
                    choices=["c1", "c2", "c3", "c3bf16", "decode256", "c4", "c5", "prefill",
                             "prefill_f32",
                             "qwen35", "proj", "proj64", "prologue"])
    ap.add_argument("--sequences", type=int, default=C3_SEQS,
                    help="C3 sequences (a smaller batch for profiling captures)")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle's check of the timed outputs (profiling runs)")
    ap.add_argument("--cpu-baselines", action="store_true",
                    help="also time the host restatement for C1, C2, C4 and a C5 slice (1 GPU)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
