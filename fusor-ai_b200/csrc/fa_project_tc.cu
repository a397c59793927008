// The qkv projection of Stack::attention_input (crates/blocks/src/layer.rs:175-209; the qkv
// Linear, project_quads in crates/kernels/src/linear.rs:52-71, f32 weights) for many rows at once
// on the tensor cores, at f32 accuracy: qkv[r][c] = sum_k x[r][k] W[c][k] + b[c].
//
// The f32 products are split in three tf32 products: with W = Wh + Wl and x = xh + xl, where
// Wh = tf32(W) (rounded to nearest) and Wl = W - Wh exactly (|Wl| <= 2^-11 |W|), the product is
// Wh xh + Wh xl + Wl xh plus Wl xl (below 2^-22 of it, left out) and the operands' own tf32
// rounding of Wl and xl (below 2^-22 as well). The tensor core's f32 accumulator adds only one
// k-block's twelve MMAs (32 values of k) before its sums are added into f32 registers: its
// additions round with a bias that grows with the chain (measured on B200: with the whole hidden
// dimension in the accumulator, a 4096-value product was 80x as far from the f64 sum as a plain
// f32 loop; with a drain every k-block, within 3x). At f32's accuracy, unlike one tf32 product
// (2^-11).
//
// A CTA = 128 output columns (the MMA's M: weight rows) x BN input rows (N: 16, 32 or 64) x one
// range of the hidden dimension. Warp roles, each running ahead of the next as far as its ring
// allows:
//   warp 0     TMA producer: 128 x 32 weight values and BN x 32 input values a k-block (both
//              128-byte swizzled rows) into a ring of raw stages;
//   warp 1     TMEM owner and MMA issuer (one thread): three tf32 MMAs per 8 values of k, each
//              k-block's twelve into the next of four TMEM buffers;
//   warps 2-9  split each raw stage in place into the high parts and a ring of low-part buffers;
//   warps 10-13 add each k-block's buffer into f32 registers (a thread = an output column, BN
//              rows), then the epilogue.
// The hidden dimension is split over consecutive CTAs when the column blocks alone would leave
// SMs idle: each CTA writes its partial sums to a workspace, and the last of a tile's CTAs to
// arrive (an arrival counter it resets) adds them in split order (deterministic), adds the bias
// and writes the rows. (A cluster per tile reducing through distributed shared memory ran in
// two waves on B200: 45 of 48 three-CTA clusters fit at once.) The RoPE + keep kernel then runs
// on the projected rows (the same kernel fa_attention_input launches, so the cache holds what
// projection-then-input keeps).
//
// Rooflines: the weight bytes from HBM (6144 x 4096 f32 weights: 100.7 MB, 15 us at the measured
// copy rate) and, for 64 rows, the three products' 9.7 GFLOP (12 us at the tf32 rate, half the
// bf16 one). Neither binds: per-stage timestamps on B200 put each CTA's k-loop at 1100-1500
// cycles a k-block, the MMA thread issuing the twelve tf32 MMAs in about 950 of them whatever N
// is (64 rows: 51-56 us a launch, against 143 us on the CUDA cores).
#include <cuda.h>
#include <cuda_runtime.h>

#include "fa_fmha_launch.h"
#include "fa_launch.cuh"
#include "fa_tc.cuh"

namespace fa {

namespace {

constexpr int kPtcThreads = 448;
constexpr int kPtcBM = 128;                      // output columns per CTA
constexpr int kPtcBK = 32;                       // f32 per 128-byte swizzled row: one k-block
constexpr int kPtcWBytes = kPtcBM * kPtcBK * 4;  // 16 KB
constexpr int kPtcKStep = 8;                     // tf32 values per MMA K step (32 bytes)
constexpr int kSplitThreads = 256;               // the split warps 2-9
constexpr int kDrainThreads = 128;               // the drain warps 10-13
constexpr int kDBufs = 4;                        // TMEM accumulator buffers
constexpr int kMaxSplits = 8;                    // splits of the hidden dimension

template <int BN>
struct PtcShape {
  static constexpr int kXBytes = BN * kPtcBK * 4;
  static constexpr int kStageBytes = kPtcWBytes + kXBytes;  // one raw stage, or one low part
  static constexpr int kStages = 200 * 1024 / kStageBytes;  // raw and low together
  // a raw stage lives from its load to its MMAs' end (the loads' latency, about 2000 cycles,
  // then the split and the MMAs), a low part from the split to its MMAs' end
  static constexpr int kLoStages = 3;
  static constexpr int kRawStages = kStages - kLoStages;
  static constexpr int kTmemCols = kDBufs * BN;             // 64, 128 or 256
  static constexpr int kBarBytes = 8 * (2 * kRawStages + 2 * kLoStages + 2 * kDBufs + 1) + 8;
  static constexpr size_t kSmemBytes = 1024 + size_t(kStages) * kStageBytes + kBarBytes;
  static_assert(BN == 16 || BN == 32 || BN == 64, "rows per tile");
  static_assert(kLoStages >= 2 && kRawStages >= 2, "at least two stages a ring");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

template <int BN>
__global__ void __launch_bounds__(kPtcThreads, 1)
    project_tc_kernel(const __grid_constant__ CUtensorMap w_map,
                      const __grid_constant__ CUtensorMap x_map, const ProjectTcArgs a) {
  using S = PtcShape<BN>;
  constexpr int SR = S::kRawStages, SL = S::kLoStages;
  constexpr uint32_t kIdesc = tc::instr_desc(2u, false, BN, kPtcBM);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* raw = smem;                          // [SR] x (W tile, x tile)
  unsigned char* lo = raw + SR * S::kStageBytes;      // [SL] x (W low tile, x low tile)
  uint64_t* bars = reinterpret_cast<uint64_t*>(lo + SL * S::kStageBytes);
  uint64_t* raw_full = bars;             // [SR] TMA bytes landed
  uint64_t* raw_empty = raw_full + SR;   // [SR] the MMAs that read the stage completed
  uint64_t* lo_full = raw_empty + SR;    // [SL] the split of the stage is written
  uint64_t* lo_empty = lo_full + SL;     // [SL] the MMAs that read the low part completed
  uint64_t* d_full = lo_empty + SL;      // [kDBufs] a k-block's products are in the buffer
  uint64_t* d_empty = d_full + kDBufs;   // [kDBufs] ... and have been added up
  uint64_t* mma_done = d_empty + kDBufs; // every MMA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int splits = a.splits;
  const int split = int(blockIdx.x) % splits;
  const int n0 = int(blockIdx.x) / splits * kPtcBM;  // first output column
  const int row0 = int(blockIdx.y) * BN;
  const int kb0 = int(int64_t(a.k_blocks) * split / splits);
  const int kb1 = int(int64_t(a.k_blocks) * (split + 1) / splits);
  const int n_kb = kb1 - kb0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 1);
    }
    for (int s = 0; s < SL; ++s) {
      mbar_init(&lo_full[s], kSplitThreads);
      mbar_init(&lo_empty[s], 1);
    }
    for (int b = 0; b < kDBufs; ++b) {
      mbar_init(&d_full[b], 1);
      mbar_init(&d_empty[b], kDrainThreads);
    }
    mbar_init(mma_done, 1);
    mbar_fence_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, S::kTmemCols);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------------------------
    if (lane == 0) {
      tc::tma_prefetch_map(&w_map);
      tc::tma_prefetch_map(&x_map);
      pdl_wait();  // the input rows written by the kernel before this one
      int issued = 0;
      for (int j = 0; j < n_kb; ++j) {
        const int st = j % SR;
        if (j >= SR && !mbar_wait(&raw_empty[st], ((j / SR) - 1) & 1, a.err)) break;
        unsigned char* dst = raw + st * S::kStageBytes;
        mbar_arrive_expect_tx(&raw_full[st], S::kStageBytes);
        const int k = (kb0 + j) * kPtcBK;
        tc::tma_load_3d(dst, &w_map, k, n0, 0, &raw_full[st]);
        tc::tma_load_3d(dst + kPtcWBytes, &x_map, k, row0, 0, &raw_full[st]);
        issued = j + 1;
      }
      // the loads in flight land before the CTA may go on (they have, unless a wait gave up)
      for (int j = max(0, issued - SR); j < issued; ++j)
        mbar_wait(&raw_full[j % SR], (j / SR) & 1, a.err);
    }
  } else if (warp == 1) {
    // ---- MMA issuer: k-block j's twelve products into TMEM buffer j % kDBufs -----------------
    if (lane == 0) {
      // The descriptors differ only in their start address (16-byte units in the low bits, and
      // shared-memory addresses stay below 2^18): one per ring, offsets added per stage and k
      // (the issue of the MMAs is on this thread's critical path).
      const uint64_t raw_desc = tc::smem_desc_sw128(smem_u32(raw), 16, 1024);
      const uint64_t lo_desc = tc::smem_desc_sw128(smem_u32(lo), 16, 1024);
      constexpr uint64_t kStageUnits = S::kStageBytes >> 4, kXUnits = kPtcWBytes >> 4;
      constexpr uint64_t kKUnits = (kPtcKStep * 4) >> 4;
      for (int j = 0; j < n_kb; ++j) {
        const int sr = j % SR, sl = j % SL, b = j % kDBufs;
        // the split of stage j (which waited for its bytes and rewrote every one of them) has
        // been written; the buffer's products of k-block j - kDBufs have been added up
        if (!mbar_wait(&lo_full[sl], (j / SL) & 1, a.err) ||
            (j >= kDBufs && !mbar_wait(&d_empty[b], ((j / kDBufs) - 1) & 1, a.err)))
          break;
        tc::fence_after_sync();
        const uint32_t d = tmem + uint32_t(b * BN);
        const uint64_t wh = raw_desc + uint64_t(sr) * kStageUnits, xh = wh + kXUnits;
        const uint64_t wl = lo_desc + uint64_t(sl) * kStageUnits, xl = wl + kXUnits;
#pragma unroll
        for (int k = 0; k < kPtcBK / kPtcKStep; ++k) {
          const uint64_t off = k * kKUnits;
          tc::mma_ss<true>(d, wh + off, xh + off, kIdesc, k > 0 ? 1u : 0u);
          tc::mma_ss<true>(d, wh + off, xl + off, kIdesc, 1u);
          tc::mma_ss<true>(d, wl + off, xh + off, kIdesc, 1u);
        }
        tc::commit(&raw_empty[sr]);
        tc::commit(&lo_empty[sl]);
        tc::commit(&d_full[b]);
      }
      // no MMA is in flight when TMEM is freed
      tc::commit(mma_done);
      mbar_wait(mma_done, 0, a.err);
    }
  } else if (warp < 10) {
    // ---- split each raw stage: high parts in place, low parts into the low ring ---------------
    const int t = threadIdx.x - 64;
    for (int j = 0; j < n_kb; ++j) {
      const int sr = j % SR, sl = j % SL;
      if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[sr], (j / SR) & 1, a.err)) ||
          (j >= SL &&
           !__all_sync(0xffffffffu, mbar_wait(&lo_empty[sl], ((j / SL) - 1) & 1, a.err))))
        break;
      float4* hi4 = reinterpret_cast<float4*>(raw + sr * S::kStageBytes);
      float4* lo4 = reinterpret_cast<float4*>(lo + sl * S::kStageBytes);
      // the W tile and the x tile are contiguous, and each low part has its tile's layout
#pragma unroll 4
      for (int i = t; i < S::kStageBytes / 16; i += kSplitThreads) {
        const float4 v = hi4[i];
        float4 h, l;
        h.x = __uint_as_float(tc::round_tf32(v.x));
        h.y = __uint_as_float(tc::round_tf32(v.y));
        h.z = __uint_as_float(tc::round_tf32(v.z));
        h.w = __uint_as_float(tc::round_tf32(v.w));
        l.x = v.x - h.x;
        l.y = v.y - h.y;
        l.z = v.z - h.z;
        l.w = v.w - h.w;
        hi4[i] = h;
        lo4[i] = l;
      }
      // generic-proxy writes become visible to the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&lo_full[sl]);
    }
  } else {
    // ---- add each k-block's products into f32 registers: this thread's TMEM lane (an output
    // column), BN columns (the rows) -------------------------------------------------------------
    const int q = warp & 3;  // the TMEM lane quarter this warp may access
    const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
    float acc[BN];
#pragma unroll
    for (int r = 0; r < BN; ++r) acc[r] = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kb; ++j) {
      const int b = j % kDBufs;
      if (!__all_sync(0xffffffffu, mbar_wait(&d_full[b], (j / kDBufs) & 1, a.err))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t base = lane_base + uint32_t(b * BN);
      if constexpr (BN == 16) {
        uint32_t d[16];
        tc::tmem_ld16_wait(base, d);
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r] += __uint_as_float(d[r]);
      } else {
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t d[32];
          tc::tmem_ld32_wait(base + c0, d);
#pragma unroll
          for (int r = 0; r < 32; ++r) acc[c0 + r] += __uint_as_float(d[r]);
        }
      }
      tc::fence_before_sync();
      mbar_arrive(&d_empty[b]);
    }
    if (!ok) atomicOr(a.err, kErrTimeout);
    // ---- epilogue: the rows' sums of this thread's column, plus the bias; with the hidden
    // dimension split, the partial sums go to the workspace and the last of the tile's CTAs to
    // arrive adds them in split order (deterministic) -----------------------------------------
    const int col = q * 32 + lane;
    const int c = n0 + col;
    const int tile = int(blockIdx.x) / splits + int(blockIdx.y) * (int(gridDim.x) / splits);
    const float bias = a.bias != nullptr && c < a.outputs ? a.bias[c] : 0.0f;
    if (splits == 1) {
#pragma unroll
      for (int r = 0; r < BN; ++r)
        if (row0 + r < a.rows && c < a.outputs)
          a.qkv[int64_t(row0 + r) * a.qkv_stride + c] = acc[r] + bias;
    } else {
      // [tile][split][BN][128]: this CTA's rows x columns, contiguous
      float* part = a.partials + (int64_t(tile) * splits + split) * BN * kPtcBM + col;
#pragma unroll
      for (int r = 0; r < BN; ++r) __stcg(part + r * kPtcBM, acc[r]);
      __threadfence();
      named_sync(1, kDrainThreads);
      __shared__ int last;
      if (threadIdx.x == 320) last = atomicAdd(a.counters + tile, 1) == splits - 1;
      named_sync(1, kDrainThreads);
      if (last) {
        __threadfence();
        // eight rows at a time, every split's value of them loaded before any is added (one
        // load latency a batch: loading row by row took about 30 us for 64 rows)
        const float* p0 = a.partials + int64_t(tile) * splits * BN * kPtcBM + col;
#pragma unroll 1
        for (int rb = 0; rb < BN && row0 + rb < a.rows; rb += 8) {
          float t[8][kMaxSplits];
#pragma unroll
          for (int sp = 0; sp < kMaxSplits; ++sp)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              t[i][sp] = sp < splits ? __ldcg(p0 + (sp * BN + rb + i) * kPtcBM) : 0.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float sum = 0.0f;
#pragma unroll
            for (int sp = 0; sp < kMaxSplits; ++sp)
              if (sp < splits) sum += t[i][sp];
            if (row0 + rb + i < a.rows && c < a.outputs)
              a.qkv[int64_t(row0 + rb + i) * a.qkv_stride + c] = sum + bias;
          }
        }
        if (threadIdx.x == 320) a.counters[tile] = 0;  // ready for the next launch
      }
    }
  }
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, S::kTmemCols);
}

template <int BN>
cudaError_t launch_bn(const ProjectTcArgs& a, const CUtensorMap& wm, const CUtensorMap& xm,
                      int col_blocks, cudaStream_t stream) {
  using S = PtcShape<BN>;
  auto kernel = project_tc_kernel<BN>;
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t e = smem_limit_once(kernel, int(S::kSmemBytes), configured);
  if (e != cudaSuccess) return e;
  const dim3 grid(unsigned(col_blocks * a.splits), unsigned((a.rows + BN - 1) / BN));
  return launch_pdl(kernel, grid, dim3(kPtcThreads), S::kSmemBytes, stream, wm, xm, a);
}

}  // namespace

int project_tc_rows_per_tile(int rows) {
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  return 64;
}

cudaError_t launch_project_tc(const ProjectTcArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  const int bn = project_tc_rows_per_tile(a.rows);
  if (a.splits < 1 || a.splits > kMaxSplits || a.k_blocks < a.splits ||
      a.k_blocks != (a.hidden + kPtcBK - 1) / kPtcBK || a.outputs <= 0 || a.qkv == nullptr ||
      (a.rows + bn - 1) / bn > 65535 ||
      (a.splits > 1 && (a.partials == nullptr || a.counters == nullptr)))
    return cudaErrorInvalidValue;
  alignas(64) CUtensorMap wm, xm;
  if (!encode_map_f32(&wm, a.weight, uint64_t(a.hidden), uint64_t(a.outputs),
                      uint64_t(a.w_stride) * 4, kPtcBK, kPtcBM) ||
      !encode_map_f32(&xm, a.x, uint64_t(a.hidden), uint64_t(a.rows), uint64_t(a.x_stride) * 4,
                      kPtcBK, uint32_t(bn)))
    return cudaErrorInvalidValue;
  const int col_blocks = (a.outputs + kPtcBM - 1) / kPtcBM;
  switch (bn) {
    case 16: return launch_bn<16>(a, wm, xm, col_blocks, stream);
    case 32: return launch_bn<32>(a, wm, xm, col_blocks, stream);
    default: return launch_bn<64>(a, wm, xm, col_blocks, stream);
  }
}

}  // namespace fa
