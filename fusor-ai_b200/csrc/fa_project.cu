// The QKV projection of Stack::attention_input (crates/blocks/src/layer.rs:175-209: the layer's
// qkv Linear, project_quads in crates/kernels/src/linear.rs:52-71, here for f32 weights) fused
// with what follows it in that function: head norm, RoPE and KvCache::keep (rope_keep_head, the
// RoPE kernel's own code, so the cache holds the keys project-then-fa_attention_input keeps).
//
// qkv[r][c] = sum_k x[r][k] * W[c][k] + b[c] for the rows r of a span (or a batch of sequences)
// and the head_dim columns c of one head unit (a query, key or value head). A CTA covers (head
// unit, block of up to 16 rows, chunk of the hidden dimension): it stages the rows' chunk of x in
// shared memory and streams the unit's weight rows, a warp reading 512 contiguous bytes of one
// weight row per load, NC output columns at a time (4, or 8 with 8 rows per pass) so that each x
// value read from shared memory feeds NC products and each weight value NR. A lane accumulates
// NR rows x NC columns over its k's; the lanes' sums are folded with a butterfly of shuffles
// that leaves row i's total in the lanes whose bits spell i (NR - 1 + log2(32 / NR) shuffles per
// column rather than 5 NR).
// With the hidden dimension split, each CTA writes its partial sums, and the last CTA of the
// (unit, row block) to arrive (an arrival counter it resets) adds them in split order and the
// bias, then runs the epilogue: a warp per row, rope_keep_head. Without a split the CTA does.
// Decode (a few rows) is bound by the weight bytes, read once from HBM; many rows by the FFMA
// pipe (f32 weights and products: no tensor cores).
#include <cuda_runtime.h>

#include "fa_launch.cuh"

namespace fa {

namespace {

constexpr int kProjectThreads = 256;
constexpr int kProjectWarps = kProjectThreads / 32;

// The warp's sums of acc[i] (i < NR): the lanes fold halves of their accumulators across lane
// bits 16, 8, ... until each holds one row, then add across the remaining bits. The result is the
// total of row folded_row<NR>(lane), in every lane; folded_owner<NR> picks one lane per row.
template <int NR>
__device__ __forceinline__ float fold_rows(float (&acc)[NR], int lane) {
  static_assert(NR == 1 || NR == 2 || NR == 4 || NR == 8, "rows per pass");
  int bit = 16;
#pragma unroll
  for (int n = NR; n > 1; n /= 2) {
    const bool upper = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? acc[i] : acc[i + n / 2];
      const float keep = upper ? acc[i + n / 2] : acc[i];
      acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
    bit >>= 1;
  }
  float v = acc[0];
#pragma unroll
  for (; bit >= 1; bit >>= 1) v += __shfl_xor_sync(0xffffffffu, v, bit);
  return v;
}

template <int NR>
__device__ __forceinline__ int folded_row(int lane) {
  int row = 0, bit = 16;
#pragma unroll
  for (int n = NR; n > 1; n /= 2) {
    if (lane & bit) row += n / 2;
    bit >>= 1;
  }
  return row;
}

template <int NR>
__device__ __forceinline__ bool folded_owner(int lane) {
  constexpr int kLowBits = 32 / NR - 1;  // the bits summed after the folds
  return (lane & kLowBits) == 0;
}

template <typename KT, int NR>
__global__ void __launch_bounds__(kProjectThreads)
    project_keep_kernel(const __grid_constant__ ProjectArgs p, const __grid_constant__ RopeArgs r) {
  constexpr int kProjectCols = NR == 8 ? 8 : 4;  // output columns a warp accumulates at once
  extern __shared__ float4 smem4[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x, rb = blockIdx.y, sp = blockIdx.z;
  const int d = r.head_dim;
  const int r0 = rb * p.row_block, nrows = min(p.row_block, p.rows - r0);
  const int padded = (nrows + NR - 1) / NR * NR;
  const int k0 = sp * p.chunk, klen = min(p.chunk, p.hidden - k0);
  float* xs = reinterpret_cast<float*>(smem4);      // [row_block][chunk]: the rows' chunk of x
  float* hs = xs + size_t(p.row_block) * p.chunk;   // [row_block][head_dim]: the unit's outputs

  // ---- stage x (zeros past the rows and past the chunk's end) --------------------------------
  const int c4 = p.chunk / 4;
  for (int i = threadIdx.x; i < padded * c4; i += kProjectThreads) {
    const int rr = i / c4, k = (i % c4) * 4;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (rr < nrows && k < klen)
      v = *reinterpret_cast<const float4*>(p.x + int64_t(r0 + rr) * p.x_stride + k0 + k);
    reinterpret_cast<float4*>(xs)[i] = v;
  }
  __syncthreads();

  // ---- products: a warp takes NC columns at a time, NR rows per pass over its k's ------------
  const bool split = p.splits > 1;
  const int64_t block_id = int64_t(unit) * gridDim.y + rb;
  float* sums = split ? p.partials + (block_id * p.splits + sp) * p.row_block * d : hs;
  const int steps = (klen + 127) / 128;  // k steps of a warp's 32 float4s
  for (int c0 = warp * kProjectCols; c0 < d; c0 += kProjectWarps * kProjectCols) {
    const float* wrow = p.weight + int64_t(unit * d + c0) * p.w_stride + k0;
    for (int g = 0; g < padded; g += NR) {
      float acc[kProjectCols][NR];
#pragma unroll
      for (int c = 0; c < kProjectCols; ++c)
#pragma unroll
        for (int i = 0; i < NR; ++i) acc[c][i] = 0.0f;
#pragma unroll 4
      for (int j = 0; j < steps; ++j) {
        const int k = j * 128 + lane * 4;
        if (k >= klen) continue;
        float4 w[kProjectCols];
#pragma unroll
        for (int c = 0; c < kProjectCols; ++c)
          w[c] = __ldg(reinterpret_cast<const float4*>(wrow + int64_t(c) * p.w_stride + k));
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          const float4 xv = *reinterpret_cast<const float4*>(xs + (g + i) * p.chunk + k);
#pragma unroll
          for (int c = 0; c < kProjectCols; ++c)
            acc[c][i] = fmaf(w[c].w, xv.w, fmaf(w[c].z, xv.z, fmaf(w[c].y, xv.y,
                                                                    fmaf(w[c].x, xv.x, acc[c][i]))));
        }
      }
#pragma unroll
      for (int c = 0; c < kProjectCols; ++c) {
        const float v = fold_rows<NR>(acc[c], lane);
        const int rr = g + folded_row<NR>(lane);
        if (folded_owner<NR>(lane) && rr < nrows) sums[rr * d + c0 + c] = v;
      }
    }
  }
  pdl_trigger();  // the attention after this kernel may be scheduled (it waits for completion)

  // ---- the unit's outputs: partials added in split order, then the bias -----------------------
  const float* bias = p.bias != nullptr ? p.bias + int64_t(unit) * d : nullptr;
  if (split) {
    __threadfence();  // the partials are visible device-wide before the arrival is counted
    __syncthreads();
    if (threadIdx.x == 0) {
      int* counter = p.counters + block_id;
      const int last = atomicAdd(counter, 1) == p.splits - 1;
      if (last) *counter = 0;  // every split has arrived: ready for the next launch
      s_last = last;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = p.partials + block_id * p.splits * p.row_block * d;
    for (int i = threadIdx.x; i < nrows * d; i += kProjectThreads) {
      float sum = 0.0f;
      for (int s = 0; s < p.splits; ++s) sum += __ldcg(base + int64_t(s) * p.row_block * d + i);
      hs[i] = bias != nullptr ? sum + bias[i % d] : sum;
    }
  } else if (bias != nullptr) {
    __syncthreads();
    for (int i = threadIdx.x; i < nrows * d; i += kProjectThreads) hs[i] += bias[i % d];
  }
  __syncthreads();
  if (p.qkv_out != nullptr)
    for (int i = threadIdx.x; i < nrows * d; i += kProjectThreads)
      p.qkv_out[int64_t(r0 + i / d) * p.qkv_out_stride + int64_t(unit) * d + i % d] = hs[i];

  // ---- epilogue: head norm, RoPE, keep (a warp per row) --------------------------------------
  for (int rr = warp; rr < nrows; rr += kProjectWarps)
    rope_keep_head<KT>(r, r0 + rr, unit, lane, hs + rr * d);
}

template <typename KT, int NR>
cudaError_t launch_nr(const ProjectArgs& p, const RopeArgs& r, size_t smem, cudaStream_t stream) {
  auto kernel = project_keep_kernel<KT, NR>;
  // the host's plans stay within 200 KB of shared memory; the limit is raised to that once
  constexpr int kMaxSmem = 200 * 1024;
  if (smem > size_t(kMaxSmem)) return cudaErrorInvalidValue;
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t e = smem_limit_once(kernel, kMaxSmem, configured);
  if (e != cudaSuccess) return e;
  const int units = r.heads + 2 * r.kv_heads;
  const dim3 grid(unsigned(units), unsigned((p.rows + p.row_block - 1) / p.row_block),
                  unsigned(p.splits));
  kernel<<<grid, kProjectThreads, smem, stream>>>(p, r);
  return cudaGetLastError();
}

template <typename KT>
cudaError_t launch_kt(int nr, const ProjectArgs& p, const RopeArgs& r, size_t smem,
                      cudaStream_t stream) {
  switch (nr) {
    case 1: return launch_nr<KT, 1>(p, r, smem, stream);
    case 4: return launch_nr<KT, 4>(p, r, smem, stream);
    case 8: return launch_nr<KT, 8>(p, r, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_project(int kt, int nr, const ProjectArgs& p, const RopeArgs& r, size_t smem,
                           cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  if (r.gate_heads != 0 || r.head_dim % 8 != 0 || p.chunk % 128 != 0 ||
      p.row_block % nr != 0)
    return cudaErrorInvalidValue;
  return kt == kKtF32 ? launch_kt<float>(nr, p, r, smem, stream)
                      : launch_kt<__nv_bfloat16>(nr, p, r, smem, stream);
}

}  // namespace fa
