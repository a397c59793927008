// The steps either side of the full-mask and gated attentions that are not attention:
//
// * The query/key prologue of the video and image DiT blocks: Wan's normalize_and_rotate
//   (crates/blocks/src/wan_dit/block.rs:109-140) and Pyramid's (pyramid_jit/block.rs:100-131)
//   RMS-normalize every token's query row and key row over their whole width (row_work.rs:57-75,
//   ops.rs:7-16), MMDiT's head_norms (mmdit/pass.rs:64-68,162-192) each head on its own; then
//   each query and key head is turned by the token's rotary angles (rope_interleaved,
//   ops.rs:87-95). One warp per (token, query | key | value row); the whole-row sum of squares
//   is a first pass over the row, the second pass reads it again (from L1/L2) head by head and
//   writes the normalized, rotated heads in f32 or bf16, the operand rows the tensor-core
//   attention reads. A memory-bound kernel: per token it reads 3 rows and writes 3 rows.
//
// * The sigmoid gate of the hybrid blocks' attention output (hybrid/attention.rs:262-295):
//   attended *= 1 / (1 + exp(-gate)), a gate per element (a gate head per query head) or one per
//   query head.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "fa_launch.cuh"
#include "fa_ptx.cuh"

namespace fa {

namespace {

constexpr int kPrologueWarps = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Row part `part` (0 queries, 1 keys) of one token: optional RMSNorm, then RoPE, into out.
template <typename O>
__device__ __forceinline__ void normalize_rotate_row(const PrologueArgs& a, int token, int part,
                                                     int lane, O* out_row) {
  const int d = a.head_dim, half = d / 2;
  const int64_t width = int64_t(a.heads) * d;
  const float* row = a.qkv + int64_t(token) * a.qkv_stride + part * width;
  const float* weight = part == 0 ? a.q_norm : a.k_norm;
  float inverse = 1.0f;
  if (a.norm == kNormRow) {
    // ops::rms_norm's mean of squares over the whole row (a tree sum rather than the CPU's
    // sequential one: the same value within a few ulps)
    float ss = 0.0f;
    if (a.vec_in) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (int64_t c = lane; c < width / 4; c += 32) {
        const float4 v = r4[c];
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
      }
    } else {
      for (int64_t c = lane; c < width; c += 32) ss = fmaf(row[c], row[c], ss);
    }
    ss = warp_sum(ss);
    inverse = 1.0f / sqrtf(ss / float(width) + a.eps);
  }
  const bool rotate = a.rope != 0 && token < a.rotated_rows;
  const float* cs = a.angles + int64_t(token) * d;
  const bool pairs_adjacent = a.rope != 1;  // interleaved pairs (2p, 2p + 1); or no rotation
  for (int h = 0; h < a.heads; ++h) {
    const float* hp = row + int64_t(h) * d;
    float x[4], y[4];
    int lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = lane + 32 * j;
      lo[j] = -1;
      x[j] = y[j] = 0.0f;
      if (p >= half) continue;
      if (pairs_adjacent) {
        lo[j] = 2 * p;
        if (a.vec_in) {
          const float2 t = *reinterpret_cast<const float2*>(hp + 2 * p);
          x[j] = t.x;
          y[j] = t.y;
        } else {
          x[j] = hp[2 * p];
          y[j] = hp[2 * p + 1];
        }
      } else {
        lo[j] = p;
        x[j] = hp[p];
        y[j] = hp[p + half];
      }
    }
    if (a.norm != kNormNone) {
      float head_inverse = inverse;
      if (a.norm == kNormHead) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss = fmaf(y[j], y[j], fmaf(x[j], x[j], ss));
        ss = warp_sum(ss);
        head_inverse = 1.0f / sqrtf(ss / float(d) + a.eps);
      }
      // whole-row weights are heads x head_dim wide; a head norm's head_dim wide
      const float* w = a.norm == kNormRow ? weight + int64_t(h) * d : weight;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (lo[j] < 0) continue;
        const int hi = pairs_adjacent ? lo[j] + 1 : lo[j] + half;
        x[j] = __fmul_rn(__fmul_rn(x[j], head_inverse), w[lo[j]]);
        y[j] = __fmul_rn(__fmul_rn(y[j], head_inverse), w[hi]);
      }
    }
    if (rotate) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (lo[j] < 0) continue;
        const int p = lane + 32 * j;
        const float c = cs[p], s = cs[half + p];
        const float nx = __fsub_rn(__fmul_rn(x[j], c), __fmul_rn(y[j], s));
        const float ny = __fadd_rn(__fmul_rn(y[j], c), __fmul_rn(x[j], s));
        x[j] = nx;
        y[j] = ny;
      }
    }
    O* op = out_row + part * width + int64_t(h) * d;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (lo[j] < 0) continue;
      if constexpr (sizeof(O) == 2) {
        if (pairs_adjacent && a.vec_out) {
          *reinterpret_cast<__nv_bfloat162*>(op + lo[j]) = __floats2bfloat162_rn(x[j], y[j]);
        } else {
          op[lo[j]] = __float2bfloat16_rn(x[j]);
          op[pairs_adjacent ? lo[j] + 1 : lo[j] + half] = __float2bfloat16_rn(y[j]);
        }
      } else {
        if (pairs_adjacent && a.vec_out) {
          *reinterpret_cast<float2*>(op + lo[j]) = make_float2(x[j], y[j]);
        } else {
          op[lo[j]] = x[j];
          op[pairs_adjacent ? lo[j] + 1 : lo[j] + half] = y[j];
        }
      }
    }
  }
}

template <typename O>
__device__ __forceinline__ void copy_values_row(const PrologueArgs& a, int token, int lane,
                                                O* out_row) {
  const int64_t width = int64_t(a.heads) * a.head_dim;
  const float* row = a.qkv + int64_t(token) * a.qkv_stride + 2 * width;
  O* op = out_row + 2 * width;
  if (a.vec_in && a.vec_out) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    for (int64_t c = lane; c < width / 4; c += 32) {
      const float4 v = r4[c];
      if constexpr (sizeof(O) == 2) {
        __nv_bfloat162 two[2] = {__floats2bfloat162_rn(v.x, v.y), __floats2bfloat162_rn(v.z, v.w)};
        *reinterpret_cast<uint2*>(op + 4 * c) = *reinterpret_cast<const uint2*>(two);
      } else {
        *reinterpret_cast<float4*>(op + 4 * c) = v;
      }
    }
    return;
  }
  for (int64_t c = lane; c < width; c += 32) {
    if constexpr (sizeof(O) == 2) op[c] = __float2bfloat16_rn(row[c]);
    else op[c] = row[c];
  }
}

template <typename O>
__global__ void __launch_bounds__(kPrologueWarps * 32) prologue_kernel(const PrologueArgs a) {
  pdl_trigger();  // the attention kernel after it may be scheduled now (it waits for this one)
  const int lane = threadIdx.x & 31;
  const int64_t item = int64_t(blockIdx.x) * kPrologueWarps + (threadIdx.x >> 5);
  if (item >= int64_t(a.tokens) * a.parts) return;
  const int token = int(item / a.parts), part = int(item % a.parts);
  O* out_row = static_cast<O*>(a.out) + int64_t(token) * a.out_stride;
  if (part == 2) copy_values_row<O>(a, token, lane, out_row);
  else normalize_rotate_row<O>(a, token, part, lane, out_row);
}

// The same for head_dim 128 and at most kRowHeads heads, streamed: persistent CTAs, each warp
// with a two-slot ring of rows in shared memory; while it works on one row (query, key or value
// part of a token) the TMA engine brings its next (one 1-D bulk copy per row), so the loads in
// flight do not depend on how many warps fit. A lane's float4 j of a row is elements 4 lane ..
// 4 lane + 3 of head j: the whole-row sum of squares (the same lane order and sum as the kernel
// above: the same inverse), then head by head the norm, the RoPE and the stores. Interleaved pairs
// (2p, 2p + 1) sit in one lane; pairs by halves (p, p + 64) in lanes l and l + 16, exchanged by
// one shuffle.
constexpr int kRowHeads = 16;
constexpr int kStreamWarps = 8;

template <typename O>
__device__ __forceinline__ void store4(O* dst, float a, float b, float c, float d) {
  if constexpr (sizeof(O) == 2) {
    __nv_bfloat162 two[2] = {__floats2bfloat162_rn(a, b), __floats2bfloat162_rn(c, d)};
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(two);
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
  }
}

// One row part (0 queries, 1 keys, 2 values) of `token`, its f32 values at `row` (shared memory).
template <typename O>
__device__ __forceinline__ void prologue128_row(const PrologueArgs& a, int token, int part,
                                                int lane, const float* row) {
  constexpr int d = 128;
  const int heads = a.heads;
  const int64_t width = int64_t(heads) * d;
  O* out = static_cast<O*>(a.out) + int64_t(token) * a.out_stride + part * width + lane * 4;
  row += lane * 4;
  if (part == 2) {  // the values, converted
    for (int j = 0; j < heads; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(row + j * d);
      store4(out + j * d, v.x, v.y, v.z, v.w);
    }
    return;
  }
  const float* weight = part == 0 ? a.q_norm : a.k_norm;
  float inverse = 1.0f;
  if (a.norm == kNormRow) {
    float ss = 0.0f;
    for (int j = 0; j < heads; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(row + j * d);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    inverse = 1.0f / sqrtf(ss / float(width) + a.eps);
  }
  const bool rotate = a.rope != 0 && token < a.rotated_rows;
  const float* cs = a.angles + int64_t(token) * d;
  float c[4] = {1.0f, 1.0f, 1.0f, 1.0f}, s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (rotate) {
    if (a.rope == 1) {  // by halves: element e = 4 (lane % 16) + t pairs with e + 64
      const float4 c4 = *reinterpret_cast<const float4*>(cs + 4 * (lane & 15));
      const float4 s4 = *reinterpret_cast<const float4*>(cs + 64 + 4 * (lane & 15));
      c[0] = c4.x; c[1] = c4.y; c[2] = c4.z; c[3] = c4.w;
      s[0] = s4.x; s[1] = s4.y; s[2] = s4.z; s[3] = s4.w;
    } else {  // interleaved: pairs 2 lane and 2 lane + 1
      const float2 c2 = *reinterpret_cast<const float2*>(cs + 2 * lane);
      const float2 s2 = *reinterpret_cast<const float2*>(cs + 64 + 2 * lane);
      c[0] = c[1] = c2.x; c[2] = c[3] = c2.y;
      s[0] = s[1] = s2.x; s[2] = s[3] = s2.y;
    }
  }
  for (int j = 0; j < heads; ++j) {
    const float4 v = *reinterpret_cast<const float4*>(row + j * d);
    float e[4] = {v.x, v.y, v.z, v.w};
    if (a.norm != kNormNone) {
      float head_inverse = inverse;
      if (a.norm == kNormHead) {
        float ss = 0.0f;
#pragma unroll
        for (int t = 0; t < 4; ++t) ss = fmaf(e[t], e[t], ss);
        ss = warp_sum(ss);
        head_inverse = 1.0f / sqrtf(ss / float(d) + a.eps);
      }
      const float4 w4 = *reinterpret_cast<const float4*>(
          (a.norm == kNormRow ? weight + j * d : weight) + lane * 4);
      const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) e[t] = __fmul_rn(__fmul_rn(e[t], head_inverse), w[t]);
    }
    if (rotate) {
      if (a.rope == 1) {
        const bool upper = lane >= 16;  // this lane holds the y of its pairs
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float other = __shfl_xor_sync(0xffffffffu, e[t], 16);
          const float x = upper ? other : e[t], y = upper ? e[t] : other;
          e[t] = upper ? __fadd_rn(__fmul_rn(y, c[t]), __fmul_rn(x, s[t]))
                       : __fsub_rn(__fmul_rn(x, c[t]), __fmul_rn(y, s[t]));
        }
      } else {
#pragma unroll
        for (int t = 0; t < 4; t += 2) {
          const float x = e[t], y = e[t + 1];
          e[t] = __fsub_rn(__fmul_rn(x, c[t]), __fmul_rn(y, s[t]));
          e[t + 1] = __fadd_rn(__fmul_rn(y, c[t]), __fmul_rn(x, s[t]));
        }
      }
    }
    store4(out + j * d, e[0], e[1], e[2], e[3]);
  }
}

template <typename O>
__global__ void __launch_bounds__(kStreamWarps * 32) prologue_stream_kernel(const PrologueArgs a) {
  pdl_trigger();  // the attention kernel after it may be scheduled now (it waits for this one)
  extern __shared__ float4 smem4[];
  __shared__ uint64_t bars[kStreamWarps][2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int width = a.heads * 128;
  const uint32_t bytes = uint32_t(width) * 4u;  // a multiple of 16: widths of whole float4s
  float* ring = reinterpret_cast<float*>(smem4) + size_t(warp) * 2 * width;
  uint64_t* bar = bars[warp];
  if (lane == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
  }
  __syncwarp();
  const int64_t items = int64_t(a.tokens) * a.parts;
  const int64_t step = int64_t(gridDim.x) * kStreamWarps;
  auto source = [&](int64_t item) {
    const int64_t token = item / a.parts, part = item % a.parts;
    return a.qkv + token * a.qkv_stride + part * int64_t(width);
  };
  int64_t item = int64_t(blockIdx.x) * kStreamWarps + warp;
  if (lane == 0 && item < items) {
    mbar_arrive_expect_tx(&bar[0], bytes);
    bulk_g2s(ring, source(item), bytes, &bar[0]);
  }
  int k = 0;  // rows this warp has taken
  bool pending = false;  // a copy issued beyond the last row waited for (a wait gave up)
  for (; item < items; item += step, ++k) {
    const int slot = k & 1;
    if (lane == 0 && item + step < items) {
      // the other slot's row was read by every lane before the __syncwarp closing the last row
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&bar[slot ^ 1], bytes);
      bulk_g2s(ring + size_t(slot ^ 1) * width, source(item + step), bytes, &bar[slot ^ 1]);
    }
    if (!__all_sync(0xffffffffu, mbar_wait(&bar[slot], (k >> 1) & 1, a.err))) {
      pending = item + step < items;
      break;
    }
    const int token = int(item / a.parts), part = int(item % a.parts);
    prologue128_row<O>(a, token, part, lane, ring + size_t(slot) * width);
    __syncwarp();
  }
  // a copy still in flight lands before the CTA may exit
  if (pending && lane == 0) mbar_wait(&bar[(k + 1) & 1], ((k + 1) >> 1) & 1, a.err);
}

// out[r][h*d + e] *= sigmoid(gate), gate = qkv[r][gate_offset + h*d + e] (per element) or
// qkv[r][gate_offset + h] (per head)
__global__ void gate_kernel(const GateArgs a) {
  const int64_t width = int64_t(a.heads) * a.head_dim;
  const int64_t total = int64_t(a.rows) * width;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / width, c = i % width;
    const float* g = a.qkv + r * a.qkv_stride + a.gate_offset;
    const float gate = a.per_head ? g[c / a.head_dim] : g[c];
    float* o = a.out + r * a.out_stride + c;
    *o = *o * (1.0f / (1.0f + expf(-gate)));
  }
}

}  // namespace

cudaError_t launch_prologue(const PrologueArgs& a, cudaStream_t stream) {
  const int64_t items = int64_t(a.tokens) * a.parts;
  if (items == 0) return cudaSuccess;
  const dim3 grid(unsigned((items + kPrologueWarps - 1) / kPrologueWarps));
  // the streamed form: head_dim 128, at most kRowHeads heads, 16-byte aligned rows (widths of
  // whole float4s), angle rows and weights
  const bool rows128 = a.head_dim == 128 && a.heads <= kRowHeads && a.vec_in && a.vec_out &&
                       (a.rope == 0 || reinterpret_cast<uintptr_t>(a.angles) % 16 == 0) &&
                       (a.norm != kNormRow || (reinterpret_cast<uintptr_t>(a.q_norm) % 16 == 0 &&
                                               reinterpret_cast<uintptr_t>(a.k_norm) % 16 == 0)) &&
                       (a.norm != kNormHead || (reinterpret_cast<uintptr_t>(a.q_norm) % 16 == 0 &&
                                                reinterpret_cast<uintptr_t>(a.k_norm) % 16 == 0));
  if (rows128) {
    // two rows in flight per warp; persistent CTAs, as many as fit on every SM
    const size_t smem = size_t(kStreamWarps) * 2 * a.heads * 128 * sizeof(float);
    // the limit raised once per device to what kRowHeads heads need
    constexpr int kMaxSmem = kStreamWarps * 2 * kRowHeads * 128 * int(sizeof(float));
    static std::atomic<bool> configured_bf16[64], configured_f32[64];
    auto kernel = a.out_bf16 ? prologue_stream_kernel<__nv_bfloat16> : prologue_stream_kernel<float>;
    cudaError_t e = smem_limit_once(kernel, kMaxSmem, a.out_bf16 ? configured_bf16 : configured_f32);
    if (e != cudaSuccess) return e;
    int per_sm = 0, sms = 0, device = 0;
    if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
      return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kStreamWarps * 32,
                                                           smem)) != cudaSuccess)
      return e;
    const int64_t ctas = std::min<int64_t>(int64_t(std::max(per_sm, 1)) * sms,
                                           (items + kStreamWarps - 1) / kStreamWarps);
    kernel<<<unsigned(ctas), kStreamWarps * 32, smem, stream>>>(a);
  } else {
    if (a.out_bf16) prologue_kernel<__nv_bfloat16><<<grid, kPrologueWarps * 32, 0, stream>>>(a);
    else prologue_kernel<float><<<grid, kPrologueWarps * 32, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_gate(const GateArgs& a, cudaStream_t stream) {
  const int64_t total = int64_t(a.rows) * a.heads * a.head_dim;
  if (total == 0) return cudaSuccess;
  const int blocks = int(std::min<int64_t>((total + 255) / 256, 148 * 8));
  gate_kernel<<<blocks, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace fa
