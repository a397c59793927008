// The attention input (Stack::attention_input + position, crates/blocks/src/layer.rs:175-234):
// optional Qwen3 head RMSNorm (ops.rs:7-16), RoPE by halves or interleaved (ops.rs:77-95) on the
// query and key heads, then KvCache::keep of the key and value heads (transformer.rs:164-180).
//
// The gated attention of the hybrid blocks (crates/blocks/src/hybrid/attention.rs:155-259) uses
// the same kernel: its rows hold a gate head per query head between the query and key heads
// (`gate_heads`, skipped here and read by the gate epilogue), and it rotates by halves only the
// first `rotary_dim` elements of a head (rope_half over head[..rotary_dim], after the head norm
// of the whole head).
//
// One warp per (row, head unit). The rotation is the reference's arithmetic bit for bit: each
// product rounded, then the difference or sum (no fused multiply-add), by the host's cos/sin
// table, so the cache holds exactly the keys the CPU path would keep. The rotated queries go to
// the workspace pre-scaled by log2(e)/sqrt(head_dim) for the base-2 softmax of the attention.
#pragma once

#include "fa_ptx.cuh"

namespace fa {

constexpr int kRopeWarps = 4;

struct KeepRow {
  void* k;       // keys of (layer, kv head 0) of this row's cache
  void* v;
  int capacity;
  int position;
};

struct RopeArgs {
  int heads, kv_heads, head_dim, rope, n_rows;
  int gate_heads;  // heads between the query and the key heads that are not rotated or kept
  int rotary_dim;  // elements of a query or key head rotated, from its first (0: head_dim)
  const float* qkv;  // row r at qkv + r*qkv_stride: heads, gate heads, kv heads, kv heads
  int64_t qkv_stride;
  const float* angles;  // row r at angles + r*rotary_dim: cosines then sines (or nullptr)
  const float* q_norm;  // optional head norms (head_dim weights each)
  const float* k_norm;
  float eps;
  float* q_out;  // rotated queries, row r at q_out + r*q_out_stride, head h at h*head_dim
  int64_t q_out_stride;
  float q_scale;         // scale applied to q_out (1 for the raw rotated queries)
  int q_out_bf16;        // q_out holds bf16 (the tensor-core path over a bf16 cache)
  int keep;              // 0: rotate queries only
  int batch;             // 0: one cache (rows[0]), positions first + r; 1: rows[r] per row
  int first;
  KeepRow keep_rows[kMaxBatchRows];
};

template <typename KT>
__device__ __forceinline__ KT to_kv(float x);
template <>
__device__ __forceinline__ float to_kv<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_kv<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Head `unit` (the qkv row's numbering: query heads, gate heads, key heads, value heads) of row
// `row`, whose head_dim values are at `head`: head norm and RoPE of a query or key head, then the
// rotated query into q_out or the key/value head kept in the row's cache. One warp.
template <typename KT>
__device__ __forceinline__ void rope_keep_head(const RopeArgs& a, int row, int unit, int lane,
                                               const float* head) {
  const bool is_query = unit < a.heads;
  if (!is_query && unit < a.heads + a.gate_heads) return;
  const int kunit = unit - a.gate_heads;  // the cache's numbering: query heads, then kv heads
  const bool is_key = !is_query && kunit < a.heads + a.kv_heads;
  if (!is_query && !a.keep) return;
  const int d = a.head_dim, half = d / 2;
  const int rd = a.rotary_dim > 0 ? a.rotary_dim : d, rhalf = rd / 2;

  // Each lane holds the pairs p = lane, lane + 32, ... (up to 4 pairs: head_dim <= 256). Pair p
  // < rotary_dim/2 is the rotated pair (p, p + rotary_dim/2) by halves or (2p, 2p + 1)
  // interleaved; past the rotated elements the pairs are (2p, 2p + 1), left as they are.
  float x[4], y[4];
  int lo[4], hi[4];
  const int pairs = (half + 31) / 32;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int p = lane + 32 * j;
    const bool live = j < pairs && p < half;
    if (a.rope == 1 && p < rhalf) { lo[j] = p; hi[j] = p + rhalf; }
    else if (p < rhalf) { lo[j] = 2 * p; hi[j] = 2 * p + 1; }
    else { lo[j] = rd + 2 * (p - rhalf); hi[j] = lo[j] + 1; }
    x[j] = live ? head[lo[j]] : 0.0f;
    y[j] = live ? head[hi[j]] : 0.0f;
    if (!live) lo[j] = -1;
  }

  if (is_query || is_key) {
    const float* weight = is_query ? a.q_norm : a.k_norm;
    if (weight != nullptr) {
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += x[j] * x[j] + y[j] * y[j];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float mean = ss / float(d);
      const float inverse = 1.0f / sqrtf(mean + a.eps);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (lo[j] < 0) continue;
        x[j] = __fmul_rn(__fmul_rn(x[j], inverse), weight[lo[j]]);
        y[j] = __fmul_rn(__fmul_rn(y[j], inverse), weight[hi[j]]);
      }
    }
    if (a.rope != 0) {
      const float* cs = a.angles + int64_t(row) * rd;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = lane + 32 * j;
        if (lo[j] < 0 || p >= rhalf) continue;
        const float c = cs[p], s = cs[rhalf + p];
        const float nx = __fsub_rn(__fmul_rn(x[j], c), __fmul_rn(y[j], s));
        const float ny = __fadd_rn(__fmul_rn(y[j], c), __fmul_rn(x[j], s));
        x[j] = nx;
        y[j] = ny;
      }
    }
  }

  if (is_query) {
    if (a.q_out == nullptr) return;
    const int64_t at = int64_t(row) * a.q_out_stride + int64_t(unit) * d;
    if (a.q_out_bf16) {
      __nv_bfloat16* q = reinterpret_cast<__nv_bfloat16*>(a.q_out) + at;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (lo[j] < 0) continue;
        q[lo[j]] = __float2bfloat16_rn(x[j] * a.q_scale);
        q[hi[j]] = __float2bfloat16_rn(y[j] * a.q_scale);
      }
      return;
    }
    float* q = a.q_out + at;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (lo[j] < 0) continue;
      q[lo[j]] = x[j] * a.q_scale;
      q[hi[j]] = y[j] * a.q_scale;
    }
    return;
  }
  const KeepRow& kr = a.keep_rows[a.batch ? row : 0];
  const int position = a.batch ? kr.position : a.first + row;
  const int kv = (kunit - a.heads) % a.kv_heads;
  // KV head blocks of capacity x head_dim (KvCache::offset, transformer.rs:263-269)
  const int64_t at = (int64_t(kv) * kr.capacity + position % kr.capacity) * d;
  KT* target = static_cast<KT*>(is_key ? kr.k : kr.v) + at;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (lo[j] < 0) continue;
    target[lo[j]] = to_kv<KT>(x[j]);
    target[hi[j]] = to_kv<KT>(y[j]);
  }
}

template <typename KT>
__global__ void __launch_bounds__(kRopeWarps * 32) rope_keep_kernel(const __grid_constant__ RopeArgs a) {
  pdl_trigger();  // the attention kernel after it may be scheduled now (it waits for this one)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x;
  const int unit = blockIdx.y * kRopeWarps + warp;
  if (unit >= a.heads + a.gate_heads + 2 * a.kv_heads) return;
  rope_keep_head<KT>(a, row, unit, lane,
                     a.qkv + int64_t(row) * a.qkv_stride + int64_t(unit) * a.head_dim);
}

// head_dim 128 with the whole head rotated, no gate heads and no head norm, over 16-byte aligned
// rows: lane l holds elements 4l .. 4l + 3 of a head (one float4). RoPE by halves pairs element
// e with e + 64, which lane l + 16 holds (one shuffle); interleaved RoPE pairs neighbours within
// the float4. The arithmetic is rope_keep_head's, element for element (each product rounded,
// then the difference or sum), so the rows kept and the queries are the same bits. (A head norm
// would add its sum of squares in another order than rope_keep_head, which the fused projection
// shares: those calls stay on rope_keep_kernel.) A warp takes R rows of one head unit, all their
// loads issued before the first row is rotated.
template <typename KT>
__device__ __forceinline__ void store4(KT* p, float4 v);
template <>
__device__ __forceinline__ void store4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t*>(&a);
  w.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = w;
}

__device__ __forceinline__ float4 shfl_xor4(float4 v, int mask) {
  return make_float4(__shfl_xor_sync(0xffffffffu, v.x, mask), __shfl_xor_sync(0xffffffffu, v.y, mask),
                     __shfl_xor_sync(0xffffffffu, v.z, mask), __shfl_xor_sync(0xffffffffu, v.w, mask));
}

template <typename KT, int R>
__global__ void __launch_bounds__(kRopeWarps * 32) rope_keep128_kernel(const __grid_constant__ RopeArgs a) {
  pdl_trigger();  // the attention kernel after it may be scheduled now (it waits for this one)
  constexpr int D = 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.y * kRopeWarps + warp;
  if (unit >= a.heads + 2 * a.kv_heads) return;
  const int row0 = blockIdx.x * R;
  const bool is_query = unit < a.heads, is_key = !is_query && unit < a.heads + a.kv_heads;
  if (!is_query && !a.keep) return;
  float4 v[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (row0 + i < a.n_rows)
      v[i] = __ldcs(reinterpret_cast<const float4*>(a.qkv + int64_t(row0 + i) * a.qkv_stride +
                                                     int64_t(unit) * D) + lane);
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int row = row0 + i;
    if (row >= a.n_rows) break;  // warp-uniform
    float4 x = v[i];
    if (is_query || is_key) {
      if (a.rope == 1) {
        // pair (e, e + 64): lanes 0-15 hold the first elements, lanes 16-31 their partners
        const float* cs = a.angles + int64_t(row) * D;
        const float4 c = reinterpret_cast<const float4*>(cs)[lane & 15];
        const float4 s = reinterpret_cast<const float4*>(cs + 64)[lane & 15];
        const float4 o = shfl_xor4(x, 16);
        if (lane < 16) {
          x = make_float4(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(o.x, s.x)),
                          __fsub_rn(__fmul_rn(x.y, c.y), __fmul_rn(o.y, s.y)),
                          __fsub_rn(__fmul_rn(x.z, c.z), __fmul_rn(o.z, s.z)),
                          __fsub_rn(__fmul_rn(x.w, c.w), __fmul_rn(o.w, s.w)));
        } else {
          x = make_float4(__fadd_rn(__fmul_rn(x.x, c.x), __fmul_rn(o.x, s.x)),
                          __fadd_rn(__fmul_rn(x.y, c.y), __fmul_rn(o.y, s.y)),
                          __fadd_rn(__fmul_rn(x.z, c.z), __fmul_rn(o.z, s.z)),
                          __fadd_rn(__fmul_rn(x.w, c.w), __fmul_rn(o.w, s.w)));
        }
      } else if (a.rope != 0) {
        // pairs (2p, 2p + 1) for p = 2l, 2l + 1: cosines and sines p of the row's table
        const float* cs = a.angles + int64_t(row) * D;
        const float2 c = reinterpret_cast<const float2*>(cs)[lane];
        const float2 s = reinterpret_cast<const float2*>(cs + 64)[lane];
        x = make_float4(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, s.x)),
                        __fadd_rn(__fmul_rn(x.y, c.x), __fmul_rn(x.x, s.x)),
                        __fsub_rn(__fmul_rn(x.z, c.y), __fmul_rn(x.w, s.y)),
                        __fadd_rn(__fmul_rn(x.w, c.y), __fmul_rn(x.z, s.y)));
      }
    }
    if (is_query) {
      if (a.q_out == nullptr) continue;
      const int64_t at = int64_t(row) * a.q_out_stride + int64_t(unit) * D + 4 * lane;
      const float4 q = make_float4(x.x * a.q_scale, x.y * a.q_scale, x.z * a.q_scale, x.w * a.q_scale);
      if (a.q_out_bf16) store4<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(a.q_out) + at, q);
      else store4<float>(a.q_out + at, q);
      continue;
    }
    const KeepRow& kr = a.keep_rows[a.batch ? row : 0];
    const int position = a.batch ? kr.position : a.first + row;
    const int kv = (unit - a.heads) % a.kv_heads;
    const int64_t at = (int64_t(kv) * kr.capacity + position % kr.capacity) * D + 4 * lane;
    store4<KT>(static_cast<KT*>(is_key ? kr.k : kr.v) + at, x);
  }
}

}  // namespace fa
