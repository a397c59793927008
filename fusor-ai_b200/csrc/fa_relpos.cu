// Transformer-XL relative-position attention of the conformer blocks
// (crates/blocks/src/conformer/attention.rs:25-159): for head h, query frame i and key frame j,
//   score(i, j) = ((q_i + u) . k_j + (q_i + v) . r_{frames-1-i+j}) / sqrt(head_dim),
// softmax over every key (a full mask), times v_j.
//
// One warp per (head, query) row; element e of a row lives on lane e % 32 (so every row load is
// one coalesced 128-byte access per 32 elements). Each lane sums its share of both products and
// one butterfly reduction gives the score; an online softmax in base 2 accumulates the output.
// Two keys per iteration keep two reductions in flight. The key, value and position rows are
// read through L1/L2 (a conformer's frames x head_dim rows are a few hundred KB per head).
#include <cuda_runtime.h>

#include "fa_launch.cuh"
#include "fa_relpos.h"

namespace fa {

namespace {

constexpr int kRelposWarps = 8;

template <int D>
__global__ void __launch_bounds__(kRelposWarps * 32) relpos_kernel(const RelposArgs a) {
  constexpr int E = D / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const int64_t item = int64_t(blockIdx.x) * kRelposWarps + (threadIdx.x >> 5);
  if (item >= int64_t(a.heads) * a.frames) return;
  const int h = int(item / a.frames), i = int(item % a.frames);
  const float* qrow = a.q + int64_t(i) * a.q_stride + int64_t(h) * D;
  float qu[E], qv[E], o[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float x = qrow[e * 32 + lane];
    qu[e] = x + a.bias_u[h * D + e * 32 + lane];  // the biased queries, f32 sums as the CPU
    qv[e] = x + a.bias_v[h * D + e * 32 + lane];
    o[e] = 0.0f;
  }
  const float* kbase = a.k + int64_t(h) * D;
  const float* vbase = a.v + int64_t(h) * D;
  // r_{frames-1-i+j}: the row of key j
  const float* rbase = a.positions + int64_t(a.frames - 1 - i) * a.positions_stride + int64_t(h) * D;
  float m = -INFINITY, l = 0.0f;
  auto partial = [&](int j) {
    const float* kr = kbase + int64_t(j) * a.kv_stride;
    const float* rr = rbase + int64_t(j) * a.positions_stride;
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) s = fmaf(qu[e], kr[e * 32 + lane], fmaf(qv[e], rr[e * 32 + lane], s));
    return s;
  };
  auto absorb = [&](int j, float s) {
    const float* vr = vbase + int64_t(j) * a.kv_stride;
    if (s > m) {  // warp-uniform: every lane holds the whole score
      const float alpha = exp2_approx(m - s);
      l *= alpha;
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] *= alpha;
      m = s;
    }
    const float p = exp2_approx(s - m);
    l += p;
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = fmaf(p, vr[e * 32 + lane], o[e]);
  };
  int j = 0;
  for (; j + 1 < a.frames; j += 2) {
    float s0 = partial(j), s1 = partial(j + 1);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, off);
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    }
    absorb(j, s0 * a.scale_log2);
    absorb(j + 1, s1 * a.scale_log2);
  }
  if (j < a.frames) {
    float s0 = partial(j);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s0 += __shfl_xor_sync(0xffffffffu, s0, off);
    absorb(j, s0 * a.scale_log2);
  }
  float* out = a.out + int64_t(i) * a.out_stride + int64_t(h) * D;
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) out[e * 32 + lane] = o[e] * inv;
}

}  // namespace

cudaError_t launch_relpos(const RelposArgs& a, int head_dim, cudaStream_t stream) {
  const int64_t items = int64_t(a.heads) * a.frames;
  if (items == 0) return cudaSuccess;
  const dim3 grid(unsigned((items + kRelposWarps - 1) / kRelposWarps));
  switch (head_dim) {
    case 32: relpos_kernel<32><<<grid, kRelposWarps * 32, 0, stream>>>(a); break;
    case 64: relpos_kernel<64><<<grid, kRelposWarps * 32, 0, stream>>>(a); break;
    case 128: relpos_kernel<128><<<grid, kRelposWarps * 32, 0, stream>>>(a); break;
    case 256: relpos_kernel<256><<<grid, kRelposWarps * 32, 0, stream>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace fa
