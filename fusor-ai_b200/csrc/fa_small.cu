// The small kernels around the attention: the RoPE + keep launch, query scaling for calls whose
// queries arrive already rotated, and the log-sum-exp merge of KV-range shards' partials.
#include <algorithm>

#include "fa_launch.cuh"

namespace fa {

namespace {

template <typename T>
__device__ __forceinline__ float load_elem(const T* p);
template <>
__device__ __forceinline__ float load_elem<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_elem<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// q_out[r][h][e] = scale * values[r * stride + offset + h * head_dim + e], in f32 or bf16
template <typename T, typename O>
__global__ void prepare_queries_kernel(const T* values, int64_t stride, int64_t offset, int rows,
                                       int heads, int head_dim, float scale, O* q_out) {
  const int64_t width = int64_t(heads) * head_dim;
  const int64_t total = int64_t(rows) * width;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / width, c = i % width;
    const float v = load_elem<T>(values + r * stride + offset + c) * scale;
    if constexpr (sizeof(O) == 2) q_out[i] = __float2bfloat16_rn(v);
    else q_out[i] = v;
  }
}

// The same over f32 rows whose elements start on 16-byte boundaries (values, offset and stride,
// and q_out): eight consecutive elements of a row per step of a thread, two 16-byte loads and
// one 16-byte (bf16) or two (f32) stores, the row found by one division per eight elements.
template <typename O>
__global__ void prepare_queries_vec_kernel(const float* values, int64_t stride, int64_t offset,
                                           int rows, int64_t width, float scale, O* q_out) {
  const int64_t per_row = width / 8;
  const int64_t total = int64_t(rows) * per_row;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    const float4* src = reinterpret_cast<const float4*>(values + r * stride + offset + c);
    float4 a = __ldcs(src), b = __ldcs(src + 1);
    a = make_float4(a.x * scale, a.y * scale, a.z * scale, a.w * scale);
    b = make_float4(b.x * scale, b.y * scale, b.z * scale, b.w * scale);
    if constexpr (sizeof(O) == 2) {
      const __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
      const __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
      uint4 w;
      w.x = *reinterpret_cast<const uint32_t*>(&p0);
      w.y = *reinterpret_cast<const uint32_t*>(&p1);
      w.z = *reinterpret_cast<const uint32_t*>(&p2);
      w.w = *reinterpret_cast<const uint32_t*>(&p3);
      *reinterpret_cast<uint4*>(q_out + r * width + c) = w;
    } else {
      float4* dst = reinterpret_cast<float4*>(q_out + r * width + c);
      dst[0] = a;
      dst[1] = b;
    }
  }
}

// out[h][e] = sum_s 2^(m_s - M) o_s[e] / sum_s 2^(m_s - M) l_s over the shards' partials.
__global__ void merge_partials_kernel(const float* partials, int shards, int heads, int head_dim,
                                      float* out) {
  const int h = blockIdx.x;
  const int64_t pitch = int64_t(heads) * (head_dim + 2);
  float mm = -INFINITY;
  for (int s = 0; s < shards; ++s) mm = fmaxf(mm, partials[s * pitch + h * (head_dim + 2)]);
  for (int e = threadIdx.x; e < head_dim; e += blockDim.x) {
    float ll = 0.0f, oo = 0.0f;
    for (int s = 0; s < shards; ++s) {
      const float* p = partials + s * pitch + h * (head_dim + 2);
      const float f = p[0] == -INFINITY ? 0.0f : exp2f(p[0] - mm);
      ll = fmaf(p[1], f, ll);
      oo = fmaf(p[2 + e], f, oo);
    }
    out[int64_t(h) * head_dim + e] = ll > 0.0f ? oo / ll : 0.0f;
  }
}

}  // namespace

namespace {

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// Whether rope_keep128_kernel takes the call: head_dim 128, the whole head rotated, no gate
// heads, no head norm, and every row and table it reads or writes on a 16-byte boundary.
bool rope128_fits(const RopeArgs& a) {
  if (a.head_dim != 128 || a.gate_heads != 0 || (a.rotary_dim != 0 && a.rotary_dim != 128))
    return false;
  if (a.q_norm != nullptr || a.k_norm != nullptr) return false;
  if (!aligned16(a.qkv) || a.qkv_stride % 4 != 0) return false;
  if (a.rope != 0 && !aligned16(a.angles)) return false;
  if (a.q_out != nullptr && (!aligned16(a.q_out) || a.q_out_stride % 4 != 0)) return false;
  return true;
}

template <typename KT>
cudaError_t launch_rope128(const RopeArgs& a, cudaStream_t stream) {
  const int units = a.heads + 2 * a.kv_heads;
  const unsigned ygrid = unsigned((units + kRopeWarps - 1) / kRopeWarps);
  // long spans: four rows per warp (more loads in flight per warp, a quarter of the blocks)
  if (a.n_rows >= 1024) {
    constexpr int R = 4;
    rope_keep128_kernel<KT, R><<<dim3(unsigned((a.n_rows + R - 1) / R), ygrid), kRopeWarps * 32, 0,
                                 stream>>>(a);
  } else {
    rope_keep128_kernel<KT, 1><<<dim3(unsigned(a.n_rows), ygrid), kRopeWarps * 32, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rope(int kt, const RopeArgs& args, cudaStream_t stream) {
  if (rope128_fits(args))
    return kt == kKtF32 ? launch_rope128<float>(args, stream)
                        : launch_rope128<__nv_bfloat16>(args, stream);
  const int units = args.heads + args.gate_heads + 2 * args.kv_heads;
  const dim3 grid(args.n_rows, (units + kRopeWarps - 1) / kRopeWarps);
  if (kt == kKtF32) rope_keep_kernel<float><<<grid, kRopeWarps * 32, 0, stream>>>(args);
  else rope_keep_kernel<__nv_bfloat16><<<grid, kRopeWarps * 32, 0, stream>>>(args);
  return cudaGetLastError();
}

cudaError_t launch_prepare_queries(int dtype, const void* values, int64_t stride, int64_t offset,
                                   int rows, int heads, int head_dim, float scale, float* q_out,
                                   cudaStream_t stream, bool out_bf16) {
  const int64_t total = int64_t(rows) * heads * head_dim;
  if (total == 0) return cudaSuccess;
  const int blocks = int(std::min<int64_t>((total + 255) / 256, 148 * 16));
  auto* qb = reinterpret_cast<__nv_bfloat16*>(q_out);
  const int64_t width = int64_t(heads) * head_dim;
  if (dtype == 0 && width % 8 == 0 && reinterpret_cast<uintptr_t>(values) % 16 == 0 &&
      offset % 4 == 0 && stride % 4 == 0 && reinterpret_cast<uintptr_t>(q_out) % 16 == 0) {
    auto* v = static_cast<const float*>(values);
    const int vblocks = int(std::min<int64_t>((total / 8 + 255) / 256, 148 * 16));
    if (out_bf16)
      prepare_queries_vec_kernel<<<vblocks, 256, 0, stream>>>(v, stride, offset, rows, width, scale, qb);
    else
      prepare_queries_vec_kernel<<<vblocks, 256, 0, stream>>>(v, stride, offset, rows, width, scale, q_out);
    return cudaGetLastError();
  }
  if (dtype == 0) {
    auto* v = static_cast<const float*>(values);
    if (out_bf16)
      prepare_queries_kernel<<<blocks, 256, 0, stream>>>(v, stride, offset, rows, heads, head_dim, scale, qb);
    else
      prepare_queries_kernel<<<blocks, 256, 0, stream>>>(v, stride, offset, rows, heads, head_dim, scale, q_out);
  } else {
    auto* v = static_cast<const __nv_bfloat16*>(values);
    if (out_bf16)
      prepare_queries_kernel<<<blocks, 256, 0, stream>>>(v, stride, offset, rows, heads, head_dim, scale, qb);
    else
      prepare_queries_kernel<<<blocks, 256, 0, stream>>>(v, stride, offset, rows, heads, head_dim, scale, q_out);
  }
  return cudaGetLastError();
}

cudaError_t launch_merge_partials(const float* partials, int shards, int heads, int head_dim,
                                  float* out, cudaStream_t stream) {
  merge_partials_kernel<<<heads, std::min(head_dim, 256), 0, stream>>>(partials, shards, heads,
                                                                     head_dim, out);
  return cudaGetLastError();
}

}  // namespace fa
