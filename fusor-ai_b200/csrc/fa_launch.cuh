// Host-side launchers of the kernels, one translation unit per head_dim (fa_inst_d*.cu), so the
// instantiations compile in parallel; the C ABI (fa_attn.cu) calls these.
#pragma once

#include <cuda_runtime.h>

#include "fa_decode.cuh"
#include "fa_rope.cuh"

namespace fa {

constexpr int kKtF32 = 0;
constexpr int kKtBf16 = 1;

// One attend launch: `grid` CTAs of the (head_dim, kt, g, batch) instantiation.
struct AttendLaunch {
  int kt;                   // kKtF32 or kKtBf16: the element type of the keys and values
  int g;                    // query heads per CTA: 1, 2, 4 or 8
  bool batch;               // BatchArgs (true) or SpanArgs (false)
  const SpanArgs* span;
  const BatchArgs* rows;
  int grid;
};

template <int D>
cudaError_t launch_attend(const AttendLaunch& launch, cudaStream_t stream);

// Keys per pipeline tile of an instantiation (the chunking granularity).
inline int tile_keys(int head_dim, int kt) {
  return kTileBytes / (head_dim * (kt == kKtF32 ? 4 : 2));
}

cudaError_t launch_rope(int kt, const RopeArgs& args, cudaStream_t stream);

// Partials of fa_attend_partial: out[h] = merge over shards.
cudaError_t launch_merge_partials(const float* partials, int shards, int heads, int head_dim,
                                  float* out, cudaStream_t stream);

// Queries of a full-mask call, f32 or bf16 operand rows, scaled into q_out (rows x heads x D).
cudaError_t launch_prepare_queries(int dtype, const void* values, int64_t stride, int64_t offset,
                                   int rows, int heads, int head_dim, float scale, float* q_out,
                                   cudaStream_t stream, bool out_bf16 = false);

}  // namespace fa
