// The relative-position attention launch as the C ABI sees it (plain data, no device code).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fa {

struct RelposArgs {
  int heads, frames;
  const float* q;  // query row i at q + i * q_stride, head h at h * head_dim
  int64_t q_stride;
  const float* k;  // key / value row j at k + j * kv_stride (v likewise)
  const float* v;
  int64_t kv_stride;
  const float* positions;  // relative-position row rel (0 .. 2 frames - 2)
  int64_t positions_stride;
  const float* bias_u;  // heads * head_dim each
  const float* bias_v;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  float* out;        // row i at out + i * out_stride
  int64_t out_stride;
};

cudaError_t launch_relpos(const RelposArgs& args, int head_dim, cudaStream_t stream);

}  // namespace fa
