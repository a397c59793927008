// The body of one per-head_dim instantiation unit: FA_HEAD_DIM is defined by the including file.
#pragma once

#include "fa_launch.cuh"

namespace fa {

namespace {

template <int D, typename KT, int G, bool BATCH, typename Args>
cudaError_t launch_one(const Args& args, int grid, cudaStream_t stream) {
  auto kernel = attend_kernel<D, KT, G, BATCH, Args>;
  constexpr size_t smem = DecodeShape<D, KT, G>::kSmemBytes;
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t e = smem_limit_once(kernel, int(smem), configured);
  if (e != cudaSuccess) return e;
  return launch_pdl_cluster(kernel, dim3(grid), dim3(kDecodeThreads), smem, stream,
                            args.c.cluster > 1 ? args.c.cluster : 1, args);
}

template <int D, typename KT, int G>
cudaError_t launch_g(const AttendLaunch& l, cudaStream_t stream) {
  return l.batch ? launch_one<D, KT, G, true>(*l.rows, l.grid, stream)
                 : launch_one<D, KT, G, false>(*l.span, l.grid, stream);
}

template <int D, typename KT>
cudaError_t launch_kt(const AttendLaunch& l, cudaStream_t stream) {
  switch (l.g) {
    case 1: return launch_g<D, KT, 1>(l, stream);
    case 2: return launch_g<D, KT, 2>(l, stream);
    case 4: return launch_g<D, KT, 4>(l, stream);
    case 8: return launch_g<D, KT, 8>(l, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

template <>
cudaError_t launch_attend<FA_HEAD_DIM>(const AttendLaunch& l, cudaStream_t stream) {
  return l.kt == kKtF32 ? launch_kt<FA_HEAD_DIM, float>(l, stream)
                        : launch_kt<FA_HEAD_DIM, __nv_bfloat16>(l, stream);
}

}  // namespace fa
