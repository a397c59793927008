// The body of one per-head_dim instantiation unit: FA_HEAD_DIM is defined by the including file.
#pragma once

#include "fa_launch.cuh"

namespace fa {

namespace {

template <int D, typename KT, int G, bool BATCH, bool PAD, typename Args>
cudaError_t launch_one(const Args& args, int grid, cudaStream_t stream) {
  auto kernel = attend_kernel<D, KT, G, BATCH, Args, PAD>;
  constexpr size_t smem = DecodeShape<D, KT, G>::kSmemBytes;
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t e = smem_limit_once(kernel, int(smem), configured);
  if (e != cudaSuccess) return e;
  return launch_pdl_cluster(kernel, dim3(grid), dim3(kDecodeThreads), smem, stream,
                            args.c.cluster > 1 ? args.c.cluster : 1, args);
}

// Head dims between the powers of two run on the next wider kernel (PAD); the narrow ones
// have no wider neighbour worth a second instantiation.
constexpr bool kPadded(int d) { return d >= 64; }

template <int D, typename KT, int G>
cudaError_t launch_g(const AttendLaunch& l, cudaStream_t stream) {
  if constexpr (kPadded(D)) {
    if (l.pad)
      return l.batch ? launch_one<D, KT, G, true, true>(*l.rows, l.grid, stream)
                     : launch_one<D, KT, G, false, true>(*l.span, l.grid, stream);
  } else if (l.pad) {
    return cudaErrorInvalidValue;
  }
  return l.batch ? launch_one<D, KT, G, true, false>(*l.rows, l.grid, stream)
                 : launch_one<D, KT, G, false, false>(*l.span, l.grid, stream);
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

template <int D, typename KT, int G, bool BATCH, typename Args, bool PAD>
int resident_one() {
  auto kernel = attend_kernel<D, KT, G, BATCH, Args, PAD>;
  constexpr size_t smem = DecodeShape<D, KT, G>::kSmemBytes;
  static std::atomic<int> cached[64];         // per instantiation, per device; 0: not asked yet
  static std::atomic<bool> configured[64];
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 0;
  int n = cached[device].load(std::memory_order_acquire);
  if (n > 0) return n;
  if (smem_limit_once(kernel, int(smem), configured) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kDecodeThreads, smem) !=
      cudaSuccess)
    return 0;
  cached[device].store(n, std::memory_order_release);
  return n;
}

template <int D, typename KT, int G>
int resident_g(const AttendLaunch& l) {
  if constexpr (kPadded(D)) {
    if (l.pad)
      return l.batch ? resident_one<D, KT, G, true, BatchArgs, true>()
                     : resident_one<D, KT, G, false, SpanArgs, true>();
  }
  return l.batch ? resident_one<D, KT, G, true, BatchArgs, false>()
                 : resident_one<D, KT, G, false, SpanArgs, false>();
}

template <int D, typename KT>
int resident_kt(const AttendLaunch& l) {
  switch (l.g) {
    case 1: return resident_g<D, KT, 1>(l);
    case 2: return resident_g<D, KT, 2>(l);
    case 4: return resident_g<D, KT, 4>(l);
    case 8: return resident_g<D, KT, 8>(l);
    default: return 0;
  }
}

}  // namespace

template <>
cudaError_t launch_attend<FA_HEAD_DIM>(const AttendLaunch& l, cudaStream_t stream) {
  return l.kt == kKtF32 ? launch_kt<FA_HEAD_DIM, float>(l, stream)
                        : launch_kt<FA_HEAD_DIM, __nv_bfloat16>(l, stream);
}

template <>
int attend_resident<FA_HEAD_DIM>(const AttendLaunch& l) {
  return l.kt == kKtF32 ? resident_kt<FA_HEAD_DIM, float>(l)
                        : resident_kt<FA_HEAD_DIM, __nv_bfloat16>(l);
}

}  // namespace fa
