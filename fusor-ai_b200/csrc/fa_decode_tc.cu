// Host side of the tensor-core decode (fa_decode_tc.cuh): its launch.
#include <cuda_runtime.h>

#include "fa_decode_tc.cuh"
#include "fa_launch.cuh"

namespace fa {

namespace {

template <int D, int kG>
cudaError_t launch_g(const DtcArgs& args, int grid, cudaStream_t stream) {
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t e = smem_limit_once(decode_tc_kernel<D, kG>, int(dtc_smem_bytes(D)), configured);
  if (e != cudaSuccess) return e;
  return launch_pdl(decode_tc_kernel<D, kG>, dim3(grid), dim3(kDtcThreads), dtc_smem_bytes(D),
                    stream, args);
}

template <int D>
cudaError_t launch_d(const DtcArgs& args, int grid, cudaStream_t stream) {
  if (args.group <= 1) return launch_g<D, 1>(args, grid, stream);
  if (args.group <= 2) return launch_g<D, 2>(args, grid, stream);
  if (args.group <= 4) return launch_g<D, 4>(args, grid, stream);
  if (args.group <= 8) return launch_g<D, 8>(args, grid, stream);
  if (args.group <= 16) return launch_g<D, 16>(args, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_decode_tc(const DtcArgs& args, int head_dim, int grid, cudaStream_t stream) {
  if (head_dim == 128) return launch_d<128>(args, grid, stream);
  if (head_dim == 256) return launch_d<256>(args, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fa
