// Host side of the tcgen05 attention kernel: TMA tensor maps (encoded through the driver entry
// point, so the library needs no link-time libcuda) and the launches of its instantiations.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "fa_fmha.cuh"
#include "fa_fmha2.cuh"
#include "fa_launch.cuh"
#include "fa_fmha_launch.h"

namespace fa {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// A 3-D map over [z][y][x] elements (x innermost, contiguous) with byte strides for y and z and
// a box of (box_x, box_y, 1), 128-byte swizzled.
bool make_map(CUtensorMap* map, bool bf16, const void* base, uint64_t x, uint64_t y, uint64_t z,
              uint64_t y_stride_bytes, uint64_t z_stride_bytes, uint32_t box_x, uint32_t box_y,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {x, y, z};
  const cuuint64_t strides[2] = {y_stride_bytes, z_stride_bytes};
  const cuuint32_t box[3] = {box_x, box_y, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int D>
cudaError_t launch_t(const FmhaLaunch& l, cudaStream_t stream) {
  using S = FmhaShape<T, D>;
  constexpr bool bf16 = sizeof(T) == 2;
  const size_t e = sizeof(T);
  CUtensorMap qm, km, vm;
  if (!make_map(&qm, bf16, l.q, D, l.q_rows, l.q_heads, l.q_row_stride * e, l.q_head_stride * e,
                S::kBlock, S::BM) ||
      !make_map(&km, bf16, l.k, D, l.kv_rows, l.kv_z, l.kv_row_stride * e, l.kv_z_stride * e,
                S::kBlock, S::BN) ||
      !make_map(&vm, bf16, l.v, D, l.kv_rows, l.kv_z, l.kv_row_stride * e, l.kv_z_stride * e,
                S::kBlock, S::BN,
                bf16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return cudaErrorInvalidValue;
  auto kernel = fmha_kernel<T, D>;
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t err = smem_limit_once(kernel, int(S::kSmemBytes), configured);
  if (err != cudaSuccess) return err;
  const int band = l.args.band_heads > 0 ? l.args.band_heads : l.args.group;
  if (band % l.args.group || l.args.heads % band) return cudaErrorInvalidValue;
  const int64_t grid = int64_t(l.args.images) * l.args.q_tiles * l.args.heads;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  return launch_pdl(kernel, dim3(unsigned(grid)), dim3(fmha_threads<T, D>()), S::kSmemBytes, stream, qm,
                    km, vm, l.args);
}

// bf16: two query tiles per CTA (fa_fmha2.cuh).
template <int D>
cudaError_t launch_bf16_pairs(const FmhaLaunch& l, cudaStream_t stream) {
  using S = Fmha2Shape<D>;
  CUtensorMap qm, km, vm;
  if (!make_map(&qm, true, l.q, D, l.q_rows, l.q_heads, l.q_row_stride * 2, l.q_head_stride * 2,
                S::kBlock, S::BM) ||
      !make_map(&km, true, l.k, D, l.kv_rows, l.kv_z, l.kv_row_stride * 2, l.kv_z_stride * 2,
                S::kBlock, S::BN) ||
      !make_map(&vm, true, l.v, D, l.kv_rows, l.kv_z, l.kv_row_stride * 2, l.kv_z_stride * 2,
                S::kBlock, S::BN))
    return cudaErrorInvalidValue;
  auto kernel = fmha2_kernel<D>;
  static std::atomic<bool> configured[64];  // per instantiation, per device
  cudaError_t err = smem_limit_once(kernel, int(S::kSmemBytes), configured);
  if (err != cudaSuccess) return err;
  const int64_t units = int64_t(l.args.images) * ((l.args.q_tiles + 1) / 2) * l.args.heads;
  int64_t grid = units;
  if (l.args.splits > 1) {
    if (l.args.splits > kFmhaMaxSplits || l.args.whole_units < 0 || l.args.whole_units > units ||
        l.args.part_o == nullptr || l.args.part_ml == nullptr || l.args.counters == nullptr)
      return cudaErrorInvalidValue;
    grid = l.args.whole_units + (units - l.args.whole_units) * l.args.splits;
  }
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  return launch_pdl(kernel, dim3(unsigned(grid)), dim3(kFmha2Threads), S::kSmemBytes, stream, qm,
                    km, vm, l.args);
}

}  // namespace

bool encode_cache_map_bf16(void* map, const void* base, uint64_t head_dim, uint64_t rows,
                           uint64_t z, uint64_t z_stride_bytes) {
  return make_map(static_cast<CUtensorMap*>(map), true, base, head_dim, rows, z, head_dim * 2,
                  z_stride_bytes, 64, 128);
}

bool encode_map_f32(void* map, const void* base, uint64_t x, uint64_t y, uint64_t y_stride_bytes,
                    uint32_t box_x, uint32_t box_y) {
  return make_map(static_cast<CUtensorMap*>(map), false, base, x, y, 1, y_stride_bytes,
                  y * y_stride_bytes, box_x, box_y);
}

bool fmha_supported(int dtype_bf16, int head_dim) {
  const bool dim = head_dim == 64 || head_dim == 128 || (head_dim == 256 && dtype_bf16);
  return dim && encode_fn() != nullptr;
}

bool fmha_splits_supported(int dtype_bf16, int head_dim) {
#ifdef FA_FMHA_ONE_TILE
  (void)dtype_bf16;
  (void)head_dim;
  return false;
#else
  return dtype_bf16 != 0 && head_dim != 256;  // head_dim 256 runs one query tile per CTA
#endif
}

int fmha_block_n(int dtype_bf16, int head_dim) {
  return (head_dim == 256 || (!dtype_bf16 && head_dim == 128)) ? 64 : 128;
}

cudaError_t launch_fmha(const FmhaLaunch& l, cudaStream_t stream) {
  if (l.bf16) {
#ifdef FA_FMHA_ONE_TILE
    if (l.head_dim == 64) return launch_t<__nv_bfloat16, 64>(l, stream);
    if (l.head_dim == 128) return launch_t<__nv_bfloat16, 128>(l, stream);
#else
    if (l.head_dim == 64) return launch_bf16_pairs<64>(l, stream);
    if (l.head_dim == 128) return launch_bf16_pairs<128>(l, stream);
#endif
    // two query tiles of head_dim 256 (S and O for each) do not fit in TMEM's 512 columns
    if (l.head_dim == 256) return launch_t<__nv_bfloat16, 256>(l, stream);
  } else {
    if (l.head_dim == 64) return launch_t<float, 64>(l, stream);
    if (l.head_dim == 128) return launch_t<float, 128>(l, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fa
