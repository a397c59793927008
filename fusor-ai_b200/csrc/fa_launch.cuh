// Host-side launchers of the kernels, one translation unit per head_dim (fa_inst_d*.cu), so the
// instantiations compile in parallel; the C ABI (fa_attn.cu) calls these.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <utility>

#include "fa_decode.cuh"
#include "fa_rope.cuh"

namespace fa {

// Launches `kernel` with programmatic stream serialization: its CTAs may be scheduled while the
// previous kernel of the stream (the RoPE + keep kernel, which triggers early) finishes; the
// kernel waits (pdl_wait) before it reads what that kernel wrote.
// With `cluster` > 1, consecutive groups of that many CTAs (along x) form a thread-block cluster.
template <typename... Params, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(cluster);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device, once per device
// (the attribute is per device): `done` is the caller's table of flags, one per device.
template <typename... Params>
cudaError_t smem_limit_once(void (*kernel)(Params...), int bytes, std::atomic<bool> (&done)[64]) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (done[device].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[device].store(true, std::memory_order_release);
  return e;
}

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, stream, 1, std::forward<Args>(args)...);
}

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
  bool pad = false;         // rows of AttendCommon::dh < D elements (the kernel's PAD form)
};

template <int D>
cudaError_t launch_attend(const AttendLaunch& launch, cudaStream_t stream);

// CTAs of the launch's instantiation that one SM holds at once (its shared memory and
// registers, cudaOccupancyMaxActiveBlocksPerMultiprocessor on the current device; asked once per
// device), or 0 if the runtime could not say.
template <int D>
int attend_resident(const AttendLaunch& launch);

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

// The query/key prologue of the DiT blocks (fa_prologue.cu).
constexpr int kNormNone = 0;
constexpr int kNormRow = 1;   // RMSNorm over the whole query (key) row
constexpr int kNormHead = 2;  // RMSNorm of each head
struct PrologueArgs {
  int tokens, heads, head_dim;
  int norm;          // kNorm*
  int rope;          // 0 none, 1 by halves, 2 interleaved
  int rotated_rows;  // tokens [0, rotated_rows) are rotated
  int parts;         // 2: queries and keys (in place); 3: and the values copied
  int vec_in;        // qkv rows start 16-byte aligned, widths multiples of 4
  int vec_out;       // out rows likewise (8-byte pairs for bf16)
  int out_bf16;
  const float* qkv;  // row t at qkv + t*qkv_stride: queries, keys, values of heads*head_dim
  int64_t qkv_stride;
  const float* q_norm;  // heads*head_dim (kNormRow) or head_dim (kNormHead) weights
  const float* k_norm;
  float eps;
  const float* angles;  // row t at angles + t*head_dim: cosines then sines
  void* out;            // row t at out + t*out_stride elements, laid out as qkv
  int64_t out_stride;
  unsigned* err;        // the device error word (a wait that gave up)
};
cudaError_t launch_prologue(const PrologueArgs& args, cudaStream_t stream);

// The sigmoid gate of the hybrid blocks' attention output (fa_prologue.cu).
struct GateArgs {
  int rows, heads, head_dim;
  int per_head;         // one gate per query head (else one per element)
  const float* qkv;     // gates at qkv + r*qkv_stride + gate_offset
  int64_t qkv_stride;
  int64_t gate_offset;
  float* out;
  int64_t out_stride;
};
cudaError_t launch_gate(const GateArgs& args, cudaStream_t stream);

// The QKV projection fused with head norm, RoPE and keep (fa_project.cu). The RopeArgs give the
// epilogue (its qkv is not read; gate_heads must be 0); grid (head units, row blocks, splits).
struct ProjectArgs {
  const float* x;        // row r at x + r*x_stride: hidden values
  int64_t x_stride;
  const float* weight;   // output column c at weight + c*w_stride: hidden values
  int64_t w_stride;
  const float* bias;     // (heads + 2 kv_heads) x head_dim values, or nullptr
  int hidden, rows;
  int row_block;         // rows per CTA, a multiple of the rows per pass
  int splits, chunk;     // splits of the hidden dimension, chunk values each (a multiple of 128)
  float* partials;       // [unit][row block][split][row_block][head_dim] when splits > 1
  int* counters;         // [unit][row block], zero between launches
  float* qkv_out;        // optional: the projected rows, before head norm and RoPE
  int64_t qkv_out_stride;
};
// nr: rows per pass (1, 4 or 8); smem: (row_block x chunk + row_block x head_dim) floats.
cudaError_t launch_project(int kt, int nr, const ProjectArgs& p, const RopeArgs& r, size_t smem,
                           cudaStream_t stream);

// The qkv projection of many rows on the tensor cores (fa_project_tc.cu): qkv = x . W^T + b in
// three tf32 products, the hidden dimension in `splits` ranges.
struct ProjectTcArgs {
  const float* x;        // row r at x + r*x_stride: hidden values (16-byte aligned rows)
  int64_t x_stride;
  const float* weight;   // output column c at weight + c*w_stride (16-byte aligned rows)
  int64_t w_stride;
  const float* bias;     // outputs values, or nullptr
  int hidden, outputs, rows;
  int k_blocks;          // (hidden + 31) / 32
  int splits;            // 1 to 8, at most k_blocks: the CTAs of a tile
  float* qkv;            // row r at qkv + r*qkv_stride
  int64_t qkv_stride;
  float* partials;       // splits > 1: [tile][split][rows per tile][128] floats
  int* counters;         // splits > 1: one per tile (column block x row tile), zero between launches
  unsigned* err;
};
// Rows per CTA tile (the MMA's N) for `rows` rows: 16, 32 or 64.
int project_tc_rows_per_tile(int rows);
cudaError_t launch_project_tc(const ProjectTcArgs& args, cudaStream_t stream);

// The tensor-core decode over bf16 caches of head_dim 128 or 256 (fa_decode_tc.cu): `grid`
// persistent CTAs.
struct DtcArgs;
cudaError_t launch_decode_tc(const DtcArgs& args, int head_dim, int grid, cudaStream_t stream);

}  // namespace fa
