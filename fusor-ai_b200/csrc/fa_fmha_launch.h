// The tcgen05 attention launch as the C ABI sees it (no CUDA device code in this header).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fa_ptx.cuh"

namespace fa {

// The tcgen05 kernel's arguments (kernel parameter; plain data).
struct FmhaArgs {
  int heads, kv_heads, group;
  int rows;            // valid query rows per image
  int images;
  int q_tiles;         // query tiles per image
  // key positions of a row: mask kind over positions first + r (cache path); for a full-mask
  // call kind is Full with end = keys
  int first, end, kind, window, state, n_ends;
  int ends[kMaxEnds];
  int q_row_base_per_image;   // Q rows of image i start at i * this (TMA y coordinate)
  int kv_row_base_per_image;  // K/V rows of image i start at i * this
  int kv_layer_base;          // TMA z of kv head 0 (layer * kv_heads for a cache)
  float scale_log2;           // log2(e) / sqrt(head_dim)
  void* out;                  // row (image * rows + r) at out + that * out_stride
  int64_t out_stride;
  int out_bf16;
  unsigned* err;
  // The two-tile kernel's schedule: units (query head, pair of query tiles), head-major; units
  // [0, whole_units) run whole, one CTA each, and with splits > 1 every later unit runs as
  // `splits` consecutive CTAs over equal shares of its KV tiles. A piece writes its rows'
  // (max, sum, unnormalised O) to part_ml / part_o (slot (tail unit x splits + piece) x 256 +
  // row of the pair); each of its 8 softmax warps counts itself in counters[tail unit x 8 +
  // warp], and the warp of the last piece to arrive merges its 32 rows, writes them out and sets
  // the counter back to zero.
  int whole_units;
  int splits;
  // 1: without splits, units run pair-major, the heaviest pairs of every head first
  int pair_major;
  // The one-tile kernel's schedule: a 1-D grid over bands of band_heads query heads (whole KV
  // groups, consecutive heads), band after band; within a band the query tiles run heaviest
  // first (later rows, for causal masks), the band's heads fastest. 0: one KV group per band.
  int band_heads;
  float* part_o;
  float* part_ml;
  int* counters;
};

constexpr int kFmhaMaxSplits = 8;


// Q, K and V as 3-D tensors of [z][row][head_dim] elements for the TMA maps: Q rows are query
// rows and z its query heads; K/V rows are key positions and z (layer x) KV heads.
struct FmhaLaunch {
  int bf16;      // operands bf16 (kind::f16) or f32 (kind::tf32)
  int head_dim;  // 64 or 128, or 256 for bf16
  const void* q;
  uint64_t q_rows, q_heads;
  uint64_t q_row_stride, q_head_stride;  // elements
  const void* k;
  const void* v;
  uint64_t kv_rows, kv_z;
  uint64_t kv_row_stride, kv_z_stride;   // elements
  const FmhaArgs& args;
};

bool fmha_supported(int dtype_bf16, int head_dim);
// Whether launch_fmha honours FmhaArgs::splits for these operands (the two-tile bf16 kernel).
bool fmha_splits_supported(int dtype_bf16, int head_dim);
// A TMA map (written to the 128 bytes at `map`, 64-byte aligned) over a bf16 cache's keys or
// values: [z][rows][head_dim] elements, z_stride_bytes apart, 64 x 128 boxes, 128-byte swizzle
// (the tensor-core decode's K and V tiles).
bool encode_cache_map_bf16(void* map, const void* base, uint64_t head_dim, uint64_t rows,
                           uint64_t z, uint64_t z_stride_bytes);
// A TMA map over a 2-D f32 array [y][x] (rows y_stride_bytes apart) with box_x x box_y boxes,
// 128-byte swizzled (box_x = 32), zero fill past the edges.
bool encode_map_f32(void* map, const void* base, uint64_t x, uint64_t y, uint64_t y_stride_bytes,
                    uint32_t box_x, uint32_t box_y);
int fmha_block_n(int dtype_bf16, int head_dim);
cudaError_t launch_fmha(const FmhaLaunch& launch, cudaStream_t stream);

}  // namespace fa
