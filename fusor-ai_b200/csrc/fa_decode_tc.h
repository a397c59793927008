// The tensor-core decode's launch arguments (the kernel: fa_decode_tc.cuh).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "fa_ptx.cuh"

namespace fa {

constexpr int kDtcD = 128;      // head_dim block of a ring entry (the M of O^T)
constexpr int kDtcKeys = 128;   // keys per tile (the M of S^T)
constexpr int kDtcN = 16;       // query heads per KV head, padded (the N of both products)
constexpr int kDtcStages = 3;
constexpr int kDtcThreads = 224;
constexpr int kDtcTileBytes = kDtcKeys * kDtcD * 2;   // one ring entry: 128 keys x 128 head_dim
constexpr int kDtcPBytes = kDtcN * kDtcKeys * 2;      // one P^T buffer: 16 rows x 256 B
constexpr int kDtcMergeBytes = 4096;
// K ring entries, of the 2 x kDtcStages the K and V rings share. At head_dim 256 a tile is two
// entries of each, and the V ring, whose tiles wait two tiles for their P.V, takes four: measured
// on B200 (`decode256`), K/V entries 3/3 0.109 ms, 4/2 0.108, 2/4 0.106.
__host__ __device__ constexpr int dtc_k_stages(int head_dim) {
  return head_dim == 256 ? 2 : kDtcStages;
}
// Q^T: 16 rows x head_dim bf16
__host__ __device__ constexpr int dtc_q_bytes(int head_dim) { return kDtcN * head_dim * 2; }
// K and V stages, two Q^T buffers, three P^T buffers, the merge's weights
__host__ __device__ constexpr size_t dtc_smem_bytes(int head_dim) {
  return size_t(2 * kDtcStages) * kDtcTileBytes + 2 * size_t(dtc_q_bytes(head_dim)) +
         3 * size_t(kDtcPBytes) + kDtcMergeBytes + 1024 /* alignment */ + 512 /* barriers */;
}

// One decode row: its cache's key and value tensor maps (device CUtensorMap, 64-byte aligned:
// [layers x kv_heads][capacity][head_dim] bf16, 64 x 128 boxes, 128-byte swizzle) and its keys,
// the cache slots b0 .. b0 + n - 1 (one run, no ring wrap).
struct DtcRow {
  const void* kmap;
  const void* vmap;
  int z0;          // layer * kv_heads
  int b0, n;
  int chunks;      // chunks of chunk_keys keys
  int unit_begin;  // first unit of this row: units are (kv head, chunk), kv head major
  int part_base;   // first partial chunk slot of this row
};

constexpr int kDtcMaxCtas = 160;     // persistent CTAs (one per SM)
constexpr int kDtcMaxUnits = 4096;   // units of one launch

struct DtcArgs {
  int heads, kv_heads, group;  // group <= kDtcN
  int n_rows, n_units;
  int chunk_keys;              // a multiple of kDtcKeys
  const float* q;              // rotated queries, row r at q + r * q_stride (heads x head_dim, f32)
  int64_t q_stride;
  float scale_log2;            // log2(e) / sqrt(head_dim)
  float* out;
  int64_t out_stride;
  float* part_o;               // chunk partials: slot (part_base + chunk) * heads + head
  float* part_ml;
  int* counters;               // per (row, kv head), zero between launches
  unsigned* err;
  DtcRow rows[kMaxBatchRows];
  // The schedule: CTA c takes units order[cta_first[c]] .. order[cta_first[c + 1] - 1], the
  // units dealt longest first to the least loaded CTA (each CTA's list longest first).
  uint16_t cta_first[kDtcMaxCtas + 1];
  uint16_t order[kDtcMaxUnits];
};
static_assert(sizeof(DtcArgs) <= 32764, "kernel parameters");

}  // namespace fa
