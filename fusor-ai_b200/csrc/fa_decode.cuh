// The memory-bound half of the hot path: RoPE + keep (Stack::attention_input, layer.rs:175-234;
// KvCache::keep, transformer.rs:164-180) and flash-decoding attention over the KvCache
// (KvCache::attend, transformer.rs:182-219, with ops::attend's arithmetic, ops.rs:310-342).
//
// attend_kernel: one CTA per (query row, KV head and up to G of its query heads, chunk of keys).
//  - A producer warp streams the chunk's key and value rows from HBM into a ring of shared-memory
//    stages with 1-D bulk copies (cp.async.bulk, completion counted on an mbarrier). The cache
//    keeps the reference's layout [layer][kv_head][slot][head_dim], so a run of positions is one
//    contiguous copy; a run that wraps a window ring, or crosses into Mask::Groups's second run,
//    is split into pieces.
//  - Four consumer warps score each key against the G query heads that share it (GQA reuse the
//    CPU path lacks: it re-reads the KV head once per query head), LPK lanes per key with 8
//    (16 for a bf16 cache) elements each, warp-shuffle reductions and an online softmax in base 2 (the queries are
//    scaled by log2(e)/sqrt(head_dim) as they are loaded).
//  - The warps' (max, sum, output) states merge in shared memory; a single-chunk row writes its
//    output, otherwise the chunk's partial goes to the workspace and the last CTA of the row
//    (an arrival counter, reset by that CTA) merges the partials by log-sum-exp.
#pragma once

#include "fa_ptx.cuh"

namespace fa {

// Shape of the split-KV CTA (compile-time tunables; the defaults are the measured best).
#ifndef FA_DECODE_WARPS
#define FA_DECODE_WARPS 4
#endif
#ifndef FA_DECODE_STAGES
#define FA_DECODE_STAGES 2
#endif
#ifndef FA_DECODE_TILE_BYTES
#define FA_DECODE_TILE_BYTES 16384
#endif
#ifndef FA_DECODE_MIN_CTAS
#define FA_DECODE_MIN_CTAS 3
#endif
constexpr int kConsumerWarps = FA_DECODE_WARPS;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = FA_DECODE_STAGES;
constexpr int kTileBytes = FA_DECODE_TILE_BYTES;  // bytes of one K (or V) tile of a stage
// Where a clustered chunk leaves its (max, sum, o) state: past the warps' merge scratch
// (<= 4 warps x 8 heads x (256 + 2) floats) in the stages' memory.
constexpr int kClusterPartialOffset = 40960;
// Chunks of a row merged within one thread-block cluster (the portable cluster size).
constexpr int kMaxClusterChunks = 8;

// Mask::keys (transformer.rs:116-128): the key positions of a row as two runs.
struct Runs {
  int b0, n0, b1, n1;
};

__host__ __device__ inline Runs mask_runs(int kind, int window, int state, int n_ends,
                                          const int* ends, int position, int end) {
  Runs r{0, 0, 0, 0};
  if (kind == 0) {  // Causal
    r.n0 = position + 1;
  } else if (kind == 1) {  // Window
    int lo = position + 1 - window;
    if (lo < 0) lo = 0;
    r.b0 = lo;
    r.n0 = position + 1 - lo;
  } else if (kind == 2 || position < state) {  // Full, or Groups before the state
    r.n0 = end;
  } else {  // Groups: the state, then the row's own group
    int g = 0;
    while (g < n_ends && ends[g] <= position) ++g;
    const int start = g == 0 ? state : ends[g - 1];
    r.n0 = state;
    r.b1 = start;
    r.n1 = (g < n_ends ? ends[g] : end) - start;
  }
  return r;
}

// The bits of key word `w` (keys kp + 32w .. kp + 32w + 31) that lie in [b, b + n).
__device__ __forceinline__ uint32_t run_word(int b, int n, int kp, int w) {
  const int base = kp + 32 * w;
  const int lo = min(max(b - base, 0), 32), hi = min(max(b + n - base, 0), 32);
  const uint32_t below_hi = hi >= 32 ? 0xffffffffu : (1u << hi) - 1u;
  const uint32_t below_lo = lo >= 32 ? 0xffffffffu : (1u << lo) - 1u;
  return below_hi & ~below_lo;
}

// Sets to -inf the scores s[0..N) of the keys kp .. kp + N - 1 that neither run of `r` covers:
// the runs become a bit mask once per 32 keys, so a key costs a bit test and a select.
template <int N>
__device__ __forceinline__ void mask_scores(const Runs& r, int kp, float* s) {
#pragma unroll
  for (int w = 0; w < N / 32; ++w) {
    const uint32_t bits = run_word(r.b0, r.n0, kp, w) | run_word(r.b1, r.n1, kp, w);
#pragma unroll
    for (int c = 0; c < 32; ++c)
      if (!((bits >> c) & 1u)) s[32 * w + c] = -INFINITY;
  }
}

template <typename KT>
struct KvElem;
template <>
struct KvElem<float> {
  static constexpr int kBytes = 4;
};
template <>
struct KvElem<__nv_bfloat16> {
  static constexpr int kBytes = 2;
};

// Elements of a key (value) row each lane holds: 8, or 16 for a bf16 cache with at most 4 query
// heads per CTA (twice the work per shuffle of the score reductions: a bf16 row carries half
// the bytes of an f32 row for the same arithmetic, so its CTA must issue fewer instructions per
// byte to keep up with HBM; more heads would spill the registers).
#ifndef FA_DECODE_BF16_EPL
#define FA_DECODE_BF16_EPL 16
#endif
#ifndef FA_DECODE_BF16_MIN_CTAS
#define FA_DECODE_BF16_MIN_CTAS 2
#endif
template <int D, typename KT, int G>
struct LaneElems {
  static constexpr int value =
      (KvElem<KT>::kBytes == 2 && G <= 4 && D / FA_DECODE_BF16_EPL >= 2) ? FA_DECODE_BF16_EPL : 8;
};

template <int D, typename KT, int G>
struct DecodeShape {
  static constexpr int kRowBytes = D * KvElem<KT>::kBytes;
  static constexpr int kLaneElems = LaneElems<D, KT, G>::value;
  static constexpr int kLanesPerKey = D / kLaneElems;
  static constexpr int kKeysPerWarp = 32 / kLanesPerKey;
  static constexpr int kTileKeys = kTileBytes / kRowBytes;
  static constexpr int kRoundKeys = kConsumerWarps * kKeysPerWarp;
  static constexpr int kRounds = kTileKeys / kRoundKeys;
  static constexpr int kElemsPerTile = kTileKeys * D;
  // resident CTAs per SM the registers are sized for: 16 elements per lane, or 8 query heads,
  // need more than a third of the register file per CTA
  static constexpr int kMinCtas =
      (kLaneElems == 16 || G >= 8) ? FA_DECODE_BF16_MIN_CTAS : FA_DECODE_MIN_CTAS;
  static_assert(kLanesPerKey >= 2 && kLanesPerKey <= 32, "head_dim 16..256");
  static_assert(kRounds * kRoundKeys == kTileKeys, "tile holds whole rounds");
  static constexpr size_t kSmemBytes = size_t(kStages) * 2 * kTileBytes + 2 * kStages * 8;
  // the warps' (max, sum, o) merge reuses the stages' memory, and so does a clustered chunk's
  // state past it
  static_assert(size_t(kConsumerWarps) * 8 * (D + 2) * 4 <= size_t(kClusterPartialOffset),
                "the merge scratch fits below the cluster state");
  static_assert(size_t(kClusterPartialOffset) + size_t(G) * (D + 2) * 4 <=
                    size_t(kStages) * 2 * kTileBytes,
                "the cluster state fits the stages");
};

// The element index of lane-slot i (0..E-1) of sub-lane `sub` in a row, LPK = D / E lanes per
// row: f32 rows are read as two float4 at sub and sub + LPK, bf16 rows as one 16-byte vector at
// sub (E = 8) or two at sub and sub + LPK (E = 16); either way each group of 8 lanes reads 128
// contiguous bytes of shared memory (no bank conflicts).
template <int D, typename KT, int E>
__device__ __forceinline__ int elem_of(int sub, int i) {
  constexpr int LPK = D / E;
  if constexpr (KvElem<KT>::kBytes == 4) {
    return i < 4 ? 4 * sub + i : 4 * (sub + LPK) + (i - 4);
  } else if constexpr (E == 8) {
    return 8 * sub + i;
  } else {
    return i < 8 ? 8 * sub + i : 8 * (sub + LPK) + (i - 8);
  }
}

// bf16 pairs of a 32-bit word as an f32 pair (the low element first).
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ void unpack_bf16x8(const uint4 a, float2* x) {
  x[0] = bf16x2_to_float2(a.x);
  x[1] = bf16x2_to_float2(a.y);
  x[2] = bf16x2_to_float2(a.z);
  x[3] = bf16x2_to_float2(a.w);
}

// A lane's E elements of a row as E/2 f32 pairs, pair i = elements (elem_of(2i), elem_of(2i+1)).
template <int D, typename KT, int E>
__device__ __forceinline__ void load_lane(const KT* row, int sub, float2 (&x)[E / 2]) {
  constexpr int LPK = D / E;
  if constexpr (KvElem<KT>::kBytes == 4) {
    static_assert(E == 8, "f32 rows: 8 elements per lane");
    const float4 a = reinterpret_cast<const float4*>(row)[sub];
    const float4 b = reinterpret_cast<const float4*>(row)[sub + LPK];
    x[0] = make_float2(a.x, a.y);
    x[1] = make_float2(a.z, a.w);
    x[2] = make_float2(b.x, b.y);
    x[3] = make_float2(b.z, b.w);
  } else if constexpr (E == 8) {
    unpack_bf16x8(reinterpret_cast<const uint4*>(row)[sub], x);
  } else {
    unpack_bf16x8(reinterpret_cast<const uint4*>(row)[sub], x);
    unpack_bf16x8(reinterpret_cast<const uint4*>(row)[sub + LPK], x + 4);
  }
}

// Two f32 lanes at once (sm_100a's paired FFMA/FMUL; each lane rounds as fmaf / __fmul_rn).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }

template <int N>
struct Log2 {
  static constexpr int value = N <= 1 ? 0 : 1 + Log2<N / 2>::value;
};
template <>
struct Log2<1> {
  static constexpr int value = 0;
};

// What every attend launch shares.
struct AttendCommon {
  int heads, kv_heads, group, hgroups;  // hgroups: CTAs per KV head (ceil(group / G))
  int64_t kv_stride;                    // elements between consecutive KV heads' blocks
  int64_t key_stride;                   // elements between consecutive key (value) rows
  const float* q;                       // rotated queries: row r at q + r*q_stride
  int64_t q_stride;
  float q_scale;                        // log2(e)/sqrt(head_dim): scores in base-2 units
  float* out;  // output row r at out + r*out_stride (heads x D), or nullptr for partial_out
  int64_t out_stride;
  float* partial_out;  // when out is nullptr: row r's merged (max, sum, o[D]) per head
  float* part_o;   // chunk partials: slot (part_base + chunk) * heads + head, D floats each
  float* part_ml;  // (max, sum) per slot
  int* counters;   // per (row, kv group) arrival counters, zero between launches
  unsigned* err;   // device error word
  int cluster;     // spans: a row's chunks are one thread-block cluster (merged in shared memory)
  int dh;          // the rows' head_dim: D, or fewer on a kernel of a wider D (PAD)
};

// One span over one cache: row r at position first + r, keys from the mask.
struct SpanArgs {
  AttendCommon c;
  const void* k;  // keys of (layer, kv head 0)
  const void* v;
  int capacity;
  int rows, first, end, kind, window, state, n_ends, chunks;
  int rows_per_image;  // rows of one image (images attend within themselves: full-mask calls)
  int keys_per_image;  // key rows between consecutive images
  int ends[kMaxEnds];
};

// Independent rows (decode sequences), each with its own cache and key runs.
struct BatchRow {
  const void* k;
  const void* v;
  int capacity;
  Runs runs;
  int chunks;      // chunks of this row
  int unit_begin;  // first CTA of this row
  int part_base;   // first partial chunk slot of this row
};
struct BatchArgs {
  AttendCommon c;
  int n;
  BatchRow rows[kMaxBatchRows];
};

// The log-sum-exp merge of one row's `chunks` partials (slot (part_base + chunk) * heads + head:
// D floats of unnormalised output, and (max, sum) in base 2) for query heads h0 .. h0 + g - 1,
// by the kThreads threads (tid 0 .. kThreads - 1) of named barrier `bar`, in the last CTA of
// the row to arrive. Each head's largest chunk max M and sum L = sum 2^(m - M) l take one warp
// per head over the chunks; the outputs sum 2^(m - M) o over the chunks with the weights staged
// in shared memory (`wts`, room for cap_chunks x G floats), each thread's output elements'
// loads of several chunks in flight. finish(h, e, M, L, o) stores element e of head h0 + h.
template <int G, int D, int kThreads, typename Finish>
__device__ __forceinline__ void merge_chunk_partials(const float* part_o, const float* part_ml,
                                                     int heads, int h0, int g, int part_base,
                                                     int chunks, float* wts, int cap_chunks,
                                                     int bar, int tid, Finish finish) {
  __shared__ float merge_m[G], merge_l[G];
  const int warp = tid >> 5, lane = tid & 31;
  const int64_t base = int64_t(part_base) * heads + h0;  // slot of (chunk 0, head h0)
  for (int h = warp; h < g; h += kThreads / 32) {
    float mm = -INFINITY;
#pragma unroll 8
    for (int ch = lane; ch < chunks; ch += 32)
      mm = fmaxf(mm, __ldcg(&part_ml[2 * (base + int64_t(ch) * heads + h)]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, off));
    float ll = 0.0f;
#pragma unroll 8
    for (int ch = lane; ch < chunks; ch += 32) {
      const int64_t slot = base + int64_t(ch) * heads + h;
      const float cm = __ldcg(&part_ml[2 * slot]);
      const float f = cm == -INFINITY ? 0.0f : exp2_approx(cm - mm);
      ll = fmaf(__ldcg(&part_ml[2 * slot + 1]), f, ll);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ll += __shfl_xor_sync(0xffffffffu, ll, off);
    if (lane == 0) {
      merge_m[h] = mm;
      merge_l[h] = ll;
    }
  }
  named_sync(bar, kThreads);
  constexpr int kPer = (G * D + kThreads - 1) / kThreads;  // output elements per thread
  const int count = g * D;
  float acc[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) acc[j] = 0.0f;
  for (int cb = 0; cb < chunks; cb += cap_chunks) {
    const int nb = min(cap_chunks, chunks - cb);
    for (int i = tid; i < nb * g; i += kThreads) {
      const int k = i / g, h = i % g;
      const float cm = __ldcg(&part_ml[2 * (base + int64_t(cb + k) * heads + h)]);
      wts[k * G + h] = cm == -INFINITY ? 0.0f : exp2_approx(cm - merge_m[h]);
    }
    named_sync(bar, kThreads);
    // the loads of 16 chunks in flight per thread (the partials are in L2: each trip is its
    // latency, and a row split 222 ways otherwise took 56 trips at the end of the launch)
#pragma unroll 16
    for (int k = 0; k < nb; ++k) {
      const float* po = part_o + (base + int64_t(cb + k) * heads) * D;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int idx = tid + j * kThreads;
        if (idx < count) acc[j] = fmaf(__ldcg(&po[idx]), wts[k * G + idx / D], acc[j]);
      }
    }
    named_sync(bar, kThreads);
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int idx = tid + j * kThreads;
    if (idx < count) finish(idx / D, idx % D, merge_m[idx / D], merge_l[idx / D], acc[j]);
  }
}

// PAD: the rows hold dh < D elements (a head_dim between the powers of two, dh a multiple of
// the 16-byte vectors: 4 for f32, 8 for bf16); they stream and sit in shared memory dh apart, the
// lanes' vectors past dh are zero, and only elements below dh are written out. The tile stays T
// rows of the D layout (fewer bytes).
template <int D, typename KT, int G, bool BATCH, typename Args, bool PAD = false>
__global__ void __launch_bounds__(kDecodeThreads, (DecodeShape<D, KT, G>::kMinCtas)) attend_kernel(const __grid_constant__ Args args) {
  using S = DecodeShape<D, KT, G>;
  constexpr int E = S::kLaneElems;
  constexpr int T = S::kTileKeys;
  constexpr int LPK = S::kLanesPerKey;
  constexpr int KPW = S::kKeysPerWarp;
  const AttendCommon& c = args.c;
  const int RD = PAD ? c.dh : D;  // elements of a row (its stride in the cache and in a tile)
  const uint32_t row_bytes = uint32_t(RD) * KvElem<KT>::kBytes;

  extern __shared__ __align__(128) unsigned char smem[];
  KT* k_tiles = reinterpret_cast<KT*>(smem);
  KT* v_tiles = reinterpret_cast<KT*>(smem + size_t(kStages) * kTileBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kStages) * 2 * kTileBytes);
  uint64_t* empty = full + kStages;
  __shared__ int last_flag;
  __shared__ int fail_flag;

  // ---- which work unit this CTA is -----------------------------------------------------------
  const int unit = blockIdx.x;
  int row, kvg, chunk, chunks, capacity, part_base;
  Runs runs;
  const KT* kbase;
  const KT* vbase;
  if constexpr (BATCH) {
    int lo = 0, hi = args.n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (args.rows[mid].unit_begin <= unit) lo = mid; else hi = mid - 1;
    }
    row = lo;
    const BatchRow& br = args.rows[row];
    chunks = br.chunks;
    const int local = unit - br.unit_begin;
    kvg = local / chunks;
    chunk = local % chunks;
    runs = br.runs;
    capacity = br.capacity;
    part_base = br.part_base;
    kbase = static_cast<const KT*>(br.k);
    vbase = static_cast<const KT*>(br.v);
  } else {
    chunks = args.chunks;
    const int per_row = c.kv_heads * c.hgroups * chunks;
    row = unit / per_row;
    const int local = unit % per_row;
    kvg = local / chunks;
    chunk = local % chunks;
    runs = mask_runs(args.kind, args.window, args.state, args.n_ends, args.ends,
                     args.first + row, args.end);
    const int image_base = (row / args.rows_per_image) * args.keys_per_image;
    runs.b0 += image_base;
    runs.b1 += image_base;
    capacity = args.capacity;
    part_base = row * chunks;
    kbase = static_cast<const KT*>(args.k);
    vbase = static_cast<const KT*>(args.v);
  }
  const int kv = kvg / c.hgroups;
  const int sg = kvg % c.hgroups;
  const int h0 = kv * c.group + sg * G;
  const int g = min(G, c.group - sg * G);
  // A batch row's KV heads are its own cache's blocks of capacity x RD.
  const int64_t kv_stride = BATCH ? int64_t(capacity) * RD : c.kv_stride;
  kbase += kv * kv_stride;
  vbase += kv * kv_stride;
  const int n = runs.n0 + runs.n1;
  const int per = ((n + chunks - 1) / chunks + T - 1) / T * T;
  const int j0 = min(n, chunk * per);
  const int j1 = min(n, j0 + per);
  const int tiles = (j1 - j0 + T - 1) / T;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_fence_init();
    fail_flag = 0;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---- producer: one elected lane streams the chunk's K/V rows -----------------------------
    if (lane == 0) {
      pdl_wait();  // the keys and values kept by the kernel before this one
      const uint64_t policy = policy_evict_first();
      int issued = 0;
      for (int t = 0; t < tiles; ++t) {
        const int s = t % kStages;
        if (!mbar_wait(&empty[s], ((t / kStages) & 1) ^ 1, c.err)) break;
        const int ja = j0 + t * T;
        const int nk = min(T, j1 - ja);
        mbar_arrive_expect_tx(&full[s], uint32_t(nk) * row_bytes * 2);
        KT* kd = k_tiles + size_t(s) * S::kElemsPerTile;
        KT* vd = v_tiles + size_t(s) * S::kElemsPerTile;
        int j = ja, at = 0;
        while (j < ja + nk) {
          int pos, left;
          if (j < runs.n0) { pos = runs.b0 + j; left = runs.n0 - j; }
          else { pos = runs.b1 + (j - runs.n0); left = n - j; }
          const int slot = pos % capacity;
          const int cnt = min(ja + nk - j, min(left, capacity - slot));
          if (c.key_stride == RD) {  // a cache: the run's rows are contiguous
            const uint32_t bytes = uint32_t(cnt) * row_bytes;
            bulk_g2s_hint(kd + size_t(at) * RD, kbase + int64_t(slot) * RD, bytes, &full[s], policy);
            bulk_g2s_hint(vd + size_t(at) * RD, vbase + int64_t(slot) * RD, bytes, &full[s], policy);
          } else {  // strided operand rows: one copy per row
            for (int i = 0; i < cnt; ++i) {
              const int64_t src = int64_t(slot + i) * c.key_stride;
              bulk_g2s_hint(kd + size_t(at + i) * RD, kbase + src, row_bytes, &full[s], policy);
              bulk_g2s_hint(vd + size_t(at + i) * RD, vbase + src, row_bytes, &full[s], policy);
            }
          }
          j += cnt;
          at += cnt;
        }
        issued = t + 1;
      }
      // Wait for this CTA's copies still in flight before it may exit.
      for (int t = max(0, issued - kStages); t < issued; ++t)
        mbar_wait(&full[t % kStages], (t / kStages) & 1, c.err);
    }
    __syncwarp();
    if (c.cluster) {  // the chunk merge's two cluster barriers
      cluster_sync();
      cluster_sync();
    }
    return;
  }

  // ---- consumers ------------------------------------------------------------------------------
  const int grp = lane / LPK;
  const int sub = lane % LPK;
  const int ctid = threadIdx.x;  // 0 .. 127
  // With 1 < G <= LPK the G head scores of a key are reduce-scattered over the key's LPK lanes
  // (log2(G) halving exchanges, then plain folding): lane `sub` ends up owning head
  // sub / (LPK / G), so the softmax of each head runs once per lane instead of once per head
  // on every lane, and the probabilities go back to all lanes by G shuffles.
  constexpr bool kScatter = G > 1 && G <= LPK;
  constexpr int kHeadLanes = kScatter ? LPK / G : LPK;
  constexpr int kLogG = Log2<G>::value;
  const int own = kScatter ? sub / kHeadLanes : 0;
  const int group_base = lane & ~(LPK - 1);

  constexpr int P = E / 2;  // f32 pairs per lane
  float2 q[G][P];
  pdl_wait();  // the rotated queries written by the kernel before this one
  const float* qrow = c.q + int64_t(row) * c.q_stride;
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int el = elem_of<D, KT, E>(sub, 2 * i);
      const int at = (h0 + h) * RD + el;
      q[h][i] = h < g && (!PAD || el < RD)
                    ? make_float2(qrow[at] * c.q_scale, qrow[at + 1] * c.q_scale)
                    : make_float2(0.0f, 0.0f);
    }
  // PAD: the lane's key vectors past the row (all or none of a vector: RD is a multiple of it)
  // read as zero, so that whatever the tile holds there cannot reach a score
  bool lane_valid[P];
#pragma unroll
  for (int i = 0; i < P; ++i) lane_valid[i] = !PAD || elem_of<D, KT, E>(sub, 2 * i) < RD;

  // m[h], l[h]: every head (per-head path) or m[0], l[0]: the lane's own head (scatter path)
  float m[G], l[G];
  float2 o[G][P];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int i = 0; i < P; ++i) o[h][i] = make_float2(0.0f, 0.0f);
  }

  bool ok = true;
  for (int t = 0; t < tiles; ++t) {
    const int s = t % kStages;
    if (!mbar_wait(&full[s], (t / kStages) & 1, c.err)) { ok = false; break; }
    const int nk = min(T, j1 - (j0 + t * T));
    const KT* kt = k_tiles + size_t(s) * S::kElemsPerTile;
    const KT* vt = v_tiles + size_t(s) * S::kElemsPerTile;
#pragma unroll 1
    for (int r = 0; r < S::kRounds; ++r) {
      const int first_key = r * S::kRoundKeys + warp * KPW;
      if (first_key >= nk) break;  // warp-uniform: no key of this warp left in the tile
      const int kr = first_key + grp;
      const bool valid = kr < nk;
      const int rr = valid ? kr : first_key;
      float2 kx[P], vx[P];
      load_lane<D, KT, E>(kt + size_t(rr) * RD, sub, kx);
      if constexpr (PAD) {
#pragma unroll
        for (int i = 0; i < P; ++i)
          if (!lane_valid[i]) kx[i] = make_float2(0.0f, 0.0f);
      }
      float part[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < P; ++i) a = fma2(q[h][i], kx[i], a);
        part[h] = a.x + a.y;
      }
      load_lane<D, KT, E>(vt + size_t(rr) * RD, sub, vx);
      if constexpr (kScatter) {
#pragma unroll
        for (int k = 0; k < kLogG; ++k) {
          const int off = LPK >> (k + 1);
          const int half = G >> (k + 1);
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int i = 0; i < half; ++i) {
            const float send = upper ? part[i] : part[i + half];
            const float keep = upper ? part[i + half] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
#pragma unroll
        for (int off = LPK >> (kLogG + 1); off >= 1; off >>= 1)
          part[0] += __shfl_xor_sync(0xffffffffu, part[0], off);
        const float sc = valid ? part[0] : -INFINITY;
        float mx = sc;
#pragma unroll
        for (int off = LPK; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const bool grew = mx > m[0];
        if (__any_sync(0xffffffffu, grew)) {
          const float alpha = grew ? exp2_approx(m[0] - mx) : 1.0f;
          if (grew) m[0] = mx;
          l[0] *= alpha;
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float ah = __shfl_sync(0xffffffffu, alpha, group_base + h * kHeadLanes);
#pragma unroll
            for (int i = 0; i < P; ++i) o[h][i] = mul2(o[h][i], make_float2(ah, ah));
          }
        }
        const float p = valid ? exp2_approx(sc - m[0]) : 0.0f;
        l[0] += p;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float ph = __shfl_sync(0xffffffffu, p, group_base + h * kHeadLanes);
#pragma unroll
          for (int i = 0; i < P; ++i) o[h][i] = fma2(make_float2(ph, ph), vx[i], o[h][i]);
        }
      } else {
        float sc[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float acc = part[h];
#pragma unroll
          for (int off = LPK / 2; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
          sc[h] = valid ? acc : -INFINITY;
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float mx = sc[h];
#pragma unroll
          for (int off = LPK; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          if (mx > m[h]) {  // warp-uniform
            const float alpha = exp2_approx(m[h] - mx);
            l[h] *= alpha;
#pragma unroll
            for (int i = 0; i < P; ++i) o[h][i] = mul2(o[h][i], make_float2(alpha, alpha));
            m[h] = mx;
          }
          const float p = valid ? exp2_approx(sc[h] - m[h]) : 0.0f;
          l[h] += p;
#pragma unroll
          for (int i = 0; i < P; ++i) o[h][i] = fma2(make_float2(p, p), vx[i], o[h][i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- merge the warp's key groups (they share the warp-uniform max) ---------------------------
  constexpr int kOwnHeads = kScatter ? 1 : G;
#pragma unroll
  for (int off = LPK; off < 32; off <<= 1) {
#pragma unroll
    for (int h = 0; h < kOwnHeads; ++h) l[h] += __shfl_xor_sync(0xffffffffu, l[h], off);
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int i = 0; i < P; ++i) {
        o[h][i].x += __shfl_xor_sync(0xffffffffu, o[h][i].x, off);
        o[h][i].y += __shfl_xor_sync(0xffffffffu, o[h][i].y, off);
      }
  }
  // All consumers are past their last tile: every copy has landed, the stages are free.
  if (!ok) fail_flag = 1;
  named_sync(1, kConsumerWarps * 32);
  if (*static_cast<volatile int*>(&fail_flag) != 0) {
    if (c.cluster) {  // every thread of the cluster reaches both of its barriers
      cluster_sync();
      cluster_sync();
    }
    return;
  }

  float* red_m = reinterpret_cast<float*>(smem);           // [warps][G]
  float* red_l = red_m + kConsumerWarps * G;               // [warps][G]
  float* red_o = red_l + kConsumerWarps * G;               // [warps][G][D]
  if constexpr (kScatter) {
    if (grp == 0 && sub % kHeadLanes == 0) {  // the lane of group 0 that owns head `own`
      red_m[warp * G + own] = m[0];
      red_l[warp * G + own] = l[0];
    }
  } else if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      red_m[warp * G + h] = m[h];
      red_l[warp * G + h] = l[h];
    }
  }
  if (grp == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int i = 0; i < P; ++i) {
        float* at = red_o + (warp * G + h) * D + elem_of<D, KT, E>(sub, 2 * i);
        at[0] = o[h][i].x;
        at[1] = o[h][i].y;
      }
  }
  named_sync(1, kConsumerWarps * 32);

  const int count = g * D;
  float* out_row = c.out != nullptr ? c.out + int64_t(row) * c.out_stride : nullptr;
  float* part_row = c.partial_out != nullptr ? c.partial_out + int64_t(row) * c.heads * (RD + 2) : nullptr;
  // The row's merged state of head h0 + h: its output, or its (max, sum, o) when partial.
  auto finish = [&](int h, int e, float mm, float ll, float oo) {
    if (PAD && e >= RD) return;
    if (out_row != nullptr) {
      out_row[(h0 + h) * RD + e] = ll > 0.0f ? oo / ll : 0.0f;
    } else {
      float* pr = part_row + (h0 + h) * (RD + 2);
      if (e == 0) { pr[0] = mm; pr[1] = ll; }
      pr[2 + e] = oo;
    }
  };
  for (int idx = ctid; idx < count; idx += kConsumerWarps * 32) {
    const int h = idx / D, e = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) mm = fmaxf(mm, red_m[w * G + h]);
    float ll = 0.0f, oo = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float wm = red_m[w * G + h];
      const float f = wm == -INFINITY ? 0.0f : exp2_approx(wm - mm);
      ll = fmaf(red_l[w * G + h], f, ll);
      oo = fmaf(red_o[(w * G + h) * D + e], f, oo);
    }
    if (chunks == 1) {
      finish(h, e, mm, ll, oo);
    } else if (c.cluster) {
      // the chunk's state for the cluster merge, in this CTA's shared memory
      float* cp = reinterpret_cast<float*>(smem + kClusterPartialOffset);
      cp[2 * G + idx] = oo;
      if (e == 0) {
        cp[h] = mm;
        cp[G + h] = ll;
      }
    } else {
      const int64_t slot = int64_t(part_base + chunk) * c.heads + (h0 + h);
      c.part_o[slot * D + e] = oo;
      if (e == 0) {
        c.part_ml[2 * slot] = mm;
        c.part_ml[2 * slot + 1] = ll;
      }
    }
  }
  if (chunks == 1) return;
  if (c.cluster) {
    // ---- the row's chunks are one cluster: CTA 0 merges their states from shared memory ----
    cluster_sync();
    if (cluster_rank() == 0) {
      const float* cp = reinterpret_cast<const float*>(smem + kClusterPartialOffset);
      for (int idx = ctid; idx < count; idx += kConsumerWarps * 32) {
        const int h = idx / D, e = idx % D;
        float mm = -INFINITY;
        for (int r = 0; r < chunks; ++r) mm = fmaxf(mm, ld_cluster_f32(cp + h, r));
        float ll = 0.0f, oo = 0.0f;
        for (int r = 0; r < chunks; ++r) {
          const float cm = ld_cluster_f32(cp + h, r);
          const float f = cm == -INFINITY ? 0.0f : exp2_approx(cm - mm);
          ll = fmaf(ld_cluster_f32(cp + G + h, r), f, ll);
          oo = fmaf(ld_cluster_f32(cp + 2 * G + idx, r), f, oo);
        }
        finish(h, e, mm, ll, oo);
      }
    }
    cluster_sync();  // no CTA leaves while CTA 0 reads its shared memory
    return;
  }

  // ---- the last CTA of this (row, KV group) merges the chunks ---------------------------------
  __threadfence();
  named_sync(1, kConsumerWarps * 32);
  int* counter = c.counters + int64_t(row) * c.kv_heads * c.hgroups + kvg;
  if (ctid == 0) {
    const int arrived = atomicAdd(counter, 1);
    last_flag = arrived == chunks - 1;
    if (last_flag) *counter = 0;  // ready for the next launch
  }
  named_sync(1, kConsumerWarps * 32);
  if (!last_flag) return;
  __threadfence();
  merge_chunk_partials<G, D, kConsumerWarps * 32>(
      c.part_o, c.part_ml, c.heads, h0, g, part_base, chunks, reinterpret_cast<float*>(smem),
      int(size_t(kStages) * 2 * kTileBytes / (4 * G)), 1, ctid, finish);
}

}  // namespace fa
