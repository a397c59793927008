// The bf16 tensor-core attention with two query tiles per CTA in ping-pong (prefill over a bf16
// cache and bf16 full-mask calls; the same semantics as fmha_kernel, fa_fmha.cuh).
//
// One CTA = 2 x 128 query rows of one query head. Warp roles:
//   warp 0      TMA producer: both Q tiles once, then K and V tiles into a 2-stage ring;
//   warp 1      TMEM owner and MMA issuer (one thread);
//   warps 2-5   softmax of query tile 0 (thread = one row, TMEM lane (warp % 4) * 32 + lane);
//   warps 6-9   softmax of query tile 1.
// TMEM: S0 | O0 | S1 | O1, 128 columns each (P_i overwrites S_i as bf16 pairs). The MMA order per
// KV tile j is PV0_j, S0_{j+1}, PV1_j, S1_{j+1}: while one softmax group works on its S, the
// tensor core runs the other group's two products, so the exponentials of one tile overlap the
// matrix products of the other (one S buffer per tile suffices: the tensor core executes one
// thread's MMAs in issue order, so PV_i reads P_i before S_i is written again).
// A query tile takes part in the KV tiles its rows see (the union of their key runs); the other
// tile's barriers count only its own participating tiles.
// Schedule (FmhaArgs::whole_units / splits): a 1-D grid over the units (query head, pair of query
// tiles), head-major (pair-major, heaviest pairs first, for a causal prefill whose K/V fits in
// L2: FmhaArgs::pair_major). The leading units run whole; with splits > 1 each later unit runs as that
// many consecutive CTAs, each over an equal share of the pair's KV tiles, so that the last waves
// of a call whose units do not fill the SMs evenly are cut into shorter pieces. A piece writes
// its rows' (max, sum, unnormalised O) partials; the last piece of the unit to finish (an
// arrival counter) merges them in log-sum-exp fashion and writes the output.
#pragma once

#include "fa_fmha.cuh"

namespace fa {

template <int D>
struct Fmha2Shape {
  static constexpr int BM = 128;   // rows of one query tile
  static constexpr int BN = 128;   // keys per KV tile
  static constexpr int kBlock = 64;  // bf16 elements per swizzled 128-byte row
  static constexpr int kDBlocks = D / kBlock;
  static constexpr int kKStep = 16;  // bf16 elements per MMA K step
  static constexpr int kStages = 2;
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;
  static constexpr int kTileCols = 256;  // TMEM columns of one query tile: S (128) then O
  static constexpr size_t kSmemUsed =
      size_t(2 * kQBytes) + size_t(kStages) * 2 * kKVBytes + 1024 /* alignment */ + 256;
  // At least 120 KB so that one CTA holds an SM: each CTA allocates all 512 TMEM columns.
  static constexpr size_t kSmemBytes = kSmemUsed > 122880 ? kSmemUsed : 122880;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
};

// The last piece of a split unit: row `orow`'s output (query head `head`) from the n_pieces
// partials (max, sum, unnormalised O) at slots slot0 + j x 256, merged in log-sum-exp fashion.
template <int D>
__device__ __forceinline__ void merge_pieces(const FmhaArgs& a, int64_t slot0, int n_pieces,
                                          int64_t orow, int head) {
  constexpr int kSlots = 256;  // rows of a pair of query tiles
  float m_max = -INFINITY;
  for (int j = 0; j < n_pieces; ++j)
    m_max = fmaxf(m_max, __ldcg(a.part_ml + 2 * (slot0 + int64_t(j) * kSlots)));
  float w[kFmhaMaxSplits];
  float l_total = 0.0f;
#pragma unroll
  for (int j = 0; j < kFmhaMaxSplits; ++j) {
    w[j] = 0.0f;
    if (j >= n_pieces) continue;
    const float* ml = a.part_ml + 2 * (slot0 + int64_t(j) * kSlots);
    const float mj = __ldcg(ml);
    if (mj == -INFINITY) continue;  // no visible key in that piece
    w[j] = exp2_approx(mj - m_max);
    l_total = fmaf(w[j], __ldcg(ml + 1), l_total);
  }
  const float inv = l_total > 0.0f ? 1.0f / l_total : 0.0f;
#pragma unroll 1
  for (int cc = 0; cc < D / 32; ++cc) {
    float acc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int j = 0; j < kFmhaMaxSplits; ++j) {
      if (j >= n_pieces || w[j] == 0.0f) continue;
      const float4* src =
          reinterpret_cast<const float4*>(a.part_o + (slot0 + int64_t(j) * kSlots) * D + cc * 32);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 v = __ldcg(src + e);
        acc[4 * e] = fmaf(w[j], v.x, acc[4 * e]);
        acc[4 * e + 1] = fmaf(w[j], v.y, acc[4 * e + 1]);
        acc[4 * e + 2] = fmaf(w[j], v.z, acc[4 * e + 2]);
        acc[4 * e + 3] = fmaf(w[j], v.w, acc[4 * e + 3]);
      }
    }
    if (a.out_bf16) {
      uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) +
                                            orow * a.out_stride + head * D + cc * 32);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        dst[e] = make_uint4(tc::pack_bf16(acc[8 * e + 0] * inv, acc[8 * e + 1] * inv),
                            tc::pack_bf16(acc[8 * e + 2] * inv, acc[8 * e + 3] * inv),
                            tc::pack_bf16(acc[8 * e + 4] * inv, acc[8 * e + 5] * inv),
                            tc::pack_bf16(acc[8 * e + 6] * inv, acc[8 * e + 7] * inv));
    } else {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow * a.out_stride +
                                              head * D + cc * 32);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        dst[e] = make_float4(acc[4 * e] * inv, acc[4 * e + 1] * inv, acc[4 * e + 2] * inv,
                             acc[4 * e + 3] * inv);
    }
  }
}

// A CTA's unit of work: query head, image, first query row of the pair, and its piece.
struct Fmha2Unit {
  int head, image, r0;
  int piece, n_pieces, tail_unit;  // n_pieces 1 for a whole unit
};

__device__ __forceinline__ Fmha2Unit fmha2_unit(const FmhaArgs& a, uint32_t cta) {
  const int pairs = (a.q_tiles + 1) / 2;
  const int per_head = a.images * pairs;
  const int whole = a.splits > 1 ? a.whole_units : per_head * a.heads;
  Fmha2Unit u;
  int unit = int(cta);
  u.piece = 0;
  u.n_pieces = 1;
  u.tail_unit = 0;
  if (unit >= whole) {
    const int p = unit - whole;
    u.tail_unit = p / a.splits;
    u.piece = p % a.splits;
    u.n_pieces = a.splits;
    unit = whole + u.tail_unit;
  }
  if (a.pair_major && a.splits <= 1) {
    // A pair's keys grow with its rows (a causal prefill from the cache's start), so the units
    // run heaviest first across every head and image (longest-processing-time order: the last
    // wave holds the lightest pairs). Every head's K/V is then read at once: the host asks for
    // this order only when that fits in L2.
    u.head = unit % a.heads;
    const int rest = unit / a.heads;
    u.image = rest % a.images;
    u.r0 = (pairs - 1 - rest / a.images) * 256;
    return u;
  }
  u.head = unit / per_head;
  const int pair_id = per_head - 1 - unit % per_head;  // heavier (later, for causal masks) first
  u.image = pair_id / pairs;
  u.r0 = (pair_id % pairs) * 256;
  return u;
}

constexpr int kFmha2Threads = 320;

template <int D>
__global__ void __launch_bounds__(kFmha2Threads, 1)
    fmha2_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                 const __grid_constant__ CUtensorMap v_map, const __grid_constant__ FmhaArgs a) {
  using S = Fmha2Shape<D>;
  constexpr int BM = S::BM, BN = S::BN;
  constexpr uint32_t kIdescQK = tc::instr_desc(1u, false, BN, BM);
  constexpr uint32_t kIdescPV = tc::instr_desc(1u, true, D, BM);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem;  // tile i at sQ + i * kQBytes
  unsigned char* sK = sQ + 2 * S::kQBytes;
  unsigned char* sV = sK + S::kStages * S::kKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + S::kStages * S::kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + S::kStages;
  uint64_t* v_full = k_empty + S::kStages;
  uint64_t* v_empty = v_full + S::kStages;
  uint64_t* s_full = v_empty + S::kStages;  // [query tile]
  uint64_t* p_full = s_full + 2;            // [query tile]
  uint64_t* o_done = p_full + 2;            // [query tile]
  uint64_t* o_final = o_done + 2;           // [query tile]: its last P.V has completed
  uint64_t* mma_drained = o_final + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Fmha2Unit u = fmha2_unit(a, ctaid_x());
  const int head = u.head, image = u.image, r0 = u.r0, piece = u.piece, n_pieces = u.n_pieces;
  const int kv = head / a.group;

  // KV tiles each query tile's rows see (the union of their key runs), and their union.
  int tb[2], te[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int first_row = r0 + i * BM;
    const int last_row = min(first_row + BM, a.rows) - 1;
    if (first_row >= a.rows) { tb[i] = te[i] = 0; continue; }
    const Runs fr = mask_runs(a.kind, a.window, a.state, a.n_ends, a.ends, a.first + first_row, a.end);
    const Runs lr = mask_runs(a.kind, a.window, a.state, a.n_ends, a.ends, a.first + last_row, a.end);
    int lo = fr.b0, hi = max(lr.b0 + lr.n0, lr.b1 + lr.n1);
    if (a.kind == 3) { lo = 0; hi = a.end; }  // Groups: every run lies in [0, end)
    tb[i] = lo / BN;
    te[i] = hi > lo ? (hi + BN - 1) / BN : tb[i];
  }
  if (n_pieces > 1) {
    // this piece's share of the union of the two tiles' KV tiles
    const bool u0 = te[0] > tb[0], u1 = te[1] > tb[1];
    const int ub = u0 && u1 ? min(tb[0], tb[1]) : (u0 ? tb[0] : tb[1]);
    const int ue = u0 && u1 ? max(te[0], te[1]) : (u0 ? te[0] : te[1]);
    const int n = (u0 || u1) ? ue - ub : 0;
    const int lo = ub + int(int64_t(n) * piece / n_pieces);
    const int hi = ub + int(int64_t(n) * (piece + 1) / n_pieces);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      tb[i] = max(tb[i], lo);
      te[i] = max(min(te[i], hi), tb[i]);
    }
  }
  const bool any0 = te[0] > tb[0], any1 = te[1] > tb[1];
  const int t0 = any0 && any1 ? min(tb[0], tb[1]) : (any0 ? tb[0] : tb[1]);
  const int t_end = any0 && any1 ? max(te[0], te[1]) : (any0 ? te[0] : te[1]);
  const int n_tiles = (any0 || any1) ? t_end - t0 : 0;
  auto part = [&](int i, int L) {  // query tile i takes part in union tile L
    const int t = t0 + L;
    return t >= tb[i] && t < te[i];
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_final[i], 1);
    }
    mbar_init(mma_drained, 1);
    mbar_fence_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer --------------------------------------------------------------------
    if (lane == 0) {
      tc::tma_prefetch_map(&q_map);
      tc::tma_prefetch_map(&k_map);
      tc::tma_prefetch_map(&v_map);
      pdl_wait();  // the queries (and a cache's kept rows) written by the kernel before this one
      mbar_arrive_expect_tx(q_full, 2 * S::kQBytes);
      const int qy = image * a.q_row_base_per_image + r0;
      for (int i = 0; i < 2; ++i)
        for (int db = 0; db < S::kDBlocks; ++db)
          tc::tma_load_3d(sQ + i * S::kQBytes + db * BM * 128, &q_map, db * S::kBlock, qy + i * BM,
                          head, q_full);
      const int kz = a.kv_layer_base + kv;
      const int ky0 = image * a.kv_row_base_per_image;
      int issued = 0;
      for (int L = 0; L < n_tiles; ++L) {
        const int st = L % S::kStages;
        const uint32_t ph = ((L / S::kStages) & 1) ^ 1;
        const int ky = ky0 + (t0 + L) * BN;
        if (!mbar_wait(&k_empty[st], ph, a.err)) break;
        mbar_arrive_expect_tx(&k_full[st], S::kKVBytes);
        for (int db = 0; db < S::kDBlocks; ++db)
          tc::tma_load_3d(sK + st * S::kKVBytes + db * BN * 128, &k_map, db * S::kBlock, ky, kz,
                          &k_full[st]);
        if (!mbar_wait(&v_empty[st], ph, a.err)) break;
        mbar_arrive_expect_tx(&v_full[st], S::kKVBytes);
        for (int db = 0; db < S::kDBlocks; ++db)
          tc::tma_load_3d(sV + st * S::kKVBytes + db * BN * 128, &v_map, db * S::kBlock, ky, kz,
                          &v_full[st]);
        issued = L + 1;
      }
      // The loads still in flight land before the CTA may exit.
      mbar_wait(q_full, 0, a.err);
      for (int L = max(0, issued - S::kStages); L < issued; ++L) {
        mbar_wait(&k_full[L % S::kStages], (L / S::kStages) & 1, a.err);
        mbar_wait(&v_full[L % S::kStages], (L / S::kStages) & 1, a.err);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------------
    if (lane == 0) {
      // The descriptors differ only in their start address (16-byte units in the low bits;
      // shared-memory addresses stay below 2^18): built once, offsets added per stage and K step
      // (the issue of the MMAs is on this thread's critical path).
      const uint64_t q_desc = tc::smem_desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc = tc::smem_desc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc = tc::smem_desc(smem_u32(sV), BN * 128, 1024, tc::kSwizzle128B);
      bool ok = mbar_wait(q_full, 0, a.err);
      int pv_count[2] = {0, 0};
      auto issue_s = [&](int i, int L) {
        const int st = L % S::kStages;
        const uint64_t qd0 = q_desc + uint64_t(i * S::kQBytes >> 4);
        const uint64_t kd0 = k_desc + uint64_t(st) * uint64_t(S::kKVBytes >> 4);
#pragma unroll
        for (int k = 0; k < D / S::kKStep; ++k) {
          const int db = k / 4, koff = (k % 4) * 32;
          tc::mma_ss<false>(tmem + i * S::kTileCols, qd0 + uint64_t((db * BM * 128 + koff) >> 4),
                            kd0 + uint64_t((db * BN * 128 + koff) >> 4), kIdescQK,
                            k > 0 ? 1u : 0u);
        }
        tc::commit(&s_full[i]);
      };
      auto issue_pv = [&](int i, int L) {
        const int st = L % S::kStages;
        const int c = pv_count[i];
        if (!mbar_wait(&p_full[i], c & 1, a.err)) return false;
        if (!mbar_wait(&v_full[st], (L / S::kStages) & 1, a.err)) return false;
        tc::fence_after_sync();
        const uint32_t p_tmem = tmem + i * S::kTileCols;
        const uint64_t vd0 = v_desc + uint64_t(st) * uint64_t(S::kKVBytes >> 4);
#pragma unroll
        for (int k = 0; k < BN / S::kKStep; ++k)
          tc::mma_ts<false>(tmem + i * S::kTileCols + 128, p_tmem + k * 8,
                            vd0 + uint64_t((k * S::kKStep * 128) >> 4), kIdescPV,
                            (c > 0 || k > 0) ? 1u : 0u);
        tc::commit(&o_done[i]);
        pv_count[i] = c + 1;
        return true;
      };
      if (ok && n_tiles > 0) {
        ok = mbar_wait(&k_full[0], 0, a.err);
        if (ok) {
          tc::fence_after_sync();
          if (part(0, 0)) issue_s(0, 0);
          if (part(1, 0)) issue_s(1, 0);
          tc::commit(&k_empty[0]);
        }
      }
      for (int L = 0; ok && L < n_tiles; ++L) {
        const bool next = L + 1 < n_tiles;
        if (next) {
          const int sn = (L + 1) % S::kStages;
          if (!mbar_wait(&k_full[sn], ((L + 1) / S::kStages) & 1, a.err)) { ok = false; break; }
          tc::fence_after_sync();
        }
        if (part(0, L) && !issue_pv(0, L)) { ok = false; break; }
        if (next && part(0, L + 1)) issue_s(0, L + 1);
        if (part(1, L) && !issue_pv(1, L)) { ok = false; break; }
        if (next && part(1, L + 1)) issue_s(1, L + 1);
        if (next) tc::commit(&k_empty[(L + 1) % S::kStages]);
        tc::commit(&v_empty[L % S::kStages]);
      }
      if (ok) {
        if (pv_count[0] > 0) tc::commit(&o_final[0]);
        if (pv_count[1] > 0) tc::commit(&o_final[1]);
      }
      // Every MMA this thread issued has completed before the CTA may free TMEM.
      tc::commit(mma_drained);
      mbar_wait(mma_drained, 0, a.err);
    }
  } else {
    // ---- softmax + epilogue of query tile i ----------------------------------------------
    const int i = warp < 6 ? 0 : 1;
    const int wq = warp & 3;  // the TMEM lane quarter this warp may access
    const int r = r0 + i * BM + wq * 32 + lane;  // this thread's query row within the image
    const bool row_valid = r < a.rows;
    const Runs runs = mask_runs(a.kind, a.window, a.state, a.n_ends, a.ends, a.first + r, a.end);
    const uint32_t lane_base = tmem + i * S::kTileCols + (uint32_t(wq * 32) << 16);
    const uint32_t o_base = lane_base + 128;
    float m_used = -INFINITY, l_sum = 0.0f;
    bool ok = true;
    int c = 0;  // this tile's participating KV tiles so far
    for (int L = 0; L < n_tiles; ++L) {
      if (!part(i, L)) continue;
      const int kp = (t0 + L) * BN;  // first key position of the tile
      // Every decision before a whole-warp tcgen05 instruction is made warp-uniform.
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[i], c & 1, a.err))) { ok = false; break; }
      tc::fence_after_sync();
      uint32_t sreg[BN];
      tc::tmem_ld128_wait(lane_base, sreg);
      float* s = reinterpret_cast<float*>(sreg);
      // A row past the end of the image's queries is never written back, and its P row reaches
      // only its own O row (the tensor-core product is row by row), so it skips the masking:
      // its Q row (the next image's query, or the TMA's zero fill) needs no -inf either.
      const bool all_in = !row_valid ||
                          (kp >= runs.b0 && kp + BN <= runs.b0 + runs.n0) ||
                          (kp >= runs.b1 && kp + BN <= runs.b1 + runs.n1);
      if (!all_in) mask_scores<BN>(runs, kp, s);
      // the tile's max in four independent chains of three-input maxima: 12 + 14 x 8 + 4 keys
      static_assert(BN == 128, "the max chains cover 128 keys");
      float mx0 = fmax3(s[0], s[1], s[2]), mx1 = fmax3(s[3], s[4], s[5]);
      float mx2 = fmax3(s[6], s[7], s[8]), mx3 = fmax3(s[9], s[10], s[11]);
#pragma unroll
      for (int cc = 12; cc < 124; cc += 8) {
        mx0 = fmax3(mx0, s[cc], s[cc + 1]);
        mx1 = fmax3(mx1, s[cc + 2], s[cc + 3]);
        mx2 = fmax3(mx2, s[cc + 4], s[cc + 5]);
        mx3 = fmax3(mx3, s[cc + 6], s[cc + 7]);
      }
      mx0 = fmax3(mx0, s[124], s[125]);
      mx1 = fmax3(mx1, s[126], s[127]);
      const float m_tile = fmax3(mx0, mx1, fmaxf(mx2, mx3)) * a.scale_log2;
      // Lazy rescale: move the reference max only when the tile's max exceeds it by 2^8 (the
      // first finite max just sets it: nothing has accumulated for the row yet).
      float alpha = 1.0f;
      if (m_tile > m_used + 8.0f || (m_used == -INFINITY && m_tile > -INFINITY)) {
        if (m_used > -INFINITY) alpha = exp2_approx(m_used - m_tile);
        m_used = m_tile;
      }
      const float ms = m_used == -INFINITY ? 0.0f : m_used;
      const float2 scale2 = make_float2(a.scale_log2, a.scale_log2);
      const float2 neg2 = make_float2(-ms, -ms);
      float2 sum2a = make_float2(0.0f, 0.0f), sum2b = make_float2(0.0f, 0.0f);
      // pairs of probabilities packed in place: sreg[cc / 2] is written only after s[cc] and
      // s[cc + 1] are read
#pragma unroll
      for (int cc = 0; cc < BN; cc += 4) {
        const float2 x0 = __ffma2_rn(make_float2(s[cc], s[cc + 1]), scale2, neg2);
        const float2 x1 = __ffma2_rn(make_float2(s[cc + 2], s[cc + 3]), scale2, neg2);
        const float2 p0 = make_float2(exp2_approx(x0.x), exp2_approx(x0.y));
        const float2 p1 = make_float2(exp2_approx(x1.x), exp2_approx(x1.y));
        sum2a = __fadd2_rn(sum2a, p0);
        sum2b = __fadd2_rn(sum2b, p1);
        sreg[cc / 2] = tc::pack_bf16(p0.x, p0.y);
        sreg[cc / 2 + 1] = tc::pack_bf16(p1.x, p1.y);
      }
#pragma unroll
      for (int cc = 0; cc < BN / 64; ++cc)
        tc::tmem_st32(lane_base + cc * 32, *reinterpret_cast<const uint32_t(*)[32]>(&sreg[cc * 32]));
      l_sum = l_sum * alpha + ((sum2a.x + sum2a.y) + (sum2b.x + sum2b.y));
      if (__any_sync(0xffffffffu, alpha != 1.0f)) {
        // O_i holds the products of this tile's earlier KV tiles. S_i of this KV tile has
        // completed, and with it (issue order) the P.V of the previous one: o_done[i] is in
        // that phase, and the next cannot start before this group's P is written. (Done after
        // P is written, so that the S row's registers are free for O's.)
        if (!__all_sync(0xffffffffu, mbar_wait(&o_done[i], (c - 1) & 1, a.err))) { ok = false; break; }
        tc::fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          tc::tmem_ld32_wait(o_base + cc * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tc::tmem_st32(o_base + cc * 32, o);
          tc::tmem_wait_st();  // the registers are free again only after the store lands
        }
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&p_full[i]);
      ++c;
    }
    const bool have = __all_sync(0xffffffffu, ok && c > 0 && mbar_wait(&o_final[i], 0, a.err));
    // The unit is decoded again from the CTA index (a volatile read: nothing of it stays live
    // through the softmax loop, whose registers are at the kernel's limit).
    const Fmha2Unit e = fmha2_unit(a, ctaid_x());
    const int64_t orow_base = int64_t(e.image) * a.rows + e.r0 + i * BM + wq * 32;  // + lane
    const bool row_ok = e.r0 + i * BM + wq * 32 + lane < a.rows;
    if (e.n_pieces > 1) {
      // ---- a piece: its partials, then the last piece of the unit merges ------------------
      const int row_in_pair = i * BM + wq * 32 + lane;
      const int64_t slot0 = int64_t(e.tail_unit) * e.n_pieces * (2 * BM) + row_in_pair;
      const int64_t slot = slot0 + int64_t(e.piece) * (2 * BM);
      if (have) {
        tc::fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          tc::tmem_ld32_wait(o_base + cc * 32, o);
          if (!row_ok) continue;
          float4* dst = reinterpret_cast<float4*>(a.part_o + slot * D + cc * 32);
#pragma unroll
          for (int x = 0; x < 8; ++x)
            dst[x] = make_float4(__uint_as_float(o[4 * x]), __uint_as_float(o[4 * x + 1]),
                                 __uint_as_float(o[4 * x + 2]), __uint_as_float(o[4 * x + 3]));
        }
      }
      if (row_ok) {
        a.part_ml[2 * slot] = have ? m_used : -INFINITY;
        a.part_ml[2 * slot + 1] = have ? l_sum : 0.0f;
      }
      // Each warp's 32 rows count their pieces on their own counter: the warp of the last piece
      // to arrive merges those rows (no barrier across the CTA's warps).
      __threadfence();  // the partials are visible device-wide before the arrival is counted
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        int* counter = a.counters + int64_t(e.tail_unit) * 8 + (i * 4 + wq);
        last = atomicAdd(counter, 1) == e.n_pieces - 1;
        if (last) *counter = 0;  // every piece has arrived: ready for the next launch
      }
      if (__shfl_sync(0xffffffffu, last, 0) != 0 && row_ok) {
        __threadfence();
        merge_pieces<D>(a, slot0, e.n_pieces, orow_base + lane, e.head);
      }
    } else if (have) {
      // ---- epilogue: O / l -----------------------------------------------------------------
      tc::fence_after_sync();
      const float inv = l_sum > 0.0f ? 1.0f / l_sum : 0.0f;
      const int64_t orow = orow_base + lane;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        tc::tmem_ld32_wait(o_base + cc * 32, o);
        if (!row_ok) continue;
        if (a.out_bf16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) +
                                                orow * a.out_stride + e.head * D + cc * 32);
#pragma unroll
          for (int x = 0; x < 4; ++x)
            dst[x] = make_uint4(
                tc::pack_bf16(__uint_as_float(o[8 * x + 0]) * inv, __uint_as_float(o[8 * x + 1]) * inv),
                tc::pack_bf16(__uint_as_float(o[8 * x + 2]) * inv, __uint_as_float(o[8 * x + 3]) * inv),
                tc::pack_bf16(__uint_as_float(o[8 * x + 4]) * inv, __uint_as_float(o[8 * x + 5]) * inv),
                tc::pack_bf16(__uint_as_float(o[8 * x + 6]) * inv, __uint_as_float(o[8 * x + 7]) * inv));
        } else {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) +
                                                  orow * a.out_stride + e.head * D + cc * 32);
#pragma unroll
          for (int x = 0; x < 8; ++x)
            dst[x] = make_float4(__uint_as_float(o[4 * x]) * inv, __uint_as_float(o[4 * x + 1]) * inv,
                                 __uint_as_float(o[4 * x + 2]) * inv, __uint_as_float(o[4 * x + 3]) * inv);
        }
      }
    }
  }

  // ---- teardown: every TMEM user is done before the owner frees it ---------------------------
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa
