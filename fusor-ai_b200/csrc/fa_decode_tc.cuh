// Decode over a bf16 cache on the tensor cores (KvCache::attend of one-row spans,
// transformer.rs:182-219, with ops::attend's semantics, ops.rs:310-342): the bf16 rows carry half
// the bytes of f32 rows for the same arithmetic, and on the CUDA cores that arithmetic, not HBM,
// bounds the split-KV kernel. Here the tensor core does the products and the CUDA cores only the
// softmax of each key.
//
// Transposed so that the keys fill the 128 rows of the MMA: per tile of 128 keys,
//   S^T (128 keys x 16) = K (128 x D head_dim) . Q^T (D x 16: the KV head's G <= 16 query
//                        heads, zero-padded),
//   O^T (D head_dim x 16) += V^T (D x 128 keys) . P^T (128 keys x 16),
// accumulators in TMEM, D = 128 or 256. The K and V rings hold 128 keys x 128 head_dim entries:
// a tile of head_dim 256 is two entries of each (its halves), S^T adds up both halves' products
// and O^T is two 128-row accumulators, so the rings' shared memory is that of head_dim 128. A
// persistent CTA per SM walks the (row, KV head, chunk of keys) units; warps:
//   warps 0, 6  TMA producers of the K and of the V entries (128-byte swizzled boxes of the
//               cache's own tensor maps, one pair per cache), 3 entries each (2 and 4 at
//               head_dim 256); plain per-CTA loads only;
//   warp 1      TMEM owner and MMA issuer (one thread): S^T_t (three S^T buffers), then
//               O^T += V^T P^T_{t-2}: the softmax has two tiles of slack;
//   warps 2-5   softmax: thread = key (TMEM lane) of S^T and head_dim row of O^T. Per tile a
//               lazy max per head (moved, and O^T rescaled, only when a score exceeds it by 2^8:
//               one OR-reducing barrier decides; then the heads' maxima over the 128 keys),
//               P^T as bf16 into shared memory (three buffers); per unit the next unit's Q^T
//               into shared memory (two buffers, so the MMAs run on across units) and at the
//               end O^T / L or the unit's partial (max, sum, o) for the chunk merge (at
//               head_dim 256 a thread keeps O^T rows d and d + 128).
#pragma once

#include "fa_decode.cuh"
#include "fa_decode_tc.h"
#include "fa_tc.cuh"

namespace fa {

// Byte offset of element (r, k) of a 16-row bf16 operand in the 128-byte swizzled K-major layout
// the descriptors below read: 64-element blocks of 16 rows x 128 bytes, the 16-byte chunks of a
// row XOR-ed with the row index within its 8-row group.
__device__ __forceinline__ uint32_t dtc_op_offset(int r, int k) {
  const int block = k >> 6, within = k & 63;
  return uint32_t(block * (kDtcN * 128) + r * 128 + ((((within >> 3) ^ (r & 7))) << 4) +
                  ((within & 7) << 1));
}

__device__ __forceinline__ void dtc_unit(const DtcArgs& a, int u, int* row, int* kv, int* j0,
                                         int* j1) {
  int lo = 0, hi = a.n_rows - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.rows[mid].unit_begin <= u) lo = mid; else hi = mid - 1;
  }
  const DtcRow& r = a.rows[lo];
  const int local = u - r.unit_begin;
  *row = lo;
  *kv = local / r.chunks;
  const int chunk = local % r.chunks;
  *j0 = chunk * a.chunk_keys;
  *j1 = min(r.n, *j0 + a.chunk_keys);
}

// kG: the group's query heads rounded up to a power of two (<= kDtcN), the per-head work of the
// softmax threads; D: the head_dim, 128 or 256.
template <int D, int kG>
__global__ void __launch_bounds__(kDtcThreads, 1) decode_tc_kernel(const __grid_constant__ DtcArgs a) {
  static_assert(D == 128 || D == 256, "head_dim");
  static_assert(dtc_smem_bytes(D) + 1024 <= 227 * 1024, "shared memory");
  constexpr int kHalves = D / kDtcD;            // ring entries per tile, O^T accumulators
  // K and V ring entries (2 * kDtcStages together)
  constexpr int KS = dtc_k_stages(D), VS = 2 * kDtcStages - KS;
  constexpr int kQBytes = dtc_q_bytes(D);
  constexpr uint32_t kIdescS = tc::instr_desc_ab(1u, false, false, kDtcN, kDtcKeys);
  constexpr uint32_t kIdescPV = tc::instr_desc_ab(1u, true, false, kDtcN, kDtcD);
  constexpr int kS = 3;            // S^T and P^T buffers
  // TMEM: S^T 0 | S^T 1 | S^T 2 | O^T (one 16-column accumulator per 128 head_dim rows)
  constexpr uint32_t kOCol = 48;
  constexpr uint32_t kTmemCols = kHalves == 1 ? 64 : 128;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sK = smem;
  unsigned char* sV = sK + KS * kDtcTileBytes;
  unsigned char* sQ = sV + VS * kDtcTileBytes;  // two buffers
  unsigned char* sP = sQ + 2 * kQBytes;                 // three buffers
  float* s_merge = reinterpret_cast<float*>(sP + kS * kDtcPBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(s_merge) +
                                               kDtcMergeBytes);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;  // [kS] S^T buffers
  uint64_t* p_full = s_full + kS;           // [kS] P^T buffers written
  uint64_t* o_done = p_full + kS;           // [2] the P.V products of even / odd tiles
  uint64_t* o_final = o_done + 2;           // a unit's last P.V
  uint64_t* q_ready = o_final + 1;          // [2] Q^T buffers written
  uint64_t* o_free = q_ready + 2;           // a unit's O^T read
  uint64_t* mma_drained = o_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drained + 1);
  __shared__ float red_max[2][4][kDtcN];
  __shared__ int red_fail[2][4];
  __shared__ float red_sum[4][kDtcN];
  __shared__ int last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < kS; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&o_done[b], 1);
      mbar_init(&q_ready[b], 128);
    }
    mbar_init(o_final, 1);
    mbar_init(o_free, 128);
    mbar_init(mma_drained, 1);
    mbar_fence_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp == 6) {
    // ---- TMA producers: warp 0 the K tiles, warp 6 the V tiles ----------------------------
    if (lane == 0) {
      const bool keys = warp == 0;
      uint64_t* full = keys ? k_full : v_full;
      uint64_t* empty = keys ? k_empty : v_empty;
      unsigned char* dst = keys ? sK : sV;
      const int stages = keys ? KS : VS;
      pdl_wait();  // the keys and values kept by the kernel before this one
      int T = 0, issued = 0;
      bool ok = true;
      for (int i = a.cta_first[blockIdx.x]; ok && i < a.cta_first[blockIdx.x + 1]; ++i) {
        int row, kv, j0, j1;
        dtc_unit(a, a.order[i], &row, &kv, &j0, &j1);
        const DtcRow& r = a.rows[row];
        const void* map = keys ? r.kmap : r.vmap;
        const int tiles = (j1 - j0 + kDtcKeys - 1) / kDtcKeys;
        for (int e = 0; e < tiles * kHalves; ++e, ++T) {
          // ring entry T: head_dim half e % kHalves of the unit's tile e / kHalves
          const int st = T % stages;
          const int t = e / kHalves, half = e % kHalves;
          if (!mbar_wait(&empty[st], ((T / stages) & 1) ^ 1, a.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[st], kDtcTileBytes);
          for (int db = 0; db < kDtcD / 64; ++db)
            tc::tma_load_3d(dst + st * kDtcTileBytes + db * (kDtcKeys * 128), map,
                            half * kDtcD + db * 64, r.b0 + j0 + t * kDtcKeys, r.z0 + kv, &full[st]);
          issued = T + 1;
        }
      }
      // The loads still in flight land before the CTA may exit.
      for (int L = max(0, issued - stages); L < issued; ++L)
        mbar_wait(&full[L % stages], (L / stages) & 1, a.err);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------------
    if (lane == 0) {
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t q_base = smem_u32(sQ), p_base = smem_u32(sP);
      bool ok = true;
      int T = 0, ui = 0;
      // O^T += V^T P^T of global tile T2 (`first`: the first of its unit, which overwrites O^T),
      // one accumulator per head_dim half (V ring entries T2 * kHalves + h)
      auto issue_pv = [&](int T2, bool first) {
        const int b = T2 % kS;
        if (first && ui > 0 && !mbar_wait(o_free, (ui - 1) & 1, a.err)) return false;
        if (!mbar_wait(&p_full[b], (T2 / kS) & 1, a.err)) return false;
#pragma unroll
        for (int h = 0; h < kHalves; ++h) {
          const int E = T2 * kHalves + h, st = E % VS;
          if (!mbar_wait(&v_full[st], (E / VS) & 1, a.err)) return false;
          tc::fence_after_sync();
#pragma unroll
          for (int k = 0; k < kDtcKeys / 16; ++k) {
            // A = V^T: the V entry's rows are keys (the K of this product), 64-element head_dim
            // blocks kDtcKeys * 128 bytes apart (M-major, 128-byte swizzle)
            const uint64_t ad = tc::smem_desc(v_base + st * kDtcTileBytes + k * 16 * 128,
                                              kDtcKeys * 128, 1024, tc::kSwizzle128B);
            const uint64_t bd = tc::smem_desc_sw128(
                p_base + b * kDtcPBytes + (k >> 2) * (kDtcN * 128) + (k & 3) * 32, 16, 1024);
            tc::mma_ss<false>(tmem + kOCol + 16 * h, ad, bd, kIdescPV,
                              (!first || k > 0) ? 1u : 0u);
          }
          tc::commit(&v_empty[st]);
        }
        tc::commit(&o_done[T2 & 1]);
        return true;
      };
      for (int i = a.cta_first[blockIdx.x]; ok && i < a.cta_first[blockIdx.x + 1]; ++i, ++ui) {
        int row, kv, j0, j1;
        dtc_unit(a, a.order[i], &row, &kv, &j0, &j1);
        const int tiles = (j1 - j0 + kDtcKeys - 1) / kDtcKeys;
        const int T0 = T;
        const int qb = ui & 1;
        if (!mbar_wait(&q_ready[qb], (ui >> 1) & 1, a.err)) { ok = false; break; }
        for (int t = 0; t < tiles; ++t, ++T) {
          // S^T of tile T over its head_dim halves (K ring entries T * kHalves + h)
#pragma unroll
          for (int h = 0; h < kHalves; ++h) {
            const int E = T * kHalves + h, st = E % KS;
            if (!mbar_wait(&k_full[st], (E / KS) & 1, a.err)) { ok = false; break; }
            tc::fence_after_sync();
#pragma unroll
            for (int k = 0; k < kDtcD / 16; ++k) {
              const int db = k >> 2, koff = (k & 3) * 32;
              const uint64_t ad = tc::smem_desc_sw128(
                  k_base + st * kDtcTileBytes + db * (kDtcKeys * 128) + koff, 16, 1024);
              const uint64_t bd = tc::smem_desc_sw128(
                  q_base + qb * kQBytes + (h * 2 + db) * (kDtcN * 128) + koff, 16, 1024);
              tc::mma_ss<false>(tmem + (T % kS) * 16, ad, bd, kIdescS,
                                (h > 0 || k > 0) ? 1u : 0u);
            }
            tc::commit(&k_empty[st]);
          }
          if (!ok) break;
          tc::commit(&s_full[T % kS]);
          // the P.V of two tiles back: S^T_{T+1} may then reuse that tile's S^T buffer
          if (t >= 2 && !issue_pv(T - 2, t == 2)) { ok = false; break; }
        }
        if (!ok) break;
        for (int t = max(0, tiles - 2); t < tiles; ++t)
          if (!issue_pv(T0 + t, t == 0)) { ok = false; break; }
        if (!ok) break;
        tc::commit(o_final);
      }
      // Every MMA this thread issued has completed before the CTA may free TMEM.
      tc::commit(mma_drained);
      mbar_wait(mma_drained, 0, a.err);
    }
  } else {
    // ---- softmax + epilogue: 128 threads, thread = key of S^T and head_dim row of O^T -------
    const int tid = threadIdx.x - 64;
    const int wq = warp & 3;              // the TMEM lane quarter this warp may access
    const int lane_row = wq * 32 + lane;  // key within a tile; head_dim element of O^T
    const int sw = warp - 2;              // this warp's slot in the cross-warp reductions
    const uint32_t lane_base = tmem + (uint32_t(wq * 32) << 16);
    // Q^T and P^T buffers start zero: the padding rows (heads >= group) stay zero.
    for (int i = tid; i < (2 * kQBytes + kS * kDtcPBytes) / 16; i += 128)
      reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
    named_sync(1, 128);
    const int g = a.group;
    // unit u's Q^T (bf16) into buffer qb, then announced to the MMA issuer
    auto write_q = [&](int u, int qb) {
      int row, kv, j0, j1;
      dtc_unit(a, u, &row, &kv, &j0, &j1);
      const float* qrow = a.q + int64_t(row) * a.q_stride + int64_t(kv * g) * D;
      unsigned char* qdst = sQ + qb * kQBytes;
      for (int i = tid; i < g * D; i += 128)
        *reinterpret_cast<__nv_bfloat16*>(qdst + dtc_op_offset(i / D, i % D)) =
            __float2bfloat16_rn(qrow[i]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&q_ready[qb]);
    };
    // A wait that gives up clears `ok` for its warp; the group leaves its loops only together,
    // at a barrier that ORs the failures (so no warp is left alone at a later barrier).
    bool ok = true;
    int T = 0, ui = 0;
    pdl_wait();  // the rotated queries written by the kernel before this one
    const int i_first = a.cta_first[blockIdx.x], i_end = a.cta_first[blockIdx.x + 1];
    if (i_first < i_end) write_q(a.order[i_first], 0);
    for (int i = i_first; i < i_end; ++i, ++ui) {
      const int u = a.order[i];
      int row, kv, j0, j1;
      dtc_unit(a, u, &row, &kv, &j0, &j1);
      const DtcRow& r = a.rows[row];
      const int tiles = (j1 - j0 + kDtcKeys - 1) / kDtcKeys;
      const int h0 = kv * g;
      // The next unit's Q^T into the other buffer: its previous unit's products have completed
      // (this group consumed their S^T).
      if (i + 1 < i_end) write_q(a.order[i + 1], (ui + 1) & 1);
      float m[kG], lp[kG];
#pragma unroll
      for (int h = 0; h < kG; ++h) {
        m[h] = -INFINITY;
        lp[h] = 0.0f;
      }
      bool failed = false;
      for (int t = 0; t < tiles; ++t, ++T) {
        const int b = T % kS;
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (T / kS) & 1, a.err));
        uint32_t sr[16];
        if (ok) {
          tc::fence_after_sync();
          tc::tmem_ld16_wait(lane_base + b * 16, sr);
        }
        const bool visible = ok && j0 + t * kDtcKeys + lane_row < j1;
        float x[kG];
        bool exceed = false;
#pragma unroll
        for (int h = 0; h < kG; ++h) {
          x[h] = (h < g && visible) ? __uint_as_float(sr[h]) * a.scale_log2 : -INFINITY;
          // the lazy max moves only for a score 2^8 above it (any finite one when it is -inf)
          exceed |= x[h] > m[h] + 8.0f;
        }
        if (named_sync_or(1, 128, exceed || !ok)) {
          // Some head's max moves (every first tile of a unit), or a wait gave up: the heads'
          // maxima over the tile's 128 keys, then the moves.
          const int rb = T & 1;
#pragma unroll
          for (int h = 0; h < kG; ++h) {
            float mx = x[h];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            if (lane == 0) red_max[rb][sw][h] = mx;
          }
          if (lane == 0) red_fail[rb][sw] = ok ? 0 : 1;
          named_sync(1, 128);
          if (red_fail[rb][0] | red_fail[rb][1] | red_fail[rb][2] | red_fail[rb][3]) {
            failed = true;
            break;
          }
          bool rescale = false;
          float alpha[kG];
#pragma unroll
          for (int h = 0; h < kG; ++h) {
            const float mt = fmaxf(fmaxf(red_max[rb][0][h], red_max[rb][1][h]),
                                   fmaxf(red_max[rb][2][h], red_max[rb][3][h]));
            alpha[h] = 1.0f;
            if (mt > m[h] + 8.0f || (m[h] == -INFINITY && mt > -INFINITY)) {
              if (m[h] > -INFINITY) {
                alpha[h] = exp2_approx(m[h] - mt);
                rescale = true;
              }
              m[h] = mt;
            }
          }
          if (rescale) {  // uniform: every thread saw the same maxima
            // O^T holds the products of this unit's tiles before T: wait for the last of them
            // (P.V of tile T - 1, on the barrier of its parity; the one before it on that
            // barrier, T - 3, completed before S^T_T, and T + 1 needs this group's P first).
#pragma unroll
            for (int h = 0; h < kG; ++h) lp[h] *= alpha[h];
            ok = __all_sync(0xffffffffu, mbar_wait(&o_done[(T - 1) & 1], ((T - 1) >> 1) & 1, a.err));
            if (ok) {
              tc::fence_after_sync();
#pragma unroll
              for (int hf = 0; hf < kHalves; ++hf) {
                uint32_t o[16];
                tc::tmem_ld16_wait(lane_base + kOCol + 16 * hf, o);
#pragma unroll
                for (int h = 0; h < kG; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
                tc::tmem_st16(lane_base + kOCol + 16 * hf, o);
                tc::tmem_wait_st();
              }
            }
          }
        }
        float p[kG];
#pragma unroll
        for (int h = 0; h < kG; ++h) {
          p[h] = (h < g && visible) ? exp2_approx(x[h] - m[h]) : 0.0f;
          lp[h] += p[h];
        }
        // P^T_T into buffer b: the P.V that read it (tile T - 3) completed before S^T_T did
        if (ok) {
          unsigned char* pb = sP + b * kDtcPBytes;
#pragma unroll
          for (int h = 0; h < kG; ++h)
            if (h < g)
              *reinterpret_cast<__nv_bfloat16*>(pb + dtc_op_offset(h, lane_row)) = __float2bfloat16_rn(p[h]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc::fence_before_sync();
          mbar_arrive(&p_full[b]);
        }
      }
      // ---- the unit's end: L per head, O^T / L (or the chunk's partial) -------------------
#pragma unroll
      for (int h = 0; h < kG; ++h) {
        float sm = lp[h];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
        if (lane == 0) red_sum[sw][h] = sm;
      }
      if (failed || named_sync_or(1, 128, !ok)) break;
      float L[kG];
#pragma unroll
      for (int h = 0; h < kG; ++h)
        L[h] = (red_sum[0][h] + red_sum[1][h]) + (red_sum[2][h] + red_sum[3][h]);
      ok = __all_sync(0xffffffffu, mbar_wait(o_final, ui & 1, a.err));
      uint32_t o[kHalves][16];
      if (ok) {
        tc::fence_after_sync();
#pragma unroll
        for (int hf = 0; hf < kHalves; ++hf) tc::tmem_ld16_wait(lane_base + kOCol + 16 * hf, o[hf]);
        tc::fence_before_sync();
        mbar_arrive(o_free);  // the next unit's first P.V may overwrite O^T
      }
      // this thread's head_dim elements: lane_row of each 128-row half
      if (r.chunks == 1) {
        if (ok) {
          float* orow = a.out + int64_t(row) * a.out_stride + int64_t(h0) * D;
#pragma unroll
          for (int hf = 0; hf < kHalves; ++hf)
#pragma unroll
            for (int h = 0; h < kG; ++h)
              if (h < g)
                orow[h * D + hf * kDtcD + lane_row] =
                    L[h] > 0.0f ? __uint_as_float(o[hf][h]) / L[h] : 0.0f;
        }
        continue;
      }
      const int chunk = (u - r.unit_begin) % r.chunks;
      const int64_t slot0 = int64_t(r.part_base + chunk) * a.heads + h0;
      if (ok) {
#pragma unroll
        for (int h = 0; h < kG; ++h) {
          if (h >= g) continue;
#pragma unroll
          for (int hf = 0; hf < kHalves; ++hf)
            a.part_o[(slot0 + h) * D + hf * kDtcD + lane_row] = __uint_as_float(o[hf][h]);
          if (lane_row == 0) {
            a.part_ml[2 * (slot0 + h)] = m[h];
            a.part_ml[2 * (slot0 + h) + 1] = L[h];
          }
        }
      }
      // the last CTA of this (row, KV head) to arrive merges the chunks
      __threadfence();
      if (named_sync_or(1, 128, !ok)) break;
      if (tid == 0) {
        int* counter = a.counters + int64_t(row) * a.kv_heads + kv;
        const int arrived = atomicAdd(counter, 1);
        last_flag = arrived == r.chunks - 1;
        if (last_flag) *counter = 0;  // ready for the next launch
      }
      named_sync(1, 128);
      if (!last_flag) continue;
      __threadfence();
      float* orow = a.out + int64_t(row) * a.out_stride;
      merge_chunk_partials<kG, D, 128>(
          a.part_o, a.part_ml, a.heads, h0, g, r.part_base, r.chunks, s_merge,
          kDtcMergeBytes / (4 * kG), 1, tid,
          [&](int h, int e, float, float ll, float oo) {
            orow[(h0 + h) * D + e] = ll > 0.0f ? oo / ll : 0.0f;
          });
    }
  }

  // ---- teardown: every TMEM user is done before the owner frees it ---------------------------
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace fa
