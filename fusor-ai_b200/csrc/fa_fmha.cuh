// The compute-bound half of the hot path: prefill (Span rows > 1) and full-mask attention as a
// tcgen05 tensor-core flash-attention forward pass (KvCache::attend over many rows,
// transformer.rs:182-219; blocks::attention::attend / dit::Within, attention.rs:79-95,
// dit.rs:135-166), with the f32 ops::attend semantics (ops.rs:310-342).
//
// One CTA = 128 query rows of one query head. Warp roles:
//   warp 0      TMA producer: Q once, then K and V tiles into a ring of shared-memory stages
//               (128-byte swizzled; tf32 V with 32-byte swizzle atoms, the MN-major tf32
//               layout; plain per-CTA loads only);
//   warp 1      TMEM owner and MMA issuer (one thread): S = Q K^T into one of two TMEM
//               buffers, then O += P V with P read from TMEM (the TS form);
//   warps 2-3   (tf32) the rounding pass: Q and every K and V tile rounded to tf32 (nearest)
//               in shared memory between the TMA's landing and the MMA that reads it; at
//               head_dim 128 also warps 8-11, so that the pass runs on all four of the SM's
//               schedulers (fmha_threads);
//   warps 4-7   softmax: thread i owns query row i (TMEM lane i); it loads its S row, masks,
//               updates the running max lazily (the output is rescaled only when the max grows
//               by more than 2^8, FA4's trick), writes P back into the S buffer (bf16 pairs, or
//               tf32) and finally normalises O and stores it.
// The MMA order S_0, S_1, PV_0, S_2, PV_1, ... keeps the tensor core on S_{j+1} while the
// softmax works on S_j (the lookahead and the buffer and stage counts are parameters of the
// shape: FmhaShape).
//
// T = __nv_bfloat16 runs kind::f16 (bf16 operands, f32 accumulation); T = float runs kind::tf32
// on f32 data (the f32-I/O path).
#pragma once

#include "fa_decode.cuh"
#include "fa_fmha_launch.h"
#include "fa_tc.cuh"

namespace fa {

// head_dim 256 (bf16 only): 64-key tiles, so that Q (64 KB) and two stages of K and V (32 KB
// each) fit in shared memory, and two S buffers of 64 columns beside O's 256 in TMEM.
template <typename T, int D>
struct FmhaShape {
  static constexpr bool kTf32 = sizeof(T) == 4;
  static constexpr int BM = 128;                               // query rows per CTA
  static constexpr int BN = (D == 256 || (kTf32 && D == 128)) ? 64 : 128;  // keys per KV tile
  static constexpr int kElem = int(sizeof(T));
  static constexpr int kBlock = 128 / kElem;                   // elements per swizzled 128 B row
  static constexpr int kDBlocks = D / kBlock;
  static constexpr int kKStep = 32 / kElem;                    // elements per MMA K step
  // S (P) buffers in TMEM, S products ahead of P.V, K and V tiles in shared memory. Measured on
  // B200 over 64-key tiles (the Qwen3.5 prefill at head_dim 256, the f32 prefill on tf32): three
  // S buffers with three K stages, or a third K or V stage alone, ran 1-2 % slower than this.
  static constexpr int kSBufs = 2;
  static constexpr int kLookahead = kSBufs - 1;
  static constexpr int kKStages = 2;
  static constexpr int kVStages = 2;
  static constexpr int kQBytes = BM * D * kElem;
  static constexpr int kKVBytes = BN * D * kElem;
  static constexpr int kSCols = BN;                            // TMEM columns of one S buffer
  static constexpr int kOCol = 256;                            // TMEM column of O
  static constexpr int kPCols = kTf32 ? BN : BN / 2;           // TMEM columns of P
  static constexpr size_t kSmemUsed = size_t(kQBytes) + size_t(kKStages + kVStages) * kKVBytes +
                                      1024 /* alignment */ + 256 /* bars */;
  // At least 120 KB so that one CTA holds an SM: each CTA allocates all 512 TMEM columns.
  static constexpr size_t kSmemBytes = kSmemUsed > 122880 ? kSmemUsed : 122880;
  static_assert(D % kBlock == 0, "head_dim a multiple of the swizzle block");
  static_assert(BN % 32 == 0 && D % 32 == 0, "TMEM loads of 32 columns");
  static_assert(kOCol + D <= 512 && kSBufs * kSCols <= kOCol, "the S buffers and O in 512 columns");
  static_assert(kSmemUsed <= 227 * 1024, "shared memory of one CTA");
};

// Threads of an instantiation: warps 0-1 (TMA, MMA), 2-3 (the tf32 rounding pass), 4-7
// (softmax), and for the f32 kernel of head_dim 128 warps 8-11 (more of the rounding pass, which
// is on the critical path of every KV tile: measured on B200 over the 8192-row f32 prefill,
// 1.618 ms with two rounding warps, 1.401 with four, 1.377 with six). The head_dim-64 f32 kernel
// keeps 256 threads: it holds 218 registers a thread, above the 168 that 384 threads allow.
template <typename T, int D>
__host__ __device__ constexpr int fmha_threads() {
  return FmhaShape<T, D>::kTf32 && D == 128 ? 384 : 256;
}
template <typename T, int D>
__host__ __device__ constexpr int fmha_conv_threads() { return fmha_threads<T, D>() - 192; }

// Rounds `bytes` of f32 shared memory to tf32 (nearest, ties away) in place, 16 bytes per
// thread per step, four steps' loads in flight at a time (the pass is on the critical path of
// every KV tile). The swizzled layout is untouched: the same function of every element.
template <int kConvThreads>
__device__ __forceinline__ void round_tile_tf32(unsigned char* tile, int bytes, int tid) {
  float4* v = reinterpret_cast<float4*>(tile);
  const int n = bytes / 16;
  int i = tid;
  for (; i + 3 * kConvThreads < n; i += 4 * kConvThreads) {
    float4 x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = v[i + k * kConvThreads];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[k].x = __uint_as_float(tc::round_tf32(x[k].x));
      x[k].y = __uint_as_float(tc::round_tf32(x[k].y));
      x[k].z = __uint_as_float(tc::round_tf32(x[k].z));
      x[k].w = __uint_as_float(tc::round_tf32(x[k].w));
      v[i + k * kConvThreads] = x[k];
    }
  }
  for (; i < n; i += kConvThreads) {
    float4 x = v[i];
    x.x = __uint_as_float(tc::round_tf32(x.x));
    x.y = __uint_as_float(tc::round_tf32(x.y));
    x.z = __uint_as_float(tc::round_tf32(x.z));
    x.w = __uint_as_float(tc::round_tf32(x.w));
    v[i] = x;
  }
}


template <typename T, int D>
__global__ void __launch_bounds__(fmha_threads<T, D>(), 1)
    fmha_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                const __grid_constant__ CUtensorMap v_map, const __grid_constant__ FmhaArgs a) {
  using S = FmhaShape<T, D>;
  constexpr int BM = S::BM, BN = S::BN;
  constexpr bool kTf32 = S::kTf32;
  constexpr uint32_t kFmt = kTf32 ? 2u : 1u;
  constexpr uint32_t kIdescQK = tc::instr_desc(kFmt, false, BN, BM);
  constexpr uint32_t kIdescPV = tc::instr_desc(kFmt, true, D, BM);

  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NB = S::kSBufs, L = S::kLookahead, KS = S::kKStages, VS = S::kVStages;
  unsigned char* sQ = smem;
  unsigned char* sK = sQ + S::kQBytes;
  unsigned char* sV = sK + KS * S::kKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * S::kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;       // [KS]
  uint64_t* k_empty = k_full + KS;   // [KS]
  uint64_t* v_full = k_empty + KS;   // [VS]
  uint64_t* v_empty = v_full + VS;   // [VS]
  uint64_t* s_full = v_empty + VS;   // [NB]
  uint64_t* p_full = s_full + NB;    // [NB]
  uint64_t* o_done = p_full + NB;    // [NB]: P.V of tile j completes phase j / NB of o_done[j % NB]
  uint64_t* o_final = o_done + NB;   // the last P.V product has completed
  uint64_t* mma_drained = o_final + 1;
  // tf32: Q, K and V tiles rounded to tf32 in place by the rounding warps before the MMA reads
  // them
  uint64_t* q_conv = mma_drained + 1;
  uint64_t* k_conv = q_conv + 1;     // [KS]
  uint64_t* v_conv = k_conv + KS;    // [VS]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_conv + VS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The CTA's query head and tile: band by band, each band's heaviest tiles first across its
  // heads (longest-processing-time order within the band; its K/V stays in L2 meanwhile).
  const int band_heads = a.band_heads > 0 ? a.band_heads : a.group;
  const int tiles = a.images * a.q_tiles;
  const int band = int(blockIdx.x) / (tiles * band_heads);
  const int in_band = int(blockIdx.x) - band * tiles * band_heads;
  const int head = band * band_heads + in_band % band_heads;
  const int kv = head / a.group;
  const int tile_id = tiles - 1 - in_band / band_heads;
  const int image = tile_id / a.q_tiles;
  const int r0 = (tile_id % a.q_tiles) * BM;
  const int r_last = min(r0 + BM, a.rows) - 1;

  // KV tiles the CTA's rows see: the union of their key runs.
  int lo, hi;
  {
    const Runs first_runs = mask_runs(a.kind, a.window, a.state, a.n_ends, a.ends, a.first + r0, a.end);
    const Runs last_runs = mask_runs(a.kind, a.window, a.state, a.n_ends, a.ends, a.first + r_last, a.end);
    lo = first_runs.b0;
    hi = max(last_runs.b0 + last_runs.n0, last_runs.b1 + last_runs.n1);
    if (a.kind == 3) { lo = 0; hi = a.end; }  // Groups: every run lies in [0, end)
  }
  const int t0 = lo / BN;
  const int n_tiles = (hi + BN - 1) / BN - t0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int st = 0; st < KS; ++st) {
      mbar_init(&k_full[st], 1);
      mbar_init(&k_empty[st], 1);
      mbar_init(&k_conv[st], fmha_conv_threads<T, D>());
    }
    for (int st = 0; st < VS; ++st) {
      mbar_init(&v_full[st], 1);
      mbar_init(&v_empty[st], 1);
      mbar_init(&v_conv[st], fmha_conv_threads<T, D>());
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&o_done[b], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(mma_drained, 1);
    mbar_init(q_conv, fmha_conv_threads<T, D>());
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
      mbar_arrive_expect_tx(q_full, S::kQBytes);
      const int qy = image * a.q_row_base_per_image + r0;
      for (int db = 0; db < S::kDBlocks; ++db)
        tc::tma_load_3d(sQ + db * BM * 128, &q_map, db * S::kBlock, qy, head, q_full);
      const int kz = a.kv_layer_base + kv;
      const int ky0 = image * a.kv_row_base_per_image;
      // In the order the MMAs take them: K_0 .. K_L, then V_j and K_{j+L+1} for each j.
      auto load_k = [&](int j) {
        const int st = j % KS;
        if (!mbar_wait(&k_empty[st], ((j / KS) & 1) ^ 1, a.err)) return false;
        mbar_arrive_expect_tx(&k_full[st], S::kKVBytes);
        for (int db = 0; db < S::kDBlocks; ++db)
          tc::tma_load_3d(sK + st * S::kKVBytes + db * BN * 128, &k_map, db * S::kBlock,
                          ky0 + (t0 + j) * BN, kz, &k_full[st]);
        return true;
      };
      auto load_v = [&](int j) {
        const int st = j % VS;
        if (!mbar_wait(&v_empty[st], ((j / VS) & 1) ^ 1, a.err)) return false;
        mbar_arrive_expect_tx(&v_full[st], S::kKVBytes);
        for (int db = 0; db < S::kDBlocks; ++db)
          tc::tma_load_3d(sV + st * S::kKVBytes + db * BN * 128, &v_map, db * S::kBlock,
                          ky0 + (t0 + j) * BN, kz, &v_full[st]);
        return true;
      };
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int j = 0; ok && j <= L && j < n_tiles; ++j)
        if ((ok = load_k(j))) k_issued = j + 1;
      for (int j = 0; ok && j < n_tiles; ++j) {
        if ((ok = load_v(j))) v_issued = j + 1;
        if (ok && j + L + 1 < n_tiles && (ok = load_k(j + L + 1))) k_issued = j + L + 2;
      }
      // The loads still in flight land before the CTA may exit (they have, unless a wait gave
      // up: every full barrier of the last stages completes once its bytes arrive).
      mbar_wait(q_full, 0, a.err);
      for (int j = max(0, k_issued - KS); j < k_issued; ++j)
        mbar_wait(&k_full[j % KS], (j / KS) & 1, a.err);
      for (int j = max(0, v_issued - VS); j < v_issued; ++j)
        mbar_wait(&v_full[j % VS], (j / VS) & 1, a.err);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------------
    if (lane == 0) {
      // The descriptors differ only in their start address (16-byte units in the low bits;
      // shared-memory addresses stay below 2^18): built once, offsets added per stage and K step
      // (the issue of the MMAs is on this thread's critical path).
      const uint64_t q_desc = tc::smem_desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc = tc::smem_desc_sw128(smem_u32(sK), 16, 1024);
      // V is the MN-major B operand: rows of 128 bytes of one head_dim block, blocks BN*128 bytes
      // apart; bf16 in 8-row 128-byte-swizzle atoms, tf32 in the only MN-major tf32 layout, 4-row
      // atoms of 32-byte chunks.
      const uint64_t v_desc =
          kTf32 ? tc::smem_desc(smem_u32(sV), BN * 128, 512, tc::kSwizzle128BAtom32B)
                : tc::smem_desc(smem_u32(sV), BN * 128, 1024, tc::kSwizzle128B);
      bool ok = mbar_wait(kTf32 ? q_conv : q_full, 0, a.err);
      auto issue_pv = [&](int j) {
        const int st = j % VS;
        const int b = j % NB;
        if (!mbar_wait(&p_full[b], (j / NB) & 1, a.err)) return false;
        if (!mbar_wait(kTf32 ? &v_conv[st] : &v_full[st], (j / VS) & 1, a.err)) return false;
        tc::fence_after_sync();
        const uint32_t p_tmem = tmem + uint32_t(b * S::kSCols);
        const uint64_t vd0 = v_desc + uint64_t(st) * uint64_t(S::kKVBytes >> 4);
#pragma unroll
        for (int k = 0; k < BN / S::kKStep; ++k)
          tc::mma_ts<kTf32>(tmem + S::kOCol, p_tmem + k * 8,
                            vd0 + uint64_t((k * S::kKStep * 128) >> 4), kIdescPV,
                            (j > 0 || k > 0) ? 1u : 0u);
        tc::commit(&o_done[b]);
        tc::commit(&v_empty[st]);
        return true;
      };
      // S_t into buffer t % NB, which held P_{t-NB}: its P.V was issued the step before (the
      // tensor core runs one thread's MMAs in issue order).
      for (int t = 0; ok && t < n_tiles + L; ++t) {
        if (t < n_tiles) {
          const int st = t % KS;
          const int b = t % NB;
          if (!mbar_wait(kTf32 ? &k_conv[st] : &k_full[st], (t / KS) & 1, a.err)) { ok = false; break; }
          tc::fence_after_sync();
          const uint64_t kd0 = k_desc + uint64_t(st) * uint64_t(S::kKVBytes >> 4);
#pragma unroll
          for (int k = 0; k < D / S::kKStep; ++k) {
            const int db = k / (128 / 32), koff = (k % (128 / 32)) * 32;
            tc::mma_ss<kTf32>(tmem + b * S::kSCols, q_desc + uint64_t((db * BM * 128 + koff) >> 4),
                              kd0 + uint64_t((db * BN * 128 + koff) >> 4), kIdescQK,
                              k > 0 ? 1u : 0u);
          }
          tc::commit(&s_full[b]);
          tc::commit(&k_empty[st]);
        }
        if (t >= L && !issue_pv(t - L)) { ok = false; break; }
      }
      if (ok && n_tiles > 0) tc::commit(o_final);
      // Every MMA this thread issued has completed before the CTA may free TMEM.
      tc::commit(mma_drained);
      mbar_wait(mma_drained, 0, a.err);
    }
  } else if (warp < 4 || warp >= 8) {
    // ---- tf32: round Q, then every K and V tile, to nearest before the MMA reads them -------
    if constexpr (kTf32) {
      const int tid = warp < 4 ? int(threadIdx.x) - 64 : int(threadIdx.x) - 192;
      auto convert = [&](uint64_t* full, uint64_t* conv, uint32_t parity, unsigned char* tile,
                         int bytes) {
        if (!mbar_wait(full, parity, a.err)) return false;
        round_tile_tf32<fmha_conv_threads<T, D>()>(tile, bytes, tid);
        // generic-proxy writes become visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(conv);
        return true;
      };
      // in the producer's order: K_0 .. K_L, then V_j and K_{j+L+1}
      auto conv_k = [&](int j) {
        return convert(&k_full[j % KS], &k_conv[j % KS], (j / KS) & 1, sK + (j % KS) * S::kKVBytes,
                       S::kKVBytes);
      };
      auto conv_v = [&](int j) {
        return convert(&v_full[j % VS], &v_conv[j % VS], (j / VS) & 1, sV + (j % VS) * S::kKVBytes,
                       S::kKVBytes);
      };
      bool ok = convert(q_full, q_conv, 0, sQ, S::kQBytes);
      for (int j = 0; ok && j <= L && j < n_tiles; ++j) ok = conv_k(j);
      for (int j = 0; ok && j < n_tiles; ++j) {
        ok = conv_v(j);
        if (ok && j + L + 1 < n_tiles) ok = conv_k(j + L + 1);
      }
    }
  } else {
    // ---- softmax + epilogue (warps 4-7) ----------------------------------------------------
    const int wq = warp - 4;
    const int r = r0 + wq * 32 + lane;  // this thread's query row within the image
    const bool row_valid = r < a.rows;
    const Runs runs = mask_runs(a.kind, a.window, a.state, a.n_ends, a.ends, a.first + r, a.end);
    const uint32_t lane_base = tmem + (uint32_t(wq * 32) << 16);
    float m_used = -INFINITY, l_sum = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j % NB;
      const int kp = (t0 + j) * BN;  // first key position of the tile
      // Every decision before a whole-warp tcgen05 instruction is made warp-uniform.
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (j / NB) & 1, a.err))) { ok = false; break; }
      tc::fence_after_sync();
      uint32_t sreg[BN];
      if constexpr (BN == 128) tc::tmem_ld128_wait(lane_base + b * S::kSCols, sreg);
      else tc::tmem_ld64_wait(lane_base + b * S::kSCols, sreg);
      float* s = reinterpret_cast<float*>(sreg);
      // A row past the end of the image's queries is never written back, and its P row reaches
      // only its own O row (the tensor-core product is row by row), so it skips the masking:
      // its Q row (the next image's query, or the TMA's zero fill) needs no -inf either.
      const bool all_in = !row_valid ||
                          (kp >= runs.b0 && kp + BN <= runs.b0 + runs.n0) ||
                          (kp >= runs.b1 && kp + BN <= runs.b1 + runs.n1);
      if (!all_in) mask_scores<BN>(runs, kp, s);
      // the tile's max in four independent chains of three-input maxima (the chain is on the
      // critical path of every tile: one dependent maximum per key took a quarter of it)
      static_assert(BN % 8 == 0, "the max chains take 8 keys a step");
      float mx0 = fmax3(s[0], s[1], -INFINITY), mx1 = fmax3(s[2], s[3], -INFINITY);
      float mx2 = fmax3(s[4], s[5], -INFINITY), mx3 = fmax3(s[6], s[7], -INFINITY);
#pragma unroll
      for (int c = 8; c < BN; c += 8) {
        mx0 = fmax3(mx0, s[c], s[c + 1]);
        mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
        mx2 = fmax3(mx2, s[c + 4], s[c + 5]);
        mx3 = fmax3(mx3, s[c + 6], s[c + 7]);
      }
      const float m_tile = fmax3(mx0, mx1, fmaxf(mx2, mx3)) * a.scale_log2;  // -inf stays -inf
      // Lazy rescale: move the reference max only when the tile's max exceeds it by 2^8 (the
      // first finite max just sets it: nothing has accumulated for the row yet).
      float alpha = 1.0f;
      if (m_tile > m_used + 8.0f || (m_used == -INFINITY && m_tile > -INFINITY)) {
        if (m_used > -INFINITY) alpha = exp2_approx(m_used - m_tile);
        m_used = m_tile;
      }
      if (__any_sync(0xffffffffu, alpha != 1.0f)) {
        // O holds PV of tiles < j: wait for PV_{j-1}, then rescale the warp's rows.
        l_sum *= alpha;
        // A parity wait names only the current or the previous phase of a barrier. Here it is
        // unambiguous: S_j has completed, and its commit tracks every MMA issued before it,
        // P.V_{j-NB} among them; the barrier of P.V_{j-1}, o_done[(j-1) % NB], was last
        // completed by P.V_{j-1-NB}, so its phase (j-1) / NB is P.V_{j-1}'s own.
        const int jb = (j - 1) % NB;
        if (!__all_sync(0xffffffffu, mbar_wait(&o_done[jb], ((j - 1) / NB) & 1, a.err))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tc::tmem_ld32_wait(lane_base + S::kOCol + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tc::tmem_st32(lane_base + S::kOCol + c * 32, o);
          tc::tmem_wait_st();  // the registers are free again only after the store lands
        }
      }
      const float ms = m_used == -INFINITY ? 0.0f : m_used;
      float sum = 0.0f;
      if constexpr (kTf32) {
        float sums[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // independent chains
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const float p = exp2_approx(fmaf(s[c], a.scale_log2, -ms));
          sums[c & 3] += p;
          sreg[c] = tc::round_tf32(p);
        }
        sum = (sums[0] + sums[1]) + (sums[2] + sums[3]);
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tc::tmem_st32(lane_base + b * S::kSCols + c * 32,
                        *reinterpret_cast<const uint32_t(*)[32]>(&sreg[c * 32]));
      } else {
        // pairs of probabilities packed in place: sreg[c / 2] is written only after s[c] and
        // s[c + 1] are read; paired FFMA/FADD, the sums in two independent chains
        const float2 scale2 = make_float2(a.scale_log2, a.scale_log2);
        const float2 neg2 = make_float2(-ms, -ms);
        float2 sum2a = make_float2(0.0f, 0.0f), sum2b = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < BN; c += 4) {
          const float2 x0 = __ffma2_rn(make_float2(s[c], s[c + 1]), scale2, neg2);
          const float2 x1 = __ffma2_rn(make_float2(s[c + 2], s[c + 3]), scale2, neg2);
          const float2 p0 = make_float2(exp2_approx(x0.x), exp2_approx(x0.y));
          const float2 p1 = make_float2(exp2_approx(x1.x), exp2_approx(x1.y));
          sum2a = __fadd2_rn(sum2a, p0);
          sum2b = __fadd2_rn(sum2b, p1);
          sreg[c / 2] = tc::pack_bf16(p0.x, p0.y);
          sreg[c / 2 + 1] = tc::pack_bf16(p1.x, p1.y);
        }
        sum = (sum2a.x + sum2a.y) + (sum2b.x + sum2b.y);
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          tc::tmem_st32(lane_base + b * S::kSCols + c * 32,
                        *reinterpret_cast<const uint32_t(*)[32]>(&sreg[c * 32]));
      }
      l_sum += sum;
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&p_full[b]);
    }
    // ---- epilogue: O / l -------------------------------------------------------------------
    // The last P.V has its own single-phase barrier: after the loop o_done may still be two
    // phases short of done, where a parity wait would match an older completed phase.
    if (__all_sync(0xffffffffu, ok && n_tiles > 0 && mbar_wait(o_final, 0, a.err))) {
      tc::fence_after_sync();
      const float inv = l_sum > 0.0f ? 1.0f / l_sum : 0.0f;
      const int64_t orow = int64_t(image) * a.rows + r;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tc::tmem_ld32_wait(lane_base + S::kOCol + c * 32, o);
        if (!row_valid) continue;
        if (a.out_bf16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) +
                                                orow * a.out_stride + head * D + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(
                tc::pack_bf16(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                tc::pack_bf16(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                tc::pack_bf16(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                tc::pack_bf16(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
        } else {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) +
                                                  orow * a.out_stride + head * D + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                 __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
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
