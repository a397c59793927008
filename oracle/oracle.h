/*
 * CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain C++ restatement of fusor-ai's f32 attention path (the Scalar backend, which is what
 * the reference runs on an x86-64 host), used by the tests as the checker and by bench.py's
 * cpu_baseline / reference arm as the timed CPU implementation. Nothing in the product library
 * (libfa_attn.so) links, loads or calls this; the product fails loudly without its CUDA path.
 *
 * Every function cites the reference file:line it restates (paths relative to the fusor-ai
 * project root). Arithmetic order follows the reference exactly: no fused multiply-adds
 * (built with -ffp-contract=off), sums in index order starting from -0.0 as Rust's f32 `sum`.
 */
#ifndef FUSOR_ORACLE_H
#define FUSOR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* crates/kernels/src/ops.rs:70-74 */
void oracle_rope_inv_freq(float base, int head_dim, float* out);
/* crates/kernels/src/ops.rs:77-85 */
void oracle_rope_half(float* head, int head_dim, const float* cos, const float* sin);
/* crates/kernels/src/ops.rs:89-95 */
void oracle_rope_interleaved(float* head, int head_dim, const float* cos, const float* sin);

/* Rotation kinds of crates/blocks/src/rotary.rs:63-86. */
enum {
  ORACLE_ROT_SEQUENCE = 0,
  ORACLE_ROT_LINEAR = 1,
  ORACLE_ROT_PARTIAL = 2,
  ORACLE_ROT_MULTIMODAL = 3,
  ORACLE_ROT_AXES = 4,
  ORACLE_ROT_MULTIMODAL_INTERLEAVED = 5,
  ORACLE_ROT_GRID = 6
};
/* Rotary::new + spatially_scaled + angles (crates/blocks/src/rotary.rs:117-178). `params` holds
 * the factor / turning count / three sections of the rotation; `position` is (temporal, height,
 * width). Writes head_dim/2 cosines and sines. Returns 0, or -1 on sections that do not cover
 * half a head. */
int oracle_rotary_angles(int kind, const int64_t* params, float base, int head_dim,
                         float spatial_scale, const int64_t* position, float* cos, float* sin);

/* crates/kernels/src/ops.rs:121-131 (Cephes expf polynomial) and 147-157. */
float oracle_exp(float x);
float oracle_exp_fast(float x);
/* crates/kernels/src/ops.rs:294-298 */
float oracle_round_bf16(float value);
/* Exponentials::apply (ops.rs:170-175) with the Scalar sweep (arch/scalar.rs:96-126). */
float oracle_exponentials_apply(int fast, float* scores, int n);
/* crates/kernels/src/ops.rs:301-306 */
void oracle_softmax(float* scores, int n);
/* crates/kernels/src/arch/scalar.rs:112-114 */
float oracle_dot(const float* left, const float* right, int n);
/* crates/kernels/src/ops.rs:7-16 (one row) */
void oracle_rms_norm(const float* x, const float* weight, float eps, int dim, float* out);

/* ops::attend (ops.rs:310-326) + weigh (329-342) for one query over `keys` rows given by
 * pointers. `scores` is scratch of `keys` floats. */
void oracle_attend(const float* query, int head_dim, int keys, const float* const* key_rows,
                   const float* const* value_rows, float* scores, float* out);

/* Mask kinds of crates/blocks/src/transformer.rs:99-111. */
enum { ORACLE_MASK_CAUSAL = 0, ORACLE_MASK_WINDOW = 1, ORACLE_MASK_FULL = 2, ORACLE_MASK_GROUPS = 3 };
typedef struct {
  int kind;
  int64_t window;
  int64_t state;
  const int64_t* ends;
  int64_t n_ends;
} oracle_mask;

/* Mask::keys (transformer.rs:116-128): the two runs of positions [r[0], r[1]) and [r[2], r[3]). */
void oracle_mask_keys(const oracle_mask* mask, int64_t position, int64_t end, int64_t* runs);

/* A KvCache (transformer.rs:134-162) over caller-owned f32 arrays of
 * layers * kv_heads * capacity * head_dim values each. */
typedef struct {
  int64_t layers, heads, kv_heads, head_dim, capacity;
  float* keys;
  float* values;
} oracle_cache;

/* KvCache::offset (transformer.rs:263-269) */
int64_t oracle_cache_offset(const oracle_cache* cache, int64_t layer, int64_t kv_head,
                            int64_t position);
/* KvCache::keep (transformer.rs:166-180) */
void oracle_cache_keep(oracle_cache* cache, int64_t layer, int64_t unit, int64_t position,
                       const float* head);
/* Transformer::run's capacity rule (transformer.rs:331-338): 1 when the span fits. */
int oracle_span_fits(const oracle_cache* cache, int64_t rows, int64_t first,
                     const oracle_mask* mask);

/* Stack::attention_input's per-head part (layer.rs:194-208 with `position` 213-234): for every
 * row and unit, optional head RMSNorm (q_norm / k_norm may be NULL), RoPE by `angles` (rows x
 * head_dim: cosines then sines; rope 0 none, 1 half, 2 interleaved) on the query and key heads,
 * in place in `qkv` (rows x stride), then keep into the cache at position first + row. */
void oracle_attention_input(oracle_cache* cache, int64_t layer, int64_t rows, int64_t first,
                            int rope, const float* angles, const float* q_norm,
                            const float* k_norm, float norm_eps, float* qkv, int64_t stride);

/* KvCache::attend (transformer.rs:185-219) for every head (one thread), into out (rows x
 * heads*head_dim). */
void oracle_cache_attend(const oracle_cache* cache, int64_t layer, int64_t rows, int64_t first,
                         const oracle_mask* mask, const float* qkv, int64_t stride, float* out);

/* The same with the reference's team split of heads (transformer.rs:196, team.rs:46-129):
 * `threads` workers, one broadcast per call, static shares. */
void oracle_cache_attend_team(const oracle_cache* cache, int64_t layer, int64_t rows,
                              int64_t first, const oracle_mask* mask, const float* qkv,
                              int64_t stride, float* out, int threads);

/* Several independent caches (sequences), each one `forward` call of one row at position
 * firsts[i] under Mask::Causal, one team run per sequence (the reference has no batching). */
void oracle_decode_batch_team(const oracle_cache* caches, int64_t batch, int64_t layer,
                              const int64_t* firsts, const float* qkv, int64_t stride,
                              float* out, int64_t out_stride, int threads);

/* The f32 full-mask attention of a blocks::attention::Call (attention.rs:24-47, row indexing of
 * 81-95 and 157-214) with the f32 ops::attend arithmetic: query rows image*queries+q, key rows
 * image*keys+k, output rows of heads*head_dim. Heads `head_begin..head_end` and queries
 * `query_begin..query_end` of each image only (a bounded sample), split over `threads`. */
void oracle_attend_call(int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t images,
                        int64_t queries, int64_t keys, const float* q, int64_t q_stride,
                        int64_t q_offset, const float* k, int64_t k_stride, int64_t k_offset,
                        const float* v, int64_t v_stride, int64_t v_offset, float* out,
                        int64_t head_begin, int64_t head_end, int64_t query_begin,
                        int64_t query_end, int threads);

/* Transformer-XL relative-position full-mask attention of one conformer layer
 * (crates/blocks/src/conformer/attention.rs:25-159): for head h, query frame i and key frame j,
 * score = ((q_i + u) . k_j + (q_i + v) . r_{frames-1-i+j}) / sqrt(head_dim), softmax over j, times
 * v_j. Rows of q/k/v at q + i*q_stride + h*head_dim (and likewise), relative-position rows at
 * positions + rel*positions_stride + h*head_dim, bias_u/bias_v of heads*head_dim, output rows of
 * heads*head_dim. */
void oracle_relpos_attend(int64_t heads, int64_t head_dim, int64_t frames, const float* q,
                          const float* k, const float* v, int64_t qkv_stride,
                          const float* positions, int64_t positions_stride, const float* bias_u,
                          const float* bias_v, float* out);

/* The query/key prologue of the DiT blocks, in place in qkv (tokens rows of `stride`: queries,
 * keys, values of heads*head_dim): norm 1 is rms_rows over the whole query row and the whole key
 * row (wan_dit/block.rs:109-126, row_work.rs:57-75; weights heads*head_dim wide), norm 2 each
 * head on its own (mmdit/pass.rs:64-68,162-176; weights head_dim wide); then tokens below
 * `rotated` have every query and key head turned by their angles row (tokens x head_dim), rope 1
 * by halves, 2 interleaved (block.rs:127-139). */
void oracle_qk_prologue(int64_t tokens, int64_t heads, int64_t head_dim, int norm, int rope,
                        int64_t rotated, const float* angles, const float* q_norm,
                        const float* k_norm, float eps, float* qkv, int64_t stride);

/* The hybrid blocks' projected heads (hybrid/attention.rs:180-235): for each row and head unit
 * of a row (query heads, gate heads when gate == 1, key heads, value heads; head_dim each),
 * queries and keys head-normed (optional) and rotated by halves in their first rotary_dim
 * elements by angles (rows x rotary_dim), gates through their sigmoid, keys and values kept at
 * first + row; with gate == 2 the per-head gates after the value heads through their sigmoid
 * too. In place in qkv. */
void oracle_gated_input(oracle_cache* cache, int64_t layer, int64_t rows, int64_t first, int gate,
                        int64_t rotary_dim, const float* angles, const float* q_norm,
                        const float* k_norm, float norm_eps, float* qkv, int64_t stride);

/* Weights::gate (hybrid/attention.rs:262-295): each query head of attention (rows x
 * heads*head_dim) times its gates from qkv as oracle_gated_input left them. */
void oracle_gate(int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim, int gate,
                 const float* qkv, int64_t stride, float* attention);

/* blocks::attention::attend's int8 approximation (crates/blocks/src/attention.rs:79-214) of one
 * image's full-mask attention, for the comparison with the f32 and bf16 paths: per (head),
 * the keys less their mean over the keys (SageAttention's smoothing) and the transposed values
 * quantized as Q7b32 rows (per block of 32: d = absmax / 63, ties-even levels clamped to +-63,
 * quant.rs:131-149), the queries and the exponentials as int8 activations (per block of 32:
 * d = absmax / 127, matmul.rs:229-260), integer dot products per block scaled by d_w * d_a,
 * scores times 1/sqrt(head_dim), Exponentials::apply (exact or fast, ops.rs:163-191), and the
 * outputs divided by the exponentials' sums. q, k, v rows `*_stride` apart (head h at
 * h * head_dim), out rows of heads * head_dim. */
void oracle_attend_int8(int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t queries,
                        int64_t keys, const float* q, int64_t q_stride, const float* k,
                        int64_t k_stride, const float* v, int64_t v_stride, int fast, float* out);

/* Joins the team's worker threads (they are started on the first threaded call). */
void oracle_team_release(void);

/* The f64 reference of the block tests (crates/blocks/tests/support/mod.rs:471-512): `heads`
 * is rows x (heads + 2 kv_heads) x head_dim doubles (already rotated), output rows x
 * heads*head_dim. Mask kinds as above plus 4 = Prefix(window) (support/mod.rs:425-446). */
void oracle_reference_attend_f64(const double* qkv_heads, int64_t rows, int64_t heads,
                                 int64_t kv_heads, int64_t head_dim, const oracle_mask* mask,
                                 double* out);

#ifdef __cplusplus
}
#endif
#endif
