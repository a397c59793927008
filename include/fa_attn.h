/*
 * fa_attn.h -- the C ABI of the B200 attention hot path of fusor-ai.
 *
 * It replaces the attention phase of blocks::transformer::Transformer::forward over a KvCache
 * (RoPE + keep + grouped-query attention; decode and prefill under every Mask) and the
 * full-mask attention of blocks::attention::attend / dit::Within. Every entry point cites the
 * fusor-ai interface it replaces (paths relative to the fusor-ai project root).
 *
 * Conventions
 *  - Plain C: pointers, sizes and status codes; no panics or aborts cross the boundary. Every
 *    function returns FA_OK (0) or an FA_ERR_* code; fa_last_error() describes the last failure
 *    of the calling thread.
 *  - Device pointers unless a name or comment says "host". `stream` is a cudaStream_t (NULL is
 *    the legacy default stream). Work is enqueued on `stream` and not waited for, except by the
 *    *_host entry points, which return when their host outputs are written.
 *  - Tensors are row-major with explicit element strides, as the reference's SharedBuf rows.
 *  - A KvCache is used from one stream at a time, as the reference uses one from one team run.
 */
#ifndef FA_ATTN_H
#define FA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define FA_OK 0
#define FA_ERR_ARG 1         /* a null pointer, a negative size, a bad enum value */
#define FA_ERR_SHAPE 2       /* heads % kv_heads != 0 (transformer.rs:389-393), a layer or row
                                count beyond what the cache or call holds (layer.rs:124-125) */
#define FA_ERR_CAPACITY 3    /* the span does not fit the cache (transformer.rs:331-338) */
#define FA_ERR_CUDA 4        /* a CUDA runtime error (allocation, launch) */
#define FA_ERR_TIMEOUT 5     /* a device-side wait gave up (see fa_device_status) */
#define FA_ERR_UNSUPPORTED 6 /* a head_dim or dtype this build has no kernel for */

/* Element types of the cache and of full-mask operands. */
#define FA_F32 0
#define FA_BF16 1

/* transformer::Mask (crates/blocks/src/transformer.rs:97-111). */
#define FA_MASK_CAUSAL 0
#define FA_MASK_WINDOW 1
#define FA_MASK_FULL 2
#define FA_MASK_GROUPS 3

/* Rotary pairing of the layer spec (crates/blocks/src/layer/spec.rs Rope; ops.rs:77-95). */
#define FA_ROPE_NONE 0
#define FA_ROPE_HALF 1
#define FA_ROPE_INTERLEAVED 2

/* rotary::Rotation (crates/blocks/src/rotary.rs:62-86). */
#define FA_ROT_SEQUENCE 0
#define FA_ROT_LINEAR 1
#define FA_ROT_PARTIAL 2
#define FA_ROT_MULTIMODAL 3
#define FA_ROT_AXES 4
#define FA_ROT_MULTIMODAL_INTERLEAVED 5
#define FA_ROT_GRID 6

/* Mask (transformer.rs:99-111). `ends` is a HOST array of n_ends group ends (Groups only). */
typedef struct {
  int32_t kind;
  int32_t window;
  int32_t state;
  int32_t n_ends;
  const int32_t* ends;
} fa_mask;

/* Span (transformer.rs:272-279): `rows` consecutive positions from `first` under `mask`. */
typedef struct {
  int32_t rows;
  int32_t first;
  fa_mask mask;
} fa_span;

/* rotary::Position (rotary.rs:27-33). */
typedef struct {
  int32_t temporal;
  int32_t height;
  int32_t width;
} fa_position;

/* A Rotary's configuration: Rotary::new(rotation, base, head_dim) (rotary.rs:117-156), with
 * params = the factor (Linear), the turning count (Partial) or the three sections; and
 * spatially_scaled(spatial_scale) (rotary.rs:161-168; 1 leaves it as it is). */
typedef struct {
  int32_t kind;
  int32_t params[3];
  float base;
  float spatial_scale;
} fa_rotation;

/* Optional Qwen3 head norms (layer.rs:220-228): device weight vectors of head_dim, or NULL. */
typedef struct {
  const float* q_norm;
  const float* k_norm;
  float eps;
} fa_head_norm;

/* blocks::attention::Operand (crates/blocks/src/attention.rs:24-31): head h of row r is the
 * head_dim values at values + r * stride + offset + h * head_dim (elements of the call dtype). */
typedef struct {
  const void* values;
  int64_t stride;
  int64_t offset;
} fa_operand;

/* blocks::attention::Call (attention.rs:33-47) without the int8 Exponentials choice: `images`
 * images of `queries` query rows over `keys` key/value rows; query row of image i is
 * i * queries + q, key row i * keys + k. `dtype` is the operands' element type (FA_F32 or
 * FA_BF16); `out_dtype` the output's. */
typedef struct {
  int32_t heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t images;
  int32_t queries;
  int32_t keys;
  fa_operand query;
  fa_operand key;
  fa_operand value;
  int32_t dtype;
  int32_t out_dtype;
} fa_call;

typedef struct fa_kvcache fa_kvcache;

/* The message of the calling thread's last failure ("" if none). */
const char* fa_last_error(void);

/* The build's capabilities: a bitmask of 1 = f32 cache, 2 = bf16 cache, 4 = tcgen05 prefill /
 * full-mask kernels, 8 = head dims between the powers of two; and the head_dim values with a
 * kernel of their own through *head_dims (may be NULL). With flag 8, a head_dim between 32 and
 * 256 that is a multiple of 4 (f32 rows) or 8 (bf16 rows) runs on the kernel of the next power
 * of two, the lanes past the head idle (Kronos' 52, Iris' 80); the tensor-core kernels take
 * 64 and 128, and 256 over bf16. */
int fa_capabilities(int32_t* flags, int32_t* head_dims, int32_t max_head_dims,
                    int32_t* n_head_dims);

/* KvCache::new(shape, capacity) / KvCache::of (transformer.rs:148-162): a zeroed cache of
 * layers x kv_heads x capacity x head_dim keys and as many values, in HBM on `device`, in the
 * reference's layout [layer][kv_head][slot = position % capacity][head_dim]. `heads` is the
 * query head count (a multiple of kv_heads). dtype FA_F32 (the reference's) or FA_BF16. */
int fa_kvcache_create(int32_t layers, int32_t heads, int32_t kv_heads, int32_t head_dim,
                      int32_t capacity, int32_t dtype, int32_t device, fa_kvcache** out);
int fa_kvcache_destroy(fa_kvcache* cache);

/* The cache's device arrays and shape, for callers that fill or read it directly. */
int fa_kvcache_data(const fa_kvcache* cache, void** keys, void** values, int32_t* shape5,
                    int32_t* dtype);

/* Reserves the per-call workspace for spans of up to `rows` rows (otherwise it grows on the
 * first call that needs more, which synchronizes the stream; do this before graph capture). */
int fa_kvcache_reserve(fa_kvcache* cache, int32_t rows);

/* KvCache::copy_rows (transformer.rs:221-239): the first `rows` rows of every (layer, kv head)
 * block, keys then values, into device buffers of layers*kv_heads*rows*head_dim elements each,
 * in block order. */
int fa_kvcache_copy_rows(const fa_kvcache* cache, int32_t rows, void* keys_out,
                         void* values_out, void* stream);
/* KvCache::put_rows (transformer.rs:241-251): puts back what fa_kvcache_copy_rows copied. */
int fa_kvcache_put_rows(fa_kvcache* cache, int32_t rows, const void* keys, const void* values,
                        void* stream);

/* Rotary::angles for `rows` positions (rotary.rs:170-178 via Stack::turn, layer.rs:140-154),
 * on the HOST, bit for bit the reference's f32 arithmetic: per row head_dim/2 cosines then
 * head_dim/2 sines (the layout of Buffers.angles, layer/buffers.rs:17-18). */
int fa_rotary_angles(const fa_rotation* rotation, int32_t head_dim, const fa_position* positions,
                     int32_t rows, float* angles_out);

/* The attention input of Stack::attention_input (layer.rs:175-234) after the QKV projection:
 * for each of span->rows rows of `qkv` (f32, qkv_stride elements apart; query heads, key
 * heads, value heads of head_dim each), head-norm (optional) and RoPE (`rope`, by `angles`:
 * rows x head_dim as fa_rotary_angles writes them; NULL when rope is FA_ROPE_NONE) the query
 * and key heads, and keep the key and value heads at position first + row (KvCache::keep,
 * transformer.rs:164-180). The rotated queries are written to q_out (rows x heads x head_dim
 * f32) when it is not NULL; qkv is not modified. */
int fa_attention_input(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t rope,
                       const float* angles, const fa_head_norm* norm, const float* qkv,
                       int64_t qkv_stride, float* q_out, void* stream);

/* The layer's qkv Linear (crates/kernels/src/linear.rs: the matrix, outputs x inputs, and the
 * optional bias) with f32 weights, on the device. */
typedef struct fa_linear {
  const float* weight;   /* output c's inputs at weight + c * weight_stride */
  int64_t weight_stride; /* elements, >= inputs; a multiple of 4 */
  const float* bias;     /* outputs values, or NULL */
  int32_t inputs;        /* the hidden width, a multiple of 4 */
  int32_t outputs;       /* (heads + 2 kv_heads) x head_dim */
} fa_linear;

/* The whole of Stack::attention_input (layer.rs:175-209) on the device: the qkv projection
 * (project_quads, linear.rs:52-71: qkv = x . W^T + b for f32 weights) of each of span->rows rows
 * of x (f32, x_stride elements apart, 16-byte aligned), fused in one kernel with what
 * fa_attention_input does after it: head norm, RoPE of the query and key heads, keep of the key
 * and value heads at position first + row, the rotated queries into q_out (rows x heads x
 * head_dim f32; may be NULL). The projected rows themselves (before head norm and RoPE) go to
 * qkv_out (qkv_out_stride apart) when it is not NULL. Sums in f32, in another order than the
 * reference's quad kernels (within float rounding of them). */
int fa_attention_input_projected(fa_kvcache* cache, int32_t layer, const fa_span* span,
                                 int32_t rope, const float* angles, const fa_head_norm* norm,
                                 const fa_linear* qkv, const float* x, int64_t x_stride,
                                 float* q_out, float* qkv_out, int64_t qkv_out_stride,
                                 void* stream);

/* The same for one decode row of each of `batch` sequences (their own caches, as in
 * fa_attention_input_batch): x row i is sequence i's input, kept at spans[i].first; the rotated
 * queries into q_out (batch rows, q_out_stride apart; may be NULL). */
int fa_attention_input_projected_batch(fa_kvcache* const* caches, const fa_span* spans,
                                       int32_t batch, int32_t layer, int32_t rope,
                                       const float* angles, const fa_head_norm* norm,
                                       const fa_linear* qkv, const float* x, int64_t x_stride,
                                       float* q_out, int64_t q_out_stride, void* stream);

/* The query half of fa_attention_input without a cache: head-norm (optional) and RoPE of the
 * `heads` query heads of each row of qkv into q_out (rows x q_out_stride f32). The ranks of a
 * KV-range-sharded decode that do not hold the new position rotate the query with this. */
int fa_rotate_queries(int32_t heads, int32_t head_dim, int32_t rows, int32_t rope,
                      const float* angles, const fa_head_norm* norm, const float* qkv,
                      int64_t qkv_stride, float* q_out, int64_t q_out_stride, void* stream);

/* KvCache::attend (transformer.rs:182-219): the span's rows' rotated queries (q: rows x
 * q_stride f32, heads x head_dim each) attend over the cache under span->mask into out (rows x
 * out_stride f32, heads x head_dim each), scores scaled by 1/sqrt(head_dim). */
int fa_attend(fa_kvcache* cache, int32_t layer, const fa_span* span, const float* q,
              int64_t q_stride, float* out, int64_t out_stride, void* stream);

/* The whole attention phase of one layer of Transformer::forward (transformer.rs:294-341 and
 * the Cached attention, 344-380): the capacity rule, then fa_attention_input, then fa_attend.
 * Replaces Cached::keep + Cached::attend behind the layer's Attention plugin (layer.rs:73-88). */
int fa_attention(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t rope,
                 const float* angles, const fa_head_norm* norm, const float* qkv,
                 int64_t qkv_stride, float* out, int64_t out_stride, void* stream);

/* fa_attention with HOST qkv, angles and out (the reference's Buffers live in host memory,
 * layer/buffers.rs:10-29): copies the rows in, runs, copies the output back and returns when
 * `out` holds it. */
int fa_attention_host(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t rope,
                      const float* angles_host, const fa_head_norm* norm, const float* qkv_host,
                      int64_t qkv_stride, float* out_host, int64_t out_stride, void* stream);

/* One decode step (Span rows = 1) of `batch` independent sequences, each with its own cache
 * (all of one shape and device), in one launch: sequence i's row is row i of qkv (qkv_stride
 * apart) at spans[i].first under spans[i].mask (any kind; a Groups mask's last end is the row's
 * position + 1), angles row i (device, batch x head_dim; NULL for FA_ROPE_NONE), output row i
 * of out. The reference runs one Transformer::forward per sequence
 * (models/ming/model/src/session.rs:268-282); batch <= 1024. */
int fa_attention_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                       int32_t layer, int32_t rope, const float* angles,
                       const fa_head_norm* norm, const float* qkv, int64_t qkv_stride,
                       float* out, int64_t out_stride, void* stream);

/* fa_attention_batch with HOST qkv, angles and out (the batched form of fa_attention_host):
 * returns when `out` holds every sequence's row. A batch of 16 or more runs as two groups of
 * consecutive sequences (the first a quarter of the keys), each its own launch: the second
 * group's rows are copied in on a copy stream while the first group attends, and the second
 * group runs on a second stream, concurrent with the first. A pinned output is stored into by
 * the kernels directly (mapped host memory); a pageable one is copied out per group. Pinned
 * host memory lets the copies overlap; pageable memory still works. The device staging, the
 * copy stream and the second stream belong to the batch's first cache: two calls whose first
 * caches are the same run one after the other, not from two host threads at once. */
int fa_attention_batch_host(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                            int32_t layer, int32_t rope, const float* angles_host,
                            const fa_head_norm* norm, const float* qkv_host, int64_t qkv_stride,
                            float* out_host, int64_t out_stride, void* stream);

/* fa_attention_batch's first half: RoPE + keep of each sequence's row into its own cache, the
 * rotated queries into q_out (batch rows, q_out_stride apart; may be NULL). */
int fa_attention_input_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                             int32_t layer, int32_t rope, const float* angles,
                             const fa_head_norm* norm, const float* qkv, int64_t qkv_stride,
                             float* q_out, int64_t q_out_stride, void* stream);

/* fa_attention_batch's second half: KvCache::attend of each sequence's rotated query row (q,
 * q_stride apart) over its own cache, all sequences in one launch. */
int fa_attend_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                    int32_t layer, const float* q, int64_t q_stride, float* out,
                    int64_t out_stride, void* stream);

/* One KV-range shard of a decode (split-KV across GPUs; the reference has no counterpart, it is
 * the sharded form of ops::attend over keys key_begin..key_end, ops.rs:310-342): the rotated
 * query row q (heads x head_dim f32) over cache positions [key_begin, key_end) of `layer`,
 * all visible, into partials: per head [max, sum, o[head_dim]] with max the largest score in
 * base-2 units (score * log2(e) / sqrt(head_dim)), sum = sum of 2^(score - max) and o the
 * unnormalised sum of 2^(score - max) * value; heads x (head_dim + 2) f32. An empty range
 * gives max = -inf, sum = 0, o = 0. */
int fa_attend_partial(fa_kvcache* cache, int32_t layer, const float* q, int32_t key_begin,
                      int32_t key_end, float* partials, void* stream);

/* The log-sum-exp merge of `shards` partials (shards x heads x (head_dim + 2) f32, as
 * fa_attend_partial writes them) into out (heads x head_dim f32). */
int fa_merge_partials(const float* partials, int32_t shards, int32_t heads, int32_t head_dim,
                      float* out, void* stream);

/* The exchange of a KV-range-sharded decode over NVLink peer memory (one process per GPU of a
 * box), in place of an all-gather of the partials and fa_merge_partials. Each rank allocates one
 * exchange buffer of fa_peer_buffer_bytes (fa_peer_alloc: zeroed, with its CUDA IPC handle),
 * the ranks swap the handles (any host channel: a process group's all-gather of objects), and
 * each maps the others' (fa_peer_open). fa_exchange_merge then stores this rank's partials in
 * every rank's buffer, each value a 64-bit word stamped with the step, waits until every rank's
 * words of the step are in its own (bounded: FA_ERR_TIMEOUT from fa_device_status after about a
 * second, the late rank left out of the merge), and merges into out (heads x head_dim f32) with
 * fa_merge_partials' arithmetic. Every rank calls it once per step, in the same order; the step
 * count lives in the buffer, so a CUDA graph of the step can be replayed. */
typedef struct fa_ipc_handle {
  unsigned char bytes[64];
} fa_ipc_handle;
int fa_peer_buffer_bytes(int32_t world, int32_t heads, int32_t head_dim, uint64_t* bytes);  /* heads <= 64 */
int fa_peer_alloc(uint64_t bytes, void** ptr, fa_ipc_handle* handle);
int fa_peer_open(const fa_ipc_handle* handle, void** ptr);
int fa_peer_close(void* ptr); /* a mapping made by fa_peer_open */
int fa_peer_free(void* ptr);  /* a buffer made by fa_peer_alloc */
/* buffers: world pointers, this rank's own at [rank] and the mappings of the others'; every
 * buffer of buffer_bytes. partials: this rank's heads x (head_dim + 2) f32 (fa_attend_partial). */
int fa_exchange_merge(void* const* buffers, uint64_t buffer_bytes, int32_t rank, int32_t world,
                      int32_t heads, int32_t head_dim, const float* partials, float* out,
                      void* stream);
/* After an exchange that gave up on a rank (FA_ERR_TIMEOUT), the ranks' step counters differ and
 * every later exchange would wait in vain: each rank synchronizes its device, the ranks meet at a
 * barrier, each clears its own buffer (buffer_bytes: its step counter and every stamped word)
 * with fa_peer_reset, which returns once it is clear, and they meet at a second barrier before
 * the next exchange. There is no counterpart in the reference (one process, no exchange); it is
 * this exchange's recovery. */
int fa_peer_reset(void* own_buffer, uint64_t buffer_bytes, void* stream);

/* blocks::attention::attend (attention.rs:79-95) and dit::Within::attend (dit.rs:135-166): full
 * (non-causal) softmax attention of every query over every key of its image, scores scaled by
 * 1/sqrt(head_dim), into out (images*queries rows of out_stride elements, heads x head_dim
 * each, in call->out_dtype). The reference's int8 SageAttention-style approximation is replaced
 * by f32 (FA_F32 operands) or bf16-in / f32-accumulate (FA_BF16) arithmetic.
 * A bf16 call whose (query head, 256-query) units leave the GPU's last wave partly idle runs
 * those units in pieces over key ranges, merged on the device; their partials live in a
 * workspace kept per (device, stream) and grown on demand (the first such call on a stream may
 * allocate device memory: make it before a stream capture). */
int fa_attend_full(const fa_call* call, void* out, int64_t out_stride, void* stream);

/* fa_attend (KvCache::attend) for callers that cannot allocate device memory when they call:
 * a host whose GPU memory is all pre-reserved by its own pool, or a latency-bound decode loop
 * that cannot take cudaMalloc's implicit synchronisation. No counterpart in the reference (its
 * attention scratch is a host Vec per thread). It runs the split-KV kernel with its partials
 * and arrival counters in one 4 MiB device array built into the library (every GPU that loads
 * the library holds it until exit) and calls no allocator: spans whose split needs more
 * scratch than that are rejected with FA_ERR_ARG. The first call on a device looks up the
 * array's device address (once per device); make that first call before any stream capture.
 * Every call on a device shares that device's array: calls whose kernels overlap on the GPU
 * (on different streams) race, and the caller must serialise them. */
int fa_attend_static(fa_kvcache* cache, int32_t layer, const fa_span* span, const float* q,
                     int64_t q_stride, float* out, int64_t out_stride, void* stream);

/* The conformer's relative-position self-attention (crates/blocks/src/conformer/attention.rs:
 * 25-159, Transformer-XL scores): for head h, query frame i and key frame j,
 * score = ((q_i + u) . k_j + (q_i + v) . r_{frames-1-i+j}) / sqrt(head_dim), softmax over every
 * key, times v_j. q, k, v: f32 operands (head h of row i at values + i*stride + offset +
 * h*head_dim); positions: the projected relative-position table, 2*frames - 1 rows
 * positions_stride apart (row frames - 1 - i + j pairs query i with key j; head h at
 * h*head_dim); bias_u, bias_v: heads*head_dim each; head_dim 32, 64, 128 or 256. */
typedef struct {
  int32_t heads;
  int32_t head_dim;
  int32_t frames;
  fa_operand query;
  fa_operand key;
  fa_operand value;
  const float* positions;
  int64_t positions_stride;
  const float* bias_u;
  const float* bias_v;
} fa_relpos_call;

int fa_attend_relpos(const fa_relpos_call* call, float* out, int64_t out_stride, void* stream);

/* Row norms of the query/key prologue. */
#define FA_NORM_NONE 0
#define FA_NORM_ROW 1  /* RMSNorm of the whole query (key) row: heads*head_dim weights */
#define FA_NORM_HEAD 2 /* RMSNorm of each head on its own: head_dim weights */

/* The query/key prologue of the DiT blocks' self-attention: Wan's normalize_and_rotate
 * (crates/blocks/src/wan_dit/block.rs:109-140) and Pyramid's (pyramid_jit/block.rs:100-131)
 * with FA_NORM_ROW, MMDiT's head_norms (mmdit/pass.rs:162-192) with FA_NORM_HEAD. */
typedef struct {
  int32_t tokens;
  int32_t heads;        /* query = key = value heads (the full-mask blocks are multi-head) */
  int32_t head_dim;
  int32_t norm;         /* FA_NORM_* */
  const float* q_norm;  /* device weights, as `norm` says (unused for FA_NORM_NONE) */
  const float* k_norm;
  float eps;
  int32_t rope;         /* FA_ROPE_NONE, FA_ROPE_HALF or FA_ROPE_INTERLEAVED (the DiTs') */
  const float* angles;  /* device, tokens x head_dim as fa_rotary_angles writes them */
  int32_t rotated_rows; /* tokens [0, rotated_rows) are rotated, the rest only normalized */
} fa_prologue;

/* Each token's query row and key row of qkv (f32 device rows qkv_stride apart: queries, keys,
 * values of heads*head_dim each) RMS-normalized and rotated, into out (tokens rows out_stride
 * elements apart, laid out as qkv, in out_dtype), the values copied beside them: the operand
 * rows of fa_attend_full. With out == qkv, FA_F32 and out_stride == qkv_stride it works in
 * place and leaves the values where they are, as the reference does. */
int fa_normalize_and_rotate(const fa_prologue* prologue, const float* qkv, int64_t qkv_stride,
                            void* out, int64_t out_stride, int32_t out_dtype, void* stream);

/* The gate of the hybrid blocks' attention output (hybrid/attention.rs:24-33). */
#define FA_GATE_NONE 0
#define FA_GATE_ELEMENTWISE 1 /* a gate head after each query head's block: per element */
#define FA_GATE_HEADWISE 2    /* one gate per query head, after the value heads */

/* The hybrid blocks' gated attention phase (hybrid/attention.rs:153-295, Weights::mix then the
 * gate): each row of qkv (f32, qkv_stride apart) holds the query heads, with FA_GATE_ELEMENTWISE
 * a gate head per query head, the key heads and the value heads (head_dim each), then with
 * FA_GATE_HEADWISE one gate per query head. Query and key heads are head-normed (optional) and
 * rotated by halves in their first rotary_dim elements by `angles` (rows x rotary_dim, as
 * fa_rotary_angles writes them for a rotary of rotary_dim), keys and values kept at first + row,
 * the queries attend over the cache under span->mask, and out (rows x out_stride f32, heads x
 * head_dim) is multiplied by the sigmoid of its gates. */
int fa_gated_attention(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t gate,
                       int32_t rotary_dim, const float* angles, const fa_head_norm* norm,
                       const float* qkv, int64_t qkv_stride, float* out, int64_t out_stride,
                       void* stream);

/* Waits for `stream` and reports whether any kernel of this library gave up a device-side wait
 * since the last call (FA_ERR_TIMEOUT, clearing the flag) or FA_OK. */
int fa_device_status(void* stream);

/* The reference's seeded generator (crates/kernels/src/rng.rs:5-52: xoshiro256** seeded by
 * SplitMix64, normals by Box-Muller), on the HOST: n standard normals into out. */
int fa_rng_fill_normal(uint64_t seed, float* out, int64_t n);

#ifdef __cplusplus
}
#endif
#endif /* FA_ATTN_H */
