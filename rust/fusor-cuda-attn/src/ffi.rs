//! The C ABI of the B200 attention kernels (`include/fa_attn.h`), as fusor-ai binds it.
//!
//! One `#[repr(C)]` struct per struct of the header, fields in the header's order, and one
//! declaration per entry point with the header's parameters; `tests/test_abi.py` checks both
//! against the header. Written to fusor-ai's conventions (its sanctioned unsafe modules carry an
//! `expect(unsafe_code)` with a reason) but not compiled in this repository: no Rust toolchain.
#![expect(unsafe_code, reason = "the C ABI of the B200 attention kernels")]
use std::ffi::{c_char, c_void};

#[repr(C)] pub struct FaMask { pub kind: i32, pub window: i32, pub state: i32, pub n_ends: i32, pub ends: *const i32 }
#[repr(C)] pub struct FaSpan { pub rows: i32, pub first: i32, pub mask: FaMask }
#[repr(C)] pub struct FaPosition { pub temporal: i32, pub height: i32, pub width: i32 }
#[repr(C)] pub struct FaRotation { pub kind: i32, pub params: [i32; 3], pub base: f32, pub spatial_scale: f32 }
#[repr(C)] pub struct FaHeadNorm { pub q_norm: *const f32, pub k_norm: *const f32, pub eps: f32 }
#[repr(C)] pub struct FaOperand { pub values: *const c_void, pub stride: i64, pub offset: i64 }
#[repr(C)] pub struct FaCall { pub heads: i32, pub kv_heads: i32, pub head_dim: i32, pub images: i32,
                              pub queries: i32, pub keys: i32, pub query: FaOperand, pub key: FaOperand,
                              pub value: FaOperand, pub dtype: i32, pub out_dtype: i32 }
#[repr(C)] pub struct FaLinear { pub weight: *const f32, pub weight_stride: i64, pub bias: *const f32, pub inputs: i32, pub outputs: i32 }
#[repr(C)] pub struct FaIpcHandle { pub bytes: [u8; 64] }
#[repr(C)] pub struct FaRelposCall { pub heads: i32, pub head_dim: i32, pub frames: i32, pub query: FaOperand,
                                    pub key: FaOperand, pub value: FaOperand, pub positions: *const f32,
                                    pub positions_stride: i64, pub bias_u: *const f32, pub bias_v: *const f32 }
#[repr(C)] pub struct FaPrologue { pub tokens: i32, pub heads: i32, pub head_dim: i32, pub norm: i32,
                                  pub q_norm: *const f32, pub k_norm: *const f32, pub eps: f32, pub rope: i32,
                                  pub angles: *const f32, pub rotated_rows: i32 }
#[repr(C)] pub struct FaKvCache { _private: [u8; 0] }

#[link(name = "fa_attn")]
unsafe extern "C" {
    // status, limits, the cache
    pub fn fa_last_error() -> *const c_char;
    pub fn fa_capabilities(flags: *mut i32, head_dims: *mut i32, max_head_dims: i32,
                           n_head_dims: *mut i32) -> i32;
    pub fn fa_device_status(stream: *mut c_void) -> i32;
    pub fn fa_kvcache_create(layers: i32, heads: i32, kv_heads: i32, head_dim: i32,
                             capacity: i32, dtype: i32, device: i32, out: *mut *mut FaKvCache) -> i32;
    pub fn fa_kvcache_destroy(cache: *mut FaKvCache) -> i32;
    pub fn fa_kvcache_data(cache: *const FaKvCache, keys: *mut *mut c_void, values: *mut *mut c_void,
                           shape5: *mut i32, dtype: *mut i32) -> i32;
    pub fn fa_kvcache_reserve(cache: *mut FaKvCache, rows: i32) -> i32;
    pub fn fa_kvcache_copy_rows(cache: *const FaKvCache, rows: i32, keys: *mut c_void,
                                values: *mut c_void, stream: *mut c_void) -> i32;
    pub fn fa_kvcache_put_rows(cache: *mut FaKvCache, rows: i32, keys: *const c_void,
                               values: *const c_void, stream: *mut c_void) -> i32;
    pub fn fa_rotary_angles(rotation: *const FaRotation, head_dim: i32,
                            positions: *const FaPosition, rows: i32, angles: *mut f32) -> i32;
    pub fn fa_rng_fill_normal(seed: u64, out: *mut f32, n: i64) -> i32;

    // the attention input: RoPE (+ head norm) + keep, optionally with the qkv projection
    pub fn fa_attention_input(cache: *mut FaKvCache, layer: i32, span: *const FaSpan, rope: i32,
                              angles: *const f32, norm: *const FaHeadNorm, qkv: *const f32,
                              qkv_stride: i64, q_out: *mut f32, stream: *mut c_void) -> i32;
    pub fn fa_attention_input_batch(caches: *const *mut FaKvCache, spans: *const FaSpan, batch: i32,
                                    layer: i32, rope: i32, angles: *const f32, norm: *const FaHeadNorm,
                                    qkv: *const f32, qkv_stride: i64, q_out: *mut f32,
                                    q_out_stride: i64, stream: *mut c_void) -> i32;
    pub fn fa_attention_input_projected(cache: *mut FaKvCache, layer: i32, span: *const FaSpan,
                                        rope: i32, angles: *const f32, norm: *const FaHeadNorm,
                                        qkv: *const FaLinear, x: *const f32, x_stride: i64,
                                        q_out: *mut f32, qkv_out: *mut f32, qkv_out_stride: i64,
                                        stream: *mut c_void) -> i32;
    pub fn fa_attention_input_projected_batch(caches: *const *mut FaKvCache, spans: *const FaSpan,
                                              batch: i32, layer: i32, rope: i32, angles: *const f32,
                                              norm: *const FaHeadNorm, qkv: *const FaLinear,
                                              x: *const f32, x_stride: i64, q_out: *mut f32,
                                              q_out_stride: i64, stream: *mut c_void) -> i32;
    pub fn fa_rotate_queries(heads: i32, head_dim: i32, rows: i32, rope: i32, angles: *const f32,
                             norm: *const FaHeadNorm, qkv: *const f32, qkv_stride: i64,
                             q_out: *mut f32, q_out_stride: i64, stream: *mut c_void) -> i32;

    // attention over a cache
    pub fn fa_attend(cache: *mut FaKvCache, layer: i32, span: *const FaSpan, q: *const f32,
                     q_stride: i64, out: *mut f32, out_stride: i64, stream: *mut c_void) -> i32;
    pub fn fa_attend_static(cache: *mut FaKvCache, layer: i32, span: *const FaSpan, q: *const f32,
                            q_stride: i64, out: *mut f32, out_stride: i64, stream: *mut c_void) -> i32;
    pub fn fa_attend_batch(caches: *const *mut FaKvCache, spans: *const FaSpan, batch: i32, layer: i32,
                           q: *const f32, q_stride: i64, out: *mut f32, out_stride: i64,
                           stream: *mut c_void) -> i32;
    pub fn fa_attention(cache: *mut FaKvCache, layer: i32, span: *const FaSpan, rope: i32,
                        angles: *const f32, norm: *const FaHeadNorm, qkv: *const f32, qkv_stride: i64,
                        out: *mut f32, out_stride: i64, stream: *mut c_void) -> i32;
    pub fn fa_attention_host(cache: *mut FaKvCache, layer: i32, span: *const FaSpan, rope: i32,
                             angles: *const f32, norm: *const FaHeadNorm, qkv: *const f32,
                             qkv_stride: i64, out: *mut f32, out_stride: i64,
                             stream: *mut c_void) -> i32;
    pub fn fa_attention_batch(caches: *const *mut FaKvCache, spans: *const FaSpan, batch: i32,
                              layer: i32, rope: i32, angles: *const f32, norm: *const FaHeadNorm,
                              qkv: *const f32, qkv_stride: i64, out: *mut f32, out_stride: i64,
                              stream: *mut c_void) -> i32;
    pub fn fa_attention_batch_host(caches: *const *mut FaKvCache, spans: *const FaSpan,
                                   batch: i32, layer: i32, rope: i32, angles: *const f32,
                                   norm: *const FaHeadNorm, qkv: *const f32, qkv_stride: i64,
                                   out: *mut f32, out_stride: i64, stream: *mut c_void) -> i32;
    pub fn fa_gated_attention(cache: *mut FaKvCache, layer: i32, span: *const FaSpan, gate: i32,
                              rotary_dim: i32, angles: *const f32, norm: *const FaHeadNorm,
                              qkv: *const f32, qkv_stride: i64, out: *mut f32, out_stride: i64,
                              stream: *mut c_void) -> i32;

    // a key range's partials, their merge, and the exchange over peer memory
    pub fn fa_attend_partial(cache: *mut FaKvCache, layer: i32, q: *const f32, key_begin: i32,
                             key_end: i32, partials: *mut f32, stream: *mut c_void) -> i32;
    pub fn fa_merge_partials(partials: *const f32, shards: i32, heads: i32, head_dim: i32,
                             out: *mut f32, stream: *mut c_void) -> i32;
    pub fn fa_peer_buffer_bytes(world: i32, heads: i32, head_dim: i32, bytes: *mut u64) -> i32;
    pub fn fa_peer_alloc(bytes: u64, ptr: *mut *mut c_void, handle: *mut FaIpcHandle) -> i32;
    pub fn fa_peer_open(handle: *const FaIpcHandle, ptr: *mut *mut c_void) -> i32;
    pub fn fa_peer_close(ptr: *mut c_void) -> i32;
    pub fn fa_peer_free(ptr: *mut c_void) -> i32;
    pub fn fa_exchange_merge(buffers: *const *mut c_void, buffer_bytes: u64, rank: i32, world: i32,
                             heads: i32, head_dim: i32, partials: *const f32, out: *mut f32,
                             stream: *mut c_void) -> i32;
    pub fn fa_peer_reset(own_buffer: *mut c_void, buffer_bytes: u64, stream: *mut c_void) -> i32;

    // full-mask attention (DiT, conformer) and its prologue
    pub fn fa_attend_full(call: *const FaCall, out: *mut c_void, out_stride: i64,
                          stream: *mut c_void) -> i32;
    pub fn fa_attend_relpos(call: *const FaRelposCall, out: *mut f32, out_stride: i64,
                            stream: *mut c_void) -> i32;
    pub fn fa_normalize_and_rotate(prologue: *const FaPrologue, qkv: *const f32, qkv_stride: i64,
                                   out: *mut c_void, out_stride: i64, out_dtype: i32,
                                   stream: *mut c_void) -> i32;
}
