//! fusor-ai's `KvCache` in GPU memory behind the fa_attn C ABI: the owning handle and the status
//! codes as a `Result`. The `Attention` adapter that plugs it into `blocks::transformer` lives in
//! `blocks` itself, since the plugin trait (crates/blocks/src/layer.rs:73-88) is crate-private:
//! a second implementation beside `Cached` whose `attend` calls `fa_attention_host` (or
//! `fa_attention` on device rows) from the team's first thread. Not compiled here: no Rust
//! toolchain.
#![expect(unsafe_code, reason = "owns a handle of the fa_attn C ABI")]

pub mod ffi;

use std::ffi::CStr;

/// A non-zero status of the ABI with `fa_last_error`'s message.
#[derive(Debug)]
pub struct Error {
    pub code: i32,
    pub message: String,
}

/// FA_ERR_CAPACITY: the reference's "the cache holds every key the span sees" panic
/// (crates/blocks/src/transformer.rs:335-338).
pub const ERR_CAPACITY: i32 = 3;

pub fn check(status: i32) -> Result<(), Error> {
    if status == 0 {
        return Ok(());
    }
    // SAFETY: fa_last_error returns this thread's NUL-terminated message, valid until the next
    // call into the library on this thread.
    let message = unsafe { CStr::from_ptr(ffi::fa_last_error()) }.to_string_lossy().into_owned();
    Err(Error { code: status, message })
}

/// `KvCache::new(Shape, capacity)` (transformer.rs:148-151) on `device`: keys and values in HBM as
/// `[layer][kv_head][slot][head_dim]`, f32 (`dtype` 0) or bf16 (1).
pub struct CudaKvCache {
    raw: *mut ffi::FaKvCache,
}

impl CudaKvCache {
    pub fn new(layers: i32, heads: i32, kv_heads: i32, head_dim: i32, capacity: i32, dtype: i32,
               device: i32) -> Result<Self, Error> {
        let mut raw = std::ptr::null_mut();
        // SAFETY: `raw` is a valid out-pointer; the library owns what it points to after.
        check(unsafe { ffi::fa_kvcache_create(layers, heads, kv_heads, head_dim, capacity, dtype,
                                              device, &mut raw) })?;
        Ok(Self { raw })
    }

    pub fn raw(&self) -> *mut ffi::FaKvCache {
        self.raw
    }
}

impl Drop for CudaKvCache {
    fn drop(&mut self) {
        // SAFETY: made by fa_kvcache_create and released once.
        unsafe { ffi::fa_kvcache_destroy(self.raw) };
    }
}

// The handle may move between threads; the library serializes what it shares per device.
unsafe impl Send for CudaKvCache {}
