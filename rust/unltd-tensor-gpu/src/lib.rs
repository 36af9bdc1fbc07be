//! B200 (sm_100a) drop-in for the quantized matvec operators of the
//! reference crate `unltd-tensor`, over the C ABI of `libunltd_gpu.so`
//! (`include/unltd_gpu.h`).
//!
//! Two layers, as in the header:
//!
//! * the reference's own signatures on host slices: [`gemv_quant`]
//!   (crates/unltd-tensor/src/quants.rs:422), [`gemv_quant_q8k`]
//!   (quants.rs:474) and [`dequantize_q4_k`] (quants.rs:534). They panic on
//!   the same conditions the CPU functions `assert!` on (quants.rs:430-452,
//!   482-505), with the library's message. Weights are uploaded on first use
//!   and cached by (address, length, dtype, shape), so a caller holding mmap
//!   views keeps its call sites; call [`forget_weights`] before unmapping.
//! * a handle API for callers that keep activations on the GPU: [`Context`]
//!   (device, stream, scratch), [`Weight`] (an uploaded, repacked tensor) and
//!   the asynchronous launches on device pointers.
//!
//! The enum [`DType`] has the ordinals of `unltd_tensor::DType`
//! (crates/unltd-tensor/src/lib.rs:19-31); inside `unltd-tensor` this module
//! would use that enum directly. Re-exported behind a feature flag, the three
//! functions replace the CPU ones without touching qwen35_forward.rs or
//! min_forward.rs:
//!
//! ```ignore
//! #[cfg(feature = "b200")] pub use unltd_tensor_gpu::{gemv_quant, gemv_quant_q8k, dequantize_q4_k};
//! #[cfg(not(feature = "b200"))] pub use quants::{gemv_quant, gemv_quant_q8k, dequantize_q4_k};
//! ```

use std::ffi::CStr;
use std::os::raw::{c_char, c_void};

/// Element types, same ordinals as `unltd_tensor::DType` (lib.rs:19-31).
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
#[repr(i32)]
pub enum DType {
    F32 = 0,
    F16 = 1,
    BF16 = 2,
    I8 = 3,
    U8 = 4,
    Q4K = 5,
    Q6K = 6,
    Q8_0 = 7,
}

/// Arithmetic of a GEMV: `F32x` follows `gemv_quant` (within 1e-4 of the f64
/// dot), `Q8kExact` is bit-identical to `gemv_quant_q8k`.
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
#[repr(i32)]
pub enum Mode {
    F32x = 0,
    Q8kExact = 1,
}

#[repr(C)]
pub struct CtxOpaque {
    _private: [u8; 0],
}
#[repr(C)]
pub struct WeightOpaque {
    _private: [u8; 0],
}

#[link(name = "unltd_gpu")]
extern "C" {
    fn unltd_last_error() -> *const c_char;
    fn unltd_abi_version() -> i32;

    fn unltd_ctx_create(device: i32, out: *mut *mut CtxOpaque) -> i32;
    fn unltd_ctx_destroy(ctx: *mut CtxOpaque) -> i32;
    fn unltd_ctx_set_stream(ctx: *mut CtxOpaque, stream: *mut c_void) -> i32;
    fn unltd_ctx_synchronize(ctx: *mut CtxOpaque) -> i32;

    fn unltd_weight_upload(ctx: *mut CtxOpaque, host_bytes: *const c_void, nbytes: usize, dtype: i32,
                           dim_in: usize, dim_out: usize, out: *mut *mut WeightOpaque) -> i32;
    fn unltd_weight_free(w: *mut WeightOpaque) -> i32;

    fn unltd_gemv(ctx: *mut CtxOpaque, w: *mut WeightOpaque, x_dev: *const f32, y_dev: *mut f32,
                  mode: i32) -> i32;
    fn unltd_gemv_argmax(ctx: *mut CtxOpaque, w: *mut WeightOpaque, x_dev: *const f32, logits_dev: *mut f32,
                         token_dev: *mut u32, mode: i32) -> i32;
    fn unltd_gemv_batch(ctx: *mut CtxOpaque, w: *mut WeightOpaque, x_dev: *const f32, y_dev: *mut f32,
                        n_seq: i32, mode: i32) -> i32;
    fn unltd_gemv_argmax_batch(ctx: *mut CtxOpaque, w: *mut WeightOpaque, x_dev: *const f32, logits_dev: *mut f32,
                               tokens_dev: *mut u32, n_seq: i32, mode: i32) -> i32;
    fn unltd_gemm(ctx: *mut CtxOpaque, w: *mut WeightOpaque, x_dev: *const f32, y_dev: *mut f32,
                  m_tokens: usize) -> i32;
    fn unltd_dequant(ctx: *mut CtxOpaque, w: *mut WeightOpaque, out_dev: *mut f32) -> i32;

    fn unltd_gemv_quant(out: *mut f32, out_len: usize, x: *const f32, x_len: usize, w: *const u8,
                        w_len: usize, dim_in: usize, dim_out: usize, dtype: i32) -> i32;
    fn unltd_gemv_quant_q8k(out: *mut f32, out_len: usize, x: *const f32, x_len: usize, w: *const u8,
                            w_len: usize, dim_in: usize, dim_out: usize, dtype: i32) -> i32;
    fn unltd_dequantize_q4_k(out: *mut f32, out_len: usize, w: *const u8, w_len: usize) -> i32;
    fn unltd_set_default_device(device: i32) -> i32;
    fn unltd_forget_host_weights() -> i32;
}

/// A failed call: the status code of the C ABI and the library's message.
#[derive(Debug, Clone)]
pub struct Error {
    pub status: i32,
    pub message: String,
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "unltd_gpu status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Error {}

fn status(rc: i32) -> Result<(), Error> {
    if rc == 0 {
        return Ok(());
    }
    let p = unsafe { unltd_last_error() };
    let message = if p.is_null() {
        String::new()
    } else {
        unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
    };
    Err(Error { status: rc, message })
}

/// The reference panics where its asserts fail; so do the drop-ins.
fn check(rc: i32, what: &str) {
    if let Err(e) = status(rc) {
        panic!("{what}: {e}");
    }
}

/// ABI version of the loaded library (`UNLTD_ABI_VERSION`).
pub fn abi_version() -> i32 {
    unsafe { unltd_abi_version() }
}

// ---- reference signatures (host slices, synchronous) ------------------------

/// Drop-in for `gemv_quant` (quants.rs:422): `out[j]` = row j of `w` (GGUF
/// bytes, `dim_out` rows of `dim_in` elements) dotted with `x`, within 1e-4
/// (normwise) of the f64 dot the CPU function computes.
pub fn gemv_quant(out: &mut [f32], x: &[f32], w: &[u8], dim_in: usize, dim_out: usize, dtype: DType) {
    let rc = unsafe {
        unltd_gemv_quant(out.as_mut_ptr(), out.len(), x.as_ptr(), x.len(), w.as_ptr(), w.len(), dim_in, dim_out,
                         dtype as i32)
    };
    check(rc, "gemv_quant");
}

/// Drop-in for `gemv_quant_q8k` (quants.rs:474): x quantized to Q8_K, the
/// integer dots and the f32 epilogue of the reference, bit for bit.
pub fn gemv_quant_q8k(out: &mut [f32], x: &[f32], w: &[u8], dim_in: usize, dim_out: usize, dtype: DType) {
    let rc = unsafe {
        unltd_gemv_quant_q8k(out.as_mut_ptr(), out.len(), x.as_ptr(), x.len(), w.as_ptr(), w.len(), dim_in,
                             dim_out, dtype as i32)
    };
    check(rc, "gemv_quant_q8k");
}

/// Drop-in for `dequantize_q4_k` (quants.rs:534), bit-exact.
pub fn dequantize_q4_k(out: &mut [f32], w: &[u8]) {
    let rc = unsafe { unltd_dequantize_q4_k(out.as_mut_ptr(), out.len(), w.as_ptr(), w.len()) };
    check(rc, "dequantize_q4_k");
}

/// Device of the default context behind the three functions above (before
/// their first call; device 0 otherwise).
pub fn set_default_device(device: i32) -> Result<(), Error> {
    status(unsafe { unltd_set_default_device(device) })
}

/// Drops the cached uploads of host weight views (before unmapping them).
pub fn forget_weights() {
    unsafe {
        unltd_forget_host_weights();
    }
}

// ---- handle API (device pointers, asynchronous on the context's stream) -----

/// A device, a stream and the scratch of the launches (`unltd_ctx`).
pub struct Context {
    h: *mut CtxOpaque,
}

impl Context {
    pub fn new(device: i32) -> Result<Self, Error> {
        let mut h = std::ptr::null_mut();
        status(unsafe { unltd_ctx_create(device, &mut h) })?;
        Ok(Context { h })
    }

    /// Launch on `stream` (a `cudaStream_t`); null restores the context's own.
    ///
    /// # Safety
    /// `stream` must be a valid CUDA stream of this context's device.
    pub unsafe fn set_stream(&self, stream: *mut c_void) -> Result<(), Error> {
        status(unltd_ctx_set_stream(self.h, stream))
    }

    /// Waits for the context's stream; reports a kernel's bounded-wait timeout.
    pub fn synchronize(&self) -> Result<(), Error> {
        status(unsafe { unltd_ctx_synchronize(self.h) })
    }

    /// Uploads a packed GGUF view (the `&[u8]` the reference borrows from the
    /// mmap, weights.rs:55-61) once and repacks it on the device.
    pub fn upload(&self, w: &[u8], dtype: DType, dim_in: usize, dim_out: usize) -> Result<Weight<'_>, Error> {
        let mut h = std::ptr::null_mut();
        status(unsafe {
            unltd_weight_upload(self.h, w.as_ptr() as *const c_void, w.len(), dtype as i32, dim_in, dim_out, &mut h)
        })?;
        Ok(Weight { h, _ctx: std::marker::PhantomData })
    }

    /// `y = W . x` on device pointers (`x_dev`: dim_in f32, `y_dev`: dim_out f32).
    ///
    /// # Safety
    /// Both pointers must be device memory of this context's device, of the sizes above.
    pub unsafe fn gemv(&self, w: &Weight<'_>, x_dev: *const f32, y_dev: *mut f32, mode: Mode) -> Result<(), Error> {
        status(unltd_gemv(self.h, w.h, x_dev, y_dev, mode as i32))
    }

    /// LM head with the greedy argmax fused (min_forward.rs:210-266 then
    /// greedy.rs:18-27); `logits_dev` may be null.
    ///
    /// # Safety
    /// Device pointers of this context's device: x dim_in f32, logits dim_out
    /// f32 (or null), token one u32.
    pub unsafe fn gemv_argmax(&self, w: &Weight<'_>, x_dev: *const f32, logits_dev: *mut f32, token_dev: *mut u32,
                              mode: Mode) -> Result<(), Error> {
        status(unltd_gemv_argmax(self.h, w.h, x_dev, logits_dev, token_dev, mode as i32))
    }

    /// Batch decode: `Y[s] = W . X[s]` for `n_seq` (1..32) sequences sharing
    /// W, each row the bits of [`Context::gemv`] in Q8K_EXACT mode on `X[s]`
    /// alone (gemv_quant_q8k per sequence, quants.rs:474-515).
    ///
    /// # Safety
    /// Device pointers of this context's device: X n_seq x dim_in f32,
    /// Y n_seq x dim_out f32.
    pub unsafe fn gemv_batch(&self, w: &Weight<'_>, x_dev: *const f32, y_dev: *mut f32, n_seq: i32)
                             -> Result<(), Error> {
        status(unltd_gemv_batch(self.h, w.h, x_dev, y_dev, n_seq, Mode::Q8kExact as i32))
    }

    /// The LM head of a batch: every sequence's logits (or null) and greedy token.
    ///
    /// # Safety
    /// Device pointers of this context's device: X n_seq x dim_in f32, logits
    /// n_seq x dim_out f32 (or null), tokens n_seq u32.
    pub unsafe fn gemv_argmax_batch(&self, w: &Weight<'_>, x_dev: *const f32, logits_dev: *mut f32,
                                    tokens_dev: *mut u32, n_seq: i32) -> Result<(), Error> {
        status(unltd_gemv_argmax_batch(self.h, w.h, x_dev, logits_dev, tokens_dev, n_seq, Mode::Q8kExact as i32))
    }

    /// Batched prefill `Y = X . W^T` over `m_tokens` rows of X.
    ///
    /// # Safety
    /// Device pointers of this context's device: X m_tokens x dim_in f32,
    /// Y m_tokens x dim_out f32.
    pub unsafe fn gemm(&self, w: &Weight<'_>, x_dev: *const f32, y_dev: *mut f32, m_tokens: usize) -> Result<(), Error> {
        status(unltd_gemm(self.h, w.h, x_dev, y_dev, m_tokens))
    }

    /// All rows dequantized to f32 (bit-exact with the reference's dequant).
    ///
    /// # Safety
    /// `out_dev`: device memory of dim_out x dim_in f32.
    pub unsafe fn dequant(&self, w: &Weight<'_>, out_dev: *mut f32) -> Result<(), Error> {
        status(unltd_dequant(self.h, w.h, out_dev))
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe {
            unltd_ctx_destroy(self.h);
        }
    }
}

/// An uploaded weight tensor; lives no longer than its [`Context`].
pub struct Weight<'c> {
    h: *mut WeightOpaque,
    _ctx: std::marker::PhantomData<&'c Context>,
}

impl Drop for Weight<'_> {
    fn drop(&mut self) {
        unsafe {
            unltd_weight_free(self.h);
        }
    }
}
