//! whisper.rs's attention path on NVIDIA B200 (sm_100a), through libwattn's
//! C ABI (`include/wattn.h`).
//!
//! * [`sys`] declares every entry point of the header, one to one.
//! * The free functions keep the reference signatures of
//!   `whisper_tensor::ops::{flash_attention_2, multi_head_attention,
//!   single_token_mha_d64}` (crates/tensor/src/ops/attention.rs:29-41, 68-78,
//!   246-254) and of the decoder's `multi_head_attention_with_cache` and
//!   `capture_cross_attention_heads` (crates/whisper/src/decoder.rs:835-845,
//!   796-806): host `&[f32]` slices in the reference layout. A non-zero
//!   status panics with the library's message, as the reference's asserts do
//!   (attention.rs:79-88).
//! * [`DeviceKvCache`] mirrors `DecoderKvCache` (decoder.rs:131-264) with
//!   the cache resident on the GPU in pages: the same methods, plus the
//!   per-layer `append` / `attend` of `decode_batch_inner`
//!   (decoder.rs:616-647) and `advance` (:765-767).
//!
//! There is no CPU fallback: head dimensions other than 64 are refused by
//! the library (`WATTN_ERR_UNSUPPORTED`), which panics here.

#![allow(non_camel_case_types)]
#![allow(clippy::too_many_arguments)]

use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};

/// Element types (`WATTN_F32`, `WATTN_F16`, `WATTN_BF16`).
pub const F32: c_int = 0;
pub const F16: c_int = 1;
pub const BF16: c_int = 2;

/// Status codes.
pub const OK: c_int = 0;
pub const ERR_INVALID: c_int = -1;
pub const ERR_UNSUPPORTED: c_int = -2;
pub const ERR_CUDA: c_int = -3;
pub const ERR_TIMEOUT: c_int = -4;
pub const ERR_NOMEM: c_int = -5;
pub const ERR_RANGE: c_int = -6;

/// The C ABI of `include/wattn.h`, declaration for declaration.
pub mod sys {
    use std::os::raw::{c_char, c_int, c_void};

    /// Opaque device-resident paged KV cache (`wattn_kv_cache`).
    #[repr(C)]
    pub struct wattn_kv_cache {
        _private: [u8; 0],
    }

    extern "C" {
        pub fn wattn_version() -> c_int;
        pub fn wattn_status_string(status: c_int) -> *const c_char;
        pub fn wattn_last_error(buf: *mut c_char, len: usize) -> c_int;
        pub fn wattn_device_status(device: c_int, status: *mut c_int) -> c_int;

        pub fn wattn_attention_fwd(q: *const c_void, k: *const c_void, v: *const c_void,
                                   o: *mut c_void, in_dtype: c_int, out_dtype: c_int,
                                   batch: c_int, t_q: c_int, t_kv: c_int, n_heads: c_int,
                                   d_head: c_int, q_row_stride: i64, kv_row_stride: i64,
                                   o_row_stride: i64, q_batch_stride: i64,
                                   kv_batch_stride: i64, o_batch_stride: i64, scale: f32,
                                   causal: c_int, q_pos_offset: c_int,
                                   stream: *mut c_void) -> c_int;

        pub fn wattn_decode_workspace_bytes(n_groups: c_int, group_size: c_int, t_kv: c_int,
                                            n_heads: c_int) -> usize;
        pub fn wattn_decode_fwd(q: *const c_void, k: *const c_void, v: *const c_void,
                                o: *mut c_void, q_dtype: c_int, kv_dtype: c_int,
                                out_dtype: c_int, n_groups: c_int, group_size: c_int,
                                t_kv: c_int, n_heads: c_int, d_head: c_int, q_row_stride: i64,
                                kv_row_stride: i64, kv_group_stride: i64, o_row_stride: i64,
                                scale: f32, workspace: *mut c_void, workspace_bytes: usize,
                                stream: *mut c_void) -> c_int;
        pub fn wattn_decode_fwd_capture(q: *const c_void, k: *const c_void, v: *const c_void,
                                        o: *mut c_void, q_dtype: c_int, kv_dtype: c_int,
                                        out_dtype: c_int, n_groups: c_int, group_size: c_int,
                                        t_kv: c_int, n_heads: c_int, d_head: c_int,
                                        q_row_stride: i64, kv_row_stride: i64,
                                        kv_group_stride: i64, o_row_stride: i64, scale: f32,
                                        workspace: *mut c_void, workspace_bytes: usize,
                                        sel_slot: *const c_int, sel_head: *const c_int,
                                        n_sel: c_int, n_selected: c_int, row_offset: c_int,
                                        capture: *mut f32, stream: *mut c_void) -> c_int;

        pub fn wattn_linear_fwd(x: *const c_void, w: *const c_void, bias: *const f32,
                                y: *mut c_void, in_dtype: c_int, out_dtype: c_int, m: c_int,
                                n: c_int, k: c_int, x_row_stride: i64, w_row_stride: i64,
                                y_row_stride: i64, stream: *mut c_void) -> c_int;
        pub fn wattn_cross_kv_project(enc: *const c_void, wk: *const c_void,
                                      wv: *const c_void, bv: *const f32, k_out: *mut c_void,
                                      v_out: *mut c_void, in_dtype: c_int, out_dtype: c_int,
                                      n_tokens: c_int, d_model: c_int, enc_row_stride: i64,
                                      kv_row_stride: i64, stream: *mut c_void) -> c_int;
        pub fn wattn_encoder_attention_workspace_bytes(batch: c_int, t: c_int,
                                                       n_heads: c_int) -> usize;
        pub fn wattn_encoder_attention(x: *const c_void, w_qkv: *const c_void,
                                       b_qkv: *const f32, w_out: *const c_void,
                                       b_out: *const f32, y: *mut c_void, in_dtype: c_int,
                                       out_dtype: c_int, batch: c_int, t: c_int,
                                       n_heads: c_int, workspace: *mut c_void,
                                       workspace_bytes: usize, stream: *mut c_void) -> c_int;
        pub fn wattn_encoder_attention_residual(x: *mut f32, ln_w: *const f32, ln_b: *const f32,
                                                w_qkv: *const c_void, b_qkv: *const f32,
                                                w_out: *const c_void, b_out: *const f32,
                                                dtype: c_int, batch: c_int, t: c_int,
                                                n_heads: c_int, workspace: *mut c_void,
                                                workspace_bytes: usize,
                                                stream: *mut c_void) -> c_int;

        pub fn wattn_decode_fwd_noalloc(q: *const c_void, k: *const c_void, v: *const c_void,
                                        o: *mut c_void, q_dtype: c_int, kv_dtype: c_int,
                                        out_dtype: c_int, n_groups: c_int, group_size: c_int,
                                        t_kv: c_int, n_heads: c_int, d_head: c_int,
                                        q_row_stride: i64, kv_row_stride: i64,
                                        kv_group_stride: i64, o_row_stride: i64, scale: f32,
                                        stream: *mut c_void) -> c_int;

        pub fn wattn_kv_create(out: *mut *mut wattn_kv_cache, n_layers: c_int, n_slots: c_int,
                               n_heads: c_int, d_head: c_int, max_ctx: c_int, page_rows: c_int,
                               n_pages: c_int, dtype: c_int) -> c_int;
        pub fn wattn_kv_destroy(cache: *mut wattn_kv_cache) -> c_int;
        pub fn wattn_kv_clear(cache: *mut wattn_kv_cache) -> c_int;
        pub fn wattn_kv_clear_slot(cache: *mut wattn_kv_cache, slot: c_int) -> c_int;
        pub fn wattn_kv_ensure_slots(cache: *mut wattn_kv_cache, n_slots: c_int) -> c_int;
        pub fn wattn_kv_copy_slot(cache: *mut wattn_kv_cache, dst: c_int, src: c_int,
                                  stream: *mut c_void) -> c_int;
        pub fn wattn_kv_assign_beams(cache: *mut wattn_kv_cache, parent_slot: *const c_int,
                                     n_branches: c_int, out_slot: *mut c_int) -> c_int;
        pub fn wattn_kv_slot_len(cache: *const wattn_kv_cache, slot: c_int,
                                 len: *mut c_int) -> c_int;
        pub fn wattn_kv_slide_to_fit(cache: *mut wattn_kv_cache, slot: c_int, n_new: c_int,
                                     max_ctx: c_int, pos: *mut c_int) -> c_int;
        pub fn wattn_kv_set_t_past(cache: *mut wattn_kv_cache, slot: c_int,
                                   n_past: c_int) -> c_int;
        pub fn wattn_kv_advance(cache: *mut wattn_kv_cache, slots: *const c_int,
                                n_tokens: *const c_int, n_seqs: c_int) -> c_int;
        pub fn wattn_kv_append(cache: *mut wattn_kv_cache, layer: c_int, slots: *const c_int,
                               n_tokens: *const c_int, n_seqs: c_int, k_rows: *const c_void,
                               v_rows: *const c_void, src_dtype: c_int, row_stride: i64,
                               stream: *mut c_void) -> c_int;
        pub fn wattn_kv_workspace_bytes(cache: *const wattn_kv_cache, n_rows: c_int) -> usize;
        pub fn wattn_kv_attend(cache: *mut wattn_kv_cache, layer: c_int, slots: *const c_int,
                               n_tokens: *const c_int, n_seqs: c_int, q: *const c_void,
                               q_dtype: c_int, q_row_stride: i64, o: *mut c_void,
                               out_dtype: c_int, o_row_stride: i64, scale: f32,
                               workspace: *mut c_void, workspace_bytes: usize,
                               stream: *mut c_void) -> c_int;
        pub fn wattn_kv_read_slot(cache: *mut wattn_kv_cache, layer: c_int, slot: c_int,
                                  which: c_int, out: *mut c_void, out_dtype: c_int,
                                  stream: *mut c_void) -> c_int;
        pub fn wattn_kv_stats(cache: *const wattn_kv_cache, pages_used: *mut c_int,
                              pages_total: *mut c_int) -> c_int;

        pub fn wattn_flash_attention_2(q: *const f32, k: *const f32, v: *const f32, t_q: usize,
                                       t_kv: usize, n_heads: usize, d_model: usize,
                                       causal: c_int, output: *mut f32) -> c_int;
        pub fn wattn_multi_head_attention(q: *const f32, k: *const f32, v: *const f32,
                                          t_q: usize, t_kv: usize, n_heads: usize,
                                          d_model: usize, causal: c_int,
                                          output: *mut f32) -> c_int;
        pub fn wattn_single_token_mha_d64(q: *const f32, k: *const f32, v: *const f32,
                                          t_kv: usize, n_heads: usize, d_model: usize,
                                          output: *mut f32) -> c_int;
        pub fn wattn_multi_head_attention_with_cache(q: *const f32, k: *const f32,
                                                     v: *const f32, n_tokens: usize,
                                                     total_tokens: usize, t_past: usize,
                                                     n_heads: usize, d_model: usize,
                                                     output: *mut f32) -> c_int;
        pub fn wattn_capture_cross_attention_heads(q: *const f32, k: *const f32,
                                                   n_tokens: usize, n_audio: usize,
                                                   n_heads: usize, d_model: usize,
                                                   sel_slot: *const c_int,
                                                   sel_head: *const c_int, n_sel: usize,
                                                   n_selected: usize, row_offset: usize,
                                                   out: *mut f32) -> c_int;
        pub fn wattn_attention_host(q: *const c_void, k: *const c_void, v: *const c_void,
                                    o: *mut c_void, in_dtype: c_int, out_dtype: c_int,
                                    batch: c_int, t_q: c_int, t_kv: c_int, n_heads: c_int,
                                    scale: f32, causal: c_int) -> c_int;
        pub fn wattn_decode_host(q: *const c_void, k: *const c_void, v: *const c_void,
                                 o: *mut c_void, q_dtype: c_int, kv_dtype: c_int,
                                 out_dtype: c_int, n_groups: c_int, group_size: c_int,
                                 t_kv: c_int, n_heads: c_int, scale: f32) -> c_int;

        pub fn wattn_selftest_bounded_wait(limit_us: c_int, stream: *mut c_void) -> c_int;
    }
}

/// The calling thread's last error message from the library.
pub fn last_error() -> String {
    let mut buf = [0 as c_char; 512];
    // SAFETY: the buffer is writable for its whole length; the library
    // NUL-terminates within `len`.
    unsafe {
        sys::wattn_last_error(buf.as_mut_ptr(), buf.len());
        CStr::from_ptr(buf.as_ptr()).to_string_lossy().into_owned()
    }
}

/// Static description of a status code.
pub fn status_string(status: c_int) -> String {
    // SAFETY: the library returns a static NUL-terminated string, never NULL.
    unsafe { CStr::from_ptr(sys::wattn_status_string(status)).to_string_lossy().into_owned() }
}

/// Panics on a non-zero status, with the library's message (the reference
/// asserts on the same argument errors; crates/ffi/src/lib.rs:2353-2375
/// turns such panics into -1 at its C API).
#[track_caller]
fn check(rc: c_int, what: &str) {
    if rc != OK {
        panic!("{what}: {} ({rc}): {}", status_string(rc), last_error());
    }
}

fn to_c(x: usize, what: &str) -> c_int {
    c_int::try_from(x).unwrap_or_else(|_| panic!("{what} = {x} does not fit a C int"))
}

// ------------------------------------------------------------ reference mirrors

/// `whisper_tensor::ops::flash_attention_2` (attention.rs:68-78): same
/// arguments and contract. q `[t_q][d_model]`, k / v `[t_kv][d_model]`,
/// output `[t_q][d_model]` (fully overwritten); head h at columns h*64.
pub fn flash_attention_2(q: &[f32], k: &[f32], v: &[f32], t_q: usize, t_kv: usize,
                         n_heads: usize, d_model: usize, causal: bool, output: &mut [f32]) {
    assert_eq!(q.len(), t_q * d_model, "q.len()");
    assert_eq!(k.len(), t_kv * d_model, "k.len()");
    assert_eq!(v.len(), t_kv * d_model, "v.len()");
    assert_eq!(output.len(), t_q * d_model, "output.len()");
    // SAFETY: the slices hold exactly the sizes the library reads and writes.
    let rc = unsafe {
        sys::wattn_flash_attention_2(q.as_ptr(), k.as_ptr(), v.as_ptr(), t_q, t_kv, n_heads,
                                     d_model, causal as c_int, output.as_mut_ptr())
    };
    check(rc, "flash_attention_2");
}

/// `whisper_tensor::ops::multi_head_attention` (attention.rs:29-41).
pub fn multi_head_attention(q: &[f32], k: &[f32], v: &[f32], t_q: usize, t_kv: usize,
                            n_heads: usize, d_model: usize, causal: bool, output: &mut [f32]) {
    flash_attention_2(q, k, v, t_q, t_kv, n_heads, d_model, causal, output);
}

/// `whisper_tensor::ops::single_token_mha_d64` (attention.rs:246-254): one
/// query row over t_kv keys, scale 1/8.
pub fn single_token_mha_d64(q: &[f32], k: &[f32], v: &[f32], t_kv: usize, n_heads: usize,
                            d_model: usize, output: &mut [f32]) {
    assert_eq!(q.len(), d_model, "q.len()");
    assert!(k.len() >= t_kv * d_model && v.len() >= t_kv * d_model, "k / v too short");
    assert_eq!(output.len(), d_model, "output.len()");
    // SAFETY: sizes checked above.
    let rc = unsafe {
        sys::wattn_single_token_mha_d64(q.as_ptr(), k.as_ptr(), v.as_ptr(), t_kv, n_heads,
                                        d_model, output.as_mut_ptr())
    };
    check(rc, "single_token_mha_d64");
}

/// `multi_head_attention_with_cache` (decoder.rs:835-845): n_tokens queries
/// at positions t_past.. over total_tokens cached rows, causal.
pub fn multi_head_attention_with_cache(q: &[f32], k: &[f32], v: &[f32], n_tokens: usize,
                                       total_tokens: usize, t_past: usize, n_heads: usize,
                                       d_model: usize, output: &mut [f32]) {
    assert_eq!(q.len(), n_tokens * d_model, "q.len()");
    assert!(k.len() >= total_tokens * d_model && v.len() >= total_tokens * d_model,
            "k / v too short");
    assert_eq!(output.len(), n_tokens * d_model, "output.len()");
    // SAFETY: sizes checked above.
    let rc = unsafe {
        sys::wattn_multi_head_attention_with_cache(q.as_ptr(), k.as_ptr(), v.as_ptr(), n_tokens,
                                                   total_tokens, t_past, n_heads, d_model,
                                                   output.as_mut_ptr())
    };
    check(rc, "multi_head_attention_with_cache");
}

/// `capture_cross_attention_heads` (decoder.rs:796-828): for every selected
/// `(slot, head)` and token t, `out[((row_offset + t) * n_selected + slot) *
/// n_audio + j]` = the head's softmax over the n_audio keys. The reference's
/// `scores` scratch is not needed.
pub fn capture_cross_attention_heads(q: &[f32], k: &[f32], n_tokens: usize, n_audio: usize,
                                     n_heads: usize, d_model: usize,
                                     selected: &[(usize, usize)], n_selected: usize,
                                     row_offset: usize, out: &mut [f32]) {
    assert_eq!(q.len(), n_tokens * d_model, "q.len()");
    assert!(k.len() >= n_audio * d_model, "k too short");
    assert!(out.len() >= (row_offset + n_tokens) * n_selected * n_audio, "out too short");
    let slots: Vec<c_int> = selected.iter().map(|&(s, _)| to_c(s, "slot")).collect();
    let heads: Vec<c_int> = selected.iter().map(|&(_, h)| to_c(h, "head")).collect();
    // SAFETY: sizes checked above; the selection arrays have selected.len() entries.
    let rc = unsafe {
        sys::wattn_capture_cross_attention_heads(q.as_ptr(), k.as_ptr(), n_tokens, n_audio,
                                                 n_heads, d_model, slots.as_ptr(),
                                                 heads.as_ptr(), selected.len(), n_selected,
                                                 row_offset, out.as_mut_ptr())
    };
    check(rc, "capture_cross_attention_heads");
}

/// Reads and clears the device status word (`WATTN_ERR_TIMEOUT` after a
/// bounded wait ran out on that device). `device < 0`: the current device.
pub fn device_status(device: i32) -> c_int {
    let mut st: c_int = 0;
    // SAFETY: `st` is a valid out-pointer.
    check(unsafe { sys::wattn_device_status(device, &mut st) }, "device_status");
    st
}

// ------------------------------------------------------------ device KV cache

/// Device-resident `DecoderKvCache` (decoder.rs:131-264): the self-attention
/// K/V of every layer and slot live in a paged pool on the GPU (f16 or bf16
/// rows); forks share pages (copy on write). Method names and meanings are
/// the reference's; `append` / `attend` / `advance` are the per-layer steps
/// of `decode_batch_inner` (decoder.rs:616-647, 765-767) over all slots at
/// once. Device pointers (`*const c_void` / `*mut c_void`) and the stream
/// are the caller's; enqueued work is asynchronous on that stream.
///
/// The reference's `k_cross` / `v_cross` (decoder.rs:137-139) are the caller's
/// device buffers here (written by `wattn_cross_kv_project`, read by
/// `wattn_decode_fwd`); `invalidate_cross` / `cross_ready` keep the
/// reference's "recompute after a new encoder pass" bookkeeping.
pub struct DeviceKvCache {
    raw: *mut sys::wattn_kv_cache,
    n_heads: usize,
    d_model: usize,
    max_ctx: usize,
    cross_ready: bool,
}

// The cache is only touched through &mut self (or &self for read-only
// queries); the library guards nothing else per cache.
unsafe impl Send for DeviceKvCache {}

impl DeviceKvCache {
    /// `DecoderKvCache::new(n_layers, n_slots, d_model)` (decoder.rs:147) for
    /// f16 rows, room for max_ctx positions per slot, 64-row pages, on the
    /// current device.
    pub fn new(n_layers: usize, n_slots: usize, d_model: usize, max_ctx: usize) -> Self {
        Self::with_options(n_layers, n_slots, d_model, max_ctx, 64, 0, F16)
    }

    /// As [`DeviceKvCache::new`] with the page size (a multiple of 64 rows),
    /// the pool size in pages (0: every slot at max_ctx plus one
    /// copy-on-write page per slot) and the row type (F16 or BF16).
    pub fn with_options(n_layers: usize, n_slots: usize, d_model: usize, max_ctx: usize,
                        page_rows: usize, n_pages: usize, dtype: c_int) -> Self {
        assert!(d_model % 64 == 0, "d_model must be n_heads * 64");
        let n_heads = d_model / 64;
        let mut raw = std::ptr::null_mut();
        // SAFETY: `raw` is a valid out-pointer.
        let rc = unsafe {
            sys::wattn_kv_create(&mut raw, to_c(n_layers, "n_layers"), to_c(n_slots, "n_slots"),
                                 to_c(n_heads, "n_heads"), 64, to_c(max_ctx, "max_ctx"),
                                 to_c(page_rows, "page_rows"), to_c(n_pages, "n_pages"), dtype)
        };
        check(rc, "DeviceKvCache::new");
        Self { raw, n_heads, d_model, max_ctx, cross_ready: false }
    }

    pub fn d_model(&self) -> usize {
        self.d_model
    }

    pub fn n_heads(&self) -> usize {
        self.n_heads
    }

    pub fn max_ctx(&self) -> usize {
        self.max_ctx
    }

    /// decoder.rs:161: every slot emptied; the pool is kept.
    pub fn clear(&mut self) {
        // SAFETY: `raw` is a live cache.
        check(unsafe { sys::wattn_kv_clear(self.raw) }, "clear");
    }

    /// decoder.rs:176: one slot emptied, the others untouched.
    pub fn clear_slot(&mut self, slot: usize) {
        // SAFETY: `raw` is a live cache; the library range-checks `slot`.
        check(unsafe { sys::wattn_kv_clear_slot(self.raw, to_c(slot, "slot")) }, "clear_slot");
    }

    /// decoder.rs:192: the cross-attention K/V must be recomputed (a new
    /// encoder pass).
    pub fn invalidate_cross(&mut self) {
        self.cross_ready = false;
    }

    /// Whether the caller's cross-attention K/V are current (set with
    /// [`DeviceKvCache::set_cross_ready`] after `wattn_cross_kv_project`).
    pub fn cross_ready(&self) -> bool {
        self.cross_ready
    }

    pub fn set_cross_ready(&mut self) {
        self.cross_ready = true;
    }

    /// decoder.rs:203: at least n_slots slots; existing slots survive.
    pub fn ensure_slots(&mut self, n_slots: usize) {
        // SAFETY: `raw` is a live cache.
        check(unsafe { sys::wattn_kv_ensure_slots(self.raw, to_c(n_slots, "n_slots")) },
              "ensure_slots");
    }

    /// decoder.rs:220: `dst` takes `src`'s history (pages shared, copied on
    /// the next write to either).
    pub fn copy_slot(&mut self, dst: usize, src: usize, stream: *mut c_void) {
        // SAFETY: `raw` is a live cache; `stream` is the caller's (or null).
        check(unsafe { sys::wattn_kv_copy_slot(self.raw, to_c(dst, "dst"), to_c(src, "src"),
                                               stream) }, "copy_slot");
    }

    /// decoder.rs:237: tokens cached in `slot`.
    pub fn slot_len(&self, slot: usize) -> usize {
        let mut n: c_int = 0;
        // SAFETY: `raw` is a live cache and `n` a valid out-pointer.
        check(unsafe { sys::wattn_kv_slot_len(self.raw, to_c(slot, "slot"), &mut n) },
              "slot_len");
        n as usize
    }

    /// decoder.rs:248: drops the oldest rows so n_new more fit in max_ctx;
    /// returns the position of the first new token.
    pub fn slide_to_fit(&mut self, slot: usize, n_new: usize, max_ctx: usize) -> usize {
        let mut pos: c_int = 0;
        // SAFETY: `raw` is a live cache and `pos` a valid out-pointer.
        check(unsafe { sys::wattn_kv_slide_to_fit(self.raw, to_c(slot, "slot"),
                                                  to_c(n_new, "n_new"),
                                                  to_c(max_ctx, "max_ctx"), &mut pos) },
              "slide_to_fit");
        pos as usize
    }

    /// The C API's rewind (`t_past = n_past`, crates/ffi/src/lib.rs:2352):
    /// rows at or past n_past are dropped by the next append.
    pub fn set_t_past(&mut self, slot: usize, n_past: usize) {
        // SAFETY: `raw` is a live cache.
        check(unsafe { sys::wattn_kv_set_t_past(self.raw, to_c(slot, "slot"),
                                                to_c(n_past, "n_past")) }, "set_t_past");
    }

    /// decoder.rs:765-767: `t_past[slots[i]] += n_tokens[i]` after the last
    /// layer of a step.
    pub fn advance(&mut self, slots: &[i32], n_tokens: &[i32]) {
        assert_eq!(slots.len(), n_tokens.len(), "slots / n_tokens");
        // SAFETY: both arrays hold slots.len() entries.
        check(unsafe { sys::wattn_kv_advance(self.raw, slots.as_ptr(), n_tokens.as_ptr(),
                                             to_c(slots.len(), "n_seqs")) }, "advance");
    }

    /// `BeamSearch::step`'s slot hand-out (crates/whisper/src/beam.rs:418-460)
    /// in one call: `parent_slot[i]` is retained branch i's parent slot; the
    /// returned vector holds each branch's slot (first child keeps the
    /// parent's, further children fork into free slots).
    pub fn assign_beams(&mut self, parent_slot: &[i32]) -> Vec<i32> {
        let mut out = vec![0i32; parent_slot.len()];
        // SAFETY: both arrays hold parent_slot.len() entries.
        check(unsafe { sys::wattn_kv_assign_beams(self.raw, parent_slot.as_ptr(),
                                                  to_c(parent_slot.len(), "n_branches"),
                                                  out.as_mut_ptr()) }, "assign_beams");
        out
    }

    /// decoder.rs:631-635: n_tokens[i] new K/V rows of slots[i] into `layer`
    /// at positions t_past.. (rows packed sequence-major, width d_model, row
    /// stride `row_stride` elements, type `src_dtype`).
    ///
    /// # Safety
    /// `k_rows` / `v_rows` must be device pointers to at least
    /// sum(n_tokens) rows of `row_stride` elements of `src_dtype`.
    pub unsafe fn append(&mut self, layer: usize, slots: &[i32], n_tokens: &[i32],
                         k_rows: *const c_void, v_rows: *const c_void, src_dtype: c_int,
                         row_stride: i64, stream: *mut c_void) {
        assert_eq!(slots.len(), n_tokens.len(), "slots / n_tokens");
        check(sys::wattn_kv_append(self.raw, to_c(layer, "layer"), slots.as_ptr(),
                                   n_tokens.as_ptr(), to_c(slots.len(), "n_seqs"), k_rows, v_rows,
                                   src_dtype, row_stride, stream), "append");
    }

    /// Workspace bytes `attend` needs for n_rows query rows.
    pub fn workspace_bytes(&self, n_rows: usize) -> usize {
        // SAFETY: `raw` is a live cache.
        unsafe { sys::wattn_kv_workspace_bytes(self.raw, to_c(n_rows, "n_rows")) }
    }

    /// `multi_head_attention_with_cache` (decoder.rs:835-892) of the rows
    /// just appended, for every slot of the step at once.
    ///
    /// # Safety
    /// `q` / `o` must be device pointers to sum(n_tokens) rows of their
    /// strides and types; `workspace` null or a zero-filled device buffer of
    /// `workspace_bytes` bytes.
    pub unsafe fn attend(&mut self, layer: usize, slots: &[i32], n_tokens: &[i32],
                         q: *const c_void, q_dtype: c_int, q_row_stride: i64, o: *mut c_void,
                         out_dtype: c_int, o_row_stride: i64, scale: f32,
                         workspace: *mut c_void, workspace_bytes: usize,
                         stream: *mut c_void) {
        assert_eq!(slots.len(), n_tokens.len(), "slots / n_tokens");
        check(sys::wattn_kv_attend(self.raw, to_c(layer, "layer"), slots.as_ptr(),
                                   n_tokens.as_ptr(), to_c(slots.len(), "n_seqs"), q, q_dtype,
                                   q_row_stride, o, out_dtype, o_row_stride, scale, workspace,
                                   workspace_bytes, stream), "attend");
    }

    /// The k_self (`which` 0) or v_self (1) rows of one slot and layer in the
    /// reference's flat layout `[t_past][d_model]` (decoder.rs:133-135).
    ///
    /// # Safety
    /// `out` must be a device pointer with room for slot_len(slot) rows of
    /// d_model elements of `out_dtype`.
    pub unsafe fn read_slot(&mut self, layer: usize, slot: usize, which: i32, out: *mut c_void,
                            out_dtype: c_int, stream: *mut c_void) {
        check(sys::wattn_kv_read_slot(self.raw, to_c(layer, "layer"), to_c(slot, "slot"), which,
                                      out, out_dtype, stream), "read_slot");
    }

    /// (pages in use, pool size in pages).
    pub fn stats(&self) -> (usize, usize) {
        let (mut used, mut total): (c_int, c_int) = (0, 0);
        // SAFETY: `raw` is a live cache; both out-pointers are valid.
        check(unsafe { sys::wattn_kv_stats(self.raw, &mut used, &mut total) }, "stats");
        (used as usize, total as usize)
    }
}

impl Drop for DeviceKvCache {
    fn drop(&mut self) {
        if !self.raw.is_null() {
            // SAFETY: `raw` came from wattn_kv_create and is destroyed once.
            unsafe { sys::wattn_kv_destroy(self.raw) };
            self.raw = std::ptr::null_mut();
        }
    }
}
