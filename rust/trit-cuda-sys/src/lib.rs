//! Bindings to libtrit_cuda.so, the B200 (sm_100a) build of the greedy
//! token loop of Trit's decoder language model.
//!
//! `ffi` holds one declaration per function of include/trit_cuda.h.
//! `GpuCausalLm` wraps them with the methods of the reference's `CausalLm`
//! (src/models/parts/causal_lm.rs:200-355): `prefix`, `generate`,
//! `generate_rows`, `answer`, `embed`, `width`, `layers`,
//! `set_ffn_scales`, `generate_additive`, `bidirectional_tokens`. A caller
//! such as `Cleaner` (src/cleanup.rs:203-208) or `Qwen3Asr`
//! (src/models/families/qwen3_asr.rs:179-181) changes only the line that
//! loads the model.
//!
//! The error and free calls carry the library's prefix
//! (`trit_cuda_last_error`, `trit_cuda_free_text`): the reference's own
//! cdylib exports `trit_last_error` and `trit_free_text`
//! (ffi/src/lib.rs:186,641), and a process that links both must not bind
//! one library's callers to the other's function.
//!
//! Not built in this repository's image (no cargo); see Cargo.toml.

use std::ffi::{c_char, c_int, c_void, CStr, CString};
use std::path::Path;
use std::ptr;

pub mod ffi {
    use super::*;

    #[repr(C)]
    pub struct TritLm {
        _p: [u8; 0],
    }
    #[repr(C)]
    pub struct TritLmPrefix {
        _p: [u8; 0],
    }
    #[repr(C)]
    pub struct TritDense {
        _p: [u8; 0],
    }

    #[link(name = "trit_cuda")]
    extern "C" {
        pub fn trit_cuda_version() -> *const c_char;
        pub fn trit_cuda_tp_id(out: *mut c_char, cap: usize) -> c_int;
        pub fn trit_cuda_last_error() -> *const c_char;
        pub fn trit_lm_inspect(model_dir: *const c_char, options_json: *const c_char) -> *mut c_char;
        pub fn trit_cuda_free_text(text: *mut c_char);
        pub fn trit_lm_load(model_dir: *const c_char, options_json: *const c_char) -> *mut TritLm;
        pub fn trit_lm_free(lm: *mut TritLm);
        pub fn trit_lm_status(lm: *const TritLm) -> *mut c_char;
        pub fn trit_lm_width(lm: *const TritLm) -> i64;
        pub fn trit_lm_layers(lm: *const TritLm) -> i64;
        pub fn trit_lm_vocab(lm: *const TritLm) -> i64;
        pub fn trit_lm_prefix(lm: *mut TritLm, ids: *const i32, n: usize) -> *mut TritLmPrefix;
        pub fn trit_lm_prefix_free(prefix: *mut TritLmPrefix);
        pub fn trit_lm_generate(
            lm: *mut TritLm, prefix: *const TritLmPrefix, prompt: *const i32, n: usize, max_new: i32,
            stop: *const i32, nstop: usize, out: *mut i32, cap: usize,
        ) -> i64;
        pub fn trit_lm_generate_rows(
            lm: *mut TritLm, rows: *const f32, nrows: usize, max_new: i32, stop: *const i32, nstop: usize,
            out: *mut i32, cap: usize,
        ) -> i64;
        pub fn trit_lm_answer(
            lm: *mut TritLm, head: *const i32, nhead: usize, audio: *const f32, naudio: usize,
            tail: *const i32, ntail: usize, max_new: i32, stop: *const i32, nstop: usize, out: *mut i32,
            cap: usize,
        ) -> i64;
        pub fn trit_lm_generate_rows_device(
            lm: *mut TritLm, rows_device: *const f32, nrows: usize, max_new: i32, stop: *const i32, nstop: usize,
            out: *mut i32, cap: usize, cuda_stream: *mut c_void,
        ) -> i64;
        pub fn trit_lm_answer_device(
            lm: *mut TritLm, head: *const i32, nhead: usize, audio_device: *const f32, naudio: usize,
            tail: *const i32, ntail: usize, max_new: i32, stop: *const i32, nstop: usize, out: *mut i32,
            cap: usize, cuda_stream: *mut c_void,
        ) -> i64;
        pub fn trit_lm_embed(lm: *mut TritLm, ids: *const i32, n: usize, out: *mut f32) -> c_int;
        pub fn trit_lm_generate_traced(
            lm: *mut TritLm, prefix: *const TritLmPrefix, prompt: *const i32, n: usize, max_new: i32,
            stop: *const i32, nstop: usize, out: *mut i32, cap: usize, logits: *mut f32,
        ) -> i64;
        pub fn trit_lm_answer_traced(
            lm: *mut TritLm, head: *const i32, nhead: usize, audio: *const f32, naudio: usize,
            tail: *const i32, ntail: usize, max_new: i32, stop: *const i32, nstop: usize, out: *mut i32,
            cap: usize, logits: *mut f32,
        ) -> i64;
        pub fn trit_lm_generate_batch(
            lm: *mut TritLm, streams: usize, prompts: *const *const i32, lens: *const usize, max_new: i32,
            stop: *const i32, nstop: usize, out: *mut i32, counts: *mut i64,
        ) -> c_int;
        pub fn trit_lm_generate_batch_prefix(
            lm: *mut TritLm, prefix: *const TritLmPrefix, streams: usize, prompts: *const *const i32,
            lens: *const usize, max_new: i32, stop: *const i32, nstop: usize, out: *mut i32, counts: *mut i64,
        ) -> c_int;
        pub fn trit_lm_prefix_pages(lm: *const TritLm, used: *mut i64, total: *mut i64) -> c_int;
        pub fn trit_lm_set_ffn_scales(lm: *mut TritLm, scales: *const f32, layers: usize, width: usize) -> c_int;
        pub fn trit_lm_generate_additive(
            lm: *mut TritLm, prompt: *const i32, n: usize, audio: *const f32, rows: usize, stop: *const i32,
            nstop: usize, out: *mut i32, cap: usize,
        ) -> i64;
        pub fn trit_lm_bidirectional_tokens(
            lm: *mut TritLm, rows: *const f32, m: usize, from: usize, out: *mut i32,
        ) -> i64;
        pub fn trit_lm_last_timing(
            lm: *const TritLm, prefill_ms: *mut f64, decode_ms: *mut f64, decode_steps: *mut i64,
            launches: *mut i64,
        ) -> c_int;
        pub fn trit_dense_q8_0(blocks: *const c_void, n: usize, k: usize, table: c_int, device: c_int)
            -> *mut TritDense;
        pub fn trit_dense_forward(layer: *mut TritDense, x: *const f32, rows: usize, out: *mut f32) -> c_int;
        pub fn trit_dense_forward_device(
            layer: *mut TritDense, x: *const f32, rows: usize, out: *mut f32, cuda_stream: *mut c_void,
        ) -> c_int;
        pub fn trit_dense_free(layer: *mut TritDense);
        pub fn trit_dense_q8_0_forward_static(
            codes: *const c_void, scales: *const c_void, n: usize, k: usize, x: *const f32, rows: usize,
            out: *mut f32, cuda_stream: *mut c_void,
        ) -> c_int;
    }
}

/// The calling thread's last error text from the library.
pub fn last_error() -> String {
    // SAFETY: the library returns a NUL-terminated string it owns, valid
    // until the next call on this thread.
    unsafe { CStr::from_ptr(ffi::trit_cuda_last_error()) }.to_string_lossy().into_owned()
}

fn ids(values: &[usize]) -> Vec<i32> {
    values.iter().map(|&t| t as i32).collect()
}

fn tokens(out: Vec<i32>, n: i64) -> Vec<usize> {
    // The reference's generate cannot fail; a failure here is a device
    // error (no GPU, out of memory), reported like its worker panics.
    assert!(n >= 0, "trit_cuda: {}", last_error());
    let mut out = out;
    out.truncate(n as usize);
    out.into_iter().map(|t| t as usize).collect()
}

/// Load options of include/trit_cuda.h (`trit_lm_load`), as JSON text.
#[derive(Clone, Debug, Default)]
pub struct Options {
    pub device: Option<i32>,
    pub kv_f32: bool,
    pub max_context: Option<usize>,
    pub max_streams: Option<usize>,
    pub config_at: String,
    pub prefix: String,
}

impl Options {
    fn json(&self) -> String {
        let mut fields = vec![
            format!("\"config_at\": {:?}", self.config_at),
            format!("\"prefix\": {:?}", self.prefix),
        ];
        if let Some(d) = self.device {
            fields.push(format!("\"device\": {d}"));
        }
        if self.kv_f32 {
            fields.push("\"kv\": \"f32\"".into());
        }
        if let Some(n) = self.max_context {
            fields.push(format!("\"max_context\": {n}"));
        }
        if let Some(n) = self.max_streams {
            fields.push(format!("\"max_streams\": {n}"));
        }
        format!("{{{}}}", fields.join(", "))
    }
}

/// `CausalLm` on a GPU (src/models/parts/causal_lm.rs), with its methods.
pub struct GpuCausalLm {
    raw: *mut ffi::TritLm,
}

/// `Prefix` (causal_lm.rs:118-122): a prompt start run once.
pub struct GpuPrefix {
    raw: *mut ffi::TritLmPrefix,
}

// SAFETY: calls on one handle take turns under the library's mutex
// (include/trit_cuda.h), as calls on one Trit engine share one team.
unsafe impl Send for GpuCausalLm {}
unsafe impl Sync for GpuCausalLm {}
unsafe impl Send for GpuPrefix {}
unsafe impl Sync for GpuPrefix {}

impl GpuCausalLm {
    /// `CausalLm::load` / `from_tensors(.., (config_at, prefix))`
    /// (causal_lm.rs:124-198) on the model folder `dir`.
    pub fn load(dir: &Path, options: &Options) -> Result<Self, String> {
        let dir = CString::new(dir.to_string_lossy().as_bytes()).map_err(|e| e.to_string())?;
        let opts = CString::new(options.json()).map_err(|e| e.to_string())?;
        // SAFETY: both strings are NUL-terminated and live across the call.
        let raw = unsafe { ffi::trit_lm_load(dir.as_ptr(), opts.as_ptr()) };
        if raw.is_null() {
            Err(last_error())
        } else {
            Ok(Self { raw })
        }
    }

    pub fn width(&self) -> usize {
        // SAFETY: `raw` is a live handle.
        unsafe { ffi::trit_lm_width(self.raw) as usize }
    }

    pub fn layers(&self) -> usize {
        // SAFETY: `raw` is a live handle.
        unsafe { ffi::trit_lm_layers(self.raw) as usize }
    }

    pub fn prefix(&self, tokens: &[usize]) -> GpuPrefix {
        let t = ids(tokens);
        // SAFETY: `t` lives across the call.
        let raw = unsafe { ffi::trit_lm_prefix(self.raw, t.as_ptr(), t.len()) };
        assert!(!raw.is_null(), "trit_cuda: {}", last_error());
        GpuPrefix { raw }
    }

    pub fn generate(&self, prompt: &[usize], prefix: Option<&GpuPrefix>, max_new: usize, stop: &[usize]) -> Vec<usize> {
        let (p, s) = (ids(prompt), ids(stop));
        let mut out = vec![0i32; max_new];
        // SAFETY: every buffer lives across the call; `out` holds `cap` ids.
        let n = unsafe {
            ffi::trit_lm_generate(
                self.raw, prefix.map_or(ptr::null(), |x| x.raw), p.as_ptr(), p.len(), max_new as i32,
                s.as_ptr(), s.len(), out.as_mut_ptr(), out.len(),
            )
        };
        tokens(out, n)
    }

    /// `generate_rows(rows, max_new, stop)`: `rows` is rows x width floats.
    pub fn generate_rows(&self, rows: &[f32], max_new: usize, stop: &[usize]) -> Vec<usize> {
        let s = ids(stop);
        let mut out = vec![0i32; max_new];
        // SAFETY: every buffer lives across the call.
        let n = unsafe {
            ffi::trit_lm_generate_rows(
                self.raw, rows.as_ptr(), rows.len() / self.width(), max_new as i32, s.as_ptr(), s.len(),
                out.as_mut_ptr(), out.len(),
            )
        };
        tokens(out, n)
    }

    pub fn answer(&self, head: &[usize], audio: &[f32], tail: &[usize], max_new: usize, stop: &[usize]) -> Vec<usize> {
        let (h, t, s) = (ids(head), ids(tail), ids(stop));
        let mut out = vec![0i32; max_new];
        // SAFETY: every buffer lives across the call.
        let n = unsafe {
            ffi::trit_lm_answer(
                self.raw, h.as_ptr(), h.len(), audio.as_ptr(), audio.len() / self.width(), t.as_ptr(), t.len(),
                max_new as i32, s.as_ptr(), s.len(), out.as_mut_ptr(), out.len(),
            )
        };
        tokens(out, n)
    }

    /// `answer` with the audio rows (`nrows` x width f32) in device memory of
    /// the model's GPU, read after the work queued on `cuda_stream` (an
    /// encoder's output that stays on the GPU).
    ///
    /// # Safety
    /// `audio_device` must point to `nrows * width` floats of device memory
    /// on the model's GPU, and `cuda_stream` must be a live stream or null.
    pub unsafe fn answer_device(
        &self, head: &[usize], audio_device: *const f32, nrows: usize, tail: &[usize], max_new: usize,
        stop: &[usize], cuda_stream: *mut c_void,
    ) -> Vec<usize> {
        let (h, t, s) = (ids(head), ids(tail), ids(stop));
        let mut out = vec![0i32; max_new];
        let n = ffi::trit_lm_answer_device(
            self.raw, h.as_ptr(), h.len(), audio_device, nrows, t.as_ptr(), t.len(), max_new as i32, s.as_ptr(),
            s.len(), out.as_mut_ptr(), out.len(), cuda_stream,
        );
        tokens(out, n)
    }

    pub fn embed(&self, ids_in: &[usize]) -> Vec<f32> {
        let t = ids(ids_in);
        let mut out = vec![0f32; t.len() * self.width()];
        // SAFETY: `out` holds n x width floats.
        let rc = unsafe { ffi::trit_lm_embed(self.raw, t.as_ptr(), t.len(), out.as_mut_ptr()) };
        assert!(rc == 0, "trit_cuda: {}", last_error());
        out
    }

    /// `set_ffn_scales(Vec<Vec<f32>>)`: one row of width floats a layer.
    pub fn set_ffn_scales(&mut self, scales: Vec<Vec<f32>>) {
        let flat: Vec<f32> = scales.iter().flatten().copied().collect();
        // SAFETY: `flat` holds layers x width floats.
        let rc = unsafe { ffi::trit_lm_set_ffn_scales(self.raw, flat.as_ptr(), scales.len(), self.width()) };
        assert!(rc == 0, "trit_cuda: {}", last_error());
    }

    pub fn generate_additive(&self, prompt: &[usize], audio: &[f32], stop: &[usize]) -> Vec<usize> {
        let (p, s) = (ids(prompt), ids(stop));
        let rows = audio.len() / self.width();
        let mut out = vec![0i32; rows + 1];
        // SAFETY: every buffer lives across the call.
        let n = unsafe {
            ffi::trit_lm_generate_additive(
                self.raw, p.as_ptr(), p.len(), audio.as_ptr(), rows, s.as_ptr(), s.len(), out.as_mut_ptr(),
                out.len(),
            )
        };
        tokens(out, n)
    }

    pub fn bidirectional_tokens(&self, rows: &[f32], from: usize) -> Vec<usize> {
        let m = rows.len() / self.width();
        let mut out = vec![0i32; m.saturating_sub(from)];
        // SAFETY: `out` holds m - from ids.
        let n = unsafe { ffi::trit_lm_bidirectional_tokens(self.raw, rows.as_ptr(), m, from, out.as_mut_ptr()) };
        tokens(out, n)
    }
}

impl Drop for GpuCausalLm {
    fn drop(&mut self) {
        // SAFETY: the handle is freed once, when no call is running on it.
        unsafe { ffi::trit_lm_free(self.raw) }
    }
}

impl Drop for GpuPrefix {
    fn drop(&mut self) {
        // SAFETY: the prefix is freed once.
        unsafe { ffi::trit_lm_prefix_free(self.raw) }
    }
}
