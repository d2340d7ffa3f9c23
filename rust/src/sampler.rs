//! rust-llama's sampler API (src/sampler.rs) on the B200 library.
//!
//! * `SamplingParams` and `Sampler` keep the reference's names, fields, defaults and
//!   signatures (sampler.rs:3-56), so `Sampler::new(params.seed)` / `sampler.sample(&logits,
//!   &params, &recent)` in model.rs:752-761, server.rs:182-187 and main.rs:552-577 work
//!   unchanged; the draw is the reference's (same token, same PRNG stream).
//! * `BatchSampler` samples many rows per call on one GPU: per-row parameters and PRNG
//!   states live on the device, logits come from host memory (`sample`) or device memory
//!   (`sample_device`, the hot path of a batched server).
use std::ffi::CStr;
use std::fmt;
use std::os::raw::c_void;

use crate::ffi;

/// sampler.rs:3-13.
#[derive(Clone, Debug)]
pub struct SamplingParams {
    pub temperature: f32,
    pub top_k: usize,
    pub top_p: f32,
    pub repetition_penalty: f32,
    /// How many trailing tokens the repetition penalty looks at; 0 = the whole history.
    pub repeat_last_n: usize,
    pub seed: u64,
}

/// sampler.rs:15-26.
impl Default for SamplingParams {
    fn default() -> Self {
        SamplingParams {
            temperature: 0.7,
            top_k: 40,
            top_p: 0.95,
            repetition_penalty: 1.1,
            repeat_last_n: 64,
            seed: 0x1234_5678_9abc_def0,
        }
    }
}

impl SamplingParams {
    fn to_ffi(&self) -> ffi::lrs_params {
        ffi::lrs_params {
            temperature: self.temperature,
            top_k: self.top_k.min(u32::MAX as usize) as u32,
            top_p: self.top_p,
            repetition_penalty: self.repetition_penalty,
            repeat_last_n: self.repeat_last_n.min(u32::MAX as usize) as u32,
            reserved: 0,
        }
    }
}

/// A status other than LRS_OK, with the library's message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct SamplerError {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for SamplerError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "{} (status {})", self.message, self.code)
    }
}

impl std::error::Error for SamplerError {}

fn check(code: i32, ctx: *const ffi::lrs_ctx) -> Result<(), SamplerError> {
    if code == ffi::LRS_OK {
        return Ok(());
    }
    let msg = unsafe {
        let p = ffi::lrs_last_error(ctx);
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    Err(SamplerError { code, message: msg })
}

/// sampler.rs:28-56: one generation stream.  The first `sample` creates a one-row
/// context on GPU 0 (`with_device` picks another).
pub struct Sampler {
    raw: *mut ffi::lrs_sampler,
}

impl Sampler {
    /// sampler.rs:33-37 (state = seed | 1).
    pub fn new(seed: u64) -> Self {
        Self::with_device(seed, 0)
    }

    pub fn with_device(seed: u64, device: i32) -> Self {
        Sampler { raw: unsafe { ffi::lrs_sampler_new(seed, device) } }
    }

    /// The PRNG state (`Sampler.state` in the reference).
    pub fn state(&self) -> u64 {
        unsafe { ffi::lrs_sampler_state(self.raw) }
    }

    /// sampler.rs:56: the reference's `sample`.  Like the reference, which panics (and
    /// aborts) on NaN probabilities, this panics when the library reports an error.
    pub fn sample(&mut self, logits: &[f32], params: &SamplingParams, recent: &[u32]) -> u32 {
        match self.try_sample(logits, params, recent) {
            Ok(t) => t,
            Err(e) => panic!("sampler: {e}"),
        }
    }

    /// `sample` returning the library's status instead of panicking.
    pub fn try_sample(&mut self, logits: &[f32], params: &SamplingParams, recent: &[u32]) -> Result<u32, SamplerError> {
        let p = params.to_ffi();
        let mut status: i32 = 0;
        let tok = unsafe {
            ffi::lrs_sampler_sample(self.raw, logits.as_ptr(), logits.len(), &p, recent.as_ptr(), recent.len(),
                                    &mut status)
        };
        if status != ffi::LRS_OK {
            let message = if status == ffi::LRS_E_NAN {
                "NaN probabilities (the reference sampler panics here)".to_string()
            } else {
                "sampling failed".to_string()
            };
            return Err(SamplerError { code: status, message });
        }
        Ok(tok)
    }
}

impl Drop for Sampler {
    fn drop(&mut self) {
        unsafe { ffi::lrs_sampler_free(self.raw) }
    }
}

/// Independent samplers, one per row, on one GPU (a context of the C ABI).  Not
/// reentrant: drive it from one thread (it is `Send`, not `Sync`).
pub struct BatchSampler {
    ctx: *mut ffi::lrs_ctx,
    max_rows: u32,
    max_vocab: u32,
    max_hist: u32,
}

unsafe impl Send for BatchSampler {}

impl BatchSampler {
    /// A context on `device` for up to `max_rows` rows of up to `max_vocab` logits and
    /// `max_hist` history ids per row.
    pub fn new(device: i32, max_rows: u32, max_vocab: u32, max_hist: u32) -> Result<Self, SamplerError> {
        let mut ctx: *mut ffi::lrs_ctx = std::ptr::null_mut();
        check(unsafe { ffi::lrs_create(device, max_rows, max_vocab, max_hist, &mut ctx) }, std::ptr::null())?;
        Ok(BatchSampler { ctx, max_rows, max_vocab, max_hist })
    }

    pub fn max_rows(&self) -> u32 {
        self.max_rows
    }
    pub fn max_vocab(&self) -> u32 {
        self.max_vocab
    }
    pub fn max_hist(&self) -> u32 {
        self.max_hist
    }

    /// Per-row parameters (their seeds are ignored: see `set_seeds`).
    pub fn set_params(&mut self, params: &[SamplingParams]) -> Result<(), SamplerError> {
        let p: Vec<ffi::lrs_params> = params.iter().map(|x| x.to_ffi()).collect();
        check(unsafe { ffi::lrs_set_params(self.ctx, p.as_ptr(), p.len() as u32) }, self.ctx)
    }

    /// `Sampler::new(seed)` for every row: state = seed | 1.
    pub fn set_seeds(&mut self, seeds: &[u64]) -> Result<(), SamplerError> {
        let st: Vec<u64> = seeds.iter().map(|&s| unsafe { ffi::lrs_seed_state(s) }).collect();
        self.set_state(&st)
    }

    pub fn set_state(&mut self, state: &[u64]) -> Result<(), SamplerError> {
        check(unsafe { ffi::lrs_set_state(self.ctx, state.as_ptr(), state.len() as u32) }, self.ctx)
    }

    pub fn get_state(&mut self, rows: u32) -> Result<Vec<u64>, SamplerError> {
        let mut st = vec![0u64; rows as usize];
        check(unsafe { ffi::lrs_get_state(self.ctx, st.as_mut_ptr(), rows) }, self.ctx)?;
        Ok(st)
    }

    /// One `Sampler::sample` per row from host memory: `logits` holds `rows` rows of `n`
    /// values (row r at r * n), `recent[r]` is row r's history (oldest first).  Returns the
    /// tokens; synchronous.
    pub fn sample(&mut self, logits: &[f32], n: usize, recent: &[&[u32]]) -> Result<Vec<u32>, SamplerError> {
        let rows = recent.len();
        if n == 0 || logits.len() < rows * n {
            return Err(SamplerError { code: ffi::LRS_E_INVALID, message: "logits shorter than rows * n".into() });
        }
        let hist_ld = recent.iter().map(|h| h.len()).max().unwrap_or(0);
        let mut hist = vec![0u32; rows * hist_ld.max(1)];
        let mut hist_len = vec![0u32; rows];
        for (r, h) in recent.iter().enumerate() {
            hist[r * hist_ld..r * hist_ld + h.len()].copy_from_slice(h);
            hist_len[r] = h.len() as u32;
        }
        let mut tokens = vec![ffi::LRS_TOKEN_NONE; rows];
        check(
            unsafe {
                ffi::lrs_sample(self.ctx, logits.as_ptr(), 0, rows as u32, n as u32, n as u64, hist.as_ptr(),
                                hist_ld as u64, hist_len.as_ptr(), tokens.as_mut_ptr(), std::ptr::null_mut())
            },
            self.ctx,
        )?;
        Ok(tokens)
    }

    /// The hot path: every pointer a device pointer, enqueued on `stream` (a cudaStream_t),
    /// no host synchronisation.  Row errors go to `d_status`; an error of an earlier launch
    /// is returned by the next call (or `poll_error`).
    ///
    /// # Safety
    /// The pointers must be valid device allocations of the sizes of lrs_sample_device.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn sample_device(
        &mut self,
        d_logits: *const f32,
        rows: u32,
        n: u32,
        ld: u64,
        d_hist: *const u32,
        hist_ld: u64,
        d_hist_len: *const u32,
        d_params: *const ffi::lrs_params,
        d_state: *mut u64,
        d_tokens: *mut u32,
        d_probs: *mut f32,
        d_status: *mut i32,
        stream: *mut c_void,
    ) -> Result<(), SamplerError> {
        check(
            ffi::lrs_sample_device(self.ctx, d_logits, rows, n, ld, d_hist, hist_ld, d_hist_len, d_params, d_state,
                                   d_tokens, d_probs, d_status, std::ptr::null_mut(), stream),
            self.ctx,
        )
    }

    /// `recent.push(next)` of a batched generation loop (model.rs:768, server.rs:187), on the
    /// device: appends each row's token to its history row (the layout `sample_device` reads)
    /// unless the row failed or drew `eos`; a full row keeps its last `keep` ids.
    ///
    /// # Safety
    /// Device pointers valid for `rows` rows (`hist_ld` ids each) on the context's GPU.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn history_append(
        &mut self,
        d_tokens: *const u32,
        d_status: *const i32,
        rows: u32,
        eos: u32,
        d_hist: *mut u32,
        hist_ld: u64,
        d_hist_len: *mut u32,
        keep: u32,
        stream: *mut c_void,
    ) -> Result<(), SamplerError> {
        check(
            ffi::lrs_history_append(d_tokens, d_status, rows, eos, d_hist, hist_ld, d_hist_len, keep, stream),
            std::ptr::null(),
        )
    }

    /// Pruned-vocabulary ids back to the full vocabulary (prune.rs:187-195 renumbers the kept
    /// ids in order): `d_out[r] = d_map[d_tokens[r]]` for rows sampled without error.
    ///
    /// # Safety
    /// Device pointers valid for `rows` tokens and `map_n` map entries on the context's GPU.
    pub unsafe fn remap_tokens(
        &mut self,
        d_tokens: *const u32,
        d_status: *const i32,
        rows: u32,
        d_map: *const u32,
        map_n: u32,
        d_out: *mut u32,
        stream: *mut c_void,
    ) -> Result<(), SamplerError> {
        check(ffi::lrs_remap_tokens(d_tokens, d_status, rows, d_map, map_n, d_out, stream), std::ptr::null())
    }

    /// Waits for the last launch and returns the error it reported, if any.
    pub fn poll_error(&mut self) -> Result<(), SamplerError> {
        check(unsafe { ffi::lrs_poll_error(self.ctx) }, self.ctx)
    }
}

impl Drop for BatchSampler {
    fn drop(&mut self) {
        unsafe {
            ffi::lrs_destroy(self.ctx);
        }
    }
}
