//! The C ABI of include/llamars_sampler.h, declared for Rust.  Every declaration here is
//! mirrored by tests/csrc/rust_abi.c, which the CPU test suite compiles against the header
//! and runs against the built library (the ABI this file assumes is checked there).
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const LRS_OK: c_int = 0;
pub const LRS_E_INVALID: c_int = -1;
pub const LRS_E_NAN: c_int = -2;
pub const LRS_E_CUDA: c_int = -3;
pub const LRS_E_NOMEM: c_int = -4;
pub const LRS_E_TIMEOUT: c_int = -5;
pub const LRS_E_NCCL: c_int = -6;
pub const LRS_E_INTERNAL: c_int = -7;
pub const LRS_TOKEN_NONE: u32 = 0xFFFF_FFFF;

/// One row's SamplingParams without the seed (sampler.rs:3-13).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq)]
pub struct lrs_params {
    pub temperature: f32,
    pub top_k: u32,
    pub top_p: f32,
    pub repetition_penalty: f32,
    pub repeat_last_n: u32,
    pub reserved: u32,
}

/// Per-row diagnostics (optional output of lrs_sample_device).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct lrs_row_info {
    pub status: i32,
    pub token: u32,
    pub path: u32,
    pub k: u32,
    pub cutoff: u32,
    pub pos: u32,
    pub max: f32,
    pub sum_exp: f32,
    pub surv_sum: f32,
    pub r0: f32,
    pub prob: f32,
    pub n_cand: u32,
    pub events: u32,
    pub cycles: [u32; 8],
    pub reserved: u32,
}

const _: () = assert!(std::mem::size_of::<lrs_params>() == 24);
const _: () = assert!(std::mem::size_of::<lrs_row_info>() == 88);

#[repr(C)]
pub struct lrs_ctx {
    _private: [u8; 0],
}
#[repr(C)]
pub struct lrs_sampler {
    _private: [u8; 0],
}

extern "C" {
    pub fn lrs_create(device: c_int, max_rows: u32, max_vocab: u32, max_hist: u32, out: *mut *mut lrs_ctx) -> c_int;
    pub fn lrs_destroy(ctx: *mut lrs_ctx) -> c_int;
    pub fn lrs_last_error(ctx: *const lrs_ctx) -> *const c_char;
    pub fn lrs_seed_state(seed: u64) -> u64;
    pub fn lrs_set_state(ctx: *mut lrs_ctx, state: *const u64, rows: u32) -> c_int;
    pub fn lrs_get_state(ctx: *mut lrs_ctx, state: *mut u64, rows: u32) -> c_int;
    pub fn lrs_set_params(ctx: *mut lrs_ctx, params: *const lrs_params, rows: u32) -> c_int;
    pub fn lrs_sample(
        ctx: *mut lrs_ctx,
        logits: *const f32,
        logits_on_device: c_int,
        rows: u32,
        n: u32,
        ld: u64,
        hist: *const u32,
        hist_ld: u64,
        hist_len: *const u32,
        out_tokens: *mut u32,
        out_probs: *mut f32,
    ) -> c_int;
    pub fn lrs_sample_device(
        ctx: *mut lrs_ctx,
        d_logits: *const f32,
        rows: u32,
        n: u32,
        ld: u64,
        d_hist: *const u32,
        hist_ld: u64,
        d_hist_len: *const u32,
        d_params: *const lrs_params,
        d_state: *mut u64,
        d_tokens: *mut u32,
        d_probs: *mut f32,
        d_status: *mut i32,
        d_info: *mut lrs_row_info,
        stream: *mut c_void,
    ) -> c_int;
    pub fn lrs_poll_error(ctx: *mut lrs_ctx) -> c_int;
    pub fn lrs_sample_device_noalloc(
        device: c_int,
        d_logits: *const f32,
        rows: u32,
        n: u32,
        ld: u64,
        d_hist: *const u32,
        hist_ld: u64,
        d_hist_len: *const u32,
        d_params: *const lrs_params,
        d_state: *mut u64,
        d_tokens: *mut u32,
        d_probs: *mut f32,
        d_status: *mut i32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn lrs_noalloc_poll_error(device: c_int, stream: *mut c_void) -> c_int;
    pub fn lrs_history_append(
        d_tokens: *const u32,
        d_status: *const i32,
        rows: u32,
        eos: u32,
        d_hist: *mut u32,
        hist_ld: u64,
        d_hist_len: *mut u32,
        keep: u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn lrs_remap_tokens(
        d_tokens: *const u32,
        d_status: *const i32,
        rows: u32,
        d_map: *const u32,
        map_n: u32,
        d_out: *mut u32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn lrs_sampler_new(seed: u64, device: c_int) -> *mut lrs_sampler;
    pub fn lrs_sampler_free(s: *mut lrs_sampler);
    pub fn lrs_sampler_state(s: *const lrs_sampler) -> u64;
    pub fn lrs_sampler_sample(
        s: *mut lrs_sampler,
        logits: *const f32,
        n: usize,
        params: *const lrs_params,
        recent: *const u32,
        recent_len: usize,
        status: *mut c_int,
    ) -> u32;
}
