//! B200 batched token sampler for rust-llama: the reference's `Sampler` / `SamplingParams`
//! API (src/sampler.rs, re-exported by src/lib.rs:54) over the C ABI of
//! include/llamars_sampler.h, plus `BatchSampler` for many rows per call.
//!
//! Not compiled in this repository's build image (it has no Rust toolchain); the ABI this
//! crate declares (src/ffi.rs) is checked by tests/csrc/rust_abi.c in the CPU test suite.
pub mod ffi;
pub mod sampler;
pub mod stream;

pub use sampler::{BatchSampler, Sampler, SamplerError, SamplingParams};
pub use stream::{ByteStream, ByteStreams};
