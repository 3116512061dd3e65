//! The B200 token sampler behind `rusticide-sampling`'s API.
//!
//! `CudaSampler` is a batched `Sampler`: one call samples many logit rows,
//! each exactly as `Sampler::sample_logits` / `greedy_logits` /
//! `sample_with_temp` would (crates/rusticide-sampling/src/sampler.rs:44-105),
//! on an sm_100a GPU through `librusticide_cuda.so`.
//!
//! Three entry points:
//!
//! * [`CudaSampler::pick_rows`]: host rows in, tokens out, safe. It is the
//!   batched form of `rusticide_model::generate::pick`
//!   (crates/rusticide-model/src/generate.rs:117-124) for the logits that
//!   `Model::forward` returns today (a host `Vec<f32>`). Each row carries its
//!   own `fastrand::Rng`, seeded as `Sampler::new(seed)` seeds its own; the
//!   row's uniform is that generator's next `f32()`, and the generator only
//!   advances on rows that consumed a draw, so a batch of one gives the
//!   reference's token sequence for the same seed.
//! * [`CudaSampler::sample_device`]: rows already in device memory (a GPU
//!   model's LM head). `unsafe`: the caller vouches for the device pointers.
//! * [`CudaSampler::sample_rows_device`]: the same with one `SamplingParams`
//!   per row, for a batch of sequences that each carry their own parameters.
//!
//! `unsafe` in this crate is limited to the FFI calls; each block states why
//! the call is sound.

#[allow(dead_code)]
mod ffi;

use std::ffi::{CStr, c_void};
use std::ptr::{self, NonNull};

use rusticide_sampling::{SamplingError, SamplingParams};

/// A failure of the library call itself (arguments, capacity, CUDA).
#[derive(Debug, thiserror::Error)]
pub enum CudaError {
    #[error("rusticide_cuda: {what} failed: {name} ({code})")]
    Call { what: &'static str, code: i32, name: String },
    #[error("rusticide_cuda ABI {found}, this crate expects {expected}")]
    AbiMismatch { found: i32, expected: i32 },
    #[error("row {row}: a bounded device wait gave up; sample the row again")]
    RowInternal { row: usize },
    #[error("{rows} rows need {need} generators, got {got}")]
    Generators { rows: usize, need: usize, got: usize },
}

fn status_name(code: i32) -> String {
    // SAFETY: rsc_status_string returns a pointer to a static NUL-terminated
    // string for every value, including unknown ones.
    let p = unsafe { ffi::rsc_status_string(code) };
    if p.is_null() {
        return format!("status {code}");
    }
    // SAFETY: non-null, static, NUL-terminated (see above).
    unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
}

fn check(what: &'static str, code: i32) -> Result<(), CudaError> {
    if code == ffi::RSC_OK {
        Ok(())
    } else {
        Err(CudaError::Call { what, code, name: status_name(code) })
    }
}

const fn to_c(p: &SamplingParams) -> ffi::RscParams {
    ffi::RscParams {
        temperature: p.temperature,
        top_k: p.top_k,
        top_p: p.top_p,
        repetition_penalty: p.repetition_penalty,
        seed: p.seed,
    }
}

/// One row's outcome, as the reference's `Result<u32, SamplingError>`.
fn row_result(status: i32, id: u32, row: usize) -> Result<Result<u32, SamplingError>, CudaError> {
    match status & ffi::RSC_ROW_CODE_MASK {
        ffi::RSC_ROW_OK => Ok(Ok(id)),
        ffi::RSC_ROW_NO_VALID_TOKENS => Ok(Err(SamplingError::NoValidTokens)),
        ffi::RSC_ROW_VOCAB_OVERFLOW => Ok(Err(SamplingError::VocabOverflow)),
        ffi::RSC_ROW_INTERNAL => Err(CudaError::RowInternal { row }),
        code => Err(CudaError::Call { what: "row status", code, name: status_name(code) }),
    }
}

/// Whether the reference consumes a draw for these params: every path but
/// the argmax one (sampler.rs:48) and greedy `pick` (generate.rs:118).
fn draws(params: &SamplingParams) -> bool {
    !(params.temperature == 0.0 || params.top_k == 1)
}

/// A sampler for batches of up to `max_rows` rows of up to `max_vocab`
/// logits on one GPU. Owns its device scratch; not `Sync`.
pub struct CudaSampler {
    raw: NonNull<ffi::RscSampler>,
    max_rows: usize,
    max_vocab: usize,
}

// SAFETY: the handle has no thread affinity; it only must not be used from two
// threads at once, which `&mut self` on every sampling method guarantees.
unsafe impl Send for CudaSampler {}

impl CudaSampler {
    /// Creates the sampler and its device scratch on `device`.
    ///
    /// # Errors
    ///
    /// `CudaError` if the library's ABI differs, the device does not exist,
    /// or the scratch cannot be allocated.
    pub fn new(device: i32, max_rows: usize, max_vocab: usize) -> Result<Self, CudaError> {
        // SAFETY: no arguments; returns a constant.
        let found = unsafe { ffi::rsc_abi_version() };
        if found != ffi::RSC_ABI_VERSION {
            return Err(CudaError::AbiMismatch { found, expected: ffi::RSC_ABI_VERSION });
        }
        let mut raw = ptr::null_mut();
        // SAFETY: `raw` is a valid out-pointer for the handle.
        check("rsc_sampler_create", unsafe {
            ffi::rsc_sampler_create(device, max_rows, max_vocab, &raw mut raw)
        })?;
        let raw = NonNull::new(raw).ok_or(CudaError::Call {
            what: "rsc_sampler_create",
            code: -1,
            name: "null handle".to_owned(),
        })?;
        Ok(Self { raw, max_rows, max_vocab })
    }

    #[must_use]
    pub const fn max_rows(&self) -> usize {
        self.max_rows
    }

    #[must_use]
    pub const fn max_vocab(&self) -> usize {
        self.max_vocab
    }

    /// Batched `generate::pick` over host rows: `logits` holds
    /// `logits.len() / vocab` dense rows; `rngs` one generator per row,
    /// advanced only for rows that drew.
    ///
    /// # Errors
    ///
    /// The outer `Err` is a failure of the call (shape, capacity, CUDA); the
    /// inner per-row `Err` is the reference's `SamplingError` for that row.
    pub fn pick_rows(
        &mut self,
        logits: &[f32],
        vocab: usize,
        params: &SamplingParams,
        rngs: &mut [fastrand::Rng],
    ) -> Result<Vec<Result<u32, SamplingError>>, CudaError> {
        if vocab == 0 || logits.len() % vocab != 0 {
            return Err(CudaError::Call {
                what: "pick_rows",
                code: ffi::RSC_ERR_INVALID_SHAPE,
                name: status_name(ffi::RSC_ERR_INVALID_SHAPE),
            });
        }
        if u32::try_from(vocab).is_err() {
            return Err(CudaError::Call {
                what: "pick_rows",
                code: ffi::RSC_ERR_VOCAB_TOO_LARGE,
                name: status_name(ffi::RSC_ERR_VOCAB_TOO_LARGE),
            });
        }
        let rows = logits.len() / vocab;
        let drawing = draws(params);
        if drawing && rngs.len() != rows {
            return Err(CudaError::Generators { rows, need: rows, got: rngs.len() });
        }
        // The next uniform of every row's generator, taken from a copy so that
        // rows which end up not drawing keep their state.
        let mut next: Vec<fastrand::Rng> = Vec::new();
        let mut uniforms: Vec<f32> = Vec::new();
        if drawing {
            next = rngs.to_vec();
            uniforms = next.iter_mut().map(fastrand::Rng::f32).collect();
        }
        let mut ids = vec![0_u32; rows];
        let mut status = vec![0_i32; rows];
        let c = to_c(params);
        // SAFETY: every host buffer is valid for the lengths passed (`rows`
        // rows of `vocab` logits; `rows` uniforms, ids and statuses); the
        // probabilities pointer is null, which the ABI allows; the handle is
        // live and used by this thread only (`&mut self`). The call is
        // synchronous, so the borrows outlive it.
        check("rsc_pick_host", unsafe {
            ffi::rsc_pick_host(
                self.raw.as_ptr(),
                logits.as_ptr(),
                rows,
                vocab,
                &raw const c,
                if drawing { uniforms.as_ptr() } else { ptr::null() },
                ids.as_mut_ptr(),
                status.as_mut_ptr(),
                ptr::null_mut(),
            )
        })?;
        let mut out = Vec::with_capacity(rows);
        for (row, (&st, &id)) in status.iter().zip(&ids).enumerate() {
            let r = row_result(st, id, row)?;
            // NoValidTokens is raised before the draw (sampler.rs:50-51, via
            // valid_probabilities), VocabOverflow after it (sampler.rs:53).
            let consumed = drawing && !matches!(r, Err(SamplingError::NoValidTokens));
            if consumed {
                rngs[row] = next[row].clone();
            }
            out.push(r);
        }
        Ok(out)
    }

    /// Batched `sample_logits` (or `pick` with `pick = true`) on device rows,
    /// asynchronous on `stream`.
    ///
    /// # Safety
    ///
    /// `d_logits` must address `rows` device rows of `vocab` f32 at a
    /// distance of `row_stride` elements; `d_uniforms` (or `d_rng_states`)
    /// `rows` device values unless every row takes the argmax branch;
    /// `d_ids`, `d_status` (and `d_probs` when non-null) `rows` device
    /// elements; all on this sampler's device and alive until `stream` has
    /// run the call; `stream` a `cudaStream_t` of that device or null.
    ///
    /// # Errors
    ///
    /// `CudaError` for a rejected argument or a launch failure.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn sample_device(
        &mut self,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        params: &SamplingParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_ids: *mut u32,
        d_status: *mut i32,
        d_probs: *mut f32,
        stream: *mut c_void,
        pick: bool,
    ) -> Result<(), CudaError> {
        let c = to_c(params);
        // SAFETY: the caller's contract above covers every pointer; the handle
        // is live and exclusively borrowed.
        let code = unsafe {
            if pick {
                ffi::rsc_pick(
                    self.raw.as_ptr(), d_logits, rows, vocab, row_stride, &raw const c,
                    d_uniforms, d_rng_states, d_ids, d_status, d_probs, stream,
                )
            } else {
                ffi::rsc_sample(
                    self.raw.as_ptr(), d_logits, rows, vocab, row_stride, &raw const c,
                    d_uniforms, d_rng_states, d_ids, d_status, d_probs, stream,
                )
            }
        };
        check(if pick { "rsc_pick" } else { "rsc_sample" }, code)
    }

    /// Batched `sample_logits` on device rows with one `SamplingParams` per
    /// row (`params[r]` for row `r`), asynchronous on `stream`; the sets are
    /// copied before the call returns.
    ///
    /// # Safety
    ///
    /// As [`CudaSampler::sample_device`], with `params.len() == rows`.
    ///
    /// # Errors
    ///
    /// `CudaError` for a rejected argument or a launch failure.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn sample_rows_device(
        &mut self,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        params: &[SamplingParams],
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_ids: *mut u32,
        d_status: *mut i32,
        d_probs: *mut f32,
        stream: *mut c_void,
    ) -> Result<(), CudaError> {
        if params.len() != rows {
            return Err(CudaError::Call {
                what: "rsc_sample_rows",
                code: ffi::RSC_ERR_INVALID_SHAPE,
                name: status_name(ffi::RSC_ERR_INVALID_SHAPE),
            });
        }
        let c: Vec<ffi::RscParams> = params.iter().map(to_c).collect();
        // SAFETY: `c` holds `rows` sets and outlives the call (the library
        // copies them before returning); the caller's contract covers the
        // device pointers; the handle is live and exclusively borrowed.
        let code = unsafe {
            ffi::rsc_sample_rows(
                self.raw.as_ptr(), d_logits, rows, vocab, row_stride, c.as_ptr(), d_uniforms,
                d_rng_states, d_ids, d_status, d_probs, stream,
            )
        };
        check("rsc_sample_rows", code)
    }

    /// Batched `greedy_logits` on device rows, asynchronous on `stream`.
    ///
    /// # Safety
    ///
    /// As [`CudaSampler::sample_device`] for `d_logits`, `d_ids`, `d_status`
    /// and `stream`.
    ///
    /// # Errors
    ///
    /// `CudaError` for a rejected argument or a launch failure.
    pub unsafe fn greedy_device(
        &mut self,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        d_ids: *mut u32,
        d_status: *mut i32,
        stream: *mut c_void,
    ) -> Result<(), CudaError> {
        // SAFETY: the caller's contract covers every pointer; the handle is
        // live and exclusively borrowed.
        check("rsc_greedy", unsafe {
            ffi::rsc_greedy(self.raw.as_ptr(), d_logits, rows, vocab, row_stride, d_ids, d_status, stream)
        })
    }

    /// Size of one row's vocab-shard record for `top_k`.
    #[must_use]
    pub fn shard_record_bytes(top_k: u32) -> usize {
        // SAFETY: pure function of its argument.
        unsafe { ffi::rsc_shard_record_bytes(top_k) }
    }

    /// Launches of the library's kernels since creation.
    #[must_use]
    pub fn launch_count(&self) -> u64 {
        // SAFETY: the handle is live.
        unsafe { ffi::rsc_launch_count(self.raw.as_ptr()) }
    }
}

impl Drop for CudaSampler {
    fn drop(&mut self) {
        // SAFETY: the handle came from rsc_sampler_create and is destroyed
        // exactly once; the library's cudaFree calls wait for work still
        // queued on the device before the scratch is released.
        let _ = unsafe { ffi::rsc_sampler_destroy(self.raw.as_ptr()) };
    }
}
