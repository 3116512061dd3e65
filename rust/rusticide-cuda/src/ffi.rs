//! Raw declarations of include/rusticide_cuda.h (ABI version 1).
//!
//! Every function is asynchronous on the `stream` it is given (a
//! `cudaStream_t`, null for the legacy default stream) except
//! `rsc_pick_host`, which returns after its host outputs are written.

use std::ffi::{c_char, c_int, c_void};

pub(crate) const RSC_ABI_VERSION: c_int = 2;

pub(crate) const RSC_OK: c_int = 0;
pub(crate) const RSC_ERR_INVALID_SHAPE: c_int = 2;
pub(crate) const RSC_ERR_VOCAB_TOO_LARGE: c_int = 3;

pub(crate) const RSC_ROW_OK: i32 = 0;
pub(crate) const RSC_ROW_NO_VALID_TOKENS: i32 = 1;
pub(crate) const RSC_ROW_VOCAB_OVERFLOW: i32 = 2;
pub(crate) const RSC_ROW_INTERNAL: i32 = 3;
pub(crate) const RSC_ROW_CODE_MASK: i32 = 0xff;

/// rsc_peer_exchange: device addresses of the arrays the ranks share.
#[repr(C)]
pub(crate) struct RscPeerExchange {
    pub d_peer_records: *const *const c_void,
    pub d_ready_records: *const u32,
    pub d_ready_results_ptrs: *const *mut u32,
    pub d_done_counter: *mut u32,
    pub d_peer_ids: *const *mut u32,
    pub d_peer_status: *const *mut i32,
    pub d_peer_probs: *const *mut f32,
}

/// `rsc_params`: `SamplingParams` field for field
/// (crates/rusticide-sampling/src/params.rs:5-12).
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct RscParams {
    pub(crate) temperature: f32,
    pub(crate) top_k: u32,
    pub(crate) top_p: f32,
    pub(crate) repetition_penalty: f32,
    pub(crate) seed: u64,
}

/// `rsc_sample_extras`.
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct RscSampleExtras {
    pub(crate) d_n_survivors: *mut u32,
    pub(crate) d_survivor_ids: *mut u32,
    pub(crate) survivor_cap: usize,
    pub(crate) d_survivor_probs: *mut f32,
    pub(crate) d_row_logsumexp: *mut f32,
    pub(crate) d_token_logprob: *mut f32,
    pub(crate) d_survivor_logprobs: *mut f32,
}

/// Opaque `rsc_sampler`.
#[repr(C)]
pub(crate) struct RscSampler {
    _private: [u8; 0],
}

unsafe extern "C" {
    pub(crate) fn rsc_status_string(status: c_int) -> *const c_char;
    pub(crate) fn rsc_abi_version() -> c_int;
    pub(crate) fn rsc_sampler_create(
        device: c_int,
        max_rows: usize,
        max_vocab: usize,
        out: *mut *mut RscSampler,
    ) -> c_int;
    pub(crate) fn rsc_sampler_destroy(sampler: *mut RscSampler) -> c_int;
    pub(crate) fn rsc_sample(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_sample_rows(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        h_params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_sample_ex(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        extras: *const RscSampleExtras,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_greedy(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_sample_with_temp(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        temperature: f32,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_pick(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_pick_host(
        sampler: *mut RscSampler,
        h_logits: *const f32,
        rows: usize,
        vocab: usize,
        params: *const RscParams,
        h_uniforms: *const f32,
        h_out_ids: *mut u32,
        h_out_status: *mut i32,
        h_out_probs: *mut f32,
    ) -> c_int;
    pub(crate) fn rsc_penalize(
        sampler: *mut RscSampler,
        d_logits: *mut f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        d_tokens: *const u32,
        n_tokens: usize,
        penalty: f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_rng_seed(
        d_seeds: *const u64,
        d_rng_states: *mut u64,
        rows: usize,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_shard_record_bytes(top_k: u32) -> usize;
    pub(crate) fn rsc_shard_partial(
        sampler: *mut RscSampler,
        d_logits: *const f32,
        rows: usize,
        shard_vocab: usize,
        row_stride: usize,
        shard_offset: usize,
        global_vocab: usize,
        params: *const RscParams,
        d_records: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_shard_merge(
        sampler: *mut RscSampler,
        d_records: *const c_void,
        n_shards: usize,
        rows: usize,
        global_vocab: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_sample_noalloc(
        d_logits: *const f32,
        rows: usize,
        vocab: usize,
        row_stride: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_lmhead_logits(
        sampler: *mut RscSampler,
        d_hidden: *const c_void,
        d_weight: *const c_void,
        rows: usize,
        dim: usize,
        vocab: usize,
        d_logits: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_lmhead_sample(
        sampler: *mut RscSampler,
        d_hidden: *const c_void,
        d_weight: *const c_void,
        rows: usize,
        dim: usize,
        vocab: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_lmhead_partial(
        sampler: *mut RscSampler,
        d_hidden: *const c_void,
        d_weight_shard: *const c_void,
        rows: usize,
        dim: usize,
        shard_vocab: usize,
        shard_offset: usize,
        global_vocab: usize,
        params: *const RscParams,
        d_records: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_expf(d_x: *const f32, d_y: *mut f32, n: usize, stream: *mut c_void) -> c_int;
    pub(crate) fn rsc_shard_merge_peers(
        sampler: *mut RscSampler,
        exchange: *const RscPeerExchange,
        step: u32,
        n_shards: usize,
        my_shard: usize,
        rows: usize,
        global_vocab: usize,
        params: *const RscParams,
        d_uniforms: *const f32,
        d_rng_states: *mut u64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_shard_collect(
        d_ready_results: *const u32,
        step: u32,
        n_shards: usize,
        rows: usize,
        d_ids: *const u32,
        d_status: *const i32,
        d_probs: *const f32,
        d_out_ids: *mut u32,
        d_out_status: *mut i32,
        d_out_probs: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_shard_publish(
        d_ready_ptrs: *const *mut u32,
        n_shards: usize,
        my_shard: usize,
        step: u32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn rsc_launch_count(sampler: *const RscSampler) -> u64;
    pub(crate) fn rsc_debug_hold_scratch(
        sampler: *mut RscSampler,
        hold: c_int,
        stream: *mut c_void,
    ) -> c_int;
}
