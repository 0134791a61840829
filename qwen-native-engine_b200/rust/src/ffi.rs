//! Raw declarations of the libqne C ABI (include/qne.h) used by this crate.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub type qne_status = i32;

#[repr(C)]
pub struct qne_model {
    _private: [u8; 0],
}

#[repr(C)]
pub struct qne_sampler {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct qne_model_info {
    pub layers: i32,
    pub hidden: i32,
    pub intermediate: i32,
    pub vocab: i32,
    pub weight_kind: i32,
    pub embed_kind: i32,
    pub tied_lm_head: i32,
    pub device: i32,
    pub weight_bytes: u64,
    pub device_bytes: u64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct qne_profile_entry {
    pub label: [c_char; 48],
    pub ms: f64,
    pub dispatches: u32,
    pub pad: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qne_sampling {
    pub temperature: f32,
    pub top_k: u32,
    pub top_p: f32,
    pub seed: u64,
    pub presence_penalty: f32,
}

pub const QNE_OK: qne_status = 0;
pub const QNE_EINVAL: qne_status = -1;
pub const QNE_ERANGE_CTX: qne_status = -2;
pub const QNE_EFORMAT: qne_status = -3;
pub const QNE_ECUDA: qne_status = -4;
pub const QNE_ETIMEOUT: qne_status = -5;
pub const QNE_ENOSNAP: qne_status = -6;
pub const QNE_ENOMEM: qne_status = -7;
pub const QNE_MAX_CONTEXT: u32 = 4096;
pub const QNE_LOAD_ANY_SHAPE: u32 = 1;

extern "C" {
    pub fn qne_last_error() -> *const c_char;
    pub fn qne_version() -> *const c_char;
    pub fn qne_model_load(
        index_json: *const c_char,
        index_len: usize,
        weights: *const c_void,
        weights_len: usize,
        device: c_int,
        out: *mut *mut qne_model,
    ) -> qne_status;
    pub fn qne_model_load_ex(
        index_json: *const c_char,
        index_len: usize,
        weights: *const c_void,
        weights_len: usize,
        device: c_int,
        flags: u32,
        out: *mut *mut qne_model,
    ) -> qne_status;
    pub fn qne_model_free(m: *mut qne_model);
    pub fn qne_model_info_get(m: *const qne_model, out: *mut qne_model_info) -> qne_status;
    pub fn qne_adapter(m: *const qne_model) -> *const c_char;
    pub fn qne_dispatches_per_token(m: *const qne_model) -> usize;
    pub fn qne_validate_tiles(tiles_json: *const c_char, len: usize) -> qne_status;
    pub fn qne_profile_token(
        m: *mut qne_model,
        out: *mut qne_profile_entry,
        cap: usize,
        n_out: *mut usize,
    ) -> qne_status;
    pub fn qne_reset(m: *mut qne_model) -> qne_status;
    pub fn qne_prefill(m: *mut qne_model, ids: *const u32, n: u32) -> qne_status;
    pub fn qne_prefill_chunk(m: *mut qne_model, ids: *const u32, n: u32, start: u32, finish_logits: c_int)
        -> qne_status;
    pub fn qne_logits(m: *mut qne_model, out: *mut f32, out_len: usize) -> qne_status;
    pub fn qne_step(m: *mut qne_model, token: u32, pos: u32, logits_out: *mut f32, out_len: usize) -> qne_status;
    pub fn qne_snapshot(m: *mut qne_model) -> qne_status;
    pub fn qne_restore(m: *mut qne_model) -> qne_status;
    pub fn qne_last_token(m: *mut qne_model, token: *mut u32, pos: *mut u32) -> qne_status;
    pub fn qne_decode(
        m: *mut qne_model,
        n: u32,
        window: u32,
        stop: *const u32,
        nstop: u32,
        ids_out: *mut u32,
        n_out: *mut u32,
    ) -> qne_status;
    pub fn qne_sampler_create(m: *mut qne_model, opts: *const qne_sampling, out: *mut *mut qne_sampler)
        -> qne_status;
    pub fn qne_sampler_free(s: *mut qne_sampler);
    pub fn qne_step_sample(
        m: *mut qne_model,
        s: *mut qne_sampler,
        token: u32,
        pos: u32,
        mask: *const u32,
        mask_tokens: u32,
        bias_token: i32,
        bias: f32,
        token_out: *mut u32,
    ) -> qne_status;
}
