//! Raw declarations of the C-ABI in `include/gpt2q.h` (libgpt2q.so).
//!
//! One `extern "C"` item per function of the header, with the header's parameter order and
//! types. The safe wrapper is the `gpt2q` crate next to this one; it restores model-lab's
//! `Gpu::new(&Engine)` / `step` / `clear_kv` (experiments/model-lab/src/gpu.rs:75,203,212).
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

pub const GPT2Q_OK: c_int = 0;
pub const GPT2Q_EARG: c_int = -1;
pub const GPT2Q_EOOM: c_int = -2;
pub const GPT2Q_ECUDA: c_int = -3;
pub const GPT2Q_ENCCL: c_int = -4;
pub const GPT2Q_ETIMEOUT: c_int = -5;
pub const GPT2Q_EUNSUP: c_int = -6;
pub const GPT2Q_NOALLOC_MAX_ROWS: c_int = 1024;

#[repr(C)]
pub struct gpt2q_handle {
    _p: [u8; 0],
}

/// Model architecture (gpt2.rs:11-19 `Meta`) plus the capacity of a handle.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct gpt2q_config {
    pub n_embd: i32,
    pub n_layer: i32,
    pub n_head: i32,
    pub n_ctx: i32,
    pub vocab: i32,
    pub ln_eps: f32,
    pub max_seqs: i32,
    pub max_tokens: i32,
}

/// One TENSORS record (format.rs:17-28 `TensorRecord`) pointing at its payload bytes.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct gpt2q_tensor_desc {
    pub name: *const c_char,
    pub atom: *const c_char,
    pub ndim: i32,
    pub shape: [i64; 2],
    pub data: *const c_void,
    pub len: u64,
}

extern "C" {
    pub fn gpt2q_create(cfg: *const gpt2q_config, t: *const gpt2q_tensor_desc, n: c_int,
                        device: c_int, out: *mut *mut gpt2q_handle) -> c_int;
    pub fn gpt2q_create_tp(cfg: *const gpt2q_config, t: *const gpt2q_tensor_desc, n: c_int, device: c_int,
                           tp_size: c_int, tp_rank: c_int, nccl_id: *const c_void,
                           out: *mut *mut gpt2q_handle) -> c_int;
    pub fn gpt2q_destroy(h: *mut gpt2q_handle);
    pub fn gpt2q_last_error(h: *const gpt2q_handle) -> *const c_char;
    pub fn gpt2q_reset_kv(h: *mut gpt2q_handle, slots: *const i32, n: c_int) -> c_int;
    pub fn gpt2q_step(h: *mut gpt2q_handle, tok: u32, pos: i32, logits: *mut f32) -> c_int;
    pub fn gpt2q_decode(h: *mut gpt2q_handle, tok: *const u32, pos: *const i32, slots: *const i32,
                        n: c_int, logits: *mut f32, next: *mut u32) -> c_int;
    pub fn gpt2q_prefill(h: *mut gpt2q_handle, toks: *const u32, offs: *const i32, slots: *const i32,
                         n: c_int, logits_last: *mut f32, next: *mut u32) -> c_int;
    pub fn gpt2q_decode_steps(h: *mut gpt2q_handle, steps: c_int, out: *mut u32) -> c_int;
    pub fn gpt2q_generate_greedy(h: *mut gpt2q_handle, toks: *const u32, offs: *const i32,
                                 n: c_int, steps: c_int, out: *mut u32) -> c_int;
    pub fn gpt2q_set_adapter(h: *mut gpt2q_handle, a: *const f32, b: *const f32, r: c_int) -> c_int;
    pub fn gpt2q_clear_adapter(h: *mut gpt2q_handle) -> c_int;
    pub fn gpt2q_nll(h: *mut gpt2q_handle, ids: *const u32, n: c_int, slot: c_int, out: *mut f64) -> c_int;
    pub fn gpt2q_dequant(h: *mut gpt2q_handle, name: *const c_char, out: *mut f32, n: u64) -> c_int;
    pub fn gpt2q_launches(h: *const gpt2q_handle) -> u64;
    pub fn gpt2q_set_stream(h: *mut gpt2q_handle, stream: *mut c_void) -> c_int;
    pub fn gpt2q_sync(h: *mut gpt2q_handle) -> c_int;
    pub fn gpt2q_profile(h: *mut gpt2q_handle, enable: c_int) -> c_int;
    pub fn gpt2q_profile_read(h: *mut gpt2q_handle, json: *mut c_char, cap: usize) -> c_int;
    pub fn gpt2q_profile_kernels(h: *mut gpt2q_handle, reps: c_int, json: *mut c_char, cap: usize) -> c_int;
    pub fn gpt2q_info(h: *mut gpt2q_handle, json: *mut c_char, cap: usize) -> c_int;
    pub fn gpt2q_argmax_noalloc(d_logits: *const f32, vocab: c_int, ld: c_int, n_rows: c_int,
                                d_next: *mut u32, stream: *mut c_void) -> c_int;
    pub fn gpt2q_rng_new(seed: u64) -> u64;
    pub fn gpt2q_quantize_q8(x: *const f32, n: usize, out: *mut u8) -> c_int;
    pub fn gpt2q_quantize_q4(x: *const f32, n: usize, out: *mut u8) -> c_int;
    pub fn gpt2q_rng_normal_f32(state: *mut u64, out: *mut f32, n: usize, stdv: f64);
    pub fn gpt2q_rng_below(state: *mut u64, out: *mut u32, n: usize, bound: u64);
    pub fn gpt2q_create_from_smt(path: *const c_char, device: c_int, max_seqs: c_int, max_tokens: c_int,
                                 verify: c_int, out: *mut *mut gpt2q_handle) -> c_int;
    pub fn gpt2q_smt_inspect(path: *const c_char, verify: c_int, json: *mut c_char, cap: usize) -> c_int;
    pub fn gpt2q_blake3(data: *const c_void, len: u64, out32: *mut u8) -> c_int;
    pub fn gpt2q_trunk_input_grad(h: *mut gpt2q_handle, ids: *const u32, n: c_int, dlogits: *const f32,
                                  dx: *mut f32, lnf_out: *mut f32) -> c_int;
    pub fn gpt2q_bwd_lin_input_grad(device: c_int, w: *const f32, dy: *const f32, rows: c_int, cols: c_int,
                                    dx: *mut f32) -> c_int;
    pub fn gpt2q_bwd_ln_backward(device: c_int, dy: *const f32, x: *const f32, g: *const f32, b: *const f32,
                                 eps: f32, n: c_int, dx: *mut f32, dg: *mut f32, db: *mut f32) -> c_int;
    pub fn gpt2q_bwd_gelu(device: c_int, x_pre: *const f32, dy: *const f32, n: c_int, dx: *mut f32) -> c_int;
    pub fn gpt2q_bwd_attn_train(device: c_int, q: *const f32, k: *const f32, v: *const f32, dy: *const f32,
                                t: c_int, hd: c_int, stride: c_int, dq: *mut f32, dk: *mut f32,
                                dv: *mut f32) -> c_int;
}
