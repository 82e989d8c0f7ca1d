// The Rust binding of include/reng_cuda.h, one to one: the file a maintainer
// adds to the reference as crates/reng-cuda/src/ffi.rs.
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

pub const RENG_OK: c_int = 0;
pub const RENG_MEM_DEVICE: c_int = 0;
pub const RENG_MEM_HOST: c_int = 1;
pub const RENG_FP8_E4M3: c_int = 0;
pub const RENG_FP8_E5M2: c_int = 1;
pub const RENG_SCALING_PCS: c_int = 0;
pub const RENG_SCALING_HW: c_int = 1;
pub const RENG_SCALING_UNIT: c_int = 2;

#[repr(C)]
pub struct reng_model { _private: [u8; 0] }

#[repr(C)]
pub struct reng_model_desc {
    pub hidden: i32, pub inter: i32, pub n_layers: i32, pub n_heads: i32,
    pub n_kv_heads: i32, pub head_dim: i32, pub vocab: i32,
    pub eps: f32, pub attn_scale: f32, pub has_qkv_bias: i32, pub weights: i32,
    pub batch: i32, pub capacity: i32, pub tp_rank: i32, pub tp_world: i32,
    pub device: i32, pub nccl_id: *const u8, pub qk_norm: i32,
}

#[repr(C)]
pub struct reng_layer_weights {
    pub wq: *const u16, pub wk: *const u16, pub wv: *const u16, pub wo: *const u16,
    pub wg: *const u16, pub wu: *const u16, pub wd: *const u16,
    pub g1: *const f32, pub g2: *const f32,
    pub bq: *const f32, pub bk: *const f32, pub bv: *const f32,
    pub qn: *const f32, pub kn: *const f32, pub no_rope: i32,
}

#[repr(C)]
pub struct reng_step_times {
    pub upload_ms: f32, pub device_ms: f32, pub readback_ms: f32,
    pub steps: i32, pub kernels_per_step: i32,
}

#[repr(C)]
pub struct reng_device_info {
    pub ordinal: i32, pub name: [c_char; 96], pub pci_bus_id: [c_char; 32],
    pub total_bytes: u64, pub sm_count: i32, pub cc_major: i32, pub cc_minor: i32,
}

#[link(name = "reng_cuda")]
extern "C" {
    pub fn reng_last_error() -> *const c_char;
    pub fn reng_version() -> c_int;
    pub fn reng_device_count(count: *mut c_int) -> c_int;
    pub fn reng_device_info_get(device: c_int, out: *mut reng_device_info) -> c_int;
    pub fn reng_fp8_encode(x: *const f32, n: i64, fmt: c_int, codes: *mut u8, stream: *mut c_void) -> c_int;
    pub fn reng_fp8_decode(codes: *const u8, n: i64, fmt: c_int, out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn reng_model_last_times(m: *const reng_model, t: *mut reng_step_times) -> c_int;
    pub fn reng_fp8_quantize(w: *const u16, rows: i64, cols: i64, fmt: c_int, scaling: c_int,
                             backoff: f32, codes: *mut u8, scales: *mut f32, exp_bias: *mut u32,
                             mem: c_int, stream: *mut c_void) -> c_int;
    pub fn reng_fp8_quantize_noalloc(w: *const u16, rows: i64, cols: i64, fmt: c_int,
                                     scaling: c_int, backoff: f32, codes: *mut u8,
                                     scales: *mut f32, exp_bias: *mut u32,
                                     stream: *mut c_void) -> c_int;
    pub fn reng_model_create(desc: *const reng_model_desc, layers: *const reng_layer_weights,
                             embed: *const u16, lm_head: *const u16, final_gamma: *const f32,
                             rope_sin: *const f32, rope_cos: *const f32, mem: c_int,
                             out: *mut *mut reng_model) -> c_int;
    pub fn reng_model_destroy(m: *mut reng_model) -> c_int;
    pub fn reng_model_prefill(m: *mut reng_model, slot: c_int, ids: *const u32, n: c_int,
                              next_id: *mut u32, last_logits: *mut f32,
                              all_logits: *mut f32) -> c_int;
    pub fn reng_model_decode(m: *mut reng_model, seeds: *const u32, n: c_int,
                             ids_out: *mut u32) -> c_int;
    pub fn reng_model_step_logits(m: *mut reng_model, ids: *const u32, logits: *mut f32,
                                  next_ids: *mut u32) -> c_int;
    pub fn reng_model_reset(m: *mut reng_model, slot: c_int) -> c_int;
    pub fn reng_model_position(m: *const reng_model, slot: c_int, pos: *mut c_int) -> c_int;
    pub fn reng_model_decode_device(m: *mut reng_model, seeds: *const u32, n: c_int,
                                    ids_out: *mut u32, stream: *mut c_void) -> c_int;
    pub fn reng_model_device_bytes(m: *const reng_model, bytes: *mut u64) -> c_int;
    pub fn reng_model_time_kernels(m: *mut reng_model, iters: c_int, ms_out: *mut f32) -> c_int;
    pub fn reng_model_time_kernels_rows(m: *mut reng_model, rows: c_int, iters: c_int, ms_out: *mut f32) -> c_int;
    pub fn reng_gemm_bf16(w: *const u16, rows: c_int, k: c_int, x: *const u16, m: c_int, y: *mut f32,
                          splits: c_int, iters: c_int, ms_out: *mut f32, mem: c_int) -> c_int;
    pub fn reng_tp_unique_id(out: *mut u8) -> c_int;
    pub fn reng_model_tp_exchange(m: *mut reng_model, kind: *mut c_int) -> c_int;
    pub fn reng_model_time_exchange(m: *mut reng_model, iters: c_int, ms_out: *mut f32) -> c_int;
    pub fn reng_tp_peer_wait_check(device: c_int) -> c_int;
}
