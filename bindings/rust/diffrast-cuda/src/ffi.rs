//! Raw bindings to include/diffrast_cuda.h, one declaration per DR_API export.
//! Pointers are device memory unless the C header says host; `stream` is a
//! cudaStream_t (null: the legacy default stream).

#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_double, c_float, c_int, c_void};

#[repr(C)]
pub struct dr_ctx {
    _private: [u8; 0],
}

pub type dr_status = c_int;
pub type dr_stream_t = *mut c_void;

pub const DR_OK: dr_status = 0;
pub const DR_INVALID_ARGUMENT: dr_status = 1;
pub const DR_TOO_LARGE: dr_status = 2;
pub const DR_NO_DEVICE: dr_status = 3;
pub const DR_TIMEOUT: dr_status = 4;
pub const DR_LAUNCH: dr_status = 5;
pub const DR_COMM: dr_status = 6;
pub const DR_OUT_OF_MEMORY: dr_status = 7;
pub const DR_INTERNAL: dr_status = 8;

pub const DR_LAYOUT_BHWC: c_int = 0;
pub const DR_LAYOUT_BCHW: c_int = 1;

pub const DR_PRECISION_REFERENCE: c_int = 0;
pub const DR_PRECISION_STRICT: c_int = 1;
pub const DR_PRECISION_FAST: c_int = 2;

pub const DR_PATH_TILE: c_int = 0;
pub const DR_PATH_REGION: c_int = 1;
pub const DR_PATH_SPLIT: c_int = 2;
pub const DR_PATH_TILE_GATHER: c_int = 3;

pub const DR_BACKWARD_TAPED: c_int = 0;
pub const DR_BACKWARD_RECOMPUTE: c_int = 1;

pub const DR_REDUCE_DIRECT: c_int = 0;
pub const DR_REDUCE_WORKGROUP: c_int = 1;

pub const DR_STOP_COMPLETED: c_int = 0;
pub const DR_STOP_CONVERGED: c_int = 1;
pub const DR_STOP_DIVERGED: c_int = 2;

pub const DR_HOST_CHUNKS_MAX: usize = 5;
pub const DR_TRIANGLE_BLOCK_STATE_BYTES: usize = 32;
pub const DR_NOALLOC_MAX_TRIANGLES: i64 = 16384;
pub const DR_NOALLOC_MAX_BATCH: i64 = 1024;
pub const DR_NOALLOC_MAX_TILES: i64 = 65536;

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct dr_fit_config {
    pub iters: i64,
    pub sigma_start: c_float,
    pub sigma_end: c_float,
    pub lr_pos: c_float,
    pub lr_color: c_float,
    pub lr_alpha: c_float,
    pub patience: i64,
    pub min_delta: c_float,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct dr_fit_report {
    pub n_losses: i64,
    pub best_iter: i64,
    pub best_loss: c_float,
    pub stop_reason: c_int,
    pub config_error: c_int,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct dr_pool_stats {
    pub hits: u64,
    pub misses: u64,
    pub bytes: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct dr_backward_timings {
    pub pack_ms: c_float,
    pub alloc_ms: c_float,
    pub dispatch_ms: c_float,
    pub readback_ms: c_float,
    pub loss_ms: c_float,
}

extern "C" {
    pub fn dr_ctx_create(device: c_int, out: *mut *mut dr_ctx) -> dr_status;
    pub fn dr_ctx_destroy(ctx: *mut dr_ctx) -> dr_status;
    pub fn dr_last_error() -> *const c_char;
    pub fn dr_status_string(s: dr_status) -> *const c_char;
    pub fn dr_params_per_triangle() -> c_int;
    pub fn dr_version() -> *const c_char;
    pub fn dr_device_name(device: c_int, buf: *mut c_char, len: usize) -> dr_status;
    pub fn dr_device_count() -> c_int;
    pub fn dr_set_background_location(ctx: *mut dr_ctx, on_device: c_int) -> dr_status;
    pub fn dr_set_precision(ctx: *mut dr_ctx, precision: c_int) -> dr_status;
    pub fn dr_set_triangle_split(ctx: *mut dr_ctx, blocks: c_int) -> dr_status;
    pub fn dr_query_path(ctx: *mut dr_ctx, b: c_int, t: c_int, h: c_int, w: c_int,
                         path: *mut c_int) -> dr_status;

    pub fn dr_render(ctx: *mut dr_ctx, params: *const c_float, background: *const c_float,
                     bg_per_scene: c_int, b: c_int, t: c_int, h: c_int, w: c_int,
                     sigma: c_float, layout: c_int, image: *mut c_float,
                     stream: dr_stream_t) -> dr_status;
    pub fn dr_loss_backward(ctx: *mut dr_ctx, params: *const c_float,
                            background: *const c_float, bg_per_scene: c_int, b: c_int,
                            t: c_int, h: c_int, w: c_int, sigma: c_float,
                            targets: *const c_float, layout: c_int, grads: *mut c_float,
                            losses: *mut c_float, image: *mut c_float,
                            stream: dr_stream_t) -> dr_status;
    pub fn dr_loss_backward_host(ctx: *mut dr_ctx, params: *const c_float,
                                 background: *const c_float, bg_per_scene: c_int, b: c_int,
                                 t: c_int, h: c_int, w: c_int, sigma: c_float,
                                 targets: *const c_float, layout: c_int, grads: *mut c_float,
                                 losses: *mut c_float, stream: dr_stream_t) -> dr_status;
    pub fn dr_host_chunks(b: c_int, lo: *mut c_int, hi: *mut c_int) -> c_int;
    pub fn dr_grad_backward(ctx: *mut dr_ctx, params: *const c_float,
                            background: *const c_float, bg_per_scene: c_int, b: c_int,
                            t: c_int, h: c_int, w: c_int, sigma: c_float,
                            grad_images: *const c_float, layout: c_int, grads: *mut c_float,
                            stream: dr_stream_t) -> dr_status;
    pub fn dr_loss_backward_sharded(ctx: *mut dr_ctx, params: *const c_float,
                                    background: *const c_float, bg_per_scene: c_int, b: c_int,
                                    t: c_int, h: c_int, w: c_int, sigma: c_float,
                                    targets: *const c_float, layout: c_int, shard: c_int,
                                    n_shards: c_int, grads: *mut c_float,
                                    loss_sums: *mut c_double, stream: dr_stream_t) -> dr_status;
    pub fn dr_triangle_block_forward(ctx: *mut dr_ctx, params: *const c_float,
                                     background: *const c_float, bg_per_scene: c_int, b: c_int,
                                     t: c_int, h: c_int, w: c_int, sigma: c_float,
                                     n_blocks: c_int, block: c_int, state: *mut c_float,
                                     stream: dr_stream_t) -> dr_status;
    pub fn dr_triangle_block_backward(ctx: *mut dr_ctx, params: *const c_float,
                                      background: *const c_float, bg_per_scene: c_int,
                                      b: c_int, t: c_int, h: c_int, w: c_int, sigma: c_float,
                                      n_blocks: c_int, block: c_int, state: *const c_float,
                                      other: *const c_float, layout: c_int, grad_input: c_int,
                                      grads: *mut c_float, losses: *mut c_float,
                                      image: *mut c_float, stream: dr_stream_t) -> dr_status;
    pub fn dr_mse_loss(ctx: *mut dr_ctx, images: *const c_float, targets: *const c_float,
                       b: c_int, n_per_image: i64, losses: *mut c_float,
                       stream: dr_stream_t) -> dr_status;
    pub fn dr_adam_step(ctx: *mut dr_ctx, params: *mut c_float, m: *mut c_float,
                        v: *mut c_float, grads: *const c_float, n: i64, lr_pos: c_float,
                        lr_color: c_float, lr_alpha: c_float, step: u32, beta1: c_float,
                        beta2: c_float, eps: c_float, project: c_int,
                        stream: dr_stream_t) -> dr_status;
    pub fn dr_fit(ctx: *mut dr_ctx, target: *const c_float, h: c_int, w: c_int,
                  init_params: *const c_float, background: *const c_float, t: c_int,
                  cfg: *const dr_fit_config, best_params: *mut c_float,
                  final_params: *mut c_float, losses: *mut c_float,
                  report: *mut dr_fit_report, stream: dr_stream_t) -> dr_status;
    pub fn dr_loss_backward_noalloc(params: *const c_float, background: *const c_float,
                                    b: c_int, t: c_int, h: c_int, w: c_int, sigma: c_float,
                                    targets: *const c_float, layout: c_int,
                                    grads: *mut c_float, losses: *mut c_float,
                                    stream: dr_stream_t) -> dr_status;
    pub fn dr_backward(ctx: *mut dr_ctx, params: *const c_float, background: *const c_float,
                       t: c_int, h: c_int, w: c_int, sigma: c_float, target: *const c_float,
                       layout: c_int, mode: c_int, grads: *mut c_float, loss: *mut c_float,
                       image: *mut c_float, stream: dr_stream_t) -> dr_status;
    pub fn dr_set_reduce_mode(ctx: *mut dr_ctx, mode: c_int) -> dr_status;
    pub fn dr_get_reduce_mode(ctx: *mut dr_ctx, mode: *mut c_int) -> dr_status;
    pub fn dr_set_deterministic(ctx: *mut dr_ctx, on: c_int) -> dr_status;
    pub fn dr_pixel_tape_bytes(b: c_int, height: c_int, width: c_int) -> u64;
    pub fn dr_render_taped(ctx: *mut dr_ctx, params: *const c_float, background: *const c_float,
                           bg_per_scene: c_int, b: c_int, t: c_int, height: c_int, width: c_int,
                           sigma: c_float, layout: c_int, image: *mut c_float, tape: *mut c_void,
                           stream: dr_stream_t) -> dr_status;
    pub fn dr_grad_backward_taped(ctx: *mut dr_ctx, params: *const c_float,
                                  background: *const c_float, bg_per_scene: c_int, b: c_int,
                                  t: c_int, height: c_int, width: c_int, sigma: c_float,
                                  grad_images: *const c_float, layout: c_int,
                                  tape: *const c_void, grads: *mut c_float,
                                  stream: dr_stream_t) -> dr_status;
    pub fn dr_get_deterministic(ctx: *mut dr_ctx, on: *mut c_int) -> dr_status;
    pub fn dr_loss_backward_timed(ctx: *mut dr_ctx, params: *const c_float,
                                  background: *const c_float, bg_per_scene: c_int, b: c_int,
                                  t: c_int, h: c_int, w: c_int, sigma: c_float,
                                  targets: *const c_float, layout: c_int, grads: *mut c_float,
                                  losses: *mut c_float, timings: *mut dr_backward_timings,
                                  stream: dr_stream_t) -> dr_status;
    pub fn dr_tape_bytes(n_tris: u64, width: u64, height: u64) -> u64;
    pub fn dr_scratch_bytes(ctx: *mut dr_ctx, b: c_int, t: c_int, h: c_int, w: c_int) -> u64;
    pub fn dr_is_discrete(device: c_int) -> c_int;
    pub fn dr_device_alloc(ctx: *mut dr_ctx, bytes: usize, out: *mut *mut c_void) -> dr_status;
    pub fn dr_device_free(ctx: *mut dr_ctx, ptr: *mut c_void) -> dr_status;
    pub fn dr_memcpy(ctx: *mut dr_ctx, dst: *mut c_void, src: *const c_void, bytes: usize,
                     stream: dr_stream_t) -> dr_status;
    pub fn dr_pool_stats_get(ctx: *mut dr_ctx, out: *mut dr_pool_stats) -> dr_status;
    pub fn dr_clear_pool(ctx: *mut dr_ctx) -> dr_status;
    pub fn dr_stream_wait(stream: dr_stream_t, timeout_s: c_double) -> dr_status;
}
