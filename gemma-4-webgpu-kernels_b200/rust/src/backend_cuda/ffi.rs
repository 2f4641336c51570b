//! Raw bindings of libgq (include/gq.h), one declaration per entry point, same
//! order of arguments. Every function returns a gq_status (0 = OK) except the
//! accessors that return a pointer or a count. Pointers named `*_dev`, `x`, `y`,
//! `out`, `ids`, `flags` … are device pointers; `*_host` and the upload payloads
//! are host pointers (copied before the call returns).
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

#[repr(C)]
pub struct GqCtx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct GqQWeight {
    _p: [u8; 0],
}
#[repr(C)]
pub struct GqGraph {
    _p: [u8; 0],
}
#[repr(C)]
pub struct GqStFile {
    _p: [u8; 0],
}
#[repr(C)]
pub struct GqChain {
    _p: [u8; 0],
}
/// gq_chain_op: one one-row MATMUL_Q call of a decode chain (mode 0 linear,
/// 1 linear_geglu with `w2` = up, 2 linear_gelu_mul_cols over `b[b_offset..]`,
/// 3 soft-capped linear).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct GqChainOp {
    pub mode: i32,
    pub w: *const GqQWeight,
    pub w2: *const GqQWeight,
    pub x: *const f32,
    pub y: *mut f32,
    pub b: *const f32,
    pub b_offset: i64,
    pub cap: f32,
}
/// gq_sample_opts: the fields of the reference's SampleOpts (src/sampler.rs:29-39).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct GqSampleOpts {
    pub temperature: f32,
    pub top_k: i32,
    pub top_p: f32,
    pub repetition_penalty: f32,
}

pub const GQ_OK: c_int = 0;
pub const GQ_ERR_INVALID_ARGUMENT: c_int = 1;
pub const GQ_ERR_UNSUPPORTED: c_int = 2;
pub const GQ_ERR_CUDA: c_int = 3;
pub const GQ_ERR_OUT_OF_MEMORY: c_int = 4;
pub const GQ_ERR_DEVICE: c_int = 5;
pub const GQ_DEVERR_BAD_ID: u32 = 0x1;
pub const GQ_DEVERR_WAIT_TIMEOUT: u32 = 0x2;
pub const GQ_DEVERR_SAMPLE_CAP: u32 = 0x4;
pub const GQ_ATTN_KPOS_ASCENDING: u32 = 0x1;
pub const GQ_ATTN_KPOS_IDENTITY: u32 = 0x2;

extern "C" {
    pub fn gq_abi_version() -> c_int;
    pub fn gq_status_string(status: c_int) -> *const c_char;
    // context (WgpuBackend::create, rust/src/backend_wgpu.rs:239-300)
    pub fn gq_ctx_create(device: c_int, out: *mut *mut GqCtx) -> c_int;
    pub fn gq_ctx_destroy(ctx: *mut GqCtx) -> c_int;
    pub fn gq_ctx_set_stream(ctx: *mut GqCtx, cuda_stream: *mut c_void) -> c_int;
    pub fn gq_ctx_get_stream(ctx: *mut GqCtx) -> *mut c_void;
    pub fn gq_ctx_num_sms(ctx: *mut GqCtx) -> c_int;
    pub fn gq_ctx_set_wait_limit(ctx: *mut GqCtx, limit_ns: u64) -> c_int;
    // decode chains: consecutive one-row linear calls in one persistent launch
    pub fn gq_chain_create(ctx: *mut GqCtx, ops: *const GqChainOp, n_ops: i32, out: *mut *mut GqChain) -> c_int;
    pub fn gq_chain_run(chain: *mut GqChain) -> c_int;
    pub fn gq_chain_reset(chain: *mut GqChain) -> c_int;
    pub fn gq_chain_destroy(chain: *mut GqChain) -> c_int;
    pub fn gq_last_error(ctx: *mut GqCtx) -> *const c_char;
    // sync / memory (Backend::{tensor, zeros, readback, flush, free_tensor})
    pub fn gq_sync(ctx: *mut GqCtx) -> c_int;
    pub fn gq_alloc(ctx: *mut GqCtx, bytes: usize, dptr: *mut *mut c_void) -> c_int;
    pub fn gq_free(ctx: *mut GqCtx, dptr: *mut c_void) -> c_int;
    pub fn gq_memcpy_h2d(ctx: *mut GqCtx, dst_dev: *mut c_void, src_host: *const c_void, bytes: usize) -> c_int;
    pub fn gq_memcpy_d2h(ctx: *mut GqCtx, dst_host: *mut c_void, src_dev: *const c_void, bytes: usize) -> c_int;
    pub fn gq_memset(ctx: *mut GqCtx, dst_dev: *mut c_void, value: c_int, bytes: usize) -> c_int;
    pub fn gq_readback(ctx: *mut GqCtx, dst_host: *mut f32, src_dev: *const f32, count: usize) -> c_int;
    // weights (Backend::quant_tensor)
    pub fn gq_qweight_upload(ctx: *mut GqCtx, qbytes: *const u8, nbytes: usize, scales: *const f32,
        nscales: usize, n: i64, k: i64, bits: i32, signed_i8: i32, group_size: i64,
        out: *mut *mut GqQWeight) -> c_int;
    pub fn gq_qweight_upload_device(ctx: *mut GqCtx, qbytes_dev: *const u8, nbytes: usize, scales: *const f32,
        nscales: usize, n: i64, k: i64, bits: i32, signed_i8: i32, group_size: i64,
        out: *mut *mut GqQWeight) -> c_int;
    pub fn gq_qweight_free(w: *mut GqQWeight) -> c_int;
    pub fn gq_qweight_info(w: *const GqQWeight, n: *mut i64, k: *mut i64, bits: *mut i32, signed_i8: *mut i32,
        group_size: *mut i64) -> c_int;
    // record / replay (the recorded command encoder, rust/src/backend_wgpu.rs:11-15)
    pub fn gq_graph_begin(ctx: *mut GqCtx) -> c_int;
    pub fn gq_graph_end(ctx: *mut GqCtx, out: *mut *mut GqGraph) -> c_int;
    pub fn gq_graph_launch(ctx: *mut GqCtx, graph: *mut GqGraph) -> c_int;
    pub fn gq_graph_destroy(graph: *mut GqGraph) -> c_int;
    // quantized linear family (MATMUL_Q MODE 0/1/2 and the fused lm_head soft-cap)
    pub fn gq_linear(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const GqQWeight, y: *mut f32) -> c_int;
    pub fn gq_linear_geglu(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, wg: *const GqQWeight,
        wu: *const GqQWeight, y: *mut f32) -> c_int;
    pub fn gq_linear_gelu_mul_cols(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const GqQWeight,
        b: *const f32, b_stride: i64, b_offset: i64, y: *mut f32) -> c_int;
    pub fn gq_linear_softcap(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const GqQWeight, cap: f32,
        y: *mut f32, ldy: i64, y_col0: i64) -> c_int;
    // vocab-sharded lm_head: the exchange fused into the shard GEMV, its completion flags, CUDA IPC
    pub fn gq_linear_softcap_peers(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const GqQWeight, cap: f32,
        y: *mut f32, ldy: i64, y_col0: i64, peer_y: *const *mut f32, npeers: i32) -> c_int;
    pub fn gq_linear_softcap_peers_signal(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const GqQWeight,
        cap: f32, y: *mut f32, ldy: i64, y_col0: i64, peer_y: *const *mut f32, npeers: i32,
        flags: *const *mut u32, sync: *mut u32, rank: i32) -> c_int;
    pub fn gq_linear_softcap_peers_sync(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const GqQWeight,
        cap: f32, y: *mut f32, ldy: i64, y_col0: i64, peer_y: *const *mut f32, npeers: i32,
        flags: *const *mut u32, sync: *mut u32, rank: i32) -> c_int;
    pub fn gq_peer_wait(ctx: *mut GqCtx, flags: *const u32, world: i32, sync: *const u32) -> c_int;
    pub fn gq_argmax_rows(ctx: *mut GqCtx, x: *const f32, m: i64, n: i64, ldx: i64, idx_base: i64,
        val: *mut f32, idx: *mut i64) -> c_int;
    // sampling on the device (src/sampler.rs:116-190) and the sharded candidate exchange
    pub fn gq_sample_rows(ctx: *mut GqCtx, logits: *const f32, m: i64, vocab: i64, ld: i64,
        opts: *const GqSampleOpts, recent: *const u32, n_recent: i64, recent_stride: i64,
        rng_state: *mut u64, tokens: *mut i32) -> c_int;
    pub fn gq_topk_rows(ctx: *mut GqCtx, logits: *const f32, m: i64, n: i64, ld: i64, idx_base: i64, k: i32,
        repetition_penalty: f32, recent: *const u32, n_recent: i64, recent_stride: i64, val: *mut f32,
        idx: *mut i64) -> c_int;
    pub fn gq_sample_candidates(ctx: *mut GqCtx, val: *const f32, idx: *const i64, m: i64, ncand: i64,
        opts: *const GqSampleOpts, rng_state: *mut u64, tokens: *mut i32) -> c_int;
    pub fn gq_ipc_get_handle(ctx: *mut GqCtx, dptr: *mut c_void, handle64: *mut u8) -> c_int;
    pub fn gq_ipc_open(ctx: *mut GqCtx, handle64: *const u8, dptr: *mut *mut c_void) -> c_int;
    pub fn gq_ipc_close(ctx: *mut GqCtx, dptr: *mut c_void) -> c_int;
    // checkpoint loading (src/safetensors.rs, src/weights.rs:37-118 restated in libgq)
    pub fn gq_st_open(path: *const c_char, out: *mut *mut GqStFile) -> c_int;
    pub fn gq_st_open_memory(bytes: *const u8, nbytes: usize, out: *mut *mut GqStFile) -> c_int;
    pub fn gq_st_close(f: *mut GqStFile) -> c_int;
    pub fn gq_st_count(f: *const GqStFile) -> i64;
    pub fn gq_st_name(f: *const GqStFile, i: i64) -> *const c_char;
    pub fn gq_st_info(f: *const GqStFile, name: *const c_char, dtype16: *mut c_char, shape8: *mut i64,
        ndim: *mut i32, data: *mut *const u8, nbytes: *mut usize) -> c_int;
    pub fn gq_st_read_f32(f: *const GqStFile, name: *const c_char, dst_host: *mut f32, count: usize) -> c_int;
    pub fn gq_bits_for(name: *const c_char, patterns: *const *const c_char, bits: *const i32, nrules: i32) -> i32;
    pub fn gq_st_resolve(logical: *const c_char, weight256: *mut c_char, scale256: *mut c_char,
        bare256: *mut c_char) -> c_int;
    pub fn gq_st_upload_quant(ctx: *mut GqCtx, f: *const GqStFile, logical: *const c_char, bits_u8: i32,
        out: *mut *mut GqQWeight) -> c_int;
    // EMBED_Q (Backend::embed_rows on a quantized table)
    pub fn gq_embed_rows(ctx: *mut GqCtx, table: *const GqQWeight, ids: *const u32, t: i64, scale: f32,
        out: *mut f32) -> c_int;
    // callers that cannot allocate: the prefill linear with library-owned scratch, and its status word
    pub fn gq_linear_prefill_static(cuda_stream: *mut c_void, x: *const f32, m: i64, k: i64, qbytes: *const u8,
        scales: *const f32, n: i64, bits: i32, signed_i8: i32, y: *mut f32) -> c_int;
    pub fn gq_linear_prefill_static_status(cuda_stream: *mut c_void, status_bits: *mut u32) -> c_int;
    // elementwise (Backend::softcap / geglu)
    pub fn gq_softcap(ctx: *mut GqCtx, x: *const f32, n: i64, cap: f32, y: *mut f32) -> c_int;
    pub fn gq_geglu(ctx: *mut GqCtx, gate: *const f32, up: *const f32, n: i64, y: *mut f32) -> c_int;
    // support ops of a decode step (rust/src/backend.rs:103-154)
    pub fn gq_rms_norm(ctx: *mut GqCtx, x: *const f32, rows: i64, d: i64, w: *const f32, eps: f32,
        y: *mut f32, y_stride: i64) -> c_int;
    pub fn gq_add_rms_norm(ctx: *mut GqCtx, residual: *const f32, x: *const f32, rows: i64, d: i64,
        w: *const f32, eps: f32, scale_by: *const f32, y: *mut f32) -> c_int;
    pub fn gq_add_rms_norm_norm(ctx: *mut GqCtx, residual: *const f32, x: *const f32, rows: i64, d: i64,
        w1: *const f32, eps: f32, scale_by: *const f32, w2: *const f32, h: *mut f32, xn: *mut f32) -> c_int;
    // one decode row: residual add + RMSNorm fused into the projection that reads it
    pub fn gq_add_norm_linear(ctx: *mut GqCtx, mode: i32, x: *const f32, residual: *const f32, k: i64,
        w_norm: *const f32, eps: f32, scale_by: *const f32, w_norm2: *const f32, h_out: *mut f32,
        w: *const GqQWeight, w_up: *const GqQWeight, b: *const f32, b_offset: i64, y: *mut f32) -> c_int;
    pub fn gq_head_norm_rope(ctx: *mut GqCtx, x: *const f32, t: i64, heads: i64, head_dim: i64, w: *const f32,
        eps: f32, positions: *const u32, theta: f32, rotary_dim: i64, y: *mut f32, y_tok_stride: i64) -> c_int;
    pub fn gq_qkv_norm_rope(ctx: *mut GqCtx, qkv: *const f32, t: i64, qkv_tok_stride: i64, hq: i64, hkv: i64,
        head_dim: i64, q_w: *const f32, k_w: *const f32, eps: f32, positions: *const u32, theta: f32,
        rotary_dim: i64, q_out: *mut f32, q_tok_stride: i64, k_out: *mut f32, k_tok_stride: i64,
        v_out: *mut f32, v_tok_stride: i64) -> c_int;
    pub fn gq_rope(ctx: *mut GqCtx, x: *const f32, t: i64, heads: i64, head_dim: i64, positions: *const u32,
        theta: f32, rotary_dim: i64, y: *mut f32, y_tok_stride: i64) -> c_int;
    pub fn gq_attention(ctx: *mut GqCtx, q: *const f32, batch: i64, t: i64, hq: i64, head_dim: i64,
        k: *const f32, v: *const f32, s: i64, hkv: i64, kv_batch_stride: i64, q_pos: *const u32,
        k_pos: *const u32, kpos_batch_stride: i64, scale: f32, sliding_window: u32, attn_softcap: f32,
        flags: u32, out: *mut f32) -> c_int;
    pub fn gq_linear_bf16(ctx: *mut GqCtx, x: *const f32, m: i64, k: i64, w: *const u16, n: i64, y: *mut f32) -> c_int;
    pub fn gq_add(ctx: *mut GqCtx, a: *const f32, b: *const f32, n: i64, y: *mut f32) -> c_int;
    pub fn gq_mul(ctx: *mut GqCtx, a: *const f32, b: *const f32, n: i64, y: *mut f32) -> c_int;
    pub fn gq_scale(ctx: *mut GqCtx, a: *const f32, n: i64, s: f32, y: *mut f32) -> c_int;
    pub fn gq_scale_by_tensor(ctx: *mut GqCtx, a: *const f32, n: i64, s: *const f32, y: *mut f32) -> c_int;
    pub fn gq_copy_rows(ctx: *mut GqCtx, src: *const f32, rows: i64, cols: i64, src_stride: i64,
        dst: *mut f32, dst_stride: i64) -> c_int;
}
