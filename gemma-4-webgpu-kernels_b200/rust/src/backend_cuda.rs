//! `CudaBackend`: the `Backend` trait (rust/src/backend.rs:88-180) on B200 through
//! libgq's C ABI (include/gq.h, bindings in `backend_cuda/ffi.rs`).
//!
//! Drop this file and the `backend_cuda/` directory into the reference crate's
//! `src/`, add `pub mod backend_cuda;` to `src/lib.rs` and the build script
//! `build.rs` beside `Cargo.toml`; `Gemma4Model<CudaBackend, _>` then runs the
//! unchanged graph (rust/src/model.rs) on the GPU. Conventions kept from the wgpu
//! backend:
//!  * methods take `&self` and are infallible: a non-zero libgq status panics
//!    with the library's message (the trait has no error channel);
//!  * ops are enqueued on the context's stream and return at once; only
//!    `readback` blocks (rust/src/backend_wgpu.rs:1-6);
//!  * the backend is single-threaded (`!Sync`), like the wgpu one
//!    (rust/src/backend_wgpu.rs:239-245).
//! Device buffers are reference counted; a buffer whose last handle drops goes back
//! to a size-keyed pool and is reused by a later allocation (a decode step asks
//! for the same shapes every token). Reuse is safe without a sync because every op
//! runs in order on the one stream. The pool is released when the backend and its
//! last tensor are gone; `free_tensor` drops a handle.
pub mod ffi;

use std::cell::RefCell;
use std::collections::HashMap;
use std::ffi::CStr;
use std::os::raw::c_void;
use std::rc::Rc;

use crate::backend::{AttnOpts, Backend, KvAppend, QuantWeight, TensorShape};

/// The context plus the pool of idle device buffers (bytes -> pointers).
struct Pool {
    ctx: *mut ffi::GqCtx,
    idle: HashMap<usize, Vec<*mut c_void>>,
}

impl Pool {
    fn check(&self, rc: i32, what: &str) {
        if rc != ffi::GQ_OK {
            let msg = unsafe { CStr::from_ptr(ffi::gq_last_error(self.ctx)) }.to_string_lossy().into_owned();
            panic!("{what}: {msg} (status {rc})");
        }
    }
    fn take(&mut self, bytes: usize) -> *mut c_void {
        if let Some(p) = self.idle.get_mut(&bytes).and_then(|v| v.pop()) {
            return p;
        }
        let mut p: *mut c_void = std::ptr::null_mut();
        let rc = unsafe { ffi::gq_alloc(self.ctx, bytes, &mut p) };
        self.check(rc, "gq_alloc");
        p
    }
    fn trim(&mut self) {
        for (_, v) in self.idle.drain() {
            for p in v {
                unsafe { ffi::gq_free(self.ctx, p) };
            }
        }
    }
}

impl Drop for Pool {
    fn drop(&mut self) {
        self.trim();
        unsafe { ffi::gq_ctx_destroy(self.ctx) };
    }
}

/// One device allocation; returned to the pool when the last handle drops.
struct DevBuf {
    ptr: *mut c_void,
    bytes: usize,
    pool: Rc<RefCell<Pool>>,
}

impl Drop for DevBuf {
    fn drop(&mut self) {
        self.pool.borrow_mut().idle.entry(self.bytes).or_default().push(self.ptr);
    }
}

/// An uploaded quantized weight (packed bytes + scales on the device); holds the
/// pool so the context outlives it.
struct QW {
    w: *mut ffi::GqQWeight,
    _pool: Rc<RefCell<Pool>>,
}

impl Drop for QW {
    fn drop(&mut self) {
        unsafe { ffi::gq_qweight_free(self.w) };
    }
}

#[derive(Clone)]
pub struct CudaTensor {
    shape: Vec<usize>,
    /// f32 contents, row-major (None for a quantized weight)
    buf: Option<Rc<DevBuf>>,
    /// bf16 copy of an f32 tensor whose values are all exactly bf16 (a weight stored
    /// as BF16 on disk, rust/src/weights.rs:11-14): the plain-weight `linear` path
    bf16: Option<Rc<DevBuf>>,
    quant: Option<Rc<QW>>,
}

impl TensorShape for CudaTensor {
    fn shape(&self) -> &[usize] {
        &self.shape
    }
}

impl CudaTensor {
    fn f32p(&self) -> *mut f32 {
        self.buf.as_ref().expect("f32 tensor expected, got a quantized weight").ptr as *mut f32
    }
    fn qw(&self) -> *const ffi::GqQWeight {
        self.quant.as_ref().expect("quantized weight expected").w
    }
}

pub struct CudaBackend {
    pool: Rc<RefCell<Pool>>,
    ctx: *mut ffi::GqCtx,
}

impl CudaBackend {
    /// A backend on CUDA device `device` (a B200), with the context's own stream.
    pub fn new(device: i32) -> Self {
        let mut ctx: *mut ffi::GqCtx = std::ptr::null_mut();
        let rc = unsafe { ffi::gq_ctx_create(device, &mut ctx) };
        if rc != ffi::GQ_OK {
            let msg = unsafe { CStr::from_ptr(ffi::gq_status_string(rc)) }.to_string_lossy().into_owned();
            panic!("gq_ctx_create(device {device}): {msg}");
        }
        let pool = Rc::new(RefCell::new(Pool { ctx, idle: HashMap::new() }));
        CudaBackend { pool, ctx }
    }

    fn ok(&self, rc: i32, what: &str) {
        self.pool.borrow().check(rc, what);
    }

    fn alloc_bytes(&self, bytes: usize) -> Rc<DevBuf> {
        let bytes = bytes.max(16);
        let ptr = self.pool.borrow_mut().take(bytes);
        Rc::new(DevBuf { ptr, bytes, pool: self.pool.clone() })
    }

    fn alloc(&self, shape: &[usize]) -> CudaTensor {
        let n: usize = shape.iter().product();
        CudaTensor { shape: shape.to_vec(), buf: Some(self.alloc_bytes(n * 4)), bf16: None, quant: None }
    }

    fn upload_u32(&self, v: &[u32]) -> Rc<DevBuf> {
        let b = self.alloc_bytes(v.len() * 4);
        self.ok(unsafe { ffi::gq_memcpy_h2d(self.ctx, b.ptr, v.as_ptr() as *const c_void, v.len() * 4) }, "upload ids");
        b
    }

    fn ew2(&self, a: &CudaTensor, b: &CudaTensor, f: unsafe extern "C" fn(*mut ffi::GqCtx, *const f32, *const f32, i64, *mut f32) -> i32, what: &str) -> CudaTensor {
        let y = self.alloc(&a.shape);
        self.ok(unsafe { f(self.ctx, a.f32p(), b.f32p(), a.size() as i64, y.f32p()) }, what);
        y
    }

    /// Rows [0, rows) x cols of `src` (row stride src_stride) into `dst` (stride dst_stride).
    fn copy_rows(&self, src: *const f32, rows: usize, cols: usize, src_stride: usize, dst: *mut f32, dst_stride: usize) {
        self.ok(unsafe { ffi::gq_copy_rows(self.ctx, src, rows as i64, cols as i64, src_stride as i64, dst, dst_stride as i64) },
            "copy_rows");
    }
}

impl Backend for CudaBackend {
    type Tensor = CudaTensor;

    fn name(&self) -> &str {
        "cuda-b200"
    }

    fn tensor(&self, data: &[f32], shape: &[usize]) -> CudaTensor {
        let t = self.alloc(shape);
        self.ok(unsafe { ffi::gq_memcpy_h2d(self.ctx, t.f32p() as *mut c_void, data.as_ptr() as *const c_void, data.len() * 4) },
            "tensor");
        // a weight that is BF16 on disk arrives as bf16-exact f32: keep a bf16 copy for `linear`
        let mut t = t;
        if shape.len() == 2 && !data.is_empty() && data.iter().all(|v| v.to_bits() & 0xFFFF == 0) {
            let h: Vec<u16> = data.iter().map(|v| (v.to_bits() >> 16) as u16).collect();
            let b = self.alloc_bytes(h.len() * 2);
            self.ok(unsafe { ffi::gq_memcpy_h2d(self.ctx, b.ptr, h.as_ptr() as *const c_void, h.len() * 2) }, "tensor bf16");
            t.bf16 = Some(b);
        }
        t
    }

    fn quant_tensor(&self, q: QuantWeight) -> CudaTensor {                      // backend.rs:95
        let mut w: *mut ffi::GqQWeight = std::ptr::null_mut();
        self.ok(unsafe { ffi::gq_qweight_upload(self.ctx, q.qbytes.as_ptr(), q.qbytes.len(), q.scales.as_ptr(),
            q.scales.len(), q.shape[0] as i64, q.shape[1] as i64, q.bits as i32, q.signed_i8 as i32,
            q.group_size as i64, &mut w) }, "quant_tensor");
        CudaTensor { shape: q.shape.to_vec(), buf: None, bf16: None, quant: Some(Rc::new(QW { w, _pool: self.pool.clone() })) }
    }

    fn zeros(&self, shape: &[usize]) -> CudaTensor {
        let t = self.alloc(shape);
        self.ok(unsafe { ffi::gq_memset(self.ctx, t.f32p() as *mut c_void, 0, t.size() * 4) }, "zeros");
        t
    }

    fn reshape(&self, x: &CudaTensor, shape: &[usize]) -> CudaTensor {
        CudaTensor { shape: shape.to_vec(), ..x.clone() }
    }

    fn embed_rows(&self, table: &CudaTensor, ids: &[u32], scale: f32) -> CudaTensor {   // :101-102
        let d = table.shape[1];
        let out = self.alloc(&[ids.len(), d]);
        let dev_ids = self.upload_u32(ids);
        match &table.quant {
            Some(q) => self.ok(unsafe { ffi::gq_embed_rows(self.ctx, q.w, dev_ids.ptr as *const u32, ids.len() as i64,
                scale, out.f32p()) }, "embed_rows"),
            None => {
                // f32 table: gather the rows, then scale (rust/src/backend_cpu.rs:139-145)
                for (i, &id) in ids.iter().enumerate() {
                    let src = unsafe { table.f32p().add(id as usize * d) };
                    let dst = unsafe { out.f32p().add(i * d) };
                    self.copy_rows(src, 1, d, d, dst, d);
                }
                self.ok(unsafe { ffi::gq_scale(self.ctx, out.f32p(), out.size() as i64, scale, out.f32p()) }, "embed scale");
            }
        }
        out
    }

    fn rms_norm(&self, x: &CudaTensor, w: Option<&CudaTensor>, eps: f32) -> CudaTensor {   // :103-104
        let d = *x.shape.last().unwrap();
        let y = self.alloc(&x.shape);
        self.ok(unsafe { ffi::gq_rms_norm(self.ctx, x.f32p(), (x.size() / d) as i64, d as i64,
            w.map_or(std::ptr::null(), |w| w.f32p() as *const f32), eps, y.f32p(), d as i64) }, "rms_norm");
        y
    }

    fn linear(&self, x: &CudaTensor, w: &CudaTensor) -> CudaTensor {              // :105-106
        let k = *x.shape.last().unwrap();
        let m = x.size() / k;
        let n = w.shape[0];
        let y = self.alloc(&[m, n]);
        if let Some(q) = &w.quant {
            self.ok(unsafe { ffi::gq_linear(self.ctx, x.f32p(), m as i64, k as i64, q.w, y.f32p()) }, "linear");
        } else {
            let h = w.bf16.as_ref().expect("linear: a plain weight must be bf16-exact (BF16 on disk)");
            self.ok(unsafe { ffi::gq_linear_bf16(self.ctx, x.f32p(), m as i64, k as i64, h.ptr as *const u16, n as i64,
                y.f32p()) }, "linear_bf16");
        }
        y
    }

    fn add(&self, a: &CudaTensor, b: &CudaTensor) -> CudaTensor {
        self.ew2(a, b, ffi::gq_add, "add")
    }

    fn mul(&self, a: &CudaTensor, b: &CudaTensor) -> CudaTensor {
        self.ew2(a, b, ffi::gq_mul, "mul")
    }

    fn scale(&self, a: &CudaTensor, s: f32) -> CudaTensor {
        let y = self.alloc(&a.shape);
        self.ok(unsafe { ffi::gq_scale(self.ctx, a.f32p(), a.size() as i64, s, y.f32p()) }, "scale");
        y
    }

    fn scale_by_tensor(&self, a: &CudaTensor, s: &CudaTensor) -> CudaTensor {
        let y = self.alloc(&a.shape);
        self.ok(unsafe { ffi::gq_scale_by_tensor(self.ctx, a.f32p(), a.size() as i64, s.f32p(), y.f32p()) },
            "scale_by_tensor");
        y
    }

    fn gelu_tanh(&self, a: &CudaTensor) -> CudaTensor {
        // gelu(a) * 1.0: the product with one is exact, so this is gelu_tanh_scalar itself
        let ones = self.tensor(&vec![1.0f32; a.size()], &[a.size()]);
        self.ew2(a, &ones, ffi::gq_geglu, "gelu_tanh")
    }

    fn geglu(&self, gate: &CudaTensor, up: &CudaTensor) -> CudaTensor {
        self.ew2(gate, up, ffi::gq_geglu, "geglu")
    }

    fn softcap(&self, a: &CudaTensor, cap: f32) -> CudaTensor {                   // :116
        let y = self.alloc(&a.shape);
        self.ok(unsafe { ffi::gq_softcap(self.ctx, a.f32p(), a.size() as i64, cap, y.f32p()) }, "softcap");
        y
    }

    fn rope(&self, x: &CudaTensor, positions: &[u32], theta: f32, head_dim: usize, heads: usize,
            rotary_dim: usize) -> CudaTensor {                                     // :118-119
        let y = self.alloc(&x.shape);
        let p = self.upload_u32(positions);
        self.ok(unsafe { ffi::gq_rope(self.ctx, x.f32p(), positions.len() as i64, heads as i64, head_dim as i64,
            p.ptr as *const u32, theta, rotary_dim as i64, y.f32p(), 0) }, "rope");
        y
    }

    fn attention(&self, q: &CudaTensor, k: &CudaTensor, v: &CudaTensor, o: &AttnOpts) -> CudaTensor {   // :120-121
        let (t, hq, dh) = (q.shape[0], q.shape[1], q.shape[2]);
        let y = self.alloc(&[t, hq * dh]);
        let (qp, kp) = (self.upload_u32(o.q_pos), self.upload_u32(o.k_pos));
        // a KV cache appends positions in order: the visible range is found by binary search
        let flags = if o.k_pos.windows(2).all(|w| w[0] < w[1]) { ffi::GQ_ATTN_KPOS_ASCENDING } else { 0 };
        self.ok(unsafe { ffi::gq_attention(self.ctx, q.f32p(), 1, t as i64, hq as i64, dh as i64, k.f32p(), v.f32p(),
            k.shape[0] as i64, k.shape[1] as i64, 0, qp.ptr as *const u32, kp.ptr as *const u32, 0, o.scale,
            o.sliding_window, o.attn_softcap, flags, y.f32p()) }, "attention");
        y
    }

    fn slice_rows(&self, x: &CudaTensor, start: usize, count: usize) -> CudaTensor {   // :122-130
        let dim = x.shape[1];
        let y = self.alloc(&[count, dim]);
        self.copy_rows(unsafe { x.f32p().add(start * dim) }, count, dim, dim, y.f32p(), dim);
        y
    }

    fn slice_cols(&self, x: &CudaTensor, offset: usize, width: usize) -> CudaTensor {
        let (rows, stride) = (x.shape[0], x.shape[1]);
        let y = self.alloc(&[rows, width]);
        self.copy_rows(unsafe { x.f32p().add(offset) }, rows, width, stride, y.f32p(), width);
        y
    }

    fn concat_rows(&self, a: Option<&CudaTensor>, b: &CudaTensor) -> CudaTensor {
        let dim: usize = b.shape[1..].iter().product();
        let ar = a.map_or(0, |a| a.shape[0]);
        let mut shape = b.shape.clone();
        shape[0] += ar;
        let y = self.alloc(&shape);
        if let Some(a) = a {
            self.copy_rows(a.f32p(), ar, dim, dim, y.f32p(), dim);
        }
        self.copy_rows(b.f32p(), b.shape[0], dim, dim, unsafe { y.f32p().add(ar * dim) }, dim);
        y
    }

    fn kv_append(&self, existing: Option<&CudaTensor>, add: &CudaTensor) -> KvAppend<CudaTensor> {
        KvAppend { tensor: self.concat_rows(existing, add), dead: existing.cloned() }
    }

    // ---- fused ops: single launches instead of the trait's compositions ----------
    fn add_rms_norm(&self, residual: &CudaTensor, x: &CudaTensor, w: &CudaTensor, eps: f32,
                    scale_by: Option<&CudaTensor>) -> CudaTensor {                // :137-144
        let d = *x.shape.last().unwrap();
        let y = self.alloc(&x.shape);
        self.ok(unsafe { ffi::gq_add_rms_norm(self.ctx, residual.f32p(), x.f32p(), (x.size() / d) as i64, d as i64,
            w.f32p(), eps, scale_by.map_or(std::ptr::null(), |s| s.f32p() as *const f32), y.f32p()) }, "add_rms_norm");
        y
    }

    fn head_norm_rope(&self, x: &CudaTensor, w: &CudaTensor, eps: f32, positions: &[u32], theta: f32,
                      head_dim: usize, heads: usize, rotary_dim: usize) -> CudaTensor {   // :148-154
        let y = self.alloc(&x.shape);
        let p = self.upload_u32(positions);
        self.ok(unsafe { ffi::gq_head_norm_rope(self.ctx, x.f32p(), positions.len() as i64, heads as i64,
            head_dim as i64, w.f32p(), eps, p.ptr as *const u32, theta, rotary_dim as i64, y.f32p(), 0) },
            "head_norm_rope");
        y
    }

    fn linear_geglu(&self, x: &CudaTensor, w_gate: &CudaTensor, w_up: &CudaTensor) -> CudaTensor {   // :155-160
        let k = *x.shape.last().unwrap();
        let m = x.size() / k;
        let y = self.alloc(&[m, w_gate.shape[0]]);
        self.ok(unsafe { ffi::gq_linear_geglu(self.ctx, x.f32p(), m as i64, k as i64, w_gate.qw(), w_up.qw(),
            y.f32p()) }, "linear_geglu");
        y
    }

    fn linear_gelu_mul_cols(&self, x: &CudaTensor, w: &CudaTensor, b: &CudaTensor, offset: usize) -> CudaTensor {   // :161-167
        let k = *x.shape.last().unwrap();
        let m = x.size() / k;
        let y = self.alloc(&[m, w.shape[0]]);
        self.ok(unsafe { ffi::gq_linear_gelu_mul_cols(self.ctx, x.f32p(), m as i64, k as i64, w.qw(), b.f32p(),
            b.shape[1] as i64, offset as i64, y.f32p()) }, "linear_gelu_mul_cols");
        y
    }

    // ---- sync / lifecycle ---------------------------------------------------------
    fn readback(&self, t: &CudaTensor) -> Vec<f32> {                            // :171
        let mut v = vec![0f32; t.size()];
        self.ok(unsafe { ffi::gq_readback(self.ctx, v.as_mut_ptr(), t.f32p(), v.len()) }, "readback");
        v
    }

    fn flush(&self) {
        self.ok(unsafe { ffi::gq_sync(self.ctx) }, "flush");
    }

    fn end_frame(&self, _keep: &[CudaTensor], also_free: Vec<CudaTensor>) {
        // the frame's intermediates went back to the pool when their handles
        // dropped; the pool keeps them for the next token's identical shapes
        drop(also_free);
    }

    fn free_tensor(&self, t: CudaTensor) {
        drop(t);
    }
}
