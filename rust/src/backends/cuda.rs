//! NVIDIA B200 backend: KernRT's per-row layer ops (embed, RMSNorm, q/k norm,
//! RoPE, SwiGLU, residual add, mul, LFM2 short conv, copy) as sm_100a kernels
//! behind the C ABI of kernrt_cuda.h, and the contractions (`project`,
//! `logits`, `kv_write`, `attention`) in the reference backend's arithmetic
//! order.  Activations live on the device and cross this API as handles;
//! `read` is the only barrier (mod.rs:8-15).
//!
//! Built only with `--features cuda`; build.rs links `libkernrt_cuda.so` from
//! the checkout named by `KERNRT_CUDA_DIR`.

use std::collections::HashMap;
use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};
use std::sync::Arc;

use super::{AttnSpec, Backend, Buf, KvSpec, ModelWeights, Proj, RopeSpec, Window};
use crate::ops::Matrix;

#[repr(C)]
struct Ctx {
    _opaque: [u8; 0],
}

/// `kernrt_window`: one query row's window (mod.rs:179-188).
#[repr(C)]
struct KernrtWindow {
    att_start: u64,
    slot: u64,
    shared_start: u64,
    shared_end: u64,
}

unsafe extern "C" {
    fn kernrt_cuda_last_error() -> *const c_char;
    fn kernrt_cuda_create(device: c_int, out: *mut *mut Ctx) -> c_int;
    fn kernrt_cuda_destroy(ctx: *mut Ctx) -> c_int;
    fn kernrt_cuda_prepare_embedding(ctx: *mut Ctx, kind: c_int, data: *const c_void, scales: *const f32,
                                     vocab: usize, dim: usize) -> c_int;
    fn kernrt_cuda_alloc(ctx: *mut Ctx, len: usize, out: *mut u64) -> c_int;
    fn kernrt_cuda_upload(ctx: *mut Ctx, data: *const f32, len: usize, out: *mut u64) -> c_int;
    fn kernrt_cuda_read(ctx: *mut Ctx, src: u64, out: *mut f32, len: usize) -> c_int;
    fn kernrt_cuda_embed(ctx: *mut Ctx, token: usize, out: u64, offset: usize) -> c_int;
    fn kernrt_cuda_copy(ctx: *mut Ctx, src: u64, src_offset: usize, dst: u64, dst_offset: usize,
                        len: usize) -> c_int;
    fn kernrt_cuda_rms_norm(ctx: *mut Ctx, out: u64, x: u64, weight: u64, rows: usize, dim: usize,
                            eps: f32) -> c_int;
    fn kernrt_cuda_qk_norm(ctx: *mut Ctx, v: u64, rows: usize, width: usize, head_size: usize,
                           weight: u64, eps: f32) -> c_int;
    fn kernrt_cuda_rope(ctx: *mut Ctx, q: u64, k: u64, q_width: usize, kv_width: usize, rows: usize,
                        positions: *const u64, n_positions: usize, head_size: usize, theta: f32,
                        interleaved: c_int) -> c_int;
    fn kernrt_cuda_add_in_place(ctx: *mut Ctx, dst: u64, src: u64, len: usize) -> c_int;
    fn kernrt_cuda_mul(ctx: *mut Ctx, out: u64, out_off: usize, a: u64, a_off: usize, b: u64, b_off: usize,
                       len: usize) -> c_int;
    fn kernrt_cuda_conv_prefill(ctx: *mut Ctx, out: u64, x: u64, kernel: u64, rows: usize, dim: usize,
                                k: usize) -> c_int;
    fn kernrt_cuda_conv_decode(ctx: *mut Ctx, out: u64, x: u64, kernel: u64, state: u64, dim: usize,
                               k: usize) -> c_int;
    fn kernrt_cuda_silu_mul(ctx: *mut Ctx, gate: u64, up: u64, len: usize) -> c_int;
    fn kernrt_cuda_prepare_matrix(ctx: *mut Ctx, kind: c_int, data: *const c_void, scales: *const f32,
                                  out_dim: usize, in_dim: usize, out: *mut u64) -> c_int;
    fn kernrt_cuda_project(ctx: *mut Ctx, w: u64, x: u64, y: u64, rows: usize) -> c_int;
    fn kernrt_cuda_project_qkv(ctx: *mut Ctx, wq: u64, wk: u64, wv: u64, x: u64, q: u64, k: u64, v: u64,
                               rows: usize) -> c_int;
    fn kernrt_cuda_project_gate_up(ctx: *mut Ctx, wg: u64, wu: u64, x: u64, gate: u64, up: u64,
                                   rows: usize) -> c_int;
    fn kernrt_cuda_logits(ctx: *mut Ctx, w: u64, x: u64, y: u64) -> c_int;
    fn kernrt_cuda_kv_prepare(ctx: *mut Ctx, n_layers: usize, kv_dim: usize, seq_len: usize) -> c_int;
    fn kernrt_cuda_kv_write(ctx: *mut Ctx, layer: usize, slots: *const u64, n_slots: usize, k: u64, v: u64,
                            rows: usize) -> c_int;
    fn kernrt_cuda_attention(ctx: *mut Ctx, q: u64, out: u64, att: u64, layer: usize,
                             windows: *const KernrtWindow, n_windows: usize, n_heads: usize, kv_mul: usize,
                             head_size: usize, kv_dim: usize, seq_len: usize) -> c_int;
}

// Storage kinds of kernrt_cuda.h (KERNRT_F32 ... KERNRT_Q8_0X4).
const KIND_F32: c_int = 0;
const KIND_BF16: c_int = 1;
const KIND_Q8_0: c_int = 2;

fn last_error() -> String {
    unsafe { CStr::from_ptr(kernrt_cuda_last_error()) }
        .to_string_lossy()
        .into_owned()
}

/// Misuse panics, as on the other backends (reference.rs:60-61, :135).
fn check(rc: c_int) {
    if rc != 0 {
        panic!("cuda backend: {}", last_error());
    }
}

pub struct Cuda {
    ctx: *mut Ctx,
    storage: &'static str,
    weights: Option<Arc<ModelWeights>>,
    /// Device handle of each `Buf` (`Buf.0` indexes this).
    handles: Vec<u64>,
    /// Device matrix of each (layer, `Proj::index`), and the classifier's.
    mats: HashMap<(usize, usize), u64>,
    classifier: u64,
}

// The context is used by one thread at a time (`&mut self` everywhere), and
// the library makes its device current on every call, so the owner may move
// between threads.
unsafe impl Send for Cuda {}

impl Drop for Cuda {
    fn drop(&mut self) {
        unsafe { kernrt_cuda_destroy(self.ctx) };
    }
}

impl Cuda {
    /// `Err` carries the detail for `BackendError` ("no CUDA device", ...).
    /// `KERNRT_CUDA_DEVICE=<n>` picks the device (default 0).
    pub fn new() -> Result<Self, String> {
        let mut ctx = std::ptr::null_mut();
        if unsafe { kernrt_cuda_create(-1, &mut ctx) } != 0 {
            return Err(last_error());
        }
        Ok(Cuda {
            ctx,
            storage: "f32",
            weights: None,
            handles: Vec::new(),
            mats: HashMap::new(),
            classifier: 0,
        })
    }

    /// The C ABI's storage kind of `m` and the pointers to hand over: f32 and
    /// bf16 as stored, Q8_0 and Q8_0x4 in the row-major Q8_0 form a device
    /// backend asks for (quant.rs:646-652).  The returned vectors keep the
    /// repacked Q8_0 bytes alive for the call.
    fn stored(m: &Matrix) -> (c_int, *const c_void, *const f32, Option<(Vec<i8>, Vec<f32>)>) {
        match m {
            Matrix::F32(t) => (KIND_F32, t.data().as_ptr().cast(), std::ptr::null(), None),
            Matrix::Bf16 { data, .. } => (KIND_BF16, data.as_ptr().cast(), std::ptr::null(), None),
            _ => {
                let (q, s) = m.to_q8_row_major().expect("quantized storage");
                let (qp, sp) = (q.as_ptr().cast(), s.as_ptr());
                (KIND_Q8_0, qp, sp, Some((q, s)))
            }
        }
    }

    fn upload_matrix(&self, m: &Matrix) -> u64 {
        let (kind, data, scales, _keep) = Self::stored(m);
        let mut h = 0u64;
        check(unsafe { kernrt_cuda_prepare_matrix(self.ctx, kind, data, scales, m.out_dim(), m.in_dim(), &mut h) });
        h
    }

    fn h(&self, b: Buf) -> u64 {
        self.handles[b.0]
    }

    fn push(&mut self, h: u64) -> Buf {
        self.handles.push(h);
        Buf(self.handles.len() - 1)
    }

    fn mat(&self, layer: usize, proj: Proj) -> u64 {
        *self
            .mats
            .get(&(layer, proj.index()))
            .expect("prepare() runs before compute")
    }
}

impl Backend for Cuda {
    fn name(&self) -> &'static str {
        "cuda"
    }

    fn storage(&self) -> &'static str {
        self.storage
    }

    fn prepare(&mut self, weights: Arc<ModelWeights>, kv: KvSpec) {
        let m = &weights.token_embedding;
        let (kind, data, scales, _keep) = Self::stored(m);
        check(unsafe { kernrt_cuda_prepare_embedding(self.ctx, kind, data, scales, m.out_dim(), m.in_dim()) });
        self.storage = m.kind();
        // Every projection a layer carries, and the classifier, once.
        for (l, layer) in weights.layers.iter().enumerate() {
            for p in Proj::ALL {
                if let Some(m) = p.matrix_opt(layer) {
                    let h = self.upload_matrix(m);
                    self.mats.insert((l, p.index()), h);
                }
            }
        }
        self.classifier = self.upload_matrix(weights.classifier());
        check(unsafe { kernrt_cuda_kv_prepare(self.ctx, kv.n_layers, kv.kv_dim, kv.seq_len) });
        self.weights = Some(weights);
    }

    fn alloc(&mut self, len: usize) -> Buf {
        let mut h = 0u64;
        check(unsafe { kernrt_cuda_alloc(self.ctx, len, &mut h) });
        self.push(h)
    }

    fn upload(&mut self, data: &[f32]) -> Buf {
        let mut h = 0u64;
        check(unsafe { kernrt_cuda_upload(self.ctx, data.as_ptr(), data.len(), &mut h) });
        self.push(h)
    }

    fn read(&mut self, src: Buf, out: &mut [f32]) {
        check(unsafe { kernrt_cuda_read(self.ctx, self.h(src), out.as_mut_ptr(), out.len()) });
    }

    fn embed(&mut self, token: usize, out: Buf, offset: usize) {
        check(unsafe { kernrt_cuda_embed(self.ctx, token, self.h(out), offset) });
    }

    fn copy(&mut self, src: Buf, src_offset: usize, dst: Buf, dst_offset: usize, len: usize) {
        check(unsafe { kernrt_cuda_copy(self.ctx, self.h(src), src_offset, self.h(dst), dst_offset, len) });
    }

    fn rms_norm(&mut self, out: Buf, x: Buf, weight: Buf, rows: usize, dim: usize, eps: f32) {
        check(unsafe { kernrt_cuda_rms_norm(self.ctx, self.h(out), self.h(x), self.h(weight), rows, dim, eps) });
    }

    fn qk_norm(&mut self, v: Buf, rows: usize, width: usize, head_size: usize, weight: Buf, eps: f32) {
        check(unsafe { kernrt_cuda_qk_norm(self.ctx, self.h(v), rows, width, head_size, self.h(weight), eps) });
    }

    fn rope(&mut self, q: Buf, k: Buf, q_width: usize, kv_width: usize, rows: usize, positions: &[usize],
            spec: RopeSpec) {
        // usize is 64 bits on every target the library builds for.
        check(unsafe {
            kernrt_cuda_rope(self.ctx, self.h(q), self.h(k), q_width, kv_width, rows, positions.as_ptr().cast(),
                             positions.len(), spec.head_size, spec.theta, spec.interleaved as c_int)
        });
    }

    fn project(&mut self, layer: usize, proj: Proj, x: Buf, y: Buf, rows: usize) {
        let w = self.mat(layer, proj);
        check(unsafe { kernrt_cuda_project(self.ctx, w, self.h(x), self.h(y), rows) });
    }

    /// One launch for the three (mod.rs:320-325 invites the override).
    fn project_qkv(&mut self, layer: usize, x: Buf, q: Buf, k: Buf, v: Buf, rows: usize) {
        let (wq, wk, wv) = (self.mat(layer, Proj::Q), self.mat(layer, Proj::K), self.mat(layer, Proj::V));
        check(unsafe {
            kernrt_cuda_project_qkv(self.ctx, wq, wk, wv, self.h(x), self.h(q), self.h(k), self.h(v), rows)
        });
    }

    fn project_gate_up(&mut self, layer: usize, x: Buf, gate: Buf, up: Buf, rows: usize) {
        let (wg, wu) = (self.mat(layer, Proj::Gate), self.mat(layer, Proj::Up));
        check(unsafe { kernrt_cuda_project_gate_up(self.ctx, wg, wu, self.h(x), self.h(gate), self.h(up), rows) });
    }

    fn kv_write(&mut self, layer: usize, slots: &[usize], k: Buf, v: Buf, rows: usize) {
        check(unsafe {
            kernrt_cuda_kv_write(self.ctx, layer, slots.as_ptr().cast(), slots.len(), self.h(k), self.h(v), rows)
        });
    }

    fn attention(&mut self, q: Buf, out: Buf, att: Buf, layer: usize, windows: &[Window], spec: AttnSpec) {
        let ws: Vec<KernrtWindow> = windows
            .iter()
            .map(|w| KernrtWindow {
                att_start: w.att_start as u64,
                slot: w.slot as u64,
                shared_start: w.shared.0 as u64,
                shared_end: w.shared.1 as u64,
            })
            .collect();
        check(unsafe {
            kernrt_cuda_attention(self.ctx, self.h(q), self.h(out), self.h(att), layer, ws.as_ptr(), ws.len(),
                                  spec.n_heads, spec.kv_mul, spec.head_size, spec.kv_dim, spec.seq_len)
        });
    }

    fn add_in_place(&mut self, dst: Buf, src: Buf, len: usize) {
        check(unsafe { kernrt_cuda_add_in_place(self.ctx, self.h(dst), self.h(src), len) });
    }

    fn mul(&mut self, out: Buf, out_off: usize, a: Buf, a_off: usize, b: Buf, b_off: usize, len: usize) {
        check(unsafe {
            kernrt_cuda_mul(self.ctx, self.h(out), out_off, self.h(a), a_off, self.h(b), b_off, len)
        });
    }

    fn conv_prefill(&mut self, out: Buf, x: Buf, kernel: Buf, rows: usize, dim: usize, k: usize) {
        check(unsafe { kernrt_cuda_conv_prefill(self.ctx, self.h(out), self.h(x), self.h(kernel), rows, dim, k) });
    }

    fn conv_decode(&mut self, out: Buf, x: Buf, kernel: Buf, state: Buf, dim: usize, k: usize) {
        check(unsafe {
            kernrt_cuda_conv_decode(self.ctx, self.h(out), self.h(x), self.h(kernel), self.h(state), dim, k)
        });
    }

    fn silu_mul(&mut self, gate: Buf, up: Buf, len: usize) {
        check(unsafe { kernrt_cuda_silu_mul(self.ctx, self.h(gate), self.h(up), len) });
    }

    fn logits(&mut self, x: Buf, y: Buf) {
        check(unsafe { kernrt_cuda_logits(self.ctx, self.classifier, self.h(x), self.h(y)) });
    }
}
