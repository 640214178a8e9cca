//! CUDA backend for diffrast on the B200 (sm_100a).
//!
//! Two surfaces over the C ABI of `libdiffrast_cuda.so` (include/diffrast_cuda.h):
//!
//! - [`GpuRasterizer`]: the `diffrast-gpu` crate's type, method for method
//!   (crates/diffrast-gpu/src/lib.rs:194-910), with the same [`GpuError`]
//!   variants, [`ReduceMode`], [`BackwardMode`], [`BackwardTimings`] and
//!   [`PoolStats`]. Scenes and canvases are the `diffrast` crate's own types.
//! - The `diffrast` crate's entry points (crates/diffrast/src/lib.rs:18-24) on
//!   the GPU: [`render`], [`render_batch`], [`render_with_tape`], [`backward`],
//!   [`backward_batch`], [`fit`], [`Fitter`] and [`Adam`], with the same
//!   signatures. They use one process-wide rasterizer on device 0 and panic
//!   where the CPU functions panic (size mismatches) and when the device fails,
//!   since their signatures have no error type.
//!
//! Results match the CPU path to the north star's tolerances (images 1e-5 abs /
//! 1e-4 rel, gradients 1e-6 abs + 1e-3 rel per element). Gradients are sums of
//! f32 atomics, so repeated calls agree to a few ulps, not bitwise. There is no
//! CPU fallback: a missing device is [`GpuError::NoAdapter`].
//!
//! This crate is not built in the repository that ships it (its image has no
//! Rust toolchain); the C ABI it binds is tested there through Python's ctypes.

mod ffi;

use std::ffi::CStr;
use std::os::raw::{c_int, c_void};
use std::ptr::{null_mut, NonNull};
use std::sync::{Mutex, OnceLock};
use std::time::Duration;

pub use diffrast::{Canvas, ConfigError, FitConfig, FitProgress, FitReport, RenderParams, Scene,
                   StepInfo, StopReason, Triangle};

/// Something went wrong talking to the GPU (diffrast-gpu/src/lib.rs:42-72).
#[derive(Debug)]
pub enum GpuError {
    NoAdapter,
    /// The device did not finish the work within [`GpuRasterizer::POLL_TIMEOUT`].
    Timeout,
    DeviceRequest(String),
    Readback(String),
    /// The requested work exceeds a device limit or is malformed.
    TooLarge(String),
}

impl std::fmt::Display for GpuError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        match self {
            Self::NoAdapter => write!(f, "no CUDA device is visible (this backend has no CPU path)"),
            Self::Timeout => write!(
                f,
                "the GPU did not finish within {:?}; it may be busy with another process",
                GpuRasterizer::POLL_TIMEOUT
            ),
            Self::DeviceRequest(m) => write!(f, "CUDA error: {m}"),
            Self::Readback(m) => write!(f, "could not read results back: {m}"),
            Self::TooLarge(m) => write!(f, "{m}"),
        }
    }
}

impl std::error::Error for GpuError {}

/// How the batched backward sums gradients (diffrast-gpu/src/lib.rs:76-84).
/// Both values run the same reduction here (warp shuffles, shared memory, one
/// global atomic per triangle, parameter and CTA); the value is kept so that
/// callers of `backward_many_full` keep compiling and behaving the same.
#[derive(Clone, Copy, Debug, PartialEq, Eq, Default)]
pub enum ReduceMode {
    Direct,
    #[default]
    Workgroup,
}

/// How the single-scene backward recovers the canvas beneath each triangle
/// (diffrast-gpu/src/lib.rs:211-220). This backend keeps no tape and does no
/// O(T^2) re-walk, so both values run the same kernel.
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum BackwardMode {
    Taped,
    Recompute,
}

/// Per-item `(loss, gradients)`, one entry per scene in a batch.
pub type BatchGradients = Vec<(f32, Vec<f32>)>;

/// Where the time of one timed batched backward went (diffrast-gpu/src/lib.rs:96-114).
/// `loss_ms` is 0: the per-image MSE is reduced inside the dispatch.
#[derive(Clone, Copy, Debug, Default)]
pub struct BackwardTimings {
    pub pack_ms: f32,
    pub alloc_ms: f32,
    pub dispatch_ms: f32,
    pub readback_ms: f32,
    pub loss_ms: f32,
}

impl BackwardTimings {
    pub fn total_ms(&self) -> f32 {
        self.pack_ms + self.alloc_ms + self.dispatch_ms + self.readback_ms + self.loss_ms
    }
}

/// Scratch-pool reuse counters (diffrast-gpu/src/lib.rs:153-158).
#[derive(Clone, Copy, Debug, Default)]
pub struct PoolStats {
    pub hits: u64,
    pub misses: u64,
    pub bytes: u64,
}

fn last_error() -> String {
    // SAFETY: dr_last_error returns a NUL-terminated thread-local string that
    // stays valid until this thread's next call into the library.
    unsafe { CStr::from_ptr(ffi::dr_last_error()).to_string_lossy().into_owned() }
}

/// Maps a dr_status onto GpuError, as include/diffrast_cuda.h documents.
fn check(status: ffi::dr_status) -> Result<(), GpuError> {
    match status {
        ffi::DR_OK => Ok(()),
        ffi::DR_NO_DEVICE => Err(GpuError::NoAdapter),
        ffi::DR_TIMEOUT => Err(GpuError::Timeout),
        ffi::DR_INVALID_ARGUMENT | ffi::DR_TOO_LARGE | ffi::DR_OUT_OF_MEMORY => {
            Err(GpuError::TooLarge(last_error()))
        }
        _ => Err(GpuError::DeviceRequest(last_error())),
    }
}

fn dim(v: usize, what: &str) -> Result<c_int, GpuError> {
    c_int::try_from(v).map_err(|_| GpuError::TooLarge(format!("{what} {v} exceeds the C ABI's int")))
}

/// The library context: owns the device scratch pool. The C side serializes
/// calls on it with its own mutex; this type is shared behind `&`.
struct Ctx(NonNull<ffi::dr_ctx>);

// SAFETY: a dr_ctx may be used from several threads (the header says so); its
// calls are serialized by its internal mutex.
unsafe impl Send for Ctx {}
unsafe impl Sync for Ctx {}

impl Ctx {
    fn raw(&self) -> *mut ffi::dr_ctx {
        self.0.as_ptr()
    }
}

impl Drop for Ctx {
    fn drop(&mut self) {
        // SAFETY: the pointer came from dr_ctx_create and is destroyed once.
        unsafe {
            ffi::dr_ctx_destroy(self.0.as_ptr());
        }
    }
}

/// A device buffer of f32 values, freed on drop.
struct DeviceBuf<'a> {
    ctx: &'a Ctx,
    ptr: *mut c_void,
    len: usize,
}

impl<'a> DeviceBuf<'a> {
    fn new(ctx: &'a Ctx, len: usize) -> Result<Self, GpuError> {
        let mut ptr = null_mut();
        // SAFETY: ctx is live; `ptr` receives a device allocation or stays null.
        check(unsafe { ffi::dr_device_alloc(ctx.raw(), len * 4, &mut ptr) })?;
        Ok(Self { ctx, ptr, len })
    }

    fn from_host(ctx: &'a Ctx, data: &[f32]) -> Result<Self, GpuError> {
        let b = Self::new(ctx, data.len())?;
        // SAFETY: both ranges hold data.len() floats; the legacy stream orders
        // the copy before any later call that reads the buffer.
        check(unsafe {
            ffi::dr_memcpy(ctx.raw(), b.ptr, data.as_ptr() as *const c_void, data.len() * 4,
                           null_mut())
        })?;
        Ok(b)
    }

    fn f32(&self) -> *const f32 {
        self.ptr as *const f32
    }

    fn f32_mut(&self) -> *mut f32 {
        self.ptr as *mut f32
    }

    /// Copies the buffer out, after a bounded wait for the work that writes it.
    fn to_host(&self, out: &mut [f32]) -> Result<(), GpuError> {
        assert_eq!(out.len(), self.len, "readback length mismatch");
        wait()?;
        // SAFETY: both ranges hold self.len floats; the device work is done.
        check(unsafe {
            ffi::dr_memcpy(self.ctx.raw(), out.as_mut_ptr() as *mut c_void, self.ptr, self.len * 4,
                           null_mut())
        })
        .map_err(|e| GpuError::Readback(e.to_string()))
    }
}

impl Drop for DeviceBuf<'_> {
    fn drop(&mut self) {
        // SAFETY: allocated by dr_device_alloc on this context.
        unsafe {
            ffi::dr_device_free(self.ctx.raw(), self.ptr);
        }
    }
}

/// The bounded wait every call ends with (POLL_TIMEOUT semantics).
fn wait() -> Result<(), GpuError> {
    // SAFETY: the null stream is the legacy default stream every call here uses.
    check(unsafe { ffi::dr_stream_wait(null_mut(), GpuRasterizer::POLL_TIMEOUT.as_secs_f64()) })
}

/// Validates a batch and returns its shared triangle count; `Ok(None)` for an
/// empty batch (diffrast-gpu/src/lib.rs:914-929).
fn check_batch(scenes: &[Scene]) -> Result<Option<usize>, GpuError> {
    let Some(first) = scenes.first() else { return Ok(None) };
    let n_tris = first.len();
    if n_tris == 0 {
        return Err(GpuError::TooLarge("scenes must contain at least one triangle".into()));
    }
    if let Some(bad) = scenes.iter().position(|s| s.len() != n_tris) {
        return Err(GpuError::TooLarge(format!(
            "batched scenes must share a triangle count: item 0 has {n_tris}, item {bad} has {}",
            scenes[bad].len()
        )));
    }
    Ok(Some(n_tris))
}

/// Flat (B, T, 10) parameters and (B, 3) backgrounds of a batch.
fn pack(scenes: &[Scene]) -> (Vec<f32>, Vec<f32>) {
    let tris = scenes.iter().flat_map(|s| s.params()).collect();
    let bgs = scenes.iter().flat_map(|s| s.background).collect();
    (tris, bgs)
}

/// The GPU rasterizer: a CUDA device with its scratch pool.
pub struct GpuRasterizer {
    ctx: Ctx,
    info: String,
    discrete: bool,
    /// Keeps each method's upload, launch and readback together.
    calls: Mutex<()>,
}

impl GpuRasterizer {
    /// How long any call waits for the device before returning
    /// [`GpuError::Timeout`] (diffrast-gpu/src/lib.rs:229).
    pub const POLL_TIMEOUT: Duration = Duration::from_secs(60);

    /// Device 0.
    pub fn new() -> Result<Self, GpuError> {
        Self::with_device(0)
    }

    pub fn with_device(device: i32) -> Result<Self, GpuError> {
        let mut raw = null_mut();
        // SAFETY: `raw` receives a context or stays null on error.
        check(unsafe { ffi::dr_ctx_create(device, &mut raw) })?;
        let ctx = Ctx(NonNull::new(raw).ok_or(GpuError::NoAdapter)?);
        let mut buf = [0 as std::os::raw::c_char; 256];
        // SAFETY: buf holds 256 bytes; the name is NUL-terminated within them.
        check(unsafe { ffi::dr_device_name(device, buf.as_mut_ptr(), buf.len()) })?;
        let name = unsafe { CStr::from_ptr(buf.as_ptr()) }.to_string_lossy().into_owned();
        let discrete = unsafe { ffi::dr_is_discrete(device) } == 1;
        Ok(Self { ctx, info: format!("{name} (CUDA)"), discrete, calls: Mutex::new(()) })
    }

    /// Human-readable description of the device in use.
    pub fn adapter_info(&self) -> &str {
        &self.info
    }

    /// Whether this is a discrete card rather than an integrated one.
    pub fn is_discrete(&self) -> bool {
        self.discrete
    }

    /// Bytes the reference's taped backward would hold for a workload. This
    /// backend keeps no tape; its own scratch is [`Self::scratch_bytes`].
    pub fn tape_bytes(n_tris: usize, width: usize, height: usize) -> u64 {
        // SAFETY: pure arithmetic in the library.
        unsafe { ffi::dr_tape_bytes(n_tris as u64, width as u64, height as u64) }
    }

    /// Device scratch a batched backward of this shape holds.
    pub fn scratch_bytes(&self, batch: usize, n_tris: usize, p: RenderParams) -> u64 {
        match (dim(batch, "batch"), dim(n_tris, "triangles"), dim(p.height, "height"),
               dim(p.width, "width")) {
            (Ok(b), Ok(t), Ok(h), Ok(w)) => unsafe {
                ffi::dr_scratch_bytes(self.ctx.raw(), b, t, h, w)
            },
            _ => 0,
        }
    }

    /// Reuse counters for the scratch pool.
    pub fn pool_stats(&self) -> PoolStats {
        let mut s = ffi::dr_pool_stats::default();
        // SAFETY: ctx is live; `s` is a valid out-pointer.
        unsafe { ffi::dr_pool_stats_get(self.ctx.raw(), &mut s) };
        PoolStats { hits: s.hits, misses: s.misses, bytes: s.bytes }
    }

    /// Frees every pooled buffer (waits for the device first).
    pub fn clear_pool(&self) {
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        // SAFETY: ctx is live.
        unsafe { ffi::dr_clear_pool(self.ctx.raw()) };
    }

    /// Render a scene on the GPU.
    pub fn render(&self, scene: &Scene, p: RenderParams) -> Result<Canvas, GpuError> {
        let (tris, bgs) = pack(std::slice::from_ref(scene));
        let data = self.render_raw(&tris, &bgs, 1, scene.len(), p)?;
        Ok(Canvas { width: p.width, height: p.height, data })
    }

    /// Render and compute gradients in one round trip; `(loss, gradients)`
    /// laid out like the CPU `diffrast::backward`.
    pub fn backward(&self, scene: &Scene, p: RenderParams,
                    target: &Canvas) -> Result<(f32, Vec<f32>), GpuError> {
        self.backward_with(scene, p, target, BackwardMode::Recompute)
    }

    /// Gradients with an explicit [`BackwardMode`] (both run the same kernel).
    pub fn backward_with(&self, scene: &Scene, p: RenderParams, target: &Canvas,
                         mode: BackwardMode) -> Result<(f32, Vec<f32>), GpuError> {
        assert_eq!(target.width, p.width, "target width mismatch");
        assert_eq!(target.height, p.height, "target height mismatch");
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        let t = scene.len();
        let params = scene.params();
        let d_params = DeviceBuf::from_host(&self.ctx, &params)?;
        let d_target = DeviceBuf::from_host(&self.ctx, &target.data)?;
        let d_grads = DeviceBuf::new(&self.ctx, t * Triangle::N_PARAMS)?;
        let d_loss = DeviceBuf::new(&self.ctx, 1)?;
        let m = match mode {
            BackwardMode::Taped => ffi::DR_BACKWARD_TAPED,
            BackwardMode::Recompute => ffi::DR_BACKWARD_RECOMPUTE,
        };
        // SAFETY: every device buffer holds what the call reads or writes; the
        // background is 3 host floats.
        check(unsafe {
            ffi::dr_backward(self.ctx.raw(), d_params.f32(), scene.background.as_ptr(),
                             dim(t, "triangles")?, dim(p.height, "height")?,
                             dim(p.width, "width")?, p.sigma, d_target.f32(), ffi::DR_LAYOUT_BHWC,
                             m, d_grads.f32_mut(), d_loss.f32_mut(), null_mut(), null_mut())
        })?;
        let mut grads = vec![0.0f32; t * Triangle::N_PARAMS];
        let mut loss = [0.0f32];
        d_loss.to_host(&mut loss)?;
        d_grads.to_host(&mut grads)?;
        Ok((loss[0], grads))
    }

    /// Render a batch in one launch; every scene must share the triangle count.
    pub fn render_many(&self, scenes: &[Scene], p: RenderParams) -> Result<Vec<Canvas>, GpuError> {
        let Some(n_tris) = check_batch(scenes)? else { return Ok(Vec::new()) };
        let (tris, bgs) = pack(scenes);
        let data = self.render_raw(&tris, &bgs, scenes.len(), n_tris, p)?;
        let px = p.width * p.height * 3;
        Ok(data
            .chunks_exact(px)
            .map(|c| Canvas { width: p.width, height: p.height, data: c.to_vec() })
            .collect())
    }

    fn render_raw(&self, tris: &[f32], bgs: &[f32], b: usize, t: usize,
                  p: RenderParams) -> Result<Vec<f32>, GpuError> {
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        let n = b * p.width * p.height * 3;
        let d_params = DeviceBuf::from_host(&self.ctx, tris)?;
        let d_image = DeviceBuf::new(&self.ctx, n)?;
        // SAFETY: params (b, t, 10) and image (b, h, w, 3) on the device; the
        // backgrounds are b * 3 host floats.
        check(unsafe {
            ffi::dr_render(self.ctx.raw(), d_params.f32(), bgs.as_ptr(), 1, dim(b, "batch")?,
                           dim(t, "triangles")?, dim(p.height, "height")?, dim(p.width, "width")?,
                           p.sigma, ffi::DR_LAYOUT_BHWC, d_image.f32_mut(), null_mut())
        })?;
        let mut out = vec![0.0f32; n];
        d_image.to_host(&mut out)?;
        Ok(out)
    }

    /// Render and differentiate a batch: one `(loss, gradients)` per scene,
    /// matching the CPU `diffrast::backward_batch`.
    pub fn backward_many(&self, scenes: &[Scene], p: RenderParams,
                         targets: &[Canvas]) -> Result<BatchGradients, GpuError> {
        let Some(n_tris) = self.check_targets(scenes, p, targets)? else { return Ok(Vec::new()) };
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        let (tris, bgs) = pack(scenes);
        let tgt: Vec<f32> = targets.iter().flat_map(|c| c.data.iter().copied()).collect();
        let b = scenes.len();
        let mut grads = vec![0.0f32; b * n_tris * Triangle::N_PARAMS];
        let mut losses = vec![0.0f32; b];
        // SAFETY: host buffers of the documented sizes; the call returns once
        // the results are in them (bounded by the library's 60 s wait).
        check(unsafe {
            ffi::dr_loss_backward_host(self.ctx.raw(), tris.as_ptr(), bgs.as_ptr(), 1,
                                       dim(b, "batch")?, dim(n_tris, "triangles")?,
                                       dim(p.height, "height")?, dim(p.width, "width")?, p.sigma,
                                       tgt.as_ptr(), ffi::DR_LAYOUT_BHWC, grads.as_mut_ptr(),
                                       losses.as_mut_ptr(), null_mut())
        })?;
        Ok(split(losses, grads, n_tris))
    }

    /// Deterministic gradient sums on this rasterizer (off by default): every
    /// later gradient call, and `fit` through it, gives bit-identical gradients
    /// call to call (fixed-point accumulation; `dr_set_deterministic`). No
    /// reference counterpart.
    pub fn set_deterministic(&self, on: bool) -> Result<(), GpuError> {
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        // SAFETY: ctx is live.
        check(unsafe { ffi::dr_set_deterministic(self.ctx.raw(), on as c_int) })
    }

    /// Whether [`Self::set_deterministic`] is on.
    pub fn deterministic(&self) -> Result<bool, GpuError> {
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        let mut on: c_int = 0;
        // SAFETY: ctx is live; `on` is an out-pointer.
        check(unsafe { ffi::dr_get_deterministic(self.ctx.raw(), &mut on) })?;
        Ok(on != 0)
    }

    /// As [`Self::backward_many`], with the phase breakdown. Phases run one
    /// after another, so this is slower; the breakdown is a diagnostic.
    pub fn backward_many_timed(&self, scenes: &[Scene], p: RenderParams, targets: &[Canvas])
                               -> Result<(BatchGradients, BackwardTimings), GpuError> {
        self.backward_many_full(scenes, p, targets, ReduceMode::default())
    }

    /// Full form: the reduce mode (accepted; one reduction either way) and the
    /// phase timings.
    pub fn backward_many_full(&self, scenes: &[Scene], p: RenderParams, targets: &[Canvas],
                              reduce: ReduceMode)
                              -> Result<(BatchGradients, BackwardTimings), GpuError> {
        let Some(n_tris) = self.check_targets(scenes, p, targets)? else {
            return Ok((Vec::new(), BackwardTimings::default()));
        };
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        let mode = match reduce {
            ReduceMode::Direct => ffi::DR_REDUCE_DIRECT,
            ReduceMode::Workgroup => ffi::DR_REDUCE_WORKGROUP,
        };
        // SAFETY: ctx is live.
        check(unsafe { ffi::dr_set_reduce_mode(self.ctx.raw(), mode) })?;
        let (tris, bgs) = pack(scenes);
        let tgt: Vec<f32> = targets.iter().flat_map(|c| c.data.iter().copied()).collect();
        let b = scenes.len();
        let mut grads = vec![0.0f32; b * n_tris * Triangle::N_PARAMS];
        let mut losses = vec![0.0f32; b];
        let mut tm = ffi::dr_backward_timings::default();
        // SAFETY: host buffers of the documented sizes; `tm` is an out-pointer.
        check(unsafe {
            ffi::dr_loss_backward_timed(self.ctx.raw(), tris.as_ptr(), bgs.as_ptr(), 1,
                                        dim(b, "batch")?, dim(n_tris, "triangles")?,
                                        dim(p.height, "height")?, dim(p.width, "width")?,
                                        p.sigma, tgt.as_ptr(), ffi::DR_LAYOUT_BHWC,
                                        grads.as_mut_ptr(), losses.as_mut_ptr(), &mut tm,
                                        null_mut())
        })?;
        let t = BackwardTimings {
            pack_ms: tm.pack_ms,
            alloc_ms: tm.alloc_ms,
            dispatch_ms: tm.dispatch_ms,
            readback_ms: tm.readback_ms,
            loss_ms: tm.loss_ms,
        };
        Ok((split(losses, grads, n_tris), t))
    }

    /// Gradients from an upstream image gradient `(batch, height, width, 3)`
    /// flattened, the autograd shape (diffrast-gpu/src/lib.rs:828-910).
    pub fn backward_many_from_grad(&self, scenes: &[Scene], p: RenderParams,
                                   grad_images: &[f32]) -> Result<Vec<Vec<f32>>, GpuError> {
        let Some(n_tris) = check_batch(scenes)? else { return Ok(Vec::new()) };
        let b = scenes.len();
        let expected = b * p.width * p.height * 3;
        if grad_images.len() != expected {
            return Err(GpuError::TooLarge(format!(
                "expected {expected} gradient values, got {}",
                grad_images.len()
            )));
        }
        let _g = self.calls.lock().expect("rasterizer mutex poisoned");
        let (tris, bgs) = pack(scenes);
        let d_params = DeviceBuf::from_host(&self.ctx, &tris)?;
        let d_gin = DeviceBuf::from_host(&self.ctx, grad_images)?;
        let d_grads = DeviceBuf::new(&self.ctx, b * n_tris * Triangle::N_PARAMS)?;
        // SAFETY: device buffers of the documented sizes; backgrounds on the host.
        check(unsafe {
            ffi::dr_grad_backward(self.ctx.raw(), d_params.f32(), bgs.as_ptr(), 1,
                                  dim(b, "batch")?, dim(n_tris, "triangles")?,
                                  dim(p.height, "height")?, dim(p.width, "width")?, p.sigma,
                                  d_gin.f32(), ffi::DR_LAYOUT_BHWC, d_grads.f32_mut(), null_mut())
        })?;
        let mut grads = vec![0.0f32; b * n_tris * Triangle::N_PARAMS];
        d_grads.to_host(&mut grads)?;
        Ok(grads.chunks_exact(n_tris * Triangle::N_PARAMS).map(|g| g.to_vec()).collect())
    }

    fn check_targets(&self, scenes: &[Scene], p: RenderParams,
                     targets: &[Canvas]) -> Result<Option<usize>, GpuError> {
        if scenes.len() != targets.len() {
            return Err(GpuError::TooLarge(format!(
                "batch mismatch: {} scenes but {} targets",
                scenes.len(),
                targets.len()
            )));
        }
        for (i, t) in targets.iter().enumerate() {
            if t.width != p.width || t.height != p.height {
                return Err(GpuError::TooLarge(format!(
                    "target {i} is {}x{}, the render is {}x{}",
                    t.width, t.height, p.width, p.height
                )));
            }
        }
        check_batch(scenes)
    }
}

fn split(losses: Vec<f32>, grads: Vec<f32>, n_tris: usize) -> BatchGradients {
    losses
        .into_iter()
        .zip(grads.chunks_exact(n_tris * Triangle::N_PARAMS))
        .map(|(l, g)| (l, g.to_vec()))
        .collect()
}

// ---------------------------------------------------------------------------
// The diffrast crate's entry points on the GPU
// ---------------------------------------------------------------------------

fn global() -> &'static GpuRasterizer {
    static GPU: OnceLock<GpuRasterizer> = OnceLock::new();
    GPU.get_or_init(|| GpuRasterizer::new().unwrap_or_else(|e| panic!("diffrast-cuda: {e}")))
}

/// `diffrast::render` (raster.rs:37-43) on the GPU.
pub fn render(scene: &Scene, p: RenderParams) -> Canvas {
    global().render(scene, p).unwrap_or_else(|e| panic!("diffrast-cuda render: {e}"))
}

/// `diffrast::render_batch` (grad.rs:210-212) on the GPU. Scenes of different
/// triangle counts render one by one (the CPU function accepts them too).
pub fn render_batch(scenes: &[Scene], p: RenderParams) -> Vec<Canvas> {
    match check_batch(scenes) {
        Ok(_) => global().render_many(scenes, p),
        Err(_) => scenes.iter().map(|s| global().render(s, p)).collect(),
    }
    .unwrap_or_else(|e| panic!("diffrast-cuda render_batch: {e}"))
}

/// What `render_with_tape` hands to `backward`. The GPU backward needs no
/// recorded patches, so this holds nothing but the triangle count it was made
/// for (grad.rs:38-50 keeps per-triangle canvas patches).
pub struct Tape {
    n_tris: usize,
}

impl Tape {
    /// Bytes held by the tape: none.
    pub fn memory_bytes(&self) -> usize {
        0
    }
}

/// `diffrast::render_with_tape` (grad.rs:56-90): the same image; the tape is empty.
pub fn render_with_tape(scene: &Scene, p: RenderParams) -> (Canvas, Tape) {
    (render(scene, p), Tape { n_tris: scene.len() })
}

/// `diffrast::backward` (grad.rs:98-131) on the GPU. The loss and gradients
/// are computed from `scene` and `target`; `rendered` must be the render of
/// `scene`, as for the CPU function.
pub fn backward(scene: &Scene, p: RenderParams, tape: &Tape, rendered: &Canvas,
                target: &Canvas) -> (f32, Vec<f32>) {
    assert_eq!(tape.n_tris, scene.len(), "tape does not match scene");
    assert_eq!(rendered.data.len(), target.data.len(), "target size mismatch");
    global().backward(scene, p, target).unwrap_or_else(|e| panic!("diffrast-cuda backward: {e}"))
}

/// `diffrast::backward_batch` (grad.rs:192-207) on the GPU.
pub fn backward_batch(scenes: &[Scene], p: RenderParams, targets: &[Canvas]) -> Vec<(f32, Vec<f32>)> {
    assert_eq!(scenes.len(), targets.len(), "batch size mismatch");
    match check_batch(scenes) {
        Ok(_) => global().backward_many(scenes, p, targets),
        Err(_) => scenes.iter().zip(targets).map(|(s, t)| global().backward(s, p, t)).collect(),
    }
    .unwrap_or_else(|e| panic!("diffrast-cuda backward_batch: {e}"))
}

/// `diffrast::Adam` (optim.rs:11-60) with its moments on the device. `step`
/// takes the same arguments; the per-parameter rates must follow the fit's
/// pattern (fit.rs:388-396: six position rates, three colour rates, one alpha
/// rate per triangle), which is what the device kernel takes.
pub struct Adam {
    m: Vec<f32>,
    v: Vec<f32>,
    t: u32,
    pub beta1: f32,
    pub beta2: f32,
    pub eps: f32,
}

impl Adam {
    pub fn new(n_params: usize) -> Self {
        Self { m: vec![0.0; n_params], v: vec![0.0; n_params], t: 0, beta1: 0.9, beta2: 0.999,
               eps: 1e-8 }
    }

    pub fn steps_taken(&self) -> u32 {
        self.t
    }

    pub fn step(&mut self, params: &mut [f32], grads: &[f32], lr: &[f32]) {
        assert_eq!(params.len(), grads.len(), "gradient length mismatch");
        assert_eq!(params.len(), lr.len(), "learning-rate length mismatch");
        assert_eq!(params.len() % Triangle::N_PARAMS, 0, "parameters come 10 per triangle");
        self.t += 1;
        if lr.is_empty() {
            return;
        }
        let (lp, lc, la) = (lr[0], lr[6], lr[9]);
        for row in lr.chunks_exact(Triangle::N_PARAMS) {
            assert!(row[..6].iter().all(|&x| x == lp) && row[6..9].iter().all(|&x| x == lc)
                        && row[9] == la,
                    "the device Adam takes one position, colour and alpha rate");
        }
        let gpu = global();
        let _g = gpu.calls.lock().expect("rasterizer mutex poisoned");
        let mut run = || -> Result<(), GpuError> {
            let dp = DeviceBuf::from_host(&gpu.ctx, params)?;
            let dm = DeviceBuf::from_host(&gpu.ctx, &self.m)?;
            let dv = DeviceBuf::from_host(&gpu.ctx, &self.v)?;
            let dg = DeviceBuf::from_host(&gpu.ctx, grads)?;
            // SAFETY: four device arrays of params.len() floats.
            check(unsafe {
                ffi::dr_adam_step(gpu.ctx.raw(), dp.f32_mut(), dm.f32_mut(), dv.f32_mut(), dg.f32(),
                                  params.len() as i64, lp, lc, la, self.t, self.beta1, self.beta2,
                                  self.eps, 0, null_mut())
            })?;
            dp.to_host(params)?;
            dm.to_host(&mut self.m)?;
            dv.to_host(&mut self.v)
        };
        run().unwrap_or_else(|e| panic!("diffrast-cuda Adam::step: {e}"));
    }
}

/// `diffrast::fit` (fit.rs:166-181) on the GPU: the reference's seeding
/// (`diffrast::Fitter::new`, StdRng from `cfg.seed`), then the iterations on
/// the device one at a time so that `on_progress` sees every step.
pub fn fit(target: &Canvas, cfg: &FitConfig,
           mut on_progress: impl FnMut(FitProgress)) -> Result<FitReport, ConfigError> {
    let mut fitter = Fitter::new(target.clone(), cfg.clone())?;
    while let Some(step) = fitter.step() {
        let scene = fitter.scene();
        on_progress(FitProgress { iter: step.iter, loss: step.loss, sigma: step.sigma,
                                  scene: &scene });
    }
    Ok(fitter.into_report())
}

/// The whole fit as one CUDA graph (`dr_fit`): no progress callback, one
/// readback at the end. The fastest form; same result as [`fit`] to rounding.
pub fn fit_graph(target: &Canvas, cfg: &FitConfig) -> Result<FitReport, ConfigError> {
    let seeded = diffrast::Fitter::new(target.clone(), cfg.clone())?;
    let init = seeded.scene().clone();
    let gpu = global();
    let _g = gpu.calls.lock().expect("rasterizer mutex poisoned");
    let t = init.len();
    let c = ffi::dr_fit_config {
        iters: cfg.iters as i64,
        sigma_start: cfg.sigma_start,
        sigma_end: cfg.sigma_end,
        lr_pos: cfg.lr_pos,
        lr_color: cfg.lr_color,
        lr_alpha: cfg.lr_alpha,
        patience: cfg.patience.map_or(-1, |p| p as i64),
        min_delta: cfg.min_delta,
    };
    let run = || -> Result<FitReport, GpuError> {
        let d_target = DeviceBuf::from_host(&gpu.ctx, &target.data)?;
        let d_init = DeviceBuf::from_host(&gpu.ctx, &init.params())?;
        let d_best = DeviceBuf::new(&gpu.ctx, t * Triangle::N_PARAMS)?;
        let d_final = DeviceBuf::new(&gpu.ctx, t * Triangle::N_PARAMS)?;
        let mut losses = vec![0.0f32; cfg.iters.max(1)];
        let mut rep = ffi::dr_fit_report::default();
        // SAFETY: device target (h, w, 3) and parameter arrays; host losses of
        // iters floats; the background is 3 host floats.
        check(unsafe {
            ffi::dr_fit(gpu.ctx.raw(), d_target.f32(), dim(target.height, "height")?,
                        dim(target.width, "width")?, d_init.f32(), init.background.as_ptr(),
                        dim(t, "triangles")?, &c, d_best.f32_mut(), d_final.f32_mut(),
                        losses.as_mut_ptr(), &mut rep, null_mut())
        })?;
        let mut best = vec![0.0f32; t * Triangle::N_PARAMS];
        d_best.to_host(&mut best)?;
        let mut scene = init.clone();
        scene.set_params(&best);
        losses.truncate(rep.n_losses as usize);
        Ok(FitReport {
            scene,
            losses,
            stop_reason: stop_reason(rep.stop_reason),
            best_iter: rep.best_iter as usize,
            best_loss: rep.best_loss,
        })
    };
    Ok(run().unwrap_or_else(|e| panic!("diffrast-cuda fit_graph: {e}")))
}

fn stop_reason(code: c_int) -> StopReason {
    match code {
        ffi::DR_STOP_CONVERGED => StopReason::Converged,
        ffi::DR_STOP_DIVERGED => StopReason::Diverged,
        _ => StopReason::Completed,
    }
}

/// `diffrast::Fitter` (fit.rs:197-336) with parameters, Adam moments and
/// gradients on the device: each step is one fused forward + loss + backward
/// launch, a 4-byte loss readback, the reference's stop logic on the host, and
/// the fused Adam + projection launch.
pub struct Fitter {
    target: Canvas,
    cfg: FitConfig,
    scene: Scene,
    best: Vec<f32>,
    params: Vec<f32>,
    m: Vec<f32>,
    v: Vec<f32>,
    losses: Vec<f32>,
    iter: usize,
    since: usize,
    best_iter: usize,
    best_loss: f32,
    stop: Option<StopReason>,
}

impl Fitter {
    pub fn new(target: Canvas, cfg: FitConfig) -> Result<Self, ConfigError> {
        let seeded = diffrast::Fitter::new(target.clone(), cfg.clone())?;
        let scene = seeded.scene().clone();
        let params = scene.params();
        let n = params.len();
        Ok(Self { target, cfg, best: params.clone(), params, m: vec![0.0; n], v: vec![0.0; n],
                  scene, losses: Vec::new(), iter: 0, since: 0, best_iter: 0,
                  best_loss: f32::INFINITY, stop: None })
    }

    /// One iteration (fit.rs:243-288); `None` once the fit has stopped.
    pub fn step(&mut self) -> Option<StepInfo> {
        if self.stop.is_some() {
            return None;
        }
        if self.iter >= self.cfg.iters {
            self.stop = Some(StopReason::Completed);
            return None;
        }
        let i = self.iter;
        let sigma = diffrast::fit::sigma_at(&self.cfg, i);
        let p = RenderParams::new(self.target.width, self.target.height, sigma);
        self.scene.set_params(&self.params);
        let (loss, grads) = global()
            .backward(&self.scene, p, &self.target)
            .unwrap_or_else(|e| panic!("diffrast-cuda Fitter::step: {e}"));
        if !loss.is_finite() {
            self.stop = Some(StopReason::Diverged);
            return None;
        }
        self.losses.push(loss);
        if loss + self.cfg.min_delta < self.best_loss {
            self.best_loss = loss;
            self.best_iter = i;
            self.best = self.params.clone();
            self.since = 0;
        } else {
            self.since += 1;
        }
        self.iter += 1;
        if let Some(pat) = self.cfg.patience {
            if self.since >= pat {
                self.stop = Some(StopReason::Converged);
                return Some(StepInfo { iter: i, loss, sigma });
            }
        }
        self.adam(&grads);
        Some(StepInfo { iter: i, loss, sigma })
    }

    fn adam(&mut self, grads: &[f32]) {
        let gpu = global();
        let _g = gpu.calls.lock().expect("rasterizer mutex poisoned");
        let t = self.iter as u32;  // Adam::t after its increment at this step
        let cfg = &self.cfg;
        let (params, m, v) = (&mut self.params, &mut self.m, &mut self.v);
        let mut run = || -> Result<(), GpuError> {
            let dp = DeviceBuf::from_host(&gpu.ctx, params)?;
            let dm = DeviceBuf::from_host(&gpu.ctx, m)?;
            let dv = DeviceBuf::from_host(&gpu.ctx, v)?;
            let dg = DeviceBuf::from_host(&gpu.ctx, grads)?;
            // SAFETY: four device arrays of params.len() floats; project = 1
            // applies fit.rs:399-424 after the update.
            check(unsafe {
                ffi::dr_adam_step(gpu.ctx.raw(), dp.f32_mut(), dm.f32_mut(), dv.f32_mut(),
                                  dg.f32(), params.len() as i64, cfg.lr_pos, cfg.lr_color,
                                  cfg.lr_alpha, t, 0.9, 0.999, 1e-8, 1, null_mut())
            })?;
            dp.to_host(params)?;
            dm.to_host(m)?;
            dv.to_host(v)
        };
        run().unwrap_or_else(|e| panic!("diffrast-cuda Fitter::step: {e}"));
    }

    /// The current scene (copied from the device state).
    pub fn scene(&self) -> Scene {
        let mut s = self.scene.clone();
        s.set_params(&self.params);
        s
    }

    pub fn target(&self) -> &Canvas {
        &self.target
    }

    pub fn iter(&self) -> usize {
        self.iter
    }

    pub fn losses(&self) -> &[f32] {
        &self.losses
    }

    pub fn best_loss(&self) -> f32 {
        self.best_loss
    }

    pub fn is_done(&self) -> bool {
        self.stop.is_some() || self.iter >= self.cfg.iters
    }

    pub fn sigma(&self) -> f32 {
        diffrast::fit::sigma_at(&self.cfg, self.iter.min(self.cfg.iters.saturating_sub(1)))
    }

    pub fn render_current(&self) -> Canvas {
        render(&self.scene(), RenderParams::new(self.target.width, self.target.height,
                                                self.sigma()))
    }

    pub fn into_report(self) -> FitReport {
        let mut scene = self.scene.clone();
        scene.set_params(&self.best);
        FitReport {
            scene,
            losses: self.losses,
            stop_reason: self.stop.unwrap_or(StopReason::Completed),
            best_iter: self.best_iter,
            best_loss: self.best_loss,
        }
    }
}

/// The library's version string.
pub fn version() -> String {
    // SAFETY: a static NUL-terminated string.
    unsafe { CStr::from_ptr(ffi::dr_version()).to_string_lossy().into_owned() }
}

/// Parameters per triangle (10), as the library reports it.
pub fn params_per_triangle() -> usize {
    // SAFETY: a constant.
    unsafe { ffi::dr_params_per_triangle() as usize }
}
