//! FFI to librwgpu.so (include/rwgpu.h): the B200 path behind rustwood's `--device gpu`.
//!
//! Drop-in for rustwood's src/ as `src/gpu_ffi.rs` (with `mod gpu_ffi;` in main.rs and
//! the `build.rs` beside this file). It replaces the cuda-oxide module loading and kernel
//! launches of `Booster::fit_inner` (src/booster.rs:227-517) and `Booster::predict`
//! (src/booster.rs:531-555); the host prep before them (`compute_boundaries`, base score)
//! stays in Rust and feeds the `cuts` and `base_score` arguments, and target encoding can
//! move to the GPU through `target_encode` below (same `Encoders` type as
//! src/encoding.rs). Error codes become `Box<dyn Error>`, so `serve_handle` keeps
//! printing `ERROR ...` lines (src/main.rs:406-409).
#![allow(non_camel_case_types)]

use std::collections::HashMap;
use std::error::Error;
use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};
use std::ptr;

pub const RW_OK: c_int = 0;
pub const RW_OBJ_LOGISTIC: i32 = 0;
pub const RW_OBJ_L2: i32 = 1;
pub const RW_N_CATEGORIES: usize = 7;

#[repr(C)]
pub struct rw_ctx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct rw_dataset {
    _p: [u8; 0],
}
#[repr(C)]
pub struct rw_dmodel {
    _p: [u8; 0],
}
#[repr(C)]
pub struct rw_encoders {
    _p: [u8; 0],
}

/// rw_train_params: the Config fields fit_inner reads (src/config.rs:19-88).
#[repr(C)]
pub struct rw_train_params {
    pub n_trees: u32,
    pub depth: u32,
    pub n_bins: u32,
    pub learning_rate: f32,
    pub lambda: f32,
    pub min_child_h: f32,
    pub subsample: f32,
    pub colsample: f32,
    pub monotone: *const i32,
    pub n_monotone: u32,
    pub subtract: i32,
    pub goss_top: f32,
    pub goss_other: f32,
    pub clamp_hessian: f32,
    pub pack4: i32,
    pub pgbm: i32,
    pub objective: i32,
    pub replicas: u32,
    pub smem_hist: i32,
    pub f16_hist: i32,
    pub int_hist: i32,
    pub int_scale: f32,
}

/// rw_profile: per-phase device time of one fit (the reference's profile categories,
/// src/booster.rs:42-52, plus the collective).
#[repr(C)]
#[derive(Default, Clone, Copy)]
pub struct rw_profile {
    pub enable: i32,
    pub total_ms: f64,
    pub category_ms: [f64; RW_N_CATEGORIES],
    pub hist_alg_bytes: f64,
    pub hist_launches: u64,
    pub kernel_launches: u64,
}

/// rw_model: a view of the Booster's model arrays (src/booster.rs:54-69).
#[repr(C)]
pub struct rw_model {
    pub n_trees: u32,
    pub depth: u32,
    pub n_features: u32,
    pub base_score: f32,
    pub feat: *const u32,
    pub thr: *const f32,
    pub thr_bin: *const u16,
    pub leafval: *const f32,
}

#[link(name = "rwgpu")]
extern "C" {
    pub fn rw_ctx_create(gpu_ids: *const c_int, n_gpus: c_int, out: *mut *mut rw_ctx) -> c_int;
    pub fn rw_ctx_create_rank(gpu_id: c_int, rank: c_int, world: c_int, nccl_id: *const c_void,
                              out: *mut *mut rw_ctx) -> c_int;
    pub fn rw_nccl_unique_id(out128: *mut c_void) -> c_int;
    pub fn rw_ctx_destroy(ctx: *mut rw_ctx);
    pub fn rw_last_error(ctx: *const rw_ctx) -> *const c_char;
    pub fn rw_ctx_stream(ctx: *const rw_ctx) -> *mut c_void;
    pub fn rw_ctx_set_timeout(ctx: *mut rw_ctx, ms: i64) -> c_int;
    pub fn rw_ctx_peer_failed(ctx: *const rw_ctx) -> c_int;
    pub fn rw_dataset_create(ctx: *mut rw_ctx, x_rowmajor: *const f32, y: *const f32, n: u64,
                             nf: u32, cuts: *const f32, n_bins: u32, pack4: i32, n_global: u64,
                             row_offset: u64, out: *mut *mut rw_dataset) -> c_int;
    pub fn rw_dataset_create_device(ctx: *mut rw_ctx, d_x: *const f32, d_y: *const f32, n: u64,
                                    nf: u32, cuts: *const f32, n_bins: u32, pack4: i32,
                                    n_global: u64, row_offset: u64,
                                    out: *mut *mut rw_dataset) -> c_int;
    pub fn rw_dataset_destroy(ds: *mut rw_dataset);
    pub fn rw_dataset_bins(ds: *const rw_dataset, out: *mut u8) -> c_int;
    pub fn rw_fit_dataset(ds: *mut rw_dataset, p: *const rw_train_params, base_score: f32,
                          feat: *mut u32, thr: *mut f32, thr_bin: *mut u16, leafval: *mut f32,
                          leafvar: *mut f32, fi_gain: *mut f32, fi_count: *mut f32,
                          prof: *mut rw_profile) -> c_int;
    pub fn rw_fit(ctx: *mut rw_ctx, p: *const rw_train_params, x_rowmajor: *const f32,
                  y: *const f32, n: u64, nf: u32, cuts: *const f32, base_score: f32,
                  feat: *mut u32, thr: *mut f32, thr_bin: *mut u16, leafval: *mut f32,
                  leafvar: *mut f32, fi_gain: *mut f32, fi_count: *mut f32,
                  prof: *mut rw_profile) -> c_int;
    pub fn rw_predict_f32(ctx: *mut rw_ctx, m: *const rw_model, x_rowmajor: *const f32, n: u64,
                          nf: u32, out: *mut f32) -> c_int;
    pub fn rw_predict_u8(ctx: *mut rw_ctx, m: *const rw_model, bins_featmajor: *const u8, n: u64,
                         nf: u32, out: *mut f32) -> c_int;
    pub fn rw_model_upload(ctx: *mut rw_ctx, m: *const rw_model, out: *mut *mut rw_dmodel) -> c_int;
    pub fn rw_model_free(dm: *mut rw_dmodel);
    pub fn rw_predict_u8_device(ctx: *mut rw_ctx, dm: *const rw_dmodel, d_bins: *const u8, n: u64,
                                ld: u64, d_out: *mut f32, kernel_ms: *mut f32) -> c_int;
    pub fn rw_predict_f32_device(ctx: *mut rw_ctx, dm: *const rw_dmodel, d_x: *const f32, n: u64,
                                 d_out: *mut f32, kernel_ms: *mut f32) -> c_int;
    pub fn rw_predict_f32_noalloc(ctx: *mut rw_ctx, m: *const rw_model, x_rowmajor: *const f32,
                                  n: u64, nf: u32, out: *mut f32) -> c_int;
    pub fn rw_predict_var_f32(ctx: *mut rw_ctx, m: *const rw_model, leafvar: *const f32,
                              x_rowmajor: *const f32, n: u64, nf: u32, out: *mut f32) -> c_int;
    pub fn rw_target_encode(ctx: *mut rw_ctx, x_rowmajor: *mut f32, y: *const f32, n: u64, nf: u32,
                            categorical: *const u32, n_cat: u32, smoothing: f32, k_folds: u32,
                            hash_buckets: u64, gmean_out: *mut f32,
                            enc_out: *mut *mut rw_encoders) -> c_int;
    pub fn rw_target_encode_device(ctx: *mut rw_ctx, d_x: *mut f32, d_y: *const f32, n: u64,
                                   nf: u32, categorical: *const u32, n_cat: u32, smoothing: f32,
                                   k_folds: u32, hash_buckets: u64, gmean_out: *mut f32,
                                   enc_out: *mut *mut rw_encoders) -> c_int;
    pub fn rw_encoders_table(enc: *const rw_encoders, i: u32, key_lo: *mut i64, n_keys: *mut u64,
                             value: *mut *const f32, present: *mut *const u8) -> c_int;
    pub fn rw_encoders_free(enc: *mut rw_encoders);
    pub fn rw_encoders_create(n_cat: u32, key_lo: *const i64, n_keys: *const u64,
                              value: *const f32, present: *const u8, gmean: f32,
                              out: *mut *mut rw_encoders) -> c_int;
    pub fn rw_target_transform(ctx: *mut rw_ctx, x_rowmajor: *mut f32, n: u64, nf: u32,
                               categorical: *const u32, n_cat: u32, enc: *const rw_encoders,
                               hash_buckets: u64) -> c_int;
    pub fn rw_model_thr_bins(m: *const rw_model, cuts: *const f32, n_bins: u32,
                             thr_bin: *mut u16) -> c_int;
    pub fn rw_compute_boundaries_device(ctx: *mut rw_ctx, d_x: *const f32, n: u64, nf: u32,
                                        n_bins: u32, sample: u64, unique: i32,
                                        out: *mut f32) -> c_int;
    pub fn rw_fit_with_boundaries(ctx: *mut rw_ctx, p: *const rw_train_params,
                                  x_rowmajor: *const f32, y: *const f32, n: u64, nf: u32,
                                  sample: u64, unique: i32, base_score: f32, cuts_out: *mut f32,
                                  feat: *mut u32, thr: *mut f32, thr_bin: *mut u16,
                                  leafval: *mut f32, leafvar: *mut f32, fi_gain: *mut f32,
                                  fi_count: *mut f32, prof: *mut rw_profile) -> c_int;
}

fn check(ctx: *const rw_ctx, rc: c_int) -> Result<(), Box<dyn Error>> {
    if rc == RW_OK {
        return Ok(());
    }
    let msg = unsafe {
        let p = rw_last_error(ctx);
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    Err(format!("rwgpu error {rc}: {msg}").into())
}

/// One context: one GPU (`CudaContext::new(cfg.gpu)`, src/booster.rs:137), or several GPUs
/// of this host driven by the library, one rank per GPU.
pub struct Context {
    raw: *mut rw_ctx,
}

impl Context {
    pub fn new(gpus: &[i32]) -> Result<Context, Box<dyn Error>> {
        let mut raw = ptr::null_mut();
        let ids: Vec<c_int> = gpus.iter().map(|&g| g as c_int).collect();
        check(ptr::null(), unsafe { rw_ctx_create(ids.as_ptr(), ids.len() as c_int, &mut raw) })?;
        Ok(Context { raw })
    }
    pub fn raw(&self) -> *mut rw_ctx {
        self.raw
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe { rw_ctx_destroy(self.raw) };
    }
}

/// The model arrays a fit fills (the Booster fields of src/booster.rs:54-69).
#[derive(Default)]
pub struct FitOut {
    pub feat: Vec<u32>,
    pub thr: Vec<f32>,
    pub thr_bin: Vec<u16>,
    pub leafval: Vec<f32>,
    /// PGBM leaf variances (filled when `p.pgbm != 0`, as fit_inner keeps `leafvar`)
    pub leafvar: Vec<f32>,
    pub fi_gain: Vec<f32>,
    pub fi_count: Vec<f32>,
    pub profile: rw_profile,
}

/// `fit_inner`'s tree loop on the GPU: x row-major [n][nf] (already target-encoded),
/// cuts [nf][n_bins - 1] from `compute_boundaries`, base_score as fit_inner computes it.
pub fn fit(ctx: &Context, p: &rw_train_params, x: &[f32], y: &[f32], nf: usize, cuts: &[f32],
           base_score: f32, profile: bool) -> Result<FitOut, Box<dyn Error>> {
    let n = y.len();
    assert_eq!(x.len(), n * nf);
    let (t, d) = (p.n_trees as usize, p.depth as usize);
    let mut o = FitOut {
        feat: vec![0; t * d],
        thr: vec![0.0; t * d],
        thr_bin: vec![0; t * d],
        leafval: vec![0.0; t << d],
        leafvar: if p.pgbm != 0 { vec![0.0; t << d] } else { Vec::new() },
        fi_gain: vec![0.0; nf],
        fi_count: vec![0.0; nf],
        profile: rw_profile { enable: profile as i32, ..Default::default() },
    };
    check(ctx.raw, unsafe {
        rw_fit(ctx.raw, p, x.as_ptr(), y.as_ptr(), n as u64, nf as u32, cuts.as_ptr(), base_score,
               o.feat.as_mut_ptr(), o.thr.as_mut_ptr(), o.thr_bin.as_mut_ptr(),
               o.leafval.as_mut_ptr(),
               if p.pgbm != 0 { o.leafvar.as_mut_ptr() } else { ptr::null_mut() },
               o.fi_gain.as_mut_ptr(),
               o.fi_count.as_mut_ptr(), &mut o.profile)
    })?;
    Ok(o)
}

/// `Booster::predict` on the GPU: raw margins of row-major x, accumulated per row in tree
/// order in f32 (bit-identical to `predict_cpu`, src/booster.rs:582-601).
pub fn predict(ctx: &Context, n_trees: usize, depth: usize, n_features: usize, base_score: f32,
               feat: &[u32], thr: &[f32], leafval: &[f32], x: &[f32])
               -> Result<Vec<f32>, Box<dyn Error>> {
    let n = x.len() / n_features.max(1);
    let m = rw_model {
        n_trees: n_trees as u32,
        depth: depth as u32,
        n_features: n_features as u32,
        base_score,
        feat: feat.as_ptr(),
        thr: thr.as_ptr(),
        thr_bin: ptr::null(),
        leafval: leafval.as_ptr(),
    };
    let mut out = vec![0.0f32; n];
    check(ctx.raw, unsafe {
        rw_predict_f32(ctx.raw, &m, x.as_ptr(), n as u64, n_features as u32, out.as_mut_ptr())
    })?;
    Ok(out)
}

/// `Booster::predict_std` (src/booster.rs:559-577): the square root of each row's summed
/// PGBM leaf variance (`predict_var` on the GPU, then `max(0).sqrt()` as the reference).
pub fn predict_std(ctx: &Context, n_trees: usize, depth: usize, n_features: usize, feat: &[u32],
                   thr: &[f32], leafvar: &[f32], x: &[f32]) -> Result<Vec<f32>, Box<dyn Error>> {
    let n = x.len() / n_features.max(1);
    let m = rw_model {
        n_trees: n_trees as u32,
        depth: depth as u32,
        n_features: n_features as u32,
        base_score: 0.0,
        feat: feat.as_ptr(),
        thr: thr.as_ptr(),
        thr_bin: ptr::null(),
        leafval: leafvar.as_ptr(),
    };
    let mut var = vec![0.0f32; n];
    check(ctx.raw, unsafe {
        rw_predict_var_f32(ctx.raw, &m, leafvar.as_ptr(), x.as_ptr(), n as u64,
                           n_features as u32, var.as_mut_ptr())
    })?;
    Ok(var.iter().map(|&v| v.max(0.0).sqrt()).collect())
}

/// `encoding::fit_transform_train` (src/encoding.rs:44-95) on the GPU: encodes the
/// categorical columns of row-major `x` in place and returns `(encoders, gmean)` in the
/// reference's types. Equal to the host function wherever its f64 sums are exact (0/1 or
/// small integer labels); `RW_ERR_UNSUPPORTED` (key range too wide for the GPU's dense
/// tables) means: call the host function instead.
pub fn target_encode(ctx: &Context, x: &mut [f32], n: usize, nf: usize, y: &[f32],
                     categorical: &[usize], smoothing: f32, k_folds: usize, hash_buckets: u64)
                     -> Result<(Vec<HashMap<i64, f32>>, f32), Box<dyn Error>> {
    assert_eq!(x.len(), n * nf);
    let cat: Vec<u32> = categorical.iter().map(|&c| c as u32).collect();
    let mut gmean = 0.0f32;
    let mut enc: *mut rw_encoders = ptr::null_mut();
    check(ctx.raw, unsafe {
        rw_target_encode(ctx.raw, x.as_mut_ptr(), y.as_ptr(), n as u64, nf as u32, cat.as_ptr(),
                         cat.len() as u32, smoothing, k_folds as u32, hash_buckets, &mut gmean,
                         &mut enc)
    })?;
    let mut out = Vec::with_capacity(cat.len());
    for i in 0..cat.len() {
        let (mut lo, mut nk) = (0i64, 0u64);
        let (mut val, mut pres): (*const f32, *const u8) = (ptr::null(), ptr::null());
        unsafe { rw_encoders_table(enc, i as u32, &mut lo, &mut nk, &mut val, &mut pres) };
        let mut m = HashMap::new();
        for j in 0..nk as usize {
            if unsafe { *pres.add(j) } != 0 {
                m.insert(lo + j as i64, unsafe { *val.add(j) });
            }
        }
        out.push(m);
    }
    unsafe { rw_encoders_free(enc) };
    Ok((out, gmean))
}
