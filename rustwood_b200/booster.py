"""Booster: the host mirror of rustwood's `Booster` (src/booster.rs) over librwgpu.

fit() performs fit_inner's host prep (target encoding, cut table, base score,
src/booster.rs:246-285) and hands the tree loop to the GPU through rw_fit_dataset;
predict() is Booster::predict (raw margins, src/booster.rs:531-555) on the GPU;
save_model()/load_model() read and write the `.rwood` v1 format byte-compatibly
(src/booster.rs:797-878). The CPU trainer (`--device cpu`, src/cpu.rs) is the
reference's own code and is not reimplemented here.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from . import _native as N
from . import encoding
from .config import LOGISTIC, Config


class Context:
    """One GPU (and optionally one NCCL rank of a multi-process job): rw_ctx_create_rank.
    Context.multi(gpus) drives several GPUs from this process: rw_ctx_create."""

    def __init__(self, gpu: int = 0, rank: int = 0, world: int = 1, nccl_id: bytes | None = None):
        h = C.c_void_p()
        idb = None if nccl_id is None else C.create_string_buffer(nccl_id, 128)
        N.check(N.lib.rw_ctx_create_rank(gpu, rank, world, idb, C.byref(h)))
        self.h = h
        self.gpu, self.rank, self.world = gpu, rank, world

    @classmethod
    def multi(cls, gpus) -> "Context":
        """One context over several GPUs of this host (one rank per GPU inside the
        library): fits shard rows and exchange histograms, scoring shards rows."""
        gpus = [int(g) for g in gpus]
        ids = (C.c_int * len(gpus))(*gpus)
        h = C.c_void_p()
        N.check(N.lib.rw_ctx_create(ids, len(gpus), C.byref(h)))
        self = cls.__new__(cls)
        self.h = h
        self.gpu, self.rank, self.world = gpus[0], 0, len(gpus)
        return self

    def close(self):
        if self.h:
            N.lib.rw_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, code: int):
        N.check(code, self.h)

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        N.check(N.lib.rw_nccl_unique_id(buf))
        return buf.raw


def train_params(cfg: Config) -> N.TrainParams:
    p = N.TrainParams()
    p.n_trees, p.depth, p.n_bins = cfg.n_trees, cfg.depth, cfg.n_bins
    p.learning_rate, p.lambda_, p.min_child_h = cfg.learning_rate, cfg.lambda_, cfg.min_child_h
    p.subsample, p.colsample = cfg.subsample, cfg.colsample
    mono = np.ascontiguousarray(cfg.monotone, dtype=np.int32)
    p._mono_keepalive = mono  # the array must outlive the call
    p.monotone = mono.ctypes.data_as(C.POINTER(C.c_int32)) if len(mono) else None
    p.n_monotone = len(mono)
    p.subtract = int(cfg.subtract)
    p.goss_top, p.goss_other, p.clamp_hessian = cfg.goss_top, cfg.goss_other, cfg.clamp_hessian
    p.pack4, p.pgbm = int(cfg.pack4), int(cfg.pgbm)
    p.objective = N.RW_OBJ_LOGISTIC if cfg.objective == LOGISTIC else N.RW_OBJ_L2
    p.replicas, p.smem_hist, p.f16_hist = cfg.replicas, int(cfg.smem_hist), int(cfg.f16_hist)
    p.int_hist, p.int_scale = int(cfg.int_hist), cfg.int_scale
    return p


def target_encode_gpu(ctx: "Context", x: np.ndarray, y: np.ndarray, categorical, smoothing: float,
                      k_folds: int = 5, hash_buckets: int = 0):
    """encoding.fit_transform_train on the GPU (rw_target_encode): x (row-major float32,
    C-contiguous) is encoded in place; returns (encoders, gmean) like the host version,
    encoders[i] a dict code -> float32. Raises N.RwError (code RW_ERR_UNSUPPORTED) when a
    feature's key range is too wide for the GPU's dense tables."""
    assert x.dtype == np.float32 and x.flags.c_contiguous
    y = N.f32c(y)
    cat = np.ascontiguousarray(categorical, np.uint32)
    gmean = C.c_float()
    enc = C.c_void_p()
    n, nf = x.shape
    ctx.check(N.lib.rw_target_encode(ctx.h, N.ptr(x), N.ptr(y), n, nf, N.ptr(cat), len(cat),
                                     float(smoothing), int(k_folds), int(hash_buckets),
                                     C.byref(gmean), C.byref(enc)))
    encoders = []
    try:
        for i in range(len(cat)):
            lo, nk = C.c_int64(), C.c_uint64()
            val, pres = C.POINTER(C.c_float)(), C.POINTER(C.c_uint8)()
            N.lib.rw_encoders_table(enc, i, C.byref(lo), C.byref(nk), C.byref(val), C.byref(pres))
            v = np.ctypeslib.as_array(val, (nk.value,)).copy() if nk.value else np.zeros(0, np.float32)
            pr = np.ctypeslib.as_array(pres, (nk.value,)).copy() if nk.value else np.zeros(0, np.uint8)
            idx = np.nonzero(pr)[0]
            encoders.append({int(lo.value + j): np.float32(v[j]) for j in idx})
    finally:
        N.lib.rw_encoders_free(enc)
    return encoders, np.float32(gmean.value)


def target_transform_gpu(ctx: "Context", x: np.ndarray, categorical, encoders, gmean,
                         hash_buckets: int = 0, max_slots: int = 1 << 26) -> bool:
    """encoding.transform on the GPU (rw_target_transform) from dense tables of the
    encoders (dicts code -> float32): x (row-major float32, C-contiguous) is transformed in
    place. Returns False, leaving x untouched, when the encoders' key ranges would need more
    than max_slots table slots (the caller then uses the host transform)."""
    assert x.dtype == np.float32 and x.flags.c_contiguous
    lo, nk, tables = [], [], []
    for m in encoders:
        if m:
            keys = np.fromiter(m.keys(), dtype=np.int64, count=len(m))
            a, b = int(keys.min()), int(keys.max())
            lo.append(a)
            nk.append(b - a + 1)
        else:
            lo.append(0)
            nk.append(0)
        if sum(nk) > max_slots:
            return False
    value = np.zeros(sum(nk), np.float32)
    present = np.zeros(sum(nk), np.uint8)
    base = 0
    for m, a, k in zip(encoders, lo, nk):
        for key, v in m.items():
            value[base + key - a] = v
            present[base + key - a] = 1
        base += k
    lo_a, nk_a = np.asarray(lo, np.int64), np.asarray(nk, np.uint64)
    cat = np.ascontiguousarray(categorical, np.uint32)
    enc = C.c_void_p()
    rc = N.lib.rw_encoders_create(len(cat), N.ptr(lo_a), N.ptr(nk_a), N.ptr(value),
                                  N.ptr(present), float(gmean), C.byref(enc))
    if rc != N.RW_OK:
        raise N.RwError(rc, "rw_encoders_create")
    try:
        n, nf = x.shape
        ctx.check(N.lib.rw_target_transform(ctx.h, N.ptr(x), n, nf, N.ptr(cat), len(cat), enc,
                                            int(hash_buckets)))
    finally:
        N.lib.rw_encoders_free(enc)
    return True


def compute_boundaries(x: np.ndarray, n_bins: int, sample: int = 200_000,
                       unique: bool = False) -> np.ndarray:
    """src/data.rs:86-146 (native)."""
    x = N.f32c(x)
    n, nf = x.shape
    out = np.empty(nf * (n_bins - 1), dtype=np.float32)
    N.lib.rw_compute_boundaries(N.ptr(x), n, nf, n_bins, sample, int(unique), N.ptr(out))
    return out


def base_score(y: np.ndarray, objective: str) -> float:
    """src/booster.rs:201-205 (native)."""
    y = N.f32c(y)
    return float(N.lib.rw_base_score(N.ptr(y), len(y),
                                     N.RW_OBJ_LOGISTIC if objective == LOGISTIC else N.RW_OBJ_L2))


class Dataset:
    """A device-resident binned training shard (rw_dataset)."""

    def __init__(self, ctx: Context, x: np.ndarray, y: np.ndarray, cuts: np.ndarray, n_bins: int,
                 pack4: bool = False, n_global: int | None = None, row_offset: int = 0):
        x, y, cuts = N.f32c(x), N.f32c(y), N.f32c(cuts)
        n, nf = x.shape
        h = C.c_void_p()
        ctx.check(N.lib.rw_dataset_create(ctx.h, N.ptr(x), N.ptr(y), n, nf, N.ptr(cuts), n_bins,
                                          int(pack4), n if n_global is None else n_global,
                                          row_offset, C.byref(h)))
        self.ctx, self.h, self.n, self.nf, self.n_bins = ctx, h, n, nf, n_bins

    @classmethod
    def from_device(cls, ctx: Context, x_ptr: int, y_ptr: int, n: int, nf: int, cuts: np.ndarray,
                    n_bins: int, pack4: bool = False, n_global: int | None = None,
                    row_offset: int = 0) -> "Dataset":
        self = cls.__new__(cls)
        cuts = N.f32c(cuts)
        h = C.c_void_p()
        ctx.check(N.lib.rw_dataset_create_device(ctx.h, C.c_void_p(x_ptr), C.c_void_p(y_ptr), n,
                                                 nf, N.ptr(cuts), n_bins, int(pack4),
                                                 n if n_global is None else n_global, row_offset,
                                                 C.byref(h)))
        self.ctx, self.h, self.n, self.nf, self.n_bins = ctx, h, n, nf, n_bins
        return self

    def bins(self) -> np.ndarray:
        out = np.empty((self.nf, self.n), dtype=np.uint8)
        self.ctx.check(N.lib.rw_dataset_bins(self.h, N.ptr(out)))
        return out

    def close(self):
        # a dataset lives in its context's memory pool: once the context is destroyed the
        # dataset's memory is gone with it and the handle must not be used again
        if self.h and self.ctx.h:
            N.lib.rw_dataset_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class FitResult:
    def __init__(self, T, D, nf):
        self.feat = np.zeros(T * D, dtype=np.uint32)
        self.thr = np.zeros(T * D, dtype=np.float32)
        self.thr_bin = np.zeros(T * D, dtype=np.uint16)
        self.leafval = np.zeros(T << D, dtype=np.float32)
        self.leafvar = np.zeros(0, dtype=np.float32)  # PGBM leaf variances (cfg.pgbm)
        self.fi_gain = np.zeros(nf, dtype=np.float32)
        self.fi_count = np.zeros(nf, dtype=np.float32)
        self.profile = N.Profile()


def fit_dataset(ds: Dataset, cfg: Config, base: float, profile: bool = False) -> FitResult:
    """rw_fit_dataset: the tree loop on a prepared dataset."""
    r = FitResult(cfg.n_trees, cfg.depth, ds.nf)
    p = train_params(cfg)
    r.profile.enable = int(profile)
    if cfg.pgbm:  # fit_inner keeps the leaf variances when cfg.pgbm (src/booster.rs:511-513)
        r.leafvar = np.zeros(cfg.n_trees << cfg.depth, dtype=np.float32)
    ds.ctx.check(N.lib.rw_fit_dataset(ds.h, C.byref(p), base, N.ptr(r.feat), N.ptr(r.thr),
                                      N.ptr(r.thr_bin), N.ptr(r.leafval),
                                      N.ptr(r.leafvar) if cfg.pgbm else None, N.ptr(r.fi_gain),
                                      N.ptr(r.fi_count), C.byref(r.profile)))
    return r


class Booster:
    """src/booster.rs:54-69 fields; GPU fit/predict through librwgpu."""

    def __init__(self, cfg: Config, ctx: Context | None = None):
        if cfg.device != "gpu":
            raise NotImplementedError(
                "this library implements the --device gpu path; the CPU trainer is src/cpu.rs")
        self.cfg = cfg
        self._ctx = ctx
        self.n_features = 0
        self.base_score = 0.0
        self.feat = np.zeros(0, np.uint32)
        self.thr = np.zeros(0, np.float32)
        self.thr_bin = np.zeros(0, np.uint16)
        self.leafval = np.zeros(0, np.float32)
        self.leafvar = np.zeros(0, np.float32)
        self.encoders: list[dict] = []
        self.gmean = 0.0
        self.fi_gain = np.zeros(0, np.float32)
        self.fi_count = np.zeros(0, np.float32)
        self.cuts = np.zeros(0, np.float32)
        self.last_profile = None

    @property
    def ctx(self) -> Context:
        """The GPU context, created on first use (model I/O needs none)."""
        if self._ctx is None:
            self._ctx = (Context.multi(self.cfg.gpus) if len(self.cfg.gpus) > 1
                         else Context(self.cfg.gpus[0] if self.cfg.gpus else self.cfg.gpu))
        return self._ctx

    # -- training ----------------------------------------------------------------
    def prepare(self, x: np.ndarray, y: np.ndarray):
        """fit_inner's host prep (src/booster.rs:246-285): returns (x_encoded, cuts, base)."""
        x, y = self._encode_train(x, y)
        cuts = compute_boundaries(x, self.cfg.n_bins, self.cfg.bin_sample, self.cfg.unique_bins)
        return x, cuts, base_score(y, self.cfg.objective)

    def _encode_train(self, x: np.ndarray, y: np.ndarray):
        """encoding::fit_transform_train of the training rows (a C-contiguous float32 copy)
        when the config has categorical features; y as float32."""
        cfg = self.cfg
        x = np.array(x, dtype=np.float32, order="C", copy=True)
        y = N.f32c(y)
        if cfg.categorical:
            # on the GPU (exact fixed-point sums); the host restatement when there is no
            # GPU or the key range is too wide for the GPU's dense tables
            try:
                self.encoders, self.gmean = target_encode_gpu(
                    self.ctx, x, y, cfg.categorical, cfg.te_smoothing, 5, cfg.cat_hash_buckets)
            except N.RwError as e:
                if e.code == N.RW_ERR_UNSUPPORTED or self._ctx is None:
                    self.encoders, self.gmean = encoding.fit_transform_train(
                        x, y, cfg.categorical, cfg.te_smoothing, 5, cfg.cat_hash_buckets)
                else:
                    raise
        return x, y

    def fit(self, x: np.ndarray, y: np.ndarray, profile: bool = False) -> float:
        """Booster::fit (src/booster.rs:169-181) for the GPU device; returns the tree-loop
        time in seconds (what the reference reports as train_s). One call of
        rw_fit_with_boundaries: the rows are uploaded once and serve both the cut table
        (compute_boundaries on the GPU, bit-identical to the host restatement) and the
        binning; the cut table comes back in self.cuts."""
        cfg = self.cfg
        x, y = self._encode_train(x, y)
        n, nf = x.shape
        base = base_score(y, cfg.objective)
        self.n_features = nf
        self.base_score = base
        cuts = np.empty(nf * (cfg.n_bins - 1), dtype=np.float32)
        r = FitResult(cfg.n_trees, cfg.depth, nf)
        p = train_params(cfg)
        r.profile.enable = int(profile)
        if cfg.pgbm:
            r.leafvar = np.zeros(cfg.n_trees << cfg.depth, dtype=np.float32)
        self.ctx.check(N.lib.rw_fit_with_boundaries(
            self.ctx.h, C.byref(p), N.ptr(x), N.ptr(y), n, nf, cfg.bin_sample,
            int(cfg.unique_bins), base, N.ptr(cuts), N.ptr(r.feat), N.ptr(r.thr),
            N.ptr(r.thr_bin), N.ptr(r.leafval), N.ptr(r.leafvar) if cfg.pgbm else None,
            N.ptr(r.fi_gain), N.ptr(r.fi_count), C.byref(r.profile)))
        self.cuts = cuts
        self._take(r)
        return r.profile.total_ms / 1e3

    def _take(self, r: FitResult):
        self.feat, self.thr, self.thr_bin, self.leafval = r.feat, r.thr, r.thr_bin, r.leafval
        self.leafvar = r.leafvar
        self.fi_gain, self.fi_count = r.fi_gain, r.fi_count
        self.last_profile = r.profile

    # -- scoring -----------------------------------------------------------------
    def model(self) -> tuple[N.Model, list]:
        m = N.Model()
        m.n_trees, m.depth, m.n_features = self.cfg.n_trees, self.cfg.depth, self.n_features
        m.base_score = self.base_score
        keep = [np.ascontiguousarray(self.feat, np.uint32), np.ascontiguousarray(self.thr, np.float32),
                np.ascontiguousarray(self.leafval, np.float32)]
        m.feat = keep[0].ctypes.data_as(C.POINTER(C.c_uint32))
        m.thr = keep[1].ctypes.data_as(C.POINTER(C.c_float))
        m.leafval = keep[2].ctypes.data_as(C.POINTER(C.c_float))
        if len(self.thr_bin) == len(self.feat) and len(self.feat):
            keep.append(np.ascontiguousarray(self.thr_bin, np.uint16))
            m.thr_bin = keep[-1].ctypes.data_as(C.POINTER(C.c_uint16))
        return m, keep

    def _encode_rows(self, x: np.ndarray) -> None:
        """encoding::transform of new rows (src/encoding.rs:96-115), in place: on the GPU
        from dense tables of the encoders (rw_target_transform), on the host when their
        key range is too wide for dense tables."""
        if not target_transform_gpu(self.ctx, x, self.cfg.categorical, self.encoders,
                                    self.gmean, self.cfg.cat_hash_buckets):
            encoding.transform(x, self.cfg.categorical, self.encoders, self.gmean,
                               self.cfg.cat_hash_buckets)

    def predict(self, x: np.ndarray) -> np.ndarray:
        """Raw margins on the GPU (Booster::predict)."""
        x = np.array(x, dtype=np.float32, order="C", copy=bool(self.cfg.categorical))
        if self.cfg.categorical:
            self._encode_rows(x)
        n = x.shape[0]
        out = np.empty(n, dtype=np.float32)
        m, _keep = self.model()
        self.ctx.check(N.lib.rw_predict_f32(self.ctx.h, C.byref(m), N.ptr(x), n, x.shape[1],
                                            N.ptr(out)))
        return out

    def predict_std(self, x: np.ndarray) -> np.ndarray:
        """Booster::predict_std (src/booster.rs:559-577): per row the square root of the
        summed PGBM leaf variances (rw_predict_var_f32), max(0).sqrt() in f32."""
        if self.cfg.n_trees and len(self.leafvar) != (self.cfg.n_trees << self.cfg.depth):
            raise RuntimeError("no leaf variances: fit with pgbm=True")
        x = np.array(x, dtype=np.float32, order="C", copy=bool(self.cfg.categorical))
        if self.cfg.categorical:
            self._encode_rows(x)
        n = x.shape[0]
        var = np.empty(n, dtype=np.float32)
        m, _keep = self.model()
        lv = np.ascontiguousarray(self.leafvar, np.float32)
        self.ctx.check(N.lib.rw_predict_var_f32(self.ctx.h, C.byref(m), N.ptr(lv), N.ptr(x), n,
                                                x.shape[1], N.ptr(var)))
        return np.sqrt(np.maximum(var, np.float32(0.0)))

    def predict_bins(self, bins_featmajor: np.ndarray) -> np.ndarray:
        """Raw margins from pre-binned feature-major u8 rows (rw_predict_u8)."""
        b = np.ascontiguousarray(bins_featmajor, dtype=np.uint8)
        nf, n = b.shape
        out = np.empty(n, dtype=np.float32)
        m, _keep = self.model()
        self.ctx.check(N.lib.rw_predict_u8(self.ctx.h, C.byref(m), N.ptr(b), n, nf, N.ptr(out)))
        return out

    def set_cut_table(self, cuts: np.ndarray, n_bins: int | None = None) -> None:
        """Recover the u8 scorer's thresholds (rw_model_thr_bins) of a model that carries
        raw thresholds only, e.g. one read from a .rwood v1 file, from the cut table it was
        trained with; predict_bins() then scores rows binned against that table."""
        nb = self.cfg.n_bins if n_bins is None else n_bins
        cuts = N.f32c(cuts)
        m, _keep = self.model()
        tb = np.zeros(len(self.feat), np.uint16)
        N.check(N.lib.rw_model_thr_bins(C.byref(m), N.ptr(cuts), nb, N.ptr(tb)))
        self.thr_bin = tb
        self.cuts = cuts

    def feature_importance(self):
        return self.fi_gain, self.fi_count

    # -- .rwood v1 (src/booster.rs:797-878) ----------------------------------------
    def save_model(self, path: str) -> None:
        cfg = self.cfg
        with open(path, "wb") as f:
            f.write(b"RWD1")
            f.write(struct.pack("<5I", 1, self.n_features, cfg.n_trees, cfg.depth,
                                int(cfg.objective == LOGISTIC)))
            f.write(struct.pack("<ffQ", self.base_score, self.gmean, cfg.cat_hash_buckets))
            f.write(struct.pack("<I", len(cfg.categorical)))
            for c in cfg.categorical:
                f.write(struct.pack("<I", c))
            for arr, dt in ((self.feat, "<u4"), (self.thr, "<f4"), (self.leafval, "<f4")):
                a = np.ascontiguousarray(arr, dtype=dt)
                f.write(struct.pack("<I", len(a)))
                f.write(a.tobytes())
            f.write(struct.pack("<I", len(self.encoders)))
            for mp in self.encoders:
                f.write(struct.pack("<I", len(mp)))
                for k in sorted(mp):
                    f.write(struct.pack("<qf", k, float(mp[k])))

    @classmethod
    def load_model(cls, path: str, ctx: Context | None = None) -> "Booster":
        with open(path, "rb") as f:
            data = f.read()
        if data[:4] != b"RWD1":
            raise ValueError("not a .rwood file")
        off = 4
        _ver, nf, nt, depth, logistic = struct.unpack_from("<5I", data, off)
        off += 20
        base, gmean, hb = struct.unpack_from("<ffQ", data, off)
        off += 16
        (ncat,) = struct.unpack_from("<I", data, off)
        off += 4
        cats = list(struct.unpack_from(f"<{ncat}I", data, off))
        off += 4 * ncat

        def arr(dt):
            nonlocal off
            (ln,) = struct.unpack_from("<I", data, off)
            off += 4
            a = np.frombuffer(data, dtype=dt, count=ln, offset=off).copy()
            off += 4 * ln
            return a

        feat, thr, leafval = arr("<u4"), arr("<f4"), arr("<f4")
        (nenc,) = struct.unpack_from("<I", data, off)
        off += 4
        encs = []
        for _ in range(nenc):
            (ml,) = struct.unpack_from("<I", data, off)
            off += 4
            mp = {}
            for _ in range(ml):
                k, v = struct.unpack_from("<qf", data, off)
                off += 12
                mp[k] = np.float32(v)
            encs.append(mp)
        cfg = Config(n_trees=nt, depth=depth, objective=LOGISTIC if logistic == 1 else "l2",
                     categorical=cats, cat_hash_buckets=hb)
        b = cls(cfg, ctx)
        b.n_features, b.base_score, b.gmean = nf, np.float32(base), np.float32(gmean)
        b.feat, b.thr, b.leafval, b.encoders = feat, thr, leafval, encs
        b.thr_bin = np.zeros(0, np.uint16)
        return b
