"""ctypes binding of include/rwgpu.h (librwgpu.so, built in-tree for sm_100a).

Importing this module loads the library; a missing library raises immediately --
there is no fallback implementation of any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librwgpu.so")

RW_OK = 0
RW_ERR = {
    -1: "RW_ERR_ARG",
    -2: "RW_ERR_OOM",
    -3: "RW_ERR_CUDA",
    -4: "RW_ERR_NCCL",
    -5: "RW_ERR_UNSUPPORTED",
    -6: "RW_ERR_TIMEOUT",
}
RW_OBJ_LOGISTIC, RW_OBJ_L2 = 0, 1
CATEGORIES = ["gradients", "zero_hist", "build_hist", "allreduce", "split_gain", "apply_split",
              "update_pred"]


class TrainParams(C.Structure):
    _fields_ = [
        ("n_trees", C.c_uint32), ("depth", C.c_uint32), ("n_bins", C.c_uint32),
        ("learning_rate", C.c_float), ("lambda_", C.c_float), ("min_child_h", C.c_float),
        ("subsample", C.c_float), ("colsample", C.c_float),
        ("monotone", C.POINTER(C.c_int32)), ("n_monotone", C.c_uint32),
        ("subtract", C.c_int32), ("goss_top", C.c_float), ("goss_other", C.c_float),
        ("clamp_hessian", C.c_float), ("pack4", C.c_int32), ("pgbm", C.c_int32),
        ("objective", C.c_int32), ("replicas", C.c_uint32), ("smem_hist", C.c_int32),
        ("f16_hist", C.c_int32), ("int_hist", C.c_int32), ("int_scale", C.c_float),
    ]


class Profile(C.Structure):
    _fields_ = [
        ("enable", C.c_int32), ("total_ms", C.c_double), ("category_ms", C.c_double * 7),
        ("hist_alg_bytes", C.c_double), ("hist_launches", C.c_uint64),
        ("kernel_launches", C.c_uint64),
    ]


class Model(C.Structure):
    _fields_ = [
        ("n_trees", C.c_uint32), ("depth", C.c_uint32), ("n_features", C.c_uint32),
        ("base_score", C.c_float), ("feat", C.POINTER(C.c_uint32)),
        ("thr", C.POINTER(C.c_float)), ("thr_bin", C.POINTER(C.c_uint16)),
        ("leafval", C.POINTER(C.c_float)),
    ]


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python rustwood_b200/build.py` "
            "(the GPU path has no fallback)")
    lib = C.CDLL(LIB_PATH)
    vp, u64, u32, i32, f32 = C.c_void_p, C.c_uint64, C.c_uint32, C.c_int32, C.c_float
    P = C.POINTER
    sig = {
        "rw_ctx_create": (i32, [P(C.c_int), C.c_int, P(vp)]),
        "rw_ctx_create_rank": (i32, [C.c_int, C.c_int, C.c_int, vp, P(vp)]),
        "rw_nccl_unique_id": (i32, [vp]),
        "rw_ctx_destroy": (None, [vp]),
        "rw_last_error": (C.c_char_p, [vp]),
        "rw_ctx_set_timeout": (i32, [vp, C.c_int64]),
        "rw_ctx_stream": (vp, [vp]),
        "rw_dataset_create": (i32, [vp, vp, vp, u64, u32, vp, u32, i32, u64, u64, P(vp)]),
        "rw_dataset_create_device": (i32, [vp, vp, vp, u64, u32, vp, u32, i32, u64, u64, P(vp)]),
        "rw_dataset_destroy": (None, [vp]),
        "rw_dataset_bins": (i32, [vp, vp]),
        "rw_fit_dataset": (i32, [vp, P(TrainParams), f32, vp, vp, vp, vp, vp, vp, vp,
                                 P(Profile)]),
        "rw_fit": (i32, [vp, P(TrainParams), vp, vp, u64, u32, vp, f32, vp, vp, vp, vp, vp, vp,
                         vp, P(Profile)]),
        "rw_predict_f32": (i32, [vp, P(Model), vp, u64, u32, vp]),
        "rw_predict_u8": (i32, [vp, P(Model), vp, u64, u32, vp]),
        "rw_model_upload": (i32, [vp, P(Model), P(vp)]),
        "rw_model_free": (None, [vp]),
        "rw_predict_u8_device": (i32, [vp, vp, vp, u64, u64, vp, P(f32)]),
        "rw_predict_f32_device": (i32, [vp, vp, vp, u64, vp, P(f32)]),
        "rw_predict_f32_noalloc": (i32, [vp, P(Model), vp, u64, u32, vp]),
        "rw_predict_var_f32": (i32, [vp, P(Model), vp, vp, u64, u32, vp]),
        "rw_target_encode": (i32, [vp, vp, vp, u64, u32, vp, u32, f32, u32, u64, vp, vp]),
        "rw_target_encode_device": (i32, [vp, vp, vp, u64, u32, vp, u32, f32, u32, u64, vp, vp]),
        "rw_encoders_table": (i32, [vp, u32, vp, vp, vp, vp]),
        "rw_encoders_free": (None, [vp]),
        "rw_encoders_create": (i32, [u32, vp, vp, vp, vp, f32, vp]),
        "rw_target_transform": (i32, [vp, vp, u64, u32, vp, u32, vp, u64]),
        "rw_compute_boundaries": (None, [vp, u64, u32, u32, u64, i32, vp]),
        "rw_base_score": (f32, [vp, u64, i32]),
        "rw_model_thr_bins": (i32, [P(Model), vp, u32, vp]),
        "rw_compute_boundaries_device": (i32, [vp, vp, u64, u32, u32, u64, i32, vp]),
        "rw_fit_with_boundaries": (i32, [vp, P(TrainParams), vp, vp, u64, u32, u64, i32, f32, vp,
                                         vp, vp, vp, vp, vp, vp, vp, P(Profile)]),
        "rw_debug_level_hist": (i32, [vp, vp, vp, vp, i32, i32, u32, i32, vp]),
        "rw_debug_expf": (i32, [vp, vp, u64, vp, vp]),
        "rw_debug_binary_version": (i32, [vp, P(i32)]),
        "rw_debug_level_step": (i32, [vp, P(TrainParams), vp, vp, vp, u32, u32, vp, vp, vp]),
        "rw_debug_peer_wait": (i32, [vp, i32, C.c_int64, P(i32), P(f32)]),
        "rw_debug_lonely_rank_ctx": (i32, [C.c_int, C.c_int64, P(vp)]),
        "rw_ctx_peer_failed": (i32, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
EXPORTED = [
    "rw_ctx_create", "rw_ctx_create_rank", "rw_nccl_unique_id", "rw_ctx_destroy",
    "rw_last_error", "rw_ctx_set_timeout", "rw_ctx_stream", "rw_dataset_create", "rw_dataset_create_device",
    "rw_dataset_destroy", "rw_dataset_bins", "rw_fit_dataset", "rw_fit", "rw_predict_f32",
    "rw_predict_u8", "rw_model_upload", "rw_model_free", "rw_predict_u8_device",
    "rw_predict_f32_device", "rw_predict_f32_noalloc", "rw_predict_var_f32",
    "rw_target_encode", "rw_target_encode_device", "rw_encoders_table", "rw_encoders_free",
    "rw_encoders_create", "rw_target_transform", "rw_compute_boundaries", "rw_base_score",
    "rw_model_thr_bins", "rw_compute_boundaries_device", "rw_fit_with_boundaries",
    "rw_debug_level_hist", "rw_debug_expf", "rw_debug_binary_version", "rw_debug_level_step",
    "rw_debug_peer_wait", "rw_debug_lonely_rank_ctx", "rw_ctx_peer_failed",
]


RW_ERR_UNSUPPORTED = -5


class RwError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{RW_ERR.get(code, code)}: {msg}")
        self.code = code


def check(code: int, ctx=None) -> None:
    if code != RW_OK:
        msg = lib.rw_last_error(ctx)
        raise RwError(code, msg.decode() if msg else "")


def ptr(a: np.ndarray | None):
    return None if a is None else C.c_void_p(a.ctypes.data)


def f32c(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)
