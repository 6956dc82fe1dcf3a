"""The C-ABI library loads and exports every entry point include/rwgpu.h declares
(no compute calls: these run without a GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle
from rustwood_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "rwgpu.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(rw_[a-z0-9_]+)\s*\(", hdr)))


def test_every_declared_symbol_is_exported():
    syms = declared_symbols()
    assert len(syms) >= 20
    lib = ctypes.CDLL(N.LIB_PATH)
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(N.EXPORTED) == syms


def test_library_build_targets_sm100a_only():
    """The build compiles SASS for sm_100a and nothing else (no PTX for JIT, no other
    arch); the GPU suite checks the loaded kernels' architecture at run time."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "rw_build", os.path.join(ROOT, "rustwood_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    cmd = mod.nvcc_command()
    gencodes = [cmd[i + 1] for i, a in enumerate(cmd) if a == "-gencode"]
    assert gencodes == ["arch=compute_100a,code=sm_100a"]


@pytest.mark.gpu
def test_loaded_kernels_run_as_sm100(ctx):
    v = ctypes.c_int32()
    ctx.check(N.lib.rw_debug_binary_version(ctx.h, ctypes.byref(v)))
    assert v.value == 100


def test_context_without_device_reports_an_error():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    h = ctypes.c_void_p()
    rc = N.lib.rw_ctx_create_rank(0, 0, 1, None, ctypes.byref(h))
    assert rc != 0
    assert N.lib.rw_last_error(None)


def test_bad_arguments_fail_cleanly():
    h = ctypes.c_void_p()
    assert N.lib.rw_ctx_create_rank(0, 2, 2, None, ctypes.byref(h)) == -1  # rank >= world
    assert N.lib.rw_ctx_create(None, 2, ctypes.byref(h)) == -1  # no GPU list
    assert N.lib.rw_ctx_create(None, 9, ctypes.byref(h)) == -1  # more GPUs than ranks allowed
    ids = (ctypes.c_int * 2)(0, 0)
    # a repeated GPU is refused before any device is touched only when devices exist; on
    # a machine without GPUs the device query fails first -- either way, an error
    assert N.lib.rw_ctx_create(ids, 2, ctypes.byref(h)) in (-1, -3)
    assert N.lib.rw_nccl_unique_id(None) == -1


@pytest.mark.parametrize("seed,n,nf,nb,uniq", [
    (0, 10_000, 5, 255, False), (1, 3_000, 3, 16, False), (2, 5_000, 4, 64, True),
    (3, 17, 2, 255, False), (4, 900, 3, 255, True), (5, 250_000, 2, 255, False),
])
def test_host_boundaries_and_base_score_match_oracle(seed, n, nf, nb, uniq):
    import rustwood_b200 as rb
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, nf)).astype(np.float32)
    x[:, 0] = np.round(x[:, 0] * 3)  # ties / low cardinality
    got = rb.compute_boundaries(x, nb, 200_000, uniq)
    want = oracle.compute_boundaries(x, nb, 200_000, uniq)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    y = (rng.random(n) < 0.3).astype(np.float32)
    for obj in ("logistic", "l2"):
        assert np.float32(rb.base_score(y, obj)) == np.float32(oracle.base_score(y, obj))


def _c_struct_fields(hdr, name):
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), hdr, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        # "uint32_t n_trees, depth" / "const float* thr" / "double category_ms[7]"
        names = decl.split(None, 1)[1] if not decl.startswith("const") else decl.split(None, 2)[2]
        for nm in names.split(","):
            fields.append(re.sub(r"[\s*]|\[.*\]", "", nm))
    return fields


def _rust_struct_fields(src, name):
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, src, re.S).group(1)
    return re.findall(r"pub (\w+):", body)


def test_rust_shim_binds_the_public_abi():
    """The Rust binding (rustwood_b200/rust/gpu_ffi.rs, what rustwood links) declares every
    public entry point of include/rwgpu.h, and its #[repr(C)] structs list the C fields in
    the C order (cargo is not available here to compile it)."""
    hdr = open(os.path.join(ROOT, "include", "rwgpu.h")).read()
    src = open(os.path.join(ROOT, "rustwood_b200", "rust", "gpu_ffi.rs")).read()
    public = [s for s in declared_symbols()
              if not s.startswith("rw_debug_") and s not in ("rw_compute_boundaries",
                                                              "rw_base_score")]
    bound = set(re.findall(r"pub fn (rw_\w+)\(", src))
    assert not [s for s in public if s not in bound], [s for s in public if s not in bound]
    for c_name in ("rw_train_params", "rw_profile", "rw_model"):
        assert _rust_struct_fields(src, c_name) == _c_struct_fields(hdr, c_name), c_name
