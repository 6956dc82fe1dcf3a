"""Training configuration: rustwood's Config (src/config.rs:19-218) and its
`--key value` token parser, kept flag-for-flag so the CLI, the `--serve` protocol and
the Python wrapper's argument lists parse unchanged."""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field

LOGISTIC, SQUARED_ERROR = "logistic", "l2"
GPU, CPU = "gpu", "cpu"


def _flag(v: str) -> bool:
    return v in ("1", "true")


@dataclass
class Config:
    """Defaults of src/config.rs:90-131."""
    data_dir: str = "data"
    n_trees: int = 500
    depth: int = 6
    learning_rate: float = 0.1
    n_bins: int = 256
    lambda_: float = 1.0
    min_child_h: float = 1e-3
    subsample: float = 1.0
    colsample: float = 1.0
    unique_bins: bool = False
    categorical: list[int] = field(default_factory=list)
    te_smoothing: float = 10.0
    cat_hash_buckets: int = 0
    monotone: list[int] = field(default_factory=list)
    subtract: bool = True
    goss_top: float = 0.0
    goss_other: float = 0.1
    clamp_hessian: float = 0.0
    pack4: bool = False
    pgbm: bool = False
    smem_hist: bool = False
    f16_hist: bool = False
    int_hist: bool = False
    int_scale: float = 16384.0
    objective: str = LOGISTIC
    bin_sample: int = 200_000
    gpu: int = 0
    # Extension (rustwood trains on one GPU): several GPUs of this host for one Booster,
    # one rank per GPU inside the library (rw_ctx_create with n_gpus > 1).
    gpus: list[int] = field(default_factory=list)
    device: str = GPU
    replicas: int = 64
    profile_out: str = ""
    dump_pred: str = ""
    save_model: str = ""
    load_model: str = ""
    latency_bench: bool = False
    throughput_bench: bool = False
    serve: bool = False

    @classmethod
    def from_tokens(cls, args: list[str]) -> "Config":
        """src/config.rs:140-218: every flag takes one value; unknown flags are errors;
        bins must be in 2..=256 and depth in 1..=12."""
        cfg = cls()
        i = 0
        while i < len(args):
            key = args[i]
            if i + 1 >= len(args):
                raise ValueError(f"missing value for {key}")
            v = args[i + 1]
            setters = {
                "--data": lambda: setattr(cfg, "data_dir", v),
                "--trees": lambda: setattr(cfg, "n_trees", int(v)),
                "--depth": lambda: setattr(cfg, "depth", int(v)),
                "--lr": lambda: setattr(cfg, "learning_rate", float(v)),
                "--bins": lambda: setattr(cfg, "n_bins", int(v)),
                "--lambda": lambda: setattr(cfg, "lambda_", float(v)),
                "--min-child": lambda: setattr(cfg, "min_child_h", float(v)),
                "--subsample": lambda: setattr(cfg, "subsample", float(v)),
                "--colsample": lambda: setattr(cfg, "colsample", float(v)),
                "--unique-bins": lambda: setattr(cfg, "unique_bins", _flag(v)),
                "--te-smoothing": lambda: setattr(cfg, "te_smoothing", float(v)),
                "--cat-hash-buckets": lambda: setattr(cfg, "cat_hash_buckets", int(v)),
                "--subtract": lambda: setattr(cfg, "subtract", _flag(v)),
                "--goss-top": lambda: setattr(cfg, "goss_top", float(v)),
                "--goss-other": lambda: setattr(cfg, "goss_other", float(v)),
                "--clamp-hessian": lambda: setattr(cfg, "clamp_hessian", float(v)),
                "--pack4": lambda: setattr(cfg, "pack4", _flag(v)),
                "--pgbm": lambda: setattr(cfg, "pgbm", _flag(v)),
                "--smem-hist": lambda: setattr(cfg, "smem_hist", _flag(v)),
                "--f16-hist": lambda: setattr(cfg, "f16_hist", _flag(v)),
                "--int-hist": lambda: setattr(cfg, "int_hist", _flag(v)),
                "--int-scale": lambda: setattr(cfg, "int_scale", float(v)),
                "--monotone": lambda: setattr(cfg, "monotone",
                                              [int(s) for s in v.split(",") if s]),
                "--categorical": lambda: setattr(cfg, "categorical",
                                                 [int(s) for s in v.split(",") if s]),
                "--bin-sample": lambda: setattr(cfg, "bin_sample", int(v)),
                "--gpu": lambda: setattr(cfg, "gpu", int(v)),
                "--gpus": lambda: setattr(cfg, "gpus", [int(s) for s in v.split(",") if s]),
                "--device": lambda: setattr(cfg, "device", _device(v)),
                "--replicas": lambda: setattr(cfg, "replicas", int(v)),
                "--profile-out": lambda: setattr(cfg, "profile_out", v),
                "--save-model": lambda: setattr(cfg, "save_model", v),
                "--load-model": lambda: setattr(cfg, "load_model", v),
                "--dump-pred": lambda: setattr(cfg, "dump_pred", v),
                "--latency-bench": lambda: setattr(cfg, "latency_bench", _flag(v)),
                "--throughput-bench": lambda: setattr(cfg, "throughput_bench", _flag(v)),
                "--serve": lambda: setattr(cfg, "serve", _flag(v)),
                "--objective": lambda: setattr(cfg, "objective", _objective(v)),
            }
            if key not in setters:
                raise ValueError(f"unknown flag {key}")
            setters[key]()
            i += 2
        if not 2 <= cfg.n_bins <= 256:
            raise ValueError("n_bins must be in 2..=256")
        if not 1 <= cfg.depth <= 12:
            raise ValueError("depth must be in 1..=12")
        return cfg

    def replace(self, **kw) -> "Config":
        return dataclasses.replace(self, **kw)


def _device(v: str) -> str:
    if v in ("gpu", "cuda"):
        return GPU
    if v in ("cpu", "host"):
        return CPU
    raise ValueError(f"unknown device {v}")


def _objective(v: str) -> str:
    if v in ("logistic", "binary"):
        return LOGISTIC
    if v in ("l2", "rmse", "reg"):
        return SQUARED_ERROR
    raise ValueError(f"unknown objective {v}")
