"""rustwood's `--serve` worker (src/main.rs:344-416) over one resident librwgpu context.

Protocol, unchanged so the Python wrapper's `_Server` (python/rustwood/__init__.py:65-102)
talks to it as to the Rust binary: every stdin line holds one tab-separated argument list
(the CLI's `--key value` tokens, src/config.rs:140-218); the worker answers with one
status line and a line `__END__`. `QUIT` (or end of input) stops it.
  - with --load-model: read the .rwood model, score the dataset's test rows (on the GPU,
    with the resident context; margins bit-identical to predict_cpu), write them with
    --dump-pred as little-endian f32, answer `OK n=<rows>`;
  - otherwise: fit on the dataset's training rows with the resident context (created
    once, on first use: the CUDA context and the library's state are paid for once per
    worker), save with --save-model, answer `OK train_s=<tree-loop seconds>`;
  - any failure answers `ERROR <stage> <message>` and the worker keeps serving.
Datasets are read from --data as src/data.rs:49-78 writes them: meta.json (n_train,
n_test, n_features) and x_train.bin, y_train.bin, x_test.bin, y_test.bin (f32 LE,
row-major).
Run: python -m rustwood_b200.serve --gpu 0   (or --gpus 0,1,... for one multi-GPU context);
rustwood_b200/rustwood runs the same module with rustwood's command line, for the Python
wrapper's RUSTWOOD_BIN.
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np


def load_dataset(d: str) -> dict:
    """Dataset::load (src/data.rs:49-78)."""
    meta = open(os.path.join(d, "meta.json")).read()

    def meta_int(key):  # the first integer after "key" (src/data.rs:31-46)
        m = re.search(r'"%s"\D*(\d+)' % re.escape(key), meta)
        if not m:
            raise ValueError(f"meta.json missing {key}")
        return int(m.group(1))

    n_train, n_test, nf = meta_int("n_train"), meta_int("n_test"), meta_int("n_features")

    def blob(name, n):
        a = np.fromfile(os.path.join(d, name), dtype="<f4")
        if a.size != n:
            raise ValueError(f"{name} size mismatch")
        return a.astype(np.float32)

    return dict(n_train=n_train, n_test=n_test, n_features=nf,
                x_train=blob("x_train.bin", n_train * nf).reshape(n_train, nf),
                y_train=blob("y_train.bin", n_train),
                x_test=blob("x_test.bin", n_test * nf).reshape(n_test, nf),
                y_test=blob("y_test.bin", n_test))


def write_dataset(d: str, x_train, y_train, x_test, y_test) -> None:
    """The on-disk layout load_dataset reads (what the reference's scripts write)."""
    os.makedirs(d, exist_ok=True)
    json.dump({"n_train": int(len(y_train)), "n_test": int(len(y_test)),
               "n_features": int(x_train.shape[1])}, open(os.path.join(d, "meta.json"), "w"))
    for name, a in (("x_train", x_train), ("y_train", y_train), ("x_test", x_test),
                    ("y_test", y_test)):
        np.ascontiguousarray(a, "<f4").tofile(os.path.join(d, name + ".bin"))


class Worker:
    """serve_handle (src/main.rs:369-416) with the resident context."""

    def __init__(self, gpus):
        self.gpus = list(gpus)
        self.ctx = None

    def context(self):
        from .booster import Context
        if self.ctx is None:
            self.ctx = Context.multi(self.gpus) if len(self.gpus) > 1 else Context(self.gpus[0])
        return self.ctx

    def handle(self, tokens: list[str]) -> str:
        from .booster import Booster
        from .config import GPU, Config
        try:
            cfg = Config.from_tokens(tokens)
        except Exception as e:  # the reference exits on a bad flag; a worker reports it
            return f"ERROR args {e}"
        try:
            ds = load_dataset(cfg.data_dir)
        except Exception as e:
            return f"ERROR data {e}"
        if cfg.load_model:
            try:
                b = Booster.load_model(cfg.load_model, self.context())
            except Exception as e:
                return f"ERROR load {e}"
            try:
                scores = b.predict(ds["x_test"])
            except Exception as e:
                return f"ERROR predict {e}"
            if cfg.dump_pred:
                try:
                    np.ascontiguousarray(scores, "<f4").tofile(cfg.dump_pred)
                except Exception as e:
                    return f"ERROR dump {e}"
            return f"OK n={len(scores)}"
        if cfg.device != GPU:
            return "ERROR new the CPU trainer is rustwood's own (src/cpu.rs)"
        try:
            b = Booster(cfg, self.context())
            t = b.fit(ds["x_train"], ds["y_train"])
        except Exception as e:
            return f"ERROR fit {e}"
        if cfg.save_model:
            try:
                b.save_model(cfg.save_model)
            except Exception as e:
                return f"ERROR save {e}"
        return f"OK train_s={t:.6f}"

    def close(self):
        if self.ctx is not None:
            self.ctx.close()
            self.ctx = None


def serve(gpus, inp=sys.stdin, out=sys.stdout) -> None:
    """The loop of src/main.rs:344-366."""
    w = Worker(gpus)
    try:
        for line in inp:
            line = line.rstrip("\r\n")
            if not line:
                continue
            if line == "QUIT":
                break
            out.write(w.handle(line.split("\t")) + "\n__END__\n")
            out.flush()
    finally:
        w.close()


def main(argv=None) -> int:
    """rustwood's command line (src/main.rs) as far as this worker goes, so the reference's
    Python wrapper can run it as its binary (rustwood_b200/rustwood): `--serve 1`, or a
    command line without `--data`, runs the line protocol on stdin; a command line with
    `--data` and no `--serve` is one request (a fit, or with --load-model a scoring run)
    whose reply goes to stdout, exit status 0 for `OK`, 1 for a failed request, 2 for a
    bad command line. --gpu / --gpus pick the devices."""
    from .config import Config
    argv = list(sys.argv[1:] if argv is None else argv)
    try:
        cfg = Config.from_tokens(argv)
    except Exception as e:
        print(f"ERROR args {e}", flush=True)
        return 2
    gpus = list(cfg.gpus) or [cfg.gpu]
    if cfg.serve or "--data" not in argv[0::2]:
        serve(gpus)
        return 0
    w = Worker(gpus)
    try:
        reply = w.handle(argv)
    finally:
        w.close()
    print(reply, flush=True)
    return 0 if reply.startswith("OK") else 1


if __name__ == "__main__":
    sys.exit(main())
