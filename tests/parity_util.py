"""Shared helpers of the GPU parity tests (engine vs oracle / golden vectors)."""
import importlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))

# Acceptance bar of the engine against fp32: the reference's own parity
# threshold (tests/test_unet_forward.cc:207, README.md:948) and >= 50 dB PSNR.
MAX_ABS = 5e-3
MIN_PSNR = 50.0


def synth_mod(pkg):
    return importlib.import_module(pkg.__name__ + ".synth")


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(str(d["meta"]))
    return d


def golden_model_dir(pkg, tmp, meta):
    synth = synth_mod(pkg)
    cfg = synth.NAFConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in meta["cfg"].items()})
    tk = {"spatial": None, "temporal_py": "py", "temporal_legacy": "legacy"}[meta["kind"]]
    path, params = synth.make_model_dir(str(tmp), cfg, meta["wseed"], tk, meta["frames"], meta["warp"])
    return path, params


def compare(out, ref):
    """(max abs diff, psnr) of two float arrays / tensors."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(out - ref)
    mse = float((d ** 2).mean())
    psnr = float("inf") if mse == 0 else 10 * np.log10(1.0 / mse)
    return float(d.max()), psnr
