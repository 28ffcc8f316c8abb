"""The oracle restatement against golden vectors from the reference's own modules."""
import json
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
import nafnet_oracle as O  # noqa: E402

GOLDEN = os.path.join(HERE, "golden")
# model and layer cases (the frame-level tiling / flip cases are in test_infer.py)
CASES = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz") and not f.startswith(("tile_", "flip_")))


def load_case(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def case_params(synth, meta):
    cfg = synth.NAFConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in meta["cfg"].items()})
    tk = {"spatial": None, "temporal_py": "py", "temporal_legacy": "legacy"}[meta["kind"]]
    specs = synth.param_specs(cfg, tk, meta["frames"], meta["warp"])
    return O.as_torch(synth.round_fp16(synth.init_params(specs, meta["wseed"])))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_golden(pkg, name):
    import importlib

    synth = importlib.import_module(pkg.__name__ + ".synth")
    z = load_case(name)
    meta = json.loads(str(z["meta"]))
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if meta["kind"] == "dcn":
        y = O.deform_conv2d(torch.from_numpy(z["x"]), torch.from_numpy(z["offsets"]),
                            torch.from_numpy(z["masks"]), torch.from_numpy(z["weight"]),
                            torch.from_numpy(z["bias"]), pad=meta["pad"], deform_groups=meta["dg"])
    else:
        p = case_params(synth, meta)
        x = torch.from_numpy(z["x"])
        fwd = {"spatial": O.nafnet_forward, "temporal_py": O.nafnet_temporal_forward,
               "temporal_legacy": O.nafnet_temporal_legacy_forward}[meta["kind"]]
        y = fwd(p, x)
    exp = torch.from_numpy(z["expected"])
    assert y.shape == exp.shape
    err = (y - exp).abs().max().item()
    assert err < 2e-5, f"{name}: oracle vs reference max abs diff {err}"
