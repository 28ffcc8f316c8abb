"""Manifest + .bin format handling (mirrors the reference's tests/test_weight_loader.cc)."""
import importlib
import json
import os

import numpy as np
import pytest


@pytest.fixture
def synth(pkg):
    return importlib.import_module(pkg.__name__ + ".synth")


@pytest.fixture
def small_manifest(tmp_path, synth):
    cfg = synth.NAFConfig(base_channels=8, enc_blocks=(1, 1), middle_blocks=1, dec_blocks=(1, 1))
    path, params = synth.make_model_dir(str(tmp_path), cfg, seed=3)
    return path, params


def test_roundtrip_names_shapes_arch(pkg, small_manifest, synth):
    path, params = small_manifest
    w = pkg.Weights(path)
    assert len(w) == len(params)
    assert w.names() == list(params.keys())
    for name, arr in params.items():
        shape, dtype = w.info(name)
        assert shape == arr.shape and dtype == "float16"
        assert name in w
    a = w.arch()
    assert a["type"] == "nafnet_residual" and a["base_channels"] == 8 and a["num_levels"] == 2


def test_missing_manifest_raises_io(pkg, tmp_path):
    with pytest.raises(pkg.DenoiserError) as e:
        pkg.Weights(str(tmp_path / "nonexistent" / "manifest.json"))
    assert e.value.code == pkg.DN_ERR_IO


def test_missing_key_is_not_found(pkg, small_manifest):
    w = pkg.Weights(small_manifest[0])
    assert "nope.weight" not in w
    with pytest.raises(pkg.NotFoundError):
        w.info("nope.weight")


def test_truncated_bin_is_rejected(pkg, small_manifest):
    path, _ = small_manifest
    man = json.load(open(path))
    f = os.path.join(os.path.dirname(path), man["layers"][3]["file"])
    data = open(f, "rb").read()
    open(f, "wb").write(data[:-2])
    with pytest.raises(pkg.DenoiserError) as e:
        pkg.Weights(path)
    assert e.value.code == pkg.DN_ERR_FORMAT and "size mismatch" in str(e.value)


def test_missing_bin_is_io_error(pkg, small_manifest):
    path, _ = small_manifest
    man = json.load(open(path))
    os.remove(os.path.join(os.path.dirname(path), man["layers"][0]["file"]))
    with pytest.raises(pkg.DenoiserError) as e:
        pkg.Weights(path)
    assert e.value.code == pkg.DN_ERR_IO


@pytest.mark.parametrize("text", ["{", '{"layers": [', '{"layers": 3}', "[1, 2]",
                                  '{"layers": [{"name": "a", "shape": [1], "dtype": "int8", "file": "x"}]}'])
def test_malformed_manifest_is_format_error(pkg, tmp_path, text):
    p = tmp_path / "manifest.json"
    p.write_text(text)
    with pytest.raises(pkg.DenoiserError) as e:
        pkg.Weights(str(p))
    assert e.value.code == pkg.DN_ERR_FORMAT


def test_reference_style_fp32_fixture(pkg, tmp_path):
    """The reference test fixture layout (FP32 layers + architecture block)."""
    wd = tmp_path / "weights"
    wd.mkdir()
    np.arange(1, 7, dtype=np.float32).tofile(wd / "layer0_weight.bin")
    np.array([0.1, 0.2], dtype=np.float32).tofile(wd / "layer0_bias.bin")
    man = {"version": "1.0", "model": "test_model", "dtype": "float32",
           "architecture": {"type": "nafnet_residual", "enc_channels": [32, 64], "num_levels": 2,
                            "base_channels": 32, "in_channels": 3, "out_channels": 3},
           "layers": [{"name": "layer0.weight", "shape": [2, 3, 1, 1], "dtype": "float32",
                       "file": "weights/layer0_weight.bin"},
                      {"name": "layer0.bias", "shape": [2], "dtype": "float32", "file": "weights/layer0_bias.bin"}]}
    (tmp_path / "manifest.json").write_text(json.dumps(man))
    w = pkg.Weights(str(tmp_path / "manifest.json"))
    assert len(w) == 2
    assert w.info("layer0.weight") == ((2, 3, 1, 1), "float32")
    assert w.arch()["num_levels"] == 2


def test_model_create_without_gpu_reports_error(pkg, small_manifest):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(pkg.DenoiserError):
        pkg.Model(small_manifest[0])
