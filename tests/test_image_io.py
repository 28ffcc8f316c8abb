"""Image codecs of the CLI (include/denoiser_b200_io.h) on the host: PNG
against PIL, EXR against OpenCV's OpenEXR codec, PPM/PFM round trips, and
the reference's pixel rules (src/io/image_io.cc:26-61: 8-bit loads as
value / 255 into 3 channels, saves clamp(v * 255 + 0.5); src/io/exr_io.cc:
76-114, 150-196: R,G,B (else Y) as FP16, saved as HALF B,G,R or Y)."""
import importlib
import os

import numpy as np
import pytest

os.environ.setdefault("OPENCV_IO_ENABLE_OPENEXR", "1")


@pytest.fixture(scope="module")
def io(pkg):
    return importlib.import_module(pkg.__name__ + ".image_io")


def rand_img(c, h, w, seed, lo=0.0, hi=1.0):
    return np.random.default_rng(seed).uniform(lo, hi, (1, c, h, w)).astype(np.float16)


def test_png_save_matches_reference_rounding_and_pil(io, tmp_path):
    PIL = pytest.importorskip("PIL.Image")
    x = rand_img(3, 13, 17, 1, -0.2, 1.2)
    p = str(tmp_path / "a.png")
    io.save(p, x)
    got = np.asarray(PIL.open(p).convert("RGB")).transpose(2, 0, 1)
    want = np.clip((x[0].astype(np.float32) * 255.0 + 0.5).astype(np.int32), 0, 255)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("mode", ["RGB", "RGBA", "L", "LA", "P", "I;16"])
def test_png_load_modes_against_pil(io, tmp_path, mode):
    PIL = pytest.importorskip("PIL.Image")
    rng = np.random.default_rng(len(mode))
    rgb = rng.integers(0, 256, (19, 23, 3), dtype=np.uint8)
    img = PIL.fromarray(rgb, "RGB")
    if mode == "I;16":
        arr16 = rng.integers(0, 65536, (19, 23), dtype=np.uint16)
        img = PIL.fromarray(arr16)
        expect = np.repeat((arr16 >> 8)[None], 3, 0)  # high byte, as an 8-bit loader keeps
    else:
        img = img.convert(mode)
        expect = np.asarray(img.convert("RGB")).transpose(2, 0, 1)
    p = str(tmp_path / "m.png")
    img.save(p, optimize=True)  # lets the encoder pick varying filter types
    got = io.load(p)
    assert got.shape == (1, 3, 19, 23)
    assert np.array_equal(got[0], (expect.astype(np.float32) / 255.0).astype(np.float16))


def test_exr_round_trip_and_opencv(io, tmp_path):
    cv2 = pytest.importorskip("cv2")
    x = rand_img(3, 21, 35, 3, -2.0, 3.0)
    p = str(tmp_path / "a.exr")
    io.save(p, x)
    assert np.array_equal(io.load(p), x)  # HALF channels: bit-exact
    got = cv2.imread(p, cv2.IMREAD_UNCHANGED)
    if got is None:
        pytest.skip("OpenCV built without OpenEXR")
    assert np.array_equal(got[..., ::-1].transpose(2, 0, 1), x[0].astype(np.float32))


@pytest.mark.parametrize("comp", [0, 1, 2, 3], ids=["none", "rle", "zips", "zip"])
@pytest.mark.parametrize("half", [True, False], ids=["half", "float"])
def test_exr_load_opencv_files(io, tmp_path, comp, half):
    cv2 = pytest.importorskip("cv2")
    rng = np.random.default_rng(comp)
    bgr = rng.uniform(-1, 4, (37, 29, 3)).astype(np.float32)
    p = str(tmp_path / "c.exr")
    params = [cv2.IMWRITE_EXR_COMPRESSION, comp, cv2.IMWRITE_EXR_TYPE,
              cv2.IMWRITE_EXR_TYPE_HALF if half else cv2.IMWRITE_EXR_TYPE_FLOAT]
    if not cv2.imwrite(p, bgr, params):
        pytest.skip("OpenCV built without OpenEXR")
    got = io.load(p)
    want = bgr[..., ::-1].transpose(2, 0, 1).astype(np.float16)
    assert got.shape == (1, 3, 37, 29)
    assert np.array_equal(got[0], want)


def test_exr_single_channel_is_y(io, tmp_path):
    x = rand_img(1, 9, 11, 4)
    p = str(tmp_path / "y.exr")
    io.save(p, x)
    assert io.probe(p) == (1, 9, 11)
    assert np.array_equal(io.load(p), x)


def test_ppm_pfm_round_trips(io, tmp_path):
    x = rand_img(3, 8, 10, 5)
    io.save(str(tmp_path / "a.pfm"), x)
    assert np.array_equal(io.load(str(tmp_path / "a.pfm")), x)
    io.save(str(tmp_path / "a.ppm"), x)
    q = np.clip((x[0].astype(np.float32) * 255.0 + 0.5).astype(np.int32), 0, 255)
    assert np.array_equal(io.load(str(tmp_path / "a.ppm"))[0], (q / 255.0).astype(np.float16))


def test_codec_errors(pkg, io, tmp_path):
    x = rand_img(3, 4, 4, 6)
    with pytest.raises(pkg.DenoiserError, match="JPEG"):
        io.save(str(tmp_path / "a.jpg"), x)
    with pytest.raises(pkg.DenoiserError):
        io.load(str(tmp_path / "missing.png"))
    (tmp_path / "bad.png").write_bytes(b"not a png at all")
    with pytest.raises(pkg.DenoiserError, match="PNG"):
        io.load(str(tmp_path / "bad.png"))
    with pytest.raises(pkg.DenoiserError, match="C=1 or C=3"):
        io.save(str(tmp_path / "a.exr"), rand_img(2, 4, 4, 7))
