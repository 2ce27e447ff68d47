"""The Backend-protocol wrappers on the GPU: CUDABackend.predict (letterbox + engine + sigmoid) and the
batching backend, which must return exactly what batch-1 predict returns for every request."""

import concurrent.futures as cf

import numpy as np
import pytest
import torch
from PIL import Image

pytestmark = pytest.mark.gpu


def _images():
    rng = np.random.default_rng(4)
    ims = [Image.fromarray(rng.integers(0, 256, (h, w, 3), dtype=np.uint8)) for h, w in ((112, 112), (90, 160), (200, 60))]
    rgba = rng.integers(0, 256, (80, 80, 4), dtype=np.uint8)
    ims.append(Image.fromarray(rgba, "RGBA"))
    return ims


def test_cuda_backend_predict(cuda_device, no_device_error):
    from foidfinder_b200.backend import CUDABackend, letterbox
    from foidfinder_b200.config import EVA02_L

    cfg = EVA02_L.with_(name="backend-112", image_size=112, depth=1)
    be = CUDABackend(None, config=cfg, device=0, seed=5)
    assert be.name == "cuda" and "B200" in be.device
    for im in _images():
        p = be.predict(im)
        assert p.shape == (cfg.num_tags,) and p.dtype == np.float32
        assert np.all((p >= 0) & (p <= 1))
        ref = torch.sigmoid(be.engine(torch.from_numpy(letterbox(im, 112, cfg.resample, cfg.pad))[None]))[0].cpu().numpy()
        np.testing.assert_array_equal(p, ref)
    be.engine.close()


def test_batching_backend_matches_batch1(cuda_device, no_device_error):
    from foidfinder_b200.backend import CUDABackend
    from foidfinder_b200.config import EVA02_L
    from foidfinder_b200.serving import BatchingBackend

    cfg = EVA02_L.with_(name="batch-112", image_size=112, depth=1)
    be = CUDABackend(None, config=cfg, device=0, seed=6)
    ims = _images() * 3
    single = [be.predict(im) for im in ims]
    bb = BatchingBackend.from_backend(be, max_batch=8, max_wait_ms=20.0)
    try:
        with cf.ThreadPoolExecutor(12) as ex:
            outs = list(ex.map(bb.predict, ims))
    finally:
        bb.close()
    assert len(bb.batches) < len(ims)
    for a, b in zip(single, outs):
        # each image's logits do not depend on its batch mates (same kernels, row-independent math)
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-6)
    be.engine.close()


CASES = [(850, 1200), (448, 900), (3, 5000), (5000, 3), (100, 37), (448, 300), (1, 1), (1500, 1400), (448, 448)]


@pytest.mark.parametrize("bicubic,fill", [(True, 255), (False, 0)])
@pytest.mark.parametrize(("w", "h"), CASES)
def test_gpu_letterbox_is_bit_exact_with_pillow(cuda_device, w, h, bicubic, fill):
    """ff_resize_pad against PIL.Image.resize + paste (the sizes of the reference's own resize test,
    tests/test_haruka.py:36-55, plus a few more), both filters."""
    from foidfinder_b200 import ops
    from foidfinder_b200.backend import letterbox_size

    S = 448
    rgb = np.random.default_rng(w * h).integers(0, 256, (h, w, 3), dtype=np.uint8)
    nh, nw = letterbox_size(h, w, S)
    canvas = Image.new("RGB", (S, S), (fill,) * 3)
    flt = Image.Resampling.BICUBIC if bicubic else Image.Resampling.BILINEAR
    canvas.paste(Image.fromarray(rgb).resize((nw, nh), flt), ((S - nw) // 2, (S - nh) // 2))
    out = torch.empty(S, S, 3, dtype=torch.uint8, device=cuda_device)
    ops.resize_pad(torch.from_numpy(rgb).to(cuda_device), nh, nw, S, out, bicubic=bicubic, fill=fill)
    np.testing.assert_array_equal(out.cpu().numpy(), np.asarray(canvas))


def test_gpu_letterbox_matches_host_letterbox(cuda_device):
    from foidfinder_b200.backend import letterbox, letterbox_gpu

    for im in _images():
        for resample, pad in (("bilinear", 0), ("bicubic", 255)):
            host = letterbox(im, 448, resample, pad)
            gpu = letterbox_gpu(im, 448, resample, pad, cuda_device).cpu().numpy()
            np.testing.assert_array_equal(gpu, host)


def _reference_sample_images():
    """The reference's preprocessing fixture shapes (tests/conftest.py:18-27): downscale, upscale and
    exact-size paths, plus an RGBA image composited onto white (seeded noise, blurred so the resize filter
    matters)."""
    from PIL import ImageFilter

    rng = np.random.default_rng(0)
    blur = ImageFilter.GaussianBlur(3)
    ims = [Image.fromarray(rng.integers(0, 256, (h, w, 3), dtype=np.uint8)).filter(blur)
           for w, h in ((1500, 2100), (700, 400), (1008, 1008))]
    return [*ims, Image.fromarray(rng.integers(0, 256, (600, 900, 4), dtype=np.uint8))]


def test_pixai_float_letterbox_matches_reference_preprocess(cuda_device):
    """ff_letterbox_aa_f16 (via backend.preprocess) against the reference's preprocess.py:16-32 restated on
    the CPU (oracle.pixai.preprocess: torch F.interpolate with antialias): the reference's own bar,
    |dpixel| < 2e-3, one fp16 step (tests/test_cuda_engine.py:29-35)."""
    from foidfinder_b200.backend import preprocess
    from oracle import pixai as P

    ims = _reference_sample_images()
    got = preprocess(ims, 1008, cuda_device).float().cpu()
    want = P.preprocess(ims, 1008).float()
    for g, w in zip(got, want):
        d = (g - w).abs()
        assert d.max().item() < 2e-3, d.max().item()
        assert (d > 0).float().mean().item() < 0.01  # only rounding ties of the fp16 step differ


@pytest.mark.parametrize("arch", ["eva02", "pixai"])
def test_engine_float_pixels_match_uint8_path(cuda_device, no_device_error, arch):
    """Engine.__call__ takes the reference's normalised float pixels (PixAICuda.__call__, engine.py:163-165).
    Pixels equal to what the uint8 path's patchify computes ((u * (1/255) - mean) / std in one fused f32
    step, then fp16) give bit-identical logits through both graphs; float32 input is cast to fp16 as the
    reference's static input does."""
    from foidfinder_b200.config import EVA02_L, PIXAI_1008
    from foidfinder_b200.engine import Engine

    if arch == "pixai":
        cfg = PIXAI_1008.with_(name="px-float", image_size=336, depth=2, window=8, global_blocks=(1,))
    else:
        cfg = EVA02_L.with_(name="eva-float", image_size=112, depth=2)
    eng = Engine(cfg, device=0, seed=4)
    u8 = torch.randint(0, 256, (2, cfg.image_size, cfg.image_size, 3), generator=torch.Generator().manual_seed(8),
                       dtype=torch.uint8)
    mean = torch.tensor(cfg.mean, dtype=torch.float32).double()
    inv_std = (1.0 / torch.tensor(cfg.std, dtype=torch.float32)).double()
    one_255 = float(np.float32(1.0 / 255.0))
    px = ((u8.double() * one_255 - mean).float().double() * inv_std).float().half()
    a = eng(u8)
    b = eng(px.to(cuda_device))
    c = eng(px.float())  # float32 on the host: moved and cast to fp16
    torch.cuda.synchronize()
    assert torch.equal(a.cpu(), b.cpu()) and torch.equal(b.cpu(), c.cpu())
    eng.close()


def test_pixai_backend_from_model_directories(cuda_device, no_device_error, tmp_path):
    """CUDABackend(model_dir) on a PixAI directory with the official fp32 checkpoint and on one with the
    reference's `foidfinder convert` int8 output: identical predictions, equal to the engine run on the
    reference's preprocessing of the same image (the CPU restatement) up to the fp16 pixel step."""
    import json

    from safetensors.torch import save_file

    from foidfinder_b200 import weights as W
    from foidfinder_b200.backend import CUDABackend
    from foidfinder_b200.config import PIXAI_1008
    from oracle import pixai as P

    cfg = PIXAI_1008.with_(name="px-dir", image_size=336, depth=2, window=8, global_blocks=(1,), num_tags=1000)
    raw = W.pixai_random_raw(cfg, seed=9)
    # `foidfinder convert` converts on the GPU when there is one (cli.py:149), as the backend does with an
    # fp32 directory: the same float32 matmul on the same device, hence the same codes
    converted = {k: v.cpu() for k, v in W.pixai_convert_checkpoint({k: v.to(cuda_device) for k, v in raw.items()},
                                                                  cfg).items()}
    for name, tensors, meta in (("official", raw, None),
                                ("converted", converted, {"format": W.PIXAI_INT8_FORMAT})):
        d = tmp_path / name
        d.mkdir()
        save_file({k: v.contiguous() for k, v in tensors.items()}, str(d / "model.safetensors"), meta)
        (d / "config.json").write_text(json.dumps({"num_classes": cfg.num_tags}))
    ims = _reference_sample_images()[1:3]
    preds = []
    for name in ("official", "converted"):
        be = CUDABackend(tmp_path / name, config=cfg, device=0)
        preds.append([be.predict(im) for im in ims])
        ref = [torch.sigmoid(be.engine(P.preprocess([im], cfg.image_size).to(cuda_device)))[0].cpu().numpy()
               for im in ims]
        for p, r in zip(preds[-1], ref):
            assert p.shape == (cfg.num_tags,)
            np.testing.assert_allclose(p, r, rtol=0, atol=5e-3)
        be.engine.close()
    for a, b in zip(*preds):
        np.testing.assert_array_equal(a, b)
