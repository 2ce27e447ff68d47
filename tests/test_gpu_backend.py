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
