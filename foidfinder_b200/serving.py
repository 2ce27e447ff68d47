"""Request batching for the serve path: many concurrent `predict(image)` calls share one CUDA-graph
replay instead of one replay each.

The reference serves every request at batch 1 on a single inference thread
(foidfinder/web.py:79 and :140-144, `backend.predict` through a one-thread executor). `BatchingBackend`
keeps the `Backend` protocol (foidfinder/backends/__init__.py:17-23) but may be called from any number
of threads: each call preprocesses its image on the calling thread, queues it, and blocks until the
batch it joined has run. A single worker thread owns the engine: it takes the first waiting request,
gathers more until `max_batch` or `max_wait_ms`, pads the batch up to the next of a few fixed sizes (one
captured graph per size), runs it, and hands every caller its own row.
"""

from __future__ import annotations

import concurrent.futures as cf
import queue
import threading
import time
from typing import Callable

import numpy as np


def batch_sizes(max_batch: int) -> list[int]:
    """Powers of two up to max_batch (and max_batch itself): the graph sizes a padded batch uses."""
    sizes, b = [], 1
    while b < max_batch:
        sizes.append(b)
        b *= 2
    return sizes + [max_batch]


class BatchingBackend:
    name = "cuda"

    def __init__(self, run_batch: Callable[[np.ndarray], np.ndarray], prepare: Callable[[object], np.ndarray],
                 device: str = "", *, max_batch: int = 32, max_wait_ms: float = 1.0):
        """run_batch: uint8 images [B, S, S, 3] -> probabilities [B, num_tags] (called on the worker thread
        only); prepare: decoded image -> uint8 [S, S, 3] (called on the submitting thread)."""
        if max_batch < 1:
            raise ValueError("max_batch must be >= 1")
        self.device = device
        self._run, self._prepare = run_batch, prepare
        self.max_batch, self.max_wait = max_batch, max_wait_ms / 1000.0
        self.sizes = batch_sizes(max_batch)
        self.batches: list[int] = []  # real request count of every batch run (for monitoring and tests)
        self._q: queue.Queue = queue.Queue()
        self._closed = False
        self._worker = threading.Thread(target=self._loop, name="foidfinder-b200-batcher", daemon=True)
        self._worker.start()

    @classmethod
    def from_backend(cls, backend, **kw) -> BatchingBackend:
        """Wraps a `backend.CUDABackend` (its engine and letterbox preprocessing)."""
        import torch

        from .backend import letterbox

        c = backend.cfg
        eng = backend.engine

        def run(images: np.ndarray) -> np.ndarray:
            with torch.no_grad():
                return torch.sigmoid(eng(torch.from_numpy(images))).cpu().numpy()

        return cls(run, lambda im: letterbox(im, c.image_size, c.resample, c.pad), backend.device, **kw)

    def submit(self, image) -> cf.Future:
        if self._closed:
            raise RuntimeError("BatchingBackend is closed")
        fut: cf.Future = cf.Future()
        self._q.put((self._prepare(image), fut))
        return fut

    def predict(self, image) -> np.ndarray:
        return self.submit(image).result()

    def _loop(self) -> None:
        while True:
            item = self._q.get()
            if item is None:
                return
            items = [item]
            deadline = time.perf_counter() + self.max_wait
            while len(items) < self.max_batch:
                left = deadline - time.perf_counter()
                try:
                    nxt = self._q.get(timeout=left) if left > 0 else self._q.get_nowait()
                except queue.Empty:
                    break
                if nxt is None:
                    self._q.put(None)  # finish this batch, then stop
                    break
                items.append(nxt)
            n = len(items)
            size = next(s for s in self.sizes if s >= n)
            imgs = np.stack([a for a, _ in items])
            if size > n:
                imgs = np.concatenate([imgs, np.zeros((size - n,) + imgs.shape[1:], imgs.dtype)])
            self.batches.append(n)
            try:
                probs = self._run(imgs)
            except BaseException as exc:  # every caller of this batch sees the failure
                for _, fut in items:
                    fut.set_exception(exc)
                continue
            for i, (_, fut) in enumerate(items):
                fut.set_result(np.asarray(probs[i]))

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self._q.put(None)
            self._worker.join()
