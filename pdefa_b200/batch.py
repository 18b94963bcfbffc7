"""BatchInference over 1..8 GPUs (replaces pdefa/python/src/pdefa/batch.py:13-70).

The reference runs `batch_size` batch-1 Sessions on a Python thread pool over one
CPU. Here one replica of the model lives on each selected GPU; a batch of images is
split into contiguous shards, each GPU runs its shard as one batched forward pass
plus the GPU decode/NMS, and only detections come back. There is no collective.
The C++ runner (pdefa_batch_run) drives all GPUs from native threads.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Sequence, Tuple

from . import _native as N
from .api import (BF16, Context, Model, PdefaError, PreprocessMeta, Session, Tensor, _check, _det_dict,
                  device_count, prepare_for_engine)


class BatchInference:
    """Batched multi-GPU inference.

    BatchInference(ctx, model, batch_size=4, num_threads=4) keeps the reference's
    signature; `batch_size` is the per-GPU micro-batch and `devices` (default: all
    visible GPUs) the replicas.
    """

    def __init__(self, ctx: Context, model: Model, batch_size: int = 4, num_threads: int = 4,
                 devices: Optional[Sequence[int]] = None, precision: Optional[int] = None):
        self.ctx = ctx
        self.model = model
        self.batch_size = int(batch_size)
        self.num_threads = int(num_threads)
        n = device_count()
        if n == 0:
            raise PdefaError("BatchInference: no CUDA device available")
        self.devices = list(devices) if devices is not None else list(range(n))
        prec = ctx.get_precision() if precision is None else int(precision)
        arr = (N.i32 * len(self.devices))(*self.devices)
        h = C.c_void_p()
        _check(N.lib().pdefa_batch_create(model.raw, len(self.devices), arr, prec, self.batch_size, C.byref(h)),
               "batch_create")
        self._handle = h

    def detect(self, images, metas: Optional[Sequence[PreprocessMeta]] = None, conf_thres: float = 0.25,
               iou_thres: float = 0.45, max_det: int = 300) -> List[List[dict]]:
        """images: [N, 3, H, W] float32 array -> per-image detection dicts."""
        import numpy as np
        x = np.ascontiguousarray(images, dtype=np.float32)
        n = x.shape[0]
        md = max(int(max_det), 0)
        counts = (N.i32 * max(n, 1))()
        dets = (N.Detection * max(n * md, 1))()
        marr = (N.PreMeta * n)(*[m.to_c() for m in metas]) if metas is not None else None
        _check(N.lib().pdefa_batch_run(self._handle, x.ctypes.data, n, marr, float(conf_thres), float(iou_thres),
                                       md, counts, dets), "batch_run")
        return [[_det_dict(dets[b * md + i]) for i in range(counts[b])] for b in range(n)]

    def run(self, image_paths: List[str], target_w: int = 640, target_h: int = 640) -> List[Tuple[Tensor, PreprocessMeta]]:
        """Reference signature (image files -> raw outputs). Needs host image decoding."""
        out = []
        for p in image_paths:
            t, meta = prepare_for_engine(p, target_w, target_h)
            s = Session(self.ctx, self.model)
            s.set_input(0, t)
            s.run()
            out.append((s.output(0), meta))
        return out

    def close(self):
        if getattr(self, "_handle", None) and N._lib is not None:
            N._lib.pdefa_batch_destroy(self._handle)
            self._handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()
