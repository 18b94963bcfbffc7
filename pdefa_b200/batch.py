"""BatchInference over 1..8 GPUs (replaces pdefa/python/src/pdefa/batch.py:13-70).

The reference runs `batch_size` batch-1 Sessions on a Python thread pool over one
CPU. Here one replica of the model lives on each selected GPU; a batch of images is
split into contiguous shards, each GPU runs its shard in micro-batches of
`batch_size` images (batched forward pass plus the GPU decode/NMS), and only
detections come back. There is no collective. The C++ runner (pdefa_batch_run)
drives all GPUs from native threads and pipelines each GPU's micro-batches over
three streams: the copy of micro-batch i+1 onto the GPU and the decode of i-1 overlap
the inference of i.
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

    # PdefaDetection (include/pdefa_b200_ext.h) as a numpy record
    DET_DTYPE = [("x1", "<f8"), ("y1", "<f8"), ("x2", "<f8"), ("y2", "<f8"), ("conf", "<f4"), ("cls", "<i4"),
                 ("anchor", "<i4"), ("reserved", "<i4")]

    def detect_arrays(self, images, metas: Optional[Sequence[PreprocessMeta]] = None, conf_thres: float = 0.25,
                      iou_thres: float = 0.45, max_det: int = 300):
        """images: [N, 3, H, W] float32 array -> (counts int32 [N], dets record array
        [N, max_det] with fields x1 y1 x2 y2 conf cls anchor); image b's detections
        are dets[b, :counts[b]], best first. Images in page-locked memory (e.g. a
        pinned torch tensor's .numpy()) reach the GPU fastest."""
        import numpy as np
        x = np.ascontiguousarray(images, dtype=np.float32)
        n = x.shape[0]
        md = max(int(max_det), 0)
        counts = np.zeros(max(n, 1), dtype=np.int32)
        dets = np.zeros((max(n, 1), max(md, 1)), dtype=self.DET_DTYPE)
        marr = (N.PreMeta * n)(*[m.to_c() for m in metas]) if metas is not None else None
        _check(N.lib().pdefa_batch_run(self._handle, x.ctypes.data, n, marr, float(conf_thres), float(iou_thres),
                                       md, counts.ctypes.data_as(C.POINTER(N.i32)),
                                       dets.ctypes.data_as(C.POINTER(N.Detection))), "batch_run")
        return counts[:n], dets[:n, :md]

    def detect_u8(self, images, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
                  pad_value: float = 0.0, conf_thres: float = 0.25, iou_thres: float = 0.45, max_det: int = 300):
        """Decoded 8-bit images -> (counts, dets, meta) like detect_arrays, boxes in
        original-image coordinates. images: [N, h, w, C] (C = 1, 3, 4) or [N, h, w]
        uint8, all of one size. Each GPU receives the pixels (a quarter of the float32
        bytes for RGB), letterboxes them into the model input exactly as the
        reference's preprocess_letterbox does, runs inference and decode with the
        letterbox meta (decode_yolo(out, meta))."""
        import numpy as np
        a = np.ascontiguousarray(images, dtype=np.uint8)
        if a.ndim == 3:
            a = a[..., None]
        if a.ndim != 4 or a.shape[3] not in (1, 3, 4):
            raise PdefaError("detect_u8: images must be uint8 [N, h, w] or [N, h, w, C] with C = 1, 3 or 4")
        n, h, w, ch = a.shape
        md = max(int(max_det), 0)
        counts = np.zeros(max(n, 1), dtype=np.int32)
        dets = np.zeros((max(n, 1), max(md, 1)), dtype=self.DET_DTYPE)
        m = N.PreMeta()
        cfg = N.PreConfig(int(target_w), int(target_h), float(scale), float(pad_value))
        _check(N.lib().pdefa_batch_run_u8(self._handle, a.ctypes.data, n, h, w, ch, C.byref(cfg), float(conf_thres),
                                          float(iou_thres), md, counts.ctypes.data_as(C.POINTER(N.i32)),
                                          dets.ctypes.data_as(C.POINTER(N.Detection)), C.byref(m)), "batch_run_u8")
        return counts[:n], dets[:n, :md], PreprocessMeta.from_c(m)

    def submit_u8(self, images, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
                  pad_value: float = 0.0, conf_thres: float = 0.25, iou_thres: float = 0.45,
                  max_det: int = 300) -> "PendingDetections":
        """detect_u8 without waiting: the frames are queued (copies, GPU letterbox,
        inference, decode) and a PendingDetections comes back at once; its result()
        gives what detect_u8 would have returned. Submitting the next frames before
        asking for the result lets their copies onto the GPU overlap the end of this
        call's work. The pending object keeps `images` and its output arrays alive;
        the caller must not modify `images` until result() returns."""
        import numpy as np
        a = np.ascontiguousarray(images, dtype=np.uint8)
        if a.ndim == 3:
            a = a[..., None]
        if a.ndim != 4 or a.shape[3] not in (1, 3, 4):
            raise PdefaError("submit_u8: images must be uint8 [N, h, w] or [N, h, w, C] with C = 1, 3 or 4")
        n, h, w, ch = a.shape
        md = max(int(max_det), 0)
        counts = np.zeros(max(n, 1), dtype=np.int32)
        dets = np.zeros((max(n, 1), max(md, 1)), dtype=self.DET_DTYPE)
        m = N.PreMeta()
        cfg = N.PreConfig(int(target_w), int(target_h), float(scale), float(pad_value))
        ticket = C.c_int64(0)
        _check(N.lib().pdefa_batch_submit_u8(self._handle, a.ctypes.data, n, h, w, ch, C.byref(cfg),
                                             float(conf_thres), float(iou_thres), md,
                                             counts.ctypes.data_as(C.POINTER(N.i32)),
                                             dets.ctypes.data_as(C.POINTER(N.Detection)), C.byref(m),
                                             C.byref(ticket)), "batch_submit_u8")
        return PendingDetections(self, ticket.value, a, counts[:n], dets[:n, :md], PreprocessMeta.from_c(m))

    def wait(self):
        """Completes every call queued by submit_u8 so far."""
        _check(N.lib().pdefa_batch_wait(self._handle, 0), "batch_wait")

    def detect(self, images, metas: Optional[Sequence[PreprocessMeta]] = None, conf_thres: float = 0.25,
               iou_thres: float = 0.45, max_det: int = 300) -> List[List[dict]]:
        """images: [N, 3, H, W] float32 array -> per-image detection dicts
        (x1, y1, x2, y2, conf, cls), best first."""
        counts, dets = self.detect_arrays(images, metas, conf_thres, iou_thres, max_det)
        out = []
        for b in range(len(counts)):
            d = dets[b, :counts[b]]
            out.append([{"x1": x1, "y1": y1, "x2": x2, "y2": y2, "conf": cf, "cls": c}
                        for x1, y1, x2, y2, cf, c in zip(d["x1"].tolist(), d["y1"].tolist(), d["x2"].tolist(),
                                                         d["y2"].tolist(), d["conf"].tolist(), d["cls"].tolist())])
        return out

    def run(self, image_paths: List[str], target_w: int = 640, target_h: int = 640) -> List[Tuple[Tensor, PreprocessMeta]]:
        """Reference signature (batch.py:45-60): image files -> [(raw output Tensor,
        letterbox meta)], one Session per image like the reference (PNG and JPEG files)."""
        out = []
        for p in image_paths:
            t, meta = prepare_for_engine(p, target_w, target_h)
            s = Session(self.ctx, self.model)
            s.set_input(0, t)
            s.run()
            y = s.output(0)
            y._session = s      # the output is borrowed from the session: keep it alive
            out.append((y, meta))
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


class PendingDetections:
    """Results of one BatchInference.submit_u8 call. result() waits for this call only
    (and for the calls queued before it) and returns (counts, dets, meta) as
    detect_u8 does."""

    def __init__(self, runner: BatchInference, ticket: int, images, counts, dets, meta):
        self._runner, self.ticket, self._images = runner, ticket, images
        self._counts, self._dets, self.meta = counts, dets, meta
        self._done = False

    def result(self):
        if not self._done:
            _check(N.lib().pdefa_batch_wait(self._runner._handle, self.ticket), "batch_wait")
            self._done = True
            self._images = None
        return self._counts, self._dets, self.meta
