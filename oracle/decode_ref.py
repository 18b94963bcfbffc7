"""CPU restatement of the reference YOLO decode + NMS.

TEST INFRASTRUCTURE ONLY. Restates pdefa/python/src/pdefa/_bindings.py:1095-1212
(decode_yolo, _iou, _nms) over a numpy [4+nc, A] float32 array with the same
float64 arithmetic and ordering rules, so GPU results can be compared exactly:

* per anchor: best class by strict '>' starting from class 0; skip if best < conf;
* box = (cx - w*0.5, cy - h*0.5, cx + w*0.5, cy + h*0.5) in float64;
* optional letterbox unmap (v - pad) * (1.0 / ratio), clamped to [0, orig];
* NMS per class, classes in order of first appearance, stable sort by conf
  descending, keep while IoU <= iou_thres against kept boxes of that class;
* final stable sort by conf descending, then truncate to max_det.
"""
from __future__ import annotations

from collections import defaultdict
from typing import List, Optional

import numpy as np


def _iou(a, b):
    x1 = a[0] if a[0] > b[0] else b[0]
    y1 = a[1] if a[1] > b[1] else b[1]
    x2 = a[2] if a[2] < b[2] else b[2]
    y2 = a[3] if a[3] < b[3] else b[3]
    w = x2 - x1
    h = y2 - y1
    if w <= 0 or h <= 0:
        return 0.0
    inter = w * h
    area_a = (a[2] - a[0]) * (a[3] - a[1])
    area_b = (b[2] - b[0]) * (b[3] - b[1])
    return inter / (area_a + area_b - inter + 1e-9)


def decode(preds: np.ndarray, meta: Optional[dict] = None, conf_thres: float = 0.25,
           iou_thres: float = 0.45, max_det: int = 300) -> List[dict]:
    """preds: [4+nc, A] float32. meta: dict with ratio, pad_x, pad_y, orig_w, orig_h."""
    p = np.asarray(preds, dtype=np.float32)
    nc = p.shape[0] - 4
    cls_scores = p[4:]
    best_c = np.zeros(p.shape[1], dtype=np.int64)
    best_s = cls_scores[0].copy()
    for c in range(1, nc):
        upd = cls_scores[c] > best_s
        best_s = np.where(upd, cls_scores[c], best_s)
        best_c = np.where(upd, c, best_c)
    cand = np.nonzero(~(best_s.astype(np.float64) < conf_thres))[0]
    boxes = []
    for i in cand:
        cx, cy, w, h = (float(p[0, i]), float(p[1, i]), float(p[2, i]), float(p[3, i]))
        boxes.append([cx - w * 0.5, cy - h * 0.5, cx + w * 0.5, cy + h * 0.5, float(best_s[i]), int(best_c[i]), int(i)])
    if not boxes:
        return []
    if meta is not None:
        scale = 1.0 / float(np.float32(meta["ratio"]))
        px, py, ow, oh = meta["pad_x"], meta["pad_y"], meta["orig_w"], meta["orig_h"]
        for b in boxes:
            for k, (pad, hi) in enumerate(((px, ow), (py, oh), (px, ow), (py, oh))):
                v = (b[k] - pad) * scale
                b[k] = 0.0 if v < 0 else (hi if v > hi else v)
    by_class = defaultdict(list)
    for i, b in enumerate(boxes):
        by_class[b[5]].append(i)
    keep = []
    for _, idxs in by_class.items():
        idxs.sort(key=lambda i: boxes[i][4], reverse=True)
        while idxs:
            cur = idxs.pop(0)
            keep.append(cur)
            if not idxs:
                break
            cb = boxes[cur]
            idxs = [j for j in idxs if _iou(cb, boxes[j]) <= iou_thres]
    keep.sort(key=lambda i: boxes[i][4], reverse=True)
    keep = keep[:max_det]
    return [{"x1": float(boxes[i][0]), "y1": float(boxes[i][1]), "x2": float(boxes[i][2]), "y2": float(boxes[i][3]),
             "conf": boxes[i][4], "cls": boxes[i][5], "anchor": boxes[i][6]} for i in keep]
