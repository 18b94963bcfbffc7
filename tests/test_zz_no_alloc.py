"""pdefa_decode_yolo_noalloc: the decode entry point for callers that cannot
allocate device memory (strict caching allocators, servers that forbid cudaMalloc
after start-up, plugin hosts that only hand out I/O buffers). Its scratch is a
built-in device array, so two calls in a row must each match the allocating
device entry point exactly (decode results are bit-exact), and sizes beyond the
built-in scratch must be refused. Collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STRUCT = 48   # sizeof(PdefaDetection)


def _lib():
    from pdefa_b200 import _native as N
    L = N.lib()
    f = L.pdefa_decode_yolo_noalloc
    f.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_double, C.c_double, C.c_int32,
                  C.c_void_p, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return L


def _decode_pair(L, torch, preds, conf, iou, max_det):
    B, ch, A = preds.shape
    d = torch.from_numpy(np.ascontiguousarray(preds)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    # allocating device entry point (caller-provided scratch)
    wb = L.pdefa_decode_work_bytes(B, A)
    work = torch.empty(wb, dtype=torch.uint8, device="cuda")
    c_ref = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    d_ref = torch.zeros(B * max_det * STRUCT, dtype=torch.uint8, device="cuda")
    assert L.pdefa_decode_yolo_device(d.data_ptr(), B, ch, A, None, conf, iou, max_det, c_ref.data_ptr(),
                                      d_ref.data_ptr(), work.data_ptr(), wb, stream) == 0
    # allocation-free entry point
    c_new = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    d_new = torch.zeros(B * max_det * STRUCT, dtype=torch.uint8, device="cuda")
    assert L.pdefa_decode_yolo_noalloc(d.data_ptr(), B, ch, A, None, conf, iou, max_det, c_new.data_ptr(),
                                       d_new.data_ptr(), stream) == 0, L.pdefa_last_error()
    torch.cuda.synchronize()
    return c_ref.cpu().numpy(), d_ref.cpu().numpy(), c_new.cpu().numpy(), d_new.cpu().numpy()


def test_noalloc_decode_matches_allocating_decode_twice(golden):
    torch = pytest.importorskip("torch")
    L = _lib()
    g = golden("decode_inputs.npz")
    first = np.stack([g["y8n_128"], g["y8n_128"][:, ::-1]]).astype(np.float32)
    adv = g["adversarial"]
    second = np.stack([adv, adv[:, ::-1], adv * np.float32(0.9)]).astype(np.float32)
    for preds, conf, iou, md in ((first, 0.25, 0.45, 300), (second, 0.3, 0.5, 40)):
        cr, dr, cn, dn = _decode_pair(L, torch, preds, conf, iou, md)
        assert (cr >= 0).all() and cr.sum() > 0
        np.testing.assert_array_equal(cn, cr)
        B = preds.shape[0]
        for b in range(B):
            n = int(cr[b])
            lo = b * md * STRUCT
            np.testing.assert_array_equal(dn[lo:lo + n * STRUCT], dr[lo:lo + n * STRUCT])


def test_noalloc_decode_rejects_oversized_calls():
    torch = pytest.importorskip("torch")
    L = _lib()
    B, ch, A = 21, 84, 8400        # 176400 candidate slots > the 174762 built in
    preds = torch.zeros((1,), dtype=torch.float32, device="cuda")
    counts = torch.zeros((B,), dtype=torch.int32, device="cuda")
    dets = torch.zeros((B * 300 * STRUCT,), dtype=torch.uint8, device="cuda")
    rc = L.pdefa_decode_yolo_noalloc(preds.data_ptr(), B, ch, A, None, 0.25, 0.45, 300, counts.data_ptr(),
                                     dets.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 7
    assert b"scratch" in L.pdefa_last_error()
