"""C-ABI checks that need no GPU: the library loads, exports every symbol the
headers declare (and every symbol of the reference pdefa.def export list), and
its host-side logic (handles, tensors, errors, model files) behaves like the
reference's (PDEFA1.0/src/api/engine_api.cpp)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import pdefa_b200 as pb
from pdefa_b200 import _native as N
from pdefa_b200.engine_file import pack_params, read_engine, unpack_params, write_engine
from pdefa_b200.yolo import build_yolov8, conv_flops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# The 77 names of pdefa/pdefa.def:4-97 (pdefa_* 14 + engine_* 63).
DEF_EXPORTS = """pdefa_version pdefa_last_error pdefa_image_load pdefa_image_free pdefa_image_width
pdefa_image_height pdefa_image_channels pdefa_image_format pdefa_image_pixels pdefa_preprocess_letterbox
pdefa_prepare_for_engine pdefa_load_image_as_tensor pdefa_map_box_to_original pdefa_map_point_to_original
engine_version engine_last_error engine_status_string engine_dtype_size engine_simd_level engine_cpu_brand
engine_context_create engine_context_destroy engine_context_set_num_threads engine_context_get_num_threads
engine_context_num_physical_cores engine_context_has_avx2 engine_context_has_avx512 engine_tensor_create
engine_tensor_create_from_data engine_tensor_data engine_tensor_shape engine_tensor_copy_from engine_tensor_copy_to
engine_tensor_numel engine_tensor_dtype engine_tensor_rank engine_tensor_destroy engine_model_load
engine_model_input_count engine_model_output_count engine_model_name engine_model_destroy engine_session_create
engine_session_set_input engine_session_run engine_session_get_output engine_session_destroy engine_run_simple
engine_model_input_info engine_model_output_info engine_session_get_stats engine_session_set_profile_callback
engine_session_clear_profile_callback engine_session_debug_intermediate engine_ops_matmul engine_ops_relu
engine_ops_silu engine_ops_add engine_ops_sub engine_ops_mul engine_ops_div engine_ops_sigmoid engine_ops_tanh
engine_ops_gelu engine_ops_clip engine_ops_softmax engine_ops_reduce_max engine_ops_reduce_sum engine_ops_reduce_mean
engine_ops_argmax engine_ops_gather engine_ops_reshape engine_ops_transpose engine_ops_concat engine_ops_stack
engine_random_randn engine_random_rand""".split()


def header_functions():
    names = set()
    for h in ("engine_c_api.h", "pdefa_c_api.h", "pdefa_b200_ext.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        names.update(re.findall(r"\b((?:engine|pdefa)_[a-z0-9_]+)\s*\(", src))
    return names


def test_def_list_has_77_entries():
    assert len(DEF_EXPORTS) == 77 and len(set(DEF_EXPORTS)) == 77


def test_library_exports_every_declared_symbol():
    L = N.lib()
    declared = header_functions()
    assert set(DEF_EXPORTS) <= declared
    for name in sorted(declared):
        assert hasattr(L, name), f"{name} not exported"


def test_status_and_version():
    L = N.lib()
    assert L.engine_status_string(0) == b"OK"
    assert L.engine_status_string(9) == b"not implemented"
    assert L.engine_dtype_size(0) == 4 and L.engine_dtype_size(2) == 2 and L.engine_dtype_size(6) == 8
    assert pb.version().startswith("1.0.3")


def test_tensor_roundtrip_host():
    a = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    t = pb.Tensor.from_numpy(a)
    assert t.shape == (2, 3, 4) and t.numel == 24 and t.ndim == 3
    np.testing.assert_array_equal(t.to_numpy(), a)
    assert t.tolist()[1][2][3] == 23.0
    t.fill(2.5)
    assert float(t.to_numpy().sum()) == 60.0
    t.copy_from_list([[[1.0] * 4] * 3] * 2)
    assert t.to_numpy().sum() == 24


def test_error_behaviour_matches_reference():
    L = N.lib()
    assert L.engine_tensor_numel(None) == 0
    h = C.c_void_p()
    shp = (N.i64 * 1)(4)
    assert L.engine_tensor_create(None, shp, 1, 0) == 1                    # NULL_PTR
    assert L.engine_tensor_create_from_data(C.byref(h), shp, 1, 0, None, 0) == 1
    data = (C.c_float * 8)()
    assert L.engine_tensor_create_from_data(C.byref(h), shp, 1, 0, data, 32) == 7   # data too large
    assert b"too large" in L.engine_last_error()
    ctx = pb.Context()
    assert L.engine_context_set_num_threads(ctx.raw, 0) == 7
    assert L.engine_context_set_num_threads(ctx.raw, -3) == 7
    ctx.set_num_threads(3)
    assert ctx.get_num_threads() == 3
    assert L.engine_context_set_num_threads(None, 2) == 2                  # INVALID_HANDLE
    bad = C.create_string_buffer(64)
    assert L.engine_tensor_numel(C.cast(bad, C.c_void_p)) == 0            # magic check


def test_model_load_and_info(tmp_path):
    g, info = build_yolov8("n", imgsz=128)
    p = str(tmp_path / "y.engine")
    write_engine(p, g)
    ctx = pb.Context()
    m = pb.Model(ctx, p)
    assert m.num_inputs == 1 and m.num_outputs == 1
    assert m.input_info(0).shape == (1, 3, 128, 128)
    assert m.output_info(0).shape == (1, 84, 336)
    assert m.name == p
    with pytest.raises(pb.PdefaError):
        pb.Model(ctx, str(tmp_path / "missing.engine"))
    bad = tmp_path / "bad.engine"
    bad.write_bytes(b"NOPE" + b"\0" * 100)
    with pytest.raises(pb.PdefaError):
        pb.Model(ctx, str(bad))


def test_engine_file_roundtrip(tmp_path):
    g, _ = build_yolov8("n", imgsz=64)
    p = str(tmp_path / "a.engine")
    write_engine(p, g)
    g2 = read_engine(p)
    assert len(g2.nodes) == len(g.nodes) and len(g2.weights) == len(g.weights)
    for a, b in zip(g.nodes, g2.nodes):
        assert a.op == b.op and a.inputs == b.inputs and a.outputs == b.outputs
    blob = pack_params(stride_h=2, pad_h=1, axis=3, eps=1e-3, fused_activation=5, leaky_slope=0.2)
    assert len(blob) == 128
    p2 = unpack_params(blob)
    assert p2["stride_h"] == 2 and p2["axis"] == 3 and p2["fused_activation"] == 5


def test_yolov8_flops_match_architecture():
    _, info = build_yolov8("n", imgsz=640)
    assert info["anchors"] == 8400
    assert abs(conv_flops(info) / 1e9 - 8.743) < 0.01
    _, info_m = build_yolov8("m", imgsz=640)
    assert abs(conv_flops(info_m) / 1e9 - 78.94) < 0.2


def test_session_without_gpu_fails_loudly(tmp_path):
    if pb.device_count() > 0:
        pytest.skip("a GPU is present")
    g, _ = build_yolov8("n", imgsz=64)
    p = str(tmp_path / "y.engine")
    write_engine(p, g)
    ctx = pb.Context()
    m = pb.Model(ctx, p)
    with pytest.raises(pb.PdefaError, match="no CUDA device"):
        pb.Session(ctx, m)
    a = pb.Tensor.from_numpy(np.ones((4, 4), np.float32))
    with pytest.raises(pb.PdefaError):
        pb.ops_matmul(a, a)


def test_box_mapping_and_images():
    meta = pb.PreprocessMeta(640, 640, 1280, 720, 0, 140, 640, 360, 0.5)
    b = pb.map_box_to_original(pb.Box(10, 150, 700, 660), meta)
    assert (b.x1, b.y1, b.x2, b.y2) == (20.0, 20.0, 1280.0, 720.0)
    x, y = pb.map_point_to_original(-5.0, 160.0, meta)
    assert (x, y) == (0.0, 40.0)
    with pytest.raises(pb.PdefaError):
        pb.prepare_for_engine("x.jpg", 640, 640)
    assert N.lib().pdefa_image_load(b"x.png") is None
    assert b"cannot read file" in N.lib().pdefa_last_error()


def test_malformed_and_unknown_files_are_reported(tmp_path):
    p = tmp_path / "a.jpg"
    p.write_bytes(b"\xff\xd8\xff\xe0" + bytes(64))          # APP0 with a zero length
    assert N.lib().pdefa_image_load(str(p).encode()) is None
    assert N.lib().pdefa_last_error().startswith(b"load_image: jpeg:")
    p.write_bytes(b"GIF89a" + bytes(64))
    assert N.lib().pdefa_image_load(str(p).encode()) is None
    assert b"unsupported format" in N.lib().pdefa_last_error()
    p.write_bytes(b"\xff\xd8")
    assert N.lib().pdefa_image_load(str(p).encode()) is None
    assert b"too small" in N.lib().pdefa_last_error()


def test_batch_submit_and_wait_argument_checks():
    """pdefa_batch_submit_u8 / pdefa_batch_wait report missing pointers with
    ENGINE_ERR_NULL_PTR (1) before touching a GPU."""
    L = N.lib()
    px = (C.c_uint8 * 12)()
    cfg = N.PreConfig(64, 64, 1.0 / 255.0, 0.0)
    counts = (N.i32 * 1)()
    dets = (N.Detection * 4)()
    ticket = C.c_int64(0)
    assert L.pdefa_batch_wait(None, 0) == 1
    assert L.pdefa_batch_submit_u8(None, px, 1, 2, 2, 3, C.byref(cfg), 0.25, 0.45, 4, counts, dets, None,
                                   C.byref(ticket)) == 1
    fake = C.create_string_buffer(64)          # never dereferenced: the ticket check comes first
    assert L.pdefa_batch_submit_u8(C.cast(fake, C.c_void_p), px, 1, 2, 2, 3, C.byref(cfg), 0.25, 0.45, 4,
                                   counts, dets, None, None) == 1


def test_decode_scratch_size_checks_do_not_wrap():
    """Sizes whose candidate-slot product overflows 64 bits are refused before any
    device work: the allocation-free decode answers ENGINE_ERR_INVALID_ARG (7), and
    the work-size query saturates instead of wrapping to a small number."""
    L = N.lib()
    f = L.pdefa_decode_yolo_noalloc
    f.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_double, C.c_double, C.c_int32,
                  C.c_void_p, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    fake = C.create_string_buffer(64)          # never dereferenced: the size check comes first
    ptr = C.cast(fake, C.c_void_p)
    for batch, anchors in ((1 << 46, 16384), (1 << 40, 1 << 23), (21, 8400)):
        assert f(ptr, batch, 84, anchors, None, 0.25, 0.45, 300, ptr, ptr, None) == 7
        assert b"scratch" in L.pdefa_last_error()
    L.pdefa_decode_work_bytes.restype = C.c_size_t
    L.pdefa_decode_work_bytes.argtypes = [C.c_int64, C.c_int64]
    assert L.pdefa_decode_work_bytes(1 << 46, 16384) == 2 ** 64 - 1
    assert L.pdefa_decode_work_bytes(2, 8400) == 2 * 8400 * 48
