"""ctypes binding of libpdefa_native.so (built in-tree by pdefa_b200.build).

The library is loaded on first use. Its C signatures are those of
include/engine_c_api.h, include/pdefa_c_api.h and include/pdefa_b200_ext.h.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libpdefa_native.so")

vp = C.c_void_p
i32, i64, u64, f32, f64, sz = C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_double, C.c_size_t
P = C.POINTER


class PreConfig(C.Structure):
    """PdefaPreprocessConfig (pdefa/include/pdefa_c_api.h:49-54)."""
    _fields_ = [("target_w", i32), ("target_h", i32), ("scale", f32), ("pad_value", f32)]


class PreMeta(C.Structure):
    """PdefaPreprocessMeta (pdefa/include/pdefa_c_api.h:56-62)."""
    _fields_ = [("target_w", i32), ("target_h", i32), ("orig_w", i32), ("orig_h", i32),
                ("pad_x", i32), ("pad_y", i32), ("scaled_w", i32), ("scaled_h", i32), ("ratio", f32)]


class SessionStats(C.Structure):
    _fields_ = [("last_run_ms", f64), ("runs", u64)]


class Detection(C.Structure):
    """PdefaDetection (include/pdefa_b200_ext.h)."""
    _fields_ = [("x1", f64), ("y1", f64), ("x2", f64), ("y2", f64), ("conf", f32),
                ("cls", i32), ("anchor", i32), ("reserved", i32)]


PROFILE_FN = C.CFUNCTYPE(None, C.c_char_p, f64, vp)

_SIGS = {
    # meta
    "engine_version": ([], C.c_char_p), "engine_last_error": ([], C.c_char_p),
    "engine_status_string": ([C.c_int], C.c_char_p), "engine_dtype_size": ([C.c_int], sz),
    "engine_simd_level": ([], C.c_char_p), "engine_cpu_brand": ([], C.c_char_p),
    "pdefa_version": ([], C.c_char_p), "pdefa_last_error": ([], C.c_char_p),
    # context
    "engine_context_create": ([P(vp)], C.c_int), "engine_context_destroy": ([vp], None),
    "engine_context_set_num_threads": ([vp, i32], C.c_int), "engine_context_get_num_threads": ([vp], i32),
    "engine_context_num_physical_cores": ([], i32), "engine_context_has_avx2": ([], i32),
    "engine_context_has_avx512": ([], i32),
    "engine_context_set_precision": ([vp, i32], C.c_int), "engine_context_get_precision": ([vp], i32),
    "engine_context_set_device": ([vp, i32], C.c_int), "engine_context_get_device": ([vp], i32),
    "engine_device_count": ([], i32), "engine_device_error": ([i32], i32),
    # tensor
    "engine_tensor_create": ([P(vp), P(i64), i32, C.c_int], C.c_int),
    "engine_tensor_create_from_data": ([P(vp), P(i64), i32, C.c_int, vp, sz], C.c_int),
    "engine_tensor_data": ([vp, P(vp), P(sz)], C.c_int),
    "engine_tensor_shape": ([vp, P(i64), P(i32)], C.c_int),
    "engine_tensor_copy_from": ([vp, vp, sz], C.c_int), "engine_tensor_copy_to": ([vp, vp, sz], C.c_int),
    "engine_tensor_numel": ([vp], i64), "engine_tensor_dtype": ([vp], C.c_int),
    "engine_tensor_rank": ([vp], i32), "engine_tensor_destroy": ([vp], None),
    # model
    "engine_model_load": ([vp, C.c_char_p, P(vp)], C.c_int),
    "engine_model_input_count": ([vp, P(i32)], C.c_int), "engine_model_output_count": ([vp, P(i32)], C.c_int),
    "engine_model_name": ([vp, P(C.c_char_p)], C.c_int), "engine_model_destroy": ([vp], None),
    "engine_model_input_info": ([vp, i32, P(C.c_char_p), P(i64), P(i32), P(C.c_int)], C.c_int),
    "engine_model_output_info": ([vp, i32, P(C.c_char_p), P(i64), P(i32), P(C.c_int)], C.c_int),
    # session
    "engine_session_create": ([vp, vp, P(vp)], C.c_int),
    "engine_session_set_input": ([vp, i32, vp], C.c_int), "engine_session_run": ([vp], C.c_int),
    "engine_session_get_output": ([vp, i32, P(vp)], C.c_int), "engine_session_destroy": ([vp], None),
    "engine_session_debug_intermediate": ([vp, i32, P(vp)], C.c_int),
    "engine_session_get_stats": ([vp, P(SessionStats)], C.c_int),
    "engine_session_set_profile_callback": ([vp, PROFILE_FN, vp], C.c_int),
    "engine_session_clear_profile_callback": ([vp], C.c_int),
    "engine_run_simple": ([C.c_char_p, P(vp), i32, P(vp), i32], C.c_int),
    "engine_session_run_device": ([vp, vp, i64, vp, vp], C.c_int),
    "engine_session_output_shape": ([vp, i32, i64, P(i64), P(i32)], C.c_int),
    "engine_session_launch_count": ([vp, i64], i64),
    "engine_session_device_output": ([vp, i32, i64, P(vp)], C.c_int),
    "engine_session_step_timing": ([vp, i64, i32], C.c_int),
    "engine_session_step_times": ([vp, i64, P(f64), i64], i64),
    "pdefa_decode_work_bytes": ([i64, i64], sz),
    "pdefa_decode_yolo_device": ([vp, i64, i64, i64, vp, f64, f64, i32, vp, vp, vp, sz, vp], C.c_int),
    "engine_model_plan_summary": ([vp, i32, i64, C.c_char_p, sz, P(i64)], C.c_int),
    "engine_model_memory_plan": ([vp, i32, i64, P(sz), P(sz)], C.c_int),
    "engine_session_keep_intermediate": ([vp, i32], C.c_int),
    # ops
    "engine_ops_add": ([vp, vp, P(vp)], C.c_int), "engine_ops_sub": ([vp, vp, P(vp)], C.c_int),
    "engine_ops_mul": ([vp, vp, P(vp)], C.c_int), "engine_ops_div": ([vp, vp, P(vp)], C.c_int),
    "engine_ops_matmul": ([vp, vp, vp], C.c_int), "engine_ops_matmul_ex": ([vp, vp, vp, i32], C.c_int),
    "engine_gemm_f32_device": ([vp, vp, vp, i64, i64, i64, i32, vp], C.c_int),
    "engine_ops_relu": ([vp], C.c_int), "engine_ops_silu": ([vp], C.c_int),
    "engine_ops_sigmoid": ([vp], C.c_int), "engine_ops_tanh": ([vp], C.c_int),
    "engine_ops_gelu": ([vp], C.c_int), "engine_ops_clip": ([vp, f32, f32], C.c_int),
    "engine_ops_softmax": ([vp, i32], C.c_int),
    "engine_ops_reduce_max": ([vp, i32, i32, P(vp)], C.c_int),
    "engine_ops_reduce_sum": ([vp, i32, i32, P(vp)], C.c_int),
    "engine_ops_reduce_mean": ([vp, i32, i32, P(vp)], C.c_int),
    "engine_ops_argmax": ([vp, i32, i32, P(vp)], C.c_int),
    "engine_ops_gather": ([vp, vp, i32, P(vp)], C.c_int),
    "engine_ops_reshape": ([vp, P(i64), i32, P(vp)], C.c_int),
    "engine_ops_transpose": ([vp, P(i32), i32, P(vp)], C.c_int),
    "engine_ops_concat": ([P(vp), i32, i32, P(vp)], C.c_int),
    "engine_ops_stack": ([P(vp), i32, i32, P(vp)], C.c_int),
    "engine_random_randn": ([P(i64), i32, u64, P(vp)], C.c_int),
    "engine_random_rand": ([P(i64), i32, u64, P(vp)], C.c_int),
    # pdefa
    "pdefa_image_load": ([C.c_char_p], vp), "pdefa_image_free": ([vp], None),
    "pdefa_image_width": ([vp], i32), "pdefa_image_height": ([vp], i32), "pdefa_image_channels": ([vp], i32),
    "pdefa_image_format": ([vp], i32), "pdefa_image_pixels": ([vp, P(sz)], vp),
    "pdefa_preprocess_letterbox": ([vp, P(PreConfig), P(vp), P(PreMeta)], C.c_int),
    "pdefa_prepare_for_engine": ([C.c_char_p, i32, i32, f32, f32, P(vp), P(PreMeta)], C.c_int),
    "pdefa_load_image_as_tensor": ([C.c_char_p, i32, i32, P(vp)], C.c_int),
    "pdefa_map_box_to_original": ([P(f32), P(PreMeta), P(f32)], C.c_int),
    "pdefa_map_point_to_original": ([P(f32), P(f32), P(PreMeta)], C.c_int),
    "pdefa_decode_yolo": ([vp, i32, i64, i64, i64, P(PreMeta), f64, f64, i32, P(i32), P(Detection), i32], C.c_int),
    "pdefa_batch_create": ([vp, i32, P(i32), i32, i64, P(vp)], C.c_int),
    "pdefa_batch_run": ([vp, vp, i64, P(PreMeta), f64, f64, i32, P(i32), P(Detection)], C.c_int),
    "pdefa_batch_destroy": ([vp], None),
    "pdefa_batch_run_u8": ([vp, vp, i64, i32, i32, i32, P(PreConfig), f64, f64, i32, P(i32), P(Detection),
                            P(PreMeta)], C.c_int),
    "pdefa_batch_submit_u8": ([vp, vp, i64, i32, i32, i32, P(PreConfig), f64, f64, i32, P(i32), P(Detection),
                               P(PreMeta), P(i64)], C.c_int),
    "pdefa_batch_wait": ([vp, i64], C.c_int),
    "pdefa_letterbox_meta": ([i32, i32, P(PreConfig), P(PreMeta)], C.c_int),
    "pdefa_letterbox_device": ([vp, i64, i32, i32, i32, P(PreConfig), vp, vp], C.c_int),
    "pdefa_letterbox": ([vp, i64, i32, i32, i32, P(PreConfig), vp, P(PreMeta), i32], C.c_int),
}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (built on demand when missing)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.isfile(LIB_PATH):
                    from . import build
                    build.build()
                L = C.CDLL(LIB_PATH)
                for name, (args, res) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = L
    return _lib
