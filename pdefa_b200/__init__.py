"""pdefa_b200 - B200-native drop-in for pdefa's YOLOv8 hot path.

The public names mirror pdefa (pdefa/python/src/pdefa/__init__.py:45-139). The
native library (lib/libpdefa_native.so, C ABI of pdefa.def plus the additive
include/pdefa_b200_ext.h) is loaded on first use.
"""
__version__ = "1.0.3-b200"

from .api import (  # noqa: F401
    BF16, FP32, TF32,
    Box, Context, EngineModel, Image, Model, PdefaError, PreprocessMeta, Session, Tensor, TensorInfo,
    _model_input_shape, cpu_brand, decode_yolo, decode_yolo_arrays, device_count, empty, from_list,
    letterbox_meta, letterbox_u8, load, load_image, load_image_as_tensor, map_box_to_original, map_point_to_original, ones,
    ops_add, ops_argmax, ops_clip, ops_concat, ops_div, ops_gather, ops_gelu, ops_matmul, ops_mul,
    ops_reduce_max, ops_reduce_mean, ops_reduce_sum, ops_relu, ops_reshape, ops_sigmoid, ops_silu,
    ops_softmax, ops_stack, ops_sub, ops_tanh, ops_transpose, prepare_for_engine, prepare_for_model,
    preprocess_letterbox, rand, randn, random_rand, random_randn, simd_level, tensor_empty, version,
    zeros,
)
from .batch import BatchInference  # noqa: F401

__all__ = [
    "PdefaError", "PreprocessMeta", "Box", "Tensor", "TensorInfo", "Context", "Model", "Session", "Image",
    "version", "simd_level", "cpu_brand", "device_count",
    "load_image", "preprocess_letterbox", "prepare_for_engine", "load_image_as_tensor",
    "map_box_to_original", "map_point_to_original", "decode_yolo", "decode_yolo_arrays", "prepare_for_model",
    "letterbox_u8", "letterbox_meta",
    "ops_matmul", "ops_relu", "ops_silu", "tensor_empty",
    "ops_add", "ops_sub", "ops_mul", "ops_div",
    "ops_sigmoid", "ops_tanh", "ops_gelu", "ops_clip", "ops_softmax",
    "ops_reduce_max", "ops_reduce_sum", "ops_reduce_mean",
    "ops_argmax", "ops_gather", "ops_reshape", "ops_transpose", "ops_concat", "ops_stack",
    "random_randn", "random_rand", "randn", "rand", "zeros", "ones", "empty", "from_list",
    "load", "EngineModel", "BatchInference", "FP32", "TF32", "BF16",
]
