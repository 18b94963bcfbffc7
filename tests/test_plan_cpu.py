"""Device-free lowering of the synthetic YOLOv8 graphs (engine_model_plan_summary):
which kernel each layer gets and which reference ops disappear into fusions."""
from collections import Counter

import pytest

import pdefa_b200 as pb
from pdefa_b200.engine_file import write_engine
from pdefa_b200.yolo import build_single_conv, build_yolov8


@pytest.fixture(scope="module")
def y8n(tmp_path_factory):
    g, info = build_yolov8("n", imgsz=640)
    p = str(tmp_path_factory.mktemp("plan") / "y8n.engine")
    write_engine(p, g)
    return pb.Model(pb.Context(), p), info


def test_bf16_plan_is_all_tensor_core_and_copy_free(y8n):
    m, info = y8n
    steps = m.plan_summary(pb.BF16, batch=256)
    kinds = Counter(k for k, _ in steps)
    # 63 convs, all on tcgen05: the stem (Cin=3, NCHW fp32 input) gathers its own
    # im2col rows (conv_stem_tc), the other 62 stream operands with TMA
    assert kinds["conv_stem_tc"] == 1 and kinds["conv_tc_bf16"] == 62
    assert kinds["yolo_head"] == 1
    # SPPF's three chained 5x5 max pools run as one launch that reads its input once
    assert kinds["pool"] == 1 and kinds["resize"] == 2
    # C2f splits are views, concats are zero-copy, residual Adds live in conv epilogues
    assert kinds["copy"] == 0 and kinds["binary"] == 0 and kinds["unary"] == 0
    assert len(steps) == 67
    assert steps[0] == ("conv_stem_tc", "/model.0/conv/Conv")


def test_fp32_plan_uses_strict_kernels_only(y8n):
    m, _ = y8n
    kinds = Counter(k for k, _ in m.plan_summary(pb.FP32, batch=1))
    assert kinds["conv_direct"] == 1 and kinds["conv_simt"] == 62 and not any(k.startswith("conv_tc") for k in kinds)


def test_tf32_plan(y8n):
    m, _ = y8n
    kinds = Counter(k for k, _ in m.plan_summary(pb.TF32, batch=4))
    assert kinds["conv_tc_tf32"] == 62


def test_unfused_head_lowers_generic_ops(y8n, monkeypatch):
    m, _ = y8n
    monkeypatch.setenv("PDEFA_NO_HEAD_FUSION", "1")
    kinds = Counter(k for k, _ in m.plan_summary(pb.FP32, batch=1))
    assert kinds["yolo_head"] == 0 and kinds["softmax"] == 1 and kinds["binary"] >= 6


def test_stem_plan(tmp_path):
    g, _ = build_single_conv(hw=640)
    p = str(tmp_path / "stem.engine")
    write_engine(p, g)
    steps = pb.Model(pb.Context(), p).plan_summary(pb.BF16, 1)
    assert [k for k, _ in steps] == ["conv_stem_tc", "copy"]     # conv + NHWC->NCHW output


@pytest.mark.parametrize("prec", [pb.FP32, pb.TF32, pb.BF16])
def test_grouped_conv_plan(tmp_path, prec):
    """Depthwise / grouped convs lower to the grouped-conv kernel in every precision."""
    g, _ = build_single_conv(cin=32, cout=32, k=3, s=1, hw=40, groups=32)
    p = str(tmp_path / "dw.engine")
    write_engine(p, g)
    kinds = [k for k, _ in pb.Model(pb.Context(), p).plan_summary(prec, 2)]
    assert "conv_grouped" in kinds and not any(k.startswith("conv_tc") for k in kinds)


def test_yolo11n_plan_lowers_attention(tmp_path):
    """YOLO11n: C3k2 and the Detect head on tcgen05 (depthwise class branches on the
    grouped-conv kernel), the C2PSA attention on matmul_heads + softmax."""
    from pdefa_b200.yolo import build_yolo11
    g, _ = build_yolo11("n", imgsz=640)
    p = str(tmp_path / "y11n.engine")
    write_engine(p, g)
    m = pb.Model(pb.Context(), p)
    for prec in (pb.BF16, pb.TF32, pb.FP32):
        kinds = Counter(k for k, _ in m.plan_summary(prec, batch=8))
        # the scale Mul and both Transposes fold into the attention products
        assert kinds["matmul_heads"] == 2 and kinds["softmax"] == 1 and kinds["binary"] == 0
        assert kinds["conv_grouped"] == 7 and kinds["yolo_head"] == 1 and kinds["resize"] == 2
    # the 8-channel C3k2 bottleneck convs (16->8 1x1, 8->16 3x3) are padded to 16
    # channels and join the other 77 convs on tcgen05
    kinds = Counter(k for k, _ in m.plan_summary(pb.BF16, batch=8))
    assert kinds["conv_stem_tc"] == 1 and kinds["conv_tc_bf16"] == 79 and kinds["conv_simt"] == 0
    assert kinds["conv_direct"] == 0


def test_memory_plan_reuses_activation_storage(y8n):
    """Live-range packing (engine_model_memory_plan): YOLOv8n-640 at 256 images keeps
    its BF16 activations in a fraction of the one-buffer-per-value footprint; the
    planner's own self-check rejects any overlap of live buffers."""
    m, _ = y8n
    packed, unpacked = m.memory_plan(pb.BF16, batch=256)
    assert unpacked > 8e9
    assert packed < 0.2 * unpacked and packed < 2e9
    p1, u1 = m.memory_plan(pb.FP32, batch=1)
    assert 0 < p1 < u1
