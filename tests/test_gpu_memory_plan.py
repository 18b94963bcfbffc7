"""Activation arena and intermediates on the GPU: with live-range reuse in place the
full graph still matches the reference golden, and an intermediate kept with
engine_session_keep_intermediate reads back (engine_session_debug_intermediate,
PDEFA1.0/src/api/engine_api.cpp:876-892) exactly as the same graph computes it when
that tensor is its output. Intermediates neither kept nor unconsumed are freed after
their last consumer, as in the reference (PDEFA1.0/src/core/session.cpp:322-337)."""
import os

import numpy as np
import pytest

import pdefa_b200 as pb
from pdefa_b200.engine_file import TensorInfo, write_engine
from pdefa_b200.yolo import build_yolov8

pytestmark = pytest.mark.gpu


def _session(path):
    ctx = pb.Context(precision=pb.FP32, device=0)
    m = pb.Model(ctx, path)
    return pb.Session(ctx, m)


def test_kept_intermediate_reads_back(tmp_path, golden):
    d = golden("yolov8n_128.npz")
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(tmp_path / "y8n.engine")
    write_engine(p, g)
    s = _session(p)
    s.keep_intermediate(8)           # /model.2/cv1 (after the fused SiLU), consumed by two Splits
    s.set_input(0, pb.Tensor.from_numpy(d["x"]))
    s.run()
    y = s.output(0).to_numpy()
    assert float(np.abs(y - d["y"]).max() / np.abs(d["y"]).max()) <= 1e-5
    t = s.debug_intermediate(8).to_numpy()
    assert t.shape == (1, 32, 32, 32)                 # engine layout: NHWC
    # the same graph with tensor 8 as its output (converted to NCHW by the session)
    g.graph_outputs = [8]
    g.output_infos = [TensorInfo("cv1", [1, 32, 32, 32])]
    p2 = str(tmp_path / "cut.engine")
    write_engine(p2, g)
    s2 = _session(p2)
    s2.set_input(0, pb.Tensor.from_numpy(d["x"]))
    s2.run()
    ref = s2.output(0).to_numpy()
    np.testing.assert_array_equal(t.transpose(0, 3, 1, 2), ref)
    # a consumed intermediate that was not kept is gone, as in the reference
    with pytest.raises(pb.PdefaError, match="intermediate not available"):
        s.debug_intermediate(11)


def test_full_graph_parity_with_arena_at_batch(tmp_path, golden):
    """A batch of 6 copies of the golden image through the packed arena: every image's
    output equals the golden (values that share storage never overlap in time)."""
    d = golden("yolov8n_128.npz")
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(tmp_path / "y8n.engine")
    write_engine(p, g)
    for prec, tol in ((pb.FP32, 1e-5), (pb.BF16, 1e-2)):
        ctx = pb.Context(precision=prec, device=0)
        s = pb.Session(ctx, pb.Model(ctx, p))
        x = np.concatenate([d["x"]] * 6)
        s.set_input(0, pb.Tensor.from_numpy(x))
        s.run()
        y = s.output(0).to_numpy()
        for b in range(6):
            assert float(np.abs(y[b] - d["y"][0]).max() / np.abs(d["y"]).max()) <= tol, (prec, b)
