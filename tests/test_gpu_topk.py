"""TopK and GatherElements (the YOLOv10 end-to-end tail ops,
PDEFA1.0/src/core/session_parts/session_ops_math.inc:321-433) against the compiled
reference engine on the same inputs: values and gathered values bit for bit, the
positions against numpy. The reference orders equal values as std::partial_sort leaves
them (unspecified); equal values are the same numbers either way, so the value outputs
still match exactly on inputs with many ties, and the positions here put the lower
position first."""
import os

import numpy as np
import pytest

import pdefa_b200 as pb
from pdefa_b200.engine_file import EngineGraph, TensorInfo, write_engine

pytestmark = pytest.mark.gpu


def build_topk_graph(shape, k, axis):
    """x -> TopK(k, axis) -> (values, positions); GatherElements(x, positions, axis);
    outputs: values, gathered values, positions."""
    g = EngineGraph()
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("x", list(shape))]
    kw = g.add_weight("k", np.array([k], dtype=np.float32))
    vals, idx = g.add_node("TopK", "/TopK", [-1, kw], n_out=2, axis=axis)
    (gat,) = g.add_node("GatherElements", "/GatherElements", [-1, idx], axis=axis)
    g.graph_outputs = [vals, gat, idx]
    out = list(shape)
    out[axis] = k if 0 < k <= shape[axis] else shape[axis]
    g.output_infos = [TensorInfo("values", out), TensorInfo("gathered", out), TensorInfo("positions", out)]
    return g


def _ours(path, x):
    ctx = pb.Context(precision=pb.FP32, device=0)
    s = pb.Session(ctx, pb.Model(ctx, path))
    s.set_input(0, pb.Tensor.from_numpy(x))
    s.run()
    return [s.output(i).to_numpy() for i in range(3)]


def _reference(path, x):
    from oracle import ref_engine as R
    if not R.available():
        pytest.skip("compiled reference engine (oracle/_ref) not built")
    return R.RefSession(path, threads=4).run_all(x, 2)   # values, gathered (positions are I32 there)


@pytest.mark.parametrize("shape,k,axis,ties", [
    ((1, 84, 1000), 100, 2, False),
    ((1, 84, 1000), 10, 1, False),
    ((1, 8400, 6), 300, 1, False),
    ((1, 24000), 300, 1, False),          # flattened class scores of the YOLOv10 tail
    ((1, 300, 80), 0, 2, False),          # k <= 0: the whole axis
    ((1, 64, 2000), 50, 2, True),         # many equal values
])
def test_topk_gather_elements_against_reference(tmp_path, shape, k, axis, ties):
    p = str(tmp_path / "topk.engine")
    write_engine(p, build_topk_graph(shape, k, axis))
    rng = np.random.default_rng(sum(shape) + k)
    x = rng.standard_normal(shape).astype(np.float32)
    if ties:
        x = np.round(x * 4) / 4
    vals, gat, pos = _ours(p, x)
    rv, rg = _reference(p, x)
    np.testing.assert_array_equal(vals, rv)
    np.testing.assert_array_equal(gat, rg)
    np.testing.assert_array_equal(gat, vals)
    # positions: a stable descending order along the axis (lower position first on ties)
    kk = vals.shape[axis]
    order = np.argsort(-x, axis=axis, kind="stable")
    exp = np.take(order, np.arange(kk), axis=axis)
    np.testing.assert_array_equal(pos.astype(np.int64), exp)


def test_topk_batch_images_independent(tmp_path):
    p = str(tmp_path / "topk_b.engine")
    write_engine(p, build_topk_graph((1, 84, 1000), 100, 2))
    x = np.random.default_rng(5).standard_normal((3, 84, 1000)).astype(np.float32)
    vb, gb, pb_ = _ours(p, x)
    for i in range(3):
        v1, g1, p1 = _ours(p, x[i:i + 1])
        np.testing.assert_array_equal(vb[i:i + 1], v1)
        np.testing.assert_array_equal(pb_[i:i + 1], p1)
