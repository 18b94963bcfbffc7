"""Failure detection without a GPU fault. PDEFA_WAIT_LIMIT_CYCLES (read when a plan is
lowered; test use only) shortens the pipeline waits of the tcgen05 conv kernel to a
few dozen SM cycles, so on a small conv they run out long before their TMA copies
land: every CTA records a code in its plan's error word, stops issuing, drains the
copies it started (those waits keep the normal limit), waits for its issued MMAs,
frees TMEM and exits. The session then reports ENGINE_ERR_RUNTIME, and because each
plan has its own error word, a session lowered earlier keeps computing correct
results, as does a new session with the normal limit."""
import os

import numpy as np
import pytest

import pdefa_b200 as pb
from pdefa_b200.engine_file import write_engine
from pdefa_b200.yolo import build_single_conv

pytestmark = pytest.mark.gpu


def _session(model, ctx, x):
    s = pb.Session(ctx, model)
    s.set_input(0, pb.Tensor.from_numpy(x))
    return s


def test_conv_wait_timeout_is_reported_and_contained(tmp_path):
    g, _ = build_single_conv(cin=64, cout=64, k=3, s=1, hw=40, seed=5)
    p = str(tmp_path / "conv.engine")
    write_engine(p, g)
    ctx = pb.Context(precision=pb.BF16, device=0)
    model = pb.Model(ctx, p)
    assert [k for k, _ in model.plan_summary(pb.BF16, 2)].count("conv_tc_bf16") == 1
    x = np.random.default_rng(9).random((2, 64, 40, 40), dtype=np.float32)

    healthy = _session(model, ctx, x)
    healthy.run()
    y0 = healthy.output(0).to_numpy().copy()
    assert np.isfinite(y0).all() and np.abs(y0).max() > 0

    os.environ["PDEFA_WAIT_LIMIT_CYCLES"] = "64"
    try:
        bad = _session(model, ctx, x)
        with pytest.raises(pb.PdefaError, match="timed out"):
            bad.run()
        # the error was cleared when it was reported; the plan keeps its short limit
        with pytest.raises(pb.PdefaError, match="timed out"):
            bad.run()
    finally:
        del os.environ["PDEFA_WAIT_LIMIT_CYCLES"]

    # the other plan's error word is its own: the earlier session is unaffected
    healthy.run()
    np.testing.assert_array_equal(healthy.output(0).to_numpy(), y0)
    # a session lowered with the normal limit computes the same result
    fresh = _session(model, ctx, x)
    fresh.run()
    np.testing.assert_array_equal(fresh.output(0).to_numpy(), y0)
