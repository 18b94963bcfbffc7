"""Single-layer micro-benchmark: one Conv-BN-SiLU layer through the engine.

    python -m pdefa_b200.layerbench --cin 64 --cout 64 --k 3 --s 1 --hw 40 --batch 512

Builds a one-conv ``.engine`` graph (``yolo.build_single_conv``), runs it on the
current GPU with per-launch CUDA-event timing and prints one JSON line per layer
with the conv launch's milliseconds, TFLOP/s, algorithmic HBM GB/s and the
fraction of the roofline (max of the FLOP and byte bounds). The graph input is
fp32 NCHW, so for Cin > 8 the plan's first launch stages it into the NHWC operand
layout; only the conv launch is reported. Used to size and profile the conv
kernels one layer shape at a time (a capture tool can target it with ``-k``).
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile


def run_layer(cin, cout, k, s, hw, batch, precision="bf16", reps=5, warmup=3, act=True):
    import torch

    import pdefa_b200 as pb
    from pdefa_b200.engine_file import write_engine
    from pdefa_b200.yolo import build_single_conv

    prec = {"bf16": pb.BF16, "tf32": pb.TF32, "fp32": pb.FP32}[precision]
    g, _ = build_single_conv(cin=cin, cout=cout, k=k, s=s, hw=hw, act=act)
    path = os.path.join(tempfile.mkdtemp(), "layer.engine")
    write_engine(path, g)
    ctx = pb.Context(precision=prec)
    model = pb.Model(ctx, path)
    sess = pb.Session(ctx, model)
    x = torch.rand((batch, cin, hw, hw), device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
    ts = torch.cuda.Stream()
    torch.cuda.set_stream(ts)
    for _ in range(warmup):
        sess.run_device(x.data_ptr(), batch, None, ts.cuda_stream)
    torch.cuda.synchronize()
    summary = model.plan_summary(prec, batch)
    sess.set_step_timing(batch, True)
    for _ in range(reps):
        sess.run_device(x.data_ptr(), batch, None, ts.cuda_stream)
    torch.cuda.synchronize()
    times = sess.step_times(batch)
    sess.set_step_timing(batch, False)
    i = next(j for j, (kind, _) in enumerate(summary) if kind.startswith("conv"))
    ms = times[i] / reps
    p = k // 2
    ho = (hw + 2 * p - k) // s + 1
    in_esz = 4 if summary[i][0] in ("conv_direct", "conv_stem_tc") or prec != pb.BF16 else 2   # fp32 graph input read in place
    out_esz = 2 if prec == pb.BF16 else 4
    flops = 2.0 * cin * cout * k * k * ho * ho * batch
    bytes_ = float((in_esz * cin * hw * hw + out_esz * cout * ho * ho) * batch)
    return {"layer": f"conv{k}x{k}s{s} {cin}->{cout} @{hw}x{hw}", "batch": batch, "kind": summary[i][0],
            "ms": ms, "tflops": flops / ms / 1e9, "gbs": bytes_ / ms / 1e6, "flops": flops, "bytes": bytes_}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--cin", type=int, default=64)
    ap.add_argument("--cout", type=int, default=64)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--s", type=int, default=1)
    ap.add_argument("--hw", type=int, default=40)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--precision", default="bf16", choices=["bf16", "tf32", "fp32"])
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--sweep-yolov8n", action="store_true",
                    help="every distinct conv shape of YOLOv8n-640 at --batch")
    args = ap.parse_args()
    peaks = {}
    pp = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            peaks = json.load(f)
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    tfl = float(peaks.get("bf16_tflops", 1590.0))
    shapes = [(args.cin, args.cout, args.k, args.s, args.hw)]
    if args.sweep_yolov8n:
        from pdefa_b200.yolo import build_yolov8
        _, info = build_yolov8("n", imgsz=640, seed=0)
        seen = []
        for _, cin, cout, k, s, h, w in info["convs"]:
            if (cin, cout, k, s, h) not in seen:
                seen.append((cin, cout, k, s, h))
        shapes = seen
    for cin, cout, k, s, hw in shapes:
        r = run_layer(cin, cout, k, s, hw, args.batch, args.precision, args.reps, args.warmup)
        t_flop = r["flops"] / tfl / 1e9
        t_byte = r["bytes"] / hbm / 1e6
        r["roofline_frac"] = max(t_flop, t_byte) / r["ms"]
        r["bound"] = "tensor" if t_flop > t_byte else "hbm"
        print(json.dumps({k2: (round(v, 4) if isinstance(v, float) else v) for k2, v in r.items()}), flush=True)


if __name__ == "__main__":
    main()
