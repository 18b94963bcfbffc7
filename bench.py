"""Throughput benchmark: YOLOv8n-640 images/s on 1..8 B200 (configs[3] of BASELINE.json).

One step = one batched forward pass of a random-init YOLOv8n over `--batch` (256)
synthetic 640x640 images per GPU with BF16 tcgen05 convolutions, followed by the GPU
decode + class-wise NMS (conf 0.25, IoU 0.45, max_det 300). One process per GPU
(torchrun); replicas are independent, so the work scales weakly and there is no
collective on the data path (one all-reduce of the timings at the end).

Printed JSON line (rank 0):
* value: images/s over all GPUs with inputs resident in HBM (seeded torch.rand on the
  device, 1.26 GB per GPU > L2, so no L2 flush is needed), device-timed with CUDA
  events, max over ranks;
* e2e: the same through the public batch API from pinned host images to host
  detections: 8-bit RGB frames at the model size, whose scale-only letterbox the stem
  conv applies as it reads them (frames of another size are letterboxed by a GPU
  kernel first), one step per call of the
  pipelined BatchInference.submit_u8 (pdefa_batch_submit_u8; step k's detections are
  read after step k+1 is queued), also as e2e.sync_value through the blocking
  detect_u8 (pdefa_batch_run_u8), and under e2e.f32_input float32 NCHW tensors
  (detect_arrays -> pdefa_batch_run); the runner pipelines micro-batches of
  --e2e-micro (256) images (copy of one overlapping the inference of the previous);
* roofline: the tcgen05 convolution kernels of the step (the dominant kernel
  family): conv FLOPs / their CUDA-event time measured inside the timed region,
  against the measured sustained BF16 peak;
* cpu_baseline: the reference CPU engine (oracle/_ref, built from the reference
  sources) + the restated reference decode on a bounded sample, rank 0 only.
`--impl reference` times that CPU path alone as the reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "YOLOv8n-640 images/sec at 1/2/4/8 B200; conv TFLOP/s vs tensor-core peak"


# DRAM bytes (read + write) per image over the 62 conv_tc launches of one YOLOv8n-640
# BF16 step: one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of a whole
# step at batch 32, divided by 32 (profiles/conv_tc_dram_traffic_yolov8n640.md). Every
# launch streams its images once, so the figure is scaled to the bench batch by images;
# at batch 32 more producer->consumer pairs stay in L2 than at 256, so it is a lower
# bound there.
CONV_TC_DRAM_BYTES_PER_IMAGE_B32 = 48.1e6


def per_layer_roofline(summary, step_ms, steps, info, B, peak_tflops, hbm_gbs, abytes):
    """(bound ms, measured ms) summed over the conv launches: each layer's bound is
    max(FLOPs / tensor peak, bytes / HBM bandwidth), bytes = activations in (fp32 for
    the stem's graph input) and out once."""
    layer_of = {name: (cin, cout, k, s, h, w) for name, cin, cout, k, s, h, w in info["convs"]}
    ideal = meas = 0.0
    for i, (kd, name) in enumerate(summary):
        key = name.strip("/").replace("/conv/Conv", "")
        if not kd.startswith("conv") or key not in layer_of:
            continue
        cin, cout, k, s, h, w = layer_of[key]
        ho, wo = (h + 2 * (k // 2) - k) // s + 1, (w + 2 * (k // 2) - k) // s + 1
        fl = 2.0 * cin * cout * k * k * ho * wo * B
        by = ((4 if kd.startswith("conv_stem") or kd == "conv_direct" else abytes) * cin * h * w
              + abytes * cout * ho * wo) * B
        ideal += max(fl / (peak_tflops * 1e12), by / (hbm_gbs * 1e9)) * 1e3
        meas += step_ms[i] / steps
    return ideal, meas


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_model(name: str, imgsz: int):
    """(graph, info) of the benchmarked model: yolov8n (the headline config), yolov8m
    (configs[4], run with --precision tf32 --batch 64) or yolo11n."""
    from pdefa_b200.yolo import build_yolo11, build_yolov8
    if name == "yolo11n":
        return build_yolo11("n", imgsz=imgsz, seed=0)
    return build_yolov8(name[-1], imgsz=imgsz, seed=0)


def cpu_reference(images: int, threads: int, model: str = "yolov8n"):
    """Reference CPU path on `images` images: engine (oracle/_ref) batch-1 + decode restatement."""
    import numpy as np
    from oracle import decode_ref, ref_engine as R
    from pdefa_b200.engine_file import write_engine
    if not R.available():
        return None
    g, _ = build_model(model, 640)
    p = os.path.join(tempfile.mkdtemp(), "y8n_ref.engine")
    write_engine(p, g)
    sess = R.RefSession(p, threads=threads)
    x = np.random.default_rng(0).random((1, 3, 640, 640), dtype=np.float32)
    sess.run(x)   # warm-up (weight caches)

    def step(n):
        t0 = time.perf_counter()
        for i in range(n):
            y = sess.run(x)
            decode_ref.decode(y[0], None, 0.25, 0.45, 300)
        return time.perf_counter() - t0
    return step


def cpu_model():
    """Host CPU model name (the line /proc/cpuinfo gives), for the CPU baseline records."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference_arm(args, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    step = cpu_reference(args.ref_images, threads, args.model)
    if step is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference engine not built (oracle/_ref missing)"}))
        return
    for _ in range(args.warmup):
        step(args.ref_images)
    ts = [step(args.ref_images) for _ in range(args.steps)]
    tot = sum(ts)
    value = args.ref_images * args.steps / tot
    sample = (f"{args.ref_images} images per step, batch-1 Session.run of the reference engine "
              f"(oracle/_ref, AVX2) + reference decode/NMS restated in Python (oracle/decode_ref.py)")
    # the reference's CPU path on configs[0], [1] and [4] (same shapes as our records)
    configs = None
    if not args.no_configs:
        import numpy as np
        from oracle import ref_engine as R
        from pdefa_b200.engine_file import write_engine
        from pdefa_b200.yolo import build_single_conv, build_yolov8
        rng = np.random.default_rng(42)
        A = rng.standard_normal((512, 512), dtype=np.float32)
        Bm = rng.standard_normal((512, 512), dtype=np.float32)
        R.time_matmul(A, Bm, 3, threads)
        mm_ms = R.time_matmul(A, Bm, 30, threads) * 1e3
        g, _ = build_single_conv(cin=3, cout=16, k=3, s=2, hw=640, act=True, seed=1)
        sp = os.path.join(tempfile.mkdtemp(), "stem.engine")
        write_engine(sp, g)
        x = np.random.default_rng(0).random((1, 3, 640, 640), dtype=np.float32)
        rs = R.RefSession(sp, threads=threads)
        rs.time_run(x, 3)
        stem_ms = rs.time_run(x, 20) * 1e3
        g, _ = build_yolov8("m", imgsz=640, seed=0)
        mp = os.path.join(tempfile.mkdtemp(), "y8m.engine")
        write_engine(mp, g)
        rm = R.RefSession(mp, threads=threads)
        rm.time_run(x, 1)
        m_s = rm.time_run(x, 3)
        configs = {"configs[0]_ops_matmul_512": {"fp32_call_ms": round(mm_ms, 4),
                                                "gflops": round(2 * 512 ** 3 / mm_ms / 1e6, 1),
                                                "api": "engine_ops_matmul (AVX2 sgemm, matmul_avx2.cpp:538-681)"},
                   "configs[1]_stem_conv": {"fp32_b1_ms": round(stem_ms, 4), "path": "Session.run, direct NHWC conv"},
                   "configs[4]_yolov8m_tf32_b64": {"images_per_s": round(1.0 / m_s, 3),
                                                   "sample": "3 images, batch-1 Session.run, FP32"}}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config(args, 1),
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "reference", "sample": sample,
                         "cpu": cpu_model()},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "configs": configs,
    }))


def run_layers(args):
    """--layer CIN,COUT,K,S,HW / --sweep-layers: one conv layer (Conv-BN-SiLU graph of
    yolo.build_single_conv) at a time through the engine, per-launch CUDA-event time
    of the conv launch, its TFLOP/s, algorithmic HBM GB/s and the fraction of its
    roofline max(FLOPs / sustained tensor peak, bytes / HBM bandwidth). One JSON line
    per layer. The graph input is fp32 NCHW, so for Cin > 8 the plan's first launch
    stages it into the NHWC operand layout; only the conv launch is reported."""
    import torch

    import pdefa_b200 as pb
    from pdefa_b200.engine_file import write_engine
    from pdefa_b200.yolo import build_single_conv, build_yolov8

    hbm, _, peak_sus, src = load_peaks()
    prec = {"bf16": pb.BF16, "tf32": pb.TF32, "fp32": pb.FP32}[args.precision]
    if args.precision == "tf32":
        peak_sus /= 2
    if args.sweep_layers:
        _, info = build_yolov8("n", imgsz=640, seed=0)
        shapes = []
        for _, cin, cout, k, s, h, w in info["convs"]:
            if (cin, cout, k, s, h) not in shapes:
                shapes.append((cin, cout, k, s, h))
    else:
        shapes = [tuple(int(v) for v in args.layer.split(","))]
    torch.cuda.set_device(0)
    ts = torch.cuda.Stream()
    torch.cuda.set_stream(ts)
    for cin, cout, k, s, hw in shapes:
        g, _ = build_single_conv(cin=cin, cout=cout, k=k, s=s, hw=hw, act=True)
        path = os.path.join(tempfile.mkdtemp(), "layer.engine")
        write_engine(path, g)
        ctx = pb.Context(precision=prec)
        model = pb.Model(ctx, path)
        sess = pb.Session(ctx, model)
        B = args.batch
        x = torch.rand((B, cin, hw, hw), device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
        for _ in range(args.warmup):
            sess.run_device(x.data_ptr(), B, None, ts.cuda_stream)
        torch.cuda.synchronize()
        summary = model.plan_summary(prec, B)
        sess.set_step_timing(B, True)
        for _ in range(args.steps):
            sess.run_device(x.data_ptr(), B, None, ts.cuda_stream)
        torch.cuda.synchronize()
        times = sess.step_times(B)
        sess.set_step_timing(B, False)
        i = next(j for j, (kind, _) in enumerate(summary) if kind.startswith("conv"))
        ms = times[i] / args.steps
        ho = (hw + 2 * (k // 2) - k) // s + 1
        in_esz = 4 if summary[i][0] in ("conv_direct", "conv_stem_tc") or prec != pb.BF16 else 2
        out_esz = 2 if prec == pb.BF16 else 4
        flops = 2.0 * cin * cout * k * k * ho * ho * B
        nbytes = float((in_esz * cin * hw * hw + out_esz * cout * ho * ho) * B)
        t_flop, t_byte = flops / peak_sus / 1e9, nbytes / hbm / 1e6
        print(json.dumps({"layer": f"conv{k}x{k}s{s} {cin}->{cout} @{hw}x{hw}", "batch": B, "kind": summary[i][0],
                          "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                          "gbs": round(nbytes / ms / 1e6, 1), "bound": "tensor" if t_flop > t_byte else "hbm",
                          "bound_ms": round(max(t_flop, t_byte), 4), "roofline_frac": round(max(t_flop, t_byte) / ms, 3),
                          "peaks": f"{src}: {peak_sus:.1f} TFLOP/s sustained, {hbm:.0f} GB/s"}), flush=True)


def measure_configs(args, local):
    """BASELINE.json configs[0], [1] and [4] on this GPU (rank 0, one GPU): per-config
    records of the same JSON line.
    * ops_matmul A[512,512] @ B[512,512] (seed 42, N(0,1)) through the C ABI
      with host tensors (engine_ops_matmul_ex: copies in, GEMM, copy out: the call a
      ctypes user makes), median over calls, per precision; plus the device GEMM alone
      (engine_gemm_f32_device on resident operands, CUDA events, mean of 200).
    * the stem Conv-BN-SiLU [1,3,640,640] -> [1,16,320,320] (3x3 s2) through
      a Session at batch 1 (FP32 strict and BF16), the conv launch's CUDA-event time and
      its HBM GB/s (fp32 input read in place, output once), also at batch 256.
    * YOLOv8m-640 random-init, TF32 tcgen05 convs, 64 images per GPU:
      images/s (inference, device-timed), conv TFLOP/s and the per-layer roofline
      fraction against the TF32 peak (half the measured BF16 sustained figure)."""
    import numpy as np
    import torch

    import pdefa_b200 as pb
    from pdefa_b200 import _native as N
    from pdefa_b200.engine_file import write_engine
    from pdefa_b200.yolo import build_single_conv, build_yolov8, conv_flops

    hbm, _, peak_sus, src = load_peaks()
    L = N.lib()
    res = {}
    # ---- configs[0]
    rng = np.random.default_rng(42)
    A = rng.standard_normal((512, 512), dtype=np.float32)
    Bm = rng.standard_normal((512, 512), dtype=np.float32)
    ta, tb = pb.Tensor.from_numpy(A), pb.Tensor.from_numpy(Bm)
    ref = A.astype(np.float64) @ Bm.astype(np.float64)
    flop = 2.0 * 512 ** 3
    da = torch.from_numpy(A).cuda()
    db = torch.from_numpy(Bm).cuda()
    dc = torch.empty((512, 512), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    mm = {}
    for name, prec in (("fp32", pb.FP32), ("tf32", pb.TF32), ("bf16", pb.BF16)):
        tc = pb.tensor_empty([512, 512])
        for _ in range(5):
            pb.ops_matmul(ta, tb, tc, precision=prec)
        ts = []
        for _ in range(30):
            t0 = time.perf_counter()
            pb.ops_matmul(ta, tb, tc, precision=prec)
            ts.append(time.perf_counter() - t0)
        ts.sort()
        call_ms = ts[len(ts) // 2] * 1e3
        err = float(np.abs(tc.to_numpy() - ref).max() / np.abs(ref).max())
        for _ in range(10):
            L.engine_gemm_f32_device(da.data_ptr(), db.data_ptr(), dc.data_ptr(), 512, 512, 512, prec, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(200):
            L.engine_gemm_f32_device(da.data_ptr(), db.data_ptr(), dc.data_ptr(), 512, 512, 512, prec, stream)
        e1.record()
        torch.cuda.synchronize()
        dev_ms = e0.elapsed_time(e1) / 200
        mm[name] = {"call_ms": round(call_ms, 4), "call_gflops": round(flop / call_ms / 1e6, 1),
                    "device_ms": round(dev_ms, 5), "device_tflops": round(flop / dev_ms / 1e9, 2),
                    "normwise_err_vs_f64": err}
    res["configs[0]_ops_matmul_512"] = {
        "api": "engine_ops_matmul_ex, host tensors (H2D of A and B, GEMM, D2H of C inside each call)", **mm}
    # ---- configs[1]
    g, _ = build_single_conv(cin=3, cout=16, k=3, s=2, hw=640, act=True, seed=1)
    path = os.path.join(tempfile.mkdtemp(), "stem.engine")
    write_engine(path, g)
    stem = {}
    for name, prec, batch in (("fp32_b1", pb.FP32, 1), ("bf16_b1", pb.BF16, 1), ("bf16_b256", pb.BF16, 256)):
        ctx = pb.Context(precision=prec, device=local)
        model = pb.Model(ctx, path)
        sess = pb.Session(ctx, model)
        x = torch.rand((batch, 3, 640, 640), device="cuda", generator=torch.Generator(device="cuda").manual_seed(0))
        for _ in range(3):
            sess.run_device(x.data_ptr(), batch, None, stream)
        torch.cuda.synchronize()
        summary = model.plan_summary(prec, batch)
        reps = 50 if batch == 1 else 5
        sess.set_step_timing(batch, True)
        for _ in range(reps):
            sess.run_device(x.data_ptr(), batch, None, stream)
        torch.cuda.synchronize()
        t = sess.step_times(batch)
        sess.set_step_timing(batch, False)
        i = next(j for j, (kd, _) in enumerate(summary) if kd.startswith("conv"))
        ms = t[i] / reps
        nbytes = (4 * 3 * 640 * 640 + (4 if prec == pb.FP32 else 2) * 16 * 320 * 320) * batch
        stem[name] = {"kernel": summary[i][0], "ms": round(ms, 5), "gbs": round(nbytes / ms / 1e6, 1),
                      "hbm_frac": round(nbytes / ms / 1e6 / hbm, 3)}
    res["configs[1]_stem_conv"] = {"bytes": "fp32 input read once + output written once", **stem}
    # ---- configs[4]
    B = 64
    g, info = build_yolov8("m", imgsz=640, seed=0)
    path = os.path.join(tempfile.mkdtemp(), "y8m.engine")
    write_engine(path, g)
    ctx = pb.Context(precision=pb.TF32, device=local)
    model = pb.Model(ctx, path)
    sess = pb.Session(ctx, model)
    x = torch.rand((B, 3, 640, 640), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    for _ in range(3):
        sess.run_device(x.data_ptr(), B, None, stream)
    torch.cuda.synchronize()
    summary = model.plan_summary(pb.TF32, B)
    steps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        sess.run_device(x.data_ptr(), B, None, stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    sess.set_step_timing(B, True)
    for _ in range(steps):
        sess.run_device(x.data_ptr(), B, None, stream)
    torch.cuda.synchronize()
    step_ms = sess.step_times(B)
    sess.set_step_timing(B, False)
    peak_tf32 = peak_sus / 2
    bound, meas = per_layer_roofline(summary, step_ms, steps, info, B, peak_tf32, hbm, 4)
    conv_ms = sum(step_ms[i] for i, (kd, _) in enumerate(summary) if kd.startswith("conv")) / steps
    flops = conv_flops(info) * B
    res["configs[4]_yolov8m_tf32_b64"] = {
        "images_per_s": round(B / ms * 1e3, 1), "ms_per_step": round(ms, 3), "conv_ms": round(conv_ms, 3),
        "conv_tflops": round(flops / conv_ms / 1e9, 1), "conv_frac_of_tf32_peak": round(flops / conv_ms / 1e9 / peak_tf32, 3),
        "conv_per_layer_roofline_frac": round(bound / meas, 3) if meas else None,
        "peak": f"{src} bf16 sustained / 2 = {peak_tf32:.1f} TFLOP/s", "step": "inference only (no decode)"}
    return res


def config(args, world):
    name = {"yolov8n": "configs[3]: YOLOv8n", "yolov8m": "configs[4]: YOLOv8m", "yolo11n": "YOLO11n"}[args.model]
    return {"workload": f"{name}-{args.imgsz} random-init, {args.precision.upper()} tcgen05 convs + GPU decode/NMS "
                        "(conf 0.25, IoU 0.45, max_det 300), independent replicas",
            "model": args.model, "imgsz": args.imgsz, "per_gpu_batch": args.batch, "global_batch": args.batch * world,
            "parallelism": f"replicas x{world}", "precision": args.precision,
            "l2": "inputs larger than L2 (1.26 GB per GPU)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--precision", default="bf16", choices=["bf16", "tf32", "fp32"])
    ap.add_argument("--model", default="yolov8n", choices=["yolov8n", "yolov8m", "yolo11n"],
                    help="yolov8n is the headline configuration")
    ap.add_argument("--e2e-steps", type=int, default=0, help="steps for the e2e leg (default: --steps)")
    ap.add_argument("--e2e-micro", type=int, default=256,
                    help="micro-batch of the e2e leg's pipelined batch runner (images per GPU launch)")
    ap.add_argument("--cpu-images", type=int, default=48, help="images in the bounded CPU baseline sample")
    ap.add_argument("--ref-images", type=int, default=4, help="images per step of the reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[0]/[1]/[4] records")
    ap.add_argument("--layers", action="store_true", help="print per-launch milliseconds to stderr")
    ap.add_argument("--layer", default="", help="CIN,COUT,K,S,HW: time one conv layer (Conv-BN-SiLU) instead")
    ap.add_argument("--sweep-layers", action="store_true", help="time every distinct YOLOv8n-640 conv shape")
    args = ap.parse_args()
    if args.layer or args.sweep_layers:
        run_layers(args)
        return
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import datetime
    import torch
    import torch.distributed as dist

    import pdefa_b200 as pb
    from pdefa_b200 import _native as N
    from pdefa_b200.engine_file import write_engine
    from pdefa_b200.replicas import job_throughput, reduce_job
    from pdefa_b200.yolo import conv_flops

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    L = N.lib()
    prec = {"bf16": pb.BF16, "tf32": pb.TF32, "fp32": pb.FP32}[args.precision]
    g, info = build_model(args.model, args.imgsz)
    tmp = tempfile.mkdtemp()
    path = os.path.join(tmp, args.model + ".engine")
    write_engine(path, g)
    ctx = pb.Context(precision=prec, device=local)
    model = pb.Model(ctx, path)
    sess = pb.Session(ctx, model)
    B = args.batch
    out_shape = sess.output_shape(B)
    ch, A = out_shape[1], out_shape[2]
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    x = torch.rand((B, 3, args.imgsz, args.imgsz), device="cuda", generator=gen)
    out_ptr = sess.device_output(B)          # decode reads the session's own output buffer
    max_det = 300
    counts = torch.empty(B, dtype=torch.int32, device="cuda")
    dets = torch.empty(B * max_det * 48, dtype=torch.uint8, device="cuda")
    wbytes = L.pdefa_decode_work_bytes(B, A)
    work = torch.empty(wbytes, dtype=torch.uint8, device="cuda")
    # An explicit (non-default) stream: every launch of the step, and the CUDA events
    # that time it, are ordered on this one stream.
    ts = torch.cuda.Stream()
    torch.cuda.set_stream(ts)
    stream = ts.cuda_stream

    def step():
        sess.run_device(x.data_ptr(), B, None, stream)
        pb.api._check(L.pdefa_decode_yolo_device(out_ptr, B, ch, A, None, 0.25, 0.45, max_det,
                                                 counts.data_ptr(), dets.data_ptr(), work.data_ptr(), wbytes,
                                                 stream), "decode")

    summary = model.plan_summary(prec, B)
    launches_per_step = len(summary) + 2          # + decode: candidate pass and per-image NMS
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sess.set_step_timing(B, True)

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = int(vis.split(",")[local]) if vis and vis.split(",")[local].strip().isdigit() else local
    sampler = ClockSampler(phys)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    step_ms = sess.step_times(B)
    sess.set_step_timing(B, False)
    if args.layers and rank == 0:
        for (k, name), v in zip(summary, step_ms):
            print(f"{v / args.steps:9.4f} ms  {k:14s} {name}", file=sys.stderr)
    # every rank processed B images per step; the job ends with the slowest rank
    ms_max, images = reduce_job(ms, B * args.steps, device=torch.device("cuda", local))
    value = job_throughput(images, ms_max)

    # roofline of the tensor-core conv family, measured inside the timed region
    hbm, peak_burst, peak_sus, peak_src = load_peaks()
    flops_img = conv_flops(info)
    tc_ms = sum(step_ms[i] for i, (k, _) in enumerate(summary) if k.startswith("conv_tc")) / args.steps
    conv_ms_all = sum(step_ms[i] for i, (k, _) in enumerate(summary) if k.startswith("conv")) / args.steps
    by_kind = {}
    for i, (k, _) in enumerate(summary):
        by_kind[k] = by_kind.get(k, 0.0) + step_ms[i] / args.steps
    # the stem (graph input, Cin 3) runs on its own kernel: excluded from the conv_tc family
    _, s_cin, s_cout, s_k, s_s, s_h, s_w = info["convs"][0]
    tc_flops = (flops_img - 2 * s_cin * s_cout * s_k * s_k * (s_h // s_s) * (s_w // s_s)) * B
    # TF32 tcgen05 runs at half the BF16 rate: its peak is half the measured BF16 figure
    peak_sus = peak_sus / 2 if args.precision == "tf32" else peak_sus
    abytes = 4 if args.precision != "bf16" else 2
    achieved = tc_flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else None
    # per-layer roofline: each conv's time bound is max(FLOPs / tensor peak, bytes /
    # HBM bandwidth), bytes = activations in (fp32 for the stem's graph input, bf16
    # otherwise) + out (bf16) once; the fraction is the sum of the bounds over the
    # sum of the measured conv times
    ideal_ms, meas_ms = per_layer_roofline(summary, step_ms, args.steps, info, B, peak_sus, hbm, abytes)
    yolov8n640 = args.imgsz == 640 and args.model == "yolov8n" and args.precision == "bf16"
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_sus, "unit": "TFLOP/s",
                "frac": (achieved / peak_sus) if achieved else None,
                "traffic": CONV_TC_DRAM_BYTES_PER_IMAGE_B32 * B / 62 if yolov8n640 else None,
                "traffic_unit": "DRAM bytes per conv_tc launch, averaged over the 62 launches of a step: "
                                "ncu capture of a batch-32 step scaled to this batch by images (a lower bound)",
                "kernel": f"conv_tc_{args.precision} ({sum(1 for k, _ in summary if k.startswith('conv_tc'))} launches/step)",
                "peak_source": f"{peak_src} bf16 sustained" + (" / 2 (tf32)" if args.precision == "tf32" else ""),
                "conv_tflops_all_convs": flops_img * B / (conv_ms_all / 1e3) / 1e12 if conv_ms_all else None,
                "conv_per_layer_roofline_frac": ideal_ms / meas_ms if meas_ms else None,
                "conv_per_layer_roofline_ms": {"bound": round(ideal_ms, 4), "measured": round(meas_ms, 4)},
                "ms_by_kernel_kind": {k: round(v, 4) for k, v in by_kind.items()},
                "decode_ms": ms_max / args.steps - sum(by_kind.values())}

    # e2e: pinned host images -> public batch API on this GPU -> host detections.
    # Headline: decoded 8-bit RGB frames (what a camera or an image decoder hands
    # over), letterboxed on the GPU (detect_u8); also the float32-tensor entry
    # (detect_arrays), whose copies are 4x larger. The runner pipelines micro-batches
    # of e2e_micro images: the copy of one onto the GPU overlaps the previous one's
    # inference.
    e2e_steps = args.e2e_steps or args.steps
    e2e_micro = max(1, min(B, args.e2e_micro))
    bi = pb.BatchInference(ctx, model, batch_size=e2e_micro, devices=[local], precision=prec)

    def timed(fn):
        fn()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            fn()
        ms, images = reduce_job((time.perf_counter() - t0) * 1e3, B * e2e_steps, device=torch.device("cuda", local))
        return job_throughput(images, ms)

    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    u8 = torch.empty((B, args.imgsz, args.imgsz, 3), dtype=torch.uint8, pin_memory=True)
    u8.copy_(torch.randint(0, 256, (B, args.imgsz, args.imgsz, 3), dtype=torch.uint8, device="cuda", generator=gen))
    u8np = u8.numpy()
    u8kw = dict(target_w=args.imgsz, target_h=args.imgsz, conf_thres=0.25, iou_thres=0.45, max_det=max_det)

    def pipelined():
        # a stream of steps through the pipelined public call: step k+1 is queued
        # before step k's detections are collected, so its frames cross PCIe while
        # step k's last micro-batches finish; every step's copies and detections are
        # inside the timed region (the last result() ends it)
        # warm-up: the runner's two lanes alternate across calls, so each lane meets
        # every micro-batch size of a step within two calls; their plans are built here
        for _ in range(3):
            bi.submit_u8(u8np, **u8kw).result()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        prev = None
        for _ in range(e2e_steps):
            cur = bi.submit_u8(u8np, **u8kw)
            if prev is not None:
                prev.result()
            prev = cur
        prev.result()
        ms, images = reduce_job((time.perf_counter() - t0) * 1e3, B * e2e_steps, device=torch.device("cuda", local))
        return job_throughput(images, ms)

    e2e_value = pipelined()
    e2e_sync_value = timed(lambda: bi.detect_u8(u8np, **u8kw))
    xh = torch.empty((B, 3, args.imgsz, args.imgsz), dtype=torch.float32, pin_memory=True)
    xh.copy_(x)
    xnp = xh.numpy()
    e2e_f32_value = timed(lambda: bi.detect_arrays(xnp, conf_thres=0.25, iou_thres=0.45, max_det=max_det))
    bi.close()

    # Host->device ceiling: every rank copies its pinned 8-bit frames to its GPU at the
    # same time (CUDA events around 5 copies), against the H2D rate the e2e leg needed
    dst = torch.empty(u8.shape, dtype=torch.uint8, device="cuda")
    dst.copy_(u8, non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    for _ in range(5):
        dst.copy_(u8, non_blocking=True)
    h1.record()
    torch.cuda.synchronize()
    h2d_ms = h0.elapsed_time(h1) / 5
    h2d_ms_max, h2d_bytes = reduce_job(h2d_ms, u8.numel(), device=torch.device("cuda", local))
    del dst
    h2d = {"ceiling_gbs_per_gpu": u8.numel() / h2d_ms / 1e6,
           "ceiling_gbs_total": h2d_bytes / h2d_ms_max / 1e6,
           "e2e_gbs_total": e2e_value * (u8.numel() / B) / 1e9,
           "how": "pinned 8-bit frames of one step copied to the GPU on all ranks at once, CUDA events"}

    configs = None
    if rank == 0 and world == 1 and not args.no_configs:
        configs = measure_configs(args, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        stepf = cpu_reference(args.cpu_images, threads, args.model)
        if stepf is not None:
            secs = stepf(args.cpu_images)
            cpu = {"value": args.cpu_images / secs, "unit": "images/s", "cores": threads, "kind": "reference",
                   "cpu": cpu_model(),
                   "sample": f"{args.cpu_images} images: reference engine (oracle/_ref) batch-1 Session.run "
                             f"+ restated reference decode/NMS (oracle/decode_ref.py, numpy argmax: a little "
                             f"faster than the reference's pure-Python decode, so the baseline is if anything "
                             f"overstated)"}

    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if prec == pb.BF16 else ("tf32" if prec == pb.TF32 else "f32"),
            "data": "synthetic (seeded uniform images, random-init weights)", "config": config(args, world),
            "clocks": clocks, "gpu_launches": launches_per_step * args.steps,
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": u8.numel(),
                    "d2h_bytes_per_step": B * 4 + B * max_det * 48, "micro_batch": e2e_micro,
                    "api": "BatchInference.submit_u8 + result() (pdefa_batch_submit_u8 / pdefa_batch_wait): "
                           f"pinned 8-bit RGB frames [{B}, {args.imgsz}, {args.imgsz}, 3] (already at the model "
                           "size: the scale-only letterbox is fused into the stem conv, which reads the 8-bit "
                           "pixels) + inference + decode, step k+1 queued before step k's detections are read",
                    "steps": e2e_steps, "warmup": 3,
                    "sync_value": e2e_sync_value,
                    "sync_api": "BatchInference.detect_u8 (pdefa_batch_run_u8), one blocking call per step",
                    "f32_input": {"value": e2e_f32_value, "h2d_bytes_per_step": xh.numel() * 4,
                                  "api": "BatchInference.detect_arrays (pdefa_batch_run), pinned float32 NCHW"},
                    "h2d": h2d},
            "roofline": roofline, "cpu_baseline": cpu,
            "conv_gflop_per_image": flops_img / 1e9,
            "configs": configs,
        }))


if __name__ == "__main__":
    main()
