"""Throughput of the fused conv/GEMM hot path on B200: images/s of the text-detection backbone
(the C2 det model, N=256 images of 3x640x640 per GPU), batch-sharded replicas.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...   (N > 1)

One step = one pass of the whole plan over one batch of synthetic input (see simdonnx_b200/configs.py).
`value` is device-resident throughput (input already in HBM, CUDA events on the session stream,
max over ranks); `e2e` is the same metric through the session's C-ABI run call with pinned host
buffers (H2D of the fp32 input and D2H of the fp32 output inside every step). Each rank prints
nothing but rank 0, which prints one JSON line.

--impl reference times the reference's own CPU algorithm (the C++ restatement of SimdOnnx's NHWC
CPU kernels under oracle/, since the C# reference cannot run here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "images/sec per B200 at 1/2/4/8 GPUs; % of fp16 tensor / HBM roofline"
HW = 640


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi clock / throttle sampling during the timed region (every 25 ms: the default timed
    region is about 0.2 s)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "25"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None}


def cpu_baseline(batch_hw: int, seconds: float = 12.0, max_images: int = 2000) -> dict:
    """The reference's CPU algorithm (oracle restatement) on all host threads, bounded sample."""
    import numpy as np

    import oracle
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs

    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    plan = configs.build_det(batch=1, hw=batch_hw)
    sess = OracleSession(plan)
    feeds = {k: f() for k, f in plan.feeds.items()}
    sess.run(feeds)  # warm-up (packs weights)
    n, t0 = 0, time.perf_counter()
    while True:
        sess.run(feeds)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= max_images:
            break
    return {"value": n / el, "unit": "images/s", "cores": threads, "kind": "port",
            "sample": f"{n} single-image runs of the C2 det model at {batch_hw}x{batch_hw} (batch 1) in {el:.1f} s; "
                      "restated reference CPU kernels (oracle/), not the reference binary"}


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    import oracle
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs

    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    per_step = max(1, args.ref_images)
    plan = configs.build_det(batch=per_step, hw=HW)
    sess = OracleSession(plan)
    feeds = {k: f() for k, f in plan.feeds.items()}
    for _ in range(args.warmup):
        sess.run(feeds)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sess.run(feeds)
    el = time.perf_counter() - t0
    v = per_step * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C5/C2 text-detection backbone (det), 3x640x640 fp32 input",
                   "images_per_step": per_step, "parallelism": "host threads"},
        "cpu_baseline": {"value": v, "unit": "images/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} image(s) per step; restated reference CPU kernels (oracle/)"},
        "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def node_times(sess, N, roofline, torch, passes: int = 3):
    """Per-node device times of a session: `passes` eager runs of its node list on the session
    stream with a CUDA event between nodes; the median per node. Returns (rows, launches per pass)."""
    n_nodes = sess.node_count()
    stream = sess.stream
    samples = [[] for _ in range(n_nodes)]
    launches = 0
    for _ in range(passes):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_nodes + 1)]
        before = int(N.lib().sdx_launch_count())
        with torch.cuda.stream(stream):
            evs[0].record(stream)
            for i in range(n_nodes):
                N.call("sdx_session_enqueue_node", sess.h, i)
                evs[i + 1].record(stream)
        evs[-1].synchronize()
        launches = int(N.lib().sdx_launch_count()) - before
        for i in range(n_nodes):
            samples[i].append(evs[i].elapsed_time(evs[i + 1]))
    rows = []
    for i, node in enumerate(sess.plan.nodes):
        cls, fl, by = roofline.node_cost(sess.plan, node)
        t = statistics.median(samples[i])
        rows.append({"node": node.name, "op": node.op, "kernel": cls, "ms": t, "bytes": by, "flops": fl,
                     "gbs": by / t / 1e6 if t > 0 else None, "tflops": fl / t / 1e9 if t > 0 else None,
                     "out": list(sess.plan.values[node.outs[0]].shape)})
    return rows, launches


def measure_extras(args, local, N, configs, roofline, torch, CudaInferenceSession) -> dict:
    """Side measurements on this GPU (not the headline): the tensor-bound half of the hot path
    (C4 UNet at N=16: images/s and, per 3x3 conv, TFLOP/s against the sustained bf16 peak), the
    single fused node C1 (N=8) and C3 rec at N=64, with fp32 logits and with the fused CTC head
    (per-step index and probability; the [N*40, 6625] logits never stored). Device-resident, CUDA
    events, K graph replays."""
    dev = torch.device("cuda", local)
    tc_peak = peaks_sustained()
    hbm, _, _ = peaks()
    out = {}
    for key, build, batch in (("unet_c4", configs.build_unet, 16), ("c1", configs.build_c1, 8),
                              ("rec_c3", configs.build_rec, 64),
                              ("rec_c3_ctc_head", lambda batch: configs.build_rec(batch=batch, ctc=True), 64)):
        plan = build(batch=batch)
        s = CudaInferenceSession(plan, device=local)
        if plan.feeds_dev:
            s.write_inputs({k: f(dev) for k, f in plan.feeds_dev.items()})
        else:
            s.write_inputs({k: f() for k, f in plan.feeds.items()})
        for _ in range(args.warmup):
            s.enqueue()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s.stream)
        for _ in range(args.steps):
            s.enqueue()
        e1.record(s.stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        rows, _ = node_times(s, N, roofline, torch)
        tot = roofline.plan_totals(s.plan)
        rec = {"batch": batch, "ms_per_step": ms, "images_per_s": batch / (ms / 1e3),
               "whole_step_tflops": tot["flops"] / ms / 1e9, "whole_step_gbs": tot["bytes"] / ms / 1e6}
        if key == "unet_c4":
            convs = [r for r in rows if r["op"] == "Conv" and r["kernel"] == "conv_tc"]
            tc_ms = sum(r["ms"] for r in convs)
            tc_fl = sum(r["flops"] for r in convs)
            rec["conv3x3_tc"] = {"launches": len(convs), "ms": tc_ms, "tflops": tc_fl / tc_ms / 1e9,
                                 "frac_of_sustained_bf16": tc_fl / tc_ms / 1e9 / tc_peak,
                                 "peak_tflops_sustained": tc_peak}
            # the ones above the ridge (FLOPs per byte > bf16 peak / HBM peak): the tensor-bound set
            ridge = tc_peak * 1e12 / (hbm * 1e9)
            tb = [r for r in convs if r["flops"] > ridge * r["bytes"]]
            tb_ms, tb_fl = sum(r["ms"] for r in tb), sum(r["flops"] for r in tb)
            if tb_ms > 0:
                rec["conv3x3_tensor_bound"] = {"launches": len(tb), "ms": tb_ms, "tflops": tb_fl / tb_ms / 1e9,
                                               "frac_of_sustained_bf16": tb_fl / tb_ms / 1e9 / tc_peak,
                                               "ridge_flop_per_byte": ridge}
            rec["per_conv"] = [{"node": r["node"], "out": r["out"], "ms": round(r["ms"], 4),
                                "tflops": round(r["tflops"], 1),
                                "frac_of_sustained_bf16": round(r["tflops"] / tc_peak, 3)} for r in convs]
        else:
            rec["node_ms_sum"] = sum(r["ms"] for r in rows)
            rec["gbs"] = tot["bytes"] / ms / 1e6
            rec["hbm_frac"] = tot["bytes"] / ms / 1e6 / hbm
        out[key] = rec
        s.close()
    return out


# DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) per launch of a kernel class of the
# det step, from one ncu capture of the session's eager pass at 64 images per GPU (every launch of the
# class averaged), scaled by 4 to the benchmark's 256 images (per-launch work is linear in images).
TRAFFIC_PER_LAUNCH = {"conv_tc_rows": 691.4e6}


def peaks_sustained() -> float:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d.get("bf16_tflops_sustained", d["bf16_tflops"])
    return 1400.0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=256, help="images per GPU per step")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-images", type=int, default=1, help="reference arm: images per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--node-times", default="", help="write per-node timings (JSON) to this path")
    ap.add_argument("--repeats", type=int, default=5, help="extra K-step timed regions (spread only)")
    ap.add_argument("--no-extras", action="store_true", help="skip the UNet / C1 / rec side measurements")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import ctypes
    from datetime import timedelta

    import numpy as np
    import torch
    import torch.distributed as dist

    from simdonnx_b200 import _native as N, configs, roofline
    from simdonnx_b200.session import CudaInferenceSession

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))

    plan = configs.build_det(batch=args.batch, hw=HW)
    dev = torch.device("cuda", local)
    # the seeded SplitMix64 input made on the device (bit-identical to synth.uniform, seconds not minutes)
    feeds_dev = {k: f(dev) for k, f in plan.feeds_dev.items()}
    sess = CudaInferenceSession(plan, device=local)
    sess.write_inputs(feeds_dev)
    stream = sess.stream
    launches0 = int(N.lib().sdx_launch_count())

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    # ---- device-resident throughput
    for _ in range(args.warmup):
        sess.enqueue()
    barrier()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        sess.enqueue()
    e1.record(stream)
    e1.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    images = args.batch * world * args.steps
    value = images / (ms / 1e3)

    # ---- repeats of the same K-step region (spread of the device-resident figure inside this run)
    rep_ms = []
    for _ in range(args.repeats):
        barrier()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for _ in range(args.steps):
            sess.enqueue()
        r1.record(stream)
        r1.synchronize()
        t = r0.elapsed_time(r1)
        if world > 1:
            tt = torch.tensor([t], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        rep_ms.append(t)
    repeats = None
    if rep_ms:
        rv = sorted(images / (t / 1e3) for t in rep_ms)
        repeats = {"n": len(rv), "steps_each": args.steps, "images_per_s_min": rv[0],
                   "images_per_s_median": statistics.median(rv), "images_per_s_max": rv[-1]}

    # ---- per-node timing passes (eager, same stream): kernel classes and the dominant one
    per_node, launches_per_step = node_times(sess, N, roofline, torch)
    classes = {}
    for r in per_node:
        c = classes.setdefault(r["kernel"], {"ms": 0.0, "flops": 0, "bytes": 0, "launches": 0})
        c["ms"] += r["ms"]
        c["flops"] += r["flops"]
        c["bytes"] += r["bytes"]
        c["launches"] += 1
    if args.node_times and rank == 0:
        with open(args.node_times, "w") as f:
            json.dump(per_node, f, indent=1)
    dom = max(classes, key=lambda k: classes[k]["ms"])
    dc = classes[dom]
    hbm, tflops, src = peaks()
    ridge = tflops * 1e12 / (hbm * 1e9)
    tensor_bound = dc["flops"] > ridge * dc["bytes"]
    if tensor_bound:
        achieved = dc["flops"] / (dc["ms"] / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops}
    else:
        achieved = dc["bytes"] / (dc["ms"] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm}
    roof.update({"kernel": dom, "launches_per_step": dc["launches"], "ms_per_step": dc["ms"],
                 "algorithmic_bytes_per_step": dc["bytes"], "algorithmic_flops_per_step": dc["flops"],
                 "peak_source": src, "traffic": TRAFFIC_PER_LAUNCH.get(dom) if args.batch == 256 else None,
                 "traffic_unit": "bytes per launch",
                 "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, det eager pass at 64 images, "
                                   "class average per launch x4",
                 "timing": "per-node CUDA events on the session stream, eager pass after the timed region"})
    tot = roofline.plan_totals(sess.plan)
    step_s = ms / 1e3 / args.steps
    extras = None
    if world == 1 and not args.no_extras:
        extras = measure_extras(args, local, N, configs, roofline, torch, CudaInferenceSession)
    whole = {"algorithmic_bytes_per_step": tot["bytes"], "algorithmic_flops_per_step": tot["flops"],
             "hbm_gbs": tot["bytes"] / step_s / 1e9, "hbm_frac": tot["bytes"] / step_s / 1e9 / hbm}

    # ---- end to end through the C-ABI run call (pinned host I/O inside each step)
    def e2e_measure(es, efeeds):
        """(pipelined, serial) seconds for K steps through the C ABI with pinned host buffers."""
        es.stage_inputs(efeeds)
        pin_in, pin_out = es.pinned_io()
        pairs = [(pin_in, pin_out), (pin_in.clone().pin_memory(), torch.empty_like(pin_out).pin_memory())]
        es.submit(*pairs[0])
        es.wait(120000)
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            es.submit(*pairs[i % 2])
        es.wait(120000)
        el = time.perf_counter() - t0
        barrier()
        t1 = time.perf_counter()
        for _ in range(args.steps):
            es.run(timeout_ms=120000, copy=False)
        el_serial = time.perf_counter() - t1
        barrier()
        if world > 1:
            t = torch.tensor([el, el_serial], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el, el_serial = float(t[0].item()), float(t[1].item())
        return el, el_serial

    e2e = None
    if not args.no_e2e:
        # (1) fp32 tensor input (the plan measured above)
        feeds = {k: t.cpu().numpy() for k, t in feeds_dev.items()}
        el_t, el_ts = e2e_measure(sess, feeds)
        tensor_e2e = {"value": images / el_t, "unit": "images/s", "h2d_bytes_per_step": sess.in_bytes,
                      "d2h_bytes_per_step": sess.out_bytes, "serial_value": images / el_ts}
        sess_bytes = (sess.in_bytes, sess.out_bytes)
        sess.close()
        # (2) image-session input: u8 RGB pixels, normalized on the device (sdx_image_to_tensor)
        iplan = configs.build_det(batch=args.batch, hw=HW, image_input=True)
        ifeeds = {k: f(dev).cpu().numpy() for k, f in iplan.feeds_dev.items()}
        isess = CudaInferenceSession(iplan, device=local)
        el_i, el_is = e2e_measure(isess, ifeeds)
        e2e = {"value": images / el_i, "unit": "images/s", "h2d_bytes_per_step": isess.in_bytes,
               "d2h_bytes_per_step": isess.out_bytes, "input": "u8 RGB images [N,640,640,3], normalized on the device",
               "timing": "host wall clock from the first of K pipelined sdx_session_submit calls (pinned host "
                         "buffers: H2D of the step's images, D2H of its fp32 probability map) to "
                         "sdx_session_wait, max over ranks",
               "serial_value": images / el_is,
               "serial_timing": "host wall clock around K synchronous sdx_session_run calls"}
        isess.close()
        del sess_bytes

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(HW)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "C5: C2 text-detection backbone, 3x640x640 fp32 input, per-GPU batch",
                       "per_gpu_batch": args.batch, "global_batch": args.batch * world, "image": [3, HW, HW],
                       "parallelism": f"replicas x{world} (batch-sharded, no collective)",
                       "l2": "inputs larger than L2 (fp32 input 1.26 GB per GPU per step)"},
            "roofline": roof, "whole_step": whole,
            "kernel_classes": {k: {"ms": round(v["ms"], 4), "launches": v["launches"]} for k, v in
                               sorted(classes.items(), key=lambda kv: -kv[1]["ms"])},
            "cpu_baseline": cpu, "e2e": e2e, "e2e_fp32_input": tensor_e2e if e2e else None,
            "repeats": repeats, "extras": extras, "gpu_launches": launches_per_step * args.steps,
            "launches_per_step": launches_per_step, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if args.no_e2e:
        sess.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    del launches0


if __name__ == "__main__":
    main()
