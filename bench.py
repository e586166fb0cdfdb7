"""Benchmark: YOLOv8n-architecture fp32 640x640 inference images/s on B200.

One step = one prepared YOLOv8n forward over a batch of 64 synthetic
640x640 images per GPU (weak scaling: every rank runs a whole-model replica
on its own batch slice).  ``value`` is measured with inputs resident in HBM;
``e2e`` repeats the same metric through the public API from pinned host
buffers (upload, forward, ``.cpu()`` of the [B, 84, 8400] result).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun every rank runs; timing is on the device (CUDA events on the
runtime stream) with a barrier + synchronize on both sides, max over ranks.
``--impl reference`` times the reference's ground-truth implementation of the
path (stock PyTorch CPU fp32 running the same unprepared model) on the host
cores of rank 0.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "YOLOv8n 640x640 fp32 images/sec"
UNIT = "images/s"
BATCH = 64
IMAGE = 640
NC = 80
ANCHORS = (IMAGE // 8) ** 2 + (IMAGE // 16) ** 2 + (IMAGE // 32) ** 2


class Spec:
    """One benchmark configuration: model, seeded synthetic input, batch per
    GPU (weak scaling) or in total (strong scaling), and the CPU sample the
    ground-truth timing runs on."""

    def __init__(self, key, metric, unit, model, inputs, batch, scaling, desc, cpu_sample):
        self.key, self.metric, self.unit = key, metric, unit
        self.model, self.inputs = model, inputs
        self.batch, self.scaling, self.desc, self.cpu_sample = batch, scaling, desc, cpu_sample

    def batch_per_gpu(self, world: int, override=None) -> int:
        b = int(override) if override else self.batch
        if self.scaling == "strong":
            if b % world:
                raise SystemExit(f"bench: total batch {b} does not split over {world} GPUs")
            return b // world
        return b


def _specs():
    import workloads as W
    return {
        "y8n": Spec("y8n", METRIC, UNIT, lambda: W.yolov8_model("n"),
                    lambda b, s: W.yolo_input(b, seed=s), BATCH, "weak",
                    "yolov8n 640x640 fp32 inference", 8),
        "y8n1": Spec("y8n1", METRIC, UNIT, lambda: W.yolov8_model("n"),
                     lambda b, s: W.yolo_input(b, seed=s), 1, "weak",
                     "yolov8n 640x640 fp32 inference", 4),
        "y8m": Spec("y8m", "YOLOv8m 640x640 fp32 images/sec", UNIT, lambda: W.yolov8_model("m"),
                    lambda b, s: W.yolo_input(b, seed=s), 256, "strong",
                    "yolov8m 640x640 fp32 inference, a batch of 256 split over the GPUs", 2),
        "r18": Spec("r18", "ResNet-18 224x224 fp32 images/sec", UNIT, W.resnet18_model,
                    lambda b, s: W.resnet18_input(b, seed=s), 32, "weak",
                    "resnet18 224x224 fp32 eval inference (softmax head)", 16),
        "mlp": Spec("mlp", "MLP 784-512-256-10 fp32 samples/sec", "samples/s", W.mlp_model,
                    lambda b, s: W.mlp_input(b, seed=s), 256, "weak",
                    "MLP 784-512-256-10 (ReLU) + softmax fp32", 256),
    }


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--workload", choices=("y8n", "y8n1", "y8m", "r18", "mlp", "c1"), default="y8n",
                   help="y8n: YOLOv8n bs64 (the headline); y8n1: YOLOv8n bs1; y8m: YOLOv8m, 256 "
                        "images split over the GPUs; r18: ResNet-18 bs32; mlp: MLP bs256; "
                        "c1: the single [1,4,320,320] x [5,4,3,3] convolution")
    p.add_argument("--batch", type=int, default=None, help="batch per GPU (total for y8m)")
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--e2e-chunks", type=int, default=4,
                   help="1 GPU: matrixman.infer chunks (upload / forward / readback overlap)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true",
                   help="skip the output check against the CPU ground truth after the timed region")
    p.add_argument("--profile-case", action="store_true",
                   help="run --steps eager forwards (no graphs, no timing) for an ncu capture")
    p.add_argument("--profile-conv", default=None, metavar="C,K,KSIZE,STRIDE,HW",
                   help="run one prepared convolution (SiLU epilogue) on a --batch x C x HW x HW "
                        "input (NCHW for C <= 3, NHWC otherwise) --steps + 1 times, for an ncu "
                        "capture of one kernel")
    p.add_argument("--conv-sweep", action="store_true",
                   help="time the tensor-core convolution alone on the YOLOv8n/m 3x3 layer shapes "
                        "at --batch (default 64): one JSON line per layer with TF/s and the fraction "
                        "of the 3xTF32 ceiling")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="mm_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        sm = []
        for r in rows:
            try:
                sm.append(float(r[1]))
            except ValueError:
                pass
            for name, flag in zip(names, r[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        smax = None
        try:
            smax = float(rows[0][2])
        except ValueError:
            pass
        load = [s for s in sm if smax and s > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(rows)}


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profile_launches(matrixman, prepared, x_dev) -> dict:
    """One eager forward with CUDA events around every native launch."""
    from matrixman_b200 import telemetry as profiling
    cfg = matrixman.config
    old_graphs, old_timing = cfg.cudaGraphs, cfg.gpuTiming
    cfg.cuda_graphs = False
    cfg.gpu_timing = True
    profiling.launch_times.records.clear()
    try:
        import torch
        with torch.no_grad():
            prepared(x_dev)
        summary = profiling.launch_times.summary()
    finally:
        cfg.cuda_graphs = old_graphs
        cfg.gpu_timing = old_timing
    return summary


def cpu_baseline(model, batch_sample: int, spec=None, min_seconds: float = 12.0) -> dict:
    """Stock PyTorch CPU fp32 on this host's cores (the reference's ground truth)."""
    import torch
    from oracle.models import cpu_model_name
    spec = spec or _specs()["y8n"]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = spec.inputs(batch_sample, 99)
    with torch.no_grad():
        model(x)  # warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            model(x)
            n += 1
            el = time.perf_counter() - t0
            if el >= min_seconds or n >= 200:
                break
    return {"value": n * batch_sample / el, "unit": spec.unit, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} forwards of the unprepared model ({spec.desc}) at batch {batch_sample} "
                      f"on torch CPU fp32 ({cpu_model_name()}, {threads} threads), {el:.1f} s"}


def output_parity(model, out_cpu, batch: int, world: int, images: int = 2, spec=None) -> dict:
    """Checker (outside every timed region): the first `images` images of each
    rank's slice of the timed step's output against the CPU ground truth (the
    unprepared model on torch CPU fp32, the same computation the CPU baseline
    times), as max |diff| / max |ref| -- the parity bar is 1e-4."""
    from oracle.models import run_cpu
    from oracle.tolerance import CONV_GEMM_REL, max_rel_err
    spec = spec or _specs()["y8n"]
    worst = 0.0
    images = min(images, batch)
    for r in range(world):
        x = spec.inputs(batch, 1000 + r)[:images]
        ref = run_cpu(model, x)
        got = out_cpu[r * batch:r * batch + images]
        worst = max(worst, max_rel_err(got, ref))
        del x
    return {"max_rel_err": worst, "bar": CONV_GEMM_REL, "ok": bool(worst < CONV_GEMM_REL),
            "images_checked": images * world,
            "what": f"first {images} images of each rank's slice of the last timed step's output"
                    + (" (gathered on rank 0)" if world > 1 else "")
                    + " vs the unprepared model on torch CPU fp32"}


def run_b200(args, spec):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        # The process group is created before the package registers its
        # PrivateUse1 device, so torch's accelerator check sees CUDA.
        from datetime import timedelta
        torch.cuda.set_device(local)
        # NCCL's version banner goes to stdout; keep rank 0's stdout to the one
        # JSON line unless the caller asked for NCCL logging.
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    import matrixman_b200 as matrixman
    import workloads as W
    from matrixman_b200 import runtime
    from matrixman_b200 import telemetry as profiling
    from matrixman_b200.replicas import PeerGather

    runtime.set_device(local)
    matrixman.init()
    rt = runtime.get_runtime(local)
    batch = spec.batch_per_gpu(world, args.batch)
    model = spec.model()
    prepared = matrixman.prepare(model)
    x_host = spec.inputs(batch, 1000 + rank)
    x_dev = matrixman.to_device(x_host, device=local)
    with torch.no_grad():
        out_tail = tuple(int(v) for v in prepared(x_dev).shape[1:])

    def barrier():
        # an all-reduce of an explicit CUDA tensor (dist.barrier would place its
        # tensor on the default accelerator, which is the matrixman device)
        if world > 1:
            t = torch.zeros(1, device=torch.device("cuda", local))
            dist.all_reduce(t)
            torch.cuda.synchronize(local)
        rt.synchronize()

    sizes = [batch] * world
    gather = None
    if world > 1:
        # Rank 0's gather buffers, written by every rank's copy engines over
        # NVLink (CUDA IPC); the copies of one step overlap the next forward.
        gather = PeerGather(out_tail, sizes, device=local)

    def step(xd):
        """One step: the replica's forward; with several ranks, plus the
        copy of this rank's output (e.g. [B, 84, 8400]) into rank 0's gather
        buffer."""
        y = prepared(xd)
        if gather is not None:
            gather.push(y)
        return y

    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):
            y = step(x_dev)
        del y
        barrier()
        clocks = ClockSampler(local)
        clocks.start()
        # untimed pre-roll so the clock sampler is up before the timed region
        t_pre = time.perf_counter()
        while time.perf_counter() - t_pre < 0.4:
            y = step(x_dev)
            rt.synchronize()
        timer = runtime.Timer(rt)
        launches0 = profiling.total_launches()
        barrier()
        timer.start()
        for _ in range(args.steps):
            y = step(x_dev)
        if gather is not None:
            gather.join(rt.stream)  # the last step's copy ends the timed region
        timer.stop()
        ms_total = timer.elapsed_ms()
        launch_calls = profiling.total_launches() - launches0
        barrier()
        clock_info = clocks.stop()
        # The last timed step's (gathered) output; its parity is checked on
        # rank 0 after the end-to-end timing (the CPU oracle's threads would
        # compete with the host thread that feeds the device).
        full = gather.collect() if gather is not None else y
        del y
    ms_step = ms_total / args.steps
    if world > 1:
        t = torch.tensor([ms_step], device=torch.device("cuda", local))
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())
    value = world * batch / (ms_step / 1e3)

    # End to end: pinned host input -> public API -> CPU result.  Each rank
    # runs the public batch API on its own slice, and its results land in its
    # own host memory (data-parallel serving: no cross-GPU traffic at all).
    # Every step's batch goes through the streaming API (matrixman.infer_stream):
    # its upload, forward and readback are all inside the timed region, and
    # they overlap those of the neighbouring steps.  One call of the batch API
    # (matrixman.infer, which overlaps chunks of a single batch) is timed too.
    e2e_steps = args.e2e_steps or max(10, min(args.steps, 30))
    x_pinned = matrixman.pinned_empty(x_host.shape)
    x_pinned.copy_(x_host)

    with torch.no_grad():
        # warm-up long enough to leave the readback pool holding every block a
        # stream of this depth keeps in flight
        for out in matrixman.infer_stream(prepared, [x_pinned] * 6, device=local):
            pass
        barrier()
        t0 = time.perf_counter()
        for out in matrixman.infer_stream(prepared, [x_pinned] * e2e_steps, device=local):
            pass
        barrier()
        e2e_s = (time.perf_counter() - t0) / e2e_steps
        for _ in range(2):
            matrixman.infer(prepared, x_pinned, chunks=args.e2e_chunks, device=local)
        barrier()
        t0 = time.perf_counter()
        for _ in range(3):
            matrixman.infer(prepared, x_pinned, chunks=args.e2e_chunks, device=local)
        barrier()
        single_s = (time.perf_counter() - t0) / 3
    if world > 1:
        t = torch.tensor([e2e_s], device=torch.device("cuda", local))
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    checked = full.cpu() if (rank == 0 and full is not None and not args.no_parity) else None
    del full
    parity = output_parity(model, checked, batch, world, spec=spec) if checked is not None else None
    out_numel = batch * world
    for v in out_tail:
        out_numel *= v
    e2e = {"value": world * batch / e2e_s, "unit": spec.unit,
           "h2d_bytes_per_step": int(x_host.numel() * 4) * world,
           "d2h_bytes_per_step": int(out_numel * 4), "ms_per_step": e2e_s * 1e3, "steps": e2e_steps,
           "api": f"matrixman.infer_stream(prepared, {e2e_steps} pinned batches of {batch})"
                  + (" on every rank, results in each rank's host memory" if world > 1 else ""),
           "single_call": {"value": world * batch / single_s, "ms": single_s * 1e3,
                           "api": f"matrixman.infer(prepared, pinned batch, chunks={args.e2e_chunks})"}}
    return {"world": world, "rank": rank, "local": local, "value": value, "ms_step": ms_step,
            "clocks": clock_info, "e2e": e2e, "launch_calls": launch_calls, "prepared": prepared,
            "x_dev": x_dev, "model": model, "macs": W.macs_per_sample(model, x_host[:1]), "batch": batch,
            "parity": parity, "gather": gather,
            "matrixman": matrixman, "dist": dist if world > 1 else None}


CONV_ENTRIES = ("mm_conv2d", "mm_conv2d_region", "mm_conv2d_tc", "mm_conv2d_tc_region", "mm_gemm")
TRAFFIC_SUMMARY = ROOT / "profiles" / "conv_tc_c64_80x80_bs128.md"


def conv_traffic_per_launch():
    """DRAM bytes (read + write) of one launch of the tensor-core convolution
    from the committed one-launch ncu capture of a representative YOLOv8n
    layer (lines ``bytes_per_launch:``, ``algorithmic_bytes_per_launch:`` and
    ``layer:``), or None."""
    if not TRAFFIC_SUMMARY.exists():
        return None
    fields = {}
    for line in TRAFFIC_SUMMARY.read_text().splitlines():
        key, sep, val = line.partition(":")
        if sep and key.strip() in ("bytes_per_launch", "algorithmic_bytes_per_launch", "layer"):
            fields[key.strip()] = val.strip()
    try:
        return {"bytes_per_launch": int(float(fields["bytes_per_launch"])),
                "algorithmic_bytes_per_launch": int(float(fields["algorithmic_bytes_per_launch"])),
                "layer": fields.get("layer", ""),
                "source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, "
                          f"{TRAFFIC_SUMMARY.relative_to(ROOT)}"}
    except (KeyError, ValueError):
        return None


def roofline(res: dict, spec=None) -> tuple[dict, int, dict]:
    """Dominant kernel family (convolution) from one event-timed eager forward.

    achieved = algorithmic conv FLOPs of one forward (2 * MACs * batch) / the
    summed device time of the conv launches.  The tensor roofline of the
    3xTF32 split is one third of the dense TF32 rate, which is half of the
    measured dense bf16 rate.
    """
    peaks = measured_peaks()
    summary = profile_launches(res["matrixman"], res["prepared"], res["x_dev"])
    total_ms = sum(v["ms"] for v in summary.values()) or 1e-9
    conv_ms = sum(summary[k]["ms"] for k in CONV_ENTRIES if k in summary)
    conv_launches = sum(summary[k]["launches"] for k in CONV_ENTRIES if k in summary)
    flops = 2.0 * res["macs"] * res["batch"]
    achieved = flops / (conv_ms / 1e3) / 1e12 if conv_ms > 0 else 0.0
    # The conv kernels run back to back inside a long step: the sustained
    # (power-capped) dense bf16 figure is the denominator.  fp32-accurate
    # 3xTF32 issues three tf32 products (tf32 runs at half the bf16 rate) per
    # algorithmic multiply-add, so its own ceiling is one sixth of that.
    peak = peaks["bf16_tflops_sustained"]
    ceiling = peak / 6.0
    kernels_per_forward = sum(v["launches"] for v in summary.values())
    # (the committed DRAM-traffic capture is one launch of a YOLOv8n layer; the
    # kernel moves its algorithmic bytes about once, so traffic ~ algorithmic)
    traffic = conv_traffic_per_launch() if spec is None or spec.key == "y8n" else None
    roof = {"bound": "tensor", "kernel": "+".join(k for k in CONV_ENTRIES if k in summary),
            "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4) if peak else None,
            "traffic": traffic["bytes_per_launch"] if traffic else None,
            "peak_basis": f"{peaks['source']} dense bf16, sustained ({peaks['bf16_tflops_sustained']} "
                          f"TF/s; burst {peaks['bf16_tflops']})",
            "ceiling_3xtf32": round(ceiling, 1), "frac_of_3xtf32_ceiling": round(achieved / ceiling, 4),
            "tensor_issue_equiv_tflops": round(achieved * 6.0, 1),
            "launches_per_forward": conv_launches, "share_of_forward": round(conv_ms / total_ms, 3),
            "forward_ms_eager_events": round(total_ms, 3)}
    if traffic:
        roof["traffic_source"] = traffic["source"]
        roof["traffic_layer"] = traffic["layer"]
        roof["traffic_algorithmic_bytes"] = traffic["algorithmic_bytes_per_launch"]
    shares = {k: {"launches": v["launches"], "ms": round(v["ms"], 4), "share": round(v["ms"] / total_ms, 4)}
              for k, v in sorted(summary.items(), key=lambda kv: -kv[1]["ms"])}
    return roof, kernels_per_forward, shares


def main():
    args = parse_args()
    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, world, rank)
    if args.profile_case:
        return run_profile_case(args)
    if args.profile_conv:
        return run_profile_conv(args)
    if args.conv_sweep:
        return run_conv_sweep(args)
    if args.workload == "c1":
        return run_c1(args)
    spec = _specs()[args.workload]
    res = run_b200(args, spec)
    roof, kernels_per_forward, shares = roofline(res, spec)
    in_bytes = res["batch"] * res["x_dev"].numel() // max(int(res["x_dev"].shape[0]), 1) * 4
    line = {
        "metric": spec.metric, "value": round(res["value"], 2), "unit": spec.unit, "n_gpus": res["world"],
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(res["ms_step"], 4),
        "higher_is_better": True, "scaling": spec.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic seeded inputs (shapes and distributions of the configuration), "
                "random-init weights (seeded)",
        "config": {"workload": f"{spec.desc}, {res['batch']} per GPU, "
                               "prepared (BN folded, NHWC, CUDA graph)"
                               + (", every step's outputs gathered in rank 0's HBM by copy-engine "
                                  "writes over NVLink (CUDA IPC), overlapped with the next forward"
                                  if res["world"] > 1 else ""),
                   "batch_per_gpu": res["batch"], "global_batch": res["batch"] * res["world"],
                   "parallelism": f"replicas{res['world']}",
                   "l2": (f"inputs larger than L2 ({in_bytes / 1e6:.0f} MB input per step per GPU)"
                          if in_bytes > 126e6 else
                          f"{in_bytes / 1e6:.1f} MB input per step, L2-resident (latency-bound config)")},
        "e2e": res["e2e"], "roofline": roof, "parity": res["parity"],
        "gpu_launches": kernels_per_forward * args.steps, "clocks": res["clocks"],
        "kernel_shares": shares,
    }
    if spec.key in ("y8n", "y8n1", "y8m"):
        line["config"]["image"] = [IMAGE, IMAGE]
    if res["world"] == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(res["model"], min(spec.cpu_sample, res["batch"] * 64), spec)
    if res["dist"] is not None:
        import torch
        if res["gather"] is not None:
            res["gather"].close()
        t = torch.zeros(1, device=torch.device("cuda", res["local"]))
        res["dist"].all_reduce(t)
        torch.cuda.synchronize(res["local"])
        res["dist"].destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_profile_case(args):
    """Eager prepared forwards (no CUDA graph, no timing) for ncu launch lists:
    one warm-up forward, then --steps forwards."""
    import torch

    import matrixman_b200 as matrixman
    import workloads as W
    matrixman.init()
    matrixman.config.cuda_graphs = False
    prepared = matrixman.prepare(W.yolov8_model("n"))
    x = matrixman.to_device(W.yolo_input(args.batch, seed=1000))
    with torch.no_grad():
        prepared(x)
        for _ in range(args.steps):
            prepared(x)
    matrixman.synchronize()
    print(json.dumps({"profile_case": "yolov8n", "batch": args.batch, "forwards": args.steps + 1}))


def run_profile_conv(args):
    import torch
    from torch import nn

    import matrixman_b200 as matrixman
    from matrixman_b200.preparation import PreparedConv2d
    c, k, ks, st, hw = (int(v) for v in args.profile_conv.split(","))
    matrixman.init()
    g = torch.Generator().manual_seed(7)
    conv = nn.Conv2d(c, k, ks, st, ks // 2)
    unit = PreparedConv2d(conv, 2)
    if c <= 3:  # stems read the image planes (NCHW), as in a model's first layer
        xd = matrixman.to_device(torch.rand(args.batch, c, hw, hw, generator=g) * 2 - 1)
    else:
        x = torch.rand(args.batch, hw, hw, c, generator=g) * 2 - 1
        xd = matrixman.to_device(x).permute(0, 3, 1, 2)
    with torch.no_grad():
        for _ in range(args.steps + 1):
            y = unit(xd)
    matrixman.synchronize()
    print(json.dumps({"profile_conv": [c, k, ks, st, hw], "batch": args.batch,
                      "launches": args.steps + 1, "out": list(y.shape)}))


# 3x3 stride-1 layer shapes of YOLOv8n / YOLOv8m at 640 x 640: (C, K, output H = W).
SWEEP_LAYERS = ((16, 16, 160), (32, 32, 80), (64, 64, 80), (64, 80, 80), (80, 80, 80), (96, 96, 80),
                (128, 128, 40), (192, 192, 40), (128, 128, 20))


def run_conv_sweep(args):
    """Per-layer throughput of the prepared tensor-core convolution (SiLU
    epilogue, NHWC input larger than L2 for the 80 x 80 and 160 x 160 layers):
    CUDA events around 5 back-to-back launches, median of 7."""
    import torch
    from torch import nn

    import matrixman_b200 as matrixman
    from matrixman_b200 import runtime as mrt
    from matrixman_b200.preparation import PreparedConv2d
    matrixman.init()
    matrixman.config.cuda_graphs = False
    rt = mrt.get_runtime(0)
    batch = args.batch or 64
    ceiling = measured_peaks()["bf16_tflops_sustained"] / 6.0
    g = torch.Generator().manual_seed(7)
    for c, k, hw in SWEEP_LAYERS:
        unit = PreparedConv2d(nn.Conv2d(c, k, 3, 1, 1), 2)
        x = torch.rand(batch, hw, hw, c, generator=g) * 2 - 1
        xd = matrixman.to_device(x).permute(0, 3, 1, 2)
        with torch.no_grad():
            y = unit(xd)
            rt.synchronize()
            times = []
            for _ in range(7):
                t = mrt.Timer(rt)
                t.start()
                for _ in range(5):
                    y = unit(xd)
                t.stop()
                times.append(t.elapsed_ms() / 5)
        ms = sorted(times)[3]
        tf = 2.0 * batch * hw * hw * k * c * 9 / (ms * 1e-3) / 1e12
        print(json.dumps({"conv_sweep": [c, k, 3, hw], "batch": batch, "ms": round(ms, 4),
                          "tflops": round(tf, 1), "frac_of_3xtf32_ceiling": round(tf / ceiling, 3)}),
              flush=True)
        del xd, y


def run_reference(args, world, rank):
    """Reference arm: the path's CPU ground truth (the unprepared model on
    torch CPU fp32, or the single convolution for c1), rank 0 only."""
    if rank != 0:
        return
    import torch
    import torch.nn.functional as F
    import workloads as W
    from oracle.models import cpu_model_name
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    steps = max(1, min(args.steps, 5))
    if args.workload == "c1":
        x, w = W.conv1_case(0)
        reps = 200  # convolutions per step (about a second of CPU work)
        with torch.no_grad():
            F.conv2d(x, w, None, 1, 1)
            t0 = time.perf_counter()
            for _ in range(steps * reps):
                F.conv2d(x, w, None, 1, 1)
            el = time.perf_counter() - t0
        value, unit, metric = steps * reps / el, "convs/s", C1_METRIC
        workload = "conv2d [1,4,320,320] x [5,4,3,3] s1 p1 fp32 on torch CPU, " \
                   f"{reps} convolutions per step"
        sample = f"{steps * reps} convolutions on {cpu_model_name()}"
        ms = el / steps * 1e3
    else:
        spec = _specs()[args.workload]
        model = spec.model()
        n = min(spec.cpu_sample, spec.batch_per_gpu(1, args.batch))
        x = spec.inputs(n, 99)
        with torch.no_grad():
            model(x)
            t0 = time.perf_counter()
            for _ in range(steps):
                model(x)
            el = time.perf_counter() - t0
        value, unit, metric = steps * n / el, spec.unit, spec.metric
        workload = f"{spec.desc} (unprepared, torch CPU fp32), bounded sample of {n} per step"
        sample = f"{steps} x batch-{n} forwards on {cpu_model_name()}"
        ms = el / steps * 1e3
    line = {
        "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": steps,
        "warmup": 1, "ms_per_step": round(ms, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic seeded inputs, random-init weights (seeded)",
        "config": {"workload": workload, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


C1_METRIC = "conv2d [1,4,320,320]x[5,4,3,3] s1 p1 fp32 convolutions/sec"
C1_BYTES = 4 * (1 * 4 * 320 * 320 + 1 * 5 * 320 * 320 + 5 * 4 * 3 * 3)  # 3,687,120 B minimal traffic


def run_c1(args):
    """Config 1: the reference's conv demo shape, one convolution per step.

    HBM-bound (3,687,120 algorithmic bytes) and launch-latency-bound.  The
    working set of one call (3.7 MB) fits in L2, so the timed steps rotate
    over 48 distinct input/output pairs (177 MB, more than the 126 MB L2).
    value: convolutions/s over K device-timed steps, the 48-call ring captured
    once as a CUDA graph and replayed (as the model benchmarks replay their
    forward), so host dispatch between launches is not timed; the same loop
    launched eagerly from Python is reported beside it; e2e: the public API
    (to_device of a pinned input, F.conv2d with the CPU weight, .cpu())."""
    import torch
    import torch.nn.functional as F

    import matrixman_b200 as matrixman
    import workloads as W
    from matrixman_b200 import ops, runtime
    from matrixman_b200 import telemetry as profiling
    from oracle import ops as O
    from oracle.models import cpu_model_name
    from oracle.tolerance import CONV_GEMM_REL, max_rel_err

    world, rank, local = dist_env()
    if world > 1:
        raise SystemExit("bench: the c1 workload is a single-GPU configuration")
    matrixman.init()
    rt = runtime.get_runtime(local)
    x, w = W.conv1_case(0)
    ring = 48
    xs = [matrixman.to_device(x * (1.0 + 0.01 * i), device=local) for i in range(ring)]
    wd = matrixman.to_device(w, device=local)
    ys = [ops.empty(rt, (1, 5, 320, 320)) for _ in range(ring)]

    def conv(i):
        ops.convolution(xs[i], wd, None, (1, 1), (1, 1), (1, 1), 1, out=ys[i])

    for i in range(max(args.warmup, 3) * ring):
        conv(i % ring)
    rt.synchronize()
    steps = max(args.steps, ring)
    clocks = ClockSampler(local)
    clocks.start()
    t_pre = time.perf_counter()
    while time.perf_counter() - t_pre < 0.4:
        conv(0)
        rt.synchronize()
    # Eager loop (host dispatch between launches included).
    timer = runtime.Timer(rt)
    timer.start()
    for i in range(steps):
        conv(i % ring)
    timer.stop()
    eager_ms = timer.elapsed_ms() / steps
    # The ring as one CUDA graph, replayed: device throughput.
    rt.synchronize()
    rt.capture_begin()
    try:
        for i in range(ring):
            conv(i)
    finally:
        graph = rt.capture_end()
    for _ in range(3):
        graph.replay()
    rt.synchronize()
    replays = (steps + ring - 1) // ring
    steps = replays * ring
    timer = runtime.Timer(rt)
    timer.start()
    for _ in range(replays):
        graph.replay()
    timer.stop()
    ms_total = timer.elapsed_ms()
    launches = steps
    clock_info = clocks.stop()
    ms = ms_total / steps
    graph.destroy()
    value = 1e3 / ms
    peaks = measured_peaks()
    achieved = C1_BYTES / (ms / 1e3) / 1e9
    y_last = ys[(steps - 1) % ring].cpu()
    ref = O.conv2d(x * (1.0 + 0.01 * ((steps - 1) % ring)), w, None, 1, 1)
    err = max_rel_err(y_last, ref)
    # End to end through the public API.
    xp = matrixman.pinned_empty(x.shape)
    xp.copy_(x)
    with torch.no_grad():
        for _ in range(5):
            F.conv2d(matrixman.to_device(xp, device=local), w, None, 1, 1).cpu()
        t0 = time.perf_counter()
        n_e2e = 200
        for _ in range(n_e2e):
            F.conv2d(matrixman.to_device(xp, device=local), w, None, 1, 1).cpu()
        e2e_s = (time.perf_counter() - t0) / n_e2e
    line = {
        "metric": C1_METRIC, "value": round(value, 1), "unit": "convs/s", "n_gpus": 1, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "x ~ U[-1,1] seeded, Kaiming-uniform weight (the reference's conv demo case)",
        "config": {"workload": "conv2d [1,4,320,320] x [5,4,3,3] s1 p1, no bias (config 1)",
                   "l2": f"timed steps rotate over {ring} input/output pairs "
                         f"({ring * C1_BYTES / 1e6:.0f} MB > 126 MB L2)",
                   "timing": f"the {ring}-call ring captured as one CUDA graph, {replays} replays",
                   "eager_loop_convs_per_s": round(1e3 / eager_ms, 1),
                   "parallelism": "single GPU"},
        "e2e": {"value": round(1.0 / e2e_s, 1), "unit": "convs/s", "h2d_bytes_per_step": int(x.numel() * 4),
                "d2h_bytes_per_step": int(5 * 320 * 320 * 4), "ms_per_step": e2e_s * 1e3,
                "api": "F.conv2d(matrixman.to_device(pinned x), cpu weight).cpu()"},
        "roofline": {"bound": "hbm", "kernel": "mm_conv2d (direct small-channel kernel)",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "algorithmic_bytes_per_launch": C1_BYTES,
                     "peak_basis": f"{peaks['source']} HBM copy bandwidth",
                     "note": "one 3.7 MB convolution per launch: launch latency, not bandwidth, "
                             "bounds a single call"},
        "parity": {"max_rel_err": err, "bar": CONV_GEMM_REL, "ok": bool(err < CONV_GEMM_REL),
                   "what": "last timed step's output vs torch CPU conv2d"},
        "gpu_launches": launches, "clocks": clock_info,
    }
    if not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        with torch.no_grad():
            F.conv2d(x, w, None, 1, 1)
            t0 = time.perf_counter()
            n = 0
            while time.perf_counter() - t0 < 10.0:
                F.conv2d(x, w, None, 1, 1)
                n += 1
            el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(n / el, 1), "unit": "convs/s", "cores": torch.get_num_threads(),
                                "kind": "port",
                                "sample": f"{n} convolutions on torch CPU fp32 ({cpu_model_name()}), {el:.1f} s"}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
