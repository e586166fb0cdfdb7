"""Per-frame YOLO benchmark that writes ``matrixman.yolo-benchmark.v1`` JSON.

Mirrors the reference runner (``drivers/matrixman/benchmarks/yolo_benchmark.py``:
frame loop at :213-297, document at :308-383): each frame is preprocessed on
the CPU exactly as the reference does (``demo/yolo_helpers.py:53-56``: cv2
INTER_LINEAR resize, BGR -> RGB, CHW float32 / 255), uploaded, run through the
prepared model, and post-processed.  Stage names and the document's keys are
the reference's.  Differences:

* frames are seeded synthetic 1920 x 1080 uint8 BGR images (no video file);
* with ``preprocess="device"`` (the default) the uint8 frame is uploaded and
  resized / converted on the device (``preprocess_frames``, bit-identical to
  the CPU path) in the stage ``device_preprocessing``, which also stands for
  the upload; ``preprocess="cpu"`` keeps the reference's CPU preprocessing;
* postprocessing runs on the device (``postprocess_detections``: filter + NMS),
  so ``explicit_readback`` moves only the kept detections; the stage
  ``device_postprocess`` covers the kernel, that readback and packaging, and
  ``readback_seconds`` / ``postprocess_seconds`` both report it;
* OpenGL-only diagnostics (``gl_calls``, texture residency) are empty.

Run: ``python -m matrixman_b200.yolo_benchmark --frames 100 --warmup 10 --json out.json``.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from pathlib import Path

import numpy as np
import torch

SCHEMA = "matrixman.yolo-benchmark.v1"
STAGES = {"cpu": ("preprocessing", "host_to_gpu_upload", "matrixman_dispatch", "device_postprocess"),
          "device": ("device_preprocessing", "matrixman_dispatch", "device_postprocess")}


def _thread_time() -> float:
    return getattr(time, "thread_time", time.process_time)()


class _Stages:
    """Per-frame stage timer: wall and thread-CPU seconds per stage name."""

    def __init__(self):
        self.values: dict[str, dict[str, float]] = {}

    def __call__(self, name: str):
        stages = self

        class _Ctx:
            def __enter__(self):
                self.w, self.t = time.perf_counter(), _thread_time()

            def __exit__(self, *exc):
                v = stages.values.setdefault(name, {"wall_seconds": 0.0, "thread_cpu_seconds": 0.0})
                v["wall_seconds"] += time.perf_counter() - self.w
                v["thread_cpu_seconds"] += _thread_time() - self.t
                return False

        return _Ctx()


def preprocess_frame(frame: np.ndarray, image_size: int) -> torch.Tensor:
    """The reference's CPU preprocessing (demo/yolo_helpers.py:53-56)."""
    import cv2

    resized = cv2.resize(frame, (image_size, image_size), interpolation=cv2.INTER_LINEAR)
    rgb = cv2.cvtColor(resized, cv2.COLOR_BGR2RGB)
    return torch.from_numpy(rgb).permute(2, 0, 1).contiguous().to(torch.float32).div_(255.0).unsqueeze(0)


def synthetic_frames(count: int, seed: int = 0, height: int = 1080, width: int = 1920):
    rng = np.random.default_rng(seed)
    for _ in range(count):
        yield rng.integers(0, 256, size=(height, width, 3), dtype=np.uint8)


def summarize(measured: list[dict]) -> dict:
    """The ``summary`` block of the document (reference :319-374, GL parts empty)."""
    n = len(measured)
    totals = [f["total_seconds"] for f in measured]
    names = sorted({name for f in measured for name in f["stages"]})
    return {
        "measured_frames": n,
        "mean_total_seconds": sum(totals) / n if n else None,
        "mean_fps": n / sum(totals) if n and sum(totals) else None,
        "mean_stage_seconds": {
            name: {m: sum(f["stages"].get(name, {}).get(m, 0.0) for f in measured) / n
                   for m in ("wall_seconds", "thread_cpu_seconds")}
            for name in names
        },
        "mean_cpu_stage_timings": {"stages": {}, "gl_calls": {}},
        "warmup_cpu_stage_timings": {},
        "warmup_gl_call_timings": {},
        "mean_process_cpu_seconds": sum(f["process_cpu_seconds"] for f in measured) / n if n else None,
        "mean_thread_cpu_seconds": sum(f["thread_cpu_seconds"] for f in measured) / n if n else None,
        "residency": {"warmup": {}, "warmup_parameter_groups": [], "first_measured_frame": {},
                      "measured_parameter_groups": [], "steady_state_measured_frames": {}},
    }


def run(frames: int = 100, warmup: int = 10, imgsz: int = 640, conf: float = 0.25,
        iou: float = 0.45, max_det: int = 300, seed: int = 0, variant: str = "n",
        preprocess: str = "device") -> dict:
    if preprocess not in STAGES:
        raise ValueError("preprocess must be 'cpu' or 'device'")
    import matrixman_b200 as matrixman
    import workloads as W

    matrixman.init()
    net = matrixman.prepare(W.yolov8_model(variant))
    measured, warmup_done, started_cpu = [], 0, time.process_time()
    with torch.no_grad():
        for frame in synthetic_frames(warmup + frames, seed):
            t0, p0, th0 = time.perf_counter(), time.process_time(), _thread_time()
            st = _Stages()
            if preprocess == "device":
                with st("device_preprocessing"):
                    gpu_input = matrixman.preprocess_frames(frame, imgsz)
            else:
                with st("preprocessing"):
                    cpu_input = preprocess_frame(frame, imgsz)
                with st("host_to_gpu_upload"):
                    gpu_input = matrixman.to_device(cpu_input)
            with st("matrixman_dispatch"):
                output = net(gpu_input)
            with st("device_postprocess"):
                dets = matrixman.postprocess_detections(output, imgsz, imgsz, conf, iou, max_det=max_det)[0]
            if warmup_done < warmup:
                warmup_done += 1
                continue
            post = st.values["device_postprocess"]["wall_seconds"]
            measured.append({
                "index": len(measured),
                "inference_seconds": st.values["matrixman_dispatch"]["wall_seconds"],
                "upload_seconds": st.values["host_to_gpu_upload" if preprocess == "cpu"
                                            else "device_preprocessing"]["wall_seconds"],
                "readback_seconds": post,
                "postprocess_seconds": post,
                "total_seconds": time.perf_counter() - t0,
                "process_cpu_seconds": time.process_time() - p0,
                "thread_cpu_seconds": _thread_time() - th0,
                "readback_bytes": max_det * 6 * 4 + 4,
                "candidates_before_nms": None,
                "detections": len(dets),
                "residency": {},
                "stages": {k: dict(v) for k, v in st.values.items()},
                "diagnostics": {},
            })
    return {
        "schema": SCHEMA,
        "backend": {"requested": "cuda", "name": "matrixman_b200",
                    "device": torch.cuda.get_device_name(0) if torch.cuda.is_available() else None},
        "variant": variant,
        "configuration": {
            "model": f"yolov8{variant} (random-init weights, seeded)",
            "video": f"synthetic 1920x1080 uint8 BGR frames (seed {seed})",
            "imgsz": imgsz, "conf": conf, "iou": iou, "warmup_frames": warmup, "preprocess": preprocess,
            "measured_frames_requested": frames,
            "environment": {k: v for k, v in os.environ.items() if k.startswith("MATRIXMAN")},
        },
        "warmup_frames_completed": warmup_done,
        "measured_frames": measured,
        "summary": summarize(measured),
        "profile": {"process_cpu_seconds": time.process_time() - started_cpu},
    }


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--frames", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--imgsz", type=int, default=640)
    p.add_argument("--conf", type=float, default=0.25)
    p.add_argument("--iou", type=float, default=0.45)
    p.add_argument("--variant", default="n")
    p.add_argument("--preprocess", choices=("device", "cpu"), default="device")
    p.add_argument("--json", type=Path, default=Path("yolo_benchmark.json"))
    args = p.parse_args(argv)
    result = run(args.frames, args.warmup, args.imgsz, args.conf, args.iou, variant=args.variant,
                 preprocess=args.preprocess)
    args.json.parent.mkdir(parents=True, exist_ok=True)
    args.json.write_text(json.dumps(result, indent=2) + "\n", encoding="utf-8")
    print(f"benchmark JSON: {args.json}  mean_fps={result['summary']['mean_fps']}")
    return 0 if len(result["measured_frames"]) == args.frames else 2


if __name__ == "__main__":
    raise SystemExit(main())
