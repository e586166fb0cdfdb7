"""Worker for the multi-GPU tests (one process per GPU, started by
tests/test_multigpu_gpu.py through torch.distributed.run).

Each rank runs the prepared YOLOv8n on its own batch slice, then
 1. gathers every rank's output into rank 0's HBM with copy-engine writes
    (PeerGather, CUDA IPC) for two consecutive steps, and
 2. gathers the same outputs with NCCL point-to-point sends (gather_to_root),
and rank 0 checks both gathers against the CPU oracle of every rank's input.
Rank 0 prints one JSON line with the errors."""

from __future__ import annotations

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", local))

    import matrixman_b200 as matrixman
    import workloads as W
    from matrixman_b200 import runtime
    from matrixman_b200.replicas import PeerGather, gather_to_root
    from oracle.models import run_cpu
    from oracle.tolerance import CONV_GEMM_REL, max_rel_err

    runtime.set_device(local)
    matrixman.init()
    model = W.yolov8_model("n")
    prepared = matrixman.prepare(model)
    sizes = [2 + (r % 2) for r in range(world)]  # uneven slices
    size = 256
    inputs = [W.yolo_input(sizes[r], seed=500 + r, size=size) for r in range(world)]
    anchors = (size // 8) ** 2 + (size // 16) ** 2 + (size // 32) ** 2
    pg = PeerGather((84, anchors), sizes, device=local)
    errs = {}
    with torch.no_grad():
        for step in range(2):  # two pushes: both gather slots are used
            scale = 1.0 if step == 0 else 0.5
            y = prepared(matrixman.to_device(inputs[rank] * scale, device=local))
            pg.push(y)
            full = pg.collect()
            if rank == 0:
                ref = torch.cat([run_cpu(model, inputs[r] * scale) for r in range(world)])
                errs[f"peer_gather_step{step}"] = max_rel_err(full.cpu(), ref)
        y = prepared(matrixman.to_device(inputs[rank], device=local))
        full = gather_to_root(y, sizes)
        if rank == 0:
            ref = torch.cat([run_cpu(model, inputs[r]) for r in range(world)])
            errs["gather_to_root"] = max_rel_err(full.cpu(), ref)
    pg.close()
    t = torch.zeros(1, device=torch.device("cuda", local))
    dist.all_reduce(t)
    torch.cuda.synchronize(local)
    dist.destroy_process_group()
    if rank == 0:
        ok = all(v < CONV_GEMM_REL for v in errs.values())
        print(json.dumps({"world": world, "errors": errs, "ok": ok}), flush=True)


if __name__ == "__main__":
    main()
