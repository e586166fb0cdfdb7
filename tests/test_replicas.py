"""Whole-model replicas: batch slicing, the rank-0 output gather (gloo ranks
on CPU), and the single-process ReplicaSet on the devices present."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from matrixman_b200.replicas import batch_slices, gather_to_root


def test_batch_slices_cover_batch_in_order():
    for batch in (0, 1, 7, 64, 256, 257):
        for parts in (1, 2, 3, 4, 8):
            sl = batch_slices(batch, parts)
            assert len(sl) == parts
            assert sl[0][0] == 0 and sl[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
            sizes = [e - s for s, e in sl]
            assert max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)


def test_infer_ramp_slices_cover_batch():
    from matrixman_b200.pipeline import ramp_slices
    assert [e - s for s, e in ramp_slices(64, 4)] == [8, 16, 24, 16]
    assert ramp_slices(0, 4) == []
    for batch in (1, 2, 3, 7, 22, 64, 65, 257):
        for chunks in (1, 2, 3, 4, 5, 8):
            sl = ramp_slices(batch, chunks)
            assert len(sl) == min(chunks, batch)
            assert sl[0][0] == 0 and sl[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
            assert all(e > s for s, e in sl)


def test_batch_slices_rejects_bad_arguments():
    with pytest.raises(ValueError):
        batch_slices(4, 0)
    with pytest.raises(ValueError):
        batch_slices(-1, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, sizes, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        start = sum(sizes[:rank])
        # rank r's slice of a global batch whose rows are their global index
        local = torch.arange(start, start + sizes[rank], dtype=torch.float32)[:, None, None].expand(
            sizes[rank], 3, 5).contiguous()
        out = gather_to_root(local, sizes)
        if rank == 0:
            queue.put(out.clone())
        else:
            queue.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("sizes", [[4, 4], [5, 3], [3, 0]])
def test_gather_to_root_gloo_world2(sizes):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, sizes, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gathered = [r for r in results if r is not None]
    assert len(gathered) == 1
    out = gathered[0]
    total = sum(sizes)
    assert out.shape == (total, 3, 5)
    expect = torch.arange(total, dtype=torch.float32)[:, None, None].expand(total, 3, 5)
    assert torch.equal(out, expect)


def _mismatch_worker(rank, world, port, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        try:
            gather_to_root(torch.zeros(2, 3), [3, 3])  # every rank claims 3 rows, has 2
            queue.put("no error")
        except ValueError:
            queue.put("ValueError")
    finally:
        dist.destroy_process_group()


def test_gather_to_root_checks_local_size():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mismatch_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    # the size check runs before any transfer, so no rank waits on another
    assert results == ["ValueError", "ValueError"]


@pytest.mark.gpu
def test_replica_set_matches_oracle(mm):
    import workloads as W
    from matrixman_b200 import runtime
    from matrixman_b200.replicas import ReplicaSet
    from oracle.tolerance import CONV_GEMM_REL, max_rel_err

    n_dev = runtime.device_count()
    devices = list(range(min(n_dev, 2)))
    model = W.yolov8_model("n")
    x = W.yolo_input(3, size=320)
    with torch.no_grad():
        ref = model(x)
    rs = ReplicaSet(model, devices)
    y = rs(x)
    assert tuple(y.shape) == tuple(ref.shape)
    assert max_rel_err(y.cpu(), ref) < CONV_GEMM_REL
