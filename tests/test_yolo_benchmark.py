"""matrixman.yolo-benchmark.v1 documents from the per-frame runner."""

import pytest

from matrixman_b200 import yolo_benchmark as yb

TOP_KEYS = {"schema", "backend", "variant", "configuration", "warmup_frames_completed",
            "measured_frames", "summary", "profile"}
FRAME_KEYS = {"index", "inference_seconds", "upload_seconds", "readback_seconds",
              "postprocess_seconds", "total_seconds", "process_cpu_seconds", "thread_cpu_seconds",
              "readback_bytes", "candidates_before_nms", "detections", "residency", "stages",
              "diagnostics"}
SUMMARY_KEYS = {"measured_frames", "mean_total_seconds", "mean_fps", "mean_stage_seconds",
                "mean_cpu_stage_timings", "warmup_cpu_stage_timings", "warmup_gl_call_timings",
                "mean_process_cpu_seconds", "mean_thread_cpu_seconds", "residency"}


def test_summary_block_means():
    frames = [{"total_seconds": t, "process_cpu_seconds": 0.5 * t, "thread_cpu_seconds": 0.25 * t,
               "stages": {"preprocessing": {"wall_seconds": t / 2, "thread_cpu_seconds": t / 4}}}
              for t in (0.1, 0.3)]
    s = yb.summarize(frames)
    assert set(s) == SUMMARY_KEYS
    assert s["measured_frames"] == 2
    assert s["mean_total_seconds"] == pytest.approx(0.2)
    assert s["mean_fps"] == pytest.approx(5.0)
    assert s["mean_stage_seconds"]["preprocessing"]["wall_seconds"] == pytest.approx(0.1)
    assert yb.summarize([])["mean_fps"] is None


@pytest.mark.gpu
@pytest.mark.parametrize("preprocess", ["device", "cpu"])
def test_runner_document(mm, preprocess):
    doc = yb.run(frames=3, warmup=1, imgsz=256, conf=0.3, iou=0.5, max_det=50, preprocess=preprocess)
    assert set(doc) == TOP_KEYS and doc["schema"] == "matrixman.yolo-benchmark.v1"
    assert doc["warmup_frames_completed"] == 1 and len(doc["measured_frames"]) == 3
    for f in doc["measured_frames"]:
        assert set(f) == FRAME_KEYS
        assert set(f["stages"]) == set(yb.STAGES[preprocess])
        assert 0 <= f["detections"] <= 50
    assert doc["summary"]["mean_fps"] > 0
