"""CPU oracle for the matrixman_b200 parity tests -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline; the product (``matrixman_b200``) never
calls it and has no CPU fallback.

What it restates.  MatrixMan's own ground truth for every op on its tensor
path is stock PyTorch CPU fp32 (the reference's diagnostics compare against
``F.conv2d`` / ``torch.softmax`` / NumPy, e.g.
drivers/matrixman/diagnostics/matrixman_conv_demo.py:57-70 and
drivers/matrixman/backends/cuda/conv2d.py:13-46), so each function in
``oracle.ops`` is the torch-CPU (or NumPy) computation of one op with the
reference's semantics, citing the reference file:line it follows.
``oracle.models`` runs whole workloads unprepared on the CPU.

How it is pinned.  ``tests/golden/make_golden.py`` imported the reference
package itself (drivers.matrixman, CPU-only parts) and recorded the outputs of
its own reference functions -- ``reference_conv2d`` (backends/cuda/conv2d.py:13),
``nearest_reference`` (backends/cuda/upsample.py:9), the BatchNorm and SiLU
known-answer formulas (backends/cuda/batch_norm.py:9-22, silu.py:9-11), the
max-pool demo cases (diagnostics/cuda_maxpool_diagnostic.py), ``_fold_pair``
(preparation.py:360-398) and the view-metadata helpers (tensor.py:161-268) --
into ``tests/golden/*.npz``.  ``tests/test_oracle_golden.py`` checks this
oracle against every one of those vectors.  The PrivateUse1 kernels of the
reference (sm_21 PTX) cannot run here (no GPU), so parity with the reference's
device code is not claimed; parity is with its CPU ground truth.
"""
