"""Build recipe for the native parts of matrixman_b200.

* ``libmatrixman_b200.so`` -- every CUDA kernel and the C ABI declared in
  ``include/matrixman_b200.h``, compiled by nvcc for sm_100a only.
* ``_matrixman_hooks*.so`` -- the C++ PrivateUse1 hooks / DeviceGuard
  extension (needs torch headers; built with torch.utils.cpp_extension).

Artefacts are written in-tree (``matrixman_b200/_lib/``) so they travel with
the repository snapshot.  Run ``python -m matrixman_b200.build``.
"""

from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "_lib"
BUILD = PKG / "_build"
LIB_NAME = "libmatrixman_b200.so"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    f"-I{ROOT / 'include'}",
]

SOURCES = ["mm_runtime.cu", "mm_ops.cu", "mm_conv_simt.cu", "mm_conv_tc.cu", "mm_detect.cu", "mm_frames.cu", "mm_train.cu"]


def _digest(paths) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(Path(p).read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, flush=True)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA sources into matrixman_b200/_lib/libmatrixman_b200.so."""
    OUT.mkdir(exist_ok=True)
    BUILD.mkdir(exist_ok=True)
    sources = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    deps = sources + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + [ROOT / "include" / "matrixman_b200.h"]
    stamp = BUILD / "lib.stamp"
    lib = OUT / LIB_NAME
    digest = _digest(deps)
    if not force and lib.exists() and stamp.exists() and stamp.read_text() == digest:
        return lib
    objs = [BUILD / (s.stem + ".o") for s in sources]
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        futs = [ex.submit(_compile, s, o, verbose) for s, o in zip(sources, objs)]
        for f in futs:
            f.result()
    tmp = OUT / (LIB_NAME + ".tmp")
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "shared", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    stamp.write_text(digest)
    return lib


def build_hooks(force: bool = False, verbose: bool = False) -> Path | None:
    """Build the C++ PrivateUse1 hooks extension in-tree (torch headers)."""
    src = CSRC / "privateuse1_hooks.cpp"
    if not src.exists():
        return None
    from torch.utils import cpp_extension  # noqa: WPS433 - build-time only

    OUT.mkdir(exist_ok=True)
    bdir = BUILD / "hooks"
    bdir.mkdir(parents=True, exist_ok=True)
    stamp = bdir / "hooks.stamp"
    digest = _digest([src])
    existing = sorted(OUT.glob("_matrixman_hooks*.so"))
    if not force and existing and stamp.exists() and stamp.read_text() == digest:
        return existing[0]
    mod = cpp_extension.load(
        name="_matrixman_hooks",
        sources=[str(src)],
        build_directory=str(bdir),
        extra_cflags=["-O2"],
        with_cuda=False,
        verbose=verbose,
        is_python_module=True,
    )
    built = Path(mod.__file__)
    target = OUT / built.name
    shutil.copy2(built, target)
    stamp.write_text(digest)
    return target


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_hooks(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(f"built {OUT / LIB_NAME}")
