"""``matrixman.config``: typed runtime settings.

Public surface follows drivers/matrixman/config.py of the reference:

* camelCase fields with snake_case aliases (config.py:73-110),
* precedence default -> ``MATRIXMAN_*`` environment -> Python override
  (config.py:349-377, 420-441),
* fields that shape the runtime (backend, tileLimit, tileSync, syncPolicy,
  activationPool, scratchPool, useDGPU) are locked once a device runtime
  exists (config.py:114-117, 581-595),
* ``keys/items/metadata/options/describe/help/show/source/asDict/reset/
  reloadFromEnvironment`` introspection, and the scratch-flag compatibility
  rules (config.py:703-713).

B200 meaning of the north-star knobs:

* ``sync_policy`` -- ``safe``: a pooled block reused on any stream first waits
  for the event recorded at its release; ``relaxed``: reuse is ordered by the
  single runtime stream only; ``auto`` resolves to ``relaxed`` because every op
  runs on one stream per device.
* ``activation_pool`` / ``scratch_pool`` -- ``safe``: released blocks are
  reusable immediately (ordering as above); ``deferred``: released blocks stay
  pending until their release event has completed.
* ``tile_limit`` -- validated, stored and reported with the reference's rules
  (a positive integer or ``auto``; default 256), and locked after init like
  the other runtime fields.  The reference uses it to bound the physical
  OpenGL tile a convolution renders into (backends/opengl/convolution.py:1299).
  On CUDA a limit the user sets (environment or Python) bounds the extent of
  one convolution launch: an output wider or taller than the limit runs as
  several launches of at most limit x limit output pixels each
  (mm_conv2d_region / mm_conv2d_tc_region), with the same result bit for
  bit.  The default value and ``auto`` mean one launch per convolution,
  whatever its size, as in the reference's CUDA backend (which never reads
  the setting).

Settings without a CUDA meaning (OpenGL diagnostics) are accepted and
reported so that existing scripts keep working; they have no effect.
"""

from __future__ import annotations

import os
from typing import Any

_TRUE = {"1", "true", "yes", "on"}
_FALSE = {"", "0", "false", "no", "off"}

_SYNC_POLICIES = ("safe", "auto", "relaxed")
_POOLS = ("safe", "deferred")
_TILE_SYNCS = ("per_tile", "end", "flush", "none")
_BACKENDS = ("auto", "opengl", "cuda")
_PROFILE_MODES = ("summary", "detail", "trace")
_CONV_ALGOS = ("auto", "simt", "tc")

# field -> (default, env var, snake alias, category, status, description)
_FIELDS: dict[str, tuple] = {
    "backend": ("auto", "MATRIXMAN_BACKEND", None, "Backend / device", "stable",
                "Selects the MatrixMan execution backend."),
    "useDGPU": (False, "MATRIXMAN_USE_DGPU", "use_dgpu", "Backend / device", "backend-specific",
                "Requests a discrete adapter (no effect on CUDA)."),
    "tileLimit": (256, "MATRIXMAN_TILE_LIMIT", "tile_limit", "OpenGL tiling", "stable",
                  "Largest output rows/columns of one convolution launch when set (default, auto: no limit)."),
    "tileSync": ("per_tile", "MATRIXMAN_TILE_SYNC", "tile_sync", "OpenGL tiling", "stable",
                 "Tiled-convolution synchronization (no effect on CUDA)."),
    "syncPolicy": ("safe", "MATRIXMAN_SYNC_POLICY", "sync_policy", "Synchronization", "stable",
                   "Pool reuse ordering: safe (event wait), auto, relaxed (stream order)."),
    "convSpatialReuse": (False, "MATRIXMAN_CONV_SPATIAL_REUSE", "conv_spatial_reuse", "Convolution",
                         "experimental", "OpenGL spatial-reuse convolution (no effect on CUDA)."),
    "activationPool": ("safe", "MATRIXMAN_ACTIVATION_POOL", "activation_pool",
                       "Memory / texture reuse", "experimental",
                       "Activation block reuse: safe or deferred until release completes."),
    "scratchPool": ("safe", "MATRIXMAN_SCRATCH_POOL", "scratch_pool", "Memory / texture reuse",
                    "experimental", "Scratch block reuse: safe or deferred until release completes."),
    "preparedExecution": (True, "MATRIXMAN_PREPARED_EXECUTION", "prepared_execution", "Convolution",
                          "experimental", "Enables prepared execution and inference folding."),
    "convDiag": (False, "MATRIXMAN_CONV_DIAG", "conv_diag", "Diagnostics", "diagnostic",
                 "Convolution diagnostic view (no effect on CUDA)."),
    "skipPreConsolidationSync": (True, "MATRIXMAN_SKIP_PRE_CONSOLIDATION_SYNC",
                                 "skip_pre_consolidation_sync", "Synchronization", "experimental",
                                 "Skips a redundant pre-consolidation synchronization point."),
    "diagnosticTiles": (False, "MATRIXMAN_DIAGNOSTIC_TILES", "diagnostic_tiles", "Diagnostics",
                        "diagnostic", "Tiled-convolution diagnostic snapshots."),
    "diagnosticRectTiles": (False, "MATRIXMAN_DIAGNOSTIC_RECT_TILES", "diagnostic_rect_tiles",
                            "Diagnostics", "diagnostic", "Rectangular diagnostic tiles."),
    "diagTileWidth": (None, "MATRIXMAN_DIAG_TILE_WIDTH", "diag_tile_width", "Diagnostics",
                      "diagnostic", "Diagnostic rectangular tile width."),
    "diagTileHeight": (None, "MATRIXMAN_DIAG_TILE_HEIGHT", "diag_tile_height", "Diagnostics",
                       "diagnostic", "Diagnostic rectangular tile height."),
    "diagTileOrder": ("normal", "MATRIXMAN_DIAG_TILE_ORDER", "diag_tile_order", "Diagnostics",
                      "diagnostic", "Diagnostic tile traversal order."),
    "diagConvWorkload": ("heavy", "MATRIXMAN_DIAG_CONV_WORKLOAD", "diag_conv_workload",
                         "Diagnostics", "diagnostic", "Compatibility diagnostic workload."),
    "profile": (False, "MATRIXMAN_PROFILE", None, "Profiling", "stable",
                "Profiler collection and report verbosity."),
    "cudaProfile": (False, "MATRIXMAN_CUDA_PROFILE", "cuda_profile", "CUDA", "backend-specific",
                    "Enables the CUDA runtime profiler."),
    "profileDetail": (False, "MATRIXMAN_PROFILE_DETAIL", "profile_detail", "Profiling",
                      "diagnostic", "Detailed profiler sections."),
    "profileDispatch": (False, "MATRIXMAN_PROFILE_DISPATCH", "profile_dispatch", "Profiling",
                        "diagnostic", "Collects PyTorch-facing dispatch timing."),
    "gpuTiming": (False, "MATRIXMAN_GPU_TIMING", "gpu_timing", "Profiling", "diagnostic",
                  "Times each op on the device with CUDA events."),
    "trace": (False, "MATRIXMAN_TRACE", None, "Profiling", "diagnostic",
              "Live execution diagnostics (true) or detailed internal diagnostics."),
    "residencyTrace": (False, "MATRIXMAN_TRACE_RESIDENCY", "residency_trace", "Profiling",
                       "diagnostic", "Prints allocation residency transitions."),
    "debug": (False, "MATRIXMAN_DEBUG", None, "Advanced / debug", "diagnostic",
              "Low-level diagnostic output."),
    "gpuPostprocess": (False, "MATRIXMAN_GPU_POSTPROCESS", "gpu_postprocess", "Advanced / debug",
                       "experimental", "Benchmark GPU postprocessing."),
    "auditCpuLeaks": (False, "MATRIXMAN_AUDIT_CPU_LEAKS", "audit_cpu_leaks", "Advanced / debug",
                      "diagnostic", "Audits unexpected CPU materialization."),
    "unsafeScratchReuse": (False, "MATRIXMAN_DEBUG_UNSAFE_SCRATCH_REUSE", "unsafe_scratch_reuse",
                           "Advanced / debug", "experimental", "Disables safe scratch reuse fencing."),
    "debugFreshScratch": (False, "MATRIXMAN_DEBUG_FRESH_SCRATCH", "debug_fresh_scratch",
                          "Advanced / debug", "diagnostic", "Fresh scratch allocations."),
    "scratchEpochPool": (False, "MATRIXMAN_SCRATCH_EPOCH_POOL", "scratch_epoch_pool",
                         "Advanced / debug", "diagnostic", "Diagnostic epoch scratch pool."),
    "debugClearReusedScratch": (False, "MATRIXMAN_DEBUG_CLEAR_REUSED_SCRATCH",
                                "debug_clear_reused_scratch", "Advanced / debug", "diagnostic",
                                "Clears reused scratch blocks."),
    "cudaDebug": (False, "MATRIXMAN_CUDA_DEBUG", "cuda_debug", "CUDA", "backend-specific",
                  "CUDA debug output (synchronises and checks after every op)."),
    "cudaDisableAsyncQueue": (False, "MATRIXMAN_CUDA_DISABLE_ASYNC_QUEUE",
                              "cuda_disable_async_queue", "CUDA", "backend-specific",
                              "Synchronise after every launch."),
    "cudaDisableAllocPool": (False, "MATRIXMAN_CUDA_DISABLE_ALLOC_POOL", "cuda_disable_alloc_pool",
                             "CUDA", "backend-specific", "Disables the caching arena."),
    "cudaDisableSpecializedConv": (False, "MATRIXMAN_CUDA_DISABLE_SPECIALIZED_CONV",
                                   "cuda_disable_specialized_conv", "CUDA", "backend-specific",
                                   "Forces the general SIMT convolution."),
    "cudaConv3x3Variant": ("plane", "MATRIXMAN_CUDA_CONV3X3_VARIANT", "cuda_conv3x3_variant",
                           "CUDA", "backend-specific", "Accepted for compatibility; kernels are chosen by shape."),
    "cudaLegacyModuleLoad": (False, "MATRIXMAN_CUDA_LEGACY_MODULE_LOAD", "cuda_legacy_module_load",
                             "CUDA", "backend-specific", "Accepted for compatibility; no effect."),
    "tileAutotuneRefresh": (False, "MATRIXMAN_TILE_AUTOTUNE_REFRESH", "tile_autotune_refresh",
                            "Advanced / debug", "diagnostic", "Accepted for compatibility; no effect."),
    "disableAutoPrepare": (False, "MATRIXMAN_DISABLE_AUTO_PREPARE", "disable_auto_prepare",
                           "Convolution", "stable", "Disables lazy model preparation."),
    # B200 additions.
    "cudaGraphs": (True, "MATRIXMAN_CUDA_GRAPHS", "cuda_graphs", "CUDA", "backend-specific",
                   "Capture prepared forwards into CUDA graphs per input shape."),
    "convAlgo": ("auto", "MATRIXMAN_CONV_ALGO", "conv_algo", "CUDA", "backend-specific",
                 "Convolution kernel: auto, simt (fp32 FFMA) or tc (tcgen05 3xTF32)."),
    "waitTimeoutMs": (600000, "MATRIXMAN_WAIT_TIMEOUT_MS", "wait_timeout_ms", "CUDA",
                      "backend-specific", "Bound on every host wait for device work."),
    "readbackCacheMb": (2048, "MATRIXMAN_READBACK_CACHE_MB", "readback_cache_mb", "CUDA",
                        "backend-specific",
                        "Page-locked host memory kept for reuse by .cpu() results (0 = off)."),
}

_BOOL_FIELDS = {f for f, spec in _FIELDS.items() if isinstance(spec[0], bool) and f != "profile"}
_RUNTIME_PROTECTED = {"backend", "useDGPU", "tileLimit", "tileSync", "syncPolicy",
                      "activationPool", "scratchPool"}
_CATEGORY_ORDER = ("Backend / device", "OpenGL tiling", "Synchronization",
                   "Memory / texture reuse", "Convolution", "Profiling", "Diagnostics", "CUDA",
                   "Advanced / debug")

_ALIASES: dict[str, str] = {}
for _f, _spec in _FIELDS.items():
    _ALIASES[_f] = _f
    if _spec[2]:
        _ALIASES[_spec[2]] = _f
_ALIASES["scratchPolicy"] = "scratchPolicy"
_ALIASES["scratch_policy"] = "scratchPolicy"
_ALIASES["gpu_preference"] = "gpu_preference"


def _public(field: str) -> str:
    if field == "useDGPU":
        return "gpu_preference"
    return _FIELDS[field][2] or field


def _as_bool(value: Any) -> bool:
    if isinstance(value, bool):
        return value
    text = str(value).strip().lower()
    if text in _TRUE:
        return True
    if text in _FALSE:
        return False
    raise ValueError(f"expected boolean value, got {value!r}")


def _choice(field: str, value: Any, choices: tuple, default: str) -> str:
    text = str(value).strip().lower() or default
    if text not in choices:
        raise ValueError(f"{field} must be one of: {', '.join(choices)}")
    return text


def parse_value(field: str, value: Any) -> Any:
    """Parse and validate one setting (same accepted spellings as the reference)."""
    if field == "trace":
        if isinstance(value, bool):
            return value
        text = str(value).strip().lower()
        if text in _TRUE:
            return True
        if text in _FALSE:
            return False
        if text == "detailed":
            return "detailed"
        raise ValueError("trace must be one of: false, true, or detailed")
    if field == "profile":
        if isinstance(value, bool):
            return "summary" if value else False
        text = str(value).strip().lower()
        if text in _FALSE:
            return False
        if text in _TRUE:
            return "summary"
        if text in _PROFILE_MODES:
            return text
        raise ValueError("profile must be one of: 0, 1, summary, detail, trace")
    if field in _BOOL_FIELDS:
        return _as_bool(value)
    if field == "tileLimit":
        if isinstance(value, str) and value.strip().lower() == "auto":
            return "auto"
        try:
            number = int(value)
        except (TypeError, ValueError) as exc:
            raise ValueError("tileLimit must be a positive integer or 'auto'") from exc
        if number <= 0:
            raise ValueError("tileLimit must be a positive integer or 'auto'")
        return number
    if field in {"diagTileWidth", "diagTileHeight"}:
        if value is None or str(value).strip() == "":
            return None
        number = int(value)
        if number <= 0:
            raise ValueError(f"{field} must be positive")
        return number
    if field == "waitTimeoutMs":
        number = int(value)
        if number <= 0:
            raise ValueError("waitTimeoutMs must be positive")
        return number
    if field == "readbackCacheMb":
        number = int(value)
        if number < 0:
            raise ValueError("readbackCacheMb must be non-negative")
        return number
    if field == "tileSync":
        return _choice("tileSync", value, _TILE_SYNCS, "per_tile")
    if field == "syncPolicy":
        return _choice("syncPolicy", value, _SYNC_POLICIES, "safe")
    if field == "activationPool":
        return _choice("activationPool", value, _POOLS, "safe")
    if field == "scratchPool":
        return _choice("scratchPool", value, _POOLS, "safe")
    if field == "convAlgo":
        return _choice("convAlgo", value, _CONV_ALGOS, "auto")
    if field == "backend":
        text = str(value).strip().lower() or "auto"
        if text not in _BACKENDS:
            raise ValueError("MatrixMan backend must be 'auto', 'cuda', or 'opengl'")
        return text
    if field in {"diagTileOrder", "diagConvWorkload", "cudaConv3x3Variant"}:
        return str(value).strip().lower()
    return value


def _validate(values: dict[str, Any]) -> None:
    fresh = bool(values.get("debugFreshScratch"))
    epoch = bool(values.get("scratchEpochPool"))
    unsafe = bool(values.get("unsafeScratchReuse"))
    clear = bool(values.get("debugClearReusedScratch"))
    if fresh and epoch:
        raise ValueError("debugFreshScratch and scratchEpochPool are incompatible")
    if unsafe and (fresh or epoch):
        raise ValueError("unsafeScratchReuse cannot be combined with fresh or epoch scratch policy")
    if clear and not epoch:
        raise ValueError("debugClearReusedScratch requires scratchEpochPool")
    if values.get("backend") == "opengl":
        raise ValueError("MatrixMan/B200 provides the CUDA backend only; backend='opengl' is "
                         "unavailable on this build")


def _runtime_active() -> bool:
    try:
        from . import runtime
        return runtime.any_initialized()
    except Exception:  # pragma: no cover - import cycles during startup
        return False


class Configuration:
    """Singleton exposed as ``matrixman.config``."""

    def __init__(self) -> None:
        object.__setattr__(self, "_values", {})
        object.__setattr__(self, "_sources", {})
        self.reloadFromEnvironment()

    # -- lifecycle ---------------------------------------------------------
    def _ensure_mutable(self, field: str) -> None:
        if field in _RUNTIME_PROTECTED and _runtime_active():
            raise RuntimeError(
                f"MatrixMan configuration '{_FIELDS[field][2] or field}' must be set before "
                "backend initialization; call matrixman.shutdown() and configure the next "
                "runtime explicitly"
            )

    def reloadFromEnvironment(self) -> None:
        values = {f: spec[0] for f, spec in _FIELDS.items()}
        sources = {f: "default" for f in _FIELDS}
        for field, spec in _FIELDS.items():
            env = spec[1]
            if env and env in os.environ:
                values[field] = parse_value(field, os.environ[env])
                sources[field] = "environment"
        _validate(values)
        for field in _RUNTIME_PROTECTED:
            if field in self._values and self._values[field] != values[field]:
                self._ensure_mutable(field)
        object.__setattr__(self, "_values", values)
        object.__setattr__(self, "_sources", sources)

    def reset(self) -> None:
        """Built-in defaults, ignoring the environment."""
        for field in _RUNTIME_PROTECTED:
            if self._values.get(field) != _FIELDS[field][0]:
                self._ensure_mutable(field)
        object.__setattr__(self, "_values", {f: spec[0] for f, spec in _FIELDS.items()})
        object.__setattr__(self, "_sources", {f: "default" for f in _FIELDS})

    def _set(self, field: str, value: Any) -> None:
        self._ensure_mutable(field)
        parsed = parse_value(field, value)
        candidate = dict(self._values)
        candidate[field] = parsed
        _validate(candidate)
        self._values[field] = parsed
        self._sources[field] = "python override"

    # -- attribute access --------------------------------------------------
    def __getattr__(self, name: str) -> Any:
        if name.startswith("_"):
            raise AttributeError(name)
        field = _ALIASES.get(name)
        if field is None:
            raise AttributeError(f"unknown MatrixMan configuration setting: {name}")
        if field == "scratchPolicy":
            return self.scratchPolicy_value()
        if field == "gpu_preference":
            return "discrete" if self._values["useDGPU"] else "integrated"
        return self._values[field]

    def __setattr__(self, name: str, value: Any) -> None:
        if name.startswith("_"):
            object.__setattr__(self, name, value)
            return
        if name in ("preferred_backend",):
            set_preferred_backend(value)
            return
        if name == "profiling":
            set_profiling(value)
            return
        field = _ALIASES.get(name)
        if field is None:
            raise AttributeError(f"unknown MatrixMan configuration setting: {name}")
        if field == "scratchPolicy":
            raise AttributeError("scratch_policy is derived from the scratch debug flags")
        if field == "gpu_preference":
            text = str(value).strip().lower()
            if isinstance(value, bool):
                self._set("useDGPU", value)
            elif text in {"discrete", "dgpu", "1", "true", "yes", "on"}:
                self._set("useDGPU", True)
            elif text in {"integrated", "igpu", "0", "false", "no", "off"}:
                self._set("useDGPU", False)
            else:
                raise ValueError("gpu_preference must be 'integrated' or 'discrete'")
            return
        self._set(field, value)

    def __dir__(self) -> list[str]:
        return sorted(set(object.__dir__(self)) | set(self.keys()))

    # -- derived -------------------------------------------------------------
    def scratchPolicy_value(self) -> str:
        v = self._values
        if v["debugFreshScratch"]:
            return "fresh"
        if v["scratchEpochPool"]:
            return "epoch"
        if v["unsafeScratchReuse"]:
            return "unsafe_reuse"
        return "safe"

    @property
    def resolvedTileLimit(self) -> int:
        value = self._values["tileLimit"]
        return 256 if value == "auto" else int(value)

    resolved_tile_limit = resolvedTileLimit

    @property
    def resolved_sync_policy(self) -> str:
        """``auto`` resolves to ``relaxed``: one runtime stream per device."""
        value = self._values["syncPolicy"]
        return "relaxed" if value == "auto" else value

    @property
    def profiling(self) -> bool:
        return bool(self._values["profile"] or self._values["cudaProfile"])

    @property
    def preferred_backend(self) -> str | None:
        return None if self._values["backend"] == "auto" else self._values["backend"]

    # -- introspection -----------------------------------------------------
    def asDict(self) -> dict[str, Any]:
        out = dict(self._values)
        out["resolvedTileLimit"] = self.resolvedTileLimit
        return out

    def keys(self) -> tuple[str, ...]:
        names = [_public(f) for f in _FIELDS]
        names.insert(names.index("scratch_pool") + 1, "scratch_policy")
        return tuple(names)

    def items(self) -> tuple[tuple[str, Any], ...]:
        return tuple((name, self.metadata(name)["current"]) for name in self.keys())

    def _field_of(self, name: str) -> str:
        field = _ALIASES.get(name)
        if field is None:
            raise ValueError(f"unknown MatrixMan configuration setting: {name}")
        return field

    def options(self, name: str) -> Any:
        return self.metadata(name)["options"]

    def metadata(self, name: str) -> dict[str, Any]:
        field = self._field_of(name)
        if field == "scratchPolicy":
            return {
                "name": "scratch_policy", "environment": None, "type": "str",
                "options": ("safe", "fresh", "epoch", "unsafe_reuse"), "default": "safe",
                "current": self.scratchPolicy_value(), "category": "Memory / texture reuse",
                "status": "diagnostic", "lifecycle": "may be changed before use",
                "description": "Effective scratch lifetime policy derived from the scratch debug flags.",
                "writable": False,
            }
        if field == "gpu_preference":
            field = "useDGPU"
        default, env, _alias, category, status, description = _FIELDS[field]
        public = _public(field)
        options: Any
        if field == "syncPolicy":
            options = _SYNC_POLICIES
        elif field in {"activationPool", "scratchPool"}:
            options = _POOLS
        elif field == "tileSync":
            options = _TILE_SYNCS
        elif field == "backend":
            options = _BACKENDS
        elif field == "convAlgo":
            options = _CONV_ALGOS
        elif field == "profile":
            options = ("off", "summary", "detail", "trace")
        elif field == "trace":
            options = (False, True, "detailed")
        elif field == "useDGPU":
            options = ("integrated", "discrete")
        elif field == "tileLimit":
            options = {"type": "int|string", "values": ("auto",), "range": "positive integer"}
        elif field in {"diagTileWidth", "diagTileHeight"}:
            options = {"type": "int|None", "range": "positive integer or None"}
        elif field in _BOOL_FIELDS:
            options = (False, True)
        else:
            options = {"type": type(default).__name__}
        if field == "profile":
            current = profile_mode()
            default = "off"
        elif field == "useDGPU":
            current = "discrete" if self._values["useDGPU"] else "integrated"
            default = "integrated"
        else:
            current = self._values[field]
        return {
            "name": public,
            "environment": env,
            "type": options["type"] if isinstance(options, dict) else (
                "bool" if field in _BOOL_FIELDS else type(default).__name__),
            "options": options,
            "default": default,
            "current": current,
            "description": description,
            "category": category,
            "lifecycle": ("set before backend initialization" if field in _RUNTIME_PROTECTED
                          else "may be changed before use"),
            "status": status,
            "writable": True,
        }

    def describe(self, name: str | None = None) -> str:
        names = (name,) if name is not None else self.keys()
        records = [self.metadata(n) for n in names]
        if name is None:
            records.sort(key=lambda r: (_CATEGORY_ORDER.index(r["category"]), r["name"]))
        lines: list[str] = []
        category = None
        for info in records:
            if name is None and info["category"] != category:
                if lines:
                    lines.append("")
                lines += [info["category"], "=" * len(info["category"]), ""]
                category = info["category"]
            lines += [info["name"], "-" * len(info["name"]), f"type: {info['type']}"]
            opts = info["options"]
            if isinstance(opts, dict):
                if "values" in opts:
                    lines.append(f"values: {' | '.join(map(str, opts['values']))}")
                if "range" in opts:
                    lines.append(f"range: {opts['range']}")
            else:
                lines.append(f"values: {' | '.join(map(str, opts))}")
            lines += [f"default: {info['default']}", f"current: {info['current']}",
                      f"category: {info['category']}", f"status: {info['status']}",
                      f"environment: {info['environment'] or 'none'}",
                      f"lifecycle: {info['lifecycle']}", f"description: {info['description']}"]
            if not info["writable"]:
                lines.append("writable: no (derived value)")
            lines.append("")
        text = "\n".join(lines).rstrip()
        print(text)
        return text

    def help(self, name: str | None = None) -> str:
        return self.describe(name)

    def source(self, name: str) -> str:
        field = self._field_of(name)
        if field == "gpu_preference":
            field = "useDGPU"
        if field == "scratchPolicy":
            srcs = [self._sources[f] for f in ("unsafeScratchReuse", "debugFreshScratch",
                                                "scratchEpochPool", "debugClearReusedScratch")]
            if "python override" in srcs:
                return "python override"
            return "environment" if "environment" in srcs else "default"
        return self._sources.get(field, "default")

    def show(self, *, as_text: bool = False) -> str | None:
        lines = ["MatrixMan configuration", "-----------------------"]
        for name in self.keys():
            info = self.metadata(name)
            value = info["current"]
            if isinstance(value, bool):
                value = str(value).lower()
            if value is None:
                value = "unset"
            lines.append(f"{name}: {value} [{self.source(name)}]")
        text = "\n".join(lines)
        if as_text:
            return text
        print(text)
        return None

    def __repr__(self) -> str:
        shown = ("backend", "tileLimit", "syncPolicy", "activationPool", "scratchPool",
                 "preparedExecution", "cudaGraphs", "convAlgo", "profile")
        return "MatrixManConfig(" + ", ".join(f"{n}={self._values[n]!r}" for n in shown) + ")"

    def __str__(self) -> str:
        return self.show(as_text=True) or ""


config = Configuration()


def profile_mode() -> str:
    value = config._values["profile"]
    if value is True:
        return "summary"
    if value in {False, None, "0", "off"}:
        return "off"
    return str(value)


def set_profiling(enabled: Any) -> bool:
    config._set("profile", enabled)
    return bool(config._values["profile"])


def set_trace(enabled: Any = True) -> Any:
    config._set("trace", enabled)
    return config._values["trace"]


def trace_enabled() -> bool:
    return config._values["trace"] in (True, "detailed")


def trace_log(message: str) -> None:
    if trace_enabled():
        print(message)


def set_preferred_backend(name: str) -> str:
    value = parse_value("backend", name)
    config._set("backend", value)
    return value


def preferred_backend() -> str | None:
    return config.preferred_backend
