"""Registration of the ``xdna`` device and the package's Python API.

Same surface as the reference's ``xdna_train/device.py`` (register 225-352,
device module 53-97, param swap 355-405, optimizer hooks 408-452, stats
648-795), on NVIDIA B200: ``xdna:i`` is CUDA device ``i`` driven through the
PrivateUse1 dispatch key, with the hot ops on the sm_100a kernels of
``libxdna_b200.so``.  The NPU-compiler machinery of the reference (IRON stream
builds, artifact families, the step autotuner) has no counterpart: kernels are
compiled ahead of time, so ``wait_for_builds`` returns at once and
``autotune_result`` reports the fixed mode.
"""
from __future__ import annotations

import functools
import os
import warnings
from pathlib import Path
from types import SimpleNamespace

import torch

_INITIALIZED = False
_C = None

_REMOVED_ENV_VARS = (  # NPU-only knobs of the reference; they have no effect here
    "XDNA_CONV3X3W", "XDNA_CONV3X3W_DW", "XDNA_CONV3X3W_MIN_MACS", "XDNA_CONV3X3W_FORCE",
    "XDNA_CONV3X3W_WEIGHT_CACHE", "XDNA_CONV3X3W_PIECES", "XDNA_CONV3X3W_SYNC_BUILD",
    "XDNA_ZERO_COPY_FALLBACK",
)


def _load_native():
    """Import the prebuilt extension.  There is no CPU fallback: a missing build
    is an error (build with ``python -m xdna_train._build``)."""
    global _C
    if _C is None:
        try:
            from . import _C as native  # noqa: N813
        except ImportError as e:
            raise RuntimeError(
                f"xdna_train native extension not built ({e}); run `python -m xdna_train._build`") from e
        _C = native
    return _C


def _device_index(device=None, optional: bool = False) -> int:
    del optional
    if device is None:
        return torch.cuda.current_device() if torch.cuda.is_available() else 0
    if isinstance(device, int):
        return device
    d = torch.device(device)
    if d.type not in ("xdna", "cuda"):
        raise ValueError(f"expected an xdna device, got {d}")
    return torch.cuda.current_device() if d.index is None else d.index


class _DeviceContext:
    """``with torch.xdna.device(i):`` -- torch.load and similar code enter it."""

    def __init__(self, device):
        self.index = _device_index(device)
        self.prev = 0

    def __enter__(self):
        self.prev = int(_C.current_device())
        _C.set_device(self.index)
        return self

    def __exit__(self, *exc):
        _C.set_device(self.prev)
        return False


class _XdnaDeviceModule:
    _utils = SimpleNamespace(_get_device_index=_device_index)
    device = _DeviceContext

    @staticmethod
    def is_available() -> bool:
        return bool(_C.is_available())

    @staticmethod
    def is_initialized() -> bool:
        return bool(_C.is_available())

    @staticmethod
    def device_count() -> int:
        return int(_C.device_count())

    @staticmethod
    def current_device() -> int:
        return int(_C.current_device())

    @staticmethod
    def set_device(device) -> None:
        _C.set_device(_device_index(device))

    @staticmethod
    def synchronize(device=None) -> None:
        _C.synchronize(-1 if device is None else _device_index(device))

    @staticmethod
    def empty_cache() -> None:
        _C.empty_cache()

    @staticmethod
    def memory_stats() -> dict[str, int]:
        return dict(_C.allocator_stats())

    @staticmethod
    def memory_allocated(device=None) -> int:
        return int(_C.allocator_stats()["allocated_bytes"])

    @staticmethod
    def get_amp_supported_dtype():
        return [torch.bfloat16, torch.float32]

    @staticmethod
    def _is_in_bad_fork() -> bool:
        return False

    @staticmethod
    def manual_seed(seed: int) -> None:
        torch.cuda.manual_seed(seed)

    @staticmethod
    def manual_seed_all(seed: int) -> None:
        torch.cuda.manual_seed_all(seed)

    @staticmethod
    def current_stream(device=None):
        return torch.cuda.current_stream(_device_index(device))


def register_xdna_device() -> None:
    """Register ``torch.device("xdna")`` (idempotent).  Import side effects are
    the reference's (device.py:225-352): PrivateUse1 renamed to ``xdna``, the
    ``torch.xdna`` module, tensor/module ``.xdna()`` methods, BF16 as the
    default autocast dtype, Parameter-preserving ``Module.to("xdna")``, backward
    on the calling thread, and the fused-optimizer pre/post hooks."""
    global _INITIALIZED
    if _INITIALIZED:
        return
    removed = [n for n in _REMOVED_ENV_VARS if n in os.environ]
    if removed:
        warnings.warn(f"{', '.join(removed)} has no effect on the B200 backend", RuntimeWarning, stacklevel=2)
    _load_native()
    current = torch._C._get_privateuse1_backend_name()
    if current == "privateuseone":
        torch.utils.rename_privateuse1_backend("xdna")
    elif current != "xdna":
        raise RuntimeError(f"PrivateUse1 is already claimed by backend {current!r}; xdna cannot coexist with it")
    # Backward on the calling thread, as the reference does (device.py:254-261);
    # XDNA_AUTOGRAD_THREAD=1 keeps PyTorch's per-device worker thread.
    if os.environ.get("XDNA_AUTOGRAD_THREAD", "0") != "1":
        torch.autograd.set_multithreading_enabled(False)
    if not hasattr(torch, "xdna"):
        torch._register_device_module("xdna", _XdnaDeviceModule)
    if not hasattr(torch.Tensor, "xdna"):
        torch.utils.generate_methods_for_privateuse1_backend(for_tensor=True, for_module=True, for_storage=False)
    torch.set_autocast_dtype("xdna", torch.bfloat16)
    _install_scoped_param_swap()
    from torch.optim.optimizer import register_optimizer_step_post_hook, register_optimizer_step_pre_hook

    register_optimizer_step_post_hook(_bump_fused_param_versions)
    if os.environ.get("XDNA_FUSED_OPTIMIZER", "1") == "1":
        register_optimizer_step_pre_hook(_prefer_fused_optimizer)
    _INITIALIZED = True


class _SwapModuleParams:
    """Keep Parameter identity across ``Module.to("xdna")`` (device.py:355-405):
    PyTorch swaps tensors in place only for backends it knows, so without this an
    optimizer built before the move would keep updating the old tensors."""

    def __enter__(self):
        self.prev = torch.__future__.get_swap_module_params_on_conversion()
        torch.__future__.set_swap_module_params_on_conversion(True)

    def __exit__(self, *exc):
        torch.__future__.set_swap_module_params_on_conversion(self.prev)


def _install_scoped_param_swap() -> None:
    module = torch.nn.Module
    if getattr(module.to, "_xdna_scoped_swap", False):
        return

    def is_xdna(device) -> bool:
        return device is not None and torch.device(device).type == "xdna"

    def scoped(fn, targets_xdna):
        @functools.wraps(fn)
        def wrapper(self, *args, **kwargs):
            if not targets_xdna(*args, **kwargs):
                return fn(self, *args, **kwargs)
            with _SwapModuleParams():
                return fn(self, *args, **kwargs)

        wrapper._xdna_scoped_swap = True
        return wrapper

    def to_targets(*args, **kwargs):
        try:
            device = torch._C._nn._parse_to(*args, **kwargs)[0]
        except Exception:
            return False
        return is_xdna(device)

    module.to = scoped(module.to, to_targets)
    module.to_empty = scoped(module.to_empty, lambda *, device=None, **k: is_xdna(device))
    if hasattr(module, "xdna"):
        module.xdna = scoped(module.xdna, lambda *a, **k: True)


def _prefer_fused_optimizer(optimizer, args, kwargs) -> None:
    """Default xdna optimizers to the fused kernels (device.py:408-436): one
    multi-tensor launch instead of ~10 foreach list ops.  Only groups that left
    both ``fused`` and ``foreach`` unset, hold only xdna floating-point params
    and have no state yet are changed."""
    if getattr(optimizer, "_xdna_fused_checked", False):
        return
    optimizer._xdna_fused_checked = True
    for group in optimizer.param_groups:
        if ("fused" not in group or group.get("fused") is not None or group.get("foreach") is not None
                or group.get("differentiable")):
            continue
        params = group["params"]
        if params and all(p.device.type == "xdna" and p.is_floating_point() and not optimizer.state.get(p)
                          for p in params):
            group["fused"] = True


def _bump_fused_param_versions(optimizer, args, kwargs) -> None:
    """Mark parameters written by a fused optimizer step as modified
    (device.py:439-452).  The C++ kernel bumps them too; this keeps the
    reference's hook for fused kernels reached another way."""
    for group in optimizer.param_groups:
        if not group.get("fused"):
            continue
        params = [p for p in group["params"] if p.device.type == "xdna"]
        if params:
            torch.autograd.graph.increment_version(params)


def try_register_xdna_device() -> bool:
    """Register if possible (called on import); warn with the cause otherwise."""
    try:
        register_xdna_device()
    except (ImportError, RuntimeError, OSError) as e:
        warnings.warn(f"xdna_train: xdna device not registered: {type(e).__name__}: {e}", RuntimeWarning,
                      stacklevel=2)
        return False
    return True


def is_available() -> bool:
    try:
        register_xdna_device()
    except (ImportError, RuntimeError, OSError):
        return False
    return _XdnaDeviceModule.is_available()


def synchronize(device=None) -> None:
    register_xdna_device()
    _XdnaDeviceModule.synchronize(device)


def empty_cache() -> None:
    register_xdna_device()
    _C.empty_cache()


def allocator_stats() -> dict[str, int]:
    register_xdna_device()
    return dict(_C.allocator_stats())


def async_dw_stats() -> dict:
    """Deferred weight-gradient state: pending / deferred / started / dropped
    jobs, early launches (kicks) and the learned dX calls per step."""
    register_xdna_device()
    return dict(_C.async_dw_stats())


def kernel_stats() -> dict[str, int]:
    """Launches of the native kernels per kind since the last reset."""
    register_xdna_device()
    return dict(_C.launch_stats())


def kernel_timer(on: bool = True) -> None:
    """Turn per-launch device timing on or off: while on, the timed launch
    sites (3x3 / 1x1 convolutions, GEMMs) record a CUDA event pair around each
    launch on its stream, with the launch's algorithmic FLOPs."""
    register_xdna_device()
    _C.kernel_timer_enable(bool(on))


def kernel_times() -> dict[str, dict[str, float]]:
    """Per label: launches, summed device milliseconds and summed algorithmic
    work (FLOPs) of the launches timed since the last read (waits for them)."""
    register_xdna_device()
    return {str(k): dict(v) for k, v in dict(_C.kernel_timer_read()).items()}


def reset_mapped_cpu_stats() -> None:
    register_xdna_device()
    _C.reset_stats()


def mapped_cpu_stats() -> dict[str, dict[str, float | int]]:
    """Per-kernel call counters (the reference's per-op host timers,
    device.py:713-727; device time is measured with CUDA events instead)."""
    register_xdna_device()
    return {str(k): {"calls": int(v), "total_ms": 0.0, "avg_ms": 0.0} for k, v in _C.launch_stats().items()}


def reset_fallback_stats() -> None:
    register_xdna_device()
    _C.reset_stats()


def fallback_stats() -> dict[str, dict[str, float | int]]:
    """Ops that ran ATen's CUDA kernels on aliases instead of a native kernel."""
    register_xdna_device()
    return {str(k): dict(v) for k, v in dict(_C.fallback_stats()).items()}


def set_npu_mode(mode: int) -> None:
    """2: all native kernels, 1: weight gradients through ATen's CUDA path,
    0: every hot op through ATen's CUDA path (A/B switch; same API as the
    reference, device.py:654-660)."""
    register_xdna_device()
    _C.set_npu_mode(int(mode))


def npu_mode() -> int:
    register_xdna_device()
    return int(_C.npu_mode())


def set_conv_paths(conv1x1=None, general=None):
    """Route the convolutions outside the 3x3 fast path (no counterpart in the
    reference, whose other convolutions all run on its CPU path):
    ``conv1x1`` -- 1x1 / stride 1 convolutions as tcgen05 GEMMs;
    ``general`` -- stems and large kernels as GEMMs over a column matrix.
    ``general`` defaults on (ResNet-50's 7x7 stem: 0.95 ms a step against
    1.17 ms in ATen's library kernels), ``conv1x1`` off (ATen's library
    kernels are still faster on ResNet-50's 1x1 layers).  ``None`` leaves a
    setting as it is.  Returns the
    settings (also ``XDNA_CONV1X1`` / ``XDNA_CONV_GENERAL`` = 0/1 at
    start-up)."""
    register_xdna_device()
    return tuple(bool(v) for v in _C.set_conv_paths(conv1x1, general))


def set_fusion(bn_epilogue=None) -> bool:
    """Fold a residual ``add_`` and a ``relu_`` that follow a training-mode
    BatchNorm on its output tensor into BatchNorm's output pass (the pass
    waits for the output's first reader, like a deferred weight gradient; a
    write into a tensor it reads runs it first).  On by default
    (``XDNA_BN_EPILOGUE=0`` at start-up turns it off); ``None`` leaves it as
    it is.  Returns the previous setting."""
    register_xdna_device()
    if bn_epilogue is None:
        return bool(_C.bn_epilogue())
    return bool(_C.set_bn_epilogue(bool(bn_epilogue)))


def wait_for_builds(timeout: float | None = None) -> bool:
    """Kernels are compiled ahead of time; nothing to wait for."""
    del timeout
    return True


def autotune_result() -> dict | None:
    """The reference's step autotuner picks an NPU mode; on B200 the mode is
    fixed (native kernels), reported in the same shape."""
    register_xdna_device()
    return {"mode": npu_mode(), "step_ms": {}}


def native_library_path() -> Path:
    register_xdna_device()
    return Path(_C.__file__).resolve()


def kernel_library_path() -> Path:
    return Path(__file__).resolve().parent / "libxdna_b200.so"


def is_xrt_backed(tensor: torch.Tensor) -> bool:
    """True for tensors whose storage is xdna device memory."""
    return tensor.device.type == "xdna"


def bo_handle(tensor: torch.Tensor) -> int:
    """Device address of the tensor's storage (the reference returned its XRT BO)."""
    register_xdna_device()
    return int(tensor.untyped_storage().data_ptr())


def coherency_state(tensor: torch.Tensor) -> int:
    """Always 0 (clean): device memory has a single copy, no host mirror."""
    del tensor
    return 0


def materialize(tensor: torch.Tensor) -> None:
    """Enqueue the deferred weight gradient of ``tensor`` now, if it has one."""
    register_xdna_device()
    _C.materialize(tensor)


def as_cuda(tensor: torch.Tensor) -> torch.Tensor:
    """Zero-copy CUDA view of an xdna tensor (for NCCL collectives)."""
    register_xdna_device()
    return _C.as_cuda(tensor)


def device_status(device: int = 0) -> int:
    """Reads and clears the device-side error word (0 = no kernel gave up)."""
    register_xdna_device()
    return int(_C.device_status(device))
