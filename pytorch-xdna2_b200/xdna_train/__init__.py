"""torch-xdna2's device backend, rebuilt for NVIDIA B200 (sm_100a).

Importing the package registers ``torch.device("xdna")`` (same side effects as
the reference's ``xdna_train/__init__.py``); ``xdna:i`` is CUDA device ``i``.
"""

from .device import (
    allocator_stats,
    as_cuda,
    async_dw_stats,
    autotune_result,
    bo_handle,
    coherency_state,
    device_status,
    empty_cache,
    fallback_stats,
    is_available,
    is_xrt_backed,
    kernel_library_path,
    kernel_stats,
    kernel_timer,
    kernel_times,
    mapped_cpu_stats,
    materialize,
    native_library_path,
    npu_mode,
    register_xdna_device,
    reset_fallback_stats,
    reset_mapped_cpu_stats,
    set_npu_mode,
    set_conv_paths,
    set_fusion,
    synchronize,
    try_register_xdna_device,
    wait_for_builds,
)

__version__ = "0.1.0"

try_register_xdna_device()

__all__ = [
    "__version__",
    "register_xdna_device",
    "try_register_xdna_device",
    "is_available",
    "synchronize",
    "empty_cache",
    "allocator_stats",
    "async_dw_stats",
    "autotune_result",
    "set_npu_mode",
    "set_conv_paths",
    "set_fusion",
    "npu_mode",
    "wait_for_builds",
    "reset_fallback_stats",
    "fallback_stats",
    "mapped_cpu_stats",
    "reset_mapped_cpu_stats",
    "kernel_stats",
    "kernel_timer",
    "kernel_times",
    "native_library_path",
    "kernel_library_path",
    "is_xrt_backed",
    "bo_handle",
    "coherency_state",
    "materialize",
    "as_cuda",
    "device_status",
]
