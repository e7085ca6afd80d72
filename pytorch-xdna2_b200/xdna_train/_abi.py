"""ctypes view of the C ABI in ``include/b2.h`` (``libxdna_b200.so``).

The PyTorch extension calls the library directly from C++; this module is the
binding a Python host without the extension (or a test) uses, and the model
for a cgo / JNI / N-API binding of the same library.  Every function takes
plain integers for device pointers and the CUDA stream.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB = None
LIB_PATH = Path(__file__).resolve().parent / "libxdna_b200.so"

B2_OK, B2_BF16, B2_F32 = 0, 0, 1

i32, i64, f32, f64, vp, sz = C.c_int, C.c_int64, C.c_float, C.c_double, C.c_void_p, C.c_size_t


class AdamTensor(C.Structure):
    _fields_ = [("param", vp), ("grad", vp), ("exp_avg", vp), ("exp_avg_sq", vp),
                ("max_exp_avg_sq", vp), ("step", vp), ("numel", i64)]


class AdamHparams(C.Structure):
    _fields_ = [("lr", f64), ("beta1", f64), ("beta2", f64), ("weight_decay", f64), ("eps", f64),
                ("amsgrad", i32), ("maximize", i32), ("adamw", i32), ("param_dtype", i32),
                ("state_dtype", i32), ("lr_tensor", vp), ("grad_scale", vp), ("found_inf", vp)]


class SgdTensor(C.Structure):
    _fields_ = [("param", vp), ("grad", vp), ("momentum_buffer", vp), ("numel", i64)]


class SgdHparams(C.Structure):
    _fields_ = [("lr", f64), ("weight_decay", f64), ("momentum", f64), ("dampening", f64),
                ("nesterov", i32), ("maximize", i32), ("is_first_step", i32), ("param_dtype", i32),
                ("lr_tensor", vp), ("grad_scale", vp), ("found_inf", vp)]


# name -> argument types (restype is int unless listed in _RESTYPES)
SIGNATURES = {
    "b2_last_error": [],
    "b2_abi_version": [],
    "b2_device_status": [i32, C.POINTER(i32)],
    "b2_pack_rows_bf16": [vp, i64, i64, i64, i64, i32, i32, i32, i32, i32, vp, vp],
    "b2_pack_rows_dbias_workspace_bytes": [i32, i32, i32, i32],
    "b2_pack_rows_dbias_bf16": [vp, i64, i64, i64, i64, i32, i32, i32, i32, i32, vp, vp, i32, vp, sz, vp],
    "b2_channel_sum_nhwc_workspace_bytes": [i32, i32, i32, i32],
    "b2_channel_sum_nhwc_bf16": [vp, i64, i64, i64, i32, i32, i32, i32, vp, i32, vp, sz, vp],
    "b2_pack_weight_fwd_bf16": [vp, i32, i32, i32, vp, vp],
    "b2_pack_weight_dgrad_bf16": [vp, i32, i32, i32, vp, vp],
    "b2_pack_weight_strided_bf16": [vp, vp, i32, i32, i32, i32, vp, vp],
    "b2_nchw_to_nhwc_bf16": [vp, vp, i32, i32, i32, vp],
    "b2_nhwc_to_nchw_bf16": [vp, vp, i32, i32, i32, vp],
    "b2_conv3x3_fwd": [vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, vp],
    "b2_conv3x3_dgrad": [vp, vp, vp, i64, i64, i64, i64, i32, i32, i32, i32, i32, vp],
    "b2_conv3x3_wgrad_workspace_bytes": [i32, i32, i32, i32, i32],
    "b2_conv3x3_wgrad": [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, sz, vp],
    "b2_conv3x3_wgrad_noalloc": [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp],
    "b2_conv3x3_fwd_nhwc": [vp, i64, i64, i64, vp, vp, vp, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, vp],
    "b2_conv3x3_dgrad_nhwc": [vp, i64, i64, i64, vp, vp, i64, i64, i64, i64, i32, i32, i32, i32, i32, vp],
    "b2_conv3x3_wgrad_nhwc": [vp, i64, i64, i64, vp, i64, i64, i64, vp, i32, i32, i32, i32, i32, i32, vp, sz, vp],
    "b2_conv3x3_wgrad_nhwc_ohwi": [vp, i64, i64, i64, vp, i64, i64, i64, vp, i32, i32, i32, i32, i32, i32, vp, sz,
                                   vp],
    "b2_conv3x3_wgrad_noalloc_max_bytes": [],
    "b2_gemm_bf16": [i32, i32, i32, i32, i32, f32, vp, i64, i64, vp, i64, i64, f32, vp, i32,
                     i64, i64, i64, vp, i64, i64, i32, vp],
    "b2_gemm_bf16_workspace_bytes": [i32, i32, i32, i32],
    "b2_gemm_bf16_ws": [i32, i32, i32, i32, i32, f32, vp, i64, i64, vp, i64, i64, f32, vp, i32,
                        i64, i64, i64, vp, i64, i64, i32, vp, sz, vp],
    "b2_fused_adam": [C.POINTER(AdamTensor), i32, C.POINTER(AdamHparams), vp],
    "b2_fused_sgd": [C.POINTER(SgdTensor), i32, C.POINTER(SgdHparams), vp],
    "b2_region_sqdiff_sum_bf16": [vp, vp, i64, vp, vp],
    "b2_region_relu_bf16": [vp, vp, i64, vp],
    "b2_region_relu_maxpool2_bf16": [vp, vp, vp, i64, i64, i64, vp],
    "b2_region_addtap_bf16": [vp, vp, vp, vp, i64, f32, vp],
    "b2_region_relu_bwd_bf16": [vp, vp, vp, vp, vp, i64, f32, vp],
    "b2_region_maxpool2_bwd_bf16": [vp, vp, vp, i64, i64, i64, vp],
    "b2_conv1x1_fwd": [vp, vp, vp, vp, i32, i64, i64, i64, i64, vp],
    "b2_conv1x1_dgrad": [vp, vp, vp, i32, i64, i64, i64, i64, vp],
    "b2_conv1x1_wgrad_workspace_bytes": [i32, i64, i64, i64, i64],
    "b2_conv1x1_wgrad": [vp, vp, vp, i32, i32, i64, i64, i64, i64, vp, sz, vp],
    "b2_gemm_splitk_workspace_bytes": [i32, i32, i32, i32],
    "b2_gemm_splitk_bf16": [i32, i32, i32, i32, i32, vp, i64, vp, i64, vp, i32, i64, vp, sz, vp],
    "b2_im2col_bf16": [vp, i64, i64, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32, i32, i64, i64,
                       i64, vp, vp],
    "b2_col2im_bf16": [vp, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32, i32, i64, i64, vp, i64, i64,
                       i64, i64, vp],
    "b2_pack_weight_khwc_bf16": [vp, i64, i64, i32, i32, i64, vp, vp],
    "b2_unpack_weight_khwc": [vp, i64, i64, i32, i32, i64, vp, i32, vp],
    "b2_batch_norm_stats_bf16": [vp, i32, i32, vp, vp, i32, vp, vp, i64, i64, i64, f32, f32, vp, sz, vp],
    "b2_batch_norm_stats_count_bf16": [vp, i32, i32, vp, vp, i32, vp, vp, i64, i64, i64, f32, f32, vp, i64, vp, sz,
                                       vp],
    "b2_batch_norm_apply_bf16": [vp, i32, vp, vp, i32, vp, vp, vp, i32, vp, i64, i64, i64, vp],
    "b2_direct_conv_weight_floats": [i64, i64, i32, i32, i32],
    "b2_direct_conv_weight": [vp, i64, i64, i32, i32, i32, vp, vp],
    "b2_direct_conv_bf16": [vp, vp, i64, i64, i64, i64, vp, i32, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, i64,
                            i64, i64, vp],
    "b2_maxpool2d_fwd": [vp, vp, vp, vp, vp, i32, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32,
                         i32, vp],
    "b2_maxpool2d_bwd": [vp, vp, vp, vp, vp, i32, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32,
                         i32, vp],
    "b2_maxpool2d_fwd_taps": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32, i32, vp],
    "b2_maxpool2d_taps_to_indices": [vp, vp, vp, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32, i32, vp],
    "b2_maxpool2d_bwd_taps": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32, i32, vp],
    "b2_cat_blocks": [vp, vp, i32, vp, i64, i64, vp],
    "b2_upsample_nearest2x": [vp, vp, i32, i32, i64, i64, i64, i64, vp],
    "b2_upsample_nearest2x_backward": [vp, vp, i32, i32, i64, i64, i64, i64, vp],
    "b2_region_bn_workspace_bytes": [i64, i64],
    "b2_batch_norm_workspace_bytes": [i64, i64, i64, i32],
    "b2_batch_norm_fwd_bf16": [vp, i32, vp, vp, i32, vp, vp, i32, vp, vp, vp, i64, i64, i64, f32, f32, vp, sz, vp],
    "b2_batch_norm_bwd_bf16": [vp, vp, i32, vp, i32, vp, vp, vp, vp, vp, i32, i64, i64, i64, vp, sz, vp],
    "b2_batch_norm_relu_bwd_bf16": [vp, vp, vp, vp, i32, vp, vp, vp, vp, vp, i32, i64, i64, i64, vp, sz, vp],
    "b2_relu_bwd_sum_bf16": [vp, vp, vp, vp, i64, vp],
    "b2_batch_norm_bwd_relu_sum_bf16": [vp, vp, vp, vp, vp, i32, vp, vp, vp, vp, vp, vp, i32, i64, i64, i64, vp, sz,
                                        vp],
    "b2_region_bn_fwd_bf16": [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, f32, f32, i32, vp, sz, vp],
    "b2_region_bn_bwd_bf16": [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, i32, vp, sz, vp],
}
_RESTYPES = {"b2_last_error": C.c_char_p, "b2_conv3x3_wgrad_workspace_bytes": sz,
             "b2_pack_rows_dbias_workspace_bytes": sz, "b2_region_bn_workspace_bytes": sz,
             "b2_conv1x1_wgrad_workspace_bytes": sz, "b2_direct_conv_weight_floats": sz, "b2_gemm_splitk_workspace_bytes": sz,
             "b2_batch_norm_workspace_bytes": sz, "b2_channel_sum_nhwc_workspace_bytes": sz,
             "b2_gemm_bf16_workspace_bytes": sz,
             "b2_conv3x3_wgrad_noalloc_max_bytes": sz}


class B2Error(RuntimeError):
    pass


def lib():
    """Load the library (raises if it was not built: there is no fallback)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.is_file():
            raise B2Error(f"{LIB_PATH} is missing; build it with `python -m xdna_train._build`")
        L = C.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, i32)
        _LIB = L
    return _LIB


def check(status: int, what: str = "") -> None:
    if status != B2_OK:
        msg = lib().b2_last_error().decode(errors="replace")
        raise B2Error(f"{what or 'b2 call'} failed with status {status}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
