"""Python face of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, as the checker; the product path (the ``xdna`` device and
``libxdna_b200.so``) never does.

* ``native()``   -- ctypes handle on ``_build/liboracle.so`` (b2_oracle.c, the
  C restatement of the reference's packing / conv-on-rows / wgrad / region /
  Adam algorithms, each function citing its reference file:line).
* ``reference()``-- ctypes handle on ``_ref/libxdna_ref.so``: the reference's
  own ``conv_pack.cpp`` and ``region_kernels.cpp`` compiled from their sources
  (``make -C oracle``), or None where the reference tree was never present.
* numpy wrappers below take and return bf16 bit patterns as ``np.uint16``.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libxdna_ref.so"

_native = None
_ref = None

u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
i32, i64, f32, f64, vp = C.c_int, C.c_int64, C.c_float, C.c_double, C.c_void_p


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def native():
    global _native
    if _native is None:
        if not LIB.is_file():
            build()
        L = C.CDLL(str(LIB))
        L.oracle_pack_rows.argtypes = [u16p, i32, i32, i32, i32, i32, u16p]
        L.oracle_pack_weight.argtypes = [u16p, i32, i32, i32, i32, u16p]
        L.oracle_conv_rows.argtypes = [u16p, u16p, vp, i32, i32, i32, i32, i32, i32, f32p]
        L.oracle_wgrad_rows.argtypes = [u16p, u16p, i32, i32, i32, i32, i32, f32p]
        L.oracle_gemm.argtypes = [u16p, u16p, vp, i32, i32, i32, f32, f32, f32p]
        L.oracle_sqdiff_sum.argtypes = [u16p, u16p, i64]
        L.oracle_sqdiff_sum.restype = f64
        L.oracle_relu.argtypes = [u16p, u16p, i64]
        L.oracle_relu_maxpool2.argtypes = [u16p, u16p, u16p, i64, i64, i64]
        L.oracle_addtap.argtypes = [vp, u16p, u16p, u16p, i64, f32]
        L.oracle_relu_bwd.argtypes = [u16p, vp, vp, vp, u16p, i64, f32]
        L.oracle_maxpool2_bwd.argtypes = [u16p, u16p, u16p, i64, i64, i64]
        L.oracle_adam_f32.argtypes = [f32p, f32p, f32p, f32p, f32p, i64, f32, f32, f32, f32, f32, f32,
                                      i32, i32, i32]
        L.oracle_bn_fwd.argtypes = [u16p, vp, vp, vp, vp, u16p, f32p, f32p, i64, i64, i64, f32, f32, f32, i32]
        L.oracle_bn_bwd.argtypes = [u16p, u16p, u16p, vp, f32p, f32p, vp, vp, vp, i64, i64, i64, f32, i32]
        _native = L
    return _native


def reference():
    """The reference's own host kernels (None if they were never built here)."""
    global _ref
    if _ref is None and REF_LIB.is_file():
        L = C.CDLL(str(REF_LIB))
        L.xdna_conv3x3w_pack_input_bf16.argtypes = [u16p, u16p, i32, i32, i32, i32, i32]
        L.xdna_region_sqdiff_sum_bf16.argtypes = [u16p, u16p, i64, i32]
        L.xdna_region_sqdiff_sum_bf16.restype = f64
        L.xdna_region_relu_bf16.argtypes = [u16p, u16p, i64, i32]
        L.xdna_region_relu_maxpool2_bf16.argtypes = [u16p, u16p, u16p, i64, i64, i64, i32]
        L.xdna_region_addtap_bf16.argtypes = [vp, u16p, u16p, u16p, i64, f32, i32]
        L.xdna_region_relu_bwd_bf16.argtypes = [u16p, vp, vp, vp, u16p, i64, f32, i32]
        L.xdna_region_maxpool2_bwd_bf16.argtypes = [u16p, u16p, u16p, i64, i64, i64, i32]
        L.xdna_region_bn_fwd_bf16.argtypes = [u16p, vp, vp, vp, vp, u16p, f32p, f32p, i64, i64, i64, f32, f32,
                                              f32, i32, i32]
        L.xdna_region_bn_bwd_bf16.argtypes = [u16p, u16p, u16p, vp, f32p, f32p, vp, vp, vp, i64, i64, i64, f32,
                                              i32, i32]
        _ref = L
    return _ref


def _ptr(a):
    return None if a is None else a.ctypes.data_as(vp)


# ---- bf16 helpers -----------------------------------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (conv3x3w_host.py:22-25)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits).astype(np.uint32) << 16).view(np.float32)


# ---- wrappers ----------------------------------------------------------------

def pack_rows(x_bits: np.ndarray, chunks: int | None = None) -> np.ndarray:
    B, Cc, H, W = x_bits.shape
    chunks = chunks or -(-Cc // 64)
    rows = np.empty((B * (H + 2) * (W + 2), chunks * 64), np.uint16)
    native().oracle_pack_rows(np.ascontiguousarray(x_bits), B, Cc, H, W, chunks, rows)
    return rows


def pack_weight(w_bits: np.ndarray, dgrad: bool = False, chunks: int | None = None) -> np.ndarray:
    Cout, Cin = w_bits.shape[:2]
    kred = Cout if dgrad else Cin
    chunks = chunks or -(-kred // 64)
    wk = np.empty(((Cin if dgrad else Cout), chunks * 576), np.uint16)
    native().oracle_pack_weight(np.ascontiguousarray(w_bits), Cout, Cin, chunks, int(dgrad), wk)
    return wk


def conv_fwd(x_bits, w_bits, bias_bits=None, relu=False) -> np.ndarray:
    """y = conv3x3(x, w) + b as float32 NCHW, computed on packed rows."""
    B, Cin, H, W = x_bits.shape
    Cout = w_bits.shape[0]
    rows = pack_rows(x_bits)
    wk = pack_weight(w_bits)
    y = np.empty((B, Cout, H, W), np.float32)
    b = None if bias_bits is None else np.ascontiguousarray(bias_bits, dtype=np.uint16)
    native().oracle_conv_rows(rows, wk, _ptr(b), B, Cin, H, W, Cout, int(relu), y)
    return y


def conv_dgrad(dy_bits, w_bits) -> np.ndarray:
    B, Cout, H, W = dy_bits.shape
    Cin = w_bits.shape[1]
    rows = pack_rows(dy_bits)
    wk = pack_weight(w_bits, dgrad=True)
    dx = np.empty((B, Cin, H, W), np.float32)
    native().oracle_conv_rows(rows, wk, None, B, Cout, H, W, Cin, 0, dx)
    return dx


def conv_wgrad(dy_bits, x_bits) -> np.ndarray:
    B, Cout, H, W = dy_bits.shape
    Cin = x_bits.shape[1]
    dw = np.empty((Cout, Cin, 3, 3), np.float32)
    native().oracle_wgrad_rows(pack_rows(dy_bits), pack_rows(x_bits), B, Cin, H, W, Cout, dw)
    return dw


def gemm(a_bits, b_bits, c=None, alpha=1.0, beta=0.0) -> np.ndarray:
    M, K = a_bits.shape
    N = b_bits.shape[1]
    d = np.empty((M, N), np.float32)
    cc = None if c is None else np.ascontiguousarray(c, dtype=np.float32)
    native().oracle_gemm(np.ascontiguousarray(a_bits), np.ascontiguousarray(b_bits), _ptr(cc), M, N, K,
                         alpha, beta, d)
    return d


def sqdiff_sum(a, b) -> float:
    return native().oracle_sqdiff_sum(np.ascontiguousarray(a), np.ascontiguousarray(b), a.size)


def relu(a):
    r = np.empty_like(a)
    native().oracle_relu(np.ascontiguousarray(a), r, a.size)
    return r


def relu_maxpool2(a):
    planes = int(np.prod(a.shape[:-2]))
    H, W = a.shape[-2:]
    r = np.empty_like(a)
    p = np.empty(a.shape[:-2] + (H // 2, W // 2), np.uint16)
    native().oracle_relu_maxpool2(np.ascontiguousarray(a), r, p, planes, H, W)
    return r, p


def addtap(base, a, b, scale):
    out = np.empty_like(a)
    bb = None if base is None else np.ascontiguousarray(base)
    native().oracle_addtap(_ptr(bb), np.ascontiguousarray(a), np.ascontiguousarray(b), out, a.size, scale)
    return out


def relu_bwd(r, base, a, b, scale):
    out = np.empty_like(r)
    args = [None if t is None else np.ascontiguousarray(t) for t in (base, a, b)]
    native().oracle_relu_bwd(np.ascontiguousarray(r), *[_ptr(t) for t in args], out, r.size, scale)
    return out


def maxpool2_bwd(x, g):
    planes = int(np.prod(x.shape[:-2]))
    H, W = x.shape[-2:]
    out = np.empty_like(x)
    native().oracle_maxpool2_bwd(np.ascontiguousarray(x), np.ascontiguousarray(g), out, planes, H, W)
    return out


def adam_f32(p, g, m, v, vmax, step, lr, beta1, beta2, wd, eps, amsgrad=False, maximize=False, adamw=False):
    """In-place on float32 arrays."""
    native().oracle_adam_f32(p, g, m, v, vmax, p.size, step, lr, beta1, beta2, wd, eps, int(amsgrad),
                             int(maximize), int(adamw))


def sgd_step(p, g, buf, lr, weight_decay=0.0, momentum=0.0, dampening=0.0, nesterov=False, maximize=False,
             first_step=False, grad_scale=None, bf16=False):
    """One fused-SGD step, the update torch.optim.SGD(fused=True) issues as
    aten::_fused_sgd_ (the op the reference's _prefer_fused_optimizer selects,
    xdna_train/device.py:408-436, and runs on its CPU through the boxed
    fallback, torch_xdna_device.cpp:5124-5260), restated in numpy: fp32
    operands, hyper-parameters in double, each intermediate rounded where the
    fused definition stores it.  Arrays hold float32 values, or bf16 bit
    patterns (np.uint16) with ``bf16``; returns new (p, g, buf) in the same
    form (g changes only with ``grad_scale``; buf is None without momentum)."""
    dec = (lambda a: bf16_value(a)) if bf16 else (lambda a: np.asarray(a, dtype=np.float32))
    enc = (lambda a: bf16_bits(a.astype(np.float32))) if bf16 else (lambda a: a.astype(np.float32))
    pf, gf = dec(p), dec(g)
    if grad_scale is not None:
        gf = (gf.astype(np.float64) / np.float64(np.float32(grad_scale))).astype(np.float32)
    g_out = enc(gf) if grad_scale is not None else g
    gg = -gf if maximize else gf
    if weight_decay != 0.0:
        gg = (gg.astype(np.float64) + weight_decay * pf.astype(np.float64)).astype(np.float32)
    b_out = None
    if momentum != 0.0:
        if first_step:
            bd = gg.astype(np.float64)
        else:
            bd = momentum * dec(buf).astype(np.float64) + (1.0 - dampening) * gg.astype(np.float64)
        b_out = enc(bd.astype(np.float32))
        gg = (gg.astype(np.float64) + momentum * bd).astype(np.float32) if nesterov else bd.astype(np.float32)
    pn = (pf.astype(np.float64) - lr * gg.astype(np.float64)).astype(np.float32)
    return enc(pn), g_out, b_out


# ---- training BatchNorm2d + activation (region_kernels.cpp:309-460) ----------

def _bn_call(fn, x, w, b, rm, rv, eps, slope, factor, update, extra=()):
    N, Cc = x.shape[:2]
    HW = int(np.prod(x.shape[2:]))
    x = np.ascontiguousarray(x, np.uint16)
    y = np.empty_like(x)
    mean = np.empty(Cc, np.float32)
    invstd = np.empty(Cc, np.float32)
    rm = None if rm is None else np.array(rm, np.uint16)
    rv = None if rv is None else np.array(rv, np.uint16)
    w = None if w is None else np.ascontiguousarray(w, np.uint16)
    b = None if b is None else np.ascontiguousarray(b, np.uint16)
    fn(x, _ptr(w), _ptr(b), _ptr(rm), _ptr(rv), y, mean, invstd, N, Cc, HW, eps, slope, factor, int(update), *extra)
    return y, mean, invstd, rm, rv


def bn_fwd(x, w, b, rm, rv, eps=1e-5, slope=0.0, factor=0.1, update=True, reference_impl=False):
    """Fused BN + activation forward on bf16 bits [N, C, ...]: (y, mean, invstd, rm', rv').

    reference_impl=True runs the reference's own compiled host kernel."""
    if reference_impl:
        return _bn_call(reference().xdna_region_bn_fwd_bf16, x, w, b, rm, rv, eps, slope, factor, update, (2,))
    return _bn_call(native().oracle_bn_fwd, x, w, b, rm, rv, eps, slope, factor, update)


def bn_bwd(dy, y, x, w, mean, invstd, slope=0.0, relu=True, need=(True, True, True), reference_impl=False):
    """Backward of the fused pair: (dx, dw, db) as bf16 bits (None where not needed)."""
    N, Cc = x.shape[:2]
    HW = int(np.prod(x.shape[2:]))
    dx = np.empty_like(x) if need[0] else None
    dw = np.empty(Cc, np.uint16) if need[1] else None
    db = np.empty(Cc, np.uint16) if need[2] else None
    w = None if w is None else np.ascontiguousarray(w, np.uint16)
    args = [np.ascontiguousarray(dy, np.uint16), np.ascontiguousarray(y, np.uint16),
            np.ascontiguousarray(x, np.uint16), _ptr(w), np.ascontiguousarray(mean, np.float32),
            np.ascontiguousarray(invstd, np.float32), _ptr(dx), _ptr(dw), _ptr(db), N, Cc, HW, slope, int(relu)]
    if reference_impl:
        reference().xdna_region_bn_bwd_bf16(*args, 2)
    else:
        native().oracle_bn_bwd(*args)
    return dx, dw, db
