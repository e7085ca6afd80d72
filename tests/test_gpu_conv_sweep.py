"""Per-shape parity over the whole 3x3 conv sweep and the
reference's strip shapes, through the C ABI.

For every C_in = C_out in {32, 64, 128, 256, 512}, H = W in {18, 36, 72, 144}
and batch in {8, 40, 128} -- the shapes `bench.py --conv-sweep` times -- the
forward, input-gradient and weight-gradient kernels run on seeded NCHW bf16
inputs (x, dY ~ N(0,1), W ~ kaiming-uniform) and are checked against an fp32
reference of the same op: max |out - ref| <= 2e-2 * max |ref| and relative L2
error <= 5e-3, the bound of the other conv tests.  The fp32 reference is
ATen's native convolution (im2col + fp32 GEMM, cuDNN off, TF32 off): cuDNN's
fp32 forward at batch 8, 512 channels, 144x144 returned wrong values for
output channels >= 192 on B200 (max error 4.7 at a scale of 5.4), where cuDNN
per image, cuDNN in bf16, the native convolution and the CPU all agreed with
this library's kernels to within 0.016.
The reference records one error per sweep shape the same way
(benchmarks/conv_shape_sweep.py:60-126); its own strip shapes
(tests/run_conv3x3w_torch.py:22-35, (4,64,16,56,64) and (2,64,20,64,128))
are added.  Batch-40 shapes write channels-last outputs from channels-last
inputs, the others NCHW.

The largest cases cover what the smaller tests cannot: the SM-pair halo
kernel at full grid occupancy (B128 C256 72x72, the conv bench's shape), the
longest split-K weight-gradient reduction (B128 C512 144x144: 2.73 M padded
rows, 2.8 GB of packed rows per operand, byte offsets past 2^31) and the
narrow kernels at every size.  Comparisons run on the device (tensors of up
to 1.36 G elements).
"""
import ctypes

import pytest
import torch

from xdna_train import _abi

pytestmark = pytest.mark.gpu

SWEEP_C = (32, 64, 128, 256, 512)
SWEEP_HW = (18, 36, 72, 144)
SWEEP_B = (8, 40, 128)
# (B, Cin, H, W, Cout, bias)
SHAPES = [(b, c, hw, hw, c, True) for c in SWEEP_C for hw in SWEEP_HW for b in SWEEP_B]
SHAPES += [(4, 64, 16, 56, 64, False), (2, 64, 20, 64, 128, True)]


def _st():
    return torch.cuda.current_stream().cuda_stream


def _rows(x):
    B, C, H, W = x.shape
    ch = -(-C // 64)
    rows = torch.empty(B * (H + 2) * (W + 2), ch * 64, dtype=torch.bfloat16, device=x.device)
    s = x.stride()
    _abi.call("b2_pack_rows_bf16", x.data_ptr(), s[0], s[1], s[2], s[3], B, C, H, W, ch, rows.data_ptr(), _st())
    return rows


def _wk(w, dgrad=False):
    Cout, Cin = w.shape[:2]
    ch = -(-(Cout if dgrad else Cin) // 64)
    wk = torch.empty(Cin if dgrad else Cout, ch * 576, dtype=torch.bfloat16, device=w.device)
    name = "b2_pack_weight_dgrad_bf16" if dgrad else "b2_pack_weight_fwd_bf16"
    _abi.call(name, w.data_ptr(), Cout, Cin, ch, wk.data_ptr(), _st())
    return wk


def _check(name, got, ref, tol=2e-2, l2=5e-3):
    d = got.float() - ref
    scale = ref.abs().max().item()
    err = d.abs().max().item()
    rel = (torch.linalg.vector_norm(d, dtype=torch.float64) /
           torch.linalg.vector_norm(ref, dtype=torch.float64).clamp_min(1e-30)).item()
    del d
    assert err <= tol * scale, f"{name}: max abs err {err:.4g} > {tol} * {scale:.4g}"
    assert rel <= l2, f"{name}: rel L2 {rel:.4g}"


def _sid(s):
    return "B{}_Ci{}_{}x{}_Co{}{}".format(*s[:5], "_bias" if s[5] else "")


@pytest.fixture
def native_fp32_conv():
    saved = (torch.backends.cudnn.enabled, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.enabled = False
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cudnn.enabled, torch.backends.cuda.matmul.allow_tf32 = saved


@pytest.mark.parametrize("shape", SHAPES, ids=[_sid(s) for s in SHAPES])
def test_conv3x3_sweep_shape_vs_fp32(cuda, native_fp32_conv, shape):
    B, Cin, H, W, Cout, has_bias = shape
    cl = B == 40
    mf = torch.channels_last if cl else torch.contiguous_format
    g = torch.Generator(device=cuda).manual_seed(B * 1000003 + Cin * 1009 + H)
    x = torch.randn(B, Cin, H, W, generator=g, device=cuda).bfloat16().contiguous(memory_format=mf)
    dy = torch.randn(B, Cout, H, W, generator=g, device=cuda).bfloat16().contiguous(memory_format=mf)
    bound = (1.0 / (9 * Cin)) ** 0.5
    w = ((torch.rand(Cout, Cin, 3, 3, generator=g, device=cuda) * 2 - 1) * bound).bfloat16()
    b = torch.randn(Cout, generator=g, device=cuda).bfloat16() if has_bias else None
    xr, dyr = _rows(x), _rows(dy)
    wf = w.float()

    # forward
    y = torch.empty(B, Cout, H, W, dtype=torch.bfloat16, device=cuda, memory_format=mf)
    wk = _wk(w)
    _abi.call("b2_conv3x3_fwd", xr.data_ptr(), wk.data_ptr(), 0 if b is None else b.data_ptr(), y.data_ptr(),
              *y.stride(), B, Cin, H, W, Cout, 0, _st())
    with torch.no_grad():
        ref = torch.nn.functional.conv2d(x.float(), wf, None if b is None else b.float(), padding=1)
    _check("fwd", y, ref)
    del y, ref, wk

    # input gradient
    dx = torch.empty(B, Cin, H, W, dtype=torch.bfloat16, device=cuda, memory_format=mf)
    wkd = _wk(w, dgrad=True)
    _abi.call("b2_conv3x3_dgrad", dyr.data_ptr(), wkd.data_ptr(), dx.data_ptr(), *dx.stride(), B, Cout, H, W, Cin,
              _st())
    with torch.no_grad():
        ref = torch.ops.aten.convolution_backward(dy.float(), x.float(), wf, None, [1, 1], [1, 1], [1, 1], False,
                                                  [0, 0], 1, [True, False, False])[0]
    _check("dgrad", dx, ref)
    del dx, ref, wkd

    # weight gradient (fp32 dW)
    ws_bytes = _abi.lib().b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    dw = torch.empty(Cout, Cin, 3, 3, dtype=torch.float32, device=cuda)
    _abi.call("b2_conv3x3_wgrad", dyr.data_ptr(), xr.data_ptr(), dw.data_ptr(), _abi.B2_F32, B, Cin, H, W, Cout,
              ws.data_ptr(), ws_bytes, _st())
    with torch.no_grad():
        ref = torch.ops.aten.convolution_backward(dy.float(), x.float(), wf, None, [1, 1], [1, 1], [1, 1], False,
                                                  [0, 0], 1, [False, True, False])[1]
    _check("wgrad", dw, ref)
    code = ctypes.c_int(-1)
    _abi.check(_abi.lib().b2_device_status(torch.cuda.current_device(), ctypes.byref(code)))
    assert code.value == 0
