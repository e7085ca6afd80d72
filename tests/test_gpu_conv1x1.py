"""1x1 convolutions (stride 1, no padding) on the tcgen05 GEMM kernels: the C
ABI against an fp32 PyTorch reference of the same op, and nn.Conv2d on the
xdna device against the reference's CPU path (stock PyTorch CPU convolution,
torch_xdna_device.cpp:4578-4603, 4828-4878), in NCHW and channels-last.
Tolerance: the north-star bound max|err| <= 2e-2 * max|ref| and rel-L2 <= 5e-3
(fp32 accumulation and one bf16 rounding).
"""
import ctypes

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import xdna_train
from xdna_train import _abi

pytestmark = pytest.mark.gpu

X = torch.device("xdna")


def st():
    return torch.cuda.current_stream().cuda_stream


def close(got, ref, tol=2e-2, l2=5e-3):
    got, ref = got.detach().float().cpu(), ref.detach().float().cpu()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= tol * scale + 1e-6, f"max abs err {err} vs scale {scale}"
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-12)).item()
    assert rel <= l2, f"rel-L2 {rel}"


@pytest.mark.parametrize("B,Cin,H,W,Cout,layout,bias", [
    (2, 64, 14, 14, 256, 1, False),
    (2, 64, 16, 16, 256, 0, True),
    (4, 256, 7, 7, 64, 1, True),
    (1, 2048, 7, 7, 512, 1, False),
    (8, 32, 16, 16, 96, 0, False),
    (3, 128, 28, 28, 128, 1, False),
])
@pytest.mark.parametrize("dw_f32", [False, True])
def test_conv1x1_abi_vs_fp32(cuda, B, Cin, H, W, Cout, layout, bias, dw_f32):
    g = torch.Generator().manual_seed(B * Cin + Cout)
    x = torch.randn(B, Cin, H, W, generator=g).bfloat16()
    w = (torch.randn(Cout, Cin, 1, 1, generator=g) / Cin ** 0.5).bfloat16()
    b = torch.randn(Cout, generator=g).bfloat16() if bias else None
    dy = torch.randn(B, Cout, H, W, generator=g).bfloat16()
    mf = torch.channels_last if layout == 1 else torch.contiguous_format
    xd = x.to(cuda).contiguous(memory_format=mf)
    dyd = dy.to(cuda).contiguous(memory_format=mf)
    wd = w.to(cuda).contiguous()
    bd = b.to(cuda) if bias else None
    y = torch.empty(B, Cout, H, W, dtype=torch.bfloat16, device=cuda).contiguous(memory_format=mf)
    _abi.call("b2_conv1x1_fwd", xd.data_ptr(), wd.data_ptr(), bd.data_ptr() if bias else None, y.data_ptr(), layout,
              B, Cin, H * W, Cout, st())
    dx = torch.empty_like(xd)
    _abi.call("b2_conv1x1_dgrad", dyd.data_ptr(), wd.data_ptr(), dx.data_ptr(), layout, B, Cin, H * W, Cout, st())
    dw = torch.empty(Cout, Cin, 1, 1, dtype=torch.float32 if dw_f32 else torch.bfloat16, device=cuda)
    nws = _abi.lib().b2_conv1x1_wgrad_workspace_bytes(layout, B, Cin, H * W, Cout)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    _abi.call("b2_conv1x1_wgrad", dyd.data_ptr(), xd.data_ptr(), dw.data_ptr(), 1 if dw_f32 else 0, layout, B, Cin,
              H * W, Cout, ws.data_ptr(), nws, st())
    torch.cuda.synchronize()
    xf, wf, dyf = x.float(), w.float(), dy.float()
    close(y, F.conv2d(xf, wf, b.float() if bias else None))
    close(dx, F.conv_transpose2d(dyf, wf))
    close(dw, torch.einsum("bohw,bihw->oi", dyf, xf)[:, :, None, None])


def test_conv1x1_rejects_bad_shapes(cuda):
    t = torch.zeros(64, dtype=torch.bfloat16, device=cuda)
    rc = _abi.lib().b2_conv1x1_fwd(t.data_ptr(), t.data_ptr(), None, t.data_ptr(), 0, 1, 6, 8, 8, st())
    assert rc != 0 and b"multiples of 8" in _abi.lib().b2_last_error()
    ws = torch.zeros(4, dtype=torch.uint8, device=cuda)
    rc = _abi.lib().b2_conv1x1_wgrad(t.data_ptr(), t.data_ptr(), t.data_ptr(), 0, 1, 1, 8, 8, 8, ws.data_ptr(), 4,
                                     st())
    assert rc == 5 and b"workspace" in _abi.lib().b2_last_error()


@pytest.fixture()
def fresh(cuda):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    saved = xdna_train.set_conv_paths()
    xdna_train.set_conv_paths(conv1x1=True, general=True)
    xdna_train.reset_fallback_stats()
    yield
    xdna_train.set_conv_paths(*saved)


@pytest.mark.parametrize("shape,cl,bias", [((4, 64, 14, 14, 256), True, False), ((4, 64, 16, 16, 128), False, True),
                                           ((2, 512, 7, 7, 2048), True, False)])
def test_conv1x1_module_vs_cpu_path(fresh, shape, cl, bias):
    B, Cin, H, W, Cout = shape
    torch.manual_seed(5)
    conv = nn.Conv2d(Cin, Cout, 1, bias=bias).bfloat16()
    x = torch.randn(B, Cin, H, W).bfloat16()
    g = torch.randn(B, Cout, H, W).bfloat16()
    mf = torch.channels_last if cl else torch.contiguous_format
    xc = x.contiguous(memory_format=mf).detach().requires_grad_()
    yc = conv(xc)
    yc.backward(g.contiguous(memory_format=mf))
    cx = nn.Conv2d(Cin, Cout, 1, bias=bias).bfloat16()
    cx.load_state_dict(conv.state_dict())
    cx = cx.to(X)
    xx = x.to(X).contiguous(memory_format=mf).detach().requires_grad_()
    yx = cx(xx)
    yx.backward(g.to(X).contiguous(memory_format=mf))
    assert yx.is_contiguous(memory_format=mf)
    close(yx, yc)
    close(xx.grad, xc.grad)
    close(cx.weight.grad, conv.weight.grad)
    if bias:
        close(cx.bias.grad, conv.bias.grad)
    k = xdna_train.kernel_stats()
    assert k.get("conv1x1.fwd", 0) >= 1 and k.get("conv1x1.dgrad", 0) >= 1 and k.get("conv1x1.wgrad", 0) >= 1
    assert "convolution_overrideable" not in xdna_train.fallback_stats()


def test_ineligible_1x1_takes_the_aten_path(fresh):
    # 6 -> 5 channels: neither the 1x1 GEMM, the column-matrix path nor the
    # direct kernel (more than 4 channels on both sides)
    conv = nn.Conv2d(6, 5, 1).bfloat16()
    x = torch.randn(2, 6, 5, 5).bfloat16()
    cx = nn.Conv2d(6, 5, 1).bfloat16()
    cx.load_state_dict(conv.state_dict())
    close(cx.to(X)(x.to(X)), conv(x))
    assert "convolution_overrideable" in xdna_train.fallback_stats()
