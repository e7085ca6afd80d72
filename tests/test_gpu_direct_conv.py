"""Direct convolutions for RGB layers: the input gradient of an output layer
(the style network's 9x9 32->3) and the forward of an input layer (its 9x9
3->32 stem) on the CUDA cores, weight gradients on ATen's library kernels.  Checked against
an fp32 reference of the reference's CPU path (the same convolution on the
CPU) with the north-star bound max|err| <= 2e-2 * max|ref| (fp32 sums, one
bf16 rounding), NCHW and channels-last, with and without bias, strided and
dilated forwards.
"""
import pytest
import torch
import torch.nn as nn

import xdna_train

pytestmark = pytest.mark.gpu

X = torch.device("xdna")


def close(got, ref, tol=2e-2, l2=1e-2):
    got, ref = got.detach().float().cpu(), ref.detach().float().cpu()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= tol * scale + 1e-6, f"max abs err {err} vs scale {scale}"
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-12)).item()
    assert rel <= l2, f"rel-L2 {rel}"


@pytest.fixture()
def fresh(cuda):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    xdna_train.reset_fallback_stats()
    yield


CASES = [
    # (B, Cin, H, W, Cout, k, stride, pad, dilation, bias, channels_last)
    (4, 32, 36, 36, 3, 9, 1, 4, 1, True, False),   # style network output layer
    (2, 32, 20, 17, 3, 9, 1, 4, 1, False, True),
    (3, 16, 13, 11, 1, 5, 1, 2, 1, True, False),
    (2, 64, 9, 9, 4, 5, 1, 2, 1, True, True),
    (2, 12, 16, 16, 3, 3, 1, 2, 2, False, False),  # dilated
    (2, 3, 15, 14, 16, 3, 2, 1, 1, True, False),   # strided RGB input layer
    (2, 4, 12, 12, 16, 7, 2, 3, 1, True, True),
    (3, 3, 20, 18, 64, 5, 1, 2, 1, True, False),
    (2, 3, 16, 16, 32, 9, 1, 4, 1, True, True),    # style network stem
]


@pytest.mark.parametrize("B,Cin,H,W,Cout,k,s,p,d,bias,cl", CASES)
def test_direct_conv_vs_fp32(fresh, B, Cin, H, W, Cout, k, s, p, d, bias, cl):
    torch.manual_seed(B * Cin + k + Cout)
    conv = nn.Conv2d(Cin, Cout, k, stride=s, padding=p, dilation=d, bias=bias).bfloat16()
    x = torch.randn(B, Cin, H, W).bfloat16()
    mf = torch.channels_last if cl else torch.contiguous_format
    ref = nn.Conv2d(Cin, Cout, k, stride=s, padding=p, dilation=d, bias=bias)
    ref.load_state_dict({n: t.float() for n, t in conv.state_dict().items()})
    xr = x.float().contiguous(memory_format=mf).detach().requires_grad_()
    yr = ref(xr)
    g = torch.randn_like(yr).bfloat16()
    yr.backward(g.float())
    cx = nn.Conv2d(Cin, Cout, k, stride=s, padding=p, dilation=d, bias=bias).bfloat16()
    cx.load_state_dict(conv.state_dict())
    cx = cx.to(X)
    xx = x.to(X).contiguous(memory_format=mf).detach().requires_grad_()
    yx = cx(xx)
    assert yx.shape == yr.shape
    if cl:
        assert yx.is_contiguous(memory_format=torch.channels_last)
    yx.backward(g.to(X).contiguous(memory_format=mf))
    close(yx, yr)
    close(xx.grad, xr.grad)
    close(cx.weight.grad, ref.weight.grad)
    if bias:
        close(cx.bias.grad, ref.bias.grad)
    kst = xdna_train.kernel_stats()
    if Cin <= 4 and 16 <= Cout <= 64 and Cin * k * k <= 512:  # RGB input layer: forward
        assert kst.get("direct_conv.fwd", 0) >= 1
        assert "convolution_overrideable" not in xdna_train.fallback_stats()
    if Cout <= 4 and Cin >= 8 and s == 1:  # RGB output layer: input gradient
        assert kst.get("direct_conv.dgrad", 0) >= 1


def test_direct_conv_abi_matches_cpu(cuda):
    """The C ABI alone: forward of a 9x9 32->3 layer against torch's CPU conv."""
    import ctypes

    from xdna_train import _abi
    torch.manual_seed(1)
    B, Cin, H, W, Cout, k = 2, 32, 24, 20, 3, 9
    x = torch.randn(B, Cin, H, W).bfloat16()
    w = (torch.randn(Cout, Cin, k, k) * 0.05).bfloat16()
    ref = torch.nn.functional.conv2d(x.float(), w.float(), padding=4)
    xd, wd = x.to(cuda), w.to(cuda)
    n = _abi.lib().b2_direct_conv_weight_floats(Cout, Cin, k, k, 0)
    wt = torch.empty(n, dtype=torch.float32, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    _abi.call("b2_direct_conv_weight", wd.data_ptr(), Cout, Cin, k, k, 0, wt.data_ptr(), st)
    y = torch.empty(B, Cout, H, W, dtype=torch.bfloat16, device=cuda)
    strides = ctypes.c_int64 * 4
    xs, ys = strides(*xd.stride()), strides(*y.stride())
    _abi.call("b2_direct_conv_bf16", xd.data_ptr(), xs, B, Cin, H, W, wt.data_ptr(), k, k, 1, 1, 4, 4, 1, 1, None,
              y.data_ptr(), ys, Cout, H, W, st)
    close(y, ref)
    # fp32 sums rounded once: within one bf16 ulp of the exact fp32 result
    assert ((y.float().cpu() - ref).abs() <= ref.abs() * 2 ** -8 + 1e-3).float().mean().item() > 0.999


def test_frozen_weight_packs_are_cached_and_invalidated(fresh):
    """A frozen 3x3 conv packs its weight once; every kind of write into the
    weight (in-place op, .data in-place op, copy_, load_state_dict) makes the
    next call repack, and the results always follow the current weights."""
    torch.manual_seed(3)
    conv = nn.Conv2d(64, 64, 3, padding=1, bias=False).bfloat16().to(X)
    conv.weight.requires_grad_(False)
    x = torch.randn(2, 64, 8, 8).bfloat16()
    xx = x.to(X)

    def ref(w):
        return torch.nn.functional.conv2d(x.float(), w.detach().float().cpu(), padding=1)

    def stats():
        s = xdna_train.async_dw_stats()
        return s["packed_weight_hits"], s["packed_weight_misses"]

    h0, m0 = stats()
    close(conv(xx), ref(conv.weight))
    close(conv(xx), ref(conv.weight))
    h1, m1 = stats()
    assert h1 - h0 >= 1 and m1 - m0 >= 1
    writes = [
        lambda w: w.mul_(0.5),
        lambda w: w.data.add_(0.01),
        lambda w: w.copy_(torch.randn(64, 64, 3, 3).bfloat16().to(X)),
        lambda w: conv.load_state_dict({"weight": torch.randn(64, 64, 3, 3).bfloat16()}),
    ]
    for write in writes:
        with torch.no_grad():
            write(conv.weight)
        close(conv(xx), ref(conv.weight))
    assert xdna_train.kernel_stats().get("pack_weight", 0) >= 1 + len(writes)
