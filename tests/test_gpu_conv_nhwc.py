"""Channels-last 3x3 convolutions read in place (b2_conv3x3_*_nhwc): the
kernels fetch x / dY through an im2col TMA map whose pixel box is the padded
grid, so they must see exactly the rows b2_pack_rows_bf16 writes -- the
forward and input gradient are compared bit for bit with the padded-row entry
points on the same inputs (the weight gradient of the wider kernels sums
64-pixel patches of tiled 4-D loads instead: to fp32 summation-order
differences, and against an fp32 reference), over shapes that reach each kernel (resident-weight narrow, tiled
128-wide, SM-pair halo with one- and two-box windows, SM-pair without halo,
all-taps narrow wgrad, tiled and SM-pair wgrad), ragged channel chunks,
channel counts below one chunk, strided channels-last views and batch 1.
Also the channels-last dbias (b2_channel_sum_nhwc_bf16) against a float64
sum, and a training step on the xdna device that runs without any padded-row
copy.
"""
import ctypes

import pytest
import torch

from xdna_train import _abi

pytestmark = pytest.mark.gpu


def _st():
    return torch.cuda.current_stream().cuda_stream


def _rows(x):
    B, C, H, W = x.shape
    ch = -(-C // 64)
    rows = torch.empty(B * (H + 2) * (W + 2), ch * 64, dtype=torch.bfloat16, device=x.device)
    _abi.call("b2_pack_rows_bf16", x.data_ptr(), *x.stride(), B, C, H, W, ch, rows.data_ptr(), _st())
    return rows


def _wk(w, dgrad=False):
    Cout, Cin = w.shape[:2]
    ch = -(-(Cout if dgrad else Cin) // 64)
    wk = torch.empty(Cin if dgrad else Cout, ch * 576, dtype=torch.bfloat16, device=w.device)
    _abi.call("b2_pack_weight_dgrad_bf16" if dgrad else "b2_pack_weight_fwd_bf16", w.data_ptr(), Cout, Cin, ch,
              wk.data_ptr(), _st())
    return wk


def _cl(t, extra=0):
    """Channels-last copy of t; with `extra`, a view of the first C channels of
    a channels-last tensor with C + extra channels (pixel stride C + extra)."""
    B, C, H, W = t.shape
    if not extra:
        return t.contiguous(memory_format=torch.channels_last)
    big = torch.zeros(B, C + extra, H, W, dtype=t.dtype, device=t.device).contiguous(memory_format=torch.channels_last)
    big[:, :C] = t
    return big[:, :C]


# (B, Cin, H, W, Cout, extra pixel stride); the kernels each reaches in the comment
SHAPES = [
    (4, 64, 16, 16, 64, 0),     # narrow: resident-weight fwd/dgrad, all-taps wgrad
    (2, 8, 9, 13, 16, 0),       # < one chunk of channels (zero-filled 8..63)
    (3, 72, 7, 11, 96, 0),      # ragged second chunk; tiled 128-wide kernels
    (2, 128, 14, 14, 128, 8),   # strided channels-last view (pixel stride 136)
    (1, 256, 10, 72, 256, 0),   # SM-pair halo, one-box window; pair wgrad; batch 1
    (2, 256, 36, 36, 320, 0),   # SM-pair halo, two-box window
    (1, 256, 3, 200, 256, 0),   # window too wide: plain SM-pair kernel
    (8, 64, 40, 56, 64, 0),     # narrow wgrad with many k-blocks
    (1, 64, 1, 9, 64, 0),       # size-1 dimensions (their strides address nothing)
]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"B{s[0]}_Ci{s[1]}_{s[2]}x{s[3]}_Co{s[4]}_x{s[5]}" for s in SHAPES])
def test_nhwc_entry_points_bit_exact_vs_padded_rows(cuda, shape):
    B, Cin, H, W, Cout, extra = shape
    g = torch.Generator(device=cuda).manual_seed(Cin * 131 + W)
    x = _cl(torch.randn(B, Cin, H, W, generator=g, device=cuda).bfloat16(), extra)
    dy = _cl(torch.randn(B, Cout, H, W, generator=g, device=cuda).bfloat16(), extra)
    w = ((torch.rand(Cout, Cin, 3, 3, generator=g, device=cuda) * 2 - 1) * (1.0 / (9 * Cin)) ** 0.5).bfloat16()
    bias = torch.randn(Cout, generator=g, device=cuda).bfloat16()
    xr, dyr, wk, wkd = _rows(x), _rows(dy), _wk(w), _wk(w, True)
    L = _abi.lib()

    def outs(c):
        return [torch.empty(B, c, H, W, dtype=torch.bfloat16, device=cuda, memory_format=torch.channels_last)
                for _ in range(2)]
    y0, y1 = outs(Cout)
    _abi.call("b2_conv3x3_fwd", xr.data_ptr(), wk.data_ptr(), bias.data_ptr(), y0.data_ptr(), *y0.stride(), B, Cin, H,
              W, Cout, 1, _st())
    _abi.call("b2_conv3x3_fwd_nhwc", x.data_ptr(), x.stride(0), x.stride(2), x.stride(3), wk.data_ptr(),
              bias.data_ptr(), y1.data_ptr(), *y1.stride(), B, Cin, H, W, Cout, 1, _st())
    dx0, dx1 = outs(Cin)
    _abi.call("b2_conv3x3_dgrad", dyr.data_ptr(), wkd.data_ptr(), dx0.data_ptr(), *dx0.stride(), B, Cout, H, W, Cin,
              _st())
    _abi.call("b2_conv3x3_dgrad_nhwc", dy.data_ptr(), dy.stride(0), dy.stride(2), dy.stride(3), wkd.data_ptr(),
              dx1.data_ptr(), *dx1.stride(), B, Cout, H, W, Cin, _st())
    wsb = L.b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout)
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda)
    dw0 = torch.empty(Cout, Cin, 3, 3, dtype=torch.float32, device=cuda)
    dw1 = torch.full_like(dw0, float("nan"))
    _abi.call("b2_conv3x3_wgrad", dyr.data_ptr(), xr.data_ptr(), dw0.data_ptr(), _abi.B2_F32, B, Cin, H, W, Cout,
              ws.data_ptr(), wsb, _st())
    _abi.call("b2_conv3x3_wgrad_nhwc", dy.data_ptr(), dy.stride(0), dy.stride(2), dy.stride(3), x.data_ptr(),
              x.stride(0), x.stride(2), x.stride(3), dw1.data_ptr(), _abi.B2_F32, B, Cin, H, W, Cout, ws.data_ptr(),
              wsb, _st())
    # the same weight gradient written in a channels-last weight's OHWI order,
    # fp32 and bf16: the same sums, bit for bit
    dw2 = torch.full((Cout, 3, 3, Cin), float("nan"), dtype=torch.float32, device=cuda)
    _abi.call("b2_conv3x3_wgrad_nhwc_ohwi", dy.data_ptr(), dy.stride(0), dy.stride(2), dy.stride(3), x.data_ptr(),
              x.stride(0), x.stride(2), x.stride(3), dw2.data_ptr(), _abi.B2_F32, B, Cin, H, W, Cout, ws.data_ptr(),
              wsb, _st())
    dw3 = torch.empty(Cout, Cin, 3, 3, dtype=torch.bfloat16, device=cuda)
    dw4 = torch.empty(Cout, 3, 3, Cin, dtype=torch.bfloat16, device=cuda)
    _abi.call("b2_conv3x3_wgrad_nhwc", dy.data_ptr(), dy.stride(0), dy.stride(2), dy.stride(3), x.data_ptr(),
              x.stride(0), x.stride(2), x.stride(3), dw3.data_ptr(), _abi.B2_BF16, B, Cin, H, W, Cout, ws.data_ptr(),
              wsb, _st())
    _abi.call("b2_conv3x3_wgrad_nhwc_ohwi", dy.data_ptr(), dy.stride(0), dy.stride(2), dy.stride(3), x.data_ptr(),
              x.stride(0), x.stride(2), x.stride(3), dw4.data_ptr(), _abi.B2_BF16, B, Cin, H, W, Cout, ws.data_ptr(),
              wsb, _st())
    torch.cuda.synchronize()
    assert torch.equal(dw2.permute(0, 3, 1, 2).view(torch.int32), dw1.view(torch.int32))
    assert torch.equal(dw4.permute(0, 3, 1, 2).view(torch.int16), dw3.view(torch.int16))
    assert torch.equal(y0, y1)
    assert torch.equal(dx0, dx1)
    # dW: the all-taps narrow kernel reads the same padded-grid k-blocks either
    # way (bit for bit); the wider kernels sum channels-last operands over
    # 64-pixel patches instead (same products, another fp32 summation order)
    d = (dw1 - dw0).abs().max().item()
    assert d <= 1e-5 * dw0.abs().max().item() + 1e-30, d
    # and the results are the convolution (fp32 reference, conv tolerance)
    ref = torch.relu(torch.nn.functional.conv2d(x.float(), w.float(), bias.float(), padding=1))
    assert (y1.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    with torch.no_grad():
        dref = torch.ops.aten.convolution_backward(dy.float(), x.float(), w.float(), None, [1, 1], [1, 1], [1, 1],
                                                   False, [0, 0], 1, [False, True, False])[1]
    assert (dw1 - dref).abs().max().item() <= 2e-2 * dref.abs().max().item()
    code = ctypes.c_int(-1)
    _abi.check(L.b2_device_status(torch.cuda.current_device(), ctypes.byref(code)))
    assert code.value == 0


def test_nhwc_entry_points_refuse_unaligned_layouts(cuda):
    L = _abi.lib()
    t = torch.zeros(1 << 16, dtype=torch.bfloat16, device=cuda)
    # 12 channels: pixel stride not a multiple of 8 elements
    st = L.b2_conv3x3_fwd_nhwc(t.data_ptr(), 12 * 64, 12 * 8, 12, t.data_ptr(), None, t.data_ptr(), 12 * 64, 1,
                               12 * 8, 12, 1, 12, 8, 8, 16, 0, _st())
    assert st == 3 and b"multiples of 8" in L.b2_last_error()


@pytest.mark.parametrize("shape", [(2, 64, 7, 9), (3, 200, 5, 5), (1, 8, 1, 1)])
def test_channel_sum_nhwc(cuda, shape):
    B, C, H, W = shape
    g = torch.Generator(device=cuda).manual_seed(C)
    x = torch.randn(B, C, H, W, generator=g, device=cuda).bfloat16().contiguous(memory_format=torch.channels_last)
    L = _abi.lib()
    wsb = L.b2_channel_sum_nhwc_workspace_bytes(B, C, H, W)
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda)
    out = torch.empty(C, dtype=torch.float32, device=cuda)
    _abi.call("b2_channel_sum_nhwc_bf16", x.data_ptr(), x.stride(0), x.stride(2), x.stride(3), B, C, H, W,
              out.data_ptr(), _abi.B2_F32, ws.data_ptr(), wsb, _st())
    torch.cuda.synchronize()
    ref = x.double().sum(dim=(0, 2, 3))
    assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-4)


def test_channels_last_training_step_makes_no_padded_copies(cuda):
    """Conv2d(64 -> 64, bias) and Conv2d(64 -> 32) on channels-last xdna
    activations: forward, dX, dbias and (deferred) dW through the in-place
    kernels -- no pack_rows launch -- and the same values as the NCHW input,
    whose activations do go through the padded-row copy."""
    import xdna_train
    xdna_train.register_xdna_device()
    X = torch.device("xdna", 0)
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Conv2d(64, 64, 3, padding=1), torch.nn.Conv2d(64, 32, 3, padding=1,
                                                                                     bias=False)).bfloat16()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 64, 20, 20, generator=g).bfloat16()
    gy = torch.randn(4, 32, 20, 20, generator=g).bfloat16()

    def run(mf):
        m = torch.nn.Sequential(*[torch.nn.Conv2d(c.in_channels, c.out_channels, 3, padding=1,
                                                  bias=c.bias is not None) for c in net]).bfloat16()
        m.load_state_dict(net.state_dict())
        m = m.to(X).to(memory_format=mf)
        xx = x.to(X).contiguous(memory_format=mf).requires_grad_()
        xdna_train.reset_mapped_cpu_stats()
        y = m(xx)
        y.backward(gy.to(X).contiguous(memory_format=mf))
        # each weight's gradient arrives in its parameter's own layout (no
        # re-layout copy by autograd): OHWI for a channels-last weight
        for p in m.parameters():
            assert p.grad.stride() == p.stride(), (p.shape, p.grad.stride(), p.stride())
        out = [y.detach().cpu(), xx.grad.cpu()] + [p.grad.cpu() for p in m.parameters()]
        return out, dict(xdna_train.kernel_stats())
    cl, ks_cl = run(torch.channels_last)
    nc, ks_nc = run(torch.contiguous_format)
    assert ks_cl.get("pack_rows", 0) == 0 and ks_cl.get("pack_rows_dbias", 0) == 0, ks_cl
    assert ks_cl.get("conv3x3.wgrad", 0) == 4 and ks_cl.get("channel_sum", 0) == 2, ks_cl
    assert ks_nc.get("pack_rows", 0) > 0
    # y and dX bit for bit; dW and dbias sum the same products in another
    # order (64-pixel patches / groups here, padded-row k-blocks there)
    for i, (a, b) in enumerate(zip(cl, nc)):
        if i < 2:
            assert torch.equal(a.contiguous(), b.contiguous()), i
        else:
            a, b = a.float(), b.float()
            assert (a - b).abs().max().item() <= 1e-2 * b.abs().max().item(), i
