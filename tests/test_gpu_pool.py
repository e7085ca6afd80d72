"""2-D max pooling on the xdna kernels against ATen on the CPU (the
reference's path for it): forward values and indices bit-exact, NaNs
included (a NaN wins, the last one in scan order; NaN payloads aside); the
backward bit-exact with ATen's fp32 CPU backward (in bf16: of the same
gradients, rounded once -- ATen's bf16 CPU kernel rounds after every add);
NCHW, channels-last, padding, dilation, ceil mode, the stem / VGG shapes.
"""
import pytest
import torch
import torch.nn.functional as F

import xdna_train

pytestmark = pytest.mark.gpu

X = torch.device("xdna")


@pytest.fixture(autouse=True)
def _fresh(cuda):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    xdna_train.reset_fallback_stats()
    yield


def bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t.view(torch.int32)


CASES = [
    # (shape, kernel, stride, padding, dilation, ceil_mode, channels_last)
    ((2, 64, 56, 56), 3, 2, 1, 1, False, True),    # ResNet stem max-pool
    ((2, 64, 56, 56), 3, 2, 1, 1, False, False),
    ((3, 16, 36, 36), 2, 2, 0, 1, False, False),   # VGG
    ((2, 6, 13, 11), 3, 2, 1, 1, True, True),      # C % 8 != 0, ceil mode
    ((2, 8, 17, 19), 3, 1, 1, 2, False, True),     # dilation
    ((1, 24, 9, 10), (3, 2), (2, 1), (1, 0), 1, True, False),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,k,s,p,d,ceil,cl", CASES)
def test_maxpool_matches_cpu(dtype, shape, k, s, p, d, ceil, cl):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).to(dtype)
    flat = x.view(-1)
    flat[torch.randperm(flat.numel(), generator=g)[: max(2, flat.numel() // 500)]] = float("nan")
    x[0, 0, 0, :3] = torch.tensor([1.0, 1.0, 1.0], dtype=dtype)  # ties: the first maximum wins
    mf = torch.channels_last if cl else torch.contiguous_format
    xc = x.contiguous(memory_format=mf).requires_grad_()
    yc, ic = F.max_pool2d(xc, k, s, p, d, ceil_mode=ceil, return_indices=True)
    gy = torch.randn(yc.shape, generator=g).to(dtype)
    yc.backward(gy)
    xx = x.to(X).contiguous(memory_format=mf).detach().requires_grad_()
    yx, ix = F.max_pool2d(xx, k, s, p, d, ceil_mode=ceil, return_indices=True)
    yx.backward(gy.to(X))
    # values bit-exact; NaN results compare as NaN (ATen's channels-last CPU
    # kernel writes a different NaN payload than its NCHW kernel)
    a, b = yx.detach().cpu(), yc.detach()
    nan_a, nan_b = torch.isnan(a), torch.isnan(b)
    assert torch.equal(nan_a, nan_b)
    assert torch.equal(bits(a.masked_fill(nan_a, 0)), bits(b.masked_fill(nan_b, 0)))
    assert torch.equal(ix.cpu(), ic)
    gx, gc = xx.grad.cpu(), xc.grad
    if dtype == torch.float32:
        assert torch.equal(bits(gx), bits(gc))
    else:
        # ATen's CPU kernel adds bf16 gradients in bf16, one rounding per add;
        # these kernels (like ATen's CUDA one) add in fp32 and round once: the
        # fp32 CPU backward of the same gradients, rounded once, is bit-equal
        ref = torch.ops.aten.max_pool2d_with_indices_backward(gy.float(), x.float().contiguous(memory_format=mf),
                                                              [k] * 2 if isinstance(k, int) else list(k),
                                                              [s] * 2 if isinstance(s, int) else list(s),
                                                              [p] * 2 if isinstance(p, int) else list(p),
                                                              [d] * 2, ceil, ic).bfloat16()
        assert torch.equal(bits(gx), bits(ref))
        assert (gx.float() - gc.float()).abs().max().item() <= 2 ** -6 * gc.float().abs().max().item()
    k_ = xdna_train.kernel_stats()
    assert k_.get("maxpool2d.fwd", 0) >= 1 and k_.get("maxpool2d.bwd", 0) >= 1
    assert "aten::max_pool2d_with_indices" not in xdna_train.fallback_stats()


def test_maxpool_module_in_a_model():
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Conv2d(3, 16, 3, padding=1), torch.nn.ReLU(), torch.nn.MaxPool2d(2))
    x = torch.randn(2, 3, 16, 16)
    ref = net(x)
    nx = torch.nn.Sequential(torch.nn.Conv2d(3, 16, 3, padding=1), torch.nn.ReLU(), torch.nn.MaxPool2d(2))
    nx.load_state_dict(net.state_dict())
    got = nx.to(X)(x.to(X))
    assert torch.allclose(got.cpu(), ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("shape,s,p,d", [((2, 64, 56, 56), 2, 1, 1), ((3, 16, 21, 19), 2, 1, 1),
                                         ((1, 64, 112, 112), 2, 1, 1),  # the stem: 448-thread rows
                                         ((1, 64, 150, 149), 2, 1, 1),  # rows over 512 units, odd W
                                         ((2, 128, 15, 16), 2, 1, 1),
                                         ((2, 8, 17, 15), 3, 1, 1), ((2, 24, 13, 13), 2, 0, 1)])
def test_window_taps_abi_match_int64_path(shape, s, p, d):
    """b2_maxpool2d_fwd_taps / taps_to_indices / bwd_taps against the int64
    path on the same inputs (NaNs and ties included): y, the expanded
    indices and dx are bit-identical."""
    import ctypes
    from xdna_train import _abi
    cuda = torch.device("cuda", 0)
    N, C, H, W = shape
    g = torch.Generator().manual_seed(sum(shape) + s)
    x = torch.randn(*shape, generator=g).bfloat16()
    flat = x.view(-1)
    flat[torch.randperm(flat.numel(), generator=g)[: max(2, flat.numel() // 300)]] = float("nan")
    x[0, :, 0, :3] = 1.0  # ties
    cl = torch.channels_last
    xd = x.to(cuda).contiguous(memory_format=cl)
    OH = (H + 2 * p - d * 2 - 1) // s + 1
    OW = (W + 2 * p - d * 2 - 1) // s + 1
    y0 = torch.empty(N, C, OH, OW, dtype=torch.bfloat16, device=cuda).contiguous(memory_format=cl)
    y1 = torch.empty_like(y0)
    ind0 = torch.empty(N, C, OH, OW, dtype=torch.int64, device=cuda).contiguous(memory_format=cl)
    ind1 = torch.empty_like(ind0)
    taps = torch.empty(N, C, OH, OW, dtype=torch.uint8, device=cuda).contiguous(memory_format=cl)
    arr = lambda t: (ctypes.c_int64 * 4)(*t.stride())  # noqa: E731
    st = torch.cuda.current_stream().cuda_stream
    geo = (N, C, H, W, OH, OW, 3, 3, s, s, p, p, d, d)
    _abi.call("b2_maxpool2d_fwd", xd.data_ptr(), arr(xd), y0.data_ptr(), ind0.data_ptr(), arr(y0), 0, *geo, st)
    _abi.call("b2_maxpool2d_fwd_taps", xd.data_ptr(), arr(xd), y1.data_ptr(), taps.data_ptr(), arr(y1), *geo, st)
    _abi.call("b2_maxpool2d_taps_to_indices", taps.data_ptr(), arr(y1), ind1.data_ptr(), *geo, st)
    dy = torch.randn(N, C, OH, OW, generator=g).bfloat16().to(cuda).contiguous(memory_format=cl)
    dx0 = torch.empty_like(xd)
    dx1 = torch.empty_like(xd)
    _abi.call("b2_maxpool2d_bwd", dy.data_ptr(), ind0.data_ptr(), arr(dy), dx0.data_ptr(), arr(dx0), 0, *geo, st)
    _abi.call("b2_maxpool2d_bwd_taps", dy.data_ptr(), taps.data_ptr(), arr(dy), dx1.data_ptr(), arr(dx1), *geo, st)
    torch.cuda.synchronize()
    assert torch.equal(bits(y0), bits(y1))
    assert torch.equal(ind0.cpu(), ind1.cpu())
    assert torch.equal(bits(dx0), bits(dx1))


def test_indices_written_only_when_read():
    """With the window taps the forward leaves ATen's int64 indices pending:
    a training step never writes them, and reading them runs the expansion
    and gives the CPU's indices."""
    x = torch.randn(2, 64, 20, 20).bfloat16()
    xx = x.to(X).contiguous(memory_format=torch.channels_last).requires_grad_()
    xdna_train.reset_fallback_stats()
    y, ind = F.max_pool2d(xx, 3, 2, 1, return_indices=True)
    y.backward(torch.ones_like(y))
    assert xdna_train.kernel_stats().get("maxpool2d.indices", 0) == 0
    _, ic = F.max_pool2d(x.contiguous(memory_format=torch.channels_last), 3, 2, 1, return_indices=True)
    assert torch.equal(ind.cpu(), ic)
    assert xdna_train.kernel_stats().get("maxpool2d.indices", 0) == 1
