"""Training-mode BatchNorm on the xdna kernels (native_batch_norm /
native_batch_norm_backward): the C ABI against the oracle in both memory
layouts, and the modules against PyTorch on the CPU -- the reference's path
for these ops (it runs ATen's CPU kernels on aliases, torch_xdna_device.cpp:
4214-4358) -- with the cases of the reference's own test
(tests/run_norm_backward.py: every output mask, BatchNorm1d/2d, InstanceNorm,
bf16 rel-L2 < 0.03, fp32 < 1e-4).
"""
import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

import xdna_train
from oracle import oracle
from xdna_train import _abi

pytestmark = pytest.mark.gpu

X = torch.device("xdna")


@pytest.fixture(autouse=True)
def _fresh(cuda):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    xdna_train.reset_fallback_stats()
    yield


def st():
    return torch.cuda.current_stream().cuda_stream


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-9)).item()


def launched(kind):
    return xdna_train.kernel_stats().get(kind, 0)


# ---- C ABI vs the oracle --------------------------------------------------------

@pytest.mark.parametrize("shape,layout", [((8, 64, 14, 14), 0), ((8, 64, 14, 14), 1), ((4, 256, 7, 7), 1),
                                          ((2, 2048, 3, 3), 1), ((3, 24, 5, 7), 1), ((40, 128, 9, 9), 0),
                                          ((64, 8, 1, 1), 0)])
@pytest.mark.parametrize("pdtype", [0, 1])
def test_batch_norm_abi_vs_oracle(cuda, shape, layout, pdtype):
    N, C, H, W = shape
    rng = np.random.default_rng(N * C + H)
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32) * 1.7 + 0.4).bfloat16()
    dy = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).bfloat16()
    pt = torch.float32 if pdtype == 1 else torch.bfloat16
    w = torch.from_numpy(rng.uniform(0.5, 1.5, C).astype(np.float32)).to(pt)
    b = torch.from_numpy(rng.standard_normal(C).astype(np.float32) * 0.3).to(pt)
    rm = torch.from_numpy(rng.standard_normal(C).astype(np.float32) * 0.1).to(pt)
    rv = torch.from_numpy(rng.uniform(0.5, 1.5, C).astype(np.float32)).to(pt)
    mf = torch.channels_last if layout == 1 else torch.contiguous_format
    xd, dyd = x.to(cuda).contiguous(memory_format=mf), dy.to(cuda).contiguous(memory_format=mf)
    wd, bd, rmd, rvd = (t.to(cuda) for t in (w, b, rm, rv))
    y = torch.empty_like(xd)
    sm = torch.empty(C, dtype=torch.float32, device=cuda)
    si = torch.empty_like(sm)
    nws = _abi.lib().b2_batch_norm_workspace_bytes(N, C, H * W, layout)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    _abi.call("b2_batch_norm_fwd_bf16", xd.data_ptr(), layout, wd.data_ptr(), bd.data_ptr(), pdtype, rmd.data_ptr(),
              rvd.data_ptr(), pdtype, y.data_ptr(), sm.data_ptr(), si.data_ptr(), N, C, H * W, ctypes.c_float(0.1),
              ctypes.c_float(1e-5), ws.data_ptr(), nws, st())
    dx = torch.empty_like(xd)
    dw = torch.empty(C, dtype=pt, device=cuda)
    db = torch.empty_like(dw)
    _abi.call("b2_batch_norm_bwd_bf16", dyd.data_ptr(), xd.data_ptr(), layout, wd.data_ptr(), pdtype, sm.data_ptr(),
              si.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), pdtype, N, C, H * W, ws.data_ptr(), nws,
              st())
    torch.cuda.synchronize()
    # oracle: the fused BN + activation with slope 1 (identity), on NCHW bf16 bits
    wb = bits(w.bfloat16())
    bb = bits(b.bfloat16())
    oy, om, oi, orm, orv = oracle.bn_fwd(bits(x), wb if pdtype == 0 else None, None, bits(rm.bfloat16()),
                                         bits(rv.bfloat16()), 1e-5, 1.0, 0.1, True)
    np.testing.assert_allclose(sm.cpu().numpy(), om, rtol=0, atol=2e-6 * max(1.0, np.abs(om).max()))
    np.testing.assert_allclose(si.cpu().numpy(), oi, rtol=2e-6)
    # y against the same affine transform in fp32 from the GPU's own statistics
    scale = w.float() * si.cpu()
    shift = b.float() - sm.cpu() * scale
    want_y = (x.float() * scale[None, :, None, None] + shift[None, :, None, None]).bfloat16()
    assert rel(y, want_y) < 4e-3
    yb = bits(y.contiguous())
    assert (yb == bits(want_y)).mean() > 0.98
    # running statistics (bf16 case: the oracle's update exactly, up to one ulp)
    if pdtype == 0:
        assert np.abs(bits(rmd).astype(int) - orm.astype(int)).max() <= 1
        assert np.abs(bits(rvd).astype(int) - orv.astype(int)).max() <= 1
    else:
        M = N * H * W
        torch.testing.assert_close(rmd.cpu(), 0.9 * rm + 0.1 * torch.from_numpy(om), rtol=1e-5, atol=1e-5)
        var = torch.from_numpy(1.0 / oi.astype(np.float64) ** 2 - 1e-5)
        torch.testing.assert_close(rvd.cpu().double(), 0.9 * rv.double() + 0.1 * var * M / (M - 1), rtol=1e-4,
                                   atol=1e-5)
    # backward from the GPU's statistics; slope 1 makes the oracle's dz = dy
    odx, odw, odb = oracle.bn_bwd(bits(dy), bits(x), bits(x), wb if pdtype == 0 else bits(w.bfloat16()),
                                  sm.cpu().numpy(), si.cpu().numpy(), 1.0, False)
    if pdtype == 1:  # the oracle reads a bf16 weight; redo dx's final scale with the fp32 one
        odx = None
    got_dx = dx.contiguous().cpu()
    if odx is not None:
        assert rel(got_dx, torch.from_numpy(oracle.bf16_value(odx))) < 4e-3
    assert rel(dw.float().cpu(), torch.from_numpy(oracle.bf16_value(odw))) < 1e-2
    assert rel(db.float().cpu(), torch.from_numpy(oracle.bf16_value(odb))) < 1e-2


# ---- modules vs the CPU (the reference's path) ------------------------------------

def _grads(make, shape, dtype, dev, input_grad=True, channels_last=False):
    torch.manual_seed(0)
    model = make().to(dtype)
    x = torch.randn(*shape, dtype=dtype)
    torch.manual_seed(1)
    w = torch.randn(*shape, dtype=dtype)
    model, x, w = model.to(dev), x.to(dev), w.to(dev)
    if channels_last:
        x = x.contiguous(memory_format=torch.channels_last)
    if input_grad:
        x.requires_grad_()
    y = model(x)
    (y * w).float().sum().backward()
    out = {"y": y.detach(), "x": x.grad if input_grad else None}
    for name, p in model.named_parameters():
        out[name] = p.grad
    for name, b in model.named_buffers():
        if b.is_floating_point():
            out[name] = b.detach()
    return out


CASES = [
    ("BatchNorm2d(affine=False)", lambda: nn.BatchNorm2d(4, affine=False), (8, 4, 6, 6), True),
    ("BatchNorm1d(affine=False)", lambda: nn.BatchNorm1d(4, affine=False), (8, 4), True),
    ("InstanceNorm2d()", lambda: nn.InstanceNorm2d(4), (8, 4, 6, 6), True),
    ("InstanceNorm1d()", lambda: nn.InstanceNorm1d(4), (8, 4, 6), True),
    ("InstanceNorm2d(affine=True)", lambda: nn.InstanceNorm2d(4, affine=True), (8, 4, 6, 6), True),
    ("BatchNorm2d(no stats, affine=False)", lambda: nn.BatchNorm2d(4, affine=False, track_running_stats=False),
     (8, 4, 6, 6), True),
    ("BatchNorm2d(), no input grad", lambda: nn.BatchNorm2d(4), (8, 4, 6, 6), False),
    ("BatchNorm2d()", lambda: nn.BatchNorm2d(4), (8, 4, 6, 6), True),
    ("BatchNorm2d(64) large", lambda: nn.BatchNorm2d(64), (16, 64, 28, 28), True),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("name,make,shape,input_grad", CASES)
def test_norm_modules_vs_cpu(dtype, name, make, shape, input_grad):
    tol = 0.03 if dtype == torch.bfloat16 else 1e-4
    ref = _grads(make, shape, dtype, "cpu", input_grad)
    got = _grads(make, shape, dtype, X, input_grad)
    for k in ref:
        assert (got[k] is None) == (ref[k] is None), k
        if ref[k] is not None:
            assert rel(got[k], ref[k]) < tol, (k, rel(got[k], ref[k]))
    if dtype == torch.bfloat16:
        assert launched("batch_norm.fwd") >= 3 and launched("batch_norm.bwd") >= 2
        assert "aten::native_batch_norm" not in xdna_train.fallback_stats()


@pytest.mark.parametrize("C,hw", [(64, 28), (256, 14), (2048, 7), (24, 9)])
def test_channels_last_batch_norm_vs_fp32(C, hw):
    """ResNet-style channels-last BatchNorm2d: errors against an fp32 CPU
    reference no larger than those of the CPU's own bf16 path (+ a floor)."""
    make = lambda: nn.BatchNorm2d(C)  # noqa: E731
    shape = (16, C, hw, hw)
    ref32 = _grads(make, shape, torch.float32, "cpu")
    cpu16 = _grads(make, shape, torch.bfloat16, "cpu", channels_last=True)
    got = _grads(make, shape, torch.bfloat16, X, channels_last=True)
    assert got["y"].is_contiguous(memory_format=torch.channels_last)
    for k in ref32:
        e_got, e_cpu = rel(got[k], ref32[k]), rel(cpu16[k], ref32[k])
        assert e_got <= 1.5 * e_cpu + 4e-3, (k, e_got, e_cpu)
    assert launched("batch_norm.fwd") >= 3 and "aten::native_batch_norm" not in xdna_train.fallback_stats()


def test_eval_mode_and_mixed_dtypes():
    torch.manual_seed(3)
    bn = nn.BatchNorm2d(16)
    x = torch.randn(4, 16, 5, 5)
    # bf16 activations with fp32 parameters and statistics (autocast-style model)
    ref = nn.BatchNorm2d(16)
    ref.load_state_dict(bn.state_dict())
    bx = bn.to(X)
    xb = x.bfloat16().to(X).requires_grad_()
    y = bx(xb)
    xr = x.bfloat16().float().requires_grad_()
    yr = ref(xr)
    assert rel(y, yr) < 1e-2
    g = torch.randn(4, 16, 5, 5)
    (y.float() * g.to(X)).sum().backward()
    (yr * g).sum().backward()
    assert rel(bx.weight.grad, ref.weight.grad) < 1e-2 and bx.weight.grad.dtype == torch.float32
    assert rel(bx.running_var, ref.running_var) < 1e-3
    assert launched("batch_norm.fwd") >= 3
    bx.eval()
    ref.eval()
    assert rel(bx(x.bfloat16().to(X)), ref(x.bfloat16().float())) < 1e-2
    assert xdna_train.fallback_stats()["aten::native_batch_norm"]["calls"] == 1


# ---- BatchNorm tails folded into the output pass ---------------------------------

def _block(cl, fused, seed=0):
    """conv -> bn -> (+ identity) -> relu_, the residual tail of a ResNet
    bottleneck, forward and backward; fused or not."""
    xdna_train.set_fusion(bn_epilogue=fused)
    torch.manual_seed(seed)
    conv = nn.Conv2d(64, 64, 3, padding=1, bias=False).bfloat16()
    bn = nn.BatchNorm2d(64).bfloat16()
    mf = torch.channels_last if cl else torch.contiguous_format
    x = torch.randn(4, 64, 14, 14).bfloat16()
    idn = torch.randn(4, 64, 14, 14).bfloat16()
    g = torch.randn(4, 64, 14, 14).bfloat16()
    conv, bn = conv.to(X), bn.to(X)
    xx = x.to(X).contiguous(memory_format=mf).requires_grad_()
    ii = idn.to(X).contiguous(memory_format=mf).requires_grad_()
    out = bn(conv(xx))
    out += ii
    out.relu_()
    out.backward(g.to(X).contiguous(memory_format=mf))
    res = {"y": out.detach().cpu(), "dx": xx.grad.cpu(), "di": ii.grad.cpu(), "dw": conv.weight.grad.cpu(),
           "dg": bn.weight.grad.cpu(), "db": bn.bias.grad.cpu(), "rm": bn.running_mean.cpu()}
    return res


@pytest.mark.parametrize("cl", [False, True])
def test_residual_add_and_relu_fold_into_batch_norm(cl):
    before = xdna_train.async_dw_stats()["folded_tails"]
    try:
        fused = _block(cl, True)
        folded = xdna_train.async_dw_stats()["folded_tails"] - before
        fb = xdna_train.fallback_stats()
        xdna_train.reset_fallback_stats()
        plain = _block(cl, False)
        fp = xdna_train.fallback_stats()
    finally:
        xdna_train.set_fusion(bn_epilogue=True)
    assert folded >= 2
    calls = lambda d, k: d.get(k, {}).get("calls", 0)  # noqa: E731
    # unfused: the residual add and the ReLU ran as ATen passes, and so did
    # BatchNorm's num_batches_tracked += 1, which the fused run advances
    # inside its statistics launch
    assert calls(fb, "aten::relu_") == 0 and calls(fp, "aten::relu_") == 1
    assert calls(fb, "aten::add_.Tensor") == 0 and calls(fp, "aten::add_.Tensor") == 2
    for k in fused:
        # the same roundings in the same order: bit-identical (zeros compared by value)
        assert torch.equal(fused[k].float(), plain[k].float()), k


def test_writes_into_a_pending_pass_inputs_run_it_first():
    """The folded pass reads x, the residual and the affine parameters when its
    output is first read: writes into any of them in between must not leak in."""
    torch.manual_seed(1)
    bn = nn.BatchNorm2d(32).bfloat16().to(X)
    x = torch.randn(2, 32, 6, 6).bfloat16()
    idn = torch.randn(2, 32, 6, 6).bfloat16()
    with torch.no_grad():
        ref = torch.relu(nn.functional.batch_norm(x.float(), None, None, bn.weight.float().cpu(),
                                                  bn.bias.float().cpu(), True) + idn.float())
        for write in (lambda xx, ii: xx.zero_(), lambda xx, ii: ii.mul_(0), lambda xx, ii: bn.weight.mul_(3),
                      lambda xx, ii: ii.copy_(torch.zeros_like(ii))):
            bn.weight.fill_(1.0)
            xx, ii = x.to(X), idn.to(X)
            y = bn(xx)
            y += ii
            y.relu_()
            write(xx, ii)
            assert (y.float().cpu() - ref).abs().max().item() <= 3e-2 * ref.abs().max().item()


# ---- the ReLU after a BatchNorm, recomputed in its backward -------------------

@pytest.mark.parametrize("shape", [(8, 64, 14, 14), (4, 256, 7, 7), (2, 2048, 3, 3), (16, 8, 5, 5)])
@pytest.mark.parametrize("pdtype", [0, 1])
def test_batch_norm_relu_bwd_abi_bit_exact(cuda, shape, pdtype):
    """b2_batch_norm_relu_bwd_bf16 (gate recomputed from x) against the two
    passes it replaces: ATen's threshold_backward(dy, y, 0) on the forward's
    ReLU output, then b2_batch_norm_bwd_bf16 -- bit for bit.  x carries exact
    zeros of the affine output, a NaN and an inf, so every branch of the gate
    is taken."""
    N, C, H, W = shape
    rng = np.random.default_rng(N + C + H)
    xn = rng.standard_normal(shape).astype(np.float32) * 1.3 + 0.2
    xn[0, 0, 0, 0] = np.nan
    xn[-1, -1, -1, -1] = np.inf
    x = torch.from_numpy(xn).bfloat16()
    dy = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).bfloat16()
    pt = torch.float32 if pdtype == 1 else torch.bfloat16
    w = torch.from_numpy(rng.uniform(0.5, 1.5, C).astype(np.float32)).to(pt)
    b = torch.from_numpy(rng.standard_normal(C).astype(np.float32) * 0.3).to(pt)
    if pdtype == 1:
        # channel 1: affine outputs z straddling 2^-134, where bf16(z) turns
        # from zero (the tie included) to the smallest positive bf16
        w[1] = 2.0 ** -140
        b[1] = 2.0 ** -134
    cl = torch.channels_last
    xd, dyd = x.to(cuda).contiguous(memory_format=cl), dy.to(cuda).contiguous(memory_format=cl)
    wd, bd = w.to(cuda), b.to(cuda)
    y = torch.empty_like(xd)
    sm = torch.empty(C, dtype=torch.float32, device=cuda)
    si = torch.empty_like(sm)
    nws = _abi.lib().b2_batch_norm_workspace_bytes(N, C, H * W, 1)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    _abi.call("b2_batch_norm_stats_bf16", xd.data_ptr(), 1, pdtype, None, None, pdtype, sm.data_ptr(), si.data_ptr(),
              N, C, H * W, ctypes.c_float(0.1), ctypes.c_float(1e-5), ws.data_ptr(), nws, st())
    _abi.call("b2_batch_norm_apply_bf16", xd.data_ptr(), 1, wd.data_ptr(), bd.data_ptr(), pdtype, sm.data_ptr(),
              si.data_ptr(), None, 1, y.data_ptr(), N, C, H * W, st())
    dz = torch.ops.aten.threshold_backward(dyd, y, 0)
    outs = {}
    for name, fn, g in (("plain", "b2_batch_norm_bwd_bf16", dz), ("fused", "b2_batch_norm_relu_bwd_bf16", dyd)):
        dx = torch.empty_like(xd)
        dw = torch.empty(C, dtype=pt, device=cuda)
        db = torch.empty_like(dw)
        if name == "plain":
            _abi.call(fn, g.data_ptr(), xd.data_ptr(), 1, wd.data_ptr(), pdtype, sm.data_ptr(), si.data_ptr(),
                      dx.data_ptr(), dw.data_ptr(), db.data_ptr(), pdtype, N, C, H * W, ws.data_ptr(), nws, st())
        else:
            _abi.call(fn, g.data_ptr(), xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), pdtype, sm.data_ptr(),
                      si.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), pdtype, N, C, H * W, ws.data_ptr(),
                      nws, st())
        torch.cuda.synchronize()
        outs[name] = (dx, dw, db)
    for a, b_ in zip(outs["plain"], outs["fused"]):
        assert torch.equal(a.view(torch.int16 if a.dtype == torch.bfloat16 else torch.int32),
                           b_.view(torch.int16 if b_.dtype == torch.bfloat16 else torch.int32))


def _relu_block(cl, gated, seed=3):
    """conv -> BatchNorm -> relu_ -> conv -> BatchNorm -> relu_ (torchvision's
    Bottleneck pattern), forward and backward on xdna; returns every gradient."""
    torch.manual_seed(seed)
    c1 = nn.Conv2d(32, 64, 3, padding=1, bias=False).bfloat16()
    b1 = nn.BatchNorm2d(64).bfloat16()
    c2 = nn.Conv2d(64, 64, 1, bias=False).bfloat16()
    b2 = nn.BatchNorm2d(64).bfloat16()
    with torch.no_grad():
        b1.weight.uniform_(0.5, 1.5)
        b1.bias.normal_(0, 0.3)
    x = torch.randn(4, 32, 12, 12).bfloat16()
    g = torch.randn(4, 64, 12, 12).bfloat16()
    mods = [m.to(X) for m in (c1, b1, c2, b2)]
    mf = torch.channels_last if cl else torch.contiguous_format
    for m in mods:
        m.to(memory_format=mf)
    xx = x.to(X).contiguous(memory_format=mf).requires_grad_()
    xdna_train.set_fusion(bn_epilogue=gated)
    out = mods[0](xx)
    out = mods[1](out)
    out.relu_()
    out = mods[2](out)
    out = mods[3](out)
    out.relu_()
    out.backward(g.to(X).contiguous(memory_format=mf))
    res = {"dx": xx.grad.cpu(), "dc1": mods[0].weight.grad.cpu(), "dg1": mods[1].weight.grad.cpu(),
           "db1": mods[1].bias.grad.cpu(), "dc2": mods[2].weight.grad.cpu(), "dg2": mods[3].weight.grad.cpu(),
           "db2": mods[3].bias.grad.cpu(), "y": out.detach().cpu()}
    return res


@pytest.mark.parametrize("cl", [False, True])
def test_relu_backward_folds_into_batch_norm_backward(cl):
    """threshold_backward of a BatchNorm output that folded the relu_ stays
    pending; the BatchNorm's backward recomputes the gate from x and never
    runs that pass (channels-last); the results equal the unfused run's bit
    for bit."""
    try:
        xdna_train.reset_fallback_stats()
        fused = _relu_block(cl, True)
        fb = xdna_train.fallback_stats()
        n_relu = launched("batch_norm.bwd_relu")
        xdna_train.reset_fallback_stats()
        plain = _relu_block(cl, False)
        fp = xdna_train.fallback_stats()
    finally:
        xdna_train.set_fusion(bn_epilogue=True)
    calls = lambda d, k: d.get(k, {}).get("calls", 0)  # noqa: E731
    if cl:
        assert n_relu > 0 and calls(fb, "aten::threshold_backward") == 0
    assert calls(fp, "aten::threshold_backward") + calls(fp, "aten::threshold_backward.grad_input") == 2
    for k in fused:
        assert torch.equal(fused[k].float(), plain[k].float()), k


def test_gated_gradient_read_elsewhere_runs_its_pass():
    """A hook that reads the pending ReLU input gradient runs its pass, and
    the BatchNorm backward then takes the plain path on it: same results."""
    torch.manual_seed(5)
    bn = nn.BatchNorm2d(16).bfloat16().to(X).to(memory_format=torch.channels_last)
    x = torch.randn(2, 16, 6, 6).bfloat16()
    g = torch.randn(2, 16, 6, 6).bfloat16()
    seen = []
    grads = []
    for hook in (False, True):
        xx = x.to(X).contiguous(memory_format=torch.channels_last).requires_grad_()
        y = bn(xx)
        if hook:
            y.register_hook(lambda t: seen.append(t.float().cpu()))
        y.relu_()
        y.backward(g.to(X).contiguous(memory_format=torch.channels_last))
        grads.append(xx.grad.cpu())
    assert seen and torch.equal(grads[0].float(), grads[1].float())


# ---- a residual block's gradient sum, fused with its ReLU backward ------------

@pytest.mark.parametrize("n", [8, 4096, 1 << 20])
def test_relu_bwd_sum_abi_bit_exact(cuda, n):
    """b2_relu_bwd_sum_bf16 against ATen's own two ops on the GPU -- a += b,
    then threshold_backward(a, y, 0) -- bit for bit, with y holding NaN, +0,
    -0 and negatives and a + b overflowing to inf and producing NaN."""
    g = torch.Generator().manual_seed(n)
    a = torch.randn(n, generator=g).bfloat16()
    b = torch.randn(n, generator=g).bfloat16()
    y = torch.randn(n, generator=g).bfloat16()
    y[:4] = torch.tensor([float("nan"), 0.0, -0.0, -1.0]).bfloat16()
    a[4:8] = torch.tensor([3e38, float("inf"), float("nan"), -3e38]).bfloat16()
    b[4:8] = torch.tensor([3e38, float("-inf"), 1.0, -3e38]).bfloat16()
    y[4:8] = 1.0
    ad, bd, yd = a.to(cuda), b.to(cuda), y.to(cuda)
    ref = torch.ops.aten.threshold_backward(ad.clone().add_(bd), yd, 0)
    dz = torch.empty_like(yd)
    _abi.call("b2_relu_bwd_sum_bf16", ad.data_ptr(), bd.data_ptr(), yd.data_ptr(), dz.data_ptr(), n, st())
    torch.cuda.synchronize()
    assert torch.equal(dz.view(torch.int16).cpu(), ref.view(torch.int16).cpu())


def _residual_stack(fused, seed=7):
    """stem conv -> BatchNorm -> relu_, then two residual blocks
    (conv -> BatchNorm -> += identity -> relu_) on channels-last xdna tensors:
    the blocks' inputs are used twice, so backward sums two gradients for each
    before the ReLU backward of the layer that made it."""
    torch.manual_seed(seed)
    convs = [nn.Conv2d(64, 64, 3, padding=1, bias=False).bfloat16() for _ in range(3)]
    bns = [nn.BatchNorm2d(64).bfloat16() for _ in range(3)]
    x = torch.randn(8, 64, 48, 48).bfloat16()
    g = torch.randn(8, 64, 48, 48).bfloat16()
    cl = torch.channels_last
    convs = [c.to(X).to(memory_format=cl) for c in convs]
    bns = [b.to(X) for b in bns]
    xx = x.to(X).contiguous(memory_format=cl).requires_grad_()
    xdna_train.set_fusion(bn_epilogue=fused)
    h = bns[0](convs[0](xx))
    h.relu_()
    for i in (1, 2):
        out = bns[i](convs[i](h))
        out += h
        out.relu_()
        h = out
    h.backward(g.to(X).contiguous(memory_format=cl))
    res = {"dx": xx.grad.cpu()}
    for i in range(3):
        res[f"dc{i}"] = convs[i].weight.grad.cpu()
        res[f"dg{i}"] = bns[i].weight.grad.cpu()
        res[f"db{i}"] = bns[i].bias.grad.cpu()
    return res


def test_gradient_sums_fold_into_relu_backward():
    """The block inputs' gradient sums stay pending, so does the ReLU backward
    that reads them, and the BatchNorm backward reading that adds, gates and
    reduces in one pass: every gradient equals the unfused run's bit for bit,
    and the separate add and ReLU-backward passes are gone."""
    try:
        xdna_train.reset_fallback_stats()
        fused = _residual_stack(True)
        fb = xdna_train.fallback_stats()
        n_sum = launched("relu_bwd_sum")
        n_bn_sum = launched("batch_norm.bwd_relu_sum")
        xdna_train.reset_fallback_stats()
        plain = _residual_stack(False)
        fp = xdna_train.fallback_stats()
    finally:
        xdna_train.set_fusion(bn_epilogue=True)
    calls = lambda d, k: d.get(k, {}).get("calls", 0)  # noqa: E731
    # both sums are made inside the BatchNorm backward that reads them
    assert n_sum == 0 and n_bn_sum == 2 * 3
    assert calls(fp, "aten::add_.Tensor") - calls(fb, "aten::add_.Tensor") >= 2
    for k in fused:
        assert torch.equal(fused[k].float(), plain[k].float()), k


@pytest.mark.parametrize("shape", [(8, 64, 14, 14), (4, 256, 7, 7), (2, 2048, 3, 3)])
@pytest.mark.parametrize("pdtype", [0, 1])
def test_batch_norm_bwd_relu_sum_abi_bit_exact(cuda, shape, pdtype):
    """b2_batch_norm_bwd_relu_sum_bf16 against b2_relu_bwd_sum_bf16 followed
    by b2_batch_norm_bwd_bf16: dz, dx, dw and db bit for bit (y with NaN and
    zeros, a + b overflowing)."""
    N, C, H, W = shape
    g = torch.Generator().manual_seed(N * C + H)
    # NHWC storage, viewed as channels-last NCHW
    flat = [torch.randn(N * H * W * C, generator=g).bfloat16() for _ in range(4)]
    flat[3][:3] = torch.tensor([float("nan"), 0.0, -0.0]).bfloat16()
    flat[1][5] = flat[2][5] = 3e38
    x, a, b, y = (f.to(cuda).view(N, H, W, C).permute(0, 3, 1, 2) for f in flat)
    assert x.is_contiguous(memory_format=torch.channels_last)
    pt = torch.float32 if pdtype == 1 else torch.bfloat16
    w = (torch.rand(C, generator=g) + 0.5).to(pt).to(cuda)
    sm = torch.randn(C, generator=g).to(cuda) * 0.1
    si = (torch.rand(C, generator=g) + 0.5).to(cuda)
    nws = _abi.lib().b2_batch_norm_workspace_bytes(N, C, H * W, 1)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    outs = {}
    for name in ("plain", "fused"):
        dz = torch.empty_like(x)
        dx = torch.empty_like(x)
        assert dz.stride() == x.stride()
        dw = torch.empty(C, dtype=pt, device=cuda)
        db = torch.empty_like(dw)
        if name == "plain":
            _abi.call("b2_relu_bwd_sum_bf16", a.data_ptr(), b.data_ptr(), y.data_ptr(), dz.data_ptr(), x.numel(), st())
            _abi.call("b2_batch_norm_bwd_bf16", dz.data_ptr(), x.data_ptr(), 1, w.data_ptr(), pdtype, sm.data_ptr(),
                      si.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), pdtype, N, C, H * W, ws.data_ptr(),
                      nws, st())
        else:
            _abi.call("b2_batch_norm_bwd_relu_sum_bf16", a.data_ptr(), b.data_ptr(), y.data_ptr(), x.data_ptr(),
                      w.data_ptr(), pdtype, sm.data_ptr(), si.data_ptr(), dz.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                      db.data_ptr(), pdtype, N, C, H * W, ws.data_ptr(), nws, st())
        torch.cuda.synchronize()
        outs[name] = (dz, dx, dw, db)
    for p_, f_ in zip(outs["plain"], outs["fused"]):
        iv = torch.int16 if p_.dtype == torch.bfloat16 else torch.int32
        assert torch.equal(p_.contiguous().view(iv).cpu(), f_.contiguous().view(iv).cpu())


# ---- the step counter advanced inside the statistics launch ------------------

@pytest.mark.parametrize("shape,layout", [((8, 64, 14, 14), 1), ((4, 24, 5, 7), 0), ((2, 2048, 3, 3), 1)])
def test_batch_norm_stats_count_abi(cuda, shape, layout):
    """b2_batch_norm_stats_count_bf16: the statistics and running statistics
    of b2_batch_norm_stats_bf16 bit for bit, and the counter advanced by the
    increment once per call (two calls in a row)."""
    N, C, H, W = shape
    rng = np.random.default_rng(C + H)
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32) * 2 + 0.5).bfloat16().to(cuda)
    if layout == 1:
        x = x.contiguous(memory_format=torch.channels_last)
    nws = _abi.lib().b2_batch_norm_workspace_bytes(N, C, H * W, layout)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    outs = []
    count = torch.tensor([41], dtype=torch.int64, device=cuda)
    for fn in ("b2_batch_norm_stats_bf16", "b2_batch_norm_stats_count_bf16"):
        rm = torch.full((C,), 0.25, dtype=torch.float32, device=cuda)
        rv = torch.full((C,), 2.0, dtype=torch.float32, device=cuda)
        sm, si = torch.empty_like(rm), torch.empty_like(rm)
        for _ in range(2):
            extra = (count.data_ptr(), 3) if fn.endswith("count_bf16") else ()
            _abi.call(fn, x.data_ptr(), layout, 1, rm.data_ptr(), rv.data_ptr(), 1, sm.data_ptr(), si.data_ptr(), N, C,
                      H * W, ctypes.c_float(0.1), ctypes.c_float(1e-5), *extra, ws.data_ptr(), nws, st())
        torch.cuda.synchronize()
        outs.append([t.cpu() for t in (sm, si, rm, rv)])
    for a, b in zip(*outs):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    assert int(count.item()) == 41 + 2 * 3
    L = _abi.lib()
    status = L.b2_batch_norm_stats_count_bf16(x.data_ptr(), layout, 1, None, None, 1, sm.data_ptr(), si.data_ptr(),
                                              N, C, H * W, ctypes.c_float(0.1), ctypes.c_float(1e-5), None, 1,
                                              ws.data_ptr(), nws, st())
    assert status != 0 and b"counter" in L.b2_last_error()


def test_num_batches_tracked_advances_inside_the_statistics_launch():
    """A training BatchNorm2d's num_batches_tracked.add_(1) takes no kernel of
    its own: the forward's statistics launch advances it (no add_ fallback);
    the count reads right after every step, after a read taken between the
    add_ and the forward (which runs the add first), and with momentum=None,
    whose forward reads the count itself."""
    torch.manual_seed(0)
    for momentum in (0.1, None):
        bn = nn.BatchNorm2d(32, momentum=momentum).bfloat16().to(X)
        ref = nn.BatchNorm2d(32, momentum=momentum).bfloat16()
        ref.load_state_dict({k: v.cpu() for k, v in bn.state_dict().items()})
        g = torch.Generator().manual_seed(3)
        xdna_train.reset_fallback_stats()
        for step in range(4):
            x = torch.randn(4, 32, 6, 6, generator=g).bfloat16()
            y = bn(x.to(X).contiguous(memory_format=torch.channels_last))
            ref(x)
            if momentum is not None and step < 3:
                assert "aten::add_.Tensor" not in xdna_train.fallback_stats(), xdna_train.fallback_stats()
            assert int(bn.num_batches_tracked.item()) == step + 1
            y.float().sum().item()
        torch.testing.assert_close(bn.running_mean.cpu(), ref.running_mean, rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(bn.running_var.cpu(), ref.running_var, rtol=2e-2, atol=2e-2)
    # a read between the increment and the forward runs the pending add
    bn = nn.BatchNorm2d(16).bfloat16().to(X)
    bn.num_batches_tracked.add_(5)
    assert int(bn.num_batches_tracked.item()) == 5
    bn(torch.randn(2, 16, 4, 4).bfloat16().to(X).contiguous(memory_format=torch.channels_last))
    assert int(bn.num_batches_tracked.item()) == 6
    # two increments with no forward between: both land
    bn.num_batches_tracked.add_(1)
    bn.num_batches_tracked.add_(2)
    bn(torch.randn(2, 16, 4, 4).bfloat16().to(X).contiguous(memory_format=torch.channels_last))
    assert int(bn.num_batches_tracked.item()) == 10
