"""Layout ops with xdna kernels (cat, nearest-2x upsample and its backward)
against ATen on the CPU, bit for bit -- the reference's own contract for its
fast host versions (tests/run_fast_layout_ops.py: copies exact, the backward's
2x2 sums in ATen's fp32 order).  Shapes follow that test: several dims and
sizes including odd, size-1 and empty ones, channels-last, explicit scales,
-0.0 gradients, and the cases that must take the ATen path (3x, arbitrary
sizes, non-contiguous), plus a cat + upsample model trained against the CPU.
"""
import pytest
import torch
import torch.nn as nn
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


def same(a, b):
    a, b = a.cpu(), b.cpu()
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    view = {2: torch.int16, 4: torch.int32, 1: torch.uint8, 8: torch.int64}[a.element_size()]
    return torch.equal(a.contiguous().view(view), b.contiguous().view(view))


def rnd(*shape, dt):
    return (torch.randn(*shape) * 3).to(dt)


def launched(kind):
    return xdna_train.kernel_stats().get(kind, 0)


def fallbacks(op):
    return xdna_train.fallback_stats().get(op, {}).get("calls", 0)


DTYPES = [torch.bfloat16, torch.float32]


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shapes,dim", [
    ([(40, 128, 36, 36), (40, 64, 36, 36), (40, 3, 36, 36)], 1),
    ([(2, 5, 7, 9), (2, 1, 7, 9)], 1),
    ([(3, 4, 5, 6), (3, 4, 5, 2)], 3),
    ([(3, 4, 5, 6), (1, 4, 5, 6)], 0),
    ([(3, 4, 5, 6), (3, 4, 2, 6), (3, 4, 1, 6)], -2),
    ([(1, 1, 1, 1), (1, 3, 1, 1)], 1),
    ([(2, 0, 3, 3), (2, 4, 3, 3)], 1),
    ([(6, 7), (6, 2)], 1),
])
def test_cat_bit_exact(dt, shapes, dim):
    ts = [rnd(*s, dt=dt) for s in shapes]
    got = torch.cat([t.to(X) for t in ts], dim)
    assert same(got, torch.cat(ts, dim))
    assert launched("cat") >= 1


@pytest.mark.parametrize("dt", DTYPES)
def test_cat_layouts_and_fallbacks(dt):
    a, b = rnd(2, 6, 5, 5, dt=dt), rnd(2, 3, 5, 5, dt=dt)
    cl = torch.channels_last
    got = torch.cat([a.to(X).contiguous(memory_format=cl), b.to(X).contiguous(memory_format=cl)], 1)
    assert same(got, torch.cat([a.contiguous(memory_format=cl), b.contiguous(memory_format=cl)], 1))
    assert got.is_contiguous(memory_format=cl)
    for d in (0, 2, 3):  # channels-last along the other dims
        assert same(torch.cat([a.to(X).contiguous(memory_format=cl)] * 2, d),
                    torch.cat([a.contiguous(memory_format=cl)] * 2, d))
    n_fast = launched("cat")
    assert same(torch.cat([a.to(X).transpose(2, 3), b.to(X).transpose(2, 3)], 1),
                torch.cat([a.transpose(2, 3), b.transpose(2, 3)], 1))
    assert same(torch.cat([a.to(X)[:, ::2], b.to(X)], 1), torch.cat([a[:, ::2], b], 1))
    assert launched("cat") == n_fast and fallbacks("aten::cat") == 2


def test_cat_many_sources_odd_bytes_and_mixed_dtypes():
    # > 32 sources (several launches), 1- and 2-byte units, legacy empty tensors
    parts = [torch.randint(0, 255, (3, k % 5 + 1, 7), dtype=torch.uint8) for k in range(45)]
    assert same(torch.cat([p.to(X) for p in parts], 1), torch.cat(parts, 1))
    h = [rnd(5, k + 1, dt=torch.float16) for k in range(3)] + [torch.empty(0, dtype=torch.float16)]
    assert same(torch.cat([t.to(X) for t in h], 1), torch.cat(h, 1))
    m = [rnd(2, 3, dt=torch.bfloat16), rnd(2, 2, dt=torch.float32)]
    assert same(torch.cat([t.to(X) for t in m], 1), torch.cat(m, 1))


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", [(40, 256, 18, 18), (2, 5, 7, 9), (1, 1, 1, 1), (3, 7, 4, 1), (2, 64, 3, 5),
                                   (4, 16, 8, 8)])
@pytest.mark.parametrize("cl", [False, True])
def test_upsample_nearest2x_fwd_bwd_bit_exact(dt, shape, cl):
    n, c, h, w = shape
    x = rnd(n, c, h, w, dt=dt)
    if cl:
        x = x.contiguous(memory_format=torch.channels_last)
    ref = F.interpolate(x, scale_factor=2, mode="nearest")
    got = F.interpolate(x.to(X), scale_factor=2, mode="nearest")
    assert same(got, ref)
    assert got.is_contiguous(memory_format=torch.channels_last if cl and c > 1 else torch.contiguous_format)
    ref = torch.ops.aten.upsample_nearest2d(x, [2 * h, 2 * w], None, None)
    assert same(torch.ops.aten.upsample_nearest2d(x.to(X), [2 * h, 2 * w], 2.0, 2.0), ref)
    g = rnd(n, c, 2 * h, 2 * w, dt=dt)
    g = g.masked_fill(torch.rand(g.shape) < 0.3, -0.0)  # ATen's sum starts at +0
    if cl:
        g = g.contiguous(memory_format=torch.channels_last)
    ref = torch.ops.aten.upsample_nearest2d_backward(g, [2 * h, 2 * w], [n, c, h, w], None, None)
    got = torch.ops.aten.upsample_nearest2d_backward(g.to(X), [2 * h, 2 * w], [n, c, h, w], None, None)
    assert same(got, ref)
    assert launched("upsample_nearest2x") >= 2 and launched("upsample_nearest2x_backward") >= 1
    assert "aten::upsample_nearest2d" not in xdna_train.fallback_stats()


@pytest.mark.parametrize("dt", DTYPES)
def test_upsample_cases_for_the_aten_path(dt):
    x = rnd(2, 3, 5, 6, dt=dt)
    assert same(F.interpolate(x.to(X), scale_factor=3, mode="nearest"), F.interpolate(x, scale_factor=3, mode="nearest"))
    assert same(F.interpolate(x.to(X), size=(11, 12), mode="nearest"), F.interpolate(x, size=(11, 12), mode="nearest"))
    xt = x.transpose(2, 3)
    assert same(F.interpolate(xt.to(X), scale_factor=2, mode="nearest"),
                F.interpolate(xt, scale_factor=2, mode="nearest"))
    g = rnd(2, 3, 10, 12, dt=dt).transpose(2, 3)
    assert same(torch.ops.aten.upsample_nearest2d_backward(g.to(X), [12, 10], [2, 3, 6, 5], None, None),
                torch.ops.aten.upsample_nearest2d_backward(g, [12, 10], [2, 3, 6, 5], None, None))
    g3 = rnd(2, 3, 15, 18, dt=dt)
    assert same(torch.ops.aten.upsample_nearest2d_backward(g3.to(X), [15, 18], [2, 3, 5, 6], None, None),
                torch.ops.aten.upsample_nearest2d_backward(g3, [15, 18], [2, 3, 5, 6], None, None))
    assert fallbacks("aten::upsample_nearest2d") == 3


def test_upsample_backward_nan_and_inf():
    g = rnd(2, 4, 6, 8, dt=torch.float32)
    g[0, 0, 0, 0] = float("nan")
    g[0, 1, 2, 3] = float("inf")
    g[0, 1, 3, 3] = float("-inf")
    g[1, 2, 4, 5] = float("-nan")
    for dt in DTYPES:
        gd = g.to(dt)
        ref = torch.ops.aten.upsample_nearest2d_backward(gd, [6, 8], [2, 4, 3, 4], None, None)
        got = torch.ops.aten.upsample_nearest2d_backward(gd.to(X), [6, 8], [2, 4, 3, 4], None, None)
        assert same(got, ref)


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.c1 = nn.Conv2d(3, 8, 3, padding=1)
        self.c2 = nn.Conv2d(8 + 3 + 8, 4, 3, padding=1)

    def forward(self, x):
        a = torch.relu(self.c1(x))
        up = F.interpolate(F.avg_pool2d(a, 2), scale_factor=2, mode="nearest")
        return self.c2(torch.cat([a, x, up], 1))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_cat_upsample_model_autograd_vs_cpu(dt):
    torch.manual_seed(0)
    m = _Net().to(dt)
    m2 = _Net().to(dt)
    m2.load_state_dict(m.state_dict())
    m2 = m2.to(X)
    x = torch.randn(4, 3, 12, 12).to(dt)
    xr, xg = x.clone().requires_grad_(), x.to(X).requires_grad_()
    yr, yg = m(xr), m2(xg)
    w = torch.randn_like(yr)
    yr.backward(w)
    yg.backward(w.to(X))
    tol = 3e-2 if dt == torch.bfloat16 else 1e-4

    def rel(a, b):
        return ((a.float().cpu() - b.float()).norm() / b.float().norm()).item()

    errs = [rel(yg.detach(), yr.detach()), rel(xg.grad, xr.grad)]
    errs += [rel(p2.grad, p1.grad) for p1, p2 in zip(m.parameters(), m2.parameters())]
    assert max(errs) < tol, errs
    # the upsample's incoming gradient is a channel slice of cat's: not
    # contiguous, so its backward takes the ATen path (as in the reference)
    assert launched("cat") >= 1 and launched("upsample_nearest2x") >= 1
