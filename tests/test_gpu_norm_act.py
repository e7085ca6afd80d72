"""regions.fuse_norm_activation on the xdna device: the fused training
BatchNorm2d + ReLU/LeakyReLU against the eager pair on xdna and an fp32 CPU
reference, with the reference's own gate (tests/run_regions_bn.py:76-87): the
fused error vs fp32 is at most 1.5x the eager error plus 6e-3, for the output,
dX, dW, dB and the running statistics, over three steps.  Then the pairing
guard and the fallbacks the reference's test checks (run_regions_bn.py:91-151).
"""
import copy

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import xdna_train
from xdna_train import regions

pytestmark = pytest.mark.gpu

X = torch.device("xdna")


@pytest.fixture(autouse=True)
def _fresh(cuda, monkeypatch):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    xdna_train.reset_fallback_stats()
    monkeypatch.setattr(regions, "NORM_ACT_MIN_BYTES", 0)
    yield


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def make_pair(C, slope, seed):
    torch.manual_seed(seed)
    bn = nn.BatchNorm2d(C)
    with torch.no_grad():
        bn.weight.uniform_(0.5, 1.5)
        bn.bias.normal_(0, 0.3)
        bn.running_mean.normal_(0, 0.1)
        bn.running_var.uniform_(0.5, 1.5)
    return bn, (nn.LeakyReLU(slope) if slope > 0 else nn.ReLU())


@pytest.mark.parametrize("N,C,H,W,slope", [(8, 64, 18, 18, 0.2), (4, 128, 9, 9, 0.2), (2, 3, 5, 7, 0.2),
                                           (1, 16, 6, 6, 0.2), (3, 1, 4, 4, 0.2), (6, 32, 11, 13, 0.0),
                                           (40, 64, 36, 36, 0.2)])
def test_fused_pair_gate_vs_eager(N, C, H, W, slope):
    bn32, act32 = make_pair(C, slope, 1)
    steps = 3
    gen = torch.Generator().manual_seed(N * 1000 + C)
    xs = [torch.randn(N, C, H, W, generator=gen) * 1.5 + 0.3 for _ in range(steps)]
    gs = [torch.randn(N, C, H, W, generator=gen) for _ in range(steps)]
    ref = copy.deepcopy(bn32)
    ref_y, ref_dx = [], []
    for x, g in zip(xs, gs):
        xr = x.bfloat16().float().requires_grad_()
        y = act32(ref(xr))
        y.backward(g.bfloat16().float())
        ref_y.append(y.detach())
        ref_dx.append(xr.grad)
    runs = {}
    for mode in ("eager", "fused"):
        bn = copy.deepcopy(bn32).to(X, torch.bfloat16)
        act = copy.deepcopy(act32)
        if mode == "fused":
            assert regions.fuse_norm_activation(bn, act)
        ys, dxs = [], []
        for x, g in zip(xs, gs):
            xd = x.bfloat16().to(X).requires_grad_()
            y = act(bn(xd))
            y.backward(g.bfloat16().to(X))
            ys.append(y.detach())
            dxs.append(xd.grad)
        runs[mode] = (ys, dxs, bn)
    if N * H * W > 1:
        assert xdna_train.kernel_stats().get("region.bn_fwd", 0) >= 3 * steps

    def errors(mode):
        ys, dxs, bn = runs[mode]
        return (max(rel(a, b) for a, b in zip(ys, ref_y)), max(rel(a, b) for a, b in zip(dxs, ref_dx)),
                rel(bn.weight.grad, ref.weight.grad), rel(bn.bias.grad, ref.bias.grad),
                rel(bn.running_mean, ref.running_mean), rel(bn.running_var, ref.running_var))

    ee, ef = errors("eager"), errors("fused")
    for name, e, f in zip(("y", "dx", "dW", "dB", "running_mean", "running_var"), ee, ef):
        assert f <= 1.5 * e + 6e-3, f"{name}: fused {f:.5f} vs eager {e:.5f}"
    assert int(runs["fused"][2].num_batches_tracked) == steps == int(runs["eager"][2].num_batches_tracked)


def test_pairing_guard_and_fallbacks():
    bn, act = make_pair(8, 0.2, 2)
    bn = bn.to(X, torch.bfloat16)
    bn_e, act_e = copy.deepcopy(bn), copy.deepcopy(act)  # eager twin, never paired
    assert regions.fuse_norm_activation(bn, act)
    assert regions.fuse_norm_activation(bn, act)            # idempotent
    assert not regions.fuse_norm_activation(bn, nn.ReLU())  # already paired with another act
    x = torch.randn(4, 8, 6, 6).bfloat16().to(X)
    assert rel(act(bn(x)), act_e(bn_e(x))) < 0.02            # activation applied exactly once
    # the tag is consumed: a second activation call on the same tensor activates
    y = bn(x)
    bn_e(x)  # keep the twin's running statistics in step
    assert act(y) is y and rel(act(y), F.leaky_relu(y, 0.2)) == 0.0
    bn.eval()
    bn_e.eval()
    assert rel(act(bn(x)), act_e(bn_e(x))) < 0.01           # eval mode: eager pair
    bn.train()
    bn_e.train()
    xt = torch.randn(4, 6, 6, 8).bfloat16().to(X).transpose(1, 3)
    yt = bn(xt)
    assert not regions.activation_pending(yt)                # non-contiguous: eager
    assert rel(act(yt), act_e(bn_e(xt))) < 0.01
    other = nn.BatchNorm2d(4, affine=False).to(X, torch.bfloat16)
    assert regions.fuse_norm_activation(other, nn.ReLU())
    assert other(torch.randn(2, 4, 3, 3).bfloat16().to(X)) is not None  # affine=False runs eagerly
    assert not regions.fuse_norm_activation(nn.BatchNorm2d(4), nn.Sigmoid())
    mom = nn.BatchNorm2d(4, momentum=None).to(X, torch.bfloat16)
    relu = nn.ReLU()
    regions.fuse_norm_activation(mom, relu)
    xm = torch.randn(2, 4, 3, 3).bfloat16().to(X)
    want = torch.relu(F.batch_norm(xm.cpu().float(), None, None, mom.weight.float().cpu(), mom.bias.float().cpu(),
                                   True, 0.1, mom.eps))
    assert rel(relu(mom(xm)), want) < 0.02                    # momentum=None: eager
    neg = nn.BatchNorm2d(8).to(X, torch.bfloat16)
    leak = nn.LeakyReLU(-0.1)
    regions.fuse_norm_activation(neg, leak)
    assert not regions.activation_pending(neg(x))            # negative slope: eager


def test_inplace_change_of_saved_input_detected():
    bn, act = make_pair(8, 0.2, 3)
    bn = bn.to(X, torch.bfloat16)
    regions.fuse_norm_activation(bn, act)
    xi = torch.randn(4, 8, 6, 6).bfloat16().to(X).requires_grad_()
    yi = act(bn(xi))
    with torch.no_grad():
        xi.mul_(2)
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        yi.sum().backward()


def test_size_threshold(monkeypatch):
    monkeypatch.setattr(regions, "NORM_ACT_MIN_BYTES", 4_000_000)
    bs, a_s = make_pair(8, 0.2, 3)
    bs = bs.to(X, torch.bfloat16)
    regions.fuse_norm_activation(bs, a_s)
    assert not regions.activation_pending(bs(torch.randn(2, 8, 4, 4).bfloat16().to(X)))
    bb, ab = make_pair(64, 0.2, 4)
    bb = bb.to(X, torch.bfloat16)
    regions.fuse_norm_activation(bb, ab)
    assert regions.activation_pending(bb(torch.randn(40, 64, 36, 36).bfloat16().to(X)))


def test_deepcopy_keeps_a_working_pair():
    bn, act = make_pair(16, 0.0, 5)
    model = nn.Sequential(bn, act).to(X, torch.bfloat16)
    regions.fuse_norm_activation(model[0], model[1])
    twin = copy.deepcopy(model)
    x = torch.randn(4, 16, 10, 10).bfloat16().to(X)
    y = twin(x)
    assert rel(y, model(x)) < 1e-2
    assert regions.paired_activation(twin[0]) is twin[1]
