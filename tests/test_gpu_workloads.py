"""BASELINE configs 1, 3, 4 and 5 end to end on the `xdna` device, each
against the same seeded run on the reference's CPU BF16 path (stock PyTorch
CPU ops).  Config 1 checks the north-star bar literally: a 200-step loss curve
within 1 % relative.  The others run a few steps at reduced batch (the CPU side
has to finish in seconds) and compare the loss trajectories."""
import copy

import pytest
import torch
import torch.nn.functional as F

import bench
import xdna_train

pytestmark = pytest.mark.gpu
X = torch.device("xdna")


@pytest.fixture(autouse=True)
def _reg(cuda):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    xdna_train.reset_mapped_cpu_stats()


def _rel(a, b):
    return abs(a - b) / max(abs(b), 1e-12)


def test_config1_readme_200_step_loss_curve_within_1pct():
    """Both sides run the fused Adam: on xdna the reference's own pre-hook
    (device.py:408-436) selects it, so its CPU path runs torch's CPU fused
    kernel.  (PyTorch's single-tensor Adam alone differs from the fused one by
    2.3 % at step 83 of this curve, CPU against CPU.)"""
    def run(dev):
        torch.manual_seed(0)
        model = torch.nn.Conv2d(128, 128, 3, padding=1).bfloat16().to(dev)
        opt = torch.optim.Adam(model.parameters(), lr=1e-3, fused=True)
        g = torch.Generator().manual_seed(1)
        x = torch.randn(16, 128, 36, 36, generator=g).bfloat16().to(dev)
        tgt = torch.zeros_like(x)
        losses = []
        for _ in range(200):
            opt.zero_grad(set_to_none=True)
            loss = F.mse_loss(model(x).float(), tgt.float())
            loss.backward()
            opt.step()
            losses.append(loss.detach())
        return torch.stack([l.float().cpu() for l in losses])
    lc, lx = run("cpu"), run(X)
    rel = ((lx - lc).abs() / lc.abs()).max().item()
    assert rel <= 0.01, f"max relative loss gap {rel}"
    assert xdna_train.kernel_stats().get("conv3x3.wgrad", 0) >= 200


def test_config3_mlp_autocast_fp32_master():
    def run(dev, kind):
        torch.manual_seed(0)
        model = bench.make_mlp().to(dev)
        opt = torch.optim.Adam(model.parameters(), lr=1e-4, fused=True)
        g = torch.Generator().manual_seed(1)
        x = torch.randn(128, 1024, generator=g).to(dev)
        tgt = torch.randn(128, 1024, generator=g).to(dev)
        out = []
        for _ in range(8):
            opt.zero_grad(set_to_none=True)
            with torch.autocast(kind, dtype=torch.bfloat16):
                loss = F.mse_loss(model(x).float(), tgt)
            loss.backward()
            opt.step()
            out.append(loss.item())
        return out, model
    lc, mc = run("cpu", "cpu")
    lx, mx = run(X, "xdna")
    for a, b in zip(lx, lc):
        assert _rel(a, b) <= 0.01, (lx, lc)
    assert mx[0].weight.dtype == torch.float32  # FP32 master weights
    assert xdna_train.kernel_stats().get("gemm", 0) >= 8 * 11  # 4 fwd + 3 dX + 4 dW per step
    assert "addmm" not in xdna_train.fallback_stats() and "mm" not in xdna_train.fallback_stats()


@pytest.mark.parametrize("fused", [False, True])
def test_config4_style_transfer_steps(fused):
    from xdna_train import regions

    def run(dev, fuse):
        torch.manual_seed(0)
        gen = bench.make_style_generator().bfloat16().to(dev)
        crit = bench.StyleLoss().bfloat16().to(dev)
        if fuse:
            assert regions.fuse_perceptual_loss(crit)
        opt = torch.optim.Adam(gen.parameters(), lr=1e-3, fused=True)
        g = torch.Generator().manual_seed(1)
        x, tgt, sty = (torch.rand(4, 3, 36, 36, generator=g).bfloat16().to(dev) for _ in range(3))
        out = []
        for _ in range(3):
            opt.zero_grad(set_to_none=True)
            loss = crit(gen(x), tgt, sty)
            loss.backward()
            opt.step()
            out.append(loss.item())
        return out
    lc = run("cpu", False)
    lx = run(X, fused)
    for a, b in zip(lx, lc):
        assert _rel(a, b) <= 0.03, (lx, lc)
    ks = xdna_train.kernel_stats()
    assert ks.get("conv3x3.fwd", 0) > 0 and ks.get("gemm", 0) > 0
    if fused:
        assert ks.get("region.relu_maxpool2", 0) > 0 and ks.get("region.sqdiff_sum", 0) > 0


@pytest.mark.parametrize("fused", [False, True])
def test_config4_reference_stylenet_steps(fused, monkeypatch):
    """The reference's own benchmark network and loss (LeakyReLU(0.2), skip
    concatenations, a 195-channel 3x3 conv, a 1x1 output conv; perceptual taps
    0, 3, 5 of ImageNet-normalised images plus L1; Adam lr 1e-4 wd 1e-5), with
    the perceptual region and every BatchNorm+LeakyReLU pair fused or not,
    against the same seeded steps on the CPU BF16 path."""
    from xdna_train import regions
    monkeypatch.setattr(regions, "NORM_ACT_MIN_BYTES", 0)

    def run(dev, fuse):
        torch.manual_seed(0)
        net = bench.RefStyleNet().bfloat16().to(dev)
        crit = bench.RefStyleLoss().bfloat16().to(dev)
        if fuse:
            assert regions.fuse_perceptual_loss(crit)
            for bn, act in net.norm_act_pairs():
                assert regions.fuse_norm_activation(bn, act)
        opt = torch.optim.Adam(net.parameters(), lr=1e-4, weight_decay=1e-5, fused=True)
        g = torch.Generator().manual_seed(1)
        x = (torch.rand(4, 3, 36, 36, generator=g) * 2 - 1).bfloat16().to(dev)
        tgt = torch.rand(4, 3, 36, 36, generator=g).bfloat16().to(dev)
        out = []
        for _ in range(3):
            loss = crit(net(x), tgt)
            opt.zero_grad(set_to_none=True)
            loss.backward()
            opt.step()
            out.append(loss.item())
        return out
    lc = run("cpu", False)
    k0 = dict(xdna_train.kernel_stats())
    lx = run(X, fused)
    for a, b in zip(lx, lc):
        assert _rel(a, b) <= 0.03, (lx, lc)
    ks = xdna_train.kernel_stats()
    ran = lambda k: ks.get(k, 0) - k0.get(k, 0)  # noqa: E731
    assert ran("conv3x3.fwd") > 0 and ran("conv3x3.dgrad") > 0 and ran("fused_adam") > 0
    if fused:
        assert ran("region.sqdiff_sum") > 0 and ran("region.bn_fwd") > 0 and ran("region.bn_bwd") > 0


def test_config5_resnet50_steps():
    """ResNet-50 (BASELINE config 5 at batch 4) against an fp32 CPU reference,
    with the reference's own kind of gate (the fused path's error no larger
    than 1.5x the CPU bf16 path's, tests/run_regions_bn.py): the first step's
    loss and the whole gradient vector; then three SGD steps lower the loss.
    In bf16 every BatchNorm output is rounded once, and 53 BatchNorms over
    batch-4 statistics compound those roundings into gradient differences of
    order one between any two bf16 implementations, so bf16 is compared with
    fp32, not with another bf16 run."""
    from torchvision.models import resnet50

    def run(dev, dtype, steps=3):
        torch.manual_seed(0)
        model = resnet50(num_classes=1000).to(dtype).to(dev).to(memory_format=torch.channels_last)
        # single-tensor SGD on every side: torch 2.11's CPU _fused_sgd_ leaves
        # bf16 parameters unchanged, so the CPU side cannot use the fused kernel
        opt = torch.optim.SGD(model.parameters(), lr=0.01, momentum=0.9, foreach=False, fused=False)
        g = torch.Generator().manual_seed(1)
        x = torch.randn(4, 3, 224, 224, generator=g).bfloat16().to(dtype).to(dev)
        x = x.contiguous(memory_format=torch.channels_last)
        y = torch.randint(0, 1000, (4,), generator=g).to(dev)
        out, grads = [], None
        for i in range(steps):
            opt.zero_grad(set_to_none=True)
            loss = F.cross_entropy(model(x).float(), y)
            loss.backward()
            if i == 0:
                grads = torch.cat([p.grad.detach().float().cpu().reshape(-1) for p in model.parameters()])
            opt.step()
            out.append(loss.item())
        return out, grads
    l32, g32 = run("cpu", torch.float32, steps=1)
    lc, gc = run("cpu", torch.bfloat16)
    lx, gx = run(X, torch.bfloat16)

    def err(g):
        return ((g - g32).norm() / g32.norm()).item()
    e_cpu, e_x = err(gc), err(gx)
    assert abs(lx[0] - l32[0]) <= 1.5 * abs(lc[0] - l32[0]) + 0.01 * abs(l32[0]), (lx[0], lc[0], l32[0])
    assert e_x <= 1.5 * e_cpu + 0.05, (e_x, e_cpu)
    assert lx[2] < lx[0] and lc[2] < lc[0], (lx, lc)
    ks = xdna_train.kernel_stats()
    assert ks.get("conv3x3.fwd", 0) >= 12 and ks.get("conv3x3.wgrad", 0) > 0 and ks.get("batch_norm.fwd", 0) > 0
