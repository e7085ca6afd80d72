"""CPU checks of the benchmark models and of the host logic around them (no
GPU): the reference's own style-transfer network and loss as rebuilt in
bench.py (structure, a BF16 training step on the CPU path, the module pattern
``regions.fuse_perceptual_loss`` matches, and that a fused loss module falls
back to its own method on CPU tensors), and the fused loss's cache of its
normalisation constants."""
import torch

import bench
from xdna_train import regions


def _tiny_batch(b=2, hw=16):
    g = torch.Generator().manual_seed(0)
    x = (torch.rand(b, 3, hw, hw, generator=g) * 2 - 1).bfloat16()
    t = torch.rand(b, 3, hw, hw, generator=g).bfloat16()
    return x, t


def test_ref_stylenet_shapes_and_pairs():
    torch.manual_seed(0)
    net = bench.RefStyleNet().bfloat16()
    x, _ = _tiny_batch()
    y = net(x)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    # encoder (3) + first halves of the 5 residual blocks + decoder (2) + head
    pairs = net.norm_act_pairs()
    assert len(pairs) == 11
    assert all(isinstance(bn, torch.nn.BatchNorm2d) and isinstance(act, torch.nn.LeakyReLU) and act.negative_slope == 0.2
               for bn, act in pairs)
    # the head sees the decoder output, the first encoder map and the input: 128 + 64 + 3 channels
    assert net.head.conv.in_channels == 195 and net.out.kernel_size == (1, 1) and net.out.bias is not None


def test_ref_style_loss_training_step_on_cpu():
    torch.manual_seed(0)
    net = bench.RefStyleNet().bfloat16()
    crit = bench.RefStyleLoss().bfloat16()
    assert not any(p.requires_grad for p in crit.parameters())
    opt = torch.optim.Adam(net.parameters(), lr=1e-4, weight_decay=1e-5)
    x, t = _tiny_batch()
    losses = []
    for _ in range(2):
        loss = crit(net(x), t)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert all(v == v and v > 0 for v in losses)
    assert all(p.grad is not None for p in net.parameters())


def test_ref_style_loss_matches_region_pattern_and_falls_back_on_cpu():
    torch.manual_seed(0)
    crit = bench.RefStyleLoss().bfloat16()
    x, t = _tiny_batch()
    x = x.requires_grad_()
    plain = crit.compute_perceptual_loss(x, t)
    (gx,) = torch.autograd.grad(plain, x)
    assert regions.fuse_perceptual_loss(crit)
    # CPU tensors are not eligible for the fused region: the module's own method runs, bit for bit
    fused = crit.compute_perceptual_loss(x, t)
    (gf,) = torch.autograd.grad(fused, x)
    assert torch.equal(fused, plain) and torch.equal(gf, gx)


def test_norm_constants_are_cached_per_tensor_version():
    """The fused perceptual loss converts the normalisation's CPU mean / std
    once per device, dtype and tensor version, not on every call."""
    import types
    fp = regions._FusedPerceptual(torch.nn.Module(), "perceptual_vgg")
    mean = torch.tensor([0.485, 0.456, 0.406])
    std = torch.tensor([0.229, 0.224, 0.225])
    norm = types.SimpleNamespace(mean=mean, std=std)
    x = torch.ones(1, 3, 2, 2, dtype=torch.bfloat16)
    xn, tn = fp._normalised(norm, x, x)
    m1, s1 = fp.consts[3], fp.consts[4]
    assert m1.shape == (1, 3, 1, 1) and m1.dtype == torch.bfloat16
    assert torch.equal(m1.flatten(), mean.bfloat16()) and torch.equal(s1.flatten(), std.bfloat16())
    assert torch.equal(xn, (x - m1) / s1) and torch.equal(tn, xn)
    fp._normalised(norm, x, x)
    assert fp.consts[3] is m1 and fp.consts[4] is s1  # no second conversion
    mean.mul_(2.0)  # an in-place write bumps the version: converted again
    fp._normalised(norm, x, x)
    assert fp.consts[3] is not m1 and torch.equal(fp.consts[3].flatten(), mean.bfloat16())
    m3 = fp.consts[3]
    other = types.SimpleNamespace(mean=mean.clone(), std=std)  # another tensor object: not the cached one
    fp._normalised(other, x, x)
    assert fp.consts[3] is not m3
    fp._normalised(other, x.float(), x.float())  # the key includes the dtype
    assert fp.consts[3].dtype == torch.float32
    # constants that are not tensors are converted on every call (nothing cached)
    lists = types.SimpleNamespace(mean=[0.5, 0.5, 0.5], std=[0.2, 0.2, 0.2])
    keep = fp.consts
    a, _ = fp._normalised(lists, x, x)
    assert fp.consts is keep and torch.equal(a, (x - 0.5) / 0.2)


def test_conv_sweep_summary():
    """`bench.py --conv-sweep` totals: FLOPs and kernel time over the three
    directions; the large-channel fraction counts only C >= 256, H >= 36."""
    def row(b, c, hw, us, frac):
        fl = 2.0 * b * hw * hw * c * c * 9 / 1e9
        return {"shape": f"B{b} C{c} HW{hw}", "batch": b, "channels": c, "hw": hw, "gflop_per_direction": fl,
                **{k: {"us": us, "tflops": 0.0, "frac": frac} for k in ("fwd", "dgrad", "wgrad")}}
    rows = [row(8, 64, 18, 10.0, 0.1), row(128, 256, 36, 100.0, 0.8), row(128, 512, 18, 50.0, 0.5),
            row(40, 512, 72, 200.0, 0.9)]
    s = bench.sweep_summary(rows)
    gflop = sum(r["gflop_per_direction"] for r in rows) * 3
    assert s["shapes"] == 4 and abs(s["sum_gflop"] - round(gflop, 1)) < 1e-9 and s["sum_us"] == 1080.0
    assert abs(s["aggregate_tflops"] - round(gflop * 1e9 / 1080e-6 / 1e12, 1)) < 1e-9
    assert s["large_channel_min_frac"] == 0.8 and abs(s["large_channel_median_frac"] - 0.85) < 1e-12
    assert bench.sweep_summary([])["aggregate_tflops"] is None
