"""CUDA graphs of training steps on the xdna device (xdna_train.graphs): a
captured step replays the eager step's kernels on the same data, so a model
trained by replays ends bit-identical to the same model trained eagerly, and
the capture's private memory pool goes back to the allocator with the graph.
"""
import gc

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import xdna_train
from xdna_train import graphs

pytestmark = pytest.mark.gpu

X = torch.device("xdna")


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.c1 = nn.Conv2d(16, 64, 3, padding=1)
        self.bn = nn.BatchNorm2d(64)
        self.c2 = nn.Conv2d(64, 64, 3, padding=1)
        self.fc = nn.Linear(64, 10)

    def forward(self, x):
        y = torch.relu(self.bn(self.c1(x)))
        y = torch.relu(self.c2(y))
        return self.fc(y.mean((2, 3)))


def make():
    torch.manual_seed(0)
    net = Net().bfloat16().to(X)
    opt = torch.optim.Adam(net.parameters(), lr=1e-3, fused=True, capturable=True)
    return net, opt


def batches(n):
    g = torch.Generator().manual_seed(5)
    return [(torch.randn(8, 16, 12, 12, generator=g).bfloat16(), torch.randint(0, 10, (8,), generator=g))
            for _ in range(n)]


@pytest.fixture()
def fresh(cuda):
    xdna_train.register_xdna_device()
    xdna_train.set_npu_mode(2)
    yield


def test_replayed_steps_match_eager_steps(fresh):
    data = batches(6)
    warmup = 2
    # eager: warm-up steps on batch 0, then one step per later batch
    net_e, opt_e = make()
    seq = [data[0]] * warmup + data[1:]
    losses_e = []
    for xb, yb in seq:
        opt_e.zero_grad(set_to_none=True)
        loss = F.cross_entropy(net_e(xb.to(X)).float(), yb.to(X))
        loss.backward()
        opt_e.step()
        losses_e.append(loss.detach().cpu())
    # graphed: the same sequence through static inputs and replays
    net_g, opt_g = make()
    xs = data[0][0].to(X)
    ys = data[0][1].to(X)

    def step():
        opt_g.zero_grad(set_to_none=True)
        loss = F.cross_entropy(net_g(xs).float(), ys)
        loss.backward()
        opt_g.step()
        return loss.detach()

    replay = graphs.make_graphed_step(step, warmup=warmup)
    assert xdna_train.allocator_stats()["graph_pools"] >= 1
    losses_g = []
    for xb, yb in data[1:]:
        xs.copy_(xb.to(X))
        ys.copy_(yb.to(X))
        losses_g.append(replay().cpu().clone())
    torch.xdna.synchronize()
    for a, b in zip(losses_e[warmup:], losses_g):
        assert torch.equal(a, b), (a, b)
    for (n, pe), pg in zip(net_e.named_parameters(), net_g.parameters()):
        assert torch.equal(pe.detach().cpu(), pg.detach().cpu()), n
    assert torch.equal(net_e.bn.running_mean.cpu(), net_g.bn.running_mean.cpu())
    assert int(net_g.bn.num_batches_tracked.item()) == warmup + len(data) - 1
    kst = xdna_train.kernel_stats()
    assert kst.get("conv3x3.fwd", 0) > 0 and kst.get("fused_adam", 0) > 0


def test_graph_pool_is_released(fresh):
    net, opt = make()
    xs = torch.randn(8, 16, 12, 12).bfloat16().to(X)
    ys = torch.randint(0, 10, (8,)).to(X)

    def step():
        opt.zero_grad(set_to_none=True)
        F.cross_entropy(net(xs).float(), ys).backward()
        opt.step()

    before = xdna_train.allocator_stats()["graph_pools"]
    replay = graphs.make_graphed_step(step, warmup=2)
    replay()
    torch.xdna.synchronize()
    assert xdna_train.allocator_stats()["graph_pools"] == before + 1
    assert xdna_train.allocator_stats()["graph_pool_bytes"] > 0
    replay.graph.reset()
    # the pool's last tensors: the captured gradients, and the packed input
    # rows the captured forward attached to the static input for its dW
    opt.zero_grad(set_to_none=True)
    del replay, step, xs, ys
    gc.collect()
    torch.xdna.synchronize()
    assert xdna_train.allocator_stats()["graph_pools"] == before


def test_fused_perceptual_loss_with_host_norm_constants_is_capturable(fresh):
    """A loss whose normalisation keeps mean / std as CPU tensors (the
    reference's benchmark loss) copies them to the device on every eager call;
    the fused perceptual loss caches those copies, so a step through it can be
    captured, and a replay gives the eager loss and input gradient."""
    import bench
    from xdna_train import regions
    torch.manual_seed(0)
    crit = bench.RefStyleLoss().bfloat16().to(X)
    assert regions.fuse_perceptual_loss(crit)
    g = torch.Generator().manual_seed(2)
    x = (torch.rand(2, 3, 16, 16, generator=g) * 2 - 1).bfloat16().to(X).requires_grad_()
    t = torch.rand(2, 3, 16, 16, generator=g).bfloat16().to(X)

    def step():
        x.grad = None
        loss = crit(x, t)
        loss.backward()
        return loss

    le = step().detach().float().cpu()
    ge = x.grad.detach().float().cpu()
    replay = graphs.make_graphed_step(step, warmup=2)
    lr = replay()
    torch.xdna.synchronize()
    assert torch.allclose(lr.detach().float().cpu(), le, rtol=1e-2, atol=0)
    assert torch.allclose(x.grad.detach().float().cpu(), ge, rtol=2e-2, atol=1e-4)
    assert xdna_train.kernel_stats().get("region.sqdiff_sum", 0) > 0
