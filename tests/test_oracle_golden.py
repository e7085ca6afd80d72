"""The CPU oracle against vectors produced by the reference itself.

Golden files come from tests/golden/make_golden.py (the reference's
conv3x3w_host.py and its region_kernels.cpp / conv_pack.cpp compiled from
source).  Bit-exact for layouts and region kernels; the oracle's conv / wgrad /
GEMM are checked against the reference's CPU path (stock PyTorch CPU ops).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cpu_path, oracle

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def host():
    return np.load(GOLD / "conv3x3w_host.npz")


@pytest.fixture(scope="module")
def reg():
    return np.load(GOLD / "regions.npz")


def test_pack_rows_matches_reference_pack_input(host):
    for i in range(4):
        B, Cc, H, W, chunks = host[f"pack{i}_meta"]
        rows = oracle.pack_rows(host[f"pack{i}_x"], int(chunks))
        assert np.array_equal(rows, host[f"pack{i}_rows"]), i


def test_weight_k_order_matches_reference(host):
    for i in range(3):
        Cout, Cin, chunks = (int(v) for v in host[f"wfwd{i}_meta"])
        w = host[f"wfwd{i}_w"]
        wk = oracle.pack_weight(w, dgrad=False, chunks=chunks)  # [Cout][K]
        ref = host[f"wfwd{i}_wk"]  # [K][128]
        assert np.array_equal(wk.T, ref[:, :Cout]), i
        assert not ref[:, Cout:].any()


def test_dgrad_weight_k_order_matches_reference(host):
    seen = 0
    for i in range(3):
        if f"wdx{i}_wk" not in host.files:
            continue
        Cout, Cin, chunks_d = (int(v) for v in host[f"wdx{i}_meta"])
        wk = oracle.pack_weight(host[f"wfwd{i}_w"], dgrad=True, chunks=chunks_d)  # [Cin][K]
        ref = host[f"wdx{i}_wk"]
        assert np.array_equal(wk.T, ref[:, :Cin]), i
        seen += 1
    assert seen >= 2


def test_output_row_convention_matches_reference_unpack(host):
    """Output pixel (b,y,x) lives in padded row (b*(H+2)+y)*(W+2)+x."""
    for i in range(2):
        B, H, W, cout = (int(v) for v in host[f"unpack{i}_meta"])
        c = oracle.bf16_value(host[f"unpack{i}_c"]).reshape(-1, 128)
        y = np.empty((B, cout, H, W), np.float32)
        for b in range(B):
            for yy in range(H):
                for xx in range(W):
                    y[b, :, yy, xx] = c[(b * (H + 2) + yy) * (W + 2) + xx, :cout]
        assert np.array_equal(y, host[f"unpack{i}_y"])


@pytest.mark.parametrize("tag", ["even", "odd"])
def test_region_kernels_bit_exact(reg, tag):
    a, b, base = reg[f"{tag}_a"], reg[f"{tag}_b"], reg[f"{tag}_base"]
    assert np.array_equal(oracle.relu(a), reg[f"{tag}_relu"])
    r, p = oracle.relu_maxpool2(a)
    assert np.array_equal(r, reg[f"{tag}_relu_r"])
    assert np.array_equal(p, reg[f"{tag}_pool"])
    assert np.array_equal(oracle.addtap(base, a, b, 0.37), reg[f"{tag}_addtap"])
    assert np.array_equal(oracle.addtap(None, a, b, -1.5), reg[f"{tag}_addtap_nobase"])
    assert np.array_equal(oracle.relu_bwd(reg[f"{tag}_relu"], base, a, b, 0.25), reg[f"{tag}_relu_bwd"])
    assert np.array_equal(oracle.relu_bwd(reg[f"{tag}_relu"], base, None, None, 0.25), reg[f"{tag}_relu_bwd_notap"])
    assert np.array_equal(oracle.maxpool2_bwd(a, reg[f"{tag}_g"]), reg[f"{tag}_maxpool_bwd"])
    sq = oracle.sqdiff_sum(reg[f"{tag}_fin_a"], reg[f"{tag}_fin_b"])
    assert abs(sq - reg[f"{tag}_sqdiff"][0]) <= 1e-5 * abs(sq)


def _bf(t):
    return oracle.bf16_bits(t.float().numpy())


@pytest.mark.parametrize("shape", [(2, 70, 5, 7, 40, True), (1, 3, 6, 4, 10, True), (2, 64, 9, 9, 128, False)])
def test_oracle_conv_matches_reference_cpu_path(shape):
    B, Cin, H, W, Cout, bias = shape
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, Cin, H, W, generator=g).bfloat16()
    w = (torch.randn(Cout, Cin, 3, 3, generator=g) * (2.0 / (9 * Cin)) ** 0.5).bfloat16()
    bb = torch.randn(Cout, generator=g).bfloat16() if bias else None
    dy = torch.randn(B, Cout, H, W, generator=g).bfloat16()
    y_ref = cpu_path.conv3x3_fwd(x, w, bb).float().numpy()
    y = oracle.conv_fwd(_bf(x), _bf(w), None if bb is None else _bf(bb))
    dx_ref, dw_ref, _ = cpu_path.conv3x3_bwd(dy, x, w)
    dx = oracle.conv_dgrad(_bf(dy), _bf(w))
    dw = oracle.conv_wgrad(_bf(dy), _bf(x))
    for got, ref in ((y, y_ref), (dx, dx_ref.float().numpy()), (dw, dw_ref.float().numpy())):
        assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()


def test_oracle_gemm_and_adam():
    g = torch.Generator().manual_seed(1)
    a = torch.randn(33, 70, generator=g).bfloat16()
    b = torch.randn(70, 45, generator=g).bfloat16()
    c = torch.randn(33, 45, generator=g)
    d = oracle.gemm(_bf(a), _bf(b), c.numpy(), alpha=0.5, beta=2.0)
    ref = 0.5 * (a.double() @ b.double()) + 2.0 * c.double()
    assert np.abs(d - ref.numpy()).max() < 1e-3
    # Adam: oracle vs the reference CPU path's torch._fused_adam_ (fp32)
    p = torch.randn(1000, generator=g)
    gr = torch.randn(1000, generator=g)
    m = torch.randn(1000, generator=g).abs() * 0.1
    v = torch.randn(1000, generator=g).abs() * 0.1
    step = torch.tensor(3.0)
    P, G, M, V = (t.clone().numpy() for t in (p, gr, m, v))
    oracle.adam_f32(P, G, M, V, np.zeros_like(P), 3.0, 1e-3, 0.9, 0.999, 0.01, 1e-8, adamw=True)
    torch._fused_adamw_([p], [gr], [m], [v], [], [step], lr=1e-3, beta1=0.9, beta2=0.999, weight_decay=0.01,
                        eps=1e-8, amsgrad=False, maximize=False)
    assert np.abs(P - p.numpy()).max() <= 1e-6
    assert np.abs(M - m.numpy()).max() <= 1e-6


def _ulps(a, b):
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


def _bf_close(got, want, floor, exact=0.995):
    """One bf16 ulp, or `floor` absolutely for near-zero differences of larger
    terms; at least `exact` of the elements bit-equal."""
    g, w = oracle.bf16_value(got), oracle.bf16_value(want)
    assert (np.abs(g - w) <= np.abs(w) * 2.0 ** -7 + floor).all()
    assert (got == want).mean() >= exact


@pytest.fixture(scope="module")
def bn():
    return np.load(GOLD / "regions_bn.npz")


def test_bn_norm_activation_matches_reference(bn):
    """Fused BatchNorm + activation: the oracle against the reference's own host
    kernels (region_kernels.cpp:309-460).  The oracle's statistics are summed in
    double, the reference's plane sums in fp32, so outputs may differ by one bf16
    ulp where a value lies on a rounding boundary, or by a small absolute amount
    where the result is a near-zero difference of larger terms."""
    for i in range(int(bn["cases"][0])):
        N, Cc, H, W, relu, affine = (int(v) for v in bn[f"c{i}_meta"])
        slope = float(bn[f"c{i}_slope"][0])
        w = bn[f"c{i}_w"] if affine else None
        b = bn[f"c{i}_b"] if affine else None
        x = bn[f"c{i}_x"]
        y, mean, invstd, rm, rv = oracle.bn_fwd(x, w, b, bn[f"c{i}_rm"], bn[f"c{i}_rv"], 1e-5, slope, 0.1, True)
        np.testing.assert_allclose(mean, bn[f"c{i}_mean"], rtol=0, atol=2e-7 * max(1.0, np.abs(mean).max()))
        np.testing.assert_allclose(invstd, bn[f"c{i}_invstd"], rtol=3e-7)
        _bf_close(y, bn[f"c{i}_y"], 1e-5 * np.abs(oracle.bf16_value(bn[f"c{i}_y"])).max())
        assert _ulps(rm, bn[f"c{i}_rm_out"]).max() <= 1 and _ulps(rv, bn[f"c{i}_rv_out"]).max() <= 1
        # backward from the reference's own statistics, on an activation with planted 0 / NaN
        dx, dw, db = oracle.bn_bwd(bn[f"c{i}_dy"], bn[f"c{i}_ybwd"], x, w, bn[f"c{i}_mean"], bn[f"c{i}_invstd"],
                                   slope, bool(relu))
        _bf_close(dx, bn[f"c{i}_dx"], 1e-5 * np.abs(oracle.bf16_value(bn[f"c{i}_dx"])).max())
        _bf_close(dw, bn[f"c{i}_dw"], 2e-6 * N * H * W, exact=0.9)
        _bf_close(db, bn[f"c{i}_db"], 2e-6 * N * H * W, exact=0.9)


@pytest.mark.parametrize("opts", [dict(momentum=0.9), dict(momentum=0.9, weight_decay=1e-4, nesterov=True),
                                  dict(momentum=0.8, dampening=0.1, maximize=True), dict(weight_decay=1e-2)])
def test_oracle_sgd_matches_reference_cpu_fused_sgd_fp32(opts):
    """The oracle's fused-SGD restatement against the reference's CPU path
    for fp32 parameters (torch's CPU _fused_sgd_, reached by the reference
    through its boxed fallback): within a few fp32 rounding steps of the
    operands' magnitude (the CPU kernel forms its products in fp32, the
    definition here in double; under cancellation the fp32 rounding of a
    product shows at the product's scale).  torch 2.11's CPU _fused_sgd_ leaves
    most bf16 parameters unchanged, so bf16 is pinned on the GPU against
    ATen's CUDA kernel instead (tests/test_gpu_sgd.py)."""
    g = torch.Generator().manual_seed(5)
    p = torch.randn(4099, generator=g)
    gr = torch.randn(4099, generator=g)
    b = torch.randn(4099, generator=g)
    has_buf = opts.get("momentum", 0.0) != 0.0
    p0, g0, b0 = p.numpy().copy(), gr.numpy().copy(), b.numpy().copy()
    want_p, _, want_b = oracle.sgd_step(p.numpy().copy(), gr.numpy().copy(), b.numpy().copy() if has_buf else None,
                                        0.1, opts.get("weight_decay", 0.0), opts.get("momentum", 0.0),
                                        opts.get("dampening", 0.0), opts.get("nesterov", False),
                                        opts.get("maximize", False), False)
    torch._fused_sgd_([p], [gr], [b] if has_buf else [], weight_decay=opts.get("weight_decay", 0.0),
                      momentum=opts.get("momentum", 0.0), lr=0.1, dampening=opts.get("dampening", 0.0),
                      nesterov=opts.get("nesterov", False), maximize=opts.get("maximize", False), is_first_step=False)
    # magnitudes of the operands each result is formed from: cancellation
    # leaves the fp32 roundings of the products at that scale
    mb = opts.get("momentum", 0.0) * np.abs(b0) + np.abs(g0) + opts.get("weight_decay", 0.0) * np.abs(p0)
    mp = np.abs(p0) + 0.1 * (mb if has_buf else np.abs(g0) + opts.get("weight_decay", 0.0) * np.abs(p0))
    assert np.all(np.abs(p.numpy() - want_p) <= 4 * np.spacing(mp.astype(np.float32)))
    if has_buf:
        assert np.all(np.abs(b.numpy() - want_b) <= 4 * np.spacing(mb.astype(np.float32)))
