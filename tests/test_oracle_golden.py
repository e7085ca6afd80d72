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
