"""Generate the golden vectors of tests/golden/ from the reference itself.

Run here (where the reference tree is mounted) with
    python tests/golden/make_golden.py [--ref /root/reference]
It needs the reference's numpy host-layout spec
(xdna_train/_designs/conv3x3w_host.py, imported from the reference tree) and
the reference's own C++ host kernels compiled from their sources by
``make -C oracle`` (oracle/_ref/libxdna_ref.so).  The outputs are small .npz
files that the tests read on any machine; the GPU box never needs the
reference.

Files
  conv3x3w_host.npz  pack_input (rows view), pack_weights / pack_weights_dx
                     (decoded K x N matrices), unpack_output cases
  regions.npz        region kernel inputs/outputs from region_kernels.cpp
  regions_bn.npz     fused BatchNorm + activation vectors from region_kernels.cpp:309-460
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import oracle  # noqa: E402


def load_host_spec(ref: Path):
    path = ref / "xdna_train" / "_designs" / "conv3x3w_host.py"
    spec = importlib.util.spec_from_file_location("conv3x3w_host", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def rows_from_groups(packed: np.ndarray, m_total: int, group_out_rows: int) -> np.ndarray:
    """[groups][chunks][GROUP_ROWS][64] -> the un-duplicated rows [m_total][chunks*64]."""
    g, ch, _, k = packed.shape
    body = packed[:, :, :group_out_rows, :].transpose(0, 2, 1, 3).reshape(g * group_out_rows, ch * k)
    return np.ascontiguousarray(body[:m_total])


# -- inverse of the reference's BFP16 weight encoding, for exactly representable
#    weights (every 8-block shares one exponent; checked by re-encoding) --------

def bfp16_decode(data: np.ndarray) -> np.ndarray:
    blk = data.reshape(-1, 9)
    exp = blk[:, :1].astype(np.int64)
    q = blk[:, 1:].astype(np.int8).astype(np.float64)
    return (q * np.ldexp(1.0, exp - 127 - 6)).astype(np.float32).reshape(-1)


def atb_unshuffle(flat: np.ndarray, K: int, Nn: int, k: int = 64, n: int = 128) -> np.ndarray:
    t = flat.reshape(Nn // n, K // k, n // 16, k // 8, 2, 8, 8)
    # forward was (Nn/n, K/k, k/8, 8, n/16, 2, 8) -> transpose(0,1,4,2,5,6,3)
    t = t.transpose(0, 1, 3, 6, 2, 4, 5).reshape(Nn // n, K // k, k, n)
    return t.transpose(1, 2, 0, 3).reshape(K, Nn)


def exact_weights(rng, Cout, Cin):
    """Values +-m/64, m in [64,127]: one shared exponent per 8-block -> exact BFP16."""
    m = rng.integers(64, 128, size=(Cout, Cin, 3, 3))
    s = rng.choice([-1.0, 1.0], size=(Cout, Cin, 3, 3))
    return (s * m / 64.0).astype(np.float32)


def make_conv3x3w_host(host, out: Path) -> None:
    rng = np.random.default_rng(1234)
    ref = oracle.reference()
    data = {}
    # ---- pack_input ----
    cases = [(2, 70, 5, 7, 2), (1, 3, 4, 4, 1), (3, 64, 6, 9, 1), (2, 130, 3, 11, 3)]
    for i, (B, Cc, H, W, chunks) in enumerate(cases):
        x = rng.standard_normal((B, Cc, H, W)).astype(np.float32)
        bits = host.bf16_bits(x)
        packed = host.pack_input(host.bf16_value(bits).reshape(x.shape), chunks)
        _, m_total, _ = host.geometry(B, H, W)
        rows = rows_from_groups(packed, m_total, host.GROUP_OUT_ROWS)
        # same bytes from the reference's C++ packer (conv_pack.cpp:352-392)
        if ref is not None:
            cpp = np.zeros(packed.shape, np.uint16)
            ref.xdna_conv3x3w_pack_input_bf16(np.ascontiguousarray(bits), cpp.reshape(-1), B, Cc, H, W, chunks)
            assert np.array_equal(cpp, packed), "conv_pack.cpp disagrees with conv3x3w_host.py"
        data[f"pack{i}_x"] = bits
        data[f"pack{i}_rows"] = rows
        data[f"pack{i}_meta"] = np.array([B, Cc, H, W, chunks])
    # ---- pack_weights (forward) and the dX variant, decoded to K x N ----
    wcases = [(128, 70, 2), (100, 64, 1), (128, 130, 3)]
    for i, (Cout, Cin, chunks) in enumerate(wcases):
        w = exact_weights(rng, Cout, Cin)
        wb = host.bf16_bits(w)
        enc = host.pack_weights(w, chunks, 0)
        K = chunks * 576
        wk = atb_unshuffle(bfp16_decode(enc), K, 128)
        # round trip: re-encoding the decoded matrix with the reference's own
        # helpers gives the reference's bytes back
        assert np.array_equal(host.bfp16_encode(host.atb_shuffle(wk)), enc)
        data[f"wfwd{i}_w"] = wb.reshape(Cout, Cin, 3, 3)
        data[f"wfwd{i}_wk"] = host.bf16_bits(wk)  # [K][N=128], exact in bf16
        data[f"wfwd{i}_meta"] = np.array([Cout, Cin, chunks])
        if ref is not None:
            # dX weights from the reference's C++ (conv_pack.cpp:474-519): the conv
            # with Cin' = Cout, Cout' = Cin; K-chunks over Cout.
            Cout_d, Cin_d = Cin, Cout  # dgrad output/input channels
            chunks_d = -(-Cout // 64)
            if Cout_d <= 128:
                nbytes = chunks_d * 9 * (128 // 16) * 8 * 2 * 8 * 9
                buf = np.zeros(nbytes, np.uint8)
                ref.xdna_conv3x3w_pack_weights_dx_bfp16.argtypes = [
                    np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"),
                    np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS"), C.c_int, C.c_int, C.c_int, C.c_int]
                ref.xdna_conv3x3w_pack_weights_dx_bfp16(np.ascontiguousarray(wb), buf, Cout, Cin, chunks_d, 0)
                wkd = atb_unshuffle(bfp16_decode(buf), chunks_d * 576, 128)
                assert np.array_equal(host.bfp16_encode(host.atb_shuffle(wkd)), buf)
                data[f"wdx{i}_wk"] = host.bf16_bits(wkd)
                data[f"wdx{i}_meta"] = np.array([Cout, Cin, chunks_d])
    # ---- unpack_output: padded-grid output rows -> NCHW ----
    for i, (B, H, W, cout) in enumerate([(2, 5, 7, 100), (1, 9, 3, 128)]):
        _, m_total, groups = host.geometry(B, H, W)
        # unpack_output reads only the first m_total rows
        c = rng.standard_normal((m_total, 128)).astype(np.float32)
        cb = host.bf16_bits(c)
        data[f"unpack{i}_c"] = cb
        data[f"unpack{i}_y"] = host.unpack_output(cb, B, H, W, cout)
        data[f"unpack{i}_meta"] = np.array([B, H, W, cout])
    np.savez_compressed(out, **data)


def make_regions(out: Path) -> None:
    ref = oracle.reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libxdna_ref.so missing: run `make -C oracle` first")
    rng = np.random.default_rng(99)
    data = {}

    def special(shape):
        x = rng.standard_normal(shape).astype(np.float32)
        flat = x.reshape(-1)
        n = flat.size
        idx = rng.choice(n, size=max(4, n // 50), replace=False)
        vals = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, 1.0, -1.0], np.float32)
        flat[idx] = vals[np.arange(idx.size) % vals.size]
        return oracle.bf16_bits(x)

    for tag, shape in (("even", (3, 4, 6, 8)), ("odd", (2, 3, 7, 5))):
        planes = shape[0] * shape[1]
        H, W = shape[2], shape[3]
        a = special(shape)
        b = special(shape)
        base = special(shape)
        n = a.size
        r = np.empty_like(a)
        ref.xdna_region_relu_bf16(a.reshape(-1), r.reshape(-1), n, 2)
        rp = np.empty_like(a)
        p = np.zeros(shape[:2] + (H // 2, W // 2), np.uint16)
        ref.xdna_region_relu_maxpool2_bf16(a.reshape(-1), rp.reshape(-1), p.reshape(-1), planes, H, W, 2)
        at = np.empty_like(a)
        ref.xdna_region_addtap_bf16(base.ctypes.data_as(C.c_void_p), a.reshape(-1), b.reshape(-1), at.reshape(-1),
                                    n, C.c_float(0.37), 2)
        at0 = np.empty_like(a)
        ref.xdna_region_addtap_bf16(None, a.reshape(-1), b.reshape(-1), at0.reshape(-1), n, C.c_float(-1.5), 2)
        rb = np.empty_like(a)
        ref.xdna_region_relu_bwd_bf16(r.reshape(-1), base.ctypes.data_as(C.c_void_p), a.ctypes.data_as(C.c_void_p),
                                      b.ctypes.data_as(C.c_void_p), rb.reshape(-1), n, C.c_float(0.25), 2)
        rb0 = np.empty_like(a)
        ref.xdna_region_relu_bwd_bf16(r.reshape(-1), base.ctypes.data_as(C.c_void_p), None, None, rb0.reshape(-1), n,
                                      C.c_float(0.25), 2)
        g = special(shape[:2] + (H // 2, W // 2))
        mb = np.empty_like(a)
        ref.xdna_region_maxpool2_bwd_bf16(a.reshape(-1), g.reshape(-1), mb.reshape(-1), planes, H, W, 2)
        fin_a = oracle.bf16_bits(rng.standard_normal(shape).astype(np.float32))
        fin_b = oracle.bf16_bits(rng.standard_normal(shape).astype(np.float32))
        sq = ref.xdna_region_sqdiff_sum_bf16(fin_a.reshape(-1), fin_b.reshape(-1), n, 2)
        data.update({f"{tag}_a": a, f"{tag}_b": b, f"{tag}_base": base, f"{tag}_relu": r, f"{tag}_relu_r": rp,
                     f"{tag}_pool": p, f"{tag}_addtap": at, f"{tag}_addtap_nobase": at0, f"{tag}_relu_bwd": rb,
                     f"{tag}_relu_bwd_notap": rb0, f"{tag}_g": g, f"{tag}_maxpool_bwd": mb, f"{tag}_fin_a": fin_a,
                     f"{tag}_fin_b": fin_b, f"{tag}_sqdiff": np.array([sq])})
    np.savez_compressed(out, **data)


def make_regions_bn(out: Path) -> None:
    """Fused BatchNorm + activation vectors from the reference's own host kernels
    (xdna_region_bn_fwd_bf16 / _bwd_bf16, region_kernels.cpp:309-460)."""
    ref = oracle.reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libxdna_ref.so missing: run `make -C oracle` first")
    rng = np.random.default_rng(7)
    data = {}
    # (N, C, H, W, slope, relu, affine): shapes after the reference test (tests/run_regions_bn.py:43-44)
    cases = [(2, 16, 18, 18, 0.2, 0, 1), (2, 3, 5, 7, 0.2, 0, 1), (3, 1, 4, 4, 0.2, 0, 1),
             (4, 8, 11, 13, 0.0, 1, 1), (4, 16, 8, 8, 0.0, 1, 0)]
    for i, (N, Cc, H, W, slope, relu, affine) in enumerate(cases):
        x = oracle.bf16_bits((rng.standard_normal((N, Cc, H, W)) * 1.5 + 0.3).astype(np.float32))
        w = oracle.bf16_bits(rng.uniform(0.5, 1.5, Cc).astype(np.float32)) if affine else None
        b = oracle.bf16_bits((rng.standard_normal(Cc) * 0.3).astype(np.float32)) if affine else None
        rm = oracle.bf16_bits((rng.standard_normal(Cc) * 0.1).astype(np.float32))
        rv = oracle.bf16_bits(rng.uniform(0.5, 1.5, Cc).astype(np.float32))
        y, mean, invstd, rm2, rv2 = oracle.bn_fwd(x, w, b, rm, rv, 1e-5, slope, 0.1, True, reference_impl=True)
        dy = oracle.bf16_bits(rng.standard_normal((N, Cc, H, W)).astype(np.float32))
        # backward on an activation with planted zeros and NaNs: pins the dz rule
        yb = y.copy().reshape(-1)
        idx = rng.choice(yb.size, size=max(2, yb.size // 40), replace=False)
        yb[idx[: idx.size // 2]] = 0x0000
        yb[idx[idx.size // 2:]] = 0x7FC0
        yb = yb.reshape(y.shape)
        dx, dw, db = oracle.bn_bwd(dy, yb, x, w, mean, invstd, slope, relu, reference_impl=True)
        data.update({f"c{i}_meta": np.array([N, Cc, H, W, relu, affine]), f"c{i}_slope": np.array([slope], np.float32),
                     f"c{i}_x": x, f"c{i}_rm": rm, f"c{i}_rv": rv, f"c{i}_y": y, f"c{i}_mean": mean,
                     f"c{i}_invstd": invstd, f"c{i}_rm_out": rm2, f"c{i}_rv_out": rv2, f"c{i}_dy": dy,
                     f"c{i}_ybwd": yb, f"c{i}_dx": dx, f"c{i}_dw": dw, f"c{i}_db": db})
        if affine:
            data.update({f"c{i}_w": w, f"c{i}_b": b})
    data["cases"] = np.array([len(cases)])
    np.savez_compressed(out, **data)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    ref = Path(args.ref)
    oracle.build()
    host = load_host_spec(ref)
    make_conv3x3w_host(host, HERE / "conv3x3w_host.npz")
    make_regions(HERE / "regions.npz")
    make_regions_bn(HERE / "regions_bn.npz")
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
