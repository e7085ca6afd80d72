// aten::convolution_overrideable / convolution_backward_overrideable on xdna.
//
// Replaces convolution_overrideable_xdna / convolution_backward_overrideable_xdna
// (torch_xdna_device.cpp:4524-4606, 4608-4885) and the conv3x3w runtimes they
// drive (:1990-2523, 2530-2771).  BF16 3x3 / stride 1 / pad 1 / dilation 1 /
// groups 1 convolutions run the sm_100a implicit-GEMM kernels:
//   forward   pack x -> padded-grid rows, pack w -> Wk, conv kernel (+bias)
//   dX        pack dy -> rows, pack w -> Wk' (flip + transpose), same kernel
//   dW        wgrad kernel over the dy rows and the x rows the forward kept,
//             deferred until the gradient is first read (see deferred.cpp)
//   dbias     sum of dy over (N, H, W)
// Channels-last x and dy (C % 8 == 0) skip the padded-row copies: the kernels
// read them in place through im2col TMA maps over the padded grid (the
// *_nhwc entry points), and dbias is a channel sum of dy.
// BF16 1x1 / stride 1 / no padding convolutions (contiguous NCHW or
// channels-last, channel counts -- and H*W for NCHW -- multiples of 8) run as
// tcgen05 GEMMs (b2_conv1x1_*): forward and dX one GEMM each, dW a split-K GEMM
// over all pixels computed with the backward.  Stems and large kernels (few
// input channels, or >= 5x5; any stride / padding / dilation) run as GEMMs
// over an explicit column matrix (b2_im2col_*, b2_gemm_splitk_bf16).
// Outputs follow the input's memory format (NCHW or channels-last), written
// directly by the kernel epilogue.  Other convolutions (and set_npu_mode(0))
// take ATen's CUDA convolution on aliases -- the reference sends them to its
// CPU path the same way (:4578-4605).
#include <ATen/ops/convolution.h>
#include <ATen/ops/convolution_backward.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {
namespace {

bool is3x3s1p1(const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride, at::IntArrayRef padding,
               at::IntArrayRef dilation, bool transposed, int64_t groups) {
  if (input.dim() != 4 || weight.dim() != 4 || transposed || groups != 1) return false;
  if (weight.size(2) != 3 || weight.size(3) != 3) return false;
  auto all = [](at::IntArrayRef v, int64_t x) {
    for (auto e : v)
      if (e != x) return false;
    return v.size() == 2;
  };
  return all(stride, 1) && all(padding, 1) && all(dilation, 1) && input.size(1) == weight.size(1);
}

bool bf16(const at::Tensor& t) { return !t.defined() || t.scalar_type() == at::kBFloat16; }

// 1x1 / stride 1 / no padding: the GEMM layout of the input (0 = NCHW,
// 1 = channels-last), or -1 when the GEMM kernels cannot take it.
int conv1x1_layout(const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride,
                   at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed, int64_t groups) {
  if (input.dim() != 4 || weight.dim() != 4 || transposed || groups != 1) return -1;
  if (weight.size(2) != 1 || weight.size(3) != 1 || input.size(1) != weight.size(1)) return -1;
  auto all = [](at::IntArrayRef v, int64_t x) {
    for (auto e : v)
      if (e != x) return false;
    return v.size() == 2;
  };
  if (!all(stride, 1) || !all(padding, 0) || !all(dilation, 1)) return -1;
  const int64_t Cin = input.size(1), Cout = weight.size(0), HW = input.size(2) * input.size(3);
  if (Cin % 8 || Cout % 8 || input.numel() == 0) return -1;
  auto aligned = [](const at::Tensor& t) { return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0; };
  if (!aligned(input)) return -1;
  if (input.suggest_memory_format() == at::MemoryFormat::ChannelsLast &&
      input.is_contiguous(at::MemoryFormat::ChannelsLast))
    return 1;
  if (input.is_contiguous() && HW % 8 == 0) return 0;
  return -1;
}

// ---- general convolutions as GEMMs over a column matrix (b2_im2col_*) -------
// Taken for the convolutions ATen's library kernels handle worst and an
// explicit column matrix handles well: few input channels (stems: 7x7 3->64,
// 9x9 3->32) or large kernels (>= 5x5).  Groups 1, bf16, Cout % 8 == 0, and a
// column matrix of at most 4 GiB.
struct GeneralConv {
  int64_t B, Cin, H, W, Cout, Ho, Wo, P, K, Kp;
  int kh, kw, sy, sx, py, px, dy, dx;
};

bool general_conv(const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride, at::IntArrayRef padding,
                  at::IntArrayRef dilation, bool transposed, int64_t groups, GeneralConv& g) {
  if (input.dim() != 4 || weight.dim() != 4 || transposed || groups != 1 || input.numel() == 0) return false;
  if (stride.size() != 2 || padding.size() != 2 || dilation.size() != 2 || input.size(1) != weight.size(1))
    return false;
  g.B = input.size(0);
  g.Cin = input.size(1);
  g.H = input.size(2);
  g.W = input.size(3);
  g.Cout = weight.size(0);
  g.kh = int(weight.size(2));
  g.kw = int(weight.size(3));
  g.sy = int(stride[0]);
  g.sx = int(stride[1]);
  g.py = int(padding[0]);
  g.px = int(padding[1]);
  g.dy = int(dilation[0]);
  g.dx = int(dilation[1]);
  if (g.Cout % 8 || g.sy < 1 || g.sx < 1 || g.dy < 1 || g.dx < 1) return false;
  if (!(g.Cin <= 16 || int64_t(g.kh) * g.kw >= 25)) return false;
  g.Ho = (g.H + 2 * g.py - int64_t(g.dy) * (g.kh - 1) - 1) / g.sy + 1;
  g.Wo = (g.W + 2 * g.px - int64_t(g.dx) * (g.kw - 1) - 1) / g.sx + 1;
  if (g.Ho <= 0 || g.Wo <= 0) return false;
  g.P = g.B * g.Ho * g.Wo;
  g.K = int64_t(g.kh) * g.kw * g.Cin;
  g.Kp = (g.K + 7) / 8 * 8;
  return g.P * g.Kp * 2 <= (int64_t(4) << 30) && g.P < INT32_MAX;
}

// Slot kind of a column matrix kept on its input's storage: a tag of the
// window geometry (kinds 0-4 are packed weights), so two convolutions of one
// input never share one.
int col_kind(const GeneralConv& g) {
  uint32_t h = 2166136261u;
  for (int v : {g.kh, g.kw, g.sy, g.sx, g.py, g.px, g.dy, g.dx}) h = (h ^ uint32_t(v)) * 16777619u;
  return int(16 + (h & 0x3fffffffu));
}

at::Tensor im2col(const at::Tensor& x, const GeneralConv& g) {
  const auto dev = x.device().index();
  at::Tensor col = empty({g.P, g.Kp}, at::kBFloat16, dev);
  materialize(x);
  XDNA_B2(b2_im2col_bf16(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), x.stride(3), g.B, g.Cin, g.H, g.W, g.kh,
                         g.kw, g.sy, g.sx, g.py, g.px, g.dy, g.dx, g.Ho, g.Wo, g.Kp, col.data_ptr(), stream(dev)));
  count_launch("im2col");
  return col;
}

// Frozen weights (no gradient wanted: a perceptual loss's feature network)
// keep their packed forms between calls; the cache drops them on any write
// into the weight's storage.  Kinds: 0 / 1 3x3 forward / input gradient,
// 2 column-matrix order, 3 / 4 direct forward / input gradient.
template <typename F>
at::Tensor cached_pack(const at::Tensor& w, int kind, F make) {
  materialize(w);
  const bool frozen = !w.requires_grad();
  if (frozen) {
    at::Tensor hit = find_packed_weight(w, kind);
    if (hit.defined()) return hit;
  }
  at::Tensor packed = make();
  if (frozen) attach_packed_weight(w, kind, packed);
  return packed;
}

at::Tensor pack_weight_khwc(const at::Tensor& weight, const GeneralConv& g) {
  return cached_pack(weight, 2, [&] {
    at::Tensor w = weight.is_contiguous() ? weight : weight.contiguous();
    materialize(w);
    at::Tensor wk = empty({g.Cout, g.Kp}, at::kBFloat16, w.device().index());
    XDNA_B2(b2_pack_weight_khwc_bf16(w.data_ptr(), g.Cout, g.Cin, g.kh, g.kw, g.Kp, wk.data_ptr(),
                                     stream(w.device().index())));
    count_launch("pack_weight_khwc");
    return wk;
  });
}

// op(A) . op(B) with split-K into a new fp32 [M][N] tensor.
at::Tensor gemm_splitk_f32(int transA, int transB, int64_t M, int64_t N, int64_t K, const at::Tensor& A, int64_t lda,
                           const at::Tensor& B, int64_t ldb, c10::DeviceIndex dev) {
  at::Tensor d = empty({M, N}, at::kFloat, dev);
  const size_t wsb = b2_gemm_splitk_workspace_bytes(int(M), int(N), int(K), B2_F32);
  at::Tensor ws = empty({int64_t((wsb + 15) / 16) * 4 + 4}, at::kFloat, dev);
  XDNA_B2(b2_gemm_splitk_bf16(transA, transB, int(M), int(N), int(K), A.data_ptr(), lda, B.data_ptr(), ldb,
                              d.data_ptr(), B2_F32, N, ws.data_ptr(), size_t(ws.numel()) * 4, stream(dev)));
  count_launch("gemm_splitk", 2);
  return d;
}

at::Tensor general_forward(const at::Tensor& input, const at::Tensor& weight, const at::Tensor& bias,
                           const GeneralConv& g) {
  const auto dev = input.device().index();
  c10::cuda::CUDAGuard guard(dev);
  at::Tensor col = im2col(input, g);
  // the weight gradient multiplies the same column matrix: kept on the
  // input's storage under its geometry (dropped when the input is written or
  // freed)
  if (at::GradMode::is_enabled() && weight.requires_grad() && g_mode.load() > 1)
    attach_packed_weight(input, col_kind(g), col);
  at::Tensor wk = pack_weight_khwc(weight, g);
  at::Tensor b = bias.defined() ? (bias.is_contiguous() ? bias : bias.contiguous()) : at::Tensor();
  if (b.defined()) materialize(b);
  const bool cl = input.suggest_memory_format() == at::MemoryFormat::ChannelsLast;
  // Y as [P][Cout] (channels-last); NCHW callers get a transposed copy
  at::Tensor y = empty({g.B, g.Cout, g.Ho, g.Wo}, at::kBFloat16, dev, at::MemoryFormat::ChannelsLast);
  XDNA_B2(b2_gemm_bf16(0, 1, int(g.P), int(g.Cout), int(g.Kp), 1.f, col.data_ptr(), g.Kp, 0, wk.data_ptr(), g.Kp, 0,
                       b.defined() ? 1.f : 0.f, b.defined() ? b.data_ptr() : nullptr, B2_BF16, 0, 1, 0, y.data_ptr(),
                       g.Cout, 0, 1, stream(dev)));
  count_launch("conv.gemm");
  if (cl) return y;
  at::Tensor yn = empty({g.B, g.Cout, g.Ho, g.Wo}, at::kBFloat16, dev);
  XDNA_B2(b2_nhwc_to_nchw_bf16(y.data_ptr(), yn.data_ptr(), int(g.B), int(g.Cout), int(g.Ho * g.Wo), stream(dev)));
  count_launch("nhwc_to_nchw");
  return yn;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> general_backward(const at::Tensor& grad_output, const at::Tensor& input,
                                                                const at::Tensor& weight, const GeneralConv& g,
                                                                std::array<bool, 3> mask) {
  const auto dev = input.device().index();
  c10::cuda::CUDAGuard guard(dev);
  // dY as [P][Cout]
  at::Tensor dy;
  if (grad_output.suggest_memory_format() == at::MemoryFormat::ChannelsLast &&
      grad_output.is_contiguous(at::MemoryFormat::ChannelsLast)) {
    dy = grad_output;
    materialize(dy);
  } else {
    at::Tensor gc = grad_output.is_contiguous() ? grad_output : grad_output.contiguous();
    materialize(gc);
    dy = empty({g.B, g.Cout, g.Ho, g.Wo}, at::kBFloat16, dev, at::MemoryFormat::ChannelsLast);
    XDNA_B2(b2_nchw_to_nhwc_bf16(gc.data_ptr(), dy.data_ptr(), int(g.B), int(g.Cout), int(g.Ho * g.Wo), stream(dev)));
    count_launch("nchw_to_nhwc");
  }
  at::Tensor dx, dw, db;
  if (mask[0]) {
    at::Tensor wk = pack_weight_khwc(weight, g);
    // dcol[P][Kp] = dY[P][Cout] . Wk[Cout][Kp]
    at::Tensor dcol = gemm_splitk_f32(0, 0, g.P, g.Kp, g.Cout, dy, g.Cout, wk, g.Kp, dev);
    const auto mf = input.suggest_memory_format() == at::MemoryFormat::ChannelsLast ? at::MemoryFormat::ChannelsLast
                                                                                     : at::MemoryFormat::Contiguous;
    dx = empty({g.B, g.Cin, g.H, g.W}, at::kBFloat16, dev, mf);
    XDNA_B2(b2_col2im_bf16(dcol.data_ptr<float>(), g.Kp, g.B, g.Cin, g.H, g.W, g.kh, g.kw, g.sy, g.sx, g.py, g.px,
                           g.dy, g.dx, g.Ho, g.Wo, dx.data_ptr(), dx.stride(0), dx.stride(1), dx.stride(2),
                           dx.stride(3), stream(dev)));
    count_launch("col2im");
  }
  if (mask[1]) {
    at::Tensor col = find_packed_weight(input, col_kind(g));
    if (!col.defined() || col.dim() != 2 || col.size(0) != g.P || col.size(1) != g.Kp) col = im2col(input, g);
    // dWk[Cout][Kp] = dY^T . col over the P pixels
    at::Tensor dwk = gemm_splitk_f32(1, 0, g.Cout, g.Kp, g.P, dy, g.Cout, col, g.Kp, dev);
    dw = empty({g.Cout, g.Cin, g.kh, g.kw}, weight.scalar_type(), dev);
    XDNA_B2(b2_unpack_weight_khwc(dwk.data_ptr<float>(), g.Cout, g.Cin, g.kh, g.kw, g.Kp, dw.data_ptr(),
                                  weight.scalar_type() == at::kFloat ? B2_F32 : B2_BF16, stream(dev)));
    count_launch("unpack_weight_khwc");
  }
  if (mask[2]) {
    count_fallback("conv.dbias");
    db = adopt(to_cuda(dy).sum(at::IntArrayRef{0, 2, 3}).to(grad_output.scalar_type()));
  }
  return {dx, dw, db};
}

at::MemoryFormat out_format(const at::Tensor& input) {
  return input.suggest_memory_format() == at::MemoryFormat::ChannelsLast ? at::MemoryFormat::ChannelsLast
                                                                          : at::MemoryFormat::Contiguous;
}

// ---- direct convolutions for RGB input / output layers (b2_direct.cu)
// An RGB output layer (9x9 32->3 in the style network) wastes nearly all of a
// tensor-core tile, and ATen's library answers its input gradient with a
// direct kernel of ~0.5 ms at B40 36x36 (45 us here); an RGB input layer's
// forward (9x9 3->32) is a short reduction.  Both run on the CUDA cores (fp32,
// one rounding); the weight gradients stay on ATen's library kernels, and 3x3
// stride-1 layers on the tensor-core path.
struct DirectConv {
  int64_t B, Cin, H, W, Cout, Ho, Wo;
  int kh, kw, sy, sx, py, px, dy, dx;
};

bool direct_conv(const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride, at::IntArrayRef padding,
                 at::IntArrayRef dilation, bool transposed, int64_t groups, DirectConv& d) {
  if (input.dim() != 4 || weight.dim() != 4 || transposed || groups != 1 || input.numel() == 0) return false;
  if (stride.size() != 2 || padding.size() != 2 || dilation.size() != 2 || input.size(1) != weight.size(1))
    return false;
  d.B = input.size(0);
  d.Cin = input.size(1);
  d.H = input.size(2);
  d.W = input.size(3);
  d.Cout = weight.size(0);
  d.kh = int(weight.size(2));
  d.kw = int(weight.size(3));
  d.sy = int(stride[0]);
  d.sx = int(stride[1]);
  d.py = int(padding[0]);
  d.px = int(padding[1]);
  d.dy = int(dilation[0]);
  d.dx = int(dilation[1]);
  // a handful of channels on one side (an RGB input or output layer), at most
  // 64 on the other (a thread holds one fp32 accumulator per output channel)
  if (std::min(d.Cin, d.Cout) > 4 || d.Cout > 64 || d.Cin > 64 || d.kh > 11 || d.kw > 11) return false;
  if (d.sy < 1 || d.sx < 1 || d.dy < 1 || d.dx < 1 || d.py < 0 || d.px < 0) return false;
  d.Ho = (d.H + 2 * d.py - int64_t(d.dy) * (d.kh - 1) - 1) / d.sy + 1;
  d.Wo = (d.W + 2 * d.px - int64_t(d.dx) * (d.kw - 1) - 1) / d.sx + 1;
  return d.Ho > 0 && d.Wo > 0;
}

at::Tensor direct_weight(const at::Tensor& weight, const DirectConv& d, int dgrad) {
  return cached_pack(weight, dgrad ? 4 : 3, [&] {
    at::Tensor w = weight.is_contiguous() ? weight : weight.contiguous();
    materialize(w);
    const size_t n = b2_direct_conv_weight_floats(d.Cout, d.Cin, d.kh, d.kw, dgrad);
    at::Tensor wt = empty({int64_t(n)}, at::kFloat, w.device().index());
    XDNA_B2(b2_direct_conv_weight(w.data_ptr(), d.Cout, d.Cin, d.kh, d.kw, dgrad, wt.data_ptr<float>(),
                                  stream(w.device().index())));
    count_launch("direct_conv.weight");
    return wt;
  });
}

at::Tensor direct_forward(const at::Tensor& input, const at::Tensor& weight, const at::Tensor& bias,
                          const DirectConv& d) {
  const auto dev = input.device().index();
  c10::cuda::CUDAGuard guard(dev);
  materialize(input);
  at::Tensor wt = direct_weight(weight, d, 0);
  at::Tensor b = bias.defined() ? (bias.is_contiguous() ? bias : bias.contiguous()) : at::Tensor();
  if (b.defined()) materialize(b);
  at::Tensor y = empty({d.B, d.Cout, d.Ho, d.Wo}, at::kBFloat16, dev, out_format(input));
  const int64_t is[4] = {input.stride(0), input.stride(1), input.stride(2), input.stride(3)};
  const int64_t os[4] = {y.stride(0), y.stride(1), y.stride(2), y.stride(3)};
  XDNA_B2(b2_direct_conv_bf16(input.data_ptr(), is, d.B, d.Cin, d.H, d.W, wt.data_ptr<float>(), d.kh, d.kw, d.sy,
                              d.sx, d.py, d.px, d.dy, d.dx, b.defined() ? b.data_ptr() : nullptr, y.data_ptr(), os,
                              d.Cout, d.Ho, d.Wo, stream(dev)));
  count_launch("direct_conv.fwd");
  return y;
}

// stride-1 input gradient as a direct convolution over dY
// A thread per output pixel keeps one fp32 accumulator per output channel and
// walks the whole reduction: efficient when many outputs share each load (>= 8
// of them) and the walk is short; with 1-4 outputs and hundreds of taps it is
// latency-bound.  So: the input gradient of an RGB output layer (Cout <= 4,
// 8 <= Cin <= 64, stride 1) and the forward of an RGB input layer (Cin <= 4,
// 16 <= Cout <= 64, Cin*kh*kw <= 512, <= 2^31 FMAs: a 224x224 batch-128 stem
// belongs on tensor cores).
bool direct_dgrad_ok(const DirectConv& d) {
  return d.Cout <= 4 && d.Cin >= 8 && d.sy == 1 && d.sx == 1 && (d.kh - 1) * d.dy >= d.py &&
         (d.kw - 1) * d.dx >= d.px && d.Cout * d.kh * d.kw <= 2592;
}

bool direct_fwd_ok(const DirectConv& d) {
  return d.Cin <= 4 && d.Cout >= 16 && d.Cin * d.kh * d.kw <= 512 &&
         d.B * d.Ho * d.Wo * d.Cin * d.kh * d.kw * d.Cout <= (int64_t(1) << 31);
}

at::Tensor direct_dgrad(const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight,
                        const DirectConv& d) {
  const auto dev = input.device().index();
  c10::cuda::CUDAGuard guard(dev);
  materialize(grad_output);
  at::Tensor wt = direct_weight(weight, d, 1);
  at::Tensor dx = empty({d.B, d.Cin, d.H, d.W}, at::kBFloat16, dev, out_format(input));
  const int64_t is[4] = {grad_output.stride(0), grad_output.stride(1), grad_output.stride(2), grad_output.stride(3)};
  const int64_t os[4] = {dx.stride(0), dx.stride(1), dx.stride(2), dx.stride(3)};
  XDNA_B2(b2_direct_conv_bf16(grad_output.data_ptr(), is, d.B, d.Cout, d.Ho, d.Wo, wt.data_ptr<float>(), d.kh, d.kw,
                              1, 1, (d.kh - 1) * d.dy - d.py, (d.kw - 1) * d.dx - d.px, d.dy, d.dx, nullptr,
                              dx.data_ptr(), os, d.Cin, d.H, d.W, stream(dev)));
  count_launch("direct_conv.dgrad");
  return dx;
}

at::Tensor contiguous_as(const at::Tensor& t, int layout) {
  const auto mf = layout == 1 ? at::MemoryFormat::ChannelsLast : at::MemoryFormat::Contiguous;
  return t.is_contiguous(mf) ? t : t.contiguous(mf);
}

at::Tensor conv1x1_forward(const at::Tensor& input, const at::Tensor& weight, const at::Tensor& bias, int layout) {
  const c10::DeviceIndex dev = input.device().index();
  c10::cuda::CUDAGuard g(dev);
  const int64_t B = input.size(0), Cin = input.size(1), H = input.size(2), W = input.size(3), Cout = weight.size(0);
  at::Tensor w = weight.is_contiguous() ? weight : weight.contiguous();
  at::Tensor b = bias.defined() ? (bias.is_contiguous() ? bias : bias.contiguous()) : at::Tensor();
  materialize(input);
  materialize(w);
  if (b.defined()) materialize(b);
  const auto mf = layout == 1 ? at::MemoryFormat::ChannelsLast : at::MemoryFormat::Contiguous;
  at::Tensor y = empty({B, Cout, H, W}, at::kBFloat16, dev, mf);
  KernelTimer kt("conv1x1.fwd", 2.0 * B * H * W * Cin * Cout, stream(dev));
  XDNA_B2(b2_conv1x1_fwd(input.data_ptr(), w.data_ptr(), b.defined() ? b.data_ptr() : nullptr, y.data_ptr(), layout, B,
                         Cin, H * W, Cout, stream(dev)));
  count_launch("conv1x1.fwd");
  return y;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> conv1x1_backward(const at::Tensor& grad_output,
                                                                const at::Tensor& input, const at::Tensor& weight,
                                                                int layout, std::array<bool, 3> mask) {
  const c10::DeviceIndex dev = input.device().index();
  c10::cuda::CUDAGuard g(dev);
  const int64_t B = input.size(0), Cin = input.size(1), H = input.size(2), W = input.size(3), Cout = weight.size(0);
  at::Tensor dy = contiguous_as(grad_output, layout);
  materialize(dy);
  materialize(input);
  at::Tensor dx, dw, db;
  if (mask[0]) {
    at::Tensor w = weight.is_contiguous() ? weight : weight.contiguous();
    materialize(w);
    dx = empty({B, Cin, H, W}, at::kBFloat16, dev,
               layout == 1 ? at::MemoryFormat::ChannelsLast : at::MemoryFormat::Contiguous);
    KernelTimer kt("conv1x1.dgrad", 2.0 * B * H * W * Cin * Cout, stream(dev));
    XDNA_B2(b2_conv1x1_dgrad(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), layout, B, Cin, H * W, Cout, stream(dev)));
    count_launch("conv1x1.dgrad");
  }
  if (mask[1]) {
    dw = empty({Cout, Cin, 1, 1}, weight.scalar_type(), dev);
    const size_t ws_bytes = b2_conv1x1_wgrad_workspace_bytes(layout, B, Cin, H * W, Cout);
    at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4 + 4}, at::kFloat, dev);
    KernelTimer kt("conv1x1.wgrad", 2.0 * B * H * W * Cin * Cout, stream(dev));
    XDNA_B2(b2_conv1x1_wgrad(dy.data_ptr(), input.data_ptr(), dw.data_ptr(),
                             weight.scalar_type() == at::kFloat ? B2_F32 : B2_BF16, layout, B, Cin, H * W, Cout,
                             ws.data_ptr(), size_t(ws.numel()) * 4, stream(dev)));
    count_launch("conv1x1.wgrad", 2);  // split-K GEMM + ordered reduce
  }
  if (mask[2]) {
    count_fallback("conv1x1.dbias");
    db = adopt(to_cuda(dy).sum(at::IntArrayRef{0, 2, 3}).to(grad_output.scalar_type()));
  }
  return {dx, dw, db};
}

int chunks_of(int64_t c) { return int((c + 63) / 64); }

at::Tensor pack_rows(const at::Tensor& x) {
  const int B = int(x.size(0)), C = int(x.size(1)), H = int(x.size(2)), W = int(x.size(3));
  const int ch = chunks_of(C);
  at::Tensor rows = empty({int64_t(B) * (H + 2) * (W + 2), int64_t(ch) * 64}, at::kBFloat16, x.device().index());
  materialize(x);
  KernelTimer kt("pack_rows", 2.0 * B * C * H * W + 2.0 * B * (H + 2) * (W + 2) * ch * 64, stream(x.device().index()));
  XDNA_B2(b2_pack_rows_bf16(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), x.stride(3), B, C, H, W, ch,
                            rows.data_ptr(), stream(x.device().index())));
  count_launch("pack_rows");
  return rows;
}

at::Tensor pack_weight(const at::Tensor& w_in, bool dgrad) {
  return cached_pack(w_in, dgrad ? 1 : 0, [&] {
    // read in place through its strides (a channels-last model's OHWI
    // weights included); only a weight with negative strides is copied
    bool strided_ok = true;
    for (int d = 0; d < 4; ++d) strided_ok = strided_ok && w_in.stride(d) >= 0;
    at::Tensor w = strided_ok ? w_in : w_in.contiguous();
    materialize(w);
    const int Cout = int(w.size(0)), Cin = int(w.size(1));
    const int ch = chunks_of(dgrad ? Cout : Cin);
    at::Tensor wk = empty({dgrad ? Cin : Cout, int64_t(ch) * 576}, at::kBFloat16, w.device().index());
    const int64_t st[4] = {w.stride(0), w.stride(1), w.stride(2), w.stride(3)};
    XDNA_B2(b2_pack_weight_strided_bf16(w.data_ptr(), st, Cout, Cin, ch, dgrad ? 1 : 0, wk.data_ptr(),
                                        stream(w.device().index())));
    count_launch("pack_weight");
    return wk;
  });
}

// dW into `gw` (raw pointer: a deferred job must not keep the gradient's
// storage alive, or an unread gradient could never be freed and dropped).
void launch_wgrad(const at::Tensor& dy_rows, const at::Tensor& x_rows, void* gw, at::ScalarType dtype,
                  c10::DeviceIndex dev, int B, int Cin, int H, int W, int Cout) {
  c10::cuda::CUDAGuard g(dev);
  const size_t ws_bytes = b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout);
  at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
  const int dt = dtype == at::kFloat ? B2_F32 : B2_BF16;
  KernelTimer kt("conv3x3.wgrad", 18.0 * B * H * W * Cin * Cout, stream(dev));
  XDNA_B2(b2_conv3x3_wgrad(dy_rows.data_ptr(), x_rows.data_ptr(), gw, dt, B, Cin, H, W, Cout, ws.data_ptr(),
                           size_t(ws.numel()) * 4, stream(dev)));
  count_launch("conv3x3.wgrad", 2);  // igemm + split-K reduce
}

bool env_flag(const char* name, bool dflt) {
  const char* s = std::getenv(name);
  return s ? std::string(s) != "0" : dflt;
}

// Channels-last activations that the 3x3 kernels read in place through an
// im2col TMA map (no padded-row copy): channel stride 1, C and the pixel
// strides multiples of 8 elements, 16-byte aligned data.  XDNA_CONV_NHWC=0
// packs them as NCHW inputs are packed (A/B switch).
bool nhwc_enabled() {
  static const bool on = env_flag("XDNA_CONV_NHWC", true);
  return on;
}

// Every 3x3 layer reads channels-last activations in place (measured on
// B200, all three directions together beat packing at every ResNet-50 and
// sweep shape tried: B128 C64 56x56 to C512 7x7, B40 C128 36x36, B128 C256
// 72x72); XDNA_CONV_NHWC=0 restores the padded-row copies.
bool nhwc_layer(int64_t, int64_t) { return true; }

bool nhwc_ok(const at::Tensor& t) {
  if (!nhwc_enabled() || t.dim() != 4 || t.numel() == 0) return false;
  if (!t.is_contiguous(at::MemoryFormat::ChannelsLast)) return false;
  // channels-last contiguous: dense pixels of C channels (the library
  // replaces the strides of size-1 dimensions by the dense ones)
  if (t.size(1) % 8) return false;
  return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0;
}

// dW from channels-last dY and x read in place (see launch_wgrad); ohwi:
// written in a channels-last weight's [Cout][3][3][Cin] order.
void launch_wgrad_nhwc(const at::Tensor& dy, const at::Tensor& x, void* gw, at::ScalarType dtype,
                       c10::DeviceIndex dev, int B, int Cin, int H, int W, int Cout, bool ohwi) {
  c10::cuda::CUDAGuard g(dev);
  materialize(dy);
  materialize(x);
  const size_t ws_bytes = b2_conv3x3_wgrad_workspace_bytes(B, Cin, H, W, Cout);
  at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
  const int dt = dtype == at::kFloat ? B2_F32 : B2_BF16;
  KernelTimer kt("conv3x3.wgrad", 18.0 * B * H * W * Cin * Cout, stream(dev));
  auto* fn = ohwi ? b2_conv3x3_wgrad_nhwc_ohwi : b2_conv3x3_wgrad_nhwc;
  XDNA_B2(fn(dy.data_ptr(), dy.stride(0), dy.stride(2), dy.stride(3), x.data_ptr(), x.stride(0), x.stride(2),
             x.stride(3), gw, dt, B, Cin, H, W, Cout, ws.data_ptr(), size_t(ws.numel()) * 4, stream(dev)));
  count_launch("conv3x3.wgrad", 2);  // igemm + split-K reduce
}

}  // namespace

// Routing of the convolutions outside the 3x3 fast path (set_conv_paths).
// Stems and large kernels take the column-matrix GEMMs by default: on
// ResNet-50 (channels-last, batch 128, one B200) the 7x7 stem costs 0.95 ms a
// step that way against 1.17 ms in ATen's library kernels (the step: 8825
// against 8693 images/s).  The 1x1 GEMMs stay off by default: ATen's library
// kernels are still faster for ResNet-50's 1x1 layers (8621 against 8999
// images/s with them on).
std::atomic<bool> g_conv1x1{env_flag("XDNA_CONV1X1", false)};
std::atomic<bool> g_conv_general{env_flag("XDNA_CONV_GENERAL", true)};

namespace {

bool conv1x1_enabled() { return g_conv1x1.load(); }
bool general_enabled() { return g_conv_general.load(); }

bool deferral_enabled() {
  static const bool on = [] {
    const char* s = std::getenv("XDNA_DEFER_DW");
    return !s || std::string(s) != "0";
  }();
  return on;
}

at::Tensor convolution_overrideable(const at::Tensor& input, const at::Tensor& weight,
                                    const std::optional<at::Tensor>& bias_opt, at::IntArrayRef stride,
                                    at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed,
                                    at::IntArrayRef output_padding, int64_t groups) {
  const at::Tensor bias = bias_opt.has_value() ? *bias_opt : at::Tensor();
  if (g_mode.load() > 0 && bf16(input) && bf16(weight) && bf16(bias)) {
    const int l1 =
        conv1x1_enabled() ? conv1x1_layout(input, weight, stride, padding, dilation, transposed, groups) : -1;
    if (l1 >= 0) return conv1x1_forward(input, weight, bias, l1);
    // an RGB input layer small enough for the direct kernel takes it; other
    // stems and large kernels the column GEMMs
    DirectConv dc;
    if (!is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups) &&
        direct_conv(input, weight, stride, padding, dilation, transposed, groups, dc) && direct_fwd_ok(dc))
      return direct_forward(input, weight, bias, dc);
    GeneralConv gc;
    if (general_enabled() && !is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups) &&
        general_conv(input, weight, stride, padding, dilation, transposed, groups, gc))
      return general_forward(input, weight, bias, gc);
  }
  const bool fast = g_mode.load() > 0 && is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups) &&
                    bf16(input) && bf16(weight) && bf16(bias) && input.numel() > 0;
  if (!fast) {
    count_fallback("convolution_overrideable");
    c10::cuda::CUDAGuard g(input.device().index());
    return adopt(at::convolution(to_cuda(input), to_cuda(weight), bias.defined() ? to_cuda(bias) : at::Tensor(),
                                 stride, padding, dilation, transposed, output_padding, groups));
  }
  c10::cuda::CUDAGuard g(input.device().index());
  const int B = int(input.size(0)), Cin = int(input.size(1)), H = int(input.size(2)), W = int(input.size(3));
  const int Cout = int(weight.size(0));
  const bool in_place = nhwc_layer(Cin, Cout) && nhwc_ok(input);
  at::Tensor rows;
  if (in_place)
    materialize(input);
  else
    rows = pack_rows(input);
  at::Tensor wk = pack_weight(weight, false);
  at::Tensor b = bias.defined() ? (bias.is_contiguous() ? bias : bias.contiguous()) : at::Tensor();
  if (b.defined()) materialize(b);
  at::Tensor y = empty({B, Cout, H, W}, at::kBFloat16, input.device().index(), out_format(input));
  KernelTimer kt("conv3x3.fwd", 18.0 * B * H * W * Cin * Cout, stream(input.device().index()));
  if (in_place)
    XDNA_B2(b2_conv3x3_fwd_nhwc(input.data_ptr(), input.stride(0), input.stride(2), input.stride(3), wk.data_ptr(),
                                b.defined() ? b.data_ptr() : nullptr, y.data_ptr(), y.stride(0), y.stride(1),
                                y.stride(2), y.stride(3), B, Cin, H, W, Cout, 0, stream(input.device().index())));
  else
    XDNA_B2(b2_conv3x3_fwd(rows.data_ptr(), wk.data_ptr(), b.defined() ? b.data_ptr() : nullptr, y.data_ptr(),
                           y.stride(0), y.stride(1), y.stride(2), y.stride(3), B, Cin, H, W, Cout, 0,
                           stream(input.device().index())));
  count_launch("conv3x3.fwd");
  // keep the packed input for the weight gradient when one will be needed
  if (!in_place && at::GradMode::is_enabled() && weight.requires_grad() && g_mode.load() > 1) attach_rows(input, rows);
  return y;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> convolution_backward_overrideable(
    const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride,
    at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed, at::IntArrayRef output_padding, int64_t groups,
    std::array<bool, 3> output_mask) {
  if (g_mode.load() > 0 && bf16(input) && bf16(weight) && bf16(grad_output)) {
    DirectConv dc;
    GeneralConv gc;
    const bool not3x3 = !is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups);
    const bool general =
        general_enabled() && not3x3 && general_conv(input, weight, stride, padding, dilation, transposed, groups, gc);
    // an RGB output layer's input gradient: the direct kernel; its weight
    // gradient from the column GEMMs (or ATen's library kernels without them)
    if (not3x3 && direct_conv(input, weight, stride, padding, dilation, transposed, groups, dc) &&
        direct_dgrad_ok(dc)) {
      at::Tensor dx = output_mask[0] ? direct_dgrad(grad_output, input, weight, dc) : at::Tensor();
      at::Tensor dw, db;
      if ((output_mask[1] || output_mask[2]) && general) {
        auto r = general_backward(grad_output, input, weight, gc, {false, output_mask[1], output_mask[2]});
        dw = std::get<1>(r);
        db = std::get<2>(r);
      } else if (output_mask[1] || output_mask[2]) {
        count_fallback("convolution_backward_overrideable.dw");
        c10::cuda::CUDAGuard g(input.device().index());
        auto r = at::convolution_backward(to_cuda(grad_output), to_cuda(input), to_cuda(weight), std::nullopt,
                                          stride, padding, dilation, transposed, output_padding, groups,
                                          {false, output_mask[1], output_mask[2]});
        if (output_mask[1]) dw = adopt(std::get<1>(r));
        if (output_mask[2]) db = adopt(std::get<2>(r));
      }
      return {dx, dw, db};
    }
    const int l1 =
        conv1x1_enabled() ? conv1x1_layout(input, weight, stride, padding, dilation, transposed, groups) : -1;
    if (l1 >= 0) return conv1x1_backward(grad_output, input, weight, l1, output_mask);
    if (general) return general_backward(grad_output, input, weight, gc, output_mask);
  }
  const bool fast = g_mode.load() > 0 && is3x3s1p1(input, weight, stride, padding, dilation, transposed, groups) &&
                    bf16(input) && bf16(weight) && bf16(grad_output) && input.numel() > 0;
  c10::cuda::CUDAGuard g(input.device().index());
  if (!fast) {
    count_fallback("convolution_backward_overrideable");
    auto r = at::convolution_backward(to_cuda(grad_output), to_cuda(input), to_cuda(weight), std::nullopt, stride,
                                      padding, dilation, transposed, output_padding, groups, output_mask);
    return {adopt(std::get<0>(r)), adopt(std::get<1>(r)), adopt(std::get<2>(r))};
  }
  const int B = int(input.size(0)), Cin = int(input.size(1)), H = int(input.size(2)), W = int(input.size(3));
  const int Cout = int(weight.size(0));
  const c10::DeviceIndex dev = input.device().index();
  at::Tensor dx, dw, db;
  // channels-last dY (and x, for dW) are read in place; otherwise packed rows
  const bool dy_cl = nhwc_layer(Cin, Cout) && nhwc_ok(grad_output);
  const bool both_cl = dy_cl && nhwc_ok(input);
  at::Tensor dy_rows;
  if (dy_cl) materialize(grad_output);
  if (output_mask[2] && dy_cl) {
    db = empty({Cout}, grad_output.scalar_type(), dev);
    const size_t ws_bytes = b2_channel_sum_nhwc_workspace_bytes(B, Cout, H, W);
    at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
    KernelTimer kt("channel_sum", 2.0 * B * H * W * Cout, stream(dev));
    XDNA_B2(b2_channel_sum_nhwc_bf16(grad_output.data_ptr(), grad_output.stride(0), grad_output.stride(2),
                                     grad_output.stride(3), B, Cout, H, W, db.data_ptr(), B2_BF16, ws.data_ptr(),
                                     size_t(ws.numel()) * 4, stream(dev)));
    count_launch("channel_sum", 2);
  } else if (output_mask[2]) {
    // the dY packer also reduces dbias (one pass over dY, deterministic order)
    const int ch = chunks_of(Cout);
    dy_rows = empty({int64_t(B) * (H + 2) * (W + 2), int64_t(ch) * 64}, at::kBFloat16, dev);
    db = empty({Cout}, grad_output.scalar_type(), dev);
    const size_t ws_bytes = b2_pack_rows_dbias_workspace_bytes(B, Cout, H, W);
    at::Tensor ws = empty({int64_t((ws_bytes + 15) / 16) * 4}, at::kFloat, dev);
    materialize(grad_output);
    XDNA_B2(b2_pack_rows_dbias_bf16(grad_output.data_ptr(), grad_output.stride(0), grad_output.stride(1),
                                    grad_output.stride(2), grad_output.stride(3), B, Cout, H, W, ch, dy_rows.data_ptr(),
                                    db.data_ptr(), B2_BF16, ws.data_ptr(), size_t(ws.numel()) * 4, stream(dev)));
    count_launch("pack_rows_dbias", 3);  // pack + two channel-sum stages
  } else if (!dy_cl) {
    dy_rows = pack_rows(grad_output);
  }
  if (output_mask[0]) {
    at::Tensor wkd = pack_weight(weight, true);
    dx = empty({B, Cin, H, W}, at::kBFloat16, dev, out_format(input));
    KernelTimer kt("conv3x3.dgrad", 18.0 * B * H * W * Cin * Cout, stream(dev));
    if (dy_cl)
      XDNA_B2(b2_conv3x3_dgrad_nhwc(grad_output.data_ptr(), grad_output.stride(0), grad_output.stride(2),
                                    grad_output.stride(3), wkd.data_ptr(), dx.data_ptr(), dx.stride(0), dx.stride(1),
                                    dx.stride(2), dx.stride(3), B, Cout, H, W, Cin, stream(dev)));
    else
      XDNA_B2(b2_conv3x3_dgrad(dy_rows.data_ptr(), wkd.data_ptr(), dx.data_ptr(), dx.stride(0), dx.stride(1),
                               dx.stride(2), dx.stride(3), B, Cout, H, W, Cin, stream(dev)));
    count_launch("conv3x3.dgrad");
  }
  if (output_mask[1]) {
    // a channels-last weight gets its gradient in its own layout (autograd
    // would otherwise copy an OIHW gradient into the parameter's strides)
    const bool ohwi = g_mode.load() > 1 && both_cl && weight.is_contiguous(at::MemoryFormat::ChannelsLast) &&
                      !weight.is_contiguous();
    dw = empty({Cout, Cin, 3, 3}, weight.scalar_type(), dev,
               ohwi ? at::MemoryFormat::ChannelsLast : at::MemoryFormat::Contiguous);
    if (g_mode.load() > 1 && both_cl) {
      // dY and x themselves are the operands: the job keeps them alive, and a
      // write into either (before_write) runs it first
      auto job = [dy = grad_output, x = input, gw = dw.data_ptr(), dtype = dw.scalar_type(), dev, B, Cin, H, W,
                  Cout, ohwi]() { launch_wgrad_nhwc(dy, x, gw, dtype, dev, B, Cin, H, W, Cout, ohwi); };
      if (deferral_enabled())
        defer_epilogue(dw, {grad_output, input}, nullptr, std::move(job));
      else
        job();
    } else if (g_mode.load() > 1) {
      if (!dy_rows.defined()) dy_rows = pack_rows(grad_output);
      at::Tensor x_rows = find_rows(input);
      if (!x_rows.defined() || x_rows.dim() != 2 || x_rows.size(0) != int64_t(B) * (H + 2) * (W + 2) ||
          x_rows.size(1) != int64_t(chunks_of(Cin)) * 64)
        x_rows = pack_rows(input);
      if (deferral_enabled()) {
        defer_write(dw, [dy_rows, x_rows, gw = dw.data_ptr(), dtype = dw.scalar_type(), dev, B, Cin, H, W, Cout]() {
          launch_wgrad(dy_rows, x_rows, gw, dtype, dev, B, Cin, H, W, Cout);
        });
      } else {
        launch_wgrad(dy_rows, x_rows, dw.data_ptr(), dw.scalar_type(), dev, B, Cin, H, W, Cout);
      }
    } else {
      // mode 1: weight gradient through ATen's CUDA path
      count_fallback("convolution_backward_overrideable.dw");
      auto r = at::convolution_backward(to_cuda(grad_output), to_cuda(input), to_cuda(weight), std::nullopt, stride,
                                        padding, dilation, transposed, output_padding, groups, {false, true, false});
      to_cuda_nosync(dw).copy_(std::get<1>(r));
    }
  }
  if (output_mask[0]) note_dgrad();
  return {dx, dw, db};
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("convolution_overrideable", convolution_overrideable);
  m.impl("convolution_backward_overrideable", convolution_backward_overrideable);
}

}  // namespace xdna
