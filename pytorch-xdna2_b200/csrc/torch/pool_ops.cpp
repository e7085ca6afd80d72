// 2-D max pooling with xdna kernels: `max_pool2d_with_indices` and its
// backward (the reference runs them on its CPU path; `nn.MaxPool2d` reaches
// them through the composite `max_pool2d`).  bf16 / fp32 4-D inputs in any
// layout (channels-last bf16 with C % 8 == 0 moves 16-byte vectors); other
// dtypes and 3-D inputs run ATen's CUDA kernels on zero-copy aliases.
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "xdna.h"

namespace xdna {
namespace {

struct Pool2d {
  int kh, kw, sh, sw, ph, pw, dh, dw;
  int64_t OH, OW;
};

int64_t out_size(int64_t in, int k, int pad, int s, int d, bool ceil_mode) {
  const int64_t num = in + 2 * pad - int64_t(d) * (k - 1) - 1 + (ceil_mode ? s - 1 : 0);
  int64_t o = (num >= 0 ? num / s : -((-num + s - 1) / s)) + 1;
  if (ceil_mode && (o - 1) * s >= in + pad) --o;
  return o;
}

bool parse(const at::Tensor& x, at::IntArrayRef k, at::IntArrayRef s, at::IntArrayRef p, at::IntArrayRef d,
           bool ceil_mode, Pool2d& g) {
  auto two = [](at::IntArrayRef v, int i, int64_t dflt) -> int64_t {
    if (v.empty()) return dflt;
    return v.size() == 1 ? v[0] : v[i];
  };
  if (x.dim() != 4 || k.empty() || k.size() > 2 || s.size() > 2 || p.size() > 2 || d.size() > 2) return false;
  g.kh = int(two(k, 0, 1));
  g.kw = int(two(k, 1, 1));
  g.sh = int(two(s, 0, g.kh));
  g.sw = int(two(s, 1, g.kw));
  g.ph = int(two(p, 0, 0));
  g.pw = int(two(p, 1, 0));
  g.dh = int(two(d, 0, 1));
  g.dw = int(two(d, 1, 1));
  if (g.kh <= 0 || g.kw <= 0 || g.sh <= 0 || g.sw <= 0 || g.dh <= 0 || g.dw <= 0 || g.ph < 0 || g.pw < 0 ||
      2 * g.ph > g.kh || 2 * g.pw > g.kw)
    return false;
  g.OH = out_size(x.size(2), g.kh, g.ph, g.sh, g.dh, ceil_mode);
  g.OW = out_size(x.size(3), g.kw, g.pw, g.sw, g.dw, ceil_mode);
  return g.OH > 0 && g.OW > 0;
}

int dtype_code(at::ScalarType t) { return t == at::kBFloat16 ? B2_BF16 : t == at::kFloat ? B2_F32 : -1; }

// Slot kind of the window taps kept on the int64 indices' storage (kinds
// below 16 are packed weights, from 16 the column matrices' geometry tags).
constexpr int kTapsSlot = 15;

// The window-tap kernels' case: channels-last bf16, C % 8 == 0, 3x3 windows
// spanning at most two strides (the backward's covering bound).
bool taps_pool(const at::Tensor& x, const Pool2d& g) {
  return x.scalar_type() == at::kBFloat16 && x.dim() == 4 &&
         x.suggest_memory_format() == at::MemoryFormat::ChannelsLast &&
         x.is_contiguous(at::MemoryFormat::ChannelsLast) && x.size(1) % 8 == 0 && g.kh == 3 && g.kw == 3 &&
         2 * (g.kh - 1) * g.dh + 2 <= 4 * g.sh && 2 * (g.kw - 1) * g.dw + 2 <= 4 * g.sw &&
         (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0;
}

std::tuple<at::Tensor, at::Tensor> max_pool2d_with_indices(const at::Tensor& self, at::IntArrayRef k,
                                                           at::IntArrayRef s, at::IntArrayRef p, at::IntArrayRef d,
                                                           bool ceil_mode) {
  Pool2d g;
  if (g_mode.load() == 0 || dtype_code(self.scalar_type()) < 0 || !parse(self, k, s, p, d, ceil_mode, g) ||
      self.numel() == 0) {
    count_fallback("aten::max_pool2d_with_indices");
    c10::cuda::CUDAGuard guard(self.device().index());
    auto r = at::max_pool2d_with_indices(to_cuda(self), k, s, p, d, ceil_mode);
    return {adopt(std::get<0>(r)), adopt(std::get<1>(r))};
  }
  const auto dev = self.device().index();
  const auto mf = self.suggest_memory_format();
  at::Tensor y = empty({self.size(0), self.size(1), g.OH, g.OW}, self.scalar_type(), dev, mf);
  at::Tensor ind = empty({self.size(0), self.size(1), g.OH, g.OW}, at::kLong, dev, mf);
  materialize(self);
  c10::cuda::CUDAGuard guard(dev);
  const int64_t xs[4] = {self.stride(0), self.stride(1), self.stride(2), self.stride(3)};
  const int64_t ys[4] = {y.stride(0), y.stride(1), y.stride(2), y.stride(3)};
  // channels-last bf16 3x3 windows: the argmax kept as window taps (1 byte an
  // element); ATen's int64 indices are written only when something reads
  // them -- the backward reads the taps (attached to the indices' storage)
  if (g_mode.load() > 1 && taps_pool(self, g)) {
    at::Tensor taps = empty({self.size(0), self.size(1), g.OH, g.OW}, at::kByte, dev, mf);
    const b2_status st =
        b2_maxpool2d_fwd_taps(self.data_ptr(), xs, y.data_ptr(), taps.data_ptr(), ys, self.size(0), self.size(1),
                              self.size(2), self.size(3), g.OH, g.OW, g.kh, g.kw, g.sh, g.sw, g.ph, g.pw, g.dh, g.dw,
                              stream(dev));
    if (st == B2_OK) {
      count_launch("maxpool2d.fwd");
      const int64_t N = self.size(0), C = self.size(1), H = self.size(2), W = self.size(3);
      defer_write(ind, [taps, ptr = ind.data_ptr<int64_t>(), ys4 = std::vector<int64_t>(ys, ys + 4), N, C, H, W, g,
                        dev]() {
        c10::cuda::CUDAGuard guard(dev);
        XDNA_B2(b2_maxpool2d_taps_to_indices(taps.data_ptr(), ys4.data(), ptr, N, C, H, W, g.OH, g.OW, g.kh, g.kw,
                                             g.sh, g.sw, g.ph, g.pw, g.dh, g.dw, stream(dev)));
        count_launch("maxpool2d.indices");
      }, /*kick=*/false);
      attach_packed_weight(ind, kTapsSlot, taps);
      return {y, ind};
    }
    TORCH_CHECK(st == B2_ERR_UNSUPPORTED, "xdna: b2_maxpool2d_fwd_taps failed (", st, "): ", b2_last_error());
  }
  XDNA_B2(b2_maxpool2d_fwd(self.data_ptr(), xs, y.data_ptr(), ind.data_ptr<int64_t>(), ys,
                           dtype_code(self.scalar_type()), self.size(0), self.size(1), self.size(2), self.size(3), g.OH,
                           g.OW, g.kh, g.kw, g.sh, g.sw, g.ph, g.pw, g.dh, g.dw, stream(dev)));
  count_launch("maxpool2d.fwd");
  return {y, ind};
}

at::Tensor max_pool2d_with_indices_backward(const at::Tensor& grad, const at::Tensor& self, at::IntArrayRef k,
                                            at::IntArrayRef s, at::IntArrayRef p, at::IntArrayRef d, bool ceil_mode,
                                            const at::Tensor& indices) {
  Pool2d g;
  const bool ok = g_mode.load() != 0 && dtype_code(self.scalar_type()) >= 0 && grad.scalar_type() == self.scalar_type() &&
                  indices.scalar_type() == at::kLong && parse(self, k, s, p, d, ceil_mode, g) &&
                  grad.dim() == 4 && indices.sizes() == grad.sizes() && grad.size(2) == g.OH && grad.size(3) == g.OW;
  if (!ok) {
    count_fallback("aten::max_pool2d_with_indices_backward");
    c10::cuda::CUDAGuard guard(self.device().index());
    return adopt(at::max_pool2d_with_indices_backward(to_cuda(grad), to_cuda(self), k, s, p, d, ceil_mode,
                                                      to_cuda(indices)));
  }
  const auto dev = self.device().index();
  // the forward's window taps, when the indices are still the forward's
  if (g_mode.load() > 1 && taps_pool(self, g) && grad.strides() == indices.strides() &&
      grad.is_contiguous(at::MemoryFormat::ChannelsLast)) {
    at::Tensor taps = find_packed_weight(indices, kTapsSlot);
    if (taps.defined() && taps.sizes() == indices.sizes() && taps.strides() == indices.strides()) {
      at::Tensor dx = empty(self.sizes(), self.scalar_type(), dev, at::MemoryFormat::ChannelsLast);
      materialize(grad);
      c10::cuda::CUDAGuard guard(dev);
      const int64_t xs[4] = {dx.stride(0), dx.stride(1), dx.stride(2), dx.stride(3)};
      const int64_t ys[4] = {grad.stride(0), grad.stride(1), grad.stride(2), grad.stride(3)};
      const b2_status st = b2_maxpool2d_bwd_taps(grad.data_ptr(), taps.data_ptr(), ys, dx.data_ptr(), xs,
                                                 self.size(0), self.size(1), self.size(2), self.size(3), g.OH, g.OW,
                                                 g.kh, g.kw, g.sh, g.sw, g.ph, g.pw, g.dh, g.dw, stream(dev));
      if (st == B2_OK) {
        count_launch("maxpool2d.bwd");
        return dx;
      }
      TORCH_CHECK(st == B2_ERR_UNSUPPORTED, "xdna: b2_maxpool2d_bwd_taps failed (", st, "): ", b2_last_error());
    }
  }
  // dy read with the indices' strides
  at::Tensor gy = grad.strides() == indices.strides() ? grad : grad.contiguous(indices.suggest_memory_format());
  at::Tensor ind = indices;
  if (gy.strides() != ind.strides()) {
    gy = grad.contiguous();
    ind = indices.contiguous();
  }
  at::Tensor dx = empty(self.sizes(), self.scalar_type(), dev, self.suggest_memory_format());
  materialize(gy);
  materialize(ind);
  c10::cuda::CUDAGuard guard(dev);
  const int64_t xs[4] = {dx.stride(0), dx.stride(1), dx.stride(2), dx.stride(3)};
  const int64_t ys[4] = {gy.stride(0), gy.stride(1), gy.stride(2), gy.stride(3)};
  XDNA_B2(b2_maxpool2d_bwd(gy.data_ptr(), ind.data_ptr<int64_t>(), ys, dx.data_ptr(), xs,
                           dtype_code(self.scalar_type()), self.size(0), self.size(1), self.size(2), self.size(3), g.OH,
                           g.OW, g.kh, g.kw, g.sh, g.sw, g.ph, g.pw, g.dh, g.dw, stream(dev)));
  count_launch("maxpool2d.bwd");
  return dx;
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("max_pool2d_with_indices", max_pool2d_with_indices);
  m.impl("max_pool2d_with_indices_backward", max_pool2d_with_indices_backward);
}

}  // namespace xdna
