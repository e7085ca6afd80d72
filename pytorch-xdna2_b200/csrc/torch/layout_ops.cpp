// Layout ops with xdna kernels: `cat`, `upsample_nearest2d` and
// `upsample_nearest2d_backward` (the reference's fast host versions,
// torch_xdna_device.cpp:3796-4175, registered at :5062-5070).
//
// Fast path (libxdna_b200 kernels, bit-exact with ATen):
//   cat       inputs of one dtype, all contiguous (NCHW order) or all
//             channels-last 4-D; output in that memory format.
//   upsample  bf16 / fp32 4-D, exactly 2x (output size 2H x 2W, scales absent
//             or 2.0), contiguous or channels-last input.
// Anything else runs ATen's CUDA kernel on zero-copy CUDA aliases, like every
// op without an xdna kernel.
#include <ATen/WrapDimUtils.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <vector>

#include "xdna.h"

namespace xdna {
namespace {

// Physical position of each logical dim, and the physical sizes, of a tensor
// in the given memory format (4-D channels-last stores N, H, W, C).
std::vector<int64_t> physical_order(int64_t ndim, bool channels_last) {
  std::vector<int64_t> order(ndim);
  for (int64_t d = 0; d < ndim; ++d) order[d] = d;
  if (channels_last) order = {0, 3, 1, 2};  // N->0, C->3, H->1, W->2
  return order;
}

bool skipped_in_cat(const at::Tensor& t) { return t.dim() == 1 && t.numel() == 0; }

at::Tensor cat_alias(const std::vector<at::Tensor>& ts, int64_t dim) {
  count_fallback("aten::cat");
  std::vector<at::Tensor> cu;
  cu.reserve(ts.size());
  for (const auto& t : ts) cu.push_back(to_cuda(t));
  c10::cuda::CUDAGuard g(ts.front().device().index());
  return adopt(at::cat(cu, dim));
}

at::Tensor cat(const at::ITensorListRef& tensors, int64_t dim) {
  std::vector<at::Tensor> all(tensors.begin(), tensors.end());
  TORCH_CHECK(!all.empty(), "torch.cat(): expected a non-empty list of Tensors");
  std::vector<at::Tensor> ts;
  for (const auto& t : all)
    if (!skipped_in_cat(t)) ts.push_back(t);
  if (ts.empty() || g_mode.load() == 0) return cat_alias(all, dim);
  const at::Tensor& first = ts.front();
  const int64_t ndim = first.dim();
  dim = c10::maybe_wrap_dim(dim, ndim);
  const auto dtype = first.scalar_type();
  const auto dev = first.device().index();
  const auto mf = first.suggest_memory_format();
  const bool cl = mf == c10::MemoryFormat::ChannelsLast;
  for (const auto& t : ts) {
    if (t.device().type() != kXdna || t.device().index() != dev || t.scalar_type() != dtype || t.dim() != ndim ||
        t.suggest_memory_format() != mf || !t.is_contiguous(mf))
      return cat_alias(all, dim);
    for (int64_t d = 0; d < ndim; ++d)
      TORCH_CHECK(d == dim || t.size(d) == first.size(d), "Sizes of tensors must match except in dimension ", dim,
                  ". Expected size ", first.size(d), " but got size ", t.size(d), " for tensor number 1 in the list.");
  }
  std::vector<int64_t> out_sizes(first.sizes().begin(), first.sizes().end());
  out_sizes[dim] = 0;
  for (const auto& t : ts) out_sizes[dim] += t.size(dim);
  at::Tensor out = empty(out_sizes, dtype, dev, mf);
  if (out.numel() == 0) return out;
  // out viewed physically as [outer, block]: outer = product of the physical
  // dims before `dim`, block = the rest (per source: its own extent of `dim`).
  const auto order = physical_order(ndim, cl);
  const int64_t pos = order[dim];
  std::vector<int64_t> phys(ndim);
  for (int64_t d = 0; d < ndim; ++d) phys[order[d]] = out_sizes[d];
  int64_t outer = 1;
  for (int64_t p = 0; p < pos; ++p) outer *= phys[p];
  const int64_t elt = int64_t(out.element_size());
  const int64_t out_block = outer ? out.numel() / outer * elt : 0;
  std::vector<const void*> srcs;
  std::vector<int64_t> blocks;
  for (const auto& t : ts) {
    materialize(t);
    srcs.push_back(t.data_ptr());
    blocks.push_back(outer ? t.numel() / outer * elt : 0);
  }
  c10::cuda::CUDAGuard g(dev);
  XDNA_B2(b2_cat_blocks(srcs.data(), blocks.data(), int(srcs.size()), out.data_ptr(), outer, out_block, stream(dev)));
  count_launch("cat");
  return out;
}

bool scales_2x(std::optional<double> sh, std::optional<double> sw) {
  return (!sh || *sh == 2.0) && (!sw || *sw == 2.0);
}

int b2_dtype(at::ScalarType t) {
  return t == at::kBFloat16 ? B2_BF16 : t == at::kFloat ? B2_F32 : -1;
}

// 0 = contiguous NCHW, 1 = channels-last, -1 = neither (ATen's output memory
// format follows the input's suggested one).
int layout_of(const at::Tensor& t) {
  const auto mf = t.suggest_memory_format();
  if (mf == c10::MemoryFormat::Contiguous && t.is_contiguous()) return 0;
  if (mf == c10::MemoryFormat::ChannelsLast && t.is_contiguous(mf)) return 1;
  return -1;
}

at::Tensor upsample_nearest2d(const at::Tensor& self, c10::SymIntArrayRef output_size, std::optional<double> sh,
                              std::optional<double> sw) {
  const auto osize = C10_AS_INTARRAYREF_SLOW(output_size);
  const int layout = self.dim() == 4 ? layout_of(self) : -1;
  if (g_mode.load() == 0 || self.dim() != 4 || osize.size() != 2 || b2_dtype(self.scalar_type()) < 0 ||
      layout < 0 || osize[0] != 2 * self.size(2) || osize[1] != 2 * self.size(3) || !scales_2x(sh, sw)) {
    count_fallback("aten::upsample_nearest2d");
    c10::cuda::CUDAGuard g(self.device().index());
    return adopt(at::upsample_nearest2d(to_cuda(self), osize, sh, sw));
  }
  const auto dev = self.device().index();
  const auto mf = layout ? c10::MemoryFormat::ChannelsLast : c10::MemoryFormat::Contiguous;
  at::Tensor out = empty({self.size(0), self.size(1), osize[0], osize[1]}, self.scalar_type(), dev, mf);
  materialize(self);
  c10::cuda::CUDAGuard g(dev);
  XDNA_B2(b2_upsample_nearest2x(self.data_ptr(), out.data_ptr(), b2_dtype(self.scalar_type()), layout, self.size(0),
                                self.size(1), self.size(2), self.size(3), stream(dev)));
  count_launch("upsample_nearest2x");
  return out;
}

at::Tensor upsample_nearest2d_backward(const at::Tensor& grad, c10::SymIntArrayRef output_size,
                                       c10::SymIntArrayRef input_size, std::optional<double> sh,
                                       std::optional<double> sw) {
  const auto osize = C10_AS_INTARRAYREF_SLOW(output_size);
  const auto isize = C10_AS_INTARRAYREF_SLOW(input_size);
  const int layout = grad.dim() == 4 ? layout_of(grad) : -1;
  const bool fast = g_mode.load() != 0 && grad.dim() == 4 && osize.size() == 2 && isize.size() == 4 &&
                    b2_dtype(grad.scalar_type()) >= 0 && layout >= 0 && scales_2x(sh, sw) &&
                    osize[0] == 2 * isize[2] && osize[1] == 2 * isize[3] && grad.size(0) == isize[0] &&
                    grad.size(1) == isize[1] && grad.size(2) == osize[0] && grad.size(3) == osize[1];
  if (!fast) {
    count_fallback("aten::upsample_nearest2d_backward");
    c10::cuda::CUDAGuard g(grad.device().index());
    return adopt(at::upsample_nearest2d_backward(to_cuda(grad), osize, isize, sh, sw));
  }
  const auto dev = grad.device().index();
  const auto mf = layout ? c10::MemoryFormat::ChannelsLast : c10::MemoryFormat::Contiguous;
  at::Tensor gi = empty(isize, grad.scalar_type(), dev, mf);
  materialize(grad);
  c10::cuda::CUDAGuard g(dev);
  XDNA_B2(b2_upsample_nearest2x_backward(grad.data_ptr(), gi.data_ptr(), b2_dtype(grad.scalar_type()), layout,
                                         isize[0], isize[1], isize[2], isize[3], stream(dev)));
  count_launch("upsample_nearest2x_backward");
  return gi;
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("cat", cat);
  m.impl("upsample_nearest2d", upsample_nearest2d);
  m.impl("upsample_nearest2d_backward", upsample_nearest2d_backward);
}

}  // namespace xdna
