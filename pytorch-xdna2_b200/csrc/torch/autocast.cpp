// torch.autocast("xdna"): the AutocastPrivateUse1 kernels, registered from
// PyTorch's own op lists exactly as its CUDA autocast does.  The reference
// registers the same lists (torch_xdna_device.cpp:5313-5344); with the default
// autocast dtype set to bfloat16 (xdna_train/device.py) conv / mm / addmm /
// bmm / linear run in BF16 and reach the hot-path kernels, while FP32-policy
// ops (losses, norms, softmax ...) run in FP32.
#include <ATen/autocast_mode.h>
#include <torch/library.h>

namespace {

#define XDNA_AUTOCAST_LOWER_PRECISION_FP(...) KERNEL_PRIVATEUSEONE(__VA_ARGS__, lower_precision_fp)
#define XDNA_AUTOCAST_FP32(...) KERNEL_PRIVATEUSEONE(__VA_ARGS__, fp32)
#define XDNA_AUTOCAST_FP32_SET_OPT_DTYPE(...) KERNEL_PRIVATEUSEONE(__VA_ARGS__, fp32_set_opt_dtype)
#define XDNA_AUTOCAST_PROMOTE(...) KERNEL_PRIVATEUSEONE(__VA_ARGS__, promote)
#define XDNA_AUTOCAST_DIFFERENT_REDISPATCH(REDISPATCH_FUNC, REGISTER_NAME, REGISTER_SIGNATURE, \
                                           REDISPATCH_SIGNATURE, POLICY)                       \
  KERNEL_DIFFERENT_REDISPATCH_SIGNATURE_PRIVATEUSEONE(REDISPATCH_FUNC, REGISTER_NAME,          \
                                                      REGISTER_SIGNATURE, REDISPATCH_SIGNATURE, POLICY)

using at::Tensor;
using c10::Scalar;
using c10::ScalarType;
using c10::IntArrayRef;
using at::Dimname;
using at::DimnameList;

// ops without an autocast policy pass straight through
TORCH_LIBRARY_IMPL(_, AutocastPrivateUse1, m) { m.fallback(torch::CppFunction::makeFallthrough()); }

TORCH_LIBRARY_IMPL(aten, AutocastPrivateUse1, m) {
  AT_FORALL_LOWER_PRECISION_FP(XDNA_AUTOCAST_LOWER_PRECISION_FP)
  AT_FORALL_FP32(XDNA_AUTOCAST_FP32)
  AT_FORALL_FP32_SET_OPT_DTYPE(XDNA_AUTOCAST_FP32_SET_OPT_DTYPE)
  AT_FORALL_DIFFERENT_REDISPATCH_SIGNATURE(XDNA_AUTOCAST_DIFFERENT_REDISPATCH)
  AT_FORALL_PROMOTE(XDNA_AUTOCAST_PROMOTE)
}

}  // namespace
