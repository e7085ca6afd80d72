// Multi-tensor fused Adam / AdamW.  One pass per element: read grad, param,
// exp_avg, exp_avg_sq (and max_exp_avg_sq), write param and the moments, all
// arithmetic in fp32.  Tensor metadata travels in the kernel parameter block
// (no device allocation); a launch covers up to kMaxTensors tensors and
// kMaxBlocks chunks of kChunk elements, larger lists take several launches.
//
// The update follows PyTorch's Adam/AdamW definition that the reference's
// `_fused_adam_` CPU path runs (reached through the boxed fallback,
// xdna_train/_native/torch_xdna_device.cpp:5124-5260):
//   g = grad / grad_scale; g = maximize ? -g : g
//   AdamW: p *= 1 - lr*wd         Adam: g = fma(wd, p, g)
//   m = fma(1-beta1, g-m, m)      v = fma((1-beta2)*g, g, beta2*v)
//   denom = sqrt(amsgrad ? max(vmax, v) : v) / sqrt(1 - beta2^t) + eps
//   p -= (lr / (1 - beta1^t)) * m / denom
// with the scalar coefficients formed in double and rounded to fp32 once.
// This operation order reproduces torch's CPU _fused_adam_ bit for bit on
// bf16 parameters (checked in tests/test_gpu_abi.py); the explicit __f*_rn /
// __fmaf_rn intrinsics keep nvcc from contracting it differently.
#include <algorithm>
#include <cmath>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kMaxTensors = 64;
constexpr int kMaxBlocks = 320;
constexpr int kChunk = 16384;
constexpr int kThreads = 256;

struct AdamArgs {
  void* param[kMaxTensors];
  const void* grad[kMaxTensors];
  void* m[kMaxTensors];
  void* v[kMaxTensors];
  void* vmax[kMaxTensors];
  const float* step[kMaxTensors];
  long long numel[kMaxTensors];
  unsigned short block_tensor[kMaxBlocks];
  int block_chunk[kMaxBlocks];
};

struct AdamScalars {
  double lr, beta1, beta2, wd, eps;
  int amsgrad, maximize, adamw;
  const float* lr_tensor;
  const float* grad_scale;
  const float* found_inf;
};

template <typename T>
__device__ __forceinline__ float ld(const void* p, long long i) {
  if constexpr (sizeof(T) == 2)
    return bf2f(static_cast<const uint16_t*>(p)[i]);
  else
    return static_cast<const float*>(p)[i];
}
template <typename T>
__device__ __forceinline__ void st(void* p, long long i, float v) {
  if constexpr (sizeof(T) == 2)
    static_cast<uint16_t*>(p)[i] = f2bf(v);
  else
    static_cast<float*>(p)[i] = v;
}

template <typename P, typename S>
__global__ void __launch_bounds__(kThreads) adam_kernel(const __grid_constant__ AdamArgs a,
                                                        const AdamScalars s) {
  if (s.found_inf && *s.found_inf != 0.f) return;
  const int t = a.block_tensor[blockIdx.x];
  const long long begin = (long long)a.block_chunk[blockIdx.x] * kChunk;
  const long long end = min(begin + kChunk, a.numel[t]);
  const double step = double(*a.step[t]);
  const double lr = s.lr_tensor ? double(*s.lr_tensor) : s.lr;
  const double bc1 = 1.0 - pow(s.beta1, step);
  const double bc2 = 1.0 - pow(s.beta2, step);
  const float step_size = float(lr / bc1);
  const float bc2_sqrt = float(sqrt(bc2));
  const float omb1 = float(1.0 - s.beta1), omb2 = float(1.0 - s.beta2), b2 = float(s.beta2);
  const float wd = float(s.wd), eps = float(s.eps);
  const float decay = float(1.0 - lr * s.wd);
  const float gscale = s.grad_scale ? *s.grad_scale : 1.f;
  void* P_ = a.param[t];
  const void* G_ = a.grad[t];
  void* M_ = a.m[t];
  void* V_ = a.v[t];
  void* X_ = a.vmax[t];
  for (long long i = begin + threadIdx.x; i < end; i += kThreads) {
    float g = ld<P>(G_, i);
    if (s.grad_scale) g = __fdiv_rn(g, gscale);
    if (s.maximize) g = -g;
    float p = ld<P>(P_, i);
    if (s.wd != 0.0) {
      if (s.adamw)
        p = __fmul_rn(p, decay);
      else
        g = __fmaf_rn(wd, p, g);
    }
    float m = ld<S>(M_, i);
    float v = ld<S>(V_, i);
    m = __fmaf_rn(omb1, __fsub_rn(g, m), m);
    v = __fmaf_rn(__fmul_rn(omb2, g), g, __fmul_rn(b2, v));
    float vv = v;
    if (s.amsgrad) {
      vv = fmaxf(ld<S>(X_, i), v);
      st<S>(X_, i, vv);
    }
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vv), bc2_sqrt), eps);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(step_size, m), denom));
    st<P>(P_, i, p);
    st<S>(M_, i, m);
    st<S>(V_, i, v);
  }
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" b2_status b2_fused_adam(const b2_adam_tensor* tensors, int n, const b2_adam_hparams* hp,
                                   void* stream) {
  if (n < 0 || (n > 0 && !tensors) || !hp) return set_error(B2_ERR_INVALID, "b2_fused_adam: bad arguments");
  if ((hp->param_dtype != B2_BF16 && hp->param_dtype != B2_F32) ||
      (hp->state_dtype != B2_BF16 && hp->state_dtype != B2_F32))
    return set_error(B2_ERR_INVALID, "b2_fused_adam: dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  AdamScalars sc{};
  sc.lr = hp->lr;
  sc.beta1 = hp->beta1;
  sc.beta2 = hp->beta2;
  sc.wd = hp->weight_decay;
  sc.eps = hp->eps;
  sc.amsgrad = hp->amsgrad;
  sc.maximize = hp->maximize;
  sc.adamw = hp->adamw;
  sc.lr_tensor = hp->lr_tensor;
  sc.grad_scale = hp->grad_scale;
  sc.found_inf = hp->found_inf;
  auto kern = hp->param_dtype == B2_F32
                  ? (hp->state_dtype == B2_F32 ? adam_kernel<float, float> : adam_kernel<float, uint16_t>)
                  : (hp->state_dtype == B2_F32 ? adam_kernel<uint16_t, float> : adam_kernel<uint16_t, uint16_t>);
  AdamArgs args;
  int nt = 0, nb = 0;
  auto flush = [&]() -> b2_status {
    if (nb == 0) return B2_OK;
    kern<<<nb, kThreads, 0, st>>>(args, sc);
    nt = 0;
    nb = 0;
    return check_cuda(cudaGetLastError(), "fused adam launch");
  };
  for (int i = 0; i < n; ++i) {
    const b2_adam_tensor& t = tensors[i];
    if (t.numel <= 0) continue;
    if (!t.param || !t.grad || !t.exp_avg || !t.exp_avg_sq || !t.step || (hp->amsgrad && !t.max_exp_avg_sq))
      return set_error(B2_ERR_INVALID, "b2_fused_adam: null pointer in tensor %d", i);
    const long long chunks = (t.numel + kChunk - 1) / kChunk;
    long long c = 0;
    while (c < chunks) {
      if (nt == kMaxTensors || nb == kMaxBlocks) B2_TRY(flush());
      args.param[nt] = t.param;
      args.grad[nt] = t.grad;
      args.m[nt] = t.exp_avg;
      args.v[nt] = t.exp_avg_sq;
      args.vmax[nt] = t.max_exp_avg_sq;
      args.step[nt] = t.step;
      args.numel[nt] = t.numel;
      while (c < chunks && nb < kMaxBlocks) {
        args.block_tensor[nb] = (unsigned short)nt;
        args.block_chunk[nb] = int(c);
        ++nb;
        ++c;
      }
      ++nt;
    }
  }
  return flush();
}
