// Multi-tensor fused Adam / AdamW.  One pass per element: read grad, param,
// exp_avg, exp_avg_sq (and max_exp_avg_sq), write param and the moments, all
// arithmetic in fp32.  Tensor metadata travels in the kernel parameter block
// (no device allocation); a launch covers up to kMaxTensors tensors, split into
// kChunk-element chunks that a grid of at most 4 CTAs per SM walks with a
// grid stride (each thread updates 4 consecutive elements per step, with
// vector loads when the tensor's arrays are aligned).
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
constexpr int kChunk = 4096;
constexpr int kThreads = 256;

struct AdamArgs {
  void* param[kMaxTensors];
  const void* grad[kMaxTensors];
  void* m[kMaxTensors];
  void* v[kMaxTensors];
  void* vmax[kMaxTensors];
  const float* step[kMaxTensors];
  long long numel[kMaxTensors];
  int chunk_begin[kMaxTensors + 1];  // prefix sums of chunks per tensor
  unsigned char vec[kMaxTensors];    // all arrays 16-byte aligned (8-element vectors)
  int ntensors;
};

struct AdamScalars {
  double lr, beta1, beta2, wd, eps;
  int amsgrad, maximize, adamw;
  const float* lr_tensor;
  const float* grad_scale;
  const float* found_inf;
};

struct Coef {
  float step_size, bc2_sqrt, omb1, omb2, b2, wd, eps, decay, gscale;
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
// 8 consecutive elements (i % 8 == 0, arrays 16-byte aligned): one 16-byte
// access for bf16, two for fp32.
template <typename T>
__device__ __forceinline__ void ld8(const void* p, long long i, float (&o)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[2 * k] = __uint_as_float(w[k] << 16);
      o[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i + 4);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  }
}
template <typename T>
__device__ __forceinline__ void st8(void* p, long long i, const float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    u.x = uint32_t(f2bf(v[0])) | (uint32_t(f2bf(v[1])) << 16);
    u.y = uint32_t(f2bf(v[2])) | (uint32_t(f2bf(v[3])) << 16);
    u.z = uint32_t(f2bf(v[4])) | (uint32_t(f2bf(v[5])) << 16);
    u.w = uint32_t(f2bf(v[6])) | (uint32_t(f2bf(v[7])) << 16);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) = u;
  } else {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__device__ __forceinline__ void update(const AdamScalars& s, const Coef& c, float g, float& p, float& m, float& v,
                                       float& vx) {
  if (s.grad_scale) g = __fdiv_rn(g, c.gscale);
  if (s.maximize) g = -g;
  if (s.wd != 0.0) {
    if (s.adamw)
      p = __fmul_rn(p, c.decay);
    else
      g = __fmaf_rn(c.wd, p, g);
  }
  m = __fmaf_rn(c.omb1, __fsub_rn(g, m), m);
  v = __fmaf_rn(__fmul_rn(c.omb2, g), g, __fmul_rn(c.b2, v));
  float vv = v;
  if (s.amsgrad) {
    vv = fmaxf(vx, v);
    vx = vv;
  }
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vv), c.bc2_sqrt), c.eps);
  p = __fsub_rn(p, __fdiv_rn(__fmul_rn(c.step_size, m), denom));
}

template <typename P, typename S>
__global__ void __launch_bounds__(kThreads) adam_kernel(const __grid_constant__ AdamArgs a, const AdamScalars s) {
  if (s.found_inf && *s.found_inf != 0.f) return;
  __shared__ Coef sc;
  const int total = a.chunk_begin[a.ntensors];
  int t = 0;
  int cur = -1;
  for (int chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    while (chunk >= a.chunk_begin[t + 1]) ++t;
    if (t != cur) {
      __syncthreads();  // everyone is done with the previous coefficients
      if (threadIdx.x == 0) {
        const double step = double(*a.step[t]);
        const double lr = s.lr_tensor ? double(*s.lr_tensor) : s.lr;
        const double bc1 = 1.0 - pow(s.beta1, step);
        const double bc2 = 1.0 - pow(s.beta2, step);
        sc.step_size = float(lr / bc1);
        sc.bc2_sqrt = float(sqrt(bc2));
        sc.omb1 = float(1.0 - s.beta1);
        sc.omb2 = float(1.0 - s.beta2);
        sc.b2 = float(s.beta2);
        sc.wd = float(s.wd);
        sc.eps = float(s.eps);
        sc.decay = float(1.0 - lr * s.wd);
        sc.gscale = s.grad_scale ? *s.grad_scale : 1.f;
      }
      __syncthreads();
      cur = t;
    }
    const Coef c = sc;
    const long long begin = (long long)(chunk - a.chunk_begin[t]) * kChunk;
    const long long end = min(begin + kChunk, a.numel[t]);
    void* P_ = a.param[t];
    const void* G_ = a.grad[t];
    void* M_ = a.m[t];
    void* V_ = a.v[t];
    void* X_ = a.vmax[t];
    if (a.vec[t]) {
      for (long long i = begin + 8 * threadIdx.x; i < end; i += 8 * kThreads) {
        if (i + 8 <= end) {
          float g[8], p[8], m[8], v[8], x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          ld8<P>(G_, i, g);
          ld8<P>(P_, i, p);
          ld8<S>(M_, i, m);
          ld8<S>(V_, i, v);
          if (s.amsgrad) ld8<S>(X_, i, x);
#pragma unroll
          for (int k = 0; k < 8; ++k) update(s, c, g[k], p[k], m[k], v[k], x[k]);
          st8<P>(P_, i, p);
          st8<S>(M_, i, m);
          st8<S>(V_, i, v);
          if (s.amsgrad) st8<S>(X_, i, x);
        } else {
          for (long long j = i; j < end; ++j) {
            float p = ld<P>(P_, j), m = ld<S>(M_, j), v = ld<S>(V_, j), x = s.amsgrad ? ld<S>(X_, j) : 0.f;
            update(s, c, ld<P>(G_, j), p, m, v, x);
            st<P>(P_, j, p);
            st<S>(M_, j, m);
            st<S>(V_, j, v);
            if (s.amsgrad) st<S>(X_, j, x);
          }
        }
      }
    } else {
      for (long long j = begin + threadIdx.x; j < end; j += kThreads) {
        float p = ld<P>(P_, j), m = ld<S>(M_, j), v = ld<S>(V_, j), x = s.amsgrad ? ld<S>(X_, j) : 0.f;
        update(s, c, ld<P>(G_, j), p, m, v, x);
        st<P>(P_, j, p);
        st<S>(M_, j, m);
        st<S>(V_, j, v);
        if (s.amsgrad) st<S>(X_, j, x);
      }
    }
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
  const int psz = hp->param_dtype == B2_F32 ? 4 : 2, ssz = hp->state_dtype == B2_F32 ? 4 : 2;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int max_grid = 4 * sm_count(dev);
  AdamArgs args;
  args.ntensors = 0;
  args.chunk_begin[0] = 0;
  auto flush = [&]() -> b2_status {
    const int total = args.chunk_begin[args.ntensors];
    if (total > 0) {
      kern<<<std::min(total, max_grid), kThreads, 0, st>>>(args, sc);
      B2_TRY(check_cuda(cudaGetLastError(), "fused adam launch"));
    }
    args.ntensors = 0;
    args.chunk_begin[0] = 0;
    return B2_OK;
  };
  auto al = [](const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; };
  for (int i = 0; i < n; ++i) {
    const b2_adam_tensor& t = tensors[i];
    if (t.numel <= 0) continue;
    if (!t.param || !t.grad || !t.exp_avg || !t.exp_avg_sq || !t.step || (hp->amsgrad && !t.max_exp_avg_sq))
      return set_error(B2_ERR_INVALID, "b2_fused_adam: null pointer in tensor %d", i);
    const long long chunks = (t.numel + kChunk - 1) / kChunk;
    if (chunks > (1LL << 30)) return set_error(B2_ERR_UNSUPPORTED, "b2_fused_adam: tensor %d too large", i);
    if (args.ntensors == kMaxTensors || args.chunk_begin[args.ntensors] + chunks > (1LL << 30)) B2_TRY(flush());
    const int k = args.ntensors;
    args.param[k] = t.param;
    args.grad[k] = t.grad;
    args.m[k] = t.exp_avg;
    args.v[k] = t.exp_avg_sq;
    args.vmax[k] = t.max_exp_avg_sq;
    args.step[k] = t.step;
    args.numel[k] = t.numel;
    args.vec[k] = al(t.param, 16) && al(t.grad, 16) && al(t.exp_avg, 16) && al(t.exp_avg_sq, 16) &&
                  (!hp->amsgrad || al(t.max_exp_avg_sq, 16));
    args.chunk_begin[k + 1] = args.chunk_begin[k] + int(chunks);
    args.ntensors = k + 1;
  }
  return flush();
}
