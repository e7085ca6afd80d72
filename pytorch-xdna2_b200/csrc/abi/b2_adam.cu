// Multi-tensor fused Adam / AdamW.  One pass per element: read grad, param,
// exp_avg, exp_avg_sq (and max_exp_avg_sq), write param and the moments, all
// arithmetic in fp32.  Tensor metadata travels in the kernel parameter block
// (no device allocation); a launch covers up to kMaxTensors tensors, split into
// kChunk-element chunks that one wave of resident CTAs walks with a grid
// stride (each thread updates two 8-element vectors per step, with 16-byte
// loads when the tensor's arrays are aligned).
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
// 8 consecutive elements (i % 8 == 0, arrays 16-byte aligned) kept as raw
// 16-byte words until used: one word for bf16, two for fp32.
template <typename T>
struct Raw8 {
  uint4 w[sizeof(T) == 2 ? 1 : 2];
};
template <typename T>
__device__ __forceinline__ void ld8(const void* p, long long i, Raw8<T>& r) {
  const uint4* q = reinterpret_cast<const uint4*>(static_cast<const T*>(p) + i);
#pragma unroll
  for (int k = 0; k < int(sizeof(T)) / 2; ++k) r.w[k] = q[k];
}
template <typename T>
__device__ __forceinline__ float elem(const Raw8<T>& r, int e) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(r.w);
  if constexpr (sizeof(T) == 2)
    return __uint_as_float((e & 1) ? (u[e >> 1] & 0xffff0000u) : (u[e >> 1] << 16));
  else
    return __uint_as_float(u[e]);
}
// Stores 8 values; bf16 through the hardware round-to-nearest-even pair
// conversion (cvt.rn.bf16x2.f32: the same result as f2bf for every non-NaN
// value, one instruction per pair).
template <typename T>
__device__ __forceinline__ void st8(void* p, long long i, const float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint32_t u[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
      u[k] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) = make_uint4(u[0], u[1], u[2], u[3]);
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
__device__ __forceinline__ void scalar_update(const AdamScalars& s, const Coef& c, void* P_, const void* G_, void* M_,
                                              void* V_, void* X_, long long j) {
  float p = ld<P>(P_, j), m = ld<S>(M_, j), v = ld<S>(V_, j), x = s.amsgrad ? ld<S>(X_, j) : 0.f;
  update(s, c, ld<P>(G_, j), p, m, v, x);
  st<P>(P_, j, p);
  st<S>(M_, j, m);
  st<S>(V_, j, v);
  if (s.amsgrad) st<S>(X_, j, x);
}

template <typename P, typename S>
__global__ void __launch_bounds__(kThreads, 3) adam_kernel(const __grid_constant__ AdamArgs a, const AdamScalars s) {
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
      // two 8-element vectors per thread, all their loads issued before the
      // math, so a warp keeps 8-10 independent 16-byte loads in flight while
      // the correctly rounded divisions and square roots of the update run
      for (long long i0 = begin + 8 * threadIdx.x; i0 < end; i0 += 16 * kThreads) {
        const long long i1 = i0 + 8 * kThreads;
        if (i0 + 8 > end || (i1 < end && i1 + 8 > end)) {  // ragged tail of the tensor
          for (long long j = i0; j < end && j < i0 + 8; ++j) scalar_update<P, S>(s, c, P_, G_, M_, V_, X_, j);
          for (long long j = i1; j < end && j < i1 + 8; ++j) scalar_update<P, S>(s, c, P_, G_, M_, V_, X_, j);
          continue;
        }
        const int nv = i1 < end ? 2 : 1;
        Raw8<P> rg[2], rp[2];
        Raw8<S> rm[2], rv[2], rx[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k < nv) {
            const long long i = k ? i1 : i0;
            ld8<P>(G_, i, rg[k]);
            ld8<P>(P_, i, rp[k]);
            ld8<S>(M_, i, rm[k]);
            ld8<S>(V_, i, rv[k]);
            if (s.amsgrad) ld8<S>(X_, i, rx[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k < nv) {
            const long long i = k ? i1 : i0;
            float p[8], m[8], v[8], x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              p[e] = elem<P>(rp[k], e);
              m[e] = elem<S>(rm[k], e);
              v[e] = elem<S>(rv[k], e);
              x[e] = s.amsgrad ? elem<S>(rx[k], e) : 0.f;
              update(s, c, elem<P>(rg[k], e), p[e], m[e], v[e], x[e]);
            }
            st8<P>(P_, i, p);
            st8<S>(M_, i, m);
            st8<S>(V_, i, v);
            if (s.amsgrad) st8<S>(X_, i, x);
          }
        }
      }
    } else {
      for (long long j = begin + threadIdx.x; j < end; j += kThreads) scalar_update<P, S>(s, c, P_, G_, M_, V_, X_, j);
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
  const int psz = hp->param_dtype == B2_F32 ? 4 : 2;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  // one wave of resident blocks (occupancy of this instantiation, per device)
  static int occ[64][4] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  int& o = occ[dev][(hp->param_dtype == B2_F32 ? 2 : 0) + (hp->state_dtype == B2_F32 ? 1 : 0)];
  if (!o) {
    int b = 0;
    B2_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, kThreads, 0), "occupancy"));
    o = std::max(1, b);
  }
  const int max_grid = o * sm_count(dev);
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
