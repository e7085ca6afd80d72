// Fused region kernels behind xdna_train.regions (the frozen-feature MSE
// loss).  Same element-wise contracts as the reference's host kernels
// (xdna_train/_native/region_kernels.cpp:1-307): bf16 storage, fp32
// arithmetic rounded once to bf16 (nearest even), ReLU keeps NaN, max-pool
// takes PyTorch's first maximum with NaN winning.  Everything except the
// squared-difference sum is bit-exact with the reference.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ bool nan_or_gt(float v, float m) { return (v > m) || (v != v); }

// NaN results follow x86 SSE propagation (first NaN operand, quieted; an
// invalid operation gives the default NaN 0xFFC00000), the arithmetic of the
// reference's host build.  With it even NaN payloads match bit for bit.
__device__ __forceinline__ float x86_nan(float r, float x, float y) {
  const uint32_t xu = __float_as_uint(x), yu = __float_as_uint(y), ru = __float_as_uint(r);
  if ((xu & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(xu | 0x00400000u);
  if ((yu & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(yu | 0x00400000u);
  if ((ru & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(0xFFC00000u);
  return r;
}
__device__ __forceinline__ float xsub(float a, float b) { return x86_nan(__fsub_rn(a, b), a, b); }
__device__ __forceinline__ float xmul(float a, float b) { return x86_nan(__fmul_rn(a, b), a, b); }
__device__ __forceinline__ float xadd(float a, float b) { return x86_nan(__fadd_rn(a, b), a, b); }

__device__ __forceinline__ uint16_t relu_bits(uint16_t a) {
  return (bf2f(a) <= 0.0f) ? uint16_t(0) : a;
}

int grid_for(long long n) {
  const long long b = (n + kThreads - 1) / kThreads;
  return int(std::max<long long>(1, std::min<long long>(b, 148LL * 32)));
}

__global__ void sqdiff_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                              long long n, double* out) {
  float acc = 0.f;
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < n;
       i += (long long)gridDim.x * kThreads) {
    const float d = __fsub_rn(bf2f(a[i]), bf2f(b[i]));
    acc = __fmaf_rn(d, d, acc);
  }
  double dacc = acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dacc += __shfl_xor_sync(0xffffffffu, dacc, o);
  __shared__ double part[kThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = dacc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0;
    for (int w = 0; w < kThreads / 32; ++w) s += part[w];
    atomicAdd(out, s);
  }
}

__global__ void relu_kernel(const uint16_t* __restrict__ a, uint16_t* __restrict__ r, long long n) {
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < n;
       i += (long long)gridDim.x * kThreads)
    r[i] = relu_bits(a[i]);
}

// One thread per 2x2 window of the ceil(H/2) x ceil(W/2) grid: writes the
// relu of the window's elements and, for complete windows, the pooled value.
__global__ void relu_maxpool2_kernel(const uint16_t* __restrict__ a, uint16_t* __restrict__ r,
                                     uint16_t* __restrict__ p, long long planes, int H, int W) {
  const int Hc = (H + 1) / 2, Wc = (W + 1) / 2;
  const int Ho = H / 2, Wo = W / 2;
  const long long total = planes * Hc * Wc;
  const bool even_w = (W & 1) == 0;
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < total;
       i += (long long)gridDim.x * kThreads) {
    const int xo = int(i % Wc);
    const int yo = int((i / Wc) % Hc);
    const long long pl = i / ((long long)Wc * Hc);
    const long long base = pl * H * W;
    const int y0 = 2 * yo, x0 = 2 * xo;
    uint16_t e[4] = {0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int yy = y0 + (k >> 1), xx = x0 + (k & 1);
      if (yy < H && xx < W) {
        e[k] = relu_bits(a[base + (long long)yy * W + xx]);
        r[base + (long long)yy * W + xx] = e[k];
      }
    }
    if (yo < Ho && xo < Wo) {
      uint16_t m;
      if (even_w) {
        // vertical pairs first, then horizontal (region_kernels.cpp:98-122)
        const float f00 = bf2f(e[0]), f01 = bf2f(e[1]), f10 = bf2f(e[2]), f11 = bf2f(e[3]);
        const bool s0 = nan_or_gt(f10, f00);
        const uint16_t m0 = s0 ? e[2] : e[0];
        const float v0 = s0 ? f10 : f00;
        const bool s1 = nan_or_gt(f11, f01);
        const uint16_t m1 = s1 ? e[3] : e[1];
        const float v1 = s1 ? f11 : f01;
        m = nan_or_gt(v1, v0) ? m1 : m0;
      } else {
        // scan order (region_kernels.cpp:169-180)
        m = e[0];
        float mv = bf2f(m);
#pragma unroll
        for (int k = 1; k < 4; ++k) {
          const float v = bf2f(e[k]);
          if (nan_or_gt(v, mv)) {
            m = e[k];
            mv = v;
          }
        }
      }
      p[pl * Ho * Wo + (long long)yo * Wo + xo] = m;
    }
  }
}

__global__ void addtap_kernel(const uint16_t* __restrict__ base, const uint16_t* __restrict__ a,
                              const uint16_t* __restrict__ b, uint16_t* __restrict__ out,
                              long long n, float scale) {
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < n;
       i += (long long)gridDim.x * kThreads) {
    // no fma contraction: the reference rounds the product and the sum apart
    const float t = xmul(scale, xsub(bf2f(a[i]), bf2f(b[i])));
    out[i] = f2bf(base ? xadd(bf2f(base[i]), t) : t);
  }
}

__global__ void relu_bwd_kernel(const uint16_t* __restrict__ r, const uint16_t* __restrict__ base,
                                const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                                uint16_t* __restrict__ out, long long n, float scale) {
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < n;
       i += (long long)gridDim.x * kThreads) {
    float g = 0.0f;
    if (base) g = bf2f(base[i]);
    if (a) g = xadd(g, xmul(scale, xsub(bf2f(a[i]), bf2f(b[i]))));
    out[i] = (bf2f(r[i]) <= 0.0f) ? uint16_t(0) : f2bf(g);
  }
}

__global__ void maxpool2_bwd_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ g,
                                    uint16_t* __restrict__ out, long long planes, int H, int W) {
  const int Hc = (H + 1) / 2, Wc = (W + 1) / 2;
  const int Ho = H / 2, Wo = W / 2;
  const long long total = planes * Hc * Wc;
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < total;
       i += (long long)gridDim.x * kThreads) {
    const int xo = int(i % Wc);
    const int yo = int((i / Wc) % Hc);
    const long long pl = i / ((long long)Wc * Hc);
    const long long base = pl * H * W;
    const int y0 = 2 * yo, x0 = 2 * xo;
    int best = -1;
    uint16_t gv = 0;
    if (yo < Ho && xo < Wo) {
      const long long o = base + (long long)y0 * W + x0;
      const float e0 = bf2f(x[o]), e1 = bf2f(x[o + 1]), e2 = bf2f(x[o + W]), e3 = bf2f(x[o + W + 1]);
      float mv = e0;
      best = 0;
      if (nan_or_gt(e1, mv)) { best = 1; mv = e1; }
      if (nan_or_gt(e2, mv)) { best = 2; mv = e2; }
      if (nan_or_gt(e3, mv)) { best = 3; }
      gv = g[pl * Ho * Wo + (long long)yo * Wo + xo];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int yy = y0 + (k >> 1), xx = x0 + (k & 1);
      if (yy < H && xx < W) out[base + (long long)yy * W + xx] = (k == best) ? gv : uint16_t(0);
    }
  }
}

}  // namespace
}  // namespace b2

using namespace b2;

#define B2_U16(p) static_cast<const uint16_t*>(p)
#define B2_STREAM static_cast<cudaStream_t>(stream)

extern "C" {

b2_status b2_region_sqdiff_sum_bf16(const void* a, const void* b, int64_t n, double* out, void* stream) {
  if (!out || n < 0 || (n > 0 && (!a || !b))) return set_error(B2_ERR_INVALID, "b2_region_sqdiff_sum_bf16: bad arguments");
  B2_TRY(check_cuda(cudaMemsetAsync(out, 0, sizeof(double), B2_STREAM), "memset"));
  if (n == 0) return B2_OK;
  sqdiff_kernel<<<grid_for(n), kThreads, 0, B2_STREAM>>>(B2_U16(a), B2_U16(b), n, out);
  return check_cuda(cudaGetLastError(), "sqdiff launch");
}

b2_status b2_region_relu_bf16(const void* a, void* r, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!a || !r))) return set_error(B2_ERR_INVALID, "b2_region_relu_bf16: bad arguments");
  if (n == 0) return B2_OK;
  relu_kernel<<<grid_for(n), kThreads, 0, B2_STREAM>>>(B2_U16(a), static_cast<uint16_t*>(r), n);
  return check_cuda(cudaGetLastError(), "relu launch");
}

b2_status b2_region_relu_maxpool2_bf16(const void* a, void* r, void* p, int64_t planes, int64_t H,
                                       int64_t W, void* stream) {
  if (planes < 0 || H < 0 || W < 0 || H > (1 << 30) || W > (1 << 30))
    return set_error(B2_ERR_INVALID, "b2_region_relu_maxpool2_bf16: bad shape");
  const long long total = planes * ((H + 1) / 2) * ((W + 1) / 2);
  if (total == 0) return B2_OK;
  if (!a || !r || (!p && H >= 2 && W >= 2)) return set_error(B2_ERR_INVALID, "b2_region_relu_maxpool2_bf16: null pointer");
  relu_maxpool2_kernel<<<grid_for(total), kThreads, 0, B2_STREAM>>>(
      B2_U16(a), static_cast<uint16_t*>(r), static_cast<uint16_t*>(p), planes, int(H), int(W));
  return check_cuda(cudaGetLastError(), "relu_maxpool2 launch");
}

b2_status b2_region_addtap_bf16(const void* base, const void* a, const void* b, void* out, int64_t n,
                                float scale, void* stream) {
  if (n < 0 || (n > 0 && (!a || !b || !out))) return set_error(B2_ERR_INVALID, "b2_region_addtap_bf16: bad arguments");
  if (n == 0) return B2_OK;
  addtap_kernel<<<grid_for(n), kThreads, 0, B2_STREAM>>>(B2_U16(base), B2_U16(a), B2_U16(b),
                                                         static_cast<uint16_t*>(out), n, scale);
  return check_cuda(cudaGetLastError(), "addtap launch");
}

b2_status b2_region_relu_bwd_bf16(const void* r, const void* base, const void* a, const void* b,
                                  void* out, int64_t n, float scale, void* stream) {
  if (n < 0 || (n > 0 && (!r || !out)) || (!a) != (!b))
    return set_error(B2_ERR_INVALID, "b2_region_relu_bwd_bf16: bad arguments");
  if (n == 0) return B2_OK;
  relu_bwd_kernel<<<grid_for(n), kThreads, 0, B2_STREAM>>>(B2_U16(r), B2_U16(base), B2_U16(a), B2_U16(b),
                                                           static_cast<uint16_t*>(out), n, scale);
  return check_cuda(cudaGetLastError(), "relu_bwd launch");
}

b2_status b2_region_maxpool2_bwd_bf16(const void* x, const void* g, void* out, int64_t planes,
                                      int64_t H, int64_t W, void* stream) {
  if (planes < 0 || H < 0 || W < 0 || H > (1 << 30) || W > (1 << 30))
    return set_error(B2_ERR_INVALID, "b2_region_maxpool2_bwd_bf16: bad shape");
  const long long total = planes * ((H + 1) / 2) * ((W + 1) / 2);
  if (total == 0) return B2_OK;
  if (!x || !out || (!g && H >= 2 && W >= 2)) return set_error(B2_ERR_INVALID, "b2_region_maxpool2_bwd_bf16: null pointer");
  maxpool2_bwd_kernel<<<grid_for(total), kThreads, 0, B2_STREAM>>>(B2_U16(x), B2_U16(g),
                                                                   static_cast<uint16_t*>(out), planes,
                                                                   int(H), int(W));
  return check_cuda(cudaGetLastError(), "maxpool2_bwd launch");
}

}  // extern "C"
