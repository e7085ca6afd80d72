// Layout ops on the device: concatenation of contiguous tensors and exact-2x
// nearest upsampling (forward and backward), for bf16 and fp32, in NCHW or
// NHWC (channels-last) memory order.  The reference runs these as OpenMP host
// loops (torch_xdna_device.cpp:3796-4175) that reproduce ATen's CPU results
// bit for bit; these kernels keep that contract:
//
//   cat / upsample forward   pure copies.
//   upsample backward        each input gradient is the sum of its 2x2 block
//                            of output gradients in fp32, starting from +0, in
//                            raster order (g[2y][2x], g[2y][2x+1], g[2y+1][2x],
//                            g[2y+1][2x+1]) -- ATen's CPU accumulation order --
//                            with x86 SSE NaN propagation, rounded once (bf16:
//                            nearest even, any NaN -> 0x7FC0 as c10::BFloat16).
//
// All are HBM-bound copies: 16-byte vector loads and stores wherever the sizes
// and addresses allow, grid-stride loops sized to the SM count.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kLayoutThreads = 256;
constexpr int kMaxCat = 32;

int layout_grid(long long units, int sms, int per_sm = 16) {
  const long long b = (units + kLayoutThreads - 1) / kLayoutThreads;
  return int(std::max<long long>(1, std::min<long long>(b, (long long)sms * per_sm)));
}

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % uintptr_t(a)) == 0; }

// ---- cat -------------------------------------------------------------------

struct CatBatch {
  const char* src[kMaxCat];
  long long block[kMaxCat];  // units per outer index
  long long off[kMaxCat];    // unit offset inside an output block
};

// blockIdx.y = source; units of sizeof(U) bytes.
template <typename U>
__global__ void __launch_bounds__(kLayoutThreads) cat_kernel(CatBatch b, U* __restrict__ dst, long long outer,
                                                             long long out_block) {
  const int i = blockIdx.y;
  const long long blk = b.block[i];
  const long long total = outer * blk;
  const U* __restrict__ src = reinterpret_cast<const U*>(b.src[i]);
  U* __restrict__ d = dst + b.off[i];
  for (long long u = (long long)blockIdx.x * kLayoutThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kLayoutThreads) {
    const long long o = u / blk;
    d[o * out_block + (u - o * blk)] = src[u];
  }
}

// ---- upsample forward ------------------------------------------------------

// NCHW: one thread per Q consecutive inputs of a row; writes 2Q outputs to
// each of the two output rows.  `rows` = N*C*H.
template <typename T, int Q>
__global__ void __launch_bounds__(kLayoutThreads) up2x_nchw_kernel(const T* __restrict__ in, T* __restrict__ out,
                                                                   long long rows, long long W) {
  const long long qpr = W / Q;
  const long long total = rows * qpr;
  for (long long u = (long long)blockIdx.x * kLayoutThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kLayoutThreads) {
    const long long row = u / qpr, q = u - row * qpr;
    alignas(16) T v[Q];
    alignas(16) T o[2 * Q];
    const T* s = in + row * W + q * Q;
    if constexpr (Q * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(v) = *reinterpret_cast<const uint4*>(s);
    } else if constexpr (Q * sizeof(T) == 8) {
      *reinterpret_cast<uint2*>(v) = *reinterpret_cast<const uint2*>(s);
    } else {
#pragma unroll
      for (int k = 0; k < Q; ++k) v[k] = s[k];
    }
#pragma unroll
    for (int k = 0; k < Q; ++k) o[2 * k] = o[2 * k + 1] = v[k];
    T* r0 = out + row * 4 * W + q * 2 * Q;  // output row 2y of the plane
    T* r1 = r0 + 2 * W;                     // output row 2y + 1
    if constexpr ((2 * Q * sizeof(T)) % 16 == 0) {
#pragma unroll
      for (int k = 0; k < int(2 * Q * sizeof(T) / 16); ++k) {
        const uint4 w = reinterpret_cast<const uint4*>(o)[k];
        reinterpret_cast<uint4*>(r0)[k] = w;
        reinterpret_cast<uint4*>(r1)[k] = w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 2 * Q; ++k) r0[k] = r1[k] = o[k];
    }
  }
}

// NHWC: one thread per output pixel and unit of U bytes along C (`cu` units
// per pixel); every output pixel copies its source pixel.
template <typename U>
__global__ void __launch_bounds__(kLayoutThreads) up2x_nhwc_kernel(const U* __restrict__ in, U* __restrict__ out,
                                                                   long long N, long long H, long long W,
                                                                   long long cu) {
  const long long total = N * 4 * H * W * cu;
  for (long long u = (long long)blockIdx.x * kLayoutThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kLayoutThreads) {
    const long long pix = u / cu, k = u - pix * cu;
    const long long ox = pix % (2 * W), oy = (pix / (2 * W)) % (2 * H), b = pix / (4 * H * W);
    out[u] = in[((b * H + (oy >> 1)) * W + (ox >> 1)) * cu + k];
  }
}

// ---- upsample backward -----------------------------------------------------

__device__ __forceinline__ float x86_add(float a, float b) {
  // x86 SSE: a NaN operand propagates quieted, the first one first; an
  // invalid operation (inf - inf) gives the default NaN 0xFFC00000.
  const float r = __fadd_rn(a, b);
  const uint32_t au = __float_as_uint(a), bu = __float_as_uint(b);
  if ((au & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(au | 0x00400000u);
  if ((bu & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(bu | 0x00400000u);
  if (r != r) return __uint_as_float(0xFFC00000u);
  return r;
}

// c10::BFloat16(float): nearest even, every NaN -> 0x7FC0.
__device__ __forceinline__ uint16_t f2bf_aten(float f) {
  if (f != f) return 0x7FC0;
  const uint32_t u = __float_as_uint(f);
  return uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

template <typename T>
__device__ __forceinline__ float ld_f(T v) {
  if constexpr (sizeof(T) == 2) return bf2f(v);
  else return v;
}
template <typename T>
__device__ __forceinline__ T st_f(float v) {
  if constexpr (sizeof(T) == 2) return f2bf_aten(v);
  else return v;
}

__device__ __forceinline__ float sum4(float a, float b, float c, float d) {
  return x86_add(x86_add(x86_add(x86_add(0.0f, a), b), c), d);
}

// NCHW: one thread per Q consecutive input gradients of a row.
template <typename T, int Q>
__global__ void __launch_bounds__(kLayoutThreads) up2x_bwd_nchw_kernel(const T* __restrict__ go, T* __restrict__ gi,
                                                                       long long rows, long long W) {
  const long long qpr = W / Q;
  const long long total = rows * qpr;
  for (long long u = (long long)blockIdx.x * kLayoutThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kLayoutThreads) {
    const long long row = u / qpr, q = u - row * qpr;
    const T* r0 = go + row * 4 * W + q * 2 * Q;
    const T* r1 = r0 + 2 * W;
    alignas(16) T a[2 * Q];
    alignas(16) T c[2 * Q];
    alignas(16) T o[Q];
    if constexpr ((2 * Q * sizeof(T)) % 16 == 0) {
#pragma unroll
      for (int k = 0; k < int(2 * Q * sizeof(T) / 16); ++k) {
        reinterpret_cast<uint4*>(a)[k] = reinterpret_cast<const uint4*>(r0)[k];
        reinterpret_cast<uint4*>(c)[k] = reinterpret_cast<const uint4*>(r1)[k];
      }
    } else {
#pragma unroll
      for (int k = 0; k < 2 * Q; ++k) {
        a[k] = r0[k];
        c[k] = r1[k];
      }
    }
#pragma unroll
    for (int k = 0; k < Q; ++k)
      o[k] = st_f<T>(sum4(ld_f(a[2 * k]), ld_f(a[2 * k + 1]), ld_f(c[2 * k]), ld_f(c[2 * k + 1])));
    T* d = gi + row * W + q * Q;
    if constexpr (Q * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(o);
    } else if constexpr (Q * sizeof(T) == 8) {
      *reinterpret_cast<uint2*>(d) = *reinterpret_cast<const uint2*>(o);
    } else {
#pragma unroll
      for (int k = 0; k < Q; ++k) d[k] = o[k];
    }
  }
}

// NHWC: one thread per input pixel and V consecutive channels (V*sizeof(T) =
// 16 bytes, or V = 1).  `C` channels per pixel.
template <typename T, int V>
__global__ void __launch_bounds__(kLayoutThreads) up2x_bwd_nhwc_kernel(const T* __restrict__ go, T* __restrict__ gi,
                                                                       long long N, long long H, long long W,
                                                                       long long C) {
  const long long cv = C / V;
  const long long total = N * H * W * cv;
  for (long long u = (long long)blockIdx.x * kLayoutThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kLayoutThreads) {
    const long long pix = u / cv, k = (u - pix * cv) * V;
    const long long x = pix % W, y = (pix / W) % H, b = pix / (H * W);
    const long long p00 = ((b * 2 * H + 2 * y) * 2 * W + 2 * x) * C + k;
    const long long p01 = p00 + C, p10 = p00 + 2 * W * C, p11 = p10 + C;
    alignas(16) T g0[V];
    alignas(16) T g1[V];
    alignas(16) T g2[V];
    alignas(16) T g3[V];
    alignas(16) T o[V];
    if constexpr (V * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(g0) = *reinterpret_cast<const uint4*>(go + p00);
      *reinterpret_cast<uint4*>(g1) = *reinterpret_cast<const uint4*>(go + p01);
      *reinterpret_cast<uint4*>(g2) = *reinterpret_cast<const uint4*>(go + p10);
      *reinterpret_cast<uint4*>(g3) = *reinterpret_cast<const uint4*>(go + p11);
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) {
        g0[e] = go[p00 + e];
        g1[e] = go[p01 + e];
        g2[e] = go[p10 + e];
        g3[e] = go[p11 + e];
      }
    }
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = st_f<T>(sum4(ld_f(g0[e]), ld_f(g1[e]), ld_f(g2[e]), ld_f(g3[e])));
    T* d = gi + pix * C + k;
    if constexpr (V * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(o);
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) d[e] = o[e];
    }
  }
}

int current_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  return sm_count(dev);
}

b2_status check_up_args(int dtype, int layout, int64_t N, int64_t C, int64_t H, int64_t W, const char* who) {
  if (dtype != B2_BF16 && dtype != B2_F32) return set_error(B2_ERR_UNSUPPORTED, "%s: dtype must be bf16 or f32", who);
  if (layout != 0 && layout != 1) return set_error(B2_ERR_INVALID, "%s: layout must be 0 (NCHW) or 1 (NHWC)", who);
  if (N < 0 || C < 0 || H < 0 || W < 0) return set_error(B2_ERR_INVALID, "%s: negative size", who);
  return B2_OK;
}

template <typename T>
b2_status up2x_fwd(const T* in, T* out, int layout, long long N, long long C, long long H, long long W,
                   cudaStream_t st) {
  const int sms = current_sms();
  if (layout == 0) {
    const long long rows = N * C * H;
    if (W % 4 == 0 && aligned(in, 4 * sizeof(T)) && aligned(out, 16)) {
      up2x_nchw_kernel<T, 4><<<layout_grid(rows * (W / 4), sms), kLayoutThreads, 0, st>>>(in, out, rows, W);
    } else {
      up2x_nchw_kernel<T, 1><<<layout_grid(rows * W, sms), kLayoutThreads, 0, st>>>(in, out, rows, W);
    }
  } else {
    const long long bytes = C * (long long)sizeof(T);
    if (bytes % 16 == 0 && aligned(in, 16) && aligned(out, 16)) {
      up2x_nhwc_kernel<uint4><<<layout_grid(N * 4 * H * W * (bytes / 16), sms), kLayoutThreads, 0, st>>>(
          reinterpret_cast<const uint4*>(in), reinterpret_cast<uint4*>(out), N, H, W, bytes / 16);
    } else {
      up2x_nhwc_kernel<T><<<layout_grid(N * 4 * H * W * C, sms), kLayoutThreads, 0, st>>>(in, out, N, H, W, C);
    }
  }
  return check_cuda(cudaGetLastError(), "upsample_nearest2x launch");
}

template <typename T>
b2_status up2x_bwd(const T* go, T* gi, int layout, long long N, long long C, long long H, long long W,
                   cudaStream_t st) {
  const int sms = current_sms();
  constexpr int kVec = 16 / sizeof(T);
  if (layout == 0) {
    const long long rows = N * C * H;
    if (W % 4 == 0 && aligned(go, 16) && aligned(gi, 4 * sizeof(T))) {
      up2x_bwd_nchw_kernel<T, 4><<<layout_grid(rows * (W / 4), sms), kLayoutThreads, 0, st>>>(go, gi, rows, W);
    } else {
      up2x_bwd_nchw_kernel<T, 1><<<layout_grid(rows * W, sms), kLayoutThreads, 0, st>>>(go, gi, rows, W);
    }
  } else {
    if (C % kVec == 0 && aligned(go, 16) && aligned(gi, 16)) {
      up2x_bwd_nhwc_kernel<T, kVec><<<layout_grid(N * H * W * (C / kVec), sms), kLayoutThreads, 0, st>>>(
          go, gi, N, H, W, C);
    } else {
      up2x_bwd_nhwc_kernel<T, 1><<<layout_grid(N * H * W * C, sms), kLayoutThreads, 0, st>>>(go, gi, N, H, W, C);
    }
  }
  return check_cuda(cudaGetLastError(), "upsample_nearest2x_backward launch");
}

template <typename U>
b2_status cat_launch(const CatBatch& b, int n, char* dst, long long outer, long long out_block_bytes,
                     long long max_units, int sms, cudaStream_t st) {
  const int gx = std::max(1, std::min(layout_grid(outer * max_units, sms), std::max(1, sms * 16 / n)));
  cat_kernel<U><<<dim3(gx, n), kLayoutThreads, 0, st>>>(b, reinterpret_cast<U*>(dst), outer,
                                                         out_block_bytes / (long long)sizeof(U));
  return check_cuda(cudaGetLastError(), "cat launch");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

b2_status b2_cat_blocks(const void* const* srcs, const int64_t* block_bytes, int n, void* dst, int64_t outer,
                        int64_t out_block_bytes, void* stream) {
  if (n < 0 || outer < 0 || out_block_bytes < 0 || (n > 0 && (!srcs || !block_bytes)))
    return set_error(B2_ERR_INVALID, "b2_cat_blocks: bad arguments");
  long long sum = 0;
  for (int i = 0; i < n; ++i) {
    if (block_bytes[i] < 0) return set_error(B2_ERR_INVALID, "b2_cat_blocks: negative block");
    if (block_bytes[i] > 0 && outer > 0 && !srcs[i]) return set_error(B2_ERR_INVALID, "b2_cat_blocks: null source");
    sum += block_bytes[i];
  }
  if (sum != out_block_bytes) return set_error(B2_ERR_INVALID, "b2_cat_blocks: blocks do not add up to the output block");
  if (outer == 0 || out_block_bytes == 0) return B2_OK;
  if (!dst) return set_error(B2_ERR_INVALID, "b2_cat_blocks: null destination");
  auto st = static_cast<cudaStream_t>(stream);
  const int sms = current_sms();
  // widest unit that divides every block, offset and address
  int unit = 16;
  auto fits = [&](int u) {
    if (out_block_bytes % u || !aligned(dst, u)) return false;
    for (int i = 0; i < n; ++i)
      if (block_bytes[i] % u || (block_bytes[i] && !aligned(srcs[i], u))) return false;
    return true;
  };
  while (unit > 1 && !fits(unit)) unit /= 2;
  long long off = 0;
  for (int first = 0; first < n; first += kMaxCat) {
    CatBatch b{};
    int m = 0;
    long long max_units = 1;
    for (int i = first; i < std::min(n, first + kMaxCat); ++i) {
      if (block_bytes[i] == 0) continue;  // nothing to copy; offset unchanged
      b.src[m] = static_cast<const char*>(srcs[i]);
      b.block[m] = block_bytes[i] / unit;
      b.off[m] = off / unit;
      max_units = std::max<long long>(max_units, b.block[m]);
      off += block_bytes[i];
      ++m;
    }
    if (m == 0) continue;
    char* d = static_cast<char*>(dst);
    b2_status s;
    switch (unit) {
      case 16: s = cat_launch<uint4>(b, m, d, outer, out_block_bytes, max_units, sms, st); break;
      case 8: s = cat_launch<uint2>(b, m, d, outer, out_block_bytes, max_units, sms, st); break;
      case 4: s = cat_launch<uint32_t>(b, m, d, outer, out_block_bytes, max_units, sms, st); break;
      case 2: s = cat_launch<uint16_t>(b, m, d, outer, out_block_bytes, max_units, sms, st); break;
      default: s = cat_launch<uint8_t>(b, m, d, outer, out_block_bytes, max_units, sms, st); break;
    }
    if (s != B2_OK) return s;
  }
  return B2_OK;
}

b2_status b2_upsample_nearest2x(const void* in, void* out, int dtype, int layout, int64_t N, int64_t C, int64_t H,
                                int64_t W, void* stream) {
  B2_TRY(check_up_args(dtype, layout, N, C, H, W, "b2_upsample_nearest2x"));
  if (N * C * H * W == 0) return B2_OK;
  if (!in || !out) return set_error(B2_ERR_INVALID, "b2_upsample_nearest2x: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == B2_BF16)
    return up2x_fwd(static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), layout, N, C, H, W, st);
  return up2x_fwd(static_cast<const float*>(in), static_cast<float*>(out), layout, N, C, H, W, st);
}

b2_status b2_upsample_nearest2x_backward(const void* go, void* gi, int dtype, int layout, int64_t N, int64_t C,
                                         int64_t H, int64_t W, void* stream) {
  B2_TRY(check_up_args(dtype, layout, N, C, H, W, "b2_upsample_nearest2x_backward"));
  if (N * C * H * W == 0) return B2_OK;
  if (!go || !gi) return set_error(B2_ERR_INVALID, "b2_upsample_nearest2x_backward: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == B2_BF16)
    return up2x_bwd(static_cast<const uint16_t*>(go), static_cast<uint16_t*>(gi), layout, N, C, H, W, st);
  return up2x_bwd(static_cast<const float*>(go), static_cast<float*>(gi), layout, N, C, H, W, st);
}

}  // extern "C"
