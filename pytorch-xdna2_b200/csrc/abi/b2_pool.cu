// 2-D max pooling with indices (forward) and its backward, bf16 / fp32, any
// kernel, stride, padding, dilation and ceil mode.  Same results as ATen
// (the reference runs these on its CPU path):
//
//   forward   the window is scanned in (kh, kw) order; a value replaces the
//             running maximum when it is greater or NaN (so the last NaN
//             wins), starting from -inf at the window's first valid position;
//             the index is h*W + w within the plane (int64).
//   backward  a gather: every input element adds, in (oh, ow) order, the
//             gradients of the outputs whose saved index is its own, in fp32,
//             and is rounded once -- no atomics, deterministic.
//
// Channels-last bf16 with C % 8 == 0 moves 16-byte channel vectors; every
// other layout goes through element strides.  HBM-bound.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kPoolThreads = 256;

struct PoolGeom {
  long long N, C, H, W, OH, OW;
  int kh, kw, sh, sw, ph, pw, dh, dw;
  // element strides of x (and dx) and of y / indices / dy
  long long xs[4], ys[4];
};

int pool_grid(long long units, int sms) {
  const long long b = (units + kPoolThreads - 1) / kPoolThreads;
  return int(std::max<long long>(1, std::min<long long>(b, (long long)sms * 16)));
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p, long long i) {
  if constexpr (sizeof(T) == 2) return bf2f(reinterpret_cast<const uint16_t*>(p)[i]);
  else return p[i];
}
template <typename T>
__device__ __forceinline__ void stf(T* p, long long i, float v) {
  if constexpr (sizeof(T) == 2) reinterpret_cast<uint16_t*>(p)[i] = f2bf(v);
  else p[i] = v;
}

// first valid tap of a window start (may be negative) and its end (exclusive)
template <typename I>
__device__ __forceinline__ void window(I o, int s, int p, int k, int d, I n, I& beg, I& end) {
  beg = o * s - p;
  end = min(beg + I(k - 1) * d + 1, n);
  while (beg < 0) beg += d;
}

// output positions whose window can cover input position i: [lo, hi)
template <typename I>
__device__ __forceinline__ void covering(I i, int s, int p, int k, int d, I on, I& lo, I& hi) {
  const I span = I(k - 1) * d + 1;
  lo = (i + p < span) ? 0 : (i + p - span) / s + 1;
  hi = min((i + p) / s + 1, on);
}

// Element-strided kernels, index type I: int when every offset fits (the
// divisions that unflatten the thread index are then 32-bit, several times
// cheaper than 64-bit ones), else long long.
template <typename T, typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_fwd_kernel(const T* __restrict__ x, PoolGeom g,
                                                                   T* __restrict__ y, int64_t* __restrict__ ind) {
  const I OW = I(g.OW), OH = I(g.OH), C = I(g.C), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * C * OH * OW;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    I r = u / OW;
    const I ow = u - r * OW;
    I r2 = r / OH;
    const I oh = r - r2 * OH;
    const I n = r2 / C, c = r2 - n * C;
    I h0, h1, w0, w1;
    window<I>(oh, g.sh, g.ph, g.kh, g.dh, H, h0, h1);
    window<I>(ow, g.sw, g.pw, g.kw, g.dw, W, w0, w1);
    const T* xp = x + n * I(g.xs[0]) + c * I(g.xs[1]);
    float best = -INFINITY;
    I bi = h0 * W + w0;
    for (I h = h0; h < h1; h += g.dh)
      for (I w = w0; w < w1; w += g.dw) {
        const float v = ldf(xp, h * I(g.xs[2]) + w * I(g.xs[3]));
        if (v > best || v != v) {
          best = v;
          bi = h * W + w;
        }
      }
    const I o = n * I(g.ys[0]) + c * I(g.ys[1]) + oh * I(g.ys[2]) + ow * I(g.ys[3]);
    stf(y, o, best);
    ind[o] = bi;
  }
}

// channels-last bf16, 8 channels per thread (C % 8 == 0, 16-byte aligned);
// index type I as for the element-strided kernels
template <typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_fwd_nhwc8_kernel(const uint16_t* __restrict__ x, PoolGeom g,
                                                                         uint16_t* __restrict__ y,
                                                                         int64_t* __restrict__ ind) {
  const I cv = I(g.C / 8), OW = I(g.OW), OH = I(g.OH), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * OH * OW * cv;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    const I r = u / cv, q = u - r * cv;
    const I r2 = r / OW, ow = r - r2 * OW;
    const I n = r2 / OH, oh = r2 - n * OH;
    I h0, h1, w0, w1;
    window<I>(oh, g.sh, g.ph, g.kh, g.dh, H, h0, h1);
    window<I>(ow, g.sw, g.pw, g.kw, g.dw, W, w0, w1);
    float best[8];
    long long bi[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      best[e] = -INFINITY;
      bi[e] = (long long)(h0 * W + w0);
    }
    const uint16_t* xp = x + n * I(g.xs[0]) + q * 8;
    for (I h = h0; h < h1; h += g.dh)
      for (I w = w0; w < w1; w += g.dw) {
        const uint4 v4 = *reinterpret_cast<const uint4*>(xp + h * I(g.xs[2]) + w * I(g.xs[3]));
        const uint32_t wd[4] = {v4.x, v4.y, v4.z, v4.w};
        const long long idx = (long long)(h * W + w);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float v = __uint_as_float((e & 1) ? (wd[e >> 1] & 0xffff0000u) : (wd[e >> 1] << 16));
          if (v > best[e] || v != v) {
            best[e] = v;
            bi[e] = idx;
          }
        }
      }
    const I o = n * I(g.ys[0]) + oh * I(g.ys[2]) + ow * I(g.ys[3]) + q * 8;
    uint4 out;
    out.x = pack_bf2(best[0], best[1]);
    out.y = pack_bf2(best[2], best[3]);
    out.z = pack_bf2(best[4], best[5]);
    out.w = pack_bf2(best[6], best[7]);
    *reinterpret_cast<uint4*>(y + o) = out;
    longlong2* ip = reinterpret_cast<longlong2*>(ind + o);
#pragma unroll
    for (int e = 0; e < 4; ++e) ip[e] = make_longlong2(bi[2 * e], bi[2 * e + 1]);
  }
}

// As maxpool_fwd_nhwc8_kernel for 3x3 windows (ResNet's stem pool): the up to
// nine window loads are all issued before the scan, which then visits the
// valid taps in the same (h, w) order -- the same maxima and indices.
//
// TAPS: instead of int64 indices, one byte per output element -- the argmax's
// position inside its window, i * kw + j for tap (hs + i*dh, ws + j*dw) of the
// window that starts at (hs, ws) = (oh*sh - ph, ow*sw - pw).  ATen's int64
// indices follow from it (maxpool_taps_to_indices_kernel), and the backward
// reads 1 byte per element instead of 8.
template <typename I, bool TAPS = false>
__global__ void __launch_bounds__(kPoolThreads) maxpool_fwd_nhwc8_k3_kernel(const uint16_t* __restrict__ x,
                                                                            PoolGeom g, uint16_t* __restrict__ y,
                                                                            int64_t* __restrict__ ind,
                                                                            uint8_t* __restrict__ taps = nullptr) {
  const I cv = I(g.C / 8), OW = I(g.OW), OH = I(g.OH), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * OH * OW * cv;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    const I r = u / cv, q = u - r * cv;
    const I r2 = r / OW, ow = r - r2 * OW;
    const I n = r2 / OH, oh = r2 - n * OH;
    I h0, h1, w0, w1;
    window<I>(oh, g.sh, g.ph, 3, g.dh, H, h0, h1);
    window<I>(ow, g.sw, g.pw, 3, g.dw, W, w0, w1);
    const uint16_t* xp = x + n * I(g.xs[0]) + q * 8;
    uint4 v[9];
    bool ok[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const I h = h0 + I(t / 3) * g.dh, w = w0 + I(t % 3) * g.dw;
      ok[t] = h < h1 && w < w1;
      v[t] = ok[t] ? __ldg(reinterpret_cast<const uint4*>(xp + h * I(g.xs[2]) + w * I(g.xs[3])))
                   : make_uint4(0, 0, 0, 0);
    }
    // window-relative position of the first valid tap (h0, w0)
    const int i0 = int((h0 - (oh * g.sh - g.ph)) / g.dh), j0 = int((w0 - (ow * g.sw - g.pw)) / g.dw);
    float best[8];
    long long bi[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      best[e] = -INFINITY;
      bi[e] = TAPS ? (long long)(i0 * 3 + j0) : (long long)(h0 * W + w0);
    }
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      if (!ok[t]) continue;
      const long long idx = TAPS ? (long long)((i0 + t / 3) * 3 + j0 + t % 3)
                                 : (long long)((h0 + I(t / 3) * g.dh) * W + w0 + I(t % 3) * g.dw);
      const uint32_t wd[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = __uint_as_float((e & 1) ? (wd[e >> 1] & 0xffff0000u) : (wd[e >> 1] << 16));
        if (f > best[e] || f != f) {
          best[e] = f;
          bi[e] = idx;
        }
      }
    }
    const I o = n * I(g.ys[0]) + oh * I(g.ys[2]) + ow * I(g.ys[3]) + q * 8;
    uint4 out;
    out.x = pack_bf2(best[0], best[1]);
    out.y = pack_bf2(best[2], best[3]);
    out.z = pack_bf2(best[4], best[5]);
    out.w = pack_bf2(best[6], best[7]);
    *reinterpret_cast<uint4*>(y + o) = out;
    if constexpr (TAPS) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        lo |= uint32_t(bi[e]) << (8 * e);
        hi |= uint32_t(bi[4 + e]) << (8 * e);
      }
      *reinterpret_cast<uint2*>(taps + o) = make_uint2(lo, hi);
    } else {
      longlong2* ip = reinterpret_cast<longlong2*>(ind + o);
#pragma unroll
      for (int e = 0; e < 4; ++e) ip[e] = make_longlong2(bi[2 * e], bi[2 * e + 1]);
    }
  }
}

// The taps forward for ResNet's stem pool (3x3 windows, stride 2, padding 1,
// no dilation): a CTA row per output row (b, oh) (grid.y), threads over its
// (ow, channel group) units, window bounds from shifts -- the same scan, the
// same maxima and taps as maxpool_fwd_nhwc8_k3_kernel<.., true>.
__global__ void __launch_bounds__(kPoolThreads) maxpool_fwd_s2k3_taps_kernel(const uint16_t* __restrict__ x,
                                                                             PoolGeom g, int cv_shift,
                                                                             uint16_t* __restrict__ y,
                                                                             uint8_t* __restrict__ taps) {
  const int H = int(g.H), W = int(g.W), OH = int(g.OH), OW = int(g.OW);
  const int row = blockIdx.y, n = row / OH, oh = row - n * OH;
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  const int ow = u >> cv_shift, q = u & ((1 << cv_shift) - 1);
  if (ow >= OW) return;
  const int hs = 2 * oh - 1, ws = 2 * ow - 1;  // window start (may be -1)
  const uint16_t* xp = x + (long long)n * g.xs[0] + q * 8;
  uint4 v[9];
  bool ok[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) {
    const int h = hs + t / 3, w = ws + t % 3;
    ok[t] = h >= 0 && h < H && w >= 0 && w < W;
    v[t] = ok[t] ? __ldg(reinterpret_cast<const uint4*>(xp + (long long)h * g.xs[2] + (long long)w * g.xs[3]))
                 : make_uint4(0, 0, 0, 0);
  }
  // the first valid tap (the general kernel's starting index)
  const int i0 = hs < 0 ? 1 : 0, j0 = ws < 0 ? 1 : 0;
  float best[8];
  int bt[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    best[e] = -INFINITY;
    bt[e] = i0 * 3 + j0;
  }
#pragma unroll
  for (int t = 0; t < 9; ++t) {
    if (!ok[t]) continue;
    const uint32_t wd[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = __uint_as_float((e & 1) ? (wd[e >> 1] & 0xffff0000u) : (wd[e >> 1] << 16));
      if (f > best[e] || f != f) {
        best[e] = f;
        bt[e] = t;
      }
    }
  }
  const long long o = (long long)n * g.ys[0] + (long long)oh * g.ys[2] + (long long)ow * g.ys[3] + q * 8;
  uint4 out;
  out.x = pack_bf2(best[0], best[1]);
  out.y = pack_bf2(best[2], best[3]);
  out.z = pack_bf2(best[4], best[5]);
  out.w = pack_bf2(best[6], best[7]);
  *reinterpret_cast<uint4*>(y + o) = out;
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    lo |= uint32_t(bt[e]) << (8 * e);
    hi |= uint32_t(bt[4 + e]) << (8 * e);
  }
  *reinterpret_cast<uint2*>(taps + o) = make_uint2(lo, hi);
}

// ATen's int64 indices (h*W + w within the plane) from the window taps.
template <typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_taps_to_indices_kernel(const uint8_t* __restrict__ taps,
                                                                               PoolGeom g,
                                                                               int64_t* __restrict__ ind) {
  const I cv = I(g.C / 8), OW = I(g.OW), OH = I(g.OH), W = I(g.W);
  const I total = I(g.N) * OH * OW * cv;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    const I r = u / cv, q = u - r * cv;
    const I r2 = r / OW, ow = r - r2 * OW;
    const I n = r2 / OH, oh = r2 - n * OH;
    const I o = n * I(g.ys[0]) + oh * I(g.ys[2]) + ow * I(g.ys[3]) + q * 8;
    const uint2 tv = *reinterpret_cast<const uint2*>(taps + o);
    const long long hs = (long long)oh * g.sh - g.ph, ws = (long long)ow * g.sw - g.pw;
    long long idx[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int t = int(((e < 4 ? tv.x : tv.y) >> (8 * (e & 3))) & 0xffu);
      idx[e] = (hs + (long long)(t / g.kw) * g.dh) * (long long)W + ws + (long long)(t % g.kw) * g.dw;
    }
    longlong2* ip = reinterpret_cast<longlong2*>(ind + o);
#pragma unroll
    for (int e = 0; e < 4; ++e) ip[e] = make_longlong2(idx[2 * e], idx[2 * e + 1]);
  }
}

template <typename T, typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_bwd_kernel(const T* __restrict__ dy,
                                                                   const int64_t* __restrict__ ind, PoolGeom g,
                                                                   T* __restrict__ dx) {
  const I OW = I(g.OW), OH = I(g.OH), C = I(g.C), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * C * H * W;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    I r = u / W;
    const I w = u - r * W;
    I r2 = r / H;
    const I h = r - r2 * H;
    const I n = r2 / C, c = r2 - n * C;
    I oh0, oh1, ow0, ow1;
    covering<I>(h, g.sh, g.ph, g.kh, g.dh, OH, oh0, oh1);
    covering<I>(w, g.sw, g.pw, g.kw, g.dw, OW, ow0, ow1);
    const long long me = (long long)h * W + w;
    const I base = n * I(g.ys[0]) + c * I(g.ys[1]);
    float s = 0.0f;
    for (I oh = oh0; oh < oh1; ++oh)
      for (I ow = ow0; ow < ow1; ++ow) {
        const I o = base + oh * I(g.ys[2]) + ow * I(g.ys[3]);
        if (ind[o] == me) s = __fadd_rn(s, ldf(dy, o));
      }
    stf(dx, n * I(g.xs[0]) + c * I(g.xs[1]) + h * I(g.xs[2]) + w * I(g.xs[3]), s);
  }
}

template <typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_bwd_nhwc8_kernel(const uint16_t* __restrict__ dy,
                                                                         const int64_t* __restrict__ ind,
                                                                         PoolGeom g, uint16_t* __restrict__ dx) {
  const I cv = I(g.C / 8), OW = I(g.OW), OH = I(g.OH), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * H * W * cv;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    const I r = u / cv, q = u - r * cv;
    const I r2 = r / W, w = r - r2 * W;
    const I n = r2 / H, h = r2 - n * H;
    I oh0, oh1, ow0, ow1;
    covering<I>(h, g.sh, g.ph, g.kh, g.dh, OH, oh0, oh1);
    covering<I>(w, g.sw, g.pw, g.kw, g.dw, OW, ow0, ow1);
    const long long me = (long long)(h * W + w);
    float s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] = 0.0f;
    for (I oh = oh0; oh < oh1; ++oh)
      for (I ow = ow0; ow < ow1; ++ow) {
        const I o = n * I(g.ys[0]) + oh * I(g.ys[2]) + ow * I(g.ys[3]) + q * 8;
        const uint4 v4 = *reinterpret_cast<const uint4*>(dy + o);
        const uint32_t wd[4] = {v4.x, v4.y, v4.z, v4.w};
        const longlong2* ip = reinterpret_cast<const longlong2*>(ind + o);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const longlong2 ii = ip[e2];
          if (ii.x == me) s[2 * e2] = __fadd_rn(s[2 * e2], __uint_as_float(wd[e2] << 16));
          if (ii.y == me) s[2 * e2 + 1] = __fadd_rn(s[2 * e2 + 1], __uint_as_float(wd[e2] & 0xffff0000u));
        }
      }
    uint4 out;
    out.x = pack_bf2(s[0], s[1]);
    out.y = pack_bf2(s[2], s[3]);
    out.z = pack_bf2(s[4], s[5]);
    out.w = pack_bf2(s[6], s[7]);
    *reinterpret_cast<uint4*>(dx + n * I(g.xs[0]) + h * I(g.xs[2]) + w * I(g.xs[3]) + q * 8) = out;
  }
}

// As maxpool_bwd_nhwc8_kernel when every input position is covered by at
// most two outputs per dimension (window span <= 2 * stride: ResNet's 3x3 /
// stride 2 pool): the up to four covering outputs' gradients and indices are
// all loaded before any is compared -- four independent 80-byte loads in
// flight per thread instead of a dependent chain -- then added in the same
// (oh, ow) order, so the results are those of the general kernel.
template <typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_bwd_nhwc8_two_kernel(const uint16_t* __restrict__ dy,
                                                                             const int64_t* __restrict__ ind,
                                                                             PoolGeom g, uint16_t* __restrict__ dx) {
  const I cv = I(g.C / 8), OW = I(g.OW), OH = I(g.OH), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * H * W * cv;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    const I r = u / cv, q = u - r * cv;
    const I r2 = r / W, w = r - r2 * W;
    const I n = r2 / H, h = r2 - n * H;
    I oh0, oh1, ow0, ow1;
    covering<I>(h, g.sh, g.ph, g.kh, g.dh, OH, oh0, oh1);
    covering<I>(w, g.sw, g.pw, g.kw, g.dw, OW, ow0, ow1);
    const long long me = (long long)(h * W + w);
    uint4 v[4];
    longlong2 ii[4][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const I oh = oh0 + (t >> 1), ow = ow0 + (t & 1);
      if (oh < oh1 && ow < ow1) {
        const I o = n * I(g.ys[0]) + oh * I(g.ys[2]) + ow * I(g.ys[3]) + q * 8;
        v[t] = __ldg(reinterpret_cast<const uint4*>(dy + o));
        const longlong2* ip = reinterpret_cast<const longlong2*>(ind + o);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) ii[t][e2] = __ldg(ip + e2);
      } else {
        v[t] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) ii[t][e2] = make_longlong2(-1, -1);  // never an input position
      }
    }
    float s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t wd[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        if (ii[t][e2].x == me) s[2 * e2] = __fadd_rn(s[2 * e2], __uint_as_float(wd[e2] << 16));
        if (ii[t][e2].y == me) s[2 * e2 + 1] = __fadd_rn(s[2 * e2 + 1], __uint_as_float(wd[e2] & 0xffff0000u));
      }
    }
    uint4 out;
    out.x = pack_bf2(s[0], s[1]);
    out.y = pack_bf2(s[2], s[3]);
    out.z = pack_bf2(s[4], s[5]);
    out.w = pack_bf2(s[6], s[7]);
    *reinterpret_cast<uint4*>(dx + n * I(g.xs[0]) + h * I(g.xs[2]) + w * I(g.xs[3]) + q * 8) = out;
  }
}

// maxpool_bwd_nhwc8_two_kernel reading the forward's window taps (1 byte per
// element) instead of int64 indices: input (h, w) matches output (oh, ow)'s
// tap when it is that window's tap ((h - hs) / dh) * kw + (w - ws) / dw.
template <typename I>
__global__ void __launch_bounds__(kPoolThreads) maxpool_bwd_nhwc8_taps_kernel(const uint16_t* __restrict__ dy,
                                                                              const uint8_t* __restrict__ taps,
                                                                              PoolGeom g, uint16_t* __restrict__ dx) {
  const I cv = I(g.C / 8), OW = I(g.OW), OH = I(g.OH), H = I(g.H), W = I(g.W);
  const I total = I(g.N) * H * W * cv;
  for (I u = I(blockIdx.x) * kPoolThreads + I(threadIdx.x); u < total; u += I(gridDim.x) * kPoolThreads) {
    const I r = u / cv, q = u - r * cv;
    const I r2 = r / W, w = r - r2 * W;
    const I n = r2 / H, h = r2 - n * H;
    I oh0, oh1, ow0, ow1;
    covering<I>(h, g.sh, g.ph, g.kh, g.dh, OH, oh0, oh1);
    covering<I>(w, g.sw, g.pw, g.kw, g.dw, OW, ow0, ow1);
    uint4 v[4];
    uint2 tv[4];
    uint32_t want[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const I oh = oh0 + (t >> 1), ow = ow0 + (t & 1);
      want[t] = 0xffffffffu;  // matches no tap byte
      if (oh < oh1 && ow < ow1) {
        const I o = n * I(g.ys[0]) + oh * I(g.ys[2]) + ow * I(g.ys[3]) + q * 8;
        v[t] = __ldg(reinterpret_cast<const uint4*>(dy + o));
        tv[t] = __ldg(reinterpret_cast<const uint2*>(taps + o));
        const I di = h - (oh * g.sh - g.ph), dj = w - (ow * g.sw - g.pw);
        if (di % g.dh == 0 && dj % g.dw == 0) want[t] = uint32_t((di / g.dh) * g.kw + dj / g.dw);
      } else {
        v[t] = make_uint4(0, 0, 0, 0);
        tv[t] = make_uint2(0, 0);
      }
    }
    float s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t wd[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t tap = ((e < 4 ? tv[t].x : tv[t].y) >> (8 * (e & 3))) & 0xffu;
        if (tap == want[t])
          s[e] = __fadd_rn(s[e], __uint_as_float((e & 1) ? (wd[e >> 1] & 0xffff0000u) : (wd[e >> 1] << 16)));
      }
    }
    uint4 out;
    out.x = pack_bf2(s[0], s[1]);
    out.y = pack_bf2(s[2], s[3]);
    out.z = pack_bf2(s[4], s[5]);
    out.w = pack_bf2(s[6], s[7]);
    *reinterpret_cast<uint4*>(dx + n * I(g.xs[0]) + h * I(g.xs[2]) + w * I(g.xs[3]) + q * 8) = out;
  }
}

// maxpool_bwd_nhwc8_taps_kernel for ResNet's stem pool (3x3 windows, stride
// 2, padding 1, no dilation; 2*OH >= H and 2*OW >= W).  A thread per output
// window (b, oh, ow, channel group) owns the 2x2 input block (2oh + a,
// 2ow + b), a, b in {0, 1}: the windows covering those inputs are (oh, ow),
// (oh, ow + 1), (oh + 1, ow) and (oh + 1, ow + 1), so four dy/taps reads make
// four dx groups (the per-input form reads 2.25 windows per input).  Window
// (oh, ow) sends taps 4/5/7/8 to (0,0)/(0,1)/(1,0)/(1,1); (oh, ow + 1) taps 3/6
// to (0,1)/(1,1); (oh + 1, ow) taps 1/2 to (1,0)/(1,1); (oh + 1, ow + 1) tap 0
// to (1,1).  Each input's adds run in the same (oh, ow) order from 0.0f as
// the general kernel's -- the same sums.  CTA row (grid.y) = (b, oh).
__global__ void __launch_bounds__(512) maxpool_bwd_s2k3_quad_kernel(const uint16_t* __restrict__ dy,
                                                                    const uint8_t* __restrict__ taps, PoolGeom g,
                                                                    int cv_shift, uint16_t* __restrict__ dx) {
  const int H = int(g.H), W = int(g.W), OH = int(g.OH), OW = int(g.OW);
  const int row = blockIdx.y, n = row / OH, oh = row - n * OH;
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  const int ow = u >> cv_shift, q = u & ((1 << cv_shift) - 1);
  if (ow >= OW) return;
  const uint16_t* dyn = dy + (long long)n * g.ys[0] + q * 8;
  const uint8_t* tn = taps + (long long)n * g.ys[0] + q * 8;
  uint4 v[4];
  uint2 tv[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int wh = oh + (t >> 1), ww = ow + (t & 1);
    if (wh < OH && ww < OW) {
      const long long o = (long long)wh * g.ys[2] + (long long)ww * g.ys[3];
      v[t] = __ldg(reinterpret_cast<const uint4*>(dyn + o));
      tv[t] = __ldg(reinterpret_cast<const uint2*>(tn + o));
    } else {
      v[t] = make_uint4(0, 0, 0, 0);
      tv[t] = make_uint2(0xffffffffu, 0xffffffffu);  // no tap matches 255
    }
  }
  float s[4][8];  // [a * 2 + b][channel]
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) s[k][e] = 0.0f;
  // tap -> owned input (a * 2 + b) for each window, -1 where the tap lies outside the block
  constexpr int kDst[4][9] = {{-1, -1, -1, -1, 0, 1, -1, 2, 3},
                              {-1, -1, -1, 1, -1, -1, 3, -1, -1},
                              {-1, 2, 3, -1, -1, -1, -1, -1, -1},
                              {3, -1, -1, -1, -1, -1, -1, -1, -1}};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t wd[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t tap = ((e < 4 ? tv[t].x : tv[t].y) >> (8 * (e & 3))) & 0xffu;
      const float f = __uint_as_float((e & 1) ? (wd[e >> 1] & 0xffff0000u) : (wd[e >> 1] << 16));
#pragma unroll
      for (int k = 0; k < 9; ++k)
        if (kDst[t][k] >= 0 && tap == uint32_t(k)) s[kDst[t][k]][e] = __fadd_rn(s[kDst[t][k]][e], f);
    }
  }
  uint16_t* dxn = dx + (long long)n * g.xs[0] + q * 8;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int h = 2 * oh + (k >> 1), w = 2 * ow + (k & 1);
    if (h >= H || w >= W) continue;
    uint4 out;
    out.x = pack_bf2(s[k][0], s[k][1]);
    out.y = pack_bf2(s[k][2], s[k][3]);
    out.z = pack_bf2(s[k][4], s[k][5]);
    out.w = pack_bf2(s[k][6], s[k][7]);
    *reinterpret_cast<uint4*>(dxn + (long long)h * g.xs[2] + (long long)w * g.xs[3]) = out;
  }
}

// Threads per CTA for a row of `units` (channel group) units: the row rounded
// up to whole warps, at most 512 (no idle tail of a fixed 256-thread CTA).
inline int row_threads(long long units) { return int(std::min<long long>(512, (units + 31) / 32 * 32)); }

bool two_cover(const PoolGeom& g) {
  return (long long)(g.kh - 1) * g.dh + 1 <= 2LL * g.sh && (long long)(g.kw - 1) * g.dw + 1 <= 2LL * g.sw;
}

b2_status make_pool(PoolGeom& g, int64_t N, int64_t C, int64_t H, int64_t W, int64_t OH, int64_t OW, int kh, int kw,
                    int sh, int sw, int ph, int pw, int dh, int dw, const int64_t* xs, const int64_t* ys,
                    const char* who) {
  if (N < 0 || C < 0 || H <= 0 || W <= 0 || OH < 0 || OW < 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || ph < 0 ||
      pw < 0 || dh <= 0 || dw <= 0 || 2 * ph > kh || 2 * pw > kw || !xs || !ys)
    return set_error(B2_ERR_INVALID, "%s: bad geometry", who);
  g = PoolGeom{N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw, dh, dw, {xs[0], xs[1], xs[2], xs[3]},
               {ys[0], ys[1], ys[2], ys[3]}};
  return B2_OK;
}

// every element offset (of x and of y, and the thread index range) fits an int
bool fits32(const PoolGeom& g) {
  auto span = [](const long long* st, long long a, long long b, long long c, long long d) {
    return (a - 1) * std::llabs(st[0]) + (b - 1) * std::llabs(st[1]) + (c - 1) * std::llabs(st[2]) +
           (d - 1) * std::llabs(st[3]);
  };
  const long long lim = (1LL << 31) - (1LL << 26);  // headroom for the grid-stride step past the end
  return g.N * g.C * g.H * g.W < lim && g.N * g.C * g.OH * g.OW < lim && span(g.xs, g.N, g.C, g.H, g.W) < lim &&
         span(g.ys, g.N, g.C, g.OH, g.OW) < lim;
}

bool nhwc8(const PoolGeom& g, const void* a, const void* b, const void* c) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return g.C % 8 == 0 && g.xs[1] == 1 && g.ys[1] == 1 && g.xs[3] % 8 == 0 && g.xs[2] % 8 == 0 && g.xs[0] % 8 == 0 &&
         g.ys[3] % 8 == 0 && g.ys[2] % 8 == 0 && g.ys[0] % 8 == 0 && al(a) && al(b) && al(c);
}

int cur_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  return sm_count(dev);
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

b2_status b2_maxpool2d_fwd(const void* x, const int64_t* x_strides, void* y, int64_t* indices,
                           const int64_t* y_strides, int dtype, int64_t N, int64_t C, int64_t H, int64_t W,
                           int64_t OH, int64_t OW, int kh, int kw, int sh, int sw, int ph, int pw, int dh, int dw,
                           void* stream) {
  PoolGeom g;
  B2_TRY(make_pool(g, N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw, dh, dw, x_strides, y_strides, "b2_maxpool2d_fwd"));
  if (dtype != B2_BF16 && dtype != B2_F32) return set_error(B2_ERR_UNSUPPORTED, "b2_maxpool2d_fwd: dtype");
  const long long total = N * C * OH * OW;
  if (total == 0) return B2_OK;
  if (!x || !y || !indices) return set_error(B2_ERR_INVALID, "b2_maxpool2d_fwd: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  const int sms = cur_sms();
  if (dtype == B2_BF16 && nhwc8(g, x, y, indices) && fits32(g) && g.kh == 3 && g.kw == 3)
    maxpool_fwd_nhwc8_k3_kernel<int><<<pool_grid(total / 8, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(y), indices);
  else if (dtype == B2_BF16 && nhwc8(g, x, y, indices) && fits32(g))
    maxpool_fwd_nhwc8_kernel<int><<<pool_grid(total / 8, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(y), indices);
  else if (dtype == B2_BF16 && nhwc8(g, x, y, indices))
    maxpool_fwd_nhwc8_kernel<long long><<<pool_grid(total / 8, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(y), indices);
  else if (dtype == B2_BF16 && fits32(g))
    maxpool_fwd_kernel<uint16_t, int><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(y), indices);
  else if (dtype == B2_BF16)
    maxpool_fwd_kernel<uint16_t, long long><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(y), indices);
  else if (fits32(g))
    maxpool_fwd_kernel<float, int><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const float*>(x), g, static_cast<float*>(y), indices);
  else
    maxpool_fwd_kernel<float, long long><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const float*>(x), g, static_cast<float*>(y), indices);
  return check_cuda(cudaGetLastError(), "maxpool fwd launch");
}

b2_status b2_maxpool2d_bwd(const void* dy, const int64_t* indices, const int64_t* y_strides, void* dx,
                           const int64_t* x_strides, int dtype, int64_t N, int64_t C, int64_t H, int64_t W,
                           int64_t OH, int64_t OW, int kh, int kw, int sh, int sw, int ph, int pw, int dh, int dw,
                           void* stream) {
  PoolGeom g;
  B2_TRY(make_pool(g, N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw, dh, dw, x_strides, y_strides, "b2_maxpool2d_bwd"));
  if (dtype != B2_BF16 && dtype != B2_F32) return set_error(B2_ERR_UNSUPPORTED, "b2_maxpool2d_bwd: dtype");
  const long long total = N * C * H * W;
  if (total == 0) return B2_OK;
  if (!dx || (N * C * OH * OW > 0 && (!dy || !indices))) return set_error(B2_ERR_INVALID, "b2_maxpool2d_bwd: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  const int sms = cur_sms();
  if (dtype == B2_BF16 && nhwc8(g, dx, dy, indices) && fits32(g) && two_cover(g))
    maxpool_bwd_nhwc8_two_kernel<int><<<pool_grid(total / 8, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(dy), indices, g, static_cast<uint16_t*>(dx));
  else if (dtype == B2_BF16 && nhwc8(g, dx, dy, indices) && fits32(g))
    maxpool_bwd_nhwc8_kernel<int><<<pool_grid(total / 8, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(dy), indices, g, static_cast<uint16_t*>(dx));
  else if (dtype == B2_BF16 && nhwc8(g, dx, dy, indices))
    maxpool_bwd_nhwc8_kernel<long long><<<pool_grid(total / 8, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(dy), indices, g, static_cast<uint16_t*>(dx));
  else if (dtype == B2_BF16 && fits32(g))
    maxpool_bwd_kernel<uint16_t, int><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(dy), indices, g, static_cast<uint16_t*>(dx));
  else if (dtype == B2_BF16)
    maxpool_bwd_kernel<uint16_t, long long><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const uint16_t*>(dy), indices, g, static_cast<uint16_t*>(dx));
  else if (fits32(g))
    maxpool_bwd_kernel<float, int><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const float*>(dy), indices, g, static_cast<float*>(dx));
  else
    maxpool_bwd_kernel<float, long long><<<pool_grid(total, sms), kPoolThreads, 0, st>>>(
        static_cast<const float*>(dy), indices, g, static_cast<float*>(dx));
  return check_cuda(cudaGetLastError(), "maxpool bwd launch");
}

}  // extern "C"

// ---- max pooling with window taps (channels-last bf16, 3x3 windows) ---------

extern "C" b2_status b2_maxpool2d_fwd_taps(const void* x, const int64_t* x_strides, void* y, void* taps,
                                           const int64_t* y_strides, int64_t N, int64_t C, int64_t H, int64_t W,
                                           int64_t OH, int64_t OW, int kh, int kw, int sh, int sw, int ph, int pw,
                                           int dh, int dw, void* stream) {
  const char* who = "b2_maxpool2d_fwd_taps";
  PoolGeom g;
  B2_TRY(make_pool(g, N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw, dh, dw, x_strides, y_strides, who));
  const long long total = N * C * OH * OW;
  if (total == 0) return B2_OK;
  if (!x || !y || !taps) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  if (kh != 3 || kw != 3 || !nhwc8(g, x, y, y) || (reinterpret_cast<uintptr_t>(taps) & 7) || !fits32(g))
    return set_error(B2_ERR_UNSUPPORTED, "%s: needs 3x3 windows over channels-last bf16 (C %% 8 == 0)", who);
  const long long cv = C / 8;
  int cv_shift = 0;
  while ((1LL << cv_shift) < cv) ++cv_shift;
  if (sh == 2 && sw == 2 && ph == 1 && pw == 1 && dh == 1 && dw == 1 && (1LL << cv_shift) == cv &&
      OW * cv < (1LL << 30) && N * OH <= 65535) {
    const dim3 grid(unsigned((OW * cv + kPoolThreads - 1) / kPoolThreads), unsigned(N * OH));
    maxpool_fwd_s2k3_taps_kernel<<<grid, kPoolThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(x), g, cv_shift, static_cast<uint16_t*>(y), static_cast<uint8_t*>(taps));
    return check_cuda(cudaGetLastError(), "maxpool fwd taps launch");
  }
  maxpool_fwd_nhwc8_k3_kernel<int, true><<<pool_grid(total / 8, cur_sms()), kPoolThreads, 0,
                                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(y), nullptr, static_cast<uint8_t*>(taps));
  return check_cuda(cudaGetLastError(), "maxpool fwd taps launch");
}

extern "C" b2_status b2_maxpool2d_taps_to_indices(const void* taps, const int64_t* y_strides, int64_t* indices,
                                                  int64_t N, int64_t C, int64_t H, int64_t W, int64_t OH, int64_t OW,
                                                  int kh, int kw, int sh, int sw, int ph, int pw, int dh, int dw,
                                                  void* stream) {
  const char* who = "b2_maxpool2d_taps_to_indices";
  PoolGeom g;
  B2_TRY(make_pool(g, N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw, dh, dw, y_strides, y_strides, who));
  const long long total = N * C * OH * OW;
  if (total == 0) return B2_OK;
  if (!taps || !indices) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  if (kh * kw > 256 || !nhwc8(g, indices, indices, indices) || (reinterpret_cast<uintptr_t>(taps) & 7) || !fits32(g))
    return set_error(B2_ERR_UNSUPPORTED, "%s: needs the channels-last layout of b2_maxpool2d_fwd_taps", who);
  maxpool_taps_to_indices_kernel<int><<<pool_grid(total / 8, cur_sms()), kPoolThreads, 0,
                                        static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(taps), g,
                                                                             indices);
  return check_cuda(cudaGetLastError(), "maxpool taps to indices launch");
}

extern "C" b2_status b2_maxpool2d_bwd_taps(const void* dy, const void* taps, const int64_t* y_strides, void* dx,
                                           const int64_t* x_strides, int64_t N, int64_t C, int64_t H, int64_t W,
                                           int64_t OH, int64_t OW, int kh, int kw, int sh, int sw, int ph, int pw,
                                           int dh, int dw, void* stream) {
  const char* who = "b2_maxpool2d_bwd_taps";
  PoolGeom g;
  B2_TRY(make_pool(g, N, C, H, W, OH, OW, kh, kw, sh, sw, ph, pw, dh, dw, x_strides, y_strides, who));
  const long long total = N * C * H * W;
  if (total == 0) return B2_OK;
  if (!dx || (N * C * OH * OW > 0 && (!dy || !taps))) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  if (kh * kw > 256 || !nhwc8(g, dx, dy, dy) || (reinterpret_cast<uintptr_t>(taps) & 7) || !fits32(g) ||
      !two_cover(g))
    return set_error(B2_ERR_UNSUPPORTED, "%s: needs channels-last bf16 and windows spanning <= 2 strides", who);
  const long long cv = C / 8;
  int cv_shift = 0;
  while ((1LL << cv_shift) < cv) ++cv_shift;
  if (kh == 3 && kw == 3 && sh == 2 && sw == 2 && ph == 1 && pw == 1 && dh == 1 && dw == 1 &&
      (1LL << cv_shift) == cv && 2 * OH >= H && 2 * OW >= W && OW * cv < (1LL << 30) && N * OH <= 65535) {
    const int bs = row_threads(OW * cv);
    const dim3 grid(unsigned((OW * cv + bs - 1) / bs), unsigned(N * OH));
    maxpool_bwd_s2k3_quad_kernel<<<grid, bs, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(dy), static_cast<const uint8_t*>(taps), g, cv_shift, static_cast<uint16_t*>(dx));
    return check_cuda(cudaGetLastError(), "maxpool bwd taps launch");
  }
  maxpool_bwd_nhwc8_taps_kernel<int><<<pool_grid(total / 8, cur_sms()), kPoolThreads, 0,
                                       static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(dy), static_cast<const uint8_t*>(taps), g, static_cast<uint16_t*>(dx));
  return check_cuda(cudaGetLastError(), "maxpool bwd taps launch");
}
