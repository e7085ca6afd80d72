// Training BatchNorm2d on bf16 activations, alone (the xdna
// native_batch_norm kernels) or fused with the ReLU / LeakyReLU applied
// directly to its output (xdna_train.regions.fuse_norm_activation).  Same
// contract as the reference's fused host kernels
// (xdna_train/_native/region_kernels.cpp:309-460):
//
//   forward     y = act(x*scale + shift), scale = w*invstd, shift = b -
//               mean*scale, act(z) = z > 0 ? z : z*slope (slope 1: plain BN),
//               one rounding to bf16; invstd = 1/sqrt(var + eps) in double from
//               the biased variance; running statistics move by `momentum`
//               towards the mean and the unbiased variance.
//   backward    dz = dy where y > 0 (or y is NaN and the activation is ReLU),
//               else dy*slope (dz = dy without an activation); db = sum dz,
//               dw = sum dz*xhat (fp32 partial sums, summed in double in a
//               fixed order, see merge_partials: deterministic);
//               dx = w*invstd*(dz - db/M - xhat*dw/M), xhat = (x - mean)*invstd.
//
// Two memory layouts:
//   NCHW  each (n, c) plane reduced in fp32 (mean, then the squared
//         deviations from it; the second read of a plane hits L1/L2), the N
//         planes of a channel merged in double, in plane order, with Chan's
//         parallel-variance formula -- the reference's statistics.
//   NHWC  (channels-last) one read of x: every thread accumulates, for 8
//         consecutive channels, sums of x - K and (x - K)^2 with K the first
//         pixel's value of the channel (a shift that keeps the variance free
//         of cancellation); block partials merged in double in a fixed order.
//
// Every elementwise expression uses explicitly rounded fp32 operations in the
// reference's order (no FMA contraction: the reference's host build has none).
//
// Memory traffic (M = N*C*HW elements, algorithmic): forward 6 B/elem (x read
// twice, y written), backward 8 B/elem for plain BN (dy and x twice, dx
// written; the second reads of tensors smaller than L2 hit L2), 12 B/elem with
// the activation (y read twice too).  NHWC forward: x once for the sums.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <map>
#include <mutex>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kBnThreads = 256;
constexpr long long kMaxSumBlocks = 1024;  // NHWC partial-sum blocks (workspace bound)
constexpr long long kMaxNhwcChannels = 2048;

// Sum over the TPP threads of a plane group (a warp, or the whole block).
template <int TPP>
__device__ __forceinline__ float group_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  if constexpr (TPP == 32) {
    return v;
  } else {
    const int w = threadIdx.x >> 5;
    __syncthreads();  // red[] may still be read from a previous call
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float s = red[0];
#pragma unroll
    for (int k = 1; k < TPP / 32; ++k) s = __fadd_rn(s, red[k]);
    return s;
  }
}

__device__ __forceinline__ void unpack8(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = __uint_as_float(w[k] << 16);
    f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float* r) {
  uint4 o;
  o.x = pack_bf2(r[0], r[1]);
  o.y = pack_bf2(r[2], r[3]);
  o.z = pack_bf2(r[4], r[5]);
  o.w = pack_bf2(r[6], r[7]);
  return o;
}

// Per-channel vectors are bf16 or fp32 (B2_BF16 / B2_F32); absent -> dflt.
__device__ __forceinline__ float ld_par(const void* p, int dt, long long c, float dflt) {
  if (!p) return dflt;
  return dt == B2_F32 ? static_cast<const float*>(p)[c] : bf2f(static_cast<const uint16_t*>(p)[c]);
}
__device__ __forceinline__ void st_par(void* p, int dt, long long c, float v) {
  if (dt == B2_F32) static_cast<float*>(p)[c] = v;
  else static_cast<uint16_t*>(p)[c] = f2bf(v);
}

// Per-channel operands of the forward.
struct BnChan {
  const void* w;
  const void* b;
  int pdtype;  // dtype of w, b
  void* rm;
  void* rv;
  int rdtype;  // dtype of rm, rv; statistics updated when both are non-null
  // a module's step counter (int64 scalar) advanced by `count_inc` in the
  // same launch (b2_batch_norm_stats_count_bf16); none when null
  long long* count = nullptr;
  long long count_inc = 0;
};

__device__ __forceinline__ void finish_stats(long long c, double mean, double var, double M, float eps,
                                             float momentum, const BnChan& ch, float* mean_out,
                                             float* invstd_out) {
  mean_out[c] = float(mean);
  invstd_out[c] = float(1.0 / sqrt(var + double(eps)));
  if (c == 0 && ch.count) *ch.count += ch.count_inc;  // one thread finishes channel 0
  if (ch.rm && ch.rv) {
    const double unbiased = M > 1.0 ? var * M / (M - 1.0) : var;
    const double f = double(momentum);
    st_par(ch.rm, ch.rdtype, c, float((1.0 - f) * double(ld_par(ch.rm, ch.rdtype, c, 0.f)) + f * mean));
    st_par(ch.rv, ch.rdtype, c, float((1.0 - f) * double(ld_par(ch.rv, ch.rdtype, c, 0.f)) + f * unbiased));
  }
}

__device__ __forceinline__ float bn_act(float xv, float scale, float shift, float slope) {
  const float z = __fadd_rn(__fmul_rn(xv, scale), shift);
  return z > 0.0f ? z : __fmul_rn(z, slope);
}

// Fused tail of the plain BatchNorm forward (the ops that followed it, run in
// the same pass with their own roundings): v = bf16(z); then, with a
// residual, v = bf16(v + r) (an fp32 add, as ATen's bf16 add); then, with
// relu, v = v > 0 ? v : 0 (NaN kept).
__device__ __forceinline__ float round_bf(float v) { return bf2f(f2bf(v)); }
__device__ __forceinline__ float bn_tail(float z, bool has_res, float res, bool relu) {
  float v = round_bf(z);
  if (has_res) v = round_bf(__fadd_rn(v, res));
  if (relu && !(v > 0.0f) && v == v) v = 0.0f;
  return v;
}

template <bool ACT>
__device__ __forceinline__ float bn_dz(float g, float yv, float slope, int relu) {
  if constexpr (!ACT) return g;
  else return ((yv > 0.0f) || (relu && yv != yv)) ? g : __fmul_rn(g, slope);
}

template <bool ACT>
__device__ __forceinline__ float bn_dx(float g, float yv, float xv, float mc, float is, float ws, float k1,
                                       float k2, float slope, int relu) {
  const float dz = bn_dz<ACT>(g, yv, slope, relu);
  const float xhat = __fmul_rn(__fsub_rn(xv, mc), is);
  return __fmul_rn(ws, __fsub_rn(__fsub_rn(dz, k1), __fmul_rn(xhat, k2)));
}

// ============================ NCHW ==========================================

// Per-plane fp32 mean and sum of squared deviations.  TPP threads per plane:
// a warp (many small planes) or the whole block (few large planes).  VEC:
// 8 elements per 16-byte load (HW % 8 == 0, so every plane starts aligned).
template <int TPP, bool VEC>
__global__ void __launch_bounds__(kBnThreads) bn_plane_stats_kernel(
    const uint16_t* __restrict__ x, long long planes, long long hw, float* __restrict__ pm,
    float* __restrict__ pq) {
  __shared__ float red[kBnThreads / 32];
  constexpr int kGroups = kBnThreads / TPP;
  const int lane = threadIdx.x % TPP;
  const long long g0 = (long long)blockIdx.x * kGroups + threadIdx.x / TPP;
  const long long gstep = (long long)gridDim.x * kGroups;
  // all threads of a block run the same number of iterations (group_sum syncs)
  const long long iters = (planes + gstep - 1) / gstep;
  for (long long it = 0; it < iters; ++it) {
    const long long pl = g0 + it * gstep;
    const bool live = pl < planes;
    const uint16_t* p = x + (live ? pl : 0) * hw;
    float s = 0.0f;
    if (live) {
      if constexpr (VEC) {
        const uint4* pv = reinterpret_cast<const uint4*>(p);
        for (long long v = lane; v < hw / 8; v += TPP) {
          float f[8];
          unpack8(__ldg(pv + v), f);
#pragma unroll
          for (int k = 0; k < 8; ++k) s = __fadd_rn(s, f[k]);
        }
      } else {
        for (long long i = lane; i < hw; i += TPP) s = __fadd_rn(s, bf2f(p[i]));
      }
    }
    const float mean = __fdiv_rn(group_sum<TPP>(s, red), float(hw));
    float q = 0.0f;
    if (live) {
      if constexpr (VEC) {
        const uint4* pv = reinterpret_cast<const uint4*>(p);
        for (long long v = lane; v < hw / 8; v += TPP) {
          float f[8];
          unpack8(__ldg(pv + v), f);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float d = __fsub_rn(f[k], mean);
            q = __fadd_rn(q, __fmul_rn(d, d));
          }
        }
      } else {
        for (long long i = lane; i < hw; i += TPP) {
          const float d = __fsub_rn(bf2f(p[i]), mean);
          q = __fadd_rn(q, __fmul_rn(d, d));
        }
      }
    }
    q = group_sum<TPP>(q, red);
    if (live && lane == 0) {
      pm[pl] = mean;
      pq[pl] = q;
    }
  }
}

// One thread per channel: Chan's merge of the N plane statistics in double,
// in plane order; mean / invstd out; running statistics.
// Channel statistics from the per-plane (mean, M2) partials: a warp per
// channel, lane l merging planes l, l+32, ... in order (Chan's parallel
// update, in double), then the lanes merged by a fixed shuffle tree --
// deterministic, and N-fold shorter dependent chains than one thread per
// channel walking all N planes.
__device__ __forceinline__ void chan_merge(double& n, double& mean, double& m2, double nb, double mb, double m2b) {
  if (nb == 0.0) return;
  if (n == 0.0) {
    n = nb;
    mean = mb;
    m2 = m2b;
    return;
  }
  const double tot = n + nb;
  const double delta = mb - mean;
  mean += delta * nb / tot;
  m2 += m2b + delta * delta * n * nb / tot;
  n = tot;
}

__global__ void bn_channel_stats_kernel(const float* __restrict__ pm, const float* __restrict__ pq,
                                        long long N, long long C, long long hw, float eps, float momentum,
                                        BnChan ch, float* __restrict__ mean_out, float* __restrict__ invstd_out) {
  const long long c = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (c >= C) return;
  const double nb = double(hw);
  double count = 0.0, mean = 0.0, m2 = 0.0;
  for (long long n = lane; n < N; n += 32) chan_merge(count, mean, m2, nb, double(pm[n * C + c]), double(pq[n * C + c]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double ob = __shfl_down_sync(0xffffffffu, count, off);
    const double om = __shfl_down_sync(0xffffffffu, mean, off);
    const double oq = __shfl_down_sync(0xffffffffu, m2, off);
    chan_merge(count, mean, m2, ob, om, oq);
  }
  if (lane == 0) {
    const double M = double(N) * nb;
    finish_stats(c, mean, m2 / M, M, eps, momentum, ch, mean_out, invstd_out);
  }
}

// y = act(x*scale + shift); one thread per 8 elements (VEC) or per element.
// EPI: the fused tail (bn_tail) with an optional residual `res` (x's layout)
// and ReLU instead of the activation.
template <bool VEC, bool EPI>
__global__ void __launch_bounds__(kBnThreads) bn_apply_kernel(
    const uint16_t* __restrict__ x, BnChan ch, const float* __restrict__ mean, const float* __restrict__ invstd,
    uint16_t* __restrict__ y, long long units, long long units_per_plane, long long C, float slope,
    const uint16_t* __restrict__ res, int relu) {
  for (long long u = (long long)blockIdx.x * kBnThreads + threadIdx.x; u < units;
       u += (long long)gridDim.x * kBnThreads) {
    const long long c = (u / units_per_plane) % C;
    const float scale = __fmul_rn(ld_par(ch.w, ch.pdtype, c, 1.0f), __ldg(invstd + c));
    const float shift = __fsub_rn(ld_par(ch.b, ch.pdtype, c, 0.0f), __fmul_rn(__ldg(mean + c), scale));
    if constexpr (VEC) {
      float f[8], r[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + u), f);
      if constexpr (EPI) {
        float q[8];
        if (res) unpack8(__ldg(reinterpret_cast<const uint4*>(res) + u), q);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          r[e] = bn_tail(__fadd_rn(__fmul_rn(f[e], scale), shift), res != nullptr, res ? q[e] : 0.f, relu != 0);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) r[e] = bn_act(f[e], scale, shift, slope);
      }
      reinterpret_cast<uint4*>(y)[u] = pack8(r);
    } else if constexpr (EPI) {
      y[u] = f2bf(bn_tail(__fadd_rn(__fmul_rn(bf2f(x[u]), scale), shift), res != nullptr, res ? bf2f(res[u]) : 0.f,
                          relu != 0));
    } else {
      y[u] = f2bf(bn_act(bf2f(x[u]), scale, shift, slope));
    }
  }
}

// Per-plane fp32 sums of dz and dz*xhat.
template <int TPP, bool VEC, bool ACT>
__global__ void __launch_bounds__(kBnThreads) bn_bwd_plane_kernel(
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y, const uint16_t* __restrict__ x,
    const float* __restrict__ mean, const float* __restrict__ invstd, long long planes, long long C,
    long long hw, float slope, int relu, float* __restrict__ ps, float* __restrict__ pt) {
  __shared__ float red[kBnThreads / 32];
  constexpr int kGroups = kBnThreads / TPP;
  const int lane = threadIdx.x % TPP;
  const long long g0 = (long long)blockIdx.x * kGroups + threadIdx.x / TPP;
  const long long gstep = (long long)gridDim.x * kGroups;
  const long long iters = (planes + gstep - 1) / gstep;
  for (long long it = 0; it < iters; ++it) {
    const long long pl = g0 + it * gstep;
    const bool live = pl < planes;
    float s1 = 0.0f, s2 = 0.0f;
    if (live) {
      const long long c = pl % C;
      const float mc = __ldg(mean + c), is = __ldg(invstd + c);
      const long long off = pl * hw;
      if constexpr (VEC) {
        const uint4* dv = reinterpret_cast<const uint4*>(dy + off);
        const uint4* yv = reinterpret_cast<const uint4*>((ACT ? y : dy) + off);
        const uint4* xv = reinterpret_cast<const uint4*>(x + off);
        for (long long v = lane; v < hw / 8; v += TPP) {
          float fg[8], fy[8], fx[8];
          unpack8(__ldg(dv + v), fg);
          if constexpr (ACT) unpack8(__ldg(yv + v), fy);
          unpack8(__ldg(xv + v), fx);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float dz = bn_dz<ACT>(fg[k], ACT ? fy[k] : 0.0f, slope, relu);
            s1 = __fadd_rn(s1, dz);
            s2 = __fadd_rn(s2, __fmul_rn(dz, __fmul_rn(__fsub_rn(fx[k], mc), is)));
          }
        }
      } else {
        for (long long i = lane; i < hw; i += TPP) {
          const float dz = bn_dz<ACT>(bf2f(dy[off + i]), ACT ? bf2f(y[off + i]) : 0.0f, slope, relu);
          s1 = __fadd_rn(s1, dz);
          s2 = __fadd_rn(s2, __fmul_rn(dz, __fmul_rn(__fsub_rn(bf2f(x[off + i]), mc), is)));
        }
      }
    }
    s1 = group_sum<TPP>(s1, red);
    s2 = group_sum<TPP>(s2, red);
    if (live && lane == 0) {
      // channel-major partials: row (channel) c holds its N plane sums
      const long long idx = (pl % C) * (planes / C) + pl / C;
      ps[idx] = s1;
      pt[idx] = s2;
    }
  }
}

// Sums of the `parts` partial sums of channel c (channel-major: pa[c*parts +
// r]) in double, in a fixed order: one block per channel; thread t adds rows
// t, t+256, t+512, ... in order (their loads issued together, coalesced across
// the block), then a fixed shuffle / shared-memory tree adds the 256 thread
// sums.  Deterministic and independent of scheduling.  Returns true in thread 0.
constexpr int kMergeThreads = 256;
constexpr int kMergeAhead = 4;

__device__ __forceinline__ bool merge_partials(const float* __restrict__ pa, const float* __restrict__ pb,
                                               long long parts, long long c, double& a, double& b) {
  __shared__ double ra[kMergeThreads / 32], rb[kMergeThreads / 32];
  const float* qa = pa + c * parts;
  const float* qb = pb + c * parts;
  double sa = 0.0, sb = 0.0;
  for (long long r0 = threadIdx.x; r0 < parts; r0 += (long long)kMergeThreads * kMergeAhead) {
    float va[kMergeAhead], vb[kMergeAhead];
#pragma unroll
    for (int i = 0; i < kMergeAhead; ++i) {
      const long long r = r0 + (long long)i * kMergeThreads;
      va[i] = r < parts ? __ldg(qa + r) : 0.0f;
      vb[i] = r < parts ? __ldg(qb + r) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < kMergeAhead; ++i) {
      sa += double(va[i]);
      sb += double(vb[i]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    ra[w] = sa;
    rb[w] = sb;
  }
  __syncthreads();
  if (threadIdx.x != 0) return false;
  a = ra[0];
  b = rb[0];
#pragma unroll
  for (int k = 1; k < kMergeThreads / 32; ++k) {
    a += ra[k];
    b += rb[k];
  }
  return true;
}

// Backward: db, dw (dtype gdtype) and the two means the dx pass needs
// (k[c] = db/M, k[C + c] = dw/M).  Grid: ceil(C/32) blocks of 256 threads.
__global__ void __launch_bounds__(kMergeThreads) bn_bwd_channel_kernel(
    const float* __restrict__ ps, const float* __restrict__ pt, long long parts, long long C, double M, void* dw,
    void* db, int gdtype, float* __restrict__ k) {
  const long long c = blockIdx.x;
  double a, bs;
  if (!merge_partials(ps, pt, parts, c, a, bs)) return;
  if (db) st_par(db, gdtype, c, float(a));
  if (dw) st_par(dw, gdtype, c, float(bs));
  k[c] = float(a / M);
  k[C + c] = float(bs / M);
}

template <bool VEC, bool ACT>
__global__ void __launch_bounds__(kBnThreads) bn_bwd_dx_kernel(
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y, const uint16_t* __restrict__ x,
    const void* w, int pdtype, const float* __restrict__ mean, const float* __restrict__ invstd,
    const float* __restrict__ k, uint16_t* __restrict__ dx, long long units, long long units_per_plane,
    long long C, float slope, int relu) {
  for (long long u = (long long)blockIdx.x * kBnThreads + threadIdx.x; u < units;
       u += (long long)gridDim.x * kBnThreads) {
    const long long c = (u / units_per_plane) % C;
    const float mc = __ldg(mean + c), is = __ldg(invstd + c);
    const float ws = __fmul_rn(ld_par(w, pdtype, c, 1.0f), is);
    const float k1 = __ldg(k + c), k2 = __ldg(k + C + c);
    if constexpr (VEC) {
      float fg[8], fy[8], fx[8], r[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(dy) + u), fg);
      if constexpr (ACT) unpack8(__ldg(reinterpret_cast<const uint4*>(y) + u), fy);
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + u), fx);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        r[e] = bn_dx<ACT>(fg[e], ACT ? fy[e] : 0.0f, fx[e], mc, is, ws, k1, k2, slope, relu);
      reinterpret_cast<uint4*>(dx)[u] = pack8(r);
    } else {
      dx[u] = f2bf(bn_dx<ACT>(bf2f(dy[u]), ACT ? bf2f(y[u]) : 0.0f, bf2f(x[u]), mc, is, ws, k1, k2, slope,
                              relu));
    }
  }
}

// ============================ NHWC ==========================================
// x viewed as [P pixels][C], C % 8 == 0, C <= kMaxNhwcChannels, 16-byte
// aligned.  A block is CV = C/8 channel groups wide and rpb = 256/CV pixel rows
// deep; thread (row pr, group cg) owns channels [8cg, 8cg+8).

struct NhwcShape {
  long long P;
  int C, CV, rpb;
};

// Sums per block and channel:  forward  a = sum(x - K), b = sum((x - K)^2)
//                              backward a = sum(dz),    b = sum(dz * xhat)
template <bool BWD, bool ACT>
__global__ void __launch_bounds__(kBnThreads) bn_nhwc_sums_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y,
    const float* __restrict__ mean, const float* __restrict__ invstd, NhwcShape sh, float slope, int relu,
    float* __restrict__ part_a, float* __restrict__ part_b) {
  extern __shared__ float red[];  // [2][rpb][C]
  const int cg = threadIdx.x % sh.CV, pr = threadIdx.x / sh.CV;
  const bool active = pr < sh.rpb;
  float a[8], b[8], k0[8], k1[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = b[e] = 0.0f;
  if (active) {
    const int c0 = cg * 8;
    if constexpr (BWD) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        k0[e] = mean[c0 + e];
        k1[e] = invstd[c0 + e];
      }
    } else {
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + cg), k0);  // shift K: the first pixel
    }
    auto accum = [&](const uint4 vx, const uint4 vg, const uint4 vy) {
      float fx[8];
      unpack8(vx, fx);
      if constexpr (BWD) {
        float fg[8], fy[8];
        unpack8(vg, fg);
        if constexpr (ACT) unpack8(vy, fy);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float dz = bn_dz<ACT>(fg[e], ACT ? fy[e] : 0.0f, slope, relu);
          a[e] = __fadd_rn(a[e], dz);
          b[e] = __fadd_rn(b[e], __fmul_rn(dz, __fmul_rn(__fsub_rn(fx[e], k0[e]), k1[e])));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = __fsub_rn(fx[e], k0[e]);
          a[e] = __fadd_rn(a[e], d);
          b[e] = __fadd_rn(b[e], __fmul_rn(d, d));
        }
      }
    };
    const uint4* x4 = reinterpret_cast<const uint4*>(x);
    const uint4* g4 = reinterpret_cast<const uint4*>(dy);
    const uint4* y4 = reinterpret_cast<const uint4*>(y);
    const uint4 zero = make_uint4(0, 0, 0, 0);
    const long long step = (long long)gridDim.x * sh.rpb;
    long long p = (long long)blockIdx.x * sh.rpb + pr;
    // four pixels' loads in flight before their additions (in pixel order)
    for (; p + 3 * step < sh.P; p += 4 * step) {
      uint4 vx[4], vg[4], vy[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const long long u = (p + i * step) * sh.CV + cg;
        vx[i] = __ldg(x4 + u);
        vg[i] = BWD ? __ldg(g4 + u) : zero;
        vy[i] = ACT ? __ldg(y4 + u) : zero;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) accum(vx[i], vg[i], vy[i]);
    }
    for (; p < sh.P; p += step) {
      const long long u = p * sh.CV + cg;
      accum(__ldg(x4 + u), BWD ? __ldg(g4 + u) : zero, ACT ? __ldg(y4 + u) : zero);
    }
    float* ra = red + (long long)pr * sh.C + cg * 8;
    float* rb = red + (long long)(sh.rpb + pr) * sh.C + cg * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ra[e] = a[e];
      rb[e] = b[e];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < sh.C; c += kBnThreads) {
    float sa = 0.0f, sb = 0.0f;
    for (int r = 0; r < sh.rpb; ++r) {
      sa = __fadd_rn(sa, red[(long long)r * sh.C + c]);
      sb = __fadd_rn(sb, red[(long long)(sh.rpb + r) * sh.C + c]);
    }
    part_a[(long long)c * gridDim.x + blockIdx.x] = sa;  // channel-major
    part_b[(long long)c * gridDim.x + blockIdx.x] = sb;
  }
}

// Forward merge of the block partials (one block per channel), statistics out.
__global__ void __launch_bounds__(kMergeThreads) bn_nhwc_stats_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ part_a, const float* __restrict__ part_b,
    long long blocks, long long C, long long P, float eps, float momentum, BnChan ch, float* __restrict__ mean_out,
    float* __restrict__ invstd_out) {
  const long long c = blockIdx.x;
  double s, q;
  if (!merge_partials(part_a, part_b, blocks, c, s, q)) return;
  const double M = double(P);
  const double shift = double(bf2f(x[c]));
  const double var = fmax(0.0, (q - s * s / M) / M);
  finish_stats(c, shift + s / M, var, M, eps, momentum, ch, mean_out, invstd_out);
}

// y = act(x*scale + shift).  FIXED: CV divides the block size, so every
// thread keeps one channel group through the grid-stride loop and holds its 8
// scales and shifts in registers; otherwise they are staged in shared memory.
template <bool FIXED, bool EPI>
__global__ void __launch_bounds__(kBnThreads) bn_nhwc_apply_kernel(
    const uint16_t* __restrict__ x, BnChan ch, const float* __restrict__ mean, const float* __restrict__ invstd,
    uint16_t* __restrict__ y, NhwcShape sh, float slope, const uint16_t* __restrict__ res, int relu) {
  extern __shared__ float tab[];  // scale[C], shift[C] (!FIXED)
  float scale[8], shift[8];
  if constexpr (FIXED) {
    const int c0 = int(threadIdx.x % sh.CV) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      scale[e] = __fmul_rn(ld_par(ch.w, ch.pdtype, c0 + e, 1.0f), invstd[c0 + e]);
      shift[e] = __fsub_rn(ld_par(ch.b, ch.pdtype, c0 + e, 0.0f), __fmul_rn(mean[c0 + e], scale[e]));
    }
  } else {
    for (int c = threadIdx.x; c < sh.C; c += kBnThreads) {
      const float sc = __fmul_rn(ld_par(ch.w, ch.pdtype, c, 1.0f), invstd[c]);
      tab[c] = sc;
      tab[sh.C + c] = __fsub_rn(ld_par(ch.b, ch.pdtype, c, 0.0f), __fmul_rn(mean[c], sc));
    }
    __syncthreads();
  }
  const long long units = sh.P * sh.CV;
  const long long stride = (long long)gridDim.x * kBnThreads;
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  const uint4* r4 = reinterpret_cast<const uint4*>(res);
  uint4* y4 = reinterpret_cast<uint4*>(y);
  const bool has_res = EPI && res != nullptr;
  auto one = [&](const uint4 v, const uint4 rv) {
    float f[8], r[8];
    unpack8(v, f);
    if constexpr (EPI) {
      float q[8];
      unpack8(rv, q);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        r[e] = bn_tail(__fadd_rn(__fmul_rn(f[e], scale[e]), shift[e]), has_res, q[e], relu != 0);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = bn_act(f[e], scale[e], shift[e], slope);
    }
    return pack8(r);
  };
  const uint4 zero4 = make_uint4(0, 0, 0, 0);
  long long u = (long long)blockIdx.x * kBnThreads + threadIdx.x;
  if constexpr (FIXED) {  // the channel group is the same for u, u + stride, ...
    for (; u + 3 * stride < units; u += 4 * stride) {
      uint4 v[4], q[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = __ldg(x4 + u + i * stride);
        q[i] = has_res ? __ldg(r4 + u + i * stride) : zero4;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) y4[u + i * stride] = one(v[i], q[i]);
    }
  }
  for (; u < units; u += stride) {
    if constexpr (!FIXED) {
      const int c0 = int(u % sh.CV) * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        scale[e] = tab[c0 + e];
        shift[e] = tab[sh.C + c0 + e];
      }
    }
    y4[u] = one(__ldg(x4 + u), has_res ? __ldg(r4 + u) : zero4);
  }
}

template <bool ACT, bool FIXED>
__global__ void __launch_bounds__(kBnThreads) bn_nhwc_dx_kernel(
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y, const uint16_t* __restrict__ x,
    const void* w, int pdtype, const float* __restrict__ mean, const float* __restrict__ invstd,
    const float* __restrict__ k, uint16_t* __restrict__ dx, NhwcShape sh, float slope, int relu) {
  extern __shared__ float tab[];  // ws[C], mean[C], invstd[C], k1[C], k2[C] (!FIXED)
  const int C = sh.C;
  float ws[8], mc[8], is[8], k1[8], k2[8];
  if constexpr (FIXED) {
    const int c0 = int(threadIdx.x % sh.CV) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = c0 + e;
      ws[e] = __fmul_rn(ld_par(w, pdtype, c, 1.0f), invstd[c]);
      mc[e] = mean[c];
      is[e] = invstd[c];
      k1[e] = k[c];
      k2[e] = k[C + c];
    }
  } else {
    for (int c = threadIdx.x; c < C; c += kBnThreads) {
      tab[c] = __fmul_rn(ld_par(w, pdtype, c, 1.0f), invstd[c]);
      tab[C + c] = mean[c];
      tab[2 * C + c] = invstd[c];
      tab[3 * C + c] = k[c];
      tab[4 * C + c] = k[C + c];
    }
    __syncthreads();
  }
  const long long units = sh.P * sh.CV;
  const long long stride = (long long)gridDim.x * kBnThreads;
  const uint4* g4 = reinterpret_cast<const uint4*>(dy);
  const uint4* y4 = reinterpret_cast<const uint4*>(y);
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  uint4* d4 = reinterpret_cast<uint4*>(dx);
  const uint4 zero = make_uint4(0, 0, 0, 0);
  auto one = [&](const uint4 vg, const uint4 vy, const uint4 vx) {
    float fg[8], fy[8], fx[8], r[8];
    unpack8(vg, fg);
    if constexpr (ACT) unpack8(vy, fy);
    unpack8(vx, fx);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      r[e] = bn_dx<ACT>(fg[e], ACT ? fy[e] : 0.0f, fx[e], mc[e], is[e], ws[e], k1[e], k2[e], slope, relu);
    return pack8(r);
  };
  long long u = (long long)blockIdx.x * kBnThreads + threadIdx.x;
  if constexpr (FIXED) {  // the channel group is the same for u, u + stride, ...
    for (; u + 3 * stride < units; u += 4 * stride) {
      uint4 vg[4], vy[4], vx[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        vg[i] = __ldg(g4 + u + i * stride);
        vy[i] = ACT ? __ldg(y4 + u + i * stride) : zero;
        vx[i] = __ldg(x4 + u + i * stride);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) d4[u + i * stride] = one(vg[i], vy[i], vx[i]);
    }
  }
  for (; u < units; u += stride) {
    if constexpr (!FIXED) {
      const int c0 = int(u % sh.CV) * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = c0 + e;
        ws[e] = tab[c];
        mc[e] = tab[C + c];
        is[e] = tab[2 * C + c];
        k1[e] = tab[3 * C + c];
        k2[e] = tab[4 * C + c];
      }
    }
    d4[u] = one(__ldg(g4 + u), ACT ? __ldg(y4 + u) : zero, __ldg(x4 + u));
  }
}

// ============================ NHWC streaming ================================
// The channels-last passes fed through shared memory.  Each CTA streams 8 KB
// chunks of its inputs (chunks b, b + G, b + 2G, ... of the 16-byte-unit
// array, u = pixel * CV + channel group) through a ring of stages that one
// producer warp fills with 1-D bulk copies (no multicast): ~96 KB per CTA in
// flight, two CTAs per SM, where the register kernels above keep at most four
// loads per thread outstanding.  256 consumer threads take units t and t + 256
// of every chunk; with CV dividing 256 a thread's channel group is t % CV in
// every chunk, so its per-channel coefficients stay in registers.  Element for
// element the same arithmetic as the register kernels (the sums kernel adds in
// another, still fixed, order).  Rounding to bf16 uses the hardware's
// round-to-nearest-even conversion, with NaNs sent through f2bf so that their
// bits stay the reference's.
//
// Chunks of kChunkUnits units are what CTAs are assigned (chunk j to CTA j mod
// G); a ring stage holds stage_units<NIN>() units of each input: the whole
// chunk for one or two inputs (16 KB copies; measured 3-4 % faster than 8 KB
// on 205 MB passes), half of it for three or four (8 KB copies, so their
// rings keep three or more stages).  A consumer thread visits the units t,
// t + 256, t + 512, t + 768 of every chunk in that order either way, so the
// sums kernels' partial sums do not depend on the input count.
constexpr int kStreamConsumers = 256;
constexpr int kStreamThreads = kStreamConsumers + 32;
constexpr int kChunkUnits = 1024;
constexpr int kRingBytes = 96 * 1024;

template <int NIN>
__host__ __device__ constexpr int stage_units() {
  return NIN <= 2 ? kChunkUnits : kChunkUnits / 2;
}
template <int NIN>
__host__ __device__ constexpr int ring_stages() {
  return kRingBytes / (NIN * stage_units<NIN>() * 16);
}
template <int NIN>
__host__ __device__ constexpr size_t ring_smem_bytes() {
  return size_t(kRingBytes) + 2 * sizeof(uint64_t) * ring_stages<NIN>() + 16;
}

__device__ __forceinline__ uint32_t pack_bf2_fast(float lo, float hi) {
  if (lo != lo || hi != hi) return pack_bf2(lo, hi);
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint4 pack8_fast(const float* r) {
  return make_uint4(pack_bf2_fast(r[0], r[1]), pack_bf2_fast(r[2], r[3]), pack_bf2_fast(r[4], r[5]),
                    pack_bf2_fast(r[6], r[7]));
}
__device__ __forceinline__ float round_bf_fast(float v) {
  return v != v ? round_bf(v) : __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float bn_tail_fast(float z, bool has_res, float res, bool relu) {
  float v = round_bf_fast(z);
  if (has_res) v = round_bf_fast(__fadd_rn(v, res));
  if (relu && !(v > 0.0f) && v == v) v = 0.0f;
  return v;
}

// Named barrier over the consumer threads (the producer warp has returned).
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kStreamConsumers) : "memory");
}

// Calls f(u, v) on the consumer threads for every unit u of this CTA's chunks,
// v[i] = src[i][u].  Returns false on a consumer whose wait gave up (status
// recorded, the other roles told through the CTA's abort flag), and on the
// producer warp, which returns once its last copy is issued.
template <int NIN, class F>
__device__ __forceinline__ bool stream_units(const uint4* const (&src)[NIN], long long units, F&& f, int* status) {
  constexpr int S = ring_stages<NIN>();
  constexpr int SU = stage_units<NIN>();
  constexpr int kStageBytes = SU * 16;
  constexpr int SPLIT = kChunkUnits / SU;
  static_assert(S >= 2 && SPLIT * SU == kChunkUnits && SU % kStreamConsumers == 0, "ring shape");
  extern __shared__ __align__(128) uint8_t ring[];
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRingBytes);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kStreamConsumers / 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const long long nchunks = (units + kChunkUnits - 1) / kChunkUnits;
  if (warp == kStreamConsumers / 32) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int last[S];
#pragma unroll
      for (int i = 0; i < S; ++i) last[i] = -1;
      bool ok = true;
      for (long long j = blockIdx.x; j < nchunks && ok; j += gridDim.x) {
        for (int h = 0; h < SPLIT; ++h) {
          const long long u0 = j * kChunkUnits + (long long)h * SU;
          if (u0 >= units) break;
          if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1, status, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bytes = uint32_t(units - u0 < SU ? units - u0 : SU) * 16u;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_arrive_expect_tx(fb, uint32_t(NIN) * bytes);
          last[s] = int(ph);
#pragma unroll
          for (int i = 0; i < NIN; ++i)
            bulk_load_1d(smem_u32(ring + (s * NIN + i) * kStageBytes), src[i] + u0, bytes, fb);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok)  // let the copies already issued land before the CTA can exit
        for (int i = 0; i < S; ++i)
          if (last[i] >= 0) mbar_wait(smem_u32(&full[i]), uint32_t(last[i]), status, nullptr);
    }
    return false;
  }
  int s = 0;
  uint32_t ph = 0;
  for (long long j = blockIdx.x; j < nchunks; j += gridDim.x) {
    for (int h = 0; h < SPLIT; ++h) {
      const long long u0 = j * kChunkUnits + (long long)h * SU;
      if (u0 >= units) break;
      if (!mbar_wait(smem_u32(&full[s]), ph, status, abort_flag)) return false;
      const int n = int(units - u0 < SU ? units - u0 : SU);
      const uint4* stg = reinterpret_cast<const uint4*>(ring + s * NIN * kStageBytes);
      for (int k = threadIdx.x; k < n; k += kStreamConsumers) {
        uint4 v[NIN];
#pragma unroll
        for (int i = 0; i < NIN; ++i) v[i] = stg[i * SU + k];
        f(u0 + k, v);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[s]));
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
    }
  }
  return true;
}

// End of a sums kernel (consumer threads): the rows R = 256 / CV of each
// channel group reduced in row order through the ring's memory (every copy
// into it has landed), one partial per channel written channel-major.
__device__ __forceinline__ void sums_tail(const float (&a)[8], const float (&b)[8], const NhwcShape& sh, int cg,
                                          bool ok, float* __restrict__ part_a, float* __restrict__ part_b) {
  extern __shared__ __align__(128) uint8_t ring[];
  float* red = reinterpret_cast<float*>(ring);  // [2][R][C]
  const int R = kStreamConsumers / sh.CV, r = threadIdx.x / sh.CV;
  consumers_sync();
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    red[r * sh.C + cg * 8 + e] = a[e];
    red[(R + r) * sh.C + cg * 8 + e] = b[e];
  }
  consumers_sync();
  if (!ok) return;
  for (int c = threadIdx.x; c < sh.C; c += kStreamConsumers) {
    float sa = 0.0f, sb = 0.0f;
    for (int q = 0; q < R; ++q) {
      sa = __fadd_rn(sa, red[q * sh.C + c]);
      sb = __fadd_rn(sb, red[(R + q) * sh.C + c]);
    }
    part_a[(long long)c * gridDim.x + blockIdx.x] = sa;  // channel-major
    part_b[(long long)c * gridDim.x + blockIdx.x] = sb;
  }
}

// The ReLU that followed a BatchNorm, recomputed from its input: the forward
// wrote y = relu(bf16(z)), z = x*scale + shift (bn_tail_fast without a
// residual), and ATen's threshold_backward passes dy where y > 0 or y is NaN,
// elsewhere the gradient is exactly +0.  bf16(z) > 0 exactly when z > 2^-134:
// the smallest positive bf16 is 2^-133, and round-to-nearest-even sends z in
// (0, 2^-134] -- the tie included -- to zero.  So the gate is !(z <= 2^-134),
// NaN passing, with no rounding.
__device__ __forceinline__ float relu_gate(float g, float xv, float scale, float shift) {
  const float z = __fadd_rn(__fmul_rn(xv, scale), shift);
  return !(z <= 0x1p-134f) ? g : 0.0f;
}

// Sums per CTA and channel (as bn_nhwc_sums_kernel): forward a = sum(x - K),
// b = sum((x - K)^2), K the first pixel; backward a = sum(dz), b = sum(dz *
// xhat).  Inputs in ring order x, dy, y.  RC (backward): dz = relu_gate(dy)
// with scale and shift from rc's w, b and the saved statistics (no y read).
template <bool BWD, bool ACT, bool RC = false>
__global__ void __launch_bounds__(kStreamThreads) bn_nhwc_stream_sums_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y,
    const float* __restrict__ mean, const float* __restrict__ invstd, NhwcShape sh, float slope, int relu,
    float* __restrict__ part_a, float* __restrict__ part_b, int* status, BnChan rc = BnChan{}) {
  static_assert(!RC || (BWD && !ACT), "the recomputed ReLU gate is a backward of plain BatchNorm");
  constexpr int NIN = BWD ? (ACT ? 3 : 2) : 1;
  const bool consumer = threadIdx.x < kStreamConsumers;
  const int cg = threadIdx.x % sh.CV;
  float a[8], b[8], k0[8], k1[8], gsc[8], gsh[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = b[e] = k0[e] = k1[e] = gsc[e] = gsh[e] = 0.0f;
  if (consumer) {
    if constexpr (BWD) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        k0[e] = mean[cg * 8 + e];
        k1[e] = invstd[cg * 8 + e];
      }
      if constexpr (RC) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          gsc[e] = __fmul_rn(ld_par(rc.w, rc.pdtype, cg * 8 + e, 1.0f), k1[e]);
          gsh[e] = __fsub_rn(ld_par(rc.b, rc.pdtype, cg * 8 + e, 0.0f), __fmul_rn(k0[e], gsc[e]));
        }
      }
    } else {
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + cg), k0);  // shift K: the first pixel
    }
  }
  const uint4* src[NIN];
  src[0] = reinterpret_cast<const uint4*>(x);
  if constexpr (BWD) src[1] = reinterpret_cast<const uint4*>(dy);
  if constexpr (ACT) src[NIN - 1] = reinterpret_cast<const uint4*>(y);
  const bool ok = stream_units<NIN>(src, sh.P * sh.CV, [&](long long, const uint4(&v)[NIN]) {
    float fx[8];
    unpack8(v[0], fx);
    if constexpr (BWD) {
      float fg[8], fy[8];
      unpack8(v[1], fg);
      if constexpr (ACT) unpack8(v[NIN - 1], fy);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float dz = RC ? relu_gate(fg[e], fx[e], gsc[e], gsh[e]) : bn_dz<ACT>(fg[e], ACT ? fy[e] : 0.0f, slope, relu);
        a[e] = __fadd_rn(a[e], dz);
        b[e] = __fadd_rn(b[e], __fmul_rn(dz, __fmul_rn(__fsub_rn(fx[e], k0[e]), k1[e])));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = __fsub_rn(fx[e], k0[e]);
        a[e] = __fadd_rn(a[e], d);
        b[e] = __fadd_rn(b[e], __fmul_rn(d, d));
      }
    }
  }, status);
  if (!consumer) return;
  sums_tail(a, b, sh, cg, ok, part_a, part_b);
}

// Backward sums of a BatchNorm whose output feeds a ReLU through a residual
// sum: the gradient at the BatchNorm's output is dz = (y > 0 or NaN) ?
// bf16(a + b) : +0 (a ReLU backward on the sum of two gradients, as
// b2_relu_bwd_sum_bf16), made here in the same pass that sums it: dz is
// written out (its other readers need it) and summed as the plain backward
// sums its dy.  Inputs in ring order x, a, b, y.
__global__ void __launch_bounds__(kStreamThreads) bn_nhwc_stream_sums_gsum_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ ga, const uint16_t* __restrict__ gb,
    const uint16_t* __restrict__ y, const float* __restrict__ mean, const float* __restrict__ invstd, NhwcShape sh,
    uint16_t* __restrict__ dz_out, float* __restrict__ part_a, float* __restrict__ part_b, int* status) {
  constexpr int NIN = 4;
  const bool consumer = threadIdx.x < kStreamConsumers;
  const int cg = threadIdx.x % sh.CV;
  float a[8], b[8], k0[8], k1[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = b[e] = k0[e] = k1[e] = 0.0f;
  if (consumer) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      k0[e] = mean[cg * 8 + e];
      k1[e] = invstd[cg * 8 + e];
    }
  }
  const uint4* src[NIN] = {reinterpret_cast<const uint4*>(x), reinterpret_cast<const uint4*>(ga),
                           reinterpret_cast<const uint4*>(gb), reinterpret_cast<const uint4*>(y)};
  uint4* d4 = reinterpret_cast<uint4*>(dz_out);
  const bool ok = stream_units<NIN>(src, sh.P * sh.CV, [&](long long u, const uint4(&v)[NIN]) {
    float fx[8], fa[8], fb[8], fy[8], dz[8];
    unpack8(v[0], fx);
    unpack8(v[1], fa);
    unpack8(v[2], fb);
    unpack8(v[3], fy);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t hb = !(fy[e] <= 0.0f) ? uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(__fadd_rn(fa[e], fb[e]))))
                                           : 0u;
      w[e >> 1] |= hb << (16 * (e & 1));
      dz[e] = __uint_as_float(hb << 16);
    }
    d4[u] = make_uint4(w[0], w[1], w[2], w[3]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      a[e] = __fadd_rn(a[e], dz[e]);
      b[e] = __fadd_rn(b[e], __fmul_rn(dz[e], __fmul_rn(__fsub_rn(fx[e], k0[e]), k1[e])));
    }
  }, status);
  if (!consumer) return;
  sums_tail(a, b, sh, cg, ok, part_a, part_b);
}

// y = act(x*scale + shift), or the fused tail (residual, ReLU) with EPI.
template <bool EPI, bool RES>
__global__ void __launch_bounds__(kStreamThreads) bn_nhwc_stream_apply_kernel(
    const uint16_t* __restrict__ x, BnChan ch, const float* __restrict__ mean, const float* __restrict__ invstd,
    uint16_t* __restrict__ y, NhwcShape sh, float slope, const uint16_t* __restrict__ res, int relu, int* status) {
  constexpr int NIN = RES ? 2 : 1;
  float scale[8], shift[8];
  if (threadIdx.x < kStreamConsumers) {
    const int c0 = int(threadIdx.x % sh.CV) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      scale[e] = __fmul_rn(ld_par(ch.w, ch.pdtype, c0 + e, 1.0f), invstd[c0 + e]);
      shift[e] = __fsub_rn(ld_par(ch.b, ch.pdtype, c0 + e, 0.0f), __fmul_rn(mean[c0 + e], scale[e]));
    }
  }
  const uint4* src[NIN];
  src[0] = reinterpret_cast<const uint4*>(x);
  if constexpr (RES) src[1] = reinterpret_cast<const uint4*>(res);
  uint4* y4 = reinterpret_cast<uint4*>(y);
  const bool rl = relu != 0;
  stream_units<NIN>(src, sh.P * sh.CV, [&](long long u, const uint4(&v)[NIN]) {
    float f[8], r[8];
    unpack8(v[0], f);
    if constexpr (EPI) {
      float q[8];
      if constexpr (RES) unpack8(v[1], q);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        r[e] = bn_tail_fast(__fadd_rn(__fmul_rn(f[e], scale[e]), shift[e]), RES, RES ? q[e] : 0.0f, rl);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = bn_act(f[e], scale[e], shift[e], slope);
    }
    y4[u] = pack8_fast(r);
  }, status);
}

// dx = w*invstd*(dz - k1 - xhat*k2); inputs in ring order dy, x, y.  RC: dz =
// relu_gate(dy) as in the sums kernel (w, b from rc).
template <bool ACT, bool RC = false>
__global__ void __launch_bounds__(kStreamThreads) bn_nhwc_stream_dx_kernel(
    const uint16_t* __restrict__ dy, const uint16_t* __restrict__ y, const uint16_t* __restrict__ x, const void* w,
    int pdtype, const float* __restrict__ mean, const float* __restrict__ invstd, const float* __restrict__ k,
    uint16_t* __restrict__ dx, NhwcShape sh, float slope, int relu, int* status, BnChan rc = BnChan{}) {
  static_assert(!RC || !ACT, "the recomputed ReLU gate is a backward of plain BatchNorm");
  constexpr int NIN = ACT ? 3 : 2;
  float ws[8], mc[8], is[8], k1[8], k2[8], gsc[8], gsh[8];
  if (threadIdx.x < kStreamConsumers) {
    const int c0 = int(threadIdx.x % sh.CV) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = c0 + e;
      ws[e] = __fmul_rn(ld_par(w, pdtype, c, 1.0f), invstd[c]);
      mc[e] = mean[c];
      is[e] = invstd[c];
      k1[e] = k[c];
      k2[e] = k[sh.C + c];
      gsc[e] = gsh[e] = 0.0f;
      if constexpr (RC) {
        gsc[e] = __fmul_rn(ld_par(rc.w, rc.pdtype, c, 1.0f), invstd[c]);
        gsh[e] = __fsub_rn(ld_par(rc.b, rc.pdtype, c, 0.0f), __fmul_rn(mean[c], gsc[e]));
      }
    }
  }
  const uint4* src[NIN];
  src[0] = reinterpret_cast<const uint4*>(dy);
  src[1] = reinterpret_cast<const uint4*>(x);
  if constexpr (ACT) src[2] = reinterpret_cast<const uint4*>(y);
  uint4* d4 = reinterpret_cast<uint4*>(dx);
  stream_units<NIN>(src, sh.P * sh.CV, [&](long long u, const uint4(&v)[NIN]) {
    float fg[8], fy[8], fx[8], r[8];
    unpack8(v[0], fg);
    unpack8(v[1], fx);
    if constexpr (ACT) unpack8(v[NIN - 1], fy);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if constexpr (RC)
        r[e] = bn_dx<false>(relu_gate(fg[e], fx[e], gsc[e], gsh[e]), 0.0f, fx[e], mc[e], is[e], ws[e], k1[e], k2[e],
                            slope, relu);
      else
        r[e] = bn_dx<ACT>(fg[e], ACT ? fy[e] : 0.0f, fx[e], mc[e], is[e], ws[e], k1[e], k2[e], slope, relu);
    }
    d4[u] = pack8_fast(r);
  }, status);
}

// ============================ launchers =====================================

// Warp-per-plane when there are enough planes to fill the GPU with warps,
// else block-per-plane.
bool warp_per_plane(long long planes, int sms) { return planes >= (long long)sms * 32; }

int stats_grid(long long planes, bool warp, int sms) {
  const long long groups = warp ? (planes + kBnThreads / 32 - 1) / (kBnThreads / 32) : planes;
  return int(std::max<long long>(1, std::min<long long>(groups, (long long)sms * 8)));
}

// Blocks of `kfn` resident per SM (cached per kernel and shared-memory size).
int resident_blocks(const void* kfn, size_t smem, int threads = kBnThreads) {
  static std::mutex mu;
  static std::map<std::pair<const void*, size_t>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find({kfn, smem});
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kfn, threads, smem) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 1;
  }
  cache[{kfn, smem}] = n;
  return n;
}

// The shared-memory streaming kernels run unless B2_BN_STREAM=0 (A/B switch),
// for channel counts whose groups divide the consumer threads.
bool stream_ok(const NhwcShape& sh) {
  static const bool on = [] {
    const char* e = std::getenv("B2_BN_STREAM");
    return !e || e[0] != '0';
  }();
  return on && kStreamConsumers % sh.CV == 0;
}

// Raises a streaming kernel's shared-memory limit to `smem` (once per device).
template <typename K>
void allow_smem(K* kfn, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, bool> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(reinterpret_cast<const void*>(kfn), dev);
  if (!done.count(key)) {
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      cudaGetLastError();
    done[key] = true;
  }
}

// Grid of a streaming kernel: one wave of resident CTAs, at most one per
// chunk and at most `cap`; raises the kernel's shared-memory limit first.
template <typename K>
int stream_grid(K* kfn, size_t smem, long long units, int sms, long long cap) {
  allow_smem(kfn, smem);
  const long long chunks = (units + kChunkUnits - 1) / kChunkUnits;
  const long long wave = (long long)sms * resident_blocks(reinterpret_cast<const void*>(kfn), smem, kStreamThreads);
  return int(std::max<long long>(1, std::min({chunks, wave, cap})));
}

// Grid-stride kernels: one full wave of resident blocks (no partial last
// wave), fewer when there is less work.
template <typename K>
int wave_grid(K* kfn, size_t smem, long long units, int sms) {
  const long long want = (units + kBnThreads - 1) / kBnThreads;
  const long long wave = (long long)sms * resident_blocks(reinterpret_cast<const void*>(kfn), smem);
  return int(std::max<long long>(1, std::min(want, wave)));
}

int elem_grid(long long units, int sms) {
  const long long b = (units + kBnThreads - 1) / kBnThreads;
  return int(std::max<long long>(1, std::min<long long>(b, (long long)sms * 16)));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

NhwcShape nhwc_shape(long long N, long long C, long long HW) {
  NhwcShape s;
  s.P = N * HW;
  s.C = int(C);
  s.CV = int(C / 8);
  s.rpb = std::max(1, kBnThreads / std::max(1, s.CV));
  return s;
}

// Partial-sum blocks for the NHWC sums kernels: every active thread sums at
// least ~16 pixels; at most one full wave (`wave`) and kMaxSumBlocks.
long long nhwc_blocks(const NhwcShape& s, long long wave) {
  const long long want = (s.P + (long long)s.rpb * 16 - 1) / ((long long)s.rpb * 16);
  return std::max<long long>(1, std::min<long long>(std::min(want, wave), kMaxSumBlocks));
}

// Upper bound of nhwc_blocks over all waves (sizes the workspace).
long long nhwc_blocks(const NhwcShape& s) {
  const long long want = (s.P + (long long)s.rpb * 16 - 1) / ((long long)s.rpb * 16);
  return std::max<long long>(1, std::min<long long>(want, kMaxSumBlocks));
}

size_t workspace_bytes(long long N, long long C, long long HW, int layout) {
  if (N <= 0 || C <= 0) return 0;
  const long long parts = layout == 0 ? N : nhwc_blocks(nhwc_shape(N, C, HW));
  // two fp32 per (part, channel), then two fp32 per channel
  return align16(2 * size_t(parts) * size_t(C) * sizeof(float)) + align16(2 * size_t(C) * sizeof(float));
}

b2_status check_common(int64_t N, int64_t C, int64_t HW, int layout, const void* ws, size_t ws_bytes,
                       const char* who) {
  if (N < 0 || C < 0 || HW < 0) return set_error(B2_ERR_INVALID, "%s: negative size", who);
  if (layout != 0 && layout != 1) return set_error(B2_ERR_INVALID, "%s: layout must be 0 (NCHW) or 1 (NHWC)", who);
  if (ws_bytes < workspace_bytes(N, C, HW, layout) || (N * C > 0 && !ws) || !aligned16(ws))
    return set_error(B2_ERR_WORKSPACE, "%s: workspace too small or misaligned", who);
  return B2_OK;
}

b2_status check_nhwc(int64_t C, std::initializer_list<const void*> ptrs, const char* who) {
  if (C % 8 != 0 || C > kMaxNhwcChannels)
    return set_error(B2_ERR_UNSUPPORTED, "%s: channels-last needs C %% 8 == 0 and C <= %lld", who,
                     (long long)kMaxNhwcChannels);
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return set_error(B2_ERR_UNSUPPORTED, "%s: channels-last needs 16-byte alignment", who);
  return B2_OK;
}

int current_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  return sm_count(dev);
}

// The statistics passes of the forward (batch mean / invstd, running
// statistics); the output is written by bn_apply.
b2_status bn_stats(const uint16_t* x, int layout, const BnChan& ch, float* mean_out, float* invstd_out, long long N,
                   long long C, long long HW, float eps, float momentum, void* workspace, cudaStream_t st,
                   const char* who) {
  const int sms = current_sms();
  if (layout == 1) {
    B2_TRY(check_nhwc(C, {x}, who));
    const NhwcShape sh = nhwc_shape(N, C, HW);
    float* pa = static_cast<float*>(workspace);
    long long blocks;
    if (stream_ok(sh)) {
      auto kfn = &bn_nhwc_stream_sums_kernel<false, false>;
      constexpr size_t smem = ring_smem_bytes<1>();
      blocks = stream_grid(kfn, smem, sh.P * sh.CV, sms, nhwc_blocks(sh));
      kfn<<<int(blocks), kStreamThreads, smem, st>>>(x, nullptr, nullptr, nullptr, nullptr, sh, 0.0f, 0, pa,
                                                      pa + blocks * C, device_status_ptr(), BnChan{});
    } else {
      const size_t red = 2 * size_t(sh.rpb) * size_t(C) * sizeof(float);
      blocks = nhwc_blocks(sh, (long long)sms * resident_blocks(reinterpret_cast<const void*>(
                                                                    &bn_nhwc_sums_kernel<false, false>), red));
      bn_nhwc_sums_kernel<false, false><<<int(blocks), kBnThreads, red, st>>>(x, nullptr, nullptr, nullptr, nullptr,
                                                                              sh, 0.0f, 0, pa, pa + blocks * C);
    }
    float* pb = pa + blocks * C;
    B2_TRY(check_cuda(cudaGetLastError(), "bn nhwc sums launch"));
    bn_nhwc_stats_kernel<<<int(C), kMergeThreads, 0, st>>>(x, pa, pb, blocks, C, sh.P, eps,
                                                                          momentum, ch, mean_out, invstd_out);
    return check_cuda(cudaGetLastError(), "bn nhwc stats launch");
  }
  const long long planes = N * C;
  float* pm = static_cast<float*>(workspace);
  float* pq = pm + planes;
  const bool vec = HW % 8 == 0 && aligned16(x);
  const bool warp = warp_per_plane(planes, sms);
  const int sg = stats_grid(planes, warp, sms);
  if (warp && vec) bn_plane_stats_kernel<32, true><<<sg, kBnThreads, 0, st>>>(x, planes, HW, pm, pq);
  else if (warp) bn_plane_stats_kernel<32, false><<<sg, kBnThreads, 0, st>>>(x, planes, HW, pm, pq);
  else if (vec) bn_plane_stats_kernel<kBnThreads, true><<<sg, kBnThreads, 0, st>>>(x, planes, HW, pm, pq);
  else bn_plane_stats_kernel<kBnThreads, false><<<sg, kBnThreads, 0, st>>>(x, planes, HW, pm, pq);
  B2_TRY(check_cuda(cudaGetLastError(), "bn stats launch"));
  bn_channel_stats_kernel<<<int((C + 3) / 4), 128, 0, st>>>(pm, pq, N, C, HW, eps, momentum, ch, mean_out,
                                                            invstd_out);
  return check_cuda(cudaGetLastError(), "bn channel launch");
}

// y = act(x*scale + shift) from the statistics; epi: the fused tail with an
// optional residual (x's layout) and ReLU instead of the activation.
template <bool EPI>
b2_status bn_apply_launch(const uint16_t* x, int layout, const BnChan& ch, const float* mean, const float* invstd,
                          uint16_t* y, long long N, long long C, long long HW, float slope, const uint16_t* res,
                          int relu, cudaStream_t st, const char* who) {
  const int sms = current_sms();
  if (layout == 1) {
    B2_TRY(check_nhwc(C, {x, y, res}, who));
    const NhwcShape sh = nhwc_shape(N, C, HW);
    if (stream_ok(sh)) {
      if (EPI && res) {
        auto kfn = &bn_nhwc_stream_apply_kernel<EPI, true>;
        constexpr size_t smem = ring_smem_bytes<2>();
        kfn<<<stream_grid(kfn, smem, sh.P * sh.CV, sms, LLONG_MAX), kStreamThreads, smem, st>>>(
            x, ch, mean, invstd, y, sh, slope, res, relu, device_status_ptr());
      } else {
        auto kfn = &bn_nhwc_stream_apply_kernel<EPI, false>;
        constexpr size_t smem = ring_smem_bytes<1>();
        kfn<<<stream_grid(kfn, smem, sh.P * sh.CV, sms, LLONG_MAX), kStreamThreads, smem, st>>>(
            x, ch, mean, invstd, y, sh, slope, nullptr, relu, device_status_ptr());
      }
    } else if (kBnThreads % sh.CV == 0)
      bn_nhwc_apply_kernel<true, EPI><<<wave_grid(&bn_nhwc_apply_kernel<true, EPI>, 0, sh.P * sh.CV, sms),
                                        kBnThreads, 0, st>>>(x, ch, mean, invstd, y, sh, slope, res, relu);
    else
      bn_nhwc_apply_kernel<false, EPI><<<elem_grid(sh.P * sh.CV, sms), kBnThreads, 2 * C * sizeof(float), st>>>(
          x, ch, mean, invstd, y, sh, slope, res, relu);
    return check_cuda(cudaGetLastError(), "bn nhwc apply launch");
  }
  const long long planes = N * C;
  const bool vec = HW % 8 == 0 && aligned16(x) && aligned16(y) && (!res || aligned16(res));
  if (vec) {
    const long long units = planes * (HW / 8);
    bn_apply_kernel<true, EPI><<<wave_grid(&bn_apply_kernel<true, EPI>, 0, units, sms), kBnThreads, 0, st>>>(
        x, ch, mean, invstd, y, units, HW / 8, C, slope, res, relu);
  } else {
    const long long units = planes * HW;
    bn_apply_kernel<false, EPI><<<elem_grid(units, sms), kBnThreads, 0, st>>>(x, ch, mean, invstd, y, units, HW, C,
                                                                              slope, res, relu);
  }
  return check_cuda(cudaGetLastError(), "bn apply launch");
}

b2_status bn_forward(const uint16_t* x, int layout, const BnChan& ch, uint16_t* y, float* mean_out,
                     float* invstd_out, long long N, long long C, long long HW, float eps, float slope,
                     float momentum, void* workspace, cudaStream_t st, const char* who) {
  if (layout == 1) B2_TRY(check_nhwc(C, {x, y}, who));
  B2_TRY(bn_stats(x, layout, ch, mean_out, invstd_out, N, C, HW, eps, momentum, workspace, st, who));
  return bn_apply_launch<false>(x, layout, ch, mean_out, invstd_out, y, N, C, HW, slope, nullptr, 0, st, who);
}

template <bool ACT>
b2_status bn_backward(const uint16_t* g, const uint16_t* yy, const uint16_t* xx, int layout, const void* w,
                      int pdtype, const float* mean, const float* invstd, uint16_t* dx, void* dw, void* db,
                      int gdtype, long long N, long long C, long long HW, float slope, int relu, void* workspace,
                      cudaStream_t st, const char* who) {
  const int sms = current_sms();
  const double M = double(N) * double(HW);
  if (layout == 1) {
    B2_TRY(check_nhwc(C, {g, yy, xx, dx}, who));
    const NhwcShape sh = nhwc_shape(N, C, HW);
    const bool stream = stream_ok(sh);
    float* pa = static_cast<float*>(workspace);
    long long blocks;
    if (stream) {
      auto kfn = &bn_nhwc_stream_sums_kernel<true, ACT>;
      constexpr size_t smem = ring_smem_bytes<ACT ? 3 : 2>();
      blocks = stream_grid(kfn, smem, sh.P * sh.CV, sms, nhwc_blocks(sh));
      kfn<<<int(blocks), kStreamThreads, smem, st>>>(xx, g, yy, mean, invstd, sh, slope, relu, pa, pa + blocks * C,
                                                      device_status_ptr(), BnChan{});
    } else {
      const size_t red = 2 * size_t(sh.rpb) * size_t(C) * sizeof(float);
      blocks = nhwc_blocks(sh, (long long)sms * resident_blocks(reinterpret_cast<const void*>(
                                                                    &bn_nhwc_sums_kernel<true, ACT>), red));
      bn_nhwc_sums_kernel<true, ACT><<<int(blocks), kBnThreads, red, st>>>(xx, g, yy, mean, invstd, sh, slope, relu,
                                                                           pa, pa + blocks * C);
    }
    float* pb = pa + blocks * C;
    float* k = reinterpret_cast<float*>(static_cast<char*>(workspace) + align16(2 * size_t(blocks) * C * sizeof(float)));
    B2_TRY(check_cuda(cudaGetLastError(), "bn nhwc bwd sums launch"));
    bn_bwd_channel_kernel<<<int(C), kMergeThreads, 0, st>>>(pa, pb, blocks, C, M, dw, db, gdtype, k);
    B2_TRY(check_cuda(cudaGetLastError(), "bn nhwc bwd channel launch"));
    if (!dx) return B2_OK;
    if (stream) {
      auto kfn = &bn_nhwc_stream_dx_kernel<ACT>;
      constexpr size_t smem = ring_smem_bytes<ACT ? 3 : 2>();
      kfn<<<stream_grid(kfn, smem, sh.P * sh.CV, sms, LLONG_MAX), kStreamThreads, smem, st>>>(
          g, yy, xx, w, pdtype, mean, invstd, k, dx, sh, slope, relu, device_status_ptr(), BnChan{});
    } else if (kBnThreads % sh.CV == 0)
      bn_nhwc_dx_kernel<ACT, true><<<wave_grid(&bn_nhwc_dx_kernel<ACT, true>, 0, sh.P * sh.CV, sms), kBnThreads, 0,
                                                                                              st>>>(
          g, yy, xx, w, pdtype, mean, invstd, k, dx, sh, slope, relu);
    else
      bn_nhwc_dx_kernel<ACT, false><<<elem_grid(sh.P * sh.CV, sms), kBnThreads, 5 * C * sizeof(float), st>>>(
          g, yy, xx, w, pdtype, mean, invstd, k, dx, sh, slope, relu);
    return check_cuda(cudaGetLastError(), "bn nhwc dx launch");
  }
  const long long planes = N * C;
  float* ps = static_cast<float*>(workspace);
  float* pt = ps + planes;
  float* k = reinterpret_cast<float*>(static_cast<char*>(workspace) + align16(2 * size_t(planes) * sizeof(float)));
  const bool vec = HW % 8 == 0 && aligned16(g) && (!ACT || aligned16(yy)) && aligned16(xx) && (!dx || aligned16(dx));
  const bool warp = warp_per_plane(planes, sms);
  const int sg = stats_grid(planes, warp, sms);
  if (warp && vec)
    bn_bwd_plane_kernel<32, true, ACT><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW, slope,
                                                                  relu, ps, pt);
  else if (warp)
    bn_bwd_plane_kernel<32, false, ACT><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW, slope,
                                                                   relu, ps, pt);
  else if (vec)
    bn_bwd_plane_kernel<kBnThreads, true, ACT><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW,
                                                                          slope, relu, ps, pt);
  else
    bn_bwd_plane_kernel<kBnThreads, false, ACT><<<sg, kBnThreads, 0, st>>>(g, yy, xx, mean, invstd, planes, C, HW,
                                                                           slope, relu, ps, pt);
  B2_TRY(check_cuda(cudaGetLastError(), "bn bwd plane launch"));
  bn_bwd_channel_kernel<<<int(C), kMergeThreads, 0, st>>>(ps, pt, N, C, M, dw, db, gdtype, k);
  B2_TRY(check_cuda(cudaGetLastError(), "bn bwd channel launch"));
  if (!dx) return B2_OK;
  if (vec) {
    const long long units = planes * (HW / 8);
    bn_bwd_dx_kernel<true, ACT><<<wave_grid(&bn_bwd_dx_kernel<true, ACT>, 0, units, sms), kBnThreads, 0, st>>>(g, yy, xx, w, pdtype, mean, invstd, k,
                                                                             dx, units, HW / 8, C, slope, relu);
  } else {
    const long long units = planes * HW;
    bn_bwd_dx_kernel<false, ACT><<<elem_grid(units, sms), kBnThreads, 0, st>>>(g, yy, xx, w, pdtype, mean, invstd,
                                                                              k, dx, units, HW, C, slope, relu);
  }
  return check_cuda(cudaGetLastError(), "bn dx launch");
}

// Backward of y = relu(bf16(BatchNorm(x))) from dL/dy, channels-last, with
// the ReLU's gate recomputed from x (no y read, no gated-gradient pass).  The
// grid is the plain backward's, so the partial sums -- and dw, db, dx -- are
// bit for bit those of ATen's threshold_backward followed by
// b2_batch_norm_bwd_bf16.
b2_status bn_relu_backward(const uint16_t* g, const uint16_t* xx, const void* w, const void* b, int pdtype,
                           const float* mean, const float* invstd, uint16_t* dx, void* dw, void* db, int gdtype,
                           long long N, long long C, long long HW, void* workspace, cudaStream_t st, const char* who) {
  B2_TRY(check_nhwc(C, {g, xx, dx}, who));
  const NhwcShape sh = nhwc_shape(N, C, HW);
  if (!stream_ok(sh))
    return set_error(B2_ERR_UNSUPPORTED, "%s: needs the streaming kernels (C/8 dividing 256, B2_BN_STREAM on)", who);
  const int sms = current_sms();
  const double M = double(N) * double(HW);
  const BnChan rc{w, b, pdtype, nullptr, nullptr, B2_F32};
  constexpr size_t smem = ring_smem_bytes<2>();
  const long long units = sh.P * sh.CV;
  const long long blocks = stream_grid(&bn_nhwc_stream_sums_kernel<true, false>, smem, units, sms, nhwc_blocks(sh));
  auto sums = &bn_nhwc_stream_sums_kernel<true, false, true>;
  allow_smem(sums, smem);
  float* pa = static_cast<float*>(workspace);
  float* pb = pa + blocks * C;
  sums<<<int(blocks), kStreamThreads, smem, st>>>(xx, g, nullptr, mean, invstd, sh, 0.0f, 0, pa, pb,
                                                  device_status_ptr(), rc);
  B2_TRY(check_cuda(cudaGetLastError(), "bn relu bwd sums launch"));
  float* k = reinterpret_cast<float*>(static_cast<char*>(workspace) + align16(2 * size_t(blocks) * C * sizeof(float)));
  bn_bwd_channel_kernel<<<int(C), kMergeThreads, 0, st>>>(pa, pb, blocks, C, M, dw, db, gdtype, k);
  B2_TRY(check_cuda(cudaGetLastError(), "bn relu bwd channel launch"));
  if (!dx) return B2_OK;
  auto dxk = &bn_nhwc_stream_dx_kernel<false, true>;
  dxk<<<stream_grid(dxk, smem, units, sms, LLONG_MAX), kStreamThreads, smem, st>>>(
      g, nullptr, xx, w, pdtype, mean, invstd, k, dx, sh, 0.0f, 0, device_status_ptr(), rc);
  return check_cuda(cudaGetLastError(), "bn relu dx launch");
}

// Backward of a BatchNorm (channels-last) whose output gradient is the ReLU
// backward of a residual sum: dz = gate(y) ? bf16(a + b) : 0 made, written to
// dz_out and summed in one pass, then the plain merge and dx passes (dx reads
// the dz just written).  The plain backward's grid, so every result is bit for
// bit b2_relu_bwd_sum_bf16 followed by b2_batch_norm_bwd_bf16.
b2_status bn_gsum_backward(const uint16_t* ga, const uint16_t* gb, const uint16_t* yy, const uint16_t* xx,
                           const void* w, int pdtype, const float* mean, const float* invstd, uint16_t* dz_out,
                           uint16_t* dx, void* dw, void* db, int gdtype, long long N, long long C, long long HW,
                           void* workspace, cudaStream_t st, const char* who) {
  B2_TRY(check_nhwc(C, {ga, gb, yy, xx, dz_out, dx}, who));
  const NhwcShape sh = nhwc_shape(N, C, HW);
  if (!stream_ok(sh))
    return set_error(B2_ERR_UNSUPPORTED, "%s: needs the streaming kernels (C/8 dividing 256, B2_BN_STREAM on)", who);
  const int sms = current_sms();
  const double M = double(N) * double(HW);
  const long long units = sh.P * sh.CV;
  constexpr size_t smem2 = ring_smem_bytes<2>();
  const long long blocks = stream_grid(&bn_nhwc_stream_sums_kernel<true, false>, smem2, units, sms, nhwc_blocks(sh));
  auto sums = &bn_nhwc_stream_sums_gsum_kernel;
  constexpr size_t smem4 = ring_smem_bytes<4>();
  allow_smem(sums, smem4);
  float* pa = static_cast<float*>(workspace);
  float* pb = pa + blocks * C;
  sums<<<int(blocks), kStreamThreads, smem4, st>>>(xx, ga, gb, yy, mean, invstd, sh, dz_out, pa, pb,
                                                   device_status_ptr());
  B2_TRY(check_cuda(cudaGetLastError(), "bn gsum sums launch"));
  float* k = reinterpret_cast<float*>(static_cast<char*>(workspace) + align16(2 * size_t(blocks) * C * sizeof(float)));
  bn_bwd_channel_kernel<<<int(C), kMergeThreads, 0, st>>>(pa, pb, blocks, C, M, dw, db, gdtype, k);
  B2_TRY(check_cuda(cudaGetLastError(), "bn gsum channel launch"));
  if (!dx) return B2_OK;
  auto dxk = &bn_nhwc_stream_dx_kernel<false>;
  dxk<<<stream_grid(dxk, smem2, units, sms, LLONG_MAX), kStreamThreads, smem2, st>>>(
      dz_out, nullptr, xx, w, pdtype, mean, invstd, k, dx, sh, 1.0f, 0, device_status_ptr(), BnChan{});
  return check_cuda(cudaGetLastError(), "bn gsum dx launch");
}

bool valid_pdtype(int dt) { return dt == B2_BF16 || dt == B2_F32; }

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

size_t b2_region_bn_workspace_bytes(int64_t N, int64_t C) { return workspace_bytes(N, C, 1, 0); }

size_t b2_batch_norm_workspace_bytes(int64_t N, int64_t C, int64_t HW, int layout) {
  return workspace_bytes(N, C, HW, layout == 1 ? 1 : 0);
}

b2_status b2_region_bn_fwd_bf16(const void* x, const void* w, const void* b, void* rm, void* rv,
                                void* y, float* mean_out, float* invstd_out, int64_t N, int64_t C,
                                int64_t HW, float eps, float slope, float factor, int update,
                                void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "b2_region_bn_fwd_bf16";
  B2_TRY(check_common(N, C, HW, 0, workspace, workspace_bytes, who));
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!x || !y || !mean_out || !invstd_out || (update && (!rm || !rv)))
    return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  const BnChan ch{w, b, B2_BF16, update ? rm : nullptr, update ? rv : nullptr, B2_BF16};
  return bn_forward(static_cast<const uint16_t*>(x), 0, ch, static_cast<uint16_t*>(y), mean_out, invstd_out, N, C,
                    HW, eps, slope, factor, workspace, static_cast<cudaStream_t>(stream), who);
}

b2_status b2_region_bn_bwd_bf16(const void* dy, const void* y, const void* x, const void* w,
                                const float* mean, const float* invstd, void* dx, void* dw, void* db,
                                int64_t N, int64_t C, int64_t HW, float slope, int relu, void* workspace,
                                size_t workspace_bytes, void* stream) {
  const char* who = "b2_region_bn_bwd_bf16";
  B2_TRY(check_common(N, C, HW, 0, workspace, workspace_bytes, who));
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!dy || !y || !x || !mean || !invstd) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  return bn_backward<true>(static_cast<const uint16_t*>(dy), static_cast<const uint16_t*>(y),
                           static_cast<const uint16_t*>(x), 0, w, B2_BF16, mean, invstd,
                           static_cast<uint16_t*>(dx), dw, db, B2_BF16, N, C, HW, slope, relu, workspace,
                           static_cast<cudaStream_t>(stream), who);
}

b2_status b2_batch_norm_fwd_bf16(const void* x, int layout, const void* w, const void* b, int pdtype, void* rm,
                                 void* rv, int rdtype, void* y, float* save_mean, float* save_invstd, int64_t N,
                                 int64_t C, int64_t HW, float momentum, float eps, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  const char* who = "b2_batch_norm_fwd_bf16";
  B2_TRY(check_common(N, C, HW, layout, workspace, workspace_bytes, who));
  if (!valid_pdtype(pdtype) || !valid_pdtype(rdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!x || !y || !save_mean || !save_invstd || (!rm) != (!rv))
    return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  const BnChan ch{w, b, pdtype, rm, rv, rdtype};
  return bn_forward(static_cast<const uint16_t*>(x), layout, ch, static_cast<uint16_t*>(y), save_mean, save_invstd,
                    N, C, HW, eps, 1.0f, momentum, workspace, static_cast<cudaStream_t>(stream), who);
}

b2_status b2_batch_norm_stats_bf16(const void* x, int layout, int pdtype, void* rm, void* rv, int rdtype,
                                   float* save_mean, float* save_invstd, int64_t N, int64_t C, int64_t HW,
                                   float momentum, float eps, void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "b2_batch_norm_stats_bf16";
  B2_TRY(check_common(N, C, HW, layout, workspace, workspace_bytes, who));
  if (!valid_pdtype(pdtype) || !valid_pdtype(rdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!x || !save_mean || !save_invstd || (!rm) != (!rv)) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  const BnChan ch{nullptr, nullptr, pdtype, rm, rv, rdtype};
  return bn_stats(static_cast<const uint16_t*>(x), layout, ch, save_mean, save_invstd, N, C, HW, eps, momentum,
                  workspace, static_cast<cudaStream_t>(stream), who);
}

b2_status b2_batch_norm_stats_count_bf16(const void* x, int layout, int pdtype, void* rm, void* rv, int rdtype,
                                         float* save_mean, float* save_invstd, int64_t N, int64_t C, int64_t HW,
                                         float momentum, float eps, int64_t* count, int64_t count_inc,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "b2_batch_norm_stats_count_bf16";
  B2_TRY(check_common(N, C, HW, layout, workspace, workspace_bytes, who));
  if (!valid_pdtype(pdtype) || !valid_pdtype(rdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (!count || (reinterpret_cast<uintptr_t>(count) & 7)) return set_error(B2_ERR_INVALID, "%s: counter", who);
  if (N * C == 0 || HW == 0) return set_error(B2_ERR_INVALID, "%s: empty input (nothing would advance the counter)", who);
  if (!x || !save_mean || !save_invstd || (!rm) != (!rv)) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  BnChan ch{nullptr, nullptr, pdtype, rm, rv, rdtype};
  ch.count = reinterpret_cast<long long*>(count);
  ch.count_inc = count_inc;
  return bn_stats(static_cast<const uint16_t*>(x), layout, ch, save_mean, save_invstd, N, C, HW, eps, momentum,
                  workspace, static_cast<cudaStream_t>(stream), who);
}

b2_status b2_batch_norm_apply_bf16(const void* x, int layout, const void* w, const void* b, int pdtype,
                                   const float* mean, const float* invstd, const void* residual, int relu, void* y,
                                   int64_t N, int64_t C, int64_t HW, void* stream) {
  const char* who = "b2_batch_norm_apply_bf16";
  if (layout != 0 && layout != 1) return set_error(B2_ERR_INVALID, "%s: layout", who);
  if (N < 0 || C < 0 || HW < 0) return set_error(B2_ERR_INVALID, "%s: negative size", who);
  if (!valid_pdtype(pdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (N * C * HW == 0) return B2_OK;
  if (!x || !y || !mean || !invstd) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  const BnChan ch{w, b, pdtype, nullptr, nullptr, B2_F32};
  auto st = static_cast<cudaStream_t>(stream);
  auto* xp = static_cast<const uint16_t*>(x);
  auto* yp = static_cast<uint16_t*>(y);
  auto* rp = static_cast<const uint16_t*>(residual);
  if (!residual && !relu) return bn_apply_launch<false>(xp, layout, ch, mean, invstd, yp, N, C, HW, 1.0f, nullptr, 0, st, who);
  return bn_apply_launch<true>(xp, layout, ch, mean, invstd, yp, N, C, HW, 1.0f, rp, relu, st, who);
}

b2_status b2_batch_norm_bwd_bf16(const void* dy, const void* x, int layout, const void* w, int pdtype,
                                 const float* save_mean, const float* save_invstd, void* dx, void* dw, void* db,
                                 int gdtype, int64_t N, int64_t C, int64_t HW, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  const char* who = "b2_batch_norm_bwd_bf16";
  B2_TRY(check_common(N, C, HW, layout, workspace, workspace_bytes, who));
  if (!valid_pdtype(pdtype) || !valid_pdtype(gdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!dy || !x || !save_mean || !save_invstd) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  return bn_backward<false>(static_cast<const uint16_t*>(dy), nullptr, static_cast<const uint16_t*>(x), layout, w,
                            pdtype, save_mean, save_invstd, static_cast<uint16_t*>(dx), dw, db, gdtype, N, C, HW,
                            1.0f, 0, workspace, static_cast<cudaStream_t>(stream), who);
}

}  // extern "C"

extern "C" b2_status b2_batch_norm_relu_bwd_bf16(const void* dy, const void* x, const void* w, const void* b,
                                                 int pdtype, const float* save_mean, const float* save_invstd,
                                                 void* dx, void* dw, void* db, int gdtype, int64_t N, int64_t C,
                                                 int64_t HW, void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "b2_batch_norm_relu_bwd_bf16";
  B2_TRY(check_common(N, C, HW, 1, workspace, workspace_bytes, who));
  if (!valid_pdtype(pdtype) || !valid_pdtype(gdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!dy || !x || !save_mean || !save_invstd) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  return bn_relu_backward(static_cast<const uint16_t*>(dy), static_cast<const uint16_t*>(x), w, b, pdtype, save_mean,
                          save_invstd, static_cast<uint16_t*>(dx), dw, db, gdtype, N, C, HW, workspace,
                          static_cast<cudaStream_t>(stream), who);
}

extern "C" b2_status b2_batch_norm_bwd_relu_sum_bf16(const void* a, const void* b, const void* y, const void* x,
                                                     const void* w, int pdtype, const float* save_mean,
                                                     const float* save_invstd, void* dz, void* dx, void* dw, void* db,
                                                     int gdtype, int64_t N, int64_t C, int64_t HW, void* workspace,
                                                     size_t workspace_bytes, void* stream) {
  const char* who = "b2_batch_norm_bwd_relu_sum_bf16";
  B2_TRY(check_common(N, C, HW, 1, workspace, workspace_bytes, who));
  if (!valid_pdtype(pdtype) || !valid_pdtype(gdtype)) return set_error(B2_ERR_UNSUPPORTED, "%s: parameter dtype", who);
  if (N * C == 0) return B2_OK;
  if (HW == 0) return set_error(B2_ERR_INVALID, "%s: empty planes", who);
  if (!a || !b || !y || !x || !dz || !save_mean || !save_invstd) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  return bn_gsum_backward(static_cast<const uint16_t*>(a), static_cast<const uint16_t*>(b),
                          static_cast<const uint16_t*>(y), static_cast<const uint16_t*>(x), w, pdtype, save_mean,
                          save_invstd, static_cast<uint16_t*>(dz), static_cast<uint16_t*>(dx), dw, db, gdtype, N, C,
                          HW, workspace, static_cast<cudaStream_t>(stream), who);
}
