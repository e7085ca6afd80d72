// Layout kernels of the general convolution path (any kernel size, stride,
// padding and dilation; groups 1): the convolution runs as tcgen05 GEMMs over
// an explicit column matrix.  The reference runs every convolution other than
// its 3x3 fast path on its CPU (torch_xdna_device.cpp:4578-4605, 4828-4878).
//
//   col    [P][Kp] bf16, P = B*Ho*Wo output pixels in (b, oy, ox) order; column
//          k = (ky*kw + kx)*Cin + ci for k < K = kh*kw*Cin, zero for K <= k < Kp
//          (Kp = K rounded up to 8: 16-byte rows for TMA); taps outside the
//          input read zero.
//   Wk     [Cout][Kp] bf16, the weight in the same (ky, kx, ci) order.
//   dcol   [P][Kp] fp32 (dY . Wk); col2im sums, for every input element, its
//          taps in (ky, kx) order -- a gather, no atomics: deterministic.
//
// Tensors are addressed through element strides, so NCHW and channels-last
// inputs and outputs need no transposition.  All HBM-bound; with channels-last
// input and Cin % 8 == 0 the column copy moves 16-byte channel vectors.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kColThreads = 256;

struct ConvGeom {
  long long B, C, H, W;       // input
  long long sb, sc, sh, sw;   // input (or dX) element strides
  int kh, kw, sy, sx, py, px, dy, dx;
  long long Ho, Wo, K, Kp;
};

int col_grid(long long units, int sms) {
  const long long b = (units + kColThreads - 1) / kColThreads;
  return int(std::max<long long>(1, std::min<long long>(b, (long long)sms * 16)));
}

// Generic column copy: one warp per pixel row (grid-stride over rows), lanes
// over the row's columns (coalesced stores).  The per-column offsets are packed
// into one word each in shared memory -- ky*dy (8 bits), kx*dx (8 bits), ci
// (16 bits) -- so an element costs one shared load, a bounds test, one global
// load and one store; the row's origin is computed once per row.
constexpr int kMaxTabK = 8192;

__global__ void __launch_bounds__(kColThreads) im2col_kernel(const uint16_t* __restrict__ x, ConvGeom g,
                                                             uint16_t* __restrict__ col) {
  __shared__ uint32_t tab[kMaxTabK];
  const int K = int(g.K), Kp = int(g.Kp);
  for (int k = threadIdx.x; k < K; k += kColThreads) {
    const int ci = k % int(g.C), tap = k / int(g.C);
    tab[k] = uint32_t((tap / g.kw) * g.dy) | (uint32_t((tap % g.kw) * g.dx) << 8) | (uint32_t(ci) << 16);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long P = g.B * g.Ho * g.Wo;
  const long long warps = (long long)gridDim.x * (kColThreads / 32);
  const uint32_t Wo = uint32_t(g.Wo), Ho = uint32_t(g.Ho);  // P < 2^31: 32-bit division is exact
  for (long long p = (long long)blockIdx.x * (kColThreads / 32) + (threadIdx.x >> 5); p < P; p += warps) {
    const uint32_t pu = uint32_t(p), q = pu / Wo;
    const uint32_t ox = pu - q * Wo, oy = q % Ho, b = q / Ho;
    const int y0 = int(oy) * g.sy - g.py, x0 = int(ox) * g.sx - g.px;
    const uint16_t* xb = x + (long long)b * g.sb;
    uint16_t* dst = col + p * Kp;
    for (int k = lane; k < Kp; k += 32) {
      uint16_t v = 0;
      if (k < K) {
        const uint32_t t = tab[k];
        const int iy = y0 + int(t & 0xffu), ix = x0 + int((t >> 8) & 0xffu);
        if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W)
          v = xb[(long long)(t >> 16) * g.sc + (long long)iy * g.sh + (long long)ix * g.sw];
      }
      dst[k] = v;
    }
  }
}

// Column copy by output rows through shared memory: a CTA takes one output
// row (b, oy) at a time and stages the kh input rows its windows read -- zero
// padded left and right, zero rows outside the image -- as [kh][Wpad][C]
// (Wpad = W + 2*px), twice: as bf16 elements and as 32-bit pairs (element e
// and e + 1), so that two adjacent columns that read adjacent elements (the
// same window row) cost one 4-byte shared load.  Thread t keeps column
// chunk j = t % J (8 columns, J = Kp / 8) for the whole kernel -- its eight
// element offsets and which of its four column pairs are adjacent sit in
// registers -- and writes that chunk for pixels ox = t / J, t / J + 256 / J,
// ... of each row as one 16-byte store.  For a stem (3 channels, 7x7) the
// input is read once per output row and a 16-byte chunk costs about four
// shared loads.
constexpr int kRowTileMaxBytes = 48 * 1024;

__global__ void __launch_bounds__(kColThreads) im2col_rowtile_kernel(const uint16_t* __restrict__ x, ConvGeom g,
                                                                     uint16_t* __restrict__ col) {
  extern __shared__ __align__(16) uint8_t rt_smem[];
  const int K = int(g.K), Kp = int(g.Kp), C = int(g.C), kh = g.kh;
  const int Wpad = int(g.W) + 2 * g.px;
  const int rowlen = Wpad * C;  // elements of one staged input row
  const int staged = kh * rowlen;
  uint32_t* pairs = reinterpret_cast<uint32_t*>(rt_smem);
  uint16_t* stage = reinterpret_cast<uint16_t*>(rt_smem + size_t(staged) * 4);
  const int Wo = int(g.Wo), J = Kp / 8, L = kColThreads / J;
  const int j = int(threadIdx.x) % J, lane = int(threadIdx.x) / J;
  // this thread's eight columns: element offsets in the stage (-1: zero)
  int o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int k = j * 8 + e;
    if (k < K) {
      const int ci = k % C, tap = k / C;
      o[e] = (tap / g.kw) * rowlen + (tap % g.kw) * g.dx * C + ci;
    } else {
      o[e] = -1;
    }
  }
  bool adj[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) adj[h] = o[2 * h] >= 0 && o[2 * h + 1] == o[2 * h] + 1;
  // channels-last input rows dense and 16-byte aligned: vector staging
  const bool dense = g.sc == 1 && g.sw == g.C && (g.W * g.C) % 8 == 0 && g.sh % 8 == 0 && g.sb % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const long long rows = g.B * g.Ho;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const int oy = int(r % g.Ho);
    const long long b = r / g.Ho;
    const uint16_t* xb = x + b * g.sb;
    __syncthreads();  // the previous row's reads of the stage are done
    if (dense) {
      // each input row is W*C contiguous elements: 16-byte loads, the zero
      // padding columns and the rows outside the image written as zeros
      const int pad = g.px * C, vr = int(g.W) * C / 8;
      for (int e = threadIdx.x; e < kh * vr; e += kColThreads) {
        const int ky = e / vr, q = e - ky * vr;
        const int iy = oy * g.sy - g.py + ky * g.dy;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (iy >= 0 && iy < g.H) v = __ldg(reinterpret_cast<const uint4*>(xb + (long long)iy * g.sh) + q);
        uint16_t* d = stage + ky * rowlen + pad + q * 8;
        const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          d[2 * h] = uint16_t(wd[h] & 0xffffu);
          d[2 * h + 1] = uint16_t(wd[h] >> 16);
        }
      }
      for (int e = threadIdx.x; e < kh * 2 * pad; e += kColThreads) {
        const int ky = e / (2 * pad), t = e - ky * 2 * pad;
        stage[ky * rowlen + (t < pad ? t : rowlen - 2 * pad + t)] = 0;
      }
    } else {
      for (int e = threadIdx.x; e < staged; e += kColThreads) {
        const int ky = e / rowlen, rem = e - ky * rowlen;
        const int ixp = rem / C, ci = rem - ixp * C;
        const int iy = oy * g.sy - g.py + ky * g.dy, ix = ixp - g.px;
        uint16_t v = 0;
        if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W)
          v = __ldg(xb + (long long)ci * g.sc + (long long)iy * g.sh + (long long)ix * g.sw);
        stage[e] = v;
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < staged; e += kColThreads)
      pairs[e] = uint32_t(stage[e]) | (e + 1 < staged ? uint32_t(stage[e + 1]) << 16 : 0u);
    __syncthreads();
    if (lane >= L) continue;
    uint16_t* dst = col + r * (long long)Wo * Kp + j * 8;
    for (int ox = lane; ox < Wo; ox += L) {
      const int base = ox * g.sx * C;
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        if (adj[h]) {
          w[h] = pairs[base + o[2 * h]];
        } else {
          const uint32_t lo = o[2 * h] >= 0 ? stage[base + o[2 * h]] : 0u;
          const uint32_t hi = o[2 * h + 1] >= 0 ? stage[base + o[2 * h + 1]] : 0u;
          w[h] = lo | (hi << 16);
        }
      }
      *reinterpret_cast<uint4*>(dst + (long long)ox * Kp) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

size_t rowtile_smem(const ConvGeom& g) {
  return size_t(g.kh) * size_t(g.W + 2 * g.px) * size_t(g.C) * 6;  // pairs (4 B) and elements (2 B)
}

// Fallback for K > kMaxTabK: one thread per column element.
// Column copy in 16-byte chunks: thread u writes columns 8j..8j+7 of pixel
// row p (u = p * Kp/8 + j), so a warp's stores cover consecutive chunks of
// consecutive rows; its eight elements are gathered one by one through the
// packed offset table (any channel count: the stems' 3 input channels leave no
// wider unit to copy).  Needs P * Kp / 8 < 2^31.
__global__ void __launch_bounds__(kColThreads) im2col_chunk8_kernel(const uint16_t* __restrict__ x, ConvGeom g,
                                                                    uint16_t* __restrict__ col) {
  __shared__ uint32_t tab[kMaxTabK];
  const int K = int(g.K), Kp = int(g.Kp);
  for (int k = threadIdx.x; k < Kp; k += kColThreads) {
    if (k < K) {
      const int ci = k % int(g.C), tap = k / int(g.C);
      tab[k] = uint32_t((tap / g.kw) * g.dy) | (uint32_t((tap % g.kw) * g.dx) << 8) | (uint32_t(ci) << 16);
    } else {
      tab[k] = 0xffffffffu;  // padding column: zero
    }
  }
  __syncthreads();
  const uint32_t J = uint32_t(Kp / 8), Wo = uint32_t(g.Wo), Ho = uint32_t(g.Ho);
  const uint32_t total = uint32_t(g.B * g.Ho * g.Wo) * J;
  const int H = int(g.H), W = int(g.W);
  for (uint32_t u = blockIdx.x * kColThreads + threadIdx.x; u < total; u += gridDim.x * kColThreads) {
    const uint32_t p = u / J, j = u - p * J;
    const uint32_t q = p / Wo;
    const uint32_t ox = p - q * Wo, oy = q % Ho, b = q / Ho;
    const int y0 = int(oy) * g.sy - g.py, x0 = int(ox) * g.sx - g.px;
    const uint16_t* xb = x + (long long)b * g.sb;
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t lo = 0, hi = 0;
      const uint32_t t0 = tab[j * 8 + 2 * h], t1 = tab[j * 8 + 2 * h + 1];
      if (t0 != 0xffffffffu) {
        const int iy = y0 + int(t0 & 0xffu), ix = x0 + int((t0 >> 8) & 0xffu);
        if (iy >= 0 && iy < H && ix >= 0 && ix < W)
          lo = __ldg(xb + (long long)(t0 >> 16) * g.sc + (long long)iy * g.sh + (long long)ix * g.sw);
      }
      if (t1 != 0xffffffffu) {
        const int iy = y0 + int(t1 & 0xffu), ix = x0 + int((t1 >> 8) & 0xffu);
        if (iy >= 0 && iy < H && ix >= 0 && ix < W)
          hi = __ldg(xb + (long long)(t1 >> 16) * g.sc + (long long)iy * g.sh + (long long)ix * g.sw);
      }
      w[h] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(col + (long long)p * Kp + j * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void __launch_bounds__(kColThreads) im2col_flat_kernel(const uint16_t* __restrict__ x, ConvGeom g,
                                                                  uint16_t* __restrict__ col) {
  const long long total = g.B * g.Ho * g.Wo * g.Kp;
  for (long long u = (long long)blockIdx.x * kColThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kColThreads) {
    const long long p = u / g.Kp, k = u - p * g.Kp;
    uint16_t v = 0;
    if (k < g.K) {
      const long long ci = k % g.C, tap = k / g.C;
      const int ky = int(tap / g.kw), kx = int(tap % g.kw);
      const long long ox = p % g.Wo, oy = (p / g.Wo) % g.Ho, b = p / (g.Wo * g.Ho);
      const long long iy = oy * g.sy - g.py + (long long)ky * g.dy;
      const long long ix = ox * g.sx - g.px + (long long)kx * g.dx;
      if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W) v = x[b * g.sb + ci * g.sc + iy * g.sh + ix * g.sw];
    }
    col[u] = v;
  }
}

// Channels-last input, C % 8 == 0: one thread per 8 channels of one tap of
// one pixel (K = kh*kw*C is then a multiple of 8, so Kp == K).
__global__ void __launch_bounds__(kColThreads) im2col_nhwc8_kernel(const uint16_t* __restrict__ x, ConvGeom g,
                                                                   uint16_t* __restrict__ col) {
  const long long cv = g.C / 8;
  const long long taps = (long long)g.kh * g.kw;
  const long long total = g.B * g.Ho * g.Wo * taps * cv;
  for (long long u = (long long)blockIdx.x * kColThreads + threadIdx.x; u < total;
       u += (long long)gridDim.x * kColThreads) {
    const long long q = u % cv, r = u / cv;
    const long long tap = r % taps, p = r / taps;
    const int ky = int(tap / g.kw), kx = int(tap % g.kw);
    const long long ox = p % g.Wo, oy = (p / g.Wo) % g.Ho, b = p / (g.Wo * g.Ho);
    const long long iy = oy * g.sy - g.py + (long long)ky * g.dy;
    const long long ix = ox * g.sx - g.px + (long long)kx * g.dx;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W)
      v = *reinterpret_cast<const uint4*>(x + b * g.sb + iy * g.sh + ix * g.sw + q * 8);
    reinterpret_cast<uint4*>(col)[u] = v;  // col row p, columns tap*C + 8q .. +8
  }
}

// dX[b, ci, y, x] = sum over (ky, kx) in order of dcol[p(oy, ox)][tap*C + ci]
// where y = oy*sy - py + ky*dy (and the same for x); one thread per element.
template <typename I>  // index type: 32-bit when every index fits
__global__ void __launch_bounds__(kColThreads) col2im_kernel(const float* __restrict__ dcol, ConvGeom g,
                                                             uint16_t* __restrict__ dxo) {
  const long long total = g.B * g.C * g.H * g.W;
  const I C = I(g.C), Wd = I(g.W), Hd = I(g.H);
  for (long long u0 = (long long)blockIdx.x * kColThreads + threadIdx.x; u0 < total;
       u0 += (long long)gridDim.x * kColThreads) {
    // channels innermost: neighbouring threads read neighbouring dcol columns
    const I u = I(u0);
    const I r = u / C, ci = u - r * C;
    const I q = r / Wd;
    const long long x = r - q * Wd, y = q % Hd, b = q / Hd;
    float s = 0.0f;
    for (int ky = 0; ky < g.kh; ++ky) {
      const long long ty = y + g.py - (long long)ky * g.dy;
      if (ty < 0 || ty % g.sy) continue;
      const long long oy = ty / g.sy;
      if (oy >= g.Ho) continue;
      for (int kx = 0; kx < g.kw; ++kx) {
        const long long tx = x + g.px - (long long)kx * g.dx;
        if (tx < 0 || tx % g.sx) continue;
        const long long ox = tx / g.sx;
        if (ox >= g.Wo) continue;
        const long long p = (b * g.Ho + oy) * g.Wo + ox;
        s = __fadd_rn(s, dcol[p * g.Kp + (long long)(ky * g.kw + kx) * g.C + ci]);
      }
    }
    dxo[b * g.sb + ci * g.sc + y * g.sh + x * g.sw] = f2bf(s);
  }
}

// Wk[co][(ky*kw + kx)*Cin + ci] = w[co][ci][ky][kx] (OIHW, contiguous), zero pad.
__global__ void pack_weight_khwc_kernel(const uint16_t* __restrict__ w, long long Cout, long long Cin, int kh, int kw,
                                        long long Kp, uint16_t* __restrict__ wk) {
  const long long K = (long long)kh * kw * Cin;
  const long long total = Cout * Kp;
  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < total;
       u += (long long)gridDim.x * blockDim.x) {
    const long long co = u / Kp, k = u - co * Kp;
    uint16_t v = 0;
    if (k < K) {
      const long long ci = k % Cin, tap = k / Cin;
      v = w[((co * Cin + ci) * kh + tap / kw) * kw + tap % kw];
    }
    wk[u] = v;
  }
}

// dw[co][ci][ky][kx] = dwk[co][(ky*kw + kx)*Cin + ci] (fp32 -> dtype).
__global__ void unpack_weight_khwc_kernel(const float* __restrict__ dwk, long long Cout, long long Cin, int kh, int kw,
                                          long long Kp, void* dw, int dtype) {
  const long long total = Cout * Cin * kh * kw;
  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < total;
       u += (long long)gridDim.x * blockDim.x) {
    const long long kx = u % kw, ky = (u / kw) % kh, ci = (u / ((long long)kw * kh)) % Cin,
                    co = u / ((long long)kw * kh * Cin);
    const float v = dwk[co * Kp + (ky * kw + kx) * Cin + ci];
    if (dtype == B2_F32) static_cast<float*>(dw)[u] = v;
    else static_cast<uint16_t*>(dw)[u] = f2bf(v);
  }
}

b2_status make_geom(ConvGeom& g, int64_t B, int64_t C, int64_t H, int64_t W, int64_t sb, int64_t sc, int64_t sh,
                    int64_t sw, int kh, int kw, int sy, int sx, int py, int px, int dy, int dx, int64_t Ho,
                    int64_t Wo, int64_t Kp, const char* who) {
  if (B < 0 || C <= 0 || H < 0 || W < 0 || kh <= 0 || kw <= 0 || sy <= 0 || sx <= 0 || py < 0 || px < 0 ||
      dy <= 0 || dx <= 0 || Ho < 0 || Wo < 0)
    return set_error(B2_ERR_INVALID, "%s: bad geometry", who);
  if (Ho != (H + 2 * py - (int64_t)dy * (kh - 1) - 1) / sy + 1 || Wo != (W + 2 * px - (int64_t)dx * (kw - 1) - 1) / sx + 1)
    return set_error(B2_ERR_INVALID, "%s: output size does not match the geometry", who);
  const int64_t K = (int64_t)kh * kw * C;
  if (Kp < K || Kp % 8) return set_error(B2_ERR_INVALID, "%s: Kp must be >= kh*kw*C and a multiple of 8", who);
  g = ConvGeom{B, C, H, W, sb, sc, sh, sw, kh, kw, sy, sx, py, px, dy, dx, Ho, Wo, K, Kp};
  return B2_OK;
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

b2_status b2_im2col_bf16(const void* x, int64_t sb, int64_t sc, int64_t sh, int64_t sw, int64_t B, int64_t C,
                         int64_t H, int64_t W, int kh, int kw, int sy, int sx, int py, int px, int dy, int dx,
                         int64_t Ho, int64_t Wo, int64_t Kp, void* col, void* stream) {
  ConvGeom g;
  B2_TRY(make_geom(g, B, C, H, W, sb, sc, sh, sw, kh, kw, sy, sx, py, px, dy, dx, Ho, Wo, Kp, "b2_im2col_bf16"));
  const long long P = B * Ho * Wo;
  if (P == 0) return B2_OK;
  if (!x || !col) return set_error(B2_ERR_INVALID, "b2_im2col_bf16: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  const int sms = cur_sms();
  const bool vec = sc == 1 && C % 8 == 0 && Kp == g.K && sw % 8 == 0 && sh % 8 == 0 && sb % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(col) & 15) == 0;
  if (vec) {
    const long long units = P * kh * kw * (C / 8);
    im2col_nhwc8_kernel<<<col_grid(units, sms), kColThreads, 0, st>>>(static_cast<const uint16_t*>(x), g,
                                                                      static_cast<uint16_t*>(col));
  } else if (g.Kp % 8 == 0 && (reinterpret_cast<uintptr_t>(col) & 15) == 0 && g.Kp / 8 <= kColThreads &&
             rowtile_smem(g) <= size_t(kRowTileMaxBytes) && g.Wo * (g.Kp / 8) < (1LL << 31)) {
    const size_t smem = rowtile_smem(g);
    const long long rows = B * Ho;
    const int grid = int(std::max<long long>(1, std::min<long long>(rows, (long long)sms * 8)));
    im2col_rowtile_kernel<<<grid, kColThreads, smem, st>>>(static_cast<const uint16_t*>(x), g,
                                                           static_cast<uint16_t*>(col));
  } else if (g.Kp <= kMaxTabK && g.Kp % 8 == 0 && g.C < 65536 && (long long)(g.kh - 1) * g.dy < 256 &&
             (long long)(g.kw - 1) * g.dx < 256 && P * (g.Kp / 8) < (1LL << 31) && H + 2 * py < (1LL << 30) &&
             W + 2 * px < (1LL << 30) && (reinterpret_cast<uintptr_t>(col) & 15) == 0) {
    im2col_chunk8_kernel<<<col_grid(P * (g.Kp / 8), sms), kColThreads, 0, st>>>(static_cast<const uint16_t*>(x), g,
                                                                                static_cast<uint16_t*>(col));
  } else if (g.K <= kMaxTabK && g.C < 65536 && (long long)(g.kh - 1) * g.dy < 256 &&
             (long long)(g.kw - 1) * g.dx < 256 && P < (1LL << 31) && H + 2 * py < (1LL << 30) &&
             W + 2 * px < (1LL << 30)) {
    const long long blocks = (P + kColThreads / 32 - 1) / (kColThreads / 32);
    const int grid = int(std::max<long long>(1, std::min<long long>(blocks, (long long)sms * 8)));
    im2col_kernel<<<grid, kColThreads, 0, st>>>(static_cast<const uint16_t*>(x), g, static_cast<uint16_t*>(col));
  } else {
    im2col_flat_kernel<<<col_grid(P * Kp, sms), kColThreads, 0, st>>>(static_cast<const uint16_t*>(x), g,
                                                                      static_cast<uint16_t*>(col));
  }
  return check_cuda(cudaGetLastError(), "im2col launch");
}

b2_status b2_col2im_bf16(const float* dcol, int64_t Kp, int64_t B, int64_t C, int64_t H, int64_t W, int kh, int kw,
                         int sy, int sx, int py, int px, int dy, int dx, int64_t Ho, int64_t Wo, void* dx_out,
                         int64_t sb, int64_t sc, int64_t sh, int64_t sw, void* stream) {
  ConvGeom g;
  B2_TRY(make_geom(g, B, C, H, W, sb, sc, sh, sw, kh, kw, sy, sx, py, px, dy, dx, Ho, Wo, Kp, "b2_col2im_bf16"));
  const long long total = B * C * H * W;
  if (total == 0) return B2_OK;
  if (!dcol || !dx_out) return set_error(B2_ERR_INVALID, "b2_col2im_bf16: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  if (total < (1LL << 31))
    col2im_kernel<uint32_t><<<col_grid(total, cur_sms()), kColThreads, 0, st>>>(dcol, g,
                                                                                static_cast<uint16_t*>(dx_out));
  else
    col2im_kernel<unsigned long long><<<col_grid(total, cur_sms()), kColThreads, 0, st>>>(
        dcol, g, static_cast<uint16_t*>(dx_out));
  return check_cuda(cudaGetLastError(), "col2im launch");
}

b2_status b2_pack_weight_khwc_bf16(const void* w, int64_t Cout, int64_t Cin, int kh, int kw, int64_t Kp, void* wk,
                                   void* stream) {
  if (Cout < 0 || Cin <= 0 || kh <= 0 || kw <= 0 || Kp < (int64_t)kh * kw * Cin || Kp % 8)
    return set_error(B2_ERR_INVALID, "b2_pack_weight_khwc_bf16: bad sizes");
  if (Cout == 0) return B2_OK;
  if (!w || !wk) return set_error(B2_ERR_INVALID, "b2_pack_weight_khwc_bf16: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  pack_weight_khwc_kernel<<<col_grid(Cout * Kp, cur_sms()), kColThreads, 0, st>>>(
      static_cast<const uint16_t*>(w), Cout, Cin, kh, kw, Kp, static_cast<uint16_t*>(wk));
  return check_cuda(cudaGetLastError(), "pack_weight_khwc launch");
}

b2_status b2_unpack_weight_khwc(const float* dwk, int64_t Cout, int64_t Cin, int kh, int kw, int64_t Kp, void* dw,
                                int dtype, void* stream) {
  if (Cout < 0 || Cin <= 0 || kh <= 0 || kw <= 0 || Kp < (int64_t)kh * kw * Cin)
    return set_error(B2_ERR_INVALID, "b2_unpack_weight_khwc: bad sizes");
  if (dtype != B2_BF16 && dtype != B2_F32) return set_error(B2_ERR_INVALID, "b2_unpack_weight_khwc: dtype");
  if (Cout == 0) return B2_OK;
  if (!dwk || !dw) return set_error(B2_ERR_INVALID, "b2_unpack_weight_khwc: null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  unpack_weight_khwc_kernel<<<col_grid(Cout * Cin * kh * kw, cur_sms()), kColThreads, 0, st>>>(dwk, Cout, Cin, kh,
                                                                                               kw, Kp, dw, dtype);
  return check_cuda(cudaGetLastError(), "unpack_weight_khwc launch");
}

}  // extern "C"
