// Layout packers: strided bf16 activations -> padded-grid rows, OIHW weights
// -> K-ordered GEMM operands (forward and dgrad), and dense NCHW <-> NHWC.
// All of them move bf16 bit patterns unchanged (bit-exact copies), staged
// through shared memory so that both the global reads and the 16-byte global
// writes are coalesced.
//
// Reference layouts: xdna_train/_designs/conv3x3w_host.py:32-78 and
// xdna_train/_native/conv_pack.cpp:352-443, 470-519.
#include <algorithm>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kCh = 64;   // channels per tile (one chunk)

// Generic strided packer: one thread per 16-byte output vector (8 channels of
// one padded pixel), threads of a warp on consecutive pixels of the same
// channel group, so each of a thread's 8 element loads is coalesced across
// the warp whenever pixels are the contiguous axis.  No shared memory and a
// thread per vector: small images (9 x 9 planes, ragged widths) get a full
// grid.  Border pixels are the trailing index range.
__global__ void __launch_bounds__(256) pack_rows_kernel(const uint16_t* __restrict__ x, long long sn,
                                                        long long sc, long long sh, long long sw,
                                                        int B, int C, int H, int W, int chunks,
                                                        uint16_t* __restrict__ rows) {
  const int wp = W + 2;
  const long long cpad = (long long)chunks * kCh;
  const int hw = H * W;
  const int groups = chunks * 8;  // 8-channel groups per pixel
  const long long interior = (long long)B * groups * hw;
  const int nb = 2 * wp + 2 * H;  // border pixels per image
  const long long total = interior + (long long)B * nb * groups;
  for (long long u = (long long)blockIdx.x * 256 + threadIdx.x; u < total; u += (long long)gridDim.x * 256) {
    if (u < interior) {
      const int p = int(u % hw);
      const long long r = u / hw;
      const int g = int(r % groups);
      const int b = int(r / groups);
      const int y = p / W, xx = p - y * W;
      const int c0 = g * 8;
      const uint16_t* src = x + b * sn + (long long)y * sh + (long long)xx * sw + (long long)c0 * sc;
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t lo = c0 + 2 * k < C ? src[(long long)(2 * k) * sc] : 0u;
        const uint32_t hi = c0 + 2 * k + 1 < C ? src[(long long)(2 * k + 1) * sc] : 0u;
        w[k] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4*>(rows + (((long long)b * (H + 2) + y + 1) * wp + xx + 1) * cpad + c0) =
          make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      const long long v = u - interior;
      const int g = int(v % groups);
      const long long r = v / groups;
      const int k = int(r % nb);
      const int b = int(r / nb);
      int yp, xp;
      if (k < wp) {
        yp = 0;
        xp = k;
      } else if (k < 2 * wp) {
        yp = H + 1;
        xp = k - wp;
      } else {
        const int j = k - 2 * wp;
        yp = 1 + (j >> 1);
        xp = (j & 1) ? W + 1 : 0;
      }
      *reinterpret_cast<uint4*>(rows + (((long long)b * (H + 2) + yp) * wp + xp) * cpad + g * 8) =
          make_uint4(0, 0, 0, 0);
    }
  }
}

// Fast path for NCHW-like inputs (pixels contiguous, W even, rows aligned to
// the vector width): one CTA writes padded row (b, yp) for one 64-channel chunk.
// Global reads are 16-, 8- or 4-byte vectors along x; the tile is transposed through
// shared memory as 32-bit pixel pairs (row pitch chosen so the 8 channel rows a
// thread gathers fall in different banks), and each thread writes two 16-byte
// channel vectors, one per pixel of its pair.
constexpr int kVecThreads = 256;
constexpr int kMaxSeg = 256;  // pixels per pass

template <int VW>  // elements per global load: 8 (16 B), 4 (8 B) or 2 (4 B)
__global__ void __launch_bounds__(kVecThreads) pack_rows_nchw_vec_kernel(
    const uint16_t* __restrict__ x, long long sn, long long sc, long long sh, int C, int H, int W, int chunks,
    int pitch_words, uint16_t* __restrict__ rows, float* __restrict__ rowsum) {
  extern __shared__ uint32_t tw[];  // [64][pitch_words]
  const int chunk = blockIdx.x % chunks;
  const int yp = (blockIdx.x / chunks) % (H + 2);
  const int b = blockIdx.x / (chunks * (H + 2));
  const int wp = W + 2;
  const long long cpad = (long long)chunks * kCh;
  uint16_t* dst_row = rows + ((long long)(b * (H + 2) + yp) * wp) * cpad + chunk * kCh;
  const int tid = threadIdx.x;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  // rowsum (optional): per padded row, the sum over x of each channel (border rows 0)
  float* rsum = rowsum ? rowsum + (long long)(b * (H + 2) + yp) * cpad + chunk * kCh : nullptr;
  if (yp == 0 || yp == H + 1) {
    for (int e = tid; e < wp * 8; e += kVecThreads)
      *reinterpret_cast<uint4*>(dst_row + (long long)(e >> 3) * cpad + (e & 7) * 8) = zero;
    if (rsum && tid < kCh) rsum[tid] = 0.f;
    return;
  }
  float csum = 0.f;
  if (tid < 16) {
    const int px = (tid < 8) ? 0 : W + 1;
    *reinterpret_cast<uint4*>(dst_row + (long long)px * cpad + (tid & 7) * 8) = zero;
  }
  const uint16_t* src = x + b * sn + (long long)(yp - 1) * sh + (long long)(chunk * kCh) * sc;
  const int cvalid = min(kCh, C - chunk * kCh);
  for (int x0 = 0; x0 < W; x0 += kMaxSeg) {
    const int seg = min(kMaxSeg, W - x0);  // multiple of VW
    const int nvec = seg / VW;
    if (x0) __syncthreads();
    for (int e = tid; e < kCh * nvec; e += kVecThreads) {
      const int c = e / nvec, v = e - c * nvec;
      const uint16_t* g = src + (long long)c * sc + x0 + v * VW;
      uint32_t* t = tw + c * pitch_words + v * (VW / 2);
      if constexpr (VW == 8) {
        uint4 val = zero;
        if (c < cvalid) val = *reinterpret_cast<const uint4*>(g);
        t[0] = val.x;
        t[1] = val.y;
        t[2] = val.z;
        t[3] = val.w;
      } else if constexpr (VW == 4) {
        uint2 val = make_uint2(0, 0);
        if (c < cvalid) val = *reinterpret_cast<const uint2*>(g);
        t[0] = val.x;
        t[1] = val.y;
      } else {
        t[0] = c < cvalid ? *reinterpret_cast<const uint32_t*>(g) : 0u;
      }
    }
    __syncthreads();
    if (rsum && tid < kCh) {  // channel tid of this row segment, in x order
      const uint32_t* t = tw + tid * pitch_words;
      for (int w = 0; w < (seg >> 1); ++w) {
        const uint32_t v = t[w];
        csum += __uint_as_float(v << 16);
        csum += __uint_as_float(v & 0xffff0000u);
      }
    }
    const int npairs = seg >> 1;
    for (int e = tid; e < npairs * 8; e += kVecThreads) {
      const int pp = e >> 3, v = e & 7;
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = tw[(v * 8 + k) * pitch_words + pp];
      uint4 lo, hi;
      lo.x = __byte_perm(w[0], w[1], 0x5410);
      lo.y = __byte_perm(w[2], w[3], 0x5410);
      lo.z = __byte_perm(w[4], w[5], 0x5410);
      lo.w = __byte_perm(w[6], w[7], 0x5410);
      hi.x = __byte_perm(w[0], w[1], 0x7632);
      hi.y = __byte_perm(w[2], w[3], 0x7632);
      hi.z = __byte_perm(w[4], w[5], 0x7632);
      hi.w = __byte_perm(w[6], w[7], 0x7632);
      const long long px = x0 + 2 * pp + 1;  // padded column of the pair's first pixel
      *reinterpret_cast<uint4*>(dst_row + px * cpad + v * 8) = lo;
      *reinterpret_cast<uint4*>(dst_row + (px + 1) * cpad + v * 8) = hi;
    }
  }
  if (rsum && tid < kCh) rsum[tid] = csum;
}

// TMA variant of the NCHW packer (W % 8 == 0, W <= 256, 16-byte strides).
// Persistent CTAs walk work items (b, y, chunk), y fastest: the TMA unit
// loads the 64-channel x W slab of image row y (channel-major, channels past
// C zero-filled) into one of two input buffers while the CTA transposes the
// other into a 128-byte-swizzled [W][64] tile, which a TMA store writes to
// padded pixels 1..W of the row.  Threads write the two border pixels of the
// row; extra items zero the top and bottom border rows.  With `rowsum`, the
// per-row channel sums (fp32, x order) are left as the generic kernel does.
constexpr int kTmaPackThreads = 256;

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}

template <bool ROWSUM>
__global__ void __launch_bounds__(kTmaPackThreads) pack_rows_nchw_tma_kernel(
    const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout, int B, int H, int W,
    int chunks, uint16_t* __restrict__ rows, float* __restrict__ rowsum, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tile = W * 128;  // bytes of one [W][64] bf16 tile; also of one [64][W] slab
  uint8_t* obuf = smem;                 // 2 output tiles (1024-aligned: W % 8 == 0)
  uint8_t* ibuf = smem + 2 * tile;      // 2 input slabs
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 4 * tile);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2);
  const int tid = threadIdx.x;
  const int wp = W + 2;
  const long long cpad = (long long)chunks * kCh;
  const long long interior = (long long)B * H * chunks;
  const long long items = interior + 2LL * B * chunks;
  if (tid == 0) {
    mbar_init(smem_u32(&full[0]), 1);
    mbar_init(smem_u32(&full[1]), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  int issued = 0;  // loads issued (thread 0)
  auto issue = [&](long long it, int s) {  // thread 0: load interior item `it` into slab s
    ++issued;
    const int y = int(it % H);
    const long long r = it / H;
    const int chunk = int(r % chunks);
    const int b = int(r / chunks);
    const uint32_t bar = smem_u32(&full[s]);
    mbar_arrive_expect_tx(bar, uint32_t(tile));
    tma_load_4d(smem_u32(ibuf + s * tile), &tin, bar, 0, y, chunk * kCh, b);
  };
  const uint4 zero = make_uint4(0, 0, 0, 0);
  long long it = blockIdx.x;
  if (tid == 0 && it < interior) issue(it, 0);
  int i = 0;      // interior items done by this CTA
  bool ok = true;
  for (; it < items; it += gridDim.x) {
    if (it >= interior) {  // a top / bottom border row: zeros (and zero row sums)
      const long long r = it - interior;
      const int chunk = int(r % chunks);
      const int top = int((r / chunks) % 2);
      const int b = int(r / (2LL * chunks));
      const int yp = top ? 0 : H + 1;
      uint16_t* dst = rows + ((long long)(b * (H + 2) + yp) * wp) * cpad + chunk * kCh;
      for (int e = tid; e < wp * 8; e += kTmaPackThreads)
        *reinterpret_cast<uint4*>(dst + (long long)(e >> 3) * cpad + (e & 7) * 8) = zero;
      if (ROWSUM && tid < kCh) rowsum[(long long)(b * (H + 2) + yp) * cpad + chunk * kCh + tid] = 0.f;
      continue;
    }
    const int s = i & 1;
    const long long nxt = it + gridDim.x;
    // slab s^1 was last read in the previous iteration, before its closing barrier
    if (tid == 0 && nxt < interior) issue(nxt, s ^ 1);
    const int y = int(it % H);
    const long long r = it / H;
    const int chunk = int(r % chunks);
    const int b = int(r / chunks);
    const long long prow = (long long)b * (H + 2) + y + 1;
    uint16_t* dst = rows + prow * wp * cpad + chunk * kCh;
    if (tid < 16) *reinterpret_cast<uint4*>(dst + (long long)(tid < 8 ? 0 : W + 1) * cpad + (tid & 7) * 8) = zero;
    if (tid == 0) bulk_wait_read<1>();  // the store issued two items ago has read tile s
    ok = mbar_wait(smem_u32(&full[s]), uint32_t((i >> 1) & 1), status, abort_flag);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const uint32_t* in32 = reinterpret_cast<const uint32_t*>(ibuf + s * tile);
    uint8_t* out = obuf + s * tile;
    const int half = W >> 1;  // pixel pairs
    for (int e = tid; e < half * 8; e += kTmaPackThreads) {
      const int pp = e % half, v = e / half;  // lanes walk pixel pairs: conflict-free slab reads
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = in32[(v * 8 + k) * half + pp];
      uint4 lo, hi;
      lo.x = __byte_perm(w[0], w[1], 0x5410);
      lo.y = __byte_perm(w[2], w[3], 0x5410);
      lo.z = __byte_perm(w[4], w[5], 0x5410);
      lo.w = __byte_perm(w[6], w[7], 0x5410);
      hi.x = __byte_perm(w[0], w[1], 0x7632);
      hi.y = __byte_perm(w[2], w[3], 0x7632);
      hi.z = __byte_perm(w[4], w[5], 0x7632);
      hi.w = __byte_perm(w[6], w[7], 0x7632);
      const int px = 2 * pp;  // 128-byte swizzle: chunk v of pixel px at v ^ (px & 7)
      *reinterpret_cast<uint4*>(out + px * 128 + ((v ^ (px & 7)) << 4)) = lo;
      *reinterpret_cast<uint4*>(out + (px + 1) * 128 + ((v ^ ((px + 1) & 7)) << 4)) = hi;
    }
    if (ROWSUM && tid < kCh) {  // channel tid of this row, in x order
      const uint32_t* t = in32 + tid * half;
      float csum = 0.f;
      for (int q = 0; q < half; ++q) {
        const uint32_t v = t[q];
        csum += __uint_as_float(v << 16);
        csum += __uint_as_float(v & 0xffff0000u);
      }
      rowsum[prow * cpad + chunk * kCh + tid] = csum;
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tma_store_2d(&tout, smem_u32(out), chunk * kCh, int(prow * wp + 1));
      bulk_commit();
    }
    ++i;
  }
  if (!ok && tid == 0) {
    // loads i .. issued-1 may still be in flight into this CTA's shared memory: let them land
    for (int q = i; q < issued; ++q) mbar_wait(smem_u32(&full[q & 1]), uint32_t((q >> 1) & 1), status, nullptr);
  }
  if (tid == 0) bulk_wait_all();
}

// Channel sums, stage 1: out[g][c] = sum of rows [64g, 64g+64) of in[.][c]
// (in = per-row sums from the packer, or the packed rows themselves).
template <typename T>
__global__ void chsum_stage1_kernel(const T* __restrict__ in, long long nrows, int ld, int C,
                                    float* __restrict__ out) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const long long r0 = (long long)blockIdx.x * 64;
  const long long r1 = r0 + 64 < nrows ? r0 + 64 : nrows;
  float s = 0.f;
  for (long long r = r0; r < r1; ++r) {
    if constexpr (sizeof(T) == 2)
      s += bf2f(in[r * ld + c]);
    else
      s += in[r * ld + c];
  }
  out[(long long)blockIdx.x * C + c] = s;
}

// Channel sums of dense channels-last pixel rows (C % 8 == 0, C <= 2048,
// 16-byte aligned rows), stage 1: block g sums rows [g*rpb, (g+1)*rpb) into
// out[g][c].  A thread owns 8 channels (16-byte loads) of every
// rows_per_iter-th row of the range, four loads in flight; the block's row
// lanes are then added in lane order: a fixed order, deterministic.
__global__ void __launch_bounds__(256) chsum_nhwc_vec_kernel(const uint16_t* __restrict__ x, long long P,
                                                              long long sw, int C, long long rpb,
                                                              float* __restrict__ out) {
  extern __shared__ float part[];  // [rows_per_iter][C]
  const int lanes = C / 8;
  const int rows_per_iter = 256 / lanes;
  const int t = threadIdx.x;
  const int rl = t / lanes, cl = t - (t / lanes) * lanes;
  const long long r0 = (long long)blockIdx.x * rpb;
  const long long r1 = r0 + rpb < P ? r0 + rpb : P;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (rl < rows_per_iter) {
    long long r = r0 + rl;
    for (; r + 3LL * rows_per_iter < r1; r += 4LL * rows_per_iter) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = *reinterpret_cast<const uint4*>(x + (r + (long long)u * rows_per_iter) * sw + cl * 8);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[2 * k] += __uint_as_float(w[k] << 16);
          acc[2 * k + 1] += __uint_as_float(w[k] & 0xffff0000u);
        }
      }
    }
    for (; r < r1; r += rows_per_iter) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + r * sw + cl * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[2 * k] += __uint_as_float(w[k] << 16);
        acc[2 * k + 1] += __uint_as_float(w[k] & 0xffff0000u);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) part[rl * C + cl * 8 + k] = acc[k];
  }
  __syncthreads();
  for (int c = t; c < C; c += 256) {
    float s = 0.f;
    for (int l = 0; l < rows_per_iter; ++l) s += part[l * C + c];
    out[(long long)blockIdx.x * C + c] = s;
  }
}

// Stage 2 for many groups: a warp per channel, lane l adding groups l, l+32,
// ... in order, then a fixed shuffle tree (deterministic), rounded once.
__global__ void chsum_stage2_warp_kernel(const float* __restrict__ in, int ngroups, int C, void* out, int dtype) {
  const int c = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (c >= C) return;
  double s = 0.0;
  for (int g = lane; g < ngroups; g += 32) s += in[(long long)g * C + c];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if (lane == 0) {
    if (dtype == B2_F32)
      static_cast<float*>(out)[c] = float(s);
    else
      static_cast<uint16_t*>(out)[c] = f2bf(float(s));
  }
}

// Stage 2: dbias[c] = sum over groups, fixed order, rounded once.
__global__ void chsum_stage2_kernel(const float* __restrict__ in, int ngroups, int C, void* out, int dtype) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double s = 0.0;
  for (int g = 0; g < ngroups; ++g) s += in[(long long)g * C + c];
  if (dtype == B2_F32)
    static_cast<float*>(out)[c] = float(s);
  else
    static_cast<uint16_t*>(out)[c] = f2bf(float(s));
}

// Channels-last inputs (channels contiguous, C % 8 == 0): a padded 16-byte copy.
__global__ void pack_rows_nhwc_vec_kernel(const uint16_t* __restrict__ x, long long sn, long long sh, long long sw,
                                          int B, int C, int H, int W, int chunks, uint16_t* __restrict__ rows) {
  const int wp = W + 2, hp = H + 2;
  const int vpr = chunks * 8;  // 16-byte vectors per padded row (pixel)
  const long long total = (long long)B * hp * wp * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int v = int(i % vpr);
    const long long p = i / vpr;
    const int xp = int(p % wp);
    const long long r = p / wp;
    const int yp = int(r % hp);
    const int b = int(r / hp);
    uint4 val = make_uint4(0, 0, 0, 0);
    const int c = v * 8;
    if (yp >= 1 && yp <= H && xp >= 1 && xp <= W && c < C)
      val = *reinterpret_cast<const uint4*>(x + b * sn + (long long)(yp - 1) * sh + (long long)(xp - 1) * sw + c);
    *reinterpret_cast<uint4*>(rows + p * (long long)(chunks * kCh) + c) = val;
  }
}

// Wk[n][chunk*576 + tap*64 + c]; forward: n = co, source w[co][chunk*64+c][tap];
// dgrad: n = ci, source w[chunk*64+c][ci][8-tap] (spatial flip + in/out swap).
// The source is read through its element strides (co, ci, ky, kx): OIHW, or
// the channels-last OHWI form of a channels-last model, without a copy.
struct WStrides {
  long long co, ci, ky, kx;
};
__global__ void pack_weight_kernel(const uint16_t* __restrict__ w, WStrides ws, int Cout, int Cin, int chunks,
                                   int dgrad, uint16_t* __restrict__ wk) {
  const int ktot = chunks * 576;
  const int nrows = dgrad ? Cin : Cout;
  const int kred = dgrad ? Cout : Cin;  // channels reduced over
  const long long total = (long long)nrows * ktot;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = int(i / ktot);
    const int k = int(i % ktot);
    const int chunk = k / 576;
    const int tap = (k % 576) / 64;
    const int c = chunk * 64 + (k % 64);
    uint16_t v = 0;
    if (c < kred) {
      const int t = dgrad ? 8 - tap : tap;
      const long long co = dgrad ? c : n, ci = dgrad ? n : c;
      v = w[co * ws.co + ci * ws.ci + (t / 3) * ws.ky + (t % 3) * ws.kx];
    }
    wk[i] = v;
  }
}

// The same packing, 8 consecutive K entries (one 16-byte store) per thread:
// unit u = (n, k8) with k = chunk*576 + tap*64 + c8*8.  Forward: the 8
// channels ci = chunk*64 + c8*8 + e of w[co][ci][tap] -- one 16-byte load
// when the channel stride is 1 (channels-last weights), else 8 loads; dgrad:
// the 8 output channels co = chunk*64 + c8*8 + e of w[co][ci][8 - tap].
// Needs the reduced channel count (Cin forward, Cout dgrad) % 8 == 0.
__global__ void pack_weight_vec_kernel(const uint16_t* __restrict__ w, WStrides ws, int Cout, int Cin, int chunks,
                                       int dgrad, uint16_t* __restrict__ wk) {
  const int k8tot = chunks * 72;  // 576 / 8
  const int nrows = dgrad ? Cin : Cout;
  const int kred = dgrad ? Cout : Cin;
  const long long total = (long long)nrows * k8tot;
  const bool vec = !dgrad && ws.ci == 1 && (ws.co % 8) == 0 && (ws.ky % 8) == 0 && (ws.kx % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = int(i / k8tot);
    const int k8 = int(i % k8tot);
    const int chunk = k8 / 72, rem = k8 % 72;
    const int tap = rem / 8, c0 = chunk * 64 + (rem % 8) * 8;
    uint4 out = make_uint4(0, 0, 0, 0);
    if (c0 < kred) {
      const int t = dgrad ? 8 - tap : tap;
      const long long tapoff = (t / 3) * ws.ky + (t % 3) * ws.kx;
      if (vec) {
        out = __ldg(reinterpret_cast<const uint4*>(w + n * ws.co + c0 + tapoff));
      } else {
        uint32_t v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const long long co = dgrad ? c0 + e : n, ci = dgrad ? n : c0 + e;
          v[e] = __ldg(w + co * ws.co + ci * ws.ci + tapoff);
        }
        out = make_uint4(v[0] | (v[1] << 16), v[2] | (v[3] << 16), v[4] | (v[5] << 16), v[6] | (v[7] << 16));
      }
    }
    reinterpret_cast<uint4*>(wk)[i] = out;
  }
}

// [B][R][S] -> [B][S][R] bf16 tile transpose (R, S arbitrary).
__global__ void __launch_bounds__(256) transpose_kernel(const uint16_t* __restrict__ src,
                                                        uint16_t* __restrict__ dst, int R, int S) {
  __shared__ uint16_t tile[64][64 + 2];
  const int tiles_s = (S + 63) / 64;
  const int tiles_r = (R + 63) / 64;
  const int ts = blockIdx.x % tiles_s;
  const int tr = (blockIdx.x / tiles_s) % tiles_r;
  const int b = blockIdx.x / (tiles_s * tiles_r);
  const uint16_t* s = src + (long long)b * R * S;
  uint16_t* d = dst + (long long)b * R * S;
  const int tid = threadIdx.x;
  for (int i = 0; i < 16; ++i) {
    const int e = i * 256 + tid;
    const int r = e / 64, c = e % 64;
    const int rr = tr * 64 + r, cc = ts * 64 + c;
    tile[r][c] = (rr < R && cc < S) ? s[(long long)rr * S + cc] : uint16_t(0);
  }
  __syncthreads();
  for (int i = 0; i < 16; ++i) {
    const int e = i * 256 + tid;
    const int c = e / 64, r = e % 64;
    const int rr = tr * 64 + r, cc = ts * 64 + c;
    if (rr < R && cc < S) d[(long long)cc * R + rr] = tile[r][c];
  }
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

// Returns the vector width of the NCHW fast path (0: not eligible).
static int nchw_vec_width(const void* x, int64_t sn, int64_t sc, int64_t sh, int64_t sw, int W) {
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
  for (int cand : {8, 4, 2})
    if (sw == 1 && W % cand == 0 && sh % cand == 0 && sc % cand == 0 && sn % cand == 0 && (xa % (2 * cand)) == 0)
      return cand;
  return 0;
}

static b2_status pack_rows_impl(const void* x, int64_t sn, int64_t sc, int64_t sh, int64_t sw, int B, int C, int H,
                                int W, int chunks, void* rows, float* rowsum, void* stream);

b2_status b2_pack_rows_bf16(const void* x, int64_t sn, int64_t sc, int64_t sh, int64_t sw, int B,
                            int C, int H, int W, int chunks, void* rows, void* stream) {
  return pack_rows_impl(x, sn, sc, sh, sw, B, C, H, W, chunks, rows, nullptr, stream);
}

size_t b2_pack_rows_dbias_workspace_bytes(int B, int C, int H, int W) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0) return 256;
  const long long cpad = ((C + 63) / 64) * 64;
  const long long prow = (long long)B * (H + 2);
  const long long m_total = prow * (W + 2);
  const long long fused = prow * cpad + ((prow + 63) / 64) * C;
  const long long generic = ((m_total + 63) / 64) * C;
  const long long floats = fused > generic ? fused : generic;
  return size_t((floats * 4 + 255) / 256 * 256);
}

b2_status b2_pack_rows_dbias_bf16(const void* x, int64_t sn, int64_t sc, int64_t sh, int64_t sw, int B, int C, int H,
                                  int W, int chunks, void* rows, void* dbias, int dbias_dtype, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (!dbias || !workspace) return set_error(B2_ERR_INVALID, "b2_pack_rows_dbias_bf16: null pointer");
  if (dbias_dtype != B2_BF16 && dbias_dtype != B2_F32)
    return set_error(B2_ERR_INVALID, "b2_pack_rows_dbias_bf16: dtype");
  if (workspace_bytes < b2_pack_rows_dbias_workspace_bytes(B, C, H, W))
    return set_error(B2_ERR_WORKSPACE, "b2_pack_rows_dbias_bf16: workspace %zu < %zu bytes", workspace_bytes,
                     b2_pack_rows_dbias_workspace_bytes(B, C, H, W));
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return set_error(B2_ERR_INVALID, "b2_pack_rows_dbias_bf16: workspace alignment");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long cpad = (long long)chunks * kCh;
  const long long prow = (long long)B * (H + 2);
  float* ws = static_cast<float*>(workspace);
  if (nchw_vec_width(x, sn, sc, sh, sw, W)) {
    // the packer itself leaves per-row channel sums: no second pass over dY
    float* rowsum = ws;
    float* groups = ws + prow * cpad;
    B2_TRY(pack_rows_impl(x, sn, sc, sh, sw, B, C, H, W, chunks, rows, rowsum, stream));
    const long long ng = (prow + 63) / 64;
    chsum_stage1_kernel<float><<<dim3(unsigned(ng), unsigned((C + 255) / 256)), 256, 0, st>>>(rowsum, prow,
                                                                                          int(cpad), C, groups);
    chsum_stage2_kernel<<<(C + 255) / 256, 256, 0, st>>>(groups, int(ng), C, dbias, dbias_dtype);
  } else {
    B2_TRY(pack_rows_impl(x, sn, sc, sh, sw, B, C, H, W, chunks, rows, nullptr, stream));
    const long long m_total = prow * (W + 2);
    const long long ng = (m_total + 63) / 64;
    chsum_stage1_kernel<uint16_t><<<dim3(unsigned(ng), unsigned((C + 255) / 256)), 256, 0, st>>>(
        static_cast<const uint16_t*>(rows), m_total, int(cpad), C, ws);
    chsum_stage2_kernel<<<(C + 255) / 256, 256, 0, st>>>(ws, int(ng), C, dbias, dbias_dtype);
  }
  return check_cuda(cudaGetLastError(), "channel-sum launch");
}

size_t b2_channel_sum_nhwc_workspace_bytes(int B, int C, int H, int W) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0) return 256;
  const long long ng = ((long long)B * H * W + 63) / 64;
  return size_t((ng * C * 4 + 255) / 256 * 256);
}

b2_status b2_channel_sum_nhwc_bf16(const void* x, int64_t sn, int64_t sh, int64_t sw, int B, int C, int H, int W,
                                   void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (!x || !out || !workspace) return set_error(B2_ERR_INVALID, "b2_channel_sum_nhwc_bf16: null pointer");
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0) return set_error(B2_ERR_INVALID, "b2_channel_sum_nhwc_bf16: bad shape");
  if (out_dtype != B2_BF16 && out_dtype != B2_F32)
    return set_error(B2_ERR_INVALID, "b2_channel_sum_nhwc_bf16: dtype");
  if (W == 1) sw = C;  // strides of size-1 dimensions address nothing
  if (H == 1) sh = (int64_t)W * sw;
  if (B == 1) sn = (int64_t)H * sh;
  if (sw < C || sh != (int64_t)W * sw || sn != (int64_t)H * sh)
    return set_error(B2_ERR_UNSUPPORTED, "b2_channel_sum_nhwc_bf16: pixels must be dense rows of sw >= C elements");
  if (workspace_bytes < b2_channel_sum_nhwc_workspace_bytes(B, C, H, W) || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return set_error(B2_ERR_WORKSPACE, "b2_channel_sum_nhwc_bf16: workspace of %zu bytes needed",
                     b2_channel_sum_nhwc_workspace_bytes(B, C, H, W));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long P = (long long)B * H * W;
  const long long ng = (P + 63) / 64;
  if (ng > 0x7fffffffLL) return set_error(B2_ERR_UNSUPPORTED, "b2_channel_sum_nhwc_bf16: too many pixels");
  float* ws = static_cast<float*>(workspace);
  if (C % 8 == 0 && C <= 2048 && sw % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // 16-byte loads over ranges of rows: up to 592 blocks (4 per SM), at most
    // ng groups, so the workspace bound above holds
    const long long rows_per_iter = 256 / (C / 8);
    const long long groups = std::min<long long>(std::min<long long>(592, ng), (P + rows_per_iter - 1) / rows_per_iter);
    const long long rpb = (P + groups - 1) / groups;
    const long long g = (P + rpb - 1) / rpb;
    const size_t smem = size_t(rows_per_iter) * C * sizeof(float);
    chsum_nhwc_vec_kernel<<<unsigned(g), 256, smem, st>>>(static_cast<const uint16_t*>(x), P, sw, C, rpb, ws);
    chsum_stage2_warp_kernel<<<(C + 7) / 8, 256, 0, st>>>(ws, int(g), C, out, out_dtype);
    return check_cuda(cudaGetLastError(), "channel-sum launch");
  }
  chsum_stage1_kernel<uint16_t><<<dim3(unsigned(ng), unsigned((C + 255) / 256)), 256, 0, st>>>(
      static_cast<const uint16_t*>(x), P, int(sw), C, ws);
  chsum_stage2_kernel<<<(C + 255) / 256, 256, 0, st>>>(ws, int(ng), C, out, out_dtype);
  return check_cuda(cudaGetLastError(), "channel-sum launch");
}

// TMA packer launch (see pack_rows_nchw_tma_kernel); B2_ERR_UNSUPPORTED when
// the tensor maps cannot describe the operands, so the caller takes the
// generic kernel.
static b2_status pack_rows_nchw_tma(const void* x, int64_t sn, int64_t sc, int64_t sh, int B, int C, int H, int W,
                                   int chunks, void* rows, float* rowsum, cudaStream_t st) {
  if ((sh * 2) % 16 || (sc * 2) % 16 || (sn * 2) % 16 || (reinterpret_cast<uintptr_t>(x) & 15))
    return B2_ERR_UNSUPPORTED;
  const long long cpad = (long long)chunks * kCh;
  const long long npix = (long long)B * (H + 2) * (W + 2);
  CUtensorMap tin, tout;
  {
    const uint64_t dims[4] = {uint64_t(W), uint64_t(H), uint64_t(C), uint64_t(B)};
    const uint64_t strides[3] = {uint64_t(sh) * 2, uint64_t(sc) * 2, uint64_t(sn) * 2};
    const uint32_t box[4] = {uint32_t(W), 1, uint32_t(kCh), 1};
    if (encode_tmap_sw(&tin, x, 4, dims, strides, box, 0) != B2_OK) return B2_ERR_UNSUPPORTED;
  }
  {
    const uint64_t dims[2] = {uint64_t(cpad), uint64_t(npix)};
    const uint64_t strides[1] = {uint64_t(cpad) * 2};
    const uint32_t box[2] = {uint32_t(kCh), uint32_t(W)};
    if (encode_tmap_sw(&tout, rows, 2, dims, strides, box, 128) != B2_OK) return B2_ERR_UNSUPPORTED;
  }
  const size_t smem = size_t(4) * W * 128 + 64 + 1024;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  auto kern = rowsum ? pack_rows_nchw_tma_kernel<true> : pack_rows_nchw_tma_kernel<false>;
  // once per device and variant, at the largest size (W = 256): no attribute
  // calls per launch, so that the packer can run inside a CUDA graph capture
  static bool configured[2][64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[rowsum ? 1 : 0][dev]) {
    B2_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(size_t(4) * 256 * 128 + 64 + 1024)),
                      "cudaFuncSetAttribute(pack smem)"));
    configured[rowsum ? 1 : 0][dev] = true;
  }
  int per_sm = 0;
  B2_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTmaPackThreads, smem),
                    "pack occupancy"));
  const long long items = (long long)B * H * chunks + 2LL * B * chunks;
  const int grid = int(std::max<long long>(1, std::min<long long>(items, (long long)std::max(1, per_sm) * sm_count(dev))));
  kern<<<grid, kTmaPackThreads, smem, st>>>(tin, tout, B, H, W, chunks, static_cast<uint16_t*>(rows), rowsum,
                                             device_status_ptr());
  return check_cuda(cudaGetLastError(), "pack_rows(nchw tma) launch");
}

static b2_status pack_rows_impl(const void* x, int64_t sn, int64_t sc, int64_t sh, int64_t sw, int B, int C, int H,
                                int W, int chunks, void* rows, float* rowsum, void* stream) {
  if (!x || !rows) return set_error(B2_ERR_INVALID, "b2_pack_rows_bf16: null pointer");
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || chunks < (C + 63) / 64)
    return set_error(B2_ERR_INVALID, "b2_pack_rows_bf16: bad shape B=%d C=%d H=%d W=%d chunks=%d", B, C,
                     H, W, chunks);
  if (reinterpret_cast<uintptr_t>(rows) & 15) return set_error(B2_ERR_INVALID, "b2_pack_rows_bf16: rows not 16-byte aligned");
  const long long blocks = (long long)B * (H + 2) * chunks;
  if (blocks >= (1LL << 31)) return set_error(B2_ERR_UNSUPPORTED, "b2_pack_rows_bf16: too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
  const int vw = nchw_vec_width(x, sn, sc, sh, sw, W);  // widest vector the strides and base allow
  if (vw == 8 && W <= 256 && H > 0) {
    b2_status rc = pack_rows_nchw_tma(x, sn, sc, sh, B, C, H, W, chunks, rows, rowsum, st);
    if (rc != B2_ERR_UNSUPPORTED) return rc;
  }
  if (vw) {
    const int seg = std::min(W, kMaxSeg);
    int pitch = seg / 2;
    while (pitch % 4 != 1) ++pitch;  // pitch = 1 mod 4 words: conflict-light gathers
    const size_t smem = size_t(kCh) * pitch * 4;
    auto* xs = static_cast<const uint16_t*>(x);
    auto* rs = static_cast<uint16_t*>(rows);
    if (vw == 8)
      pack_rows_nchw_vec_kernel<8><<<unsigned(blocks), kVecThreads, smem, st>>>(xs, sn, sc, sh, C, H, W, chunks,
                                                                               pitch, rs, rowsum);
    else if (vw == 4)
      pack_rows_nchw_vec_kernel<4><<<unsigned(blocks), kVecThreads, smem, st>>>(xs, sn, sc, sh, C, H, W, chunks,
                                                                               pitch, rs, rowsum);
    else
      pack_rows_nchw_vec_kernel<2><<<unsigned(blocks), kVecThreads, smem, st>>>(xs, sn, sc, sh, C, H, W, chunks,
                                                                               pitch, rs, rowsum);
    return check_cuda(cudaGetLastError(), "pack_rows(nchw) launch");
  }
  if (sc == 1 && C % 8 == 0 && sw % 8 == 0 && sh % 8 == 0 && sn % 8 == 0 && (xa & 15) == 0) {
    const long long total = (long long)B * (H + 2) * (W + 2) * chunks * 8;
    const int grid = int(std::min<long long>((total + 255) / 256, 148LL * 16));
    pack_rows_nhwc_vec_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(x), sn, sh, sw, B, C, H, W, chunks,
                                                    static_cast<uint16_t*>(rows));
    return check_cuda(cudaGetLastError(), "pack_rows(nhwc) launch");
  }
  if ((long long)H * W >= (1LL << 31)) return set_error(B2_ERR_UNSUPPORTED, "b2_pack_rows_bf16: too large");
  const long long vecs = (long long)B * chunks * 8 * ((long long)H * W + 2LL * (W + 2) + 2LL * H);
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int grid = int(std::max<long long>(1, std::min<long long>((vecs + 255) / 256, (long long)sm_count(dev) * 16)));
  pack_rows_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(x), sn, sc, sh, sw, B, C, H, W, chunks,
                                         static_cast<uint16_t*>(rows));
  return check_cuda(cudaGetLastError(), "pack_rows launch");
}

static b2_status pack_weight(const void* w, WStrides ws, int Cout, int Cin, int chunks, int dgrad, void* wk,
                             void* stream, const char* name) {
  if (!w || !wk) return set_error(B2_ERR_INVALID, "%s: null pointer", name);
  const int kred = dgrad ? Cout : Cin;
  if (Cout <= 0 || Cin <= 0 || chunks < (kred + 63) / 64) return set_error(B2_ERR_INVALID, "%s: bad shape", name);
  if (ws.co < 0 || ws.ci < 0 || ws.ky < 0 || ws.kx < 0) return set_error(B2_ERR_INVALID, "%s: negative stride", name);
  const long long total = (long long)(dgrad ? Cin : Cout) * chunks * 576;
  if (kred % 8 == 0 && (reinterpret_cast<uintptr_t>(wk) & 15) == 0) {
    const int blocks = int(std::min<long long>((total / 8 + 255) / 256, 148LL * 8));
    pack_weight_vec_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(w), ws, Cout, Cin, chunks, dgrad, static_cast<uint16_t*>(wk));
    return check_cuda(cudaGetLastError(), "pack_weight launch");
  }
  const int blocks = int(std::min<long long>((total + 255) / 256, 148LL * 8));
  pack_weight_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), ws, Cout, Cin, chunks, dgrad, static_cast<uint16_t*>(wk));
  return check_cuda(cudaGetLastError(), "pack_weight launch");
}

b2_status b2_pack_weight_fwd_bf16(const void* w, int Cout, int Cin, int chunks, void* wk, void* stream) {
  return pack_weight(w, WStrides{9LL * Cin, 9, 3, 1}, Cout, Cin, chunks, 0, wk, stream, "b2_pack_weight_fwd_bf16");
}

b2_status b2_pack_weight_dgrad_bf16(const void* w, int Cout, int Cin, int chunks_o, void* wk,
                                    void* stream) {
  return pack_weight(w, WStrides{9LL * Cin, 9, 3, 1}, Cout, Cin, chunks_o, 1, wk, stream,
                     "b2_pack_weight_dgrad_bf16");
}

b2_status b2_pack_weight_strided_bf16(const void* w, const int64_t* strides, int Cout, int Cin, int chunks,
                                      int dgrad, void* wk, void* stream) {
  if (!strides) return set_error(B2_ERR_INVALID, "b2_pack_weight_strided_bf16: null strides");
  return pack_weight(w, WStrides{strides[0], strides[1], strides[2], strides[3]}, Cout, Cin, chunks, dgrad ? 1 : 0,
                     wk, stream, "b2_pack_weight_strided_bf16");
}

static b2_status transpose(const void* src, void* dst, int B, int R, int S, void* stream, const char* name) {
  if (!src || !dst) return set_error(B2_ERR_INVALID, "%s: null pointer", name);
  if (B <= 0 || R <= 0 || S <= 0) return set_error(B2_ERR_INVALID, "%s: bad shape", name);
  const long long blocks = (long long)B * ((R + 63) / 64) * ((S + 63) / 64);
  if (blocks >= (1LL << 31)) return set_error(B2_ERR_UNSUPPORTED, "%s: too large", name);
  transpose_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), R, S);
  return check_cuda(cudaGetLastError(), name);
}

b2_status b2_nchw_to_nhwc_bf16(const void* src, void* dst, int B, int C, int HW, void* stream) {
  return transpose(src, dst, B, C, HW, stream, "b2_nchw_to_nhwc_bf16");
}

b2_status b2_nhwc_to_nchw_bf16(const void* src, void* dst, int B, int C, int HW, void* stream) {
  return transpose(src, dst, B, HW, C, stream, "b2_nhwc_to_nchw_bf16");
}

}  // extern "C"
