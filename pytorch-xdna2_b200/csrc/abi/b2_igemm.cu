// tcgen05 implicit-GEMM kernels for sm_100a: 3x3/s1/p1 convolution forward
// and dgrad, convolution wgrad, and dense (batched) bf16 GEMM.  Activations
// come as padded-grid rows (b2_pack_rows_bf16) or, channels-last, straight
// from the caller's tensor through an im2col TMA map whose pixel box is the
// padded grid (the *_nhwc entry points: no packing pass).
//
// One persistent, warp-specialized kernel template serves all of them:
//   warp 0      TMA producer: fills a STAGES-deep ring of shared-memory
//               operand tiles (A: 128 x 64, B: BN x 64 bf16, 128-byte swizzle)
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16)
//               into a double-buffered fp32 accumulator in tensor memory
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, fused bias / ReLU /
//               alpha-beta, bf16 rounding and the store in the caller's layout
// The epilogue of tile i overlaps the mainloop of tile i+1.
//
// The convolution is the reference's conv3x3w formulation
// (xdna_train/_designs/conv3x3w.py:1-38): output rows are padded-grid pixels,
// so tap (dy,dx) of output row p is input row p + dy*(W+2) + dx and the im2col
// is nothing but a row offset in the TMA coordinate of the A tile.  K order is
// (chunk, dy, dx, c) as in conv3x3w_host.py:66-78.  Wgrad reduces over the
// padded rows with both operands M/N-major, so the same packed buffers serve
// forward, dgrad and wgrad (the reference's dW also reuses the packed X and dY,
// torch_xdna_device.cpp:1968-1985, 2660-2679).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kABytes = BM * BK * 2;

enum Kind : int { kConv = 0, kWgrad = 1, kGemm = 2 };

struct Params {
  // tile space
  int tiles_m, tiles_n, splits, batch;
  int num_kb;        // k-blocks of a full reduction
  int kb_per_split;  // wgrad split-K
  // conv geometry (padded grid)
  int wp, hp, H, W, m_total;
  int a_row_shift;   // wgrad: dY rows are read shifted by W+3
  int ci_blocks;     // wgrad: BN-wide input-channel blocks per tap
  // output
  int M, N;                      // valid output extents
  void* out;
  long long osn, osc, osh, osw;  // conv: element strides; gemm: osn = batch stride, osh = ldd
  const uint16_t* bias;
  int relu;
  float alpha, beta;
  const void* cin;
  int cin_dtype;
  long long c_sm, c_sn, c_sb;
  float* partial;                // wgrad partial sums [splits][9][M][N]; gemm split-K [splits][M][N]
  int* status;
  // GEMM extensions (1x1 convolutions)
  int a_bcast;       // A has one batch slice, shared by every batch
  int kb_per_batch;  // > 0: the reduction runs over the batch slices too (k-block kb is in slice kb / kb_per_batch)
  int gemm_split;    // 1: tile-space slices are split-K ranges writing fp32 partials
  int tma_store;     // GEMM: bf16 D written by TMA stores of shared-memory staged boxes
  int win_boxes, win_box_rows;  // conv halo kernel: the A window is win_boxes TMA boxes of win_box_rows rows
  int win_bufs;                 // resident-weight halo kernel: window buffers in flight (<= kMaxWinBufs)
  // activation operands read as padded-grid rows: bit 0 for the first map
  // (A, the halo window, wgrad's dY), bit 1 for the second (wgrad's X);
  // set = an im2col map over a channels-last tensor, clear = packed rows
  int src_im2col;
  // weight gradient over channels-last dY and X with tiled 4-D loads: k-block
  // kb is the patch_wb x patch_hb pixel patch (kb % patch_nx, kb / patch_nx %
  // patch_ny) of image kb / (patch_nx * patch_ny) (patch_wb * patch_hb == 64);
  // X for tap (dy, dx) is the same patch moved by (dx - 1, dy - 1), the image
  // border and the patch's overhang read as zeros.  0 = padded-row k-blocks.
  int patch_wb, patch_hb, patch_nx, patch_ny;
};

// Origin (x0, y0, n) of the pixel patch of k-block kb (Params::patch_*).
__device__ __forceinline__ void patch_origin(const Params& p, int kb, int& x0, int& y0, int& n) {
  const int bx = kb % p.patch_nx;
  const int t = kb / p.patch_nx;
  const int by = t % p.patch_ny;
  n = t / p.patch_ny;
  x0 = bx * p.patch_wb;
  y0 = by * p.patch_hb;
}

template <int BN>
struct Smem {
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
};

// GEMM output staging: per epilogue warp two 32-row bf16 boxes, one filled
// while the TMA store of the other reads it.  Boxes are 64 columns wide
// (128-byte rows, 128-byte swizzle) when the warp's half of the tile has 64
// or more columns, else 32 (64-byte rows, 64-byte swizzle).
template <int BN>
constexpr int epi_box_cols() {
  return BN >= 128 ? 64 : 32;
}
template <int BN>
constexpr int epi_box_bytes() {
  return 32 * epi_box_cols<BN>() * 2;
}
// TS: the GEMM writes bf16 D through TMA stores of staged boxes (short
// reductions, where the epilogue is the bottleneck); long reductions drop
// the staging for a deeper operand ring and store directly.
template <int KIND, int BN, bool TS = (KIND == kGemm)>
constexpr int epi_stage_bytes() {
  return (KIND == kGemm && TS) ? kEpiWarps * 2 * epi_box_bytes<BN>() : 0;
}

__device__ __forceinline__ void decode_tile(int kind, const Params& p, int t, int& mt, int& nt,
                                            int& bz, int& tap, int& kb0, int& kb1) {
  tap = 0;
  bz = 0;
  if (kind == kConv) {
    nt = t % p.tiles_n;
    mt = t / p.tiles_n;
    kb0 = 0;
    kb1 = p.num_kb;
  } else if (kind == kWgrad) {
    nt = t % p.ci_blocks;
    t /= p.ci_blocks;
    tap = t % 9;
    t /= 9;
    mt = t % p.tiles_m;
    int s = t / p.tiles_m;
    bz = s;
    kb0 = s * p.kb_per_split;
    kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  } else {
    nt = t % p.tiles_n;
    t /= p.tiles_n;
    mt = t % p.tiles_m;
    bz = t / p.tiles_m;
    if (p.gemm_split) {
      kb0 = bz * p.kb_per_split;
      kb1 = min(p.num_kb, kb0 + p.kb_per_split);
    } else {
      kb0 = 0;
      kb1 = p.num_kb;
    }
  }
}

__device__ __forceinline__ int total_tiles(int kind, const Params& p) {
  if (kind == kConv) return p.tiles_m * p.tiles_n;
  if (kind == kWgrad) return p.splits * p.tiles_m * 9 * p.ci_blocks;
  return p.batch * p.tiles_m * p.tiles_n;
}

// ---------------------------------------------------------------------------
// epilogues.  Thread owns accumulator row `row` of the tile; r[] holds columns
// [col0, col0+32) as fp32 bit patterns.  bf16 rounding uses the hardware
// round-to-nearest-even conversion (cvt.rn.bf16x2.f32).  Per-column vectors
// (bias) are read once per chunk by the warp and broadcast with shuffles.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cvt2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint16_t cvt1(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Output row of a conv tile: base pointer of pixel (b, y, x), or null when the
// padded-grid row is a border / tail row that produces nothing.
__device__ __forceinline__ uint16_t* conv_row_base_at(const Params& p, int prow) {
  if (prow >= p.m_total) return nullptr;
  const int plane = p.hp * p.wp;
  const int b = prow / plane;
  const int rem = prow - b * plane;
  const int y = rem / p.wp;
  const int x = rem - y * p.wp;
  if (y >= p.H || x >= p.W) return nullptr;
  return static_cast<uint16_t*>(p.out) + b * p.osn + y * p.osh + x * p.osw;
}
__device__ __forceinline__ uint16_t* conv_row_base(const Params& p, int mt, int row) {
  return conv_row_base_at(p, mt * BM + row);
}

__device__ __forceinline__ void epi_conv(const Params& p, uint16_t* base, int col0, int lane,
                                         const uint32_t (&r)[32]) {
  const bool full = col0 + 32 <= p.N;
  float v[32];
  // uniform branches outside the element loops (see gemm_values); without a
  // bias the accumulator still gets + 0.0f, which turns a -0 sum into +0 as
  // an accumulation that starts from zero does
  if (p.bias) {
    float bl = 0.f;
    if (col0 + lane < p.N) bl = bf2f(p.bias[col0 + lane]);
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]) + __shfl_sync(0xffffffffu, bl, c);
  } else {
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]) + 0.f;
  }
  if (p.relu) {
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = fmaxf(v[c], 0.f);
  }
  if (!base) return;
  if (p.osc == 1 && full && ((reinterpret_cast<uintptr_t>(base + col0) & 15) == 0)) {
    uint4* dst = reinterpret_cast<uint4*>(base + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[q] = make_uint4(cvt2(v[q * 8 + 0], v[q * 8 + 1]), cvt2(v[q * 8 + 2], v[q * 8 + 3]),
                          cvt2(v[q * 8 + 4], v[q * 8 + 5]), cvt2(v[q * 8 + 6], v[q * 8 + 7]));
    return;
  }
  uint16_t* q = base + (long long)col0 * p.osc;
  if (full) {
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      *q = cvt1(v[c]);
      q += p.osc;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      if (col0 + c < p.N) *q = cvt1(v[c]);
      q += p.osc;
    }
  }
}

__device__ __forceinline__ void epi_wgrad_co(const Params& p, int split, int tap, int co, int col0,
                                             const uint32_t (&r)[32]) {
  if (co >= p.M) return;
  float* dst = p.partial + ((((long long)split * 9 + tap) * p.M + co) * p.N);
  if (col0 + 32 <= p.N && (p.N % 4) == 0) {
    float4* d4 = reinterpret_cast<float4*>(dst + col0);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      d4[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                          __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    return;
  }
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (col0 + c < p.N) dst[col0 + c] = __uint_as_float(r[c]);
}
__device__ __forceinline__ void epi_wgrad(const Params& p, int split, int tap, int mt, int col0, int row,
                                          const uint32_t (&r)[32]) {
  epi_wgrad_co(p, split, tap, mt * BM + row, col0, r);
}

__device__ __forceinline__ float load_c(const Params& p, long long i) {
  return p.cin_dtype == B2_F32 ? static_cast<const float*>(p.cin)[i]
                               : bf2f(static_cast<const uint16_t*>(p.cin)[i]);
}

// alpha * acc + beta * C for columns [col0, col0+32) of output row m
__device__ __forceinline__ void gemm_values(const Params& p, int bz, int m, int col0, int lane,
                                            const uint32_t (&r)[32], float (&v)[32]) {
  // Branch once on the uniform parameters: a per-element test would be
  // compiled into 32 predicated address computations and loads that cost
  // more than the rest of the epilogue even when beta is 0.
  const float alpha = p.alpha, beta = p.beta;
  if (beta == 0.f) {
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = alpha * __uint_as_float(r[c]);
  } else if (p.c_sm == 0) {
    // C broadcast along rows (a bias vector): one load per lane, shuffled
    float cl = 0.f;
    if (col0 + lane < p.N) cl = load_c(p, bz * p.c_sb + (long long)(col0 + lane) * p.c_sn);
#pragma unroll
    for (int c = 0; c < 32; ++c)
      v[c] = alpha * __uint_as_float(r[c]) + beta * __shfl_sync(0xffffffffu, cl, c);
  } else {
    const bool row_ok = m < p.M;
    const long long base = bz * p.c_sb + (long long)m * p.c_sm;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      float a = alpha * __uint_as_float(r[c]);
      if (row_ok && col0 + c < p.N) a += beta * load_c(p, base + (long long)(col0 + c) * p.c_sn);
      v[c] = a;
    }
  }
}

__device__ __forceinline__ void epi_gemm(const Params& p, int bz, int mt, int col0, int row, int lane,
                                         const uint32_t (&r)[32]) {
  const int m = mt * BM + row;
  float v[32];
  gemm_values(p, bz, m, col0, lane, r, v);
  if (m >= p.M) return;
  uint16_t* base = static_cast<uint16_t*>(p.out) + bz * p.osn + (long long)m * p.osh;
  if (col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(base + col0) & 15) == 0)) {
    uint4* dst = reinterpret_cast<uint4*>(base + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[q] = make_uint4(cvt2(v[q * 8 + 0], v[q * 8 + 1]), cvt2(v[q * 8 + 2], v[q * 8 + 3]),
                          cvt2(v[q * 8 + 4], v[q * 8 + 5]), cvt2(v[q * 8 + 6], v[q * 8 + 7]));
    return;
  }
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (col0 + c < p.N) base[col0 + c] = cvt1(v[c]);
}

// split-K GEMM: fp32 partial sums of split `split`, [splits][M][N]
__device__ __forceinline__ void epi_gemm_partial(const Params& p, int split, int m, int col0,
                                                 const uint32_t (&r)[32]) {
  if (m >= p.M) return;
  float* dst = p.partial + ((long long)split * p.M + m) * p.N;
  if (col0 + 32 <= p.N && (p.N % 4) == 0) {
    float4* d4 = reinterpret_cast<float4*>(dst + col0);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      d4[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                          __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    return;
  }
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (col0 + c < p.N) dst[col0 + c] = __uint_as_float(r[c]);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int BN, int STAGES, int KIND, bool A_MN, bool B_MN, bool TS = (KIND == kGemm)>
__global__ void __launch_bounds__(kThreads, 1)
    igemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                 const __grid_constant__ CUtensorMap tma_b,
                 const __grid_constant__ CUtensorMap tma_d, const Params p) {
  constexpr int kStageBytes = Smem<BN>::kStageBytes;
  constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
  constexpr uint32_t kTmemCols = 2 * BN;  // double-buffered accumulator

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* epi_stage = smem + STAGES * kStageBytes;  // 1024-aligned: stage sizes are KB multiples
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + epi_stage_bytes<KIND, BN, TS>());
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), kEpiWarps);
    }
    mbar_init(smem_u32(mma_done), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = total_tiles(KIND, p);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ producer ------------------------------
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      int last_par[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int mt, nt, bz, tap, kb0, kb1;
        decode_tile(KIND, p, t, mt, nt, bz, tap, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, kStageBytes);
          last_par[stage] = int(phase);
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
          if constexpr (KIND == kConv) {
            const int chunk = kb / 9, tp = kb - chunk * 9;
            const int dy = tp / 3, dx = tp - dy * 3;
            load_rows<false>(sa, &tma_a, fb, chunk * BK, mt * BM + dy * p.wp + dx, p.src_im2col & 1, p.wp,
                             p.wp * p.hp);
            tma_load_3d(sb, &tma_b, fb, kb * BK, nt * BN, 0);
          } else if constexpr (KIND == kWgrad) {
            const int dy = tap / 3, dx = tap - dy * 3;
            if (p.patch_wb) {
              int x0, y0, n;
              patch_origin(p, kb, x0, y0, n);
              tma_load_4d(sa, &tma_a, fb, mt * BM, x0, y0, n);
              tma_load_4d(sa + 8192, &tma_a, fb, mt * BM + 64, x0, y0, n);
#pragma unroll
              for (int h = 0; h < BN / 64; ++h)
                tma_load_4d(sb + h * 8192, &tma_b, fb, nt * BN + h * 64, x0 + dx - 1, y0 + dy - 1, n);
            } else {
              const int plane = p.wp * p.hp;
              load_rows<false>(sa, &tma_a, fb, mt * BM, kb * BK + p.a_row_shift, p.src_im2col & 1, p.wp, plane);
              load_rows<false>(sa + 8192, &tma_a, fb, mt * BM + 64, kb * BK + p.a_row_shift, p.src_im2col & 1,
                               p.wp, plane);
#pragma unroll
              for (int h = 0; h < BN / 64; ++h)
                load_rows<false>(sb + h * 8192, &tma_b, fb, nt * BN + h * 64, kb * BK + dy * p.wp + dx,
                                 p.src_im2col & 2, p.wp, plane);
            }
          } else {
            // slice (z) and k offset of this k-block for A and B
            int za = bz, zb = bz, k0 = kb * BK;
            if (p.kb_per_batch > 0) {
              za = zb = kb / p.kb_per_batch;
              k0 = (kb - za * p.kb_per_batch) * BK;
            } else if (p.gemm_split) {
              za = zb = 0;
            }
            if (p.a_bcast) za = 0;
            if constexpr (A_MN) {
              tma_load_3d(sa, &tma_a, fb, mt * BM, k0, za);
              tma_load_3d(sa + 8192, &tma_a, fb, mt * BM + 64, k0, za);
            } else {
              tma_load_3d(sa, &tma_a, fb, k0, mt * BM, za);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int h = 0; h < BN / 64; ++h)
                tma_load_3d(sb + h * 8192, &tma_b, fb, nt * BN + h * 64, k0, zb);
            } else {
              tma_load_3d(sb, &tma_b, fb, k0, nt * BN, zb);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(smem_u32(&full[s]), uint32_t(last_par[s]), p.status, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ----------------------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      // stage-0 descriptors, stepped by offsets in 16-byte units (shared
      // addresses stay below 2^18: no carry out of the start-address field)
      const uint64_t a_desc0 = A_MN ? smem_desc_sw128(smem_u32(smem), 8192, 1024)
                                    : smem_desc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = B_MN ? smem_desc_sw128(smem_u32(smem) + kABytes, 8192, 1024)
                                    : smem_desc_sw128(smem_u32(smem) + kABytes, 16, 1024);
      constexpr uint32_t kAStep = A_MN ? 128u : 2u;  // one 16-deep k step: 16 rows or 32 bytes
      constexpr uint32_t kBStep = B_MN ? 128u : 2u;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int mt, nt, bz, tap, kb0, kb1;
        decode_tile(KIND, p, t, mt, nt, bz, tap, kb0, kb1);
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t soff = (uint32_t(stage) * uint32_t(kStageBytes)) >> 4;
          const uint32_t first = kb > kb0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_f16(d_tmem, a_desc0 + soff + kAStep * k, b_desc0 + soff + kBStep * k, kIdesc,
                       (first | uint32_t(k)) ? 1u : 0u);
          tc_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&tfull[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // All MMAs of this CTA have completed once mma_done flips.
      tc_commit(smem_u32(mma_done));
      mbar_wait(smem_u32(mma_done), 0, p.status, nullptr);
    }
    __syncwarp();
  } else {
    // -------------------------------- epilogue ------------------------------
    // 8 warps: two per tensor-memory lane quarter, each draining half of the
    // accumulator's columns.
    const int quarter = warp & 3;  // tensor-memory lane quarter this warp may read
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    constexpr int kChunks = BN / 64;  // 32-column chunks per half
    int acc = 0;
    uint32_t acc_phase = 0;
    constexpr int kBoxCols = epi_box_cols<BN>();
    constexpr int kBoxBytes = epi_box_bytes<BN>();
    uint8_t* epi_buf = epi_stage + (warp - 2) * 2 * kBoxBytes;  // GEMM output staging of this warp
    int epi_sel = 0;
    (void)epi_buf;
    (void)epi_sel;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      int mt, nt, bz, tap, kb0, kb1;
      decode_tile(KIND, p, t, mt, nt, bz, tap, kb0, kb1);
      uint16_t* obase = nullptr;
      if constexpr (KIND == kConv) obase = conv_row_base(p, mt, row);
      bool ok = mbar_wait(smem_u32(&tfull[acc]), acc_phase, p.status, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + half * (BN / 2));
      if (KIND == kGemm && TS && p.tma_store) {
        // Stage each 32-row box of the warp's columns in shared memory (the
        // swizzle puts 16-byte chunk q of row `lane` at chunk q ^ (lane & 7)
        // for 128-byte rows, q ^ ((lane >> 1) & 3) for 64-byte rows, so the
        // eight rows of each store phase hit distinct banks) and let the TMA
        // unit write it out in whole rows; rows past M / columns past N are
        // clipped by the tensor map.
        constexpr int kSub = kBoxCols / 32;
#pragma unroll 1
        for (int j = 0; j < (BN / 2) / kBoxCols; ++j) {
          const int c0 = nt * BN + half * (BN / 2) + j * kBoxCols;
          uint32_t r[kSub][32];
#pragma unroll
          for (int u = 0; u < kSub; ++u) tmem_ld32(taddr + j * kBoxCols + u * 32, r[u]);
          tc_wait_ld();
          uint32_t packed[kBoxCols / 2];
#pragma unroll
          for (int u = 0; u < kSub; ++u) {
            float v[32];
            gemm_values(p, bz, mt * BM + row, c0 + u * 32, lane, r[u], v);
#pragma unroll
            for (int c = 0; c < 16; ++c) packed[u * 16 + c] = cvt2(v[2 * c], v[2 * c + 1]);
          }
          if (lane == 0) bulk_wait_read<1>();  // this buffer's previous store has read it
          __syncwarp();
          uint8_t* buf = epi_buf + epi_sel * kBoxBytes;
#pragma unroll
          for (int q = 0; q < kBoxCols / 8; ++q) {
            const int phys = kBoxCols == 64 ? (q ^ (lane & 7)) : (q ^ ((lane >> 1) & 3));
            *reinterpret_cast<uint4*>(buf + lane * (kBoxCols * 2) + (phys << 4)) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tma_d, smem_u32(buf), c0, mt * BM + quarter * 32, bz);
            bulk_commit();
          }
          epi_sel ^= 1;
        }
      } else {
#pragma unroll 1
      for (int j = 0; j < kChunks; ++j) {
        uint32_t r[32];
        tmem_ld32(taddr + j * 32, r);
        tc_wait_ld();
        const int col0 = nt * BN + half * (BN / 2) + j * 32;
        if constexpr (KIND == kConv) {
          epi_conv(p, obase, col0, lane, r);
        } else if constexpr (KIND == kWgrad) {
          epi_wgrad(p, bz, tap, mt, col0, row, r);
        } else if (p.gemm_split) {
          epi_gemm_partial(p, bz, mt * BM + row, col0, r);
        } else {
          epi_gemm(p, bz, mt, col0, row, lane, r);
        }
      }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if constexpr (KIND == kGemm) {
      if (lane == 0) bulk_wait_all();  // stores done before the CTA's shared memory goes away
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// The SM-pair variant for the conv (fwd / dgrad) with Cout > 128: a cluster of
// two CTAs computes a 256-pixel x 256-channel tile with tcgen05.mma
// .cta_group::2 (M=256, N=256).  Each CTA TMA-loads its own 128 A rows and its
// own 128-row half of the B tile (no multicast; the loads signal the leader
// CTA's "full" barrier, which expects both CTAs' bytes), so per k-block each
// SM stages 32 KB instead of 48 KB and the ring is 6 stages deep.  The leader's
// single MMA thread issues for both SMs and commits to the "empty" / "tmem full"
// barriers of both CTAs at once; each CTA drains its own 128 accumulator rows
// (all 256 columns) and releases the accumulator buffer through the leader's
// "tmem empty" barrier.  Same bounded waits as the single-CTA kernel.
// ---------------------------------------------------------------------------
template <int STAGES, int KIND, int PBN = 256, bool A_MN = (KIND == kWgrad), bool B_MN = (KIND == kWgrad)>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    igemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                      const Params p) {
  static_assert(PBN == 256 || PBN == 128, "pair tile width");
  constexpr int BN = PBN;            // N per pair tile
  constexpr int kBHalf = PBN / 2;    // B rows each CTA loads
  constexpr int kStageBytes = kABytes + kBHalf * BK * 2;
  constexpr uint32_t kIdesc = idesc_bf16_f32(256, BN, A_MN, B_MN);
  constexpr uint32_t kTmemCols = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 2 * kEpiWarps);
    }
    mbar_init(smem_u32(mma_done), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialized before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // conv: tiles (256-pixel block, 256-channel block); wgrad: (split, 256-co
  // block, tap, 256-ci block); GEMM: (slice or split, 256-row block, PBN-column
  // block) -- as in decode_tile with M tiles of 256
  const int ntiles = KIND == kConv   ? p.tiles_m * p.tiles_n
                     : KIND == kGemm ? p.batch * p.tiles_m * p.tiles_n
                                     : p.splits * p.tiles_m * 9 * p.ci_blocks;
  auto decode = [&](int t, int& mt, int& nt, int& split, int& tap, int& kb0, int& kb1) {
    if (KIND == kGemm) {
      nt = t % p.tiles_n;
      t /= p.tiles_n;
      mt = t % p.tiles_m;
      split = t / p.tiles_m;  // batch slice, or split-K range
      tap = 0;
      kb0 = p.gemm_split ? split * p.kb_per_split : 0;
      kb1 = p.gemm_split ? min(p.num_kb, kb0 + p.kb_per_split) : p.num_kb;
    } else if (KIND == kConv) {
      nt = t % p.tiles_n;
      mt = t / p.tiles_n;
      split = 0;
      tap = 0;
      kb0 = 0;
      kb1 = p.num_kb;
    } else {
      nt = t % p.ci_blocks;
      t /= p.ci_blocks;
      tap = t % 9;
      t /= 9;
      mt = t % p.tiles_m;
      split = t / p.tiles_m;
      kb0 = split * p.kb_per_split;
      kb1 = min(p.num_kb, kb0 + p.kb_per_split);
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ producer (both CTAs) -----------------
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      int last_par[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        int mt, nt, split, tap, kb0, kb1;
        decode(t, mt, nt, split, tap, kb0, kb1);
        const int row0 = mt * 256 + int(rank) * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = smem_u32(&full[stage]);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * kStageBytes);
          last_par[stage] = int(phase);
          const uint32_t fb = mapa_shared(fb_local, 0);
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
          if constexpr (KIND == kConv) {
            const int chunk = kb / 9, tp = kb - chunk * 9;
            const int dy = tp / 3, dx = tp - dy * 3;
            load_rows<true>(sa, &tma_a, fb, chunk * BK, row0 + dy * p.wp + dx, p.src_im2col & 1, p.wp,
                            p.wp * p.hp);
            tma_load_3d_pair(sb, &tma_b, fb, kb * BK, nt * BN + int(rank) * kBHalf, 0);
          } else if constexpr (KIND == kGemm) {
            // this CTA's 128 rows of A and its half of the tile's B columns
            const int za = (p.gemm_split || p.a_bcast) ? 0 : split, zb = p.gemm_split ? 0 : split;
            const int k0 = kb * BK;
            const int n0 = nt * BN + int(rank) * kBHalf;
            if constexpr (A_MN) {
              tma_load_3d_pair(sa, &tma_a, fb, row0, k0, za);
              tma_load_3d_pair(sa + 8192, &tma_a, fb, row0 + 64, k0, za);
            } else {
              tma_load_3d_pair(sa, &tma_a, fb, k0, row0, za);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int h = 0; h < kBHalf / 64; ++h) tma_load_3d_pair(sb + h * 8192, &tma_b, fb, n0 + h * 64, k0, zb);
            } else {
              tma_load_3d_pair(sb, &tma_b, fb, k0, n0, zb);
            }
          } else {
            // A = dY rows (co contiguous), this CTA's 128 co; B = X rows shifted by the tap
            const int dy = tap / 3, dx = tap - dy * 3;
            const int ci0 = nt * BN + int(rank) * kBHalf;
            if (p.patch_wb) {
              int x0, y0, n;
              patch_origin(p, kb, x0, y0, n);
              tma_load_4d_pair(sa, &tma_a, fb, row0, x0, y0, n);
              tma_load_4d_pair(sa + 8192, &tma_a, fb, row0 + 64, x0, y0, n);
              tma_load_4d_pair(sb, &tma_b, fb, ci0, x0 + dx - 1, y0 + dy - 1, n);
              tma_load_4d_pair(sb + 8192, &tma_b, fb, ci0 + 64, x0 + dx - 1, y0 + dy - 1, n);
            } else {
              const int plane = p.wp * p.hp;
              const bool ia = p.src_im2col & 1, ib = p.src_im2col & 2;
              load_rows<true>(sa, &tma_a, fb, row0, kb * BK + p.a_row_shift, ia, p.wp, plane);
              load_rows<true>(sa + 8192, &tma_a, fb, row0 + 64, kb * BK + p.a_row_shift, ia, p.wp, plane);
              load_rows<true>(sb, &tma_b, fb, ci0, kb * BK + dy * p.wp + dx, ib, p.wp, plane);
              load_rows<true>(sb + 8192, &tma_b, fb, ci0 + 64, kb * BK + dy * p.wp + dx, ib, p.wp, plane);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && leader) {
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(smem_u32(&full[s]), uint32_t(last_par[s]), p.status, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------ MMA issuer (leader CTA) --------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        int mt, nt, split, tap, kb0, kb1;
        decode(t, mt, nt, split, tap, kb0, kb1);
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc_sw128(sa + k * 2048, 8192, 1024) : smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(sb + k * 2048, 8192, 1024) : smem_desc_sw128(sb + k * 32, 16, 1024);
            tc_mma_pair(d_tmem, ad, bd, kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(smem_u32(&empty[stage]), uint16_t(0x3));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair_mc(smem_u32(&tfull[acc]), uint16_t(0x3));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      tc_commit_pair(smem_u32(mma_done));
      mbar_wait(smem_u32(mma_done), 0, p.status, nullptr);
    }
    __syncwarp();
  } else {
    // -------------------------------- epilogue (both CTAs) ------------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    constexpr int kChunks = BN / 64;
    const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty[0]), 0), mapa_shared(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < ntiles; t += nclusters) {
      int mt, nt, split, tap, kb0, kb1;
      decode(t, mt, nt, split, tap, kb0, kb1);
      const int grow = mt * 256 + int(rank) * 128 + row;  // pixel (conv) or co (wgrad) of this thread
      uint16_t* obase = nullptr;
      if constexpr (KIND == kConv) obase = conv_row_base_at(p, grow);
      bool ok = mbar_wait(smem_u32(&tfull[acc]), acc_phase, p.status, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + half * (BN / 2));
#pragma unroll 1
      for (int j = 0; j < kChunks; ++j) {
        uint32_t r[32];
        tmem_ld32(taddr + j * 32, r);
        tc_wait_ld();
        const int col0 = nt * BN + half * (BN / 2) + j * 32;
        if constexpr (KIND == kConv)
          epi_conv(p, obase, col0, lane, r);
        else if constexpr (KIND == kGemm) {
          if (p.gemm_split)
            epi_gemm_partial(p, split, grow, col0, r);
          else
            epi_gemm(p, split, mt * 2 + int(rank), col0, row, lane, r);
        } else
          epi_wgrad_co(p, split, tap, grow, col0, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(smem_u32(&tempty[acc]));
        else
          mbar_arrive_remote(tempty_leader[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its pair may still signal or read it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}


// Row offset of tap (dy, dx) = (tap / 3, tap % 3) in a padded grid of row pitch wp.
__device__ __forceinline__ int tap_shift(int tap, int wp) {
  const int dy = tap / 3;
  return dy * wp + (tap - dy * 3);
}

// ---------------------------------------------------------------------------
// The SM-pair conv kernel with the A halo loaded once per 64-channel chunk.
// The nine taps of a chunk read the same padded rows shifted by dy*(W+2)+dx,
// so each CTA loads one window of 128 + 2*(W+2) + 2 rows per chunk into a
// double-buffered A slot and the MMA takes tap (dy, dx) as a descriptor that
// starts that many rows into the window (the 128-byte swizzle phase follows
// the address, so any row start works); only B (this CTA's 128
// rows of the tap's weight slice) streams per tap, through an NB-deep ring.
// Per k-block an SM stages 16 KB instead of 32 KB, cutting the L2-to-SM
// traffic of the wide convolutions (3.23 GB per launch at B64 C256 72x72).
// Barriers, bounded waits, TMEM handling and the epilogue are those of
// igemm_pair_kernel.  (A 128-wide version for 65-128 output channels, M=256
// x N=128 pair MMAs with a 6- or a 12-deep B ring, measured 3-7 % slower than
// the single-CTA kernel there, although it moves 2.7x fewer bytes from L2.)
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    igemm_pair_halo_kernel(const __grid_constant__ CUtensorMap tma_win, const __grid_constant__ CUtensorMap tma_b,
                           const Params p) {
  constexpr int BN = 256;
  constexpr int kBHalf = 128;
  constexpr uint32_t kBBytes = kBHalf * BK * 2;  // 16 KB
  constexpr uint32_t kIdesc = idesc_bf16_f32(256, BN, false, false);
  constexpr uint32_t kTmemCols = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t box_bytes = uint32_t(p.win_box_rows) * 128u;
  const uint32_t a_bytes = uint32_t(p.win_boxes) * box_bytes;  // one A window slot (1024-byte multiple)
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + 2 * a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + NB * kBBytes);
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + 2;
  uint64_t* b_full = bars + 4;
  uint64_t* b_empty = b_full + NB;
  uint64_t* tfull = b_empty + NB;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  const int chunks = p.num_kb / 9;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&a_full[s]), 1);
      mbar_init(smem_u32(&a_empty[s]), 1);
      mbar_init(smem_u32(&tfull[s]), 1);
      mbar_init(smem_u32(&tempty[s]), 2 * kEpiWarps);
    }
    for (int s = 0; s < NB; ++s) {
      mbar_init(smem_u32(&b_full[s]), 1);
      mbar_init(smem_u32(&b_empty[s]), 1);
    }
    mbar_init(smem_u32(mma_done), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ producer (both CTAs) -----------------
      tma_prefetch_desc(&tma_win);
      tma_prefetch_desc(&tma_b);
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      int a_last[2] = {-1, -1};
      int b_last[NB];
#pragma unroll
      for (int s = 0; s < NB; ++s) b_last[s] = -1;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        const int nt = t % p.tiles_n, mt = t / p.tiles_n;
        const int row0 = mt * 256 + int(rank) * 128;
        for (int ch = 0; ch < chunks && ok; ++ch) {
          if (!mbar_wait(smem_u32(&a_empty[as]), aph ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fa_local = smem_u32(&a_full[as]);
          if (leader) mbar_arrive_expect_tx(fa_local, 2 * a_bytes);
          a_last[as] = int(aph);
          const uint32_t fa = mapa_shared(fa_local, 0);
          const uint32_t sa = smem_u32(a_base + as * a_bytes);
          for (int i = 0; i < p.win_boxes; ++i)
            load_rows<true>(sa + i * box_bytes, &tma_win, fa, ch * BK, row0 + i * p.win_box_rows, p.src_im2col & 1,
                            p.wp, p.wp * p.hp);
          if (++as == 2) {
            as = 0;
            aph ^= 1;
          }
          for (int tap = 0; tap < 9; ++tap) {
            if (!mbar_wait(smem_u32(&b_empty[bs]), bph ^ 1, p.status, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t fb_local = smem_u32(&b_full[bs]);
            if (leader) mbar_arrive_expect_tx(fb_local, 2 * kBBytes);
            b_last[bs] = int(bph);
            const uint32_t fb = mapa_shared(fb_local, 0);
            tma_load_3d_pair(smem_u32(b_base + bs * kBBytes), &tma_b, fb, (ch * 9 + tap) * BK,
                             nt * BN + int(rank) * kBHalf, 0);
            if (++bs == NB) {
              bs = 0;
              bph ^= 1;
            }
          }
        }
      }
      if (!ok && leader) {
        for (int s = 0; s < 2; ++s)
          if (a_last[s] >= 0) mbar_wait(smem_u32(&a_full[s]), uint32_t(a_last[s]), p.status, nullptr);
        for (int s = 0; s < NB; ++s)
          if (b_last[s] >= 0) mbar_wait(smem_u32(&b_full[s]), uint32_t(b_last[s]), p.status, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------ MMA issuer (leader CTA) --------------
      int as = 0, bs = 0, acc = 0;
      uint32_t aph = 0, bph = 0, acc_phase = 0;
      bool ok = true;
      const uint64_t a_desc0 = smem_desc_sw128(smem_u32(a_base), 16, 1024);
      const uint64_t b_desc0 = smem_desc_sw128(smem_u32(b_base), 16, 1024);
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int ch = 0; ch < chunks && ok; ++ch) {
          if (!mbar_wait(smem_u32(&a_full[as]), aph, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors stepped by offsets in 16-byte units (window row =
          // 8 units); shared addresses stay below 2^18
          const uint64_t a_desc = a_desc0 + uint64_t((uint32_t(as) * a_bytes) >> 4);
          for (int tap = 0; tap < 9; ++tap) {
            if (!mbar_wait(smem_u32(&b_full[bs]), bph, p.status, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = a_desc + uint32_t(tap_shift(tap, p.wp)) * 8u;
            const uint64_t bd = b_desc0 + (uint32_t(bs) * kBBytes >> 4);
            const uint32_t first = (ch > 0 || tap > 0) ? 1u : 0u;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              tc_mma_pair(d_tmem, ad + uint32_t(2 * k), bd + uint32_t(2 * k), kIdesc, (first | uint32_t(k)) ? 1u : 0u);
            tc_commit_pair_mc(smem_u32(&b_empty[bs]), uint16_t(0x3));
            if (++bs == NB) {
              bs = 0;
              bph ^= 1;
            }
          }
          if (!ok) break;
          tc_commit_pair_mc(smem_u32(&a_empty[as]), uint16_t(0x3));
          if (++as == 2) {
            as = 0;
            aph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair_mc(smem_u32(&tfull[acc]), uint16_t(0x3));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      tc_commit_pair(smem_u32(mma_done));
      mbar_wait(smem_u32(mma_done), 0, p.status, nullptr);
    }
    __syncwarp();
  } else {
    // -------------------------------- epilogue (both CTAs) ------------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    constexpr int kChunks = BN / 64;
    const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty[0]), 0), mapa_shared(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < ntiles; t += nclusters) {
      const int nt = t % p.tiles_n, mt = t / p.tiles_n;
      uint16_t* obase = conv_row_base_at(p, mt * 256 + int(rank) * 128 + row);
      bool ok = mbar_wait(smem_u32(&tfull[acc]), acc_phase, p.status, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + half * (BN / 2));
#pragma unroll 1
      for (int j = 0; j < kChunks; ++j) {
        uint32_t r[32];
        tmem_ld32(taddr + j * 32, r);
        tc_wait_ld();
        epi_conv(p, obase, nt * BN + half * (BN / 2) + j * 32, lane, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(smem_u32(&tempty[acc]));
        else
          mbar_arrive_remote(tempty_leader[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}



// Narrow convolutions (Cin <= 64, Cout <= 64) with the weights resident: a
// 64-wide output tile needs 9 taps x 64 x 64 weights (72 KB), the same for
// every tile, and a 128-row tile of one 64-channel chunk does only 1152
// cycles of MMA work.  Streaming A per tap and B per tile moved 216 KB per
// tile through L2, more than the TMA pipeline's bytes in flight can cover at
// that MMA rate.  Here each persistent CTA loads the whole weight slice once,
// then streams only the padded input window of each tile (128 + 2(W+2) + 2
// rows, loaded once and read by all nine taps as row-shifted descriptors,
// as in the SM-pair halo kernel), with as many windows in flight as shared
// memory holds.
constexpr int kMaxWinBufs = 6;

__global__ void __launch_bounds__(kThreads, 1)
    igemm_halo_bres_kernel(const __grid_constant__ CUtensorMap tma_win, const __grid_constant__ CUtensorMap tma_b,
                           const Params p) {
  constexpr int BN = 64;
  constexpr uint32_t kTapBytes = BN * BK * 2;  // 8 KB
  constexpr uint32_t kWBytes = 9 * kTapBytes;  // 72 KB
  constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, false, false);
  constexpr uint32_t kTmemCols = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int NW = p.win_bufs;
  const uint32_t box_bytes = uint32_t(p.win_box_rows) * 128u;
  const uint32_t a_bytes = uint32_t(p.win_boxes) * box_bytes;
  uint8_t* w_base = smem;
  uint8_t* a_base = smem + kWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(a_base + NW * a_bytes);
  uint64_t* w_full = bars;
  uint64_t* a_full = bars + 1;
  uint64_t* a_empty = a_full + kMaxWinBufs;
  uint64_t* tfull = a_empty + kMaxWinBufs;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(w_full), 1);
    for (int s = 0; s < NW; ++s) {
      mbar_init(smem_u32(&a_full[s]), 1);
      mbar_init(smem_u32(&a_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&tfull[s]), 1);
      mbar_init(smem_u32(&tempty[s]), kEpiWarps);
    }
    mbar_init(smem_u32(mma_done), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = p.tiles_m;  // one 64-wide column tile

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ producer ------------------------------
      tma_prefetch_desc(&tma_win);
      tma_prefetch_desc(&tma_b);
      const uint32_t fw = smem_u32(w_full);
      mbar_arrive_expect_tx(fw, kWBytes);
      for (int tap = 0; tap < 9; ++tap) tma_load_3d(smem_u32(w_base + tap * kTapBytes), &tma_b, fw, tap * BK, 0, 0);
      int as = 0;
      uint32_t aph = 0;
      int a_last[kMaxWinBufs];
      for (int s = 0; s < kMaxWinBufs; ++s) a_last[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        if (!mbar_wait(smem_u32(&a_empty[as]), aph ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fa = smem_u32(&a_full[as]);
        mbar_arrive_expect_tx(fa, a_bytes);
        a_last[as] = int(aph);
        const uint32_t sa = smem_u32(a_base + as * a_bytes);
        for (int i = 0; i < p.win_boxes; ++i)
          load_rows<false>(sa + i * box_bytes, &tma_win, fa, 0, t * BM + i * p.win_box_rows, p.src_im2col & 1, p.wp,
                           p.wp * p.hp);
        if (++as == NW) {
          as = 0;
          aph ^= 1;
        }
      }
      // the weights and every issued window land before the CTA may exit
      mbar_wait(fw, 0, p.status, nullptr);
      if (!ok)
        for (int s = 0; s < NW; ++s)
          if (a_last[s] >= 0) mbar_wait(smem_u32(&a_full[s]), uint32_t(a_last[s]), p.status, nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ----------------------------
      int as = 0, acc = 0;
      uint32_t aph = 0, acc_phase = 0;
      bool ok = mbar_wait(smem_u32(w_full), 0, p.status, abort_flag);
      tc_fence_after();
      // At 64 output columns an MMA is ~32 cycles of tensor work, so the
      // issuing thread must not rebuild descriptors per instruction: build
      // them once and step them by offsets (the start-address field counts 16
      // bytes; every shared-memory address here is below 2^18, so additions
      // never carry out of the field).
      const uint64_t a_desc0 = smem_desc_sw128(smem_u32(a_base), 16, 1024);
      const uint64_t w_desc0 = smem_desc_sw128(smem_u32(w_base), 16, 1024);
      uint32_t a_off[9];
#pragma unroll
      for (int tap = 0; tap < 9; ++tap) a_off[tap] = uint32_t(tap_shift(tap, p.wp)) * 8u;  // rows of 128 B
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        if (!mbar_wait(smem_u32(&a_full[as]), aph, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        const uint64_t a_desc = a_desc0 + uint64_t((uint32_t(as) * a_bytes) >> 4);
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_f16(d_tmem, a_desc + a_off[tap] + uint32_t(2 * k), w_desc0 + uint32_t((tap * kTapBytes + k * 32) >> 4),
                       kIdesc, (tap > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&a_empty[as]));
        if (++as == NW) {
          as = 0;
          aph ^= 1;
        }
        tc_commit(smem_u32(&tfull[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      tc_commit(smem_u32(mma_done));
      mbar_wait(smem_u32(mma_done), 0, p.status, nullptr);
    }
    __syncwarp();
  } else {
    // -------------------------------- epilogue ------------------------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      uint16_t* obase = conv_row_base(p, t, row);
      bool ok = mbar_wait(smem_u32(&tfull[acc]), acc_phase, p.status, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + half * (BN / 2));
      uint32_t r[32];
      tmem_ld32(taddr, r);
      tc_wait_ld();
      epi_conv(p, obase, half * (BN / 2), lane, r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}


// Weight gradient of narrow convolutions (Cin <= 64, Cout <= 64).  The tiled
// wgrad kernel runs one tile per tap, so each 64-pixel k-block reloads dY and
// X for every tap, and a 64-channel Cout fills only half of its 128-row MMA.
// Here a persistent CTA owns a range of 128-pixel k-blocks (split-K) and all
// nine taps: per k-block it loads the dY block once (128 pixels x 64 output
// channels) and the input window once (128 + 2(W+2) + 2 padded rows x 64
// input channels).  The MMA's M rows are two taps' input channels: rows 0-63
// read the window `s1` rows in, rows 64-127 `s2` rows in (the two 64-element
// halves of an M-major operand sit the descriptor's leading byte offset
// apart, here (s2 - s1) rows).  Taps pair as (0,1) (2,3) (4,5) (6,7) (7,8);
// the last accumulator keeps only its tap-8 half.  Five 128 x 64 fp32
// accumulators (320 TMEM columns) hold the CTA's sums until its last k-block;
// the epilogue writes them as this split's partials [split][tap][co][ci],
// which wgrad_reduce_kernel adds in split order.
constexpr int kNarrowWgradPix = 128;  // pixels (padded rows) per k-block

__global__ void __launch_bounds__(kThreads, 1)
    igemm_wgrad_narrow_kernel(const __grid_constant__ CUtensorMap tma_dy, const __grid_constant__ CUtensorMap tma_x,
                              const Params p) {
  constexpr int BN = 64;
  constexpr uint32_t kDyBytes = kNarrowWgradPix * 128;  // 16 KB
  constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, true, true);
  constexpr uint32_t kTmemCols = 512;  // 5 x 64 used

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int NS = p.win_bufs;
  const uint32_t box_bytes = uint32_t(p.win_box_rows) * 128u;
  const uint32_t stage_bytes = kDyBytes + uint32_t(p.win_boxes) * box_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = full + kMaxWinBufs;
  uint64_t* tfull = empty + kMaxWinBufs;
  uint64_t* mma_done = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int split = blockIdx.x;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(tfull), 1);
    mbar_init(smem_u32(mma_done), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ producer ------------------------------
      tma_prefetch_desc(&tma_dy);
      tma_prefetch_desc(&tma_x);
      int st = 0;
      uint32_t ph = 0;
      int last[kMaxWinBufs];
      for (int s = 0; s < kMaxWinBufs; ++s) last[s] = -1;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(smem_u32(&empty[st]), ph ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t f = smem_u32(&full[st]);
        mbar_arrive_expect_tx(f, stage_bytes);
        last[st] = int(ph);
        const uint32_t sd = smem_u32(smem + st * stage_bytes);
        const int row0 = kb * kNarrowWgradPix;
        load_rows<false>(sd, &tma_dy, f, 0, row0 + p.a_row_shift, p.src_im2col & 1, p.wp, p.wp * p.hp);
        for (int i = 0; i < p.win_boxes; ++i)
          load_rows<false>(sd + kDyBytes + i * box_bytes, &tma_x, f, 0, row0 + i * p.win_box_rows, p.src_im2col & 2,
                           p.wp, p.wp * p.hp);
        if (++st == NS) {
          st = 0;
          ph ^= 1;
        }
      }
      if (!ok)
        for (int s = 0; s < NS; ++s)
          if (last[s] >= 0) mbar_wait(smem_u32(&full[s]), uint32_t(last[s]), p.status, nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ----------------------------
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      // descriptors built once for stage 0 and stepped by offsets (see the
      // resident-weight kernel): per tap pair its window start s1 and the
      // leading byte offset (s2 - s1) rows to the second tap's half
      uint64_t a_desc0[5];
#pragma unroll
      for (int a = 0; a < 5; ++a) {
        const int s1 = tap_shift(a < 4 ? 2 * a : 7, p.wp);
        const int s2 = tap_shift(a < 4 ? 2 * a + 1 : 8, p.wp);
        a_desc0[a] = smem_desc_sw128(smem_u32(smem) + kDyBytes + uint32_t(s1) * 128u, uint32_t(s2 - s1) * 128u, 1024);
      }
      const uint64_t d_desc0 = smem_desc_sw128(smem_u32(smem), 8192, 1024);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(smem_u32(&full[st]), ph, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t soff = (uint32_t(st) * stage_bytes) >> 4;
        const uint32_t first = kb > kb0 ? 1u : 0u;
#pragma unroll
        for (int a = 0; a < 5; ++a) {
#pragma unroll
          for (int k = 0; k < kNarrowWgradPix / 16; ++k)
            tc_mma_f16(tmem_base + uint32_t(a * BN), a_desc0[a] + soff + uint32_t(128 * k),
                       d_desc0 + soff + uint32_t(128 * k), kIdesc, (first | uint32_t(k)) ? 1u : 0u);
        }
        tc_commit(smem_u32(&empty[st]));
        if (++st == NS) {
          st = 0;
          ph ^= 1;
        }
      }
      if (ok) tc_commit(smem_u32(tfull));
      tc_commit(smem_u32(mma_done));
      mbar_wait(smem_u32(mma_done), 0, p.status, nullptr);
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // -------------------------------- epilogue ------------------------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int ci = row & 63;
    bool ok = kb1 > kb0 && mbar_wait(smem_u32(tfull), 0, p.status, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int a = 0; a < 5; ++a) {
        if (a == 4 && row < 64) continue;  // the duplicate tap-7 half (warp-uniform)
        const int tap = a < 4 ? 2 * a + (row >> 6) : 8;
        uint32_t r[32];
        tmem_ld32(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(a * BN + half * 32), r);
        tc_wait_ld();
        if (ci < p.N) {
          float* dst = p.partial + ((long long)split * 9 + tap) * p.M * p.N + ci;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int co = half * 32 + c;
            if (co < p.M) dst[(long long)co * p.N] = __uint_as_float(r[c]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Deterministic split-K reduction: dw[co][ci][tap] = sum_s partial[s][tap][co][ci].
// D[m][n] = alpha * (partial[0][m][n] + partial[1][m][n] + ...), in split order.
// The same sum four columns at a time (N % 4 == 0, 16-byte aligned partials;
// D rows aligned for 8-byte bf16 or 16-byte fp32 stores): a 2-D grid of
// column groups x rows, no 64-bit index division, every split's load of a
// group issued before the additions, which run in split order from +0.
__global__ void __launch_bounds__(256) gemm_split_reduce_vec_kernel(const float4* __restrict__ partial, int splits,
                                                                    int M, int N4, float alpha, void* D, int d_dtype,
                                                                    long long ldd, float beta, const void* C,
                                                                    int c_dtype, long long c_sm, long long c_sn) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= N4) return;
  const long long plane4 = (long long)M * N4;
  for (int m = blockIdx.y; m < M; m += gridDim.y) {
    const long long i = (long long)m * N4 + q;
    float4 v[8];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < splits; k0 += 8) {
      const int nk = splits - k0 < 8 ? splits - k0 : 8;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nk) v[k] = __ldg(partial + (long long)(k0 + k) * plane4 + i);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nk) {
          acc.x += v[k].x;
          acc.y += v[k].y;
          acc.z += v[k].z;
          acc.w += v[k].w;
        }
    }
    float r[4] = {acc.x * alpha, acc.y * alpha, acc.z * alpha, acc.w * alpha};
    const long long n0 = 4LL * q;
    if (beta != 0.f) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const long long ci = m * c_sm + (n0 + e) * c_sn;
        r[e] += beta * (c_dtype == B2_F32 ? static_cast<const float*>(C)[ci]
                                          : bf2f(static_cast<const uint16_t*>(C)[ci]));
      }
    }
    if (d_dtype == B2_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(D) + m * ldd + n0) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(D) + m * ldd + n0) =
          make_uint2(pack_bf2(r[0], r[1]), pack_bf2(r[2], r[3]));
    }
  }
}

__global__ void gemm_split_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N, float alpha,
                                         void* D, int d_dtype, long long ldd, float beta = 0.f,
                                         const void* C = nullptr, int c_dtype = B2_BF16, long long c_sm = 0,
                                         long long c_sn = 0) {
  const long long total = (long long)M * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += partial[k * total + i];
    s *= alpha;
    const long long m = i / N, n = i - m * N;
    if (beta != 0.f) {
      const long long ci = m * c_sm + n * c_sn;
      s += beta * (c_dtype == B2_F32 ? static_cast<const float*>(C)[ci] : bf2f(static_cast<const uint16_t*>(C)[ci]));
    }
    if (d_dtype == B2_F32)
      static_cast<float*>(D)[m * ldd + n] = s;
    else
      static_cast<uint16_t*>(D)[m * ldd + n] = f2bf(s);
  }
}

// ohwi: dw in [Cout][3][3][Cin] order (a channels-last weight's layout),
// which also reads the [tap][Cout][Cin] partials contiguously; otherwise OIHW.
// Same sums, in the same split order, either way.
__global__ void wgrad_reduce_kernel(const float* __restrict__ partial, void* dw, int dtype,
                                    int splits, int Cout, int Cin, bool ohwi = false) {
  const long long total = (long long)Cout * Cin * 9;
  const long long plane = (long long)9 * Cout * Cin;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int tap, ci, co;
    if (ohwi) {
      ci = int(i % Cin);
      const long long ct = i / Cin;
      tap = int(ct % 9);
      co = int(ct / 9);
    } else {
      tap = int(i % 9);
      const long long oc = i / 9;
      ci = int(oc % Cin);
      co = int(oc / Cin);
    }
    const float* src = partial + ((long long)tap * Cout + co) * Cin + ci;
    // eight splits' loads issued together, then added in split order (the
    // same sums as one load per add, without a load latency per split)
    float s = 0.f;
    for (int k0 = 0; k0 < splits; k0 += 8) {
      const int nk = splits - k0 < 8 ? splits - k0 : 8;
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = k < nk ? __ldg(src + (long long)(k0 + k) * plane) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nk) s += v[k];
    }
    if (dtype == B2_F32)
      static_cast<float*>(dw)[i] = s;
    else
      static_cast<uint16_t*>(dw)[i] = f2bf(s);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int BN, int STAGES, int KIND, bool TS = (KIND == kGemm)>
constexpr size_t smem_bytes() {
  return size_t(STAGES) * Smem<BN>::kStageBytes + epi_stage_bytes<KIND, BN, TS>() + 1024 /*align*/ + 256 /*barriers*/;
}

template <int BN, int STAGES, int KIND, bool A_MN, bool B_MN, bool TS = (KIND == kGemm)>
b2_status launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int tiles,
                 cudaStream_t st, const CUtensorMap* td = nullptr) {
  auto kern = igemm_kernel<BN, STAGES, KIND, A_MN, B_MN, TS>;
  constexpr size_t smem = smem_bytes<BN, STAGES, KIND, TS>();
  static_assert(smem <= 232448, "shared memory per block");
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[dev]) {
    B2_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                      "cudaFuncSetAttribute(smem)"));
    configured[dev] = true;
  }
  if (tiles <= 0) return B2_OK;
  const int grid = std::min(tiles, sm_count(dev));
  static const CUtensorMap kNoMap{};  // kinds without a TMA store never read it
  Params q = p;
  if (!TS) q.tma_store = 0;
  kern<<<grid, kThreads, smem, st>>>(ta, tb, td ? *td : kNoMap, q);
  return check_cuda(cudaGetLastError(), "igemm launch");
}

constexpr int kStages64 = 8;
constexpr int kStages128 = 6;
constexpr int kStages256 = 4;
// the GEMM kind gives up operand stages for its output staging
constexpr int kGemmStages64 = 8;
constexpr int kGemmStages128 = 5;
constexpr int kGemmStages256 = 3;
constexpr int kGemmDeep64 = 9;  // without the store staging
constexpr int kGemmDeep128 = 7;
constexpr int kGemmDeep256 = 4;
constexpr int kStagesPair = 6;

template <int KIND, int PBN = 256, bool A_MN = (KIND == kWgrad), bool B_MN = (KIND == kWgrad)>
b2_status launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int tiles, cudaStream_t st) {
  // 128-wide pair tiles stage 24 KB per k-block: two more stages fit
  constexpr int kSt = PBN == 256 ? kStagesPair : kStagesPair + 2;
  auto kern = igemm_pair_kernel<kSt, KIND, PBN, A_MN, B_MN>;
  constexpr size_t smem = size_t(kSt) * (kABytes + (PBN / 2) * BK * 2) + 1024 + 256;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[dev]) {
    B2_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                      "cudaFuncSetAttribute(smem, pair)"));
    configured[dev] = true;
  }
  if (tiles <= 0) return B2_OK;
  const int clusters = std::min(tiles, sm_count(dev) / 2);
  kern<<<2 * clusters, kThreads, smem, st>>>(ta, tb, p);
  return check_cuda(cudaGetLastError(), "igemm pair launch");
}

constexpr int kHaloB = 6;                       // B ring depth of the halo kernel
constexpr size_t kHaloMaxSmem = 227 * 1024;

// Window geometry of the halo kernel for padded width wp: TMA boxes of at most
// 256 rows, each a multiple of 8 rows; 0 boxes when the window and a ring of
// `b_ring_bytes` do not fit in shared memory.  (Single-CTA versions of the
// kernel, with a 6-deep and with a 10-24-deep B ring, were measured 3-8 %
// slower than the per-tap loads on 64- and 128-channel layers: there the MMA
// issue rate of the narrow tiles binds, not L2.)
void halo_window(int wp, size_t b_ring_bytes, int& boxes, int& box_rows) {
  const int need = 128 + 2 * wp + 2;
  boxes = (need + 255) / 256;
  box_rows = ((need + boxes - 1) / boxes + 7) / 8 * 8;
  const size_t smem = 2 * size_t(boxes) * box_rows * 128 + b_ring_bytes + 1024 + 512;
  if (smem > kHaloMaxSmem) boxes = 0;
}

// Resident-weight halo launch (Cin <= 64, Cout <= 64): the 72 KB weight
// slice plus p.win_bufs windows of the geometry halo_window gave.
constexpr size_t kBresWeightBytes = 9 * 64 * BK * 2;

int bres_window_buffers(int win_bytes) {
  if (win_bytes <= 0) return 0;
  const size_t room = kHaloMaxSmem - kBresWeightBytes - 1024 - 256;
  const int n = int(std::min<size_t>(kMaxWinBufs, room / size_t(win_bytes)));
  return n >= 2 ? n : 0;
}

b2_status launch_halo_bres(const CUtensorMap& twin, const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  const size_t smem = kBresWeightBytes + size_t(p.win_bufs) * p.win_boxes * p.win_box_rows * 128 + 1024 + 256;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[dev]) {  // once, at the largest size accepted
    B2_TRY(check_cuda(cudaFuncSetAttribute(igemm_halo_bres_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(kHaloMaxSmem)),
                      "cudaFuncSetAttribute(smem, halo bres)"));
    configured[dev] = true;
  }
  if (p.tiles_m <= 0) return B2_OK;
  igemm_halo_bres_kernel<<<std::min(p.tiles_m, sm_count(dev)), kThreads, smem, st>>>(twin, tb, p);
  return check_cuda(cudaGetLastError(), "igemm halo bres launch");
}

b2_status launch_pair_halo(const CUtensorMap& twin, const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  auto kern = igemm_pair_halo_kernel<kHaloB>;
  const size_t smem = 2 * size_t(p.win_boxes) * p.win_box_rows * 128 + size_t(kHaloB) * 128 * BK * 2 + 1024 + 512;
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[dev]) {  // once, at the largest window accepted
    B2_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kHaloMaxSmem)),
                      "cudaFuncSetAttribute(smem, pair halo)"));
    configured[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  if (tiles <= 0) return B2_OK;
  const int clusters = std::min(tiles, sm_count(dev) / 2);
  kern<<<2 * clusters, kThreads, smem, st>>>(twin, tb, p);
  return check_cuda(cudaGetLastError(), "igemm pair halo launch");
}

// The halo kernel for wide convolutions unless B2_CONV_HALO=0 (A/B switch).
bool halo_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_CONV_HALO");
    return !e || e[0] != '0';
  }();
  return on;
}

// Resident-weight halo kernel for Cin <= 64, Cout <= 64 unless B2_CONV_BRES=0
// (A/B switch; 1.3-1.5x the per-tap kernel on 32- and 64-channel layers).
bool bres_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_CONV_BRES");
    return !(e && e[0] == '0') && halo_enabled();
  }();
  return on;
}

// All-taps weight-gradient kernel for Cin, Cout <= 64 unless B2_WGRAD_NARROW=0.
bool narrow_wgrad_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_WGRAD_NARROW");
    return !(e && e[0] == '0') && halo_enabled();
  }();
  return on;
}

// Pixel-patch k-blocks for the weight gradient of channels-last operands
// unless B2_WGRAD_PATCH=0 (A/B switch: the im2col padded-row k-blocks).
bool patch_wgrad_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_WGRAD_PATCH");
    return !e || e[0] != '0';
  }();
  return on;
}

// SM-pair tiles for GEMMs only with B2_GEMM_PAIR=1: measured on B200 they
// run no faster than the single-CTA tiles on the MLP's shapes (M = 512:
// 27 us for 512 x 4096 x 4096 either way, 12.4 against 10.6 us for the
// weight gradients; ncu: both latency-bound, tensor pipe ~47 % of active
// cycles with L2 at 23-27 % of peak), so they are off by default.
bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_GEMM_PAIR");
    return e && e[0] == '1';
  }();
  return on;
}

template <int BN, int STAGES, bool TS>
b2_status launch_gemm(bool amn, bool bmn, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int tiles,
                      cudaStream_t st, const CUtensorMap* td) {
  if (!amn && !bmn) return launch<BN, STAGES, kGemm, false, false, TS>(ta, tb, p, tiles, st, td);
  if (!amn && bmn) return launch<BN, STAGES, kGemm, false, true, TS>(ta, tb, p, tiles, st, td);
  if (amn && !bmn) return launch<BN, STAGES, kGemm, true, false, TS>(ta, tb, p, tiles, st, td);
  return launch<BN, STAGES, kGemm, true, true, TS>(ta, tb, p, tiles, st, td);
}

// SM-pair MMA for wide convolutions unless B2_PAIR_MMA=0 (A/B switch).
bool pair_mma_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_PAIR_MMA");
    return !e || e[0] != '0';
  }();
  return on;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// An activation operand of the conv kernels: padded-grid rows written by
// b2_pack_rows_bf16, or a channels-last tensor (channel stride 1, element
// strides sn / sh / sw) read through an im2col map whose pixel box is the
// padded grid -- the kernels see the same rows either way.
struct ActSrc {
  const void* ptr = nullptr;
  bool nhwc = false;
  int64_t sn = 0, sh = 0, sw = 0;
};

ActSrc rows_src(const void* rows) {
  ActSrc a;
  a.ptr = rows;
  return a;
}

// The stride of a dimension of size 1 is never used to address an element
// (frameworks leave any value there, e.g. 1): give such dimensions the
// dense stride so they pass the TMA stride rules.
void normalize_act(ActSrc& a, int B, int C, int H, int W) {
  if (!a.nhwc) return;
  if (W == 1) a.sw = C;
  if (H == 1) a.sh = int64_t(W) * a.sw;
  if (B == 1) a.sn = int64_t(H) * a.sh;
}

b2_status check_act(const ActSrc& a, int C, const char* name, const char* what) {
  if (!a.ptr) return set_error(B2_ERR_INVALID, "%s: null %s", name, what);
  if (!aligned16(a.ptr)) return set_error(B2_ERR_INVALID, "%s: %s must be 16-byte aligned", name, what);
  if (a.nhwc && (C % 8 || a.sn % 8 || a.sh % 8 || a.sw % 8 || a.sn <= 0 || a.sh <= 0 || a.sw < C))
    return set_error(B2_ERR_UNSUPPORTED,
                     "%s: channels-last %s needs C %% 8 == 0 and pixel strides that are multiples of 8 elements",
                     name, what);
  return B2_OK;
}

// A map of `box_rows` padded-grid rows x 64 channels over operand `a`.
b2_status rows_map(CUtensorMap* m, const ActSrc& a, int B, int C, int H, int W, uint32_t box_rows) {
  if (a.nhwc) return encode_tmap_padded_nhwc(m, a.ptr, B, C, H, W, a.sn, a.sh, a.sw, box_rows);
  const uint64_t cpad = uint64_t((C + 63) / 64) * 64;
  const uint64_t m_total = uint64_t(B) * uint64_t(H + 2) * uint64_t(W + 2);
  const uint64_t dims[3] = {cpad, m_total, 1};
  const uint64_t strides[2] = {cpad * 2, cpad * 2 * m_total};
  const uint32_t box[3] = {64, box_rows, 1};
  return encode_tmap(m, a.ptr, 3, dims, strides, box, true);
}

b2_status conv_common(ActSrc xs, const void* wk, const uint16_t* bias, void* y, int64_t sn,
                      int64_t sc, int64_t sh, int64_t sw, int B, int Cin, int H, int W, int Cout,
                      int relu, cudaStream_t st, const char* name) {
  if (!wk || !y) return set_error(B2_ERR_INVALID, "%s: null pointer", name);
  if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0)
    return set_error(B2_ERR_INVALID, "%s: bad shape B=%d C=%d H=%d W=%d Cout=%d", name, B, Cin, H, W, Cout);
  normalize_act(xs, B, Cin, H, W);
  B2_TRY(check_act(xs, Cin, name, "input"));
  if (!aligned16(wk)) return set_error(B2_ERR_INVALID, "%s: operands must be 16-byte aligned", name);
  const long long m_total = (long long)B * (H + 2) * (W + 2);
  if (m_total + 2LL * (W + 2) + 2 + BM >= (1LL << 31))
    return set_error(B2_ERR_UNSUPPORTED, "%s: %lld padded rows exceed the 32-bit TMA coordinate range", name, m_total);
  const int chunks = (Cin + 63) / 64;
  const int cpad = chunks * 64;
  const int ktot = chunks * 9 * 64;
  const bool wide = Cout > 128 && (Cout % 256 == 0 || Cout % 256 > 128);
  const bool pair = wide && pair_mma_enabled();
  const bool narrow = Cout <= 64;  // 64-wide tiles: no MMA work on padding columns
  const int BN = wide ? 256 : narrow ? 64 : 128;
  const uint32_t b_box = pair ? 128u : uint32_t(BN);  // the pair kernel loads half of B per CTA

  (void)cpad;
  CUtensorMap ta, tb;
  B2_TRY(rows_map(&ta, xs, B, Cin, H, W, BM));
  {
    const uint64_t dims[3] = {uint64_t(ktot), uint64_t(Cout), 1};
    const uint64_t strides[2] = {uint64_t(ktot) * 2, uint64_t(ktot) * 2 * Cout};
    const uint32_t box[3] = {64, b_box, 1};
    B2_TRY(encode_tmap(&tb, wk, 3, dims, strides, box, true));
  }
  Params p{};
  p.tiles_m = int((m_total + BM - 1) / BM);
  p.tiles_n = (Cout + BN - 1) / BN;
  p.splits = 1;
  p.batch = 1;
  p.num_kb = chunks * 9;
  p.kb_per_split = p.num_kb;
  p.wp = W + 2;
  p.hp = H + 2;
  p.H = H;
  p.W = W;
  p.m_total = int(m_total);
  p.M = int(m_total);
  p.N = Cout;
  p.out = y;
  p.osn = sn;
  p.osc = sc;
  p.osh = sh;
  p.osw = sw;
  p.bias = bias;
  p.relu = relu;
  p.alpha = 1.f;
  p.status = device_status_ptr();
  p.src_im2col = xs.nhwc ? 1 : 0;
  const int tiles = p.tiles_m * p.tiles_n;
  if (pair) {
    Params pp = p;
    pp.tiles_m = int((m_total + 255) / 256);  // 256-pixel tiles
    int boxes = 0, box_rows = 0;
    if (halo_enabled()) halo_window(W + 2, size_t(kHaloB) * 128 * BK * 2, boxes, box_rows);
    if (boxes > 0) {
      CUtensorMap twin;
      B2_TRY(rows_map(&twin, xs, B, Cin, H, W, uint32_t(box_rows)));
      pp.win_boxes = boxes;
      pp.win_box_rows = box_rows;
      return launch_pair_halo(twin, tb, pp, st);
    }
    return launch_pair<kConv>(ta, tb, pp, pp.tiles_m * pp.tiles_n, st);
  }
  if (narrow && chunks == 1 && bres_enabled()) {
    int boxes = 0, box_rows = 0;
    halo_window(W + 2, kBresWeightBytes, boxes, box_rows);
    const int bufs = boxes > 0 ? bres_window_buffers(boxes * box_rows * 128) : 0;
    if (bufs > 0) {
      CUtensorMap twin;
      B2_TRY(rows_map(&twin, xs, B, Cin, H, W, uint32_t(box_rows)));
      Params ph = p;
      ph.win_boxes = boxes;
      ph.win_box_rows = box_rows;
      ph.win_bufs = bufs;
      return launch_halo_bres(twin, tb, ph, st);
    }
  }
  if (wide) return launch<256, kStages256, kConv, false, false>(ta, tb, p, tiles, st);
  if (narrow) return launch<64, kStages64, kConv, false, false>(ta, tb, p, tiles, st);
  return launch<128, kStages128, kConv, false, false>(ta, tb, p, tiles, st);
}

struct WgradPlan {
  int BN, ci_blocks, tiles_m, num_kb, splits, kb_per_split;
  int wb = 0, hb = 0, nx = 0, ny = 0;  // pixel patches of channels-last operands (0: padded rows)
  bool pair;  // SM-pair kernel: 256-co x 256-ci tiles per cluster of two CTAs
  long long m_total;
  size_t workspace;
};

// The 64-pixel patch (wb x hb, powers of two) that covers an H x W image
// with the fewest padded pixels; ties go to the wider patch.
void choose_patch(int H, int W, int& wb, int& hb) {
  long long best = -1;
  for (int e = 6; e >= 0; --e) {
    const int cw = 1 << e, chh = BK / cw;
    const long long area = (long long)((W + cw - 1) / cw) * cw * (long long)((H + chh - 1) / chh) * chh;
    if (best < 0 || area < best) {
      best = area;
      wb = cw;
      hb = chh;
    }
  }
}

WgradPlan wgrad_plan(int B, int Cin, int H, int W, int Cout, int sms, bool allow_pair, bool patches = false) {
  WgradPlan w{};
  w.m_total = (long long)B * (H + 2) * (W + 2);
  w.pair = allow_pair && Cin > 128 && Cout > 128;
  w.BN = Cin > 128 ? 256 : Cin > 64 ? 128 : 64;
  w.ci_blocks = (Cin + w.BN - 1) / w.BN;
  w.tiles_m = (Cout + (w.pair ? 255 : BM - 1)) / (w.pair ? 256 : BM);
  w.num_kb = int((w.m_total + BK - 1) / BK);
  if (patches) {
    choose_patch(H, W, w.wb, w.hb);
    w.nx = (W + w.wb - 1) / w.wb;
    w.ny = (H + w.hb - 1) / w.hb;
    w.num_kb = B * w.nx * w.ny;
  }
  // Split-K so that the tiles fill the SMs (pairs of SMs for the pair kernel)
  // in whole waves: tiles are long (thousands of k-blocks), so a partial last
  // wave would idle SMs for a whole tile's duration.
  const int units = w.pair ? sms / 2 : sms;
  const int base = w.tiles_m * 9 * w.ci_blocks;
  int splits = base >= units ? 1 : units / base;
  splits = std::max(1, std::min(splits, w.num_kb / 16));
  w.kb_per_split = (w.num_kb + splits - 1) / splits;
  w.splits = (w.num_kb + w.kb_per_split - 1) / w.kb_per_split;
  w.workspace = size_t(w.splits) * 9 * size_t(Cout) * size_t(Cin) * sizeof(float);
  return w;
}

// Plan of the narrow wgrad kernel (Cin <= 64, Cout <= 64): 128-pixel
// k-blocks split over the SMs (at least 2 per CTA), the input window of
// halo_window's geometry, as many stages (dY block + window) as fit.  ok =
// false when the shape is not narrow or the window does not fit.
struct NarrowWgradPlan {
  bool ok = false;
  int num_kb = 0, splits = 0, kb_per_split = 0, boxes = 0, box_rows = 0, stages = 0;
  long long m_total = 0;
  size_t workspace = 0, smem = 0;
};

NarrowWgradPlan narrow_wgrad_plan(int B, int Cin, int H, int W, int Cout, int sms) {
  NarrowWgradPlan w;
  if (Cin > 64 || Cout > 64 || !narrow_wgrad_enabled()) return w;
  w.m_total = (long long)B * (H + 2) * (W + 2);
  const size_t dy_bytes = size_t(kNarrowWgradPix) * 128;
  halo_window(W + 2, 2 * dy_bytes, w.boxes, w.box_rows);
  if (w.boxes <= 0) return w;
  const size_t stage = dy_bytes + size_t(w.boxes) * w.box_rows * 128;
  w.stages = int(std::min<size_t>(kMaxWinBufs, (kHaloMaxSmem - 1024 - 256) / stage));
  if (w.stages < 2) return w;
  w.smem = size_t(w.stages) * stage + 1024 + 256;
  w.num_kb = int((w.m_total + kNarrowWgradPix - 1) / kNarrowWgradPix);
  // fewer k-blocks than SMs: the tiled kernel's 9 x tiles parallelism wins
  if (w.num_kb < sms) return w;
  int splits = std::max(1, std::min(sms, w.num_kb / 2));
  w.kb_per_split = (w.num_kb + splits - 1) / splits;
  w.splits = (w.num_kb + w.kb_per_split - 1) / w.kb_per_split;
  w.workspace = size_t(w.splits) * 9 * size_t(Cout) * size_t(Cin) * sizeof(float);
  w.ok = true;
  return w;
}

b2_status launch_wgrad_narrow(const CUtensorMap& tdy, const CUtensorMap& tx, const Params& p, size_t smem,
                              int splits, cudaStream_t st) {
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  if (!configured[dev]) {  // once, at the largest size accepted
    B2_TRY(check_cuda(cudaFuncSetAttribute(igemm_wgrad_narrow_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(kHaloMaxSmem)),
                      "cudaFuncSetAttribute(smem, narrow wgrad)"));
    configured[dev] = true;
  }
  igemm_wgrad_narrow_kernel<<<splits, kThreads, smem, st>>>(tdy, tx, p);
  return check_cuda(cudaGetLastError(), "narrow wgrad launch");
}

// One GEMM call, D[z] = alpha * op(A[z]) * op(B[z]) + beta * C[z] (bf16 in, fp32
// accumulate), with the extensions the 1x1 convolutions need:
//   a_bcast    A has a single slice used for every z;
//   k_batched  the reduction also runs over the `batch` slices of A and B
//              (one output slice): sum_z op(A[z]) op(B[z]);
//   partial    split-K: `splits` fp32 partials [splits][M][N] in `partial`,
//              summed in split order into D (dtype d_dtype, alpha only); also
//              with one split, for an fp32 D.
struct GemmCall {
  int transA = 0, transB = 0, M = 0, N = 0, K = 0;
  float alpha = 1.f;
  const void* A = nullptr;
  int64_t lda = 0, strideA = 0;
  const void* B = nullptr;
  int64_t ldb = 0, strideB = 0;
  float beta = 0.f;
  const void* C = nullptr;
  int c_dtype = B2_BF16;
  int64_t c_sm = 0, c_sn = 0, c_sb = 0;
  void* D = nullptr;
  int64_t ldd = 0, strideD = 0;
  int batch = 1;
  bool a_bcast = false, k_batched = false;
  int splits = 1;
  float* partial = nullptr;
  int d_dtype = B2_BF16;
  bool partial_is_d = false;  // one split, fp32 D with ldd == N: the partial is D itself
  int bn = 0;                 // output tile width; 0: gemm_tile_n's choice
};

// Output tile width: the widest the output allows.  A tcgen05.mma of M = 128
// and K = 16 occupies the tensor pipe for the same time whatever its N (up to
// 256): measured on B200, back-to-back MMAs with operands resident in shared
// memory take 138 cycles each at N = 64, 128 and 256, so a 128-wide tile runs
// the pipe at half the rate of a 256-wide one.  Few output tiles are made up
// for by splitting the reduction (gemm_plain_splits), not by narrower tiles.
int gemm_widest_tile(int N) { return N > 128 ? 256 : N > 64 ? 128 : 64; }

int gemm_tile_n(int /*M*/, int N, int /*batch*/, int /*sms*/) { return gemm_widest_tile(N); }

// Split-K of a plain GEMM whose tiles occupy under three quarters of the SMs:
// enough splits for about one wave, at most 8, and at least 16 k-blocks per
// split -- the fp32 partials and their ordered reduction cost a few
// microseconds (measured on B200: 512 x 4096 x 1024 ran 10.4 us in 64 tiles
// unsplit, 17 us in two splits of 8 k-blocks; 512 x 4096 x 4096 25 us either
// as 128 narrow tiles or as 2 x 64 wide ones).
int gemm_plain_splits(int M, int N, int K, int batch, int sms) {
  if (batch != 1) return 1;
  const int bn = gemm_widest_tile(N);
  const long long tiles = (long long)((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  const long long kb = (K + BK - 1) / BK;
  if (tiles * 4 >= (long long)sms * 3) return 1;
  return int(std::max<long long>(1, std::min<long long>({(long long)sms / tiles, kb / 16, 8})));
}

b2_status gemm_core(const GemmCall& g, cudaStream_t st) {
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int BN = g.bn ? g.bn : gemm_tile_n(g.M, g.N, g.partial ? 1 : g.batch, sm_count(dev));
  const uint64_t bt = uint64_t(g.batch);
  const uint64_t bta = g.a_bcast ? 1 : bt;
  CUtensorMap ta, tb;
  if (!g.transA) {  // A [M][K], K contiguous -> K-major
    const uint64_t dims[3] = {uint64_t(g.K), uint64_t(g.M), bta};
    const uint64_t strides[2] = {uint64_t(g.lda) * 2, uint64_t(bta > 1 ? g.strideA : g.lda * g.M) * 2};
    const uint32_t box[3] = {64, BM, 1};
    B2_TRY(encode_tmap(&ta, g.A, 3, dims, strides, box, true));
  } else {  // A stored [K][M], M contiguous -> MN-major
    const uint64_t dims[3] = {uint64_t(g.M), uint64_t(g.K), bta};
    const uint64_t strides[2] = {uint64_t(g.lda) * 2, uint64_t(bta > 1 ? g.strideA : g.lda * g.K) * 2};
    const uint32_t box[3] = {64, 64, 1};
    B2_TRY(encode_tmap(&ta, g.A, 3, dims, strides, box, true));
  }
  if (g.transB) {  // B stored [N][K] -> K-major
    const uint64_t dims[3] = {uint64_t(g.K), uint64_t(g.N), bt};
    const uint64_t strides[2] = {uint64_t(g.ldb) * 2, uint64_t(bt > 1 ? g.strideB : g.ldb * g.N) * 2};
    const uint32_t box[3] = {64, uint32_t(BN), 1};
    B2_TRY(encode_tmap(&tb, g.B, 3, dims, strides, box, true));
  } else {  // B [K][N], N contiguous -> MN-major
    const uint64_t dims[3] = {uint64_t(g.N), uint64_t(g.K), bt};
    const uint64_t strides[2] = {uint64_t(g.ldb) * 2, uint64_t(bt > 1 ? g.strideB : g.ldb * g.K) * 2};
    const uint32_t box[3] = {64, 64, 1};
    B2_TRY(encode_tmap(&tb, g.B, 3, dims, strides, box, true));
  }
  Params p{};
  p.tiles_m = (g.M + BM - 1) / BM;
  p.tiles_n = (g.N + BN - 1) / BN;
  const int kb_slice = (g.K + BK - 1) / BK;
  p.num_kb = g.k_batched ? kb_slice * g.batch : kb_slice;
  p.kb_per_batch = g.k_batched ? kb_slice : 0;
  p.a_bcast = g.a_bcast ? 1 : 0;
  p.splits = 1;
  if (g.partial) {
    // alpha and beta * C are applied by the reduction
    p.gemm_split = 1;
    p.kb_per_split = (p.num_kb + std::max(1, g.splits) - 1) / std::max(1, g.splits);
    p.batch = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;  // tile-space slices = splits
    p.partial = g.partial;
  } else {
    p.kb_per_split = p.num_kb;
    p.batch = g.k_batched ? 1 : g.batch;
  }
  p.M = g.M;
  p.N = g.N;
  p.out = g.D;
  p.osn = g.strideD;
  p.osh = g.ldd;
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.cin = g.C;
  p.cin_dtype = g.c_dtype;
  p.c_sm = g.c_sm;
  p.c_sn = g.c_sn;
  p.c_sb = g.c_sb;
  p.status = device_status_ptr();
  // bf16 D through TMA stores: 32 x 32 boxes of a {N, M, batch} map (16-byte
  // aligned base and row / slice strides; the box is clipped at M and N)
  CUtensorMap td;
  const CUtensorMap* tdp = nullptr;
  if (!p.gemm_split && g.D && aligned16(g.D) && g.ldd % 8 == 0 && g.ldd >= g.N &&
      (p.batch <= 1 || g.strideD % 8 == 0)) {
    const uint64_t nb = uint64_t(std::max(1, p.batch));
    const uint64_t dims[3] = {uint64_t(g.N), uint64_t(g.M), nb};
    const uint64_t strides[2] = {uint64_t(g.ldd) * 2, uint64_t(nb > 1 ? g.strideD : g.ldd * g.M) * 2};
    const uint32_t bc = BN >= 128 ? 64 : 32;  // epi_box_cols<BN>()
    const uint32_t box[3] = {bc, 32, 1};
    if (encode_tmap_sw(&td, g.D, 3, dims, strides, box, int(bc * 2)) == B2_OK) {
      tdp = &td;
      p.tma_store = 1;
    }
  }
  const bool amn = g.transA != 0, bmn = g.transB == 0;
  b2_status rc;
  // SM-pair tiles (256 rows x PBN columns, tcgen05.mma.cta_group::2): each SM
  // stages its own 128 A rows and half of the tile's B columns, so per MMA it
  // moves a quarter (PBN 256) to an eighth less from L2 than a single-CTA
  // tile.  Taken when the pair tiles still give most SMs work.
  int pbn = 0;
  if (gemm_pair_enabled() && !g.k_batched && g.M > 128 && BN == 256) pbn = 256;
  if (pbn) {
    Params pp = p;
    pp.tiles_m = (g.M + 255) / 256;
    pp.tiles_n = (g.N + pbn - 1) / pbn;
    pp.tma_store = 0;
    if (g.transB) {  // re-encode B (K-major, stored [N][K]): a box is this CTA's half of the tile's columns
      const uint64_t bt2 = uint64_t(g.batch);
      const uint64_t dims[3] = {uint64_t(g.K), uint64_t(g.N), bt2};
      const uint64_t strides[2] = {uint64_t(g.ldb) * 2, uint64_t(bt2 > 1 ? g.strideB : g.ldb * g.N) * 2};
      const uint32_t box[3] = {64, uint32_t(pbn / 2), 1};
      B2_TRY(encode_tmap(&tb, g.B, 3, dims, strides, box, true));
    }
    const int ptiles = pp.batch * pp.tiles_m * pp.tiles_n;
    if (pbn == 256) {
      if (!amn && !bmn) rc = launch_pair<kGemm, 256, false, false>(ta, tb, pp, ptiles, st);
      else if (!amn && bmn) rc = launch_pair<kGemm, 256, false, true>(ta, tb, pp, ptiles, st);
      else if (amn && !bmn) rc = launch_pair<kGemm, 256, true, false>(ta, tb, pp, ptiles, st);
      else rc = launch_pair<kGemm, 256, true, true>(ta, tb, pp, ptiles, st);
    } else {
      if (!amn && !bmn) rc = launch_pair<kGemm, 128, false, false>(ta, tb, pp, ptiles, st);
      else if (!amn && bmn) rc = launch_pair<kGemm, 128, false, true>(ta, tb, pp, ptiles, st);
      else if (amn && !bmn) rc = launch_pair<kGemm, 128, true, false>(ta, tb, pp, ptiles, st);
      else rc = launch_pair<kGemm, 128, true, true>(ta, tb, pp, ptiles, st);
    }
  } else {
  const int tiles = p.batch * p.tiles_m * p.tiles_n;
  // split-K partials are fp32 and never go through the TMA-store staging:
  // its shared memory buys more operand stages instead.  (Plain GEMMs keep
  // the staging even for long reductions: without it the direct stores of
  // a one-tile-per-SM grid cost more than the deeper ring gains -- measured
  // on B200, 512 x 4096 x 4096 26.2 against 26.8 us, 4096 x 4096 x 512 23.6
  // against 28.1 us.)
  if (p.gemm_split) {
    if (BN == 256) rc = launch_gemm<256, kGemmDeep256, false>(amn, bmn, ta, tb, p, tiles, st, nullptr);
    else if (BN == 128) rc = launch_gemm<128, kGemmDeep128, false>(amn, bmn, ta, tb, p, tiles, st, nullptr);
    else rc = launch_gemm<64, kGemmDeep64, false>(amn, bmn, ta, tb, p, tiles, st, nullptr);
  } else if (BN == 256) {
    rc = launch_gemm<256, kGemmStages256, true>(amn, bmn, ta, tb, p, tiles, st, tdp);
  } else if (BN == 128) {
    rc = launch_gemm<128, kGemmStages128, true>(amn, bmn, ta, tb, p, tiles, st, tdp);
  } else {
    rc = launch_gemm<64, kGemmStages64, true>(amn, bmn, ta, tb, p, tiles, st, tdp);
  }
  }
  if (rc != B2_OK || !p.gemm_split || g.partial_is_d) return rc;
  const long long total = (long long)g.M * g.N;
  const int threads = 256;
  const bool dvec = g.d_dtype == B2_F32 ? (aligned16(g.D) && g.ldd % 4 == 0)
                                        : ((reinterpret_cast<uintptr_t>(g.D) & 7) == 0 && g.ldd % 4 == 0);
  if (g.N % 4 == 0 && aligned16(g.partial) && dvec) {
    const int n4 = g.N / 4;
    const dim3 grid(unsigned((n4 + threads - 1) / threads), unsigned(std::min(g.M, 65535)));
    gemm_split_reduce_vec_kernel<<<grid, threads, 0, st>>>(reinterpret_cast<const float4*>(g.partial), p.batch, g.M,
                                                            n4, g.alpha, g.D, g.d_dtype, g.ldd, g.beta, g.C,
                                                            g.c_dtype, g.c_sm, g.c_sn);
    return check_cuda(cudaGetLastError(), "gemm split reduce launch");
  }
  const int blocks = int(std::max<long long>(1, std::min<long long>((total + threads - 1) / threads, 148LL * 8)));
  gemm_split_reduce_kernel<<<blocks, threads, 0, st>>>(g.partial, p.batch, g.M, g.N, g.alpha, g.D, g.d_dtype, g.ldd,
                                                       g.beta, g.C, g.c_dtype, g.c_sm, g.c_sn);
  return check_cuda(cudaGetLastError(), "gemm split reduce launch");
}

// Split-K plan for a reduction-heavy GEMM (1x1 wgrad): enough splits for one
// wave over the SMs, at least 16 k-blocks per split.
int gemm_splits(int M, int N, long long num_kb, int sms) {
  const int BN = gemm_widest_tile(N);
  const long long tiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  long long splits = tiles >= sms ? 1 : sms / tiles;
  splits = std::max<long long>(1, std::min<long long>(splits, num_kb / 16));
  const long long kps = (num_kb + splits - 1) / splits;
  return int((num_kb + kps - 1) / kps);
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

b2_status b2_conv3x3_fwd(const void* x_rows, const void* wk, const void* bias, void* y, int64_t ysn,
                         int64_t ysc, int64_t ysh, int64_t ysw, int B, int Cin, int H, int W,
                         int Cout, int relu, void* stream) {
  return conv_common(rows_src(x_rows), wk, static_cast<const uint16_t*>(bias), y, ysn, ysc, ysh, ysw, B, Cin,
                     H, W, Cout, relu, static_cast<cudaStream_t>(stream), "b2_conv3x3_fwd");
}

b2_status b2_conv3x3_dgrad(const void* dy_rows, const void* wk_dgrad, void* dx, int64_t sn,
                           int64_t sc, int64_t sh, int64_t sw, int B, int Cout, int H, int W,
                           int Cin, void* stream) {
  return conv_common(rows_src(dy_rows), wk_dgrad, nullptr, dx, sn, sc, sh, sw, B, Cout, H, W, Cin, 0,
                     static_cast<cudaStream_t>(stream), "b2_conv3x3_dgrad");
}

size_t b2_conv3x3_wgrad_workspace_bytes(int B, int Cin, int H, int W, int Cout) {
  if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0) return 16;
  int dev = 0;
  cudaGetDevice(&dev);
  const NarrowWgradPlan nw = narrow_wgrad_plan(B, Cin, H, W, Cout, sm_count(dev));
  if (nw.ok) return std::max<size_t>(16, nw.workspace);
  // the larger of the padded-row and the pixel-patch plans (channels-last operands)
  return std::max<size_t>({size_t(16), wgrad_plan(B, Cin, H, W, Cout, sm_count(dev), pair_mma_enabled()).workspace,
                           wgrad_plan(B, Cin, H, W, Cout, sm_count(dev), pair_mma_enabled(), true).workspace});
}

static b2_status wgrad_common(ActSrc dys, ActSrc xs, void* dw, int dw_dtype, int B, int Cin, int H,
                              int W, int Cout, void* workspace, size_t workspace_bytes, void* stream,
                              const char* name, bool ohwi = false) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!dw || !workspace) return set_error(B2_ERR_INVALID, "%s: null pointer", name);
  if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0) return set_error(B2_ERR_INVALID, "%s: bad shape", name);
  if (dw_dtype != B2_BF16 && dw_dtype != B2_F32) return set_error(B2_ERR_INVALID, "%s: dtype", name);
  normalize_act(dys, B, Cout, H, W);
  normalize_act(xs, B, Cin, H, W);
  B2_TRY(check_act(dys, Cout, name, "dY"));
  B2_TRY(check_act(xs, Cin, name, "input"));
  if (!aligned16(workspace)) return set_error(B2_ERR_INVALID, "%s: workspace must be 16-byte aligned", name);
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const NarrowWgradPlan nw = narrow_wgrad_plan(B, Cin, H, W, Cout, sm_count(dev));
  if (nw.ok) {
    if (nw.m_total + 2LL * (W + 2) + 2 + W + 3 + kNarrowWgradPix >= (1LL << 31))
      return set_error(B2_ERR_UNSUPPORTED, "%s: too many padded rows", name);
    if (workspace_bytes < nw.workspace)
      return set_error(B2_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", name, workspace_bytes, nw.workspace);
    CUtensorMap tdy, tx;
    B2_TRY(rows_map(&tdy, dys, B, Cout, H, W, uint32_t(kNarrowWgradPix)));
    B2_TRY(rows_map(&tx, xs, B, Cin, H, W, uint32_t(nw.box_rows)));
    Params p{};
    p.splits = nw.splits;
    p.num_kb = nw.num_kb;
    p.kb_per_split = nw.kb_per_split;
    p.wp = W + 2;
    p.hp = H + 2;
    p.H = H;
    p.W = W;
    p.m_total = int(nw.m_total);
    p.a_row_shift = W + 3;
    p.M = Cout;
    p.N = Cin;
    p.win_boxes = nw.boxes;
    p.win_box_rows = nw.box_rows;
    p.win_bufs = nw.stages;
    p.partial = static_cast<float*>(workspace);
    p.alpha = 1.f;
    p.status = device_status_ptr();
    p.src_im2col = (dys.nhwc ? 1 : 0) | (xs.nhwc ? 2 : 0);
    B2_TRY(launch_wgrad_narrow(tdy, tx, p, nw.smem, nw.splits, st));
    const long long total = (long long)Cout * Cin * 9;
    const int blocks = int(std::min<long long>((total + 255) / 256, 148LL * 16));
    wgrad_reduce_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(workspace), dw, dw_dtype, nw.splits,
                                                Cout, Cin, ohwi);
    return check_cuda(cudaGetLastError(), "wgrad reduce launch");
  }
  // Channels-last dY and X: k-blocks are 64-pixel patches fetched by tiled
  // 4-D loads (an im2col load of 64 pixels costs about twice a tiled one).
  const bool patches = dys.nhwc && xs.nhwc && patch_wgrad_enabled();
  const WgradPlan w = wgrad_plan(B, Cin, H, W, Cout, sm_count(dev), pair_mma_enabled(), patches);
  if (!patches && w.m_total + 2LL * (W + 2) + 2 + W + 3 + BK >= (1LL << 31))
    return set_error(B2_ERR_UNSUPPORTED, "%s: too many padded rows", name);
  if (workspace_bytes < w.workspace)
    return set_error(B2_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", name, workspace_bytes, w.workspace);
  CUtensorMap ta, tb;
  if (patches) {
    const uint32_t box[4] = {64, uint32_t(w.wb), uint32_t(w.hb), 1};
    const uint64_t dd[4] = {uint64_t(Cout), uint64_t(W), uint64_t(H), uint64_t(B)};
    const uint64_t ds[3] = {uint64_t(dys.sw) * 2, uint64_t(dys.sh) * 2, uint64_t(dys.sn) * 2};
    B2_TRY(encode_tmap(&ta, dys.ptr, 4, dd, ds, box, true));
    const uint64_t xd[4] = {uint64_t(Cin), uint64_t(W), uint64_t(H), uint64_t(B)};
    const uint64_t xst[3] = {uint64_t(xs.sw) * 2, uint64_t(xs.sh) * 2, uint64_t(xs.sn) * 2};
    B2_TRY(encode_tmap(&tb, xs.ptr, 4, xd, xst, box, true));
  } else {
    B2_TRY(rows_map(&ta, dys, B, Cout, H, W, 64));
    B2_TRY(rows_map(&tb, xs, B, Cin, H, W, 64));
  }
  Params p{};
  p.tiles_m = w.tiles_m;
  p.tiles_n = 1;
  p.splits = w.splits;
  p.batch = 1;
  p.num_kb = w.num_kb;
  p.kb_per_split = w.kb_per_split;
  p.wp = W + 2;
  p.hp = H + 2;
  p.H = H;
  p.W = W;
  p.m_total = int(w.m_total);
  p.a_row_shift = W + 3;
  p.ci_blocks = w.ci_blocks;
  p.M = Cout;
  p.N = Cin;
  p.partial = static_cast<float*>(workspace);
  p.alpha = 1.f;
  p.status = device_status_ptr();
  p.src_im2col = (dys.nhwc ? 1 : 0) | (xs.nhwc ? 2 : 0);
  p.patch_wb = w.wb;
  p.patch_hb = w.hb;
  p.patch_nx = w.nx;
  p.patch_ny = w.ny;
  const int tiles = w.splits * w.tiles_m * 9 * w.ci_blocks;
  if (w.pair)
    B2_TRY(launch_pair<kWgrad>(ta, tb, p, tiles, st));
  else if (w.BN == 256)
    B2_TRY((launch<256, kStages256, kWgrad, true, true>(ta, tb, p, tiles, st)));
  else if (w.BN == 64)
    B2_TRY((launch<64, kStages64, kWgrad, true, true>(ta, tb, p, tiles, st)));
  else
    B2_TRY((launch<128, kStages128, kWgrad, true, true>(ta, tb, p, tiles, st)));
  const long long total = (long long)Cout * Cin * 9;
  const int threads = 256;
  const int blocks = int(std::min<long long>((total + threads - 1) / threads, 148LL * 16));
  wgrad_reduce_kernel<<<blocks, threads, 0, st>>>(static_cast<const float*>(workspace), dw, dw_dtype,
                                                  w.splits, Cout, Cin, ohwi);
  return check_cuda(cudaGetLastError(), "wgrad reduce launch");
}

b2_status b2_conv3x3_wgrad(const void* dy_rows, const void* x_rows, void* dw, int dw_dtype, int B, int Cin, int H,
                           int W, int Cout, void* workspace, size_t workspace_bytes, void* stream) {
  return wgrad_common(rows_src(dy_rows), rows_src(x_rows), dw, dw_dtype, B, Cin, H, W, Cout, workspace,
                      workspace_bytes, stream, "b2_conv3x3_wgrad");
}

// ---- channels-last operands read in place (no padded-row copy) ------------
static ActSrc nhwc_src(const void* t, int64_t sn, int64_t sh, int64_t sw) {
  ActSrc a;
  a.ptr = t;
  a.nhwc = true;
  a.sn = sn;
  a.sh = sh;
  a.sw = sw;
  return a;
}

b2_status b2_conv3x3_fwd_nhwc(const void* x, int64_t xsn, int64_t xsh, int64_t xsw, const void* wk,
                              const void* bias, void* y, int64_t ysn, int64_t ysc, int64_t ysh, int64_t ysw, int B,
                              int Cin, int H, int W, int Cout, int relu, void* stream) {
  return conv_common(nhwc_src(x, xsn, xsh, xsw), wk, static_cast<const uint16_t*>(bias), y, ysn, ysc, ysh, ysw, B,
                     Cin, H, W, Cout, relu, static_cast<cudaStream_t>(stream), "b2_conv3x3_fwd_nhwc");
}

b2_status b2_conv3x3_dgrad_nhwc(const void* dy, int64_t dsn, int64_t dsh, int64_t dsw, const void* wk_dgrad,
                                void* dx, int64_t sn, int64_t sc, int64_t sh, int64_t sw, int B, int Cout, int H,
                                int W, int Cin, void* stream) {
  return conv_common(nhwc_src(dy, dsn, dsh, dsw), wk_dgrad, nullptr, dx, sn, sc, sh, sw, B, Cout, H, W, Cin, 0,
                     static_cast<cudaStream_t>(stream), "b2_conv3x3_dgrad_nhwc");
}

b2_status b2_conv3x3_wgrad_nhwc(const void* dy, int64_t dsn, int64_t dsh, int64_t dsw, const void* x, int64_t xsn,
                                int64_t xsh, int64_t xsw, void* dw, int dw_dtype, int B, int Cin, int H, int W,
                                int Cout, void* workspace, size_t workspace_bytes, void* stream) {
  return wgrad_common(nhwc_src(dy, dsn, dsh, dsw), nhwc_src(x, xsn, xsh, xsw), dw, dw_dtype, B, Cin, H, W, Cout,
                      workspace, workspace_bytes, stream, "b2_conv3x3_wgrad_nhwc");
}

b2_status b2_conv3x3_wgrad_nhwc_ohwi(const void* dy, int64_t dsn, int64_t dsh, int64_t dsw, const void* x,
                                     int64_t xsn, int64_t xsh, int64_t xsw, void* dw, int dw_dtype, int B, int Cin,
                                     int H, int W, int Cout, void* workspace, size_t workspace_bytes, void* stream) {
  return wgrad_common(nhwc_src(dy, dsn, dsh, dsw), nhwc_src(x, xsn, xsh, xsw), dw, dw_dtype, B, Cin, H, W, Cout,
                      workspace, workspace_bytes, stream, "b2_conv3x3_wgrad_nhwc_ohwi", true);
}

b2_status b2_gemm_bf16(int transA, int transB, int M, int N, int K, float alpha, const void* A,
                       int64_t lda, int64_t strideA, const void* Bm, int64_t ldb, int64_t strideB,
                       float beta, const void* C, int c_dtype, int64_t c_sm, int64_t c_sn,
                       int64_t c_sb, void* D, int64_t ldd, int64_t strideD, int batch,
                       void* stream) {
  return b2_gemm_bf16_ws(transA, transB, M, N, K, alpha, A, lda, strideA, Bm, ldb, strideB, beta, C, c_dtype, c_sm,
                         c_sn, c_sb, D, ldd, strideD, batch, nullptr, 0, stream);
}

size_t b2_gemm_bf16_workspace_bytes(int M, int N, int K, int batch) {
  if (M <= 0 || N <= 0 || K <= 0 || batch != 1) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int sp = gemm_plain_splits(M, N, K, batch, sm_count(dev));
  return sp > 1 ? size_t(sp) * size_t(M) * size_t(N) * sizeof(float) : 0;
}

b2_status b2_gemm_bf16_ws(int transA, int transB, int M, int N, int K, float alpha, const void* A, int64_t lda,
                          int64_t strideA, const void* Bm, int64_t ldb, int64_t strideB, float beta, const void* C,
                          int c_dtype, int64_t c_sm, int64_t c_sn, int64_t c_sb, void* D, int64_t ldd,
                          int64_t strideD, int batch, void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M < 0 || N < 0 || K < 0 || batch < 0) return set_error(B2_ERR_INVALID, "b2_gemm_bf16: negative size");
  if (M == 0 || N == 0 || batch == 0) return B2_OK;
  if (!A || !Bm || !D) return set_error(B2_ERR_INVALID, "b2_gemm_bf16: null pointer");
  if (beta != 0.f && !C) return set_error(B2_ERR_INVALID, "b2_gemm_bf16: beta != 0 needs C");
  if (c_dtype != B2_BF16 && c_dtype != B2_F32) return set_error(B2_ERR_INVALID, "b2_gemm_bf16: c dtype");
  if (K == 0) return set_error(B2_ERR_UNSUPPORTED, "b2_gemm_bf16: K == 0");
  if (!aligned16(A) || !aligned16(Bm) || lda % 8 || ldb % 8 || (batch > 1 && (strideA % 8 || strideB % 8)))
    return set_error(B2_ERR_UNSUPPORTED, "b2_gemm_bf16: operands need 16-byte aligned rows");
  GemmCall g;
  g.transA = transA;
  g.transB = transB;
  g.M = M;
  g.N = N;
  g.K = K;
  g.alpha = alpha;
  g.A = A;
  g.lda = lda;
  g.strideA = strideA;
  g.B = Bm;
  g.ldb = ldb;
  g.strideB = strideB;
  g.beta = beta;
  g.C = C;
  g.c_dtype = c_dtype;
  g.c_sm = c_sm;
  g.c_sn = c_sn;
  g.c_sb = c_sb;
  g.D = D;
  g.ldd = ldd;
  g.strideD = strideD;
  g.batch = batch;
  // too few output tiles for the SMs: split the reduction when the caller
  // gave room for the fp32 partial sums (added in split order: deterministic)
  const size_t need = b2_gemm_bf16_workspace_bytes(M, N, K, batch);
  if (need > 0 && workspace && workspace_bytes >= need && aligned16(workspace)) {
    int dev = 0;
    B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
    g.splits = gemm_plain_splits(M, N, K, batch, sm_count(dev));
    g.partial = static_cast<float*>(workspace);
    g.d_dtype = B2_BF16;
  }
  return gemm_core(g, st);
}

// ---- 1x1 convolutions (stride 1, no padding) as GEMMs ----------------------
// layout 0: NCHW (per image, X[b] is [Cin][HW]); 1: NHWC (X is [B*HW][Cin]).
// Weights [Cout][Cin] (OIHW with 1x1 kernels), bf16; every row stride must be
// a multiple of 8 elements (16 bytes) and every pointer 16-byte aligned.

size_t b2_gemm_splitk_workspace_bytes(int M, int N, int K, int d_dtype) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int splits = gemm_splits(M, N, (K + BK - 1) / BK, sm_count(dev));
  if (splits == 1 && d_dtype == B2_F32) return 0;  // a dense fp32 D takes the sums directly
  return size_t(splits) * size_t(M) * size_t(N) * sizeof(float);
}

b2_status b2_gemm_splitk_bf16(int transA, int transB, int M, int N, int K, const void* A, int64_t lda,
                              const void* Bm, int64_t ldb, void* D, int d_dtype, int64_t ldd, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) return set_error(B2_ERR_INVALID, "b2_gemm_splitk_bf16: negative size");
  if (d_dtype != B2_BF16 && d_dtype != B2_F32) return set_error(B2_ERR_INVALID, "b2_gemm_splitk_bf16: D dtype");
  if (M == 0 || N == 0) return B2_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!A || !Bm || !D) return set_error(B2_ERR_INVALID, "b2_gemm_splitk_bf16: null pointer");
  if (!aligned16(A) || !aligned16(Bm) || lda % 8 || ldb % 8)
    return set_error(B2_ERR_UNSUPPORTED, "b2_gemm_splitk_bf16: operands need 16-byte aligned rows");
  if (K == 0) {
    if (ldd != N) return set_error(B2_ERR_UNSUPPORTED, "b2_gemm_splitk_bf16: K == 0 needs a dense D");
    return check_cuda(cudaMemsetAsync(D, 0, size_t(M) * N * (d_dtype == B2_F32 ? 4 : 2), st), "memset");
  }
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int splits = gemm_splits(M, N, (K + BK - 1) / BK, sm_count(dev));
  GemmCall g;
  g.transA = transA;
  g.transB = transB;
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = A;
  g.lda = lda;
  g.B = Bm;
  g.ldb = ldb;
  g.D = D;
  g.ldd = ldd;
  g.d_dtype = d_dtype;
  g.splits = splits;
  g.bn = gemm_widest_tile(N);  // the tile width gemm_splits planned for
  if (splits == 1 && d_dtype == B2_F32 && ldd == N && aligned16(D)) {
    g.partial = static_cast<float*>(D);
    g.partial_is_d = true;
  } else {
    const size_t need = size_t(splits) * size_t(M) * size_t(N) * sizeof(float);
    if (workspace_bytes < need || !workspace || !aligned16(workspace))
      return set_error(B2_ERR_WORKSPACE, "b2_gemm_splitk_bf16: workspace of %zu bytes needed", need);
    g.partial = static_cast<float*>(workspace);
  }
  return gemm_core(g, st);
}

static b2_status conv1x1_check(const char* who, int layout, int64_t B, int64_t Cin, int64_t HW, int64_t Cout,
                               std::initializer_list<const void*> ptrs) {
  if (layout != 0 && layout != 1) return set_error(B2_ERR_INVALID, "%s: layout must be 0 (NCHW) or 1 (NHWC)", who);
  if (B < 0 || Cin < 0 || HW < 0 || Cout < 0) return set_error(B2_ERR_INVALID, "%s: negative size", who);
  if (B * HW > INT32_MAX || Cin > INT32_MAX || Cout > INT32_MAX)
    return set_error(B2_ERR_UNSUPPORTED, "%s: too large", who);
  for (const void* q : ptrs)
    if (!q) return set_error(B2_ERR_INVALID, "%s: null pointer", who);
  for (const void* q : ptrs)
    if (!aligned16(q)) return set_error(B2_ERR_UNSUPPORTED, "%s: 16-byte alignment needed", who);
  if (Cin % 8 || Cout % 8 || (layout == 0 && HW % 8))
    return set_error(B2_ERR_UNSUPPORTED, "%s: channel counts (and HW for NCHW) must be multiples of 8", who);
  return B2_OK;
}

b2_status b2_conv1x1_fwd(const void* x, const void* w, const void* bias, void* y, int layout, int64_t B,
                         int64_t Cin, int64_t HW, int64_t Cout, void* stream) {
  B2_TRY(conv1x1_check("b2_conv1x1_fwd", layout, B, Cin, HW, Cout, {x, w, y}));
  if (B * HW == 0 || Cout == 0) return B2_OK;
  if (Cin == 0) return set_error(B2_ERR_UNSUPPORTED, "b2_conv1x1_fwd: Cin == 0");
  GemmCall g;
  if (layout == 1) {  // Y[P][Cout] = X[P][Cin] . W^T
    g.transA = 0; g.transB = 1;
    g.M = int(B * HW); g.N = int(Cout); g.K = int(Cin);
    g.A = x; g.lda = Cin; g.B = w; g.ldb = Cin;
    g.D = y; g.ldd = Cout;
    if (bias) { g.beta = 1.f; g.C = bias; g.c_sm = 0; g.c_sn = 1; }
  } else {  // Y[b][Cout][HW] = W[Cout][Cin] . X[b][Cin][HW]
    g.transA = 0; g.transB = 0;
    g.M = int(Cout); g.N = int(HW); g.K = int(Cin);
    g.A = w; g.lda = Cin; g.a_bcast = true;
    g.B = x; g.ldb = HW; g.strideB = Cin * HW;
    g.D = y; g.ldd = HW; g.strideD = Cout * HW;
    g.batch = int(B);
    if (bias) { g.beta = 1.f; g.C = bias; g.c_sm = 1; g.c_sn = 0; }
  }
  return gemm_core(g, static_cast<cudaStream_t>(stream));
}

b2_status b2_conv1x1_dgrad(const void* dy, const void* w, void* dx, int layout, int64_t B, int64_t Cin,
                           int64_t HW, int64_t Cout, void* stream) {
  B2_TRY(conv1x1_check("b2_conv1x1_dgrad", layout, B, Cin, HW, Cout, {dy, w, dx}));
  if (B * HW == 0 || Cin == 0) return B2_OK;
  if (Cout == 0) return set_error(B2_ERR_UNSUPPORTED, "b2_conv1x1_dgrad: Cout == 0");
  GemmCall g;
  if (layout == 1) {  // dX[P][Cin] = dY[P][Cout] . W[Cout][Cin]
    g.transA = 0; g.transB = 0;
    g.M = int(B * HW); g.N = int(Cin); g.K = int(Cout);
    g.A = dy; g.lda = Cout; g.B = w; g.ldb = Cin;
    g.D = dx; g.ldd = Cin;
  } else {  // dX[b][Cin][HW] = W^T[Cin][Cout] . dY[b][Cout][HW]
    g.transA = 1; g.transB = 0;
    g.M = int(Cin); g.N = int(HW); g.K = int(Cout);
    g.A = w; g.lda = Cin; g.a_bcast = true;
    g.B = dy; g.ldb = HW; g.strideB = Cout * HW;
    g.D = dx; g.ldd = HW; g.strideD = Cin * HW;
    g.batch = int(B);
  }
  return gemm_core(g, static_cast<cudaStream_t>(stream));
}

static int conv1x1_wgrad_splits(int layout, int64_t B, int64_t Cin, int64_t HW, int64_t Cout, int sms) {
  const long long num_kb = layout == 1 ? (B * HW + BK - 1) / BK : B * ((HW + BK - 1) / BK);
  return gemm_splits(int(Cout), int(Cin), num_kb, sms);
}

size_t b2_conv1x1_wgrad_workspace_bytes(int layout, int64_t B, int64_t Cin, int64_t HW, int64_t Cout) {
  if (B * HW <= 0 || Cin <= 0 || Cout <= 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int splits = conv1x1_wgrad_splits(layout, B, Cin, HW, Cout, sm_count(dev));
  return size_t(splits) * size_t(Cout) * size_t(Cin) * sizeof(float);
}

b2_status b2_conv1x1_wgrad(const void* dy, const void* x, void* dw, int dw_dtype, int layout, int64_t B,
                           int64_t Cin, int64_t HW, int64_t Cout, void* workspace, size_t workspace_bytes,
                           void* stream) {
  B2_TRY(conv1x1_check("b2_conv1x1_wgrad", layout, B, Cin, HW, Cout, {dy, x, dw}));
  if (dw_dtype != B2_BF16 && dw_dtype != B2_F32) return set_error(B2_ERR_INVALID, "b2_conv1x1_wgrad: dw dtype");
  if (Cin == 0 || Cout == 0) return B2_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B * HW == 0) {  // empty reduction: dW = 0
    const size_t bytes = size_t(Cout) * size_t(Cin) * (dw_dtype == B2_F32 ? 4 : 2);
    return check_cuda(cudaMemsetAsync(dw, 0, bytes, st), "b2_conv1x1_wgrad: memset");
  }
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const int splits = conv1x1_wgrad_splits(layout, B, Cin, HW, Cout, sm_count(dev));
  const size_t need = size_t(splits) * size_t(Cout) * size_t(Cin) * sizeof(float);
  if (workspace_bytes < need || !workspace || !aligned16(workspace))
    return set_error(B2_ERR_WORKSPACE, "b2_conv1x1_wgrad: workspace of %zu bytes needed", need);
  GemmCall g;
  g.M = int(Cout);
  g.N = int(Cin);
  if (layout == 1) {  // dW[Cout][Cin] = dY^T . X over the P pixels
    g.transA = 1; g.transB = 0;
    g.K = int(B * HW);
    g.A = dy; g.lda = Cout; g.B = x; g.ldb = Cin;
  } else {  // dW = sum_b dY[b][Cout][HW] . X[b]^T
    g.transA = 0; g.transB = 1;
    g.K = int(HW);
    g.A = dy; g.lda = HW; g.strideA = Cout * HW;
    g.B = x; g.ldb = HW; g.strideB = Cin * HW;
    g.batch = int(B);
    g.k_batched = true;
  }
  g.D = dw;
  g.ldd = Cin;
  g.d_dtype = dw_dtype;
  // split-K partials (also with one split: dW may be fp32), reduced in order
  g.splits = splits;
  g.partial = static_cast<float*>(workspace);
  g.bn = gemm_widest_tile(int(Cin));  // the tile width gemm_splits planned for
  return gemm_core(g, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Weight gradient without any allocation.
//
// b2_conv3x3_wgrad needs a caller-provided workspace for its split-K partial
// sums.  Some callers cannot provide one: a host framework that has already
// reserved all device memory for its own pool, or a latency-critical loop that
// must never reach cudaMalloc (which can synchronize the whole device).  For
// them this variant keeps the partial sums in one fixed device array that
// lives as long as the library is loaded on each GPU.
//   * Limit: kNoAllocScratchBytes (16 MiB).  If the usual split-K plan needs
//     more, fewer splits are used; if even one split (9*Cout*Cin floats) does
//     not fit, the call fails with B2_ERR_WORKSPACE.
//   * The array's device address is looked up once per device, on the first
//     call made with that device current (cudaGetSymbolAddress); make that
//     first call before any stream capture.  The cached address is valid for
//     the lifetime of the device's primary context: a cudaDeviceReset in the
//     same process invalidates it.
//   * Every call reuses the same array.  Each call overwrites every partial
//     sum it later reads, so nothing has to be cleared between calls, but two
//     calls that overlap on the GPU (different streams, or different host
//     threads) race on it: serialize them.
// ---------------------------------------------------------------------------
namespace b2 {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

std::mutex g_noalloc_mu;
float* g_noalloc_addr[64] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
b2_status noalloc_scratch(float** out) {
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev < 0 || dev >= 64) return set_error(B2_ERR_INVALID, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    B2_TRY(check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)"));
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_addr[dev];
  return B2_OK;
}

}  // namespace
}  // namespace b2

extern "C" {

size_t b2_conv3x3_wgrad_noalloc_max_bytes(void) { return b2::kNoAllocScratchBytes; }

b2_status b2_conv3x3_wgrad_noalloc(const void* dy_rows, const void* x_rows, void* dw, int dw_dtype, int B, int Cin,
                                   int H, int W, int Cout, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!dy_rows || !x_rows || !dw) return set_error(B2_ERR_INVALID, "b2_conv3x3_wgrad_noalloc: null pointer");
  if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0)
    return set_error(B2_ERR_INVALID, "b2_conv3x3_wgrad_noalloc: bad shape");
  if (dw_dtype != B2_BF16 && dw_dtype != B2_F32) return set_error(B2_ERR_INVALID, "b2_conv3x3_wgrad_noalloc: dtype");
  if (!aligned16(dy_rows) || !aligned16(x_rows))
    return set_error(B2_ERR_INVALID, "b2_conv3x3_wgrad_noalloc: operands must be 16-byte aligned");
  const size_t per_split = size_t(9) * size_t(Cout) * size_t(Cin) * sizeof(float);
  if (per_split > kNoAllocScratchBytes)
    return set_error(B2_ERR_WORKSPACE,
                     "b2_conv3x3_wgrad_noalloc: Cout*Cin = %d*%d needs %zu bytes of partial sums, more than the "
                     "fixed %zu-byte scratch; use b2_conv3x3_wgrad with a workspace",
                     Cout, Cin, per_split, kNoAllocScratchBytes);
  int dev = 0;
  B2_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  WgradPlan w = wgrad_plan(B, Cin, H, W, Cout, sm_count(dev), /*allow_pair=*/false);
  if (w.m_total + 2LL * (W + 2) + 2 + W + 3 + BK >= (1LL << 31))
    return set_error(B2_ERR_UNSUPPORTED, "b2_conv3x3_wgrad_noalloc: too many padded rows");
  if (w.workspace > kNoAllocScratchBytes) {  // fewer splits, same result up to fp32 summation order
    const int max_splits = int(kNoAllocScratchBytes / per_split);
    w.kb_per_split = (w.num_kb + max_splits - 1) / max_splits;
    w.splits = (w.num_kb + w.kb_per_split - 1) / w.kb_per_split;
    w.workspace = size_t(w.splits) * per_split;
  }
  float* scratch = nullptr;
  B2_TRY(noalloc_scratch(&scratch));
  const int cpo = ((Cout + 63) / 64) * 64;
  const int cpi = ((Cin + 63) / 64) * 64;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[3] = {uint64_t(cpo), uint64_t(w.m_total), 1};
    const uint64_t strides[2] = {uint64_t(cpo) * 2, uint64_t(cpo) * 2 * w.m_total};
    const uint32_t box[3] = {64, 64, 1};
    B2_TRY(encode_tmap(&ta, dy_rows, 3, dims, strides, box, true));
  }
  {
    const uint64_t dims[3] = {uint64_t(cpi), uint64_t(w.m_total), 1};
    const uint64_t strides[2] = {uint64_t(cpi) * 2, uint64_t(cpi) * 2 * w.m_total};
    const uint32_t box[3] = {64, 64, 1};
    B2_TRY(encode_tmap(&tb, x_rows, 3, dims, strides, box, true));
  }
  Params p{};
  p.tiles_m = w.tiles_m;
  p.tiles_n = 1;
  p.splits = w.splits;
  p.batch = 1;
  p.num_kb = w.num_kb;
  p.kb_per_split = w.kb_per_split;
  p.wp = W + 2;
  p.hp = H + 2;
  p.H = H;
  p.W = W;
  p.m_total = int(w.m_total);
  p.a_row_shift = W + 3;
  p.ci_blocks = w.ci_blocks;
  p.M = Cout;
  p.N = Cin;
  p.partial = scratch;
  p.alpha = 1.f;
  p.status = device_status_ptr();
  const int tiles = w.splits * w.tiles_m * 9 * w.ci_blocks;
  if (w.BN == 256)
    B2_TRY((launch<256, kStages256, kWgrad, true, true>(ta, tb, p, tiles, st)));
  else if (w.BN == 64)
    B2_TRY((launch<64, kStages64, kWgrad, true, true>(ta, tb, p, tiles, st)));
  else
    B2_TRY((launch<128, kStages128, kWgrad, true, true>(ta, tb, p, tiles, st)));
  const long long total = (long long)Cout * Cin * 9;
  const int threads = 256;
  const int blocks = int(std::min<long long>((total + threads - 1) / threads, 148LL * 16));
  wgrad_reduce_kernel<<<blocks, threads, 0, st>>>(scratch, dw, dw_dtype, w.splits, Cout, Cin);
  return check_cuda(cudaGetLastError(), "wgrad reduce launch (no-alloc)");
}

}  // extern "C"
