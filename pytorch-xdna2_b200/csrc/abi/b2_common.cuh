// Shared device helpers for libxdna_b200: bf16 conversions, mbarrier / TMA /
// tcgen05 wrappers written as inline PTX for sm_100a, and the per-device
// status word that kernels use to report a wait that ran out of its limit.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2.h"

namespace b2 {

// ---------------------------------------------------------------------------
// host-side error plumbing (b2_runtime.cu)
// ---------------------------------------------------------------------------
b2_status set_error(b2_status code, const char* fmt, ...);
b2_status check_cuda(cudaError_t e, const char* what);
// Encodes a tiled TMA descriptor through the driver entry point (no libcuda
// link dependency, so the library also loads on machines without a driver).
b2_status encode_tmap(CUtensorMap* map, const void* base, int rank,
                      const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, bool swizzle128);
// Same, with the shared-memory swizzle given in bytes (0, 64 or 128).
b2_status encode_tmap_sw(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);
// Encodes an im2col TMA descriptor over a channels-last bf16 activation
// [B][H][W][C] (element strides sn, sh, sw; channel stride 1) whose pixel
// box is the zero-padded grid: traversal runs over h in [-1, H] and w in
// [-1, W] of each image in turn, so `box_rows` consecutive "pixels" from a
// start (w, h, n) are exactly the padded-grid rows of b2_pack_rows_bf16,
// padding positions and channels >= C filled with zeros.  64 channels per
// pixel, 128-byte swizzle (the same shared-memory image as a tiled load of
// the packed rows).
b2_status encode_tmap_padded_nhwc(CUtensorMap* map, const void* base, int B, int C, int H, int W, int64_t sn,
                                  int64_t sh, int64_t sw, uint32_t box_rows);
int sm_count(int device);
int* device_status_ptr();  // address of the device status word (current device)

#define B2_TRY(expr)                      \
  do {                                    \
    b2_status _s = (expr);                \
    if (_s != B2_OK) return _s;           \
  } while (0)

// ---------------------------------------------------------------------------
// numerics
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf2f(uint16_t v) {
  return __uint_as_float(uint32_t(v) << 16);
}
// Round to nearest even, NaN -> quiet NaN (matches the reference's f2bf,
// region_kernels.cpp:37-43, and __float2bfloat16_rn).
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  uint32_t rounded = (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
  uint32_t qnan = (u >> 16) | 0x40u;
  return uint16_t(((u & 0x7fffffffu) > 0x7f800000u) ? qnan : rounded);
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
}

// ---------------------------------------------------------------------------
// status word + bounded waits
// ---------------------------------------------------------------------------
// Waits give up after this many nanoseconds of %globaltimer; the kernel then
// records B2_ERR_TIMEOUT and unwinds instead of hanging the GPU.
constexpr unsigned long long kWaitLimitNs = 20ull * 1000 * 1000 * 1000;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with `parity` to complete.  Returns false (and records
// B2_ERR_TIMEOUT) if it did not within kWaitLimitNs, or if another role of
// this CTA already gave up (*abort set).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        record_status(status, B2_ERR_TIMEOUT);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map,
                                            uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Tiled load of a 4-D map (channels-last activation: c, w, h, n); any of w,
// h may be negative or past the end (zero fill).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// im2col-mode load of a 4-D channels-last map: 64 channels from c of the
// pixels the map's box traverses from (w, h, n); zero im2col offsets.
__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c, int w,
                                                   int h, int n) {
  const uint16_t z = 0;
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(z), "h"(z)
      : "memory");
}
// Tiled store shared -> global (bulk async-group of the issuing thread).  The
// box is clipped at the tensor's bounds, so partial edge tiles need no masks.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// 1-D bulk copy of `bytes` from global memory into this CTA's shared memory,
// completing on the mbarrier `bar` (both addresses 16-byte aligned, bytes a
// multiple of 16; no multicast).
__device__ __forceinline__ void bulk_load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until all of this thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Makes this thread's shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 in, fp32 acc).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive fp32 columns: thread t of the warp gets row
// (lane quarter base + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// ---------------------------------------------------------------------------
// two-CTA (SM pair) variants: cluster of 2, one MMA issuer for both SMs
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory that completes on an mbarrier of
// either CTA of the pair (the pair's leader counts both CTAs' bytes).  No
// multicast: each CTA loads its own operand halves.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// The 4-D tiled form of tma_load_3d_pair (no multicast).
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// The im2col form of tma_load_3d_pair (no multicast).
__device__ __forceinline__ void tma_load_im2col_4d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                        int c, int w, int h, int n) {
  const uint16_t z = 0;
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c), "r"(w), "r"(h), "r"(n), "h"(z), "h"(z)
      : "memory");
}
// `nrows` (the map's box) consecutive padded-grid rows of 64 channels from
// channel c0, starting at padded row r, from either packed rows (a tiled 2-D
// map) or a channels-last tensor (an encode_tmap_padded_nhwc map): the same
// shared-memory image either way.  Row r of a grid of pitch wp and plane
// rows per image is pixel (r / plane, (r % plane) / wp - 1, r % wp - 1); rows
// past the last image start at n = B and read zeros.
template <bool PAIR>
__device__ __forceinline__ void load_rows(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int r,
                                          bool im2col, int wp, int plane) {
  if (!im2col) {
    if constexpr (PAIR)
      tma_load_3d_pair(dst, map, bar, c0, r, 0);
    else
      tma_load_3d(dst, map, bar, c0, r, 0);
    return;
  }
  const int n = r / plane;
  const int rem = r - n * plane;
  const int yy = rem / wp;
  const int xx = rem - yy * wp;
  if constexpr (PAIR)
    tma_load_im2col_4d_pair(dst, map, bar, c0, xx - 1, yy - 1, n);
  else
    tma_load_im2col_4d(dst, map, bar, c0, xx - 1, yy - 1, n);
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (both CTAs' tensor memory) (+)= A (rows 0-127 from this CTA's smem, 128-255
// from the peer's) * B (N split the same way), kind::f16.
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once, on the barrier at this shared offset in every CTA of `mask`,
// when this thread's issued pair MMAs have completed.
__device__ __forceinline__ void tc_commit_pair_mc(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile
// (tcgen05 "version 1" descriptor): start address, leading-dimension byte
// offset, stride-dimension byte offset, layout type 2 = SWIZZLE_128B.
//   K-major  : rows of 64 bf16 (128 B) along K; SBO = 1024 B between 8-row
//              groups; LBO unused.
//   MN-major : rows of 64 bf16 along M/N, one row per k; SBO = 1024 B between
//              8-k groups, LBO = byte stride between 64-wide M/N blocks.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo,
                                                    uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  d |= uint64_t(2) << 61;  // SWIZZLE_128B
  return d;
}

// An operand that starts `row` 128-byte rows into a 1024-byte aligned block
// written by a 128-byte-swizzled TMA load (any row, also row % 8 != 0) takes
// the block's descriptor with row * 8 added to the start-address field (16-byte
// units): the swizzle phase of each row follows the shared-memory address bits
// on both sides, so the start address alone selects the rows and the matrix
// base offset field stays 0 (checked against the unshifted loads:
// tests/test_gpu_abi.py conv cases on the halo kernels).  The kernels step
// descriptors this way; every shared address is below 2^18, so the 14-bit
// field never carries.

// Instruction descriptor, kind::f16: bf16 x bf16 -> fp32, M x N, operand majors.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                      // D format fp32
         | (1u << 7)                    // A format bf16
         | (1u << 10)                   // B format bf16
         | (uint32_t(a_mn) << 15)       // A major (0 = K)
         | (uint32_t(b_mn) << 16)       // B major (0 = K)
         | (uint32_t(N >> 3) << 17)     // N / 8
         | (uint32_t(M >> 4) << 24);    // M / 16
}

}  // namespace b2
