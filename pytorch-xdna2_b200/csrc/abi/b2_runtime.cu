// Runtime pieces of libxdna_b200: thread-local last error, CUDA error
// mapping, TMA descriptor encoding through the driver entry point, SM count
// cache and the per-device status word that kernels write on a failed wait.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "b2_common.cuh"

namespace {

thread_local char g_last_error[512] = "";

// One status word per device.  Its device address is looked up once per
// device (cudaGetSymbolAddress with that device current) and handed to every
// kernel as a plain pointer.
__device__ int g_device_status;

constexpr int kMaxDevices = 64;
int* g_status_addr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
PFN_cuTensorMapEncodeIm2col_v12000 g_encode_im2col = nullptr;

}  // namespace

namespace b2 {

b2_status set_error(b2_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
  va_end(ap);
  return code;
}

b2_status check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B2_OK;
  return set_error(B2_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status_addr[dev] = static_cast<int*>(p);
  }
  return g_status_addr[dev];
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sm_count[device]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        n <= 0)
      n = 148;
    g_sm_count[device] = n;
  }
  return g_sm_count[device];
}

b2_status encode_tmap(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  return encode_tmap_sw(map, base, rank, dims, strides_bytes, box, swizzle128 ? 128 : 0);
}

b2_status encode_tmap_sw(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q{};
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return set_error(B2_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(B2_ERR_UNSUPPORTED, "TMA base address %p not 16-byte aligned", base);
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) {
      if (strides_bytes[i] % 16 != 0)
        return set_error(B2_ERR_UNSUPPORTED, "TMA stride %llu not a multiple of 16 bytes",
                         (unsigned long long)strides_bytes[i]);
      gstride[i] = strides_bytes[i];
    }
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), gdim,
                        gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                        : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(B2_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return B2_OK;
}

b2_status encode_tmap_padded_nhwc(CUtensorMap* map, const void* base, int B, int C, int H, int W, int64_t sn,
                                  int64_t sh, int64_t sw, uint32_t box_rows) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode_im2col) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q{};
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return set_error(B2_ERR_CUDA, "cuTensorMapEncodeIm2col entry point unavailable");
      g_encode_im2col = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(fn);
    }
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(B2_ERR_UNSUPPORTED, "TMA base address %p not 16-byte aligned", base);
  if (C % 8 || sw % 8 || sh % 8 || sn % 8 || sw < C || box_rows < 1 || box_rows > 256)
    return set_error(B2_ERR_UNSUPPORTED, "channels-last operand: C and the pixel strides must be multiples of 8");
  cuuint64_t gdim[4] = {cuuint64_t(C), cuuint64_t(W), cuuint64_t(H), cuuint64_t(B)};
  cuuint64_t gstride[3] = {cuuint64_t(sw) * 2, cuuint64_t(sh) * 2, cuuint64_t(sn) * 2};
  const int lower[2] = {-1, -1};  // the padded grid: one zero row / column before ...
  const int upper[2] = {1, 1};    // ... and after the image
  cuuint32_t estride[4] = {1, 1, 1, 1};
  CUresult r = g_encode_im2col(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), gdim, gstride,
                               lower, upper, 64, box_rows, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(B2_ERR_CUDA, "cuTensorMapEncodeIm2col failed (%d)", int(r));
  return B2_OK;
}

}  // namespace b2

extern "C" {

const char* b2_last_error(void) { return g_last_error; }

int b2_abi_version(void) { return 1; }

b2_status b2_device_status(int device, int* code) {
  if (!code) return b2::set_error(B2_ERR_INVALID, "b2_device_status: null code");
  int prev = 0;
  B2_TRY(b2::check_cuda(cudaGetDevice(&prev), "cudaGetDevice"));
  B2_TRY(b2::check_cuda(cudaSetDevice(device), "cudaSetDevice"));
  b2_status st = B2_OK;
  int* p = b2::device_status_ptr();
  if (!p) {
    st = b2::set_error(B2_ERR_CUDA, "device status word unavailable");
  } else {
    int v = 0, zero = 0;
    st = b2::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    if (st == B2_OK) st = b2::check_cuda(cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost), "read status");
    if (st == B2_OK) st = b2::check_cuda(cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice), "clear status");
    *code = v;
  }
  cudaSetDevice(prev);
  return st;
}

}  // extern "C"
