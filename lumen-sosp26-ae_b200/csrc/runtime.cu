// Process-wide runtime pieces of liblumen_b200.so: device properties, the device
// status word, and tensor-map encoding through the driver entry point (the
// library does not link libcuda; it asks the runtime for cuTensorMapEncodeTiled).
#include <mutex>

#include "lumen_b200_internal.h"

namespace b200 {

namespace {
constexpr int kMaxDevices = 64;
__device__ int g_status_word;

std::mutex g_mu;
int g_sm_count[kMaxDevices];
int* g_status_ptr[kMaxDevices];

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_encode) return g_encode;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) !=
          cudaSuccess ||
      qres != cudaDriverEntryPointSuccess)
    return nullptr;
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return g_encode;
}
}  // namespace

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

int encode_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t gdim[5];
  cuuint64_t gstr[5];
  cuuint32_t bdim[5];
  cuuint32_t estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstr[i] = strides_bytes[i];
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                        const_cast<void*>(base), gdim, gstr, bdim, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

int encode_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld_bytes,
                      uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstr[1] = {ld_bytes};
  const cuuint32_t bdim[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstr, bdim, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS ? 0 : -1;
}

int encode_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                        uint64_t ld_elems, uint32_t box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {ld_elems * 2};
  const uint32_t box[2] = {64, box_rows};
  return encode_tmap_bf16(map, base, 2, dims, strides, box);
}

}  // namespace b200

extern "C" const char* lumen_b200_version(void) { return "lumen_b200 0.1 sm_100a"; }

extern "C" int lumen_b200_sm_count(void) {
  const int n = b200::device_sm_count();
  return n > 0 ? n : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_device_status(int* status) {
  if (!status) return LUMEN_B200_EINVAL;
  int* p = b200::device_status_word();
  if (!p) return LUMEN_B200_ECUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return LUMEN_B200_ECUDA;
  if (cudaMemcpy(status, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return LUMEN_B200_ECUDA;
  return *status == 0 ? LUMEN_B200_OK : LUMEN_B200_EDEVICE;
}

extern "C" int lumen_b200_clear_status(void) {
  int* p = b200::device_status_word();
  if (!p) return LUMEN_B200_ECUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return LUMEN_B200_ECUDA;
  return cudaMemset(p, 0, sizeof(int)) == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_status_snapshot(int* host_dst, void* stream) {
  if (!host_dst) return LUMEN_B200_EINVAL;
  int* p = b200::device_status_word();
  if (!p) return LUMEN_B200_ECUDA;
  return cudaMemcpyAsync(host_dst, p, sizeof(int), cudaMemcpyDeviceToHost,
                         static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? LUMEN_B200_OK
             : LUMEN_B200_ECUDA;
}
