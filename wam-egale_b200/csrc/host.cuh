// Host-side helpers shared by the C-ABI entry points: error reporting,
// TMA tensor-map encoding (driver entry point fetched through the runtime, so
// the library does not link libcuda directly) and per-device properties.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <utility>
#include <string>

#include "../../include/wamb.h"

namespace wamb {

inline thread_local std::string g_last_error;

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define WAMB_CHECK_CUDA(expr)                                                              \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return ::wamb::fail(WAMB_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

#define WAMB_REQUIRE(cond, code, ...)                 \
  do {                                                \
    if (!(cond)) return ::wamb::fail(code, __VA_ARGS__); \
  } while (0)

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D tensor map over a row-major matrix [rows, cols] with row stride
// `ld` elements. Box = box_cols x box_rows, 128-byte swizzle, zero fill
// outside the matrix.
inline int make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                        uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                        uint32_t box_cols) {
  auto fn = encode_fn();
  WAMB_REQUIRE(fn != nullptr, WAMB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  WAMB_REQUIRE(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, WAMB_ERR_ALIGN,
               "tensor base %p not 16-byte aligned", ptr);
  WAMB_REQUIRE((ld * elem_bytes) % 16 == 0, WAMB_ERR_ALIGN, "row stride %llu not 16-byte aligned",
               (unsigned long long)ld);
  WAMB_REQUIRE(rows > 0 && cols > 0, WAMB_ERR_SHAPE, "empty tensor map");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  WAMB_REQUIRE(r == CUDA_SUCCESS, WAMB_ERR_CUDA, "cuTensorMapEncodeTiled error %d", (int)r);
  return WAMB_OK;
}

inline int make_tmap_bf16(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols,
                          uint64_t ld, uint32_t box_rows) {
  return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, ld, box_rows, 64);
}

// E4M3 operand: 128 bytes (= 128 elements) of K per box row.
inline int make_tmap_e4m3(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols,
                          uint64_t ld, uint32_t box_rows) {
  return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, cols, ld, box_rows, 128);
}

// Launch with programmatic stream serialization (see pdl_wait in
// common.cuh); WAMB_PDL=0 in the environment turns it off (plain launches).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WAMB_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                         Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  WAMB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  return WAMB_OK;
}

struct DeviceInfo {
  int sms = 0;
};

inline int device_info(DeviceInfo* out) {
  static DeviceInfo cache[64];
  static std::mutex mu;
  int dev = 0;
  WAMB_CHECK_CUDA(cudaGetDevice(&dev));
  WAMB_REQUIRE(dev >= 0 && dev < 64, WAMB_ERR_CUDA, "device index %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].sms == 0) {
    int sms = 0;
    WAMB_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    int major = 0, minor = 0;
    WAMB_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    WAMB_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    WAMB_REQUIRE(major == 10 && minor == 0, WAMB_ERR_DEVICE,
                 "this library is built for sm_100a (B200); device %d is sm_%d%d", dev, major,
                 minor);
    cache[dev].sms = sms;
  }
  *out = cache[dev];
  return WAMB_OK;
}

inline bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace wamb
