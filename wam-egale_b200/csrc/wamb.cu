// libwamb.so: the single translation unit of the B200 Wan-DiT block library.
// The C-ABI declared in include/wamb.h is defined here; kernels live in the
// included headers.
#include "common.cuh"
#include "host.cuh"
#include "linear.cuh"

extern "C" {

const char* wamb_last_error(void) { return wamb::g_last_error.c_str(); }

int wamb_abi_version(void) { return 100; }

int wamb_device_status(void* stream, int* device_code) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  WAMB_CHECK_CUDA(cudaStreamSynchronize(s));
  int v = 0;
  WAMB_CHECK_CUDA(cudaMemcpyFromSymbol(&v, wamb::g_error, sizeof(int)));
  const int zero = 0;
  WAMB_CHECK_CUDA(cudaMemcpyToSymbol(wamb::g_error, &zero, sizeof(int)));
  if (device_code) *device_code = v;
  return WAMB_OK;
}

int wamb_linear(const wamb_linear_args* args, void* stream) {
  return wamb::linear_impl(args, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
