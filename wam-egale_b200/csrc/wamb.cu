// libwamb.so: the single translation unit of the B200 Wan-DiT block library.
// The C-ABI declared in include/wamb.h is defined here; kernels live in the
// included headers.
#include "common.cuh"
#include "host.cuh"
#include "linear.cuh"
#include "block.cuh"

namespace wamb {

// Scratch of wamb_block_forward_noalloc: a fixed device array, so that the
// entry point never calls the allocator. Host code must not pass the symbol
// itself to a kernel (on the host it only names the array); its device
// address is looked up once per device with cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[WAMB_NOALLOC_SCRATCH_BYTES];

inline int noalloc_scratch_address(void** out) {
  static void* addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  WAMB_CHECK_CUDA(cudaGetDevice(&dev));
  WAMB_REQUIRE(dev >= 0 && dev < 64, WAMB_ERR_CUDA, "device index %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    WAMB_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    WAMB_REQUIRE(p != nullptr && reinterpret_cast<uintptr_t>(p) % 256 == 0, WAMB_ERR_CUDA,
                 "scratch array address %p", p);
    addr[dev] = p;
  }
  *out = addr[dev];
  return WAMB_OK;
}

}  // namespace wamb

extern "C" {

const char* wamb_last_error(void) { return wamb::g_last_error.c_str(); }

int wamb_abi_version(void) { return 102; }

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

int wamb_quantize_rows(const void* x, int64_t ldx, int32_t x_is_f32, int32_t m, int32_t k, void* out,
                       int64_t ldo, float* scale, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(m >= 0 && k > 0 && k % 8 == 0, WAMB_ERR_SHAPE, "quantize: m >= 0, k %% 8 == 0");
  WAMB_REQUIRE(x_is_f32 == 0 || x_is_f32 == 1, WAMB_ERR_ARG, "x_is_f32 must be 0 or 1");
  WAMB_REQUIRE(ldx >= k && ldo >= k && ldx % 8 == 0 && ldo % 16 == 0, WAMB_ERR_ALIGN, "ldx / ldo");
  WAMB_REQUIRE(x && out && scale && aligned16(x) && aligned16(out) && aligned16(scale), WAMB_ERR_ALIGN,
               "null or misaligned pointer");
  QuantParams p{};
  p.x = x; p.ldx = ldx; p.x_f32 = x_is_f32; p.M = m; p.K = k;
  p.out = static_cast<uint8_t*>(out); p.ldo = ldo; p.scale = scale;
  return launch_quant(p, static_cast<cudaStream_t>(stream));
}

int wamb_attention(const wamb_attention_args* args, void* stream) {
  return wamb::attention_impl(args, static_cast<cudaStream_t>(stream));
}

size_t wamb_block_workspace_bytes(const wamb_block_args* args) {
  if (args == nullptr) return 0;
  return wamb::block_layout(args).total;
}

size_t wamb_block_workspace_layout(const wamb_block_args* args, int64_t* offsets) {
  if (args == nullptr) return 0;
  const wamb::BlockLayout L = wamb::block_layout(args);
  if (offsets != nullptr)
    for (int i = 0; i < WAMB_TAP_COUNT; ++i) offsets[i] = L.off[i];
  return L.total;
}

int wamb_block_forward(const wamb_block_args* args, void* stream) {
  return wamb::block_forward_impl(args, static_cast<cudaStream_t>(stream));
}

int wamb_block_forward_noalloc(const wamb_block_args* args, void* stream) {
  if (args == nullptr) return wamb::fail(WAMB_ERR_ARG, "null args");
  // The block's minimum workspace must fit; the optional split-K scratch is
  // used when the array has room for it too.
  const size_t need = wamb::block_layout(args).minimum;
  if (need > WAMB_NOALLOC_SCRATCH_BYTES)
    return wamb::fail(WAMB_ERR_WORKSPACE,
                      "this block call needs %zu bytes of scratch; the no-allocation entry point "
                      "has %u (use wamb_block_forward with a workspace)",
                      need, WAMB_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = wamb::noalloc_scratch_address(&scratch);
  if (rc) return rc;
  wamb_block_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = WAMB_NOALLOC_SCRATCH_BYTES;
  return wamb::block_forward_impl(&a, static_cast<cudaStream_t>(stream));
}

int wamb_cross_kv(const wamb_block_args* args, void* k_out, void* v_out, void* stream) {
  if (args == nullptr) return wamb::fail(WAMB_ERR_ARG, "null args");
  return wamb::cross_kv_impl(args, k_out, v_out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
