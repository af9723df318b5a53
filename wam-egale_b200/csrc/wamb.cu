// libwamb.so: the single translation unit of the B200 Wan-DiT block library.
// The C-ABI declared in include/wamb.h is defined here; kernels live in the
// included headers.
#include "common.cuh"
#include "host.cuh"
#include "linear.cuh"
#include "block.cuh"
#include "model.cuh"
#include "speculative.cuh"

#include <cmath>

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

int wamb_abi_version(void) { return 107; }

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
  using namespace wamb;
  if (args == nullptr || args->sk_workspace == nullptr) return linear_impl(args, static_cast<cudaStream_t>(stream));
  WAMB_REQUIRE(reinterpret_cast<uintptr_t>(args->sk_workspace) % 256 == 0, WAMB_ERR_ALIGN,
               "sk_workspace must be 256-byte aligned");
  SkBuffers sk;
  if (args->sk_workspace_bytes >= SK_FLAG_BYTES) {
    uint8_t* w = static_cast<uint8_t*>(args->sk_workspace);
    sk.flags = reinterpret_cast<int*>(w);
    sk.part = reinterpret_cast<float*>(w + SK_FLAG_BYTES);
    sk.part_bytes = args->sk_workspace_bytes - SK_FLAG_BYTES;
  }
  return linear_impl(args, static_cast<cudaStream_t>(stream), false, false, 0, false, &sk);
}

size_t wamb_linear_sk_bytes(void) {
  wamb::DeviceInfo di;
  if (wamb::device_info(&di) != WAMB_OK) return 0;
  return wamb::SK_FLAG_BYTES + wamb::sk_part_bytes(di.sms);
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
  using namespace wamb;
  if (args == nullptr || args->split_workspace == nullptr)
    return attention_impl(args, static_cast<cudaStream_t>(stream));
  WAMB_REQUIRE(reinterpret_cast<uintptr_t>(args->split_workspace) % 256 == 0, WAMB_ERR_ALIGN,
               "split_workspace must be 256-byte aligned");
  AttnSplitBuffers sb;
  if (args->split_workspace_bytes >= ATT_COUNT_BYTES) {
    uint8_t* w = static_cast<uint8_t*>(args->split_workspace);
    sb.count = reinterpret_cast<int*>(w);
    sb.part = reinterpret_cast<float*>(w + ATT_COUNT_BYTES);
    sb.part_bytes = args->split_workspace_bytes - ATT_COUNT_BYTES;
  }
  return attention_impl(args, static_cast<cudaStream_t>(stream), false, &sb);
}

size_t wamb_attention_split_bytes(const wamb_attention_args* args) {
  using namespace wamb;
  if (args == nullptr) return 0;
  DeviceInfo di;
  if (device_info(&di) != WAMB_OK) return 0;
  const size_t part = attn_part_bytes(args, di.sms, args->kv_splits);
  return part > 0 ? ATT_COUNT_BYTES + part : 0;
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
  const size_t need = wamb::block_layout(args).total;
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

int wamb_timestep_embedding(const float* t, int32_t n, int32_t dim, void* out, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(n >= 0 && dim > 0 && dim % 2 == 0, WAMB_ERR_SHAPE, "timestep embedding: n >= 0, even dim");
  if (n == 0) return WAMB_OK;
  WAMB_REQUIRE(t && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(timestep_embed_kernel, dim3(elem_grid(static_cast<long long>(n) * dim / 2, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       t, n, dim, static_cast<__nv_bfloat16*>(out));
}

int wamb_silu(const void* x, int64_t ldx, int32_t x_is_f32, int32_t m, int32_t n, void* out, int64_t ldo,
              void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(m >= 0 && n > 0 && ldx >= n && ldo >= n, WAMB_ERR_SHAPE, "silu shape");
  if (m == 0) return WAMB_OK;
  WAMB_REQUIRE(x && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(silu_kernel, dim3(elem_grid(static_cast<long long>(m) * n, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       
      x, ldx, x_is_f32, m, n, static_cast<__nv_bfloat16*>(out), ldo);
}

int wamb_embed_gather(const void* x, int32_t b, int32_t c, int32_t f, int32_t h, int32_t w, int32_t p1,
                      int32_t p2, int32_t p3, void* out, int32_t ldo, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(b >= 0 && c > 0 && f > 0 && h > 0 && w > 0 && p1 > 0 && p2 > 0 && p3 > 0 &&
                   f % p1 == 0 && h % p2 == 0 && w % p3 == 0 && ldo >= c * p1 * p2 * p3,
               WAMB_ERR_SHAPE, "embed gather shape");
  if (b == 0) return WAMB_OK;
  WAMB_REQUIRE(x && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  GatherParams p{static_cast<const __nv_bfloat16*>(x), b, c, f, h, w, p1, p2, p3,
                 static_cast<__nv_bfloat16*>(out), ldo};
  const long long total = static_cast<long long>(b) * (f / p1) * (h / p2) * (w / p3) * ldo;
  return launch_kernel(embed_gather_kernel, dim3(elem_grid(total, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       p);
}

int wamb_output_norm(const void* x, int32_t x_is_f32, int32_t m, int32_t d, double eps, const float* table,
                     const void* temb, int32_t temb_is_f32, int32_t temb_len, int32_t rows_per_batch,
                     void* out, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(m >= 0 && rows_per_batch > 0 && (temb_len == 1 || temb_len == rows_per_batch) &&
                   m % rows_per_batch == 0,
               WAMB_ERR_SHAPE, "output norm shape");
  WAMB_REQUIRE(row_vpt(d) > 0, WAMB_ERR_SHAPE, "d=%d unsupported by the row kernels", d);
  if (m == 0) return WAMB_OK;
  WAMB_REQUIRE(x && table && temb && out, WAMB_ERR_ARG, "null pointer");
  LnParams p{};
  p.x = x; p.x_f32 = x_is_f32; p.ldx = d;
  p.out = static_cast<__nv_bfloat16*>(out); p.ldo = d;
  p.M = m; p.D = d; p.eps = static_cast<float>(eps); p.affine = 0;
  p.table = table; p.temb = temb; p.temb_f32 = temb_is_f32; p.temb_L = temb_len;
  p.rows_per_batch = rows_per_batch; p.shift_idx = 0; p.scale_idx = 1; p.temb_rows = 1;
  return launch_ln(p, static_cast<cudaStream_t>(stream));
}

int wamb_copy_cols(const void* x, int64_t ldx_bytes, int32_t m, int32_t n_bytes, void* out, int64_t ldo_bytes,
                   void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(m >= 0 && n_bytes > 0 && ldx_bytes >= n_bytes && ldo_bytes >= n_bytes, WAMB_ERR_SHAPE,
               "copy_cols shape");
  if (m == 0) return WAMB_OK;
  WAMB_REQUIRE(x && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(copy_cols_kernel, dim3(elem_grid(static_cast<long long>(m) * n_bytes, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const uint8_t*>(x), ldx_bytes, m, n_bytes,
                                                          static_cast<uint8_t*>(out), ldo_bytes);
}

int wamb_repeat_rows(const void* x, int32_t rows, int32_t row_bytes, int32_t repeat, void* out, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(rows >= 0 && row_bytes > 0 && repeat >= 1, WAMB_ERR_SHAPE, "repeat_rows shape");
  if (rows == 0) return WAMB_OK;
  WAMB_REQUIRE(x && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(repeat_rows_kernel, dim3(elem_grid(static_cast<long long>(rows) * repeat * row_bytes, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const uint8_t*>(x), rows, row_bytes, repeat,
                                                            static_cast<uint8_t*>(out));
}

int wamb_flow_step_cl(void* sample, int32_t sample_is_f32, const void* v, int32_t v_is_f32, int32_t b, int32_t c,
                      int64_t l, float dsigma, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(b >= 0 && c > 0 && l >= 0, WAMB_ERR_SHAPE, "flow step shape");
  const long long n = static_cast<long long>(b) * c * l;
  if (n == 0) return WAMB_OK;
  WAMB_REQUIRE(sample && v, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(flow_step_cl_kernel, dim3(elem_grid(n, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       
      sample, sample_is_f32, v, v_is_f32, b, c, l, dsigma);
}

int wamb_flow_step(void* sample, int32_t sample_is_f32, const void* v, int32_t v_is_f32, int64_t n, float dsigma,
                   void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(n >= 0, WAMB_ERR_SHAPE, "flow step size");
  if (n == 0) return WAMB_OK;
  WAMB_REQUIRE(sample && v, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(flow_step_kernel, dim3(elem_grid(n, di.sms)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       sample, sample_is_f32, v, v_is_f32, n, dsigma);
}

// ------------------------------------------------- speculative decoding
int wamb_draft_forward(const wamb_draft_params* p, const void* state, const void* previous, int32_t io_is_f32,
                       const float* scalars, int32_t batch, void* out, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(p != nullptr, WAMB_ERR_ARG, "null draft params");
  WAMB_REQUIRE(p->tokens == DR_T && p->width == DR_E && p->heads == DR_H && p->ffn == DR_F, WAMB_ERR_SHAPE,
               "draft shape tokens %d width %d heads %d ffn %d (supported: %d, %d, %d, %d)", p->tokens, p->width,
               p->heads, p->ffn, DR_T, DR_E, DR_H, DR_F);
  WAMB_REQUIRE(p->channels >= 1 && p->channels <= DR_AMAX, WAMB_ERR_SHAPE, "draft channels %d (1..%d)",
               p->channels, DR_AMAX);
  WAMB_REQUIRE(batch >= 0 && (io_is_f32 == 0 || io_is_f32 == 1), WAMB_ERR_ARG, "batch / dtype");
  if (batch == 0) return WAMB_OK;
  const float* w[] = {p->embed_w, p->embed_b, p->position, p->in_proj_w, p->in_proj_b, p->out_proj_w,
                      p->out_proj_b, p->linear1_w, p->linear1_b, p->linear2_w, p->linear2_b, p->norm1_w,
                      p->norm1_b, p->norm2_w, p->norm2_b, p->head_w, p->head_b, p->feature_mean,
                      p->feature_std, p->residual_mean, p->residual_std};
  for (const float* x : w) WAMB_REQUIRE(x != nullptr, WAMB_ERR_ARG, "null draft weight");
  WAMB_REQUIRE(state && previous && scalars && out, WAMB_ERR_ARG, "null draft input / output");
  static bool configured[64] = {};
  int dev = 0;
  WAMB_CHECK_CUDA(cudaGetDevice(&dev));
  WAMB_REQUIRE(dev >= 0 && dev < 64, WAMB_ERR_CUDA, "device index %d", dev);
  if (!configured[dev]) {
    WAMB_CHECK_CUDA(cudaFuncSetAttribute(draft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         DraftSmem::BYTES));
    configured[dev] = true;
  }
  DraftArgs a{};
  a.A = p->channels;
  a.eps = p->ln_eps;
  a.embed_w = p->embed_w; a.embed_b = p->embed_b; a.position = p->position;
  a.ln1_w = p->norm1_w; a.ln1_b = p->norm1_b; a.in_w = p->in_proj_w; a.in_b = p->in_proj_b;
  a.out_w = p->out_proj_w; a.out_b = p->out_proj_b; a.ln2_w = p->norm2_w; a.ln2_b = p->norm2_b;
  a.l1_w = p->linear1_w; a.l1_b = p->linear1_b; a.l2_w = p->linear2_w; a.l2_b = p->linear2_b;
  a.head_w = p->head_w; a.head_b = p->head_b;
  a.fmean = p->feature_mean; a.fstd = p->feature_std; a.rmean = p->residual_mean; a.rstd = p->residual_std;
  a.state = state; a.previous = previous; a.io_f32 = io_is_f32; a.scalars = scalars; a.out = out;
  return launch_kernel(draft_kernel, dim3(batch), dim3(DR_THREADS), DraftSmem::BYTES,
                       static_cast<cudaStream_t>(stream), a);
}

int wamb_spec_scores(const void* draft, const void* target, int32_t io_is_f32, int64_t n, int32_t edges,
                     const int32_t* draft_rows, const int32_t* target_rows, const float* scales,
                     int32_t scale_inside, float* scores, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(edges >= 0 && edges <= SPEC_MAX_EDGES && n > 0, WAMB_ERR_SHAPE, "edges %d (0..%d), n %lld", edges,
               SPEC_MAX_EDGES, static_cast<long long>(n));
  if (edges == 0) return WAMB_OK;
  WAMB_REQUIRE(draft && target && draft_rows && target_rows && scales && scores, WAMB_ERR_ARG, "null pointer");
  SpecEdges e{};
  e.n = edges;
  e.scale_inside = scale_inside ? 1 : 0;
  for (int k = 0; k < edges; ++k) {
    WAMB_REQUIRE(draft_rows[k] >= 0 && target_rows[k] >= 0, WAMB_ERR_ARG, "negative row");
    e.d[k] = draft_rows[k];
    e.t[k] = target_rows[k];
    e.scale[k] = scales[k];
  }
  return launch_kernel(spec_scores_kernel, dim3(edges), dim3(256), 0, static_cast<cudaStream_t>(stream), draft,
                       target, io_is_f32, static_cast<long long>(n), e, scores);
}

int wamb_spec_route(const float* scores, int32_t mode, double tau, int32_t* route, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(mode >= 0 && mode <= 2, WAMB_ERR_ARG, "route mode %d", mode);
  WAMB_REQUIRE(mode != 0 || (std::isfinite(tau) && tau >= 0.0), WAMB_ERR_ARG, "tau must be finite and >= 0");
  WAMB_REQUIRE(scores && route, WAMB_ERR_ARG, "null pointer");
  return launch_kernel(spec_route_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), scores, mode,
                       tau, route);
}

int wamb_spec_expand(const void* base, const void* dirs, int32_t io_is_f32, int32_t rows, int32_t fan, int64_t n,
                     float delta, void* out, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(rows >= 0 && fan >= 1 && n >= 0, WAMB_ERR_SHAPE, "rows / fan / n");
  if (rows == 0 || n == 0) return WAMB_OK;
  WAMB_REQUIRE(base && dirs && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(spec_expand_kernel, dim3(elem_grid(static_cast<long long>(rows) * n, di.sms)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), base, dirs, out, io_is_f32, rows, fan,
                       static_cast<long long>(n), delta);
}

int wamb_spec_commit(const int32_t* route, const void* values, const void* tree, int32_t io_is_f32, int64_t n,
                     float delta0, float delta1, float delta2, void* state_out, void* previous_out, void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(n >= 0, WAMB_ERR_SHAPE, "n");
  if (n == 0) return WAMB_OK;
  WAMB_REQUIRE(route && values && tree && state_out && previous_out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(spec_commit_kernel, dim3(elem_grid(n, di.sms)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), route, values, tree, io_is_f32, static_cast<long long>(n),
                       delta0, delta1, delta2, state_out, previous_out);
}

int wamb_cfg_combine(const void* cond, const void* uncond, int32_t io_is_f32, int64_t n, float scale, void* out,
                     void* stream) {
  using namespace wamb;
  WAMB_REQUIRE(n >= 0, WAMB_ERR_SHAPE, "n");
  if (n == 0) return WAMB_OK;
  WAMB_REQUIRE(cond && uncond && out, WAMB_ERR_ARG, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  return launch_kernel(cfg_combine_kernel, dim3(elem_grid(n, di.sms)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), cond, uncond, out, io_is_f32, static_cast<long long>(n),
                       scale);
}

}  // extern "C"
