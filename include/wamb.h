/*
 * wamb.h - C ABI of the B200 (sm_100a) Wan-DiT transformer block library
 * (libwamb.so).
 *
 * Plain pointers and sizes only: every tensor is a device pointer to a
 * contiguous row-major array whose dtype is stated beside it. All calls are
 * asynchronous on the given CUDA stream (a cudaStream_t passed as void*; NULL
 * = legacy default stream) and return 0 on success or a wamb_status code;
 * wamb_last_error() then describes the failure (thread-local). Kernel-side
 * failures (a bounded device wait that expired, a KV-cache contract error
 * found on the device) are recorded in a per-device error word that
 * wamb_device_status() reads.
 *
 * Each entry point names the interface of the reference project
 * (qingyiyi/WAM-egale, paths under 算子研究/wam_ops/ and
 * 投机采样/wam-p0-worktree/wan_va/modules/model.py) that it replaces.
 */
#ifndef WAMB_H
#define WAMB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WAMB_API __attribute__((visibility("default")))
#else
#define WAMB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum wamb_status {
  WAMB_OK = 0,
  WAMB_ERR_ARG = 1,       /* null pointer / unsupported option */
  WAMB_ERR_SHAPE = 2,     /* dimension outside the supported contract */
  WAMB_ERR_ALIGN = 3,     /* pointer or stride not 16-byte aligned */
  WAMB_ERR_CUDA = 4,      /* CUDA runtime / driver error */
  WAMB_ERR_KV = 5,        /* KV-cache contract violation (host-detectable) */
  WAMB_ERR_DEVICE = 6,    /* wrong GPU architecture */
  WAMB_ERR_WORKSPACE = 7, /* workspace missing or too small */
  WAMB_ERR_DEVICE_STATUS = 8 /* a kernel recorded an error (see wamb_device_status) */
};

/* Device error codes returned through wamb_device_status(). */
enum wamb_device_code {
  WAMB_DEV_OK = 0,
  WAMB_DEV_WAIT_TIMEOUT = 1,  /* a bounded mbarrier wait expired; kernel returned early */
  WAMB_DEV_KV_LAYOUT = 2,     /* KV pool metadata inconsistent */
  WAMB_DEV_BAD_ROW = 3,       /* candidate_cache_rows entry outside [0, pool_batch) */
  WAMB_DEV_POOL_FULL = 4      /* not enough slots even after eviction */
};

/* Thread-local text of the last host-side failure. */
WAMB_API const char* wamb_last_error(void);
/* ABI version (major * 100 + minor). */
WAMB_API int wamb_abi_version(void);
/* Synchronises `stream`, then returns the current device's error word in
 * *device_code and clears it. Returns WAMB_OK or WAMB_ERR_CUDA. */
WAMB_API int wamb_device_status(void* stream, int* device_code);

/* Epilogues of wamb_linear (values of wamb_linear_args.epilogue). */
enum wamb_epilogue {
  WAMB_EPI_BIAS = 0,     /* out = bf16(A W^T + b) */
  WAMB_EPI_GELU = 1,     /* out = bf16(gelu_tanh(A W^T + b)) */
  WAMB_EPI_RES = 2,      /* out = bf16(res + (A W^T + b)) */
  WAMB_EPI_RES_GATE = 3, /* out = bf16(res + (A W^T + b) * (table[g] + temb[b, l, g])) */
  WAMB_EPI_SILU = 4      /* out = silu(A W^T + b) (timestep embedder) */
};

/*
 * Dense projection Y = A W^T + b on the tcgen05 tensor cores, with a fused
 * epilogue. Replaces the reference's cuBLASLt `linear(x, w, b)`
 * (算子研究/wam_ops/baseline/csrc/gemm.h:35-77) and the fused FFN1+GELU
 * `ffn1_gelu_out` (算子研究/wam_ops/optimized/csrc/ffn.cu:100-104); the
 * residual epilogues replace `residual_kernel` (baseline/csrc/block.cu:90-102).
 *
 * The N output columns are split into `groups` (1..3) equal column groups;
 * group g reads weight[g] ([n_per_group, K] bf16) and bias[g] ([n_per_group]
 * bf16, may be NULL). Requirements: K % 64 == 0, n_per_group % 64 == 0,
 * lda / ldo / ldr multiples of 8, all pointers 16-byte aligned.
 */
typedef struct wamb_linear_args {
  const void* a;          /* [M, lda] bf16 */
  int64_t lda;
  int32_t m, k;
  int32_t groups;
  int32_t n_per_group;
  const void* weight[3];  /* [n_per_group, K] bf16 each */
  const void* bias[3];    /* [n_per_group] bf16 each, or NULL */
  void* out;              /* [M, ldo] bf16, or fp32 when out_is_f32 */
  int64_t ldo;
  int32_t epilogue;       /* enum wamb_epilogue */
  const void* res;        /* [M, ldr] bf16 (RES / RES_GATE), or fp32 when res_is_f32 */
  int64_t ldr;
  int32_t res_is_f32, out_is_f32;
  /* RES_GATE: gate = table[gate_index*D + col] + temb[((b*temb_len + l)*6 + gate_index)*D + col]
   * with b = row / rows_per_batch and l = 0 if temb_len == 1 else row % rows_per_batch. */
  const float* table;     /* [6, D] fp32 */
  const void* temb;       /* [B, temb_len, 6, D] fp32 (temb_is_f32) or bf16 */
  int32_t temb_is_f32;
  int32_t temb_len;
  int32_t rows_per_batch;
  int32_t gate_index;
  int32_t dim;            /* D (= N for the gated epilogue) */
  /* FP8 operands (no counterpart in the reference, which is bf16-only,
   * baseline/csrc/gemm.h:36-38). a_is_fp8 = 1: A is [M, lda] E4M3 bytes with
   * the per-row scale a_scale[M] (fp32), weight[g] is [n_per_group, K] E4M3
   * with the per-output-channel scale w_scale[g][n_per_group] (fp32); the
   * fp32 accumulator is multiplied by a_scale[row] * w_scale[g][col] before
   * the bias and the epilogue. Requires K % 128 == 0 and lda % 16 == 0. */
  int32_t a_is_fp8;
  const float* a_scale;
  const float* w_scale[3];
  /* Optional stream-K scratch for M >= 512 (NULL: none) of
   * wamb_linear_sk_bytes() bytes, 256-byte aligned, zero-filled before its
   * first use (the library leaves its flags zero after every call). With
   * it, a GEMM whose 256 x 256 tiles leave the last round over the SM pairs
   * partly filled shares that round's k-blocks evenly over all pairs; the
   * partial sums of a shared tile are added in a fixed order, so results do
   * not depend on timing. Calls that share it must be ordered on one stream. */
  void* sk_workspace;
  size_t sk_workspace_bytes;
} wamb_linear_args;
/* When the output tiles would leave SMs idle (small M), wamb_linear splits K
 * across the CTAs of a thread-block cluster: their fp32 partials meet in the
 * cluster's shared memory and are summed in split order, so the result does
 * not depend on timing and no workspace is needed. */

WAMB_API int wamb_linear(const wamb_linear_args* args, void* stream);
/* Bytes of wamb_linear_args.sk_workspace on the current device. */
WAMB_API size_t wamb_linear_sk_bytes(void);

/*
 * Row-wise E4M3 quantization (no counterpart in the reference):
 *   amax[r]  = max(max_c |x[r, c]|, 1e-20)
 *   scale[r] = amax[r] / 448
 *   out[r,c] = e4m3(x[r, c] * (448 / amax[r]))  (round to nearest even, saturating)
 * x is [m, ldx] bf16, or fp32 when x_is_f32; out is [m, ldo] bytes.
 * Gives the per-token activation scales of the FP8 path and, applied to a
 * weight [N, K], its per-output-channel scales. Requires k % 8 == 0, ldx and
 * ldo multiples of 16 bytes / 8 elements, 16-byte aligned pointers.
 */
WAMB_API int wamb_quantize_rows(const void* x, int64_t ldx, int32_t x_is_f32, int32_t m, int32_t k,
                                void* out, int64_t ldo, float* scale, void* stream);

/*
 * Flash attention (non-causal, head_dim 128) on the tcgen05 tensor cores.
 * Replaces the reference's FA2 `sdpa(q, k, v, scale)`
 * (算子研究/wam_ops/optimized/csrc/attention.cu:121-181) and the pack + SDPA
 * pair of its KV path (baseline/csrc/block.cu:213-224, 228-260): keys are read
 * in place from up to two sources.
 *   Query row r of batch row b is q[(b*q_rows + r)*ldq + q_col + h*128 + d].
 *   Source 0: batch row b reads rows src0_batch_stride * s(b) + [tile rows],
 *     s(b) = src0_map[b] if src0_map, 0 if src0_broadcast, else b; the
 *     tiles are `tiles` (int32 pairs (first row, length <= 128), count in
 *     device memory at *n_tiles) or, when tiles is NULL, [0, src0_len) in
 *     128-row pieces. K at column k0_col + h*128 of k0, V likewise of v0.
 *   Source 1 (optional, k1 != NULL): the q_rows own rows b*q_rows + [0, q_rows)
 *     of k1 / v1 (candidate verification: history + private suffix).
 * Output: out[(b*q_rows + r)*ldo + h*128 + d], bf16.
 */
typedef struct wamb_attention_args {
  int32_t batch, heads, q_rows;
  const void* q; int64_t ldq; int64_t q_total_rows; int32_t q_col;
  const void* k0; const void* v0; int64_t ld0; int64_t src0_total_rows;
  int32_t k0_col, v0_col;
  int32_t src0_batch_stride;
  const int64_t* src0_map;
  int32_t src0_broadcast;
  const int32_t* tiles; const int32_t* n_tiles;
  int32_t src0_len;
  const void* k1; const void* v1; int64_t ld1; int32_t k1_col, v1_col;
  void* out; int64_t ldo;
  /* Optional split-key scratch (NULL: none) of
   * wamb_attention_split_bytes(args) bytes, 256-byte aligned and zero-filled
   * before its first use (the library leaves its counters zero after every
   * call). With it, when the (query tile pair, head, batch row) items alone
   * would leave SMs idle, their keys are shared out: for queries longer
   * than 128 rows and kv_splits 0 or 1, key tiles are cut evenly over one
   * CTA per SM (stream-K); otherwise each item's keys are split over
   * kv_splits CTAs (0: chosen by the library, 1: never). The CTA that
   * completes an item merges its partial softmax results in key order
   * (results do not depend on timing). Not used with candidate rows
   * (src0_map). Calls sharing it must be ordered on one stream. */
  void* split_workspace;
  size_t split_workspace_bytes;
  int32_t kv_splits;
} wamb_attention_args;

WAMB_API int wamb_attention(const wamb_attention_args* args, void* stream);
/* Bytes of split_workspace that this call shape needs (0: it never splits). */
WAMB_API size_t wamb_attention_split_bytes(const wamb_attention_args* args);

/*
 * One Wan-DiT transformer block forward (WanTransformerBlock.forward,
 * 投机采样/wam-p0-worktree/wan_va/modules/model.py:741-794, with
 * WanAttention.forward :595-691 and the "original" KV cache :547-593).
 * Replaces the reference's native entry
 *   forward(weights[27], x, context, temb, freq, cache[5], candidate_rows,
 *           update, eps[7], debug, ...)
 * of 算子研究/wam_ops/baseline/csrc/block.cu:262-311 and
 * 算子研究/wam_ops/optimized/csrc/whole_layer.cu:1080-1229.
 *
 * weights[27] follow the reference order (baseline/native.py:31-46):
 *  0 scale_shift_table [1,6,D] fp32 | 1,2 norm2 gamma,beta [D] fp32 (NULL: norm2 is Identity)
 *  3..10 self to_q W,b / to_k W,b / to_v W,b / to_out W,b (W [D,D] bf16, b [D] bf16)
 *  11,12 self norm_q / norm_k gamma [D] bf16
 *  13..20 cross to_q / to_k / to_v / to_out (W,b) | 21,22 cross norm_q / norm_k gamma
 *  23,24 ffn proj W [F,D], b [F] | 25,26 ffn out W [D,F], b [D]     (all bf16)
 * eps[7]: norm1, norm2, norm3, self q, self k, cross q, cross k.
 *
 * Self KV cache (optional; cache_k NULL = no cache): the reference schema
 * k, v [pool_batch, pool, H, 128] bf16, id [pool] int64, mask/is_pred [pool]
 * bool (1 byte). update 0/1/2 as update_cache; the cache is mutated in place
 * exactly as the reference does (new rows written, ids/is_pred set, mask set
 * and, for update 0, restored). candidate_rows [batch] int64 selects the
 * read-only candidate-verification path (update must be 0).
 *
 * Cross K/V: either cross_k/cross_v precomputed ([context_batch, C, D] bf16,
 * from wamb_cross_kv), or computed per call from `context`. context_rows
 * ([batch] int64, optional) maps each batch row to its context row;
 * otherwise context_batch must be batch or 1.
 *
 * Numerics: fp32 math everywhere except the tensor-core operands; the
 * residual stream (after self- and cross-attention) stays fp32 inside the
 * block, so only the GEMM / attention operands and the output are rounded to
 * bf16 (the reference also rounds the two intermediate residuals).
 *
 * Scratch: `workspace` of wamb_block_workspace_bytes() bytes (caller-owned,
 * 256-byte aligned); intermediates stay there after the call (debug taps).
 */
typedef struct wamb_block_args {
  int32_t batch, tokens, dim, heads, ffn_dim;
  int32_t context_tokens, context_batch;
  const void* weights[27];
  double eps[7];
  const void* x;                 /* [batch, tokens, dim] bf16, or fp32 when x_is_f32 */
  int32_t x_is_f32, out_is_f32;  /* fp32 residual stream in/out (30-layer stacks) */
  const void* context;           /* [context_batch, context_tokens, dim] bf16 or NULL */
  const void* cross_k;           /* [context_batch, context_tokens, dim] bf16 or NULL */
  const void* cross_v;
  const int64_t* context_rows;   /* [batch] or NULL */
  const void* temb;              /* [batch, temb_len, 6, dim] */
  int32_t temb_len, temb_is_f32;
  const float* freq;             /* complex64 as float pairs [freq_batch, tokens, 64, 2] or NULL */
  int32_t freq_batch;
  void* cache_k; void* cache_v;
  int64_t* cache_id; uint8_t* cache_mask; uint8_t* cache_pred;
  int32_t pool, pool_batch;
  const int64_t* candidate_rows; /* [batch] or NULL */
  int32_t update;
  void* out;                     /* [batch, tokens, dim] bf16, or fp32 when out_is_f32 */
  void* workspace; size_t workspace_bytes;
  /* FP8-E4M3 weight path (no counterpart in the reference). fp8 = 1 runs the
   * eight GEMMs of the step (self q/k/v/out, cross q/out, FFN proj/out) on
   * w8[i] ([N, K] E4M3, i in 3, 5, 7, 9, 13, 19, 23, 25) with the
   * per-output-channel scales w8_scale[i] (fp32 [N], from
   * wamb_quantize_rows), and E4M3 activations with per-token scales, written
   * by the producing LayerNorm (LN1, LN2, LN3) or by a row-quantize pass
   * (self/cross attention output, GELU output). weights[] must still hold the
   * bf16 tensors (biases, norms, and the cross K/V projections 15/17 stay
   * bf16). */
  int32_t fp8;
  const void* w8[27];
  const float* w8_scale[27];
  /* chained = 1 declares that the work just before this call on `stream` is
   * a wamb_block_forward (or _noalloc) call with the same batch, tokens,
   * dims, context shape, cache presence and fp8 mode, i.e. the previous
   * layer of a stack: the KV bookkeeping kernel (cache only) then starts
   * beside that call's last GEMM instead of after it. chained = 0 (the
   * default) makes it wait for all earlier work on the stream first, which
   * is required when that work may have written this layer's cache
   * metadata or used a workspace of another layout. */
  int32_t chained;
} wamb_block_args;

/* Named intermediates kept in the workspace (byte offsets; -1 = absent).
 * The workspace must be zero-filled before its first use (cudaMemset once
 * at allocation): its first bytes hold the stream-K flags of the two-CTA
 * GEMMs, which every call leaves zero again. Calls of any shape may share
 * one workspace. After a call that recorded a device error, zero it again. */
enum wamb_tap {
  WAMB_TAP_MODULATED1 = 0,  /* [M, D]   LN1 + modulation */
  WAMB_TAP_QKV = 1,         /* [M, 3D]  q | k | v (q,k after RMS + RoPE unless in the pool) */
  WAMB_TAP_SELF_ATTN = 2,   /* [M, D] */
  WAMB_TAP_RESIDUAL1 = 3,   /* [M, D] fp32 (the residual stream stays fp32 inside the block) */
  WAMB_TAP_NORM2 = 4,       /* [M, D] */
  WAMB_TAP_CROSS_Q = 5,     /* [M, D]   after RMS */
  WAMB_TAP_CROSS_K = 6,     /* [Bc*C, D] after RMS (computed per call only) */
  WAMB_TAP_CROSS_V = 7,
  WAMB_TAP_CROSS_ATTN = 8,  /* [M, D] */
  WAMB_TAP_RESIDUAL2 = 9,   /* [M, D] fp32 */
  WAMB_TAP_MODULATED3 = 10, /* [M, D] */
  WAMB_TAP_GELU = 11,       /* [M, F] */
  WAMB_TAP_KV_SLOTS = 12,   /* [tokens] int32 pool slot of each new token */
  WAMB_TAP_KV_TILES = 13,   /* [pool] int32 pairs */
  WAMB_TAP_KV_COUNTS = 14,  /* [2] int32: tiles, visible slots */
  WAMB_TAP_A8 = 15,         /* fp8 only: [M, F] E4M3, the last quantized GEMM input */
  WAMB_TAP_A8_SCALE = 16,   /* fp8 only: [M] fp32 per-row scales of WAMB_TAP_A8 */
  WAMB_TAP_SK_FLAGS = 17,   /* zero region at offset 0 of every layout: stream-K flags of the
                               two-CTA GEMMs, then split-key counters of the self attention */
  WAMB_TAP_SK_PART = 18,    /* stream-K fp32 partials (M >= 512 only) */
  WAMB_TAP_ATTN_PART = 19,  /* partials of the self attention when its items do not fill whole waves */
  WAMB_TAP_COUNT = 20
};

WAMB_API size_t wamb_block_workspace_bytes(const wamb_block_args* args);
/* Fills offsets[WAMB_TAP_COUNT]; returns the workspace size. */
WAMB_API size_t wamb_block_workspace_layout(const wamb_block_args* args, int64_t* offsets);
WAMB_API int wamb_block_forward(const wamb_block_args* args, void* stream);

/*
 * wamb_block_forward without a caller-provided workspace. This entry point
 * has no counterpart in the reference. It is for callers that cannot
 * allocate device memory where they run the block: serving loops that keep
 * cudaMalloc / cudaFree off their path (both can synchronise the device and
 * stall every stream), and hosts that reach the library through a thin FFI
 * (ctypes, cgo, JNI) and own no device allocator with which to provide a
 * workspace.
 *
 * The scratch is a fixed array of WAMB_NOALLOC_SCRATCH_BYTES in device
 * memory, defined once in the library; every GPU that loads libwamb.so holds
 * it until the process exits. A call whose workspace need
 * (wamb_block_workspace_bytes) exceeds it returns WAMB_ERR_WORKSPACE and
 * launches nothing. args->workspace and args->workspace_bytes are ignored;
 * everything else is as for wamb_block_forward. The first call on a device
 * looks up the array's device address with cudaGetSymbolAddress and keeps
 * it for the life of the process: make that first call before any stream
 * capture on the device, and do not use the library across a
 * cudaDeviceReset of it (the kept address would be stale). All calls share
 * the one array and it keeps the last call's contents (nothing in it needs
 * to start at zero): calls that can overlap on the GPU, e.g. on two streams
 * without ordering, race on it; calls ordered on one stream do not, as long
 * as `chained` is set only as its comment states.
 * Allocates nothing: no cudaMalloc, no cudaFree.
 */
#define WAMB_NOALLOC_SCRATCH_BYTES (32u << 20)
WAMB_API int wamb_block_forward_noalloc(const wamb_block_args* args, void* stream);

/*
 * Cross-attention K/V of one block for a fixed context (the reference's
 * WholeLayerBlock.prepare_context(context, precompute=True),
 * 算子研究/wam_ops/optimized/whole_layer.py:41-67):
 *   k = RMSNorm(context W_k^T + b_k) * gamma_k,  v = context W_v^T + b_v.
 * weights/eps as in wamb_block_args (entries 15..18, 22 and eps[6] are read);
 * k_out, v_out: [context_batch * context_tokens, dim] bf16, two distinct
 * 16-byte aligned buffers. Two kernels: the K and V projections as one GEMM
 * launch (two weight groups, each writing its own output), then the RMSNorm
 * of K in place.
 */
WAMB_API int wamb_cross_kv(const wamb_block_args* args, void* k_out, void* v_out, void* stream);

/*
 * Glue of the whole-model forward (WanTransformer3DModel.forward,
 * 投机采样/wam-p0-worktree/wan_va/modules/model.py:1060-1116) and of the
 * flow-match scheduler step (wan_va/utils/scheduler.py:78-89), so that a
 * denoise step can run end to end on the device. All are asynchronous on
 * `stream`, allocate nothing and return 0 or a wamb_status.
 */

/* Sinusoidal timestep features, diffusers Timesteps(num_channels=dim,
 * flip_sin_to_cos=True, downscale_freq_shift=0) (model.py:213-215):
 * out[i] = [cos(t_i f), sin(t_i f)], f_k = exp(-ln(10000) k / (dim/2)).
 * t: [n] fp32, out: [n, dim] bf16, dim even. */
WAMB_API int wamb_timestep_embedding(const float* t, int32_t n, int32_t dim, void* out, void* stream);

/* out = bf16(silu(x)), x [m, ldx] bf16 or fp32 (x_is_f32), out [m, ldo]. */
WAMB_API int wamb_silu(const void* x, int64_t ldx, int32_t x_is_f32, int32_t m, int32_t n, void* out,
                       int64_t ldo, void* stream);

/* Patchify gather of the latent / action input embedding (model.py:1064-1077):
 * x [b, c, f, h, w] bf16 -> out [b, (f/p1)(h/p2)(w/p3), ldo] bf16 with column
 * (c p1 p2 p3) order and columns [c*p1*p2*p3, ldo) zero (ldo pads K to a
 * multiple of 64 for wamb_linear). p1 = p2 = p3 = 1 is the action rearrange. */
WAMB_API int wamb_embed_gather(const void* x, int32_t b, int32_t c, int32_t f, int32_t h, int32_t w,
                               int32_t p1, int32_t p2, int32_t p3, void* out, int32_t ldo, void* stream);

/* Output norm with its modulation (model.py:1099-1106): out = bf16(LN(x) *
 * (1 + table[1] + temb) + table[0] + temb), LN without affine in fp32;
 * x [m, d] bf16 or fp32, table [2, d] fp32, temb [m / rows_per_batch,
 * temb_len, d] fp32 or bf16 with temb_len 1 or rows_per_batch. */
WAMB_API int wamb_output_norm(const void* x, int32_t x_is_f32, int32_t m, int32_t d, double eps,
                              const float* table, const void* temb, int32_t temb_is_f32,
                              int32_t temb_len, int32_t rows_per_batch, void* out, void* stream);

/* out[r, 0:n_bytes] = x[r, 0:n_bytes] (strided rows, byte counts). */
WAMB_API int wamb_copy_cols(const void* x, int64_t ldx_bytes, int32_t m, int32_t n_bytes, void* out,
                            int64_t ldo_bytes, void* stream);

/* The same step with the velocity in the model's output layout:
 * sample [b, c, l] (the input layout 'b c f h w', l = f*h*w) += v[b, l, c] * dsigma. */
WAMB_API int wamb_flow_step_cl(void* sample, int32_t sample_is_f32, const void* v, int32_t v_is_f32,
                               int32_t b, int32_t c, int64_t l, float dsigma, void* stream);

/* torch.repeat_interleave over rows: out[r * repeat + k] = x[r] (row_bytes each). */
WAMB_API int wamb_repeat_rows(const void* x, int32_t rows, int32_t row_bytes, int32_t repeat, void* out,
                              void* stream);

/* Flow-match Euler step in place: sample += v * dsigma over n elements
 * (sample and v bf16 or fp32), dsigma = sigma_next - sigma. */
WAMB_API int wamb_flow_step(void* sample, int32_t sample_is_f32, const void* v, int32_t v_is_f32,
                            int64_t n, float dsigma, void* stream);

/* ------------------------------------------------------------------------
 * Speculative action decoding around the target model (the reference's K2/B2
 * loop, fastwam-base/fullcode-v1/real_speculative.py:32-109): the draft
 * predictor, the tree states, edge scores, route choice and commit. States and
 * directions are row-major [rows, n] (n = positions x action channels), bf16
 * or fp32 (io_is_f32). The element maps round as torch's ops on those dtypes.
 * ------------------------------------------------------------------------ */

/* FastWAM DirectionPredictor weights (fullcode-v1/draft.py:10-20), fp32, with
 * the reference's state_dict layout: embed [width, 2A+3], position [tokens,
 * width], TransformerEncoderLayer(width, heads, ffn, GELU, pre-norm) with
 * in_proj [3 width, width], out_proj, linear1 [ffn, width], linear2 [width,
 * ffn], norm1 / norm2, head [2A, width], and the normalization buffers.
 * Supported shape: tokens 32, width 64, heads 4, ffn 256, channels A <= 16. */
typedef struct wamb_draft_params {
  int32_t tokens, channels, width, heads, ffn;
  float ln_eps;
  const float* embed_w; const float* embed_b; const float* position;
  const float* in_proj_w; const float* in_proj_b; const float* out_proj_w; const float* out_proj_b;
  const float* linear1_w; const float* linear1_b; const float* linear2_w; const float* linear2_b;
  const float* norm1_w; const float* norm1_b; const float* norm2_w; const float* norm2_b;
  const float* head_w; const float* head_b;
  const float* feature_mean; const float* feature_std;     /* [2 tokens A + 3] */
  const float* residual_mean; const float* residual_std;   /* [tokens A] */
} wamb_draft_params;

/* DirectionPredictor.decode (draft.py:26-36) for `batch` rows: state and
 * previous [batch, tokens*A] (time-major, io dtype), scalars [batch, 3] fp32
 * -> out [batch, 2, tokens*A] (io dtype): the two candidate directions. */
WAMB_API int wamb_draft_forward(const wamb_draft_params* p, const void* state, const void* previous,
                                int32_t io_is_f32, const float* scalars, int32_t batch, void* out, void* stream);

/* Weighted L2 per tree edge k < edges (at most 16): scores[k] =
 * ||draft[draft_rows[k]] - target[target_rows[k]]|| * |scales[k]|, or with
 * scale_inside = 1 ||(draft - target) * scales[k]|| (p0_k3_b2.py:220-232).
 * The row and scale arrays are host memory; scores fp32 on the device. */
WAMB_API int wamb_spec_scores(const void* draft, const void* target, int32_t io_is_f32, int64_t n, int32_t edges,
                              const int32_t* draft_rows, const int32_t* target_rows, const float* scales,
                              int32_t scale_inside, float* scores, void* stream);

/* Route on the device, route [4] int32:
 *   mode 0: K2/B2 (real_speculative.py:13-23) over scores first[2],
 *           second[4] (2 + 2 parent + child) and threshold tau ->
 *           (depth, parent, child, 0)
 *   mode 1 / 2: K3/B2 greedy / global (p0_k3_b2.py:258-283) over first[2],
 *           second[2][2], third[2][2][2] -> (3, parent, child, grandchild) */
WAMB_API int wamb_spec_route(const float* scores, int32_t mode, double tau, int32_t* route, void* stream);

/* Tree states: out[r] = base[r / fan] + dirs[r] * delta, r < rows. */
WAMB_API int wamb_spec_expand(const void* base, const void* dirs, int32_t io_is_f32, int32_t rows, int32_t fan,
                              int64_t n, float delta, void* out, void* stream);

/* K2/B2 commit from a device route (depth, parent, child): row sel = 0,
 * 1 + parent or 3 + 2 parent + child of the packed tree [7, n] (state,
 * parents, leaves) and of the target values [7, n]:
 * state_out = tree[sel] + values[sel] * delta_depth, previous_out =
 * values[sel] (state_out may be tree row 0). */
WAMB_API int wamb_spec_commit(const int32_t* route, const void* values, const void* tree, int32_t io_is_f32,
                              int64_t n, float delta0, float delta1, float delta2, void* state_out,
                              void* previous_out, void* stream);

/* Classifier-free guidance of packed [conditional | unconditional] rows
 * (wan_va_server.py:1936-1941): out = uncond + scale * (cond - uncond) when
 * scale > 1, else cond. */
WAMB_API int wamb_cfg_combine(const void* cond, const void* uncond, int32_t io_is_f32, int64_t n, float scale,
                              void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WAMB_H */
