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
  WAMB_EPI_RES_GATE = 3  /* out = bf16(res + (A W^T + b) * (table[g] + temb[b, l, g])) */
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
  void* out;              /* [M, ldo] bf16 */
  int64_t ldo;
  int32_t epilogue;       /* enum wamb_epilogue */
  const void* res;        /* [M, ldr] bf16 (RES / RES_GATE) */
  int64_t ldr;
  /* RES_GATE: gate = table[gate_index*D + col] + temb[((b*temb_len + l)*6 + gate_index)*D + col]
   * with b = row / rows_per_batch and l = 0 if temb_len == 1 else row % rows_per_batch. */
  const float* table;     /* [6, D] fp32 */
  const void* temb;       /* [B, temb_len, 6, D] fp32 (temb_is_f32) or bf16 */
  int32_t temb_is_f32;
  int32_t temb_len;
  int32_t rows_per_batch;
  int32_t gate_index;
  int32_t dim;            /* D (= N for the gated epilogue) */
} wamb_linear_args;

WAMB_API int wamb_linear(const wamb_linear_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WAMB_H */
