// Glue of the whole-model forward around the block stack
// (投机采样/wam-p0-worktree/wan_va/modules/model.py:1060-1116) and of the
// flow-match scheduler step (wan_va/utils/scheduler.py:78-89):
//   timestep_embed_kernel  sinusoidal timestep features (diffusers Timesteps
//                          with flip_sin_to_cos=True, downscale_freq_shift=0,
//                          model.py:213-215)
//   silu_kernel            SiLU before the timestep projection (model.py:236)
//   embed_gather_kernel    'b c (f p1) (h p2) (w p3) -> b (f h w) (c p1 p2 p3)'
//                          (model.py:1069-1077; p = 1 gives the action
//                          rearrange of :1064-1066), zero-padded to a K the
//                          GEMM accepts
//   copy_cols_kernel       first n columns of a padded GEMM output
//   repeat_rows_kernel     torch.repeat_interleave of rows (the per-frame
//                          timestep embedding expanded to every token,
//                          model.py:1088-1092)
//   flow_step_kernel       prev = sample + v * (sigma_next - sigma)
// All are memory-bound element maps (grid-stride loops).
#pragma once
#include "common.cuh"

namespace wamb {

__global__ void timestep_embed_kernel(const float* t, int n, int dim, __nv_bfloat16* out) {
  pdl_wait();
  const int half = dim / 2;
  const long long total = static_cast<long long>(n) * half;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = e / half;
    const int i = static_cast<int>(e - row * half);
    // freq_i = exp(-ln(10000) * i / half), computed like the reference in fp32
    const float f = expf(-9.210340371976184f * static_cast<float>(i) / static_cast<float>(half));
    const float a = t[row] * f;
    out[row * dim + i] = __float2bfloat16_rn(cosf(a));
    out[row * dim + half + i] = __float2bfloat16_rn(sinf(a));
  }
}

__global__ void silu_kernel(const void* x, long long ldx, int x_f32, int m, int n, __nv_bfloat16* out,
                            long long ldo) {
  pdl_wait();
  const long long total = static_cast<long long>(m) * n;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / n;
    const int c = static_cast<int>(e - r * n);
    const float v = x_f32 ? static_cast<const float*>(x)[r * ldx + c]
                          : __bfloat162float(static_cast<const __nv_bfloat16*>(x)[r * ldx + c]);
    out[r * ldo + c] = __float2bfloat16_rn(v / (1.f + expf(-v)));
  }
}

struct GatherParams {
  const __nv_bfloat16* x;   // [B, C, F, H, W]
  int B, C, F, H, W, p1, p2, p3;
  __nv_bfloat16* out;       // [B, L, ldo], columns [C*p1*p2*p3, ldo) zeroed
  int ldo;
};

__global__ void embed_gather_kernel(const GatherParams p) {
  pdl_wait();
  const int Fn = p.F / p.p1, Hn = p.H / p.p2, Wn = p.W / p.p3;
  const long long L = static_cast<long long>(Fn) * Hn * Wn;
  const int K = p.C * p.p1 * p.p2 * p.p3;
  const long long total = p.B * L * p.ldo;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(e % p.ldo);
    const long long bl = e / p.ldo;
    const long long l = bl % L;
    const int b = static_cast<int>(bl / L);
    __nv_bfloat16 v = __float2bfloat16_rn(0.f);
    if (k < K) {
      const int a3 = k % p.p3, a2 = (k / p.p3) % p.p2, a1 = (k / (p.p3 * p.p2)) % p.p1;
      const int c = k / (p.p3 * p.p2 * p.p1);
      const int wi = static_cast<int>(l % Wn), hi = static_cast<int>((l / Wn) % Hn);
      const int fi = static_cast<int>(l / (static_cast<long long>(Wn) * Hn));
      const long long src = ((((static_cast<long long>(b) * p.C + c) * p.F + fi * p.p1 + a1) * p.H +
                              hi * p.p2 + a2) * p.W) + wi * p.p3 + a3;
      v = p.x[src];
    }
    p.out[e] = v;
  }
}

__global__ void copy_cols_kernel(const uint8_t* x, long long ldx_bytes, int m, int n_bytes, uint8_t* out,
                                 long long ldo_bytes) {
  pdl_wait();
  const long long total = static_cast<long long>(m) * n_bytes;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / n_bytes;
    const int c = static_cast<int>(e - r * n_bytes);
    out[r * ldo_bytes + c] = x[r * ldx_bytes + c];
  }
}

__global__ void repeat_rows_kernel(const uint8_t* x, int rows, int row_bytes, int repeat, uint8_t* out) {
  pdl_wait();
  const long long total = static_cast<long long>(rows) * repeat * row_bytes;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / row_bytes;
    const int c = static_cast<int>(e - r * row_bytes);
    out[e] = x[(r / repeat) * row_bytes + c];
  }
}

__global__ void flow_step_kernel(void* sample, int s_f32, const void* v, int v_f32, long long n,
                                 float dsigma) {
  pdl_wait();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float vv = v_f32 ? static_cast<const float*>(v)[i]
                           : __bfloat162float(static_cast<const __nv_bfloat16*>(v)[i]);
    if (s_f32) {
      float* s = static_cast<float*>(sample);
      s[i] = s[i] + vv * dsigma;
    } else {
      __nv_bfloat16* s = static_cast<__nv_bfloat16*>(sample);
      s[i] = __float2bfloat16_rn(__bfloat162float(s[i]) + vv * dsigma);
    }
  }
}

// The same step with the velocity in token layout: sample [B, C, L]
// (channels first, the model's input layout), v [B, L, C] (its output).
__global__ void flow_step_cl_kernel(void* sample, int s_f32, const void* v, int v_f32, int B, int C,
                                    long long L, float dsigma) {
  pdl_wait();
  const long long n = static_cast<long long>(B) * C * L;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long l = i % L;
    const long long bc = i / L;
    const int c = static_cast<int>(bc % C);
    const long long b = bc / C;
    const long long vi = (b * L + l) * C + c;
    const float vv = v_f32 ? static_cast<const float*>(v)[vi]
                           : __bfloat162float(static_cast<const __nv_bfloat16*>(v)[vi]);
    if (s_f32) {
      float* s = static_cast<float*>(sample);
      s[i] = s[i] + vv * dsigma;
    } else {
      __nv_bfloat16* s = static_cast<__nv_bfloat16*>(sample);
      s[i] = __float2bfloat16_rn(__bfloat162float(s[i]) + vv * dsigma);
    }
  }
}

// Grid for an element map of `total` items: up to 8 CTAs of 256 per SM.
inline int elem_grid(long long total, int sms) {
  long long g = (total + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 8;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace wamb
