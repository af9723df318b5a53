// Speculative action decoding around the target model: the pieces of the
// reference's K2/B2 loop (fastwam-base/fullcode-v1/real_speculative.py:32-109)
// other than the target forward itself.
//   draft_kernel        FastWAM DirectionPredictor (fullcode-v1/draft.py:10-42),
//                       one CTA per state row: 32 positions x 64 features,
//                       fp32 on the CUDA cores (54 k parameters and ~1.8 M
//                       multiply-adds a row, far below a tensor-core tile)
//   spec_scores_kernel  weighted L2 of draft vs target direction per tree
//                       edge (real_speculative.py:75-77; p0_k3_b2.py:220-232)
//   spec_route_kernel   the K2/B2 depth-then-cost route (real_speculative.py:13-23)
//                       or the K3/B2 greedy / global route (p0_k3_b2.py:258-283)
//   spec_expand_kernel  tree states out[r] = base[r / fan] + dir[r] * delta
//   spec_commit_kernel  state and previous direction of the accepted route
//                       (real_speculative.py:82-96)
//   cfg_combine_kernel  uncond + s * (cond - uncond) (wan_va_server.py:1936-1941)
// The element maps round exactly as torch's fp32 (or bf16 opmath) ops do: no
// fused multiply-add where the reference has a separate product and sum.
#pragma once
#include "common.cuh"

namespace wamb {

constexpr int DR_T = 32, DR_E = 64, DR_H = 4, DR_HD = 16, DR_F = 256, DR_THREADS = 256;
constexpr int DR_AMAX = 16;   // action channels per position, at most
// Shared-memory row strides (floats), odd so that the 32 lanes of a warp
// (lane = position) reading one column hit 32 different banks.
constexpr int DR_XS = 37, DR_ES = 65, DR_QS = 193, DR_FS = 257, DR_AS = 33;

struct DraftSmem {
  static constexpr int XIN = 0;                        // [T][DR_XS] normalized features
  static constexpr int H = XIN + DR_T * DR_XS;         // [T][DR_ES] residual stream
  static constexpr int Y = H + DR_T * DR_ES;           // [T][DR_ES] LayerNorm output
  static constexpr int QKV = Y + DR_T * DR_ES;         // [T][DR_QS]
  static constexpr int ATT = QKV + DR_T * DR_QS;       // [H][T][DR_AS] probabilities
  static constexpr int O = ATT + DR_H * DR_T * DR_AS;  // [T][DR_ES] attention output
  static constexpr int U = QKV;                        // [T][DR_FS] FFN hidden, over QKV..O
  static constexpr int HEAD = O + DR_T * DR_ES;        // [T][DR_AS] head output
  static constexpr int FLOATS = HEAD + DR_T * DR_AS;
  static_assert(U + DR_T * DR_FS <= HEAD, "FFN hidden overlaps the head output");
  static constexpr uint32_t BYTES = FLOATS * 4;
};

struct DraftArgs {
  int A;                 // action channels per position (<= DR_AMAX)
  float eps;             // LayerNorm epsilon
  const float *embed_w, *embed_b, *position, *ln1_w, *ln1_b, *in_w, *in_b, *out_w, *out_b;
  const float *ln2_w, *ln2_b, *l1_w, *l1_b, *l2_w, *l2_b, *head_w, *head_b;
  const float *fmean, *fstd, *rmean, *rstd;
  const void* state;     // [B, T * A] bf16 or fp32
  const void* previous;  // [B, T * A]
  int io_f32;
  const float* scalars;  // [B, 3]
  void* out;             // [B, 2, T * A]
};

WAMB_DEV float ld_io(const void* p, long long i, int f32) {
  return f32 ? static_cast<const float*>(p)[i] : __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
WAMB_DEV void st_io(void* p, long long i, int f32, float v) {
  if (f32) static_cast<float*>(p)[i] = v;
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// out[t][j] (stride os) = act(in[t] . W[j] + b[j]) for the 32 positions
// t = lane, columns j = warp, warp + 8, ... W is row-major [J][K] in global
// memory (warp-broadcast reads). MODE 0: store, 1: add into out (residual),
// 2: store the exact GELU 0.5 x (1 + erf(x / sqrt 2)).
template <int MODE>
WAMB_DEV void dr_linear(const float* in, int is, int K, const float* __restrict__ W, const float* __restrict__ b,
                        int J, float* out, int os) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* x = in + lane * is;
  for (int j = warp; j < J; j += DR_THREADS / 32) {
    const float* w = W + static_cast<long long>(j) * K;
    float acc = 0.f;
#pragma unroll 8
    for (int k = 0; k < K; ++k) acc = fmaf(x[k], __ldg(w + k), acc);
    acc = __fadd_rn(acc, __ldg(b + j));
    if constexpr (MODE == 2) acc = 0.5f * acc * (1.f + erff(acc * 0.7071067811865476f));
    if constexpr (MODE == 1) out[lane * os + j] = __fadd_rn(out[lane * os + j], acc);
    else out[lane * os + j] = acc;
  }
}

// LayerNorm over the 64 features of each position (warp per position).
WAMB_DEV void dr_layernorm(const float* in, float* out, const float* g, const float* b, float eps) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t = warp; t < DR_T; t += DR_THREADS / 32) {
    const float a = in[t * DR_ES + lane], c = in[t * DR_ES + lane + 32];
    float s = a + c;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / 64.f;
    const float da = a - mean, dc = c - mean;
    float v = da * da + dc * dc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float rstd = 1.f / sqrtf(v / 64.f + eps);
    out[t * DR_ES + lane] = da * rstd * __ldg(g + lane) + __ldg(b + lane);
    out[t * DR_ES + lane + 32] = dc * rstd * __ldg(g + lane + 32) + __ldg(b + lane + 32);
  }
}

__global__ void __launch_bounds__(DR_THREADS, 1) draft_kernel(const DraftArgs a) {
  pdl_wait();
  extern __shared__ float dsm[];
  using S = DraftSmem;
  float* xin = dsm + S::XIN;
  float* h = dsm + S::H;
  float* y = dsm + S::Y;
  float* qkv = dsm + S::QKV;
  float* att = dsm + S::ATT;
  float* o = dsm + S::O;
  float* u = dsm + S::U;
  float* head = dsm + S::HEAD;
  const int b = blockIdx.x, A = a.A, IN = 2 * A + 3, NS = DR_T * A;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long row = static_cast<long long>(b) * NS;
  // Normalized features of each position: [state (A) | previous (A) | 3 scalars].
  for (int idx = threadIdx.x; idx < DR_T * IN; idx += DR_THREADS) {
    const int t = idx / IN, k = idx - t * IN;
    float raw;
    int f;
    if (k < A) {
      f = t * A + k;
      raw = ld_io(a.state, row + f, a.io_f32);
    } else if (k < 2 * A) {
      f = NS + t * A + k - A;
      raw = ld_io(a.previous, row + t * A + k - A, a.io_f32);
    } else {
      f = 2 * NS + k - 2 * A;
      raw = a.scalars[b * 3 + k - 2 * A];
    }
    xin[t * DR_XS + k] = __fdiv_rn(__fsub_rn(raw, __ldg(a.fmean + f)), __ldg(a.fstd + f));
  }
  __syncthreads();
  dr_linear<0>(xin, DR_XS, IN, a.embed_w, a.embed_b, DR_E, h, DR_ES);
  __syncthreads();
  for (int idx = threadIdx.x; idx < DR_T * DR_E; idx += DR_THREADS) {
    const int t = idx / DR_E, e = idx - t * DR_E;
    h[t * DR_ES + e] = __fadd_rn(h[t * DR_ES + e], __ldg(a.position + idx));
  }
  __syncthreads();
  // Self attention block: h += out_proj(softmax(q k^T / 4) v) of LN1(h).
  dr_layernorm(h, y, a.ln1_w, a.ln1_b, a.eps);
  __syncthreads();
  dr_linear<0>(y, DR_ES, DR_E, a.in_w, a.in_b, 3 * DR_E, qkv, DR_QS);
  __syncthreads();
  for (int r = warp; r < DR_H * DR_T; r += DR_THREADS / 32) {   // (head, query) rows; lane = key
    const int hh = r / DR_T, t = r - hh * DR_T;
    const float* q = qkv + t * DR_QS + hh * DR_HD;
    const float* k = qkv + lane * DR_QS + DR_E + hh * DR_HD;
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < DR_HD; ++d) s = fmaf(q[d], k[d], s);
    s *= 0.25f;   // 1 / sqrt(16), exact
    float m = s;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float e = expf(s - m);
    float sum = e;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    att[(hh * DR_T + t) * DR_AS + lane] = e / sum;
  }
  __syncthreads();
  for (int col = warp; col < DR_E; col += DR_THREADS / 32) {   // lane = query
    const int hh = col / DR_HD;
    const float* p = att + (hh * DR_T + lane) * DR_AS;
    float acc = 0.f;
#pragma unroll 8
    for (int key = 0; key < DR_T; ++key) acc = fmaf(p[key], qkv[key * DR_QS + 2 * DR_E + col], acc);
    o[lane * DR_ES + col] = acc;
  }
  __syncthreads();
  dr_linear<1>(o, DR_ES, DR_E, a.out_w, a.out_b, DR_E, h, DR_ES);
  __syncthreads();
  // Feed-forward block: h += linear2(gelu(linear1(LN2(h)))).
  dr_layernorm(h, y, a.ln2_w, a.ln2_b, a.eps);
  __syncthreads();
  dr_linear<2>(y, DR_ES, DR_E, a.l1_w, a.l1_b, DR_F, u, DR_FS);
  __syncthreads();
  dr_linear<1>(u, DR_FS, DR_F, a.l2_w, a.l2_b, DR_E, h, DR_ES);
  __syncthreads();
  dr_linear<0>(h, DR_ES, DR_E, a.head_w, a.head_b, 2 * A, head, DR_AS);
  __syncthreads();
  // Decode: previous + (center +/- spread) * residual_std + residual_mean.
  for (int idx = threadIdx.x; idx < NS; idx += DR_THREADS) {
    const int t = idx / A, c = idx - t * A;
    const float center = head[t * DR_AS + c], spread = head[t * DR_AS + A + c];
    const float prev = ld_io(a.previous, row + idx, a.io_f32);
    const float sd = __ldg(a.rstd + idx), mu = __ldg(a.rmean + idx);
    const long long o0 = static_cast<long long>(b) * 2 * NS + idx;
    st_io(a.out, o0, a.io_f32, __fadd_rn(__fadd_rn(prev, __fmul_rn(__fadd_rn(center, spread), sd)), mu));
    st_io(a.out, o0 + NS, a.io_f32, __fadd_rn(__fadd_rn(prev, __fmul_rn(__fsub_rn(center, spread), sd)), mu));
  }
}

// ------------------------------------------------------------ tree scoring
constexpr int SPEC_MAX_EDGES = 16;
struct SpecEdges {
  int n;
  int d[SPEC_MAX_EDGES], t[SPEC_MAX_EDGES];
  float scale[SPEC_MAX_EDGES];
  int scale_inside;
};

// One CTA per edge: sqrt(sum (draft[d] - target[t])^2) * |scale|, or with
// the scale inside the sum.
__global__ void spec_scores_kernel(const void* draft, const void* target, int io_f32, long long n, SpecEdges e,
                                   float* scores) {
  pdl_wait();
  __shared__ float red[32];
  const int k = blockIdx.x;
  const long long d0 = static_cast<long long>(e.d[k]) * n, t0 = static_cast<long long>(e.t[k]) * n;
  const float sc = e.scale[k];
  float s = 0.f;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    float r = __fsub_rn(ld_io(draft, d0 + i, io_f32), ld_io(target, t0 + i, io_f32));
    if (e.scale_inside) r = __fmul_rn(r, sc);
    s = fmaf(r, r, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    const float nrm = sqrtf(t);
    scores[k] = e.scale_inside ? nrm : __fmul_rn(nrm, fabsf(sc));
  }
}

// Route from the scores, on one thread (comparisons and sums in double, as
// the reference compares Python floats).
//   mode 0  K2/B2: scores = first[2], second[4] (index 2 + 2p + c); route =
//           (depth, parent, child, 0), the deepest route whose edges stay
//           within tau, then the lowest a + b, then the lowest (p, c)
//   mode 1  K3/B2 greedy, 2 global: scores = first[2], second[2][2],
//           third[2][2][2]; route = (3, parent, child, grandchild)
__global__ void spec_route_kernel(const float* scores, int mode, double tau, int* route) {
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (mode == 0) {
    int bd = -1, bp = 0, bc = 0;
    double bcost = 0.0;
    for (int p = 0; p < 2; ++p)
      for (int c = 0; c < 2; ++c) {
        const double x = scores[p], y = scores[2 + 2 * p + c];
        const int depth = x > tau ? 0 : (y > tau ? 1 : 2);
        const double cost = x + y;
        if (depth > bd || (depth == bd && cost < bcost)) {   // (p, c) ascend: first wins ties
          bd = depth;
          bcost = cost;
          bp = p;
          bc = c;
        }
      }
    route[0] = bd;
    route[1] = bp;
    route[2] = bc;
    route[3] = 0;
    return;
  }
  const float* f = scores;
  const float* s = scores + 2;   // [p][c]
  const float* t = scores + 6;   // [p][c][g]
  int p = 0, c = 0, g = 0;
  if (mode == 1) {
    p = static_cast<double>(f[1]) < static_cast<double>(f[0]) ? 1 : 0;
    c = static_cast<double>(s[2 * p + 1]) < static_cast<double>(s[2 * p]) ? 1 : 0;
    g = static_cast<double>(t[4 * p + 2 * c + 1]) < static_cast<double>(t[4 * p + 2 * c]) ? 1 : 0;
  } else {
    double best = 0.0;
    bool first = true;
    for (int pp = 0; pp < 2; ++pp)
      for (int cc = 0; cc < 2; ++cc)
        for (int gg = 0; gg < 2; ++gg) {
          const double cost = static_cast<double>(f[pp]) + static_cast<double>(s[2 * pp + cc]) +
                              static_cast<double>(t[4 * pp + 2 * cc + gg]);
          if (first || cost < best) {
            first = false;
            best = cost;
            p = pp;
            c = cc;
            g = gg;
          }
        }
  }
  route[0] = 3;
  route[1] = p;
  route[2] = c;
  route[3] = g;
}

// out[r] = base[r / fan] + dirs[r] * delta for r < rows (n elements a row).
__global__ void spec_expand_kernel(const void* base, const void* dirs, void* out, int io_f32, int rows, int fan,
                                   long long n, float delta) {
  pdl_wait();
  const long long total = static_cast<long long>(rows) * n;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / n, i = e - r * n;
    const float x = ld_io(base, (r / fan) * n + i, io_f32);
    const float v = ld_io(dirs, e, io_f32);
    st_io(out, e, io_f32, __fadd_rn(x, __fmul_rn(v, delta)));
  }
}

// The accepted route's update: row sel = 0 (depth 0), 1 + p (depth 1) or
// 3 + 2p + c (depth 2) of the packed tree (state, parents, leaves) and of the
// target values; state_out = tree[sel] + values[sel] * delta_depth,
// previous_out = values[sel].
__global__ void spec_commit_kernel(const int* route, const void* values, const void* tree, int io_f32, long long n,
                                   float d0, float d1, float d2, void* state_out, void* previous_out) {
  pdl_wait();
  // The route comes from device memory: clamp it to the tree (rows 0..6).
  const int depth = min(max(route[0], 0), 2), p = route[1] & 1, c = route[2] & 1;
  const int sel = depth <= 0 ? 0 : (depth == 1 ? 1 + p : 3 + 2 * p + c);
  const float delta = depth <= 0 ? d0 : (depth == 1 ? d1 : d2);
  const long long r0 = static_cast<long long>(sel) * n;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = ld_io(values, r0 + i, io_f32);
    const float x = ld_io(tree, r0 + i, io_f32);
    st_io(state_out, i, io_f32, __fadd_rn(x, __fmul_rn(v, delta)));
    st_io(previous_out, i, io_f32, v);
  }
}

// CFG: uncond + s * (cond - uncond) for s > 1, else cond; bf16 tensors round
// after each op (torch's bf16 elementwise ops with fp32 opmath).
__global__ void cfg_combine_kernel(const void* cond, const void* uncond, void* out, int io_f32, long long n,
                                   float scale) {
  pdl_wait();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float c = ld_io(cond, i, io_f32);
    if (!(scale > 1.f)) {
      st_io(out, i, io_f32, c);
      continue;
    }
    const float u = ld_io(uncond, i, io_f32);
    float d = __fsub_rn(c, u);
    if (!io_f32) d = __bfloat162float(__float2bfloat16_rn(d));
    float m = __fmul_rn(scale, d);
    if (!io_f32) m = __bfloat162float(__float2bfloat16_rn(m));
    st_io(out, i, io_f32, __fadd_rn(u, m));
  }
}

}  // namespace wamb
