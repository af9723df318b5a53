// Persistent tcgen05 GEMM for the block's dense projections:
//   out[M, N] = epilogue( A[M, K] * W[N, K]^T + bias[N] )
// A and W are bf16 row-major (K contiguous), or E4M3 with a per-row scale
// for A and a per-output-channel scale for W; accumulation is fp32 in TMEM.
//
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producer (A tile 128 rows x 128 bytes, W tile BN rows x
//               128 bytes, 128B swizzle: 64 bf16 or 128 E4M3 of K)
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: tcgen05.ld -> bias / GELU / residual / gate -> bf16 or fp32 stores;
//               two warps per TMEM lane quarter, each on half of the tile's columns
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the MMAs of tile i+1.
//
// Small M (cluster split-K, CL = true): when the output tiles alone would
// leave SMs idle, each tile is computed by a cluster of `splits` CTAs, one
// per K range. A split's fp32 partial goes from TMEM into its own shared
// memory (over the drained TMA ring); after a cluster barrier each CTA sums
// one row band of the tile over all splits' shared memory (DSMEM, split
// order) and runs the epilogue on it. Wider tiles and all SMs streaming
// weights matter at small M: an SM's TMA ring ingests ~90 GB/s, and every
// k-block of a 64-column tile spends two thirds of that on re-reading A.
//
// The output columns may be split into up to three groups that each read a
// different weight tensor (the separate to_q / to_k / to_v Linear weights of
// the reference, model.py:318-320), so no concatenated weight copy is needed.
#pragma once
#include "common.cuh"

namespace wamb {

enum GemmEpilogue : int {
  EPI_BIAS = 0,      // bf16(acc + b)
  EPI_GELU = 1,      // bf16(gelu_tanh(acc + b))                 FFN1, model.py:733-735
  EPI_RES = 2,       // bf16(res + (acc + b))                    cross-attn residual, model.py:783
  EPI_RES_GATE = 3,  // bf16(res + (acc + b) * (table + temb))   gated residuals, model.py:771,792
  EPI_SILU = 4,      // silu(acc + b)                            TimestepEmbedding linear_1 (diffusers)
};

struct GemmParams {
  int M, N, K;
  int n_per_group;                   // columns per weight group (N = groups * n_per_group)
  const __nv_bfloat16* bias[3];      // per group, may be null
  void* out;                         // [M, ldo] bf16, or fp32 when out_f32
  long long ldo;                     // output row stride (elements)
  int epi;
  const void* res;                   // residual [M, ldr] bf16, or fp32 when res_f32
  long long ldr;
  int res_f32, out_f32;
  // Gate = table[gate_idx, col] + temb[b, l, gate_idx, col]  (model.py:751-759)
  const float* table;                // [6, D] fp32
  const void* temb;                  // [B, L, 6, D] fp32 or bf16
  int temb_f32, temb_L, rows_per_batch, gate_idx, D;
  // E4M3 operands: acc * a_scale[row] * w_scale[group][col] (null for bf16)
  const float* a_scale;
  const float* w_scale[3];
  // 1: the weights were last written two or more kernels before this one
  // in the stream (the block forward), so the one-CTA kernel requests the
  // weight tiles of its first ring stages before griddepcontrol.wait; with
  // implicit triggers, that writer finished before the previous kernel began.
  int w_early;
  int trigger;   // 1: trigger the dependent grid early (a GEMM with w_early follows)
  // Cluster split-K (one-CTA kernel, small M): CTA u = tile * splits + s of
  // a cluster of `splits` CTAs sums k-blocks [s * kb_per_split,
  // (s + 1) * kb_per_split); the cluster reduces its partials through
  // shared memory (gemm_cluster_reduce). splits = 1: no split.
  int splits, kb_per_split;
  // != 0: the columns of weight group g go to out + g * out_gstride
  // (elements) at their local column, instead of column g * n_per_group of
  // one [M, ldo] output (separate K and V outputs of one launch).
  long long out_gstride;
  // 1: trigger the dependent grid right after griddepcontrol.wait (every
  // earlier grid is then complete); the block's last GEMM sets it so that
  // the next block's KV layout kernel, which waits only before exiting,
  // overlaps this GEMM's last tiles.
  int trigger_after;
  // Stream-K (two-CTA kernel, gemm2.cuh): the last sk_tiles tiles (0: none)
  // are shared evenly over all pairs by k-blocks; a tile shared by several
  // pairs is finished by the pair holding its last k-block from the other
  // pairs' fp32 partials in sk_part ([pairs][8 chunks][8 groups][256 rows][4]),
  // each announced by one flag per producing warp in sk_flags ([pairs][16],
  // zero before the launch and zero again after it).
  int sk_tiles;
  float* sk_part;
  int* sk_flags;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;          // bf16 elements per k-block (128 bytes)
constexpr int GEMM_BK8 = 128;        // E4M3 elements per k-block (128 bytes)
constexpr int GEMM_THREADS = 320;
constexpr int GEMM_EPI_WARPS = 8;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr uint32_t B_BYTES = BN * GEMM_BK * 2;
  // tcgen05.alloc takes a power of two of at least 32 columns.
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128
                                        : 2 * BN <= 256 ? 256 : 512;
  static constexpr uint32_t BAR_OFF = STAGES * (A_BYTES + B_BYTES);
  static constexpr uint32_t NBARS = 2 * STAGES + 6;
  static constexpr uint32_t TOTAL = 1024 + BAR_OFF + NBARS * 8 + 16;
  // Cluster split-K (64/128-column tiles): over the ring once the MMAs are
  // done, this split's fp32 partial [128][PART_LD] and the receive slots
  // [splits][R][PART_LD] of the other splits' rows of this CTA's band (R =
  // ceil(128 / splits); splits * R <= 133 for splits <= 8). The 4-float pad
  // keeps the row-per-thread stores free of bank conflicts.
  static constexpr uint32_t PART_LD = BN + 4;
  static constexpr uint32_t PART_BYTES = 128 * PART_LD * 4;
  static constexpr bool CL_FITS = PART_BYTES + 133 * PART_LD * 4 <= BAR_OFF;
};

WAMB_DEV float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3): the formula of the
  // reference's gelu_kernel (baseline/csrc/block.cu:119-124), evaluated as
  // x / (1 + exp(-2u)) (since 1 + tanh(u) = 2 / (1 + exp(-2u))) with one
  // ex2.approx and one approximate reciprocal: relative error ~1e-6, against
  // 2^-9 for the bf16 rounding that follows. x -> -inf gives x / inf = -0.
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float u = k0 * fmaf(k1 * x * x, x, x);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(u * -2.8853900817779268f));  // -2 log2(e) u
  return __fdividef(x, 1.f + e);
}

// x * sigmoid(x) = x / (1 + exp(-x)): one ex2.approx and one approximate
// reciprocal (relative error ~1e-6); x -> -inf gives x / inf = -0.
WAMB_DEV float silu(float x) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  return __fdividef(x, 1.f + e);
}

// Per-row context of the epilogue (the calling thread's output row).
struct EpiRow {
  bool valid;
  int g, n_local0;
  long long out_adj;                 // added to row * ldo + col (out_gstride)
  const __nv_bfloat16* bias;
  const float* wscale;
  float ascale;
  const float* gate_tab;
  const float* gate_f32;
  const __nv_bfloat16* gate_bf;
};

WAMB_DEV EpiRow epi_row(const GemmParams& p, int row, int n0) {
  EpiRow e;
  e.valid = row < p.M;
  e.g = n0 / p.n_per_group;
  e.n_local0 = n0 - e.g * p.n_per_group;
  e.out_adj = p.out_gstride != 0 ? e.g * (p.out_gstride - p.n_per_group) : 0;
  e.bias = e.g == 0 ? p.bias[0] : (e.g == 1 ? p.bias[1] : p.bias[2]);
  e.wscale = e.g == 0 ? p.w_scale[0] : (e.g == 1 ? p.w_scale[1] : p.w_scale[2]);
  e.ascale = p.a_scale != nullptr && e.valid ? __ldg(p.a_scale + row) : 1.f;
  e.gate_tab = nullptr;
  e.gate_f32 = nullptr;
  e.gate_bf = nullptr;
  if (p.epi == EPI_RES_GATE && e.valid) {
    const int b = row / p.rows_per_batch, tok = row - b * p.rows_per_batch;
    const long long l = p.temb_L == 1 ? 0 : tok;
    const long long off = ((static_cast<long long>(b) * p.temb_L + l) * 6 + p.gate_idx) * p.D;
    e.gate_tab = p.table + static_cast<long long>(p.gate_idx) * p.D;
    if (p.temb_f32) e.gate_f32 = static_cast<const float*>(p.temb) + off;
    else e.gate_bf = static_cast<const __nv_bfloat16*>(p.temb) + off;
  }
  return e;
}

// Raw residual words of W columns starting at `col` (W/4 x 128 bits for
// fp32, W/8 for bf16).
template <int W>
WAMB_DEV void epi_fetch_res(const GemmParams& p, int row, int col, uint4 (&r)[W / 4]) {
  if (p.res_f32) {
    const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const float*>(p.res) + row * p.ldr + col);
#pragma unroll
    for (int j = 0; j < W / 4; ++j) r[j] = __ldg(rp + j);
  } else {
    const uint4* rp =
        reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.res) + row * p.ldr + col);
#pragma unroll
    for (int j = 0; j < W / 8; ++j) r[j] = __ldg(rp + j);
  }
}

// W consecutive accumulator values v of the row at output column `col`
// (column `lcol` of the weight group) -> E4M3 scales, bias, then GELU /
// SiLU or the gate of EPI_RES_GATE: everything before the residual add.
template <int W>
WAMB_DEV void epi_value(const GemmParams& p, const EpiRow& e, float (&v)[W], int col, int lcol) {
  if (p.a_scale != nullptr) {
    const float4* sp = reinterpret_cast<const float4*>(e.wscale + lcol);
#pragma unroll
    for (int j = 0; j < W / 4; ++j) {
      const float4 w = __ldg(sp + j);
      v[4 * j] *= e.ascale * w.x;
      v[4 * j + 1] *= e.ascale * w.y;
      v[4 * j + 2] *= e.ascale * w.z;
      v[4 * j + 3] *= e.ascale * w.w;
    }
  }
  if (e.bias != nullptr) {
    const uint4* bp = reinterpret_cast<const uint4*>(e.bias + lcol);
#pragma unroll
    for (int j = 0; j < W / 8; ++j) {
      const uint4 w = __ldg(bp + j);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16(ws[h]);
        v[8 * j + 2 * h] += f.x;
        v[8 * j + 2 * h + 1] += f.y;
      }
    }
  }
  if (p.epi == EPI_GELU) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = gelu_tanh(v[j]);
  } else if (p.epi == EPI_SILU) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = silu(v[j]);
  } else if (p.epi == EPI_RES || p.epi == EPI_RES_GATE) {
    if (p.epi == EPI_RES_GATE) {
#pragma unroll
      for (int j = 0; j < W; j += 4) {
        const float4 tb = __ldg(reinterpret_cast<const float4*>(e.gate_tab + col + j));
        float4 te;
        if (e.gate_f32 != nullptr) {
          te = __ldg(reinterpret_cast<const float4*>(e.gate_f32 + col + j));
        } else {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(e.gate_bf + col + j));
          const float2 a = unpack_bf16(w.x), b2 = unpack_bf16(w.y);
          te = make_float4(a.x, a.y, b2.x, b2.y);
        }
        v[j] *= tb.x + te.x;
        v[j + 1] *= tb.y + te.y;
        v[j + 2] *= tb.z + te.z;
        v[j + 3] *= tb.w + te.w;
      }
    }
  }
}

// W consecutive accumulator values v of the row at output column `col`
// (column `lcol` of the weight group): epi_value, then the residual of the
// residual epilogues (raw words `res`), then bf16 or fp32 stores.
template <int W>
WAMB_DEV void epi_apply(const GemmParams& p, const EpiRow& e, float (&v)[W], int row, int col, int lcol,
                        const uint4 (&res)[W / 4]) {
  epi_value<W>(p, e, v, col, lcol);
  if (p.epi == EPI_RES || p.epi == EPI_RES_GATE) {
    if (p.res_f32) {
#pragma unroll
      for (int j = 0; j < W / 4; ++j) {
        v[4 * j] += __uint_as_float(res[j].x);
        v[4 * j + 1] += __uint_as_float(res[j].y);
        v[4 * j + 2] += __uint_as_float(res[j].z);
        v[4 * j + 3] += __uint_as_float(res[j].w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < W / 8; ++j) {
        const uint32_t ws[4] = {res[j].x, res[j].y, res[j].z, res[j].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = unpack_bf16(ws[h]);
          v[8 * j + 2 * h] += f.x;
          v[8 * j + 2 * h + 1] += f.y;
        }
      }
    }
  }
  if (p.out_f32) {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row * p.ldo + col + e.out_adj);
#pragma unroll
    for (int j = 0; j < W / 4; ++j) op[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint4* op = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + row * p.ldo + col + e.out_adj);
#pragma unroll
    for (int j = 0; j < W / 8; ++j) {
      uint4 w;
      w.x = pack_bf16(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
      op[j] = w;
    }
  }
}

// One 32-column chunk c of the tile starting at output column n0.
WAMB_DEV void epi_chunk(const GemmParams& p, const EpiRow& e, float (&v)[32], int row, int n0, int c,
                        const uint4 (&res)[8]) {
  epi_apply<32>(p, e, v, row, n0 + c * 32, e.n_local0 + c * 32, res);
}

// Epilogue of one output tile for the calling thread's row: 32-column
// chunks [c0, c1) of the fp32 accumulator at TMEM address `taddr` (this
// warp's lane quarter, column 0 of the tile). Every lane must call it
// (tcgen05.ld is warp-collective); rows >= M only skip the stores.
WAMB_DEV void gemm_epilogue_tile(const GemmParams& p, uint32_t taddr, int row, int n0, int c0,
                                 int c1) {
  const EpiRow e = epi_row(p, row, n0);
  // Residual rows are fetched one chunk ahead, so their DRAM latency
  // overlaps the previous chunk.
  const bool has_res = e.valid && (p.epi == EPI_RES || p.epi == EPI_RES_GATE);
  uint4 rnext[8];
  if (has_res) epi_fetch_res<32>(p, row, n0 + c0 * 32, rnext);
#pragma unroll 1
  for (int c = c0; c < c1; ++c) {
    uint4 rcur[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) rcur[j] = rnext[j];
    if (has_res && c + 1 < c1) epi_fetch_res<32>(p, row, n0 + (c + 1) * 32, rnext);
    float v[32];
    tmem_ld32(taddr + c * 32, v);
    tmem_wait_ld();
    if (!e.valid) continue;
    epi_chunk(p, e, v, row, n0, c, rcur);
  }
}

// Epilogue of one output tile through a per-warp staging buffer (32 rows x
// 32 fp32, 4 KB, 16-byte groups XOR-swizzled by row so that both the
// row-per-lane and the row-major accesses are free of bank conflicts), for
// the residual and fp32-output epilogues: the residual reads and the output
// stores become row-major warp accesses (4 rows x 128 contiguous bytes per
// instruction) instead of 32 rows x 16 bytes. `row0` is the warp's first
// row (lane l holds row row0 + l of the accumulator); residual words are
// requested one chunk ahead and kept raw until they are staged.
WAMB_DEV void sts4(uint32_t a, float4 x) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x.x), "f"(x.y), "f"(x.z), "f"(x.w)
               : "memory");
}
WAMB_DEV float4 lds4(uint32_t a) {
  float4 x;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w) : "r"(a)
               : "memory");
  return x;
}

// NC (3 or 4) 32-column chunks [c0, c0 + NC) of one tile. The residual of chunks
// c0 and c0 + 1 is requested before `wait_acc` (the wait for the
// accumulator: the residual does not depend on it), and each later chunk's
// two chunks ahead, so its DRAM latency overlaps the accumulator wait and
// two chunks of work. Residual loads and output stores carry the streaming
// cache hint (ld/st .cs: evict first), so the streamed rows do not push the
// mainloop's A and weight tiles out of L2. Returns false if wait_acc gave up.
template <int NC, class WaitAcc>
WAMB_DEV bool gemm_epilogue_tile_staged(const GemmParams& p, uint32_t taddr, int row0, int lane, int n0,
                                        int c0, uint32_t st, WaitAcc&& wait_acc) {
  const int row = row0 + lane;
  const EpiRow e = epi_row(p, row, n0);
  const bool has_res = p.epi == EPI_RES || p.epi == EPI_RES_GATE;
  const int rs = lane >> 3, f = lane & 7;   // row-major role: rows i*4 + rs, 16-byte group f
  // Staging byte offsets: row r, group g at r * 128 + ((g ^ (r & 7)) * 16).
  // Row-major role: rows i*4 + rs have r & 7 = rs + 4 (i & 1).
  const uint32_t rm_even = st + rs * 128 + ((f ^ rs) << 4);
  const uint32_t rm_odd = st + rs * 128 + ((f ^ (rs + 4)) << 4);
  const uint32_t own = st + lane * 128;
  auto rm = [&](int i) { return ((i & 1) ? rm_odd : rm_even) + i * 512; };
  auto own_at = [&](int j) { return own + ((j ^ (lane & 7)) << 4); };
  uint4 ra[8], rb[8];
  auto fetch = [&](int c, uint4 (&r8)[8]) {
    const int col = n0 + c * 32 + f * 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = row0 + i * 4 + rs;
      if (r >= p.M) {
        r8[i] = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      if (p.res_f32) {
        r8[i] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const float*>(p.res) + r * p.ldr + col));
      } else {
        const uint2 w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.res) + r * p.ldr + col));
        r8[i].x = w.x;
        r8[i].y = w.y;
      }
    }
  };
  if (has_res) {
    fetch(c0, ra);
    fetch(c0 + 1, rb);
  }
  if (!wait_acc()) return false;
  static_assert(NC >= 2, "the residual of two chunks is requested ahead");
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = c0 + k;
    uint4 (&rc)[8] = (k & 1) ? rb : ra;
    if (has_res) {
      // This chunk's residual into the staging buffer, then the request of
      // the chunk two ahead into the freed registers.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 x;
        if (p.res_f32) {
          x = make_float4(__uint_as_float(rc[i].x), __uint_as_float(rc[i].y), __uint_as_float(rc[i].z),
                          __uint_as_float(rc[i].w));
        } else {
          const float2 a = unpack_bf16(rc[i].x), b = unpack_bf16(rc[i].y);
          x = make_float4(a.x, a.y, b.x, b.y);
        }
        sts4(rm(i), x);
      }
      if (k + 2 < NC) fetch(c + 2, rc);
    }
    float v[32];
    tmem_ld32(taddr + c * 32, v);
    tmem_wait_ld();
    if (e.valid) epi_value<32>(p, e, v, n0 + c * 32, e.n_local0 + c * 32);
    if (has_res) {
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = lds4(own_at(j));
        v[4 * j] += x.x;
        v[4 * j + 1] += x.y;
        v[4 * j + 2] += x.z;
        v[4 * j + 3] += x.w;
      }
      __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) sts4(own_at(j), make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
    __syncwarp();
    const long long col = n0 + c * 32 + f * 4 + e.out_adj;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = row0 + i * 4 + rs;
      if (r >= p.M) continue;
      const float4 x = lds4(rm(i));
      if (p.out_f32) {
        __stcs(reinterpret_cast<float4*>(static_cast<float*>(p.out) + r * p.ldo + col), x);
      } else {
        uint2 w;
        w.x = pack_bf16(x.x, x.y);
        w.y = pack_bf16(x.z, x.w);
        __stcs(reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + r * p.ldo + col), w);
      }
    }
    __syncwarp();
  }
  return true;
}

// Cluster split-K, step 1, for one warp slice (rows q*32.., chunks
// [c0, c1)): this split's fp32 accumulator rows from TMEM into its local
// partial, then made visible to the bulk-copy (async) proxy.
template <int BN>
WAMB_DEV void gemm_part_to_smem(uint32_t taddr, float* part, int row_in_tile, int c0, int c1) {
  constexpr int LD = BN + 4;
#pragma unroll 1
  for (int c = c0; c < c1; ++c) {
    float v[32];
    tmem_ld32(taddr + c * 32, v);
    tmem_wait_ld();
    float4* dst = reinterpret_cast<float4*>(part + row_in_tile * LD + c * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  fence_proxy_async();
}

// Epilogue operands of 8 consecutive output columns of one row, requested
// ahead of the accumulator values (epi_load8: loads only, nothing that waits
// for them) and applied in epi_apply's order (epi_finish8).
struct EpiOps8 {
  uint4 bias;        // 8 bf16 (has_bias)
  float4 w[2];       // w_scale (E4M3 operands)
  float ascale;
  float4 tab[2];     // gate table row (EPI_RES_GATE)
  float4 tef[2];     // fp32 temb gate row, or
  uint4 teb;         // bf16 temb gate row
  uint4 res[2];      // raw residual words
  long long out_adj; // EpiRow::out_adj
  bool has_bias;
};

WAMB_DEV void epi_load8(const GemmParams& p, const EpiRow& e, int row, int col, int lcol, EpiOps8& o) {
  o.has_bias = e.bias != nullptr;
  o.out_adj = e.out_adj;
  if (o.has_bias) o.bias = __ldg(reinterpret_cast<const uint4*>(e.bias + lcol));
  o.ascale = e.ascale;
  if (p.a_scale != nullptr) {
    const float4* sp = reinterpret_cast<const float4*>(e.wscale + lcol);
    o.w[0] = __ldg(sp);
    o.w[1] = __ldg(sp + 1);
  }
  if (p.epi == EPI_RES_GATE) {
    o.tab[0] = __ldg(reinterpret_cast<const float4*>(e.gate_tab + col));
    o.tab[1] = __ldg(reinterpret_cast<const float4*>(e.gate_tab + col + 4));
    if (e.gate_f32 != nullptr) {
      o.tef[0] = __ldg(reinterpret_cast<const float4*>(e.gate_f32 + col));
      o.tef[1] = __ldg(reinterpret_cast<const float4*>(e.gate_f32 + col + 4));
    } else {
      o.teb = __ldg(reinterpret_cast<const uint4*>(e.gate_bf + col));
    }
  }
  if (p.epi == EPI_RES || p.epi == EPI_RES_GATE) epi_fetch_res<8>(p, row, col, o.res);
}

WAMB_DEV void epi_finish8(const GemmParams& p, const EpiOps8& o, float (&v)[8], int row, int col) {
  if (p.a_scale != nullptr) {
    const float ws[8] = {o.w[0].x, o.w[0].y, o.w[0].z, o.w[0].w, o.w[1].x, o.w[1].y, o.w[1].z, o.w[1].w};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= o.ascale * ws[j];
  }
  if (o.has_bias) {
    const uint32_t ws[4] = {o.bias.x, o.bias.y, o.bias.z, o.bias.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = unpack_bf16(ws[h]);
      v[2 * h] += f.x;
      v[2 * h + 1] += f.y;
    }
  }
  if (p.epi == EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = gelu_tanh(v[j]);
  } else if (p.epi == EPI_SILU) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = silu(v[j]);
  } else if (p.epi == EPI_RES || p.epi == EPI_RES_GATE) {
    if (p.epi == EPI_RES_GATE) {
      const float tb[8] = {o.tab[0].x, o.tab[0].y, o.tab[0].z, o.tab[0].w,
                           o.tab[1].x, o.tab[1].y, o.tab[1].z, o.tab[1].w};
      float te[8];
      if (p.temb_f32) {
        te[0] = o.tef[0].x; te[1] = o.tef[0].y; te[2] = o.tef[0].z; te[3] = o.tef[0].w;
        te[4] = o.tef[1].x; te[5] = o.tef[1].y; te[6] = o.tef[1].z; te[7] = o.tef[1].w;
      } else {
        const uint32_t ws[4] = {o.teb.x, o.teb.y, o.teb.z, o.teb.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = unpack_bf16(ws[h]);
          te[2 * h] = f.x;
          te[2 * h + 1] = f.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= tb[j] + te[j];
    }
    if (p.res_f32) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        v[4 * j] += __uint_as_float(o.res[j].x);
        v[4 * j + 1] += __uint_as_float(o.res[j].y);
        v[4 * j + 2] += __uint_as_float(o.res[j].z);
        v[4 * j + 3] += __uint_as_float(o.res[j].w);
      }
    } else {
      const uint32_t ws[4] = {o.res[0].x, o.res[0].y, o.res[0].z, o.res[0].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16(ws[h]);
        v[2 * h] += f.x;
        v[2 * h + 1] += f.y;
      }
    }
  }
  if (p.out_f32) {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row * p.ldo + col + o.out_adj);
    op[0] = make_float4(v[0], v[1], v[2], v[3]);
    op[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 w;
    w.x = pack_bf16(v[0], v[1]);
    w.y = pack_bf16(v[2], v[3]);
    w.z = pack_bf16(v[4], v[5]);
    w.w = pack_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + row * p.ldo + col + o.out_adj) = w;
  }
}

// Cluster split-K, step 3, for the epilogue threads, once the other
// splits' rows of this CTA's band [rank * R, rank * R + R) arrived in its
// receive slots (recv_bar): each thread takes 8-column groups of the band,
// requests the group's epilogue operands, sums the splits in split order
// (its own from the local partial; the result does not depend on timing)
// and runs the epilogue. The next group's operands are requested before the
// current group is summed.
template <int BN>
WAMB_DEV void gemm_cluster_reduce(const GemmParams& p, const float* part, const float* recv, uint32_t recv_bar,
                                  volatile int* abort_flag, int rank, int m_blk, int n0, int etid,
                                  int nthreads) {
  constexpr int LD = BN + 4;
  constexpr int G = BN / 8;   // 8-column groups per row
  const int splits = p.splits;
  const int R = (128 + splits - 1) / splits;
  const int r0 = rank * R, r1 = min(128, r0 + R);
  const int items = (r1 - r0) * G;
  EpiOps8 nxt;
  auto prefetch = [&](int it) {
    const int rr = r0 + it / G, g = it - (it / G) * G;
    const int row = m_blk * GEMM_BM + rr;
    if (row < p.M) {
      const EpiRow e = epi_row(p, row, n0);
      epi_load8(p, e, row, n0 + g * 8, e.n_local0 + g * 8, nxt);
    }
  };
  if (etid < items) prefetch(etid);
  mbar_wait(recv_bar, 0, abort_flag);   // bounded; on abort the sums are garbage
  for (int it = etid; it < items; it += nthreads) {
    const int rr = r0 + it / G, g = it - (it / G) * G;
    const int row = m_blk * GEMM_BM + rr;
    const EpiOps8 cur = nxt;
    if (it + nthreads < items) prefetch(it + nthreads);
    if (row >= p.M) continue;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      if (s2 < splits) {
        const float* src = s2 == rank ? part + rr * LD + g * 8 : recv + (s2 * R + rr - r0) * LD + g * 8;
        const float4 lo = *reinterpret_cast<const float4*>(src);
        const float4 hi = *reinterpret_cast<const float4*>(src + 4);
        v[0] += lo.x; v[1] += lo.y; v[2] += lo.z; v[3] += lo.w;
        v[4] += hi.x; v[5] += hi.y; v[6] += hi.z; v[7] += hi.w;
      }
    }
    epi_finish8(p, cur, v, row, n0 + g * 8);
  }
}

template <int BN, int STAGES, bool F8, bool CL>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                   const GemmParams p) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * STAGES;
  const uint32_t tfull0 = empty0 + 8 * STAGES;
  const uint32_t tempty0 = tfull0 + 16;
  const uint32_t drain = tempty0 + 16;
  const uint32_t recv_bar = drain + 8;   // cluster split-K: the band's incoming rows
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = p.N / BN;
  const int num_tiles = num_m * num_n;
  constexpr int KB = F8 ? GEMM_BK8 : GEMM_BK;
  const int num_kb = p.K / KB;
  const int splits = CL && p.splits > 1 ? p.splits : 1;
  const int num_units = num_tiles * splits;   // unit u: tile u / splits, split u % splits
  auto unit_kb = [&](int u, int& kb0, int& kb1) {
    if (splits == 1) { kb0 = 0; kb1 = num_kb; return; }
    kb0 = (u % splits) * p.kb_per_split;
    kb1 = min(num_kb, kb0 + p.kb_per_split);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, GEMM_EPI_WARPS);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_init(recv_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB0);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool cl_ok = false;   // cluster split-K: this thread saw the accumulator complete
  // Weight tile source of unit u: tensor map and first row.
  auto unit_b = [&](int u, const CUtensorMap*& mb, int& n_local) {
    const int n0 = (u / splits / num_m) * BN;
    const int g = n0 / p.n_per_group;
    n_local = n0 - g * p.n_per_group;
    mb = g == 0 ? &tmB0 : (g == 1 ? &tmB1 : &tmB2);
  };
  // Early weight loads: the first ring stages of this CTA's first unit (the
  // stages are free, so no empty wait); their A halves follow the wait.
  int pre = 0;
  if (p.w_early && warp == 0 && lane == 0 && static_cast<int>(blockIdx.x) < num_units) {
    const CUtensorMap* mb;
    int n_local, kb0, kb1;
    unit_b(blockIdx.x, mb, n_local);
    unit_kb(blockIdx.x, kb0, kb1);
    pre = min(STAGES, kb1 - kb0);
    for (int s = 0; s < pre; ++s) {
      mbar_arrive_expect_tx(full0 + 8 * s, L::A_BYTES + L::B_BYTES);
      tma_load_2d(smem_u32(sB + s * L::B_BYTES), mb, full0 + 8 * s, (kb0 + s) * KB, n_local);
    }
  }
  if (p.trigger) pdl_trigger();
  pdl_wait();   // inputs of the previous kernel are complete from here on
  if (p.trigger_after) pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      int it = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const int m_blk = (u / splits) % num_m;
        const CUtensorMap* mb;
        int n_local;
        unit_b(u, mb, n_local);
        int kb0, kb1;
        unit_kb(u, kb0, kb1);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (it < pre) {   // weight half already requested
            tma_load_2d(smem_u32(sA + s * L::A_BYTES), &tmA, full0 + 8 * s, kb * KB, m_blk * GEMM_BM);
            continue;
          }
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(full0 + 8 * s, L::A_BYTES + L::B_BYTES);
          tma_load_2d(smem_u32(sA + s * L::A_BYTES), &tmA, full0 + 8 * s, kb * KB, m_blk * GEMM_BM);
          tma_load_2d(smem_u32(sB + s * L::B_BYTES), mb, full0 + 8 * s, kb * KB, n_local);
        }
        if (!ok) break;
      }
      // Teardown: wait for the last load issued into each stage to land
      // (early weight loads included when an abort stopped the loop first).
      if (it < pre) it = pre;
      for (int s = 0; s < STAGES; ++s) {
        if (it > s) {
          const int last = s + ((it - 1 - s) / STAGES) * STAGES;
          mbar_wait_teardown(full0 + 8 * s, (last / STAGES) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------------- MMA issuer
      constexpr uint32_t IDESC = F8 ? idesc_e4m3(GEMM_BM, BN) : idesc_bf16(GEMM_BM, BN, 0);
      int it = 0, tc = 0;
      for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++tc) {
        const int acc = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait(tempty0 + 8 * acc, aph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int kb0, kb1;
        unit_kb(u, kb0, kb1);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * L::A_BYTES);
          const uint32_t b_base = smem_u32(sB + s * L::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes of K per k-block
            const uint64_t ad = sw128_desc(a_base + kk * 32, 16, 1024);
            const uint64_t bd = sw128_desc(b_base + kk * 32, 16, 1024);
            const uint32_t accum = kb > kb0 || kk > 0;
            if constexpr (F8) umma_e4m3(d_tmem, ad, bd, IDESC, accum);
            else umma_bf16(d_tmem, ad, bd, IDESC, accum);
          }
          umma_commit(empty0 + 8 * s);
        }
        if (!ok) break;
        umma_commit(tfull0 + 8 * acc);
      }
      // Teardown: all MMAs issued by this thread must finish before TMEM is freed.
      umma_commit(drain);
      mbar_wait_teardown(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter accessible to this warp
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    int tc = 0;
    if constexpr (CL) {
      // One unit per CTA (accumulator 0, phase 0); the push and reduction
      // follow the role branches, where every thread takes the cluster
      // barriers whatever happened here.
      cl_ok = static_cast<int>(blockIdx.x) < num_units && mbar_wait(tfull0, 0, abort_flag);
      tc_fence_after();
    }
    for (int u = blockIdx.x; !CL && u < num_units; u += gridDim.x, ++tc) {
      const int acc = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      if (!mbar_wait(tfull0 + 8 * acc, aph, abort_flag)) break;
      tc_fence_after();
      const int t = u / splits;
      const int m_blk = t % num_m, n_blk = t / num_m;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      const int row = m_blk * GEMM_BM + row_in_tile;
      const int c0 = half * (BN / 64), c1 = (half + 1) * (BN / 64);
      gemm_epilogue_tile(p, taddr, row, n_blk * BN, c0, c1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * acc);   // accumulator free for the next unit
    }
  }

  if constexpr (CL) {
    static_assert(!CL || L::CL_FITS, "cluster split-K buffers do not fit the ring");
    // The cluster's CTAs are the splits of one tile; CTA r owns rows
    // [r * R, r * R + R). Each writes its partial locally and announces the
    // bytes its band will receive; after barrier A (every split's MMAs are
    // done and its partial written, so every ring is free) one thread sends
    // each other CTA its band by bulk copy; owners reduce; barrier C keeps
    // every CTA alive until the copies out of its partial have landed.
    float* part = reinterpret_cast<float*>(smem);
    float* recv = reinterpret_cast<float*>(smem + L::PART_BYTES);
    const int rank = static_cast<int>(cluster_rank());
    const int R = (128 + splits - 1) / splits;
    auto band_rows = [&](int r) { return max(0, min(128, r * R + R) - r * R); };
    if (warp >= 2 && __all_sync(0xffffffffu, cl_ok)) {
      const int q = warp & 3, half = (warp - 2) >> 2;
      gemm_part_to_smem<BN>(tmem_base + (static_cast<uint32_t>(q * 32) << 16), part, q * 32 + lane,
                            half * (BN / 64), (half + 1) * (BN / 64));
    }
    if (threadIdx.x == 64)
      mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((splits - 1) * band_rows(rank) * L::PART_LD * 4));
    __syncwarp();
    cluster_sync_all();   // barrier A
    if (threadIdx.x == 32) {
      for (int o = 0; o < splits; ++o) {
        if (o == rank || band_rows(o) == 0) continue;
        bulk_copy_to_peer(map_to_rank(smem_u32(recv) + static_cast<uint32_t>(rank * R * L::PART_LD * 4), o),
                          smem_u32(part) + static_cast<uint32_t>(o * R * L::PART_LD * 4),
                          static_cast<uint32_t>(band_rows(o) * L::PART_LD * 4), map_to_rank(recv_bar, o));
      }
    }
    if (warp >= 2) {
      const int t = blockIdx.x / splits;
      gemm_cluster_reduce<BN>(p, part, recv, recv_bar, abort_flag, rank, t % num_m, (t / num_m) * BN,
                              threadIdx.x - 64, GEMM_EPI_WARPS * 32);
    }
    __syncwarp();
    cluster_sync_all();   // barrier C
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace wamb
