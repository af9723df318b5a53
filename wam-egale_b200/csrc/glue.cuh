// Memory-bound glue kernels of the block (one CTA per token row, 128-bit
// vector loads, warp-shuffle reductions, fp32 math):
//   ln_kernel        LayerNorm (no affine) + adaLN modulation   model.py:761-763, 786-788
//                    LayerNorm (fp32 affine)                      model.py:775-776 (norm2)
//                    optionally written as E4M3 + per-row scale (FP8 path)
//   quant_rows_kernel per-row E4M3 quantization of a bf16 / fp32 matrix
//   rms_rope_kernel  RMSNorm across all heads (* gamma) + 3D RoPE, K/V written
//                    into the caller's KV-pool slots              model.py:609-623, 577-589
//   kv_layout_kernel slot allocation with id eviction, run-tile list of the
//                    visible KV, mask restore for update_cache=0  model.py:547-593, 667-686
#pragma once
#include "common.cuh"

namespace wamb {

// ---------------------------------------------------------------- helpers
template <int NWARPS>
WAMB_DEV float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // protect `red` from the previous use
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NWARPS; ++i) t += red[i];
  return t;
}

WAMB_DEV void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float2 t = unpack_bf16(ws[h]);
    f[2 * h] = t.x;
    f[2 * h + 1] = t.y;
  }
}
WAMB_DEV void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 w;
  w.x = pack_bf16(f[0], f[1]);
  w.y = pack_bf16(f[2], f[3]);
  w.z = pack_bf16(f[4], f[5]);
  w.w = pack_bf16(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = w;
}
WAMB_DEV void load8f(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
// Modulation row: table[idx, col..col+8] + temb[..., idx, col..col+8] (model.py:751-759).
// temb_rows: modulation rows per token in temb (6 for the blocks; 1 for the
// output norm, whose single temb row is added to both table rows, model.py:1100).
WAMB_DEV void load_mod8(const float* table, const void* temb, int temb_f32, long long temb_off,
                        int idx, int D, int col, float (&f)[8], int temb_rows = 6) {
  float t[8];
  load8f(table + static_cast<long long>(idx) * D + col, f);
  const long long o = temb_off + (temb_rows > 1 ? static_cast<long long>(idx) * D : 0) + col;
  if (temb_f32) load8f(static_cast<const float*>(temb) + o, t);
  else load8(static_cast<const __nv_bfloat16*>(temb) + o, t);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] += t[i];
}

// ------------------------------------------------------------ LayerNorm
struct LnParams {
  const void* x;          // [M, ldx] bf16, or fp32 when x_f32
  long long ldx;
  int x_f32;
  __nv_bfloat16* out;
  long long ldo;
  int M, D;
  float eps;
  int affine;             // 1: y = LN(x) * gamma + beta ; 0: y = LN(x) * (1 + scale) + shift
                          // 2: y = x (identity norm2, only the bf16 cast)
  const float* gamma;
  const float* beta;
  uint8_t* out8;          // non-null: write E4M3 [M, ldo] + out_scale[M] instead of bf16
  float* out_scale;
  const float* table;     // [6, D]
  const void* temb;       // [B, L, temb_rows, D]
  int temb_f32, temb_L, rows_per_batch, shift_idx, scale_idx;
  int temb_rows;          // 0 or 6: the blocks' 6 modulation rows; 1: the output norm
  int trigger;            // 1: trigger the dependent grid early (a GEMM follows)
};

// Rows per CTA of ln_kernel for large M: two rows share one load of the
// modulation (or gamma / beta) vectors and one pair of barriers per
// reduction (four rows measured slower at D 3072: 128 registers left two
// CTAs per SM, too few to keep loads in flight through the reductions).
// Small M (fewer CTAs than SMs at that count) runs one row per CTA, with the
// modulation loads issued before the reductions.
__host__ __device__ constexpr int ln_rows(int vpt) { return vpt <= 4 ? 2 : 1; }

template <int VPT, int R>
__global__ void ln_kernel(const LnParams p) {
  if (p.trigger) pdl_trigger();
  pdl_wait();
  __shared__ float red[32 * R];
  const int row0 = blockIdx.x * R;
  const int nthr = blockDim.x;
  const int nw = nthr >> 5;
  // All R rows are loaded up front (R * VPT * 16 B in flight per thread).
  float v[R][VPT][8];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r < p.M ? row0 + r : p.M - 1;  // tail rows: recompute the last row, no store
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const long long off = static_cast<long long>(row) * p.ldx + (i * nthr + threadIdx.x) * 8;
      if (p.x_f32) load8f(static_cast<const float*>(p.x) + off, v[r][i]);
      else load8(static_cast<const __nv_bfloat16*>(p.x) + off, v[r][i]);
    }
  }
  // Block reductions of R values at once (number of warps known only at run time).
  auto reduce = [&](float (&a)[R], bool is_max) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, a[r], o);
        a[r] = is_max ? fmaxf(a[r], t) : a[r] + t;
      }
    __syncthreads();  // protect `red` from the previous use
    if ((threadIdx.x & 31) == 0)
#pragma unroll
      for (int r = 0; r < R; ++r) red[(threadIdx.x >> 5) * R + r] = a[r];
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float t = is_max ? 0.f : 0.f;
      for (int w = 0; w < nw; ++w) t = is_max ? fmaxf(t, red[w * R + r]) : t + red[w * R + r];
      a[r] = t;
    }
  };
  // Row output: bf16, or E4M3 with the row scale amax / 448 (quant_rows_kernel rule).
  auto emit = [&]() {
    if (p.out8 == nullptr) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (row0 + r >= p.M) continue;
        __nv_bfloat16* orow = p.out + static_cast<long long>(row0 + r) * p.ldo;
#pragma unroll
        for (int i = 0; i < VPT; ++i) store8(orow + (i * nthr + threadIdx.x) * 8, v[r][i]);
      }
      return;
    }
    float am[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      am[r] = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) am[r] = fmaxf(am[r], fabsf(v[r][i][j]));
    }
    reduce(am, true);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row0 + r >= p.M) continue;
      const float amax = fmaxf(am[r], 1e-20f);
      const float inv = 448.f / amax;
      if (threadIdx.x == 0) p.out_scale[row0 + r] = amax / 448.f;
      uint8_t* orow = p.out8 + static_cast<long long>(row0 + r) * p.ldo;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = v[r][i][j] * inv;
        *reinterpret_cast<uint2*>(orow + (i * nthr + threadIdx.x) * 8) = pack_e4m3x8(t);
      }
    }
  };
  if (p.affine == 2) {
    emit();
    return;
  }
  // Per-column multiplier / offset: gamma / beta (affine), or 1 + scale /
  // shift of the row's (batch, token) modulation, reloaded only when it
  // changes between consecutive rows.
  long long key[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    key[r] = 0;
    if (p.affine == 0) {
      const int row = row0 + r < p.M ? row0 + r : p.M - 1;
      const int b = row / p.rows_per_batch, tok = row - b * p.rows_per_batch;
      const long long l = p.temb_L == 1 ? 0 : tok;
      key[r] = (static_cast<long long>(b) * p.temb_L + l) * (p.temb_rows == 1 ? 1 : 6) * p.D;
    }
  }
  auto load_mul_add = [&](int r, int col, float (&mul)[8], float (&add)[8]) {
    if (p.affine) {
      load8f(p.gamma + col, mul);
      load8f(p.beta + col, add);
    } else {
      const int tr = p.temb_rows == 1 ? 1 : 6;
      load_mod8(p.table, p.temb, p.temb_f32, key[r], p.scale_idx, p.D, col, mul, tr);
      load_mod8(p.table, p.temb, p.temb_f32, key[r], p.shift_idx, p.D, col, add, tr);
    }
  };
  // One row per CTA: fetch the row's vectors now, so that their latency
  // overlaps the two reductions.
  float mul1[R == 1 ? VPT : 1][8], add1[R == 1 ? VPT : 1][8];
  if constexpr (R == 1) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) load_mul_add(0, (i * nthr + threadIdx.x) * 8, mul1[i], add1[i]);
  }
  float mean[R], var[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    mean[r] = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) mean[r] += v[r][i][j];
  }
  reduce(mean, false);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    mean[r] /= p.D;
    var[r] = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[r][i][j] - mean[r];
        var[r] += d * d;
      }
  }
  reduce(var, false);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int col = (i * nthr + threadIdx.x) * 8;
    float mul[8], add[8];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if constexpr (R == 1) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          mul[j] = mul1[i][j];
          add[j] = add1[i][j];
        }
      } else if (r == 0 || key[r] != key[r - 1]) {
        load_mul_add(r, col, mul, add);
      }
      const float one = p.affine ? 0.f : 1.f;   // the modulation multiplies by 1 + scale
      const float rstd = rsqrtf(var[r] / p.D + p.eps);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[r][i][j] = (v[r][i][j] - mean[r]) * rstd * (mul[j] + one) + add[j];
    }
  }
  emit();
}

// Warp-per-row LayerNorm for D % 256 == 0 (the block's widths), one CTA
// of 8 warps per SM. Rows reach shared memory by bulk copies (TMA engine,
// completing on one mbarrier per slot): every warp keeps two fp32 or four
// bf16 row slots and requests the next row for a slot as soon as it has
// taken that slot's row into registers, so ~192 KB of rows per SM are in
// flight while the warps normalize. Each lane holds 8 values of each
// 256-column group of its row: both reductions are warp shuffles over
// eight independent partial sums, with no block barrier on a row's path.
// The CTA's `rpc` rows lie in one batch row of the modulation, whose
// per-column multiplier and offset (1 + scale and shift, or gamma and beta)
// are staged in shared memory once instead of every row re-reading four
// fp32 D-vectors from L2; per-token modulation (temb_L > 1) stages the
// table part and adds each row's temb. Grid: batch rows x `cpb` CTAs (the
// affine modes: one batch of M rows).
WAMB_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
WAMB_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Four consecutive temb values (fp32 or bf16) as fp32.
WAMB_DEV float4 load_temb4(const void* temb, int f32, long long off) {
  if (f32) return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(temb) + off));
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(temb) + off));
  const float2 a = unpack_bf16(w.x), b = unpack_bf16(w.y);
  return make_float4(a.x, a.y, b.x, b.y);
}
// `bytes` (a multiple of 16; both addresses 16-byte aligned) from global
// into this CTA's shared memory by the TMA engine, completing as
// transaction bytes on the mbarrier `bar`.
WAMB_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

constexpr int LNW_WARPS = 10;

// Row slots per warp: one fp32 row or three bf16 rows (120 / 180 KB of rows
// in flight per SM at D 3072). Ten warps of ~168 registers: the kernel is
// bound by each warp's instruction latency, not by DRAM, so more warps pay
// more than deeper slots (8 warps with 2 / 4 slots: LN1 28.0, LN2 23.5 us
// at M 7040; 10 warps: 24.1, 21.6 us; 12 warps with 1 / 2 slots: 24.5,
// 21.8 us).
__host__ __device__ constexpr int ln_warp_slots(int x_f32) { return x_f32 ? 1 : 3; }
constexpr int LNW_MAX_SLOTS = 4;
// Dynamic shared memory of ln_warp_kernel: multiplier and offset [2][D]
// fp32, the row slots of every warp, one mbarrier per slot, the abort flag.
__host__ __device__ constexpr size_t ln_warp_smem(int D, int x_f32) {
  return 8ull * D + static_cast<size_t>(ln_warp_slots(x_f32)) * LNW_WARPS * D * (x_f32 ? 4 : 2) +
         8ull * LNW_MAX_SLOTS * LNW_WARPS + 16;
}

template <int NV>
__global__ void __launch_bounds__(LNW_WARPS * 32, 1) ln_warp_kernel(const LnParams p, int rpc, int cpb) {
  extern __shared__ __align__(16) uint8_t ln_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.D;
  const uint32_t row_bytes = static_cast<uint32_t>(D) * (p.x_f32 ? 4 : 2);
  const int NS = ln_warp_slots(p.x_f32);
  float* smul = reinterpret_cast<float*>(ln_smem);
  float* sadd = smul + D;
  uint8_t* slots = ln_smem + 8 * D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(slots + NS * LNW_WARPS * row_bytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + LNW_MAX_SLOTS * LNW_WARPS);
  if (threadIdx.x == 0) {
    for (int i = 0; i < LNW_MAX_SLOTS * LNW_WARPS; ++i) mbar_init(smem_u32(bars + i), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (p.trigger) pdl_trigger();
  pdl_wait();
  const int rpb = p.affine ? p.M : p.rows_per_batch;
  const int b = blockIdx.x / cpb, chunk = blockIdx.x - b * cpb;
  const int r_begin = b * rpb + chunk * rpc;
  const int r_end = min(min(r_begin + rpc, (b + 1) * rpb), p.M);
  const int nk = r_end - r_begin > warp ? (r_end - r_begin - warp + LNW_WARPS - 1) / LNW_WARPS : 0;
  const uint8_t* xb = static_cast<const uint8_t*>(p.x);
  const long long x_row_bytes = p.ldx * (p.x_f32 ? 4 : 2);
  const uint32_t slot0 = smem_u32(slots + warp * NS * row_bytes);
  const uint32_t bar0 = smem_u32(bars + LNW_MAX_SLOTS * warp);
  auto request = [&](int k) {   // row k of this warp into slot k % NS (lane 0)
    const int row = r_begin + warp + k * LNW_WARPS;
    const int sl = k % NS;
    mbar_arrive_expect_tx(bar0 + 8 * sl, row_bytes);
    bulk_load(slot0 + sl * row_bytes, xb + row * x_row_bytes, row_bytes, bar0 + 8 * sl);
  };
  int issued = 0;
  if (lane == 0)
    for (; issued < NS && issued < nk; ++issued) request(issued);
  issued = __shfl_sync(0xffffffffu, issued, 0);

  const int tr = p.temb_rows == 1 ? 1 : 6;
  const int ts = tr == 1 ? 0 : p.scale_idx, th = tr == 1 ? 0 : p.shift_idx;   // temb rows of scale / shift
  const bool per_token = p.affine == 0 && p.temb_L > 1;
  if (p.affine != 2) {
    const long long toff = static_cast<long long>(b) * p.temb_L * tr * D;   // token 0 of batch row b
    for (int c = threadIdx.x * 4; c < D; c += LNW_WARPS * 32 * 4) {
      float4 m, a;
      if (p.affine == 1) {
        m = __ldg(reinterpret_cast<const float4*>(p.gamma + c));
        a = __ldg(reinterpret_cast<const float4*>(p.beta + c));
      } else {
        m = __ldg(reinterpret_cast<const float4*>(p.table + static_cast<long long>(p.scale_idx) * D + c));
        a = __ldg(reinterpret_cast<const float4*>(p.table + static_cast<long long>(p.shift_idx) * D + c));
        m.x += 1.f; m.y += 1.f; m.z += 1.f; m.w += 1.f;   // the modulation multiplies by 1 + scale
        if (!per_token) {
          const float4 tm = load_temb4(p.temb, p.temb_f32, toff + static_cast<long long>(ts) * D + c);
          const float4 ta = load_temb4(p.temb, p.temb_f32, toff + static_cast<long long>(th) * D + c);
          m.x += tm.x; m.y += tm.y; m.z += tm.z; m.w += tm.w;
          a.x += ta.x; a.y += ta.y; a.z += ta.z; a.w += ta.w;
        }
      }
      *reinterpret_cast<float4*>(smul + c) = m;
      *reinterpret_cast<float4*>(sadd + c) = a;
    }
  }
  __syncthreads();

  // Lane l holds columns [i * 256 + l * 4, +4) and [i * 256 + 128 + l * 4,
  // +4) of each 256-column group i: every warp access to a row or to the
  // staged vectors is contiguous (fp32: 512 B, bf16: 256 B), free of bank
  // conflicts.
  auto col_of = [&](int i, int h) { return i * 256 + h * 128 + lane * 4; };
  int k = 0;
  for (; k < nk; ++k) {
    const int row = r_begin + warp + k * LNW_WARPS;
    if (!mbar_wait(bar0 + 8 * (k % NS), (k / NS) & 1, abort_flag)) break;
    // The row as fp32 pairs: v[i][2h + e] holds columns col_of(i, h) + 2e,
    // + 1. The arithmetic below runs on the pairs (sm_100 f32x2), one
    // instruction per two columns, in the same order and rounding as
    // separate fp32 operations.
    uint64_t v[NV][4];
    const uint8_t* srow = slots + (warp * NS + k % NS) * row_bytes;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = col_of(i, h);
        if (p.x_f32) {
          const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(reinterpret_cast<const float*>(srow) + col);
          v[i][2 * h] = x.x;
          v[i][2 * h + 1] = x.y;
        } else {
          const uint2 x = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(srow) + col);
          const float2 a = unpack_bf16(x.x), c = unpack_bf16(x.y);
          v[i][2 * h] = f2(a.x, a.y);
          v[i][2 * h + 1] = f2(c.x, c.y);
        }
      }
    __syncwarp();
    if (issued < nk) {   // the slot is free again: request the row NS ahead
      if (lane == 0) {
        fence_proxy_async();
        request(issued);
      }
      ++issued;
    }
    if (p.affine != 2) {
      // Eight independent partial sums per lane (short dependency chains),
      // as four pairs.
      auto row_sum = [&](const uint64_t (&s2)[4]) {
        const float2 a = f2_split(s2[0]), b = f2_split(s2[1]), c = f2_split(s2[2]), d = f2_split(s2[3]);
        return warp_sum(((a.x + a.y) + (b.x + b.y)) + ((c.x + c.y) + (d.x + d.y)));
      };
      uint64_t s2[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s2[j] = fadd2(s2[j], v[i][j]);
      const float mean = row_sum(s2) / D;
      const uint64_t mean2 = f2(mean, mean);
#pragma unroll
      for (int j = 0; j < 4; ++j) s2[j] = f2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t d = fsub2(v[i][j], mean2);
          s2[j] = ffma2(d, d, s2[j]);
        }
      const float var = row_sum(s2) / D;
      const float rstd = rsqrtf(var + p.eps);
      const uint64_t rstd2 = f2(rstd, rstd);
      long long trow = 0;
      if (per_token) {
        const int tok = row - b * rpb;
        trow = (static_cast<long long>(b) * p.temb_L + tok) * tr * D;
      }
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = col_of(i, h);
          ulonglong2 m = *reinterpret_cast<const ulonglong2*>(smul + col);
          ulonglong2 a = *reinterpret_cast<const ulonglong2*>(sadd + col);
          if (per_token) {
            const float4 tm = load_temb4(p.temb, p.temb_f32, trow + static_cast<long long>(ts) * D + col);
            const float4 ta = load_temb4(p.temb, p.temb_f32, trow + static_cast<long long>(th) * D + col);
            m.x = fadd2(m.x, f2(tm.x, tm.y));
            m.y = fadd2(m.y, f2(tm.z, tm.w));
            a.x = fadd2(a.x, f2(ta.x, ta.y));
            a.y = fadd2(a.y, f2(ta.z, ta.w));
          }
          // (x - mean) * rstd * (1 + scale) + shift, or * gamma + beta
          v[i][2 * h] = ffma2(fmul2(fsub2(v[i][2 * h], mean2), rstd2), m.x, a.x);
          v[i][2 * h + 1] = ffma2(fmul2(fsub2(v[i][2 * h + 1], mean2), rstd2), m.y, a.y);
        }
    }
    if (p.out8 == nullptr) {
      __nv_bfloat16* orow = p.out + static_cast<long long>(row) * p.ldo;
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h)
        {
          const float2 x = f2_split(v[i][2 * h]), y = f2_split(v[i][2 * h + 1]);
          *reinterpret_cast<uint2*>(orow + col_of(i, h)) = make_uint2(pack_bf16(x.x, x.y), pack_bf16(y.x, y.y));
        }
    } else {
      // E4M3 with the row scale amax / 448 (the quant_rows_kernel rule).
      float am = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = f2_split(v[i][j]);
          am = fmaxf(am, fmaxf(fabsf(x.x), fabsf(x.y)));
        }
      const float amax = fmaxf(warp_max(am), 1e-20f);
      const float inv = 448.f / amax;
      if (lane == 0) p.out_scale[row] = amax / 448.f;
      uint8_t* orow = p.out8 + static_cast<long long>(row) * p.ldo;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = f2_split(v[i][j]);
          t[2 * j] = x.x * inv;
          t[2 * j + 1] = x.y * inv;
        }
        const uint2 q = pack_e4m3x8(t);   // bytes 0-3: group h = 0, bytes 4-7: h = 1
        *reinterpret_cast<uint32_t*>(orow + col_of(i, 0)) = q.x;
        *reinterpret_cast<uint32_t*>(orow + col_of(i, 1)) = q.y;
      }
    }
  }
  // After an abort, the copies still in flight must land before the CTA's
  // shared memory goes away.
  if (lane == 0)
    for (int j = k; j < issued; ++j) mbar_wait_teardown(bar0 + 8 * (j % NS), (j / NS) & 1);
}

// --------------------------------------------------- row E4M3 quantization
struct QuantParams {
  const void* x;          // [M, ldx] bf16, or fp32 when x_f32
  long long ldx;
  int x_f32;
  int M, K;
  uint8_t* out;           // [M, ldo] E4M3
  long long ldo;
  float* scale;           // [M]: amax / 448
};

// One CTA per row: amax over the row (pass 1), then E4M3(x * 448 / amax)
// (pass 2, re-reading the row from L1/L2).
__global__ void __launch_bounds__(256) quant_rows_kernel(const QuantParams p) {
  pdl_wait();
  __shared__ float red[8];
  const long long row = blockIdx.x;
  float am = 0.f;
  for (int c = threadIdx.x * 8; c < p.K; c += 256 * 8) {
    float f[8];
    if (p.x_f32) load8f(static_cast<const float*>(p.x) + row * p.ldx + c, f);
    else load8(static_cast<const __nv_bfloat16*>(p.x) + row * p.ldx + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(f[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
  __syncthreads();
  am = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) am = fmaxf(am, red[i]);
  const float amax = fmaxf(am, 1e-20f);
  const float inv = 448.f / amax;
  if (threadIdx.x == 0) p.scale[row] = amax / 448.f;
  for (int c = threadIdx.x * 8; c < p.K; c += 256 * 8) {
    float f[8];
    if (p.x_f32) load8f(static_cast<const float*>(p.x) + row * p.ldx + c, f);
    else load8(static_cast<const __nv_bfloat16*>(p.x) + row * p.ldx + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] *= inv;
    *reinterpret_cast<uint2*>(p.out + row * p.ldo + c) = pack_e4m3x8(f);
  }
}

// ------------------------------------------------------- RMSNorm + RoPE
struct RmsParams {
  __nv_bfloat16* x;        // [M, ld]: section 0 at column 0, section 1 at column D, V at 2D
  long long ld;
  int M, D, rows_per_batch;
  int sections;            // 1 or 2
  const __nv_bfloat16* gamma[2];
  float eps[2];
  const float2* freq;      // complex64 [freq_batch, rows_per_batch, 64] or null (no RoPE)
  int freq_batch;
  // Optional KV-pool destination for section 1 (K) and the V columns.
  __nv_bfloat16* pool_k;
  __nv_bfloat16* pool_v;
  long long pool;          // slots per pool batch row
  const int* slots;        // [rows_per_batch] pool slot of each new token
};

template <int VPT>
__global__ void rms_rope_kernel(const RmsParams p) {
  pdl_wait();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nthr = blockDim.x;
  const int nw = nthr >> 5;
  const int b = row / p.rows_per_batch, tok = row - b * p.rows_per_batch;
  __nv_bfloat16* xr = p.x + static_cast<long long>(row) * p.ld;
  auto reduce = [&](float a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
  };
  bool to_pool = p.pool_k != nullptr;
  long long dst_row = 0;
  if (to_pool) {
    const int slot = p.slots[tok];
    // kv_layout_kernel writes -1 when it rejected the call: skip the pool write.
    if (slot < 0 || slot >= p.pool) return;
    dst_row = static_cast<long long>(b) * p.pool + slot;
  }
  for (int s = 0; s < p.sections; ++s) {
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      load8(xr + s * p.D + (i * nthr + threadIdx.x) * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
    const float rstd = rsqrtf(reduce(ss) / p.D + (s == 0 ? p.eps[0] : p.eps[1]));
    __nv_bfloat16* dst = (s == 1 && to_pool) ? p.pool_k + dst_row * p.D : xr + s * p.D;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int col = (i * nthr + threadIdx.x) * 8;
      float g[8], y[8];
      load8((s == 0 ? p.gamma[0] : p.gamma[1]) + col, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = v[i][j] * rstd * g[j];
      if (p.freq != nullptr) {
        // Pairs (2j, 2j+1) of each 128-wide head rotate by freq[b?, tok, j]
        // (model.py:614-621, complex multiply).
        const int fb = p.freq_batch == 1 ? 0 : b;
        const float4* f = reinterpret_cast<const float4*>(
            p.freq + (static_cast<long long>(fb) * p.rows_per_batch + tok) * 64 + ((col & 127) >> 1));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4 c = f[h];  // (re0, im0, re1, im1)
          const float a0 = y[4 * h], b0 = y[4 * h + 1], a1 = y[4 * h + 2], b1 = y[4 * h + 3];
          y[4 * h] = a0 * c.x - b0 * c.y;
          y[4 * h + 1] = a0 * c.y + b0 * c.x;
          y[4 * h + 2] = a1 * c.z - b1 * c.w;
          y[4 * h + 3] = a1 * c.w + b1 * c.z;
        }
      }
      store8(dst + col, y);
    }
  }
  if (to_pool) {
    const uint4* src = reinterpret_cast<const uint4*>(xr + 2 * static_cast<long long>(p.D));
    uint4* dst = reinterpret_cast<uint4*>(p.pool_v + dst_row * p.D);
    for (int i = threadIdx.x; i < p.D / 8; i += nthr) dst[i] = src[i];
  }
}

// Warp-per-row variant of rms_rope_kernel for large M (the LayerNorm's
// design): one CTA of RMSW_WARPS warps per SM, a contiguous range of rows
// per CTA, one warp per row. A row's sections (q | k, adjacent in the row,
// and the V section after them when K and V go to pool slots) arrive in a
// shared-memory slot by one bulk copy, rmsw_slots() slots per warp, so the
// next rows are in flight while one is normalized; gamma is
// staged in shared memory once per CTA. Lane l holds columns [i*256 + h*128
// + 4l, +4) of each section, so its two RoPE pairs are the same for every
// head: one float4 of the row's frequencies per lane. The same arithmetic
// as rms_rope_kernel per element (x * rstd * gamma, then the rotation);
// the sum of squares is reduced in another order.
constexpr int RMSW_WARPS = 10;
__host__ __device__ constexpr int rmsw_slots(int sections) { return sections == 2 ? 1 : 3; }
// row_sections: the sections each slot holds (sections, + 1 for V).
__host__ __device__ constexpr size_t rmsw_smem(int D, int sections, int row_sections) {
  return 4ull * sections * D + static_cast<size_t>(rmsw_slots(sections)) * RMSW_WARPS * row_sections * D * 2 +
         8ull * 3 * RMSW_WARPS + 16;
}

template <int NV>
__global__ void __launch_bounds__(RMSW_WARPS * 32, 1) rms_warp_kernel(const RmsParams p, int rpc) {
  extern __shared__ __align__(16) uint8_t rm_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.D, SEC = p.sections;
  const int NS = rmsw_slots(SEC);
  const bool to_pool = p.pool_k != nullptr;
  const uint32_t row_bytes = static_cast<uint32_t>(SEC + (to_pool ? 1 : 0)) * D * 2;
  float* sg = reinterpret_cast<float*>(rm_smem);                       // gamma [SEC][D]
  uint8_t* slots = rm_smem + 4 * SEC * D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(slots + static_cast<size_t>(NS) * RMSW_WARPS * row_bytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * RMSW_WARPS);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3 * RMSW_WARPS; ++i) mbar_init(smem_u32(bars + i), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int s2 = 0; s2 < SEC; ++s2)
    for (int c = threadIdx.x * 8; c < D; c += RMSW_WARPS * 32 * 8) {
      float g[8];
      load8((s2 == 0 ? p.gamma[0] : p.gamma[1]) + c, g);
      *reinterpret_cast<float4*>(sg + s2 * D + c) = make_float4(g[0], g[1], g[2], g[3]);
      *reinterpret_cast<float4*>(sg + s2 * D + c + 4) = make_float4(g[4], g[5], g[6], g[7]);
    }
  __syncthreads();
  pdl_wait();
  const int r_begin = blockIdx.x * rpc;
  const int r_end = min(r_begin + rpc, p.M);
  const int nk = r_end - r_begin > warp ? (r_end - r_begin - warp + RMSW_WARPS - 1) / RMSW_WARPS : 0;
  const uint32_t slot0 = smem_u32(slots + static_cast<size_t>(warp) * NS * row_bytes);
  const uint32_t bar0 = smem_u32(bars + 3 * warp);
  auto request = [&](int k) {   // row k of this warp into slot k % NS (lane 0)
    const int row = r_begin + warp + k * RMSW_WARPS;
    const int sl = k % NS;
    mbar_arrive_expect_tx(bar0 + 8 * sl, row_bytes);
    bulk_load(slot0 + sl * row_bytes, p.x + static_cast<long long>(row) * p.ld, row_bytes, bar0 + 8 * sl);
  };
  int issued = 0;
  if (lane == 0)
    for (; issued < NS && issued < nk; ++issued) request(issued);
  issued = __shfl_sync(0xffffffffu, issued, 0);
  auto col_of = [&](int i, int h) { return i * 256 + h * 128 + lane * 4; };
  int k = 0;
  for (; k < nk; ++k) {
    const int row = r_begin + warp + k * RMSW_WARPS;
    const int b = row / p.rows_per_batch, tok = row - b * p.rows_per_batch;
    if (!mbar_wait(bar0 + 8 * (k % NS), (k / NS) & 1, abort_flag)) break;
    const __nv_bfloat16* srow = reinterpret_cast<const __nv_bfloat16*>(slots + static_cast<size_t>(warp * NS + k % NS) * row_bytes);
    long long dst_row = 0;
    bool skip = false;
    if (to_pool) {
      const int slot = p.slots[tok];
      skip = slot < 0 || slot >= p.pool;   // kv_layout_kernel rejected the call: no pool write
      dst_row = static_cast<long long>(b) * p.pool + slot;
    }
    float4 fr = make_float4(1.f, 0.f, 1.f, 0.f);
    if (p.freq != nullptr && !skip) {
      const int fb = p.freq_batch == 1 ? 0 : b;
      fr = __ldg(reinterpret_cast<const float4*>(p.freq + (static_cast<long long>(fb) * p.rows_per_batch + tok) * 64) + lane);
    }
    for (int s2 = 0; s2 < SEC && !skip; ++s2) {
      float v[NV][8];
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint2 x = *reinterpret_cast<const uint2*>(srow + s2 * D + col_of(i, h));
          const float2 a = unpack_bf16(x.x), c = unpack_bf16(x.y);
          v[i][4 * h] = a.x; v[i][4 * h + 1] = a.y; v[i][4 * h + 2] = c.x; v[i][4 * h + 3] = c.y;
        }
      float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) s8[j] = fmaf(v[i][j], v[i][j], s8[j]);
      const float ss = warp_sum(((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
      const float rstd = rsqrtf(ss / D + (s2 == 0 ? p.eps[0] : p.eps[1]));
      __nv_bfloat16* dst = (s2 == 1 && to_pool) ? p.pool_k + dst_row * D
                                                : p.x + static_cast<long long>(row) * p.ld + s2 * D;
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = col_of(i, h);
          const float4 g = *reinterpret_cast<const float4*>(sg + s2 * D + col);
          float y[4] = {v[i][4 * h] * rstd * g.x, v[i][4 * h + 1] * rstd * g.y, v[i][4 * h + 2] * rstd * g.z,
                        v[i][4 * h + 3] * rstd * g.w};
          if (p.freq != nullptr) {
            // Pairs (2j, 2j+1) of each 128-wide head rotate by freq[b?, tok, j]
            // (model.py:614-621, complex multiply).
            const float a0 = y[0], b0 = y[1], a1 = y[2], b1 = y[3];
            y[0] = a0 * fr.x - b0 * fr.y;
            y[1] = a0 * fr.y + b0 * fr.x;
            y[2] = a1 * fr.z - b1 * fr.w;
            y[3] = a1 * fr.w + b1 * fr.z;
          }
          *reinterpret_cast<uint2*>(dst + col) = make_uint2(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]));
        }
    }
    if (to_pool && !skip) {
      // V from the slot into its pool row: every chunk loaded, then stored.
      const uint4* sv = reinterpret_cast<const uint4*>(srow + 2 * D);
      uint4* vdst = reinterpret_cast<uint4*>(p.pool_v + dst_row * D);
      uint4 vv[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) vv[i] = sv[lane + 32 * i];
#pragma unroll
      for (int i = 0; i < NV; ++i) vdst[lane + 32 * i] = vv[i];
    }
    __syncwarp();
    if (issued < nk) {   // the slot is free again: request the row NS ahead
      if (lane == 0) {
        fence_proxy_async();
        request(issued);
      }
      ++issued;
    }
  }
  // After an abort, the copies still in flight must land before the CTA's
  // shared memory goes away.
  if (lane == 0)
    for (int j = k; j < issued; ++j) mbar_wait_teardown(bar0 + 8 * (j % NS), (j / NS) & 1);
}

// ------------------------------------------------------------ KV layout
// One CTA of 1024 threads. The pool mask is staged in shared memory; each
// thread owns a contiguous segment of slots so that block scans follow the
// physical slot order (the order of mask.nonzero() in the reference).
constexpr int KV_THREADS = 1024;
constexpr int KV_MAX_POOL = 16384;
constexpr int KV_TILE = 128;

struct KvParams {
  uint8_t* mask;            // [pool] bool
  long long* ids;           // [pool] int64
  uint8_t* pred;            // [pool] bool
  int pool;
  int q;                    // new tokens per batch row
  int update;               // 0 / 1 / 2
  int candidate;            // read-only candidate verification
  const long long* rows;    // [batch] candidate history rows
  int batch, pool_batch;
  int* new_slots;           // [q]   out: pool slot of each new token
  int2* tiles;              // [pool] out: (first slot, length) of each visible run piece
  int* counts;              // [2]   out: number of tiles, number of visible slots
  int early;                // 1: start before griddepcontrol.wait (the caller vouches that the
                            //    previous grid is a same-layout block's last GEMM)
};

WAMB_DEV int warp_incl_scan(int v) {
  const int l = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (l >= o) v += t;
  }
  return v;
}

// Exclusive scan over the block in thread order; returns the prefix and the total.
WAMB_DEV int block_excl_scan(int v, int* sh, int* total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int inc = warp_incl_scan(v);
  __syncthreads();
  if (l == 31) sh[w] = inc;
  __syncthreads();
  if (w == 0) {
    const int s = sh[l];
    const int si = warp_incl_scan(s);
    sh[l] = si - s;
    if (l == 31) sh[32] = si;
  }
  __syncthreads();
  const int res = sh[w] + inc - v;
  *total = sh[32];
  return res;
}

WAMB_DEV long long block_min_ll(long long v, long long* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t < v ? t : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  long long r = sh[0];
  for (int i = 1; i < KV_THREADS / 32; ++i) r = sh[i] < r ? sh[i] : r;
  return r;
}
WAMB_DEV long long block_max_ll(long long v, long long* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  long long r = sh[0];
  for (int i = 1; i < KV_THREADS / 32; ++i) r = sh[i] > r ? sh[i] : r;
  return r;
}

// Nonzero bytes of a 32-bit word -> 1, zero bytes -> 0 (bit 8k of the
// shifted ORs covers bits 8k..8k+7 of x).
WAMB_DEV uint32_t bytes_nonzero(uint32_t x) {
  x |= x >> 4;
  x |= x >> 2;
  x |= x >> 1;
  return x & 0x01010101u;
}

// With p.early = 1 (a chained block call: the previous grid is the last
// GEMM of a block call with the same workspace layout) the kernel starts
// without waiting and runs beside that GEMM's last tiles: it reads only the
// cache metadata of its own layer and writes that metadata and the block's
// slot / tile scratch, whose readers in the previous call (RMS+RoPE and
// attention) precede the previous call's last GEMM, and that GEMM triggers
// its dependents only after its own griddepcontrol.wait (trigger_after);
// with the same layout the scratch lies apart from everything that GEMM
// reads or writes. Otherwise (p.early = 0) it waits first: the previous
// grid may have written this metadata, or the stream may carry another
// layout whose buffers overlap this scratch. Either way it waits before
// exiting, so its completion implies every earlier grid's (the next kernel,
// LN1, reads that GEMM's output); it triggers LN1 at once, so LN1's CTAs are
// resident and start as soon as it exits.
__global__ void __launch_bounds__(KV_THREADS, 1) kv_layout_kernel(const KvParams p) {
  pdl_trigger();
  if (!p.early) pdl_wait();
  constexpr int SEG_MAX = KV_MAX_POOL / KV_THREADS;   // slots per thread at most
  __shared__ __align__(16) uint8_t m[KV_MAX_POOL];
  __shared__ int sh[33];
  __shared__ long long shl[32];
  __shared__ int s_err;
  const int seg = (p.pool + KV_THREADS - 1) / KV_THREADS;
  const int lo = threadIdx.x * seg;
  const int hi = min(p.pool, lo + seg);
  if (threadIdx.x == 0) s_err = 0;
  // Stage the mask as 0/1 bytes, 16 per load when the base allows it (one
  // round trip for pools up to 16 K slots).
  int vec_end = 0;
  if ((reinterpret_cast<uintptr_t>(p.mask) & 15) == 0) {
    vec_end = p.pool & ~15;
    for (int i = threadIdx.x; i < (vec_end >> 4); i += KV_THREADS) {
      const uint4 w = reinterpret_cast<const uint4*>(p.mask)[i];
      reinterpret_cast<uint4*>(m)[i] =
          make_uint4(bytes_nonzero(w.x), bytes_nonzero(w.y), bytes_nonzero(w.z), bytes_nonzero(w.w));
    }
  }
  for (int i = vec_end + threadIdx.x; i < p.pool; i += KV_THREADS) m[i] = p.mask[i] ? 1 : 0;
  // This thread's slot ids, all loads in flight at once (allocation only).
  long long idr[SEG_MAX];
  if (!p.candidate) {
#pragma unroll
    for (int k = 0; k < SEG_MAX; ++k) idr[k] = lo + k < hi ? p.ids[lo + k] : -1;
  }
  __syncthreads();
  int total = 0;

  if (p.candidate) {
    for (int i = threadIdx.x; i < p.batch; i += KV_THREADS)
      if (p.rows[i] < 0 || p.rows[i] >= p.pool_batch) s_err = 3;
  } else {
    // free slots before allocation
    int nfree = 0;
    for (int i = lo; i < hi; ++i) nfree += !m[i];
    block_excl_scan(nfree, sh, &total);
    int need = p.q - total;
    // Evict the smallest ids, lowest slot first among equal ids (model.py:553-563).
    for (int iter = 0; need > 0 && iter <= p.pool; ++iter) {
      long long mn = LLONG_MAX;
#pragma unroll
      for (int k = 0; k < SEG_MAX; ++k)
        if (lo + k < hi && m[lo + k] && idr[k] < mn) mn = idr[k];
      mn = block_min_ll(mn, shl);
      if (mn == LLONG_MAX) {
        if (threadIdx.x == 0) s_err = 4;
        break;
      }
      int c = 0;
#pragma unroll
      for (int k = 0; k < SEG_MAX; ++k) c += lo + k < hi && m[lo + k] && idr[k] == mn;
      const int before = block_excl_scan(c, sh, &total);
      int r = before;
#pragma unroll
      for (int k = 0; k < SEG_MAX; ++k) {
        if (lo + k < hi && m[lo + k] && idr[k] == mn) {
          if (r < need) {
            m[lo + k] = 0;
            idr[k] = -1;
            p.ids[lo + k] = -1;
          }
          ++r;
        }
      }
      need -= total < need ? total : need;
      __syncthreads();
    }
    __syncthreads();
    if (s_err == 0) {
      // next id = max(valid ids) + 1, or 0 (model.py:565-571)
      long long mx = -1;
#pragma unroll
      for (int k = 0; k < SEG_MAX; ++k)
        if (lo + k < hi && m[lo + k] && idr[k] > mx) mx = idr[k];
      mx = block_max_ll(mx, shl);
      const long long next = mx < 0 ? 0 : mx + 1;
      // first q free slots in physical order (model.py:551, 564)
      nfree = 0;
      for (int i = lo; i < hi; ++i) nfree += !m[i];
      int r = block_excl_scan(nfree, sh, &total);
      __syncthreads();
      for (int i = lo; i < hi; ++i) {
        if (!m[i]) {
          if (r < p.q) {
            p.new_slots[r] = i;
            m[i] = 1;
            p.ids[i] = next;
            p.pred[i] = p.update == 1 ? 1 : 0;
          }
          ++r;
        }
      }
    }
  }
  __syncthreads();

  // Run-tile list: maximal runs of visible slots inside each 128-slot window.
  // A tile starts at a visible slot whose predecessor is hidden or in the
  // previous window, and ends at a visible slot whose successor is hidden or
  // in the next window; the k-th start and the k-th end (in slot order)
  // belong to tile k, so two scans pair them without walking the runs.
  {
    auto is_start = [&](int i) { return m[i] && (i % KV_TILE == 0 || !m[i - 1]); };
    auto is_end = [&](int i) { return m[i] && ((i + 1) % KV_TILE == 0 || i + 1 == p.pool || !m[i + 1]); };
    int nt = 0, ne = 0, nv = 0;
    for (int i = lo; i < hi; ++i) {
      nv += m[i];
      nt += is_start(i);
      ne += is_end(i);
    }
    int vis = 0, ntiles = 0, nends = 0;
    const int t0 = block_excl_scan(nt, sh, &ntiles);
    const int e0 = block_excl_scan(ne, sh, &nends);
    block_excl_scan(nv, sh, &vis);
    int t = t0;
    for (int i = lo; i < hi; ++i)
      if (is_start(i)) p.tiles[t++].x = i;
    __syncthreads();   // every start is written (block-scope global visibility)
    int e = e0;
    for (int i = lo; i < hi; ++i)
      if (is_end(i)) {
        p.tiles[e].y = i + 1 - p.tiles[e].x;
        ++e;
      }
    if (s_err && !p.candidate)
      for (int i = threadIdx.x; i < p.q; i += KV_THREADS) p.new_slots[i] = -1;
    if (threadIdx.x == 0) {
      p.counts[0] = s_err ? 0 : ntiles;
      p.counts[1] = s_err ? 0 : vis;
      if (s_err) record_error(s_err);
    }
  }
  __syncthreads();
  // update_cache == 0 restores the mask of the new slots (model.py:592-593, 684-686).
  if (!p.candidate && p.update == 0 && s_err == 0) {
    for (int i = threadIdx.x; i < p.q; i += KV_THREADS) m[p.new_slots[i]] = 0;
  }
  __syncthreads();
  if (!p.candidate)
    for (int i = threadIdx.x; i < p.pool; i += KV_THREADS) p.mask[i] = m[i];
  pdl_wait();
}

}  // namespace wamb
