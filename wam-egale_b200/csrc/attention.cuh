// tcgen05 flash attention (non-causal, head_dim 128, scale 1/sqrt(128)):
//   out[b, q, h, :] = softmax(Q[b, q, h] K[b, :, h]^T / sqrt(128)) V[b, :, h]
// the reference's custom_sdpa (model.py:37-40) for self and cross attention.
//
// One CTA per (256 query rows = two 128-row tiles A and B, head, batch row);
// both tiles share every K/V tile that is loaded. 320 threads:
//   warps 0..7  softmax: warps 0-3 on tile A, warps 4-7 on tile B, both
//               tiles at the same time, one thread per query row (its TMEM
//               lane), all 128 keys of the tile, so no cross-thread
//               reduction is needed. S is read from TMEM, P written back to
//               TMEM as packed bf16 over the S columns, O rescaled in TMEM
//               only when the row max grows by more than 2^8 (the final
//               O / l uses the same stale max, so the result is exact).
//               Three quarters of the exp2s run on the MUFU (ex2.approx),
//               one quarter as a cubic on the FMA pipe with packed f32x2
//               arithmetic. Each warp signals the MMA issuer with one
//               arrival (a shared-memory barrier op per thread would queue
//               behind the tensor core's operand reads).
//   warp 8      TMA producer: Q once, then K_0, V_0, K_1, V_1, ... through
//               one 5-slot ring (the order both are consumed and released in)
//   warp 9      TMEM owner; its lane 0 issues the MMAs, in the order
//               PV_A(j), S_A(j+1), PV_B(j), S_B(j+1): while one tile's
//               softmax runs the tensor core works on the other tile.
//               S = Q K^T reads both operands from SMEM; O += P V reads P
//               from TMEM and V from SMEM as an MN-major operand.
// A CTA with a single query tile (q_rows <= 128, or the last 128 rows of a
// longer query) would leave slot B idle and lose the ping-pong, so it splits
// its keys instead: slot A takes key tiles [0, ceil(n/2)), slot B the rest,
// both against Q_A, and the epilogue merges the two partial softmaxes.
// TMEM columns: S/P of A [0,128), S/P of B [128,256), O_A [256,384), O_B [384,512).
// SMEM: Q_A, Q_B and a 5-slot K/V ring of 128 rows x 128 bf16 tiles (224 KB).
//
// Keys come from up to two sources:
//   source 0  the KV pool (or a contiguous K/V tensor), read as a list of
//             (first row, length <= 128) tiles: either a device-side tile list
//             written by kv_layout_kernel (visible pool slots, so no gather or
//             pack copy is needed) or a contiguous range;
//   source 1  the call's own K/V rows (candidate verification appends each
//             candidate's private K/V to the shared history, model.py:654-660).
// Partial tiles: S columns past the tile length are masked to -inf, V rows
// past it (up to the next multiple of 16) are zeroed before the PV MMA, and
// only ceil(len/16) K-steps are issued, so stale pool rows never contribute.
#pragma once
#include "common.cuh"

namespace wamb {

constexpr int ATT_THREADS = 320;
constexpr int ATT_PRODUCER_WARP = 8;
constexpr int ATT_MMA_WARP = 9;
constexpr uint32_t ATT_TILE_BYTES = 128 * 128 * 2;  // 128 rows x 128 bf16
constexpr uint32_t ATT_ATOM = 128 * 128;            // one 64-column half: 128 rows x 128 B
constexpr float ATT_RESCALE_LOG2 = 8.f;             // rescale O only when the max grows > 2^8
constexpr int ATT_SLOTS = 5;                        // K/V ring: load L = 2j (K_j) or 2j+1 (V_j)
// 2^f ~= C0 + f (C1 + f (C2 + f C3)) for f in [-0.5, 0.5]: minimax relative
// error 7.5e-5 (tests/test_host_exp2_cubic.py recomputes the fit), far below bf16's 2^-9 for P.
constexpr float ATT_EXP2_C0 = 0.9999281167984009f;
constexpr float ATT_EXP2_C1 = 0.6932609677314758f;
constexpr float ATT_EXP2_C2 = 0.2426108419895172f;
constexpr float ATT_EXP2_C3 = 0.05517144873738289f;

WAMB_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
WAMB_DEV float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for a pair on the FMA pipe: x clamped to >= -125, rounded to n + f with
// |f| <= 1/2 by the 1.5 * 2^23 shifter, 2^f from the cubic, n added to the
// exponent field (the shifter's bit pattern vanishes from (bits << 23)).
WAMB_DEV uint64_t ex2_poly2(uint64_t x2) {
  const float2 xv = f2_split(x2);
  const uint64_t x = f2(fmaxf(xv.x, -125.f), fmaxf(xv.y, -125.f));
  const uint64_t shifter = f2(12582912.f, 12582912.f);
  const uint64_t t = fadd2(x, shifter);
  const uint64_t f = fsub2(x, fsub2(t, shifter));
  uint64_t p = ffma2(f, f2(ATT_EXP2_C3, ATT_EXP2_C3), f2(ATT_EXP2_C2, ATT_EXP2_C2));
  p = ffma2(p, f, f2(ATT_EXP2_C1, ATT_EXP2_C1));
  p = ffma2(p, f, f2(ATT_EXP2_C0, ATT_EXP2_C0));
  const float2 pv = f2_split(p), tv = f2_split(t);
  return f2(__int_as_float(__float_as_int(pv.x) + (__float_as_int(tv.x) << 23)),
            __int_as_float(__float_as_int(pv.y) + (__float_as_int(tv.y) << 23)));
}
struct AttnParams {
  int trigger;              // 1: trigger the dependent grid early (a GEMM follows)
  int heads;
  int q_rows;               // query rows per batch row
  __nv_bfloat16* out;       // [B * q_rows, ldo], head h at columns [h*128, h*128+128)
  long long ldo;
  float scale_log2;         // log2(e) / sqrt(head_dim)
  int q_col;                // column of head 0 in the Q tensor
  // source 0
  int src0_batch_stride;    // rows between consecutive source-0 batch rows
  const long long* src0_map;  // batch row -> source-0 batch row (candidate rows), or null
  int src0_broadcast;       // 1: every batch row reads source-0 batch row 0
  const int2* tiles;        // device tile list or null
  const int* n_tiles;       // device count of `tiles`
  int src0_len;             // contiguous length when tiles == null
  int k0_col, v0_col;
  // source 1 (own rows of this call)
  int has_src1;
  int k1_col, v1_col;
  // Grouped candidates (launched as clusters of group_ctas = G x R CTAs
  // along z, G * q_rows <= 128, source-0 rows by src0_map): cluster c holds
  // batch rows [c G, c G + G) and its CTA k works for row c G + k / R. When
  // the G rows read the same source-0 row, the CTAs share one query tile
  // holding all G candidates, split the key tiles (source 0, then the G
  // candidates' own keys as one block-diagonal tile) into group_ctas
  // ranges and merge (m, l, O): CTA k owns q_rows / R rows of its
  // candidate, slice k % R.
  int group;
  int group_ctas;
  // Split keys (ungrouped kernel, kv_splits > 1, blockIdx.z = batch row x
  // kv_splits + split): when the query tiles alone would leave SMs idle,
  // each (query tile pair, head, batch row) item is computed by kv_splits
  // CTAs over consecutive key-tile ranges. Each writes its rows' partial
  // (O relative to its max m, unnormalized, and m, l) to its slot of
  // kv_part ([item][split] x ATT_PART_BYTES); the CTA that brings the item's
  // counter in kv_count (zero between launches) to kv_splits merges the
  // partials in split order, writes the output and resets the counter.
  int kv_splits;
  float* kv_part;
  int* kv_count;
  // attn_ot_kernel only (a persistent 1-D grid of G CTAs): items are (query
  // tile pair, head, batch row) with the pair fastest, ot_items of them,
  // ot_qpairs pairs per (head, batch row). Items [0, ot_dp_items) go whole
  // to CTAs round-robin; with ot_sk the key tiles of the rest are shared
  // evenly over the G CTAs (stream-K), partials in kv_part ([G][2] slots of
  // ATT_PART_FLOATS) and one counter per item in kv_count.
  int ot_items, ot_qpairs, ot_dp_items, ot_sk;
};

// One split-key partial: O [32 four-column groups][256 rows][4] fp32 (so
// that for a fixed group the threads of consecutive rows touch one
// contiguous run), then m [256] and l [256].
constexpr size_t ATT_PART_FLOATS = 256 * 128 + 2 * 256;
constexpr int ATT_MAX_SPLITS = 4;
constexpr size_t ATT_PART_BYTES = ATT_PART_FLOATS * 4;

struct AttnSmem {
  static constexpr uint32_t Q_OFF = 0;                                    // Q_A, Q_B
  static constexpr uint32_t RING_OFF = Q_OFF + 2 * ATT_TILE_BYTES;        // K/V ring
  static constexpr uint32_t BAR_OFF = RING_OFF + ATT_SLOTS * ATT_TILE_BYTES;
  // q_full, full[5], empty[5], s_full[2], p_full[2], o_done, drain, recv
  static constexpr uint32_t NBARS = 18;
  // Grouped candidates, over the ring once the MMAs are done: this CTA's
  // partial O [128][PART_LD] fp32, m [128], l [128], then one receive slot
  // per sender of q_rows x (PART_LD + 2) floats (128 rows in all).
  static constexpr uint32_t PART_LD = 132;
  static constexpr uint32_t PART_O = RING_OFF;
  static constexpr uint32_t PART_M = PART_O + 128 * PART_LD * 4;
  static constexpr uint32_t PART_L = PART_M + 128 * 4;
  static constexpr uint32_t RECV = PART_L + 128 * 4;
  static_assert(RECV + 128 * (PART_LD + 2) * 4 <= BAR_OFF, "grouped exchange does not fit the ring");
  static constexpr uint32_t TOTAL = 1024 + BAR_OFF + NBARS * 8 + 16;
  static_assert(TOTAL <= 232448, "attention shared memory exceeds 227 KB");
};

struct KvTile {
  int row;      // first row in the source tensor
  int len;      // valid rows (1..128)
  int src;      // 0 or 1
};

WAMB_DEV KvTile att_tile(const AttnParams& p, int j, int n0, int b) {
  KvTile t;
  if (j < n0) {
    int start, len;
    if (p.tiles != nullptr) {
      const int2 e = p.tiles[j];
      start = e.x;
      len = e.y;
    } else {
      start = j * 128;
      len = min(128, p.src0_len - start);
    }
    const long long srow = p.src0_map ? p.src0_map[b] : (p.src0_broadcast ? 0 : b);
    t.row = static_cast<int>(srow * p.src0_batch_stride + start);
    t.len = len;
    t.src = 0;
  } else {
    const int start = (j - n0) * 128;
    t.row = b * p.q_rows + start;
    t.len = min(128, p.q_rows - start);
    t.src = 1;
  }
  return t;
}

// Split keys: the last of an item's S CTAs to finish merges the S partials
// (in split order, so the result does not depend on timing), writes the
// bf16 output and resets the item's counter. Called by the 256 softmax
// threads (threads 0..255: thread i is row i of the item's 256 query rows)
// after each wrote its partial.
WAMB_DEV void att_split_merge(const AttnParams& p, int item, int S, int q0, int b, int h, bool has_b,
                              volatile int* abort_flag, volatile int* last_split) {
  // Split keys: the last of the item's S CTAs to finish merges the S
  // partials (split order, so the result does not depend on timing).
  __threadfence();
  asm volatile("bar.sync 2, 256;" ::: "memory");
  if (threadIdx.x == 0) *last_split = atomicAdd(p.kv_count + item, 1) == S - 1;
  asm volatile("bar.sync 2, 256;" ::: "memory");
  if (*last_split) {
    __threadfence();
    const int prow = threadIdx.x;   // 0..255
    const int qr = q0 + prow;
    const bool has_row = (has_b || prow < 128) && qr < p.q_rows;
    if (has_row) {
      const float* b0p = p.kv_part + static_cast<size_t>(item) * S * ATT_PART_FLOATS;
      float M = -INFINITY;
      for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, __ldcg(b0p + s2 * ATT_PART_FLOATS + 256 * 128 + prow));
      float w[ATT_MAX_SPLITS], den = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < ATT_MAX_SPLITS; ++s2) {
        w[s2] = 0.f;
        if (s2 < S) {
          const float* bs = b0p + s2 * ATT_PART_FLOATS;
          const float ms = __ldcg(bs + 256 * 128 + prow);
          w[s2] = ms == -INFINITY ? 0.f : exp2f(ms - M);
          den += w[s2] * __ldcg(bs + 256 * 128 + 256 + prow);
        }
      }
      const float inv = (!*abort_flag && den > 0.f) ? 1.f / den : 0.f;
      __nv_bfloat16* orow = p.out + (static_cast<long long>(b) * p.q_rows + qr) * p.ldo + h * 128;
      // Eight four-column groups of every split in flight at once (a
      // rolled loop of dependent L2 round trips cost ~20 us per item).
#pragma unroll 1
      for (int j0 = 0; j0 < 32; j0 += 8) {
        float4 v[ATT_MAX_SPLITS][8];
#pragma unroll
        for (int s2 = 0; s2 < ATT_MAX_SPLITS; ++s2)
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            v[s2][jj] = s2 < S ? __ldcg(reinterpret_cast<const float4*>(b0p + s2 * ATT_PART_FLOATS) +
                                        (j0 + jj) * 256 + prow)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int s2 = 0; s2 < ATT_MAX_SPLITS; ++s2) {
            acc.x += w[s2] * v[s2][jj].x;
            acc.y += w[s2] * v[s2][jj].y;
            acc.z += w[s2] * v[s2][jj].z;
            acc.w += w[s2] * v[s2][jj].w;
          }
          *reinterpret_cast<uint2*>(orow + 4 * (j0 + jj)) =
              make_uint2(pack_bf16(acc.x * inv, acc.y * inv), pack_bf16(acc.z * inv, acc.w * inv));
        }
      }
    }
    if (threadIdx.x == 0) p.kv_count[item] = 0;   // ready for the next launch
  }
}

// GROUPED: the grouped-candidate variant (cluster launch); false compiles
// the kernel without any of that code.
template <bool GROUPED>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                   const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                   const __grid_constant__ CUtensorMap tmV1, const AttnParams p) {
  using L = AttnSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sQ = smem_u32(smem + L::Q_OFF);
  const uint32_t sRing = smem_u32(smem + L::RING_OFF);
  const uint32_t bar0 = smem_u32(smem + L::BAR_OFF);
  const uint32_t q_full = bar0;
  const uint32_t full = bar0 + 8;         // [5] by ring slot
  const uint32_t empty = bar0 + 48;       // [5]
  const uint32_t s_full = bar0 + 88;      // [2] by query tile
  const uint32_t p_full = bar0 + 104;     // [2] by query tile
  const uint32_t o_done = bar0 + 120;
  const uint32_t drain = bar0 + 128;
  const uint32_t recv_bar = bar0 + 136;   // grouped: the other CTAs' partials of this CTA's rows
  // Ring load L (the L-th K or V tile in consumption order; K_j = 2j and
  // V_j = 2j+1 without split-KV) lives in slot L % 5, phase (L / 5) & 1.
  auto slot_addr = [&](int L) { return sRing + (L % ATT_SLOTS) * ATT_TILE_BYTES; };
  auto slot_full = [&](int L) { return full + 8 * (L % ATT_SLOTS); };
  auto slot_empty = [&](int L) { return empty + 8 * (L % ATT_SLOTS); };
  auto slot_phase = [&](int L) { return static_cast<uint32_t>((L / ATT_SLOTS) & 1); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_split = reinterpret_cast<volatile int*>(tmem_slot + 2);   // split keys: this CTA merges

  if (p.trigger) pdl_trigger();
  pdl_wait();   // the tile list and Q/K/V of the previous kernels are complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = !GROUPED && p.kv_splits > 1 ? p.kv_splits : 1;
  const int C = GROUPED && p.group_ctas > 1 ? p.group_ctas : 1;   // CTAs of a cluster
  const int G = GROUPED && p.group > 1 ? p.group : 1;             // its batch rows
  const int R = C / G;                                            // CTAs per batch row
  const int crank = GROUPED ? static_cast<int>(blockIdx.z) % C : 0;
  const int b = GROUPED ? static_cast<int>(blockIdx.z) / C * G + crank / R : static_cast<int>(blockIdx.z) / S;
  const int sidx = GROUPED ? 0 : static_cast<int>(blockIdx.z) - b * S, h = blockIdx.y;
  const int q0 = blockIdx.x * 256;
  const int item = (b * gridDim.y + h) * gridDim.x + blockIdx.x;   // split keys: the item's counter / slots
  const int n0 = p.tiles != nullptr ? *p.n_tiles : (p.src0_len + 127) / 128;
  // Grouped candidates: the cluster's G batch rows share their source-0 row
  // (checked here, so every CTA of the cluster decides alike). Otherwise
  // each row is computed alone by the first of its R CTAs; the others idle.
  const int b0 = b - b % G;
  bool grouped = GROUPED && C > 1;
  for (int i = 1; grouped && i < G; ++i) grouped = p.src0_map[b0 + i] == p.src0_map[b0];
  const bool idle = GROUPED && !grouped && crank % R != 0;
  // Key tiles of this CTA: [kv_lo, kv_lo + n) of the tile space (source 0,
  // then source 1; grouped: source 0, then the group's own-key tile n0).
  const int n_all = grouped ? n0 + 1 : n0 + (p.has_src1 ? (p.q_rows + 127) / 128 : 0);
  const int kv_lo = grouped ? crank * n_all / C : sidx * n_all / S;
  const int n = idle ? 0 : grouped ? (crank + 1) * n_all / C - kv_lo : (sidx + 1) * n_all / S - kv_lo;
  const bool has_b = !grouped && q0 + 128 < p.q_rows;   // the second query tile holds rows
  auto tile_of = [&](int j) {   // this CTA's j-th key tile
    const int jj = kv_lo + j;
    if (grouped && jj == n0) {
      KvTile t;
      t.row = b0 * p.q_rows;
      t.len = G * p.q_rows;
      t.src = 1;
      return t;
    }
    return att_tile(p, jj, n0, b);
  };
  // Split-KV: a CTA with one query tile runs its keys as two halves, [0, nA)
  // in TMEM slot A and [nA, n) in slot B (both against Q_A), so the two-slot
  // ping-pong still overlaps softmax with MMAs; the epilogue merges the halves.
  const bool split = !has_b && n >= 2;
  const int nA = split ? (n + 1) >> 1 : n;
  const int nB = split ? n - nA : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ATT_SLOTS; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + 8 * i, 1);
      mbar_init(p_full + 8 * i, 4);   // one arrival per softmax warp of the tile
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    mbar_init(recv_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == ATT_MMA_WARP) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == ATT_PRODUCER_WARP) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      const int qrow = grouped ? b0 * p.q_rows : b * p.q_rows + q0;
      const int qcol = p.q_col + h * 128;
      mbar_arrive_expect_tx(q_full, (has_b ? 2 : 1) * ATT_TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, qcol, qrow);
      tma_load_2d(sQ + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow);
      if (has_b) {
        tma_load_2d(sQ + ATT_TILE_BYTES, &tmQ, q_full, qcol, qrow + 128);
        tma_load_2d(sQ + ATT_TILE_BYTES + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow + 128);
      }
      auto src_of = [&](const KvTile& t, const CUtensorMap*& mk, const CUtensorMap*& mv, int& kc,
                        int& vc) {
        mk = t.src ? &tmK1 : &tmK0;
        mv = t.src ? &tmV1 : &tmV0;
        kc = (t.src ? p.k1_col : p.k0_col) + h * 128;
        vc = (t.src ? p.v1_col : p.v0_col) + h * 128;
      };
      int issued = 0;   // ring loads issued
      bool go = true;
      auto emit = [&](int j, bool is_v) {
        if (!go) return;
        const int L = issued;
        const KvTile t = tile_of(j);
        const CUtensorMap *mk, *mv;
        int kc, vc;
        src_of(t, mk, mv, kc, vc);
        if (!mbar_wait(slot_empty(L), slot_phase(L) ^ 1, abort_flag)) { go = false; return; }
        const CUtensorMap* m = is_v ? mv : mk;
        const int col = is_v ? vc : kc;
        mbar_arrive_expect_tx(slot_full(L), ATT_TILE_BYTES);
        tma_load_2d(slot_addr(L), m, slot_full(L), col, t.row);
        tma_load_2d(slot_addr(L) + ATT_ATOM, m, slot_full(L), col + 64, t.row);
        issued = L + 1;
      };
      if (split) {
        // K_A(0), K_B(0), then V_A(j), K_A(j+1), V_B(j), K_B(j+1): the MMA order.
        emit(0, false);
        emit(nA, false);
        for (int j = 0; j < nA; ++j) {
          emit(j, true);
          if (j + 1 < nA) emit(j + 1, false);
          if (j < nB) {
            emit(nA + j, true);
            if (j + 1 < nB) emit(nA + j + 1, false);
          }
        }
      } else {
        for (int j = 0; j < n; ++j) {
          emit(j, false);
          emit(j, true);
        }
      }
      // Teardown: loads still in flight must land before the CTA exits.
      mbar_wait_teardown(q_full, 0);
      for (int L = max(0, issued - ATT_SLOTS); L < issued; ++L)
        mbar_wait_teardown(slot_full(L), slot_phase(L));
    }
  } else if (warp == ATT_MMA_WARP) {
   if (lane == 0) {
    // ------------------------------------------------ MMA issuer (lane 0)
    constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0);
    constexpr uint32_t IDESC_O = idesc_bf16(128, 128, 1);
    const int ntq = has_b ? 2 : 1;
    // S_t = Q K^T into TMEM columns [t*128, t*128+128); Q at qb, K at ring address kb.
    auto issue_s = [&](int t, uint32_t qb, uint32_t kb) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * ATT_ATOM + (kk & 3) * 32;
        umma_bf16(tmem + t * 128, sw128_desc(qb + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                  IDESC_S, kk > 0);
      }
      umma_commit(s_full + 8 * t);
    };
    // O_t += P_t V (V at ring address vb); P_t is packed bf16 in TMEM columns [t*128, t*128+64).
    auto issue_pv = [&](int t, uint32_t vb, int ksteps, bool acc) {
      for (int kk = 0; kk < ksteps; ++kk)
        umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                     sw128_desc(vb + kk * 2048, ATT_ATOM, 1024), IDESC_O, acc || kk > 0);
    };
    // Zero V rows [len, 16*ceil(len/16)) of ring load L in both 64-column halves.
    auto zero_v_tail = [&](int L, int len) {
      if (len & 15) {
        uint8_t* vt = smem + L::RING_OFF + (L % ATT_SLOTS) * ATT_TILE_BYTES;
        const int r0 = len, r1 = ((len + 15) >> 4) * 16;
        for (int i = 0; i < (r1 - r0) * 16; ++i) {
          const int r = r0 + (i >> 4), c = i & 15;
          uint8_t* dst = vt + (c >> 3) * ATT_ATOM + r * 128 + (c & 7) * 16;
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
      }
    };
    auto wait_full = [&](int L) { return mbar_wait(slot_full(L), slot_phase(L), abort_flag); };
    bool ok = mbar_wait(q_full, 0, abort_flag);
    if (split) {
      // Loads: K_A(0) = 0, K_B(0) = 1, then V_A(j), K_A(j+1), V_B(j), K_B(j+1).
      for (int t = 0; ok && t < 2; ++t) {
        ok = wait_full(t);
        if (ok) {
          tc_fence_after();
          issue_s(t, sQ, slot_addr(t));
          umma_commit(slot_empty(t));
        }
      }
      int Lc = 2;
      for (int j = 0; ok && j < nA; ++j) {
        for (int t = 0; ok && t < 2; ++t) {
          const int nt = t ? nB : nA;
          if (j >= nt) break;
          const int len = tile_of(t ? nA + j : j).len;
          if (!wait_full(Lc)) { ok = false; break; }
          zero_v_tail(Lc, len);
          if (!mbar_wait(p_full + 8 * t, j & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, slot_addr(Lc), (len + 15) >> 4, j > 0);
          umma_commit(slot_empty(Lc));
          ++Lc;
          if (j + 1 < nt) {
            if (!wait_full(Lc)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, sQ, slot_addr(Lc));
            umma_commit(slot_empty(Lc));
            ++Lc;
          }
        }
      }
    }
    if (!split && ok && n > 0) {
      ok = wait_full(0);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < ntq; ++t) issue_s(t, sQ + t * ATT_TILE_BYTES, slot_addr(0));
        umma_commit(slot_empty(0));
      }
    }
    for (int j = 0; !split && ok && j < n; ++j) {
      const KvTile tl = tile_of(j);
      const int ksteps = (tl.len + 15) >> 4;
      if (!wait_full(2 * j + 1)) break;
      zero_v_tail(2 * j + 1, tl.len);
      const bool next = j + 1 < n;
      bool knext = false;
      for (int t = 0; t < ntq; ++t) {
        if (!mbar_wait(p_full + 8 * t, j & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        issue_pv(t, slot_addr(2 * j + 1), ksteps, j > 0);
        if (t == ntq - 1) umma_commit(slot_empty(2 * j + 1));
        if (next) {
          if (!knext) {
            if (!wait_full(2 * j + 2)) { ok = false; break; }
            tc_fence_after();
            knext = true;
          }
          issue_s(t, sQ + t * ATT_TILE_BYTES, slot_addr(2 * j + 2));
        }
      }
      if (ok && next) umma_commit(slot_empty(2 * j + 2));
    }
    umma_commit(o_done);
    umma_commit(drain);
    mbar_wait_teardown(drain, 0);
   }
    __syncwarp();
  } else {
    // -------------------------------------------------- softmax / epilogue
    const int t = warp >> 2;          // query tile of this warp
    const int wq = warp & 3;          // TMEM lane quarter
    const int r = wq * 32 + lane;     // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const bool active = t == 0 || has_b || split;
    const int nt = split ? (t ? nB : nA) : n;   // key tiles of this slot
    const int kv0 = split && t ? nA : 0;        // its first key tile
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; active && ok && j < nt; ++j) {
      // Valid key columns [lo, hi): the tile's length, or in the group's own
      // keys only the row's candidate (a row sees only its own keys).
      int lo = 0, hi = tile_of(kv0 + j).len;
      if (grouped && kv_lo + kv0 + j == n0) {
        lo = (r / p.q_rows) * p.q_rows;
        hi = min(lo + p.q_rows, hi);   // rows past the G candidates see none
      }
      if (!mbar_wait(s_full + 8 * t, j & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t32[32];
        tmem_ld32(tmem + lane_base + t * 128 + c * 32, t32);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t32[i];
      }
      tmem_wait_ld();
      if (lo > 0 || hi < 128) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i < lo || i >= hi) s[i] = -INFINITY;
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        mx0 = fmax3(mx0, s[i], s[i + 1]);
        mx1 = fmax3(mx1, s[64 + i], s[64 + i + 1]);
      }
      const float mx = fmaxf(mx0, mx1) * p.scale_log2;
      // Keep the stale max unless the new one exceeds it by more than 2^8.
      const bool grow = mx > m_used + ATT_RESCALE_LOG2;
      const float m_new = grow ? mx : m_used;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = grow ? exp2f(m_used - m_use) : 1.f;
      const uint64_t scale2 = f2(p.scale_log2, p.scale_log2);
      const uint64_t neg_m2 = f2(-m_use, -m_use);
      uint64_t sum2 = f2(0.f, 0.f);
      // Four chunks of 32 keys; in each, keys 0..23 take the MUFU exp2 and
      // keys 24..31 the cubic. P of keys [32 c, +32) -> packed TMEM columns
      // [t*128 + 16 c, +16).
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 12; ++i) {
          const int k = 32 * c + 2 * i;
          const float2 x = f2_split(ffma2(f2(s[k], s[k + 1]), scale2, neg_m2));
          const float a = ex2_mufu(x.x), bb = ex2_mufu(x.y);
          sum2 = fadd2(sum2, f2(a, bb));
          pk[i] = pack_bf16(a, bb);
        }
#pragma unroll
        for (int i = 12; i < 16; ++i) {
          const int k = 32 * c + 2 * i;
          const uint64_t e = ex2_poly2(ffma2(f2(s[k], s[k + 1]), scale2, neg_m2));
          sum2 = fadd2(sum2, e);
          const float2 ev = f2_split(e);
          pk[i] = pack_bf16(ev.x, ev.y);
        }
        tmem_st16u(tmem + lane_base + t * 128 + c * 16, pk);
      }
      const float2 sv = f2_split(sum2);
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O_t is stable: S_t(j) was issued after PV_t(j-1) and has completed.
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          const uint32_t oc = 256 + t * 128 + c * 32;
          tmem_ld32(tmem + lane_base + oc, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tmem + lane_base + oc, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + 8 * t);
      l = l * alpha + (sv.x + sv.y);
      m_used = m_new;
    }
    if (split) {
      // Merge the halves. Each slot's O and l are relative to its own stale
      // max m; the row's result is (2^(mA-M) O_A + 2^(mB-M) O_B) /
      // (2^(mA-M) lA + 2^(mB-M) lB), M = max(mA, mB). The (m, l) pairs meet
      // in the unused Q_B tile; warps of slot A store output columns [0, 64),
      // warps of slot B columns [64, 128) of the same rows.
      if (ok) ok = mbar_wait(o_done, 0, abort_flag);
      tc_fence_after();
      float* xch = reinterpret_cast<float*>(smem + L::Q_OFF + ATT_TILE_BYTES);
      xch[t * 256 + r] = m_used;
      xch[t * 256 + 128 + r] = l;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float m_o = xch[(t ^ 1) * 256 + r], l_o = xch[(t ^ 1) * 256 + 128 + r];
      const float mA = t ? m_o : m_used, lA = t ? l_o : l;
      const float mB = t ? m_used : m_o, lB = t ? l : l_o;
      const float M = fmaxf(mA, mB);
      const float aA = mA == -INFINITY ? 0.f : exp2f(mA - M);
      const float aB = mB == -INFINITY ? 0.f : exp2f(mB - M);
      const float den = aA * lA + aB * lB;
      if (grouped) {
        // This CTA's partial of the row: O relative to M, unnormalized.
        float* po = reinterpret_cast<float*>(smem + L::PART_O) + r * L::PART_LD + t * 64;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float oa[32], ob[32];
          tmem_ld32(tmem + lane_base + 256 + t * 64 + c * 32, oa);
          tmem_ld32(tmem + lane_base + 384 + t * 64 + c * 32, ob);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 8; ++k)
            reinterpret_cast<float4*>(po + c * 32)[k] =
                make_float4(oa[4 * k] * aA + ob[4 * k] * aB, oa[4 * k + 1] * aA + ob[4 * k + 1] * aB,
                            oa[4 * k + 2] * aA + ob[4 * k + 2] * aB, oa[4 * k + 3] * aA + ob[4 * k + 3] * aB);
        }
        if (t == 0) {
          reinterpret_cast<float*>(smem + L::PART_M)[r] = ok ? M : -INFINITY;
          reinterpret_cast<float*>(smem + L::PART_L)[r] = ok ? den : 0.f;
        }
      }
      if (S > 1) {
        // Split keys: this CTA's partial of the row (tile A rows only).
        float* base = p.kv_part + (static_cast<size_t>(item) * S + sidx) * ATT_PART_FLOATS;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float oa[32], ob[32];
          tmem_ld32(tmem + lane_base + 256 + t * 64 + c * 32, oa);
          tmem_ld32(tmem + lane_base + 384 + t * 64 + c * 32, ob);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int j = t * 16 + c * 8 + k;   // four-column group
            reinterpret_cast<float4*>(base)[j * 256 + r] =
                make_float4(oa[4 * k] * aA + ob[4 * k] * aB, oa[4 * k + 1] * aA + ob[4 * k + 1] * aB,
                            oa[4 * k + 2] * aA + ob[4 * k + 2] * aB, oa[4 * k + 3] * aA + ob[4 * k + 3] * aB);
          }
        }
        if (t == 0) {
          base[256 * 128 + r] = ok ? M : -INFINITY;
          base[256 * 128 + 256 + r] = ok ? den : 0.f;
        }
      }
      const float inv = (ok && !*abort_flag && den > 0.f) ? 1.f / den : 0.f;
      const float sA = aA * inv, sB = aB * inv;
      const int qr = q0 + r;
      const bool store = !grouped && S == 1 && qr < p.q_rows;
      __nv_bfloat16* orow = p.out + (static_cast<long long>(b) * p.q_rows + qr) * p.ldo + h * 128 + t * 64;
#pragma unroll 1
      for (int c = 0; !grouped && c < 2; ++c) {
        float oa[32], ob[32];
        tmem_ld32(tmem + lane_base + 256 + t * 64 + c * 32, oa);
        tmem_ld32(tmem + lane_base + 384 + t * 64 + c * 32, ob);
        tmem_wait_ld();
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = oa[8 * k + i] * sA + ob[8 * k + i] * sB;
            uint4 w;
            w.x = pack_bf16(v[0], v[1]);
            w.y = pack_bf16(v[2], v[3]);
            w.z = pack_bf16(v[4], v[5]);
            w.w = pack_bf16(v[6], v[7]);
            dst[k] = w;
          }
        }
      }
    } else if (active && grouped) {
      // One key tile (or none): this CTA's partial is slot A's O, m, l.
      if (ok && n > 0) ok = mbar_wait(o_done, 0, abort_flag);
      tc_fence_after();
      float* po = reinterpret_cast<float*>(smem + L::PART_O) + r * L::PART_LD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        if (n > 0) {
          tmem_ld32(tmem + lane_base + 256 + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          reinterpret_cast<float4*>(po + c * 32)[k] = make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
      }
      reinterpret_cast<float*>(smem + L::PART_M)[r] = ok && n > 0 ? m_used : -INFINITY;
      reinterpret_cast<float*>(smem + L::PART_L)[r] = ok && n > 0 ? l : 0.f;
    } else if (active && S > 1) {
      // Split keys: this CTA's partial of tile t's rows (zeros without keys).
      if (ok && n > 0) ok = mbar_wait(o_done, 0, abort_flag);
      tc_fence_after();
      float* base = p.kv_part + (static_cast<size_t>(item) * S + sidx) * ATT_PART_FLOATS;
      const int prow = t * 128 + r;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        if (n > 0) {
          tmem_ld32(tmem + lane_base + 256 + t * 128 + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          reinterpret_cast<float4*>(base)[(c * 8 + k) * 256 + prow] =
              make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
      }
      base[256 * 128 + prow] = ok && n > 0 ? m_used : -INFINITY;
      base[256 * 128 + 256 + prow] = ok && n > 0 ? l : 0.f;
    } else if (active) {
      if (ok && n > 0) ok = mbar_wait(o_done, 0, abort_flag);
      tc_fence_after();
      const int qr = q0 + t * 128 + r;
      const bool store = qr < p.q_rows && !idle;
      __nv_bfloat16* orow = p.out + (static_cast<long long>(b) * p.q_rows + qr) * p.ldo + h * 128;
      const float inv = (ok && n > 0 && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + 256 + t * 128 + c * 32, o);
        tmem_wait_ld();
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4 w;
            w.x = pack_bf16(o[8 * k + 0] * inv, o[8 * k + 1] * inv);
            w.y = pack_bf16(o[8 * k + 2] * inv, o[8 * k + 3] * inv);
            w.z = pack_bf16(o[8 * k + 4] * inv, o[8 * k + 5] * inv);
            w.w = pack_bf16(o[8 * k + 6] * inv, o[8 * k + 7] * inv);
            dst[k] = w;
          }
        }
      }
    }
  }

  if (S > 1 && warp < 8) att_split_merge(p, item, S, q0, b, h, has_b, abort_flag, last_split);
  if (grouped) {
    // Exchange: CTA k owns rows [(k % R) ro, + ro) of candidate b0 + k / R
    // (ro = q_rows / R, rows own0 + [0, ro) of the group tile). Each CTA
    // announces the bytes its rows will receive, barrier A (every partial is
    // written; every CTA's MMAs and loads are done, so its ring is free),
    // one thread sends each owner its rows (O, m, l) by bulk copy into slot
    // `crank`, owners merge in sender order (the result does not depend on
    // timing), barrier C keeps every CTA alive until its copies out landed.
    const int qr = p.q_rows;
    const int ro = qr / R;
    const int own0 = (crank / R) * qr + (crank % R) * ro;
    const uint32_t slot_bytes = static_cast<uint32_t>(ro * (L::PART_LD + 2) * 4);
    const float* part_o = reinterpret_cast<const float*>(smem + L::PART_O);
    const float* part_m = reinterpret_cast<const float*>(smem + L::PART_M);
    const float* part_l = reinterpret_cast<const float*>(smem + L::PART_L);
    const uint8_t* recv = smem + L::RECV;
    if (threadIdx.x < 256) fence_proxy_async();
    if (threadIdx.x == 0) mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(C - 1) * slot_bytes);
    __syncwarp();
    cluster_sync_all();   // barrier A
    if (threadIdx.x == ATT_MMA_WARP * 32) {
      for (int o = 0; o < C; ++o) {
        if (o == crank) continue;
        const int orow0 = (o / R) * qr + (o % R) * ro;
        const uint32_t dst = map_to_rank(smem_u32(recv) + static_cast<uint32_t>(crank) * slot_bytes, o);
        const uint32_t bar = map_to_rank(recv_bar, o);
        bulk_copy_to_peer(dst, smem_u32(part_o + orow0 * L::PART_LD), ro * L::PART_LD * 4, bar);
        bulk_copy_to_peer(dst + ro * L::PART_LD * 4, smem_u32(part_m + orow0), ro * 4, bar);
        bulk_copy_to_peer(dst + ro * L::PART_LD * 4 + ro * 4, smem_u32(part_l + orow0), ro * 4, bar);
      }
    }
    if (threadIdx.x < 256) {
      const bool ok = mbar_wait(recv_bar, 0, abort_flag);
      // 16-column groups of this CTA's rows.
      for (int it = threadIdx.x; it < ro * 8; it += 256) {
        const int rr = it >> 3, cg = (it & 7) * 16;
        const int own = own0 + rr;
        float ms[8], ls[8];
        float M = -INFINITY;
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          ms[s2] = -INFINITY;
          ls[s2] = 0.f;
          if (s2 < C) {
            const float* rm = reinterpret_cast<const float*>(recv + s2 * slot_bytes) + ro * L::PART_LD;
            ms[s2] = s2 == crank ? part_m[own] : rm[rr];
            ls[s2] = s2 == crank ? part_l[own] : rm[ro + rr];
            M = fmaxf(M, ms[s2]);
          }
        }
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
        float den = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          if (s2 < C) {
            const float w = ms[s2] == -INFINITY ? 0.f : exp2f(ms[s2] - M);
            den += w * ls[s2];
            const float* src = s2 == crank
                                   ? part_o + own * L::PART_LD + cg
                                   : reinterpret_cast<const float*>(recv + s2 * slot_bytes) + rr * L::PART_LD + cg;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float4 v = reinterpret_cast<const float4*>(src)[k];
              acc[4 * k] += w * v.x;
              acc[4 * k + 1] += w * v.y;
              acc[4 * k + 2] += w * v.z;
              acc[4 * k + 3] += w * v.w;
            }
          }
        }
        const float inv = (ok && !*abort_flag && den > 0.f) ? 1.f / den : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(
            p.out + (static_cast<long long>(b0) * qr + own) * p.ldo + h * 128 + cg);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          uint4 w;
          w.x = pack_bf16(acc[8 * k + 0] * inv, acc[8 * k + 1] * inv);
          w.y = pack_bf16(acc[8 * k + 2] * inv, acc[8 * k + 3] * inv);
          w.z = pack_bf16(acc[8 * k + 4] * inv, acc[8 * k + 5] * inv);
          w.w = pack_bf16(acc[8 * k + 6] * inv, acc[8 * k + 7] * inv);
          dst[k] = w;
        }
      }
    }
    __syncwarp();
    cluster_sync_all();   // barrier C
  }
  tc_fence_before();
  __syncthreads();
  if (warp == ATT_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wamb
