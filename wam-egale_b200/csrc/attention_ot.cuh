// Attention with the output transposed in TMEM, for queries longer than one
// tile (same inputs, outputs and split-key partials as attn_tc_kernel):
//
//   S_t = Q_t K_j^T      one query tile t in {A, B} (128 rows) per MMA, N 128 keys
//   O^T += V_j^T P_j^T   both tiles in one MMA: M 128 head dims, N 256 queries
//
// An N 256 tcgen05.mma costs little more than an N 128 one (measured ~1.15x
// for twice the work), and with head dim 128 the usual O += P V can only be
// N 128; here the P V product runs as half as many N 256 instructions. P
// goes to shared memory (the B operand, K-major: [256 queries][128 keys]),
// V_j is the A operand read MN-major straight from its tile, and O^T (lane =
// head dim, column = query) fills TMEM columns [256, 512). S_A and S_B keep
// columns [0, 128) and [128, 256); each is free again as soon as its softmax
// warps have loaded it, so S(j+1) is computed while the softmax of tile j
// runs, and only the P buffer orders one key tile's softmax after the
// previous key tile's O^T update.
//
// 320 threads: warps 0-3 softmax of tile A, 4-7 of tile B (one thread per
// query row, all 128 keys), warp 8 TMA producer, warp 9 TMEM owner whose
// lane 0 issues the MMAs. A CTA always runs both tiles (rows past q_rows
// compute on zero-filled queries and are not stored).
//
// Row max growth: O^T column q must be scaled by alpha_q before the next
// O^T update. Rows keep their stale max unless it grows by more than 2^8
// (as in attn_tc_kernel), so this is rare; when any row of the CTA grows,
// all 8 softmax warps rescale their 32-lane x 128-column slab of O^T after
// the previous update completed.
//
// SMEM: Q_A, Q_B (64 KB), a 3-slot K/V ring (96 KB) in consumption order
// K_0, K_1, V_0, K_2, V_1, ..., the P buffer (64 KB), per-row alpha / 1/l.
#pragma once
#include "attention.cuh"

namespace wamb {

constexpr int ATO_SLOTS = 3;
// exp2 of keys 2i, 2i + 1 of every 32 on the MUFU for i < ATO_MUFU_PAIRS,
// the rest as the cubic on the FMA pipe. One cfg2 chunk (CUDA events): 12
// pairs 78.5 us, 11 pairs 79.2 us, 10 pairs 81.1 us.
constexpr int ATO_MUFU_PAIRS = 12;

struct AttnOtSmem {
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t RING_OFF = 2 * ATT_TILE_BYTES;
  static constexpr uint32_t P_OFF = RING_OFF + ATO_SLOTS * ATT_TILE_BYTES;
  static constexpr uint32_t P_ATOM = 256 * 128;                          // 256 rows x 64 keys x 2 B
  static constexpr uint32_t ROW_OFF = P_OFF + 2 * P_ATOM;                // float[256]: alpha, then 1/l
  static constexpr uint32_t BAR_OFF = ROW_OFF + 256 * 4;
  // q_full, full[3], empty[3], s_full[2], s_free[2], p_full, p_free, o_done, drain
  static constexpr uint32_t NBARS = 15;
  // After the barriers: TMEM address, abort flag, split flag, spare, then
  // the softmax warps' grow flags [2 key-tile parities][8 warps].
  static constexpr uint32_t TOTAL = 1024 + BAR_OFF + NBARS * 8 + 16 + 64;
  static_assert(TOTAL <= 232448, "attention shared memory exceeds 227 KB");
  // Epilogue staging over the ring and the P buffer once every MMA is done:
  // fp32 O [256 rows][128] (split keys) or bf16 O [256 rows][128].
  static_assert(RING_OFF + 256 * 128 * 4 <= ROW_OFF, "output staging does not fit");
};

WAMB_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_ot_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                   const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                   const __grid_constant__ CUtensorMap tmV1, const AttnParams p) {
  using L = AttnOtSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sQ = smem_u32(smem + L::Q_OFF);
  const uint32_t sRing = smem_u32(smem + L::RING_OFF);
  const uint32_t sP = smem_u32(smem + L::P_OFF);
  float* row_f = reinterpret_cast<float*>(smem + L::ROW_OFF);
  const uint32_t bar0 = smem_u32(smem + L::BAR_OFF);
  const uint32_t q_full = bar0;
  const uint32_t full = bar0 + 8;               // [3] by ring slot
  const uint32_t empty = full + 8 * ATO_SLOTS;  // [3]
  const uint32_t s_full = empty + 8 * ATO_SLOTS;   // [2] by query tile
  const uint32_t s_free = s_full + 16;          // [2] by query tile
  const uint32_t p_full = s_free + 16;
  const uint32_t p_free = p_full + 8;
  const uint32_t o_done = p_free + 8;
  const uint32_t drain = o_done + 8;
  auto slot_addr = [&](int L) { return sRing + (L % ATO_SLOTS) * ATT_TILE_BYTES; };
  auto slot_full = [&](int L) { return full + 8 * (L % ATO_SLOTS); };
  auto slot_empty = [&](int L) { return empty + 8 * (L % ATO_SLOTS); };
  auto slot_phase = [&](int L) { return static_cast<uint32_t>((L / ATO_SLOTS) & 1); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_split = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* grow_w = reinterpret_cast<volatile int*>(tmem_slot + 4);   // [2][8]

  if (p.trigger) pdl_trigger();
  pdl_wait();   // the tile list and Q/K/V of the previous kernels are complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.kv_splits > 1 ? p.kv_splits : 1;
  const int b = static_cast<int>(blockIdx.z) / S, sidx = static_cast<int>(blockIdx.z) - b * S, h = blockIdx.y;
  const int q0 = blockIdx.x * 256;
  const int item = (b * gridDim.y + h) * gridDim.x + blockIdx.x;
  const int n0 = p.tiles != nullptr ? *p.n_tiles : (p.src0_len + 127) / 128;
  const int n_all = n0 + (p.has_src1 ? (p.q_rows + 127) / 128 : 0);
  const int kv_lo = sidx * n_all / S;
  const int n = (sidx + 1) * n_all / S - kv_lo;
  auto tile_of = [&](int j) { return att_tile(p, kv_lo + j, n0, b); };
  // Ring load L -> key tile and K/V: K_0, then per j: K_{j+1} (if any), V_j.
  auto load_of = [&](int L, int& j, bool& is_v) {
    if (L == 0) { j = 0; is_v = false; return; }
    if (n == 1) { j = 0; is_v = true; return; }
    const int m = L - 1;            // pairs (K_{j+1}, V_j) for j < n - 1, then V_{n-1}
    if (m < 2 * (n - 1)) { j = (m >> 1) + (m & 1 ? 0 : 1); is_v = (m & 1) != 0; return; }
    j = n - 1;
    is_v = true;
  };
  const int n_loads = 2 * n;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ATO_SLOTS; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + 8 * i, 1);
      mbar_init(s_free + 8 * i, 4);   // the tile's four softmax warps loaded S
    }
    mbar_init(p_full, 8);             // all eight softmax warps wrote P
    mbar_init(p_free, 1);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
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
      const int qrow = b * p.q_rows + q0;
      const int qcol = p.q_col + h * 128;
      mbar_arrive_expect_tx(q_full, 2 * ATT_TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, qcol, qrow);
      tma_load_2d(sQ + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow);
      tma_load_2d(sQ + ATT_TILE_BYTES, &tmQ, q_full, qcol, qrow + 128);
      tma_load_2d(sQ + ATT_TILE_BYTES + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow + 128);
      int issued = 0;
      for (int L = 0; L < n_loads; ++L) {
        int j;
        bool is_v;
        load_of(L, j, is_v);
        const KvTile t = tile_of(j);
        const CUtensorMap* m = is_v ? (t.src ? &tmV1 : &tmV0) : (t.src ? &tmK1 : &tmK0);
        const int col = (is_v ? (t.src ? p.v1_col : p.v0_col) : (t.src ? p.k1_col : p.k0_col)) + h * 128;
        if (!mbar_wait(slot_empty(L), slot_phase(L) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(slot_full(L), ATT_TILE_BYTES);
        tma_load_2d(slot_addr(L), m, slot_full(L), col, t.row);
        tma_load_2d(slot_addr(L) + ATT_ATOM, m, slot_full(L), col + 64, t.row);
        issued = L + 1;
      }
      // Teardown: loads still in flight must land before the CTA exits.
      mbar_wait_teardown(q_full, 0);
      for (int L = max(0, issued - ATO_SLOTS); L < issued; ++L) mbar_wait_teardown(slot_full(L), slot_phase(L));
    }
  } else if (warp == ATT_MMA_WARP) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer (lane 0)
      constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0);
      // O^T: M 128 (head dim), N 256 (queries); A = V_j read MN-major, B = P K-major.
      constexpr uint32_t IDESC_O = idesc_bf16(128, 256, 0) | (1u << 15);
      auto issue_s = [&](int t, uint32_t kb) {
        const uint32_t qb = sQ + t * ATT_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * ATT_ATOM + (kk & 3) * 32;
          umma_bf16(tmem + t * 128, sw128_desc(qb + off, 16, 1024), sw128_desc(kb + off, 16, 1024), IDESC_S,
                    kk > 0);
        }
        umma_commit(s_full + 8 * t);
      };
      auto issue_pv = [&](uint32_t vb, int ksteps, bool acc) {
        for (int kk = 0; kk < ksteps; ++kk)
          umma_bf16(tmem + 256, sw128_desc(vb + kk * 2048, ATT_ATOM, 1024),
                    sw128_desc(sP + (kk >> 2) * L::P_ATOM + (kk & 3) * 32, 16, 1024), IDESC_O, acc || kk > 0);
      };
      // Zero V rows [len, 16*ceil(len/16)) of ring load Lv: P is 0 there, but
      // stale pool rows must not meet it.
      auto zero_v_tail = [&](int Lv, int len) {
        if (len & 15) {
          uint8_t* vt = smem + L::RING_OFF + (Lv % ATO_SLOTS) * ATT_TILE_BYTES;
          const int r0 = len, r1 = ((len + 15) >> 4) * 16;
          for (int i = 0; i < (r1 - r0) * 16; ++i) {
            const int r = r0 + (i >> 4), c = i & 15;
            *reinterpret_cast<uint4*>(vt + (c >> 3) * ATT_ATOM + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async();
        }
      };
      auto wait_full = [&](int Lx) { return mbar_wait(slot_full(Lx), slot_phase(Lx), abort_flag); };
      bool ok = mbar_wait(q_full, 0, abort_flag) && n > 0 && wait_full(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, slot_addr(0));
        issue_s(1, slot_addr(0));
        umma_commit(slot_empty(0));
      }
      int Lc = 1;
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) {
          // S(j+1) into the S columns the softmax of tile j has loaded.
          if (!wait_full(Lc)) { ok = false; break; }
          for (int t = 0; t < 2; ++t) {
            if (!mbar_wait(s_free + 8 * t, j & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, slot_addr(Lc));
          }
          if (!ok) break;
          umma_commit(slot_empty(Lc));
          ++Lc;
        }
        const int len = tile_of(j).len;
        if (!wait_full(Lc)) { ok = false; break; }
        zero_v_tail(Lc, len);
        if (!mbar_wait(p_full, j & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        issue_pv(slot_addr(Lc), (len + 15) >> 4, j > 0);
        umma_commit(p_free);
        umma_commit(slot_empty(Lc));
        ++Lc;
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
    const int r = wq * 32 + lane;     // query row within the tile == TMEM lane of S
    const int q = t * 128 + r;        // row of the CTA's 256 (P row, O^T column)
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // Every warp runs every key tile, its named barriers included, even after
    // an abort (the waits then return at once and the work is skipped), so no
    // warp is left at a barrier.
    for (int j = 0; j < n; ++j) {
      const int hi = tile_of(j).len;   // valid key columns [0, hi)
      if (ok) ok = mbar_wait(s_full + 8 * t, j & 1, abort_flag);
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
      // S_t is in registers: the MMA warp may compute S_t(j+1) over it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free + 8 * t);
      if (hi < 128) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= hi) s[i] = -INFINITY;
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        mx0 = fmax3(mx0, s[i], s[i + 1]);
        mx1 = fmax3(mx1, s[32 + i], s[32 + i + 1]);
        mx2 = fmax3(mx2, s[64 + i], s[64 + i + 1]);
        mx3 = fmax3(mx3, s[96 + i], s[96 + i + 1]);
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * p.scale_log2;
      // Keep the stale max unless the new one exceeds it by more than 2^8.
      const bool grow = mx > m_used + ATT_RESCALE_LOG2;
      const float m_new = grow ? mx : m_used;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = grow ? exp2f(m_used - m_use) : 1.f;
      const uint64_t scale2 = f2(p.scale_log2, p.scale_log2);
      const uint64_t neg_m2 = f2(-m_use, -m_use);
      uint64_t sum2 = f2(0.f, 0.f), sum2p = f2(0.f, 0.f);
      // P as packed bf16 pairs: keys 2 ATO_MUFU_PAIRS .. 31 of every 32 take
      // the cubic, the rest the MUFU exp2.
      uint32_t pk[64];
      // exp2 of keys [32 c, 32 c + 32) into pk[16 c, 16 c + 16).
      auto exp_chunk = [&](int c) {
#pragma unroll
        for (int i = 0; i < ATO_MUFU_PAIRS; ++i) {
          const int k = 32 * c + 2 * i;
          const float2 x = f2_split(ffma2(f2(s[k], s[k + 1]), scale2, neg_m2));
          const float a = ex2_mufu(x.x), bb = ex2_mufu(x.y);
          sum2 = fadd2(sum2, f2(a, bb));
          pk[16 * c + i] = pack_bf16(a, bb);
        }
#pragma unroll
        for (int i = ATO_MUFU_PAIRS; i < 16; ++i) {
          const int k = 32 * c + 2 * i;
          const uint64_t e = ex2_poly2(ffma2(f2(s[k], s[k + 1]), scale2, neg_m2));
          sum2p = fadd2(sum2p, e);
          const float2 ev = f2_split(e);
          pk[16 * c + i] = pack_bf16(ev.x, ev.y);
        }
      };
      // P row q into the K-major SW128 buffer: 16-byte chunk c of the row's
      // 64-key atom at ((c ^ (q & 7)) * 16).
      auto store_p = [&](int c) {
        const uint32_t addr = sP + (c >> 3) * L::P_ATOM + q * 128 + (((c & 7) ^ (q & 7)) << 4);
        st_shared_v4(addr, pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      };
      // The first three quarters of the keys, then (the previous O^T update
      // having read P) their P goes out while the last quarter is computed,
      // so most of P's 64 KB of shared-memory stores overlap the exp2s.
#pragma unroll
      for (int c = 0; c < 3; ++c) exp_chunk(c);
      if (j > 0) {
        // The previous O^T update has read P and written O^T.
        if (ok) ok = mbar_wait(p_free, (j - 1) & 1, abort_flag);
        tc_fence_after();
        // Rows whose max grew: scale their O^T columns (all 8 warps, each
        // its 32 head dims x its tile's 128 queries) before the next update.
        // One flag per warp, in two sets by key-tile parity (a warp running
        // a tile ahead writes the other set), so the usual tile without
        // growth costs one named barrier; a growth costs two more (the
        // alphas are written, then every warp has read them).
        volatile int* gw = grow_w + (j & 1) * 8;
        const bool g_any = __any_sync(0xffffffffu, grow);
        if (lane == 0) gw[warp] = g_any ? 1 : 0;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const bool rescale = (gw[0] | gw[1] | gw[2] | gw[3] | gw[4] | gw[5] | gw[6] | gw[7]) != 0;
        if (rescale) {
          row_f[q] = alpha;
          asm volatile("bar.sync 1, 256;" ::: "memory");
          if (ok) {
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              float o[32];
              const uint32_t oc = 256 + t * 128 + c * 32;
              tmem_ld32(tmem + lane_base + oc, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= row_f[t * 128 + c * 32 + i];
              tmem_st32(tmem + lane_base + oc, o);
            }
            tmem_wait_st();
          }
          asm volatile("bar.sync 1, 256;" ::: "memory");   // every warp read the alphas
        }
      }
#pragma unroll
      for (int c = 0; c < 12; ++c) store_p(c);
      exp_chunk(3);
#pragma unroll
      for (int c = 12; c < 16; ++c) store_p(c);
      const float2 sv = f2_split(fadd2(sum2, sum2p));
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      l = l * alpha + (sv.x + sv.y);
      m_used = m_new;
    }
    if (ok && n > 0) ok = mbar_wait(o_done, 0, abort_flag);
    tc_fence_after();
    // Epilogue: O^T slab (head dims [32 wq, +32), queries of tile t) through
    // shared memory (the drained ring and P buffer) to row-major output.
    if (S > 1) {
      // Split keys: this CTA's partial (O unnormalized relative to m, then m, l).
      float* stage = reinterpret_cast<float*>(smem + L::RING_OFF);   // [256][128] fp32
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + 256 + t * 128 + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) stage[(t * 128 + c * 32 + i) * 128 + wq * 32 + lane] = n > 0 ? o[i] : 0.f;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      float* base = p.kv_part + (static_cast<size_t>(item) * S + sidx) * ATT_PART_FLOATS;
      const int prow = threadIdx.x;   // 0..255
#pragma unroll 4
      for (int jg = 0; jg < 32; ++jg)
        reinterpret_cast<float4*>(base)[jg * 256 + prow] = *reinterpret_cast<const float4*>(stage + prow * 128 + 4 * jg);
      base[256 * 128 + q] = ok && n > 0 ? m_used : -INFINITY;
      base[256 * 128 + 256 + q] = ok && n > 0 ? l : 0.f;
      att_split_merge(p, item, S, q0, b, h, true, abort_flag, last_split);
    } else {
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem + L::RING_OFF);   // [256][128] bf16
      row_f[q] = (ok && !*abort_flag && l > 0.f) ? 1.f / l : 0.f;
      asm volatile("bar.sync 1, 256;" ::: "memory");
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + 256 + t * 128 + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qq = t * 128 + c * 32 + i;
          stage[qq * 128 + wq * 32 + lane] = __float2bfloat16_rn(o[i] * row_f[qq]);
        }
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      // Row-major copy out: 256 rows x 256 bytes, 16 bytes per thread step.
      for (int i = threadIdx.x; i < 256 * 16; i += 256) {
        const int rr = i >> 4, ch = i & 15;
        if (q0 + rr < p.q_rows)
          *reinterpret_cast<uint4*>(p.out + (static_cast<long long>(b) * p.q_rows + q0 + rr) * p.ldo + h * 128 +
                                    ch * 8) = reinterpret_cast<const uint4*>(stage + rr * 128)[ch];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == ATT_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wamb
