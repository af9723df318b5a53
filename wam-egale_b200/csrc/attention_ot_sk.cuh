// Stream-K variant of attn_ot_kernel (same tiles, MMAs and softmax) for
// calls whose whole items would leave SMs idle, on a persistent grid.
//
// An item is (query tile pair, head, batch row), n key tiles long. With I
// items on G CTAs, items [0, dp) go whole to CTAs round-robin (dp = the
// whole waves but the last, so the CTAs of one wave share their heads' K/V
// in L2), and the key tiles of the remaining items are cut into G equal
// ranges, one per CTA: a CTA then runs a sequence of segments (item, key
// tiles [ja, jb)). A segment over a whole item writes its rows; a partial
// one writes O (relative to its row max m), m and l to the CTA's partial
// slot (0 for its first stream-K segment, 1 for its last) and adds one to
// the item's counter; the CTA that brings it to the item's segment count
// combines the partials in key order (the result does not depend on
// timing), writes the rows and resets the counter. Every wait in the
// kernel is on this CTA's own barriers: no CTA waits for another.
//
// Across segments the ring, the S buffers and the P buffer keep running
// (phases count key tiles over the whole CTA); Q is reloaded once the last
// S MMAs of a segment completed (q_empty), and the first O^T update of a
// segment waits until the epilogue of the previous one has read O^T out of
// TMEM (o_free). A pair whose tile B holds no query row (the last 128 or
// fewer rows) skips S_B and runs O^T as N 128 MMAs; that tile's softmax
// warps still run every step on whatever S_B holds (its P rows are not read
// and none of its rows is stored), which measured faster than masking them.
//
// SMEM as attn_ot_kernel, the P buffer also being the bf16 output staging
// of a whole item (the ring keeps loading the next segment).
#pragma once
#include "attention_ot.cuh"

namespace wamb {

struct AttnOtSkSmem {
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t RING_OFF = 2 * ATT_TILE_BYTES;
  static constexpr uint32_t P_OFF = RING_OFF + ATO_SLOTS * ATT_TILE_BYTES;
  static constexpr uint32_t P_ATOM = 256 * 128;                          // 256 rows x 64 keys x 2 B
  static constexpr uint32_t ROW_OFF = P_OFF + 2 * P_ATOM;                // float[256]: alpha, then 1/l
  static constexpr uint32_t BAR_OFF = ROW_OFF + 256 * 4;
  // q_full, q_empty, full[3], empty[3], s_full[2], s_free[2], p_full, p_free,
  // o_done, o_free, drain
  static constexpr uint32_t NBARS = 17;
  // After the barriers: TMEM address, abort flag, spare, segment flag, then
  // the softmax warps' grow flags [2 key-tile parities][8 warps].
  static constexpr uint32_t TOTAL = 1024 + BAR_OFF + NBARS * 8 + 16 + 64;
  static_assert(TOTAL <= 232448, "attention shared memory exceeds 227 KB");
  // bf16 output staging [256 rows][128] over the P buffer.
  static_assert(256 * 128 * 2 <= 2 * P_ATOM, "output staging does not fit");
};

// ---------------------------------------------------------- the schedule
// Work of CTA c of G: its round-robin items c, c + G, ... below dp, then
// its stream-K units [u0, u1) (unit x: key tile x % n of item dp + x / n).
struct OtSched {
  int G, c, n, dp, ndp, nsk;
  long long U, u0, u1;
};

// First stream-K unit of CTA c (c = G: the end).
WAMB_DEV long long ot_bound(long long U, int G, int c) { return static_cast<long long>(c) * U / G; }

// Stream-K units of a launch of G CTAs over items of n key tiles, 0 for
// whole items only: at least 8 key tiles per CTA, and every item over at
// most ATT_MAX_SPLITS CTAs (ceil(n / q) + 1 is the most an item meets).
WAMB_DEV long long ot_sk_units(const AttnParams& p, int n, int G) {
  if (!p.ot_sk || n <= 0 || p.kv_part == nullptr || p.kv_count == nullptr || p.ot_dp_items >= p.ot_items) return 0;
  const long long U = static_cast<long long>(p.ot_items - p.ot_dp_items) * n;
  const long long q = U / G;   // the fewest units of a CTA
  return q >= 8 && (n + q - 1) / q + 1 <= ATT_MAX_SPLITS ? U : 0;
}

WAMB_DEV OtSched ot_schedule(const AttnParams& p, int n) {
  OtSched s;
  s.G = static_cast<int>(gridDim.x);
  s.c = static_cast<int>(blockIdx.x);
  s.n = n;
  s.U = ot_sk_units(p, n, s.G);
  s.dp = s.U == 0 ? p.ot_items : p.ot_dp_items;   // whole items only without stream-K
  s.ndp = s.c < s.dp ? (s.dp - s.c + s.G - 1) / s.G : 0;
  s.u0 = ot_bound(s.U, s.G, s.c);
  s.u1 = ot_bound(s.U, s.G, s.c + 1);
  s.nsk = s.u1 > s.u0 ? static_cast<int>((s.u1 - 1) / n - s.u0 / n + 1) : 0;
  return s;
}

struct OtSeg {
  int item, ja, jb;
  int slot;   // -1: the whole item; else this CTA's partial slot
};

// Segment k of this CTA (k < ndp + nsk).
WAMB_DEV OtSeg ot_segment(const OtSched& s, int k) {
  OtSeg g;
  if (k < s.ndp) {
    g.item = s.c + k * s.G;
    g.ja = 0;
    g.jb = s.n;
    g.slot = -1;
    return g;
  }
  k -= s.ndp;
  const long long i = s.u0 / s.n + k;
  const long long a = max(s.u0, i * s.n), e = min(s.u1, (i + 1) * s.n);
  g.item = s.dp + static_cast<int>(i);
  g.ja = static_cast<int>(a - i * s.n);
  g.jb = static_cast<int>(e - i * s.n);
  g.slot = (g.ja == 0 && g.jb == s.n) ? -1 : (k == 0 ? 0 : 1);
  return g;
}

// CTAs c0, c0 + 1, ..., c0 + ns - 1 hold the partials of stream-K item r
// (relative to dp), in key order.
WAMB_DEV void ot_item_ctas(const OtSched& s, long long r, int& c0, int& ns) {
  auto cta_of = [&](long long x) { return static_cast<int>(((x + 1) * s.G - 1) / s.U); };
  c0 = cta_of(r * s.n);
  ns = cta_of((r + 1) * s.n - 1) - c0 + 1;
}

// One partial: O [256 queries][128 head dims] fp32 (row-major, so that a
// warp's store of one query's 32 head dims is one 128-byte line), then
// m [256] and l [256].
WAMB_DEV float* ot_part(const AttnParams& p, int c, int slot) {
  return p.kv_part + (static_cast<size_t>(c) * 2 + slot) * ATT_PART_FLOATS;
}

// Merge of NS stream-K partials, rows r0 .. r0 + 7 of an item by one warp:
// lane the head dims [4 lane, 4 lane + 4); all NS partials of the 8 rows
// are loaded at once, then combined in key order with the weights
// exp2(m_s - M) / sum_s exp2(m_s - M) l_s (lanes 0..7 compute one row's).
template <int NS>
WAMB_DEV void ot_merge_rows(const AttnParams& p, const float* const (&part)[ATT_MAX_SPLITS], int q0, int r0, int b,
                            int h) {
  const int lane = threadIdx.x & 31;
  float wt[NS], inv;
  {
    const int q = r0 + (lane & 7);
    float m[NS], M = -INFINITY, den = 0.f;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      m[k] = __ldcg(part[k] + 256 * 128 + q);
      M = fmaxf(M, m[k]);
    }
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      wt[k] = m[k] == -INFINITY ? 0.f : exp2f(m[k] - M);
      den += wt[k] * __ldcg(part[k] + 256 * 128 + 256 + q);
    }
    inv = den > 0.f ? 1.f / den : 0.f;
  }
  float4 v[NS][8];
#pragma unroll
  for (int rr = 0; rr < 8; ++rr)
#pragma unroll
    for (int k = 0; k < NS; ++k) v[k][rr] = __ldcg(reinterpret_cast<const float4*>(part[k] + (r0 + rr) * 128) + lane);
#pragma unroll
  for (int rr = 0; rr < 8; ++rr) {
    float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const float wk = __shfl_sync(0xffffffffu, wt[k], rr);
      a[0] += wk * v[k][rr].x;
      a[1] += wk * v[k][rr].y;
      a[2] += wk * v[k][rr].z;
      a[3] += wk * v[k][rr].w;
    }
    const float iv = __shfl_sync(0xffffffffu, inv, rr);
    if (q0 + r0 + rr < p.q_rows)
      *reinterpret_cast<uint2*>(p.out + (static_cast<long long>(b) * p.q_rows + q0 + r0 + rr) * p.ldo + h * 128 +
                                4 * lane) = make_uint2(pack_bf16(a[0] * iv, a[1] * iv), pack_bf16(a[2] * iv, a[3] * iv));
  }
}

// Merge of stream-K item `item` by the 256 softmax threads of the CTA that
// completed it: warp w takes rows [32 w, 32 w + 32) in four steps.
template <int NS>
WAMB_DEV void ot_merge_item(const AttnParams& p, const float* const (&part)[ATT_MAX_SPLITS], int q0, int b, int h) {
  const int w = threadIdx.x >> 5;
#pragma unroll 1
  for (int r0 = 32 * w; r0 < 32 * w + 32 && q0 + r0 < p.q_rows; r0 += 8) ot_merge_rows<NS>(p, part, q0, r0, b, h);
}

WAMB_DEV void ot_merge(const AttnParams& p, const OtSched& s, int item, int q0, int b, int h) {
  int c0, ns;
  const long long r = item - s.dp;
  ot_item_ctas(s, r, c0, ns);
  const float* part[ATT_MAX_SPLITS];
#pragma unroll
  for (int k = 0; k < ATT_MAX_SPLITS; ++k) {
    const int c = c0 + min(k, ns - 1);
    part[k] = ot_part(p, c, ot_bound(s.U, s.G, c) / s.n == r ? 0 : 1);
  }
  static_assert(ATT_MAX_SPLITS == 4, "merge cases");
  if (ns == 2) ot_merge_item<2>(p, part, q0, b, h);
  else if (ns == 3) ot_merge_item<3>(p, part, q0, b, h);
  else ot_merge_item<4>(p, part, q0, b, h);
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_ot_sk_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                   const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                   const __grid_constant__ CUtensorMap tmV1, const AttnParams p) {
  using L = AttnOtSkSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sQ = smem_u32(smem + L::Q_OFF);
  const uint32_t sRing = smem_u32(smem + L::RING_OFF);
  const uint32_t sP = smem_u32(smem + L::P_OFF);
  float* row_f = reinterpret_cast<float*>(smem + L::ROW_OFF);
  const uint32_t bar0 = smem_u32(smem + L::BAR_OFF);
  const uint32_t q_full = bar0;
  const uint32_t q_empty = bar0 + 8;
  const uint32_t full = bar0 + 16;              // [3] by ring slot
  const uint32_t empty = full + 8 * ATO_SLOTS;  // [3]
  const uint32_t s_full = empty + 8 * ATO_SLOTS;   // [2] by query tile
  const uint32_t s_free = s_full + 16;          // [2] by query tile
  const uint32_t p_full = s_free + 16;
  const uint32_t p_free = p_full + 8;
  const uint32_t o_done = p_free + 8;
  const uint32_t o_free = o_done + 8;
  const uint32_t drain = o_free + 8;
  auto slot_addr = [&](int x) { return sRing + (x % ATO_SLOTS) * ATT_TILE_BYTES; };
  auto slot_full = [&](int x) { return full + 8 * (x % ATO_SLOTS); };
  auto slot_empty = [&](int x) { return empty + 8 * (x % ATO_SLOTS); };
  auto slot_phase = [&](int x) { return static_cast<uint32_t>((x / ATO_SLOTS) & 1); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* grow_w = reinterpret_cast<volatile int*>(tmem_slot + 4);   // [2][8]
  volatile int* last_seg = reinterpret_cast<volatile int*>(tmem_slot + 3);

  if (p.trigger) pdl_trigger();
  pdl_wait();   // the tile list and Q/K/V of the previous kernels are complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = p.tiles != nullptr ? *p.n_tiles : (p.src0_len + 127) / 128;
  const int n_all = n0 + (p.has_src1 ? (p.q_rows + 127) / 128 : 0);
  const OtSched sc = ot_schedule(p, n_all);
  const int nseg = sc.ndp + sc.nsk;
  // Item -> batch row, head, first query row of its pair.
  auto coords = [&](int item, int& b, int& h, int& q0) {
    const int bh = item / p.ot_qpairs;
    q0 = (item - bh * p.ot_qpairs) * 256;
    h = bh % p.heads;
    b = bh / p.heads;
  };
  if (n_all == 0) {
    // No keys: the rows are zero (every segment is a whole item here).
    for (int k = 0; k < nseg; ++k) {
      int b, h, q0;
      coords(ot_segment(sc, k).item, b, h, q0);
      for (int i = threadIdx.x; i < 256 * 16; i += ATT_THREADS) {
        const int rr = i >> 4, ch = i & 15;
        if (q0 + rr < p.q_rows)
          *reinterpret_cast<uint4*>(p.out + (static_cast<long long>(b) * p.q_rows + q0 + rr) * p.ldo + h * 128 +
                                    ch * 8) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }
  // Ring load x of a segment of n key tiles -> key tile and K/V: K_0, then
  // per j: K_{j+1} (if any), V_j.
  auto load_of = [](int x, int n, int& j, bool& is_v) {
    if (x == 0) { j = 0; is_v = false; return; }
    if (n == 1) { j = 0; is_v = true; return; }
    const int m = x - 1;            // pairs (K_{j+1}, V_j) for j < n - 1, then V_{n-1}
    if (m < 2 * (n - 1)) { j = (m >> 1) + (m & 1 ? 0 : 1); is_v = (m & 1) != 0; return; }
    j = n - 1;
    is_v = true;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
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
    mbar_init(o_free, 8);             // all eight softmax warps read O^T
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
      int issued = 0, nq = 0;
      bool ok = true;
      for (int k = 0; ok && k < nseg; ++k) {
        const OtSeg sg = ot_segment(sc, k);
        int b, h, q0;
        coords(sg.item, b, h, q0);
        const bool has_b = q0 + 128 < p.q_rows;
        const int n = sg.jb - sg.ja;
        // Q of this segment once the previous segment's S MMAs completed.
        if (k > 0 && !mbar_wait(q_empty, (k - 1) & 1, abort_flag)) break;
        const int qrow = b * p.q_rows + q0;
        const int qcol = p.q_col + h * 128;
        mbar_arrive_expect_tx(q_full, (has_b ? 2 : 1) * ATT_TILE_BYTES);
        tma_load_2d(sQ, &tmQ, q_full, qcol, qrow);
        tma_load_2d(sQ + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow);
        if (has_b) {
          tma_load_2d(sQ + ATT_TILE_BYTES, &tmQ, q_full, qcol, qrow + 128);
          tma_load_2d(sQ + ATT_TILE_BYTES + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow + 128);
        }
        nq = k + 1;
        for (int x = 0; x < 2 * n; ++x) {
          int j;
          bool is_v;
          load_of(x, n, j, is_v);
          const KvTile t = att_tile(p, sg.ja + j, n0, b);
          const CUtensorMap* m = is_v ? (t.src ? &tmV1 : &tmV0) : (t.src ? &tmK1 : &tmK0);
          const int col = (is_v ? (t.src ? p.v1_col : p.v0_col) : (t.src ? p.k1_col : p.k0_col)) + h * 128;
          if (!mbar_wait(slot_empty(issued), slot_phase(issued) ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(slot_full(issued), ATT_TILE_BYTES);
          tma_load_2d(slot_addr(issued), m, slot_full(issued), col, t.row);
          tma_load_2d(slot_addr(issued) + ATT_ATOM, m, slot_full(issued), col + 64, t.row);
          ++issued;
        }
      }
      // Teardown: loads still in flight must land before the CTA exits.
      if (nq > 0) mbar_wait_teardown(q_full, (nq - 1) & 1);
      for (int x = max(0, issued - ATO_SLOTS); x < issued; ++x) mbar_wait_teardown(slot_full(x), slot_phase(x));
    }
  } else if (warp == ATT_MMA_WARP) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer (lane 0)
      constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0);
      // O^T: M 128 (head dim), N 256 (queries) or 128 (tile A alone); A = V_j
      // read MN-major, B = P K-major.
      constexpr uint32_t IDESC_O = idesc_bf16(128, 256, 0) | (1u << 15);
      constexpr uint32_t IDESC_O1 = idesc_bf16(128, 128, 0) | (1u << 15);
      auto issue_s = [&](int t, uint32_t kb) {
        const uint32_t qb = sQ + t * ATT_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * ATT_ATOM + (kk & 3) * 32;
          umma_bf16(tmem + t * 128, sw128_desc(qb + off, 16, 1024), sw128_desc(kb + off, 16, 1024), IDESC_S,
                    kk > 0);
        }
      };
      auto issue_pv = [&](uint32_t vb, int ksteps, bool acc, bool has_b) {
        for (int kk = 0; kk < ksteps; ++kk)
          umma_bf16(tmem + 256, sw128_desc(vb + kk * 2048, ATT_ATOM, 1024),
                    sw128_desc(sP + (kk >> 2) * L::P_ATOM + (kk & 3) * 32, 16, 1024), has_b ? IDESC_O : IDESC_O1,
                    acc || kk > 0);
      };
      // Zero V rows [len, 16*ceil(len/16)) of ring load x: P is 0 there, but
      // stale pool rows must not meet it.
      auto zero_v_tail = [&](int x, int len) {
        if (len & 15) {
          uint8_t* vt = smem + L::RING_OFF + (x % ATO_SLOTS) * ATT_TILE_BYTES;
          const int r0 = len, r1 = ((len + 15) >> 4) * 16;
          for (int i = 0; i < (r1 - r0) * 16; ++i) {
            const int r = r0 + (i >> 4), c = i & 15;
            *reinterpret_cast<uint4*>(vt + (c >> 3) * ATT_ATOM + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async();
        }
      };
      auto wait_full = [&](int x) { return mbar_wait(slot_full(x), slot_phase(x), abort_flag); };
      int lc = 0, g = 0;   // ring loads consumed, key tiles done (whole CTA)
      bool ok = true;
      // S_t of key tile gj (ring load x): into S columns the softmax of key
      // tile gj - 1 has loaded; tile B only when it holds query rows.
      auto s_step = [&](int gj, int x, bool has_b) {
        for (int t = 0; t < 2; ++t) {
          if (gj > 0 && !mbar_wait(s_free + 8 * t, (gj - 1) & 1, abort_flag)) return false;
          tc_fence_after();
          if (t == 0 || has_b) issue_s(t, slot_addr(x));
          umma_commit(s_full + 8 * t);
        }
        umma_commit(slot_empty(x));
        return true;
      };
      for (int k = 0; ok && k < nseg; ++k) {
        const OtSeg sg = ot_segment(sc, k);
        int b, h, q0;
        coords(sg.item, b, h, q0);
        const bool has_b = q0 + 128 < p.q_rows;
        const int n = sg.jb - sg.ja;
        if (!mbar_wait(q_full, k & 1, abort_flag) || !wait_full(lc)) { ok = false; break; }
        tc_fence_after();
        if (!s_step(g, lc, has_b)) { ok = false; break; }
        ++lc;
        if (n == 1) umma_commit(q_empty);
        for (int j = 0; j < n; ++j) {
          if (j + 1 < n) {
            if (!wait_full(lc)) { ok = false; break; }
            tc_fence_after();
            if (!s_step(g + j + 1, lc, has_b)) { ok = false; break; }
            ++lc;
            if (j + 2 == n) umma_commit(q_empty);   // the segment's last S MMAs read Q
          }
          const int len = att_tile(p, sg.ja + j, n0, b).len;
          if (!wait_full(lc)) { ok = false; break; }
          zero_v_tail(lc, len);
          if (!mbar_wait(p_full, (g + j) & 1, abort_flag)) { ok = false; break; }
          // The first update of a segment overwrites O^T: the previous
          // segment's epilogue must have read it.
          if (j == 0 && k > 0 && !mbar_wait(o_free, (k - 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(slot_addr(lc), (len + 15) >> 4, j > 0, has_b);
          umma_commit(p_free);
          umma_commit(slot_empty(lc));
          ++lc;
        }
        if (!ok) break;
        umma_commit(o_done);
        g += n;
      }
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
    const int d = wq * 32 + lane;     // head dim == TMEM lane of O^T
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    bool ok = true;
    int g = 0;
    // Every warp runs every segment and key tile, its named barriers
    // included, even after an abort (the waits then return at once and the
    // work is skipped), so no warp is left at a barrier.
    for (int k = 0; k < nseg; ++k) {
      const OtSeg sg = ot_segment(sc, k);
      int b, h, q0;
      coords(sg.item, b, h, q0);
      // A tile B without query rows: its softmax runs on stale S_B (the MMA
      // warp skips S_B and reads only P's tile A rows); none of its rows is
      // read back from TMEM or stored.
      const bool active = t == 0 || q0 + 128 < p.q_rows;
      const int n = sg.jb - sg.ja;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const int gj = g + j;
        const int hi = att_tile(p, sg.ja + j, n0, b).len;   // valid key columns [0, hi)
        if (ok) ok = mbar_wait(s_full + 8 * t, gj & 1, abort_flag);
        tc_fence_after();
        bool grow;
        float m_new, alpha, lsum;
        uint32_t pk[64];
        float s[128];
        uint64_t sum2 = f2(0.f, 0.f), sum2p = f2(0.f, 0.f), scale2 = 0, neg_m2 = 0;
        // exp2 of keys [32 c, 32 c + 32) into pk[16 c, 16 c + 16): keys 24..31
        // of every 32 take the cubic, the rest the MUFU exp2 (as in
        // attn_tc_kernel).
        auto exp_chunk = [&](int c) {
#pragma unroll
          for (int i = 0; i < 12; ++i) {
            const int kk = 32 * c + 2 * i;
            const float2 x = f2_split(ffma2(f2(s[kk], s[kk + 1]), scale2, neg_m2));
            const float a = ex2_mufu(x.x), bb = ex2_mufu(x.y);
            sum2 = fadd2(sum2, f2(a, bb));
            pk[16 * c + i] = pack_bf16(a, bb);
          }
#pragma unroll
          for (int i = 12; i < 16; ++i) {
            const int kk = 32 * c + 2 * i;
            const uint64_t e = ex2_poly2(ffma2(f2(s[kk], s[kk + 1]), scale2, neg_m2));
            sum2p = fadd2(sum2p, e);
            const float2 ev = f2_split(e);
            pk[16 * c + i] = pack_bf16(ev.x, ev.y);
          }
        };
        // P row q into the K-major SW128 buffer: 16-byte chunk c of the
        // row's 64-key atom at ((c ^ (q & 7)) * 16).
        auto store_p = [&](int c) {
          const uint32_t addr = sP + (c >> 3) * L::P_ATOM + q * 128 + (((c & 7) ^ (q & 7)) << 4);
          st_shared_v4(addr, pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        };
        {
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
          grow = mx > m_used + ATT_RESCALE_LOG2;
          m_new = grow ? mx : m_used;
          const float m_use = m_new == -INFINITY ? 0.f : m_new;
          alpha = grow ? exp2f(m_used - m_use) : 1.f;
          scale2 = f2(p.scale_log2, p.scale_log2);
          neg_m2 = f2(-m_use, -m_use);
          // The first three quarters of the keys, then (the previous O^T
          // update having read P) their P goes out while the last quarter is
          // computed, as in attn_ot_kernel.
#pragma unroll
          for (int c = 0; c < 3; ++c) exp_chunk(c);
        }
        if (j > 0) {
          // The previous O^T update has read P and written O^T.
          if (ok) ok = mbar_wait(p_free, (gj - 1) & 1, abort_flag);
          tc_fence_after();
          // Rows whose max grew: scale their O^T columns before the next
          // update. Grow flags as in attn_ot_kernel, the set chosen by the
          // CTA's key-tile count (the epilogues between segments are named
          // barriers of all eight warps too, so a set is read by every warp
          // before it is written again).
          volatile int* gw = grow_w + (gj & 1) * 8;
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
            asm volatile("bar.sync 1, 256;" ::: "memory");
          }
        }
#pragma unroll
        for (int c = 0; c < 12; ++c) store_p(c);
        exp_chunk(3);
#pragma unroll
        for (int c = 12; c < 16; ++c) store_p(c);
        {
          const float2 sv = f2_split(fadd2(sum2, sum2p));
          lsum = sv.x + sv.y;
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        l = l * alpha + lsum;
        m_used = m_new;
      }
      if (ok) ok = mbar_wait(o_done, k & 1, abort_flag);
      tc_fence_after();
      if (sg.slot >= 0) {
        // Partial: O (32 queries of head dim d per load, one 128-byte line
        // per query and warp) straight to the CTA's slot, then m and l of
        // row q; the last of the item's segments to arrive merges.
        float* base = ot_part(p, sc.c, sg.slot);
        if (active) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_base + 256 + t * 128 + c * 32, o);
            tmem_wait_ld();
            float* dst = base + (t * 128 + c * 32) * 128 + d;
#pragma unroll
            for (int i = 0; i < 32; ++i) dst[i * 128] = o[i];
          }
          base[128 * 256 + q] = ok ? m_used : -INFINITY;
          base[128 * 256 + 256 + q] = ok ? l : 0.f;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free);
        int c0, ns;
        ot_item_ctas(sc, sg.item - sc.dp, c0, ns);
        __threadfence();
        asm volatile("bar.sync 2, 256;" ::: "memory");
        if (threadIdx.x == 0) *last_seg = atomicAdd(p.kv_count + sg.item, 1) == ns - 1;
        asm volatile("bar.sync 2, 256;" ::: "memory");
        if (*last_seg) {
          __threadfence();
          ot_merge(p, sc, sg.item, q0, b, h);
          if (threadIdx.x == 0) p.kv_count[sg.item] = 0;   // ready for the next launch
        }
        asm volatile("bar.sync 2, 256;" ::: "memory");     // every thread read last_seg
      } else {
        // Whole item: O^T slab (head dims [32 wq, +32), queries of tile t)
        // through the P buffer (free: the segment's updates are done) to
        // row-major output.
        __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem + L::P_OFF);   // [256][128] bf16
        row_f[q] = (ok && !*abort_flag && l > 0.f) ? 1.f / l : 0.f;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (active) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_base + 256 + t * 128 + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int qq = t * 128 + c * 32 + i;
              stage[qq * 128 + d] = __float2bfloat16_rn(o[i] * row_f[qq]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free);
        asm volatile("bar.sync 1, 256;" ::: "memory");
        // Row-major copy out: 256 rows x 256 bytes, 16 bytes per thread step.
        for (int i = threadIdx.x; i < 256 * 16; i += 256) {
          const int rr = i >> 4, ch = i & 15;
          if (q0 + rr < p.q_rows)
            *reinterpret_cast<uint4*>(p.out + (static_cast<long long>(b) * p.q_rows + q0 + rr) * p.ldo + h * 128 +
                                      ch * 8) = reinterpret_cast<const uint4*>(stage + rr * 128)[ch];
        }
        // The P buffer and row_f are written again by the next segment.
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
      g += n;
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
