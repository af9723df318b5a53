// Two-CTA (cta_group::2) variant of the tcgen05 GEMM for large M:
// a cluster of 2 CTAs computes a 256 x BN output tile (BN 256 or 192) with
// M=256 tcgen05.mma instructions issued by the leader CTA. Each CTA loads
// its own 128 rows of A and its own BN / 2 of the tile's BN weight rows, so
// a CTA moves 32 KB (BN 256) or 28 KB (BN 192) per 64-wide k-block instead
// of 48 / 40 KB for a 128 x BN tile on one SM: the shared weight tile
// crosses the L2 -> SM path once per pair.
//
// Barriers (per CTA):
//   full[s]    leader only: one arrive_expect_tx (both CTAs' bytes); both
//              CTAs' TMA loads complete_tx on the leader's barrier
//   empty[s]   both CTAs: one arrival from the leader's commit (sent to both)
//   tfull[a]   both CTAs: one arrival from the leader's commit (sent to both)
//   tempty[a]  leader only: 16 arrivals, one per epilogue warp of either CTA
//   bye        exit handshake: the other CTA arrives once (remote arrive)
// TMEM: 2 accumulators x BN columns per CTA (rows 0-127 of the tile in the
// leader's TMEM, rows 128-255 in the peer's).
//
// Stream-K (GemmParams::sk_tiles): the first tiles run as before, one tile
// per pair per round, in the wave order that keeps few weight column blocks
// in flight (A and those weights stay in L2). The tiles x k-blocks units of
// the last sk_tiles tiles (the partly filled last round, plus the full
// round before it when the last one is less than half filled, so that a
// tile is shared by two or three pairs, not dozens) are cut into one equal
// contiguous share per pair. A pair walks its share from the highest unit
// down, in segments cut at tile boundaries. A segment without the tile's
// last k-block is a producer: its fp32 partial goes to the pair's slot of
// sk_part and each epilogue warp raises its flag. The segment holding the
// last k-block (and not the first) finishes the tile: while its own MMAs
// run, its epilogue warps sum the lower pairs' partials (in a fixed order)
// into the pair's other TMEM accumulator, free by then, and the epilogue
// adds that sum to the tile's accumulator; they clear the flags they read.
// Walking down puts a pair's producer segment first and its finisher
// segment last, and the finisher of a tile is the highest pair on it, so
// partials are ready when they are needed and no pair waits on a pair that
// starts after it.
#pragma once
#include "gemm.cuh"

namespace wamb {

constexpr int GEMM2_STAGES = 6;

template <int BN>
struct Gemm2Smem {
  static_assert(BN == 256 || BN == 192, "two-CTA tiles are 256 or 192 columns wide");
  static constexpr uint32_t A_BYTES = 128 * 128;        // this CTA's 128 rows of A x 128 bytes of K
  static constexpr uint32_t B_BYTES = (BN / 2) * 128;   // this CTA's BN / 2 of BN weight rows
  static constexpr uint32_t BAR_OFF = GEMM2_STAGES * (A_BYTES + B_BYTES);
  static constexpr uint32_t NBARS = 2 * GEMM2_STAGES + 6;
  // Epilogue staging (gemm_epilogue_tile_staged): 4 KB per epilogue warp.
  // After the barriers: the TMEM address, the abort flag, then the pair's
  // stream-K segment table (SegTable, 64 bytes).
  static constexpr uint32_t TAB_OFF = BAR_OFF + NBARS * 8 + 16;
  static constexpr uint32_t STAGE_OFF = (TAB_OFF + 64 + 15) & ~15u;
  static constexpr uint32_t TOTAL = 1024 + STAGE_OFF + GEMM_EPI_WARPS * 4096;
  static_assert(TOTAL <= 232448, "2-CTA GEMM shared memory exceeds 227 KB");
};

WAMB_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// TMA load into this CTA's shared memory that completes on the mbarrier at
// `bar_cluster` (the leader CTA's full barrier).
WAMB_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                               int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
WAMB_DEV void umma2_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
WAMB_DEV void umma2_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at this offset in both CTAs of the pair when
// all previously issued tcgen05 ops of this thread complete.
WAMB_DEV void umma2_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Same, arriving only on this CTA's barrier (every tcgen05 op of a kernel
// uses one cta_group, so the teardown drain needs the ::2 form too).
WAMB_DEV void umma2_commit_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// One output tile's k-block range processed by a pair.
struct Seg {
  int t, kb0, kb1;
  bool producer, finisher;
};

// The pair's stream-K segments (at most three: a share is less than two
// tiles of k-blocks), computed once per CTA by thread 0 into shared memory
// so that the roles carry only a tile and a table index through their loops.
// Share of pair q: units [q U / npairs, (q + 1) U / npairs) of the last
// sk_tiles tiles (tile-major, counted from dp_end), walked in descending
// order and cut at tile boundaries. 32-bit: sk_tiles < 2 x pairs (<= 256),
// so U and q * U stay far below 2^31 for any K up to 2^20.
struct SegTable {
  int n;          // segments
  int dp_end;     // tiles below it run whole, one per pair per round
  int t[3], kb0[3], kb1[3];
  int q_lo[3];    // producer pairs [q_lo, pair) of a finisher segment; pair otherwise
};
static_assert(sizeof(SegTable) <= 64, "segment table exceeds its shared-memory slot");

WAMB_DEV void sk_table_build(SegTable& tb, int sk_tiles, int pair, int npairs, int num_tiles, int num_kb) {
  tb.n = 0;
  tb.dp_end = num_tiles - sk_tiles;
  const int U = sk_tiles * num_kb;
  const int lo = pair * U / npairs;
  for (int i = (pair + 1) * U / npairs - 1; i >= lo && tb.n < 3;) {
    const int tt = i / num_kb, base = tt * num_kb;
    const int seg_lo = lo > base ? lo : base;
    const int k = tb.n++;
    tb.t[k] = tb.dp_end + tt;
    tb.kb0[k] = seg_lo - base;
    tb.kb1[k] = i + 1 - base;
    int q_lo = pair;
    if (tb.kb1[k] == num_kb && tb.kb0[k] != 0)   // finisher: the lower pairs on this tile
      for (int qq = pair - 1; qq >= 0 && (qq + 1) * U / npairs > base; --qq) q_lo = qq;
    tb.q_lo[k] = q_lo;
    i = seg_lo - 1;
  }
}

// Segment s of the pair: whole tiles first, then the table's entries.
struct SegCursor {
  int t, k;
  WAMB_DEV bool next(const SegTable& tb, int npairs, int num_kb, Seg& s, int& q_lo) {
    if (t < tb.dp_end) {
      s = Seg{t, 0, num_kb, false, false};
      q_lo = -1;
      t += npairs;
      return true;
    }
    if (k >= tb.n) return false;
    s.t = tb.t[k];
    s.kb0 = tb.kb0[k];
    s.kb1 = tb.kb1[k];
    s.producer = s.kb1 != num_kb;
    s.finisher = !s.producer && s.kb0 != 0;
    q_lo = tb.q_lo[k];
    ++k;
    return true;
  }
};

WAMB_DEV void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
WAMB_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait of a warp for a stream-K partial's flag: lane 0 polls with
// a growing sleep (hundreds of finisher warps must not flood L2 with
// acquire loads while the producers' MMAs still run), then every lane
// acquires the flag itself, so that its own loads of the partial are
// ordered after the producer's stores. Returns false on abort / timeout.
WAMB_DEV bool sk_wait_flag(const int* f, volatile int* abort_flag) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) {
    const uint64_t t0 = globaltimer();
    uint32_t ns = 64;
    while (ld_acquire_gpu(f) == 0) {
      if (*abort_flag) { ok = false; break; }
      if (globaltimer() - t0 > WAMB_WAIT_TIMEOUT_NS) {
        *abort_flag = 1;
        record_error(1);
        ok = false;
        break;
      }
      __nanosleep(ns);
      ns = ns < 1024 ? 2 * ns : ns;
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)ld_acquire_gpu(f);
  return ok;
}

// Stream-K (sk_tiles > 0) is used with BN 256 only: the partial slots and
// their layout hold 256 x 256 tiles.
template <bool F8, int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                    const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                    const GemmParams p) {
  using L = Gemm2Smem<BN>;
  constexpr int STAGES = GEMM2_STAGES;
  constexpr int NCH = BN / 64;   // 32-column chunks per epilogue warp (two warps per lane quarter)
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
  const uint32_t bye = drain + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  SegTable& segtab = *reinterpret_cast<SegTable*>(smem + L::TAB_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (p.M + 255) / 256;
  const int num_n = p.N / BN;
  const int num_tiles = num_m * num_n;
  constexpr int KB = F8 ? GEMM_BK8 : GEMM_BK;
  const int num_kb = p.K / KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 2 * GEMM_EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(bye, 1);
    *abort_flag = 0;
    sk_table_build(segtab, p.sk_tiles, blockIdx.x >> 1, gridDim.x >> 1, ((p.M + 255) / 256) * (p.N / BN),
                   p.K / (F8 ? GEMM_BK8 : GEMM_BK));
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB0);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  // Both CTAs' barriers and TMEM exist before any cross-CTA signal.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();   // inputs of the previous kernel are complete from here on
  if (p.trigger_after) pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      int it = 0;
      SegCursor cur{pair, 0};
      Seg sg;
      int q_unused;
      while (!*abort_flag && cur.next(segtab, npairs, num_kb, sg, q_unused)) {
        const int t = sg.t;
        const int m_blk = t % num_m, n_blk = t / num_m;
        const int n0 = n_blk * BN;
        const int g = n0 / p.n_per_group;
        const int n_local = n0 - g * p.n_per_group;
        const CUtensorMap* mb = g == 0 ? &tmB0 : (g == 1 ? &tmB1 : &tmB2);
        bool ok = true;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag)) { ok = false; break; }
          const uint32_t full_leader = map_to_rank(full0 + 8 * s, 0);
          if (leader) mbar_arrive_expect_tx(full0 + 8 * s, 2 * (L::A_BYTES + L::B_BYTES));
          tma_load_2d_pair(smem_u32(sA + s * L::A_BYTES), &tmA, full_leader, kb * KB,
                           m_blk * 256 + rank * 128);
          tma_load_2d_pair(smem_u32(sB + s * L::B_BYTES), mb, full_leader, kb * KB,
                           n_local + rank * (BN / 2));
        }
        if (!ok) break;
      }
      // Teardown: this CTA's last loads must land before it may exit (their
      // completion is counted on the leader's barrier, so wait on the
      // consumer side instead: the final empty arrivals).
      for (int s = 0; s < STAGES; ++s) {
        if (it > s) {
          const int last = s + ((it - 1 - s) / STAGES) * STAGES;
          mbar_wait_teardown(empty0 + 8 * s, (last / STAGES) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // --------------------------------------------------- MMA issuer (leader)
      constexpr uint32_t IDESC = F8 ? idesc_e4m3(256, BN) : idesc_bf16(256, BN, 0);
      int it = 0, tc = 0;
      SegCursor cur{pair, 0};
      Seg sg;
      int q_unused;
      for (; cur.next(segtab, npairs, num_kb, sg, q_unused); ++tc) {
        const int acc = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait(tempty0 + 8 * acc, aph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
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
            const uint32_t accum = kb > sg.kb0 || kk > 0;
            if constexpr (F8) umma2_e4m3(d_tmem, ad, bd, IDESC, accum);
            else umma2_bf16(d_tmem, ad, bd, IDESC, accum);
          }
          umma2_commit_both(empty0 + 8 * s);
        }
        if (!ok) break;
        umma2_commit_both(tfull0 + 8 * acc);
      }
      // Teardown: all MMAs issued by this thread must finish before TMEM is freed.
      umma2_commit_local(drain);
      mbar_wait_teardown(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter accessible to this warp
    const int half = (warp - 2) >> 2;  // columns [half * BN / 2, + BN / 2)
    const int c0 = half * NCH, nch = NCH;
    const int row_in_tile = static_cast<int>(rank) * 128 + q * 32 + lane;
    const uint32_t tempty_leader0 = map_to_rank(tempty0, 0);
    // Every tile's epilogue goes through the warp's staging buffer.
    const uint32_t stage = smem_u32(smem + L::STAGE_OFF + (warp - 2) * 4096);
    // Stream-K: this warp's partial rows / chunks in a pair's slot, and its flag.
    const int wslot = static_cast<int>(rank) * 8 + (warp - 2);
    // Layout [slot][chunk][4-column group j][256 rows][4]: for a fixed j the
    // lanes (consecutive rows) of a warp touch one contiguous 512-byte run.
    auto part_at = [&](int slot, int c, int j) {
      return reinterpret_cast<float4*>(p.sk_part) + ((static_cast<size_t>(slot) * 8 + c) * 8 + j) * 256 + row_in_tile;
    };
    int tc = 0;
    SegCursor cur{pair, 0};
    Seg sg;
    int q_lo;
    for (; cur.next(segtab, npairs, num_kb, sg, q_lo); ++tc) {
      const int t = sg.t;
      const int acc = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      const int m_blk = t % num_m, n_blk = t / num_m;
      const int row = m_blk * 256 + row_in_tile;
      const int n0 = n_blk * BN;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      bool ok;
      if (sg.producer) {
        // This pair's partial of the tile into its slot, then the flag.
        ok = mbar_wait(tfull0 + 8 * acc, aph, abort_flag);
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c = c0; c < c0 + nch; ++c) {
            float v[32];
            tmem_ld32(taddr + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) *part_at(pair, c, j) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
          __threadfence();
          __syncwarp();
          if (lane == 0) st_release_gpu(p.sk_flags + pair * 16 + wslot, 1);
        }
      } else {
        // Finisher: the lower pairs [q_lo, pair) hold the tile's other
        // k-blocks (q_lo = pair: none; whole tiles: -1, none).
        if (q_lo < 0) q_lo = pair;
        // The producers' partials, summed in a fixed order (highest pair
        // first), into the other accumulator of this warp's TMEM slice (the
        // finisher segment is the pair's last, so its epilogue is done)
        // while this segment's MMAs still run.
        const uint32_t tsum = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + (acc ^ 1) * BN;
        bool pre = true;
        for (int qq = q_lo; pre && qq < pair; ++qq) pre = sk_wait_flag(p.sk_flags + qq * 16 + wslot, abort_flag);
        if (pre && q_lo < pair) {
#pragma unroll 1
          for (int c = c0; c < c0 + nch; ++c) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
#pragma unroll 1
            for (int qq = pair - 1; qq >= q_lo; --qq) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 x = __ldcg(part_at(qq, c, j));
                v[4 * j] += x.x;
                v[4 * j + 1] += x.y;
                v[4 * j + 2] += x.z;
                v[4 * j + 3] += x.w;
              }
            }
            tmem_st32(tsum + c * 32, v);
          }
          tmem_wait_st();
        }
        bool ready = pre;
        if (pre && q_lo < pair) {
          // Once this segment's accumulator is complete, add the sum into it
          // (TMEM to TMEM), before the epilogue and its residual requests.
          ready = mbar_wait(tfull0 + 8 * acc, aph, abort_flag);
          if (ready) {
            tc_fence_after();
#pragma unroll 1
            for (int c = c0; c < c0 + nch; ++c) {
              float v[32], w[32];
              tmem_ld32(taddr + c * 32, v);
              tmem_ld32(tsum + c * 32, w);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += w[j];
              tmem_st32(taddr + c * 32, v);
            }
            tmem_wait_st();
          }
        }
        auto wait_acc = [&]() {
          if (q_lo < pair) return true;   // waited for above
          if (!mbar_wait(tfull0 + 8 * acc, aph, abort_flag)) return false;
          tc_fence_after();
          return true;
        };
        ok = ready && gemm_epilogue_tile_staged<NCH>(p, taddr, row - lane, lane, n0, c0, stage, wait_acc);
        if (ok && q_lo < pair) {
          __syncwarp();
          if (lane == 0)
            for (int qq = q_lo; qq < pair; ++qq) p.sk_flags[qq * 16 + wslot] = 0;   // consumed
        }
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_leader0 + 8 * acc);
    }
  }

  // Exit handshake: neither CTA leaves (or frees TMEM) while the other may
  // still signal its barriers or read its shared memory.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_remote(map_to_rank(bye, rank ^ 1));
    mbar_wait_teardown(bye, 0);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(512u)
                 : "memory");
  }
}

}  // namespace wamb
