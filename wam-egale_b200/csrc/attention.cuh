// tcgen05 flash attention (non-causal, head_dim 128, scale 1/sqrt(128)):
//   out[b, q, h, :] = softmax(Q[b, q, h] K[b, :, h]^T / sqrt(128)) V[b, :, h]
// the reference's custom_sdpa (model.py:37-40) for self and cross attention.
//
// One CTA per (256 query rows = two 128-row tiles A and B, head, batch row);
// both tiles share every K/V tile that is loaded. 320 threads:
//   warps 0..3  softmax of tile A, warps 4..7 softmax of tile B: one thread
//               per query row; S read from TMEM, P written back to TMEM as
//               packed bf16 over the S columns, O rescaled in TMEM only when
//               the row max grows by more than 2^8 (the final O / l uses the
//               same stale max, so the result is exact)
//   warp 8      TMA producer: Q once, K and V tiles double-buffered
//   warp 9      TMEM owner + MMA issuer, in the order
//               PV_A(j), S_A(j+1), PV_B(j), S_B(j+1): while one tile's
//               softmax runs the tensor core works on the other tile.
//               S = Q K^T reads both operands from SMEM; O += P V reads P
//               from TMEM and V from SMEM as an MN-major operand.
// TMEM columns: S/P of A [0,128), S/P of B [128,256), O_A [256,384), O_B [384,512).
// SMEM: Q_A, Q_B, K x2, V x2 tiles of 128 rows x 128 bf16 (192 KB).
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
constexpr uint32_t ATT_TILE_BYTES = 128 * 128 * 2;  // 128 rows x 128 bf16
constexpr uint32_t ATT_ATOM = 128 * 128;            // one 64-column half: 128 rows x 128 B
constexpr float ATT_RESCALE_LOG2 = 8.f;             // rescale O only when the max grows > 2^8

struct AttnParams {
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
};

struct AttnSmem {
  static constexpr uint32_t Q_OFF = 0;                               // Q_A, Q_B
  static constexpr uint32_t K_OFF = Q_OFF + 2 * ATT_TILE_BYTES;      // K x2
  static constexpr uint32_t V_OFF = K_OFF + 2 * ATT_TILE_BYTES;      // V x2
  static constexpr uint32_t BAR_OFF = V_OFF + 2 * ATT_TILE_BYTES;
  // q_full, k_full[2], v_full[2], k_empty[2], v_empty[2], s_full[2], p_full[2], o_done, drain
  static constexpr uint32_t NBARS = 16;
  static constexpr uint32_t TOTAL = 1024 + BAR_OFF + NBARS * 8 + 16;
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

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                   const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                   const __grid_constant__ CUtensorMap tmV1, const AttnParams p) {
  using L = AttnSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sQ = smem_u32(smem + L::Q_OFF);
  const uint32_t sK = smem_u32(smem + L::K_OFF);
  const uint32_t sV = smem_u32(smem + L::V_OFF);
  const uint32_t bar0 = smem_u32(smem + L::BAR_OFF);
  const uint32_t q_full = bar0;
  const uint32_t k_full = bar0 + 8;       // [2] by stage
  const uint32_t v_full = bar0 + 24;      // [2]
  const uint32_t k_empty = bar0 + 40;     // [2]
  const uint32_t v_empty = bar0 + 56;     // [2]
  const uint32_t s_full = bar0 + 72;      // [2] by query tile
  const uint32_t p_full = bar0 + 88;      // [2] by query tile
  const uint32_t o_done = bar0 + 104;
  const uint32_t drain = bar0 + 112;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = blockIdx.x * 256;
  const bool has_b = q0 + 128 < p.q_rows;   // the second query tile holds rows
  const int n0 = p.tiles != nullptr ? *p.n_tiles : (p.src0_len + 127) / 128;
  const int n1 = p.has_src1 ? (p.q_rows + 127) / 128 : 0;
  const int n = n0 + n1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full + 8 * i, 1);
      mbar_init(v_full + 8 * i, 1);
      mbar_init(k_empty + 8 * i, 1);
      mbar_init(v_empty + 8 * i, 1);
      mbar_init(s_full + 8 * i, 1);
      mbar_init(p_full + 8 * i, 128);
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      const int qrow = b * p.q_rows + q0;
      const int qcol = p.q_col + h * 128;
      mbar_arrive_expect_tx(q_full, (has_b ? 2 : 1) * ATT_TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, qcol, qrow);
      tma_load_2d(sQ + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow);
      if (has_b) {
        tma_load_2d(sQ + ATT_TILE_BYTES, &tmQ, q_full, qcol, qrow + 128);
        tma_load_2d(sQ + ATT_TILE_BYTES + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow + 128);
      }
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const KvTile t = att_tile(p, j, n0, b);
        const CUtensorMap* mk = t.src ? &tmK1 : &tmK0;
        const CUtensorMap* mv = t.src ? &tmV1 : &tmV0;
        const int kc = (t.src ? p.k1_col : p.k0_col) + h * 128;
        const int vc = (t.src ? p.v1_col : p.v0_col) + h * 128;
        if (!mbar_wait(k_empty + 8 * st, ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(k_full + 8 * st, ATT_TILE_BYTES);
        tma_load_2d(sK + st * ATT_TILE_BYTES, mk, k_full + 8 * st, kc, t.row);
        tma_load_2d(sK + st * ATT_TILE_BYTES + ATT_ATOM, mk, k_full + 8 * st, kc + 64, t.row);
        if (!mbar_wait(v_empty + 8 * st, ph ^ 1, abort_flag)) { issued = 2 * j + 1; break; }
        mbar_arrive_expect_tx(v_full + 8 * st, ATT_TILE_BYTES);
        tma_load_2d(sV + st * ATT_TILE_BYTES, mv, v_full + 8 * st, vc, t.row);
        tma_load_2d(sV + st * ATT_TILE_BYTES + ATT_ATOM, mv, v_full + 8 * st, vc + 64, t.row);
        issued = 2 * j + 2;
      }
      // Teardown: loads still in flight must land before the CTA exits.
      mbar_wait_teardown(q_full, 0);
      for (int i = issued - 1; i >= 0 && i >= issued - 4; --i) {
        const int j = i >> 1;
        const uint32_t bar = (i & 1) ? v_full + 8 * (j & 1) : k_full + 8 * (j & 1);
        mbar_wait_teardown(bar, (j >> 1) & 1);
      }
    }
  } else if (warp == 9) {
    // --------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0);
    constexpr uint32_t IDESC_O = idesc_bf16(128, 128, 1);
    const int ntq = has_b ? 2 : 1;
    // S_t = Q_t K^T (stage st) into TMEM columns [t*128, t*128+128).
    auto issue_s = [&](int t, int st) {
      if (lane == 0) {
        const uint32_t qb = sQ + t * ATT_TILE_BYTES;
        const uint32_t kb = sK + st * ATT_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * ATT_ATOM + (kk & 3) * 32;
          umma_bf16(tmem + t * 128, sw128_desc(qb + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                    IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * t);
      }
    };
    // O_t += P_t V (stage st); P_t is packed bf16 in TMEM columns [t*128, t*128+64).
    auto issue_pv = [&](int t, int st, int ksteps, bool acc) {
      if (lane == 0) {
        const uint32_t vb = sV + st * ATT_TILE_BYTES;
        for (int kk = 0; kk < ksteps; ++kk)
          umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                       sw128_desc(vb + kk * 2048, ATT_ATOM, 1024), IDESC_O, acc || kk > 0);
      }
    };
    bool ok = mbar_wait(q_full, 0, abort_flag);
    if (ok && n > 0) {
      ok = mbar_wait(k_full, 0, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < ntq; ++t) issue_s(t, 0);
        if (lane == 0) umma_commit(k_empty);
      }
      __syncwarp();
    }
    for (int j = 0; ok && j < n; ++j) {
      const int st = j & 1;
      const KvTile tl = att_tile(p, j, n0, b);
      const int ksteps = (tl.len + 15) >> 4;
      if (!mbar_wait(v_full + 8 * st, (j >> 1) & 1, abort_flag)) break;
      if (tl.len & 15) {
        // Zero V rows [len, 16*ksteps) in both 64-column halves.
        uint8_t* vt = smem + L::V_OFF + st * ATT_TILE_BYTES;
        const int r0 = tl.len, r1 = ksteps * 16;
        for (int i = lane; i < (r1 - r0) * 16; i += 32) {
          const int r = r0 + (i >> 4), c = i & 15;
          uint8_t* dst = vt + (c >> 3) * ATT_ATOM + r * 128 + (c & 7) * 16;
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
        __syncwarp();
      }
      const bool next = j + 1 < n;
      const int nst = (j + 1) & 1;
      bool knext = false;
      for (int t = 0; t < ntq; ++t) {
        if (!mbar_wait(p_full + 8 * t, j & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        issue_pv(t, st, ksteps, j > 0);
        if (t == ntq - 1 && lane == 0) umma_commit(v_empty + 8 * st);
        if (next) {
          if (!knext) {
            if (!mbar_wait(k_full + 8 * nst, ((j + 1) >> 1) & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            knext = true;
          }
          issue_s(t, nst);
        }
        __syncwarp();
      }
      if (ok && next && lane == 0) umma_commit(k_empty + 8 * nst);
      __syncwarp();
    }
    if (lane == 0) {
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
    const uint32_t s_col = t * 128, o_col = 256 + t * 128;
    float m_used = -INFINITY, l = 0.f;  // running max (scaled log2 units) and row sum
    bool ok = t == 0 || has_b;
    for (int j = 0; ok && j < n; ++j) {
      if (!mbar_wait(s_full + 8 * t, j & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t32[32];
        tmem_ld32(tmem + lane_base + s_col + c * 32, t32);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t32[i];
      }
      tmem_wait_ld();
      const int len = att_tile(p, j, n0, b).len;
      if (len < 128) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= len) s[i] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) mx = fmaxf(mx, s[i]);
      mx *= p.scale_log2;
      // Keep the stale max unless the new one exceeds it by more than 2^8.
      const bool grow = mx > m_used + ATT_RESCALE_LOG2;
      const float m_new = grow ? mx : m_used;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = grow ? exp2f(m_used - m_use) : 1.f;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = exp2f(fmaf(s[c * 64 + 2 * i], p.scale_log2, -m_use));
          const float bb = exp2f(fmaf(s[c * 64 + 2 * i + 1], p.scale_log2, -m_use));
          rs += a + bb;
          pk[i] = pack_bf16(a, bb);
        }
        tmem_st32u(tmem + lane_base + s_col + c * 32, pk);
      }
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O_t is stable: S_t(j) was issued after PV_t(j-1) and has completed.
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_base + o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tmem + lane_base + o_col + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full + 8 * t);
      l = l * alpha + rs;
      m_used = m_new;
    }
    if (t == 0 || has_b) {
      if (ok && n > 0) ok = mbar_wait(o_done, 0, abort_flag);
      tc_fence_after();
      const int qr = q0 + t * 128 + r;
      const bool store = qr < p.q_rows;
      __nv_bfloat16* orow = p.out + (static_cast<long long>(b) * p.q_rows + qr) * p.ldo + h * 128;
      const float inv = (ok && n > 0 && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + o_col + c * 32, o);
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

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wamb
