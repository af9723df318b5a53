// tcgen05 flash attention (non-causal, head_dim 128, scale 1/sqrt(128)):
//   out[b, q, h, :] = softmax(Q[b, q, h] K[b, :, h]^T / sqrt(128)) V[b, :, h]
// the reference's custom_sdpa (model.py:37-40) for self and cross attention.
//
// One CTA per (128-row query tile, head, batch row); 192 threads:
//   warps 0..3  softmax: one thread per query row; S read from TMEM, P written
//               as bf16 into a 128B-swizzled SMEM tile, O rescaled in TMEM,
//               final O / l written to global memory
//   warp 4      TMA producer: Q once, K and V tiles double-buffered
//   warp 5      TMEM owner + MMA issuer: S_j = Q K_j^T into one of two TMEM
//               S buffers, O += P_j V_j (V is an MN-major operand)
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384).
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

constexpr int ATT_THREADS = 192;
constexpr uint32_t ATT_TILE_BYTES = 128 * 128 * 2;  // 128 rows x 128 bf16
constexpr uint32_t ATT_ATOM = 128 * 128;            // one 64-column half: 128 rows x 128 B

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
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t K_OFF = Q_OFF + ATT_TILE_BYTES;
  static constexpr uint32_t V_OFF = K_OFF + 2 * ATT_TILE_BYTES;
  static constexpr uint32_t P_OFF = V_OFF + 2 * ATT_TILE_BYTES;
  static constexpr uint32_t BAR_OFF = P_OFF + ATT_TILE_BYTES;
  // q_full, k_full[2], v_full[2], k_empty[2], v_empty[2], s_full[2], s_empty[2],
  // p_full, pv_done, drain
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
  uint8_t* sP_ptr = smem + L::P_OFF;
  const uint32_t sP = smem_u32(sP_ptr);
  const uint32_t bar0 = smem_u32(smem + L::BAR_OFF);
  const uint32_t q_full = bar0;
  const uint32_t k_full = bar0 + 8;       // [2]
  const uint32_t v_full = bar0 + 24;      // [2]
  const uint32_t k_empty = bar0 + 40;     // [2]
  const uint32_t v_empty = bar0 + 56;     // [2]
  const uint32_t s_full = bar0 + 72;      // [2]
  const uint32_t s_empty = bar0 + 88;     // [2]
  const uint32_t p_full = bar0 + 104;
  const uint32_t pv_done = bar0 + 112;
  const uint32_t drain = bar0 + 120;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = blockIdx.x * 128;
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
      mbar_init(s_empty + 8 * i, 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      const int qrow = b * p.q_rows + q0;
      const int qcol = p.q_col + h * 128;
      mbar_arrive_expect_tx(q_full, ATT_TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, qcol, qrow);
      tma_load_2d(sQ + ATT_ATOM, &tmQ, q_full, qcol + 64, qrow);
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
  } else if (warp == 5) {
    // --------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0);
    constexpr uint32_t IDESC_O = idesc_bf16(128, 128, 1);
    bool ok = mbar_wait(q_full, 0, abort_flag);
    auto issue_s = [&](int j) -> bool {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!mbar_wait(k_full + 8 * st, ph, abort_flag)) return false;
      if (!mbar_wait(s_empty + 8 * st, ph ^ 1, abort_flag)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kb = sK + st * ATT_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * ATT_ATOM + (kk & 3) * 32;
          umma_bf16(tmem + st * 128, sw128_desc(sQ + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                    IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * st);
        umma_commit(k_empty + 8 * st);
      }
      __syncwarp();
      return true;
    };
    if (ok && n > 0) ok = issue_s(0);
    for (int j = 0; ok && j < n; ++j) {
      if (j + 1 < n && !issue_s(j + 1)) break;
      const int st = j & 1;
      if (!mbar_wait(p_full, j & 1, abort_flag)) break;
      if (!mbar_wait(v_full + 8 * st, (j >> 1) & 1, abort_flag)) break;
      const KvTile t = att_tile(p, j, n0, b);
      const int ksteps = (t.len + 15) >> 4;
      if (t.len & 15) {
        // Zero V rows [len, 16*ksteps) in both 64-column halves.
        uint8_t* vt = smem + L::V_OFF + st * ATT_TILE_BYTES;
        const int r0 = t.len, r1 = ksteps * 16;
        for (int i = lane; i < (r1 - r0) * 16; i += 32) {
          const int r = r0 + (i >> 4), c = i & 15;
          uint8_t* dst = vt + (c >> 3) * ATT_ATOM + r * 128 + (c & 7) * 16;
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vb = sV + st * ATT_TILE_BYTES;
        for (int kk = 0; kk < ksteps; ++kk) {
          const uint32_t poff = (kk >> 2) * ATT_ATOM + (kk & 3) * 32;
          umma_bf16(tmem + 256, sw128_desc(sP + poff, 16, 1024),
                    sw128_desc(vb + kk * 2048, ATT_ATOM, 1024), IDESC_O, (j > 0 || kk > 0));
        }
        umma_commit(pv_done);
        umma_commit(v_empty + 8 * st);
      }
      __syncwarp();
    }
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait_teardown(drain, 0);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------- softmax / epilogue
    const int r = warp * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(s_full + 8 * sb, (j >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t32[32];
        tmem_ld32(tmem + lane_base + sb * 128 + c * 32, t32);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t32[i];
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_empty + 8 * sb);
      const int len = att_tile(p, j, n0, b).len;
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        if (i >= len) s[i] = -INFINITY;
        mx = fmaxf(mx, s[i]);
      }
      const float m_new = fmaxf(m, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f((m - m_use) * p.scale_log2);
      const float bias = -m_use * p.scale_log2;
      float rs = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        s[i] = exp2f(fmaf(s[i], p.scale_log2, bias));
        rs += s[i];
      }
      if (j > 0) {
        if (!mbar_wait(pv_done, (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
      }
      // P row -> swizzled K-major SMEM tile (two 64-key halves).
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 w;
        w.x = pack_bf16(s[8 * c + 0], s[8 * c + 1]);
        w.y = pack_bf16(s[8 * c + 2], s[8 * c + 3]);
        w.z = pack_bf16(s[8 * c + 4], s[8 * c + 5]);
        w.w = pack_bf16(s[8 * c + 6], s[8 * c + 7]);
        uint8_t* dst = sP_ptr + (c >> 3) * ATT_ATOM + r * 128 + (((c & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = w;
      }
      fence_proxy_async();
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_base + 256 + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tmem + lane_base + 256 + c * 32, o);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(p_full);
      l = l * alpha + rs;
      m = m_new;
    }
    if (ok && n > 0) ok = mbar_wait(pv_done, (n - 1) & 1, abort_flag);
    tc_fence_after();
    const int qr = q0 + r;
    const bool store = qr < p.q_rows;
    __nv_bfloat16* orow = p.out + (static_cast<long long>(b) * p.q_rows + qr) * p.ldo + h * 128;
    const float inv = (ok && n > 0 && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float o[32];
      tmem_ld32(tmem + lane_base + 256 + c * 32, o);
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

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wamb
