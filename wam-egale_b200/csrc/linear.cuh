// Host launcher of the tcgen05 GEMM (gemm.cuh): tile-width choice, tensor
// maps, argument checks.
#pragma once
#include "gemm.cuh"
#include "gemm2.cuh"
#include "host.cuh"

#include <algorithm>

namespace wamb {

template <int BN, int STAGES, bool F8>
inline int launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap* tb, const GemmParams& p,
                          int sms, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  static bool configured[64] = {};
  int dev = 0;
  WAMB_CHECK_CUDA(cudaGetDevice(&dev));
  if (!configured[dev]) {
    WAMB_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES, F8, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    configured[dev] = true;
  }
  const int tiles = ((p.M + GEMM_BM - 1) / GEMM_BM) * (p.N / BN) * (p.splits > 1 ? p.splits : 1);
  const int grid = tiles < sms ? tiles : sms;
  return launch_kernel(gemm_tc_kernel<BN, STAGES, F8, false>, dim3(grid), dim3(GEMM_THREADS), L::TOTAL, stream,
                       ta, tb[0], tb[1], tb[2], p);
}

// Cluster split-K launch configuration: p.splits CTAs per cluster, one
// cluster per output tile.
template <int BN, int STAGES, bool F8>
inline cudaLaunchConfig_t cluster_config(int splits, int grid, cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = GemmSmem<BN, STAGES>::TOTAL;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Clusters of `splits` CTAs of the cluster split-K kernel that fit on the
// device at once (1 CTA per SM; the clusters of a GPC must fit its SMs).
// Queried once per device and size.
template <int BN, int STAGES, bool F8>
inline int cluster_capacity(int splits, int sms) {
  static int cap[64][9] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || splits < 2 || splits > 8) return 0;
  if (cap[dev][splits] == 0) {
    int n = 0;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = cluster_config<BN, STAGES, F8>(splits, splits * (sms / splits), nullptr, attr);
    if (cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES, F8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmSmem<BN, STAGES>::TOTAL) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, STAGES, F8, true>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    cap[dev][splits] = n > 0 ? n : -1;
  }
  return cap[dev][splits] > 0 ? cap[dev][splits] : 0;
}

template <int BN, int STAGES, bool F8>
inline int launch_gemm_cl(const CUtensorMap& ta, const CUtensorMap* tb, const GemmParams& p,
                          cudaStream_t stream) {
  const int grid = ((p.M + GEMM_BM - 1) / GEMM_BM) * (p.N / BN) * p.splits;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = cluster_config<BN, STAGES, F8>(p.splits, grid, stream, attr);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  WAMB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, STAGES, F8, true>, ta, tb[0], tb[1], tb[2], p));
  return WAMB_OK;
}

// Two-CTA launch: clusters of 2 along x, one cluster per pair of SMs.
template <int BN>
inline cudaLaunchConfig_t gemm2_config(cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = Gemm2Smem<BN>::TOTAL;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Co-resident clusters (SM pairs) of the two-CTA kernel on the current
// device (queried once per device; 74 on B200). It is also the number of
// stream-K partial slots a launch needs.
template <bool F8, int BN = 256>
inline int gemm2_resident(int sms) {
  static int resident[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (resident[dev] == 0) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = gemm2_config<BN>(nullptr, attr);
    cfg.gridDim = dim3(sms, 1, 1);
    int n = 0;
    if (cudaFuncSetAttribute(gemm_tc2_kernel<F8, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Gemm2Smem<BN>::TOTAL) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<F8, BN>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    resident[dev] = n > 0 ? n : -1;
  }
  return resident[dev] > 0 ? resident[dev] : 0;
}

// Stream-K scratch: one flag per epilogue warp of each pair (zero between
// launches), then one 256 x 256 fp32 partial per pair.
constexpr size_t SK_FLAG_BYTES = 128 * 16 * 4;    // up to 128 pairs
constexpr size_t SK_SLOT_BYTES = 256 * 256 * 4;
inline size_t sk_part_bytes(int sms) {
  const int r = std::max(gemm2_resident<false>(sms), gemm2_resident<true>(sms));
  return static_cast<size_t>(r > 0 ? r : sms / 2) * SK_SLOT_BYTES;
}

struct SkBuffers {
  int* flags = nullptr;     // SK_FLAG_BYTES, zero
  float* part = nullptr;    // sk_part_bytes()
  size_t part_bytes = 0;
};

template <bool F8, int BN>
inline int launch_gemm2(const CUtensorMap& ta, const CUtensorMap* tb, const GemmParams& p, int sms,
                        cudaStream_t stream) {
  const int resident = gemm2_resident<F8, BN>(sms);
  WAMB_REQUIRE(resident > 0, WAMB_ERR_CUDA, "two-CTA GEMM cannot be resident on this device");
  WAMB_REQUIRE(!p.sk_tiles || (BN == 256 && resident <= 128), WAMB_ERR_CUDA,
               "stream-K needs 256-column tiles and at most 128 SM pairs");
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = gemm2_config<BN>(stream, attr);
  const int tiles = ((p.M + 255) / 256) * (p.N / BN);
  // Stream-K shares the last round over every resident pair (one partial slot each).
  const int pairs = p.sk_tiles ? resident : (tiles < resident ? tiles : resident);
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  WAMB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<F8, BN>, ta, tb[0], tb[1], tb[2], p));
  return WAMB_OK;
}

// Tile plan of the one-CTA kernel: tile width (256/192/128/64 columns) and
// cluster split-K factor, from a cost model measured on B200 at small M:
//   * the TMA ring of one SM ingests ~90 GB/s of A + weight tiles while
//     the MMAs consume them, and each k-block moves (128 + BN) x 128 bytes,
//     so narrow tiles spend most of an SM's ingest on re-reading A;
//   * the weights stream from HBM at no more than ~6 TB/s in all;
//   * an output tile's epilogue costs ~1 + BN/128 us; a split tile's
//     cluster reduction ~1.5 + BN/128 (0.7 + 2/splits) us;
//   * split plans use 64- or 128-column tiles (cluster_capacity_bn).
// Splits need all clusters co-resident (capacity queried per device), at
// least 4 k-blocks each and splits x tiles <= SMs.
struct TilePlan {
  int bn, splits, kb_per_split;
  double cost_us = 0.0;   // the cost model's estimate of the plan
};

// Split plans use 64- or 128-column tiles: a 256-column tile's fp32
// partial and receive slots do not fit its ring.
template <bool F8>
inline int cluster_capacity_bn(int bn, int splits, int sms) {
  switch (bn) {
    case 128: return cluster_capacity<128, 6, F8>(splits, sms);
    case 64: return cluster_capacity<64, 8, F8>(splits, sms);
    default: return 0;
  }
}

inline TilePlan plan_tiles(int M, int N, int n_per_group, int num_kb, int sms, bool f8) {
  constexpr double kIngestGBs = 90.0, kDramGBs = 6000.0;
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  const double t_dram = static_cast<double>(N) * num_kb * 128.0 / (kDramGBs * 1e3);   // us
  TilePlan best{0, 1, num_kb};
  double best_t = 1e300;
  const int cands[4] = {256, 192, 128, 64};
  for (int bn : cands) {
    if (n_per_group % bn) continue;
    const long long tiles = static_cast<long long>(num_m) * (N / bn);
    const double kb_us = (128.0 + bn) * 128.0 / (kIngestGBs * 1e3);   // one k-block of one SM
    const long long waves = (tiles + sms - 1) / sms;
    const double t1 = std::max(waves * num_kb * kb_us, t_dram) + 1.0 + bn / 128.0;
    if (t1 < best_t) {
      best_t = t1;
      best = TilePlan{bn, 1, num_kb};
    }
    for (int sp = 2; sp <= 8; ++sp) {
      const int kbps = (num_kb + sp - 1) / sp;
      const int eff = (num_kb + kbps - 1) / kbps;   // no empty split
      if (eff != sp || kbps < 4 || tiles * sp > sms) continue;
      const int cap = f8 ? cluster_capacity_bn<true>(bn, sp, sms) : cluster_capacity_bn<false>(bn, sp, sms);
      if (tiles > cap) continue;
      const double t = std::max(kbps * kb_us, t_dram) + 1.5 + bn / 128.0 * (0.7 + 2.0 / sp);
      if (t < best_t) {
        best_t = t;
        best = TilePlan{bn, sp, kbps};
      }
    }
  }
  best.cost_us = best_t;
  return best;
}

// Tile width of the 2-CTA kernel for a GEMM of this shape (M >= 512), or 0
// for the one-CTA kernel. Stream-K (sk: every pair gets an equal share of
// the last round) needs 256-column tiles. Otherwise 256 x 256 tiles when
// the weight groups split into them and there are enough to give every SM
// pair one, and, for the residual epilogues, 256 x 192 tiles when
// plan_tiles' cost model, applied to a pair, rates them faster than that
// choice: an SM ingests (128 + BN / 2) x 128 bytes per k-block (A rows plus
// its half of the weight rows) at ~90 GB/s, tiles run in rounds over the SM
// pairs, an epilogue costs ~1 + BN / 128 us. At M 880, N 3072 that is one
// round of 64 pair tiles, 28 KB per SM per k-block, against 112 one-CTA
// 128 x 192 tiles moving 40 KB per k-block. Measured there (CUDA events,
// weights from HBM): the gated fp32 residual 31.1 -> 28.4 us, whose reads
// the pair kernel's staged epilogue requests two chunks ahead; a bias-only
// epilogue 22.4 -> 24.8 us, so those keep the one-CTA plan.
inline int gemm_pair_bn(int M, long long N, int n_per_group, int num_kb, int sms, bool f8, int epi,
                        bool sk = false) {
  if (M < 512) return 0;
  const bool c256 = n_per_group % 256 == 0, c192 = n_per_group % 192 == 0;
  if (sk) return c256 ? 256 : 0;
  const int pairs = sms / 2;
  const double t_dram = static_cast<double>(N) * num_kb * 128.0 / (6000.0 * 1e3);   // us
  auto cost = [&](int bn) {
    const long long tiles = static_cast<long long>((M + 255) / 256) * (N / bn);
    const long long rounds = (tiles + pairs - 1) / pairs;
    return std::max(rounds * num_kb * ((128.0 + bn / 2) * 128.0 / (90.0 * 1e3)), t_dram) + 1.0 + bn / 128.0;
  };
  const long long t256 = c256 ? static_cast<long long>((M + 255) / 256) * (N / 256) : 0;
  int best = c256 && t256 >= pairs ? 256 : 0;
  const double best_t = best ? cost(256) : plan_tiles(M, static_cast<int>(N), n_per_group, num_kb, sms, f8).cost_us;
  const bool res = epi == WAMB_EPI_RES || epi == WAMB_EPI_RES_GATE;
  if (c192 && res && cost(192) < best_t) best = 192;
  return best;
}

// Tiles of a pair GEMM that stream-K shares over the pairs (0: none): the
// partly filled last round when it holds at least half as many tiles as
// there are pairs, else that round plus the full one before it (a share is
// then at least one tile of k-blocks, so that a tile is split between two or
// three pairs, not dozens); none when the tiles divide evenly, or when a
// GEMM of less than one round has too few tiles to share that way. Only for
// long K (>= 128 k-blocks, the FFN output projections): the partial
// exchange and the split tiles' second epilogue cost a launch ~6 us, which
// measured more than the idle pairs at K 3072 (M 880: O projection 24 ->
// 32 us, QKV 43 -> 52 us) and less at K 14336 (M 880: FFN2 93 -> 74 us).
constexpr int SK_MIN_KB = 128;
inline int gemm_sk_tiles(int M, long long N, int num_kb, int sms) {
  const int r = gemm2_resident<false>(sms);
  if (M < 512 || num_kb < SK_MIN_KB || r <= 0 || r > 128) return 0;
  const long long tiles = ((M + 255) / 256) * (N / 256);
  const long long rem = tiles % r, full = tiles / r;
  long long sk = 0;
  if (rem == 0) sk = 0;
  else if (2 * rem >= r) sk = rem;
  else if (full >= 1) sk = rem + r;
  return sk * num_kb >= r ? static_cast<int>(sk) : 0;
}
inline bool gemm_use_sk(int M, long long N, int num_kb, int sms) { return gemm_sk_tiles(M, N, num_kb, sms) > 0; }

// w_early: the caller guarantees that the weights were last written two or
// more kernels before this GEMM in the stream (GemmParams::w_early).
// trigger: the next kernel is a GEMM with w_early (GemmParams::trigger).
// out_gstride != 0: weight group g writes its n_per_group columns to
// out + g * out_gstride elements (separate outputs of one launch, ldo each).
// trigger_after: GemmParams::trigger_after.
// sk: stream-K scratch (flags zero on entry); null or too small: no stream-K.
inline int linear_impl(const wamb_linear_args* a, cudaStream_t stream, bool w_early = false,
                       bool trigger = false, long long out_gstride = 0, bool trigger_after = false,
                       const SkBuffers* sk = nullptr) {
  WAMB_REQUIRE(a != nullptr, WAMB_ERR_ARG, "null args");
  WAMB_REQUIRE(a->groups >= 1 && a->groups <= 3, WAMB_ERR_ARG, "groups must be 1..3");
  WAMB_REQUIRE(a->m >= 0 && a->k > 0 && a->n_per_group > 0, WAMB_ERR_SHAPE, "bad M/K/N");
  WAMB_REQUIRE(a->a_is_fp8 == 0 || a->a_is_fp8 == 1, WAMB_ERR_ARG, "a_is_fp8 must be 0 or 1");
  const bool f8 = a->a_is_fp8 == 1;
  WAMB_REQUIRE(a->k % (f8 ? GEMM_BK8 : GEMM_BK) == 0, WAMB_ERR_SHAPE, "K=%d must be a multiple of %d",
               a->k, f8 ? GEMM_BK8 : GEMM_BK);
  WAMB_REQUIRE(a->n_per_group % 64 == 0, WAMB_ERR_SHAPE, "N per group=%d must be a multiple of 64",
               a->n_per_group);
  WAMB_REQUIRE(a->lda >= a->k && a->lda % (f8 ? 16 : 8) == 0, WAMB_ERR_ALIGN, "lda");
  const long long N = static_cast<long long>(a->groups) * a->n_per_group;
  WAMB_REQUIRE(a->ldo >= (out_gstride != 0 ? a->n_per_group : N) && a->ldo % 8 == 0, WAMB_ERR_ALIGN, "ldo");
  WAMB_REQUIRE(out_gstride % 8 == 0, WAMB_ERR_ALIGN, "group output stride");
  WAMB_REQUIRE(a->out_is_f32 == 0 || a->out_is_f32 == 1, WAMB_ERR_ARG, "out_is_f32");
  WAMB_REQUIRE(a->res_is_f32 == 0 || a->res_is_f32 == 1, WAMB_ERR_ARG, "res_is_f32");
  WAMB_REQUIRE(a->a && a->out, WAMB_ERR_ARG, "null A/out");
  WAMB_REQUIRE(aligned16(a->a) && aligned16(a->out), WAMB_ERR_ALIGN, "A/out alignment");
  for (int g = 0; g < a->groups; ++g) {
    WAMB_REQUIRE(a->weight[g] && aligned16(a->weight[g]), WAMB_ERR_ARG, "weight[%d]", g);
    WAMB_REQUIRE(!a->bias[g] || aligned16(a->bias[g]), WAMB_ERR_ALIGN, "bias[%d]", g);
    if (f8)
      WAMB_REQUIRE(a->w_scale[g] && aligned16(a->w_scale[g]), WAMB_ERR_ARG, "w_scale[%d]", g);
  }
  if (f8) WAMB_REQUIRE(a->a_scale != nullptr, WAMB_ERR_ARG, "a_scale");
  WAMB_REQUIRE(a->epilogue >= 0 && a->epilogue <= 4, WAMB_ERR_ARG, "epilogue");
  if (a->epilogue == WAMB_EPI_RES || a->epilogue == WAMB_EPI_RES_GATE) {
    WAMB_REQUIRE(a->res && aligned16(a->res) && a->ldr >= N && a->ldr % 8 == 0, WAMB_ERR_ARG,
                 "residual");
  }
  if (a->epilogue == WAMB_EPI_RES_GATE) {
    WAMB_REQUIRE(a->table && a->temb && aligned16(a->table) && aligned16(a->temb), WAMB_ERR_ARG,
                 "gate tables");
    WAMB_REQUIRE(a->dim == N && a->dim % 8 == 0, WAMB_ERR_SHAPE, "gate dim must equal N");
    WAMB_REQUIRE(a->rows_per_batch > 0 && a->temb_len >= 1 &&
                     (a->temb_len == 1 || a->temb_len == a->rows_per_batch),
                 WAMB_ERR_SHAPE, "temb_len must be 1 or rows_per_batch");
    WAMB_REQUIRE(a->gate_index >= 0 && a->gate_index < 6, WAMB_ERR_ARG, "gate_index");
  }
  if (a->m == 0) return WAMB_OK;
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;

  const bool sk_ok = sk != nullptr && sk->flags != nullptr && sk->part != nullptr && a->n_per_group % 256 == 0 &&
                     sk->part_bytes >= sk_part_bytes(di.sms) &&
                     gemm_use_sk(a->m, N, a->k / (f8 ? GEMM_BK8 : GEMM_BK), di.sms);
  const int num_kb = a->k / (f8 ? GEMM_BK8 : GEMM_BK);
  const int pbn = gemm_pair_bn(a->m, N, a->n_per_group, num_kb, di.sms, f8, a->epilogue, sk_ok);
  const bool pair = pbn != 0;
  TilePlan tp{pbn, 1, num_kb};
  if (!pair) tp = plan_tiles(a->m, static_cast<int>(N), a->n_per_group, num_kb, di.sms, f8);
  const int bn = tp.bn;
  CUtensorMap ta, tb[3];
  auto tmap = f8 ? make_tmap_e4m3 : make_tmap_bf16;
  rc = tmap(&ta, a->a, a->m, a->k, a->lda, 128);
  if (rc) return rc;
  for (int g = 0; g < 3; ++g) {
    const int src = g < a->groups ? g : 0;
    rc = tmap(&tb[g], a->weight[src], a->n_per_group, a->k, a->k, pair ? pbn / 2 : bn);
    if (rc) return rc;
  }
  GemmParams p{};
  p.M = a->m;
  p.N = static_cast<int>(N);
  p.K = a->k;
  p.n_per_group = a->n_per_group;
  for (int g = 0; g < 3; ++g)
    p.bias[g] = g < a->groups ? static_cast<const __nv_bfloat16*>(a->bias[g]) : nullptr;
  p.out = a->out;
  p.ldo = a->ldo;
  p.epi = a->epilogue;
  p.res = a->res;
  p.ldr = a->ldr;
  p.res_f32 = a->res_is_f32;
  p.out_f32 = a->out_is_f32;
  p.table = a->table;
  p.temb = a->temb;
  p.temb_f32 = a->temb_is_f32;
  p.temb_L = a->temb_len;
  p.rows_per_batch = a->rows_per_batch > 0 ? a->rows_per_batch : 1;
  p.gate_idx = a->gate_index;
  p.D = a->dim;
  if (f8) {
    p.a_scale = a->a_scale;
    for (int g = 0; g < 3; ++g) p.w_scale[g] = g < a->groups ? a->w_scale[g] : nullptr;
  }
  p.w_early = w_early ? 1 : 0;
  p.trigger = trigger ? 1 : 0;
  p.splits = tp.splits;
  p.kb_per_split = tp.kb_per_split;
  p.out_gstride = out_gstride;
  p.trigger_after = trigger_after ? 1 : 0;
  if (pair && sk_ok && pbn == 256) {
    p.sk_tiles = gemm_sk_tiles(a->m, N, a->k / (f8 ? GEMM_BK8 : GEMM_BK), di.sms);
    p.sk_flags = sk->flags;
    p.sk_part = sk->part;
  }
  auto launch = [&](auto f8c) {
    constexpr bool F8 = decltype(f8c)::value;
    if (pair) return pbn == 256 ? launch_gemm2<F8, 256>(ta, tb, p, di.sms, stream)
                                : launch_gemm2<F8, 192>(ta, tb, p, di.sms, stream);
    if (tp.splits > 1) {
      if (bn == 128) return launch_gemm_cl<128, 6, F8>(ta, tb, p, stream);
      return launch_gemm_cl<64, 8, F8>(ta, tb, p, stream);
    }
    switch (bn) {
      case 256: return launch_gemm_bn<256, 4, F8>(ta, tb, p, di.sms, stream);
      case 192: return launch_gemm_bn<192, 5, F8>(ta, tb, p, di.sms, stream);
      case 128: return launch_gemm_bn<128, 6, F8>(ta, tb, p, di.sms, stream);
      default: return launch_gemm_bn<64, 8, F8>(ta, tb, p, di.sms, stream);
    }
  };
  return f8 ? launch(std::true_type{}) : launch(std::false_type{});
}

}  // namespace wamb
