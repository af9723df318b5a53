// Host launcher of the tcgen05 GEMM (gemm.cuh): tile-width choice, tensor
// maps, argument checks.
#pragma once
#include "gemm.cuh"
#include "gemm2.cuh"
#include "host.cuh"

namespace wamb {

template <int BN, int STAGES, bool F8>
inline int launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap* tb, const GemmParams& p,
                          int sms, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  static bool configured[64] = {};
  int dev = 0;
  WAMB_CHECK_CUDA(cudaGetDevice(&dev));
  if (!configured[dev]) {
    WAMB_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES, F8>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    configured[dev] = true;
  }
  const int tiles = ((p.M + GEMM_BM - 1) / GEMM_BM) * (p.N / BN) * (p.splits > 1 ? p.splits : 1);
  const int grid = tiles < sms ? tiles : sms;
  return launch_kernel(gemm_tc_kernel<BN, STAGES, F8>, dim3(grid), dim3(GEMM_THREADS), L::TOTAL, stream, ta, tb[0],
                       tb[1], tb[2], p);
}

// Two-CTA launch: clusters of 2 along x, one cluster per pair of SMs.
template <bool F8>
inline int launch_gemm2(const CUtensorMap& ta, const CUtensorMap* tb, const GemmParams& p, int sms,
                        cudaStream_t stream) {
  static int resident[64] = {};  // co-resident clusters per device, 0 = not queried
  int dev = 0;
  WAMB_CHECK_CUDA(cudaGetDevice(&dev));
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = Gemm2Smem::TOTAL;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (resident[dev] == 0) {
    WAMB_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<F8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Gemm2Smem::TOTAL));
    cfg.gridDim = dim3(sms, 1, 1);
    int n = 0;
    WAMB_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<F8>, &cfg));
    resident[dev] = n > 0 ? n : 1;
  }
  const int tiles = ((p.M + 255) / 256) * (p.N / 256);
  const int pairs = tiles < resident[dev] ? tiles : resident[dev];
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  WAMB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<F8>, ta, tb[0], tb[1], tb[2], p));
  return WAMB_OK;
}

// Picks the widest tile (256/128/64 columns) that still gives every SM a
// tile; falls back to the narrowest legal width for small problems.
inline int choose_bn(int M, int N, int n_per_group, int sms) {
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  const int cands[3] = {256, 128, 64};
  int best = 0;
  for (int c : cands) {
    if (n_per_group % c) continue;
    if (best == 0) best = c;
    if (static_cast<long long>(num_m) * (N / c) >= sms) return c;
    best = c;
  }
  return best;
}

// Split-K plan of the one-CTA kernel: when the output tiles at the chosen
// width leave SMs idle (small M: the verify batch, a short chunk), use
// 128-wide tiles and split K so that tiles x splits fills the SMs, each
// split keeping at least 32 k-blocks (measured on B200 at M 128: a 6-way
// split of K 14336 takes the FFN-out GEMM from 66 to 45 us, while 2-3 way
// splits of K 3072 are slower than the unsplit kernel).
// Returns splits (1 = none).
struct SplitPlan {
  int bn, splits, kb_per_split;
};
constexpr int kSplitCounterBytes = 256 * 1024;   // room for 8 counters per tile of up to 8192 tiles

inline SplitPlan plan_split(int M, int N, int n_per_group, int num_kb, int sms, int bn0) {
  SplitPlan sp{bn0, 1, num_kb};
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  if (static_cast<long long>(num_m) * (N / bn0) >= sms) return sp;
  const int bn = n_per_group % 128 == 0 ? 128 : bn0;
  const int tiles = num_m * (N / bn);
  int s = sms / tiles;
  if (s > num_kb / 32) s = num_kb / 32;
  if (s < 2) return sp;
  sp.bn = bn;
  sp.kb_per_split = (num_kb + s - 1) / s;
  sp.splits = (num_kb + sp.kb_per_split - 1) / sp.kb_per_split;   // no empty split
  return sp;
}

// Workspace bytes a split plan needs: counters, then [tiles][splits][128][bn] fp32.
inline size_t split_bytes(int M, int N, const SplitPlan& sp) {
  if (sp.splits <= 1) return 0;
  const size_t tiles = static_cast<size_t>((M + GEMM_BM - 1) / GEMM_BM) * (N / sp.bn);
  return kSplitCounterBytes + tiles * sp.splits * 128 * sp.bn * 4;
}

// Largest split-K scratch any plan can take on a GPU of up to kSplitMaxSms
// SMs: units = tiles x splits <= SMs, each unit's partial 128 x 128 fp32.
constexpr int kSplitMaxSms = 160;
constexpr size_t kSplitReserveBytes =
    static_cast<size_t>(kSplitCounterBytes) + static_cast<size_t>(kSplitMaxSms) * 128 * 128 * 4;

// Whether a GEMM of this shape would split K on a B200 (148 SMs): the block
// reserves split-K scratch only when one of its GEMMs would.
inline bool gemm_would_split(int M, int N, int n_per_group, int K, bool f8) {
  constexpr int sms = 148;
  if (M <= 0) return false;
  const long long pair_tiles = ((M + 255) / 256) * (N / 256);
  if (M >= 512 && n_per_group % 256 == 0 && pair_tiles >= sms / 2) return false;
  const int bn0 = choose_bn(M, N, n_per_group, sms);
  return plan_split(M, N, n_per_group, K / (f8 ? GEMM_BK8 : GEMM_BK), sms, bn0).splits > 1;
}

// counters_zero: the caller guarantees the workspace's counter area is zero
// (the block zeroes it once per call; split GEMMs leave it zero).
inline int linear_impl(const wamb_linear_args* a, cudaStream_t stream, bool counters_zero = false) {
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
  WAMB_REQUIRE(a->ldo >= N && a->ldo % 8 == 0, WAMB_ERR_ALIGN, "ldo");
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

  // 2-CTA 256 x 256 tiles when the weight groups split into 256-wide tiles
  // and there are enough of them to give every SM pair one; otherwise one
  // CTA per 128 x BN tile.
  const long long pair_tiles = ((a->m + 255) / 256) * (N / 256);
  const bool pair = a->m >= 512 && a->n_per_group % 256 == 0 && pair_tiles >= di.sms / 2;
  int bn = pair ? 256 : choose_bn(a->m, static_cast<int>(N), a->n_per_group, di.sms);
  SplitPlan sp{bn, 1, 0};
  if (!pair && a->split_ws != nullptr) {
    sp = plan_split(a->m, static_cast<int>(N), a->n_per_group, a->k / (f8 ? GEMM_BK8 : GEMM_BK), di.sms, bn);
    if (sp.splits > 1) {
      WAMB_REQUIRE(reinterpret_cast<uintptr_t>(a->split_ws) % 256 == 0, WAMB_ERR_ALIGN,
                   "split workspace must be 256-byte aligned");
      const size_t tiles = static_cast<size_t>((a->m + GEMM_BM - 1) / GEMM_BM) * (N / sp.bn);
      if (tiles * GEMM_EPI_WARPS * sizeof(int) > static_cast<size_t>(kSplitCounterBytes) ||
          split_bytes(a->m, static_cast<int>(N), sp) > static_cast<size_t>(a->split_ws_bytes))
        sp = SplitPlan{bn, 1, 0};   // too little room: no split
      else
        bn = sp.bn;
    }
  }
  CUtensorMap ta, tb[3];
  auto tmap = f8 ? make_tmap_e4m3 : make_tmap_bf16;
  rc = tmap(&ta, a->a, a->m, a->k, a->lda, 128);
  if (rc) return rc;
  for (int g = 0; g < 3; ++g) {
    const int src = g < a->groups ? g : 0;
    rc = tmap(&tb[g], a->weight[src], a->n_per_group, a->k, a->k, pair ? 128 : bn);
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
  p.splits = sp.splits;
  if (sp.splits > 1) {
    uint8_t* ws = static_cast<uint8_t*>(a->split_ws);
    p.kb_per_split = sp.kb_per_split;
    p.cnt = reinterpret_cast<int*>(ws);
    p.part = reinterpret_cast<float*>(ws + kSplitCounterBytes);
    const size_t tiles = static_cast<size_t>((a->m + GEMM_BM - 1) / GEMM_BM) * (N / sp.bn);
    if (!counters_zero) WAMB_CHECK_CUDA(cudaMemsetAsync(ws, 0, tiles * GEMM_EPI_WARPS * sizeof(int), stream));
  }
  auto launch = [&](auto f8c) {
    constexpr bool F8 = decltype(f8c)::value;
    if (pair) return launch_gemm2<F8>(ta, tb, p, di.sms, stream);
    switch (bn) {
      case 256: return launch_gemm_bn<256, 4, F8>(ta, tb, p, di.sms, stream);
      case 128: return launch_gemm_bn<128, 6, F8>(ta, tb, p, di.sms, stream);
      default: return launch_gemm_bn<64, 8, F8>(ta, tb, p, di.sms, stream);
    }
  };
  return f8 ? launch(std::true_type{}) : launch(std::false_type{});
}

}  // namespace wamb
