// Host side of the SVD-MLP library: C ABI, weight packing, workspace carving,
// split-K planning, tensor-map encoding and launches of the sm_100a kernels.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "../../include/svdmlp.h"
#include "gemm_sm100.cuh"
#include "gemv_sm100.cuh"
#include "layer_decode_sm100.cuh"
#include "peer_sm100.cuh"

using bf16 = __nv_bfloat16;

namespace svdmlp {

// ------------------------------------------------------------------ state
static thread_local int g_last_cuda_error = 0;
static std::atomic<int64_t> g_launches{0};
static int g_split_override[8] = {0, 0, 0, 0, 0, 0, 0, 0};
static unsigned long long g_wait_limit_ns = 2000000000ull;  // 2 s: far above any legal wait
static constexpr int kLayerDecodeMaxM = 64;        // largest M the whole-layer decode kernel handles
// Measured on B200 (8B layer, three rotated weight copies, with a residual;
// whole-layer kernel / per-stage kernels): 2 tokens 75.3 / 82.5 us, 4 tokens
// 77.3 / 83.3, 6 tokens 81.6 / 83.6, 8 tokens 91.1 / 84.4, 16 tokens
// 88.2 / 87.0 (r = 1911 at 8 tokens: 70.1 / 65.9).
static constexpr int kLayerDecodeDefaultMaxM = 6;
static int g_layer_decode_max_m = kLayerDecodeDefaultMaxM;
// L2 prefetch window of the whole-layer decode kernel's weight stream (slots
// beyond the one loading).  Off: with weights that are not already in L2 the
// extra requests only compete with the stage's slowest units (8B layer,
// three rotated weight copies: M = 1 72.9 us off vs 75.0 us with one slot).
static int g_pf_ahead = 0, g_pf_wait = 0;
// Programmatic dependent launch of the whole-layer decode kernel: 0 = off,
// k >= 1 = on, each CTA prefetching k units' weights before its wait.
// Whole-layer decode launches: 0 plain, 1 overlapped (programmatic dependent
// launch), k >= 2 overlapped and each CTA requests into L2 the weights of k - 1
// units before it waits.  Measured at one token (8B layer, rotated weights):
// plain 78.0 us, overlapped 74.7, with one unit requested 77.4.
static int g_layer_decode_pdl = 1;
// Prefill stage chaining: M-tile groups per stage (0: off).  Off by default:
// under the 1 kW power cap that sustained prefill runs at, filling the SMs a
// stage's tail leaves idle only lowers the clock of the others (measured
// 330 vs 334 us per layer at M = 1024, 1575 vs 1485 MHz), and two groups
// read the gate/up weights from HBM twice.
static int g_chain_groups = 0;    // L2 prefetch window of the whole-layer decode kernel (slots)
static unsigned long long* g_trace = nullptr;  // whole-layer decode timeline (diagnostics)

// Optional per-stage event timing (a diagnostics pass; off by default).
struct TimedLaunch {
  int stage;
  cudaEvent_t start, stop;
};
static std::mutex g_timing_mu;
static bool g_timing = false;
static std::vector<TimedLaunch> g_timed;
static size_t g_timed_used = 0;

static int cuda_fail(cudaError_t e) {
  g_last_cuda_error = static_cast<int>(e);
  return SVDMLP_ERR_CUDA;
}
#define SVD_CUDA(call)                         \
  do {                                         \
    cudaError_t e_ = (call);                   \
    if (e_ != cudaSuccess) return cuda_fail(e_); \
  } while (0)
#define SVD_CHECK(...)      \
  do {                      \
    int s_ = (__VA_ARGS__); \
    if (s_ != SVDMLP_OK) return s_; \
  } while (0)

static int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
static int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool attrs_set = false;
};
static std::mutex g_dev_mu;
static DeviceInfo g_dev[64];

static int device_info(DeviceInfo** out) {
  int dev = 0;
  SVD_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return SVDMLP_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sms == 0) {
    SVD_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    SVD_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
  }
  if (d.major != 10) return SVDMLP_ERR_DEVICE;
  *out = &d;
  return SVDMLP_OK;
}

// Number of SMs used for planning: the current device's, or 148 (B200) when
// no device is visible (workspace sizing on a host without a GPU).
static int planning_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
    return sms;
  cudaGetLastError();
  return 148;
}

// ------------------------------------------------------------- tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

enum class DT { BF16, F16, F32 };

// 2-D row-major tensor [outer, inner] with leading dimension `ld` elements.
static int make_map(CUtensorMap* map, const void* base, DT dt, int64_t inner, int64_t outer, int64_t ld,
                    uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return cuda_fail(cudaErrorInitializationError);
  const int elt = dt == DT::F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * elt) % 16 != 0) return SVDMLP_ERR_ALIGNMENT;
  const CUtensorMapDataType t = dt == DT::F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                : dt == DT::F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elt)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return SVDMLP_ERR_ALIGNMENT;
  return SVDMLP_OK;
}

// Operand tile map: rows of 64 16-bit elements (128 bytes, 128-byte swizzle).
static int operand_map(CUtensorMap* m, const void* base, bool f16, int64_t k, int64_t rows, int64_t ld,
                       int box_rows) {
  return make_map(m, base, f16 ? DT::F16 : DT::BF16, k, rows, ld, 64, static_cast<uint32_t>(box_rows),
                  CU_TENSOR_MAP_SWIZZLE_128B);
}
// Output map: 32 x 32 boxes (16-bit: 64-byte rows, 64B swizzle; fp32: 128-byte rows, 128B swizzle).
template <class Cfg>
static int output_map(CUtensorMap* m, const void* base, int64_t n, int64_t rows, int64_t ld) {
  const DT dt = Cfg::OUT == OUT_F32 ? DT::F32 : Cfg::OUT == OUT_F16 ? DT::F16 : DT::BF16;
  return make_map(m, base, dt, n, rows, ld, 32, 32,
                  dt == DT::F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// Packed weights are stored tile-major: [16-row group][64-column k-block]
// tiles of 16 x 64 elements, each tile 2 KB contiguous and row-major inside.
// A 4-D tensor map (64, 16, k-blocks, groups) reads a box of `box_rows` rows
// (a multiple of 16) of one k-block as box_rows/16 contiguous 2 KB runs and
// lays it out in shared memory exactly as a 2-D [box_rows x 64] box would,
// with the 128-byte swizzle.  Rows beyond N and columns beyond K are zero in
// the packed buffer.
static int64_t tiled_bytes(int64_t n, int64_t k) { return round_up(n, 16) * round_up(k, 64) * 2; }

static int tiled_map(CUtensorMap* map, const void* base, bool f16, int64_t n, int64_t k, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return cuda_fail(cudaErrorInitializationError);
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || box_rows % 16 != 0 || box_rows > 256)
    return SVDMLP_ERR_ALIGNMENT;
  const int64_t kb = cdiv(k, 64), groups = cdiv(n, 16);
  cuuint64_t dims[4] = {64, 16, static_cast<cuuint64_t>(kb), static_cast<cuuint64_t>(groups)};
  cuuint64_t strides[3] = {128, 2048, static_cast<cuuint64_t>(kb * 2048)};
  cuuint32_t box[4] = {64, 16, 1, static_cast<cuuint32_t>(box_rows / 16)};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return SVDMLP_ERR_ALIGNMENT;
  return SVDMLP_OK;
}

// ------------------------------------------------------------------ planner
struct Plan {
  int m_tiles, n_tiles, k_blocks, splits, kb_per_split, units, grid;
  // split tail (CTA-pair plans): units [tail_start, units) split the last
  // wave's tiles `tail_splits` ways; -1: none
  int tail_start = -1, tail_splits = 1, tail_kb_per_split = 0;
};
// Split tail of the CTA-pair plans (on by default; svdmlp_set_split_tail).
static int g_split_tail = 1;

// One-CTA plans (decode-sized M): chooses the split-K factor that minimises a
// wave-quantisation cost model in units of one k-block's MMA time: rounds of
// units over the SMs times the k-blocks per unit, plus a per-unit pipeline
// and epilogue overhead, plus the fix-up traffic of the partial tiles (valid
// rows only), which is latency-bound at roughly 20 bytes per SM cycle.
static Plan plan_gemm(int M, int N, int K, int BN, int NB, int sms, int forced_splits) {
  Plan p{};
  p.m_tiles = static_cast<int>(cdiv(M, 128));
  p.n_tiles = static_cast<int>(cdiv(N, BN));
  p.k_blocks = static_cast<int>(cdiv(K, 64));
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  const double rows = static_cast<double>(std::min(M, 128));
  int best_s = 1;
  if (forced_splits > 0) {
    best_s = std::min(forced_splits, p.k_blocks);
  } else {
    double best = 1e30;
    for (int s = 1; s <= 32; ++s) {
      const int kbs = static_cast<int>(cdiv(p.k_blocks, s));
      if (s > 1 && kbs < 2) break;
      const int s_eff = static_cast<int>(cdiv(p.k_blocks, kbs));
      if (s > 1 && s_eff != s) continue;
      const int64_t units = tiles * s_eff;
      const int64_t rounds = cdiv(units, sms);
      double cost = static_cast<double>(rounds) * (kbs + 1.5);
      if (s_eff > 1) cost += 1.0 + 2.0 * s_eff * rows * BN * NB * 4.0 / 20.0 / 512.0;
      if (cost < best * 0.97) {
        best = cost;
        best_s = s_eff;
      }
    }
  }
  p.kb_per_split = static_cast<int>(cdiv(p.k_blocks, best_s));
  p.splits = static_cast<int>(cdiv(p.k_blocks, p.kb_per_split));
  p.units = static_cast<int>(tiles * p.splits);
  p.grid = std::min(p.units, sms);
  return p;
}

// CTA-pair plans (prefill-sized M): 256-row tiles, no split-K, one cluster of
// two CTAs per pair of SMs.
// CTA-pair plans (prefill).  Split-K over the pairs when it fills more of the
// waves (tiles x splits over sms/2 pairs) than the extra fix-up costs: each
// split writes an fp32 partial of its 256 x BN tile, and once all splits are
// in, every split sums a share of the tile's 32-column chunks (modelled as ~10
// k-blocks of work), while the partials stay within kPairPartialBudget (not
// for the dual-store X.[u_g|u_u] tile).
static constexpr int64_t kPairPartialBudget = 48ll << 20;
// L2 bytes one group of M-tiles' A rows may take (of 126 MB; the rest holds
// the weight tiles in flight, outputs and partials).
static constexpr int64_t kL2GroupBytes = 40ll << 20;
static constexpr double kL2Bytes = 96.0 * (1 << 20);  // L2 a GEMM's A operand can count on keeping
static Plan plan_gemm_pair(int M, int N, int K, int BN, int sms, bool allow_split = false, int forced_splits = 0,
                           int nb = 1) {
  Plan p{};
  p.m_tiles = static_cast<int>(cdiv(M, 256));
  p.n_tiles = static_cast<int>(cdiv(N, BN));
  p.k_blocks = static_cast<int>(cdiv(K, 64));
  const int pairs = std::max(1, sms / 2);
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  int best_s = 1;
  if (allow_split) {
    if (forced_splits > 0) {
      best_s = std::min(forced_splits, p.k_blocks);
    } else {
      double best = 1e30;
      for (int s = 1; s <= 4; ++s) {
        const int kbs = static_cast<int>(cdiv(p.k_blocks, s));
        if (s > 1 && (kbs < 8 || tiles * s * 2 * nb * 128 * BN * 4 > kPairPartialBudget)) break;
        const double cost = static_cast<double>(cdiv(tiles * s, pairs)) * kbs + (s > 1 ? 10.0 : 0.0);
        if (cost < best * 0.95) {
          best = cost;
          best_s = s;
        }
      }
    }
  }
  p.kb_per_split = static_cast<int>(cdiv(p.k_blocks, best_s));
  p.splits = static_cast<int>(cdiv(p.k_blocks, p.kb_per_split));
  p.units = static_cast<int>(tiles) * p.splits;
  // Split tail: when whole waves are unsplit and the last wave is partial,
  // its tiles are split over K across the pairs that wave would leave idle
  // (8B layer at 1024 tokens: the dual gate/up GEMM's 256 tiles are 3 waves
  // of 74 pairs plus 34 tiles, whose 2-way splits take 68 pairs for half as
  // long).  Same k-block cost model as above, including the fix-up.
  if (allow_split && forced_splits <= 0 && g_split_tail && p.splits == 1) {
    const int64_t waves = tiles / pairs, rem = tiles - waves * pairs;
    const double plain = static_cast<double>(cdiv(tiles, pairs)) * p.k_blocks;
    double best_tail = plain * 0.95;
    for (int st = 2; st <= 4 && waves >= 1 && rem > 0; ++st) {
      const int kbs = static_cast<int>(cdiv(p.k_blocks, st));
      if (rem * st > pairs || kbs < 8 || rem * st * 2 * nb * 128 * BN * 4 > kPairPartialBudget) break;
      const double cost = static_cast<double>(waves) * p.k_blocks + kbs + 10.0;
      if (cost < best_tail) {
        best_tail = cost;
        p.tail_start = static_cast<int>(waves * pairs);
        p.tail_kb_per_split = kbs;
        p.tail_splits = static_cast<int>(cdiv(p.k_blocks, kbs));
      }
    }
    if (p.tail_start >= 0) p.units = p.tail_start + static_cast<int>(rem) * p.tail_splits;
  }
  p.grid = 2 * std::min(p.units, pairs);
  return p;
}

template <class Cfg>
static Plan plan_for(int M, int N, int K, int sms, int forced_splits) {
  if constexpr (Cfg::CTAS == 2)
    return plan_gemm_pair(M, N, K, Cfg::BN, sms, Cfg::EPI != EPI_DUAL_STORE, forced_splits, Cfg::NB);
  else return plan_gemm(M, N, K, Cfg::BN, Cfg::NB, sms, forced_splits);
}

// Token counts above this use the CTA-pair kernels; below, one-CTA kernels
// with split-K stream the weights across all SMs.
// Smallest M run on the CTA-pair GEMMs (below it: the one-CTA and streaming
// decode kernels).  Tunable at run time down to kPairMinMLowest; workspaces are
// sized for any threshold in that range.
static constexpr int kPairMinMDefault = 129;
static constexpr int kPairMinMLowest = 17;
static int g_pair_min_m = kPairMinMDefault;

// Split choice for a weight-streaming (decode) stage, from a model fitted to
// B200 measurements of these kernels: a CTA streams about 60 GB/s (its
// in-flight weight bytes over ~1.6 us of memory latency), the GPU about
// 7 TB/s; every extra unit a CTA runs in a stage costs about one latency, and
// split-K adds a ~4 us chain to the stage (partial stores, the arrival
// atomic, the last split's reads and stores), plus, when the last split sums
// every partial, a memory round trip per four splits per 16 tokens.
static constexpr double kHbmBytesPerUs = 7.0e6;
static constexpr double kCtaBytesPerUs = 6.0e4;
static Plan plan_stream(int M, int tok, int N, int K, int nb, int slots, int forced_splits,
                        bool spread_fixup = false) {
  Plan p{};
  p.m_tiles = 1;
  p.n_tiles = static_cast<int>(cdiv(N, 128));
  p.k_blocks = static_cast<int>(cdiv(K, 64));
  const int tv16 = static_cast<int>(cdiv(std::min(M, tok), 16));
  const double total = static_cast<double>(p.n_tiles) * p.k_blocks * 16384.0 * nb;
  int best_s = 1;
  if (forced_splits > 0) {
    best_s = std::min(forced_splits, p.k_blocks);
  } else {
    double best = 1e30;
    for (int s = 1; s <= 24; ++s) {
      const int kbs = static_cast<int>(cdiv(p.k_blocks, s));
      if (s > 1 && kbs < 2) break;
      const int s_eff = static_cast<int>(cdiv(p.k_blocks, kbs));
      if (s > 1 && s_eff != s) continue;
      const int64_t units = static_cast<int64_t>(p.n_tiles) * s_eff;
      const double rounds = static_cast<double>(cdiv(units, slots));
      const double busiest = rounds * kbs * 16384.0 * nb;
      double us = std::max(total / kHbmBytesPerUs, busiest / kCtaBytesPerUs) + 1.5 * rounds;
      // The last split of a tile sums every partial (cost grows with the split
      // count and the token chunks); in the spread fix-up every split sums
      // 1/S of the tile's token rows in parallel, a constant hand-off.
      if (s_eff > 1) us += spread_fixup ? 4.0 : 4.0 + 1.0 * static_cast<double>(cdiv(s_eff, 4) - 1) * tv16;
      if (us < best * 0.97) {
        best = us;
        best_s = s_eff;
      }
    }
  }
  p.kb_per_split = static_cast<int>(cdiv(p.k_blocks, best_s));
  p.splits = static_cast<int>(cdiv(p.k_blocks, p.kb_per_split));
  p.units = p.n_tiles * p.splits;
  p.grid = std::min(p.units, slots);
  return p;
}

// Decode plans of the per-stage streaming kernels: 128-row weight panels
// split along K over the CTA slots (two per SM where the footprint allows).
template <class Cfg>
static Plan plan_dec(int M, int N, int K, int sms, int forced_splits) {
#ifndef SVDMLP_DEC_CTAS_PER_SM
#define SVDMLP_DEC_CTAS_PER_SM 2
#endif
  const int slots = (Cfg::TWO_PER_SM ? SVDMLP_DEC_CTAS_PER_SM : 1) * sms;
  // Above 16 tokens the per-stage kernels use the spread fix-up (gemv_sm100.cuh).
  const bool spread = std::min(M, Cfg::TOK) > 16;
  if (spread && Cfg::NB == 1 && forced_splits <= 0) {
    // One-branch stages: the smallest split count that gives at least 1.2
    // units per SM.  Split sweeps of the 8B layer at 32 and 128 tokens, ratios
    // 0.6 and 0.9, put this within ~3 us of the best (X.[u_g,u_u] 4-6,
    // H.u_down 8-12, T.v_down 4-6 splits); the stream model above
    // under-splits these stages by 2-9 us.
    const int n_tiles = static_cast<int>(cdiv(N, Cfg::BM));
    const int k_blocks = static_cast<int>(cdiv(K, Cfg::BK));
    const int want = static_cast<int>(std::min<int64_t>(k_blocks / 2, cdiv(static_cast<int64_t>(12 * sms), 10LL * n_tiles)));
    return plan_stream(M, Cfg::TOK, N, K, Cfg::NB, slots, std::max(1, want), true);
  }
  return plan_stream(M, Cfg::TOK, N, K, Cfg::NB, slots, forced_splits, spread);
}

// One stage of the whole-layer decode kernel (all stages share `slots` CTAs).
static Plan plan_layer_stage(int M, int tok, int N, int K, int nb, int slots, int forced_splits) {
  Plan p = plan_stream(M, tok, N, K, nb, slots, forced_splits);
  p.grid = slots;
  return p;
}

// CTAs per SM of the whole-layer decode kernel.  Two fit (shared memory and
// TMEM allow it) but measure slower than one: the weight stream is bound by
// HBM and the TMA path, not by copies in flight, and twice the CTAs only
// lengthen each stage's tail.
static constexpr int kLayerDecodeCtasPerSm = 1;
// Shared-memory ring depth (slots of two weight and two token tiles) of the
// whole-layer decode kernel for 16- and 64-token tiles.
#ifndef SVDMLP_LD_RING16
#define SVDMLP_LD_RING16 5
#endif
#ifndef SVDMLP_LD_RING64
#define SVDMLP_LD_RING64 4
#endif

// Partial bytes of the whole-layer decode kernel (all four stages at once).
// The contracted decode schedule (16-token tiles): the gate/up stage's units
// also multiply their H tile by u_down, writing fp32 partials of T per ff tile.
// svdmlp_forward uses it for M <= g_decode_contract tokens.  Measured on B200
// (8B layer, three rotated weight copies): M = 1 74.4 vs 76.0 us at r = 2867
// and 58.0 vs 62.1 us at r = 1911; at 2 tokens 79.4 vs 77.8 and 63.0 vs 64.3;
// from 4 tokens on slower (the partials grow with the tokens).
static constexpr int kDecodeContractDefault = 1;
static int g_decode_contract = kDecodeContractDefault;
static int64_t contract_partials(const svdmlp_layout* L) {
  return round_up(cdiv(L->ff, 128) * 16 * round_up(L->r_d, 128) * 4, 256);
}

// Partial bytes of the whole-layer decode kernel (all four stages at once),
// the larger of the plain and the contracted schedule.
static int64_t layer_decode_partials(const svdmlp_layout* L, int M, int sms) {
  const int tok = M <= 16 ? 16 : 64;
  const int slots = kLayerDecodeCtasPerSm * sms;
  const int shapes[4][3] = {{2 * L->rp_gu, L->d, 1}, {L->ff, L->r_gu, 2}, {L->r_d, L->ff, 1}, {L->d, L->r_d, 1}};
  int64_t by_stage[4] = {0, 0, 0, 0};
  for (int st = 0; st < 4; ++st) {
    const Plan pl =
        plan_layer_stage(M, tok, shapes[st][0], shapes[st][1], shapes[st][2], slots, g_split_override[st]);
    if (pl.splits > 1) by_stage[st] = round_up(static_cast<int64_t>(pl.units) * 2 * 128 * tok * 4, 256);
  }
  const int64_t plain = by_stage[0] + by_stage[1] + by_stage[2] + by_stage[3];
  const int64_t contracted = tok == 16 ? by_stage[0] + by_stage[3] + contract_partials(L) : 0;
  return std::max(plain, contracted);
}

template <class Cfg>
static int64_t dec_partial_bytes(const Plan& p) {
  if (p.splits <= 1) return 0;
  return static_cast<int64_t>(p.units) * Cfg::NB * Cfg::BM * Cfg::TOK * 4;
}

// Bytes of split-K partials a plan needs (NB accumulators of BM x BN fp32).
static int64_t partial_bytes(const Plan& p, int BN, int NB, int ctas = 1) {
  if (p.tail_start >= 0) return static_cast<int64_t>(p.units - p.tail_start) * ctas * NB * 128 * BN * 4;
  if (p.splits <= 1) return 0;
  return static_cast<int64_t>(p.units) * ctas * NB * 128 * BN * 4;
}

// ------------------------------------------------------------ kernel configs
// Tile choices of the prefill kernels (compile-time; the defaults are the
// tuned values, other values serve tile sweeps).
// Dual gate/up tile: 256 x 256 per branch (one TMEM buffer of 2 x 256
// columns, 3 pipeline stages in 225 KB of shared memory).  The widest tile
// wins: 7.6 KB of operands per MFLOP against 8.2 for 256 x 224 and 11.4 for
// 256 x 128, and fewer tiles per launch, although operand traffic is not the
// bound (with no operand loads at all the stage still takes 0.92 of its time)
// (config 1: 256 x 128 double-buffered 199 us, 256 x 224 166 -> 139 us with
// the tile-major weights; 256 x 256 with the split tail 275 vs 280 us per
// layer in short runs, 312 vs 317 us sustained).
#ifndef SVDMLP_GU_BN
#define SVDMLP_GU_BN 256      // per-branch N of the dual gate/up tile
#endif
#ifndef SVDMLP_GU_STAGES
#define SVDMLP_GU_STAGES 3
#endif
#ifndef SVDMLP_GU_EPI_WARPS
#define SVDMLP_GU_EPI_WARPS 8
#endif
#ifndef SVDMLP_DENSE_GU_STAGES
#define SVDMLP_DENSE_GU_STAGES 4
#endif
#ifndef SVDMLP_PLAIN_STAGES
#define SVDMLP_PLAIN_STAGES 6
#endif
#ifndef SVDMLP_PLAIN_EPI_WARPS
#define SVDMLP_PLAIN_EPI_WARPS 4
#endif
#ifndef SVDMLP_XU_BN
#define SVDMLP_XU_BN 256      // N of the X.[u_g|u_u] tile
#endif
#ifndef SVDMLP_DU_BN
#define SVDMLP_DU_BN 256      // N of the H.u_down tile
#endif
#ifndef SVDMLP_DV_BN
#define SVDMLP_DV_BN 256      // N of the T.v_down tile
#endif
constexpr int kGuBn = SVDMLP_GU_BN, kGuSt = SVDMLP_GU_STAGES, kGuEw = SVDMLP_GU_EPI_WARPS;
constexpr int kXuBn = SVDMLP_XU_BN, kDuBn = SVDMLP_DU_BN, kDvBn = SVDMLP_DV_BN;
constexpr int kDgSt = SVDMLP_DENSE_GU_STAGES;
constexpr int kPlSt = SVDMLP_PLAIN_STAGES, kPlEw = SVDMLP_PLAIN_EPI_WARPS;

// Prefill (M > 128): CTA pairs, 256-row tiles.
//                          BN     NB shared STG    epilogue   fp16-in out       CTAs epi-warps
// X.[u_g|u_u] at prefill as one dual-store tile: 256 x (2 x 160) per CTA pair,
// the A tile read once for both halves (57.6 operand bytes per MMA cycle per
// SM against 64 for 256 x 256) and 18 x 4 = 72 tiles for 74 pairs at 1024
// tokens (256-wide tiles: 92, i.e. 1.24 waves).
#ifndef SVDMLP_XUD_BN
#define SVDMLP_XUD_BN 160
#endif
#ifndef SVDMLP_XUD_STAGES
#define SVDMLP_XUD_STAGES 5
#endif
using CfgXUd    = GemmCfg<SVDMLP_XUD_BN, 2, true, SVDMLP_XUD_STAGES, EPI_DUAL_STORE, false, OUT_F16, 2, 8>;
using CfgXU     = GemmCfg<kXuBn,   1, false, kPlSt, EPI_PLAIN,  false, OUT_F16,  2, kPlEw>;  // X.[u_g|u_u] -> XU
using CfgGU     = GemmCfg<kGuBn, 2, false, kGuSt, EPI_SWIGLU, true,  OUT_F16,  2, kGuEw>;  // XU.v -> H (internal)
using CfgGUbf   = GemmCfg<kGuBn, 2, false, kGuSt, EPI_SWIGLU, true,  OUT_BF16, 2, kGuEw>;  // XU.v -> H (to caller)
using CfgDU     = GemmCfg<kDuBn,   1, false, kPlSt, EPI_PLAIN,  true,  OUT_F16,  2, kPlEw>;  // H.u_down -> T
using CfgDUbf   = GemmCfg<kDuBn,   1, false, kPlSt, EPI_PLAIN,  false, OUT_F16,  2, kPlEw>;  // bf16 H.u_down
using CfgDUf32  = GemmCfg<kDuBn,   1, false, kPlSt, EPI_PLAIN,  true,  OUT_F32,  2, kPlEw>;  // H.u_down -> fp32 (TP)
using CfgDV     = GemmCfg<kDvBn,   1, false, kPlSt, EPI_PLAIN,  true,  OUT_BF16, 2, kPlEw>;  // T.v_down -> y
using CfgDVres  = GemmCfg<kDvBn,   1, false, kPlSt, EPI_RESID,  true,  OUT_BF16, 2, kPlEw>;  // + residual
using CfgDenseGU = GemmCfg<kGuBn, 2, true, kDgSt, EPI_SWIGLU, false, OUT_F16,  2, kGuEw>;  // X.[w_g|w_u] -> H
using CfgGemm   = GemmCfg<256,   1, false, kPlSt, EPI_PLAIN,  false, OUT_BF16, 2, kPlEw, false>;  // row-major B
// Decode (M <= 128): one CTA per tile, split-K across the SMs.
using CfgXU1     = GemmCfg<256, 1, false, 4, EPI_PLAIN,  false, OUT_F16>;
using CfgGU1     = GemmCfg<128, 2, false, 3, EPI_SWIGLU, true,  OUT_F16>;
using CfgGUbf1   = GemmCfg<128, 2, false, 3, EPI_SWIGLU, true,  OUT_BF16>;
using CfgDU1     = GemmCfg<256, 1, false, 4, EPI_PLAIN,  true,  OUT_F16>;
using CfgDUbf1   = GemmCfg<256, 1, false, 4, EPI_PLAIN,  false, OUT_F16>;
using CfgDUf321  = GemmCfg<256, 1, false, 4, EPI_PLAIN,  true,  OUT_F32>;
using CfgDV1     = GemmCfg<256, 1, false, 4, EPI_PLAIN,  true,  OUT_BF16>;
using CfgDVres1  = GemmCfg<256, 1, false, 4, EPI_RESID,  true,  OUT_BF16>;
using CfgDenseGU1 = GemmCfg<128, 2, true, 4, EPI_SWIGLU, false, OUT_F16>;
using CfgGemm1   = GemmCfg<256, 1, false, 4, EPI_PLAIN,  false, OUT_BF16, 1, 4, false>;
// Decode (M <= 128): swapped-operand weight-streaming kernels (gemv_sm100.cuh),
// one set per token tile TOK (the MMA N).  TOK <= 64 sets stay within 113 KB
// of shared memory and 256 TMEM columns so that two CTAs share an SM.
template <int TOK>
struct DecSet {
  static constexpr int PST = TOK == 16 ? 5 : TOK == 64 ? 4 : 3;  // stages, one-branch kernels
  static constexpr int DST = TOK == 64 ? 2 : TOK == 16 ? 2 : 3;  // stages, dual kernels (TOK <= 64: two CTAs per SM)
  using XU = DecCfg<TOK, 1, PST, EPI_PLAIN, false, OUT_F16>;
  using GU = DecCfg<TOK, 2, DST, EPI_SWIGLU, true, OUT_F16>;
  using DU = DecCfg<TOK, 1, PST, EPI_PLAIN, true, OUT_F16>;
  using DUf32 = DecCfg<TOK, 1, PST, EPI_PLAIN, true, OUT_F32>;
  using DV = DecCfg<TOK, 1, PST, EPI_PLAIN, true, OUT_BF16>;
  using DVres = DecCfg<TOK, 1, PST, EPI_RESID, true, OUT_BF16>;
  using DGU = DecCfg<TOK, 2, DST, EPI_SWIGLU, false, OUT_F16>;  // dense X.[w_g|w_u] (bf16 operands)
};
using Dec16 = DecSet<16>;
using Dec64 = DecSet<64>;
using Dec128 = DecSet<128>;

enum Stage : int {
  ST_XU = 0, ST_GATEUP = 1, ST_DOWN_U = 2, ST_DOWN_V = 3, ST_DENSE_GU = 4, ST_DENSE_D = 5, ST_GEMM = 6,
  ST_LAYER_DECODE = 7  // timing id of the whole-layer decode kernel
};

// Workspace carving.  The control block holds the error word (int 0) and the
// split-K counters; the rest holds the intermediates.
// One link of a chained prefill layer (gemm_sm100.cuh): the counters a stage
// waits on and the ones it publishes to.
struct ChainLink {
  const int* dep;    // previous stage's M-tile counters (null: the first stage)
  int dep_target;    // 2 x the previous stage's N-tiles (both CTAs of a pair publish)
  int* pub;          // this stage's M-tile counters (null: the last stage)
  int* reset;        // last stage: the chain's counter block
  int* exit_count;   // last stage: exit counter
  int m_group;       // M-tiles per unit group
};

struct Workspace {
  int* err;
  int* counters;
  __half* xu;  // [M, 2*rp_gu]  fp16
  __half* h;   // [M, ld_ff]    fp16 (or bf16 staging of a caller's H)
  __half* t;   // [M, rp_d]     fp16
  bf16* xs;   // [M, ld_d] staging for unaligned x
  bf16* ys;   // [M, ld_d] staging for unaligned y
  float* partials;
  int64_t partial_cap;
  // When the split-K partials of a plan do not fit in partial_cap: false
  // fails the call with SVDMLP_ERR_WORKSPACE, true runs the GEMM unsplit.
  bool unsplit_if_short = false;
  const ChainLink* chain = nullptr;  // set for the stages of a chained prefill layer
  // Fused RMSNorm of a decoder block (see GemmParams): the stage that reads
  // the block input scales rows by the norm; the residual stage writes the
  // next block's statistics.
  const float* norm_stats = nullptr;
  int norm_parts = 0, norm_dim = 0, stats_ld = 0;
  float norm_eps = 0.0f;
  float* out_stats = nullptr;
  // Tensor-parallel exchange fused into the H.u_down epilogue (the CTA-pair
  // GEMM only; see GemmPush).
  const GemmPush* push = nullptr;
};

static constexpr int64_t kCtlBytes = 256;
static constexpr int64_t kPackStatusBytes = 256;  // trailing block of a packed layer (its status word)
// Split-K arrival counters: a fixed 1 MiB region (262144 tiles) right after
// the control block, so that every entry point and layout carves it at the
// same place and svdmlp_workspace_init zeroes exactly it.
static constexpr int64_t kCounterBytes = 1 << 20;
// The last 64 KiB of the counter region hold the chained-prefill counters:
// [3 stages][kChainStride M-tiles] and one exit counter.
static constexpr int64_t kChainOffsetInts = (kCounterBytes - 65536) / 4;
static int64_t counters_bytes(const svdmlp_layout*, int) { return kCounterBytes; }

template <class Cfg>
static int64_t stage_partials(int M, int N, int K, int sms, int stage) {
  const Plan p = plan_for<Cfg>(M, N, K, sms, g_split_override[stage]);
  return partial_bytes(p, Cfg::BN, Cfg::NB, Cfg::CTAS);
}

template <class Set>
static int64_t dec_set_partials(const svdmlp_layout* L, int M, int sms) {
  int64_t b = 0;
  if (L->kind == SVDMLP_KIND_DENSE) {
    b = std::max(b, dec_partial_bytes<typename Set::DGU>(
                        plan_dec<typename Set::DGU>(M, L->ff, L->d, sms, g_split_override[ST_DENSE_GU])));
    return std::max(b, dec_partial_bytes<typename Set::DV>(
                           plan_dec<typename Set::DV>(M, L->d, L->ff, sms, g_split_override[ST_DENSE_D])));
  }
  if (L->r_gu > 0) {
    b = std::max(b, dec_partial_bytes<typename Set::XU>(
                        plan_dec<typename Set::XU>(M, 2 * L->rp_gu, L->d, sms, g_split_override[ST_XU])));
    b = std::max(b, dec_partial_bytes<typename Set::GU>(
                        plan_dec<typename Set::GU>(M, L->ff, L->r_gu, sms, g_split_override[ST_GATEUP])));
  }
  if (L->r_d > 0) {
    b = std::max(b, dec_partial_bytes<typename Set::DU>(
                        plan_dec<typename Set::DU>(M, L->r_d, L->ff, sms, g_split_override[ST_DOWN_U])));
    b = std::max(b, dec_partial_bytes<typename Set::DV>(
                        plan_dec<typename Set::DV>(M, L->d, L->r_d, sms, g_split_override[ST_DOWN_V])));
  }
  return b;
}

// Largest split-K partial buffer any M <= max_m can ask for: the one-CTA and
// decode kernels (M <= 128) and the CTA-pair GEMMs (any M >= kPairMinMLowest,
// so that every run-time threshold fits; the planner caps their partials at
// kPairPartialBudget, forced split counts may exceed it), evaluated on every
// 256-row step.
static int64_t max_partials(const svdmlp_layout* L, int max_m, int sms) {
  const int M = std::min(max_m, kPairMinMDefault - 1);
  int64_t best = 0;
  // Partials grow with the M-tiles: every 256-row step below max_m, and
  // max_m itself (whose last M-tile may be partial).
  for (int step = kPairMinMLowest;; step = step < 256 ? 256 : step + 256) {
    const int mp = std::min(step, max_m);
    if (mp < kPairMinMLowest) break;
    if (L->kind == SVDMLP_KIND_SVD) {
      if (L->r_gu > 0) best = std::max(best, stage_partials<CfgGU>(mp, L->ff, L->r_gu, sms, ST_GATEUP));
      if (L->r_d > 0) {
        best = std::max(best, stage_partials<CfgDU>(mp, L->r_d, L->ff, sms, ST_DOWN_U));
        best = std::max(best, stage_partials<CfgDUf32>(mp, L->r_d, L->ff, sms, ST_DOWN_U));
        best = std::max(best, stage_partials<CfgDV>(mp, L->d, L->r_d, sms, ST_DOWN_V));
      }
    } else {
      best = std::max(best, stage_partials<CfgDenseGU>(mp, L->ff, L->d, sms, ST_DENSE_GU));
      best = std::max(best, stage_partials<CfgDV>(mp, L->d, L->ff, sms, ST_DENSE_D));
    }
    if (mp >= max_m) break;
  }
  if (L->kind == SVDMLP_KIND_SVD) {
    if (L->r_gu > 0) {
      best = std::max(best, stage_partials<CfgXU1>(M, 2 * L->rp_gu, L->d, sms, ST_XU));
      best = std::max(best, stage_partials<CfgGU1>(M, L->ff, L->r_gu, sms, ST_GATEUP));
    }
    if (L->r_d > 0) {
      best = std::max(best, stage_partials<CfgDU1>(M, L->r_d, L->ff, sms, ST_DOWN_U));
      best = std::max(best, stage_partials<CfgDV1>(M, L->d, L->r_d, sms, ST_DOWN_V));
    }
  }
  if (L->kind == SVDMLP_KIND_SVD && L->r_gu > 0 && L->r_d > 0) {
    for (int m : {1, 16, 17, 64}) {
      if (m > max_m) break;
      best = std::max(best, layer_decode_partials(L, m, sms));
    }
  }
  {
    for (int m : {1, 16, 17, 64, 65, 128}) {
      if (m > max_m) break;
      if (m <= 16) best = std::max(best, dec_set_partials<Dec16>(L, m, sms));
      else if (m <= 64) best = std::max(best, dec_set_partials<Dec64>(L, m, sms));
      else best = std::max(best, dec_set_partials<Dec128>(L, m, sms));
    }
  }
  return round_up(best, 256);
}

static int64_t ws_bytes_for(const svdmlp_layout* L, int max_m, int sms) {
  const int64_t M = max_m;
  int64_t b = kCtlBytes + counters_bytes(L, max_m);
  b += round_up(M * 2 * L->rp_gu * 2, 256);
  b += round_up(M * L->ld_ff * 2, 256);
  b += round_up(M * L->rp_d * 2, 256);
  b += 2 * round_up(M * L->ld_d * 2, 256);
  b += max_partials(L, max_m, sms);
  return b;
}

static int carve(const svdmlp_layout* L, int M, void* ws, int64_t ws_bytes, Workspace* w) {
  if (!ws) return SVDMLP_ERR_INVALID_VALUE;
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return SVDMLP_ERR_ALIGNMENT;
  const int sms = planning_sms();
  const int64_t need = ws_bytes_for(L, M, sms);
  if (ws_bytes < need) return SVDMLP_ERR_WORKSPACE;
  uint8_t* p = static_cast<uint8_t*>(ws);
  w->err = reinterpret_cast<int*>(p);
  p += kCtlBytes;
  w->counters = reinterpret_cast<int*>(p);
  p += counters_bytes(L, M);
  w->xu = reinterpret_cast<__half*>(p);
  p += round_up(static_cast<int64_t>(M) * 2 * L->rp_gu * 2, 256);
  w->h = reinterpret_cast<__half*>(p);
  p += round_up(static_cast<int64_t>(M) * L->ld_ff * 2, 256);
  w->t = reinterpret_cast<__half*>(p);
  p += round_up(static_cast<int64_t>(M) * L->rp_d * 2, 256);
  w->xs = reinterpret_cast<bf16*>(p);
  p += round_up(static_cast<int64_t>(M) * L->ld_d * 2, 256);
  w->ys = reinterpret_cast<bf16*>(p);
  p += round_up(static_cast<int64_t>(M) * L->ld_d * 2, 256);
  w->partials = reinterpret_cast<float*>(p);
  w->partial_cap = static_cast<uint8_t*>(ws) + ws_bytes - p;
  return SVDMLP_OK;
}

// ------------------------------------------------------------------ launches
template <class Cfg>
static int launch_gemm(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& b, const CUtensorMap& b2,
                       const CUtensorMap& out, const CUtensorMap& out2, int M, int N, int K, int stage, const Workspace& w,
                       const bf16* residual, int64_t ld_res, cudaStream_t stream) {
  // Only a residual stage whose tiles hold whole 128-column slices, one
  // epilogue thread per row, writes the block statistics.
  if (w.out_stats != nullptr && !(Cfg::EPI == EPI_RESID && Cfg::BN % 128 == 0 && Cfg::EPI_WARPS == 4))
    return SVDMLP_ERR_INVALID_VALUE;
  DeviceInfo* dev = nullptr;
  SVD_CHECK(device_info(&dev));
  static std::mutex mu;
  {
    // The dynamic shared memory opt-in is a per-function attribute; set it on
    // first use for each device.
    int cur = 0;
    SVD_CUDA(cudaGetDevice(&cur));
    static uint64_t done_mask = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!(done_mask & (1ull << cur))) {
      SVD_CUDA(cudaFuncSetAttribute(gemm_sm100_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::SMEM_BYTES));
      done_mask |= 1ull << cur;
    }
  }
  Plan pl = plan_for<Cfg>(M, N, K, dev->sms, g_split_override[stage]);
  // chained stages publish whole tiles, and the block statistics are written
  // per tile row by the unsplit epilogue: unsplit
  if ((partial_bytes(pl, Cfg::BN, Cfg::NB, Cfg::CTAS) > w.partial_cap && w.unsplit_if_short) ||
      ((w.chain || w.out_stats || w.norm_stats) && (pl.splits > 1 || pl.tail_start >= 0)))
    pl = plan_for<Cfg>(M, N, K, dev->sms, 1);
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.k_blocks = pl.k_blocks;
  p.splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.num_units = pl.units;
  p.tail_start = pl.tail_start >= 0 ? pl.tail_start : pl.units;
  p.tail_splits = pl.tail_splits;
  p.tail_kb_per_split = pl.tail_kb_per_split;
  p.norm_stats = w.norm_stats;
  p.norm_parts = w.norm_parts;
  p.norm_dim = w.norm_dim;
  p.norm_eps = w.norm_eps;
  p.stats_ld = w.stats_ld;
  p.out_stats = w.out_stats;
  p.partials = w.partials;
  p.counters = w.counters;
  p.err = w.err;
  p.timeout_ns = g_wait_limit_ns;
  p.residual = residual;
  p.ld_residual = ld_res;
  if (w.push != nullptr) {
    if constexpr (kPushable<Cfg> && Cfg::CTAS == 2) p.push = *w.push;
    else return SVDMLP_ERR_INVALID_VALUE;
  }
  // Unit raster, from an estimate of HBM traffic.  m-fastest (one group):
  // the weights are read once, A once if it fits in L2, else once per span
  // of N-tiles that one wave of pairs covers.  Grouped: M-tiles in groups
  // whose A rows fit in kL2GroupBytes, A read once, the weights once per
  // group.  Grouping pays for very long M (32 K tokens: ~10x less traffic).
  p.m_group = pl.m_tiles;
  if constexpr (Cfg::CTAS == 2) {
    const double a_tile = static_cast<double>(Cfg::TILE_M) * K * 2 * Cfg::NA;
    const double a_total = a_tile * pl.m_tiles;
    const double b_total = static_cast<double>(N) * K * 2 * Cfg::NB;
    const double waves_n = std::max(1.0, (dev->sms / 2.0) / pl.m_tiles);  // N-tiles one wave spans
    const double t0 = b_total + (a_total > kL2Bytes ? a_total * pl.n_tiles / waves_n : a_total);
    const int g = static_cast<int>(std::max(1.0, std::min<double>(pl.m_tiles, kL2GroupBytes / a_tile)));
    const double t1 = a_total + b_total * static_cast<double>(cdiv(pl.m_tiles, g));
    if (g < pl.m_tiles && t1 < 0.7 * t0) p.m_group = g;
  }
  if (w.chain) {
    // Chained stages are CTA-pair, unsplit plans by construction of the caller.
    if (Cfg::CTAS != 2 || pl.splits != 1 || pl.tail_start >= 0 || pl.m_tiles > kChainStride)
      return SVDMLP_ERR_INVALID_VALUE;
    p.m_group = std::min(w.chain->m_group, pl.m_tiles);
    p.dep = w.chain->dep;
    p.dep_target = w.chain->dep_target;
    p.pub = w.chain->pub;
    p.reset = w.chain->reset;
    p.exit_count = w.chain->exit_count;
  }
  if (partial_bytes(pl, Cfg::BN, Cfg::NB, Cfg::CTAS) > w.partial_cap) return SVDMLP_ERR_WORKSPACE;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = Cfg::CTAS;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  TimedLaunch* tl = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    if (g_timing && g_timed_used < g_timed.size()) {
      tl = &g_timed[g_timed_used++];
      tl->stage = stage;
    }
  }
  if (tl) SVD_CUDA(cudaEventRecord(tl->start, stream));
  SVD_CUDA(cudaLaunchKernelEx(&cfg, gemm_sm100_kernel<Cfg>, a, a2, b, b2, out, out2, p));
  if (tl) SVD_CUDA(cudaEventRecord(tl->stop, stream));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SVDMLP_OK;
}

template <class Cfg>
static int launch_gemv(const CUtensorMap& x, const CUtensorMap& x2, const CUtensorMap& wm, const CUtensorMap& wm2,
                       void* out, int64_t ld_out, int M, int N, int K, int stage, const Workspace& w,
                       const bf16* residual, int64_t ld_res, cudaStream_t stream) {
  DeviceInfo* dev = nullptr;
  SVD_CHECK(device_info(&dev));
  static std::mutex mu;
  {
    int cur = 0;
    SVD_CUDA(cudaGetDevice(&cur));
    static uint64_t done_mask = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!(done_mask & (1ull << cur))) {
      SVD_CUDA(cudaFuncSetAttribute(gemv_sm100_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::SMEM_BYTES));
      SVD_CUDA(cudaFuncSetAttribute(gemv_sm100_kernel<Cfg>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
      done_mask |= 1ull << cur;
    }
  }
  Plan pl = plan_dec<Cfg>(M, N, K, dev->sms, g_split_override[stage]);
  if (dec_partial_bytes<Cfg>(pl) > w.partial_cap) {
    if (!w.unsplit_if_short) return SVDMLP_ERR_WORKSPACE;
    pl = plan_dec<Cfg>(M, N, K, dev->sms, 1);
  }
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = 1;
  p.n_tiles = pl.n_tiles;
  p.k_blocks = pl.k_blocks;
  p.splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.num_units = pl.units;
  p.tail_start = pl.units;
  p.tail_splits = 1;
  p.norm_stats = w.norm_stats;
  p.norm_parts = w.norm_parts;
  p.norm_dim = w.norm_dim;
  p.norm_eps = w.norm_eps;
  p.stats_ld = w.stats_ld;
  p.out_stats = w.out_stats;
  p.partials = w.partials;
  p.counters = w.counters;
  p.err = w.err;
  p.timeout_ns = g_wait_limit_ns;
  p.residual = residual;
  p.ld_residual = ld_res;
  if (w.push != nullptr) return SVDMLP_ERR_INVALID_VALUE;  // the fused exchange runs on the CTA-pair GEMM only
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TimedLaunch* tl = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    if (g_timing && g_timed_used < g_timed.size()) {
      tl = &g_timed[g_timed_used++];
      tl->stage = stage;
    }
  }
  if (tl) SVD_CUDA(cudaEventRecord(tl->start, stream));
  SVD_CUDA(cudaLaunchKernelEx(&cfg, gemv_sm100_kernel<Cfg>, x, x2, wm, wm2, out, static_cast<long long>(ld_out), p));
  if (tl) SVD_CUDA(cudaEventRecord(tl->stop, stream));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SVDMLP_OK;
}

// ----------------------------------------------------------- small kernels
template <typename T>
SVD_DEV T from_float(float v);
template <>
SVD_DEV bf16 from_float<bf16>(float v) { return __float2bfloat16(v); }
template <>
SVD_DEV __half from_float<__half>(float v) { return __float2half_rn(fminf(fmaxf(v, -65504.f), 65504.f)); }

// Conversion to the stored type that also reports values fp16 cannot hold
// (|v| > 65504 or NaN) in `*range`: they are saturated, never silently.
template <typename TO>
SVD_DEV TO checked_from_float(float v, int* range) {
  if constexpr (std::is_same<TO, __half>::value) {
    if (range != nullptr && f16_out_of_range(v)) atomicOr(range, 1);
  }
  return from_float<TO>(v);
}

// dst[i][j] = src[j][i] (bf16 in, bf16 or fp16 out); zero outside the source.
template <typename TO>
__global__ void transpose_pack_kernel(const bf16* __restrict__ src, long long ld_src, int rows, int cols,
                                      TO* __restrict__ dst, long long ld_dst, int dst_rows, int dst_cols) {
  __shared__ float tile[32][33];
  const int i0 = blockIdx.y * 32;  // dst rows  == src columns
  const int j0 = blockIdx.x * 32;  // dst cols  == src rows
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int j = j0 + k, i = i0 + threadIdx.x;
    tile[k][threadIdx.x] = (j < rows && i < cols) ? __bfloat162float(src[static_cast<long long>(j) * ld_src + i]) : 0.f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int i = i0 + k, j = j0 + threadIdx.x;
    if (i < dst_rows && j < dst_cols) dst[static_cast<long long>(i) * ld_dst + j] = from_float<TO>(tile[threadIdx.x][k]);
  }
}

// Packs src [rows, cols] (row-major bf16) transposed into rows [row0,
// row0 + cols) of a tiled K-major matrix with K = rows: element (n, k) of the
// destination is src[k][n - row0], stored at tile (n / 16, k / 64), offset
// (n % 16) * 64 + k % 64.  `kb_count` is the number of 64-column k-blocks of
// the destination; destination columns k >= rows are written as zero.
// `kscale` (nullable): each source row k is multiplied by kscale[k] in fp32
// before the conversion (a decoder block's RMSNorm weight folded into the
// first factors).
template <typename TO>
__global__ void tiled_pack_kernel(const bf16* __restrict__ src, long long ld_src, int rows, int cols,
                                  TO* __restrict__ dst, int row0, int kb_count, int* range,
                                  const bf16* __restrict__ kscale) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.x * 32;  // destination column (k) == source row
  const int n0 = blockIdx.y * 32;  // destination row offset within [0, cols)
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int k = k0 + y, n = n0 + threadIdx.x;
    float val = (k < rows && n < cols) ? __bfloat162float(src[static_cast<long long>(k) * ld_src + n]) : 0.f;
    if (kscale != nullptr && k < rows) val *= __bfloat162float(kscale[k]);
    tile[y][threadIdx.x] = val;
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int n = n0 + y, k = k0 + threadIdx.x;
    if (n < cols && k < kb_count * 64) {
      const int gn = row0 + n;
      const long long off = (static_cast<long long>(gn / 16) * kb_count + k / 64) * 1024 + (gn % 16) * 64 + (k % 64);
      dst[off] = checked_from_float<TO>(tile[threadIdx.x][y], range);
    }
  }
}

// 2-D element-wise conversion with leading dimensions (fp32 -> fp16, bf16 -> fp16).
template <typename TI, typename TO>
__global__ void convert_kernel(const TI* __restrict__ src, long long ld_src, TO* __restrict__ dst, long long ld_dst,
                               int rows, int cols, int* range) {
  const long long total = static_cast<long long>(rows) * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols, c = i % cols;
    float v;
    if constexpr (std::is_same<TI, float>::value) v = src[r * ld_src + c];
    else v = __bfloat162float(src[r * ld_src + c]);
    dst[r * ld_dst + c] = checked_from_float<TO>(v, range);
  }
}

__global__ void rmsnorm_kernel(const bf16* __restrict__ x, long long ld_x, const bf16* __restrict__ w,
                               bf16* __restrict__ y, long long ld_y, int n, float eps) {
  const bf16* xr = x + static_cast<long long>(blockIdx.x) * ld_x;
  bf16* yr = y + static_cast<long long>(blockIdx.x) * ld_y;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __bfloat162float(xr[i]);
    ss += v * v;
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    yr[i] = __float2bfloat16(__bfloat162float(xr[i]) * rstd * __bfloat162float(w[i]));
}

// Per row of x [M, n], the sum of squares of each 128-column slice:
// stats[row * ld_stats + slice] (the statistics a block's fused RMSNorm reads
// for the first block of a stack; later blocks get them from the previous
// block's residual epilogue).  One CTA per row, a warp per slice.
__global__ void row_sumsq_kernel(const bf16* __restrict__ x, long long ld_x, int n, float* __restrict__ stats,
                                 long long ld_stats) {
  const bf16* xr = x + static_cast<long long>(blockIdx.x) * ld_x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int slices = (n + 127) / 128;
  for (int sl = warp; sl < slices; sl += nwarps) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = sl * 128 + j * 32 + lane;
      const float v = c < n ? __bfloat162float(xr[c]) : 0.f;
      ss += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) stats[static_cast<long long>(blockIdx.x) * ld_stats + sl] = ss;
  }
}

// One CTA that waits, bounded, on an mbarrier nothing will complete.
__global__ void wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtx ctx{&abort_flag, err, limit_ns};
    mbar_wait(&bar, 0, ctx, SITE_PROBE);
  }
}

template <typename TI, typename TO>
static int launch_convert(const TI* src, int64_t ld_src, TO* dst, int64_t ld_dst, int rows, int cols, int* range,
                          cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(rows) * cols;
  const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(cdiv(total, 256), 148 * 16)));
  convert_kernel<TI, TO><<<blocks, 256, 0, s>>>(src, ld_src, dst, ld_dst, rows, cols, range);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

template <typename TO>
static int launch_tiled_pack(const void* src, int64_t ld_src, int rows, int cols, void* dst, int row0, int64_t k,
                             int* range, cudaStream_t s, const void* kscale = nullptr) {
  if (!src || !dst || rows <= 0 || cols <= 0 || ld_src < cols || row0 % 16 != 0) return SVDMLP_ERR_INVALID_VALUE;
  const int kb = static_cast<int>(cdiv(k, 64));
  dim3 grid(static_cast<unsigned>(cdiv(static_cast<int64_t>(kb) * 64, 32)), static_cast<unsigned>(cdiv(cols, 32)));
  tiled_pack_kernel<TO><<<grid, dim3(32, 8), 0, s>>>(static_cast<const bf16*>(src), ld_src, rows, cols,
                                                     static_cast<TO*>(dst), row0, kb, range,
                                                     static_cast<const bf16*>(kscale));
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

template <typename TO>
static int launch_transpose(const void* src, int64_t ld_src, int rows, int cols, void* dst, int64_t ld_dst,
                            int dst_rows, int dst_cols, cudaStream_t s) {
  if (!src || !dst || rows <= 0 || cols <= 0 || dst_rows <= 0 || dst_cols <= 0 || ld_src < cols ||
      ld_dst < dst_cols)
    return SVDMLP_ERR_INVALID_VALUE;
  dim3 grid(static_cast<unsigned>(cdiv(dst_cols, 32)), static_cast<unsigned>(cdiv(dst_rows, 32)));
  transpose_pack_kernel<TO><<<grid, dim3(32, 8), 0, s>>>(static_cast<const bf16*>(src), ld_src, rows, cols,
                                                         static_cast<TO*>(dst), ld_dst, dst_rows, dst_cols);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

// ------------------------------------------------------------ validation
static bool aligned16(const void* p, int64_t ld) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && ld % 8 == 0;
}

static int check_layout(const svdmlp_layout* L) {
  if (!L || L->d <= 0 || L->ff <= 0) return SVDMLP_ERR_INVALID_VALUE;
  if (L->kind != SVDMLP_KIND_SVD && L->kind != SVDMLP_KIND_DENSE) return SVDMLP_ERR_INVALID_VALUE;
  return SVDMLP_OK;
}

// Brings a bf16 activation matrix to a TMA-legal buffer (16-byte aligned
// rows), copying it into workspace staging when the caller's stride is not.
static int stage_in(const void* src, int64_t ld, int rows, int cols, void* staging, int64_t ld_staging,
                    const void** out, int64_t* out_ld, cudaStream_t s) {
  if (aligned16(src, ld)) {
    *out = src;
    *out_ld = ld;
    return SVDMLP_OK;
  }
  SVD_CUDA(cudaMemcpy2DAsync(staging, ld_staging * 2, src, ld * 2, static_cast<size_t>(cols) * 2, rows,
                             cudaMemcpyDeviceToDevice, s));
  *out = staging;
  *out_ld = ld_staging;
  return SVDMLP_OK;
}

static int finish_output(void* target, int64_t ld_target, const void* staged, int64_t ld_staged, int M, int cols,
                         cudaStream_t s) {
  if (staged == target) return SVDMLP_OK;
  SVD_CUDA(cudaMemcpy2DAsync(target, ld_target * 2, staged, ld_staged * 2, static_cast<size_t>(cols) * 2, M,
                             cudaMemcpyDeviceToDevice, s));
  return SVDMLP_OK;
}

// ------------------------------------------------------------------ stages
// A K-major operand: `rows` rows of `k` 16-bit elements, leading dim `ld`.
struct Operand {
  const void* ptr;
  bool f16;
  int64_t k, rows, ld;
};
struct Output {
  void* ptr;
  int64_t n, rows, ld;
};

template <class Cfg>
static int gemm_cfg(const Operand& a, const Operand& a2, const Operand& b, const Operand& b2, const Output& o, int M,
                    int N, int K, int stage, const Workspace& w, const void* residual, int64_t ld_res,
                    cudaStream_t s, const Output* o2 = nullptr) {
  CUtensorMap ma, ma2, mb, mb2, mo, mo2;
  SVD_CHECK(operand_map(&ma, a.ptr, a.f16, a.k, a.rows, a.ld, Cfg::BM));
  SVD_CHECK(operand_map(&ma2, a2.ptr, a2.f16, a2.k, a2.rows, a2.ld, Cfg::BM));
  if constexpr (Cfg::B_TILED) {
    SVD_CHECK(tiled_map(&mb, b.ptr, b.f16, b.rows, b.k, Cfg::B_ROWS));
    SVD_CHECK(tiled_map(&mb2, b2.ptr, b2.f16, b2.rows, b2.k, Cfg::B_ROWS));
  } else {
    SVD_CHECK(operand_map(&mb, b.ptr, b.f16, b.k, b.rows, b.ld, Cfg::B_ROWS));
    SVD_CHECK(operand_map(&mb2, b2.ptr, b2.f16, b2.k, b2.rows, b2.ld, Cfg::B_ROWS));
  }
  SVD_CHECK(output_map<Cfg>(&mo, o.ptr, o.n, o.rows, o.ld));
  if (o2) SVD_CHECK(output_map<Cfg>(&mo2, o2->ptr, o2->n, o2->rows, o2->ld));
  else mo2 = mo;
  return launch_gemm<Cfg>(ma, ma2, mb, mb2, mo, mo2, M, N, K, stage, w, static_cast<const bf16*>(residual), ld_res,
                          s);
}

// Runs one GEMM stage with the CTA-pair config for prefill-sized M and the
// one-CTA split-K config for decode-sized M.
template <class CPair, class COne>
static int gemm_stage(const Operand& a, const Operand& a2, const Operand& b, const Operand& b2, const Output& o,
                      int M, int N, int K, int stage, const Workspace& w, cudaStream_t s,
                      const void* residual = nullptr, int64_t ld_res = 0) {
  if (M >= g_pair_min_m) return gemm_cfg<CPair>(a, a2, b, b2, o, M, N, K, stage, w, residual, ld_res, s);
  return gemm_cfg<COne>(a, a2, b, b2, o, M, N, K, stage, w, residual, ld_res, s);
}

template <class Cfg>
static int gemv_cfg(const Operand& x, const Operand& x2, const Operand& wt, const Operand& wt2, const Output& o, int M,
                    int N, int K, int stage, const Workspace& w, const void* residual, int64_t ld_res,
                    cudaStream_t s) {
  CUtensorMap mx, mx2, mw, mw2;
  SVD_CHECK(operand_map(&mx, x.ptr, x.f16, x.k, x.rows, x.ld, Cfg::TOK));
  SVD_CHECK(operand_map(&mx2, x2.ptr, x2.f16, x2.k, x2.rows, x2.ld, Cfg::TOK));
  SVD_CHECK(tiled_map(&mw, wt.ptr, wt.f16, wt.rows, wt.k, Cfg::BM));
  SVD_CHECK(tiled_map(&mw2, wt2.ptr, wt2.f16, wt2.rows, wt2.k, Cfg::BM));
  const int64_t elt = Cfg::OUT == OUT_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(o.ptr) % elt) != 0) return SVDMLP_ERR_ALIGNMENT;
  return launch_gemv<Cfg>(mx, mx2, mw, mw2, o.ptr, o.ld, M, N, K, stage, w, static_cast<const bf16*>(residual), ld_res,
                          s);
}

// Like gemm_stage, with the swapped-operand streaming kernels for M <= 128:
// `Pick` maps a DecSet to the stage's config.
template <class CPair, template <class> class Pick>
static int gemm_stage_dec(const Operand& a, const Operand& a2, const Operand& b, const Operand& b2, const Output& o,
                          int M, int N, int K, int stage, const Workspace& w, cudaStream_t s,
                          const void* residual = nullptr, int64_t ld_res = 0) {
  if (M >= g_pair_min_m) return gemm_cfg<CPair>(a, a2, b, b2, o, M, N, K, stage, w, residual, ld_res, s);
  if (M <= 16) return gemv_cfg<Pick<Dec16>>(a, a2, b, b2, o, M, N, K, stage, w, residual, ld_res, s);
  if (M <= 64) return gemv_cfg<Pick<Dec64>>(a, a2, b, b2, o, M, N, K, stage, w, residual, ld_res, s);
  return gemv_cfg<Pick<Dec128>>(a, a2, b, b2, o, M, N, K, stage, w, residual, ld_res, s);
}
template <class S> using PickXU = typename S::XU;
template <class S> using PickGU = typename S::GU;
template <class S> using PickDU = typename S::DU;
template <class S> using PickDUf32 = typename S::DUf32;
template <class S> using PickDV = typename S::DV;
template <class S> using PickDVres = typename S::DVres;
template <class S> using PickDGU = typename S::DGU;

// Stage 1 + 2: h = silu(X.u_g.v_g) * (X.u_u.v_u); `h_bf16` selects the
// caller-facing bf16 output instead of the internal fp16 H.
// XU = X . [u_g|u_u]  (fp16, [M, 2 rp_gu])
static int run_xu(const svdmlp_layout* L, const uint8_t* packed, const void* x, int64_t ldx, int M,
                  const Workspace& w, cudaStream_t s, void* xu_out = nullptr, int64_t ld_xu = 0) {
  const int64_t n1 = 2LL * L->rp_gu;
  const Operand xa{x, false, L->d, M, ldx};
  __half* xu = xu_out ? static_cast<__half*>(xu_out) : w.xu;  // the workspace's XU or a caller's buffer
  const int64_t ldo = xu_out ? ld_xu : n1;
  if (M >= g_pair_min_m) {
    // the two halves of the packed w1 (rp_gu is a whole number of 16-row groups)
    const uint8_t* w1 = packed + L->off_w1;
    const Operand wg{w1, false, L->d, L->rp_gu, L->ld_d};
    const Operand wu{w1 + tiled_bytes(L->rp_gu, L->d), false, L->d, L->rp_gu, L->ld_d};
    const Output og{xu, L->rp_gu, M, ldo};
    const Output ou{xu + L->rp_gu, L->rp_gu, M, ldo};
    return gemm_cfg<CfgXUd>(xa, xa, wg, wu, og, M, L->rp_gu, L->d, ST_XU, w, nullptr, 0, s, &ou);
  }
  const Operand w1{packed + L->off_w1, false, L->d, n1, L->ld_d};
  return gemm_stage_dec<CfgXU, PickXU>(xa, xa, w1, w1, Output{xu, n1, M, ldo}, M, static_cast<int>(n1), L->d,
                                       ST_XU, w, s);
}

// H = silu(XU_g . v_g) * (XU_u . v_u)
static int run_gu(const svdmlp_layout* L, const uint8_t* packed, int M, void* h, int64_t ldh, bool h_bf16,
                  const Workspace& w, cudaStream_t s, const void* xu_in = nullptr, int64_t ld_xu = 0) {
  const int64_t n1 = 2LL * L->rp_gu;
  const __half* xu = xu_in ? static_cast<const __half*>(xu_in) : w.xu;
  const int64_t ldi = xu_in ? ld_xu : n1;
  const Operand ag{xu, true, L->r_gu, M, ldi};
  const Operand au{xu + L->rp_gu, true, L->r_gu, M, ldi};
  const Operand bg{packed + L->off_vg, true, L->r_gu, L->ff, L->rp_gu};
  const Operand bu{packed + L->off_vu, true, L->r_gu, L->ff, L->rp_gu};
  const Output ho{h, L->ff, M, ldh};
  if (h_bf16) return gemm_stage<CfgGUbf, CfgGUbf1>(ag, au, bg, bu, ho, M, L->ff, L->r_gu, ST_GATEUP, w, s);
  return gemm_stage_dec<CfgGU, PickGU>(ag, au, bg, bu, ho, M, L->ff, L->r_gu, ST_GATEUP, w, s);
}

static int run_gate_up(const svdmlp_layout* L, const uint8_t* packed, const void* x, int64_t ldx, int M, void* h,
                       int64_t ldh, bool h_bf16, const Workspace& w, cudaStream_t s) {
  SVD_CHECK(run_xu(L, packed, x, ldx, M, w, s));
  return run_gu(L, packed, M, h, ldh, h_bf16, w, s);
}

// Stage 3: H . u_down -> T (fp16, workspace) or an fp32 partial.  `h_f16`
// says whether H is fp16 (it must then match an fp16 ud) or bf16 (bf16 ud).
// T = H . u_down into the workspace, or into a caller's fp32 (`partial`) or
// fp16 (`partial16`) buffer for the tensor-parallel all-reduce.
static int run_down_u(const svdmlp_layout* L, const uint8_t* packed, const void* h, int64_t ldh, bool h_f16, int M,
                      float* partial, int64_t ldp, const Workspace& w, cudaStream_t s, void* partial16 = nullptr) {
  const Operand ha{h, h_f16, L->ff, M, ldh};
  const Operand ud{packed + L->off_ud, h_f16, L->ff, L->r_d, L->ld_ff};
  if (partial16) {
    if (!h_f16) return SVDMLP_ERR_DTYPE;
    return gemm_stage_dec<CfgDU, PickDU>(ha, ha, ud, ud, Output{partial16, L->r_d, M, ldp}, M, L->r_d, L->ff,
                                         ST_DOWN_U, w, s);
  }
  if (partial) {
    if (!h_f16) return SVDMLP_ERR_DTYPE;
    return gemm_stage_dec<CfgDUf32, PickDUf32>(ha, ha, ud, ud, Output{partial, L->r_d, M, ldp}, M, L->r_d, L->ff,
                                               ST_DOWN_U, w, s);
  }
  const Output to{w.t, L->r_d, M, L->rp_d};
  if (h_f16) return gemm_stage_dec<CfgDU, PickDU>(ha, ha, ud, ud, to, M, L->r_d, L->ff, ST_DOWN_U, w, s);
  return gemm_stage<CfgDUbf, CfgDUbf1>(ha, ha, ud, ud, to, M, L->r_d, L->ff, ST_DOWN_U, w, s);
}

// Stage 4: T . v_down (+ residual) -> y (bf16)
// y = T . v_down (+ residual), T the workspace's fp16 T or a caller's fp16 buffer.
static int run_down_v(const svdmlp_layout* L, const uint8_t* packed, int M, void* y, int64_t ldy,
                      const void* residual, int64_t ld_res, const Workspace& w, cudaStream_t s,
                      const void* t = nullptr, int64_t ldt = 0) {
  const Operand ta{t ? t : w.t, true, L->r_d, M, t ? ldt : L->rp_d};
  const Operand vd{packed + L->off_vd, true, L->r_d, L->d, L->rp_d};
  const Output yo{y, L->d, M, ldy};
  if (residual)
    return gemm_stage_dec<CfgDVres, PickDVres>(ta, ta, vd, vd, yo, M, L->d, L->r_d, ST_DOWN_V, w, s, residual,
                                               ld_res);
  return gemm_stage_dec<CfgDV, PickDV>(ta, ta, vd, vd, yo, M, L->d, L->r_d, ST_DOWN_V, w, s);
}

// Dense SwiGLU: H = silu(X.w_g) * (X.w_u) (fp16), y = H.w_d (+ residual).
static int run_dense(const svdmlp_layout* L, const uint8_t* packed, const void* x, int64_t ldx, int M, void* y,
                     int64_t ldy, const void* residual, int64_t ld_res, const Workspace& w, cudaStream_t s) {
  const Operand xa{x, false, L->d, M, ldx};
  const Operand bg{packed + L->off_vg, false, L->d, L->ff, L->ld_d};
  const Operand bu{packed + L->off_vu, false, L->d, L->ff, L->ld_d};
  // below the CTA-pair threshold both stages stream their weights on the
  // swapped-operand decode kernels, as the SVD layer's stages do
  SVD_CHECK(gemm_stage_dec<CfgDenseGU, PickDGU>(xa, xa, bg, bu, Output{w.h, L->ff, M, L->ld_ff}, M, L->ff, L->d,
                                               ST_DENSE_GU, w, s));
  const Operand ha{w.h, true, L->ff, M, L->ld_ff};
  const Operand bd{packed + L->off_ud, true, L->ff, L->d, L->ld_ff};
  const Output yo{y, L->d, M, ldy};
  if (residual)
    return gemm_stage_dec<CfgDVres, PickDVres>(ha, ha, bd, bd, yo, M, L->d, L->ff, ST_DENSE_D, w, s, residual,
                                               ld_res);
  return gemm_stage_dec<CfgDV, PickDV>(ha, ha, bd, bd, yo, M, L->d, L->ff, ST_DENSE_D, w, s);
}

// The whole layer for M <= 64 in one persistent launch (layer_decode_sm100.cuh).
//
// The launch is an ordinary one, not a cooperative one.  A CTA only ever waits
// for units claimed before its own, and only running CTAs claim units, so the
// earliest unfinished unit always has its inputs complete and the grid makes
// progress however many of its CTAs are resident.  (The runtime's occupancy
// query reports one CTA per SM for every kernel that allocates tensor memory,
// which would cap a cooperative grid at one CTA per SM; the hardware runs as
// many as shared memory and the 512 TMEM columns allow.)
template <int TOK, int STAGES>
static int launch_layer_decode(LayerDecParams& prm, cudaStream_t s, int sms) {
  using Cfg = LayerDecCfg<TOK, STAGES>;
  static std::mutex mu;
  int cur = 0;
  SVD_CUDA(cudaGetDevice(&cur));
  {
    static uint64_t done_mask = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!(done_mask & (1ull << cur))) {
      SVD_CUDA(cudaFuncSetAttribute(layer_decode_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::SMEM_BYTES));
      // all of the unified L1/shared storage as shared memory: two CTAs per SM
      SVD_CUDA(cudaFuncSetAttribute(layer_decode_kernel<Cfg>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
      done_mask |= 1ull << cur;
    }
  }
  int smem_sm = 0, smem_resv = 0;
  SVD_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, cur));
  SVD_CUDA(cudaDeviceGetAttribute(&smem_resv, cudaDevAttrReservedSharedMemoryPerBlock, cur));
  const int by_smem = smem_sm / (Cfg::SMEM_BYTES + smem_resv);
  const int by_tmem = 512 / static_cast<int>(Cfg::TMEM_COLS);
  const int per_sm = std::min(kLayerDecodeCtasPerSm, std::min(by_smem, by_tmem));
  if (per_sm < 1) return SVDMLP_ERR_BUDGET;
  const int grid = std::min(prm.total_units, per_sm * sms);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_layer_decode_pdl > 0 ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TimedLaunch* tl = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    if (g_timing && g_timed_used < g_timed.size()) {
      tl = &g_timed[g_timed_used++];
      tl->stage = ST_LAYER_DECODE;
    }
  }
  if (tl) SVD_CUDA(cudaEventRecord(tl->start, s));
  SVD_CUDA(cudaLaunchKernelEx(&cfg, layer_decode_kernel<Cfg>, prm));
  if (tl) SVD_CUDA(cudaEventRecord(tl->stop, s));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SVDMLP_OK;
}

// `contract`: the contracted schedule (16-token tiles, full layers with fp16
// u_down): stage 1 runs CONTRACT units (SwiGLU tile -> shared memory ->
// . u_down, fp32 T partials per ff tile), stage 2 REDUCE units (T summed in
// tile order, rounded to fp16 once), stage 3 T . v_down as usual.
static int run_layer_decode(const svdmlp_layout* L, const uint8_t* P, const void* x, int64_t ldx, int M, void* y,
                            int64_t ldy, const void* residual, int64_t ld_res, const Workspace& w, cudaStream_t s,
                            bool contract = false) {
  DeviceInfo* dev = nullptr;
  SVD_CHECK(device_info(&dev));
  const int tok = M <= 16 ? 16 : 64;
  contract = contract && tok == 16 && L->ud_f16 != 0;
  const int slots = kLayerDecodeCtasPerSm * dev->sms;  // the planning grid; the launch checks that it fits
  LayerDecParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.num_stages = 4;
  prm.M = M;
  prm.err = w.err;
  prm.timeout_ns = g_wait_limit_ns;
  prm.residual = static_cast<const bf16*>(residual);
  prm.ld_residual = ld_res;
  prm.done = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(w.err) + 64);
  prm.exit_count = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(w.err) + 96);
  prm.next_unit = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(w.err) + 128);
  prm.trace = g_trace;
  prm.pf_ahead = g_pf_ahead;
  prm.pf_wait = g_pf_wait;
  prm.pdl_units = std::max(0, g_layer_decode_pdl - 1);
  prm.norm_stats = w.norm_stats;
  prm.norm_parts = w.norm_parts;
  prm.norm_dim = w.norm_dim;
  prm.norm_eps = w.norm_eps;
  prm.stats_ld = w.stats_ld;
  const int64_t n1 = 2LL * L->rp_gu;
  // stage operands: token tiles (box TOK rows) and weight panels (box 128 rows)
  struct Spec {
    const void *x, *x2;
    bool xf16;
    int64_t xk, xld;
    const void *w, *w2;
    int64_t wrows, wld;
    void* out;
    int64_t ld_out;
    int nb, epi, out_kind;
  } spec[4] = {
      {x, x, false, L->d, ldx, P + L->off_w1, P + L->off_w1, n1, L->ld_d, w.xu, n1, 1, EPI_PLAIN, OUT_F16},
      {w.xu, w.xu + L->rp_gu, true, L->r_gu, n1, P + L->off_vg, P + L->off_vu, L->ff, L->rp_gu, w.h, L->ld_ff, 2,
       EPI_SWIGLU, OUT_F16},
      {w.h, w.h, true, L->ff, L->ld_ff, P + L->off_ud, P + L->off_ud, L->r_d, L->ld_ff, w.t, L->rp_d, 1, EPI_PLAIN,
       OUT_F16},
      {w.t, w.t, true, L->r_d, L->rp_d, P + L->off_vd, P + L->off_vd, L->d, L->rp_d, y, ldy, 1,
       residual ? EPI_RESID : EPI_PLAIN, OUT_BF16},
  };
  float* part = w.partials;
  int64_t part_left = w.partial_cap;
  int base = 0;
  for (int st = 0; st < 4; ++st) {
    DecStage& d = prm.st[st];
    const Spec& sp = spec[st];
    d.kind = KIND_GEMM;
    if (contract && st == 2) {
      // REDUCE: 32 features of T per unit, reading stage 1's partials
      const DecStage& c1 = prm.st[1];
      d.kind = KIND_REDUCE;
      d.out = w.t;
      d.ld_out = L->rp_d;
      d.N = L->r_d;
      d.n_tiles = static_cast<int>(cdiv(L->r_d, 32));
      d.splits = 1;
      d.units = d.n_tiles;
      d.unit_base = base;
      d.t_slots = c1.n_tiles;
      d.t_ld = c1.t_ld;
      d.tpart = c1.tpart;
      d.out_kind = OUT_F16;
      base += d.units;
      continue;
    }
    SVD_CHECK(operand_map(&d.x, sp.x, sp.xf16, sp.xk, M, sp.xld, tok));
    SVD_CHECK(operand_map(&d.x2, sp.x2, sp.xf16, sp.xk, M, sp.xld, tok));
    SVD_CHECK(tiled_map(&d.w, sp.w, sp.xf16, sp.wrows, sp.xk, 128));
    SVD_CHECK(tiled_map(&d.w2, sp.w2, sp.xf16, sp.wrows, sp.xk, 128));
    const int N = static_cast<int>(st == 0 ? n1 : sp.wrows);
    const int K = static_cast<int>(sp.xk);
    const bool con = contract && st == 1;
    // CONTRACT units hold a whole ff tile (the SwiGLU needs full sums)
    Plan pl = plan_layer_stage(M, tok, N, K, sp.nb, slots, con ? 1 : g_split_override[st]);
    int64_t pb = pl.splits > 1 ? round_up(static_cast<int64_t>(pl.units) * 2 * 128 * tok * 4, 256) : 0;
    if (con) {
      d.kind = KIND_CONTRACT;
      SVD_CHECK(tiled_map(&d.w3, P + L->off_ud, true, L->r_d, L->ff, 128));
      d.r_tiles = static_cast<int>(cdiv(L->r_d, 128));
      d.ff_kb = static_cast<int>(cdiv(L->ff, 64));
      d.t_ld = static_cast<int>(round_up(L->r_d, 128));
      pb = contract_partials(L);
      if (pb > part_left) return SVDMLP_ERR_WORKSPACE;
      d.tpart = part;
    }
    if (pb > part_left) {
      if (!w.unsplit_if_short) return SVDMLP_ERR_WORKSPACE;
      pl = plan_layer_stage(M, tok, N, K, sp.nb, slots, 1);
      pb = 0;
    }
    d.out = con ? nullptr : sp.out;
    d.norm = (st == 0 && w.norm_stats != nullptr) ? 1 : 0;
    d.out_stats = st == 3 ? w.out_stats : nullptr;
    d.ld_out = sp.ld_out;
    d.partials = part;
    d.tile_counters = w.counters + st * 65536;
    d.N = N;
    d.K = K;
    d.n_tiles = pl.n_tiles;
    d.k_blocks = pl.k_blocks;
    d.splits = pl.splits;
    d.kb_per_split = pl.kb_per_split;
    d.units = pl.units;
    d.unit_base = base;
    d.nb = sp.nb;
    d.in_f16 = sp.xf16 ? 1 : 0;
    d.epi = sp.epi;
    d.out_kind = sp.out_kind;
    base += pl.units;
    part += pb / 4;
    part_left -= pb;
  }
  prm.total_units = prm.st[prm.num_stages - 1].unit_base + prm.st[prm.num_stages - 1].units;
  if (tok == 16) return launch_layer_decode<16, SVDMLP_LD_RING16>(prm, s, dev->sms);
  return launch_layer_decode<64, SVDMLP_LD_RING64>(prm, s, dev->sms);
}

// Output target: the caller's buffer when TMA-legal, else workspace staging.
struct OutTarget {
  void* ptr;
  int64_t ld;
};
static OutTarget out_target(void* y, int64_t ldy, void* staging, int64_t ld_staging) {
  if (aligned16(y, ldy)) return {y, ldy};
  return {staging, ld_staging};
}

}  // namespace svdmlp

using namespace svdmlp;

// =================================================================== C ABI
extern "C" {

const char* svdmlp_status_string(int status) {
  switch (status) {
    case SVDMLP_OK: return "ok";
    case SVDMLP_ERR_INVALID_VALUE: return "invalid value: sizes must be positive integers and pointers non-null";
    case SVDMLP_ERR_SHAPE_MISMATCH: return "shape mismatch: contraction dimensions do not match";
    case SVDMLP_ERR_ALIGNMENT: return "alignment: pointers and leading dimensions must be 16-byte aligned";
    case SVDMLP_ERR_DTYPE: return "unsupported dtype: inputs must all be bfloat16";
    case SVDMLP_ERR_WORKSPACE: return "workspace too small";
    case SVDMLP_ERR_DEVICE_TIMEOUT: return "device-side wait exceeded its limit";
    case SVDMLP_ERR_CUDA: return "CUDA error";
    case SVDMLP_ERR_BUDGET: return "SMEM/TMEM budget exceeds the device";
    case SVDMLP_ERR_DEVICE: return "device is not an sm_100 (B200) GPU";
    case SVDMLP_ERR_RANGE:
      return "value out of fp16 range: an intermediate or an fp16-packed weight exceeded 65504 (or was NaN) and was "
             "saturated";
    default: return "unknown status";
  }
}

int svdmlp_last_cuda_error(void) { return g_last_cuda_error; }

int64_t svdmlp_launch_count(void) { return g_launches.load(); }

int svdmlp_layout_init(svdmlp_layout* L, int d, int ff, int r_gu, int r_d) {
  if (!L || d <= 0 || ff <= 0 || r_gu < 0 || r_d < 0 || (r_gu == 0 && r_d == 0)) return SVDMLP_ERR_INVALID_VALUE;
  std::memset(L, 0, sizeof(*L));
  L->kind = SVDMLP_KIND_SVD;
  L->d = d;
  L->ff = ff;
  L->r_gu = r_gu;
  L->r_d = r_d;
  L->rp_gu = static_cast<int32_t>(round_up(r_gu, 16));  // the up half of w1 starts on a 16-row group
  L->rp_d = static_cast<int32_t>(round_up(r_d, 8));
  L->ld_d = static_cast<int32_t>(round_up(d, 8));
  L->ld_ff = static_cast<int32_t>(round_up(ff, 8));
  L->ud_f16 = r_gu > 0 ? 1 : 0;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += round_up(bytes, 256);
    return o;
  };
  L->off_w1 = take(tiled_bytes(2LL * L->rp_gu, d));  // [2*rp_gu, d]
  L->off_vg = take(tiled_bytes(ff, r_gu));            // [ff, r_gu]
  L->off_vu = take(tiled_bytes(ff, r_gu));
  L->off_ud = take(tiled_bytes(r_d, ff));             // [r_d, ff]
  L->off_vd = take(tiled_bytes(d, r_d));              // [d, r_d]
  L->off_status = take(kPackStatusBytes);             // pack status word (fp16 range)
  L->packed_bytes = off;
  return SVDMLP_OK;
}

int svdmlp_dense_layout_init(svdmlp_layout* L, int d, int ff) {
  if (!L || d <= 0 || ff <= 0) return SVDMLP_ERR_INVALID_VALUE;
  std::memset(L, 0, sizeof(*L));
  L->kind = SVDMLP_KIND_DENSE;
  L->d = d;
  L->ff = ff;
  L->ld_d = static_cast<int32_t>(round_up(d, 8));
  L->ld_ff = static_cast<int32_t>(round_up(ff, 8));
  L->ud_f16 = 1;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += round_up(bytes, 256);
    return o;
  };
  L->off_vg = take(tiled_bytes(ff, d));  // [ff, d]
  L->off_vu = take(tiled_bytes(ff, d));
  L->off_ud = take(tiled_bytes(d, ff));  // [d, ff]
  L->off_status = take(kPackStatusBytes);
  L->packed_bytes = off;
  return SVDMLP_OK;
}

int svdmlp_transpose_pack(const void* src, int64_t ld_src, int rows, int cols, void* dst, int64_t ld_dst,
                          int dst_rows, int dst_cols, void* stream) {
  return launch_transpose<bf16>(src, ld_src, rows, cols, dst, ld_dst, dst_rows, dst_cols,
                                static_cast<cudaStream_t>(stream));
}

static int pack_impl(const svdmlp_layout* L, const void* u_gate, int64_t ld_ug, const void* v_gate, int64_t ld_vg,
                     const void* u_up, int64_t ld_uu, const void* v_up, int64_t ld_vu, const void* u_down,
                     int64_t ld_ud, const void* v_down, int64_t ld_vd, void* packed, void* stream,
                     const void* norm_w);

int svdmlp_pack(const svdmlp_layout* L, const void* u_gate, int64_t ld_ug, const void* v_gate, int64_t ld_vg,
                const void* u_up, int64_t ld_uu, const void* v_up, int64_t ld_vu, const void* u_down, int64_t ld_ud,
                const void* v_down, int64_t ld_vd, void* packed, void* stream) {
  return pack_impl(L, u_gate, ld_ug, v_gate, ld_vg, u_up, ld_uu, v_up, ld_vu, u_down, ld_ud, v_down, ld_vd, packed,
                   stream, nullptr);
}

int svdmlp_pack_block(const svdmlp_layout* L, const void* norm_weight, const void* u_gate, int64_t ld_ug,
                      const void* v_gate, int64_t ld_vg, const void* u_up, int64_t ld_uu, const void* v_up,
                      int64_t ld_vu, const void* u_down, int64_t ld_ud, const void* v_down, int64_t ld_vd,
                      void* packed, void* stream) {
  if (!norm_weight) return SVDMLP_ERR_INVALID_VALUE;
  return pack_impl(L, u_gate, ld_ug, v_gate, ld_vg, u_up, ld_uu, v_up, ld_vu, u_down, ld_ud, v_down, ld_vd, packed,
                   stream, norm_weight);
}

}  // extern "C"

static int pack_impl(const svdmlp_layout* L, const void* u_gate, int64_t ld_ug, const void* v_gate, int64_t ld_vg,
                     const void* u_up, int64_t ld_uu, const void* v_up, int64_t ld_vu, const void* u_down,
                     int64_t ld_ud, const void* v_down, int64_t ld_vd, void* packed, void* stream,
                     const void* norm_w) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || !packed) return SVDMLP_ERR_INVALID_VALUE;
  if ((reinterpret_cast<uintptr_t>(packed) & 255u) != 0) return SVDMLP_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* P = static_cast<uint8_t*>(packed);
  SVD_CUDA(cudaMemsetAsync(P, 0, static_cast<size_t>(L->packed_bytes), s));
  int* range = reinterpret_cast<int*>(P + L->off_status);  // set if an fp16-packed weight saturates
  if (L->r_gu > 0) {
    if (!u_gate || !v_gate || !u_up || !v_up) return SVDMLP_ERR_INVALID_VALUE;
    // w1 [2*rp_gu, d] (bf16: it multiplies the bf16 input X): u_gate^T, then u_up^T
    SVD_CHECK(launch_tiled_pack<bf16>(u_gate, ld_ug, L->d, L->r_gu, P + L->off_w1, 0, L->d, range, s, norm_w));
    SVD_CHECK(launch_tiled_pack<bf16>(u_up, ld_uu, L->d, L->r_gu, P + L->off_w1, L->rp_gu, L->d, range, s, norm_w));
    // v [r, ff] -> v^T [ff, r] (fp16: it multiplies the fp16 XU)
    SVD_CHECK(launch_tiled_pack<__half>(v_gate, ld_vg, L->r_gu, L->ff, P + L->off_vg, 0, L->r_gu, range, s));
    SVD_CHECK(launch_tiled_pack<__half>(v_up, ld_vu, L->r_gu, L->ff, P + L->off_vu, 0, L->r_gu, range, s));
  }
  if (L->r_d > 0) {
    if (!u_down || !v_down) return SVDMLP_ERR_INVALID_VALUE;
    // u_down [ff, r_d] -> [r_d, ff];  v_down [r_d, d] -> [d, r_d]
    if (L->ud_f16)
      SVD_CHECK(launch_tiled_pack<__half>(u_down, ld_ud, L->ff, L->r_d, P + L->off_ud, 0, L->ff, range, s));
    else
      SVD_CHECK(launch_tiled_pack<bf16>(u_down, ld_ud, L->ff, L->r_d, P + L->off_ud, 0, L->ff, range, s));
    SVD_CHECK(launch_tiled_pack<__half>(v_down, ld_vd, L->r_d, L->d, P + L->off_vd, 0, L->r_d, range, s));
  }
  return SVDMLP_OK;
}

extern "C" {

int svdmlp_dense_pack(const svdmlp_layout* L, const void* w_gate, int64_t ld_wg, const void* w_up, int64_t ld_wu,
                      const void* w_down, int64_t ld_wd, void* packed, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_DENSE || !packed || !w_gate || !w_up || !w_down) return SVDMLP_ERR_INVALID_VALUE;
  if ((reinterpret_cast<uintptr_t>(packed) & 255u) != 0) return SVDMLP_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* P = static_cast<uint8_t*>(packed);
  SVD_CUDA(cudaMemsetAsync(P, 0, static_cast<size_t>(L->packed_bytes), s));
  int* range = reinterpret_cast<int*>(P + L->off_status);
  SVD_CHECK(launch_tiled_pack<bf16>(w_gate, ld_wg, L->d, L->ff, P + L->off_vg, 0, L->d, range, s));
  SVD_CHECK(launch_tiled_pack<bf16>(w_up, ld_wu, L->d, L->ff, P + L->off_vu, 0, L->d, range, s));
  SVD_CHECK(launch_tiled_pack<__half>(w_down, ld_wd, L->ff, L->d, P + L->off_ud, 0, L->ff, range, s));
  return SVDMLP_OK;
}

int64_t svdmlp_workspace_bytes(const svdmlp_layout* L, int max_m) {
  if (check_layout(L) != SVDMLP_OK || max_m <= 0) return SVDMLP_ERR_INVALID_VALUE;
  return ws_bytes_for(L, max_m, planning_sms());
}

int svdmlp_workspace_init(void* ws, int64_t ws_bytes, void* stream) {
  if (!ws || ws_bytes < kCtlBytes) return SVDMLP_ERR_INVALID_VALUE;
  // The control block and the split-K counters sit at the front.
  const int64_t n = std::min<int64_t>(ws_bytes, kCtlBytes + kCounterBytes);
  SVD_CUDA(cudaMemsetAsync(ws, 0, static_cast<size_t>(n), static_cast<cudaStream_t>(stream)));
  return SVDMLP_OK;
}

// Reads the two words of a device error block (wait-timeout site, fp16 range
// flag) after the stream has drained; a set word maps to its status.
static int read_error_block(const void* block, cudaStream_t s, int* status) {
  SVD_CUDA(cudaStreamSynchronize(s));
  int words[2] = {0, 0};
  SVD_CUDA(cudaMemcpyAsync(words, block, sizeof(words), cudaMemcpyDeviceToHost, s));
  SVD_CUDA(cudaStreamSynchronize(s));
  *status = words[0] != 0 ? SVDMLP_ERR_DEVICE_TIMEOUT : words[1] != 0 ? SVDMLP_ERR_RANGE : SVDMLP_OK;
  return SVDMLP_OK;
}

int svdmlp_check_device_status(void* ws, int64_t ws_bytes, void* stream) {
  if (!ws || ws_bytes < kCtlBytes) return SVDMLP_ERR_INVALID_VALUE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int status = SVDMLP_OK;
  SVD_CHECK(read_error_block(ws, s, &status));
  if (status == SVDMLP_ERR_DEVICE_TIMEOUT) {
    // a wait that gave up may leave counters behind: clear the whole block
    SVD_CHECK(svdmlp_workspace_init(ws, ws_bytes, stream));
    SVD_CUDA(cudaStreamSynchronize(s));
  } else if (status == SVDMLP_ERR_RANGE) {
    SVD_CUDA(cudaMemsetAsync(static_cast<int*>(ws) + kRangeWord, 0, sizeof(int), s));
    SVD_CUDA(cudaStreamSynchronize(s));
  }
  return status;
}

int svdmlp_pack_status(const svdmlp_layout* L, const void* packed, void* stream) {
  SVD_CHECK(check_layout(L));
  if (!packed) return SVDMLP_ERR_INVALID_VALUE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SVD_CUDA(cudaStreamSynchronize(s));
  int word = 0;
  SVD_CUDA(cudaMemcpyAsync(&word, static_cast<const uint8_t*>(packed) + L->off_status, sizeof(int),
                           cudaMemcpyDeviceToHost, s));
  SVD_CUDA(cudaStreamSynchronize(s));
  return word != 0 ? SVDMLP_ERR_RANGE : SVDMLP_OK;
}

int svdmlp_gate_up(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* h,
                   int64_t ldh, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || !packed || !x || !h || M <= 0 || ldx < L->d || ldh < L->ff)
    return SVDMLP_ERR_INVALID_VALUE;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  const OutTarget ht = out_target(h, ldh, w.h, L->ld_ff);
  SVD_CHECK(run_gate_up(L, static_cast<const uint8_t*>(packed), xa, ldxa, M, ht.ptr, ht.ld, true, w, s));
  return finish_output(h, ldh, ht.ptr, ht.ld, M, L->ff, s);
}

// Caller-facing bf16 H into the form the layout's ud expects.
static int stage_h(const svdmlp_layout* L, const void* h, int64_t ldh, int M, const Workspace& w, const void** ha,
                   int64_t* ldha, cudaStream_t s) {
  if (L->ud_f16) {
    SVD_CHECK(launch_convert<bf16, __half>(static_cast<const bf16*>(h), ldh, w.h, L->ld_ff, M, L->ff, w.err + kRangeWord, s));
    *ha = w.h;
    *ldha = L->ld_ff;
    return SVDMLP_OK;
  }
  return stage_in(h, ldh, M, L->ff, w.h, L->ld_ff, ha, ldha, s);
}

int svdmlp_xuv(const svdmlp_layout* L, const void* packed, const void* h, int64_t ldh, int M, void* y,
               int64_t ldy, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_d <= 0 || !packed || !h || !y || M <= 0 || ldh < L->ff || ldy < L->d)
    return SVDMLP_ERR_INVALID_VALUE;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* ha;
  int64_t ldha;
  SVD_CHECK(stage_h(L, h, ldh, M, w, &ha, &ldha, s));
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  SVD_CHECK(run_down_u(L, P, ha, ldha, L->ud_f16 != 0, M, nullptr, 0, w, s));
  const OutTarget yt = out_target(y, ldy, w.ys, L->ld_d);
  SVD_CHECK(run_down_v(L, P, M, yt.ptr, yt.ld, nullptr, 0, w, s));
  return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
}

static int forward_impl(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* y,
                        int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes, void* stream,
                        bool contract);

int svdmlp_forward(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* y,
                   int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes, void* stream) {
  return forward_impl(L, packed, x, ldx, M, y, ldy, residual, ld_res, ws, ws_bytes, stream, M <= g_decode_contract);
}

int svdmlp_forward_contracted(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M,
                              void* y, int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes,
                              void* stream) {
  return forward_impl(L, packed, x, ldx, M, y, ldy, residual, ld_res, ws, ws_bytes, stream, true);
}

int svdmlp_set_decode_contract(int max_m) {
  if (max_m > 16) return SVDMLP_ERR_INVALID_VALUE;
  g_decode_contract = max_m < 0 ? kDecodeContractDefault : max_m;
  return SVDMLP_OK;
}

}  // extern "C"

static int forward_impl(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* y,
                        int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes, void* stream,
                        bool contract) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || L->r_d <= 0 || !packed || !x || !y || M <= 0 ||
      ldx < L->d || ldy < L->d || (residual && ld_res < L->d))
    return SVDMLP_ERR_INVALID_VALUE;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  if (M <= g_layer_decode_max_m || (contract && M <= 16)) {
    // Decode sizes: the whole layer in one launch (the contracted schedule
    // always runs there); its stores need no TMA alignment, and the residual
    // is read in place (it must not alias y).
    return run_layer_decode(L, P, xa, ldxa, M, y, ldy, residual, ld_res, w, s, contract);
  }
  const OutTarget yt = out_target(y, ldy, w.ys, L->ld_d);
  const void* res = nullptr;
  int64_t ldr = 0;
  const bool residual_in_place = residual && aligned16(residual, ld_res);
  if (M >= g_pair_min_m && g_chain_groups > 0 && cdiv(M, 256) <= kChainStride && (!residual || residual_in_place)) {
    // Prefill: the four stages as a chain (gemm_sm100.cuh), each stage
    // starting on the M-tile groups its predecessor has completed.
    int* base = w.counters + kChainOffsetInts;
    const int nt_xu = static_cast<int>(cdiv(L->rp_gu, CfgXUd::BN));
    const int nt_gu = static_cast<int>(cdiv(L->ff, CfgGU::BN));
    const int nt_du = static_cast<int>(cdiv(L->r_d, CfgDU::BN));
    const int mg = static_cast<int>(cdiv(cdiv(M, 256), g_chain_groups));  // M-tiles per group
    const ChainLink links[4] = {
        {nullptr, 0, base, nullptr, nullptr, mg},
        {base, 2 * nt_xu, base + kChainStride, nullptr, nullptr, mg},
        {base + kChainStride, 2 * nt_gu, base + 2 * kChainStride, nullptr, nullptr, mg},
        {base + 2 * kChainStride, 2 * nt_du, nullptr, base, base + 3 * kChainStride, mg}};
    Workspace wc[4] = {w, w, w, w};
    for (int i = 0; i < 4; ++i) wc[i].chain = &links[i];
    SVD_CHECK(run_xu(L, P, xa, ldxa, M, wc[0], s));
    SVD_CHECK(run_gu(L, P, M, w.h, L->ld_ff, false, wc[1], s));
    SVD_CHECK(run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, 0, wc[2], s));
    if (residual) {
      res = residual;
      ldr = ld_res;
    }
    SVD_CHECK(run_down_v(L, P, M, yt.ptr, yt.ld, res, ldr, wc[3], s));
    return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
  }
  SVD_CHECK(run_gate_up(L, P, xa, ldxa, M, w.h, L->ld_ff, false, w, s));
  SVD_CHECK(run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, 0, w, s));
  // An unaligned residual is staged in the x staging buffer once x is consumed.
  if (residual) SVD_CHECK(stage_in(residual, ld_res, M, L->d, w.xs, L->ld_d, &res, &ldr, s));
  SVD_CHECK(run_down_v(L, P, M, yt.ptr, yt.ld, res, ldr, w, s));
  return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
}

extern "C" {

int svdmlp_row_sumsq(const void* x, int64_t ldx, int M, int n, float* stats, int64_t ld_stats, void* stream) {
  if (!x || !stats || M <= 0 || n <= 0 || ldx < n || ld_stats < cdiv(n, 128)) return SVDMLP_ERR_INVALID_VALUE;
  row_sumsq_kernel<<<static_cast<unsigned>(M), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(x), ldx, n, stats, ld_stats);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_forward_block(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* y,
                         int64_t ldy, const float* x_stats, int64_t ld_stats, float* y_stats, float eps, void* ws,
                         int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || L->r_d <= 0 || !packed || !x || !y || !x_stats || M <= 0 ||
      ldx < L->d || ldy < L->d || ld_stats < cdiv(L->d, 128) || !(eps >= 0.0f) || x == y)
    return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(x, ldx)) return SVDMLP_ERR_ALIGNMENT;  // x is also the residual, read in place
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  Workspace wn = w, wo = w;  // the first stage (norm) and the residual stage (statistics)
  wn.norm_stats = x_stats;
  wn.norm_parts = static_cast<int>(cdiv(L->d, 128));
  wn.norm_dim = L->d;
  wn.norm_eps = eps;
  wn.stats_ld = static_cast<int>(ld_stats);
  wo.stats_ld = static_cast<int>(ld_stats);
  wo.out_stats = y_stats;
  if (M <= g_layer_decode_max_m || M <= g_decode_contract) {
    Workspace wb = wn;
    wb.out_stats = y_stats;
    return run_layer_decode(L, P, x, ldx, M, y, ldy, x, ldx, wb, s, M <= g_decode_contract);
  }
  const OutTarget yt = out_target(y, ldy, w.ys, L->ld_d);
  SVD_CHECK(run_xu(L, P, x, ldx, M, wn, s));
  SVD_CHECK(run_gu(L, P, M, w.h, L->ld_ff, false, w, s));
  SVD_CHECK(run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, 0, w, s));
  SVD_CHECK(run_down_v(L, P, M, yt.ptr, yt.ld, x, ldx, wo, s));
  return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
}

int svdmlp_dense_forward(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* y,
                         int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes,
                         void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_DENSE || !packed || !x || !y || M <= 0 || ldx < L->d || ldy < L->d ||
      (residual && ld_res < L->d))
    return SVDMLP_ERR_INVALID_VALUE;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  const OutTarget yt = out_target(y, ldy, w.ys, L->ld_d);
  const void* res = nullptr;
  int64_t ldr = 0;
  if (residual) SVD_CHECK(stage_in(residual, ld_res, M, L->d, w.xs, L->ld_d, &res, &ldr, s));
  SVD_CHECK(run_dense(L, P, xa, ldxa, M, yt.ptr, yt.ld, res, ldr, w, s));
  return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
}

int svdmlp_forward_partial(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M,
                           float* partial, int64_t ldp, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || L->r_d <= 0 || !packed || !x || !partial || M <= 0 ||
      ldx < L->d || ldp < L->r_d)
    return SVDMLP_ERR_INVALID_VALUE;
  if ((reinterpret_cast<uintptr_t>(partial) & 15u) != 0 || ldp % 4 != 0) return SVDMLP_ERR_ALIGNMENT;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  SVD_CHECK(run_gate_up(L, P, xa, ldxa, M, w.h, L->ld_ff, false, w, s));
  return run_down_u(L, P, w.h, L->ld_ff, true, M, partial, ldp, w, s);
}

int svdmlp_down_partial(const svdmlp_layout* L, const void* packed, const void* h, int64_t ldh, int M,
                        float* partial, int64_t ldp, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_d <= 0 || !packed || !h || !partial || M <= 0 || ldh < L->ff ||
      ldp < L->r_d)
    return SVDMLP_ERR_INVALID_VALUE;
  if (!L->ud_f16) return SVDMLP_ERR_DTYPE;
  if ((reinterpret_cast<uintptr_t>(partial) & 15u) != 0 || ldp % 4 != 0) return SVDMLP_ERR_ALIGNMENT;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* ha;
  int64_t ldha;
  SVD_CHECK(stage_h(L, h, ldh, M, w, &ha, &ldha, s));
  return run_down_u(L, static_cast<const uint8_t*>(packed), ha, ldha, true, M, partial, ldp, w, s);
}

int svdmlp_forward_partial_f16(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M,
                               void* partial, int64_t ldp, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || L->r_d <= 0 || !packed || !x || !partial || M <= 0 ||
      ldx < L->d || ldp < L->r_d)
    return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(partial, ldp)) return SVDMLP_ERR_ALIGNMENT;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  SVD_CHECK(run_gate_up(L, P, xa, ldxa, M, w.h, L->ld_ff, false, w, s));
  return run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, ldp, w, s, partial);
}

int svdmlp_xu_project(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M, void* xu,
                      int64_t ld_xu, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || !packed || !x || !xu || M <= 0 || ldx < L->d ||
      ld_xu < 2LL * L->rp_gu)
    return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(xu, ld_xu)) return SVDMLP_ERR_ALIGNMENT;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  return run_xu(L, static_cast<const uint8_t*>(packed), xa, ldxa, M, w, s, xu, ld_xu);
}

int svdmlp_partial_from_xu_f16(const svdmlp_layout* L, const void* packed, const void* xu, int64_t ld_xu, int M,
                               void* partial, int64_t ldp, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || L->r_d <= 0 || !packed || !xu || !partial || M <= 0 ||
      ld_xu < 2LL * L->rp_gu || ldp < L->r_d)
    return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(xu, ld_xu) || !aligned16(partial, ldp)) return SVDMLP_ERR_ALIGNMENT;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  SVD_CHECK(run_gu(L, P, M, w.h, L->ld_ff, false, w, s, xu, ld_xu));
  return run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, ldp, w, s, partial);
}

int svdmlp_down_finish_f16(const svdmlp_layout* L, const void* packed, const void* partial, int64_t ldp, int M,
                           void* y, int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes,
                           void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_d <= 0 || !packed || !partial || !y || M <= 0 || ldp < L->r_d ||
      ldy < L->d || (residual && ld_res < L->d))
    return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(partial, ldp)) return SVDMLP_ERR_ALIGNMENT;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const OutTarget yt = out_target(y, ldy, w.ys, L->ld_d);
  const void* res = nullptr;
  int64_t ldr = 0;
  if (residual) SVD_CHECK(stage_in(residual, ld_res, M, L->d, w.xs, L->ld_d, &res, &ldr, s));
  SVD_CHECK(run_down_v(L, static_cast<const uint8_t*>(packed), M, yt.ptr, yt.ld, res, ldr, w, s, partial, ldp));
  return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
}

int svdmlp_down_finish(const svdmlp_layout* L, const void* packed, const float* partial, int64_t ldp, int M,
                       void* y, int64_t ldy, const void* residual, int64_t ld_res, void* ws, int64_t ws_bytes,
                       void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_d <= 0 || !packed || !partial || !y || M <= 0 || ldp < L->r_d ||
      ldy < L->d || (residual && ld_res < L->d))
    return SVDMLP_ERR_INVALID_VALUE;
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SVD_CHECK(launch_convert<float, __half>(partial, ldp, w.t, L->rp_d, M, L->r_d, w.err + kRangeWord, s));
  const OutTarget yt = out_target(y, ldy, w.ys, L->ld_d);
  const void* res = nullptr;
  int64_t ldr = 0;
  if (residual) SVD_CHECK(stage_in(residual, ld_res, M, L->d, w.xs, L->ld_d, &res, &ldr, s));
  SVD_CHECK(run_down_v(L, static_cast<const uint8_t*>(packed), M, yt.ptr, yt.ld, res, ldr, w, s));
  return finish_output(y, ldy, yt.ptr, yt.ld, M, L->d, s);
}

int64_t svdmlp_gemm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return SVDMLP_ERR_INVALID_VALUE;
  const int sms = planning_sms();
  const Plan pl = M >= g_pair_min_m ? plan_for<CfgGemm>(M, N, K, sms, g_split_override[ST_GEMM])
                                 : plan_for<CfgGemm1>(M, N, K, sms, g_split_override[ST_GEMM]);
  const int64_t part = M >= g_pair_min_m ? partial_bytes(pl, CfgGemm::BN, 1, 2) : partial_bytes(pl, CfgGemm1::BN, 1);
  return kCtlBytes + kCounterBytes + round_up(part, 256);
}

int svdmlp_gemm(const void* a, int64_t lda, const void* bt, int64_t ldb, void* c, int64_t ldc, int M, int N, int K,
                void* ws, int64_t ws_bytes, void* stream) {
  if (!a || !bt || !c || M <= 0 || N <= 0 || K <= 0 || lda < K || ldb < K || ldc < N) return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(a, lda) || !aligned16(bt, ldb) || !aligned16(c, ldc)) return SVDMLP_ERR_ALIGNMENT;
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return SVDMLP_ERR_INVALID_VALUE;
  const int64_t need = svdmlp_gemm_workspace_bytes(M, N, K);
  if (ws_bytes < need) return SVDMLP_ERR_WORKSPACE;
  const int64_t cnt = kCounterBytes;
  Workspace w{};
  uint8_t* p = static_cast<uint8_t*>(ws);
  w.err = reinterpret_cast<int*>(p);
  w.counters = reinterpret_cast<int*>(p + kCtlBytes);
  w.partials = reinterpret_cast<float*>(p + kCtlBytes + cnt);
  w.partial_cap = ws_bytes - kCtlBytes - cnt;
  const Operand ao{a, false, K, M, lda};
  const Operand bo{bt, false, K, N, ldb};
  return gemm_stage<CfgGemm, CfgGemm1>(ao, ao, bo, bo, Output{c, N, M, ldc}, M, N, K, ST_GEMM, w,
                                       static_cast<cudaStream_t>(stream));
}

int svdmlp_rmsnorm(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, int M, int n, float eps,
                   void* stream) {
  if (!x || !w || !y || M <= 0 || n <= 0 || ldx < n || ldy < n || !(eps >= 0.f)) return SVDMLP_ERR_INVALID_VALUE;
  rmsnorm_kernel<<<static_cast<unsigned>(M), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(x), ldx, static_cast<const bf16*>(w), static_cast<bf16*>(y), ldy, n, eps);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_debug_wait_timeout(void* ws, int64_t ws_bytes, int64_t limit_ns, void* stream) {
  if (!ws || ws_bytes < kCtlBytes || limit_ns <= 0) return SVDMLP_ERR_INVALID_VALUE;
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<int*>(ws),
                                                                      static_cast<unsigned long long>(limit_ns));
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_stage_timing(int enable) {
  std::lock_guard<std::mutex> lock(g_timing_mu);
  if (enable && g_timed.empty()) {
    g_timed.resize(4096);
    for (auto& t : g_timed) {
      SVD_CUDA(cudaEventCreate(&t.start));
      SVD_CUDA(cudaEventCreate(&t.stop));
    }
  }
  g_timing = enable != 0;
  g_timed_used = 0;
  return SVDMLP_OK;
}

int svdmlp_stage_times(double* ms_out, int64_t* counts_out, int n) {
  if (!ms_out || !counts_out || n <= 0) return SVDMLP_ERR_INVALID_VALUE;
  std::lock_guard<std::mutex> lock(g_timing_mu);
  for (int i = 0; i < n; ++i) {
    ms_out[i] = 0.0;
    counts_out[i] = 0;
  }
  for (size_t i = 0; i < g_timed_used; ++i) {
    SVD_CUDA(cudaEventSynchronize(g_timed[i].stop));
    float ms = 0.f;
    SVD_CUDA(cudaEventElapsedTime(&ms, g_timed[i].start, g_timed[i].stop));
    const int st = g_timed[i].stage;
    if (st >= 0 && st < n) {
      ms_out[st] += ms;
      counts_out[st] += 1;
    }
  }
  g_timed_used = 0;
  return SVDMLP_OK;
}

int svdmlp_set_trace_buffer(void* buffer, int64_t bytes) {
  // 296 CTAs x 64 events x 16 bytes is the largest timeline one launch writes
  if (buffer && bytes < 2 * 148 * 64 * 16) return SVDMLP_ERR_INVALID_VALUE;
  g_trace = static_cast<unsigned long long*>(buffer);
  return SVDMLP_OK;
}

int svdmlp_set_layer_decode(int max_m) {
  if (max_m > kLayerDecodeMaxM) return SVDMLP_ERR_INVALID_VALUE;
  g_layer_decode_max_m = max_m < 0 ? kLayerDecodeDefaultMaxM : max_m;
  return SVDMLP_OK;
}

int svdmlp_set_decode_prefetch(int ahead_slots, int wait_slots) {
  if (ahead_slots < 0 || ahead_slots > 64 || wait_slots < 0 || wait_slots > 64) return SVDMLP_ERR_INVALID_VALUE;
  g_pf_ahead = ahead_slots;
  g_pf_wait = wait_slots;
  return SVDMLP_OK;
}

int svdmlp_set_decode_overlap(int mode) {
  if (mode < 0 || mode > 8) return SVDMLP_ERR_INVALID_VALUE;
  g_layer_decode_pdl = mode;
  return SVDMLP_OK;
}

int svdmlp_set_pair_min_m(int m) {
  if (m > kPairMinMDefault) return SVDMLP_ERR_INVALID_VALUE;
  g_pair_min_m = m < 0 ? kPairMinMDefault : std::max(m, kPairMinMLowest);
  return SVDMLP_OK;
}

int svdmlp_set_prefill_chain(int groups) {
  if (groups < 0 || groups > 64) return SVDMLP_ERR_INVALID_VALUE;
  g_chain_groups = groups;
  return SVDMLP_OK;
}

int svdmlp_set_split_tail(int enable) {
  if (enable != 0 && enable != 1) return SVDMLP_ERR_INVALID_VALUE;
  g_split_tail = enable;
  return SVDMLP_OK;
}

int svdmlp_set_split_override(int stage, int splits) {
  if (stage < 0 || stage >= 8 || splits < 0 || splits > 64) return SVDMLP_ERR_INVALID_VALUE;
  g_split_override[stage] = splits;
  return SVDMLP_OK;
}

// ----------------------------------------------------------------------------
// XUV down operator with library-owned scratch, for callers that cannot
// allocate device memory: plugins hosted by a runtime that owns every device
// allocation and hands the plugin only its input and output buffers, and code
// that runs where cudaMalloc is not allowed.  The scratch (control block,
// split-K counters, the rank-r intermediate, the fp16 copy of H and, when they
// fit, split-K partials) lives in this file-scope device array, one copy per
// GPU that loads the library, kept until the process exits.
// ----------------------------------------------------------------------------
static constexpr int64_t kStaticScratchBytes = 8LL << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
static std::mutex g_static_mu;
static void* g_static_scratch_dev[64] = {};

// Device address of g_static_scratch on the current device.  The host-side
// name is only a stand-in; the address must come from cudaGetSymbolAddress,
// called once per device with that device current.
static int static_scratch_address(void** out) {
  int dev = 0;
  SVD_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return SVDMLP_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_scratch_dev[dev]) {
    void* p = nullptr;
    SVD_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
    if (!p) return SVDMLP_ERR_CUDA;
    g_static_scratch_dev[dev] = p;
  }
  *out = g_static_scratch_dev[dev];
  return SVDMLP_OK;
}

int svdmlp_xuv_noalloc(const svdmlp_layout* L, const void* packed, const void* h, int64_t ldh, int M, void* y,
                       int64_t ldy, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_d <= 0 || !packed || !h || !y || M <= 0 || ldh < L->ff || ldy < L->d)
    return SVDMLP_ERR_INVALID_VALUE;
  if (!aligned16(h, ldh) || !aligned16(y, ldy)) return SVDMLP_ERR_ALIGNMENT;
  const int64_t cnt = round_up(cdiv(M, 128) * cdiv(std::max(L->r_d, L->d), 128) * 4, 256);
  const int64_t t_bytes = round_up(static_cast<int64_t>(M) * L->rp_d * 2, 256);
  const int64_t h_bytes = L->ud_f16 ? round_up(static_cast<int64_t>(M) * L->ld_ff * 2, 256) : 0;
  const int64_t need = kCtlBytes + cnt + t_bytes + h_bytes;
  if (need > kStaticScratchBytes) return SVDMLP_ERR_WORKSPACE;
  void* base = nullptr;
  SVD_CHECK(static_scratch_address(&base));
  uint8_t* p = static_cast<uint8_t*>(base);
  Workspace w{};
  w.err = reinterpret_cast<int*>(p);
  w.counters = reinterpret_cast<int*>(p + kCtlBytes);
  w.t = reinterpret_cast<__half*>(p + kCtlBytes + cnt);
  w.h = reinterpret_cast<__half*>(p + kCtlBytes + cnt + t_bytes);
  w.partials = reinterpret_cast<float*>(p + need);
  w.partial_cap = kStaticScratchBytes - need;
  w.unsplit_if_short = true;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: the error word and the
  // split-K counters must start at zero.
  SVD_CUDA(cudaMemsetAsync(p, 0, static_cast<size_t>(kCtlBytes + cnt), s));
  const void* ha = h;
  int64_t ldha = ldh;
  if (L->ud_f16) {
    SVD_CHECK(launch_convert<bf16, __half>(static_cast<const bf16*>(h), ldh, w.h, L->ld_ff, M, L->ff, w.err + kRangeWord, s));
    ha = w.h;
    ldha = L->ld_ff;
  }
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  SVD_CHECK(run_down_u(L, P, ha, ldha, L->ud_f16 != 0, M, nullptr, 0, w, s));
  return run_down_v(L, P, M, y, ldy, nullptr, 0, w, s);
}

int svdmlp_xuv_noalloc_status(void* stream) {
  void* base = nullptr;
  SVD_CHECK(static_scratch_address(&base));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int status = SVDMLP_OK;
  SVD_CHECK(read_error_block(base, s, &status));
  if (status != SVDMLP_OK) {
    // both words; the counters are cleared by the next call's own reset
    SVD_CUDA(cudaMemsetAsync(base, 0, 2 * sizeof(int), s));
    SVD_CUDA(cudaStreamSynchronize(s));
  }
  return status;
}

}  // extern "C"

// Compile-time resources of the kernel configuration a stage runs with at M
// tokens (the per-stage kernels; M <= 128 uses the swapped-operand decode
// set for its token tile).
namespace svdmlp {
template <class Cfg>
static void pair_tile_info(int* o) {
  o[0] = Cfg::TILE_M;
  o[1] = Cfg::EPI == EPI_DUAL_STORE ? 2 * Cfg::BN : Cfg::BN;
  o[2] = Cfg::BK;
  o[3] = Cfg::STAGES;
  o[4] = Cfg::SMEM_BYTES;
  o[5] = static_cast<int>(Cfg::TMEM_COLS);
  o[6] = Cfg::THREADS;
  o[7] = Cfg::CTAS;
}
template <class Cfg>
static void dec_tile_info(int* o) {
  o[0] = Cfg::TOK;
  o[1] = Cfg::BM;
  o[2] = Cfg::BK;
  o[3] = Cfg::STAGES;
  o[4] = Cfg::SMEM_BYTES;
  o[5] = static_cast<int>(Cfg::TMEM_COLS);
  o[6] = 192;
  o[7] = 1;
}
template <class Set>
static void dec_set_info(int stage, int* o) {
  if (stage == ST_XU) dec_tile_info<typename Set::XU>(o);
  else if (stage == ST_GATEUP) dec_tile_info<typename Set::GU>(o);
  else if (stage == ST_DOWN_U) dec_tile_info<typename Set::DU>(o);
  else if (stage == ST_DENSE_GU) dec_tile_info<typename Set::DGU>(o);
  else dec_tile_info<typename Set::DV>(o);
}
}  // namespace svdmlp

extern "C" {

int svdmlp_tile_info(int stage, int M, int* out8) {
  if (!out8 || M <= 0 || stage < 0 || stage > ST_GEMM) return SVDMLP_ERR_INVALID_VALUE;
  const bool pair = M >= g_pair_min_m;
  switch (stage) {
    case ST_XU: pair ? pair_tile_info<CfgXUd>(out8) : void(); break;
    case ST_GATEUP: pair ? pair_tile_info<CfgGU>(out8) : void(); break;
    case ST_DOWN_U: pair ? pair_tile_info<CfgDU>(out8) : void(); break;
    case ST_DOWN_V: pair ? pair_tile_info<CfgDV>(out8) : void(); break;
    case ST_DENSE_GU: pair ? pair_tile_info<CfgDenseGU>(out8) : pair_tile_info<CfgDenseGU1>(out8); break;
    case ST_DENSE_D: pair ? pair_tile_info<CfgDV>(out8) : pair_tile_info<CfgDV1>(out8); break;
    default: pair ? pair_tile_info<CfgGemm>(out8) : pair_tile_info<CfgGemm1>(out8); break;
  }
  if (!pair && stage <= ST_DENSE_D) {
    if (M <= 16) dec_set_info<Dec16>(stage, out8);
    else if (M <= 64) dec_set_info<Dec64>(stage, out8);
    else dec_set_info<Dec128>(stage, out8);
  }
  return SVDMLP_OK;
}

int svdmlp_plan_info(int stage, int M, int N, int K, int* out6) {
  if (!out6 || M <= 0 || N <= 0 || K <= 0 || stage < 0 || stage >= 8) return SVDMLP_ERR_INVALID_VALUE;
  const bool dual = stage == ST_GATEUP || stage == ST_DENSE_GU;
  const int nb = dual ? 2 : 1;
  const int tok = M <= 16 ? 16 : M <= 64 ? 64 : 128;
  const int pair_bn = dual ? CfgGU::BN : stage == ST_XU ? CfgXUd::BN : stage == ST_DOWN_U ? CfgDU::BN
                    : stage == ST_DOWN_V || stage == ST_DENSE_D ? CfgDV::BN : CfgGemm::BN;
  // prefill X.[u_g|u_u] is a dual-store tile over the two halves of N
  const int pair_n = stage == ST_XU ? (N + 1) / 2 : N;
  // below the pair threshold: the plan of the per-stage decode kernel for M
  // (the same function the launches use)
  auto dec_plan = [&](auto set) -> Plan {
    using Set = decltype(set);
    return dual ? plan_dec<typename Set::GU>(M, N, K, planning_sms(), g_split_override[stage])
                : plan_dec<typename Set::XU>(M, N, K, planning_sms(), g_split_override[stage]);
  };
  const Plan p = M >= g_pair_min_m ? plan_gemm_pair(M, pair_n, K, pair_bn, planning_sms(), stage != ST_XU,
                                                g_split_override[stage], nb)
                 : tok == 16         ? dec_plan(Dec16{})
                 : tok == 64         ? dec_plan(Dec64{})
                                     : dec_plan(Dec128{});
  out6[0] = p.m_tiles;
  out6[1] = p.n_tiles;
  out6[2] = p.k_blocks;
  out6[3] = p.splits;
  out6[4] = p.units;
  out6[5] = p.grid;
  return SVDMLP_OK;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Collectives over NVLink peer memory (peer_sm100.cuh).
namespace svdmlp {
static int make_peer_args(void* const* bases, int world, int rank, PeerArgs* a) {
  if (!bases || world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world) return SVDMLP_ERR_INVALID_VALUE;
  std::memset(a, 0, sizeof(*a));
  for (int i = 0; i < world; ++i) {
    if (!bases[i] || (reinterpret_cast<uintptr_t>(bases[i]) & 255u) != 0) return SVDMLP_ERR_ALIGNMENT;
    a->base[i] = static_cast<unsigned char*>(bases[i]);
  }
  a->world = world;
  a->rank = rank;
  a->limit_ns = g_wait_limit_ns;
  return SVDMLP_OK;
}

// CTAs of a collective: enough for `vectors` 16-byte elements at four per
// thread, at most one per SM.  Small exchanges (decode sizes) then run on a few
// CTAs and wait on a few barriers instead of one per SM.  The grid depends only
// on the sizes, so every rank launches the same one.
static int peer_grid(int64_t vectors, unsigned* grid) {
  DeviceInfo* dev = nullptr;
  SVD_CHECK(device_info(&dev));
  const int64_t want = cdiv(vectors, static_cast<int64_t>(kPeerThreads) * kPeerUnroll);
  *grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, std::min(kPeerMaxCtas, dev->sms))));
  return SVDMLP_OK;
}

static bool peer_matrix_ok(int64_t off, int m, int64_t row_bytes, int64_t ld_bytes) {
  return m > 0 && row_bytes > 0 && row_bytes % 16 == 0 && ld_bytes >= row_bytes && ld_bytes % 16 == 0 &&
         off >= kPeerSignalBytes && off % 16 == 0;
}
}  // namespace svdmlp

extern "C" {

int64_t svdmlp_peer_signal_bytes(void) { return kPeerSignalBytes; }

int svdmlp_peer_alloc(int64_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes <= kPeerSignalBytes) return SVDMLP_ERR_INVALID_VALUE;
  void* p = nullptr;
  SVD_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer maps it
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return SVDMLP_ERR_CUDA;
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return SVDMLP_OK;
}

int svdmlp_peer_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return SVDMLP_ERR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  SVD_CUDA(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return SVDMLP_OK;
}

int svdmlp_peer_close(void* peer_ptr) {
  if (!peer_ptr) return SVDMLP_ERR_INVALID_VALUE;
  SVD_CUDA(cudaIpcCloseMemHandle(peer_ptr));
  return SVDMLP_OK;
}

int svdmlp_peer_free(void* ptr) {
  if (!ptr) return SVDMLP_ERR_INVALID_VALUE;
  SVD_CUDA(cudaFree(ptr));
  return SVDMLP_OK;
}

int64_t svdmlp_peer_scratch_bytes(int world, int m, int c) {
  if (world < 1 || world > kPeerMaxRanks || m <= 0 || c <= 0) return 0;
  return 2LL * world * cdiv(m, world) * c * 2;
}

int svdmlp_peer_allreduce_f16(void* const* bases, int world, int rank, int64_t off, int m, int c, int64_t ld,
                              int64_t off_scratch, void* stream) {
  PeerArgs a;
  SVD_CHECK(make_peer_args(bases, world, rank, &a));
  if (c <= 0 || c % 8 != 0 || !peer_matrix_ok(off, m, 2LL * c, 2 * ld) || off_scratch < kPeerSignalBytes ||
      off_scratch % 16 != 0)
    return SVDMLP_ERR_INVALID_VALUE;
  unsigned grid = 0;
  SVD_CHECK(peer_grid(static_cast<int64_t>(m) * (c / 8), &grid));
  peer_allreduce_f16_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, off, m, c, ld,
                                                                                         off_scratch);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_peer_reduce_scatter_f16(void* const* bases, int world, int rank, int64_t off, int m, int c, int64_t ld,
                                   int64_t off_scratch, void* out, int64_t ld_out, void* stream) {
  PeerArgs a;
  SVD_CHECK(make_peer_args(bases, world, rank, &a));
  if (c <= 0 || c % 8 != 0 || !peer_matrix_ok(off, m, 2LL * c, 2 * ld) || off_scratch < kPeerSignalBytes ||
      off_scratch % 16 != 0 || !out || ld_out < c || ld_out % 8 != 0)
    return SVDMLP_ERR_INVALID_VALUE;
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) return SVDMLP_ERR_ALIGNMENT;
  unsigned grid = 0;
  SVD_CHECK(peer_grid(static_cast<int64_t>(m) * (c / 8), &grid));
  peer_reduce_scatter_f16_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      a, off, m, c, ld, off_scratch, static_cast<unsigned char*>(out), ld_out);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_peer_allgather(void* const* bases, int world, int rank, int64_t off, int m, int64_t row_bytes,
                          int64_t ld_bytes, void* stream) {
  PeerArgs a;
  SVD_CHECK(make_peer_args(bases, world, rank, &a));
  if (!peer_matrix_ok(off, m, row_bytes, ld_bytes)) return SVDMLP_ERR_INVALID_VALUE;
  unsigned grid = 0;
  SVD_CHECK(peer_grid(static_cast<int64_t>(m) * (row_bytes / 16), &grid));
  peer_allgather_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, off, m, row_bytes,
                                                                                     ld_bytes);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int64_t svdmlp_peer_slots_bytes(int world, int slot_rows, int64_t ld_slot) {
  if (world < 1 || world > kPeerMaxRanks || slot_rows <= 0 || ld_slot <= 0 || ld_slot % 8 != 0) return 0;
  return 2LL * world * slot_rows * ld_slot * 2;
}

int svdmlp_forward_partial_f16_peer(const svdmlp_layout* L, const void* packed, const void* x, int64_t ldx, int M,
                                    void* const* bases, int world, int rank, int64_t off_slots, int slot_rows,
                                    int64_t ld_slot, void* ws, int64_t ws_bytes, void* stream) {
  SVD_CHECK(check_layout(L));
  if (L->kind != SVDMLP_KIND_SVD || L->r_gu <= 0 || L->r_d <= 0 || !packed || !x || M <= 0 || ldx < L->d ||
      M > slot_rows || ld_slot < L->r_d || ld_slot % 8 != 0 || off_slots < kPeerSignalBytes || off_slots % 16 != 0)
    return SVDMLP_ERR_INVALID_VALUE;
  PeerArgs a;
  SVD_CHECK(make_peer_args(bases, world, rank, &a));
  Workspace w{};
  SVD_CHECK(carve(L, M, ws, ws_bytes, &w));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* P = static_cast<const uint8_t*>(packed);
  const void* xa;
  int64_t ldxa;
  SVD_CHECK(stage_in(x, ldx, M, L->d, w.xs, L->ld_d, &xa, &ldxa, s));
  SVD_CHECK(run_gate_up(L, P, xa, ldxa, M, w.h, L->ld_ff, false, w, s));
  if (M >= g_pair_min_m) {
    // the CTA-pair H.u_down GEMM stores its rows straight into the slots
    static_assert(kPushMaxRanks == kPeerMaxRanks, "one slot per rank");
    GemmPush push{};
    const long long slot_bytes = static_cast<long long>(slot_rows) * ld_slot * 2;
    for (int q = 0; q < world; ++q) {
      push.dst[q] = a.base[q] + off_slots + rank * slot_bytes;
      push.flag[q] = reinterpret_cast<unsigned*>(&reinterpret_cast<PeerSignal*>(a.base[q])->ctl[kPushFlagWord + rank]);
    }
    PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[rank]);
    push.epoch = reinterpret_cast<unsigned*>(&me->ctl[kPushEpochWord]);
    push.exit_count = reinterpret_cast<unsigned*>(&me->ctl[kPushExitWord]);
    push.parity_bytes = world * slot_bytes;
    push.ld = ld_slot;
    push.n = world;
    push.rank = rank;
    Workspace wp = w;
    wp.push = &push;
    // the output map (over the workspace's T) is built but not written
    return run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, L->rp_d, wp, s, w.t);
  }
  // decode sizes: the partial goes to the workspace's T, then into the slots
  SVD_CHECK(run_down_u(L, P, w.h, L->ld_ff, true, M, nullptr, L->rp_d, w, s, w.t));
  unsigned grid = 0;
  SVD_CHECK(peer_grid(static_cast<int64_t>(M) * (ld_slot / 8), &grid));
  peer_push_slots_kernel<<<grid, kPeerThreads, 0, s>>>(a, reinterpret_cast<const unsigned char*>(w.t), L->rp_d,
                                                       off_slots, M, slot_rows, L->r_d, ld_slot);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_peer_sum_f16(void* const* bases, int world, int rank, int64_t off_slots, int slot_rows, int m, int c,
                        int64_t ld_slot, void* out, int64_t ld_out, void* stream) {
  PeerArgs a;
  SVD_CHECK(make_peer_args(bases, world, rank, &a));
  if (m <= 0 || m > slot_rows || c <= 0 || c % 8 != 0 || ld_slot < c || ld_slot % 8 != 0 || off_slots < kPeerSignalBytes ||
      off_slots % 16 != 0 || !out || ld_out < c || ld_out % 8 != 0)
    return SVDMLP_ERR_INVALID_VALUE;
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) return SVDMLP_ERR_ALIGNMENT;
  unsigned grid = 0;
  SVD_CHECK(peer_grid(static_cast<int64_t>(m) * (c / 8), &grid));
  peer_sum_slots_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      a, off_slots, m, slot_rows, c, ld_slot, static_cast<unsigned char*>(out), ld_out);
  SVD_CUDA(cudaGetLastError());
  g_launches.fetch_add(1);
  return SVDMLP_OK;
}

int svdmlp_peer_check_status(void* own_base, void* stream) {
  if (!own_base) return SVDMLP_ERR_INVALID_VALUE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int status = SVDMLP_OK;
  SVD_CHECK(read_error_block(own_base, s, &status));
  if (status == SVDMLP_ERR_RANGE) {
    SVD_CUDA(cudaMemsetAsync(static_cast<int*>(own_base) + kRangeWord, 0, sizeof(int), s));
    SVD_CUDA(cudaStreamSynchronize(s));
  }
  return status;
}

}  // extern "C"
