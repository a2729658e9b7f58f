// Whole-layer decode kernel (M <= 64 tokens) for sm_100a: the four GEMM
// stages of one SVD MLP layer in one persistent launch.
//
//   stage 0  XU = X . [u_g|u_u]                 (bf16 -> fp16)
//   stage 1  H  = silu(XU_g . v_g) * (XU_u . v_u)   (fp16, dual)
//   stage 2  T  = H . u_down                    (fp16)
//   stage 3  y  = T . v_down (+ residual)       (bf16)
//
// At decode sizes every stage streams its factor matrix from HBM once; the
// work is the weight bytes.  Running the stages as separate kernels pays a
// launch, a pipeline ramp and a split-K hand-off per stage.  Here all units
// of all stages form one list that the running CTAs claim in order, and
// a stage's units wait (bounded) on a per-stage "tiles done" counter before
// they load their activation tiles.  The weight tiles never depend on an
// earlier stage, so the producer fetches them before it waits: the weight
// stream runs on across stage boundaries.
//
// Each unit is a 128-row panel of a stage's weight (the MMA M) over a K range
// (split-K), times the tokens (the MMA N, TOK = 16 or 64, zero-filled beyond
// M).  Units are claimed dynamically: the producer takes the next unit index
// from a global counter and passes it to the MMA and epilogue warps through a
// small shared-memory queue, so busy and idle CTAs even out at every stage
// boundary.  CTA i starts with unit i and claims from the counter after that,
// so a unit only ever waits on units of the first wave or claimed before it.
// The grid is at most one CTA per SM, and the launch waits for the previous
// grid before any unit is taken, so every CTA of the first wave is resident;
// were one not (another context holding SMs), the bounded dependency wait
// would end the launch with a timeout status instead of hanging.
// A shared-memory slot holds two weight tiles and two token tiles: the
// two branches (gate, up) of one k-block for the dual stage, or two
// consecutive k-blocks for the other stages.  The split of a tile that
// finishes last sums the fp32 partials in split order (deterministic), runs
// the epilogue and bumps the stage's done counter.  The last CTA to leave
// resets the counters.
//
// Roles: warps 0-3 epilogue, warp 4 TMA producer, warp 5 TMEM allocator and
// MMA issuer.  Every wait is bounded (ptx.cuh).
#pragma once

#include "gemv_sm100.cuh"

namespace svdmlp {

// Unit kinds of a stage.  GEMM: a 128-row weight panel over a K range (the
// four stages of the plain schedule).  CONTRACT (the contracted schedule's
// gate/up stage): one ff tile of the SwiGLU GEMM over the whole rank, its H
// tile kept in shared memory and multiplied at once by the u_down columns of
// that ff slice, all rank tiles; the fp32 product is this tile's partial of
// T = H . u_down.  REDUCE: 32 features of T summed over every CONTRACT tile's
// partial in tile order (deterministic) and rounded to fp16 once.
enum DecKind : int { KIND_GEMM = 0, KIND_CONTRACT = 1, KIND_REDUCE = 2 };

struct alignas(64) DecStage {
  CUtensorMap x, x2, w, w2;  // token operand(s) [M, K] (2-D) and packed tiled weight(s) [N, K] (4-D)
  CUtensorMap w3;            // CONTRACT: packed u_down^T [r, ff], 128-row boxes
  void* out;
  long long ld_out;
  float* partials;   // [tiles][splits][nb][TOK][128] fp32 (token-major)
  int* tile_counters;
  int N, K, n_tiles, k_blocks, splits, kb_per_split, units, unit_base;
  int nb;            // 1, or 2 for the dual SwiGLU stage
  int in_f16;        // operand type: fp16 (1) or bf16 (0)
  int epi;           // EPI_PLAIN, EPI_SWIGLU or EPI_RESID
  int out_kind;      // OUT_BF16, OUT_F16 or OUT_F32
  int kind;          // DecKind
  // CONTRACT: rank tiles of u_down (128 rows), u_down k-blocks over ff, and the
  // T partials [ff tile][TOK tokens][t_ld] fp32; REDUCE reads them (t_slots
  // tiles) and writes fp16 T (out, ld_out; N = rank).
  int r_tiles, ff_kb, t_ld, t_slots;
  float* tpart;
  // fused RMSNorm: `norm` (the first stage) scales each token's outputs by
  // its row scale; `out_stats` (the EPI_RESID stage) receives each token's
  // sum of squares of its bf16 outputs per 128-feature tile.
  int norm;
  float* out_stats;
};

struct LayerDecParams {
  DecStage st[4];
  int num_stages, M, total_units;
  int* done;        // [4] tiles completed per stage in this launch
  int* exit_count;  // CTAs that have left
  int* next_unit;   // unit claim counter
  int* err;
  unsigned long long timeout_ns;
  // L2 prefetch window of the weight stream, in slots: while streaming, the
  // producer keeps the next `pf_ahead` slots of its unit requested from HBM
  // into L2; while a unit waits on the previous stage it requests up to
  // `pf_wait` slots beyond those it has already loaded to shared memory.
  int pf_ahead, pf_wait;
  // units blockIdx.x + j * gridDim.x (j < pdl_units) whose weights a CTA
  // prefetches to L2 before it waits for the previous grid
  int pdl_units;
  const __nv_bfloat16* residual;
  long long ld_residual;
  // Fused RMSNorm of a decoder block: the previous block's per-slice sums of
  // squares of this block's input, [M][stats_ld], norm_parts slices of the
  // norm_dim features; also the row stride of the stages' out_stats.
  const float* norm_stats;
  int norm_parts, norm_dim, stats_ld;
  float norm_eps;
  // Optional timeline (null: off): per CTA kTraceEvents pairs of
  // (tag | unit << 8, globaltimer ns).
  unsigned long long* trace;
};

// Trace tags of the whole-layer decode kernel.
enum TraceTag : unsigned { TR_START = 1, TR_CLAIM = 2, TR_DEP_BEGIN = 3, TR_DEP_END = 4, TR_UNIT_DONE = 5, TR_END = 6 };
constexpr int kTraceEvents = 64;

SVD_DEV void trace_event(const LayerDecParams& p, int& n, unsigned tag, int unit) {
  if (p.trace == nullptr || n >= kTraceEvents) return;
  unsigned long long* e = p.trace + (static_cast<size_t>(blockIdx.x) * kTraceEvents + n) * 2;
  e[0] = static_cast<unsigned long long>(tag) | (static_cast<unsigned long long>(unit + 1) << 8);
  e[1] = global_timer_ns();
  ++n;
}

template <int TOK_, int STAGES_>
struct LayerDecCfg {
  static constexpr int BM = 128, BK = 64, TOK = TOK_, STAGES = STAGES_;
  static constexpr int W_BYTES = BM * BK * 2;
  static constexpr int X_BYTES = TOK * BK * 2;
  static constexpr int SLOT_BYTES = 2 * W_BYTES + 2 * X_BYTES;
  static constexpr int ACC_BUFS = 2;
  static constexpr int ACC_STRIDE = 2 * TOK;
  // The contracted schedule (16-token tiles only) keeps T accumulators for up
  // to T_CHUNK rank tiles after the two SwiGLU accumulator buffers: all 512
  // columns.  64-token tiles run the plain schedule only.
  static constexpr bool CONTRACT = TOK == 16;
  static constexpr int T_COL0 = ACC_BUFS * ACC_STRIDE;
  static constexpr uint32_t TMEM_COLS =
      CONTRACT ? 512 : ACC_BUFS * ACC_STRIDE <= 64 ? 64 : ACC_BUFS * ACC_STRIDE <= 128 ? 128 : 256;
  static constexpr int T_CHUNK = CONTRACT ? (512 - T_COL0) / TOK : 0;  // rank tiles per TMEM pass
  static constexpr int OFF_W = 0;                        // [slot][2] weight tiles
  static constexpr int OFF_X = STAGES * 2 * W_BYTES;     // [slot][2] token tiles
  // CONTRACT: the H tile as the B operand of its u_down product, two
  // [TOK x 64] K-major 128B-swizzled tiles (ff k-blocks 2f and 2f + 1)
  static constexpr int OFF_H = OFF_X + STAGES * 2 * X_BYTES;
  static constexpr int H_BYTES = CONTRACT ? 2 * X_BYTES : 0;
  // REDUCE: [4 slot groups][TOK tokens][32 features] fp32 partial sums
  static constexpr int OFF_RED = OFF_H + H_BYTES;
  static constexpr int RED_BYTES = CONTRACT ? 4 * TOK * 32 * 4 : 0;
  static constexpr int OFF_RSTD = OFF_RED + RED_BYTES;     // fused RMSNorm: row scale per token
  static constexpr int OFF_SS = OFF_RSTD + TOK * 4;        // [4 warps][16 tokens] sums of squares
  static constexpr int OFF_BAR = OFF_SS + 4 * 16 * 4;
  static constexpr int QUEUE = 4;  // claimed units in flight per CTA
  // + h_ready, h_empty, t_full, t_empty for CONTRACT units
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 1 + 2 * QUEUE + 4;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 64 + 4 * QUEUE + 1024;
  static_assert(X_BYTES % 1024 == 0, "token tiles stay 1024-byte aligned");
  static_assert(SMEM_BYTES <= 227 * 1024, "fits one CTA's shared memory");
  static_assert(TOK == 16 || TOK == 64, "16 or 64 tokens per tile");
};

struct LdUnit {
  int s, n_t, ks, kb0, kb1;
};

SVD_DEV LdUnit layer_dec_unit(const LayerDecParams& p, int u) {
  int s = 0;
  while (s + 1 < p.num_stages && u >= p.st[s + 1].unit_base) ++s;
  const DecStage& st = p.st[s];
  const int local = u - st.unit_base;
  LdUnit c;
  c.s = s;
  c.ks = local % st.splits;
  c.n_t = local / st.splits;
  c.kb0 = c.ks * st.kb_per_split;
  c.kb1 = min(c.kb0 + st.kb_per_split, st.k_blocks);
  return c;
}

// Shared-memory slots a unit occupies: one per k-block for the dual stage
// (two branches), one per pair of k-blocks otherwise; a CONTRACT unit adds one
// slot per rank tile (the two u_down k-blocks of its ff slice); REDUCE units
// load nothing.
SVD_DEV int unit_slots(const LayerDecParams& p, const LdUnit& c) {
  const DecStage& st = p.st[c.s];
  if (st.kind == KIND_REDUCE) return 0;
  const int nk = c.kb1 - c.kb0;
  if (st.kind == KIND_CONTRACT) return nk + st.r_tiles;
  return st.nb == 2 ? nk : (nk + 1) / 2;
}

// Split-K fix-up of the first 16-token chunk with few tokens: this thread's
// feature row of every split's partial (JM splits and TM tokens at most, all
// loads in flight at once), summed in split order into v (and w for the dual
// stage).  `slot` is the element distance between two splits' partials (two
// branches each).
template <int JM, int TM, int SLOT>
SVD_DEV void ld_sum_splits(const float* base, int splits, int tv, bool dual, float (&v)[16], float (&w)[16]) {
  constexpr int BM = 128;
  float g[JM][TM], u[JM][TM];
#pragma unroll
  for (int j = 0; j < JM; ++j) {
    const float* src = base + static_cast<size_t>(j * 2) * SLOT;
#pragma unroll
    for (int t = 0; t < TM; ++t) {
      const bool ld = j < splits && t < tv;
      g[j][t] = ld ? __ldcg(src + t * BM) : 0.f;
      u[j][t] = ld && dual ? __ldcg(src + SLOT + t * BM) : 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < JM; ++j) {
    if (j < splits) {
#pragma unroll
      for (int t = 0; t < TM; ++t) {
        v[t] += g[j][t];
        w[t] += u[j][t];
      }
    }
  }
}

// Stores one 16-token chunk of a unit's outputs (thread = feature f of the
// 128-row tile; all 128 epilogue threads call it together).  The first stage
// of a fused block scales token t by its RMSNorm row scale; an EPI_RESID
// stage with out_stats also writes each token's sum of squares of its bf16
// outputs over the tile's 128 features (summed across the four warps in
// warp order).
template <int TOK>
SVD_DEV void ld_store_chunk(const LayerDecParams& p, const DecStage& st, int f, int t0, float (&v)[16],
                            const float* rstd, float* ss_smem, int n_t) {
  if (st.norm) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= rstd[min(t0 + j, TOK - 1)];
  }
  float ss[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    ss[j] = 0.0f;
    const int t = t0 + j;
    if (t < p.M && f < st.N) {
      float x = v[j];
      if (st.epi == EPI_RESID) x += __bfloat162float(p.residual[static_cast<long long>(t) * p.ld_residual + f]);
      const long long off = static_cast<long long>(t) * st.ld_out + f;
      if (st.out_kind == OUT_F32) static_cast<float*>(st.out)[off] = x;
      else if (st.out_kind == OUT_F16) {
        if (f16_out_of_range(x)) flag_range(p.err);  // reported, never silent
        static_cast<__half*>(st.out)[off] = __float2half_rn(fminf(fmaxf(x, -65504.f), 65504.f));
      } else {
        const __nv_bfloat16 b = __float2bfloat16(x);
        static_cast<__nv_bfloat16*>(st.out)[off] = b;
        const float r = __bfloat162float(b);
        ss[j] = r * r;
      }
    }
  }
  if (st.out_stats != nullptr) {
    const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float a = ss[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) ss_smem[warp * 16 + j] = a;
    }
    named_barrier_sync(5, 128);
    if (threadIdx.x < 16 && t0 + static_cast<int>(threadIdx.x) < p.M) {
      const int j = static_cast<int>(threadIdx.x);
      const float tot = ss_smem[j] + ss_smem[16 + j] + ss_smem[32 + j] + ss_smem[48 + j];
      st.out_stats[static_cast<long long>(t0 + j) * p.stats_ld + n_t] = tot;
    }
    named_barrier_sync(5, 128);  // the buffer is free for the next chunk
  }
}

template <class Cfg>
__global__ void __launch_bounds__(192) layer_decode_kernel(const __grid_constant__ LayerDecParams p) {
  constexpr int STAGES = Cfg::STAGES;
  constexpr int TOK = Cfg::TOK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + Cfg::ACC_BUFS;
  uint64_t* drain = acc_empty + Cfg::ACC_BUFS;
  uint64_t* q_full = drain + 1;            // [QUEUE] producer -> MMA, epilogue
  uint64_t* q_empty = q_full + Cfg::QUEUE; // [QUEUE] MMA + 4 epilogue warps -> producer
  // CONTRACT units: H tile written (epilogue -> MMA), H tile read (MMA ->
  // epilogue), T accumulators of a rank-tile chunk full (MMA -> epilogue) and
  // drained (4 epilogue warps -> MMA)
  uint64_t* h_ready = q_empty + Cfg::QUEUE;
  uint64_t* h_empty = h_ready + 1;
  uint64_t* t_full = h_ready + 2;
  uint64_t* t_empty = h_ready + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* epi_abort = reinterpret_cast<volatile int*>(tmem_slot + 3);
  volatile int* unit_q = reinterpret_cast<volatile int*>(smem + Cfg::OFF_MISC + 64);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  // Programmatic dependent launch: the next launch on the stream may start its
  // CTAs as soon as SMs free up (they wait for this grid before touching any
  // state it writes), so the next layer's weight stream overlaps this one's tail.
  grid_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < Cfg::ACC_BUFS; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < Cfg::QUEUE; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 5);
    }
    mbar_init(h_ready, 1);
    mbar_init(h_empty, 1);
    mbar_init(t_full, 1);
    mbar_init(t_empty, 4);
    *abort_flag = 0;
    *fix_flag = 0;
    *epi_abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 4 && lane == 0) {
    for (int s = 0; s < p.num_stages; ++s) {
      if (p.st[s].kind == KIND_REDUCE) continue;  // no tensor maps
      prefetch_tensormap(&p.st[s].x);
      prefetch_tensormap(&p.st[s].w);
      if (p.st[s].nb == 2) {
        prefetch_tensormap(&p.st[s].x2);
        prefetch_tensormap(&p.st[s].w2);
      }
      if (p.st[s].kind == KIND_CONTRACT) prefetch_tensormap(&p.st[s].w3);
    }
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.err, p.timeout_ns};

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // k-blocks of slot i of unit c: dual -> kb0 + i (both branches);
      // otherwise kb0 + 2i and kb0 + 2i + 1 (the second may not exist).
      // weights are read once per call: evict them from L2 first, before the
      // activations and split-K partials that are read again
      const uint64_t wpol = l2_policy_weight_stream();
      auto slot_w = [&](const LdUnit& c, int i, int sl) {
        const DecStage& st = p.st[c.s];
        uint8_t* w0 = smem + Cfg::OFF_W + (sl * 2) * Cfg::W_BYTES;
        uint8_t* w1 = w0 + Cfg::W_BYTES;
        // weights: packed tile-major layout, 4-D loads at (k-block, 16-row group)
        const int grp = c.n_t * Cfg::BM / 16;
        if (st.kind == KIND_CONTRACT && i >= c.kb1 - c.kb0) {
          // u_down^T rows of rank tile j, the two k-blocks of this ff slice
          const int j = i - (c.kb1 - c.kb0), kbu = 2 * c.n_t;
          tma_load_4d_hint(&st.w3, &full[sl], w0, kbu, j * (Cfg::BM / 16), wpol);
          if (kbu + 1 < st.ff_kb) tma_load_4d_hint(&st.w3, &full[sl], w1, kbu + 1, j * (Cfg::BM / 16), wpol);
        } else if (st.nb == 2) {
          tma_load_4d_hint(&st.w, &full[sl], w0, c.kb0 + i, grp, wpol);
          tma_load_4d_hint(&st.w2, &full[sl], w1, c.kb0 + i, grp, wpol);
        } else {
          tma_load_4d_hint(&st.w, &full[sl], w0, c.kb0 + 2 * i, grp, wpol);
          if (c.kb0 + 2 * i + 1 < c.kb1) tma_load_4d_hint(&st.w, &full[sl], w1, c.kb0 + 2 * i + 1, grp, wpol);
        }
      };
      auto slot_x = [&](const LdUnit& c, int i, int sl) {
        const DecStage& st = p.st[c.s];
        uint8_t* x0 = smem + Cfg::OFF_X + (sl * 2) * Cfg::X_BYTES;
        uint8_t* x1 = x0 + Cfg::X_BYTES;
        if (st.kind == KIND_CONTRACT && i >= c.kb1 - c.kb0) return;  // the H tile is already in shared memory
        if (st.nb == 2) {
          tma_load_2d(&st.x, &full[sl], x0, (c.kb0 + i) * Cfg::BK, 0);
          tma_load_2d(&st.x2, &full[sl], x1, (c.kb0 + i) * Cfg::BK, 0);
        } else {
          tma_load_2d(&st.x, &full[sl], x0, (c.kb0 + 2 * i) * Cfg::BK, 0);
          if (c.kb0 + 2 * i + 1 < c.kb1) tma_load_2d(&st.x, &full[sl], x1, (c.kb0 + 2 * i + 1) * Cfg::BK, 0);
        }
      };
      auto slot_pf = [&](const LdUnit& c, int i) {
        const DecStage& st = p.st[c.s];
        const int grp = c.n_t * Cfg::BM / 16;
        if (st.kind == KIND_CONTRACT && i >= c.kb1 - c.kb0) {
          const int j = i - (c.kb1 - c.kb0), kbu = 2 * c.n_t;
          tma_prefetch_4d(&st.w3, kbu, j * (Cfg::BM / 16));
          if (kbu + 1 < st.ff_kb) tma_prefetch_4d(&st.w3, kbu + 1, j * (Cfg::BM / 16));
        } else if (st.nb == 2) {
          tma_prefetch_4d(&st.w, c.kb0 + i, grp);
          tma_prefetch_4d(&st.w2, c.kb0 + i, grp);
        } else {
          tma_prefetch_4d(&st.w, c.kb0 + 2 * i, grp);
          if (c.kb0 + 2 * i + 1 < c.kb1) tma_prefetch_4d(&st.w, c.kb0 + 2 * i + 1, grp);
        }
      };
      auto slot_bytes = [&](const LdUnit& c, int i) -> uint32_t {
        const DecStage& st = p.st[c.s];
        if (st.kind == KIND_CONTRACT && i >= c.kb1 - c.kb0)
          return (2 * c.n_t + 1 < st.ff_kb ? 2u : 1u) * Cfg::W_BYTES;
        const bool two = st.nb == 2 || c.kb0 + 2 * i + 1 < c.kb1;
        return (two ? 2u : 1u) * (Cfg::W_BYTES + Cfg::X_BYTES);
      };
      int it = 0;  // slot index over the whole run
      bool ok = true;
      // Weights are never written by a kernel: before waiting for the previous
      // grid, request into L2 the weights of the units the CTAs will most
      // likely claim first (blockIdx.x, then one grid further per round).
      // Everything else (claims, activations, counters, partials) comes
      // after the wait.
      for (int j = 0; j < p.pdl_units; ++j) {
        const int u0 = static_cast<int>(blockIdx.x) + j * static_cast<int>(gridDim.x);
        if (u0 >= p.total_units) break;
        const LdUnit c0 = layer_dec_unit(p, u0);
        const int n0 = unit_slots(p, c0);
        for (int i = 0; i < n0; ++i) slot_pf(c0, i);
      }
      grid_dependency_wait();
      int ready_stage = 0;  // stages whose inputs are known complete (stage 0 always)
      int ntr = 0;          // producer trace events (slots [0, 40))
      trace_event(p, ntr, TR_START, -1);
      for (int qi = 0; ok; ++qi) {
        // claim the next unit and hand it to the MMA and epilogue warps
        const int qs = qi % Cfg::QUEUE;
        if (!mbar_wait(&q_empty[qs], (static_cast<uint32_t>(qi / Cfg::QUEUE) & 1u) ^ 1u, ctx, SITE_PRODUCER_EMPTY)) {
          ok = false;
          unit_q[qs] = -1;
          mbar_arrive(&q_full[qs]);
          break;
        }
        // The first unit of every CTA is its own index (no atomic: at launch
        // the claim would queue behind every CTA's weight prefetches); later
        // units come from the shared counter, in order after the first wave.
        const int u = qi == 0 ? static_cast<int>(blockIdx.x)
                              : static_cast<int>(gridDim.x) + atomicAdd(p.next_unit, 1);
        unit_q[qs] = u < p.total_units ? u : -1;
        mbar_arrive(&q_full[qs]);  // release: the unit id is visible to the waiters
        if (u >= p.total_units) break;
        if (ntr < 40) trace_event(p, ntr, TR_CLAIM, u);
        const LdUnit c = layer_dec_unit(p, u);
        const int ns = unit_slots(p, c);
        // REDUCE units load nothing, but the producer still waits for the
        // CONTRACT stage before it claims again: CTAs with nothing else to do
        // would otherwise queue several reduce units each and run them one
        // after another at the end.
        if (p.st[c.s].kind == KIND_REDUCE) {
          if (c.s > ready_stage) {
            if (!wait_counter_geq(&p.done[c.s - 1], p.st[c.s - 1].n_tiles, ctx, SITE_DEPENDENCY)) ok = false;
            ready_stage = c.s;
          }
          continue;
        }
        int i = 0;
        int pf = 0;  // slots of this unit requested so far (to L2 or shared memory)
        if (c.s > ready_stage) {
          // Weights first: as many slots as the ring frees up, then wait for
          // the previous stage, then the token tiles of those slots.
          int pre = 0;
          for (; pre < min(ns, STAGES); ++pre) {
            const int sl = (it + pre) % STAGES;
            const uint32_t ph = static_cast<uint32_t>((it + pre) / STAGES) & 1u;
            if (!mbar_wait(&empty[sl], ph ^ 1u, ctx, SITE_PRODUCER_EMPTY)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[sl], slot_bytes(c, pre));
            slot_w(c, pre, sl);
          }
          if (!ok) break;
          for (pf = pre; pf < min(ns, pre + p.pf_wait); ++pf) slot_pf(c, pf);
          if (ntr < 40) trace_event(p, ntr, TR_DEP_BEGIN, u);
          if (!wait_counter_geq(&p.done[c.s - 1], p.st[c.s - 1].n_tiles, ctx, SITE_DEPENDENCY)) {
            // Complete the slots already announced with their token tiles so
            // the barrier phases stay consistent, then stop.
            ok = false;
          }
          if (ntr < 40) trace_event(p, ntr, TR_DEP_END, u);
          fence_proxy_async_global();
          for (int j = 0; j < pre; ++j) slot_x(c, j, (it + j) % STAGES);
          it += pre;
          i = pre;
          ready_stage = c.s;
          if (!ok) break;
        }
        for (; i < ns; ++i, ++it) {
          const int sl = it % STAGES;
          const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
          if (pf < i + 1) pf = i + 1;
          for (; pf < min(ns, i + 1 + p.pf_ahead); ++pf) slot_pf(c, pf);
          if (!mbar_wait(&empty[sl], ph ^ 1u, ctx, SITE_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[sl], slot_bytes(c, i));
          slot_w(c, i, sl);
          slot_x(c, i, sl);
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        if (it > s) {
          const int last = s + ((it - 1 - s) / STAGES) * STAGES;
          mbar_wait(&full[s], static_cast<uint32_t>(last / STAGES) & 1u, ctx, SITE_DRAIN_LOADS, false);
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    grid_dependency_wait();
    if (lane == 0) {
      const uint32_t idesc_bf = make_idesc_16bit(Cfg::BM, TOK, false);
      const uint32_t idesc_h = make_idesc_16bit(Cfg::BM, TOK, true);
      int it = 0, acc_it = 0;
      int cu = 0, tc = 0;  // CONTRACT units and T chunks issued by this CTA
      bool ok = true;
      for (int qi = 0; ok; ++qi) {
        const int qs = qi % Cfg::QUEUE;
        if (!mbar_wait(&q_full[qs], static_cast<uint32_t>(qi / Cfg::QUEUE) & 1u, ctx, SITE_MMA_FULL)) break;
        const int u = unit_q[qs];
        mbar_arrive(&q_empty[qs]);
        if (u < 0) break;
        const LdUnit c = layer_dec_unit(p, u);
        const DecStage& st = p.st[c.s];
        if (st.kind == KIND_REDUCE) continue;  // no MMA: the epilogue sums partials
        const uint32_t idesc = st.in_f16 ? idesc_h : idesc_bf;
        // the SwiGLU accumulation over the rank (a CONTRACT unit's first phase)
        const int ns = st.kind == KIND_CONTRACT ? c.kb1 - c.kb0 : unit_slots(p, c);
        const int b = acc_it % Cfg::ACC_BUFS;
        const uint32_t aph = static_cast<uint32_t>(acc_it / Cfg::ACC_BUFS) & 1u;
        if (!mbar_wait(&acc_empty[b], aph ^ 1u, ctx, SITE_MMA_ACC_EMPTY)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(b * Cfg::ACC_STRIDE);
        for (int i = 0; i < ns; ++i, ++it) {
          const int sl = it % STAGES;
          const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
          if (!mbar_wait(&full[sl], ph, ctx, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w0 = smem_addr(smem + Cfg::OFF_W + (sl * 2) * Cfg::W_BYTES);
          const uint32_t x0 = smem_addr(smem + Cfg::OFF_X + (sl * 2) * Cfg::X_BYTES);
          const bool dual = st.nb == 2;
          const bool second = dual || c.kb0 + 2 * i + 1 < c.kb1;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !second) break;
            const uint32_t wa = w0 + h * Cfg::W_BYTES, xa = x0 + h * Cfg::X_BYTES;
            const uint32_t dd = dual ? d + h * TOK : d;
#pragma unroll
            for (int k = 0; k < Cfg::BK / 16; ++k) {
              const bool first = i == 0 && k == 0 && (dual || h == 0);
              umma_f16kind(dd, make_sw128_desc(wa + k * 32), make_sw128_desc(xa + k * 32), idesc, first ? 0u : 1u);
            }
          }
          umma_commit(&empty[sl]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
        ++acc_it;
        if constexpr (Cfg::CONTRACT) {
          if (st.kind == KIND_CONTRACT) {
            // Second phase: T partial [rank tile x TOK] = u_down^T[tile, ff slice]
            // . H[ff slice, TOK], for every rank tile, in chunks of T_CHUNK tiles
            // of TMEM columns; the H tile comes from shared memory.
            if (!mbar_wait(h_ready, static_cast<uint32_t>(cu) & 1u, ctx, SITE_MMA_FULL)) break;
            tc_fence_after();
            const uint32_t hb = smem_addr(smem + Cfg::OFF_H);
            const bool two = 2 * c.n_t + 1 < st.ff_kb;
            for (int j0 = 0; j0 < st.r_tiles && ok; j0 += Cfg::T_CHUNK) {
              const int j1 = min(st.r_tiles, j0 + Cfg::T_CHUNK);
              if (!mbar_wait(t_empty, (static_cast<uint32_t>(tc) & 1u) ^ 1u, ctx, SITE_MMA_ACC_EMPTY)) {
                ok = false;
                break;
              }
              tc_fence_after();
              for (int j = j0; j < j1; ++j, ++it) {
                const int sl = it % STAGES;
                const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
                if (!mbar_wait(&full[sl], ph, ctx, SITE_MMA_FULL)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                const uint32_t w0 = smem_addr(smem + Cfg::OFF_W + (sl * 2) * Cfg::W_BYTES);
                const uint32_t dT = tmem_base + static_cast<uint32_t>(Cfg::T_COL0 + (j - j0) * TOK);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  if (h == 1 && !two) break;
#pragma unroll
                  for (int k = 0; k < Cfg::BK / 16; ++k)
                    umma_f16kind(dT, make_sw128_desc(w0 + h * Cfg::W_BYTES + k * 32),
                                 make_sw128_desc(hb + h * Cfg::X_BYTES + k * 32), idesc_h, (h | k) ? 1u : 0u);
                }
                umma_commit(&empty[sl]);
              }
              if (!ok) break;
              umma_commit(t_full);
              ++tc;
            }
            if (!ok) break;
            umma_commit(h_empty);  // the H tile may be overwritten once these MMAs are done
            ++cu;
          }
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, ctx, SITE_DRAIN_MMA, false);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    grid_dependency_wait();
    const int q = warp;
    int acc_it = 0;
    int ecu = 0, etc = 0;  // CONTRACT units and T chunks drained by this CTA
    float* rstd = reinterpret_cast<float*>(smem + Cfg::OFF_RSTD);
    float* ss_smem = reinterpret_cast<float*>(smem + Cfg::OFF_SS);
    if (p.norm_stats != nullptr) {
      // fused RMSNorm: each token's row scale, from the previous block's
      // per-slice sums of squares, summed in slice order
      for (int t = threadIdx.x; t < min(p.M, TOK); t += 128)
        rstd[t] = norm_row_scale(p.norm_stats, p.stats_ld, p.norm_parts, p.norm_dim, p.norm_eps, t);
      named_barrier_sync(1, 128);
    }
    int ntr = 40;  // epilogue trace events (slots [40, 64))
    for (int qi = 0;; ++qi) {
      const int qs = qi % Cfg::QUEUE;
      bool qok = mbar_wait(&q_full[qs], static_cast<uint32_t>(qi / Cfg::QUEUE) & 1u, ctx, SITE_EPI_ACC_FULL);
      qok = __all_sync(0xffffffffu, qok);
      // The four warps take the same decision (a timed-out wait in any of
      // them stops all), so that none is left alone at a named barrier.
      if (!qok && lane == 0) *epi_abort = 1;
      named_barrier_sync(2, 128);
      if (*epi_abort) break;
      const int u = unit_q[qs];  // the same entry for all four warps
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[qs]);
      if (u < 0) break;
      const LdUnit c = layer_dec_unit(p, u);
      const DecStage& st = p.st[c.s];
      if constexpr (Cfg::CONTRACT) {
        if (st.kind == KIND_REDUCE) {
          // 32 features of T: wait (bounded) for every CONTRACT tile, sum its
          // partials in tile order -- four slot groups (one per warp), then the
          // groups in order -- round once to fp16 and publish.
          if (threadIdx.x == 0) {
            if (ntr < kTraceEvents - 1) trace_event(p, ntr, TR_DEP_BEGIN, u);
            *fix_flag = wait_counter_geq(&p.done[c.s - 1], p.st[c.s - 1].n_tiles, ctx, SITE_DEPENDENCY) ? 1 : 0;
            if (ntr < kTraceEvents - 1) trace_event(p, ntr, TR_DEP_END, u);
          }
          // thread 0's acquire load saw every CONTRACT tile's release; the
          // CTA barrier orders the other threads' reads after it
          named_barrier_sync(1, 128);
          if (!*fix_flag) break;  // the same for all four warps
          const int tv = min(p.M, TOK);
          const int feat = c.n_t * 32 + static_cast<int>(lane);
          const int S = st.t_slots, g0 = q * S / 4, g1 = (q + 1) * S / 4;
          const float* base = st.tpart + feat;
          const size_t slot_stride = static_cast<size_t>(TOK) * st.t_ld;
          // Each thread sums its group's slots in slot order, in registers:
          // one token with 32 loads in flight, more tokens four at a time with
          // 8 slots x 4 tokens in flight (the reduction is latency-bound).
          float* red = reinterpret_cast<float*>(smem + Cfg::OFF_RED);
          if (tv == 1) {
            float acc = 0.f;
            for (int b0 = g0; b0 < g1; b0 += 32) {
              float l[32];
#pragma unroll
              for (int k = 0; k < 32; ++k) l[k] = b0 + k < g1 ? __ldcg(base + (b0 + k) * slot_stride) : 0.f;
#pragma unroll
              for (int k = 0; k < 32; ++k) acc += l[k];
            }
            red[q * TOK * 32 + lane] = acc;
          } else {
            for (int t0 = 0; t0 < tv; t0 += 4) {
              float acc[4] = {0.f, 0.f, 0.f, 0.f};
              for (int b0 = g0; b0 < g1; b0 += 8) {
                float l[8][4];
#pragma unroll
                for (int k = 0; k < 8; ++k)
#pragma unroll
                  for (int t = 0; t < 4; ++t)
                    l[k][t] = (b0 + k < g1 && t0 + t < tv)
                                  ? __ldcg(base + (b0 + k) * slot_stride + static_cast<size_t>(t0 + t) * st.t_ld)
                                  : 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
#pragma unroll
                  for (int t = 0; t < 4; ++t) acc[t] += l[k][t];
              }
#pragma unroll
              for (int t = 0; t < 4; ++t)
                if (t0 + t < tv) red[(q * TOK + t0 + t) * 32 + lane] = acc[t];
            }
          }
          named_barrier_sync(1, 128);
          if (q == 0 && feat < st.N) {
            __half* o = static_cast<__half*>(st.out);
            for (int t = 0; t < tv; ++t) {
              float sum = red[(0 * TOK + t) * 32 + lane];
              sum += red[(1 * TOK + t) * 32 + lane];
              sum += red[(2 * TOK + t) * 32 + lane];
              sum += red[(3 * TOK + t) * 32 + lane];
              if (f16_out_of_range(sum)) flag_range(p.err);
              o[static_cast<long long>(t) * st.ld_out + feat] = __float2half_rn(fminf(fmaxf(sum, -65504.f), 65504.f));
            }
          }
          named_barrier_sync(1, 128);  // stores before the release; the buffer free for the next unit
          if (threadIdx.x == 0) red_add_release_gpu(&p.done[c.s], 1);
          if (threadIdx.x == 0 && ntr < kTraceEvents - 1) trace_event(p, ntr, TR_UNIT_DONE, u);
          continue;
        }
      }
      const int b = acc_it % Cfg::ACC_BUFS;
      const uint32_t aph = static_cast<uint32_t>(acc_it / Cfg::ACC_BUFS) & 1u;
      bool ok = mbar_wait(&acc_full[b], aph, ctx, SITE_EPI_ACC_FULL);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) *epi_abort = 1;
      named_barrier_sync(2, 128);
      if (*epi_abort) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * Cfg::ACC_STRIDE);
      const int row = q * 32 + static_cast<int>(lane);
      const int f = c.n_t * Cfg::BM + row;
      const int tv = min(p.M, TOK);
      const bool dual = st.nb == 2;
      constexpr int NCH = TOK / 16;
      const size_t tile_slot = static_cast<size_t>(c.n_t) * st.splits;
      // token-major partial: a warp's 32 features of one token are one 128-byte line
      float* slot = st.partials + ((tile_slot + c.ks) * 2) * (Cfg::BM * TOK) + row;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        uint32_t rg[16], ru[16];
        tmem_ld_x16(tacc + ch * 16, rg);
        tmem_ld_x16(tacc + TOK + ch * 16, ru);  // unused columns for one-branch stages
        tmem_ld_wait();
        if (ch == NCH - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (16 * ch >= tv) continue;
        float v[16], w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __uint_as_float(rg[j]);
          w[j] = __uint_as_float(ru[j]);
        }
        if (st.splits == 1) {
          if (dual) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = silu_mul(v[j], w[j]);
          }
          if (Cfg::CONTRACT && st.kind == KIND_CONTRACT) {
            // H tile -> shared memory, as the B operand [TOK tokens x 128 ff]
            // of this unit's u_down product: two K-major [TOK x 64] tiles in
            // the 128-byte swizzle (16-byte chunk c of row t at c ^ (t % 8)).
            // The previous CONTRACT unit's MMAs must be done reading it.
            bool hok = ecu == 0 || mbar_wait(h_empty, static_cast<uint32_t>(ecu - 1) & 1u, ctx, SITE_EPI_ACC_FULL);
            hok = __all_sync(0xffffffffu, hok);
            if (!hok && lane == 0) *epi_abort = 1;
            bool bad = false;
            uint8_t* ht = smem + Cfg::OFF_H + (row >> 6) * Cfg::X_BYTES;
            const int col = row & 63;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              if (t < tv) bad |= f16_out_of_range(v[t]);
              const __half hv = __float2half_rn(fminf(fmaxf(v[t], -65504.f), 65504.f));
              *reinterpret_cast<__half*>(ht + t * 128 + (((col >> 3) ^ (t & 7)) << 4) + (col & 7) * 2) = hv;
            }
            if (bad) flag_range(p.err);
            fence_proxy_async_smem();
            named_barrier_sync(1, 128);
            if (threadIdx.x == 0 && !*epi_abort) mbar_arrive(h_ready);
          } else {
            ld_store_chunk<TOK>(p, st, f, 16 * ch, v, rstd, ss_smem, c.n_t);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (16 * ch + j < tv) {
              __stcg(slot + (16 * ch + j) * Cfg::BM, v[j]);
              if (dual) __stcg(slot + Cfg::BM * TOK + (16 * ch + j) * Cfg::BM, w[j]);
            }
          }
        }
      }
      if (Cfg::CONTRACT && st.kind == KIND_CONTRACT) {
        if (*epi_abort) break;
        // Second phase: this ff tile's partial of T, rank tile by rank tile,
        // token-major [TOK][t_ld] fp32 in the tile's slot (a warp's 32
        // features of one token are one 128-byte line).
        const int tv2 = min(p.M, TOK);
        float* dst = st.tpart + static_cast<size_t>(c.n_t) * TOK * st.t_ld;
        bool tok = true;
        for (int j0 = 0; j0 < st.r_tiles && tok; j0 += Cfg::T_CHUNK) {
          const int j1 = min(st.r_tiles, j0 + Cfg::T_CHUNK);
          tok = mbar_wait(t_full, static_cast<uint32_t>(etc) & 1u, ctx, SITE_EPI_ACC_FULL);
          tok = __all_sync(0xffffffffu, tok);
          if (!tok) break;
          tc_fence_after();
          for (int j = j0; j < j1; ++j) {
            uint32_t r16[16];
            tmem_ld_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(Cfg::T_COL0 + (j - j0) * TOK), r16);
            tmem_ld_wait();
            const int fr = j * Cfg::BM + row;
            if (fr < st.N) {
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (t < tv2) __stcg(dst + static_cast<size_t>(t) * st.t_ld + fr, __uint_as_float(r16[t]));
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(t_empty);
          ++etc;
        }
        if (!tok && lane == 0) *epi_abort = 1;
        named_barrier_sync(2, 128);
        if (*epi_abort) break;
        ++ecu;
      }
      bool finished = st.splits == 1;  // this unit completed its tile
      if (st.splits > 1) {
        // Every thread's partial stores, then one acq_rel increment: the
        // barrier orders the stores before it and the release is cumulative.
        named_barrier_sync(1, 128);
        if (threadIdx.x == 0) {
          const int old = atom_add_acq_rel_gpu(&st.tile_counters[c.n_t], 1);
          *fix_flag = (old == st.splits - 1) ? 1 : 0;
        }
        named_barrier_sync(1, 128);
        if (*fix_flag) {
          const float* base = st.partials + (tile_slot * 2) * (Cfg::BM * TOK) + row;
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            if (16 * ch >= tv) continue;
            float v[16], w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              v[j] = 0.f;
              w[j] = 0.f;
            }
            // Few tokens: every split's loads in flight at once (one round trip
            // instead of one per pair of splits); the sum is in split order.
            if (tv <= 4 && st.splits <= 8) {
              ld_sum_splits<8, 4, Cfg::BM * TOK>(base, st.splits, tv, dual, v, w);
            } else if (tv <= 8 && st.splits <= 4) {
              ld_sum_splits<4, 8, Cfg::BM * TOK>(base, st.splits, tv, dual, v, w);
            } else {
            // Two splits' loads in flight per step (one 128-byte line per warp
            // and token); the sum is in split order.
#pragma unroll 1
            for (int s0 = 0; s0 < st.splits; s0 += 2) {
              float g[2][16], u[2][16];
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const bool have = s0 + j < st.splits;
                const float* src = base + static_cast<size_t>((s0 + j) * 2) * (Cfg::BM * TOK) + 16 * ch * Cfg::BM;
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                  const bool ld = have && 16 * ch + t < tv;
                  g[j][t] = ld ? __ldcg(src + t * Cfg::BM) : 0.f;
                  u[j][t] = ld && dual ? __ldcg(src + Cfg::BM * TOK + t * Cfg::BM) : 0.f;
                }
              }
#pragma unroll
              for (int j = 0; j < 2; ++j) {
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                  v[t] += g[j][t];
                  w[t] += u[j][t];
                }
              }
            }
            }
            if (dual) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = silu_mul(v[j], w[j]);
            }
            ld_store_chunk<TOK>(p, st, f, 16 * ch, v, rstd, ss_smem, c.n_t);
          }
          finished = true;
          named_barrier_sync(1, 128);
          if (threadIdx.x == 0) st.tile_counters[c.n_t] = 0;
        }
      }
      if (finished) {
        // Publish the tile: every thread's stores, then one release increment.
        named_barrier_sync(1, 128);
        if (threadIdx.x == 0) red_add_release_gpu(&p.done[c.s], 1);
      }
      if (threadIdx.x == 0 && ntr < kTraceEvents - 1) trace_event(p, ntr, TR_UNIT_DONE, u);
      ++acc_it;
    }
  }

  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    int ntr = kTraceEvents - 1;
    trace_event(p, ntr, TR_END, -1);
    // The last CTA to leave re-arms the counters for the next launch.
    __threadfence();
    const int e = atomicAdd(p.exit_count, 1);
    if (e == static_cast<int>(gridDim.x) - 1) {
      for (int s = 0; s < 4; ++s) atomicExch(&p.done[s], 0);
      atomicExch(p.next_unit, 0);
      atomicExch(p.exit_count, 0);
      __threadfence();
    }
  }
}

}  // namespace svdmlp
