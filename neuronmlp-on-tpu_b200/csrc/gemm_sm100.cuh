// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M, N] = epilogue( A[M, K] . B[N, K]^T )        (both operands K-major)
//
// Dual form (NB == 2): two accumulators per tile, C = silu(A.Bg^T) * (A2.Bu^T);
// this is the fused low-rank gate/up operator's second stage (the SwiGLU
// epilogue of kernels/reference.py:54-72 applied on fp32 accumulators).
// Dual-store form (EPI_DUAL_STORE, NB == 2, shared A): C1 = A.B1^T and
// C2 = A.B2^T, two output maps; the first stage X.[u_g|u_u] as one tile of
// 2 x BN columns that reads its A tile once for both halves.
//
// Operands are bf16 or fp16 (both the same type in one MMA); the output is
// bf16, fp16 or fp32.  The SVD layer keeps its rank-r and ff intermediates in
// fp16: its unit roundoff (2^-11) is 8x smaller than bf16's, at the same
// tensor-core rate, which keeps the layer well inside the max-abs error bound
// that bf16 intermediates overshoot.
//
// Roles (one CTA per SM):
//   warps 0..E-1  epilogue (E = 4 or 8): TMEM -> registers -> (math) ->
//                 swizzled smem -> TMA store
//   warp  E       TMA producer: STAGES-deep smem ring of 128B-swizzled K-major tiles
//   warp  E+1     TMEM allocator + single-thread tcgen05.mma issuer
// Accumulators are double-buffered in TMEM when two fit in its 512 columns,
// so that the epilogue of one tile overlaps the main loop of the next; wider
// tiles use one buffer that the epilogue releases as soon as its TMEM reads
// have returned.
//
// CTAS == 2 (a cluster of two CTAs on two SMs): a tile is 256 x BN; each CTA
// loads its own 128 rows of A and half (BN/2 rows) of B, and the even CTA
// issues tcgen05.mma.cta_group::2, which reads both CTAs' shared memory and
// writes each CTA's 128 accumulator rows into its own TMEM.  Each SM thus
// streams half of the B tile, halving the shared-memory and L2 traffic per
// FLOP against a one-SM 128 x BN tile.  Loads of both CTAs complete on the
// even CTA's `full` barrier; MMA commits arrive on the `empty` / `acc_full`
// barriers of both CTAs; both epilogues release the accumulator on the even
// CTA's `acc_empty` barrier.
//
// Work units are (m_tile, split, n_tile), ordered in groups of `m_group`
// M-tiles: within a group m runs fastest, so the CTAs that run at the same
// time share the same weight (B) tile (read from HBM once per group and
// served from L2 to the group's other M-tiles), and the groups complete one
// after another.
//
// Chained stages (the four GEMMs of one prefill layer): instead of waiting for
// the whole previous launch (griddepcontrol.wait), a stage waits per M-tile on
// counters that the previous stage bumps once a tile's output is in global
// memory, and it lets its own dependents launch at once.  The next stage's
// CTAs therefore take the SMs that the previous stage's tail leaves idle and
// start on the M-tile groups that are already complete.  A launch only starts
// once every CTA of its predecessor is resident, and every wait points to an
// earlier launch, so the chain cannot deadlock.  The last stage's last CTA
// resets the counters.
//
// Split-K: every split writes an fp32 partial tile (its valid rows) to the
// workspace and bumps a per-tile counter.  One-CTA tiles: the split that
// arrives last sums all partials in split order (deterministic) and runs the
// epilogue; nothing waits on another CTA.  CTA pairs (prefill H.u_down, whose
// 48 tiles at 1024 tokens fill only 48 of 74 pairs): every split of a tile
// waits, bounded, for all splits and sums its share of the 32-column chunks,
// in split order.  Units are ordered splits-fastest, so the lowest unfinished
// tile always has all its splits running or done, and the waits end.
#pragma once

#include "ptx.cuh"

namespace svdmlp {

enum EpiKind : int { EPI_PLAIN = 0, EPI_SWIGLU = 1, EPI_RESID = 2, EPI_DUAL_STORE = 3 };
enum OutKind : int { OUT_BF16 = 0, OUT_F16 = 1, OUT_F32 = 2 };

// Error sites recorded in the device error word when a bounded wait expires.
enum ErrSite : int {
  SITE_PRODUCER_EMPTY = 1,
  SITE_MMA_FULL = 2,
  SITE_MMA_ACC_EMPTY = 3,
  SITE_EPI_ACC_FULL = 4,
  SITE_DRAIN_LOADS = 5,
  SITE_DRAIN_MMA = 6,
  SITE_PROBE = 7,
  SITE_DEPENDENCY = 8,
};

// Tensor-parallel exchange fused into the epilogue of the H.u_down GEMM
// (n == 0: none).  Every fp16 output row goes, with 16-byte stores, into
// this rank's slot of every rank's peer buffer (over NVLink; the own buffer
// included) instead of through the output tensor map.  The two slot sets
// alternate from call to call (the parity of this rank's call counter), so a
// rank one call ahead never overwrites a slot a peer still reads.  When every
// CTA of the launch is done, the last one publishes the new count into each
// peer's flag word for this rank (release, system scope).
constexpr int kPushMaxRanks = 8;
struct GemmPush {
  unsigned char* dst[kPushMaxRanks];  // this rank's slot (parity 0) in every rank's buffer
  unsigned* flag[kPushMaxRanks];      // this rank's flag word in every rank's signal area
  unsigned* epoch;                    // this rank's call counter
  unsigned* exit_count;               // CTAs of the launch that are done
  long long parity_bytes;             // distance between the two slot sets
  long long ld;                       // row stride of a slot (elements)
  int n, rank;                        // ranks (0: no exchange), this rank
};

struct GemmParams {
  int M, N, K;  // N is the per-branch width for dual GEMMs
  int m_tiles, n_tiles, k_blocks;
  int splits, kb_per_split;
  int num_units;
  float* partials;  // split-K partial tiles  [tiles][splits][NB][BM*BN]
  int* counters;    // split-K arrival counters [tiles], zero between launches
  int* err;         // device error word
  unsigned long long timeout_ns;
  const __nv_bfloat16* residual;  // EPI_RESID: C = acc + residual (bf16)
  long long ld_residual;
  int m_group;       // M-tiles per group of the unit order (m_tiles: one group, m fastest)
  // Split tail: units [tail_start, num_units) are the last (partial) wave's
  // tiles split `tail_splits` ways over K (tail_kb_per_split k-blocks each);
  // units before it follow `splits`.  tail_start == num_units: no split tail.
  int tail_start, tail_splits, tail_kb_per_split;
  // Fused RMSNorm of a decoder block.  norm_stats (the block's first GEMM,
  // whose weights carry the norm's column weights): output row i is scaled
  // by rsqrt(sum_j norm_stats[i * stats_ld + j] / norm_dim + norm_eps), the
  // sum over j < norm_parts in order.  out_stats (an EPI_RESID stage): for
  // each row, the sum of squares of its bf16 outputs in every 128-column
  // slice, stored at out_stats[row * stats_ld + slice] -- the next block's
  // norm_stats.
  const float* norm_stats;
  int norm_parts, norm_dim, stats_ld;
  float norm_eps;
  float* out_stats;
  // Chained stages (null: not chained, wait for the whole previous launch).
  const int* dep;    // previous stage's per-M-tile tile counters
  int dep_target;    // count that marks an M-tile of the previous stage complete
  int* pub;          // this stage's per-M-tile counters, bumped by each CTA per tile
  int* reset;        // last stage: counters [3][kChainStride] cleared by the last CTA
  int* exit_count;   // last stage: CTAs that have left
  GemmPush push;
};

constexpr int kChainStride = 4096;  // M-tile counters per chained stage

template <int BN_, int NB_, bool SHARED_A_, int STAGES_, int EPI_, bool IN_F16_, int OUT_, int CTAS_ = 1,
          int EPI_WARPS_ = 4, bool B_TILED_ = true>
struct GemmCfg {
  // B (the weight operand) in the packed tile-major layout (4-D tensor map,
  // 2 KB contiguous tiles) or row-major (2-D tensor map).
  static constexpr bool B_TILED = B_TILED_;
  static constexpr int BM = 128, BK = 64;  // rows per CTA, K per stage
  static constexpr int BN = BN_, NB = NB_, STAGES = STAGES_, EPI = EPI_, OUT = OUT_, CTAS = CTAS_;
  // Epilogue warps: 4 (one per TMEM lane quarter) or 8 (two per quarter,
  // each taking every other 32-column chunk).  Warps EPI_WARPS and
  // EPI_WARPS + 1 are the TMA producer and the MMA issuer.
  static constexpr int EPI_WARPS = EPI_WARPS_;
  static constexpr int THREADS = 32 * (EPI_WARPS + 2);
  static constexpr int PRODUCER_WARP = EPI_WARPS, MMA_WARP = EPI_WARPS + 1;
  static constexpr bool IN_F16 = IN_F16_;
  static constexpr bool SHARED_A = SHARED_A_;
  static constexpr int NA = (NB == 2 && !SHARED_A) ? 2 : 1;
  static constexpr int TILE_M = BM * CTAS;  // rows of one work unit
  static constexpr int B_ROWS = BN / CTAS;  // rows of B loaded by each CTA
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static_assert(CTAS == 1 || CTAS == 2, "one CTA or a CTA pair per tile");
  static_assert(B_ROWS % 8 == 0, "B half-tile must hold whole 8-row core-matrix groups");
  static_assert(!B_TILED || B_ROWS % 16 == 0, "tiled B loads whole 16-row groups");
  static_assert(NB == 1 || NB == 2, "one or two accumulators per tile");
  static_assert(NB == 1 || EPI == EPI_SWIGLU || EPI == EPI_DUAL_STORE, "dual GEMMs: SwiGLU or two outputs");
  static_assert(EPI != EPI_DUAL_STORE || (NB == 2 && SHARED_A && CTAS == 2), "dual-store: shared A, CTA pairs");
  static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "four or eight epilogue warps");
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = NA * A_BYTES + NB * B_BYTES;  // per CTA
  static constexpr bool IS_F32 = (OUT == OUT_F32);
  static constexpr int OUT_ELT = IS_F32 ? 4 : 2;
  static constexpr int STG_BYTES = 32 * 32 * OUT_ELT;  // one 32x32 output box per warp buffer
  static constexpr int BSTRIDE = BN <= 128 ? 128 : 256;  // TMEM columns between the two branches
  static constexpr int ACC_STRIDE = NB * BSTRIDE;        // TMEM columns per accumulator buffer
  // Two accumulator buffers when they fit in 512 TMEM columns (the epilogue
  // of one tile overlaps the next tile's main loop); one otherwise.
  static constexpr int ACC_BUFS = 2 * ACC_STRIDE <= 512 ? 2 : 1;
  static_assert(ACC_BUFS * ACC_STRIDE <= 512, "accumulators must fit in 512 TMEM columns");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t IDESC = make_idesc_16bit(TILE_M, BN, IN_F16);

  static constexpr int OFF_A = 0;
  static constexpr int OFF_A2 = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_B = OFF_A2 + (NA == 2 ? STAGES * A_BYTES : 0);
  static constexpr int OFF_B2 = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_STG = OFF_B2 + (NB == 2 ? STAGES * B_BYTES : 0);
  static constexpr int OFF_BAR = OFF_STG + EPI_WARPS * 2 * STG_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;  // + slack for 1024-byte alignment
  static_assert(B_BYTES % 1024 == 0, "operand stage buffers must stay 1024-byte aligned");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

struct UnitCoord {
  int m_t, n_t, ks, kb0, kb1, tile;
  int nsplit;  // splits of this unit's tile
  int pslot;   // partial slot of split 0 of this tile
};

SVD_DEV UnitCoord decode_unit(const GemmParams& p, int u) {
  UnitCoord c;
  // splits fastest: the units of one tile are consecutive, so the lowest
  // unfinished tile always has every split running or done (the pair split-K
  // fix-up waits for all splits of its tile).
  int v, kbp;
  if (u < p.tail_start) {
    c.nsplit = p.splits;
    c.ks = u % p.splits;
    v = u / p.splits;
    kbp = p.kb_per_split;
    c.pslot = v * p.splits;
  } else {
    // the split tail: tiles after the full waves (whose units are unsplit)
    const int t = u - p.tail_start;
    c.nsplit = p.tail_splits;
    c.ks = t % p.tail_splits;
    v = p.tail_start / p.splits + t / p.tail_splits;
    kbp = p.tail_kb_per_split;
    c.pslot = (t / p.tail_splits) * p.tail_splits;
  }
  const int group_units = p.m_group * p.n_tiles;
  const int g = v / group_units;
  const int gm = min(p.m_group, p.m_tiles - g * p.m_group);  // M-tiles in this (possibly last, short) group
  const int in_g = v - g * group_units;
  c.m_t = g * p.m_group + in_g % gm;
  c.n_t = in_g / gm;
  c.kb0 = c.ks * kbp;
  c.kb1 = min(c.kb0 + kbp, p.k_blocks);
  c.tile = c.n_t * p.m_tiles + c.m_t;
  if (u < p.tail_start) c.pslot = c.tile * p.splits;
  return c;
}

// Writes one 32-row x 32-column output box (this warp's rows) through a
// swizzled staging buffer and a TMA store.  `v` holds this thread's row.
template <class Cfg>
SVD_DEV void store_box(const CUtensorMap* tm_out, uint8_t* stg_warp, int& stg_buf, const float (&v)[32], int x,
                       int y, int M, int N, int* err) {
  const uint32_t lane = lane_id();
  uint8_t* stg = stg_warp + stg_buf * Cfg::STG_BYTES;
  if constexpr (Cfg::OUT == OUT_F16) {
    // Saturated fp16 intermediates are reported, never silent.  Rows and
    // columns outside the output hold zeros (zero-filled operands), so the
    // whole box can be checked.
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 32; ++j) bad |= f16_out_of_range(v[j]);
    if (__any_sync(0xffffffffu, bad) && lane == 0) flag_range(err);
  }
  // The TMA store issued two boxes ago used this buffer; make sure it has
  // finished reading it (at most one group, the other buffer's, may remain).
  if (lane == 0) bulk_wait_group_read<1>();
  __syncwarp();
  if constexpr (Cfg::IS_F32) {
    // 128-byte rows, 128-byte swizzle: 16-byte chunk j lands at j ^ (row & 7).
    const uint32_t base = smem_addr(stg) + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t phys = static_cast<uint32_t>(j) ^ (lane & 7u);
      st_shared_v4(base + phys * 16, __float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                   __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
    }
  } else {
    // 64-byte rows, 64-byte swizzle: 16-byte chunk j lands at j ^ ((row >> 1) & 3).
    const uint32_t base = smem_addr(stg) + lane * 64;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t phys = static_cast<uint32_t>(j) ^ ((lane >> 1) & 3u);
      if constexpr (Cfg::OUT == OUT_F16)
        st_shared_v4(base + phys * 16, pack_f16x2_sat(v[8 * j], v[8 * j + 1]), pack_f16x2_sat(v[8 * j + 2], v[8 * j + 3]),
                     pack_f16x2_sat(v[8 * j + 4], v[8 * j + 5]), pack_f16x2_sat(v[8 * j + 6], v[8 * j + 7]));
      else
        st_shared_v4(base + phys * 16, pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                     pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    // Boxes that lie wholly outside the output (rows >= M or columns >= N)
    // are skipped; partly outside boxes are clipped by the TMA unit.
    if (y < M && x < N) tma_store_2d(tm_out, stg, x, y);
    bulk_commit_group();
  }
  stg_buf ^= 1;
}

// Configurations whose epilogue can run the fused exchange (fp16 rows of a
// plain GEMM: the tensor-parallel partial of T = H . u_down).  Its blocks are
// pairs of consecutive 32-column chunks of one warp: four epilogue warps (each
// walks every chunk of its rows in order) and tiles of whole 64-column pairs.
template <class Cfg>
constexpr bool kPushable = Cfg::OUT == OUT_F16 && Cfg::EPI == EPI_PLAIN && Cfg::NB == 1 && Cfg::EPI_WARPS == 4 &&
                           Cfg::BN % 64 == 0;

// Output boxes of the fused exchange, in pairs: box `half` (0 or 1) of a
// 32 x 64 block (lane = row y0 + lane, columns col..col+31 of the box) goes,
// as fp16 with saturation and zeros at or past column N, into half `half` of
// the warp's two staging buffers; after the second box the block is read back
// row-wise and stored into every rank's slot, so that each store instruction
// writes four whole 128-byte row segments (16-byte stores from 32 different
// rows cost NVLink far more per byte).  All lanes call it together.
template <class Cfg>
SVD_DEV void push_box(const GemmParams& p, uint8_t* stg, long long parity_off, const float (&v)[32], int col, int y0,
                      int half) {
  const uint32_t lane = lane_id();
  bool bad = false;
  uint32_t h[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float lo = col + 2 * j < p.N ? v[2 * j] : 0.0f;
    const float hi = col + 2 * j + 1 < p.N ? v[2 * j + 1] : 0.0f;
    bad |= f16_out_of_range(lo) || f16_out_of_range(hi);
    h[j] = pack_f16x2_sat(lo, hi);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) flag_range(p.err);
  // 64-byte rows per box, 16-byte chunk j of row r at j ^ ((r >> 1) & 3)
  const uint32_t base = smem_addr(stg);
  if (half == 0) __syncwarp();  // the previous block's reads of both buffers are done
  const uint32_t box = base + static_cast<uint32_t>(half) * Cfg::STG_BYTES;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    st_shared_v4(box + lane * 64 + ((static_cast<uint32_t>(j) ^ ((lane >> 1) & 3u)) * 16), h[4 * j], h[4 * j + 1],
                 h[4 * j + 2], h[4 * j + 3]);
  if (half == 0) return;
  __syncwarp();
  const int c16 = static_cast<int>(lane & 7u);  // 16-byte chunk of the 128-byte row segment
  const uint32_t src = base + static_cast<uint32_t>(c16 >> 2) * Cfg::STG_BYTES;
  const int col0 = col - 32 + 8 * c16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + static_cast<int>(lane >> 3);
    const uint4 val = ld_shared_v4(src + r * 64 + ((static_cast<uint32_t>(c16 & 3) ^ ((static_cast<uint32_t>(r) >> 1) & 3u)) * 16));
    const int row = y0 + r;
    if (row < p.M && col0 < p.push.ld) {
      const long long off = parity_off + (static_cast<long long>(row) * p.push.ld + col0) * 2;
#pragma unroll 1
      for (int q = 0; q < p.push.n; ++q) *reinterpret_cast<uint4*>(p.push.dst[q] + off) = val;
    }
  }
}

SVD_DEV float silu_mul(float g, float u) {
  // g * sigmoid(g) * u; for g << 0 the denominator overflows to +inf and the
  // quotient is the correct limit 0.
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// Fused RMSNorm row scale rsqrt(sum_j stats[row, j] / dim + eps).  The sum
// runs in j order (every kernel computes the same value from the same
// statistics), with sixteen loads in flight at a time.
SVD_DEV float norm_row_scale(const float* stats, long long ld, int parts, int dim, float eps, int row) {
  const float* s = stats + static_cast<long long>(row) * ld;
  float sum = 0.0f;
  for (int j0 = 0; j0 < parts; j0 += 16) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = j0 + j < parts ? s[j0 + j] : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) sum += v[j];  // + 0.0f past the end leaves the sum as it is
  }
  return rsqrtf(sum / static_cast<float>(dim) + eps);
}

// Applies the epilogue to one 32-column chunk of this thread's row.
template <class Cfg>
SVD_DEV void epilogue_math(const GemmParams& p, float (&v)[32], const float (&u)[32], int row, int col) {
  if constexpr (Cfg::EPI == EPI_SWIGLU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu_mul(v[j], u[j]);
  } else if constexpr (Cfg::EPI == EPI_RESID) {
    if (row < p.M) {
      const __nv_bfloat16* r = p.residual + static_cast<long long>(row) * p.ld_residual + col;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (col + 8 * q + 8 <= p.N) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(r + 8 * q));
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            v[8 * q + 2 * e] += f.x;
            v[8 * q + 2 * e + 1] += f.y;
          }
        }
      }
    }
  }
}

// acc += t0 then acc += t1, element by element (the split order).
SVD_DEV void add_partials(float (&acc)[32], const float4 (&t0)[8], const float4 (&t1)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    acc[4 * j] += t0[j].x;
    acc[4 * j + 1] += t0[j].y;
    acc[4 * j + 2] += t0[j].z;
    acc[4 * j + 3] += t0[j].w;
    acc[4 * j] += t1[j].x;
    acc[4 * j + 1] += t1[j].y;
    acc[4 * j + 2] += t1[j].z;
    acc[4 * j + 3] += t1[j].w;
  }
}

// Weight (B) tiles of the CTA-pair GEMMs are loaded with an L2 evict-first
// policy (1) or the default policy (0).
#ifndef SVDMLP_B_EVICT_FIRST
#define SVDMLP_B_EVICT_FIRST 1
#endif

template <class Cfg>
SVD_DEV void issue_stage_loads(const CUtensorMap* tm_a, const CUtensorMap* tm_a2, const CUtensorMap* tm_b,
                               const CUtensorMap* tm_b2, uint8_t* smem, int s, uint64_t* full_local,
                               uint32_t full_leader, int kx, int a_row, int b_row, bool do_a = true,
                               bool do_b = true) {
  uint8_t* a = smem + Cfg::OFF_A + s * Cfg::A_BYTES;
  uint8_t* a2 = smem + Cfg::OFF_A2 + s * Cfg::A_BYTES;
  uint8_t* b = smem + Cfg::OFF_B + s * Cfg::B_BYTES;
  uint8_t* b2 = smem + Cfg::OFF_B2 + s * Cfg::B_BYTES;
  const int kb = kx / Cfg::BK, grp = b_row / 16;
  if constexpr (Cfg::CTAS == 1) {
    if (do_a) {
      tma_load_2d(tm_a, full_local, a, kx, a_row);
      if constexpr (Cfg::NA == 2) tma_load_2d(tm_a2, full_local, a2, kx, a_row);
    }
    if (!do_b) return;
    if constexpr (Cfg::B_TILED) {
      tma_load_4d(tm_b, full_local, b, kb, grp);
      if constexpr (Cfg::NB == 2) tma_load_4d(tm_b2, full_local, b2, kb, grp);
    } else {
      tma_load_2d(tm_b, full_local, b, kx, b_row);
      if constexpr (Cfg::NB == 2) tma_load_2d(tm_b2, full_local, b2, kx, b_row);
    }
  } else {
    if (do_a) {
      tma_load_2d_pair(tm_a, full_leader, a, kx, a_row);
      if constexpr (Cfg::NA == 2) tma_load_2d_pair(tm_a2, full_leader, a2, kx, a_row);
    }
    if (!do_b) return;
    if constexpr (Cfg::B_TILED) {
#if SVDMLP_B_EVICT_FIRST
      const uint64_t pol = l2_policy_evict_first();
      tma_load_4d_pair_hint(tm_b, full_leader, b, kb, grp, pol);
      if constexpr (Cfg::NB == 2) tma_load_4d_pair_hint(tm_b2, full_leader, b2, kb, grp, pol);
#else
      tma_load_4d_pair(tm_b, full_leader, b, kb, grp);
      if constexpr (Cfg::NB == 2) tma_load_4d_pair(tm_b2, full_leader, b2, kb, grp);
#endif
    } else {
      tma_load_2d_pair(tm_b, full_leader, b, kx, b_row);
      if constexpr (Cfg::NB == 2) tma_load_2d_pair(tm_b2, full_leader, b2, kx, b_row);
    }
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_a2,
                      const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b2,
                      const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_out2,
                      const GemmParams p) {
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool PAIR = Cfg::CTAS == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* epi_abort = reinterpret_cast<volatile int*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int unit_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], Cfg::EPI_WARPS * Cfg::CTAS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *fix_flag = 0;
    *epi_abort = 0;
    fence_mbarrier_init();
  }
  if (warp == Cfg::PRODUCER_WARP && lane == 0) {
    prefetch_tensormap(&tm_a);
    if (Cfg::NA == 2) prefetch_tensormap(&tm_a2);
    prefetch_tensormap(&tm_b);
    if (Cfg::NB == 2) prefetch_tensormap(&tm_b2);
    prefetch_tensormap(&tm_out);
    if (Cfg::EPI == EPI_DUAL_STORE) prefetch_tensormap(&tm_out2);
  }
  if (warp == Cfg::MMA_WARP) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.err, p.timeout_ns};
  unsigned push_epoch = 0;  // the fused exchange's call counter, read by the epilogue

  if (warp == Cfg::PRODUCER_WARP) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const bool chained = p.dep != nullptr || p.pub != nullptr;
      // Inputs of an unchained launch (and of a chain's first stage) come from
      // the previous launch as a whole.  The first stage waits for it before
      // it lets the chain's later stages launch: those trust the counters,
      // which the previous chain's last stage clears just before it completes.
      if (p.dep == nullptr) grid_dependency_wait();
      if (chained) grid_launch_dependents();  // the next stage may take SMs as this one drains
      const uint32_t full_leader0 = PAIR ? mapa_shared(smem_addr(&full[0]), 0) : 0u;
      int it = 0;
      bool ok = true;
      for (int u = unit0; u < p.num_units && ok; u += unit_step) {
        const UnitCoord c = decode_unit(p, u);
        const int a_row = c.m_t * Cfg::TILE_M + static_cast<int>(rank) * Cfg::BM;
        const int b_row = c.n_t * Cfg::BN + static_cast<int>(rank) * Cfg::B_ROWS;
        int kb = c.kb0;
        if (p.dep != nullptr && ld_acquire_gpu(&p.dep[c.m_t]) < p.dep_target) {
          // Weights first (they do not depend on the previous stage): as many
          // stages as the ring frees, then the wait, then those stages' A tiles.
          int pre = 0;
          for (; pre < min(STAGES, c.kb1 - c.kb0); ++pre) {
            const int s = (it + pre) % STAGES;
            const uint32_t ph = static_cast<uint32_t>((it + pre) / STAGES) & 1u;
            if (!mbar_wait(&empty[s], ph ^ 1u, ctx, SITE_PRODUCER_EMPTY)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES * Cfg::CTAS);
            issue_stage_loads<Cfg>(&tm_a, &tm_a2, &tm_b, &tm_b2, smem, s, &full[s], full_leader0 + 8u * s,
                                   (c.kb0 + pre) * Cfg::BK, a_row, b_row, false, true);
          }
          // On a timeout the announced stages still get their A tiles, so that
          // every barrier phase completes; the error word reports the failure.
          if (ok && !wait_counter_geq(&p.dep[c.m_t], p.dep_target, ctx, SITE_DEPENDENCY)) ok = false;
          fence_proxy_async_global();
          for (int j = 0; j < pre; ++j)
            issue_stage_loads<Cfg>(&tm_a, &tm_a2, &tm_b, &tm_b2, smem, (it + j) % STAGES, &full[(it + j) % STAGES],
                                   full_leader0 + 8u * ((it + j) % STAGES), (c.kb0 + j) * Cfg::BK, a_row, b_row,
                                   true, false);
          it += pre;
          kb += pre;
          if (!ok) break;
        } else if (p.dep != nullptr) {
          fence_proxy_async_global();
        }
        for (; kb < c.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, ctx, SITE_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES * Cfg::CTAS);
          issue_stage_loads<Cfg>(&tm_a, &tm_a2, &tm_b, &tm_b2, smem, s, &full[s], full_leader0 + 8u * s,
                                 kb * Cfg::BK, a_row, b_row);
        }
      }
      if (!chained) grid_launch_dependents();
      // Drain: every stage's most recent load must have landed before the CTA
      // may exit (on the normal path these waits return at once).  In a pair
      // the loads complete on the even CTA's barrier, so the odd CTA waits for
      // the MMA that consumed them (its `empty` barrier) instead.
      for (int s = 0; s < STAGES; ++s) {
        if (it > s) {
          const int last = s + ((it - 1 - s) / STAGES) * STAGES;
          const uint32_t par = static_cast<uint32_t>(last / STAGES) & 1u;
          if (PAIR && !leader)
            mbar_wait(&empty[s], par, ctx, SITE_DRAIN_LOADS, false);
          else
            mbar_wait(&full[s], par, ctx, SITE_DRAIN_LOADS, false);
        }
      }
    }
    __syncwarp();
  } else if (warp == Cfg::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int it = 0, acc_it = 0;
      bool ok = true;
      for (int u = unit0; u < p.num_units && ok; u += unit_step) {
        const UnitCoord c = decode_unit(p, u);
        const int b = acc_it % Cfg::ACC_BUFS;
        const uint32_t aph = static_cast<uint32_t>(acc_it / Cfg::ACC_BUFS) & 1u;
        if (!mbar_wait(&acc_empty[b], aph ^ 1u, ctx, SITE_MMA_ACC_EMPTY)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(b * Cfg::ACC_STRIDE);
        for (int kb = c.kb0; kb < c.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, ctx, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + Cfg::OFF_A + s * Cfg::A_BYTES);
          const uint32_t a2_addr = Cfg::NA == 2 ? smem_addr(smem + Cfg::OFF_A2 + s * Cfg::A_BYTES) : a_addr;
          const uint32_t b_addr = smem_addr(smem + Cfg::OFF_B + s * Cfg::B_BYTES);
          const uint32_t b2_addr = smem_addr(smem + Cfg::OFF_B2 + s * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            const uint32_t acc = (kb > c.kb0 || k > 0) ? 1u : 0u;
            const uint64_t ad = make_sw128_desc(a_addr + k * 32), bd = make_sw128_desc(b_addr + k * 32);
            if constexpr (PAIR) umma_f16kind_pair(d, ad, bd, Cfg::IDESC, acc);
            else umma_f16kind(d, ad, bd, Cfg::IDESC, acc);
            if constexpr (Cfg::NB == 2) {
              const uint64_t ad2 = make_sw128_desc(a2_addr + k * 32), bd2 = make_sw128_desc(b2_addr + k * 32);
              if constexpr (PAIR) umma_f16kind_pair(d + Cfg::BSTRIDE, ad2, bd2, Cfg::IDESC, acc);
              else umma_f16kind(d + Cfg::BSTRIDE, ad2, bd2, Cfg::IDESC, acc);
            }
          }
          // frees the smem stage (of both CTAs) once these MMAs have read it
          if constexpr (PAIR) umma_commit_pair_multicast(&empty[s], 0x3);
          else umma_commit(&empty[s]);
        }
        if (!ok) break;
        // accumulator ready for the epilogue (of both CTAs)
        if constexpr (PAIR) umma_commit_pair_multicast(&acc_full[b], 0x3);
        else umma_commit(&acc_full[b]);
        ++acc_it;
      }
      // Drain: all issued MMAs must be complete before TMEM is released.
      if constexpr (PAIR) umma_commit_pair(drain);
      else umma_commit(drain);
      mbar_wait(drain, 0, ctx, SITE_DRAIN_MMA, false);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;          // TMEM lane quarter == rows [32q, 32q + 32) of this CTA's rows
    const int half = warp >> 2;      // with eight epilogue warps: which chunks this warp takes
    constexpr int CH_STEP = Cfg::EPI_WARPS / 4;
    constexpr int NCH = Cfg::BN / 32;
    uint8_t* stg_warp = smem + Cfg::OFF_STG + warp * 2 * Cfg::STG_BYTES;
    const uint32_t acc_empty_leader0 = PAIR ? mapa_shared(smem_addr(&acc_empty[0]), 0) : 0u;
    constexpr int EPI_THREADS = 32 * Cfg::EPI_WARPS;
    int stg_buf = 0;
    int acc_it = 0;
    // The fused norm's statistics come from the previous launch: wait for it
    // (as the producer does) so that each unit's row scale can be read before
    // its accumulator is ready.
    if (p.norm_stats != nullptr) grid_dependency_wait();
    // The fused exchange writes the slot set of this call's parity.  The
    // counter was moved by the previous exchange's last CTA, in an earlier
    // launch.
    long long push_off = 0;
    if constexpr (kPushable<Cfg>) {
      if (p.push.n > 0) {
        grid_dependency_wait();
        push_epoch = *reinterpret_cast<volatile unsigned*>(p.push.epoch);
        push_off = (push_epoch & 1u) ? p.push.parity_bytes : 0;
      }
    }
    for (int u = unit0; u < p.num_units; u += unit_step) {
      const UnitCoord c = decode_unit(p, u);
      const int b = acc_it % Cfg::ACC_BUFS;
      const uint32_t aph = static_cast<uint32_t>(acc_it / Cfg::ACC_BUFS) & 1u;
      const int row_base = c.m_t * Cfg::TILE_M + static_cast<int>(rank) * Cfg::BM;  // this CTA's first row
      const int row_in_tile = q * 32 + static_cast<int>(lane);
      const int grow = row_base + row_in_tile;
      float rscale = 1.0f;  // RMSNorm row scale (1 without a fused norm)
      if (p.norm_stats != nullptr && c.nsplit == 1 && grow < p.M)
        rscale = norm_row_scale(p.norm_stats, p.stats_ld, p.norm_parts, p.norm_dim, p.norm_eps, grow);
      bool ok = mbar_wait(&acc_full[b], aph, ctx, SITE_EPI_ACC_FULL);
      ok = __all_sync(0xffffffffu, ok);
      // The epilogue warps take the same decision, so that none of them is
      // left alone at a named barrier below.
      if (!ok && lane == 0) *epi_abort = 1;
      named_barrier_sync(2, EPI_THREADS);
      if (*epi_abort) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * Cfg::ACC_STRIDE);
      const int n0 = c.n_t * Cfg::BN;
      const int y_box = row_base + q * 32;

      if (c.nsplit == 1) {
        float slice_ss[Cfg::BN / 128 > 0 ? Cfg::BN / 128 : 1] = {};
#pragma unroll 1
        for (int ch = half; ch < NCH; ch += CH_STEP) {
          uint32_t rg[32];
          uint32_t ru[32];
          tmem_ld_x32(tacc + ch * 32, rg);
          if constexpr (Cfg::NB == 2) tmem_ld_x32(tacc + Cfg::BSTRIDE + ch * 32, ru);
          tmem_ld_wait();
          if (ch + CH_STEP >= NCH) {
            // This warp's TMEM reads of the buffer have all returned: release it.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (PAIR) mbar_arrive_cluster(acc_empty_leader0 + 8u * b);
              else mbar_arrive(&acc_empty[b]);
            }
          }
          float v[32], w[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __uint_as_float(rg[j]);
            w[j] = Cfg::NB == 2 ? __uint_as_float(ru[j]) : 0.0f;
          }
          epilogue_math<Cfg>(p, v, w, grow, n0 + ch * 32);
          if (p.norm_stats != nullptr) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] *= rscale;
              w[j] *= rscale;
            }
          }
          if constexpr (Cfg::EPI == EPI_RESID && Cfg::BN % 128 == 0 && CH_STEP == 1) {
            if (p.out_stats != nullptr) {
              float ss = 0.0f;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float r = __bfloat162float(__float2bfloat16(v[j]));  // the value the next block reads
                ss += r * r;
              }
              slice_ss[ch / 4] += ss;
            }
          }
          if constexpr (kPushable<Cfg>) {
            if (p.push.n > 0) push_box<Cfg>(p, stg_warp, push_off, v, n0 + ch * 32, y_box, ch & 1);
            else store_box<Cfg>(&tm_out, stg_warp, stg_buf, v, n0 + ch * 32, y_box, p.M, p.N, p.err);
          } else {
            store_box<Cfg>(&tm_out, stg_warp, stg_buf, v, n0 + ch * 32, y_box, p.M, p.N, p.err);
          }
          if constexpr (Cfg::EPI == EPI_DUAL_STORE)
            store_box<Cfg>(&tm_out2, stg_warp, stg_buf, w, n0 + ch * 32, y_box, p.M, p.N, p.err);
        }
        if constexpr (Cfg::EPI == EPI_RESID && Cfg::BN % 128 == 0 && CH_STEP == 1) {
          if (p.out_stats != nullptr && grow < p.M) {
#pragma unroll
            for (int sl = 0; sl < Cfg::BN / 128; ++sl)
              if (n0 + sl * 128 < p.N) p.out_stats[static_cast<long long>(grow) * p.stats_ld + n0 / 128 + sl] = slice_ss[sl];
          }
        }
        if (p.pub != nullptr) {
          // Publish this CTA's rows of the tile: each warp's output boxes are
          // written, then one release increment once every epilogue warp is here.
          if (lane == 0) {
            bulk_wait_group<0>();
            fence_proxy_async_global();
          }
          __syncwarp();
          named_barrier_sync(3, EPI_THREADS);
          if (threadIdx.x == 0) red_add_release_gpu(&p.pub[c.m_t], 1);
        }
      } else {
        // Split-K.  Each split writes its fp32 partial (this CTA's rows) and
        // bumps the (tile, CTA) counter.  One CTA per tile: the split that
        // arrives last sums all partials in split order and runs the
        // epilogue.  CTA pairs: a 256 x BN partial tile is too much for one
        // CTA to read, so every split waits (bounded) until all are in and
        // sums the 32-column chunks ch = ks (mod splits); a second pass over
        // the counter lets the last one to finish re-arm it.
        const int ctile = c.tile * Cfg::CTAS + static_cast<int>(rank);
        const size_t tile_elems = static_cast<size_t>(Cfg::NB) * (Cfg::BM * Cfg::BN);
        float* slot = p.partials + static_cast<size_t>((c.pslot + c.ks) * Cfg::CTAS + rank) * tile_elems;
        const bool row_ok = grow < p.M;
#pragma unroll 1
        for (int ch = half; ch < NCH; ch += CH_STEP) {
#pragma unroll
          for (int br = 0; br < Cfg::NB; ++br) {
            uint32_t r[32];
            tmem_ld_x32(tacc + br * Cfg::BSTRIDE + ch * 32, r);
            tmem_ld_wait();
            if (row_ok) {
              // [chunk][float4 j][128 rows]: a warp's 32 rows of one float4
              // column are 512 contiguous bytes
              float4* dst = reinterpret_cast<float4*>(slot + static_cast<size_t>(br) * (Cfg::BM * Cfg::BN) +
                                                      ch * (Cfg::BM * 32)) + row_in_tile;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                __stcg(dst + j * Cfg::BM, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                      __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {  // TMEM no longer needed for this unit
          if constexpr (PAIR) mbar_arrive_cluster(acc_empty_leader0 + 8u * b);
          else mbar_arrive(&acc_empty[b]);
        }
        __threadfence();
        named_barrier_sync(1, EPI_THREADS);
        if (threadIdx.x == 0) {
          const int old = atomicAdd(&p.counters[ctile], 1);
          int go = PAIR ? 1 : (old == c.nsplit - 1 ? 1 : 0);
          if (PAIR && !wait_counter_geq(&p.counters[ctile], c.nsplit, ctx, SITE_DEPENDENCY)) go = 0;
          *fix_flag = go;
        }
        named_barrier_sync(1, EPI_THREADS);
        if (*fix_flag) {
          __threadfence();
          const float* base = p.partials + static_cast<size_t>(c.pslot * Cfg::CTAS + rank) * tile_elems;
          const size_t split_stride = static_cast<size_t>(Cfg::CTAS) * tile_elems;
#pragma unroll 1
          for (int ch = half; ch < NCH; ch += CH_STEP) {
            // the same for every lane of the warp; the fused exchange hands
            // out whole pairs of chunks (its 128-byte row segments)
            if (PAIR && (p.push.n > 0 ? (ch >> 1) % c.nsplit : ch % c.nsplit) != c.ks) continue;
            float v[32], w[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = 0.0f;
              w[j] = 0.0f;
            }
            if (row_ok) {
#pragma unroll 1
              for (int s = 0; s < c.nsplit; s += 2) {
                // two splits' loads in flight per step; the sum order is the split order
                const bool two = s + 1 < c.nsplit;
                const float* src0 = base + static_cast<size_t>(s) * split_stride + ch * (Cfg::BM * 32);
                const float* src1 = src0 + split_stride;
#pragma unroll
                for (int br = 0; br < Cfg::NB; ++br) {
                  const float4* s0 = reinterpret_cast<const float4*>(src0 + br * (Cfg::BM * Cfg::BN)) + row_in_tile;
                  const float4* s1 = reinterpret_cast<const float4*>(src1 + br * (Cfg::BM * Cfg::BN)) + row_in_tile;
                  float4 t0[8], t1[8];
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                    t0[j] = __ldcg(s0 + j * Cfg::BM);
                    t1[j] = two ? __ldcg(s1 + j * Cfg::BM) : make_float4(0.f, 0.f, 0.f, 0.f);
                  }
                  if (br == 0) add_partials(v, t0, t1);
                  else add_partials(w, t0, t1);
                }
              }
            }
            epilogue_math<Cfg>(p, v, w, grow, n0 + ch * 32);
            if constexpr (kPushable<Cfg>) {
              if (p.push.n > 0) push_box<Cfg>(p, stg_warp, push_off, v, n0 + ch * 32, y_box, ch & 1);
              else store_box<Cfg>(&tm_out, stg_warp, stg_buf, v, n0 + ch * 32, y_box, p.M, p.N, p.err);
            } else {
              store_box<Cfg>(&tm_out, stg_warp, stg_buf, v, n0 + ch * 32, y_box, p.M, p.N, p.err);
            }
            if constexpr (Cfg::EPI == EPI_DUAL_STORE)
              store_box<Cfg>(&tm_out2, stg_warp, stg_buf, w, n0 + ch * 32, y_box, p.M, p.N, p.err);
          }
        }
        named_barrier_sync(1, EPI_THREADS);
        if (threadIdx.x == 0) {
          if constexpr (!PAIR) {
            if (*fix_flag) p.counters[ctile] = 0;
          } else {
            const int old = atomicAdd(&p.counters[ctile], 1);
            if (old == 2 * c.nsplit - 1) p.counters[ctile] = 0;
          }
        }
      }
      ++acc_it;
    }
    if (lane == 0) bulk_wait_group<0>();  // all output boxes written before exit
    __syncwarp();
    // This thread's stores into the peers' slots are ordered before the
    // publish below (system scope: the peers read them).
    if constexpr (kPushable<Cfg>) {
      if (p.push.n > 0) __threadfence_system();
    }
  }

  __syncthreads();
  if constexpr (kPushable<Cfg>) {
    if (p.push.n > 0 && threadIdx.x == 0) {
      // thread 0 is an epilogue thread: push_epoch is this launch's count
      const unsigned done = atom_add_acq_rel_gpu(p.push.exit_count, 1u);
      if (done == gridDim.x - 1) {
        // every CTA's rows are out: publish the new count to every peer
        fence_acq_rel_sys();
        for (int q = 0; q < p.push.n; ++q)
          if (q != p.push.rank) st_release_sys(p.push.flag[q], push_epoch + 1u);
        *p.push.exit_count = 0;
        *p.push.epoch = push_epoch + 1u;
        __threadfence();
      }
    }
  }
  if (p.exit_count != nullptr && threadIdx.x == 0) {
    // Last stage of a chain: the last CTA to leave clears the chain's
    // counters (every wait on them has returned by now) for the next launch.
    __threadfence();
    const int e = atomicAdd(p.exit_count, 1);
    if (e == static_cast<int>(gridDim.x) - 1) {
      for (int st = 0; st < 3; ++st)
        for (int m = 0; m < p.m_tiles; ++m) atomicExch(&p.reset[st * kChainStride + m], 0);
      atomicExch(p.exit_count, 0);
      __threadfence();
    }
  }
  if constexpr (PAIR) cluster_sync();  // the peer's MMAs and arrivals are done
  if (warp == Cfg::MMA_WARP) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace svdmlp
