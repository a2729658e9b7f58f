// Decode-size (M <= 128 tokens) tcgen05 kernel for sm_100a: HBM streaming of
// the weight (factor) matrices with the operands swapped.  TOK (the MMA N) is
// 16, 64 or 128 tokens.
//
//   C[M, N] = epilogue( X[M, K] . W[N, K]^T )
//
// The weight tile is the MMA's A operand (128 rows of N, the MMA M) and the
// tokens are the MMA's N (TOK = 16..128, zero-filled beyond M by the TMA
// unit), so the tensor core does little wasted work and the activation tile
// is small.  The accumulator in TMEM is transposed: TMEM lane = output
// feature, column = token.  The epilogue moves each 16-token chunk through
// shared memory (one thread per feature writes a column of an fp32
// [16][128] tile) and then writes whole output rows: a warp stores the 128
// features of one token (256 bytes of fp16/bf16) with 8-byte vectors, so
// every store fills whole 128-byte lines.  Per-token scattered 2-byte stores
// (one half-line per warp and token) cost ~50 ns each under a full weight
// stream; full-line stores do not.
//
// Dual form (NB == 2): C = silu(X.Wg^T) * (X2.Wu^T), the decode gate/up stage.
//
// Weight bytes dominate; the kernel is built to keep HBM busy:
//  - split-K spreads each 128-row weight panel over several CTAs, so that
//    every SM streams; the split that arrives last sums the fp32 partials of
//    its feature (all splits' loads issued together, summed in split order:
//    deterministic) and runs the epilogue;
//  - the producer fetches the first stages' weight tiles before waiting on
//    the previous kernel (griddepcontrol.wait): weights never depend on it,
//    and with <= 256 TMEM columns and ~100 KB of shared memory a CTA of this
//    kernel can share an SM with the previous kernel's last CTAs, so the
//    weight stream of the next stage starts during the tail of the last.
//
// Roles: warps 0-3 epilogue, warp 4 TMA producer, warp 5 TMEM allocator and
// single-thread MMA issuer.  All waits are bounded (see ptx.cuh).
#pragma once

#include "gemm_sm100.cuh"

namespace svdmlp {

template <int TOK_, int NB_, int STAGES_, int EPI_, bool IN_F16_, int OUT_, int ACC_BUFS_ = 2>
struct DecCfg {
  static constexpr int BM = 128, BK = 64;  // weight rows per tile, K per stage
  static constexpr int TOK = TOK_, NB = NB_, STAGES = STAGES_, EPI = EPI_, OUT = OUT_, ACC_BUFS = ACC_BUFS_;
  static constexpr bool IN_F16 = IN_F16_;
  static_assert(TOK == 16 || TOK == 32 || TOK == 64 || TOK == 128, "tokens per tile: 16, 32, 64 or 128");
  static_assert(NB == 1 || EPI == EPI_SWIGLU, "dual decode GEMMs use the SwiGLU epilogue");
  static constexpr int W_BYTES = BM * BK * 2;
  static constexpr int X_BYTES = TOK * BK * 2;
  static_assert(X_BYTES % 1024 == 0, "activation tiles stay 1024-byte aligned");
  static constexpr int W_STAGE_BYTES = NB * W_BYTES;
  static constexpr int STAGE_BYTES = NB * (W_BYTES + X_BYTES);
  static constexpr int ACC_STRIDE = NB * TOK;  // TMEM columns per accumulator buffer
  static constexpr int ACC_COLS = ACC_BUFS * ACC_STRIDE;
  static constexpr uint32_t TMEM_COLS =
      ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128 : ACC_COLS <= 256 ? 256 : 512;
  static_assert(ACC_COLS <= 512, "accumulators must fit in 512 TMEM columns");
  // Two CTAs per SM (the next kernel's CTA beside the last CTAs of the
  // previous one) need <= 256 TMEM columns and <= ~113 KB of shared memory each.
  static constexpr bool TWO_PER_SM = TMEM_COLS <= 256;
  static constexpr uint32_t IDESC = make_idesc_16bit(BM, TOK, IN_F16);
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = OFF_W + STAGES * NB * W_BYTES;
  static constexpr int STG_BYTES = 16 * BM * 4;  // fp32 [16 tokens][128 features] output staging
  static constexpr int OFF_STG = OFF_X + STAGES * NB * X_BYTES;
  static constexpr int OFF_BAR = OFF_STG + STG_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_RSTD = OFF_MISC + 64;  // fused RMSNorm: the row scale of each token
  static constexpr int SMEM_BYTES = OFF_RSTD + TOK * 4 + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
  static_assert(!TWO_PER_SM || SMEM_BYTES <= 113 * 1024, "two CTAs per SM need <= 113 KB of shared memory each");
};

struct DecUnit {
  int n_t, ks, kb0, kb1;
};

SVD_DEV DecUnit decode_dec_unit(const GemmParams& p, int u) {
  DecUnit c;
  c.ks = u % p.splits;
  c.n_t = u / p.splits;
  c.kb0 = c.ks * p.kb_per_split;
  c.kb1 = min(c.kb0 + p.kb_per_split, p.k_blocks);
  return c;
}

// Writes four consecutive features [f, f + 4) of token t: epilogue residual,
// conversion and a vector store when all four are inside N (scalar tail
// otherwise).  Rows and the output base are 16-byte aligned.
// Returns the sum of squares of the bf16 values it stored (0 for other
// output types), for the fused RMSNorm statistics of the next block.
template <class Cfg>
SVD_DEV float dec_store4(const GemmParams& p, void* out, long long ld_out, int t, int f, float4 v) {
  if (t >= p.M || f >= p.N) return 0.0f;
  float x[4] = {v.x, v.y, v.z, v.w};
  const bool full = f + 4 <= p.N;
  if constexpr (Cfg::EPI == EPI_RESID) {
    const __nv_bfloat16* r = p.residual + static_cast<long long>(t) * p.ld_residual + f;
    if (full) {
      const uint2 w = *reinterpret_cast<const uint2*>(r);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
      x[0] += a.x;
      x[1] += a.y;
      x[2] += b.x;
      x[3] += b.y;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (f + j < p.N) x[j] += __bfloat162float(r[j]);
    }
  }
  const long long off = static_cast<long long>(t) * ld_out + f;
  if constexpr (Cfg::OUT == OUT_F32) {
    float* o = static_cast<float*>(out) + off;
    if (full) *reinterpret_cast<float4*>(o) = make_float4(x[0], x[1], x[2], x[3]);
    else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (f + j < p.N) o[j] = x[j];
    }
  } else if constexpr (Cfg::OUT == OUT_F16) {
    __half* o = static_cast<__half*>(out) + off;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) bad |= (full || f + j < p.N) && f16_out_of_range(x[j]);
    if (bad) flag_range(p.err);  // saturated fp16 intermediates are reported, never silent
    if (full) *reinterpret_cast<uint2*>(o) = make_uint2(pack_f16x2_sat(x[0], x[1]), pack_f16x2_sat(x[2], x[3]));
    else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (f + j < p.N) o[j] = __float2half_rn(fminf(fmaxf(x[j], -65504.f), 65504.f));
    }
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + off;
    if (full) *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (f + j < p.N) o[j] = __float2bfloat16(x[j]);
    }
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float r = f + j < p.N ? __bfloat162float(__float2bfloat16(x[j])) : 0.0f;
      ss += r * r;
    }
    return ss;
  }
  return 0.0f;
}

SVD_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <class Cfg>
__global__ void __launch_bounds__(192)
    gemv_sm100_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_x2,
                      const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                      void* out, long long ld_out, const GemmParams p) {
  constexpr int STAGES = Cfg::STAGES;
  constexpr int TOK = Cfg::TOK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + Cfg::ACC_BUFS;
  uint64_t* drain = acc_empty + Cfg::ACC_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* epi_abort = reinterpret_cast<volatile int*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();

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
    *abort_flag = 0;
    *fix_flag = 0;
    *epi_abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&tm_x);
    if (Cfg::NB == 2) prefetch_tensormap(&tm_x2);
    prefetch_tensormap(&tm_w);
    if (Cfg::NB == 2) prefetch_tensormap(&tm_w2);
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
      // weights: packed tile-major layout, 4-D loads at (k-block, 16-row group),
      // read once per call, so evicted from L2 before activations and partials
      const uint64_t wpol = l2_policy_weight_stream();
      auto w_loads = [&](int s, int kx, int row) {
        tma_load_4d_hint(&tm_w, &full[s], smem + Cfg::OFF_W + (s * Cfg::NB) * Cfg::W_BYTES, kx / Cfg::BK, row / 16,
                         wpol);
        if constexpr (Cfg::NB == 2)
          tma_load_4d_hint(&tm_w2, &full[s], smem + Cfg::OFF_W + (s * Cfg::NB + 1) * Cfg::W_BYTES, kx / Cfg::BK,
                           row / 16, wpol);
      };
      auto x_loads = [&](int s, int kx) {
        tma_load_2d(&tm_x, &full[s], smem + Cfg::OFF_X + (s * Cfg::NB) * Cfg::X_BYTES, kx, 0);
        if constexpr (Cfg::NB == 2)
          tma_load_2d(&tm_x2, &full[s], smem + Cfg::OFF_X + (s * Cfg::NB + 1) * Cfg::X_BYTES, kx, 0);
      };
      // Weights do not depend on the previous kernel: fetch the first stages'
      // weight tiles before waiting for it, then their activations.
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < p.num_units) {
        const DecUnit c = decode_dec_unit(p, blockIdx.x);
        pre = min(STAGES, c.kb1 - c.kb0);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], Cfg::STAGE_BYTES);
          w_loads(i, (c.kb0 + i) * Cfg::BK, c.n_t * Cfg::BM);
        }
      }
      grid_dependency_wait();
      if (pre > 0) {
        const DecUnit c = decode_dec_unit(p, blockIdx.x);
        for (int i = 0; i < pre; ++i) x_loads(i, (c.kb0 + i) * Cfg::BK);
      }
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        const DecUnit c = decode_dec_unit(p, u);
        for (int kb = c.kb0; kb < c.kb1; ++kb, ++it) {
          if (it < pre) continue;  // issued above
          const int s = it % STAGES;
          const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, ctx, SITE_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          w_loads(s, kb * Cfg::BK, c.n_t * Cfg::BM);
          x_loads(s, kb * Cfg::BK);
        }
      }
      grid_launch_dependents();
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
    if (lane == 0) {
      int it = 0, acc_it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        const DecUnit c = decode_dec_unit(p, u);
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
#pragma unroll
          for (int br = 0; br < Cfg::NB; ++br) {
            const uint32_t w_addr = smem_addr(smem + Cfg::OFF_W + (s * Cfg::NB + br) * Cfg::W_BYTES);
            const uint32_t x_addr = smem_addr(smem + Cfg::OFF_X + (s * Cfg::NB + br) * Cfg::X_BYTES);
#pragma unroll
            for (int k = 0; k < Cfg::BK / 16; ++k) {
              const uint32_t acc = (kb > c.kb0 || k > 0) ? 1u : 0u;
              umma_f16kind(d + br * TOK, make_sw128_desc(w_addr + k * 32), make_sw128_desc(x_addr + k * 32),
                           Cfg::IDESC, acc);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
        ++acc_it;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, ctx, SITE_DRAIN_MMA, false);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp;
    int acc_it = 0;
    float* rstd = reinterpret_cast<float*>(smem + Cfg::OFF_RSTD);
    if (p.norm_stats != nullptr) {
      // fused RMSNorm: the row scale of each token, from the previous
      // block's per-slice sums of squares (written by the previous kernel)
      grid_dependency_wait();
      for (int t = threadIdx.x; t < min(p.M, TOK); t += 128)
        rstd[t] = norm_row_scale(p.norm_stats, p.stats_ld, p.norm_parts, p.norm_dim, p.norm_eps, t);
      named_barrier_sync(1, 128);
    }
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
      const DecUnit c = decode_dec_unit(p, u);
      const int b = acc_it % Cfg::ACC_BUFS;
      const uint32_t aph = static_cast<uint32_t>(acc_it / Cfg::ACC_BUFS) & 1u;
      bool ok = mbar_wait(&acc_full[b], aph, ctx, SITE_EPI_ACC_FULL);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) *epi_abort = 1;
      named_barrier_sync(2, 128);
      if (*epi_abort) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * Cfg::ACC_STRIDE);
      const int row = q * 32 + static_cast<int>(lane);   // feature within the 128-row panel
      const int tv = min(p.M, TOK);                      // valid tokens
      constexpr int NCH = TOK / 16;
      // Partial slot of this split: [tile][split][branch][TOK tokens][128 features] fp32,
      // token-major so that a warp's 32 features of one token are one 128-byte line.
      const size_t tile_slot = static_cast<size_t>(c.n_t) * p.splits;
      float* slot = p.partials + ((tile_slot + c.ks) * Cfg::NB) * (Cfg::BM * TOK) + row;
      float* stg = reinterpret_cast<float*>(smem + Cfg::OFF_STG);
      const int f0 = c.n_t * Cfg::BM;
#pragma unroll 1
      for (int ch = 0; ch < NCH; ++ch) {
        uint32_t rg[16], ru[16];
        tmem_ld_x16(tacc + ch * 16, rg);
        if constexpr (Cfg::NB == 2) tmem_ld_x16(tacc + TOK + ch * 16, ru);
        tmem_ld_wait();
        if (ch == NCH - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);  // every TMEM read has returned
        }
        if (16 * ch >= tv) continue;  // the same for all four warps
        float v[16], w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __uint_as_float(rg[j]);
          w[j] = Cfg::NB == 2 ? __uint_as_float(ru[j]) : 0.f;
        }
        if (p.splits == 1) {
          if constexpr (Cfg::EPI == EPI_SWIGLU) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = silu_mul(v[j], w[j]);
          }
          if (p.norm_stats != nullptr) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] *= rstd[min(16 * ch + j, TOK - 1)];
          }
          // column `row` of the fp32 [16 tokens][128 features] staging tile
#pragma unroll
          for (int j = 0; j < 16; ++j) stg[j * Cfg::BM + row] = v[j];
          named_barrier_sync(3, 128);
          // whole rows: thread -> (token row, feature quad), a warp per row
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int idx = static_cast<int>(threadIdx.x) + 128 * i;
            const int rr = idx >> 5, c4 = idx & 31;
            const float4 x = *reinterpret_cast<const float4*>(stg + rr * Cfg::BM + 4 * c4);
            const float ss = warp_sum(dec_store4<Cfg>(p, out, ld_out, 16 * ch + rr, f0 + 4 * c4, x));
            // one warp holds one token's 128 features: its slice sum of squares
            if (p.out_stats != nullptr && lane == 0 && 16 * ch + rr < p.M)
              p.out_stats[static_cast<long long>(16 * ch + rr) * p.stats_ld + c.n_t] = ss;
          }
          named_barrier_sync(3, 128);  // read before the next chunk overwrites it
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (16 * ch + j < tv) {
              __stcg(slot + (16 * ch + j) * Cfg::BM, v[j]);
              if constexpr (Cfg::NB == 2) __stcg(slot + Cfg::BM * TOK + (16 * ch + j) * Cfg::BM, w[j]);
            }
          }
        }
      }
      if (p.splits > 1) {
        // Fix-up.  Up to 16 tokens: the split that arrives last sums every
        // split's partial (tiny).  Beyond that the reads of S fp32 partial
        // tiles are too much for one CTA, so every split of the tile waits
        // (bounded) until all S partials are in and sums the token rows
        // r = ks (mod S); a second pass over the same counter lets the last
        // one to finish reset it.
        const bool spread = tv > 16;
        __threadfence();
        named_barrier_sync(1, 128);
        if (threadIdx.x == 0) {
          const int old = atomicAdd(&p.counters[c.n_t], 1);
          int go = spread ? 1 : (old == p.splits - 1 ? 1 : 0);
          if (spread && !wait_counter_geq(&p.counters[c.n_t], p.splits, ctx, SITE_DEPENDENCY)) go = 0;
          *fix_flag = go;
        }
        named_barrier_sync(1, 128);
        if (*fix_flag) {
          __threadfence();
          // Row-vector mapping (thread -> token row, feature quad): the
          // token-major partials are read as whole 512-byte rows, up to four
          // splits' loads in flight, summed in split order.
          const float* base = p.partials + (tile_slot * Cfg::NB) * (Cfg::BM * TOK);
          constexpr int VI = Cfg::NB == 2 ? 2 : 4;  // row vectors per thread and pass
          const int r0 = spread ? c.ks : 0, rstep = spread ? p.splits : 1;
          const int rows = (tv - r0 + rstep - 1) / rstep;  // token rows this CTA sums
#pragma unroll 1
          for (int lr0 = 0; lr0 < rows; lr0 += 4 * VI) {
            float4 g[VI], uacc[VI];
            int tt[VI], ff[VI];
#pragma unroll
            for (int i = 0; i < VI; ++i) {
              const int idx = static_cast<int>(threadIdx.x) + 128 * i;
              const int lr = lr0 + (idx >> 5);
              tt[i] = lr < rows ? r0 + lr * rstep : TOK;  // TOK: no row
              ff[i] = 4 * (idx & 31);
              g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
              uacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll 1
            for (int s0 = 0; s0 < p.splits; s0 += 4) {
              float4 lg[4][VI], lu[4][VI];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int i = 0; i < VI; ++i) {
                  const bool ld = s0 + j < p.splits && tt[i] < tv;
                  const float* src = base + static_cast<size_t>((s0 + j) * Cfg::NB) * (Cfg::BM * TOK) +
                                     (ld ? tt[i] : 0) * Cfg::BM + ff[i];
                  lg[j][i] = ld ? __ldcg(reinterpret_cast<const float4*>(src)) : make_float4(0.f, 0.f, 0.f, 0.f);
                  if constexpr (Cfg::NB == 2)
                    lu[j][i] = ld ? __ldcg(reinterpret_cast<const float4*>(src + Cfg::BM * TOK))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                }
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int i = 0; i < VI; ++i) {
                  g[i].x += lg[j][i].x;
                  g[i].y += lg[j][i].y;
                  g[i].z += lg[j][i].z;
                  g[i].w += lg[j][i].w;
                  if constexpr (Cfg::NB == 2) {
                    uacc[i].x += lu[j][i].x;
                    uacc[i].y += lu[j][i].y;
                    uacc[i].z += lu[j][i].z;
                    uacc[i].w += lu[j][i].w;
                  }
                }
              }
            }
#pragma unroll
            for (int i = 0; i < VI; ++i) {
              if constexpr (Cfg::EPI == EPI_SWIGLU) {
                g[i].x = silu_mul(g[i].x, uacc[i].x);
                g[i].y = silu_mul(g[i].y, uacc[i].y);
                g[i].z = silu_mul(g[i].z, uacc[i].z);
                g[i].w = silu_mul(g[i].w, uacc[i].w);
              }
              if (p.norm_stats != nullptr && tt[i] < tv) {
                const float sc = rstd[tt[i]];
                g[i].x *= sc;
                g[i].y *= sc;
                g[i].z *= sc;
                g[i].w *= sc;
              }
              // a warp's lanes hold one token row (tt is the same across the warp)
              const float ss = warp_sum(tt[i] < tv ? dec_store4<Cfg>(p, out, ld_out, tt[i], f0 + ff[i], g[i]) : 0.0f);
              if (p.out_stats != nullptr && lane == 0 && tt[i] < tv)
                p.out_stats[static_cast<long long>(tt[i]) * p.stats_ld + c.n_t] = ss;
            }
          }
        }
        named_barrier_sync(1, 128);
        if (threadIdx.x == 0) {
          if (!spread) {
            if (*fix_flag) p.counters[c.n_t] = 0;
          } else {
            // second pass: the last split to finish its rows re-arms the counter
            const int old = atomicAdd(&p.counters[c.n_t], 1);
            if (old == 2 * p.splits - 1) p.counters[c.n_t] = 0;
          }
        }
      }
      ++acc_it;
    }
  }

  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace svdmlp
