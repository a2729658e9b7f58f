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
// feature, column = token.  Each epilogue thread owns one output feature and
// writes out[t][f] for t < M (consecutive features across a warp, so the
// stores coalesce).
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
  static constexpr int OFF_BAR = OFF_X + STAGES * NB * X_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
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

// Stores tokens [t0, t0 + 16) of feature f (bounds-checked against M and N).
template <class Cfg>
SVD_DEV void dec_store_chunk(const GemmParams& p, void* out, long long ld_out, int f, int t0, const float (&v)[16]) {
  if (f >= p.N) return;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int t = t0 + j;
    if (t < p.M) {
      float x = v[j];
      if constexpr (Cfg::EPI == EPI_RESID) x += __bfloat162float(p.residual[static_cast<long long>(t) * p.ld_residual + f]);
      const long long off = static_cast<long long>(t) * ld_out + f;
      if constexpr (Cfg::OUT == OUT_F32) static_cast<float*>(out)[off] = x;
      else if constexpr (Cfg::OUT == OUT_F16)
        static_cast<__half*>(out)[off] = __float2half_rn(fminf(fmaxf(x, -65504.f), 65504.f));
      else static_cast<__nv_bfloat16*>(out)[off] = __float2bfloat16(x);
    }
  }
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
      // weights: packed tile-major layout, 4-D loads at (k-block, 16-row group)
      auto w_loads = [&](int s, int kx, int row) {
        tma_load_4d(&tm_w, &full[s], smem + Cfg::OFF_W + (s * Cfg::NB) * Cfg::W_BYTES, kx / Cfg::BK, row / 16);
        if constexpr (Cfg::NB == 2)
          tma_load_4d(&tm_w2, &full[s], smem + Cfg::OFF_W + (s * Cfg::NB + 1) * Cfg::W_BYTES, kx / Cfg::BK, row / 16);
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
      const int f = c.n_t * Cfg::BM + row;
      const int tv = min(p.M, TOK);                      // valid tokens
      constexpr int NCH = TOK / 16;
      // Partial slot of this split: [tile][split][branch][128 features][TOK tokens] fp32.
      const size_t tile_slot = static_cast<size_t>(c.n_t) * p.splits;
      float* slot = p.partials + ((tile_slot + c.ks) * Cfg::NB) * (Cfg::BM * TOK) + static_cast<size_t>(row) * TOK;
#pragma unroll
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
        if (16 * ch >= tv) continue;
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
          dec_store_chunk<Cfg>(p, out, ld_out, f, 16 * ch, v);
        } else {
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            __stcg(reinterpret_cast<float4*>(slot + 16 * ch) + j4,
                   make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]));
            if constexpr (Cfg::NB == 2)
              __stcg(reinterpret_cast<float4*>(slot + Cfg::BM * TOK + 16 * ch) + j4,
                     make_float4(w[4 * j4], w[4 * j4 + 1], w[4 * j4 + 2], w[4 * j4 + 3]));
          }
        }
      }
      if (p.splits > 1) {
        __threadfence();
        named_barrier_sync(1, 128);
        if (threadIdx.x == 0) {
          const int old = atomicAdd(&p.counters[c.n_t], 1);
          *fix_flag = (old == p.splits - 1) ? 1 : 0;
        }
        named_barrier_sync(1, 128);
        if (*fix_flag) {
          __threadfence();
          const float* base = p.partials + (tile_slot * Cfg::NB) * (Cfg::BM * TOK) + static_cast<size_t>(row) * TOK;
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            if (16 * ch >= tv) continue;
            float v[16], w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              v[j] = 0.f;
              w[j] = 0.f;
            }
            // Up to 4 splits' loads in flight per step; the sum is in split order.
#pragma unroll 1
            for (int s0 = 0; s0 < p.splits; s0 += 4) {
              float4 g4[4][4], u4[4][4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const bool have = s0 + j < p.splits;
                const float* src = base + static_cast<size_t>((s0 + j) * Cfg::NB) * (Cfg::BM * TOK) + 16 * ch;
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                  g4[j][j4] = have ? __ldcg(reinterpret_cast<const float4*>(src) + j4) : make_float4(0.f, 0.f, 0.f, 0.f);
                  if constexpr (Cfg::NB == 2)
                    u4[j][j4] = have ? __ldcg(reinterpret_cast<const float4*>(src + Cfg::BM * TOK) + j4)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                  v[4 * j4] += g4[j][j4].x;
                  v[4 * j4 + 1] += g4[j][j4].y;
                  v[4 * j4 + 2] += g4[j][j4].z;
                  v[4 * j4 + 3] += g4[j][j4].w;
                  if constexpr (Cfg::NB == 2) {
                    w[4 * j4] += u4[j][j4].x;
                    w[4 * j4 + 1] += u4[j][j4].y;
                    w[4 * j4 + 2] += u4[j][j4].z;
                    w[4 * j4 + 3] += u4[j][j4].w;
                  }
                }
              }
            }
            if constexpr (Cfg::EPI == EPI_SWIGLU) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = silu_mul(v[j], w[j]);
            }
            dec_store_chunk<Cfg>(p, out, ld_out, f, 16 * ch, v);
          }
          named_barrier_sync(1, 128);
          if (threadIdx.x == 0) p.counters[c.n_t] = 0;
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
