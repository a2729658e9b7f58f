// Thin inline-PTX wrappers for the sm_100a features the SVD-MLP kernels use:
// mbarriers (with bounded waits), TMA tensor loads/stores, tcgen05 MMA with
// TMEM accumulators, TMEM loads, programmatic dependent launch.
//
// Every wait in this library is bounded: a wait that runs past its limit
// records an error code in global memory, raises a CTA-wide abort flag and
// returns false so that the caller can drain its in-flight copies, free TMEM
// and leave the kernel.  Nothing here traps.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#define SVD_DEV __device__ __forceinline__

namespace svdmlp {

SVD_DEV uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SVD_DEV uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

SVD_DEV uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ----------------------------------------------------------------- mbarrier
SVD_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

SVD_DEV void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

SVD_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

SVD_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

SVD_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Context for bounded waits.  `abort_flag` lives in shared memory and is seen
// by every role of the CTA; `err` is the device-wide error word that the host
// reads back with svdmlp_check_device_status().
struct WaitCtx {
  volatile int* abort_flag;
  int* err;
  uint64_t limit_ns;
};

// Waits until the phase with `parity` of `bar` completes.  Returns false if
// the CTA was aborted or the wait exceeded ctx.limit_ns (then `site` is
// recorded in the error word).  When `honour_abort` is false the wait ignores
// the abort flag (used while draining copies that are still in flight).
SVD_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx, int site,
                       bool honour_abort = true) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 31u) == 0u) {
      if (honour_abort && *ctx.abort_flag) return false;
      if (global_timer_ns() - t0 > ctx.limit_ns) {
        *ctx.abort_flag = 1;
        atomicCAS(ctx.err, 0, site);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------- TMA
SVD_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

SVD_DEV void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// 4-D tile load: the packed weight layout [16-row group][k-block][16][64]
// (see tiled_weight_map in svdmlp.cu); coordinates (0, 0, k-block, group).
SVD_DEV void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(0), "r"(c2), "r"(c3)
      : "memory");
}

// tma_load_4d with an L2 cache policy (see l2_policy_evict_first).
SVD_DEV void tma_load_4d_hint(const CUtensorMap* map, uint64_t* bar, void* dst, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(0), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// L2 prefetch of the same 4-D tile (no shared memory, no barrier): pulls the
// tile's lines into L2 so that a later tma_load_4d of it hits there.
SVD_DEV void tma_prefetch_4d(const CUtensorMap* map, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(0), "r"(c2), "r"(c3)
               : "memory");
}

SVD_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
}

SVD_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
SVD_DEV void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
SVD_DEV void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

SVD_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// --------------------------------------------------------------- tcgen05/TMEM
SVD_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}

SVD_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

SVD_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

SVD_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SVD_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored as rows of
// 128 bytes (64 bf16) with the 128-byte swizzle that TMA writes.  Eight-row
// core-matrix groups are 1024 bytes apart (stride byte offset); the leading
// byte offset is unused for swizzled K-major layouts.  Bits: start address
// [0,14), LBO [16,30), SBO [32,46), descriptor version 1 at [46,48), layout
// type 2 (128B swizzle) at [61,64).
SVD_DEV uint64_t make_sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: A and B both bf16 (or
// both fp16), fp32 accumulator, both operands K-major, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc_16bit(int M, int N, bool f16) {
  return (1u << 4)                                    // D format: f32
         | ((f16 ? 0u : 1u) << 7)                     // A format: f16 = 0, bf16 = 1
         | ((f16 ? 0u : 1u) << 10)                    // B format: f16 = 0, bf16 = 1
         | (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);     // M / 16
}

SVD_DEV void umma_f16kind(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation issued so far by this
// thread has completed.
SVD_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread i of the warp receives
// row (lane_base + i), columns [col, col + 32).
SVD_DEV void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

SVD_DEV void tmem_ld_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

SVD_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------ programmatic dependent launch
SVD_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SVD_DEV void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ 2-SM (CTA pair)
SVD_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at the same offset in CTA `rank`.
SVD_DEV uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

SVD_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (shared::cluster address).
SVD_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA load into this CTA's shared memory whose completion is signalled on an
// mbarrier of either CTA of the pair (`bar_cluster` is a shared::cluster address).
SVD_DEV void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

SVD_DEV void tma_load_4d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(0), "r"(c2), "r"(c3)
      : "memory");
}

// The same load with an L2 cache policy (createpolicy): used for weight tiles,
// which every CTA pair reads once, so that they leave L2 before the
// activations and split-K partials that are read again.
SVD_DEV void tma_load_4d_pair_hint(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int c2, int c3,
                                   uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(0), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

SVD_DEV uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// The policy of the decode kernels' weight stream: evict-first (1) or the
// normal policy (0).
#ifndef SVDMLP_W_EVICT_FIRST
#define SVDMLP_W_EVICT_FIRST 1
#endif
SVD_DEV uint64_t l2_policy_weight_stream() {
#if SVDMLP_W_EVICT_FIRST
  return l2_policy_evict_first();
#else
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
#endif
}

SVD_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
SVD_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
SVD_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// MMA over the CTA pair: A rows split across the two CTAs (M = 256), B rows
// split across them (N/2 each); issued by the even CTA only.
SVD_DEV void umma_f16kind_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at the same offset in every CTA of `cta_mask`
// when all prior tcgen05 operations of this thread have completed.
SVD_DEV void umma_commit_pair_multicast(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_addr(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrives on `bar` of the issuing CTA when this thread's tcgen05 ops complete.
SVD_DEV void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// ------------------------------------------------ cross-CTA dependency counters
SVD_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Atomic add with acquire-release semantics at GPU scope; returns the old
// value.  Release is cumulative: writes that happen before it in this CTA
// (ordered by a barrier) are published with it.
SVD_DEV int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Fire-and-forget add with release semantics at GPU scope.
SVD_DEV void red_add_release_gpu(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's earlier generic-proxy view of global memory before its
// later async-proxy (TMA) accesses.
SVD_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Waits until *ctr >= target (bounded like mbar_wait; the counter is written
// by other running CTAs of the same grid).
SVD_DEV bool wait_counter_geq(const int* ctr, int target, const WaitCtx& ctx, int site) {
  if (ld_acquire_gpu(ctr) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_gpu(ctr) >= target) return true;
    __nanosleep(32);
    if ((i & 15u) == 0u) {
      if (*ctx.abort_flag) return false;
      if (global_timer_ns() - t0 > ctx.limit_ns) {
        *ctx.abort_flag = 1;
        atomicCAS(ctx.err, 0, site);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------- misc
SVD_DEV void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

SVD_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

SVD_DEV uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

SVD_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// fp16 pair with saturation to the largest finite fp16 (65504) instead of inf.
SVD_DEV uint32_t pack_f16x2_sat(float lo, float hi) {
  lo = fminf(fmaxf(lo, -65504.0f), 65504.0f);
  hi = fminf(fmaxf(hi, -65504.0f), 65504.0f);
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// True when v cannot be stored as a finite fp16 without saturating: |v| above
// the largest finite fp16, or NaN (the comparison is false for NaN).
SVD_DEV bool f16_out_of_range(float v) { return !(fabsf(v) <= 65504.0f); }

// Word 1 of the device error block: set to 1 when an fp16 intermediate (or
// an fp16-packed weight) had to be saturated.  Word 0 holds the wait-timeout
// site.  The host reads both back (svdmlp_check_device_status).
constexpr int kRangeWord = 1;
SVD_DEV void flag_range(int* err) { atomicOr(err + kRangeWord, 1); }

// System-scope ordering for flags that other GPUs read (peer memory).
SVD_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

SVD_DEV unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

SVD_DEV void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Atomic add with acquire-release semantics at GPU scope; returns the old value.
SVD_DEV unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

}  // namespace svdmlp
