// Collectives of the tensor-parallel layer over NVLink peer memory.
//
// One process per GPU.  Every rank allocates one buffer that its peers map
// (CUDA IPC); the buffers have the same layout on every rank: a signal area at
// offset 0, then the matrices the collectives move, at offsets the caller
// chooses.  A kernel gets every rank's buffer as mapped in this process
// (`base[i]`, this rank's own at `base[rank]`) and moves rows with plain
// 16-byte loads and stores over NVLink: no TMA, no multicast.
//
// Rows are owned in blocks: rank q owns rows [q R, min(M, (q + 1) R)),
// R = ceil(M / world).
//
// Synchronisation: each CTA keeps an epoch (a call counter in its own
// signal area).  A barrier is: every CTA b writes epoch + 1 into slot
// [b][rank] of each peer's flag array (release, system scope) and waits until
// each peer has written the same value into slot [b][peer] of its own array
// (read relaxed, then an acquire fence).  Every rank launches the same
// kernels with the same grids, so the epochs agree.  A barrier that waits
// longer than the limit
// records the site in the signal area's error word and the CTA returns
// without moving its epoch: the group then stays in error (every later
// barrier times out) until it is rebuilt.
#pragma once

#include "ptx.cuh"

namespace svdmlp {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerMaxCtas = 256;
constexpr int kPeerThreads = 512;

// Sites recorded in the signal area's error word.
enum PeerSite : int { SITE_PEER_START = 21, SITE_PEER_MID = 22, SITE_PEER_END = 23, SITE_PEER_SUM = 24 };

// Words of the signal area's ctl block used by the fused exchange (the
// H.u_down GEMM or peer_push_slots_kernel fills the slots, then
// peer_sum_slots_kernel sums them): this rank's call counter, the exit
// counter of the launch that fills the slots, and from word kPushFlagWord on
// the count each rank has published into this rank's area.
constexpr int kPushEpochWord = 8, kPushExitWord = 9, kPushFlagWord = 16;
static_assert(kPushFlagWord + kPeerMaxRanks <= 64, "ctl words");

struct PeerSignal {
  int ctl[64];                                    // word 0: timeout site; word 1: fp16 range flag
  unsigned epoch[kPeerMaxCtas];                   // per CTA: barrier calls completed
  unsigned flag[3][kPeerMaxCtas][kPeerMaxRanks];  // start / mid / end barriers
};
constexpr long long kPeerSignalBytes = 32 * 1024;
static_assert(sizeof(PeerSignal) <= kPeerSignalBytes, "signal area");

struct PeerArgs {
  unsigned char* base[kPeerMaxRanks];  // each rank's buffer as mapped in this process
  int world, rank;
  unsigned long long limit_ns;
};

// The barrier of kind `kind` (0 start, 1 mid, 2 end) for this CTA.  All
// threads call it; returns false (in every thread) when a wait timed out.
SVD_DEV bool peer_barrier(const PeerArgs& a, int kind, unsigned epoch) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < static_cast<unsigned>(a.world)) {
    const int p = static_cast<int>(threadIdx.x);
    PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[a.rank]);
    PeerSignal* peer = reinterpret_cast<PeerSignal*>(a.base[p]);
    // This CTA's earlier stores (ordered before this point by the barrier
    // above) become visible to the peer before the flag does.
    fence_acq_rel_sys();
    st_release_sys(&peer->flag[kind][blockIdx.x][a.rank], epoch);
    // Spin on plain (relaxed) reads; one fence after the flag is seen makes
    // the peer's stores visible to this CTA (acquire).
    const unsigned* mine = &me->flag[kind][blockIdx.x][p];
    if (ld_relaxed_sys(mine) != epoch) {
      const unsigned long long t0 = global_timer_ns();
      for (unsigned i = 1;; ++i) {
        if (ld_relaxed_sys(mine) == epoch) break;
        if ((i & 63u) == 0u && global_timer_ns() - t0 > a.limit_ns) {
          atomicCAS(&me->ctl[0], 0, SITE_PEER_START + kind);
          ok = false;
          break;
        }
      }
    }
    fence_acq_rel_sys();
  }
  return __syncthreads_and(ok) != 0;
}

SVD_DEV unsigned peer_epoch_next(const PeerArgs& a) {
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) s_epoch = reinterpret_cast<PeerSignal*>(a.base[a.rank])->epoch[blockIdx.x] + 1u;
  __syncthreads();
  return s_epoch;
}

SVD_DEV void peer_epoch_commit(const PeerArgs& a, unsigned epoch) {
  if (threadIdx.x == 0) reinterpret_cast<PeerSignal*>(a.base[a.rank])->epoch[blockIdx.x] = epoch;
}

// Work split.  Every phase walks one owner's block of rows as a flat list of
// 16-byte vectors, element i going to CTA (i / blockDim) mod gridDim, the same
// way on every rank and in every phase.  So the per-CTA barriers are enough:
// when CTA b has passed a barrier, CTA b of every rank has finished the
// elements it handles in the phase before, and those are the only elements
// CTA b handles in the phase after.
constexpr int kPeerUnroll = 4;

struct PeerBlock {
  int r0, rows;  // first row and row count of an owner's block
};

SVD_DEV PeerBlock peer_block(int m, int world, int owner) {
  const int rows_per = (m + world - 1) / world;
  const int r0 = min(m, owner * rows_per);
  return PeerBlock{r0, min(m, r0 + rows_per) - r0};
}

// fp16 slots of the reduce scatter: [2 parities][world][rows_per][c], dense.
SVD_DEV long long peer_slot_off(long long off_s, int parity, int world, int src, int rows_per, int j, int c, int v) {
  return off_s + ((static_cast<long long>((parity * world + src)) * rows_per + j) * c + v * 8) * 2;
}

// Phase A of the reduce scatter: this rank's partial rows of every other
// owner q go into slot [parity][rank] of q's scratch (stores over NVLink).
SVD_DEV void peer_push_partials(const PeerArgs& a, long long off, int m, int c, long long ld, long long off_s,
                                int parity) {
  const int rows_per = (m + a.world - 1) / a.world;
  const int vpr = c / 8;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const unsigned char* mine = a.base[a.rank];
  for (int q = 0; q < a.world; ++q) {
    if (q == a.rank) continue;
    const PeerBlock blk = peer_block(m, a.world, q);
    const long long n = static_cast<long long>(blk.rows) * vpr;
    unsigned char* dst_base = a.base[q];
    for (long long i0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i0 < n;
         i0 += kPeerUnroll * stride) {
      uint4 val[kPeerUnroll];
#pragma unroll
      for (int u = 0; u < kPeerUnroll; ++u) {
        const long long i = i0 + u * stride;
        if (i < n) {
          const int j = static_cast<int>(i / vpr), v = static_cast<int>(i % vpr);
          val[u] = *reinterpret_cast<const uint4*>(mine + off + (static_cast<long long>(blk.r0 + j) * ld + v * 8) * 2);
        }
      }
#pragma unroll
      for (int u = 0; u < kPeerUnroll; ++u) {
        const long long i = i0 + u * stride;
        if (i < n) {
          const int j = static_cast<int>(i / vpr), v = static_cast<int>(i % vpr);
          *reinterpret_cast<uint4*>(dst_base + peer_slot_off(off_s, parity, a.world, a.rank, rows_per, j, c, v)) =
              val[u];
        }
      }
    }
  }
}

// Phase B: this rank's rows summed over the ranks in rank order (its own
// partial from `off`, the others from its scratch slots), in fp32, rounded
// once to fp16.  The result goes to `out` (row j of the block at
// out + j * ld_out elements) and, when push_rows, to the same rows of every
// other rank's matrix at `off` (stores over NVLink).
SVD_DEV void peer_reduce_block(const PeerArgs& a, long long off, int m, int c, long long ld, long long off_s,
                               int parity, unsigned char* out, long long ld_out, bool push_rows, int* range_word) {
  const int rows_per = (m + a.world - 1) / a.world;
  const int vpr = c / 8;
  const PeerBlock blk = peer_block(m, a.world, a.rank);
  const long long n = static_cast<long long>(blk.rows) * vpr;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const unsigned char* mine = a.base[a.rank];
  bool bad = false;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const int j = static_cast<int>(i / vpr), v = static_cast<int>(i % vpr);
    const long long row_off = (static_cast<long long>(blk.r0 + j) * ld + v * 8) * 2;
    uint4 in[kPeerMaxRanks];
#pragma unroll
    for (int p = 0; p < kPeerMaxRanks; ++p) {
      if (p < a.world) {
        const unsigned char* src =
            p == a.rank ? mine + off + row_off : mine + peer_slot_off(off_s, parity, a.world, p, rows_per, j, c, v);
        in[p] = p == a.rank ? *reinterpret_cast<const uint4*>(src) : __ldcg(reinterpret_cast<const uint4*>(src));
      }
    }
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int p = 0; p < kPeerMaxRanks; ++p) {
      if (p < a.world) {
        const __half2* h = reinterpret_cast<const __half2*>(&in[p]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      bad |= f16_out_of_range(acc[2 * e]) || f16_out_of_range(acc[2 * e + 1]);
      ow[e] = pack_f16x2_sat(acc[2 * e], acc[2 * e + 1]);
    }
    *reinterpret_cast<uint4*>(out + (static_cast<long long>(j) * ld_out + v * 8) * 2) = o;
    if (push_rows) {
#pragma unroll
      for (int p = 0; p < kPeerMaxRanks; ++p)
        if (p < a.world && p != a.rank) *reinterpret_cast<uint4*>(a.base[p] + off + row_off) = o;
    }
  }
  // one flag per CTA (a saturated matrix would otherwise send an atomic per thread)
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(range_word, 1);
}

// ------------------------------------------------------------ fused exchange
// Slots of the fused exchange: [2 parities][world][slot_rows][ld] fp16 at
// off_s of every rank's buffer; slot [parity][q] holds rank q's partial in its
// first m rows.  The slot size is fixed by the buffer, not by the call, so
// calls of different sizes never overlap the other parity's slots.
SVD_DEV long long push_slot_off(long long off_s, int parity, int world, int src, int slot_rows, long long ld) {
  return off_s + (static_cast<long long>(parity * world + src) * slot_rows) * ld * 2;
}

// The last CTA of a launch that filled this rank's slots publishes the new
// count to every peer and moves this rank's counter (thread 0 calls it after
// a __syncthreads that follows every thread's system-scope fence).
SVD_DEV void push_publish(const PeerArgs& a, unsigned epoch) {
  PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[a.rank]);
  unsigned* exit_word = reinterpret_cast<unsigned*>(&me->ctl[kPushExitWord]);
  if (atom_add_acq_rel_gpu(exit_word, 1u) == gridDim.x - 1) {
    fence_acq_rel_sys();
    for (int q = 0; q < a.world; ++q) {
      if (q == a.rank) continue;
      PeerSignal* peer = reinterpret_cast<PeerSignal*>(a.base[q]);
      st_release_sys(reinterpret_cast<unsigned*>(&peer->ctl[kPushFlagWord + a.rank]), epoch + 1u);
    }
    *exit_word = 0;
    me->ctl[kPushEpochWord] = static_cast<int>(epoch + 1u);
    __threadfence();
  }
}

// The fused exchange for a partial that is already in local memory (decode
// sizes, whose GEMMs are not the CTA-pair kernel): this rank's fp16 partial
// [m, c_valid] (row stride ld_src) goes into its slot of every rank's buffer,
// the own included; columns from c_valid up to ld are stored as zeros.
__global__ void __launch_bounds__(kPeerThreads) peer_push_slots_kernel(PeerArgs a, const unsigned char* src,
                                                                       long long ld_src, long long off_s, int m,
                                                                       int slot_rows, int c_valid, long long ld) {
  PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[a.rank]);
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(&me->ctl[kPushEpochWord]);
  const int parity = static_cast<int>(epoch & 1u);
  const long long vpr = ld / 8;
  const long long n = static_cast<long long>(m) * vpr;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long slot = push_slot_off(off_s, parity, a.world, a.rank, slot_rows, ld);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const long long j = i / vpr;
    const int v = static_cast<int>(i % vpr);
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (v * 8 + 8 <= c_valid) {
      val = *reinterpret_cast<const uint4*>(src + (j * ld_src + v * 8) * 2);
    } else if (v * 8 < c_valid) {
      // the ragged last vector: the columns past c_valid become zeros
      const unsigned short* h = reinterpret_cast<const unsigned short*>(src) + j * ld_src + v * 8;
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t lo = v * 8 + 2 * k < c_valid ? h[2 * k] : 0u;
        const uint32_t hi = v * 8 + 2 * k + 1 < c_valid ? h[2 * k + 1] : 0u;
        w[k] = lo | (hi << 16);
      }
      val = make_uint4(w[0], w[1], w[2], w[3]);
    }
#pragma unroll
    for (int q = 0; q < kPeerMaxRanks; ++q)
      if (q < a.world) *reinterpret_cast<uint4*>(a.base[q] + slot + (j * ld + v * 8) * 2) = val;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) push_publish(a, epoch);
}

// The other half of the fused exchange: once every peer has published this
// call's count, this rank sums the ranks' slots in rank order in fp32 and
// rounds once to fp16 (the same arithmetic as the all-reduce above, so every
// rank gets the same bits) into `out` [m, c] (row stride ld_out).  A peer that
// does not publish within the limit leaves `out` unwritten and the timeout
// site in the error word.
__global__ void __launch_bounds__(kPeerThreads) peer_sum_slots_kernel(PeerArgs a, long long off_s, int m,
                                                                      int slot_rows, int c, long long ld,
                                                                      unsigned char* out, long long ld_out) {
  PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[a.rank]);
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned*>(&me->ctl[kPushEpochWord]);
  __syncthreads();
  const unsigned epoch = s_epoch;  // moved by this call's fill, in the launch before
  const int parity = static_cast<int>((epoch - 1u) & 1u);
  bool ok = true;
  if (threadIdx.x < static_cast<unsigned>(a.world) && static_cast<int>(threadIdx.x) != a.rank) {
    const unsigned* f = reinterpret_cast<const unsigned*>(&me->ctl[kPushFlagWord + threadIdx.x]);
    if (static_cast<int>(ld_relaxed_sys(f) - epoch) < 0) {
      const unsigned long long t0 = global_timer_ns();
      for (unsigned i = 1;; ++i) {
        if (static_cast<int>(ld_relaxed_sys(f) - epoch) >= 0) break;
        if ((i & 63u) == 0u && global_timer_ns() - t0 > a.limit_ns) {
          atomicCAS(&me->ctl[0], 0, SITE_PEER_SUM);
          ok = false;
          break;
        }
      }
    }
    fence_acq_rel_sys();
  }
  if (!__syncthreads_and(ok)) return;
  const int vpr = c / 8;
  const long long n = static_cast<long long>(m) * vpr;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const unsigned char* mine = a.base[a.rank];
  bool bad = false;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const long long j = i / vpr;
    const int v = static_cast<int>(i % vpr);
    uint4 in[kPeerMaxRanks];
#pragma unroll
    for (int q = 0; q < kPeerMaxRanks; ++q)
      if (q < a.world)
        in[q] = __ldcg(reinterpret_cast<const uint4*>(mine + push_slot_off(off_s, parity, a.world, q, slot_rows, ld) +
                                                     (j * ld + v * 8) * 2));
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int q = 0; q < kPeerMaxRanks; ++q) {
      if (q < a.world) {
        const __half2* h = reinterpret_cast<const __half2*>(&in[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      bad |= f16_out_of_range(acc[2 * e]) || f16_out_of_range(acc[2 * e + 1]);
      ow[e] = pack_f16x2_sat(acc[2 * e], acc[2 * e + 1]);
    }
    *reinterpret_cast<uint4*>(out + (j * ld_out + v * 8) * 2) = o;
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(&me->ctl[kRangeWord], 1);
}

// In-place all-reduce (sum) of an fp16 [m, c] matrix at `off` (row stride ld
// elements).  Every rank pushes its partial rows of each owner to that owner;
// each owner sums its rows and pushes the result to every rank.
__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_f16_kernel(PeerArgs a, long long off, int m, int c,
                                                                          long long ld, long long off_s) {
  const unsigned epoch = peer_epoch_next(a);
  PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[a.rank]);
  const int parity = static_cast<int>(epoch & 1u);
  peer_push_partials(a, off, m, c, ld, off_s, parity);
  if (!peer_barrier(a, 0, epoch)) return;  // every rank's partials of my rows are here
  const PeerBlock blk = peer_block(m, a.world, a.rank);
  peer_reduce_block(a, off, m, c, ld, off_s, parity, a.base[a.rank] + off + static_cast<long long>(blk.r0) * ld * 2,
                    ld, true, &me->ctl[kRangeWord]);
  if (!peer_barrier(a, 2, epoch)) return;  // every owner's sums are here
  peer_epoch_commit(a, epoch);
}

// Reduce-scatter of an fp16 [m, c] matrix: this rank's rows, summed over the
// ranks, into `out` (a local matrix, row stride ld_out).  The scratch slots
// alternate between two parities from call to call, so a rank that is one
// call ahead writes the other set; one barrier per call.
__global__ void __launch_bounds__(kPeerThreads) peer_reduce_scatter_f16_kernel(PeerArgs a, long long off, int m,
                                                                               int c, long long ld, long long off_s,
                                                                               unsigned char* out,
                                                                               long long ld_out) {
  const unsigned epoch = peer_epoch_next(a);
  PeerSignal* me = reinterpret_cast<PeerSignal*>(a.base[a.rank]);
  const int parity = static_cast<int>(epoch & 1u);
  peer_push_partials(a, off, m, c, ld, off_s, parity);
  if (!peer_barrier(a, 0, epoch)) return;
  peer_reduce_block(a, off, m, c, ld, off_s, parity, out, ld_out, false, &me->ctl[kRangeWord]);
  peer_epoch_commit(a, epoch);
}

// All-gather of row blocks: every rank wrote its own rows at `off`; it pushes
// them into every other rank's matrix.  The first barrier makes sure no rank
// still reads the rows about to be overwritten (it has reached this call);
// the second that every rank's rows have arrived.
__global__ void __launch_bounds__(kPeerThreads) peer_allgather_kernel(PeerArgs a, long long off, int m,
                                                                      long long row_bytes, long long ld_bytes) {
  const unsigned epoch = peer_epoch_next(a);
  if (!peer_barrier(a, 0, epoch)) return;
  const PeerBlock blk = peer_block(m, a.world, a.rank);
  const long long vpr = row_bytes / 16;
  const long long n = blk.rows * vpr;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const unsigned char* mine = a.base[a.rank];
  for (long long i0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i0 < n;
       i0 += kPeerUnroll * stride) {
    uint4 val[kPeerUnroll];
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const long long i = i0 + u * stride;
      if (i < n) val[u] = *reinterpret_cast<const uint4*>(mine + off + (blk.r0 + i / vpr) * ld_bytes + (i % vpr) * 16);
    }
#pragma unroll
    for (int p = 0; p < kPeerMaxRanks; ++p) {
      if (p < a.world && p != a.rank) {
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) {
          const long long i = i0 + u * stride;
          if (i < n) *reinterpret_cast<uint4*>(a.base[p] + off + (blk.r0 + i / vpr) * ld_bytes + (i % vpr) * 16) = val[u];
        }
      }
    }
  }
  if (!peer_barrier(a, 2, epoch)) return;
  peer_epoch_commit(a, epoch);
}

}  // namespace svdmlp
