/*
 * svdmlp.h -- C ABI of the B200 (sm_100a) SVD-compressed LLaMA MLP library.
 *
 * The library computes one SwiGLU MLP layer whose gate, up and down weights are
 * low-rank factor pairs:
 *
 *     H   = SiLU((X . u_gate) . v_gate) * ((X . u_up) . v_up)      "gate/up"
 *     out = (H . u_down) . v_down                                 "XUV down"
 *
 * with bf16 inputs and outputs, fp32 accumulation, and the three intermediates
 * (X.u, H and H.u_down) rounded once each to fp16 (see svdmlp_layout).
 * Factor names follow the reference Python (kernels/reference.py:54-93):
 * u_* is the first factor [in, r], v_* the second factor [r, out].
 *
 * Conventions
 *  - Every entry point returns an int status: 0 = SVDMLP_OK, negative = error.
 *  - All device buffers are owned by the caller; no entry point allocates
 *    device memory except svdmlp_peer_alloc (the buffer peers map, freed with
 *    svdmlp_peer_free), and none synchronises the stream except the status
 *    reads (svdmlp_check_device_status, svdmlp_pack_status,
 *    svdmlp_xuv_noalloc_status, svdmlp_peer_check_status) and
 *    svdmlp_peer_alloc.
 *  - Matrices are row-major bf16 (uint16 storage) with an explicit leading
 *    dimension in elements; `void*` pointers are device pointers.
 *  - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL is the
 *    legacy default stream).
 *  - Weights are packed once (svdmlp_pack) into K-major, TMA-legal layouts;
 *    the reference rebuilds/pads its weights outside timing in the same way
 *    (test_speedup.py:809-812, _pad at test_speedup.py:52).
 */
#ifndef SVDMLP_H_
#define SVDMLP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define SVDMLP_OK 0
#define SVDMLP_ERR_INVALID_VALUE (-1)   /* non-positive size, NULL pointer        */
#define SVDMLP_ERR_SHAPE_MISMATCH (-2)  /* contraction dims / gate-up shapes      */
#define SVDMLP_ERR_ALIGNMENT (-3)       /* pointer or leading dim not 16-byte legal */
#define SVDMLP_ERR_DTYPE (-4)           /* unsupported element type                */
#define SVDMLP_ERR_WORKSPACE (-5)       /* workspace too small                     */
#define SVDMLP_ERR_DEVICE_TIMEOUT (-6)  /* a bounded device-side wait expired      */
#define SVDMLP_ERR_CUDA (-7)            /* CUDA runtime/driver error               */
#define SVDMLP_ERR_BUDGET (-8)          /* SMEM/TMEM budget exceeds the device     */
#define SVDMLP_ERR_DEVICE (-9)          /* device is not sm_100 (B200 class)       */
#define SVDMLP_ERR_RANGE (-10)          /* an fp16 intermediate or fp16-packed weight
                                           exceeded 65504 (or was NaN) and was saturated */

/* Human-readable text for a status code. */
const char* svdmlp_status_string(int status);

/* Last CUDA error code seen by the library on this thread (0 if none). */
int svdmlp_last_cuda_error(void);

/* ------------------------------------------------------------------ layout */
#define SVDMLP_KIND_SVD 1   /* low-rank factor pairs                     */
#define SVDMLP_KIND_DENSE 2 /* dense SwiGLU weights, same kernels        */

/*
 * Packed-weight layout of one MLP layer.  Filled by svdmlp_layout_init() /
 * svdmlp_dense_layout_init(); callers treat it as read-only.
 *
 * SVD kind (ranks r_gu for gate and up, r_d for down; a rank of 0 leaves that
 * half out, so a down-only layout serves xuv_matmul and a gate/up-only layout
 * serves fused_gate_up), each a K-major matrix [N rows, K]:
 *   w1 [2*rp_gu, d]    bf16  rows [0,r_gu) = u_gate^T, rows [rp_gu, rp_gu+r_gu) = u_up^T
 *   vg [ff, r_gu]      fp16  v_gate^T
 *   vu [ff, r_gu]      fp16  v_up^T
 *   ud [r_d, ff]       fp16  u_down^T  (bf16 when r_gu == 0, see ud_f16)
 *   vd [d, r_d]        fp16  v_down^T
 * Dense kind:
 *   vg [ff, d] bf16 w_gate^T,  vu [ff, d] bf16 w_up^T,  ud [d, ff] fp16 w_down^T
 * Every matrix is stored tile-major: tiles of 16 rows x 64 columns, 2 KB
 * each, ordered [row group][column block], row-major inside a tile; N is
 * padded to 16 and K to 64 with zeros.  rp_gu is a multiple of 16; rp_d and
 * the ld_* (leading dimensions of the activations X, H and T in the
 * workspace) are multiples of 8 elements (16 bytes).
 *
 * Precision: inputs and outputs are bf16.  The intermediates X.u (rank r),
 * H (ff) and H.u_down (rank r) are kept in fp16 (saturating at +-65504), so
 * every weight that multiplies an intermediate is packed as fp16.  bf16 ->
 * fp16 is exact for magnitudes in [2^-14, 65504]; smaller weights become fp16
 * subnormals (absolute error <= 2^-25).  All accumulation is fp32.
 *
 * Range: a value that fp16 cannot hold (|v| > 65504, or NaN) is saturated to
 * +-65504 and never passes silently.  Weights are checked when packed
 * (svdmlp_pack_status); intermediates when they are stored, which sets the
 * range word of the workspace's error block (svdmlp_check_device_status
 * then reports SVDMLP_ERR_RANGE).  Activation outliers of a few hundred times
 * the typical row scale square in H = SiLU(g) * u and reach this limit.
 */
typedef struct svdmlp_layout {
  int32_t kind;
  int32_t d, ff, r_gu, r_d;
  int32_t rp_gu, rp_d, ld_d, ld_ff;
  int32_t ud_f16; /* 1: ud is stored as fp16 (full layers), 0: bf16 (down-only layouts) */
  int64_t off_w1, off_vg, off_vu, off_ud, off_vd; /* byte offsets into the packed buffer */
  int64_t off_status; /* 256-byte block holding the pack status word (see svdmlp_pack_status) */
  int64_t packed_bytes;
} svdmlp_layout;

/* SVD layer layout.  Replaces the rank/shape planning of the reference
 * launchers (test_speedup.py:169-191, _fusion_shape test_speedup.py:267-299).
 * Errors: INVALID_VALUE if d or ff <= 0, or r_gu < 0, r_d < 0, or both ranks 0. */
int svdmlp_layout_init(svdmlp_layout* layout, int d, int ff, int r_gu, int r_d);

/* Dense SwiGLU layer layout (the dense arm, kernels/reference.py:96-106). */
int svdmlp_dense_layout_init(svdmlp_layout* layout, int d, int ff);

/*
 * Packs the six factors (natural reference layouts, row-major bf16) into
 * `packed` (layout->packed_bytes bytes, 256-byte aligned).  Factors of a
 * half that the layout leaves out may be NULL.
 *   u_gate, u_up [d, r_gu]   v_gate, v_up [r_gu, ff]
 *   u_down [ff, r_d]         v_down [r_d, d]
 * Replaces the loader transposes of the reference (models/hf_svd.py:130-196)
 * and the padding in test_speedup.py:514-518, 538-543.
 */
int svdmlp_pack(const svdmlp_layout* layout, const void* u_gate, int64_t ld_u_gate, const void* v_gate,
                int64_t ld_v_gate, const void* u_up, int64_t ld_u_up, const void* v_up, int64_t ld_v_up,
                const void* u_down, int64_t ld_u_down, const void* v_down, int64_t ld_v_down, void* packed,
                void* stream);

/* Synchronises `stream`, then reports SVDMLP_ERR_RANGE if svdmlp_pack or
 * svdmlp_dense_pack saturated a weight stored as fp16 (|w| > 65504 or NaN)
 * into this packed buffer, else SVDMLP_OK.  Packing is a set-up step; the
 * Python API calls this after every pack. */
int svdmlp_pack_status(const svdmlp_layout* layout, const void* packed, void* stream);

/* svdmlp_pack for a decoder block with a fused RMSNorm: the norm's weight
 * norm_weight [d] (bf16) is folded into the first factors (row k of u_gate
 * and u_up times norm_weight[k], in fp32, rounded once), since
 * (x * rstd * w) . u = rstd * (x . diag(w) u).  The layout is svdmlp_layout_init's.
 * Use the packed layer with svdmlp_forward_block. */
int svdmlp_pack_block(const svdmlp_layout* layout, const void* norm_weight, const void* u_gate, int64_t ld_u_gate,
                      const void* v_gate, int64_t ld_v_gate, const void* u_up, int64_t ld_u_up, const void* v_up,
                      int64_t ld_v_up, const void* u_down, int64_t ld_u_down, const void* v_down, int64_t ld_v_down,
                      void* packed, void* stream);

/* Packs dense weights w_gate, w_up [d, ff] and w_down [ff, d]. */
int svdmlp_dense_pack(const svdmlp_layout* layout, const void* w_gate, int64_t ld_w_gate, const void* w_up,
                      int64_t ld_w_up, const void* w_down, int64_t ld_w_down, void* packed, void* stream);

/* --------------------------------------------------------------- workspace */
/* Bytes of workspace needed by any entry point below for up to `max_m` tokens. */
int64_t svdmlp_workspace_bytes(const svdmlp_layout* layout, int max_m);

/* Zeroes the workspace control block (error word and split-K counters).
 * Call once after allocating a workspace; the kernels keep it clean after. */
int svdmlp_workspace_init(void* workspace, int64_t workspace_bytes, void* stream);

/* Synchronises `stream`, then reports SVDMLP_ERR_DEVICE_TIMEOUT if a device
 * wait expired in an earlier launch on this workspace, SVDMLP_ERR_RANGE if an
 * fp16 intermediate was saturated (see svdmlp_layout), SVDMLP_ERR_CUDA on a
 * sticky CUDA error, else SVDMLP_OK.  A reported condition is cleared (the
 * control block re-armed), so the next call reports only later launches. */
int svdmlp_check_device_status(void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- operators */
/*
 * Fused low-rank gate/up operator: h[M, ff] = SiLU(x.u_gate.v_gate) * (x.u_up.v_up).
 * Replaces kernels/reference.py:54-72 (fused_gate_up_ref), the Pallas
 * launcher fused_mlp_up_T (test_speedup.py:522-544, which returns the
 * transpose; this returns the natural [M, ff] layout) and
 * pallas_ops.fused_gate_up (called at bench/smoke.py:81-83).
 */
int svdmlp_gate_up(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m, void* h,
                   int64_t ld_h, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * XUV down operator: y[M, d] = (h . u_down) . v_down.
 * Replaces kernels/reference.py:75-82 (fused_xuv_ref), the Pallas launcher
 * fused_three_mm_XTUV (test_speedup.py:500-519) and pallas_ops.xuv_matmul
 * (bench/latency.py:346, bench/profile_xuv.py:32-39).
 */
int svdmlp_xuv(const svdmlp_layout* layout, const void* packed, const void* h, int64_t ld_h, int m, void* y,
               int64_t ld_y, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Full SVD layer y = xuv(gate_up(x)) (two operators, four GEMM launches).
 * Replaces kernels/reference.py:85-93 (svd_mlp_ref),
 * svd_mlp_with_fused_kernel (test_speedup.py:631-655) and pallas_ops.svd_mlp
 * (bench/latency.py:402-404, models/modeling_llama.py:851-862).
 * With a non-NULL `residual` (ld_residual) the result is y = residual + mlp(x),
 * added in the last GEMM's epilogue (the decoder's residual,
 * models/modeling_llama.py:998-1002).
 */
int svdmlp_forward(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m, void* y,
                   int64_t ld_y, const void* residual, int64_t ld_residual, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * The contracted layer: the same y = xuv(gate_up(x)) (+ residual), with the
 * gate/up operator fused through . u_down as the reference's contracted path
 * does (pallas_ops.contracted_svd_mlp, models/modeling_llama.py:865-886,
 * bench/all_mlp_layers.py:491-503).  At M <= 16 tokens (the whole-layer decode
 * kernel) each SwiGLU tile of H stays in shared memory and is multiplied by
 * its slice of u_down at once, so H is never written: T = H . u_down is
 * summed from fp32 per-tile partials in a fixed order (deterministic) and
 * rounded to fp16 once.  Above 16 tokens it runs the two-operator path: a
 * prefill contraction would move r / 256 (~11 at r = 2867) times more partial
 * sums than the H it saves, and H stays in L2 between the kernels anyway.
 */
int svdmlp_forward_contracted(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m,
                              void* y, int64_t ld_y, const void* residual, int64_t ld_residual, void* workspace,
                              int64_t workspace_bytes, void* stream);

/* svdmlp_forward runs layers of M <= max_m tokens on the contracted schedule
 * above and other decode sizes on four GEMM stages.  Default 1 (measured on
 * B200: the contracted schedule is faster at one token, slower from four);
 * 0 turns it off, a negative value restores the default; at most 16. */
int svdmlp_set_decode_contract(int max_m);

/*
 * One MLP block of a decoder stack with the RMSNorm fused in:
 *   y = x + mlp(RMSNorm(x)),  RMSNorm(x) = x * rsqrt(mean(x^2) + eps) * w
 * (models/modeling_llama.py:245-262, 998-1002; bench/e2e_block.py:72-75,
 * 264-278), `packed` from svdmlp_pack_block.  No separate norm launch: the
 * first GEMM scales its output rows by rsqrt(sum(x_stats[row]) / d + eps),
 * and the last GEMM's residual epilogue writes y_stats, the same statistics of
 * y for the next block.  x_stats / y_stats: fp32 [M, ld_stats], one sum of
 * squares per 128-column slice of the row (ld_stats >= ceil(d / 128));
 * svdmlp_row_sumsq computes them for the stack's input; y_stats may be NULL.
 * x must be 16-byte aligned (it is read in place as the residual) and must
 * not alias y.
 */
int svdmlp_forward_block(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m,
                         void* y, int64_t ld_y, const float* x_stats, int64_t ld_stats, float* y_stats, float eps,
                         void* workspace, int64_t workspace_bytes, void* stream);

/* stats[row * ld_stats + s] = sum of squares of x[row, 128 s : 128 (s + 1)]
 * (bf16 x [M, n]); ld_stats >= ceil(n / 128). */
int svdmlp_row_sumsq(const void* x, int64_t ld_x, int m, int n, float* stats, int64_t ld_stats, void* stream);

/*
 * Dense SwiGLU layer y = (SiLU(x.w_gate) * (x.w_up)) . w_down from the same
 * kernels.  Replaces kernels/reference.py:96-106 (dense_mlp_ref), nki_baseline
 * (test_speedup.py:669-678) and pallas_ops.dense_mlp
 * (models/modeling_llama.py:930-937).  `residual` as in svdmlp_forward.
 */
int svdmlp_dense_forward(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m,
                         void* y, int64_t ld_y, const void* residual, int64_t ld_residual, void* workspace,
                         int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------ tensor parallel (ff) */
/*
 * First half of the down operator on an ff-shard: partial[M, r_d] (fp32) =
 * h_p . u_down_p, where h_p = [M, ff/P] and u_down_p = rows of u_down owned by
 * this rank.  The caller all-reduces `partial` (sum) across ranks, then calls
 * svdmlp_down_finish.  The reference has no multi-device path
 * (models/README.md:26-27); this is the exchange point of the ff-sharded
 * layer.
 */
int svdmlp_down_partial(const svdmlp_layout* layout, const void* packed, const void* h, int64_t ld_h, int m,
                        float* partial, int64_t ld_partial, void* workspace, int64_t workspace_bytes, void* stream);

/* Stages 1-3 of an ff-shard in one call: partial[M, r_d] (fp32) =
 * gate_up_p(x) . u_down_p, the rank-local contribution that is all-reduced. */
int svdmlp_forward_partial(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m,
                           float* partial, int64_t ld_partial, void* workspace, int64_t workspace_bytes,
                           void* stream);

/* Second half: y[M, d] = fp16(partial) . v_down (+ residual if non-NULL). */
int svdmlp_down_finish(const svdmlp_layout* layout, const void* packed, const float* partial,
                       int64_t ld_partial, int m, void* y, int64_t ld_y, const void* residual,
                       int64_t ld_residual, void* workspace, int64_t workspace_bytes, void* stream);

/* The same exchange with an fp16 partial (half the all-reduce bytes; the
 * sum is the fp16 T that the single-GPU layer also rounds to): down_u writes
 * fp16 partial[M, r_d] directly, and svdmlp_down_finish_f16 reads the summed
 * fp16 buffer as the A operand of . v_down.  partial: 16-byte aligned,
 * ld_partial a multiple of 8, else SVDMLP_ERR_ALIGNMENT.  The caller reduces
 * it with an fp16 sum (ncclHalf). */
int svdmlp_forward_partial_f16(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x,
                               int m, void* partial, int64_t ld_partial, void* workspace,
                               int64_t workspace_bytes, void* stream);
int svdmlp_down_finish_f16(const svdmlp_layout* layout, const void* packed, const void* partial,
                           int64_t ld_partial, int m, void* y, int64_t ld_y, const void* residual,
                           int64_t ld_residual, void* workspace, int64_t workspace_bytes, void* stream);

/* The all-gather split of the replicated stages (X . [u_g|u_u] sharded over
 * M, then all-gathered; for layers whose replicated stages outweigh two more
 * collectives).  Per rank of P:
 *   svdmlp_xu_project on its M/P rows -> fp16 XU rows [M/P, 2*rp_gu];
 *   all-gather XU over ranks (rows);
 *   svdmlp_partial_from_xu_f16 on all M rows (this rank's ff shard) -> fp16
 *     partial [M, r_d];
 *   reduce-scatter the partial over ranks (rows, sum);
 *   svdmlp_down_finish_f16 on its M/P rows; all-gather y over ranks.
 * xu: 16-byte aligned, ld_xu >= 2*rp_gu and a multiple of 8. */
int svdmlp_xu_project(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x, int m,
                      void* xu, int64_t ld_xu, void* workspace, int64_t workspace_bytes, void* stream);
int svdmlp_partial_from_xu_f16(const svdmlp_layout* layout, const void* packed, const void* xu, int64_t ld_xu,
                               int m, void* partial, int64_t ld_partial, void* workspace,
                               int64_t workspace_bytes, void* stream);

/*
 * XUV down operator, y[M, d] = (h . u_down) . v_down, that allocates nothing
 * and takes no workspace.  It has no counterpart in the reference.
 *
 * For callers that cannot allocate device memory: plugins hosted by a runtime
 * that owns every device allocation and passes the plugin only its input and
 * output buffers, and code that runs where cudaMalloc is not allowed.  The
 * caller passes h and y (16-byte aligned, leading dimensions multiples of 8
 * elements, else SVDMLP_ERR_ALIGNMENT); the scratch lives in a file-scope
 * device array of 8 MiB inside the library, which every GPU that loads the
 * library holds until the process exits.
 *
 * Limit: 256 + 4*ceil(M/128)*ceil(max(r_d, d)/128) (rounded up to 256) +
 * 2*M*rp_d (rounded up to 256) + [full layers, ud_f16 = 1] 2*M*ld_ff (rounded
 * up to 256) bytes must fit in 8 MiB; larger M is rejected with
 * SVDMLP_ERR_WORKSPACE before any work is enqueued.  Split-K partials use the
 * rest of the array when they fit; otherwise the GEMMs run unsplit.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current), so that first call should
 * come before any stream capture.  Every call shares the one array and clears
 * its error word and counters at the start; calls that overlap on the GPU
 * (different streams, or different host threads on one device) race on it.
 */
int svdmlp_xuv_noalloc(const svdmlp_layout* layout, const void* packed, const void* h, int64_t ld_h, int m,
                       void* y, int64_t ld_y, void* stream);

/*
 * Status of the svdmlp_xuv_noalloc calls on the current device since its last
 * call started (that call clears the array's error block first): synchronises
 * `stream`, then reports SVDMLP_ERR_DEVICE_TIMEOUT if a bounded device wait
 * expired, SVDMLP_ERR_RANGE if an fp16 intermediate was saturated, else
 * SVDMLP_OK, and clears what it reported.  Like the entry point it allocates
 * nothing; its error block is the one inside the library's static array.
 */
int svdmlp_xuv_noalloc_status(void* stream);

/* --------------------------------------------------------- building blocks */
/*
 * c[M, N] = a[M, K] . b[K, N] given b pre-transposed as bt[N, K] (K-major):
 * the dense GEMM of the reference's nki_matmul_fully_optimized_
 * (test_speedup.py:548-615) and pallas_ops.dense_matmul
 * (bench/diagnose_down.py:121), on the same tcgen05 kernel.
 */
int svdmlp_gemm(const void* a, int64_t ld_a, const void* bt, int64_t ld_bt, void* c, int64_t ld_c, int m, int n,
                int k, void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace bytes svdmlp_gemm needs for this shape (control block, split-K
 * counters and partials). */
int64_t svdmlp_gemm_workspace_bytes(int m, int n, int k);

/* dst[i][j] = src[j][i] for i < cols, j < rows; zero for i < dst_rows, j < dst_cols outside. */
int svdmlp_transpose_pack(const void* src, int64_t ld_src, int rows, int cols, void* dst, int64_t ld_dst,
                          int dst_rows, int dst_cols, void* stream);

/* RMSNorm y = x * rsqrt(mean(x^2) + eps) * w over rows of length n (bf16 in/out,
 * fp32 math); the decoder norm of models/modeling_llama.py:245-262. */
int svdmlp_rmsnorm(const void* x, int64_t ld_x, const void* w, void* y, int64_t ld_y, int m, int n, float eps,
                   void* stream);

/* --------------------------------------------------------------- diagnostics */
/*
 * Launches one CTA whose only work is a bounded wait on an mbarrier that
 * nothing completes, with a limit of `limit_ns` nanoseconds.  The wait expires,
 * records the timeout in the workspace error word and the kernel returns;
 * svdmlp_check_device_status() then reports SVDMLP_ERR_DEVICE_TIMEOUT.  Used by
 * the failure-detection tests; the device context stays usable.
 */
int svdmlp_debug_wait_timeout(void* workspace, int64_t workspace_bytes, int64_t limit_ns, void* stream);

/*
 * Tuning hooks (the analogue of the reference's block autotuner,
 * bench/tune.py:34-100).  Stage ids: 0 = X.[u_g|u_u], 1 = gate/up SwiGLU GEMM,
 * 2 = H.u_down, 3 = T.v_down, 4 = dense gate/up, 5 = dense down,
 * 6 = svdmlp_gemm.  `splits` = 0 restores the built-in split-K planner.
 * svdmlp_plan_info writes {m_tiles, n_tiles, k_blocks, splits, units, grid}.
 */
int svdmlp_set_split_override(int stage, int splits);

/* Split tail of the CTA-pair GEMMs (1, the default): when a stage's tiles
 * fill whole waves of CTA pairs plus a partial last wave, and the planner
 * leaves the stage unsplit, the last wave's tiles are split over K across the
 * pairs that wave would leave idle.  0 turns it off (every tile whole). */
int svdmlp_set_split_tail(int enable);

/* svdmlp_forward runs layers of M <= max_m tokens as one whole-layer decode
 * kernel and larger ones as four per-stage kernels (the contracted schedule,
 * svdmlp_set_decode_contract, always runs on the whole-layer kernel).  max_m = 0
 * turns the plain whole-layer schedule off, a negative value restores the
 * default (6: measured on B200 the whole-layer kernel wins up to six tokens and
 * the per-stage kernels from eight); at most 64. */
int svdmlp_set_layer_decode(int max_m);

/* L2 prefetch window of the whole-layer decode kernel's weight stream, in
 * shared-memory slots (two 16 KB weight tiles each): `ahead_slots` beyond the
 * slot being loaded while a unit streams, `wait_slots` beyond the slots
 * already loaded while a unit waits for the previous stage.  0 turns a window
 * off (the default for both); both are at most 64. */
int svdmlp_set_decode_prefetch(int ahead_slots, int wait_slots);

/* mode >= 1 (default 1) launches the whole-layer decode kernel with
 * programmatic dependent launch: its CTAs start on SMs that the previous
 * kernel on the stream has left and wait for that kernel before touching
 * anything it writes; with mode >= 2 each CTA first requests into L2 the
 * weights of mode - 1 units (measured slower: their requests compete with the
 * previous kernel's tail).  0 launches it plainly.  At most 8. */
int svdmlp_set_decode_overlap(int mode);

/* Layers (and svdmlp_gemm calls) of M >= m tokens run on the CTA-pair GEMMs,
 * smaller ones on the decode kernels.  Default 129; values below 17 act as 17;
 * a negative value restores the default; above 129 is invalid. */
int svdmlp_set_pair_min_m(int m);

/* Prefill layers (M > 128) in svdmlp_forward run their four GEMMs as a chain:
 * each stage waits per 256-row M-tile on counters the previous stage
 * publishes, instead of on the whole previous launch, and each stage's units
 * are ordered in `groups` groups of M-tiles that complete one after another,
 * so that a stage starts on its first group while its predecessor finishes
 * the last.  0 (the default) turns chaining off: each stage waits for the
 * previous launch.  Under the power cap that sustained prefill runs at on B200
 * chaining measures neutral, so it is opt-in. */
int svdmlp_set_prefill_chain(int groups);

/* Timeline of the whole-layer decode kernel (tracing; NULL turns it off).
 * Each launch writes, per CTA, 64 pairs of uint64 (tag | (unit + 1) << 8,
 * globaltimer ns): tags 1 start, 2 unit claimed, 3/4 dependency wait
 * begin/end, 5 unit epilogue done, 6 exit.  `buffer` is a device buffer of at
 * least 2 * SMs * 64 * 16 bytes, zeroed by the caller. */
int svdmlp_set_trace_buffer(void* buffer, int64_t bytes);
int svdmlp_plan_info(int stage, int m, int n, int k, int* out6);

/* Compile-time resources of the kernel a stage runs with at m tokens (the
 * B200 counterpart of the reference's tile tables and VMEM estimates,
 * test_speedup.py:169-191, 303-317): out8 = {tile rows (activation rows per
 * tile: 256 for CTA pairs, the token tile at decode sizes), tile columns
 * (output features per tile), K per pipeline stage, pipeline stages, shared
 * memory bytes per CTA, TMEM columns per CTA, threads per CTA, CTAs per tile}. */
int svdmlp_tile_info(int stage, int m, int* out8);

/*
 * Per-stage timing for profiling passes: with timing enabled every GEMM launch
 * is bracketed by CUDA events on its stream (which serialises it with its
 * neighbours); svdmlp_stage_times() waits for them and returns, per stage id,
 * the summed milliseconds and launch counts, then resets.  Off by default.
 */
int svdmlp_stage_timing(int enable);
int svdmlp_stage_times(double* ms_out, int64_t* counts_out, int n);

/* Number of kernel launches the library has enqueued since load (all entry points). */
int64_t svdmlp_launch_count(void);

/*
 * Collectives of the ff-sharded layer over NVLink peer memory, one process per
 * GPU.  The reference has no multi-device path (models/README.md:26-27); these
 * are the exchanges of the tensor-parallel layer (the all-reduce of the
 * [M, r_down] partial, and the all-gather / reduce-scatter of its split form),
 * done by the library's own kernels with plain stores between GPUs (NVLink).
 *
 * Every rank allocates one peer buffer of the same size and layout
 * (svdmlp_peer_alloc, zeroed; its first svdmlp_peer_signal_bytes() bytes are
 * the group's signal area), sends the 64-byte handle to the other ranks, and
 * maps theirs (svdmlp_peer_open; not its own).  A collective gets `bases`, the
 * `world` buffers as mapped in this process in rank order (bases[rank] = its
 * own), and a matrix at byte offset `off` of every buffer (off >= the signal
 * area, 16-byte aligned; rows of 16-byte multiples).  Row blocks: rank q owns
 * rows [q R, min(M, (q + 1) R)), R = ceil(M / world).  Every rank must make the
 * same collective calls in the same order on its own stream; each call waits
 * (bounded) for the others.  A wait that expires leaves the group in error:
 * svdmlp_peer_check_status reports SVDMLP_ERR_DEVICE_TIMEOUT from then on, and
 * the buffers must be freed and allocated again.  world <= 8.
 */
int64_t svdmlp_peer_signal_bytes(void);
int svdmlp_peer_alloc(int64_t bytes, void** ptr, void* handle);
int svdmlp_peer_open(const void* handle, void** peer_ptr);
int svdmlp_peer_close(void* peer_ptr);
int svdmlp_peer_free(void* ptr);

/* In-place sum of the fp16 [M, c] matrix (row stride ld elements; c and ld
 * multiples of 8) over the ranks: the reduced rows replace every rank's copy.
 * Every rank stores its partial rows of each owner into that owner's scratch
 * (at byte offset off_scratch, svdmlp_peer_scratch_bytes(world, m, c) bytes,
 * not overlapping the matrix); each owner sums its rows in rank order in fp32,
 * rounds once to fp16 (every rank gets the same bits) and stores them into
 * every rank's matrix.  A sum beyond fp16's range sets the range flag that
 * svdmlp_peer_check_status reports. */
int64_t svdmlp_peer_scratch_bytes(int world, int m, int c);
int svdmlp_peer_allreduce_f16(void* const* bases, int world, int rank, int64_t off, int m, int c, int64_t ld,
                              int64_t off_scratch, void* stream);

/* This rank's rows of the same sum into `out` (a local fp16 [R, c] matrix,
 * row stride ld_out). */
int svdmlp_peer_reduce_scatter_f16(void* const* bases, int world, int rank, int64_t off, int m, int c, int64_t ld,
                                   int64_t off_scratch, void* out, int64_t ld_out, void* stream);

/* Each rank has written its own rows of an [M, row_bytes] matrix (row stride
 * ld_bytes) in its buffer; stores them into every other rank's copy. */
int svdmlp_peer_allgather(void* const* bases, int world, int rank, int64_t off, int m, int64_t row_bytes,
                          int64_t ld_bytes, void* stream);

/* Reads this rank's group error block (synchronises the stream): an expired
 * wait (SVDMLP_ERR_DEVICE_TIMEOUT, sticky) or a saturated fp16 sum
 * (SVDMLP_ERR_RANGE, cleared by the read). */
int svdmlp_peer_check_status(void* own_base, void* stream);

/* The tensor-parallel all-reduce fused into the GEMM that produces it (the
 * reference has no multi-device path, models/README.md:26-27; this is the
 * exchange of the ff-sharded layer, replacing svdmlp_forward_partial_f16 +
 * svdmlp_peer_allreduce_f16).
 *
 * Slots: two sets (alternating from call to call) of one fp16
 * [slot_rows, ld_slot] slot per rank, svdmlp_peer_slots_bytes(world,
 * slot_rows, ld_slot) bytes at byte offset off_slots of every rank's buffer
 * (off_slots >= the signal area, 16-byte aligned; ld_slot a multiple of 8).
 * A call of M <= slot_rows rows uses the first M rows of each slot; keep
 * slot_rows fixed for a buffer.
 *
 * svdmlp_forward_partial_f16_peer runs stages 1-3 of this rank's ff shard
 * (as svdmlp_forward_partial_f16) and stores its fp16 partial [M, r_d] into
 * its slot of every rank's buffer: at CTA-pair sizes (M >= the pair
 * threshold) the H.u_down GEMM's epilogue stores each row over NVLink as its
 * tile finishes, so the transfer overlaps the GEMM; below it, one more kernel
 * copies the finished partial.  The last CTA then publishes this rank's call
 * count to every peer.  svdmlp_peer_sum_f16 waits (bounded) until every peer
 * has published the same count and writes the ranks' partials summed in rank
 * order in fp32, rounded once to fp16, into `out` [m, c] (row stride ld_out):
 * the same bits as svdmlp_peer_allreduce_f16, on every rank.  Every rank makes
 * both calls, in this order, on its own stream, for every layer call. */
int64_t svdmlp_peer_slots_bytes(int world, int slot_rows, int64_t ld_slot);
int svdmlp_forward_partial_f16_peer(const svdmlp_layout* layout, const void* packed, const void* x, int64_t ld_x,
                                    int M, void* const* bases, int world, int rank, int64_t off_slots, int slot_rows,
                                    int64_t ld_slot, void* workspace, int64_t workspace_bytes, void* stream);
int svdmlp_peer_sum_f16(void* const* bases, int world, int rank, int64_t off_slots, int slot_rows, int m, int c,
                        int64_t ld_slot, void* out, int64_t ld_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SVDMLP_H_ */
