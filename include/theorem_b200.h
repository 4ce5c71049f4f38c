/* theorem_b200.h -- C ABI of the B200 (sm_100a) Theorem forward hot path.
 *
 * Four ops, each replacing one `custom_kernel` of the reference
 * (yhinai/Theorem, `kernels/<op>/kernel.py`). All pointers are device
 * pointers to dense, contiguous tensors in the layouts documented per entry
 * point; sizes are element counts. Every call is asynchronous on `stream`
 * (NULL = the legacy default stream), allocates nothing, never mutates its
 * inputs, and returns a thm_status. A CUDA error of the launch itself is
 * reported as THM_ERR_CUDA; an in-kernel wait that ran out of time is
 * reported later through thm_get_device_status().
 *
 * No CPU fallback exists: without a B200-class device the entry points
 * return THM_ERR_CUDA / THM_ERR_UNSUPPORTED.
 */
#ifndef THEOREM_B200_H_
#define THEOREM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t / CUstream. */
typedef struct CUstream_st* thm_stream_t;

typedef enum {
  THM_OK = 0,
  THM_ERR_INVALID = 1,     /* bad shape / size / null pointer */
  THM_ERR_UNSUPPORTED = 2, /* valid for the reference but not built here (e.g. K=96) */
  THM_ERR_ALIGNMENT = 3,   /* pointer not 16-byte aligned */
  THM_ERR_CUDA = 4,        /* CUDA launch / runtime error */
  THM_ERR_TIMEOUT = 5,     /* an in-kernel bounded wait gave up (device status) */
  THM_ERR_NO_DRIVER = 6    /* driver entry point (tensor maps) unavailable */
} thm_status;

typedef enum { THM_F32 = 0, THM_BF16 = 1 } thm_dtype;
typedef enum { THM_LAYOUT_BDS = 0, THM_LAYOUT_BSD = 1 } thm_conv_layout;
typedef enum { THM_ACT_NONE = 0, THM_ACT_SILU = 1 } thm_activation;

/* ---------------------------------------------------------------------------
 * causal_conv1d -- replaces kernels/causal_conv1d/kernel.py:170-230
 * (custom_kernel; Triton causal_conv1d_kernel :44-117).
 *
 *   out[b,d,t] = act(bias[d] + sum_{k<W} weight[d,k] * x[b,d,t-W+1+k]),
 *   x[...,t<0] = 0.
 *
 * layout THM_LAYOUT_BDS: x, out [B, D, S] (the reference layout, fp32 only).
 * layout THM_LAYOUT_BSD: x, out [B, S, D] channel-last (fp32 or bf16), as the
 *   gated-DeltaNet chain produces them; D % 4 == 0.
 * weight [D, W] and bias [D] are fp32. 1 <= W <= 64 (BDS: W <= 8, BSD:
 * W in {2,3,4} take the unrolled fast paths).
 * l2norm_group (BSD only): 0, or G in {16,32,64,128}: after the
 *   activation every run of G consecutive channels of a time step is scaled
 *   by 1/sqrt(sum of squares + 1e-6) (the chain's q/k L2 norm over a head).
 * ------------------------------------------------------------------------- */
int thm_causal_conv1d_fwd(const void* x, const float* weight, const float* bias, void* out, int B, int D,
                          int S, int W, int layout, int dtype, int activation, int l2norm_group,
                          thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * causal_conv1d on two inputs of the same shape in one launch -- no reference
 * counterpart of its own: it is thm_causal_conv1d_fwd (THM_LAYOUT_BSD) applied
 * to (x0, weight0, bias0) -> out0 and to (x1, weight1, bias1) -> out1, with the
 * same B, D, S, W, dtype, activation and l2norm_group, and results bit-identical
 * to those two calls. The gated-DeltaNet layer runs its q and k projections'
 * convs this way: one grid of 2B sequences wastes less on its last, partly filled
 * wave than two grids of B. Where the TMA path does not apply (D * elem % 16 != 0,
 * W not in {2,3,4}) it issues the two single-conv launches.
 * ------------------------------------------------------------------------- */
int thm_causal_conv1d_pair_fwd(const void* x0, const float* weight0, const float* bias0, void* out0,
                               const void* x1, const float* weight1, const float* bias1, void* out1, int B, int D,
                               int S, int W, int dtype, int activation, int l2norm_group, thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * recompute_w_u -- replaces kernels/recompute_w_u/kernel.py:192-248
 * (_launch / custom_kernel; Triton recompute_w_u_kernel :73-186).
 *
 * Per 64-token chunk:  w = A (k * beta * exp(g)),  u = A (v * beta).
 *   k [B,T,H,K], v [B,T,H,V] in `dtype`; beta, g [B,T,H] fp32;
 *   A [B,T,H,64] fp32 (row t of its chunk's matrix at position t);
 *   w [B,T,H,K], u [B,T,H,V] written in `dtype`.
 * a_mode  0: A is read from `A` (the reference contract).
 * a_mode -1: A is computed in-kernel as (I - M)^-1 (the reference's upstream
 *            producer, kernels/recompute_w_u/reference.py:48-91),
 * a_mode +1: A = (I + M)^-1 (gated DeltaNet), with
 *            M = strict_tril(beta_i k_i.k_j exp(g_i - g_j)); `A` is ignored and
 *            may be NULL; if A_out != NULL the computed A is stored there fp32.
 * T % 64 == 0; K in {64, 128}; V in {64, 128}.
 * ------------------------------------------------------------------------- */
int thm_recompute_w_u_fwd(const void* k, const void* v, const float* beta, const float* A, const float* g,
                          void* w, void* u, float* A_out, int B, int T, int H, int K, int V, int dtype,
                          int a_mode, thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * recompute_w_u with the v projection's conv folded in -- replaces the pair
 * kernels/causal_conv1d (kernel.py:170-230, on the v projection, activation
 * as given, no norm) -> kernels/recompute_w_u/kernel.py:192-248, which the
 * layer chains (docs/ARCHITECTURE.md:200-235) with v read only by the second.
 *
 *   v = act(conv_b + sum_k conv_w[:, k] * xv[t - 3 + k])  (causal, zero before
 *   each sequence's first token), then w, u as thm_recompute_w_u_fwd with
 *   a_mode +1 / -1; v itself is never written. xv [B,T,H*V] bf16 (the layer's
 *   channel-last projection), conv_w [H*V, 4], conv_b [H*V] fp32; k, beta, g,
 *   w, u, A_out as thm_recompute_w_u_fwd. v equals thm_causal_conv1d_fwd's
 *   bf16 output bit for bit, so w and u equal the two-launch path's.
 * bf16 only; conv_width 4; T % 64 == 0; K, V in {64, 128}.
 * ------------------------------------------------------------------------- */
int thm_recompute_w_u_conv_fwd(const void* k, const void* xv, const float* conv_w, const float* conv_b,
                               const float* beta, const float* g, void* w, void* u, float* A_out, int B, int T,
                               int H, int K, int V, int conv_width, int activation, int a_mode,
                               thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * build_A -- the upstream producer of recompute_w_u's A
 * (kernels/recompute_w_u/reference.py:48-91, `_build_A`), for callers that
 * pass A to thm_recompute_w_u_fwd with a_mode 0.
 *
 *   A_c = (I + sign * M_c)^-1,  M_c = strict_tril(beta_i k_i.k_j exp(g_i - g_j))
 * per 64-token chunk c; sign = -1 is the reference (I - M)^-1, +1 gated
 * DeltaNet's (I + M)^-1. k [B,T,H,K] in `dtype`; beta, g [B,T,H] fp32;
 * A [B,T,H,64] fp32 (row t of its chunk's matrix at position t).
 * T % 64 == 0; K in {64, 128}.
 * ------------------------------------------------------------------------- */
int thm_build_A_fwd(const void* k, const float* beta, const float* g, float* A, int B, int T, int H, int K,
                    int dtype, int sign, thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * chunk_local_cumsum -- the upstream producer of g: the reference's
 * generators form g as a per-chunk cumulative sum of per-token log-decay
 * increments (kernels/chunk_fwd_h/reference.py:41-45,
 * kernels/recompute_w_u/reference.py:103-106).
 *
 *   g[b, c*64 + i, h] = scale * sum_{j <= i} g_inc[b, c*64 + j, h]
 * g_inc, g [B,T,H] fp32 (g may be g_inc: in place); T % 64 == 0.
 * ------------------------------------------------------------------------- */
int thm_chunk_local_cumsum_fwd(const float* g_inc, float* g, int B, int T, int H, float scale,
                               thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * chunk_fwd_h -- replaces kernels/chunk_fwd_h/kernel.py:141-191
 * (custom_kernel; Triton chunk_fwd_h_kernel :61-138).
 *
 * mode 0 (reference): state = state*exp(g_end) + k_c^T (v_c * exp(g_end-g_c));
 *   h[b,c,h] = state AFTER chunk c.  `w`, `h0`, `v_new`, `final_state` must be
 *   NULL.
 * mode 1 (gated delta rule): with h_c the state entering chunk c (h_0 = h0,
 *   or 0 when h0 == NULL):
 *     v_new_c = u_c - w_c h_c
 *     h_{c+1} = exp(g_last) h_c + (k_c * exp(g_last - g_c))^T v_new_c
 *   h[b,c,h] = h_c (state BEFORE chunk c); `v` is u; v_new (optional)
 *   [B,T,H,V] in `dtype`; final_state (optional) [B,H,K,V] fp32 = h_NT.
 *   In mode 1 h may be NULL (no per-chunk states are written), e.g. when
 *   only the final state of a sequence segment is wanted.
 * k, w [B,T,H,K], v [B,T,H,V] in `dtype`; g [B,T,H] fp32;
 * h [B,T/64,H,K,V] in `h_dtype` (THM_F32 as the reference, or THM_BF16: the
 * state itself is always carried in fp32, only the stored copy is rounded);
 * h0 [B,H,K,V] fp32. T % 64 == 0; K in {64, 128}; V in {64, 128}.
 * ------------------------------------------------------------------------- */
int thm_chunk_fwd_h_fwd(const void* k, const void* w, const void* v, const float* g, const float* h0,
                        void* h, void* v_new, float* final_state, int B, int T, int H, int K, int V,
                        int dtype, int h_dtype, int mode, thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * chunk_fwd_o -- replaces kernels/chunk_fwd_o/kernel.py:146-212
 * (custom_kernel; Triton _chunk_fwd_o_kernel :52-136).
 *
 *   o = scale * ( tril_{s<=t}((q k^T) * exp(g_t - g_s)) v + (q * exp(g)) h[c] )
 * q, k [B,T,H,K], v [B,T,H,V], o [B,T,H,V] in `dtype`; g [B,T,H] fp32;
 * h [B,T/64,H,K,V] in `h_dtype` (used as given for chunk c).
 * T % 64 == 0; K in {64, 128}; V % 64 == 0, V <= 512 (h_dtype THM_BF16:
 * dtype THM_BF16 and V in {64, 128}, run by a persistent warp-specialized
 * kernel; h_dtype THM_F32: one CTA per (b, h, chunk, 64-wide V tile)).
 * ------------------------------------------------------------------------- */
int thm_chunk_fwd_o_fwd(const void* q, const void* k, const void* v, const float* g, const void* h, void* o,
                        float scale, int B, int T, int H, int K, int V, int dtype, int h_dtype,
                        thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * gated_delta_fwd_ho -- chunk_fwd_h (mode 1) and chunk_fwd_o fused: the
 * reference composes kernels/chunk_fwd_h/kernel.py:141-191 and
 * kernels/chunk_fwd_o/kernel.py:146-212 through HBM (h and v_new written,
 * then read back); this entry point produces the same o without either.
 *
 *   h_0 = h0 (or 0);  v_new_c = u_c - w_c h_c;
 *   h_{c+1} = exp(g_last) h_c + (k_c * exp(g_last - g_c))^T v_new_c
 *   o_c = scale * ( tril_{s<=t}((q k^T) * exp(g_t - g_s)) v_new_c + (q * exp(g)) h_c )
 * q, k, w [B,T,H,K], u [B,T,H,V], o [B,T,H,V] in `dtype`; g [B,T,H] fp32;
 * h0 (optional) and final_state (optional, = h_NT) [B,H,K,V] fp32.
 * The state is carried in fp32; it is rounded to bf16 only as an MMA operand,
 * and v_new once to bf16, as the separate ops do with a bf16 h.
 * Built for dtype THM_BF16, K = V = 128, T % 64 == 0 (else THM_ERR_UNSUPPORTED).
 * ------------------------------------------------------------------------- */
int thm_gated_delta_fwd_ho(const void* q, const void* k, const void* w, const void* u, const float* g,
                           const float* h0, void* o, float* final_state, float scale, int B, int T, int H, int K,
                           int V, int dtype, thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * thm_sp_prefix_fold -- states entering consecutive segments of a sequence
 * split along T (sequence parallel). The delta-rule recurrence of a segment
 * (kernels/chunk_fwd_h/kernel.py:61-138 with the delta rule) maps its entering
 * state affinely, h_out = M h_in + S; for R segments in order:
 *
 *   out[0] = x0 (or 0 when x0 is NULL),  out[r+1] = M[r] out[r] + S[r]
 *
 * for r < nout - 1. M [nout-1, BH, K, K], S [nout-1, BH, K, V], x0 [BH, K, V],
 * out [nout, BH, K, V], all fp32. K <= 128, K % 4 == 0, V % 32 == 0. No
 * reference counterpart as one call (the reference has no sequence-parallel
 * path); it replaces a loop of small batched matrix products.
 * ------------------------------------------------------------------------- */
int thm_sp_prefix_fold(const float* M, const float* S, const float* x0, float* out, int nout, int BH, int K, int V,
                       thm_stream_t stream);

/* ---------------------------------------------------------------------------
 * Utilities
 * ------------------------------------------------------------------------- */
/* Human-readable name of a thm_status. */
const char* thm_status_string(int status);

/* Reads (and, if reset != 0, clears) the device status word on the current
 * device: THM_OK, or the first in-kernel error (THM_ERR_TIMEOUT) recorded by
 * any kernel of this library since the last reset. Synchronizes the device. */
int thm_get_device_status(int* device_status, int reset);

/* ABI version: (major << 16) | minor. */
int thm_version(void);

/* Test hook for the timeout path: launches one warp that waits, through the
 * same bounded mbarrier wait every kernel here uses, on a barrier nobody
 * arrives on, for limit_ns nanoseconds (1e3 .. 1e8). The wait runs out, the
 * kernel records THM_ERR_TIMEOUT in the device status word and returns (no
 * TMA or tensor-core work is in flight), so thm_get_device_status() then
 * reports THM_ERR_TIMEOUT until reset; if waited_out (device int) is not NULL
 * it receives 1 when the wait ran out, 0 otherwise. No reference counterpart as
 * a call: it stands in for the reference harness's per-cell failure recording
 * (benchmarks/pytorch_baseline.py:99-110), which a test can trigger on demand. */
int thm_selftest_wait_timeout(long long limit_ns, int* waited_out, thm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* THEOREM_B200_H_ */
