/* gated_delta_b200.h -- C ABI of the B200 (sm_100a) chunked gated delta rule.
 *
 * The reference (AbstractEyes/Mac-ai-engineering, package macai) reaches its GPU code through Metal kernels compiled by
 * torch.mps.compile_shader and dispatched as lib.<kernel>(...). Each entry point below replaces one of those dispatch
 * sites (cited as reference file:line), or one autograd step that sequences them. Every function:
 *   - takes raw device pointers, sizes and a CUDA stream (cudaStream_t passed as void*), no torch types;
 *   - allocates nothing: intermediates live in a caller-provided workspace of gd_workspace_bytes() (for
 *     gd_forward_noalloc, in a fixed array inside the library: see its comment);
 *   - launches on the given stream and does not synchronise (graph-capturable), except gd_read_error and
 *     gd_forward_noalloc, which are described on their own;
 *   - returns a status code (GD_OK or a GD_ERR_*) and never aborts or traps.
 *
 * Layouts (all contiguous, row-major):
 *   q, k        [B, T, HK, DK]   dtype GD_FLOAT32 / GD_FLOAT16 / GD_BFLOAT16 (q, k, v, o, do share one dtype)
 *   v, o, do    [B, T, H, DV]    H = value heads; HK = key heads, H % HK == 0 (HK < H: each key head serves H/HK
 *                                consecutive value heads, the repeat_interleave of the Qwen3.5 layer)
 *   g, beta     [B, T, H]        float32 (g = log decay <= 0)
 *   s0, sT, dsT, ds0 [B, H, DK, DV] float32
 *   dg, dbeta   [B, T, H]        float32;  dq, dk [B, T, HK, DK] and dv [B, T, H, DV] in the q/k/v dtype
 * Supported head widths: DK = DV = 128 (the Qwen3.5 / Qwen3-Next shapes). Chunk length 64 (fixed).
 */
#ifndef GATED_DELTA_B200_H
#define GATED_DELTA_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define GD_OK 0
#define GD_ERR_ARG 1       /* null pointer, unknown dtype or flag */
#define GD_ERR_SHAPE 2     /* unsupported sizes (head widths, H % HK) */
#define GD_ERR_ALIGN 3     /* a pointer is not 16-byte aligned */
#define GD_ERR_WORKSPACE 4 /* workspace smaller than gd_workspace_bytes() */
#define GD_ERR_LAUNCH 5    /* the CUDA launch failed */
#define GD_ERR_TIMEOUT 6   /* a bounded device-side wait gave up (recorded in the workspace's error word) */
#define GD_ERR_DEVICE 7    /* the current device is not sm_100 */
#define GD_ERR_SCRATCH 8   /* gd_forward_noalloc: the sizes need more than its fixed 64 MiB scratch array */

/* dtypes of q / k / v / o / do and of dq / dk / dv */
#define GD_FLOAT32 0
#define GD_FLOAT16 1
#define GD_BFLOAT16 2

/* flags */
#define GD_L2NORM 1        /* use_qk_l2norm_in_kernel: q and k rows are l2-normalised (eps 1e-6) in the prep kernel */
#define GD_STORE_STATES 2  /* the state pass keeps each chunk's entering state S_c and Vn for the backward */
#define GD_SCALE_Q 4       /* q is multiplied by DK^-1/2 (after the l2 norm): the drop-in's query scaling */
#define GD_STATES_STORED 8 /* gd_backward: the workspace already holds the states (gd_forward with GD_STORE_STATES) */
/* gd_fwd_state: the value split of the sequential pass. Without this flag the forward pass with O (no
 * GD_STORE_STATES) runs four CTAs per (value head, batch row or sequence), 32 value columns each, when all of them fit
 * on the GPU at once (4 x heads x rows <= SMs), else two CTAs of 64 columns (the reference's VALUE_SPLIT chosen from
 * the head-rows and the SM count, src/macai/gated_delta/op.py:75-87); with it, always two. The high-level entry points
 * (gd_forward, ...) use the automatic choice. */
#define GD_WIDE_STATE_PASS 16
/* Bits 16-23 (with GD_SCALE_Q): the caller's key head width when its q and k rows are zero-padded to the built width
 * 128 (a width of 32, 64 or 96 runs exactly in the 128-wide kernels: zero key dimensions change neither the l2 norms
 * nor the states, zero value columns stay zero); the query scale is then that width^-1/2. 0: the built width. The
 * high-level entry points pass these bits on. */
#define GD_KEY_WIDTH(dk) (((dk) & 0xff) << 16)
#define GD_KEY_WIDTH_MASK 0x00ff0000
/* Test only (never set in production): gd_fwd_state's MMA-issuing thread first waits on a barrier that nothing
 * signals, with a ~1 ms budget. The wait expires, the kernel records GD_ERR_TIMEOUT at stage 28 in the error word,
 * every role of the CTA gives up in its own bounded wait (~2 s) with no product or copy left in flight, and the CTA
 * frees its TMEM and returns: gd_read_error then reports (GD_ERR_TIMEOUT, 28), and the context stays usable. The
 * high-level entry points (gd_forward, gd_backward, ...) do not pass it on. */
#define GD_TEST_WAIT_EXPIRES 0x40000000

/* Text for a status code. */
const char* gd_status_string(int status);

/* Workspace bytes for one call of these sizes. for_backward != 0: enough for gd_backward (and for gd_forward). */
size_t gd_workspace_bytes(int B, int T, int H, int HK, int DK, int DV, int for_backward);

/* Per chunk (64 tokens) of every (batch row, value head), all independent: the l2 prologue of q and k, the in-chunk
 * cumulative log decay G, M = (Q K^T) * exp(G_i - G_j) (lower, diagonal included), the inverse A = (I + L)^-1 of
 * L = diag(beta) (K K^T) * exp(G_i - G_j) (strictly lower), W = A diag(beta gamma) K and U = A diag(beta) V, all into
 * the workspace.
 * Replaces: lib.gdc_prep (src/macai/gated_delta/op.py:63-72, kernel _chunked.py:220-313) and the fused prologue
 * l2n_fwd_* (src/macai/gated_delta/_norm.py:27-43, applied at op.py:276-278), with W and U of gdc_fwd's first stage. */
int gd_prep(const void* q, const void* k, const void* v, const float* g, const float* beta, int dtype, int B, int T,
            int H, int HK, int DK, int DV, int flags, void* workspace, size_t workspace_bytes, void* stream);

/* The sequential state pass, per (batch row, value head) with its value columns split over two or four CTAs (see
 * GD_WIDE_STATE_PASS): for each chunk in order,
 * Vn = U - W S, O = diag(gamma) Q S + M Vn, S <- exp(G_last) S + K^T diag(e) Vn; writes o (q's dtype) and, when sT is
 * not NULL, the final state. s0 NULL = zero initial state. flags & GD_STORE_STATES: also keeps S_c and Vn per chunk in
 * the workspace (the backward's recompute, o and sT then may be NULL; or the stored-states forward, with o).
 * Replaces: lib.gdc_fwd (src/macai/gated_delta/op.py:159 and :217, kernel _chunked.py:315-659). Requires gd_prep. */
int gd_fwd_state(const float* s0, void* o, float* sT, int dtype, int B, int T, int H, int HK, int DK, int DV,
                 int flags, void* workspace, size_t workspace_bytes, void* stream);

/* The reverse state pass, per (batch row, value head) with its value columns split over two CTAs, chunks last to
 * first, carrying dS:
 * dVn = M^T dO + diag(e) K dS, dS <- exp(G_last) dS + (diag(gamma) Q)^T dO - W^T dVn; keeps dS_{c+1} and dVn per
 * chunk in the workspace and writes ds0 (may be NULL). dsT NULL = zero. Requires gd_prep and
 * gd_fwd_state(GD_STORE_STATES) on the same workspace.
 * Replaces: lib.gdc_bwd_state (src/macai/gated_delta/op.py:234, kernel _chunked.py:661-903). */
int gd_bwd_state(const void* d_o, const float* dsT, float* ds0, int dtype, int B, int T, int H, int HK, int DK, int DV,
                 int flags, void* workspace, size_t workspace_bytes, void* stream);

/* Every per-chunk gradient, per (chunk, key head, batch row) item (persistent CTAs, one per SM, walk the items), all
 * independent and without atomics: dq, dk (through the l2 prologue when GD_L2NORM; summed over the value heads of a
 * key head in a fixed order), dv, dg (with the in-chunk reverse cumulative sum) and dbeta. Requires gd_bwd_state on the same workspace.
 * Replaces: lib.gdc_bwd_chunk (src/macai/gated_delta/op.py:241-242, kernel _chunked.py:905-1177) and the fused
 * prologue's backward l2n_bwd_* (src/macai/gated_delta/_norm.py:44-56, applied at :102-114). */
int gd_bwd_chunk(const void* q, const void* k, const void* v, const float* beta, const void* d_o, void* dq, void* dk,
                 void* dv, float* dg, float* dbeta, int dtype, int B, int T, int H, int HK, int DK, int DV, int flags,
                 void* workspace, size_t workspace_bytes, void* stream);

/* The forward of the autograd function: gd_prep then gd_fwd_state. flags & GD_STORE_STATES: the training forward of
 * the stored-states mode (the reference's op.RECOMPUTE_STATES = False, op.py:27-33, :142, :151-155, :165-167): the
 * workspace must hold gd_workspace_bytes(..., 1), and afterwards holds every chunk matrix, state and Vn the backward
 * reads; keep it unchanged for gd_backward(GD_STATES_STORED). Outputs are the same bits in both modes when the plain
 * training forward passes GD_WIDE_STATE_PASS (as the drop-in does when autograd records the call): the stored-states
 * forward always runs the two-CTA state pass. Without GD_WIDE_STATE_PASS and GD_STORE_STATES the state pass picks its
 * value split from the head-rows and the SM count (GD_WIDE_STATE_PASS above).
 * Replaces: GatedDeltaRule.forward (src/macai/gated_delta/op.py:119-185) as called by the drop-in (op.py:296). */
int gd_forward(const void* q, const void* k, const void* v, const float* g, const float* beta, const float* s0,
               void* o, float* sT, int dtype, int B, int T, int H, int HK, int DK, int DV, int flags, void* workspace,
               size_t workspace_bytes, void* stream);

/* The backward with the chunk states recomputed from the inputs: gd_prep, gd_fwd_state(GD_STORE_STATES),
 * gd_bwd_state, gd_bwd_chunk. d_o / dsT NULL = zero cotangents; ds0 may be NULL. flags & GD_STATES_STORED: the
 * workspace comes from gd_forward(GD_STORE_STATES) on the same inputs and the recompute is skipped (g and s0 are then
 * not read); the gradients are the same bits in both modes.
 * Replaces: GatedDeltaRule.backward in its recompute mode (src/macai/gated_delta/op.py:187-243, :207-218) and its
 * stored mode (ctx.mode "chunked", op.py:204-206). */
int gd_backward(const void* q, const void* k, const void* v, const float* g, const float* beta, const float* s0,
                const void* d_o, const float* dsT, void* dq, void* dk, void* dv, float* dg, float* dbeta, float* ds0,
                int dtype, int B, int T, int H, int HK, int DK, int DV, int flags, void* workspace,
                size_t workspace_bytes, void* stream);

/* Synchronises the stream and returns the first device-side failure recorded in the workspace's error word (GD_OK if
 * none), with the kernel stage that recorded it in *where (may be NULL); then clears the word. */
int gd_read_error(void* workspace, void* stream, int* where);

/* gd_forward for callers that cannot allocate device memory: a program whose device memory all belongs to another
 * allocator (a serving engine's reserved pool, a host framework that owns the GPU), or a caller that may not risk the
 * device synchronisation cudaMalloc / cudaFree can cause. Same arguments and results as gd_forward, without the
 * workspace: the intermediates go to one fixed 64 MiB device array inside the library (enough for
 * gd_workspace_bytes(..., 0) <= 64 MiB, e.g. 16 value heads x 1,984 tokens); larger sizes return GD_ERR_SCRATCH
 * before any device call. The library allocates nothing either: the array is static device memory, held until the
 * process exits on each GPU where this code has been loaded.
 *   - The first call on a device (that device current) looks the array's device address up with
 *     cudaGetSymbolAddress and keeps it; make that first call before any stream capture. The address belongs to the
 *     device's current context: after cudaDeviceReset the next call finds a new context and looks it up again (make
 *     that call before any capture, too).
 *   - flags as gd_forward's, except GD_STORE_STATES (GD_ERR_ARG): the stored-states forward's workspace must be kept
 *     until the backward, which the shared array cannot promise.
 *   - All calls on a device share the array. Each call clears the part that must start at zero (the error word) on
 *     its stream; calls whose work overlaps on the GPU race on the array, so the caller serialises them.
 *   - device_status NULL: asynchronous like gd_forward. Otherwise the call waits for its stream and stores the
 *     kernels' own status (GD_OK, or GD_ERR_TIMEOUT) in *device_status.
 * No counterpart in the reference: its Metal path allocates through torch. */
int gd_forward_noalloc(const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* s0, void* o, float* sT, int dtype, int B, int T, int H, int HK, int DK, int DV,
                       int flags, void* stream, int* device_status);

/* ---- packed rows (cu_seqlens) ----
 * N sequences concatenated along the token axis: q, k [T, HK, DK], v, o, do [T, H, DV], g, beta, dg, dbeta [T, H]
 * (one batch row of T rows in all), sequence n at rows cu_seqlens[n] .. cu_seqlens[n + 1] - 1 (cu_seqlens: N + 1
 * device int32, cu_seqlens[0] = 0, non-decreasing, cu_seqlens[N] = T; the kernels clamp any other input into range
 * rather than read out of bounds, but its results are then undefined). Every sequence runs as its own row: states
 * restart at its first token, s0 / sT / dsT / ds0 are [N, H, DK, DV] (s0, dsT NULL = zero), a sequence without tokens
 * passes its state through. Each sequence starts a new chunk; the results equal N separate calls. The chunk table is
 * built on the device from cu_seqlens (no host synchronisation: graph-capturable); o, dq, dk, dv are formed
 * chunk-aligned in the workspace and copied to the packed rows at the end.
 * Replaces: the drop-in's cu_seqlens argument, which the reference refuses (src/macai/gated_delta/op.py:270-273;
 * design note docs/prior_art_gated_delta.md:310-312), with fla's packed-sequence semantics (transformers' call site
 * passes cu_seqlens= to fla's kernel, layer/_qwen3_5.py:163-165). */
size_t gd_workspace_bytes_packed(int N, int T, int H, int HK, int DK, int DV, int for_backward);

/* gd_forward over packed rows (flags as gd_forward's, GD_STORE_STATES included). */
int gd_forward_packed(const void* q, const void* k, const void* v, const float* g, const float* beta,
                      const float* s0, void* o, float* sT, const int* cu_seqlens, int N, int dtype, int T, int H,
                      int HK, int DK, int DV, int flags, void* workspace, size_t workspace_bytes, void* stream);

/* gd_backward over packed rows (flags as gd_backward's, GD_STATES_STORED included: the workspace then comes from
 * gd_forward_packed with GD_STORE_STATES on the same inputs and cu_seqlens). */
int gd_backward_packed(const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* s0, const void* d_o, const float* dsT, void* dq, void* dk, void* dv, float* dg,
                       float* dbeta, float* ds0, const int* cu_seqlens, int N, int dtype, int T, int H, int HK, int DK,
                       int DV, int flags, void* workspace, size_t workspace_bytes, void* stream);

/* ---- the layer's gates (the step before the rule) ----
 * beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) (softplus with PyTorch's threshold of 20), both float32,
 * from b, a [n = rows * H] in `dtype` and A_log, dt_bias [H] in `wdtype` (GD_FLOAT32 / GD_FLOAT16 / GD_BFLOAT16);
 * element i belongs to head i % H. n < 2^31. No allocation, asynchronous on `stream`.
 * Replaces: the reference's one-pass gates kernels gates_fwd_* (src/macai/layer/_gates.py:27-35, :51-56, dispatched at
 * :91-92) and their autograd function's forward (:84-95). */
int gd_gates_fwd(const void* b, const void* a, const void* A_log, const void* dt_bias, float* beta, float* g,
                 int dtype, int wdtype, long long n, int H, void* stream);

/* Bytes of workspace gd_gates_bwd needs when it forms dA_log or ddt_bias (0 for invalid sizes). */
size_t gd_gates_workspace_bytes(long long n, int H);

/* db = dbeta * beta * (1 - beta), da = dg * (-exp(A_log)) * sigmoid(a + dt_bias) (1 above the threshold), in `dtype`;
 * dbeta / dg NULL = zero cotangents. dA_log = sum over rows of dg * g and ddt_bias = sum over rows of da (before its
 * cast), in `wdtype`, when not NULL (then `workspace` holds gd_gates_workspace_bytes(n, H)); the sums are taken in a
 * fixed order (no atomics: the same bits every run).
 * Replaces: gates_bwd_* (src/macai/layer/_gates.py:38-48, :57-63, dispatched at :105-106) and the autograd
 * function's reductions for trained gates (:108-116). */
int gd_gates_bwd(const void* b, const void* a, const void* A_log, const void* dt_bias, const float* dbeta,
                 const float* dg, void* db, void* da, void* dA_log, void* ddt_bias, int dtype, int wdtype, long long n,
                 int H, void* workspace, size_t workspace_bytes, void* stream);

/* ---- the gated RMSNorm on the rule's output (the step after the rule) ----
 * o = (w * (x * rsqrt(mean(x^2) + eps)).to(dtype) * silu(z)).to(dtype) over `rows` rows of width D (one value head
 * each), with transformers' rounding points: the product with w is rounded to `dtype` again when `wdtype` == `dtype`.
 * x, z, o: [rows, D] in `dtype`; w: [D] in `dtype` or GD_FLOAT32. D % 4 == 0, 0 < D <= 1024; every pointer 16-byte
 * aligned. No allocation, asynchronous on `stream`.
 * Replaces: the reference's gnorm_fwd_* kernels (src/macai/layer/_gated_norm.py:28-53, :107-114, dispatched at
 * :166-167) and their autograd function's forward (:157-171). */
int gd_gnorm_fwd(const void* x, const void* z, const void* w, void* o, int dtype, int wdtype, long long rows, int D,
                 float eps, void* stream);

/* Bytes of workspace gd_gnorm_bwd needs when it forms dw (0 for invalid sizes). */
size_t gd_gnorm_workspace_bytes(long long rows, int D);

/* dx, dz [rows, D] in `dtype` from dout (fp32 math, one rounding each; r recomputed from x). dw = the sum over rows of
 * dout * silu(z) * x_hat.to(dtype), in `wdtype`, when not NULL (then `workspace` holds gd_gnorm_workspace_bytes(rows,
 * D)); the sum is taken in a fixed order (no atomics: the same bits every run).
 * Replaces: gnorm_bwd_* (src/macai/layer/_gated_norm.py:55-104, :115-124, dispatched at :188-190), the weight
 * gradient's column sum col_sum (:127-137, :192-196) and the autograd function's backward (:172-197). */
int gd_gnorm_bwd(const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw,
                 int dtype, int wdtype, long long rows, int D, float eps, void* workspace, size_t workspace_bytes,
                 void* stream);

/* ---- the convolution path (the step that produces the rule's q, k, v) ----
 * u[t, c] = sum_j w[c, j] x[t - 3 + j, c] (depthwise causal, kernel 4, no bias, zero before each row's start) and
 * y = silu(u) on the fp32 u, over x [B, T, C] in `dtype` (the input projection's output read in place), written as the
 * rule's inputs: q, k [B, T, H_v, DK] in `dtype` from channels [0, KD) and [KD, 2 KD), each of the KD / DK key heads
 * written REP times (value head h REP + r); v [B, T, H_v, DV] in fp32 from channels [2 KD, C).
 * w: [C, 4] in `dtype` or GD_FLOAT32. Requires C = 2 KD + VD, KD % DK == 0, VD % DV == 0, (KD / DK) REP == VD / DV,
 * and C, KD, DK, DV multiples of 8 (16-bit) or 4 (fp32); x, q, k, v 16-byte aligned. No allocation, asynchronous.
 * Replaces: the reference's conv_fwd_* kernels (src/macai/layer/_conv.py:52-83, :139-146, dispatched at :201-203) and
 * their autograd function's forward (:191-207). */
int gd_conv_fwd(const void* x, const void* w, void* q, void* k, float* v, int dtype, int wdtype, int B, int T, int C,
                int KD, int DK, int REP, int DV, void* stream);

/* Bytes of workspace gd_conv_bwd needs when it forms dw (0 for invalid sizes). */
size_t gd_conv_workspace_bytes(int B, int T, int C);

/* dx [B, T, C] in `dtype` from dq, dk (in `dtype`, summed over the REP value heads of each key head) and dv (fp32);
 * any of the three NULL = a zero cotangent. u is recomputed from x. dw [C, 4] = the sum over rows and steps of
 * du[t, c] x[t - 3 + j, c], in `wdtype`, when not NULL (then `workspace` holds gd_conv_workspace_bytes(B, T, C)); the
 * sum is taken in a fixed order (no atomics: the same bits every run).
 * Replaces: conv_bwd_* (src/macai/layer/_conv.py:84-137, :147-156, dispatched at :228-230), the weight gradient's
 * sum dw_sum (:158-167, :232-236) and the autograd function's backward (:208-237). */
int gd_conv_bwd(const void* x, const void* w, const void* dq, const void* dk, const float* dv, void* dx, void* dw,
                int dtype, int wdtype, int B, int T, int C, int KD, int DK, int REP, int DV, void* workspace,
                size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GATED_DELTA_B200_H */
