/*
 * dc_attn.h — C ABI of the B200 (sm_100a) DC-attention forward.
 *
 * DC ("dynamically composable multi-head") attention forward for one layer:
 *   L_h   = scale * Q_h K_h^T                         (per head)
 *   S     = compose_pre(L)                            (across the HPG heads of a group)
 *   P_h   = softmax_s(mask(S_h))                      (causal, sliding window, seq_lens)
 *   P'    = compose_post(P)
 *   out_h = P'_h V_h
 * compose(a)[h] = [identity] a[h] + sum_h' a[h'] w[g,h',h]
 *               + sum_r qw2[b,t,r,h] sum_h' qw1[b,t,h',r] a[h']
 *               + sum_r kw2[b,s,r,h] sum_h' kw1[b,s,h',r] a[h']
 *               + (qdd[b,t,h] + kdd[b,s,h]) a[h]
 *               + sum_j qmat[b,t,h,j] a[g*HPG + j]
 *
 * The reference project (Lisennlp/dc_triton_opt) exposes this path through
 * pybind11/torch bindings only; the entry points below are the plain-pointer
 * equivalents those bindings would call:
 *   - dc_attn_fwd           replaces the general forward named by the project
 *                           (superset of dc_attention_torch.py:22-258)
 *   - dc_attn_fwd_residual  replaces dc_hopper_cuda/dc_hopper_api.cpp:17-28
 *                           (forward_hpg4_wide_ref / _opt / _cluster, kernel
 *                           dc_hopper_kernel.cu:639-687) and
 *                           dc_fused_cuda/kernel.cu:1350-1431
 *                           (dc_onekernel_v4_fwd_cuda), i.e. the residual
 *                           rank-1 form with six [B,T,N] weight tensors.
 *
 * Conventions (mirroring the reference bindings):
 *   - all pointers are device pointers owned by the caller; the library
 *     allocates nothing and never synchronises;
 *   - work is enqueued on `stream` (a cudaStream_t passed as void*; NULL =
 *     legacy default stream) and is asynchronous;
 *   - the return value is 0 on success or a negative DC_ERR_* code; the
 *     message of the last error on the calling thread is returned by
 *     dc_attn_last_error();
 *   - errors found on the device after a launch (a bounded wait inside a
 *     kernel that ran out: the kernel then skips the rest of its work and the
 *     output is not valid) are written to an error word, the caller's
 *     err_flag or the library's own per-device word, and read back with
 *     dc_attn_read_error().
 */
#ifndef DC_ATTN_H_
#define DC_ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DC_ATTN_ABI_VERSION 2

#if defined(_WIN32)
#define DC_API __declspec(dllexport)
#else
#define DC_API __attribute__((visibility("default")))
#endif

/* element type of q, k, v, out and the per-token composition weights */
enum dc_dtype { DC_DTYPE_BF16 = 0, DC_DTYPE_FP16 = 1 };

enum dc_status {
  DC_OK = 0,
  DC_ERR_NULL = -1,        /* a required pointer is NULL                       */
  DC_ERR_SHAPE = -2,       /* inconsistent or out-of-range sizes               */
  DC_ERR_DTYPE = -3,       /* unknown dtype                                    */
  DC_ERR_UNSUPPORTED = -4, /* valid request the selected kernel cannot handle  */
  DC_ERR_ALIGN = -5,       /* a pointer or stride breaks the 16-byte rule      */
  DC_ERR_LAUNCH = -6,      /* CUDA launch / attribute error                    */
  DC_ERR_DEVICE = -7       /* no sm_100 device / device query failed           */
};

/* kernel selection (dc_attn_params.kernel) */
enum dc_kernel {
  DC_KERNEL_AUTO = 0, /* fastest kernel that supports the request            */
  DC_KERNEL_SIMT = 1, /* general CUDA-core kernel: every term, any window    */
  DC_KERNEL_TC = 2,   /* tcgen05/TMEM/TMA kernel, single pass (windows up to
                         three key tiles, heads per group <= 8)              */
  DC_KERNEL_TCS = 3,  /* tcgen05 two-pass streaming kernel (any window incl.
                         full causal, heads per group <= 8)                  */
  DC_KERNEL_TCM = 4   /* two-pass streaming kernel with the static head mix
                         on the tensor cores (16 or 32 heads per group)     */
};

/* One composition term set (pre: on logits, post: on probabilities).
 * Every pointer may be NULL (term absent).  Per-token tensors are contiguous
 * in the params' dtype; w is fp32.  Shapes use B,T,H,G,R,HPG=H/G of the call. */
typedef struct dc_terms {
  int32_t identity;    /* non-zero: add a[h] (the reference's residual "+ L")   */
  const float *w;      /* [G, HPG, HPG]  static head mix, a'[h] += a[h'] w[g,h',h] */
  const void *qw1;     /* [B, T, H, R]   query-wise rank-R, first factor        */
  const void *qw2;     /* [B, T, R, H]   query-wise rank-R, second factor       */
  const void *kw1;     /* [B, T, H, R]   key-wise rank-R (indexed by the key)   */
  const void *kw2;     /* [B, T, R, H]                                          */
  const void *qdd;     /* [B, T, H]      query-wise diagonal gate               */
  const void *kdd;     /* [B, T, H]      key-wise diagonal gate                 */
  const void *qmat;    /* [B, T, H, HPG] per-query full mix inside the group    */
} dc_terms;

typedef struct dc_attn_params {
  int32_t abi_version;     /* must be DC_ATTN_ABI_VERSION                        */
  int32_t B, T, H, D, G, R;
  int32_t window;          /* > 0: key s visible iff t-window < s <= t; <= 0: full causal */
  float scale;             /* softmax scale applied to q.k                        */
  int32_t dtype;           /* enum dc_dtype                                       */
  int32_t kernel;          /* enum dc_kernel                                      */
  const void *q, *k, *v;   /* [B, T, H, D] contiguous                             */
  void *out;               /* out[b*out_sb + t*out_st + h*out_sh + d]             */
  int64_t out_sb, out_st, out_sh; /* element strides; d is contiguous             */
  const int32_t *seq_lens; /* [B] keys s >= seq_lens[b] are masked; NULL = T      */
  int32_t *err_flag;       /* optional device int32; a kernel whose bounded wait runs
                              out writes its DC_DEV_ERR_* code here (first code
                              wins).  NULL = the library's per-device error word  */
  dc_terms pre, post;
  uint32_t wait_us;        /* limit of every wait inside a kernel, microseconds;
                              0 = 2 s                                             */
  int32_t test_flags;      /* testing only, 0 in normal use (DC_TEST_*)           */
} dc_attn_params;

/* dc_attn_params.test_flags: the loading warp issues no loads, so every wait
 * of the launch runs out after wait_us and the kernel reports a timeout.  It
 * lets a test exercise the device-error path without a fault. */
#define DC_TEST_SKIP_LOADS 1

/* Device error codes (written to the error word, read by dc_attn_read_error). */
enum dc_dev_error {
  DC_DEV_OK = 0,
  DC_DEV_ERR_TIMEOUT_Q = 1,    /* query tile never arrived            */
  DC_DEV_ERR_TIMEOUT_FULL = 2, /* key / value tile never arrived      */
  DC_DEV_ERR_TIMEOUT_FREE = 3, /* ring slot never released            */
  DC_DEV_ERR_TIMEOUT_S = 4,    /* logits never completed              */
  DC_DEV_ERR_TIMEOUT_P = 5,    /* probabilities never written         */
  DC_DEV_ERR_TIMEOUT_O = 6     /* output accumulator never completed  */
};

/* General forward.  Returns DC_OK or a DC_ERR_* code. */
DC_API int dc_attn_fwd(const dc_attn_params *p, void *stream);

/* Residual rank-1 form of the reference (six [B,T,N] weights, identity
 * residual), output [B,T,N,D] written with the given element strides.
 * window <= 0 means full causal.  chunk_size is accepted for signature parity
 * with the reference and does not change the result. */
DC_API int dc_attn_fwd_residual(const void *q, const void *k, const void *v,
                         const void *pre_w1, const void *pre_w2, const void *pre_dd,
                         const void *post_w1, const void *post_w2, const void *post_dd,
                         void *out, int64_t out_sb, int64_t out_st, int64_t out_sh,
                         const int32_t *seq_lens, int32_t B, int32_t T, int32_t N,
                         int32_t D, int32_t G, float scaling, int32_t window,
                         int32_t chunk_size, int32_t dtype, void *stream);

/* Forward with q and k in 8-bit float (e4m3, one byte per element, [B,T,H,D]
 * contiguous) and per-tensor scales: the logits are
 * p->scale * q_scale * k_scale * (q8 . k8), with QK^T on the tensor cores in
 * e4m3 (tcgen05 kind::f8f6f4) and fp32 accumulation.  v, out and every weight
 * stay in p->dtype (bf16 / fp16), and so do the probabilities fed to P'V.
 * Runs the single-pass tensor-core kernel: heads per group 1, 2, 4 or 8,
 * D = 128, windows of at most three key tiles; other calls return
 * DC_ERR_UNSUPPORTED.  The reference names fp8 only as a later experiment
 * (fa3_dc_hopper_plan.md:113-116); no counterpart kernel. */
DC_API int dc_attn_fwd_fp8qk(const dc_attn_params *p, float q_scale, float k_scale, void *stream);

/* Packed variable-length batch: p->B must be 1 and p->T the total token count;
 * q, k, v, out and every per-token weight hold the sequences back to back,
 * sequence i being tokens [cu_seqlens[i], cu_seqlens[i+1]) (host array of
 * nseq + 1 non-decreasing values, cu_seqlens[0] = 0, cu_seqlens[nseq] = T).
 * Attention never crosses a sequence boundary.  p->seq_lens must be NULL.
 * Runs of consecutive sequences of equal length are launched together as one
 * batch; each run is one dc_attn_fwd launch on `stream`.  The reference
 * masks keys by seq_lens only (triton_dc_onekernel_v4_h100.py:661-664); this
 * packed layout has no counterpart there.  Returns DC_OK or a DC_ERR_* code
 * (the first failing run's). */
DC_API int dc_attn_fwd_varlen(const dc_attn_params *p, const int32_t *cu_seqlens, int32_t nseq, void *stream);

/* Producer of the per-token composition weights from the hidden states x
 * (DCFormer's dynamic weight projection; the reference has no code for this
 * step, its weights arrive precomputed):
 *   hidden = gelu(x W1), [M, I];   dw = hidden W2;   dd = tanh(x Wdd).
 * All matrices row-major in `dtype`; M = tokens (B*T), Dm and I multiples of
 * 32, H even.  Outputs (dtype, caller-owned, contiguous):
 *   dw[0..3] = pre qw1 [M,H,R], pre qw2 [M,R,H], pre kw1 [M,H,R], pre kw2 [M,R,H],
 *   dw[4..7] = the same for the post set    (W2 is [I, 8*H*R] in that order);
 *   dd[0..3] = pre qdd, pre kdd, post qdd, post kdd, [M,H] each
 *                                           (Wdd is [Dm, 4*H] in that order).
 * `hidden` is a caller-owned workspace of M*I elements. */
typedef struct dc_proj_params {
  int32_t M, Dm, I, H, R, dtype;
  const void *x;    /* [M, Dm]       */
  const void *w1;   /* [Dm, I]       */
  const void *w2;   /* [I, 8*H*R]    */
  const void *wdd;  /* [Dm, 4*H]     */
  void *hidden;     /* [M, I] workspace */
  void *dw[8];
  void *dd[4];
} dc_proj_params;

DC_API int dc_proj_weights(const dc_proj_params *p, void *stream);

/* Largest M * I (tokens x MLP width) that dc_proj_weights_noalloc accepts:
 * its `hidden` activations live in a fixed 8 MiB device array. */
#define DC_PROJ_NOALLOC_MAX_HIDDEN (4 * 1024 * 1024)

/* dc_proj_weights for callers that cannot allocate device memory: code that
 * runs where cudaMalloc is unavailable or forbidden (inside a custom
 * allocator's own callbacks, under a framework that owns every byte of the
 * device through a memory pool, or in a tightly budgeted inference server
 * that admits no allocation after start-up) still has to produce the
 * weights.  The caller passes inputs and outputs as usual; p->hidden is
 * ignored.  The intermediate activations go to a library-owned
 * `static __device__` array of DC_PROJ_NOALLOC_MAX_HIDDEN elements, which every
 * GPU that loads this library holds until the process exits.  Calls with
 * M * I above that limit return DC_ERR_SHAPE.  The first call on a device
 * looks the array's device address up (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  All calls share
 * the one array: calls that may run at the same time on the GPU (different
 * streams without ordering) race on it.  Nothing in the array needs to start
 * at zero (every element a call reads it has written first).  No cudaMalloc,
 * cudaFree or allocating library routine is called.  No counterpart in the
 * reference. */
DC_API int dc_proj_weights_noalloc(const dc_proj_params *p, void *stream);

/* Gradients of one composition term set, fp32, caller-owned; a NULL pointer
 * means the gradient is not wanted.  Shapes as in dc_terms.  The per-token
 * gradients are written; w is a sum over every (b, t) and is zeroed by the
 * library before it accumulates. */
typedef struct dc_term_grads {
  float *w;     /* [G, HPG, HPG]  */
  float *qw1;   /* [B, T, H, R]   */
  float *qw2;   /* [B, T, R, H]   */
  float *qdd;   /* [B, T, H]      */
  float *qmat;  /* [B, T, H, HPG] */
} dc_term_grads;

typedef struct dc_attn_bwd_params {
  dc_attn_params fwd;  /* the forward call being differentiated (out, out
                          strides, kernel, wait_us and test_flags unused) */
  const void *dout;    /* [B, T, H, D] contiguous, dtype of the forward     */
  void *dq;            /* [B, T, H, D] contiguous, dtype of the forward     */
  float *dk, *dv;      /* [B, T, H, D] contiguous fp32: zeroed, then
                          accumulated by the library (keys are shared by
                          neighbouring query blocks)                        */
  dc_term_grads dpre, dpost;
} dc_attn_bwd_params;

/* Backward of dc_attn_fwd for the query-side term family (identity, w,
 * qw1/qw2 of rank <= 2, qdd, qmat; key-wise terms are not covered) and
 * heads per group in {1, 2, 4, 8, 16, 32}, D = 128, windows whose key span
 * fits one block (any practical sliding window; full causal only for short
 * T).  Replaces TritonDCResidual.backward (triton_dc_residual.py:1707-1892),
 * which returns dq in the input dtype and dk, dv and the six weight
 * gradients in fp32, as here.  Everything is recomputed from q, k, v and the
 * weights; no forward state is needed.  Returns DC_OK or a DC_ERR_* code. */
DC_API int dc_attn_bwd(const dc_attn_bwd_params *p, void *stream);

/* sizeof(dc_attn_bwd_params) in this build. */
DC_API int dc_attn_bwd_params_size(void);

/* Read the device error word `err_flag` (NULL = the library's word on the
 * current device) after the work queued on `stream` so far: the call enqueues
 * a copy on `stream` and synchronises with it.  Returns the DC_DEV_* code
 * (0 = no error) or a negative DC_ERR_* code if the copy failed.  With
 * clear != 0 the word is reset to 0 afterwards.  No counterpart in the
 * reference, whose kernels never wait on a barrier that can stay open. */
DC_API int dc_attn_read_error(int32_t *err_flag, int clear, void *stream);

/* The kernel (enum dc_kernel) the last successful dc_attn_fwd call on the
 * calling thread launched, 0 if none yet. */
DC_API int dc_attn_last_kernel(void);

/* Which kernel DC_KERNEL_AUTO would pick for *p (enum dc_kernel), or a
 * negative DC_ERR_* code if no kernel supports the request. */
DC_API int dc_attn_select_kernel(const dc_attn_params *p);

/* Message of the last error on the calling thread ("" if none). */
DC_API const char *dc_attn_last_error(void);

/* Library ABI version (DC_ATTN_ABI_VERSION of the build). */
DC_API int dc_attn_abi_version(void);

/* sizeof(dc_attn_params) in this build, so FFI bindings can check their
 * struct mirror. */
DC_API int dc_attn_params_size(void);

#ifdef __cplusplus
}
#endif

#endif /* DC_ATTN_H_ */
