/*
 * hlm_b200.h -- C ABI of the hackable-lm B200 operator library (libhlm_b200.so).
 *
 * Hand-written sm_100a CUDA kernels for the fused operator hot path of
 * hackable-lm: residual-add + RMSNorm, QKV projection + QK-norm + RoPE,
 * SwiGLU, and the fused LM-head + cross-entropy loss, each forward and
 * backward.
 *
 * Conventions (every entry point):
 *   - All tensor arguments are DEVICE pointers owned by the caller.  The
 *     library never allocates or frees device memory; where a kernel needs
 *     scratch memory the caller passes a workspace whose size comes from the
 *     matching *_workspace_bytes() query.
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued on it and
 *     nothing synchronises the host.
 *   - Return value: HLM_OK (0) or a negative HLM_ERR_* code.  Nothing traps,
 *     exits or throws across this boundary.  hlm_strerror() names a code.
 *   - dtype codes: HLM_F32, HLM_BF16, HLM_F16.  The tensor-core paths
 *     (QKV, LM head, GEMM) take bf16 operands.
 *   - Kernels that wait on other warps bound every wait; a wait that runs out
 *     records a code in a device error word read by hlm_device_error_get().
 *
 * Reference citations are paths inside the hackable-lm repository.
 */
#ifndef HLM_B200_H_
#define HLM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HLM_OK 0
#define HLM_ERR_INVALID_ARG (-1)  /* null pointer, negative size, bad rank */
#define HLM_ERR_UNSUPPORTED (-2)  /* shape / dtype / stride / alignment not supported */
#define HLM_ERR_LAUNCH (-3)       /* CUDA launch or runtime error */
#define HLM_ERR_WORKSPACE (-4)    /* workspace smaller than required */
#define HLM_ERR_DRIVER (-5)       /* driver entry point / tensor-map encode failed */

#define HLM_F32 0
#define HLM_BF16 1
#define HLM_F16 2

/* Library version (major*10000 + minor*100 + patch). */
int hlm_version(void);

/* Static string naming an HLM_* return code. */
const char* hlm_strerror(int code);

/* Copy the device error word (0 = none) to *out; synchronises `stream`.
 * Test and diagnostics use only. */
int hlm_device_error_get(int* out, void* stream);

/* Reset the device error word to 0 (stream-ordered). */
int hlm_device_error_clear(void* stream);

/* Codes of the device error word.  A kernel whose bounded wait runs out
 * records the first code (later ones are dropped), drains its own in-flight
 * copies, frees its tensor memory and returns; nothing traps. */
#define HLM_DEVERR_NONE 0
#define HLM_DEVERR_TIMEOUT_FULL 1       /* MMA issuer waited too long for a TMA stage */
#define HLM_DEVERR_TIMEOUT_EMPTY 2      /* producer waited too long for a free stage */
#define HLM_DEVERR_TIMEOUT_TMEM_FULL 3  /* epilogue waited too long for an accumulator */
#define HLM_DEVERR_TIMEOUT_TMEM_EMPTY 4 /* MMA issuer waited too long for the epilogue */
#define HLM_DEVERR_TIMEOUT_DRAIN 5      /* teardown drain of in-flight TMA copies ran out */
#define HLM_DEVERR_BAD_TMEM 6           /* tcgen05.alloc returned an unexpected address */
#define HLM_DEVERR_SELFTEST_TIMEOUT 7   /* hlm_selftest_bounded_wait ran out, as it should */
#define HLM_DEVERR_TIMEOUT_EPI_LOAD 8   /* an epilogue waited too long for its own TMA input load */
#define HLM_DEVERR_TIMEOUT_PEER 9       /* an epilogue waited too long for its cluster peers' row sums */

/* Self-test of the bounded waits: one warp waits on an mbarrier that nothing
 * arrives at, with the same wait helper the GEMM roles use (scope 0: CTA-scope
 * acquire; 1: cluster-scope acquire) and a limit of limit_us microseconds
 * (1 .. 1000000) instead of the kernels' 1 s.  When the limit runs out the
 * kernel records HLM_DEVERR_SELFTEST_TIMEOUT and returns, leaving the context
 * usable.  Asynchronous on `stream`; read the result with
 * hlm_device_error_get. */
int hlm_selftest_bounded_wait(int64_t limit_us, int scope, void* stream);

/* Number of kernels this library has launched in this process (all devices).
 * Lets a harness count the library's own launches inside a timed region. */
uint64_t hlm_launch_count(void);

/* Kernel ids for hlm_profile_begin / hlm_profile_end. */
#define HLM_KERNEL_LM_LOGITS 1     /* LM head: logits GEMM + softmax statistics */
#define HLM_KERNEL_LM_DLOGITS 2    /* LM head: in-place softmax - onehot */
#define HLM_KERNEL_LM_DX 3         /* LM head: grad_hidden GEMM */
#define HLM_KERNEL_LM_DW 4         /* LM head: grad_weight GEMM */
#define HLM_KERNEL_QKV_FWD 5       /* QKV GEMM + norm/RoPE epilogue */
#define HLM_KERNEL_QKV_BWD_NORM 6  /* QKV backward: norm/RoPE backward */
#define HLM_KERNEL_QKV_DX 7        /* QKV backward: grad_x GEMM */
#define HLM_KERNEL_QKV_DW 8        /* QKV backward: grad_w GEMM */
#define HLM_KERNEL_SWIGLU_FWD 9
#define HLM_KERNEL_SWIGLU_BWD 10
#define HLM_KERNEL_RMSNORM_FWD 11
#define HLM_KERNEL_RMSNORM_BWD 12
#define HLM_KERNEL_QK_ROPE_FWD 13
#define HLM_KERNEL_QK_ROPE_BWD 14
#define HLM_KERNEL_GEMM 15
#define HLM_KERNEL_GATE_UP 16      /* gate_up GEMM + SwiGLU epilogue */
#define HLM_KERNEL_SWIGLU_DOWN_BWD 17 /* down grad_h GEMM + SwiGLU backward epilogue */
#define HLM_KERNEL_PROJ_NORM 18    /* o_proj / down GEMM + residual add + RMSNorm epilogue */
#define HLM_KERNEL_ATTN_FWD 19     /* attention forward (causal / sliding window) */
#define HLM_KERNEL_ATTN_BWD 20     /* attention backward (its three launches) */
#define HLM_KERNEL_MAX 21

/* Start timing every launch of kernel `kernel_id`: launch i records
 * start_events[i] immediately before and stop_events[i] immediately after
 * it, on the launching stream (cudaEvent_t handles created by the caller),
 * for i < capacity.  Profiling use only; not for use during graph capture. */
int hlm_profile_begin(int kernel_id, void* const* start_events, void* const* stop_events,
                      int capacity);

/* Stop timing kernel `kernel_id`; *launches receives how many launches
 * happened since hlm_profile_begin (may exceed the capacity). */
int hlm_profile_end(int kernel_id, int* launches);

/* ------------------------------------------------------------------------
 * SwiGLU
 * ------------------------------------------------------------------------ */

/* out[r, j] = silu(gate_up[r, j]) * gate_up[r, hidden + j]
 * gate_up: contiguous [rows, 2*hidden]; out: contiguous [rows, hidden].
 * Replaces torch.ops.hackable_lm.swiglu (kernels.py:388-402) and its
 * Triton kernel _swiglu_kernel (kernels.py:343-358). */
int hlm_swiglu_fwd(const void* gate_up, void* out, int64_t rows, int64_t hidden, int dtype,
                   void* stream);

/* grad_gate_up[r, j]          = g * up * s * (1 + gate * (1 - s))
 * grad_gate_up[r, hidden + j] = g * gate * s,   s = sigmoid(gate)
 * Replaces torch.ops.hackable_lm.swiglu_backward (kernels.py:404-419) and
 * _swiglu_backward_kernel (kernels.py:365-386). */
int hlm_swiglu_bwd(const void* gate_up, const void* grad_out, void* grad_gate_up, int64_t rows,
                   int64_t hidden, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Residual add + RMSNorm
 * ------------------------------------------------------------------------ */

/* out  = residual + branch                      (rounded to dtype)
 * norm = out * rsqrt(mean(out^2) + eps) [* weight]
 * residual may be NULL: then x = branch, `out` is not written, and the call
 * is the plain RMSNorm of kernels.rms_norm (kernels.py:245-247) /
 * model.rms_norm_torch (model.py:14-16).  weight may be NULL (weightless,
 * as in the model).  All row-major contiguous [rows, cols].
 * Replaces model.residual_rms_norm (model.py:73-75). */
int hlm_residual_rms_norm_fwd(const void* residual, const void* branch, const void* weight,
                              void* out, void* norm, int64_t rows, int64_t cols, float eps,
                              int dtype, void* stream);

/* Backward of hlm_residual_rms_norm_fwd, given the saved pre-norm x (= out).
 *   grad_in = grad_out + r*(g*w) - x*r^3*mean((g*w)*x),   r = rsqrt(mean(x^2)+eps)
 * grad_out may be NULL (treated as zero).  grad_in receives the gradient of
 * both residual and branch.  If weight != NULL, grad_weight[cols] (dtype) is
 * written = sum_rows g * x * r, reduced deterministically through `workspace`
 * (fp32, hlm_rms_norm_bwd_workspace_bytes bytes). */
int hlm_residual_rms_norm_bwd(const void* x, const void* weight, const void* grad_out,
                              const void* grad_norm, void* grad_in, void* grad_weight,
                              void* workspace, size_t workspace_bytes, int64_t rows,
                              int64_t cols, float eps, int dtype, void* stream);
size_t hlm_rms_norm_bwd_workspace_bytes(int64_t rows, int64_t cols);

/* Allocation-free variant of hlm_residual_rms_norm_bwd for the weighted case
 * (weight and grad_weight required), for callers that cannot allocate device
 * memory when they call it: hosts that plan every device byte up front, and
 * code that must not stall the device (cudaMalloc/cudaFree synchronise).
 * No counterpart in the reference: it has no caller-allocated-workspace
 * convention to avoid.
 *   - Scratch (the dweight partial sums) lives in a fixed 4 MiB array inside
 *     the library, held on every GPU that loads it until the process exits.
 *   - cols must be <= HLM_NOALLOC_RMS_MAX_COLS, else HLM_ERR_UNSUPPORTED.
 *   - Each call made outside stream capture looks up the array's device
 *     address on the current device (so a context re-created after
 *     cudaDeviceReset is handled); a call inside a capture reuses the address
 *     of an earlier uncaptured call on that device, and is refused with
 *     HLM_ERR_UNSUPPORTED when there was none: make the first call on each
 *     device outside any stream capture.
 *   - Calls share the array: calls that overlap on the GPU (different streams,
 *     different threads) race and must be serialised by the caller.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 * Results are identical to hlm_residual_rms_norm_bwd with a workspace. */
#define HLM_NOALLOC_RMS_MAX_COLS 1024
int hlm_residual_rms_norm_bwd_noalloc(const void* x, const void* weight, const void* grad_out,
                                      const void* grad_norm, void* grad_in, void* grad_weight,
                                      int64_t rows, int64_t cols, float eps, int dtype,
                                      void* stream);

/* ------------------------------------------------------------------------
 * QK-norm + partial rotate-half RoPE (standalone, strided inputs)
 * ------------------------------------------------------------------------ */

/* For every head vector x of q [B,T,Hq,D] and k [B,T,Hk,D] (element strides
 * q_strides[4], k_strides[4], any layout):
 *   z = x * rsqrt(mean(x^2) + eps)
 *   out[d]        = z[d]*c[d] - z[d+h]*s[d]      for d <  h = rotary_dim/2
 *   out[d]        = z[d]*c[d-h] + z[d-h]*s[d-h]  for h <= d < rotary_dim
 *   out[d]        = z[d]                         for d >= rotary_dim
 * with c/s = cos/sin[t, .] ([T, rotary_dim] tables of which only the first
 * half is read, as in _apply_partial_rope (kernels.py:670-676); row stride
 * cs_stride_t, dtype cs_dtype).  q_out/k_out are contiguous [B,T,H,D] in `dtype`.
 * Replaces torch.ops.hackable_lm.qk_norm_rope (kernels.py:505-539) and
 * _qk_norm_rope_kernel (kernels.py:446-503). */
int hlm_qk_norm_rope_fwd(const void* q, const void* k, const void* cos, const void* sin,
                         void* q_out, void* k_out, int64_t B, int64_t T, int64_t Hq, int64_t Hk,
                         int64_t D, int64_t rotary_dim, const int64_t* q_strides,
                         const int64_t* k_strides, int64_t cs_stride_t, int cs_dtype, float eps,
                         int dtype, void* stream);

/* Backward: g_n = inverse rotation of the output gradient, then
 * dx = inv * (g_n - z * mean(g_n * z)).  q/k are the saved pre-norm inputs
 * (strided as above); grad_q/grad_k and the results are contiguous.
 * Replaces torch.ops.hackable_lm.qk_norm_rope_backward (kernels.py:614-658)
 * and _qk_norm_rope_backward_kernel (kernels.py:546-612). */
int hlm_qk_norm_rope_bwd(const void* q, const void* k, const void* grad_q, const void* grad_k,
                         const void* cos, const void* sin, void* grad_q_in, void* grad_k_in,
                         int64_t B, int64_t T, int64_t Hq, int64_t Hk, int64_t D,
                         int64_t rotary_dim, const int64_t* q_strides, const int64_t* k_strides,
                         int64_t cs_stride_t, int cs_dtype, float eps, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Fused QKV projection + QK-norm + RoPE (tcgen05 GEMM, head-split epilogue)
 * ------------------------------------------------------------------------ */

/* x [B*T, C] bf16 (row-major), w_qkv [(Hq+2*Hk)*D, C] bf16 (nn.Linear
 * layout).  Computes qkv = x @ w_qkv^T in fp32 on the tensor cores and, per
 * 128-wide head tile in the epilogue: q/k heads -> RMSNorm over D + RoPE
 * (position t = row mod T) -> q_out/k_out; v heads -> v_out.  Outputs are
 * contiguous [B,T,H,D] bf16.  rstd [B*T, Hq+Hk] fp32 receives the per-head
 * 1/rms used by the backward.  D must be 128.
 * Replaces QKVProjection._project + fwd_triton (model.py:92-99, 117-126). */
int hlm_qkv_rope_fwd(const void* x, const void* w_qkv, const void* cos, const void* sin,
                     void* q_out, void* k_out, void* v_out, float* rstd, int64_t B, int64_t T,
                     int64_t C, int64_t Hq, int64_t Hk, int64_t D, int64_t rotary_dim,
                     int64_t cs_stride_t, int cs_dtype, float eps, void* stream);

/* Backward of hlm_qkv_rope_fwd.  From the saved outputs q_out/k_out and
 * rstd, recovers the normalised vectors, applies the norm/RoPE backward to
 * grad_q/grad_k (contiguous [B,T,H,D] bf16), then computes on the tensor
 * cores grad_x = [dq|dk|dv] @ w_qkv and grad_w = [dq|dk|dv]^T @ x.
 * grad_x or grad_w may be NULL (not needed).  Workspace bytes from
 * hlm_qkv_rope_bwd_workspace_bytes.  With both requested, grad_w runs on the
 * library's per-device side stream beside grad_x, forked from `stream` and
 * joined back into it before the call returns (stream-ordered, capturable).
 * Replaces the autograd backward of QKVProjection.fwd_triton: view/split
 * backward + _qk_norm_rope_backward (kernels.py:711-735) + the qkv_proj
 * nn.Linear dgrad/wgrad. */
int hlm_qkv_rope_bwd(const void* x, const void* w_qkv, const void* q_out, const void* k_out,
                     const float* rstd, const void* cos, const void* sin, const void* grad_q,
                     const void* grad_k, const void* grad_v, void* grad_x, void* grad_w,
                     void* workspace, size_t workspace_bytes, int64_t B, int64_t T, int64_t C,
                     int64_t Hq, int64_t Hk, int64_t D, int64_t rotary_dim, int64_t cs_stride_t,
                     int cs_dtype, float eps, void* stream);
size_t hlm_qkv_rope_bwd_workspace_bytes(int64_t B, int64_t T, int64_t C, int64_t Hq, int64_t Hk,
                                        int64_t D);

/* ------------------------------------------------------------------------
 * Fused LM head + cross-entropy (forward and backward in one call)
 * ------------------------------------------------------------------------ */

/* hidden [n_tokens, C] bf16, weight [V, C] bf16, targets [n_tokens] int64.
 * Rows whose target equals ignore_index contribute no loss and no gradient;
 * the loss is the mean over the other rows (F.cross_entropy semantics with
 * ignore_index).  Writes the scalar loss (fp32, device) and, when non-NULL,
 * grad_hidden [n_tokens, C] and grad_weight [V, C] (bf16) = d(loss)/d(.).
 * Logits are produced tile by tile on the tensor cores; full fp32 logits are
 * never materialised.  chunk_tokens bounds the token rows processed per
 * pass (0 = choose automatically); the workspace size depends on it.
 * Replaces _TritonFusedLinearCrossEntropy.forward (kernels.py:878-931) and
 * _linear_ce_kernel (kernels.py:291-318). */
int hlm_lm_head_ce(const void* hidden, const void* weight, const int64_t* targets, float* loss,
                   void* grad_hidden, void* grad_weight, void* workspace, size_t workspace_bytes,
                   int64_t n_tokens, int64_t C, int64_t V, int64_t ignore_index,
                   int64_t chunk_tokens, void* stream);
size_t hlm_lm_head_ce_workspace_bytes(int64_t n_tokens, int64_t C, int64_t V,
                                      int64_t chunk_tokens);

/* data[i] *= *scale for i < n (scale is a device fp32 scalar).  Backward of
 * the fused LM head, replacing _scale_saved_grad (kernels.py:872-875). */
int hlm_scale_by_device_scalar(void* data, const float* scale, int64_t n, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * MLP: gate_up projection with the SwiGLU activation in its epilogue
 * ------------------------------------------------------------------------ */

/* gate_up projection + SwiGLU in one CTA-pair tcgen05 GEMM.  Replaces
 * GateUpProjection.fwd_triton (model.py:291-292): gate_up = x @ W^T followed by
 * swiglu_triton (kernels.py:743-753).  x [M, C] bf16 row-major, w_gate_up
 * [2H, C] bf16 (gate rows first, then up rows, the reference's packed
 * layout); writes gate_up [M, 2H] bf16 (kept for the backward) and
 * h = silu(gate) * up [M, H] bf16 (fp32 math on the bf16-rounded gate/up).
 * Requires C % 64 == 0, H % 128 == 0, 16-byte aligned pointers. */
int hlm_gate_up_swiglu_fwd(const void* x, const void* w_gate_up, void* gate_up_out, void* h_out,
                           int64_t M, int64_t C, int64_t H, void* stream);

/* Backward through the down projection and the SwiGLU in one CTA-pair tcgen05
 * GEMM: grad_h = grad_y @ W_down (rounded to bf16, the dtype of the reference's
 * F.linear backward output, model.py:301-304), then the SwiGLU backward of
 * _swiglu_backward (kernels.py:690-700) on the saved gate_up, written as
 * grad_gate_up [M, 2H] bf16; grad_h itself never goes to memory.  grad_y
 * [M, C], w_down [C, H] (the nn.Linear weight of the down projection),
 * gate_up [M, 2H], all bf16 row-major.  Requires C % 64 == 0, H % 256 == 0,
 * 16-byte aligned pointers.  (The down projection's weight gradient and the
 * gate_up GEMM's input gradients are separate GEMMs.) */
int hlm_swiglu_down_bwd(const void* grad_y, const void* w_down, const void* gate_up,
                        void* grad_gate_up, int64_t M, int64_t C, int64_t H, void* stream);

/* ------------------------------------------------------------------------
 * Output / down projection with the residual add and RMSNorm in its epilogue
 * ------------------------------------------------------------------------ */

/* branch = y @ w^T (rounded to bf16, the reference's F.linear output),
 * out = residual + branch (rounded to bf16), norm = out * rsqrt(mean(out^2) +
 * eps) over each row of N values (fp32 math on the bf16 out), all in one
 * tcgen05 GEMM whose epilogue sees whole rows: the N columns of a 128-row
 * block are split over a cluster of N / BN CTAs (BN = 256, or 128 when N is
 * not a multiple of 256), which exchange their per-row sums of squares
 * through distributed shared memory.  Replaces OutputProjection.fwd_torch
 * (model.py:253-264) and DownProjection.fwd_torch (model.py:303-304): the
 * nn.Linear GEMM followed by residual_rms_norm (model.py:73-75).
 * y [M, K], w [N, K] (the nn.Linear weight), residual / out / norm [M, N], all
 * bf16 row-major, 16-byte aligned.  Requires K % 64 == 0 and N a multiple of
 * 128 with N <= 1024 (N = 1..4 times 256, or 1..4 times 128); other shapes
 * return HLM_ERR_UNSUPPORTED. */
int hlm_proj_residual_rms_norm_fwd(const void* y, const void* w, const void* residual, void* out,
                                   void* norm, int64_t M, int64_t K, int64_t N, float eps,
                                   void* stream);

/* ------------------------------------------------------------------------
 * Attention forward (causal, optional sliding window), head_dim 128
 * ------------------------------------------------------------------------ */

/* out[b,t,h,:] = softmax over keys k with 0 <= t - k < window of
 * (q[b,t,h,:] . k[b,k,hk,:]) * scale, times v[b,k,hk,:]; hk = h / (H / Hk).
 * lse[b,h,t] = log(sum_k exp(scale * q . k)) (natural log, fp32), the
 * statistics a FlashAttention-style backward takes.  window <= 0 or >= T means
 * full causal.  q, out [B, T, H, 128] and k, v [B, T, Hk, 128] bf16 contiguous
 * (the layout hlm_qkv_rope_fwd writes).  Requires T % 128 == 0, H % Hk == 0,
 * 16-byte aligned pointers.  Replaces the FlashAttention / SDPA call of
 * kernels.scaled_dot_product_attention (kernels.py:774-847) with the window
 * convention (window - 1, 0) of kernels.py:839. */
int hlm_attention_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int64_t B,
                      int64_t T, int64_t H, int64_t Hk, int64_t D, int64_t window, float scale,
                      void* stream);

/* Gradients of hlm_attention_fwd: dq, dk, dv [B, T, H, 128] bf16 from grad_out
 * and the forward's q, k, v, out and lse (natural log, [B, H, T] fp32), the same
 * mask (window <= 0 or >= T: full causal), H == Hk.  workspace: at least
 * hlm_attention_bwd_workspace_bytes(B, T, H, D) bytes (an fp32 dq accumulator,
 * the per-row dot(dO, O) and the log-sum-exp in base 2), 16-byte aligned.  Replaces the backward of the
 * FlashAttention / SDPA call of kernels.scaled_dot_product_attention
 * (kernels.py:774-847) with the window convention (window - 1, 0) of
 * kernels.py:839.  Other shapes return HLM_ERR_UNSUPPORTED. */
size_t hlm_attention_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D);
int hlm_attention_bwd(const void* grad_out, const void* q, const void* k, const void* v, const void* out,
                      const float* lse, void* dq, void* dk, void* dv, void* workspace,
                      size_t workspace_bytes, int64_t B, int64_t T, int64_t H, int64_t Hk, int64_t D,
                      int64_t window, float scale, void* stream);

/* ------------------------------------------------------------------------
 * Plain tcgen05 GEMM (building block; also used by tests)
 * ------------------------------------------------------------------------ */

/* D[M,N] = A[M,K] * B[N,K]^T (+ D if accumulate), bf16 operands, fp32
 * accumulation.  A is K-major (row-major [M][lda]) unless a_mn_major, in
 * which case it is stored [K][lda] with M contiguous; likewise B is
 * [N][ldb] (K-major) or [K][ldb] (N-major).  D is row-major [M][ldd] of
 * d_dtype (HLM_BF16 or HLM_F32).  Leading dimensions must be multiples of
 * 8 elements and base pointers 16-byte aligned.
 * Replaces the cuBLAS GEMMs under nn.Linear / torch.mm on this path
 * (model.py:94; kernels.py:913, 920, 922). */
int hlm_gemm_bf16(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                  int a_mn_major, int b_mn_major, int64_t lda, int64_t ldb, int64_t ldd,
                  int d_dtype, int accumulate, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HLM_B200_H_ */
