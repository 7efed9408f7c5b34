/*
 * mt_b200.h -- C ABI of the B200 (sm_100a) transformer-op hot path.
 *
 * Every entry point takes plain device pointers, element counts, element
 * strides and a cudaStream_t (passed as void*), launches its kernels on that
 * stream and returns an mt_status code.  No entry point allocates device
 * memory: scratch buffers ("workspace") are passed in by the caller, whose
 * size is given by the matching *_workspace_bytes function.
 *
 * Each entry point names the reference operator it replaces
 * (duoan/mega-trading, paths relative to the project root).  The reference
 * binds those operators as Python functions; the Python mirror in
 * mega_trading_b200/kernels/ keeps their names, signatures and errors and
 * calls these functions through ctypes.
 *
 * dtype codes: MT_F32 = 0, MT_F16 = 1, MT_BF16 = 2.
 */
#ifndef MT_B200_H
#define MT_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define MT_API __attribute__((visibility("default")))
#else
#define MT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum mt_dtype { MT_F32 = 0, MT_F16 = 1, MT_BF16 = 2 };

enum mt_status {
  MT_OK = 0,
  MT_ERR_INVALID_ARGUMENT = 1,   /* shape / size / pointer mismatch            */
  MT_ERR_UNSUPPORTED_DTYPE = 2,  /* dtype combination not implemented          */
  MT_ERR_UNSUPPORTED_LAYOUT = 3, /* stride or alignment the kernel cannot take */
  MT_ERR_UNSUPPORTED_ARCH = 4,   /* device is not sm_100                       */
  MT_ERR_LAUNCH = 5,             /* CUDA launch / runtime error                */
  MT_ERR_DEVICE_TIMEOUT = 6,     /* a bounded device-side wait gave up         */
  MT_ERR_WORKSPACE = 7,          /* workspace pointer null or too small        */
  MT_ERR_TENSOR_MAP = 8          /* cuTensorMapEncodeTiled rejected a layout   */
};

/* Human-readable text for a status code (static storage). */
MT_API const char* mt_status_string(int status);

/* Library version, and the compute capability the library was built for (100). */
MT_API int mt_version(void);
MT_API int mt_built_arch(void);

/* Last CUDA error text seen by the library on this host thread (static storage). */
MT_API const char* mt_last_error(void);

/*
 * Device status word.  The tcgen05 kernels take a pointer to one uint32 in
 * device memory (caller-owned, zero-initialised).  A bounded wait that gives
 * up writes a nonzero code there and the kernel returns early instead of
 * hanging.  The host reads it back with an ordinary copy.
 *   bit layout: (kernel_id << 16) | wait_site
 */

/* Test hook for the bounded waits (no counterpart in the reference).  Launches
 * one small kernel that allocates TMEM and waits on an mbarrier through the
 * same bounded wait the tcgen05 kernels use, with a limit of limit_cycles SM
 * clock cycles (1 .. 4e9).  complete = 0: nothing arrives, the wait gives up,
 * the kernel writes (15 << 16) | 1 to *status, frees its TMEM and returns;
 * complete = 1: the barrier completes and *status is left alone.  Blocks until
 * the kernel has finished (it synchronises the stream) and returns
 * MT_ERR_DEVICE_TIMEOUT when *status is nonzero afterwards.  *status must be
 * zero-initialised device memory. */
MT_API int mt_debug_wait_timeout(int64_t limit_cycles, int complete, uint32_t* status,
                                 void* stream);

/* Timing hook (no counterpart in the reference).  Two caller-owned CUDA
 * events (CUevent / cudaEvent_t handles, created by the caller) that the next
 * calls on this host thread record on their stream right before and right
 * after their main kernel (the tcgen05 attention kernels), so a caller can time
 * that kernel alone inside a multi-kernel operator.  Both NULL disables it. */
MT_API int mt_set_timing_events(void* before_main, void* after_main);

/* Launch counter (no counterpart in the reference): the number of kernels this
 * library has launched successfully in the process so far, over all devices
 * and host threads.  A caller takes the difference around a region to count
 * the library's kernels in it. */
MT_API int64_t mt_launch_count(void);

/* ---------------------------------------------------------------------
 * RMSNorm   replaces triton_rms_norm (src/mega_trading/kernels/triton_ops.py:11-15,
 *           forward kernel :528-538, backward :633-665 + torch sum :183)
 *   y[r, :] = x[r, :] * rstd[r] * w,   rstd[r] = rsqrt(mean(x[r, :]^2) + eps)
 * x, y: [rows, dim] contiguous; w: [dim]; rstd: [rows] fp32 (output).
 * Math in fp32 for every dtype.
 * ------------------------------------------------------------------- */
MT_API int mt_rms_norm_fwd(const void* x, int x_dtype, const void* w, int w_dtype,
                    void* y, int y_dtype, float* rstd, int64_t rows,
                    int64_t dim, float eps, void* stream);

/* Workspace (bytes) for mt_rms_norm_bwd / mt_add_rms_norm_bwd: fp32 per-block
 * partial sums of dW. */
MT_API int64_t mt_rms_norm_bwd_workspace_bytes(int64_t rows, int64_t dim);

/* dx = rstd * (dy*w - x * rstd^2 * mean(dy*w*x));  dw = sum_rows dy * x * rstd.
 * dx: [rows, dim] in dx_dtype; dw: [dim] in dw_dtype (fully written, not
 * accumulated). */
MT_API int mt_rms_norm_bwd(const void* x, int x_dtype, const void* w, int w_dtype,
                    const float* rstd, const void* dy, int dy_dtype, void* dx,
                    int dx_dtype, void* dw, int dw_dtype, void* workspace,
                    int64_t workspace_bytes, int64_t rows, int64_t dim,
                    void* stream);

/* RMSNorm backward for callers that cannot allocate device memory where they
 * call it.  No counterpart in the reference: it exists for hosts that bind this
 * C ABI without a device allocator of their own at the call site (an FFI
 * caller, or code running while another runtime owns the device memory
 * pool), and for code that must not call cudaMalloc/cudaFree in its step
 * because they synchronise the device.  Same math and arguments as
 * mt_rms_norm_bwd minus the workspace: the dW partials live in a 4 MiB
 * static device array inside the library (held by every GPU that loads it).
 * Limits: dim <= 4096 (larger returns MT_ERR_WORKSPACE).  The first call on a
 * device looks up the array's device address; make that first call before any
 * stream capture.  All calls on a device share the array and it keeps the
 * last call's contents (each call overwrites what it reads), so two calls that
 * can run at the same time on one device, e.g. on two streams, race: order
 * them on one stream. */
MT_API int mt_rms_norm_bwd_noalloc(const void* x, int x_dtype, const void* w, int w_dtype,
                                   const float* rstd, const void* dy, int dy_dtype, void* dx,
                                   int dx_dtype, void* dw, int dw_dtype, int64_t rows,
                                   int64_t dim, void* stream);

/* ---------------------------------------------------------------------
 * Fused residual add + RMSNorm   replaces triton_add_rms_norm
 *   (src/mega_trading/kernels/triton_ops.py:18-42, forward kernel :541-566,
 *    backward kernel :569-608 + torch sum :287)
 *   new_residual = hidden + residual;  normed = RMSNorm(new_residual)
 * All activations share one dtype (act_dtype); w has w_dtype.
 * ------------------------------------------------------------------- */
MT_API int mt_add_rms_norm_fwd(const void* hidden, const void* residual, int act_dtype,
                        const void* w, int w_dtype, void* new_residual,
                        int res_dtype, void* normed, int normed_dtype,
                        float* rstd, int64_t rows, int64_t dim, float eps,
                        void* stream);

/* grad_input = grad_new_residual + dNorm(grad_normed);  the reference returns
 * the same tensor for hidden and residual (triton_ops.py:291). */
MT_API int mt_add_rms_norm_bwd(const void* new_residual, int res_dtype, const void* w,
                        int w_dtype, const float* rstd,
                        const void* grad_new_residual, int gres_dtype,
                        const void* grad_normed, int gnorm_dtype,
                        void* grad_input, int gin_dtype, void* dw, int dw_dtype,
                        void* workspace, int64_t workspace_bytes, int64_t rows,
                        int64_t dim, void* stream);

/* mt_add_rms_norm_bwd that also writes grad_input rounded to gnorm_dtype into
 * grad_branch ([rows, dim]).  For a wide residual stream (fp32 new_residual and
 * grad_input) feeding a narrower branch (bf16 hidden): both add inputs take the
 * same gradient, one per dtype, from one pass.  No counterpart kernel in the
 * reference, where autocast casts the shared gradient in a separate op
 * (residual adds of src/mega_trading/model.py:185-186 under the autocast of
 * trainer.py:336). */
MT_API int mt_add_rms_norm_bwd_dual(const void* new_residual, int res_dtype, const void* w,
                             int w_dtype, const float* rstd,
                             const void* grad_new_residual, int gres_dtype,
                             const void* grad_normed, int gnorm_dtype,
                             void* grad_input, int gin_dtype, void* grad_branch,
                             void* dw, int dw_dtype, void* workspace,
                             int64_t workspace_bytes, int64_t rows, int64_t dim,
                             void* stream);

/* ---------------------------------------------------------------------
 * RoPE (interleaved pairs)   replaces triton_apply_rope
 *   (src/mega_trading/kernels/triton_ops.py:45-54, _launch_rope_kernel
 *    :477-525, _rope_kernel :690-761)
 *   out[2i]   = x[2i]*cos[t,i] - x[2i+1]*sin[t,i]
 *   out[2i+1] = x[2i]*sin[t,i] + x[2i+1]*cos[t,i]
 * Backward is the same call with negate_sin = 1.
 * q: [B, Hq, T, D], k: [B, Hk, T, D] with arbitrary element strides
 * (qs[4], ks[4], qos[4], kos[4] = strides of q, k, q_out, k_out in elements);
 * cos/sin: [T, D/2] with strides cs[2], ss[2].  One dtype for all tensors.
 * ------------------------------------------------------------------- */
MT_API int mt_rope(const void* q, const void* k, const void* cos, const void* sin,
            void* q_out, void* k_out, int dtype, int64_t B, int64_t Hq,
            int64_t Hk, int64_t T, int64_t D, const int64_t* qs,
            const int64_t* ks, const int64_t* qos, const int64_t* kos,
            const int64_t* cs, const int64_t* ss, int negate_sin, void* stream);

/* ---------------------------------------------------------------------
 * SwiGLU gate   replaces triton_swiglu_gate
 *   (src/mega_trading/kernels/triton_ops.py:57-61, forward :774-782,
 *    backward :799-819)
 *   y = silu(g) * u, silu evaluated in fp32 and rounded to u's dtype first.
 * g, u, y: n contiguous elements.
 * ------------------------------------------------------------------- */
MT_API int mt_swiglu_fwd(const void* g, const void* u, void* y, int dtype, int64_t n,
                  void* stream);
MT_API int mt_swiglu_bwd(const void* g, const void* u, const void* dy, void* dg,
                  void* du, int dtype, int64_t n, void* stream);

/* Packed variant for a single GEMM against concatenated [w1; w3] weights:
 * gu is [rows, 2*inter] = [gate | up] per row, y is [rows, inter]; the
 * backward writes the packed gradient dgu [rows, 2*inter].  bf16/fp16,
 * inter % 8 == 0.  Same math as mt_swiglu_fwd / mt_swiglu_bwd. */
MT_API int mt_swiglu_packed_fwd(const void* gu, void* y, int dtype, int64_t rows,
                                int64_t inter, void* stream);
MT_API int mt_swiglu_packed_bwd(const void* gu, const void* dy, void* dgu, int dtype,
                                int64_t rows, int64_t inter, void* stream);

/* ---------------------------------------------------------------------
 * Causal GQA flash attention (tcgen05 + TMEM + TMA)   replaces triton_attention
 *   (src/mega_trading/kernels/triton_attention.py:12-24, forward :27-78 and
 *    kernels :260-478, backward :80-111 and :134-245, :481-747)
 * q/o: [B, Hq, T, D], k/v: [B, Hkv, T, D], Hq = Hkv * repeats, element
 * strides qs[4] etc. (innermost stride must be 1, other strides multiples of
 * 8 elements), D in {32, 64}, dtype bf16 or fp16.
 * lse: [B, Hq, T] fp32 contiguous (natural-log logsumexp of scaled scores).
 * scale: softmax scale (1/sqrt(D) in the reference).
 * workspace: device scratch of mt_attention_fwd_workspace_bytes() bytes.
 * status: device uint32 (see above).
 * ------------------------------------------------------------------- */
MT_API int mt_attention_fwd(const void* q, const void* k, const void* v, void* o,
                     float* lse, int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                     int64_t T, int64_t D, const int64_t* qs, const int64_t* ks,
                     const int64_t* vs, const int64_t* os, float scale,
                     void* workspace, int64_t workspace_bytes,
                     uint32_t* status, void* stream);

/* Workspace for the forward (16-byte aligned): the persistent kernel's work
 * counter, zeroed on the stream by every call.  One call at a time per
 * workspace. */
MT_API int64_t mt_attention_fwd_workspace_bytes(int64_t B, int64_t Hq, int64_t T,
                                                int64_t D);

/* Workspace for the backward: fp32 delta and -lse*log2(e) [B*Hq*Tp], fp32 dQ
 * accumulator [B*Hq*Tp*D] and the persistent kernel's work counter,
 * Tp = T rounded up to 128. */
MT_API int64_t mt_attention_bwd_workspace_bytes(int64_t B, int64_t Hq, int64_t T,
                                         int64_t D);

MT_API int mt_attention_bwd(const void* q, const void* k, const void* v,
                     const void* o, const float* lse, const void* dout,
                     void* dq, void* dk, void* dv, int dtype, int64_t B,
                     int64_t Hq, int64_t Hkv, int64_t T, int64_t D,
                     const int64_t* qs, const int64_t* ks, const int64_t* vs,
                     const int64_t* os, const int64_t* dos, const int64_t* dqs,
                     const int64_t* dks, const int64_t* dvs, float scale,
                     void* workspace, int64_t workspace_bytes, uint32_t* status,
                     void* stream);

/* mt_attention_bwd with the RoPE backward folded in: q and k are the ROTATED
 * query/key the forward consumed, and dq / dk come back as the gradients of
 * the un-rotated query/key (interleaved-pair RoPE of
 * src/mega_trading/model.py:286-316, run backwards).  Each dq / dk row is
 * rotated by -theta(t) in fp32 before its one rounding, so no rotated-gradient
 * tensor is written.  rope_cos / rope_sin: [T, D/2] tables in dtype with row
 * stride rope_ld (a multiple of 4 elements, pointers 8-byte aligned).  No
 * counterpart entry in the reference, which runs triton_apply_rope's backward
 * as a separate kernel (kernels/triton_ops.py:187-214). */
MT_API int mt_attention_rope_bwd(const void* q, const void* k, const void* v,
                          const void* o, const float* lse, const void* dout,
                          void* dq, void* dk, void* dv, int dtype, int64_t B,
                          int64_t Hq, int64_t Hkv, int64_t T, int64_t D,
                          const int64_t* qs, const int64_t* ks, const int64_t* vs,
                          const int64_t* os, const int64_t* dos, const int64_t* dqs,
                          const int64_t* dks, const int64_t* dvs, float scale,
                          const void* rope_cos, const void* rope_sin, int64_t rope_ld,
                          void* workspace, int64_t workspace_bytes, uint32_t* status,
                          void* stream);


/* ---------------------------------------------------------------------
 * SwiGLU MLP GEMMs   replace the w1 / w3 projections + triton_swiglu_gate
 *   forward and the w2 input-gradient GEMM + gate backward of SwiGLU
 *   (src/mega_trading/model.py:249-256; kernels/triton_ops.py:57-61,
 *   forward :774-782, backward :799-819).  tcgen05 GEMMs with the gate in
 *   the epilogue; no counterpart kernel in the reference.
 * Layout: the gate/up weight w13 [2I, K] and the saved activation gu [M, 2I]
 *   are interleaved in blocks of 128: rows (columns) 256b .. 256b+127 hold
 *   w1 (gate) block b, 256b+128 .. 256b+255 hold w3 (up) block b.
 * Forward:  gu = round(x w13^T);  y = round(round(silu(g)) * u)   [M, I].
 * Backward: dy = round(dout w2)   (w2t = w2^T [I, H], dout [M, H]);
 *           dgate = dy u s (1 + g (1 - s)), dup = dy round(g s), s = sigmoid(g),
 *           written to dgu [M, 2I] in the interleaved layout.
 * I must be a multiple of 256, K (H) a multiple of 8; 16-bit dtypes; all
 * tensors contiguous row-major, 16-byte aligned.
 * ------------------------------------------------------------------- */
MT_API int mt_swiglu_gemm_fwd(const void* x, const void* w13, void* gu, void* y,
                       int dtype, int64_t M, int64_t K, int64_t I,
                       uint32_t* status, void* stream);
MT_API int mt_swiglu_gemm_bwd(const void* dout, const void* w2t, const void* gu,
                       void* dgu, int dtype, int64_t M, int64_t H, int64_t I,
                       uint32_t* status, void* stream);

/* ---------------------------------------------------------------------
 * QKV projection + RoPE   replaces the q/k/v projections and
 *   RotaryEmbedding / triton_apply_rope forward of LlamaAttention
 *   (src/mega_trading/model.py:218-226, 286-294; kernels/triton_ops.py:45-54).
 *   tcgen05 GEMM qkv = round(x w^T) whose epilogue rotates the first
 *   rot_cols columns (the q and k heads) of each row by the RoPE tables at
 *   position t = row % seq: interleaved pairs (e c - o s, e s + o c), tables
 *   rope_cos / rope_sin [seq, head_dim/2] in dtype with row stride rope_ld
 *   (a multiple of 8).  x [M, K], w [N, K], qkv [M, N] row-major; M a
 *   multiple of seq, N a multiple of 256, head_dim 32 or 64, rot_cols a
 *   multiple of head_dim.  No counterpart kernel in the reference.
 * ------------------------------------------------------------------- */
MT_API int mt_qkv_rope_gemm(const void* x, const void* w, void* qkv,
                     const void* rope_cos, const void* rope_sin, int64_t rope_ld,
                     int dtype, int64_t M, int64_t K, int64_t N, int64_t rot_cols,
                     int64_t seq, int64_t head_dim, uint32_t* status,
                     void* stream);

/* ---------------------------------------------------------------------
 * Fused linear + cross-entropy   replaces triton_fused_linear_cross_entropy
 *   (src/mega_trading/kernels/triton_ops.py:64-92, :294-411, row kernel
 *    :822-887; torch path :99-112)
 * hidden: [N, K] and weight: [V, K], contiguous, bf16 or fp16, K % 8 == 0;
 * labels: [N] int64 (labels_i64 = 1) or int32; rows whose label equals
 * ignore_index contribute no loss and no gradient.
 *
 * Forward: loss = mean over valid rows of (logsumexp(hidden W^T) - z_label),
 * 0 when no row is valid.  The logits live only in TMEM/registers.
 * lse2_out (optional): [N + 3] fp32 = per-row logsumexp in log2 units followed
 * by {loss, n_valid, 1/n_valid}; it is the input of the backward.
 * ------------------------------------------------------------------- */
MT_API int64_t mt_fused_ce_workspace_bytes(int64_t N, int64_t V);
MT_API int mt_fused_ce_fwd(const void* hidden, const void* weight, const void* labels,
                           int labels_i64, int64_t ignore_index, int dtype, int64_t N,
                           int64_t V, int64_t K, float* loss, float* lse2_out,
                           void* workspace, int64_t workspace_bytes, uint32_t* status,
                           void* stream);

/* Backward: dhidden = dZ W  [N, K]  and  dweight = dZ^T hidden  [V, K] with
 *   dZ = (softmax(hidden W^T) - onehot(label)) * grad_out / n_valid
 * (rows with an ignored or out-of-range label contribute nothing), the
 * gradients the reference computes chunk by chunk with two library GEMMs over
 * a materialised logits chunk (kernels/triton_ops.py:359-389).  Here the
 * logit tiles are recomputed on chip, rounded to dtype and multiplied out of
 * shared memory: dZ never reaches global memory and the products accumulate
 * in fp32 (TMEM).  lse2_scal: the forward's lse2_out; grad_out: device fp32
 * scalar.  dhidden / dweight: contiguous, written completely in dh_dtype /
 * dw_dtype (MT_F32, MT_BF16 or MT_F16); either may be NULL to skip it.
 * workspace: mt_fused_ce_bwd_workspace_bytes(N, V, K) bytes, 256-byte aligned. */
MT_API int64_t mt_fused_ce_bwd_workspace_bytes(int64_t N, int64_t V, int64_t K);
MT_API int mt_fused_ce_bwd(const void* hidden, const void* weight, const void* labels,
                           int labels_i64, int64_t ignore_index, int dtype, int64_t N,
                           int64_t V, int64_t K, const float* lse2_scal, const float* grad_out,
                           void* dhidden, int dh_dtype, void* dweight, int dw_dtype,
                           void* workspace, int64_t workspace_bytes, uint32_t* status,
                           void* stream);

/* ---------------------------------------------------------------------
 * Fused AdamW with 16-bit weight copies   replaces torch.optim.AdamW(fused=True)
 *   (src/mega_trading/trainer.py:535-545) plus the per-forward bf16 weight
 *   casts of the reference's autocast (trainer.py:336); no counterpart kernel
 *   in the reference.
 * One launch updates every tensor of the table (decoupled weight decay,
 * bias-corrected moments, torch.optim.AdamW semantics):
 *   p -= lr*wd*p ; m = b1*m + (1-b1)*g ; v = b2*v + (1-b2)*g*g ;
 *   p -= step_size * m / (sqrt(v) / bias_correction2_sqrt + eps)
 * with step_size = lr / (1 - b1^t), bias_correction2_sqrt = sqrt(1 - b2^t)
 * computed by the caller for the tensors' common step t.  skip_if_set: NULL,
 * or a device status word (see above); when it holds a nonzero code at launch
 * time the kernel changes nothing, so a step whose kernels gave up on a wait
 * (partial gradients) never reaches the weights.  Then, when shadow is
 * not NULL, the updated value rounded to shadow_dtype (bf16 or fp16) is
 * stored at shadow[(j / shadow_block) * shadow_stride + j % shadow_block] for
 * element j: shadow_block = numel for a contiguous copy; a copy interleaved
 * with other tensors in blocks of rows uses the block size and the distance
 * between its blocks (shadow_block < 2^32).
 * tensors: DEVICE array of n_tensors entries sorted by offset, offsets the
 * prefix sums of numel (offset[0] = 0); total = sum of numel.  All fp32
 * pointers distinct per tensor.
 * ------------------------------------------------------------------- */
typedef struct MtAdamWTensor {
  float* param;          /* fp32 master weights, updated in place */
  const float* grad;     /* fp32 gradient                          */
  float* exp_avg;        /* fp32 first moment                      */
  float* exp_avg_sq;     /* fp32 second moment                     */
  void* shadow;          /* 16-bit copy of the updated weights, or NULL */
  int64_t numel;
  int64_t shadow_block;
  int64_t shadow_stride;
  int64_t offset;        /* first index of this tensor in the flattened space */
} MtAdamWTensor;

MT_API int mt_adamw_step(const MtAdamWTensor* tensors, int n_tensors, int64_t total,
                         int shadow_dtype, float lr, float beta1, float beta2, float eps,
                         float weight_decay, float step_size, float bias_correction2_sqrt,
                         const uint32_t* skip_if_set, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MT_B200_H */
