/*
 * soupb200.h — C ABI of the B200 (sm_100a) fused QLoRA ops.
 *
 * Every entry point takes plain device pointers, element counts and strides
 * (in elements), a dtype code and a cudaStream_t (passed as void*), launches
 * asynchronously on that stream and returns a status code. Nothing allocates:
 * outputs and scratch buffers are the caller's. No entry point synchronises
 * the stream.
 *
 * The reference (Python + Triton) exposes these ops through its autograd
 * Functions; each declaration below names the reference interface it
 * replaces (paths relative to the reference project root).
 */
#ifndef SOUPB200_H
#define SOUPB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define SOUP_OK 0
#define SOUP_ERR_INVALID 1      /* bad pointer, size, stride or dtype            */
#define SOUP_ERR_UNSUPPORTED 2  /* valid but not handled (alignment, dtype mix)  */
#define SOUP_ERR_CUDA 3         /* a CUDA runtime call or launch failed          */
#define SOUP_ERR_WORKSPACE 4    /* workspace too small                           */
#define SOUP_ERR_DEVICE 5       /* a device-side bounded wait timed out          */

/* ---- dtype codes --------------------------------------------------------- */
#define SOUP_F32 0
#define SOUP_F16 1
#define SOUP_BF16 2

/* Library version and the last CUDA error text seen by this thread. */
int soup_version(void);
const char* soup_last_error(void);

/* Device error word written by bounded waits in the GEMM kernels (0 = none).
 * Reads and clears it in one atomic step on the device (a code written
 * meanwhile by a kernel on another stream stays for the next read), then
 * synchronises the given stream. Codes: 0x101 producer, 0x102 MMA issuer,
 * 0x103 epilogue wait expired, 0x104 a stream-K partial never became
 * ready. No counterpart in the reference (its Triton kernels have no
 * device-side waits). */
int soup_device_error(void* stream, int* out_code);

/* Time limit of every mbarrier wait inside the GEMM kernels launched after
 * this call (all devices): 0 restores the default of 2 s; otherwise at least
 * 1 ms. A wait that expires records its code in the device error word, the
 * kernel drains its copies and MMAs (each drain wait bounded by the same
 * limit), frees its TMEM and returns. No counterpart in the reference. */
int soup_set_wait_limit_ns(uint64_t ns);

/* ---- RMSNorm -------------------------------------------------------------
 * Replaces solution/kernels/rmsnorm.py:22-57 (_rms_norm_fwd_kernel) and the
 * launch in FastRMSNormFunction.forward (rmsnorm.py:102-134).
 * x, y: [rows, cols] with row strides; weight: [cols]; rstd: [rows] fp32 out.
 * y = (x * rstd) * w, rstd = 1/sqrt(mean(x^2) + eps), fp32 math. */
int soup_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight, void* y,
                     int64_t y_row_stride, float* rstd, int64_t rows, int64_t cols, float eps,
                     int x_dtype, int w_dtype, void* stream);

/* Replaces solution/kernels/rmsnorm.py:60-96 (_rms_norm_bwd_dx_kernel) and
 * the eager dw reduction at rmsnorm.py:161-167, fused into one launch.
 * dx = rstd*(dy*w - (x/cols)*rstd^2*sum(dy*w*x)); dw = sum_rows dy*x*rstd.
 * dw may be NULL (weight frozen). When dw is given, workspace must hold
 * soup_rmsnorm_bwd_workspace_bytes(rows, cols) bytes; the dw reduction is
 * deterministic (fixed-order per-block partials, no data atomics). */
size_t soup_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t cols);
int soup_rmsnorm_bwd(const void* dy, int64_t dy_row_stride, const void* x, int64_t x_row_stride,
                     const void* weight, const float* rstd, void* dx, int64_t dx_row_stride,
                     void* dw, void* workspace, size_t workspace_bytes, int64_t rows,
                     int64_t cols, int x_dtype, int w_dtype, void* stream);

/* RMSNorm backward that allocates nothing. No counterpart in the reference:
 * it exists for callers that cannot give the library a scratch buffer, such as
 * code running under an allocator that already owns all device memory, or host
 * code that must avoid cudaMalloc because it can synchronise the device.
 * Same arguments and results as soup_rmsnorm_bwd without the workspace: the dw
 * partial rows go to a 4 MiB array built into the library (every GPU that
 * loads the library holds it until exit). The partials are one fp32 row of
 * `cols` per CTA, at most 3 CTAs per SM on the vector path (cols up to about
 * 2360 on a 148-SM B200, e.g. hidden sizes 1536 and 2048); calls needing more
 * than 4 MiB return SOUP_ERR_WORKSPACE. The first call on a device looks up the array's device
 * address (under a lock, so first calls from several host threads are safe) and
 * keeps it for the life of the process; make that first call before any stream
 * capture, and do not call this entry point again on a device after a
 * cudaDeviceReset of it (the kept address would be stale). All calls share
 * the array, so calls whose kernels overlap on the GPU (other streams, other
 * host threads) race: serialise them. */
int soup_rmsnorm_bwd_noalloc(const void* dy, int64_t dy_row_stride, const void* x,
                             int64_t x_row_stride, const void* weight, const float* rstd,
                             void* dx, int64_t dx_row_stride, void* dw, int64_t rows,
                             int64_t cols, int x_dtype, int w_dtype, void* stream);

/* ---- SwiGLU --------------------------------------------------------------
 * Replaces solution/kernels/swiglu.py:20-50 (_custom_swiglu_fwd_kernel).
 * out = g*sigmoid(g)*u on [rows, cols] with independent row strides. */
int soup_swiglu_fwd(const void* gate, int64_t gate_row_stride, const void* up,
                    int64_t up_row_stride, void* out, int64_t out_row_stride, int64_t rows,
                    int64_t cols, int dtype, void* stream);

/* Replaces solution/kernels/swiglu.py:53-95 (_custom_swiglu_bwd_kernel);
 * sigmoid is recomputed from gate. dgate/dup may alias gate/up (in place). */
int soup_swiglu_bwd(const void* dy, int64_t dy_row_stride, const void* gate,
                    int64_t gate_row_stride, const void* up, int64_t up_row_stride, void* dgate,
                    int64_t dgate_row_stride, void* dup, int64_t dup_row_stride, int64_t rows,
                    int64_t cols, int dtype, void* stream);

/* ---- RoPE (rotate-half) ----------------------------------------------------
 * Replaces solution/kernels/rope.py:20-67 (_fused_rope_2d_fwd_kernel) and the
 * two launches of patch_qwen2_rope (rope.py:217-218): Q and K in one launch.
 * Tensors are [B, H, S, D] with strides {b, h, s} (last dim contiguous);
 * cos/sin are indexed [b*cos_sb + s*cos_ss + d] for d < D/2 (the reference
 * reads the first half only). k/k_out may be NULL with hk = 0. inverse != 0
 * applies the transpose rotation (backward, rope.py:70-117). */
int soup_rope(const void* q, const int64_t* q_strides, void* q_out, const int64_t* q_out_strides,
              int64_t hq, const void* k, const int64_t* k_strides, void* k_out,
              const int64_t* k_out_strides, int64_t hk, const void* cos, const void* sin,
              int64_t cos_sb, int64_t cos_ss, int64_t batch, int64_t seq, int64_t head_dim,
              int dtype, int cos_dtype, int inverse, void* stream);

/* ---- Cross-entropy on a logits buffer ------------------------------------
 * Replaces solution/kernels/chunked_ce.py:32-128
 * (_chunked_cross_entropy_fused_kernel): per-row loss, entropy, top-1 hit,
 * and (write_grad != 0) the in-place overwrite of the logits with
 * (softmax - onehot)/denominator (0 for ignored rows). */
int soup_ce_rows(void* logits, int64_t row_stride, const int64_t* targets, float* losses,
                 float* entropies, int32_t* correct, int64_t rows, int64_t vocab,
                 float denominator, int64_t ignore_index, int dtype, int write_grad,
                 void* stream);

/* ---- Fused lm_head cross-entropy (tcgen05 GEMMs) -------------------------
 * Replaces chunk_cross_entropy_triton (chunked_ce.py:183-264) driven by
 * TritonChunkedHeadLoss.forward (chunked_ce.py:271-304): the logits GEMM with
 * an online-softmax epilogue, the per-row metrics, the logits' gradient (kept
 * factored: per-row factors times the stored exponentials exp(z - c_row), no
 * [rows, vocab] pass between the GEMMs), the input gradient and (new, no
 * reference counterpart) the lm_head gradient.
 * hidden [rows, dim] (row stride h_ld) and weight [vocab, dim] (row stride
 * w_ld) are both in_dtype: BF16, or F16 (the reference's own operand type: it
 * rounds the chunk and a cached copy of W to fp16 for its GEMMs,
 * chunked_ce.py:170-180,196-199); fp32 accumulation either way. The logits'
 * gradient is kept in bf16, so with F16 operands the dX GEMM reads weight_bwd,
 * a bf16 copy of the weight [vocab, dim] (row stride wb_ld); with BF16 it is
 * ignored (may be NULL). targets [rows] int64.
 * Outputs: losses/entropies [rows] fp32, correct [rows] int32,
 * sums[2] fp32 = {sum of losses, sum of hits} (may be NULL),
 * dhidden [rows, dim] in dh_dtype F32 or BF16 (NULL: no input gradient),
 * dweight [vocab, dim] (NULL: no lm_head gradient; dtype dw_dtype F32 or
 * BF16; accumulate_dw != 0 adds to its contents). Gradients are scaled by
 * 1/denominator (the caller's grad_output scale is applied outside).
 * workspace: see soup_ce_linear_workspace_bytes. */
size_t soup_ce_linear_workspace_bytes(int64_t rows, int64_t vocab, int64_t dim);
int soup_ce_linear(const void* hidden, int64_t h_ld, const void* weight, int64_t w_ld, int in_dtype,
                   const void* weight_bwd, int64_t wb_ld, const int64_t* targets, int64_t rows,
                   int64_t vocab, int64_t dim, float denominator, int64_t ignore_index,
                   float* losses, float* entropies, int32_t* correct, float* sums, void* dhidden,
                   int dh_dtype, void* dweight, int dw_dtype, int accumulate_dw, void* workspace,
                   size_t workspace_bytes, void* stream);

/* The lm_head gradient from the state that a preceding soup_ce_linear call
 * with a non-NULL dhidden left in `workspace` (same rows/vocab/dim/hidden):
 * dweight (+)= grad_scale[0] * dL^T H, where grad_scale is an optional device
 * fp32 scalar (the upstream gradient of the loss; NULL = 1). The workspace
 * holds dL factored as diag(s) E (E = exp(logit - c_row) in bf16 with the
 * target entries corrected, s = exp(c_row - lse_row) / denominator per row);
 * this call scales the hidden rows by s into the workspace and runs one GEMM.
 * Lets an autograd backward apply its upstream gradient inside the GEMM
 * epilogue instead of in a separate pass over the [vocab, dim] gradient.
 * hidden has the in_dtype (BF16 or F16) given to soup_ce_linear.
 * Extends chunked_ce.py:307-311 (the reference's head is frozen and has no
 * gradient). */
int soup_ce_linear_dweight(void* workspace, size_t workspace_bytes, const void* hidden,
                           int64_t h_ld, int in_dtype, int64_t rows, int64_t vocab, int64_t dim,
                           const float* grad_scale, void* dweight, int dw_dtype, int accumulate_dw,
                           void* stream);

/* ---- Vocab-parallel fused CE (the lm_head rows sharded over ranks) -----------
 * No counterpart in the reference (single GPU only). A rank holding rows
 * [vocab_offset, vocab_offset + vocab_shard) of W runs:
 *   1. soup_ce_vp_forward: logits GEMM over its shard with the online-softmax
 *      epilogue; states[rows][5] = {max, sum exp, sum z*exp, global argmax
 *      (int32 bits), target logit or 0}; the shard's row-shifted exponentials
 *      exp(z - c_row) stay in workspace (c_row: the target logit when the
 *      target is in the shard, else the shard's first column, + a margin);
 *   2. (caller) all-gather the states of all ranks into states_all[nranks][rows][5];
 *   3. soup_ce_vp_combine: merges the ranks' states per row in rank order
 *      (argmax ties keep the smaller index): losses, entropies, correct, the
 *      global lse [rows] and optional sums[2];
 *   4. soup_ce_vp_backward: the per-row gradient factors from the global lse
 *      (the shard's buffer is not rewritten), this rank's partial dhidden =
 *      dL_shard W_shard (F32 or BF16) and its dW_shard = dL_shard^T H (local,
 *      no exchange);
 *   5. (caller) sum the partial dhidden over ranks (a reduce-scatter over
 *      token blocks, or an all-reduce).
 * hidden and the shard are in_dtype (BF16 or F16, as for soup_ce_linear);
 * with F16 the backward's dX GEMM reads weight_shard_bwd, a bf16 copy of the
 * shard (NULL with BF16).
 * Same row semantics as chunked_ce.py:46-128. */
size_t soup_ce_vp_workspace_bytes(int64_t rows, int64_t vocab_shard, int64_t dim);
int soup_ce_vp_forward(const void* hidden, int64_t h_ld, const void* weight_shard, int64_t w_ld,
                       int in_dtype, const int64_t* targets, int64_t rows, int64_t vocab_shard,
                       int64_t vocab_offset, int64_t dim, float* states, void* workspace,
                       size_t workspace_bytes, void* stream);
int soup_ce_vp_combine(const float* states_all, int nranks, const int64_t* targets, int64_t rows,
                       int64_t vocab_total, int64_t ignore_index, float* losses, float* entropies,
                       int32_t* correct, float* lse, float* sums, void* stream);
int soup_ce_vp_backward(void* workspace, size_t workspace_bytes, const void* hidden, int64_t h_ld,
                        const void* weight_shard, int64_t w_ld, int in_dtype,
                        const void* weight_shard_bwd, int64_t wb_ld, const int64_t* targets,
                        int64_t rows, int64_t vocab_shard, int64_t vocab_offset, int64_t dim,
                        const float* lse, float denominator, int64_t ignore_index,
                        void* dhidden_partial, int dh_dtype, void* dweight_shard, int dw_dtype,
                        int accumulate_dw, void* stream);

/* Stage timing for measurement: while set (n > 0), each soup_ce_linear call on
 * this host thread records events[i] on its stream after stage i:
 * 0 row shifts + logits GEMM, 1 row statistics (+ the gated fallback GEMM),
 * 2 sums, 3 dX GEMM, 4 dX reduce, 5 dW GEMM
 * (a stage that does not run records nothing). n = 0 clears. The events are
 * cudaEvent_t handles owned by the caller. */
int soup_set_stage_events(void** events, int n);

/* ---- Causal grouped-query flash attention (head dim 128, bf16) ---------------
 * No kernel in the reference: its Qwen2 attention is torch SDPA, called by
 * transformers' sdpa_attention_forward from Qwen2Attention.forward. q is
 * [batch, heads, seq, 128], k and v [batch, kv_heads, seq, 128] (heads a
 * multiple of kv_heads), each with element strides {b, h, s} (multiples of 8)
 * and a contiguous last dimension, 16-byte aligned. out = softmax(scale q k^T
 * [+ causal mask]) v as bf16 [batch, seq, heads, 128] (contiguous), lse =
 * log-sum-exp of the scaled logits per query, fp32 [batch, heads, S_pad] with
 * rows padded to S_pad = seq rounded up to 128 (the padding is not written). */
int soup_attention_fwd(const void* q, const int64_t* q_strides, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq,
                       int64_t head_dim, float scale, int causal, void* out, float* lse,
                       void* stream);

/* Backward of soup_attention_fwd: dq [batch, seq, heads, 128], dk and dv
 * [batch, seq, kv_heads, 128] (bf16, contiguous) from q, k, v (as given to the
 * forward), its out and lse, and dout = dL/d out ([batch, seq, heads, 128]
 * contiguous). P is recomputed from lse; dK / dV are accumulated per query
 * head in fp32 and summed over each KV head's group in a fixed order, dQ per
 * query tile over the key tiles (no atomics: reproducible). workspace: see
 * soup_attention_bwd_workspace_bytes (row dot products dout . out, the
 * log-sum-exp in base-2 units, and the fp32 per-head partials). */
size_t soup_attention_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq);
int soup_attention_bwd(const void* q, const int64_t* q_strides, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       const void* out, const void* dout, const float* lse, int64_t batch,
                       int64_t heads, int64_t kv_heads, int64_t seq, int64_t head_dim, float scale,
                       int causal, void* dq, void* dk, void* dv, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---- NF4 base weights for the QLoRA step ------------------------------------
 * No kernel in the reference: there the 4-bit base layers come from
 * bitsandbytes (Linear4bit, blocksize 64; harness/eval_adapter.py:26-28 loads
 * them). Blockwise absmax quantisation to the nearest of 16 code values
 * (code16: host array, sorted ascending, normalised to [-1, 1]); packed[n/2],
 * two 4-bit indices per byte, the earlier element in the high nibble;
 * absmax[n/64] fp32. Ties between two codes pick the lower index. */
int soup_nf4_quantize(const void* weight, int64_t n, int dtype, int blocksize, const float* code16,
                      uint8_t* packed, float* absmax, void* stream);
/* out[i] = code16[index_i] * absmax[i / 64] in dtype (16-byte aligned buffers). */
int soup_nf4_dequant(const uint8_t* packed, const float* absmax, int64_t n, int blocksize,
                     const float* code16, void* out, int dtype, void* stream);

/* ---- Stream-K scratch of the tcgen05 GEMMs (this device) -------------------
 * The pair GEMMs (every launch with one k split: the fused CE's logits and dW
 * products, the QLoRA step's GEMMs below) run their last, partial wave as
 * stream-K when the current device has a registered workspace and that
 * saves enough: the k blocks of the tiles that do not fill a whole wave of
 * CTA pairs are spread evenly over the pairs, and the pair holding a tile's
 * last k block adds the other parts' fp32 partials (in a fixed order;
 * results are reproducible) before the epilogue. Otherwise the tail runs as
 * a partial wave.
 * soup_gemm_stream_k_workspace_bytes: the size that covers every launch on
 * the current device. soup_gemm_set_stream_k_workspace: registers `ws`
 * (256-byte aligned, at least that size, zero-filled before the first
 * launch; the kernels leave it zero-filled) for later launches on the
 * current device, or none (NULL). Launches that use it must be ordered (one
 * stream, or streams that wait on each other): they share its slots. A
 * launch that ended with the device wait code 0x104 (soup_device_error) may
 * leave it non-zero; zero it again before the next launch. No counterpart
 * in the reference (its GEMMs are cuBLAS calls from PyTorch). */
size_t soup_gemm_stream_k_workspace_bytes(void);
int soup_gemm_set_stream_k_workspace(void* ws, size_t bytes);
/* A launch runs its tail as stream-K only if that shortens its longest
 * segment by at least `kblocks` k blocks of 64 against a whole tile (the
 * finishing pairs' waits and adds cost about 20 on B200); negative: the
 * default, 24. For tuning and tests; all devices, later launches. */
int soup_gemm_set_stream_k_min_saved(int kblocks);

/* ---- Plain tcgen05 GEMM (building block, exposed for tests) ---------------
 * C[m, n] = alpha * sum_k A(m, k) * B(n, k) (+ C if accumulate), bf16 inputs,
 * fp32 accumulation. a_mn_major = 0: A stored [M, K] (lda >= K); 1: stored
 * [K, M] (lda >= M). b_mn_major = 0: B stored [N, K]; 1: stored [K, N].
 * c_dtype F32 or BF16, C stored [M, N] with row stride ldc. */
int soup_gemm_bf16(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb,
                   int b_mn_major, void* c, int64_t ldc, int c_dtype, int64_t m, int64_t n,
                   int64_t k, float alpha, int accumulate, void* stream);

/* Diagnostic launch of the expiry path of the bounded waits: the same GEMM as
 * soup_gemm_bf16 (A [m, k] and B [n, k] K-major bf16, C [m, n] bf16, row
 * strides k, k, n) whose TMA producer withholds the second k-block of its
 * first tile, so the MMA issuer's wait for it can never be satisfied and
 * expires after wait_ns (1 ms .. 2 s). The kernel then records the code in the
 * device error word (read it with soup_device_error) and returns; C is left
 * partly unwritten. Requires k >= 128. Nothing in the fused ops calls it; it
 * exists so a test can show that an expired wait ends the kernel with an error
 * status and leaves the device usable. No counterpart in the reference. */
int soup_gemm_wait_expiry_check(const void* a, const void* b, void* c, int64_t m, int64_t n,
                                int64_t k, uint64_t wait_ns, void* stream);

/* ---- Base GEMM plus a rank-r update in the same accumulator (QLoRA linears) --
 * C[m, n] = alpha * (sum_k A(m,k) B(n,k) + sum_{j<r} A2(m,j) B2(n,j)) + bias[n]
 *           (+ C if accumulate).
 * A2 has A's majorness (a_mn_major = 0: stored [M, r], lda2 >= r; 1: stored
 * [r, M], lda2 >= M) and B2 has B's (b_mn_major = 0: stored [N, r]; 1: stored
 * [r, N]); the update is one or more extra 64-deep k-blocks of the same
 * tcgen05 GEMM, zero-filled beyond r, so y = x W^T + (x A^T)(s B)^T or
 * dx = dy W + (dy B)(s A) costs no pass over C of its own. r = 0: plain GEMM.
 * bias: optional bf16 [N] (NULL: none). All row strides 16-byte aligned.
 * No counterpart in the reference: there the LoRA linears are peft modules
 * over bitsandbytes 4-bit layers, each term its own GEMM. */
int soup_gemm_bf16_lora(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb,
                        int b_mn_major, const void* a2, int64_t lda2, const void* b2, int64_t ldb2,
                        int64_t r, const void* bias, void* c, int64_t ldc, int c_dtype, int64_t m,
                        int64_t n, int64_t k, float alpha, int accumulate, void* stream);

/* ---- Gate/up GEMM of a SwiGLU MLP with the activation in its epilogue ------
 * B = gate and up weights [2*inter, k] (K-major, bf16) with their rows
 * interleaved in blocks of 128: rows [256c, 256c+128) are gate rows
 * [128c, 128c+128) and the next 128 the same up rows; A = x [m, k]; the
 * optional rank-r segment (a2 [m, r], b2 [2*inter, r], same row order as B)
 * and bias ([2*inter], same order) as in soup_gemm_bf16_lora. Each 256-column
 * tile holds g and u for 128 intermediate columns; they are rounded to bf16
 * as a plain GEMM output would be, then
 *   mode 0: h = silu(g) * u -> h [m, inter] (row stride ldh); with y != NULL
 *           g and u also go to y [m, 2*inter] (row stride ldy, B's row order)
 *   mode 1: h holds dh [m, inter]; dg, du -> y [m, 2*inter] (B's row order)
 * with the arithmetic of soup_swiglu_fwd / soup_swiglu_bwd (bit-identical to
 * the unfused GEMM + SwiGLU kernels). inter % 128 == 0; rows 16-byte aligned.
 * Replaces the reference MLP's gate_proj / up_proj GEMMs plus its SwiGLU
 * kernels (solution/kernels/swiglu.py:20-95, 173-221), where the gate/up
 * outputs make a round trip through memory. */
int soup_gemm_bf16_lora_swiglu(const void* a, int64_t lda, const void* b, int64_t ldb,
                               const void* a2, int64_t lda2, const void* b2, int64_t ldb2, int64_t r,
                               const void* bias, int mode, void* h, int64_t ldh, void* y, int64_t ldy,
                               int64_t m, int64_t inter, int64_t k, void* stream);

/* The down projection's input gradient with the SwiGLU backward in its epilogue:
 * dh = a [m, k] b [k, inter] (+ a2 [m, r] b2 [r, inter]; b and b2 row-major, i.e.
 * the down weight [k, inter] and the scaled LoRA A [r, inter] as stored) is
 * rounded to bf16 as a plain GEMM output would be, and with g, u read from y
 * [m, 2*inter] (row stride ldy, the interleaved order of
 * soup_gemm_bf16_lora_swiglu's B rows) dg and du overwrite them in y: the
 * output of this call is [dg | du] in place of [g | u] (bit-identical to
 * soup_gemm_bf16_lora + soup_swiglu_bwd). inter % 128 == 0; rows 16-byte
 * aligned. Replaces the reference MLP's down_proj backward plus its SwiGLU
 * backward kernel (solution/kernels/swiglu.py:60-95, 197-214), where dh makes a
 * round trip through memory. */
int soup_gemm_bf16_lora_dswiglu(const void* a, int64_t lda, const void* b, int64_t ldb,
                                const void* a2, int64_t lda2, const void* b2, int64_t ldb2,
                                int64_t r, void* y, int64_t ldy, int64_t m, int64_t inter,
                                int64_t k, void* stream);

/* ---- Rank-r products of the LoRA linears (n <= 64) ---------------------------
 * C[m, n] = sum_k A(m, k) B(n, k) on the tensor cores, fp32 accumulation.
 * A: a_mn_major = 0 stored [m, k] (lda >= k), 1 stored [k, m] (lda >= m);
 * B: stored [n, k] (ldb >= k); bf16, rows 16-byte aligned. Outputs, any of:
 *   c  != NULL: c[i * ldc + j]  = bf16(alpha * C[i, j])
 *   ct != NULL: ct[j * ldct + i] = bf16(alpha * C[i, j])   (the transpose)
 *   g  != NULL: fp32 g[i * ldg + j] += alpha * C[i, j]
 *               (g_transposed: g[j * ldg + i] += alpha * C[i, j])
 * The four products of a LoRA linear y = x W^T + s (x A^T) B^T are
 *   xa = x (sA)^T (a = x, b = sA; ct = xa^T for gB), dxa = dy B (a = dy,
 *   b = B^T; ct = dxa^T for gA), gA += s dxa^T x (a = x MN-major, b = dxa^T,
 *   g = A.grad transposed), gB += dy^T xa (a = dy MN-major, b = xa^T, g = B.grad).
 * Deterministic (fixed summation order). No counterpart in the reference:
 * there these are four GEMMs of peft's LoRA Linear (lora_A, lora_B and their
 * autograd) over the bitsandbytes 4-bit base layer. */
int soup_lora_rank_gemm(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb,
                        int64_t m, int64_t n, int64_t k, void* c, int64_t ldc, void* ct, int64_t ldct,
                        float* g, int64_t ldg, int g_transposed, float alpha, void* stream);

/* gB of the members of a projection group in one pass over dy: C = dy^T xa with
 * a = dy stored [k = tokens, m = the group's output rows] (MN-major) and
 * b = xa^T [n = stacked rank, k]; member j (0 <= j < nmem <= 4) owns rows
 * [row_off[j], row_off[j+1]) of C (interleaved != 0: 128-row blocks taken in
 * turn, block t belonging to member t % nmem, each member's rows a multiple of
 * 128) and rank columns [col_off[j], col_off[j+1]), and receives
 * g[j][local row * ldg[j] + col - col_off[j]] += alpha * C[row, col]. */
int soup_lora_rank_grad_group(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                              int64_t k, int nmem, int interleaved, const int64_t* row_off,
                              const int64_t* col_off, float* const* g, const int64_t* ldg, float alpha,
                              void* stream);

/* Both rank products of one LoRA output gradient dy [m, n] in one pass over it
 * (no reference counterpart; replaces peft's two products through cuBLAS,
 * dxa = dy B and gB = dy^T xa, for the wide gate/up gradient):
 *   dxa [m, r] bf16 = dy bt^T     bt = B^T [r, n] (row stride ldbt)
 *   g   [n, r] fp32 = dy^T xt^T   xt = xa^T [r, m] (row stride ldxt), written (not added)
 * r <= 64. Each 128 x 128 tile of dy is loaded once and feeds both tcgen05
 * products; fp32 partials of each CTA block go to `workspace` (at least
 * soup_lora_rank_dual_workspace_bytes(m, n, r), 16-byte aligned) and a second
 * kernel sums them in a fixed order. */
size_t soup_lora_rank_dual_workspace_bytes(int64_t m, int64_t n, int64_t r);
int soup_lora_rank_dual(const void* dy, int64_t lddy, const void* bt, int64_t ldbt, const void* xt,
                        int64_t ldxt, int64_t m, int64_t n, int64_t r, void* dxa, int64_t lddxa, float* g,
                        int64_t ldg, void* workspace, size_t workspace_bytes, void* stream);

/* ---- AdamW over flat fp32 buffers (the QLoRA step's optimiser) ------------
 * One pass over n elements: param, exp_avg, exp_avg_sq updated in place from
 * grad with torch.optim.AdamW's decoupled weight decay; `step` is a device
 * fp32 scalar holding the step count t including this update (so the call can
 * be recorded in a CUDA graph). With param16 != NULL (BF16 or F16) the updated
 * parameters are also written in 16 bits, the first n_scaled of them
 * multiplied by `scale`. Replaces the reference trainer's optimiser step (HF
 * Trainer AdamW over the peft LoRA parameters; `soup train` with
 * task/task.yaml:10-22); the reference has no kernel of its own for it. */
int soup_adamw_flat(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n,
                    const float* step, float lr, float beta1, float beta2, float eps,
                    float weight_decay, void* param16, int param16_dtype, int64_t n_scaled,
                    float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SOUPB200_H */
