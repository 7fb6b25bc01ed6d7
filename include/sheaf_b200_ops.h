/* sheaf_b200 kernel-library entry points (C ABI).
 *
 * Each entry point runs one fused op of Sheaf's compiled fwd+VJP graphs on
 * caller-owned device memory, asynchronously on the caller's CUDA stream
 * (`stream` is a cudaStream_t; NULL = the legacy default stream). They are
 * the building blocks the module executor (sheaf_b200.h) schedules, exported
 * so the primitive-op sweep and the parity tests can drive one kernel at a
 * time. All return 0 on success and a non-zero SB_OPERR_* code otherwise.
 *
 * Element types use the IREE HAL element-type codes that Sheaf's runtime
 * passes today (sheaf/src/runtime/iree_ffi.rs:32-36).
 */
#ifndef SHEAF_B200_OPS_H_
#define SHEAF_B200_OPS_H_

#include <stddef.h>
#include <stdint.h>

#ifndef SB_API
#define SB_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SB_ELEM_F16 0x21000010u
#define SB_ELEM_F32 0x21000020u
#define SB_ELEM_BF16 0x22000010u
#define SB_ELEM_I32 0x10000020u

#define SB_OPERR_ARGS 1        /* bad shape, null pointer or unsupported dtype */
#define SB_OPERR_TMA 2         /* operand not 16-byte aligned for TMA */
#define SB_OPERR_LAUNCH 4      /* kernel launch failed */
#define SB_OPERR_WORKSPACE 5   /* workspace missing or too small */
#define SB_OPERR_SCRATCH 6     /* size beyond a fixed built-in scratch array */

/* C[M,N] = op(A) @ op(B), fp32 accumulation.
 * Replaces `stablehlo.dot_general` with contracting_dims = [1] x [0]
 * (sheaf/src/lowering/stablehlo/dot_ops.rs:32-79) and, through trans_a /
 * trans_b, the swapaxes operands of the `@` VJP
 * (sheaf/src/autodiff/reverse.rs:585-689).
 *   elem    : SB_ELEM_BF16 (tcgen05 tensor cores) or SB_ELEM_F32 (CUDA cores)
 *   trans_a : 0 -> A stored [M,K] row-major (row stride lda);
 *             1 -> A stored [K,M] (op(A) = A^T)
 *   trans_b : 0 -> B stored [K,N]; 1 -> B stored [N,K] (op(B) = B^T)
 *   c_elem  : SB_ELEM_F32 or SB_ELEM_BF16 output (ldc = row stride)
 *   workspace: fp32 scratch for split-K partials, at least
 *             sb_op_matmul_workspace_size(...) bytes (may be NULL when 0). */
SB_API int sb_op_matmul(uint32_t elem, const void* a, int64_t lda, int trans_a, const void* b, int64_t ldb, int trans_b,
                 int32_t m, int32_t n, int32_t k, void* c, int64_t ldc, uint32_t c_elem, void* workspace,
                 size_t workspace_bytes, void* stream);
SB_API size_t sb_op_matmul_workspace_size(uint32_t elem, int trans_a, int trans_b, int32_t m, int32_t n, int32_t k);
/* The matmul fused with the MLP activation, as the nanoGPT plan runs the fc
 * layer: u = A @ B^T (B stored [N,K]) rounded to the element type, then
 * y = gelu(u) and dy = gelu'(u) in the epilogue (lib/nn.shf:10-11 and its
 * derivative through the tanh, reverse.rs:969-975), both [M,N] with row
 * stride ldc in the element type. No workspace. */
SB_API int sb_op_matmul_gelu(uint32_t elem, const void* a, int64_t lda, const void* b, int64_t ldb, int32_t m,
                             int32_t n, int32_t k, void* y, void* dy, int64_t ldc, void* stream);
/* The matmul with a multiplicative epilogue, as the nanoGPT plan runs the
 * fc2 VJP through the GELU: C = (op(A) @ op(B)) * aux elementwise (the `*`
 * VJP rule fused into the dot_general, reverse.rs:551-583), aux [M,N] with
 * row stride ldaux in the element type; trans_a / trans_b as sb_op_matmul. */
SB_API int sb_op_matmul_mul(uint32_t elem, const void* a, int64_t lda, int trans_a, const void* b, int64_t ldb,
                            int trans_b, int32_t m, int32_t n, int32_t k, const void* aux, int64_t ldaux, void* c,
                            int64_t ldc, void* stream);

/* Layer norm without beta over the last dim (examples/nanogpt/model.shf:11-14:
 * (x - mean) / sqrt(var + 1e-5) * gamma, two-pass population variance as in
 * sheaf/src/lowering/codegen/reduction_builtins.rs:287-358).
 *   x f32 [rows, d]; gamma, y of type `elem` (SB_ELEM_BF16 / SB_ELEM_F32);
 *   mean, rstd f32 [rows] saved for the VJP. d must be a multiple of 4. */
SB_API int sb_op_layernorm_fwd(uint32_t elem, const void* x, const void* gamma, void* y, void* mean, void* rstd,
                               int32_t rows, int32_t d, void* stream);
/* VJP (the `/`, `-`, `sqrt`, `var`, `mean` rules of
 * sheaf/src/autodiff/reverse.rs:551-583,847-914,961-967, composed):
 *   dres (f32 [rows, d]) += dx; dgamma (`elem`, [d]) = sum_rows dy * xhat.
 *   dy is f32. */
SB_API size_t sb_op_layernorm_bwd_workspace_size(int32_t rows, int32_t d);
SB_API int sb_op_layernorm_bwd(uint32_t elem, const void* dy, const void* x, const void* mean, const void* rstd,
                               const void* gamma, void* dres, void* dgamma, void* workspace, size_t workspace_bytes,
                               int32_t rows, int32_t d, void* stream);

/* The same layer-norm VJP for callers that cannot allocate device memory
 * while they run (a host runtime that owns the device heap through its own
 * allocator and passes only finished buffers and a stream, or a
 * latency-critical loop that cannot afford cudaMalloc's device-wide
 * synchronisation). No counterpart in the reference: it exists for such
 * callers of this library. It takes no workspace: the dgamma partial sums go
 * to a fixed 128 KB array compiled into the library (held on every GPU that
 * uses it until the library is unloaded). d must be a multiple of 4 and at
 * most 4096; a larger d returns SB_OPERR_SCRATCH before any GPU work.
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture. All calls
 * share the array, so calls that overlap on the GPU race: serialise them.
 * Allocates nothing (no cudaMalloc / cudaFree). */
SB_API int sb_op_layernorm_bwd_noalloc(uint32_t elem, const void* dy, const void* x, const void* mean,
                                       const void* rstd, const void* gamma, void* dres, void* dgamma, int32_t rows,
                                       int32_t d, void* stream);

/* cross-entropy-loss fused with its VJP (sheaf/lib/nn.shf:28-30,44-50):
 *   loss_f32[0] = -mean_r log_softmax(logits[r])[targets[r]];
 *   dlogits = (softmax(logits) - one_hot(targets)) / rows.
 * logits / dlogits of type `elem` with row strides ld / ldd; targets are f32
 * class ids. As in the reference's one_hot (an f32 compare against an iota,
 * sheaf/src/lowering/stablehlo/tensor_ops.rs:163-217), a target that is not
 * exactly an integer in [0, v) selects no class: its row adds nothing to the
 * loss (which still divides by every row) and its dlogits row is zero. */
SB_API size_t sb_op_cross_entropy_workspace_size(int32_t rows);
SB_API int sb_op_cross_entropy(uint32_t elem, const void* logits, int64_t ld, int32_t rows, int32_t v,
                               const void* targets, void* dlogits, int64_t ldd, void* workspace,
                               size_t workspace_bytes, void* loss_f32, void* stream);

/* GELU, tanh form (sheaf/lib/nn.shf:10-11), elementwise over n values of
 * type `elem`: y = gelu(x). The VJP (chain rule through the inlined tanh /
 * multiply / add ops, sheaf/src/autodiff/reverse.rs:969-975) is
 * dx = g * gelu'(x). Inside the fused plans GELU lives in GEMM epilogues;
 * these standalone forms serve the primitive sweep and other graphs. */
SB_API int sb_op_gelu_fwd(uint32_t elem, const void* x, void* y, int64_t n, void* stream);
SB_API int sb_op_gelu_bwd(uint32_t elem, const void* x, const void* g, void* dx, int64_t n, void* stream);

/* Token + position embedding: x[n] = wte[clamp(ids[n])] + wpe[n % t] (f32 out)
 * (`stablehlo.convert` + `stablehlo.gather`,
 * sheaf/src/lowering/stablehlo/indexing_ops.rs:416-484; wpe `slice`). */
SB_API int sb_op_embedding_fwd(uint32_t elem, const void* ids, const void* wte, const void* wpe, void* x,
                               int32_t ntok, int32_t t, int32_t v, int32_t d, void* stream);
/* Embedding VJP as a scatter-add (the reference's one-hot matmul,
 * sheaf/src/autodiff/reverse.rs:1077-1122) and the wpe slice VJP (pad,
 * sheaf/src/lowering/codegen/builtins.rs:208-271): dx f32 [b*t, d] ->
 * dwte [v, d], dwpe [p, d] (rows >= t zero), both of type `elem`. The
 * one-hot compares the f32 id with an f32 iota, so an id that is not exactly
 * an integer in [0, v) adds nothing (the forward gather instead truncates
 * and clamps it). */
SB_API size_t sb_op_embedding_bwd_workspace_size(int32_t v, int32_t d);
SB_API int sb_op_embedding_bwd(uint32_t elem, const void* ids, const void* dx, int32_t b, int32_t t, int32_t p,
                               int32_t v, int32_t d, void* dwte, void* dwpe, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Fused causal self-attention over the packed projection qkv [b*t, 3*h*hd]
 * (q | k | v, head j at columns j*hd), as examples/nanogpt/model.shf:55-70
 * computes it: softmax(where(tril, q k^T / sqrt(hd), -1e10)) v, heads merged
 * to o [b*t, h*hd]; lse f32 [b*h*t] (log-sum-exp of the scaled scores) is
 * saved for the VJP. hd is 32 or 64. */
SB_API int sb_op_attention_fwd(uint32_t elem, const void* qkv, void* o, void* lse, int32_t b, int32_t t, int32_t h,
                               int32_t hd, void* stream);
/* VJP: dqkv [b*t, 3*h*hd] (dq | dk | dv) from qkv, o, do and lse. */
SB_API size_t sb_op_attention_bwd_workspace_size(uint32_t elem, int32_t b, int32_t t, int32_t h, int32_t hd);
SB_API int sb_op_attention_bwd(uint32_t elem, const void* qkv, const void* o, const void* dout, const void* lse,
                               void* dqkv, void* workspace, size_t workspace_bytes, int32_t b, int32_t t, int32_t h,
                               int32_t hd, void* stream);

/* Optimizer step of nanoGPT's train-step (examples/nanogpt/train.shf:29-32):
 * clip-by-global-norm(g, max_norm) then adamw-step(params, g, m, v, t, lr, b1,
 * b2, eps, wd) as sheaf/lib/optim.shf:19-32,42-51 define them, over n_leaves
 * tensors of element type `elem` (f32 or bf16) at once. The pointer arrays
 * are host arrays of device pointers; counts[i] is leaf i's element count.
 * t and lr are device f32 scalars; t_out receives t + 1. params_out / m_out /
 * v_out may alias params / m / v. max_norm <= 0 disables clipping; norm_out
 * (device f32, optional) receives the global norm of the unclipped gradients.
 * Replaces the optimizer part of the compiled train-step module (IREE
 * dispatches behind iree_runtime_session_call_by_name,
 * sheaf/src/runtime/iree_session.rs:576-583). */
SB_API size_t sb_op_adamw_workspace_size(const int64_t* counts, int32_t n_leaves);
SB_API int sb_op_adamw_step(uint32_t elem, int32_t n_leaves, const int64_t* counts, const void* const* grads,
                            const void* const* params, const void* const* m, const void* const* v,
                            void* const* params_out, void* const* m_out, void* const* v_out, const void* t,
                            void* t_out, const void* lr, float b1, float b2, float eps, float wd, float max_norm,
                            void* norm_out, void* workspace, size_t workspace_bytes, void* stream);
/* Global norm sqrt(sum_i sum(g_i^2)) of n_leaves gradient tensors
 * (sheaf/lib/optim.shf:42-45), f32 accumulation, written to norm_out. */
SB_API int sb_op_global_norm(uint32_t elem, int32_t n_leaves, const int64_t* counts, const void* const* grads,
                             void* norm_out, void* workspace, size_t workspace_bytes, void* stream);

/* get-batch of examples/nanogpt/train.shf:15-21 on the device: x, y
 * [batch, block] f32 token ids, rows starting at random-randint(key, [batch],
 * 0, n - block - 1) (sheaf/src/core/prng.rs:124-134) in `data` (n f32 ids);
 * y is x shifted by one. `key` is four f32 limbs (prng.rs:29-40); all
 * pointers are device memory. Requires 0 < n - block - 1 <= 2^24. */
SB_API int sb_op_get_batch(const void* data, int64_t n, const void* key, int32_t block, int32_t batch, void* x,
                           void* y, void* stream);
/* random-split of `key` into n child keys written as [n, 4] f32 limbs
 * (child i = threefry(key, [i, 1]), prng.rs:81-84, random_ops.rs:146-162). */
SB_API int sb_op_random_split(const void* key, int32_t n, void* out, void* stream);

/* Reads and clears the device error word that bounded waits inside the
 * kernels set (0 = no error, 1 = a barrier wait timed out). Synchronizes
 * the device. */
SB_API int sb_op_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SHEAF_B200_OPS_H_ */
