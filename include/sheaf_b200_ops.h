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

/* Reads and clears the device error word that bounded waits inside the
 * kernels set (0 = no error, 1 = a barrier wait timed out). Synchronizes
 * the device. */
SB_API int sb_op_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SHEAF_B200_OPS_H_ */
