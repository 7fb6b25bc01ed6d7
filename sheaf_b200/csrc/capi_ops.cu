// C-ABI wrappers of the kernel library (include/sheaf_b200_ops.h).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/sheaf_b200_ops.h"
#include "sb_kernels.h"

namespace sb {

// One device word per process that kernels' bounded waits write on timeout.
int* device_error_word() {
  static int* word = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    if (cudaMalloc(&word, sizeof(int)) == cudaSuccess) cudaMemset(word, 0, sizeof(int));
  });
  return word;
}

static bool fill_matmul_desc(GemmDesc& d, uint32_t elem, const void* a, int64_t lda, int trans_a, const void* b,
                             int64_t ldb, int trans_b, int32_t m, int32_t n, int32_t k) {
  if (elem != SB_ELEM_BF16 && elem != SB_ELEM_F32) return false;
  if (m <= 0 || n <= 0 || k <= 0) return false;
  d.A = a;
  d.lda = lda;
  d.a_mn = trans_a != 0;
  d.B = b;
  d.ldb = ldb;
  d.b_mn = trans_b == 0;  // B stored [K,N] is N-major for the kernel
  d.M = m;
  d.N = n;
  d.K = k;
  d.epi = EPI_STORE;
  return true;
}

}  // namespace sb

extern "C" {

size_t sb_op_matmul_workspace_size(uint32_t elem, int trans_a, int trans_b, int32_t m, int32_t n, int32_t k) {
  sb::GemmDesc d;
  if (!sb::fill_matmul_desc(d, elem, nullptr, 0, trans_a, nullptr, 0, trans_b, m, n, k)) return 0;
  return sb::gemm_workspace_bytes(d, elem == SB_ELEM_BF16);
}

int sb_op_matmul(uint32_t elem, const void* a, int64_t lda, int trans_a, const void* b, int64_t ldb, int trans_b,
                 int32_t m, int32_t n, int32_t k, void* c, int64_t ldc, uint32_t c_elem, void* workspace,
                 size_t workspace_bytes, void* stream) {
  sb::GemmDesc d;
  if (!a || !b || !c) return SB_OPERR_ARGS;
  if (!sb::fill_matmul_desc(d, elem, a, lda, trans_a, b, ldb, trans_b, m, n, k)) return SB_OPERR_ARGS;
  if (c_elem != SB_ELEM_F32 && c_elem != SB_ELEM_BF16) return SB_OPERR_ARGS;
  if (elem == SB_ELEM_F32 && c_elem != SB_ELEM_F32) return SB_OPERR_ARGS;
  d.out = c;
  d.ldo = ldc;
  d.out_f32 = (c_elem == SB_ELEM_F32);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (elem == SB_ELEM_BF16)
    return sb::gemm_bf16(d, static_cast<float*>(workspace), workspace_bytes, s, sb::device_error_word());
  return sb::gemm_f32(d, static_cast<float*>(workspace), workspace_bytes, s, sb::device_error_word());
}

int sb_op_device_error(void) {
  int* w = sb::device_error_word();
  if (!w) return -1;
  int v = 0;
  cudaDeviceSynchronize();
  cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  cudaMemset(w, 0, sizeof(int));
  return v;
}

}  // extern "C"
