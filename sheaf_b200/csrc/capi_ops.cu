// C-ABI wrappers of the kernel library (include/sheaf_b200_ops.h).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/sheaf_b200_ops.h"
#include "sb_kernels.h"
#include "sb_nn.h"

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

int sb_op_matmul_gelu(uint32_t elem, const void* a, int64_t lda, const void* b, int64_t ldb, int32_t m, int32_t n,
                      int32_t k, void* y, void* dy, int64_t ldc, void* stream) {
  sb::GemmDesc d;
  if (!a || !b || !y || !dy) return SB_OPERR_ARGS;
  if (!sb::fill_matmul_desc(d, elem, a, lda, 0, b, ldb, 1, m, n, k)) return SB_OPERR_ARGS;
  d.out = y;
  d.ldo = ldc;
  d.out_f32 = elem == SB_ELEM_F32;
  d.epi = sb::EPI_GELU;
  d.out2 = dy;
  d.ldo2 = ldc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (elem == SB_ELEM_BF16) return sb::gemm_bf16(d, nullptr, 0, s, sb::device_error_word());
  return sb::gemm_f32(d, nullptr, 0, s, sb::device_error_word());
}

int sb_op_matmul_mul(uint32_t elem, const void* a, int64_t lda, int trans_a, const void* b, int64_t ldb, int trans_b,
                     int32_t m, int32_t n, int32_t k, const void* aux, int64_t ldaux, void* c, int64_t ldc,
                     void* stream) {
  sb::GemmDesc d;
  if (!a || !b || !aux || !c) return SB_OPERR_ARGS;
  if (!sb::fill_matmul_desc(d, elem, a, lda, trans_a, b, ldb, trans_b, m, n, k)) return SB_OPERR_ARGS;
  d.out = c;
  d.ldo = ldc;
  d.out_f32 = elem == SB_ELEM_F32;
  d.epi = sb::EPI_MUL;
  d.aux = aux;
  d.ldaux = ldaux;
  d.aux_f32 = elem == SB_ELEM_F32;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (elem == SB_ELEM_BF16) return sb::gemm_bf16(d, nullptr, 0, s, sb::device_error_word());
  return sb::gemm_f32(d, nullptr, 0, s, sb::device_error_word());
}

static bool float_elem(uint32_t e) { return e == SB_ELEM_BF16 || e == SB_ELEM_F32; }

int sb_op_layernorm_fwd(uint32_t elem, const void* x, const void* gamma, void* y, void* mean, void* rstd,
                        int32_t rows, int32_t d, void* stream) {
  if (!float_elem(elem) || !x || !gamma || !y || !mean || !rstd) return SB_OPERR_ARGS;
  const bool f = elem == SB_ELEM_F32;
  return sb::layernorm_fwd(x, true, gamma, f, y, f, static_cast<float*>(mean),
                           static_cast<float*>(rstd), rows, d, static_cast<cudaStream_t>(stream));
}

size_t sb_op_layernorm_bwd_workspace_size(int32_t rows, int32_t d) { return sb::layernorm_bwd_workspace_bytes(rows, d); }

int sb_op_layernorm_bwd(uint32_t elem, const void* dy, const void* x, const void* mean, const void* rstd,
                        const void* gamma, void* dres, void* dgamma, void* workspace, size_t workspace_bytes,
                        int32_t rows, int32_t d, void* stream) {
  if (!float_elem(elem) || !dy || !x || !mean || !rstd || !gamma || !dres || !dgamma) return SB_OPERR_ARGS;
  if (workspace_bytes < sb::layernorm_bwd_workspace_bytes(rows, d) || !workspace) return SB_OPERR_WORKSPACE;
  const bool f = elem == SB_ELEM_F32;
  return sb::layernorm_bwd(dy, true, x, true, static_cast<const float*>(mean),
                           static_cast<const float*>(rstd), gamma, f, dres, dres, dgamma, f,
                           static_cast<float*>(workspace), rows, d, static_cast<cudaStream_t>(stream));
}

size_t sb_op_cross_entropy_workspace_size(int32_t rows) { return sb::cross_entropy_workspace_bytes(rows); }

int sb_op_cross_entropy(uint32_t elem, const void* logits, int64_t ld, int32_t rows, int32_t v, const void* targets,
                        void* dlogits, int64_t ldd, void* workspace, size_t workspace_bytes, void* loss_f32,
                        void* stream) {
  if (!float_elem(elem) || !logits || !targets || !dlogits || !loss_f32) return SB_OPERR_ARGS;
  if (!workspace || workspace_bytes < sb::cross_entropy_workspace_bytes(rows)) return SB_OPERR_WORKSPACE;
  return sb::cross_entropy_fwd_bwd(logits, elem == SB_ELEM_F32, ld, rows, v, static_cast<const float*>(targets),
                                   dlogits, ldd, static_cast<float*>(workspace), static_cast<float*>(loss_f32),
                                   nullptr, static_cast<cudaStream_t>(stream));
}

int sb_op_gelu_fwd(uint32_t elem, const void* x, void* y, int64_t n, void* stream) {
  if (!float_elem(elem) || !x || !y || n <= 0) return SB_OPERR_ARGS;
  return sb::gelu(x, nullptr, y, elem == SB_ELEM_F32, false, n, static_cast<cudaStream_t>(stream));
}

int sb_op_gelu_bwd(uint32_t elem, const void* x, const void* g, void* dx, int64_t n, void* stream) {
  if (!float_elem(elem) || !x || !g || !dx || n <= 0) return SB_OPERR_ARGS;
  return sb::gelu(x, g, dx, elem == SB_ELEM_F32, true, n, static_cast<cudaStream_t>(stream));
}

int sb_op_embedding_fwd(uint32_t elem, const void* ids, const void* wte, const void* wpe, void* x, int32_t ntok,
                        int32_t t, int32_t v, int32_t d, void* stream) {
  if (!float_elem(elem) || !ids || !wte || !wpe || !x || t <= 0 || v <= 0) return SB_OPERR_ARGS;
  return sb::embedding_fwd(static_cast<const float*>(ids), wte, wpe, elem == SB_ELEM_F32, x, true,
                           ntok, t, v, d, static_cast<cudaStream_t>(stream));
}

size_t sb_op_embedding_bwd_workspace_size(int32_t v, int32_t d) { return sb::embedding_bwd_workspace_bytes(v, d); }

int sb_op_embedding_bwd(uint32_t elem, const void* ids, const void* dx, int32_t b, int32_t t, int32_t p, int32_t v,
                        int32_t d, void* dwte, void* dwpe, void* workspace, size_t workspace_bytes, void* stream) {
  if (!float_elem(elem) || !ids || !dx || !dwte || !dwpe || p < t) return SB_OPERR_ARGS;
  if (workspace_bytes < sb::embedding_bwd_workspace_bytes(v, d)) return SB_OPERR_WORKSPACE;
  return sb::embedding_bwd(static_cast<const float*>(ids), dx, true, b, t, p, v, d, dwte, dwpe,
                           elem == SB_ELEM_F32, static_cast<float*>(workspace), static_cast<cudaStream_t>(stream));
}

int sb_op_attention_fwd(uint32_t elem, const void* qkv, void* o, void* lse, int32_t b, int32_t t, int32_t h,
                        int32_t hd, void* stream) {
  if (!float_elem(elem) || !qkv || !o || !lse || b <= 0 || t <= 0 || h <= 0) return SB_OPERR_ARGS;
  return sb::attention_fwd(qkv, elem == SB_ELEM_F32, o, static_cast<float*>(lse), sb::AttnShape{b, t, h, hd},
                           static_cast<cudaStream_t>(stream));
}

size_t sb_op_attention_bwd_workspace_size(uint32_t elem, int32_t b, int32_t t, int32_t h, int32_t hd) {
  return sb::attention_bwd_workspace_bytes(elem == SB_ELEM_F32, sb::AttnShape{b, t, h, hd});
}

int sb_op_attention_bwd(uint32_t elem, const void* qkv, const void* o, const void* dout, const void* lse, void* dqkv,
                        void* workspace, size_t workspace_bytes, int32_t b, int32_t t, int32_t h, int32_t hd,
                        void* stream) {
  if (!float_elem(elem) || !qkv || !o || !dout || !lse || !dqkv) return SB_OPERR_ARGS;
  const sb::AttnShape sh{b, t, h, hd};
  if (!workspace || workspace_bytes < sb::attention_bwd_workspace_bytes(elem == SB_ELEM_F32, sh))
    return SB_OPERR_WORKSPACE;
  return sb::attention_bwd(qkv, o, dout, static_cast<const float*>(lse), elem == SB_ELEM_F32, dqkv,
                           static_cast<float*>(workspace), sh, static_cast<cudaStream_t>(stream));
}

size_t sb_op_adamw_workspace_size(const int64_t* counts, int32_t n_leaves) {
  if (!counts || n_leaves <= 0) return 0;
  return sb::optimizer_workspace_bytes(counts, n_leaves);
}

int sb_op_adamw_step(uint32_t elem, int32_t n_leaves, const int64_t* counts, const void* const* grads,
                     const void* const* params, const void* const* m, const void* const* v, void* const* params_out,
                     void* const* m_out, void* const* v_out, const void* t, void* t_out, const void* lr, float b1,
                     float b2, float eps, float wd, float max_norm, void* norm_out, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!float_elem(elem) || !params || !t || !t_out || !lr) return SB_OPERR_ARGS;
  return sb::optimizer_step(elem == SB_ELEM_BF16, n_leaves, counts, grads, params, m, v, params_out, m_out, v_out,
                            static_cast<const float*>(t), static_cast<float*>(t_out), static_cast<const float*>(lr),
                            b1, b2, eps, wd, max_norm, static_cast<float*>(norm_out), workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream));
}

int sb_op_get_batch(const void* data, int64_t n, const void* key, int32_t block, int32_t batch, void* x, void* y,
                    void* stream) {
  return sb::get_batch(static_cast<const float*>(data), n, static_cast<const float*>(key), block, batch,
                       static_cast<float*>(x), static_cast<float*>(y), static_cast<cudaStream_t>(stream));
}

int sb_op_random_split(const void* key, int32_t n, void* out, void* stream) {
  return sb::random_split(static_cast<const float*>(key), n, static_cast<float*>(out),
                          static_cast<cudaStream_t>(stream));
}

int sb_op_global_norm(uint32_t elem, int32_t n_leaves, const int64_t* counts, const void* const* grads,
                      void* norm_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!float_elem(elem) || !norm_out) return SB_OPERR_ARGS;
  return sb::optimizer_step(elem == SB_ELEM_BF16, n_leaves, counts, grads, nullptr, nullptr, nullptr, nullptr,
                            nullptr, nullptr, nullptr, nullptr, nullptr, 0.f, 0.f, 0.f, 0.f, 0.f,
                            static_cast<float*>(norm_out), workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream));
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
