// fp32 GEMMs on the tcgen05 tensor cores by the bf16x6 split (Henry, Tang and
// Heinecke, "Leveraging the bfloat16 Artificial Intelligence Datatype For
// Higher-Precision Computations", ARITH 2019): every f32 operand value is
// written as the sum of three bf16 parts,
//   x0 = bf16(x),  x1 = bf16(x - x0),  x2 = bf16(x - x0 - x1)
// (each difference exact in f32), and
//   a * b ~= a0 b0 + a0 b1 + a1 b0 + a0 b2 + a1 b1 + a2 b0,
// dropping the three products below 2^-24 of |a b|. A bf16 x bf16 product is
// exact in f32, so laying the six part pairs out along K (A' = [a0 a0 a1 a0
// a1 a2], B' = [b0 b1 b0 b2 b1 b0], K' = 6 K) turns the f32 product into one
// bf16 GEMM with f32 accumulation, whose error is that of an f32
// accumulation of the 6 K exact terms -- the 1e-5 parity bar of the fp32
// path holds, as for the CUDA-core FFMA GEMM it replaces on large shapes.
//
// The tensor cores' own accumulation of a long chain loses low-order bits
// (measured on this part: 7e-7 of the largest output at K' = 2304, 1.8e-5 at
// K' = 9216-12288, against 2e-6 for the FFMA kernel); as Ootomo and Yokota
// ("Recovering single precision accuracy from Tensor Cores while surpassing
// the FP32 theoretical peak performance", IJHPCA 2022) do, the chains are kept
// short and their partial sums added in round-to-nearest f32 on the CUDA
// cores: the product always runs split-K with at most kSplitK terms of K' per
// split, the splits summed by the split-K reduction.
//
// The split copies keep the operand's storage order (K-major [rows, K] ->
// [rows, 6K]; MN-major [K, cols] -> [6K, cols]), so the bf16 kernel reads them
// exactly as it would read the f32 operand. Epilogues other than a plain store
// (GELU, multiply, add, accumulate) run as one f32 elementwise pass after the
// product, which split-K leaves in an f32 temporary (the bf16 kernel's own
// GELU epilogue rounds u to bf16 first, which the fp32 module does not).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "sb_kernels.h"

namespace sb {

namespace {

// Part j of the six along K, for A (first) and B (second).
__constant__ int kPartA[6] = {0, 0, 1, 0, 1, 2};
__constant__ int kPartB[6] = {0, 1, 0, 2, 1, 0};

// x -> its three bf16 parts.
__device__ __forceinline__ void split3(float x, __nv_bfloat16 (&p)[3]) {
  p[0] = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(p[0]);
  p[1] = __float2bfloat16_rn(r1);
  p[2] = __float2bfloat16_rn(r1 - __bfloat162float(p[1]));
}

// Writes the six-part copy of a stored [rows, cols] f32 matrix (row stride
// ld). k_major: K runs along cols, the copy is [rows, 6 cols] with part block
// j at columns j*cols; otherwise K runs along rows, the copy is [6 rows, cols]
// with block j at rows j*rows. which = 0 for A's part order, 1 for B's.
__global__ void split6_kernel(const float* __restrict__ x, long rows, long cols, long ld, bool k_major, int which,
                              __nv_bfloat16* __restrict__ out) {
  const long total = rows * cols;
  for (long e = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = e / cols, c = e % cols;
    __nv_bfloat16 p[3];
    split3(x[r * ld + c], p);
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const __nv_bfloat16 v = p[which ? kPartB[j] : kPartA[j]];
      if (k_major)
        out[r * 6 * cols + j * cols + c] = v;
      else
        out[(j * rows + r) * cols + c] = v;
    }
  }
}

constexpr int kSplitK = 1536;

__device__ __forceinline__ float gelu_f32(float x) {
  const float inner = x + 0.044715f * (x * (x * x));
  return 0.5f * (x * (1.0f + tanhf(0.7978846f * inner)));
}
__device__ __forceinline__ float gelu_df32(float x) {
  const float x2 = x * x;
  const float t = tanhf(0.7978846f * (x + 0.044715f * (x * x2)));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * 0.7978846f * (1.0f + 0.134145f * x2);
}

// u [M, N] (row stride N) -> out = gelu(u), out2 = gelu'(u); out = u * aux;
// out = u + aux; or out += u.
__global__ void epilogue_f32_kernel(const float* __restrict__ u, long M, long N, int epi, float* __restrict__ out,
                                    long ldo, float* __restrict__ out2, long ldo2, const float* __restrict__ aux,
                                    long ldaux) {
  const long total = M * N;
  for (long e = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = e / N, c = e % N;
    const float v = u[e];
    if (epi == EPI_GELU) {
      out[r * ldo + c] = gelu_f32(v);
      out2[r * ldo2 + c] = gelu_df32(v);
    } else if (epi == EPI_MUL) {
      out[r * ldo + c] = v * aux[r * ldaux + c];
    } else if (epi == EPI_ADD) {
      out[r * ldo + c] = v + aux[r * ldaux + c];
    } else {  // EPI_ACCUM
      out[r * ldo + c] += v;
    }
  }
}

int blocks_for(long n) {
  const long b = (n + 255) / 256;
  return static_cast<int>(std::max<long>(1, std::min<long>(b, 16L * num_sms())));
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// The bf16 GEMM over the split copies (operands filled in by the caller).
bool needs_tmp(const GemmDesc& d) { return d.epi != EPI_STORE; }

GemmDesc split_desc(const GemmDesc& d) {
  GemmDesc e = d;
  e.K = 6 * d.K;
  e.lda = d.a_mn ? d.M : 6L * d.K;
  e.ldb = d.b_mn ? d.N : 6L * d.K;
  if (needs_tmp(d)) {  // product into an f32 temporary first
    e.epi = EPI_STORE;
    e.ldo = d.N;
    e.aux = nullptr;
    e.out2 = nullptr;
  }
  e.out_f32 = true;
  e.splits = std::max(2, (e.K + kSplitK - 1) / kSplitK);
  e.max_splits = 0;
  e.max_ctas = 0;
  e.max_pair_splits = 0;
  return e;
}

}  // namespace

// Large enough for the split to pay (below it the FFMA kernel's launch is
// cheaper than three launches), with the f32 output addressable by TMA.
bool gemm_f32_use_emulation(const GemmDesc& d) {
  static const bool ffma = [] {
    const char* e = std::getenv("SHEAF_B200_F32_GEMM");
    return e && std::strcmp(e, "ffma") == 0;
  }();
  if (ffma) return false;
  const double work = static_cast<double>(d.M) * d.N * d.K;
  // split-K partial rows (and the f32 output of a plain store, written by
  // TMA) must be 16-byte multiples
  const bool tma_out = (d.N % 4) == 0 && (needs_tmp(d) ||
                                          ((d.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(d.out) & 15) == 0));
  // the bf16 split copies' rows must be 16-byte multiples too: 6K bf16 for a
  // K-major copy, M (or N) bf16 for an MN-major one
  const bool a_ok = d.a_mn ? (d.M % 8) == 0 : (d.K % 4) == 0;
  const bool b_ok = d.b_mn ? (d.N % 8) == 0 : (d.K % 4) == 0;
  return work >= 6.7e7 && d.M >= 64 && d.N >= 64 && tma_out && a_ok && b_ok;
}

size_t gemm_f32_emulated_workspace_bytes(const GemmDesc& d) {
  const size_t a = up256(6 * static_cast<size_t>(d.M) * d.K * 2);
  const size_t b = up256(6 * static_cast<size_t>(d.N) * d.K * 2);
  const size_t t = needs_tmp(d) ? up256(static_cast<size_t>(d.M) * d.N * 4) : 0;
  return a + b + t + gemm_workspace_bytes(split_desc(d), true);
}

int gemm_f32_emulated(const GemmDesc& d, void* workspace, size_t workspace_bytes, cudaStream_t s, int* err) {
  if (!workspace || workspace_bytes < gemm_f32_emulated_workspace_bytes(d)) return 5;
  char* w = static_cast<char*>(workspace);
  __nv_bfloat16* a6 = reinterpret_cast<__nv_bfloat16*>(w);
  w += up256(6 * static_cast<size_t>(d.M) * d.K * 2);
  __nv_bfloat16* b6 = reinterpret_cast<__nv_bfloat16*>(w);
  w += up256(6 * static_cast<size_t>(d.N) * d.K * 2);
  float* tmp = nullptr;
  if (needs_tmp(d)) {
    tmp = reinterpret_cast<float*>(w);
    w += up256(static_cast<size_t>(d.M) * d.N * 4);
  }
  const size_t rest = workspace_bytes - static_cast<size_t>(w - static_cast<char*>(workspace));
  // A stored [M, K] (K-major) or [K, M]; B stored [N, K] or [K, N]
  const long ar = d.a_mn ? d.K : d.M, ac = d.a_mn ? d.M : d.K;
  const long br = d.b_mn ? d.K : d.N, bc = d.b_mn ? d.N : d.K;
  split6_kernel<<<blocks_for(ar * ac), 256, 0, s>>>(static_cast<const float*>(d.A), ar, ac, d.lda, !d.a_mn, 0, a6);
  split6_kernel<<<blocks_for(br * bc), 256, 0, s>>>(static_cast<const float*>(d.B), br, bc, d.ldb, !d.b_mn, 1, b6);
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  GemmDesc e = split_desc(d);
  e.A = a6;
  e.B = b6;
  if (tmp) e.out = tmp;
  if (int rc = gemm_bf16(e, reinterpret_cast<float*>(w), rest, s, err)) return rc;
  if (tmp) {
    epilogue_f32_kernel<<<blocks_for(static_cast<long>(d.M) * d.N), 256, 0, s>>>(
        tmp, d.M, d.N, d.epi, static_cast<float*>(d.out), d.ldo, static_cast<float*>(d.out2), d.ldo2,
        static_cast<const float*>(d.aux), d.ldaux);
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
  }
  return 0;
}

}  // namespace sb
