// fp32 GEMM on the CUDA cores: the fp32 path of `stablehlo.dot_general`
// (lowering/stablehlo/dot_ops.rs:12-229) and of the `@` VJP
// (autodiff/reverse.rs:585-689). Exact fp32 multiply-add accumulation keeps
// results within 1e-5 relative of an fp32 CPU evaluation, which tf32 tensor
// cores (10-bit mantissa) would not.
//
// 128x128 output tile per CTA, 256 threads, 8x8 outputs per thread in two
// 4x4 quadrants (conflict-free float4 reads of the smem panels), BK = 16,
// register-staged double buffering of the global loads. Split-K over a fp32
// workspace for the long-K weight-gradient contractions.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "sb_kernels.h"

namespace sb {

namespace {

constexpr int TM = 128, TN = 128, TK = 16;

struct F32Args {
  const float* A;
  long lda;
  const float* B;
  long ldb;
  int M, N, K;
  int splits, k_per_split;
  int epi;
  float* out;
  long ldo;
  const float* aux;
  long ldaux;
  float* out2;
  long ldo2;
  long split_stride;
};

// gelu(x) = 0.5 * (x * (1 + tanh(0.7978846 * (x + 0.044715 * (x * (x * x))))))
// (lib/nn.shf:10-11) and its derivative by the chain rule of those primitive
// ops, from one tanh.
__device__ __forceinline__ void gelu_and_grad32(float x, float& g, float& d) {
  const float x2 = x * x;
  const float t = tanhf(0.7978846f * (x + 0.044715f * (x * x2)));
  g = 0.5f * (x * (1.0f + t));
  d = 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * 0.7978846f * (1.0f + 0.134145f * x2);
}

// Loads a TK x 128 panel of an operand into registers (8 values/thread).
//   K-major operand (X[mn*ld + k]) : thread t -> mn = t/2, k = (t%2)*8 .. +7
//   MN-major operand (X[k*ld + mn]): thread t -> k = t/16, mn = (t%16)*8 .. +7
template <bool MN>
__device__ __forceinline__ void load_panel(const float* __restrict__ X, long ld, int mn_total, int k_total, int mn0,
                                           int k0, float (&r)[8]) {
  const int t = threadIdx.x;
  if (!MN) {
    const int mn = mn0 + t / 2, k = k0 + (t % 2) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = (mn < mn_total && k + j < k_total) ? X[static_cast<long>(mn) * ld + k + j] : 0.f;
  } else {
    const int k = k0 + t / 16, mn = mn0 + (t % 16) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = (k < k_total && mn + j < mn_total) ? X[static_cast<long>(k) * ld + mn + j] : 0.f;
  }
}

template <bool MN>
__device__ __forceinline__ void store_panel(float (*S)[TM], const float (&r)[8]) {
  const int t = threadIdx.x;
  if (!MN) {
    const int mn = t / 2, k = (t % 2) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) S[k + j][mn] = r[j];
  } else {
    const int k = t / 16, mn = (t % 16) * 8;
    *reinterpret_cast<float4*>(&S[k][mn]) = make_float4(r[0], r[1], r[2], r[3]);
    *reinterpret_cast<float4*>(&S[k][mn + 4]) = make_float4(r[4], r[5], r[6], r[7]);
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(256) gemm_f32_kernel(F32Args a) {
  __shared__ __align__(16) float As[2][TK][TM];
  __shared__ __align__(16) float Bs[2][TK][TN];

  const int split = blockIdx.z;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int kbeg = split * a.k_per_split;
  const int kend = min(a.K, kbeg + a.k_per_split);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float ra[8], rb[8];
  load_panel<A_MN>(a.A, a.lda, a.M, kend, m0, kbeg, ra);
  load_panel<B_MN>(a.B, a.ldb, a.N, kend, n0, kbeg, rb);
  store_panel<A_MN>(As[0], ra);
  store_panel<B_MN>(Bs[0], rb);
  __syncthreads();

  int buf = 0;
  for (int k0 = kbeg; k0 < kend; k0 += TK) {
    const bool more = k0 + TK < kend;
    if (more) {
      load_panel<A_MN>(a.A, a.lda, a.M, kend, m0, k0 + TK, ra);
      load_panel<B_MN>(a.B, a.ldb, a.N, kend, n0, k0 + TK, rb);
    }
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float av[8], bv[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
      av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      store_panel<A_MN>(As[buf ^ 1], ra);
      store_panel<B_MN>(Bs[buf ^ 1], rb);
    }
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (col >= a.N) continue;
      const float v = acc[i][j];
      const long o = static_cast<long>(row) * a.ldo + col;
      switch (a.epi) {
        case EPI_STORE: a.out[split * a.split_stride + o] = v; break;
        case EPI_ADD: a.out[o] = a.aux[static_cast<long>(row) * a.ldaux + col] + v; break;
        case EPI_GELU: {
          float g, dg;
          gelu_and_grad32(v, g, dg);
          a.out[o] = g;
          a.out2[static_cast<long>(row) * a.ldo2 + col] = dg;
          break;
        }
        case EPI_ACCUM: a.out[o] += v; break;
        default: a.out[o] = v * a.aux[static_cast<long>(row) * a.ldaux + col]; break;  // EPI_MUL
      }
    }
  }
}

__global__ void splitk_reduce_f32(const float* __restrict__ ws, int splits, long slice, int M, int N, float* out,
                                  long ldo) {
  const long total = static_cast<long>(M) * N;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[s * slice + i];
    out[(i / N) * ldo + (i % N)] = acc;
  }
}

struct F32Plan {
  int splits, k_per_split;
};

F32Plan f32_plan(const GemmDesc& d) {
  const int tiles = ((d.M + TM - 1) / TM) * ((d.N + TN - 1) / TN);
  int splits = d.splits;
  if (splits <= 0) {
    splits = 1;
    if (d.epi == EPI_STORE && tiles * 2 <= num_sms() && d.K >= 1024) splits = std::min(num_sms() / tiles, d.K / 256);
  }
  if (d.epi != EPI_STORE) splits = 1;
  splits = std::max(1, splits);
  int kps = (d.K + splits - 1) / splits;
  kps = (kps + TK - 1) / TK * TK;
  splits = (d.K + kps - 1) / kps;
  return {splits, kps};
}

}  // namespace

size_t gemm_f32_workspace_bytes(const GemmDesc& d) {
  F32Plan p = f32_plan(d);
  const size_t ffma = p.splits <= 1 ? 0 : static_cast<size_t>(p.splits) * d.M * d.N * sizeof(float);
  // enough for either path: the choice also depends on the output's alignment
  return gemm_f32_use_emulation(d) ? std::max(ffma, gemm_f32_emulated_workspace_bytes(d)) : ffma;
}

int gemm_f32(const GemmDesc& d, float* workspace, size_t workspace_bytes, cudaStream_t s, int* err) {
  if (d.M <= 0 || d.N <= 0 || d.K <= 0) return 1;
  if (gemm_f32_use_emulation(d) && workspace && workspace_bytes >= gemm_f32_emulated_workspace_bytes(d))
    return gemm_f32_emulated(d, workspace, workspace_bytes, s, err);
  F32Plan p = f32_plan(d);
  F32Args a{};
  a.A = static_cast<const float*>(d.A);
  a.lda = d.lda;
  a.B = static_cast<const float*>(d.B);
  a.ldb = d.ldb;
  a.M = d.M;
  a.N = d.N;
  a.K = d.K;
  a.splits = p.splits;
  a.k_per_split = p.k_per_split;
  a.epi = d.epi;
  const bool split = p.splits > 1;
  if (split) {
    const size_t need = static_cast<size_t>(p.splits) * d.M * d.N * sizeof(float);
    if (!workspace || workspace_bytes < need) return 5;
    a.out = workspace;
    a.ldo = d.N;
    a.split_stride = static_cast<long>(d.M) * d.N;
  } else {
    a.out = static_cast<float*>(d.out);
    a.ldo = d.ldo;
    a.aux = static_cast<const float*>(d.aux);
    a.ldaux = d.ldaux;
    a.out2 = static_cast<float*>(d.out2);
    a.ldo2 = d.ldo2;
  }
  dim3 grid((d.N + TN - 1) / TN, (d.M + TM - 1) / TM, p.splits);
  if (!d.a_mn && !d.b_mn) gemm_f32_kernel<false, false><<<grid, 256, 0, s>>>(a);
  else if (!d.a_mn && d.b_mn) gemm_f32_kernel<false, true><<<grid, 256, 0, s>>>(a);
  else if (d.a_mn && d.b_mn) gemm_f32_kernel<true, true><<<grid, 256, 0, s>>>(a);
  else gemm_f32_kernel<true, false><<<grid, 256, 0, s>>>(a);
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  if (split) {
    const long total = static_cast<long>(d.M) * d.N;
    const int blocks = static_cast<int>(std::min<long>((total + 255) / 256, 4L * num_sms()));
    splitk_reduce_f32<<<blocks, 256, 0, s>>>(workspace, p.splits, total, d.M, d.N, static_cast<float*>(d.out), d.ldo);
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
  }
  return 0;
}

}  // namespace sb
