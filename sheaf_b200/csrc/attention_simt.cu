// Causal self-attention on the CUDA cores (fp32 operands): the fp32 path of
// the nanoGPT attention block (examples/nanogpt/model.shf:55-70):
//   s = (q @ k^T) / sqrt(Hd); s = where(tril(ones[T,T]) == 1, s, -1e10);
//   p = softmax(s); o = p @ v, heads merged back to [B*T, D].
// exp(-1e10 - max) is exactly 0 in fp32, so masked keys are skipped.
// The VJP follows the `@`, `/`, `where` and softmax rules
// (autodiff/reverse.rs:585-689, 551-583, 1014-1019, 814-828):
//   dv = p^T do; dp = do v^T; ds = p * (dp - rowsum(do * o)); dq = ds k / sqrt(Hd);
//   dk = ds^T q / sqrt(Hd)  (rowsum(dp * p) == rowsum(do * o)).
// q/k/v are read in place from the packed projection output [B*T, 3*D].
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "sb_nn.h"

namespace sb {

namespace {

constexpr int kQB = 64;  // query rows per CTA (8 warps x 8 rows)
constexpr int kKC = 32;  // keys per shared-memory chunk
constexpr int kRPW = 4;  // backward: rows per warp
constexpr int kBQB = 8 * kRPW;  // backward: rows per CTA
constexpr int kMaxHd = 128;

template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ void stf(T* p, float v);
template <>
__device__ __forceinline__ void stf<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Forward. grid (ceil(T/64), B*H), 256 threads. DPL = Hd/32 dims per lane.
template <typename T, int DPL>
__global__ void __launch_bounds__(256) attn_fwd_simt(const T* __restrict__ qkv, T* __restrict__ out,
                                                     float* __restrict__ lse, int B, int Tn, int H, float inv_scale) {
  constexpr int Hd = DPL * 32;
  __shared__ float sQ[kQB][Hd];
  __shared__ float sK[kKC][Hd + 1];
  __shared__ float sV[kKC][Hd];
  const int D = H * Hd;
  const long ld = 3L * D;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kQB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const T* base = qkv + static_cast<long>(b) * Tn * ld;

  for (int i = threadIdx.x; i < kQB * Hd; i += blockDim.x) {
    const int r = i / Hd, d = i % Hd;
    sQ[r][d] = (q0 + r < Tn) ? ldf(base + static_cast<long>(q0 + r) * ld + h * Hd + d) : 0.f;
  }
  float m[8], l[8], o[8][DPL];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[i][j] = 0.f;
  }
  const int q_last = min(q0 + kQB, Tn) - 1;
  for (int k0 = 0; k0 <= q_last; k0 += kKC) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKC * Hd; i += blockDim.x) {
      const int r = i / Hd, d = i % Hd;
      const bool ok = k0 + r < Tn;
      sK[r][d] = ok ? ldf(base + static_cast<long>(k0 + r) * ld + D + h * Hd + d) : 0.f;
      sV[r][d] = ok ? ldf(base + static_cast<long>(k0 + r) * ld + 2 * D + h * Hd + d) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = warp * 8 + i;
      const int row = q0 + r;
      if (row >= Tn || k0 > row) continue;
      const int key = k0 + lane;
      float s = 0.f;
#pragma unroll 16
      for (int d = 0; d < Hd; ++d) s = fmaf(sQ[r][d], sK[lane][d], s);
      s = s / inv_scale;
      const bool valid = key <= row && key < Tn;
      const float cmax = wmax(valid ? s : -INFINITY);
      const float mn = fmaxf(m[i], cmax);
      const float p = valid ? expf(s - mn) : 0.f;
      const float corr = expf(m[i] - mn);
      l[i] = l[i] * corr + wsum(p);
      m[i] = mn;
#pragma unroll
      for (int j = 0; j < DPL; ++j) o[i][j] *= corr;
      for (int kk = 0; kk < kKC; ++kk) {
        const float pk = __shfl_sync(0xffffffffu, p, kk);
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[i][j] = fmaf(pk, sV[kk][lane + 32 * j], o[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = q0 + warp * 8 + i;
    if (row >= Tn) continue;
    T* orow = out + (static_cast<long>(b) * Tn + row) * D + h * Hd;
#pragma unroll
    for (int j = 0; j < DPL; ++j) stf(orow + lane + 32 * j, o[i][j] / l[i]);
    if (lane == 0) lse[static_cast<long>(bh) * Tn + row] = m[i] + logf(l[i]);
  }
}

// delta[bh*T + t] = sum_d dO[t, h, d] * O[t, h, d]
template <typename T>
__global__ void attn_delta(const T* __restrict__ out, const T* __restrict__ dout, float* __restrict__ delta, int B,
                           int Tn, int H, int Hd) {
  const int D = H * Hd;
  const long rows = static_cast<long>(B) * H * Tn;
  const int warps = blockDim.x / 32, lane = threadIdx.x & 31;
  for (long r = blockIdx.x * static_cast<long>(warps) + threadIdx.x / 32; r < rows;
       r += static_cast<long>(gridDim.x) * warps) {
    const long bh = r / Tn;
    const int t = static_cast<int>(r % Tn), b = static_cast<int>(bh / H), h = static_cast<int>(bh % H);
    const long off = (static_cast<long>(b) * Tn + t) * D + h * Hd;
    float acc = 0.f;
    for (int d = lane; d < Hd; d += 32) acc += ldf(dout + off + d) * ldf(out + off + d);
    acc = wsum(acc);
    if (lane == 0) delta[r] = acc;
  }
}

// dQ. Same tiling as the forward: per query row, loop over keys <= row.
template <typename T, int DPL>
__global__ void __launch_bounds__(256) attn_bwd_dq_simt(const T* __restrict__ qkv, const T* __restrict__ dout,
                                                        const float* __restrict__ lse,
                                                        const float* __restrict__ delta, T* __restrict__ dqkv, int B,
                                                        int Tn, int H, float inv_scale) {
  constexpr int Hd = DPL * 32;
  __shared__ float sQ[kBQB][Hd];
  __shared__ float sdO[kBQB][Hd];
  __shared__ float sK[kKC][Hd + 1];
  __shared__ float sV[kKC][Hd + 1];
  const int D = H * Hd;
  const long ld = 3L * D;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kBQB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const T* base = qkv + static_cast<long>(b) * Tn * ld;
  const T* dob = dout + static_cast<long>(b) * Tn * D;
  for (int i = threadIdx.x; i < kBQB * Hd; i += blockDim.x) {
    const int r = i / Hd, d = i % Hd;
    const bool ok = q0 + r < Tn;
    sQ[r][d] = ok ? ldf(base + static_cast<long>(q0 + r) * ld + h * Hd + d) : 0.f;
    sdO[r][d] = ok ? ldf(dob + static_cast<long>(q0 + r) * D + h * Hd + d) : 0.f;
  }
  float dq[kRPW][DPL], L[kRPW], Dl[kRPW];
#pragma unroll
  for (int i = 0; i < kRPW; ++i) {
    const int row = min(q0 + warp * kRPW + i, Tn - 1);
    L[i] = lse[static_cast<long>(bh) * Tn + row];
    Dl[i] = delta[static_cast<long>(bh) * Tn + row];
#pragma unroll
    for (int j = 0; j < DPL; ++j) dq[i][j] = 0.f;
  }
  const int q_last = min(q0 + kBQB, Tn) - 1;
  for (int k0 = 0; k0 <= q_last; k0 += kKC) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKC * Hd; i += blockDim.x) {
      const int r = i / Hd, d = i % Hd;
      const bool ok = k0 + r < Tn;
      sK[r][d] = ok ? ldf(base + static_cast<long>(k0 + r) * ld + D + h * Hd + d) : 0.f;
      sV[r][d] = ok ? ldf(base + static_cast<long>(k0 + r) * ld + 2 * D + h * Hd + d) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kRPW; ++i) {
      const int r = warp * kRPW + i;
      const int row = q0 + r;
      if (row >= Tn || k0 > row) continue;
      const int key = k0 + lane;
      float s = 0.f, dp = 0.f;
#pragma unroll 16
      for (int d = 0; d < Hd; ++d) {
        s = fmaf(sQ[r][d], sK[lane][d], s);
        dp = fmaf(sdO[r][d], sV[lane][d], dp);
      }
      s = s / inv_scale;
      const bool valid = key <= row && key < Tn;
      const float p = valid ? expf(s - L[i]) : 0.f;
      const float ds = p * (dp - Dl[i]) / inv_scale;
      for (int kk = 0; kk < kKC; ++kk) {
        const float dsk = __shfl_sync(0xffffffffu, ds, kk);
#pragma unroll
        for (int j = 0; j < DPL; ++j) dq[i][j] = fmaf(dsk, sK[kk][lane + 32 * j], dq[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kRPW; ++i) {
    const int row = q0 + warp * kRPW + i;
    if (row >= Tn) continue;
    T* d = dqkv + (static_cast<long>(b) * Tn + row) * ld + h * Hd;
#pragma unroll
    for (int j = 0; j < DPL; ++j) stf(d + lane + 32 * j, dq[i][j]);
  }
}

// dK, dV. Per key row (8 per warp, 64 per CTA), loop over queries >= key.
template <typename T, int DPL>
__global__ void __launch_bounds__(256) attn_bwd_dkv_simt(const T* __restrict__ qkv, const T* __restrict__ dout,
                                                         const float* __restrict__ lse,
                                                         const float* __restrict__ delta, T* __restrict__ dqkv, int B,
                                                         int Tn, int H, float inv_scale) {
  constexpr int Hd = DPL * 32;
  __shared__ float sK[kBQB][Hd];
  __shared__ float sV[kBQB][Hd];
  __shared__ float sQ[kKC][Hd + 1];
  __shared__ float sdO[kKC][Hd + 1];
  __shared__ float sL[kKC], sD[kKC];
  const int D = H * Hd;
  const long ld = 3L * D;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int k0 = blockIdx.x * kBQB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const T* base = qkv + static_cast<long>(b) * Tn * ld;
  const T* dob = dout + static_cast<long>(b) * Tn * D;
  for (int i = threadIdx.x; i < kBQB * Hd; i += blockDim.x) {
    const int r = i / Hd, d = i % Hd;
    const bool ok = k0 + r < Tn;
    sK[r][d] = ok ? ldf(base + static_cast<long>(k0 + r) * ld + D + h * Hd + d) : 0.f;
    sV[r][d] = ok ? ldf(base + static_cast<long>(k0 + r) * ld + 2 * D + h * Hd + d) : 0.f;
  }
  float dk[kRPW][DPL], dv[kRPW][DPL];
#pragma unroll
  for (int i = 0; i < kRPW; ++i)
#pragma unroll
    for (int j = 0; j < DPL; ++j) dk[i][j] = dv[i][j] = 0.f;
  for (int qc = (k0 / kKC) * kKC; qc < Tn; qc += kKC) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKC * Hd; i += blockDim.x) {
      const int r = i / Hd, d = i % Hd;
      const bool ok = qc + r < Tn;
      sQ[r][d] = ok ? ldf(base + static_cast<long>(qc + r) * ld + h * Hd + d) : 0.f;
      sdO[r][d] = ok ? ldf(dob + static_cast<long>(qc + r) * D + h * Hd + d) : 0.f;
    }
    if (threadIdx.x < kKC) {
      const int q = qc + threadIdx.x;
      sL[threadIdx.x] = q < Tn ? lse[static_cast<long>(bh) * Tn + q] : 0.f;
      sD[threadIdx.x] = q < Tn ? delta[static_cast<long>(bh) * Tn + q] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kRPW; ++i) {
      const int r = warp * kRPW + i;
      const int key = k0 + r;
      if (key >= Tn || qc + kKC - 1 < key) continue;
      const int q = qc + lane;
      float s = 0.f, dp = 0.f;
#pragma unroll 16
      for (int d = 0; d < Hd; ++d) {
        s = fmaf(sQ[lane][d], sK[r][d], s);
        dp = fmaf(sdO[lane][d], sV[r][d], dp);
      }
      s = s / inv_scale;
      const bool valid = key <= q && q < Tn;
      const float p = valid ? expf(s - sL[lane]) : 0.f;
      const float ds = p * (dp - sD[lane]) / inv_scale;
      for (int qq = 0; qq < kKC; ++qq) {
        const float pq = __shfl_sync(0xffffffffu, p, qq);
        const float dsq = __shfl_sync(0xffffffffu, ds, qq);
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          dv[i][j] = fmaf(pq, sdO[qq][lane + 32 * j], dv[i][j]);
          dk[i][j] = fmaf(dsq, sQ[qq][lane + 32 * j], dk[i][j]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kRPW; ++i) {
    const int key = k0 + warp * kRPW + i;
    if (key >= Tn) continue;
    T* d = dqkv + (static_cast<long>(b) * Tn + key) * ld + h * Hd;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      stf(d + D + lane + 32 * j, dk[i][j]);
      stf(d + 2 * D + lane + 32 * j, dv[i][j]);
    }
  }
}

template <typename T>
int attn_fwd_t(const T* qkv, T* o, float* lse, const AttnShape& sh, cudaStream_t s) {
  dim3 grid((sh.T + kQB - 1) / kQB, sh.B * sh.H);
  const float sc = sqrtf(static_cast<float>(sh.Hd));
  switch (sh.Hd) {
    case 32: attn_fwd_simt<T, 1><<<grid, 256, 0, s>>>(qkv, o, lse, sh.B, sh.T, sh.H, sc); break;
    case 64: attn_fwd_simt<T, 2><<<grid, 256, 0, s>>>(qkv, o, lse, sh.B, sh.T, sh.H, sc); break;
    default: return 1;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

template <typename T>
int attn_bwd_t(const T* qkv, const T* o, const T* dout, const float* lse, T* dqkv, float* ws, const AttnShape& sh,
               cudaStream_t s) {
  const long rows = static_cast<long>(sh.B) * sh.H * sh.T;
  const int g = static_cast<int>(std::min<long>((rows + 7) / 8, 8L * num_sms_cached()));
  attn_delta<T><<<g, 256, 0, s>>>(o, dout, ws, sh.B, sh.T, sh.H, sh.Hd);
  dim3 grid((sh.T + kBQB - 1) / kBQB, sh.B * sh.H);
  const float sc = sqrtf(static_cast<float>(sh.Hd));
  switch (sh.Hd) {
    case 32:
      attn_bwd_dq_simt<T, 1><<<grid, 256, 0, s>>>(qkv, dout, lse, ws, dqkv, sh.B, sh.T, sh.H, sc);
      attn_bwd_dkv_simt<T, 1><<<grid, 256, 0, s>>>(qkv, dout, lse, ws, dqkv, sh.B, sh.T, sh.H, sc);
      break;
    case 64:
      attn_bwd_dq_simt<T, 2><<<grid, 256, 0, s>>>(qkv, dout, lse, ws, dqkv, sh.B, sh.T, sh.H, sc);
      attn_bwd_dkv_simt<T, 2><<<grid, 256, 0, s>>>(qkv, dout, lse, ws, dqkv, sh.B, sh.T, sh.H, sc);
      break;
    default: return 1;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace

int attention_delta_bf16(const void* o, const void* dout, float* delta, const AttnShape& sh, cudaStream_t s) {
  const long rows = static_cast<long>(sh.B) * sh.H * sh.T;
  const int g = static_cast<int>(std::min<long>((rows + 7) / 8, 8L * num_sms_cached()));
  attn_delta<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(o),
                                               static_cast<const __nv_bfloat16*>(dout), delta, sh.B, sh.T, sh.H,
                                               sh.Hd);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int attention_fwd_simt(const void* qkv, bool f32, void* o, float* lse, const AttnShape& sh, cudaStream_t s) {
  if (f32) return attn_fwd_t(static_cast<const float*>(qkv), static_cast<float*>(o), lse, sh, s);
  return attn_fwd_t(static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(o), lse, sh, s);
}

int attention_bwd_simt(const void* qkv, const void* o, const void* dout, const float* lse, bool f32, void* dqkv,
                       float* ws, const AttnShape& sh, cudaStream_t s) {
  if (f32)
    return attn_bwd_t(static_cast<const float*>(qkv), static_cast<const float*>(o), static_cast<const float*>(dout),
                      lse, static_cast<float*>(dqkv), ws, sh, s);
  return attn_bwd_t(static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(o),
                    static_cast<const __nv_bfloat16*>(dout), lse, static_cast<__nv_bfloat16*>(dqkv), ws, sh, s);
}

}  // namespace sb
