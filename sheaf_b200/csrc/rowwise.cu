// Bandwidth-bound row-wise kernels of the nanoGPT fwd+VJP step:
//   * layer-norm without beta, forward and VJP   (examples/nanogpt/model.shf:11-14;
//     two-pass population variance, lowering/codegen/reduction_builtins.rs:287-358;
//     VJP from the `/`, `-`, `sqrt`, `var`, `mean` rules, autodiff/reverse.rs:551-583,
//     847-914, 961-967)
//   * cross-entropy loss with its VJP fused       (lib/nn.shf:28-30,44-50; one-hot
//     via iota/compare/select, lowering/stablehlo/tensor_ops.rs:163-217)
//   * token + position embedding gather and its scatter-add VJP
//     (lowering/stablehlo/indexing_ops.rs:416-484, autodiff/reverse.rs:1077-1122,
//     slice_grad/pad lowering/codegen/builtins.rs:208-271)
// All loads/stores are 128-bit vectorised where the row layout allows; row
// reductions use warp shuffles (plus shared memory across warps).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "sb_nn.h"
#define SB_PDL_FAMILY 1
#include "sb_launch.cuh"

namespace sb {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The class an f32 token id selects in a one-hot built as
// compare(id, iota) in f32 (tensor_ops.rs:163-217): the id itself when it is
// exactly an integer in [0, V), else -1 (no class: an all-zero one-hot row).
// The forward gather instead truncates and clamps (indexing_ops.rs:416-484).
__device__ __forceinline__ int one_hot_class(float f, int V) {
  const int i = static_cast<int>(f);
  return (static_cast<float>(i) == f && i >= 0 && i < V) ? i : -1;
}

template <typename T>
__device__ __forceinline__ float load1(const T* p);
template <>
__device__ __forceinline__ float load1<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load1<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ void store1(T* p, float v);
template <>
__device__ __forceinline__ void store1<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store1<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// Loads 4 consecutive elements as floats (16-byte aligned for f32, 8 for bf16).
template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x), b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float4 v);
template <>
__device__ __forceinline__ void store4<float>(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// ---------------------------------------------------------------------------
// Layer norm (no beta). One warp per row; each lane holds VPT float4 chunks
// (lane*4 + j*128). D must be a multiple of 4 and <= VPT*128.
// ---------------------------------------------------------------------------

// y = (x - mean) * rstd * gamma, rstd = 1 / sqrt(var + 1e-5); one warp per
// row, two rows per iteration so that both rows' loads are in flight.
template <int VPT, typename TO, typename TX>
__device__ __forceinline__ void ln_fwd_row(const float4 (&v)[VPT], int lane, int D, const void* gamma, int gamma_f32,
                                           TO* yr, float* mean_out, float* rstd_out, int row, TX* xc) {
  if (xc) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = lane * 4 + j * 128;
      if (c < D) store4(xc + c, v[j]);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = lane * 4 + j * 128;
    if (c < D) {
      const float a = v[j].x - mean, b = v[j].y - mean, cc = v[j].z - mean, d = v[j].w - mean;
      q += (a * a + b * b) + (cc * cc + d * d);
    }
  }
  const float var = warp_sum(q) / static_cast<float>(D);
  const float rstd = 1.0f / sqrtf(var + 1e-5f);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = lane * 4 + j * 128;
    if (c < D) {
      const float4 g = gamma_f32 ? load4(static_cast<const float*>(gamma) + c)
                                 : load4(static_cast<const __nv_bfloat16*>(gamma) + c);
      store4(yr + c, make_float4(((v[j].x - mean) * rstd) * g.x, ((v[j].y - mean) * rstd) * g.y,
                                 ((v[j].z - mean) * rstd) * g.z, ((v[j].w - mean) * rstd) * g.w));
    }
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// x (and its optional copy) is the residual stream: f32, or bf16 in a bf16
// module, as the module computes it.
template <int VPT, typename TX, typename TO>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const TX* __restrict__ x, const void* __restrict__ gamma,
                                                     int gamma_f32, TO* __restrict__ y, float* __restrict__ mean_out,
                                                     float* __restrict__ rstd_out, int rows, int D,
                                                     TX* __restrict__ x_copy) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * warps;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += 2 * stride) {
    const int row2 = row + stride;
    const bool two = row2 < rows;
    float4 v[VPT], w[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = lane * 4 + j * 128;
      v[j] = (c < D) ? load4(x + static_cast<long>(row) * D + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      w[j] = (c < D && two) ? load4(x + static_cast<long>(row2) * D + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    ln_fwd_row<VPT, TO, TX>(v, lane, D, gamma, gamma_f32, y + static_cast<long>(row) * D, mean_out, rstd_out, row,
                            x_copy ? x_copy + static_cast<long>(row) * D : nullptr);
    if (two)
      ln_fwd_row<VPT, TO, TX>(w, lane, D, gamma, gamma_f32, y + static_cast<long>(row2) * D, mean_out, rstd_out, row2,
                              x_copy ? x_copy + static_cast<long>(row2) * D : nullptr);
  }
}

// dx = rstd * (dxh - mean(dxh) - xhat * mean(dxh * xhat)), dxh = dy * gamma.
// dres_out = dres_in + dx (the residual stream's gradient, in the type of x:
// f32, or bf16 rounded once per add in a bf16 module; without ACC dres_in is
// zero and not read; it may alias dres_out: every element is read once, by the thread
// that then writes it, so the no-alias qualifiers only let loads of later
// rows move ahead of stores to earlier ones); per-block partial sums of
// dgamma = sum_rows dy * xhat into dgamma_part[blockIdx.x][D].
// x, dy and dres of a row are loaded together (the dres read does not wait
// for the row reductions); gamma is re-read from L1 per row to keep the
// register count low. Rows up to 384 wide run 24 warps per block, one block
// per SM, so there is one dgamma partial row per SM.
// Rows up to 768 wide run 12 warps per block (about 150 registers: one block
// per SM, 12 warps instead of 8), wider ones 8.
template <int VPT>
constexpr int ln_bwd_warps() { return VPT <= 3 ? 24 : VPT <= 6 ? 12 : 8; }

template <int VPT, typename TI, typename TX, bool ACC>
__global__ void __launch_bounds__(32 * ln_bwd_warps<VPT>(), 1) ln_bwd_kernel(const TI* __restrict__ dy, const TX* __restrict__ x,
                                                        const float* __restrict__ mean_in,
                                                        const float* __restrict__ rstd_in,
                                                        const void* __restrict__ gamma, int gamma_f32,
                                                        const TX* __restrict__ dres_in, TX* __restrict__ dres_out,
                                                        float* __restrict__ dgamma_part, int rows, int D) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm_dg[];  // [warps][D]
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  float4 dg[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) dg[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int row = blockIdx.x * warps + warp; row < rows; row += gridDim.x * warps) {
    const long off = static_cast<long>(row) * D;
    const float mean = mean_in[row], rstd = rstd_in[row];
    float4 xh[VPT], dxh[VPT], r[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = lane * 4 + j * 128;
      const bool in = c < D;
      xh[j] = in ? load4(x + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      dxh[j] = in ? load4(dy + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      r[j] = (ACC && in) ? load4(dres_in + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = lane * 4 + j * 128;
      if (c < D) {
        const float4 g = gamma_f32 ? load4(static_cast<const float*>(gamma) + c)
                                   : load4(static_cast<const __nv_bfloat16*>(gamma) + c);
        xh[j] = make_float4((xh[j].x - mean) * rstd, (xh[j].y - mean) * rstd, (xh[j].z - mean) * rstd,
                            (xh[j].w - mean) * rstd);
        dg[j].x += dxh[j].x * xh[j].x;
        dg[j].y += dxh[j].y * xh[j].y;
        dg[j].z += dxh[j].z * xh[j].z;
        dg[j].w += dxh[j].w * xh[j].w;
        dxh[j] = make_float4(dxh[j].x * g.x, dxh[j].y * g.y, dxh[j].z * g.z, dxh[j].w * g.w);
        s1 += (dxh[j].x + dxh[j].y) + (dxh[j].z + dxh[j].w);
        s2 += (dxh[j].x * xh[j].x + dxh[j].y * xh[j].y) + (dxh[j].z * xh[j].z + dxh[j].w * xh[j].w);
      }
    }
    const float c1 = warp_sum(s1) / static_cast<float>(D);
    const float c2 = warp_sum(s2) / static_cast<float>(D);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = lane * 4 + j * 128;
      if (c < D) {
        r[j].x += rstd * (dxh[j].x - c1 - xh[j].x * c2);
        r[j].y += rstd * (dxh[j].y - c1 - xh[j].y * c2);
        r[j].z += rstd * (dxh[j].z - c1 - xh[j].z * c2);
        r[j].w += rstd * (dxh[j].w - c1 - xh[j].w * c2);
        store4(dres_out + off + c, r[j]);
      }
    }
  }
  // reduce dgamma over the block's warps, in a fixed order
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = lane * 4 + j * 128;
    if (c < D) *reinterpret_cast<float4*>(&sm_dg[warp * D + c]) = dg[j];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < warps; ++w) acc += sm_dg[w * D + c];
    dgamma_part[static_cast<long>(blockIdx.x) * D + c] = acc;
  }
}

// ---------------------------------------------------------------------------
// Layer norm for wide rows (D >= 1024): one block per row, each thread owning
// CPT float4 column chunks (c = (j * threads + tid) * 4) of every row the
// block visits, so no thread holds more than CPT x 16 bytes of a row in
// registers and many rows are in flight per SM. Row sums go through warp
// shuffles and one shared-memory word per warp, read back in warp order by
// every thread (the same order for all rows: deterministic).
// ---------------------------------------------------------------------------

__device__ __forceinline__ float block_sum_ordered(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int warps = blockDim.x >> 5;
  for (int w = 0; w < warps; ++w) t += red[w];
  return t;
}

template <int CPT, typename TX, typename TO>
__global__ void __launch_bounds__(256) ln_fwd_wide_kernel(const TX* __restrict__ x, const void* __restrict__ gamma,
                                                          int gamma_f32, TO* __restrict__ y,
                                                          float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                          int rows, int D, TX* __restrict__ x_copy) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red1[32], red2[32];
  const int nt = blockDim.x, tid = threadIdx.x;
  float4 g[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = (j * nt + tid) * 4;
    g[j] = c < D ? (gamma_f32 ? load4(static_cast<const float*>(gamma) + c)
                              : load4(static_cast<const __nv_bfloat16*>(gamma) + c))
                 : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long off = static_cast<long>(row) * D;
    float4 v[CPT];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = (j * nt + tid) * 4;
      v[j] = c < D ? load4(x + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    if (x_copy) {
#pragma unroll
      for (int j = 0; j < CPT; ++j) {
        const int c = (j * nt + tid) * 4;
        if (c < D) store4(x_copy + off + c, v[j]);
      }
    }
    const float mean = block_sum_ordered(s, red1) / static_cast<float>(D);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = (j * nt + tid) * 4;
      if (c < D) {
        const float a = v[j].x - mean, b = v[j].y - mean, cc = v[j].z - mean, d = v[j].w - mean;
        q += (a * a + b * b) + (cc * cc + d * d);
      }
    }
    const float var = block_sum_ordered(q, red2) / static_cast<float>(D);
    const float rstd = 1.0f / sqrtf(var + 1e-5f);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = (j * nt + tid) * 4;
      if (c < D)
        store4(y + off + c, make_float4(((v[j].x - mean) * rstd) * g[j].x, ((v[j].y - mean) * rstd) * g[j].y,
                                        ((v[j].z - mean) * rstd) * g[j].z, ((v[j].w - mean) * rstd) * g[j].w));
    }
    if (tid == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

template <int CPT, typename TI, typename TX, bool ACC>
__global__ void __launch_bounds__(256) ln_bwd_wide_kernel(const TI* __restrict__ dy, const TX* __restrict__ x,
                                                          const float* __restrict__ mean_in,
                                                          const float* __restrict__ rstd_in,
                                                          const void* __restrict__ gamma, int gamma_f32,
                                                          const TX* __restrict__ dres_in, TX* __restrict__ dres_out,
                                                          float* __restrict__ dgamma_part, int rows, int D) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red1[32], red2[32];
  const int nt = blockDim.x, tid = threadIdx.x;
  float4 g[CPT], dg[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = (j * nt + tid) * 4;
    g[j] = c < D ? (gamma_f32 ? load4(static_cast<const float*>(gamma) + c)
                              : load4(static_cast<const __nv_bfloat16*>(gamma) + c))
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    dg[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long off = static_cast<long>(row) * D;
    const float mean = mean_in[row], rstd = rstd_in[row];
    float4 xh[CPT], dxh[CPT], r[CPT];
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = (j * nt + tid) * 4;
      const bool in = c < D;
      xh[j] = in ? load4(x + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      dxh[j] = in ? load4(dy + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      r[j] = (ACC && in) ? load4(dres_in + off + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = (j * nt + tid) * 4;
      if (c < D) {
        xh[j] = make_float4((xh[j].x - mean) * rstd, (xh[j].y - mean) * rstd, (xh[j].z - mean) * rstd,
                            (xh[j].w - mean) * rstd);
        dg[j].x += dxh[j].x * xh[j].x;
        dg[j].y += dxh[j].y * xh[j].y;
        dg[j].z += dxh[j].z * xh[j].z;
        dg[j].w += dxh[j].w * xh[j].w;
        dxh[j] = make_float4(dxh[j].x * g[j].x, dxh[j].y * g[j].y, dxh[j].z * g[j].z, dxh[j].w * g[j].w);
        s1 += (dxh[j].x + dxh[j].y) + (dxh[j].z + dxh[j].w);
        s2 += (dxh[j].x * xh[j].x + dxh[j].y * xh[j].y) + (dxh[j].z * xh[j].z + dxh[j].w * xh[j].w);
      }
    }
    const float c1 = block_sum_ordered(s1, red1) / static_cast<float>(D);
    const float c2 = block_sum_ordered(s2, red2) / static_cast<float>(D);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = (j * nt + tid) * 4;
      if (c < D) {
        r[j].x += rstd * (dxh[j].x - c1 - xh[j].x * c2);
        r[j].y += rstd * (dxh[j].y - c1 - xh[j].y * c2);
        r[j].z += rstd * (dxh[j].z - c1 - xh[j].z * c2);
        r[j].w += rstd * (dxh[j].w - c1 - xh[j].w * c2);
        store4(dres_out + off + c, r[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = (j * nt + tid) * 4;
    if (c < D) *reinterpret_cast<float4*>(&dgamma_part[static_cast<long>(blockIdx.x) * D + c]) = dg[j];
  }
}

// out[c] = sum_b part[b][c] in a fixed order, written as f32 or bf16. Block
// of 1024 threads per 32 columns: warp w sums partial rows w, w+32, ... (lane =
// column, coalesced), then the 32 warp sums are combined in order. Many short
// per-warp chains: the kernel is bound by load latency, not bytes.
__global__ void __launch_bounds__(1024) column_sum_kernel(const float* __restrict__ part, int nparts, long D, void* out,
                                                          int out_f32) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long c = static_cast<long>(blockIdx.x) * 32 + lane;
  float acc = 0.f;
  if (c < D) {
#pragma unroll 4
    for (int b = warp; b < nparts; b += 32) acc += part[static_cast<long>(b) * D + c];
  }
  sm[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < D) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 32; ++w) t += sm[w][lane];
    if (out_f32)
      static_cast<float*>(out)[c] = t;
    else
      static_cast<__nv_bfloat16*>(out)[c] = __float2bfloat16_rn(t);
  }
}

int column_sum(const float* part, int nparts, long D, void* out, bool out_f32, cudaStream_t s) {
  launch_pdl(column_sum_kernel, dim3(static_cast<unsigned>((D + 31) / 32)), dim3(1024), 0, s, part, nparts, D, out,
             out_f32);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

// ---------------------------------------------------------------------------
// Cross-entropy: per row r, lse = log-sum-exp, row contribution lp[y] =
// x[y] - lse, dlogits = (softmax - onehot(y)) * (1/rows). One warp per row.
// ---------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(256) ce_fwd_bwd_kernel(const T* __restrict__ logits, long ld, int rows, int V,
                                                         const float* __restrict__ targets, T* __restrict__ dlogits,
                                                         long ldd, float* __restrict__ row_part, float inv_rows) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  __shared__ float sm_part[32];
  float part = 0.f;
  for (int row = blockIdx.x * warps + warp; row < rows; row += gridDim.x * warps) {
    const T* lr = logits + static_cast<long>(row) * ld;
    float m = -INFINITY, s = 0.f;
    for (int c = lane; c < V; c += 32) {
      const float v = load1(lr + c);
      const float nm = fmaxf(m, v);
      s = s * expf(m - nm) + expf(v - nm);
      m = nm;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, m2);
      s = s * expf(m - nm) + s2 * expf(m2 - nm);
      m = nm;
    }
    const float logs = logf(s);
    // one_hot(y) compares the f32 target with an f32 iota: a fractional or
    // out-of-range target matches no class, adds nothing to the loss and
    // gets a zero gradient row ((softmax * sum(one_hot) - one_hot) / rows)
    const int y = one_hot_class(targets[row], V);
    if (lane == 0 && y >= 0) part += (load1(lr + y) - m) - logs;
    T* dr = dlogits + static_cast<long>(row) * ldd;
    const float hit = y >= 0 ? 1.f : 0.f;
    for (int c = lane; c < V; c += 32) {
      const float p = expf((load1(lr + c) - m) - logs);
      store1(dr + c, (p * hit - (c == y ? 1.f : 0.f)) * inv_rows);
    }
  }
  if (lane == 0) sm_part[warp] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int w = 0; w < warps; ++w) acc += sm_part[w];
    row_part[blockIdx.x] = acc;
  }
}

// Cross-entropy for wide rows (GPT-2's 50304-entry vocabulary): one block
// per row, 16-byte loads and stores. Pass 1 keeps an online (max, sum of
// exp) per thread over 16-byte chunks, merged across the block; pass 2
// re-reads the row (from L2: a row is at most a few hundred KB and the rows
// in flight fit in L2) and writes dlogits. The row's loss term is read by
// thread 0; each block sums its rows' terms in order into row_part.
constexpr int kCeWideThreads = 256;
constexpr int kCeWideBlocksPerSm = 3;  // the kernel's launch bound

template <typename T>
__device__ __forceinline__ void load_vec16(const T* p, float (&v)[16 / sizeof(T)]);
template <>
__device__ __forceinline__ void load_vec16<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load_vec16<float>(const float* p, float (&v)[4]) {
  const float4 u = *reinterpret_cast<const float4*>(p);
  v[0] = u.x;
  v[1] = u.y;
  v[2] = u.z;
  v[3] = u.w;
}
template <typename T>
__device__ __forceinline__ void store_vec16(T* p, const float (&v)[16 / sizeof(T)]);
template <>
__device__ __forceinline__ void store_vec16<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store_vec16<float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

// 2^x from the hardware approximation (PTX ex2.approx.ftz.f32: relative
// error about 2^-22, far below the bf16 rounding of dlogits and the f32
// parity bar).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Scores are handled in log2 units (x * log2 e), so every exponential is one
// ex2. Four 16-byte chunks per thread are loaded before any is used.
template <typename T>
__global__ void __launch_bounds__(kCeWideThreads, kCeWideBlocksPerSm) ce_wide_kernel(const T* __restrict__ logits, long ld, int rows,
                                                                 int V, const float* __restrict__ targets,
                                                                 T* __restrict__ dlogits, long ldd,
                                                                 float* __restrict__ row_part, float inv_rows) {
  pdl_wait();
  pdl_trigger();
  constexpr int E = 16 / sizeof(T);
  constexpr int W = kCeWideThreads / 32;
  constexpr int U = 4;
  constexpr float kL2e = 1.4426950408889634f;
  __shared__ float sm_m[W], sm_s[W];
  __shared__ float sm_row[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  const int nvec = V / E;  // whole 16-byte chunks; the tail (V % E) is done by scalar accesses
  float part = 0.f;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* lr = logits + static_cast<long>(row) * ld;
    float m = -INFINITY, sum = 0.f;  // running max (log2 units) and sum of 2^(x - m)
    for (int i0 = threadIdx.x; i0 < nvec; i0 += U * kCeWideThreads) {
      float v[U][E];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kCeWideThreads;
        if (i < nvec) {
          load_vec16(lr + static_cast<long>(i) * E, v[u]);
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) v[u][e] = -INFINITY;
        }
      }
      // the max over raw values (log2 e > 0 keeps the order), then one FMA
      // per value into log2 units inside the exponential
      float cm = -INFINITY;
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int e = 0; e < E; ++e) cm = fmaxf(cm, v[u][e]);
      const float nm = fmaxf(m, cm * kL2e);
      float acc = m == -INFINITY ? 0.f : sum * ex2_fast(m - nm);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int e = 0; e < E; ++e) acc += ex2_fast(fmaf(v[u][e], kL2e, -nm));
      sum = acc;
      m = nm;
    }
    for (int c = nvec * E + threadIdx.x; c < V; c += kCeWideThreads) {
      const float v = load1(lr + c) * kL2e;
      const float nm = fmaxf(m, v);
      sum = (m == -INFINITY ? 0.f : sum * ex2_fast(m - nm)) + ex2_fast(v - nm);
      m = nm;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, sum, o);
      const float nm = fmaxf(m, m2);
      // a lane that saw nothing has m = -inf, sum = 0: its term is 0
      sum = (m == -INFINITY ? 0.f : sum * ex2_fast(m - nm)) + (m2 == -INFINITY ? 0.f : s2 * ex2_fast(m2 - nm));
      m = nm;
    }
    if (lane == 0) {
      sm_m[warp] = m;
      sm_s[warp] = sum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bm = sm_m[0], bs = sm_s[0];
      for (int w = 1; w < W; ++w) {  // fixed order
        const float nm = fmaxf(bm, sm_m[w]);
        bs = (bm == -INFINITY ? 0.f : bs * ex2_fast(bm - nm)) +
             (sm_m[w] == -INFINITY ? 0.f : sm_s[w] * ex2_fast(sm_m[w] - nm));
        bm = nm;
      }
      const float lse2 = bm + log2f(bs);  // log-sum-exp in log2 units
      sm_row[0] = lse2;
      const int y = one_hot_class(targets[row], V);
      sm_row[1] = static_cast<float>(y);
      if (y >= 0) part += (load1(lr + y) * kL2e - lse2) * (1.0f / kL2e);
    }
    __syncthreads();
    const float lse2 = sm_row[0];
    const int y = static_cast<int>(sm_row[1]);
    const float hit = y >= 0 ? inv_rows : 0.f;
    // softmax / rows = 2^(x log2 e - lse2 + log2(1 / rows)); a row without a
    // class gets 2^-inf = 0
    const float off = y >= 0 ? lse2 - log2f(inv_rows) : INFINITY;
    T* dr = dlogits + static_cast<long>(row) * ldd;
    for (int i0 = threadIdx.x; i0 < nvec; i0 += U * kCeWideThreads) {
      float v[U][E];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kCeWideThreads;
        if (i < nvec) load_vec16(lr + static_cast<long>(i) * E, v[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kCeWideThreads;
        if (i < nvec) {
#pragma unroll
          for (int e = 0; e < E; ++e) v[u][e] = ex2_fast(fmaf(v[u][e], kL2e, -off));
          const int rel = y - i * E;  // the one-hot's column, if it lies in this chunk
          if (rel >= 0 && rel < E) {
#pragma unroll
            for (int e = 0; e < E; ++e)
              if (e == rel) v[u][e] -= inv_rows;
          }
          store_vec16(dr + static_cast<long>(i) * E, v[u]);
        }
      }
    }
    for (int c = nvec * E + threadIdx.x; c < V; c += kCeWideThreads)
      store1(dr + c, ex2_fast(fmaf(load1(lr + c), kL2e, -lse2)) * hit - (c == y ? inv_rows : 0.f));
    __syncthreads();  // sm_m / sm_row are rewritten by the next row
  }
  if (threadIdx.x == 0) row_part[blockIdx.x] = part;
}

// loss = -(sum of block partials) / rows, written as f32 and/or bf16.
__global__ void ce_finish_kernel(const float* __restrict__ part, int nparts, float inv_rows, float* loss_f32,
                                 __nv_bfloat16* loss_bf16) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[256];
  float acc = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) acc += part[i];
  sm[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) sm[threadIdx.x] += sm[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float loss = -sm[0] * inv_rows;
    if (loss_f32) *loss_f32 = loss;
    if (loss_bf16) *loss_bf16 = __float2bfloat16_rn(loss);
  }
}

// ---------------------------------------------------------------------------
// Embedding: x[b*T+t, :] = wte[clamp(id)] + wpe[t]   (residual stream: f32,
// or the bf16 sum a bf16 module computes)
// ---------------------------------------------------------------------------

template <typename TW, typename TX>
__global__ void embed_fwd_kernel(const float* __restrict__ ids, const TW* __restrict__ wte,
                                 const TW* __restrict__ wpe, TX* __restrict__ x, int ntok, int T, int V, int D) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  for (int n = blockIdx.x * warps + threadIdx.x / 32; n < ntok; n += gridDim.x * warps) {
    int id = static_cast<int>(ids[n]);
    id = min(max(id, 0), V - 1);
    const TW* a = wte + static_cast<long>(id) * D;
    const TW* p = wpe + static_cast<long>(n % T) * D;
    TX* o = x + static_cast<long>(n) * D;
    for (int c = lane * 4; c < D; c += 128) {
      const float4 u = load4(a + c), w = load4(p + c);
      store4(o + c, make_float4(u.x + w.x, u.y + w.y, u.z + w.z, u.w + w.w));
    }
  }
}

// dwte for a small vocabulary, deterministic: block b accumulates the tokens
// [b*chunk, (b+1)*chunk) in order into a private [V, D] copy in shared memory
// (thread = column, so no two threads touch one word), then writes it to
// part[b]; the partials are summed in block order by column_sum.
template <typename TD>
__global__ void embed_bwd_priv_kernel(const float* __restrict__ ids, const TD* __restrict__ dx, int ntok, int V,
                                      int D, int chunk, float* __restrict__ part) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float acc[];
  const int VD = V * D;
  for (int i = threadIdx.x; i < VD; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();
  const int t0 = blockIdx.x * chunk, t1 = min(ntok, t0 + chunk);
  const int c = threadIdx.x;  // one column per thread (blockDim >= D)
  for (int t = t0; t < t1; t += 8) {
    int id[8];
    float g[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int tt = t + u;
      id[u] = (tt < t1) ? one_hot_class(ids[tt], V) : -1;
      g[u] = (tt < t1 && c < D) ? load1(dx + static_cast<long>(tt) * D + c) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (id[u] >= 0 && id[u] < V && c < D) acc[id[u] * D + c] += g[u];
  }
  __syncthreads();
  float* p = part + static_cast<long>(blockIdx.x) * VD;
  for (int i = threadIdx.x; i < VD; i += blockDim.x) p[i] = acc[i];
}

constexpr int kEmbedPrivBlocks = 148;

// dwte for a large vocabulary: fp32 atomics into a zeroed f32 accumulator.
template <typename TD>
__global__ void embed_bwd_atomic_kernel(const float* __restrict__ ids, const TD* __restrict__ dx, int ntok, int V,
                                        int D, float* __restrict__ acc) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  for (int n = blockIdx.x * warps + threadIdx.x / 32; n < ntok; n += gridDim.x * warps) {
    const int id = one_hot_class(ids[n], V);
    if (id < 0) continue;
    const TD* g = dx + static_cast<long>(n) * D;
    float* o = acc + static_cast<long>(id) * D;
    for (int c = lane; c < D; c += 32) atomicAdd(o + c, load1(g + c));
  }
}

// one_hot(ids, V) as the reference's embedding VJP builds it (compare of the
// f32 id with an f32 iota, tensor_ops.rs:163-217), bf16 [ntok, Vp]; columns
// V..Vp-1 are zero. Its transpose times the token gradients is dwte
// (reverse.rs:1108-1121).
__global__ void onehot_kernel(const float* __restrict__ ids, int ntok, int V, int Vp, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const long total = static_cast<long>(ntok) * Vp;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long n = i / Vp;
    const int v = static_cast<int>(i % Vp);
    out[i] = __float2bfloat16_rn(one_hot_class(ids[n], V) == v ? 1.f : 0.f);
  }
}

// dwpe[t, :] = sum_b dx[b*T + t, :] for t < T; rows T..P-1 are zero (pad).
template <typename TD>
__global__ void embed_bwd_pos_kernel(const TD* __restrict__ dx, int B, int T, int P, int D, void* dwpe,
                                     int out_f32) {
  pdl_wait();
  pdl_trigger();
  const long total = static_cast<long>(P) * D;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long t = i / D, c = i % D;
    float acc = 0.f;
    if (t < T) {
      // eight rows' loads in flight, summed in batch order
      int b = 0;
      for (; b + 8 <= B; b += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = load1(dx + (static_cast<long>(b + u) * T + t) * D + c);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc += v[u];
      }
      for (; b < B; ++b) acc += load1(dx + (static_cast<long>(b) * T + t) * D + c);
    }
    if (out_f32)
      static_cast<float*>(dwpe)[i] = acc;
    else
      static_cast<__nv_bfloat16*>(dwpe)[i] = __float2bfloat16_rn(acc);
  }
}

// Standalone GELU (tanh form, lib/nn.shf:10-11) and its VJP, 8 elements per
// thread per iteration (16-byte bf16 / 2 x 16-byte f32 accesses).
__device__ __forceinline__ float gelu_f(float x) {
  const float inner = x + 0.044715f * (x * (x * x));
  return 0.5f * (x * (1.0f + tanhf(0.7978846f * inner)));
}
__device__ __forceinline__ float gelu_df(float x) {
  const float x2 = x * x;
  const float t = tanhf(0.7978846f * (x + 0.044715f * (x * x2)));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * 0.7978846f * (1.0f + 0.134145f * x2);
}

template <typename T, bool BWD>
__global__ void gelu_kernel(const T* __restrict__ x, const T* __restrict__ g, T* __restrict__ y, long n) {
  pdl_wait();
  pdl_trigger();
  const long n8 = n / 8;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float4 a0 = load4(x + 8 * i), a1 = load4(x + 8 * i + 4);
    float4 r0, r1;
    if (BWD) {
      const float4 g0 = load4(g + 8 * i), g1 = load4(g + 8 * i + 4);
      r0 = make_float4(g0.x * gelu_df(a0.x), g0.y * gelu_df(a0.y), g0.z * gelu_df(a0.z), g0.w * gelu_df(a0.w));
      r1 = make_float4(g1.x * gelu_df(a1.x), g1.y * gelu_df(a1.y), g1.z * gelu_df(a1.z), g1.w * gelu_df(a1.w));
    } else {
      r0 = make_float4(gelu_f(a0.x), gelu_f(a0.y), gelu_f(a0.z), gelu_f(a0.w));
      r1 = make_float4(gelu_f(a1.x), gelu_f(a1.y), gelu_f(a1.z), gelu_f(a1.w));
    }
    store4(y + 8 * i, r0);
    store4(y + 8 * i + 4, r1);
  }
  for (long i = n8 * 8 + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float a = load1(x + i);
    store1(y + i, BWD ? load1(g + i) * gelu_df(a) : gelu_f(a));
  }
}

// bf16 GELU / GELU-VJP: 16-byte loads and stores (8 values), tanh from the
// hardware approximation (PTX tanh.approx.f32, one MUFU op; its relative
// error, about 2^-11, is below the bf16 rounding of the result). The f32
// path keeps tanhf.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BWD>
__global__ void __launch_bounds__(256) gelu_bf16_kernel(const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ g,
                                                        __nv_bfloat16* __restrict__ y, long n) {
  pdl_wait();
  pdl_trigger();
  const long n8 = n / 8;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float a[8], gv[8], r[8];
    load_vec16(x + 8 * i, a);
    if (BWD) load_vec16(g + 8 * i, gv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = a[e], v2 = v * v;
      const float t = tanh_fast(0.7978846f * (v + 0.044715f * (v * v2)));
      if (BWD)
        r[e] = gv[e] * (0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * 0.7978846f * (1.0f + 0.134145f * v2));
      else
        r[e] = 0.5f * (v * (1.0f + t));
    }
    store_vec16(y + 8 * i, r);
  }
  for (long i = n8 * 8 + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float v = __bfloat162float(x[i]), v2 = v * v;
    const float t = tanh_fast(0.7978846f * (v + 0.044715f * (v * v2)));
    const float r = BWD ? __bfloat162float(g[i]) *
                              (0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * 0.7978846f * (1.0f + 0.134145f * v2))
                        : 0.5f * (v * (1.0f + t));
    y[i] = __float2bfloat16_rn(r);
  }
}

__global__ void convert_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, long n) {
  pdl_wait();
  pdl_trigger();
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

int grid_for(long work_items, int per_block) {
  const long b = (work_items + per_block - 1) / per_block;
  return static_cast<int>(std::max<long>(1, std::min<long>(b, 16L * num_sms_cached())));
}

}  // namespace

int num_sms_cached() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

#define SB_LN_DISPATCH(VPT_EXPR, LAUNCH)          \
  do {                                            \
    const int vpt_ = (VPT_EXPR);                  \
    if (vpt_ <= 1) { constexpr int V = 1; LAUNCH; } \
    else if (vpt_ <= 2) { constexpr int V = 2; LAUNCH; } \
    else if (vpt_ <= 3) { constexpr int V = 3; LAUNCH; } \
    else if (vpt_ <= 4) { constexpr int V = 4; LAUNCH; } \
    else if (vpt_ <= 6) { constexpr int V = 6; LAUNCH; } \
    else if (vpt_ <= 8) { constexpr int V = 8; LAUNCH; } \
    else if (vpt_ <= 16) { constexpr int V = 16; LAUNCH; } \
    else if (vpt_ <= 32) { constexpr int V = 32; LAUNCH; } \
    else return 1;                                \
  } while (0)

// Rows at least this wide take the block-per-row kernels.
constexpr int kLnWideMin = 1024;

namespace {
// Threads per row (a multiple of 32, at most 256) and float4 chunks per
// thread of the wide layer-norm kernels.
int ln_wide_threads(int D) { return std::min(256, (D / 4 + 31) / 32 * 32); }
int ln_wide_cpt(int D) { return (D / 4 + ln_wide_threads(D) - 1) / ln_wide_threads(D); }
int ln_wide_grid(int rows) { return std::max(1, std::min(rows, 4 * num_sms_cached())); }
}  // namespace

#define SB_LN_WIDE_DISPATCH(CPT_EXPR, LAUNCH)              \
  do {                                                     \
    const int cpt_ = (CPT_EXPR);                           \
    if (cpt_ <= 1) { constexpr int C = 1; LAUNCH; }        \
    else if (cpt_ <= 2) { constexpr int C = 2; LAUNCH; }   \
    else if (cpt_ <= 4) { constexpr int C = 4; LAUNCH; }   \
    else if (cpt_ <= 8) { constexpr int C = 8; LAUNCH; }   \
    else return 1;                                         \
  } while (0)

namespace {
template <typename TX, typename TO>
int layernorm_fwd_t(const TX* x, const void* gamma, bool gamma_f32, TO* y, float* mean, float* rstd, int rows, int D,
                    cudaStream_t s, TX* x_copy) {
  if (D >= kLnWideMin) {
    const int nt = ln_wide_threads(D), grid = ln_wide_grid(rows);
    SB_LN_WIDE_DISPATCH(ln_wide_cpt(D), (launch_pdl((ln_fwd_wide_kernel<C, TX, TO>), dim3(grid), dim3(nt), 0, s, x,
                                                    gamma, gamma_f32, y, mean, rstd, rows, D, x_copy)));
  } else {
    const int warps = 8;
    const int grid = std::min((rows + 2 * warps - 1) / (2 * warps), 4 * num_sms_cached());
    SB_LN_DISPATCH((D + 127) / 128, (launch_pdl((ln_fwd_kernel<V, TX, TO>), dim3(grid), dim3(warps * 32), 0, s, x,
                                                gamma, gamma_f32, y, mean, rstd, rows, D, x_copy)));
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}
}  // namespace

int layernorm_fwd(const void* x, bool x_f32, const void* gamma, bool gamma_f32, void* y, bool y_f32, float* mean,
                  float* rstd, int rows, int D, cudaStream_t s, void* x_copy) {
  if (rows <= 0 || D <= 0 || (D & 3)) return 1;
  using bf = __nv_bfloat16;
  if (x_f32) {
    const float* xf = static_cast<const float*>(x);
    float* cf = static_cast<float*>(x_copy);
    return y_f32 ? layernorm_fwd_t(xf, gamma, gamma_f32, static_cast<float*>(y), mean, rstd, rows, D, s, cf)
                 : layernorm_fwd_t(xf, gamma, gamma_f32, static_cast<bf*>(y), mean, rstd, rows, D, s, cf);
  }
  if (y_f32) return 1;  // a bf16 residual stream feeds bf16 outputs only
  return layernorm_fwd_t(static_cast<const bf*>(x), gamma, gamma_f32, static_cast<bf*>(y), mean, rstd, rows, D, s,
                         static_cast<bf*>(x_copy));
}

namespace {
// Blocks of the layer-norm VJP: one per SM (fewer for short inputs).
int ln_bwd_grid(int rows, int warps) { return std::max(1, std::min((rows + warps - 1) / warps, num_sms_cached())); }
int ln_bwd_warps_for(int D) {
  const int vpt = (D + 127) / 128;
  return vpt <= 3 ? 24 : vpt <= 6 ? 12 : 8;
}
}  // namespace

size_t layernorm_bwd_workspace_bytes(int rows, int D) {
  if (D >= kLnWideMin) return static_cast<size_t>(ln_wide_grid(rows)) * D * sizeof(float);
  return static_cast<size_t>(ln_bwd_grid(rows, ln_bwd_warps_for(D))) * D * sizeof(float);
}

namespace {
template <typename TI, typename TX>
int layernorm_bwd_t(const TI* dy, const TX* x, const float* mean, const float* rstd, const void* gamma,
                    bool gamma_f32, const TX* __restrict__ dres_in, TX* __restrict__ dres_out, void* dgamma, bool dgamma_f32, float* ws,
                    int rows, int D, cudaStream_t s) {
  if (D >= kLnWideMin) {
    const int nt = ln_wide_threads(D), grid = ln_wide_grid(rows);
    if (dres_in)
      SB_LN_WIDE_DISPATCH(ln_wide_cpt(D), (launch_pdl((ln_bwd_wide_kernel<C, TI, TX, true>), dim3(grid), dim3(nt), 0, s,
                                                      dy, x, mean, rstd, gamma, gamma_f32, dres_in, dres_out, ws, rows,
                                                      D)));
    else
      SB_LN_WIDE_DISPATCH(ln_wide_cpt(D), (launch_pdl((ln_bwd_wide_kernel<C, TI, TX, false>), dim3(grid), dim3(nt), 0,
                                                      s, dy, x, mean, rstd, gamma, gamma_f32, dres_in, dres_out, ws,
                                                      rows, D)));
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
    return column_sum(ws, grid, D, dgamma, dgamma_f32, s);
  }
  const int warps = ln_bwd_warps_for(D);
  const int grid = ln_bwd_grid(rows, warps);
  const size_t smem = static_cast<size_t>(warps) * D * sizeof(float);
  if (smem > 200 * 1024) return 1;
  SB_LN_DISPATCH((D + 127) / 128, ({
    auto k = dres_in ? ln_bwd_kernel<V, TI, TX, true> : ln_bwd_kernel<V, TI, TX, false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    launch_pdl(k, dim3(grid), dim3(warps * 32), smem, s, dy, x, mean, rstd, gamma, gamma_f32, dres_in, dres_out, ws,
               rows, D);
  }));
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  return column_sum(ws, grid, D, dgamma, dgamma_f32, s);
}
}  // namespace

int layernorm_bwd(const void* dy, bool dy_f32, const void* x, bool x_f32, const float* mean, const float* rstd,
                  const void* gamma, bool gamma_f32, const void* dres_in, void* dres_out, void* dgamma,
                  bool dgamma_f32, float* ws, int rows, int D, cudaStream_t s) {
  if (rows <= 0 || D <= 0 || (D & 3) || !dres_out) return 1;
  using bf = __nv_bfloat16;
  if (x_f32) {
    const float* xf = static_cast<const float*>(x);
    const float* ri = static_cast<const float*>(dres_in);
    float* ro = static_cast<float*>(dres_out);
    return dy_f32 ? layernorm_bwd_t(static_cast<const float*>(dy), xf, mean, rstd, gamma, gamma_f32, ri, ro, dgamma,
                                    dgamma_f32, ws, rows, D, s)
                  : layernorm_bwd_t(static_cast<const bf*>(dy), xf, mean, rstd, gamma, gamma_f32, ri, ro, dgamma,
                                    dgamma_f32, ws, rows, D, s);
  }
  if (dy_f32) return 1;  // a bf16 residual stream comes with bf16 gradients
  return layernorm_bwd_t(static_cast<const bf*>(dy), static_cast<const bf*>(x), mean, rstd, gamma, gamma_f32,
                         static_cast<const bf*>(dres_in), static_cast<bf*>(dres_out), dgamma, dgamma_f32, ws, rows, D,
                         s);
}

// Same VJP with the number of blocks capped at `max_blocks`, so that the
// dgamma partial sums fit a caller-provided scratch of max_blocks * D floats.
int layernorm_bwd_capped(const float* dy, const float* x, const float* mean, const float* rstd, const void* gamma,
                         bool gamma_f32, float* dres, void* dgamma, bool dgamma_f32, float* scratch, int max_blocks,
                         int rows, int D, cudaStream_t s) {
  if (rows <= 0 || D <= 0 || (D & 3) || max_blocks <= 0) return 1;
  if (D >= kLnWideMin) {  // the kernel layernorm_bwd uses at this width, on fewer blocks
    const int nt = ln_wide_threads(D), grid = std::min(ln_wide_grid(rows), max_blocks);
    SB_LN_WIDE_DISPATCH(ln_wide_cpt(D), (launch_pdl((ln_bwd_wide_kernel<C, float, float, true>), dim3(grid), dim3(nt), 0, s, dy, x,
                                                    mean, rstd, gamma, gamma_f32, dres, dres, scratch, rows, D)));
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
    return column_sum(scratch, grid, D, dgamma, dgamma_f32, s);
  }
  const int warps = 8;
  const int grid = std::min(std::min((rows + warps - 1) / warps, 2 * num_sms_cached()), max_blocks);
  const size_t smem = static_cast<size_t>(warps) * D * sizeof(float);
  if (smem > 200 * 1024) return 1;
  SB_LN_DISPATCH((D + 127) / 128, ({
    auto k = ln_bwd_kernel<V, float, float, true>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    launch_pdl(k, dim3(grid), dim3(warps * 32), smem, s, dy, x, mean, rstd, gamma, gamma_f32, dres, dres, scratch,
               rows, D);
  }));
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  return column_sum(scratch, grid, D, dgamma, dgamma_f32, s);
}

size_t cross_entropy_workspace_bytes(int rows) {
  return static_cast<size_t>(std::min((rows + 7) / 8, 4 * num_sms_cached())) * sizeof(float);
}

int cross_entropy_fwd_bwd(const void* logits, bool f32, long ld, int rows, int V, const float* targets, void* dlogits,
                          long ldd, float* ws, float* loss_f32, __nv_bfloat16* loss_bf16, cudaStream_t s) {
  if (rows <= 0 || V <= 0) return 1;
  const int warps = 8;
  int grid = std::min((rows + warps - 1) / warps, 4 * num_sms_cached());
  const float inv = 1.0f / static_cast<float>(rows);
  const size_t es = f32 ? 4 : 2;
  const bool aligned = ((reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(dlogits) |
                         (static_cast<uintptr_t>(ld) * es) | (static_cast<uintptr_t>(ldd) * es)) & 15) == 0;
  if (V >= 2048 && aligned) {
    // a block per row, grid-striding over rows. bf16: one wave of resident
    // blocks (kCeWideBlocksPerSm per SM), so that no second, partial wave
    // runs its rows at a third of the occupancy (GPT-2-small's logits: 454 ->
    // 383 us); f32 rows, twice the bytes, measured faster with the longer
    // grid (742 vs 771 us). The grid stays <= the workspace's partial count.
    if (!f32) grid = std::min(grid, kCeWideBlocksPerSm * num_sms_cached());
    if (f32)
      launch_pdl((ce_wide_kernel<float>), dim3(grid), dim3(kCeWideThreads), 0, s, static_cast<const float*>(logits),
                 ld, rows, V, targets, static_cast<float*>(dlogits), ldd, ws, inv);
    else
      launch_pdl((ce_wide_kernel<__nv_bfloat16>), dim3(grid), dim3(kCeWideThreads), 0, s,
                 static_cast<const __nv_bfloat16*>(logits), ld, rows, V, targets,
                 static_cast<__nv_bfloat16*>(dlogits), ldd, ws, inv);
  } else if (f32)
    launch_pdl((ce_fwd_bwd_kernel<float>), dim3(grid), dim3(warps * 32), 0, s, static_cast<const float*>(logits), ld,
               rows, V, targets, static_cast<float*>(dlogits), ldd, ws, inv);
  else
    launch_pdl((ce_fwd_bwd_kernel<__nv_bfloat16>), dim3(grid), dim3(warps * 32), 0, s,
               static_cast<const __nv_bfloat16*>(logits), ld, rows, V, targets, static_cast<__nv_bfloat16*>(dlogits),
               ldd, ws, inv);
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  launch_pdl(ce_finish_kernel, dim3(1), dim3(256), 0, s, ws, grid, inv, loss_f32, loss_bf16);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int embedding_fwd(const float* ids, const void* wte, const void* wpe, bool f32, void* x, bool x_f32, int ntok, int T,
                  int V, int D, cudaStream_t s) {
  if (ntok <= 0 || (D & 3)) return 1;
  using bf = __nv_bfloat16;
  const int grid = std::min((ntok + 7) / 8, 8 * num_sms_cached());
  if (f32 && x_f32)
    launch_pdl((embed_fwd_kernel<float, float>), dim3(grid), dim3(256), 0, s, ids, static_cast<const float*>(wte),
               static_cast<const float*>(wpe), static_cast<float*>(x), ntok, T, V, D);
  else if (!f32 && x_f32)
    launch_pdl((embed_fwd_kernel<bf, float>), dim3(grid), dim3(256), 0, s, ids, static_cast<const bf*>(wte),
               static_cast<const bf*>(wpe), static_cast<float*>(x), ntok, T, V, D);
  else if (!f32)
    launch_pdl((embed_fwd_kernel<bf, bf>), dim3(grid), dim3(256), 0, s, ids, static_cast<const bf*>(wte),
               static_cast<const bf*>(wpe), static_cast<bf*>(x), ntok, T, V, D);
  else
    return 1;  // f32 tables feed an f32 residual stream
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

static bool embed_small(int V, int D) { return static_cast<size_t>(V) * D * sizeof(float) <= 160 * 1024 && D <= 1024; }

size_t embedding_bwd_workspace_bytes(int V, int D) {
  return embed_small(V, D) ? static_cast<size_t>(kEmbedPrivBlocks) * V * D * sizeof(float)
                           : static_cast<size_t>(V) * D * sizeof(float);
}

namespace {
template <typename TD>
int embedding_bwd_t(const float* ids, const TD* dx, int B, int T, int P, int V, int D, void* dwte, void* dwpe,
                    bool out_f32, float* ws, cudaStream_t s) {
  const int ntok = B * T;
  if (embed_small(V, D)) {
    if (!ws) return 5;
    const int chunk = (ntok + kEmbedPrivBlocks - 1) / kEmbedPrivBlocks;
    const size_t smem = static_cast<size_t>(V) * D * sizeof(float);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(embed_bwd_priv_kernel<TD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    launch_pdl(embed_bwd_priv_kernel<TD>, dim3(kEmbedPrivBlocks), dim3((D + 31) / 32 * 32), smem, s, ids, dx, ntok, V,
               D, chunk, ws);
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
    if (column_sum(ws, kEmbedPrivBlocks, static_cast<long>(V) * D, dwte, out_f32, s)) return 4;
  } else {
    float* acc = out_f32 ? static_cast<float*>(dwte) : ws;
    if (!acc) return 5;
    cudaMemsetAsync(acc, 0, static_cast<size_t>(V) * D * sizeof(float), s);
    launch_pdl(embed_bwd_atomic_kernel<TD>, dim3(std::min((ntok + 7) / 8, 8 * num_sms_cached())), dim3(256), 0, s,
               ids, dx, ntok, V, D, acc);
    if (!out_f32) {
      const long n = static_cast<long>(V) * D;
      launch_pdl(convert_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, acc, static_cast<__nv_bfloat16*>(dwte), n);
    }
  }
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  const long total = static_cast<long>(P) * D;
  launch_pdl(embed_bwd_pos_kernel<TD>, dim3(grid_for(total, 256)), dim3(256), 0, s, dx, B, T, P, D, dwpe,
             static_cast<int>(out_f32));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}
}  // namespace

int embedding_bwd(const float* ids, const void* dx, bool dx_f32, int B, int T, int P, int V, int D, void* dwte,
                  void* dwpe, bool out_f32, float* ws, cudaStream_t s) {
  return dx_f32 ? embedding_bwd_t(ids, static_cast<const float*>(dx), B, T, P, V, D, dwte, dwpe, out_f32, ws, s)
                : embedding_bwd_t(ids, static_cast<const __nv_bfloat16*>(dx), B, T, P, V, D, dwte, dwpe, out_f32, ws,
                                  s);
}

int embedding_onehot(const float* ids, int ntok, int V, int Vp, __nv_bfloat16* out, cudaStream_t s) {
  if (ntok <= 0 || V <= 0 || Vp < V) return 1;
  const long n = static_cast<long>(ntok) * Vp;
  launch_pdl(onehot_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, ids, ntok, V, Vp, out);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int embedding_pos_bwd(const void* dx, bool dx_f32, int B, int T, int P, int D, void* dwpe, bool out_f32,
                      cudaStream_t s) {
  const long total = static_cast<long>(P) * D;
  if (dx_f32)
    launch_pdl(embed_bwd_pos_kernel<float>, dim3(grid_for(total, 256)), dim3(256), 0, s,
               static_cast<const float*>(dx), B, T, P, D, dwpe, static_cast<int>(out_f32));
  else
    launch_pdl(embed_bwd_pos_kernel<__nv_bfloat16>, dim3(grid_for(total, 256)), dim3(256), 0, s,
               static_cast<const __nv_bfloat16*>(dx), B, T, P, D, dwpe, static_cast<int>(out_f32));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int gelu(const void* x, const void* g, void* y, bool f32, bool bwd, long n, cudaStream_t s) {
  if (n <= 0) return 1;
  const int blocks = grid_for((n + 7) / 8, 256);
  if (f32) {
    if (bwd)
      launch_pdl((gelu_kernel<float, true>), dim3(blocks), dim3(256), 0, s, static_cast<const float*>(x),
                 static_cast<const float*>(g), static_cast<float*>(y), n);
    else
      launch_pdl((gelu_kernel<float, false>), dim3(blocks), dim3(256), 0, s, static_cast<const float*>(x), nullptr,
                 static_cast<float*>(y), n);
  } else {
    using B = __nv_bfloat16;
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                      (bwd ? reinterpret_cast<uintptr_t>(g) : 0)) & 15) == 0;
    if (al && bwd)
      launch_pdl((gelu_bf16_kernel<true>), dim3(blocks), dim3(256), 0, s, static_cast<const B*>(x),
                 static_cast<const B*>(g), static_cast<B*>(y), n);
    else if (al)
      launch_pdl((gelu_bf16_kernel<false>), dim3(blocks), dim3(256), 0, s, static_cast<const B*>(x), nullptr,
                 static_cast<B*>(y), n);
    else if (bwd)
      launch_pdl((gelu_kernel<B, true>), dim3(blocks), dim3(256), 0, s, static_cast<const B*>(x),
                 static_cast<const B*>(g), static_cast<B*>(y), n);
    else
      launch_pdl((gelu_kernel<B, false>), dim3(blocks), dim3(256), 0, s, static_cast<const B*>(x), nullptr,
                 static_cast<B*>(y), n);
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int convert_f32_to_bf16(const float* in, __nv_bfloat16* out, long n, cudaStream_t s) {
  launch_pdl(convert_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, in, out, n);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace sb
