// Token sampling of nanoGPT's generate-token (examples/nanogpt/model.shf:
// 116-125) on the device, one CTA per sequence:
//   last = logits[last position] / temp; [vals idx] = top_k(last, k);
//   probs = softmax(vals); [new-key subkey] = random-split(key);
//   next = idx[choice(subkey, k, :p probs)]   (random_ops.rs:164-180)
// then the window slides by one (append-and-roll) and the key advances, so a
// CUDA graph of forward + this kernel can be replayed once per token.
//
// The PRNG is Threefry2x32-20 over keys held as four 16-bit f32 limbs
// (sheaf/src/core/prng.rs:29-97): split child i = threefry(key, [i, 1]),
// sample bits = threefry(key, [index, 0]), uniform = (bits >> 8) * 2^-24.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sb_nn.h"
#include "sb_prng.cuh"
#define SB_PDL_FAMILY 3
#include "sb_launch.cuh"

namespace sb {

namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

// a precedes b: larger value first, equal values by smaller index (stable)
__device__ __forceinline__ bool before(float va, int ia, float vb, int ib) { return va > vb || (va == vb && ia < ib); }

template <typename T>
__global__ void __launch_bounds__(256) sample_kernel(const T* __restrict__ logits, long ld, int T_, int V, int vp2,
                                                    int top_k, float temp, float* __restrict__ ids,
                                                    float* __restrict__ keys, float* __restrict__ tokens, int n_new,
                                                    int* __restrict__ step, float* __restrict__ step_logits) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sh[];
  float* vals = sh;                                    // [vp2]
  int* idx = reinterpret_cast<int*>(vals + vp2);       // [vp2]
  float* win = reinterpret_cast<float*>(idx + vp2);    // [T_]
  __shared__ float s_token;
  const int b = blockIdx.x;
  const int s = *step;
  const T* row = logits + (static_cast<long>(b) * T_ + (T_ - 1)) * ld;
  for (int v = threadIdx.x; v < vp2; v += blockDim.x) {
    if (v < V) {
      const float x = to_f32<T>(row[v]);
      if (step_logits && s < n_new) step_logits[(static_cast<long>(s) * gridDim.x + b) * V + v] = x;
      vals[v] = x / temp;  // (/ logits temp), model.shf:120
      idx[v] = v;
    } else {
      vals[v] = -INFINITY;
      idx[v] = 0x7FFFFFFF;
    }
  }
  for (int t = threadIdx.x; t < T_; t += blockDim.x) win[t] = ids[static_cast<long>(b) * T_ + t];
  __syncthreads();
  // bitonic sort, descending by (value, -index)
  for (int size = 2; size <= vp2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < vp2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float vi = vals[i], vj = vals[j];
          const int ii = idx[i], ij = idx[j];
          const bool swap = desc ? before(vj, ij, vi, ii) : before(vi, ii, vj, ij);
          if (swap) {
            vals[i] = vj;
            vals[j] = vi;
            idx[i] = ij;
            idx[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    const int k = min(top_k, V);
    // softmax over the k largest (lib/nn.shf:24-26), sums in order
    const float m = vals[0];
    float sum = 0.f;
    for (int i = 0; i < k; ++i) {
      const float e = expf(vals[i] - m);
      vals[i] = e;
      sum += e;
    }
    // [new-key subkey] = random-split(key); u = uniform(subkey, [])
    uint32_t w0, w1, n0, n1, u0, u1, bits, unused;
    key_decode(keys + 4 * b, w0, w1);
    threefry2x32(w0, w1, 0u, 1u, n0, n1);
    threefry2x32(w0, w1, 1u, 1u, u0, u1);
    threefry2x32(u0, u1, 0u, 0u, bits, unused);
    const float u = uniform_from_bits(bits);
    // choice: index = min(k - count(cumsum > u), k - 1)
    float c = 0.f;
    int count = 0;
    for (int i = 0; i < k; ++i) {
      c += vals[i] / sum;
      count += (c > u) ? 1 : 0;
    }
    const int pick = min(k - count, k - 1);
    const float token = static_cast<float>(idx[pick]);
    if (s < n_new) tokens[static_cast<long>(b) * n_new + s] = token;
    key_encode(n0, n1, keys + 4 * b);
    s_token = token;
  }
  __syncthreads();
  // append-and-roll: drop the oldest id, append the sampled one
  for (int t = threadIdx.x; t < T_; t += blockDim.x)
    ids[static_cast<long>(b) * T_ + t] = (t + 1 < T_) ? win[t + 1] : s_token;
}

__global__ void advance_step_kernel(int* step) {
  pdl_wait();
  pdl_trigger();
  *step += 1;
}

}  // namespace

int sample_step(const void* logits, bool logits_f32, long ld, int B, int T, int V, int top_k, float temperature,
                float* ids, float* keys, float* tokens, int n_new, int* step, float* step_logits, cudaStream_t s) {
  if (B <= 0 || T <= 0 || V <= 0 || top_k <= 0 || !(temperature > 0.f) || V > kSampleMaxVocab) return 1;
  int vp2 = 1;
  while (vp2 < V) vp2 <<= 1;
  const size_t smem = static_cast<size_t>(vp2) * 8 + static_cast<size_t>(T) * 4;
  if (smem > 200 * 1024) return 1;
  if (logits_f32) {
    auto k = sample_kernel<float>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    launch_pdl(k, dim3(B), dim3(256), smem, s, static_cast<const float*>(logits), ld, T, V, vp2, top_k, temperature,
               ids, keys, tokens, n_new, step, step_logits);
  } else {
    auto k = sample_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    launch_pdl(k, dim3(B), dim3(256), smem, s, static_cast<const __nv_bfloat16*>(logits), ld, T, V, vp2, top_k,
               temperature, ids, keys, tokens, n_new, step, step_logits);
  }
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  launch_pdl(advance_step_kernel, dim3(1), dim3(1), 0, s, step);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace sb
