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

#include "hlo_kernels.h"
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

// ---- vocabularies beyond one CTA's shared-memory sort (GPT-2's 50304) ----
// logits / temp of every sequence's last position go to a [B, V] buffer
// (recording the raw logits too), are sorted per sequence with the stable
// chunked merge sort (value descending, index ascending on ties), and one
// CTA per sequence then takes the softmax over the k largest, the cumulative
// sum and the choice with block-wide scans.

template <typename T>
__global__ void sample_prep_kernel(const T* __restrict__ logits, long ld, int T_, int V, float temp,
                                   const int* __restrict__ step, int n_new, float* __restrict__ step_logits,
                                   float* __restrict__ vals) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int s = *step;
  const T* row = logits + (static_cast<long>(b) * T_ + (T_ - 1)) * ld;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V; v += gridDim.x * blockDim.x) {
    const float x = to_f32<T>(row[v]);
    if (step_logits && s < n_new) step_logits[(static_cast<long>(s) * gridDim.y + b) * V + v] = x;
    vals[static_cast<long>(b) * V + v] = x / temp;  // (/ logits temp), model.shf:120
  }
}

constexpr int kSampleWideThreads = 1024;

// Inclusive scan of one value per thread over the block (fixed order).
__device__ __forceinline__ float block_inclusive_scan(float v, float* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  float before = 0.f;
  for (int w = 0; w < warp; ++w) before += warp_tot[w];
  __syncthreads();
  return v + before;
}

__global__ void __launch_bounds__(kSampleWideThreads) sample_wide_kernel(
    const float* __restrict__ sorted, const int32_t* __restrict__ order, int T_, int V, int top_k,
    float* __restrict__ ids, float* __restrict__ keys, float* __restrict__ tokens, int n_new,
    const int* __restrict__ step) {
  pdl_wait();
  pdl_trigger();
  __shared__ float warp_tot[32];
  __shared__ int s_first;
  __shared__ float s_token;
  const int b = blockIdx.x;
  const int s = *step;
  const int k = min(top_k, V);
  const float* vb = sorted + static_cast<long>(b) * V;
  const float m = vb[0];
  // thread t owns the contiguous run [t*per, (t+1)*per) of the k sorted values
  const int per = (k + kSampleWideThreads - 1) / kSampleWideThreads;
  const int lo = min(k, threadIdx.x * per), hi = min(k, lo + per);
  float part = 0.f;
  for (int i = lo; i < hi; ++i) part += expf(vb[i] - m);
  const float incl = block_inclusive_scan(part, warp_tot);
  if (threadIdx.x == blockDim.x - 1) warp_tot[31] = incl;  // the total (written after the scan's last read)
  __syncthreads();
  const float sum = warp_tot[31];
  // [new-key subkey] = random-split(key); u = uniform(subkey, [])
  uint32_t w0, w1, n0, n1, u0, u1, bits, unused;
  key_decode(keys + 4 * b, w0, w1);
  threefry2x32(w0, w1, 0u, 1u, n0, n1);
  threefry2x32(w0, w1, 1u, 1u, u0, u1);
  threefry2x32(u0, u1, 0u, 0u, bits, unused);
  const float u = uniform_from_bits(bits);
  // choice: the first index whose cumulative probability exceeds u
  // (= min(k - count(cumsum > u), k - 1), the cumsum being non-decreasing)
  if (threadIdx.x == 0) s_first = k - 1;
  __syncthreads();
  float run = incl - part;
  for (int i = lo; i < hi; ++i) {
    run += expf(vb[i] - m);
    if (run / sum > u) {
      atomicMin(&s_first, i);
      break;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float token = static_cast<float>(order[static_cast<long>(b) * V + s_first]);
    if (s < n_new) tokens[static_cast<long>(b) * n_new + s] = token;
    key_encode(n0, n1, keys + 4 * b);
    s_token = token;
  }
  __syncthreads();
  // append-and-roll (read the whole window before any thread writes)
  float* win = ids + static_cast<long>(b) * T_;
  float mine[4];
  int cnt = 0;
  for (int t = threadIdx.x; t < T_ && cnt < 4; t += blockDim.x) mine[cnt++] = (t + 1 < T_) ? win[t + 1] : s_token;
  __syncthreads();
  cnt = 0;
  for (int t = threadIdx.x; t < T_ && cnt < 4; t += blockDim.x) win[t] = mine[cnt++];
}

__global__ void advance_step_kernel(int* step) {
  pdl_wait();
  pdl_trigger();
  *step += 1;
}

}  // namespace

size_t sample_workspace_bytes(int B, int V) {
  if (V <= kSampleSmemVocab) return 0;
  const size_t bv = static_cast<size_t>(B) * V;
  return 2 * bv * sizeof(float) + bv * sizeof(int32_t) + 256 * 3 + hlo::sort_rows_workspace_bytes(B, V);
}

int sample_step(const void* logits, bool logits_f32, long ld, int B, int T, int V, int top_k, float temperature,
                float* ids, float* keys, float* tokens, int n_new, int* step, float* step_logits, void* ws,
                size_t ws_bytes, cudaStream_t s) {
  if (B <= 0 || T <= 0 || V <= 0 || top_k <= 0 || !(temperature > 0.f) || V > kSampleMaxVocab) return 1;
  if (V > kSampleSmemVocab) {
    if (!ws || ws_bytes < sample_workspace_bytes(B, V) || T > 4 * kSampleWideThreads || B > 65535) return 1;
    const size_t bv = static_cast<size_t>(B) * V;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    char* w = static_cast<char*>(ws);
    float* vals = reinterpret_cast<float*>(w);
    float* sorted = reinterpret_cast<float*>(w + up(bv * 4));
    int32_t* order = reinterpret_cast<int32_t*>(w + up(bv * 4) * 2);
    void* sort_ws = w + up(bv * 4) * 2 + up(bv * 4);
    const size_t sort_bytes = hlo::sort_rows_workspace_bytes(B, V);
    const dim3 pg(static_cast<unsigned>((V + 255) / 256), static_cast<unsigned>(B));
    if (logits_f32)
      launch_pdl(sample_prep_kernel<float>, pg, dim3(256), 0, s, static_cast<const float*>(logits), ld, T, V,
                 temperature, step, n_new, step_logits, vals);
    else
      launch_pdl(sample_prep_kernel<__nv_bfloat16>, pg, dim3(256), 0, s, static_cast<const __nv_bfloat16*>(logits),
                 ld, T, V, temperature, step, n_new, step_logits, vals);
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
    if (int rc = hlo::sort_rows(vals, hlo::DT_F32, nullptr, sorted, order, B, V, true, sort_ws, sort_bytes, s))
      return rc;
    launch_pdl(sample_wide_kernel, dim3(B), dim3(kSampleWideThreads), 0, s, sorted, order, T, V, top_k, ids, keys,
               tokens, n_new, step);
    if (cudaPeekAtLastError() != cudaSuccess) return 4;
    launch_pdl(advance_step_kernel, dim3(1), dim3(1), 0, s, step);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
  }
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
