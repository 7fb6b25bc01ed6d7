// Optimizer step of nanoGPT's train-step (examples/nanogpt/train.shf:26-33):
// clip-by-global-norm (lib/optim.shf:42-51) then adamw-step
// (lib/optim.shf:19-32), over every parameter leaf at once.
//
// The leaves are cut into chunks of kChunk elements (a chunk never spans two
// leaves). Pass 1 writes one sum of g*g per chunk; a single-thread pass sums
// the chunk partials in chunk order (deterministic for any grid) and derives
// the device scalars the update reads: clip factor, t + 1 and the two bias
// corrections. Pass 2 updates p, m, v elementwise. Everything stays on the
// device, so the whole step can sit in a CUDA graph.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "sb_nn.h"
#define SB_PDL_FAMILY 3
#include "sb_launch.cuh"

namespace sb {

namespace {

constexpr int kChunk = 4096;
constexpr int kThreads = 256;
constexpr int kOptLeavesPerLaunch = 32;  // leaf table passed by value to each launch

struct OptLeaves {
  const void* g[kOptLeavesPerLaunch];
  const void* p[kOptLeavesPerLaunch];
  const void* m[kOptLeavesPerLaunch];
  const void* v[kOptLeavesPerLaunch];
  void* p_out[kOptLeavesPerLaunch];
  void* m_out[kOptLeavesPerLaunch];
  void* v_out[kOptLeavesPerLaunch];
  long n[kOptLeavesPerLaunch];
  int cstart[kOptLeavesPerLaunch + 1];  // first chunk of each leaf (chunk ids are global)
  int count;
};

// Scalars written by the finish pass: [0] clip factor, [1] 1 / (1 - b1^t'),
// [2] 1 / (1 - b2^t'), [3] lr.
struct OptScalars {
  float factor, bcm, bcv, lr;
};

template <typename T>
__device__ __forceinline__ float ld(const T* p, long i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, long i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, long i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void st(T* p, long i, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, long i, float v) {
  p[i] = v;
}
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, long i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// Leaf of a global chunk id within this launch's table.
__device__ __forceinline__ int leaf_of(const OptLeaves& t, int c) {
  int l = 0;
  while (l + 1 < t.count && t.cstart[l + 1] <= c) ++l;
  return l;
}

// Pass 1: part[c] = sum over chunk c of g*g (f32 accumulation; fixed order:
// thread-strided then a fixed tree over the block).
template <typename T>
__global__ void __launch_bounds__(kThreads) sumsq_kernel(OptLeaves t, float* __restrict__ part) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kThreads];
  const int c0 = t.cstart[0], c1 = t.cstart[t.count];
  for (int c = c0 + static_cast<int>(blockIdx.x); c < c1; c += gridDim.x) {
    const int l = leaf_of(t, c);
    const T* g = static_cast<const T*>(t.g[l]);
    const long b = static_cast<long>(c - t.cstart[l]) * kChunk;
    const long e = min(b + kChunk, t.n[l]);
    float s = 0.f;
    for (long i = b + threadIdx.x; i < e; i += kThreads) {
      const float x = ld<T>(g, i);
      s = fmaf(x, x, s);
    }
    red[threadIdx.x] = s;
    __syncthreads();
    for (int w = kThreads / 2; w > 0; w >>= 1) {
      if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) part[c] = red[0];
    __syncthreads();
  }
}

// Finish: norm = sqrt(sum part), factor = min(1, max_norm / (norm + 1e-8))
// (1 without clipping), t' = t + 1 and the bias corrections
// (lib/optim.shf:20-25, 48-51). One thread: the partials are summed in order.
__global__ void opt_finish_kernel(const float* __restrict__ part, int nchunks, const float* __restrict__ t_in,
                                  float* __restrict__ t_out, const float* __restrict__ lr, float b1, float b2,
                                  float max_norm, OptScalars* __restrict__ sc, float* __restrict__ norm_out) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double acc = 0.0;
  for (int c = 0; c < nchunks; ++c) acc += static_cast<double>(part[c]);
  const float norm = sqrtf(static_cast<float>(acc));
  if (norm_out) *norm_out = norm;
  if (!sc) return;  // norm only
  const float factor = max_norm > 0.f ? fminf(1.0f, max_norm / (norm + 1e-8f)) : 1.0f;
  const float tn = *t_in + 1.0f;
  sc->factor = factor;
  sc->bcm = 1.0f / (1.0f - powf(b1, tn));
  sc->bcv = 1.0f / (1.0f - powf(b2, tn));
  sc->lr = *lr;
  if (t_out) *t_out = tn;
}

// Pass 2 (lib/optim.shf:19-32 after :48-51): g' = g * factor (factor cast
// like g); m' = b1 m + (1-b1) g'; v' = b2 v + (1-b2) g'^2;
// p' = p - lr (wd p + m' bcm / (sqrt(v' bcv) + eps)). Computed in f32, stored
// in the leaf's element type; outputs may alias inputs.
template <typename T>
__global__ void __launch_bounds__(kThreads) adamw_kernel(OptLeaves t, const OptScalars* __restrict__ sc, float b1,
                                                         float b2, float eps, float wd) {
  pdl_wait();
  pdl_trigger();
  T fac_t;
  st<T>(&fac_t, 0, sc->factor);
  const float fl = ld<T>(&fac_t, 0);  // the clip factor in the leaf's type
  const float bcm = sc->bcm, bcv = sc->bcv, lr = sc->lr;
  const int c0 = t.cstart[0], c1 = t.cstart[t.count];
  for (int c = c0 + static_cast<int>(blockIdx.x); c < c1; c += gridDim.x) {
    const int l = leaf_of(t, c);
    const T* g = static_cast<const T*>(t.g[l]);
    const T* p = static_cast<const T*>(t.p[l]);
    const T* m = static_cast<const T*>(t.m[l]);
    const T* v = static_cast<const T*>(t.v[l]);
    T* po = static_cast<T*>(t.p_out[l]);
    T* mo = static_cast<T*>(t.m_out[l]);
    T* vo = static_cast<T*>(t.v_out[l]);
    const long b = static_cast<long>(c - t.cstart[l]) * kChunk;
    const long e = min(b + kChunk, t.n[l]);
    for (long i = b + threadIdx.x; i < e; i += kThreads) {
      T gt;
      st<T>(&gt, 0, ld<T>(g, i) * fl);
      const float gc = ld<T>(&gt, 0);
      const float mn = b1 * ld<T>(m, i) + (1.0f - b1) * gc;
      const float vn = b2 * ld<T>(v, i) + (1.0f - b2) * (gc * gc);
      const float pv = ld<T>(p, i);
      const float pn = pv - lr * (wd * pv + (mn * bcm) / (sqrtf(vn * bcv) + eps));
      st<T>(mo, i, mn);
      st<T>(vo, i, vn);
      st<T>(po, i, pn);
    }
  }
}

int chunks_of(long n) { return static_cast<int>((n + kChunk - 1) / kChunk); }

}  // namespace

size_t optimizer_workspace_bytes(const int64_t* counts, int n_leaves) {
  long chunks = 0;
  for (int i = 0; i < n_leaves; ++i) chunks += chunks_of(counts[i]);
  return static_cast<size_t>(chunks) * sizeof(float) + 256;
}

int optimizer_step(bool bf16, int n_leaves, const int64_t* counts, const void* const* grads,
                   const void* const* params, const void* const* m, const void* const* v, void* const* params_out,
                   void* const* m_out, void* const* v_out, const float* t_in, float* t_out, const float* lr,
                   float b1, float b2, float eps, float wd, float max_norm, float* norm_out, void* workspace,
                   size_t workspace_bytes, cudaStream_t s) {
  if (n_leaves <= 0 || !counts || !grads) return 1;
  const bool update = params != nullptr;
  if (update && (!m || !v || !params_out || !m_out || !v_out || !t_in || !lr)) return 1;
  if (!update && !norm_out) return 1;
  long total_chunks = 0;
  for (int i = 0; i < n_leaves; ++i) {
    if (counts[i] <= 0 || !grads[i]) return 1;
    if (update && (!params[i] || !m[i] || !v[i] || !params_out[i] || !m_out[i] || !v_out[i])) return 1;
    total_chunks += chunks_of(counts[i]);
  }
  if (total_chunks >= (1L << 30)) return 1;
  const size_t need = static_cast<size_t>(total_chunks) * sizeof(float) + 256;
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15)) return 5;
  float* part = static_cast<float*>(workspace);
  OptScalars* sc = reinterpret_cast<OptScalars*>(
      (reinterpret_cast<uintptr_t>(part + total_chunks) + 15) & ~static_cast<uintptr_t>(15));
  const int grid_cap = 4 * num_sms_cached();

  // tables of at most kOptLeavesPerLaunch leaves; chunk ids continue across tables
  auto table = [&](int first, int cnt, int cbase) {
    OptLeaves t{};
    t.count = cnt;
    int c = cbase;
    for (int j = 0; j < cnt; ++j) {
      const int i = first + j;
      t.g[j] = grads[i];
      if (update) {
        t.p[j] = params[i];
        t.m[j] = m[i];
        t.v[j] = v[i];
        t.p_out[j] = params_out[i];
        t.m_out[j] = m_out[i];
        t.v_out[j] = v_out[i];
      }
      t.n[j] = counts[i];
      t.cstart[j] = c;
      c += chunks_of(counts[i]);
    }
    t.cstart[cnt] = c;
    return t;
  };
  int cbase = 0;
  for (int first = 0; first < n_leaves; first += kOptLeavesPerLaunch) {
    const int cnt = std::min(kOptLeavesPerLaunch, n_leaves - first);
    OptLeaves t = table(first, cnt, cbase);
    const int nch = t.cstart[cnt] - cbase;
    const int grid = std::min(nch, grid_cap);
    if (bf16)
      launch_pdl((sumsq_kernel<__nv_bfloat16>), dim3(grid), dim3(kThreads), 0, s, t, part);
    else
      launch_pdl((sumsq_kernel<float>), dim3(grid), dim3(kThreads), 0, s, t, part);
    cbase = t.cstart[cnt];
  }
  launch_pdl(opt_finish_kernel, dim3(1), dim3(32), 0, s, part, static_cast<int>(total_chunks), t_in,
             update ? t_out : nullptr, lr, b1, b2, max_norm, update ? sc : nullptr, norm_out);
  if (update) {
    cbase = 0;
    for (int first = 0; first < n_leaves; first += kOptLeavesPerLaunch) {
      const int cnt = std::min(kOptLeavesPerLaunch, n_leaves - first);
      OptLeaves t = table(first, cnt, cbase);
      const int nch = t.cstart[cnt] - cbase;
      const int grid = std::min(nch, grid_cap);
      if (bf16)
        launch_pdl((adamw_kernel<__nv_bfloat16>), dim3(grid), dim3(kThreads), 0, s, t, sc, b1, b2, eps, wd);
      else
        launch_pdl((adamw_kernel<float>), dim3(grid), dim3(kThreads), 0, s, t, sc, b1, b2, eps, wd);
      cbase = t.cstart[cnt];
    }
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace sb
