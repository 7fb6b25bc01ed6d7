// Generic device kernels behind the StableHLO executor (stablehlo.cpp): one
// kernel family per StableHLO op of the surface Sheaf's emitter prints
// (sheaf/src/lowering/stablehlo/*.rs). Each op computes in fp32 registers and
// rounds to its declared element type on store, so bf16 modules round after
// every op as the reference's per-op bf16 execution does.
//
// Element types: f32, bf16, f16, i32 (also used for the PRNG's u32 words),
// i1 (one byte per element). Shapes have rank <= kMaxRank; index maps are
// passed by value.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "hlo_kernels.h"
#include "sb_kernels.h"

namespace sb {
namespace hlo {

namespace {

__device__ __forceinline__ float ld(const void* p, long i, int dt) {
  switch (dt) {
    case DT_F32: return static_cast<const float*>(p)[i];
    case DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case DT_F16: return __half2float(static_cast<const __half*>(p)[i]);
    case DT_I32: return static_cast<float>(static_cast<const int32_t*>(p)[i]);
    default: return static_cast<const uint8_t*>(p)[i] ? 1.f : 0.f;
  }
}

__device__ __forceinline__ void st(void* p, long i, int dt, float v) {
  switch (dt) {
    case DT_F32: static_cast<float*>(p)[i] = v; break;
    case DT_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case DT_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case DT_I32: static_cast<int32_t*>(p)[i] = static_cast<int32_t>(v); break;  // truncation (fptosi)
    default: static_cast<uint8_t*>(p)[i] = (v != 0.f) ? 1 : 0; break;
  }
}

__device__ __forceinline__ uint32_t ldu(const void* p, long i) { return static_cast<const uint32_t*>(p)[i]; }

#define SB_GRID_LOOP(i, n) \
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < (n); i += static_cast<long>(gridDim.x) * blockDim.x)

__device__ float apply_unary(int op, float x) {
  switch (op) {
    case U_NEG: return -x;
    case U_ABS: return fabsf(x);
    case U_EXP: return expf(x);
    case U_LOG: return logf(x);
    case U_SQRT: return sqrtf(x);
    case U_RSQRT: return rsqrtf(x);
    case U_TANH: return tanhf(x);
    case U_SIN: return sinf(x);
    case U_COS: return cosf(x);
    case U_FLOOR: return floorf(x);
    case U_CEIL: return ceilf(x);
    case U_SIGN: return (x > 0.f) ? 1.f : ((x < 0.f) ? -1.f : x);
    case U_LOGISTIC: return 1.f / (1.f + expf(-x));
    case U_NOT: return x != 0.f ? 0.f : 1.f;
    case U_LOG1P: return log1pf(x);
    case U_EXPM1: return expm1f(x);
    default: return x;  // U_COPY
  }
}

__device__ float apply_binary(int op, float a, float b) {
  switch (op) {
    case B_ADD: return a + b;
    case B_SUB: return a - b;
    case B_MUL: return a * b;
    case B_DIV: return a / b;
    case B_POW: return powf(a, b);
    case B_MAX: return fmaxf(a, b);
    case B_MIN: return fminf(a, b);
    case B_REM: return fmodf(a, b);
    case B_FLOORDIV: return floorf(a / b);
    case B_ATAN2: return atan2f(a, b);
    case B_AND: return (a != 0.f && b != 0.f) ? 1.f : 0.f;
    case B_OR: return (a != 0.f || b != 0.f) ? 1.f : 0.f;
    default: return a;
  }
}

__device__ uint32_t apply_binary_u32(int op, uint32_t a, uint32_t b) {
  switch (op) {
    case B_ADD: return a + b;
    case B_SUB: return a - b;
    case B_MUL: return a * b;
    case B_AND: return a & b;
    case B_OR: return a | b;
    case B_XOR: return a ^ b;
    case B_SHL: return b >= 32 ? 0u : (a << b);
    case B_SHR: return b >= 32 ? 0u : (a >> b);
    case B_MAX: return static_cast<uint32_t>(max(static_cast<int32_t>(a), static_cast<int32_t>(b)));
    case B_MIN: return static_cast<uint32_t>(min(static_cast<int32_t>(a), static_cast<int32_t>(b)));
    default: return a;
  }
}

__global__ void unary_kernel(const void* a, void* out, long n, int op, int dta, int dto) {
  SB_GRID_LOOP(i, n) st(out, i, dto, apply_unary(op, ld(a, i, dta)));
}

__global__ void binary_kernel(const void* a, const void* b, void* out, long n, int op, int dt) {
  if (dt == DT_I32) {
    SB_GRID_LOOP(i, n) static_cast<uint32_t*>(out)[i] = apply_binary_u32(op, ldu(a, i), ldu(b, i));
  } else if (dt == DT_I1) {
    SB_GRID_LOOP(i, n) {
      const uint8_t x = static_cast<const uint8_t*>(a)[i] != 0, y = static_cast<const uint8_t*>(b)[i] != 0;
      uint8_t r = 0;
      if (op == B_AND) r = x & y;
      else if (op == B_OR) r = x | y;
      else if (op == B_XOR) r = x ^ y;
      static_cast<uint8_t*>(out)[i] = r;
    }
  } else {
    SB_GRID_LOOP(i, n) st(out, i, dt, apply_binary(op, ld(a, i, dt), ld(b, i, dt)));
  }
}

__global__ void clamp_kernel(const void* lo, long nlo, const void* x, const void* hi, long nhi, void* out, long n,
                             int dt) {
  SB_GRID_LOOP(i, n) {
    const float l = ld(lo, nlo == 1 ? 0 : i, dt), h = ld(hi, nhi == 1 ? 0 : i, dt);
    st(out, i, dt, fminf(fmaxf(ld(x, i, dt), l), h));
  }
}

__global__ void compare_kernel(const void* a, const void* b, uint8_t* out, long n, int dir, int dt) {
  SB_GRID_LOOP(i, n) {
    bool r;
    if (dt == DT_I32) {
      const int32_t x = static_cast<const int32_t*>(a)[i], y = static_cast<const int32_t*>(b)[i];
      r = dir == C_EQ ? x == y : dir == C_NE ? x != y : dir == C_LT ? x < y : dir == C_LE ? x <= y : dir == C_GT ? x > y : x >= y;
    } else {
      const float x = ld(a, i, dt), y = ld(b, i, dt);
      r = dir == C_EQ ? x == y : dir == C_NE ? x != y : dir == C_LT ? x < y : dir == C_LE ? x <= y : dir == C_GT ? x > y : x >= y;
    }
    out[i] = r ? 1 : 0;
  }
}

__global__ void select_kernel(const uint8_t* p, long np, const void* a, const void* b, void* out, long n, int dt,
                              int esize) {
  SB_GRID_LOOP(i, n) {
    const bool c = p[np == 1 ? 0 : i] != 0;
    const char* src = static_cast<const char*>(c ? a : b) + i * esize;
    char* dst = static_cast<char*>(out) + i * esize;
    for (int k = 0; k < esize; ++k) dst[k] = src[k];
  }
}

__global__ void convert_kernel_g(const void* a, int dta, void* out, int dto, long n) {
  if (dta == DT_I32 && dto == DT_I32) {
    SB_GRID_LOOP(i, n) static_cast<int32_t*>(out)[i] = static_cast<const int32_t*>(a)[i];
  } else if (dta == DT_I32) {
    // integer -> float: exact for |v| < 2^24, as the PRNG's 16-bit limbs are
    SB_GRID_LOOP(i, n) st(out, i, dto, static_cast<float>(static_cast<const int32_t*>(a)[i]));
  } else if (dto == DT_I32) {
    SB_GRID_LOOP(i, n) {
      const float v = ld(a, i, dta);
      static_cast<int32_t*>(out)[i] = (v != v) ? 0 : static_cast<int32_t>(fmaxf(fminf(v, 2147483520.f), -2147483648.f));
    }
  } else {
    SB_GRID_LOOP(i, n) st(out, i, dto, ld(a, i, dta));
  }
}

// Generic index remap: out[i] = in[src(i)], src = base + sum_d (c_d - offset_d)
// * stride_d over the output coordinates c. With `check`, coordinates outside
// [0, extent_d) are not copied: they take the pad value if one is given and
// are left untouched otherwise (concatenate writes one operand at a time).
__global__ void remap_kernel(const void* in, void* out, long n, int esize, IndexMap m) {
  SB_GRID_LOOP(i, n) {
    long rem = i, src = m.base;
    bool ok = true;
    for (int d = m.rank - 1; d >= 0; --d) {
      const long c = rem % m.out_shape[d];
      rem /= m.out_shape[d];
      const long ci = c - m.offset[d];
      if (m.check && (ci < 0 || ci >= m.extent[d])) ok = false;
      src += ci * m.stride[d];
    }
    char* dst = static_cast<char*>(out) + i * esize;
    if (ok) {
      const char* sp = static_cast<const char*>(in) + src * esize;
      for (int k = 0; k < esize; ++k) dst[k] = sp[k];
    } else if (m.pad_value) {
      const char* sp = static_cast<const char*>(m.pad_value);
      for (int k = 0; k < esize; ++k) dst[k] = sp[k];
    }
  }
}

__global__ void iota_kernel(void* out, long n, int dt, long inner, long dim_extent) {
  SB_GRID_LOOP(i, n) {
    const long c = (i / inner) % dim_extent;
    if (dt == DT_I32)
      static_cast<int32_t*>(out)[i] = static_cast<int32_t>(c);
    else
      st(out, i, dt, static_cast<float>(c));
  }
}

// Reduction of the middle axis of [outer, red, inner] (a run of contiguous
// reduced axes). fp32 accumulation in index order, initialised with `init`.
__global__ void reduce_kernel(const void* in, void* out, long outer, long red, long inner, int op, float init,
                              const void* init_ptr, int dt) {
  SB_GRID_LOOP(i, outer * inner) {
    const long o = i / inner, k = i % inner;
    float acc = init_ptr ? ld(init_ptr, 0, dt) : init;
    if (dt == DT_I32) {
      uint32_t a = init_ptr ? ldu(init_ptr, 0) : static_cast<uint32_t>(static_cast<int32_t>(init));
      for (long r = 0; r < red; ++r) a = apply_binary_u32(op, a, ldu(in, (o * red + r) * inner + k));
      static_cast<uint32_t*>(out)[i] = a;
      continue;
    }
    for (long r = 0; r < red; ++r) acc = apply_binary(op, acc, ld(in, (o * red + r) * inner + k, dt));
    st(out, i, dt, acc);
  }
}

// Batched GEMM on canonical layouts: C[b, m, n] = sum_k A[b, m, k] * B[b, k, n],
// fp32 accumulation, 16x16 output tile per block with a 16-deep smem panel.
__global__ void bgemm_kernel(const void* A, const void* B, void* C, int M, int N, int K, long sa, long sb, long sc,
                             int dta, int dtb, int dtc) {
  __shared__ float As[16][17], Bs[16][17];
  const int b = blockIdx.z;
  const int row = blockIdx.y * 16 + threadIdx.y, col = blockIdx.x * 16 + threadIdx.x;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
    As[threadIdx.y][threadIdx.x] = (row < M && ka < K) ? ld(A, b * sa + static_cast<long>(row) * K + ka, dta) : 0.f;
    Bs[threadIdx.y][threadIdx.x] = (kb < K && col < N) ? ld(B, b * sb + static_cast<long>(kb) * N + col, dtb) : 0.f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) acc = fmaf(As[threadIdx.y][kk], Bs[kk][threadIdx.x], acc);
    __syncthreads();
  }
  if (row < M && col < N) st(C, b * sc + static_cast<long>(row) * N + col, dtc, acc);
}

// Row gather (the form Sheaf emits: collapsed_slice_dims = [0],
// start_index_map = [0]): out[r, :] = operand[clamp(idx[r]), :].
__global__ void gather_rows_kernel(const void* operand, const int32_t* idx, void* out, long rows, long V, long width,
                                   int esize) {
  SB_GRID_LOOP(i, rows * width) {
    const long r = i / width, c = i % width;
    long v = idx[r];
    v = v < 0 ? 0 : (v >= V ? V - 1 : v);
    const char* s = static_cast<const char*>(operand) + (v * width + c) * esize;
    char* d = static_cast<char*>(out) + i * esize;
    for (int k = 0; k < esize; ++k) d[k] = s[k];
  }
}

// Clamped start of axis k (StableHLO dynamic_slice / dynamic_update_slice).
__device__ __forceinline__ long dyn_start(const DynSlice& d, int k) {
  long v = *d.start[k];
  const long hi = d.shape[k] - d.size[k];
  return v < 0 ? 0 : (v > hi ? hi : v);
}

// out[c] = in[start + c] over the slice coordinates c.
__global__ void dyn_slice_kernel(const void* in, void* out, long n, int esize, DynSlice d) {
  SB_GRID_LOOP(i, n) {
    long rem = i, src = 0, stride = 1;
    for (int k = d.rank - 1; k >= 0; --k) {
      const long c = rem % d.size[k];
      rem /= d.size[k];
      src += (dyn_start(d, k) + c) * stride;
      stride *= d.shape[k];
    }
    const char* sp = static_cast<const char*>(in) + src * esize;
    char* dp = static_cast<char*>(out) + i * esize;
    for (int b = 0; b < esize; ++b) dp[b] = sp[b];
  }
}

// out[start + c] = upd[c] over the update's coordinates c.
__global__ void dyn_update_kernel(void* out, const void* upd, long n, int esize, DynSlice d) {
  SB_GRID_LOOP(i, n) {
    long rem = i, dst = 0, stride = 1;
    for (int k = d.rank - 1; k >= 0; --k) {
      const long c = rem % d.size[k];
      rem /= d.size[k];
      dst += (dyn_start(d, k) + c) * stride;
      stride *= d.shape[k];
    }
    const char* sp = static_cast<const char*>(upd) + i * esize;
    char* dp = static_cast<char*>(out) + dst * esize;
    for (int b = 0; b < esize; ++b) dp[b] = sp[b];
  }
}

// One CTA per row: bitonic sort of (key, position) pairs in shared memory,
// position breaking ties so the order is stable; padding sorts last.
__global__ void __launch_bounds__(512) sort_rows_kernel(const void* keys, int key_dt, const int32_t* payload,
                                                        void* out_keys, int32_t* out_payload, int n, int np2,
                                                        int descending) {
  extern __shared__ float sk[];
  int* pos = reinterpret_cast<int*>(sk + np2);
  const long row = blockIdx.x;
  for (int i = threadIdx.x; i < np2; i += blockDim.x) {
    if (i < n) {
      const float v = ld(keys, row * n + i, key_dt);
      sk[i] = descending ? v : -v;  // sort descending on the (possibly negated) key
      pos[i] = i;
    } else {
      sk[i] = -INFINITY;
      pos[i] = 0x7FFFFFFF;
    }
  }
  __syncthreads();
  for (int size = 2; size <= np2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const float vi = sk[i], vj = sk[j];
          const int pi = pos[i], pj = pos[j];
          // does element j belong before element i?
          const bool j_first = vj > vi || (vj == vi && pj < pi);
          const bool i_first = vi > vj || (vi == vj && pi < pj);
          const bool swap = ((i & size) == 0) ? j_first : i_first;
          if (swap) {
            sk[i] = vj;
            sk[j] = vi;
            pos[i] = pj;
            pos[j] = pi;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int p = pos[i];
    // the key is copied from its source (exact, also for bf16 and -0.0)
    const long src = row * n + p, dst = row * n + i;
    if (key_dt == DT_BF16)
      static_cast<__nv_bfloat16*>(out_keys)[dst] = static_cast<const __nv_bfloat16*>(keys)[src];
    else
      static_cast<float*>(out_keys)[dst] = static_cast<const float*>(keys)[src];
    out_payload[dst] = payload ? payload[src] : p;  // no payload: the source positions
  }
}

int blocks_for(long n) { return static_cast<int>(std::max<long>(1, std::min<long>((n + 255) / 256, 32L * num_sms()))); }

}  // namespace

int dt_size(int dt) { return dt == DT_F32 || dt == DT_I32 ? 4 : (dt == DT_I1 ? 1 : 2); }

int unary(const void* a, void* out, long n, int op, int dta, int dto, cudaStream_t s) {
  if (n == 0) return 0;
  unary_kernel<<<blocks_for(n), 256, 0, s>>>(a, out, n, op, dta, dto);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int binary(const void* a, const void* b, void* out, long n, int op, int dt, cudaStream_t s) {
  if (n == 0) return 0;
  binary_kernel<<<blocks_for(n), 256, 0, s>>>(a, b, out, n, op, dt);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int clamp(const void* lo, long nlo, const void* x, const void* hi, long nhi, void* out, long n, int dt,
          cudaStream_t s) {
  if (n == 0) return 0;
  clamp_kernel<<<blocks_for(n), 256, 0, s>>>(lo, nlo, x, hi, nhi, out, n, dt);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int compare(const void* a, const void* b, void* out, long n, int dir, int dt, cudaStream_t s) {
  if (n == 0) return 0;
  compare_kernel<<<blocks_for(n), 256, 0, s>>>(a, b, static_cast<uint8_t*>(out), n, dir, dt);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int select(const void* p, long np, const void* a, const void* b, void* out, long n, int dt, cudaStream_t s) {
  if (n == 0) return 0;
  select_kernel<<<blocks_for(n), 256, 0, s>>>(static_cast<const uint8_t*>(p), np, a, b, out, n, dt, dt_size(dt));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int convert(const void* a, int dta, void* out, int dto, long n, cudaStream_t s) {
  if (n == 0) return 0;
  convert_kernel_g<<<blocks_for(n), 256, 0, s>>>(a, dta, out, dto, n);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int remap(const void* in, void* out, long n, int dt, const IndexMap& m, cudaStream_t s) {
  if (n == 0) return 0;
  remap_kernel<<<blocks_for(n), 256, 0, s>>>(in, out, n, dt_size(dt), m);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int iota(void* out, long n, int dt, long inner, long dim_extent, cudaStream_t s) {
  if (n == 0) return 0;
  iota_kernel<<<blocks_for(n), 256, 0, s>>>(out, n, dt, inner, dim_extent);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int reduce(const void* in, void* out, long outer, long red, long inner, int op, float init, const void* init_ptr,
           int dt, cudaStream_t s) {
  if (outer * inner == 0) return 0;
  reduce_kernel<<<blocks_for(outer * inner), 256, 0, s>>>(in, out, outer, red, inner, op, init, init_ptr, dt);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int bgemm(const void* A, const void* B, void* C, int batch, int M, int N, int K, int dta, int dtb, int dtc,
          cudaStream_t s) {
  if (batch == 0 || M == 0 || N == 0) return 0;
  dim3 grid((N + 15) / 16, (M + 15) / 16, batch);
  bgemm_kernel<<<grid, dim3(16, 16), 0, s>>>(A, B, C, M, N, K, static_cast<long>(M) * K, static_cast<long>(K) * N,
                                              static_cast<long>(M) * N, dta, dtb, dtc);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int gather_rows(const void* operand, const void* idx, void* out, long rows, long V, long width, int dt, cudaStream_t s) {
  if (rows * width == 0) return 0;
  gather_rows_kernel<<<blocks_for(rows * width), 256, 0, s>>>(operand, static_cast<const int32_t*>(idx), out, rows, V,
                                                             width, dt_size(dt));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int dynamic_slice(const void* in, void* out, int dt, const DynSlice& d, cudaStream_t s) {
  long n = 1;
  for (int k = 0; k < d.rank; ++k) n *= d.size[k];
  if (n == 0) return 0;
  dyn_slice_kernel<<<blocks_for(n), 256, 0, s>>>(in, out, n, dt_size(dt), d);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int dynamic_update(void* out, const void* upd, int dt, const DynSlice& d, cudaStream_t s) {
  long n = 1;
  for (int k = 0; k < d.rank; ++k) n *= d.size[k];
  if (n == 0) return 0;
  dyn_update_kernel<<<blocks_for(n), 256, 0, s>>>(out, upd, n, dt_size(dt), d);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

// ---------------------------------------------------------------------------
// Rows longer than one CTA's shared memory holds: a stable sort on 64-bit
// composite keys, (order-preserving image of the key) << 32 | position, so
// that ascending unsigned order is (key in the requested direction, then
// position) and every composite is distinct. -0.0 is folded into +0.0 (the
// two compare equal, so they keep their positions' order). Chunks of
// kSortChunk composites are sorted in shared memory, then runs are merged
// pairwise in global memory (merge path: each thread finds its split of the
// two runs by binary search, then merges kSortIpt outputs); a last pass
// copies the keys and payload of each position into place.
// ---------------------------------------------------------------------------

constexpr int kSortChunk = 8192;
constexpr int kSortIpt = 8;

__device__ __forceinline__ uint64_t sort_composite(float v, int pos, int descending) {
  if (v == 0.f) v = 0.f;  // -0.0 -> +0.0
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending float order as unsigned order
  if (descending) u = ~u;
  return (static_cast<uint64_t>(u) << 32) | static_cast<uint32_t>(pos);
}

__global__ void __launch_bounds__(1024) sort_chunk_kernel(const void* keys, int key_dt, int n, int npad,
                                                          int descending, uint64_t* out) {
  extern __shared__ uint64_t sk[];  // kSortChunk composites (64 KB, dynamic)
  const long row = blockIdx.y;
  const int base = blockIdx.x * kSortChunk;
  for (int i = threadIdx.x; i < kSortChunk; i += blockDim.x) {
    const int pos = base + i;
    sk[i] = pos < n ? sort_composite(ld(keys, row * n + pos, key_dt), pos, descending) : ~0ull;
  }
  __syncthreads();
  for (int size = 2; size <= kSortChunk; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < kSortChunk; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const uint64_t a = sk[i], b = sk[j];
          const bool up = (i & size) == 0;
          if (up ? (b < a) : (a < b)) {
            sk[i] = b;
            sk[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  uint64_t* o = out + row * npad + base;
  for (int i = threadIdx.x; i < kSortChunk; i += blockDim.x) o[i] = sk[i];
}

// Merges the run pairs of length `run` of every row (npad composites a row).
__global__ void __launch_bounds__(256) sort_merge_kernel(const uint64_t* in, uint64_t* out, int npad, int run) {
  const long row = blockIdx.y;
  const long k0 = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) * kSortIpt;
  if (k0 >= npad) return;
  const long base = k0 / (2L * run) * (2L * run);
  const uint64_t* A = in + row * npad + base;
  const long lenA = min(static_cast<long>(run), npad - base);
  const uint64_t* Bp = A + lenA;
  const long lenB = max(0L, min(static_cast<long>(run), npad - base - lenA));
  const long k = k0 - base;
  long lo = max(0L, k - lenB), hi = min(k, lenA);
  while (lo < hi) {  // i = number of A elements among the first k outputs
    const long mid = (lo + hi) >> 1;
    if (A[mid] <= Bp[k - 1 - mid])
      lo = mid + 1;
    else
      hi = mid;
  }
  long i = lo, j = k - lo;
  uint64_t* o = out + row * npad + base + k;
  const long cnt = min(static_cast<long>(kSortIpt), lenA + lenB - k);
  for (long t = 0; t < cnt; ++t) {
    const bool takeA = j >= lenB || (i < lenA && A[i] <= Bp[j]);
    o[t] = takeA ? A[i++] : Bp[j++];
  }
}

__global__ void sort_gather_kernel(const uint64_t* sorted, int npad, const void* keys, int key_dt,
                                   const int32_t* payload, void* out_keys, int32_t* out_payload, long rows, int n) {
  const long total = rows * n;
  const int es = key_dt == DT_F32 ? 4 : 2;
  for (long e = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long>(gridDim.x) * blockDim.x) {
    const long row = e / n, i = e % n;
    const long src = row * n + static_cast<uint32_t>(sorted[row * npad + i]);
    out_payload[e] = payload ? payload[src] : static_cast<int32_t>(src - row * n);
    const char* kp = static_cast<const char*>(keys) + src * es;
    char* op = static_cast<char*>(out_keys) + e * es;
    for (int b = 0; b < es; ++b) op[b] = kp[b];
  }
}

size_t sort_rows_workspace_bytes(long rows, int n) {
  if (n <= kSortSmemRow) return 0;
  const long npad = (static_cast<long>(n) + kSortChunk - 1) / kSortChunk * kSortChunk;
  return static_cast<size_t>(2 * rows * npad) * sizeof(uint64_t);
}

int sort_rows(const void* keys, int key_dt, const int32_t* payload, void* out_keys, int32_t* out_payload, long rows,
              int n, bool descending, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (rows == 0 || n == 0) return 0;
  if (n > kSortMaxRow || (key_dt != DT_F32 && key_dt != DT_BF16)) return 1;
  if (n > kSortSmemRow) {
    if (!ws || ws_bytes < sort_rows_workspace_bytes(rows, n) || rows > 65535) return 1;
    const int npad = (n + kSortChunk - 1) / kSortChunk * kSortChunk;
    uint64_t* a = static_cast<uint64_t*>(ws);
    uint64_t* b = a + rows * npad;
    const size_t csm = kSortChunk * sizeof(uint64_t);
    if (cudaFuncSetAttribute(sort_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(csm)) !=
        cudaSuccess)
      return 3;
    sort_chunk_kernel<<<dim3(npad / kSortChunk, static_cast<unsigned>(rows)), 1024, csm, s>>>(
        keys, key_dt, n, npad, descending ? 1 : 0, a);
    for (int run = kSortChunk; run < npad; run *= 2) {
      const long threads = (npad + kSortIpt - 1) / kSortIpt;
      sort_merge_kernel<<<dim3(static_cast<unsigned>((threads + 255) / 256), static_cast<unsigned>(rows)), 256, 0,
                          s>>>(a, b, npad, run);
      std::swap(a, b);
    }
    sort_gather_kernel<<<blocks_for(rows * n), 256, 0, s>>>(a, npad, keys, key_dt, payload, out_keys, out_payload,
                                                           rows, n);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
  }
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  const size_t smem = static_cast<size_t>(np2) * 8;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(sort_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess)
    return 3;
  sort_rows_kernel<<<static_cast<unsigned>(rows), 512, smem, s>>>(keys, key_dt, payload, out_keys, out_payload, n,
                                                                   np2, descending ? 1 : 0);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace hlo
}  // namespace sb
