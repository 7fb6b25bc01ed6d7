// Device side of nanoGPT's data path: the key chain and get-batch of
// examples/nanogpt/train.shf:15-21,70-73, so a training loop draws its
// batches from a token array resident in HBM with no host work per step.
//   [k1 k2] = random-split key                       (random_ops.rs:146-162)
//   starts  = random-randint k1 [batch] 0 (len - block - 1)   (prng.rs:124-134)
//   x = data[starts + arange(block)], y = data[starts + arange(block) + 1]
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "sb_nn.h"
#include "sb_prng.cuh"

namespace sb {

namespace {

// One CTA per batch row: the row's start from the key's sampling bits for
// flat index b (f32 arithmetic as the reference's randint), then a
// coalesced copy of the window and of the window shifted by one.
__global__ void get_batch_kernel(const float* __restrict__ data, const float* __restrict__ key, int block, float high,
                                 float* __restrict__ x, float* __restrict__ y) {
  const int b = blockIdx.x;
  uint32_t w0, w1, bits, unused;
  key_decode(key, w0, w1);
  threefry2x32(w0, w1, static_cast<uint32_t>(b), 0u, bits, unused);
  const float u = uniform_from_bits(bits);
  float v = floorf(__fmul_rn(u, high)) + 0.0f;  // low = 0
  v = fminf(v, high - 1.0f);
  v = fmaxf(v, 0.0f);
  const long start = static_cast<long>(v);
  const long row = static_cast<long>(b) * block;
  for (int t = threadIdx.x; t < block; t += blockDim.x) {
    x[row + t] = data[start + t];
    y[row + t] = data[start + t + 1];
  }
}

// child i of random-split: threefry(key, [i, 1]) as four limbs
__global__ void random_split_kernel(const float* __restrict__ key, int n, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t w0, w1, c0, c1;
  key_decode(key, w0, w1);
  threefry2x32(w0, w1, static_cast<uint32_t>(i), 1u, c0, c1);
  key_encode(c0, c1, out + 4 * i);
}

}  // namespace

int get_batch(const float* data, long n, const float* key, int block, int batch, float* x, float* y, cudaStream_t s) {
  const long hi = n - block - 1;  // exclusive upper bound of the start
  if (!data || !key || !x || !y || block <= 0 || batch <= 0 || hi <= 0 || hi > (1L << 24)) return 1;
  get_batch_kernel<<<batch, 256, 0, s>>>(data, key, block, static_cast<float>(hi), x, y);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

int random_split(const float* key, int n, float* out, cudaStream_t s) {
  if (!key || !out || n <= 0) return 1;
  random_split_kernel<<<(n + 127) / 128, 128, 0, s>>>(key, n, out);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace sb
