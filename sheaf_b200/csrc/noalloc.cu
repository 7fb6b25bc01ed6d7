// Layer-norm VJP entry point that allocates nothing (sb_op_layernorm_bwd_noalloc).
//
// Some callers cannot allocate device memory while they run: a host runtime
// that owns the whole device heap through its own allocator and hands a
// kernel library only finished buffers and a stream (for example the Rust
// shim in front of this library, or a serving process that carves all of
// HBM into a fixed arena at start-up), and latency-critical loops in which
// cudaMalloc's implicit device-wide synchronisation is not acceptable.
// sb_op_layernorm_bwd needs a caller-provided workspace for its partial sums
// of dgamma; this variant keeps that scratch in a fixed array compiled into
// the library instead, so the caller passes only inputs and outputs.
//
// The array lives in device memory for as long as the library is loaded, on
// every GPU that uses it: kScratchFloats floats (128 KB). Every call shares
// it, so calls that overlap on the GPU (on different streams, or from
// different host threads) race on it and must be serialised by the caller.
#include <cuda_runtime.h>

#include <map>
#include <mutex>

#include "../../include/sheaf_b200_ops.h"
#include "sb_nn.h"

namespace sb {
namespace {

// dgamma partial sums: one row of D floats per block of the VJP kernel.
constexpr int kScratchFloats = 32768;
// Largest row width accepted: the scratch must hold the partials of at
// least 8 blocks.
constexpr int kMaxWidth = kScratchFloats / 8;

static __device__ __align__(256) float g_ln_bwd_scratch[kScratchFloats];

// Device address of g_ln_bwd_scratch on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current, on the first call there) and cached
// for the life of the process. A device reset (cudaDeviceReset, or anything
// else that destroys the primary context) unloads the module and can place
// the array elsewhere when it is loaded again: after one, reload the library
// before calling this entry point again (every other object of the library,
// sessions and modules included, is lost with the context too).
float* scratch_on_current_device(int* rc) {
  static std::mutex mu;
  static std::map<int, float*> by_device;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    *rc = SB_OPERR_LAUNCH;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  auto it = by_device.find(dev);
  if (it != by_device.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ln_bwd_scratch) != cudaSuccess || p == nullptr) {
    *rc = SB_OPERR_LAUNCH;
    return nullptr;
  }
  by_device[dev] = static_cast<float*>(p);
  return static_cast<float*>(p);
}

}  // namespace
}  // namespace sb

extern "C" int sb_op_layernorm_bwd_noalloc(uint32_t elem, const void* dy, const void* x, const void* mean,
                                           const void* rstd, const void* gamma, void* dres, void* dgamma,
                                           int32_t rows, int32_t d, void* stream) {
  if ((elem != SB_ELEM_BF16 && elem != SB_ELEM_F32) || !dy || !x || !mean || !rstd || !gamma || !dres || !dgamma ||
      rows <= 0 || d <= 0 || (d & 3))
    return SB_OPERR_ARGS;
  if (d > sb::kMaxWidth) return SB_OPERR_SCRATCH;
  int rc = 0;
  float* scratch = sb::scratch_on_current_device(&rc);
  if (!scratch) return rc;
  // Every block overwrites its own row of partials before column_sum reads
  // it, so nothing left in the array by an earlier call is ever read.
  const bool f = elem == SB_ELEM_F32;
  return sb::layernorm_bwd_capped(static_cast<const float*>(dy), static_cast<const float*>(x),
                                  static_cast<const float*>(mean), static_cast<const float*>(rstd), gamma, f,
                                  static_cast<float*>(dres), dgamma, f, scratch, sb::kScratchFloats / d, rows, d,
                                  static_cast<cudaStream_t>(stream));
}
