// Executor runtime behind the C ABI (include/sheaf_b200.h): sessions, device
// buffers, modules. Replaces the IREE runtime objects Sheaf drives today
// (sheaf/src/runtime/iree_session.rs, device_buffer.rs, buffer_cache.rs).
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/sheaf_b200.h"

namespace sb {

// Owned error object handed across the C ABI (NULL status = OK).
struct StatusObj {
  int code;
  std::string message;
};

sb_status make_status(int code, const std::string& msg);
#define SB_RETURN_IF(cond, code, msg) \
  do {                                \
    if (cond) return ::sb::make_status((code), (msg)); \
  } while (0)
#define SB_CUDA_TRY(expr)                                                                       \
  do {                                                                                          \
    cudaError_t e_ = (expr);                                                                    \
    if (e_ != cudaSuccess)                                                                      \
      return ::sb::make_status(SB_STATUS_INTERNAL, std::string(#expr ": ") + cudaGetErrorString(e_)); \
  } while (0)
#define SB_TRY(expr)              \
  do {                            \
    sb_status s_ = (expr);        \
    if (s_) return s_;            \
  } while (0)

size_t elem_size(uint32_t elem);
bool elem_supported(uint32_t elem);

struct Session;

// A device allocation from the session's stream-ordered pool. Buffers are
// views (offset + shape) into one; it is returned to the pool when the last
// view is released.
struct Allocation {
  Session* session;
  void* ptr;
  size_t bytes;
  std::atomic<int> refs{1};
};

struct Buffer {
  std::atomic<int> refs{1};
  Session* session;
  Allocation* alloc;
  size_t offset;
  std::vector<int64_t> shape;
  uint32_t elem;
  size_t bytes() const;
  void* data() const { return static_cast<char*>(alloc->ptr) + offset; }
};

// A loaded module: named functions executed on the session stream.
struct Module {
  std::string name;
  virtual ~Module() = default;
  virtual bool has_function(const std::string& fn) const = 0;
  virtual sb_status call(Session& s, const std::string& fn, const std::vector<Buffer*>& in,
                         std::vector<Buffer*>& out) = 0;
  // Releases CUDA graphs and device state before the session goes away.
  virtual void teardown() {}
  // With `on` false, calls run on this rank's inputs alone even when the
  // session belongs to a data-parallel group (no gradient all-reduce).
  virtual void set_collectives(bool on) { (void)on; }
};

struct Comm;  // NCCL communicator wrapper (comm.cpp)

struct Session {
  std::atomic<int> refs{1};
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t comm_stream = nullptr;
  cudaMemPool_t pool = nullptr;
  int* err_word = nullptr;  // device word written by bounded waits
  std::mutex mu;            // guards modules / plan state; released before GPU waits
  std::map<std::string, std::unique_ptr<Module>> modules;
  Comm* comm = nullptr;
  int rank = 0, world = 1;
  // statistics (dispatch profile in the spirit of iree_session.rs:250-297)
  uint64_t calls = 0, graph_replays = 0, graph_captures = 0, kernel_launches = 0;
};

sb_status session_alloc(Session& s, size_t bytes, Allocation** out);
void allocation_release(Allocation* a);
Buffer* buffer_new(Session& s, Allocation* a, size_t offset, std::vector<int64_t> shape, uint32_t elem);
sb_status buffer_create(Session& s, const std::vector<int64_t>& shape, uint32_t elem, Buffer** out);
void buffer_release(Buffer* b);

// Builds the fused nanoGPT value-and-grad module (gpt_vag.cpp).
struct GptShape {
  int n_layer, n_head, n_embd, block_size, vocab, batch, seq;
  uint32_t elem;  // SB_ELEM_BF16 or SB_ELEM_F32 (parameter / compute type)
};
struct AdamwConfig {
  float b1, b2, eps, wd, max_norm;
};
struct SamplerConfig {
  int n_new, top_k;
  float temperature;
};
// With `adamw`, the module also runs the train-step function (VAG + clip +
// AdamW in one graph); with `sampler`, the generate function (window forward
// + top-k sampling per token, one graph replayed per token).
sb_status make_gpt_vag_module(Session& s, const std::string& name, const GptShape& g, std::unique_ptr<Module>* out,
                              const AdamwConfig* adamw = nullptr, const SamplerConfig* sampler = nullptr);

// Parses StableHLO text and maps it onto the kernel library (stablehlo.cpp).
sb_status load_stablehlo_module(Session& s, const char* text, size_t len, std::unique_ptr<Module>* out);
std::string describe_stablehlo_module(Module* m);
sb_status validate_stablehlo(const char* text, size_t len, std::string* summary);

// NCCL data-parallel group (comm.cpp).
sb_status comm_init(Session& s, const void* unique_id, size_t id_bytes, int rank, int world);
sb_status comm_get_unique_id(void* out, size_t bytes);
sb_status comm_allreduce_avg(Session& s, void* data, size_t count, uint32_t elem, cudaStream_t stream);
void comm_destroy(Session& s, bool abort = false);

}  // namespace sb

// The opaque C-ABI handle types are the runtime objects themselves.
struct sb_status_s : sb::StatusObj {};
struct sb_session_s : sb::Session {};
struct sb_buffer_s : sb::Buffer {};
