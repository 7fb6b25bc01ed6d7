// Sessions, the stream-ordered device pool, buffers and the exported C ABI
// (include/sheaf_b200.h).
//
// Replaces Sheaf's IREE session (sheaf/src/runtime/iree_session.rs), its
// buffer views (device_buffer.rs) and the identity-keyed upload cache
// (buffer_cache.rs): device memory comes from a CUDA memory pool with an
// unlimited release threshold, so freed blocks are recycled in stream order
// instead of being returned to the driver.
#include "runtime.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <thread>

#include "sb_kernels.h"
#include "sb_nn.h"

namespace sb {

sb_status make_status(int code, const std::string& msg) {
  auto* s = new sb_status_s();
  s->code = code;
  s->message = msg;
  return s;
}

size_t elem_size(uint32_t elem) {
  switch (elem) {
    case SB_ELEM_F32:
    case SB_ELEM_I32: return 4;
    case SB_ELEM_BF16:
    case SB_ELEM_F16: return 2;
    default: return 0;
  }
}

bool elem_supported(uint32_t elem) { return elem_size(elem) != 0; }

size_t Buffer::bytes() const {
  size_t n = 1;
  for (int64_t d : shape) n *= static_cast<size_t>(d);
  return n * elem_size(elem);
}

sb_status session_alloc(Session& s, size_t bytes, Allocation** out) {
  void* p = nullptr;
  const size_t sz = bytes ? (bytes + 255) & ~size_t(255) : 256;
  cudaError_t e = cudaMallocFromPoolAsync(&p, sz, s.pool, s.stream);
  if (e != cudaSuccess)
    return make_status(SB_STATUS_RESOURCE_EXHAUSTED, std::string("device pool allocation failed: ") + cudaGetErrorString(e));
  auto* a = new Allocation();
  a->session = &s;
  a->ptr = p;
  a->bytes = sz;
  *out = a;
  s.refs.fetch_add(1);
  return nullptr;
}

void session_release_ref(Session* s);

void allocation_release(Allocation* a) {
  if (!a) return;
  if (a->refs.fetch_sub(1) == 1) {
    Session* s = a->session;
    cudaSetDevice(s->device);
    cudaFreeAsync(a->ptr, s->stream);
    delete a;
    session_release_ref(s);
  }
}

Buffer* buffer_new(Session& s, Allocation* a, size_t offset, std::vector<int64_t> shape, uint32_t elem) {
  auto* b = new sb_buffer_s();
  b->session = &s;
  b->alloc = a;
  b->offset = offset;
  b->shape = std::move(shape);
  b->elem = elem;
  return b;
}

sb_status buffer_create(Session& s, const std::vector<int64_t>& shape, uint32_t elem, Buffer** out) {
  SB_RETURN_IF(!elem_supported(elem), SB_STATUS_INVALID_ARGUMENT, "unsupported element type");
  size_t n = elem_size(elem);
  for (int64_t d : shape) {
    SB_RETURN_IF(d < 0, SB_STATUS_INVALID_ARGUMENT, "negative dimension");
    n *= static_cast<size_t>(d);
  }
  Allocation* a = nullptr;
  SB_TRY(session_alloc(s, n, &a));
  *out = buffer_new(s, a, 0, shape, elem);
  return nullptr;
}

void buffer_release(Buffer* b) {
  if (!b) return;
  if (b->refs.fetch_sub(1) == 1) {
    allocation_release(b->alloc);
    delete static_cast<sb_buffer_s*>(b);
  }
}

void session_release_ref(Session* s) {
  if (s->refs.fetch_sub(1) == 1) {
    cudaSetDevice(s->device);
    cudaStreamSynchronize(s->stream);
    for (auto& kv : s->modules) kv.second->teardown();
    s->modules.clear();
    if (s->comm) comm_destroy(*s);
    if (s->err_word) cudaFree(s->err_word);
    if (s->comm_stream) cudaStreamDestroy(s->comm_stream);
    cudaStreamDestroy(s->stream);
    cudaMemPoolDestroy(s->pool);
    delete static_cast<sb_session_s*>(s);
  }
}

// Waits for `stream` with a deadline; returns DEADLINE_EXCEEDED on timeout.
sb_status wait_stream(cudaStream_t stream, int64_t timeout_ns) {
  cudaEvent_t ev;
  SB_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaEventRecord(ev, stream);
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      cudaEventDestroy(ev);
      return make_status(SB_STATUS_INTERNAL, std::string("device error: ") + cudaGetErrorString(q));
    }
    if (timeout_ns >= 0) {
      const auto el = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0);
      if (el.count() > timeout_ns) {
        cudaEventDestroy(ev);
        return make_status(SB_STATUS_DEADLINE_EXCEEDED, "timed out waiting for the device");
      }
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  cudaEventDestroy(ev);
  return nullptr;
}

}  // namespace sb

using namespace sb;

extern "C" {

bool sb_status_is_ok(sb_status s) { return s == nullptr; }
int sb_status_code(sb_status s) { return s ? s->code : SB_STATUS_OK; }
const char* sb_status_message(sb_status s) { return s ? s->message.c_str() : "OK"; }
void sb_status_free(sb_status s) { delete s; }

sb_status sb_session_create(int device_ordinal, sb_session** out) {
  SB_RETURN_IF(!out, SB_STATUS_INVALID_ARGUMENT, "out_session is null");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
    return make_status(SB_STATUS_UNAVAILABLE, "no CUDA device");
  SB_RETURN_IF(device_ordinal < 0 || device_ordinal >= count, SB_STATUS_INVALID_ARGUMENT, "bad device ordinal");
  cudaDeviceProp prop;
  SB_CUDA_TRY(cudaGetDeviceProperties(&prop, device_ordinal));
  if (prop.major != 10)
    return make_status(SB_STATUS_UNAVAILABLE, "sheaf_b200 kernels are built for sm_100a; device is sm_" +
                                                  std::to_string(prop.major) + std::to_string(prop.minor));
  SB_CUDA_TRY(cudaSetDevice(device_ordinal));
  auto* s = new sb_session_s();
  s->device = device_ordinal;
  // the session's streams take the highest priority: side streams of a
  // module (weight gradients) fill the SMs the critical path leaves idle
  int least = 0, greatest = 0;
  SB_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  SB_CUDA_TRY(cudaStreamCreateWithPriority(&s->stream, cudaStreamNonBlocking, greatest));
  SB_CUDA_TRY(cudaStreamCreateWithPriority(&s->comm_stream, cudaStreamNonBlocking, greatest));
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.handleTypes = cudaMemHandleTypeNone;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = device_ordinal;
  SB_CUDA_TRY(cudaMemPoolCreate(&s->pool, &props));
  uint64_t threshold = UINT64_MAX;
  cudaMemPoolSetAttribute(s->pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  SB_CUDA_TRY(cudaMalloc(&s->err_word, sizeof(int)));
  SB_CUDA_TRY(cudaMemset(s->err_word, 0, sizeof(int)));
  *out = s;
  return nullptr;
}

void sb_session_retain(sb_session* s) {
  if (s) s->refs.fetch_add(1);
}

void sb_session_release(sb_session* s) {
  if (s) session_release_ref(s);
}

sb_status sb_session_synchronize(sb_session* s, int64_t timeout_ns) {
  SB_RETURN_IF(!s, SB_STATUS_INVALID_ARGUMENT, "null session");
  cudaSetDevice(s->device);
  SB_TRY(wait_stream(s->stream, timeout_ns));
  int err = 0;
  SB_CUDA_TRY(cudaMemcpy(&err, s->err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    cudaMemset(s->err_word, 0, sizeof(int));
    return make_status(SB_STATUS_DEADLINE_EXCEEDED, "a kernel's bounded wait timed out (device error word " +
                                                        std::to_string(err) + ")");
  }
  return nullptr;
}

void* sb_session_stream(sb_session* s) { return s ? static_cast<void*>(s->stream) : nullptr; }

sb_status sb_session_get_stats(sb_session* s, sb_session_stats* out) {
  SB_RETURN_IF(!s || !out, SB_STATUS_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  out->calls = s->calls;
  out->graph_captures = s->graph_captures;
  out->graph_replays = s->graph_replays;
  out->kernel_launches = s->kernel_launches;
  return nullptr;
}

sb_status sb_buffer_alloc(sb_session* s, const int64_t* shape, size_t rank, uint32_t elem, sb_buffer** out) {
  SB_RETURN_IF(!s || !out || (rank && !shape), SB_STATUS_INVALID_ARGUMENT, "null argument");
  cudaSetDevice(s->device);
  Buffer* b = nullptr;
  SB_TRY(buffer_create(*s, std::vector<int64_t>(shape, shape + rank), elem, &b));
  *out = static_cast<sb_buffer*>(b);
  return nullptr;
}

sb_status sb_buffer_alloc_copy(sb_session* s, const int64_t* shape, size_t rank, uint32_t elem, const void* host,
                               size_t bytes, sb_buffer** out) {
  SB_RETURN_IF(!host && bytes, SB_STATUS_INVALID_ARGUMENT, "null host pointer");
  sb_buffer* b = nullptr;
  SB_TRY(sb_buffer_alloc(s, shape, rank, elem, &b));
  if (b->bytes() != bytes) {
    buffer_release(b);
    return make_status(SB_STATUS_INVALID_ARGUMENT, "byte length does not match shape and element type");
  }
  if (bytes) {
    cudaError_t e = cudaMemcpyAsync(b->data(), host, bytes, cudaMemcpyHostToDevice, s->stream);
    if (e != cudaSuccess) {
      buffer_release(b);
      return make_status(SB_STATUS_INTERNAL, cudaGetErrorString(e));
    }
  }
  *out = b;
  return nullptr;
}

sb_status sb_buffer_h2d(sb_buffer* b, const void* host, size_t bytes) {
  SB_RETURN_IF(!b || (!host && bytes), SB_STATUS_INVALID_ARGUMENT, "null argument");
  SB_RETURN_IF(bytes != b->bytes(), SB_STATUS_INVALID_ARGUMENT, "byte length mismatch");
  cudaSetDevice(b->session->device);
  SB_CUDA_TRY(cudaMemcpyAsync(b->data(), host, bytes, cudaMemcpyHostToDevice, b->session->stream));
  return nullptr;
}

sb_status sb_buffer_d2h(sb_buffer* b, void* host, size_t bytes, int64_t timeout_ns) {
  SB_RETURN_IF(!b || (!host && bytes), SB_STATUS_INVALID_ARGUMENT, "null argument");
  SB_RETURN_IF(bytes > b->bytes(), SB_STATUS_INVALID_ARGUMENT, "read past end of buffer");
  Session& s = *b->session;
  cudaSetDevice(s.device);
  SB_TRY(wait_stream(s.stream, timeout_ns));
  SB_CUDA_TRY(cudaMemcpyAsync(host, b->data(), bytes, cudaMemcpyDeviceToHost, s.stream));
  return wait_stream(s.stream, timeout_ns);
}

void sb_buffer_retain(sb_buffer* b) {
  if (b) b->refs.fetch_add(1);
}
void sb_buffer_release(sb_buffer* b) { buffer_release(b); }
void sb_buffer_release_many(sb_buffer* const* bufs, size_t n) {
  if (!bufs) return;
  for (size_t i = 0; i < n; ++i)
    if (bufs[i]) buffer_release(bufs[i]);
}
size_t sb_buffer_rank(const sb_buffer* b) { return b ? b->shape.size() : 0; }
int64_t sb_buffer_dim(const sb_buffer* b, size_t axis) {
  return (b && axis < b->shape.size()) ? b->shape[axis] : -1;
}
uint32_t sb_buffer_elem_type(const sb_buffer* b) { return b ? b->elem : 0; }
size_t sb_buffer_byte_length(const sb_buffer* b) { return b ? b->bytes() : 0; }
void* sb_buffer_device_ptr(const sb_buffer* b) { return b ? b->data() : nullptr; }

sb_status sb_module_create_gpt_vag(sb_session* s, const char* name, const sb_gpt_config* c) {
  SB_RETURN_IF(!s || !name || !c, SB_STATUS_INVALID_ARGUMENT, "null argument");
  cudaSetDevice(s->device);
  GptShape g{c->n_layer, c->n_head, c->n_embd, c->block_size, c->vocab_size, c->batch, c->seq, c->elem_type};
  std::unique_ptr<Module> m;
  SB_TRY(make_gpt_vag_module(*s, name, g, &m));
  std::lock_guard<std::mutex> lk(s->mu);
  if (auto it = s->modules.find(name); it != s->modules.end()) it->second->teardown();
  s->modules[name] = std::move(m);
  return nullptr;
}

sb_status sb_module_create_gpt_train(sb_session* s, const char* name, const sb_gpt_config* c,
                                     const sb_adamw_config* o) {
  SB_RETURN_IF(!s || !name || !c || !o, SB_STATUS_INVALID_ARGUMENT, "null argument");
  SB_RETURN_IF(!(o->b1 >= 0.f && o->b1 < 1.f && o->b2 >= 0.f && o->b2 < 1.f && o->eps >= 0.f),
               SB_STATUS_INVALID_ARGUMENT, "adamw: b1, b2 must lie in [0, 1) and eps >= 0");
  cudaSetDevice(s->device);
  GptShape g{c->n_layer, c->n_head, c->n_embd, c->block_size, c->vocab_size, c->batch, c->seq, c->elem_type};
  AdamwConfig a{o->b1, o->b2, o->eps, o->weight_decay, o->max_norm};
  std::unique_ptr<Module> m;
  SB_TRY(make_gpt_vag_module(*s, name, g, &m, &a));
  std::lock_guard<std::mutex> lk(s->mu);
  if (auto it = s->modules.find(name); it != s->modules.end()) it->second->teardown();
  s->modules[name] = std::move(m);
  return nullptr;
}

sb_status sb_module_create_gpt_sampler(sb_session* s, const char* name, const sb_gpt_config* c,
                                       const sb_sampler_config* o) {
  SB_RETURN_IF(!s || !name || !c || !o, SB_STATUS_INVALID_ARGUMENT, "null argument");
  SB_RETURN_IF(c->seq != c->block_size, SB_STATUS_INVALID_ARGUMENT, "sampler: seq must equal block_size");
  cudaSetDevice(s->device);
  GptShape g{c->n_layer, c->n_head, c->n_embd, c->block_size, c->vocab_size, c->batch, c->seq, c->elem_type};
  SamplerConfig sc{o->n_new, o->top_k, o->temperature};
  std::unique_ptr<Module> m;
  SB_TRY(make_gpt_vag_module(*s, name, g, &m, nullptr, &sc));
  std::lock_guard<std::mutex> lk(s->mu);
  if (auto it = s->modules.find(name); it != s->modules.end()) it->second->teardown();
  s->modules[name] = std::move(m);
  return nullptr;
}

sb_status sb_module_load_stablehlo(sb_session* s, const char* text, size_t len, const char** out_name) {
  SB_RETURN_IF(!s || !text, SB_STATUS_INVALID_ARGUMENT, "null argument");
  cudaSetDevice(s->device);
  std::unique_ptr<Module> m;
  SB_TRY(load_stablehlo_module(*s, text, len, &m));
  std::lock_guard<std::mutex> lk(s->mu);
  const std::string name = m->name;
  if (auto it = s->modules.find(name); it != s->modules.end()) it->second->teardown();
  auto& slot = s->modules[name];
  slot = std::move(m);
  if (out_name) *out_name = slot->name.c_str();
  return nullptr;
}

sb_status sb_stablehlo_validate(const char* text, size_t length, char* buf, size_t capacity) {
  SB_RETURN_IF(!text || (!buf && capacity), SB_STATUS_INVALID_ARGUMENT, "null argument");
  std::string summary;
  SB_TRY(validate_stablehlo(text, length, &summary));
  if (capacity) {
    const size_t n = std::min(capacity - 1, summary.size());
    std::memcpy(buf, summary.data(), n);
    buf[n] = '\0';
  }
  return nullptr;
}

sb_status sb_module_describe(sb_session* s, const char* module_name, char* buf, size_t capacity) {
  SB_RETURN_IF(!s || !module_name || (!buf && capacity), SB_STATUS_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  auto it = s->modules.find(module_name);
  if (it == s->modules.end()) return make_status(SB_STATUS_NOT_FOUND, std::string("module not loaded: ") + module_name);
  const std::string d = describe_stablehlo_module(it->second.get());
  if (capacity) {
    const size_t n = std::min(capacity - 1, d.size());
    std::memcpy(buf, d.data(), n);
    buf[n] = '\0';
  }
  return nullptr;
}

sb_status sb_call(sb_session* s, const char* qualified_name, sb_buffer* const* inputs, size_t in_count,
                  sb_buffer** outputs, size_t out_capacity, size_t* out_count) {
  SB_RETURN_IF(!s || !qualified_name || (in_count && !inputs) || !out_count, SB_STATUS_INVALID_ARGUMENT,
               "null argument");
  const std::string q(qualified_name);
  const size_t dot = q.rfind('.');
  SB_RETURN_IF(dot == std::string::npos, SB_STATUS_INVALID_ARGUMENT, "expected <module>.<function>");
  const std::string mod = q.substr(0, dot), fn = q.substr(dot + 1);
  cudaSetDevice(s->device);
  // a runtime error left by the caller's own CUDA work must not be reported
  // as a failure of this call's launches
  (void)cudaGetLastError();
  std::vector<Buffer*> in(inputs, inputs + in_count);
  for (Buffer* b : in) {
    SB_RETURN_IF(!b, SB_STATUS_INVALID_ARGUMENT, "null input buffer");
    SB_RETURN_IF(b->session != s, SB_STATUS_INVALID_ARGUMENT, "input buffer belongs to another session");
  }
  std::vector<Buffer*> out;
  {
    std::lock_guard<std::mutex> lk(s->mu);
    auto it = s->modules.find(mod);
    if (it == s->modules.end()) return make_status(SB_STATUS_NOT_FOUND, "module not loaded: " + mod);
    if (!it->second->has_function(fn)) return make_status(SB_STATUS_NOT_FOUND, "function not found: " + q);
    s->calls++;
    SB_TRY(it->second->call(*s, fn, in, out));
  }
  if (out.size() > out_capacity) {
    for (Buffer* b : out) buffer_release(b);
    return make_status(SB_STATUS_INVALID_ARGUMENT, "output capacity too small: need " + std::to_string(out.size()));
  }
  for (size_t i = 0; i < out.size(); ++i) outputs[i] = static_cast<sb_buffer*>(out[i]);
  *out_count = out.size();
  return nullptr;
}

}  // extern "C"
