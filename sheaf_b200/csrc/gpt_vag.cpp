// The fused nanoGPT value_and_grad module.
//
// Executes the graph Sheaf compiles for
//   ((value-and-grad (fn [p] (cross-entropy-loss (gpt-forward x p config) y))) params)
// (examples/nanogpt/train.shf:26-28, model.shf:85-113, lib/nn.shf:44-50) as a
// fixed schedule of library kernels instead of IREE dispatches:
//   forward : embedding gather + wpe slice; per layer LN -> QKV GEMM ->
//             fused causal attention -> proj GEMM (+residual) -> LN ->
//             fc GEMM (+GELU epilogue) -> fc2 GEMM (+residual); each LN also
//             copies its input to the next residual buffer, into which the
//             residual GEMM accumulates with bulk tensor reduce-adds (the
//             residual stream in the module's element type: a bf16 module
//             adds and rounds in bf16, as its compiled graph does);
//             final LN -> head GEMM -> fused cross-entropy fwd+VJP
//   backward: the `@` VJP GEMMs (dX with K-major / N-major operands, dW
//             contracted over all tokens with split-K), GELU-VJP fused in the
//             dX epilogue, LN VJP accumulating into the residual gradient,
//             fused attention VJP, embedding scatter-add + wpe pad.
// Inputs follow the module signature Sheaf's compile_vag produces
// (jit/vag.rs:126-141): the params pytree leaves (sorted keys, buffer_convert.rs
// :218-246), then the captured x and y token ids (f32). Outputs are
// (loss, grad leaves...) (jit/vag.rs:565-574).
//
// Schedule: parameters are copied into plan-owned slots (one batched-copy
// launch), the compute sequence is replayed from a CUDA graph, and the
// gradients + loss are copied into one fresh pool allocation that backs all
// the output buffers. With a data-parallel group, per-layer gradient buckets
// are all-reduced on a second stream as soon as the layer's weight gradients
// are complete, overlapping the rest of the backward pass.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "runtime.h"
#include "sb_kernels.h"
#include "sb_nn.h"

namespace sb {

namespace {

constexpr int kMaxSegs = 48;

struct CopySegs {
  const char* src[kMaxSegs];
  char* dst[kMaxSegs];
  unsigned long long bytes[kMaxSegs];
  int n;
};

__global__ void batched_copy_kernel(CopySegs c) {
  const int seg = blockIdx.y;
  if (seg >= c.n) return;
  const char* s = c.src[seg];
  char* d = c.dst[seg];
  const size_t n = c.bytes[seg];
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0) {
    const size_t n16 = n / 16;
    for (size_t i = tid; i < n16; i += stride) reinterpret_cast<uint4*>(d)[i] = reinterpret_cast<const uint4*>(s)[i];
    for (size_t i = n16 * 16 + tid; i < n; i += stride) d[i] = s[i];
  } else {
    for (size_t i = tid; i < n; i += stride) d[i] = s[i];
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

class GptVagModule : public Module {
 public:
  GptShape g{};
  bool bf = true;
  size_t es = 2;
  int L = 0, H = 0, D = 0, V = 0, P = 0, B = 0, T = 0, N = 0, ldl = 0;
  std::vector<std::vector<int64_t>> shapes;
  std::vector<size_t> offs;
  size_t grads_bytes = 0, loss_off = 0, out_bytes = 0;

  std::vector<void*> owned;
  char* params = nullptr;
  char* grads = nullptr;  // gradients followed by the loss (output element type)
  float* ids = nullptr;   // x ids [N] then y ids [N]
  float* loss_f32 = nullptr;
  std::vector<void*> xs, xmid;  // residual stream, model element type
  std::vector<float*> mean1, rstd1, mean2, rstd2, lse;
  float *meanf = nullptr, *rstdf = nullptr;
  std::vector<void*> h1, h2, qkv, att, gder, gact;  // gder = gelu'(u) saved for the VJP
  void *hf = nullptr, *logits = nullptr, *dlogits = nullptr;
  // gradient of the residual stream: f32, updated in place (f32 module), or
  // two bf16 buffers the layer-norm VJPs read and write in turn (bf16)
  float* dres = nullptr;
  void* dres_bf = nullptr;
  void* dh = nullptr;  // dy of the layer-norm VJPs, model element type (as the module materialises it)
  void *du = nullptr, *dout = nullptr, *dqkv = nullptr;
  __nv_bfloat16* onehot = nullptr;  // bf16 one-hot [N, ldl] of the x ids (small vocabularies, bf16 plan)
  float* ws = nullptr;
  size_t ws_bytes = 0;

  // train-step (with an AdamW configuration): m, v copied in (parameter
  // layout), t and lr, and the updated state [loss | m | params | t | v]
  bool train = false;
  AdamwConfig opt{};
  char* mbuf = nullptr;
  char* vbuf = nullptr;
  float* tl = nullptr;  // tl[0] = t, tl[1] = lr
  char* state = nullptr;
  size_t st_m = 0, st_p = 0, st_t = 0, st_v = 0, st_bytes = 0;
  float* opt_ws = nullptr;
  size_t opt_ws_bytes = 0;

  // sampling (generate): keys [B, 4], tokens [B, n_new], the device step
  // counter and the last-position logits of every step [n_new, B, V]
  bool sampler = false;
  int n_new = 0, top_k = 0;
  float temperature = 1.f;
  float* keys_buf = nullptr;
  float* tokens_buf = nullptr;
  int* step_ctr = nullptr;
  float* step_logits = nullptr;
  size_t gen_tok = 0, gen_ids = 0, gen_keys = 0, gen_logits = 0, gen_bytes = 0;
  void* sample_ws = nullptr;  // the long-vocabulary sort's scratch
  size_t sample_ws_bytes = 0;

  // one captured graph per function (value_and_grad, train_step, one token
  // of generate), its kernel nodes and the eager runs before the capture
  enum Mode { kVag, kTrain, kSample, kModes };
  cudaGraphExec_t exec[kModes] = {};
  bool exec_dp[kModes] = {};  // whether the captured graph holds the all-reduce
  uint64_t kernels[kModes] = {};
  int eager[kModes] = {};
  bool use_graph = true;
  std::vector<cudaEvent_t> bucket_events;
  cudaEvent_t comm_done = nullptr;

  // bf16 backward: the weight-gradient GEMMs run on a low-priority side
  // stream beside the critical path (dX GEMMs, layer-norm and attention
  // VJPs), filling the SMs its tails leave idle. The operands they read are
  // double-buffered (residual gradient by writer, dU and dqkv by layer parity) so the
  // critical path only waits for a dW GEMM before overwriting its operand.
  bool dw_side = false;
  cudaStream_t wst = nullptr;
  float* ws_w = nullptr;  // split-K workspace of the side stream
  size_t ws_w_bytes = 0;
  void *dres_bf2 = nullptr, *du2 = nullptr, *dqkv2 = nullptr;
  std::vector<cudaEvent_t> xev;

  ~GptVagModule() override { teardown(); }

  void teardown() override {
    for (auto& e : exec) {
      if (e) cudaGraphExecDestroy(e);
      e = nullptr;
    }
    for (auto e : bucket_events) cudaEventDestroy(e);
    bucket_events.clear();
    if (comm_done) cudaEventDestroy(comm_done);
    comm_done = nullptr;
    for (auto e : xev) cudaEventDestroy(e);
    xev.clear();
    if (wst) cudaStreamDestroy(wst);
    wst = nullptr;
    for (void* p : owned) cudaFree(p);
    owned.clear();
  }

  // false: calls skip the gradient all-reduce even in a data-parallel
  // session (the front door's first-call check compares per-rank results)
  bool collectives = true;
  void set_collectives(bool on) override { collectives = on; }
  bool group(const Session& s) const { return collectives && s.comm != nullptr && s.world > 1; }

  bool has_function(const std::string& fn) const override {
    return fn == "value_and_grad" || (train && fn == "train_step") || (sampler && fn == "generate");
  }

  // Parameter pointers the kernels read: the plan-owned slots, or (for
  // value_and_grad on resident, 256-byte-aligned parameter buffers) the input
  // buffers themselves, read in place as the reference's DeviceBuffer inputs
  // are (iree_session.rs:505-519). A captured graph records the pointer set it
  // was captured with and is recaptured when a call brings another one.
  std::vector<void*> pin;
  std::vector<void*> exec_pin[kModes];
  void* Pp(int i) const { return pin[i]; }
  void* slot(int i) const { return params + offs[i]; }
  // Points the plan at `ptrs` for the next run of `mode`.
  sb_status use_params(const std::vector<void*>& ptrs, Mode mode, cudaStream_t st) {
    pin = ptrs;
    if (exec[mode] && exec_pin[mode] != pin) {
      SB_CUDA_TRY(cudaStreamSynchronize(st));
      cudaGraphExecDestroy(exec[mode]);
      exec[mode] = nullptr;
    }
    return nullptr;
  }
  std::vector<void*> slots() const {
    std::vector<void*> v(shapes.size());
    for (size_t i = 0; i < shapes.size(); ++i) v[i] = slot(static_cast<int>(i));
    return v;
  }
  void* Gp(int i) const { return grads + offs[i]; }

  sb_status dev(size_t bytes, void** p) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return make_status(SB_STATUS_RESOURCE_EXHAUSTED, "plan allocation failed");
    owned.push_back(*p);
    return nullptr;
  }
  template <typename T>
  sb_status devt(size_t count, T** p) {
    void* v = nullptr;
    SB_TRY(dev(count * sizeof(T), &v));
    *p = static_cast<T*>(v);
    return nullptr;
  }

  GemmDesc desc(const void* A, long lda, bool a_mn, const void* Bm, long ldb, bool b_mn, int M, int Nn, int K,
                void* out, long ldo, bool out_f32) const {
    GemmDesc d;
    d.A = A;
    d.lda = lda;
    d.a_mn = a_mn;
    d.B = Bm;
    d.ldb = ldb;
    d.b_mn = b_mn;
    d.M = M;
    d.N = Nn;
    d.K = K;
    d.out = out;
    d.ldo = ldo;
    d.out_f32 = out_f32;
    return d;
  }

  // Weight-gradient GEMMs beside the critical path split their token
  // dimension over at most 108 CTAs, and CTA-pair tiles at most 6 ways: they
  // then occupy about three quarters of the SMs and leave the rest to the
  // critical path's kernels. Measured on nanoGPT-char (ms/step): at most 6
  // splits for every GEMM 2.304; the same with the 384 x 384 proj weight
  // gradient on 6 tiles x 18 splits (the CTA cap) 2.266-2.274, x 24 splits
  // 2.281; the CTA cap alone (pair tiles at 9-10 splits) 2.305; the
  // full-GPU choice for every GEMM slower still. With the bf16 residual
  // stream: 2.107-2.109 at 108 CTAs, 2.118-2.119 at 132, 2.161-2.163 at 84. On GPT-2-small the CTA cap
  // puts the fc and fc2 weight gradients (36 pair tiles each) on one split
  // instead of two: 9.26-9.30 -> 9.00-9.08 ms/step.
  static constexpr int kSideCtas = 108;
  static constexpr int kSidePairSplits = 6;

  int gemm(const GemmDesc& d0, cudaStream_t st, int* err, bool side = false) const {
    GemmDesc d = d0;
    if (side) {
      d.max_ctas = kSideCtas;
      d.max_pair_splits = kSidePairSplits;
    }
    float* w = side ? ws_w : ws;
    const size_t wb = side ? ws_w_bytes : ws_bytes;
    return bf ? gemm_bf16(d, w, wb, st, err) : gemm_f32(d, w, wb, st, err);
  }

  // All GEMMs of one step (used for workspace sizing).
  std::vector<GemmDesc> all_gemms() const {
    std::vector<GemmDesc> v;
    const bool f = !bf;
    v.push_back(desc(nullptr, D, false, nullptr, D, false, N, 3 * D, D, nullptr, 3 * D, f));
    v.push_back(desc(nullptr, D, false, nullptr, D, false, N, D, D, nullptr, D, true));
    v.push_back(desc(nullptr, D, false, nullptr, D, false, N, 4 * D, D, nullptr, 4 * D, f));
    v.push_back(desc(nullptr, 4 * D, false, nullptr, 4 * D, false, N, D, 4 * D, nullptr, D, true));
    v.push_back(desc(nullptr, D, false, nullptr, D, false, N, V, D, nullptr, ldl, f));
    v.push_back(desc(nullptr, ldl, false, nullptr, D, true, N, D, V, nullptr, D, true));
    v.push_back(desc(nullptr, ldl, true, nullptr, D, true, V, D, N, nullptr, D, f));
    v.push_back(desc(nullptr, D, true, nullptr, 4 * D, true, D, 4 * D, N, nullptr, 4 * D, f));
    v.push_back(desc(nullptr, 4 * D, true, nullptr, D, true, 4 * D, D, N, nullptr, D, f));
    v.push_back(desc(nullptr, D, true, nullptr, D, true, D, D, N, nullptr, D, f));
    v.push_back(desc(nullptr, 3 * D, true, nullptr, D, true, 3 * D, D, N, nullptr, D, f));
    return v;
  }

  sb_status build(const std::string& nm, const GptShape& shape, const AdamwConfig* adamw,
                  const SamplerConfig* smp) {
    name = nm;
    g = shape;
    SB_RETURN_IF(g.elem != SB_ELEM_BF16 && g.elem != SB_ELEM_F32, SB_STATUS_INVALID_ARGUMENT,
                 "gpt module element type must be bf16 or f32");
    SB_RETURN_IF(g.n_layer <= 0 || g.n_head <= 0 || g.n_embd <= 0 || g.vocab <= 0 || g.batch <= 0 || g.seq <= 0,
                 SB_STATUS_INVALID_ARGUMENT, "non-positive gpt dimension");
    SB_RETURN_IF(g.n_embd % g.n_head != 0, SB_STATUS_INVALID_ARGUMENT, "n_embd must be divisible by n_head");
    SB_RETURN_IF(g.seq > g.block_size, SB_STATUS_INVALID_ARGUMENT, "seq exceeds block_size (wpe rows)");
    const int hd = g.n_embd / g.n_head;
    SB_RETURN_IF(hd != 64 && hd != 32, SB_STATUS_UNIMPLEMENTED, "attention head dim must be 32 or 64");
    SB_RETURN_IF(g.n_embd % 64 != 0, SB_STATUS_UNIMPLEMENTED, "n_embd must be a multiple of 64");
    bf = g.elem == SB_ELEM_BF16;
    es = bf ? 2 : 4;
    L = g.n_layer;
    H = g.n_head;
    D = g.n_embd;
    V = g.vocab;
    P = g.block_size;
    B = g.batch;
    T = g.seq;
    N = B * T;
    ldl = (V + 7) / 8 * 8;
    use_graph = !(std::getenv("SHEAF_B200_GRAPH") && std::string(std::getenv("SHEAF_B200_GRAPH")) == "0");

    shapes.push_back({V, D});
    for (int l = 0; l < L; ++l) {
      shapes.push_back({3 * D, D});
      shapes.push_back({D, D});
      shapes.push_back({D});
      shapes.push_back({D});
      shapes.push_back({4 * D, D});
      shapes.push_back({D, 4 * D});
    }
    shapes.push_back({D});
    shapes.push_back({P, D});
    shapes.push_back({V, D});
    size_t off = 0;
    for (auto& s : shapes) {
      offs.push_back(off);
      size_t n = es;
      for (auto d : s) n *= static_cast<size_t>(d);
      off = align256(off + n);
    }
    grads_bytes = off;
    loss_off = off;
    out_bytes = align256(off + 4);

    void* v;
    SB_TRY(dev(grads_bytes, &v));
    params = static_cast<char*>(v);
    pin = slots();
    SB_TRY(dev(out_bytes, &v));
    grads = static_cast<char*>(v);
    cudaMemset(grads, 0, out_bytes);
    SB_TRY(devt(2 * static_cast<size_t>(N), &ids));
    SB_TRY(devt(4, &loss_f32));
    const size_t nd = static_cast<size_t>(N) * D;
    for (int l = 0; l <= L; ++l) {
      void* q;
      SB_TRY(dev(nd * es, &q));
      xs.push_back(q);
    }
    for (int l = 0; l < L; ++l) {
      float* p;
      void* q;
      SB_TRY(dev(nd * es, &q));
      xmid.push_back(q);
      for (auto* vec : {&mean1, &rstd1, &mean2, &rstd2}) {
        SB_TRY(devt(N, &p));
        vec->push_back(p);
      }
      SB_TRY(devt(static_cast<size_t>(B) * H * T, &p));
      lse.push_back(p);
      SB_TRY(dev(nd * es, &q));
      h1.push_back(q);
      SB_TRY(dev(nd * es, &q));
      h2.push_back(q);
      SB_TRY(dev(3 * nd * es, &q));
      qkv.push_back(q);
      SB_TRY(dev(nd * es, &q));
      att.push_back(q);
      SB_TRY(dev(4 * nd * es, &q));
      gder.push_back(q);
      SB_TRY(dev(4 * nd * es, &q));
      gact.push_back(q);
    }
    SB_TRY(devt(N, &meanf));
    SB_TRY(devt(N, &rstdf));
    SB_TRY(dev(nd * es, &hf));
    SB_TRY(dev(static_cast<size_t>(N) * ldl * es, &logits));
    SB_TRY(dev(static_cast<size_t>(N) * ldl * es, &dlogits));
    cudaMemset(logits, 0, static_cast<size_t>(N) * ldl * es);
    cudaMemset(dlogits, 0, static_cast<size_t>(N) * ldl * es);
    if (bf) {
      SB_TRY(dev(nd * 2, &dres_bf));
      SB_TRY(dev(nd * 2, &dres_bf2));
    } else {
      SB_TRY(devt(nd, &dres));
    }
    SB_TRY(dev(nd * es, &dh));
    SB_TRY(dev(4 * nd * es, &du));
    SB_TRY(dev(nd * es, &dout));
    SB_TRY(dev(3 * nd * es, &dqkv));
    if (bf && V <= 256) {
      void* oh = nullptr;
      SB_TRY(dev(static_cast<size_t>(N) * ldl * 2, &oh));
      onehot = static_cast<__nv_bfloat16*>(oh);
    }

    size_t w = 0;
    for (auto& d : all_gemms()) w = std::max(w, gemm_workspace_bytes(d, bf));
    w = std::max(w, layernorm_bwd_workspace_bytes(N, D));
    w = std::max(w, cross_entropy_workspace_bytes(N));
    w = std::max(w, attention_bwd_workspace_bytes(!bf, AttnShape{B, T, H, D / H}));
    w = std::max(w, embedding_bwd_workspace_bytes(V, D));
    ws_bytes = align256(w);
    SB_TRY(devt(ws_bytes / 4 + 64, &ws));

    const char* side_env = std::getenv("SHEAF_B200_DW_STREAM");
    dw_side = bf && !smp && !(side_env && std::string(side_env) == "0");
    if (dw_side) {
      int least = 0, greatest = 0;
      SB_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
      SB_CUDA_TRY(cudaStreamCreateWithPriority(&wst, cudaStreamNonBlocking, least));
      size_t w2 = 0;
      for (auto& d : all_gemms())
        if (d.K == N) w2 = std::max(w2, gemm_workspace_bytes(d, bf));  // the dW GEMMs contract over tokens
      ws_w_bytes = align256(w2);
      SB_TRY(devt(ws_w_bytes / 4 + 64, &ws_w));
      SB_TRY(dev(4 * nd * es, &du2));
      SB_TRY(dev(3 * nd * es, &dqkv2));
      for (int i = 0; i < 8 * L + 8; ++i) {
        cudaEvent_t e;
        SB_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        xev.push_back(e);
      }
    }

    if (adamw) {
      train = true;
      opt = *adamw;
      SB_TRY(dev(grads_bytes, &v));
      mbuf = static_cast<char*>(v);
      SB_TRY(dev(grads_bytes, &v));
      vbuf = static_cast<char*>(v);
      SB_TRY(devt(64, &tl));
      st_m = 256;
      st_p = st_m + grads_bytes;
      st_t = st_p + grads_bytes;
      st_v = st_t + 256;
      st_bytes = st_v + grads_bytes;
      SB_TRY(dev(st_bytes, &v));
      state = static_cast<char*>(v);
      cudaMemset(state, 0, st_bytes);
      std::vector<int64_t> cnt = leaf_counts();
      opt_ws_bytes = align256(optimizer_workspace_bytes(cnt.data(), static_cast<int>(cnt.size())));
      SB_TRY(devt(opt_ws_bytes / 4 + 64, &opt_ws));
    }
    if (smp) {
      SB_RETURN_IF(smp->n_new <= 0 || smp->top_k <= 0 || !(smp->temperature > 0.f), SB_STATUS_INVALID_ARGUMENT,
                   "sampler: n_new and top_k must be positive, temperature > 0");
      SB_RETURN_IF(V > kSampleMaxVocab || (V > kSampleSmemVocab && T > 4096), SB_STATUS_UNIMPLEMENTED,
                   "sampler: vocabulary or window beyond the on-device sort");
      sampler = true;
      n_new = smp->n_new;
      top_k = smp->top_k;
      temperature = smp->temperature;
      SB_TRY(devt(static_cast<size_t>(B) * 4, &keys_buf));
      SB_TRY(devt(static_cast<size_t>(B) * n_new, &tokens_buf));
      SB_TRY(devt(64, &step_ctr));
      SB_TRY(devt(static_cast<size_t>(n_new) * B * V, &step_logits));
      sample_ws_bytes = sample_workspace_bytes(B, V);
      if (sample_ws_bytes) SB_TRY(dev(sample_ws_bytes, &sample_ws));
      // outputs of generate: tokens | ids | keys | step logits (all f32)
      gen_tok = 0;
      gen_ids = align256(gen_tok + static_cast<size_t>(B) * n_new * 4);
      gen_keys = align256(gen_ids + static_cast<size_t>(N) * 4);
      gen_logits = align256(gen_keys + static_cast<size_t>(B) * 16);
      gen_bytes = align256(gen_logits + static_cast<size_t>(n_new) * B * V * 4);
    }
    return nullptr;
  }

  std::vector<int64_t> leaf_counts() const {
    std::vector<int64_t> c;
    for (auto& sh : shapes) {
      int64_t n = 1;
      for (auto d : sh) n *= d;
      c.push_back(n);
    }
    return c;
  }

  // Launches the whole fwd+VJP step on `st` (optionally with the gradient
  // all-reduce on the session's comm stream).
  sb_status enqueue(Session& s, cudaStream_t st, Mode mode) {
    const bool train_step = mode == kTrain;
    int* err = s.err_word;
    const bool f32 = !bf;
    const bool dp = group(s);
    const AttnShape ash{B, T, H, D / H};
    int rc = 0;
#define SB_K(expr)                                                                                  \
  do {                                                                                              \
    rc = (expr);                                                                                    \
    if (rc) return make_status(SB_STATUS_INTERNAL, std::string("launch failed (") + std::to_string(rc) + "): " #expr); \
  } while (0)
    const int iw = 3 + 6 * L, ip = 2 + 6 * L, ilnf = 1 + 6 * L;

    // ---- forward
    SB_K(embedding_fwd(ids, Pp(iw), Pp(ip), f32, xs[0], f32, N, T, V, D, st));
    for (int l = 0; l < L; ++l) {
      const int b0 = 1 + 6 * l;
      // LN1 also copies x into xmid, which the proj GEMM then accumulates into
      SB_K(layernorm_fwd(xs[l], f32, Pp(b0 + 2), f32, h1[l], f32, mean1[l], rstd1[l], N, D, st, xmid[l]));
      SB_K(gemm(desc(h1[l], D, false, Pp(b0 + 0), D, false, N, 3 * D, D, qkv[l], 3 * D, f32), st, err));
      SB_K(attention_fwd(qkv[l], f32, att[l], lse[l], ash, st));
      {
        GemmDesc d = desc(att[l], D, false, Pp(b0 + 1), D, false, N, D, D, xmid[l], D, f32);
        d.epi = EPI_ACCUM;  // xmid = x + att @ Wproj^T
        SB_K(gemm(d, st, err));
      }
      SB_K(layernorm_fwd(xmid[l], f32, Pp(b0 + 3), f32, h2[l], f32, mean2[l], rstd2[l], N, D, st, xs[l + 1]));
      {
        GemmDesc d = desc(h2[l], D, false, Pp(b0 + 4), D, false, N, 4 * D, D, gact[l], 4 * D, f32);
        d.epi = EPI_GELU;
        d.out2 = gder[l];
        d.ldo2 = 4 * D;
        SB_K(gemm(d, st, err));
      }
      {
        GemmDesc d = desc(gact[l], 4 * D, false, Pp(b0 + 5), 4 * D, false, N, D, 4 * D, xs[l + 1], D, f32);
        d.epi = EPI_ACCUM;  // x' = xmid + gelu(...) @ Wfc2^T
        SB_K(gemm(d, st, err));
      }
    }
    SB_K(layernorm_fwd(xs[L], f32, Pp(ilnf), f32, hf, f32, meanf, rstdf, N, D, st));
    SB_K(gemm(desc(hf, D, false, Pp(0), D, false, N, V, D, logits, ldl, f32), st, err));
    if (mode == kSample) {
      SB_K(sample_step(logits, f32, ldl, B, T, V, top_k, temperature, ids, keys_buf, tokens_buf, n_new, step_ctr,
                       step_logits, sample_ws, sample_ws_bytes, st));
      return nullptr;
    }
    SB_K(cross_entropy_fwd_bwd(logits, f32, ldl, N, V, ids + N, dlogits, ldl, ws, loss_f32, nullptr, st));

    // ---- backward
    SB_K(gemm(desc(dlogits, ldl, false, Pp(0), D, true, N, D, V, dh, D, f32), st, err));
    SB_K(gemm(desc(dlogits, ldl, true, hf, D, true, V, D, N, Gp(0), D, f32), st, err));
    // residual-stream gradient buffers: r0 is written by the LN_f and LN1
    // VJPs, r1 by LN2's (the same f32 buffer in an f32 module)
    void* r0 = bf ? dres_bf : static_cast<void*>(dres);
    void* r1 = bf ? dres_bf2 : r0;
    SB_K(layernorm_bwd(dh, f32, xs[L], f32, meanf, rstdf, Pp(ilnf), f32, nullptr, r0, Gp(ilnf), f32, ws, N, D, st));
    int bucket = 0;
    // the all-reduce of a bucket waits for the main stream and, when given,
    // a side-stream mark
    auto launch_bucket = [&](size_t lo_off, size_t hi_off, cudaEvent_t side_ev) -> sb_status {
      if (!dp) return nullptr;
      cudaEvent_t ev = bucket_events[bucket++];
      SB_CUDA_TRY(cudaEventRecord(ev, st));
      SB_CUDA_TRY(cudaStreamWaitEvent(s.comm_stream, ev, 0));
      if (side_ev) SB_CUDA_TRY(cudaStreamWaitEvent(s.comm_stream, side_ev, 0));
      return comm_allreduce_avg(s, grads + lo_off, (hi_off - lo_off) / es, g.elem, s.comm_stream);
    };
    SB_TRY(launch_bucket(offs[0], offs[1], nullptr));

    // Weight gradients go to the side stream (in line when there is none).
    cudaStream_t sst = dw_side ? wst : st;
    int nev = 0;
    auto fork = [&]() -> sb_status {  // the side stream waits for the main stream's work so far
      if (!dw_side) return nullptr;
      cudaEvent_t e = xev[nev++];
      SB_CUDA_TRY(cudaEventRecord(e, st));
      SB_CUDA_TRY(cudaStreamWaitEvent(wst, e, 0));
      return nullptr;
    };
    auto mark = [&](cudaEvent_t& e) -> sb_status {  // a point on the side stream
      if (!dw_side) return nullptr;
      e = xev[nev++];
      SB_CUDA_TRY(cudaEventRecord(e, wst));
      return nullptr;
    };
    auto wait = [&](cudaEvent_t e) -> sb_status {  // the main stream waits for a side-stream point
      if (dw_side && e) SB_CUDA_TRY(cudaStreamWaitEvent(st, e, 0));
      return nullptr;
    };
    std::vector<cudaEvent_t> ev_fc2(L, nullptr), ev_fc(L, nullptr), ev_proj(L, nullptr), ev_qkv(L, nullptr);
    for (int l = L - 1; l >= 0; --l) {
      const int b0 = 1 + 6 * l;
      void* dul = (dw_side && (l & 1)) ? du2 : du;
      void* dql = (dw_side && (l & 1)) ? dqkv2 : dqkv;
      SB_TRY(fork());
      SB_K(gemm(desc(r0, D, true, gact[l], 4 * D, true, D, 4 * D, N, Gp(b0 + 5), 4 * D, f32), sst, err, dw_side));
      SB_TRY(mark(ev_fc2[l]));
      if (l + 2 < L) SB_TRY(wait(ev_fc[l + 2]));  // dU buffer last read by dW_fc two layers up
      {
        GemmDesc d = desc(r0, D, false, Pp(b0 + 5), 4 * D, true, N, 4 * D, D, dul, 4 * D, f32);
        d.epi = EPI_MUL;
        d.aux = gder[l];
        d.ldaux = 4 * D;
        d.aux_f32 = f32;
        SB_K(gemm(d, st, err));
      }
      SB_TRY(fork());
      SB_K(gemm(desc(dul, 4 * D, true, h2[l], D, true, 4 * D, D, N, Gp(b0 + 4), D, f32), sst, err, dw_side));
      SB_TRY(mark(ev_fc[l]));
      SB_K(gemm(desc(dul, 4 * D, false, Pp(b0 + 4), D, true, N, D, 4 * D, dh, D, f32), st, err));
      if (l + 1 < L) SB_TRY(wait(ev_proj[l + 1]));  // r1 last read by dW_proj one layer up
      SB_K(layernorm_bwd(dh, f32, xmid[l], f32, mean2[l], rstd2[l], Pp(b0 + 3), f32, r0, r1, Gp(b0 + 3), f32,
                         ws, N, D, st));
      SB_TRY(fork());
      SB_K(gemm(desc(r1, D, true, att[l], D, true, D, D, N, Gp(b0 + 1), D, f32), sst, err, dw_side));
      SB_TRY(mark(ev_proj[l]));
      SB_K(gemm(desc(r1, D, false, Pp(b0 + 1), D, true, N, D, D, dout, D, f32), st, err));
      if (l + 2 < L) SB_TRY(wait(ev_qkv[l + 2]));  // dqkv buffer last read by dW_qkv two layers up
      SB_K(attention_bwd(qkv[l], att[l], dout, lse[l], f32, dql, ws, ash, st));
      SB_TRY(fork());
      SB_K(gemm(desc(dql, 3 * D, true, h1[l], D, true, 3 * D, D, N, Gp(b0 + 0), D, f32), sst, err, dw_side));
      SB_TRY(mark(ev_qkv[l]));
      SB_K(gemm(desc(dql, 3 * D, false, Pp(b0 + 0), D, true, N, D, 3 * D, dh, D, f32), st, err));
      SB_TRY(wait(ev_fc2[l]));  // r0 last read by dW_fc2 of this layer
      SB_K(layernorm_bwd(dh, f32, xs[l], f32, mean1[l], rstd1[l], Pp(b0 + 2), f32, r1, r0, Gp(b0 + 2), f32, ws,
                         N, D, st));
      // layer l's six gradients (plus ln_f after the last layer) are final
      SB_TRY(launch_bucket(offs[b0], l == L - 1 ? offs[ip] : offs[b0 + 6], ev_qkv[l]));
    }
    if (dw_side) {  // join: the main stream waits for every weight gradient
      cudaEvent_t e = xev[nev++];
      SB_CUDA_TRY(cudaEventRecord(e, wst));
      SB_CUDA_TRY(cudaStreamWaitEvent(st, e, 0));
    }
    if (onehot) {
      // the reference's one-hot matmul (reverse.rs:1108-1121) on the tensor
      // cores: dwte = one_hot(x)^T [V, N] x dres (bf16) [N, D], the shape
      // of the head's weight gradient
      SB_K(embedding_onehot(ids, N, V, ldl, onehot, st));
      SB_K(gemm(desc(onehot, ldl, true, r0, D, true, V, D, N, Gp(iw), D, false), st, err));
      SB_K(embedding_pos_bwd(r0, f32, B, T, P, D, Gp(ip), false, st));
    } else {
      SB_K(embedding_bwd(ids, r0, f32, B, T, P, V, D, Gp(iw), Gp(ip), f32, ws, st));
    }
    SB_TRY(launch_bucket(offs[ip], grads_bytes, nullptr));
    if (dp) {
      SB_TRY(comm_allreduce_avg(s, loss_f32, 1, SB_ELEM_F32, s.comm_stream));
      SB_CUDA_TRY(cudaEventRecord(comm_done, s.comm_stream));
      SB_CUDA_TRY(cudaStreamWaitEvent(st, comm_done, 0));
    }
    char* loss_dst = train_step ? state : grads + loss_off;
    if (bf)
      SB_K(convert_f32_to_bf16(loss_f32, reinterpret_cast<__nv_bfloat16*>(loss_dst), 1, st));
    else
      SB_CUDA_TRY(cudaMemcpyAsync(loss_dst, loss_f32, 4, cudaMemcpyDeviceToDevice, st));
    if (train_step) {
      // clip-by-global-norm + adamw-step over the (averaged) gradients
      // (train.shf:29-32), written into the state block
      const int n = static_cast<int>(shapes.size());
      std::vector<int64_t> cnt = leaf_counts();
      std::vector<const void*> gp(n), pp(n), mp(n), vp(n);
      std::vector<void*> po(n), mo(n), vo(n);
      for (int i = 0; i < n; ++i) {
        gp[i] = Gp(i);
        pp[i] = Pp(i);
        mp[i] = mbuf + offs[i];
        vp[i] = vbuf + offs[i];
        po[i] = state + st_p + offs[i];
        mo[i] = state + st_m + offs[i];
        vo[i] = state + st_v + offs[i];
      }
      SB_K(optimizer_step(bf, n, cnt.data(), gp.data(), pp.data(), mp.data(), vp.data(), po.data(), mo.data(),
                          vo.data(), tl, reinterpret_cast<float*>(state + st_t), tl + 1, opt.b1, opt.b2, opt.eps,
                          opt.wd, opt.max_norm, nullptr, opt_ws, opt_ws_bytes, st));
    }
#undef SB_K
    return nullptr;
  }

  sb_status check_leaf(const Buffer* b, size_t i, const char* what) const {
    SB_RETURN_IF(b->elem != g.elem, SB_STATUS_INVALID_ARGUMENT, std::string(what) + " " + std::to_string(i) +
                                                                   ": element type");
    SB_RETURN_IF(b->shape != shapes[i], SB_STATUS_INVALID_ARGUMENT, std::string(what) + " " + std::to_string(i) +
                                                                       ": shape");
    return nullptr;
  }
  sb_status check_ids(const Buffer* b) const {
    SB_RETURN_IF(b->elem != SB_ELEM_F32, SB_STATUS_INVALID_ARGUMENT, "token ids must be f32");
    SB_RETURN_IF(b->shape != std::vector<int64_t>({B, T}), SB_STATUS_INVALID_ARGUMENT,
                 "token ids must be [batch, seq]");
    return nullptr;
  }
  sb_status check_f32_scalar(const Buffer* b, const char* what) const {
    SB_RETURN_IF(b->elem != SB_ELEM_F32 || !b->shape.empty(), SB_STATUS_INVALID_ARGUMENT,
                 std::string(what) + " must be an f32 scalar");
    return nullptr;
  }

  // value_and_grad: leaves..., x, y
  sb_status check_inputs(const std::vector<Buffer*>& in) const {
    const size_t nleaf = shapes.size();
    SB_RETURN_IF(in.size() != nleaf + 2, SB_STATUS_INVALID_ARGUMENT,
                 "value_and_grad expects " + std::to_string(nleaf + 2) + " inputs, got " + std::to_string(in.size()));
    for (size_t i = 0; i < nleaf; ++i) SB_TRY(check_leaf(in[i], i, "leaf"));
    SB_TRY(check_ids(in[nleaf]));
    SB_TRY(check_ids(in[nleaf + 1]));
    return nullptr;
  }

  // train_step: loss, m..., params..., t, v..., x, y, lr
  sb_status check_train_inputs(const std::vector<Buffer*>& in) const {
    const size_t n = shapes.size();
    SB_RETURN_IF(in.size() != 3 * n + 5, SB_STATUS_INVALID_ARGUMENT,
                 "train_step expects " + std::to_string(3 * n + 5) + " inputs, got " + std::to_string(in.size()));
    SB_RETURN_IF(!in[0]->shape.empty(), SB_STATUS_INVALID_ARGUMENT, "state loss must be a scalar");
    for (size_t i = 0; i < n; ++i) {
      SB_TRY(check_leaf(in[1 + i], i, "m leaf"));
      SB_TRY(check_leaf(in[1 + n + i], i, "param leaf"));
      SB_TRY(check_leaf(in[2 + 2 * n + i], i, "v leaf"));
    }
    SB_TRY(check_f32_scalar(in[1 + 2 * n], "t"));
    SB_TRY(check_ids(in[2 + 3 * n]));
    SB_TRY(check_ids(in[3 + 3 * n]));
    SB_TRY(check_f32_scalar(in[4 + 3 * n], "lr"));
    return nullptr;
  }

  // generate: leaves..., ids [batch, block], keys [batch, 4]
  sb_status check_gen_inputs(const std::vector<Buffer*>& in) const {
    const size_t n = shapes.size();
    SB_RETURN_IF(in.size() != n + 2, SB_STATUS_INVALID_ARGUMENT,
                 "generate expects " + std::to_string(n + 2) + " inputs, got " + std::to_string(in.size()));
    for (size_t i = 0; i < n; ++i) SB_TRY(check_leaf(in[i], i, "leaf"));
    SB_TRY(check_ids(in[n]));
    SB_RETURN_IF(in[n + 1]->elem != SB_ELEM_F32 || in[n + 1]->shape != std::vector<int64_t>({B, 4}),
                 SB_STATUS_INVALID_ARGUMENT, "keys must be f32 [batch, 4]");
    return nullptr;
  }

  using Seg = std::pair<const void*, std::pair<void*, size_t>>;

  // Copies every input into its plan-owned slot with batched-copy launches.
  sb_status copy_segs(Session& s, const std::vector<Seg>& segs, cudaStream_t st) {
    for (size_t base = 0; base < segs.size(); base += kMaxSegs) {
      CopySegs c{};
      c.n = static_cast<int>(std::min<size_t>(kMaxSegs, segs.size() - base));
      size_t maxb = 0;
      for (int j = 0; j < c.n; ++j) {
        c.src[j] = static_cast<const char*>(segs[base + j].first);
        c.dst[j] = static_cast<char*>(segs[base + j].second.first);
        c.bytes[j] = segs[base + j].second.second;
        maxb = std::max<size_t>(maxb, c.bytes[j]);
      }
      const int gx = static_cast<int>(std::min<size_t>((maxb / 16 + 255) / 256 + 1, 64));
      batched_copy_kernel<<<dim3(gx, c.n), 256, 0, st>>>(c);
      SB_CUDA_TRY(cudaPeekAtLastError());
      s.kernel_launches++;
    }
    return nullptr;
  }

  sb_status copy_in(Session& s, const std::vector<Buffer*>& in, cudaStream_t st) {
    std::vector<void*> direct(shapes.size());
    bool aligned = true;
    for (size_t i = 0; i < shapes.size(); ++i) {
      direct[i] = in[i]->data();
      aligned = aligned && (reinterpret_cast<uintptr_t>(direct[i]) & 255) == 0;
    }
    SB_TRY(use_params(aligned ? direct : slots(), kVag, st));
    std::vector<Seg> segs;
    if (!aligned)
      for (size_t i = 0; i < shapes.size(); ++i) segs.push_back({in[i]->data(), {slot(static_cast<int>(i)), in[i]->bytes()}});
    segs.push_back({in[shapes.size()]->data(), {ids, static_cast<size_t>(N) * 4}});
    segs.push_back({in[shapes.size() + 1]->data(), {ids + N, static_cast<size_t>(N) * 4}});
    return copy_segs(s, segs, st);
  }

  sb_status copy_in_train(Session& s, const std::vector<Buffer*>& in, cudaStream_t st) {
    const size_t n = shapes.size();
    SB_TRY(use_params(slots(), kTrain, st));
    std::vector<Seg> segs;
    for (size_t i = 0; i < n; ++i) {
      segs.push_back({in[1 + i]->data(), {mbuf + offs[i], in[1 + i]->bytes()}});
      segs.push_back({in[1 + n + i]->data(), {slot(static_cast<int>(i)), in[1 + n + i]->bytes()}});
      segs.push_back({in[2 + 2 * n + i]->data(), {vbuf + offs[i], in[2 + 2 * n + i]->bytes()}});
    }
    segs.push_back({in[1 + 2 * n]->data(), {tl, 4}});
    segs.push_back({in[4 + 3 * n]->data(), {tl + 1, 4}});
    segs.push_back({in[2 + 3 * n]->data(), {ids, static_cast<size_t>(N) * 4}});
    segs.push_back({in[3 + 3 * n]->data(), {ids + N, static_cast<size_t>(N) * 4}});
    return copy_segs(s, segs, st);
  }

  sb_status copy_in_gen(Session& s, const std::vector<Buffer*>& in, cudaStream_t st) {
    const size_t n = shapes.size();
    SB_TRY(use_params(slots(), kSample, st));
    std::vector<Seg> segs;
    for (size_t i = 0; i < n; ++i) segs.push_back({in[i]->data(), {slot(static_cast<int>(i)), in[i]->bytes()}});
    segs.push_back({in[n]->data(), {ids, static_cast<size_t>(N) * 4}});
    segs.push_back({in[n + 1]->data(), {keys_buf, static_cast<size_t>(B) * 16}});
    SB_TRY(copy_segs(s, segs, st));
    SB_CUDA_TRY(cudaMemsetAsync(step_ctr, 0, sizeof(int), st));
    return nullptr;
  }

  // Runs the step: eagerly on the first call of a function, then from the
  // CUDA graph captured on the second.
  sb_status run(Session& s, cudaStream_t st, Mode mode) {
    cudaGraphExec_t& ex = exec[mode];
    uint64_t& nk = kernels[mode];
    const bool dp = group(s) && mode != kSample;
    if (!use_graph || eager[mode] < 1) {
      SB_TRY(enqueue(s, st, mode));
      ++eager[mode];
      return nullptr;
    }
    if (ex && exec_dp[mode] != dp) {  // joined or left a group since the capture
      SB_CUDA_TRY(cudaStreamSynchronize(st));
      cudaGraphExecDestroy(ex);
      ex = nullptr;
    }
    if (!ex) {
      exec_dp[mode] = dp;
      exec_pin[mode] = pin;
      cudaGraph_t graph = nullptr;
      SB_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      sb_status e = enqueue(s, st, mode);
      cudaError_t ce = cudaStreamEndCapture(st, &graph);
      if (e) {
        if (graph) cudaGraphDestroy(graph);
        return e;
      }
      if (ce != cudaSuccess) return make_status(SB_STATUS_INTERNAL, std::string("graph capture: ") + cudaGetErrorString(ce));
      size_t nnodes = 0;
      cudaGraphGetNodes(graph, nullptr, &nnodes);
      std::vector<cudaGraphNode_t> nodes(nnodes);
      cudaGraphGetNodes(graph, nodes.data(), &nnodes);
      nk = 0;
      for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++nk;
      }
      // NCCL's own kernels (one per bucket all-reduce and one for the loss)
      // are not library kernels
      if (dp) nk -= std::min<uint64_t>(nk, static_cast<uint64_t>(L) + 3);
      // honour the streams' priorities captured into the kernel nodes
      ce = cudaGraphInstantiate(&ex, graph, cudaGraphInstantiateFlagUseNodePriority);
      cudaGraphDestroy(graph);
      if (ce != cudaSuccess) return make_status(SB_STATUS_INTERNAL, std::string("graph instantiate: ") + cudaGetErrorString(ce));
      s.graph_captures++;
    }
    SB_CUDA_TRY(cudaGraphLaunch(ex, st));
    s.graph_replays++;
    s.kernel_launches += nk;
    return nullptr;
  }

  sb_status call(Session& s, const std::string& fn, const std::vector<Buffer*>& in,
                 std::vector<Buffer*>& out) override {
    SB_RETURN_IF(!has_function(fn), SB_STATUS_NOT_FOUND, "unknown function " + fn);
    cudaStream_t st = s.stream;
    const int n = static_cast<int>(shapes.size());
    Allocation* a = nullptr;
    if (fn == "generate") {
      // n_new tokens: the graph of one token (window forward + sampling) is
      // replayed, the device step counter moving every replay along
      SB_TRY(check_gen_inputs(in));
      SB_TRY(copy_in_gen(s, in, st));
      for (int i = 0; i < n_new; ++i) SB_TRY(run(s, st, kSample));
      SB_TRY(session_alloc(s, gen_bytes, &a));
      char* o = static_cast<char*>(a->ptr);
      SB_CUDA_TRY(cudaMemcpyAsync(o + gen_tok, tokens_buf, static_cast<size_t>(B) * n_new * 4,
                                  cudaMemcpyDeviceToDevice, st));
      SB_CUDA_TRY(cudaMemcpyAsync(o + gen_ids, ids, static_cast<size_t>(N) * 4, cudaMemcpyDeviceToDevice, st));
      SB_CUDA_TRY(cudaMemcpyAsync(o + gen_keys, keys_buf, static_cast<size_t>(B) * 16, cudaMemcpyDeviceToDevice, st));
      SB_CUDA_TRY(cudaMemcpyAsync(o + gen_logits, step_logits, static_cast<size_t>(n_new) * B * V * 4,
                                  cudaMemcpyDeviceToDevice, st));
      a->refs.store(4);
      out.push_back(buffer_new(s, a, gen_tok, {B, n_new}, SB_ELEM_F32));
      out.push_back(buffer_new(s, a, gen_ids, {B, T}, SB_ELEM_F32));
      out.push_back(buffer_new(s, a, gen_keys, {B, 4}, SB_ELEM_F32));
      out.push_back(buffer_new(s, a, gen_logits, {n_new, B, V}, SB_ELEM_F32));
      return nullptr;
    }
    const bool train_step = fn == "train_step";
    SB_TRY(train_step ? check_train_inputs(in) : check_inputs(in));
    const bool dp = group(s);
    if (dp && bucket_events.empty()) {
      for (int i = 0; i < L + 2; ++i) {
        cudaEvent_t e;
        SB_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        bucket_events.push_back(e);
      }
      SB_CUDA_TRY(cudaEventCreateWithFlags(&comm_done, cudaEventDisableTiming));
    }
    SB_TRY(train_step ? copy_in_train(s, in, st) : copy_in(s, in, st));
    SB_TRY(run(s, st, train_step ? kTrain : kVag));
    if (!train_step) {
      // outputs: one pool allocation holds every gradient and the loss
      SB_TRY(session_alloc(s, out_bytes, &a));
      SB_CUDA_TRY(cudaMemcpyAsync(a->ptr, grads, out_bytes, cudaMemcpyDeviceToDevice, st));
      a->refs.store(n + 1);
      out.push_back(buffer_new(s, a, loss_off, {}, g.elem));
      for (int i = 0; i < n; ++i) out.push_back(buffer_new(s, a, offs[i], shapes[i], g.elem));
      return nullptr;
    }
    // the updated state [loss | m | params | t | v] in one pool allocation
    SB_TRY(session_alloc(s, st_bytes, &a));
    SB_CUDA_TRY(cudaMemcpyAsync(a->ptr, state, st_bytes, cudaMemcpyDeviceToDevice, st));
    a->refs.store(3 * n + 2);
    out.push_back(buffer_new(s, a, 0, {}, g.elem));
    for (int i = 0; i < n; ++i) out.push_back(buffer_new(s, a, st_m + offs[i], shapes[i], g.elem));
    for (int i = 0; i < n; ++i) out.push_back(buffer_new(s, a, st_p + offs[i], shapes[i], g.elem));
    out.push_back(buffer_new(s, a, st_t, {}, SB_ELEM_F32));
    for (int i = 0; i < n; ++i) out.push_back(buffer_new(s, a, st_v + offs[i], shapes[i], g.elem));
    return nullptr;
  }
};

}  // namespace

sb_status make_gpt_vag_module(Session& s, const std::string& name, const GptShape& g, std::unique_ptr<Module>* out,
                              const AdamwConfig* adamw, const SamplerConfig* sampler) {
  auto m = std::make_unique<GptVagModule>();
  sb_status st = m->build(name, g, adamw, sampler);
  if (st) return st;
  *out = std::move(m);
  return nullptr;
}

}  // namespace sb
