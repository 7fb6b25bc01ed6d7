// Host launch interface of the non-GEMM kernels (internal to the library).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>

#include "sb_kernels.h"

namespace sb {

// Vocabularies up to this size use the deterministic per-row embedding VJP;
// larger ones accumulate with fp32 atomics.
constexpr int kEmbedSmallVocab = 4096;

int num_sms_cached();
int* device_error_word();

// y = (x - mean) / sqrt(var + 1e-5) * gamma over the last dim (rows x D).
// x is the residual stream, f32 (x_f32) or bf16; a bf16 x takes a bf16 y.
// x_copy (optional, x's type, [rows, D]) receives a copy of x: the base that
// a following residual GEMM accumulates into (EPI_ACCUM).
int layernorm_fwd(const void* x, bool x_f32, const void* gamma, bool gamma_f32, void* y, bool y_f32, float* mean,
                  float* rstd, int rows, int D, cudaStream_t s, void* x_copy = nullptr);
// dres_out = dres_in + LN-VJP(dy) (dres_in null: zero; it may alias
// dres_out); dgamma = sum_rows dy * xhat. x and the residual gradients are
// f32 (x_f32) or bf16; a bf16 x takes a bf16 dy.
size_t layernorm_bwd_workspace_bytes(int rows, int D);
int layernorm_bwd(const void* dy, bool dy_f32, const void* x, bool x_f32, const float* mean, const float* rstd,
                  const void* gamma, bool gamma_f32, const void* dres_in, void* dres_out, void* dgamma,
                  bool dgamma_f32, float* ws, int rows, int D, cudaStream_t s);

// layernorm_bwd (f32 dy) with at most `max_blocks` blocks; `scratch` holds
// max_blocks * D floats of dgamma partials.
int layernorm_bwd_capped(const float* dy, const float* x, const float* mean, const float* rstd, const void* gamma,
                         bool gamma_f32, float* dres, void* dgamma, bool dgamma_f32, float* scratch, int max_blocks,
                         int rows, int D, cudaStream_t s);

// loss = -mean(log_softmax(logits)[target]); dlogits = (softmax - onehot) / rows.
size_t cross_entropy_workspace_bytes(int rows);
int cross_entropy_fwd_bwd(const void* logits, bool f32, long ld, int rows, int V, const float* targets, void* dlogits,
                          long ldd, float* ws, float* loss_f32, __nv_bfloat16* loss_bf16, cudaStream_t s);

// x[b*T+t] = wte[clamp(ids)] + wpe[t]: tables f32 (f32) or bf16; x f32
// (x_f32) or, from bf16 tables, the bf16-rounded sum.
int embedding_fwd(const float* ids, const void* wte, const void* wpe, bool f32, void* x, bool x_f32, int ntok, int T,
                  int V, int D, cudaStream_t s);
// dwte = scatter-add of dx rows by id; dwpe[t] = sum_b dx[b,t] (rows >= T zero).
size_t embedding_bwd_workspace_bytes(int V, int D);
int embedding_bwd(const float* ids, const void* dx, bool dx_f32, int B, int T, int P, int V, int D, void* dwte, void* dwpe,
                  bool out_f32, float* ws, cudaStream_t s);

// The embedding VJP in two parts, for a plan that computes dwte itself as
// one_hot(ids)^T dx on the tensor cores: the bf16 one-hot [ntok, Vp] (columns
// >= V zero; an id that is not exactly an integer in [0, V) has no class)
// and dwpe alone.
int embedding_onehot(const float* ids, int ntok, int V, int Vp, __nv_bfloat16* out, cudaStream_t s);
int embedding_pos_bwd(const void* dx, bool dx_f32, int B, int T, int P, int D, void* dwpe, bool out_f32,
                      cudaStream_t s);

int convert_f32_to_bf16(const float* in, __nv_bfloat16* out, long n, cudaStream_t s);
// y = gelu(x) or, with bwd, y = g * gelu'(x), elementwise over n values.
int gelu(const void* x, const void* g, void* y, bool f32, bool bwd, long n, cudaStream_t s);

// Causal attention over packed qkv [B*T, 3*D] (q | k | v, heads of Hd=D/H
// columns), o [B*T, D], lse [B*H*T] (natural-log units of the scaled scores).
struct AttnShape {
  int B, T, H, Hd;
};
int attention_fwd(const void* qkv, bool f32, void* o, float* lse, const AttnShape& sh, cudaStream_t s);
// dqkv [B*T, 3*D] from dO, O, qkv, lse. `ws` holds B*H*T floats (row dots)
// plus, for the tensor-core path, a f32 dQ accumulator.
size_t attention_bwd_workspace_bytes(bool f32, const AttnShape& sh);
int attention_bwd(const void* qkv, const void* o, const void* dout, const float* lse, bool f32, void* dqkv, float* ws,
                  const AttnShape& sh, cudaStream_t s);

// get-batch of examples/nanogpt/train.shf:15-21 on the device: batch rows
// of `block` token ids (f32) from `data` (n ids) at starts drawn with
// random-randint from `key` (four f32 limbs); y is x shifted by one. The
// start bound n - block - 1 must be positive and at most 2^24 (exact in f32).
int get_batch(const float* data, long n, const float* key, int block, int batch, float* x, float* y, cudaStream_t s);
// random-split `key` into n children, written as [n, 4] limbs.
int random_split(const float* key, int n, float* out, cudaStream_t s);

// One token of nanoGPT's generate-token for B sequences (window T, vocab V
// at most kSampleMaxVocab): samples from the last position's logits
// (row b*T + T-1, row stride ld), writes tokens[b * n_new + *step], advances
// each sequence's key [B, 4] and its id window [B, T] in place, records the
// raw last-position logits in step_logits [n_new, B, V] (optional) and
// increments *step. Vocabularies up to kSampleSmemVocab sort in one CTA's
// shared memory and need no workspace; larger ones (window T <= 4096) take
// sample_workspace_bytes(B, V) of scratch.
constexpr int kSampleSmemVocab = 4096;
constexpr int kSampleMaxVocab = 1 << 24;
size_t sample_workspace_bytes(int B, int V);
int sample_step(const void* logits, bool logits_f32, long ld, int B, int T, int V, int top_k, float temperature,
                float* ids, float* keys, float* tokens, int n_new, int* step, float* step_logits, void* ws,
                size_t ws_bytes, cudaStream_t s);

// Global gradient norm, and with `params` the clip-by-global-norm + AdamW
// step of nanoGPT's train-step over n_leaves tensors of one element type
// (pointer arrays on the host, tensors on the device). t_in, lr: device f32
// scalars; t_out <- t_in + 1. Outputs may alias inputs. max_norm <= 0: no
// clipping. norm_out (optional): the global norm of the unclipped gradients.
size_t optimizer_workspace_bytes(const int64_t* counts, int n_leaves);
int optimizer_step(bool bf16, int n_leaves, const int64_t* counts, const void* const* grads,
                   const void* const* params, const void* const* m, const void* const* v, void* const* params_out,
                   void* const* m_out, void* const* v_out, const float* t_in, float* t_out, const float* lr,
                   float b1, float b2, float eps, float wd, float max_norm, float* norm_out, void* workspace,
                   size_t workspace_bytes, cudaStream_t s);

}  // namespace sb
