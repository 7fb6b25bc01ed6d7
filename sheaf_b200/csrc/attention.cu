// Attention dispatch: bf16 operands with head dim 64 run on the tcgen05 tensor
// cores (attention_tc.cu); fp32 operands (and other head dims) on the CUDA
// cores (attention_simt.cu).
#include <algorithm>

#include "sb_nn.h"

namespace sb {

int attention_fwd_simt(const void* qkv, bool f32, void* o, float* lse, const AttnShape& sh, cudaStream_t s);
int attention_bwd_simt(const void* qkv, const void* o, const void* dout, const float* lse, bool f32, void* dqkv,
                       float* ws, const AttnShape& sh, cudaStream_t s);
bool attention_tc_supported(const AttnShape& sh);
int attention_fwd_tc(const void* qkv, void* o, float* lse, const AttnShape& sh, cudaStream_t s, int* err);
size_t attention_bwd_tc_workspace_bytes(const AttnShape& sh);
int attention_bwd_tc(const void* qkv, const void* o, const void* dout, const float* lse, void* dqkv, float* ws,
                     const AttnShape& sh, cudaStream_t s, int* err);

static bool use_tc(bool f32, const AttnShape& sh) { return !f32 && attention_tc_supported(sh); }

size_t attention_bwd_workspace_bytes(bool f32, const AttnShape& sh) {
  const size_t simt = static_cast<size_t>(sh.B) * sh.H * sh.T * sizeof(float);
  return use_tc(f32, sh) ? std::max(simt, attention_bwd_tc_workspace_bytes(sh)) : simt;
}

int attention_fwd(const void* qkv, bool f32, void* o, float* lse, const AttnShape& sh, cudaStream_t s) {
  if (use_tc(f32, sh)) return attention_fwd_tc(qkv, o, lse, sh, s, device_error_word());
  return attention_fwd_simt(qkv, f32, o, lse, sh, s);
}

int attention_bwd(const void* qkv, const void* o, const void* dout, const float* lse, bool f32, void* dqkv, float* ws,
                  const AttnShape& sh, cudaStream_t s) {
  if (use_tc(f32, sh)) return attention_bwd_tc(qkv, o, dout, lse, dqkv, ws, sh, s, device_error_word());
  return attention_bwd_simt(qkv, o, dout, lse, f32, dqkv, ws, sh, s);
}

}  // namespace sb
