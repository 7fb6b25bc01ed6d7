// Attention dispatch: fp32 operands run on the CUDA cores (attention_simt.cu),
// bf16 operands on the tcgen05 tensor cores (attention_tc.cu).
#include "sb_nn.h"

namespace sb {

int attention_fwd_simt(const void* qkv, bool f32, void* o, float* lse, const AttnShape& sh, cudaStream_t s);
int attention_bwd_simt(const void* qkv, const void* o, const void* dout, const float* lse, bool f32, void* dqkv,
                       float* ws, const AttnShape& sh, cudaStream_t s);

size_t attention_bwd_workspace_bytes(bool /*f32*/, const AttnShape& sh) {
  return static_cast<size_t>(sh.B) * sh.H * sh.T * sizeof(float);
}

int attention_fwd(const void* qkv, bool f32, void* o, float* lse, const AttnShape& sh, cudaStream_t s) {
  return attention_fwd_simt(qkv, f32, o, lse, sh, s);
}

int attention_bwd(const void* qkv, const void* o, const void* dout, const float* lse, bool f32, void* dqkv, float* ws,
                  const AttnShape& sh, cudaStream_t s) {
  return attention_bwd_simt(qkv, o, dout, lse, f32, dqkv, ws, sh, s);
}

}  // namespace sb
