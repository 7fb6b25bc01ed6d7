// Host-side launch interface of the kernel library (internal to the shared
// library; the exported C ABI lives in include/sheaf_b200*.h).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace sb {

// Epilogue applied to each accumulator tile of a GEMM.
enum EpiKind : int {
  EPI_STORE = 0,     // out = acc
  EPI_ADD = 1,       // out = acc + aux            (aux may alias out; f32 only)
  EPI_GELU = 2,      // u = acc; out = gelu(u); out2 = gelu'(u)  (out2 feeds EPI_MUL in the VJP)
  EPI_MUL = 3,       // out = acc * aux            (aux = gelu'(u) saved by EPI_GELU)
  EPI_ACCUM = 4,     // out += acc                 (f32 or bf16 out; no split-K)
};

// C[M,N] = A[M,K] * B[N,K]^T with either operand stored K-major (rows of K)
// or MN-major (stored transposed: [K, M] / [K, N] row-major).
struct GemmDesc {
  const void* A = nullptr;
  long lda = 0;       // row stride (elements) of A as stored
  bool a_mn = false;  // A stored as [K, M]
  const void* B = nullptr;
  long ldb = 0;
  bool b_mn = false;  // B stored as [K, N]
  int M = 0, N = 0, K = 0;
  int epi = EPI_STORE;
  void* out = nullptr;
  long ldo = 0;
  bool out_f32 = false;
  const void* aux = nullptr;
  long ldaux = 0;
  bool aux_f32 = false;
  void* out2 = nullptr;
  long ldo2 = 0;
  int splits = 0;  // 0 = choose; 1 = no split-K (split-K only with EPI_STORE)
  int bn = 0;      // 0 = choose tile width (64, 128, 192, 256; 384 runs on CTA pairs)
  int pair = -1;   // 256-row tiles on CTA pairs: -1 = when the tile allows, 0 = never
  int max_splits = 0;  // cap on the chosen split-K factor (0 = none)
  int max_ctas = 0;    // cap on the CTAs the chosen split-K factor occupies (0 = none)
  int max_pair_splits = 0;  // cap on the chosen split-K factor of CTA-pair tiles (0 = none)
};

// bf16 operands on tcgen05 tensor cores (fp32 accumulation in TMEM).
// `workspace` (fp32) is used for split-K partial sums; returns 0 on success.
int gemm_bf16(const GemmDesc& d, float* workspace, size_t workspace_bytes, cudaStream_t s, int* err);
// fp32 operands: on the tensor cores by the bf16x6 split (one bf16 GEMM over
// K' = 6K with f32 accumulation, gemm_emul.cu) when the problem is large and
// the workspace holds the split copies, else on the CUDA cores (FFMA).
int gemm_f32(const GemmDesc& d, float* workspace, size_t workspace_bytes, cudaStream_t s, int* err);
bool gemm_f32_use_emulation(const GemmDesc& d);
size_t gemm_f32_emulated_workspace_bytes(const GemmDesc& d);
int gemm_f32_emulated(const GemmDesc& d, void* workspace, size_t workspace_bytes, cudaStream_t s, int* err);
// Bytes of split-K workspace gemm_* would use for this problem (0 if none).
size_t gemm_workspace_bytes(const GemmDesc& d, bool bf16);
size_t gemm_f32_workspace_bytes(const GemmDesc& d);

int num_sms();

// 2-D bf16 TMA descriptor over a row-major [rows, cols] matrix (row stride
// `ld` elements), box {box_cols, box_rows}, 128-byte swizzle, zero fill.
// `map` points at a CUtensorMap (64-byte aligned storage).
bool make_tma_2d_bf16(void* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows);
bool make_tma_2d_f32(void* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows);
bool make_tma_3d_bf16(void* map, const void* base, long d0, long d1, long d2, long ld1, long ld2, int box0,
                      int box1);

}  // namespace sb
