// Generic StableHLO op kernels (hlo_kernels.cu) used by the module executor.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace sb {
namespace hlo {

enum Dt : int { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2, DT_I32 = 3, DT_I1 = 4 };

enum Unary : int {
  U_COPY = 0, U_NEG, U_ABS, U_EXP, U_LOG, U_SQRT, U_RSQRT, U_TANH, U_SIN, U_COS, U_FLOOR, U_CEIL, U_SIGN,
  U_LOGISTIC, U_NOT, U_LOG1P, U_EXPM1,
};

enum Binary : int {
  B_ADD = 0, B_SUB, B_MUL, B_DIV, B_POW, B_MAX, B_MIN, B_REM, B_FLOORDIV, B_ATAN2, B_AND, B_OR, B_XOR, B_SHL, B_SHR,
};

enum Cmp : int { C_EQ = 0, C_NE, C_LT, C_LE, C_GT, C_GE };

constexpr int kMaxRank = 8;

struct IndexMap {
  int rank = 0;
  long out_shape[kMaxRank] = {};
  long stride[kMaxRank] = {};  // source-element stride per output axis
  long offset[kMaxRank] = {};  // subtracted from the output coordinate first
  long extent[kMaxRank] = {};  // valid range of (coordinate - offset) when check
  long base = 0;
  bool check = false;
  const void* pad_value = nullptr;  // device pointer to one element
};

// dynamic_slice / dynamic_update_slice: start indices are device i32
// scalars, clamped on the device to [0, shape_d - size_d] as StableHLO
// specifies; `shape` is the operand (slice) or result (update) shape and
// `size` the slice sizes or the update's shape.
struct DynSlice {
  int rank = 0;
  long shape[kMaxRank] = {};
  long size[kMaxRank] = {};
  const int32_t* start[kMaxRank] = {};
};

// Longest row the sort kernel handles (one CTA sorts a row in shared memory).
// Rows up to kSortSmemRow sort in one CTA's shared memory; longer rows (up to
// kSortMaxRow) take a chunked merge sort with sort_rows_workspace_bytes of scratch.
constexpr int kSortSmemRow = 16384;
constexpr int kSortMaxRow = 1 << 24;

int dt_size(int dt);
int unary(const void* a, void* out, long n, int op, int dta, int dto, cudaStream_t s);
int binary(const void* a, const void* b, void* out, long n, int op, int dt, cudaStream_t s);
int clamp(const void* lo, long nlo, const void* x, const void* hi, long nhi, void* out, long n, int dt, cudaStream_t s);
int compare(const void* a, const void* b, void* out, long n, int dir, int dt, cudaStream_t s);
int select(const void* p, long np, const void* a, const void* b, void* out, long n, int dt, cudaStream_t s);
int convert(const void* a, int dta, void* out, int dto, long n, cudaStream_t s);
int remap(const void* in, void* out, long n, int dt, const IndexMap& m, cudaStream_t s);
int iota(void* out, long n, int dt, long inner, long dim_extent, cudaStream_t s);
int reduce(const void* in, void* out, long outer, long red, long inner, int op, float init, const void* init_ptr,
           int dt, cudaStream_t s);
int bgemm(const void* A, const void* B, void* C, int batch, int M, int N, int K, int dta, int dtb, int dtc,
          cudaStream_t s);
int gather_rows(const void* operand, const void* idx, void* out, long rows, long V, long width, int dt, cudaStream_t s);
int dynamic_slice(const void* in, void* out, int dt, const DynSlice& d, cudaStream_t s);
// Writes `upd` into `out` (already holding the operand) at the clamped starts.
int dynamic_update(void* out, const void* upd, int dt, const DynSlice& d, cudaStream_t s);
// Stable sort of `rows` rows of n keys (f32 or bf16) along the last axis,
// carrying an i32 payload: descending for a GT comparator, ascending for LT;
// equal keys keep their input order.
// Stable sort of each of `rows` rows of n keys (descending or ascending),
// the payload permuted alike (payload null: out_payload receives the source
// positions). Rows longer than kSortSmemRow need sort_rows_workspace_bytes
// of scratch in `ws`.
size_t sort_rows_workspace_bytes(long rows, int n);
int sort_rows(const void* keys, int key_dt, const int32_t* payload, void* out_keys, int32_t* out_payload, long rows,
              int n, bool descending, void* ws, size_t ws_bytes, cudaStream_t s);

}  // namespace hlo
}  // namespace sb
