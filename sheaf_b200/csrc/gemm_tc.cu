// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the `stablehlo.dot_general` dispatches that Sheaf's `@` lowers to
// (lowering/stablehlo/dot_ops.rs:12-229) and the two GEMMs of its VJP
// (autodiff/reverse.rs:585-689: dA = adj @ swapaxes(B), dB = swapaxes(A) @ adj,
// followed by the batch reduction of maybe_unbroadcast, reverse.rs:360-376).
// The weight gradient is contracted over all B*T tokens in one GEMM (split-K
// across CTAs) instead of B per-batch partial products plus a reduce.
//
// Kernel structure (one CTA per SM, persistent over output tiles):
//   warp 0     : TMA producer (one lane), STAGES-deep smem ring
//   warp 1     : TMEM allocator + single-thread UMMA issuer (M=128, N=BN, K=16)
//   warps 2..3 : idle (keep the epilogue warpgroups aligned)
//   warps 4..11: two epilogue warpgroups; group g drains TMEM accumulator
//                buffer g. Warp w owns TMEM lanes 32*(w%4)..+31 (32 output
//                rows). Each 32-row x 128-byte block of the tile is converted
//                in registers (fused epilogue), written to the warp's
//                128B-swizzled 4 KB staging slot and stored with a TMA bulk
//                tensor store.
// Accumulators are double-buffered in TMEM (2*BN columns): the MMA warp fills
// one buffer while the other group's epilogue drains the other, and the two
// groups' epilogues (global aux loads, math, stores) overlap each other.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "sb_kernels.h"
#define SB_PDL_FAMILY 0
#include "sb_launch.cuh"
#include "sb_ptx.cuh"

namespace sb {

int pdl_mask() {
  static const int mask = [] {
    const char* e = std::getenv("SHEAF_B200_PDL");
    return e ? std::atoi(e) : 0x5;
  }();
  return mask;
}


namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr uint32_t kABytes = kBM * kBK * 2;
constexpr uint32_t kSlotBytes = 32 * 128;  // one 32-row x 128-byte staging block

// Staging slots per epilogue warp: two (conversion overlaps the previous
// store) except for the single-CTA 256-wide tile, whose 4-stage operand ring
// leaves room for one.
__host__ __device__ constexpr int staging_slots(int bn, bool pair) { return (bn >= 256 && !pair) ? 1 : 2; }
__host__ __device__ constexpr uint32_t staging_bytes(int bn, bool pair) {
  return 8u * staging_slots(bn, pair) * kSlotBytes;
}

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles;
  int splits, kb_per_split, kb_total;
  int epi;
  int out_f32;     // output element type (split-K partials are f32)
  int partial;     // split-K: rows of split s start at s * m_tiles * 128
  const void* aux;
  long ldaux;
  int* err;
};

// Hardware tanh (PTX tanh.approx.f32, one MUFU op; relative error about
// 2^-11, below the 2^-9 rounding of the bf16 results it feeds).
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// gelu(x) = 0.5 * (x * (1 + tanh(0.7978846 * (x + 0.044715 * (x * (x * x))))))
// (lib/nn.shf:10-11) and its derivative by the chain rule of those primitive
// ops, from one tanh: the forward epilogue saves gelu'(u) for the VJP. Two
// elements at a time with packed f32x2 arithmetic (sm_100: one instruction
// per pair for each multiply / fma, the same IEEE single-precision operations
// and roundings as the scalar expressions), which halves the epilogue's
// floating-point instruction count.
__device__ __forceinline__ void gelu_and_grad2(float2 x, float2& g, float2& d) {
  const float2 x2 = __fmul2_rn(x, x);
  const float2 s = __ffma2_rn(make_float2(0.044715f, 0.044715f), __fmul2_rn(x, x2), x);
  const float2 arg = __fmul2_rn(make_float2(0.7978846f, 0.7978846f), s);
  const float2 t = make_float2(tanh_approx(arg.x), tanh_approx(arg.y));
  const float2 hx = __fmul2_rn(make_float2(0.5f, 0.5f), x);
  g = __ffma2_rn(hx, t, hx);  // 0.5 x (1 + t)
  // gelu'(x) = 0.5 (1 + t) + 0.5 x (1 - t^2) 0.7978846 (1 + 3 * 0.044715 x^2)
  const float2 a0 = __ffma2_rn(make_float2(0.5f, 0.5f), t, make_float2(0.5f, 0.5f));
  const float2 omt = __ffma2_rn(make_float2(-t.x, -t.y), t, make_float2(1.0f, 1.0f));
  const float2 poly =
      __ffma2_rn(make_float2(0.7978846f * 0.134145f, 0.7978846f * 0.134145f), x2, make_float2(0.7978846f, 0.7978846f));
  d = __ffma2_rn(__fmul2_rn(hx, omt), poly, a0);
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  return (2 * bn <= 32) ? 32 : (2 * bn <= 64) ? 64 : (2 * bn <= 128) ? 128 : (2 * bn <= 256) ? 256 : 512;
}

// Shared memory per CTA: STAGES x (A tile + this CTA's B rows), staging,
// barriers. A CTA of a pair (PAIR) holds half of the B tile's BN rows.
template <int BN, int STAGES, bool PAIR>
constexpr size_t smem_bytes_for() {
  return 1024 /*alignment slack*/ + static_cast<size_t>(STAGES) * (kABytes + (PAIR ? BN / 2 : BN) * kBK * 2) +
         staging_bytes(BN, PAIR) + (2 * STAGES + 4) * sizeof(uint64_t) + 16;
}

// PAIR: launched as clusters of two CTAs on two SMs that compute a 256 x BN
// tile with tcgen05.mma.cta_group::2 (M = 256). CTA rank r loads A rows
// 256*mt + 128r .. +127 and B rows BN*nt + (BN/2)r .. +BN/2-1 into its own
// shared memory, the loads of both completing on rank 0's `full` barrier;
// rank 0 issues the MMAs, whose completion is signalled to the `empty` and
// `tfull` barriers of both CTAs; each CTA's epilogue drains the 128
// accumulator rows in its own TMEM and arrives on rank 0's `tempty`. Halving
// the B bytes per SM leaves room for deeper operand pipelines.
//
// BN = 384 (pairs only) covers N = 384 in one tile with two UMMAs per K step,
// N = 256 into accumulator columns 0..255 and N = 128 into 256..383; each CTA
// holds B rows 128r .. +127 and 256 + 64r .. +63 of the tile. One 384-column
// accumulator fills the TMEM, so there is a single accumulator buffer. Per
// byte of operands loaded it does twice the MMA work of 192-wide tiles.
template <int BN, bool A_MN, bool B_MN, int STAGES, bool PAIR>
__global__ void __launch_bounds__(384, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2, GemmArgs a) {
  constexpr int BH = PAIR ? BN / 2 : BN;  // B rows (N) loaded by this CTA
  constexpr uint32_t kBBytes = BH * kBK * 2;
  constexpr uint32_t kTmemCols = tmem_cols_for(BN);
  constexpr int kRowsPerTile = PAIR ? 2 * kBM : kBM;
  constexpr bool kWide = PAIR && BN == 384;
  constexpr int kAcc = kWide ? 1 : 2;  // accumulator buffers in TMEM
  static_assert(BN % 64 == 0 && BN >= 64 && (BN <= 256 || kWide), "tile width must be 64, 128, 192, 256 (or 384 on pairs)");
  static_assert(!PAIR || (BH % 64 == 0), "pair tiles split B into 64-row halves");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  uint8_t* sStg = sB + STAGES * kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + staging_bytes(BN, PAIR));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int cta0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);  // work-unit stride base
  const int ncta = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], PAIR ? 16 : 8);  // every epilogue warp (of both CTAs)
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    tma_prefetch_desc(&tmC2);
  }
  // operands come from the preceding kernel and the outputs may be its
  // operands: no global access, and no TMEM allocation, before this
  pdl_wait();
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  else
    __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles = a.m_tiles * a.n_tiles;
  const int units = tiles * a.splits;

  if (warp == 0) {
    if (lane == 0) {
      // with PAIR, both CTAs' loads complete on rank 0's full[s], which rank
      // 0 arms with the bytes of both halves
      const uint32_t full0 = PAIR ? mapa_shared(smem_u32(full), 0) : smem_u32(full);
      uint32_t it = 0;
      for (int u = cta0; u < units; u += ncta) {
        const int split = u % a.splits;
        const int tile = u / a.splits;
        const int mt = tile % a.m_tiles, nt = tile / a.m_tiles;
        const int arow = mt * kRowsPerTile + static_cast<int>(rank) * kBM;
        const int brow = nt * BN + static_cast<int>(rank) * BH;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.kb_total, kb0 + a.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, a.err, abort_flag)) goto done;
          uint8_t* da = sA + s * kABytes;
          uint8_t* db = sB + s * kBBytes;
          if constexpr (PAIR) {
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (kABytes + kBBytes));
            const uint32_t fb = full0 + s * 8;
            if (!A_MN) {
              tma_load_2d_pair(da, &tmA, fb, kb * kBK, arow);
            } else {
              tma_load_2d_pair(da, &tmA, fb, arow, kb * kBK);
              tma_load_2d_pair(da + 8192, &tmA, fb, arow + 64, kb * kBK);
            }
            if constexpr (kWide) {
              // three 64-row (K-major) or 64-column (MN-major) boxes: rows
              // 128r, 128r + 64 (N = 256 UMMA) and 256 + 64r (N = 128 UMMA)
#pragma unroll
              for (int j = 0; j < 3; ++j) {
                const int pos = nt * BN + (j < 2 ? static_cast<int>(rank) * 128 + j * 64 : 256 + static_cast<int>(rank) * 64);
                if (!B_MN)
                  tma_load_2d_pair(db + j * 8192, &tmB, fb, kb * kBK, pos);
                else
                  tma_load_2d_pair(db + j * 8192, &tmB, fb, pos, kb * kBK);
              }
            } else if (!B_MN) {
              tma_load_2d_pair(db, &tmB, fb, kb * kBK, brow);
            } else {
#pragma unroll
              for (int j = 0; j < BH / 64; ++j) tma_load_2d_pair(db + j * 8192, &tmB, fb, brow + j * 64, kb * kBK);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
            if (!A_MN) {
              tma_load_2d(da, &tmA, &full[s], kb * kBK, arow);
            } else {
              tma_load_2d(da, &tmA, &full[s], arow, kb * kBK);
              tma_load_2d(da + 8192, &tmA, &full[s], arow + 64, kb * kBK);
            }
            if (!B_MN) {
              tma_load_2d(db, &tmB, &full[s], kb * kBK, brow);
            } else {
#pragma unroll
              for (int j = 0; j < BH / 64; ++j) tma_load_2d(db + j * 8192, &tmB, &full[s], brow + j * 64, kb * kBK);
            }
          }
        }
      }
      // wait for the final release of every stage, so that no UMMA commit
      // can still arrive on this CTA's barriers after it exits
      for (int i = 0; i < STAGES; ++i, ++it)
        if (!mbar_wait(&empty[it % STAGES], ((it / STAGES) & 1) ^ 1, a.err, abort_flag)) break;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kRowsPerTile, kWide ? 256 : BN, A_MN, B_MN);
      constexpr uint32_t idesc_hi = make_idesc_bf16(kRowsPerTile, 128, A_MN, B_MN);  // wide tiles' N = 128 part
      uint32_t it = 0;
      int local = 0;
      for (int u = cta0; u < units; u += ncta, ++local) {
        const int split = u % a.splits;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.kb_total, kb0 + a.kb_per_split);
        const int as = local % kAcc;
        const uint32_t aph = (local / kAcc) & 1;
        if (!mbar_wait(&tempty[as], aph ^ 1, a.err, abort_flag)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + as * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, a.err, abort_flag)) goto done;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * kABytes);
          const uint32_t b_addr = smem_u32(sB + s * kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            if constexpr (kWide) {
              const uint64_t bd_hi = B_MN ? make_sw128_desc(b_addr + 16384 + kk * 2048, 8192, 1024)
                                          : make_sw128_desc(b_addr + 16384 + kk * 32, 16, 1024);
              umma_f16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
              umma_f16_pair(d_tmem + 256, ad, bd_hi, idesc_hi, (kb > kb0 || kk > 0) ? 1u : 0u);
            } else if constexpr (PAIR) {
              umma_f16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            } else {
              umma_f16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            }
          }
          if constexpr (PAIR)
            umma_commit_pair(&empty[s]);
          else
            umma_commit(&empty[s]);
        }
        if constexpr (PAIR)
          umma_commit_pair(&tfull[as]);
        else
          umma_commit(&tfull[as]);
      }
      if constexpr (PAIR) {
        // the peer's epilogue arrives remotely on tempty: wait for the
        // releases of the last accumulator buffers before leaving
        for (int i = 0; i < kAcc; ++i, ++local)
          if (!mbar_wait(&tempty[local % kAcc], ((local / kAcc) & 1) ^ 1, a.err, abort_flag)) break;
      }
    }
  } else if (warp >= 4) {
    // Two epilogue warpgroups drain every tile together, group eg taking one
    // half of the tile's column blocks, so a tile's drain (the last one's is
    // not hidden behind a main loop) takes half as long; warp w reads TMEM
    // lanes 32*(w%4) .. +31.
    const int q = warp & 3;
    const int eg = (warp >> 2) - 1;
    constexpr int kBlocksBf16 = BN / 64, kBlocksF32 = BN / 32;  // 128-byte column blocks per tile row
    const int cb16 = eg ? (kBlocksBf16 + 1) / 2 : 0, ce16 = eg ? kBlocksBf16 : (kBlocksBf16 + 1) / 2;
    const int cb32 = eg ? kBlocksF32 / 2 : 0, ce32 = eg ? kBlocksF32 : kBlocksF32 / 2;
    constexpr int kSlots = staging_slots(BN, PAIR);
    const uint32_t stg = smem_u32(sStg) + (warp - 4) * kSlots * kSlotBytes;
    uint32_t cc = 0;  // bulk stores issued by this warp (lane 0 commits them)
    // Writes the warp's 32-row x 128-byte block into a swizzled staging slot
    // and stores it with a bulk tensor store, or, with `accumulate`, adds it
    // into global memory with a bulk tensor reduce-add (the add runs in L2).
    // L2 policy for outputs nothing reads soon (gelu'(u), read by the VJP
    // only): evict first, so they do not push the next kernel's operands out
    uint64_t evict_first_policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(evict_first_policy));
    // the next staging slot, once the bulk store that last used it has read it
    auto acquire_slot = [&]() {
      const uint32_t slot = stg + (cc % kSlots) * kSlotBytes;
      if (cc >= static_cast<uint32_t>(kSlots)) {
        if (lane == 0) bulk_wait_read<kSlots - 1>();
        __syncwarp();
      }
      return slot;
    };
    auto stage = [&](const uint32_t(&w)[32], const CUtensorMap* map, int x, int y, bool accumulate,
                     bool evict_first = false, uint32_t held_slot = 0) {
      const uint32_t slot = held_slot ? held_slot : acquire_slot();
      st_row128_sw(slot, lane, w);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (accumulate)
          asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::
                           "l"(reinterpret_cast<uint64_t>(map)),
                       "r"(slot), "r"(x), "r"(y)
                       : "memory");
        else if (evict_first)
          asm volatile(
              "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                  reinterpret_cast<uint64_t>(map)),
              "r"(slot), "r"(x), "r"(y), "l"(evict_first_policy)
              : "memory");
        else
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                           reinterpret_cast<uint64_t>(map)),
                       "r"(slot), "r"(x), "r"(y)
                       : "memory");
        bulk_commit();
      }
      ++cc;
    };
    int local = 0;
    const uint32_t tempty0 = PAIR ? mapa_shared(smem_u32(tempty), 0) : smem_u32(tempty);
    for (int u = cta0; u < units; u += ncta, ++local) {
      const int split = u % a.splits;
      const int tile = u / a.splits;
      const int mt = tile % a.m_tiles, nt = tile / a.m_tiles;
      const int as = local % kAcc;
      const uint32_t aph = (local / kAcc) & 1;
      const int row0 = mt * kRowsPerTile + static_cast<int>(rank) * kBM + q * 32;
      const int row = row0 + lane;
      if ((a.epi == EPI_ADD || a.epi == EPI_MUL) && row < a.M) {
        // pull this row's aux segment of the tile towards L2 while the
        // accumulator is still being computed
        const int esz = a.epi == EPI_ADD ? 4 : 2;
        const int c0 = nt * BN + (a.epi == EPI_ADD ? cb32 * 32 : cb16 * 64);
        const int c1 = min(a.N, nt * BN + (a.epi == EPI_ADD ? ce32 * 32 : ce16 * 64));
        const char* ap = static_cast<const char*>(a.aux) + static_cast<long>(row) * a.ldaux * esz;
        for (int off = c0 * esz; off < c1 * esz; off += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(ap + off));
      }
      if (!mbar_wait(&tfull[as], aph, a.err, abort_flag)) break;
      tc_fence_after();
      const int store_y = a.partial ? split * a.m_tiles * kRowsPerTile + row0 : row0;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + as * BN;
      if (a.out_f32) {
        // 32 f32 columns (128 B) per block: STORE, ADD, or ACCUM (reduce-add
        // into the residual stream)
#pragma unroll 1
        for (int c = cb32; c < ce32; ++c) {
          const int col0 = nt * BN + c * 32;
          if (col0 >= a.N) break;
          uint32_t v[32];
          tmem_ld32(t_row + c * 32, v);
          tmem_wait_ld();
          if (a.epi == EPI_ADD && row < a.M) {
            const float* x = static_cast<const float*>(a.aux) + static_cast<long>(row) * a.ldaux + col0;
            if (col0 + 32 <= a.N) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 r = *reinterpret_cast<const float4*>(x + j);
                v[j] = __float_as_uint(__uint_as_float(v[j]) + r.x);
                v[j + 1] = __float_as_uint(__uint_as_float(v[j + 1]) + r.y);
                v[j + 2] = __float_as_uint(__uint_as_float(v[j + 2]) + r.z);
                v[j + 3] = __float_as_uint(__uint_as_float(v[j + 3]) + r.w);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < a.N) v[j] = __float_as_uint(__uint_as_float(v[j]) + x[j]);
            }
          }
          stage(v, &tmC, col0, store_y, a.epi == EPI_ACCUM);
        }
      } else {
        // 64 bf16 columns (128 B) per block: STORE, ACCUM (bf16 reduce-add
        // into the residual stream: x + bf16(acc) rounded to bf16, as the
        // module's bf16 add), GELU (two outputs), MUL
#pragma unroll 1
        for (int c = cb16; c < ce16; ++c) {
          const int col0 = nt * BN + c * 64;
          if (col0 >= a.N) break;
          uint32_t v0[32], v1[32];
          tmem_ld32(t_row + c * 64, v0);
          tmem_ld32(t_row + c * 64 + 32, v1);
          tmem_wait_ld();
          uint32_t w[32];
          if (a.epi == EPI_STORE || a.epi == EPI_ACCUM) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              w[j] = pack_bf16x2(__uint_as_float(v0[2 * j]), __uint_as_float(v0[2 * j + 1]));
              w[16 + j] = pack_bf16x2(__uint_as_float(v1[2 * j]), __uint_as_float(v1[2 * j + 1]));
            }
            stage(w, &tmC, col0, store_y, a.epi == EPI_ACCUM);
          } else if (a.epi == EPI_GELU) {
            // u is the bf16-rounded product, as the module's dot_general
            // result (rounded in pairs: the paired conversion keeps the
            // special-function pipe free for the tanh)
            uint32_t g[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float2 ya, yb, da, db;
              const uint32_t r0 = pack_bf16x2(__uint_as_float(v0[2 * j]), __uint_as_float(v0[2 * j + 1]));
              const uint32_t r1 = pack_bf16x2(__uint_as_float(v1[2 * j]), __uint_as_float(v1[2 * j + 1]));
              gelu_and_grad2(make_float2(__uint_as_float(r0 << 16), __uint_as_float(r0 & 0xFFFF0000u)), ya, da);
              gelu_and_grad2(make_float2(__uint_as_float(r1 << 16), __uint_as_float(r1 & 0xFFFF0000u)), yb, db);
              w[j] = pack_bf16x2(ya.x, ya.y);
              w[16 + j] = pack_bf16x2(yb.x, yb.y);
              g[j] = pack_bf16x2(da.x, da.y);
              g[16 + j] = pack_bf16x2(db.x, db.y);
            }
            if constexpr (kSlots >= 2) {
              // both outputs of the block in one go: the two slots written,
              // one proxy fence and one warp sync, both stores in one bulk
              // group (every block of this launch does the same, so a group
              // always covers both slots: wait for all earlier reads)
              const uint32_t s0 = stg, s1 = stg + kSlotBytes;
              if (cc > 0) {
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
              }
              st_row128_sw(s0, lane, w);
              st_row128_sw(s1, lane, g);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                                 reinterpret_cast<uint64_t>(&tmC)),
                             "r"(s0), "r"(col0), "r"(store_y)
                             : "memory");
                asm volatile(
                    "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                        reinterpret_cast<uint64_t>(&tmC2)),
                    "r"(s1), "r"(col0), "r"(store_y), "l"(evict_first_policy)
                    : "memory");
                bulk_commit();
              }
              cc += 2;
            } else {
              stage(w, &tmC, col0, store_y, false);
              stage(g, &tmC2, col0, store_y, false, true);
            }
          } else {  // EPI_MUL: acc * aux (bf16)
            // The warp's 32 x 64 aux block goes through the staging slot the
            // result will leave from: coalesced loads (4 rows of 128 B per
            // instruction) into the swizzled slot, then each lane reads its
            // own row (a row per lane straight from global memory touches 32
            // lines per instruction).
            const __nv_bfloat16* ab = static_cast<const __nv_bfloat16*>(a.aux);
            const int ch = lane & 7;
            uint4 av[8];  // all eight loads in flight before any is stored
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int grow = row0 + 4 * k + (lane >> 3), gcol = col0 + 8 * ch;
              av[k] = make_uint4(0u, 0u, 0u, 0u);
              if (grow < a.M) {
                const __nv_bfloat16* src = ab + static_cast<long>(grow) * a.ldaux + gcol;
                if (gcol + 8 <= a.N) {
                  av[k] = *reinterpret_cast<const uint4*>(src);
                } else if (gcol < a.N) {
                  uint32_t e[4] = {0u, 0u, 0u, 0u};
                  for (int t = 0; t < 8 && gcol + t < a.N; ++t)
                    e[t >> 1] |= static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(src)[t]) << (16 * (t & 1));
                  av[k] = make_uint4(e[0], e[1], e[2], e[3]);
                }
              }
            }
            const uint32_t slot = acquire_slot();
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int r = 4 * k + (lane >> 3);
              st_shared_v4(slot + r * 128 + ((ch ^ (r & 7)) << 4), av[k].x, av[k].y, av[k].z, av[k].w);
            }
            __syncwarp();
            uint32_t uw[32];
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const uint4 t = ld_shared_v4(slot + lane * 128 + ((ch ^ (lane & 7)) << 4));
              uw[4 * ch] = t.x;
              uw[4 * ch + 1] = t.y;
              uw[4 * ch + 2] = t.z;
              uw[4 * ch + 3] = t.w;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              w[j] = pack_bf16x2(__uint_as_float(v0[2 * j]) * bf16_bits_to_f32(uw[j] & 0xFFFFu),
                                 __uint_as_float(v0[2 * j + 1]) * bf16_bits_to_f32(uw[j] >> 16));
              w[16 + j] = pack_bf16x2(__uint_as_float(v1[2 * j]) * bf16_bits_to_f32(uw[16 + j] & 0xFFFFu),
                                      __uint_as_float(v1[2 * j + 1]) * bf16_bits_to_f32(uw[16 + j] >> 16));
            }
            stage(w, &tmC, col0, store_y, false, false, slot);  // each lane overwrites only its own row
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(tempty0 + as * 8);  // rank 0's tempty[as]
        else
          mbar_arrive(&tempty[as]);
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

done:
  __syncwarp();
  tc_fence_before();
  if constexpr (PAIR) {
    // neither CTA frees TMEM or leaves while the pair's MMAs, commits or
    // remote arrivals may still touch it
    cluster_sync();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem_base, kTmemCols);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, kTmemCols);
    }
  }
}

// Sums split-K partial slices in split order: out[r, c] = sum_s ws[s][r][c]
// (slice = elements between splits, partial rows of N floats). Four columns
// per thread; the loads of all splits are issued ahead of the in-order adds.
__global__ void splitk_reduce_kernel(const float4* __restrict__ ws, int splits, long slice4, int M, int nq, void* out,
                                     long ldo, int out_f32) {
  pdl_wait();
  pdl_trigger();
  const long total = static_cast<long>(M) * nq;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float4 acc = ws[i];
#pragma unroll 4
    for (int s = 1; s < splits; ++s) {
      const float4 v = ws[s * slice4 + i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const long r = i / nq;
    const long c = (i - r * nq) * 4;
    if (out_f32) {
      float* o = static_cast<float*>(out) + r * ldo + c;
      o[0] = acc.x;
      o[1] = acc.y;
      o[2] = acc.z;
      o[3] = acc.w;
    } else {
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + r * ldo + c;
      const uint32_t lo = pack_bf16x2(acc.x, acc.y), hi = pack_bf16x2(acc.z, acc.w);
      const uintptr_t al = reinterpret_cast<uintptr_t>(o);
      if ((al & 7) == 0) {
        *reinterpret_cast<uint2*>(o) = make_uint2(lo, hi);
      } else if ((al & 3) == 0) {
        reinterpret_cast<uint32_t*>(o)[0] = lo;
        reinterpret_cast<uint32_t*>(o)[1] = hi;
      } else {
        uint16_t* h = reinterpret_cast<uint16_t*>(o);
        h[0] = static_cast<uint16_t>(lo);
        h[1] = static_cast<uint16_t>(lo >> 16);
        h[2] = static_cast<uint16_t>(hi);
        h[3] = static_cast<uint16_t>(hi >> 16);
      }
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D tensor map over a row-major [rows, cols] matrix with row stride `ld`
// elements; box = {box_cols (inner), box_rows}, 128-byte swizzle,
// out-of-bounds elements read as zero (and are not written by stores).
bool make_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, long rows, long cols, long ld,
              int box_cols, int box_rows) {
  auto fn = get_encode_fn();
  if (!fn || !base) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || ((ld * esize) & 15) != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_map_bf16(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols, ld, box_cols, box_rows);
}

template <int BN, bool A_MN, bool B_MN, int STAGES, bool PAIR>
int launch_tc(const GemmDesc& d, const GemmArgs& args, void* out, long ldo, long out_rows, int grid, cudaStream_t s) {
  alignas(64) CUtensorMap ta, tb, tc, tc2;
  bool ok;
  if (!A_MN)
    ok = make_map_bf16(&ta, d.A, d.M, d.K, d.lda, kBK, kBM);
  else
    ok = make_map_bf16(&ta, d.A, d.K, d.M, d.lda, 64, kBK);
  if (!ok) return 2;
  if (!B_MN)
    ok = make_map_bf16(&tb, d.B, d.N, d.K, d.ldb, kBK, PAIR ? (BN == 384 ? 64 : BN / 2) : BN);
  else
    ok = make_map_bf16(&tb, d.B, d.K, d.N, d.ldb, 64, kBK);
  if (!ok) return 2;
  if (args.out_f32)
    ok = make_map(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out, out_rows, d.N, ldo, 32, 32);
  else
    ok = make_map_bf16(&tc, out, out_rows, d.N, ldo, 64, 32);
  if (!ok) return 2;
  if (args.epi == EPI_GELU) {
    if (!make_map_bf16(&tc2, d.out2, d.M, d.N, d.ldo2, 64, 32)) return 2;
  } else {
    tc2 = tc;
  }
  constexpr size_t smem = smem_bytes_for<BN, STAGES, PAIR>();
  static_assert(smem <= 232448, "shared memory budget");
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, STAGES, PAIR>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return 3;
    attr_set = true;
  }
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(384);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl_mask() & 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, tc2, args) != cudaSuccess) return 4;
  } else {
    if (launch_pdl(kern, dim3(grid), dim3(384), smem, s, ta, tb, tc, tc2, args) != cudaSuccess) return 4;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

template <int BN, int STAGES, bool PAIR>
int dispatch_major(const GemmDesc& d, const GemmArgs& a, void* out, long ldo, long rows, int grid, cudaStream_t s) {
  if (!d.a_mn && !d.b_mn) return launch_tc<BN, false, false, STAGES, PAIR>(d, a, out, ldo, rows, grid, s);
  if (!d.a_mn && d.b_mn) return launch_tc<BN, false, true, STAGES, PAIR>(d, a, out, ldo, rows, grid, s);
  if (d.a_mn && d.b_mn) return launch_tc<BN, true, true, STAGES, PAIR>(d, a, out, ldo, rows, grid, s);
  return launch_tc<BN, true, false, STAGES, PAIR>(d, a, out, ldo, rows, grid, s);
}

struct Plan {
  int bn, m_tiles, n_tiles, kb_total, splits, kb_per_split;
  bool pair;          // 256-row tiles on CTA pairs (tcgen05 cta_group::2)
  int rows_per_tile;  // 128, or 256 for pair tiles
};

Plan plan_for(const GemmDesc& d) {
  Plan p;
  p.bn = d.bn;
  if (p.bn == 0) {
    // tile width among {64, 128, 192, 256} with the least column padding,
    // the wider one on ties: a 128 x N x 16 UMMA costs about the same for
    // every N <= 256, so full-width tiles do the most work per instruction
    // (N = 384 -> 192 x 2, N = 1152 -> 192 x 6, N = 1536 -> 256 x 6)
    p.bn = 64;
    long best = (d.N + 63) / 64 * 64L;
    for (int bn : {128, 192, 256}) {
      const long padded = static_cast<long>((d.N + bn - 1) / bn) * bn;
      if (padded <= best) {
        best = padded;
        p.bn = bn;
      }
    }
    // A dependent chain of 128 x N x 16 UMMAs costs about 123 cycles each
    // for N <= 192 and 129 for N = 256 (measured), so a 256-wide grid with a
    // half-empty last column of tiles can still win on rounds of tiles:
    // N = 1152 at M = 16384 runs 5 rounds of 256-wide tiles (5 x 129) instead
    // of 6 rounds of 192-wide ones (6 x 123).
    if (p.bn == 192) {
      const long m128 = (d.M + kBM - 1) / kBM;
      const long r192 = (m128 * ((d.N + 191) / 192) + num_sms() - 1) / num_sms();
      const long r256 = (m128 * ((d.N + 255) / 256) + num_sms() - 1) / num_sms();
      if (r256 * 129 < r192 * 123) p.bn = 256;
    }
  }
  // 256-row tiles on CTA pairs for tiles 256 or 128 wide (192-wide pair tiles
  // measured slower in the step) when padding M to 256 rows wastes little
  // (M = 384 would run 512 rows: a third more work per SM than 128-row tiles)
  // 257..384 columns: one 384-wide pair tile per 256 rows instead of two
  // 192-wide tiles per 128 rows (half the operand bytes per MMA), over many
  // rows or a long K (the dW GEMMs); a short-K GEMM over few rows runs one
  // tile per pair, where the single accumulator buffer costs more than that
  // saves (measured slower for M = 1024..8192 at K = 384)
  const bool long_k = d.K >= 4096 && d.M >= 1024;  // dW GEMMs: a half-empty last pair tile costs little
  const bool pair_rows = d.pair != 0 && (d.M % (2 * kBM) == 0 || d.M >= 4096 || long_k);
  if (d.bn == 0 && p.bn == 192 && d.N > 256 && d.N <= 384 && pair_rows && (d.M >= 4096 || d.K >= 4096))
    p.bn = 384;
  p.pair = p.bn == 384 || ((p.bn == 256 || p.bn == 128) && pair_rows);
  p.rows_per_tile = p.pair ? 2 * kBM : kBM;
  p.m_tiles = (d.M + p.rows_per_tile - 1) / p.rows_per_tile;
  p.n_tiles = (d.N + p.bn - 1) / p.bn;
  p.kb_total = (d.K + kBK - 1) / kBK;
  const int tiles = p.m_tiles * p.n_tiles;
  int splits = d.splits;
  if (splits <= 0) {
    splits = 1;
    const int slots = p.pair ? num_sms() / 2 : num_sms();  // tiles in flight at once
    if (d.epi == EPI_STORE && d.N % 4 == 0 && tiles * 2 <= slots && p.kb_total >= 8)
      splits = std::min(slots / tiles, p.kb_total / 4);
    if (d.max_splits > 0) splits = std::min(splits, d.max_splits);
    if (d.max_ctas > 0) splits = std::min(splits, std::max(1, d.max_ctas / (tiles * (p.pair ? 2 : 1))));
    if (d.max_pair_splits > 0 && p.pair) splits = std::min(splits, d.max_pair_splits);
  }
  if (d.epi != EPI_STORE || d.N % 4 != 0) splits = 1;  // partial rows of N floats must be 16-byte multiples
  splits = std::max(1, std::min(splits, p.kb_total));
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  return p;
}

}  // namespace

bool make_tma_2d_bf16(void* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows) {
  return make_map_bf16(static_cast<CUtensorMap*>(map), base, rows, cols, ld, box_cols, box_rows);
}

// 3-D tiled map over a [d2, d1, d0] bf16 tensor (d0 innermost, row strides
// ld1 and ld2 elements), 128-byte swizzle; coordinates past d1 are clipped,
// so a per-batch view stops stores at the end of each batch element.
bool make_tma_3d_bf16(void* map, const void* base, long d0, long d1, long d2, long ld1, long ld2, int box0,
                      int box1) {
  auto fn = get_encode_fn();
  if (!fn || !base) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || ((ld1 * 2) & 15) != 0 || ((ld2 * 2) & 15) != 0) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld1 * 2), static_cast<cuuint64_t>(ld2 * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tma_2d_f32(void* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows) {
  return make_map(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, rows, cols, ld, box_cols,
                  box_rows);
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

size_t gemm_workspace_bytes(const GemmDesc& d, bool bf16) {
  if (!bf16) return gemm_f32_workspace_bytes(d);
  Plan p = plan_for(d);
  if (p.splits <= 1) return 0;
  return static_cast<size_t>(p.splits) * p.m_tiles * p.rows_per_tile * d.N * sizeof(float);
}

int gemm_bf16(const GemmDesc& d, float* workspace, size_t workspace_bytes, cudaStream_t s, int* err) {
  if (d.M <= 0 || d.N <= 0 || d.K <= 0) return 1;
  const bool f32_epi = d.epi == EPI_ADD || ((d.epi == EPI_STORE || d.epi == EPI_ACCUM) && d.out_f32);
  if ((d.epi == EPI_ADD && !d.out_f32) || ((d.epi == EPI_GELU || d.epi == EPI_MUL) && d.out_f32)) return 1;
  Plan p = plan_for(d);
  GemmArgs a{};
  a.M = d.M;
  a.N = d.N;
  a.K = d.K;
  a.m_tiles = p.m_tiles;
  a.n_tiles = p.n_tiles;
  a.splits = p.splits;
  a.kb_per_split = p.kb_per_split;
  a.kb_total = p.kb_total;
  a.epi = d.epi;
  a.err = err;
  a.aux = d.aux;
  a.ldaux = d.ldaux;
  const bool split = p.splits > 1;
  void* out = d.out;
  long ldo = d.ldo, rows = d.M;
  if (split) {
    const size_t need = static_cast<size_t>(p.splits) * p.m_tiles * p.rows_per_tile * d.N * sizeof(float);
    if (!workspace || workspace_bytes < need) return 5;
    out = workspace;
    ldo = d.N;
    rows = static_cast<long>(p.splits) * p.m_tiles * p.rows_per_tile;
    a.out_f32 = 1;
    a.partial = 1;
  } else {
    a.out_f32 = f32_epi ? 1 : 0;
    a.partial = 0;
  }
  if (d.aux && (((reinterpret_cast<uintptr_t>(d.aux) & 15) != 0) || ((d.ldaux * (d.aux_f32 ? 4 : 2)) & 15) != 0))
    return 2;
  const int units = p.m_tiles * p.n_tiles * p.splits;
  const int grid = p.pair ? 2 * std::min(units, num_sms() / 2) : std::min(units, num_sms());
  int rc;
  switch (p.bn) {
    case 256:
      rc = p.pair ? dispatch_major<256, 5, true>(d, a, out, ldo, rows, grid, s)
                  : dispatch_major<256, 4, false>(d, a, out, ldo, rows, grid, s);
      break;
    case 384: rc = dispatch_major<384, 4, true>(d, a, out, ldo, rows, grid, s); break;
    case 192: rc = dispatch_major<192, 4, false>(d, a, out, ldo, rows, grid, s); break;
    case 128:
      rc = p.pair ? dispatch_major<128, 6, true>(d, a, out, ldo, rows, grid, s)
                  : dispatch_major<128, 5, false>(d, a, out, ldo, rows, grid, s);
      break;
    case 64: rc = dispatch_major<64, 6, false>(d, a, out, ldo, rows, grid, s); break;
    default: return 6;
  }
  if (rc) return rc;
  if (split) {
    const long total = static_cast<long>(d.M) * (d.N / 4);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<long>((total + threads - 1) / threads, 8L * num_sms()));
    if (launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(threads), 0, s,
                   reinterpret_cast<const float4*>(workspace), p.splits,
                   static_cast<long>(p.m_tiles) * p.rows_per_tile * d.N / 4, d.M, d.N / 4, d.out, d.ldo,
                   static_cast<int>(d.out_f32)) != cudaSuccess)
      return 4;
  }
  return 0;
}

}  // namespace sb
