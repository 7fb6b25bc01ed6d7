// Fused causal self-attention on the tcgen05 tensor cores (bf16 operands,
// fp32 accumulation in TMEM): the nanoGPT attention block
// (examples/nanogpt/model.shf:55-70)
//   s = (q @ k^T) / sqrt(Hd); s = where(tril(ones[T,T]) == 1, s, -1e10);
//   p = softmax(s) (lib/nn.shf:24-26); o = p @ v; heads merged to [B*T, D]
// and its VJP (the `@`, `/`, `where` and softmax rules of
// autodiff/reverse.rs:585-689, 551-583, 1014-1019, 814-828).
// Masked scores contribute exp(-1e10 - max) == 0, so masked keys are skipped.
//
// Forward, persistent over (batch, head, 128-query tile) items, two CTAs per
// SM; 192 threads:
//   warp 0    TMA: Q tile per item (two slots), K/V tiles of 128 keys (one
//             slot each)
//   warp 1    TMEM owner + single-thread UMMA issuer:
//             S = Q K^T (M=128, N=128, K=64) into TMEM;
//             O_j = P V (M=128, N=64, K=128) into TMEM
//   warps 2-5 softmax: thread = query row; reads its S row from TMEM, keeps
//             the running max / sum, writes P (bf16, 128B-swizzled K-major)
//             to shared memory for the P V UMMA, accumulates O_j in registers.
// Backward, persistent (one CTA per SM) over (batch, head, 128-key tile) work
// items, each looping over the query tiles at or after its key tile:
//   S^T = K Q^T and dP^T = V dO^T into TMEM (thread = key row);
//   P^T, dS^T = P^T * (dP^T - delta) / sqrt(Hd) written to shared memory;
//   dV += P^T dO, dK += dS^T Q (accumulated in TMEM across query tiles);
//   dQ_i = dS K (the dS^T tile read as an MN-major operand), added into an
//   fp32 dQ buffer with TMA bulk reduce-adds, converted to bf16 at the end.
// Q/K/V/dO tiles are 128 rows x 64 bf16 (128-byte rows), the same smem tile
// serving as a K-major operand (rows = M/N) and an MN-major one (rows = K).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "sb_kernels.h"
#include "sb_nn.h"
#include "sb_ptx.cuh"
#define SB_PDL_FAMILY 2
#include "sb_launch.cuh"

namespace sb {

namespace {

constexpr int kT = 128;   // rows per tile
constexpr int kHd = 64;   // head dim handled by the tensor-core path
constexpr uint32_t kTileBytes = kT * kHd * 2;  // 16 KB
constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  int B, T, H, D;
  int ntiles;  // ceil(T / 128)
  float scale;  // 1 / sqrt(Hd)
  __nv_bfloat16* out;
  float* lse;
  const __nv_bfloat16* o;     // backward: forward output [B*T, D]
  const __nv_bfloat16* dout;  // backward: upstream gradient [B*T, D]
  float* dq_acc;
  __nv_bfloat16* dqkv;
  int* err;
};

// Writes 32 bf16 values (columns 32c .. 32c+31 of row r) into a 128-row,
// 128-column tile stored as two 64-column K-major SW128 atoms of 16 KB.
__device__ __forceinline__ void store_row32(uint32_t tile, int r, int c, const uint32_t (&pk)[16]) {
  const uint32_t row = tile + (c >> 1) * 16384 + r * 128;
  const int c0 = (c & 1) * 4;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    st_shared_v4(row + (((c0 + k) ^ (r & 7)) << 4), pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
}

__device__ __forceinline__ uint64_t kdesc(uint32_t tile, int kk) {  // K-major, 64-wide K atom
  return make_sw128_desc(tile + kk * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t kdesc2(uint32_t tile, int kk) {  // K-major, K=128 as two atoms
  return make_sw128_desc(tile + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mndesc(uint32_t tile, int kk, uint32_t lbo) {  // MN-major, K rows
  return make_sw128_desc(tile + kk * 2048, lbo, 1024);
}

// j-th work item of this CTA. Items come longest first; rounds of gridDim.x
// items alternate direction, so the CTAs that took the last long items of one
// round take the first short ones of the next and no CTA ends up with a long
// item more than the others plus a short one.
__device__ __forceinline__ int item_of(int j) {
  const int g = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
  return j * g + ((j & 1) ? g - 1 - b : b);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------

constexpr size_t kFwdSmem = 1024 + 2 * kTileBytes /*Q x2*/ + kTileBytes /*K*/ + kTileBytes /*V*/ +
                            2 * kTileBytes /*P*/ + 16 * 8 + 16;

// Forward work item u: query tile qt = ntiles - 1 - u / (B*H) (long rows
// first), head bh = u % (B*H).
__device__ __forceinline__ void fwd_item(const AttnArgs& a, int u, int& qt, int& bh, int& h, int& row0) {
  const int bhn = a.B * a.H;
  qt = a.ntiles - 1 - u / bhn;
  bh = u % bhn;
  h = bh % a.H;
  row0 = (bh / a.H) * a.T;
}

// ~98 KB of shared memory and 256 TMEM columns: two CTAs per SM, so one CTA's
// softmax overlaps the other's loads and UMMAs. Persistent over (batch, head,
// query-tile) items: Q is double buffered and the K / V slots and every
// barrier phase continue across items, so the next item's loads overlap the
// current item's softmax.
__global__ void __launch_bounds__(192, 2) attn_fwd_tc(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;  // [2]
  uint8_t* sK = sQ + 2 * kTileBytes;
  uint8_t* sV = sK + kTileBytes;
  uint8_t* sP = sV + kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kTileBytes);
  uint64_t* q_full = bars + 0;   // [2]
  uint64_t* q_empty = bars + 2;  // [2]
  uint64_t* k_full = bars + 4;
  uint64_t* k_empty = bars + 5;
  uint64_t* v_full = bars + 6;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 8;
  uint64_t* p_full = bars + 9;
  uint64_t* o_full = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nitems = a.B * a.H * a.ntiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 11; ++i) mbar_init(&bars[i], i == 9 ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  // inputs come from the preceding kernel: no global access, and no TMEM
  // allocation, before this
  pdl_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    // K_c is reloaded once S_{c-1} has consumed the single K slot, V_c once
    // P_{c-1} V_{c-1} has consumed the V slot (c counts key tiles across
    // items); both land during softmax.
    if (lane == 0) {
      uint32_t c = 0;
      int j = 0;
      bool ok = true;
      for (int u = item_of(j); u < nitems && ok; u = item_of(++j)) {
        int qt, bh, h, row0;
        fwd_item(a, u, qt, bh, h, row0);
        const int qb = j & 1;
        if (!mbar_wait(&q_empty[qb], ((j >> 1) & 1) ^ 1, a.err, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qb], kTileBytes);
        tma_load_2d(sQ + qb * kTileBytes, &tm, &q_full[qb], h * kHd, row0 + qt * kT);
        for (int kv = 0; kv <= qt; ++kv, ++c) {
          const uint32_t ph = (c & 1) ^ 1;
          if (!mbar_wait(k_empty, ph, a.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(k_full, kTileBytes);
          tma_load_2d(sK, &tm, k_full, a.D + h * kHd, row0 + kv * kT);
          if (!mbar_wait(v_empty, ph, a.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(v_full, kTileBytes);
          tma_load_2d(sV, &tm, v_full, 2 * a.D + h * kHd, row0 + kv * kT);
        }
      }
      // no UMMA commit may arrive on this CTA's barriers after it exits
      if (ok) {
        mbar_wait(k_empty, (c & 1) ^ 1, a.err, abort_flag);
        mbar_wait(v_empty, (c & 1) ^ 1, a.err, abort_flag);
        for (int i = 0; i < 2; ++i, ++j) mbar_wait(&q_empty[j & 1], ((j >> 1) & 1) ^ 1, a.err, abort_flag);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = make_idesc_bf16(128, 64, false, true);
      const uint32_t p_addr = smem_u32(sP);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      uint32_t c = 0;
      int j = 0;
      bool ok = true;
      for (int u = item_of(j); u < nitems && ok; u = item_of(++j)) {
        int qt, bh, h, row0;
        fwd_item(a, u, qt, bh, h, row0);
        const int qb = j & 1;
        if (!mbar_wait(&q_full[qb], (j >> 1) & 1, a.err, abort_flag)) break;
        const uint32_t q_addr = smem_u32(sQ + qb * kTileBytes);
        for (int kv = 0; kv <= qt; ++kv, ++c) {
          const uint32_t ph = c & 1;
          if (!mbar_wait(k_full, ph, a.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(tS, kdesc(q_addr, kk), kdesc(k_addr, kk), idS, kk > 0);
          umma_commit(s_full);
          umma_commit(k_empty);
          if (kv == qt) umma_commit(&q_empty[qb]);  // the item's last read of Q
          if (!mbar_wait(p_full, ph, a.err, abort_flag) || !mbar_wait(v_full, ph, a.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) umma_f16(tO, kdesc2(p_addr, kk), mndesc(v_addr, kk, 8192), idO, kk > 0);
          umma_commit(o_full);
          umma_commit(v_empty);
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl = a.scale * kLog2e;  // scores -> log2 units
    const uint32_t p_addr = smem_u32(sP);
    uint32_t c = 0;
    bool ok = true;
    int n = 0;  // items of this CTA
    for (int u = item_of(n); u < nitems && ok; u = item_of(++n)) {
      int qt, bh, h, row0;
      fwd_item(a, u, qt, bh, h, row0);
      const int q = qt * kT + r;
      float m = -INFINITY, l = 0.f;
      float o[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) o[i] = 0.f;
      for (int j = 0; j <= qt; ++j, ++c) {
        if (!mbar_wait(s_full, c & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Causal mask: only the diagonal tile (j == qt) has masked keys. There,
        // chunk cc (keys 32cc..32cc+31 of the tile) is fully visible to this
        // warp's rows 32*quarter.. for cc < quarter, fully masked for
        // cc > quarter, and masked above the diagonal (t > lane) for
        // cc == quarter.
        const int clast = (j == qt) ? quarter : 3;
        float mx = -INFINITY;  // over raw scores (sl > 0)
#pragma unroll 1
        for (int cc = 0; cc <= clast; ++cc) {
          uint32_t v[32];
          tmem_ld32(tS + lane_base + cc * 32, v);
          tmem_wait_ld();
          if (j == qt && cc == quarter) {
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (t <= lane) mx = fmaxf(mx, __uint_as_float(v[t]));
          } else {
#pragma unroll
            for (int t = 0; t < 32; ++t) mx = fmaxf(mx, __uint_as_float(v[t]));
          }
        }
        const float mn = fmaxf(m, mx * sl);
        const float corr = ex2_approx(m - mn);
        float rs = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t pk[16];
          if (cc > clast) {
#pragma unroll
            for (int t = 0; t < 16; ++t) pk[t] = 0u;
          } else {
            uint32_t v[32];
            tmem_ld32(tS + lane_base + cc * 32, v);
            tmem_wait_ld();
            const bool part = (j == qt && cc == quarter);
#pragma unroll
            for (int t = 0; t < 32; t += 2) {
              float p0 = ex2_approx(fmaf(__uint_as_float(v[t]), sl, -mn));
              float p1 = ex2_approx(fmaf(__uint_as_float(v[t + 1]), sl, -mn));
              if (part) {
                p0 = (t <= lane) ? p0 : 0.f;
                p1 = (t + 1 <= lane) ? p1 : 0.f;
              }
              rs += p0 + p1;
              pk[t >> 1] = pack_bf16x2(p0, p1);
            }
          }
          store_row32(p_addr, r, cc, pk);
        }
        l = l * corr + rs;
        m = mn;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (!mbar_wait(o_full, c & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t v0[32], v1[32];
        tmem_ld32(tO + lane_base, v0);
        tmem_ld32(tO + lane_base + 32, v1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o[i] = o[i] * corr + __uint_as_float(v0[i]);
          o[32 + i] = o[32 + i] * corr + __uint_as_float(v1[i]);
        }
        tc_fence_before();
      }
      if (ok) {
        // O leaves through the (now idle) P buffer: each lane writes its row
        // swizzled, then every store instruction covers 4 rows x 128 B
        // (a row per lane straight to global memory touches 32 lines)
        const float inv = 1.f / l;
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = pack_bf16x2(o[2 * i] * inv, o[2 * i + 1] * inv);
        st_row128_sw(p_addr, r, w);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int rr = quarter * 32 + 4 * k + (lane >> 3), ch = lane & 7;
          const uint4 v = ld_shared_v4(p_addr + rr * 128 + ((ch ^ (rr & 7)) << 4));
          if (qt * kT + rr < a.T)
            *reinterpret_cast<uint4*>(a.out + static_cast<long>(row0 + qt * kT + rr) * a.D + h * kHd + ch * 8) = v;
        }
        __syncwarp();  // the next item's P rows overwrite what the other lanes read
        // natural-log log-sum-exp of the scaled scores
        if (q < a.T) a.lse[static_cast<long>(bh) * a.T + q] = (m + log2f(l)) / kLog2e;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------

constexpr int kBwdSoftmaxWarps = 8;
constexpr int kBwdThreads = 32 * (2 + kBwdSoftmaxWarps);
constexpr size_t kBwdSmem = 1024 + 4 * kTileBytes /*K,V x2*/ + 4 * kTileBytes /*Q,dO x2*/ +
                            4 * kTileBytes /*P^T, dS^T*/ + 4 * kT * 4 /*lse, delta x2*/ + 24 * 8 + 16;

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t smem_src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_src), "r"(x), "r"(y)
               : "memory");
}

// Work item u of the VJP: key tile kt = u / (B*H) (long items first), head
// bh = u % (B*H); it loops over the query tiles kt .. ntiles-1.
struct BwdItem {
  int kt, bh, h, row0, nq, b;
};
__device__ __forceinline__ BwdItem bwd_item(const AttnArgs& a, int u) {
  BwdItem w;
  const int bhn = a.B * a.H;
  w.kt = u / bhn;
  w.bh = u % bhn;
  w.b = w.bh / a.H;
  w.h = w.bh % a.H;
  w.row0 = w.b * a.T;
  w.nq = a.ntiles - w.kt;
  return w;
}

// Persistent VJP: one CTA per SM loops over work items. K/V are double
// buffered and the Q/dO ring runs across items, so the next item's loads
// land while the current one computes; lse/delta of the next query tile are
// loaded one tile ahead; dK/dV leave through swizzled staging and TMA stores.
// Warp 0 loads, warp 1 issues the UMMAs, warps 2-9 compute P^T / dS^T and
// drain dQ / dK / dV: two warps per TMEM lane quarter (the warp's index mod
// 4), each owning one 64-column half of its 32 rows -- query chunks 2h and
// 2h+1 of P^T and dS^T (SW128 atom h), dQ columns 32h..32h+31, and dK (h = 0)
// or dV (h = 1) -- so each sub-partition runs two of these warps and one's
// TMEM loads and exponentials overlap the other's. A warp stages its dQ
// reduce-adds and its dK / dV stores in its own rows of atom h of dS^T and
// P^T, which no UMMA reads between the commit it waited for and the next
// tile's softmax.
__global__ void __launch_bounds__(kBwdThreads, 1) attn_bwd_tc(const __grid_constant__ CUtensorMap tm_qkv,
                                                      const __grid_constant__ CUtensorMap tm_do,
                                                      const __grid_constant__ CUtensorMap tm_dq,
                                                      const __grid_constant__ CUtensorMap tm_dkv, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm;                       // [2]
  uint8_t* sV = sK + 2 * kTileBytes;      // [2]
  uint8_t* sQ = sV + 2 * kTileBytes;      // [2]
  uint8_t* sdO = sQ + 2 * kTileBytes;     // [2]
  uint8_t* sPT = sdO + 2 * kTileBytes;    // 32 KB; also dK (first atom) / dV (second atom) staging
  uint8_t* sdST = sPT + 2 * kTileBytes;   // 32 KB; also dQ staging
  float* sLse = reinterpret_cast<float*>(sdST + 2 * kTileBytes);  // [2][128]
  float* sDel = sLse + 2 * kT;                                // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDel + 2 * kT);
  uint64_t* kv_full = bars + 0;     // [2]
  uint64_t* kv_empty = bars + 2;    // [2]
  uint64_t* qd_full = bars + 4;     // [2]
  uint64_t* qd_empty = bars + 6;    // [2]
  uint64_t* st_full = bars + 8;
  uint64_t* p_full = bars + 9;
  uint64_t* dq_full = bars + 10;
  uint64_t* dq_empty = bars + 11;
  uint64_t* acc_full = bars + 12;
  uint64_t* acc_empty = bars + 13;
  uint64_t* stats_full = bars + 14;  // [2]: the softmax warps wrote lse / delta of a query tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nitems = a.B * a.H * a.ntiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&stats_full[i], kBwdSoftmaxWarps);
    }
    mbar_init(st_full, 1);
    mbar_init(p_full, kBwdSoftmaxWarps);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, kBwdSoftmaxWarps);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kBwdSoftmaxWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    tma_prefetch_desc(&tm_dkv);
  }
  // inputs come from the preceding kernel: no global access, and no TMEM
  // allocation, before this
  pdl_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tST = tmem, tdPT = tmem + 128, tdV = tmem + 256, tdK = tmem + 320, tdQ = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t g = 0;  // query tiles loaded by this CTA
      int j = 0;       // items of this CTA
      bool ok = true;
      for (int u = item_of(j); u < nitems && ok; u = item_of(++j)) {
        const BwdItem w = bwd_item(a, u);
        const int kb = j & 1;
        if (!mbar_wait(&kv_empty[kb], ((j >> 1) & 1) ^ 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[kb], 2 * kTileBytes);
        tma_load_2d(sK + kb * kTileBytes, &tm_qkv, &kv_full[kb], a.D + w.h * kHd, w.row0 + w.kt * kT);
        tma_load_2d(sV + kb * kTileBytes, &tm_qkv, &kv_full[kb], 2 * a.D + w.h * kHd, w.row0 + w.kt * kT);
        for (int it = 0; it < w.nq; ++it, ++g) {
          const int s = g & 1, i = w.kt + it;
          if (!mbar_wait(&qd_empty[s], ((g >> 1) & 1) ^ 1, a.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&qd_full[s], 2 * kTileBytes);
          tma_load_2d(sQ + s * kTileBytes, &tm_qkv, &qd_full[s], w.h * kHd, w.row0 + i * kT);
          tma_load_2d(sdO + s * kTileBytes, &tm_do, &qd_full[s], w.h * kHd, w.row0 + i * kT);
        }
      }
      // wait for the final releases of every buffer, so that no UMMA commit
      // arrives on this CTA's barriers after it exits
      if (ok) {
        for (int i = 0; i < 2; ++i, ++g)
          if (!mbar_wait(&qd_empty[g & 1], ((g >> 1) & 1) ^ 1, a.err, abort_flag)) break;
        for (int i = 0; i < 2; ++i, ++j)
          if (!mbar_wait(&kv_empty[j & 1], ((j >> 1) & 1) ^ 1, a.err, abort_flag)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idKV = make_idesc_bf16(128, 64, false, true);
      constexpr uint32_t idQ = make_idesc_bf16(128, 64, true, true);
      const uint32_t pt_addr = smem_u32(sPT), dst_addr = smem_u32(sdST);
      uint32_t g = 0;
      int j = 0;
      bool ok = true;
      for (int u = item_of(j); u < nitems && ok; u = item_of(++j)) {
        const BwdItem w = bwd_item(a, u);
        const int kb = j & 1;
        if (!mbar_wait(&kv_full[kb], (j >> 1) & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + kb * kTileBytes), v_addr = smem_u32(sV + kb * kTileBytes);
        for (int it = 0; it < w.nq; ++it, ++g) {
          const int s = g & 1;
          if (!mbar_wait(&qd_full[s], (g >> 1) & 1, a.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + s * kTileBytes), do_addr = smem_u32(sdO + s * kTileBytes);
          // S^T, dP^T overwrite what the softmax warps read for tile g-1
          // (they arrived on p_full(g-1) before this point)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(tST, kdesc(k_addr, kk), kdesc(q_addr, kk), idS, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(tdPT, kdesc(v_addr, kk), kdesc(do_addr, kk), idS, kk > 0);
          umma_commit(st_full);
          if (!mbar_wait(p_full, g & 1, a.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (it == 0 && j > 0) {  // the previous item's dK / dV have been read out
            if (!mbar_wait(acc_empty, (j - 1) & 1, a.err, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tdV, kdesc2(pt_addr, kk), mndesc(do_addr, kk, 8192), idKV, (it > 0 || kk > 0));
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tdK, kdesc2(dst_addr, kk), mndesc(q_addr, kk, 8192), idKV, (it > 0 || kk > 0));
          if (g > 0) {
            if (!mbar_wait(dq_empty, (g - 1) & 1, a.err, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tdQ, mndesc(dst_addr, kk, 16384), mndesc(k_addr, kk, 8192), idQ, kk > 0);
          umma_commit(dq_full);
          umma_commit(&qd_empty[s]);
        }
        if (!ok) break;
        umma_commit(acc_full);
        umma_commit(&kv_empty[kb]);
      }
    }
  } else {
    const int quarter = warp & 3;        // TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;    // 64-column half of those rows
    const int tid = quarter * 32 + lane;  // 0..127: key row (S^T, dK, dV) / query row (dQ)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl = a.scale * kLog2e;
    const float2 sl2 = make_float2(sl, sl), sc2 = make_float2(a.scale, a.scale);
    const uint32_t pt_addr = smem_u32(sPT), dst_addr = smem_u32(sdST);
    // this warp's 32 rows of atom `half` of P^T and of dS^T (4 KB each)
    const uint32_t own_pt = pt_addr + half * 16384 + quarter * 4096;
    const uint32_t own_dst = dst_addr + half * 16384 + quarter * 4096;
    // Per query row of tile i of head bh into buffer s: lse (log2 units) and
    // delta * scale, delta = rowsum(dO * O). Issued one tile ahead so that
    // the global loads overlap the previous tile's UMMAs.
    // delta of the quarter's 32 rows with coalesced loads, half of them per
    // warp: instruction k reads rows 16h + 4k .. +3 (eight lanes a row, 16
    // bytes each; all eight loads in flight first), the eight partial dot
    // products of a row are summed by shuffles.
    auto load_row_stats = [&](const BwdItem& w, int i, int s) {
      const int q = i * kT + tid;
      const int ch = lane & 7;
      const int r0 = quarter * 32 + half * 16;
      uint4 ov[4], dv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int qk = i * kT + r0 + 4 * k + (lane >> 3);
        ov[k] = dv[k] = make_uint4(0u, 0u, 0u, 0u);
        if (qk < a.T) {
          const long off = static_cast<long>(w.row0 + qk) * a.D + w.h * kHd + ch * 8;
          ov[k] = *reinterpret_cast<const uint4*>(a.o + off);
          dv[k] = *reinterpret_cast<const uint4*>(a.dout + off);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t ow[4] = {ov[k].x, ov[k].y, ov[k].z, ov[k].w}, dw[4] = {dv[k].x, dv[k].y, dv[k].z, dv[k].w};
        float dl = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dl += bf16_bits_to_f32(static_cast<uint16_t>(ow[e] & 0xFFFFu)) *
                bf16_bits_to_f32(static_cast<uint16_t>(dw[e] & 0xFFFFu));
          dl += bf16_bits_to_f32(static_cast<uint16_t>(ow[e] >> 16)) * bf16_bits_to_f32(static_cast<uint16_t>(dw[e] >> 16));
        }
        dl += __shfl_xor_sync(0xffffffffu, dl, 4);
        dl += __shfl_xor_sync(0xffffffffu, dl, 2);
        dl += __shfl_xor_sync(0xffffffffu, dl, 1);
        if (ch == 0) sDel[s * kT + r0 + 4 * k + (lane >> 3)] = dl * a.scale;
      }
      if (half == 0) sLse[s * kT + tid] = (q < a.T) ? a.lse[static_cast<long>(w.bh) * a.T + q] * kLog2e : INFINITY;
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats_full[s]);
    };
    // Stats buffer s is rewritten for tile g+2 only after this thread passed
    // st_full(g+1), which the MMA warp commits after every warp's p_full(g):
    // no reader of the tile-g values is left by then.
    bool ok = true;
    uint32_t g = 0;
    int j = 0;
    if (static_cast<int>(blockIdx.x) < nitems) {
      const BwdItem w0 = bwd_item(a, blockIdx.x);
      load_row_stats(w0, w0.kt, 0);
    }
    for (int u = item_of(j); u < nitems && ok; u = item_of(++j)) {
      const BwdItem w = bwd_item(a, u);
      const int key = w.kt * kT + tid;
      for (int it = 0; it < w.nq; ++it, ++g) {
        const int s = g & 1, i = w.kt + it;
        if (!mbar_wait(st_full, g & 1, a.err, abort_flag) ||
            !mbar_wait(&stats_full[s], (g >> 1) & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // this warp's rows of P^T / dS^T held its previous dQ / dK / dV staging
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        const float* lse2 = sLse + s * kT;
        const float* del = sDel + s * kT;
        // Causal mask (key <= query) matters only on the diagonal tile i == kt:
        // there this warp's keys 32*quarter + lane see query chunk c (queries
        // 32c..32c+31 of the tile) fully for c > quarter, not at all for
        // c < quarter (P = dS = 0), and for t >= lane when c == quarter.
        const int cfirst = (i == w.kt) ? quarter : 0;
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
          uint32_t pp[16], pd[16];
          if (c < cfirst) {
#pragma unroll
            for (int t = 0; t < 16; ++t) pp[t] = pd[t] = 0u;
          } else {
            uint32_t sv[32], dv[32];
            tmem_ld32(tST + lane_base + c * 32, sv);
            tmem_ld32(tdPT + lane_base + c * 32, dv);
            tmem_wait_ld();
            const bool part = (i == w.kt && c == quarter);
#pragma unroll
            for (int t = 0; t < 32; t += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(lse2 + c * 32 + t);
              const float4 d4 = *reinterpret_cast<const float4*>(del + c * 32 + t);
              // packed f32x2 arithmetic: the same single-precision fma / mul
              // per element, one instruction per pair
              const float2 e01 = __ffma2_rn(make_float2(__uint_as_float(sv[t]), __uint_as_float(sv[t + 1])), sl2,
                                            make_float2(-l4.x, -l4.y));
              const float2 e23 = __ffma2_rn(make_float2(__uint_as_float(sv[t + 2]), __uint_as_float(sv[t + 3])), sl2,
                                            make_float2(-l4.z, -l4.w));
              float p[4] = {ex2_approx(e01.x), ex2_approx(e01.y), ex2_approx(e23.x), ex2_approx(e23.y)};
              if (part) {
#pragma unroll
                for (int uu = 0; uu < 4; ++uu)
                  if (t + uu < lane) p[uu] = 0.f;
              }
              const float2 f01 = __ffma2_rn(make_float2(__uint_as_float(dv[t]), __uint_as_float(dv[t + 1])), sc2,
                                            make_float2(-d4.x, -d4.y));
              const float2 f23 = __ffma2_rn(make_float2(__uint_as_float(dv[t + 2]), __uint_as_float(dv[t + 3])), sc2,
                                            make_float2(-d4.z, -d4.w));
              const float2 d01 = __fmul2_rn(make_float2(p[0], p[1]), f01);
              const float2 d23 = __fmul2_rn(make_float2(p[2], p[3]), f23);
              pp[t >> 1] = pack_bf16x2(p[0], p[1]);
              pp[(t >> 1) + 1] = pack_bf16x2(p[2], p[3]);
              pd[t >> 1] = pack_bf16x2(d01.x, d01.y);
              pd[(t >> 1) + 1] = pack_bf16x2(d23.x, d23.y);
            }
          }
          store_row32(pt_addr, tid, c, pp);
          store_row32(dst_addr, tid, c, pd);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        // lse / delta of the next query tile (of this item or the next one)
        if (it + 1 < w.nq) {
          load_row_stats(w, i + 1, s ^ 1);
        } else if (item_of(j + 1) < nitems) {
          const BwdItem wn = bwd_item(a, item_of(j + 1));
          load_row_stats(wn, wn.kt, s ^ 1);
        }
        // dQ tile partial: TMEM lane = query row of tile i
        if (!mbar_wait(dq_full, g & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t qv[32];
        tmem_ld32(tdQ + lane_base + half * 32, qv);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
        // This warp's 32 query rows x 32 columns of dQ are added into the fp32
        // accumulator with one bulk tensor reduce-add staged in the warp's own
        // dS^T rows (the dK and dQ UMMAs that read them have completed). Rows
        // past T hold exact zeros (their P and dS are zero).
        st_row128_sw(own_dst, lane, qv);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tm_dq, own_dst, w.h * kHd + half * 32, w.row0 + i * kT + quarter * 32);
          bulk_commit();
        }
      }
      if (!ok) break;
      // dK (half 0) or dV (half 1) of this item: TMEM -> bf16 -> the warp's
      // own rows of P^T (no bulk copy reads them: the dQ staging is in dS^T)
      // -> TMA store clipped at T
      if (!mbar_wait(acc_full, j & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tacc = half ? tdV : tdK;
      uint32_t x0[32], x1[32];
      tmem_ld32(tacc + lane_base, x0);
      tmem_ld32(tacc + lane_base + 32, x1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      uint32_t wx[32];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        wx[t] = pack_bf16x2(__uint_as_float(x0[2 * t]), __uint_as_float(x0[2 * t + 1]));
        wx[16 + t] = pack_bf16x2(__uint_as_float(x1[2 * t]), __uint_as_float(x1[2 * t + 1]));
      }
      st_row128_sw(own_pt, lane, wx);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tm_dkv, own_pt, (1 + half) * a.D + w.h * kHd, w.kt * kT + quarter * 32, w.b);
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dq (bf16, columns [0, D) of dqkv) = dq_acc (f32 [rows, D]). Block
// (tx, ty): ty rows, each thread 8 consecutive values of a row per step (two
// 16-byte loads, one 16-byte store); D is a multiple of 8 (64 per head).
__global__ void dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dqkv, long rows, int D) {
  pdl_wait();
  pdl_trigger();
  const long r = static_cast<long>(blockIdx.x) * blockDim.y + threadIdx.y;
  if (r >= rows) return;
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    const float4* src = reinterpret_cast<const float4*>(acc + r * D + c);
    const float4 v0 = src[0], v1 = src[1];
    uint4 u;
    u.x = pack_bf16x2(v0.x, v0.y);
    u.y = pack_bf16x2(v0.z, v0.w);
    u.z = pack_bf16x2(v1.x, v1.y);
    u.w = pack_bf16x2(v1.z, v1.w);
    *reinterpret_cast<uint4*>(dqkv + r * 3 * D + c) = u;
  }
}

}  // namespace

bool attention_tc_supported(const AttnShape& sh) { return sh.Hd == kHd && sh.T >= 1 && sh.B >= 1 && sh.H >= 1; }

int attention_fwd_tc(const void* qkv, void* o, float* lse, const AttnShape& sh, cudaStream_t s, int* err) {
  const int D = sh.H * sh.Hd, N = sh.B * sh.T;
  alignas(64) CUtensorMap tm;
  if (!make_tma_2d_bf16(&tm, qkv, N, 3L * D, 3L * D, 64, kT)) return 2;
  AttnArgs a{};
  a.B = sh.B;
  a.T = sh.T;
  a.H = sh.H;
  a.D = D;
  a.ntiles = (sh.T + kT - 1) / kT;
  a.scale = 1.0f / sqrtf(static_cast<float>(sh.Hd));
  a.out = static_cast<__nv_bfloat16*>(o);
  a.lse = lse;
  a.err = err;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kFwdSmem)) !=
        cudaSuccess)
      return 3;
    attr = true;
  }
  launch_pdl(attn_fwd_tc, dim3(std::min(sh.B * sh.H * a.ntiles, 2 * num_sms())), dim3(192), kFwdSmem, s, tm, a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

size_t attention_bwd_tc_workspace_bytes(const AttnShape& sh) {
  return static_cast<size_t>(sh.B) * sh.T * sh.H * sh.Hd * sizeof(float);
}

int attention_bwd_tc(const void* qkv, const void* o, const void* dout, const float* lse, void* dqkv, float* ws,
                     const AttnShape& sh, cudaStream_t s, int* err) {
  const int D = sh.H * sh.Hd, N = sh.B * sh.T;
  float* dq_acc = ws;
  if (cudaMemsetAsync(dq_acc, 0, static_cast<size_t>(N) * D * sizeof(float), s) != cudaSuccess) return 4;
  alignas(64) CUtensorMap tq, td, tdq, tdkv;
  if (!make_tma_2d_bf16(&tq, qkv, N, 3L * D, 3L * D, 64, kT)) return 2;
  if (!make_tma_2d_bf16(&td, dout, N, D, D, 64, kT)) return 2;
  if (!make_tma_2d_f32(&tdq, dq_acc, N, D, D, 32, 32)) return 2;
  // dK / dV stores through a [B, T, 3D] view, clipped at T per batch element
  if (!make_tma_3d_bf16(&tdkv, dqkv, 3L * D, sh.T, sh.B, 3L * D, static_cast<long>(sh.T) * 3 * D, 64, 32)) return 2;
  AttnArgs a{};
  a.B = sh.B;
  a.T = sh.T;
  a.H = sh.H;
  a.D = D;
  a.ntiles = (sh.T + kT - 1) / kT;
  a.scale = 1.0f / sqrtf(static_cast<float>(sh.Hd));
  a.lse = const_cast<float*>(lse);
  a.o = static_cast<const __nv_bfloat16*>(o);
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.dq_acc = dq_acc;
  a.dqkv = static_cast<__nv_bfloat16*>(dqkv);
  a.err = err;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBwdSmem)) !=
        cudaSuccess)
      return 3;
    attr = true;
  }
  const int items = sh.B * sh.H * a.ntiles;
  launch_pdl(attn_bwd_tc, dim3(std::min(items, num_sms())), dim3(kBwdThreads), kBwdSmem, s, tq, td, tdq, tdkv, a);
  if (cudaPeekAtLastError() != cudaSuccess) return 4;
  const int tx = std::min(D / 8, 128), ty = std::max(1, 384 / tx);
  launch_pdl(dq_convert_kernel, dim3((N + ty - 1) / ty), dim3(tx, ty), 0, s, dq_acc, static_cast<__nv_bfloat16*>(dqkv),
             static_cast<long>(N), D);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace sb
