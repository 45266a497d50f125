// Backward main kernel for B200 (sm_100a): dK/dV-stationary, tcgen05 MMAs
// accumulating S^T, dP^T, dV, dK and dQ in tensor memory.
//
// Computes what the reference backward main kernel computes
// (wan_flash/bwd_sm90.py of Quarky93/wan-flash, `_mma_m_block` :947-1046):
// for one 128-row KV block it walks the query blocks and forms
//     S^T  = K Q^T                      P^T = exp2(S^T * scale_log2 - lse_log2)
//     dP^T = V dO^T                     dS^T = P^T * (dP^T - D)
//     dV  += P^T dO                     dK  += dS^T Q         dQ_blk = dS K
// with dQ reduced into an fp32 accumulator, D and lse_log2 from the
// preprocess kernel (+inf lse_log2 on pad query rows makes the m-tail
// self-masking, bwd_sm90.py:167-172), the K tail masked by the row predicate
// (:967-985), dK scaled once in the epilogue (:930) and dV never scaled.
//
// Blackwell schedule (one CTA per (KV block[, split], head, batch)):
//   warps 0-3  "dS" warpgroup: thread = one KV row; P^T, dS^T, epilogue
//   warps 4-7  "dQ" warpgroup: thread = one query row; drains dQ from TMEM
//              and reduces it into dq_accum with vector fp32 reductions
//   warp  8    tcgen05.mma issuer + TMEM owner
//   warp  9    TMA producer (K/V once, Q/dO double-buffered)
//
//   TMEM (512 columns): S^T [0,128) (P^T bf16 overwrites [0,64); dQ reuses
//   all of it after the dV MMA has read P^T), dP^T [128,256), dV [256,384),
//   dK [384,512).  dS^T goes to shared memory (128B-swizzled, [kv][q]); the
//   dK MMA reads it K-major and the dQ MMA reads the same bytes MN-major.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

namespace bwd {
constexpr int kThreads = 320;
constexpr uint32_t kBoxBytes = 128 * 128;       // 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kBoxBytes;  // 128 rows x 128 bf16
constexpr uint32_t kOffK = 0;
constexpr uint32_t kOffV = kOffK + kTileBytes;
constexpr uint32_t kOffQ = kOffV + kTileBytes;     // 2 stages
constexpr uint32_t kOffdO = kOffQ + 2 * kTileBytes;  // 2 stages
constexpr uint32_t kOffdS = kOffdO + 2 * kTileBytes;
constexpr uint32_t kOffBar = kOffdS + kTileBytes;
constexpr int kBarKvFull = 0;
constexpr int kBarQdoFull = 1;   // + stage
constexpr int kBarQdoEmpty = 3;  // + stage
constexpr int kBarSFull = 5;
constexpr int kBarDpFull = 6;
constexpr int kBarPReady = 7;
constexpr int kBarDsReady = 8;
constexpr int kBarDsEmpty = 9;
constexpr int kBarDqFull = 10;
constexpr int kBarDqDrained = 11;
constexpr int kBarDkvFull = 12;
constexpr int kBarDrain = 13;
constexpr int kNumBars = 14;
constexpr uint32_t kOffTmemHolder = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemHolder + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "backward shared memory exceeds the sm_100 per-CTA limit");
}  // namespace bwd

size_t bwd_smem_bytes() { return bwd::kSmemBytes; }

enum : uint32_t { kRoleDs = 11, kRoleDq = 12, kRoleBwdMma = 13, kRoleBwdLoad = 14, kRoleEpi = 15 };

__device__ __forceinline__ float4 ldg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__global__ void __launch_bounds__(bwd::kThreads, 1)
    wf_bwd_main_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       BwdParams p) {
  using namespace bwd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmemHolder);

  const int warp = (int)warp_id();
  const int lane = (int)lane_id();
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int nb = blockIdx.x % p.n_blocks;
  const int split = blockIdx.x / p.n_blocks;
  const int n0 = nb * 128;
  const int m_begin = split * p.m_chunk;
  const int m_end = min(m_begin + p.m_chunk, p.m_blocks);
  const int cnt = m_end - m_begin;
  if (cnt <= 0) return;  // empty split: nothing to add (uniform for the CTA)
  const size_t bh = (size_t)b * p.h + h;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bar(i), (i == kBarPReady || i == kBarDsReady || i == kBarDqDrained) ? 128u : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 9) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_expect_tx(bar(kBarKvFull), 2 * kTileBytes);
      for (int x = 0; x < 2; ++x) {
        tma_load_4d(sbase + kOffK + x * kBoxBytes, &tm_k, bar(kBarKvFull), x * 64, n0, h, b);
        tma_load_4d(sbase + kOffV + x * kBoxBytes, &tm_v, bar(kBarKvFull), x * 64, n0, h, b);
      }
      int issued[2] = {0, 0};
      for (int u = 0; u < cnt; ++u) {
        const int st = u & 1, use = u >> 1;
        if (use > 0 && !mbar_wait(bar(kBarQdoEmpty + st), (use - 1) & 1, abort_flag, kRoleBwdLoad, 3 + st)) break;
        const int m = (m_begin + u) * 128;
        mbar_expect_tx(bar(kBarQdoFull + st), 2 * kTileBytes);
        for (int x = 0; x < 2; ++x) {
          tma_load_4d(sbase + kOffQ + st * kTileBytes + x * kBoxBytes, &tm_q, bar(kBarQdoFull + st), x * 64, m, h, b);
          tma_load_4d(sbase + kOffdO + st * kTileBytes + x * kBoxBytes, &tm_do, bar(kBarQdoFull + st), x * 64, m, h,
                      b);
        }
        issued[st] = use + 1;
      }
      if (*abort_flag) {
        mbar_wait_drain(bar(kBarKvFull), 0);
        for (int st = 0; st < 2; ++st)
          if (issued[st] > 0) mbar_wait_drain(bar(kBarQdoFull + st), (issued[st] - 1) & 1);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t id_kk = idesc_bf16(128, 128, 0, 0);  // A, B K-major
      constexpr uint32_t id_kb = idesc_bf16(128, 128, 0, 1);  // A K-major (or TMEM), B MN-major
      constexpr uint32_t id_mm = idesc_bf16(128, 128, 1, 1);  // A, B MN-major
      const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;
      const uint32_t sK = sbase + kOffK, sV = sbase + kOffV, sdS = sbase + kOffdS;
      bool ok = mbar_wait(bar(kBarKvFull), 0, abort_flag, kRoleBwdMma, 0);
      tc_fence_after();
      for (int u = 0; u < cnt && ok; ++u) {
        const int st = u & 1;
        const uint32_t sQ = sbase + kOffQ + st * kTileBytes, sdO = sbase + kOffdO + st * kTileBytes;
        if (!(ok = mbar_wait(bar(kBarQdoFull + st), (u >> 1) & 1, abort_flag, kRoleBwdMma, 1 + st))) break;
        tc_fence_after();
        // dP^T = V dO^T  (the dP region was released when dS(u-1) was signalled)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * kBoxBytes + (ks & 3) * 32);
          mma_ss(tdP, sdesc(sV + off, 16, 1024), sdesc(sdO + off, 16, 1024), id_kk, ks > 0);
        }
        mma_commit(bar(kBarDpFull));
        // S^T = K Q^T once dQ(u-1) has left the shared S/dQ columns
        if (u > 0) {
          if (!(ok = mbar_wait(bar(kBarDqDrained), (u - 1) & 1, abort_flag, kRoleBwdMma, 11))) break;
          tc_fence_after();
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * kBoxBytes + (ks & 3) * 32);
          mma_ss(tS, sdesc(sK + off, 16, 1024), sdesc(sQ + off, 16, 1024), id_kk, ks > 0);
        }
        mma_commit(bar(kBarSFull));
        // dV += P^T dO   (P^T from TMEM)
        if (!(ok = mbar_wait(bar(kBarPReady), u & 1, abort_flag, kRoleBwdMma, 7))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts(tdV, tS + ks * 8, sdesc(sdO + ks * 2048, kBoxBytes, 1024), id_kb, (u > 0 || ks > 0) ? 1u : 0u);
        // dK += dS^T Q   (dS^T from smem, K-major)
        if (!(ok = mbar_wait(bar(kBarDsReady), u & 1, abort_flag, kRoleBwdMma, 8))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * kBoxBytes + (ks & 3) * 32);
          mma_ss(tdK, sdesc(sdS + off, 16, 1024), sdesc(sQ + ks * 2048, kBoxBytes, 1024), id_kb,
                 (u > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(bar(kBarQdoEmpty + st));
        // dQ_blk = dS K   (same dS bytes read MN-major), into the S^T columns
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss(tS, sdesc(sdS + ks * 2048, kBoxBytes, 1024), sdesc(sK + ks * 2048, kBoxBytes, 1024), id_mm, ks > 0);
        mma_commit(bar(kBarDqFull));
        mma_commit(bar(kBarDsEmpty));
      }
      if (ok) mma_commit(bar(kBarDkvFull));
      mma_commit(bar(kBarDrain));
      mbar_wait_drain(bar(kBarDrain), 0);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------- dS warpgroup
    const int wq = warp;
    const int r = wq * 32 + lane;  // KV row within the block
    const bool kv_valid = (n0 + r) < p.skv;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base, tdP = tS + 128, tdV = tS + 256, tdK = tS + 384;
    uint8_t* sdS = smem + kOffdS;
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int u = 0; u < cnt; ++u) {
      const size_t row0 = bh * (size_t)p.sq_rounded + (size_t)(m_begin + u) * 128;
      const float* lse_blk = p.lse_log2 + row0;
      const float* d_blk = p.dpsum + row0;
      if (!(ok = mbar_wait(bar(kBarSFull), u & 1, abort_flag, kRoleDs, 5))) break;
      tc_fence_after();
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) reg_fence32(s[c]);
      // P^T = exp2(S^T * scale_log2 - lse_log2[q]); zero on K-tail rows
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 L = ldg_f4(lse_blk + c * 32 + v * 4);
          float pv[4];
          pv[0] = ex2_approx(fmaf(__uint_as_float(s[c][4 * v + 0]), sl2, -L.x));
          pv[1] = ex2_approx(fmaf(__uint_as_float(s[c][4 * v + 1]), sl2, -L.y));
          pv[2] = ex2_approx(fmaf(__uint_as_float(s[c][4 * v + 2]), sl2, -L.z));
          pv[3] = ex2_approx(fmaf(__uint_as_float(s[c][4 * v + 3]), sl2, -L.w));
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (!kv_valid) pv[e] = 0.f;
            s[c][4 * v + e] = __float_as_uint(pv[e]);
          }
          pk[2 * v] = pack_bf16(pv[0], pv[1]);
          pk[2 * v + 1] = pack_bf16(pv[2], pv[3]);
        }
        tmem_st16(tS + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarPReady));
      // dS^T = P^T * (dP^T - D[q])
      if (!(ok = mbar_wait(bar(kBarDpFull), u & 1, abort_flag, kRoleDs, 6))) break;
      tc_fence_after();
      if (u > 0 && !(ok = mbar_wait(bar(kBarDsEmpty), (u - 1) & 1, abort_flag, kRoleDs, 9))) break;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t dp[32];
        tmem_ld32(tdP + c * 32, dp);
        tmem_wait_ld();
        reg_fence32(dp);
        uint32_t pk[16];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 D = ldg_f4(d_blk + c * 32 + v * 4);
          const float d0 = __uint_as_float(s[c][4 * v + 0]) * (__uint_as_float(dp[4 * v + 0]) - D.x);
          const float d1 = __uint_as_float(s[c][4 * v + 1]) * (__uint_as_float(dp[4 * v + 1]) - D.y);
          const float d2 = __uint_as_float(s[c][4 * v + 2]) * (__uint_as_float(dp[4 * v + 2]) - D.z);
          const float d3 = __uint_as_float(s[c][4 * v + 3]) * (__uint_as_float(dp[4 * v + 3]) - D.w);
          pk[2 * v] = pack_bf16(d0, d1);
          pk[2 * v + 1] = pack_bf16(d2, d3);
        }
        // row r of dS^T: q columns [32c, 32c+32) = 4 chunks of 16 B in sub-tile c/2
        uint8_t* sub = sdS + (c >> 1) * kBoxBytes;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint32_t off = sw128_offset((uint32_t)r, (uint32_t)((c & 1) * 4 + v));
          *reinterpret_cast<uint4*>(sub + off) = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(kBarDsReady));
    }
    // ----------------------------------------------------------- epilogue
    if (ok) ok = mbar_wait(bar(kBarDkvFull), 0, abort_flag, kRoleEpi, 12);
    if (ok) {
      tc_fence_after();
      const int kv = n0 + r;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {  // 0 = dV (unscaled), 1 = dK (scaled)
        const uint32_t tsrc = which ? tdK : tdV;
        const float mul = which ? p.scale : 1.f;
        void* dst = which ? p.dk : p.dv;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t a[32];
          tmem_ld32(tsrc + c * 32, a);
          tmem_wait_ld();
          reg_fence32(a);
          if (!p.accum_dkv) {
            if (kv_valid) {
              __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(dst) + (((size_t)b * p.skv + kv) * p.h + h) * 128;
#pragma unroll
              for (int v = 0; v < 4; ++v)
                st_global_v4(row + c * 32 + v * 8,
                             pack_bf16(__uint_as_float(a[8 * v + 0]) * mul, __uint_as_float(a[8 * v + 1]) * mul),
                             pack_bf16(__uint_as_float(a[8 * v + 2]) * mul, __uint_as_float(a[8 * v + 3]) * mul),
                             pack_bf16(__uint_as_float(a[8 * v + 4]) * mul, __uint_as_float(a[8 * v + 5]) * mul),
                             pack_bf16(__uint_as_float(a[8 * v + 6]) * mul, __uint_as_float(a[8 * v + 7]) * mul));
            }
          } else {
            float* tile = reinterpret_cast<float*>(dst) + (bh * (size_t)p.n_blocks + nb) * 16384 + (size_t)r * 4;
#pragma unroll
            for (int g = 0; g < 8; ++g)
              red_add_v4(tile + (size_t)(c * 8 + g) * 512, __uint_as_float(a[4 * g + 0]) * mul,
                         __uint_as_float(a[4 * g + 1]) * mul, __uint_as_float(a[4 * g + 2]) * mul,
                         __uint_as_float(a[4 * g + 3]) * mul);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------- dQ warpgroup
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // query row within the block
    const uint32_t tQ = tmem + ((uint32_t)(wq * 32) << 16);
    for (int u = 0; u < cnt; ++u) {
      if (!mbar_wait(bar(kBarDqFull), u & 1, abort_flag, kRoleDq, 10)) break;
      tc_fence_after();
      uint32_t q[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tQ + c * 32, q[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) reg_fence32(q[c]);
      tc_fence_before();
      mbar_arrive(bar(kBarDqDrained));
      float* tile = p.dq_accum + (bh * (size_t)p.m_blocks + (m_begin + u)) * 16384 + (size_t)r * 4;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int g = 0; g < 8; ++g)
          red_add_v4(tile + (size_t)(c * 8 + g) * 512, __uint_as_float(q[c][4 * g + 0]),
                     __uint_as_float(q[c][4 * g + 1]), __uint_as_float(q[c][4 * g + 2]),
                     __uint_as_float(q[c][4 * g + 3]));
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tmem, 512);
}

}  // namespace wf
