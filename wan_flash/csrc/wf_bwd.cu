// Backward main kernel for B200 (sm_100a): dK/dV-stationary, tcgen05 MMAs
// accumulating S^T, dP^T, dV, dK and dQ in tensor memory.
//
// Computes what the reference backward main kernel computes
// (wan_flash/bwd_sm90.py of Quarky93/wan-flash, `_mma_m_block` :947-1046):
// for one 128-row KV block it walks the query blocks and forms
//     S^T  = K Q^T                      P^T = exp2(S^T * scale_log2 - lse * log2(e))
//     dP^T = V dO^T                     dS^T = P^T * (dP^T - D)
//     dV  += P^T dO                     dK  += dS^T Q         dQ_blk = dS K
// with dQ reduced into an fp32 accumulator, D and lse_log2 from the
// preprocess kernel (stored negated: -inf on pad query rows makes the m-tail
// self-masking, as the +inf lse_log2 sentinel of bwd_sm90.py:167-172), the K tail masked by a row predicate
// (:967-985), dK scaled once in the epilogue (:930) and dV never scaled.
//
// Blackwell schedule (one CTA per (KV block[, split], head, batch)):
//   warps 0-3   elementwise WG A: thread = one KV row, query columns [0, 64)
//   warps 4-7   elementwise WG B: thread = one KV row, query columns [64, 128)
//   warps 8-11  dQ WG: thread = one query row; drains dQ from TMEM and
//               reduces it into dq_accum with bulk async reductions staged
//               through a dedicated buffer
//   warp  12    tcgen05.mma issuer + TMEM owner
//   warp  13    TMA producer (K/V once; Q, -lse*log2(e), D double-buffered;
//               dO single-buffered, refilled between dV(u) and dP(u+1))
//   warps 14-15 idle (complete warpgroup 3 so it can give registers back)
//
//   TMEM (512 columns): S^T [0,128) -- P^T (bf16) overwrites [0,32) (WG A)
//   and [64,96) (WG B), each inside the columns that WG has already read;
//   dP^T [128,256) -- dS^T (bf16) overwrites it the same way as the A operand
//   of the dK MMA, and dQ reuses all of it once dK has read dS^T; dV
//   [256,384); dK [384,512).  dS^T also goes to shared memory (128B-swizzled,
//   [kv][q]), read MN-major by the dQ MMA.
//   A separate 32 KB buffer stages dQ for the bulk reductions.
//
//   MMA order for query block u:  dV(u)  S(u+1)  dK(u)  dQ(u)  dP(u+1)
//   (dV and dK take their A operand from TMEM; S, dP and dQ read both from
//   shared memory)
//   S(u+1) only needs dV(u) to have read P^T(u) (in-order tensor pipe), so
//   the next exponentials start while dK/dQ of this block run; dP(u+1)
//   waits for the dQ warpgroup to have read dQ(u) out of the dP columns.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

namespace bwd {
constexpr int kThreads = 512;
// register split (launch: 512 x 128 = 65536):
//   2 elementwise WGs 128 x 152 + dQ WG 128 x 152 + WG3 128 x 56 = 65536
constexpr uint32_t kRegsEw = 152;
constexpr uint32_t kRegsDq = 152;
constexpr uint32_t kRegsOther = 56;
constexpr uint32_t kBoxBytes = 128 * 128;       // 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kBoxBytes;  // 128 rows x 128 bf16
constexpr uint32_t kOffK = 0;
constexpr uint32_t kOffV = kOffK + kTileBytes;
constexpr uint32_t kOffQ = kOffV + kTileBytes;       // 2 stages
constexpr uint32_t kOffdO = kOffQ + 2 * kTileBytes;  // 1 stage (free after dV, refilled before dP)
constexpr uint32_t kOffdS = kOffdO + kTileBytes;
constexpr uint32_t kOffX = kOffdS + kTileBytes;      // dQ staging for the bulk reductions (32 KB)
constexpr uint32_t kOffLse = kOffX + kTileBytes;     // 2 stages x 128 fp32 (-lse * log2 e)
constexpr uint32_t kOffD = kOffLse + 2 * 512;        // 2 stages x 128 fp32
constexpr uint32_t kOffBar = kOffD + 2 * 512;
constexpr int kBarKvFull = 0;
constexpr int kBarQFull = 1;     // + stage (with -lse*log2e and D of the block)
constexpr int kBarQEmpty = 3;    // + stage
constexpr int kBarDoFull = 5;
constexpr int kBarDoEmpty = 6;
constexpr int kBarSFull = 7;
constexpr int kBarDpFull = 8;
constexpr int kBarPReady = 9;
constexpr int kBarDsReady = 10;
constexpr int kBarDsEmpty = 11;
constexpr int kBarDqFull = 12;
constexpr int kBarDqDrained = 13;
constexpr int kBarDkvFull = 14;
constexpr int kBarDrain = 15;
constexpr int kBarXchgFull = 16;   // the dQ warpgroup has written a half-tile into the staging buffer
constexpr int kBarXchgDone = 17;   // the staging buffer is free again (previous bulk read done)
constexpr int kBarEpiGo = 18;      // deterministic split-M: earlier splits have added their dK/dV
constexpr int kBarEpiDone = 19;    // deterministic split-M: this CTA's dK/dV reductions are issued
constexpr int kNumBars = 20;
constexpr uint32_t kOffTmemHolder = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemHolder + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemLimit = 232448;  // sm_100 opt-in maximum per CTA
// Request what fits: the base is re-aligned to 1024 B at run time and the
// kernel checks that the aligned layout still fits (it normally needs no pad).
constexpr uint32_t kSmemBytes = (kSmemUsed + 1024 <= kSmemLimit) ? kSmemUsed + 1024 : kSmemLimit;
static_assert(kSmemUsed <= kSmemLimit, "backward shared memory exceeds the sm_100 per-CTA limit");
}  // namespace bwd

size_t bwd_smem_bytes() { return bwd::kSmemBytes; }

enum : uint32_t { kRoleEw = 11, kRoleDq = 12, kRoleBwdMma = 13, kRoleBwdLoad = 14, kRoleEpi = 15 };

__device__ __forceinline__ uint32_t dynamic_smem_size() {
  uint32_t r;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}

__global__ void __launch_bounds__(bwd::kThreads, 1)
    wf_bwd_main_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       BwdParams p) {
  using namespace bwd;
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  uint8_t* smem = reinterpret_cast<uint8_t*>((raw + 1023) & ~uintptr_t(1023));
  if ((uint32_t)(reinterpret_cast<uintptr_t>(smem) - raw) + kSmemUsed > dynamic_smem_size()) {
    // the aligned layout does not fit: report and leave (uniform for the CTA)
    if (threadIdx.x == 0) atomicCAS(&g_err_code, 0u, (unsigned)WF_ERR_SMEM_ALIGN);
    return;
  }
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
  // The CTAs of a head resident at the same time walk the same Q/dO tiles
  // together, so each tile is fetched from HBM about once and served to the
  // others from L2.  Successive waves (one CTA per SM, `p.wave` CTAs) walk in
  // alternating directions: a wave starts on the query blocks whose Q/dO
  // tiles and dQ accumulator lines the previous wave touched last, which are
  // still in L2.  (A walk rotated by the KV block index, spreading the dQ
  // reductions over more lines, measured 1-2 % slower.)  Deterministic mode
  // walks every CTA forwards: it relies on KV block nb meeting each query
  // block just after KV block nb-1.  A CTA's direction depends only on its
  // grid position, so dK/dV stay bitwise reproducible at nsplit = 1.
  const unsigned lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const bool reverse = !p.deterministic && p.wave > 0 && ((lin / (unsigned)p.wave) & 1u);
  auto qblock = [&](int u) -> int { return reverse ? m_end - 1 - u : m_begin + u; };
  if (cnt <= 0) return;  // empty split: nothing to add (uniform for the CTA)
  const size_t bh = (size_t)b * p.h + h;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      // per-thread arrivals (measured faster here than one arrival per warp)
      const bool ew = (i == kBarPReady || i == kBarDsReady);
      const uint32_t count = (ew || i == kBarEpiDone) ? 256u
                             : (i == kBarDqDrained || i == kBarXchgDone || i == kBarXchgFull) ? 128u : 1u;
      mbar_init(bar(i), count);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 12) {
    tmem_alloc(smem_u32(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // Launched as a programmatic dependent of the preprocess: q, k, v, dO were
  // complete before it started, so barrier set-up, TMEM allocation and the
  // K/V loads overlap its tail; -lse*log2(e), D and the zeroed dQ
  // accumulator are touched only after griddep_wait() (the TMA producer,
  // before the first -lse/D load; the dQ reducing thread, before its first
  // reduction).  The convert that follows may be scheduled early too.
  griddep_launch_dependents();

  if (warp >= 14) {
    regs_dec<kRegsOther>();  // idle warps of warpgroup 3
  } else if (warp == 13) {
    regs_dec<kRegsOther>();
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
      griddep_wait();  // the preprocess has written -lse*log2(e) and D
      int issued0 = 0, issued1 = 0, issued_do = 0;  // completed uses per buffer (for the abort drain)
      for (int u = 0; u < cnt; ++u) {
        const int st = u & 1, use = u >> 1;
        const int m = qblock(u);
        if (use > 0 && !mbar_wait(bar(kBarQEmpty + st), (use - 1) & 1, abort_flag, kRoleBwdLoad, 3 + st)) break;
        const uint32_t qfull = bar(kBarQFull + st);
        mbar_expect_tx(qfull, kTileBytes + 1024);
        for (int x = 0; x < 2; ++x)
          tma_load_4d(sbase + kOffQ + st * kTileBytes + x * kBoxBytes, &tm_q, qfull, x * 64, m * 128, h, b);
        const size_t row0 = bh * (size_t)p.sq_rounded + (size_t)m * 128;
        bulk_load(sbase + kOffLse + st * 512, p.neg_lse_log2 + row0, 512, qfull);
        bulk_load(sbase + kOffD + st * 512, p.dpsum + row0, 512, qfull);
        if (st) issued1 = use + 1; else issued0 = use + 1;
        // dO has one buffer: refill it once dV of the previous block has read it
        if (u > 0 && !mbar_wait(bar(kBarDoEmpty), (u - 1) & 1, abort_flag, kRoleBwdLoad, 6)) break;
        mbar_expect_tx(bar(kBarDoFull), kTileBytes);
        for (int x = 0; x < 2; ++x)
          tma_load_4d(sbase + kOffdO + x * kBoxBytes, &tm_do, bar(kBarDoFull), x * 64, m * 128, h, b);
        issued_do = u + 1;
      }
      if (*abort_flag) {
        mbar_wait_drain(bar(kBarKvFull), 0);
        if (issued0 > 0) mbar_wait_drain(bar(kBarQFull + 0), (issued0 - 1) & 1);
        if (issued1 > 0) mbar_wait_drain(bar(kBarQFull + 1), (issued1 - 1) & 1);
        if (issued_do > 0) mbar_wait_drain(bar(kBarDoFull), (issued_do - 1) & 1);
      }
    }
  } else if (warp == 12) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ MMA
    // (converged warp: every lane computes descriptors and waits, one
    // elected lane issues each tcgen05 instruction)
    {
      constexpr uint32_t id_kk = idesc_bf16(128, 128, 0, 0);  // A, B K-major
      constexpr uint32_t id_kb = idesc_bf16(128, 128, 0, 1);  // A K-major (or TMEM), B MN-major
      constexpr uint32_t id_mm = idesc_bf16(128, 128, 1, 1);  // A, B MN-major
      const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;
      // K-major operand descriptors advance 32 B per 16-element K step inside
      // a 64-column box and 16 KB to the next box; MN-major ones use the 16 KB
      // box stride as LBO and advance 2 KB per 16 rows of K (desc_add adds
      // the offset to the encoded start-address field).
      const uint64_t dK_k = sdesc(sbase + kOffK, 16, 1024);
      const uint64_t dV_k = sdesc(sbase + kOffV, 16, 1024);
      const uint64_t dK_mn = sdesc(sbase + kOffK, kBoxBytes, 1024);
      const uint64_t dS_mn = sdesc(sbase + kOffdS, kBoxBytes, 1024);
      auto koff = [](int ks) -> uint32_t { return (uint32_t)((ks >> 2) * kBoxBytes + (ks & 3) * 32); };
      auto moff = [](int ks) -> uint32_t { return (uint32_t)(ks * 2048); };
      auto issue_s = [&](int st) {  // S^T = K Q^T
        const uint64_t q_k = sdesc(sbase + kOffQ + st * kTileBytes, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) mma_ss_e(tS, desc_add(dK_k, koff(ks)), desc_add(q_k, koff(ks)), id_kk, ks > 0);
        mma_commit_e(bar(kBarSFull));
      };
      const uint64_t do_k = sdesc(sbase + kOffdO, 16, 1024);
      const uint64_t do_mn = sdesc(sbase + kOffdO, kBoxBytes, 1024);
      auto issue_dp = [&]() {  // dP^T = V dO^T
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) mma_ss_e(tdP, desc_add(dV_k, koff(ks)), desc_add(do_k, koff(ks)), id_kk, ks > 0);
        mma_commit_e(bar(kBarDpFull));
      };
      bool ok = mbar_wait_warp(bar(kBarKvFull), 0, abort_flag, kRoleBwdMma, 0) &&
                mbar_wait_warp(bar(kBarQFull + 0), 0, abort_flag, kRoleBwdMma, 1) &&
                mbar_wait_warp(bar(kBarDoFull), 0, abort_flag, kRoleBwdMma, 5);
      if (ok) {
        tc_fence_after();
        issue_dp();
        issue_s(0);
      }
      for (int u = 0; u < cnt && ok; ++u) {
        const int st = u & 1;
        // dV += P^T dO   (P^T from TMEM: query 0-63 in columns [0,32), 64-127 in [64,96))
        if (!(ok = mbar_wait_warp(bar(kBarPReady), u & 1, abort_flag, kRoleBwdMma, 7))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts_e(tdV, tS + (ks >> 2) * 64 + (ks & 3) * 8, desc_add(do_mn, moff(ks)), id_kb, (u > 0 || ks > 0) ? 1u : 0u);
        mma_commit_e(bar(kBarDoEmpty));  // dO(u) is read by dP(u) and dV(u) only
        // S^T(u+1): the S columns are free once dV(u) has read P^T(u)
        if (u + 1 < cnt) {
          if (!(ok = mbar_wait_warp(bar(kBarQFull + ((u + 1) & 1)), ((u + 1) >> 1) & 1, abort_flag, kRoleBwdMma, 1)))
            break;
          tc_fence_after();
          issue_s((u + 1) & 1);
        }
        // dK += dS^T Q   (dS^T from TMEM: query 0-63 in dP columns [0,32), 64-127 in [64,96))
        if (!(ok = mbar_wait_warp(bar(kBarDsReady), u & 1, abort_flag, kRoleBwdMma, 8))) break;
        tc_fence_after();
        const uint64_t q_mn = sdesc(sbase + kOffQ + st * kTileBytes, kBoxBytes, 1024);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts_e(tdK, tdP + (ks >> 2) * 64 + (ks & 3) * 8, desc_add(q_mn, moff(ks)), id_kb, (u > 0 || ks > 0) ? 1u : 0u);
        mma_commit_e(bar(kBarQEmpty + st));
        // dQ_blk = dS K   (same dS bytes read MN-major) into the dP^T columns
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) mma_ss_e(tdP, desc_add(dS_mn, moff(ks)), desc_add(dK_mn, moff(ks)), id_mm, ks > 0);
        mma_commit_e(bar(kBarDqFull));
        mma_commit_e(bar(kBarDsEmpty));
        // dP^T(u+1) once dQ(u) has been read out of those columns and dO(u+1) is in
        if (u + 1 < cnt) {
          if (!(ok = mbar_wait_warp(bar(kBarDqDrained), u & 1, abort_flag, kRoleBwdMma, 11))) break;
          if (!(ok = mbar_wait_warp(bar(kBarDoFull), (u + 1) & 1, abort_flag, kRoleBwdMma, 5))) break;
          tc_fence_after();
          issue_dp();
        }
      }
      if (ok) mma_commit_e(bar(kBarDkvFull));
      mma_commit_e(bar(kBarDrain));
      mbar_wait_drain(bar(kBarDrain), 0);
    }
  } else if (warp < 8) {
    regs_inc<kRegsEw>();
    // ---------------------------------------------- elementwise warpgroups
    const int half = warp >> 2;   // 0: query columns [0,64), 1: [64,128)
    const int wq = warp & 3;      // TMEM lane quadrant: KV rows [32 wq, 32 wq + 32)
    // S^T and dP^T are read 16 lanes at a time (16x256b): thread t holds KV
    // rows 32 wq + 16 g + 8 e + t/4 (g, e in {0, 1}) and, in repetition j,
    // query columns 64 half + 8 j + 2 (t%4) + {0, 1}.  Four threads share a
    // row and eight column pairs a warp, so the per-column -lse*log2(e) and D
    // are 16 shared-memory values per thread per block (32 when each thread
    // owned a whole 64-column row).
    const int tq = lane & 3;
    const int tr = lane >> 2;
    auto kv_row = [&](int g, int e) -> int { return wq * 32 + 16 * g + 8 * e + tr; };
    bool kv_ok[2][2];
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int e = 0; e < 2; ++e) kv_ok[g][e] = (n0 + kv_row(g, e)) < p.skv;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    constexpr uint32_t kLane16 = 16u << 16;
    const uint32_t tS = tmem + lane_base + (uint32_t)(half * 64);
    const uint32_t tdP = tmem + lane_base + 128u + (uint32_t)(half * 64);
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    const uint32_t sdS = sbase + kOffdS + (uint32_t)half * kBoxBytes;
    bool ok = true;
    for (int u = 0; u < cnt; ++u) {
      const int st = u & 1;
      const float* snl = reinterpret_cast<const float*>(smem + kOffLse + st * 512) + half * 64 + 2 * tq;
      const float* sD = reinterpret_cast<const float*>(smem + kOffD + st * 512) + half * 64 + 2 * tq;
      if (!(ok = mbar_wait(bar(kBarSFull), u & 1, abort_flag, kRoleEw, 5))) break;
      // -lse*log2(e) / D of this block arrived with Q/dO (already complete; this
      // wait makes the bulk-copied bytes visible to these threads)
      if (!(ok = mbar_wait(bar(kBarQFull + st), (u >> 1) & 1, abort_flag, kRoleEw, 1))) break;
      tc_fence_after();
      uint32_t s[2][32];
      tmem_ld_16x256b_x8(tS, s[0]);
      tmem_ld_16x256b_x8(tS + kLane16, s[1]);
      uint64_t nl[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 L = *reinterpret_cast<const float2*>(snl + 8 * j);
        nl[j] = f2_pack(L.x, L.y);
      }
      tmem_wait_ld();
      reg_fence32(s[0]);
      reg_fence32(s[1]);
      // P^T = 2^(S^T * scale_log2 + neg_lse_log2[q]) on the MUFU pipe; rows past
      // the K tail are zeroed.  P^T goes back to TMEM as bf16 pairs over the
      // already-read S^T columns (packed column 64 half + 4 j + t%4).
      uint64_t pp[2][16];
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[g][4 * j + 2 * e]), __uint_as_float(s[g][4 * j + 2 * e + 1])),
                                      sl2x2, nl[j]);
            pp[g][2 * j + e] = exp2_mufu2(x);
            float p0, p1;
            f2_unpack(pp[g][2 * j + e], p0, p1);
            pk[2 * j + e] = kv_ok[g][e] ? pack_bf16(p0, p1) : 0u;
          }
        tmem_st_16x128b_x8(tS + (g ? kLane16 : 0u), pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarPReady));
      // dS^T = P^T * (dP^T - D[q])
      if (!(ok = mbar_wait(bar(kBarDpFull), u & 1, abort_flag, kRoleEw, 6))) break;
      tc_fence_after();
      uint32_t dp[2][32];
      tmem_ld_16x256b_x8(tdP, dp[0]);
      tmem_ld_16x256b_x8(tdP + kLane16, dp[1]);
      tmem_wait_ld();
      reg_fence32(dp[0]);
      reg_fence32(dp[1]);
      tc_fence_before();  // the dP columns are read; dQ(u) may overwrite them after dS_ready
      if (u > 0 && !(ok = mbar_wait(bar(kBarDsEmpty), (u - 1) & 1, abort_flag, kRoleEw, 9))) break;
      const uint64_t m1x2 = f2_pack(-1.f, -1.f);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 D = *reinterpret_cast<const float2*>(sD + 8 * j);
          const uint64_t d2 = f2_pack(D.x, D.y);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const uint64_t dpp = f2_pack(__uint_as_float(dp[g][4 * j + 2 * e]), __uint_as_float(dp[g][4 * j + 2 * e + 1]));
            float d0, d1;
            f2_unpack(f2_mul(pp[g][2 * j + e], f2_fma(d2, m1x2, dpp)), d0, d1);
            pk[2 * j + e] = kv_ok[g][e] ? pack_bf16(d0, d1) : 0u;
            // row of dS^T in shared memory for the dQ MMA (128B-swizzled
            // [kv][q] box of this half): 4 bytes of the 16-byte chunk j
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + sw128_offset((uint32_t)kv_row(g, e), (uint32_t)j) +
                                                          4u * (uint32_t)tq),
                         "r"(pk[2 * j + e])
                         : "memory");
          }
        }
        // dS^T as the A operand of the dK MMA: bf16 pairs over this
        // warpgroup's (already read) dP^T columns
        tmem_st_16x128b_x8(tdP + (g ? kLane16 : 0u), pk);
      }
      fence_proxy_async_smem();
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarDsReady));
    }
    // the epilogue reads dV / dK rows 32 x 32b: thread = one KV row
    const int r = wq * 32 + lane;
    const bool kv_valid = (n0 + r) < p.skv;
    // ----------------------------------------------------------- epilogue
    // WG A writes dV (unscaled), WG B writes dK (scaled by softmax_scale)
    if (ok) ok = mbar_wait(bar(kBarDkvFull), 0, abort_flag, kRoleEpi, 12);
    const bool ordered = p.accum_dkv && p.deterministic;
    int* kv_sem = ordered ? p.dkv_sem + bh * (size_t)p.n_blocks + nb : nullptr;
    if (ok && ordered) {
      // splits 0..split-1 add their dK/dV for this KV block first
      if (threadIdx.x == 0) {
        if (counter_wait_eq(kv_sem, split, abort_flag, kRoleEpi, 20)) mbar_arrive(bar(kBarEpiGo));
      }
      ok = mbar_wait(bar(kBarEpiGo), 0, abort_flag, kRoleEpi, 18);
    }
    if (ok) {
      tc_fence_after();
      const int kv = n0 + r;
      const uint32_t tsrc = tmem + lane_base + (half ? 384u : 256u);
      const float mul = half ? p.scale : 1.f;
      void* dst = half ? p.dk : p.dv;
#pragma unroll
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
          float* tile = reinterpret_cast<float*>(dst) + (bh * (size_t)p.n_blocks + nb) * 16384 +
                        (size_t)(r >> 6) * 8192 + (size_t)(r & 63) * 4;
#pragma unroll
          for (int g = 0; g < 8; ++g)
            red_add_v4(tile + (size_t)(c * 8 + g) * 256, __uint_as_float(a[4 * g + 0]) * mul,
                       __uint_as_float(a[4 * g + 1]) * mul, __uint_as_float(a[4 * g + 2]) * mul,
                       __uint_as_float(a[4 * g + 3]) * mul);
        }
      }
      if (ordered) {
        __threadfence();
        mbar_arrive(bar(kBarEpiDone));
        if (threadIdx.x == 0 && mbar_wait(bar(kBarEpiDone), 0, abort_flag, kRoleEpi, 19)) {
          __threadfence();
          st_release_gpu(kv_sem, split + 1);
        }
      }
    }
  } else {
    regs_inc<kRegsDq>();
    // ------------------------------------------------------- dQ warpgroup
    // dQ(u) leaves TMEM into registers (then the dP^T columns are free for
    // dP(u+1)), goes through a dedicated 32 KB staging buffer in two column
    // halves and is reduced into dq_accum by two bulk cp.reduce.async per
    // half (the accumulator's 128-row tile is [2 row halves][32 groups of 4
    // columns][64 rows][4], so one column half of one row half is 16
    // contiguous KB).  The bulk engine, not the per-SMSP
    // load/store pipe, carries the reduction, which keeps that pipe free for
    // the TMEM, shared-memory and mbarrier traffic of the other warps.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // query row within the block
    const uint32_t tQ = tmem + ((uint32_t)(wq * 32) << 16) + 128u;  // dQ lives in the dP^T columns
    const uint32_t sx = sbase + kOffX;
    uint8_t* xb = smem + kOffX;
    const bool leader = (threadIdx.x == 256);
    if (leader) griddep_wait();  // the preprocess has zeroed dq_accum
    int* const q_sem = p.deterministic ? p.dq_sem + bh * (size_t)p.m_blocks : nullptr;
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
      float* tile = p.dq_accum + (bh * (size_t)p.m_blocks + qblock(u)) * 16384;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        // the staging buffer is free once the previous bulk reduction has read it
        if (leader) bulk_wait_read_all();
        mbar_arrive(bar(kBarXchgDone));
        if (!mbar_wait(bar(kBarXchgDone), (2 * u + half) & 1, abort_flag, kRoleDq, 16)) break;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc)
#pragma unroll
          for (int g = 0; g < 8; ++g)
            *reinterpret_cast<uint4*>(xb + (((r >> 6) * 16 + cc * 8 + g) * 64 + (r & 63)) * 16) =
                make_uint4(q[2 * half + cc][4 * g + 0], q[2 * half + cc][4 * g + 1], q[2 * half + cc][4 * g + 2],
                           q[2 * half + cc][4 * g + 3]);
        fence_proxy_async_smem();
        mbar_arrive(bar(kBarXchgFull));
        if (leader) {
          if (!mbar_wait(bar(kBarXchgFull), (2 * u + half) & 1, abort_flag, kRoleDq, 15)) break;
          if (q_sem != nullptr && half == 0) {
            // KV blocks 0..nb-1 add their contributions to this query block first
            if (!counter_wait_eq(q_sem + qblock(u), nb, abort_flag, kRoleDq, 20)) break;
            fence_proxy_async_global();
          }
          bulk_reduce_add_f32(tile + half * 4096, sx, 16384);
          bulk_reduce_add_f32(tile + 8192 + half * 4096, sx + 16384, 16384);
          bulk_commit_group();
          if (q_sem != nullptr && half == 1) {
            bulk_wait_all();  // the reductions have landed in global memory
            fence_proxy_async_global();
            st_release_gpu(q_sem + qblock(u), nb + 1);
          }
        }
      }
      if (*abort_flag) break;
    }
    if (leader) bulk_wait_all();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 12) tmem_dealloc(tmem, 512);
}

}  // namespace wf
