// Backward main kernel, CTA-pair form (cluster of 2, tcgen05 cta_group::2).
//
// Same mathematics as wf_bwd_main_kernel (wf_bwd.cu) and the reference main
// kernel (wan_flash/bwd_sm90.py of Quarky93/wan-flash, `_mma_m_block`
// :947-1046): for a KV tile walk the query blocks and form
//     S^T  = K Q^T                      P^T = exp2(S^T * scale_log2 - lse * log2(e))
//     dP^T = V dO^T                     dS^T = P^T * (dP^T - D)
//     dV  += P^T dO                     dK  += dS^T Q         dQ_blk = dS K
// The reference's `cluster_n = 2` pairs adjacent KV blocks of a head and
// multicasts Q/dO into both CTAs (features.py:55-70).  Here the pair shares
// the work instead of the loads: one thread of the leader CTA issues 2-SM
// MMAs over the pair's 256 KV rows, so
//   * S^T, dP^T, dV, dK are M = 256 MMAs: each CTA supplies its own 128 KV
//     rows of A (K, V from smem; P^T, dS^T from its TMEM) and HALF of the B
//     operand (Q / dO: 64 query rows for S^T and dP^T, 64 head-dim columns
//     for dK and dV), so each SM reads half of every Q / dO tile from shared
//     memory;
//   * dQ = dS K is one M = 128 MMA over K = 256 KV rows: CTA r supplies query
//     rows [64r, 64r+64) of dS (both KV halves: the peer writes its half of
//     dS into this CTA's shared memory) and head-dim columns [64r, 64r+64) of
//     K, and receives dQ rows [64r, 64r+64) in TMEM.  The pair therefore
//     reduces ONE dQ partial per 256 KV rows into the fp32 accumulator, half
//     the reduction traffic of two independent CTAs.
//
// Roles per CTA (512 threads; both CTAs run every role except the MMA issue):
//   warps 0-3   elementwise WG A: thread = one KV row, query columns [0, 64)
//   warps 4-7   elementwise WG B: thread = one KV row, query columns [64, 128)
//   warps 8-11  dQ WG: drains this CTA's 64 dQ rows (lane l holds row l%64,
//               head-dim half l/64) and reduces them with two 16 KB bulk
//               reductions per query block
//   warp  12    TMEM owner (both CTAs); MMA issuer (leader CTA only)
//   warp  13    TMA producer A: K, V, the pair's K half; Q / dO query-row
//               halves (S^T, dP^T operands); lse / D
//   warp  14    dS exchange: one bulk shared::cta -> shared::cluster copy per
//               query block of the dS rows the peer's dQ MMA needs
//   warp  15    TMA producer B: Q / dO head-dim halves (dK, dV operands)
//
// dS exchange: the elementwise warpgroup whose query columns belong to the
// peer writes its dS rows into a local 16 KB staging buffer (plain stores),
// and warp 14 moves the block with one asynchronous bulk copy that completes
// on the peer's mbarrier.  The leader's dQ MMA waits for its own incoming
// block and, through a relay arrival from the peer's warp 14, for the
// peer's; dK only waits for dS^T in TMEM.
//
// Synchronisation: the leader's MMA thread waits on leader-side mbarriers
// that count both CTAs -- TMA bytes of both CTAs (cta_group::2 loads signal
// the leader's barrier; the leader arms it with the total), and per-warp
// release.cluster arrivals of both CTAs' elementwise / dQ warps.  MMA
// completions are committed to the same barrier offset in both CTAs.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

namespace bwd2 {
constexpr int kThreads = 512;
constexpr uint32_t kRegsEw = 152;
constexpr uint32_t kRegsDq = 152;
constexpr uint32_t kRegsOther = 56;
constexpr uint32_t kBox = 128 * 128;     // 128 rows x 64 bf16 (one swizzle-128 box)
constexpr uint32_t kHalfBox = 64 * 128;  // 64 rows x 64 bf16
// shared memory (identical offsets in both CTAs of the pair)
constexpr uint32_t kOffK = 0;                      // own 128 KV rows of K, d [0,64) | [64,128)   (S^T A)
constexpr uint32_t kOffV = kOffK + 2 * kBox;       // own 128 KV rows of V                       (dP^T A)
constexpr uint32_t kOffKd = kOffV + 2 * kBox;      // the pair's 256 K rows, this CTA's d-half   (dQ B)
constexpr uint32_t kOffQk = kOffKd + 2 * kBox;     // Q, this CTA's 64 query rows, all d         (S^T B)
constexpr uint32_t kOffQn = kOffQk + 2 * kHalfBox; // Q, 128 query rows, this CTA's d-half       (dK B)
constexpr uint32_t kOffOk = kOffQn + kBox;         // dO, this CTA's 64 query rows, all d        (dP^T B)
constexpr uint32_t kOffOn = kOffOk + 2 * kHalfBox; // dO, 128 query rows, this CTA's d-half      (dV B)
constexpr uint32_t kOffdS = kOffOn + kBox;         // dS, 256 KV rows x this CTA's 64 query cols (dQ A)
constexpr uint32_t kOffX = kOffdS + 2 * kBox;      // dQ staging, one head-dim half: [16 groups][64 rows][4] fp32
constexpr uint32_t kOffDso = kOffX + 16384;        // outgoing dS rows for the peer: [128 KV rows][64 q cols] bf16
constexpr uint32_t kOffLse = kOffDso + 16384;      // 2 stages x 128 fp32 (-lse * log2 e)
constexpr uint32_t kOffD = kOffLse + 2 * 512;      // 2 stages x 128 fp32
constexpr uint32_t kOffBar = kOffD + 2 * 512;
// leader-side barriers (only the leader's copies are used)
constexpr int kBarKvFull = 0;
constexpr int kBarQkFull = 1;
constexpr int kBarQnFull = 2;
constexpr int kBarOkFull = 3;
constexpr int kBarOnFull = 4;
constexpr int kBarPReady = 5;     // 16 warps (8 per CTA)
constexpr int kBarDsReady = 6;    // 16 warps
constexpr int kBarDqDrained = 7;  // 8 warps (4 per CTA)
// barriers in both CTAs, arrived by MMA commits to the pair
constexpr int kBarQkEmpty = 8;
constexpr int kBarQnEmpty = 9;
constexpr int kBarOkEmpty = 10;
constexpr int kBarOnEmpty = 11;
constexpr int kBarSFull = 12;
constexpr int kBarDpFull = 13;
constexpr int kBarDsEmpty = 14;
constexpr int kBarDqFull = 15;
constexpr int kBarDkvFull = 16;
// local barriers
constexpr int kBarLseFull = 17;   // + stage
constexpr int kBarLseEmpty = 19;  // + stage, 8 warps
constexpr int kBarXFull = 21;     // 4 dQ warps
constexpr int kBarXFree = 22;     // 4 dQ warps
constexpr int kBarDrain = 23;
constexpr int kBarDsIn = 24;      // incoming dS rows from the peer (bulk-copy bytes)
constexpr int kBarDsInPeer = 25;  // leader only: the peer's incoming block has landed (relay)
constexpr int kBarDsoFull = 26;   // 4 warps of the warpgroup that writes the outgoing rows
constexpr int kNumBars = 27;
constexpr uint32_t kOffTmemHolder = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemHolder + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemLimit = 232448;
constexpr uint32_t kSmemBytes = (kSmemUsed + 1024 <= kSmemLimit) ? kSmemUsed + 1024 : kSmemLimit;
static_assert(kSmemUsed <= kSmemLimit, "pair backward shared memory exceeds the sm_100 per-CTA limit");
constexpr uint16_t kPairMask = 0x3;
}  // namespace bwd2

size_t bwd2_smem_bytes() { return bwd2::kSmemBytes; }

enum : uint32_t { kRoleEw2 = 21, kRoleDq2 = 22, kRoleMma2 = 23, kRoleLoad2 = 24, kRoleEpi2 = 25, kRoleEx2 = 26 };

__device__ __forceinline__ uint32_t dyn_smem_size2() {
  uint32_t r;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}

__global__ void __launch_bounds__(bwd2::kThreads, 1)
    wf_bwd2_main_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_q64,
                        const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_do64,
                        BwdParams p) {
  using namespace bwd2;
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  uint8_t* smem = reinterpret_cast<uint8_t*>((raw + 1023) & ~uintptr_t(1023));
  if ((uint32_t)(reinterpret_cast<uintptr_t>(smem) - raw) + kSmemUsed > dyn_smem_size2()) {
    // the aligned layout does not fit (same for both CTAs of the pair)
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
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int n_pairs = (p.n_blocks + 1) >> 1;
  const int pair = (int)(blockIdx.x >> 1) % n_pairs;
  const int split = (int)(blockIdx.x >> 1) / n_pairs;
  const int pair_n0 = pair * 256;
  const int n0 = pair_n0 + 128 * (int)rank;  // this CTA's KV rows
  const int m_begin = split * p.m_chunk;
  const int m_end = min(m_begin + p.m_chunk, p.m_blocks);
  const int cnt = m_end - m_begin;
  // Query-block order, rotated per KV tile: CTAs that run at the same time
  // then load different Q/dO tiles and reduce into different dQ tiles,
  // instead of every resident CTA of a head hitting the same L2 lines.
  const int rot = cnt > 0 ? pair % cnt : 0;
  auto qblock = [&](int u) -> int { int j = u + rot; return m_begin + (j >= cnt ? j - cnt : j); };
  if (cnt <= 0) return;  // same for both CTAs of the pair
  const size_t bh = (size_t)b * p.h + h;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t count = 1;
      if (i == kBarPReady || i == kBarDsReady) count = 16;  // per-warp arrivals of both CTAs
      else if (i == kBarDqDrained) count = 8;               // 4 dQ warps of each CTA
      else if (i == kBarLseEmpty || i == kBarLseEmpty + 1) count = 8;  // this CTA's elementwise warps
      else if (i == kBarXFull || i == kBarXFree || i == kBarDsoFull) count = 4;  // per-warp arrivals
      mbar_init(bar(i), count);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 12) {
    tmem_alloc_pair(smem_u32(tmem_holder), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // programmatic dependent of the preprocess (as the single-CTA kernel):
  // -lse*log2(e), D and dq_accum only after griddep_wait()
  griddep_launch_dependents();
  const bool leader = (rank == 0);
  auto lbar = [&](int i) -> uint32_t { return mapa_shared(bar(i), 0); };  // the leader's barrier

  if (warp == 15) {
    regs_dec<kRegsOther>();
    // ------------------------------------------- TMA producer B (MN-major halves)
    if (lane == 0) {
      const int dh = 64 * (int)rank;  // this CTA's head-dim half
      bool ok = true;
      for (int u = 0; u < cnt && ok; ++u) {
        const int qrow = qblock(u) * 128;
        // dO head-dim half for dV(u): free once dV(u-1) has read it
        if (u > 0 && !(ok = mbar_wait(bar(kBarOnEmpty), (u - 1) & 1, abort_flag, kRoleLoad2, 11))) break;
        if (leader) mbar_expect_tx(bar(kBarOnFull), 2 * kBox);
        tma_load_4d_pair(sbase + kOffOn, &tm_do, lbar(kBarOnFull), dh, qrow, h, b);
        // Q head-dim half for dK(u): free once dK(u-1) has read it
        if (u > 0 && !(ok = mbar_wait(bar(kBarQnEmpty), (u - 1) & 1, abort_flag, kRoleLoad2, 9))) break;
        if (leader) mbar_expect_tx(bar(kBarQnFull), 2 * kBox);
        tma_load_4d_pair(sbase + kOffQn, &tm_q, lbar(kBarQnFull), dh, qrow, h, b);
      }
    }
  } else if (warp == 14) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------- dS exchange
    if (lane == 0) {
      const uint32_t peer = rank ^ 1u;
      // this CTA's KV rows land in rows [128*rank, +128) of the peer's dS buffer
      const uint32_t dst = mapa_shared(sbase + kOffdS + 16384u * rank, peer);
      const uint32_t dst_bar = mapa_shared(bar(kBarDsIn), peer);
      const uint32_t relay = lbar(kBarDsInPeer);
      // The staging buffer needs no separate release: its writers wait for
      // dQ(u-1) to finish (DsEmpty) before writing block u, and dQ(u-1) ran
      // only after both CTAs' incoming blocks of u-1 had landed.  The same
      // wait covers the peer's destination rows.
      for (int u = 0; u < cnt; ++u) {
        mbar_expect_tx(bar(kBarDsIn), 16384);  // arm: the peer's block for this query block
        if (!mbar_wait(bar(kBarDsoFull), u & 1, abort_flag, kRoleEx2, 26)) break;
        bulk_copy_to_cluster(dst, sbase + kOffDso, 16384, dst_bar);
        // the incoming block must land before this barrier is armed again
        if (!mbar_wait(bar(kBarDsIn), u & 1, abort_flag, kRoleEx2, 24)) break;
        if (!leader) mbar_arrive_cluster(relay);  // the leader's dQ MMA also needs this CTA's rows
      }
    }
  } else if (warp == 13) {
    regs_dec<kRegsOther>();
    // ------------------------------------------- TMA producer A (K-major halves)
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_q64);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_do64);
      const int dh = 64 * (int)rank;  // this CTA's head-dim half
      if (leader) mbar_expect_tx(bar(kBarKvFull), 2 * 6 * kBox);
      for (int x = 0; x < 2; ++x) {
        tma_load_4d_pair(sbase + kOffK + x * kBox, &tm_k, lbar(kBarKvFull), x * 64, n0, h, b);
        tma_load_4d_pair(sbase + kOffV + x * kBox, &tm_v, lbar(kBarKvFull), x * 64, n0, h, b);
        tma_load_4d_pair(sbase + kOffKd + x * kBox, &tm_k, lbar(kBarKvFull), dh, pair_n0 + 128 * x, h, b);
      }
      griddep_wait();  // the preprocess has written -lse*log2(e) and D
      int lse_issued[2] = {0, 0};
      bool ok = true;
      for (int u = 0; u < cnt && ok; ++u) {
        const int m = qblock(u);
        const int qrow = m * 128;
        const int st = u & 1;
        // Q rows of this CTA for S^T(u): free once S^T(u-1) has read them
        if (u > 0 && !(ok = mbar_wait(bar(kBarQkEmpty), (u - 1) & 1, abort_flag, kRoleLoad2, 8))) break;
        if (leader) mbar_expect_tx(bar(kBarQkFull), 2 * 2 * kHalfBox);
        for (int x = 0; x < 2; ++x)
          tma_load_4d_pair(sbase + kOffQk + x * kHalfBox, &tm_q64, lbar(kBarQkFull), x * 64, qrow + 64 * (int)rank, h,
                           b);
        // -lse*log2(e) and D of the block for this CTA's elementwise warps
        if (u >= 2 && !(ok = mbar_wait(bar(kBarLseEmpty + st), ((u >> 1) - 1) & 1, abort_flag, kRoleLoad2, 19 + st)))
          break;
        const uint32_t lfull = bar(kBarLseFull + st);
        mbar_expect_tx(lfull, 1024);
        const size_t row0 = bh * (size_t)p.sq_rounded + (size_t)qrow;
        bulk_load(sbase + kOffLse + st * 512, p.neg_lse_log2 + row0, 512, lfull);
        bulk_load(sbase + kOffD + st * 512, p.dpsum + row0, 512, lfull);
        lse_issued[st] = (u >> 1) + 1;
        // dO rows of this CTA for dP^T(u): free once dP^T(u-1) has read them
        if (u > 0 && !(ok = mbar_wait(bar(kBarOkEmpty), (u - 1) & 1, abort_flag, kRoleLoad2, 10))) break;
        if (leader) mbar_expect_tx(bar(kBarOkFull), 2 * 2 * kHalfBox);
        for (int x = 0; x < 2; ++x)
          tma_load_4d_pair(sbase + kOffOk + x * kHalfBox, &tm_do64, lbar(kBarOkFull), x * 64, qrow + 64 * (int)rank, h,
                           b);
      }
      if (*abort_flag) {
        // the local lse/D copies are the only ones this CTA can wait for
        for (int s = 0; s < 2; ++s)
          if (lse_issued[s] > 0) mbar_wait_drain(bar(kBarLseFull + s), (lse_issued[s] - 1) & 1);
      }
    }
  } else if (warp == 12) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ MMA
    if (leader) {  // converged warp: all lanes wait and form descriptors, elected lanes issue
      constexpr uint32_t id_s = idesc_bf16(256, 128, 0, 0);   // S^T, dP^T: A, B K-major
      constexpr uint32_t id_kv = idesc_bf16(256, 128, 0, 1);  // dV, dK: A in TMEM, B MN-major
      constexpr uint32_t id_q = idesc_bf16(128, 128, 1, 1);   // dQ: A, B MN-major
      const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;
      const uint64_t k_k = sdesc(sbase + kOffK, 16, 1024);
      const uint64_t v_k = sdesc(sbase + kOffV, 16, 1024);
      const uint64_t qk_k = sdesc(sbase + kOffQk, 16, 1024);
      const uint64_t ok_k = sdesc(sbase + kOffOk, 16, 1024);
      const uint64_t qn_mn = sdesc(sbase + kOffQn, kBox, 1024);
      const uint64_t on_mn = sdesc(sbase + kOffOn, kBox, 1024);
      const uint64_t ds_mn = sdesc(sbase + kOffdS, kBox, 1024);
      const uint64_t kd_mn = sdesc(sbase + kOffKd, kBox, 1024);
      // K-major: 32 B per 16-element K step inside a 64-column box; the next
      // box is 16 KB (128-row A tiles) or 8 KB (64-row B halves) further.
      // MN-major: 2 KB per 16 rows of K.
      auto koff = [](int ks) -> uint32_t { return (uint32_t)((ks >> 2) * kBox + (ks & 3) * 32); };
      auto hoff = [](int ks) -> uint32_t { return (uint32_t)((ks >> 2) * kHalfBox + (ks & 3) * 32); };
      auto issue_s = [&]() {  // S^T = K Q^T over the pair
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss_pair_e(tS, desc_add(k_k, koff(ks)), desc_add(qk_k, hoff(ks)), id_s, ks > 0);
        mma_commit_pair_e(bar(kBarSFull), kPairMask);
        mma_commit_pair_e(bar(kBarQkEmpty), kPairMask);
      };
      auto issue_dp = [&]() {  // dP^T = V dO^T over the pair
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss_pair_e(tdP, desc_add(v_k, koff(ks)), desc_add(ok_k, hoff(ks)), id_s, ks > 0);
        mma_commit_pair_e(bar(kBarDpFull), kPairMask);
        mma_commit_pair_e(bar(kBarOkEmpty), kPairMask);
      };
      bool ok = mbar_wait_warp(bar(kBarKvFull), 0, abort_flag, kRoleMma2, 0) &&
                mbar_wait_warp(bar(kBarOkFull), 0, abort_flag, kRoleMma2, 3) &&
                mbar_wait_warp(bar(kBarQkFull), 0, abort_flag, kRoleMma2, 1);
      if (ok) {
        tc_fence_after();
        issue_dp();
        issue_s();
      }
      for (int u = 0; u < cnt && ok; ++u) {
        // dV += P^T dO   (P^T from TMEM: query 0-63 in columns [0,32), 64-127 in [64,96))
        if (!(ok = mbar_wait_warp(bar(kBarPReady), u & 1, abort_flag, kRoleMma2, 5))) break;
        if (!(ok = mbar_wait_warp(bar(kBarOnFull), u & 1, abort_flag, kRoleMma2, 4))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts_pair_e(tdV, tS + (ks >> 2) * 64 + (ks & 3) * 8, desc_add(on_mn, ks * 2048), id_kv,
                      (u > 0 || ks > 0) ? 1u : 0u);
        mma_commit_pair_e(bar(kBarOnEmpty), kPairMask);
        // S^T(u+1): the S columns are free once dV(u) has read P^T(u)
        if (u + 1 < cnt) {
          if (!(ok = mbar_wait_warp(bar(kBarQkFull), (u + 1) & 1, abort_flag, kRoleMma2, 1))) break;
          tc_fence_after();
          issue_s();
        }
        // dK += dS^T Q   (dS^T from TMEM over the dP^T columns)
        if (!(ok = mbar_wait_warp(bar(kBarDsReady), u & 1, abort_flag, kRoleMma2, 6))) break;
        if (!(ok = mbar_wait_warp(bar(kBarQnFull), u & 1, abort_flag, kRoleMma2, 2))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts_pair_e(tdK, tdP + (ks >> 2) * 64 + (ks & 3) * 8, desc_add(qn_mn, ks * 2048), id_kv,
                      (u > 0 || ks > 0) ? 1u : 0u);
        mma_commit_pair_e(bar(kBarQnEmpty), kPairMask);
        // dQ needs the dS rows exchanged between the CTAs: this CTA's incoming
        // block (bulk-copy bytes) and the peer's (relayed by its warp 14)
        if (!(ok = mbar_wait_warp(bar(kBarDsIn), u & 1, abort_flag, kRoleMma2, 24))) break;
        if (!(ok = mbar_wait_warp(bar(kBarDsInPeer), u & 1, abort_flag, kRoleMma2, 25))) break;
        // dQ rows of each CTA = dS K over the pair's 256 KV rows, into the dP^T columns
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          mma_ss_pair_e(tdP, desc_add(ds_mn, ks * 2048), desc_add(kd_mn, ks * 2048), id_q, ks > 0);
        mma_commit_pair_e(bar(kBarDqFull), kPairMask);
        mma_commit_pair_e(bar(kBarDsEmpty), kPairMask);
        // dP^T(u+1) once both CTAs have drained dQ(u) from those columns
        if (u + 1 < cnt) {
          if (!(ok = mbar_wait_warp(bar(kBarDqDrained), u & 1, abort_flag, kRoleMma2, 7))) break;
          if (!(ok = mbar_wait_warp(bar(kBarOkFull), (u + 1) & 1, abort_flag, kRoleMma2, 3))) break;
          tc_fence_after();
          issue_dp();
        }
      }
      if (ok) mma_commit_pair_e(bar(kBarDkvFull), kPairMask);
      mma_commit_pair_e(bar(kBarDrain), 0x1);
      mbar_wait_drain(bar(kBarDrain), 0);
    }
  } else if (warp < 8) {
    regs_inc<kRegsEw>();
    // ---------------------------------------------- elementwise warpgroups
    const int half = warp >> 2;   // query columns [64*half, +64), owned by CTA `half` for dQ
    const int wq = warp & 3;
    const int r = wq * 32 + lane; // KV row within this CTA
    const bool kv_valid = (n0 + r) < p.skv;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + (uint32_t)(half * 64);
    const uint32_t tdP = tmem + lane_base + 128u + (uint32_t)(half * 64);
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    // dS rows: query columns owned by this CTA go to row 128*rank + r of the
    // local dS buffer; the peer's go to row r of the outgoing staging buffer
    const bool ds_local = (half == (int)rank);  // warp-uniform
    uint8_t* const ds_base = ds_local ? smem + kOffdS + 16384 * rank : smem + kOffDso;
    const uint32_t pready = lbar(kBarPReady), dsready = lbar(kBarDsReady);
    bool ok = true;
    for (int u = 0; u < cnt; ++u) {
      const int st = u & 1;
      const float* snl = reinterpret_cast<const float*>(smem + kOffLse + st * 512) + half * 64;
      const float* sD = reinterpret_cast<const float*>(smem + kOffD + st * 512) + half * 64;
      if (!(ok = mbar_wait(bar(kBarSFull), u & 1, abort_flag, kRoleEw2, 12))) break;
      if (!(ok = mbar_wait(bar(kBarLseFull + st), (u >> 1) & 1, abort_flag, kRoleEw2, 17 + st))) break;
      tc_fence_after();
      uint32_t s[2][32];
      tmem_ld32(tS, s[0]);
      tmem_ld32(tS + 32, s[1]);
      tmem_wait_ld();
      reg_fence32(s[0]);
      reg_fence32(s[1]);
      uint64_t pp[2][16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 L = *reinterpret_cast<const float4*>(snl + c * 32 + v * 4);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int i = 2 * v + e;
            const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[c][2 * i]), __uint_as_float(s[c][2 * i + 1])), sl2x2,
                                      e ? f2_pack(L.z, L.w) : f2_pack(L.x, L.y));
            pp[c][i] = exp2_mufu2(x);
            float p0, p1;
            f2_unpack(pp[c][i], p0, p1);
            pk[i] = kv_valid ? pack_bf16(p0, p1) : 0u;
          }
        }
        tmem_st16(tS + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(pready);
      // dS^T = P^T * (dP^T - D[q])
      if (!(ok = mbar_wait(bar(kBarDpFull), u & 1, abort_flag, kRoleEw2, 13))) break;
      tc_fence_after();
      uint32_t dp[2][32];
      tmem_ld32(tdP, dp[0]);
      tmem_ld32(tdP + 32, dp[1]);
      tmem_wait_ld();
      reg_fence32(dp[0]);
      reg_fence32(dp[1]);
      if (u > 0 && !(ok = mbar_wait(bar(kBarDsEmpty), (u - 1) & 1, abort_flag, kRoleEw2, 14))) break;
      const uint64_t m1x2 = f2_pack(-1.f, -1.f);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 D = *reinterpret_cast<const float4*>(sD + c * 32 + v * 4);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int i = 2 * v + e;
            const uint64_t dpp = f2_pack(__uint_as_float(dp[c][2 * i]), __uint_as_float(dp[c][2 * i + 1]));
            const uint64_t t = f2_fma(e ? f2_pack(D.z, D.w) : f2_pack(D.x, D.y), m1x2, dpp);
            float d0, d1;
            f2_unpack(f2_mul(pp[c][i], t), d0, d1);
            pk[i] = kv_valid ? pack_bf16(d0, d1) : 0u;
          }
        }
        // dS^T as the A operand of the dK MMA, over this warpgroup's dP^T columns
        tmem_st16(tdP + c * 16, pk);
        // row r of this warpgroup's dS block, query columns [32c, 32c+32) of this half
#pragma unroll
        for (int v = 0; v < 4; ++v)
          *reinterpret_cast<uint4*>(ds_base + sw128_offset((uint32_t)r, (uint32_t)(c * 4 + v))) =
              make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
      }
      fence_proxy_async_smem();
      if (!ds_local) mbar_arrive_warp(bar(kBarDsoFull));  // the exchange warp may copy the block
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_cluster(dsready);
        mbar_arrive(bar(kBarLseEmpty + st));
      }
    }
    // ----------------------------------------------------------- epilogue
    if (ok) ok = mbar_wait(bar(kBarDkvFull), 0, abort_flag, kRoleEpi2, 16);
    if (ok) {  // every lane runs the (warp-collective) TMEM loads; stores are per row
      tc_fence_after();
      const int kv = n0 + r;
      const uint32_t tsrc = tmem + lane_base + (half ? 384u : 256u);
      const float mul = half ? p.scale : 1.f;
      void* dst = half ? p.dk : p.dv;
      const int nb = n0 >> 7;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t a[32];
        tmem_ld32(tsrc + c * 32, a);
        tmem_wait_ld();
        reg_fence32(a);
        if (!kv_valid) continue;
        if (!p.accum_dkv) {
          __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(dst) + (((size_t)b * p.skv + kv) * p.h + h) * 128;
#pragma unroll
          for (int v = 0; v < 4; ++v)
            st_global_v4(row + c * 32 + v * 8,
                         pack_bf16(__uint_as_float(a[8 * v + 0]) * mul, __uint_as_float(a[8 * v + 1]) * mul),
                         pack_bf16(__uint_as_float(a[8 * v + 2]) * mul, __uint_as_float(a[8 * v + 3]) * mul),
                         pack_bf16(__uint_as_float(a[8 * v + 4]) * mul, __uint_as_float(a[8 * v + 5]) * mul),
                         pack_bf16(__uint_as_float(a[8 * v + 6]) * mul, __uint_as_float(a[8 * v + 7]) * mul));
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
    }
  } else {
    regs_inc<kRegsDq>();
    // ------------------------------------------------------- dQ warpgroup
    // This CTA's dQ rows of the pair's M = 128 MMA sit in TMEM columns
    // [128, 192): lane l holds query row 64*rank + l%64, head-dim columns
    // [64*(l/64), +64).  Each head-dim half is staged in turn as [16 groups
    // of 4 columns][64 rows][4] -- one contiguous 16 KB piece of the
    // accumulator's run for this row half -- and reduced by one bulk
    // cp.reduce.async (two per query block).
    const int wq = warp & 3;
    const int l = wq * 32 + lane;
    const int row = l & 63, dh = l >> 6;
    const uint32_t tQ = tmem + ((uint32_t)(wq * 32) << 16) + 128u;
    const uint32_t sx = sbase + kOffX;
    uint8_t* xb = smem + kOffX;
    const bool lead_thr = (threadIdx.x == 256);
    if (lead_thr) griddep_wait();  // the preprocess has zeroed dq_accum
    const uint32_t drained = lbar(kBarDqDrained);
    for (int u = 0; u < cnt; ++u) {
      if (!mbar_wait(bar(kBarDqFull), u & 1, abort_flag, kRoleDq2, 15)) break;
      tc_fence_after();
      uint32_t q[2][32];
      tmem_ld32(tQ, q[0]);
      tmem_ld32(tQ + 32, q[1]);
      tmem_wait_ld();
      reg_fence32(q[0]);
      reg_fence32(q[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(drained);
      float* run = p.dq_accum + (bh * (size_t)p.m_blocks + qblock(u)) * 16384 + rank * 8192;
      bool ok = true;
      for (int hh = 0; hh < 2 && ok; ++hh) {
        const uint32_t ph = (uint32_t)(2 * u + hh) & 1u;
        // the staging buffer is free once the previous bulk reduction has read it
        if (lead_thr) bulk_wait_read_all();
        mbar_arrive_warp(bar(kBarXFree));
        if (!(ok = mbar_wait(bar(kBarXFree), ph, abort_flag, kRoleDq2, 22))) break;
        if (dh == hh) {  // warp-uniform: warps 0-1 hold head-dim half 0, warps 2-3 half 1
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int g = 0; g < 8; ++g)
              *reinterpret_cast<uint4*>(xb + ((c * 8 + g) * 64 + row) * 16) =
                  make_uint4(q[c][4 * g + 0], q[c][4 * g + 1], q[c][4 * g + 2], q[c][4 * g + 3]);
          fence_proxy_async_smem();
        }
        mbar_arrive_warp(bar(kBarXFull));
        if (lead_thr) {
          if (!(ok = mbar_wait(bar(kBarXFull), ph, abort_flag, kRoleDq2, 21))) break;
          bulk_reduce_add_f32(run + hh * 4096, sx, 16384);
          bulk_commit_group();
        }
      }
      if (!ok || *abort_flag) break;
    }
    if (lead_thr) bulk_wait_all();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs and the peer's remote stores / arrivals are done
  tc_fence_after();
  if (warp == 12) tmem_dealloc_pair(tmem, 512);
}

}  // namespace wf
