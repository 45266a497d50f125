// Forward attention, CTA-pair form: a cluster of two CTAs along the query
// axis issues 2-SM tensor-core MMAs (tcgen05 cta_group::2, M = 256).
//
// Same computation as wf_fwd_kernel (wf_fwd.cu) and the reference forward
// (wan_flash/fwd_sm90.py of Quarky93/wan-flash: `softmax_step` :330-379,
// `rescale_O` :381-395, `apply_seqlenk_mask` :397-420, finalize :866-941).
// The reference's cluster (2, 1) pairs two query tiles and multicasts each
// K/V tile into both CTAs (features.py:28-42).  Here the pair shares the
// K/V tiles through the MMA instead of through the load:
//   * S_t = Q_t K^T is one M = 256 MMA: each CTA supplies its own 128 query
//     rows of A (Q_t) and HALF of B (64 of the block's 128 keys);
//   * O_t += P_t V is one M = 256 MMA: each CTA supplies its own P_t (A, in
//     its tensor memory) and half of B (64 of the 128 head-dim columns of V).
// So each SM loads half of every K/V tile, reads 3/4 of the shared-memory
// operand bytes of the single-CTA kernel, and the leader's MMA warp issues
// one instruction where two single-CTA kernels would issue two.
//
// Work: the cluster owns 512 query rows (two 256-row items) of one (batch,
// head); CTA r takes rows [256 r, 256 r + 256) of them as two 128-row tiles,
// walks every KV block (ragged tail first, masked) and writes its own O and
// LSE.  A CTA whose rows all lie past sq computes padding and stores
// nothing.
//
// Roles per CTA (384 threads):
//   warps 0-3  softmax for query tile 0 (thread = one query row)
//   warps 4-7  softmax for query tile 1
//   warp  8    TMEM owner (both CTAs, cta_group::2 allocation); MMA issuer
//              (leader CTA only: converged warp, one elected lane)
//   warp  9    TMA producer: own Q tiles, own K/V halves (counted on the
//              leader's barriers; the leader arms them with both CTAs' bytes)
//   warp  10   O store (TMA tensor stores of this CTA's tiles)
//   warp  11   idle (completes warpgroup 2 for the register split)
//
// Synchronisation: loads of both CTAs complete on the leader's full
// barriers; the softmax warps of both CTAs arrive (one per warp) on the
// leader's P barriers; every MMA completion is committed to the same barrier
// in both CTAs (S ready, O ready, K/V slot free).  No load is multicast.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

namespace fwd2 {
constexpr int kThreads = 384;
// register split (launch: 384 x 168 = 64512): softmax WGs 2 x 128 x 208 + WG2 128 x 88
constexpr uint32_t kRegsSoftmax = 208;
constexpr uint32_t kRegsOther = 88;
constexpr int kSlots = 8;                   // K/V ring: K halves and V halves alternate
constexpr uint32_t kBox = 128 * 128;        // 128 rows x 64 bf16 (one 128B-swizzled box)
constexpr uint32_t kHalfBox = 64 * 128;     // 64 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kBox;   // 128 rows x 128 bf16
constexpr uint32_t kSlotBytes = kBox;       // K half: 64 keys x 128 d (two 8 KB boxes); V half: 128 keys x 64 d
constexpr uint32_t kOffQ = 0;               // 2 query tiles
constexpr uint32_t kOffKV = 2 * kTileBytes;
constexpr uint32_t kOffOStage = kOffKV + kSlots * kSlotBytes;
constexpr uint32_t kOffBar = kOffOStage + kTileBytes;
constexpr int kBarQFull = 0;                      // + tile   (leader: both CTAs' tile t)
constexpr int kBarKvFull = 2;                     // + slot   (leader: both CTAs' halves)
constexpr int kBarKvEmpty = kBarKvFull + kSlots;  // + slot   (each CTA: MMA commit to both)
constexpr int kBarSFull = kBarKvEmpty + kSlots;   // + tile   (each CTA)
constexpr int kBarPFull = kBarSFull + 2;          // + 2 * tile + half (leader: 8 softmax warps)
constexpr int kBarOFull = kBarPFull + 4;          // + tile   (each CTA)
constexpr int kBarDrain = kBarOFull + 2;          // leader
constexpr int kBarOStaged = kBarDrain + 1;        // local: O tile in the stage (one arrival per warp)
constexpr int kBarOStageFree = kBarOStaged + 1;   // local: stage read by the tensor store
constexpr int kNumBars = kBarOStageFree + 1;
constexpr uint32_t kOffTmemHolder = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemHolder + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "pair forward shared memory exceeds the sm_100 per-CTA limit");
constexpr uint16_t kPairMask = 0x3;
}  // namespace fwd2

size_t fwd2_smem_bytes() { return fwd2::kSmemBytes; }

enum : uint32_t { kRoleSm2 = 31, kRoleMmaF2 = 33, kRoleLoadF2 = 34, kRoleStoreF2 = 35 };

__global__ void __launch_bounds__(fwd2::kThreads, 1)
    wf_fwd2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k64,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, FwdParams p) {
  using namespace fwd2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmemHolder);

  const int warp = (int)warp_id();
  const int lane = (int)lane_id();
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const bool leader = (rank == 0);
  const int n_cl = (p.n_pairs + 1) >> 1;  // clusters per (batch, head)
  const int cl = (int)(blockIdx.x >> 1);
  const int hb = cl / n_cl;
  const int m0 = ((cl % n_cl) * 2 + (int)rank) * 256;  // this CTA's first query row
  const int h = hb % p.h;
  const int b = hb / p.h;
  const int n_blocks = p.n_blocks[0];

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarQFull + t), 1);
      mbar_init(bar(kBarSFull + t), 1);
      mbar_init(bar(kBarPFull + 2 * t), 8);  // 4 softmax warps of each CTA
      mbar_init(bar(kBarPFull + 2 * t + 1), 8);
      mbar_init(bar(kBarOFull + t), 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(bar(kBarKvFull + s), 1);
      mbar_init(bar(kBarKvEmpty + s), 1);
    }
    mbar_init(bar(kBarDrain), 1);
    mbar_init(bar(kBarOStaged), 4);
    mbar_init(bar(kBarOStageFree), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc_pair(smem_u32(tmem_holder), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrival or copy
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  auto lbar = [&](int i) -> uint32_t { return mapa_shared(bar(i), 0); };  // the leader's barrier

  if (warp == 11) {
    regs_dec<kRegsOther>();
  } else if (warp == 10) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------ O store
    if (lane == 0) {
      tma_prefetch_desc(&tm_o);
      for (int t = 0; t < 2; ++t) {
        if (!mbar_wait(bar(kBarOStaged), (uint32_t)t, abort_flag, kRoleStoreF2, 50 + t)) break;
        if (m0 + t * 128 < p.sq) {  // a tile wholly past sq stores nothing
          for (int x = 0; x < 2; ++x) tma_store_4d(&tm_o, sbase + kOffOStage + x * kBox, x * 64, m0 + t * 128, h, b);
          bulk_commit_group();
          bulk_wait_read_all();
        }
        mbar_arrive(bar(kBarOStageFree));
      }
      bulk_wait_all();
    }
  } else if (warp == 9) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k64);
      tma_prefetch_desc(&tm_v);
      for (int t = 0; t < 2; ++t) {
        if (leader) mbar_expect_tx(bar(kBarQFull + t), 2 * kTileBytes);
        for (int x = 0; x < 2; ++x)
          tma_load_4d_pair(sbase + kOffQ + t * kTileBytes + x * kBox, &tm_q, lbar(kBarQFull + t), x * 64,
                           m0 + t * 128, h, b);
      }
      int u = 0;  // K/V units in walk order: K(j) = 2i, V(j) = 2i + 1 for the i-th block walked
      for (int it = 0; it < n_blocks; ++it) {
        const int j = (it == 0) ? (n_blocks - 1) : (it - 1);  // ragged tail first
        bool ok = true;
        for (int kv = 0; kv < 2; ++kv, ++u) {
          const int slot = u % kSlots, use = u / kSlots;
          if (use > 0 && !(ok = mbar_wait(bar(kBarKvEmpty + slot), (use - 1) & 1, abort_flag, kRoleLoadF2, 100 + slot)))
            break;
          const uint32_t dst = sbase + kOffKV + slot * kSlotBytes;
          if (leader) mbar_expect_tx(bar(kBarKvFull + slot), 2 * kSlotBytes);
          if (kv == 0) {  // keys [64 r, 64 r + 64) of the block, all head dims (two 64-column boxes)
            for (int x = 0; x < 2; ++x)
              tma_load_4d_pair(dst + x * kHalfBox, &tm_k64, lbar(kBarKvFull + slot), x * 64, j * 128 + 64 * (int)rank,
                               h, b);
          } else {        // all 128 keys, head dims [64 r, 64 r + 64)
            tma_load_4d_pair(dst, &tm_v, lbar(kBarKvFull + slot), 64 * (int)rank, j * 128, h, b);
          }
        }
        if (!ok) break;
      }
      if (*abort_flag && leader) {
        // drain: every copy either CTA issued completes on the leader's
        // barriers, so once these phases complete no copy is in flight into
        // either CTA (the peer waits at the closing cluster barrier)
        for (int t = 0; t < 2; ++t) mbar_wait_drain(bar(kBarQFull + t), 0);
        for (int sl = 0; sl < kSlots && sl < u; ++sl)  // u units were issued; slot sl took the last of its uses
          mbar_wait_drain(bar(kBarKvFull + sl), ((u - 1 - sl) / kSlots) & 1);
      }
    }
  } else if (warp == 8) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ MMA
    if (leader) {  // converged warp: all lanes wait and form descriptors, elected lanes issue
      constexpr uint32_t id_s = idesc_bf16(256, 128, 0, 0);   // A (Q), B (K half) K-major
      constexpr uint32_t id_pv = idesc_bf16(256, 128, 0, 1);  // A (P) in TMEM, B (V half) MN-major
      const uint32_t sQ = sbase + kOffQ;
      const uint32_t sKV = sbase + kOffKV;
      // K-major: 32 B per 16-element K step inside a 64-column box, then the
      // next box (16 KB for the 128-row Q tile, 8 KB for the 64-row K half);
      // MN-major V half: 2 KB per 16 keys.
      auto issue_s = [&](int t, int slot) {
        const uint64_t a0 = sdesc(sQ + t * kTileBytes, 16, 1024);
        const uint64_t b0 = sdesc(sKV + slot * kSlotBytes, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss_pair_ee(tmem + (uint32_t)(t * 128), desc_add(a0, (uint32_t)((ks >> 2) * kBox + (ks & 3) * 32)),
                         desc_add(b0, (uint32_t)((ks >> 2) * kHalfBox + (ks & 3) * 32)), id_s, ks > 0);
      };
      int pv_phase[2] = {0, 0};
      bool ok = true;
      auto issue_pv = [&](int t, int slot_v, bool acc) -> bool {
        const uint64_t b0 = sdesc(sKV + slot_v * kSlotBytes, kBox, 1024);
        for (int half = 0; half < 2; ++half) {
          if (!mbar_wait_warp(bar(kBarPFull + 2 * t + half), (uint32_t)pv_phase[t] & 1, abort_flag, kRoleMmaF2,
                              20 + 2 * t + half))
            return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int ks = half * 4 + kk;
            mma_ts_pair_ee(tmem + 256u + (uint32_t)(t * 128), tmem + (uint32_t)(t * 128 + ks * 8),
                           desc_add(b0, (uint32_t)(ks * 2048)), id_pv, (acc || ks > 0) ? 1u : 0u);
          }
        }
        pv_phase[t]++;
        return true;
      };
      // block g (walk order) issues PV_t(g-1) before S_t(g) for each tile
      for (int g = 0; g < n_blocks && ok; ++g) {
        const int uk = 2 * g, slot_k = uk % kSlots;
        if (!(ok = mbar_wait_warp(bar(kBarKvFull + slot_k), (uk / kSlots) & 1, abort_flag, kRoleMmaF2, 10 + slot_k)))
          break;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t) {
          if (g > 0) {
            const int uv = 2 * (g - 1) + 1, slot_v = uv % kSlots;
            if (t == 0 && !(ok = mbar_wait_warp(bar(kBarKvFull + slot_v), (uv / kSlots) & 1, abort_flag, kRoleMmaF2,
                                                 10 + slot_v)))
              break;
            if (!(ok = issue_pv(t, slot_v, g > 1))) break;
            if (t == 1) mma_commit_pair_ee(bar(kBarKvEmpty + slot_v), kPairMask);
          }
          if (g == 0) {
            if (!(ok = mbar_wait_warp(bar(kBarQFull + t), 0, abort_flag, kRoleMmaF2, t))) break;
            tc_fence_after();
          }
          issue_s(t, slot_k);
          mma_commit_pair_ee(bar(kBarSFull + t), kPairMask);
        }
        if (ok) mma_commit_pair_ee(bar(kBarKvEmpty + slot_k), kPairMask);
      }
      if (ok) {
        const int uv = 2 * (n_blocks - 1) + 1, slot_v = uv % kSlots;
        ok = mbar_wait_warp(bar(kBarKvFull + slot_v), (uv / kSlots) & 1, abort_flag, kRoleMmaF2, 10 + slot_v);
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = issue_pv(t, slot_v, n_blocks > 1))) break;
          mma_commit_pair_ee(bar(kBarOFull + t), kPairMask);
        }
        if (ok) mma_commit_pair_ee(bar(kBarKvEmpty + slot_v), kPairMask);
      }
      // drain the tensor pipe before TMEM can be released
      mma_commit_pair_ee(bar(kBarDrain), 0x1);
      mbar_wait_drain(bar(kBarDrain), 0);
    }
  } else {
    regs_inc<kRegsSoftmax>();
    // -------------------------------------------------------------- softmax
    const int t = warp >> 2;  // query tile
    const int wq = warp & 3;  // TMEM lane quadrant
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + (uint32_t)(t * 128);
    const uint32_t tO = tmem + lane_base + 256u + (uint32_t)(t * 128);
    const uint32_t pfull0 = lbar(kBarPFull + 2 * t), pfull1 = lbar(kBarPFull + 2 * t + 1);
    const float sl2 = p.scale_log2;
    const float thr = p.rescale_threshold;
    const int tail_valid = p.skv[0] - (n_blocks - 1) * 128;  // 1..128
    float m_s = -INFINITY;  // running reference max, in scaled log2 units
    float l = 0.f;          // running row sum (relative to m_s)
    bool ok = true;
    for (int it = 0; it < n_blocks; ++it) {
      if (!(ok = mbar_wait(bar(kBarSFull + t), (uint32_t)it & 1, abort_flag, kRoleSm2, 30 + t))) break;
      tc_fence_after();
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) reg_fence32(s[c]);
      if (it == 0 && tail_valid < 128) {
        // first (ragged tail) block: keys past skv do not exist
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i >= tail_valid) s[c][i] = __float_as_uint(-INFINITY);
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i)
          mx[i & 3] = fmax3(mx[i & 3], __uint_as_float(s[c][2 * i]), __uint_as_float(s[c][2 * i + 1]));
      const float mnew_s = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
      if (it == 0) {
        m_s = mnew_s;
      } else {
        // move the reference max only when the row max grew past the threshold
        const bool need = mnew_s - m_s > thr;
        if (__any_sync(0xffffffffu, need)) {
          const float factor = need ? ex2_approx(m_s - mnew_s) : 1.f;
          if (need) {
            l *= factor;
            m_s = mnew_s;
          }
          // O_t holds the sum through block it-1 (the commit that signalled S_t(it) covers PV_t(it-1))
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t o[16];
            tmem_ld16(tO + c * 16, o);
            tmem_wait_ld();
            reg_fence16(o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st16(tO + c * 16, o);
          }
        }
      }
      const uint64_t sl2x2 = f2_pack(sl2, sl2), negx2 = f2_pack(-m_s, -m_s);
      float bsum = fwd_exp_half(s, 0, tS, sl2x2, negx2);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(pfull0);
      bsum += fwd_exp_half(s, 2, tS, sl2x2, negx2);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(pfull1);
      l += bsum;
    }
    // --------------------------------------------------------- epilogue
    if (ok) ok = mbar_wait(bar(kBarOFull + t), 0, abort_flag, kRoleSm2, 40 + t);
    if (ok && t == 1) ok = mbar_wait(bar(kBarOStageFree), 0, abort_flag, kRoleSm2, 46);
    if (ok) {
      tc_fence_after();
      const int r = wq * 32 + lane;  // row within the tile
      const int row = m0 + t * 128 + r;
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      // tile 0 stages first; tile 1 waited above until the store of tile 0 had read the stage
      {
        const uint32_t stage = sbase + kOffOStage + (uint32_t)r * 128u;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          reg_fence32(o);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack_bf16(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const uint32_t chunk = (uint32_t)((c & 1) * 4 + v);  // 16-byte chunk within the 64-column box
            st_shared_v4(stage + (uint32_t)(c >> 1) * kBox + ((chunk ^ ((uint32_t)r & 7u)) << 4), pk[4 * v],
                         pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarOStaged));
      if (row < p.sq) {
        // natural-log LSE; -inf when the row sum is zero or not finite
        const float lse = (l > 0.f && l == l) ? (m_s + log2f(l)) * 0.69314718055994531f : -INFINITY;
        p.lse[0][((size_t)b * p.h + h) * p.sq + row] = lse;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs into this CTA's TMEM and the peer's arrivals are done
  tc_fence_after();
  if (warp == 8) tmem_dealloc_pair(tmem, 512);
}

}  // namespace wf
