// Forward attention kernel for B200 (sm_100a): tcgen05 MMAs with S and O
// accumulators in tensor memory, TMA-fed Q/K/V, warp-specialised roles.
//
// Follows the computation of the reference forward (wan_flash/fwd_sm90.py of
// Quarky93/wan-flash): softmax in the exp2 domain with the max-shift
// rescale skip (`softmax_step` :330-379, `rescale_O` :381-395), masked
// ragged KV tail peeled as the first step (`apply_seqlenk_mask` :397-420,
// descending KV walk), packed RN bf16 converts (:48-61), and the finalize
// LSE = (m * scale_log2 + log2(sum)) * ln2 (:866-876).  The schedule is a
// Blackwell design of its own:
//
//   CTA = 2 query tiles of 128 rows (256 rows) of one (batch, head).
//   warps 0-3  softmax for query tile 0  (thread = one query row)
//   warps 4-7  softmax for query tile 1
//   warp  8    tcgen05.mma issuer (one thread) + TMEM owner
//   warp  9    TMA producer (one thread)
//   warps 10-11 idle (complete warpgroup 2 so it can give registers back)
//
//   TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
//   P_t (bf16, 64 columns) overwrites the first half of S_t once S_t is read.
//
//   MMA order per KV block j:  PV0(j-1) S0(j) PV1(j-1) S1(j)  -- softmax of
//   tile 0 overlaps the tensor work of tile 1 and vice versa.  P_t is
//   produced in two key halves with their own barriers, so PV_t starts on
//   keys 0-63 while the softmax still exponentiates keys 64-127.  The tensor
//   pipe executes tcgen05.mma in issue order, so S_t(j) never overwrites
//   P_t(j-1) before PV_t(j-1) has read it, and the commit that signals
//   "S_t(j) ready" also covers PV_t(j-1) -- O_t is final for block j-1 when
//   the softmax sees S_t(j), which is when it may rescale O_t in place.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

namespace fwd {
constexpr int kThreads = 384;
// register split (launch: 384 x 168 = 64512): softmax WGs 2 x 128 x 208 + WG2 128 x 88 = 64512
constexpr uint32_t kRegsSoftmax = 208;
constexpr uint32_t kRegsOther = 88;
constexpr int kKvSlots = 4;
constexpr uint32_t kBoxBytes = 128 * 128;        // 128 rows x 64 bf16 (one 128B-swizzled box)
constexpr uint32_t kTileBytes = 2 * kBoxBytes;   // 128 rows x 128 bf16
constexpr uint32_t kOffQ = 0;                    // 2 query tiles
constexpr uint32_t kOffKV = 2 * kTileBytes;      // kKvSlots tiles (K and V alternate)
constexpr uint32_t kOffBar = kOffKV + kKvSlots * kTileBytes;
// barrier indices
constexpr int kBarQFull = 0;
constexpr int kBarKvFull = 1;                    // + slot
constexpr int kBarKvEmpty = kBarKvFull + kKvSlots;
constexpr int kBarSFull = kBarKvEmpty + kKvSlots;  // + tile
constexpr int kBarPFull = kBarSFull + 2;      // + 2 * tile + half (keys 0-63 / 64-127)
constexpr int kBarOFull = kBarPFull + 4;
constexpr int kBarDrain = kBarOFull + 2;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kOffTmemHolder = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemHolder + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + alignment slack
}  // namespace fwd

size_t fwd_smem_bytes() { return fwd::kSmemBytes; }

// role ids recorded on a wait timeout
enum : uint32_t { kRoleSoftmax0 = 1, kRoleSoftmax1 = 2, kRoleMma = 3, kRoleLoad = 4 };

// Exponentials of half a 128-column block (two 32-column chunks starting at
// chunk c0) for this thread's row: P = 2^(s * scale_log2 - m) is stored to
// TMEM as bf16 pairs over the already-read S columns and the fp32 partial
// row sum is returned.  Packed f32x2 math keeps the instruction count low:
// the softmax warps share their SMSPs with the MMA-issuing warp, whose issue
// rate sets the tensor pipe's.  kFwdPolyEvery > 0 routes one pair in
// kFwdPolyEvery through the FMA-pipe polynomial exp2 instead of MUFU (off by
// default: on B200 it costs more issue slots than the MUFU time it saves).
constexpr int kFwdPolyEvery = 0;

__device__ __forceinline__ float fwd_exp_half(const uint32_t (&s)[4][32], int c0, uint32_t tS, uint64_t sl2x2,
                                              uint64_t negx2) {
  uint64_t acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = f2_pack(0.f, 0.f);
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const int c = c0 + cc;
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[c][2 * i]), __uint_as_float(s[c][2 * i + 1])), sl2x2, negx2);
      const uint64_t pp =
          (kFwdPolyEvery > 0 && (i % kFwdPolyEvery) == kFwdPolyEvery - 1) ? exp2_poly2(x) : exp2_mufu2(x);
      acc[i & 3] = f2_add(acc[i & 3], pp);
      float p0, p1;
      f2_unpack(pp, p0, p1);
      pk[i] = pack_bf16(p0, p1);
    }
    tmem_st16(tS + c * 16, pk);
  }
  float a0, a1;
  f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), a0, a1);
  return a0 + a1;
}

__global__ void __launch_bounds__(fwd::kThreads, 1)
    wf_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, FwdParams p) {
  using namespace fwd;
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
  const int m0 = blockIdx.x * 256;
  const int n_blocks = p.n_blocks;

  if (threadIdx.x == 0) {
    mbar_init(bar(kBarQFull), 1);
    for (int s = 0; s < kKvSlots; ++s) {
      mbar_init(bar(kBarKvFull + s), 1);
      mbar_init(bar(kBarKvEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarSFull + t), 1);
      mbar_init(bar(kBarPFull + 2 * t), 4);  // one arrival per softmax warp
      mbar_init(bar(kBarPFull + 2 * t + 1), 4);
      mbar_init(bar(kBarOFull + t), 1);
    }
    mbar_init(bar(kBarDrain), 1);
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

  if (warp >= 10) {
    regs_dec<kRegsOther>();  // idle warps of warpgroup 2
  } else if (warp == 9) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_expect_tx(bar(kBarQFull), 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        for (int x = 0; x < 2; ++x)
          tma_load_4d(sbase + kOffQ + t * kTileBytes + x * kBoxBytes, &tm_q, bar(kBarQFull), x * 64,
                      m0 + t * 128, h, b);
      int issued[kKvSlots] = {0, 0, 0, 0};
      bool ok = true;
      for (int it = 0; it < n_blocks && ok; ++it) {
        const int j = (it == 0) ? (n_blocks - 1) : (it - 1);
        for (int kv = 0; kv < 2 && ok; ++kv) {  // 0 = K, 1 = V
          const int u = 2 * it + kv;
          const int slot = u % kKvSlots;
          const int use = u / kKvSlots;
          if (use > 0) ok = mbar_wait(bar(kBarKvEmpty + slot), (use - 1) & 1, abort_flag, kRoleLoad, 100 + slot);
          if (!ok) break;
          mbar_expect_tx(bar(kBarKvFull + slot), kTileBytes);
          const CUtensorMap* tm = kv ? &tm_v : &tm_k;
          for (int x = 0; x < 2; ++x)
            tma_load_4d(sbase + kOffKV + slot * kTileBytes + x * kBoxBytes, tm, bar(kBarKvFull + slot),
                        x * 64, j * 128, h, b);
          issued[slot] = use + 1;
        }
      }
      if (*abort_flag) {
        // drain: let every issued copy land before the CTA can exit
        mbar_wait_drain(bar(kBarQFull), 0);
        for (int s = 0; s < kKvSlots; ++s)
          if (issued[s] > 0) mbar_wait_drain(bar(kBarKvFull + s), (issued[s] - 1) & 1);
      }
    }
  } else if (warp == 8) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ MMA
    {  // converged warp: all lanes wait and form descriptors, elected lanes issue
      constexpr uint32_t idesc_qk = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16(128, 128, 0, 1);
      const uint32_t sQ = sbase + kOffQ;
      const uint32_t sKV = sbase + kOffKV;
      bool ok = mbar_wait_warp(bar(kBarQFull), 0, abort_flag, kRoleMma, 0);
      tc_fence_after();
      int pv_phase[2] = {0, 0};
      auto issue_s = [&](int t, int slot_k) {
        const uint32_t d = tmem + (uint32_t)(t * 128);
        const uint64_t a0 = sdesc(sQ + t * kTileBytes, 16, 1024);
        const uint64_t b0 = sdesc(sKV + slot_k * kTileBytes, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * kBoxBytes + (ks & 3) * 32);
          mma_ss_e(d, desc_add(a0, off), desc_add(b0, off), idesc_qk, ks > 0);
        }
      };
      // O_t += P_t V over keys [64*half, 64*half + 64) once that half of P_t
      // has been written (P_t: bf16 pairs in S_t columns [0, 64))
      auto issue_pv_half = [&](int t, int half, int slot_v, bool acc) -> bool {
        if (!mbar_wait_warp(bar(kBarPFull + 2 * t + half), (uint32_t)pv_phase[t] & 1, abort_flag, kRoleMma, 20 + 2 * t + half))
          return false;
        tc_fence_after();
        const uint32_t d = tmem + 256u + (uint32_t)(t * 128);
        const uint32_t a = tmem + (uint32_t)(t * 128);
        const uint64_t b0 = sdesc(sKV + slot_v * kTileBytes, kBoxBytes, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int ks = half * 4 + kk;
          mma_ts_e(d, a + ks * 8, desc_add(b0, (uint32_t)(ks * 2048)), idesc_pv, (acc || ks > 0) ? 1u : 0u);
        }
        return true;
      };
      auto issue_pv = [&](int t, int slot_v, bool acc) -> bool {
        const bool r = issue_pv_half(t, 0, slot_v, acc) && issue_pv_half(t, 1, slot_v, acc);
        pv_phase[t]++;
        return r;
      };
      for (int it = 0; it < n_blocks && ok; ++it) {
        const int uk = 2 * it, slot_k = uk % kKvSlots;
        ok = mbar_wait_warp(bar(kBarKvFull + slot_k), (uk / kKvSlots) & 1, abort_flag, kRoleMma, 10 + slot_k);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t) {
          if (it > 0) {
            const int uv = 2 * (it - 1) + 1, slot_v = uv % kKvSlots;
            if (t == 0) {
              ok = mbar_wait_warp(bar(kBarKvFull + slot_v), (uv / kKvSlots) & 1, abort_flag, kRoleMma, 10 + slot_v);
              if (!ok) break;
            }
            if (!(ok = issue_pv(t, slot_v, it - 1 > 0))) break;
            if (t == 1) mma_commit_e(bar(kBarKvEmpty + slot_v));
          }
          issue_s(t, slot_k);
          mma_commit_e(bar(kBarSFull + t));
        }
        if (ok) mma_commit_e(bar(kBarKvEmpty + slot_k));
      }
      if (ok) {
        const int uv = 2 * (n_blocks - 1) + 1, slot_v = uv % kKvSlots;
        ok = mbar_wait_warp(bar(kBarKvFull + slot_v), (uv / kKvSlots) & 1, abort_flag, kRoleMma, 10 + slot_v);
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = issue_pv(t, slot_v, n_blocks - 1 > 0))) break;
          mma_commit_e(bar(kBarOFull + t));
        }
        if (ok) mma_commit_e(bar(kBarKvEmpty + slot_v));
      }
      // drain the tensor pipe before TMEM can be released
      mma_commit_e(bar(kBarDrain));
      mbar_wait_drain(bar(kBarDrain), 0);
    }
  } else {
    regs_inc<kRegsSoftmax>();
    // -------------------------------------------------------------- softmax
    const int t = warp >> 2;           // query tile
    const int wq = warp & 3;           // TMEM lane quadrant
    const uint32_t role = t ? kRoleSoftmax1 : kRoleSoftmax0;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + (uint32_t)(t * 128);
    const uint32_t tO = tmem + lane_base + 256u + (uint32_t)(t * 128);
    const float sl2 = p.scale_log2;
    const float thr = p.rescale_threshold;
    const int tail_valid = p.skv - (n_blocks - 1) * 128;  // 1..128
    float m_s = -INFINITY;  // running reference max, in scaled log2 units
    float l = 0.f;          // running row sum (relative to m_s)
    bool ok = true;
    for (int it = 0; it < n_blocks; ++it) {
      ok = mbar_wait(bar(kBarSFull + t), it & 1, abort_flag, role, 30 + t);
      if (!ok) break;
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
        // move the reference max only when the row max grew past the rescale
        // threshold (exact by max-shift invariance; rare after a few blocks)
        const bool need = mnew_s - m_s > thr;
        if (__any_sync(0xffffffffu, need)) {
          const float factor = need ? ex2_approx(m_s - mnew_s) : 1.f;
          if (need) {
            l *= factor;
            m_s = mnew_s;
          }
          // O_t holds the sum through block it-1 (its PV completed before S_t(it) was signalled)
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
      // P in two halves: the PV MMA on keys 0-63 starts while keys 64-127
      // are still being exponentiated
      const uint64_t sl2x2 = f2_pack(sl2, sl2), negx2 = f2_pack(-m_s, -m_s);
      float bsum = fwd_exp_half(s, 0, tS, sl2x2, negx2);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(bar(kBarPFull + 2 * t));
      bsum += fwd_exp_half(s, 2, tS, sl2x2, negx2);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(bar(kBarPFull + 2 * t + 1));
      l += bsum;
    }
    // ----------------------------------------------------------- epilogue
    if (ok) ok = mbar_wait(bar(kBarOFull + t), 0, abort_flag, role, 40 + t);
    if (ok) {
      tc_fence_after();
      const int row = m0 + t * 128 + wq * 32 + lane;
      const bool valid = row < p.sq;
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + (((size_t)b * p.sq + (valid ? row : 0)) * p.h + h) * 128;
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
        if (valid) {
#pragma unroll
          for (int v = 0; v < 4; ++v)
            st_global_v4(orow + c * 32 + v * 8, pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      if (valid) {
        // natural-log LSE; -inf when the row sum is zero or not finite
        const float lse = (l > 0.f && l == l) ? (m_s + log2f(l)) * 0.69314718055994531f : -INFINITY;
        p.lse[((size_t)b * p.h + h) * p.sq + row] = lse;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tmem, 512);
}

}  // namespace wf
