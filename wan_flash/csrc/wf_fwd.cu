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
//   work item = 2 query tiles of 128 rows (256 rows) of one (batch, head).
//   A work item walks one KV context, or two (the I2V text and image
//   contexts of the same query rows, kMode 2) as consecutive segments.
//   A CTA runs items blockIdx.x, blockIdx.x + gridDim.x, ...: one item per
//   CTA (grid = all items), or persistent (grid = SM count) for short KV
//   sequences, where the per-item prologue and epilogue would otherwise
//   leave the tensor pipe idle: the next item's Q load overlaps the current
//   item's last blocks and its first QK^T the current item's last PV.
//   warps 0-3  softmax for query tile 0  (thread = one query row)
//   warps 4-7  softmax for query tile 1
//   warp  8    tcgen05.mma issuer (converged warp, one elected lane per
//              instruction) + TMEM owner
//   warp  9    TMA producer (one thread)
//   warp  10   O store: one thread sends each staged O tile out with TMA
//   warp  11   idle (completes warpgroup 2 so it can give registers back)
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
constexpr uint32_t kOffOStage = kOffKV + kKvSlots * kTileBytes;  // one O tile (bf16, two swizzled boxes)
constexpr uint32_t kOffBar = kOffOStage + kTileBytes;
// barrier indices
constexpr int kBarQFull = 0;                     // + tile
constexpr int kBarQEmpty = 2;                    // + tile
constexpr int kBarKvFull = 4;                    // + slot
constexpr int kBarKvEmpty = kBarKvFull + kKvSlots;
constexpr int kBarSFull = kBarKvEmpty + kKvSlots;  // + tile
constexpr int kBarPFull = kBarSFull + 2;      // + 2 * tile + half (keys 0-63 / 64-127)
constexpr int kBarOFull = kBarPFull + 4;
constexpr int kBarDrain = kBarOFull + 2;
constexpr int kBarOStaged = kBarDrain + 1;       // O tile written to the stage (one arrival per warp)
constexpr int kBarOStageFree = kBarOStaged + 1;  // stage read by the tensor store
constexpr int kNumBars = kBarOStageFree + 1;
constexpr uint32_t kOffTmemHolder = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemHolder + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + alignment slack
}  // namespace fwd

size_t fwd_smem_bytes() { return fwd::kSmemBytes; }

// role ids recorded on a wait timeout
enum : uint32_t { kRoleSoftmax0 = 1, kRoleSoftmax1 = 2, kRoleMma = 3, kRoleLoad = 4, kRoleStore = 5 };

// Exponentials of half a 128-column block (two 32-column chunks starting at
// chunk c0) for this thread's row: P = 2^(s * scale_log2 - m) is stored to
// TMEM as bf16 pairs over the already-read S columns and the fp32 partial
// row sum is returned.  Packed f32x2 math keeps the instruction count low:
// the softmax warps share their SMSPs with the MMA-issuing warp, whose issue
// rate sets the tensor pipe's.
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
      const uint64_t pp = exp2_mufu2(x);
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

// kMode 0: one KV context; 1: one context whose ragged tail holds at most 64
// keys and runs as a 64-key block; 2: two KV contexts (segments) attended
// by the same query rows, each with its own softmax, output and LSE (the
// Wan I2V text + image cross attention), tail width decided per segment.
// Separate instantiations, so the common case carries none of the others.
template <int kMode>
__global__ void __launch_bounds__(fwd::kThreads, 1)
    wf_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k0,
                  const __grid_constant__ CUtensorMap tm_v0, const __grid_constant__ CUtensorMap tm_o0,
                  const __grid_constant__ CUtensorMap tm_k1, const __grid_constant__ CUtensorMap tm_v1,
                  const __grid_constant__ CUtensorMap tm_o1, FwdParams p) {
  using namespace fwd;
  // Segment loops stay rolled and per-segment parameters are read with
  // constant indices: an unrolled copy of the block loops, or the parameter
  // arrays copied to local memory for a run-time index, each cost the
  // two-context kernel 7-25 % against two one-context launches.
  constexpr int kSegs = (kMode == 2) ? 2 : 1;
  // a segment whose ragged tail holds at most 64 keys runs it 64 keys wide
  auto seg_narrow = [&](int seg) -> bool {
    if constexpr (kMode == 2)
      return (seg ? p.skv[1] : p.skv[0]) - ((seg ? p.n_blocks[1] : p.n_blocks[0]) - 1) * 128 <= 64;
    else
      return kMode == 1;
  };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmemHolder);

  const int warp = (int)warp_id();
  const int lane = (int)lane_id();
  // work item = 256 query rows (two 128-row tiles) of one (batch, head);
  // item i covers rows 256 * (i % n_pairs) of head (i / n_pairs) % h
  auto item_coords = [&](int item, int& m0, int& h, int& b) {
    const int pair = item % p.n_pairs;
    const int hb = item / p.n_pairs;
    m0 = pair * 256;
    h = hb % p.h;
    b = hb / p.h;
  };

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarQFull + t), 1);
      mbar_init(bar(kBarQEmpty + t), 1);
    }
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
    mbar_init(bar(kBarOStaged), 4);
    mbar_init(bar(kBarOStageFree), 1);
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

  if (warp == 11) {
    regs_dec<kRegsOther>();  // idle warp of warpgroup 2
  } else if (warp == 10) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------ O store
    // The softmax warps of tile 0 and tile 1 take turns on the one stage
    // buffer (item order, tile 0 first: the MMA completes O_0 of an item
    // before O_1, and O_1 before the next item's O_0).
    if (lane == 0) {
      tma_prefetch_desc(&tm_o0);
      if (kSegs > 1) tma_prefetch_desc(&tm_o1);
      int n = 0;  // tiles stored
      bool ok = true;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x) {
        int m0, h, b;
        item_coords(item, m0, h, b);
        #pragma unroll 1
        for (int seg = 0; seg < kSegs && ok; ++seg) {
          const CUtensorMap* tm_o = seg ? &tm_o1 : &tm_o0;
          for (int t = 0; t < 2; ++t, ++n) {
            ok = mbar_wait(bar(kBarOStaged), (uint32_t)n & 1, abort_flag, kRoleStore, 50 + t);
            if (!ok) break;
            for (int x = 0; x < 2; ++x)
              tma_store_4d(tm_o, sbase + kOffOStage + x * kBoxBytes, x * 64, m0 + t * 128, h, b);
            bulk_commit_group();
            bulk_wait_read_all();
            mbar_arrive(bar(kBarOStageFree));
          }
        }
      }
      bulk_wait_all();
    }
  } else if (warp == 9) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k0);
      tma_prefetch_desc(&tm_v0);
      if (kSegs > 1) {
        tma_prefetch_desc(&tm_k1);
        tma_prefetch_desc(&tm_v1);
      }
      int q_issued[2] = {0, 0};                // Q loads per tile buffer
      int issued[kKvSlots] = {0, 0, 0, 0};     // K/V loads per ring slot
      int u = 0;                               // K/V units (K and V of a block alternate)
      bool ok = true;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x) {
        int m0, h, b;
        item_coords(item, m0, h, b);
        #pragma unroll 1
        for (int seg = 0; seg < kSegs && ok; ++seg) {
        const int n_blocks = (seg ? p.n_blocks[1] : p.n_blocks[0]);
        const CUtensorMap* tm_k = seg ? &tm_k1 : &tm_k0;
        const CUtensorMap* tm_v = seg ? &tm_v1 : &tm_v0;
        for (int it = 0; it < n_blocks && ok; ++it) {
          const int j = (it == 0) ? (n_blocks - 1) : (it - 1);
          for (int kv = 0; kv < 2 && ok; ++kv, ++u) {  // 0 = K, 1 = V
            const int slot = u % kKvSlots;
            const int use = u / kKvSlots;
            if (use > 0) ok = mbar_wait(bar(kBarKvEmpty + slot), (use - 1) & 1, abort_flag, kRoleLoad, 100 + slot);
            if (!ok) break;
            mbar_expect_tx(bar(kBarKvFull + slot), kTileBytes);
            const CUtensorMap* tm = kv ? tm_v : tm_k;
            for (int x = 0; x < 2; ++x)
              tma_load_4d(sbase + kOffKV + slot * kTileBytes + x * kBoxBytes, tm, bar(kBarKvFull + slot),
                          x * 64, j * 128, h, b);
            issued[slot] = use + 1;
            if (seg == 0 && it == 0 && kv == 0) {
              // the item's Q tiles go between its first K and V: each buffer
              // is refilled once the previous item's last S MMA on it has
              // completed, which is after that item's last K arrived
              for (int t = 0; t < 2 && ok; ++t) {
                if (q_issued[t] > 0)
                  ok = mbar_wait(bar(kBarQEmpty + t), (q_issued[t] - 1) & 1, abort_flag, kRoleLoad, 90 + t);
                if (!ok) break;
                mbar_expect_tx(bar(kBarQFull + t), kTileBytes);
                for (int x = 0; x < 2; ++x)
                  tma_load_4d(sbase + kOffQ + t * kTileBytes + x * kBoxBytes, &tm_q, bar(kBarQFull + t), x * 64,
                              m0 + t * 128, h, b);
                q_issued[t]++;
              }
            }
          }
        }
        }
      }
      if (*abort_flag) {
        // drain: let every issued copy land before the CTA can exit
        for (int t = 0; t < 2; ++t)
          if (q_issued[t] > 0) mbar_wait_drain(bar(kBarQFull + t), (q_issued[t] - 1) & 1);
        for (int s = 0; s < kKvSlots; ++s)
          if (issued[s] > 0) mbar_wait_drain(bar(kBarKvFull + s), (issued[s] - 1) & 1);
      }
    }
  } else if (warp == 8) {
    regs_dec<kRegsOther>();
    // ------------------------------------------------------------------ MMA
    {  // converged warp: all lanes wait and form descriptors, elected lanes issue
      constexpr uint32_t idesc_qk = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_qk_narrow = idesc_bf16(128, 64, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16(128, 128, 0, 1);
      // a ragged tail of at most 64 keys (e.g. 257 = 2 x 128 + 1) runs as a
      // 64-key block: QK^T with N = 64 and PV over keys 0-63 only
      const uint32_t sQ = sbase + kOffQ;
      const uint32_t sKV = sbase + kOffKV;
      bool ok = true;
      int pv_phase[2] = {0, 0};
      auto issue_s = [&](int t, int slot_k, bool narrow) {
        const uint32_t d = tmem + (uint32_t)(t * 128);
        const uint64_t a0 = sdesc(sQ + t * kTileBytes, 16, 1024);
        const uint64_t b0 = sdesc(sKV + slot_k * kTileBytes, 16, 1024);
        const uint32_t idesc = narrow ? idesc_qk_narrow : idesc_qk;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * kBoxBytes + (ks & 3) * 32);
          mma_ss_e(d, desc_add(a0, off), desc_add(b0, off), idesc, ks > 0);
        }
      };
      // O_t += P_t V over keys [64*half, 64*half + 64) once that half of P_t
      // has been written (P_t: bf16 pairs in S_t columns [0, 64))
      auto issue_pv_half = [&](int t, int half, int slot_v, bool acc, bool narrow) -> bool {
        if (!mbar_wait_warp(bar(kBarPFull + 2 * t + half), (uint32_t)pv_phase[t] & 1, abort_flag, kRoleMma, 20 + 2 * t + half))
          return false;
        if (narrow && half == 1) return true;  // keys 64-127 of a narrow tail do not exist
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
      auto issue_pv = [&](int t, int slot_v, bool acc, bool narrow) -> bool {
        const bool r = issue_pv_half(t, 0, slot_v, acc, narrow) && issue_pv_half(t, 1, slot_v, acc, narrow);
        pv_phase[t]++;
        return r;
      };
      // One flat pipeline over the blocks of all this CTA's items: global
      // block g issues PV_t(g-1) before S_t(g) for each tile, so the last PV
      // of an item interleaves with the first QK^T of the next one.
      int g = 0;                 // blocks issued so far (K of block g = unit 2g, V = 2g+1)
      int prev_it = 0;           // position of block g-1 within its segment
      bool prev_last = false;    // block g-1 ends its segment: its PV completes O
      bool prev_narrow = false;  // block g-1 is a 64-key-wide tail
      int n_items_done = 0;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x, ++n_items_done) {
        #pragma unroll 1
        for (int seg = 0; seg < kSegs && ok; ++seg) {
        const int n_blocks = (seg ? p.n_blocks[1] : p.n_blocks[0]);
        const bool narrow_tail = seg_narrow(seg);
        for (int it = 0; it < n_blocks && ok; ++it, ++g) {
          const int uk = 2 * g, slot_k = uk % kKvSlots;
          ok = mbar_wait_warp(bar(kBarKvFull + slot_k), (uk / kKvSlots) & 1, abort_flag, kRoleMma, 10 + slot_k);
          if (!ok) break;
          tc_fence_after();
          for (int t = 0; t < 2 && ok; ++t) {
            if (g > 0) {
              const int uv = 2 * (g - 1) + 1, slot_v = uv % kKvSlots;
              if (t == 0) {
                ok = mbar_wait_warp(bar(kBarKvFull + slot_v), (uv / kKvSlots) & 1, abort_flag, kRoleMma, 10 + slot_v);
                if (!ok) break;
              }
              if (!(ok = issue_pv(t, slot_v, prev_it > 0, prev_narrow))) break;
              if (prev_last) mma_commit_e(bar(kBarOFull + t));
              if (t == 1) mma_commit_e(bar(kBarKvEmpty + slot_v));
            }
            if (seg == 0 && it == 0) {
              ok = mbar_wait_warp(bar(kBarQFull + t), (uint32_t)n_items_done & 1, abort_flag, kRoleMma, t);
              if (!ok) break;
              tc_fence_after();
            }
            issue_s(t, slot_k, it == 0 && narrow_tail);
            mma_commit_e(bar(kBarSFull + t));
            if (seg == kSegs - 1 && it == n_blocks - 1) mma_commit_e(bar(kBarQEmpty + t));
          }
          if (ok) mma_commit_e(bar(kBarKvEmpty + slot_k));
          prev_it = it;
          prev_last = (it == n_blocks - 1);
          prev_narrow = (it == 0) && narrow_tail;
        }
        }
      }
      if (ok && g > 0) {
        const int uv = 2 * (g - 1) + 1, slot_v = uv % kKvSlots;
        ok = mbar_wait_warp(bar(kBarKvFull + slot_v), (uv / kKvSlots) & 1, abort_flag, kRoleMma, 10 + slot_v);
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = issue_pv(t, slot_v, prev_it > 0, prev_narrow))) break;
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
    bool ok = true;
    int s_waits = 0;     // S_t tiles consumed (SFull_t phase)
    int n_segs_done = 0;
    for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x) {
      #pragma unroll 1
      for (int seg = 0; seg < kSegs && ok; ++seg, ++n_segs_done) {
      const int n_blocks = (seg ? p.n_blocks[1] : p.n_blocks[0]);
      const int tail_valid = (seg ? p.skv[1] : p.skv[0]) - (n_blocks - 1) * 128;  // 1..128
      float m_s = -INFINITY;  // running reference max, in scaled log2 units
      float l = 0.f;          // running row sum (relative to m_s)
      int it0 = 0;
      if (kMode != 0 && seg_narrow(seg)) {
        // the ragged tail holds at most 64 keys: S columns 0-63 only, one P
        // half (the MMA warp skips PV over keys 64-127)
        ok = mbar_wait(bar(kBarSFull + t), (uint32_t)s_waits & 1, abort_flag, role, 30 + t);
        if (!ok) break;
        ++s_waits;
        tc_fence_after();
        uint32_t s[4][32];
        tmem_ld32(tS, s[0]);
        tmem_ld32(tS + 32, s[1]);
        tmem_wait_ld();
        reg_fence32(s[0]);
        reg_fence32(s[1]);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i >= tail_valid) s[c][i] = __float_as_uint(-INFINITY);
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 16; ++i)
            mx[i & 1] = fmax3(mx[i & 1], __uint_as_float(s[c][2 * i]), __uint_as_float(s[c][2 * i + 1]));
        m_s = fmaxf(mx[0], mx[1]) * sl2;
        const uint64_t sl2x2 = f2_pack(sl2, sl2), negx2 = f2_pack(-m_s, -m_s);
        l = fwd_exp_half(s, 0, tS, sl2x2, negx2);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive_warp(bar(kBarPFull + 2 * t));
        mbar_arrive_warp(bar(kBarPFull + 2 * t + 1));
        it0 = 1;
      }
      for (int it = it0; it < n_blocks; ++it, ++s_waits) {
        ok = mbar_wait(bar(kBarSFull + t), (uint32_t)s_waits & 1, abort_flag, role, 30 + t);
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
        // are still being exponentiated.  The arrivals also tell the MMA warp
        // that this item's O_t readout (the epilogue below, in program order
        // before the next item's first P) is complete.
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
      // --------------------------------------------------------- epilogue
      if (ok) ok = mbar_wait(bar(kBarOFull + t), (uint32_t)n_segs_done & 1, abort_flag, role, 40 + t);
      if (!ok) break;
      tc_fence_after();
      int m0, h, b;
      item_coords(item, m0, h, b);
      const int r = wq * 32 + lane;  // row within the tile
      const int row = m0 + t * 128 + r;
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      // O_t / l as bf16 into the stage (two 128B-swizzled boxes of 64
      // columns, the tensor store's layout) once the previous tile's store
      // has read it
      const int use = 2 * n_segs_done + t;
      if (use > 0) ok = mbar_wait(bar(kBarOStageFree), (uint32_t)(use - 1) & 1, abort_flag, role, 45 + t);
      if (!ok) break;
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
          st_shared_v4(stage + (uint32_t)(c >> 1) * kBoxBytes + ((chunk ^ ((uint32_t)r & 7u)) << 4), pk[4 * v],
                       pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarOStaged));
      if (row < p.sq) {
        // natural-log LSE; -inf when the row sum is zero or not finite
        const float lse = (l > 0.f && l == l) ? (m_s + log2f(l)) * 0.69314718055994531f : -INFINITY;
        (seg ? p.lse[1] : p.lse[0])[((size_t)b * p.h + h) * p.sq + row] = lse;
      }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tmem, 512);
}

#define WF_FWD_INSTANTIATE(MODE)                                                                            \
  template __global__ void wf_fwd_kernel<MODE>(                                                                   \
      const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap, \
      const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap, \
      const __grid_constant__ CUtensorMap, FwdParams);
WF_FWD_INSTANTIATE(0)
WF_FWD_INSTANTIATE(1)
WF_FWD_INSTANTIATE(2)
#undef WF_FWD_INSTANTIATE

}  // namespace wf
