// Memory-bound kernels of the backward chain: the preprocess (rowsum(O*dO),
// lse -> -lse*log2(e), zero the dQ accumulator) and the fp32-accumulator ->
// bf16 convert.  Both are plain coalesced loads/stores sized for HBM.
//
// Reference counterparts (Quarky93/wan-flash): WanFlashBwdPreprocessSm90,
// wan_flash/bwd_sm90.py:99-235 (D at :195-217, zero dQaccum :219-228,
// lse_log2 with +inf pad rows and -inf -> 0 at :230-235; stored negated here,
// so pad rows hold -inf and the main kernel needs one fused multiply-add per
// exponent) and
// WanFlashBwdPostprocessSm90, wan_flash/bwd_sm90.py:1140-1308.  The
// accumulator here is stored in 128-row tiles of [2 row halves][32 groups of
// 4 columns][64 rows][4] (each 64-row half is one contiguous 32 KB run, the
// unit the backward main kernels reduce into), not the reference's WGMMA
// fragment order.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float bf16_dot2(uint32_t a, uint32_t b) {
  const float a0 = __uint_as_float(a << 16), a1 = __uint_as_float(a & 0xFFFF0000u);
  const float b0 = __uint_as_float(b << 16), b1 = __uint_as_float(b & 0xFFFF0000u);
  return fmaf(a0, b0, a1 * b1);
}

// grid (sq_rounded / 64, h, b), 256 threads: 16 threads per row (8 bf16 each),
// 16 rows per pass, 4 passes.
__global__ void __launch_bounds__(256) wf_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o,
                                                         const __nv_bfloat16* __restrict__ dO,
                                                         const float* __restrict__ lse, float* __restrict__ dpsum,
                                                         float* __restrict__ neg_lse_log2,
                                                         float* __restrict__ dq_accum, int sq, int sq_rounded,
                                                         int h_total) {
  // the main kernel (launched as a programmatic dependent) may be scheduled
  // as soon as every CTA of this grid is running; it waits for this grid's
  // completion before reading what is written here
  griddep_launch_dependents();
  const int h = blockIdx.y, b = blockIdx.z;
  const size_t bh = (size_t)b * h_total + h;
  const int row0 = blockIdx.x * 64;
  const int sub = threadIdx.x & 15;
  const int rr = threadIdx.x >> 4;
#pragma unroll
  for (int pass = 0; pass < 4; ++pass) {
    const int s = row0 + pass * 16 + rr;
    float acc = 0.f;
    if (s < sq) {
      const size_t off = (((size_t)b * sq + s) * h_total + h) * 128 + sub * 8;
      const uint4 a = ldg_u4(o + off);
      const uint4 c = ldg_u4(dO + off);
      acc = bf16_dot2(a.x, c.x) + bf16_dot2(a.y, c.y) + bf16_dot2(a.z, c.z) + bf16_dot2(a.w, c.w);
    }
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (sub == 0) {
      float nl2 = -INFINITY;  // pad rows: P = exp2(-inf) = 0
      if (s < sq) {
        const float l = lse[bh * sq + s];
        nl2 = (l == -INFINITY) ? 0.f : -(l * 1.4426950408889634f);
      }
      dpsum[bh * sq_rounded + s] = acc;
      neg_lse_log2[bh * sq_rounded + s] = nl2;
    }
  }
  // zero rows [row0, row0 + 64) of the tiled dQ accumulator: one 64-row half,
  // a contiguous 32 KB run (no accumulator: a second KV context's
  // preprocess, adding into one the first context's call zeroed)
  if (dq_accum == nullptr) return;
  const int m = row0 >> 7, half = (row0 >> 6) & 1;
  float4* run = reinterpret_cast<float4*>(dq_accum + (bh * (size_t)(sq_rounded >> 7) + m) * 16384 + half * 8192);
#pragma unroll
  for (int i = 0; i < 8; ++i) run[threadIdx.x + i * 256] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// grid (s_rounded / 32, h, b), 256 threads; tile of 32 rows x 128 columns.
__global__ void __launch_bounds__(256) wf_convert_kernel(const float* __restrict__ accum,
                                                         __nv_bfloat16* __restrict__ out, float scale, int s_len,
                                                         int s_rounded, int h_total) {
  __shared__ float tile[32][132];
  // launched as a programmatic dependent of the kernel that filled `accum`
  // (the backward main kernel, or the previous convert): wait for it
  griddep_launch_dependents();
  griddep_wait();
  const int h = blockIdx.y, b = blockIdx.z;
  const size_t bh = (size_t)b * h_total + h;
  const int row0 = blockIdx.x * 32;
  const int m = row0 >> 7, half = (row0 >> 6) & 1, r0 = row0 & 63;
  const float4* src =
      reinterpret_cast<const float4*>(accum + (bh * (size_t)(s_rounded >> 7) + m) * 16384 + half * 8192);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + i * 256;  // 0..1023 = 32 groups x 32 rows
    const int g = idx >> 5, rw = idx & 31;
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(src + g * 64 + r0 + rw));
    tile[rw][4 * g + 0] = v.x;
    tile[rw][4 * g + 1] = v.y;
    tile[rw][4 * g + 2] = v.z;
    tile[rw][4 * g + 3] = v.w;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int idx = threadIdx.x + i * 256;  // 0..511 = 32 rows x 16 chunks of 8
    const int rw = idx >> 4, ch = idx & 15;
    const int s = row0 + rw;
    if (s < s_len) {
      const float* t = &tile[rw][ch * 8];
      uint4 w;
      w.x = pack_bf16(t[0] * scale, t[1] * scale);
      w.y = pack_bf16(t[2] * scale, t[3] * scale);
      w.z = pack_bf16(t[4] * scale, t[5] * scale);
      w.w = pack_bf16(t[6] * scale, t[7] * scale);
      *reinterpret_cast<uint4*>(out + (((size_t)b * s_len + s) * h_total + h) * 128 + ch * 8) = w;
    }
  }
}

}  // namespace wf
