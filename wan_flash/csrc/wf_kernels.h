// Kernel parameter blocks and launch-side declarations shared by the kernel
// translation units and the C ABI (wf_capi.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

namespace wf {

struct FwdParams {
  float* lse[2];           // per KV segment: (b, h, sq) natural-log LSE
  int sq, h;
  int skv[2];              // per KV segment (segment 1 only in the two-context kernel)
  int n_blocks[2];         // ceil(skv / 128)
  int n_pairs;             // ceil(sq / 256): work items per (batch, head)
  int n_items;             // b * h * n_pairs
  float scale_log2;        // log2(e) / sqrt(128)
  float rescale_threshold; // log2 units
};

struct BwdParams {
  const float* neg_lse_log2;  // (b, h, sq_rounded): -lse * log2(e), -inf on pad rows
  const float* dpsum;      // (b, h, sq_rounded)
  float* dq_accum;         // tiled, b*h*sq_rounded*128
  void* dk;                // bf16 (b, skv, h, 128) or fp32 tiled accumulator
  void* dv;
  int sq, skv, h;
  int sq_rounded, m_blocks, n_blocks, skv_rounded;
  int n_blocks_padded;     // n_blocks rounded up to the 2-CTA cluster size
  int accum_dkv;           // 1: dk/dv are fp32 tiled accumulators (split-M)
  int m_chunk;             // split-M: m-blocks per CTA
  float scale;             // 1/sqrt(128)
  float scale_log2;        // log2(e)/sqrt(128)
  int* dq_sem;             // deterministic: (b*h, m_blocks) dQ contributions added so far
  int* dkv_sem;            // deterministic, split-M: (b*h, n_blocks) splits added so far
  int deterministic;
  int wave;                // CTAs resident at once (one per SM): the serpentine walk's period
};

template <int kMode>
__global__ void wf_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k0,
                              const __grid_constant__ CUtensorMap tm_v0, const __grid_constant__ CUtensorMap tm_o0,
                              const __grid_constant__ CUtensorMap tm_k1, const __grid_constant__ CUtensorMap tm_v1,
                              const __grid_constant__ CUtensorMap tm_o1, FwdParams p);
__global__ void wf_fwd2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k64,
                               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                               FwdParams p);
__global__ void wf_bwd_main_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                                   BwdParams p);
__global__ void wf_bwd2_main_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_q64,
                                    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                                    const __grid_constant__ CUtensorMap tm_do,
                                    const __grid_constant__ CUtensorMap tm_do64, BwdParams p);
__global__ void wf_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dO,
                                  const float* __restrict__ lse, float* __restrict__ dpsum,
                                  float* __restrict__ neg_lse_log2, float* __restrict__ dq_accum, int sq,
                                  int sq_rounded, int h);
__global__ void wf_convert_kernel(const float* __restrict__ accum, __nv_bfloat16* __restrict__ out, float scale,
                                  int s, int s_rounded, int h);

size_t fwd_smem_bytes();
size_t fwd2_smem_bytes();
size_t bwd_smem_bytes();
size_t bwd2_smem_bytes();

// wf_fwd with cluster_m = 0 (auto), one KV context, one item per CTA: true =
// the CTA-pair kernel.
constexpr bool kFwdPairDefault = true;
// wf_bwd_main with cluster_n = 0 (auto): true = the CTA-pair kernel.
constexpr bool kBwdPairDefault = false;

constexpr int kFwdThreads = 384;
// wf_fwd with scheduler = 0 (auto): persistent grid when KV has at most this
// many 128-key blocks.
constexpr int kFwdPersistMaxBlocks = 64;
constexpr int kBwdThreads = 512;

}  // namespace wf
