// C ABI of the Wan attention hot path (declared in include/wan_flash.h).
//
// Host side of each launch: argument checks, TMA tensor-map encoding
// (driver entry point fetched through the runtime, so the library has no
// link-time dependency on libcuda), one-time per-device kernel attributes,
// and the launch on the caller's stream.  Nothing here allocates device
// memory: every buffer is the caller's.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "wan_flash.h"
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

namespace {

thread_local char t_last_error[512] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(WF_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
EncodeTiledFn g_encode = nullptr;
constexpr int kMaxDevices = 64;
bool g_dev_ready[kMaxDevices] = {false};
int g_dev_sms[kMaxDevices] = {0};

int get_encode(EncodeTiledFn* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(WF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable (%s)", cudaGetErrorName(e));
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = g_encode;
  return WF_OK;
}

// Per-device one-time set-up: verify sm_100, record the SM count, opt the
// big kernels into their dynamic shared memory.
int device_setup(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(WF_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  *dev_out = dev;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_dev_ready[dev]) return WF_OK;
  int major = 0, minor = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10 || minor != 0)
    return fail(WF_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major, minor);
  e = cudaFuncSetAttribute(wf_fwd_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fwd smem)");
  e = cudaFuncSetAttribute(wf_fwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fwd narrow smem)");
  e = cudaFuncSetAttribute(wf_fwd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fwd dual smem)");
  e = cudaFuncSetAttribute(wf_fwd2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd2_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fwd pair smem)");
  e = cudaFuncSetAttribute(wf_bwd_main_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bwd_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bwd smem)");
  e = cudaFuncSetAttribute(wf_bwd2_main_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bwd2_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bwd pair smem)");
  g_dev_sms[dev] = sms;
  g_dev_ready[dev] = true;
  return WF_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 4-D map over a contiguous (b, s, h, 128) bf16 tensor: dims {d, s, h, b},
// box {64, rows, 1, 1} with the 128-byte swizzle (rows x 128-byte box).
int make_bshd_map(CUtensorMap* map, const void* ptr, int b, int s, int h, int rows = 128) {
  EncodeTiledFn enc;
  int rc = get_encode(&enc);
  if (rc) return rc;
  const cuuint64_t dims[4] = {128, (cuuint64_t)s, (cuuint64_t)h, (cuuint64_t)b};
  const cuuint64_t strides[3] = {(cuuint64_t)h * 256, 256, (cuuint64_t)s * h * 256};
  const cuuint32_t box[4] = {64, (cuuint32_t)rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for (%d,%d,%d,128)", (int)r, b, s, h);
  return WF_OK;
}

int check_dims(int b, int s1, int s2, int h) {
  if (b < 0 || s1 < 0 || s2 < 0 || h < 0) return fail(WF_ERR_INVALID_ARG, "negative size");
  if (h > 65535 || b > 65535) return fail(WF_ERR_UNSUPPORTED, "h=%d / b=%d exceed the grid limits", h, b);
  // TMA coordinates and strides: s*h*256 must stay below 2^40
  if ((double)s1 * h * 256.0 >= 1099511627776.0 || (double)s2 * h * 256.0 >= 1099511627776.0)
    return fail(WF_ERR_UNSUPPORTED, "sequence too long for a TMA stride");
  return WF_OK;
}

// Launch through cudaLaunchKernelEx with programmatic stream serialization
// (programmatic dependent launch: the kernel may start while the previous
// kernel of the stream finishes; it calls griddep_wait() before touching that
// kernel's results) and, for cluster_x > 1, a 1-D cluster.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  lc.attrs = attr;
  lc.numAttrs = n;
  return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return WF_OK;
}

}  // namespace

// Self-test of the bounded-wait machinery: one thread waits on an mbarrier that
// nothing arrives on.  No copies or MMAs are in flight, so the expiry path is
// exercised without any risk to the context.
__global__ void wf_selftest_wait_kernel() {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, 99u, 99u);
}

// Forward over one KV context, or two contexts attended by the same query
// rows (each with its own softmax, output and LSE) in one launch.
static int fwd_launch(const void* q, int n_ctx, const void* const* k, const void* const* v, void* const* o,
                      float* const* lse, const int* skv, int b, int sq, int h, const wf_fwd_cfg* cfg,
                      void* stream) {
  int rc;
  for (int c = 0; c < n_ctx; ++c)
    if ((rc = check_dims(b, sq, skv[c], h))) return rc;
  if (b == 0 || sq == 0 || h == 0) return WF_OK;
  if (!q) return fail(WF_ERR_INVALID_ARG, "null pointer");
  for (int c = 0; c < n_ctx; ++c) {
    if (skv[c] == 0) return fail(WF_ERR_UNSUPPORTED, "skv == 0: attention over an empty key set");
    if (!k[c] || !v[c] || !o[c] || !lse[c]) return fail(WF_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(q) || !aligned16(k[c]) || !aligned16(v[c]) || !aligned16(o[c]) ||
        (reinterpret_cast<uintptr_t>(lse[c]) & 3))
      return fail(WF_ERR_MISALIGNED, "q/k/v/o must be 16-byte aligned and lse 4-byte aligned");
  }
  int dev;
  if ((rc = device_setup(&dev))) return rc;
  CUtensorMap mq, mk[2], mv[2], mo[2];
  if ((rc = make_bshd_map(&mq, q, b, sq, h))) return rc;
  for (int c = 0; c < n_ctx; ++c)
    if ((rc = make_bshd_map(&mk[c], k[c], b, skv[c], h)) || (rc = make_bshd_map(&mv[c], v[c], b, skv[c], h)) ||
        (rc = make_bshd_map(&mo[c], o[c], b, sq, h)))
      return rc;
  if (n_ctx == 1) {  // the one-context kernels never read the second segment's maps
    mk[1] = mk[0];
    mv[1] = mv[0];
    mo[1] = mo[0];
  }
  FwdParams p;
  p.sq = sq;
  p.h = h;
  int total_blocks = 0;
  for (int c = 0; c < 2; ++c) {
    const int cc = c < n_ctx ? c : 0;
    p.lse[c] = lse[cc];
    p.skv[c] = skv[cc];
    p.n_blocks[c] = (skv[cc] + 127) / 128;
    if (c < n_ctx) total_blocks += p.n_blocks[c];
  }
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  p.rescale_threshold = cfg ? cfg->rescale_threshold : 8.0f;
  p.n_pairs = (sq + 255) / 256;
  const long long n_items = (long long)p.n_pairs * h * b;
  if (n_items > 0x7fffffffLL) return fail(WF_ERR_UNSUPPORTED, "%lld work items exceed the grid limit", n_items);
  p.n_items = (int)n_items;
  const int sched = cfg ? cfg->scheduler : 0;
  if (sched < 0 || sched > 2) return fail(WF_ERR_INVALID_ARG, "scheduler %d not in {0, 1, 2}", sched);
  if (cfg && cfg->num_sms < 0) return fail(WF_ERR_INVALID_ARG, "num_sms %d < 0", cfg->num_sms);
  const int sms = (cfg && cfg->num_sms > 0) ? cfg->num_sms : g_dev_sms[dev];
  const bool persistent = sched == 2 || (sched == 0 && total_blocks <= kFwdPersistMaxBlocks);
  const int grid = persistent ? (int)std::min<long long>(n_items, sms) : p.n_items;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int cluster_m = cfg ? cfg->cluster_m : 0;
  if (cluster_m < 0 || cluster_m > 2) return fail(WF_ERR_INVALID_ARG, "cluster_m %d not in {0, 1, 2}", cluster_m);
  if (cluster_m == 2 && (n_ctx != 1 || persistent))
    return fail(WF_ERR_UNSUPPORTED, "cluster_m = 2 needs one KV context and the one-item-per-CTA schedule");
  if (n_ctx == 1 && !persistent && (cluster_m == 2 || (cluster_m == 0 && kFwdPairDefault))) {
    // CTA pairs: one cluster of 2 per 512 query rows of a (batch, head)
    CUtensorMap mk64;
    if ((rc = make_bshd_map(&mk64, k[0], b, skv[0], h, 64))) return rc;
    const long long n_cl = (long long)((p.n_pairs + 1) / 2) * h * b;
    if (2 * n_cl > 0x7fffffffLL) return fail(WF_ERR_UNSUPPORTED, "%lld clusters exceed the grid limit", n_cl);
    cudaError_t e = launch_ex(wf_fwd2_kernel, dim3((unsigned)(2 * n_cl)), dim3(kFwdThreads), fwd2_smem_bytes(), st,
                              false, 2u, mq, mk64, mv[0], mo[0], p);
    if (e != cudaSuccess) return cuda_fail(e, "wf_fwd pair launch");
    return launch_check("wf_fwd pair launch");
  }
  const size_t smem = fwd_smem_bytes();
  if (n_ctx == 2)
    wf_fwd_kernel<2><<<grid, kFwdThreads, smem, st>>>(mq, mk[0], mv[0], mo[0], mk[1], mv[1], mo[1], p);
  else if (skv[0] - (p.n_blocks[0] - 1) * 128 <= 64)
    wf_fwd_kernel<1><<<grid, kFwdThreads, smem, st>>>(mq, mk[0], mv[0], mo[0], mk[1], mv[1], mo[1], p);
  else
    wf_fwd_kernel<0><<<grid, kFwdThreads, smem, st>>>(mq, mk[0], mv[0], mo[0], mk[1], mv[1], mo[1], p);
  return launch_check("wf_fwd launch");
}

}  // namespace wf

using namespace wf;

extern "C" {

int wf_version(void) { return 100; }

int wf_last_error(char* buf, int len) {
  if (!buf || len <= 0) return WF_ERR_INVALID_ARG;
  snprintf(buf, (size_t)len, "%s", t_last_error);
  return WF_OK;
}

int wf_num_sms(void) {
  int dev = 0;
  if (device_setup(&dev)) return 0;
  return g_dev_sms[dev];
}

int wf_set_wait_limit_ns(unsigned long long ns) {
  if (ns == 0) return fail(WF_ERR_INVALID_ARG, "wait limit must be > 0");
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(wait limit)");
  return WF_OK;
}

int wf_device_status(unsigned int* info) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned int code = 0, inf[4] = {0, 0, 0, 0};
  e = cudaMemcpyFromSymbol(&code, g_err_code, sizeof(code));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(err)");
  e = cudaMemcpyFromSymbol(inf, g_err_info, sizeof(inf));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(info)");
  if (info) memcpy(info, inf, sizeof(inf));
  if (code != 0) {
    const unsigned int zero[5] = {0, 0, 0, 0, 0};
    cudaMemcpyToSymbol(g_err_code, zero, sizeof(unsigned int));
    cudaMemcpyToSymbol(g_err_info, zero + 1, sizeof(inf));
    return fail((int)code, "device error %d: block (%u,%u,%u) role %u tag %u", (int)code, inf[0] & 0xFFFF,
                inf[0] >> 16, inf[1], inf[2], inf[3]);
  }
  return WF_OK;
}

int wf_selftest_wait_timeout(unsigned long long limit_ns, unsigned int* info) {
  int dev, rc;
  if ((rc = device_setup(&dev))) return rc;
  if ((rc = wf_device_status(nullptr))) return rc;  // start from a clean error word
  unsigned long long old_limit = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&old_limit, g_wait_limit_ns, sizeof(old_limit));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(wait limit)");
  if ((rc = wf_set_wait_limit_ns(limit_ns))) return rc;
  wf_selftest_wait_kernel<<<1, 32>>>();
  e = cudaGetLastError();
  const int status = (e == cudaSuccess) ? wf_device_status(info) : cuda_fail(e, "selftest launch");
  const int rc2 = wf_set_wait_limit_ns(old_limit);
  return status != WF_OK ? status : rc2;
}

int wf_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int b, int sq, int skv, int h,
           const wf_fwd_cfg* cfg, void* stream) {
  const void* ks[1] = {k};
  const void* vs[1] = {v};
  void* os[1] = {o};
  float* lses[1] = {lse};
  const int skvs[1] = {skv};
  return fwd_launch(q, 1, ks, vs, os, lses, skvs, b, sq, h, cfg, stream);
}

int wf_fwd_dual(const void* q, const void* k0, const void* v0, const void* k1, const void* v1, void* o0, void* o1,
                float* lse0, float* lse1, int b, int sq, int skv0, int skv1, int h, const wf_fwd_cfg* cfg,
                void* stream) {
  const void* ks[2] = {k0, k1};
  const void* vs[2] = {v0, v1};
  void* os[2] = {o0, o1};
  float* lses[2] = {lse0, lse1};
  const int skvs[2] = {skv0, skv1};
  return fwd_launch(q, 2, ks, vs, os, lses, skvs, b, sq, h, cfg, stream);
}

int wf_bwd_pre(const void* o, const void* dO, const float* lse, float* dpsum, float* neg_lse_log2, float* dq_accum, int b,
               int sq, int sq_rounded, int h, void* stream) {
  int rc = check_dims(b, sq, sq_rounded, h);
  if (rc) return rc;
  if (sq_rounded != (sq + 127) / 128 * 128) return fail(WF_ERR_INVALID_ARG, "sq_rounded must be ceil(sq/128)*128");
  if (b == 0 || sq == 0 || h == 0) return WF_OK;
  if (!o || !dO || !lse || !dpsum || !neg_lse_log2) return fail(WF_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(o) || !aligned16(dO) || !aligned16(dpsum) || !aligned16(neg_lse_log2) ||
      (dq_accum && !aligned16(dq_accum)))
    return fail(WF_ERR_MISALIGNED, "o/dO/dpsum/neg_lse_log2/dq_accum must be 16-byte aligned");
  int dev;
  if ((rc = device_setup(&dev))) return rc;
  dim3 grid(sq_rounded / 64, h, b);
  wf_bwd_pre_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(dO), lse, dpsum, neg_lse_log2,
      dq_accum, sq, sq_rounded, h);
  return launch_check("wf_bwd_pre launch");
}

int wf_bwd_main(const void* q, const void* k, const void* v, const void* dO, const float* neg_lse_log2,
                const float* dpsum, float* dq_accum, void* dk, void* dv, int b, int sq, int skv, int h,
                const wf_bwd_cfg* cfg, void* stream) {
  int rc = check_dims(b, sq, skv, h);
  if (rc) return rc;
  if (b == 0 || h == 0 || skv == 0) return WF_OK;
  if (sq == 0) return fail(WF_ERR_UNSUPPORTED, "sq == 0: the caller must zero dk/dv");
  if (!q || !k || !v || !dO || !neg_lse_log2 || !dpsum || !dq_accum || !dk || !dv)
    return fail(WF_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dO) || !aligned16(neg_lse_log2) ||
      !aligned16(dpsum) || !aligned16(dq_accum) || !aligned16(dk) || !aligned16(dv))
    return fail(WF_ERR_MISALIGNED, "all buffers must be 16-byte aligned");
  const int nsplit = cfg ? cfg->nsplit : 1;
  const int cluster_n = cfg ? cfg->cluster_n : 0;
  if (cluster_n < 0 || cluster_n > 2) return fail(WF_ERR_INVALID_ARG, "cluster_n=%d must be 0 (auto), 1 or 2", cluster_n);
  const int deterministic = cfg ? cfg->deterministic : 0;
  const bool pdl = !(cfg && cfg->pdl_off);
  if (deterministic && (!cfg->sem || (reinterpret_cast<uintptr_t>(cfg->sem) & 3)))
    return fail(WF_ERR_INVALID_ARG, "deterministic mode needs a 4-byte aligned sem workspace");
  if (deterministic && cluster_n == 2)
    return fail(WF_ERR_UNSUPPORTED, "deterministic mode runs on the single-CTA kernel (cluster_n 0 or 1)");
  int dev;
  if ((rc = device_setup(&dev))) return rc;
  BwdParams p;
  p.neg_lse_log2 = neg_lse_log2;
  p.dpsum = dpsum;
  p.dq_accum = dq_accum;
  p.dk = dk;
  p.dv = dv;
  p.sq = sq;
  p.skv = skv;
  p.h = h;
  p.m_blocks = (sq + 127) / 128;
  p.sq_rounded = p.m_blocks * 128;
  p.n_blocks = (skv + 127) / 128;
  p.skv_rounded = p.n_blocks * 128;
  if (nsplit < 1 || nsplit > p.m_blocks) return fail(WF_ERR_INVALID_ARG, "nsplit=%d outside [1, %d]", nsplit, p.m_blocks);
  p.m_chunk = (p.m_blocks + nsplit - 1) / nsplit;
  p.accum_dkv = nsplit > 1 ? 1 : 0;
  p.scale = (float)(1.0 / std::sqrt(128.0));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  p.deterministic = deterministic ? 1 : 0;
  p.wave = g_dev_sms[dev];
  p.dq_sem = deterministic ? cfg->sem : nullptr;
  p.dkv_sem = deterministic ? cfg->sem + (size_t)b * h * p.m_blocks : nullptr;
  CUtensorMap mq, mk, mv, mdo;
  if ((rc = make_bshd_map(&mq, q, b, sq, h)) || (rc = make_bshd_map(&mk, k, b, skv, h)) ||
      (rc = make_bshd_map(&mv, v, b, skv, h)) || (rc = make_bshd_map(&mdo, dO, b, sq, h)))
    return rc;
  const int splits = (p.m_blocks + p.m_chunk - 1) / p.m_chunk;  // every split owns >= 1 m-block
  const bool use_pair = !deterministic && (cluster_n == 0 ? kBwdPairDefault : cluster_n == 2);
  if (!use_pair) {
    p.n_blocks_padded = p.n_blocks;
    dim3 grid(p.n_blocks * splits, h, b);
    cudaError_t e = launch_ex(wf_bwd_main_kernel, grid, dim3(kBwdThreads), bwd_smem_bytes(),
                              reinterpret_cast<cudaStream_t>(stream), pdl, 1u, mq, mk, mv, mdo, p);
    if (e != cudaSuccess) return cuda_fail(e, "wf_bwd_main launch");
    return launch_check("wf_bwd_main launch");
  }
  // CTA pairs over adjacent KV blocks (cluster of 2, 2-SM MMAs)
  CUtensorMap mq64, mdo64;
  if ((rc = make_bshd_map(&mq64, q, b, sq, h, 64)) || (rc = make_bshd_map(&mdo64, dO, b, sq, h, 64))) return rc;
  const int n_pairs = (p.n_blocks + 1) / 2;
  p.n_blocks_padded = 2 * n_pairs;
  cudaError_t e = launch_ex(wf_bwd2_main_kernel, dim3(2 * n_pairs * splits, h, b), dim3(kBwdThreads),
                            bwd2_smem_bytes(), reinterpret_cast<cudaStream_t>(stream), pdl, 2u, mq, mq64, mk, mv, mdo,
                            mdo64, p);
  if (e != cudaSuccess) return cuda_fail(e, "wf_bwd_main (pair) launch");
  return launch_check("wf_bwd_main (pair) launch");
}

int wf_bwd_convert(const float* accum, void* out, float scale, int b, int s, int h, void* stream) {
  int rc = check_dims(b, s, s, h);
  if (rc) return rc;
  if (b == 0 || s == 0 || h == 0) return WF_OK;
  if (!accum || !out) return fail(WF_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(accum) || !aligned16(out)) return fail(WF_ERR_MISALIGNED, "accum/out must be 16-byte aligned");
  int dev;
  if ((rc = device_setup(&dev))) return rc;
  const int s_rounded = (s + 127) / 128 * 128;
  dim3 grid(s_rounded / 32, h, b);
  // a programmatic dependent of the kernel that filled `accum`
  cudaError_t e = launch_ex(wf_convert_kernel, grid, dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), true, 1u,
                            accum, reinterpret_cast<__nv_bfloat16*>(out), scale, s, s_rounded, h);
  if (e != cudaSuccess) return cuda_fail(e, "wf_bwd_convert launch");
  return launch_check("wf_bwd_convert launch");
}

}  // extern "C"
