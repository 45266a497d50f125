// wf_bwd_noalloc: the whole backward chain (preprocess, main, dQ convert)
// with its fp32 workspaces in a fixed device array compiled into the library
// instead of caller-provided buffers.
//
// Who needs it: callers that can hand this library their tensors but cannot
// allocate device memory at call time -- a host runtime or plugin framework
// that owns every device allocation and gives a plugin only its inputs and
// outputs, or a caller on a latency-critical path that must not pay for
// cudaMalloc's implicit device synchronisation.  wf_bwd_main needs three
// workspaces (rowsum(o*dO), -lse*log2(e), the fp32 dQ accumulator); here they
// live in `g_noalloc_scratch`, a file-scope array every GPU that loads the
// library holds until the process exits.
//
// Limits and rules (also stated at the declaration in include/wan_flash.h):
//   * at most kNoAllocMaxRows = b * h * ceil(sq/128)*128 query rows
//     (64 MiB of scratch, 520 bytes per row); larger calls are rejected with
//     WF_ERR_UNSUPPORTED before any device work;
//   * split-M is not used (nsplit = 1): dk/dv are written directly;
//   * every call shares the one array: calls whose work overlaps on the GPU
//     (different streams, or different host threads without ordering) race on
//     it.  The dQ accumulator is cleared by the preprocess kernel of every call,
//     so nothing carries over from the previous call's contents.
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture begins.
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "wan_flash.h"
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB
constexpr size_t kNoAllocBytesPerRow = (2 + 128) * sizeof(float);
constexpr size_t kNoAllocMaxRows = kNoAllocScratchBytes / kNoAllocBytesPerRow / 128 * 128;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on device `dev` (current), looked up once.
int noalloc_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return WF_OK;
}
}  // namespace
}  // namespace wf

extern "C" int wf_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse,
                              const void* dO, void* dq, void* dk, void* dv, int b, int sq, int skv, int h,
                              void* stream) {
  using namespace wf;
  if (b < 0 || sq < 0 || skv < 0 || h < 0) return fail(WF_ERR_INVALID_ARG, "negative size");
  if (b == 0 || h == 0 || sq == 0 || skv == 0)
    return fail(WF_ERR_UNSUPPORTED, "wf_bwd_noalloc needs b, h, sq, skv > 0");
  const size_t sq_rounded = (size_t(sq) + 127) / 128 * 128;
  const size_t rows = size_t(b) * size_t(h) * sq_rounded;
  if (rows > kNoAllocMaxRows)
    return fail(WF_ERR_UNSUPPORTED,
                "wf_bwd_noalloc: b*h*ceil(sq/128)*128 = %zu query rows exceeds the built-in scratch limit of %zu rows "
                "(64 MiB); use wf_bwd_pre/wf_bwd_main/wf_bwd_convert with caller workspaces",
                rows, kNoAllocMaxRows);
  if (!dq) return fail(WF_ERR_INVALID_ARG, "null pointer");
  int dev, rc;
  if ((rc = device_setup(&dev))) return rc;
  void* base = nullptr;
  if ((rc = noalloc_scratch(dev, &base))) return rc;
  float* dpsum = reinterpret_cast<float*>(base);
  float* neg_lse_log2 = dpsum + rows;
  float* dq_accum = neg_lse_log2 + rows;
  if ((rc = wf_bwd_pre(o, dO, lse, dpsum, neg_lse_log2, dq_accum, b, sq, (int)sq_rounded, h, stream))) return rc;
  wf_bwd_cfg cfg = {1, 0, 0, 0, nullptr};
  if ((rc = wf_bwd_main(q, k, v, dO, neg_lse_log2, dpsum, dq_accum, dk, dv, b, sq, skv, h, &cfg, stream))) return rc;
  return wf_bwd_convert(dq_accum, dq, (float)(1.0 / std::sqrt(128.0)), b, sq, h, stream);
}
