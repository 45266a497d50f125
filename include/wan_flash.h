/*
 * wan_flash.h -- C ABI of the B200 (sm_100a) Wan attention hot path.
 *
 * The reference (Quarky93/wan-flash) has no native library: its Python
 * driver `wan_flash/interface.py` JIT-compiles CuTeDSL kernels and calls the
 * compiled launchers directly.  Each entry point below replaces one of those
 * compiled-launch calls and keeps its argument meaning; the Python package
 * `wan_flash` (interface.py) binds them with ctypes exactly where the
 * reference calls its compiled kernels.
 *
 * Conventions
 *   - Tensors are caller-owned device memory, contiguous, in the reference's
 *     layouts: q/k/v/o/dO/dq/dk/dv (b, s, h, 128) bf16; lse (b, h, s) fp32
 *     natural log; workspaces as documented per call.
 *   - bf16 buffers and fp32 workspaces must be 16-byte aligned.
 *   - Every call is enqueued on `stream` (a cudaStream_t, 0 = legacy default)
 *     and does not synchronise.  Calls are thread-safe.
 *   - Return 0 (WF_OK) or a negative wf_status; never abort.  A message for
 *     the last failure of the calling thread is available from
 *     wf_last_error().
 *   - Device-side failures (a bounded wait that ran out) do not trap; they
 *     set a device error word that wf_device_status() reads.
 */
#ifndef WAN_FLASH_H_
#define WAN_FLASH_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum wf_status {
  WF_OK = 0,
  WF_ERR_INVALID_ARG = -1,   /* null pointer, negative size, bad config      */
  WF_ERR_UNSUPPORTED = -2,   /* outside the Wan contract (e.g. head_dim)     */
  WF_ERR_MISALIGNED = -3,    /* a buffer is not 16-byte aligned              */
  WF_ERR_CUDA = -4,          /* CUDA runtime / driver call failed            */
  WF_ERR_NO_DEVICE = -5,     /* current device is not an sm_100 part         */
  WF_ERR_WAIT_TIMEOUT = -6,  /* device: a bounded mbarrier wait expired      */
  WF_ERR_SMEM_ALIGN = -7     /* device: dynamic shared memory misaligned     */
} wf_status;

#define WF_HEAD_DIM 128

/* Forward options (mirror FwdFeatures, wan_flash/features.py:28-42). */
typedef struct wf_fwd_cfg {
  float rescale_threshold; /* skip the O rescale while the running max grew
                              by <= this many log2 units; 0 = always rescale */
  int scheduler;           /* 0 = auto (persistent when skv <= 8192),
                              1 = one CTA per 256-row work item,
                              2 = persistent (min(items, num_sms) CTAs)      */
  int num_sms;             /* persistent grid size; 0 = the device's SMs     */
  int cluster_m;           /* 0 = auto (2 for one KV context on the
                              one-item-per-CTA schedule, else 1),
                              1 = one CTA per 256-row work item,
                              2 = CTA pairs along the query axis (cluster of
                              2, 2-SM tensor-core MMAs, each CTA loading half
                              of every K/V tile: the reference's cluster
                              (2, 1) without multicast loads); one KV context
                              and the one-item-per-CTA schedule only        */
} wf_fwd_cfg;

/* Backward options (mirror BwdFeatures, wan_flash/features.py:45-70). */
typedef struct wf_bwd_cfg {
  int nsplit;        /* split-M factor >= 1; with nsplit > 1 dk/dv arguments of
                        wf_bwd_main are fp32 accumulators (zeroed by the caller) */
  int cluster_n;     /* 0 = auto, 1 = one CTA per KV block, 2 = CTA pairs over
                        adjacent KV blocks (cluster of 2, 2-SM tensor-core MMAs;
                        the reference's cluster_n = 2 without multicast loads) */
  int deterministic; /* 1 = add the fp32 dQ (and split-M dK/dV) contributions in
                        KV-block (split) order: bitwise-reproducible gradients,
                        slower; single-CTA kernel only; needs `sem` */
  int pdl_off;       /* 1 = launch the main kernel without programmatic dependent
                        launch (default 0: it may start while the preceding
                        wf_bwd_pre finishes -- barrier set-up, TMEM allocation
                        and the K/V loads overlap the preprocess's tail -- and
                        waits for it before reading its outputs) */
  int* sem;          /* deterministic only: b*h*(ceil(sq/128) + ceil(skv/128))
                        int32, zeroed by the caller before each wf_bwd_main */
} wf_bwd_cfg;

/*
 * Forward: o = softmax(q k^T / sqrt(128)) v and lse (natural log).
 * Replaces the compiled WanFlashFwdSm90 launch `_compile_cache[key](*cargs,
 * stream)` of wan_flash/interface.py:74 (kernel: wan_flash/fwd_sm90.py:184-308).
 *   q (b, sq, h, 128) bf16; k, v (b, skv, h, 128) bf16
 *   o (b, sq, h, 128) bf16; lse (b, h, sq) fp32
 */
int wf_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int b, int sq, int skv,
           int h, const wf_fwd_cfg* cfg, void* stream);

/*
 * Two-context forward (no reference counterpart; the Wan I2V cross
 * attention, where the same query rows attend a text context and an image
 * context and the model adds the two outputs): o_c = softmax(q k_c^T /
 * sqrt(128)) v_c and lse_c for c = 0, 1 in one launch, each 256-row query
 * block loaded once for both.  Same layouts as wf_fwd; each context's
 * softmax, output and LSE are independent (o_0 and o_1 are what two wf_fwd
 * calls would write, bitwise).
 */
int wf_fwd_dual(const void* q, const void* k0, const void* v0, const void* k1, const void* v1, void* o0, void* o1,
                float* lse0, float* lse1, int b, int sq, int skv0, int skv1, int h, const wf_fwd_cfg* cfg,
                void* stream);

/*
 * Backward preprocess: dpsum = rowsum(o * dO) (fp32), neg_lse_log2 =
 * -lse * log2(e) (-inf on pad rows, lse == -inf mapped to 0; the reference's
 * lse_log2 workspace, negated), and zero dq_accum.
 * Replaces `compiled[0](*pre_args, stream)` of wan_flash/interface.py:190
 * (WanFlashBwdPreprocessSm90, wan_flash/bwd_sm90.py:99-235).
 *   dpsum, neg_lse_log2: (b, h, sq_rounded) fp32, sq_rounded = ceil(sq/128)*128
 *   dq_accum: b*h*sq_rounded*128 fp32 in 128-row tiles, see wf_bwd_convert;
 *   may be NULL (left untouched: the second KV context of a two-context
 *   backward adds into the accumulator the first context's call zeroed)
 */
int wf_bwd_pre(const void* o, const void* dO, const float* lse, float* dpsum, float* neg_lse_log2,
               float* dq_accum, int b, int sq, int sq_rounded, int h, void* stream);

/*
 * Backward main (dK/dV-stationary): dk, dv, and dQ partial sums
 * (fp32 reductions into dq_accum, unscaled).
 * Replaces `compiled[1](*main_args, stream)` of wan_flash/interface.py:191
 * (WanFlashBwdSm90, wan_flash/bwd_sm90.py:381-507), launched, as there
 * (use_pdl=True, bwd_sm90.py:498-506), as a programmatic dependent of the
 * preceding kernel (normally wf_bwd_pre; see wf_bwd_cfg.pdl_off).
 *   nsplit == 1: dk, dv are bf16 (b, skv, h, 128) outputs (dk scaled).
 *   nsplit  > 1: dk, dv are fp32 accumulators of b*h*skv_rounded*128 floats
 *                in the tiled layout of dq_accum (skv_rounded =
 *                ceil(skv/128)*128), zeroed by the caller; dk is scaled.
 */
int wf_bwd_main(const void* q, const void* k, const void* v, const void* dO, const float* neg_lse_log2,
                const float* dpsum, float* dq_accum, void* dk, void* dv, int b, int sq, int skv, int h,
                const wf_bwd_cfg* cfg, void* stream);

/*
 * Convert a tiled fp32 accumulator to bf16 (b, s, h, 128): out = accum * scale.
 * Tiled layout: for (b, h, 128-row block m) a 128x128 tile stored as
 * [2 row halves][32 column groups of 4][64 rows][4] -- element (row r, col c)
 * of block m at ((b*h_total + h)*m_blocks + m)*16384 + (r/64)*8192 +
 * ((c/4)*64 + r%64)*4 + c%4.
 * Replaces `compiled[2](*post_args, stream)` (dQ) and, under split-M,
 * `compiled[3](...)` (dK, dV) of wan_flash/interface.py:192-195
 * (WanFlashBwdPostprocessSm90, wan_flash/bwd_sm90.py:1140-1308).  Launched
 * as a programmatic dependent of the preceding kernel (the main kernel or the
 * previous convert), whose completion it waits for before reading `accum`.
 */
int wf_bwd_convert(const float* accum, void* out, float scale, int b, int s, int h, void* stream);

/*
 * Backward without caller workspaces: the whole chain of wf_bwd_pre,
 * wf_bwd_main (nsplit = 1) and wf_bwd_convert, with the three fp32
 * workspaces taken from a 64 MiB array compiled into this library.  It has
 * no counterpart in the reference.  It exists for callers that can pass
 * tensors but cannot allocate device memory at call time -- a plugin host
 * that owns every device allocation, or a latency-critical caller that cannot
 * afford cudaMalloc's implicit synchronisation.  It never allocates.
 *   q, k, v, o, dO, dq, dk, dv: as wan_flash_bwd; lse (b, h, sq) natural log.
 *   Limit: b * h * ceil(sq/128)*128 <= 129,024 query rows (520 bytes of
 *   scratch each); larger calls return WF_ERR_UNSUPPORTED before any work.
 *   All calls share the one array: calls that overlap on the GPU race.
 *   The first call on a device looks up the array's address; make it before
 *   any stream capture.
 */
int wf_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse, const void* dO,
                   void* dq, void* dk, void* dv, int b, int sq, int skv, int h, void* stream);

/* Message for the last failed call on this thread (empty if none). */
int wf_last_error(char* buf, int len);

/*
 * Synchronise the current device and read (and clear) the device error word
 * written by kernels whose bounded waits expired.  Returns WF_OK or the
 * recorded wf_status; `info` (may be NULL) receives 4 words: block x|y<<16,
 * block z, role, barrier tag.
 */
int wf_device_status(unsigned int* info);

/* Set the device-side wait limit in nanoseconds (default 2^31). */
int wf_set_wait_limit_ns(unsigned long long ns);

/*
 * Self-test of device-side failure detection: launches one thread that waits
 * on an mbarrier nothing arrives on, with the wait limit set to `limit_ns`,
 * synchronises, and returns what wf_device_status reports (WF_ERR_WAIT_TIMEOUT
 * when the machinery works; `info` as in wf_device_status).  The previous
 * limit is restored.  No reference counterpart (the reference has no failure
 * detection); nothing is in flight, so the expiry cannot harm the context.
 */
int wf_selftest_wait_timeout(unsigned long long limit_ns, unsigned int* info);

/* Number of SMs of the current device (0 on error). */
int wf_num_sms(void);

/* Library version: 100 * major + minor. */
int wf_version(void);

#ifdef __cplusplus
}
#endif

#endif /* WAN_FLASH_H_ */
