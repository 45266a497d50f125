/*
 * A plain C host of the C ABI (include/wan_flash.h): what a C or C++ caller,
 * or another language's FFI, does with libwanflash.so.  Device memory comes
 * from the CUDA runtime; inputs are seeded bf16 from an LCG.  Runs the
 * forward and the full backward chain (wf_bwd_pre, wf_bwd_main,
 * wf_bwd_convert) on a small problem and checks o, lse, dq, dk, dv against
 * a double-precision reference computed here, then wf_bwd_noalloc against
 * the chain.  Exit status 0 = all checks passed.
 *
 *   gcc -O2 -std=c11 -I include tests/c_host/wf_c_host.c -o wf_c_host \
 *       -L wan_flash -lwanflash -L /usr/local/cuda/lib64 -lcudart -lm \
 *       -Wl,-rpath,<dir of libwanflash.so>
 */
#include <cuda_runtime_api.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "wan_flash.h"

#define B 1
#define H 2
#define SQ 300
#define SKV 200
#define D 128

static uint64_t g_state = 0x9E3779B97F4A7C15ull;

static float lcg_normalish(void) {
  /* sum of 4 uniforms, centred and scaled to unit variance */
  float acc = 0.f;
  for (int i = 0; i < 4; ++i) {
    g_state = g_state * 6364136223846793005ull + 1442695040888963407ull;
    acc += (float)((g_state >> 40) & 0xFFFFFF) / 16777216.0f;
  }
  return (acc - 2.0f) * 1.7320508f;
}

static uint16_t f2bf(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

#define CK(x)                                                                            \
  do {                                                                                   \
    cudaError_t e_ = (x);                                                                \
    if (e_ != cudaSuccess) {                                                             \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
      return 2;                                                                          \
    }                                                                                    \
  } while (0)

#define WF(x)                                                                         \
  do {                                                                                \
    int rc_ = (x);                                                                    \
    if (rc_ != WF_OK) {                                                               \
      char msg_[512];                                                                 \
      wf_last_error(msg_, sizeof msg_);                                               \
      fprintf(stderr, "%s:%d %s -> %d (%s)\n", __FILE__, __LINE__, #x, rc_, msg_); \
      return 3;                                                                       \
    }                                                                                 \
  } while (0)

/* element (b, s, h, d) of a (B, S, H, D) tensor */
#define AT(s, h, d, S) (((size_t)(s) * H + (h)) * D + (d))

static double rel_l2(const uint16_t* got, const double* ref, size_t n) {
  double num = 0, den = 0;
  for (size_t i = 0; i < n; ++i) {
    const double g = bf2f(got[i]), r = ref[i];
    num += (g - r) * (g - r);
    den += r * r;
  }
  return sqrt(num / (den > 0 ? den : 1e-300));
}

int main(void) {
  const size_t nq = (size_t)B * SQ * H * D, nk = (size_t)B * SKV * H * D;
  uint16_t *hq = malloc(nq * 2), *hk = malloc(nk * 2), *hv = malloc(nk * 2), *hdo = malloc(nq * 2);
  uint16_t *ho = malloc(nq * 2), *hdq = malloc(nq * 2), *hdk = malloc(nk * 2), *hdv = malloc(nk * 2);
  uint16_t *hdq2 = malloc(nq * 2), *hdk2 = malloc(nk * 2), *hdv2 = malloc(nk * 2);
  float* hlse = malloc((size_t)B * H * SQ * 4);
  for (size_t i = 0; i < nq; ++i) hq[i] = f2bf(lcg_normalish());
  for (size_t i = 0; i < nk; ++i) hk[i] = f2bf(lcg_normalish());
  for (size_t i = 0; i < nk; ++i) hv[i] = f2bf(lcg_normalish());
  for (size_t i = 0; i < nq; ++i) hdo[i] = f2bf(lcg_normalish());

  void *q, *k, *v, *o, *dO, *dq, *dk, *dv;
  float *lse, *dpsum, *nl, *dqa;
  const int sq_r = (SQ + 127) / 128 * 128;
  CK(cudaMalloc(&q, nq * 2));
  CK(cudaMalloc(&k, nk * 2));
  CK(cudaMalloc(&v, nk * 2));
  CK(cudaMalloc(&o, nq * 2));
  CK(cudaMalloc(&dO, nq * 2));
  CK(cudaMalloc(&dq, nq * 2));
  CK(cudaMalloc(&dk, nk * 2));
  CK(cudaMalloc(&dv, nk * 2));
  CK(cudaMalloc((void**)&lse, (size_t)B * H * SQ * 4));
  CK(cudaMalloc((void**)&dpsum, (size_t)B * H * sq_r * 4));
  CK(cudaMalloc((void**)&nl, (size_t)B * H * sq_r * 4));
  CK(cudaMalloc((void**)&dqa, (size_t)B * H * sq_r * D * 4));
  CK(cudaMemcpy(q, hq, nq * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(k, hk, nk * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(v, hv, nk * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dO, hdo, nq * 2, cudaMemcpyHostToDevice));

  printf("wan_flash C ABI version %d, %d SMs\n", wf_version(), wf_num_sms());
  wf_fwd_cfg fcfg = {8.0f, 0, 0};
  WF(wf_fwd(q, k, v, o, lse, B, SQ, SKV, H, &fcfg, NULL));
  wf_bwd_cfg bcfg;
  memset(&bcfg, 0, sizeof bcfg);
  bcfg.nsplit = 1;
  bcfg.cluster_n = 1;
  WF(wf_bwd_pre(o, dO, lse, dpsum, nl, dqa, B, SQ, sq_r, H, NULL));
  WF(wf_bwd_main(q, k, v, dO, nl, dpsum, dqa, dk, dv, B, SQ, SKV, H, &bcfg, NULL));
  WF(wf_bwd_convert(dqa, dq, (float)(1.0 / sqrt((double)D)), B, SQ, H, NULL));
  CK(cudaDeviceSynchronize());
  WF(wf_device_status(NULL));
  CK(cudaMemcpy(ho, o, nq * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(hlse, lse, (size_t)B * H * SQ * 4, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(hdq, dq, nq * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(hdk, dk, nk * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(hdv, dv, nk * 2, cudaMemcpyDeviceToHost));

  /* the same backward through the no-workspace entry point */
  WF(wf_bwd_noalloc(q, k, v, o, lse, dO, dq, dk, dv, B, SQ, SKV, H, NULL));
  CK(cudaDeviceSynchronize());
  WF(wf_device_status(NULL));
  CK(cudaMemcpy(hdq2, dq, nq * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(hdk2, dk, nk * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(hdv2, dv, nk * 2, cudaMemcpyDeviceToHost));

  /* double-precision reference from the bf16 inputs; the backward uses the
     kernel's own o (rounded to bf16), as the reference's tests do */
  const double scale = 1.0 / sqrt((double)D);
  double* ro = calloc(nq, sizeof(double));
  double* rdq = calloc(nq, sizeof(double));
  double* rdk = calloc(nk, sizeof(double));
  double* rdv = calloc(nk, sizeof(double));
  double* p = malloc((size_t)SKV * sizeof(double));
  double* dp = malloc((size_t)SKV * sizeof(double));
  double lse_err = 0;
  for (int h = 0; h < H; ++h)
    for (int i = 0; i < SQ; ++i) {
      double m = -INFINITY, l = 0;
      for (int j = 0; j < SKV; ++j) {
        double s = 0;
        for (int d = 0; d < D; ++d) s += (double)bf2f(hq[AT(i, h, d, SQ)]) * bf2f(hk[AT(j, h, d, SKV)]);
        p[j] = s * scale;
        if (p[j] > m) m = p[j];
      }
      for (int j = 0; j < SKV; ++j) l += exp(p[j] - m);
      const double lse_ref = m + log(l);
      const double e = fabs(lse_ref - hlse[(size_t)h * SQ + i]);
      if (e > lse_err) lse_err = e;
      for (int j = 0; j < SKV; ++j) p[j] = exp(p[j] - lse_ref);
      for (int d = 0; d < D; ++d) {
        double acc = 0;
        for (int j = 0; j < SKV; ++j) acc += p[j] * bf2f(hv[AT(j, h, d, SKV)]);
        ro[AT(i, h, d, SQ)] = acc;
      }
      double Di = 0;
      for (int d = 0; d < D; ++d) Di += (double)bf2f(hdo[AT(i, h, d, SQ)]) * bf2f(ho[AT(i, h, d, SQ)]);
      for (int j = 0; j < SKV; ++j) {
        double s = 0;
        for (int d = 0; d < D; ++d) s += (double)bf2f(hdo[AT(i, h, d, SQ)]) * bf2f(hv[AT(j, h, d, SKV)]);
        dp[j] = p[j] * (s - Di) * scale; /* dS */
      }
      for (int j = 0; j < SKV; ++j)
        for (int d = 0; d < D; ++d) {
          rdv[AT(j, h, d, SKV)] += p[j] * bf2f(hdo[AT(i, h, d, SQ)]);
          rdk[AT(j, h, d, SKV)] += dp[j] * bf2f(hq[AT(i, h, d, SQ)]);
          rdq[AT(i, h, d, SQ)] += dp[j] * bf2f(hk[AT(j, h, d, SKV)]);
        }
    }
  const double tol = 4.5e-3;
  const double e_o = rel_l2(ho, ro, nq), e_dq = rel_l2(hdq, rdq, nq), e_dk = rel_l2(hdk, rdk, nk),
               e_dv = rel_l2(hdv, rdv, nk);
  const double e2_dq = rel_l2(hdq2, rdq, nq), e2_dk = rel_l2(hdk2, rdk, nk), e2_dv = rel_l2(hdv2, rdv, nk);
  printf("rel_l2 o %.3e dq %.3e dk %.3e dv %.3e | noalloc dq %.3e dk %.3e dv %.3e | lse abs %.3e\n", e_o, e_dq,
         e_dk, e_dv, e2_dq, e2_dk, e2_dv, lse_err);
  const int ok = e_o <= tol && e_dq <= tol && e_dk <= tol && e_dv <= tol && e2_dq <= tol && e2_dk <= tol &&
                 e2_dv <= tol && lse_err <= 1e-5;
  printf("%s\n", ok ? "C host: OK" : "C host: FAILED");
  return ok ? 0 : 1;
}
