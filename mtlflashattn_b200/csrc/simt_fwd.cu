// The fp32 CUDA-core forward (fa_simt_fwd.cuh) in a translation unit of its own, compiled
// WITHOUT fast math (IEEE division, accurate expf / tanhf / logf, no flush to zero) so the
// accuracy path keeps its fp32 error bar at large logits and under softcap; the rest of
// libmfa.so is built with --use_fast_math. mfa_api.cu calls simt_forward through the
// declaration below.
#include <cuda_runtime.h>

#include "fa_simt_fwd.cuh"

namespace mfa {

// Launches the forward for resolved arguments; returns 0 (MFA_OK) or 2 (MFA_ERR_UNSUPPORTED: a
// grid beyond 2^31 CTAs).
int simt_forward(FwdArgs a, int dtype, int D, cudaStream_t st) {
  // 32-row CTAs unless that leaves most of the GPU idle: below two CTAs per SM, 8-row CTAs with
  // 16 threads per row (config 1, B=1 H=4 L=1024: 128 CTAs -> 512)
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t wide_grid = (int64_t)((a.max_lq + simt::rows_per_cta<4>() - 1) /
                                      simt::rows_per_cta<4>()) * a.Hq * a.B;
  const bool narrow = wide_grid < 2ll * sms;
  const int bm = narrow ? simt::rows_per_cta<16>() : simt::rows_per_cta<4>();
  a.num_row_blocks = (a.max_lq + bm - 1) / bm;
  const int64_t grid = (int64_t)a.num_row_blocks * a.Hq * a.B;
  if (grid == 0) return 0;
  if (grid >= (1ll << 31)) return 2;
  const int dp = D <= 32 ? 32 : (D <= 64 ? 64 : 128);
#define MFA_SIMT_TPR(T, DPV)                                                          \
  do {                                                                                \
    if (narrow) fa_fwd_simt<T, DPV, 16><<<(unsigned)grid, simt::kThreads, 0, st>>>(a); \
    else fa_fwd_simt<T, DPV, 4><<<(unsigned)grid, simt::kThreads, 0, st>>>(a);         \
  } while (0)
#define MFA_SIMT_LAUNCH(T)                          \
  do {                                              \
    if (dp == 32) MFA_SIMT_TPR(T, 32);              \
    else if (dp == 64) MFA_SIMT_TPR(T, 64);         \
    else MFA_SIMT_TPR(T, 128);                      \
  } while (0)
  if (dtype == 2) MFA_SIMT_LAUNCH(float);
  else if (dtype == 1) MFA_SIMT_LAUNCH(__nv_bfloat16);
  else MFA_SIMT_LAUNCH(__half);
#undef MFA_SIMT_LAUNCH
#undef MFA_SIMT_TPR
  return 0;
}

}  // namespace mfa
