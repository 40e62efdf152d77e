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
  a.num_row_blocks = (a.max_lq + simt::BM - 1) / simt::BM;
  const int64_t grid = (int64_t)a.num_row_blocks * a.Hq * a.B;
  if (grid == 0) return 0;
  if (grid >= (1ll << 31)) return 2;
  const int dp = D <= 32 ? 32 : (D <= 64 ? 64 : 128);
#define MFA_SIMT_LAUNCH(T)                                                           \
  do {                                                                               \
    if (dp == 32) fa_fwd_simt<T, 32><<<(unsigned)grid, simt::kThreads, 0, st>>>(a);  \
    else if (dp == 64) fa_fwd_simt<T, 64><<<(unsigned)grid, simt::kThreads, 0, st>>>(a); \
    else fa_fwd_simt<T, 128><<<(unsigned)grid, simt::kThreads, 0, st>>>(a);          \
  } while (0)
  if (dtype == 2) MFA_SIMT_LAUNCH(float);
  else if (dtype == 1) MFA_SIMT_LAUNCH(__nv_bfloat16);
  else MFA_SIMT_LAUNCH(__half);
#undef MFA_SIMT_LAUNCH
  return 0;
}

}  // namespace mfa
