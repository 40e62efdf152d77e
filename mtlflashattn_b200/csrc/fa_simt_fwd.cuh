// Accuracy-first flash-attention forward on the CUDA cores (fp32 FMA), for every input the
// tcgen05 kernel does not take: fp32 inputs, head dims that are not a multiple of 8, strides or
// pointers that TMA cannot address. It reads q/k/v through arbitrary (batch, seq, head) strides,
// so no layout copy is ever made.
//
// CTA = 128 threads = 32 query rows x 4 threads per row (or 8 rows x 16 threads for small
// launches); keys stream in blocks of 16 through shared memory. Online softmax in fp32 with expf; semantics of the reference's chunked-fp32
// tier (metal_flash_attn/_kernel.py:1165-1208) and of its scalar v0 kernel (_kernel.py:32-87).
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace mfa {
namespace simt {
constexpr int BN = 16;
constexpr int kThreads = 128;
// TPR threads share a query row: 4 (32 rows per CTA) normally, 16 (8 rows per CTA) when a
// launch would otherwise leave SMs idle, so small problems get four times the CTAs.
template <int TPR>
__host__ __device__ constexpr int rows_per_cta() { return kThreads / TPR; }
}  // namespace simt

template <typename T>
__device__ __forceinline__ void store_elem(const FwdArgs& a, void* row_ptr, int col, float v) {
  if (a.o_dtype == 2) {
    reinterpret_cast<float*>(row_ptr)[col] = v;
  } else if (a.o_dtype == 1) {
    reinterpret_cast<__nv_bfloat16*>(row_ptr)[col] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(row_ptr)[col] = __float2half_rn(v);
  }
}

template <typename T, int DP, int TPR = 4>
__global__ void __launch_bounds__(simt::kThreads) fa_fwd_simt(const __grid_constant__ FwdArgs a) {
  using namespace simt;
  static_assert(TPR == 4 || TPR == 16, "threads per row");
  constexpr int BM = rows_per_cta<TPR>();
  constexpr int NC = DP / TPR;  // output columns per thread
  __shared__ float sQ[BM][DP + 1];
  __shared__ float sK[BN][DP + 1];
  __shared__ float sV[BN][DP];
  __shared__ float sP[BM][BN + 1];

  const int HB = a.Hq * a.B;
  const int idx = blockIdx.x;
  const int rb = a.num_row_blocks - 1 - idx / HB;
  const int hb = idx % HB;
  const int h = hb % a.Hq;
  const int b = hb / a.Hq;
  const int hk = h / a.group;
  const SeqView sv = seq_view(a, b);
  const int r0 = rb * BM;
  if (r0 >= sv.lq) return;

  const T* qp = reinterpret_cast<const T*>(a.q);
  const T* kp = reinterpret_cast<const T*>(a.k);
  const T* vp = reinterpret_cast<const T*>(a.v);
  const int tid = threadIdx.x;
  const int r = tid / TPR;
  const int sub = tid % TPR;
  const int64_t row = (int64_t)r0 + r;
  const int D = a.D;

  for (int e = tid; e < BM * DP; e += kThreads) {
    const int rr = e / DP, d = e % DP;
    float val = 0.f;
    if (r0 + rr < sv.lq && d < D)
      val = to_f32<T>(qp[(int64_t)sv.qb * a.q_sb + (int64_t)(sv.q0 + r0 + rr) * a.q_ss +
                         (int64_t)h * a.q_sh + d]);
    sQ[rr][d] = val;
  }

  const int r_last = min(r0 + BM, sv.lq) - 1;
  const int klo = key_range(a, sv, r0).lo;
  const int khi = key_range(a, sv, r_last).hi;
  const KeyRange kr = key_range(a, sv, row);
  const float slope = a.alibi != nullptr ? a.alibi[(int64_t)b * a.Hq + h] : 0.f;
  const float centre = (float)(row + sv.off);

  float m = -INFINITY, l = 0.f;
  float acc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) acc[c] = 0.f;

  for (int kb0 = (khi > klo ? (klo / BN) * BN : khi); kb0 < khi; kb0 += BN) {
    __syncthreads();
    for (int e = tid; e < BN * DP; e += kThreads) {
      const int kk = e / DP, d = e % DP;
      float kv = 0.f, vv = 0.f;
      if (kb0 + kk < sv.lk && d < D) {
        const int64_t krow = (int64_t)(sv.k0 + kb0 + kk);
        kv = to_f32<T>(kp[(int64_t)sv.kb * a.k_sb + krow * a.k_ss + (int64_t)hk * a.k_sh + d]);
        vv = to_f32<T>(vp[(int64_t)sv.kb * a.v_sb + krow * a.v_ss + (int64_t)hk * a.v_sh + d]);
      }
      sK[kk][d] = kv;
      sV[kk][d] = vv;
    }
    __syncthreads();

    float s[BN / TPR];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < BN / TPR; ++i) {
      const int kk = sub + TPR * i;
      float dot = 0.f;
#pragma unroll 8
      for (int d = 0; d < DP; ++d) dot = fmaf(sQ[r][d], sK[kk][d], dot);
      float val = dot * a.scale;
      if (a.softcap > 0.f) val = a.softcap * tanhf(val / a.softcap);
      const int key = kb0 + kk;
      if (a.alibi != nullptr) val -= slope * fabsf(centre - (float)(key + a.k_pos_offset));
      s[i] = (key >= kr.lo && key < kr.hi) ? val : -INFINITY;
      mx = fmaxf(mx, s[i]);
    }
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m, mx);
    float corr = 1.f;
    float ls = 0.f;
    if (m_new != -INFINITY) {
      corr = (m == -INFINITY) ? 0.f : expf(m - m_new);
#pragma unroll
      for (int i = 0; i < BN / TPR; ++i) {
        const float p = (s[i] == -INFINITY) ? 0.f : expf(s[i] - m_new);
        sP[r][sub + TPR * i] = p;
        ls += p;
      }
    } else {
#pragma unroll
      for (int i = 0; i < BN / TPR; ++i) sP[r][sub + TPR * i] = 0.f;
    }
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    l = l * corr + ls;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[c] *= corr;
#pragma unroll 4
    for (int kk = 0; kk < BN; ++kk) {
      const float p = sP[r][kk];
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = fmaf(p, sV[kk][sub + TPR * c], acc[c]);
    }
  }

  if (row < sv.lq) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t esz = a.o_dtype == 2 ? 4 : 2;
    uint8_t* orow = reinterpret_cast<uint8_t*>(a.o) +
                    esz * ((int64_t)sv.qb * a.o_sb + (int64_t)(sv.q0 + row) * a.o_ss + (int64_t)h * a.o_sh);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int d = sub + TPR * c;
      if (d < D) store_elem<T>(a, orow, d, acc[c] * inv);
    }
    if (sub == 0 && a.lse != nullptr)
      a.lse[(int64_t)sv.qb * a.lse_sb + (int64_t)h * a.lse_sh + sv.q0 + row] =
          l > 0.f ? m + logf(l) : -INFINITY;
  }
}

}  // namespace mfa
