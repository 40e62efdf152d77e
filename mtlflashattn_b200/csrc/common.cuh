// Kernel-side argument block and the masking rules shared by both attention kernels.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mfa {

// Resolved arguments as both kernels read them. Strides are in elements.
constexpr int kMaxPeers = 8;  // GPUs one split-KV launch can scatter its partial rows to

// Debug build (-DMFA_CHECKS=1): every TMA tile coordinate and every output row address is
// checked against the launch's extents before use; a failed check stores MFA_ERR_CHECK (8) in
// the error word, skips the access and ends the CTA's waits (no trap, no fault).
#ifndef MFA_CHECKS
#define MFA_CHECKS 0
#endif
constexpr int kErrCheck = 8;

struct FwdArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  int64_t o_sb, o_ss, o_sh;
  int64_t lse_sb, lse_sh;
  int B, Hq, Hkv, Lq, Lk, D;
  int group;  // Hq / Hkv
  const int* cu_q;
  const int* cu_k;
  int max_lq;
  float scale, softcap;
  int causal, wl, wr;
  const float* alibi;
  int o_dtype;  // 0 fp16, 1 bf16, 2 fp32
  int o_vec16;  // 1 if every output row segment is 16-byte aligned (vector stores allowed)
  int k_pos_offset;
  int lk_total;  // 0 = per-sequence Lk
  int* err;
  int num_row_blocks;  // row blocks per (batch, head) for this launch's kernel
  // CTA order: (batch, head) pairs in groups of group_hb (whole KV groups, sized so one group's
  // K/V fits comfortably in L2), groups one after the other, heaviest row blocks first within
  // a group; group_hb = B * Hq is one group (plain heaviest-first order)
  int group_hb;
  // key split within one launch (1 = none): CTA (row block, batch, head, split) covers the local
  // keys [split * split_keys, (split + 1) * split_keys) and writes its partial output at
  // o + split * o_split_stride and its row log-sum-exp at lse + split * lse_split_stride
  int num_splits;
  int split_keys;
  int64_t o_split_stride;
  int64_t lse_split_stride;
  // query heads packed per KV head (tcgen05 kernel only): 0 = off, else a CTA serves one
  // (batch, KV head) and its tile row r is query position r >> pack_shift of query head
  // hk * 2^pack_shift + (r & (2^pack_shift - 1)); the 2^pack_shift heads of a KV group share
  // every K/V block load
  int pack_shift;
  // sequences of a varlen launch (B before the split merge views the packed rows as one batch)
  int nseq;
  // split-KV over several GPUs (peer_n > 0; dense launches only): query row R is owned by GPU
  // R / peer_rows, and this launch's fp32 partial row and row log-sum-exp go straight into that
  // GPU's receive buffers (peer-mapped device pointers), in slot peer_slot of each:
  // peer_o[g] + peer_slot * peer_slot_o holds [peer_rows][B][Hq][D] (o_* strides below), and
  // peer_lse[g] + peer_slot * peer_slot_lse holds [B*Hq][peer_rows] (lse_* strides)
  int peer_n, peer_rows, peer_slot;
  int64_t peer_slot_o, peer_slot_lse;
  float* peer_o[kMaxPeers];
  float* peer_lse[kMaxPeers];
};

// One (batch, sequence) view after resolving dense vs varlen.
struct SeqView {
  int q0, lq;   // first row (absolute for varlen, 0 for dense) and query length
  int k0, lk;   // first key row and local key count
  int qb, kb;   // batch coordinate for strided addressing (0 for varlen)
  int off;      // centre offset: centre(i) = i + off, in global key positions
};

__device__ __forceinline__ SeqView seq_view(const FwdArgs& a, int b) {
  SeqView s;
  if (a.cu_q != nullptr) {
    s.q0 = a.cu_q[b];
    s.lq = a.cu_q[b + 1] - s.q0;
    s.k0 = a.cu_k[b];
    s.lk = a.cu_k[b + 1] - s.k0;
    s.qb = 0;
    s.kb = 0;
  } else {
    s.q0 = 0;
    s.lq = a.Lq;
    s.k0 = 0;
    s.lk = a.Lk;
    s.qb = b;
    s.kb = b;
  }
  const int lk_tot = a.lk_total > 0 ? a.lk_total : s.lk;
  s.off = lk_tot - s.lq;
  return s;
}

// Local key interval [lo, hi) that row i of a sequence may attend (bottom-right aligned causal
// and sliding window, restricted to the local keys [0, lk)). Rule of _flash_torch
// (metal_flash_attn/_kernel.py:1196-1203) and of the v0 kernel's kmin/kmax (_kernel.py:59-64).
struct KeyRange {
  int lo, hi;
};
__device__ __forceinline__ KeyRange key_range(const FwdArgs& a, const SeqView& s, int64_t i) {
  const int64_t centre = i + s.off;
  int64_t lo = a.wl >= 0 ? centre - a.wl : INT64_MIN / 4;
  int64_t hi = INT64_MAX / 4;
  if (a.causal) hi = centre + 1;
  if (a.wr >= 0) hi = hi < centre + a.wr + 1 ? hi : centre + a.wr + 1;
  lo -= a.k_pos_offset;
  hi -= a.k_pos_offset;
  if (lo < 0) lo = 0;
  if (hi > s.lk) hi = s.lk;
  KeyRange r;
  r.lo = static_cast<int>(lo > s.lk ? s.lk : lo);
  r.hi = static_cast<int>(hi < 0 ? 0 : hi);
  return r;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

// Pack two fp32 values into one 32-bit word of 16-bit values, `lo` in the low half.
template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Store `n` (<= 32) consecutive fp32 values of one output row, converting to o_dtype.
__device__ __forceinline__ void store_row_chunk(const FwdArgs& a, void* row_ptr, int col0,
                                                const float* vals, int n) {
  if (a.o_dtype == 2) {
    float* p = reinterpret_cast<float*>(row_ptr) + col0;
    if (a.o_vec16 && n == 32) {  // 16-byte stores (also the unit of a remote write over NVLink)
      float4* dst = reinterpret_cast<float4*>(p);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[i] = make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
      return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < n) p[i] = vals[i];
    return;
  }
  uint16_t* p = reinterpret_cast<uint16_t*>(row_ptr) + col0;
  if (a.o_vec16 && n == 32) {
    uint32_t w[16];
    if (a.o_dtype == 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = pack2<true>(vals[2 * i], vals[2 * i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = pack2<false>(vals[2 * i], vals[2 * i + 1]);
    }
    uint4* dst = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < n) {
      if (a.o_dtype == 1) {
        __nv_bfloat16 h = __float2bfloat16_rn(vals[i]);
        p[i] = *reinterpret_cast<uint16_t*>(&h);
      } else {
        __half h = __float2half_rn(vals[i]);
        p[i] = *reinterpret_cast<uint16_t*>(&h);
      }
    }
  }
}

// tanh from its exponential form, tanh(y) = 1 - 2 / (exp(2y) + 1), with the hardware exp2.
// |y| is clamped at 15 where tanh is 1 to fp32 precision. Absolute error stays near 1e-7,
// so a softcap of 30 moves a logit by ~3e-6 at most.
__device__ __forceinline__ float tanh_exp2(float y) {
  y = fminf(fmaxf(y, -15.f), 15.f);
  float t;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(y * 2.8853900817779268f));  // 2*log2(e)
  return 1.f - __fdividef(2.f, t + 1.f);
}

}  // namespace mfa
