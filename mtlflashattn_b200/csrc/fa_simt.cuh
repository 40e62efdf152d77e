// CUDA-core helper kernels of the library: the split-KV merges (within one launch, across GPUs,
// and of caller-held partials) and the bounded-wait self-test. Their exponentials and logs
// weigh partial results only, so the library's fast-math build serves them; the fp32 forward
// itself (fa_simt_fwd.cuh) is compiled separately with IEEE-accurate math.
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace mfa {

// Pointers of up to kMaxParts split-KV partials, passed by value as a kernel argument.
constexpr int kMaxParts = 64;
struct PartPtrs {
  const float* o[kMaxParts];
  const float* lse[kMaxParts];
};

// Log-sum-exp merge of n split-KV partials: one warp per (row, head), lanes over D.
template <typename TO>
__global__ void lse_combine_kernel(const __grid_constant__ PartPtrs pp, int n, int rows, int H,
                                   int D, TO* o, float* lse_out) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)rows * H) return;
  const int row = (int)(w / H), h = (int)(w % H);
  const int64_t li = (int64_t)h * rows + row;
  float mx = -INFINITY;
  for (int g = 0; g < n; ++g) mx = fmaxf(mx, pp.lse[g][li]);
  float tot = 0.f;
  if (mx != -INFINITY)
    for (int g = 0; g < n; ++g) tot += expf(pp.lse[g][li] - mx);
  const float lse = mx == -INFINITY ? -INFINITY : mx + logf(tot);
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    if (lse != -INFINITY)
      for (int g = 0; g < n; ++g) {
        const float lg = pp.lse[g][li];
        if (lg != -INFINITY) acc = fmaf(expf(lg - lse), pp.o[g][((int64_t)row * H + h) * D + d], acc);
      }
    if constexpr (sizeof(TO) == 4) {
      o[((int64_t)row * H + h) * D + d] = acc;
    } else {
      o[((int64_t)row * H + h) * D + d] = TO(acc);
    }
  }
  if (lane == 0 && lse_out != nullptr) lse_out[li] = lse;
}

// Weighted sum of n split-KV partials against a log-sum-exp computed elsewhere (the first half
// of a merge whose partials live on several GPUs): o = sum_g exp(lse_g - lse_ref) o_g, with a
// term of 0 where lse_g or lse_ref is -inf. When lse_ref is the log-sum-exp of every partial of
// the row on every GPU, the per-GPU sums add up (a reduce-scatter) to the exact merged row, so
// no second pass over the output is needed. One warp per (row, head); each lane owns four
// consecutive columns (16-byte loads) when D % 4 == 0 and every pointer is 16-byte aligned.
template <typename TO>
__global__ void lse_rescale_sum_kernel(const __grid_constant__ PartPtrs pp, int n, int rows,
                                       int H, int D, const float* __restrict__ lse_ref, TO* o,
                                       int vec4) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)rows * H) return;
  const int row = (int)(w / H), h = (int)(w % H);
  const int64_t li = (int64_t)h * rows + row;
  const int64_t oi = ((int64_t)row * H + h) * D;
  const float ref = lse_ref[li];
  float wg[kMaxParts];
#pragma unroll 4
  for (int g = 0; g < n; ++g) {
    const float lg = pp.lse[g][li];
    wg[g] = (lg == -INFINITY || ref == -INFINITY) ? 0.f : expf(lg - ref);
  }
  auto put = [&](int d, float v) {
    if constexpr (sizeof(TO) == 4) {
      o[oi + d] = v;
    } else {
      o[oi + d] = TO(v);
    }
  };
  if (vec4) {
    for (int c = 4 * lane; c < D; c += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int g = 0; g < n; ++g) {
        if (wg[g] == 0.f) continue;  // also skips partials that were never written (-inf rows)
        const float4 x = *reinterpret_cast<const float4*>(pp.o[g] + oi + c);
        acc.x = fmaf(wg[g], x.x, acc.x);
        acc.y = fmaf(wg[g], x.y, acc.y);
        acc.z = fmaf(wg[g], x.z, acc.z);
        acc.w = fmaf(wg[g], x.w, acc.w);
      }
      if constexpr (sizeof(TO) == 4) {
        *reinterpret_cast<float4*>(o + oi + c) = acc;
      } else {
        put(c, acc.x);
        put(c + 1, acc.y);
        put(c + 2, acc.z);
        put(c + 3, acc.w);
      }
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      float acc = 0.f;
      for (int g = 0; g < n; ++g)
        if (wg[g] != 0.f) acc = fmaf(wg[g], pp.o[g][oi + d], acc);
      put(d, acc);
    }
  }
}

// Local merge of n partials of the same rows held in one buffer (the receive buffer of a
// split-KV over GPUs): parts fp32 [n][rows][H][D] (partial g at parts + g * part_stride), each
// normalised by its own softmax sum, lses fp32 [n][H][rows] (lses + g * lse_stride). Writes
// o [rows][H][D] in TO and optionally lse_out [H][rows]: lse = log sum_g exp(lse_g),
// o = sum_g exp(lse_g - lse) o_g; rows no partial attends get 0 and -inf. One warp per
// (row, head); lanes own four consecutive columns when vec4.
template <typename TO>
__global__ void lse_merge_kernel(const float* __restrict__ parts, const float* __restrict__ lses,
                                 int n, int rows, int H, int D, int64_t part_stride,
                                 int64_t lse_stride, TO* o, float* lse_out, int vec4) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)rows * H) return;
  const int row = (int)(w / H), h = (int)(w % H);
  const int64_t li = (int64_t)h * rows + row;
  const int64_t oi = ((int64_t)row * H + h) * D;
  float mx = -INFINITY;
  for (int g = 0; g < n; ++g) mx = fmaxf(mx, lses[g * lse_stride + li]);
  float tot = 0.f;
  if (mx != -INFINITY)
    for (int g = 0; g < n; ++g) {
      const float lg = lses[g * lse_stride + li];
      if (lg != -INFINITY) tot += expf(lg - mx);
    }
  const float lse = mx == -INFINITY ? -INFINITY : mx + logf(tot);
  const float inv = mx == -INFINITY ? 0.f : 1.f / tot;
  auto put = [&](int d, float v) {
    if constexpr (sizeof(TO) == 4) {
      o[oi + d] = v;
    } else {
      o[oi + d] = TO(v);
    }
  };
  if (vec4) {
    for (int c = 4 * lane; c < D; c += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int g = 0; g < n && mx != -INFINITY; ++g) {
        const float lg = lses[g * lse_stride + li];
        if (lg == -INFINITY) continue;  // a partial that saw no key of this row
        const float wg = expf(lg - mx) * inv;
        const float4 x = *reinterpret_cast<const float4*>(parts + g * part_stride + oi + c);
        acc.x = fmaf(wg, x.x, acc.x);
        acc.y = fmaf(wg, x.y, acc.y);
        acc.z = fmaf(wg, x.z, acc.z);
        acc.w = fmaf(wg, x.w, acc.w);
      }
      if constexpr (sizeof(TO) == 4) {
        *reinterpret_cast<float4*>(o + oi + c) = acc;
      } else {
        put(c, acc.x);
        put(c + 1, acc.y);
        put(c + 2, acc.z);
        put(c + 3, acc.w);
      }
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      float acc = 0.f;
      for (int g = 0; g < n && mx != -INFINITY; ++g) {
        const float lg = lses[g * lse_stride + li];
        if (lg != -INFINITY) acc = fmaf(expf(lg - mx) * inv, parts[g * part_stride + oi + d], acc);
      }
      put(d, acc);
    }
  }
  if (lane == 0 && lse_out != nullptr) lse_out[li] = lse;
}

// Merge of a row window from partials held by several GPUs (the pull side of a split-KV over
// GPUs): partial g is fp32 [rows_total][H][D] at pp.o[g] (a peer-mapped pointer when another GPU
// holds it) with its row log-sum-exp [H][rows_total] at pp.lse[g]. Rows [row0, row0 + nrows)
// are merged into o [nrows][H][D] (TO) and optionally lse_out [H][nrows]. Plain loads, one warp
// per (row, head), four consecutive columns per lane when vec4.
template <typename TO>
__global__ void lse_merge_rows_kernel(const __grid_constant__ PartPtrs pp, int n, int rows_total,
                                      int row0, int nrows, int H, int D, TO* o, float* lse_out,
                                      int vec4) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)nrows * H) return;
  const int r = (int)(w / H), h = (int)(w % H);
  const int64_t li = (int64_t)h * rows_total + row0 + r;
  const int64_t si = ((int64_t)(row0 + r) * H + h) * D;
  const int64_t oi = ((int64_t)r * H + h) * D;
  float lg[kMaxParts];
  float mx = -INFINITY;
  for (int g = 0; g < n; ++g) {
    lg[g] = pp.lse[g][li];
    mx = fmaxf(mx, lg[g]);
  }
  float tot = 0.f;
  if (mx != -INFINITY)
    for (int g = 0; g < n; ++g)
      if (lg[g] != -INFINITY) tot += expf(lg[g] - mx);
  const float inv = mx == -INFINITY ? 0.f : 1.f / tot;
  for (int g = 0; g < n; ++g) lg[g] = (lg[g] == -INFINITY || mx == -INFINITY) ? 0.f : expf(lg[g] - mx) * inv;
  auto put = [&](int d, float v) {
    if constexpr (sizeof(TO) == 4) {
      o[oi + d] = v;
    } else {
      o[oi + d] = TO(v);
    }
  };
  if (vec4) {
    for (int c = 4 * lane; c < D; c += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int g = 0; g < n; ++g) {
        if (lg[g] == 0.f) continue;  // a partial that saw no key of this row
        const float4 x = *reinterpret_cast<const float4*>(pp.o[g] + si + c);
        acc.x = fmaf(lg[g], x.x, acc.x);
        acc.y = fmaf(lg[g], x.y, acc.y);
        acc.z = fmaf(lg[g], x.z, acc.z);
        acc.w = fmaf(lg[g], x.w, acc.w);
      }
      if constexpr (sizeof(TO) == 4) {
        *reinterpret_cast<float4*>(o + oi + c) = acc;
      } else {
        put(c, acc.x);
        put(c + 1, acc.y);
        put(c + 2, acc.z);
        put(c + 3, acc.w);
      }
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      float acc = 0.f;
      for (int g = 0; g < n; ++g)
        if (lg[g] != 0.f) acc = fmaf(lg[g], pp.o[g][si + d], acc);
      put(d, acc);
    }
  }
  if (lane == 0 && lse_out != nullptr)
    lse_out[(int64_t)h * nrows + r] = mx == -INFINITY ? -INFINITY : mx + logf(tot);
}

// Merge of the key splits of one launch (dense layout): partial outputs ws_o fp32
// [split][B][Lq][Hq][D] normalised by their own sums, row log-sum-exp ws_lse [split][B][Hq][Lq].
// One block of kCombineThreads per (batch, head, row). The split weights exp(lse_s - max) are
// computed in parallel into shared memory (a.num_splits floats of dynamic shared memory); then
// warp w sums the splits w, w + 8, ... of the row, each lane four columns with 16-byte loads, so
// a thread's loads are independent of one another; the eight warp sums meet in shared memory
// and the final row is written in the caller's dtype and strides. D is a multiple of 8 (the
// tcgen05 path's requirement) and the workspace is 256-byte aligned, so the loads are aligned.
// The kernel is launched as a programmatic dependent of the forward: griddepcontrol.wait holds
// it until the forward grid has finished and its writes are visible.
constexpr int kCombineThreads = 256;
constexpr int kCombineWarps = kCombineThreads / 32;
__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int w = 1; w < kCombineWarps; ++w) v = is_max ? fmaxf(v, red[w]) : v + red[w];
  return v;
}

template <typename TO>
__global__ void __launch_bounds__(kCombineThreads)
    split_combine_kernel(const FwdArgs a, const float* __restrict__ ws_o,
                         const float* __restrict__ ws_lse, TO* o, float* lse_out) {
  extern __shared__ float sw[];  // [num_splits]
  __shared__ float red[kCombineWarps];
  __shared__ float4 part[kCombineWarps][32];  // per-warp column sums (D <= 128)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t w = blockIdx.x;
  const int row = (int)(w % a.Lq);
  const int bh = (int)(w / a.Lq);
  const int h = bh % a.Hq, b = bh / a.Hq;
  // varlen: only the packed rows of this launch's sequences hold partials; a launch over some of
  // the sequences of a larger packed batch leaves every other row (and its slots) alone
  if (a.cu_q != nullptr && (row < a.cu_q[0] || row >= a.cu_q[a.nseq])) return;
  const int64_t li = ((int64_t)b * a.Hq + h) * a.Lq + row;
  const int64_t lstride = (int64_t)a.B * a.Hq * a.Lq;
  const int64_t ostride = lstride * a.D;
  const int64_t oi = (((int64_t)b * a.Lq + row) * a.Hq + h) * a.D;
  const int S = a.num_splits;
  float mx = -INFINITY;
  for (int s = threadIdx.x; s < S; s += kCombineThreads) mx = fmaxf(mx, ws_lse[s * lstride + li]);
  mx = block_reduce(mx, true, red);
  float tot = 0.f;
  for (int s = threadIdx.x; s < S; s += kCombineThreads) {
    const float ls = ws_lse[s * lstride + li];
    const float e = (mx == -INFINITY || ls == -INFINITY) ? 0.f : expf(ls - mx);
    sw[s] = e;
    tot += e;
  }
  tot = block_reduce(tot, false, red);  // its barriers also publish sw
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool has_cols = 4 * lane < a.D;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (has_cols) {
    const float4* src = reinterpret_cast<const float4*>(ws_o + oi) + lane;
    const int64_t step = ostride / 4;  // float4 per split
#pragma unroll 4
    for (int s = warp; s < S; s += kCombineWarps) {
      const float4 x = src[s * step];
      const float ws = sw[s];
      acc.x = fmaf(ws, x.x, acc.x);
      acc.y = fmaf(ws, x.y, acc.y);
      acc.z = fmaf(ws, x.z, acc.z);
      acc.w = fmaf(ws, x.w, acc.w);
    }
  }
  part[warp][lane] = acc;
  __syncthreads();
  // thread t < D writes column t: the sum over the warps of lane t/4's component t%4
  TO* orow = o + (int64_t)b * a.o_sb + (int64_t)row * a.o_ss + (int64_t)h * a.o_sh;
  for (int d = threadIdx.x; d < a.D; d += kCombineThreads) {
    const float* pc = reinterpret_cast<const float*>(&part[0][0]) + d;  // column d of warp 0
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < kCombineWarps; ++q) v += pc[q * 128];
    v *= inv;
    if constexpr (sizeof(TO) == 4) {
      orow[d] = v;
    } else {
      orow[d] = TO(v);
    }
  }
  if (threadIdx.x == 0 && lse_out != nullptr)
    lse_out[(int64_t)b * a.lse_sb + (int64_t)h * a.lse_sh + row] =
        tot > 0.f ? mx + logf(tot) : -INFINITY;
}

// Self-test of the bounded wait every pipelined kernel uses: one thread waits on an mbarrier
// that nothing ever arrives on, gives up after `timeout_ns` of device time and reports
// MFA_ERR_TIMEOUT (4) in *err, exactly as a stalled attention CTA does. No fault, trap or hang.
__global__ void wait_timeout_selftest(int* err, uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const bool ok = mbar_wait(&bar, 0, &abort_flag, timeout_ns);
  *err = ok ? 0 : 4;
}

}  // namespace mfa
