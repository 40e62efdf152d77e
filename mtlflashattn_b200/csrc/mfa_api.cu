// C ABI of libmfa.so (declared in include/mfa.h): argument checks, kernel choice, TMA tensor
// maps and launches. Replaces the tier dispatch of the reference's flash_attn_forward
// (metal_flash_attn/_kernel.py:1052-1153) and its Metal launchers (_kernel.py:1288-1420).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/mfa.h"
#include "fa_simt.cuh"
#include "fa_sm100.cuh"

namespace mfa {
// The fp32 CUDA-core forward, compiled in simt_fwd.cu without fast math.
int simt_forward(FwdArgs a, int dtype, int D, cudaStream_t st);
}  // namespace mfa

static_assert(mfa::kMaxPeers == MFA_MAX_PEERS, "peer table size differs from the header's");
static_assert(mfa::kErrCheck == MFA_ERR_CHECK, "device check status differs from the header's");

namespace mfa {
namespace {

// ------------------------------------------------------------------ host fault injection
// MFA_FAULT=<site>[,<site>...] makes the named entry point fail before it launches anything,
// so callers' error handling can be tested without touching a GPU. Sites: fwd, combine.
bool fault_injected(const char* site) {
  const char* env = std::getenv("MFA_FAULT");
  if (env == nullptr || *env == 0) return false;
  const size_t n = std::strlen(site);
  for (const char* p = env; *p;) {
    const char* e = std::strchr(p, ',');
    const size_t len = e ? (size_t)(e - p) : std::strlen(p);
    if (len == n && std::strncmp(p, site, n) == 0) return true;
    if (!e) break;
    p = e + 1;
  }
  return false;
}

// ------------------------------------------------------------------ NVTX
// Host-side range around each launching entry point, named after it, so an nsys / ncu timeline
// shows which library call queued which kernels. NVTX v3 is header-only: with no tool attached
// a push/pop is a test of a null function pointer.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};

// ------------------------------------------------------------------ driver entry point
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct DevInfo {
  int major = -1, minor = -1, sms = 0;
};
DevInfo dev_info(int dev) {
  static std::mutex mu;
  static DevInfo cache[64];
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0 || dev >= 64) return DevInfo{};
  if (cache[dev].major < 0) {
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&cache[dev].minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return cache[dev];
}

// cudaFuncSetAttribute once per (kernel, device).
template <typename K>
cudaError_t ensure_smem(K kernel, int dev, int bytes) {
  static std::mutex mu;
  static const void* seen[256];
  static int seen_dev[256];
  static int nseen = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < nseen; ++i)
    if (seen[i] == (const void*)kernel && seen_dev[i] == dev) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  // all of the SM's unified L1/shared storage as shared memory (two one-tile CTAs per SM)
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess && nseen < 256) {
    seen[nseen] = (const void*)kernel;
    seen_dev[nseen] = dev;
    ++nseen;
  }
  return e;
}

int esize(int dtype) { return dtype == MFA_FP32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Argument checks. Mirrors the checks the reference makes before any tier runs
// (metal_flash_attn/__init__.py:28-59, 84-90; _kernel.py:1070-1074, 1145-1147).
int validate(const mfa_fwd_params* p) {
  if (p == nullptr) return MFA_ERR_INVALID;
  if (p->dtype < 0 || p->dtype > 2) return MFA_ERR_UNSUPPORTED;
  const int od = p->o_dtype < 0 ? p->dtype : p->o_dtype;
  if (od > 2) return MFA_ERR_UNSUPPORTED;
  if (p->D < 1 || p->D > 128) return MFA_ERR_UNSUPPORTED;
  if (p->B < 0 || p->Hq < 1 || p->Hkv < 1 || p->Hq % p->Hkv != 0) return MFA_ERR_INVALID;
  if (!(p->softcap >= 0.f)) return MFA_ERR_INVALID;
  if (p->win_left < -1 || p->win_right < -1) return MFA_ERR_INVALID;
  const bool varlen = p->cu_q != nullptr || p->cu_k != nullptr;
  if (varlen && (p->cu_q == nullptr || p->cu_k == nullptr)) return MFA_ERR_INVALID;
  if (!varlen && (p->Lq < 0 || p->Lk < 0)) return MFA_ERR_INVALID;
  if (varlen && p->max_lq < 0) return MFA_ERR_INVALID;
  if (p->B == 0 || (!varlen && p->Lq == 0) || (varlen && p->max_lq == 0)) return MFA_OK;
  if (p->q == nullptr || p->o == nullptr) return MFA_ERR_INVALID;
  if ((p->k == nullptr || p->v == nullptr) && p->Lk > 0) return MFA_ERR_INVALID;
  return MFA_OK;
}

FwdArgs resolve(const mfa_fwd_params* p) {
  FwdArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = p->q;
  a.k = p->k;
  a.v = p->v;
  a.o = p->o;
  a.lse = p->lse;
  a.q_sb = p->q_stride[0]; a.q_ss = p->q_stride[1]; a.q_sh = p->q_stride[2];
  a.k_sb = p->k_stride[0]; a.k_ss = p->k_stride[1]; a.k_sh = p->k_stride[2];
  a.v_sb = p->v_stride[0]; a.v_ss = p->v_stride[1]; a.v_sh = p->v_stride[2];
  a.o_sb = p->o_stride[0]; a.o_ss = p->o_stride[1]; a.o_sh = p->o_stride[2];
  a.lse_sb = p->lse_stride[0];
  a.lse_sh = p->lse_stride[1];
  a.B = p->B;
  a.Hq = p->Hq;
  a.Hkv = p->Hkv;
  a.Lq = p->Lq;
  a.Lk = p->Lk;
  a.D = p->D;
  a.group = p->Hq / p->Hkv;
  a.cu_q = p->cu_q;
  a.cu_k = p->cu_k;
  a.max_lq = p->cu_q ? p->max_lq : p->Lq;
  a.scale = p->scale;
  a.softcap = p->softcap;
  a.causal = p->causal ? 1 : 0;
  a.wl = p->win_left;
  a.wr = p->win_right;
  a.alibi = p->alibi;
  a.o_dtype = p->o_dtype < 0 ? p->dtype : p->o_dtype;
  const int oes = esize(a.o_dtype);
  a.o_vec16 = aligned16(p->o) && (a.o_ss * oes) % 16 == 0 && (a.o_sh * oes) % 16 == 0 &&
              (p->cu_q != nullptr || (a.o_sb * oes) % 16 == 0);
  a.k_pos_offset = p->k_pos_offset;
  a.lk_total = p->lk_total;
  a.err = p->err;
  a.num_splits = 1;
  a.nseq = p->B;
  return a;
}

// ---- key split within one launch (decode-like shapes)
// When the (row block, batch, head) CTAs of a dense launch cover well under two waves of the
// GPU and there are enough keys, each CTA's keys are cut into `splits` ranges run by separate
// CTAs; their partial rows are merged by split_combine_kernel. Ranges are whole 128-key blocks
// and each holds at least two blocks.
struct SplitPlan {
  int splits = 1;
  int split_keys = 0;
  size_t bytes = 0;
};
// Bias mode of the tcgen05 kernel: 2 softcap, 1 ALiBi or a non-positive scale, 0 plain.
int sm100_gen(const mfa_fwd_params* p) {
  return p->softcap > 0.f ? 2 : (!(p->scale > 0.f) || p->alibi != nullptr) ? 1 : 0;
}
int sm100_tiles_rt(bool wide, int gen);

// Query heads packed per KV head (log2; 0 = none). Decode-like launches (fewer than 128 query
// rows per sequence) of a GQA/MQA model put the query heads of one KV group into the rows of one
// tile, so each K/V block is loaded once for the whole group instead of once per query head.
// The group must be a power of two up to 16: the packed Q box is (64, group, 128 / group).
int pack_shift_for(const mfa_fwd_params* p) {
#if MFA_PACK_GQA
  const int g = p->Hq / p->Hkv;
  const int max_lq = p->cu_q != nullptr ? p->max_lq : p->Lq;
  if (g < 2 || g > 16 || (g & (g - 1)) != 0 || max_lq >= 128) return 0;
  int s = 0;
  while ((1 << s) < g) ++s;
  return s;
#else
  (void)p;
  return 0;
#endif
}

// Decode-like launches (query heads packed, or at most 128 query rows per sequence) run the
// kPack instantiation in one-tile CTAs, two per SM: a second tile would mostly stay empty, and
// two CTAs per SM overlap the load -> QK -> softmax -> PV chain of one key block with another's.
bool sm100_short(const mfa_fwd_params* p) {
  const int max_lq = p->cu_q != nullptr ? p->max_lq : p->Lq;
  return pack_shift_for(p) > 0 || max_lq <= 128;
}
// Tiles per CTA of the tcgen05 kernel for these params.
int sm100_tiles_for(const mfa_fwd_params* p) {
  return sm100_short(p) ? 1 : sm100_tiles_rt(p->D > 64, sm100_gen(p));
}

#ifndef MFA_MAX_SPLITS
#define MFA_MAX_SPLITS 128
#endif
#ifndef MFA_SPLIT_MIN_BLOCKS
#define MFA_SPLIT_MIN_BLOCKS 8  // key blocks per split at least
#endif

// Splits fill one wave of resident CTAs (7/8 of the slots: a split CTA that lands in a second
// wave doubles the launch's span) with at least 8 key blocks each (below that the per-CTA setup
// and the merge outweigh the gain). Measured on B200 over decode shapes from 1 to 128 query
// rows and 2K to 128K keys, this picks the fastest split count or one within a few percent.
// Varlen launches split by the longest sequence's keys (max_lk); every split CTA of a shorter
// sequence whose keys end before its range writes an empty partial (weight 0 in the merge), and
// the last split takes all keys past its start, so an understated max_lk loses nothing.
SplitPlan plan_splits(const mfa_fwd_params* p, int sms) {
  SplitPlan sp;
  const bool varlen = p->cu_q != nullptr;
  const int64_t lq = varlen ? p->max_lq : p->Lq;
  const int64_t lk = varlen ? p->max_lk : p->Lk;
  if (p->B == 0 || lq <= 0 || lk <= 0) return sp;
  const int ps = pack_shift_for(p);
  const int tiles = sm100_tiles_for(p);
  const int64_t rows_per_cta = (int64_t)tiles * 128;
  const int64_t slots = (int64_t)sms * (tiles == 1 ? 2 : 1);  // resident CTAs
  const int64_t row_blocks = ((lq << ps) + rows_per_cta - 1) / rows_per_cta;
  const int64_t ctas = row_blocks * (p->Hq >> ps) * p->B;
  const int64_t key_blocks = (lk + 127) / 128;
  int64_t s = (slots - slots / 8) / ctas;
  s = s < key_blocks / MFA_SPLIT_MIN_BLOCKS ? s : key_blocks / MFA_SPLIT_MIN_BLOCKS;
  s = s < MFA_MAX_SPLITS ? s : MFA_MAX_SPLITS;
  if (s < 2) return sp;
  const int64_t blocks_per = (key_blocks + s - 1) / s;
  sp.split_keys = (int)(blocks_per * 128);
  sp.splits = (int)((lk + sp.split_keys - 1) / sp.split_keys);
  if (sp.splits < 2) return SplitPlan{};
  // partial rows: [B][Lq][Hq] dense, [total_q][Hq] varlen (Lq carries total_q)
  const size_t rows = (size_t)(varlen ? 1 : p->B) * p->Hq * p->Lq;
  sp.bytes = (size_t)sp.splits * rows * ((size_t)p->D + 1) * sizeof(float) + 256;
  return sp;
}

// tcgen05 path eligibility: 16-bit inputs, D a multiple of 8 (TMA needs 16-byte strides),
// 16-byte aligned bases and strides, and an sm_100 device.
bool tc_eligible(const mfa_fwd_params* p, const DevInfo& di) {
  if (di.major != 10 || di.minor != 0) return false;
  if (p->dtype != MFA_FP16 && p->dtype != MFA_BF16) return false;
  if (p->D % 8 != 0) return false;
  const void* ptrs[3] = {p->q, p->k, p->v};
  const int64_t* strides[3] = {p->q_stride, p->k_stride, p->v_stride};
  const bool varlen = p->cu_q != nullptr;
  for (int i = 0; i < 3; ++i) {
    if (!aligned16(ptrs[i])) return false;
    const int64_t extent[3] = {varlen ? 1 : p->B, i == 0 ? p->Lq : p->Lk, i == 0 ? p->Hq : p->Hkv};
    for (int d = 0; d < 3; ++d) {
      if (extent[d] <= 1) continue;  // a unit dimension's stride is never used
      const int64_t s = strides[i][d] * 2;
      if (s <= 0 || s % 16 != 0 || s >= (1ll << 40)) return false;
    }
  }
  return true;
}

int pick_kernel(const mfa_fwd_params* p, int dev) {
  const DevInfo di = dev_info(dev);
  if (p->kernel == MFA_KERNEL_SIMT) return MFA_KERNEL_SIMT;
  // An empty key set has nothing to stream; the CUDA-core kernel writes the zero rows.
  const bool ok = tc_eligible(p, di) && p->Lk > 0;
  if (p->kernel == MFA_KERNEL_TCGEN05) return ok ? MFA_KERNEL_TCGEN05 : -MFA_ERR_UNSUPPORTED;
  return ok ? MFA_KERNEL_TCGEN05 : MFA_KERNEL_SIMT;
}

// 4-D tensor map over (D, H, S, B) with a (64, 1, 128, 1) box and 128-byte swizzle.
int encode_map(CUtensorMap* m, const void* base, int dtype, int D, int H, int64_t S, int B,
             const int64_t* stride /* batch, seq, head (elements) */, int box_h = 1,
             int rows = 128) {
  auto fn = encode_fn();
  if (fn == nullptr) return MFA_ERR_CUDA;
  const int64_t es = 2;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)(S > 0 ? S : 1),
                        (cuuint64_t)(B > 0 ? B : 1)};
  int64_t sh = stride[2] * es, ss = stride[1] * es, sbt = stride[0] * es;
  // a unit dimension's stride is never used, but must be encodable
  if (H <= 1) sh = 16;
  if (S <= 1) ss = 16;
  if (B <= 1) sbt = 16;
  cuuint64_t strides[3] = {(cuuint64_t)sh, (cuuint64_t)ss, (cuuint64_t)sbt};
  cuuint32_t box[4] = {64, (cuuint32_t)box_h, (cuuint32_t)(rows / box_h), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, dtype == MFA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MFA_OK : MFA_ERR_CUDA;
}

// Tensor maps are pure functions of (base, dtype, D, H, S, B, strides, box), so repeated calls
// on the same buffers (a decode loop, a benchmark, every layer of a model with a static
// allocator) reuse the encoded map instead of calling cuTensorMapEncodeTiled three or four
// times per forward. A small direct-mapped table under one mutex; a miss encodes and replaces
// the slot. Encoding costs ~1-2 us of host time per map; the lookup is a hash and a compare.
struct MapKey {
  const void* base;
  int64_t S, stride[3];
  int dtype, D, H, B, box_h, rows;
  bool operator==(const MapKey& o) const {
    return base == o.base && S == o.S && stride[0] == o.stride[0] && stride[1] == o.stride[1] &&
           stride[2] == o.stride[2] && dtype == o.dtype && D == o.D && H == o.H && B == o.B &&
           box_h == o.box_h && rows == o.rows;
  }
};
constexpr int kMapSlots = 256;
struct MapSlot {
  bool used = false;
  MapKey key;
  CUtensorMap map;
};

int make_map(CUtensorMap* m, const void* base, int dtype, int D, int H, int64_t S, int B,
             const int64_t* stride, int box_h = 1, int rows = 128) {
  static std::mutex mu;
  static MapSlot slots[kMapSlots];
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  key.base = base;
  key.S = S;
  key.stride[0] = stride[0];
  key.stride[1] = stride[1];
  key.stride[2] = stride[2];
  key.dtype = dtype;
  key.D = D;
  key.H = H;
  key.B = B;
  key.box_h = box_h;
  key.rows = rows;
  uint64_t h = reinterpret_cast<uintptr_t>(base) >> 4;
  const int64_t mix[8] = {S, stride[0], stride[1], stride[2], dtype, D, H,
                          ((int64_t)B * 64 + box_h) * 512 + rows};
  for (int i = 0; i < 8; ++i) h = (h ^ (uint64_t)mix[i]) * 0x100000001b3ull;
  MapSlot& sl = slots[(h ^ (h >> 29)) % kMapSlots];
  {
    std::lock_guard<std::mutex> g(mu);
    if (sl.used && sl.key == key) {
      *m = sl.map;
      return MFA_OK;
    }
  }
  const int rc = encode_map(m, base, dtype, D, H, S, B, stride, box_h, rows);
  if (rc == MFA_OK) {
    std::lock_guard<std::mutex> g(mu);
    sl.used = true;
    sl.key = key;
    sl.map = *m;
  }
  return rc;
}

// Tiles per CTA of the tcgen05 kernel fa_fwd_sm100<DP, *, GEN> (its default template argument).
template <int DP, int GEN>
constexpr int sm100_tiles() {
  return DefaultTiles<DP, DefaultCG<GEN, DP>::value, GEN>::value;
}
int sm100_tiles_rt(bool wide, int gen) {
  if (wide) return gen == 2 ? sm100_tiles<128, 2>() : gen == 1 ? sm100_tiles<128, 1>() : sm100_tiles<128, 0>();
  return gen == 2 ? sm100_tiles<64, 2>() : gen == 1 ? sm100_tiles<64, 1>() : sm100_tiles<64, 0>();
}

// K/V bytes of the (batch, head) pairs whose CTAs run together (see run_sm100). Measured with
// ncu on B200, B=1 H=16 L=8192 D=128 causal (67 MB of K/V): 64 MB groups (all heads at once)
// read 137-141 MB of DRAM per launch against 100.7 MB of compulsory Q/K/V, 32 MB groups (8
// heads) read 100.7 MB, in the same time (263 us). The 126 MB L2 does not keep 67 MB of K/V
// that every SM reads, so the group budget is a quarter of it.
#ifndef MFA_L2_GROUP_MB
#define MFA_L2_GROUP_MB 32
#endif

// Keys per K/V block of the instantiation launch_sm100 will pick (BlockKeys on the host).
template <int DP, int GEN, bool SHORT>
constexpr int sm100_kbn() {
  return SHORT ? sm100::BlockKeys<DP, GEN, 1, 1, true>::value
               : sm100::BlockKeys<DP, GEN, DefaultCG<GEN, DP>::value, sm100_tiles<DP, GEN>(),
                                        false>::value;
}
int sm100_kbn_rt(bool wide, int gen, bool short_rows) {
#define MFA_KBN(DP)                                                                          \
  (short_rows ? (gen == 2 ? sm100_kbn<DP, 2, true>() : gen == 1 ? sm100_kbn<DP, 1, true>()  \
                                                                : sm100_kbn<DP, 0, true>())  \
              : (gen == 2 ? sm100_kbn<DP, 2, false>() : gen == 1 ? sm100_kbn<DP, 1, false>() \
                                                                 : sm100_kbn<DP, 0, false>()))
  return wide ? MFA_KBN(128) : MFA_KBN(64);
#undef MFA_KBN
}

// SHORT: the one-tile, one-column-group kPack instantiation (sm100_short).
template <int DP, bool BF16, int GEN, bool SHORT>
int launch_sm100(const Sm100Args& args, int dev, int64_t grid, cudaStream_t st) {
  constexpr int CG = SHORT ? 1 : DefaultCG<GEN, DP>::value;
  constexpr int TILES = SHORT ? 1 : sm100_tiles<DP, GEN>();
  auto k = fa_fwd_sm100<DP, BF16, GEN, CG, TILES, SHORT>;
  using R = sm100::Roles<CG, TILES>;
  constexpr int KBN = sm100::BlockKeys<DP, GEN, CG, TILES, SHORT>::value;
  const int smem = (int)sm100::Cfg<DP, TILES, KBN>::SMEM;
  // The kernel re-splits its registers with setmaxnreg assuming exactly kLaunchRegs per thread
  // at launch; a build that launched with fewer would make setmaxnreg.inc wait forever.
  static std::atomic<int> launch_regs{-1};
  int regs = launch_regs.load(std::memory_order_relaxed);
  if (regs < 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) return MFA_ERR_CUDA;
    regs = fa.numRegs;
    launch_regs.store(regs, std::memory_order_relaxed);
  }
  if (regs != R::kLaunchRegs) return MFA_ERR_UNSUPPORTED;
  if (ensure_smem(k, dev, smem) != cudaSuccess) return MFA_ERR_CUDA;
  k<<<(unsigned)grid, R::kThreads, smem, st>>>(args);
  return MFA_OK;
}

int launch_combine(const FwdArgs& fin, const float* ws_o, const float* ws_lse, void* o,
                   float* lse, cudaStream_t st) {
  const int64_t rows = (int64_t)fin.B * fin.Hq * fin.Lq;
  if (rows == 0) return MFA_OK;
  if (rows >= (1ll << 31)) return MFA_ERR_UNSUPPORTED;
  // a programmatic dependent launch: the merge grid is set up while the forward drains and
  // waits (griddepcontrol.wait) for its completion before reading the partials
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = (size_t)fin.num_splits * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (fin.o_dtype == MFA_FP32)
    e = cudaLaunchKernelEx(&cfg, split_combine_kernel<float>, fin, ws_o, ws_lse, (float*)o, lse);
  else if (fin.o_dtype == MFA_BF16)
    e = cudaLaunchKernelEx(&cfg, split_combine_kernel<__nv_bfloat16>, fin, ws_o, ws_lse,
                           (__nv_bfloat16*)o, lse);
  else
    e = cudaLaunchKernelEx(&cfg, split_combine_kernel<__half>, fin, ws_o, ws_lse, (__half*)o, lse);
  return e == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int run_sm100(const mfa_fwd_params* p, FwdArgs a, int dev, cudaStream_t st,
              const SplitPlan& split, void* workspace) {
  Sm100Args args;
  std::memset(&args, 0, sizeof(args));
  const bool varlen = p->cu_q != nullptr;
  const int64_t Sq = varlen ? p->Lq : p->Lq;  // varlen: Lq carries total_q
  const int64_t Sk = varlen ? p->Lk : p->Lk;
  const int Bm = varlen ? 1 : p->B;
  int rc;
  if ((rc = make_map(&args.tq, p->q, p->dtype, p->D, p->Hq, Sq, Bm, p->q_stride)) != MFA_OK) return rc;
  // K / V boxes are one block of keys of the instantiation that will run
  const int kbn = sm100_kbn_rt(p->D > 64, sm100_gen(p), sm100_short(p));
  if ((rc = make_map(&args.tk, p->k, p->dtype, p->D, p->Hkv, Sk, Bm, p->k_stride, 1, kbn)) != MFA_OK)
    return rc;
  if ((rc = make_map(&args.tv, p->v, p->dtype, p->D, p->Hkv, Sk, Bm, p->v_stride, 1, kbn)) != MFA_OK)
    return rc;
  const int gen = sm100_gen(p);
  const bool wide = p->D > 64;
  const bool short_rows = sm100_short(p);
  const int rows_per_cta = (short_rows ? 1 : sm100_tiles_rt(wide, gen)) * sm100::BM;
  a.pack_shift = pack_shift_for(p);
  const int heads = p->Hq >> a.pack_shift;  // per batch: query heads, or KV heads when packed
  if (a.pack_shift > 0 &&
      (rc = make_map(&args.tqp, p->q, p->dtype, p->D, p->Hq, Sq, Bm, p->q_stride,
                     1 << a.pack_shift)) != MFA_OK)
    return rc;
  a.num_row_blocks = (int)((((int64_t)a.max_lq << a.pack_shift) + rows_per_cta - 1) / rows_per_cta);
  {
    // K/V bytes of one KV head of one sequence; groups of whole KV groups whose K/V stays
    // within MFA_L2_GROUP_MB of L2 (all of them when everything fits)
    const int64_t kv_unit = (int64_t)(varlen ? p->max_lk : p->Lk) * p->D * 2 * 2;
    int64_t units = kv_unit > 0 ? ((int64_t)MFA_L2_GROUP_MB << 20) / kv_unit : (1ll << 30);
    if (units < 1) units = 1;
    const int64_t all = (int64_t)heads * a.B;
    const int64_t ghb = units * (p->Hq / p->Hkv >> a.pack_shift);
    a.group_hb = (int)(ghb < all ? ghb : all);
  }
  FwdArgs fin = a;  // the caller's output, for the split merge
  fin.num_splits = split.splits;
  if (varlen) fin.B = 1;  // the merge walks the packed rows [total_q][Hq] as one batch
  float* ws_o = nullptr;
  float* ws_lse = nullptr;
  if (split.splits > 1) {
    // partials: fp32 [split][B][Lq][Hq][D] and row lse [split][B][Hq][Lq] in the workspace
    uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255;
    ws_o = reinterpret_cast<float*>(base);
    const int64_t rows = (int64_t)(varlen ? 1 : p->B) * p->Hq * p->Lq;
    ws_lse = ws_o + (int64_t)split.splits * rows * p->D;
    a.o = ws_o;
    a.o_dtype = MFA_FP32;
    a.o_sb = (int64_t)p->Lq * p->Hq * p->D;
    a.o_ss = (int64_t)p->Hq * p->D;
    a.o_sh = p->D;
    a.o_vec16 = 0;
    a.lse = ws_lse;
    a.lse_sb = (int64_t)p->Hq * p->Lq;
    a.lse_sh = p->Lq;
    a.num_splits = split.splits;
    a.split_keys = split.split_keys;
    a.o_split_stride = rows * p->D;
    a.lse_split_stride = rows;
  }
  args.a = a;
  int64_t grid = (int64_t)a.num_row_blocks * heads * a.B * a.num_splits;
  if (varlen && p->cu_q_host != nullptr && p->B <= kMaxTileSeqs) {
    // exact CTA list: each non-empty sequence's row blocks x heads x splits, longest first
    struct SeqBlocks {
      int seq, nrb;
    };
    SeqBlocks sb[kMaxTileSeqs];
    int n = 0;
    for (int i = 0; i < p->B; ++i) {
      const int64_t rows = (int64_t)(p->cu_q_host[i + 1] - p->cu_q_host[i]) << a.pack_shift;
      if (rows <= 0) continue;  // no query rows: nothing to compute or write
      sb[n++] = SeqBlocks{i, (int)((rows + rows_per_cta - 1) / rows_per_cta)};
    }
    std::stable_sort(sb, sb + n, [](const SeqBlocks& x, const SeqBlocks& y) { return x.nrb > y.nrb; });
    args.tl.n = n;
    args.tl.off[0] = 0;
    int64_t total = 0;
    for (int i = 0; i < n; ++i) {
      args.tl.seq[i] = sb[i].seq;
      total += (int64_t)sb[i].nrb * heads * a.num_splits;
      if (total >= (1ll << 31)) return MFA_ERR_UNSUPPORTED;
      args.tl.off[i + 1] = (int)total;
    }
    grid = total;
  }
  if (grid == 0) return MFA_OK;
  if (grid >= (1ll << 31)) return MFA_ERR_UNSUPPORTED;
  const bool bf = p->dtype == MFA_BF16;
#define MFA_SM100(DP, BF, G)                                                     \
  do {                                                                           \
    const int rc_ = short_rows ? launch_sm100<DP, BF, G, true>(args, dev, grid, st)   \
                               : launch_sm100<DP, BF, G, false>(args, dev, grid, st); \
    if (rc_ != MFA_OK || split.splits < 2) return rc_;                           \
    return launch_combine(fin, ws_o, ws_lse, p->o, p->lse, st);                  \
  } while (0)
  if (wide) {
    if (bf) {
      if (gen == 2) MFA_SM100(128, true, 2);
      if (gen == 1) MFA_SM100(128, true, 1);
      MFA_SM100(128, true, 0);
    }
    if (gen == 2) MFA_SM100(128, false, 2);
    if (gen == 1) MFA_SM100(128, false, 1);
    MFA_SM100(128, false, 0);
  }
  if (bf) {
    if (gen == 2) MFA_SM100(64, true, 2);
    if (gen == 1) MFA_SM100(64, true, 1);
    MFA_SM100(64, true, 0);
  }
  if (gen == 2) MFA_SM100(64, false, 2);
  if (gen == 1) MFA_SM100(64, false, 1);
  MFA_SM100(64, false, 0);
#undef MFA_SM100
}

int run_simt(const mfa_fwd_params* p, const FwdArgs& a, cudaStream_t st) {
  return simt_forward(a, p->dtype, p->D, st) == 0 ? MFA_OK : MFA_ERR_UNSUPPORTED;
}

// ------------------------------------------------------------------ no-allocation variant
// Scratch for mfa_fwd_noalloc: the split-KV partials live in this fixed device array instead of
// a caller-provided workspace. Every GPU that loads the library holds it until the process
// exits. Host code must not pass the symbol itself to a kernel (on the host it only names a
// shadow variable); noalloc_scratch() resolves its device address for the current device.
constexpr size_t kNoAllocScratchBytes = 16u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on `dev` (the current device), looked up once per device.
int noalloc_scratch(int dev, void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  if (dev < 0 || dev >= 64) return MFA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return MFA_ERR_CUDA;
    addr[dev] = p;
  }
  *out = addr[dev];
  return MFA_OK;
}

#include "staged.inc"

}  // namespace
}  // namespace mfa

extern "C" {

int mfa_abi_version(void) { return MFA_ABI_VERSION; }

const char* mfa_status_string(int s) {
  switch (s) {
    case MFA_OK: return "ok";
    case MFA_ERR_INVALID: return "invalid argument";
    case MFA_ERR_UNSUPPORTED: return "unsupported shape, dtype or kernel for this input";
    case MFA_ERR_CUDA: return "CUDA error";
    case MFA_ERR_TIMEOUT: return "in-kernel wait timed out";
    case MFA_ERR_NO_DEVICE: return "no usable CUDA device";
    case MFA_ERR_FAULT_INJECTED: return "fault injected (MFA_FAULT)";
    case MFA_ERR_CHECK: return "a device-side check of an MFA_CHECKS build failed";
    case MFA_ERR_SCRATCH_TOO_SMALL:
      return "problem needs more split-KV scratch than mfa_fwd_noalloc's fixed 16 MiB buffer";
    default: return "unknown status";
  }
}

size_t mfa_fwd_workspace_size(const mfa_fwd_params* p) {
  if (mfa::validate(p) != MFA_OK) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (mfa::pick_kernel(p, dev) != MFA_KERNEL_TCGEN05) return 0;
  return mfa::plan_splits(p, mfa::dev_info(dev).sms).bytes;
}

int mfa_fwd_num_splits(const mfa_fwd_params* p) {
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return -rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -MFA_ERR_NO_DEVICE;
  if (mfa::pick_kernel(p, dev) != MFA_KERNEL_TCGEN05 || p->workspace == nullptr) return 1;
  const mfa::SplitPlan sp = mfa::plan_splits(p, mfa::dev_info(dev).sms);
  return (sp.splits > 1 && p->workspace_bytes >= sp.bytes) ? sp.splits : 1;
}

int mfa_fwd_packed_heads(const mfa_fwd_params* p) {
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return -rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -MFA_ERR_NO_DEVICE;
  if (mfa::pick_kernel(p, dev) != MFA_KERNEL_TCGEN05) return 1;
  return 1 << mfa::pack_shift_for(p);
}

int mfa_select_kernel(const mfa_fwd_params* p) {
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return -rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -MFA_ERR_NO_DEVICE;
  return mfa::pick_kernel(p, dev);
}

int mfa_fwd(const mfa_fwd_params* p, void* stream) {
  if (mfa::fault_injected("fwd")) return MFA_ERR_FAULT_INJECTED;
  mfa::NvtxRange range("mfa_fwd");
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return rc;
  const bool varlen = p->cu_q != nullptr;
  if (p->B == 0 || (!varlen && p->Lq == 0) || (varlen && p->max_lq == 0)) return MFA_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MFA_ERR_NO_DEVICE;
  const int kern = mfa::pick_kernel(p, dev);
  if (kern < 0) return -kern;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  mfa::FwdArgs a = mfa::resolve(p);
  mfa::SplitPlan split;
  if (kern == MFA_KERNEL_TCGEN05 && p->workspace != nullptr) {
    split = mfa::plan_splits(p, mfa::dev_info(dev).sms);
    if (split.splits > 1 && p->workspace_bytes < split.bytes) split = mfa::SplitPlan{};
  }
  rc = kern == MFA_KERNEL_TCGEN05 ? mfa::run_sm100(p, a, dev, st, split, p->workspace)
                                  : mfa::run_simt(p, a, st);
  if (rc != MFA_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_fwd_noalloc(const mfa_fwd_params* p, void* stream) {
  if (p == nullptr) return MFA_ERR_INVALID;
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return rc;
  mfa_fwd_params q = *p;  // same call, with the library's own scratch as the workspace
  q.workspace = nullptr;
  q.workspace_bytes = 0;
  const size_t need = mfa_fwd_workspace_size(&q);
  if (need > 0) {
    if (need > mfa::kNoAllocScratchBytes) return MFA_ERR_SCRATCH_TOO_SMALL;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MFA_ERR_NO_DEVICE;
    void* scratch = nullptr;
    if ((rc = mfa::noalloc_scratch(dev, &scratch)) != MFA_OK) return rc;
    q.workspace = scratch;
    q.workspace_bytes = mfa::kNoAllocScratchBytes;
  }
  return mfa_fwd(&q, stream);
}

int mfa_fwd_staged(const mfa_fwd_params* p, const mfa_host_io* io, void* stream) {
  if (mfa::fault_injected("fwd")) return MFA_ERR_FAULT_INJECTED;
  mfa::NvtxRange range("mfa_fwd_staged");
  if (io == nullptr) return MFA_ERR_INVALID;
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return rc;
  return mfa::run_staged(p, io, reinterpret_cast<cudaStream_t>(stream));
}

int mfa_selftest_wait_timeout(int32_t* err, uint32_t timeout_us, void* stream) {
  if (err == nullptr || timeout_us == 0 || timeout_us > 10000000u) return MFA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  mfa::wait_timeout_selftest<<<1, 32, 0, st>>>(err, (uint64_t)timeout_us * 1000ull);
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_lse_combine(const float* const* o_part, const float* const* lse_part, int32_t n,
                    int32_t rows, int32_t H, int32_t D, void* o, int32_t o_dtype, float* lse,
                    void* stream) {
  if (mfa::fault_injected("combine")) return MFA_ERR_FAULT_INJECTED;
  if (n < 1 || n > mfa::kMaxParts || rows < 0 || H < 1 || D < 1 || o_dtype < 0 || o_dtype > 2)
    return MFA_ERR_INVALID;
  if (rows == 0) return MFA_OK;
  if (o_part == nullptr || lse_part == nullptr || o == nullptr) return MFA_ERR_INVALID;
  mfa::PartPtrs pp;
  std::memset(&pp, 0, sizeof(pp));
  for (int g = 0; g < n; ++g) {
    if (o_part[g] == nullptr || lse_part[g] == nullptr) return MFA_ERR_INVALID;
    pp.o[g] = o_part[g];
    pp.lse[g] = lse_part[g];
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  const int64_t warps = (int64_t)rows * H;
  const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
  if (o_dtype == MFA_FP32)
    mfa::lse_combine_kernel<float><<<blocks, 256, 0, st>>>(pp, n, rows, H, D, (float*)o, lse);
  else if (o_dtype == MFA_BF16)
    mfa::lse_combine_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(pp, n, rows, H, D, (__nv_bfloat16*)o, lse);
  else
    mfa::lse_combine_kernel<__half><<<blocks, 256, 0, st>>>(pp, n, rows, H, D, (__half*)o, lse);
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_lse_rescale_sum(const float* const* o_part, const float* const* lse_part, int32_t n,
                        int32_t rows, int32_t H, int32_t D, const float* lse_ref, void* o,
                        int32_t o_dtype, void* stream) {
  if (mfa::fault_injected("combine")) return MFA_ERR_FAULT_INJECTED;
  if (n < 1 || n > mfa::kMaxParts || rows < 0 || H < 1 || D < 1 || o_dtype < 0 || o_dtype > 2)
    return MFA_ERR_INVALID;
  if (rows == 0) return MFA_OK;
  if (o_part == nullptr || lse_part == nullptr || o == nullptr || lse_ref == nullptr)
    return MFA_ERR_INVALID;
  mfa::PartPtrs pp;
  std::memset(&pp, 0, sizeof(pp));
  bool vec4 = D % 4 == 0 && mfa::aligned16(o);
  for (int g = 0; g < n; ++g) {
    if (o_part[g] == nullptr || lse_part[g] == nullptr) return MFA_ERR_INVALID;
    pp.o[g] = o_part[g];
    pp.lse[g] = lse_part[g];
    vec4 = vec4 && mfa::aligned16(o_part[g]);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  const int64_t warps = (int64_t)rows * H;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks >= (1ll << 31)) return MFA_ERR_UNSUPPORTED;
  const unsigned nb = (unsigned)blocks;
  const int v4 = vec4 ? 1 : 0;
  if (o_dtype == MFA_FP32)
    mfa::lse_rescale_sum_kernel<float><<<nb, 256, 0, st>>>(pp, n, rows, H, D, lse_ref, (float*)o, v4);
  else if (o_dtype == MFA_BF16)
    mfa::lse_rescale_sum_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(pp, n, rows, H, D, lse_ref,
                                                                  (__nv_bfloat16*)o, v4);
  else
    mfa::lse_rescale_sum_kernel<__half><<<nb, 256, 0, st>>>(pp, n, rows, H, D, lse_ref, (__half*)o, v4);
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_fwd_scatter(const mfa_fwd_params* p, const mfa_peer_scatter* sc, void* stream) {
  if (mfa::fault_injected("fwd")) return MFA_ERR_FAULT_INJECTED;
  mfa::NvtxRange range("mfa_fwd_scatter");
  if (sc == nullptr) return MFA_ERR_INVALID;
  int rc = mfa::validate(p);
  if (rc != MFA_OK) return rc;
  if (p->cu_q != nullptr) return MFA_ERR_UNSUPPORTED;  // dense launches only
  if (sc->n_peers < 1 || sc->n_peers > mfa::kMaxPeers || sc->rows_per_peer < 1 || sc->slot < 0)
    return MFA_ERR_INVALID;
  if ((int64_t)p->Lq > (int64_t)sc->n_peers * sc->rows_per_peer) return MFA_ERR_INVALID;
  for (int g = 0; g < sc->n_peers; ++g) {
    if (sc->o_recv[g] == nullptr || sc->lse_recv[g] == nullptr) return MFA_ERR_INVALID;
    if (!mfa::aligned16(sc->o_recv[g])) return MFA_ERR_INVALID;
  }
  if (p->B == 0 || p->Lq == 0) return MFA_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MFA_ERR_NO_DEVICE;
  if (mfa::pick_kernel(p, dev) != MFA_KERNEL_TCGEN05) return MFA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  mfa::FwdArgs a = mfa::resolve(p);
  const int64_t rows = sc->rows_per_peer;
  a.o = sc->o_recv[0];
  a.o_dtype = MFA_FP32;
  a.o_sb = (int64_t)p->Hq * p->D;
  a.o_ss = (int64_t)p->B * p->Hq * p->D;
  a.o_sh = p->D;
  a.o_vec16 = 1;  // D % 8 == 0 (tcgen05) and 256-byte aligned receive buffers
  a.lse = sc->lse_recv[0];
  a.lse_sb = (int64_t)p->Hq * rows;
  a.lse_sh = rows;
  a.peer_n = sc->n_peers;
  a.peer_rows = sc->rows_per_peer;
  a.peer_slot = sc->slot;
  a.peer_slot_o = rows * p->B * p->Hq * p->D;
  a.peer_slot_lse = rows * p->B * p->Hq;
  for (int g = 0; g < sc->n_peers; ++g) {
    a.peer_o[g] = sc->o_recv[g];
    a.peer_lse[g] = sc->lse_recv[g];
  }
  rc = mfa::run_sm100(p, a, dev, st, mfa::SplitPlan{}, nullptr);
  if (rc != MFA_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_lse_merge(const float* o_parts, const float* lse_parts, int32_t n, int32_t rows,
                  int32_t H, int32_t D, void* o, int32_t o_dtype, float* lse, void* stream) {
  if (mfa::fault_injected("combine")) return MFA_ERR_FAULT_INJECTED;
  mfa::NvtxRange range("mfa_lse_merge");
  if (n < 1 || rows < 0 || H < 1 || D < 1 || o_dtype < 0 || o_dtype > 2) return MFA_ERR_INVALID;
  if (rows == 0) return MFA_OK;
  if (o_parts == nullptr || lse_parts == nullptr || o == nullptr) return MFA_ERR_INVALID;
  const int64_t part_stride = (int64_t)rows * H * D, lse_stride = (int64_t)rows * H;
  const int v4 = (D % 4 == 0 && mfa::aligned16(o_parts) && mfa::aligned16(o)) ? 1 : 0;
  const int64_t blocks = ((int64_t)rows * H * 32 + 255) / 256;
  if (blocks >= (1ll << 31)) return MFA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  const unsigned nb = (unsigned)blocks;
  if (o_dtype == MFA_FP32)
    mfa::lse_merge_kernel<float><<<nb, 256, 0, st>>>(o_parts, lse_parts, n, rows, H, D,
                                                      part_stride, lse_stride, (float*)o, lse, v4);
  else if (o_dtype == MFA_BF16)
    mfa::lse_merge_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(
        o_parts, lse_parts, n, rows, H, D, part_stride, lse_stride, (__nv_bfloat16*)o, lse, v4);
  else
    mfa::lse_merge_kernel<__half><<<nb, 256, 0, st>>>(o_parts, lse_parts, n, rows, H, D,
                                                       part_stride, lse_stride, (__half*)o, lse, v4);
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes == 0) return MFA_ERR_INVALID;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MFA_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return MFA_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return MFA_OK;
}

int mfa_peer_open(const void* ipc_handle, void** ptr) {
  if (ptr == nullptr || ipc_handle == nullptr) return MFA_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? MFA_OK
             : MFA_ERR_CUDA;
}

int mfa_peer_close(void* ptr) {
  if (ptr == nullptr) return MFA_ERR_INVALID;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_peer_free(void* ptr) {
  if (ptr == nullptr) return MFA_ERR_INVALID;
  return cudaFree(ptr) == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

int mfa_lse_merge_rows(const float* const* o_parts, const float* const* lse_parts, int32_t n,
                       int32_t rows_total, int32_t row0, int32_t nrows, int32_t H, int32_t D,
                       void* o, int32_t o_dtype, float* lse, void* stream) {
  if (mfa::fault_injected("combine")) return MFA_ERR_FAULT_INJECTED;
  mfa::NvtxRange range("mfa_lse_merge_rows");
  if (n < 1 || n > mfa::kMaxParts || rows_total < 0 || row0 < 0 || nrows < 0 ||
      (int64_t)row0 + nrows > rows_total || H < 1 || D < 1 || o_dtype < 0 || o_dtype > 2)
    return MFA_ERR_INVALID;
  if (nrows == 0) return MFA_OK;
  if (o_parts == nullptr || lse_parts == nullptr || o == nullptr) return MFA_ERR_INVALID;
  mfa::PartPtrs pp;
  std::memset(&pp, 0, sizeof(pp));
  bool vec4 = D % 4 == 0 && mfa::aligned16(o);
  for (int g = 0; g < n; ++g) {
    if (o_parts[g] == nullptr || lse_parts[g] == nullptr) return MFA_ERR_INVALID;
    pp.o[g] = o_parts[g];
    pp.lse[g] = lse_parts[g];
    vec4 = vec4 && mfa::aligned16(o_parts[g]);
  }
  const int64_t blocks = ((int64_t)nrows * H * 32 + 255) / 256;
  if (blocks >= (1ll << 31)) return MFA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  const unsigned nb = (unsigned)blocks;
  const int v4 = vec4 ? 1 : 0;
  if (o_dtype == MFA_FP32)
    mfa::lse_merge_rows_kernel<float><<<nb, 256, 0, st>>>(pp, n, rows_total, row0, nrows, H, D,
                                                           (float*)o, lse, v4);
  else if (o_dtype == MFA_BF16)
    mfa::lse_merge_rows_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(
        pp, n, rows_total, row0, nrows, H, D, (__nv_bfloat16*)o, lse, v4);
  else
    mfa::lse_merge_rows_kernel<__half><<<nb, 256, 0, st>>>(pp, n, rows_total, row0, nrows, H, D,
                                                            (__half*)o, lse, v4);
  return cudaGetLastError() == cudaSuccess ? MFA_OK : MFA_ERR_CUDA;
}

}  // extern "C"
