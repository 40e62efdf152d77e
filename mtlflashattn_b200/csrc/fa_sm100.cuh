// Flash-attention forward for B200 (sm_100a): TMA -> mbarrier ring -> tcgen05.mma with TMEM
// accumulators -> fp32 online softmax in registers -> P -> P.V on tcgen05.
//
// One CTA owns 256 query rows of one (batch, head) as two 128-row tiles (t = 0, 1) and streams
// the key/value blocks (128 keys each) that any of those rows may attend. For D = 64 with one
// column group (no softcap) a CTA owns one 128-row tile (TILES = 1) and two CTAs share each
// SM: their MMA warps issue independently, so the two tiles' softmax phases do not run in
// lock-step (+1.4% on B=1 H=16 L=8192 causal, +2.7% with 1 of 8 exponential pairs on the FMA
// pipe).
//
//   warpgroups 0 .. TILES*CG-1   softmax: tile t = wg / CG, key columns [cg*128/CG,
//                                (cg+1)*128/CG) with cg = wg % CG (TMEM lanes 0-127, one
//                                query row per thread)
//   warp W = 4*CG*TILES          TMA producer: Q tiles once, then K_j, V_j into a ring of NSLOT
//   warp W+1                     TMEM allocator + single-thread tcgen05.mma issuer
//   warps W+2, W+3               idle (they complete the last warpgroup)
// With CG = 2 each row's 128 scores are split over two threads in two warpgroups that exchange
// their partial row maxima (and, at the end, row sums) through shared memory behind a named
// barrier: twice the softmax warps per SM sub-partition to hide the TMEM / MUFU latencies.
// Registers: the softmax warpgroups raise theirs and the producer/MMA warpgroup lowers its
// with setmaxnreg (Roles<CG, TILES> below), so each softmax thread keeps its share of a row of
// S in registers without spilling.
//
// TMEM columns (512 allocated with two tiles, 256 with one): S_t at [128t, 128t+128), O_t
// after all S tiles, and at D = 64 P_t in its own 64 columns after all O tiles (Cfg below).
// At D = 128, P_t (16-bit, two per column) overwrites the first 64 columns of S_t once S_t is in
// registers.
// The MMA warp issues, per key block j:  PV0_j, S0_{j+1}, PV1_j, S1_{j+1}.  tcgen05 MMAs of
// one thread execute in issue order, so S_t(j+1) never overwrites P_t(j) before PV_t(j) read it,
// and the commit that publishes S_t(j+1) also covers PV_t(j); that is what lets the softmax
// warps rescale O_t in place right after they see S_t(j+1). With CG = 1 the softmax publishes P_t in
// two key halves on separate mbarriers and the MMA warp issues the first four P.V MMAs while
// the second half is still being computed (measured +5% on the plain path; quarters: +1-3%).
// (At D = 128, a variant that released S_t to the MMA as soon as it was in registers, with P
// in shared memory and an event-driven issuer, measured 5-20% slower on every BASELINE
// configuration.)
//
// Semantics follow the reference's chunked-fp32 tier (metal_flash_attn/_kernel.py:1165-1208):
// scale, softcap, ALiBi, bottom-right causal and sliding window, fully masked rows -> 0.
// The online softmax keeps a stale row maximum until it grows by more than 2^8 (log2 domain),
// so O is rescaled rarely; the final 1/l uses the same maximum as O, so the result is exact.
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace mfa {

// Exact CTA list of a varlen launch whose sequence lengths the host knows (n > 0): sequences in
// the order seq[0..n), longest first; sequence seq[i] owns CTAs [off[i], off[i+1]) of the grid,
// its row blocks x heads x splits and nothing else, so no CTA lands past a sequence's last row.
constexpr int kMaxTileSeqs = 256;
struct TileList {
  int n;
  int seq[kMaxTileSeqs];
  int off[kMaxTileSeqs + 1];
};

struct Sm100Args {
  CUtensorMap tq, tk, tv;  // 4-D maps (D, H, S, B), box (64, 1, 128, 1), 128B swizzle
  // head-packed query map: box (64, 2^pack_shift, 128 >> pack_shift, 1), rows head-fastest
  CUtensorMap tqp;
  FwdArgs a;
  TileList tl;
};

namespace sm100 {

constexpr int BM = 128;  // query rows per tile (TMEM lanes)
constexpr int BN = 128;  // keys per block

// Thread roles and register budget for CG column groups per tile and TILES 128-row tiles per
// CTA. TILES = 1 CTAs are sized so that two of them share an SM (half the TMEM columns, half
// the registers, under half the shared memory).
template <int CG, int TILES = 2>
struct Roles {
  static_assert(TILES == 2 || CG <= 2, "one-tile CTAs use one or two column groups");
  static constexpr int kSoftWarps = 4 * CG * TILES;
  static constexpr int kProducer = kSoftWarps;
  static constexpr int kMma = kSoftWarps + 1;
  static constexpr int kThreads = 128 * (TILES * CG + 1);
  static constexpr int kCtasPerSm = TILES == 1 ? 2 : 1;
  // registers per thread at launch: the register file (65536) over the threads of the CTAs
  // that share an SM, rounded down to a multiple of 8
  static constexpr int kLaunchRegs = (65536 / (kThreads * kCtasPerSm)) / 8 * 8;
  static constexpr int kSoftmaxRegs = TILES == 1 ? (CG == 1 ? 184 : 96) : CG == 1 ? 208 : 104;
  static constexpr int kOtherRegs = TILES == 1 ? (CG == 1 ? 72 : 48) : CG == 1 ? 88 : 64;
  static constexpr int NC = 128 / CG;  // score columns per softmax thread
  static_assert(TILES * CG * 128 * kSoftmaxRegs + 128 * kOtherRegs <= kThreads * kLaunchRegs,
                "setmaxnreg split exceeds the launch register budget");
};

// KBN keys per K/V block (128; 64 for the MFA_BN64_D128 variant of the D = 128 plain kernel).
template <int DP, int TILES = 2, int KBN = 128>
struct Cfg {
  static constexpr int NCH = DP / 64;                    // 128-byte column chunks per row
  static constexpr uint32_t CHUNK = 128u * 128u;         // one Q chunk of 128 rows: 16 KB
  static constexpr uint32_t TILE = NCH * CHUNK;          // Q tile
  static constexpr uint32_t KCHUNK = (uint32_t)KBN * 128u;  // one K / V chunk of KBN rows
  static constexpr uint32_t KTILE = NCH * KCHUNK;        // K / V block
  static constexpr int NSLOT = KBN == 64 ? 8
                               : DP == 128 ? (TILES == 1 ? 2 : 3) : TILES == 1 ? 5 : 6;  // ring
  static constexpr uint32_t BAR_OFF = TILES * TILE + NSLOT * KTILE;
  static constexpr uint32_t XCH_OFF = BAR_OFF + 256;     // [parity][tile][cg][row] fp32 (CG = 2)
  // TMEM columns: S_t at KBN t, O_t at TMEM_O + DP t, and (decoupled) P_t at TMEM_P + KBN/2 t.
  // D = 64 (and D = 128 with 64-key blocks) leaves room for P in its own columns and S is
  // released to the MMA as soon as it is in registers (see "decoupled" below). Otherwise P
  // aliases S.
  static constexpr bool DECOUPLED = DP == 64 || KBN == 64;
  static constexpr uint32_t TMEM_S = (uint32_t)KBN;      // columns of one tile's S
  static constexpr uint32_t TMEM_O = (uint32_t)KBN * TILES;
  static constexpr uint32_t TMEM_P = (uint32_t)KBN * TILES + (uint32_t)DP * TILES;
  static constexpr uint32_t TMEM_COLS = TILES == 1 ? 256 : 512;
  static_assert(!DECOUPLED || TMEM_P + (uint32_t)(KBN / 2) * TILES <= TMEM_COLS, "TMEM plan");
  static constexpr uint32_t SMEM = XCH_OFF + 4096 + 1024;  // + alignment slack
};

// Keys per K/V block of an instantiation (host and device agree through this).
#ifndef MFA_BN64_D128
#define MFA_BN64_D128 0
#endif
template <int DP, int kBias, int CG, int TILES, bool kPack>
struct BlockKeys {
  static constexpr int value =
      (MFA_BN64_D128 && DP == 128 && kBias == 0 && CG == 1 && TILES == 2 && !kPack) ? 64 : 128;
};

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version field.
// K-major tiles (Q, K): SBO = 1024 B between 8-row groups; LBO unused (1).
// MN-major tile (V as the B operand of P.V): LBO = 16 KB between 64-column chunks,
// SBO = 1024 B between 8-key groups.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor for kind::f16: fp32 accumulator, A/B fp16 (0) or bf16 (1).
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace sm100

// kEmu: of every 8 pairs of probabilities, how many are computed with exp2_poly2 on the FMA
// pipe instead of MUFU.EX2 (balances the two pipes). Used by one-tile D = 64 CTAs only; at
// D = 128 and in two-tile CTAs it measured no gain.
#ifndef MFA_EMU64
#define MFA_EMU64 1
#endif
#ifndef MFA_EMU128
#define MFA_EMU128 0
#endif
// The same for the softcap kernel (kBias = 2), which is MUFU-bound: two MUFU operations per
// score (tanh and the softmax ex2). Measured on B200, config 3 (fp16 D = 128, softcap 30,
// window 1024/1024), TFLOP/s: ex2+rcp tanh 365 (kEmu 0), 368 (2), 362 (4); hardware tanh
// 424 (0), 442 (2), 429 (4).
// kHalfExp: of every 8 pairs of probabilities of the plain kernel (kBias = 0), how many are
// computed by one packed 16-bit MUFU ex2 (ex2_x2: two results per operation, P in its final
// 16-bit type with no conversion) instead of two fp32 ones. Halves the MUFU time of those
// pairs; the argument is rounded to 16 bits first.
#ifndef MFA_HALF_EXP64
#define MFA_HALF_EXP64 0
#endif
#ifndef MFA_HALF_EXP128
#define MFA_HALF_EXP128 0
#endif
#ifndef MFA_EMU_SOFTCAP
#define MFA_EMU_SOFTCAP 2
#endif
// Softcap tanh: 1 = the hardware tanh.approx.f32 (one MUFU operation; its error, ~2^-11
// relative, moves a logit by at most cap * 2^-11, and config 3's output error against the fp32
// oracle stayed at 1.4e-4); 0 = 1 - 2 / (2^(2 y log2e) + 1) with MUFU ex2 and a reciprocal
// (MUFU or Newton, MFA_RCP_EMU), two MUFU operations.
#ifndef MFA_SOFTCAP_TANH
#define MFA_SOFTCAP_TANH 1
#endif
// Score transform, a template parameter of the kernel:
//   kBias = 0  x = s                        (c = scale*log2e folded into the exponent)
//   kBias = 1  x = log2e*(s*scale - slope*|centre - key|)   (any scale, ALiBi optional)
//   kBias = 2  x = log2e*(softcap(s*scale) - slope*|centre - key|)
// Column groups per tile; see the role table above. Measured on B200: the plain path loses 9-17%
// with CG = 2. The softcap path gained from CG = 2 while its tanh took two MUFU operations;
// with the hardware tanh, CG = 1 in one-tile CTAs (two per SM) is faster on config 3 (fp16
// D = 128, softcap 30, window 1024/1024): 447 TFLOP/s (CG 2, two tiles) -> 455 (CG 1, two
// tiles) -> 504 (CG 1, one tile; two CTAs per SM issue their MMAs independently and the row
// max needs no exchange between threads). The ALiBi path (kBias = 1) uses CG = 1 since its
// bias became two packed FMAs per pair of scores on all but the diagonal blocks (+43% on varlen
// GQA ALiBi, +55% on dense causal D = 128 ALiBi over CG = 2 with the general bias). Separate
// kBias = 1 / 2 kernels (rather than one kernel testing softcap at run time) cut the CG = 2
// register spills and gained 11-13% on the softcap and ALiBi configurations.
#ifndef MFA_CG_PLAIN
#define MFA_CG_PLAIN 1
#endif
#ifndef MFA_CG_SOFTCAP
#define MFA_CG_SOFTCAP 1
#endif
#ifndef MFA_CG_LINEAR
#define MFA_CG_LINEAR 1
#endif
// ALiBi kernel: bias as two packed FMAs on key blocks that lie on one side of the rows' centres.
#ifndef MFA_PACK_GQA
#define MFA_PACK_GQA 1  // pack the query heads of a KV group into tile rows on decode shapes
#endif
#ifndef MFA_ALIBI_LINEAR
#define MFA_ALIBI_LINEAR 1
#endif
// Softcap: of every 8 pairs of scores, how many take the reciprocal on the FMA pipe (Newton)
// instead of MUFU.RCP; 2 balances the pipes best on B200 (+1.5% on config 3, 8: -5%).
#ifndef MFA_RCP_EMU
#define MFA_RCP_EMU 2
#endif
#ifndef MFA_PPARTS
#define MFA_PPARTS 2
#endif
// D = 64 (P in its own TMEM columns): 1 = compute all exponentials of a block before waiting for
// the previous block's P.V (which only the P stores need), 0 = wait first.
#ifndef MFA_LATE_PV_WAIT
#define MFA_LATE_PV_WAIT 0
#endif
#ifndef MFA_CG_PLAIN64
#define MFA_CG_PLAIN64 MFA_CG_PLAIN
#endif
template <int kBias, int DP = 128>
struct DefaultCG {
  static constexpr int value = kBias == 2   ? MFA_CG_SOFTCAP
                               : kBias == 1 ? MFA_CG_LINEAR
                               : DP == 64   ? MFA_CG_PLAIN64
                                            : MFA_CG_PLAIN;
};
// Tiles per CTA: two 128-row tiles share each K/V block in one CTA, except (MFA_TILES64 = 1)
// D = 64 with one column group, where one-tile CTAs run two per SM. MFA_TILES128 = 1 does the
// same at D = 128 (measured slower: every K/V block is fetched by two CTAs).
#ifndef MFA_TILES64
#define MFA_TILES64 1
#endif
#ifndef MFA_TILES128
#define MFA_TILES128 2
#endif
// ... and the softcap kernel at D = 128 (one-tile CTAs: +11% on config 3, above).
#ifndef MFA_TILES128_SOFTCAP
#define MFA_TILES128_SOFTCAP 1
#endif
// Two column groups in one-tile D = 64 CTAs (four softmax warps per SM sub-partition) when
// MFA_TILES64_CG2 = 1.
#ifndef MFA_TILES64_CG2
#define MFA_TILES64_CG2 2
#endif
template <int DP, int CG, int kBias = 0>
struct DefaultTiles {
  static constexpr int value = CG != 1 ? (DP == 64 ? MFA_TILES64_CG2 : 2)
                               : DP == 64 ? MFA_TILES64
                               : kBias == 2 ? MFA_TILES128_SOFTCAP : MFA_TILES128;
};
template <bool B>
struct BoolC {
  static constexpr bool value = B;
};
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// kPack: the row mapping of decode-like launches (query heads packed per KV head, one-tile CTAs);
// the other instantiations fold pack_shift to 0 at compile time.
template <int DP, bool kBF16, int kBias, int CG = DefaultCG<kBias, DP>::value,
          int TILES = DefaultTiles<DP, CG, kBias>::value, bool kPack = false,
          int kEmu = (kBias == 2 ? MFA_EMU_SOFTCAP
                                 : DP == 64 ? (TILES == 1 ? MFA_EMU64 : 0) : MFA_EMU128),
          int kHalfExp = (kBias == 0 ? (DP == 64 ? MFA_HALF_EXP64 : MFA_HALF_EXP128) : 0)>
__global__ void __launch_bounds__(sm100::Roles<CG, TILES>::kThreads,
                                  sm100::Roles<CG, TILES>::kCtasPerSm)
    fa_fwd_sm100(const __grid_constant__ Sm100Args args) {
  using namespace sm100;
  constexpr int KBN = BlockKeys<DP, kBias, CG, TILES, kPack>::value;
  using C = Cfg<DP, TILES, KBN>;
  using R = Roles<CG, TILES>;
  constexpr int kSoftmaxRegs = R::kSoftmaxRegs;
  constexpr int kOtherRegs = R::kOtherRegs;
  constexpr int NC = KBN / CG;  // score columns per softmax thread
  // P_t is published to the MMA in this many key parts (one part with CG = 2, where both
  // column groups' halves are needed before the P.V MMAs of a part could start anyway).
  constexpr int kPParts = CG == 1 ? MFA_PPARTS : 1;
  const FwdArgs& a = args.a;
  constexpr bool kGeneral = kBias != 0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sb = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = sb;
  uint8_t* sKV = sb + TILES * C::TILE;  // K / V ring: NSLOT blocks of C::KTILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + C::BAR_OFF);
  uint64_t* q_full = bars;                 // [2]
  uint64_t* kv_full = bars + 2;            // [NSLOT]
  uint64_t* kv_empty = kv_full + C::NSLOT; // [NSLOT]
  uint64_t* s_full = kv_empty + C::NSLOT;  // [2]
  uint64_t* p_full = s_full + 2;           // [2][kPParts]: tile, key part
  uint64_t* o_full = p_full + 2 * kPParts; // [2]
  uint64_t* s_free = o_full + 2;           // [2] decoupled only
  uint64_t* pv_done = s_free + 2;          // [2] decoupled only
  uint64_t* mma_done = pv_done + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(sb + C::XCH_OFF);

  // ---- work decode: heaviest row blocks first across all (batch, head)
  // (groups of (batch, head) pairs whose K/V fits in L2, one after the other)
  const int idx = blockIdx.x;
  // head-packed: one CTA per (batch, KV head); tile row r is position r >> ps of query head
  // (hk << ps) + (r & pmask). Unpacked (ps = 0): one CTA per (batch, query head), r = position.
  const int ps = kPack ? a.pack_shift : 0;
  const int pmask = (1 << ps) - 1;
  const int heads = a.Hq >> ps;
  int rb, split, hu, b;
  if (args.tl.n > 0) {
    // exact varlen list: find the sequence, then within it groups of group_hb heads (L2), each
    // group's row blocks heaviest first, the splits of a row block side by side
    int lo = 0, hi = args.tl.n - 1;
    while (lo < hi) {  // the last i with off[i] <= idx
      const int mid = (lo + hi + 1) >> 1;
      if (args.tl.off[mid] <= idx) lo = mid; else hi = mid - 1;
    }
    b = args.tl.seq[lo];
    const int ri0 = idx - args.tl.off[lo];
    const int nrb = (args.tl.off[lo + 1] - args.tl.off[lo]) / (heads * a.num_splits);
    const int gh = min(a.group_hb, heads);
    const int per_full = nrb * gh * a.num_splits;
    const int g = ri0 / per_full;
    const int gsz = min(gh, heads - g * gh) * a.num_splits;  // CTAs per row block in group g
    const int ri = ri0 - g * per_full;
    rb = nrb - 1 - ri / gsz;
    split = (ri % gsz) % a.num_splits;
    hu = g * gh + (ri % gsz) / a.num_splits;
  } else {
    const int per_group = a.num_row_blocks * a.group_hb * a.num_splits;
    const int grp = idx / per_group;
    const int hb0 = grp * a.group_hb;
    const int GHS = min(a.group_hb, heads * a.B - hb0) * a.num_splits;  // CTAs per row block
    const int ri = idx - grp * per_group;
    rb = a.num_row_blocks - 1 - ri / GHS;
    split = (ri % GHS) % a.num_splits;  // splits of one row block run side by side
    const int hb = hb0 + (ri % GHS) / a.num_splits;
    hu = hb % heads;  // query head, or KV head when packed
    b = hb / heads;
  }
  const int hk = ps ? hu : hu / a.group;
  const SeqView sv = seq_view(a, b);
  const int rows = sv.lq << ps;  // tile rows of this (batch, head unit)
  const int r0 = rb * TILES * BM;
  // a split launch is followed by its merge, launched as a programmatic dependent: let it be
  // scheduled now (it waits for this grid's completion before reading anything)
  if (a.num_splits > 1) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (r0 >= rows) return;  // whole CTA leaves before touching barriers or TMEM
  // tiles holding at least one row (a last row block may leave the second tile empty)
  const int nt = (TILES == 2 && r0 + BM < rows) ? 2 : 1;

  const int r_last = min(r0 + TILES * BM, rows) - 1;
  // union of the rows' key intervals: lo and hi are nondecreasing in the position
  int klo = key_range(a, sv, r0 >> ps).lo;
  int khi = key_range(a, sv, r_last >> ps).hi;
  if (a.num_splits > 1) {
    klo = max(klo, split * a.split_keys);
    if (split + 1 < a.num_splits) khi = min(khi, (split + 1) * a.split_keys);
  }
  const int jb = klo / KBN;
  const int n = khi > klo ? (khi + KBN - 1) / KBN - jb : 0;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&q_full[0], 1);
    mbar_init(&q_full[1], 1);
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      for (int q = 0; q < kPParts; ++q) mbar_init(&p_full[kPParts * t + q], 4 * CG);
      mbar_init(&o_full[t], 1);
      mbar_init(&s_free[t], 4 * CG);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == R::kMma) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == R::kProducer && lane == 0) {
    tma_prefetch_map(ps ? &args.tqp : &args.tq);
    tma_prefetch_map(&args.tk);
    tma_prefetch_map(&args.tv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= R::kMma + 1) {
    regs_dec<kOtherRegs>();  // idle warps of the producer/MMA warpgroup
  } else if (warp == R::kProducer) {
    regs_dec<kOtherRegs>();
    // ------------------------------------------------------------ TMA producer
    if (n > 0) {
      if (lane == 0) {
        for (int t = 0; t < nt; ++t) {
          const int qpos = sv.q0 + ((r0 + t * BM) >> ps);
          if constexpr (MFA_CHECKS) {
            const int h_hi = ps ? ((hk + 1) << ps) : hu + 1;  // one past the last head loaded
            if (qpos < 0 || qpos >= (a.cu_q != nullptr ? a.Lq : sv.lq) || h_hi > a.Hq ||
                (a.cu_q == nullptr && sv.qb >= a.B)) {
              if (a.err != nullptr) atomicExch(a.err, kErrCheck);
              *abort_flag = 1;
              break;
            }
          }
          mbar_expect_tx(&q_full[t], C::TILE);
          for (int c = 0; c < C::NCH; ++c) {
            if (ps)
              tma_load_4d(sQ + t * C::TILE + c * C::CHUNK, &args.tqp, &q_full[t], 64 * c, hk << ps,
                          qpos, sv.qb);
            else
              tma_load_4d(sQ + t * C::TILE + c * C::CHUNK, &args.tq, &q_full[t], 64 * c, hu, qpos,
                          sv.qb);
          }
        }
      }
      for (int it = 0; it < 2 * n; ++it) {
        const int slot = it % C::NSLOT;
        const uint32_t ph = (uint32_t)(it / C::NSLOT) & 1u;
        bool ok = mbar_wait(&kv_empty[slot], ph ^ 1u, abort_flag);
        if (!__all_sync(kFull, ok)) break;
        if (lane == 0) {
          const int j = jb + (it >> 1);
          const CUtensorMap* m = (it & 1) ? &args.tv : &args.tk;
          if constexpr (MFA_CHECKS) {
            const int krow = sv.k0 + j * KBN;
            if (j < 0 || j * KBN >= sv.lk || krow < 0 || krow >= a.Lk || hk < 0 || hk >= a.Hkv ||
                (a.cu_q == nullptr && sv.kb >= a.B)) {
              if (a.err != nullptr) atomicExch(a.err, kErrCheck);
              *abort_flag = 1;
            }
          }
          if (!(MFA_CHECKS && *abort_flag)) {
            mbar_expect_tx(&kv_full[slot], C::KTILE);
            for (int c = 0; c < C::NCH; ++c)
              tma_load_4d(sKV + slot * C::KTILE + c * C::KCHUNK, m, &kv_full[slot], 64 * c, hk,
                          sv.k0 + j * KBN, sv.kb);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == R::kMma) {
    // ------------------------------------------------------------ MMA issuer (one thread)
    regs_dec<kOtherRegs>();
    if (n > 0 && lane == 0) {
      constexpr uint32_t kIdQK = idesc_f16(kBF16, BM, KBN, false);
      constexpr uint32_t kIdPV = idesc_f16(kBF16, BM, DP, true);
      const uint32_t sQa = smem_u32(sQ);
      const uint32_t sKVa = smem_u32(sKV);
      // Descriptors are built once; each MMA only adds a compile-time offset to the 14-bit
      // start-address field (shared-memory addresses < 256 KB never carry out of it). Building
      // them per MMA made the single issuing thread, not the tensor pipe, the bottleneck.
      const uint64_t dQ = desc_sw128(sQa, 16, 1024);
      const uint64_t dK = desc_sw128(sKVa, 16, 1024);
      const uint64_t dV = desc_sw128(sKVa, C::KCHUNK, 1024);
      auto qk = [&](int t, int it) {  // S_t = Q_t K^T, K in ring item `it`
        const uint64_t a0 = dQ + ((t * C::TILE) >> 4);
        const uint64_t b0 = dK + (((it % C::NSLOT) * C::KTILE) >> 4);
        const uint32_t d = tmem + C::TMEM_S * t;
#pragma unroll
        for (int k = 0; k < DP / 16; ++k) {
          const uint32_t koff_a = ((k >> 2) * C::CHUNK + (k & 3) * 32) >> 4;
          const uint32_t koff_b = ((k >> 2) * C::KCHUNK + (k & 3) * 32) >> 4;
          mma_ss(d, a0 + koff_a, b0 + koff_b, kIdQK, k > 0);
        }
      };
      // O_t (+)= P_t V, V in ring item `it`. P_t arrives in kPParts key parts; the MMAs of a
      // part run while the softmax is still producing the next one.
      auto pv = [&](int t, int it, bool acc, int j) {
        const uint64_t b0 = dV + (((it % C::NSLOT) * C::KTILE) >> 4);
        const uint32_t d = tmem + C::TMEM_O + DP * t;
        const uint32_t pa = tmem + (C::DECOUPLED ? C::TMEM_P + (KBN / 2) * t : C::TMEM_S * t);
#pragma unroll
        for (int q = 0; q < kPParts; ++q) {
          if (!mbar_wait(&p_full[kPParts * t + q], (uint32_t)j & 1u, abort_flag)) return false;
          tc_fence_after();
#pragma unroll
          for (int k = q * (KBN / 16 / kPParts); k < (q + 1) * (KBN / 16 / kPParts); ++k)
            mma_ts(d, pa + k * 8, b0 + ((k * 2048) >> 4), kIdPV, (acc || k > 0) ? 1u : 0u);
        }
        return true;
      };
      auto ring_wait = [&](int it) {
        return mbar_wait(&kv_full[it % C::NSLOT], (uint32_t)(it / C::NSLOT) & 1u, abort_flag);
      };
      // The issue loop is compiled for one and for two active tiles (a last row block may
      // leave the second tile empty), so the loop itself carries no tile-count tests.
      auto issue = [&](auto two) {
        constexpr bool kTwo = decltype(two)::value;
        bool ok = mbar_wait(&q_full[0], 0, abort_flag) &&
                  (!kTwo || mbar_wait(&q_full[1], 0, abort_flag)) && ring_wait(0);
        if (ok) {
          tc_fence_after();
          qk(0, 0);
          tc_commit(&s_full[0]);
          if (kTwo) {
            qk(1, 0);
            tc_commit(&s_full[1]);
          }
          tc_commit(&kv_empty[0]);
        }
        if constexpr (C::DECOUPLED) {
          // Per block j: S0(j+1) and S1(j+1) as soon as each softmax has S_t(j) in registers,
          // then P0(j) V_j and P1(j) V_j as each P arrives; pv_done[t] tells the softmax when
          // O_t and P_t are free again.
          for (int j = 0; j < n && ok; ++j) {
            const int itV = 2 * j + 1, itK = 2 * j + 2;
            if (j + 1 < n) {
              ok = ring_wait(itK) && mbar_wait(&s_free[0], (uint32_t)j & 1u, abort_flag);
              if (!ok) break;
              tc_fence_after();
              qk(0, itK);
              tc_commit(&s_full[0]);
              if (kTwo) {
                if (!(ok = mbar_wait(&s_free[1], (uint32_t)j & 1u, abort_flag))) break;
                tc_fence_after();
                qk(1, itK);
                tc_commit(&s_full[1]);
              }
              tc_commit(&kv_empty[itK % C::NSLOT]);
            }
            ok = ring_wait(itV) && pv(0, itV, j > 0, j);
            if (!ok) break;
            tc_commit(&pv_done[0]);
            if (kTwo) {
              if (!(ok = pv(1, itV, j > 0, j))) break;
              tc_commit(&pv_done[1]);
            }
            tc_commit(&kv_empty[itV % C::NSLOT]);
          }
        } else {
        for (int j = 0; j < n && ok; ++j) {
          const int itV = 2 * j + 1, itK = 2 * j + 2;
          const bool more = j + 1 < n;
          ok = ring_wait(itV) && pv(0, itV, j > 0, j);
          if (!ok) break;
          if (!more) tc_commit(&o_full[0]);
          if (more) {
            if (!(ok = ring_wait(itK))) break;
            tc_fence_after();
            qk(0, itK);
            tc_commit(&s_full[0]);
          }
          if (kTwo) {
            if (!(ok = pv(1, itV, j > 0, j))) break;
          }
          tc_commit(&kv_empty[itV % C::NSLOT]);
          if (kTwo && !more) tc_commit(&o_full[1]);
          if (more) {
            if (kTwo) {
              qk(1, itK);
              tc_commit(&s_full[1]);
            }
            tc_commit(&kv_empty[itK % C::NSLOT]);
          }
        }
        }
      };
      if constexpr (TILES == 2) {
        if (nt == 2) issue(BoolC<true>{}); else issue(BoolC<false>{});
      } else {
        issue(BoolC<false>{});
      }
      // Drain: every MMA issued above has completed before TMEM is released.
      tc_commit(mma_done);
      if (!mbar_wait_drain(mma_done, 0)) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    regs_inc<kSoftmaxRegs>();
    const int wg = warp >> 2;
    const int t = wg / CG;          // tile
    const int cg = wg % CG;         // column group within the row
    const int col0 = cg * NC;       // first score column of this thread
    const int wq = warp & 3;        // TMEM lane quarter
    const int rt = wq * 32 + lane;  // row within tile
    const int trow = r0 + t * BM + rt;  // tile row within the (batch, head unit)
    const int64_t row = trow >> ps;     // query position within the sequence
    const int h = ps ? (hk << ps) + (trow & pmask) : hu;  // query head of this row
    const int nj = (TILES == 1 || t < nt) ? n : 0;  // key blocks this tile runs (0: empty tile)
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + C::TMEM_S * t;
    const uint32_t tO = tmem + lane_base + C::TMEM_O + t * DP;
    const KeyRange kr = key_range(a, sv, row);
    // tile-uniform interval extremes for the "block needs no mask" test
    const int tile_lo_max = key_range(a, sv, (r0 + t * BM + BM - 1) >> ps).lo;
    const int tile_hi_min = key_range(a, sv, (r0 + t * BM) >> ps).hi;
    constexpr float kLog2e = 1.4426950408889634f;
    // x (the values kept in registers) times c is the logit in log2 units
    const float c = kGeneral ? 1.f : a.scale * kLog2e;
    float slope_l2 = 0.f;  // ALiBi slope in log2 units
    if (kGeneral && a.alibi != nullptr) slope_l2 = a.alibi[(int64_t)b * a.Hq + h] * kLog2e;
    const float cap = a.softcap;
    // softcap: x = cap*log2e*tanh(y) with tanh(y) = 1 - 2/(2^(2*log2e*y) + 1), y = s*scale/cap
    const float sc_in = cap > 0.f ? a.scale * 2.f * kLog2e / cap : 0.f;
    const float sc_a = cap * kLog2e, sc_b = -2.f * cap * kLog2e;
    const float sc_tin = cap > 0.f ? a.scale / cap : 0.f;  // hardware tanh: y = s*scale/cap
    const float pl_scale = a.scale * kLog2e;  // no softcap: x = s*scale*log2e
    const float centre = (float)(row + sv.off);
    // partner exchange slots: xch[parity][t][cg][row]
    auto xslot = [&](int parity, int g) { return xch + ((parity * 2 + t) * 2 + g) * 128 + rt; };

    float m_used = -INFINITY;  // in x units
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      ok = __all_sync(kFull, mbar_wait(&s_full[t], (uint32_t)j & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[NC];
#pragma unroll
      for (int q = 0; q < NC / 32; ++q) tmem_ld32(tS + col0 + 32 * q, r + 32 * q);
      tmem_ld_wait32(r);
#pragma unroll
      for (int q = 1; q < NC / 32; ++q) tmem_ld_tie32(r + 32 * q);
      if constexpr (C::DECOUPLED) {  // S_t is in registers: the MMA may write S_t(j+1)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t]);
      }
      float x[NC];
      const int c0 = (jb + j) * KBN + col0;  // local key index of x[0]
      const bool need_mask = ((jb + j) * KBN < tile_lo_max) || ((jb + j) * KBN + KBN > tile_hi_min);
      // ALiBi on a block whose keys all lie on one side of the centre of every row of this
      // warp (every causal block but the diagonal): |centre - key| is linear in the key index,
      // so the bias is one packed FMA, slope' * i + base, and x = s * scale + bias another.
      bool linear_bias = false;
      float lb_slope = 0.f, lb_base = 0.f;
      if constexpr (kBias == 1 && MFA_ALIBI_LINEAR) {
        const float kp0 = (float)(c0 + a.k_pos_offset);  // key position of x[0]
        // smallest and largest centre among the warp's rows (positions ascend with the lane)
        const int wr0 = r0 + t * BM + wq * 32;
        const float wmin = (float)((int64_t)(wr0 >> ps) + sv.off);
        const float wmax = (float)((int64_t)((wr0 + 31) >> ps) + sv.off);
        const bool left = kp0 + (float)(NC - 1) <= wmin, right = kp0 >= wmax;
        linear_bias = left || right;
        lb_slope = left ? slope_l2 : -slope_l2;  // bias = -slope |c - k| = lb_slope (k - c)
        lb_base = lb_slope * (kp0 - centre);
      }
      if (kBias == 1 && linear_bias) {
        const uint64_t sl2 = f2pack(lb_slope, lb_slope), base2 = f2pack(lb_base, lb_base);
        const uint64_t sc2 = f2pack(pl_scale, pl_scale);
#pragma unroll
        for (int i = 0; i < NC; i += 2) {
          const uint64_t s2 = f2pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
          const uint64_t b2 = ffma2(sl2, f2pack((float)i, (float)(i + 1)), base2);
          f2unpack(ffma2(s2, sc2, b2), x[i], x[i + 1]);
        }
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < NC; ++i) {
            const int kl = c0 + i;
            if (kl < kr.lo || kl >= kr.hi) x[i] = -INFINITY;
          }
        }
      } else if constexpr (kGeneral) {
        // x = log2(e) * (softcap(s * scale) - slope * |centre - key|)
        const float d0 = centre - (float)(c0 + a.k_pos_offset);  // centre - key for i = 0
#pragma unroll
        for (int i = 0; i < NC; i += 2) {
          uint64_t s2 = f2pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
          uint64_t x2;
          if constexpr (kBias == 2 && MFA_SOFTCAP_TANH) {
            float ya, yb;
            f2unpack(fmul2(s2, f2pack(sc_tin, sc_tin)), ya, yb);
            x2 = fmul2(f2pack(tanh_hw(ya), tanh_hw(yb)), f2pack(sc_a, sc_a));
          } else if constexpr (kBias == 2) {
            float ya, yb;
            f2unpack(fmul2(s2, f2pack(sc_in, sc_in)), ya, yb);
            // no clamp needed: 2^y overflows to +inf -> rcp = 0 -> tanh = 1; 2^y -> 0 -> tanh = -1
            const uint64_t e2 = fadd2(f2pack(ex2(ya), ex2(yb)), f2pack(1.f, 1.f));
            float ea, eb;
            f2unpack(e2, ea, eb);
            uint64_t r2;
            if (((i >> 1) & 7) < MFA_RCP_EMU) {
              // reciprocal on the FMA pipe: the guess bits(1/d) ~ kRcpSeed - bits(d) (relative
              // error <= 0.051; the constant is fitted by csrc/fit_rcp_seed.py) and three Newton
              // steps r += r(1 - d r) (error < 1e-7 after fp32 rounding); d >= 1 is clamped below
              // 2^126 so the guess stays a normal number (1/d < 1.2e-38 is 0 for the logit anyway)
              constexpr int kRcpSeed = 0x7EF311C2;
              ea = fminf(ea, 8.5e37f);
              eb = fminf(eb, 8.5e37f);
              const uint64_t nd = f2pack(-ea, -eb), one = f2pack(1.f, 1.f);
              r2 = f2pack(__int_as_float(kRcpSeed - __float_as_int(ea)),
                          __int_as_float(kRcpSeed - __float_as_int(eb)));
#pragma unroll
              for (int it = 0; it < 3; ++it) r2 = ffma2(r2, ffma2(nd, r2, one), r2);
            } else {
              r2 = f2pack(rcp(ea), rcp(eb));
            }
            x2 = ffma2(r2, f2pack(sc_b, sc_b), f2pack(sc_a, sc_a));
          } else {
            x2 = fmul2(s2, f2pack(pl_scale, pl_scale));
          }
          if (slope_l2 != 0.f) {
            float da = fabsf(d0 - (float)i), db = fabsf(d0 - (float)(i + 1));
            x2 = ffma2(f2pack(da, db), f2pack(-slope_l2, -slope_l2), x2);
          }
          f2unpack(x2, x[i], x[i + 1]);
        }
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < NC; ++i) {
            const int kl = c0 + i;
            if (kl < kr.lo || kl >= kr.hi) x[i] = -INFINITY;
          }
        }
      } else {
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < NC; ++i) {
            const int kl = c0 + i;
            x[i] = (kl < kr.lo || kl >= kr.hi) ? -INFINITY : __uint_as_float(r[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < NC; ++i) x[i] = __uint_as_float(r[i]);
        }
      }
      float mx0 = fmax3(x[0], x[1], x[2]), mx1 = fmax3(x[3], x[4], x[5]);
      float mx2 = fmax3(x[6], x[7], x[8]), mx3 = fmax3(x[9], x[10], x[11]);
#pragma unroll
      for (int i = 12; i < NC - 4; i += 8) {
        mx0 = fmax3(mx0, x[i], x[i + 1]);
        mx1 = fmax3(mx1, x[i + 2], x[i + 3]);
        mx2 = fmax3(mx2, x[i + 4], x[i + 5]);
        mx3 = fmax3(mx3, x[i + 6], x[i + 7]);
      }
      mx0 = fmax3(mx0, x[NC - 4], x[NC - 3]);
      mx1 = fmax3(mx1, x[NC - 2], x[NC - 1]);
      float mrow = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      if constexpr (CG == 2) {
        // combine with the partner thread that holds the other half of this row
        *xslot(j & 1, cg) = mrow;
        named_barrier(1 + t, 256);
        mrow = fmaxf(mrow, *xslot(j & 1, cg ^ 1));
      }
      // kLate: the exponentials of block j run before the wait for P_t(j-1) V_{j-1}, which
      // only the P stores (and a rare O rescale) need
      constexpr bool kLate = C::DECOUPLED && MFA_LATE_PV_WAIT;
      bool pv_waited = j == 0 || !C::DECOUPLED;
      if constexpr (C::DECOUPLED && !kLate) {  // O_t, P_t busy until P_t(j-1) V_{j-1} is done
        if (j > 0) {
          ok = __all_sync(kFull, mbar_wait(&pv_done[t], (uint32_t)(j - 1) & 1u, abort_flag));
          if (!ok) break;
          tc_fence_after();
          pv_waited = true;
        }
      }
      const float m_new = fmaxf(m_used, mrow);
      const bool grow = (m_new - m_used) * c > 8.f;  // false when both are -inf (NaN compare)
      if (__any_sync(kFull, grow)) {  // same rows in both halves -> same decision
        if (kLate && !pv_waited) {
          ok = __all_sync(kFull, mbar_wait(&pv_done[t], (uint32_t)(j - 1) & 1u, abort_flag));
          if (!ok) break;
          tc_fence_after();
          pv_waited = true;
        }
        const float factor = (m_used == -INFINITY) ? 0.f : ex2((m_used - m_new) * c);
        if (j > 0) {
          // O_t is idle here: decoupled, after pv_done; aliased, because the commit that
          // published S_t(j) also covered PV_t(j-1).
#pragma unroll 1
          for (int cc = cg * (DP / CG); cc < (cg + 1) * (DP / CG); cc += 32) {
            uint32_t o[32];
            tmem_ld32(tO + cc, o);
            tmem_ld_wait32(o);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const uint64_t v2 = fmul2(u2pack(o[i], o[i + 1]), f2pack(factor, factor));
              u2unpack(v2, o[i], o[i + 1]);
            }
            tmem_st32(tO + cc, o);
          }
        }
        l *= factor;
        m_used = m_new;
      }
      const float ref = (m_used == -INFINITY) ? 0.f : m_used * c;
      // p = 2^(x*c - ref): a fraction kEmu/8 of the pairs on the FMA pipe, the rest on MUFU
      const uint64_t c2 = f2pack(c, c), nref2 = f2pack(-ref, -ref);
      uint64_t acc0 = f2pack(0.f, 0.f), acc1 = acc0;
      uint32_t pk_all[kLate ? NC / 2 : 1];  // kLate: all of P_t(j) until the stores may start
      const uint32_t tP = (C::DECOUPLED ? tmem + lane_base + C::TMEM_P + t * (KBN / 2) : tS) + col0 / 2;
      auto publish = [&](int cc, const uint32_t* pk) {
        // P_t: its own columns (decoupled) or over the first 64 columns of S_t
        tmem_st16(tP + 16 * cc, pk);
        if constexpr (kPParts > 1) {
          if ((cc + 1) % (NC / 32 / kPParts) == 0 && cc + 1 < NC / 32) {  // an early part
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[kPParts * t + (cc + 1) / (NC / 32 / kPParts) - 1]);
          }
        }
      };
#pragma unroll
      for (int cc = 0; cc < NC / 32; ++cc) {  // 32 keys -> 16 packed words per step
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = 32 * cc + 2 * i;
          const uint64_t t2 = ffma2(f2pack(x[e], x[e + 1]), c2, nref2);
          if ((i & 7) >= 8 - kHalfExp) {
            // one MUFU operation for the pair; P is produced in its 16-bit type directly and
            // the row sum adds exactly the values P.V will use
            float ta, tb;
            f2unpack(t2, ta, tb);
            const uint32_t ph = ex2_x2<kBF16>(pack2<kBF16>(ta, tb));
            pk[i] = ph;
            float p0, p1;
            if constexpr (kBF16) {
              p0 = __uint_as_float(ph << 16);
              p1 = __uint_as_float(ph & 0xFFFF0000u);
            } else {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ph));
              p0 = f.x;
              p1 = f.y;
            }
            if (i & 1) acc1 = fadd2(acc1, f2pack(p0, p1)); else acc0 = fadd2(acc0, f2pack(p0, p1));
            continue;
          }
          uint64_t p2;
          if ((i & 7) < kEmu) {
            p2 = exp2_poly2(t2);
          } else {
            float ta, tb;
            f2unpack(t2, ta, tb);
            p2 = f2pack(ex2(ta), ex2(tb));
          }
          if (i & 1) acc1 = fadd2(acc1, p2); else acc0 = fadd2(acc0, p2);
          float p0, p1;
          f2unpack(p2, p0, p1);
          pk[i] = pack2<kBF16>(p0, p1);
        }
        if constexpr (kLate) {
#pragma unroll
          for (int i = 0; i < 16; ++i) pk_all[16 * cc + i] = pk[i];
        } else {
          publish(cc, pk);
        }
      }
      if constexpr (kLate) {
        if (!pv_waited) {
          ok = __all_sync(kFull, mbar_wait(&pv_done[t], (uint32_t)(j - 1) & 1u, abort_flag));
          if (!ok) break;
          tc_fence_after();
        }
#pragma unroll
        for (int cc = 0; cc < NC / 32; ++cc) publish(cc, pk_all + 16 * cc);
      }
      float la, lb;
      f2unpack(fadd2(acc0, acc1), la, lb);
      l += la + lb;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[kPParts * t + kPParts - 1]);
    }
    if (ok && nj > 0) {
      ok = __all_sync(kFull, C::DECOUPLED
                                 ? mbar_wait(&pv_done[t], (uint32_t)(nj - 1) & 1u, abort_flag)
                                 : mbar_wait(&o_full[t], 0, abort_flag));
    }
    if constexpr (CG == 2) {
      // row sum = both halves (both threads of a row agree on ok: same barrier waits)
      *xslot(nj & 1, cg) = l;
      named_barrier(1 + t, 256);
      l += *xslot(nj & 1, cg ^ 1);
    }
    if (ok) {
      tc_fence_after();
      bool store = row < sv.lq;
      // a split launch's partial rows live in a workspace sized by Lq (varlen: total_q); a
      // caller whose Lq understates cu_q[B] gets an error word instead of a write past its end
      if (store && a.num_splits > 1 && sv.q0 + row >= a.Lq) {
        store = false;
        if (a.err != nullptr) atomicExch(a.err, 1 /*MFA_ERR_INVALID*/);
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint8_t* orow = nullptr;
      // output row: this GPU's buffer, or (split-KV over GPUs) the owning GPU's receive slot
      int64_t orow_idx = sv.q0 + row;
      float* lse_base = a.lse;
      uint8_t* obase = reinterpret_cast<uint8_t*>(a.o);
      if constexpr (MFA_CHECKS) {
        const bool bad = store && (h < 0 || h >= a.Hq || orow_idx < 0 ||
                                   (a.peer_n > 0 ? orow_idx >= (int64_t)a.peer_n * a.peer_rows
                                                 : orow_idx >= (a.cu_q != nullptr ? a.Lq : sv.lq)));
        if (bad) {
          if (a.err != nullptr) atomicExch(a.err, kErrCheck);
          store = false;
        }
      }
      if (a.peer_n > 0 && store) {  // the host checked Lq <= peer_n * peer_rows
        const int owner = (int)(orow_idx / a.peer_rows);
        orow_idx -= (int64_t)owner * a.peer_rows;
        obase = reinterpret_cast<uint8_t*>(a.peer_o[owner] + a.peer_slot * a.peer_slot_o);
        lse_base = a.peer_lse[owner] + a.peer_slot * a.peer_slot_lse;
      }
      if (store) {
        const int64_t esz = a.o_dtype == 2 ? 4 : 2;
        orow = obase + esz * ((int64_t)split * a.o_split_stride + (int64_t)sv.qb * a.o_sb +
                              orow_idx * a.o_ss + (int64_t)h * a.o_sh);
      }
#pragma unroll 1
      for (int cc = cg * (DP / CG); cc < (cg + 1) * (DP / CG); cc += 32) {
        float vals[32];
        if (nj > 0) {
          uint32_t o[32];
          tmem_ld32(tO + cc, o);
          tmem_ld_wait32(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) vals[i] = __uint_as_float(o[i]) * inv;
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) vals[i] = 0.f;
        }
        const int nc = min(32, a.D - cc);
        if (store && nc > 0) store_row_chunk(a, orow, cc, vals, nc);
      }
      if (store && cg == 0 && lse_base != nullptr) {
        const float lse = l > 0.f ? (m_used * c + __log2f(l)) * 0.6931471805599453f : -INFINITY;
        lse_base[(int64_t)split * a.lse_split_stride + (int64_t)sv.qb * a.lse_sb +
                 (int64_t)h * a.lse_sh + orow_idx] = lse;
      }
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == R::kMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && a.err != nullptr) atomicExch(a.err, 4 /*MFA_ERR_TIMEOUT*/);
}

}  // namespace mfa
