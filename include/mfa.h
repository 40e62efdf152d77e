/*
 * mfa.h — C ABI of libmfa.so, the B200 (sm_100a) flash-attention forward engine.
 *
 * This library replaces the kernel-tier layer that sits under the reference's boundary
 * function `flash_attn_forward` (metal_flash_attn/_kernel.py:1052-1153). That function picks
 * one of the Metal tiers v0/v1/v2/v2r (metal_flash_attn/_kernel.py:974-985) and launches it
 * through torch.mps.compile_shader (e.g. metal_flash_attn/_kernel.py:1309-1312, 1416-1419).
 * Here the same boundary is one C call, `mfa_fwd`, with plain device pointers, element strides
 * and scalars; no torch types cross it.
 *
 * Semantics (identical to the reference's chunked-fp32 torch tier,
 * metal_flash_attn/_kernel.py:1165-1208):
 *   s  = (q . k) * scale
 *   s  = softcap * tanh(s / softcap)              if softcap > 0
 *   s -= alibi[b*Hq + h] * |center - j|           if alibi != NULL
 *   masked (-inf) unless kmin <= j < kmax, with center = i + (Lk - Lq) (bottom-right),
 *     causal: j <= center; win_left >= 0: j >= center - win_left;
 *     win_right >= 0: j <= center + win_right
 *   o  = softmax(s) @ v ; a row with no unmasked key is 0 (nan_to_num, _kernel.py:1206)
 * GQA/MQA: query head h reads kv head h / (Hq / Hkv).
 *
 * Ownership: the caller owns every buffer. Launches are asynchronous on the caller's stream.
 * No C++ exception crosses the ABI; every entry returns an mfa_status.
 * The library is reentrant and safe to call from several host threads.
 */
#ifndef MFA_H_
#define MFA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MFA_ABI_VERSION 8

/* Status codes. The Python layer maps them to the reference's exception types. */
enum mfa_status {
  MFA_OK = 0,
  MFA_ERR_INVALID = 1,        /* bad argument (ValueError in the reference) */
  MFA_ERR_UNSUPPORTED = 2,    /* feature or shape not supported (NotImplementedError) */
  MFA_ERR_CUDA = 3,           /* CUDA runtime / driver failure (RuntimeError) */
  MFA_ERR_TIMEOUT = 4,        /* a bounded in-kernel wait expired; output is invalid */
  MFA_ERR_NO_DEVICE = 5,      /* no usable sm_100 device for the requested kernel */
  MFA_ERR_FAULT_INJECTED = 6, /* host-side fault injection (MFA_FAULT env) fired */
  MFA_ERR_SCRATCH_TOO_SMALL = 7, /* mfa_fwd_noalloc: the problem needs more than its scratch */
  MFA_ERR_CHECK = 8             /* (in *err) a device-side bounds check of a build with
                                   -DMFA_CHECKS=1 failed; the access was skipped */
};

enum mfa_dtype { MFA_FP16 = 0, MFA_BF16 = 1, MFA_FP32 = 2 };

/* Kernel choice. AUTO picks TCGEN05 when eligible (fp16/bf16, D % 8 == 0, 16-byte aligned
 * strides and pointers, sm_100 device), else SIMT. */
enum mfa_kernel { MFA_KERNEL_AUTO = 0, MFA_KERNEL_TCGEN05 = 1, MFA_KERNEL_SIMT = 2 };

typedef struct mfa_fwd_params {
  const void* q;  /* [B, Lq, Hq, D] logical; any (batch, seq, head) strides, last dim stride 1 */
  const void* k;  /* [B, Lk, Hkv, D] */
  const void* v;  /* [B, Lk, Hkv, D] */
  void* o;        /* [B, Lq, Hq, D] in o_dtype */
  float* lse;     /* optional [B, Hq, Lq] natural-log sum-exp of each row (-inf if empty) */
  int64_t q_stride[3]; /* element strides: batch, seq, head */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t lse_stride[2]; /* batch, head; the row stride is 1 */
  int32_t B, Hq, Hkv, Lq, Lk, D;
  /* varlen: device int32 [B+1] cumulative lengths, or NULL for dense. With varlen the batch
   * strides are ignored, rows are absolute token indices, Lq/Lk hold the total token counts
   * (total_q, total_k) and max_lq must be >= every per-sequence query length. With a
   * workspace (or mfa_fwd_noalloc) Lq must also be >= cu_q[B]: split partial rows are addressed
   * by packed row, and a row at or past Lq is not stored but reported as MFA_ERR_INVALID in
   * *err. A launch over some of the sequences of a larger packed batch touches only the rows
   * [cu_q[0], cu_q[B]) of o and lse. */
  const int32_t* cu_q;
  const int32_t* cu_k;
  int32_t max_lq, max_lk;
  float scale;
  float softcap;       /* 0 disables */
  int32_t causal;      /* bottom-right aligned */
  int32_t win_left;    /* -1 = unbounded */
  int32_t win_right;   /* -1 = unbounded */
  const float* alibi;  /* optional device fp32 [B*Hq] slopes */
  int32_t dtype;       /* mfa_dtype of q/k/v */
  int32_t o_dtype;     /* mfa_dtype of o; -1 = same as dtype */
  /* split-KV: local key j is global key j + k_pos_offset; lk_total is the global key count
   * used for the bottom-right centre (0 = use Lk). */
  int32_t k_pos_offset;
  int32_t lk_total;
  int32_t kernel;      /* mfa_kernel */
  int32_t* err;        /* optional device int; a kernel that times out stores MFA_ERR_TIMEOUT,
                          a split launch whose varlen rows pass Lq stores MFA_ERR_INVALID */
  /* Optional caller-owned device scratch for splitting the keys of one launch over several
   * CTAs when there are too few query rows to fill the GPU (decode-like Lq). Size it with
   * mfa_fwd_workspace_size; NULL or too small simply disables the split. */
  void* workspace;
  size_t workspace_bytes;
  /* varlen, optional: a HOST copy of cu_q ([B + 1]). With it (and B <= 256) the launch runs
   * exactly the CTAs the sequences need, longest sequence first, instead of max_lq's row
   * blocks for every sequence with the surplus CTAs exiting at once. */
  const int32_t* cu_q_host;
} mfa_fwd_params;

/* Attention forward. Replaces the tier dispatch under flash_attn_forward
 * (metal_flash_attn/_kernel.py:1052-1153) and every Metal launcher it calls
 * (_kernel.py:1288-1420). Returns MFA_OK or an error; a launch error is reported here,
 * a kernel-side timeout through p->err. */
int mfa_fwd(const mfa_fwd_params* p, void* cuda_stream);

/* mfa_fwd for callers that cannot allocate device memory (no counterpart in the reference).
 * Some callers cannot call cudaMalloc during a forward: code running under an allocator that
 * owns all device memory, a custom memory pool, or a real-time loop that must not take the
 * allocator's locks or trigger an implicit synchronisation. This entry point takes the same
 * params (their workspace fields are ignored) and allocates nothing: when the keys are split
 * over extra CTAs, the partial results go to a fixed 16 MiB device array inside the library,
 * which every GPU that loads libmfa.so holds until the process exits. A problem that would
 * need more than 16 MiB of that scratch is rejected with MFA_ERR_SCRATCH_TOO_SMALL (use
 * mfa_fwd with a workspace for it); problems that do not split need no scratch at all.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture. The address is kept for
 * the life of the process: do not use this entry point across a cudaDeviceReset (or any other
 * teardown of the device's primary context), after which the kept address is stale. All calls share the
 * one array: calls whose kernels can overlap on the GPU (different streams, or several host
 * threads) race on it and must be serialised by the caller. Nothing in it needs to start at
 * zero: each call overwrites every slot it reads. */
int mfa_fwd_noalloc(const mfa_fwd_params* p, void* cuda_stream);

/* Bytes of workspace mfa_fwd can use for these params on the current device (0 when it would
 * not split the keys). No counterpart in the reference, whose tiers never split keys. */
size_t mfa_fwd_workspace_size(const mfa_fwd_params* p);

/* Number of key splits mfa_fwd would use for these params with the workspace they carry (1 =
 * no split), or a negative mfa_status. Lets callers and tests see the plan. */
int mfa_fwd_num_splits(const mfa_fwd_params* p);

/* Query heads mfa_fwd packs into the rows of one tile per KV head for these params (1 = none),
 * or a negative mfa_status. Decode-like GQA/MQA calls (fewer than 128 query rows per sequence,
 * a power-of-two group of at most 16) load each K/V block once per KV group instead of once per
 * query head. No counterpart in the reference, which runs one threadgroup row per query head. */
int mfa_fwd_packed_heads(const mfa_fwd_params* p);

/* Which kernel mfa_fwd would run for these params (mfa_kernel value, never AUTO), or a
 * negative mfa_status if the call would be rejected. Replaces the label logic of the
 * reference's trace (_effective_kernel_label, metal_flash_attn/_kernel.py:995-1019). */
int mfa_select_kernel(const mfa_fwd_params* p);

/* Log-sum-exp merge of n partial results over disjoint key sets (split-KV). Partial g has
 * o_part[g] fp32 [rows, H, D] (row stride H*D, head stride D) normalised by its own sum, and
 * lse_part[g] fp32 [H, rows]. Writes o (o_dtype, same layout) and optionally lse [H, rows].
 * No counterpart in the reference (its tiers never split keys); the merge restates
 * lse = log sum_g exp(lse_g), o = sum_g exp(lse_g - lse) o_g. */
int mfa_lse_combine(const float* const* o_part, const float* const* lse_part, int32_t n,
                    int32_t rows, int32_t H, int32_t D, void* o, int32_t o_dtype,
                    float* lse, void* cuda_stream);

/* First half of a split-KV merge whose partials live on several GPUs (no counterpart in the
 * reference). With o_part/lse_part laid out as in mfa_lse_combine and lse_ref fp32 [H, rows]
 * the log-sum-exp of the row over every partial on every GPU, writes
 * o[row, h, :] = sum_g exp(lse_g - lse_ref) o_g[row, h, :] (terms with lse_g or lse_ref = -inf
 * are 0). Summing these over the GPUs (an NCCL reduce-scatter by query rows) gives the exact
 * merged rows: the second half of the merge is the collective itself. */
int mfa_lse_rescale_sum(const float* const* o_part, const float* const* lse_part, int32_t n,
                        int32_t rows, int32_t H, int32_t D, const float* lse_ref, void* o,
                        int32_t o_dtype, void* cuda_stream);

/* ---- split-KV over several GPUs, merged through peer memory (no counterpart in the
 * reference, which runs on one Apple GPU). The query rows are owned by GPUs in contiguous
 * blocks of rows_per_peer; every GPU holds some of the keys. mfa_fwd_scatter runs this GPU's
 * forward over its keys and its epilogue stores each fp32 partial row (normalised by its own
 * softmax sum) and the row log-sum-exp straight into the OWNING GPU's receive buffers, slot
 * `slot`, with plain stores over NVLink, so the exchange overlaps the attention itself. After
 * every GPU's scatter has completed (the caller orders that, e.g. with an NCCL all-reduce on a
 * one-element tensor), each GPU merges the slots of its own rows locally with mfa_lse_merge.
 * Receive buffers come from mfa_peer_alloc on their own GPU and are mapped on the others with
 * mfa_peer_open (CUDA IPC handles of MFA_IPC_HANDLE_BYTES bytes, exchanged by the caller). */
#define MFA_MAX_PEERS 8
#define MFA_IPC_HANDLE_BYTES 64
typedef struct mfa_peer_scatter {
  int32_t n_peers;        /* GPUs owning query rows (1..MFA_MAX_PEERS) */
  int32_t rows_per_peer;  /* GPU g owns rows [g * rows_per_peer, (g + 1) * rows_per_peer) */
  int32_t slot;           /* slot of this launch in every receive buffer (e.g. its rank) */
  float* o_recv[MFA_MAX_PEERS];   /* GPU g's receive buffer, mapped here: fp32
                                     [slots][rows_per_peer][B][Hq][D], 16-byte aligned */
  float* lse_recv[MFA_MAX_PEERS]; /* fp32 [slots][B * Hq][rows_per_peer] */
} mfa_peer_scatter;

/* mfa_fwd with its output scattered by query row to the owning GPUs (see above). Dense inputs,
 * the tcgen05 kernel (fp16/bf16, D % 8 == 0); p->o and p->lse are ignored, p->Lq must be
 * <= n_peers * rows_per_peer, and the caller guarantees every slot index < the buffers' slot
 * count. p->k_pos_offset / p->lk_total place this GPU's keys in the whole sequence. */
int mfa_fwd_scatter(const mfa_fwd_params* p, const mfa_peer_scatter* s, void* cuda_stream);

/* Local log-sum-exp merge of n partials of the same rows: o_parts fp32 [n][rows][H][D],
 * lse_parts fp32 [n][H][rows] (a receive buffer as mfa_fwd_scatter fills it, H = B * Hq).
 * Writes o [rows][H][D] in o_dtype and, if lse != NULL, lse [H][rows]. */
int mfa_lse_merge(const float* o_parts, const float* lse_parts, int32_t n, int32_t rows,
                  int32_t H, int32_t D, void* o, int32_t o_dtype, float* lse, void* cuda_stream);

/* The pull side of a split-KV over GPUs (no counterpart in the reference): each GPU has run
 * its forward over its keys into its own fp32 partial buffer [rows_total][H][D] with row
 * log-sum-exp [H][rows_total] (an ordinary mfa_fwd with o_dtype fp32 and lse); after all have
 * finished, every GPU merges ITS rows [row0, row0 + nrows) from all n partials, reading the
 * other GPUs' buffers through peer mappings (mfa_peer_open) with plain loads over NVLink.
 * Writes o [nrows][H][D] in o_dtype and, if lse != NULL, lse [H][nrows]. */
int mfa_lse_merge_rows(const float* const* o_parts, const float* const* lse_parts, int32_t n,
                       int32_t rows_total, int32_t row0, int32_t nrows, int32_t H, int32_t D,
                       void* o, int32_t o_dtype, float* lse, void* cuda_stream);

/* Receive buffers for mfa_fwd_scatter: device memory on the current GPU plus its CUDA IPC
 * handle (MFA_IPC_HANDLE_BYTES bytes written to ipc_handle). */
int mfa_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another GPU's receive buffer (from its IPC handle) into this process. */
int mfa_peer_open(const void* ipc_handle, void** ptr);
int mfa_peer_close(void* ptr);   /* unmap a buffer mapped by mfa_peer_open */
int mfa_peer_free(void* ptr);    /* free a buffer from mfa_peer_alloc */

/* Host buffers of mfa_fwd_staged. */
typedef struct {
  const void *q, *k, *v; /* inputs in host memory (pinned for overlap), laid out with the same
                            strides as the device buffers p->q, p->k, p->v */
  void* o;               /* output in host memory, same strides as p->o */
  const int32_t* cu_q;   /* varlen only: host copies of p->cu_q / p->cu_k ([B + 1]) */
  const int32_t* cu_k;
  int32_t chunks;        /* pipeline pieces: 0 = automatic (about half a wave of 256-row
                            CTAs per piece, at most 16), 1 = copy, compute, copy back */
} mfa_host_io;

/* Forward of host-resident inputs into a host-resident output (no counterpart in the
 * reference, whose tensors live on the device already). p describes the problem and names
 * device buffers of the same layout that serve as staging areas (p->lse, if set, stays on the
 * device). The problem is cut into pieces: runs of query rows of each batch (each needing only
 * the key prefix its last row can attend: causal and right-windowed inputs start computing
 * before all keys have arrived) or runs of whole varlen sequences. The host-to-device copy of
 * piece c+1, the forward of piece c and the device-to-host copy of piece c-1 overlap, on two
 * internal streams joined to cuda_stream by events: when the call's work on cuda_stream is
 * complete, io->o holds the result. Results equal one mfa_fwd call on the whole problem. */
int mfa_fwd_staged(const mfa_fwd_params* p, const mfa_host_io* io, void* cuda_stream);

/* Failure-detection self-test (no counterpart in the reference): launches one thread that waits
 * on an mbarrier nothing arrives on, with the same bounded wait the attention kernels use but a
 * limit of timeout_us microseconds, and stores MFA_ERR_TIMEOUT (or 0) in the device int *err.
 * Shows that a stalled wait ends with a status the host can read and leaves the context usable;
 * it faults, traps or hangs nothing. */
int mfa_selftest_wait_timeout(int32_t* err, uint32_t timeout_us, void* cuda_stream);

const char* mfa_status_string(int status);
int mfa_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MFA_H_ */
