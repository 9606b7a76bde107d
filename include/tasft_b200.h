/*
 * tasft_b200.h -- C ABI of libtasft_b200.so, the B200 (sm_100a) implementation of
 * TASFT's gated block-sparse attention path.
 *
 * Conventions
 *   - Every pointer in an args struct is a DEVICE pointer unless its comment says
 *     otherwise. The caller owns every buffer, including the workspace whose size
 *     the matching *_workspace_size() call returns. The library keeps no allocation,
 *     with one exception: tasft_bsa_decode_fwd_noalloc's static per-device scratch
 *     array of tasft_decode_noalloc_capacity() bytes.
 *   - Strides are in ELEMENTS (int64). Tensors are 4-D [batch, heads, seq, dim]
 *     unless stated; the innermost (dim) stride must be 1.
 *   - Launches are asynchronous on the given stream; no call synchronises the host.
 *   - Return value: TASFT_OK (0) or a negative status for an argument error found on
 *     the host before anything is launched. Errors that only the device can see
 *     (an index out of range, a bounded wait that ran out) are OR-ed into the
 *     optional `err` word (TASFT_DEVERR_* bits) and never trap the GPU.
 *
 * Reference interfaces replaced (v-code01/tasft, paths inside that project):
 *   tasft_gate_mask_build      AttnGate.forward           tasft/modules/attn_gate.py:377-485
 *   tasft_mask_from_scores     soft >= tau (+ tril)       tasft/modules/attn_gate.py:466-477
 *   tasft_qkv_rope_pool        _prepare_qkv head split + rotary + the gate's pooling
 *                              tasft/modules/tasft_attention.py:615-742, attn_gate.py:351-375
 *   tasft_mask_to_kept         bool mask & block tril     tasft/kernels/block_sparse_fa.py:497-508
 *   tasft_calibrate_tau        the weight-norm estimate of per-layer sparsity
 *                                                         tasft/bundle/export.py:327-360
 *   tasft_bsa_prefill_fwd      _block_sparse_attn_fwd_kernel launch
 *                                                         tasft/kernels/block_sparse_fa.py:454-552
 *   tasft_bsa_decode_fwd       (none: new capability; the reference delegates decode
 *                              to vLLM's dense forward, tasft/inference/vllm_patch.py:189-196)
 *   tasft_bsa_decode_combine   (none: split-KV (m,l,o) merge for multi-GPU decode)
 *   tasft_gate_target_fwd      TASFTAttention scores + compute_gate_target
 *                              tasft/modules/tasft_attention.py:427-458,
 *                              tasft/training/objectives.py:128-185
 *   tasft_attention_train_fwd  TASFTAttention._training_forward scores + softmax + P V and
 *                              compute_gate_target, fused (tasft_attention.py:427-466)
 *   tasft_gate_target_from_scores  compute_gate_target on a score tensor
 *                              tasft/training/objectives.py:128-185
 *   tasft_gate_loss_fwd_bwd    compute_gate_loss + compute_sparsity_loss (+ grad)
 *                              tasft/training/objectives.py:187-241
 *   tasft_gate_bwd             autograd of AttnGate.forward to its parameters
 *                              tasft/modules/attn_gate.py:442-459
 */
#ifndef TASFT_B200_H_
#define TASFT_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define TASFT_API __attribute__((visibility("default")))
#else
#define TASFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TASFT_ABI_VERSION 3

/* status codes (host-side, returned) */
#define TASFT_OK                  0
#define TASFT_ERR_INVALID_ARG    -1  /* null pointer, bad shape, bad stride */
#define TASFT_ERR_UNSUPPORTED    -2  /* dtype / head_dim / block size not built */
#define TASFT_ERR_CUDA           -3  /* a CUDA runtime call failed */
#define TASFT_ERR_WORKSPACE      -4  /* workspace missing or too small */
#define TASFT_ERR_TOO_LARGE      -5  /* a size exceeds a fixed capacity */

/* device error word bits (OR-ed into *err when err != NULL) */
#define TASFT_DEVERR_INDEX        1  /* a kept index outside [0, NB_k) was skipped */
#define TASFT_DEVERR_TIMEOUT      2  /* a bounded wait gave up */
#define TASFT_DEVERR_ORDER        4  /* a kept list was not strictly ascending */

/* element types */
#define TASFT_F32   0
#define TASFT_BF16  1
#define TASFT_F16   2

typedef void* tasft_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* ------------------------------------------------------------------------- */
/* AttnGate: pooled pair-MLP scores, hard mask and kept-block lists          */
/* ------------------------------------------------------------------------- */
typedef struct {
  const void* q;          /* [B, Hq, Sq, D]  dtype */
  const void* k;          /* [B, Hk, Sk, D]  dtype, Hq % Hk == 0 (GQA: K shared per group) */
  int64_t q_stride[4];
  int64_t k_stride[4];
  int32_t B, Hq, Hk, Sq, Sk, D;
  int32_t block;          /* tokens per block (any positive value) */
  int32_t dtype;          /* TASFT_F32 / TASFT_BF16 / TASFT_F16 */
  int32_t hidden;         /* gate MLP width, <= 256 */
  const float* w_in;      /* [hidden, 2D] fp32 row-major (nn.Linear weight) */
  const float* b_in;      /* [hidden] fp32 */
  const float* w_out;     /* [hidden] fp32 */
  int32_t causal;         /* zero blocks j > i when NB_q == NB_k (reference semantics) */
  float tau;              /* hard = soft >= tau */
  float* soft;            /* out [B, Hq, NBq, NBk] fp32 (required) */
  uint8_t* hard;          /* out [B, Hq, NBq, NBk] bool, or NULL */
  int32_t* kept_idx;      /* out [B, Hq, NBq, NBk] ascending kept k-blocks, -1 padded, or NULL */
  int32_t* kept_cnt;      /* out [B, Hq, NBq], or NULL (required with kept_idx) */
  int32_t* num_kept;      /* out scalar: total kept blocks over the full grid, or NULL */
  float* pooled_q;        /* out [B, Hq, NBq, D] fp32 block means, or NULL */
  float* pooled_k;        /* out [B, Hk, NBk, D] fp32 block means, or NULL */
  void* workspace;        /* tasft_gate_workspace_size() bytes */
  int64_t workspace_bytes;
} tasft_gate_args;

/* Workspace of tasft_gate_mask_build: the projected block rows plus the fp32 block means
 * (ABI 2 added `D`). */
TASFT_API int64_t tasft_gate_workspace_size(int32_t B, int32_t Hq, int32_t Hk, int32_t Sq, int32_t Sk,
                                  int32_t block, int32_t hidden, int32_t D);
/* Pooled-input mode: with q == k == NULL, pooled_q / pooled_k are INPUTS (the block means
 * from tasft_qkv_rope_pool) and the pooling pass is skipped; hidden 32 or 64, D % 4 == 0. */
TASFT_API int tasft_gate_mask_build(const tasft_gate_args* args, tasft_stream_t stream);

/* Q/K/V projection epilogue: head split [B, S, H*D] -> [B, H, S, D], rotary embedding of
 * Q and K (x * cos + rotate_half(x) * sin, each op rounded to the dtype as the reference's
 * element-wise ops are), and the fp32 block means of the rotated Q and K that AttnGate pools
 * (zero padding counts). Replaces TASFTAttention._prepare_qkv's view / transpose / rotary
 * (tasft/modules/tasft_attention.py:615-742, :872-908) and the gate's pooling pass
 * (tasft/modules/attn_gate.py:351-375); K/V are not repeated per q-head. Pass the means
 * to tasft_gate_mask_build with q = k = NULL (pooled-input mode). */
typedef struct {
  const void* q_in;       /* [B, S, Hq*D] rows; element strides (batch, token) below, D contiguous */
  const void* k_in;       /* [B, S, Hk*D] */
  const void* v_in;       /* [B, S, Hk*D] */
  int64_t q_in_stride[2], k_in_stride[2], v_in_stride[2];
  const void* cos;        /* [B or 1, S, D] (HF layout, halves duplicated); unused when rope == 0 */
  const void* sin;
  int64_t cs_stride[2];   /* batch stride (0 = shared over the batch), token stride */
  void* q_out;            /* [B, Hq, S, D] contiguous */
  void* k_out;            /* [B, Hk, S, D] contiguous */
  void* v_out;            /* [B, Hk, S, D] contiguous */
  float* pooled_q;        /* out [B, Hq, NB, D] fp32 block means of the rotated Q, or NULL */
  float* pooled_k;        /* out [B, Hk, NB, D], or NULL */
  int32_t B, Hq, Hk, S, D;
  int32_t block;          /* gate block size (tokens) */
  int32_t dtype;
  int32_t rope;           /* 1 = apply the rotary embedding to Q and K, 0 = layout only */
} tasft_qkv_args;
TASFT_API int tasft_qkv_rope_pool(const tasft_qkv_args* args, tasft_stream_t stream);

/* Threshold given fp32 scores: hard = (soft >= tau) (& block tril when causal),
 * ascending kept lists, counts and the total. Bit-exact with the reference's
 * `soft >= tau` on the same scores. */
typedef struct {
  const float* soft;      /* [rows, NBk] fp32, rows = B*H*NBq, row-major */
  int64_t rows;
  int32_t NBq, NBk;       /* row r is q-block (r % NBq) */
  int32_t causal;         /* also drop k-block > q-block */
  float tau;
  uint8_t* hard;          /* out [rows, NBk] or NULL */
  int32_t* kept_idx;      /* out [rows, NBk] -1 padded, or NULL */
  int32_t* kept_cnt;      /* out [rows] or NULL */
  int32_t* num_kept;      /* out scalar or NULL */
} tasft_threshold_args;
TASFT_API int tasft_mask_from_scores(const tasft_threshold_args* args, tasft_stream_t stream);

/* Threshold calibration: tau = the keep-th largest of n gate scores (exact radix select),
 * so that `soft >= tau` keeps `keep` blocks (more only on ties at tau). Replaces the
 * weight-norm sparsity estimate of tasft/bundle/export.py:327-360 with a measured per-layer
 * tau. keep <= 0 gives +inf (keep nothing), keep > n gives -inf (keep everything). */
typedef struct {
  const float* scores;    /* [n] fp32 gate scores (the full grid, causal zeros included) */
  int64_t n;
  int64_t keep;
  float* tau;             /* out device scalar */
  int64_t* kept;          /* out device scalar: count of scores >= tau, or NULL */
} tasft_calib_args;
TASFT_API int tasft_calibrate_tau(const tasft_calib_args* args, tasft_stream_t stream);

/* Bool block mask -> ascending kept lists (the reference kernel's visiting order). */
typedef struct {
  const uint8_t* mask;    /* [rows, NBk] bool, row-major */
  int64_t rows;
  int32_t NBq, NBk;
  int32_t causal;         /* AND with the block lower triangle, as the reference host does */
  int32_t* kept_idx;      /* out [rows, NBk] -1 padded */
  int32_t* kept_cnt;      /* out [rows] */
  int32_t* num_kept;      /* out scalar or NULL */
} tasft_mask_args;
TASFT_API int tasft_mask_to_kept(const tasft_mask_args* args, tasft_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Block-sparse prefill attention                                            */
/* ------------------------------------------------------------------------- */
typedef struct {
  const void* q;          /* [B, Hq, S, D] */
  const void* k;          /* [B, Hk, S, D], Hq % Hk == 0 */
  const void* v;          /* [B, Hk, S, D] */
  void* out;              /* [B, Hq, S, D] */
  int64_t q_stride[4], k_stride[4], v_stride[4], o_stride[4];
  int32_t B, Hq, Hk, S, D;
  int32_t block;          /* 32, 64 or 128 */
  int32_t dtype;
  int32_t causal;
  float scale;            /* softmax scale, normally 1/sqrt(D) */
  const int32_t* kept_idx;/* [B, Hm, NB, NB] ascending kept k-blocks per (b, head, q-block) */
  const int32_t* kept_cnt;/* [B, Hm, NB] */
  int32_t Hm;             /* heads of the lists: Hq (per q-head) or Hk (per kv-head) */
  int32_t* err;           /* optional device error word */
  int32_t force_simt;     /* 1 = use the CUDA-core kernel even where tcgen05 applies (testing) */
  int32_t qb_lo, qb_hi;   /* q-block window [qb_lo, qb_hi) (one rank's share of a long sequence);
                             qb_hi <= 0: every q-block. The tcgen05 kernel visits only the window's
                             tiles and leaves the other output rows untouched (the CUDA-core kernel
                             computes every row); padded layout only */
} tasft_prefill_args;
TASFT_API int tasft_bsa_prefill_fwd(const tasft_prefill_args* args, tasft_stream_t stream);

/* Prefill of a batch of sequences of different lengths packed along the token axis (the
 * layout vLLM hands its attention backend). Replaces the reference's vLLM prefill, which
 * flattens the batch into one causal sequence so sequences attend across their
 * boundaries (tasft/inference/vllm_patch.py:172-196); here each sequence attends only
 * within itself. `base` is read as for tasft_bsa_prefill_fwd except:
 *   base.q / k / v / out   packed [total, H, D]; strides given as [1, H, token, D]: the
 *                          first is never stepped (pass total*H*D), e.g. {T*H*D, D, H*D, 1}
 *   base.B                 number of sequences; base.S = longest sequence (NB = ceil(S/block))
 *   kept lists             [B, Hm, NB, NB] per sequence, as for the padded call
 * Sequence b is rows [cu_seqlens[b], cu_seqlens[b+1]). Same dtypes, blocks and head dims
 * as tasft_bsa_prefill_fwd (tensor cores for bf16/fp16, block 64, D 64/128; the CUDA-core
 * kernel otherwise, or with base.force_simt). */
typedef struct {
  tasft_prefill_args base;
  const int32_t* cu_seqlens; /* device [B + 1], ascending, cu_seqlens[0] = 0 */
  int32_t total;             /* cu_seqlens[B] */
} tasft_prefill_varlen_args;
TASFT_API int tasft_bsa_prefill_varlen_fwd(const tasft_prefill_varlen_args* args, tasft_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Block-sparse decode (one query token per sequence), split-KV               */
/* ------------------------------------------------------------------------- */
typedef struct {
  const void* q;          /* [B, Hq, D] */
  const void* k_cache;    /* [B, Hk, L, D] */
  const void* v_cache;    /* [B, Hk, L, D] */
  void* out;              /* [B, Hq, D] (may be NULL when only partials are wanted) */
  int64_t q_stride[3], k_stride[4], v_stride[4], o_stride[3];
  int32_t B, Hq, Hk, L, D;
  int32_t block;
  int32_t dtype;
  float scale;
  const int32_t* kv_len;  /* [B] valid cache length per sequence (<= L) */
  const int32_t* kept_idx;/* [B, Hk, NBmax] ascending kept blocks per (sequence, kv-head) */
  const int32_t* kept_cnt;/* [B, Hk] */
  int32_t nb_max;         /* row length of kept_idx */
  int32_t num_splits;     /* 0 = choose; else CTAs per (sequence, kv-head) */
  float* part_o;          /* optional out [B, Hq, D] fp32 normalised partial (for cross-GPU combine) */
  float* part_ml;         /* optional out [B, Hq, 2] fp32 (m, l) in base-e units */
  void* workspace;        /* tasft_decode_workspace_size() bytes; the call clears its ticket prefix */
  int64_t workspace_bytes;
  int32_t* err;
  int32_t kv_offset;      /* tokens before this cache's first row (one rank's slab of a longer
                             sequence): valid rows = clamp(kv_len - kv_offset, 0, L); 0 otherwise */
} tasft_decode_args;
TASFT_API int64_t tasft_decode_workspace_size(int32_t B, int32_t Hq, int32_t Hk, int32_t D, int32_t max_splits);
TASFT_API int tasft_bsa_decode_fwd(const tasft_decode_args* args, tasft_stream_t stream);

/* Same computation as tasft_bsa_decode_fwd, for callers that cannot allocate device
 * memory (a plugin whose host owns every allocation, a serving loop that must not call
 * cudaMalloc). No counterpart in the reference. The split-KV scratch is a fixed
 * per-device array of tasft_decode_noalloc_capacity() bytes (4 MiB) inside the library;
 * args->workspace is ignored. The first call on a device looks the array up and should
 * come before any stream capture. The address is cached per device for the life of the
 * process; after cudaDeviceReset on that device the entry point must not be called again. All calls on a device share the array: calls that
 * overlap on the GPU race; order them on one stream. A call that needs more scratch than
 * the capacity returns TASFT_ERR_TOO_LARGE without launching. Nothing is allocated. */
TASFT_API int tasft_bsa_decode_fwd_noalloc(const tasft_decode_args* args, tasft_stream_t stream);
TASFT_API int64_t tasft_decode_noalloc_capacity(void);

/* Block-sparse decode over a PAGED KV cache (vLLM's flash layout). No counterpart in the
 * reference: its vLLM backend runs decode dense over paged caches
 * (tasft/inference/vllm_patch.py:189-196); this is the sparse replacement for that call.
 * `base` is read as for tasft_bsa_decode_fwd except:
 *   base.k_cache / base.v_cache  page pools [num_pages, page_size, Hk, D]
 *   base.k_stride / base.v_stride element strides of those pools (stride[3] == 1)
 *   base.L                       logical capacity = max_pages * page_size
 * Logical token t of sequence b lives in page block_table[b * max_pages + t / page_size]
 * at row t % page_size. Kept lists stay in logical 64-token blocks. bf16/fp16, D 64 or
 * 128, block 64, page_size 16, 32, 64 or 128. A table entry outside [0, num_pages) is
 * skipped and reported as TASFT_DEVERR_INDEX. */
typedef struct {
  tasft_decode_args base;
  const int32_t* block_table; /* [B, max_pages] */
  int32_t max_pages;
  int32_t page_size;
  int32_t num_pages;
} tasft_paged_decode_args;
TASFT_API int tasft_bsa_decode_paged_fwd(const tasft_paged_decode_args* args, tasft_stream_t stream);

/* Merge G partial results (normalised o, m, l) into the final output. */
typedef struct {
  const float* part_o;    /* [G, rows, D] fp32 */
  const float* part_ml;   /* [G, rows, 2] fp32 */
  int32_t G;
  int64_t rows;           /* B * Hq */
  int32_t D;
  void* out;              /* [rows, D] contiguous, dtype */
  int32_t dtype;
} tasft_combine_args;
TASFT_API int tasft_bsa_decode_combine(const tasft_combine_args* args, tasft_stream_t stream);

/* Cross-GPU merge of split-KV decode partials over peer memory, in place of an NCCL
 * all-gather + tasft_bsa_decode_combine. No counterpart in the reference (it has no
 * sparse decode). Each rank owns a mailbox (tasft_peer_alloc of
 * tasft_peer_mailbox_bytes(world, rows, D) bytes, zeroed) and maps every other rank's
 * mailbox with tasft_ipc_handle / tasft_ipc_open (CUDA IPC; one process per GPU). A call
 * pushes this rank's partial into every mailbox with plain stores, raises its flag in each,
 * waits for all ranks' flags in its own mailbox (bounded by timeout_ns; on expiry
 * TASFT_DEVERR_TIMEOUT is OR-ed into *err and the exchange must be rebuilt) and writes
 * the merged output. Every rank must make the same sequence of calls; the per-rank epoch
 * counter lives on the device, so a step that contains the call can be replayed from a
 * CUDA graph. */
typedef struct {
  const float* part_o;    /* [rows, D] this rank's normalised partial output */
  const float* part_ml;   /* [rows, 2] its (m, l), base e */
  int64_t rows;           /* B * Hq */
  int32_t D;              /* even; part_o and part_ml 8-byte aligned */
  int32_t world, rank;    /* world <= 8 (one NVLink node) */
  void* const* mailboxes; /* device array [world] of device pointers: rank r's mailbox (own or IPC-mapped) */
  uint32_t* epoch;        /* device scalar of this rank, zero before the first call */
  void* out;              /* [rows, D] dtype */
  int32_t dtype;
  uint64_t timeout_ns;    /* bound of the wait for the other ranks */
  int32_t* err;           /* optional device error word */
} tasft_peer_combine_args;
TASFT_API int64_t tasft_peer_mailbox_bytes(int32_t world, int64_t rows, int32_t D);

/* Split-KV decode with the cross-GPU merge fused in: one call runs this rank's decode over its
 * slab of the cache, and the kernel that merges the rank's splits also pushes the rank's
 * (o, m, l) rows straight into every rank's mailbox (plain 8-byte stores through the IPC
 * mappings, each word carrying the call's epoch beside its value, so no fence or flag),
 * waits (bounded by timeout_ns; TASFT_DEVERR_TIMEOUT into args->err on expiry) for every
 * rank's rows in its own mailbox and writes the merged output to args->out. Replaces tasft_bsa_decode_fwd (with part_o / part_ml) followed by
 * tasft_peer_combine; same mailboxes (tasft_peer_mailbox_bytes, tasft_peer_alloc,
 * tasft_ipc_*) and epoch, so the two may be mixed in one sequence of calls that every rank
 * makes alike. bf16 / f16, block 64, D 64 / 128, group <= 8, world <= 8; needs a workspace
 * (at least 2 splits). No counterpart in the reference (it has no sparse decode). */
typedef struct {
  void* const* mailboxes; /* device array [world] of device pointers, as in tasft_peer_combine_args */
  uint32_t* epoch;        /* device scalar of this rank */
  int32_t world, rank;
  uint64_t timeout_ns;
} tasft_decode_peer_args;
TASFT_API int tasft_bsa_decode_peer_fwd(const tasft_decode_args* args, const tasft_decode_peer_args* peer,
                                        tasft_stream_t stream);
TASFT_API int tasft_peer_alloc(int64_t bytes, void** ptr);
TASFT_API int tasft_peer_free(void* ptr);
TASFT_API int tasft_ipc_handle(void* ptr, uint8_t* handle64);
TASFT_API int tasft_ipc_open(const uint8_t* handle64, void** ptr);
TASFT_API int tasft_ipc_close(void* ptr);
TASFT_API int tasft_peer_combine(const tasft_peer_combine_args* args, tasft_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Training-time gate target, losses and gate backward                       */
/* ------------------------------------------------------------------------- */
typedef struct {
  const void* q;          /* [B, Hq, S, D] */
  const void* k;          /* [B, Hk, S, D] */
  int64_t q_stride[4], k_stride[4];
  int32_t B, Hq, Hk, S, D;
  int32_t block;
  int32_t dtype;
  float scale;            /* 1/sqrt(D) */
  int32_t emulate_bf16_scores; /* round block maxima as the reference's bf16 (QK^T)*scale */
  float temperature;      /* 1 = compute_gate_target; 2 = the alternate target */
  float clamp;            /* <= 0: none; else clamp finite maxima to [-clamp, clamp] */
  float* block_max;       /* out [B, Hq, NB, NB] fp32 (upper triangle = -inf), or NULL */
  float* target;          /* out [B, Hq, NB, NB] fp32 softmax over the NB*NB grid */
  void* workspace;        /* tasft_gate_target_workspace_size() bytes */
  int64_t workspace_bytes;
  int32_t force_simt;
  int32_t* err;
} tasft_target_args;
TASFT_API int64_t tasft_gate_target_workspace_size(int32_t B, int32_t Hq, int32_t S, int32_t block);
TASFT_API int tasft_gate_target_fwd(const tasft_target_args* args, tasft_stream_t stream);

/* Gate target from a score tensor the caller already holds, e.g. the pre-softmax
 * attention scores [B, H, Sq, Sk] a training forward kept (-inf above the diagonal):
 * -inf padding to whole blocks, block x block max-pool, optional clamp of finite maxima,
 * softmax over the NBq*NBk grid divided by `temperature`. Replaces
 * TASFTObjective.compute_gate_target (tasft/training/objectives.py:128-185; temperature 1,
 * no clamp) and TASFTAttention._compute_gate_target (tasft/modules/tasft_attention.py:
 * 220-290; temperature 2, clamp 50). Reads the whole tensor once (HBM-bound) and reports
 * NaN (bit 0) and +inf (bit 1) in *flags, which the reference rejects. */
typedef struct {
  const void* scores;     /* [B, H, Sq, Sk] dtype */
  int64_t stride[4];
  int32_t B, H, Sq, Sk;
  int32_t block;          /* 1..1024 */
  int32_t dtype;
  float temperature;      /* softmax divides the maxima by this (<= 0: 1) */
  float clamp;            /* <= 0: none; else clamp finite maxima to [-clamp, clamp] */
  float* block_max;       /* out [B, H, NBq, NBk] fp32, or NULL (then the workspace holds it) */
  float* target;          /* out [B, H, NBq, NBk] fp32 */
  int32_t* flags;         /* optional device word, OR-ed: 1 = NaN seen, 2 = +inf seen */
  void* workspace;        /* tasft_scores_target_workspace_size() bytes when block_max is NULL */
  int64_t workspace_bytes;
} tasft_scores_target_args;
TASFT_API int64_t tasft_scores_target_workspace_size(int32_t B, int32_t H, int32_t Sq, int32_t Sk, int32_t block);
TASFT_API int tasft_gate_target_from_scores(const tasft_scores_target_args* args, tasft_stream_t stream);

/* Training forward in one pass: the attention output of tasft_bsa_prefill_fwd (pass kept
 * lists with every causal block for the reference's dense training attention) and, from
 * the same on-chip S tiles, the block maxima of the scores (the S x S score tensor is never
 * formed) and their softmax target. Replaces TASFTAttention._training_forward's
 * scores / softmax / P V (tasft/modules/tasft_attention.py:427-466) plus
 * TASFTObjective.compute_gate_target (tasft/training/objectives.py:128-185). Only the
 * tcgen05 shapes (bf16/fp16, block 64, D 64/128, padded layout); other shapes return
 * TASFT_ERR_UNSUPPORTED (use tasft_bsa_prefill_fwd + tasft_gate_target_fwd). */
typedef struct {
  tasft_prefill_args base;
  float* block_max;       /* out [B, Hq, NB, NB] fp32: max of (Q K^T) * scale per visited tile, -inf elsewhere */
  float* target;          /* out [B, Hq, NB, NB] fp32 softmax over the grid, or NULL */
  float temperature;      /* 1 = compute_gate_target; 2 = TASFTAttention._compute_gate_target */
  float clamp;            /* <= 0: none; else clamp finite maxima to [-clamp, clamp] before the softmax */
  int32_t emulate_bf16_scores; /* round the maxima as the reference's bf16 (Q K^T) * scale */
} tasft_train_fwd_args;
TASFT_API int tasft_attention_train_fwd(const tasft_train_fwd_args* args, tasft_stream_t stream);

typedef struct {
  const float* soft;      /* [B, H, NB, NB] gate scores */
  const float* target;    /* [B, H, NB, NB] */
  int32_t B, H, NBq, NBk;
  float tau_target;       /* sparsity target */
  float w_kl, w_sparse;   /* d_soft = w_kl dKL/dsoft + w_sparse dSparse/dsoft */
  float* kl;              /* out scalar: KL(target || gate), batchmean */
  float* sparse;          /* out scalar: (mean(soft) - tau)^2 */
  float* d_soft;          /* out [B, H, NB, NB] or NULL */
  void* workspace;        /* tasft_gate_loss_workspace_size() bytes */
  int64_t workspace_bytes;
} tasft_loss_args;
TASFT_API int64_t tasft_gate_loss_workspace_size(int32_t B, int32_t H);
TASFT_API int tasft_gate_loss_fwd_bwd(const tasft_loss_args* args, tasft_stream_t stream);

typedef struct {
  const float* pooled_q;  /* [B, Hq, NBq, D] from tasft_gate_mask_build */
  const float* pooled_k;  /* [B, Hk, NBk, D] */
  const float* d_soft;    /* [B, Hq, NBq, NBk] upstream gradient of the soft scores */
  const float* soft;      /* [B, Hq, NBq, NBk] the forward soft scores */
  int32_t B, Hq, Hk, NBq, NBk, D, hidden;
  int32_t causal;
  const float* w_in;      /* [hidden, 2D] */
  const float* b_in;      /* [hidden] */
  const float* w_out;     /* [hidden] */
  float* d_w_in;          /* out [hidden, 2D] (overwritten) */
  float* d_b_in;          /* out [hidden] */
  float* d_w_out;         /* out [hidden] */
  float* d_pooled_q;      /* out [B, Hq, NBq, D] or NULL */
  float* d_pooled_k;      /* out [B, Hk, NBk, D] or NULL */
  void* workspace;        /* tasft_gate_bwd_workspace_size() bytes */
  int64_t workspace_bytes;
} tasft_gate_bwd_args;
TASFT_API int64_t tasft_gate_bwd_workspace_size(int32_t B, int32_t Hq, int32_t Hk, int32_t NBq, int32_t NBk,
                                      int32_t hidden);
TASFT_API int tasft_gate_bwd(const tasft_gate_bwd_args* args, tasft_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Misc                                                                      */
/* ------------------------------------------------------------------------- */
TASFT_API const char* tasft_status_string(int status);
TASFT_API int tasft_abi_version(void);
/* Number of kernels this library launched since load (for launch accounting). */
TASFT_API int64_t tasft_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* TASFT_B200_H_ */
