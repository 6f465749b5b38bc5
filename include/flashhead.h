/*
 * flashhead.h - C ABI of the B200 (sm_100a) FlashHead decode-step LM head.
 *
 * FlashHead replaces the dense LM head h x W_vocab^T with a two-stage
 * retrieval over balanced token clusters (K clusters of `cluster_size`
 * tokens):
 *   stage 1  score the K cluster centroids against the hidden state and pick
 *            the top n_probes clusters (or draw them, in sampling mode);
 *   stage 2  score only the tokens of the probed clusters and return the
 *            argmax token (or a sample from the candidates' softmax).
 *
 * The reference implementation is Python/Triton (embedl/flash-head,
 * src/flash_head/flash_head.py and src/flash_head/fused.py); it has no native
 * interface. Each entry point below names the reference function whose
 * behaviour it replaces. The Python package `flash_head` binds these
 * functions with ctypes (flash_head/_lib.py).
 *
 * Conventions
 *   - Every pointer argument named hidden/w_perm/... is a DEVICE pointer; the
 *     library never allocates, frees, or synchronises, and never reads device
 *     memory on the host, so every call can be captured in a CUDA graph.
 *   - Scratch memory is caller-owned: size it with fh_workspace_bytes() and
 *     zero-fill it once before its first use. A workspace may be reused by
 *     consecutive calls on one stream, with any row count that fits; calls
 *     that may overlap on the GPU need separate workspaces.
 *   - All functions return FH_OK (0) or an fh_status code; the message of
 *     the last failure on the calling thread is available from
 *     fh_last_error(). Launch errors are reported as FH_ERR_CUDA.
 *   - stream is a cudaStream_t (NULL = legacy default stream).
 *   - Hidden-state pointers (device ones, and page-locked host ones read by
 *     the kernels directly) must be 16-byte aligned; misaligned ones are
 *     refused with FH_ERR_INVALID_ARGUMENT by every entry point that takes
 *     them.
 *   - Ties: probe selection prefers the smaller cluster id, the greedy token
 *     the smaller vocab id (fused.py:161-163).
 */
#ifndef FLASHHEAD_H
#define FLASHHEAD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FH_API __attribute__((visibility("default")))

typedef struct CUstream_st *fh_stream_t; /* identical to cudaStream_t */

typedef enum fh_status {
  FH_OK = 0,
  FH_ERR_INVALID_ARGUMENT = 1,
  FH_ERR_CUDA = 2,
  FH_ERR_WORKSPACE = 3,
  FH_ERR_UNSUPPORTED = 4
} fh_status;

typedef enum fh_dtype {
  FH_BF16 = 0,
  FH_FP16 = 1,
  FH_FP8_E4M3 = 2,
  FH_FP32 = 3
} fh_dtype;

/*
 * Device buffers of one FlashHead, laid out by the loader
 * (flash_head/flash_head.py), which owns them for the head's lifetime.
 *
 *   w_perm        [K * cluster_size, hidden]  weight_dtype (bf16/fp16): LM-head
 *                 rows in cluster order (flash_head.py:162-168)
 *   vocab_map     [K * cluster_size] int32: vocab id of every w_perm row
 *                 (the reference's vocab_maps, flash_head.py:100-118)
 *   cluster_w     [K, hidden] score_dtype: L2-normalised centroids for greedy
 *                 stage 1 (flash_head.py:158-160); fp8 rows carry
 *   cluster_scale [K] fp32 per-row dequantisation scale (NULL unless fp8)
 *   centroid_w    [K, hidden] sample_dtype: RAW centroids (transposed) used
 *                 by sampling stage 1 (flash_head.py:203-205); may be NULL
 *                 when sampling is not used
 *   centroid_scale[K] fp32 (NULL unless sample_dtype is fp8)
 *   special_slots [n_special] int32: w_perm row of every special token that
 *                 is always scored (flash_head.py:171-188, :239-249)
 *   cluster_base  global id of local cluster 0 (tensor-parallel shards; 0
 *                 for an unsharded head). Sampling noise is keyed by global
 *                 ids, so results do not depend on the shard count.
 */
typedef struct fh_head_desc {
  int32_t hidden;       /* D */
  int32_t n_clusters;   /* K (local clusters of this shard) */
  int32_t cluster_size; /* cap, 1..32 */
  int32_t n_probes;     /* p, 1..min(K_total, 4096) */
  int32_t weight_dtype; /* fh_dtype of w_perm and hidden states: BF16/FP16 */
  int32_t score_dtype;  /* fh_dtype of cluster_w: FP8_E4M3 or weight_dtype */
  int32_t sample_dtype; /* fh_dtype of centroid_w: FP8_E4M3 or weight_dtype */
  int32_t n_special;
  int32_t cluster_base;
  int32_t flags;        /* FH_FLAG_* bits, 0 by default */
  const void *w_perm;
  const int32_t *vocab_map;
  const void *cluster_w;
  const float *cluster_scale;
  const void *centroid_w;
  const float *centroid_scale;
  const int32_t *special_slots;
} fh_head_desc;

/* fh_head_desc.flags */
#define FH_FLAG_NO_FUSED 1u      /* always use the three-kernel path */
#define FH_FLAG_TEST_TIMEOUT 2u  /* test only: the fused step's grid barrier
                                    waits for one CTA more than it launches and
                                    gives up after ~1 ms, setting error bit 1 */

typedef struct fh_head fh_head; /* opaque, host memory only */

/* Library identification and error reporting. */
FH_API int fh_version(void);
FH_API const char *fh_last_error(void);

/* Validate a descriptor and make a handle (host memory only; no device work).
 * Replaces FlashHead.__init__ argument checks (flash_head.py:136-188). */
FH_API int fh_head_create(const fh_head_desc *desc, fh_head **out);
FH_API int fh_head_destroy(fh_head *head);

/* Bytes of caller-provided scratch for a call with `rows` hidden states. */
FH_API size_t fh_workspace_bytes(const fh_head *head, int rows);

/*
 * Byte offset, within a workspace, of a 32-bit word in which the one-kernel
 * step (used for up to 4 rows) records failures of its bounded waits: bit 0
 * = the grid barrier timed out, bit 1 = a bulk-copy wait timed out. The
 * kernel still completes (its outputs are then meaningless). The word is
 * sticky: the caller reads it (after synchronising) and clears it.
 */
FH_API size_t fh_workspace_error_offset(void);

/*
 * Kernel launches one fh_get_next_token / fh_get_next_token_sample call makes
 * for `rows` hidden states on the current device: 1 when the one-kernel step
 * applies (rows <= 4 and supported shapes); from 5 rows stage 1 runs on the
 * tensor cores ([an f16 copy of bf16 rows for an fp8 stage-1 matrix], one
 * stage-1 kernel per 256 rows, the selection), followed for 5..15 rows by
 * the block-sparse stage 2 and for 16+ rows by [the special tokens] and,
 * per 256 rows, the cluster-major tensor-core stage 2 (up to 256 rows the
 * selection fills its index, above that an index kernel per 256 rows; the
 * tile builder; the stage-2 kernel, whose last CTA publishes the ids);
 * 3 for the CUDA-core stage kernels (unsupported shapes). Memsets are not
 * counted.
 */
FH_API int fh_step_kernel_count(const fh_head *head, int rows, int do_sample);

/*
 * Greedy next token for `rows` hidden states [rows, hidden]:
 * out_ids[rows] (int64). Replaces FlashHead.get_next_token(h) on its fused
 * greedy branch (flash_head.py:277-321: cluster_linear + topk +
 * block_sparse_argmax_atomic) and on its special-token / tiebreak branch
 * (:323-334), which differs from it only in tie handling.
 */
FH_API int fh_get_next_token(const fh_head *head, const void *hidden, int rows,
                             int64_t *out_ids, void *workspace,
                             size_t workspace_bytes, fh_stream_t stream);

/*
 * Greedy next token with HOST buffers: hidden_host [rows, hidden],
 * out_ids_host [rows] int64. The call brings the hidden states to the device,
 * runs fh_get_next_token on the workspace and returns once the ids are in
 * out_ids_host. Page-locked buffers are read and written by the kernels
 * directly (a small copy kernel in, the step's own id stores out): the call
 * marks out_ids_host with -1 and returns as soon as every row has been
 * overwritten, possibly before the kernel's last instructions retire (later
 * work on `stream` is ordered after it; reuse the workspace on the same
 * stream); after 20 ms it falls back to synchronising `stream`. Pageable
 * buffers go through cudaMemcpyAsync and a stream synchronisation.
 * For C and C++ callers that keep the decode state on the host; the
 * reference's get_next_token (flash_head.py:277-334) takes device tensors.
 * The workspace must hold fh_workspace_bytes_host(head, rows) bytes (the
 * device staging of inputs and ids sits at its end).
 */
FH_API size_t fh_workspace_bytes_host(const fh_head *head, int rows);
FH_API int fh_get_next_token_host(const fh_head *head, const void *hidden_host, int rows,
                                  int64_t *out_ids_host, void *workspace,
                                  size_t workspace_bytes, fh_stream_t stream);

/*
 * Greedy next token WITHOUT a workspace argument; nothing is allocated. No
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they need a token, e.g. code running while a CUDA graph
 * is being captured, a latency-critical thread that must not enter the
 * allocator, or a host runtime whose fixed memory pool forbids cudaMalloc.
 *
 * Its scratch is a fixed array inside this library (FH_NOALLOC_SCRATCH_BYTES
 * bytes of device memory that every GPU loading the library holds until the
 * process exits). Limits: rows <= FH_NOALLOC_MAX_ROWS, n_clusters <=
 * FH_NOALLOC_MAX_CLUSTERS, n_probes <= FH_NOALLOC_MAX_PROBES; larger requests
 * return FH_ERR_UNSUPPORTED. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current: make that
 * first call before capturing a CUDA graph. Every call uses the same array
 * and clears what must start at zero itself; calls that may run at the same
 * time on the GPU (other streams, other threads) race on it, so the caller
 * must serialise them. Results equal fh_get_next_token's three-kernel path.
 */
#define FH_NOALLOC_MAX_ROWS 4
#define FH_NOALLOC_MAX_CLUSTERS 16384
#define FH_NOALLOC_MAX_PROBES 4096
#define FH_NOALLOC_SCRATCH_BYTES 328192
FH_API int fh_get_next_token_noalloc(const fh_head *head, const void *hidden, int rows,
                                     int64_t *out_ids, fh_stream_t stream);

/*
 * Sampled next token: probes drawn without replacement with probabilities
 * softmax(h.C/T) over the raw centroids, then one token drawn from
 * softmax(logit/T) over the candidates (flash_head.py:202-211, :326-328).
 * Randomness is Philox-4x32-10 keyed by (seed, offset, row, id); rows are
 * independent draws. Replaces get_next_token(h, do_sample=True, temperature).
 */
FH_API int fh_get_next_token_sample(const fh_head *head, const void *hidden,
                                    int rows, float temperature, uint64_t seed,
                                    uint64_t offset, int64_t *out_ids,
                                    void *workspace, size_t workspace_bytes,
                                    fh_stream_t stream);

/*
 * Stage 1 only: probed clusters [rows, n_probes] (int32, ascending cluster id)
 * and optionally the stage-1 scores [rows, K] (fp32; in sampling mode the
 * Gumbel-perturbed keys). Replaces FlashHead._get_top_clusters
 * (flash_head.py:190-221).
 */
FH_API int fh_top_clusters(const fh_head *head, const void *hidden, int rows,
                           int do_sample, float temperature, uint64_t seed,
                           uint64_t offset, int32_t *out_probes,
                           float *out_scores, void *workspace,
                           size_t workspace_bytes, fh_stream_t stream);

/*
 * Stage-1 scores only: out_scores [rows, K] fp32 = h . cluster_w^T (times the
 * fp8 row scale); in sampling mode the Gumbel-perturbed keys
 * h . centroid_w^T / T + G. Replaces the reference's cluster_linear(h)
 * (flash_head.py:213) / F.linear(h, centroids.t()) (:203-205). Needs no
 * workspace.
 */
FH_API int fh_cluster_scores(const fh_head *head, const void *hidden, int rows,
                             int do_sample, float temperature, uint64_t seed,
                             uint64_t offset, float *out_scores,
                             fh_stream_t stream);

/*
 * Stage 2 only, for given probe lists probes [rows, n_probes] (int32 cluster
 * ids; ids outside [0, K) are skipped): out_ids[rows]. The head's
 * block_sparse_argmax_atomic (fused.py:167-188) plus its special tokens, or
 * the within-candidate sample when do_sample != 0. Unlike the other entry
 * points this one does not reset the workspace's accumulator first: the
 * workspace must be zero-filled before its first use (and after a failed
 * call); every completed call leaves it zeroed.
 */
FH_API int fh_stage2_next_token(const fh_head *head, const void *hidden,
                                int rows, const int32_t *probes, int do_sample,
                                float temperature, uint64_t seed,
                                uint64_t offset, int64_t *out_ids,
                                void *workspace, size_t workspace_bytes,
                                fh_stream_t stream);

/*
 * Full-vocabulary next token over w_perm (greedy, or sampled at temperature
 * when do_sample != 0). Replaces the dense branch of get_next_token for
 * hidden_states.shape[0] > 10 (flash_head.py:292-301). Calls of 16+ rows run
 * one tcgen05 GEMM kernel per 256 rows with the argmax (or, sampling, the
 * Gumbel-max) in its epilogue, so the logits stay on chip; fewer rows run the
 * block-sparse stage 2 over every cluster.
 * Ties go to the smallest vocab id; logits are f32 sums of the 16-bit
 * products, so ids equal the exact argmax up to f32 rounding of near-ties.
 */
FH_API int fh_dense_next_token(const fh_head *head, const void *hidden,
                               int rows, int do_sample, float temperature,
                               uint64_t seed, uint64_t offset,
                               int64_t *out_ids, void *workspace,
                               size_t workspace_bytes, fh_stream_t stream);

/*
 * Stateless block-sparse kernels with the reference's argument layout
 * (fused.py). hs [T, D] (dtype), w_perm [K*cap*D] (dtype), ci [T, P] int64
 * cluster ids, vocab_maps [K*cap] int64. Cluster ids outside [0, K) are
 * skipped; a row left without candidates yields 4294967295, as the
 * reference's sentinel unpacks.
 */
/* fused.py:82-93: out [T, P*cap] logits (dtype). */
FH_API int fh_block_sparse_logits(const void *hs, int T, int D,
                                  const void *w_perm, const int64_t *ci, int P,
                                  int n_clusters, int cluster_size, int dtype,
                                  void *out, fh_stream_t stream);
/* fused.py:96-116: out_max [T, P] (dtype), out_vocab [T, P] int64. */
FH_API int fh_block_sparse_logits_argmax(const void *hs, int T, int D,
                                         const void *w_perm, const int64_t *ci,
                                         int P, const int64_t *vocab_maps,
                                         int n_clusters, int cluster_size,
                                         int dtype, void *out_max,
                                         int64_t *out_vocab,
                                         fh_stream_t stream);
/*
 * Speculative decoding with FlashHead ids (replaces the per-element host loop
 * of the reference's RejectionSampler hook, patches/rejection_sampler.py:55-76).
 * Per request b (batch requests, drafts draft_ids[cu[b-1] .. cu[b]) with
 * cu = cu_num_draft, an inclusive prefix sum, int32 on the device):
 * out_ids[b, j] = draft token j while it equals target_ids at the same flat
 * position; the first mismatch writes the target's token there and ends the
 * row; when every draft is accepted, bonus_ids[b] goes to position n (also
 * for n = 0, as vLLM's rejection sampler does; the reference's loop leaves
 * such rows empty). Other positions hold `placeholder`. out_ids is
 * [batch, max_spec_len + 1] int32; max_spec_len 0..4096.
 */
FH_API int fh_spec_accept(const int32_t *draft_ids, const int32_t *target_ids,
                          const int32_t *bonus_ids, const int32_t *cu_num_draft, int batch,
                          int max_spec_len, int32_t placeholder, int32_t *out_ids,
                          fh_stream_t stream);

/* fused.py:167-188: out [T] int64 next-token ids. */
FH_API int fh_block_sparse_argmax_atomic(const void *hs, int T, int D,
                                         const void *w_perm, const int64_t *ci,
                                         int P, const int64_t *vocab_maps,
                                         int n_clusters, int cluster_size,
                                         int dtype, int64_t *out,
                                         fh_stream_t stream);

/*
 * Tensor-parallel steps (clusters partitioned across ranks; no reference
 * counterpart: the reference replicates the head on every rank,
 * loading.py:144-164). The caller moves the candidate words between ranks
 * (an all-gather and a max all-reduce, e.g. NCCL):
 *   1. fh_tp_local_candidates: local stage 1 + local top-p ->
 *      cand[rows, n_probes] packed words (mono(score) << 32 | ~global id),
 *      as int64 with the top bit flipped so signed order == unsigned order.
 *   2. all-gather cand over R ranks -> all_cand[R, rows, n_probes]
 *   3. fh_tp_select_and_score: global top-p over all_cand, stage 2 on the
 *      probes this shard owns (+ its special tokens) -> best[rows] packed
 *      (mono(logit) << 32 | ~vocab id), same int64 encoding
 *   4. max all-reduce of best over ranks
 *   5. fh_tp_finalize: best -> out_ids[rows]
 */
FH_API int fh_tp_local_candidates(const fh_head *head, const void *hidden,
                                  int rows, int do_sample, float temperature,
                                  uint64_t seed, uint64_t offset,
                                  int64_t *cand, void *workspace,
                                  size_t workspace_bytes, fh_stream_t stream);
FH_API int fh_tp_select_and_score(const fh_head *head, const void *hidden,
                                  int rows, int n_ranks,
                                  const int64_t *all_cand, int do_sample,
                                  float temperature, uint64_t seed,
                                  uint64_t offset, int64_t *best,
                                  void *workspace, size_t workspace_bytes,
                                  fh_stream_t stream);
FH_API int fh_tp_finalize(const int64_t *best, int rows, int64_t *out_ids,
                          fh_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHHEAD_H */
