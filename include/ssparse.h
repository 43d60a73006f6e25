/*
 * ssparse.h -- C ABI of libssparse.so, the sm_100a routed block-sparse attention path for
 * streaming (chunk-autoregressive) Wan-DiT video diffusion.
 *
 * Conventions shared by every entry point
 *   - Plain pointers to device memory, sizes as int / int64_t, a cudaStream_t passed as void*.
 *     No torch types cross this boundary.
 *   - The caller allocates every buffer (inputs, outputs, workspace). The library never allocates,
 *     frees or synchronises; work is enqueued on the caller's stream, so the entry points that
 *     take their buffers from the caller can be captured into a CUDA graph once
 *     ss_prepare_device() has run on that device.
 *   - Return value: 0 on success, a cudaError_t value (< 1000) if a CUDA call failed, or one of
 *     the SS_ERR_* codes below for invalid arguments (checked on the host before any launch).
 *   - Device-side faults (non-finite router score, a pipeline wait that timed out) are reported
 *     by OR-ing SS_DEV_* bits into an optional device int (`status`), which the caller reads when
 *     it chooses to synchronise. Kernels never trap.
 *   - Layouts: one batch element (B = 1, as in the reference); token-major activations
 *     q[Lq][H][D], k/v[Lk][H][D] in bf16 with row stride H*D elements; D = 128.
 *
 * Reference interfaces replaced (paths are inside the jurky123/streaming_sparse repository):
 *   ss_router      <- project (migration/unified_router/opt8/projection.py:11-14),
 *                     prototype pooling segment (migration/unified_router/opt19/prototype.py:43-49),
 *                     block-score GEMM _coarse + top-k _top (migration/unified_router/opt16/route.py:34-55,
 *                     route() :90-113), forced-set policy (local_experiments/video_runtime_v1/
 *                     pipeline_graph.py:140-151) and fixed_page_select (local_experiments/
 *                     video_runtime_v1/fixed_page_select.py:34-41)
 *   ss_router_pool_keys, ss_router_cached <- Cache.refresh_history / Cache.current
 *                     (migration/unified_router/opt23/pipeline.py:22-34): history pooled once per
 *                     commit, the current chunk pooled per call
 *   ss_router_fast <- the tensor-core projection/score GEMM (migration/unified_router/opt8/
 *                     projection.py:4-14, `_coarse` in opt16/route.py:34-47)
 *   ss_attention   <- exact(q,k,v,ids,workspace) (local_experiments/video_runtime_v1/attention.py:15-24)
 *                     wrapping _attn_fwd (local_experiments/gap_exact_round_kernel.py:4-137), and the
 *                     sm_80 C ABI `run` (local_experiments/video_runtime_v1/csrc/fixed15_attention.cu:407-409)
 *   ss_quant_k_pages, ss_attention_i8 <- the INT8-QK path: `_quant` and `_shared` with INT8=True
 *                     (migration/unified_router/opt23/attention.py:6-58), called by the Sparge
 *                     pipeline (migration/unified_router/opt24/pipeline.py:23-25, sparge.py:38-43)
 *   ss_lse_merge   <- merge (local_experiments/video_runtime_v1/attention.py:40-45),
 *                     _merge_restore (migration/unified_router/opt21/attention.py:7-15)
 *   ss_cache_append<- the cache roll + write in CausalWanSelfAttention.forward
 *                     (wan/modules/causal_model.py:216-246) and commit_fixed15
 *                     (local_experiments/video_runtime_v1/csrc/fixed15_attention.cu:453-458)
 *   ss_cache_rope_shift <- the anchor rebase shift_temporal_ (local_experiments/anchor_rebase.py:8-18)
 *                     as applied to the cache's first frame by set_phase
 *                     (reproduction/vbench_current/phase.py:4-9)
 *   ss_qkv_norm_rope <- the fused projection hook project_cached_rotary
 *                     (wan/modules/causal_model.py:116-128, 241-246; local_experiments/
 *                     video_runtime_v1/rms_mean.py:38-72): q/k RMSNorm + RoPE, k/v into the cache
 *   ss_adaln       <- WanLayerNorm + modulation (wan/modules/causal_model.py:332, 344-345, 383)
 *                     and the affine norm3 (wan/modules/causal_model.py:285-287)
 *   ss_rms_norm    <- WanRMSNorm (wan/modules/model.py:70-86) of the cross-attention query (:172)
 *   ss_gate_residual <- the gated residual adds (wan/modules/causal_model.py:337, 348-349)
 */
#ifndef SSPARSE_H_
#define SSPARSE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* host-side argument errors */
#define SS_ERR_SHAPE 1001       /* inconsistent or unsupported sizes */
#define SS_ERR_POINTER 1002     /* null or misaligned pointer */
#define SS_ERR_WORKSPACE 1003   /* workspace too small */
#define SS_ERR_BUDGET 1004      /* extra > number of unforced blocks */
#define SS_ERR_SMEM 1005        /* the id lists do not fit the attention kernel's shared memory */
#define SS_ERR_DRIVER 1006      /* cuTensorMapEncodeTiled unavailable or failed */
#define SS_ERR_DEVICE 1007      /* current device ordinal >= SS_MAX_DEVICES */

/* Devices per process the library keeps per-device state for (ordinals 0 .. 63). */
#define SS_MAX_DEVICES 64

/* device-side status bits (OR-ed into *status) */
#define SS_DEV_NONFINITE 0x1    /* a router score was NaN or +-inf */
#define SS_DEV_TIMEOUT 0x2      /* an mbarrier wait in the attention kernel ran out of budget */
#define SS_DEV_BADID 0x4        /* a block id in the LUT was out of range */

/* Library version (major*100 + minor). */
int ss_version(void);

/* One-time per-device setup (kernel attributes such as the dynamic shared memory size).
   Call once per device before capturing any ss_* call into a CUDA graph. Idempotent. */
int ss_prepare_device(void);

/* ------------------------------------------------------------------------------------------ */
/* Router: mean-pooled query/key blocks -> per-head projections -> block scores -> top-k.       */
/* ------------------------------------------------------------------------------------------ */

/* Bytes of workspace ss_router and ss_router_cached need for these sizes (R = projection width,
 * 64 in the reference). */
int ss_router_workspace_bytes(int H, int Lq, int Lk, int R, int block, size_t *bytes);

/* Bytes of workspace ss_router_fast (and ss_router_ring with fast != 0) needs: the exact mode's
 * workspace followed by the tensor-core scores and key norms. */
int ss_router_fast_workspace_bytes(int H, int Lq, int Lk, int R, int block, size_t *bytes);

/* Route one chunk-layer.
 *   q       [Lq][H][128] bf16, the current chunk's queries (RoPE applied)
 *   k       [Lk][H][128] bf16, the visible KV window; its last Lq rows are the current chunk
 *   wq, wk  [H][128][R] fp32 per-head projections
 *   block   query/KV block size in tokens (64 or 128); last blocks may be partial
 *   sink_tokens  tokens at the start of the window that are always kept (0 = no sink)
 *   extra   number of blocks chosen by score per query block, outside the forced set
 *   ids     [H][qb][n_ids] int32 out, ascending block ids; n_ids must equal forced + extra
 *           (forced = blocks overlapping [0, sink_tokens) or [Lk-Lq, Lk))
 *   mask    [H][qb][kb] uint8 out (optional, may be NULL): 1 where a block is selected
 *   scores  [H][qb][kb] fp32 out (optional, may be NULL): the block scores
 * Scores are computed in exact fp32 with a fixed summation order (sequential token sums, one
 * divide by the valid count, fmaf in ascending index order), -0 is canonicalised to +0, and
 * ties go to the lower block index, so the ids are bit-identical to the CPU oracle. */
int ss_router(const void *q, const void *k, const float *wq, const float *wk,
              int H, int Lq, int Lk, int R, int block, int sink_tokens, int extra,
              int32_t *ids, int n_ids, uint8_t *mask, float *scores,
              void *workspace, size_t workspace_bytes, int *status, void *stream);

/* Pool and project key blocks [j0, j1) of the window k into rows j0 .. j1-1 of kh
 * [H][kh_rows][R] fp32 (kh_rows >= the window's block count), with the arithmetic of ss_router.
 * Replaces the commit-time history pooling `Cache.refresh_history`
 * (migration/unified_router/opt23/pipeline.py:22-29): the history's key blocks change only when
 * the window is committed (a new chunk, a roll, a rewrite of sink rows), so they are pooled once
 * per commit and reused by every denoising call of the chunk through ss_router_cached. */
int ss_router_pool_keys(const void *k, const float *wk, int H, int Lk, int R, int block, int j0, int j1,
                        float *kh, int kh_rows, int *status, void *stream);

/* ss_router with the first n_cached key blocks' projections taken from kh [H][kh_rows][R]
 * (written by ss_router_pool_keys or an earlier ss_router_cached on the same window rows): only
 * the query blocks and key blocks [n_cached, kb) are pooled, and their key projections are
 * written into kh rows n_cached .. kb-1. Results are bit-identical to ss_router whenever rows
 * [0, n_cached) of kh hold the projections of this window's blocks. Replaces the per-call
 * `Cache.current` pooling of the current chunk (migration/unified_router/opt23/pipeline.py:30-34).
 * k holds window rows [k_row0, Lk) (k_row0 <= n_cached * block): a rank of a KV-sharded group,
 * which stores only its own history blocks, passes the window's tail (the history rows of the
 * block the current chunk starts in, then the chunk) with the gathered history projections in kh.
 * workspace: ss_router_workspace_bytes for these sizes (only its query half is used). */
int ss_router_cached(const void *q, const void *k, int k_row0, const float *wq, const float *wk,
                     int H, int Lq, int Lk, int R, int block, int sink_tokens, int extra,
                     float *kh, int kh_rows, int n_cached,
                     int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                     void *workspace, size_t workspace_bytes, int *status, void *stream);

/* The router with its block-score GEMM on the tensor cores (tcgen05 kind::tf32, each fp32
 * operand split into a tf32 part and its remainder, three products accumulated in fp32), for
 * R = 32 or 64. The fast scores are within 2^-13 * |qh_i| * |kh_j| of the exact mode's; a query
 * block whose threshold is tied, or whose lowest selected score minus that bound does not exceed
 * the highest unselected candidate's score plus it, is scored again in exact fp32 with
 * ss_router's arithmetic, so ids and mask are bit-identical to ss_router / ss_router_cached.
 * Arguments as ss_router_cached, except:
 *   kh      may be NULL (with n_cached = k_row0 = 0): every key block pooled into the workspace
 *   scores  (optional) receives the tensor-core scores
 *   rescored (optional) device int, incremented once per query block scored again
 *   workspace  ss_router_fast_workspace_bytes for these sizes (the fast mode's scores live there too)
 * Replaces the tensor-core projection and score GEMM of the reference's Triton router
 * (migration/unified_router/opt8/projection.py:4-14, `_coarse` in migration/unified_router/
 * opt16/route.py:34-47) with its top-k (`_top`, :49-55). */
int ss_router_fast(const void *q, const void *k, int k_row0, const float *wq, const float *wk,
                   int H, int Lq, int Lk, int R, int block, int sink_tokens, int extra,
                   float *kh, int kh_rows, int n_cached,
                   int32_t *ids, int n_ids, uint8_t *mask, float *scores, int *rescored,
                   void *workspace, size_t workspace_bytes, int *status, void *stream);

/* ---- ring-buffer KV cache (O(chunk) eviction) ----------------------------------------------- *
 * A ring cache keeps the window's first S = ring_sink rows at physical rows [0, S) and the rest
 * in a ring of C = ring_cap rows at [S, S + C): window row t >= S sits at physical row
 * S + ((t - S + ring_head) mod C). A roll of the window then moves only the ring's head instead
 * of the rows. The cache also holds rows [S + C, S + C + 64) = a copy of ring rows [0, 64), and,
 * when S is not a multiple of 64, a copy of the sink's last S mod 64 rows at ring rows
 * ring_head - S mod 64 .. ring_head - 1, so that every 64-row sub-block of the window is one
 * contiguous physical range (kept by ss_cache_append_ring / ss_cache_ring_refresh). Physical rows:
 * S + C + 64; the window (Lk rows, starting at the cache's row 0) needs Lk - S + S mod 64 <= C.
 * ring_head_dev (optional, device int): where the head lives for calls captured in a CUDA graph.
 * When it is given the kernels read the head from it at run time (ring_head must still be the
 * current head, for the host checks), and ss_cache_append_ring moves it on after its copies.
 * The reference's paged store advances the same kind of cursor over whole pages
 * (`PageStore.commit`: write = sink + (end - sink) % (history_pages - sink),
 * local_experiments/review_v1/runtime.py:38-46); here it runs per token, because the frames
 * (1560 tokens) are not whole 64-token sub-blocks, and the window's block grid, and so every
 * block id, stays that of the shifted cache. */

/* ss_router_pool_keys over a ring cache k (S + C + 64 rows). */
int ss_router_pool_keys_ring(const void *k, const float *wk, int H, int Lk, int R, int block, int j0, int j1,
                             float *kh, int kh_rows, int ring_sink, int ring_cap, int ring_head,
                             const int *ring_head_dev, int *status, void *stream);

/* The router over a ring cache k: the exact mode (fast = 0, ss_router / ss_router_cached) or the
 * tensor-core mode (fast != 0, ss_router_fast), the first n_cached key blocks' projections from kh
 * when kh is not NULL. Results equal those of the same call on the shifted (contiguous) window. */
int ss_router_ring(const void *q, const void *k, const float *wq, const float *wk,
                   int H, int Lq, int Lk, int R, int block, int sink_tokens, int extra,
                   float *kh, int kh_rows, int n_cached,
                   int32_t *ids, int n_ids, uint8_t *mask, float *scores, int *rescored, int fast,
                   int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev,
                   void *workspace, size_t workspace_bytes, int *status, void *stream);

/* Bytes of the static device array used by ss_router_noalloc (8 MiB per device that loads the
   library, held until the process exits). */
#define SS_ROUTER_STATIC_SCRATCH_BYTES (8u << 20)

/* ss_router for callers that cannot allocate device memory: no workspace argument and no
 * allocation. This entry point has no counterpart in the reference (whose router ops allocate
 * their intermediates through torch). It serves hosts whose device memory is handed out by their
 * own fixed pool (so a cudaMalloc or a torch allocation per call is unavailable or fails), and
 * hosts binding the library from a language that has no device allocator of its own.
 *   - The intermediates (ss_router_workspace_bytes for these sizes) live in one static device
 *     array of SS_ROUTER_STATIC_SCRATCH_BYTES per device; larger problems return
 *     SS_ERR_WORKSPACE before anything is launched (about 4.9 MB at a 98 280-token window with
 *     12 heads and 64-token blocks).
 *   - The first call on a device looks up that device's address of the array
 *     (cudaGetSymbolAddress, with the device current); make that first call before capturing
 *     any stream on that device. The address is kept per (device, CUDA context): after
 *     cudaDeviceReset the next call sees a new context and looks the address up again, so that
 *     call, too, must come before any capture.
 *   - All calls on a device share the array: calls that overlap on the GPU (different streams
 *     or host threads) race, so the caller serialises them. Nothing in the array needs to start
 *     at zero: a call that completes writes every value it reads.
 *   - Whenever *status comes back non-zero, ids, mask and scores of that call are undefined:
 *     a pooling wait that timed out leaves projections unwritten, and the scoring then reads the
 *     previous call's values from the shared array.
 *   - Device ordinals >= SS_MAX_DEVICES are refused with SS_ERR_DEVICE.
 * Other arguments, results and status codes are those of ss_router. */
int ss_router_noalloc(const void *q, const void *k, const float *wq, const float *wk,
                      int H, int Lq, int Lk, int R, int block, int sink_tokens, int extra,
                      int32_t *ids, int n_ids, uint8_t *mask, float *scores, int *status,
                      void *stream);

/* ------------------------------------------------------------------------------------------ */
/* Block-sparse attention (tcgen05 / TMEM / TMA, sm_100a).                                     */
/* ------------------------------------------------------------------------------------------ */

/* out[t][h][:] = softmax(q[t,h,:] . K_sel^T * scale) V_sel over the valid tokens of the blocks
 * listed for t's query block in ids[h][t / block][0..n_ids) (ascending or not; entries < 0 are
 * ignored). out_dtype: 0 = bf16, 1 = fp32. lse (optional): [H][Lq] fp32 natural-log
 * log-sum-exp of the scaled scores. q, k, v 16-byte aligned and out 32-byte aligned
 * (SS_ERR_POINTER otherwise). */
int ss_attention(const void *q, const void *k, const void *v, const int32_t *ids,
                 int H, int Lq, int Lk, int block, int n_ids, float scale,
                 void *out, int out_dtype, float *lse, int *status, void *stream);

/* Largest n_ids ss_attention accepts for these sizes (its block lists live in shared memory). */
int ss_attention_max_ids(int Lk, int block, int *max_ids);

/* ss_attention with a caller workspace that balances a problem of one to two tiles per SM, or of
 * half a tile per SM or less: when the 128-row tiles (ceil(Lq/128) * H) are at least as many as
 * the SMs and fewer than twice as many, or at most half as many (and long enough that a piece
 * keeps 8 steps), each CTA takes an equal share of the tiles' work, a tile shared by several CTAs is cut at its step list, every piece leaves
 * its normalised partial and LSE in the workspace, and a second kernel merges the pieces (the
 * arithmetic of ss_lse_merge). Larger problems run exactly as ss_attention. Same arguments and
 * results as ss_attention (within fp32 rounding of the merge for split tiles). workspace:
 * ss_attention_workspace_bytes bytes (0 = this size never splits), 256-byte aligned; it keeps
 * nothing between calls. No counterpart in the reference (its kernel launches one program per
 * query block and page group). */
int ss_attention_workspace_bytes(int H, int Lq, size_t *bytes);
int ss_attention_ws(const void *q, const void *k, const void *v, const int32_t *ids,
                    int H, int Lq, int Lk, int block, int n_ids, float scale,
                    void *out, int out_dtype, float *lse, int *status,
                    void *workspace, size_t workspace_bytes, void *stream);

/* ss_attention_ws over a ring cache k, v (S + C + 64 rows each; see ss_router_ring). */
int ss_attention_ring(const void *q, const void *k, const void *v, const int32_t *ids,
                      int H, int Lq, int Lk, int block, int n_ids, float scale,
                      void *out, int out_dtype, float *lse, int *status,
                      int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev,
                      void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------------ */
/* INT8-QK block-sparse attention (the reference's SpargeAttn-style path).                      */
/* ------------------------------------------------------------------------------------------ */

/* Quantise the key pages [p0, p1) of the window k [Lk][H][128] bf16 (page p = tokens
 * [64p, 64p + 64), the last page possibly partial): per page and head, scale = max(max|k| / 127,
 * 1e-10) in fp32 and k_i8 = round-half-even(k / scale) (IEEE divide) into k_i8 [Lk][H][128] int8,
 * the scale into ks [H][ceil(Lk/64)] fp32. Replaces `_quant` / `Quantized.history` / `.current`
 * (migration/unified_router/opt23/attention.py:6-28): history pages are quantised once per commit,
 * the pages the current chunk touches per call. k and k_i8 16-byte aligned. */
int ss_quant_k_pages(const void *k, int H, int Lk, int p0, int p1, int8_t *k_i8, float *ks, void *stream);

/* ss_attention with the scores taken in int8: q [Lq][H][128] bf16 is quantised per 32-row group
 * and head inside the kernel (the scale rule of ss_quant_k_pages), the logits are the exact int32
 * dot products with k_i8 times (q scale * ks[page]) times scale * log2(e) (fp32, rounded after each
 * product), softmax in base 2, P rounded to bf16 for the P.V product (fp32 accumulation), v bf16.
 * ids, block, n_ids, out (0 = bf16, 1 = fp32), lse (natural log, optional) and status as in
 * ss_attention; out, q, k_i8, v 16-byte aligned; at most 4096 pages (Lk <= 262144). Replaces the
 * INT8 attention of migration/unified_router/opt23/attention.py:30-58 (`_shared`, INT8=True) and
 * the Sparge call of opt24/sparge.py:38-43 / opt24/pipeline.py:23-25. Plain windows (ring caches:
 * ss_attention_i8_ring).
 * workspace (optional, 256-byte aligned, ss_attention_i8_workspace_bytes bytes; NULL = none): when
 * the 128-row tiles would leave a partial wave (two CTAs per SM), each tile's step list is cut into
 * 2-4 equal pieces whose normalised partials and LSEs go to the workspace and are combined by the
 * arithmetic of ss_lse_merge (results equal within fp32 rounding of the merge); it keeps nothing
 * between calls. */
int ss_attention_i8_workspace_bytes(int H, int Lq, size_t *bytes);
int ss_attention_i8(const void *q, const int8_t *k_i8, const float *ks, const void *v, const int32_t *ids,
                    int H, int Lq, int Lk, int block, int n_ids, float scale,
                    void *out, int out_dtype, float *lse, int *status,
                    void *workspace, size_t workspace_bytes, void *stream);

/* The INT8-QK path over a ring cache (ring arguments as in ss_router_ring): k (bf16), k_i8 and v
 * hold the ring's physical rows (S + C + 64 each); a page is a 64-row range of window rows, which
 * the ring keeps contiguous, so its int8 rows sit where its bf16 rows sit. Same results, bit for
 * bit, as the plain-window calls on the same window. Replaces the same reference code as the plain
 * entry points, over the ring cursor of local_experiments/review_v1/runtime.py:38-46. */
int ss_quant_k_pages_ring(const void *k, int H, int Lk, int p0, int p1, int8_t *k_i8, float *ks,
                          int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev, void *stream);
int ss_attention_i8_ring(const void *q, const int8_t *k_i8, const float *ks, const void *v, const int32_t *ids,
                         int H, int Lq, int Lk, int block, int n_ids, float scale,
                         void *out, int out_dtype, float *lse, int *status,
                         int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev,
                         void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------------ */
/* Log-sum-exp merge of partial attention results.                                             */
/* ------------------------------------------------------------------------------------------ */

/* o_parts [P][Lq][H][128] fp32, lse_parts [P][H][Lq] fp32 (natural log; -inf = empty part).
 * out [Lq][H][128] (out_dtype 0 = bf16, 1 = fp32) = sum_p exp(lse_p - L) o_p with
 * L = logsumexp_p lse_p; lse_out [H][Lq] (optional) = L. */
int ss_lse_merge(const float *o_parts, const float *lse_parts, int P, int H, int Lq,
                 void *out, int out_dtype, float *lse_out, void *stream);

/* ------------------------------------------------------------------------------------------ */
/* KV-block sharding across the GPUs of a node: partials merged over peer memory.              */
/* ------------------------------------------------------------------------------------------ */
/* With the window split block-cyclically over P ranks (one GPU each), every rank attends over its
 * own blocks (ss_attention with lse) and the partials are combined by the LSE merge of
 * ss_lse_merge. These entry points do that combine with the partials left where they were
 * written: each rank opens the others' buffers once (CUDA IPC), and per call a flag barrier makes
 * the partials visible, then one kernel reads all P of them through peer pointers and writes the
 * merged rows. No counterpart in the reference, whose runtime runs one video per GPU
 * (local_experiments/video_runtime_v1/batch.py:29-37) and merges splits inside one GPU
 * (migration/unified_router/opt21/attention.py:7-15). The caller allocates every buffer. */

#define SS_MAX_PEERS 8
#define SS_IPC_HANDLE_BYTES 64

/* Export the allocation holding device pointer ptr: handle (SS_IPC_HANDLE_BYTES bytes) and the
   offset of ptr inside that allocation, to be sent to the other processes of the node. */
int ss_ipc_handle(const void *ptr, void *handle, size_t *offset);
/* Map another process's exported allocation into the current device's context (peer access
   enabled); *ptr = mapped base + offset. */
int ss_ipc_open(const void *handle, size_t offset, void **ptr);
/* Unmap a pointer returned by ss_ipc_open (same offset). */
int ss_ipc_close(void *ptr, size_t offset);

/* flags: P device pointers (flags[p] = rank p's int array of >= P entries, zeroed before first
 * use, the others opened with ss_ipc_open); epoch: this rank's device int counter (zeroed before
 * first use), advanced by one per call on the device, so a call captured in a CUDA graph posts a
 * new epoch at every replay. Posts the epoch into slot `rank` of every rank's array, then waits
 * until this rank's slots 0..P-1 all hold it or a later one. Every rank makes the same number of
 * calls. Writes enqueued before the barrier on each rank are visible to every rank's work
 * enqueued after it. A wait that runs out (about 2 s) sets SS_DEV_TIMEOUT in *status instead of
 * hanging. */
int ss_peer_barrier(int *const *flags, int rank, int P, int *epoch, int *status, void *stream);

/* Rows [row0, row1) of out [Lq][H][128] (out_dtype 0 = bf16, 1 = fp32) =
 * sum_p exp(lse_p - L) o_p with L = logsumexp_p lse_p, where o_parts[p] is part p's [Lq][H][128]
 * output (part_dtype 0 = bf16, 1 = fp32) and lse_parts[p] its [H][Lq] natural-log LSE (-inf = the
 * part saw no token), both device pointers that may live on other GPUs (ss_ipc_open); the o_parts
 * and out 16-byte aligned. lse_out [H][Lq] (optional) receives L for those rows.
 * P <= SS_MAX_PEERS. Arithmetic of ss_lse_merge (the same values, bit for bit). */
int ss_lse_merge_peers(const void *const *o_parts, const float *const *lse_parts, int P, int part_dtype,
                       int H, int Lq, int row0, int row1, void *out, int out_dtype, float *lse_out,
                       void *stream);

/* KV-block sharding with the exchange fused into the kernels. Rank `slot` of P stores the window
 * blocks j with j % P == slot, packed in order into its k, v (Lk rows: local block j / P); ids
 * are the window's block ids as the router gives them (every rank the same), and the kernel keeps
 * this rank's. It attends over them (ss_attention_ws arguments) and its epilogue stores each partial row straight into
 * the buffers of the rank that owns the row: row t belongs to rank d = t / rows (rows * P >= Lq)
 * and goes to o_parts[d] [P][rows][H][128] (part_dtype 0 = bf16, 1 = fp32; 32-byte aligned) at
 * [slot][t - d * rows], its natural-log LSE to lse_parts[d] [P][H][rows] at [slot][h][t - d *
 * rows] (-inf where the rank saw no token). o_parts / lse_parts: every rank's buffers, this
 * rank's own and the others' opened with ss_ipc_open. After a ss_peer_barrier, rank d merges its
 * rows from its own memory with ss_lse_merge_gather. */
int ss_attention_kv_parts(const void *q, const void *k, const void *v, const int32_t *ids,
                          int H, int Lq, int Lk, int block, int n_ids, float scale,
                          void *const *o_parts, float *const *lse_parts, int P, int rows, int slot,
                          int part_dtype, int *status, void *workspace, size_t workspace_bytes,
                          void *stream);

/* ss_lse_merge_peers whose merged rows are stored into each of outs[0 .. n_out) (device pointers,
 * this GPU's or peers', 16-byte aligned; row r of the parts goes to row r of every outs[d]), so a
 * rank merging the rows it owns also delivers them to every rank. n_out <= SS_MAX_PEERS.
 * flags (optional, NULL = none): the merge is first preceded by the barrier of ss_peer_barrier
 * over the P ranks (flags, rank, epoch, status as there), so that the partials the peers pushed
 * before it are visible: one warp posts the epoch, and the merge's CTAs wait for the peers'
 * posts before they read. With row0 == row1 only the barrier runs. */
int ss_lse_merge_gather(const void *const *o_parts, const float *const *lse_parts, int P, int part_dtype,
                        int H, int Lq, int row0, int row1, void *const *outs, int n_out, int out_dtype,
                        int *const *flags, int rank, int *epoch, int *status, void *stream);

/* Head sharding: ss_attention_ws over this rank's H heads (global heads h0 .. h0 + H - 1 of
 * out_heads) whose output rows go straight into all P ranks' [Lq][out_heads][128] buffers
 * (outs[p], this rank's own and the others' opened with ss_ipc_open; out_dtype 0 = bf16, 1 =
 * fp32; 32-byte aligned): row t of local head h is stored at element ((t * out_heads) + h0 + h) *
 * 128 of every outs[p], by the attention kernel's epilogue (and the split merge), so the
 * all-gather of the heads' outputs travels over NVLink inside the attention instead of after it.
 * lse (optional) is this rank's [H][Lq]. After a ss_peer_barrier on every rank, each rank's buffer
 * holds every head's rows. 1 <= P <= SS_MAX_PEERS, 0 <= h0, h0 + H <= out_heads. ring_cap > 0:
 * k, v are a ring cache of this rank's heads (as ss_attention_ring); ring_cap = 0: the window's
 * rows in order (the other ring arguments ignored). Replaces, per
 * rank, the reference's attention(q, k, v) call of the patched model
 * (self_forcing_adapter.py:109) on a head slice plus an all-gather of the slices. */
int ss_attention_heads(const void *q, const void *k, const void *v, const int32_t *ids,
                       int H, int Lq, int Lk, int block, int n_ids, float scale,
                       void *const *outs, int P, int out_heads, int h0, int out_dtype, float *lse,
                       int *status, int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev,
                       void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------------ */
/* KV cache append / evict.                                                                    */
/* ------------------------------------------------------------------------------------------ */

/* Apply one chunk write to a [cap][H][128] bf16 K/V cache with the rolling-window semantics of
 * CausalWanSelfAttention (sink kept, oldest non-sink tokens evicted by a left shift):
 *   local_attn      nonzero if the model uses a local window (eviction enabled)
 *   global_end, local_end  the cache's index state before the write
 *   current_start, n_new   the chunk's absolute start token and length
 *   sink_tokens     sink length in tokens
 *   k_new, v_new    [n_new][H][128] bf16 with token stride new_stride (elements)
 *   out_local_end   receives the new local end index (the window is [max(0,end-W), end))
 * The shift moves rows in chunks no longer than the eviction distance, so it never reads a row
 * that an earlier chunk of the same call has overwritten. All stores are 16-byte vectors. */
int ss_cache_append(void *k_cache, void *v_cache, int cap, int H,
                    const void *k_new, const void *v_new, int64_t new_stride, int n_new,
                    int local_attn, int64_t global_end, int64_t local_end,
                    int64_t current_start, int sink_tokens, int64_t *out_local_end,
                    void *stream);

/* ss_cache_append on a ring cache (see ss_router_ring): the same window, index arithmetic and
 * results, but a roll moves the ring's head by the evicted row count instead of shifting the
 * window's rows, so a call writes only the chunk's n_new rows, their copies among the mirrored
 * rows, and the sink's last S mod 64 rows before the new head. cap = the window's capacity in
 * rows (the cache holds sink_tokens + ring_cap + 64 physical rows), ring_cap >= cap -
 * sink_tokens + sink_tokens mod 64. *out_ring_head receives the head after the call. */
int ss_cache_append_ring(void *k_cache, void *v_cache, int cap, int H,
                         const void *k_new, const void *v_new, int64_t new_stride, int n_new,
                         int local_attn, int64_t global_end, int64_t local_end,
                         int64_t current_start, int sink_tokens, int ring_cap, int ring_head, int *ring_head_dev,
                         int64_t *out_local_end, int *out_ring_head, void *stream);

/* Rewrite the copy of the sink's last sink_tokens mod 64 rows before the ring's head (and its
 * mirrored rows), after the sink rows changed outside ss_cache_append_ring (an anchor rebase). */
int ss_cache_ring_refresh(void *k_cache, void *v_cache, int H, int sink_tokens, int ring_cap, int ring_head,
                          const int *ring_head_dev, void *stream);

/* After a ring write placed by the device head (ss_qkv_norm_rope_ring): when the write rolled
 * (evicted > 0) or wrote sink rows (refresh != 0), the sink's last sink_tokens mod 64 rows are
 * repeated before the head after the roll; then the head moves on by evicted. */
int ss_cache_ring_commit(void *k_cache, void *v_cache, int H, int sink_tokens, int ring_cap,
                         int *ring_head_dev, int evicted, int refresh, void *stream);

/* Rotate the first `pairs` complex pairs (elements 2p, 2p+1) of every head of rows [0, n) of a
 * key tensor [n][H][128] bf16 by phase[p] = (cos, sin) (float64 [pairs][2], device memory):
 * float64 products and sums, then double -> float -> bf16. src rows at stride src_ld elements,
 * dst rows at dst_ld; dst may equal src (in place); when it does not, the rows are copied first
 * so the other pairs come through unchanged. Used to re-rotate a snapshot of the anchor (sink)
 * frame's keys to a new temporal position. */
int ss_cache_rope_shift(const void *src, int64_t src_ld, void *dst, int64_t dst_ld, int n, int H,
                        int pairs, const double *phase, void *stream);

/* ---- per-token kernels of the DiT layer around the attention (one CTA per token row) ---- */

/* q/k/v rows of one chunk from a fused [n][>= 3*d] projection (q at column 0, k at d, v at 2d;
 * d = H*128; row stride qkv_ld elements). For q and k: RMSNorm over the d columns (fp32 mean of
 * squares, + eps, rsqrt), rounded to bf16, times the bf16 norm weight (rounded), then rotated
 * pairwise (2i, 2i+1) by the row's table cos_t/sin_t [n][64] fp32 (pair index = column % 128 / 2).
 * q goes to q_out (row stride q_ld); k and the untouched v go to k_out / v_out (row stride kv_ld),
 * which may be the cache rows the chunk occupies. All pointers 16-byte aligned, strides multiples
 * of 8 elements, d/8 <= 1024. */
int ss_qkv_norm_rope(const void *qkv, int64_t qkv_ld, int n, int H, const void *norm_q,
                     const void *norm_k, float eps, const float *cos_t, const float *sin_t,
                     void *q_out, int64_t q_ld, void *k_out, void *v_out, int64_t kv_ld,
                     void *stream);

/* ss_qkv_norm_rope writing k and v into a ring-buffer cache (see ss_router_ring): row r goes to
 * the physical row of window row t0 + r with the head (*ring_head_dev + evicted) mod C, the head
 * after this write's roll, and once more among the mirrored rows when its ring row is below 64.
 * Follow it with ss_cache_ring_commit (same evicted). */
int ss_qkv_norm_rope_ring(const void *qkv, int64_t qkv_ld, int n, int H, const void *norm_q,
                          const void *norm_k, float eps, const float *cos_t, const float *sin_t,
                          void *q_out, int64_t q_ld, void *k_cache, void *v_cache, int64_t kv_ld,
                          int ring_sink, int ring_cap, int64_t t0, const int *ring_head_dev, int evicted,
                          void *stream);

/* Head sharding: ss_qkv_norm_rope (ring_cap = 0) or ss_qkv_norm_rope_ring (ring_cap > 0) over
 * the H heads of qkv -- the RMSNorm still over the whole width H*128 -- writing only heads h0 ..
 * h0 + nh - 1: to q_out [n][nh][128] (row stride q_ld) and to k/v rows of nh heads (row stride
 * kv_ld), so a rank's cache holds its own heads only. */
int ss_qkv_norm_rope_heads(const void *qkv, int64_t qkv_ld, int n, int H, const void *norm_q,
                           const void *norm_k, float eps, const float *cos_t, const float *sin_t, int h0, int nh,
                           void *q_out, int64_t q_ld, void *k_out, void *v_out, int64_t kv_ld,
                           int ring_sink, int ring_cap, int64_t t0, const int *ring_head_dev, int evicted,
                           void *stream);

/* LayerNorm of the n rows of x [n][d] bf16 (no affine, fp32 statistics, rounded to bf16), then
 * EITHER modulation with the row's frame f = row / frame_tokens:
 *     out = bf16(ln * (1 + scale[f*mod_ld + c]) + shift[f*mod_ld + c])   (shift/scale fp32)
 * OR affine: out = bf16(((x - mean) * rstd) * weight + bias) (weight/bias bf16 [d]).
 * Exactly one of (shift, scale) and (weight, bias) is given. d a multiple of 8, d/8 <= 1024. */
int ss_adaln(const void *x, int n, int d, int frame_tokens, const float *shift, const float *scale,
             int64_t mod_ld, const void *weight, const void *bias, float eps, void *out,
             void *stream);

/* out [n][d] bf16 = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight), x rows at stride x_ld,
 * weight bf16 [d]. */
int ss_rms_norm(const void *x, int64_t x_ld, int n, int d, const void *weight, float eps, void *out,
                void *stream);

/* In place on x [n][d] bf16 (contiguous rows): x = bf16(x + bf16(y * gate[f])) with
 * f = row / frame_tokens and gate fp32 rows of stride gate_ld, or x = bf16(x + y) when gate is
 * NULL. y rows at stride y_ld elements. */
int ss_gate_residual(void *x, const void *y, int64_t y_ld, int n, int d, int frame_tokens,
                     const float *gate, int64_t gate_ld, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SSPARSE_H_ */
