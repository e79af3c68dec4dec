/*
 * spa_b200.h -- C ABI of the B200 (sm_100a) sparse paged-attention library.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t, enqueues
 * its work on that stream and returns immediately (no host synchronisation).  No
 * function allocates device memory; callers pass a workspace when one is needed
 * and query its size first.  Return value: SPA_OK (0) or a spa_status code.
 *
 * The reference (divagr18/attention) is Python + Triton; each function below names
 * the reference function or Triton launch it replaces.
 */
#ifndef SPA_B200_H
#define SPA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* spa_stream_t; /* same type as cudaStream_t */

typedef enum {
  SPA_OK = 0,
  SPA_ERR_INVALID = 1,     /* bad shape, pointer, alignment or argument */
  SPA_ERR_UNSUPPORTED = 2, /* valid request the library does not implement */
  SPA_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  SPA_ERR_WORKSPACE = 4,   /* workspace pointer missing or too small */
  SPA_ERR_TIMEOUT = 5      /* a bounded device-side wait gave up */
} spa_status;

typedef enum { SPA_F32 = 0, SPA_F16 = 1, SPA_BF16 = 2 } spa_dtype;

/*
 * Where the K/V rows of a (sequence b, kv head h, token t) live.  A "row" is the
 * head_dim contiguous elements of one token of one head.  Row index:
 *
 *   page = page_table ? page_table[b * table_stride + t / page_size] : t / page_size
 *   row  = b * batch_stride_rows + page * page_stride_rows
 *        + h * head_stride_rows + t % page_size
 *
 * Shared page pool [num_pages, Hkv, P, D]:   batch_stride_rows = 0,
 *     page_stride_rows = Hkv * P, head_stride_rows = P, page_table = [B, max_pages].
 * Reference contiguous layout [B, H, L, D] (triton_paged_attention.py:56,139):
 *     batch_stride_rows = H * L, page_stride_rows = P, head_stride_rows = L,
 *     page_table = NULL.
 * k and v share the layout.  total_rows bounds every row the kernels may touch.
 */
typedef struct {
  const void* k;
  const void* v;
  int64_t total_rows;
  int64_t batch_stride_rows;
  int64_t page_stride_rows;
  int64_t head_stride_rows;
  const int32_t* page_table;
  int32_t table_stride;
  int32_t page_size;
} spa_kv_layout;

/* Library version and build information (NUL-terminated, static storage). */
const char* spa_version(void);

/* CUDA runtime error text of the last call in this host thread that returned
 * SPA_ERR_CUDA ("" if none); static storage. */
const char* spa_last_error(void);

/* Reads and clears the library's device-side error word on the current device
 * (nonzero after a bounded wait gave up or a kernel saw an invalid page id).  Bits:
 * 1 a bounded wait gave up, 2 an invalid page id was skipped, 4 an embedding row id
 * outside its table (spa_embed_rms_norm).
 * Synchronises the current device.  Returns SPA_OK or SPA_ERR_CUDA. */
int spa_device_error(uint32_t* out_flags);

/* Copies `bytes` from src to dst on `stream` with a kernel (16-byte accesses when
 * both pointers and the size are multiples of 16).  Meant for small transfers
 * between device memory and mapped pinned host memory, where a kernel's loads and
 * stores cost less latency than a copy-engine transfer.  The kernel is launched as a
 * programmatic dependent of the previous kernel on the stream and waits for it
 * before reading.  No reference counterpart (the reference moves tensors with
 * torch copies).  Returns SPA_OK, SPA_ERR_INVALID or SPA_ERR_CUDA. */
int spa_copy(void* dst, const void* src, size_t bytes, spa_stream_t stream);

/* Device address of pinned, mapped host memory (cudaHostGetDevicePointer; equal to
 * the host address under unified addressing), for kernels that read their inputs
 * from, or write results to, host memory directly.  SPA_ERR_INVALID when `host` is
 * not such memory. */
int spa_host_device_pointer(void* host, void** device);

/*
 * Page summaries: summary[b, h, g, :] = mean of K rows of logical page g of
 * sequence b, kv head h, for g < n_pages (the routable, historical pages).
 * Accumulated in fp64 in token order, stored fp32.  Optional superblock
 * summaries: super[b, h, s, :] = mean of K over pages [s*superblock,
 * min((s+1)*superblock, n_pages)), accumulated in fp64 from the page sums.
 * Replaces: keys[:, :, :hist].view(B,H,hist/P,P,D).mean(3)
 *   (triton_paged_gather_decode_benchmark.py:61, triton_paged_decode_benchmark.py:71).
 * page_sums64: workspace of B*Hkv*n_pages*D doubles (required when super != NULL).
 */
int spa_summaries_build(const spa_kv_layout* kv, int batch, int kv_heads,
                        int head_dim, int dtype, int n_pages, float* summaries,
                        int superblock, float* super_summaries,
                        double* page_sums64, spa_stream_t stream);

/*
 * Router: score[b, g] = scale * mean_h (q[b, h, :] . summary[b, h / group, g, :])
 * in fp32 with one fixed summation order, then the top_m pages by descending
 * score, ties to the lower page index, written as int64 [B, top_m] in
 * descending-score order.  Optional scores_out: fp32 [B, n_pages].
 * Requires q_heads / kv_heads <= 16.
 * Replaces: select_blocks (triton_paged_gather_decode_benchmark.py:16-17,
 *   triton_promotion_cache_benchmark.py:16-17) and the routing half of
 *   paged_candidates (triton_paged_decode_benchmark.py:29-30).
 */
int spa_router_topm(const void* q, int q_dtype, int batch, int q_heads,
                    int kv_heads, int head_dim, const float* summaries,
                    int n_pages, double scale, int top_m, int64_t* selected,
                    float* scores_out, spa_stream_t stream);

/*
 * Two-level (tree) router: score superblocks with super_summaries, keep the
 * top_super, then score only the pages inside them with page summaries and keep
 * top_m.  Same scoring, ordering and tie rule as spa_router_topm.
 * Replaces the block->token hierarchy of hierarchical_retrieval
 *   (benchmark_decode_attention.py:58-67) with superblock->page levels.
 */
int spa_router_tree_topm(const void* q, int q_dtype, int batch, int q_heads,
                         int kv_heads, int head_dim,
                         const float* super_summaries, int n_super,
                         const float* summaries, int n_pages, int superblock,
                         int top_super, double scale, int top_m,
                         int64_t* selected, spa_stream_t stream);

/*
 * Periodic causal router for prefill: for every update position
 * p_u = (u+1)*router_stride - 1 (u < seq_len / router_stride) and head h, scores the
 * blocks g with (g+1)*block_size - 1 <= p_u by q[b,h,p_u] . summary[b,h,g] (fp32,
 * fixed order), keeps the top_m (ties to the lower block) in descending order and
 * pads unfilled slots with -1.  q: [B, H, S, D]; summaries fp32 [B, H, n_blocks, D];
 * out int64 [B, H, U, top_m].
 * Replaces: periodic_router (triton_prefill_router_overhead.py:16-34), whose Python
 *   loop issues one topk per update position.
 */
int spa_periodic_router(const void* q, int q_dtype, int batch, int heads,
                        int seq_len, int head_dim, const float* summaries,
                        int n_blocks, int block_size, int router_stride,
                        int top_m, int64_t* out, spa_stream_t stream);

/*
 * Split-K paged decode attention.  For each sequence b and query head h
 * (kv head h / (q_heads / kv_heads)):
 *   out[b,h] = softmax(q . K_C^T * scale) V_C
 * over the candidate token set C (one softmax over all of it):
 *   selected == NULL:  C = [lo_b, ctx_b) where ctx_b = context_lens[b] and
 *                      lo_b = max(0, ctx_b - local_window) (local_window <= 0:
 *                      the whole context).
 *   selected != NULL:  C = [ctx_b - local_window, ctx_b) followed by the
 *                      top_m logical pages selected[b, :] (int64), each
 *                      page_size tokens.
 * q: [B, Hq, D]; out: [B, Hq, D] (same dtype as q).
 * Replaces: paged_decode_attention_kernel launch (triton_paged_attention.py:56-81)
 *   and paged_gather_decode_attention_kernel launch (:139-168).
 * workspace: spa_decode_workspace_size() bytes of device memory (per-split
 *   partial outputs and log-sum-exps of the global split merge; no initial
 *   contents are required).
 *   Requires batch * kv_heads <= 65536.
 */
size_t spa_decode_workspace_size(int batch, int q_heads, int kv_heads,
                                 int head_dim, int max_candidates);

int spa_paged_decode(const void* q, int dtype, int batch, int q_heads,
                     int kv_heads, int head_dim, const spa_kv_layout* kv,
                     const int32_t* context_lens, int local_window,
                     const int64_t* selected, int top_m, int max_candidates,
                     double scale, void* out, void* workspace,
                     size_t workspace_bytes, spa_stream_t stream);

/*
 * The selected-pages form of spa_paged_decode under the name of the kernel it
 * replaces, paged_gather_decode_attention (triton_paged_attention.py:139-168):
 * selected must be non-NULL and top_m > 0 (SPA_ERR_INVALID otherwise); the
 * arguments and results are those of spa_paged_decode.
 */
int spa_paged_gather_decode(const void* q, int dtype, int batch, int q_heads,
                            int kv_heads, int head_dim, const spa_kv_layout* kv,
                            const int32_t* context_lens, int local_window,
                            const int64_t* selected, int top_m,
                            int max_candidates, double scale, void* out,
                            void* workspace, size_t workspace_bytes,
                            spa_stream_t stream);

/*
 * Split plan of the tensor-core decode for this shape on the current device:
 * *nsplit CTAs per (sequence, kv head); *cluster_merge = 1 when they form one
 * thread-block cluster and merge on chip (one kernel launch), 0 when partials go
 * to the workspace and a merge kernel follows (two launches; one when nsplit = 1).
 * No reference counterpart (the reference's Triton launch has one program per
 * (batch, head), triton_paged_attention.py:74-80).
 */
int spa_decode_plan(int batch, int q_heads, int kv_heads, int max_candidates,
                    int* nsplit, int* cluster_merge);

/*
 * Span gather decode: as spa_paged_decode with selected pages, but the candidates
 * after the local window are n_spans spans of span_width consecutive tokens starting
 * at token starts[b, j] (int64; negative = empty slot; tokens at or past the context
 * are dropped).  workspace: spa_decode_workspace_size(batch, q_heads, kv_heads,
 * head_dim, local_window + n_spans * (span_width + 128)) bytes.
 * Replaces: span_gather_decode_attention_kernel launch (triton_paged_attention.py:210-224).
 */
int spa_span_gather_decode(const void* q, int dtype, int batch, int q_heads,
                           int kv_heads, int head_dim, const spa_kv_layout* kv,
                           const int32_t* context_lens, int local_window,
                           const int64_t* starts, int n_spans, int span_width,
                           double scale, void* out, void* workspace,
                           size_t workspace_bytes, spa_stream_t stream);

/*
 * One routed sparse decode step: router then gather decode.  For bf16/fp16,
 * head_dim 64 or 128, at most 8 kv heads, top_m <= 32 and a split plan that merges
 * each (sequence, kv head) pair's splits in one cluster, it is ONE kernel launch in
 * which every decode cluster scores its sequence's summaries, selects the pages
 * (the same pages, bit for bit, as spa_router_tree_topm / spa_router_topm) and
 * streams them, the local window loading meanwhile; otherwise the router and the
 * decode are enqueued as chained kernels (the decode starts while the router runs
 * and streams the local window before it reads the page ids)
 * (spa_set_step_fusion chooses).  super_summaries != NULL: two-level router
 * (spa_router_tree_topm); NULL: single level over n_pages (spa_router_topm).
 * router_scale multiplies the router score, attn_scale the attention logits.
 * selected: int64 [B, top_m] (written); out: [B, Hq, D]; workspace as for
 * spa_paged_decode with max_candidates = local_window + top_m * page_size.
 * Every input except `selected` must be complete when this call is enqueued.
 * Replaces the timed unit paged_gather_decode_attention(q, K, V,
 *   select_blocks(q, summaries, m), ...) of triton_paged_gather_decode_benchmark.py:69
 *   and triton_promotion_cache_benchmark.py:59.
 */
int spa_sparse_decode_step(const void* q, int dtype, int batch, int q_heads,
                           int kv_heads, int head_dim, const spa_kv_layout* kv,
                           const int32_t* context_lens, int local_window,
                           const float* super_summaries, int n_super,
                           const float* summaries, int n_pages, int superblock,
                           int top_super, int top_m, double router_scale,
                           double attn_scale, int64_t* selected, void* out,
                           void* workspace, size_t workspace_bytes,
                           spa_stream_t stream);

/*
 * spa_sparse_decode_step with host buffers (the per-call form of a serving loop without a
 * session): query_host, selected_host [batch, top_m] and out_host are pinned, mapped host
 * memory (cudaHostAlloc / torch pin_memory; anything else returns SPA_ERR_INVALID before a
 * launch).  A copy kernel reads the query into query_dev (device, batch*q_heads*head_dim
 * elements), the step starts during that copy and writes the output and a copy of the
 * page ids into the host buffers (selected_dev, device [batch, top_m], holds the ids the
 * decode reads).  Nothing goes through a copy engine; the results are complete on the host
 * when the stream's work is.  The reference's equivalent is the timed call of
 * triton_paged_gather_decode_benchmark.py:71 with its inputs copied in and outputs read back.
 */
int spa_sparse_decode_step_host(const void* query_host, void* query_dev, int dtype, int batch, int q_heads,
                                int kv_heads, int head_dim, const spa_kv_layout* kv, const int32_t* context_lens,
                                int local_window, const float* super_summaries, int n_super,
                                const float* summaries, int n_pages, int superblock, int top_super, int top_m,
                                double router_scale, double attn_scale, int64_t* selected_dev,
                                int64_t* selected_host, void* out_host, void* workspace, size_t workspace_bytes,
                                spa_stream_t stream);

/*
 * spa_sparse_decode_step for a chain of dependent launches (a model's decode step): the
 * first kernel is launched as a programmatic dependent of the kernel enqueued before it
 * and waits for that kernel to complete before its first read, so it is resident and
 * ready when its inputs are; kernels enqueued after it as programmatic dependents may
 * start while it runs.  Same arguments and results as spa_sparse_decode_step.  No
 * counterpart in the reference.
 */
int spa_sparse_decode_step_chained(const void* q, int dtype, int batch, int q_heads,
                                   int kv_heads, int head_dim, const spa_kv_layout* kv,
                                   const int32_t* context_lens, int local_window,
                                   const float* super_summaries, int n_super,
                                   const float* summaries, int n_pages, int superblock,
                                   int top_super, int top_m, double router_scale,
                                   double attn_scale, int64_t* selected, void* out,
                                   void* workspace, size_t workspace_bytes,
                                   spa_stream_t stream);

/*
 * spa_sparse_decode_step over a kv-head slice: one rank's (sequence, kv head)
 * shard of a decode batch.  q [B, q_heads, D] holds every query head of each
 * sequence and the summaries every one of the kv_heads kv heads (the router scores
 * with all of them, so every shard of a sequence selects the same pages); the
 * decode covers kv heads [kv_head_begin, kv_head_begin + kv_head_count), which
 * the layout kv addresses as its kv heads 0 .. kv_head_count-1, and writes out
 * [B, kv_head_count * q_heads / kv_heads, D] (those kv heads' query heads).
 * selected [B, top_m] as for spa_sparse_decode_step; workspace for
 * (B, kv_head_count * q_heads / kv_heads, kv_head_count) heads.
 * Extends spa_sparse_decode_step (same reference unit) to the multi-GPU split of a
 * batch; kv_head_begin = 0, kv_head_count = kv_heads is spa_sparse_decode_step.
 */
int spa_sparse_decode_step_heads(const void* q, int dtype, int batch, int q_heads,
                                 int kv_heads, int head_dim, int kv_head_begin,
                                 int kv_head_count, const spa_kv_layout* kv,
                                 const int32_t* context_lens, int local_window,
                                 const float* super_summaries, int n_super,
                                 const float* summaries, int n_pages,
                                 int superblock, int top_super, int top_m,
                                 double router_scale, double attn_scale,
                                 int64_t* selected, void* out, void* workspace,
                                 size_t workspace_bytes, spa_stream_t stream);

/*
 * Kernel launches one spa_sparse_decode_step (or _heads with kv_head_count kv
 * heads; <= 0: all) of this shape enqueues, with the current fusion mode and a
 * page-pool layout whose page size is page_size: 1 (the single routing +
 * decode kernel), 2 (router, decode) or 3 (router, decode, split merge).
 * No counterpart in the reference (lets a caller count kernels per step).
 */
int spa_sparse_step_launches(int dtype, int batch, int q_heads, int kv_heads,
                             int head_dim, int kv_head_count, int local_window,
                             int page_size, int top_m, int* launches);

/*
 * Step fusion switch for the library (process-wide): 1 (default) runs the steps
 * that qualify as one launch, 0 always chains the router and decode launches.
 * Returns the previous mode; other values only query it.  Both modes give the
 * same pages and the same outputs.  No counterpart in the reference (a tuning
 * and A/B switch of this library).
 */
int spa_set_step_fusion(int mode);

/*
 * Allocation-free spa_paged_decode, for callers that cannot allocate device
 * memory or pass a workspace (a serving engine that owns all of HBM through its
 * own pool, a plugin interface with no workspace argument).  No counterpart in
 * the reference, which allocates through PyTorch.
 * Same arguments and results as spa_paged_decode, minus the workspace: the
 * split-K partials go to a scratch array of SPA_DECODE_STATIC_SCRATCH_BYTES
 * compiled into the library (held in device memory of every GPU that loads it
 * until the process exits).  Returns SPA_ERR_WORKSPACE when
 * spa_decode_workspace_size() of the request exceeds that size.
 * Allocates nothing.  Every call looks up the scratch's device address in the
 * CUDA context current on the calling thread (cudaGetSymbolAddress), so it works
 * from the runtime's primary context, from a host's own driver context and after
 * a device reset alike; the first lookup in a context loads the library's device
 * code into it, so make the first call in each context before any stream capture.
 * All calls on a device share the one array: calls
 * whose kernels can overlap on the GPU (different streams, no ordering) race and
 * must be serialised by the caller.  Nothing in the array needs clearing: every
 * split writes its slot before the merge reads it.
 */
#define SPA_DECODE_STATIC_SCRATCH_BYTES (4u << 20)
int spa_paged_decode_noalloc(const void* q, int dtype, int batch, int q_heads,
                             int kv_heads, int head_dim,
                             const spa_kv_layout* kv,
                             const int32_t* context_lens, int local_window,
                             const int64_t* selected, int top_m,
                             int max_candidates, double scale, void* out,
                             spa_stream_t stream);

/*
 * KV append: writes k_new/v_new [B, Hkv, D] at token positions[b] of sequence b
 * (the row given by the layout).  Replaces the tail overwrite of
 * page_decode (triton_kvcache_transformer_decode.py:51-55).
 */
int spa_kv_append(const spa_kv_layout* kv, int dtype, int batch, int kv_heads,
                  int head_dim, const void* k_new, const void* v_new,
                  const int32_t* positions, spa_stream_t stream);

/*
 * Causal sliding-window local prefill, q/k/v/out [B, H, S, D] contiguous:
 *   out[b,h,i] = softmax_{j in [i-W+1, i]} (q_i . k_j * D^-1/2) v_j
 * Optional halo (sequence-parallel chunk): k_halo/v_halo [B, H, halo_len, D]
 * hold the halo_len keys that precede this chunk; query i then sees keys
 * i+halo_len-W+1 .. i+halo_len of the concatenation [halo ; k].
 * Only query rows [row_begin, row_end) are computed (row_end <= 0: seq_len), so
 * rows that need no halo can run while the halo is still in flight.
 * Replaces: local_causal_prefill_kernel launch (triton_local_prefill.py:61-81).
 */
int spa_local_prefill(const void* q, const void* k, const void* v, int dtype,
                      int batch, int heads, int seq_len, int head_dim,
                      int window, const void* k_halo, const void* v_halo,
                      int halo_len, int row_begin, int row_end, void* out,
                      spa_stream_t stream);

/*
 * SMs the tensor-core prefill leaves free (process-wide, default 0): its persistent
 * grid is min(work items, SMs - n).  A sequence-parallel rank sets it while its halo
 * exchange is in flight, so the exchange's copy kernels find SMs to run on beside the
 * prefill instead of waiting for its last CTA.  Returns the previous value; a negative
 * n only queries it.  No counterpart in the reference.
 */
int spa_set_prefill_sm_reserve(int n);

/*
 * Promotion cache update (one table of `slots` entries per row r < rows):
 * page[r, i] (int32, -1 = free) and last_hit[r, i] (int32).  With the row's
 * selected pages sel[r, 0..top_m) at decode step `step`:
 *   1. a selected page already present gets last_hit = step;
 *   2. entries with step - last_hit >= ttl are freed (page = -1);
 *   3. each new selected page (in selection order) takes the free slot with
 *      the lowest index, else evicts the entry with the smallest last_hit,
 *      ties to the smallest page id.
 * Requires top_m <= slots; duplicate ids in one selection count once.
 * step_dev != NULL: the step is read from that device int32 instead of `step`
 * (for calls captured once in a CUDA graph and replayed every step).
 * Replaces the host-side promoted-id swap of triton_promotion_cache_benchmark.py:53-60
 *   with a fixed-TTL policy (evaluate_promotion_ttl.py:134-135).
 */
int spa_promotion_update(int32_t* pages, int32_t* last_hit, int rows,
                         int slots, const int64_t* selected, int top_m,
                         int step, const int32_t* step_dev, int ttl,
                         spa_stream_t stream);

/*
 * Promotion refresh gate (one decision per decode step for the whole batch, on the
 * device).  Policies of evaluate_promotion_ttl.py:125-139 and train_refresh_head.py:
 *   SPA_GATE_TTL        refresh when step % ttl == 0 (step from step_dev if non-NULL)
 *   SPA_GATE_SIGNATURE  refresh when signature [batch, sig_len] (token ids) differs
 *                       from cached_signature
 *   SPA_GATE_DRIFT      refresh when mean_b (1 - cos(state[b], cached_state[b])) >
 *                       threshold (cos as torch.nn.functional.cosine_similarity)
 *   SPA_GATE_LEARNED    refresh when mean_b sigmoid(head(state[b], cached_state[b])) >=
 *                       threshold; head = Linear(4*width, hidden) (w1 [hidden, 4*width],
 *                       b1 [hidden]) -> exact GELU -> Linear(hidden, 1) (w2 [hidden], b2 [1])
 *                       over [state, cached, |state - cached|, state * cached]
 * gate[2] (device int32): gate[0] receives the decision (1 = route); gate[1] is nonzero
 * once a gated router has promoted a selection (zero it to start over: the next step
 * then always routes).  On refresh, cached_state / cached_signature (when given) take
 * the current values.  score_out (optional, device float): the batch mean compared with
 * the threshold.  States are fp32 [batch, width].
 * Replaces the host-side should_refresh logic of the reference's promotion-reuse loops.
 */
enum { SPA_GATE_TTL = 0, SPA_GATE_SIGNATURE = 1, SPA_GATE_DRIFT = 2, SPA_GATE_LEARNED = 3 };
typedef struct spa_refresh_gate_args {
  int mode;
  int batch;
  int ttl;
  int step;
  const int32_t* step_dev;
  const int64_t* signature;
  int64_t* cached_signature;
  int sig_len;
  const float* state;
  float* cached_state;
  int width;
  const float* w1;
  const float* b1;
  const float* w2;
  const float* b2;
  int hidden;
  float threshold;
  int32_t* gate;
  float* score_out;
} spa_refresh_gate_args;
int spa_refresh_gate(const spa_refresh_gate_args* args, spa_stream_t stream);

/*
 * Gated routers and step: as spa_router_topm / spa_router_tree_topm /
 * spa_sparse_decode_step, with promotion reuse.  When gate[0] == 0 and gate[1] != 0 the
 * router reads no summary and copies promoted [batch, top_m] into selected; otherwise it
 * routes, then copies selected into promoted and sets gate[1] = 1.  (The reference reuses
 * promoted ids in place of routing: triton_promotion_cache_benchmark.py:53-60.)
 */
int spa_router_topm_gated(const void* q, int q_dtype, int batch, int q_heads,
                          int kv_heads, int head_dim, const float* summaries,
                          int n_pages, double scale, int top_m, int64_t* selected,
                          int32_t* gate, int64_t* promoted, spa_stream_t stream);
int spa_router_tree_topm_gated(const void* q, int q_dtype, int batch, int q_heads,
                               int kv_heads, int head_dim,
                               const float* super_summaries, int n_super,
                               const float* summaries, int n_pages, int superblock,
                               int top_super, double scale, int top_m,
                               int64_t* selected, int32_t* gate, int64_t* promoted,
                               spa_stream_t stream);
int spa_sparse_decode_step_gated(const void* q, int dtype, int batch, int q_heads,
                                 int kv_heads, int head_dim, const spa_kv_layout* kv,
                                 const int32_t* context_lens, int local_window,
                                 const float* super_summaries, int n_super,
                                 const float* summaries, int n_pages, int superblock,
                                 int top_super, int top_m, double router_scale,
                                 double attn_scale, int64_t* selected, void* out,
                                 void* workspace, size_t workspace_bytes,
                                 int32_t* gate, int64_t* promoted, spa_stream_t stream);

/*
 * Prepared sparse decode step for a serving loop (no reference counterpart: the
 * reference times select_blocks + paged_gather_decode_attention,
 * triton_paged_gather_decode_benchmark.py:69, from Python).  The session keeps every
 * argument of spa_sparse_decode_step[_gated]; the query of step `slot` is read from
 * query[slot] (mapped pinned host memory, see spa_host_device_pointer) and the results
 * go to result_host[slot] (output [B, Hq, D] at offset 0, page ids [B, top_m] int64 at
 * result_sel_offset), as io_mode says:
 *   SPA_SESSION_DIRECT_IN: the kernels read query[slot]; spa_copy returns result_bytes
 *     from result_dev (same layout) after the decode;
 *   SPA_SESSION_COPY_IN: spa_copy brings the query into query_dev first (one PCIe read),
 *     results as above;
 *   SPA_SESSION_ROUTER_IN_DIRECT_OUT: the router reads query[slot] and leaves a device
 *     copy in query_dev for the decode; the decode writes the output and the router a
 *     copy of the page ids straight to result_host[slot] (no copy kernels);
 *   SPA_SESSION_COPY_IN_DIRECT_OUT: spa_copy into query_dev, direct results.
 * The page ids the decode reads always sit in result_dev at result_sel_offset.
 * spa_session_create synchronises the device, runs one step and captures each slot's
 * launches as a CUDA graph.  Two slots double-buffer the host side:
 * spa_session_wait(s, slot) blocks until the last step enqueued on that slot has
 * completed; spa_session_step(s, slot, stream) enqueues a step (one graph launch and one
 * event record, no synchronisation).  gate/promoted may be NULL (ungated).
 */
typedef enum spa_session_io_mode {
  SPA_SESSION_DIRECT_IN = 0,
  SPA_SESSION_COPY_IN = 1,
  SPA_SESSION_ROUTER_IN_DIRECT_OUT = 2,
  SPA_SESSION_COPY_IN_DIRECT_OUT = 3
} spa_session_io_mode;
typedef struct spa_session_params {
  int dtype, batch, q_heads, kv_heads, head_dim;
  spa_kv_layout kv;
  const int32_t* context_lens;
  int local_window;
  const float* super_summaries; /* NULL: single-level router */
  int n_super;
  const float* summaries;
  int n_pages, superblock, top_super, top_m;
  double router_scale, attn_scale;
  void* workspace;
  size_t workspace_bytes;
  int32_t* gate;
  int64_t* promoted;
  int io_mode;           /* spa_session_io_mode */
  const void* query[2];
  void* query_dev;       /* [B, Hq, D] device buffer (every mode but SPA_SESSION_DIRECT_IN) */
  size_t query_bytes;    /* B * Hq * D * element size */
  void* result_dev;
  size_t result_sel_offset, result_bytes;
  void* result_host[2];
} spa_session_params;
typedef struct spa_session spa_session;
int spa_session_create(const spa_session_params* params, spa_session** out);
int spa_session_wait(spa_session* session, int slot);
int spa_session_step(spa_session* session, int slot, spa_stream_t stream);
int spa_session_destroy(spa_session* session);

/*
 * RMSNorm of `rows` rows of `dim` elements, for the integrated decoder's model:
 * out[r, i] = (x[r, i] * rsqrt(mean_j x[r, j]^2 + eps)) * weight[i], fp32 arithmetic,
 * x, weight and out of type dtype, contiguous.  One launch instead of the chain of
 * elementwise and reduction ops of its torch form (the decoder's norm, standing in for
 * the LayerNorm of train_tiny_transformer.py:178-190).
 */
int spa_rms_norm(const void* x, const void* weight, void* out, int rows, int dim, double eps, int dtype,
                 spa_stream_t stream);

/*
 * The decoder's residual add fused with the RMSNorm after it (one launch instead of two):
 * x_out[r, i] = dtype(x[r, i] + delta[r, i]) (rounded once, as a separate elementwise add
 * rounds it), out = spa_rms_norm(x_out).  x_out may be x itself (an in-place residual
 * stream); it must not overlap delta.  Same arguments and checks as spa_rms_norm; delta
 * and x_out are required when rows > 0.
 */
int spa_add_rms_norm(const void* x, const void* delta, const void* weight, void* x_out, void* out, int rows, int dim,
                     double eps, int dtype, spa_stream_t stream);

/*
 * The start of a decode step fused into one launch: the token and position embedding
 * lookup and the first RMSNorm (train_tiny_transformer.py:259,270, then the first block's
 * norm):  x_out[r] = dtype(table[ids[r]] + pos_table[positions[r]]), out = spa_rms_norm(x_out).
 * table [table_rows, dim] and pos_table [pos_rows, dim] of type dtype; ids int64 and
 * positions int32, [rows], in device memory.  An id outside its table raises device error
 * bit 4 (spa_device_error) and gives a zero row.
 */
int spa_embed_rms_norm(const void* table, int64_t table_rows, const int64_t* ids, const void* pos_table,
                       int64_t pos_rows, const int32_t* positions, const void* weight, void* x_out, void* out,
                       int rows, int dim, double eps, int dtype, spa_stream_t stream);

/*
 * Linear layer for 1..4 rows (the decoder's batch at decode time, where a library GEMM is
 * launch-bound): out[m, n] = act(dtype(x[m, :] . weight[n, :] + bias[n])), weight
 * [out_features, in_features] row-major (a torch Linear weight), bias optional (NULL).
 * fp32 products and sums, one rounding to dtype; activation 0 none, 1 exact GELU
 * (0.5 f (1 + erf(f / sqrt 2)) on the rounded value, rounded again).  out is of type dtype,
 * or fp32 holding the dtype-rounded values when out_f32 = 1.  x, weight, bias, out
 * contiguous.  rows > 4 returns SPA_ERR_INVALID.
 */
int spa_linear(const void* x, const void* weight, const void* bias, void* out, int rows, int in_features,
               int out_features, int activation, int out_f32, int dtype, spa_stream_t stream);

/* The RMSNorm in front of a spa_linear, fused into it (spa_norm_linear). */
typedef struct spa_norm_prologue {
  const void* delta;        /* added to x before the norm, rounded to dtype (NULL: none) */
  const int64_t* ids;       /* embedding mode: x row m is x[ids[m]] (NULL: row m) */
  int64_t id_limit;         /* rows of the x table (embedding mode) */
  const int32_t* delta_ids; /* embedding mode: delta row m is delta[delta_ids[m]] */
  int64_t delta_limit;      /* rows of the delta table (embedding mode) */
  const void* norm_weight;  /* RMSNorm weight [in_features], required */
  double eps;
  void* x_out;              /* receives the summed rows [rows, in_features] (NULL: not kept);
                               must not overlap x or delta */
} spa_norm_prologue;

/*
 * spa_linear applied to RMSNorm(x (+ delta)) in one launch: every CTA normalises the rows
 * itself, bit-identical to spa_add_rms_norm / spa_embed_rms_norm / spa_rms_norm (same
 * arithmetic and reduction order; in_features is the norm width), and one CTA stores the
 * summed rows to x_out.  With ids, the rows come from embedding tables as in
 * spa_embed_rms_norm (delta and delta_ids then required).  With append (NULL: none), the
 * output columns [k_col, k_col + kv_heads*head_dim) and [v_col, ...) of row m are also
 * the new K and V of batch row m, stored into the pools exactly as spa_kv_append stores
 * them (reference: the K/V cache write of triton_kvcache_transformer_decode.py:51-55).
 * Errors as spa_linear, plus SPA_ERR_INVALID without norm or norm_weight or with an
 * inconsistent append; an id outside its table raises device error bit 4 and gives a zero
 * row, a page outside the pools bit 2.
 */
/*
 * End of a greedy decode step in one launch: token[r] = argmax of logits[r, 0..cols) (fp32,
 * torch.argmax's rules: NaN counts as the largest value, the first index among equal
 * values), and counters[0..n_counters) each incremented by one (the decoder's position,
 * context length and step counter; NULL when n_counters is 0).
 */
int spa_argmax_advance(const float* logits, int rows, int cols, int64_t* token, int32_t* counters, int n_counters,
                       spa_stream_t stream);

/*
 * spa_argmax_advance that also logs the token: log[positions[r] * rows + r] = token[r] for
 * 0 <= positions[r] < log_len (positions are read before the counters advance; they may be
 * the first rows entries of counters).  A decoder keeps its generated tokens on the device
 * this way, with no copy between two graph replays.  rows <= 256 (one CTA serves every row).
 * No reference counterpart (the reference appends tokens on the host).
 */
int spa_argmax_advance_log(const float* logits, int rows, int cols, int64_t* token, int32_t* counters,
                           int n_counters, const int32_t* positions, int64_t* log, int log_len,
                           spa_stream_t stream);

/* The new token's K/V append fused into a spa_norm_linear epilogue (the QKV projection). */
typedef struct spa_kv_append_epilogue {
  spa_kv_layout kv;         /* K/V pools and page table, as for spa_kv_append */
  const int32_t* positions; /* [rows] token position of batch row m (negative: not stored) */
  int k_col;                /* first output column of K (kv_heads * head_dim columns, head-major) */
  int v_col;                /* first output column of V */
  int kv_heads;
  int head_dim;
  void* q_out;              /* optional [rows, q_width] of the output dtype: also receives output
                               columns [q_col, q_col + q_width) (the query, contiguous for the
                               attention step at any batch size); NULL: none */
  int q_col;
  int q_width;
} spa_kv_append_epilogue;

int spa_norm_linear(const void* x, const spa_norm_prologue* norm, const void* weight, const void* bias, void* out,
                    int rows, int in_features, int out_features, int activation, int out_f32, int dtype,
                    const spa_kv_append_epilogue* append, spa_stream_t stream);

/*
 * spa_linear / spa_norm_linear for a chain of dependent launches (a decode step): the
 * kernel is launched as a programmatic dependent of the kernel enqueued before it on the
 * stream and starts streaming its weight rows while that kernel still runs; every other
 * input is read, and every output written, only after that kernel has completed.  The
 * caller guarantees that weight, bias and the norm weight are not written by the kernel
 * enqueued immediately before (model weights during inference).  Same arguments and
 * results as the unchained forms.  No counterpart in the reference (its decode step is a
 * sequence of PyTorch calls).
 */
int spa_linear_chained(const void* x, const void* weight, const void* bias, void* out, int rows,
                       int in_features, int out_features, int activation, int out_f32, int dtype,
                       spa_stream_t stream);
int spa_norm_linear_chained(const void* x, const spa_norm_prologue* norm, const void* weight, const void* bias,
                            void* out, int rows, int in_features, int out_features, int activation, int out_f32,
                            int dtype, const spa_kv_append_epilogue* append, spa_stream_t stream);

/*
 * The integrated decoder's whole decode step in ONE launch (the KV-cache model decode of
 * triton_kvcache_transformer_decode.py:35-66 -- per layer the block of
 * train_tiny_transformer.py:134-190 with RMSNorm -- re-built around the paged cache, with
 * the router of triton_paged_gather_decode_benchmark.py:16-17 over the routable pages, the
 * gather decode of triton_paged_attention.py:139-168 over the local window + selected
 * pages, and the fixed-TTL promotion table of evaluate_promotion_ttl.py:134-135):
 *
 *   x = emb[token] + pos_emb[position];  per layer:  h = RMSNorm(x, norm1);
 *   qkv = h W_qkv^T + b (the new token's K and V stored at `position` in the layer's pools);
 *   selected = top-m of the router scores (ties to the lower page) over pages [0, n_pages);
 *   att = attention over the last local_window tokens then the selected pages;
 *   x = x + att W_out^T + b;  x = x + fc2(GELU(fc1(RMSNorm(x, norm2))));
 *   logits = RMSNorm(x, norm_f) head^T (fp32 of the rounded products);
 *   token = argmax(logits) (torch.argmax's rules), token_log[position, b] = token;
 *   promotion update of every (layer, b) row with its selection at step counters[2B];
 *   counters += 1 (positions [B], context lengths [B], step).
 *
 * The linear layers, norms and router use the arithmetic of spa_norm_linear / spa_linear /
 * spa_router_topm (bit-identical for the same inputs); the attention agrees with
 * spa_paged_gather_decode to rounding.  One cooperative grid of one CTA per SM; the phases
 * exchange data through the workspace (spa_decoder_step_workspace_size bytes, 256-byte
 * aligned, zero-filled before the first step and kept between steps).  Limits: batch 1..4,
 * layers 1..8, head_dim 32/64/128, d_model <= 512, d_model / ffn / vocab multiples of 8,
 * top_m <= 32, max pages per sequence <= 4096, promotion slots <= 512; weights 16-byte
 * aligned.  After a step that reported SPA_DEVERR_WAIT_TIMEOUT, zero the workspace again.
 */
#define SPA_DECODER_MAX_LAYERS 8
typedef struct spa_decoder_layer {
  const void* norm1;         /* [d_model] */
  const void* qkv_w;         /* [3 d_model, d_model] (q, k, v blocks, head-major) */
  const void* qkv_b;         /* [3 d_model] or NULL */
  const void* out_w;         /* [d_model, d_model] */
  const void* out_b;         /* [d_model] or NULL */
  const void* norm2;         /* [d_model] */
  const void* fc1_w;         /* [ffn, d_model] */
  const void* fc1_b;         /* [ffn] or NULL */
  const void* fc2_w;         /* [d_model, ffn] */
  const void* fc2_b;         /* [d_model] or NULL */
  void* k_pool;              /* the layer's pools, addressed by spa_decoder_step_params.kv */
  void* v_pool;
  const float* summaries;    /* [batch, heads, n_pages, head_dim] fp32 page mean keys (n_pages > 0) */
} spa_decoder_layer;

typedef struct spa_decoder_step_params {
  int dtype, batch, d_model, heads, ffn, vocab, layers;
  int local_window, top_m, n_pages;
  int max_pages;             /* pages per sequence when kv.page_table is NULL */
  double eps, router_scale, attn_scale;
  const void* emb;           /* [emb_rows, d_model] */
  int64_t emb_rows;
  const void* pos_emb;       /* [pos_rows, d_model] */
  int64_t pos_rows;
  const void* norm_f;        /* [d_model] */
  const void* head_w;        /* [vocab, d_model] */
  spa_decoder_layer layer[SPA_DECODER_MAX_LAYERS];
  spa_kv_layout kv;          /* page geometry and table shared by every layer (k, v unused) */
  int64_t* token;            /* [batch]: this step's tokens in, the greedy next tokens out */
  int32_t* counters;         /* [2 batch + 1]: positions, context lengths, step */
  float* logits;             /* [batch, vocab] */
  int64_t* token_log;        /* [log_len, batch] or NULL */
  int log_len;
  int64_t* selected;         /* [layers, batch, max(min(top_m, n_pages), 1)] (-1 when none) */
  int32_t* promo_pages;      /* [layers * batch, promo_slots] or NULL (no promotion table) */
  int32_t* promo_last_hit;
  int promo_slots, promo_ttl;
  void* workspace;
  size_t workspace_bytes;
} spa_decoder_step_params;

size_t spa_decoder_step_workspace_size(const spa_decoder_step_params* params);
int spa_decoder_step(const spa_decoder_step_params* params, spa_stream_t stream);

/*
 * Diagnostic for the failure path: one kernel waits on an mbarrier that nothing
 * completes, with the library's bounded wait limited to `cycles` (1 .. 4e9 clock
 * cycles).  The wait gives up, the kernel returns, and spa_device_error then reports
 * the wait-timeout bit (1).  No reference counterpart.
 */
int spa_debug_wait_timeout(long long cycles, spa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SPA_B200_H */
