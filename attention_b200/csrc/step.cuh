// One sparse decode step.  Where the shape allows (bf16/fp16, head_dim 64 or 128, the
// splits of each (sequence, kv head) pair merged in one cluster, at most 8 kv heads), it
// is ONE launch: decode_mma_kernel's route instantiation, in which every decode cluster
// scores its sequence's summaries itself, selects the pages and streams them; the
// local-window chunks load while it routes.  Otherwise: the router (cluster kernel), then
// the split-K gather decode launched as its programmatic dependent (its grid starts while
// the router runs and streams the local window before it waits for the page ids).
//
// Reference: the timed unit of triton_paged_gather_decode_benchmark.py:69 and
// triton_promotion_cache_benchmark.py:59 --
//   paged_gather_decode_attention(q, K, V, select_blocks(q, summaries, m), ...).
#pragma once

#include "decode.cuh"
#include "router.cuh"

namespace spa {

// 1 (default): steps whose shape the single-launch kernel serves run as one launch (the
// decode clusters route their sequence themselves); 0: router launch, then decode launch.
inline int& step_fusion_mode() {
  static int mode = 1;
  return mode;
}

// Whether a step of this form runs as one launch (the route instantiation of the decode).
inline bool step_fusable(bool fast, bool gated, bool router_copies_query, int kv_heads, int top_m) {
  return step_fusion_mode() != 0 && fast && !gated && !router_copies_query && kv_heads <= kRouterKvBatch &&
         top_m <= DecodeSmem<128, kDecodeStages>::kSelCap;
}

// The step's split plan: the decode's, except that a fused step whose pairs are too few for
// the decode's cluster plan still takes clusters of kMaxClusterSplits splits (the routing
// needs the splits of a pair in one cluster) when they fit on the GPU twice over.
inline SplitPlan step_plan(int batch, int q_heads, int kv_heads, int max_cand, bool fusable) {
  SplitPlan plan = decode_plan(batch, q_heads, kv_heads, max_cand);
  if (fusable && !plan.cluster && static_cast<int64_t>(batch) * kv_heads * kMaxClusterSplits <= 2 * device_sm_count())
    plan = {kMaxClusterSplits, true};
  return plan;
}

// Router-side argument checks of a step (the ones router_tree_impl / router_topm_impl make).
inline int step_route_checks(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                             const float* super_summaries, int n_super, const float* summaries, int n_pages,
                             int superblock, int top_super, int top_m) {
  int rc = router_common_checks(q, dtype, batch, q_heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!summaries || n_pages <= 0 || top_m <= 0) return SPA_ERR_INVALID;
  if (!super_summaries) return top_m > n_pages ? SPA_ERR_INVALID : SPA_OK;
  if (superblock <= 0 || n_super != (n_pages + superblock - 1) / superblock) return SPA_ERR_INVALID;
  if (top_super <= 0 || top_super > n_super || top_super > 64) return SPA_ERR_INVALID;
  const int last = n_pages - (n_super - 1) * superblock;
  const int min_cand = (top_super - 1) * superblock + (last < superblock ? last : superblock);
  return top_m > min_cand ? SPA_ERR_INVALID : SPA_OK;
}

// One routed decode step.  q [B, q_heads, D] holds every query head of each sequence and
// the summaries every kv head (the router's inputs); the decode covers kv heads
// [kv_begin, kv_begin + kv_count) (kv_count < 0: all), whose K/V the layout addresses
// (kv_count heads) and whose query heads the output [B, kv_count * group, D] receives.
int sparse_step_impl(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                     const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                     const float* super_summaries, int n_super, const float* summaries, int n_pages, int superblock,
                     int top_super, int top_m, double router_scale, double attn_scale, int64_t* selected, void* out,
                     void* workspace, size_t workspace_bytes, int32_t* gate, int64_t* promoted,
                     spa_stream_t stream, void* q_copy = nullptr, int64_t* selected_copy = nullptr,
                     bool router_pdl = false, int kv_begin = 0, int kv_count = -1) {
  if (!q || !out || !kv || !kv->k || !kv->v || !context_lens || !summaries || !selected) return SPA_ERR_INVALID;
  if (dtype != SPA_F16 && dtype != SPA_BF16 && dtype != SPA_F32) return SPA_ERR_INVALID;
  if (local_window < 0 || top_m <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads) return SPA_ERR_INVALID;
  if (kv_count < 0) kv_count = kv_heads;
  if (kv_begin < 0 || kv_count <= 0 || kv_begin + kv_count > kv_heads) return SPA_ERR_INVALID;
  if ((gate == nullptr) != (promoted == nullptr)) return SPA_ERR_INVALID;
  const int group = q_heads / kv_heads;
  spa::DecodeArgs a{};
  a.out = out;
  a.B = batch;
  a.Hq = kv_count * group;
  a.Hkv = kv_count;
  a.group = group;
  a.D = head_dim;
  a.q_batch_heads = q_heads;
  a.q_head_offset = kv_begin * group;
  a.addr = make_kv_addr(*kv);
  a.ctx_lens = context_lens;
  a.local_window = local_window;
  a.selected = selected;
  a.top_m = top_m;
  a.span_len = 0;
  const int max_cand = local_window + top_m * kv->page_size;
  const bool linear_rows = !kv->page_table && kv->page_stride_rows == kv->page_size;
  const bool fast = dtype != SPA_F32 && (head_dim == 64 || head_dim == 128) && group <= 16 &&
                    (kv->page_size % spa::kChunk == 0 || linear_rows) && kv->total_rows < (1ll << 31) &&
                    reinterpret_cast<uintptr_t>(kv->k) % 16 == 0 && reinterpret_cast<uintptr_t>(kv->v) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(q) % 4 == 0;
  const bool fusable = step_fusable(fast, gate != nullptr, q_copy != nullptr, kv_heads, top_m);
  const spa::SplitPlan plan = step_plan(batch, a.Hq, a.Hkv, max_cand, fusable);
  a.nsplit = plan.nsplit;
  a.scale = static_cast<float>(attn_scale);
  a.scale_log2 = static_cast<float>(attn_scale * 1.4426950408889634);
  a.part_o = nullptr;
  a.part_lse = nullptr;
  {
    const size_t need = spa_decode_workspace_size(batch, a.Hq, a.Hkv, head_dim, max_cand);
    if (need && (!workspace || workspace_bytes < need)) return SPA_ERR_WORKSPACE;
    a.part_o = static_cast<float*>(workspace);
    a.part_lse = need ? a.part_o + static_cast<size_t>(batch) * a.Hq * a.nsplit * head_dim : nullptr;
  }
  a.cluster_merge = fast && plan.cluster;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  // ---- one launch: the decode clusters route their sequence themselves
  if (fusable && plan.cluster && plan.nsplit >= 2) {
    int rc = step_route_checks(q, dtype, batch, q_heads, kv_heads, head_dim, super_summaries, n_super, summaries,
                               n_pages, superblock, top_super, top_m);
    if (rc) return rc;
    a.q = q;
    a.early_local = 0;  // the kernel waits for its predecessor (when launched as its dependent) first
    a.q_after_wait = 0;
    a.route.q_heads = q_heads;
    a.route.kv_heads = kv_heads;
    a.route.supers = super_summaries;
    a.route.n_super = super_summaries ? n_super : 0;
    a.route.superblock = super_summaries ? superblock : 0;
    a.route.top_super = super_summaries ? top_super : 0;
    a.route.summaries = summaries;
    a.route.n_pages = n_pages;
    a.route.scale = static_cast<float>(router_scale);
    a.route.selected = selected;
    a.route.selected_copy = selected_copy;
    // with router_pdl (the session's copy-in precedes it) launched as that kernel's
    // programmatic dependent; it waits for it before its first read either way.  Not by
    // default: a step launched early behind a running step only holds SM slots there.
    if (dtype == SPA_F16)
      rc = head_dim == 128 ? launch_decode_mma<__half, 128, true>(*kv, dtype, a, st, router_pdl)
                           : launch_decode_mma<__half, 64, true>(*kv, dtype, a, st, router_pdl);
    else
      rc = head_dim == 128 ? launch_decode_mma<__nv_bfloat16, 128, true>(*kv, dtype, a, st, router_pdl)
                           : launch_decode_mma<__nv_bfloat16, 64, true>(*kv, dtype, a, st, router_pdl);
    if (rc != SPA_ERR_UNSUPPORTED) return rc;  // else (scratch too large): the two launches below
  }

  // ---- router launch, then the decode launched as its programmatic dependent
  int rc;
  if (super_summaries)
    rc = router_tree_impl(q, dtype, batch, q_heads, kv_heads, head_dim, super_summaries, n_super, summaries, n_pages,
                          superblock, top_super, router_scale, top_m, selected, gate, promoted, stream, q_copy,
                          selected_copy, router_pdl);
  else
    rc = router_topm_impl(q, dtype, batch, q_heads, kv_heads, head_dim, summaries, n_pages, router_scale, top_m,
                          selected, nullptr, gate, promoted, stream, q_copy, selected_copy, router_pdl);
  if (rc) return rc;
  // with q_copy the query lives in host memory: the decode reads the router's device copy
  a.q = q_copy ? q_copy : q;
  a.early_local = 1;
  // the query is written by a kernel still running when the decode launches (the router's
  // copy, or the copy-in the router waits for): read it after the wait
  a.q_after_wait = q_copy != nullptr || router_pdl;
  switch (dtype) {
    case SPA_F32:
      return spa::launch_decode<float>(*kv, dtype, a, false, st);
    case SPA_F16:
      return spa::launch_decode<__half>(*kv, dtype, a, fast, st);
    default:
      return spa::launch_decode<__nv_bfloat16>(*kv, dtype, a, fast, st);
  }
}
}  // namespace spa

extern "C" int spa_sparse_decode_step(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                                      const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                                      const float* super_summaries, int n_super, const float* summaries,
                                      int n_pages, int superblock, int top_super, int top_m, double router_scale,
                                      double attn_scale, int64_t* selected, void* out, void* workspace,
                                      size_t workspace_bytes, spa_stream_t stream) {
  return spa::sparse_step_impl(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window,
                               super_summaries, n_super, summaries, n_pages, superblock, top_super, top_m,
                               router_scale, attn_scale, selected, out, workspace, workspace_bytes, nullptr, nullptr,
                               stream);
}

extern "C" int spa_sparse_decode_step_chained(const void* q, int dtype, int batch, int q_heads, int kv_heads,
                                              int head_dim, const spa_kv_layout* kv, const int32_t* context_lens,
                                              int local_window, const float* super_summaries, int n_super,
                                              const float* summaries, int n_pages, int superblock, int top_super,
                                              int top_m, double router_scale, double attn_scale, int64_t* selected,
                                              void* out, void* workspace, size_t workspace_bytes,
                                              spa_stream_t stream) {
  return spa::sparse_step_impl(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window,
                               super_summaries, n_super, summaries, n_pages, superblock, top_super, top_m,
                               router_scale, attn_scale, selected, out, workspace, workspace_bytes, nullptr, nullptr,
                               stream, nullptr, nullptr, /*router_pdl=*/true);
}

extern "C" int spa_sparse_decode_step_gated(const void* q, int dtype, int batch, int q_heads, int kv_heads,
                                            int head_dim, const spa_kv_layout* kv, const int32_t* context_lens,
                                            int local_window, const float* super_summaries, int n_super,
                                            const float* summaries, int n_pages, int superblock, int top_super,
                                            int top_m, double router_scale, double attn_scale, int64_t* selected,
                                            void* out, void* workspace, size_t workspace_bytes, int32_t* gate,
                                            int64_t* promoted, spa_stream_t stream) {
  if (!gate || !promoted) return SPA_ERR_INVALID;
  return spa::sparse_step_impl(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window,
                               super_summaries, n_super, summaries, n_pages, superblock, top_super, top_m,
                               router_scale, attn_scale, selected, out, workspace, workspace_bytes, gate, promoted,
                               stream);
}

extern "C" int spa_sparse_decode_step_heads(const void* q, int dtype, int batch, int q_heads, int kv_heads,
                                            int head_dim, int kv_head_begin, int kv_head_count,
                                            const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                                            const float* super_summaries, int n_super, const float* summaries,
                                            int n_pages, int superblock, int top_super, int top_m,
                                            double router_scale, double attn_scale, int64_t* selected, void* out,
                                            void* workspace, size_t workspace_bytes, spa_stream_t stream) {
  if (kv_head_count <= 0) return SPA_ERR_INVALID;
  return spa::sparse_step_impl(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window,
                               super_summaries, n_super, summaries, n_pages, superblock, top_super, top_m,
                               router_scale, attn_scale, selected, out, workspace, workspace_bytes, nullptr, nullptr,
                               stream, nullptr, nullptr, false, kv_head_begin, kv_head_count);
}

extern "C" int spa_sparse_step_launches(int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                                        int kv_head_count, int local_window, int page_size, int top_m,
                                        int* launches) {
  if (!launches || batch <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || page_size <= 0 ||
      top_m <= 0 || local_window < 0)
    return SPA_ERR_INVALID;
  if (kv_head_count <= 0) kv_head_count = kv_heads;
  const int group = q_heads / kv_heads;
  const int hq = kv_head_count * group;
  const bool fast = dtype != SPA_F32 && (head_dim == 64 || head_dim == 128) && group <= 16 &&
                    page_size % spa::kChunk == 0;
  const bool fusable = spa::step_fusable(fast, false, false, kv_heads, top_m);
  const spa::SplitPlan plan =
      spa::step_plan(batch, hq, kv_head_count, local_window + top_m * page_size, fusable);
  if (fusable && plan.cluster && plan.nsplit >= 2)
    *launches = 1;  // one kernel: routing + decode
  else
    *launches = 2 + ((fast && plan.cluster) || plan.nsplit <= 1 ? 0 : 1);  // router, decode (+ split merge)
  return SPA_OK;
}

extern "C" int spa_set_step_fusion(int mode) {
  const int prev = spa::step_fusion_mode();
  if (mode == 0 || mode == 1) spa::step_fusion_mode() = mode;
  return prev;
}
