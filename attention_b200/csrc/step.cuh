// One sparse decode step: router (cluster kernel) -> split-K gather decode -> split merge,
// chained with programmatic dependent launch.  The decode grid starts while the router
// runs and streams its local-window chunks before it waits for the router's page ids.
//
// Reference: the timed unit of triton_paged_gather_decode_benchmark.py:69 and
// triton_promotion_cache_benchmark.py:59 --
//   paged_gather_decode_attention(q, K, V, select_blocks(q, summaries, m), ...).
#pragma once

#include "decode.cuh"
#include "router.cuh"

namespace spa {
int sparse_step_impl(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                     const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                     const float* super_summaries, int n_super, const float* summaries, int n_pages, int superblock,
                     int top_super, int top_m, double router_scale, double attn_scale, int64_t* selected, void* out,
                     void* workspace, size_t workspace_bytes, int32_t* gate, int64_t* promoted,
                     spa_stream_t stream, void* q_copy = nullptr, int64_t* selected_copy = nullptr,
                     bool router_pdl = false) {
  if (!q || !out || !kv || !kv->k || !kv->v || !context_lens || !summaries || !selected) return SPA_ERR_INVALID;
  if (dtype != SPA_F16 && dtype != SPA_BF16 && dtype != SPA_F32) return SPA_ERR_INVALID;
  if (local_window < 0 || top_m <= 0) return SPA_ERR_INVALID;
  int rc;
  if (super_summaries)
    rc = router_tree_impl(q, dtype, batch, q_heads, kv_heads, head_dim, super_summaries, n_super, summaries, n_pages,
                          superblock, top_super, router_scale, top_m, selected, gate, promoted, stream, q_copy,
                          selected_copy, router_pdl);
  else
    rc = router_topm_impl(q, dtype, batch, q_heads, kv_heads, head_dim, summaries, n_pages, router_scale, top_m,
                          selected, nullptr, gate, promoted, stream, q_copy, selected_copy, router_pdl);
  if (rc) return rc;
  spa::DecodeArgs a;
  // with q_copy the query lives in host memory: the decode reads the router's device copy
  a.q = q_copy ? q_copy : q;
  a.out = out;
  a.B = batch;
  a.Hq = q_heads;
  a.Hkv = kv_heads;
  a.group = q_heads / kv_heads;
  a.D = head_dim;
  a.addr = make_kv_addr(*kv);
  a.ctx_lens = context_lens;
  a.local_window = local_window;
  a.selected = selected;
  a.top_m = top_m;
  a.span_len = 0;
  const int max_cand = local_window + top_m * kv->page_size;
  const spa::SplitPlan plan = spa::decode_plan(batch, q_heads, kv_heads, max_cand);
  a.nsplit = plan.nsplit;
  a.scale = static_cast<float>(attn_scale);
  a.scale_log2 = static_cast<float>(attn_scale * 1.4426950408889634);
  a.part_o = nullptr;
  a.part_lse = nullptr;
  a.early_local = 1;
  // the query is written by a kernel still running when the decode launches (the router's
  // copy, or the copy-in the router waits for): read it after the wait
  a.q_after_wait = q_copy != nullptr || router_pdl;
  {
    const size_t need = spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_cand);
    if (need && (!workspace || workspace_bytes < need)) return SPA_ERR_WORKSPACE;
    a.part_o = static_cast<float*>(workspace);
    a.part_lse = need ? a.part_o + static_cast<size_t>(batch) * q_heads * a.nsplit * head_dim : nullptr;
  }
  const bool linear_rows = !kv->page_table && kv->page_stride_rows == kv->page_size;
  const bool fast = dtype != SPA_F32 && (head_dim == 64 || head_dim == 128) && a.group <= 16 &&
                    (kv->page_size % spa::kChunk == 0 || linear_rows) && kv->total_rows < (1ll << 31) &&
                    reinterpret_cast<uintptr_t>(kv->k) % 16 == 0 && reinterpret_cast<uintptr_t>(kv->v) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(q) % 4 == 0;
  a.cluster_merge = fast && plan.cluster;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
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
