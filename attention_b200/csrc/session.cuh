// Prepared sparse decode step for a serving loop: the fused step (router -> gather decode,
// chained with programmatic dependent launch) with the step's query taken from, and its
// results returned to, mapped pinned host memory, captured once per slot as a CUDA graph.
// Nothing goes through a copy engine, and the host cost per step is one graph launch and
// one event record.  io_mode chooses how the bytes cross PCIe (spa_session_io_mode).
//
// Two slots double-buffer the host buffers: spa_session_wait(s, slot) blocks until the
// last step that used the slot has completed (its query may then be overwritten and its
// results read); spa_session_step(s, slot, stream) enqueues the next one.
//
// Reference: the timed unit of triton_paged_gather_decode_benchmark.py:69 with the query
// copied in and the result read back every step.
#pragma once

#include "runtime.cuh"
#include "step.cuh"

struct spa_session {
  spa_session_params p;
  cudaEvent_t done[2];
  cudaGraphExec_t exec[2];
};

namespace {
// The step's launches for one slot (eager or under capture).
int session_enqueue(const spa_session_params& p, int slot, cudaStream_t st) {
  const spa_stream_t ss = reinterpret_cast<spa_stream_t>(st);
  unsigned char* res = static_cast<unsigned char*>(p.result_dev);
  unsigned char* host = static_cast<unsigned char*>(p.result_host[slot]);
  int64_t* sel_dev = reinterpret_cast<int64_t*>(res + p.result_sel_offset);
  const bool copy_in = p.io_mode == SPA_SESSION_COPY_IN || p.io_mode == SPA_SESSION_COPY_IN_DIRECT_OUT;
  const bool router_in = p.io_mode == SPA_SESSION_ROUTER_IN_DIRECT_OUT;
  const bool direct_out = p.io_mode == SPA_SESSION_ROUTER_IN_DIRECT_OUT || p.io_mode == SPA_SESSION_COPY_IN_DIRECT_OUT;
  const void* q = p.query[slot];
  int rc;
  if (copy_in) {
    // one PCIe read of the query per step, then every CTA reads it from device memory; the
    // router launches during the copy and waits for it before its first read
    rc = spa::copy_launch(p.query_dev, q, p.query_bytes, ss, /*release_early=*/!p.gate);
    if (rc) return rc;
    q = p.query_dev;
  }
  // direct_out: the decode writes the output, and the router a copy of the page ids,
  // straight into the slot's host buffer; router_in: the router reads the query from host
  // memory and leaves a device copy in query_dev for the decode
  rc = spa::sparse_step_impl(q, p.dtype, p.batch, p.q_heads, p.kv_heads, p.head_dim, &p.kv, p.context_lens,
                             p.local_window, p.super_summaries, p.n_super, p.summaries, p.n_pages, p.superblock,
                             p.top_super, p.top_m, p.router_scale, p.attn_scale, sel_dev, direct_out ? host : res,
                             p.workspace, p.workspace_bytes, p.gate, p.promoted, ss, router_in ? p.query_dev : nullptr,
                             direct_out ? reinterpret_cast<int64_t*>(host + p.result_sel_offset) : nullptr,
                             /*router_pdl=*/copy_in && !p.gate);
  if (rc || direct_out) return rc;
  return spa_copy(p.result_host[slot], res, p.result_bytes, ss);
}

void session_release(spa_session* s) {
  for (int k = 0; k < 2; ++k) {
    if (s->exec[k]) cudaGraphExecDestroy(s->exec[k]);
    if (s->done[k]) cudaEventDestroy(s->done[k]);
  }
  delete s;
}
}  // namespace

extern "C" int spa_session_create(const spa_session_params* p, spa_session** out) {
  if (!p || !out) return SPA_ERR_INVALID;
  *out = nullptr;
  if (!p->query[0] || !p->query[1] || !p->result_host[0] || !p->result_host[1] || !p->result_dev)
    return SPA_ERR_INVALID;
  if (p->top_m <= 0 || p->batch <= 0 || p->q_heads <= 0 || p->head_dim <= 0) return SPA_ERR_INVALID;
  if (p->io_mode < SPA_SESSION_DIRECT_IN || p->io_mode > SPA_SESSION_COPY_IN_DIRECT_OUT) return SPA_ERR_INVALID;
  if (p->io_mode != SPA_SESSION_DIRECT_IN &&
      (!p->query_dev ||
       p->query_bytes != static_cast<size_t>(p->batch) * p->q_heads * p->head_dim * dtype_size(p->dtype)))
    return SPA_ERR_INVALID;
  const size_t out_bytes = static_cast<size_t>(p->batch) * p->q_heads * p->head_dim * dtype_size(p->dtype);
  const size_t sel_bytes = static_cast<size_t>(p->batch) * p->top_m * sizeof(int64_t);
  if (p->result_sel_offset < out_bytes || p->result_sel_offset % 8 != 0 ||
      p->result_bytes < p->result_sel_offset + sel_bytes)
    return SPA_ERR_INVALID;
  spa_session* s = new spa_session;
  s->p = *p;
  s->done[0] = s->done[1] = nullptr;
  s->exec[0] = s->exec[1] = nullptr;
  cudaStream_t cs = nullptr;
  int rc = SPA_OK;
  // the inputs (summaries, page table, pool) may still be in flight on any stream
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
  for (int k = 0; k < 2 && e == cudaSuccess; ++k) e = cudaEventCreateWithFlags(&s->done[k], cudaEventDisableTiming);
  // one eager step first (kernel attributes, TMA descriptors), then one capture per slot
  if (e == cudaSuccess) rc = session_enqueue(s->p, 0, cs);
  if (e == cudaSuccess && rc == SPA_OK) e = cudaStreamSynchronize(cs);
  for (int k = 0; k < 2 && e == cudaSuccess && rc == SPA_OK; ++k) {
    cudaGraph_t g = nullptr;
    e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) break;
    rc = session_enqueue(s->p, k, cs);
    const cudaError_t e2 = cudaStreamEndCapture(cs, &g);
    if (rc == SPA_OK) e = e2;
    if (e == cudaSuccess && rc == SPA_OK) e = cudaGraphInstantiate(&s->exec[k], g, 0);
    if (g) cudaGraphDestroy(g);
  }
  if (cs) cudaStreamDestroy(cs);
  if (e != cudaSuccess || rc != SPA_OK) {
    session_release(s);
    if (rc != SPA_OK) return rc;
    SPA_CHECK_CUDA(e);
  }
  *out = s;
  return SPA_OK;
}

extern "C" int spa_session_wait(spa_session* s, int slot) {
  if (!s || slot < 0 || slot > 1) return SPA_ERR_INVALID;
  SPA_CHECK_CUDA(cudaEventSynchronize(s->done[slot]));
  return SPA_OK;
}

extern "C" int spa_session_step(spa_session* s, int slot, spa_stream_t stream) {
  if (!s || slot < 0 || slot > 1) return SPA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SPA_CHECK_CUDA(cudaGraphLaunch(s->exec[slot], st));
  SPA_CHECK_CUDA(cudaEventRecord(s->done[slot], st));
  return SPA_OK;
}

extern "C" int spa_session_destroy(spa_session* s) {
  if (!s) return SPA_OK;
  for (int k = 0; k < 2; ++k) cudaEventSynchronize(s->done[k]);
  session_release(s);
  return SPA_OK;
}

// One sparse decode step with host buffers, for a caller that does not hold a session: the
// query is read from pinned host memory by a copy kernel into query_dev (one PCIe read),
// the step (one launch where it fuses) starts during that copy and writes its output, and
// a copy of the page ids, straight into pinned host memory.  No copy engine and one host
// call per step.  The copy waits for the stream's earlier work before it is launched, so
// a step enqueued behind another takes no SM slots while that one runs.
extern "C" int spa_sparse_decode_step_host(const void* query_host, void* query_dev, int dtype, int batch,
                                           int q_heads, int kv_heads, int head_dim, const spa_kv_layout* kv,
                                           const int32_t* context_lens, int local_window,
                                           const float* super_summaries, int n_super, const float* summaries,
                                           int n_pages, int superblock, int top_super, int top_m,
                                           double router_scale, double attn_scale, int64_t* selected_dev,
                                           int64_t* selected_host, void* out_host, void* workspace,
                                           size_t workspace_bytes, spa_stream_t stream) {
  if (!query_host || !query_dev || !selected_dev || !selected_host || !out_host) return SPA_ERR_INVALID;
  if (batch <= 0 || q_heads <= 0 || head_dim <= 0 || top_m <= 0) return SPA_ERR_INVALID;
  // the three host buffers must be pinned and mapped (their device addresses are used)
  void* qh = nullptr;
  void* sh = nullptr;
  void* oh = nullptr;
  if (cudaHostGetDevicePointer(&qh, const_cast<void*>(query_host), 0) != cudaSuccess ||
      cudaHostGetDevicePointer(&sh, selected_host, 0) != cudaSuccess ||
      cudaHostGetDevicePointer(&oh, out_host, 0) != cudaSuccess) {
    cudaGetLastError();  // not pinned host memory: clear the error state
    return SPA_ERR_INVALID;
  }
  const size_t elem = dtype == SPA_F32 ? 4 : 2;
  const size_t q_bytes = static_cast<size_t>(batch) * q_heads * head_dim * elem;
  int rc = spa::copy_launch(query_dev, qh, q_bytes, stream, /*release_early=*/true, /*pdl=*/false);
  if (rc) return rc;
  return spa::sparse_step_impl(query_dev, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens,
                               local_window, super_summaries, n_super, summaries, n_pages, superblock, top_super,
                               top_m, router_scale, attn_scale, selected_dev, oh, workspace, workspace_bytes,
                               nullptr, nullptr, stream, nullptr, static_cast<int64_t*>(sh), /*router_pdl=*/true);
}
