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
