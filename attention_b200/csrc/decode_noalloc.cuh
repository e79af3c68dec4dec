// Allocation-free variant of spa_paged_decode.
//
// Some callers cannot allocate device memory at the point where they decode: a
// serving engine that owns every byte of HBM through its own pool, or a plugin
// host whose interface has no way to hand the plugin a workspace.  This entry
// point takes the split-K partials from a fixed scratch array compiled into the
// library instead of a caller workspace.  The array lives in device memory of
// every GPU that loads the library, for the life of the process.
#pragma once

#include "decode.cuh"

namespace spa {

// The scratch itself.  Host code must never pass this name to a kernel: on the host
// it is only a stand-in, and the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_decode_scratch[SPA_DECODE_STATIC_SCRATCH_BYTES];

// Device address of g_decode_scratch in the context current on the calling thread, or
// nullptr on failure.  Looked up on every call rather than cached: a cached address
// belongs to the context it was looked up in, and a caller may decode from another
// context on the same device (a plugin host's own driver context) or after a device
// reset, where a cached address would point at memory the current context does not
// own.  The first lookup in a context loads the library's device code into it.
inline void* decode_scratch_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess) return nullptr;
  return p;
}

}  // namespace spa

extern "C" int spa_paged_decode_noalloc(const void* q, int dtype, int batch, int q_heads, int kv_heads,
                                        int head_dim, const spa_kv_layout* kv, const int32_t* context_lens,
                                        int local_window, const int64_t* selected, int top_m, int max_candidates,
                                        double scale, void* out, spa_stream_t stream) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || max_candidates < 0) return SPA_ERR_INVALID;
  const size_t need = spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_candidates);
  if (need > SPA_DECODE_STATIC_SCRATCH_BYTES) return SPA_ERR_WORKSPACE;
  // resolved on every call, also when this request needs no scratch, so the first call
  // in a context always does the lookup (callers are told to make it before any capture)
  void* scratch = spa::decode_scratch_ptr();
  if (!scratch) return SPA_ERR_CUDA;
  return spa_paged_decode(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window, selected,
                          top_m, max_candidates, scale, out, need > 0 ? scratch : nullptr, need, stream);
}
