// Single translation unit of the library: every kernel source is included here so
// the device error word and helpers are shared without relocatable device code.
#include "common.cuh"
#include "runtime.cuh"
#include "router.cuh"
#include "decode.cuh"
#include "decode_noalloc.cuh"
#include "step.cuh"
#include "gate.cuh"
#include "session.cuh"
#include "model.cuh"
#include "cache.cuh"
#include "decoder_step.cuh"
#include "prefill_generic.cuh"
#include "prefill_sm100.cuh"

extern "C" int spa_local_prefill(const void* q, const void* k, const void* v, int dtype, int batch, int heads,
                                 int seq_len, int head_dim, int window, const void* k_halo, const void* v_halo,
                                 int halo_len, int row_begin, int row_end, void* out, spa_stream_t stream) {
  if (!q || !k || !v || !out || !dtype_ok(dtype)) return SPA_ERR_INVALID;
  if (batch <= 0 || heads <= 0 || seq_len <= 0 || head_dim <= 0 || head_dim > 256 || window <= 0)
    return SPA_ERR_INVALID;
  if (halo_len < 0 || (halo_len > 0 && (!k_halo || !v_halo))) return SPA_ERR_INVALID;
  if (row_end <= 0) row_end = seq_len;
  if (row_begin < 0 || row_begin >= row_end || row_end > seq_len) return SPA_ERR_INVALID;
  spa::PrefillArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.k_halo = k_halo;
  a.v_halo = v_halo;
  a.out = out;
  a.B = batch;
  a.H = heads;
  a.S = seq_len;
  a.D = head_dim;
  a.W = window;
  a.halo = halo_len;
  a.row0 = row_begin;
  a.row1 = row_end;
  a.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(head_dim)));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype != SPA_F32 && spa::prefill_sm100_supported(a, dtype)) {
    return dtype == SPA_F16 ? spa::launch_prefill_sm100<__half>(a, dtype, st)
                            : spa::launch_prefill_sm100<__nv_bfloat16>(a, dtype, st);
  }
  switch (dtype) {
    case SPA_F32:
      return spa::launch_prefill_generic<float>(a, st);
    case SPA_F16:
      return spa::launch_prefill_generic<__half>(a, st);
    default:
      return spa::launch_prefill_generic<__nv_bfloat16>(a, st);
  }
}
