// KV append and the promotion-cache table update.
#pragma once

#include "common.cuh"

namespace spa {

// grid (B, Hkv), block = head_dim threads (<= 256).  Writes token positions[b].
// Reference: the tail K/V overwrite of page_decode (triton_kvcache_transformer_decode.py:51-55).
template <typename T>
__global__ void kv_append_kernel(T* __restrict__ k, T* __restrict__ v, KvAddr addr, int head_dim,
                                 const T* __restrict__ k_new, const T* __restrict__ v_new,
                                 const int32_t* __restrict__ positions) {
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int pos = positions[b];
  if (pos < 0 || d >= head_dim) return;
  const int64_t row = addr.row(b, h, pos);
  if (row < 0 || row >= addr.total_rows) {
    if (d == 0) spa_raise(SPA_DEVERR_BAD_PAGE);
    return;
  }
  const int64_t src = (static_cast<int64_t>(b) * gridDim.y + h) * head_dim + d;
  k[row * head_dim + d] = k_new[src];
  v[row * head_dim + d] = v_new[src];
}

// One warp per table row, the row's slots staged in shared memory.  Policy: hits refresh
// last_hit, then entries idle for >= ttl steps are freed, then new pages, in selection
// order, fill the lowest free slot or evict the least recently hit entry (ties: smallest
// page id).  The scans over slots are warp-parallel; the inserts stay sequential, as the
// policy defines them.  Reference policy: fixed-TTL refresh of promoted ids,
// evaluate_promotion_ttl.py:134-135; promoted-id reuse,
// triton_promotion_cache_benchmark.py:53-60.
//
// promotion_row_update: the update of one table row by one (converged) warp.  sel_src is the
// row's selection [top_m]; sel, pg and lh are the warp's shared-memory staging ([top_m],
// [slots], [slots]).
__device__ __forceinline__ void promotion_row_update(int32_t* __restrict__ pg_g, int32_t* __restrict__ lh_g,
                                                     const int64_t* __restrict__ sel_src, int top_m, int slots,
                                                     int step, int ttl, int64_t* sel, int32_t* pg, int32_t* lh) {
  const int lane = threadIdx.x & 31;
  // the row's selection is staged with the table (loads in flight together), so the
  // per-page loops below read shared memory, not one global load per page
  for (int j = lane; j < top_m; j += 32) sel[j] = sel_src[j];
  for (int i = lane; i < slots; i += 32) {
    pg[i] = pg_g[i];
    lh[i] = lh_g[i];
  }
  __syncwarp();
  // hits refresh last_hit
  for (int j = 0; j < top_m; ++j) {
    const int64_t id = sel[j];
    if (id < 0) continue;
    for (int i = lane; i < slots; i += 32)
      if (pg[i] == static_cast<int32_t>(id)) lh[i] = step;
  }
  __syncwarp();
  // idle entries expire
  for (int i = lane; i < slots; i += 32)
    if (pg[i] >= 0 && step - lh[i] >= ttl) pg[i] = -1;
  __syncwarp();
  // inserts, one selected page after another
  for (int j = 0; j < top_m; ++j) {
    const int64_t id64 = sel[j];
    if (id64 < 0 || id64 > 0x7fffffff) continue;
    const int32_t id = static_cast<int32_t>(id64);
    bool present = false;
    int free_slot = -1;
    for (int base = 0; base < slots; base += 32) {
      const int i = base + lane;
      const bool in = i < slots;
      present |= __any_sync(0xffffffffu, in && pg[i] == id);
      const unsigned fr = __ballot_sync(0xffffffffu, in && pg[i] < 0);
      if (free_slot < 0 && fr) free_slot = base + __ffs(fr) - 1;
    }
    if (present) continue;
    int slot = free_slot;
    if (slot < 0) {
      // least recently hit, ties to the smallest page id (ids in a row are distinct)
      int bl = 0x7fffffff, bp = 0x7fffffff, bi = 0x7fffffff;
      for (int i = lane; i < slots; i += 32)
        if (lh[i] < bl || (lh[i] == bl && pg[i] < bp)) {
          bl = lh[i];
          bp = pg[i];
          bi = i;
        }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const int ol = __shfl_xor_sync(0xffffffffu, bl, off), op = __shfl_xor_sync(0xffffffffu, bp, off),
                  oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ol < bl || (ol == bl && (op < bp || (op == bp && oi < bi)))) {
          bl = ol;
          bp = op;
          bi = oi;
        }
      }
      slot = bi;
    }
    if (lane == 0) {
      pg[slot] = id;
      lh[slot] = step;
    }
    __syncwarp();
  }
  for (int i = lane; i < slots; i += 32) {
    pg_g[i] = pg[i];
    lh_g[i] = lh[i];
  }
}

__global__ void __launch_bounds__(32) promotion_update_kernel(int32_t* __restrict__ pages,
                                                              int32_t* __restrict__ last_hit, int rows, int slots,
                                                              const int64_t* __restrict__ selected, int top_m,
                                                              int step_arg, const int32_t* __restrict__ step_dev,
                                                              int ttl) {
  extern __shared__ int64_t promo_smem[];  // sel [top_m], then pg [slots], lh [slots]
  // launched as a programmatic dependent of the kernel before it: every read after it completes
  pdl_trigger();
  pdl_block();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int step = step_dev ? *step_dev : step_arg;
  int64_t* sel = promo_smem;
  int32_t* pg = reinterpret_cast<int32_t*>(sel + top_m);
  promotion_row_update(pages + static_cast<int64_t>(r) * slots, last_hit + static_cast<int64_t>(r) * slots,
                       selected + static_cast<int64_t>(r) * top_m, top_m, slots, step, ttl, sel, pg, pg + slots);
}

}  // namespace spa

extern "C" int spa_kv_append(const spa_kv_layout* kv, int dtype, int batch, int kv_heads, int head_dim,
                             const void* k_new, const void* v_new, const int32_t* positions, spa_stream_t stream) {
  if (!kv || !kv->k || !kv->v || !k_new || !v_new || !positions || !dtype_ok(dtype)) return SPA_ERR_INVALID;
  if (batch <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim > 256 || kv->page_size <= 0) return SPA_ERR_INVALID;
  if (kv->page_table && kv->table_stride <= 0) return SPA_ERR_INVALID;
  const KvAddr addr = make_kv_addr(*kv);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(batch, kv_heads);
  if (dtype == SPA_F32)
    spa::kv_append_kernel<float><<<grid, head_dim, 0, st>>>(
        static_cast<float*>(const_cast<void*>(kv->k)), static_cast<float*>(const_cast<void*>(kv->v)), addr,
        head_dim, static_cast<const float*>(k_new), static_cast<const float*>(v_new), positions);
  else if (dtype == SPA_F16)
    spa::kv_append_kernel<__half><<<grid, head_dim, 0, st>>>(
        static_cast<__half*>(const_cast<void*>(kv->k)), static_cast<__half*>(const_cast<void*>(kv->v)), addr,
        head_dim, static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), positions);
  else
    spa::kv_append_kernel<__nv_bfloat16><<<grid, head_dim, 0, st>>>(
        static_cast<__nv_bfloat16*>(const_cast<void*>(kv->k)), static_cast<__nv_bfloat16*>(const_cast<void*>(kv->v)),
        addr, head_dim, static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new),
        positions);
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}

extern "C" int spa_promotion_update(int32_t* pages, int32_t* last_hit, int rows, int slots, const int64_t* selected,
                                    int top_m, int step, const int32_t* step_dev, int ttl, spa_stream_t stream) {
  if (!pages || !last_hit || !selected || rows <= 0 || slots <= 0 || top_m <= 0 || top_m > slots || ttl <= 0)
    return SPA_ERR_INVALID;
  if (slots > 8192) return SPA_ERR_UNSUPPORTED;  // the row is staged in shared memory
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = sizeof(int64_t) * static_cast<size_t>(top_m) + sizeof(int32_t) * 2 * static_cast<size_t>(slots);
  SPA_CHECK_CUDA(spa_set_smem_once(spa::promotion_update_kernel, static_cast<int>(smem)));
  SPA_CHECK_CUDA(spa::launch_ex(spa::promotion_update_kernel, dim3(rows), dim3(32), smem, st, true, 1, pages,
                                 last_hit, rows, slots, selected, top_m, step, step_dev, ttl));
  return SPA_OK;
}
