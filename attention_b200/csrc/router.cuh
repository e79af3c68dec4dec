// Page summaries and the page router (single level and superblock -> page tree).
//
// Canonical arithmetic (the oracle restates exactly this order, so scores and
// therefore selections are bit-identical):
//   page sum   S[b,h,g,d] = ((K[t0,d] + K[t0+1,d]) + ...) in fp64, tokens in order
//   summary    = fp32(S / page_size)                              (fp64 divide)
//   super sum  = ((S[g0] + S[g0+1]) + ...) over the superblock's pages in order
//   super      = fp32(super sum / (pages_in_super * page_size))
//   qg[kvh,d]  = ((q[h0,d] + q[h0+1,d]) + ...) over the kv head's query heads, fp64
//   dot_kvh    = per lane l: sum_k qg[kvh, l+32k] * summ[kvh, l+32k]  (k ascending,
//                separate multiply and add), then xor-butterfly over lanes with
//                offsets 16, 8, 4, 2, 1
//   score      = ((dot_0 + dot_1) + ...) over kv heads, / q_heads, * scale
// Selection: descending score, ties to the lower page index.
//
// Reference: select_blocks (triton_paged_gather_decode_benchmark.py:16-17) computes
// einsum("bhd,bhgd->bhg").mean(1).topk(m); summaries at :61.  Grouping the q heads
// of one kv head first is the same sum (reference Hq == Hkv: groups of one).
#pragma once

#include "common.cuh"

namespace spa {

// ---------------------------------------------------------------------------
// summaries: grid (n_pages, Hkv, B), block = head_dim threads (<= 256)
template <typename T>
__global__ void page_summaries_kernel(const T* __restrict__ k, KvAddr addr, int head_dim, int n_pages,
                                      float* __restrict__ summaries, double* __restrict__ sums64) {
  const int g = blockIdx.x, h = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  if (d >= head_dim) return;
  const int P = addr.page_size;
  const int64_t row0 = addr.row(b, h, g * P);
  double acc = 0.0;
  if (row0 < 0 || row0 + P > addr.total_rows) {
    spa_raise(SPA_DEVERR_BAD_PAGE);
  } else {
    const T* p = k + row0 * head_dim + d;
    for (int t = 0; t < P; ++t) acc = __dadd_rn(acc, to_f64(p[static_cast<int64_t>(t) * head_dim]));
  }
  const int64_t o = ((static_cast<int64_t>(b) * gridDim.y + h) * n_pages + g) * head_dim + d;
  summaries[o] = __double2float_rn(__ddiv_rn(acc, static_cast<double>(P)));
  if (sums64) sums64[o] = acc;
}

// grid (n_super, Hkv, B), block = head_dim threads
__global__ void super_summaries_kernel(const double* __restrict__ sums64, int head_dim, int n_pages,
                                       int superblock, int page_size, float* __restrict__ super_out) {
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  if (d >= head_dim) return;
  const int g0 = s * superblock;
  const int g1 = min(g0 + superblock, n_pages);
  const double* p = sums64 + ((static_cast<int64_t>(b) * gridDim.y + h) * n_pages) * head_dim + d;
  double acc = 0.0;
  for (int g = g0; g < g1; ++g) acc = __dadd_rn(acc, p[static_cast<int64_t>(g) * head_dim]);
  const double n = static_cast<double>(g1 - g0) * static_cast<double>(page_size);
  super_out[((static_cast<int64_t>(b) * gridDim.y + h) * gridDim.x + s) * head_dim + d] =
      __double2float_rn(__ddiv_rn(acc, n));
}

// ---------------------------------------------------------------------------
// scoring helpers
constexpr int kRouterMaxHeadDim = 256;
constexpr int kRouterMaxKvHeads = 64;

// qg (fp64, [Hkv][D]) into shared memory; group sums in head order.
template <typename T>
__device__ void load_group_query(const T* __restrict__ q, int b, int q_heads, int kv_heads, int head_dim,
                                 double* __restrict__ qg) {
  const int group = q_heads / kv_heads;
  for (int i = threadIdx.x; i < kv_heads * head_dim; i += blockDim.x) {
    const int kvh = i / head_dim, d = i - kvh * head_dim;
    const T* qp = q + (static_cast<int64_t>(b) * q_heads + kvh * group) * head_dim + d;
    double acc = 0.0;
    for (int j = 0; j < group; ++j) acc = __dadd_rn(acc, to_f64(qp[static_cast<int64_t>(j) * head_dim]));
    qg[i] = acc;
  }
}

// Score of one page by one warp (all lanes return the same value).
// summ points at summary[b, 0, g, 0]; kv_stride = elements between kv heads.
__device__ __forceinline__ double warp_page_score(const double* __restrict__ qg, const float* __restrict__ summ,
                                                  int64_t kv_stride, int kv_heads, int head_dim, int q_heads,
                                                  double scale) {
  const int lane = threadIdx.x & 31;
  double total = 0.0;
  for (int kvh = 0; kvh < kv_heads; ++kvh) {
    const float* s = summ + kvh * kv_stride;
    const double* qq = qg + kvh * head_dim;
    double part = 0.0;
    for (int d = lane; d < head_dim; d += 32)
      part = __dadd_rn(part, __dmul_rn(qq[d], static_cast<double>(__ldg(s + d))));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part = __dadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
    total = __dadd_rn(total, part);
  }
  return __dmul_rn(__ddiv_rn(total, static_cast<double>(q_heads)), scale);
}

// (score, index) ordering: a beats b when its score is larger, or equal with a lower index.
__device__ __forceinline__ bool beats(double sa, int ia, double sb, int ib) {
  return sa > sb || (sa == sb && ia < ib);
}

// Block-wide top-m over cand_score[0..n) (indices cand_idx[0..n)), written in
// descending order to out[0..m).  Chosen entries are overwritten with -inf and
// index INT_MAX.  Uses red_s / red_i scratch of blockDim.x/32 entries.
__device__ void block_topm(double* cand_score, int* cand_idx, int n, int m, int64_t* out, double* red_s,
                           int* red_i, int* chosen_pos) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int r = 0; r < m; ++r) {
    double bs = -INFINITY;
    int bi = 0x7fffffff, bp = -1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      if (cand_idx[i] != 0x7fffffff && (bp < 0 || beats(cand_score[i], cand_idx[i], bs, bi))) {
        bs = cand_score[i];
        bi = cand_idx[i];
        bp = i;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const double os = __shfl_xor_sync(0xffffffffu, bs, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const int op = __shfl_xor_sync(0xffffffffu, bp, off);
      if (op >= 0 && (bp < 0 || beats(os, oi, bs, bi))) {
        bs = os;
        bi = oi;
        bp = op;
      }
    }
    if (lane == 0) {
      red_s[warp] = bs;
      red_i[warp] = bp;  // position; the index is read back from cand_idx
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int best = -1;
      for (int w = 0; w < nwarps; ++w) {
        const int p = red_i[w];
        if (p < 0) continue;
        if (best < 0 || beats(cand_score[p], cand_idx[p], cand_score[best], cand_idx[best])) best = p;
      }
      *chosen_pos = best;
      out[r] = best >= 0 ? static_cast<int64_t>(cand_idx[best]) : -1;
      if (best >= 0) cand_idx[best] = 0x7fffffff;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// single-level router: grid (B), block 256; dynamic smem: qg + scores + idx
template <typename T>
__global__ void __launch_bounds__(256) router_topm_kernel(const T* __restrict__ q, int q_heads, int kv_heads,
                                                          int head_dim, const float* __restrict__ summaries,
                                                          int n_pages, double scale, int top_m,
                                                          int64_t* __restrict__ selected,
                                                          double* __restrict__ scores_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* qg = reinterpret_cast<double*>(smem_raw);
  double* sc = qg + kv_heads * head_dim;
  int* ix = reinterpret_cast<int*>(sc + n_pages);
  __shared__ double red_s[8];
  __shared__ int red_i[8];
  __shared__ int chosen;
  const int b = blockIdx.x;
  load_group_query(q, b, q_heads, kv_heads, head_dim, qg);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int64_t kv_stride = static_cast<int64_t>(n_pages) * head_dim;
  const float* base = summaries + static_cast<int64_t>(b) * kv_heads * kv_stride;
  for (int g = warp; g < n_pages; g += nwarps) {
    const double s = warp_page_score(qg, base + static_cast<int64_t>(g) * head_dim, kv_stride, kv_heads,
                                     head_dim, q_heads, scale);
    if (lane == 0) {
      sc[g] = s;
      ix[g] = g;
      if (scores_out) scores_out[static_cast<int64_t>(b) * n_pages + g] = s;
    }
  }
  __syncthreads();
  block_topm(sc, ix, n_pages, top_m, selected + static_cast<int64_t>(b) * top_m, red_s, red_i, &chosen);
}

// ---------------------------------------------------------------------------
// tree router: grid (B), block 256.  Level 1 over n_super superblocks, level 2
// over the pages of the top_super chosen superblocks.
template <typename T>
__global__ void __launch_bounds__(256) router_tree_kernel(const T* __restrict__ q, int q_heads, int kv_heads,
                                                          int head_dim, const float* __restrict__ supers,
                                                          int n_super, const float* __restrict__ summaries,
                                                          int n_pages, int superblock, int top_super,
                                                          double scale, int top_m,
                                                          int64_t* __restrict__ selected) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* qg = reinterpret_cast<double*>(smem_raw);
  const int cand_cap = max(n_super, top_super * superblock);
  double* sc = qg + kv_heads * head_dim;
  int* ix = reinterpret_cast<int*>(sc + cand_cap);
  int64_t* chosen_super = reinterpret_cast<int64_t*>(ix + cand_cap + (cand_cap & 1));
  __shared__ double red_s[8];
  __shared__ int red_i[8];
  __shared__ int chosen;
  const int b = blockIdx.x;
  load_group_query(q, b, q_heads, kv_heads, head_dim, qg);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  // level 1
  {
    const int64_t kv_stride = static_cast<int64_t>(n_super) * head_dim;
    const float* base = supers + static_cast<int64_t>(b) * kv_heads * kv_stride;
    for (int s = warp; s < n_super; s += nwarps) {
      const double v = warp_page_score(qg, base + static_cast<int64_t>(s) * head_dim, kv_stride, kv_heads,
                                       head_dim, q_heads, scale);
      if (lane == 0) {
        sc[s] = v;
        ix[s] = s;
      }
    }
    __syncthreads();
    block_topm(sc, ix, n_super, top_super, chosen_super, red_s, red_i, &chosen);
  }
  // level 2: candidate pages listed superblock by superblock (selection order)
  __shared__ int cand_start[64];
  __shared__ int n_cand;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < top_super; ++j) {
      cand_start[j] = n;
      const int s = static_cast<int>(chosen_super[j]);
      const int g0 = s * superblock, g1 = min(g0 + superblock, n_pages);
      n += max(0, g1 - g0);
    }
    n_cand = n;
  }
  __syncthreads();
  const int nc = n_cand;
  {
    const int64_t kv_stride = static_cast<int64_t>(n_pages) * head_dim;
    const float* base = summaries + static_cast<int64_t>(b) * kv_heads * kv_stride;
    for (int c = warp; c < nc; c += nwarps) {
      int j = 0;
      while (j + 1 < top_super && cand_start[j + 1] <= c) ++j;
      const int g = static_cast<int>(chosen_super[j]) * superblock + (c - cand_start[j]);
      const double v = warp_page_score(qg, base + static_cast<int64_t>(g) * head_dim, kv_stride, kv_heads,
                                       head_dim, q_heads, scale);
      if (lane == 0) {
        sc[c] = v;
        ix[c] = g;
      }
    }
  }
  __syncthreads();
  block_topm(sc, ix, nc, top_m, selected + static_cast<int64_t>(b) * top_m, red_s, red_i, &chosen);
}

}  // namespace spa

// ---------------------------------------------------------------------------
// C ABI
extern "C" int spa_summaries_build(const spa_kv_layout* kv, int batch, int kv_heads, int head_dim, int dtype,
                                   int n_pages, float* summaries, int superblock, float* super_summaries,
                                   double* page_sums64, spa_stream_t stream) {
  if (!kv || !kv->k || !summaries || batch <= 0 || kv_heads <= 0 || n_pages <= 0 || kv->page_size <= 0)
    return SPA_ERR_INVALID;
  if (head_dim <= 0 || head_dim > spa::kRouterMaxHeadDim || !dtype_ok(dtype)) return SPA_ERR_INVALID;
  if (super_summaries && (superblock <= 0 || !page_sums64)) return SPA_ERR_INVALID;
  const KvAddr addr = make_kv_addr(*kv);
  dim3 grid(n_pages, kv_heads, batch);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SPA_F32:
      spa::page_summaries_kernel<float><<<grid, head_dim, 0, st>>>(static_cast<const float*>(kv->k), addr,
                                                                   head_dim, n_pages, summaries, page_sums64);
      break;
    case SPA_F16:
      spa::page_summaries_kernel<__half><<<grid, head_dim, 0, st>>>(static_cast<const __half*>(kv->k), addr,
                                                                    head_dim, n_pages, summaries, page_sums64);
      break;
    default:
      spa::page_summaries_kernel<__nv_bfloat16><<<grid, head_dim, 0, st>>>(
          static_cast<const __nv_bfloat16*>(kv->k), addr, head_dim, n_pages, summaries, page_sums64);
  }
  SPA_CHECK_CUDA(cudaGetLastError());
  if (super_summaries) {
    const int n_super = (n_pages + superblock - 1) / superblock;
    spa::super_summaries_kernel<<<dim3(n_super, kv_heads, batch), head_dim, 0, st>>>(
        page_sums64, head_dim, n_pages, superblock, kv->page_size, super_summaries);
    SPA_CHECK_CUDA(cudaGetLastError());
  }
  return SPA_OK;
}

namespace {
int router_common_checks(const void* q, int q_dtype, int batch, int q_heads, int kv_heads, int head_dim) {
  if (!q || batch <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads) return SPA_ERR_INVALID;
  if (head_dim <= 0 || head_dim > spa::kRouterMaxHeadDim || !dtype_ok(q_dtype)) return SPA_ERR_INVALID;
  if (kv_heads > spa::kRouterMaxKvHeads) return SPA_ERR_UNSUPPORTED;
  return SPA_OK;
}
}  // namespace

extern "C" int spa_router_topm(const void* q, int q_dtype, int batch, int q_heads, int kv_heads, int head_dim,
                               const float* summaries, int n_pages, double scale, int top_m, int64_t* selected,
                               double* scores_out, spa_stream_t stream) {
  int rc = router_common_checks(q, q_dtype, batch, q_heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!summaries || !selected || n_pages <= 0 || top_m <= 0 || top_m > n_pages) return SPA_ERR_INVALID;
  const size_t smem = sizeof(double) * (kv_heads * head_dim + n_pages) + sizeof(int) * n_pages;
  if (smem > 200 * 1024) return SPA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define SPA_LAUNCH_ROUTER(T)                                                                               \
  do {                                                                                                     \
    if (smem > 48 * 1024)                                                                                  \
      SPA_CHECK_CUDA(spa_set_smem_once(spa::router_topm_kernel<T>, (int)smem));                          \
    spa::router_topm_kernel<T><<<batch, 256, smem, st>>>(static_cast<const T*>(q), q_heads, kv_heads,     \
                                                         head_dim, summaries, n_pages, scale, top_m,      \
                                                         selected, scores_out);                            \
  } while (0)
  if (q_dtype == SPA_F32)
    SPA_LAUNCH_ROUTER(float);
  else if (q_dtype == SPA_F16)
    SPA_LAUNCH_ROUTER(__half);
  else
    SPA_LAUNCH_ROUTER(__nv_bfloat16);
#undef SPA_LAUNCH_ROUTER
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}

extern "C" int spa_router_tree_topm(const void* q, int q_dtype, int batch, int q_heads, int kv_heads,
                                    int head_dim, const float* super_summaries, int n_super,
                                    const float* summaries, int n_pages, int superblock, int top_super,
                                    double scale, int top_m, int64_t* selected, spa_stream_t stream) {
  int rc = router_common_checks(q, q_dtype, batch, q_heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!super_summaries || !summaries || !selected || n_pages <= 0 || superblock <= 0) return SPA_ERR_INVALID;
  if (n_super != (n_pages + superblock - 1) / superblock) return SPA_ERR_INVALID;
  if (top_super <= 0 || top_super > n_super || top_super > 64 || top_m <= 0) return SPA_ERR_INVALID;
  // the smallest possible candidate count: the top_super smallest superblocks
  const int last = n_pages - (n_super - 1) * superblock;
  const int min_cand = (top_super - 1) * superblock + (last < superblock ? last : superblock);
  if (top_m > min_cand) return SPA_ERR_INVALID;
  const int cand_cap = n_super > top_super * superblock ? n_super : top_super * superblock;
  const size_t smem = sizeof(double) * (kv_heads * head_dim + cand_cap) + sizeof(int) * (cand_cap + 1) +
                      sizeof(int64_t) * (top_super + 1);
  if (smem > 200 * 1024) return SPA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define SPA_LAUNCH_TREE(T)                                                                                  \
  do {                                                                                                      \
    if (smem > 48 * 1024)                                                                                   \
      SPA_CHECK_CUDA(spa_set_smem_once(spa::router_tree_kernel<T>, (int)smem));                           \
    spa::router_tree_kernel<T><<<batch, 256, smem, st>>>(static_cast<const T*>(q), q_heads, kv_heads,      \
                                                         head_dim, super_summaries, n_super, summaries,    \
                                                         n_pages, superblock, top_super, scale, top_m,     \
                                                         selected);                                         \
  } while (0)
  if (q_dtype == SPA_F32)
    SPA_LAUNCH_TREE(float);
  else if (q_dtype == SPA_F16)
    SPA_LAUNCH_TREE(__half);
  else
    SPA_LAUNCH_TREE(__nv_bfloat16);
#undef SPA_LAUNCH_TREE
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}
