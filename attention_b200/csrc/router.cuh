// Page summaries and the page router (single level and superblock -> page tree).
//
// Canonical arithmetic (the oracle restates exactly this order, so scores and
// therefore selections are bit-identical):
//   page sum   S[b,h,g,d] = ((K[t0,d] + K[t0+1,d]) + ...) in fp64, tokens in order
//   summary    = fp32(S / page_size)                              (fp64 divide)
//   super sum  = ((S[g0] + S[g0+1]) + ...) over the superblock's pages in order
//   super      = fp32(super sum / (pages_in_super * page_size))
//   qg[kvh,d]  = ((q[h0,d] + q[h0+1,d]) + ...) over the kv head's query heads, fp32
//   dot_kvh    = per lane l: sum_k qg[kvh, l+32k] * summ[kvh, l+32k]  (k ascending,
//                fp32, separate multiply and add), then xor-butterfly over lanes with
//                offsets 16, 8, 4, 2, 1
//   score      = ((dot_0 + dot_1) + ...) over kv heads, / q_heads, * fp32(scale), fp32
// Selection: descending score, ties to the lower page index.  Scores are fp32, the
// precision of the reference's own einsum router.
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

// (score, index) ordering: a beats b when its score is larger, or equal with a lower index.
__device__ __forceinline__ bool beats(float sa, int ia, float sb, int ib) {
  return sa > sb || (sa == sb && ia < ib);
}

// Block-wide top-m over cand_score[0..n) (indices cand_idx[0..n)), written in
// descending order to out[0..m).  Chosen entries are overwritten with -inf and
// index INT_MAX.  Uses red_s / red_i scratch of blockDim.x/32 entries.
__device__ __noinline__ void block_topm(float* cand_score, int* cand_idx, int n, int m, int64_t* out, float* red_s,
                           int* red_i, int* chosen_pos) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int r = 0; r < m; ++r) {
    float bs = -INFINITY;
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
      const float os = __shfl_xor_sync(0xffffffffu, bs, off);
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
// Cluster router.  One cluster of kRouterCluster CTAs per batch row.  Candidate c of a
// level is owned by CTA rank c % kRouterCluster and scored by one warp: each lane loads
// its lane-strided slices of the candidate's summary rows for a batch of kv heads
// (independent loads, one memory round trip), forms the lane partials, and the heads'
// butterflies run interleaved.  Lane 0..7 push the score into the shared memory of the
// CTAs that select from it (st.shared::cluster): after level 1 of the tree every CTA
// selects the same top_super superblocks from the same scores; after the last level rank
// 0 selects the top_m pages.  One cluster barrier per level orders the pushes before the
// selection.  Tree mode: level 1 over superblocks, level 2 over the pages of the chosen
// superblocks.  Both levels run through one copy of the scoring loop: the kernel is
// latency-bound, and its instructions, fetched afresh every step, are part of that.
constexpr int kRouterCluster = 8;
constexpr int kRouterThreads = 256;
constexpr int kRouterKvBatch = 8;  // kv heads per register batch

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

struct RouterArgs {
  const void* q;
  int q_heads, kv_heads, head_dim;
  const float* supers;     // [B, Hkv, n_super, D] (tree mode) or nullptr
  const float* summaries;  // [B, Hkv, n_pages, D]
  int n_super, n_pages, superblock, top_super, top_m;
  float scale;
  int64_t* selected;  // [B, top_m]
  float* scores_out;  // [B, n_pages] (single-level mode) or nullptr
  // promotion refresh gate or nullptr: gate[0] = refresh decision of this step,
  // gate[1] = a selection has been promoted; promoted [B, top_m] holds it
  int32_t* gate = nullptr;
  int64_t* promoted = nullptr;
  // fused step with its query in host memory: q_copy [B, Hq, D] receives a device copy of
  // the query for the decode (rank r of a row's cluster writes the r-th eighth of the row),
  // selected_copy [B, top_m] a second copy of the selection (host memory)
  void* q_copy = nullptr;
  int64_t* selected_copy = nullptr;
  // launched as a programmatic dependent of the kernel that produces its query (the
  // session's copy-in): waits for it before any read.  Its own dependents (the decode)
  // may launch before that wait ends, so they must read the query only after theirs.
  int pdl_wait = 0;
};

// qg (fp32, [Hkv][D]) for batch row b, summed over each kv head's query heads in
// order.  The raw query row [Hq, D] is first copied to shared memory with 16-byte
// loads, four per thread in flight (one memory round trip for rows up to 16 KB).
template <typename T>
__device__ void load_group_query(const T* __restrict__ q, int b, int q_heads, int kv_heads, int head_dim,
                                 T* __restrict__ qraw, float* __restrict__ qg) {
  const int n = q_heads * head_dim;
  const int nvec = n * static_cast<int>(sizeof(T)) / 16;
  const uint4* src = reinterpret_cast<const uint4*>(q + static_cast<int64_t>(b) * n);
  const int nt = static_cast<int>(blockDim.x);
#pragma unroll 1
  for (int v0 = threadIdx.x; v0 < nvec; v0 += 4 * nt) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v0 + u * nt < nvec) r[u] = __ldg(src + v0 + u * nt);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v0 + u * nt < nvec) reinterpret_cast<uint4*>(qraw)[v0 + u * nt] = r[u];
  }
  __syncthreads();
  const int group = (kv_heads & (kv_heads - 1)) == 0 ? q_heads >> (__ffs(kv_heads) - 1) : q_heads / kv_heads;
#pragma unroll 1
  for (int i = threadIdx.x; i < kv_heads * head_dim; i += nt) {
    const int kvh = (head_dim & (head_dim - 1)) == 0 ? i >> (__ffs(head_dim) - 1) : i / head_dim;
    const int d = i - kvh * head_dim;
    float acc = 0.f;
    for (int j = 0; j < group; ++j) acc = __fadd_rn(acc, to_f32(qraw[(kvh * group + j) * head_dim + d]));
    qg[i] = acc;
  }
}

// One warp's view of a candidate: its lane-strided summary values (NS slices of 32,
// head_dim <= 32 * NS) for up to kRouterKvBatch kv heads, in registers.
template <int NS>
struct CandRows {
  float v[kRouterKvBatch][NS];
};

// Rows of kv heads [k0, k0 + kRouterKvBatch) of the candidate whose head-0 row is `base`.
template <int NS>
__device__ __forceinline__ void load_cand_rows(CandRows<NS>& r, const float* base, int64_t kv_stride, int k0,
                                               int kv_heads, int head_dim) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int u = 0; u < kRouterKvBatch; ++u) {
    const bool hv = k0 + u < kv_heads;
    const float* row = base + static_cast<int64_t>(hv ? k0 + u : k0) * kv_stride;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int d = lane + 32 * k;
      r.v[u][k] = (hv && d < head_dim) ? __ldg(row + d) : 0.f;
    }
  }
}

// Adds the kv heads [k0, k0+kRouterKvBatch) of one candidate to `total` in the canonical
// order: lane partials over the lane's slice, xor butterflies, kv heads in order.
template <int NS>
__device__ __forceinline__ float accumulate_cand(const CandRows<NS>& r, const float* qg, int k0, int kv_heads,
                                                 int head_dim, float total) {
  const int lane = threadIdx.x & 31;
  float part[kRouterKvBatch];
#pragma unroll
  for (int u = 0; u < kRouterKvBatch; ++u) {
    const float* qq = qg + (k0 + u < kv_heads ? k0 + u : k0) * head_dim;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int d = lane + 32 * k;
      if (d < head_dim) acc = __fadd_rn(acc, __fmul_rn(qq[d], r.v[u][k]));
    }
    part[u] = acc;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int u = 0; u < kRouterKvBatch; ++u) part[u] = __fadd_rn(part[u], __shfl_xor_sync(0xffffffffu, part[u], off));
#pragma unroll
  for (int u = 0; u < kRouterKvBatch; ++u)
    if (k0 + u < kv_heads) total = __fadd_rn(total, part[u]);
  return total;
}

// T threads (a power of two dividing 32) share one candidate's rank count: candidate i
// goes to out[rank_i], rank_i = number of candidates that beat it.  One pass, one barrier.
__device__ void block_topm_rank(const float* sc, const int* id, int n, int m, int64_t* out) {
  int T = 1;
  while (T < 32 && T * 2 * n <= static_cast<int>(blockDim.x)) T *= 2;
  const int per_round = static_cast<int>(blockDim.x) >> (__ffs(T) - 1);
  for (int base = 0; base < n; base += per_round) {
    // T is a power of two
    const int i = base + (static_cast<int>(threadIdx.x) >> (__ffs(T) - 1)), part = static_cast<int>(threadIdx.x) & (T - 1);
    int r = 0;
    float si = 0.f;
    int ii = 0;
    if (i < n) {
      si = sc[i];
      ii = id[i];
      for (int j = part; j < n; j += T) r += beats(sc[j], id[j], si, ii) ? 1 : 0;
    }
    for (int off = T / 2; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
    if (i < n && part == 0 && r < m) out[r] = ii;
  }
  __syncthreads();
}

__device__ __forceinline__ void select_top(float* sc, int* id, int n, int m, int64_t* out, float* red_s, int* red_i,
                                           int* pos) {
  if (n <= 2048)
    block_topm_rank(sc, id, n, m, out);
  else
    block_topm(sc, id, n, m, out, red_s, red_i, pos);
}

// Candidates of the last level: the pages of the chosen superblocks (tree) or every page.
__host__ __device__ inline int router_level2_cap(const RouterArgs& a) {
  return a.supers ? a.top_super * a.superblock : a.n_pages;
}

// Dynamic shared memory of router_cluster_kernel: chosen [top_super] i64, qg [Hkv*D],
// level-1 scores [n_super], level-2 scores [level-2 cap], ids [max of both], query row.
__host__ __device__ inline size_t router_smem_bytes(const RouterArgs& a, size_t q_row_bytes) {
  const size_t n1 = a.supers ? a.n_super : 0, n2 = router_level2_cap(a);
  const size_t base = sizeof(int64_t) * (a.top_super > 0 ? a.top_super : 1) +
                      sizeof(float) * (static_cast<size_t>(a.kv_heads) * a.head_dim + n1 + n2) +
                      sizeof(int) * ((n1 > n2 ? n1 : n2) + 4);
  return ((base + 15) & ~size_t(15)) + q_row_bytes + 16;
}

// The gated router's reuse step, out of line (it runs only while the gate is closed, and
// the routing path's code stays compact): rank 0 copies the promoted pages into this
// step's selection, and each CTA its eighth of the query row into q_copy when given.
template <typename T>
__device__ __noinline__ void router_reuse_promoted(const int64_t* promoted, int64_t* selected, int64_t* selected_copy,
                                                   const T* q, T* q_copy, int b, int rank, int top_m, int row_elems) {
  if (rank == 0) {
    for (int j = threadIdx.x; j < top_m; j += blockDim.x) {
      const int64_t v = promoted[static_cast<int64_t>(b) * top_m + j];
      selected[static_cast<int64_t>(b) * top_m + j] = v;
      if (selected_copy) selected_copy[static_cast<int64_t>(b) * top_m + j] = v;
    }
  }
  if (q_copy) {
    const int nvec = row_elems * static_cast<int>(sizeof(T)) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(q + static_cast<int64_t>(b) * row_elems);
    uint4* dst = reinterpret_cast<uint4*>(q_copy + static_cast<int64_t>(b) * row_elems);
    const int v0 = nvec * rank / kRouterCluster, v1 = nvec * (rank + 1) / kRouterCluster;
    for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
  }
}

// grid (kRouterCluster, B), cluster (kRouterCluster, 1, 1), block kRouterThreads.
// PIPE (single-level routing, kv heads <= kRouterKvBatch, several candidates per warp):
// each warp requests its next candidate's rows before it scores the current one, so a
// warp's candidates cost one memory round trip instead of one each.
template <typename T, int NS, bool PIPE>
__global__ void __launch_bounds__(kRouterThreads) router_cluster_kernel(const RouterArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int hkv = a.kv_heads, D = a.head_dim;
  const bool tree = a.supers != nullptr;
  const int n1 = tree ? a.n_super : 0, n2 = router_level2_cap(a);
  int64_t* chosen = reinterpret_cast<int64_t*>(smem_raw);                         // [top_super]
  float* qg = reinterpret_cast<float*>(chosen + (a.top_super > 0 ? a.top_super : 1));  // [Hkv*D]
  float* score1 = qg + hkv * D;  // [n1]: every CTA's pushes of level 1
  float* score2 = score1 + n1;   // [n2]: pushes of the last level (read by rank 0)
  int* ids = reinterpret_cast<int*>(score2 + n2);
  T* qraw = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(ids + (n1 > n2 ? n1 : n2) + 4) + 15) & ~uintptr_t(15));
  __shared__ float red_s[kRouterThreads / 32];
  __shared__ int red_i[kRouterThreads / 32];
  __shared__ int chosen_pos;
  __shared__ int cand_start[65];

  pdl_trigger();
  const int b = blockIdx.y;
  const int rank = static_cast<int>(cluster_rank());
  if (a.pdl_wait) pdl_block();  // the copied query (launched as the copy's dependent)
  // every thread arrives now and waits once the query is in: every CTA of the cluster is
  // then running, so pushes into peers' shared memory are safe.  Gated, the arrival waits
  // for the gate's decision (a reusing cluster leaves before any cluster barrier).
  if (!a.gate) cluster_arrive_relaxed();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kRouterThreads / 32;
  const float* sup_tab = tree ? a.supers + static_cast<int64_t>(b) * hkv * a.n_super * D : nullptr;
  const float* page_tab = a.summaries + static_cast<int64_t>(b) * hkv * a.n_pages * D;
  const int64_t sup_stride = static_cast<int64_t>(a.n_super) * D;
  const int64_t page_stride = static_cast<int64_t>(a.n_pages) * D;
  const int first_level = tree ? 1 : 2;
  // the rows of the warp's first candidate (first kv-head batch) are requested before the
  // query row, so both loads are in flight together.  Gated, both were written before the
  // gate kernel started, so they load while the gate decides.
  CandRows<NS> rows;
  int n_cand = tree ? a.n_super : a.n_pages;
  if (rank + warp * kRouterCluster < n_cand)
    load_cand_rows(rows, (tree ? sup_tab : page_tab) + static_cast<int64_t>(rank + warp * kRouterCluster) * D,
                   tree ? sup_stride : page_stride, 0, hkv, D);
  load_group_query(static_cast<const T*>(a.q), b, a.q_heads, hkv, D, qraw, qg);
  if (a.gate) {
    pdl_block();  // the gate kernel's decision (launched as its dependent)
    if (a.gate[0] == 0 && a.gate[1] != 0) {
      // promotion reuse: the refresh gate is closed, so the promoted pages are this step's
      // selection and no summary beyond the first rows is read.  The flags are the same for
      // every CTA, so whole clusters leave here together, before any cluster barrier.
      router_reuse_promoted<T>(a.promoted, a.selected, a.selected_copy, static_cast<const T*>(a.q),
                               static_cast<T*>(a.q_copy), b, rank, a.top_m, a.q_heads * a.head_dim);
      return;
    }
    cluster_arrive_relaxed();
  }
  __syncthreads();
  if (a.q_copy) {
    // the decode reads the query from q_copy: this CTA's eighth of the staged row
    const int nvec = a.q_heads * D * static_cast<int>(sizeof(T)) / 16;
    uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(a.q_copy) + static_cast<int64_t>(b) * a.q_heads * D);
    const int v0 = nvec * rank / kRouterCluster, v1 = nvec * (rank + 1) / kRouterCluster;
    for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = reinterpret_cast<const uint4*>(qraw)[v];
  }
  cluster_wait();
  auto page_of = [&](int c) {  // page of level-2 candidate c (tree)
    int j = 0;
    while (j + 1 < a.top_super && cand_start[j + 1] <= c) ++j;
    return static_cast<int>(chosen[j]) * a.superblock + (c - cand_start[j]);
  };
#pragma unroll 1
  for (int level = first_level; level <= 2; ++level) {
    const float* tab = level == 1 ? sup_tab : page_tab;
    const int64_t kv_stride = level == 1 ? sup_stride : page_stride;
    float* dst = level == 1 ? score1 : score2;
    const int nl = n_cand > rank ? (n_cand - 1 - rank) / kRouterCluster + 1 : 0;
#pragma unroll 1
    for (int i = warp; i < nl; i += nwarps) {
      const int c = rank + i * kRouterCluster;
      const int g = (level == 2 && tree) ? page_of(c) : c;
      const float* base = tab + static_cast<int64_t>(g) * D;
      float total = 0.f;
      if constexpr (PIPE) {
        // rows holds this candidate (requested with the query, or in the previous pass)
        CandRows<NS> next;
        if (i + nwarps < nl)
          load_cand_rows(next, tab + static_cast<int64_t>(c + nwarps * kRouterCluster) * D, kv_stride, 0, hkv, D);
        total = accumulate_cand(rows, qg, 0, hkv, D, total);
        rows = next;
      } else {
#pragma unroll 1
        for (int k0 = 0; k0 < hkv; k0 += kRouterKvBatch) {
          if (level != first_level || i != warp || k0 != 0) load_cand_rows(rows, base, kv_stride, k0, hkv, D);
          total = accumulate_cand(rows, qg, k0, hkv, D, total);
        }
      }
      const float v = __fmul_rn(__fdiv_rn(total, static_cast<float>(a.q_heads)), a.scale);
      if (level == 1) {
        if (lane < kRouterCluster) st_dsmem(dst + c, lane, v);  // every CTA selects superblocks
      } else if (lane == 0) {
        st_dsmem(dst + c, 0, v);  // rank 0 selects pages
        if (a.scores_out) a.scores_out[static_cast<int64_t>(b) * a.n_pages + c] = v;
      }
    }
    cluster_barrier();  // this level's pushes are visible to the selecting CTAs
    if (level == 1) {
      for (int c = threadIdx.x; c < n_cand; c += blockDim.x) ids[c] = c;
      __syncthreads();
      select_top(score1, ids, n_cand, a.top_super, chosen, red_s, red_i, &chosen_pos);
      if (threadIdx.x == 0) {
        int n = 0;
        for (int j = 0; j < a.top_super; ++j) {
          cand_start[j] = n;
          const int g0 = static_cast<int>(chosen[j]) * a.superblock, g1 = min(g0 + a.superblock, a.n_pages);
          n += max(0, g1 - g0);
        }
        cand_start[a.top_super] = n;
      }
      __syncthreads();
      n_cand = cand_start[a.top_super];
    } else if (rank == 0) {
      for (int c = threadIdx.x; c < n_cand; c += blockDim.x) ids[c] = tree ? page_of(c) : c;
      __syncthreads();
      select_top(score2, ids, n_cand, a.top_m, a.selected + static_cast<int64_t>(b) * a.top_m, red_s, red_i,
                 &chosen_pos);
      if (a.selected_copy) {
        __syncthreads();
        for (int j = threadIdx.x; j < a.top_m; j += blockDim.x)
          a.selected_copy[static_cast<int64_t>(b) * a.top_m + j] = a.selected[static_cast<int64_t>(b) * a.top_m + j];
      }
    }
  }
  if (a.gate && rank == 0) {
    // a routed step becomes the promoted selection
    __syncthreads();
    for (int j = threadIdx.x; j < a.top_m; j += blockDim.x)
      a.promoted[static_cast<int64_t>(b) * a.top_m + j] = a.selected[static_cast<int64_t>(b) * a.top_m + j];
    if (threadIdx.x == 0) a.gate[1] = 1;
  }
}

template <typename T, int NS, bool PIPE>
int launch_router_ns(const RouterArgs& a, int batch, cudaStream_t st) {
  const size_t smem = router_smem_bytes(a, static_cast<size_t>(a.q_heads) * a.head_dim * sizeof(T));
  if (smem > 200 * 1024) return SPA_ERR_UNSUPPORTED;
  auto kern = router_cluster_kernel<T, NS, PIPE>;
  SPA_CHECK_CUDA(spa_set_smem_once(kern, static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kRouterCluster, batch, 1);
  cfg.blockDim = dim3(kRouterThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRouterCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // gated: launched as a programmatic dependent of the gate kernel, which it waits for
  // (griddepcontrol.wait) before reading the decision
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (a.gate || a.pdl_wait) ? 2 : 1;
  SPA_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  return SPA_OK;
}

// One instantiation per head_dim class: the lane slices of a summary row are unrolled
// exactly, so the scoring loop carries no dead slices.
template <typename T>
int launch_router(const RouterArgs& a, int batch, cudaStream_t st) {
  // single level with more candidates than one per warp: prefetching scoring loop
  const bool pipe = !a.supers && a.kv_heads <= kRouterKvBatch && a.n_pages > kRouterCluster * (kRouterThreads / 32);
  if (pipe) {
    if (a.head_dim <= 32) return launch_router_ns<T, 1, true>(a, batch, st);
    if (a.head_dim <= 64) return launch_router_ns<T, 2, true>(a, batch, st);
    if (a.head_dim <= 128) return launch_router_ns<T, 4, true>(a, batch, st);
    return launch_router_ns<T, 8, true>(a, batch, st);
  }
  if (a.head_dim <= 32) return launch_router_ns<T, 1, false>(a, batch, st);
  if (a.head_dim <= 64) return launch_router_ns<T, 2, false>(a, batch, st);
  if (a.head_dim <= 128) return launch_router_ns<T, 4, false>(a, batch, st);
  return launch_router_ns<T, 8, false>(a, batch, st);
}

// ---------------------------------------------------------------------------
// Periodic causal router: grid (U, H, B), block 256.  Update u routes the query at
// position (u+1)*stride-1 of head h against that head's block summaries, over the
// blocks that end at or before it; top-m by the canonical fp32 score of one head
// (lane partials + butterfly), ties to the lower block, unfilled slots -1.
// Reference: periodic_router (triton_prefill_router_overhead.py:16-34).
template <typename T>
__global__ void __launch_bounds__(256) periodic_router_kernel(const T* __restrict__ q, int seq_len, int head_dim,
                                                              const float* __restrict__ summaries, int n_blocks,
                                                              int block_size, int stride, int top_m,
                                                              int64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int u = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = gridDim.y, U = gridDim.x;
  float* sc = reinterpret_cast<float*>(smem_raw);   // [n_blocks]
  int* id = reinterpret_cast<int*>(sc + n_blocks);   // [n_blocks]
  float* qv = reinterpret_cast<float*>(id + n_blocks);  // [head_dim]
  const int pos = (u + 1) * stride - 1;
  const int64_t bh = static_cast<int64_t>(b) * H + h;
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) qv[d] = to_f32(q[(bh * seq_len + pos) * head_dim + d]);
  __syncthreads();
  const int avail = min(n_blocks, (pos + 1) / block_size);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int g = warp; g < avail; g += nwarps) {
    const float* sv = summaries + (bh * n_blocks + g) * head_dim;
    float part = 0.f;
    for (int d = lane; d < head_dim; d += 32) part = __fadd_rn(part, __fmul_rn(qv[d], __ldg(sv + d)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
    if (lane == 0) {
      sc[g] = __fadd_rn(0.f, part);
      id[g] = g;
    }
  }
  __syncthreads();
  int64_t* o = out + (bh * U + u) * top_m;
  const int cnt = min(top_m, avail);
  for (int j = cnt + threadIdx.x; j < top_m; j += blockDim.x) o[j] = -1;
  if (cnt > 0) {
    for (int i = threadIdx.x; i < avail; i += blockDim.x) {
      const float si = sc[i];
      int r = 0;
      for (int j = 0; j < avail; ++j) r += beats(sc[j], id[j], si, i) ? 1 : 0;
      if (r < cnt) o[r] = i;
    }
  }
}


// Tiled form of the periodic router for top_m <= MCAP: a CTA (8 warps) routes kPrUpdates
// consecutive updates of one head, so each block summary is read once for all of them;
// the scores are the canonical ones above (lane partials over d = lane + 32k in order,
// butterfly, __fadd_rn(0, .)), and each update's top-m comes from per-lane sorted lists
// of MCAP entries merged across the warp, in the same (score desc, block asc) order.
constexpr int kPrUpdates = 8;

template <typename T, int NS, int MCAP>
__global__ void __launch_bounds__(256) periodic_router_tiled_kernel(const T* __restrict__ q, int seq_len,
                                                                     int head_dim,
                                                                     const float* __restrict__ summaries,
                                                                     int n_blocks, int block_size, int stride,
                                                                     int top_m, int64_t* __restrict__ out) {
  extern __shared__ __align__(16) float pr_smem[];
  const int h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
  const int U = seq_len / stride;
  const int u0 = blockIdx.x * kPrUpdates;
  const int nu = min(kPrUpdates, U - u0);
  const int64_t bh = static_cast<int64_t>(b) * H + h;
  float* qv = pr_smem;                                  // [kPrUpdates][32 * NS]
  float* sc = pr_smem + kPrUpdates * 32 * NS;           // [kPrUpdates][n_blocks]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto avail_of = [&](int u) { return min(n_blocks, (u + 1) * stride / block_size); };
  for (int i = threadIdx.x; i < kPrUpdates * 32 * NS; i += blockDim.x) {
    const int u = i / (32 * NS), d = i - u * (32 * NS);
    const int pos = (u0 + u + 1) * stride - 1;
    qv[i] = (u < nu && d < head_dim) ? to_f32(q[(bh * seq_len + pos) * head_dim + d]) : 0.f;
  }
  __syncthreads();
  int av[kPrUpdates];
#pragma unroll
  for (int u = 0; u < kPrUpdates; ++u) av[u] = u < nu ? avail_of(u0 + u) : 0;
  const int max_av = avail_of(u0 + nu - 1);  // availability grows with u
  for (int g = warp; g < max_av; g += 8) {
    const float* sv = summaries + (bh * n_blocks + g) * head_dim;
    float s[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) s[k] = (lane + 32 * k < head_dim) ? __ldg(sv + lane + 32 * k) : 0.f;
    float part[kPrUpdates];
#pragma unroll
    for (int u = 0; u < kPrUpdates; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < NS; ++k)
        if (lane + 32 * k < head_dim) acc = __fadd_rn(acc, __fmul_rn(qv[u * 32 * NS + lane + 32 * k], s[k]));
      part[u] = acc;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < kPrUpdates; ++u) part[u] = __fadd_rn(part[u], __shfl_xor_sync(0xffffffffu, part[u], off));
    if (lane == 0) {
#pragma unroll
      for (int u = 0; u < kPrUpdates; ++u)
        if (g < av[u]) sc[static_cast<int64_t>(u) * n_blocks + g] = __fadd_rn(0.f, part[u]);
    }
  }
  __syncthreads();
  if (warp >= nu) return;
  // warp `warp` selects for update u0 + warp
  const int avail = av[warp];
  const float* su = sc + static_cast<int64_t>(warp) * n_blocks;
  int64_t* o = out + (bh * U + u0 + warp) * top_m;
  const int cnt = min(top_m, avail);
  for (int j = cnt + lane; j < top_m; j += 32) o[j] = -1;
  float ls[MCAP];
  int li[MCAP];
#pragma unroll
  for (int k = 0; k < MCAP; ++k) {
    ls[k] = -INFINITY;
    li[k] = 0x7fffffff;
  }
  for (int g = lane; g < avail; g += 32) {
    float cs = su[g];
    int ci = g;
#pragma unroll
    for (int k = 0; k < MCAP; ++k) {
      if (beats(cs, ci, ls[k], li[k])) {
        const float ts = ls[k];
        const int ti = li[k];
        ls[k] = cs;
        li[k] = ci;
        cs = ts;
        ci = ti;
      }
    }
  }
  for (int r = 0; r < cnt; ++r) {
    float bs = ls[0];
    int bi = li[0], bl = lane;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off), ol = __shfl_xor_sync(0xffffffffu, bl, off);
      if (beats(os, oi, bs, bi)) {
        bs = os;
        bi = oi;
        bl = ol;
      }
    }
    if (lane == 0) o[r] = bi;
    if (lane == bl) {
#pragma unroll
      for (int k = 0; k + 1 < MCAP; ++k) {
        ls[k] = ls[k + 1];
        li[k] = li[k + 1];
      }
      ls[MCAP - 1] = -INFINITY;
      li[MCAP - 1] = 0x7fffffff;
    }
  }
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
  // the query row is staged with 16-byte loads
  const size_t qbytes = static_cast<size_t>(q_heads) * head_dim * dtype_size(q_dtype);
  if (reinterpret_cast<uintptr_t>(q) % 16 != 0 || qbytes % 16 != 0 || qbytes > 64 * 1024) return SPA_ERR_UNSUPPORTED;
  return SPA_OK;
}
}  // namespace

namespace spa {
int router_topm_impl(const void* q, int q_dtype, int batch, int q_heads, int kv_heads, int head_dim,
                     const float* summaries, int n_pages, double scale, int top_m, int64_t* selected,
                     float* scores_out, int32_t* gate, int64_t* promoted, spa_stream_t stream,
                     void* q_copy, int64_t* selected_copy, bool pdl_wait) {
  if ((gate == nullptr) != (promoted == nullptr)) return SPA_ERR_INVALID;
  int rc = router_common_checks(q, q_dtype, batch, q_heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!summaries || !selected || n_pages <= 0 || top_m <= 0 || top_m > n_pages) return SPA_ERR_INVALID;
  if (batch > 65535) return SPA_ERR_UNSUPPORTED;
  spa::RouterArgs a;
  a.q = q;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.head_dim = head_dim;
  a.supers = nullptr;
  a.summaries = summaries;
  a.n_super = 0;
  a.n_pages = n_pages;
  a.superblock = 0;
  a.top_super = 0;
  a.top_m = top_m;
  a.scale = static_cast<float>(scale);
  a.selected = selected;
  a.scores_out = scores_out;
  a.gate = gate;
  a.promoted = promoted;
  a.q_copy = q_copy;
  a.selected_copy = selected_copy;
  a.pdl_wait = pdl_wait;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (q_dtype == SPA_F32) return spa::launch_router<float>(a, batch, st);
  if (q_dtype == SPA_F16) return spa::launch_router<__half>(a, batch, st);
  return spa::launch_router<__nv_bfloat16>(a, batch, st);
}

int router_tree_impl(const void* q, int q_dtype, int batch, int q_heads, int kv_heads, int head_dim,
                     const float* super_summaries, int n_super, const float* summaries, int n_pages, int superblock,
                     int top_super, double scale, int top_m, int64_t* selected, int32_t* gate, int64_t* promoted,
                     spa_stream_t stream, void* q_copy, int64_t* selected_copy, bool pdl_wait) {
  if ((gate == nullptr) != (promoted == nullptr)) return SPA_ERR_INVALID;
  int rc = router_common_checks(q, q_dtype, batch, q_heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!super_summaries || !summaries || !selected || n_pages <= 0 || superblock <= 0) return SPA_ERR_INVALID;
  if (n_super != (n_pages + superblock - 1) / superblock) return SPA_ERR_INVALID;
  if (top_super <= 0 || top_super > n_super || top_super > 64 || top_m <= 0) return SPA_ERR_INVALID;
  // the smallest possible candidate count: the top_super smallest superblocks
  const int last = n_pages - (n_super - 1) * superblock;
  const int min_cand = (top_super - 1) * superblock + (last < superblock ? last : superblock);
  if (top_m > min_cand) return SPA_ERR_INVALID;
  if (batch > 65535) return SPA_ERR_UNSUPPORTED;
  spa::RouterArgs a;
  a.q = q;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.head_dim = head_dim;
  a.supers = super_summaries;
  a.summaries = summaries;
  a.n_super = n_super;
  a.n_pages = n_pages;
  a.superblock = superblock;
  a.top_super = top_super;
  a.top_m = top_m;
  a.scale = static_cast<float>(scale);
  a.selected = selected;
  a.scores_out = nullptr;
  a.gate = gate;
  a.promoted = promoted;
  a.q_copy = q_copy;
  a.selected_copy = selected_copy;
  a.pdl_wait = pdl_wait;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (q_dtype == SPA_F32) return spa::launch_router<float>(a, batch, st);
  if (q_dtype == SPA_F16) return spa::launch_router<__half>(a, batch, st);
  return spa::launch_router<__nv_bfloat16>(a, batch, st);
}
}  // namespace spa

extern "C" int spa_router_topm(const void* q, int q_dtype, int batch, int q_heads, int kv_heads, int head_dim,
                               const float* summaries, int n_pages, double scale, int top_m, int64_t* selected,
                               float* scores_out, spa_stream_t stream) {
  return spa::router_topm_impl(q, q_dtype, batch, q_heads, kv_heads, head_dim, summaries, n_pages, scale, top_m,
                               selected, scores_out, nullptr, nullptr, stream, nullptr, nullptr, false);
}

extern "C" int spa_router_topm_gated(const void* q, int q_dtype, int batch, int q_heads, int kv_heads, int head_dim,
                                     const float* summaries, int n_pages, double scale, int top_m, int64_t* selected,
                                     int32_t* gate, int64_t* promoted, spa_stream_t stream) {
  if (!gate || !promoted) return SPA_ERR_INVALID;
  return spa::router_topm_impl(q, q_dtype, batch, q_heads, kv_heads, head_dim, summaries, n_pages, scale, top_m,
                               selected, nullptr, gate, promoted, stream, nullptr, nullptr, false);
}

extern "C" int spa_router_tree_topm(const void* q, int q_dtype, int batch, int q_heads, int kv_heads,
                                    int head_dim, const float* super_summaries, int n_super,
                                    const float* summaries, int n_pages, int superblock, int top_super,
                                    double scale, int top_m, int64_t* selected, spa_stream_t stream) {
  return spa::router_tree_impl(q, q_dtype, batch, q_heads, kv_heads, head_dim, super_summaries, n_super, summaries,
                               n_pages, superblock, top_super, scale, top_m, selected, nullptr, nullptr, stream, nullptr,
                               nullptr, false);
}

extern "C" int spa_router_tree_topm_gated(const void* q, int q_dtype, int batch, int q_heads, int kv_heads,
                                          int head_dim, const float* super_summaries, int n_super,
                                          const float* summaries, int n_pages, int superblock, int top_super,
                                          double scale, int top_m, int64_t* selected, int32_t* gate,
                                          int64_t* promoted, spa_stream_t stream) {
  if (!gate || !promoted) return SPA_ERR_INVALID;
  return spa::router_tree_impl(q, q_dtype, batch, q_heads, kv_heads, head_dim, super_summaries, n_super, summaries,
                               n_pages, superblock, top_super, scale, top_m, selected, gate, promoted, stream, nullptr,
                               nullptr, false);
}

extern "C" int spa_periodic_router(const void* q, int q_dtype, int batch, int heads, int seq_len, int head_dim,
                                   const float* summaries, int n_blocks, int block_size, int router_stride,
                                   int top_m, int64_t* out, spa_stream_t stream) {
  if (!q || !summaries || !out || !dtype_ok(q_dtype) || batch <= 0 || heads <= 0 || seq_len <= 0) return SPA_ERR_INVALID;
  if (head_dim <= 0 || head_dim > 256 || n_blocks <= 0 || block_size <= 0 || router_stride <= 0 || top_m <= 0)
    return SPA_ERR_INVALID;
  const int U = seq_len / router_stride;
  if (U <= 0) return SPA_ERR_INVALID;
  if (heads > 65535 || batch > 65535) return SPA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // tiled form: top_m <= 16 and the scores of kPrUpdates updates in shared memory
  // NS: the kernel's slices of 32 (2, 4 or 8), which also size its query rows in shared memory
  const int ns = head_dim <= 64 ? 2 : head_dim <= 128 ? 4 : 8;
  const size_t tsmem = sizeof(float) * spa::kPrUpdates * (32 * static_cast<size_t>(ns) + n_blocks);
  if (top_m <= 16 && tsmem <= 200 * 1024) {
    dim3 tgrid((U + spa::kPrUpdates - 1) / spa::kPrUpdates, heads, batch);
#define SPA_LAUNCH_PR_TILED(T, NS, MC)                                                                      \
  do {                                                                                                      \
    auto kern = spa::periodic_router_tiled_kernel<T, NS, MC>;                                               \
    SPA_CHECK_CUDA(spa_set_smem_once(kern, static_cast<int>(tsmem)));                                       \
    kern<<<tgrid, 256, tsmem, st>>>(static_cast<const T*>(q), seq_len, head_dim, summaries, n_blocks,       \
                                    block_size, router_stride, top_m, out);                                 \
  } while (0)
#define SPA_LAUNCH_PR_NS(T, MC)                \
  do {                                         \
    if (ns == 2)                               \
      SPA_LAUNCH_PR_TILED(T, 2, MC);           \
    else if (ns == 4)                          \
      SPA_LAUNCH_PR_TILED(T, 4, MC);           \
    else                                       \
      SPA_LAUNCH_PR_TILED(T, 8, MC);           \
  } while (0)
#define SPA_LAUNCH_PR_M(T)                     \
  do {                                         \
    if (top_m <= 4)                            \
      SPA_LAUNCH_PR_NS(T, 4);                  \
    else                                       \
      SPA_LAUNCH_PR_NS(T, 16);                 \
  } while (0)
    if (q_dtype == SPA_F32)
      SPA_LAUNCH_PR_M(float);
    else if (q_dtype == SPA_F16)
      SPA_LAUNCH_PR_M(__half);
    else
      SPA_LAUNCH_PR_M(__nv_bfloat16);
#undef SPA_LAUNCH_PR_M
#undef SPA_LAUNCH_PR_NS
#undef SPA_LAUNCH_PR_TILED
    SPA_CHECK_CUDA(cudaGetLastError());
    return SPA_OK;
  }
  const size_t smem = sizeof(float) * n_blocks + sizeof(int) * n_blocks + sizeof(float) * head_dim + 16;
  if (smem > 200 * 1024) return SPA_ERR_UNSUPPORTED;
  dim3 grid(U, heads, batch);
#define SPA_LAUNCH_PERIODIC(T)                                                                              \
  do {                                                                                                      \
    SPA_CHECK_CUDA(spa_set_smem_once(spa::periodic_router_kernel<T>, static_cast<int>(smem)));              \
    spa::periodic_router_kernel<T><<<grid, 256, smem, st>>>(static_cast<const T*>(q), seq_len, head_dim,     \
                                                            summaries, n_blocks, block_size, router_stride,  \
                                                            top_m, out);                                      \
  } while (0)
  if (q_dtype == SPA_F32)
    SPA_LAUNCH_PERIODIC(float);
  else if (q_dtype == SPA_F16)
    SPA_LAUNCH_PERIODIC(__half);
  else
    SPA_LAUNCH_PERIODIC(__nv_bfloat16);
#undef SPA_LAUNCH_PERIODIC
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}
