// Split-K paged decode attention (dense over a context, or local window + selected pages).
//
// Reference kernels: paged_decode_attention_kernel (triton_paged_attention.py:20-53) and
// paged_gather_decode_attention_kernel (:84-136).  Both stream candidates through one
// online softmax per (b, h); candidate c of the gather kernel is token ctx-W+c for c < W,
// else sel[b,(c-W)//P]*P + (c-W)%P (:111-122).  Here the candidates are cut into chunks of
// 64 tokens that never straddle a page, every (b, kv head) is split over `nsplit` CTAs,
// and each CTA serves all `group` query heads that share the kv head (GQA packing).
//
// Fast path (bf16/fp16, D in {64,128}): one producer warp streams K and V chunks with
// 2D TMA loads (128-byte swizzle) into a STAGES-deep mbarrier ring; four consumer warps
// each take 16 tokens of a chunk and run QK^T and PV on mma.sync m16n8k16 with the
// query heads as the (zero-padded) M dimension.  Partials (normalised O, log2-sum-exp)
// go to the workspace and a small kernel merges the splits.
#pragma once

#include <utility>

#include "common.cuh"
#include "router.cuh"

namespace spa {

// In-kernel routing (the route instantiation of decode_mma_kernel): the router inputs of
// the sequences the decode serves.  The query rows a.q hold q_heads heads of head_dim D
// for every sequence; the summaries cover kv_heads kv heads (all heads of the sequence,
// also when the decode covers only a slice of them).
struct FusedRoute {
  int q_heads, kv_heads;
  const float* supers;  // [B, kv_heads, n_super, D] (two levels) or nullptr (one level)
  int n_super, superblock, top_super;
  const float* summaries;  // [B, kv_heads, n_pages, D]
  int n_pages;
  float scale;
  int64_t* selected;       // [B, top_m]: the selection, written once per sequence
  int64_t* selected_copy;  // [B, top_m] second copy (host memory of a session) or nullptr
};

struct DecodeArgs {
  const void* q;
  void* out;
  int B, Hq, Hkv, group, D;
  // query head h (of Hq) of sequence b is row b * q_batch_heads + q_head_offset + h of a.q:
  // q_batch_heads = Hq and q_head_offset = 0 unless the decode covers a kv-head slice of
  // a wider query row
  int q_batch_heads, q_head_offset;
  KvAddr addr;
  const int32_t* ctx_lens;
  int local_window;
  const int64_t* selected;
  int top_m;
  // 0: selected[] are logical pages of page_size tokens.  > 0: selected[] are first
  // tokens of spans of span_len tokens (span_gather_decode_attention).
  int span_len;
  int nsplit;
  float scale_log2;  // softmax scale * log2(e)
  float scale;
  float* part_o;    // [B*Hq, nsplit, D]       (global-merge path)
  float* part_lse;  // [B*Hq, nsplit] log2-sum-exp
  int cluster_merge;  // splits of a pair form one cluster and merge through DSMEM
  // Launched right after the router (programmatic dependent launch) with every input
  // except `selected` already complete: local-window chunks may stream before the
  // router finishes.  Otherwise the kernel waits for its predecessor before any read.
  int early_local;
  // with early_local: the query is written by the kernel this one overlaps (the router's
  // device copy of a query held in host memory), so the consumers read it after the wait
  int q_after_wait;
  FusedRoute route;  // read by the route instantiation only
};

struct ChunkPlan {
  int lo, hi, seg_a, n_seg, cpp, n_total, ctx;
};

__device__ __forceinline__ ChunkPlan make_plan_ctx(const DecodeArgs& a, int ctx, int chunk) {
  ChunkPlan p;
  p.ctx = ctx;
  int lo = 0;
  if (a.selected || a.local_window > 0) lo = max(0, ctx - max(a.local_window, 0));
  p.lo = lo;
  p.hi = ctx;
  p.seg_a = (lo / chunk) * chunk;
  p.n_seg = ctx > lo ? (ctx - p.seg_a + chunk - 1) / chunk : 0;
  // span starts are arbitrary tokens: their chunks are chunk-aligned, so one extra chunk
  p.cpp = !a.selected ? 0 : a.span_len > 0 ? (a.span_len + chunk - 1) / chunk + 1 : (a.addr.page_size + chunk - 1) / chunk;
  p.n_total = p.n_seg + (a.selected ? a.top_m * p.cpp : 0);
  return p;
}
__device__ __forceinline__ ChunkPlan make_plan(const DecodeArgs& a, int b, int chunk) {
  return make_plan_ctx(a, a.ctx_lens[b], chunk);
}

struct ChunkInfo {
  int t0, vlo, vhi;  // tokens [t0, t0+chunk) are loaded; [vlo, vhi) are candidates
};

// sel_row: the sequence's selected ids (a.selected + b * top_m, or a copy of them)
// Reads every field of the argument block once.  Kernel parameters live in the constant
// bank; a field first read after the wait for the router would add a constant-cache miss
// to that path, so each thread touches them all at kernel start.
__device__ __forceinline__ void touch_args(const DecodeArgs& a) {
  uint64_t x = reinterpret_cast<uint64_t>(a.q) ^ reinterpret_cast<uint64_t>(a.out) ^
               reinterpret_cast<uint64_t>(a.ctx_lens) ^ reinterpret_cast<uint64_t>(a.selected) ^
               reinterpret_cast<uint64_t>(a.part_o) ^ reinterpret_cast<uint64_t>(a.part_lse) ^
               reinterpret_cast<uint64_t>(a.addr.page_table);
  x ^= static_cast<uint64_t>(a.addr.batch_stride_rows ^ a.addr.page_stride_rows ^ a.addr.head_stride_rows ^
                             a.addr.total_rows);
  x ^= static_cast<uint64_t>(a.B ^ a.Hq ^ a.Hkv ^ a.group ^ a.D ^ a.addr.table_stride ^ a.addr.page_size ^
                             a.local_window ^ a.top_m ^ a.span_len ^ a.nsplit ^ a.cluster_merge ^ a.early_local ^
                             a.q_after_wait);
  x ^= static_cast<uint64_t>(__float_as_uint(a.scale_log2) ^ __float_as_uint(a.scale));
  asm volatile("" ::"l"(x));
}

__device__ __forceinline__ ChunkInfo chunk_info(const DecodeArgs& a, const ChunkPlan& p, const int64_t* sel_row,
                                                int k, int chunk) {
  ChunkInfo c;
  if (k < p.n_seg) {
    c.t0 = p.seg_a + k * chunk;
    c.vlo = max(c.t0, p.lo);
    c.vhi = min(c.t0 + chunk, p.hi);
  } else {
    const int kk = k - p.n_seg;
    // chunks per page is a power of two for power-of-two pages: a shift, not a division
    const int j = (p.cpp & (p.cpp - 1)) == 0 ? kk >> (__ffs(p.cpp) - 1) : kk / p.cpp, ci = kk - j * p.cpp;
    const int64_t lp = sel_row[j];
    const int P = a.addr.page_size;
    if (a.span_len > 0) {
      // span [lp, lp + span_len) in chunk-aligned pieces, clipped to the context
      if (lp < 0 || lp >= p.ctx) {
        if (lp >= p.ctx) spa_raise(SPA_DEVERR_BAD_PAGE);
        c.t0 = 0;
        c.vlo = c.vhi = 0;
      } else {
        const int start = static_cast<int>(lp);
        c.t0 = (start / chunk) * chunk + ci * chunk;
        c.vlo = max(c.t0, start);
        c.vhi = min(min(c.t0 + chunk, start + a.span_len), p.ctx);
        if (c.vlo >= c.vhi) c.vlo = c.vhi = 0;
      }
      return c;
    }
    if (lp < 0 || lp * P >= p.ctx) {
      // -1 marks an unfilled slot; anything else past the context is an input error
      if (lp >= 0) spa_raise(SPA_DEVERR_BAD_PAGE);
      c.t0 = 0;
      c.vlo = c.vhi = 0;
    } else {
      c.t0 = static_cast<int>(lp) * P + ci * chunk;
      c.vlo = c.t0;
      c.vhi = min(min(c.t0 + chunk, static_cast<int>(lp + 1) * P), p.ctx);
    }
  }
  return c;
}

// ---------------------------------------------------------------------------
// Fast path
constexpr int kChunk = 64;
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;

template <int D, int STAGES>
struct DecodeSmem {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = kChunk * 128;
  static constexpr int kKvBytes = kBoxes * kBoxBytes;
  static constexpr int kStageBytes = 2 * kKvBytes;
  static constexpr int kRingBytes = STAGES * kStageBytes;
  static constexpr int kTabCap = 2048;  // page-table entries prefetched into shared memory
  static constexpr int kSelCap = 32;    // selected ids prefetched into shared memory
  // + barriers, chunk info, page table, selected ids (the cluster receive buffer follows)
  // (+32: the routing and merge exchange barriers)
  static constexpr int kBytes = kRingBytes + STAGES * 16 + STAGES * 16 + 32 + kTabCap * 4 + kSelCap * 8 + 1024;
};

template <int D>
__device__ __forceinline__ uint32_t swz_addr(uint32_t base, int row, int c16) {
  // 16-byte chunk c16 of token row `row` in a [kChunk rows x 128 B] box array with SWIZZLE_128B
  constexpr int kBoxBytes = kChunk * 128;
  return base + (c16 >> 3) * kBoxBytes + row * 128 + (((c16 & 7) ^ (row & 7)) << 4);
}

// ---------------------------------------------------------------------------
// In-kernel routing.  The splits of one (sequence, kv head) pair form a cluster of ns CTAs;
// the cluster selects its sequence's pages itself, with the arithmetic of
// router_cluster_kernel (query heads summed per kv head, lane-strided partial dots and
// xor butterflies, kv heads in order, / q_heads, * scale; ties to the lower page), so
// the pages are the ones spa_router_tree_topm / spa_router_topm return, bit for bit.
// Every cluster serving the same sequence computes the same selection from the same
// inputs: no exchange between clusters, no grid-wide wait.  Candidate c of a level is
// scored by CTA c % ns (one warp per candidate, up to CB candidates' rows in flight per
// warp) and its score pushed into every CTA of the cluster; after one cluster barrier per
// level every CTA ranks the same scores.  Scratch: the last ring stage, free until the
// producer issues its first chunk after the selection.
template <int NS>
struct RouteCfg {
  static constexpr int kCB = NS >= 8 ? 1 : 8 / NS;  // candidates per warp in flight
};

__host__ __device__ inline size_t route_align16(size_t x) { return (x + 15) & ~size_t(15); }

// The query row is staged through the consumer warps' registers: at most this many 16-byte
// pieces per consumer thread (q_heads * head_dim * elem <= kRouteQVec * 16 * 128).
constexpr int kRouteQVec = 4;
constexpr int kRouteStagers = 128;  // the consumer warps

// The router's first loads, issued at kernel entry together with the split plan's: this
// warp's first batch of first-level candidate rows and this thread's pieces of the query
// row (consumed by fused_route).
template <int NS>
struct RoutePrefetch {
  CandRows<NS> rows[RouteCfg<NS>::kCB];
  uint4 q[kRouteQVec];
};

template <typename T, int NS>
__device__ __forceinline__ void route_prefetch(const DecodeArgs& a, int b, int rank, int ns, RoutePrefetch<NS>& pf) {
  constexpr int CB = RouteCfg<NS>::kCB;
  const FusedRoute& r = a.route;
  constexpr int D = NS * 32;  // the kernel's head_dim
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5;
  // every route field is read here once: parameters sit in the constant bank, and a field
  // first read after a cluster barrier would put a constant-cache miss on the chain
  uint64_t x = reinterpret_cast<uint64_t>(r.supers) ^ reinterpret_cast<uint64_t>(r.summaries) ^
               reinterpret_cast<uint64_t>(r.selected) ^ reinterpret_cast<uint64_t>(r.selected_copy);
  x ^= static_cast<uint64_t>(r.q_heads ^ r.kv_heads ^ r.n_super ^ r.superblock ^ r.top_super ^ r.n_pages ^
                             __float_as_int(r.scale));
  asm volatile("" ::"l"(x));
  const bool tree = r.supers != nullptr;
  const int n_cand = tree ? r.n_super : r.n_pages;
  const float* tab = tree ? r.supers + static_cast<int64_t>(b) * r.kv_heads * r.n_super * D
                          : r.summaries + static_cast<int64_t>(b) * r.kv_heads * r.n_pages * D;
  const int64_t stride = static_cast<int64_t>(tree ? r.n_super : r.n_pages) * D;
  const int nl = n_cand > rank ? (n_cand - 1 - rank) / ns + 1 : 0;
  // two levels: the consumer warps score level 1 (the producer joins at level 2)
  const int nws = tree ? kConsumerWarps : nw;
  if (warp < nws) {
#pragma unroll
    for (int u = 0; u < CB; ++u) {
      const int i = warp + u * nws;
      if (i < nl) load_cand_rows(pf.rows[u], tab + static_cast<int64_t>(rank + i * ns) * D, stride, 0, r.kv_heads, D);
    }
  }
  const int nvec = r.q_heads * D * static_cast<int>(sizeof(T)) / 16;
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) + static_cast<int64_t>(b) * r.q_heads * D);
  if (threadIdx.x < kRouteStagers) {
#pragma unroll
    for (int u = 0; u < kRouteQVec; ++u) {
      const int v = threadIdx.x + u * kRouteStagers;
      if (v < nvec) pf.q[u] = __ldg(src + v);
    }
  }
}

// Scratch bytes of fused_route (layout below); must fit in one ring stage.
__host__ __device__ inline size_t route_scratch_bytes(const FusedRoute& r, int head_dim, size_t elem) {
  const size_t n1 = r.supers ? r.n_super : 0, n2 = r.supers ? static_cast<size_t>(r.top_super) * r.superblock
                                                            : static_cast<size_t>(r.n_pages);
  return route_align16(static_cast<size_t>(r.q_heads) * head_dim * elem) +
         route_align16(sizeof(float) * static_cast<size_t>(r.kv_heads) * head_dim) +
         route_align16(sizeof(uint64_t) * n1) + route_align16(sizeof(uint64_t) * n2) +
         route_align16(sizeof(int64_t) * (r.top_super > 0 ? r.top_super : 1));
}

// A candidate's rank key: the score mapped to an order-preserving unsigned integer in the
// high half (-0 folded into +0, so equal scores stay equal), the id inverted in the low half
// -- key_a > key_b exactly when a beats b (higher score, or equal score and lower id), so
// ranking is one unsigned 64-bit compare per pair.  0 <= id <= 0x7FFFFFFF.
__device__ __forceinline__ uint64_t rank_key(float score, int id) {
  uint32_t u = __float_as_uint(score);
  if (u == 0x80000000u) u = 0u;
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<uint64_t>(u) << 32) | static_cast<uint32_t>(0x7FFFFFFF - id);
}
__device__ __forceinline__ int key_id(uint64_t key) { return 0x7FFFFFFF - static_cast<int>(static_cast<uint32_t>(key)); }

__device__ __forceinline__ void st_dsmem_u64(uint64_t* local_ptr, int rank, uint64_t v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local_ptr)), "r"(rank));
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(ra), "l"(v) : "memory");
}

// Asynchronous stores into a peer CTA's shared memory that complete transaction bytes on an
// mbarrier in that CTA (st.async): the receiver waits for the byte count it expects, so no
// cluster-wide barrier orders the exchange.
__device__ __forceinline__ uint32_t peer_addr(const void* local_ptr, int rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local_ptr)), "r"(rank));
  return ra;
}
__device__ __forceinline__ void st_async_b64(uint32_t raddr, uint64_t v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(raddr), "l"(v),
               "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async_v4(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   raddr),
               "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
               "r"(__float_as_uint(v.w)), "r"(rbar)
               : "memory");
}

// Top-m of the n rank keys (16-byte aligned): the thread of candidate t counts the keys
// above its own with broadcast 16-byte shared reads (two keys per read); out[rank] = id
// for rank < m.  Ranks are distinct (ids are), so out[0..min(n, m)) is filled once each.
__device__ __forceinline__ void key_select(const uint64_t* keys, int n, int m, int64_t* out) {
  const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(keys);
  const int n2 = n & ~1;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const uint64_t kt = keys[t];
    int r = 0;
#pragma unroll 8
    for (int j = 0; j < n2; j += 2) {
      const ulonglong2 v = k2[j >> 1];
      r += (v.x > kt ? 1 : 0) + (v.y > kt ? 1 : 0);
    }
    if (n & 1) r += keys[n - 1] > kt ? 1 : 0;
    if (r < m && kt != 0) out[r] = key_id(kt);  // key 0: an empty candidate slot
  }
  __syncthreads();
}

// Half-warp scoring: half h of a warp scores one candidate.  Lane hl of the half holds the
// canonical partial sums of lanes hl and hl + 16 (d = lane + 32k, k ascending, separate
// multiply and add); their sum is the canonical butterfly's first step (offset 16: fp
// addition is commutative bit for bit), and offsets 8, 4, 2, 1 stay inside the half, so
// the score equals accumulate_cand's bit for bit with half the shuffles per candidate.
template <int NS>
struct HalfRows {
  float v[kRouterKvBatch][2 * NS];
};
template <int NS>
__device__ __forceinline__ void load_half_rows(HalfRows<NS>& r, const float* base, int64_t kv_stride, int kv_heads) {
  const int hl = threadIdx.x & 15;
#pragma unroll
  for (int u = 0; u < kRouterKvBatch; ++u) {
    const bool hv = u < kv_heads;
    const float* row = base + static_cast<int64_t>(hv ? u : 0) * kv_stride;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      r.v[u][2 * k] = hv ? __ldg(row + hl + 32 * k) : 0.f;
      r.v[u][2 * k + 1] = hv ? __ldg(row + hl + 16 + 32 * k) : 0.f;
    }
  }
}
template <int NS>
__device__ __forceinline__ float accumulate_half(const HalfRows<NS>& r, const float* qg, int kv_heads) {
  constexpr int D = NS * 32;
  const int hl = threadIdx.x & 15;
  float part[kRouterKvBatch];
#pragma unroll
  for (int u = 0; u < kRouterKvBatch; ++u) {
    const float* qq = qg + (u < kv_heads ? u : 0) * D;
    float pa = 0.f, pb = 0.f;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      pa = __fadd_rn(pa, __fmul_rn(qq[hl + 32 * k], r.v[u][2 * k]));
      pb = __fadd_rn(pb, __fmul_rn(qq[hl + 16 + 32 * k], r.v[u][2 * k + 1]));
    }
    part[u] = __fadd_rn(pa, pb);
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1)
#pragma unroll
    for (int u = 0; u < kRouterKvBatch; ++u) part[u] = __fadd_rn(part[u], __shfl_xor_sync(0xffffffffu, part[u], off));
  float total = 0.f;
#pragma unroll
  for (int u = 0; u < kRouterKvBatch; ++u)
    if (u < kv_heads) total = __fadd_rn(total, part[u]);
  return total;
}

// Called by every thread of the CTA.  Ends with the top_m logical pages of sequence b in
// sel_s (descending score, -1 for slots without a candidate), visible to the whole CTA.
template <typename T, int NS>
__device__ __forceinline__ void fused_route(const DecodeArgs& a, int b, int rank, int ns, unsigned char* scratch,
                                         int64_t* sel_s, bool write_out, RoutePrefetch<NS>& pf, uint64_t* xbar) {
  constexpr int CB = RouteCfg<NS>::kCB;
  const FusedRoute& r = a.route;
  constexpr int D = NS * 32;  // the kernel's head_dim
  const int hkv = r.kv_heads, top_m = a.top_m;
  const bool tree = r.supers != nullptr;
  const int n1 = tree ? r.n_super : 0, n2 = tree ? r.top_super * r.superblock : r.n_pages;
  // scratch: query row, per-kv-head query sums, rank keys of both levels, chosen
  // superblocks, candidate offsets (route_scratch_bytes)
  unsigned char* sp = scratch;
  T* qraw = reinterpret_cast<T*>(sp);
  sp += route_align16(static_cast<size_t>(r.q_heads) * D * sizeof(T));
  float* qg = reinterpret_cast<float*>(sp);
  sp += route_align16(sizeof(float) * static_cast<size_t>(hkv) * D);
  uint64_t* k1 = reinterpret_cast<uint64_t*>(sp);
  sp += route_align16(sizeof(uint64_t) * n1);
  uint64_t* k2 = reinterpret_cast<uint64_t*>(sp);
  sp += route_align16(sizeof(uint64_t) * n2);
  int64_t* chosen = reinterpret_cast<int64_t*>(sp);
  // score = total / q_heads * scale; for a power-of-two head count the division is a
  // multiplication by the exact reciprocal (the same correctly rounded quotient)
  const bool hq_pow2 = (r.q_heads & (r.q_heads - 1)) == 0;
  const float inv_hq = 1.0f / static_cast<float>(r.q_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float* sup_tab = tree ? r.supers + static_cast<int64_t>(b) * hkv * r.n_super * D : nullptr;
  const float* page_tab = r.summaries + static_cast<int64_t>(b) * hkv * r.n_pages * D;
  const int64_t sup_stride = static_cast<int64_t>(r.n_super) * D, page_stride = static_cast<int64_t>(r.n_pages) * D;
  for (int j = threadIdx.x; j < top_m; j += blockDim.x) sel_s[j] = -1;

  // the first batch of this warp's first-level candidate rows and the query row were
  // requested at kernel entry (route_prefetch): stage the query, sum it per kv head
  int n_cand = tree ? n1 : n2;
  int nl;
  CandRows<NS>* rows = pf.rows;
  if (threadIdx.x < kRouteStagers) {  // the consumer warps; the producer joins after them
    const int nvec = r.q_heads * D * static_cast<int>(sizeof(T)) / 16;
#pragma unroll
    for (int u = 0; u < kRouteQVec; ++u) {
      const int v = threadIdx.x + u * kRouteStagers;
      if (v < nvec) reinterpret_cast<uint4*>(qraw)[v] = pf.q[u];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kRouteStagers) : "memory");
    // qg[kvh][8c .. 8c+8): the kv head's query heads added in order, one 16-byte piece
    // of each head row per load (all of a thread's loads issue before the adds)
    const int group = r.q_heads / hkv;
    constexpr int kPieces = D / 8;  // 16-byte pieces of a 16-bit head row
    const uint4* qv = reinterpret_cast<const uint4*>(qraw);
    for (int w = threadIdx.x; w < hkv * kPieces; w += kRouteStagers) {
      const int kvh = w / kPieces, c = w - kvh * kPieces;
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 4
      for (int j = 0; j < group; ++j) {
        const uint4 v = qv[(kvh * group + j) * kPieces + c];
        const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], to_f32(h[e]));
      }
      float4* dst4 = reinterpret_cast<float4*>(qg + kvh * D + 8 * c);
      dst4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  // the per-kv-head sums are complete for the threads that score next: two levels, the
  // consumer warps (the producer, still issuing the local window, scores only at level 2,
  // after the level-1 selection's block barrier); one level, everyone
  if (tree) {
    if (threadIdx.x < kRouteStagers) asm volatile("bar.sync 1, %0;" ::"n"(kRouteStagers) : "memory");
  } else {
    __syncthreads();
  }
  cluster_wait();  // every CTA of the cluster runs (its exchange barriers initialised)
  // this CTA receives every candidate's key of a level: 8 bytes per candidate slot (two
  // levels: n_super superblocks, then top_super * superblock page slots)
  if (threadIdx.x == 0) {
    if (tree) mbar_arrive_expect_tx(&xbar[0], static_cast<uint32_t>(n1) * 8u);
    mbar_arrive_expect_tx(&xbar[1], static_cast<uint32_t>(n2) * 8u);
  }
  // level-2 slot c of two levels: page c % superblock of the (c / superblock)-th chosen
  // superblock; slots past the last page (a partial last superblock) carry key 0
  const bool sb_pow2 = (r.superblock & (r.superblock - 1)) == 0;
  const int sb_lg = __ffs(r.superblock) - 1;
  auto page_of = [&](int c) {
    const int j = sb_pow2 ? c >> sb_lg : c / r.superblock;
    return static_cast<int>(chosen[j]) * r.superblock + (c - j * r.superblock);
  };
  const int first_level = tree ? 1 : 2;
#pragma unroll 1
  for (int level = first_level; level <= 2; ++level) {
    const float* tab = level == 1 ? sup_tab : page_tab;
    const int64_t kv_stride = level == 1 ? sup_stride : page_stride;
    uint64_t* dst = level == 1 ? k1 : k2;
    nl = n_cand > rank ? (n_cand - 1 - rank) / ns + 1 : 0;
    const int nws = level == 1 ? kConsumerWarps : nw;  // scoring warps of this level
    if (level == 2 && tree) {
      // two levels, level 2: half-warps, one candidate pair per warp in flight
      constexpr int HB = 1;
      const int half = lane >> 4, hl = lane & 15;
      const int npairs = (nl + 1) >> 1;
#pragma unroll 1
      for (int p0 = warp; p0 < npairs; p0 += nws * HB) {
        HalfRows<NS> hr[HB];
#pragma unroll
        for (int hb = 0; hb < HB; ++hb) {
          const int pr = p0 + hb * nws, i = 2 * pr + half;
          if (pr < npairs) {
            // a half without a candidate (odd count) reads a valid row and discards it
            int g = i < nl ? page_of(rank + i * ns) : 0;
            if (g >= r.n_pages) g = r.n_pages - 1;  // empty slot: any valid row, key 0 below
            load_half_rows(hr[hb], page_tab + static_cast<int64_t>(g) * D, page_stride, hkv);
          }
        }
#pragma unroll
        for (int hb = 0; hb < HB; ++hb) {
          const int pr = p0 + hb * nws, i = 2 * pr + half;
          if (pr < npairs) {
            const float total = accumulate_half(hr[hb], qg, hkv);
            if (i < nl && hl < ns) {
              const int c = rank + i * ns;
              const int g = page_of(c);
              const float q = hq_pow2 ? __fmul_rn(total, inv_hq) : __fdiv_rn(total, static_cast<float>(r.q_heads));
              const uint64_t key = g < r.n_pages ? rank_key(__fmul_rn(q, r.scale), g) : 0ull;
              st_async_b64(peer_addr(k2 + c, hl), key, peer_addr(&xbar[1], hl));
            }
          }
        }
      }
    } else {
#pragma unroll 1
    for (int i0 = warp; warp < nws && i0 < nl; i0 += nws * CB) {
      if (level != first_level || i0 != warp) {
#pragma unroll
        for (int u = 0; u < CB; ++u) {
          const int i = i0 + u * nws;
          if (i < nl) {
            const int c = rank + i * ns;
            int g = (level == 2 && tree) ? page_of(c) : c;
            if (g >= r.n_pages) g = r.n_pages - 1;  // empty slot: any valid row, key 0 below
            load_cand_rows(rows[u], tab + static_cast<int64_t>(g) * D, kv_stride, 0, hkv, D);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < CB; ++u) {
        const int i = i0 + u * nws;
        if (i < nl) {
          const int c = rank + i * ns;
          const int g = (level == 2 && tree) ? page_of(c) : c;
          const float total = accumulate_cand(rows[u], qg, 0, hkv, D, 0.f);
          const float q = hq_pow2 ? __fmul_rn(total, inv_hq) : __fdiv_rn(total, static_cast<float>(r.q_heads));
          const uint64_t key = g < r.n_pages || level == 1 ? rank_key(__fmul_rn(q, r.scale), g) : 0ull;
          if (lane < ns) st_async_b64(peer_addr(dst + c, lane), key, peer_addr(&xbar[level - 1], lane));
        }
      }
    }
    }
    // every candidate's key of this level is in this CTA (a lost store ends the wait with
    // the error word set)
    mbar_wait_bounded(&xbar[level - 1], 0);
    if (level == 1) {
      key_select(k1, n_cand, r.top_super, chosen);
      n_cand = n2;
    } else {
      key_select(k2, n_cand, top_m, sel_s);
    }
  }
  if (write_out) {
    for (int j = threadIdx.x; j < top_m; j += blockDim.x) {
      const int64_t v = sel_s[j];
      r.selected[static_cast<int64_t>(b) * top_m + j] = v;
      if (r.selected_copy) r.selected_copy[static_cast<int64_t>(b) * top_m + j] = v;
    }
  }
  // the scratch (written by this CTA and pushed into by its peers) becomes a TMA
  // destination next: order the generic-proxy accesses before the async-proxy writes
  fence_proxy_async_smem();
  __syncthreads();
}

template <typename T, int D, int STAGES, bool ROUTE = false>
__global__ void __launch_bounds__(kDecodeThreads, ROUTE ? 2 : 0) decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                     const __grid_constant__ CUtensorMap vmap,
                                                                     const DecodeArgs a) {
  using S = DecodeSmem<D, STAGES>;
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte aligned base (128-byte swizzle atoms), taken by indexing the shared array so
  // the compiler keeps every access through it in the shared address space
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kRingBytes);
  uint64_t* empty = full + STAGES;
  // exchange barriers of the routing instantiation: level-1 keys, level-2 keys, merge
  // partials (each counts the bytes its CTA's peers store into it)
  uint64_t* xbar = empty + STAGES;
  int4* info = reinterpret_cast<int4*>(xbar + 4);
  int32_t* tab = reinterpret_cast<int32_t*>(info + STAGES);
  int64_t* sel_s = reinterpret_cast<int64_t*>(tab + S::kTabCap);
  // partials pushed by the cluster's splits for the columns this CTA merges
  float* recv = reinterpret_cast<float*>(sel_s + S::kSelCap);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool cluster_push = a.cluster_merge && a.nsplit > 1;
  pdl_trigger();
  touch_args(a);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    if (ROUTE)
      for (int k = 0; k < 3; ++k) mbar_init(&xbar[k], 1);
    fence_mbar_init();
  }
  // routing CTAs (and merging splits) store into their peers' shared memory: every CTA
  // arrives now, after its barriers are initialised, and waits before its first remote store
  if (ROUTE || cluster_push) cluster_arrive_relaxed();
  if (!a.early_local) pdl_block();
  // routing: the router's first loads go out now, with the prologue's
  RoutePrefetch<(ROUTE ? D / 32 : 1)> pf;
  if constexpr (ROUTE) route_prefetch<T, D / 32>(a, b, split, a.nsplit, pf);
  // prologue loads issued together (one memory round trip): the producer's page-table row
  // and selected ids, every thread's context length.  With early_local the selected ids
  // come from the kernel this one overlaps, so they are read after it completes; routing
  // CTAs select the pages themselves.
  const int tstride = a.addr.table_stride;
  const bool use_tab = a.addr.page_table != nullptr && tstride <= S::kTabCap;
  const bool sel_early = !ROUTE && a.selected && !a.early_local && a.top_m <= S::kSelCap;
  int32_t tab_r[16];
  int64_t sel_r = -1;
  if (warp == kConsumerWarps) {
    if (use_tab) {
      const int32_t* src = a.addr.page_table + static_cast<int64_t>(b) * tstride;
#pragma unroll
      for (int u = 0; u < 16; ++u) tab_r[u] = lane + 32 * u < tstride ? __ldg(src + lane + 32 * u) : -1;
    }
    if (sel_early && lane < a.top_m) sel_r = a.selected[static_cast<int64_t>(b) * a.top_m + lane];
  }
  // this split's chunks: the local-window chunks and the selected chunks are divided among
  // the splits separately: each split gets an equal share of the selected chunks, the ones
  // that wait for the router in the fused step, on top of at most its share of the local ones
  struct SplitWork {
    ChunkPlan plan;
    int c_l0, c_s0, n_local, nk;
  };
  auto split_work = [&](int ctx) -> SplitWork {
    SplitWork w;
    w.plan = make_plan_ctx(a, ctx, kChunk);
    const int n_sel_chunks = w.plan.n_total - w.plan.n_seg;
    // bounds of an even division of n items into nsplit parts (32-bit arithmetic while the
    // products fit, which is every realistic context)
    auto part_of = [&](int n, int s_) -> int {
      return n <= (1 << 22) ? n * s_ / a.nsplit : static_cast<int>(static_cast<int64_t>(n) * s_ / a.nsplit);
    };
    w.c_l0 = part_of(w.plan.n_seg, split);
    const int c_l1 = part_of(w.plan.n_seg, split + 1);
    w.c_s0 = w.plan.n_seg + part_of(n_sel_chunks, split);
    const int c_s1 = w.plan.n_seg + part_of(n_sel_chunks, split + 1);
    w.n_local = c_l1 - w.c_l0;
    w.nk = w.n_local + (c_s1 - w.c_s0);
    return w;
  };
  // routing: the context length is requested now and used by the producer before routing
  // and by the consumers only after it, so its round trip is not on their path
  const int ctx_b = a.ctx_lens[b];
  SplitWork sw{};
  if constexpr (ROUTE) {
    __syncthreads();  // the barrier initialisation is visible to every thread
    if (warp == kConsumerWarps) sw = split_work(ctx_b);
  } else {
    sw = split_work(ctx_b);
    __syncthreads();
  }

  // ------------------------------------------------------------ producer
  bool ok = true;
  auto row_of = [&](int t) -> long long {
    if (!use_tab) return a.addr.row(b, kvh, t);
    const int ps = a.addr.page_size;
    const int lp = (ps & (ps - 1)) == 0 ? t >> (__ffs(ps) - 1) : t / ps;
    if (lp < 0 || lp >= tstride) return -1;
    const int32_t pg = tab[lp];
    if (pg < 0) return -1;
    return b * a.addr.batch_stride_rows + static_cast<long long>(pg) * a.addr.page_stride_rows +
           kvh * a.addr.head_stride_rows + (t - lp * a.addr.page_size);
  };
  // issues this split's chunks [lo, hi) into the ring (producer warp; lane 0 issues)
  auto produce = [&](int lo, int hi, const int64_t* sel_row) {
    const uint64_t policy = l2_policy_evict_first();
    for (int base = lo; base < hi && ok; base += 32) {
      ChunkInfo ci{0, 0, 0};
      long long row = -1;
      if (base + lane < hi) {
        const int idx = base + lane;  // this split's idx-th chunk
        ci = chunk_info(a, sw.plan, sel_row, idx < sw.n_local ? sw.c_l0 + idx : sw.c_s0 + (idx - sw.n_local),
                        kChunk);
        if (ci.vlo < ci.vhi) {
          row = row_of(ci.t0);
          if (row < 0 || row >= a.addr.total_rows) {
            spa_raise(SPA_DEVERR_BAD_PAGE);
            row = -1;
          }
        }
      }
      const int cnt = min(32, hi - base);
      for (int j = 0; j < cnt; ++j) {
        const int i = base + j;
        const int t0 = __shfl_sync(0xffffffffu, ci.t0, j);
        const int vlo = __shfl_sync(0xffffffffu, ci.vlo, j);
        const int vhi = __shfl_sync(0xffffffffu, ci.vhi, j);
        const long long r = __shfl_sync(0xffffffffu, row, j);
        if (lane == 0) {
          const int stage = i % STAGES;
          if (i >= STAGES && !mbar_wait_bounded(&empty[stage], ((i / STAGES) - 1) & 1)) ok = false;
          if (ok) {
            info[stage] = make_int4(t0, r >= 0 ? vlo : 0, r >= 0 ? vhi : 0, 0);
            uint64_t* bar = &full[stage];
            if (r >= 0) {
              mbar_arrive_expect_tx(bar, S::kStageBytes);
              unsigned char* dst = smem + stage * S::kStageBytes;
              tma_load_3d_hint(dst, &kmap, bar, 0, static_cast<int>(r), 0, policy);
              tma_load_3d_hint(dst + S::kKvBytes, &vmap, bar, 0, static_cast<int>(r), 0, policy);
            } else {
              mbar_arrive(bar);
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
    }
  };
  // routing: the local-window chunks that fit in the ring before its last stage (the
  // router's scratch) load while the cluster selects; the rest follow the selection
  const int n_early = ROUTE ? min(sw.n_local, STAGES - 1) : sw.n_local;
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    // the sequence's page-table row: the first 512 entries were loaded with the plan,
    // the rest (long rows) here with independent loads
    if (use_tab) {
      const int32_t* src = a.addr.page_table + static_cast<int64_t>(b) * tstride;
#pragma unroll
      for (int u = 0; u < 16; ++u)
        if (lane + 32 * u < tstride) tab[lane + 32 * u] = tab_r[u];
      for (int e0 = lane + 32 * 16; e0 < tstride; e0 += 32 * 16) {
        int32_t r[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) r[u] = e0 + 32 * u < tstride ? __ldg(src + e0 + 32 * u) : -1;
#pragma unroll
        for (int u = 0; u < 16; ++u)
          if (e0 + 32 * u < tstride) tab[e0 + 32 * u] = r[u];
      }
    }
    if (sel_early && lane < a.top_m) sel_s[lane] = sel_r;
    __syncwarp();
    if constexpr (ROUTE) {
      produce(0, n_early, nullptr);
    } else {
      const int64_t* sel_row =
          sel_early ? sel_s : (a.selected ? a.selected + static_cast<int64_t>(b) * a.top_m : nullptr);
      // chunks [0, n_local) of this split are local-window chunks (no router output needed);
      // with early_local they are issued before waiting for the router.
      for (int part = 0; part < 2 && ok; ++part) {
        const int lo = part ? sw.n_local : 0, hi = part ? sw.nk : sw.n_local;
        if (part == 1 && a.early_local) {
          pdl_block();
          // the router has completed: its selected ids for this sequence, one round trip
          if (a.selected && a.top_m <= S::kSelCap) {
            if (lane < a.top_m) sel_s[lane] = a.selected[static_cast<int64_t>(b) * a.top_m + lane];
            __syncwarp();
            sel_row = sel_s;
          }
        }
        produce(lo, hi, sel_row);
      }
      // every thread of every CTA in a merging cluster completes both cluster phases
      if (cluster_push) {
        cluster_wait();
        cluster_barrier();
      }
      return;
    }
  }
  if constexpr (ROUTE) {
    // every thread routes (the producer warp too, after its early chunks)
    fused_route<T, D / 32>(a, b, split, a.nsplit, smem + (STAGES - 1) * S::kStageBytes, sel_s,
                           split == 0 && kvh == 0, pf, xbar);
    if (warp == kConsumerWarps) {
      produce(n_early, sw.nk, sel_s);
      return;
    }
    sw = split_work(ctx_b);  // the consumers' chunk count
  }

  // -------------------------------------------------------------- consumers
  using Mma = MmaOp<T>;
  const int group = a.group;
  const int g0 = lane >> 2, tig = lane & 3;
  uint32_t qa[D / 16][4];
  {
    if (a.q_after_wait) pdl_block();
    const T* qb =
        static_cast<const T*>(a.q) + (static_cast<int64_t>(b) * a.q_batch_heads + a.q_head_offset + kvh * group) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int col = ks * 16 + tig * 2;
      qa[ks][0] = g0 < group ? *reinterpret_cast<const uint32_t*>(qb + g0 * D + col) : 0u;
      qa[ks][1] = g0 + 8 < group ? *reinterpret_cast<const uint32_t*>(qb + (g0 + 8) * D + col) : 0u;
      qa[ks][2] = g0 < group ? *reinterpret_cast<const uint32_t*>(qb + g0 * D + col + 8) : 0u;
      qa[ks][3] = g0 + 8 < group ? *reinterpret_cast<const uint32_t*>(qb + (g0 + 8) * D + col + 8) : 0u;
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  const int rbase = warp * 16;
  const int mi = lane >> 3, mr = lane & 7;
  ok = true;
  const int nk = sw.nk;
  for (int i = 0; i < nk; ++i) {
    const int stage = i % STAGES;
    // warp-uniform outcome: lanes must agree before any aligned barrier below
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[stage], (i / STAGES) & 1))) {
      ok = false;
      break;
    }
    const int4 ci = info[stage];
    const int tw0 = ci.x + rbase;
    const bool any = ci.y < ci.z && tw0 < ci.z && tw0 + 16 > ci.y;
    if (any) {
      const uint32_t sk = smem_u32(smem + stage * S::kStageBytes);
      const uint32_t sv = sk + S::kKvBytes;
      const bool partial = tw0 < ci.y || tw0 + 16 > ci.z;
      if (partial) {
        // zero the V rows of non-candidate tokens so 0 * (stale bits) cannot make NaN
        unsigned char* vrow = smem + stage * S::kStageBytes + S::kKvBytes;
        for (int e = lane; e < 16 * S::kBoxes * 8; e += 32) {
          const int r = e / (S::kBoxes * 8), rem = e - r * (S::kBoxes * 8);
          const int bx = rem >> 3, c = rem & 7;
          const int tok = tw0 + r;
          if (tok < ci.y || tok >= ci.z)
            *reinterpret_cast<int4*>(vrow + bx * S::kBoxBytes + (rbase + r) * 128 + c * 16) = make_int4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      float s[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t kb[4];
        ldmatrix_x4(kb, swz_addr<D>(sk, rbase + (mi >> 1) * 8 + mr, 2 * ks + (mi & 1)));
        Mma::run(s[0], qa[ks], kb[0], kb[1]);
        Mma::run(s[1], qa[ks], kb[2], kb[3]);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = tw0 + j * 8 + tig * 2 + (e & 1);
          s[j][e] = (tok >= ci.y && tok < ci.z) ? s[j][e] * a.scale_log2 : -INFINITY;
        }
      float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = fast_exp2(m0 - mu0), al1 = fast_exp2(m1 - mu1);
      float p[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        p[j][0] = fast_exp2(s[j][0] - mu0);
        p[j][1] = fast_exp2(s[j][1] - mu0);
        p[j][2] = fast_exp2(s[j][2] - mu1);
        p[j][3] = fast_exp2(s[j][3] - mu1);
      }
      l0 = l0 * al0 + (p[0][0] + p[0][1] + p[1][0] + p[1][1]);
      l1 = l1 * al1 + (p[0][2] + p[0][3] + p[1][2] + p[1][3]);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        acc[n][0] *= al0;
        acc[n][1] *= al0;
        acc[n][2] *= al1;
        acc[n][3] *= al1;
      }
      uint32_t pa[4];
      pa[0] = Mma::pack(p[0][0], p[0][1]);
      pa[1] = Mma::pack(p[0][2], p[0][3]);
      pa[2] = Mma::pack(p[1][0], p[1][1]);
      pa[3] = Mma::pack(p[1][2], p[1][3]);
#pragma unroll
      for (int nd = 0; nd < D / 16; ++nd) {
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, swz_addr<D>(sv, rbase + (mi & 1) * 8 + mr, 2 * nd + (mi >> 1)));
        Mma::run(acc[2 * nd], pa, vb[0], vb[1]);
        Mma::run(acc[2 * nd + 1], pa, vb[2], vb[3]);
      }
      if (partial) fence_proxy_async_smem();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
  if (!ok) {  // error word already raised; outputs of this split are undefined
    if (cluster_push && !ROUTE) {
      cluster_wait();
      cluster_barrier();
    }
    return;
  }

  // ------------------------------------------------ merge the four warps (shared memory)
  // Each consumer warp holds (m, l, O) of its 16 token rows for every query head.  The
  // real rows go to padded shared-memory rows (conflict-free float2 stores) and the
  // CTA combines them into one normalised partial (O, log2-sum-exp) per head.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  constexpr int LD = D + 8;
  float* red = reinterpret_cast<float*>(smem);                 // [warp][group][LD]
  float* ml = red + kConsumerWarps * group * LD;               // [warp][group][2]
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");  // ring reads done
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = g0 + 8 * half;
    if (row >= group) continue;
    float* dst = red + (warp * group + row) * LD + tig * 2;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<float2*>(dst + n * 8) = make_float2(acc[n][2 * half], acc[n][2 * half + 1]);
    if (tig == 0) {
      ml[(warp * group + row) * 2] = half ? m1 : m0;
      ml[(warp * group + row) * 2 + 1] = half ? l1 : l0;
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
  // per head, once: the warps' weights exp2(m_w - M) / L and the log2-sum-exp
  float* fw = ml + kConsumerWarps * group * 2;   // [group][kConsumerWarps]
  float* row_lse = fw + group * kConsumerWarps;  // [group]
  if (threadIdx.x < group) {
    const int row = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, ml[(w * group + row) * 2]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float e[kConsumerWarps], L = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      e[w] = fast_exp2(ml[(w * group + row) * 2] - Mu);
      L += ml[(w * group + row) * 2 + 1] * e[w];
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) fw[row * kConsumerWarps + w] = e[w] * inv;
    row_lse[row] = L > 0.f ? M + __log2f(L) : -INFINITY;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
  const int64_t bh0 = static_cast<int64_t>(b) * a.Hq + kvh * group;
  const int ns = a.nsplit;
  // cluster merge: rank r merges output columns [r*D/ns, (r+1)*D/ns) of every head; every
  // split pushes its normalised partial of those columns, and its log-sum-exps, into rank
  // r's receive buffer (recv_lse [split][group], recv_o [split][group][wmax])
  // a power-of-two split count (8 in the fused step) turns the divisions by ns into shifts
  const bool ns_pow2 = (ns & (ns - 1)) == 0;
  const int ns_lg = __ffs(ns) - 1;
  auto div_ns = [&](int x) { return ns_pow2 ? x >> ns_lg : x / ns; };
  const int wmax = div_ns(D + ns - 1);
  float* recv_lse = recv;
  float* recv_o = recv + ((ns * group + 3) & ~3);  // 16-byte aligned
  // equal column slices of a multiple of 4: 16-byte loads and remote stores
  const bool vec4 = cluster_push && (ns_pow2 ? (D & (4 * ns - 1)) == 0 : D % (4 * ns) == 0);
  // every CTA of the cluster runs: remote stores are safe (routing CTAs waited before routing)
  if (cluster_push && !ROUTE) cluster_wait();
  if (ROUTE && cluster_push && threadIdx.x == 0) {
    // this CTA receives, from each of the ns splits, one log-sum-exp and its column slice
    // per head
    const int w_self = div_ns((split + 1) * D) - div_ns(split * D);
    mbar_arrive_expect_tx(&xbar[2], static_cast<uint32_t>(ns * group * (1 + w_self)) * 4u);
  }
  if (vec4) {
    for (int idx = threadIdx.x; idx < group * (D / 4); idx += kConsumerWarps * 32) {
      const int row = idx / (D / 4), col = (idx - row * (D / 4)) * 4;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float4 r4 = *reinterpret_cast<const float4*>(red + (w * group + row) * LD + col);
        const float f = fw[row * kConsumerWarps + w];
        o.x = fmaf(r4.x, f, o.x);
        o.y = fmaf(r4.y, f, o.y);
        o.z = fmaf(r4.z, f, o.z);
        o.w = fmaf(r4.w, f, o.w);
      }
      const int r = col * ns / D;  // slices are exactly wmax = D / ns wide
      float* dst = recv_o + (split * group + row) * wmax + (col - r * wmax);
      if constexpr (ROUTE)
        st_async_v4(peer_addr(dst, r), o, peer_addr(&xbar[2], r));
      else
        st_dsmem_v4(dst, r, o);
    }
  }
  for (int idx = threadIdx.x; !vec4 && idx < group * D; idx += kConsumerWarps * 32) {
    const int row = idx / D, col = idx - row * D;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w)
      o = fmaf(red[(w * group + row) * LD + col], fw[row * kConsumerWarps + w], o);
    if (ns == 1) {
      static_cast<T*>(a.out)[(bh0 + row) * D + col] = from_f32<T>(o);
    } else if (cluster_push) {
      const int r = ((col + 1) * ns - 1) / D;  // the rank whose column slice holds col
      float* dst = recv_o + (split * group + row) * wmax + (col - r * D / ns);
      if constexpr (ROUTE)
        st_async_f32(peer_addr(dst, r), o, peer_addr(&xbar[2], r));
      else
        st_dsmem(dst, r, o);
    } else {
      a.part_o[((bh0 + row) * ns + split) * D + col] = o;
      if (col == 0) a.part_lse[(bh0 + row) * ns + split] = row_lse[row];
    }
  }
  if (!cluster_push) return;
  for (int i = threadIdx.x; i < group * ns; i += kConsumerWarps * 32) {
    const int row = div_ns(i), r = i - row * ns;
    if constexpr (ROUTE)
      st_async_f32(peer_addr(recv_lse + split * group + row, r), row_lse[row], peer_addr(&xbar[2], r));
    else
      st_dsmem(recv_lse + split * group + row, r, row_lse[row]);
  }
  // every split's pushes are visible in the receive buffers (routing instantiation: this
  // CTA's byte count; a lost store ends the wait with the error word set)
  if constexpr (ROUTE)
    mbar_wait_bounded(&xbar[2], 0);
  else
    cluster_barrier();
  // after the barrier this CTA reads only its own shared memory: no second barrier
  const int c0 = div_ns(split * D), c1 = div_ns((split + 1) * D), w = c1 - c0;
  for (int idx = threadIdx.x; idx < group * w; idx += kConsumerWarps * 32) {
    const int row = ns_pow2 ? idx * ns / D : idx / w, j = idx - row * w;
    float M = -INFINITY;
    for (int s2 = 0; s2 < ns; ++s2) M = fmaxf(M, recv_lse[s2 * group + row]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float W = 0.f, O = 0.f;
    for (int s2 = 0; s2 < ns; ++s2) {
      const float f = fast_exp2(recv_lse[s2 * group + row] - Mu);
      W += f;
      O = fmaf(recv_o[(s2 * group + row) * wmax + j], f, O);
    }
    static_cast<T*>(a.out)[(bh0 + row) * D + c0 + j] = from_f32<T>(W > 0.f ? O / W : 0.f);
  }
}

// ---------------------------------------------------------------------------
// Generic path: one warp per (b, q head, split); any dtype, head_dim <= 256,
// any page size.  fp32 math with accurate expf.
constexpr int kGenericChunk = 16;

template <typename T>
__global__ void __launch_bounds__(32) decode_generic_kernel(const T* __restrict__ k, const T* __restrict__ v,
                                                            const DecodeArgs a) {
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z, lane = threadIdx.x;
  pdl_trigger();
  pdl_block();
  const int kvh = h / a.group, D = a.D;
  const ChunkPlan plan = make_plan(a, b, kGenericChunk);
  const int k0 = static_cast<int>(static_cast<int64_t>(plan.n_total) * split / a.nsplit);
  const int k1 = static_cast<int>(static_cast<int64_t>(plan.n_total) * (split + 1) / a.nsplit);
  float qv[8], acc[8];
  const T* qp = static_cast<const T*>(a.q) + (static_cast<int64_t>(b) * a.q_batch_heads + a.q_head_offset + h) * D;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int d = lane + 32 * e;
    qv[e] = d < D ? to_f32(qp[d]) : 0.f;
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int kk = k0; kk < k1; ++kk) {
    const ChunkInfo ci =
        chunk_info(a, plan, a.selected ? a.selected + static_cast<int64_t>(b) * a.top_m : nullptr, kk, kGenericChunk);
    for (int t = ci.vlo; t < ci.vhi; ++t) {
      const int64_t row = a.addr.row(b, kvh, t);
      if (row < 0 || row >= a.addr.total_rows) {
        if (lane == 0) spa_raise(SPA_DEVERR_BAD_PAGE);
        continue;
      }
      const T* kr = k + row * D;
      const T* vr = v + row * D;
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = lane + 32 * e;
        if (d < D) dot = fmaf(qv[e], to_f32(kr[d]), dot);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const float sc = dot * a.scale;
      const float mn = fmaxf(m, sc);
      const float alpha = expf(m - mn);  // m = -inf -> 0
      const float p = expf(sc - mn);
      l = l * alpha + p;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = lane + 32 * e;
        acc[e] = acc[e] * alpha + (d < D ? p * to_f32(vr[d]) : 0.f);
      }
      m = mn;
    }
  }
  const int64_t bh = static_cast<int64_t>(b) * a.Hq + h;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int d = lane + 32 * e;
    if (d >= D) continue;
    const float o = l > 0.f ? acc[e] / l : 0.f;
    if (a.nsplit == 1)
      static_cast<T*>(a.out)[bh * D + d] = from_f32<T>(o);
    else
      a.part_o[(bh * a.nsplit + split) * D + d] = o;
  }
  if (a.nsplit > 1 && lane == 0)
    a.part_lse[bh * a.nsplit + split] = l > 0.f ? m * 1.4426950408889634f + log2f(l) : -INFINITY;
}

// ---------------------------------------------------------------------------
// Split merge: grid (B*Hq), block kMergeThreads.  Thread t owns column t % D of slot
// group t / D; the slot groups' weighted sums are added in shared memory.
constexpr int kMergeThreads = 512;
constexpr int kMergeMaxSlots = 1024;

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) decode_combine_kernel(const float* __restrict__ part_o,
                                                                       const float* __restrict__ part_lse,
                                                                       int nslots, int D, T* __restrict__ out) {
  constexpr int kRegSlots = 16;  // partials a thread holds in registers per batch
  pdl_block();
  __shared__ float w[kMergeMaxSlots];
  __shared__ float red[kMergeThreads];
  __shared__ float s_max, s_inv;
  const int64_t bh = blockIdx.x;
  const int groups = max(1, static_cast<int>(blockDim.x) / D);
  const int d = threadIdx.x % D, g = threadIdx.x / D;
  const float* base = part_o + bh * nslots * static_cast<int64_t>(D) + d;
  // issue this thread's first batch of partial loads before the weights are known
  float v[kRegSlots];
#pragma unroll
  for (int u = 0; u < kRegSlots; ++u) {
    const int s = g + u * groups;
    v[u] = (g < groups && s < nslots) ? __ldcg(base + static_cast<int64_t>(s) * D) : 0.f;
  }
  const float* lse = part_lse + bh * nslots;
  for (int s = threadIdx.x; s < nslots; s += blockDim.x) w[s] = __ldcg(lse + s);
  __syncthreads();
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (int s = threadIdx.x; s < nslots; s += 32) M = fmaxf(M, w[s]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float Mu = M == -INFINITY ? 0.f : M;
    float W = 0.f;
    for (int s = threadIdx.x; s < nslots; s += 32) W += exp2f(w[s] - Mu);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) W += __shfl_xor_sync(0xffffffffu, W, off);
    if (threadIdx.x == 0) {
      s_max = Mu;
      s_inv = W > 0.f ? 1.f / W : 0.f;
    }
  }
  __syncthreads();
  const float mx = s_max;
  float o = 0.f;
  if (g < groups) {
#pragma unroll
    for (int u = 0; u < kRegSlots; ++u) {
      const int s = g + u * groups;
      if (s < nslots) o += v[u] * exp2f(w[s] - mx);
    }
    for (int s = g + kRegSlots * groups; s < nslots; s += groups)
      o += __ldcg(base + static_cast<int64_t>(s) * D) * exp2f(w[s] - mx);
  }
  red[threadIdx.x] = o;
  __syncthreads();
  if (threadIdx.x < D) {
    float t = 0.f;
    for (int gg = 0; gg < groups; ++gg) t += red[gg * D + threadIdx.x];
    out[bh * D + threadIdx.x] = from_f32<T>(t * s_inv);
  }
}

// ---------------------------------------------------------------------------
// host planning
inline int device_sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Split plan per (b, kv head).  Target ~2 CTAs per SM with >= 2 chunks per split.  Up to
// kMaxClusterSplits splits form a thread-block cluster that merges through distributed
// shared memory; pairs too few to fill the GPU that way use more splits with global
// partials and a merge kernel.
constexpr int kMaxClusterSplits = 8;
struct SplitPlan {
  int nsplit;
  bool cluster;
};
inline SplitPlan decode_plan(int batch, int q_heads, int kv_heads, int max_candidates) {
  const int pairs = batch * kv_heads;
  const int group = q_heads / kv_heads;
  const int slots = device_sm_count() * 2;
  const int chunks = max_candidates / kChunk + 2;
  int ns = pairs >= slots ? 1 : slots / pairs;
  const int cap = chunks / 2 > 1 ? chunks / 2 : 1;
  if (ns > cap) ns = cap;
  if (ns > 256) ns = 256;
  if (ns < 1) ns = 1;
  if (ns <= kMaxClusterSplits) return {ns, ns > 1};
  // 8-CTA clusters still give every SM at least one CTA: prefer them
  if (static_cast<int64_t>(pairs) * kMaxClusterSplits >= device_sm_count()) return {kMaxClusterSplits, true};
  // few chunks per pair (at most 3 per split of 8): the wider split would not shorten the
  // per-split chain, and 8 splits merged in a cluster save the separate merge launch
  if (chunks <= 3 * kMaxClusterSplits) return {kMaxClusterSplits, true};
  (void)group;
  return {ns, false};
}
inline int decode_nsplit(int batch, int q_heads, int kv_heads, int max_candidates) {
  return decode_plan(batch, q_heads, kv_heads, max_candidates).nsplit;
}

constexpr int kDecodeStages = 3;

// Launch with programmatic stream serialization (when pdl: the kernel may start before its
// predecessor in the stream completes and orders its reads with griddepcontrol.wait) and,
// when cluster_x > 1, thread-block clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                       Args&&... args) {
  return launch_ex(kern, grid, block, smem, st, pdl, 1, std::forward<Args>(args)...);
}

// ROUTE: the instantiation that selects the pages itself (fused_route); it needs the
// splits of a pair in one cluster and the router's scratch within one ring stage.
// pdl: launch as a programmatic dependent of the previous kernel in the stream (the
// kernel waits for it before its first read unless early_local says otherwise).
template <typename T, int D, bool ROUTE = false>
int launch_decode_mma(const spa_kv_layout& kv, int dtype, const DecodeArgs& a, cudaStream_t st, bool pdl = false) {
  using S = DecodeSmem<D, kDecodeStages>;
  if (ROUTE && (!a.cluster_merge || route_scratch_bytes(a.route, D, sizeof(T)) > static_cast<size_t>(S::kStageBytes) ||
                static_cast<size_t>(a.route.q_heads) * D * sizeof(T) > kRouteQVec * 16 * kRouteStagers))
    return SPA_ERR_UNSUPPORTED;
  CUtensorMap kmap, vmap;
  // one TMA load per chunk of K (and of V) covers both 64-column slabs of a row
  if (!spa_make_tensor_map_row_halves(&kmap, kv.k, dtype, kv.total_rows, D, kChunk)) return SPA_ERR_INVALID;
  if (!spa_make_tensor_map_row_halves(&vmap, kv.v, dtype, kv.total_rows, D, kChunk)) return SPA_ERR_INVALID;
  auto kern = decode_mma_kernel<T, D, kDecodeStages, ROUTE>;
  // the receive buffer of the cluster merge: [ns][group] log-sum-exps + [ns][group][ceil(D/ns)]
  const int ns = a.nsplit;
  const size_t recv = a.cluster_merge && ns > 1
                          ? sizeof(float) * (((static_cast<size_t>(ns) * a.group + 3) & ~size_t(3)) +
                                             static_cast<size_t>(ns) * a.group * ((D + ns - 1) / ns))
                          : 0;
  const size_t smem = S::kBytes + recv;
  SPA_CHECK_CUDA(spa_set_smem_once(kern, static_cast<int>(smem)));
  SPA_CHECK_CUDA(launch_ex(kern, dim3(a.nsplit, a.Hkv, a.B), dim3(kDecodeThreads), smem, st,
                           a.early_local != 0 || pdl, a.cluster_merge ? a.nsplit : 1, kmap, vmap, a));
  return SPA_OK;
}

template <typename T>
int launch_decode(const spa_kv_layout& kv, int dtype, DecodeArgs a, bool fast, cudaStream_t st) {
  const int nslots = a.nsplit;
  if (fast) {
    const int rc = a.D == 128 ? launch_decode_mma<T, 128>(kv, dtype, a, st) : launch_decode_mma<T, 64>(kv, dtype, a, st);
    if (rc || a.cluster_merge || nslots <= 1) return rc;
  } else {
    decode_generic_kernel<T><<<dim3(a.nsplit, a.Hq, a.B), 32, 0, st>>>(static_cast<const T*>(kv.k),
                                                                        static_cast<const T*>(kv.v), a);
    SPA_CHECK_CUDA(cudaGetLastError());
  }
  if (nslots > 1)
    SPA_CHECK_CUDA(launch_pdl(decode_combine_kernel<T>, dim3(a.B * a.Hq), dim3(kMergeThreads), 0, st, true,
                              a.part_o, a.part_lse, nslots, a.D, static_cast<T*>(a.out)));
  return SPA_OK;
}

template <>
int launch_decode<float>(const spa_kv_layout& kv, int dtype, DecodeArgs a, bool, cudaStream_t st) {
  (void)dtype;
  decode_generic_kernel<float><<<dim3(a.nsplit, a.Hq, a.B), 32, 0, st>>>(static_cast<const float*>(kv.k),
                                                                          static_cast<const float*>(kv.v), a);
  SPA_CHECK_CUDA(cudaGetLastError());
  if (a.nsplit > 1) {
    decode_combine_kernel<float><<<a.B * a.Hq, kMergeThreads, 0, st>>>(a.part_o, a.part_lse, a.nsplit, a.D,
                                                                        static_cast<float*>(a.out));
    SPA_CHECK_CUDA(cudaGetLastError());
  }
  return SPA_OK;
}

}  // namespace spa

// ---------------------------------------------------------------------------
// C ABI
extern "C" size_t spa_decode_workspace_size(int batch, int q_heads, int kv_heads, int head_dim,
                                            int max_candidates) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || max_candidates < 0) return 0;
  // one partial slot per split per head on the global-merge path; clusters merge on chip,
  // but the generic (CUDA-core) kernel always uses global partials
  const int slots = spa::decode_nsplit(batch, q_heads, kv_heads, max_candidates);
  if (slots <= 1) return 0;
  return static_cast<size_t>(batch) * q_heads * slots * (head_dim + 1) * sizeof(float);
}

extern "C" int spa_decode_plan(int batch, int q_heads, int kv_heads, int max_candidates, int* nsplit,
                               int* cluster_merge) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || max_candidates < 0 || !nsplit || !cluster_merge)
    return SPA_ERR_INVALID;
  const spa::SplitPlan plan = spa::decode_plan(batch, q_heads, kv_heads, max_candidates);
  *nsplit = plan.nsplit;
  *cluster_merge = plan.cluster ? 1 : 0;
  return SPA_OK;
}

namespace spa {
int paged_decode_impl(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                      const spa_kv_layout* kv, const int32_t* context_lens, int local_window, const int64_t* selected,
                      int top_m, int span_len, int max_candidates, double scale, void* out, void* workspace,
                      size_t workspace_bytes, spa_stream_t stream);
}

extern "C" int spa_paged_decode(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                                const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                                const int64_t* selected, int top_m, int max_candidates, double scale, void* out,
                                void* workspace, size_t workspace_bytes, spa_stream_t stream) {
  return spa::paged_decode_impl(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window,
                                selected, top_m, 0, max_candidates, scale, out, workspace, workspace_bytes, stream);
}

extern "C" int spa_paged_gather_decode(const void* q, int dtype, int batch, int q_heads, int kv_heads,
                                       int head_dim, const spa_kv_layout* kv, const int32_t* context_lens,
                                       int local_window, const int64_t* selected, int top_m, int max_candidates,
                                       double scale, void* out, void* workspace, size_t workspace_bytes,
                                       spa_stream_t stream) {
  if (!selected || top_m <= 0) return SPA_ERR_INVALID;
  return spa_paged_decode(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window, selected,
                          top_m, max_candidates, scale, out, workspace, workspace_bytes, stream);
}

extern "C" int spa_span_gather_decode(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                                      const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                                      const int64_t* starts, int n_spans, int span_width, double scale, void* out,
                                      void* workspace, size_t workspace_bytes, spa_stream_t stream) {
  if (!starts || n_spans <= 0 || span_width <= 0) return SPA_ERR_INVALID;
  return spa::paged_decode_impl(q, dtype, batch, q_heads, kv_heads, head_dim, kv, context_lens, local_window, starts,
                                n_spans, span_width, local_window + n_spans * (span_width + 2 * spa::kChunk), scale,
                                out, workspace, workspace_bytes, stream);
}

int spa::paged_decode_impl(const void* q, int dtype, int batch, int q_heads, int kv_heads, int head_dim,
                           const spa_kv_layout* kv, const int32_t* context_lens, int local_window,
                           const int64_t* selected, int top_m, int span_len, int max_candidates, double scale,
                           void* out, void* workspace, size_t workspace_bytes, spa_stream_t stream) {
  if (!q || !out || !kv || !kv->k || !kv->v || !context_lens) return SPA_ERR_INVALID;
  if (!dtype_ok(dtype) || batch <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads) return SPA_ERR_INVALID;
  if (head_dim <= 0 || head_dim > 256 || kv->page_size <= 0 || kv->total_rows <= 0) return SPA_ERR_INVALID;
  if (local_window < 0 || max_candidates < 0 || (selected && top_m <= 0)) return SPA_ERR_INVALID;
  if (kv->page_table && kv->table_stride <= 0) return SPA_ERR_INVALID;
  spa::DecodeArgs a{};
  a.q = q;
  a.out = out;
  a.B = batch;
  a.Hq = q_heads;
  a.Hkv = kv_heads;
  a.group = q_heads / kv_heads;
  a.D = head_dim;
  a.q_batch_heads = q_heads;
  a.q_head_offset = 0;
  a.addr = make_kv_addr(*kv);
  a.ctx_lens = context_lens;
  a.local_window = local_window;
  a.selected = selected;
  a.top_m = selected ? top_m : 0;
  a.span_len = selected ? span_len : 0;
  const spa::SplitPlan plan = spa::decode_plan(batch, q_heads, kv_heads, max_candidates);
  a.nsplit = plan.nsplit;
  a.scale = static_cast<float>(scale);
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.part_o = nullptr;
  a.part_lse = nullptr;
  a.early_local = 0;
  a.q_after_wait = 0;
  {
    const size_t need = spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_candidates);
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
