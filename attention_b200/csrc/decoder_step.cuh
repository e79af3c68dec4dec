// The integrated decoder's whole decode step as ONE persistent kernel: the model of
// attention_b200/decoder.py (the reference's tiny decoder block, train_tiny_transformer.py:
// 134-190, with RMSNorm; its KV-cache page decode, triton_kvcache_transformer_decode.py:
// 35-66, re-built around the paged cache, the router and the promotion table).
//
// Why: at batch <= 4 every piece of the step is a few-microsecond latency chain (weight
// GEMVs of 0.5-4 MB, a router over ~130 pages, a decode over ~1.2k tokens per head), and a
// chain of ~22 dependent launches pays a launch and a grid drain per piece.  Here one
// cooperative grid of one 256-thread CTA per SM runs every phase of every layer:
//
//   per layer:  A  embed / residual add + RMSNorm + QKV (K/V appended, query kept)
//               R  router scores of the routable pages (canonical fp32 order)
//               D  top-m selection, gather decode of 64-token items, split merge
//               O  output projection
//               C  residual add + RMSNorm + fc1 + GELU
//               F  fc2
//   then:       H  residual add + RMSNorm + vocabulary head (fp32 logits) + argmax
//               (CTA 0) greedy token, token log, promotion update, counters += 1
//
// Phases hand data to one another through "flagged words" in global memory: a 64-bit word
// holds a 32-bit payload (one fp32, or two 16-bit elements) and, in its high half, the
// launch's epoch (launch counter + 1).  A consumer spins (bounded) on exactly the words it
// needs until they carry this launch's epoch; a 64-bit aligned store is single-copy atomic,
// so value and flag arrive together and no grid-wide barrier is needed.  Every phase of
// every layer has its own words, so nothing is overwritten within a launch.  Weight rows of
// a phase are requested before the CTA waits for the phase's inputs.
//
// Decode partials (one per 64-candidate item) are flagged words too: the CTA that owns a
// (row, head)'s first item, a window chunk that needs no selection, merges the head's
// partials once all of its own items are done and publishes the head's output.
//
// The linear layers and norms use the arithmetic of linear_rows_kernel / rms_norm_kernel
// (same lane mapping, fma order, reductions and roundings), the router the canonical fp32
// order of router_cluster_kernel, and the promotion update promotion_row_update; only the
// attention's split structure differs from the multi-launch form (fp32 partials, accurate
// expf), so its outputs agree to rounding.
#pragma once

#include "common.cuh"

namespace spa {

constexpr int kDsThreads = 256;
constexpr int kDsWarps = kDsThreads / 32;
// Threads of a CTA that poll flagged words: every CTA waits for the same few words, and
// hundreds of threads per CTA spinning on them saturate the L2 slices that hold them (and
// delay the very stores they wait for); one warp per CTA keeps that traffic small.
constexpr int kDsPollers = 32;
constexpr int kDsChunk = 64;        // candidate tokens per decode item
constexpr int kDsMaxRows = 4;       // batch rows
constexpr int kDsMaxLayers = SPA_DECODER_MAX_LAYERS;
constexpr int kDsMaxPages = 4096;   // routable pages per row (selection keys staged in shared memory)
constexpr int kDsMaxTopM = 32;
constexpr int kDsMaxWidth = 512;    // d_model (norm rows held in registers: 2 elements per thread)
constexpr int kDsMaxSlots = 512;    // promotion slots per row
constexpr int kDsMaxSumRegs = kDsMaxWidth / 32;  // router: heads * head_dim / 32 summary values per lane

struct DsLayer {
  const void *norm1, *qkv_w, *qkv_b, *out_w, *out_b, *norm2, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
  void *k, *v;
  const float* summ;
};

// Word offsets of one layer's flagged words (per batch row: row stride in words).
struct DsWords {
  int64_t xin, qkv, score, attn, o, xmid, hid, mlp, per_layer;
};

struct DsArgs {
  int B, D, H, Dh, F, V, L, P, W, top_m, m, msel, n, n_cap, slots, ttl, log_len, nchmax, G;
  float eps, rscale, ascale;
  const void *emb, *pos, *norm_f, *head;
  int64_t emb_rows, pos_rows;
  DsLayer layer[kDsMaxLayers];
  KvAddr addr;
  int64_t* token;
  int32_t* counters;
  float* logits;
  int64_t* log;
  int64_t* selected;
  int32_t *ppages, *plast;
  uint32_t* seq;
  uint64_t* words;    // layer i's words at words + i * wo.per_layer; then the argmax candidates
  uint64_t* cand;     // [G][B][2]
  uint64_t* pwords;   // decode partials, flagged words [L][B][H][nchmax][Dh + 2]
  uint32_t* ctrs;     // phase arrival counters [2 launch parities][6 L + 1]
  DsWords wo;
  int smem_bytes;
};

// ---------------------------------------------------------------- flagged words
__device__ __forceinline__ uint64_t fw_load(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t fw_load_acquire(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fw_store(uint64_t* p, uint32_t payload, uint32_t epoch) {
  const uint64_t v = (static_cast<uint64_t>(epoch) << 32) | payload;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fw_store_release(uint64_t* p, uint32_t payload, uint32_t epoch) {
  const uint64_t v = (static_cast<uint64_t>(epoch) << 32) | payload;
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Spins until *p carries `epoch`; returns its payload.  Bounded: after SPA_WAIT_CYCLES (or at
// once when another bounded wait on the device has given up) it raises the timeout bit and
// returns 0.
template <bool kAcquire = false>
__device__ __noinline__ uint32_t fw_wait(const uint64_t* p, uint32_t epoch) {
  const long long t0 = clock64();
  uint32_t spins = 0;
  while (true) {
    const uint64_t v = kAcquire ? fw_load_acquire(p) : fw_load(p);
    if (static_cast<uint32_t>(v >> 32) == epoch) return static_cast<uint32_t>(v);
    if ((++spins & 63u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(&g_spa_error_flags) & SPA_DEVERR_WAIT_TIMEOUT) return 0;
      if (clock64() - t0 > SPA_WAIT_CYCLES) {
        spa_raise(SPA_DEVERR_WAIT_TIMEOUT);
        return 0;
      }
    }
  }
}
// Spins (one thread, bounded like fw_wait) until *ctr >= target; acquire, so the stores that
// the counted arrivals released are visible to the caller's CTA after its next barrier.
__device__ __noinline__ void ds_wait_count(const uint32_t* ctr, uint32_t target) {
  const long long t0 = clock64();
  uint32_t spins = 0;
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return;
    if ((++spins & 63u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(&g_spa_error_flags) & SPA_DEVERR_WAIT_TIMEOUT) return;
      if (clock64() - t0 > SPA_WAIT_CYCLES) {
        spa_raise(SPA_DEVERR_WAIT_TIMEOUT);
        return;
      }
    }
  }
}

// Payloads of the flagged words [0, n) of src into dst[0, n) (shared memory), read by
// threads [0, nthreads) with four requests in flight each; the caller synchronises the CTA
// before the others use dst.  One copy of this code serves every phase.
__device__ __noinline__ void ds_poll(const uint64_t* src, int n, uint32_t epoch, uint32_t* dst, int nthreads) {
  if (static_cast<int>(threadIdx.x) >= nthreads) return;
  for (int base = threadIdx.x; base < n; base += 4 * nthreads) {
    uint64_t v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * nthreads;
      v[u] = i < n ? fw_load(src + i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * nthreads;
      if (i < n) dst[i] = static_cast<uint32_t>(v[u] >> 32) == epoch ? static_cast<uint32_t>(v[u]) : fw_wait(src + i, epoch);
    }
  }
}

// E elements of T per 32-bit payload.
template <typename T>
struct DsPack {
  static constexpr int E = 4 / static_cast<int>(sizeof(T));
  static __device__ __forceinline__ uint32_t pack(const T* e) {
    if constexpr (sizeof(T) == 4) {
      return __float_as_uint(*reinterpret_cast<const float*>(e));
    } else {
      const uint16_t lo = *reinterpret_cast<const uint16_t*>(e), hi = *reinterpret_cast<const uint16_t*>(e + 1);
      return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
  }
  static __device__ __forceinline__ void unpack(uint32_t w, T* e) {
    if constexpr (sizeof(T) == 4) {
      *reinterpret_cast<uint32_t*>(e) = w;
    } else {
      reinterpret_cast<uint16_t*>(e)[0] = static_cast<uint16_t>(w & 0xffffu);
      reinterpret_cast<uint16_t*>(e)[1] = static_cast<uint16_t>(w >> 16);
    }
  }
};

// ---------------------------------------------------------------- shared memory plan
struct DsSmem {
  int bufA, bufB, xs, qf, ks, vs, sc, tval, red, po, mrg, keys, scw, sel, part, argv, argi, misc, promo, wbar, wst,
      wslot, tab, total;
};
__host__ __device__ inline int ds_align(int x) { return (x + 15) & ~15; }
__host__ __device__ inline DsSmem ds_smem_plan(int esize, int B, int D, int F, int Dh, int n_cap, int top_m,
                                               int slots, int nchmax, int layers, int grid, int table_stride) {
  DsSmem s;
  int o = 0;
  const int kmax = D > F ? D : F;
  s.bufA = o; o += ds_align(B * D * esize);
  s.bufB = o; o += ds_align(B * D * esize);
  s.xs = o; o += ds_align(B * kmax * esize);
  s.qf = o; o += ds_align(B * D * 4);
  s.ks = o; o += ds_align(kDsChunk * Dh * esize);
  s.vs = o; o += ds_align(kDsChunk * Dh * esize);
  s.sc = o; o += ds_align(kDsChunk * 4);
  s.tval = o; o += ds_align(kDsChunk * 4);
  s.red = o; o += ds_align(kDsThreads * 4);
  s.po = o; o += ds_align((Dh + 2) * 4);
  s.mrg = o; o += ds_align(nchmax * (Dh + 2) * 4);
  s.keys = o; o += ds_align((n_cap + 2) * 8);
  // polled payloads: a row's scores, or every worker's argmax candidates
  s.scw = o; o += ds_align((n_cap > 2 * grid * B ? n_cap : 2 * grid * B) * 4);
  s.sel = o; o += ds_align(layers * kDsMaxRows * (top_m > 0 ? top_m : 1) * 8);
  s.part = o; o += ds_align(kDsMaxRows * 8 * 4);
  s.argv = o; o += ds_align(kDsWarps * kDsMaxRows * 4);
  s.argi = o; o += ds_align(kDsWarps * kDsMaxRows * 4);
  s.misc = o; o += ds_align(64);
  s.promo = o; o += ds_align(kDsWarps * ((top_m > 0 ? top_m : 1) + slots) * 8);
  s.wbar = o; o += ds_align(kDsWarps * 8);
  // a warp's weight slot holds one column group of the widest layer (E * esize = 4 bytes
  // per input feature), or several groups of a narrower one
  s.wslot = ds_align(4 * kmax);
  s.wst = o; o += kDsWarps * s.wslot;
  s.tab = o; o += ds_align(B * table_stride * 4);  // the page-table rows, staged once
  s.total = o;
  return s;
}

// ---------------------------------------------------------------- GEMV pieces
// A warp computes groups of E adjacent output columns (one flagged word per row).  The
// warp's weight rows of a phase are staged in its shared-memory slot by one bulk copy per
// group (TMA, cp.async.bulk, no multicast), issued before the CTA waits for the phase's
// inputs; the products then read shared memory in a rolled loop.  This code runs once per
// phase on each SM, so it is kept small: unrolled per-column register pipelines made the
// products instruction-fetch bound.

// 1D bulk copy of `bytes` from global memory into this CTA's shared memory, completing
// transaction bytes on `bar`.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// acc[e] = sum_k w[e * K + k] * x[k] for the E rows of a column group and one input row
// (16-byte aligned, shared or global memory): lane chunks k = (lane + 32 u) * kVec, u
// ascending, fma in element order, then the xor butterfly -- linear_rows_kernel's order.
template <typename T>
__device__ __noinline__ void ds_dot_rows(const T* w, const T* x, int K, float (&acc)[DsPack<T>::E]) {
  constexpr int E = DsPack<T>::E, kVec = 16 / static_cast<int>(sizeof(T));
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
#pragma unroll 1
  for (int k = lane * kVec; k < K; k += 32 * kVec) {
    const uint4 xv = *reinterpret_cast<const uint4*>(x + k);
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = dot16<T>(*reinterpret_cast<const uint4*>(w + e * K + k), xv, acc[e]);
  }
#pragma unroll
  for (int e = 0; e < E; ++e)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], off);
}



__device__ __forceinline__ int ds_pick_int(const int (&a)[kDsMaxRows], int m) {
  int v = a[0];
#pragma unroll
  for (int k = 1; k < kDsMaxRows; ++k)
    if (m == k) v = a[k];
  return v;
}

// The payload of one flagged word of this launch (waiting, bounded, if it has not arrived).
__device__ __forceinline__ uint32_t fw_get(const uint64_t* p, uint32_t epoch) {
  const uint64_t v = fw_load(p);
  return static_cast<uint32_t>(v >> 32) == epoch ? static_cast<uint32_t>(v) : fw_wait(p, epoch);
}

// B rows of `width` elements from flagged words (row stride `stride` words) into dst
// [B][width] (the poller threads read; the caller synchronises the CTA).  Not inlined: the
// phases share one copy of the code (each SM runs a phase once per layer, so inlined
// copies would be fetched cold every time).
template <typename T>
__device__ __forceinline__ void ds_stage_words(const uint64_t* src, int width, int stride, int B, T* dst,
                                               uint32_t epoch) {
  // a payload holds E consecutive elements in memory order, so it lands in dst as is
  const int nw = width / DsPack<T>::E;
  if (stride == nw) {
    ds_poll(src, B * nw, epoch, reinterpret_cast<uint32_t*>(dst), kDsThreads);
  } else {
    for (int m = 0; m < B; ++m)
      ds_poll(src + static_cast<int64_t>(m) * stride, nw, epoch, reinterpret_cast<uint32_t*>(dst + m * width),
              kDsThreads);
  }
}

// The top-m pages of one row (CTA-wide): its n scores from flagged words, rank keys, and
// key_select's ranking (higher score first, ties to the lower page) into out[0, m).
__device__ __noinline__ void ds_select_row(const uint64_t* score_words, int n, int m, uint32_t epoch, uint32_t* scw,
                                           uint64_t* keys, int64_t* out) {
  ds_poll(score_words, n, epoch, scw, kDsThreads);
  __syncthreads();
  for (int t = threadIdx.x; t < n; t += kDsThreads) keys[t] = rank_key(__uint_as_float(scw[t]), t);
  __syncthreads();
  key_select(keys, n, m, out);  // ends with __syncthreads
}

// The promotion update of rows [0, rows) with their selections (one warp per row).
__device__ __noinline__ void ds_promotion(int32_t* pages, int32_t* last_hit, const int64_t* selected, int rows,
                                          int msel, int slots, int step, int ttl, int64_t* stage) {
  const int warp = threadIdx.x >> 5;
  int64_t* psel = stage + warp * (msel + slots);
  int32_t* ppg = reinterpret_cast<int32_t*>(psel + msel);
  for (int r = warp; r < rows; r += kDsWarps)
    promotion_row_update(pages + static_cast<int64_t>(r) * slots, last_hit + static_cast<int64_t>(r) * slots,
                         selected + static_cast<int64_t>(r) * msel, msel, slots, step, ttl, psel, ppg, ppg + slots);
}

// Residual add + RMSNorm of B rows of width D: bufA (+ bufB) hold the inputs as T.
// rms_norm_kernel's mapping and order (threads 0..255, element i = thread + 256 u); the
// normalised rows go to xs, the summed rows back to bufA.  Rows in bad_mask give zeros.
// Called by every thread of the CTA (two barriers inside).
// The thread's norm weights (elements thread and thread + 256) come in w0, w1: they are read
// before the phase waits for its inputs (ds_norm_weights).
static_assert(kDsMaxWidth == 512, "the norm holds two elements per thread");
template <typename T>
__device__ __forceinline__ float2 ds_norm_weights(const T* __restrict__ nw, int D) {
  const int i = threadIdx.x;
  return make_float2(i < D ? to_f32(nw[i]) : 0.f, i + 256 < D ? to_f32(nw[i + 256]) : 0.f);
}
template <typename T>
__device__ __noinline__ void ds_norm_rows(T* bufA, const T* bufB, T* xs, float* npart, float w0, float w1, bool add,
                                          int bad_mask, int B, int D, float eps) {
  constexpr int kHeld = kDsMaxWidth / 256;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float held[kDsMaxRows][kHeld];
  const float wn[kHeld] = {w0, w1};
  if (tid < 256) {
#pragma unroll
    for (int u = 0; u < kHeld; ++u) {
      const int i = tid + u * 256;
#pragma unroll
      for (int m = 0; m < kDsMaxRows; ++m) {
        float v = 0.f;
        if (m < B && i < D && !((bad_mask >> m) & 1)) {
          v = to_f32(bufA[m * D + i]);
          if (add) v = to_f32(from_f32<T>(v + to_f32(bufB[m * D + i])));
        }
        held[m][u] = v;
      }
    }
#pragma unroll
    for (int m = 0; m < kDsMaxRows; ++m) {
      if (m >= B) break;
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < kHeld; ++u) {
        const int i = tid + u * 256;
        if (i < D) ss = fmaf(held[m][u], held[m][u], ss);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) npart[m * 8 + warp] = ss;
    }
  }
  __syncthreads();
  if (tid < 256) {
#pragma unroll
    for (int m = 0; m < kDsMaxRows; ++m) {
      if (m >= B) break;
      float tot = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) tot += npart[m * 8 + k];
      const float r = rsqrtf(tot / static_cast<float>(D) + eps);
      const bool bad = (bad_mask >> m) & 1;
#pragma unroll
      for (int u = 0; u < kHeld; ++u) {
        const int i = tid + u * 256;
        if (i < D) {
          xs[m * D + i] = bad ? from_f32<T>(0.f) : from_f32<T>(held[m][u] * r * wn[u]);
          bufA[m * D + i] = from_f32<T>(held[m][u]);
        }
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- the kernel
// One CTA of kDsThreads per SM, launched cooperatively (every CTA resident at once: a CTA
// spins only on words that CTAs already running will write).  DH = head_dim.
template <typename T, int DH>
__global__ void __launch_bounds__(kDsThreads, 1) decoder_step_kernel(const __grid_constant__ DsArgs a) {
  extern __shared__ __align__(16) unsigned char ds_smem[];
  constexpr int E = DsPack<T>::E;
  constexpr int kVec = 16 / static_cast<int>(sizeof(T));
  constexpr int NSL = DH / 32;  // summary / query values per lane and head
  const int tstride = a.addr.page_table ? a.addr.table_stride : 0;
  const DsSmem sp =
      ds_smem_plan(sizeof(T), a.B, a.D, a.F, DH, a.n_cap, a.top_m, a.slots, a.nchmax, a.L, a.G, tstride);
  T* bufA = reinterpret_cast<T*>(ds_smem + sp.bufA);
  T* bufB = reinterpret_cast<T*>(ds_smem + sp.bufB);
  T* xs = reinterpret_cast<T*>(ds_smem + sp.xs);
  float* qf = reinterpret_cast<float*>(ds_smem + sp.qf);
  T* ks = reinterpret_cast<T*>(ds_smem + sp.ks);
  T* vs = reinterpret_cast<T*>(ds_smem + sp.vs);
  float* sc = reinterpret_cast<float*>(ds_smem + sp.sc);
  int* tval = reinterpret_cast<int*>(ds_smem + sp.tval);
  float* red = reinterpret_cast<float*>(ds_smem + sp.red);
  float* po = reinterpret_cast<float*>(ds_smem + sp.po);
  float* mrg = reinterpret_cast<float*>(ds_smem + sp.mrg);  // [nchmax][DH + 2]
  uint64_t* keys = reinterpret_cast<uint64_t*>(ds_smem + sp.keys);
  uint32_t* scw = reinterpret_cast<uint32_t*>(ds_smem + sp.scw);
  int64_t* selrow = reinterpret_cast<int64_t*>(ds_smem + sp.sel);  // [layers][kDsMaxRows][msel]
  float* npart = reinterpret_cast<float*>(ds_smem + sp.part);       // [kDsMaxRows][8]
  float* argv = reinterpret_cast<float*>(ds_smem + sp.argv);        // [warps][kDsMaxRows]
  int* argi = reinterpret_cast<int*>(ds_smem + sp.argi);
  int* misc = reinterpret_cast<int*>(ds_smem + sp.misc);
  // misc: [0..3] position, [4..7] context length, [8] step, [9] epoch, [10] merge flag,
  //       [11..14] row selected by this CTA in the current layer
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the last CTA is the service CTA (selections and the promotion table, off the critical
  // path); the others, G of them, are the workers every phase is spread over
  const int B = a.B, D = a.D, H = a.H, G = a.G - 1;
  const int wD = D / E, wF = a.F / E;
  const int n = a.n, msel = a.msel, m_sel = a.m;

  if (tid < kDsMaxRows) {
    misc[tid] = tid < B ? a.counters[tid] : -1;
    misc[4 + tid] = tid < B ? a.counters[B + tid] : 0;
  }
  uint64_t* wbar = reinterpret_cast<uint64_t*>(ds_smem + sp.wbar);  // [warps], one per weight slot
  unsigned char* wst = ds_smem + sp.wst + (threadIdx.x >> 5) * sp.wslot;
  if (tid == 0) {
    misc[8] = a.counters[2 * B];
    misc[9] = static_cast<int>(*reinterpret_cast<volatile uint32_t*>(a.seq) + 1u);
    for (int w = 0; w < kDsWarps; ++w) mbar_init(&wbar[w], 1);
  }
  __syncthreads();
  uint32_t wpar = 0;  // phase parity of this warp's weight barrier
  int32_t* tab = reinterpret_cast<int32_t*>(ds_smem + sp.tab);  // [B][tstride]
  for (int i = tid; i < B * tstride; i += kDsThreads) tab[i] = a.addr.page_table[i];  // rows b < B are contiguous
  __syncthreads();
  // KvAddr::row with the page-table rows read from shared memory
  auto kv_row = [&](int b, int h, int t) -> int64_t {
    const int lp = t / a.addr.page_size;
    int64_t pg = lp;
    if (tstride) {
      if (lp >= tstride) return -1;
      pg = tab[b * tstride + lp];
      if (pg < 0) return -1;
    }
    return b * a.addr.batch_stride_rows + pg * a.addr.page_stride_rows + h * a.addr.head_stride_rows +
           (t - lp * a.addr.page_size);
  };
  const uint32_t epoch = static_cast<uint32_t>(misc[9]);
  const int posv[kDsMaxRows] = {misc[0], misc[1], misc[2], misc[3]};

  auto norm_rows = [&](float2 nw, bool add, int bad_mask) {
    ds_norm_rows<T>(bufA, bufB, xs, npart, nw.x, nw.y, add, bad_mask, B, D, a.eps);
  };
  // CTA 0 publishes the summed rows (bufA) as flagged words
  auto publish_rows = [&](uint64_t* dst) {
    if (blockIdx.x != 0) return;
    for (int i = tid; i < B * wD; i += kDsThreads) {
      const int m = i / wD, w = i - m * wD;
      fw_store(dst + i, DsPack<T>::pack(bufA + m * D + w * E), epoch);
    }
  };
  // B rows of `width` elements from flagged words (row stride `stride` words) into dst [B][width]
  auto stage_words = [&](const uint64_t* src, int width, int stride, T* dst) {
    ds_stage_words<T>(src, width, stride, B, dst, epoch);
  };
  // One linear layer over xs ([B][K]) for N = groups * E columns: group g (columns g*E ..
  // g*E+E-1) belongs to CTA g mod G, warp (g / G) mod warps.  gemv_issue stages the warp's
  // groups (as many as its slot holds) before the caller waits for the phase's inputs;
  // gemv_run waits for them and computes every group and row, emit(g, m, acc).
  struct GemvPre {
    int staged;
    float bias[E];  // the warp's first group's bias (0 without one), read before the wait
  };
  auto gemv_issue = [&](const void* w, const void* bias, int N, int K) {
    const int ngroups = N / E;
    GemvPre pre;
    const int g0 = blockIdx.x + G * warp;
#pragma unroll
    for (int e = 0; e < E; ++e)
      pre.bias[e] = bias && g0 < ngroups ? to_f32(static_cast<const T*>(bias)[g0 * E + e]) : 0.f;
    const int gbytes = 4 * K;  // E columns of K elements
    const int fit = sp.wslot / gbytes;
    int cnt = 0;
    for (int g = blockIdx.x + G * warp; g < ngroups && cnt < fit; g += G * kDsWarps) ++cnt;
    __syncwarp();  // every lane is done with the slot's previous contents
    if (cnt > 0 && lane == 0) {
      fence_proxy_async_smem();  // the slot's generic-proxy reads come before the copies' writes
      mbar_arrive_expect_tx(&wbar[warp], static_cast<uint32_t>(cnt * gbytes));
      int g = blockIdx.x + G * warp;
      for (int j = 0; j < cnt; ++j, g += G * kDsWarps)
        bulk_g2s(wst + j * gbytes, static_cast<const T*>(w) + static_cast<int64_t>(g) * E * K,
                 static_cast<uint32_t>(gbytes), &wbar[warp]);
    }
    pre.staged = cnt;
    return pre;
  };
  auto gemv_run = [&](const void* w, const void* bias, int N, int K, const GemvPre& pre, auto&& emit) {
    const int ngroups = N / E;
    const int staged = pre.staged;
    if (staged > 0) {
      mbar_wait_bounded(&wbar[warp], wpar);
      wpar ^= 1u;
    }
    int j = 0;
    for (int g = blockIdx.x + G * warp; g < ngroups; g += G * kDsWarps, ++j) {
      const T* wr = j < staged ? reinterpret_cast<const T*>(wst + j * 4 * K)
                               : static_cast<const T*>(w) + static_cast<int64_t>(g) * E * K;
      float bv[E];
#pragma unroll
      for (int e = 0; e < E; ++e)
        bv[e] = j == 0 ? pre.bias[e] : (bias ? to_f32(static_cast<const T*>(bias)[g * E + e]) : 0.f);
#pragma unroll 1
      for (int m = 0; m < B; ++m) {
        float acc[E];
        ds_dot_rows<T>(wr, xs + m * K, K, acc);
        if (bias) {
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] += bv[e];
        }
        emit(g, m, acc);
      }
    }
  };
  // rounding to T (the bias is already added), optional exact GELU (linear_rows_kernel's
  // epilogue), in every lane
  auto epilogue = [&](bool gelu, float (&acc)[E], T (&y)[E]) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      T t = from_f32<T>(acc[e]);
      if (gelu) {
        const float f = to_f32(t);
        t = from_f32<T>(f * 0.5f * (1.f + erff(f * 0.70710678118654752f)));
      }
      y[e] = t;
    }
  };

  // top-m of row b of layer li (CTA-wide): rank keys of the row's scores, key_select's
  // ranking (higher score first, ties to the lower page) into sel_of(li, b)
  auto sel_of = [&](int li, int b) { return selrow + (li * kDsMaxRows + b) * msel; };
  auto select_row = [&](int li, int b) {
    ds_select_row(a.words + static_cast<int64_t>(li) * a.wo.per_layer + a.wo.score + static_cast<int64_t>(b) * a.n_cap,
                  n, m_sel, epoch, scw, keys, sel_of(li, b));
  };

  // Phase hand-offs: every worker CTA adds 1 to the phase's counter once its stores of the
  // phase are done (one release add after a barrier); a consumer CTA has one thread wait
  // until all G workers have arrived (acquire), then reads the phase's words in one round.
  // Counters: per layer 0 QKV, 1 scores, 2 attention, 3 output projection, 4 fc1, 5 fc2;
  // 6 L the argmax candidates.  The launch uses the set of its epoch's parity; CTA 0 clears
  // the other set at the end for the next launch.
  const int nctr = 6 * a.L + 1;
  uint32_t* ctr = a.ctrs + (epoch & 1u) * nctr;
  auto arrive = [&](int idx) {
    __syncthreads();
    if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr + idx) : "memory");
  };
  auto wait_all = [&](int idx) {
    if (tid == 0) ds_wait_count(ctr + idx, static_cast<uint32_t>(G));
    __syncthreads();
  };

  if (blockIdx.x == a.G - 1) {
    // service CTA: every layer's selections as the layer's scores arrive, then the
    // promotion update of every (layer, row) with them.  Its first word (in its own
    // candidate slot) tells CTA 0 that it has read the counters and the launch counter.
    if (tid == 0) fw_store_release(a.cand + static_cast<int64_t>(G) * B * 2, 1u, epoch);
    for (int li = 0; li < a.L; ++li) {
      if (m_sel > 0) wait_all(li * 6 + 1);
      for (int b = 0; b < B; ++b) {
        int64_t* dst = a.selected + (static_cast<int64_t>(li) * B + b) * msel;
        if (m_sel > 0) {
          select_row(li, b);
          if (tid < msel) dst[tid] = sel_of(li, b)[tid];
        } else if (tid == 0) {
          dst[0] = -1;
        }
      }
    }
    const int step = misc[8];
    __syncthreads();
    if (a.ppages)
      ds_promotion(a.ppages, a.plast, a.selected, a.L * B, msel, a.slots, step, a.ttl,
                   reinterpret_cast<int64_t*>(ds_smem + sp.promo));
    return;
  }

  for (int li = 0; li < a.L; ++li) {
    const DsLayer& ly = a.layer[li];
    uint64_t* wl = a.words + static_cast<int64_t>(li) * a.wo.per_layer;
    uint64_t* w_xin = wl + a.wo.xin;
    uint64_t* w_qkv = wl + a.wo.qkv;
    uint64_t* w_score = wl + a.wo.score;
    uint64_t* w_attn = wl + a.wo.attn;
    uint64_t* w_o = wl + a.wo.o;
    uint64_t* w_xmid = wl + a.wo.xmid;
    uint64_t* w_hid = wl + a.wo.hid;
    uint64_t* w_mlp = wl + a.wo.mlp;

    // ---------------------------------------------------------- A: QKV
    {
      const GemvPre pre = gemv_issue(ly.qkv_w, ly.qkv_b, 3 * D, D);
      const float2 nw1 = ds_norm_weights(static_cast<const T*>(ly.norm1), D);
      int bad = 0;
      __syncthreads();  // xs / bufA / bufB of the previous phase are free
      if (li == 0) {
        // token + position embedding rows (rms_norm_kernel's lookup rules)
        const T* emb = static_cast<const T*>(a.emb);
        const T* pos = static_cast<const T*>(a.pos);
        for (int m = 0; m < B; ++m) {
          const int64_t ti = a.token[m];
          const int64_t pi = posv[m];
          if (ti < 0 || ti >= a.emb_rows || pi < 0 || pi >= a.pos_rows) {
            bad |= 1 << m;
            continue;
          }
          for (int i = tid; i < D; i += kDsThreads) {
            bufA[m * D + i] = emb[ti * D + i];
            bufB[m * D + i] = pos[pi * D + i];
          }
        }
        if (bad && blockIdx.x == 0 && tid == 0) spa_raise(SPA_DEVERR_BAD_INDEX);
      } else {
        const uint64_t* pl = a.words + static_cast<int64_t>(li - 1) * a.wo.per_layer;
        wait_all((li - 1) * 6 + 5);
        stage_words(pl + a.wo.xmid, D, wD, bufA);
        stage_words(pl + a.wo.mlp, D, wD, bufB);
      }
      __syncthreads();
      norm_rows(nw1, true, bad);
      publish_rows(w_xin);
      gemv_run(ly.qkv_w, ly.qkv_b, 3 * D, D, pre, [&](int g, int m, float (&acc)[E]) {
        T y[E];
        epilogue(false, acc, y);
        if (lane == 0) {
          fw_store(w_qkv + static_cast<int64_t>(m) * 3 * wD + g, DsPack<T>::pack(y), epoch);
          const int pos = ds_pick_int(posv, m);
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const int c = g * E + e;
            if (c < D || pos < 0) continue;
            // the new token's K / V (spa_kv_append's store)
            const bool isk = c < 2 * D;
            const int rel = isk ? c - D : c - 2 * D;
            const int h = rel / DH, j = rel - h * DH;
            const int64_t row = kv_row(m, h, pos);
            if (row < 0 || row >= a.addr.total_rows)
              spa_raise(SPA_DEVERR_BAD_PAGE);
            else
              static_cast<T*>(isk ? ly.k : ly.v)[row * DH + j] = y[e];
          }
        }
      });
      arrive(li * 6 + 0);
    }

    // ---------------------------------------------------------- R: router scores
    // One warp per (row b, page): the canonical fp32 order (per kv head: 32 lane-strided
    // partial sums, separate multiply and add, xor butterfly; kv heads in order; / Hq, *
    // scale).  The page's summary rows are requested before the query is waited for.
    {
      const int pairs = B * n;
      const int pr0 = blockIdx.x + G * warp;
      float sv[kDsMaxSumRegs];
      auto load_rows = [&](int p) {
        const int b = p / n, pg = p - b * n;
#pragma unroll
        for (int u = 0; u < kDsMaxSumRegs; ++u) {
          const int h = u / NSL, k = u - h * NSL;
          sv[u] = h < H ? __ldg(ly.summ + ((static_cast<int64_t>(b) * H + h) * n + pg) * DH + lane + 32 * k) : 0.f;
        }
      };
      if (pr0 < pairs) load_rows(pr0);
      // the query rows as the router's per-kv-head sums (group of one: 0 + q)
      wait_all(li * 6 + 0);
      stage_words(w_qkv, D, 3 * wD, bufA);  // the query columns of every row
      if (tid < kDsMaxRows) misc[11 + tid] = 0;
      __syncthreads();
      for (int i = tid; i < B * D; i += kDsThreads) qf[i] = __fadd_rn(0.f, to_f32(bufA[i]));
      __syncthreads();
      for (int pr = pr0; pr < pairs; pr += G * kDsWarps) {
        if (pr != pr0) load_rows(pr);
        const int b = pr / n, pg = pr - b * n;
        float total = 0.f;
#pragma unroll
        for (int h = 0; h < kDsMaxSumRegs / NSL; ++h) {
          if (h >= H) break;
          float part = 0.f;
#pragma unroll
          for (int k = 0; k < NSL; ++k) part = __fadd_rn(part, __fmul_rn(qf[b * D + h * DH + lane + 32 * k], sv[h * NSL + k]));
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
          total = __fadd_rn(total, part);
        }
        const float v = __fmul_rn(__fdiv_rn(total, static_cast<float>(H)), a.rscale);
        if (lane == 0) fw_store(w_score + static_cast<int64_t>(b) * a.n_cap + pg, __float_as_uint(v), epoch);
      }
      arrive(li * 6 + 1);
    }

    // ---------------------------------------------------------- D: select + decode + merge
    {
      const int nbh = B * H;
      const int nitems = a.nchmax * nbh;
      for (int it = blockIdx.x; it < nitems; it += G) {
        const int k = it / nbh, r = it - k * nbh, b = r / H, h = r - b * H;
        const int ctx = misc[4 + b];
        const int lo = ctx > a.W ? ctx - a.W : 0;
        const int nwin = ctx - lo;
        const int nc = nwin + m_sel * a.P;
        const int nch = (nc + kDsChunk - 1) / kDsChunk;
        if (k >= nch) continue;
        const int c0 = k * kDsChunk;
        if (m_sel > 0 && c0 + kDsChunk > nwin && !misc[11 + b]) {
          wait_all(li * 6 + 1);
          select_row(li, b);
          if (tid == 0) misc[11 + b] = 1;
          __syncthreads();
        }
        const int pos_b = misc[b];
        // K / V of the item's 64 candidates (the window first, then the selected pages in
        // selection order); the step's own token comes from the QKV words
        constexpr int kPieces = DH / kVec;
        for (int i = tid; i < kDsChunk * kPieces; i += kDsThreads) {
          const int s = i / kPieces, pc = i - s * kPieces;
          const int c = c0 + s;
          bool ok = false;
          uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
          if (c < nc) {
            const int tok = c < nwin ? lo + c
                                     : static_cast<int>(sel_of(li, b)[(c - nwin) / a.P]) * a.P + (c - nwin) % a.P;
            if (tok == pos_b) {
              const uint64_t* kw = w_qkv + static_cast<int64_t>(b) * 3 * wD + (D + h * DH + pc * kVec) / E;
              uint32_t* kd = reinterpret_cast<uint32_t*>(&kv4);
              uint32_t* vd = reinterpret_cast<uint32_t*>(&vv4);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                kd[u] = fw_get(kw + u, epoch);
                vd[u] = fw_get(kw + wD + u, epoch);
              }
              ok = true;
            } else {
              const int64_t row = kv_row(b, h, tok);
              if (row >= 0 && row < a.addr.total_rows) {
                kv4 = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(ly.k) + row * DH + pc * kVec));
                vv4 = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(ly.v) + row * DH + pc * kVec));
                ok = true;
              } else {
                spa_raise(SPA_DEVERR_BAD_PAGE);
              }
            }
          }
          *reinterpret_cast<uint4*>(ks + s * DH + pc * kVec) = kv4;
          *reinterpret_cast<uint4*>(vs + s * DH + pc * kVec) = vv4;
          if (pc == 0) tval[s] = ok ? 1 : 0;
        }
        __syncthreads();
        // scores: warp w takes candidates w * (chunk / warps) onwards
#pragma unroll 1
        for (int u = 0; u < kDsChunk / kDsWarps; ++u) {
          const int s = warp * (kDsChunk / kDsWarps) + u;
          float acc = 0.f;
#pragma unroll
          for (int kk = 0; kk < NSL; ++kk) {
            const int d = lane + 32 * kk;
            acc = fmaf(qf[b * D + h * DH + d], to_f32(ks[s * DH + d]), acc);
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
          if (lane == 0) sc[s] = tval[s] ? acc * a.ascale : -INFINITY;
        }
        __syncthreads();
        if (warp == 0) {
          const float s0 = sc[lane], s1 = sc[lane + 32];
          float mx = fmaxf(s0, s1);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          const float p0 = s0 == -INFINITY ? 0.f : expf(s0 - mx);
          const float p1 = s1 == -INFINITY ? 0.f : expf(s1 - mx);
          float l = p0 + p1;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
          sc[lane] = p0;
          sc[lane + 32] = p1;
          if (lane == 0) {
            po[DH] = mx;
            po[DH + 1] = l;
          }
        }
        __syncthreads();
        {
          constexpr int kGroups = kDsThreads / DH;
          const int j = tid % DH, grp = tid / DH;
          float o = 0.f;
#pragma unroll 4
          for (int s = grp; s < kDsChunk; s += kGroups) o = fmaf(sc[s], to_f32(vs[s * DH + j]), o);
          red[grp * DH + j] = o;
          __syncthreads();
          if (tid < DH) {
            float t = 0.f;
#pragma unroll
            for (int q = 0; q < kGroups; ++q) t += red[q * DH + tid];
            po[tid] = t;
          }
        }
        __syncthreads();
        // the item's partial (output row, max, sum) as flagged words
        const int64_t bh = (static_cast<int64_t>(li) * B + b) * H + h;
        if (tid < DH + 2) fw_store(a.pwords + (bh * a.nchmax + k) * (DH + 2) + tid, __float_as_uint(po[tid]), epoch);
        __syncthreads();  // po is reused by the next item
      }
      // merges: the CTA of a (row, head)'s first item (a window chunk, which needs no
      // selection) merges every partial of the row-head (log-sum-exp) and publishes its
      // output, after all of its own items -- no CTA waits while it holds unfinished items
      for (int r = blockIdx.x; r < nbh; r += G) {
        const int b = r / H, h = r - b * H;
        const int ctx = misc[4 + b];
        const int nwin = ctx - (ctx > a.W ? ctx - a.W : 0);
        const int nch = (nwin + m_sel * a.P + kDsChunk - 1) / kDsChunk;
        const int64_t bh = (static_cast<int64_t>(li) * B + b) * H + h;
        ds_poll(a.pwords + bh * a.nchmax * (DH + 2), nch * (DH + 2), epoch, reinterpret_cast<uint32_t*>(mrg),
                kDsThreads);
        __syncthreads();
        T* res = reinterpret_cast<T*>(red);
        if (tid < DH) {
          float M = -INFINITY;
          for (int q = 0; q < nch; ++q) M = fmaxf(M, mrg[q * (DH + 2) + DH]);
          float ls = 0.f, o = 0.f;
          for (int q = 0; q < nch; ++q) {
            const float mq = mrg[q * (DH + 2) + DH];
            const float wq = mq == -INFINITY ? 0.f : expf(mq - M);
            ls = fmaf(mrg[q * (DH + 2) + DH + 1], wq, ls);
            o = fmaf(mrg[q * (DH + 2) + tid], wq, o);
          }
          res[tid] = from_f32<T>(ls > 0.f ? o / ls : 0.f);
        }
        __syncthreads();
        if (tid < DH / E)
          fw_store(w_attn + static_cast<int64_t>(b) * wD + (h * DH) / E + tid, DsPack<T>::pack(res + tid * E), epoch);
        __syncthreads();
      }
      arrive(li * 6 + 2);
    }

    // ---------------------------------------------------------- O: output projection
    {
      const GemvPre pre = gemv_issue(ly.out_w, ly.out_b, D, D);
      __syncthreads();
      wait_all(li * 6 + 2);
      stage_words(w_attn, D, wD, xs);
      __syncthreads();
      gemv_run(ly.out_w, ly.out_b, D, D, pre, [&](int g, int m, float (&acc)[E]) {
        T y[E];
        epilogue(false, acc, y);
        if (lane == 0) fw_store(w_o + static_cast<int64_t>(m) * wD + g, DsPack<T>::pack(y), epoch);
      });
      arrive(li * 6 + 3);
    }

    // ---------------------------------------------------------- C: norm2 + fc1 + GELU
    {
      const GemvPre pre = gemv_issue(ly.fc1_w, ly.fc1_b, a.F, D);
      const float2 nw2 = ds_norm_weights(static_cast<const T*>(ly.norm2), D);
      __syncthreads();
      wait_all(li * 6 + 3);
      stage_words(w_xin, D, wD, bufA);
      stage_words(w_o, D, wD, bufB);
      __syncthreads();
      norm_rows(nw2, true, 0);
      publish_rows(w_xmid);
      gemv_run(ly.fc1_w, ly.fc1_b, a.F, D, pre, [&](int g, int m, float (&acc)[E]) {
        T y[E];
        epilogue(true, acc, y);
        if (lane == 0) fw_store(w_hid + static_cast<int64_t>(m) * wF + g, DsPack<T>::pack(y), epoch);
      });
      arrive(li * 6 + 4);
    }

    // ---------------------------------------------------------- F: fc2
    {
      const GemvPre pre = gemv_issue(ly.fc2_w, ly.fc2_b, D, a.F);
      __syncthreads();
      wait_all(li * 6 + 4);
      stage_words(w_hid, a.F, wF, xs);
      __syncthreads();
      gemv_run(ly.fc2_w, ly.fc2_b, D, a.F, pre, [&](int g, int m, float (&acc)[E]) {
        T y[E];
        epilogue(false, acc, y);
        if (lane == 0) fw_store(w_mlp + static_cast<int64_t>(m) * wD + g, DsPack<T>::pack(y), epoch);
      });
      arrive(li * 6 + 5);
    }
  }

  // ------------------------------------------------------------ H: norm_f + head + argmax
  {
    const GemvPre pre = gemv_issue(a.head, nullptr, a.V, D);
    const float2 nwf = ds_norm_weights(static_cast<const T*>(a.norm_f), D);
    __syncthreads();
    const uint64_t* pl = a.words + static_cast<int64_t>(a.L - 1) * a.wo.per_layer;
    wait_all((a.L - 1) * 6 + 5);
    stage_words(pl + a.wo.xmid, D, wD, bufA);
    stage_words(pl + a.wo.mlp, D, wD, bufB);
    __syncthreads();
    norm_rows(nwf, true, 0);
    // fp32 logits of the rounded products; the warp's best (value, column) per row in lane m
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    gemv_run(a.head, nullptr, a.V, D, pre, [&](int g, int m, float (&acc)[E]) {
      T y[E];
      epilogue(false, acc, y);
      if (lane == m) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int c = g * E + e;
          const float f = to_f32(y[e]);
          a.logits[static_cast<int64_t>(m) * a.V + c] = f;
          if (argmax_beats(f, c, bv, bi)) {
            bv = f;
            bi = c;
          }
        }
      }
    });
    if (lane < kDsMaxRows) {
      argv[warp * kDsMaxRows + lane] = bv;
      argi[warp * kDsMaxRows + lane] = bi;
    }
    __syncthreads();
    if (tid < B) {
      float v = -INFINITY;
      int i = 0x7fffffff;
      for (int w = 0; w < kDsWarps; ++w)
        if (argmax_beats(argv[w * kDsMaxRows + tid], argi[w * kDsMaxRows + tid], v, i)) {
          v = argv[w * kDsMaxRows + tid];
          i = argi[w * kDsMaxRows + tid];
        }
      uint64_t* cw = a.cand + (static_cast<int64_t>(blockIdx.x) * B + tid) * 2;
      fw_store(cw, __float_as_uint(v), epoch);
      fw_store(cw + 1, static_cast<uint32_t>(i), epoch);
    }
    // release (cumulative over the barrier): this CTA's logits, its candidates and its reads
    // of the step counters come before its arrival
    arrive(6 * a.L);
  }

  // ------------------------------------------------------------ CTA 0: token and counters
  if (blockIdx.x != 0) return;
  // every worker's best (value, column) of every row, polled with relaxed loads; an acquire
  // fence after all of them.  argmax_beats is a total order, so the reduction order does not
  // change the winner.
  wait_all(6 * a.L);
  ds_poll(a.cand, G * B * 2, epoch, scw, kDsThreads);
  __syncthreads();
  if (warp < B) {
    const int m = warp;
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int c = lane; c < G; c += 32) {
      const float cv = __uint_as_float(scw[(c * B + m) * 2]);
      const int ci = static_cast<int>(scw[(c * B + m) * 2 + 1]);
      if (argmax_beats(cv, ci, v, i)) {
        v = cv;
        i = ci;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, i, off);
      if (argmax_beats(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (lane == 0) {
      a.token[m] = i;
      const int p = posv[m];
      if (a.log && p >= 0 && p < a.log_len) a.log[static_cast<int64_t>(p) * B + m] = i;
    }
  }
  if (tid == 0) {
    fw_get(a.cand + static_cast<int64_t>(G) * B * 2, epoch);
    asm volatile("fence.acq_rel.gpu;" ::: "memory");  // the counter updates come after that read
  }
  __syncthreads();
  // every worker has read the counters and the launch counter (their candidate words come
  // after those reads), and so has the service CTA (its first word)
  if (tid < 2 * B + 1) a.counters[tid] += 1;
  // the next launch's arrival counters start from zero
  uint32_t* ctr_next = a.ctrs + ((epoch + 1u) & 1u) * nctr;
  for (int i = tid; i < nctr; i += kDsThreads) ctr_next[i] = 0;
  if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.seq) = epoch;
}

// ---------------------------------------------------------------- host side
struct DsLayout {
  DsWords wo;
  int64_t cand_words;
  size_t seq_off, words_off, cand_off, parts_off, ctr_off, bytes;
  int nchmax;
};

inline DsLayout ds_layout(int esize, int B, int D, int H, int F, int L, int n_cap, int W, int top_m, int P, int G) {
  DsLayout l;
  const int E = 4 / esize;
  const int64_t wD = D / E, wF = F / E;
  l.wo.xin = 0;
  l.wo.qkv = l.wo.xin + B * wD;
  l.wo.score = l.wo.qkv + B * 3 * wD;
  l.wo.attn = l.wo.score + static_cast<int64_t>(B) * n_cap;
  l.wo.o = l.wo.attn + B * wD;
  l.wo.xmid = l.wo.o + B * wD;
  l.wo.hid = l.wo.xmid + B * wD;
  l.wo.mlp = l.wo.hid + B * wF;
  l.wo.per_layer = l.wo.mlp + B * wD;
  l.nchmax = static_cast<int>((static_cast<int64_t>(W) + static_cast<int64_t>(top_m) * P + kDsChunk - 1) / kDsChunk);
  if (l.nchmax < 1) l.nchmax = 1;
  l.cand_words = static_cast<int64_t>(G) * B * 2;
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  const int Dh = D / H;
  l.seq_off = 0;
  l.words_off = 256;
  l.cand_off = up(l.words_off + sizeof(uint64_t) * static_cast<size_t>(L) * l.wo.per_layer);
  l.parts_off = up(l.cand_off + sizeof(uint64_t) * static_cast<size_t>(l.cand_words));
  l.ctr_off =
      up(l.parts_off + sizeof(uint64_t) * static_cast<size_t>(L) * B * H * l.nchmax * static_cast<size_t>(Dh + 2));
  l.bytes = up(l.ctr_off + sizeof(uint32_t) * 2 * static_cast<size_t>(6 * L + 1));
  return l;
}

inline int ds_table_pages(const spa_decoder_step_params* p) {
  return p->kv.page_table ? p->kv.table_stride : p->max_pages;
}

// Shape checks shared by the size query and the step.
inline int ds_check(const spa_decoder_step_params* p) {
  if (!p || !dtype_ok(p->dtype)) return SPA_ERR_INVALID;
  if (p->batch < 1 || p->layers < 1 || p->heads < 1 || p->d_model < 1 || p->ffn < 1 || p->vocab < 1)
    return SPA_ERR_INVALID;
  if (p->d_model % p->heads || p->local_window < 0 || p->top_m < 0 || p->n_pages < 0 || p->kv.page_size < 1 ||
      p->max_pages < 0)
    return SPA_ERR_INVALID;
  const int dh = p->d_model / p->heads;
  if (p->batch > kDsMaxRows || p->layers > kDsMaxLayers || (dh != 32 && dh != 64 && dh != 128) ||
      p->d_model > kDsMaxWidth || p->d_model % 8 || p->ffn % 8 || p->vocab % 8 || p->top_m > kDsMaxTopM ||
      p->promo_slots > kDsMaxSlots)
    return SPA_ERR_UNSUPPORTED;
  const int cap = ds_table_pages(p);
  if (cap < 0 || cap > kDsMaxPages || p->n_pages > cap) return SPA_ERR_UNSUPPORTED;
  return SPA_OK;
}

template <typename T, int DH>
int ds_launch(const DsArgs& a, int smem, cudaStream_t st) {
  auto kern = decoder_step_kernel<T, DH>;
  SPA_CHECK_CUDA(spa_set_smem_once(kern, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.G);
  cfg.blockDim = dim3(kDsThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SPA_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  return SPA_OK;
}

template <typename T>
int ds_dispatch(const DsArgs& a, int smem, cudaStream_t st) {
  switch (a.Dh) {
    case 32:
      return ds_launch<T, 32>(a, smem, st);
    case 64:
      return ds_launch<T, 64>(a, smem, st);
    default:
      return ds_launch<T, 128>(a, smem, st);
  }
}
}  // namespace spa

extern "C" size_t spa_decoder_step_workspace_size(const spa_decoder_step_params* p) {
  if (spa::ds_check(p) != SPA_OK) return 0;
  const spa::DsLayout l =
      spa::ds_layout(static_cast<int>(dtype_size(p->dtype)), p->batch, p->d_model, p->heads, p->ffn, p->layers,
                     spa::ds_table_pages(p), p->local_window, p->top_m, p->kv.page_size, spa::device_sm_count());
  return l.bytes;
}

extern "C" int spa_decoder_step(const spa_decoder_step_params* p, spa_stream_t stream) {
  const int chk = spa::ds_check(p);
  if (chk != SPA_OK) return chk;
  const int B = p->batch, D = p->d_model, L = p->layers, esize = static_cast<int>(dtype_size(p->dtype));
  auto a16 = [](const void* q) { return q && reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (!a16(p->emb) || !a16(p->pos_emb) || !p->norm_f || !a16(p->head_w) || p->emb_rows < 1 || p->pos_rows < 1 ||
      !p->token || !p->counters || !p->logits || !p->selected || !p->workspace || !p->kv.page_size ||
      (p->kv.page_table && p->kv.table_stride < 1) || (p->promo_pages && (!p->promo_last_hit || p->promo_slots < 1 ||
                                                                         p->promo_ttl < 1)) ||
      (p->token_log && p->log_len < 1) || reinterpret_cast<uintptr_t>(p->workspace) % 256)
    return SPA_ERR_INVALID;
  const int m = p->top_m < p->n_pages ? p->top_m : p->n_pages;
  for (int i = 0; i < L; ++i) {
    const spa_decoder_layer& y = p->layer[i];
    if (!y.norm1 || !a16(y.qkv_w) || !a16(y.out_w) || !y.norm2 || !a16(y.fc1_w) || !a16(y.fc2_w) || !y.k_pool ||
        !y.v_pool || (m > 0 && !y.summaries) || reinterpret_cast<uintptr_t>(y.k_pool) % 16 ||
        reinterpret_cast<uintptr_t>(y.v_pool) % 16)
      return SPA_ERR_INVALID;
  }
  const int G = spa::device_sm_count();
  if (G < 2) return SPA_ERR_UNSUPPORTED;
  const int cap = spa::ds_table_pages(p);
  const spa::DsLayout l =
      spa::ds_layout(esize, B, D, p->heads, p->ffn, L, cap, p->local_window, p->top_m, p->kv.page_size, G);
  if (p->workspace_bytes < l.bytes) return SPA_ERR_WORKSPACE;
  const spa::DsSmem sp =
      spa::ds_smem_plan(esize, B, D, p->ffn, D / p->heads, cap, p->top_m, p->promo_slots, l.nchmax, L, G,
                        p->kv.page_table ? p->kv.table_stride : 0);
  if (sp.total > 227 * 1024) return SPA_ERR_UNSUPPORTED;
  spa::DsArgs a{};
  a.B = B;
  a.D = D;
  a.H = p->heads;
  a.Dh = D / p->heads;
  a.F = p->ffn;
  a.V = p->vocab;
  a.L = L;
  a.P = p->kv.page_size;
  a.W = p->local_window;
  a.top_m = p->top_m;
  a.m = m;
  a.msel = m > 0 ? m : 1;
  a.n = p->n_pages;
  a.n_cap = cap;
  a.slots = p->promo_pages ? p->promo_slots : 0;
  a.ttl = p->promo_ttl;
  a.log_len = p->token_log ? p->log_len : 0;
  a.nchmax = l.nchmax;
  a.G = G;
  a.eps = static_cast<float>(p->eps);
  a.rscale = static_cast<float>(p->router_scale);
  a.ascale = static_cast<float>(p->attn_scale);
  a.emb = p->emb;
  a.pos = p->pos_emb;
  a.norm_f = p->norm_f;
  a.head = p->head_w;
  a.emb_rows = p->emb_rows;
  a.pos_rows = p->pos_rows;
  for (int i = 0; i < L; ++i) {
    const spa_decoder_layer& y = p->layer[i];
    a.layer[i] = spa::DsLayer{y.norm1, y.qkv_w, y.qkv_b, y.out_w, y.out_b, y.norm2, y.fc1_w,
                              y.fc1_b, y.fc2_w, y.fc2_b, y.k_pool, y.v_pool, y.summaries};
  }
  a.addr = make_kv_addr(p->kv);
  a.token = p->token;
  a.counters = p->counters;
  a.logits = p->logits;
  a.log = p->token_log;
  a.selected = p->selected;
  a.ppages = p->promo_pages;
  a.plast = p->promo_last_hit;
  unsigned char* ws = static_cast<unsigned char*>(p->workspace);
  a.seq = reinterpret_cast<uint32_t*>(ws + l.seq_off);
  a.words = reinterpret_cast<uint64_t*>(ws + l.words_off);
  a.cand = reinterpret_cast<uint64_t*>(ws + l.cand_off);
  a.pwords = reinterpret_cast<uint64_t*>(ws + l.parts_off);
  a.ctrs = reinterpret_cast<uint32_t*>(ws + l.ctr_off);
  a.wo = l.wo;
  a.smem_bytes = sp.total;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->dtype == SPA_F32) return spa::ds_dispatch<float>(a, sp.total, st);
  if (p->dtype == SPA_F16) return spa::ds_dispatch<__half>(a, sp.total, st);
  return spa::ds_dispatch<__nv_bfloat16>(a, sp.total, st);
}
