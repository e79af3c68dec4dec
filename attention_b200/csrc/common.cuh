// Shared device helpers for the sm_100a sparse paged-attention kernels:
// dtype conversion, the library error word, bounded mbarrier waits, TMA
// (cp.async.bulk.tensor) loads, ldmatrix and mma.sync wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spa_b200.h"

// Last CUDA runtime error an entry point returned SPA_ERR_CUDA for, per host thread
// (read by spa_last_error()).
inline cudaError_t& spa_last_cuda_error() {
  static thread_local cudaError_t e = cudaSuccess;
  return e;
}

#define SPA_CHECK_CUDA(expr)                          \
  do {                                                \
    cudaError_t _e = (expr);                          \
    if (_e != cudaSuccess) {                          \
      spa_last_cuda_error() = _e;                     \
      return SPA_ERR_CUDA;                            \
    }                                                 \
  } while (0)

// Bits of the device-side error word (read by spa_device_error()).
enum : uint32_t {
  SPA_DEVERR_WAIT_TIMEOUT = 1u,   // a bounded mbarrier / flag wait gave up
  SPA_DEVERR_BAD_PAGE = 2u,       // a page id outside the table / pool was skipped
  SPA_DEVERR_BAD_INDEX = 4u,      // a token or position id outside its embedding table
};

// ~2 s at 1.9 GHz: far above any legitimate wait, small enough that a lost
// arrival ends the kernel instead of hanging the GPU.
#define SPA_WAIT_CYCLES (4000000000ll)

// Defined once: every kernel source is compiled in one translation unit (spa_b200.cu).
__device__ uint32_t g_spa_error_flags = 0;

__device__ __forceinline__ void spa_raise(uint32_t bit) { atomicOr(&g_spa_error_flags, bit); }

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
__device__ __forceinline__ double to_f64(T x) { return static_cast<double>(to_f32<T>(x)); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete.  Returns false (and
// raises SPA_DEVERR_WAIT_TIMEOUT) if it has not completed after SPA_WAIT_CYCLES.
// Once any wait on the device has given up, every other bounded wait returns at
// once (the error word is polled), so a broken pipeline ends within one bound.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit_cycles = SPA_WAIT_CYCLES) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(&g_spa_error_flags) & SPA_DEVERR_WAIT_TIMEOUT) return false;
      if (clock64() - t0 > limit_cycles) {
        spa_raise(SPA_DEVERR_WAIT_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA
// 3D tiled tensor load into shared memory with an L2 eviction-priority hint (createpolicy
// result); completion is signalled on `bar` as transaction bytes.  x (innermost
// coordinate) times the element size must be a multiple of 16 B.
__device__ __forceinline__ void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                                 int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- mma.sync
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <typename T>
struct MmaOp;
template <>
struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct MmaOp<__half> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Programmatic dependent launch and thread-block-cluster helpers.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Barrier over every running thread of every CTA in the cluster (threads that have
// exited are not counted).
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split cluster barrier: every thread arrives once at kernel start (relaxed) and waits
// before its first store into a peer's shared memory, which guarantees every CTA of the
// cluster is running by then.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void st_dsmem(float* local_ptr, int rank, float v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local_ptr)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
__device__ __forceinline__ void st_dsmem_v4(float* local_ptr, int rank, float4 v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local_ptr)), "r"(rank));
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(ra), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void pdl_block() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// True in exactly one lane of the (converged, full) warp: the lowest one.
__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred;
  asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
  return pred != 0;
}

// max(a, b, c) in one instruction (three-input max, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

// Row index of (sequence b, kv head h, logical token t) under a spa_kv_layout.
struct KvAddr {
  int64_t batch_stride_rows, page_stride_rows, head_stride_rows, total_rows;
  const int32_t* page_table;
  int32_t table_stride, page_size;

  // Physical page of logical page lp, or -1 when lp is outside the table row or the
  // table entry is negative.
  __device__ __forceinline__ int64_t page_of(int b, int lp) const {
    if (lp < 0) return -1;
    if (!page_table) return lp;
    if (lp >= table_stride) return -1;
    const int32_t p = page_table[static_cast<int64_t>(b) * table_stride + lp];
    return p < 0 ? -1 : static_cast<int64_t>(p);
  }
  // Row of token t (t >= 0), or -1 when its page is invalid (callers also bound
  // the row by total_rows).
  __device__ __forceinline__ int64_t row(int b, int h, int t) const {
    const int lp = t / page_size;
    const int64_t pg = page_of(b, lp);
    if (pg < 0) return -1;
    return b * batch_stride_rows + pg * page_stride_rows + h * head_stride_rows + (t - lp * page_size);
  }
};

inline KvAddr make_kv_addr(const spa_kv_layout& kv) {
  KvAddr a;
  a.batch_stride_rows = kv.batch_stride_rows;
  a.page_stride_rows = kv.page_stride_rows;
  a.head_stride_rows = kv.head_stride_rows;
  a.total_rows = kv.total_rows;
  a.page_table = kv.page_table;
  a.table_stride = kv.table_stride;
  a.page_size = kv.page_size;
  return a;
}

inline size_t dtype_size(int dtype) { return dtype == SPA_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == SPA_F32 || dtype == SPA_F16 || dtype == SPA_BF16; }

// Host: sets a kernel's dynamic shared memory limit once per (kernel, device).
cudaError_t spa_set_smem_limit(const void* kernel, int bytes);
template <typename K>
inline cudaError_t spa_set_smem_once(K kernel, int bytes) {
  return spa_set_smem_limit(reinterpret_cast<const void*>(kernel), bytes);
}

// Host: a [rows, cols] row-major buffer seen as [cols / w][rows][w], w = 128 bytes of
// elements, with box [all slabs, box_rows, w] and 128-byte swizzle: one load brings box_rows
// full rows, slab after slab, exactly as one 2D [box_rows, w] box per slab would.
bool spa_make_tensor_map_row_halves(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols,
                                    uint32_t box_rows);
// Host: 3D view [bh, rows, d] of a contiguous [B, H, rows, D] tensor, box [1, 128, 64], 128-byte swizzle.
bool spa_make_tensor_map_3d(CUtensorMap* out, const void* base, int dtype, uint64_t d, uint64_t rows, uint64_t bh);
