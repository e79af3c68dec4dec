// Library runtime: device error word, version string, TMA descriptor encoding
// (through the driver entry point, so the library needs no -lcuda) with a small
// host-side cache keyed by (base, shape, box, dtype).
#pragma once

#include <mutex>
#include <unordered_map>

#include "common.cuh"

extern "C" const char* spa_version(void) {
  return "spa_b200 0.2 (sm_100a; tcgen05 prefill, TMA+mma.sync paged decode, fp32 cluster router)";
}

namespace spa {
// One thread waits on an mbarrier that nothing arrives on; the bounded wait gives up
// after `cycles` and raises SPA_DEVERR_WAIT_TIMEOUT.
__global__ void debug_wait_timeout_kernel(long long cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, cycles);
}
}  // namespace spa

extern "C" int spa_debug_wait_timeout(long long cycles, spa_stream_t stream) {
  if (cycles <= 0 || cycles > SPA_WAIT_CYCLES) return SPA_ERR_INVALID;
  spa::debug_wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(cycles);
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}

extern "C" const char* spa_last_error(void) {
  const cudaError_t e = spa_last_cuda_error();
  return e == cudaSuccess ? "" : cudaGetErrorString(e);
}

extern "C" int spa_device_error(uint32_t* out_flags) {
  if (!out_flags) return SPA_ERR_INVALID;
  SPA_CHECK_CUDA(cudaDeviceSynchronize());
  uint32_t v = 0, zero = 0;
  SPA_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_spa_error_flags, sizeof(v)));
  SPA_CHECK_CUDA(cudaMemcpyToSymbol(g_spa_error_flags, &zero, sizeof(zero)));
  *out_flags = v;
  return SPA_OK;
}

namespace spa {
// Byte copy for small transfers between device memory and mapped pinned host memory:
// 16-byte accesses when both ends and the size allow, bytes otherwise.  Launched as a
// programmatic dependent of the previous kernel on the stream, it waits for that kernel
// (griddepcontrol.wait) before the first read, so its launch overlaps that kernel's tail.
// With release_early it also lets its own programmatic dependent launch at once; that
// dependent must wait (griddepcontrol.wait) before it reads anything this copy writes.
__global__ void __launch_bounds__(256) copy_bytes_kernel(unsigned char* __restrict__ dst,
                                                         const unsigned char* __restrict__ src, size_t bytes,
                                                         int vec16, int release_early) {
  if (release_early) pdl_trigger();
  pdl_block();
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t nth = static_cast<size_t>(gridDim.x) * blockDim.x;
  if (vec16) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (size_t i = tid; i < bytes / 16; i += nth) d[i] = s[i];
  } else {
    for (size_t i = tid; i < bytes; i += nth) dst[i] = src[i];
  }
}

// pdl: launched as a programmatic dependent of the kernel before it (it waits for that
// kernel's completion at entry either way); without it the launch itself waits, so the
// copy's CTAs take no SM slots while that kernel runs.
int copy_launch(void* dst, const void* src, size_t bytes, spa_stream_t stream, bool release_early, bool pdl = true) {
  if (!dst || !src) return SPA_ERR_INVALID;
  if (bytes == 0) return SPA_OK;
  const int vec16 = (reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) % 16 == 0;
  const size_t units = vec16 ? bytes / 16 : bytes;
  const size_t blocks = (units + 255) / 256;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks < 64 ? blocks : 64), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SPA_CHECK_CUDA(cudaLaunchKernelEx(&cfg, spa::copy_bytes_kernel, static_cast<unsigned char*>(dst),
                                    static_cast<const unsigned char*>(src), bytes, vec16,
                                    release_early ? 1 : 0));
  return SPA_OK;
}
}  // namespace spa

extern "C" int spa_copy(void* dst, const void* src, size_t bytes, spa_stream_t stream) {
  return spa::copy_launch(dst, src, bytes, stream, false);
}

extern "C" int spa_host_device_pointer(void* host, void** device) {
  if (!host || !device) return SPA_ERR_INVALID;
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, host, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not pinned and mapped: clear the sticky-free error state
    return SPA_ERR_INVALID;
  }
  *device = d;
  return SPA_OK;
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  uintptr_t base;
  uint64_t rows, cols, depth;
  uint32_t box_rows, box_cols;
  int dtype, swz, dev;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && depth == o.depth && box_rows == o.box_rows &&
           box_cols == o.box_cols && dtype == o.dtype && swz == o.swz && dev == o.dev;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = k.base * 1000003u;
    h ^= k.rows + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= k.cols * 31 + k.depth * 65599 + k.box_rows * 131 + k.box_cols * 7 + k.dtype * 3 + k.swz + k.dev * 977;
    return h;
  }
};

}  // namespace

cudaError_t spa_set_smem_limit(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> done;  // (kernel, device) -> bytes set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) << 8) ^ static_cast<uint64_t>(dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}

namespace {
// depth == 0: 2D [rows, cols]; depth > 0: 3D [depth, rows, cols] with box depth 1.
bool make_tensor_map(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols, uint64_t depth,
                     uint32_t box_rows, uint32_t box_cols, bool swizzle128) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, depth, box_rows, box_cols, dtype, swizzle128 ? 1 : 0,
             dev};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  const size_t es = dtype_size(dtype);
  if ((cols * es) % 16 != 0) return false;
  CUtensorMapDataType dt = dtype == SPA_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == SPA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint32_t rank = depth ? 3 : 2;
  cuuint64_t dims[3] = {cols, rows, depth};
  cuuint64_t strides[2] = {cols * es, rows * cols * es};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(out, dt, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return true;
}
}  // namespace

bool spa_make_tensor_map_row_halves(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols,
                                    uint32_t box_rows) {
  // [rows, cols] seen as [cols / w][rows][w] with w = 128 bytes of elements: one box of
  // box_rows rows covers every w-column slab, laid out in shared memory slab by slab
  // (the same bytes, swizzle included, as one 2D box per slab)
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t es = dtype_size(dtype);
  const uint64_t w = 128 / es;
  if (cols % w != 0 || cols / w > 256 || reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, 0, box_rows, static_cast<uint32_t>(w), dtype, 2, dev};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  CUtensorMapDataType dt = dtype == SPA_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == SPA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[3] = {w, rows, cols / w};
  cuuint64_t strides[2] = {cols * es, 128};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(w), box_rows, static_cast<cuuint32_t>(cols / w)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(out, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return true;
}

bool spa_make_tensor_map_3d(CUtensorMap* out, const void* base, int dtype, uint64_t d, uint64_t rows, uint64_t bh) {
  return make_tensor_map(out, base, dtype, rows, d, bh, 128, 64, true);
}
