// Model glue of the integrated decoder that would otherwise cost a chain of small library
// launches per use: the decoder's RMSNorm (standing in for the LayerNorm of the reference
// model, train_tiny_transformer.py:178-190) as one kernel instead of nine elementwise and
// reduction ops.
//   out[r, i] = T((x[r, i] * rsqrt(mean_j x[r, j]^2 + eps)) * w[i]), arithmetic in fp32
#pragma once

#include "common.cuh"

namespace spa {
// one CTA of 256 threads per row
template <typename T>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                       T* __restrict__ out, int dim, float eps) {
  __shared__ float part[8];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = to_f32(xr[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += part[k];
  const float r = rsqrtf(tot / static_cast<float>(dim) + eps);
  T* outr = out + row * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) outr[i] = from_f32<T>(to_f32(xr[i]) * r * to_f32(w[i]));
}
}  // namespace spa

extern "C" int spa_rms_norm(const void* x, const void* weight, void* out, int rows, int dim, double eps, int dtype,
                            spa_stream_t stream) {
  if (rows < 0 || dim <= 0 || !dtype_ok(dtype)) return SPA_ERR_INVALID;
  if (rows == 0) return SPA_OK;
  if (!x || !weight || !out) return SPA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float e = static_cast<float>(eps);
  if (dtype == SPA_F32)
    spa::rms_norm_kernel<float><<<rows, 256, 0, st>>>(static_cast<const float*>(x), static_cast<const float*>(weight),
                                                      static_cast<float*>(out), dim, e);
  else if (dtype == SPA_F16)
    spa::rms_norm_kernel<__half><<<rows, 256, 0, st>>>(static_cast<const __half*>(x),
                                                       static_cast<const __half*>(weight), static_cast<__half*>(out),
                                                       dim, e);
  else
    spa::rms_norm_kernel<__nv_bfloat16><<<rows, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                              static_cast<const __nv_bfloat16*>(weight),
                                                              static_cast<__nv_bfloat16*>(out), dim, e);
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}
