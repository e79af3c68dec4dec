// Causal sliding-window prefill, CUDA-core path: any dtype, head_dim <= 256.
// One warp per query row, fp32 online softmax with accurate expf.  Serves the
// shapes the tensor-core kernel does not (fp32, head_dim outside {64, 128}).
//
// Reference: local_causal_prefill_kernel (triton_local_prefill.py:17-58): query i
// attends keys [i-W+1, i]; keys before position 0 carry no mass (:48-53).
#pragma once

#include "common.cuh"

namespace spa {

struct PrefillArgs {
  const void *q, *k, *v, *k_halo, *v_halo;
  void* out;
  int B, H, S, D, W, halo;
  int row0, row1;  // query rows computed: [row0, row1)
  float scale;
};

// grid (ceil(S/4), H, B), block 128
template <typename T>
__global__ void __launch_bounds__(128) prefill_generic_kernel(const PrefillArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = a.row0 + blockIdx.x * 4 + warp, h = blockIdx.y, b = blockIdx.z;
  if (i >= a.row1) return;
  const int D = a.D;
  const int64_t bh = static_cast<int64_t>(b) * a.H + h;
  const T* qp = static_cast<const T*>(a.q) + (bh * a.S + i) * D;
  float qv[8], acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int d = lane + 32 * e;
    qv[e] = d < D ? to_f32(qp[d]) : 0.f;
    acc[e] = 0.f;
  }
  // positions in the concatenation [halo ; keys]
  const int ci = i + a.halo;
  const int c0 = max(0, ci - a.W + 1);
  float m = -INFINITY, l = 0.f;
  for (int c = c0; c <= ci; ++c) {
    const T *kr, *vr;
    if (c < a.halo) {
      kr = static_cast<const T*>(a.k_halo) + (bh * a.halo + c) * D;
      vr = static_cast<const T*>(a.v_halo) + (bh * a.halo + c) * D;
    } else {
      kr = static_cast<const T*>(a.k) + (bh * a.S + (c - a.halo)) * D;
      vr = static_cast<const T*>(a.v) + (bh * a.S + (c - a.halo)) * D;
    }
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
    const float alpha = expf(m - mn);
    const float p = expf(sc - mn);
    l = l * alpha + p;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int d = lane + 32 * e;
      acc[e] = acc[e] * alpha + (d < D ? p * to_f32(vr[d]) : 0.f);
    }
    m = mn;
  }
  T* op = static_cast<T*>(a.out) + (bh * a.S + i) * D;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int d = lane + 32 * e;
    if (d < D) op[d] = from_f32<T>(acc[e] / l);
  }
}

template <typename T>
int launch_prefill_generic(const PrefillArgs& a, cudaStream_t st) {
  prefill_generic_kernel<T><<<dim3((a.row1 - a.row0 + 3) / 4, a.H, a.B), 128, 0, st>>>(a);
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}

}  // namespace spa
