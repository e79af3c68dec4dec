// Promotion refresh gate: whether this decode step re-routes or reuses the promoted
// selection, decided on the device for the whole batch (one decision per step, as in the
// reference's strategies).  Reference policies (evaluate_promotion_ttl.py:125-139 and the
// learned head of train_refresh_head.py:24-31, decision at its evaluate()):
//   TTL        refresh when step % ttl == 0
//   SIGNATURE  refresh when the query signature (token ids) differs from the one at the
//              last refresh
//   DRIFT      refresh when the batch mean of 1 - cos(state, state at last refresh)
//              exceeds the threshold
//   LEARNED    refresh when the batch mean of sigmoid(head(state, cached)) reaches the
//              threshold; head = Linear(4W, H) -> GELU -> Linear(H, 1) over
//              [state, cached, |state - cached|, state * cached]
// A step with nothing promoted yet always refreshes.  On refresh the cached state and
// signature become the current ones.
#pragma once

#include "common.cuh"

namespace spa {

// 32 warps: at batch 4 and width 4096 each warp reduces 512 values with all of its loads
// in flight at once
constexpr int kGateThreads = 1024;

__device__ __forceinline__ float gate_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// single CTA; dynamic shared memory: [batch] row values, then [batch * hidden] (learned)
__global__ void __launch_bounds__(kGateThreads) refresh_gate_kernel(const spa_refresh_gate_args a) {
  extern __shared__ float gsm[];
  float* row_val = gsm;             // [batch]
  float* unit_val = gsm + a.batch;  // [batch * hidden] (learned) or [batch * warps per row * 3] (drift)
  // a gated router launched after this kernel may start now; it waits for this grid to
  // complete before it reads the decision
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ int mismatch;
  __shared__ int decision;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = kGateThreads / 32;
  if (threadIdx.x == 0) mismatch = 0;
  __syncthreads();
  const int W = a.width;
  if (a.mode == SPA_GATE_SIGNATURE) {
    const int64_t n = static_cast<int64_t>(a.batch) * a.sig_len;
    int diff = 0;
    for (int64_t i = threadIdx.x; i < n; i += kGateThreads) diff |= a.signature[i] != a.cached_signature[i];
    if (__syncthreads_or(diff) && threadIdx.x == 0) mismatch = 1;
  } else if (a.mode == SPA_GATE_DRIFT) {
    // torch cosine_similarity: (x / max(|x|, eps)) . (y / max(|y|, eps)), eps = 1e-8.
    // Each row is cut into `wpr` contiguous segments, one warp each; the segment partials
    // are added in segment order (deterministic).
    const int wpr = a.batch >= nw ? 1 : nw / a.batch;
    const int seg = (W + wpr - 1) / wpr;
    const bool vec = (W % 4 == 0) && (seg % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.state) |
                                                          reinterpret_cast<uintptr_t>(a.cached_state)) % 16 == 0);
    for (int t = warp; t < a.batch * wpr; t += nw) {
      const int b = t / wpr, sidx = t - b * wpr;
      const int k0 = sidx * seg, k1 = min(W, k0 + seg);
      const float* x = a.state + static_cast<int64_t>(b) * W;
      const float* y = a.cached_state + static_cast<int64_t>(b) * W;
      float xy = 0.f, xx = 0.f, yy = 0.f;
      if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(x + k0);
        const float4* y4 = reinterpret_cast<const float4*>(y + k0);
        const int n4 = (k1 - k0) / 4;
#pragma unroll 4
        for (int i = lane; i < n4; i += 32) {
          const float4 u = x4[i], v = y4[i];
          xy = fmaf(u.x, v.x, fmaf(u.y, v.y, fmaf(u.z, v.z, fmaf(u.w, v.w, xy))));
          xx = fmaf(u.x, u.x, fmaf(u.y, u.y, fmaf(u.z, u.z, fmaf(u.w, u.w, xx))));
          yy = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, yy))));
        }
      } else {
        for (int k = k0 + lane; k < k1; k += 32) {
          const float u = x[k], v = y[k];
          xy = fmaf(u, v, xy);
          xx = fmaf(u, u, xx);
          yy = fmaf(v, v, yy);
        }
      }
      xy = gate_warp_sum(xy);
      xx = gate_warp_sum(xx);
      yy = gate_warp_sum(yy);
      if (lane == 0) {
        unit_val[3 * t] = xy;
        unit_val[3 * t + 1] = xx;
        unit_val[3 * t + 2] = yy;
      }
    }
    __syncthreads();
    for (int b = threadIdx.x; b < a.batch; b += kGateThreads) {
      float xy = 0.f, xx = 0.f, yy = 0.f;
      for (int sidx = 0; sidx < wpr; ++sidx) {
        xy += unit_val[3 * (b * wpr + sidx)];
        xx += unit_val[3 * (b * wpr + sidx) + 1];
        yy += unit_val[3 * (b * wpr + sidx) + 2];
      }
      row_val[b] = 1.f - xy / (fmaxf(sqrtf(xx), 1e-8f) * fmaxf(sqrtf(yy), 1e-8f));
    }
  } else if (a.mode == SPA_GATE_LEARNED) {
    // one warp per (row, hidden unit): GELU(w1[u] . features(row) + b1[u]) * w2[u]
    const int tasks = a.batch * a.hidden;
    for (int t = warp; t < tasks; t += nw) {
      const int b = t / a.hidden, u = t - b * a.hidden;
      const float* x = a.state + static_cast<int64_t>(b) * W;
      const float* y = a.cached_state + static_cast<int64_t>(b) * W;
      const float* w = a.w1 + static_cast<int64_t>(u) * 4 * W;
      float acc = 0.f;
      for (int k = lane; k < W; k += 32) {
        const float c = x[k], p = y[k];
        acc = fmaf(w[k], c, acc);
        acc = fmaf(w[W + k], p, acc);
        acc = fmaf(w[2 * W + k], fabsf(c - p), acc);
        acc = fmaf(w[3 * W + k], c * p, acc);
      }
      acc = gate_warp_sum(acc);
      if (lane == 0) {
        const float h = acc + a.b1[u];
        unit_val[t] = 0.5f * h * (1.f + erff(h * 0.7071067811865476f)) * a.w2[u];
      }
    }
    __syncthreads();
    for (int b = threadIdx.x; b < a.batch; b += kGateThreads) {
      float logit = a.b2[0];
      for (int u = 0; u < a.hidden; ++u) logit += unit_val[b * a.hidden + u];
      row_val[b] = 1.f / (1.f + expf(-logit));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int refresh = a.gate[1] == 0;  // nothing promoted yet
    float mean = 0.f;
    if (a.mode == SPA_GATE_TTL) {
      const int step = a.step_dev ? *a.step_dev : a.step;
      refresh |= step % a.ttl == 0;
    } else if (a.mode == SPA_GATE_SIGNATURE) {
      refresh |= mismatch;
    } else {
      float sum = 0.f;
      for (int b = 0; b < a.batch; ++b) sum += row_val[b];  // row order: deterministic
      mean = sum / static_cast<float>(a.batch);
      refresh |= a.mode == SPA_GATE_DRIFT ? (mean > a.threshold) : (mean >= a.threshold);
    }
    if (a.score_out) *a.score_out = mean;
    a.gate[0] = refresh;
    decision = refresh;
  }
  __syncthreads();
  if (!decision) return;
  // refresh: the current state and signature become the cached ones.  The router waits for
  // this grid to complete, so the copy issues four independent loads per thread before
  // its stores: one memory round trip per 4 x kGateThreads vectors, not one per element.
  if (a.cached_state && a.state) {
    const int64_t n = static_cast<int64_t>(a.batch) * W;
    const bool vec4 = n % 4 == 0 && ((reinterpret_cast<uintptr_t>(a.state) |
                                      reinterpret_cast<uintptr_t>(a.cached_state)) % 16 == 0);
    if (vec4) {
      const float4* src = reinterpret_cast<const float4*>(a.state);
      float4* dst = reinterpret_cast<float4*>(a.cached_state);
      const int64_t n4 = n / 4;
      for (int64_t i0 = threadIdx.x; i0 < n4; i0 += 4 * kGateThreads) {
        float4 r[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * kGateThreads < n4) r[u] = src[i0 + u * kGateThreads];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * kGateThreads < n4) dst[i0 + u * kGateThreads] = r[u];
      }
    } else {
      for (int64_t i0 = threadIdx.x; i0 < n; i0 += 4 * kGateThreads) {
        float r[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * kGateThreads < n) r[u] = a.state[i0 + u * kGateThreads];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * kGateThreads < n) a.cached_state[i0 + u * kGateThreads] = r[u];
      }
    }
  }
  if (a.cached_signature && a.signature) {
    const int64_t n = static_cast<int64_t>(a.batch) * a.sig_len;
    for (int64_t i = threadIdx.x; i < n; i += kGateThreads) a.cached_signature[i] = a.signature[i];
  }
}

}  // namespace spa

extern "C" int spa_refresh_gate(const spa_refresh_gate_args* args, spa_stream_t stream) {
  if (!args || !args->gate || args->batch <= 0) return SPA_ERR_INVALID;
  const spa_refresh_gate_args& a = *args;
  size_t smem = sizeof(float) * static_cast<size_t>(a.batch);
  switch (a.mode) {
    case SPA_GATE_TTL:
      if (a.ttl <= 0 || (!a.step_dev && a.step < 0)) return SPA_ERR_INVALID;
      break;
    case SPA_GATE_SIGNATURE:
      if (!a.signature || !a.cached_signature || a.sig_len <= 0) return SPA_ERR_INVALID;
      break;
    case SPA_GATE_DRIFT: {
      if (!a.state || !a.cached_state || a.width <= 0) return SPA_ERR_INVALID;
      const int nw = spa::kGateThreads / 32;
      const int wpr = a.batch >= nw ? 1 : nw / a.batch;
      smem += sizeof(float) * 3 * static_cast<size_t>(a.batch) * wpr;
      break;
    }
    case SPA_GATE_LEARNED:
      if (!a.state || !a.cached_state || a.width <= 0 || !a.w1 || !a.b1 || !a.w2 || !a.b2 || a.hidden <= 0)
        return SPA_ERR_INVALID;
      smem += sizeof(float) * static_cast<size_t>(a.batch) * a.hidden;
      break;
    default:
      return SPA_ERR_INVALID;
  }
  if (smem > 200 * 1024) return SPA_ERR_UNSUPPORTED;
  SPA_CHECK_CUDA(spa_set_smem_once(spa::refresh_gate_kernel, static_cast<int>(smem)));
  spa::refresh_gate_kernel<<<1, spa::kGateThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}
