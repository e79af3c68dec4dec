// Model glue of the integrated decoder that would otherwise cost a chain of small library
// launches per use: the decoder's RMSNorm (standing in for the LayerNorm of the reference
// model, train_tiny_transformer.py:178-190) as one kernel instead of nine elementwise and
// reduction ops, optionally fused with the residual add before it or with the token and
// position embedding lookup that starts a step (train_tiny_transformer.py:259,270).
//   out[r, i] = T((x[r, i] * rsqrt(mean_j x[r, j]^2 + eps)) * w[i]), arithmetic in fp32
#pragma once

#include "common.cuh"

namespace spa {
// One CTA of 256 threads per row.  Row r's input is x[x_rows ? x_rows[r] : r], plus
// delta[delta_rows ? delta_rows[r] : r] when delta is given; the sum is rounded to T, as a
// separate elementwise add of two T tensors rounds it.  x_out (when given) receives the
// input row and may be x itself (the second pass then reads the row back from x_out, the
// same thread's own writes); it must not overlap delta.  A row index outside [0, limit)
// raises SPA_DEVERR_BAD_INDEX and gives zero rows.
template <typename T>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* x, const int64_t* __restrict__ x_rows, int64_t x_limit,
                                                       const T* delta, const int32_t* __restrict__ delta_rows,
                                                       int64_t delta_limit, const T* __restrict__ w, T* x_out,
                                                       T* __restrict__ out, int dim, float eps) {
  __shared__ float part[8];
  const int64_t row = blockIdx.x;
  const int64_t xi = x_rows ? x_rows[row] : row;
  const int64_t di = delta_rows ? static_cast<int64_t>(delta_rows[row]) : row;
  T* outr = out + row * dim;
  T* xo = x_out ? x_out + row * dim : nullptr;
  if ((x_rows && (xi < 0 || xi >= x_limit)) || (delta && delta_rows && (di < 0 || di >= delta_limit))) {
    if (threadIdx.x == 0) spa_raise(SPA_DEVERR_BAD_INDEX);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      outr[i] = from_f32<T>(0.f);
      if (xo) xo[i] = from_f32<T>(0.f);
    }
    return;
  }
  const T* xr = x + xi * dim;
  const T* dr = delta ? delta + di * dim : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = to_f32(xr[i]);
    if (dr) {
      const T sum = from_f32<T>(v + to_f32(dr[i]));
      v = to_f32(sum);
      if (xo) xo[i] = sum;
    } else if (xo) {
      xo[i] = xr[i];
    }
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
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = xo ? to_f32(xo[i]) : (dr ? to_f32(from_f32<T>(to_f32(xr[i]) + to_f32(dr[i]))) : to_f32(xr[i]));
    outr[i] = from_f32<T>(v * r * to_f32(w[i]));
  }
}

template <typename T>
void launch_rms_norm(const void* x, const int64_t* x_rows, int64_t x_limit, const void* delta,
                     const int32_t* delta_rows, int64_t delta_limit, const void* w, void* x_out, void* out, int rows,
                     int dim, float eps, cudaStream_t st) {
  rms_norm_kernel<T><<<rows, 256, 0, st>>>(static_cast<const T*>(x), x_rows, x_limit, static_cast<const T*>(delta),
                                           delta_rows, delta_limit, static_cast<const T*>(w), static_cast<T*>(x_out),
                                           static_cast<T*>(out), dim, eps);
}

int rms_norm_impl(const void* x, const int64_t* x_rows, int64_t x_limit, const void* delta, const int32_t* delta_rows,
                  int64_t delta_limit, const void* w, void* x_out, void* out, int rows, int dim, double eps, int dtype,
                  spa_stream_t stream) {
  if (rows < 0 || dim <= 0 || !dtype_ok(dtype)) return SPA_ERR_INVALID;
  if (rows == 0) return SPA_OK;
  if (!x || !w || !out) return SPA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float e = static_cast<float>(eps);
  if (dtype == SPA_F32)
    launch_rms_norm<float>(x, x_rows, x_limit, delta, delta_rows, delta_limit, w, x_out, out, rows, dim, e, st);
  else if (dtype == SPA_F16)
    launch_rms_norm<__half>(x, x_rows, x_limit, delta, delta_rows, delta_limit, w, x_out, out, rows, dim, e, st);
  else
    launch_rms_norm<__nv_bfloat16>(x, x_rows, x_limit, delta, delta_rows, delta_limit, w, x_out, out, rows, dim, e,
                                   st);
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}

// Linear layer for a handful of rows (the decoder's batch at decode time), where a library
// GEMM is launch- and latency-bound: y[m, n] = act(T(x[m, :] . w[n, :] + b[n])), w [N, K]
// row-major as a torch Linear weight.  One warp per output column n: its lanes read the
// weight row with 16-byte loads (all of a 2048-element slice in flight) while the CTA
// stages x in shared memory; fp32 products and sums, one warp reduction, one rounding to
// T (as the GEMM's output is rounded), then the activation: exact GELU,
// 0.5 f (1 + erf(f / sqrt 2)) in fp32, rounded again.  out_f32 stores float(y).
constexpr int kLinearMaxRows = 4;
constexpr int kLinearWarps = 8;
constexpr int kLinearBatch = 8;  // 16-byte weight loads per lane in flight
constexpr int kNormHeld = 4;     // norm prologue: row elements per thread held in registers

template <typename T>
__device__ __forceinline__ float dot16(const uint4& wv, const uint4& xv, float acc) {
  const T* we = reinterpret_cast<const T*>(&wv);
  const T* xe = reinterpret_cast<const T*>(&xv);
#pragma unroll
  for (int j = 0; j < static_cast<int>(16 / sizeof(T)); ++j) acc = fmaf(to_f32(we[j]), to_f32(xe[j]), acc);
  return acc;
}

// Optional prologue: the rows fed to the product are RMSNorm(x (+ delta)) computed by every
// CTA for itself with the arithmetic of rms_norm_kernel (same thread-to-element mapping and
// reduction order, so the normalised rows are bit-identical to a separate norm launch),
// and CTA 0 stores the summed rows to x_out.  ids / delta_ids select table rows as in
// rms_norm_kernel (embedding lookup).
struct LinearPro {
  const void* delta;
  const int64_t* ids;
  int64_t id_limit;
  const int32_t* delta_ids;
  int64_t delta_limit;
  const void* norm_w;
  void* x_out;
  float eps;
};

// Optional epilogue: output columns [k_col, k_col + Hkv*D) and [v_col, v_col + Hkv*D) are
// also the new token's K and V of batch row m, stored into the paged pools at
// positions[m] as spa_kv_append stores them (negative position: not stored; a row outside
// the pools raises SPA_DEVERR_BAD_PAGE).
struct LinearAppend {
  KvAddr addr;
  void* k;
  void* v;
  const int32_t* positions;
  int k_col, v_col, kv_heads, head_dim;
  void* q_out;  // also receives output columns [q_col, q_col + q_width), [rows, q_width]
  int q_col, q_width;
};

template <typename T>
__global__ void __launch_bounds__(kLinearWarps * 32) linear_rows_kernel(const T* __restrict__ x,
                                                                        const T* __restrict__ w,
                                                                        const T* __restrict__ bias,
                                                                        void* __restrict__ out, int rows, int K,
                                                                        int N, int gelu, int out_f32, int vec,
                                                                        int chained, const LinearPro pro,
                                                                        const LinearAppend app) {
  extern __shared__ __align__(16) unsigned char linear_smem[];
  T* xs = reinterpret_cast<T*>(linear_smem);  // [rows][K]
  constexpr int kVec = 16 / sizeof(T);        // elements per 16-byte load
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kLinearWarps + warp;
  const T* wr = w + static_cast<int64_t>(n < N ? n : 0) * K;
  // the first weight batch is requested before x is staged; chained (launched as a
  // programmatic dependent of the kernel before it), before that kernel has completed too
  // -- the weights are not its outputs -- and everything else after it has
  uint4 r[kLinearBatch];
  auto first_weights = [&] {
    if (vec && n < N) {
#pragma unroll
      for (int u = 0; u < kLinearBatch; ++u) {
        const int k = (lane + 32 * u) * kVec;
        if (k < K) r[u] = __ldg(reinterpret_cast<const uint4*>(wr + k));
      }
    }
  };
  pdl_trigger();
  if (chained) first_weights();
  pdl_block();
  if (!chained) first_weights();
  const int total = rows * K;
  if (pro.norm_w) {
    __shared__ float part[kLinearMaxRows][kLinearWarps];
    const T* dl = static_cast<const T*>(pro.delta);
    const T* nw = static_cast<const T*>(pro.norm_w);
    T* xo = blockIdx.x == 0 ? static_cast<T*>(pro.x_out) : nullptr;
    const T* xr[kLinearMaxRows];
    const T* dr[kLinearMaxRows];
    bool bad[kLinearMaxRows];
#pragma unroll
    for (int m = 0; m < kLinearMaxRows; ++m) {
      const int mm = m < rows ? m : 0;
      const int64_t xi = pro.ids ? pro.ids[mm] : mm;
      const int64_t di = pro.delta_ids ? static_cast<int64_t>(pro.delta_ids[mm]) : mm;
      bad[m] = (pro.ids && (xi < 0 || xi >= pro.id_limit)) || (dl && pro.delta_ids && (di < 0 || di >= pro.delta_limit));
      xr[m] = x + (bad[m] ? 0 : xi) * K;
      dr[m] = dl ? dl + (bad[m] ? 0 : di) * K : nullptr;
    }
    auto value = [&](int m, int i) -> float {
      if (bad[m]) return 0.f;
      const float v = to_f32(xr[m][i]);
      return dr[m] ? to_f32(from_f32<T>(v + to_f32(dr[m][i]))) : v;
    };
    if (blockIdx.x == 0 && threadIdx.x == 0)
      for (int m = 0; m < rows; ++m)
        if (bad[m]) spa_raise(SPA_DEVERR_BAD_INDEX);
    if (K <= kNormHeld * kLinearWarps * 32) {
      // every element this thread owns (i = threadIdx.x + u * blockDim.x) and its norm
      // weight requested at once and held in registers: one memory round trip
      float held[kLinearMaxRows][kNormHeld];
      float wn[kNormHeld];
#pragma unroll
      for (int u = 0; u < kNormHeld; ++u) {
        const int i = threadIdx.x + u * blockDim.x;
        wn[u] = i < K ? to_f32(nw[i]) : 0.f;
#pragma unroll
        for (int m = 0; m < kLinearMaxRows; ++m) held[m][u] = m < rows && i < K ? value(m, i) : 0.f;
      }
#pragma unroll
      for (int m = 0; m < kLinearMaxRows; ++m) {
        if (m >= rows) break;
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < kNormHeld; ++u) {
          const int i = threadIdx.x + u * blockDim.x;
          if (i < K) {
            if (xo) xo[m * K + i] = from_f32<T>(held[m][u]);
            ss = fmaf(held[m][u], held[m][u], ss);
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) part[m][warp] = ss;
      }
      __syncthreads();
#pragma unroll
      for (int m = 0; m < kLinearMaxRows; ++m) {
        if (m >= rows) break;
        float tot = 0.f;
#pragma unroll
        for (int k = 0; k < kLinearWarps; ++k) tot += part[m][k];
        const float r = rsqrtf(tot / static_cast<float>(K) + pro.eps);
#pragma unroll
        for (int u = 0; u < kNormHeld; ++u) {
          const int i = threadIdx.x + u * blockDim.x;
          if (i < K) xs[m * K + i] = bad[m] ? from_f32<T>(0.f) : from_f32<T>(held[m][u] * r * wn[u]);
        }
      }
    } else {
#pragma unroll
      for (int m = 0; m < kLinearMaxRows; ++m) {
        if (m >= rows) break;
        float ss = 0.f;
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
          const float v = value(m, i);
          if (xo) xo[m * K + i] = from_f32<T>(v);
          ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) part[m][warp] = ss;
      }
      __syncthreads();
#pragma unroll
      for (int m = 0; m < kLinearMaxRows; ++m) {
        if (m >= rows) break;
        float tot = 0.f;
#pragma unroll
        for (int k = 0; k < kLinearWarps; ++k) tot += part[m][k];
        const float r = rsqrtf(tot / static_cast<float>(K) + pro.eps);
        for (int i = threadIdx.x; i < K; i += blockDim.x)
          xs[m * K + i] = bad[m] ? from_f32<T>(0.f) : from_f32<T>(value(m, i) * r * to_f32(nw[i]));
      }
    }
  } else if (vec) {
    for (int i = threadIdx.x; i < total / kVec; i += blockDim.x)
      reinterpret_cast<uint4*>(xs)[i] = __ldg(reinterpret_cast<const uint4*>(x) + i);
  } else {
    for (int i = threadIdx.x; i < total; i += blockDim.x) xs[i] = x[i];
  }
  __syncthreads();
  if (n >= N) return;
  float acc[kLinearMaxRows];
#pragma unroll
  for (int m = 0; m < kLinearMaxRows; ++m) acc[m] = 0.f;
  if (vec) {
    for (int base = 0; base < K; base += 32 * kVec * kLinearBatch) {
      if (base > 0) {
#pragma unroll
        for (int u = 0; u < kLinearBatch; ++u) {
          const int k = base + (lane + 32 * u) * kVec;
          if (k < K) r[u] = __ldg(reinterpret_cast<const uint4*>(wr + k));
        }
      }
#pragma unroll
      for (int u = 0; u < kLinearBatch; ++u) {
        const int k = base + (lane + 32 * u) * kVec;
        if (k < K) {
#pragma unroll
          for (int m = 0; m < kLinearMaxRows; ++m)
            if (m < rows) acc[m] = dot16<T>(r[u], *reinterpret_cast<const uint4*>(xs + m * K + k), acc[m]);
        }
      }
    }
  } else {
    for (int k = lane; k < K; k += 32) {
      const float wv = to_f32(wr[k]);
#pragma unroll
      for (int m = 0; m < kLinearMaxRows; ++m)
        if (m < rows) acc[m] = fmaf(wv, to_f32(xs[m * K + k]), acc[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < kLinearMaxRows; ++m)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], off);
  if (lane < rows) {
    float v = acc[0];
#pragma unroll
    for (int m = 1; m < kLinearMaxRows; ++m)
      if (lane == m) v = acc[m];
    if (bias) v += to_f32(bias[n]);
    T y = from_f32<T>(v);
    if (gelu) {
      const float f = to_f32(y);
      y = from_f32<T>(f * 0.5f * (1.f + erff(f * 0.70710678118654752f)));
    }
    const int64_t o = static_cast<int64_t>(lane) * N + n;
    if (out_f32)
      static_cast<float*>(out)[o] = to_f32(y);
    else
      static_cast<T*>(out)[o] = y;
    if (app.q_out && n >= app.q_col && n < app.q_col + app.q_width)
      static_cast<T*>(app.q_out)[static_cast<int64_t>(lane) * app.q_width + (n - app.q_col)] = y;
    if (app.k) {
      const int width = app.kv_heads * app.head_dim;
      T* pool = nullptr;
      int rel = 0;
      if (n >= app.k_col && n < app.k_col + width) {
        pool = static_cast<T*>(app.k);
        rel = n - app.k_col;
      } else if (n >= app.v_col && n < app.v_col + width) {
        pool = static_cast<T*>(app.v);
        rel = n - app.v_col;
      }
      const int pos = pool ? app.positions[lane] : -1;
      if (pos >= 0) {
        const int h = rel / app.head_dim, j = rel - h * app.head_dim;
        const int64_t row = app.addr.row(lane, h, pos);
        if (row < 0 || row >= app.addr.total_rows)
          spa_raise(SPA_DEVERR_BAD_PAGE);
        else
          pool[row * app.head_dim + j] = y;
      }
    }
  }
}

template <typename T>
int launch_linear(const void* x, const void* w, const void* bias, void* out, int rows, int K, int N, int gelu,
                  int out_f32, int chained, const LinearPro& pro, const LinearAppend& app, cudaStream_t st) {
  constexpr int kVec = 16 / sizeof(T);
  const size_t smem = static_cast<size_t>(rows) * K * sizeof(T);
  if (smem > 200 * 1024) return SPA_ERR_UNSUPPORTED;
  // the 16-byte path needs aligned weight rows, and aligned x when x is staged as is
  const int vec = K % kVec == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                  (pro.norm_w || reinterpret_cast<uintptr_t>(x) % 16 == 0);
  auto kern = linear_rows_kernel<T>;
  SPA_CHECK_CUDA(spa_set_smem_once(kern, static_cast<int>(smem)));
  SPA_CHECK_CUDA(launch_ex(kern, dim3((N + kLinearWarps - 1) / kLinearWarps), dim3(kLinearWarps * 32), smem, st,
                           chained != 0, 1, static_cast<const T*>(x), static_cast<const T*>(w),
                           static_cast<const T*>(bias), out, rows, K, N, gelu, out_f32, vec, chained, pro, app));
  return SPA_OK;
}
}  // namespace spa

extern "C" int spa_rms_norm(const void* x, const void* weight, void* out, int rows, int dim, double eps, int dtype,
                            spa_stream_t stream) {
  return spa::rms_norm_impl(x, nullptr, 0, nullptr, nullptr, 0, weight, nullptr, out, rows, dim, eps, dtype,
                            stream);
}

extern "C" int spa_add_rms_norm(const void* x, const void* delta, const void* weight, void* x_out, void* out, int rows,
                                int dim, double eps, int dtype, spa_stream_t stream) {
  if (rows > 0 && (!delta || !x_out)) return SPA_ERR_INVALID;
  return spa::rms_norm_impl(x, nullptr, 0, delta, nullptr, 0, weight, x_out, out, rows, dim, eps, dtype, stream);
}

extern "C" int spa_embed_rms_norm(const void* table, int64_t table_rows, const int64_t* ids, const void* pos_table,
                                  int64_t pos_rows, const int32_t* positions, const void* weight, void* x_out,
                                  void* out, int rows, int dim, double eps, int dtype, spa_stream_t stream) {
  if (rows > 0 && (!ids || !pos_table || !positions || !x_out || table_rows <= 0 || pos_rows <= 0))
    return SPA_ERR_INVALID;
  return spa::rms_norm_impl(table, ids, table_rows, pos_table, positions, pos_rows, weight, x_out, out, rows, dim, eps,
                            dtype, stream);
}

namespace spa {
// Greedy token choice at the end of a decode step: the index of the largest logit with
// torch.argmax's rules (NaN counts as the largest value; among equal values the first
// index).  One CTA per row, or with a token log one CTA for every row (it reads each row's
// position before any counter moves).  CTA 0 then adds 1 to each of the step's counters
// (position, context length, step), which every earlier kernel of the step has already read.
// A thread requests kArgmaxBatch logits of a row at once, so a row costs one memory round
// trip per kArgmaxBatch * blockDim.x columns; the comparison is a total order, so the
// visiting order does not change the winner.
constexpr int kArgmaxBatch = 16;
constexpr int kArgmaxLogRows = 256;

__device__ __forceinline__ bool argmax_beats(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ia < ib;
}

__global__ void __launch_bounds__(256) argmax_advance_kernel(const float* __restrict__ logits, int rows, int cols,
                                                             int64_t* __restrict__ token, int32_t* counters,
                                                             int n_counters, const int32_t* positions,
                                                             int64_t* __restrict__ log, int log_len) {
  __shared__ float bv[8];
  __shared__ int bi[8];
  __shared__ int lpos[kArgmaxLogRows];
  // launched as a programmatic dependent of the kernel before it: every read after it completes
  pdl_trigger();
  pdl_block();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (log)
    for (int j = threadIdx.x; j < rows; j += blockDim.x) lpos[j] = positions[j];
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* lr = logits + static_cast<int64_t>(row) * cols;
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int base = 0; base < cols; base += kArgmaxBatch * blockDim.x) {
      float xv[kArgmaxBatch];
#pragma unroll
      for (int u = 0; u < kArgmaxBatch; ++u) {
        const int c = base + threadIdx.x + u * blockDim.x;
        xv[u] = c < cols ? lr[c] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kArgmaxBatch; ++u) {
        const int c = base + threadIdx.x + u * blockDim.x;
        if (c < cols && argmax_beats(xv[u], c, v, i)) {
          v = xv[u];
          i = c;
        }
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
      bv[warp] = v;
      bi[warp] = i;
    }
    __syncthreads();  // also orders every lpos read before the counter updates below
    if (threadIdx.x == 0) {
      for (int w = 1; w < 8; ++w)
        if (argmax_beats(bv[w], bi[w], v, i)) {
          v = bv[w];
          i = bi[w];
        }
      token[row] = i;
      if (log) {
        const int p = lpos[row];
        if (p >= 0 && p < log_len) log[static_cast<int64_t>(p) * rows + row] = i;
      }
    }
    __syncthreads();  // bv / bi are reused by the next row
  }
  if (blockIdx.x == 0)
    for (int c = threadIdx.x; c < n_counters; c += blockDim.x) counters[c] += 1;
}
}  // namespace spa

extern "C" int spa_argmax_advance(const float* logits, int rows, int cols, int64_t* token, int32_t* counters,
                                  int n_counters, spa_stream_t stream) {
  if (rows < 0 || cols <= 0 || n_counters < 0 || (n_counters > 0 && !counters)) return SPA_ERR_INVALID;
  if (rows == 0) return SPA_OK;
  if (!logits || !token) return SPA_ERR_INVALID;
  SPA_CHECK_CUDA(spa::launch_ex(spa::argmax_advance_kernel, dim3(rows), dim3(256), 0,
                                 reinterpret_cast<cudaStream_t>(stream), true, 1, logits, rows, cols, token, counters,
                                 n_counters, static_cast<const int32_t*>(nullptr), static_cast<int64_t*>(nullptr), 0));
  return SPA_OK;
}

extern "C" int spa_argmax_advance_log(const float* logits, int rows, int cols, int64_t* token, int32_t* counters,
                                      int n_counters, const int32_t* positions, int64_t* log, int log_len,
                                      spa_stream_t stream) {
  if (rows < 0 || cols <= 0 || n_counters < 0 || (n_counters > 0 && !counters) || log_len < 0 ||
      rows > spa::kArgmaxLogRows)
    return SPA_ERR_INVALID;
  if (rows == 0) return SPA_OK;
  if (!logits || !token || !positions || (log_len > 0 && !log)) return SPA_ERR_INVALID;
  SPA_CHECK_CUDA(spa::launch_ex(spa::argmax_advance_kernel, dim3(1), dim3(256), 0,
                                 reinterpret_cast<cudaStream_t>(stream), true, 1, logits, rows, cols, token, counters,
                                 n_counters, positions, log_len > 0 ? log : static_cast<int64_t*>(nullptr), log_len));
  return SPA_OK;
}

namespace spa {
int linear_impl(const void* x, const void* weight, const void* bias, void* out, int rows, int in_features,
                int out_features, int activation, int out_f32, int dtype, const LinearPro& pro,
                const LinearAppend& app, spa_stream_t stream, int chained = 0) {
  if (rows < 0 || rows > kLinearMaxRows || in_features <= 0 || out_features <= 0 || !dtype_ok(dtype) ||
      (activation != 0 && activation != 1) || (out_f32 != 0 && out_f32 != 1))
    return SPA_ERR_INVALID;
  if (rows == 0) return SPA_OK;
  if (!x || !weight || !out) return SPA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPA_F32)
    return launch_linear<float>(x, weight, bias, out, rows, in_features, out_features, activation, out_f32, chained, pro,
                                app, st);
  if (dtype == SPA_F16)
    return launch_linear<__half>(x, weight, bias, out, rows, in_features, out_features, activation, out_f32, chained, pro,
                                 app, st);
  return launch_linear<__nv_bfloat16>(x, weight, bias, out, rows, in_features, out_features, activation, out_f32, chained,
                                      pro, app, st);
}
}  // namespace spa

extern "C" int spa_linear(const void* x, const void* weight, const void* bias, void* out, int rows, int in_features,
                          int out_features, int activation, int out_f32, int dtype, spa_stream_t stream) {
  const spa::LinearPro pro{};
  const spa::LinearAppend app{};
  return spa::linear_impl(x, weight, bias, out, rows, in_features, out_features, activation, out_f32, dtype, pro, app,
                          stream);
}

extern "C" int spa_linear_chained(const void* x, const void* weight, const void* bias, void* out, int rows,
                                  int in_features, int out_features, int activation, int out_f32, int dtype,
                                  spa_stream_t stream) {
  const spa::LinearPro pro{};
  const spa::LinearAppend app{};
  return spa::linear_impl(x, weight, bias, out, rows, in_features, out_features, activation, out_f32, dtype, pro, app,
                          stream, 1);
}

namespace spa {
int norm_linear_impl(const void* x, const spa_norm_prologue* norm, const void* weight, const void* bias, void* out,
                     int rows, int in_features, int out_features, int activation, int out_f32, int dtype,
                     const spa_kv_append_epilogue* append, spa_stream_t stream, int chained) {
  if (!norm || !norm->norm_weight) return SPA_ERR_INVALID;
  spa::LinearAppend app{};
  if (append) {
    const spa_kv_layout& kv = append->kv;
    const int64_t width = static_cast<int64_t>(append->kv_heads) * append->head_dim;
    if (!kv.k || !kv.v || !append->positions || kv.page_size <= 0 || append->kv_heads <= 0 ||
        append->head_dim <= 0 || (kv.page_table && kv.table_stride <= 0) || append->k_col < 0 || append->v_col < 0 ||
        append->k_col + width > out_features || append->v_col + width > out_features)
      return SPA_ERR_INVALID;
    app.addr = make_kv_addr(kv);
    app.k = const_cast<void*>(kv.k);
    app.v = const_cast<void*>(kv.v);
    app.positions = append->positions;
    app.k_col = append->k_col;
    app.v_col = append->v_col;
    app.kv_heads = append->kv_heads;
    app.head_dim = append->head_dim;
    if (append->q_out) {
      if (out_f32 || append->q_col < 0 || append->q_width <= 0 ||
          static_cast<int64_t>(append->q_col) + append->q_width > out_features)
        return SPA_ERR_INVALID;
      app.q_out = append->q_out;
      app.q_col = append->q_col;
      app.q_width = append->q_width;
    }
  }
  if (norm->ids && (norm->id_limit <= 0 || !norm->delta || !norm->delta_ids || norm->delta_limit <= 0))
    return SPA_ERR_INVALID;
  spa::LinearPro pro{};
  pro.delta = norm->delta;
  pro.ids = norm->ids;
  pro.id_limit = norm->id_limit;
  pro.delta_ids = norm->delta_ids;
  pro.delta_limit = norm->delta_limit;
  pro.norm_w = norm->norm_weight;
  pro.x_out = norm->x_out;
  pro.eps = static_cast<float>(norm->eps);
  return spa::linear_impl(x, weight, bias, out, rows, in_features, out_features, activation, out_f32, dtype, pro, app,
                          stream, chained);
}
}  // namespace spa

extern "C" int spa_norm_linear(const void* x, const spa_norm_prologue* norm, const void* weight, const void* bias,
                               void* out, int rows, int in_features, int out_features, int activation, int out_f32,
                               int dtype, const spa_kv_append_epilogue* append, spa_stream_t stream) {
  return spa::norm_linear_impl(x, norm, weight, bias, out, rows, in_features, out_features, activation, out_f32, dtype,
                               append, stream, 0);
}

extern "C" int spa_norm_linear_chained(const void* x, const spa_norm_prologue* norm, const void* weight,
                                       const void* bias, void* out, int rows, int in_features, int out_features,
                                       int activation, int out_f32, int dtype, const spa_kv_append_epilogue* append,
                                       spa_stream_t stream) {
  return spa::norm_linear_impl(x, norm, weight, bias, out, rows, in_features, out_features, activation, out_f32, dtype,
                               append, stream, 1);
}
