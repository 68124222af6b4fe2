// dense.cuh -- single-query dense attention pieces behind the NumPy-facing API
// (standard_attention, Path A/B/D/F softmax and value sums, Path F masks).
// Reference: helix_online_kv/compressed_attention.py:38-55, 60-80, 136-160,
// 230-254, 259-310.  Scores and weights follow NumPy's dtype rules: a Python
// float scale keeps float32, a NumPy float64 scale promotes to float64.
#pragma once
#include "hokv_common.cuh"

namespace hokv {

// scores[t] = (q . K[t]) * scale for masked-in tokens, -1e9 otherwise.
// The dot is fp32 (one FMA chain); the scale multiply is fp32 or fp64
// (mul_f64) and the result is stored as f32 or f64 (store_f64).
__global__ void k_dense_scores(const float* __restrict__ q, const float* __restrict__ K, int D, int64_t S,
                               double scale, int mul_f64, int store_f64, const uint8_t* __restrict__ mask,
                               void* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (t >= S) return;
  float acc = 0.f;
  for (int d = lane; d < D; d += 32) acc = fmaf(q[d], K[t * D + d], acc);
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane != 0) return;
  const bool in = mask == nullptr || mask[t] != 0;
  if (store_f64) {
    reinterpret_cast<double*>(scores)[t] = in ? (double)acc * scale : -1e9;
  } else {
    float v;
    if (!in) v = -1e9f;
    else if (mul_f64) v = (float)((double)acc * scale);
    else v = fmul(acc, (float)scale);
    reinterpret_cast<float*>(scores)[t] = v;
  }
}

// Softmax over n values (f32 or f64 storage), computed in f64, one CTA.
__global__ void __launch_bounds__(1024) k_softmax(const void* __restrict__ in, int f64, int64_t n,
                                                  void* __restrict__ out) {
  __shared__ double red[32];
  __shared__ double s_max, s_sum;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto get = [&](int64_t i) -> double {
    return f64 ? reinterpret_cast<const double*>(in)[i] : (double)reinterpret_cast<const float*>(in)[i];
  };
  double m = -INFINITY;
  for (int64_t i = tid; i < n; i += blockDim.x) m = fmax(m, get(i));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0) { double M = red[0]; for (int w = 1; w < (int)(blockDim.x / 32); ++w) M = fmax(M, red[w]); s_max = M; }
  __syncthreads();
  double s = 0.0;
  for (int64_t i = tid; i < n; i += blockDim.x) s += exp(get(i) - s_max);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (tid == 0) { double T = 0; for (int w = 0; w < (int)(blockDim.x / 32); ++w) T += red[w]; s_sum = T; }
  __syncthreads();
  for (int64_t i = tid; i < n; i += blockDim.x) {
    const double w = exp(get(i) - s_max) / s_sum;
    if (f64) reinterpret_cast<double*>(out)[i] = w;
    else reinterpret_cast<float*>(out)[i] = (float)w;
  }
}

// out[d] = sum_t w[t] * V[t][d] (f64 accumulation), stored f32 or f64.
__global__ void k_weighted_sum(const void* __restrict__ w, int w_f64, const float* __restrict__ V, int D, int64_t S,
                               void* __restrict__ out, int out_f64) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  double acc = 0.0;
  for (int64_t t = 0; t < S; ++t) {
    const double wt = w_f64 ? reinterpret_cast<const double*>(w)[t] : (double)reinterpret_cast<const float*>(w)[t];
    acc += wt * (double)V[t * D + d];
  }
  if (out_f64) reinterpret_cast<double*>(out)[d] = acc;
  else reinterpret_cast<float*>(out)[d] = (float)acc;
}

// Path F: keep the top_p clusters by coarse score (ties: the higher index wins,
// as in the tail of a stable ascending sort), then mask tokens whose code is kept.
__global__ void __launch_bounds__(256) k_prefilter_mask(const float* __restrict__ coarse, int k,
                                                        const uint8_t* __restrict__ codes, int64_t S, int top_p,
                                                        uint8_t* __restrict__ mask) {
  __shared__ uint8_t keep[256];
  for (int j = threadIdx.x; j < 256; j += blockDim.x) {
    uint8_t kj = 0;
    if (j < k) {
      const float sj = coarse[j];
      int rank = 0;
      for (int i = 0; i < k; ++i) {
        const float si = coarse[i];
        rank += (si > sj) || (si == sj && i > j);
      }
      kj = rank < top_p;
    }
    keep[j] = kj;
  }
  __syncthreads();
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < S; t += (int64_t)gridDim.x * blockDim.x)
    mask[t] = keep[codes[t]];
}

__global__ void k_scale_f32_to_f64(const float* __restrict__ in, int64_t n, double scale, double* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (double)in[i] * scale;
}

}  // namespace hokv
