// hokv_math.cuh -- fp32 arithmetic in the exact orders NumPy uses on the
// reference path, shared by the device kernels and a host build (g++) that the
// CPU test-suite checks against the golden fixtures.
//
// Orders (NumPy 2.3 + OpenBLAS 0.3.30, x86-64 AVX-512 kernels):
//  * np.sum / np.mean of a contiguous float32 array: numpy's pairwise sum
//    (8 accumulators over blocks of <= 128, halving split above that);
//    mean = f32(f64(sum) / n).
//  * np.sum(x**2, axis=1) of a row: the same pairwise sum over the row.
//  * (1 x d) @ (d x k), the GEMV shape: d == 4 -> (p0+p1)+(p2+p3); d == 8 ->
//    pairwise tree of the 8 products; d % 8 == 0, d >= 16 -> 8 lane
//    accumulators (first product, then FMA per 8-chunk), lanes folded
//    i <- i + i+4, then (a0+a1)+(a2+a3).
//  * (N x d) @ (d x k) with N >= 5: one FMA chain per output, ascending d.
//  * N in [2, 4], d >= 32 (d % 16 == 0): 16 FMA lanes, pairwise tree fold.
//  * column mean over rows (np.mean(X, axis=0)): sequential row adds.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define HD __host__ __device__ __forceinline__
#define HDF __host__ __device__
#else
#include <cmath>
#define HD inline
#define HDF inline
#endif

namespace hokv {

// Round-to-nearest fp32 primitives that the compiler may not contract.
#if defined(__CUDA_ARCH__)
HD float fadd(float a, float b) { return __fadd_rn(a, b); }
HD float fsub(float a, float b) { return __fsub_rn(a, b); }
HD float fmul(float a, float b) { return __fmul_rn(a, b); }
HD float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
HD double dadd(double a, double b) { return __dadd_rn(a, b); }
HD double dsub(double a, double b) { return __dsub_rn(a, b); }
HD double dmul(double a, double b) { return __dmul_rn(a, b); }
#else
HD float fadd(float a, float b) { volatile float r = a + b; return r; }
HD float fsub(float a, float b) { volatile float r = a - b; return r; }
HD float fmul(float a, float b) { volatile float r = a * b; return r; }
HD float ffma(float a, float b, float c) { return std::fmaf(a, b, c); }
HD double dadd(double a, double b) { volatile double r = a + b; return r; }
HD double dsub(double a, double b) { volatile double r = a - b; return r; }
HD double dmul(double a, double b) { volatile double r = a * b; return r; }
#endif

enum DotOrder { DOT_SEQ_FMA = 0, DOT_GEMV = 1, DOT_L16_PAIR = 2 };

// numpy pairwise sum of g(i), i in [0, n), for n <= 128 (one block).
template <typename Gen>
HD float pw_block_idx(int64_t base, int n, Gen g) {
  if (n < 8) {
    float r = 0.f;
    for (int i = 0; i < n; ++i) r = fadd(r, g(base + i));
    return r;
  }
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = g(base + j);
  int i = 8;
  for (; i < n - (n % 8); i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = fadd(r[j], g(base + i + j));
  }
  float res = fadd(fadd(fadd(r[0], r[1]), fadd(r[2], r[3])),
                   fadd(fadd(r[4], r[5]), fadd(r[6], r[7])));
  for (; i < n; ++i) res = fadd(res, g(base + i));
  return res;
}

// numpy pairwise sum of g(i) for any n: halves split at a multiple of 8 down
// to blocks of <= 128.  Evaluated as an explicit post-order walk (no device
// recursion, so kernels keep a statically known stack size).
template <typename Gen>
HD float pw_sum_idx(int64_t n, Gen g) {
  if (n <= 128) return pw_block_idx(0, (int)n, g);
  int64_t fs[32], fm[32];
  float fl[32];
  int st[32];
  int sp = 1;
  fs[0] = 0; fm[0] = n; st[0] = 0;
  float ret = 0.f;
  while (sp > 0) {
    const int t = sp - 1;
    const int64_t s = fs[t], m = fm[t];
    if (st[t] == 0) {
      if (m <= 128) { ret = pw_block_idx(s, (int)m, g); --sp; continue; }
      int64_t h = m / 2;
      h -= h % 8;
      st[t] = 1;
      fs[sp] = s; fm[sp] = h; st[sp] = 0; ++sp;
    } else if (st[t] == 1) {
      fl[t] = ret;
      int64_t h = m / 2;
      h -= h % 8;
      st[t] = 2;
      fs[sp] = s + h; fm[sp] = m - h; st[sp] = 0; ++sp;
    } else {
      ret = fadd(fl[t], ret);
      --sp;
    }
  }
  return ret;
}

struct Ident { HD float operator()(float v) const { return v; } };
struct Square { HD float operator()(float v) const { return fmul(v, v); } };

template <typename F>
struct PtrGen {
  const float* x;
  F f;
  HD float operator()(int64_t i) const { return f(x[i]); }
};

// numpy pairwise sum of f(x[i]).
template <typename F>
HD float pw_sum(const float* x, int64_t n, F f) { return pw_sum_idx(n, PtrGen<F>{x, f}); }

HD float sum_sq(const float* x, int n) { return pw_sum(x, n, Square()); }

// Dot products in the BLAS orders (a, b contiguous, length d).
HD float dot_seqfma(const float* a, const float* b, int d) {
  float acc = 0.f;
  for (int i = 0; i < d; ++i) acc = ffma(a[i], b[i], acc);
  return acc;
}

HD float dot_gemv(const float* a, const float* b, int d) {
  if (d == 4) {
    return fadd(fadd(fmul(a[0], b[0]), fmul(a[1], b[1])),
                fadd(fmul(a[2], b[2]), fmul(a[3], b[3])));
  }
  if (d == 8) {
    float p[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = fmul(a[i], b[i]);
    return fadd(fadd(fadd(p[0], p[1]), fadd(p[2], p[3])), fadd(fadd(p[4], p[5]), fadd(p[6], p[7])));
  }
  if (d >= 16 && (d % 8) == 0) {
    float r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = fmul(a[i], b[i]);
    for (int c = 8; c < d; c += 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = ffma(a[c + i], b[c + i], r[i]);
    }
    float h0 = fadd(r[0], r[4]), h1 = fadd(r[1], r[5]), h2 = fadd(r[2], r[6]), h3 = fadd(r[3], r[7]);
    return fadd(fadd(h0, h1), fadd(h2, h3));
  }
  return dot_seqfma(a, b, d);
}

HD float dot_l16pair(const float* a, const float* b, int d) {
  if (d < 32 || (d % 16) != 0) return dot_seqfma(a, b, d);
  float r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = fmul(a[i], b[i]);
  for (int c = 16; c < d; c += 16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = ffma(a[c + i], b[c + i], r[i]);
  }
#pragma unroll
  for (int w = 16; w > 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w / 2; ++i) r[i] = fadd(r[2 * i], r[2 * i + 1]);
  }
  return r[0];
}

HD float dot_order(int order, const float* a, const float* b, int d) {
  if (order == DOT_GEMV) return dot_gemv(a, b, d);
  if (order == DOT_L16_PAIR) return dot_l16pair(a, b, d);
  return dot_seqfma(a, b, d);
}

// The order NumPy's matmul takes for an (n_rows x d) @ (d x k) product.
HD int dot_order_for(int64_t n_rows, int d) {
  if (n_rows == 1) return DOT_GEMV;
  if (n_rows <= 4 && d >= 32) return DOT_L16_PAIR;
  return DOT_SEQ_FMA;
}

// ((|x|^2 - 2 x.c) + |c|^2), the reference's L2 expansion.
HD float l2_expansion(float x2, float dot, float c2) {
  return fadd(fsub(x2, fmul(2.f, dot)), c2);
}

// Order-preserving map of an fp32 value to uint32 (larger float -> larger key).
HD uint32_t ord_f32(float f) {
#if defined(__CUDA_ARCH__)
  uint32_t u = __float_as_uint(f);
#else
  union { float f; uint32_t u; } c; c.f = f; uint32_t u = c.u;
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
HD float unord_f32(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  union { float f; uint32_t u; } c; c.u = u; return c.f;
#endif
}
// Selection key: higher score first, then lower token index.
HD uint64_t sel_key(float score, uint32_t idx) {
  return ((uint64_t)ord_f32(score) << 32) | (uint64_t)(0xffffffffu - idx);
}
HD uint32_t key_idx(uint64_t key) { return 0xffffffffu - (uint32_t)(key & 0xffffffffu); }
HD float key_score(uint64_t key) { return unord_f32((uint32_t)(key >> 32)); }

// np.percentile(sorted, linspace(0, 100, k))[i] (method 'linear'), cast f32.
HD float percentile_linear(const float* sorted, int64_t n, int k, int i) {
  double q = (k > 1) ? ((double)i * (100.0 / (double)(k - 1))) : 0.0;
  if (k > 1 && i == k - 1) q = 100.0;
  q = q / 100.0;
  double vi = (double)(n - 1) * q;
  int64_t lo, hi;
  double g;
#if defined(__CUDA_ARCH__)
  double fl = floor(vi);
#else
  double fl = std::floor(vi);
#endif
  if (vi >= (double)(n - 1)) { lo = hi = n - 1; g = vi - fl; }
  else { lo = (int64_t)fl; hi = lo + 1; g = vi - fl; }
  float a = sorted[lo], b = sorted[hi];
  float d = fsub(b, a);
  double r = (g >= 0.5) ? dsub((double)b, dmul((double)d, dsub(1.0, g)))
                         : dadd((double)a, dmul((double)d, g));
  return (float)r;
}

// np.linspace(0, n - 1, k).astype(int)[i]
HD int64_t linspace_pick(int64_t n, int k, int i) {
  if (k <= 1) return 0;
  if (i == k - 1) return n - 1;
  double step = (double)(n - 1) / (double)(k - 1);
  double y = (double)i * step;
  return (int64_t)y;
}

}  // namespace hokv
