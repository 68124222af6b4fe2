// Host build of the library's fp32 arithmetic (hokv_math.cuh) so the CPU test
// suite can check the exact-order design against the reference fixtures.
#include <stdint.h>
#include "hokv_math.cuh"

extern "C" {

void host_pq_tables(const float* q, int M, int sd, const float* cents, int slots, const int* k, float* T, int t_cols,
                    int order) {
  for (int s = 0; s < M; ++s)
    for (int j = 0; j < t_cols; ++j)
      T[s * t_cols + j] = j < k[s] ? hokv::dot_order(order, q + s * sd, cents + ((int64_t)s * slots + j) * sd, sd) : 0.f;
}

// argmin_j ((|x|^2 - 2 x.c_j) + |c_j|^2), first minimum.
void host_l2_argmin(const float* x, int64_t n, int d, const float* cents, int k, int order, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    const float* xi = x + i * d;
    const float x2 = hokv::sum_sq(xi, d);
    float best = 0.f;
    int bj = 0;
    for (int j = 0; j < k; ++j) {
      const float* c = cents + (int64_t)j * d;
      const float dd = hokv::l2_expansion(x2, hokv::dot_order(order, xi, c, d), hokv::sum_sq(c, d));
      if (j == 0 || dd < best) { best = dd; bj = j; }
    }
    out[i] = (uint8_t)bj;
  }
}

float host_pw_sum(const float* x, int64_t n) { return hokv::pw_sum(x, n, hokv::Ident()); }

void host_percentiles(const float* sorted, int64_t n, int k, float* out) {
  for (int i = 0; i < k; ++i) out[i] = hokv::percentile_linear(sorted, n, k, i);
}

int64_t host_linspace_pick(int64_t n, int k, int i) { return hokv::linspace_pick(n, k, i); }

int host_dot_order_for(int64_t n, int d) { return hokv::dot_order_for(n, d); }

// Exact CDC-03 score of one token: ((0 + T0[c0]) + T1[c1]) + ... then * scale.
float host_adc_score(const float* T, int M, int t_cols, const uint8_t* code, float scale) {
  float acc = 0.f;
  for (int s = 0; s < M; ++s) acc = hokv::fadd(acc, T[s * t_cols + code[s]]);
  return hokv::fmul(acc, scale);
}
}
