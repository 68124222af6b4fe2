// codec.cuh -- codebook calibration and nearest-centroid assignment.
//
// Reference semantics (helix_online_kv):
//  * OnlineCodebook (codebook.py:57-221): k = min(n_clusters, #unique values),
//    np.percentile init, Lloyd with argmin |x - c| (first minimum) and
//    per-cluster np.mean, stop when max |shift| < rtol * (c[-1] - c[0]).
//  * VectorCodebook (vector_codebook.py:95-242): k = min(n_clusters, #unique
//    rows), init = rows at linspace positions of argsort(|x|), Lloyd with the
//    L2 expansion ((|x|^2 - 2 x.c) + |c|^2) and column means, stop when
//    max |c_new - c_old| < rtol * (max|x| - min|x|).
// Every reduction follows NumPy's order (see hokv_math.cuh), so centroids and
// indices match the reference bit for bit on the same BLAS orders.
#pragma once
#include "hokv_common.cuh"

namespace hokv {

// ---- 1-D nearest centroid, first minimum ---------------------------------
__device__ __forceinline__ int nearest_brute(const float* c, int k, float x) {
  float best = fabsf(fsub(x, c[0]));
  int bj = 0;
  for (int j = 1; j < k; ++j) {
    const float d = fabsf(fsub(x, c[j]));
    if (d < best) { best = d; bj = j; }
  }
  return bj;
}

// Centroids sorted non-decreasing: |fl(x - c_j)| is valley shaped in j, so
// the first minimum is next to the insertion point (or left of it on ties).
__device__ __forceinline__ int nearest_sorted(const float* c, int k, float x) {
  int lo = 0, hi = k;  // first j with c[j] >= x
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (c[mid] < x) lo = mid + 1; else hi = mid;
  }
  const int p = lo;
  if (p == 0) return 0;
  int j;
  float m;
  if (p == k) { j = k - 1; m = fabsf(fsub(x, c[j])); }
  else {
    const float dl = fabsf(fsub(x, c[p - 1])), dr = fabsf(fsub(x, c[p]));
    if (dr < dl) return p;
    j = p - 1; m = dl;
  }
  while (j > 0 && fabsf(fsub(x, c[j - 1])) == m) --j;
  return j;
}

__global__ void k_scalar_assign(const void* __restrict__ vals, int dtype, int64_t n, int64_t vstride,
                                const float* __restrict__ cents, int k, int64_t cstride,
                                uint8_t* __restrict__ out, int64_t ostride) {
  __shared__ float c[256];
  __shared__ int s_sorted;
  const int set = blockIdx.y;
  for (int i = threadIdx.x; i < k; i += blockDim.x) c[i] = cents[(int64_t)set * cstride + i];
  if (threadIdx.x == 0) s_sorted = 1;
  __syncthreads();
  for (int i = threadIdx.x; i + 1 < k; i += blockDim.x)
    if (!(c[i] <= c[i + 1])) s_sorted = 0;
  __syncthreads();
  const bool sorted = s_sorted != 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = load_as_f32(vals, dtype, (int64_t)set * vstride + i);
    const int j = sorted ? nearest_sorted(c, k, x) : nearest_brute(c, k, x);
    out[(int64_t)set * ostride + i] = (uint8_t)j;
  }
}

__global__ void k_scalar_decode(const uint8_t* __restrict__ idx, int64_t n, const float* __restrict__ c, int k,
                                float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int j = idx[i];
    if (j >= k) { dev_flag(HOKV_ERR_DEVICE_INPUT); j = 0; }
    out[i] = c[j];
  }
}

// ---- stable counting sort of items by cluster id (one CTA) -----------------
// Writes members[] grouped by cluster, original order inside a cluster, and
// off[0..k] (exclusive offsets, off[k] = n).  cid(i) gives the cluster of item
// i (0..k-1); val(i) the value stored.  Block size must be 1024.
struct ScatterSmem {
  uint16_t warp_cnt[32][256];
  int run[256];
  int tile_tot[256];
};

template <typename CidF, typename ValT, typename ValF>
__device__ void stable_group(int64_t n, int k, CidF cid, ValF val, ValT* members, int* off, ScatterSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // counts -> offsets
  for (int j = tid; j < 256; j += blockDim.x) sm.run[j] = 0;
  __syncthreads();
  for (int64_t i = tid; i < n; i += blockDim.x) atomicAdd(&sm.run[cid(i)], 1);
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int j = 0; j < k; ++j) { const int t = sm.run[j]; off[j] = acc; sm.run[j] = acc; acc += t; }
    off[k] = acc;
  }
  for (int i = tid; i < 32 * 256; i += blockDim.x) (&sm.warp_cnt[0][0])[i] = 0;
  __syncthreads();
  for (int64_t base = 0; base < n; base += blockDim.x) {
    const int64_t i = base + tid;
    const bool valid = i < n;
    const int c = valid ? cid(i) : 256 + lane;   // unique dummy ids for the tail
    const unsigned peers = __match_any_sync(0xffffffffu, c);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (valid && rank == 0) sm.warp_cnt[warp][c] = (uint16_t)__popc(peers);
    __syncthreads();
    for (int j = tid; j < k; j += blockDim.x) {
      int r = 0;
      for (int w = 0; w < 32; ++w) { const int t = sm.warp_cnt[w][j]; sm.warp_cnt[w][j] = (uint16_t)r; r += t; }
      sm.tile_tot[j] = r;
    }
    __syncthreads();
    if (valid) members[sm.run[c] + sm.warp_cnt[warp][c] + rank] = val(i);
    __syncthreads();
    for (int j = tid; j < k; j += blockDim.x) {
      sm.run[j] += sm.tile_tot[j];
      for (int w = 0; w < 32; ++w) sm.warp_cnt[w][j] = 0;
    }
    __syncthreads();
  }
}

// ---- 1-D k-means, one CTA (1024 threads) per set ---------------------------
struct SKmSmem {
  float c[256], cn[256];
  int off[257];
  ScatterSmem sc;
  int uniq, sorted;
  float maxd;
};

__global__ void __launch_bounds__(1024) k_scalar_kmeans(const float* __restrict__ data, int64_t n, int64_t dstride,
                                                        const float* __restrict__ sorted_all, int n_clusters,
                                                        int max_iters, double rtol, float* __restrict__ cents_out,
                                                        int* __restrict__ k_out, int* __restrict__ it_out,
                                                        double* __restrict__ mse_out, uint8_t* __restrict__ assign_ws,
                                                        float* __restrict__ member_ws, uint8_t* __restrict__ assign_out) {
  __shared__ SKmSmem sm;
  const int set = blockIdx.x, tid = threadIdx.x;
  const float* x = data + (int64_t)set * dstride;
  const float* srt = sorted_all + (int64_t)set * n;
  uint8_t* asg = assign_ws + (int64_t)set * n;
  float* mem = member_ws + (int64_t)set * n;
  if (tid == 0) sm.uniq = 1;
  __syncthreads();
  {
    int local = 0;
    for (int64_t i = 1 + tid; i < n; i += blockDim.x) local += (srt[i] != srt[i - 1]) ? 1 : 0;
    if (local) atomicAdd(&sm.uniq, local);
  }
  __syncthreads();
  const int k = min(n_clusters, sm.uniq);
  for (int j = tid; j < k; j += blockDim.x) sm.c[j] = percentile_linear(srt, n, k, j);
  __syncthreads();
  double span = (double)fsub(sm.c[k - 1], sm.c[0]);
  if (span < 1e-30) span = 1.0;
  const double tol = rtol * span;
  int iters = 0;
  for (int it = 1; it <= max_iters; ++it) {
    iters = it;
    if (tid == 0) sm.sorted = 1;
    __syncthreads();
    for (int j = tid; j + 1 < k; j += blockDim.x)
      if (!(sm.c[j] <= sm.c[j + 1])) sm.sorted = 0;
    __syncthreads();
    const bool srtd = sm.sorted != 0;
    for (int64_t i = tid; i < n; i += blockDim.x)
      asg[i] = (uint8_t)(srtd ? nearest_sorted(sm.c, k, x[i]) : nearest_brute(sm.c, k, x[i]));
    __syncthreads();
    stable_group(n, k, [&](int64_t i) { return (int)asg[i]; }, [&](int64_t i) { return x[i]; }, mem, sm.off, sm.sc);
    for (int j = tid; j < k; j += blockDim.x) {
      const int cnt = sm.off[j + 1] - sm.off[j];
      sm.cn[j] = cnt ? (float)((double)pw_sum(mem + sm.off[j], cnt, Ident()) / (double)cnt) : sm.c[j];
    }
    if (tid == 0) sm.maxd = 0.f;
    __syncthreads();
    if (tid < 32) {
      float m = 0.f;
      for (int j = tid; j < k; j += 32) m = fmaxf(m, fabsf(fsub(sm.cn[j], sm.c[j])));
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (tid == 0) sm.maxd = m;
    }
    __syncthreads();
    const float maxd = sm.maxd;
    for (int j = tid; j < k; j += blockDim.x) sm.c[j] = sm.cn[j];
    __syncthreads();
    if ((double)maxd < tol) break;
  }
  for (int j = tid; j < n_clusters; j += blockDim.x) cents_out[(int64_t)set * n_clusters + j] = j < k ? sm.c[j] : 0.f;
  if (assign_out)
    for (int64_t i = tid; i < n; i += blockDim.x) assign_out[(int64_t)set * n + i] = asg[i];
  // calibration MSE: mean((x - c[a])^2) in numpy's pairwise order
  for (int64_t i = tid; i < n; i += blockDim.x) {
    const float d = fsub(x[i], sm.c[asg[i]]);
    mem[i] = fmul(d, d);
  }
  __syncthreads();
  if (tid == 0) {
    k_out[set] = k;
    it_out[set] = iters;
    mse_out[set] = (double)(float)((double)pw_sum(mem, n, Ident()) / (double)n);
  }
}

// EMA drift step for one codebook (codebook.py:146-176): one CTA.
__global__ void __launch_bounds__(1024) k_scalar_ema(const float* __restrict__ vals, int64_t n,
                                                     float* __restrict__ cents, int k, float alpha,
                                                     uint8_t* __restrict__ asg, float* __restrict__ mem) {
  __shared__ float c[256];
  __shared__ int off[257];
  __shared__ ScatterSmem sc;
  __shared__ int s_sorted;
  const int tid = threadIdx.x;
  for (int j = tid; j < k; j += blockDim.x) c[j] = cents[j];
  if (tid == 0) s_sorted = 1;
  __syncthreads();
  for (int j = tid; j + 1 < k; j += blockDim.x) if (!(c[j] <= c[j + 1])) s_sorted = 0;
  __syncthreads();
  const bool srtd = s_sorted != 0;
  for (int64_t i = tid; i < n; i += blockDim.x) asg[i] = (uint8_t)(srtd ? nearest_sorted(c, k, vals[i]) : nearest_brute(c, k, vals[i]));
  __syncthreads();
  stable_group(n, k, [&](int64_t i) { return (int)asg[i]; }, [&](int64_t i) { return vals[i]; }, mem, off, sc);
  const float a1 = (float)(1.0 - (double)alpha), a = alpha;
  for (int j = tid; j < k; j += blockDim.x) {
    const int cnt = off[j + 1] - off[j];
    if (cnt) {
      const float mean = (float)((double)pw_sum(mem + off[j], cnt, Ident()) / (double)cnt);
      cents[j] = fadd(fmul(a1, c[j]), fmul(a, mean));
    }
  }
}

// Squared error / dot / norms for quantization_error and cosine_similarity.
__global__ void __launch_bounds__(1024) k_recon_stats(const float* __restrict__ x, const float* __restrict__ r,
                                                      int64_t n, float* __restrict__ tmp, double* __restrict__ out4) {
  __shared__ double red[3][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  double a = 0, bb = 0, c = 0;
  for (int64_t i = tid; i < n; i += blockDim.x) {
    const float d = fsub(x[i], r[i]);
    tmp[i] = fmul(d, d);
    a += (double)x[i] * (double)r[i];
    bb += (double)x[i] * (double)x[i];
    c += (double)r[i] * (double)r[i];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    bb += __shfl_xor_sync(0xffffffffu, bb, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  if (lane == 0) { red[0][warp] = a; red[1][warp] = bb; red[2][warp] = c; }
  __syncthreads();
  if (tid == 0) {
    double A = 0, Bv = 0, C = 0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) { A += red[0][w]; Bv += red[1][w]; C += red[2][w]; }
    out4[0] = (double)pw_sum(tmp, n, Ident());
    out4[1] = A; out4[2] = Bv; out4[3] = C;
  }
}

// ---- vector / product assignment ------------------------------------------
// grid (ceil(n / 64), M, n_sets), 256 threads; one warp per (vector, subspace).
__global__ void __launch_bounds__(256) k_pq_assign(const void* __restrict__ x, int dtype, int64_t n, int64_t xrs,
                                                   int64_t xss, int M, int sd, const float* __restrict__ cents,
                                                   int slots, int64_t css, const int* __restrict__ kk, int64_t kss,
                                                   uint8_t* __restrict__ out, int64_t ors, int64_t oss, int order,
                                                   int use_smem) {
  extern __shared__ float sm[];
  const int s = blockIdx.y, set = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int k = kk[(int64_t)set * kss + s];
  k = k < 1 ? 1 : (k > slots ? slots : k);
  const float* cg = cents + (int64_t)set * css + (int64_t)s * slots * sd;
  const int rstride = use_smem ? sd + 1 : sd;
  float* c2 = sm;                       // [256]
  float* xs = sm + 256;                 // [8][sd]
  float* cs = xs + 8 * sd;              // [k][sd + 1] (if use_smem)
  const float* crow0 = use_smem ? cs : cg;
  if (use_smem)
    for (int i = tid; i < k * sd; i += blockDim.x) cs[(i / sd) * rstride + (i % sd)] = cg[i];
  __syncthreads();
  for (int j = tid; j < k; j += blockDim.x) c2[j] = sum_sq(crow0 + (int64_t)j * rstride, sd);
  __syncthreads();
  const int64_t v0 = (int64_t)blockIdx.x * 64;
  for (int vi = warp; vi < 64; vi += 8) {
    const int64_t i = v0 + vi;
    if (i >= n) break;
    float* xw = xs + warp * sd;
    for (int d = lane; d < sd; d += 32)
      xw[d] = load_as_f32(x, dtype, (int64_t)set * xss + i * xrs + (int64_t)s * sd + d);
    __syncwarp();
    const float x2 = sum_sq(xw, sd);
    float best = INFINITY;
    int bj = 0x7fffffff;
    for (int j = lane; j < k; j += 32) {
      const float dot = dot_order(order, xw, crow0 + (int64_t)j * rstride, sd);
      const float dd = l2_expansion(x2, dot, c2[j]);
      if (dd < best || bj == 0x7fffffff) { best = dd; bj = j; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ob < best || (ob == best && oj < bj)) { best = ob; bj = oj; }
    }
    if (lane == 0) out[(int64_t)set * oss + i * ors + s] = (uint8_t)(bj == 0x7fffffff ? 0 : bj);
    __syncwarp();
  }
}

// Batched assignment in the sequential-FMA order (BLAS sgemm with >= 5 rows,
// the order every prefill-sized batch gets), SD in {4, 8}: grid
// (ceil(n / (256 V)), M, n_sets), 256 threads, V vectors per thread held in
// registers against every centroid of the subspace, read from shared memory
// as broadcasts (SD * V <= 32 keeps the vectors in registers).  Same
// arithmetic and tie rule (lowest index) as k_pq_assign.
template <int SD, int V>
__global__ void __launch_bounds__(256) k_pq_assign_seq(const void* __restrict__ x, int dtype, int64_t n, int64_t xrs,
                                                       int64_t xss, const float* __restrict__ cents, int slots,
                                                       int64_t css, const int* __restrict__ kk, int64_t kss,
                                                       uint8_t* __restrict__ out, int64_t ors, int64_t oss) {
  __shared__ float cs[256 * SD];
  __shared__ float c2[256];
  const int s = blockIdx.y, set = blockIdx.z;
  const int tid = threadIdx.x;
  int k = kk[(int64_t)set * kss + s];
  k = k < 1 ? 1 : (k > slots ? slots : k);
  const float* cg = cents + (int64_t)set * css + (int64_t)s * slots * SD;
  for (int i = tid; i < k * SD; i += blockDim.x) cs[i] = cg[i];
  __syncthreads();
  for (int j = tid; j < k; j += blockDim.x) c2[j] = sum_sq(cs + j * SD, SD);
  float xv[V][SD], x2[V], best[V];
  int bj[V];
  const int64_t i0 = (int64_t)blockIdx.x * 256 * V + tid;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int64_t i = i0 + (int64_t)v * 256;
    const int64_t base = (int64_t)set * xss + (i < n ? i : 0) * xrs + (int64_t)s * SD;
#pragma unroll
    for (int d = 0; d < SD; ++d) xv[v][d] = load_as_f32(x, dtype, base + d);
    x2[v] = sum_sq(xv[v], SD);
    best[v] = INFINITY;
    bj[v] = 0x7fffffff;
  }
  __syncthreads();
  if (i0 >= n) return;   // no vector of this thread in range (small batches): nothing to score
  // vectors v < nv of this block's threads can be in range (the same for the
  // whole block, so the branch below does not diverge)
  const int64_t left = n - (int64_t)blockIdx.x * 256 * V;
  const int nv = left >= 256 * V ? V : (int)((left + 255) / 256);
  for (int j = 0; j < k; ++j) {
    float c[SD];
#pragma unroll
    for (int d = 0; d < SD; ++d) c[d] = cs[j * SD + d];
    const float cj2 = c2[j];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (v >= nv) break;
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < SD; ++d) acc = ffma(xv[v][d], c[d], acc);
      const float dd = l2_expansion(x2[v], acc, cj2);
      if (dd < best[v] || bj[v] == 0x7fffffff) { best[v] = dd; bj[v] = j; }
    }
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int64_t i = i0 + (int64_t)v * 256;
    if (i < n) out[(int64_t)set * oss + i * ors + s] = (uint8_t)bj[v];
  }
}

__device__ __forceinline__ float kv_to_f32(float v) { return v; }
__device__ __forceinline__ float kv_to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float kv_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// Tier aging: PQ codes of the tokens [cold_from[b], cold_to[b]) of every
// (sequence b, KV head h) from the exact key store, written in place into the
// code store.  grid (gx, H_kv, B), 256 threads, one warp per (token,
// subspace) item; the arithmetic and tie rule are those of k_pq_assign.
template <typename KVT>
__global__ void __launch_bounds__(256) k_age_tokens(const KVT* __restrict__ k, int64_t kv_sb, int64_t kv_sh, int D,
                                                    int M, int sd, const float* __restrict__ cb, int64_t cb_sb,
                                                    int64_t cb_sh, int slots, const int* __restrict__ cbk,
                                                    int64_t cbk_sb, int64_t cbk_sh, uint8_t* __restrict__ codes,
                                                    int64_t c_sb, int64_t c_sh, int CS, const int* __restrict__ from,
                                                    const int* __restrict__ to, int64_t cap, int order) {
  __shared__ float xs[8][32];
  const int h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int t0 = from[b], t1 = to[b];
  if (t0 < 0 || t1 > cap || t0 > t1) {
    dev_flag(HOKV_ERR_DEVICE_INPUT);
    return;
  }
  const int64_t n_items = (int64_t)(t1 - t0) * M;
  const KVT* kb = k + (int64_t)b * kv_sb + (int64_t)h * kv_sh;
  const float* cbase = cb + (int64_t)b * cb_sb + (int64_t)h * cb_sh;
  const int* kcount = cbk + (int64_t)b * cbk_sb + (int64_t)h * cbk_sh;
  uint8_t* cout = codes + (int64_t)b * c_sb + (int64_t)h * c_sh;
  float* xw = xs[warp];
  for (int64_t it = (int64_t)blockIdx.x * 8 + warp; it < n_items; it += (int64_t)gridDim.x * 8) {
    const int64_t t = t0 + it / M;
    const int s = (int)(it - (it / M) * M);
    int kk = kcount[s];
    kk = kk < 1 ? 1 : (kk > slots ? slots : kk);
    if (lane < sd) xw[lane] = kv_to_f32(kb[t * D + (int64_t)s * sd + lane]);
    __syncwarp();
    const float x2 = sum_sq(xw, sd);
    const float* cs = cbase + (int64_t)s * slots * sd;
    float best = INFINITY;
    int bj = 0x7fffffff;
    for (int j = lane; j < kk; j += 32) {
      const float* crow = cs + (int64_t)j * sd;
      const float dd = l2_expansion(x2, dot_order(order, xw, crow, sd), sum_sq(crow, sd));
      if (dd < best || bj == 0x7fffffff) { best = dd; bj = j; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ob < best || (ob == best && oj < bj)) { best = ob; bj = oj; }
    }
    if (lane == 0) cout[t * CS + s] = (uint8_t)(bj == 0x7fffffff ? 0 : bj);
    __syncwarp();
  }
}

__global__ void k_pq_decode(const uint8_t* __restrict__ codes, int64_t n, int64_t crs, int M, int sd,
                            const float* __restrict__ cents, int slots, float* __restrict__ out) {
  const int64_t total = n * M * sd;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / (M * sd);
    const int rem = (int)(e - i * M * sd);
    const int s = rem / sd, d = rem - s * sd;
    int j = codes[i * crs + s];
    if (j >= slots) { dev_flag(HOKV_ERR_DEVICE_INPUT); j = 0; }
    out[e] = cents[((int64_t)s * slots + j) * sd + d];
  }
}

// ---- vector k-means, one CTA (1024 threads) per set --------------------------
// Work layout per set (global workspace): asg[n] int, x2[n] f32, mem[n] int,
// order[n] int, err[n*sd] f32.  Shared: centroids [k][sd] + new + |c|^2.
__device__ __forceinline__ int row_cmp(const float* a, const float* b, int sd) {
  for (int d = 0; d < sd; ++d) {
    if (a[d] < b[d]) return -1;
    if (a[d] > b[d]) return 1;
  }
  return 0;
}

__global__ void __launch_bounds__(1024) k_vq_kmeans(const float* __restrict__ data, int64_t n, int sd, int64_t drs,
                                                    int64_t dss, int n_clusters, int max_iters, double rtol,
                                                    float* __restrict__ cents_out, int slots, int* __restrict__ k_out,
                                                    int* __restrict__ it_out, double* __restrict__ mse_out,
                                                    unsigned char* __restrict__ ws, int64_t ws_per_set) {
  extern __shared__ __align__(16) unsigned char smraw[];
  __shared__ ScatterSmem sc;
  __shared__ int off[257];
  __shared__ int s_uniq;
  __shared__ float s_maxd, s_nmin, s_nmax;
  const int set = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const float* X = data + (int64_t)set * dss;
  unsigned char* w = ws + (int64_t)set * ws_per_set;
  int* asg = reinterpret_cast<int*>(w);
  float* x2 = reinterpret_cast<float*>(w + 4 * n);
  int* mem = reinterpret_cast<int*>(w + 8 * n);
  uint64_t* keys = reinterpret_cast<uint64_t*>(w + 12 * n + (8 - (12 * n) % 8) % 8);
  float* err = reinterpret_cast<float*>(keys + n);
  float* C = reinterpret_cast<float*>(smraw);          // [n_clusters][sd]
  float* Cn = C + (int64_t)n_clusters * sd;            // [n_clusters][sd]
  float* c2 = Cn + (int64_t)n_clusters * sd;           // [n_clusters]
  int* ordr = reinterpret_cast<int*>(c2 + n_clusters); // [npow2] sort scratch (indices)

  int npow = 1;
  while (npow < n) npow <<= 1;
  auto row = [&](int64_t i) { return X + i * drs; };

  // 1. unique rows: bitonic sort of row indices lexicographically
  for (int i = tid; i < npow; i += blockDim.x) ordr[i] = i < n ? i : -1;
  __syncthreads();
  for (int kk = 2; kk <= npow; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < npow; i += blockDim.x) {
        const int l = i ^ jj;
        if (l > i) {
          const int a = ordr[i], bq = ordr[l];
          int cmp;
          if (a < 0) cmp = (bq < 0) ? 0 : 1;
          else if (bq < 0) cmp = -1;
          else cmp = row_cmp(row(a), row(bq), sd);
          const bool up = (i & kk) == 0;
          if ((up && cmp > 0) || (!up && cmp < 0)) { ordr[i] = bq; ordr[l] = a; }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) s_uniq = n > 0 ? 1 : 0;
  __syncthreads();
  {
    int local = 0;
    for (int64_t i = 1 + tid; i < n; i += blockDim.x) local += row_cmp(row(ordr[i]), row(ordr[i - 1]), sd) != 0;
    if (local) atomicAdd(&s_uniq, local);
  }
  // 2. norms, 3. stable argsort of norms (key = norm bits, index)
  for (int64_t i = tid; i < n; i += blockDim.x) {
    x2[i] = sum_sq(row(i), sd);
    keys[i] = ((uint64_t)ord_f32(sqrtf(x2[i])) << 32) | (uint64_t)i;
  }
  __syncthreads();
  for (int i = tid; i < npow; i += blockDim.x) ordr[i] = i < n ? i : -1;
  __syncthreads();
  for (int kk = 2; kk <= npow; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < npow; i += blockDim.x) {
        const int l = i ^ jj;
        if (l > i) {
          const int a = ordr[i], bq = ordr[l];
          const uint64_t ka = a < 0 ? ~0ull : keys[a], kb = bq < 0 ? ~0ull : keys[bq];
          const bool up = (i & kk) == 0;
          if ((up && ka > kb) || (!up && ka < kb)) { ordr[i] = bq; ordr[l] = a; }
        }
      }
      __syncthreads();
    }
  }
  const int k = min(n_clusters, s_uniq);
  if (tid == 0) {
    s_nmin = unord_f32((uint32_t)(keys[ordr[0]] >> 32));
    s_nmax = unord_f32((uint32_t)(keys[ordr[n - 1]] >> 32));
  }
  // 4. init centroids from linspace picks of the norm order
  for (int e = tid; e < k * sd; e += blockDim.x) {
    const int j = e / sd, d = e - j * sd;
    C[e] = row(ordr[linspace_pick(n, k, j)])[d];
  }
  __syncthreads();
  double span = (double)fsub(s_nmax, s_nmin);
  if (span < 1e-30) span = 1.0;
  const double tol = rtol * span;
  const int order = dot_order_for(n, sd);
  int iters = 0;
  for (int it = 1; it <= max_iters; ++it) {
    iters = it;
    for (int j = tid; j < k; j += blockDim.x) c2[j] = sum_sq(C + j * sd, sd);
    __syncthreads();
    for (int64_t i = tid; i < n; i += blockDim.x) {
      const float* xi = row(i);
      float best = INFINITY;
      int bj = 0;
      for (int j = 0; j < k; ++j) {
        const float dd = l2_expansion(x2[i], dot_order(order, xi, C + j * sd, sd), c2[j]);
        if (dd < best || j == 0) { best = dd; bj = j; }
      }
      asg[i] = bj;
    }
    __syncthreads();
    stable_group(n, k, [&](int64_t i) { return asg[i]; }, [&](int64_t i) { return (int)i; }, mem, off, sc);
    for (int e = tid; e < k * sd; e += blockDim.x) {
      const int j = e / sd, d = e - j * sd;
      const int cnt = off[j + 1] - off[j];
      if (cnt) {
        float acc = row(mem[off[j]])[d];
        for (int m = 1; m < cnt; ++m) acc = fadd(acc, row(mem[off[j] + m])[d]);
        Cn[e] = (float)((double)acc / (double)cnt);
      } else {
        Cn[e] = C[e];
      }
    }
    if (tid == 0) s_maxd = 0.f;
    __syncthreads();
    for (int j = tid; j < k; j += blockDim.x) {
      const float* cn = Cn + j * sd;
      const float* co = C + j * sd;
      const float ss = pw_sum_idx(sd, [&](int64_t d) { const float df = fsub(cn[d], co[d]); return fmul(df, df); });
      atomicMax(reinterpret_cast<int*>(&s_maxd), __float_as_int(sqrtf(ss)));  // >= 0
    }
    __syncthreads();
    const float maxd = s_maxd;
    for (int e = tid; e < k * sd; e += blockDim.x) C[e] = Cn[e];
    __syncthreads();
    if ((double)maxd < tol) break;
  }
  (void)lane;
  float* co = cents_out + (int64_t)set * slots * sd;
  for (int e = tid; e < slots * sd; e += blockDim.x) co[e] = e < k * sd ? C[e] : 0.f;
  for (int64_t e = tid; e < n * sd; e += blockDim.x) {
    const int64_t i = e / sd;
    const int d = (int)(e - i * sd);
    const float df = fsub(row(i)[d], C[asg[i] * sd + d]);
    err[e] = fmul(df, df);
  }
  __syncthreads();
  if (tid == 0) {
    k_out[set] = k;
    it_out[set] = iters;
    mse_out[set] = (double)(float)((double)pw_sum(err, n * sd, Ident()) / (double)(n * sd));
  }
}

// ---- binned value output (Paths B / D) --------------------------------------
__global__ void k_value_bins(const double* __restrict__ w, int64_t n, const uint8_t* __restrict__ codes, int64_t crs,
                             int M, double* __restrict__ bins) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n * M; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / M;
    const int s = (int)(e - t * M);
    atomicAdd(&bins[s * 256 + codes[t * crs + s]], w[t]);
  }
}
__global__ void k_value_out(const double* __restrict__ bins, int M, int sd, const float* __restrict__ cents, int slots,
                            const int* __restrict__ kk, float* __restrict__ out) {
  const int s = blockIdx.x;
  const int k = min(kk[s], slots);
  for (int d = threadIdx.x; d < sd; d += blockDim.x) {
    double acc = 0.0;
    for (int j = 0; j < k; ++j) acc += bins[s * 256 + j] * (double)cents[((int64_t)s * slots + j) * sd + d];
    out[s * sd + d] = (float)acc;
  }
}

}  // namespace hokv
