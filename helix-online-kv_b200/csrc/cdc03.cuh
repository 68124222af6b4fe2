// cdc03.cuh -- PQ lookup tables, ADC scoring and CDC-03 decode attention.
//
// Decode step, per layer:
//   K6 k6_candidates  grid (chunks, B*H_kv): builds the per-KV-head sub-tables
//      for the G query heads of the GQA group, quantises them to 8-bit entries
//      in a bank-conflict-free shared-memory layout, streams the uint8 PQ codes
//      of one chunk of cold tokens, and emits the token indices whose 8-bit
//      score lies within the proven error band of the chunk's top-k boundary.
//   K7 k7_select_attend  grid (B*H_kv*G): rebuilds the exact fp32 sub-table of
//      one query head, rescores the candidates in the reference's summation
//      order, selects sinks + top-(k - sinks) exactly (ties to the lower index)
//      and runs exact softmax attention over the selected cold tokens plus the
//      hot window, gathering fp16/bf16 K/V rows straight into registers.
//
// Reference: helix_online_kv/compressed_attention.py:315-412 (hybrid_pq_attention),
// product_codebook.py:172-227 (tables, gather).
#pragma once
#include "hokv_common.cuh"

namespace hokv {

constexpr int K6_THREADS = 256;
constexpr int K6_CHUNK_MAX = 4096;   // tokens per K6 CTA (16 per thread)
constexpr int CAND_MAX = 512;        // candidates per (unit, chunk, head)
constexpr int K7_THREADS = 256;
constexpr int K7_CAP = 2048;         // key buffer of the exact selection
constexpr int TOPK_MAX = 1024;       // largest top_k with k < S_c

struct Cdc03P {
  int B, Hkv, G, D, M, sd, CS, slots, top_k, sink, hot;
  float scale;
  int lut_order;
  const void* q; int q_dtype; int64_t q_sb;
  void* out; int out_dtype; int64_t out_sb;
  const void* k; const void* v; int64_t kv_sb, kv_sh;
  int64_t cap;
  const uint8_t* codes; int64_t c_sb, c_sh;
  const float* cb; int64_t cb_sb, cb_sh;
  const int* cbk; int64_t cbk_sb, cbk_sh;
  const int* seq_len;
  int* sel_idx; float* sel_score; int* sel_count;
  uint32_t* cand_idx; int* cand_cnt;
  int n_chunks, chunk, GT;
};

// Per-sequence geometry of the cold range, identical in K6 and K7.
struct ColdRange {
  int S, Sc, k, sink, kp;
};
__device__ __forceinline__ ColdRange cold_range(const Cdc03P& p, int b) {
  ColdRange r;
  int S = p.seq_len[b];
  if (S < 0 || (int64_t)S > p.cap) { dev_flag(HOKV_ERR_DEVICE_INPUT); S = S < 0 ? 0 : (int)p.cap; }
  r.S = S;
  r.Sc = S - p.hot > 0 ? S - p.hot : 0;
  r.k = p.top_k < r.Sc ? p.top_k : r.Sc;
  r.sink = p.sink < r.Sc ? p.sink : r.Sc;
  r.kp = r.k - r.sink;
  return r;
}

// ---------------------------------------------------------------------------
// Quantised sub-table geometry.  Entry = G 8-bit codes of one (subspace s,
// centroid j).  Rows are 128 B (one shared-memory wavefront).  Lane L at step
// u reads subspace (u + L) mod CS, and each row stores copies / row blocks
// such that the lanes of one wavefront always hit distinct columns: every
// lookup is bank-conflict free whatever the code bytes are.
// ---------------------------------------------------------------------------
template <int CS, int GT>
struct QGeo {
  static constexpr int EW = (GT <= 4) ? 4 : 8;
  static constexpr int COLS = 128 / EW;
  static constexpr int RB = (CS > COLS) ? CS / COLS : 1;
  static constexpr int BYTES = RB * 256 * 128;
  static constexpr int NACC = (GT == 8) ? 4 : (GT == 4 ? 2 : 1);
  static constexpr int W = CS / 4;
  __device__ static __forceinline__ int col_of(int lane, int s) {
    return (CS <= COLS) ? (((lane % COLS) / CS) * CS + s) : (s % COLS);
  }
  __device__ static __forceinline__ int rb_of(int s) { return (CS <= COLS) ? 0 : s / COLS; }
};

template <int W>
__device__ __forceinline__ void load_code(const uint8_t* p, uint32_t (&w)[W]) {
  if constexpr (W == 1) {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else if constexpr (W == 2) {
    uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (W == 4) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
    uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    uint4 c = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = c.x; w[5] = c.y; w[6] = c.z; w[7] = c.w;
  }
}

// Rotate a W-word byte string left by r bytes: out byte u = in byte (u + r) mod 4W.
template <int W>
__device__ __forceinline__ void rotate_bytes(uint32_t (&w)[W], int r) {
  const int rw = r >> 2, rb = r & 3;
#pragma unroll
  for (int bit = 1; bit < W; bit <<= 1) {
    uint32_t t[W];
    const bool on = (rw & bit) != 0;
#pragma unroll
    for (int i = 0; i < W; ++i) t[i] = on ? w[(i + bit) % W] : w[i];
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = t[i];
  }
  uint32_t t[W];
#pragma unroll
  for (int i = 0; i < W; ++i) t[i] = __funnelshift_r(w[i], w[(i + 1) % W], 8 * rb);
#pragma unroll
  for (int i = 0; i < W; ++i) w[i] = t[i];
}

// Sub-table values for one centroid row: T[g][s][j] = q_g[s-slice] . c  (BLAS order).
template <int SD>
__device__ __forceinline__ void lut_row(const float* __restrict__ sq, int D, const float* __restrict__ crow,
                                        int s, int order, int GT, float* outv /*[GT]*/) {
  float c[SD];
#pragma unroll
  for (int i = 0; i < SD; ++i) c[i] = __ldg(crow + i);
  for (int g = 0; g < GT; ++g) outv[g] = dot_order(order, sq + g * D + s * SD, c, SD);
}

template <int CS, int GT>
__global__ void __launch_bounds__(K6_THREADS, 2) k6_candidates(Cdc03P p) {
  using Q = QGeo<CS, GT>;
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* qlut = smem;
  float* T = reinterpret_cast<float*>(smem + Q::BYTES);            // [GT][CS][256] while building
  uint16_t* apx = reinterpret_cast<uint16_t*>(smem + Q::BYTES);    // [GT][chunk] afterwards
  const int regionA = max(GT * CS * 1024, GT * p.chunk * 2);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + Q::BYTES + regionA);  // [GT][256]
  float* sq = reinterpret_cast<float*>(smem + Q::BYTES + regionA + GT * 1024);  // [GT][D]
  __shared__ float s_lo[GT * CS], s_hi[GT * CS], s_inv[GT];
  __shared__ int s_margin[GT], s_thr[GT], s_cnt[GT];

  const int u = blockIdx.y, c = blockIdx.x;
  const int b = u / p.Hkv, h = u - b * p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ColdRange cr = cold_range(p, b);
  const int lo_t = max(c * p.chunk, cr.sink), hi_t = min((c + 1) * p.chunk, cr.Sc);
  int* cnt_out = p.cand_cnt + ((int64_t)u * p.n_chunks + c) * GT;
  if (cr.k >= cr.Sc || cr.kp <= 0 || lo_t >= hi_t) {
    if (tid < GT) cnt_out[tid] = 0;
    return;
  }
  const int D = p.D, M = p.M, sd = p.sd;

  // ---- queries of the GQA group -> shared f32 -----------------------------
  for (int i = tid; i < GT * D; i += K6_THREADS) {
    int g = i / D, d = i - g * D;
    sq[i] = (g < p.G) ? load_as_f32(p.q, p.q_dtype, (int64_t)b * p.q_sb + (int64_t)(h * p.G + g) * D + d) : 0.f;
  }
  for (int i = tid; i < GT * 256; i += K6_THREADS) hist[i] = 0;
  if (tid < GT) s_cnt[tid] = 0;
  __syncthreads();

  // ---- exact sub-tables (fp32, BLAS order) into region A --------------------
  const float* cbase = p.cb + (int64_t)b * p.cb_sb + (int64_t)h * p.cb_sh;
  const int* kbase = p.cbk + (int64_t)b * p.cbk_sb + (int64_t)h * p.cbk_sh;
  {
    const int j = tid;  // K6_THREADS == 256 slots
    float vals[GT];
    for (int s = 0; s < M; ++s) {
      int ks = kbase[s];
      ks = ks < 0 ? 0 : (ks > p.slots ? p.slots : ks);
      if (j < ks) {
        const float* crow = cbase + ((int64_t)s * p.slots + j) * sd;
        switch (sd) {
          case 4: lut_row<4>(sq, D, crow, s, p.lut_order, GT, vals); break;
          case 8: lut_row<8>(sq, D, crow, s, p.lut_order, GT, vals); break;
          case 16: lut_row<16>(sq, D, crow, s, p.lut_order, GT, vals); break;
          case 32: lut_row<32>(sq, D, crow, s, p.lut_order, GT, vals); break;
          default:
            for (int g = 0; g < GT; ++g) vals[g] = dot_order(p.lut_order, sq + g * D + s * sd, crow, sd);
        }
      } else {
#pragma unroll
        for (int g = 0; g < GT; ++g) vals[g] = 0.f;
      }
#pragma unroll
      for (int g = 0; g < GT; ++g) T[(g * CS + s) * 256 + j] = vals[g];
    }
  }
  __syncthreads();

  // ---- per (head, subspace) value range -----------------------------------
  for (int pr = warp; pr < GT * M; pr += K6_THREADS / 32) {
    const int g = pr / M, s = pr - g * M;
    const float* row = T + (g * CS + s) * 256;
    float mn = row[lane], mx = row[lane];
#pragma unroll
    for (int i = 1; i < 8; ++i) { float v = row[lane + 32 * i]; mn = fminf(mn, v); mx = fmaxf(mx, v); }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) { s_lo[g * CS + s] = mn; s_hi[g * CS + s] = mx; }
  }
  __syncthreads();
  if (tid < GT) {
    const int g = tid;
    float rmax = 0.f;
    double sa = 0.0;
    for (int s = 0; s < M; ++s) {
      float lo = s_lo[g * CS + s], hi = s_hi[g * CS + s];
      rmax = fmaxf(rmax, hi - lo);
      sa += fmax(fabs((double)lo), fabs((double)hi));
    }
    // Error budget in code units: rounding of each entry (<= 0.5 + fp32 slop)
    // for both tokens of a comparison, plus the fp32 summation error of the
    // exact scores and ties created by the final scale multiply.
    const double delta = rmax > 0.f ? (double)rmax / 255.0 : 1.0;
    const double e_f = (double)(M + 1) * ldexp(1.0, -22) * sa / delta;
    const bool ok_scale = (p.scale > 0.f) && isfinite(p.scale) && isfinite(sa);
    s_inv[g] = rmax > 0.f ? 255.f / rmax : 0.f;
    s_margin[g] = ok_scale ? (int)ceil((double)M * 1.0002 + e_f) : (1 << 30);
  }
  __syncthreads();

  // ---- quantised, replicated sub-tables -----------------------------------
  {
    const int j = tid;
    for (int rb = 0; rb < Q::RB; ++rb) {
#pragma unroll 4
      for (int i = 0; i < Q::COLS; ++i) {
        const int col = (i + lane) & (Q::COLS - 1);
        const int s = (CS <= Q::COLS) ? (col % CS) : (rb * Q::COLS + col);
        uint32_t code[GT];
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          uint32_t cv = 0;
          if (s < M) {
            float x = __fmul_rn(__fsub_rn(T[(g * CS + s) * 256 + j], s_lo[g * CS + s]), s_inv[g]);
            x = fminf(fmaxf(rintf(x), 0.f), 255.f);
            cv = (uint32_t)x;
          }
          code[g] = cv;
        }
        const int e = (rb * 256 + j) * Q::COLS + col;
        if constexpr (GT == 1) {
          reinterpret_cast<uint32_t*>(qlut)[e] = code[0];
        } else if constexpr (GT == 2) {
          reinterpret_cast<uint32_t*>(qlut)[e] = code[0] | (code[1] << 16);
        } else if constexpr (GT == 4) {
          reinterpret_cast<uint32_t*>(qlut)[e] = code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
        } else {
          uint2 v;
          v.x = code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
          v.y = code[4] | (code[5] << 8) | (code[6] << 16) | (code[7] << 24);
          reinterpret_cast<uint2*>(qlut)[e] = v;
        }
      }
    }
  }
  __syncthreads();   // region A (T) is dead from here on; reused for apx

  // ---- stream the chunk's codes: 8-bit approximate scores ------------------
  const uint8_t* codes = p.codes + (int64_t)b * p.c_sb + (int64_t)h * p.c_sh;
  const int r = lane % CS;
  int colidx[CS];
#pragma unroll
  for (int uu = 0; uu < CS; ++uu) {
    const int s = (uu + r) % CS;
    colidx[uu] = Q::rb_of(s) * 256 * Q::COLS + Q::col_of(lane, s);
  }
  int mxv[GT];
#pragma unroll
  for (int g = 0; g < GT; ++g) mxv[g] = -1;
  const int base = c * p.chunk;
  const int tpt = p.chunk / K6_THREADS;
  constexpr int U = 4;
  for (int it0 = 0; it0 < tpt; it0 += U) {
    uint32_t w[U][Q::W];
    bool valid[U];
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const int t = base + (it0 + q) * K6_THREADS + tid;
      valid[q] = (it0 + q < tpt) && t >= lo_t && t < hi_t;
      if (valid[q]) load_code<Q::W>(codes + (int64_t)t * CS, w[q]);
      else {
#pragma unroll
        for (int i = 0; i < Q::W; ++i) w[q][i] = 0;
      }
    }
#pragma unroll
    for (int q = 0; q < U; ++q) {
      if (it0 + q >= tpt) break;
      rotate_bytes<Q::W>(w[q], r);
      uint32_t acc[Q::NACC];
#pragma unroll
      for (int a = 0; a < Q::NACC; ++a) acc[a] = 0;
#pragma unroll
      for (int uu = 0; uu < CS; ++uu) {
        const uint32_t byte = (w[q][uu >> 2] >> (8 * (uu & 3))) & 0xffu;
        const int e = colidx[uu] + (int)byte * Q::COLS;
        if constexpr (Q::EW == 4) {
          const uint32_t x = reinterpret_cast<const uint32_t*>(qlut)[e];
          if constexpr (GT <= 2) {
            acc[0] += x;
          } else {
            acc[0] += x & 0x00ff00ffu;
            acc[1] += (x >> 8) & 0x00ff00ffu;
          }
        } else {
          const uint2 x = reinterpret_cast<const uint2*>(qlut)[e];
          acc[0] += x.x & 0x00ff00ffu;
          acc[1] += (x.x >> 8) & 0x00ff00ffu;
          acc[2] += x.y & 0x00ff00ffu;
          acc[3] += (x.y >> 8) & 0x00ff00ffu;
        }
      }
      int a[GT];
      if constexpr (GT == 1) {
        a[0] = (int)acc[0];
      } else if constexpr (GT == 2) {
        a[0] = (int)(acc[0] & 0xffffu); a[1] = (int)(acc[0] >> 16);
      } else {
        // acc[0] = h0 | h2<<16, acc[1] = h1 | h3<<16 (, acc[2] = h4 | h6<<16, acc[3] = h5 | h7<<16)
        a[0] = (int)(acc[0] & 0xffffu); a[2] = (int)(acc[0] >> 16);
        a[1] = (int)(acc[1] & 0xffffu); a[3] = (int)(acc[1] >> 16);
        if constexpr (GT == 8) {
          a[4] = (int)(acc[2] & 0xffffu); a[6] = (int)(acc[2] >> 16);
          a[5] = (int)(acc[3] & 0xffffu); a[7] = (int)(acc[3] >> 16);
        }
      }
      const int lt = (it0 + q) * K6_THREADS + tid;
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        apx[g * p.chunk + lt] = (uint16_t)a[g];
        if (valid[q]) mxv[g] = max(mxv[g], a[g]);
      }
    }
  }

  // ---- lower bound of the k'-th largest approximate score ------------------
  int sh = 0;
  while (((M * 255) >> sh) > 255) ++sh;
#pragma unroll
  for (int g = 0; g < GT; ++g)
    if (mxv[g] >= 0) atomicAdd(&hist[g * 256 + (mxv[g] >> sh)], 1u);
  __syncthreads();
  if (warp < GT) {
    const int g = warp;
    const uint32_t* hg = hist + g * 256;
    uint32_t ls = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) ls += hg[lane * 8 + i];
    uint32_t suf = ls;  // inclusive suffix over lanes >= lane
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t t = __shfl_down_sync(0xffffffffu, suf, o);
      if (lane + o < 32) suf += t;
    }
    const uint32_t kp = (uint32_t)cr.kp;
    const unsigned ball = __ballot_sync(0xffffffffu, suf >= kp);
    int thr = -(1 << 30);
    if (ball != 0u) {
      const int lstar = 31 - __clz((int)ball);
      const uint32_t above = __shfl_sync(0xffffffffu, suf - ls, lstar);
      int bstar = -1;
      if (lane == lstar) {
        uint32_t cum = above;
        for (int i = 7; i >= 0; --i) {
          cum += hg[lane * 8 + i];
          if (cum >= kp) { bstar = lane * 8 + i; break; }
        }
      }
      bstar = __shfl_sync(0xffffffffu, bstar, lstar);
      thr = (bstar << sh) - s_margin[g];
    }
    if (lane == 0) s_thr[g] = (s_margin[g] >= (1 << 30)) ? -(1 << 30) : thr;
  }
  __syncthreads();

  // ---- emit candidates ------------------------------------------------------
  uint32_t* cand = p.cand_idx + ((int64_t)u * p.n_chunks + c) * GT * CAND_MAX;
  for (int it = 0; it < tpt; ++it) {
    const int t = base + it * K6_THREADS + tid;
    const bool valid = t >= lo_t && t < hi_t;
    const int lt = it * K6_THREADS + tid;
    for (int g = 0; g < p.G; ++g) {
      const bool pred = valid && ((int)apx[g * p.chunk + lt] >= s_thr[g]);
      const unsigned m = __ballot_sync(0xffffffffu, pred);
      if (m) {
        const int leader = __ffs(m) - 1;
        int basep = 0;
        if (lane == leader) basep = atomicAdd(&s_cnt[g], __popc(m));
        basep = __shfl_sync(0xffffffffu, basep, leader);
        const int slot = basep + __popc(m & ((1u << lane) - 1u));
        if (pred && slot < CAND_MAX) cand[g * CAND_MAX + slot] = (uint32_t)t;
      }
    }
  }
  __syncthreads();
  if (tid < GT) cnt_out[tid] = (tid < p.G && s_cnt[tid] > CAND_MAX) ? -1 : s_cnt[tid];
}

// ---------------------------------------------------------------------------
// Block-wide exact selection: keep the m largest of n unique 64-bit keys in
// keys[0..m).  Histogram refinement on the key range; each round narrows the
// range containing the m-th key by >= 2^9, so it ends in <= 8 rounds.
// ---------------------------------------------------------------------------
struct SelShared {
  unsigned long long lo, hi, thr;
  int need, done, bstar, above, binc, n_out;
};

template <int NT>
__device__ void select_topm(uint64_t* keys, int n, int m, uint32_t* hist, SelShared* sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = NT / 32;
  __shared__ unsigned long long red_lo[NW], red_hi[NW];
  if (n <= m) return;
  unsigned long long lo = ~0ull, hi = 0ull;
  for (int i = tid; i < n; i += NT) { unsigned long long k = keys[i]; lo = k < lo ? k : lo; hi = k > hi ? k : hi; }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    unsigned long long a = __shfl_xor_sync(0xffffffffu, lo, o), c = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = a < lo ? a : lo; hi = c > hi ? c : hi;
  }
  if (lane == 0) { red_lo[warp] = lo; red_hi[warp] = hi; }
  __syncthreads();
  if (tid == 0) {
    unsigned long long L = red_lo[0], H = red_hi[0];
    for (int w = 1; w < NW; ++w) { L = red_lo[w] < L ? red_lo[w] : L; H = red_hi[w] > H ? red_hi[w] : H; }
    sh->lo = L; sh->hi = H; sh->need = m; sh->done = 0;
  }
  __syncthreads();
  for (int round = 0; round < 10; ++round) {
    const unsigned long long L = sh->lo, H = sh->hi;
    const unsigned long long range = H - L;
    const int bits = range ? 64 - __clzll((long long)range) : 0;
    const int shift = bits > 10 ? bits - 10 : 0;
    const int nb = (int)(range >> shift) + 1;
    for (int i = tid; i < nb; i += NT) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += NT) {
      const unsigned long long k = keys[i];
      if (k >= L && k <= H) atomicAdd(&hist[(int)((k - L) >> shift)], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      const int need = sh->need;
      uint32_t ls = 0;
      for (int i = 0; i < 32; ++i) { int bb = lane * 32 + i; if (bb < nb) ls += hist[bb]; }
      uint32_t suf = ls;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t t = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += t;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, suf >= (uint32_t)need);
      const int lstar = ball ? 31 - __clz((int)ball) : 0;
      const uint32_t above0 = __shfl_sync(0xffffffffu, suf - ls, lstar);
      if (lane == lstar) {
        uint32_t cum = above0;
        int bs = lane * 32, ab = (int)above0, bc = 0;
        for (int i = 31; i >= 0; --i) {
          int bb = lane * 32 + i;
          if (bb >= nb) continue;
          if (cum + hist[bb] >= (uint32_t)need) { bs = bb; ab = (int)cum; bc = (int)hist[bb]; break; }
          cum += hist[bb];
        }
        sh->bstar = bs; sh->above = ab; sh->binc = bc;
        const unsigned long long nlo = L + ((unsigned long long)bs << shift);
        const int nneed = need - ab;
        if (bc == nneed || shift == 0) {
          sh->thr = nlo; sh->done = 1;
        } else {
          unsigned long long nhi = nlo + ((1ull << shift) - 1ull);
          sh->lo = nlo; sh->hi = nhi < H ? nhi : H; sh->need = nneed;
        }
      }
    }
    __syncthreads();
    if (sh->done) break;
  }
  if (!sh->done) { if (tid == 0) { sh->thr = sh->lo; dev_flag(HOKV_ERR_TIMEOUT); } }
  __syncthreads();
  const unsigned long long thr = sh->thr;
  constexpr int PER = K7_CAP / NT;
  unsigned long long mine[PER];
  bool take[PER];
#pragma unroll
  for (int r = 0; r < PER; ++r) {
    const int i = tid + r * NT;
    take[r] = false;
    mine[r] = 0ull;
    if (i < n) { mine[r] = keys[i]; take[r] = mine[r] >= thr; }
  }
  if (tid == 0) sh->n_out = 0;
  __syncthreads();
#pragma unroll
  for (int r = 0; r < PER; ++r) {
    if (take[r]) {
      int slot = atomicAdd(&sh->n_out, 1);
      if (slot < m) keys[slot] = mine[r];
    }
  }
  __syncthreads();
}

template <int D>
struct AttnGeo {
  static constexpr int DPL = (D <= 128) ? 4 : D / 32;   // dims per lane
  static constexpr int LPT = D / DPL;                    // lanes per token
  static constexpr int SUB = 32 / LPT;                   // tokens per warp step
};

template <typename KVT, int DPL>
__device__ __forceinline__ void load_row(const KVT* p, float (&o)[DPL]) {
#pragma unroll
  for (int i = 0; i < DPL; i += 4) {
    float4 f = load4<KVT>(p + i);
    o[i] = f.x; o[i + 1] = f.y; o[i + 2] = f.z; o[i + 3] = f.w;
  }
}

template <int D, typename KVT>
__global__ void __launch_bounds__(K7_THREADS) k7_select_attend(Cdc03P p) {
  using A = AttnGeo<D>;
  constexpr int NW = K7_THREADS / 32;
  constexpr int U = 4;
  extern __shared__ __align__(16) unsigned char smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);                        // [K7_CAP]
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + K7_CAP * 8);           // [1024]
  int* sel = reinterpret_cast<int*>(smem + K7_CAP * 8 + 4096);               // [TOPK_MAX]
  float* part = reinterpret_cast<float*>(smem + K7_CAP * 8 + 4096 + TOPK_MAX * 4);  // [NW][D + 2]
  float* T = part + NW * (D + 2);                                            // [M][256]
  __shared__ float s_q[D];
  __shared__ int s_n;
  __shared__ SelShared s_sel;

  const int Hq = p.Hkv * p.G;
  const int u = blockIdx.x / p.G, g = blockIdx.x - (blockIdx.x / p.G) * p.G;
  const int b = u / p.Hkv, h = u - b * p.Hkv;
  const int hq = h * p.G + g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ColdRange cr = cold_range(p, b);

  for (int d = tid; d < D; d += K7_THREADS)
    s_q[d] = load_as_f32(p.q, p.q_dtype, (int64_t)b * p.q_sb + (int64_t)hq * D + d);
  if (tid == 0) s_n = 0;
  __syncthreads();

  // ---- which cold tokens are attended --------------------------------------
  int n_sel;
  bool explicit_sel = false;
  if (cr.k >= cr.Sc) {
    n_sel = cr.Sc;
  } else if (cr.kp <= 0) {
    n_sel = cr.sink;
  } else {
    explicit_sel = true;
    const int M = p.M, sd = p.sd;
    const float* cbase = p.cb + (int64_t)b * p.cb_sb + (int64_t)h * p.cb_sh;
    const int* kbase = p.cbk + (int64_t)b * p.cbk_sb + (int64_t)h * p.cbk_sh;
    for (int i = tid; i < M * 256; i += K7_THREADS) {
      const int s = i >> 8, j = i & 255;
      int ks = kbase[s];
      ks = ks < 0 ? 0 : (ks > p.slots ? p.slots : ks);
      T[i] = (j < ks) ? dot_order(p.lut_order, s_q + s * sd, cbase + ((int64_t)s * p.slots + j) * sd, sd) : 0.f;
    }
    __syncthreads();
    const uint8_t* codes = p.codes + (int64_t)b * p.c_sb + (int64_t)h * p.c_sh;
    const float scale = p.scale;
    for (int c = 0; c < p.n_chunks; ++c) {
      const int clo = max(c * p.chunk, cr.sink), chi = min((c + 1) * p.chunk, cr.Sc);
      if (clo >= chi) continue;
      const int cnt = p.cand_cnt[((int64_t)u * p.n_chunks + c) * p.GT + g];
      const uint32_t* cl = p.cand_idx + (((int64_t)u * p.n_chunks + c) * p.GT + g) * CAND_MAX;
      const int ntok = (cnt >= 0) ? min(cnt, CAND_MAX) : (chi - clo);
      for (int base = 0; base < ntok; base += K7_THREADS) {
        if (s_n + K7_THREADS > K7_CAP) {
          select_topm<K7_THREADS>(keys, s_n, cr.kp, hist, &s_sel);
          if (tid == 0) s_n = min(s_n, cr.kp);
          __syncthreads();
        }
        const int i = base + tid;
        if (i < ntok) {
          const int t = (cnt >= 0) ? (int)cl[i] : clo + i;
          const uint8_t* row = codes + (int64_t)t * p.CS;
          float sum = 0.f;
          for (int s = 0; s < M; ++s) sum = fadd(sum, T[s * 256 + row[s]]);
          const float sc = fmul(sum, scale);
          const int slot = atomicAdd(&s_n, 1);
          keys[slot] = sel_key(sc, (uint32_t)t);
        }
        __syncthreads();
      }
    }
    const int n = s_n;
    if (n > cr.kp) select_topm<K7_THREADS>(keys, n, cr.kp, hist, &s_sel);
    const int m = min(n, cr.kp);
    for (int i = tid; i < cr.sink; i += K7_THREADS) sel[i] = i;
    for (int i = tid; i < m; i += K7_THREADS) sel[cr.sink + i] = (int)key_idx(keys[i]);
    n_sel = cr.sink + m;
    __syncthreads();
  }

  // ---- exact attention over selected cold tokens + hot window ---------------
  const int n_hot = cr.S - cr.Sc;
  const int n_tot = n_sel + n_hot;
  const KVT* kb = reinterpret_cast<const KVT*>(p.k) + (int64_t)b * p.kv_sb + (int64_t)h * p.kv_sh;
  const KVT* vb = reinterpret_cast<const KVT*>(p.v) + (int64_t)b * p.kv_sb + (int64_t)h * p.kv_sh;
  const int sub = lane / A::LPT, sl = lane - sub * A::LPT;
  float qv[A::DPL];
#pragma unroll
  for (int i = 0; i < A::DPL; ++i) qv[i] = s_q[sl * A::DPL + i];
  float m_run = -INFINITY, l_run = 0.f, acc[A::DPL];
#pragma unroll
  for (int i = 0; i < A::DPL; ++i) acc[i] = 0.f;
  const bool want_scores = p.sel_score != nullptr;
  const int sel_cap = max(p.top_k, p.sink);   // sinks are kept even when top_k < sink_tokens
  const int64_t sel_base = ((int64_t)b * Hq + hq) * sel_cap;
  constexpr int STEP = NW * A::SUB * U;
  for (int ib = warp * A::SUB * U; ib < n_tot; ib += STEP) {
    float kf[U][A::DPL], vf[U][A::DPL];
    bool valid[U];
#pragma unroll
    for (int r = 0; r < U; ++r) {
      const int i = ib + r * A::SUB + sub;
      valid[r] = i < n_tot;
      if (valid[r]) {
        const int t = (i < n_sel) ? (explicit_sel ? sel[i] : i) : (cr.Sc + (i - n_sel));
        load_row<KVT, A::DPL>(kb + (int64_t)t * D + sl * A::DPL, kf[r]);
        load_row<KVT, A::DPL>(vb + (int64_t)t * D + sl * A::DPL, vf[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < U; ++r) {
      float s = 0.f;
      if (valid[r]) {
#pragma unroll
        for (int i = 0; i < A::DPL; ++i) s = fmaf(qv[i], kf[r][i], s);
      }
#pragma unroll
      for (int o = A::LPT / 2; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (valid[r]) {
        s *= p.scale;
        const int i = ib + r * A::SUB + sub;
        if (want_scores && sl == 0 && i < n_sel && i < sel_cap) p.sel_score[sel_base + i] = s;
        const float mn = fmaxf(m_run, s);
        const float corr = __expf(m_run - mn);
        const float pe = __expf(s - mn);
        l_run = l_run * corr + pe;
#pragma unroll
        for (int d = 0; d < A::DPL; ++d) acc[d] = acc[d] * corr + pe * vf[r][d];
        m_run = mn;
      }
    }
  }
  // combine the SUB token groups of this warp
#pragma unroll
  for (int o = A::LPT; o < 32; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m_run, o);
    const float lo = __shfl_xor_sync(0xffffffffu, l_run, o);
    const float mn = fmaxf(m_run, mo);
    const float a = (m_run == -INFINITY) ? 0.f : __expf(m_run - mn);
    const float c = (mo == -INFINITY) ? 0.f : __expf(mo - mn);
    l_run = l_run * a + lo * c;
#pragma unroll
    for (int d = 0; d < A::DPL; ++d) {
      const float ao = __shfl_xor_sync(0xffffffffu, acc[d], o);
      acc[d] = acc[d] * a + ao * c;
    }
    m_run = mn;
  }
  float* pw = part + warp * (D + 2);
  if (sub == 0) {
#pragma unroll
    for (int d = 0; d < A::DPL; ++d) pw[sl * A::DPL + d] = acc[d];
    if (sl == 0) { pw[D] = m_run; pw[D + 1] = l_run; }
  }
  __syncthreads();
  for (int d = tid; d < D; d += K7_THREADS) {
    float M_ = -INFINITY;
    for (int w = 0; w < NW; ++w) M_ = fmaxf(M_, part[w * (D + 2) + D]);
    float num = 0.f, den = 0.f;
    if (M_ != -INFINITY) {
      for (int w = 0; w < NW; ++w) {
        const float mw = part[w * (D + 2) + D];
        if (mw == -INFINITY) continue;
        const float f = __expf(mw - M_);
        num += part[w * (D + 2) + d] * f;
        den += part[w * (D + 2) + D + 1] * f;
      }
    }
    const float o = den > 0.f ? num / den : 0.f;
    store_from_f32(p.out, p.out_dtype, (int64_t)b * p.out_sb + (int64_t)hq * D + d, o);
  }
  if (p.sel_idx) {
    for (int i = tid; i < sel_cap; i += K7_THREADS) {
      int t = -1;
      if (i < n_sel) t = explicit_sel ? sel[i] : i;
      p.sel_idx[sel_base + i] = t;
      if (want_scores && i >= n_sel) p.sel_score[sel_base + i] = -INFINITY;
    }
  }
  if (p.sel_count && tid == 0) p.sel_count[(int64_t)b * Hq + hq] = n_sel;
}

// ---------------------------------------------------------------------------
// Sub-tables for the API (ProductCodebook.precompute_distance_tables).
// grid (n_q, M), block 256: one (query, subspace) row of t_cols entries.
// ---------------------------------------------------------------------------
__global__ void k_pq_tables(const float* __restrict__ q, int M, int sd, const float* __restrict__ cents,
                            int slots, int64_t cent_set_stride, const int* __restrict__ k, int64_t k_set_stride,
                            const int* __restrict__ set_of_q, float* __restrict__ tables, int t_cols, int order) {
  const int i = blockIdx.x, s = blockIdx.y;
  const int set = set_of_q ? set_of_q[i] : i;
  const float* qs = q + (int64_t)i * M * sd + s * sd;
  int ks = k[(int64_t)set * k_set_stride + s];
  ks = ks < 0 ? 0 : (ks > slots ? slots : ks);
  const float* cb = cents + (int64_t)set * cent_set_stride + (int64_t)s * slots * sd;
  float* out = tables + ((int64_t)i * M + s) * t_cols;
  for (int j = threadIdx.x; j < t_cols; j += blockDim.x)
    out[j] = (j < ks) ? dot_order(order, qs, cb + (int64_t)j * sd, sd) : 0.f;
}

// ProductCodebook.gather_pq_scores: ((0 + T0[c0]) + T1[c1]) + ... [* scale]
__global__ void k_pq_gather(const float* __restrict__ tables, int M, int t_cols, const uint8_t* __restrict__ codes,
                            int64_t n, int64_t row_stride, int apply_scale, float scale, float* __restrict__ out) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* r = codes + t * row_stride;
    float acc = 0.f;
    for (int s = 0; s < M; ++s) {
      int j = r[s];
      if (j >= t_cols) { dev_flag(HOKV_ERR_DEVICE_INPUT); j = 0; }
      acc = fadd(acc, tables[s * t_cols + j]);
    }
    out[t] = apply_scale ? fmul(acc, scale) : acc;
  }
}

// ---------------------------------------------------------------------------
// K8 Path A fused Q.K^T over scalar-VQ codes (triton_attention.py:25-120).
// The 256-entry codebook is held 32 times in shared memory, copy L at bank L,
// so lane L's lookups never conflict whatever the indices are.
// ---------------------------------------------------------------------------
template <typename IT, typename ACC>
__global__ void __launch_bounds__(256) k_scalar_vq_qkt(const float* __restrict__ q, const IT* __restrict__ idx,
                                                       int64_t S, int D, int64_t stride, const float* __restrict__ cbk,
                                                       int k, float scale, float* __restrict__ scores) {
  __shared__ float rep[256 * 32];
  extern __shared__ float sq[];
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
    const int j = i >> 5;
    rep[i] = (j < k) ? cbk[j] : 0.f;
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) sq[d] = q[d];
  __syncthreads();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= S) return;
  const IT* row = idx + t * stride;
  ACC acc = 0;
  for (int d = 0; d < D; ++d) {
    int j = (int)row[d];
    if (j < 0 || j >= 256) { dev_flag(HOKV_ERR_DEVICE_INPUT); j = 0; }
    acc += (ACC)sq[d] * (ACC)rep[j * 32 + lane];
  }
  scores[t] = (float)(acc * (ACC)scale);
}

}  // namespace hokv
