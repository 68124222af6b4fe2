// cdc03.cuh -- PQ lookup tables, ADC scoring and CDC-03 decode attention.
//
// Decode step, per layer, two kernels chained with programmatic dependent
// launch (K7 starts its hot-window attention while K6 runs):
//   K6 k6_candidates  grid (min(chunks, 8), B*H_kv), one thread-block cluster
//      per (sequence, KV head): the CTAs build the exact fp32 sub-tables
//      T[g][s][j] = q_g[s-slice] . C_s[j] of the G query heads of the GQA
//      group (BLAS order) and their quantised image (codes of floor(65535 / M)
//      levels in 16-bit lanes, laid out so every shared-memory lookup is bank
//      conflict free); each CTA streams the uint8 PQ codes of its 2048-token
//      chunks into registers, sums quantised entries per token in integer
//      lanes, pools a score histogram over the cluster, and emits every token
//      whose score lies within the proven error band of the unit's k'-th
//      score, rescored exactly (reference summation order) into a selection key.
//   K7 k7_select_attend  grid (B*H_kv*G): attends the hot window before it
//      waits for K6, selects sinks + top-(k - sinks) of the candidate keys
//      (ties to the lower token index) and finishes softmax attention over them.
//
// Reference: helix_online_kv/compressed_attention.py:315-412 (hybrid_pq_attention),
// product_codebook.py:172-227 (tables, gather).
#pragma once
#include "hokv_common.cuh"
#include <cooperative_groups.h>
#include <climits>
#include <type_traits>

namespace hokv {

constexpr int K6_THREADS = 256;
constexpr int K6_FIRST_ROWS = 128;  // codebook rows per subspace staged before the live counts are read

constexpr int CAND_MAX = 512;        // candidates per (unit, chunk, head)
constexpr int K7_THREADS = 256;
constexpr int K7_CAP = 1024;         // key buffer of the exact selection (rank counting)
constexpr int TOPK_MAX = 1024;       // largest top_k with k < S_c
// K6 chunks per (sequence, KV head): a CTA then scores at most 31 chunks, so
// none of its 16-bit histogram counters can exceed 31 x 2048 = 63,488
// (507,904 cold tokens per sequence)
constexpr int MAX_CHUNKS = 248;

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
  // workspace
  uint64_t* cand_key;     // [units][chunks][GT][CAND_MAX] selection keys of listed candidates (K6 -> K7)
  int* cand_cnt;          // [units][chunks][GT]   listed count, -1 when the list overflowed
  unsigned char* qimg;    // [units][qimg_bytes]     quantised sub-table images (exchanged in the cluster)
  float* texact;          // [units][GT][CS][256]    exact sub-tables (K6 rescoring, K7 rescans)
  int* margin;            // [units][GT]             error band in code units
  int n_chunks, chunk, GT, qimg_bytes;
  int kv_es;              // bytes per K/V element
};

// Per-sequence geometry of the cold range, identical in all three kernels.
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

// ---- async copies and programmatic dependent launch ------------------------
// Hint: bring the 16-byte-aligned interior of [base + off, base + off + nbytes)
// into L2 with one bulk prefetch (nothing happens when it is empty).
__device__ __forceinline__ void prefetch_l2(const void* base, int64_t off, int64_t nbytes) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(base) + (uintptr_t)off;
  const uintptr_t lo = (a0 + 15) & ~(uintptr_t)15, hi = (a0 + (uintptr_t)nbytes) & ~(uintptr_t)15;
  if (nbytes > 0 && hi > lo)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((uint32_t)(hi - lo)) : "memory");
}

// Hint: the 128-byte lines of [base + off, base + off + nbytes) into L2, one
// prefetch instruction a line (cheap to issue from many threads; the bulk
// prefetch above goes through the CTA's asynchronous copy unit, one at a time).
__device__ __forceinline__ void prefetch_lines_l2(const void* base, int64_t off, int64_t nbytes) {
  const char* a = static_cast<const char*>(base) + off;
  for (int64_t o = 0; o < nbytes; o += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(a + o));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
// Let the next kernel in the stream start its independent prologue now.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
// Block until the previous kernel in the stream has completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// ---------------------------------------------------------------------------
// Quantised sub-table geometry.  One entry holds the codes of the GT query
// heads for one (subspace s, centroid j) in 16-bit lanes: GT <= 2 -> 4 bytes,
// GT = 4 -> 8 bytes {h0|h2, h1|h3}, GT = 8 -> 16 bytes.  Rows are 128 B (one
// shared-memory wavefront of COLS lanes).  Lane L at step u reads subspace
// (u + L) mod CS; each row holds copies (or row blocks) placed so that the
// lanes of one wavefront always hit distinct columns, whatever the codes are.
// ---------------------------------------------------------------------------
template <int CS, int GT>
struct QGeo {
  static constexpr int EW = (GT <= 2) ? 4 : (GT == 4 ? 8 : 16);
  static constexpr int COLS = 128 / EW;
  static constexpr int RB = (CS > COLS) ? CS / COLS : 1;
  static constexpr int NC = (CS < COLS) ? COLS / CS : 1;
  static constexpr int BYTES = RB * 256 * 128;
  static constexpr int NACC = (GT == 8) ? 4 : (GT == 4 ? 2 : 1);
  static constexpr int W = CS / 4;
  __host__ __device__ static constexpr int col_of(int lane, int s) {
    return (CS <= COLS) ? (((lane % COLS) / CS) * CS + s) : (s % COLS);
  }
  __host__ __device__ static constexpr int rb_of(int s) { return (CS <= COLS) ? 0 : s / COLS; }
};

__host__ __device__ __forceinline__ int qmax_for(int M) { return 65535 / M; }

template <int GT>
__device__ __forceinline__ int approx_of(const uint32_t* acc, int g) {
  // packing: acc[0] = h0 | h2 << 16, acc[1] = h1 | h3 << 16, acc[2] = h4 | h6 << 16, acc[3] = h5 | h7 << 16
  if constexpr (GT == 1) return (int)acc[0];
  else if constexpr (GT == 2) return (int)(g == 0 ? (acc[0] & 0xffffu) : (acc[0] >> 16));
  else {
    const uint32_t a = acc[(g >> 2) * 2 + (g & 1)];
    return (int)((g & 2) ? (a >> 16) : (a & 0xffffu));
  }
}

template <int W>
__device__ __forceinline__ void load_code(const uint8_t* p, uint32_t (&w)[W]) {
  if constexpr (W == 1) {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else if constexpr (W == 2) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (W == 4) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(p) + 1);
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

// Exact sub-table entry: the GEMV order of NumPy/OpenBLAS for (1 x SD) @ (SD x k)
// (hokv_math.cuh dot_gemv), so the value equals the reference's bit for bit;
// the paired products and sums of the 4- and 8-dim orders run as fp32x2
// operations, which round each lane as its scalar twin does.
template <int SD>
__device__ __forceinline__ float lut_dot(const float* q, const float* c) {
  if constexpr (SD == 4) {
    const float2 a = __fmul2_rn(make_float2(q[0], q[2]), make_float2(c[0], c[2]));
    const float2 b = __fmul2_rn(make_float2(q[1], q[3]), make_float2(c[1], c[3]));
    const float2 s = __fadd2_rn(a, b);   // {p0 + p1, p2 + p3}
    return fadd(s.x, s.y);
  } else if constexpr (SD == 8) {
    float2 pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = __fmul2_rn(make_float2(q[i], q[i + 4]), make_float2(c[i], c[i + 4]));
    const float2 s = __fadd2_rn(__fadd2_rn(pr[0], pr[1]), __fadd2_rn(pr[2], pr[3]));
    return fadd(s.x, s.y);   // ((p0+p1)+(p2+p3)) + ((p4+p5)+(p6+p7))
  } else {
    return dot_gemv(q, c, SD);
  }
}

// Quantisation of one head's tables from the per-subspace ranges [lo, hi]
// (0 included where a subspace has fewer than 256 centroids): a common step
// delta = max range / qmax, and the error band, in code units, that covers
// entry rounding (<= 0.5 + fp32 slop) for both tokens of a comparison, the
// fp32 summation error of the exact scores and ties created by the final
// scale multiply.  A margin of 2^30 marks a scale that cannot rank.
struct QuantScale {
  float inv;
  int margin;
};
// The step and band computed by one warp: lane s takes subspace s (and
// s + 32); the largest range and the sum sa of max(|lo|, |hi|) are warp
// reductions.  The band is
//   margin = ceil(M * 1.0002 + (M + 1) 2^-22 sa / delta),  delta = rmax / qmax,
// evaluated in fp32 with every rounding pushed upward (sa, the quotient and
// the sum each scaled by 1 + 2^-20, more than the relative error of the
// at most 7 fp32 additions and 4 products and quotients behind them), so the
// margin is never below the exact value of the formula; at worst it is one
// code unit wider, which admits a few more candidates and changes no
// selection.  A band past 2^30, or a scale that cannot rank, gives 2^30.
// Every lane returns the result.
__device__ __forceinline__ QuantScale quant_scale_warp(const float* lo, const float* hi, int M, float scale,
                                                       int lane) {
  const int qmax = qmax_for(M);
  float rmax = 0.f, sa = 0.f;
  for (int s = lane; s < M; s += 32) {
    rmax = fmaxf(rmax, hi[s] - lo[s]);
    sa += fmaxf(fabsf(lo[s]), fabsf(hi[s]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
  }
  constexpr float UP = 1.f + 0x1p-20f;
  const float sa_up = sa * UP;
  float e_f = (float)(M + 1) * 0x1p-22f * sa_up;
  if (rmax > 0.f) e_f = e_f * (float)qmax / rmax * UP;   // / delta
  const float band = ((float)M * 1.0002f + e_f) * UP;
  const bool ok_scale = (scale > 0.f) && isfinite(scale) && isfinite(sa) && band < 1.0e9f;
  QuantScale r;
  r.inv = rmax > 0.f ? (float)qmax / rmax : 0.f;
  r.margin = ok_scale ? (int)ceilf(band) : (1 << 30);
  return r;
}

__device__ __forceinline__ uint16_t quant_code(float t, float lo, float inv, int qmax) {
  float x = __fmul_rn(__fsub_rn(t, lo), inv);
  x = fminf(fmaxf(rintf(x), 0.f), (float)qmax);
  return (uint16_t)x;
}

// ===========================================================================
// K6: candidate stream, grid (min(chunks, 8), B*H_kv), 256 threads, 8 tokens
// of a 2048-token chunk per thread.  The CTAs of one (b, KV head) form a
// thread-block cluster that builds the unit's tables itself (each CTA one
// block of subspaces; ranges exchanged through distributed shared memory, the
// quantised image through L2) and pools its score histograms, so the
// threshold is the unit-wide k'-th score at any context length.
// ===========================================================================
constexpr int K6_TPT = 8;
constexpr int K6_CHUNK = K6_THREADS * K6_TPT;   // 2048 tokens
constexpr int K6_CLUSTER_MAX = 8;
constexpr int HBINS = 1024;                      // score histogram bins per head
constexpr int HWORDS = HBINS / 2;                // two 16-bit counters per word
constexpr int HSHIFT = 6;                        // bin = approx >> 6 (approx <= 65535)

// Cluster barrier halves (every thread of every CTA of the cluster arrives,
// then waits, once per phase).  `arrive` releases this thread's earlier
// shared and global writes to the cluster; `wait` acquires them.
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

// Per-lane coarse counts of one CTA's packed histograms: coarse[g * 32 + L] =
// items of head g in bins [32L, 32L + 32) (words [16L, 16L + 16)).  Threads
// [0, GT * 32); lane L's 16 words as four 16-byte loads, rotated by lane so
// that a quarter warp spreads over the bank groups.
template <int GT>
__device__ __forceinline__ void coarse_counts(const uint32_t* hist, uint32_t* coarse) {
  static_assert(HWORDS == 512, "32 lanes x 16 words");
  const int i = threadIdx.x;
  if (i >= GT * 32) return;
  const int g = i >> 5, lane = i & 31;
  const uint4* h4 = reinterpret_cast<const uint4*>(hist + g * HWORDS);
  uint32_t ls = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 v = h4[lane * 4 + ((k + lane) & 3)];
    ls += (v.x & 0xffffu) + (v.x >> 16) + (v.y & 0xffffu) + (v.y >> 16) + (v.z & 0xffffu) + (v.z >> 16) +
          (v.w & 0xffffu) + (v.w >> 16);
  }
  coarse[i] = ls;
}

// Largest bin b of head g's histogram pooled over the R CTAs of the cluster
// (HWORDS words per CTA, bin 2i in the low half of word i) such that at least
// kp items lie in bins >= b; -1 if the cluster holds fewer than kp items.  One
// warp, reading the other CTAs' shared memory: first the R coarse counts of
// each lane's 32 bins, then the R copies of the 16 words of the lane range
// that holds b.  Counts are summed in 32 bits (no saturation).  The caller
// has made every CTA's `hist` and `coarse` visible (cluster barrier) and
// keeps them unchanged until every CTA has passed this call (the next).
__device__ __forceinline__ int top_bin_cluster(const uint32_t* hist_g, const uint32_t* coarse_g, uint32_t kp,
                                               int lane, int R) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  uint32_t ls = 0;
#pragma unroll
  for (int rk = 0; rk < K6_CLUSTER_MAX; ++rk)
    if (rk < R) ls += cl.map_shared_rank(const_cast<uint32_t*>(coarse_g), (unsigned)rk)[lane];
  uint32_t suf = ls;   // items in lanes >= this one's bins
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += t;
  }
  const unsigned ball = __ballot_sync(0xffffffffu, suf >= kp);
  if (ball == 0u) return -1;
  const int lstar = 31 - __clz((int)ball);
  // inside lane lstar's 32 bins: lane j takes bin 32 * lstar + j (bin 2i is the
  // low half of word i), and the warp finds the highest j whose suffix count,
  // with the items above the range, still reaches kp
  const uint32_t above = __shfl_sync(0xffffffffu, suf - ls, lstar);
  uint32_t c = 0;
#pragma unroll
  for (int rk = 0; rk < K6_CLUSTER_MAX; ++rk) {
    if (rk < R) {
      const uint32_t w = cl.map_shared_rank(const_cast<uint32_t*>(hist_g), (unsigned)rk)[lstar * 16 + (lane >> 1)];
      c += (lane & 1) ? (w >> 16) : (w & 0xffffu);
    }
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(0xffffffffu, c, o);
    if (lane + o < 32) c += t;
  }
  const unsigned b2 = __ballot_sync(0xffffffffu, above + c >= kp);
  return lstar * 32 + (31 - __clz((int)b2));
}

// Resident CTAs per SM: 4 (64 registers) unless the score lanes need more.
template <int CS, int GT>
constexpr int k6_min_blocks() { return ((GT == 8 && CS >= 16) || (CS == 32 && GT >= 4)) ? 3 : 4; }

// Dot phase of the in-cluster table build: thread j computes entry j of the
// subspaces [s_begin, s_end) for the GT query heads of the group, stores the
// exact fp32 value (for the exact rescoring), folds it into the
// per-(head, subspace) range and keeps the first two subspaces' values in
// registers for the quantisation.  Row (s, j) of the codebook is at
// rows + ((s - s_off) * slots + j) * SD.
template <int GT, int SD>
__device__ __forceinline__ void lut_dot_row(const Cdc03P& p, int u, const float* rows, int s_off, const float* sq,
                                            const int* s_k, int s, unsigned (*s_lo)[32], unsigned (*s_hi)[32],
                                            float (&tv)[GT]) {
  const int j = threadIdx.x, lane = j & 31;
  const bool live = j < s_k[s];
  float c[SD];
  const float* row = rows + ((int64_t)(s - s_off) * p.slots + j) * SD;
#pragma unroll
  for (int d = 0; d < SD; ++d) c[d] = live ? row[d] : 0.f;
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    const float t = live ? lut_dot<SD>(sq + g * p.D + s * SD, c) : 0.f;
    tv[g] = t;
    p.texact[(((int64_t)u * GT + g) * p.CS + s) * 256 + j] = t;
    const unsigned o = ord_f32(t);
    const unsigned mn = __reduce_min_sync(0xffffffffu, o), mx = __reduce_max_sync(0xffffffffu, o);
    if (lane == 0) { atomicMin(&s_lo[g][s], mn); atomicMax(&s_hi[g][s], mx); }
  }
}

template <int GT, int SD>
__device__ __forceinline__ void lut_dots(const Cdc03P& p, int u, const float* rows, int s_off, const float* sq,
                                         const int* s_k, int s_begin, int s_end, unsigned (*s_lo)[32],
                                         unsigned (*s_hi)[32], float (&tv)[2][GT]) {
  if (s_begin < s_end) lut_dot_row<GT, SD>(p, u, rows, s_off, sq, s_k, s_begin, s_lo, s_hi, tv[0]);
  if (s_begin + 1 < s_end) lut_dot_row<GT, SD>(p, u, rows, s_off, sq, s_k, s_begin + 1, s_lo, s_hi, tv[1]);
  for (int s = s_begin + 2; s < s_end; ++s) {
    float tmp[GT];
    lut_dot_row<GT, SD>(p, u, rows, s_off, sq, s_k, s, s_lo, s_hi, tmp);
  }
}

// Quantised entry (EW bytes, GT 16-bit lanes) of subspace sx, row j, into the
// unit's image in global memory, every copy of the column.
// 16-bit lane of head g: GT <= 2 -> u32 lane g; GT = 4 -> {h0|h2, h1|h3};
// GT = 8 -> {h0|h2, h1|h3, h4|h6, h5|h7}.
template <int CS, int GT>
__device__ __forceinline__ void put_entry(unsigned char* img, int sx, int j, const uint32_t* code) {
  using Q = QGeo<CS, GT>;
  uint32_t e32[Q::EW / 4];
#pragma unroll
  for (int i = 0; i < Q::EW / 4; ++i) e32[i] = 0u;
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    const int l16 = (GT <= 2) ? g : ((g >> 2) * 4 + (g & 1) * 2 + ((g & 2) >> 1));
    e32[l16 >> 1] |= code[g] << (16 * (l16 & 1));
  }
  for (int copy = 0; copy < Q::NC; ++copy) {
    const int e = (Q::rb_of(sx) * 256 + j) * Q::COLS + copy * CS + (sx % Q::COLS);
    if constexpr (Q::EW == 4) reinterpret_cast<uint32_t*>(img)[e] = e32[0];
    else if constexpr (Q::EW == 8) reinterpret_cast<uint2*>(img)[e] = make_uint2(e32[0], e32[1]);
    else reinterpret_cast<uint4*>(img)[e] = make_uint4(e32[0], e32[1], e32[2], e32[3]);
  }
}

// Chunk c of the unit is handled by CTA c % R of the cluster (R <= 8).  With
// one chunk per CTA its scores stay in registers between the histogram and the
// candidate list; with more (long contexts) the CTA scores its chunks twice:
// once for the histogram, once, after the unit-wide threshold, for the list.
template <int CS, int GT>
__global__ void __launch_bounds__(K6_THREADS, k6_min_blocks<CS, GT>()) k6_candidates(Cdc03P p) {
  using Q = QGeo<CS, GT>;
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* qlut = smem;                                              // Q::BYTES
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + Q::BYTES);           // [GT][HWORDS]
  uint32_t* coarse = hist + GT * HWORDS;                                   // [GT][32] per-lane counts
  __shared__ int s_margin[GT], s_thr[GT], s_cnt[GT], s_nl[GT];

  pdl_launch_dependents();
  const int scta = blockIdx.y * gridDim.x + blockIdx.x;   // phase-stamp slot (profiling build)
  stamp(0, scta, 0);
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int R = (int)cl.num_blocks(), me = (int)cl.block_rank();
  const int u = blockIdx.y;
  const int b = u / p.Hkv, h = u - b * p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ColdRange cr = cold_range(p, b);
  const int n_mine = (p.n_chunks - me + R - 1) / R;   // chunks me, me + R, ...
  if (cr.k >= cr.Sc || cr.kp <= 0) {      // the same for every CTA of the unit
    for (int i = 0; i < n_mine; ++i)
      if (tid < GT) p.cand_cnt[((int64_t)u * p.n_chunks + me + i * R) * GT + tid] = 0;
    return;
  }
  const int M = p.M;
  const uint8_t* gcodes = p.codes + (int64_t)b * p.c_sb + (int64_t)h * p.c_sh;
  constexpr int HT = K6_TPT / 2;
  uint32_t w[HT][Q::W];
  const int c0 = me;
  {
    // ---- tables built by the cluster: each CTA computes a block of subspaces
    // (whole 16-byte groups of the image), the ranges go to every CTA through
    // distributed shared memory, the quantised entries to the unit's image in
    // global memory, from where every CTA loads the whole image
    __shared__ unsigned s_lo[GT][32], s_hi[GT][32];
    __shared__ float f_lo[GT][32], f_hi[GT][32], s_inv[GT];
    __shared__ int s_k[32];
    cluster_arrive_relaxed();   // phase A: this CTA runs
    constexpr int GS = 16 / Q::EW;                 // subspaces per 16-byte group
    const int ngm = (M + GS - 1) / GS;             // groups holding real subspaces
    const int grp0 = me * ngm / R, grp1 = (me + 1) * ngm / R;
    const int s_begin = grp0 * GS, s_end = min(grp1 * GS, M);
    const float* cbase = p.cb + (int64_t)b * p.cb_sb + (int64_t)h * p.cb_sh;
    // own codebook rows into shared memory (the image space is free until the
    // image is loaded), with the queries: the first K6_FIRST_ROWS rows of each
    // subspace now, the live rows past them (if any) once the counts are known
    const int64_t per_s = (int64_t)p.slots * p.sd;                           // floats per subspace
    const int64_t blk = (int64_t)max(0, s_end - s_begin) * per_s;
    const bool staged = blk * 4 <= Q::BYTES;
    const float* src = cbase + (int64_t)s_begin * per_s;
    const int first = min(p.slots, K6_FIRST_ROWS);
    const int row16 = p.sd / 4;                                              // 16-byte pieces per row
    if (staged) {   // 32-bit index math: a staged block holds at most Q::BYTES
      const int per_sub = first * row16;
      const int n16 = (s_end - s_begin) * per_sub;
      for (int i = tid; i < n16; i += K6_THREADS) {
        const int sr = i / per_sub;
        const int off = sr * (int)per_s + (i - sr * per_sub) * 4;
        cp_async16(qlut + off * 4, src + off);
      }
    }
    float* sq = reinterpret_cast<float*>(hist);   // [GT][D], dead before the histograms
    for (int i = tid; i < GT * p.D; i += K6_THREADS) {
      const int g = i / p.D, d = i - g * p.D;
      sq[i] = g < p.G ? load_as_f32(p.q, p.q_dtype, (int64_t)b * p.q_sb + (int64_t)(h * p.G + g) * p.D + d) : 0.f;
    }
    if (tid < M) {
      const int ks = p.cbk[(int64_t)b * p.cbk_sb + (int64_t)h * p.cbk_sh + tid];
      s_k[tid] = ks < 0 ? 0 : (ks > p.slots ? p.slots : ks);
    }
    if (tid < GT * 32) { s_lo[tid / 32][tid % 32] = 0xffffffffu; s_hi[tid / 32][tid % 32] = 0u; }
    cp_async_wait_all();
    __syncthreads();
    stamp(0, scta, 1);   // codebook rows and queries staged
    if (staged && p.slots > first) {
      bool more = false;   // the same in every thread: the counts are in shared memory
      for (int sx = s_begin; sx < s_end; ++sx) more |= s_k[sx] > first;
      if (more) {
        for (int sx = s_begin; sx < s_end; ++sx) {
          const int64_t base = (int64_t)(sx - s_begin) * per_s + (int64_t)first * p.sd;
          const int64_t n16 = (int64_t)max(0, s_k[sx] - first) * row16;
          for (int64_t i = tid; i < n16; i += K6_THREADS) cp_async16(qlut + (base + i * 4) * 4, src + base + i * 4);
        }
        cp_async_wait_all();
        __syncthreads();
      }
    }
    float tv[2][GT];
    const float* rows = staged ? reinterpret_cast<const float*>(qlut) : cbase;
    const int s_off = staged ? s_begin : 0;
    switch (p.sd) {
      case 4: lut_dots<GT, 4>(p, u, rows, s_off, sq, s_k, s_begin, s_end, s_lo, s_hi, tv); break;
      case 8: lut_dots<GT, 8>(p, u, rows, s_off, sq, s_k, s_begin, s_end, s_lo, s_hi, tv); break;
      case 16: lut_dots<GT, 16>(p, u, rows, s_off, sq, s_k, s_begin, s_end, s_lo, s_hi, tv); break;
      case 32: lut_dots<GT, 32>(p, u, rows, s_off, sq, s_k, s_begin, s_end, s_lo, s_hi, tv); break;
      default: dev_flag(HOKV_ERR_DEVICE_INPUT);
    }
    // this CTA's codes into L2 while the cluster exchanges and quantises the
    // tables (issued after the table reads, which are on the critical path):
    // one bulk prefetch per chunk from one thread, so the load/store pipe
    // stays free for the phases that follow (the 16-byte-aligned interior of
    // each chunk; a prefetch is only a hint)
    if (tid == 0) {
      for (int i = 0; i < n_mine; ++i) {
        const int t0 = (me + i * R) * K6_CHUNK;
        prefetch_l2(gcodes, (int64_t)t0 * CS, (int64_t)max(0, min(t0 + K6_CHUNK, cr.Sc) - t0) * CS);
      }
    }
    // the K and V rows k7 reads whatever the selection (the hot window and the
    // sink tokens) into L2 meanwhile, by the last CTA of the cluster
    if (tid == 32 && me == R - 1) {
      const int64_t rb = (int64_t)p.D * p.kv_es, base = ((int64_t)b * p.kv_sb + (int64_t)h * p.kv_sh) * p.kv_es;
      prefetch_l2(p.k, base + cr.Sc * rb, (int64_t)(cr.S - cr.Sc) * rb);
      prefetch_l2(p.v, base + cr.Sc * rb, (int64_t)(cr.S - cr.Sc) * rb);
      prefetch_l2(p.k, base, (int64_t)cr.sink * rb);
      prefetch_l2(p.v, base, (int64_t)cr.sink * rb);
    }
    __syncthreads();
    stamp(0, scta, 2);   // dots done
    cluster_wait();             // phase A: every CTA of the cluster runs
    if (tid < GT * 32) {        // own ranges into every CTA
      const int g = tid / 32, sx = tid % 32;
      if (sx >= s_begin && sx < s_end) {
        float lo = unord_f32(s_lo[g][sx]), hi = unord_f32(s_hi[g][sx]);
        if (s_k[sx] < 256) { lo = fminf(lo, 0.f); hi = fmaxf(hi, 0.f); }   // zero-padded entries
        for (int rk = 0; rk < R; ++rk) {
          cl.map_shared_rank(&f_lo[0][0], (unsigned)rk)[g * 32 + sx] = lo;
          cl.map_shared_rank(&f_hi[0][0], (unsigned)rk)[g * 32 + sx] = hi;
        }
      }
    }
    for (int i = tid; i < GT * HWORDS; i += K6_THREADS) hist[i] = 0;
    if (tid < GT) s_cnt[tid] = 0;
    cluster_arrive();
    cluster_wait();             // phase B: all ranges in every CTA
    stamp(0, scta, 3);   // ranges exchanged
    if (warp < GT) {   // one warp per head
      const QuantScale qs = quant_scale_warp(f_lo[warp], f_hi[warp], M, p.scale, lane);
      if (lane == 0) {
        s_inv[warp] = qs.inv;
        s_margin[warp] = qs.margin;
        if (me == 0) p.margin[(int64_t)u * GT + warp] = qs.margin;
      }
    }
    __syncthreads();
    stamp(0, scta, 4);   // quantisation step known
    unsigned char* gimg = p.qimg + (int64_t)u * p.qimg_bytes;
    {
      const int qmax = qmax_for(M), j = tid;
      uint32_t code[GT];
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int sx = s_begin + kk;
        if (sx < s_end) {
#pragma unroll
          for (int g = 0; g < GT; ++g) code[g] = quant_code(tv[kk][g], f_lo[g][sx], s_inv[g], qmax);
          put_entry<CS, GT>(gimg, sx, j, code);
        }
      }
      for (int sx = s_begin + 2; sx < s_end; ++sx) {
#pragma unroll
        for (int g = 0; g < GT; ++g)
          code[g] = quant_code(p.texact[(((int64_t)u * GT + g) * CS + sx) * 256 + j], f_lo[g][sx], s_inv[g], qmax);
        put_entry<CS, GT>(gimg, sx, j, code);
      }
      // padding subspaces [M, CS): zero entries, written by the owner of the
      // group (rank 0 for groups without a real subspace)
#pragma unroll
      for (int g = 0; g < GT; ++g) code[g] = 0u;
      for (int sx = M; sx < CS; ++sx) {
        const int grp = sx / GS;
        const int own = grp < ngm ? ((grp + 1) * R - 1) / ngm : 0;
        if (own == me) put_entry<CS, GT>(gimg, sx, j, code);
      }
    }
    stamp(0, scta, 5);   // own image entries written
    cluster_arrive();           // phase C: the image is complete in memory
#pragma unroll
    for (int it = 0; it < HT; ++it) {   // first codes of the first chunk meanwhile
      const int t = c0 * K6_CHUNK + it * K6_THREADS + tid;
      if (t < cr.Sc) load_code<Q::W>(gcodes + (int64_t)t * CS, w[it]);
      else {
#pragma unroll
        for (int i = 0; i < Q::W; ++i) w[it][i] = 0;
      }
    }
    cluster_wait();
    stamp(0, scta, 6);   // every CTA's image entries written
    for (int i = tid; i < Q::BYTES / 16; i += K6_THREADS) cp_async16(qlut + i * 16, gimg + (int64_t)i * 16);
    cp_async_wait_all();
    __syncthreads();
    stamp(0, scta, 7);   // image in shared memory
  }

  // ---- quantised scores of one chunk, kept in registers ----------------------
  const int r = lane % CS;
  int colidx[CS];
#pragma unroll
  for (int uu = 0; uu < CS; ++uu) {
    const int s = (uu + r) % CS;
    colidx[uu] = Q::rb_of(s) * 256 * Q::COLS + Q::col_of(lane, s);
  }
  uint32_t accs[K6_TPT][Q::NACC];
  auto load_half = [&](int t0, int half) {
#pragma unroll
    for (int it = 0; it < HT; ++it) {
      const int t = t0 + (half * HT + it) * K6_THREADS + tid;
      if (t < cr.Sc) load_code<Q::W>(gcodes + (int64_t)t * CS, w[it]);
      else {
#pragma unroll
        for (int i = 0; i < Q::W; ++i) w[it][i] = 0;
      }
    }
  };
  // scores of chunk c into accs (first half of its codes already in w when
  // preloaded); with to_hist every in-range score goes to the histograms
  auto score_chunk = [&](int c, bool preloaded, bool to_hist) {
    const int t0 = c * K6_CHUNK;
    const int lo_t = max(t0, cr.sink), hi_t = min(t0 + K6_CHUNK, cr.Sc);
    if (!preloaded) load_half(t0, 0);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      if (half == 1) load_half(t0, 1);
#pragma unroll
      for (int it = 0; it < HT; ++it) {
        const int ti = half * HT + it;
        const int t = t0 + ti * K6_THREADS + tid;
#pragma unroll
        for (int a = 0; a < Q::NACC; ++a) accs[ti][a] = 0;
        rotate_bytes<Q::W>(w[it], r);
#pragma unroll
        for (int uu = 0; uu < CS; ++uu) {
          const uint32_t byte = (w[it][uu >> 2] >> (8 * (uu & 3))) & 0xffu;
          const int e = colidx[uu] + (int)byte * Q::COLS;
          if constexpr (Q::EW == 4) {
            accs[ti][0] += reinterpret_cast<const uint32_t*>(qlut)[e];
          } else if constexpr (Q::EW == 8) {
            const uint2 x = reinterpret_cast<const uint2*>(qlut)[e];
            accs[ti][0] += x.x; accs[ti][1] += x.y;
          } else {
            const uint4 x = reinterpret_cast<const uint4*>(qlut)[e];
            accs[ti][0] += x.x; accs[ti][1] += x.y; accs[ti][2] += x.z; accs[ti][3] += x.w;
          }
        }
        if (to_hist && t >= lo_t && t < hi_t) {
          if constexpr (GT == 1) {
            const int bin = approx_of<GT>(accs[ti], 0) >> HSHIFT;
            atomicAdd(&hist[bin >> 1], 1u << (16 * (bin & 1)));
          } else {
            // straight from the packed lanes: the bin of a 16-bit score v is
            // v >> 6, its word v >> 7, its half bit 6 of v
            static_assert(HSHIFT == 6 && HWORDS == 512, "bin arithmetic below");
            static_assert((MAX_CHUNKS + K6_CLUSTER_MAX - 1) / K6_CLUSTER_MAX * K6_CHUNK <= 65535,
                          "a CTA's 16-bit bin counters cannot overflow");
#pragma unroll
            for (int a = 0; a < Q::NACC; ++a) {
              const uint32_t x = accs[ti][a];
              const int gl = (GT == 2) ? 0 : (a >> 1) * 4 + (a & 1), gh = (GT == 2) ? 1 : gl + 2;
              atomicAdd(&hist[gl * HWORDS + ((x >> 7) & (HWORDS - 1))], 1u << ((x >> 2) & 16u));
              atomicAdd(&hist[gh * HWORDS + (x >> 23)], 1u << ((x >> 18) & 16u));
            }
          }
        }
      }
    }
  };

  // candidates of chunk c from accs: list (token per (head, slot)), exact
  // rescoring into selection keys, count (-1 when the list overflowed)
  uint32_t* list = hist;   // [GT][CAND_MAX], the histograms are dead by then
  static_assert(CAND_MAX <= HWORDS, "candidate list must fit the histogram space");
  auto emit_chunk = [&](int c) {
    const int t0 = c * K6_CHUNK;
    const int lo_t = max(t0, cr.sink), hi_t = min(t0 + K6_CHUNK, cr.Sc);
    {   // candidates as one bit per (token, head) of this thread; the warp
        // visits only the bits some lane has set, twice: per-warp counts (one
        // atomic per (warp, head)), then the slots, in (token, head) order
      using MT = typename std::conditional<(K6_TPT * GT <= 32), uint32_t, unsigned long long>::type;
      MT mask = 0;
      int thr[GT];
#pragma unroll
      for (int g = 0; g < GT; ++g) thr[g] = g < p.G ? s_thr[g] : INT_MAX;   // padded heads list nothing
#pragma unroll
      for (int ti = 0; ti < K6_TPT; ++ti) {
        const int t = t0 + ti * K6_THREADS + tid;
        const bool valid = t >= lo_t && t < hi_t;
#pragma unroll
        for (int g = 0; g < GT; ++g)
          if (valid && approx_of<GT>(accs[ti], g) >= thr[g]) mask |= (MT)1 << (ti * GT + g);
      }
      MT um;
      if constexpr (sizeof(MT) == 4) {
        um = __reduce_or_sync(0xffffffffu, mask);
      } else {
        um = ((MT)__reduce_or_sync(0xffffffffu, (unsigned)(mask >> 32)) << 32) |
             (MT)__reduce_or_sync(0xffffffffu, (unsigned)mask);
      }
      auto low_bit = [](MT x) { return sizeof(MT) == 4 ? __ffs((unsigned)x) - 1 : __ffsll((long long)x) - 1; };
      int mine = 0;   // lane g: this warp's candidates of head g
      for (MT r = um; r; r &= r - 1) {
        const int bit = low_bit(r);
        const unsigned m = __ballot_sync(0xffffffffu, (unsigned)(mask >> bit) & 1u);
        if (lane == (bit & (GT - 1))) mine += __popc(m);
      }
      int run = 0;    // lane g: next slot of head g
      if (lane < p.G && mine > 0) run = atomicAdd(&s_cnt[lane], mine);
      for (MT r = um; r; r &= r - 1) {
        const int bit = low_bit(r), g = bit & (GT - 1), ti = bit / GT;
        const bool pred = (unsigned)(mask >> bit) & 1u;
        const unsigned m = __ballot_sync(0xffffffffu, pred);
        const int slot = __shfl_sync(0xffffffffu, run, g) + __popc(m & ((1u << lane) - 1u));
        if (pred && slot < CAND_MAX) list[g * CAND_MAX + slot] = (uint32_t)(t0 + ti * K6_THREADS + tid);
        if (lane == g) run += __popc(m);
      }
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int g = 0; g < GT; ++g) { s_nl[g] = acc; acc += (g < p.G) ? min(s_cnt[g], CAND_MAX) : 0; }
    }
    __syncthreads();
    const int n_items = s_nl[GT - 1] + ((GT - 1 < p.G) ? min(s_cnt[GT - 1], CAND_MAX) : 0);
    uint64_t* keys = p.cand_key + ((int64_t)u * p.n_chunks + c) * GT * CAND_MAX;
    const float scale = p.scale;
    for (int i = tid; i < n_items; i += K6_THREADS) {
      int g = 0;
#pragma unroll
      for (int k = 1; k < GT; ++k) if (i >= s_nl[k]) g = k;
      const int slot = i - s_nl[g];
      if (s_cnt[g] > CAND_MAX) continue;   // overflowed: the chunk is rescanned exactly
      const uint32_t t = list[g * CAND_MAX + slot];
      uint32_t cw[Q::W];
      load_code<Q::W>(gcodes + (int64_t)t * CS, cw);
      const float* tex = p.texact + ((int64_t)u * GT + g) * CS * 256;
      float e[CS];
#pragma unroll
      for (int s = 0; s < CS; ++s) e[s] = (s < M) ? __ldcg(tex + s * 256 + ((cw[s >> 2] >> (8 * (s & 3))) & 0xffu)) : 0.f;
      float sum = 0.f;   // reference order: ((0 + T0[c0]) + T1[c1]) + ...
#pragma unroll
      for (int s = 0; s < CS; ++s) if (s < M) sum = fadd(sum, e[s]);
      keys[g * CAND_MAX + slot] = sel_key(fmul(sum, scale), t);
      // the candidate's K and V rows into L2 for k7's attention over the
      // selected tokens (a hint; every head's copy of a token prefetches it)
      const int64_t rb = (int64_t)p.D * p.kv_es;
      const int64_t ro = ((int64_t)b * p.kv_sb + (int64_t)h * p.kv_sh) * p.kv_es + (int64_t)t * rb;
      prefetch_lines_l2(p.k, ro, rb);
      prefetch_lines_l2(p.v, ro, rb);
    }
    __syncthreads();
    if (tid < GT) {
      p.cand_cnt[((int64_t)u * p.n_chunks + c) * GT + tid] =
          (tid < p.G && s_cnt[tid] > CAND_MAX) ? -1 : (tid < p.G ? s_cnt[tid] : 0);
      s_cnt[tid] = 0;
    }
    __syncthreads();
  };

  // ---- histograms of every own chunk, pooled; threshold ----------------------
  for (int i = 0; i < n_mine; ++i) score_chunk(me + i * R, i == 0, true);
  stamp(0, scta, 8);   // own chunks scored (thread 0)
  // the unit-wide threshold straight from every CTA's histograms: per-lane
  // coarse counts, one cluster barrier, then each head's warp reads the R
  // coarse counts and the R copies of one 32-bin range through distributed
  // shared memory
  __syncthreads();
  coarse_counts<GT>(hist, coarse);
  cluster_arrive();
  cluster_wait();   // every CTA's histograms and coarse counts are complete
  stamp(0, scta, 9);   // histograms complete in the cluster
  if (warp < GT) {
    const int g = warp;
    const int bstar = top_bin_cluster(hist + g * HWORDS, coarse + g * 32, (uint32_t)cr.kp, lane, R);
    if (lane == 0)
      s_thr[g] = (s_margin[g] >= (1 << 30) || bstar < 0) ? -(1 << 30) : (bstar << HSHIFT) - s_margin[g];
  }
  cluster_arrive();   // this CTA no longer reads the others' histograms
  __syncthreads();
  stamp(0, scta, 10);   // threshold known
  cluster_wait();     // nor does any other CTA read this one's: the list may reuse them

  // ---- candidates: the last scored chunk from registers, the others scored again
  emit_chunk(me + (n_mine - 1) * R);
  for (int i = 0; i + 1 < n_mine; ++i) {
    score_chunk(me + i * R, false, false);
    emit_chunk(me + i * R);
  }
  stamp(0, scta, 11);  // candidates listed and rescored
}

template <int D, typename KVT>
struct AttnGeo {
  // dims per lane: 16 bytes of a row, or D / 32 when that is more
  static constexpr int DPL = (16 / (int)sizeof(KVT)) > D / 32 ? 16 / (int)sizeof(KVT) : D / 32;
  static constexpr int LPT = D / DPL;                    // lanes per token
  static constexpr int SUB = 32 / LPT;                   // tokens per warp step
};

// One lane's slice of a K/V row kept as stored (16-bit values two to a word)
// and widened to fp32 where it is used: twice the rows in flight per register
// than fp32 copies.
template <typename KVT, int DPL>
struct RawRow {
  static constexpr int NW = DPL * (int)sizeof(KVT) / 4;
  uint32_t w[NW];
};

template <typename KVT, int DPL>
__device__ __forceinline__ void load_raw(const KVT* p, RawRow<KVT, DPL>& r) {
  constexpr int NW = RawRow<KVT, DPL>::NW;
  static_assert(NW == 2 || NW % 4 == 0, "row slice of 8 or 16k bytes");
  if constexpr (NW == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    r.w[0] = v.x; r.w[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < NW / 4; ++i) {
      const uint4 v = reinterpret_cast<const uint4*>(p)[i];
      r.w[4 * i] = v.x; r.w[4 * i + 1] = v.y; r.w[4 * i + 2] = v.z; r.w[4 * i + 3] = v.w;
    }
  }
}

template <typename KVT, int DPL>
__device__ __forceinline__ void unpack_raw(const RawRow<KVT, DPL>& r, float (&o)[DPL]) {
  if constexpr (std::is_same<KVT, float>::value) {
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[i] = __uint_as_float(r.w[i]);
  } else if constexpr (std::is_same<KVT, __nv_bfloat16>::value) {
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) {   // bf16 is the top half of an fp32
      o[2 * i] = __uint_as_float(r.w[i] << 16);
      o[2 * i + 1] = __uint_as_float(r.w[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r.w[i]));
      o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
  }
}

// ===========================================================================
// K7: exact selection and attention, grid (B*H_kv*G), 256 threads.
// ===========================================================================
template <int D, typename KVT>
struct Attn {
  using A = AttnGeo<D, KVT>;
  static constexpr int NW = K7_THREADS / 32;
  static constexpr int U = 8;   // row slices in flight per lane
  float qv[A::DPL];
  float m_run, l_run, acc[A::DPL];
  int sub, sl;

  __device__ void init(const float* s_q, int lane) {
    sub = lane / A::LPT;
    sl = lane - sub * A::LPT;
#pragma unroll
    for (int i = 0; i < A::DPL; ++i) { qv[i] = s_q[sl * A::DPL + i]; acc[i] = 0.f; }
    m_run = -INFINITY;
    l_run = 0.f;
  }

  // Online softmax over tokens i in [0, n) with token index tok(i); the U
  // scores of a step are reduced together, then folded in with one rescale.
  template <typename TokF, typename ScoreF>
  __device__ void run(const KVT* kb, const KVT* vb, int n, int warp, float scale, TokF tok, ScoreF on_score) {
    constexpr int STEP = NW * A::SUB * U;
    for (int ib = warp * A::SUB * U; ib < n; ib += STEP) {
      RawRow<KVT, A::DPL> kr[U], vr[U];
      float s[U];
      bool valid[U];
#pragma unroll
      for (int r = 0; r < U; ++r) {
        const int i = ib + r * A::SUB + sub;
        valid[r] = i < n;
        if (valid[r]) {
          const int t = tok(i);
          load_raw<KVT, A::DPL>(kb + (int64_t)t * D + sl * A::DPL, kr[r]);
          load_raw<KVT, A::DPL>(vb + (int64_t)t * D + sl * A::DPL, vr[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < U; ++r) {
        s[r] = 0.f;
        if (valid[r]) {
          float kf[A::DPL];
          unpack_raw<KVT, A::DPL>(kr[r], kf);
#pragma unroll
          for (int i = 0; i < A::DPL; ++i) s[r] = fmaf(qv[i], kf[i], s[r]);
        }
      }
#pragma unroll
      for (int o = A::LPT / 2; o; o >>= 1) {
#pragma unroll
        for (int r = 0; r < U; ++r) s[r] += __shfl_xor_sync(0xffffffffu, s[r], o);
      }
      float mloc = -INFINITY;
#pragma unroll
      for (int r = 0; r < U; ++r) {
        if (valid[r]) {
          s[r] *= scale;
          on_score(ib + r * A::SUB + sub, s[r]);
          mloc = fmaxf(mloc, s[r]);
        }
      }
      if (mloc != -INFINITY) {
        const float mn = fmaxf(m_run, mloc);
        const float corr = __expf(m_run - mn);
        l_run *= corr;
#pragma unroll
        for (int d = 0; d < A::DPL; ++d) acc[d] *= corr;
#pragma unroll
        for (int r = 0; r < U; ++r) {
          if (valid[r]) {
            const float pe = __expf(s[r] - mn);
            l_run += pe;
            float vf[A::DPL];
            unpack_raw<KVT, A::DPL>(vr[r], vf);
#pragma unroll
            for (int d = 0; d < A::DPL; ++d) acc[d] = fmaf(pe, vf[d], acc[d]);
          }
        }
        m_run = mn;
      }
    }
  }
};

constexpr int K7_RANK_MAX = K7_CAP;   // up to this many keys, selection by rank counting
constexpr int K7_FAST_SLOTS = 64;     // list slots per chunk read with the counts
static_assert(8 * K7_FAST_SLOTS + 4 <= K7_CAP && K7_FAST_SLOTS <= CAND_MAX && K7_FAST_SLOTS == 64,
              "fast path: two slots per lane, every chunk's keys fit the key buffer");
static_assert(K7_THREADS == 256, "k7_select_attend clears a 256-bin histogram with one thread per bin");

// Shared memory that caches the keys of the radix selection (long contexts),
// when they fit: 8192 keys.
constexpr int K7_KEYCACHE_BYTES = 65536;

template <int D, typename KVT>
__global__ void __launch_bounds__(K7_THREADS) k7_select_attend(Cdc03P p) {
  using A = AttnGeo<D, KVT>;
  using AT = Attn<D, KVT>;
  constexpr int NW = AT::NW;
  extern __shared__ __align__(16) unsigned char smem[];
  float* T = reinterpret_cast<float*>(smem);                                 // [M][256] exact sub-table
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem + p.M * 1024);           // [K7_CAP]
  uint32_t* hist = reinterpret_cast<uint32_t*>(keys + K7_CAP);               // [256]
  int* sel = reinterpret_cast<int*>(hist + 256);                             // [TOPK_MAX]
  float* part = reinterpret_cast<float*>(sel + TOPK_MAX);                    // [NW][D + 2]
  __shared__ float s_q[D];
  __shared__ int s_n, s_over, s_cnt[MAX_CHUNKS], s_off[MAX_CHUNKS + 1];

  const int Hq = p.Hkv * p.G;
  const int u = blockIdx.x / p.G, g = blockIdx.x - (blockIdx.x / p.G) * p.G;
  const int b = u / p.Hkv, h = u - b * p.Hkv;
  const int hq = h * p.G + g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ColdRange cr = cold_range(p, b);
  const bool topk_mode = !(cr.k >= cr.Sc) && cr.kp > 0;
  const KVT* kb = reinterpret_cast<const KVT*>(p.k) + (int64_t)b * p.kv_sb + (int64_t)h * p.kv_sh;
  const KVT* vb = reinterpret_cast<const KVT*>(p.v) + (int64_t)b * p.kv_sb + (int64_t)h * p.kv_sh;
  const float scale = p.scale;
  const bool want_scores = p.sel_score != nullptr;
  const int sel_cap = max(p.top_k, p.sink);   // sinks are kept even when top_k < sink_tokens
  const int64_t sel_base = ((int64_t)b * Hq + hq) * sel_cap;

  stamp(1, blockIdx.x, 0);
  for (int d = tid; d < D; d += K7_THREADS)
    s_q[d] = load_as_f32(p.q, p.q_dtype, (int64_t)b * p.q_sb + (int64_t)hq * D + d);
  if (tid == 0) s_n = 0;
  __syncthreads();
  AT at;
  at.init(s_q, lane);

  // key cache of the radix selection (long contexts)
  uint64_t* kc = reinterpret_cast<uint64_t*>(part + NW * (D + 2));

  // ---- hot window: independent of the candidate stage, done before waiting
  // (rows straight from memory, 16 in flight per warp for 16-bit K/V)
  const int n_hot = cr.S - cr.Sc;
  at.run(kb, vb, n_hot, warp, scale, [&](int i) { return cr.Sc + i; }, [](int, float) {});

  stamp(1, blockIdx.x, 1);   // hot window attended (thread 0)
  // ---- wait for the candidate stage ------------------------------------------
  pdl_wait();
  stamp(1, blockIdx.x, 2);   // candidate stage complete

  int n_sel;
  bool explicit_sel = false;
  if (cr.k >= cr.Sc) {
    n_sel = cr.Sc;
  } else if (cr.kp <= 0) {
    n_sel = cr.sink;
  } else {
    explicit_sel = true;
    const int M = p.M;
    const int64_t cbase_idx = (int64_t)u * p.n_chunks * p.GT;
    // common case in one memory round trip, the counts read together with the
    // first list slots (the slots below the count are kept): up to NW chunks,
    // warp c reads chunk c and its first 64 slots; up to 2 NW chunks, chunks c
    // and c + NW, 32 slots each
    const bool two = p.n_chunks > NW;
    const int slots = two ? K7_FAST_SLOTS / 2 : K7_FAST_SLOTS;
    bool fast = p.n_chunks <= 2 * NW;
    int cnt0 = 0, cnt1 = 0;
    uint64_t k0 = 0ull, k1 = 0ull;
    const int c0 = warp, c1 = warp + NW;
    if (fast && c0 < p.n_chunks) {
      const int64_t li = cbase_idx + (int64_t)c0 * p.GT + g;
      cnt0 = __ldcg(p.cand_cnt + li);
      k0 = __ldcg(p.cand_key + li * CAND_MAX + lane);
      if (!two) k1 = __ldcg(p.cand_key + li * CAND_MAX + lane + 32);
      if (lane == 0) s_cnt[c0] = cnt0;
    }
    if (fast && two && c1 < p.n_chunks) {
      const int64_t li = cbase_idx + (int64_t)c1 * p.GT + g;
      cnt1 = __ldcg(p.cand_cnt + li);
      k1 = __ldcg(p.cand_key + li * CAND_MAX + lane);
      if (lane == 0) s_cnt[c1] = cnt1;
    }
    fast = !__syncthreads_or(!fast || (c0 < p.n_chunks && (cnt0 < 0 || cnt0 > slots)) ||
                             (two && c1 < p.n_chunks && (cnt1 < 0 || cnt1 > slots)));
    if (fast) {
      int off0 = 0, off1 = 0, n_all = 0;
      for (int c = 0; c < p.n_chunks; ++c) {
        const int x = s_cnt[c];
        off0 += c < c0 ? x : 0;
        off1 += c < c1 ? x : 0;
        n_all += x;
      }
      if (c0 < p.n_chunks) {
        if (lane < cnt0) keys[off0 + lane] = k0;
        if (!two && lane + 32 < cnt0) keys[off0 + lane + 32] = k1;
      }
      if (two && c1 < p.n_chunks && lane < cnt1) keys[off1 + lane] = k1;
      for (int i = tid; i < cr.sink; i += K7_THREADS) sel[i] = i;
      if (tid < 4) keys[n_all + tid] = 0ull;   // padding to a multiple of 4: a zero key beats none
      if (tid == 0) s_n = min(n_all, cr.kp);
      __syncthreads();
      const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(keys);
      const int n4 = (n_all + 3) >> 2;
      for (int i = tid; i < n_all; i += K7_THREADS) {   // position = rank: a fixed order
        const uint64_t x = keys[i];
        int rank = 0;
#pragma unroll 4
        for (int j = 0; j < n4; ++j) {
          const ulonglong2 a = k2[2 * j], c = k2[2 * j + 1];
          rank += (int)(a.x > x) + (int)(a.y > x) + (int)(c.x > x) + (int)(c.y > x);
        }
        if (rank < cr.kp) sel[cr.sink + rank] = (int)key_idx(x);
      }
    } else {
      for (int c = tid; c < p.n_chunks; c += K7_THREADS) s_cnt[c] = p.cand_cnt[cbase_idx + (int64_t)c * p.GT + g];
      __syncthreads();
      if (tid == 0) {
        int acc = 0, over = 0;
        for (int c = 0; c < p.n_chunks; ++c) { s_off[c] = acc; acc += s_cnt[c] > 0 ? s_cnt[c] : 0; over |= s_cnt[c] < 0; }
        s_off[p.n_chunks] = acc;
        s_over = over;
      }
      __syncthreads();
      if (s_over) {   // exact sub-table of this head, for the rescan of overflowed chunks
        const float* tex = p.texact + ((int64_t)u * p.GT + g) * p.CS * 256;
        for (int i = tid; i < M * 64; i += K7_THREADS) cp_async16(T + i * 4, tex + i * 4);
      }
      const int n_listed = s_off[p.n_chunks];
      for (int i = tid; i < cr.sink; i += K7_THREADS) sel[i] = i;
      if (!s_over && n_listed <= K7_RANK_MAX) {
        // few keys: gathered into shared memory; a key is selected when fewer
        // than k' keys beat it (keys are unique)
        for (int li = tid; li < n_listed; li += K7_THREADS) {
          int lo = 0, hi = p.n_chunks - 1;   // chunk c with s_off[c] <= li < s_off[c + 1]
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_off[mid] <= li) lo = mid; else hi = mid - 1;
          }
          keys[li] = p.cand_key[(cbase_idx + (int64_t)lo * p.GT + g) * CAND_MAX + (li - s_off[lo])];
        }
        if (tid == 0) s_n = min(n_listed, cr.kp);
        __syncthreads();
        for (int i = tid; i < n_listed; i += K7_THREADS) {   // position = rank: a fixed order
          const uint64_t x = keys[i];
          int rank = 0;
          for (int j = 0; j < n_listed; ++j) rank += keys[j] > x;
          if (rank < cr.kp) sel[cr.sink + rank] = (int)key_idx(x);
        }
      } else {
        // many keys (chunk-local thresholds of long contexts) or overflowed
        // lists: radix select of the k'-th largest key, 8 bits a round, over the
        // listed keys and the exact keys of every token of an overflowed chunk
        // (recomputed each round from the exact sub-table); the selection is
        // exactly the keys >= that key
        cp_async_wait_all();
        const uint8_t* codes = p.codes + (int64_t)b * p.c_sb + (int64_t)h * p.c_sh;
        __shared__ int s_ooff[MAX_CHUNKS], s_nall;   // overflowed chunks: key positions after the listed keys
        auto for_each_source_key = [&](auto fn) {
          // listed keys: flat index, 8 loads in flight per thread
          constexpr int UK = 8;
          for (int base = tid; base < n_listed; base += UK * K7_THREADS) {
            uint64_t kk[UK];
  #pragma unroll
            for (int r = 0; r < UK; ++r) {
              const int li = base + r * K7_THREADS;
              kk[r] = 0ull;
              if (li < n_listed) {
                int lo = 0, hi = p.n_chunks - 1;   // chunk c with s_off[c] <= li < s_off[c + 1]
                while (lo < hi) {
                  const int mid = (lo + hi + 1) >> 1;
                  if (s_off[mid] <= li) lo = mid; else hi = mid - 1;
                }
                kk[r] = __ldcg(p.cand_key + (cbase_idx + (int64_t)lo * p.GT + g) * CAND_MAX + (li - s_off[lo]));
              }
            }
  #pragma unroll
            for (int r = 0; r < UK; ++r)
              if (base + r * K7_THREADS < n_listed) fn(kk[r], base + r * K7_THREADS);
          }
          // overflowed chunks: exact keys of every non-sink token
          for (int c = 0; c < p.n_chunks; ++c) {
            if (s_cnt[c] >= 0) {
              continue;
            } else {
              const int clo = max(c * p.chunk, cr.sink), chi = min((c + 1) * p.chunk, cr.Sc);
              for (int t = clo + tid; t < chi; t += K7_THREADS) {
                const uint32_t* row = reinterpret_cast<const uint32_t*>(codes + (int64_t)t * p.CS);
                uint32_t cw[8];
  #pragma unroll
                for (int w = 0; w < 8; ++w) cw[w] = (w < p.CS / 4) ? __ldg(row + w) : 0u;   // one row, loads in flight together
                float sum = 0.f;
                for (int s2 = 0; s2 < M; ++s2) sum = fadd(sum, T[s2 * 256 + ((cw[s2 >> 2] >> (8 * (s2 & 3))) & 0xffu)]);
                fn(sel_key(fmul(sum, scale), (uint32_t)t), n_listed + s_ooff[c] + (t - clo));
              }
            }
          }
        };
        // every key once into the (idle) row staging space when they fit there
        if (tid == 0) {
          int acc = 0;
          for (int c = 0; c < p.n_chunks; ++c) {
            s_ooff[c] = acc;
            if (s_cnt[c] < 0) acc += max(0, min((c + 1) * p.chunk, cr.Sc) - max(c * p.chunk, cr.sink));
          }
          s_nall = n_listed + acc;
        }
        __syncthreads();
          const int kc_cap = K7_KEYCACHE_BYTES / 8;
        const bool cached = s_nall <= kc_cap;
        if (cached) {
          for_each_source_key([&](uint64_t key, int pos) { kc[pos] = key; });
          __syncthreads();
        }
        auto for_each_key = [&](auto fn) {
          if (cached) {
            for (int i = tid; i < s_nall; i += K7_THREADS) fn(kc[i]);
          } else {
            for_each_source_key([&](uint64_t key, int) { fn(key); });
          }
        };
        __shared__ unsigned long long s_pre, s_msk;
        __shared__ int s_need, s_done;
        if (tid == 0) { s_pre = 0ull; s_msk = 0ull; s_need = cr.kp; s_done = 0; }
        __syncthreads();
        for (int shift = 56; shift >= 0; shift -= 8) {
          if (s_done) break;   // uniform: read after a barrier
          hist[tid] = 0;       // K7_THREADS == 256 bins
          __syncthreads();
          const unsigned long long pre = s_pre, msk = s_msk;
          for_each_key([&](uint64_t key) {
            if ((key & msk) == pre) atomicAdd(&hist[(int)((key >> shift) & 255u)], 1u);
          });
          __syncthreads();
          if (warp == 0) {
            const int need = s_need;
            uint32_t ls = 0;
  #pragma unroll
            for (int i = 0; i < 8; ++i) ls += hist[lane * 8 + i];
            uint32_t suf = ls;
  #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t t = __shfl_down_sync(0xffffffffu, suf, o);
              if (lane + o < 32) suf += t;
            }
            const unsigned ball = __ballot_sync(0xffffffffu, suf >= (uint32_t)need);
            if (ball == 0u) {
              if (lane == 0) s_done = 1;   // fewer matching keys than needed: take them all
            } else {
              const int lstar = 31 - __clz((int)ball);
              if (lane == lstar) {
                uint32_t cum = suf - ls;
                for (int i = 7; i >= 0; --i) {
                  const int d = lane * 8 + i;
                  const uint32_t hd = hist[d];
                  if (cum + hd >= (uint32_t)need) {
                    const int rest = need - (int)cum;
                    s_pre = pre | ((unsigned long long)d << shift);
                    s_msk = msk | (255ull << shift);
                    s_need = rest;
                    if ((int)hd == rest || shift == 0) s_done = 1;
                    break;
                  }
                  cum += hd;
                }
              }
            }
          }
          __syncthreads();
        }
        if (tid == 0) s_n = 0;
        __syncthreads();
        const unsigned long long thr = s_pre;
        for_each_key([&](uint64_t key) {
          if (key >= thr) {
            const int slot = atomicAdd(&s_n, 1);
            if (slot < K7_CAP) keys[slot] = key;
          }
        });
        __syncthreads();
        const int m = min(min(s_n, cr.kp), K7_CAP);
        for (int i = tid; i < m; i += K7_THREADS) {   // position = rank among the selected: a fixed order
          const uint64_t x = keys[i];
          int rank = 0;
          for (int j = 0; j < m; ++j) rank += keys[j] > x;
          sel[cr.sink + rank] = (int)key_idx(x);
        }
      }
    }   // general path
    __syncthreads();
    n_sel = cr.sink + min(s_n, cr.kp);
    __syncthreads();
  }
  stamp(1, blockIdx.x, 3);   // selection done

  // ---- exact attention over the selected cold tokens, rows straight from
  // memory (16 rows in flight per warp: one round trip for 128 rows)
  at.run(kb, vb, n_sel, warp, scale, [&](int i) { return explicit_sel ? sel[i] : i; }, [&](int i, float s) {
    if (want_scores && at.sl == 0 && i < sel_cap) p.sel_score[sel_base + i] = s;
  });

  stamp(1, blockIdx.x, 4);   // selected tokens attended (thread 0)
  // combine the SUB token groups of this warp, then the warps
#pragma unroll
  for (int o = A::LPT; o < 32; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, at.m_run, o);
    const float lo = __shfl_xor_sync(0xffffffffu, at.l_run, o);
    const float mn = fmaxf(at.m_run, mo);
    const float a = (at.m_run == -INFINITY) ? 0.f : __expf(at.m_run - mn);
    const float c = (mo == -INFINITY) ? 0.f : __expf(mo - mn);
    at.l_run = at.l_run * a + lo * c;
#pragma unroll
    for (int d = 0; d < A::DPL; ++d) {
      const float ao = __shfl_xor_sync(0xffffffffu, at.acc[d], o);
      at.acc[d] = at.acc[d] * a + ao * c;
    }
    at.m_run = mn;
  }
  float* pw = part + warp * (D + 2);
  if (at.sub == 0) {
#pragma unroll
    for (int d = 0; d < A::DPL; ++d) pw[at.sl * A::DPL + d] = at.acc[d];
    if (at.sl == 0) { pw[D] = at.m_run; pw[D + 1] = at.l_run; }
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
  stamp(1, blockIdx.x, 5);
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

// The same for uint8 codes with head_dim = 16 * LPT (LPT = 1..32 lanes per
// token) and 16-byte-aligned rows: LPT lanes share a token, each loads 16
// codes with one 16-byte load (a warp reads 32 / LPT whole rows, contiguous
// when the rows are), looks them up in the lane-replicated codebook (bank of
// lane L = L: conflict-free for any code) and multiplies by its 16 query
// values kept in registers; the LPT partial sums are added by shuffles.  A
// grid-stride loop, so each CTA fills the replicated codebook once.
template <int LPT, typename ACC>
__global__ void __launch_bounds__(256) k_scalar_vq_qkt_u8v(const float* __restrict__ q, const uint8_t* __restrict__ idx,
                                                           int64_t S, int64_t stride, const float* __restrict__ cbk,
                                                           int k, float scale, float* __restrict__ scores) {
  __shared__ float rep[256 * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
    const int j = i >> 5;
    rep[i] = (j < k) ? cbk[j] : 0.f;
  }
  const int sub = lane % LPT;   // this lane's 16 dims: [16 sub, 16 sub + 16)
  float qv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) qv[i] = q[sub * 16 + i];
  __syncthreads();
  constexpr int TPW = 32 / LPT;   // tokens per warp and step
  const int64_t step = (int64_t)gridDim.x * 8 * TPW;
  for (int64_t t0 = ((int64_t)blockIdx.x * 8 + warp) * TPW; t0 < S; t0 += step) {
    const int64_t t = t0 + lane / LPT;
    ACC acc = 0;
    if (t < S) {
      const uint4 w = *reinterpret_cast<const uint4*>(idx + t * stride + sub * 16);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = (int)((ws[i >> 2] >> (8 * (i & 3))) & 0xffu);
        acc += (ACC)qv[i] * (ACC)rep[j * 32 + lane];
      }
    }
#pragma unroll
    for (int o = LPT / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (sub == 0 && t < S) scores[t] = (float)(acc * (ACC)scale);
  }
}

}  // namespace hokv
