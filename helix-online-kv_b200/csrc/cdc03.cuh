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
#include <type_traits>

namespace hokv {

constexpr int K6_THREADS = 256;
constexpr int K6_CHUNK_MAX = 4096;   // tokens per K6 CTA (16 per thread)
constexpr int CAND_MAX = 512;        // candidates per (unit, chunk, head)
constexpr int K7_THREADS = 256;
constexpr int K7_CAP = 2048;         // key buffer of the exact selection
constexpr int TOPK_MAX = 1024;       // largest top_k with k < S_c
constexpr int MAX_CHUNKS = 512;      // K6 chunks per (sequence, KV head)

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
  uint32_t* cand_idx; int* cand_cnt; uint8_t* cand_code;
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

// ---- async copies and programmatic dependent launch ------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
// Let the next kernel in the stream start its independent prologue now.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
// Block until the previous kernel in the stream has completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Rows [0, lim) of every subspace of one (sequence, KV head) codebook are
// staged in shared memory as stage[s][j][sd]; lim keeps the stage <= 64 KB.
__device__ __forceinline__ int stage_rows(int slots, int D) {
  const int lim = 16384 / D;  // D floats per (row of all subspaces) -> 64 KB
  return slots < lim ? slots : lim;
}

__device__ __forceinline__ void stage_codebook(float* stage, const float* cb, int M, int slots, int sd, int lim,
                                               int tid, int nthreads) {
  // bytes per subspace block = lim * sd * 4 (multiple of 16 for sd % 4 == 0)
  const int per_s = lim * sd / 4;  // 16-byte pieces per subspace
  const int total = M * per_s;
  for (int i = tid; i < total; i += nthreads) {
    const int s = i / per_s, r = i - s * per_s;
    cp_async16(stage + (int64_t)s * lim * sd + r * 4, cb + (int64_t)s * slots * sd + r * 4);
  }
}

// Rotate W words so that out[i] = in[(i + r) % W] (r dynamic, W a power of two).
template <int W, typename T>
__device__ __forceinline__ void rotate_words(T (&w)[W], int r) {
#pragma unroll
  for (int bit = 1; bit < W; bit <<= 1) {
    T t[W];
    const bool on = (r & bit) != 0;
#pragma unroll
    for (int i = 0; i < W; ++i) t[i] = on ? w[(i + bit) % W] : w[i];
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = t[i];
  }
}

template <int CS, int GT, int TPTM>
__global__ void __launch_bounds__(K6_THREADS, 2) k6_candidates(Cdc03P p) {
  using Q = QGeo<CS, GT>;
  static_assert(CS <= Q::COLS, "one row block");
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* qlut = smem;                                            // Q::BYTES
  float* stage = reinterpret_cast<float*>(smem + Q::BYTES);              // codebook rows, then codes
  const int stage_bytes = max(64 * 1024, p.chunk * CS);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + Q::BYTES + stage_bytes);  // [GT][256]
  float* sq = reinterpret_cast<float*>(hist + GT * 256);                 // [GT][D]
  __shared__ unsigned s_lo[GT * CS], s_hi[GT * CS];
  __shared__ float s_inv[GT], s_lof[GT * CS];
  __shared__ int s_margin[GT], s_thr[GT], s_cnt[GT], s_k[32];

  pdl_launch_dependents();
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
  const float* cbase = p.cb + (int64_t)b * p.cb_sb + (int64_t)h * p.cb_sh;
  const int lim = stage_rows(p.slots, D);
  const bool staged = (sd % 4) == 0;

  // ---- prologue: stage the codebook, load queries and counts ----------------
  if (staged) stage_codebook(stage, cbase, M, p.slots, sd, lim, tid, K6_THREADS);
  for (int i = tid; i < GT * D; i += K6_THREADS) {
    const int g = i / D, d = i - g * D;
    sq[i] = (g < p.G) ? load_as_f32(p.q, p.q_dtype, (int64_t)b * p.q_sb + (int64_t)(h * p.G + g) * D + d) : 0.f;
  }
  if (tid < M) {
    int ks = p.cbk[(int64_t)b * p.cbk_sb + (int64_t)h * p.cbk_sh + tid];
    s_k[tid] = ks < 0 ? 0 : (ks > p.slots ? p.slots : ks);
  }
  for (int i = tid; i < GT * 256; i += K6_THREADS) hist[i] = 0;
  for (int i = tid; i < GT * CS; i += K6_THREADS) { s_lo[i] = 0xffffffffu; s_hi[i] = 0u; }
  if (tid < GT) s_cnt[tid] = 0;
  cp_async_wait_all();
  __syncthreads();

  // exact sub-table value T[g][s][j] in the reference's BLAS order; j = tid
  const int j = tid;
  auto tval = [&](int g, int s) -> float {
    if (j >= s_k[s]) return 0.f;
    const float* row = (staged && j < lim) ? stage + ((int64_t)s * lim + j) * sd
                                           : cbase + ((int64_t)s * p.slots + j) * sd;
    return dot_order(p.lut_order, sq + g * D + s * sd, row, sd);
  };

  // ---- pass 1: per (head, subspace) value ranges -----------------------------
  for (int s = 0; s < M; ++s) {
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      const unsigned o = ord_f32(tval(g, s));
      const unsigned mn = __reduce_min_sync(0xffffffffu, o), mx = __reduce_max_sync(0xffffffffu, o);
      if (lane == 0) { atomicMin(&s_lo[g * CS + s], mn); atomicMax(&s_hi[g * CS + s], mx); }
    }
  }
  __syncthreads();
  if (tid < GT) {
    const int g = tid;
    float rmax = 0.f;
    double sa = 0.0;
    for (int s = 0; s < M; ++s) {
      const float lo = unord_f32(s_lo[g * CS + s]), hi = unord_f32(s_hi[g * CS + s]);
      s_lof[g * CS + s] = lo;
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

  // ---- pass 2: quantise and store the replicated 8-bit sub-tables -----------
  {
    using EntT = typename std::conditional<Q::EW == 4, uint32_t, uint2>::type;
    EntT w[CS];
#pragma unroll
    for (int s = 0; s < CS; ++s) {
      uint32_t code[GT];
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        uint32_t cv = 0;
        if (s < M) {
          float x = __fmul_rn(__fsub_rn(tval(g, s), s_lof[g * CS + s]), s_inv[g]);
          x = fminf(fmaxf(rintf(x), 0.f), 255.f);
          cv = (uint32_t)x;
        }
        code[g] = cv;
      }
      if constexpr (GT == 1) w[s] = code[0];
      else if constexpr (GT == 2) w[s] = code[0] | (code[1] << 16);
      else if constexpr (GT == 4) w[s] = code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
      else {
        uint2 v;
        v.x = code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
        v.y = code[4] | (code[5] << 8) | (code[6] << 16) | (code[7] << 24);
        w[s] = v;
      }
    }
    // lane L writes subspace (i + L) mod CS at step i: distinct columns per wavefront
    rotate_words<CS>(w, lane % CS);
    constexpr int NC = Q::COLS / CS;
#pragma unroll
    for (int cp = 0; cp < NC; ++cp) {
      const int copy = (cp + (lane % Q::COLS) / CS) % NC;
#pragma unroll
      for (int i = 0; i < CS; ++i) {
        const int col = copy * CS + ((i + lane) % CS);
        reinterpret_cast<EntT*>(qlut)[j * Q::COLS + col] = w[i];
      }
    }
  }
  __syncthreads();  // codebook stage is dead: reuse it for the chunk's codes

  // ---- stage the chunk's codes -------------------------------------------------
  const int t0 = c * p.chunk;
  const int ntok = min(p.chunk, cr.Sc - t0);
  const uint8_t* gcodes = p.codes + (int64_t)b * p.c_sb + (int64_t)h * p.c_sh + (int64_t)t0 * CS;
  {
    const int n16 = (ntok * CS + 15) / 16;
    unsigned char* dst = reinterpret_cast<unsigned char*>(stage);
    for (int i = tid; i < n16; i += K6_THREADS) cp_async16(dst + i * 16, gcodes + (int64_t)i * 16);
    cp_async_wait_all();
  }
  __syncthreads();

  // ---- 8-bit approximate scores, kept in registers ---------------------------
  const unsigned char* scodes = reinterpret_cast<const unsigned char*>(stage);
  const int r = lane % CS;
  int colidx[CS];
#pragma unroll
  for (int uu = 0; uu < CS; ++uu) colidx[uu] = Q::col_of(lane, (uu + r) % CS);
  uint32_t accs[TPTM][Q::NACC];
  int mxv[GT];
#pragma unroll
  for (int g = 0; g < GT; ++g) mxv[g] = -1;
  const int tpt = p.chunk / K6_THREADS;
#pragma unroll
  for (int it = 0; it < TPTM; ++it) {
#pragma unroll
    for (int a = 0; a < Q::NACC; ++a) accs[it][a] = 0;
    if (it >= tpt) continue;
    const int lt = it * K6_THREADS + tid;
    const int t = t0 + lt;
    const bool valid = t >= lo_t && t < hi_t;
    uint32_t w[Q::W];
    if constexpr (Q::W == 1) w[0] = *reinterpret_cast<const uint32_t*>(scodes + lt * CS);
    else if constexpr (Q::W == 2) { const uint2 v = *reinterpret_cast<const uint2*>(scodes + lt * CS); w[0] = v.x; w[1] = v.y; }
    else {
#pragma unroll
      for (int q4 = 0; q4 < Q::W / 4; ++q4) {
        const uint4 v = *reinterpret_cast<const uint4*>(scodes + lt * CS + q4 * 16);
        w[q4 * 4 + 0] = v.x; w[q4 * 4 + 1] = v.y; w[q4 * 4 + 2] = v.z; w[q4 * 4 + 3] = v.w;
      }
    }
    rotate_bytes<Q::W>(w, r);
#pragma unroll
    for (int uu = 0; uu < CS; ++uu) {
      const uint32_t byte = (w[uu >> 2] >> (8 * (uu & 3))) & 0xffu;
      const int e = colidx[uu] + (int)byte * Q::COLS;
      if constexpr (Q::EW == 4) {
        const uint32_t x = reinterpret_cast<const uint32_t*>(qlut)[e];
        if constexpr (GT <= 2) {
          accs[it][0] += x;
        } else {
          accs[it][0] += x & 0x00ff00ffu;
          accs[it][1] += (x >> 8) & 0x00ff00ffu;
        }
      } else {
        const uint2 x = reinterpret_cast<const uint2*>(qlut)[e];
        accs[it][0] += x.x & 0x00ff00ffu;
        accs[it][1] += (x.x >> 8) & 0x00ff00ffu;
        accs[it][2] += x.y & 0x00ff00ffu;
        accs[it][3] += (x.y >> 8) & 0x00ff00ffu;
      }
    }
    if (valid) {
#pragma unroll
      for (int g = 0; g < GT; ++g) mxv[g] = max(mxv[g], approx_of<GT>(accs[it], g));
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
    uint32_t suf = ls;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_down_sync(0xffffffffu, suf, o);
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

  // ---- emit candidates: token index and its code row --------------------------
  const int64_t cbase_idx = ((int64_t)u * p.n_chunks + c) * GT * CAND_MAX;
  uint32_t* cand = p.cand_idx + cbase_idx;
  uint8_t* ccode = p.cand_code + cbase_idx * CS;
#pragma unroll
  for (int it = 0; it < TPTM; ++it) {
    if (it >= tpt) break;
    const int lt = it * K6_THREADS + tid;
    const int t = t0 + lt;
    const bool valid = t >= lo_t && t < hi_t;
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      if (g >= p.G) break;   // uniform across the block
      const bool pred = valid && approx_of<GT>(accs[it], g) >= s_thr[g];
      const unsigned m = __ballot_sync(0xffffffffu, pred);
      if (m) {
        const int leader = __ffs(m) - 1;
        int basep = 0;
        if (lane == leader) basep = atomicAdd(&s_cnt[g], __popc(m));
        basep = __shfl_sync(0xffffffffu, basep, leader);
        const int slot = basep + __popc(m & ((1u << lane) - 1u));
        if (pred && slot < CAND_MAX) {
          cand[g * CAND_MAX + slot] = (uint32_t)t;
          uint8_t* dst = ccode + ((int64_t)g * CAND_MAX + slot) * CS;
#pragma unroll
          for (int q4 = 0; q4 < CS; q4 += 4)
            *reinterpret_cast<uint32_t*>(dst + q4) = *reinterpret_cast<const uint32_t*>(scodes + lt * CS + q4);
        }
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
  constexpr int U = 8;
  extern __shared__ __align__(16) unsigned char smem[];
  float* T = reinterpret_cast<float*>(smem);                                 // [M][256] exact sub-table
  unsigned char* X = smem + p.M * 1024;                                      // prologue: codebook stage;
  float* stage = reinterpret_cast<float*>(X);                                // afterwards the buffers below
  uint64_t* keys = reinterpret_cast<uint64_t*>(X);                           // [K7_CAP]
  uint32_t* hist = reinterpret_cast<uint32_t*>(X + K7_CAP * 8);              // [1024]
  int* sel = reinterpret_cast<int*>(X + K7_CAP * 8 + 4096);                  // [TOPK_MAX]
  float* part = reinterpret_cast<float*>(X + K7_CAP * 8 + 4096 + TOPK_MAX * 4);  // [NW][D + 2]
  __shared__ float s_q[D];
  __shared__ int s_n, s_k[32], s_cnt[MAX_CHUNKS], s_off[MAX_CHUNKS + 1];
  __shared__ SelShared s_sel;

  const int Hq = p.Hkv * p.G;
  const int u = blockIdx.x / p.G, g = blockIdx.x - (blockIdx.x / p.G) * p.G;
  const int b = u / p.Hkv, h = u - b * p.Hkv;
  const int hq = h * p.G + g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ColdRange cr = cold_range(p, b);
  const bool topk_mode = !(cr.k >= cr.Sc) && cr.kp > 0;

  // ---- prologue (independent of the candidate stage): q, exact sub-table ----
  for (int d = tid; d < D; d += K7_THREADS)
    s_q[d] = load_as_f32(p.q, p.q_dtype, (int64_t)b * p.q_sb + (int64_t)hq * D + d);
  if (tid == 0) s_n = 0;
  const int M = p.M, sd = p.sd;
  const float* cbase = p.cb + (int64_t)b * p.cb_sb + (int64_t)h * p.cb_sh;
  const int lim = stage_rows(p.slots, p.M * sd);
  const bool staged = (sd % 4) == 0;
  if (topk_mode) {
    if (staged) stage_codebook(stage, cbase, M, p.slots, sd, lim, tid, K7_THREADS);
    if (tid < M) {
      int ks = p.cbk[(int64_t)b * p.cbk_sb + (int64_t)h * p.cbk_sh + tid];
      s_k[tid] = ks < 0 ? 0 : (ks > p.slots ? p.slots : ks);
    }
    cp_async_wait_all();
  }
  __syncthreads();
  if (topk_mode) {
    for (int i = tid; i < M * 256; i += K7_THREADS) {
      const int s = i >> 8, j = i & 255;
      float t = 0.f;
      if (j < s_k[s]) {
        const float* row = (staged && j < lim) ? stage + ((int64_t)s * lim + j) * sd
                                               : cbase + ((int64_t)s * p.slots + j) * sd;
        t = dot_order(p.lut_order, s_q + s * sd, row, sd);
      }
      T[i] = t;
    }
  }
  // ---- wait for the candidate stage ------------------------------------------
  pdl_wait();
  __syncthreads();

  int n_sel;
  bool explicit_sel = false;
  if (cr.k >= cr.Sc) {
    n_sel = cr.Sc;
  } else if (cr.kp <= 0) {
    n_sel = cr.sink;
  } else {
    explicit_sel = true;
    const float scale = p.scale;
    const int64_t cbase_idx = (int64_t)u * p.n_chunks * p.GT;
    // candidate counts of every chunk (-1: list overflowed, rescan the chunk)
    for (int c = tid; c < p.n_chunks; c += K7_THREADS) s_cnt[c] = p.cand_cnt[cbase_idx + (int64_t)c * p.GT + g];
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int c = 0; c < p.n_chunks; ++c) { s_off[c] = acc; acc += s_cnt[c] > 0 ? s_cnt[c] : 0; }
      s_off[p.n_chunks] = acc;
    }
    __syncthreads();
    const int n_listed = s_off[p.n_chunks];
    // listed candidates: index + code row written by the candidate stage
    for (int base = 0; base < n_listed; base += K7_THREADS) {
      if (s_n + K7_THREADS > K7_CAP) {
        select_topm<K7_THREADS>(keys, s_n, cr.kp, hist, &s_sel);
        if (tid == 0) s_n = min(s_n, cr.kp);
        __syncthreads();
      }
      const int i = base + tid;
      if (i < n_listed) {
        int lo = 0, hi = p.n_chunks - 1;   // chunk c with s_off[c] <= i < s_off[c + 1]
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_off[mid] <= i) lo = mid; else hi = mid - 1;
        }
        const int c = lo;
        const int slot = i - s_off[c];
        const int64_t e = (cbase_idx + (int64_t)c * p.GT + g) * CAND_MAX + slot;
        const uint32_t t = p.cand_idx[e];
        const uint8_t* row = p.cand_code + e * p.CS;
        float sum = 0.f;
        for (int s = 0; s < M; ++s) sum = fadd(sum, T[s * 256 + row[s]]);
        keys[atomicAdd(&s_n, 1)] = sel_key(fmul(sum, scale), t);
      }
      __syncthreads();
    }
    // overflowed chunks: rescan every non-sink token of the chunk
    const uint8_t* codes = p.codes + (int64_t)b * p.c_sb + (int64_t)h * p.c_sh;
    for (int c = 0; c < p.n_chunks; ++c) {
      if (s_cnt[c] >= 0) continue;
      const int clo = max(c * p.chunk, cr.sink), chi = min((c + 1) * p.chunk, cr.Sc);
      for (int base = clo; base < chi; base += K7_THREADS) {
        if (s_n + K7_THREADS > K7_CAP) {
          select_topm<K7_THREADS>(keys, s_n, cr.kp, hist, &s_sel);
          if (tid == 0) s_n = min(s_n, cr.kp);
          __syncthreads();
        }
        const int t = base + tid;
        if (t < chi) {
          const uint8_t* row = codes + (int64_t)t * p.CS;
          float sum = 0.f;
          for (int s = 0; s < M; ++s) sum = fadd(sum, T[s * 256 + row[s]]);
          keys[atomicAdd(&s_n, 1)] = sel_key(fmul(sum, scale), (uint32_t)t);
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
