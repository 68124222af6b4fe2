// assign_tc.cuh -- nearest-centroid assignment of batched f16/bf16 vectors
// with a tensor-core screen (tcgen05, accumulators in tensor memory) and an
// exact fp32 rescoring, bit-exact with the reference.
//
// Reference: vector_codebook.py:95-119 (VectorCodebook.assign) per subspace,
// product_codebook.py:118-145 (ProductCodebook.assign): for (N x d) @ (d x k)
// with N >= 5 rows the distance is ((|x|^2 - 2 x.c) + |c|^2) with x.c one fp32
// FMA chain in ascending d (hokv_math.cuh, DOT_SEQ_FMA) and the first minimum
// wins.
//
// Screen.  Per 128-row tile of one subspace, the tensor cores compute
//   s_j = x . c_j - |c_j|^2 / 2       (argmax s  <->  argmin distance)
// in tf32 with fp32 accumulation: x (f16/bf16 values, exact in tf32; fp32
// values split as x_hi + x_lo the same way) times c = c_hi + c_lo (c_hi = c
// rounded to tf32, c_lo = c - c_hi, exact in fp32; x_lo c_lo is left out),
// plus an appended K chunk [1, 1, 0..] x [-|c|^2_hi / 2, -|c|^2_lo / 2, 0..]
// that folds the centroid norms in; centroid slots past the live count get
// -2^99 there and never win.  Each thread owns one row (one TMEM lane): it
// finds the largest s over the row (tcgen05.ld, 32 columns at a time), then
// every centroid with s_j >= max - delta is a candidate, where delta bounds
// twice the screen's error plus the reference's own rounding:
//   E_tc = (n_terms + 2) 2^-22 (3 |x|_1 Cmax + Csq_max)   (tensor-core sums,
//          truncation of c_lo, x_lo and the norm's low part to tf32, and the
//          omitted x_lo c_lo),
//   E_ex = 2^-22 ((d + 1) |x|_1 Cmax + |x|^2 + Csq_max)   (fp32 FMA chain and
//          the two roundings of the expansion),
//   delta = 1.25 (E_ex + 2 E_tc),
// with Cmax = the largest |c_ji| and Csq_max the largest |c_j|^2 of the
// subspace's live centroids.  The exact minimiser always is a candidate
// (s_j* >= s_max - E_ex - 2 E_tc).  Candidates are rescored in the
// reference's fp32 order and the lowest index among equal distances wins, so
// the code equals the reference's bit for bit.
//
// Layout.  Operands sit in shared memory as K-major core matrices without
// swizzle (8 rows x 16 bytes, 128 contiguous bytes): element (r, k) of a
// tile with KE elements per row lives at
//   (r / 8) * (KE / 4) * 128 + (k / 4) * 128 + (r % 8) * 16 + (k % 4) * 4
// bytes, so one K = 8 slice is two adjacent core-matrix columns (leading
// byte offset 128, stride byte offset (KE / 4) * 128).  A CTA keeps one
// (set, subspace) codebook staged and loops over row tiles; one elected thread
// issues the MMAs and commits them to an mbarrier, every wait is bounded.
#pragma once
#include "hokv_common.cuh"

namespace hokv {

constexpr int TC_ROWS = 128;          // rows per tile = TMEM lanes = epilogue threads
constexpr int TC_TMEM_COLS = 256;     // fp32 accumulator columns: two stages of 128 or one of 256
constexpr int TC_MIN_ROWS = 256;      // smaller batches stay on the CUDA-core kernels
constexpr unsigned long long TC_WAIT_NS = 1000000000ull;   // an mbarrier wait gives up after one second

// tf32 value nearest to x (ties away from zero) in an fp32 container.
__device__ __forceinline__ float tf32_round(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Shared-memory matrix descriptor: K-major, no swizzle, 128-byte core-matrix
// columns (leading byte offset) and `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3ffffu) >> 4);          // start address, bits 0-13
  d |= (uint64_t)(128u >> 4) << 16;                  // leading byte offset, bits 16-29
  d |= (uint64_t)((sbo & 0x3ffffu) >> 4) << 32;      // stride byte offset, bits 32-45
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  return d;                                          // base offset 0, no swizzle
}

// Instruction descriptor of kind::tf32: fp32 accumulator, A and B tf32,
// both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t umma_idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, int accumulate) {
  const uint32_t no_mask = 0u;   // no output lane disabled
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(no_mask));
}

__device__ __forceinline__ void umma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait until the mbarrier's phase `parity` completes; false when TC_WAIT_NS
// passed first.  Each try_wait may suspend the thread in hardware for up to
// 0.1 ms (its time hint), so a blocked warp issues few instructions.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, unsigned parity) {
  const uint32_t a = smem_u32(mbar);
  const uint32_t hint_ns = 100000u;
  unsigned long long t0 = 0;
  for (int i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(hint_ns)
        : "memory");
    if (done) return true;
    if (i == 0) t0 = global_ns();
    else if (global_ns() - t0 > TC_WAIT_NS) return false;
  }
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (r, k) in a K-major core-matrix tile with ke
// elements per row.
__device__ __forceinline__ uint32_t cm_off(int r, int k, int ke) {
  return (uint32_t)((r >> 3) * (ke >> 2) * 128 + (k >> 2) * 128 + (r & 7) * 16 + (k & 3) * 4);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mbar)) : "memory");
}

constexpr int TC_PRODUCERS = 64;      // threads (two warps) filling A tiles

// The SD values of one row as fp32: 16-byte loads when the row start is
// 16-byte aligned and SD fills whole loads, element loads otherwise.
template <int SD>
__device__ __forceinline__ void tc_load_row(const void* x, int dtype, int64_t base, float (&xv)[SD]) {
  if (dtype == HOKV_F32) {
    const float* px = reinterpret_cast<const float*>(x) + base;
    if (SD % 4 == 0 && (reinterpret_cast<uintptr_t>(px) & 15) == 0) {
#pragma unroll
      for (int d = 0; d < SD; d += 4) {
        const float4 v = *reinterpret_cast<const float4*>(px + d);
        xv[d] = v.x; xv[d + 1] = v.y; xv[d + 2] = v.z; xv[d + 3] = v.w;
      }
      return;
    }
  } else {
    const uint16_t* px = reinterpret_cast<const uint16_t*>(x) + base;
    if (SD % 8 == 0 && (reinterpret_cast<uintptr_t>(px) & 15) == 0) {
#pragma unroll
      for (int d = 0; d < SD; d += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(px + d);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (dtype == HOKV_BF16) {
            xv[d + 2 * e] = __uint_as_float(w[e] << 16);
            xv[d + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
          } else {
            const __half2 hh = *reinterpret_cast<const __half2*>(&w[e]);
            const float2 f = __half22float2(hh);
            xv[d + 2 * e] = f.x;
            xv[d + 2 * e + 1] = f.y;
          }
        }
      }
      return;
    }
  }
#pragma unroll
  for (int d = 0; d < SD; ++d) xv[d] = load_as_f32(x, dtype, base + d);
}
constexpr int TC_CTA = 2 * TC_ROWS + TC_PRODUCERS + 32;   // 2 x 4 epilogue warps, 2 producer warps, 1 MMA warp

// Tile geometry of k_pq_assign_tc: K slices of x (KX), B and A row lengths,
// and the A ring depth that keeps two CTAs per SM where it can (at most 113 KB
// of shared memory each), one otherwise; STAGES == 0 marks a variant that does
// not fit (the CUDA-core kernel handles it).
template <int SD, bool SPLIT>
struct TcGeo {
  static constexpr int KX = (SD + 7) / 8;
  static constexpr int KL = 8 * KX;
  static constexpr int KE = KL + 8;
  static constexpr int KA = SPLIT ? 2 * KL + 8 : KL + 8;
  static constexpr int A_BYTES = TC_ROWS * KA * 4;
  static constexpr int SIDE_BYTES = TC_ROWS * (SD + 2) * 4;
  static constexpr int XCH = 8 * TC_ROWS * 4;   // the epilogue groups' exchange rows
  static constexpr int FIXED = 256 * KE * 4 + 256 * KL * 4 + 256 * 4 + XCH + 256;
  static constexpr int PER = A_BYTES + SIDE_BYTES;
  static constexpr int S2 = (113 * 1024 - FIXED) / PER;
  static constexpr int S1 = (227 * 1024 - FIXED) / PER;
  static constexpr int STAGES = S2 >= 2 ? (S2 > 4 ? 4 : S2) : (S1 >= 1 ? (S1 > 4 ? 4 : S1) : 0);
  static constexpr int SMEM = FIXED + (STAGES > 0 ? STAGES : 1) * PER;
};

// grid (CTAs), TC_CTA threads; CTA c takes (set, subspace) pair c % pairs and
// tile group c / pairs.  Roles:
//   warps 0-3, 7-10  two epilogue groups: thread r of a group owns row r of
//              a tile (TMEM lane r); group g takes the tiles of accumulator
//              stage g, so two tiles' epilogues run at once (with a single
//              256-column stage, group 0 takes every tile);
//   warps 4-5  producers: x rows of the next tiles into a TC_STAGES ring of
//              A tiles (x_hi, [1, 1, 0..], x_lo in core-matrix layout) plus
//              the fp32 row, |x|^2 and |x|_1 the epilogue needs;
//   warp 6     lane 0 issues the MMAs of a tile into one of the accumulator
//              stages (two of 128 columns, or one of 256 when more than 128
//              centroids are live) and commits them to that stage's mbarrier.
// mbarriers: a_full[s] (64 producer arrivals), a_empty[s] (the 4 warps of the
// epilogue group that took the tile), acc_full[a] (the commit), acc_empty[a]
// (4 epilogue warps).  Every wait is
// bounded; a wait that gives up sets HOKV_ERR_TIMEOUT and the CTA drains.
// Shared memory: B_hi [256][KE], B_lo [256][KL], |c|^2 [256], the exchange
// rows of the two epilogue groups [8][128], then per stage
// A [128][KA] and the rows [128][SD] + |x|^2 [128] + |x|_1 [128], then the
// barriers and control words.
template <int SD, bool SPLIT>
__global__ void __launch_bounds__(TC_CTA, TcGeo<SD, SPLIT>::S2 >= 2 ? 2 : 1) k_pq_assign_tc(const void* __restrict__ x, int dtype, int64_t n, int64_t xrs,
                                                          int64_t xss, const float* __restrict__ cents, int slots,
                                                          int64_t css, const int* __restrict__ kk, int64_t kss,
                                                          uint8_t* __restrict__ out, int64_t ors, int64_t oss, int M,
                                                          int n_sets, int groups) {
  using TG = TcGeo<SD, SPLIT>;
  constexpr int KX = TG::KX, KL = TG::KL, KE = TG::KE, KA = TG::KA;
  constexpr int A_BYTES = TG::A_BYTES, SIDE_BYTES = TG::SIDE_BYTES, TC_STAGES = TG::STAGES;
  static_assert(TC_STAGES >= 1, "variant does not fit in shared memory");
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  unsigned char* sBh = tc_smem;                                  // 256 x KE
  unsigned char* sBl = sBh + 256 * KE * 4;                       // 256 x KL
  float* csq = reinterpret_cast<float*>(sBl + 256 * KL * 4);     // [256]
  float* xch = csq + 256;                                        // [8][TC_ROWS] epilogue exchange
  unsigned char* ring = reinterpret_cast<unsigned char*>(xch + 8 * TC_ROWS);   // TC_STAGES x (A, side)
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + TC_STAGES * (A_BYTES + SIDE_BYTES));
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + TC_STAGES;
  uint64_t* acc_full = bars + 2 * TC_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* ctl = reinterpret_cast<uint32_t*>(acc_empty + 2);   // [0] tmem, [1] Cmax, [2] Csq_max, [3] abort

  const int pairs = M * n_sets;
  const int pair = blockIdx.x % pairs, grp = blockIdx.x / pairs;
  const int s = pair % M, set = pair / M;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int k = kk[(int64_t)set * kss + s];
  k = k < 1 ? 1 : (k > slots ? slots : k);
  // MMA N: live slots rounded up to 32, so every 32-column chunk the epilogue
  // reads holds computed values (slots past the live count score -2^98)
  const int np = (k + 31) & ~31;
  const int n_acc = np <= 128 ? 2 : 1;            // accumulator stages in the 256 columns
  const float* cg = cents + (int64_t)set * css + (int64_t)s * slots * SD;
  const int64_t n_tiles = (n + TC_ROWS - 1) / TC_ROWS;
  const int64_t t_begin = n_tiles * grp / groups, t_end = n_tiles * (grp + 1) / groups;
  constexpr bool split = SPLIT;                   // fp32 inputs: x = x_hi + x_lo

  if (warp == 6) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(ctl)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < TC_STAGES; ++i) {
      mbar_init(&a_full[i], TC_PRODUCERS);
      mbar_init(&a_empty[i], n_acc == 1 ? 8 : 4);   // both epilogue groups take every tile with one stage
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], n_acc == 1 ? 8 : 4);
    }
    ctl[1] = 0u;
    ctl[2] = 0u;
    ctl[3] = 0u;
  }
  __syncthreads();
  // B: split centroids, exact norms, bounds (slots past the live count never win)
  for (int j = tid; j < 256; j += TC_CTA) {
    float c[SD];
    const bool live = j < k;
#pragma unroll
    for (int d = 0; d < SD; ++d) c[d] = live ? cg[(int64_t)j * SD + d] : 0.f;
    const float c2 = live ? sum_sq(c, SD) : 0.f;
    csq[j] = c2;
    float cm = 0.f;
#pragma unroll
    for (int d = 0; d < KL; ++d) {
      const float v = d < SD ? c[d] : 0.f;
      const float hi = tf32_round(v);
      *reinterpret_cast<float*>(sBh + cm_off(j, d, KE)) = hi;
      *reinterpret_cast<float*>(sBl + cm_off(j, d, KL)) = v - hi;
      cm = fmaxf(cm, fabsf(v));
    }
    const float c2h = tf32_round(c2);
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      float v = 0.f;
      if (d == 0) v = live ? -0.5f * c2h : -0x1p99f;
      if (d == 1) v = live ? -0.5f * (c2 - c2h) : 0.f;
      *reinterpret_cast<float*>(sBh + cm_off(j, KL + d, KE)) = v;
    }
    if (live) {
      atomicMax(&ctl[1], __float_as_uint(cm));   // non-negative floats order as their bits
      atomicMax(&ctl[2], __float_as_uint(c2));
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl[0];
  const float cmax = __uint_as_float(ctl[1]), csqmax = __uint_as_float(ctl[2]);
  volatile uint32_t* abort_flag = &ctl[3];
  auto give_up = [&]() { if (atomicExch(const_cast<uint32_t*>(abort_flag), 1u) == 0u) dev_flag(HOKV_ERR_TIMEOUT); };

  if (warp < 4 || warp >= 7) {
    // ---- epilogue: one row per thread (TMEM lane).  With two accumulator
    //      stages (up to 128 live centroids) group g (warps 0-3 / 7-10) takes
    //      the tiles of stage g; with one 256-column stage both groups take
    //      every tile, group g its columns [128 g, 128 g + 128), and they
    //      combine the row maximum, the candidate counts and the best
    //      candidate through shared memory at a named barrier (id 1) ----------
    const int g = warp < 4 ? 0 : 1, quad = warp & 3, r = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    constexpr float N_TERMS = 3 * KL + 2;
    const int nch = np >> 5;
    const bool halves = n_acc == 1;                         // column split between the groups
    const int c_lo = halves ? g * 4 : 0, c_hi = halves ? min(nch, g * 4 + 4) : nch;
    float* xm = xch;                                        // [2][TC_ROWS] half maxima
    int* xt = reinterpret_cast<int*>(xch + 2 * TC_ROWS);    // [2][TC_ROWS] candidate counts
    float* xd = xch + 4 * TC_ROWS;                          // [2][TC_ROWS] best distances
    int* xj = reinterpret_cast<int*>(xch + 6 * TC_ROWS);    // [2][TC_ROWS] best slots
    auto pair_sync = [&]() { asm volatile("bar.sync 1, 256;" ::: "memory"); };
    int64_t it = 0;
    for (int64_t tile = t_begin; tile < t_end; ++tile, ++it) {
      const int st = (int)(it % TC_STAGES), a = (int)(it % n_acc);
      if (!halves && a != g) continue;   // the other group's tile
      const unsigned ph_a = (unsigned)((it / n_acc) & 1);
      bool ok = !*abort_flag && mbar_wait(&a_full[st], (unsigned)((it / TC_STAGES) & 1)) && mbar_wait(&acc_full[a], ph_a);
      if (halves) {   // both groups leave together (the named barriers below need all 8 warps)
        uint32_t r_ok;
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.and.pred q, 1, 256, p;\n\t"
                     "selp.u32 %0, 1, 0, q;\n\t}\n" : "=r"(r_ok) : "r"((uint32_t)ok) : "memory");
        ok = r_ok != 0;
      }
      if (!ok) {
        give_up();
        break;
      }
      tc_fence_after();
      const float* side = reinterpret_cast<const float*>(ring + st * (A_BYTES + SIDE_BYTES) + A_BYTES);
      const float x2 = side[TC_ROWS * SD + r], xa = side[TC_ROWS * (SD + 1) + r];
      const uint32_t col0 = lane_base + (uint32_t)(a * 128);
      float cmaxs[8];
      float m = -INFINITY;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        cmaxs[c] = -INFINITY;
        if (c >= c_lo && c < c_hi) {
          float v[32];
          tmem_ld32(col0 + c * 32, v);
#pragma unroll
          for (int w = 16; w > 1; w >>= 1)
#pragma unroll
            for (int q = 0; q < w; ++q) v[q] = fmaxf(v[q], v[q + w]);
          cmaxs[c] = fmaxf(v[0], v[1]);
          m = fmaxf(m, cmaxs[c]);
        }
      }
      if (halves) {
        xm[g * TC_ROWS + r] = m;
        pair_sync();
        m = fmaxf(m, xm[(1 - g) * TC_ROWS + r]);
      }
      const float e_tc = (N_TERMS + 2.f) * 0x1p-22f * (3.f * xa * cmax + csqmax);
      const float e_ex = 0x1p-22f * ((float)(SD + 1) * xa * cmax + x2 + csqmax);
      const float thr = m - 1.25f * (e_ex + 2.f * e_tc);
      // candidates as one bit per column of each needed chunk
      uint32_t cmask[8];
      int total = 0;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        cmask[c] = 0u;
        const bool need = c >= c_lo && c < c_hi && cmaxs[c] >= thr;
        if (__any_sync(0xffffffffu, need)) {
          float v[32];
          tmem_ld32(col0 + c * 32, v);
          if (need) {
            uint32_t msk = 0u;
#pragma unroll
            for (int q = 0; q < 32; ++q) msk |= (uint32_t)(v[q] >= thr) << q;
            cmask[c] = msk;
            total += __popc(msk);
          }
        }
      }
      if (halves) {
        xt[g * TC_ROWS + r] = total;
        pair_sync();
        total += xt[(1 - g) * TC_ROWS + r];
      }
      // one candidate is the minimiser; several are rescored exactly, in slot
      // order (the row read back from shared memory)
      float best = INFINITY;
      int bj = 0x7fffffff;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        for (uint32_t msk = cmask[c]; msk; msk &= msk - 1u) {
          const int j = c * 32 + __ffs(msk) - 1;
          if (total == 1) { bj = j; break; }
          float acc = 0.f;
#pragma unroll
          for (int d = 0; d < SD; ++d) {
            const float cd = *reinterpret_cast<const float*>(sBh + cm_off(j, d, KE)) +
                             *reinterpret_cast<const float*>(sBl + cm_off(j, d, KL));   // c_hi + c_lo = c
            acc = ffma(side[d * TC_ROWS + r], cd, acc);
          }
          const float dd = l2_expansion(x2, acc, csq[j]);
          if (dd < best || bj == 0x7fffffff) { best = dd; bj = j; }
        }
      }
      if (halves) {   // group 1's slots are all above group 0's: ties keep group 0's
        xd[g * TC_ROWS + r] = best;
        xj[g * TC_ROWS + r] = bj;
        pair_sync();
        const float ob = xd[(1 - g) * TC_ROWS + r];
        const int oj = xj[(1 - g) * TC_ROWS + r];
        if (g == 0 && oj != 0x7fffffff && (bj == 0x7fffffff || ob < best)) bj = oj;
      }
      const int64_t i = tile * TC_ROWS + r;
      if ((!halves || g == 0) && i < n) out[(int64_t)set * oss + i * ors + s] = (uint8_t)(bj == 0x7fffffff ? 0 : bj);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {   // 4 arrivals per group that took the tile
        mbar_arrive(&acc_empty[a]);
        mbar_arrive(&a_empty[st]);
      }
    }
  } else if (warp < 6) {
    // ---- producers: the next tiles' rows into the A ring -------------------
    const int pt = tid - TC_ROWS;   // 0..63: rows pt and pt + 64 of a tile
    int64_t it = 0;
    for (int64_t tile = t_begin; tile < t_end; ++tile, ++it) {
      const int st = (int)(it % TC_STAGES);
      const unsigned ph = (unsigned)(((it / TC_STAGES) & 1) ^ 1);   // the first pass finds every slot free
      if (*abort_flag || !mbar_wait(&a_empty[st], ph)) { give_up(); break; }
      unsigned char* A = ring + st * (A_BYTES + SIDE_BYTES);
      float* side = reinterpret_cast<float*>(A + A_BYTES);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = pt + h * 64;
        const int64_t i = tile * TC_ROWS + r;
        const bool valid = i < n;
        const int64_t base = (int64_t)set * xss + (valid ? i : 0) * xrs + (int64_t)s * SD;
        float xv[SD];
        if (valid) tc_load_row<SD>(x, dtype, base, xv);
        else {
#pragma unroll
          for (int d = 0; d < SD; ++d) xv[d] = 0.f;
        }
        float xa = 0.f;
#pragma unroll
        for (int d = 0; d < SD; ++d) xa += fabsf(xv[d]);
        // 16-byte stores: four consecutive K elements of a row are one
        // core-matrix row slice (conflict-free across the warp's rows)
#pragma unroll
        for (int d4 = 0; d4 < KL / 4; ++d4) {
          float hv[4], lv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = d4 * 4 + e;
            const float v = d < SD ? xv[d] : 0.f;
            hv[e] = split ? tf32_round(v) : v;
            lv[e] = v - hv[e];
          }
          *reinterpret_cast<float4*>(A + cm_off(r, d4 * 4, KA)) = make_float4(hv[0], hv[1], hv[2], hv[3]);
          if (split)
            *reinterpret_cast<float4*>(A + cm_off(r, KL + 8 + d4 * 4, KA)) = make_float4(lv[0], lv[1], lv[2], lv[3]);
        }
        *reinterpret_cast<float4*>(A + cm_off(r, KL, KA)) = make_float4(1.f, 1.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(A + cm_off(r, KL + 4, KA)) = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int d = 0; d < SD; ++d) side[d * TC_ROWS + r] = xv[d];   // [dim][row]: conflict-free
        side[TC_ROWS * SD + r] = sum_sq(xv, SD);
        side[TC_ROWS * (SD + 1) + r] = xa;
      }
      fence_async_smem();
      mbar_arrive(&a_full[st]);
    }
  } else if (lane == 0) {
    // ---- MMA issue --------------------------------------------------------------
    const uint32_t idesc = umma_idesc_tf32(np);
    const uint32_t aBh = smem_u32(sBh), aBl = smem_u32(sBl);
    constexpr uint32_t sbo_a = (KA / 4) * 128, sbo_h = (KE / 4) * 128, sbo_l = (KL / 4) * 128;
    int64_t it = 0;
    for (int64_t tile = t_begin; tile < t_end; ++tile, ++it) {
      const int st = (int)(it % TC_STAGES), a = (int)(it % n_acc);
      const unsigned ph_full = (unsigned)((it / TC_STAGES) & 1);
      const unsigned ph_empty = (unsigned)(((it / n_acc) & 1) ^ 1);
      if (*abort_flag || !mbar_wait(&a_full[st], ph_full) || !mbar_wait(&acc_empty[a], ph_empty)) {
        give_up();
        break;
      }
      tc_fence_after();
      const uint32_t aA = smem_u32(ring + st * (A_BYTES + SIDE_BYTES));
      const uint32_t d = tmem + (uint32_t)(a * 128);
#pragma unroll
      for (int kc = 0; kc < KX; ++kc)   // x_hi . c_hi
        umma_tf32(d, umma_desc(aA + kc * 256, sbo_a), umma_desc(aBh + kc * 256, sbo_h), idesc, kc > 0);
      // [1, 1, 0..] . [-|c|^2_hi / 2, -|c|^2_lo / 2, 0..]
      umma_tf32(d, umma_desc(aA + KX * 256, sbo_a), umma_desc(aBh + KX * 256, sbo_h), idesc, 1);
#pragma unroll
      for (int kc = 0; kc < KX; ++kc)   // x_hi . c_lo
        umma_tf32(d, umma_desc(aA + kc * 256, sbo_a), umma_desc(aBl + kc * 256, sbo_l), idesc, 1);
      if (split) {
#pragma unroll
        for (int kc = 0; kc < KX; ++kc)   // x_lo . c_hi
          umma_tf32(d, umma_desc(aA + (KX + 1 + kc) * 256, sbo_a), umma_desc(aBh + kc * 256, sbo_h), idesc, 1);
      }
      umma_commit(&acc_full[a]);
    }
    // the last commits: wait (bounded) until this thread's MMAs are done
    if (it > 0) {
      const int64_t last = it - 1;
      (void)mbar_wait(&acc_full[last % n_acc], (unsigned)((last / n_acc) & 1));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 6) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

}  // namespace hokv
