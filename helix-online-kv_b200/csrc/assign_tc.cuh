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

constexpr int TC_ROWS = 128;          // rows per tile = TMEM lanes = threads
constexpr int TC_THREADS = 128;
constexpr int TC_TMEM_COLS = 256;     // fp32 accumulator columns (centroid slots)
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
// passed first.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, unsigned parity) {
  const uint32_t a = smem_u32(mbar);
  const unsigned long long t0 = global_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (global_ns() - t0 > TC_WAIT_NS) return false;
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

// grid (M, tile groups, n_sets), TC_THREADS threads.  KX = ceil(SD / 8) K
// slices of x; shared memory: A [128][KA] (x_hi, [1, 1, 0..], x_lo), B_hi
// [256][KE] (c_hi, norms), B_lo [256][KL] (c_lo), with KL = 8 KX,
// KE = KL + 8, KA = 2 KL + 8; |c|^2 [256], then the control words.
template <int SD>
__global__ void __launch_bounds__(TC_THREADS) k_pq_assign_tc(const void* __restrict__ x, int dtype, int64_t n,
                                                           int64_t xrs, int64_t xss, const float* __restrict__ cents,
                                                           int slots, int64_t css, const int* __restrict__ kk,
                                                           int64_t kss, uint8_t* __restrict__ out, int64_t ors,
                                                           int64_t oss) {
  constexpr int KX = (SD + 7) / 8;
  constexpr int KL = 8 * KX;
  constexpr int KE = KL + 8;
  constexpr int KA = 2 * KL + 8;
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  unsigned char* sA = tc_smem;                              // 128 x KA
  unsigned char* sBh = sA + TC_ROWS * KA * 4;               // 256 x KE
  unsigned char* sBl = sBh + 256 * KE * 4;                  // 256 x KL
  float* csq = reinterpret_cast<float*>(sBl + 256 * KL * 4);   // [256]
  uint64_t* mbar = reinterpret_cast<uint64_t*>(csq + 256);
  uint32_t* ctl = reinterpret_cast<uint32_t*>(mbar + 1);   // [0] tmem base, [1] Cmax ord, [2] Csq_max ord, [3] failed

  const int s = blockIdx.x, set = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5;
  int k = kk[(int64_t)set * kss + s];
  k = k < 1 ? 1 : (k > slots ? slots : k);
  const int np = (k + 15) & ~15;                            // MMA N: live slots rounded up to 16
  const float* cg = cents + (int64_t)set * css + (int64_t)s * slots * SD;

  if (warp == 0) {   // tensor memory for the accumulator (the whole warp allocates)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(ctl)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(mbar, 1);
    ctl[1] = 0u;
    ctl[2] = 0u;
    ctl[3] = 0u;
  }
  __syncthreads();
  // B: split centroids, norms, bounds
  for (int j = tid; j < 256; j += TC_THREADS) {
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl[0];
  const float cmax = __uint_as_float(ctl[1]), csqmax = __uint_as_float(ctl[2]);
  const uint32_t idesc = umma_idesc_tf32(np);
  const uint32_t aA = smem_u32(sA), aBh = smem_u32(sBh), aBl = smem_u32(sBl);
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  constexpr float N_TERMS = 3 * KL + 2;
  const bool split = dtype == HOKV_F32;   // fp32 inputs: x = x_hi + x_lo

  const int64_t n_tiles = (n + TC_ROWS - 1) / TC_ROWS;
  unsigned phase = 0;
  for (int64_t tile = blockIdx.y; tile < n_tiles; tile += gridDim.y) {
    const int64_t i = tile * TC_ROWS + tid;
    const bool valid = i < n;
    // A row of this thread: x slice, then [1, 1, 0..]
    float xv[SD];
    const int64_t base = (int64_t)set * xss + (valid ? i : 0) * xrs + (int64_t)s * SD;
#pragma unroll
    for (int d = 0; d < SD; ++d) xv[d] = valid ? load_as_f32(x, dtype, base + d) : 0.f;
    float xa = 0.f;
#pragma unroll
    for (int d = 0; d < KL; ++d) {
      const float v = d < SD ? xv[d] : 0.f;
      const float hi = split ? tf32_round(v) : v;
      *reinterpret_cast<float*>(sA + cm_off(tid, d, KA)) = hi;
      *reinterpret_cast<float*>(sA + cm_off(tid, KL + 8 + d, KA)) = v - hi;
      xa += fabsf(v);
    }
#pragma unroll
    for (int d = 0; d < 8; ++d) *reinterpret_cast<float*>(sA + cm_off(tid, KL + d, KA)) = d < 2 ? 1.f : 0.f;
    const float x2 = sum_sq(xv, SD);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t sbo_a = (KA / 4) * 128, sbo_h = (KE / 4) * 128, sbo_l = (KL / 4) * 128;
#pragma unroll
      for (int kc = 0; kc < KX; ++kc)   // x_hi . c_hi
        umma_tf32(tmem, umma_desc(aA + kc * 256, sbo_a), umma_desc(aBh + kc * 256, sbo_h), idesc, kc > 0);
      // [1, 1, 0..] . [-|c|^2_hi / 2, -|c|^2_lo / 2, 0..]
      umma_tf32(tmem, umma_desc(aA + KX * 256, sbo_a), umma_desc(aBh + KX * 256, sbo_h), idesc, 1);
#pragma unroll
      for (int kc = 0; kc < KX; ++kc)   // x_hi . c_lo
        umma_tf32(tmem, umma_desc(aA + kc * 256, sbo_a), umma_desc(aBl + kc * 256, sbo_l), idesc, 1);
      if (split) {
#pragma unroll
        for (int kc = 0; kc < KX; ++kc)   // x_lo . c_hi
          umma_tf32(tmem, umma_desc(aA + (KX + 1 + kc) * 256, sbo_a), umma_desc(aBh + kc * 256, sbo_h), idesc, 1);
      }
      umma_commit(mbar);
    }
    const bool ok = mbar_wait(mbar, phase);
    if (__syncthreads_or(!ok)) {   // the same answer in every thread
      if (tid == 0) { dev_flag(HOKV_ERR_TIMEOUT); ctl[3] = 1u; }
      (void)mbar_wait(mbar, phase);   // the MMAs may still be running: one more bounded wait
      break;
    }
    phase ^= 1u;
    tc_fence_after();
    // pass 1: the row's largest screen value and each 32-column chunk's
    const int nch = (np + 31) >> 5;   // 32-column chunks holding the np MMA columns
    float cmaxs[8];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      cmaxs[c] = -INFINITY;
      if (c < nch) {
        float v[32];
        tmem_ld32(lane_base + c * 32, v);
        float mc = -INFINITY;
#pragma unroll
        for (int q = 0; q < 32; ++q) mc = fmaxf(mc, (c * 32 + q < np) ? v[q] : -INFINITY);
        cmaxs[c] = mc;
        m = fmaxf(m, mc);
      }
    }
    const float e_tc = (N_TERMS + 2.f) * 0x1p-22f * (3.f * xa * cmax + csqmax);
    const float e_ex = 0x1p-22f * ((float)(SD + 1) * xa * cmax + x2 + csqmax);
    const float thr = m - 1.25f * (e_ex + 2.f * e_tc);
    // pass 2: exact distances of the candidates, ascending slot order, first minimum
    float best = INFINITY;
    int bj = 0x7fffffff;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const bool need = c < nch && cmaxs[c] >= thr;
      if (__any_sync(0xffffffffu, need)) {
        float v[32];
        tmem_ld32(lane_base + c * 32, v);
        if (need) {
          for (int q = 0; q < 32; ++q) {
            const int j = c * 32 + q;
            if (j < k && v[q] >= thr) {
              float acc = 0.f;
#pragma unroll
              for (int d = 0; d < SD; ++d) {
                const float cd = *reinterpret_cast<const float*>(sBh + cm_off(j, d, KE)) +
                                 *reinterpret_cast<const float*>(sBl + cm_off(j, d, KL));   // exact: c_hi + c_lo = c
                acc = ffma(xv[d], cd, acc);
              }
              const float dd = l2_expansion(x2, acc, csq[j]);
              if (dd < best || bj == 0x7fffffff) { best = dd; bj = j; }
            }
          }
        }
      }
    }
    if (valid) out[(int64_t)set * oss + i * ors + s] = (uint8_t)(bj == 0x7fffffff ? 0 : bj);
    tc_fence_before();
    __syncthreads();   // every lane read: the accumulator may be overwritten
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

}  // namespace hokv
