// prefill.cuh -- exact causal attention over many query tokens (prefill and
// the layers kept exact), FlashAttention-style on the tensor cores.
//
// The reference runs these through the model's own attention (its exact
// layers and every prefill see the dense K/V, compressed_cache.py:73-105);
// here one launch covers a layer: grid (query tiles, query heads, batch), one
// CTA per 128 query rows of one head, looping over key/value tiles of BN
// tokens up to the causal limit.  Per tile:
//   S = Q K^T            tcgen05.mma kind::f16 (f16 or bf16 operands in shared
//                        memory, fp32 accumulator: BN columns of tensor memory)
//   P = exp2(S * scale * log2 e - m)   one thread per row (its TMEM lane),
//                        written back as f16/bf16 in shared memory
//   O += P V             tcgen05.mma into D more columns of tensor memory
// with the online softmax's running maximum m raised lazily: O and the running
// sum are rescaled only when a row's maximum grows by more than 2^8 (the
// exponentials stay below 2^8, the normalisation by the same m at the end
// makes the result independent of when m was raised).
//
// Operands are K-major core matrices without swizzle (8 rows x 16 bytes,
// 128 contiguous bytes): element (r, k) of a tile with KE 16-bit elements per
// row lives at (r / 8) (KE / 8) 128 + (k / 8) 128 + (r % 8) 16 + (k % 8) 2
// bytes; one K = 16 step of an MMA is two adjacent core-matrix columns.  Q and
// K tiles are copied in that layout with cp.async; V^T (the B operand of
// P V, K = tokens) is built from raw V rows with ldmatrix.trans.  Keys past
// the sequence and queries past the last row are zero-filled and masked.
// One elected thread issues the MMAs and commits them to mbarriers; every
// wait is bounded and decided for the whole CTA at once.
#pragma once
#include <type_traits>
#include "assign_tc.cuh"

namespace hokv {

constexpr int PF_ROWS = 128;     // query rows per CTA = TMEM lanes = threads
constexpr int PF_TMEM_COLS = 256;

template <int D>
struct PfGeo {
  static constexpr int BN = D == 64 ? 128 : 64;      // key/value tokens per tile
  static constexpr int VR_STRIDE = D * 2 + 16;       // padded raw V row (conflict-free ldmatrix)
  static constexpr int Q_BYTES = PF_ROWS * D * 2;
  static constexpr int K_BYTES = BN * D * 2;
  static constexpr int VR_BYTES = BN * VR_STRIDE;
  static constexpr int VT_BYTES = D * BN * 2;
  static constexpr int P_BYTES = PF_ROWS * BN * 2;
  static constexpr int SMEM = Q_BYTES + K_BYTES + VR_BYTES + VT_BYTES + P_BYTES + 64;
  static constexpr int O_COL = 128;                  // O accumulator columns [128, 128 + D)
};

__device__ __forceinline__ uint32_t cm16(int r, int k, int ke) {
  return (uint32_t)((r >> 3) * (ke >> 3) * 128 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// Instruction descriptor of kind::f16: fp32 accumulator, A and B both f16
// (fmt 0) or both bf16 (fmt 1), K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t umma_idesc_f16(int n, int bf16) {
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(PF_ROWS >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, int accumulate) {
  const uint32_t no_mask = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(no_mask));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16-byte global -> shared copy; src_bytes = 0 fills zeros (src not read).
__device__ __forceinline__ void pf_cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void pf_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void pf_cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct PfArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int Sq, Skv, Hq, G;
  int64_t qsb, qsh, qss, ksb, ksh, kss, vsb, vsh, vss, osb, osh, oss;   // element strides
  float scale_log2;   // softmax scale * log2(e)
  int causal;
};

// grid (query tiles, Hq, B), PF_ROWS threads.  Thread r owns query row r of
// the tile (TMEM lane r).
template <int D, typename T>
__global__ void __launch_bounds__(PF_ROWS, 1) k_prefill_attn(const PfArgs p) {
  using PG = PfGeo<D>;
  constexpr int BN = PG::BN;
  constexpr int BF = sizeof(T) == 2 && !std::is_same<T, __half>::value ? 1 : 0;
  extern __shared__ __align__(1024) unsigned char pf_smem[];
  unsigned char* sQ = pf_smem;
  unsigned char* sK = sQ + PG::Q_BYTES;
  unsigned char* sVr = sK + PG::K_BYTES;
  unsigned char* sVt = sVr + PG::VR_BYTES;
  unsigned char* sP = sVt + PG::VT_BYTES;
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sP + PG::P_BYTES);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_o + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_qt = (p.Sq + PF_ROWS - 1) / PF_ROWS;
  const int qt = n_qt - 1 - (int)blockIdx.x;          // the longest (causal) tiles first
  const int hq = blockIdx.y, b = blockIdx.z, hk = hq / p.G;
  const int q0 = qt * PF_ROWS;
  const int off = p.Skv - p.Sq;                       // absolute position of query row 0
  const T* qg = reinterpret_cast<const T*>(p.q) + b * p.qsb + hq * p.qsh;
  const T* kg = reinterpret_cast<const T*>(p.k) + b * p.ksb + hk * p.ksh;
  const T* vg = reinterpret_cast<const T*>(p.v) + b * p.vsb + hk * p.vsh;
  const int last_pos = off + min(q0 + PF_ROWS, p.Sq) - 1;
  const int kv_end = p.causal ? min(p.Skv, last_pos + 1) : p.Skv;
  const int n_kt = (kv_end + BN - 1) / BN;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(PF_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
  }

  // ---- prologue: Q tile, K and V of tile 0 ----------------------------------
  constexpr int QCH = D / 8;   // 16-byte chunks per row
  for (int i = tid; i < PF_ROWS * QCH; i += PF_ROWS) {
    const int r = i / QCH, c = i % QCH;
    const bool in = q0 + r < p.Sq;
    pf_cp_async16(sQ + cm16(r, c * 8, D), qg + (in ? (int64_t)(q0 + r) * p.qss + c * 8 : 0), in ? 16 : 0);
  }
  auto load_k = [&](int kt) {
    for (int i = tid; i < BN * QCH; i += PF_ROWS) {
      const int r = i / QCH, c = i % QCH, t = kt * BN + r;
      const bool in = t < p.Skv;
      pf_cp_async16(sK + cm16(r, c * 8, D), kg + (in ? (int64_t)t * p.kss + c * 8 : 0), in ? 16 : 0);
    }
  };
  auto load_v = [&](int kt) {
    for (int i = tid; i < BN * QCH; i += PF_ROWS) {
      const int r = i / QCH, c = i % QCH, t = kt * BN + r;
      const bool in = t < p.Skv;
      pf_cp_async16(sVr + r * PG::VR_STRIDE + c * 16, vg + (in ? (int64_t)t * p.vss + c * 8 : 0), in ? 16 : 0);
    }
  };
  load_k(0);
  load_v(0);
  pf_cp_commit();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t idesc_s = umma_idesc_f16(BN, BF), idesc_o = umma_idesc_f16(D, BF);
  const int pos = off + q0 + tid;                     // this row's absolute position
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;   // the same on every thread: each wait's outcome is and-ed over the CTA

  for (int kt = 0; kt < n_kt; ++kt) {
    // (a) K_kt and V_kt are in shared memory
    pf_cp_wait_all();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // (b) S = Q K^T into columns [0, BN)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kc = 0; kc < D / 16; ++kc)
        umma_f16(tmem, umma_desc(smem_u32(sQ) + kc * 256, (D / 8) * 128), umma_desc(smem_u32(sK) + kc * 256, (D / 8) * 128),
                 idesc_s, kc > 0);
      umma_commit(bar_s);
    }
    // (c) the previous P V has finished reading V^T and P
    if (kt > 0) {
      ok = __syncthreads_and(mbar_wait(bar_o, (unsigned)((kt - 1) & 1)));
      if (!ok) break;
      tc_fence_after();
    }
    // (d) V^T of this tile from the raw rows: each ldmatrix.x4.trans moves four
    //     8 x 8 blocks (8 tokens x 32 dims)
    for (int blk = warp; blk < (BN / 8) * (D / 32); blk += PF_ROWS / 32) {
      const int ck = blk / (D / 32), d0 = (blk % (D / 32)) * 32;
      const unsigned char* src = sVr + (ck * 8 + (lane & 7)) * PG::VR_STRIDE + (d0 + 8 * (lane >> 3)) * 2;
      uint32_t r0, r1, r2, r3;
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                   : "r"(smem_u32(src)));
      const int dr = lane >> 2, kk = ck * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(sVt + cm16(d0 + dr, kk, BN)) = r0;
      *reinterpret_cast<uint32_t*>(sVt + cm16(d0 + 8 + dr, kk, BN)) = r1;
      *reinterpret_cast<uint32_t*>(sVt + cm16(d0 + 16 + dr, kk, BN)) = r2;
      *reinterpret_cast<uint32_t*>(sVt + cm16(d0 + 24 + dr, kk, BN)) = r3;
    }
    __syncthreads();
    if (kt + 1 < n_kt) load_v(kt + 1);                // raw V rows are free again
    // (e) S is ready; K may be overwritten
    ok = __syncthreads_and(mbar_wait(bar_s, (unsigned)(kt & 1)));
    if (!ok) break;
    tc_fence_after();
    if (kt + 1 < n_kt) load_k(kt + 1);
    pf_cp_commit();
    // (f) softmax of this row: maximum, lazy rescale, P
    const int t0 = kt * BN;
    const bool masked = t0 + BN > p.Skv || (p.causal && t0 + BN - 1 > off + q0);
    float mt = -INFINITY;
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld32(lane_base + c * 32, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int t = t0 + c * 32 + j;
        const bool live = !masked || (t < p.Skv && (!p.causal || t <= pos));
        mt = fmaxf(mt, live ? v[j] * p.scale_log2 : -INFINITY);
      }
    }
    const bool grow = mt > m_run + 8.f;
    const float m_new = grow ? mt : m_run;
    const float f = grow ? exp2f(m_run - m_new) : 1.f;   // 0 on the first tile
    if (kt > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(lane_base + PG::O_COL + c * 32, o);
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] *= f;
        tmem_st32(lane_base + PG::O_COL + c * 32, o);
      }
    }
    l_run *= f;
    m_run = m_new;
    float ls = 0.f;
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld32(lane_base + c * 32, v);
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float e[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int j = j8 * 8 + h * 2 + u;
            const int t = t0 + c * 32 + j;
            const bool live = !masked || (t < p.Skv && (!p.causal || t <= pos));
            e[u] = live ? exp2f(v[j] * p.scale_log2 - m_run) : 0.f;
            ls += e[u];
          }
          w[h] = pack2<T>(e[0], e[1]);
        }
        *reinterpret_cast<uint4*>(sP + cm16(tid, c * 32 + j8 * 8, BN)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    l_run += ls;
    // (g) O += P V^T
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kc = 0; kc < BN / 16; ++kc)
        umma_f16(tmem + PG::O_COL, umma_desc(smem_u32(sP) + kc * 256, (BN / 8) * 128),
                 umma_desc(smem_u32(sVt) + kc * 256, (BN / 8) * 128), idesc_o, kt > 0 || kc > 0);
      umma_commit(bar_o);
    }
  }
  pf_cp_wait_all();
  // ---- epilogue: O / l ---------------------------------------------------------
  if (ok && n_kt > 0) ok = __syncthreads_and(mbar_wait(bar_o, (unsigned)((n_kt - 1) & 1)));
  if (!ok) {
    if (tid == 0) dev_flag(HOKV_ERR_TIMEOUT);
  } else if (n_kt > 0) {
    tc_fence_after();
    const float inv = 1.f / l_run;
    const bool row_ok = q0 + tid < p.Sq;
    T* og = reinterpret_cast<T*>(p.out) + b * p.osb + hq * p.osh + (int64_t)(q0 + tid) * p.oss;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float o[32];
      tmem_ld32(lane_base + PG::O_COL + c * 32, o);
      if (row_ok) {
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          uint4 w;
          w.x = pack2<T>(o[j8 * 8 + 0] * inv, o[j8 * 8 + 1] * inv);
          w.y = pack2<T>(o[j8 * 8 + 2] * inv, o[j8 * 8 + 3] * inv);
          w.z = pack2<T>(o[j8 * 8 + 4] * inv, o[j8 * 8 + 5] * inv);
          w.w = pack2<T>(o[j8 * 8 + 6] * inv, o[j8 * 8 + 7] * inv);
          *reinterpret_cast<uint4*>(og + c * 32 + j8 * 8) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS));
  }
}

}  // namespace hokv
