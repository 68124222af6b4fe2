// prefill.cuh -- exact causal attention over many query tokens (prefill and
// the layers kept exact), FlashAttention-style on the tensor cores.
//
// The reference runs these through the model's own attention (its exact
// layers and every prefill see the dense K/V, compressed_cache.py:72-105);
// here one launch covers a layer.  Grid (query-tile pairs, query heads,
// batch): a CTA owns 2 x 128 query rows of one head and loops over key/value
// tiles of BN tokens up to the causal limit.  Per tile and query tile q:
//   S_q = Q_q K^T         tcgen05.mma kind::f16 (f16 or bf16 operands in
//                         shared memory, fp32 accumulator in tensor memory)
//   P_q = 2^(S_q * scale * log2 e - m)   one thread per query row (its TMEM
//                         lane), rounded to the input type into shared memory
//   O_q += P_q V          tcgen05.mma into tensor memory
// The two query tiles take turns on the tensor cores: while the softmax
// warps of one tile work, the other tile's products run.  The running
// maximum m is raised lazily: O and the running sum are rescaled only when a
// row's maximum grows by more than 8 (log2 units), so P stays below 2^8 and
// the final normalisation by the same m gives the exact softmax.
//
// Roles (320 threads): warps 0-3 the softmax of query tile 0 (thread = row =
// TMEM lane), warps 4-7 that of tile 1, warp 8 lane 0 loads the tiles with
// TMA (cp.async.bulk.tensor, completion counted in bytes on mbarriers), warp 9
// lane 0 issues the MMAs and commits them to mbarriers.  K and V stream
// through a ring of PF_STAGES tiles, so the loads run up to three tiles ahead
// of the products.
//
// Shared-memory tiles use the 128-byte swizzle of TMA and the tensor cores:
// a tile of R rows x C 16-bit columns is C / 64 column blocks of R rows x
// 128 bytes (64 elements), 16-byte chunk j of row r stored at chunk j ^ (r %
// 8), 8-row groups 1024 bytes apart.  TMA writes Q, K and V tiles in that
// layout from the (b, h, s) strided tensors; the softmax threads write P in
// it.  Q, K and P are read K-major (an MMA K step of 16 columns is 32 bytes
// inside a column block); V (rows = tokens) is read in place as the MN-major B
// of P V: 64-dim column blocks and 8-token groups.  No transposition anywhere.
// Keys past the sequence and queries past the last row are zero-filled by TMA
// and masked.  Every wait is bounded; a wait that gives up stops the CTA's roles
// and sets HOKV_ERR_TIMEOUT.
#pragma once
#include <cuda.h>
#include <type_traits>
#include "assign_tc.cuh"

namespace hokv {

constexpr int PF_ROWS = 128;                 // rows of a query tile = TMEM lanes
constexpr int PF_THREADS = 320;              // 8 softmax warps, 1 load warp, 1 MMA warp
constexpr int PF_TMEM_COLS = 512;            // S_0, S_1 (128 each), O_0, O_1 (128 each)
constexpr int PF_STAGES = 4;                 // K/V ring depth

template <int D>
struct PfGeo {
  static constexpr int BN = D == 64 ? 128 : 64;            // key/value tokens per tile
  static constexpr int Q_BYTES = PF_ROWS * D * 2;          // one query tile
  static constexpr int KV_BYTES = BN * D * 2;              // one K or V tile
  static constexpr int P_BYTES = PF_ROWS * BN * 2;         // one P tile
  static constexpr int SMEM = 2 * Q_BYTES + 2 * PF_STAGES * KV_BYTES + 2 * P_BYTES + 128;   // 224 KB + barriers
};

// Byte offset of element (r, k) (k a multiple of 8: the start of a 16-byte
// chunk) in a 128-byte-swizzled tile of `rows` rows.
__device__ __forceinline__ uint32_t sw128_off(int r, int k, int rows) {
  return (uint32_t)((k >> 6) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4));
}

// Shared-memory matrix descriptor with the 128-byte swizzle: leading and
// stride byte offsets given (sm_100 version bit, base offset 0: every tile
// starts on a 1024-byte boundary).
__device__ __forceinline__ uint64_t umma_desc_sw(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3ffffu) >> 4);
  d |= (uint64_t)((lbo & 0x3ffffu) >> 4) << 16;
  d |= (uint64_t)((sbo & 0x3ffffu) >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;   // 128-byte swizzle
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, A and B both f16
// (fmt 0) or both bf16 (fmt 1), A K-major, B K-major or (b_mn) MN-major,
// M = 128, N = n.
__device__ __forceinline__ uint32_t umma_idesc_f16(int n, int bf16, int b_mn) {
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)(b_mn ? 1 : 0) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(PF_ROWS >> 4) << 24);
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

// TMA tile load of a 4-D tensor map (no multicast) into this CTA's shared
// memory, completion counted in bytes on `bar`.
__device__ __forceinline__ void pf_tma4(void* dst, const void* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void pf_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

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

// 32 consecutive fp32 TMEM columns of this thread's lane, without waiting
// (tcgen05.wait::ld before the values are used).
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 2^x (MUFU ex2, flush-to-zero); the softmax weights are rounded to 16 bits
// afterwards, far coarser than its error.
__device__ __forceinline__ float pf_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Largest raw score of this thread's row of S (BN TMEM columns from
// s_addr); with MASK, columns j >= lim do not count.
template <bool MASK, int BN>
__device__ __forceinline__ float pf_row_max(uint32_t s_addr, int lim) {
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    tmem_ld32(s_addr + c * 32, v);
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      m0 = fmaxf(m0, MASK && c * 32 + j >= lim ? -INFINITY : v[j]);
      m1 = fmaxf(m1, MASK && c * 32 + j + 1 >= lim ? -INFINITY : v[j + 1]);
    }
  }
  return fmaxf(m0, m1);
}

// P = 2^(S * sl2 + nm) of this thread's row into the chunk-major P tile
// (row `row` of PF_ROWS, BN columns), masked columns 0; returns the row's sum
// of P (fp32, before rounding to T).
template <bool MASK, int BN, typename T>
__device__ __forceinline__ float pf_emit(uint32_t s_addr, unsigned char* sP, int row, float sl2, float nm, int lim) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    tmem_ld32(s_addr + c * 32, v);
#pragma unroll
    for (int j8 = 0; j8 < 4; ++j8) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int j = j8 * 8 + h * 2;
        float e0 = pf_ex2(fmaf(v[j], sl2, nm)), e1 = pf_ex2(fmaf(v[j + 1], sl2, nm));
        if (MASK) {
          e0 = c * 32 + j < lim ? e0 : 0.f;
          e1 = c * 32 + j + 1 < lim ? e1 : 0.f;
        }
        s0 += e0;
        s1 += e1;
        w[h] = pack2<T>(e0, e1);
      }
      *reinterpret_cast<uint4*>(sP + sw128_off(row, c * 32 + j8 * 8, PF_ROWS)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  return s0 + s1;
}

// Single-pass form for 64-column tiles: the row of S stays in registers
// (va: columns 0-31, vb: 32-63) between the maximum and the exponentials.
template <bool MASK>
__device__ __forceinline__ float pf_max_regs(const float (&va)[32], const float (&vb)[32], int lim) {
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    m0 = fmaxf(m0, MASK && j >= lim ? -INFINITY : va[j]);
    m1 = fmaxf(m1, MASK && 32 + j >= lim ? -INFINITY : vb[j]);
  }
  return fmaxf(m0, m1);
}

// Exponent arguments and the running sum use packed fp32 x 2 operations
// (one instruction per column pair); `rowp` is the row's byte offset in its
// P column block and x7 its swizzle key (row % 8).
template <bool MASK, typename T>
__device__ __forceinline__ float pf_emit_regs(const float (&v)[32], int c, unsigned char* sP, uint32_t rowp, int x7,
                                              float sl2, float nm, int lim) {
  float2 acc = make_float2(0.f, 0.f);
  const float2 sl = make_float2(sl2, sl2), nn = make_float2(nm, nm);
#pragma unroll
  for (int j8 = 0; j8 < 4; ++j8) {
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int j = j8 * 8 + h * 2;
      const float2 a = __ffma2_rn(make_float2(v[j], v[j + 1]), sl, nn);
      float2 e = make_float2(pf_ex2(a.x), pf_ex2(a.y));
      if (MASK) {
        e.x = c * 32 + j < lim ? e.x : 0.f;
        e.y = c * 32 + j + 1 < lim ? e.y : 0.f;
      }
      acc = __fadd2_rn(acc, e);
      w[h] = pack2<T>(e.x, e.y);
    }
    const int col = c * 32 + j8 * 8;   // chunk (col % 64) / 8 of column block col / 64
    *reinterpret_cast<uint4*>(sP + (col >> 6) * PF_ROWS * 128 + rowp + ((((col & 63) >> 3) ^ x7) << 4)) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
  return acc.x + acc.y;
}

// Tensor maps of q, k and v as 4-D (head dim, then the token, head and
// batch dims in ascending stride order); slot_* give each dim's coordinate
// position (1-3) in that map.
struct alignas(64) PfMaps {
  CUtensorMap q, k, v;
};

struct PfArgs {
  void* out;
  int Sq, Skv, Hq, G;
  int64_t osb, osh, oss;   // output element strides
  int q_slot_t, q_slot_h, q_slot_b, kv_slot_t, kv_slot_h, kv_slot_b;
  float scale_log2;        // softmax scale * log2(e)
  int causal;
};

__device__ __forceinline__ void pf_coords(int slot_t, int slot_h, int slot_b, int t, int h, int b, int (&c)[4]) {
  c[0] = 0;
  c[slot_t] = t;
  c[slot_h] = h;
  c[slot_b] = b;
}

// Warp-uniform bounded wait (every lane of the calling warp waits on `bar`).
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, unsigned parity, volatile uint32_t* abort_flag) {
  const bool ok = !*abort_flag && mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// grid (ceil(Sq / 256), Hq, B), PF_THREADS threads.
template <int D, typename T>
__global__ void __launch_bounds__(PF_THREADS, 1) k_prefill_attn(const __grid_constant__ PfMaps maps, const PfArgs p) {
  using PG = PfGeo<D>;
  constexpr int BN = PG::BN;
  constexpr int BF = std::is_same<T, __half>::value ? 0 : 1;
  extern __shared__ __align__(1024) unsigned char pf_smem[];
  unsigned char* sQ = pf_smem;                                   // [2 tiles][Q_BYTES]
  unsigned char* sK = sQ + 2 * PG::Q_BYTES;                      // [PF_STAGES][KV_BYTES]
  unsigned char* sV = sK + PF_STAGES * PG::KV_BYTES;             // [PF_STAGES][KV_BYTES]
  unsigned char* sP = sV + PF_STAGES * PG::KV_BYTES;             // [2 tiles][P_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * PG::P_BYTES);
  uint64_t* q_full = bars;                          // TMA bytes
  uint64_t* kv_full = bars + 1;                     // [PF_STAGES] TMA bytes
  uint64_t* kv_empty = kv_full + PF_STAGES;         // [PF_STAGES] MMA commit
  uint64_t* s_full = kv_empty + PF_STAGES;          // [2] MMA commit
  uint64_t* p_full = s_full + 2;                    // [2] softmax warps (4)
  uint64_t* o_final = p_full + 2;                   // [2] MMA commit
  uint32_t* ctl = reinterpret_cast<uint32_t*>(o_final + 2);      // [0] tmem base, [1] abort
  volatile uint32_t* abort_flag = &ctl[1];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_pairs = (p.Sq + 2 * PF_ROWS - 1) / (2 * PF_ROWS);
  const int q0 = (n_pairs - 1 - (int)blockIdx.x) * 2 * PF_ROWS;   // the longest (causal) tiles first
  const int hq = blockIdx.y, b = blockIdx.z, hk = hq / p.G;
  const int off = p.Skv - p.Sq;                                   // absolute position of query row 0
  int n_kt_q[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int base = q0 + q * PF_ROWS;
    if (base >= p.Sq) {
      n_kt_q[q] = 0;
    } else {
      const int last_pos = off + min(base + PF_ROWS, p.Sq) - 1;
      const int kv_end = p.causal ? min(p.Skv, last_pos + 1) : p.Skv;
      n_kt_q[q] = (kv_end + BN - 1) / BN;
    }
  }
  const int n_kt = max(n_kt_q[0], n_kt_q[1]);

  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(ctl)),
                 "r"(PF_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < PF_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
    }
    ctl[1] = 0u;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl[0];
  auto give_up = [&]() {
    if (atomicExch(const_cast<uint32_t*>(abort_flag), 1u) == 0u) dev_flag(HOKV_ERR_TIMEOUT);
  };

  if (warp < 8) {
    // ---- softmax of query tile q, one row per thread ------------------------------
    const int q = warp >> 2, row = tid & (PF_ROWS - 1);
    const int base = q0 + q * PF_ROWS;
    const int pos = off + base + row;                 // this row's absolute position
    const uint32_t lane_sel = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_sel + (uint32_t)(q * 128);
    const uint32_t o_addr = tmem + lane_sel + (uint32_t)(256 + q * 128);
    unsigned char* sPq = sP + q * PG::P_BYTES;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int kt = 0; kt < n_kt_q[q]; ++kt) {
      if (!pf_wait_warp(&s_full[q], (unsigned)(kt & 1), abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int t0 = kt * BN;
      const bool masked = t0 + BN > p.Skv || (p.causal && t0 + BN - 1 > off + base);   // warp-uniform
      const int lim = (p.causal ? min(p.Skv, pos + 1) : p.Skv) - t0;
      float va[32], vb[32];   // BN == 64: the row of S, read once
      if constexpr (BN == 64) {   // both loads in flight, one wait
        tmem_ld32_nw(s_addr, va);
        tmem_ld32_nw(s_addr + 32, vb);
        tmem_wait_ld();
      }
      float mt;
      if constexpr (BN == 64)
        mt = masked ? pf_max_regs<true>(va, vb, lim) : pf_max_regs<false>(va, vb, lim);
      else
        mt = masked ? pf_row_max<true, BN>(s_addr, lim) : pf_row_max<false, BN>(s_addr, lim);
      mt *= p.scale_log2;
      const bool grow = mt > m_run + 8.f;
      const float m_new = grow ? mt : m_run;
      const float f = grow ? pf_ex2(m_run - m_new) : 1.f;   // 0 on the first tile
      // O_q was last written by P V of the previous tile, which completed
      // before S of this one (one issuing thread, in order)
      if (kt > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(o_addr + c * 32, o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= f;
          tmem_st32(o_addr + c * 32, o);
        }
      }
      m_run = m_new;
      float ls;
      if constexpr (BN == 64) {
        const uint32_t rowp = (uint32_t)((row >> 3) * 1024 + (row & 7) * 128);
        ls = masked ? pf_emit_regs<true, T>(va, 0, sPq, rowp, row & 7, p.scale_log2, -m_run, lim) +
                          pf_emit_regs<true, T>(vb, 1, sPq, rowp, row & 7, p.scale_log2, -m_run, lim)
                    : pf_emit_regs<false, T>(va, 0, sPq, rowp, row & 7, p.scale_log2, -m_run, lim) +
                          pf_emit_regs<false, T>(vb, 1, sPq, rowp, row & 7, p.scale_log2, -m_run, lim);
      } else {
        ls = masked ? pf_emit<true, BN, T>(s_addr, sPq, row, p.scale_log2, -m_run, lim)
                    : pf_emit<false, BN, T>(s_addr, sPq, row, p.scale_log2, -m_run, lim);
      }
      l_run = l_run * f + ls;
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[q]);
    }
    if (n_kt_q[q] > 0) {
      if (!ok || !pf_wait_warp(&o_final[q], 0u, abort_flag)) {
        give_up();
      } else {
        tc_fence_after();
        const float inv = 1.f / l_run;
        const bool row_ok = base + row < p.Sq;
        T* og = reinterpret_cast<T*>(p.out) + b * p.osb + hq * p.osh + (int64_t)(base + row) * p.oss;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(o_addr + c * 32, o);
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
    }
  } else if (warp == 8) {
    // ---- loads (lane 0): both query tiles, then K and V tiles through the ring ----
    if (lane == 0) {
      int c[4];
      pf_expect_tx(q_full, 2 * PG::Q_BYTES);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        pf_coords(p.q_slot_t, p.q_slot_h, p.q_slot_b, q0 + q * PF_ROWS, hq, b, c);
#pragma unroll
        for (int a = 0; a < D / 64; ++a)
          pf_tma4(sQ + q * PG::Q_BYTES + a * PF_ROWS * 128, &maps.q, a * 64, c[1], c[2], c[3], q_full);
      }
      for (int kt = 0; kt < n_kt; ++kt) {
        const int st = kt % PF_STAGES;   // use kt / PF_STAGES of the stage waits for the previous use's release
        if (kt >= PF_STAGES &&
            (*abort_flag || !mbar_wait(&kv_empty[st], (unsigned)((kt / PF_STAGES + 1) & 1)))) {
          give_up();
          break;
        }
        pf_coords(p.kv_slot_t, p.kv_slot_h, p.kv_slot_b, kt * BN, hk, b, c);
        pf_expect_tx(&kv_full[st], 2 * PG::KV_BYTES);
#pragma unroll
        for (int a = 0; a < D / 64; ++a) {
          pf_tma4(sK + st * PG::KV_BYTES + a * BN * 128, &maps.k, a * 64, c[1], c[2], c[3], &kv_full[st]);
          pf_tma4(sV + st * PG::KV_BYTES + a * BN * 128, &maps.v, a * 64, c[1], c[2], c[3], &kv_full[st]);
        }
      }
    }
  } else if (lane == 0) {
    // ---- MMA issue -----------------------------------------------------------------
    const uint32_t idesc_s = umma_idesc_f16(BN, BF, 0), idesc_o = umma_idesc_f16(D, BF, 1);
    const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
    bool ok = !*abort_flag && mbar_wait(q_full, 0u);
    auto issue_s = [&](int q, int kt) {   // S_q = Q_q K(kt)^T, committed to s_full[q]
      const uint32_t a = aQ + q * PG::Q_BYTES, bk = aK + (kt % PF_STAGES) * PG::KV_BYTES;
#pragma unroll
      for (int kc = 0; kc < D / 16; ++kc)   // K step kc: column block kc / 4, 32 bytes per step inside it
        umma_f16(tmem + (uint32_t)(q * 128), umma_desc_sw(a + (kc >> 2) * PF_ROWS * 128 + (kc & 3) * 32, 16, 1024),
                 umma_desc_sw(bk + (kc >> 2) * BN * 128 + (kc & 3) * 32, 16, 1024), idesc_s, kc > 0);
      umma_commit(&s_full[q]);
    };
    auto wait_kv = [&](int kt) {
      if (ok && !(*abort_flag) && mbar_wait(&kv_full[kt % PF_STAGES], (unsigned)((kt / PF_STAGES) & 1))) {
        tc_fence_after();
      } else {
        ok = false;
      }
    };
    if (ok) tc_fence_after();
    if (ok && n_kt > 0) {
      wait_kv(0);
      if (ok) {
#pragma unroll
        for (int q = 0; q < 2; ++q)
          if (n_kt_q[q] > 0) issue_s(q, 0);
      }
    }
    for (int kt = 0; ok && kt < n_kt; ++kt) {
      bool next_ready = false;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (kt < n_kt_q[q]) {
          // P_q(kt) written, S_q(kt) read: O_q += P_q V(kt)
          if (*abort_flag || !mbar_wait(&p_full[q], (unsigned)(kt & 1))) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = aP + q * PG::P_BYTES, bv = aV + (kt % PF_STAGES) * PG::KV_BYTES;
#pragma unroll
          for (int kc = 0; kc < BN / 16; ++kc)
            umma_f16(tmem + (uint32_t)(256 + q * 128),
                     umma_desc_sw(a + (kc >> 2) * PF_ROWS * 128 + (kc & 3) * 32, 16, 1024),
                     umma_desc_sw(bv + kc * 2048, BN * 128, 1024), idesc_o, kt > 0 || kc > 0);
          if (kt == n_kt_q[q] - 1) umma_commit(&o_final[q]);
        }
        if (kt + 1 < n_kt_q[q]) {
          if (!next_ready) {
            wait_kv(kt + 1);
            if (!ok) break;
            next_ready = true;
          }
          issue_s(q, kt + 1);
        }
      }
      if (ok) umma_commit(&kv_empty[kt % PF_STAGES]);   // the stage is free once these products finish
    }
    if (!ok) give_up();
  }
  // every role is done: the last products were awaited by the softmax warps
  // (o_final), or the CTA gave up
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS));
  }
}

}  // namespace hokv
