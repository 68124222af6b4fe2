/*
 * hokv.h -- C ABI of the B200 (sm_100a) compressed-KV hot path.
 *
 * Every entry point takes plain device pointers, sizes and strides plus a
 * cudaStream_t passed as `void*` (NULL = the legacy default stream).  The
 * library writes only caller-provided outputs and allocates nothing; entry
 * points that need scratch space take a `workspace` pointer whose size the
 * matching *_workspace_size() call reports.  Calls are asynchronous on the
 * given stream; a non-zero return value is an hokv_status and
 * hokv_last_error() gives a one-line message (thread-local).  Invalid inputs
 * that only the device can see (a code byte beyond the codebook, a bounded
 * wait that ran out) set a device-side flag that hokv_device_status() reads.
 *
 * Each declaration names the reference (echo313unfolding/helix-online-kv)
 * interface it replaces, as helix_online_kv/<file>:<line>.
 */
#ifndef HOKV_H
#define HOKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HOKV_ABI_VERSION 1

typedef enum hokv_status {
  HOKV_OK = 0,
  HOKV_ERR_INVALID = 1,      /* bad shape, stride, alignment or argument   */
  HOKV_ERR_UNSUPPORTED = 2,  /* valid but outside the compiled variants     */
  HOKV_ERR_CUDA = 3,         /* a CUDA runtime call failed                  */
  HOKV_ERR_TIMEOUT = 4,      /* a bounded device wait ran out               */
  HOKV_ERR_DEVICE_INPUT = 5, /* the device found invalid data (e.g. codes)  */
  HOKV_ERR_WORKSPACE = 6     /* workspace missing or too small              */
} hokv_status;

/* element types */
enum { HOKV_F32 = 0, HOKV_F16 = 1, HOKV_BF16 = 2, HOKV_U8 = 3, HOKV_I32 = 4, HOKV_F64 = 5 };

/* Summation order of an fp32 dot product.  NumPy hands `a @ b` to BLAS; the
 * order depends on the call shape.  GEMV is the order of a (1 x d) @ (d x k)
 * product (sub-table builds and single-vector assignment), SEQ_FMA the order
 * of an (N x d) @ (d x k) product with N >= 5, L16_PAIR the order for
 * 2 <= N <= 4 with d >= 32.  hokv_dot_order_for() picks one for a call shape. */
enum { HOKV_DOT_SEQ_FMA = 0, HOKV_DOT_GEMV = 1, HOKV_DOT_L16_PAIR = 2 };

int hokv_abi_version(void);
const char* hokv_status_string(int status);
const char* hokv_last_error(void);
int hokv_dot_order_for(int64_t n_rows, int dim);
/* Synchronises `stream`, returns and clears the device-side status flag. */
int hokv_device_status(void* stream);

/* ------------------------------------------------------------------------
 * Scalar codebook (Path A / layer state)
 * ---------------------------------------------------------------------- */

/* OnlineCodebook.assign -- codebook.py:86-99.  argmin_j |x - c_j| with the
 * first minimum, x given as f32/f16/bf16 (`dtype`).  n_sets independent
 * problems: values[set*values_stride + i], centroids[set*cent_stride + j],
 * out[set*out_stride + i]. */
int hokv_scalar_assign(const void* values, int dtype, int64_t n, int64_t values_stride,
                       const float* centroids, int k, int64_t cent_stride,
                       uint8_t* out, int64_t out_stride, int n_sets, void* stream);

/* OnlineCodebook.decode -- codebook.py:101-112 (out = centroids[idx]). */
int hokv_scalar_decode(const uint8_t* idx, int64_t n, const float* centroids, int k,
                       float* out, void* stream);

/* OnlineCodebook.finalize_calibration + _fit_kmeans -- codebook.py:57-84,178-221.
 * n_sets independent 1-D k-means fits over data[set*data_stride + i], i < n.
 * Per set writes centroids[set*n_clusters + j] (j < k), k_out[set],
 * iters_out[set], mse_out[set] (f64) and, if non-NULL, the last assignment
 * assign_out[set*n + i]. */
size_t hokv_scalar_kmeans_workspace_size(int64_t n, int n_sets);
int hokv_scalar_kmeans(const float* data, int64_t n, int64_t data_stride, int n_sets,
                       int n_clusters, int max_iters, double rtol,
                       float* centroids, int* k_out, int* iters_out, double* mse_out,
                       uint8_t* assign_out, void* workspace, size_t workspace_bytes,
                       void* stream);

/* OnlineCodebook.maybe_update_centroids EMA step -- codebook.py:146-176 (the
 * caller applies the drift threshold).  centroids updated in place. */
int hokv_scalar_ema(const float* values, int64_t n, float* centroids, int k, float alpha,
                    void* workspace, size_t workspace_bytes, void* stream);
size_t hokv_scalar_ema_workspace_size(int64_t n);

/* quantization_error / cosine_similarity of all three codebooks
 * (codebook.py:114-144, vector_codebook.py:166-183, product_codebook.py:231-250):
 * out4[0] = sum((x - r)^2) in numpy's float32 pairwise order, out4[1] = x.r,
 * out4[2] = |x|^2, out4[3] = |r|^2 (f64).  r is given densely; the workspace
 * holds n floats. */
int hokv_recon_stats(const float* x, const float* r, int64_t n, double* out4,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Path A fused Q.K^T over scalar-VQ codes -- triton_attention.py:25-120.
 * scores[t] = scale * sum_d q[d] * codebook[idx[t*idx_stride + d]], idx u8 or
 * i32 (`idx_dtype`).  accum_f64 != 0 accumulates in f64 (NumPy-tight). */
int hokv_scalar_vq_qkt(const float* q, const void* idx, int idx_dtype, int64_t seq_len,
                       int head_dim, int64_t idx_stride, const float* codebook, int k,
                       float scale, int accum_f64, float* scores, void* stream);

/* ------------------------------------------------------------------------
 * Vector / product codebooks
 * ---------------------------------------------------------------------- */

/* VectorCodebook.assign / ProductCodebook.assign -- vector_codebook.py:95-119,
 * product_codebook.py:118-145.  Vectors x[set][i][M*sub_dim] (f32/f16/bf16,
 * row stride x_row_stride elements), centroids cents[set][s][slot][sub_dim]
 * f32 (cb_slots slots per subspace), counts k[set][s].  Writes
 * out[set][i*out_row_stride + s] = argmin_j ((|x_s|^2 - 2 x_s.c_j) + |c_j|^2).
 * VQ is the case M = 1.  dot_order is one of HOKV_DOT_*. */
int hokv_pq_assign(const void* x, int x_dtype, int64_t n, int64_t x_row_stride,
                   int64_t x_set_stride, int M, int sub_dim,
                   const float* cents, int cb_slots, int64_t cent_set_stride,
                   const int* k, int64_t k_set_stride,
                   uint8_t* out, int64_t out_row_stride, int64_t out_set_stride,
                   int n_sets, int dot_order, void* stream);

/* ProductCodebook.decode / VectorCodebook.decode -- product_codebook.py:147-168. */
int hokv_pq_decode(const uint8_t* codes, int64_t n, int64_t code_row_stride, int M,
                   int sub_dim, const float* cents, int cb_slots, float* out, void* stream);

/* VectorCodebook._fit_kmeans -- vector_codebook.py:185-242, batched over
 * n_sets independent fits (ProductCodebook runs one per subspace,
 * product_codebook.py:86-116).  data[set][i][sub_dim] (row stride
 * data_row_stride, set stride data_set_stride, f32).  Writes
 * cents[set][slot][sub_dim] (cb_slots >= n_clusters), k_out, iters_out,
 * mse_out (f64) per set. */
size_t hokv_vq_kmeans_workspace_size(int64_t n, int sub_dim, int n_sets);
int hokv_vq_kmeans(const float* data, int64_t n, int sub_dim, int64_t data_row_stride,
                   int64_t data_set_stride, int n_sets, int n_clusters, int max_iters,
                   double rtol, float* cents, int cb_slots, int* k_out, int* iters_out,
                   double* mse_out, void* workspace, size_t workspace_bytes,
                   void* stream);

/* ProductCodebook.precompute_distance_tables -- product_codebook.py:172-205
 * (VectorCodebook.precompute_query_scores, vector_codebook.py:136-148, is the
 * case M = 1).  n_q queries q[i][M*sub_dim] f32, each against codebook set
 * set_of_q[i] (NULL: set i).  tables[i][s][j] for j < t_cols; zero where
 * j >= k[s]. */
int hokv_pq_tables(const float* q, int n_q, int M, int sub_dim, const float* cents,
                   int cb_slots, int64_t cent_set_stride, const int* k,
                   int64_t k_set_stride, const int* set_of_q, float* tables, int t_cols,
                   void* stream);

/* ProductCodebook.gather_pq_scores -- product_codebook.py:207-227, times an
 * optional f32 scale (pq_attention_scores, compressed_attention.py:165-184):
 * scores[t] = (((0 + T[0][c0]) + T[1][c1]) + ...) [* scale].  Codes beyond
 * t_cols raise the device flag.  VQ gather_scores is the case M = 1. */
int hokv_pq_gather(const float* tables, int M, int t_cols, const uint8_t* codes,
                   int64_t seq_len, int64_t code_row_stride, int apply_scale, float scale,
                   float* scores, void* stream);

/* Binned value output of Paths B and D -- compressed_attention.py:110-133 and
 * 187-227: bins_s[j] = sum of weights (f64) of tokens with code j in
 * subspace s; out[s*sub_dim + d] = f32(sum_j bins_s[j] * C_s[j][d]). */
int hokv_pq_value_output(const double* weights, int64_t seq_len, const uint8_t* codes,
                         int64_t code_row_stride, int M, int sub_dim, const float* cents,
                         int cb_slots, const int* k, float* out, void* workspace,
                         size_t workspace_bytes, void* stream);
size_t hokv_pq_value_output_workspace_size(int M);

/* ------------------------------------------------------------------------
 * Dense single-query pieces behind the NumPy-facing attention paths
 * ---------------------------------------------------------------------- */

/* standard_attention -- compressed_attention.py:38-55 (and the masked form of
 * Path F, :259-310).  q [D], K/V [S][D] f32.  scores[t] = (q . K[t]) * scale
 * (the product in f64 when mul_f64), -1e9 where mask[t] == 0 (mask may be
 * NULL); store_flags bit 0: scores stored f64, bit 1: out stored f64.  Then
 * w = softmax(scores) and out = sum_t w[t] V[t] (f64 accumulation).
 * workspace: seq_len * 8 bytes. */
int hokv_dense_attention(const float* q, const float* K, const float* V, int head_dim,
                         int64_t seq_len, int mul_f64, double scale, int store_flags,
                         const uint8_t* mask, void* scores, void* out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Exact multi-token attention (prefill, and every step of the layers kept
 * exact): out = softmax(q k^T * scale [causal]) v per query head, with
 * q_heads / kv_heads query heads sharing a KV head.  The reference hands the
 * exact K/V its cache returns to the model's own attention
 * (compressed_cache.py:72-105, parent DynamicCache.update); this replaces that
 * call.  q [batch, q_heads, q_len, head_dim], k/v [batch, kv_heads, kv_len,
 * head_dim], out [batch, q_heads, q_len, head_dim], each through its own
 * element strides (b, h, s; dims contiguous, strides multiples of 8
 * elements, pointers 16-byte aligned).  Causal: query i sits at position
 * kv_len - q_len + i and sees keys 0..that position (kv_len >= q_len).
 * f16/bf16 (HOKV_F16/HOKV_BF16, out in the same type), head_dim 64 or 128;
 * other cases return HOKV_ERR_UNSUPPORTED.  fp32 accumulation; the softmax
 * weights are rounded to the input type before the second product, as
 * FlashAttention does. */
int hokv_prefill_attention(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                           int q_heads, int kv_heads, int q_len, int kv_len, int head_dim, int64_t q_stride_b,
                           int64_t q_stride_h, int64_t q_stride_s, int64_t k_stride_b, int64_t k_stride_h,
                           int64_t k_stride_s, int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
                           int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, float scale,
                           int causal, void* stream);

/* scipy.special.softmax over n values stored f32 (is_f64 = 0) or f64, computed
 * in f64 (compressed_attention.py:31-33). */
int hokv_softmax(const void* in, int is_f64, int64_t n, void* out, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Path F cluster filter -- compressed_attention.py:289-300: keep the top_p
 * clusters by coarse score, mask[t] = code[t] is kept. */
int hokv_prefilter_mask(const float* coarse, int k, const uint8_t* codes, int64_t seq_len,
                        int top_p, uint8_t* mask, void* stream);

/* out[i] = (double)in[i] * scale: a float32 array times a NumPy float64 scalar. */
int hokv_scale_f32_to_f64(const float* in, int64_t n, double scale, double* out, void* stream);

/* ------------------------------------------------------------------------
 * CDC-03 decode attention (Path G) -- compressed_attention.py:315-412, with an
 * exact hot window: tokens [0, S_c) with S_c = max(0, seq_len[b] - hot_window)
 * are cold and ranked by the PQ score (sinks always kept, then the top
 * (top_k - sink) by score, ties to the lower token index); tokens [S_c, seq_len)
 * are always attended.  Exact softmax(q.K^T * scale) . V over the union.
 * hot_window = 0 is hybrid_pq_attention itself.
 * ---------------------------------------------------------------------- */
typedef struct hokv_cdc03_args {
  int batch;        /* B sequences                                          */
  int kv_heads;     /* H_kv                                                 */
  int q_per_kv;     /* G = H_q / H_kv, 1..8 (GQA group)                     */
  int head_dim;     /* D: 32, 64, 128 or 256                                */
  int n_subspaces;  /* M real PQ subspaces                                   */
  int sub_dim;      /* dims per subspace, M * sub_dim <= D (0: D / M)       */
  int code_bytes;   /* bytes per token in the code store: 4, 8, 16, 32 >= M */
  int cb_slots;     /* centroid slots per subspace in the codebook store    */
  int top_k;        /* CDC-03 budget, sinks included                        */
  int sink_tokens;
  int hot_window;
  float scale;
  int lut_order;    /* HOKV_DOT_* of the sub-table dot products (GEMV)      */
  /* q[b][hq][d], hq = h*G + g; out likewise                                */
  const void* q; int q_dtype; int64_t q_stride_b;
  void* out; int out_dtype; int64_t out_stride_b;
  /* exact store k/v[b][h][t][d] (f16, bf16 or f32), strides in elements   */
  const void* k; const void* v; int kv_dtype; int64_t kv_stride_b, kv_stride_h;
  int64_t capacity; /* tokens per (b, h) in the stores (multiple of 16)     */
  /* PQ codes codes[b][h][t][code_bytes], strides in bytes (16-B aligned)   */
  const uint8_t* codes; int64_t code_stride_b, code_stride_h;
  /* codebook cb[b][h][s][slot][sub_dim] f32, counts cb_k[b][h][s] int32    */
  const float* codebook; int64_t cb_stride_b, cb_stride_h;
  const int* cb_k; int64_t cbk_stride_b, cbk_stride_h;
  const int* seq_len; /* [B] device int32, tokens valid per sequence       */
  /* optional outputs (NULL to skip): selected cold tokens per query head,
   * sel_idx/sel_score[b][hq][max(top_k, sink_tokens)] (unsorted, -1 / -inf
   * padded) and sel_count[b][hq]                                          */
  int* sel_idx; float* sel_score; int* sel_count;
  void* workspace; size_t workspace_bytes;
} hokv_cdc03_args;

/* Scratch bytes the stages below need for `a`.  HOKV_ERR_UNSUPPORTED when
 * capacity - hot_window exceeds 248 chunks of 2048 tokens (507,904), where the
 * candidate stage's 16-bit histogram counters could overflow. */
int hokv_cdc03_workspace_size(const hokv_cdc03_args* a, size_t* bytes);
/* Both stages below, in order, on `stream`. */
int hokv_cdc03_decode(const hokv_cdc03_args* a, void* stream);
/* Stage 1 (precompute_distance_tables + gather_pq_scores + the first half of
 * the selection, product_codebook.py:172-227, compressed_attention.py:362-383):
 * build the sub-tables, stream the PQ codes scored with quantised 16-bit
 * tables, and write, per (sequence, KV head, chunk, query head), the tokens
 * that can still reach the top-k with their exact scores (selection keys)
 * into the workspace. */
int hokv_cdc03_candidates(const hokv_cdc03_args* a, void* stream);
/* Stage 2 (compressed_attention.py:384-403): exact top-k of the candidate
 * keys with sinks, softmax attention over the selected cold tokens plus the
 * hot window.  Reads the workspace stage 1 wrote. */
int hokv_cdc03_attend(const hokv_cdc03_args* a, void* stream);

/* hokv_cdc03_decode for callers that cannot allocate device memory.  No
 * counterpart in the reference (its NumPy path allocates as it goes).
 *
 * Who needs it: a plugin loaded by a serving runtime that reserves nearly all
 * HBM for its own KV pool at start-up and hands its plugins no allocator.
 * There cudaMalloc either fails for lack of memory or, since it synchronises
 * with the device, stalls a decode step that must not block; the caller also
 * has no spare buffer to pass as `workspace`.
 *
 * What it does: the same two stages as hokv_cdc03_decode, with the scratch
 * taken from one array of HOKV_CDC03_NOALLOC_SCRATCH_BYTES that the library
 * itself holds on every device it is loaded on, until the process exits.
 * a->workspace and a->workspace_bytes are ignored; inputs and outputs stay
 * the caller's.  A configuration whose hokv_cdc03_workspace_size exceeds the
 * limit is rejected with HOKV_ERR_WORKSPACE before anything is launched
 * (16 MiB covers 8 sequences x 8 KV heads x 4 query heads at 16K tokens with
 * 16 subspaces).  The library allocates nothing on this path.
 *
 * The first call on a device looks up the array's device address (with that
 * device current) and keeps it; make that first call before any stream
 * capture.  All calls on a device share the array and nothing in it has to
 * start at zero: each call writes every scratch byte it later reads, so the
 * previous call's contents are harmless.  Calls that overlap on the GPU
 * (other streams, other host threads) race on the array: order them. */
#define HOKV_CDC03_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int hokv_cdc03_decode_noalloc(const hokv_cdc03_args* a, void* stream);

/* ------------------------------------------------------------------------
 * Tier aging (AgingPolicy.tier_boundary, aging_policy.py:42-56, applied in
 * place): for every (b, h) assign the PQ code of each token in
 * [cold_from[b], cold_to[b]) from the exact store and write it into the
 * code store.  The reference computes the boundary but never moves tokens
 * (compressed_cache.py:51); this is the device-side demotion step.
 * Uses the store fields of `a` (k, kv_dtype, strides, capacity, codes,
 * codebook, cb_k, n_subspaces, sub_dim, code_bytes, cb_slots); cold_from and
 * cold_to are device int32 [batch].  dot_order as for hokv_pq_assign
 * (hokv_dot_order_for(1, sub_dim) reproduces a one-token assign, the decode
 * step's case).  A range outside [0, capacity] sets HOKV_ERR_DEVICE_INPUT
 * in the device status and leaves that sequence's codes untouched.
 * ---------------------------------------------------------------------- */
int hokv_age_tokens(const hokv_cdc03_args* a, const int* cold_from, const int* cold_to,
                    int dot_order, void* stream);

/* ------------------------------------------------------------------------
 * Profiling.  No counterpart in the reference.  A library built with
 * -DHOKV_STAMPS records, in the two decode kernels, the %globaltimer value
 * (ns) at each phase boundary, thread 0 of every CTA: out[k][cta][phase] for
 * kernel k (0: candidate stage, cta = blockIdx.y * gridDim.x + blockIdx.x;
 * 1: attention stage, cta = blockIdx.x; 2: reserved), 4096 CTAs x 16 phases
 * each, the last launch's values.  n_values must be at least 3 * 4096 * 16.
 * The product build returns HOKV_ERR_UNSUPPORTED.
 * ---------------------------------------------------------------------- */
int hokv_phase_stamps(uint64_t* out, size_t n_values);

#ifdef __cplusplus
}
#endif
#endif /* HOKV_H */
