// hokv_lib.cu -- C ABI of the B200 compressed-KV hot path (declared in
// include/hokv.h).  One translation unit: all kernels share the device status
// flag below.  Host code validates arguments, picks template variants and
// launches on the caller's stream; it allocates nothing.
#include <cub/device/device_radix_sort.cuh>

#include "hokv_common.cuh"
#include "cdc03.cuh"
#include "codec.cuh"
#include "dense.cuh"
#include "assign_tc.cuh"
#include "prefill.cuh"

#include <map>
#include <mutex>
#include <string>
#include <utility>

namespace hokv {


static thread_local std::string t_err;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return HOKV_OK;
}

static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
static inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
static inline bool is_pow2_in(int v, int lo, int hi) { return v >= lo && v <= hi && (v & (v - 1)) == 0; }
static inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Raise a kernel's dynamic shared-memory limit once per (device, kernel), so
// calls made later (e.g. inside CUDA-graph capture) issue no attribute change.
template <typename K>
static int ensure_smem(K kernel, size_t bytes) {
  // Static plus dynamic shared memory above 48 KB needs the opt-in even when
  // the dynamic part alone is below it, so raise the limit for any request.
  if (bytes == 0) return HOKV_OK;
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return HOKV_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "cudaFuncSetAttribute(%zu B): %s", bytes, cudaGetErrorString(e));
  done[key] = bytes;
  return HOKV_OK;
}

// Extended launch: `pdl` allows a programmatic (early) start behind the
// previous kernel of the stream; cluster_x > 0 groups cluster_x consecutive
// blocks along x into one thread-block cluster.
template <typename K>
static int launch_ex(K kernel, dim3 grid, dim3 block, size_t sm, cudaStream_t st, const Cdc03P& p, const char* what,
                     bool pdl, int cluster_x = 0) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = sm;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 0) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // do not leave the error for the next call to report
    return fail(HOKV_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  }
  return check_launch(what);
}

// Stage 1: one thread-block cluster of min(chunks, K6_CLUSTER_MAX) CTAs per
// unit builds the tables and streams the candidates (ordinary launch: it
// reads the queries).
template <int CS, int GT>
static int launch_stage1(const Cdc03P& p, cudaStream_t st) {
  using Q = QGeo<CS, GT>;
  if (p.chunk != K6_CHUNK) return fail(HOKV_ERR_INVALID, "cdc03: chunk %d != %d", p.chunk, K6_CHUNK);
  const size_t sm = Q::BYTES + (size_t)GT * (HWORDS + 32) * 4;   // table image, histograms, coarse counts
  const int R = std::min(p.n_chunks, K6_CLUSTER_MAX);
  if (int e = ensure_smem(k6_candidates<CS, GT>, sm)) return e;
  return launch_ex(k6_candidates<CS, GT>, dim3((unsigned)R, (unsigned)(p.B * p.Hkv)), dim3(K6_THREADS), sm, st, p,
                   "k6_candidates", false, R);
}

static int dispatch_stage1(const Cdc03P& p, cudaStream_t st) {
#define HOKV_S1(cs_, gt_) if (p.CS == cs_ && p.GT == gt_) return launch_stage1<cs_, gt_>(p, st);
  HOKV_S1(4, 1) HOKV_S1(4, 2) HOKV_S1(4, 4) HOKV_S1(4, 8)
  HOKV_S1(8, 1) HOKV_S1(8, 2) HOKV_S1(8, 4) HOKV_S1(8, 8)
  HOKV_S1(16, 1) HOKV_S1(16, 2) HOKV_S1(16, 4) HOKV_S1(16, 8)
  HOKV_S1(32, 1) HOKV_S1(32, 2) HOKV_S1(32, 4)
#undef HOKV_S1
  return fail(HOKV_ERR_UNSUPPORTED, "cdc03: no candidate-stage variant for code_bytes=%d group=%d", p.CS, p.GT);
}

static int qimg_bytes_for(int CS, int GT) {
  const int ew = GT <= 2 ? 4 : (GT == 4 ? 8 : 16);
  const int cols = 128 / ew;
  const int rb = CS > cols ? CS / cols : 1;
  return rb * 256 * 128;
}

// Stage 2: K7, programmatic launch (hot-window attention overlaps K6).
template <int D, typename KVT>
static int launch_k7(const Cdc03P& p, cudaStream_t st) {
  const size_t sm = (size_t)p.M * 1024 + (size_t)K7_CAP * 8 + 1024 + (size_t)TOPK_MAX * 4 +
                    (size_t)(K7_THREADS / 32) * (D + 2) * 4 + (size_t)K7_KEYCACHE_BYTES;
  if (int e = ensure_smem(k7_select_attend<D, KVT>, sm)) return e;
  return launch_ex(k7_select_attend<D, KVT>, dim3((unsigned)(p.B * p.Hkv * p.G)), dim3(K7_THREADS), sm, st, p,
                   "k7_select_attend", true);
}

template <typename KVT>
static int dispatch_k7_t(const Cdc03P& p, cudaStream_t st) {
  switch (p.D) {
    case 32: return launch_k7<32, KVT>(p, st);
    case 64: return launch_k7<64, KVT>(p, st);
    case 128: return launch_k7<128, KVT>(p, st);
    case 256: return launch_k7<256, KVT>(p, st);
  }
  return fail(HOKV_ERR_UNSUPPORTED, "cdc03: head_dim %d", p.D);
}

static int dispatch_k7(const Cdc03P& p, int kv_dtype, cudaStream_t st) {
  if (kv_dtype == HOKV_BF16) return dispatch_k7_t<__nv_bfloat16>(p, st);
  if (kv_dtype == HOKV_F16) return dispatch_k7_t<__half>(p, st);
  if (kv_dtype == HOKV_F32) return dispatch_k7_t<float>(p, st);
  return fail(HOKV_ERR_UNSUPPORTED, "cdc03: kv dtype %d", kv_dtype);
}

}  // namespace hokv

using namespace hokv;

extern "C" {

int hokv_abi_version(void) { return HOKV_ABI_VERSION; }

const char* hokv_status_string(int s) {
  switch (s) {
    case HOKV_OK: return "ok";
    case HOKV_ERR_INVALID: return "invalid argument";
    case HOKV_ERR_UNSUPPORTED: return "unsupported configuration";
    case HOKV_ERR_CUDA: return "CUDA error";
    case HOKV_ERR_TIMEOUT: return "bounded device wait ran out";
    case HOKV_ERR_DEVICE_INPUT: return "device found invalid input";
    case HOKV_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

const char* hokv_last_error(void) { return t_err.c_str(); }

int hokv_dot_order_for(int64_t n_rows, int dim) { return dot_order_for(n_rows, dim); }

int hokv_device_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(S(stream));
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "stream sync: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(int));
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_dev_status, &zero, sizeof(int));
    return fail(v, "device reported: %s", hokv_status_string(v));
  }
  return HOKV_OK;
}

// ---------------------------------------------------------------- scalar ---
int hokv_scalar_assign(const void* values, int dtype, int64_t n, int64_t values_stride, const float* centroids,
                       int k, int64_t cent_stride, uint8_t* out, int64_t out_stride, int n_sets, void* stream) {
  HOKV_REQUIRE(n >= 0 && n_sets >= 1, "scalar_assign: n=%lld n_sets=%d", (long long)n, n_sets);
  HOKV_REQUIRE(k >= 1 && k <= 256, "scalar_assign: k=%d not in [1, 256]", k);
  HOKV_REQUIRE(dtype == HOKV_F32 || dtype == HOKV_F16 || dtype == HOKV_BF16, "scalar_assign: dtype %d", dtype);
  if (n == 0) return HOKV_OK;
  HOKV_REQUIRE(values && centroids && out, "scalar_assign: null pointer");
  dim3 grid((unsigned)std::min<int64_t>(cdiv(n, 256), 1024), (unsigned)n_sets);
  k_scalar_assign<<<grid, 256, 0, S(stream)>>>(values, dtype, n, values_stride, centroids, k, cent_stride, out,
                                               out_stride);
  return check_launch("k_scalar_assign");
}

int hokv_scalar_decode(const uint8_t* idx, int64_t n, const float* centroids, int k, float* out, void* stream) {
  HOKV_REQUIRE(n >= 0 && k >= 1 && k <= 256, "scalar_decode: n=%lld k=%d", (long long)n, k);
  if (n == 0) return HOKV_OK;
  k_scalar_decode<<<(unsigned)std::min<int64_t>(cdiv(n, 256), 4096), 256, 0, S(stream)>>>(idx, n, centroids, k, out);
  return check_launch("k_scalar_decode");
}

static size_t cub_sort_bytes(int64_t n) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortKeys(nullptr, bytes, (const float*)nullptr, (float*)nullptr, (int)n);
  return bytes;
}

static inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

size_t hokv_scalar_kmeans_workspace_size(int64_t n, int n_sets) {
  return a256((size_t)n * n_sets * 4) + a256((size_t)n * n_sets) + a256((size_t)n * n_sets * 4) + a256(cub_sort_bytes(n));
}

int hokv_scalar_kmeans(const float* data, int64_t n, int64_t data_stride, int n_sets, int n_clusters, int max_iters,
                       double rtol, float* centroids, int* k_out, int* iters_out, double* mse_out,
                       uint8_t* assign_out, void* workspace, size_t workspace_bytes, void* stream) {
  HOKV_REQUIRE(n >= 1 && n < (1ll << 31), "scalar_kmeans: n=%lld", (long long)n);
  HOKV_REQUIRE(n_sets >= 1 && n_clusters >= 1 && n_clusters <= 256, "scalar_kmeans: n_sets=%d n_clusters=%d", n_sets,
               n_clusters);
  HOKV_REQUIRE(max_iters >= 0, "scalar_kmeans: max_iters=%d", max_iters);
  const size_t need = hokv_scalar_kmeans_workspace_size(n, n_sets);
  if (!workspace || workspace_bytes < need)
    return fail(HOKV_ERR_WORKSPACE, "scalar_kmeans: workspace %zu < %zu", workspace_bytes, need);
  unsigned char* w = static_cast<unsigned char*>(workspace);
  float* sorted = reinterpret_cast<float*>(w);
  w += a256((size_t)n * n_sets * 4);
  uint8_t* asg = w;
  w += a256((size_t)n * n_sets);
  float* mem = reinterpret_cast<float*>(w);
  w += a256((size_t)n * n_sets * 4);
  size_t tb = cub_sort_bytes(n);
  for (int s = 0; s < n_sets; ++s) {
    cudaError_t e = cub::DeviceRadixSort::SortKeys(w, tb, data + (int64_t)s * data_stride, sorted + (int64_t)s * n,
                                                   (int)n, 0, 32, S(stream));
    if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "scalar_kmeans sort: %s", cudaGetErrorString(e));
  }
  if (max_iters == 0) max_iters = 0;
  k_scalar_kmeans<<<n_sets, 1024, 0, S(stream)>>>(data, n, data_stride, sorted, n_clusters, max_iters, rtol,
                                                  centroids, k_out, iters_out, mse_out, asg, mem, assign_out);
  return check_launch("k_scalar_kmeans");
}

size_t hokv_scalar_ema_workspace_size(int64_t n) { return a256((size_t)n) + a256((size_t)n * 4); }

int hokv_scalar_ema(const float* values, int64_t n, float* centroids, int k, float alpha, void* workspace,
                    size_t workspace_bytes, void* stream) {
  HOKV_REQUIRE(n >= 1 && k >= 1 && k <= 256, "scalar_ema: n=%lld k=%d", (long long)n, k);
  if (!workspace || workspace_bytes < hokv_scalar_ema_workspace_size(n))
    return fail(HOKV_ERR_WORKSPACE, "scalar_ema: workspace too small");
  uint8_t* asg = static_cast<uint8_t*>(workspace);
  float* mem = reinterpret_cast<float*>(asg + a256((size_t)n));
  k_scalar_ema<<<1, 1024, 0, S(stream)>>>(values, n, centroids, k, alpha, asg, mem);
  return check_launch("k_scalar_ema");
}

int hokv_recon_stats(const float* x, const float* r, int64_t n, double* out4, void* workspace,
                     size_t workspace_bytes, void* stream) {
  HOKV_REQUIRE(n >= 1 && x && r && out4, "recon_stats: bad arguments");
  if (!workspace || workspace_bytes < (size_t)n * 4) return fail(HOKV_ERR_WORKSPACE, "recon_stats: workspace");
  float* tmp = static_cast<float*>(workspace);
  k_recon_stats<<<1, 1024, 0, S(stream)>>>(x, r, n, tmp, out4);
  return check_launch("k_recon_stats");
}

int hokv_scalar_vq_qkt(const float* q, const void* idx, int idx_dtype, int64_t seq_len, int head_dim,
                       int64_t idx_stride, const float* codebook, int k, float scale, int accum_f64, float* scores,
                       void* stream) {
  HOKV_REQUIRE(seq_len >= 0 && head_dim >= 1 && head_dim <= 4096, "scalar_vq_qkt: seq_len=%lld head_dim=%d",
               (long long)seq_len, head_dim);
  HOKV_REQUIRE(k >= 1 && k <= 256, "scalar_vq_qkt: k=%d", k);
  HOKV_REQUIRE(idx_dtype == HOKV_U8 || idx_dtype == HOKV_I32, "scalar_vq_qkt: idx dtype %d", idx_dtype);
  if (seq_len == 0) return HOKV_OK;
  if (idx_dtype == HOKV_U8 && head_dim % 16 == 0 && (head_dim / 16) <= 32 && ((head_dim / 16) & (head_dim / 16 - 1)) == 0 &&
      idx_stride % 16 == 0 && aligned(idx, 16)) {
    // coalesced 16-byte code loads, lanes of a token combined by shuffles
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int lpt = head_dim / 16;
    const int64_t per_cta = 8 * (32 / lpt);   // warps x tokens per step
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(seq_len, per_cta), (int64_t)n_sm * 6));
#define HOKV_QKT(L_)                                                                                              \
  if (lpt == L_) {                                                                                              \
    if (accum_f64)                                                                                              \
      k_scalar_vq_qkt_u8v<L_, double><<<grid, 256, 0, S(stream)>>>(q, (const uint8_t*)idx, seq_len, idx_stride,  \
                                                                    codebook, k, scale, scores);                \
    else                                                                                                        \
      k_scalar_vq_qkt_u8v<L_, float><<<grid, 256, 0, S(stream)>>>(q, (const uint8_t*)idx, seq_len, idx_stride,   \
                                                                   codebook, k, scale, scores);                 \
    return check_launch("k_scalar_vq_qkt_u8v");                                                                 \
  }
    HOKV_QKT(1) HOKV_QKT(2) HOKV_QKT(4) HOKV_QKT(8) HOKV_QKT(16) HOKV_QKT(32)
#undef HOKV_QKT
  }
  const unsigned grid = (unsigned)cdiv(seq_len, 256);
  const size_t sm = (size_t)head_dim * 4;
  if (idx_dtype == HOKV_U8) {
    if (accum_f64)
      k_scalar_vq_qkt<uint8_t, double><<<grid, 256, sm, S(stream)>>>(q, (const uint8_t*)idx, seq_len, head_dim,
                                                                      idx_stride, codebook, k, scale, scores);
    else
      k_scalar_vq_qkt<uint8_t, float><<<grid, 256, sm, S(stream)>>>(q, (const uint8_t*)idx, seq_len, head_dim,
                                                                     idx_stride, codebook, k, scale, scores);
  } else {
    if (accum_f64)
      k_scalar_vq_qkt<int32_t, double><<<grid, 256, sm, S(stream)>>>(q, (const int32_t*)idx, seq_len, head_dim,
                                                                      idx_stride, codebook, k, scale, scores);
    else
      k_scalar_vq_qkt<int32_t, float><<<grid, 256, sm, S(stream)>>>(q, (const int32_t*)idx, seq_len, head_dim,
                                                                     idx_stride, codebook, k, scale, scores);
  }
  return check_launch("k_scalar_vq_qkt");
}

// ------------------------------------------------------------ vector / PQ ---
}  // extern "C"

namespace hokv {
// HOKV_OK when launched, -1 when no tensor-core variant fits (the caller
// takes the CUDA-core kernels), else an error status.
template <int SD, bool SPLIT>
static int launch_assign_tc_sd(const void* x, int x_dtype, int64_t n, int64_t xrs, int64_t xss, int M,
                               const float* cents, int slots, int64_t css, const int* k, int64_t kss, uint8_t* out,
                               int64_t ors, int64_t oss, int n_sets, cudaStream_t st) {
  using TG = TcGeo<SD, SPLIT>;
  if constexpr (TG::STAGES == 0) {
    return -1;
  } else {
    // at most two CTAs per SM: each holds TC_TMEM_COLS of the 512 tensor-memory columns
    const size_t sm = std::max<size_t>((size_t)TG::SMEM, 80 * 1024);
    if (int e = ensure_smem(k_pq_assign_tc<SD, SPLIT>, sm)) return e;
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int64_t n_tiles = cdiv(n, TC_ROWS);
    const int64_t pairs = (int64_t)M * n_sets;
    // persistent CTAs: every (set, subspace) pair split into tile groups,
    // about two CTAs per SM over the whole grid
    const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(n_tiles, cdiv(2 * n_sm, pairs)));
    if (pairs * groups > (int64_t)INT32_MAX) return fail(HOKV_ERR_UNSUPPORTED, "pq_assign: grid too large");
    k_pq_assign_tc<SD, SPLIT><<<(unsigned)(pairs * groups), TC_CTA, sm, st>>>(
        x, x_dtype, n, xrs, xss, cents, slots, css, k, kss, out, ors, oss, M, n_sets, (int)groups);
    return check_launch("k_pq_assign_tc");
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time libcuda dependency).
typedef CUresult (*PfEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PfEncodeFn pf_encoder() {
  static std::once_flag once;
  static PfEncodeFn fn = nullptr;
  std::call_once(once, []() {
    cudaDriverEntryPointQueryResult qr;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfEncodeFn>(f);
  });
  return fn;
}

// A [batch, heads, tokens, dim] tensor with element strides (sb, sh, ss) as a
// 4-D tensor map for 128-byte-swizzled boxes of 64 dims x `box_rows` tokens:
// dim 0 = the head dim, dims 1-3 = tokens, heads, batch sorted by stride (a
// dim of extent 1 takes the stride its place needs); *slot_* return each
// dim's position.  HOKV_ERR_UNSUPPORTED when the strides do not nest.
static int pf_tensor_map(CUtensorMap* m, const void* base, int dtype, int dim, int64_t tokens, int64_t ss,
                         int64_t heads, int64_t sh, int64_t batch, int64_t sb, int box_rows, int* slot_t,
                         int* slot_h, int* slot_b) {
  PfEncodeFn enc = pf_encoder();
  if (!enc) return fail(HOKV_ERR_CUDA, "prefill_attention: cuTensorMapEncodeTiled unavailable");
  int64_t ext[3] = {tokens, heads, batch}, str[3] = {ss, sh, sb};
  int order[3] = {0, 1, 2};
  for (int i = 0; i < 3; ++i)   // ascending stride; extent-1 dims last
    for (int j = i + 1; j < 3; ++j) {
      const bool sw = (ext[order[j]] > 1 && ext[order[i]] == 1) ||
                      ((ext[order[j]] > 1) == (ext[order[i]] > 1) && str[order[j]] < str[order[i]]);
      if (sw) std::swap(order[i], order[j]);
    }
  cuuint64_t gdim[4] = {(cuuint64_t)dim, 0, 0, 0};
  cuuint64_t gstr[3];
  int64_t need = (int64_t)dim;   // elements the next stride must cover
  for (int i = 0; i < 3; ++i) {
    const int d = order[i];
    gdim[i + 1] = (cuuint64_t)ext[d];
    int64_t s = str[d];
    if (ext[d] == 1) s = need;
    if (s < need)
      return fail(HOKV_ERR_UNSUPPORTED, "prefill_attention: strides (%lld, %lld, %lld) do not nest",
                  (long long)ss, (long long)sh, (long long)sb);
    gstr[i] = (cuuint64_t)s * 2;
    need = s * ext[d];
    if (d == 0) *slot_t = i + 1;
    if (d == 1) *slot_h = i + 1;
    if (d == 2) *slot_b = i + 1;
  }
  cuuint32_t es[4] = {1, 1, 1, 1};
  cuuint32_t bx[4] = {64, 1, 1, 1};   // 64 dims x box_rows tokens x 1 head x 1 sequence
  bx[*slot_t] = (cuuint32_t)box_rows;
  const CUresult r = enc(m, dtype == HOKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         4, const_cast<void*>(base), gdim, gstr, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HOKV_ERR_UNSUPPORTED, "prefill_attention: tensor map encode failed (%d)", (int)r);
  return HOKV_OK;
}

static int launch_assign_tc(const void* x, int x_dtype, int64_t n, int64_t xrs, int64_t xss, int M, int sd,
                            const float* cents, int slots, int64_t css, const int* k, int64_t kss, uint8_t* out,
                            int64_t ors, int64_t oss, int n_sets, cudaStream_t st) {
  const bool split = x_dtype == HOKV_F32;
#define HOKV_TC(sd_)                                                                                              \
  if (sd == sd_)                                                                                                 \
    return split ? launch_assign_tc_sd<sd_, true>(x, x_dtype, n, xrs, xss, M, cents, slots, css, k, kss, out, ors, \
                                                  oss, n_sets, st)                                              \
                 : launch_assign_tc_sd<sd_, false>(x, x_dtype, n, xrs, xss, M, cents, slots, css, k, kss, out,    \
                                                   ors, oss, n_sets, st);
  HOKV_TC(4) HOKV_TC(8) HOKV_TC(16) HOKV_TC(32) HOKV_TC(64)
#undef HOKV_TC
  return -1;
}
}  // namespace hokv

extern "C" {

int hokv_pq_assign(const void* x, int x_dtype, int64_t n, int64_t x_row_stride, int64_t x_set_stride, int M,
                   int sub_dim, const float* cents, int cb_slots, int64_t cent_set_stride, const int* k,
                   int64_t k_set_stride, uint8_t* out, int64_t out_row_stride, int64_t out_set_stride, int n_sets,
                   int dot_order, void* stream) {
  HOKV_REQUIRE(n >= 0 && M >= 1 && sub_dim >= 1 && n_sets >= 1, "pq_assign: n=%lld M=%d sub_dim=%d", (long long)n, M,
               sub_dim);
  HOKV_REQUIRE(cb_slots >= 1 && cb_slots <= 256, "pq_assign: cb_slots=%d", cb_slots);
  HOKV_REQUIRE(dot_order >= 0 && dot_order <= 2, "pq_assign: dot_order=%d", dot_order);
  HOKV_REQUIRE(x_dtype == HOKV_F32 || x_dtype == HOKV_F16 || x_dtype == HOKV_BF16, "pq_assign: dtype %d", x_dtype);
  HOKV_REQUIRE(sub_dim <= 1024, "pq_assign: sub_dim %d > 1024", sub_dim);
  if (n == 0) return HOKV_OK;
  if (dot_order == DOT_SEQ_FMA && n >= TC_MIN_ROWS &&
      (sub_dim == 4 || sub_dim == 8 || sub_dim == 16 || sub_dim == 32 || sub_dim == 64) && M <= 65535 &&
      n_sets <= 65535) {
    // prefill-sized batches: tensor-core screen, exact rescoring
    const int st = launch_assign_tc(x, x_dtype, n, x_row_stride, x_set_stride, M, sub_dim, cents, cb_slots,
                                    cent_set_stride, k, k_set_stride, out, out_row_stride, out_set_stride, n_sets,
                                    S(stream));
    if (st != -1) return st;
  }
  if (dot_order == DOT_SEQ_FMA && (sub_dim == 4 || sub_dim == 8) && n >= 64) {
    // mid-sized batches: register-tiled kernel, same arithmetic (below 64
    // rows most of its threads would have no row; the warp-per-vector kernel
    // below splits the centroids over the lanes instead)
    HOKV_REQUIRE(cdiv(n, 1024) < (1ll << 31) && M <= 65535 && n_sets <= 65535, "pq_assign: grid too large");
    const dim3 grid((unsigned)cdiv(n, 1024), (unsigned)M, (unsigned)n_sets);
#define HOKV_PQA(sd_, v_)                                                                                          \
  if (sub_dim == sd_) {                                                                                          \
    k_pq_assign_seq<sd_, v_><<<grid, 256, 0, S(stream)>>>(x, x_dtype, n, x_row_stride, x_set_stride, cents,       \
                                                        cb_slots, cent_set_stride, k, k_set_stride, out,          \
                                                        out_row_stride, out_set_stride);                          \
    return check_launch("k_pq_assign_seq");                                                                      \
  }
    HOKV_PQA(4, 4) HOKV_PQA(8, 4)
#undef HOKV_PQA
  }
  size_t sm = (256 + 8 * (size_t)sub_dim) * 4;
  const size_t cb_sm = (size_t)cb_slots * (sub_dim + 1) * 4;
  int use_smem = (sm + cb_sm) <= 160 * 1024;
  if (use_smem) sm += cb_sm;
  if (int st = ensure_smem(k_pq_assign, sm)) return st;
  HOKV_REQUIRE(cdiv(n, 64) < (1ll << 31) && M <= 65535 && n_sets <= 65535, "pq_assign: grid too large");
  dim3 grid((unsigned)cdiv(n, 64), (unsigned)M, (unsigned)n_sets);
  k_pq_assign<<<grid, 256, sm, S(stream)>>>(x, x_dtype, n, x_row_stride, x_set_stride, M, sub_dim, cents, cb_slots,
                                            cent_set_stride, k, k_set_stride, out, out_row_stride, out_set_stride,
                                            dot_order, use_smem);
  return check_launch("k_pq_assign");
}

int hokv_pq_decode(const uint8_t* codes, int64_t n, int64_t code_row_stride, int M, int sub_dim, const float* cents,
                   int cb_slots, float* out, void* stream) {
  HOKV_REQUIRE(n >= 0 && M >= 1 && sub_dim >= 1 && cb_slots >= 1 && cb_slots <= 256, "pq_decode: bad shape");
  if (n == 0) return HOKV_OK;
  const int64_t total = n * M * sub_dim;
  k_pq_decode<<<(unsigned)std::min<int64_t>(cdiv(total, 256), 8192), 256, 0, S(stream)>>>(codes, n, code_row_stride,
                                                                                           M, sub_dim, cents,
                                                                                           cb_slots, out);
  return check_launch("k_pq_decode");
}

static size_t vq_ws_per_set(int64_t n, int sd, int n_clusters) {
  // asg, x2, mem (4 B each), keys (8 B, aligned), err (n*sd f32), Cn (k*sd f32)
  size_t b = 12 * (size_t)n;
  b += (8 - b % 8) % 8;
  b += 8 * (size_t)n + 4 * (size_t)n * sd + 4 * (size_t)n_clusters * sd;
  return a256(b);
}

size_t hokv_vq_kmeans_workspace_size(int64_t n, int sub_dim, int n_sets) {
  return vq_ws_per_set(n, sub_dim, 256) * (size_t)n_sets;
}

int hokv_vq_kmeans(const float* data, int64_t n, int sub_dim, int64_t data_row_stride, int64_t data_set_stride,
                   int n_sets, int n_clusters, int max_iters, double rtol, float* cents, int cb_slots, int* k_out,
                   int* iters_out, double* mse_out, void* workspace, size_t workspace_bytes, void* stream) {
  HOKV_REQUIRE(n >= 1 && n <= 8192, "vq_kmeans: n=%lld not in [1, 8192]", (long long)n);
  HOKV_REQUIRE(sub_dim >= 1 && n_sets >= 1, "vq_kmeans: sub_dim=%d n_sets=%d", sub_dim, n_sets);
  HOKV_REQUIRE(n_clusters >= 1 && n_clusters <= 256 && cb_slots >= n_clusters && cb_slots <= 256,
               "vq_kmeans: n_clusters=%d cb_slots=%d", n_clusters, cb_slots);
  if ((int64_t)n_clusters * sub_dim > 32768)
    return fail(HOKV_ERR_UNSUPPORTED, "vq_kmeans: n_clusters*sub_dim=%lld exceeds 32768",
                (long long)n_clusters * sub_dim);
  const size_t per = vq_ws_per_set(n, sub_dim, 256);
  if (!workspace || workspace_bytes < per * (size_t)n_sets)
    return fail(HOKV_ERR_WORKSPACE, "vq_kmeans: workspace %zu < %zu", workspace_bytes, per * (size_t)n_sets);
  int npow = 1;
  while (npow < n) npow <<= 1;
  const size_t sm = (size_t)n_clusters * sub_dim * 4 * 2 + (size_t)n_clusters * 4 + (size_t)npow * 4;
  if (int st = ensure_smem(k_vq_kmeans, sm)) return st;
  k_vq_kmeans<<<n_sets, 1024, sm, S(stream)>>>(data, n, sub_dim, data_row_stride, data_set_stride, n_clusters,
                                              max_iters, rtol, cents, cb_slots, k_out, iters_out, mse_out,
                                              static_cast<unsigned char*>(workspace), (int64_t)per);
  return check_launch("k_vq_kmeans");
}

int hokv_pq_tables(const float* q, int n_q, int M, int sub_dim, const float* cents, int cb_slots,
                   int64_t cent_set_stride, const int* k, int64_t k_set_stride, const int* set_of_q, float* tables,
                   int t_cols, void* stream) {
  HOKV_REQUIRE(n_q >= 1 && M >= 1 && sub_dim >= 1 && t_cols >= 1, "pq_tables: bad shape");
  HOKV_REQUIRE(cb_slots >= 1 && cb_slots <= 256 && M <= 65535, "pq_tables: cb_slots=%d M=%d", cb_slots, M);
  dim3 grid((unsigned)n_q, (unsigned)M);
  k_pq_tables<<<grid, 256, 0, S(stream)>>>(q, M, sub_dim, cents, cb_slots, cent_set_stride, k, k_set_stride, set_of_q,
                                           tables, t_cols, DOT_GEMV);
  return check_launch("k_pq_tables");
}

int hokv_pq_gather(const float* tables, int M, int t_cols, const uint8_t* codes, int64_t seq_len,
                   int64_t code_row_stride, int apply_scale, float scale, float* scores, void* stream) {
  HOKV_REQUIRE(M >= 1 && t_cols >= 1 && seq_len >= 0, "pq_gather: bad shape");
  if (seq_len == 0) return HOKV_OK;
  k_pq_gather<<<(unsigned)std::min<int64_t>(cdiv(seq_len, 256), 4096), 256, 0, S(stream)>>>(
      tables, M, t_cols, codes, seq_len, code_row_stride, apply_scale, scale, scores);
  return check_launch("k_pq_gather");
}

size_t hokv_pq_value_output_workspace_size(int M) { return (size_t)M * 256 * sizeof(double); }

int hokv_pq_value_output(const double* weights, int64_t seq_len, const uint8_t* codes, int64_t code_row_stride, int M,
                         int sub_dim, const float* cents, int cb_slots, const int* k, float* out, void* workspace,
                         size_t workspace_bytes, void* stream) {
  HOKV_REQUIRE(seq_len >= 0 && M >= 1 && sub_dim >= 1 && cb_slots >= 1 && cb_slots <= 256, "pq_value_output: shape");
  if (!workspace || workspace_bytes < hokv_pq_value_output_workspace_size(M))
    return fail(HOKV_ERR_WORKSPACE, "pq_value_output: workspace too small");
  double* bins = static_cast<double*>(workspace);
  cudaError_t e = cudaMemsetAsync(bins, 0, hokv_pq_value_output_workspace_size(M), S(stream));
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "pq_value_output memset: %s", cudaGetErrorString(e));
  if (seq_len > 0)
    k_value_bins<<<(unsigned)std::min<int64_t>(cdiv(seq_len * M, 256), 4096), 256, 0, S(stream)>>>(
        weights, seq_len, codes, code_row_stride, M, bins);
  k_value_out<<<M, 128, 0, S(stream)>>>(bins, M, sub_dim, cents, cb_slots, k, out);
  return check_launch("k_value_out");
}

// ------------------------------------------------------------------ CDC-03 ---
static int gt_of(int G) { return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; }

struct Plan {
  int n_chunks, chunk, GT, qimg_bytes;
  size_t cand_key_bytes, cand_cnt_bytes, qimg_total, texact_bytes, margin_bytes;
  size_t total() const {
    return cand_key_bytes + cand_cnt_bytes + qimg_total + texact_bytes + margin_bytes;
  }
};

static int plan_cdc03(const hokv_cdc03_args* a, Plan* pl) {
  HOKV_REQUIRE(a, "cdc03: null args");
  HOKV_REQUIRE(a->batch >= 1 && a->kv_heads >= 1, "cdc03: batch=%d kv_heads=%d", a->batch, a->kv_heads);
  HOKV_REQUIRE(a->q_per_kv >= 1 && a->q_per_kv <= 8, "cdc03: q_per_kv=%d not in [1, 8]", a->q_per_kv);
  HOKV_REQUIRE(a->head_dim == 32 || a->head_dim == 64 || a->head_dim == 128 || a->head_dim == 256,
               "cdc03: head_dim=%d not in {32, 64, 128, 256}", a->head_dim);
  HOKV_REQUIRE(a->n_subspaces >= 1, "cdc03: n_subspaces=%d", a->n_subspaces);
  {
    const int sd = a->sub_dim > 0 ? a->sub_dim : a->head_dim / a->n_subspaces;
    HOKV_REQUIRE(sd >= 1 && a->n_subspaces * sd <= a->head_dim && (a->sub_dim > 0 || a->head_dim % a->n_subspaces == 0),
                 "cdc03: M=%d x sub_dim=%d does not fit head_dim=%d", a->n_subspaces, sd, a->head_dim);
  }
  HOKV_REQUIRE(is_pow2_in(a->code_bytes, 4, 32) && a->n_subspaces <= a->code_bytes,
               "cdc03: code_bytes=%d (M=%d)", a->code_bytes, a->n_subspaces);
  HOKV_REQUIRE(a->cb_slots >= 1 && a->cb_slots <= 256, "cdc03: cb_slots=%d", a->cb_slots);
  HOKV_REQUIRE(a->top_k >= 0 && a->sink_tokens >= 0 && a->hot_window >= 0, "cdc03: negative budget");
  HOKV_REQUIRE(a->capacity >= 1 && a->capacity < (1ll << 30), "cdc03: capacity=%lld", (long long)a->capacity);
  HOKV_REQUIRE(a->q && a->out && a->k && a->v && a->codes && a->codebook && a->cb_k && a->seq_len,
               "cdc03: null pointer");
  HOKV_REQUIRE(a->kv_dtype == HOKV_F16 || a->kv_dtype == HOKV_BF16 || a->kv_dtype == HOKV_F32,
               "cdc03: kv dtype %d", a->kv_dtype);
  HOKV_REQUIRE(a->q_dtype == HOKV_F32 || a->q_dtype == HOKV_F16 || a->q_dtype == HOKV_BF16, "cdc03: q dtype");
  HOKV_REQUIRE(a->out_dtype == HOKV_F32 || a->out_dtype == HOKV_F16 || a->out_dtype == HOKV_BF16, "cdc03: out dtype");
  HOKV_REQUIRE(aligned(a->codes, 16) && a->code_stride_b % 16 == 0 && a->code_stride_h % 16 == 0,
               "cdc03: code store must be 16-byte aligned with 16-byte strides");
  HOKV_REQUIRE(aligned(a->k, 16) && aligned(a->v, 16) && a->kv_stride_b % 8 == 0 && a->kv_stride_h % 8 == 0,
               "cdc03: K/V stores must be 16-byte aligned with strides multiple of 8 elements");
  const int64_t cold_cap = std::max<int64_t>(0, a->capacity - a->hot_window);
  if (a->top_k > TOPK_MAX && a->top_k < cold_cap)
    return fail(HOKV_ERR_UNSUPPORTED, "cdc03: top_k=%d > %d with a longer cold range", a->top_k, TOPK_MAX);
  const int units = a->batch * a->kv_heads;
  pl->GT = gt_of(a->q_per_kv);
  HOKV_REQUIRE(!(pl->GT == 8 && a->code_bytes > 16), "cdc03: q_per_kv > 4 needs code_bytes <= 16");
  {
    const int sd = a->sub_dim > 0 ? a->sub_dim : a->head_dim / a->n_subspaces;
    if (!(sd == 4 || sd == 8 || sd == 16 || sd == 32))
      return fail(HOKV_ERR_UNSUPPORTED, "cdc03: sub_dim %d not in {4, 8, 16, 32}", sd);
    if (a->lut_order != HOKV_DOT_GEMV)
      return fail(HOKV_ERR_UNSUPPORTED, "cdc03: sub-tables use the GEMV dot order (lut_order = %d)", a->lut_order);
  }
  pl->chunk = K6_CHUNK;
  pl->n_chunks = (int)std::max<int64_t>(1, cdiv(cold_cap, K6_CHUNK));
  if (pl->n_chunks > MAX_CHUNKS)
    return fail(HOKV_ERR_UNSUPPORTED, "cdc03: capacity %lld needs %d chunks > %d", (long long)a->capacity,
                pl->n_chunks, MAX_CHUNKS);
  const size_t slots = (size_t)units * pl->n_chunks * pl->GT * CAND_MAX;
  pl->cand_key_bytes = a256(slots * 8);
  pl->cand_cnt_bytes = a256((size_t)units * pl->n_chunks * pl->GT * 4);
  pl->qimg_bytes = qimg_bytes_for(a->code_bytes, pl->GT);
  pl->qimg_total = a256((size_t)units * pl->qimg_bytes);
  pl->texact_bytes = a256((size_t)units * pl->GT * a->code_bytes * 256 * 4);
  pl->margin_bytes = a256((size_t)units * pl->GT * 4);
  return HOKV_OK;
}

int hokv_cdc03_workspace_size(const hokv_cdc03_args* a, size_t* bytes) {
  Plan pl;
  if (int st = plan_cdc03(a, &pl)) return st;
  *bytes = pl.total();
  return HOKV_OK;
}

static Cdc03P make_params(const hokv_cdc03_args* a, const Plan& pl) {
  Cdc03P p;
  p.B = a->batch; p.Hkv = a->kv_heads; p.G = a->q_per_kv; p.D = a->head_dim; p.M = a->n_subspaces;
  p.sd = a->sub_dim > 0 ? a->sub_dim : a->head_dim / a->n_subspaces; p.CS = a->code_bytes; p.slots = a->cb_slots; p.top_k = a->top_k;
  p.sink = a->sink_tokens; p.hot = a->hot_window; p.scale = a->scale; p.lut_order = a->lut_order;
  p.q = a->q; p.q_dtype = a->q_dtype; p.q_sb = a->q_stride_b;
  p.out = a->out; p.out_dtype = a->out_dtype; p.out_sb = a->out_stride_b;
  p.k = a->k; p.v = a->v; p.kv_sb = a->kv_stride_b; p.kv_sh = a->kv_stride_h; p.cap = a->capacity;
  p.kv_es = a->kv_dtype == HOKV_F32 ? 4 : 2;
  p.codes = a->codes; p.c_sb = a->code_stride_b; p.c_sh = a->code_stride_h;
  p.cb = a->codebook; p.cb_sb = a->cb_stride_b; p.cb_sh = a->cb_stride_h;
  p.cbk = a->cb_k; p.cbk_sb = a->cbk_stride_b; p.cbk_sh = a->cbk_stride_h;
  p.seq_len = a->seq_len;
  p.sel_idx = a->sel_idx; p.sel_score = a->sel_score; p.sel_count = a->sel_count;
  unsigned char* w = static_cast<unsigned char*>(a->workspace);
  p.cand_key = reinterpret_cast<uint64_t*>(w);
  p.cand_cnt = reinterpret_cast<int*>(w + pl.cand_key_bytes);
  w += pl.cand_key_bytes + pl.cand_cnt_bytes;
  p.qimg = w;
  w += pl.qimg_total;
  p.texact = reinterpret_cast<float*>(w);
  w += pl.texact_bytes;
  p.margin = reinterpret_cast<int*>(w);
  p.qimg_bytes = pl.qimg_bytes;
  p.n_chunks = pl.n_chunks; p.chunk = pl.chunk; p.GT = pl.GT;
  return p;
}

static int cdc03_prepare(const hokv_cdc03_args* a, Cdc03P* p) {
  Plan pl;
  if (int st = plan_cdc03(a, &pl)) return st;
  const size_t need = pl.total();
  if (!a->workspace || a->workspace_bytes < need)
    return fail(HOKV_ERR_WORKSPACE, "cdc03: workspace %zu < %zu", a->workspace_bytes, need);
  HOKV_REQUIRE(aligned(a->workspace, 16), "cdc03: workspace must be 16-byte aligned");
  *p = make_params(a, pl);
  return HOKV_OK;
}

int hokv_cdc03_candidates(const hokv_cdc03_args* a, void* stream) {
  Cdc03P p;
  if (int st = cdc03_prepare(a, &p)) return st;
  return dispatch_stage1(p, S(stream));
}

int hokv_cdc03_attend(const hokv_cdc03_args* a, void* stream) {
  Cdc03P p;
  if (int st = cdc03_prepare(a, &p)) return st;
  return dispatch_k7(p, a->kv_dtype, S(stream));
}

int hokv_cdc03_decode(const hokv_cdc03_args* a, void* stream) {
  Cdc03P p;
  if (int st = cdc03_prepare(a, &p)) return st;
  if (int st = dispatch_stage1(p, S(stream))) return st;
  return dispatch_k7(p, a->kv_dtype, S(stream));
}

// ---------------------------------------------------------------------------
// hokv_cdc03_decode with library-owned scratch: for callers that cannot
// allocate device memory (see hokv.h).  The array lives in this file; host
// code only ever uses the device address cudaGetSymbolAddress returns for it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_cdc03_scratch[HOKV_CDC03_NOALLOC_SCRATCH_BYTES];

// Device address of g_cdc03_scratch on the current device, looked up once per
// device (with that device current) and kept.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static std::map<int, void*> addr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "cdc03_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> g(mu);
  auto it = addr.find(dev);
  if (it == addr.end()) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_cdc03_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      (void)cudaGetLastError();
      return fail(HOKV_ERR_CUDA, "cdc03_decode_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                  cudaGetErrorString(e));
    }
    it = addr.emplace(dev, ptr).first;
  }
  *out = it->second;
  return HOKV_OK;
}

int hokv_cdc03_decode_noalloc(const hokv_cdc03_args* a, void* stream) {
  HOKV_REQUIRE(a, "cdc03_decode_noalloc: null args");
  size_t need = 0;
  if (int st = hokv_cdc03_workspace_size(a, &need)) return st;
  if (need > HOKV_CDC03_NOALLOC_SCRATCH_BYTES)
    return fail(HOKV_ERR_WORKSPACE,
                "cdc03_decode_noalloc: this configuration needs %zu bytes of scratch, more than the %zu bytes the "
                "library holds; use hokv_cdc03_decode with a caller-provided workspace",
                need, (size_t)HOKV_CDC03_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  hokv_cdc03_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = HOKV_CDC03_NOALLOC_SCRATCH_BYTES;
  return hokv_cdc03_decode(&b, stream);
}

int hokv_phase_stamps(uint64_t* out, size_t n_values) {
#ifdef HOKV_STAMPS
  const size_t all = (size_t)3 * STAMP_CTAS * STAMP_N;
  HOKV_REQUIRE(out && n_values >= all, "phase_stamps: need %zu values", all);
  cudaError_t e = cudaMemcpyFromSymbol(out, g_stamps, all * sizeof(uint64_t));
  if (e != cudaSuccess) return fail(HOKV_ERR_CUDA, "phase_stamps: %s", cudaGetErrorString(e));
  return HOKV_OK;
#else
  (void)out; (void)n_values;
  return fail(HOKV_ERR_UNSUPPORTED, "phase_stamps: this library was built without -DHOKV_STAMPS");
#endif
}

int hokv_dense_attention(const float* q, const float* K, const float* V, int head_dim, int64_t seq_len, int mul_f64,
                         double scale, int store_flags, const uint8_t* mask, void* scores, void* out, void* workspace,
                         size_t workspace_bytes, void* stream) {
  HOKV_REQUIRE(head_dim >= 1 && seq_len >= 1 && q && K && V && scores && out, "dense_attention: bad arguments");
  if (!workspace || workspace_bytes < (size_t)seq_len * 8) return fail(HOKV_ERR_WORKSPACE, "dense_attention: workspace");
  const int sf64 = store_flags & 1, of64 = (store_flags >> 1) & 1;
  k_dense_scores<<<(unsigned)cdiv(seq_len * 32, 256), 256, 0, S(stream)>>>(q, K, head_dim, seq_len, scale, mul_f64, sf64,
                                                                         mask, scores);
  k_softmax<<<1, 1024, 0, S(stream)>>>(scores, sf64, seq_len, workspace);
  k_weighted_sum<<<(unsigned)cdiv(head_dim, 128), 128, 0, S(stream)>>>(workspace, sf64, V, head_dim, seq_len, out, of64);
  return check_launch("dense_attention");
}

int hokv_softmax(const void* in, int is_f64, int64_t n, void* out, void* workspace, size_t workspace_bytes,
                 void* stream) {
  (void)workspace; (void)workspace_bytes;
  HOKV_REQUIRE(n >= 1 && in && out, "softmax: bad arguments");
  k_softmax<<<1, 1024, 0, S(stream)>>>(in, is_f64, n, out);
  return check_launch("k_softmax");
}

int hokv_prefilter_mask(const float* coarse, int k, const uint8_t* codes, int64_t seq_len, int top_p, uint8_t* mask,
                        void* stream) {
  HOKV_REQUIRE(k >= 1 && k <= 256 && seq_len >= 0 && top_p >= 0, "prefilter_mask: k=%d top_p=%d", k, top_p);
  if (seq_len == 0) return HOKV_OK;
  k_prefilter_mask<<<(unsigned)std::min<int64_t>(cdiv(seq_len, 256), 1024), 256, 0, S(stream)>>>(coarse, k, codes,
                                                                                                  seq_len, top_p, mask);
  return check_launch("k_prefilter_mask");
}

int hokv_scale_f32_to_f64(const float* in, int64_t n, double scale, double* out, void* stream) {
  HOKV_REQUIRE(n >= 0 && (n == 0 || (in && out)), "scale_f32_to_f64: bad arguments");
  if (n == 0) return HOKV_OK;
  k_scale_f32_to_f64<<<(unsigned)std::min<int64_t>(cdiv(n, 256), 4096), 256, 0, S(stream)>>>(in, n, scale, out);
  return check_launch("k_scale_f32_to_f64");
}

int hokv_age_tokens(const hokv_cdc03_args* a, const int* cold_from, const int* cold_to, int dot_order, void* stream) {
  HOKV_REQUIRE(a && cold_from && cold_to, "age_tokens: null argument");
  HOKV_REQUIRE(a->batch >= 1 && a->kv_heads >= 1 && a->batch <= 65535 && a->kv_heads <= 65535,
               "age_tokens: batch=%d kv_heads=%d", a->batch, a->kv_heads);
  HOKV_REQUIRE(a->n_subspaces >= 1 && a->n_subspaces <= a->code_bytes && a->code_bytes <= 32,
               "age_tokens: M=%d code_bytes=%d", a->n_subspaces, a->code_bytes);
  const int sd = a->sub_dim > 0 ? a->sub_dim : a->head_dim / a->n_subspaces;
  HOKV_REQUIRE(sd >= 1 && sd <= 32 && a->n_subspaces * sd <= a->head_dim, "age_tokens: sub_dim %d", sd);
  HOKV_REQUIRE(a->cb_slots >= 1 && a->cb_slots <= 256, "age_tokens: cb_slots=%d", a->cb_slots);
  HOKV_REQUIRE(dot_order >= 0 && dot_order <= 2, "age_tokens: dot_order=%d", dot_order);
  HOKV_REQUIRE(a->k && a->codes && a->codebook && a->cb_k, "age_tokens: null store pointer");
  HOKV_REQUIRE(a->capacity >= 1, "age_tokens: capacity=%lld", (long long)a->capacity);
  const int64_t items = a->capacity * a->n_subspaces;
  const unsigned gx = (unsigned)std::min<int64_t>(64, std::max<int64_t>(1, cdiv(items, 8 * 32)));
  const dim3 grid(gx, (unsigned)a->kv_heads, (unsigned)a->batch);
#define HOKV_AGE(T)                                                                                                 \
  k_age_tokens<T><<<grid, 256, 0, S(stream)>>>(reinterpret_cast<const T*>(a->k), a->kv_stride_b, a->kv_stride_h,   \
                                               a->head_dim, a->n_subspaces, sd, a->codebook, a->cb_stride_b,       \
                                               a->cb_stride_h, a->cb_slots, a->cb_k, a->cbk_stride_b,              \
                                               a->cbk_stride_h, const_cast<uint8_t*>(a->codes), a->code_stride_b, a->code_stride_h, \
                                               a->code_bytes, cold_from, cold_to, a->capacity, dot_order)
  if (a->kv_dtype == HOKV_BF16) HOKV_AGE(__nv_bfloat16);
  else if (a->kv_dtype == HOKV_F16) HOKV_AGE(__half);
  else if (a->kv_dtype == HOKV_F32) HOKV_AGE(float);
  else return fail(HOKV_ERR_INVALID, "age_tokens: kv dtype %d", a->kv_dtype);
#undef HOKV_AGE
  return check_launch("k_age_tokens");
}

int hokv_prefill_attention(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                           int q_heads, int kv_heads, int q_len, int kv_len, int head_dim, int64_t q_stride_b,
                           int64_t q_stride_h, int64_t q_stride_s, int64_t k_stride_b, int64_t k_stride_h,
                           int64_t k_stride_s, int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
                           int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, float scale,
                           int causal, void* stream) {
  HOKV_REQUIRE(q && k && v && out, "prefill_attention: null pointer");
  HOKV_REQUIRE(batch >= 1 && batch <= 65535 && q_heads >= 1 && q_heads <= 65535 && kv_heads >= 1 &&
                   q_heads % kv_heads == 0,
               "prefill_attention: batch=%d q_heads=%d kv_heads=%d", batch, q_heads, kv_heads);
  HOKV_REQUIRE(q_len >= 1 && kv_len >= 1 && (!causal || kv_len >= q_len),
               "prefill_attention: q_len=%d kv_len=%d causal=%d (a causal call needs kv_len >= q_len)", q_len,
               kv_len, causal);
  if (dtype != HOKV_F16 && dtype != HOKV_BF16)
    return fail(HOKV_ERR_UNSUPPORTED, "prefill_attention: dtype %d (f16 and bf16 only)", dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(HOKV_ERR_UNSUPPORTED, "prefill_attention: head_dim %d (64 and 128 only)", head_dim);
  // 16-byte rows: every row start and every stride a multiple of 8 elements
  const int64_t st[12] = {q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h, k_stride_s,
                          v_stride_b, v_stride_h, v_stride_s, out_stride_b, out_stride_h, out_stride_s};
  for (int i = 0; i < 12; ++i)
    HOKV_REQUIRE(st[i] % 8 == 0 && st[i] >= 0, "prefill_attention: stride %lld not a multiple of 8 elements",
                 (long long)st[i]);
  HOKV_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16),
               "prefill_attention: pointers must be 16-byte aligned");
  HOKV_REQUIRE(k_stride_b == v_stride_b && k_stride_h == v_stride_h && k_stride_s == v_stride_s,
               "prefill_attention: k and v must share their strides");
  PfMaps maps;
  PfArgs p;
  if (int e = pf_tensor_map(&maps.q, q, dtype, head_dim, q_len, q_stride_s, q_heads, q_stride_h, batch, q_stride_b,
                            PF_ROWS, &p.q_slot_t, &p.q_slot_h, &p.q_slot_b))
    return e;
  const int bn = head_dim == 64 ? PfGeo<64>::BN : PfGeo<128>::BN;
  if (int e = pf_tensor_map(&maps.k, k, dtype, head_dim, kv_len, k_stride_s, kv_heads, k_stride_h, batch, k_stride_b,
                            bn, &p.kv_slot_t, &p.kv_slot_h, &p.kv_slot_b))
    return e;
  int ts, hs, bs;
  if (int e = pf_tensor_map(&maps.v, v, dtype, head_dim, kv_len, v_stride_s, kv_heads, v_stride_h, batch, v_stride_b,
                            bn, &ts, &hs, &bs))
    return e;
  p.out = out;
  p.Sq = q_len;
  p.Skv = kv_len;
  p.Hq = q_heads;
  p.G = q_heads / kv_heads;
  p.osb = out_stride_b; p.osh = out_stride_h; p.oss = out_stride_s;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  const dim3 grid((unsigned)cdiv(q_len, 2 * PF_ROWS), (unsigned)q_heads, (unsigned)batch);
#define HOKV_PF(D_, T_)                                                                                  \
  {                                                                                                    \
    if (int e = ensure_smem(k_prefill_attn<D_, T_>, PfGeo<D_>::SMEM)) return e;                        \
    k_prefill_attn<D_, T_><<<grid, PF_THREADS, PfGeo<D_>::SMEM, S(stream)>>>(maps, p);                 \
    return check_launch("k_prefill_attn");                                                            \
  }
  if (head_dim == 64 && dtype == HOKV_F16) HOKV_PF(64, __half)
  if (head_dim == 64) HOKV_PF(64, __nv_bfloat16)
  if (dtype == HOKV_F16) HOKV_PF(128, __half)
  HOKV_PF(128, __nv_bfloat16)
#undef HOKV_PF
}


}  // extern "C"
