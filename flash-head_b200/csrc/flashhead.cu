// C ABI of the FlashHead decode-step head (declared in include/flashhead.h).
//
// Host code only validates arguments, lays out the caller's workspace and
// launches kernels on the caller's stream: it never allocates, synchronises
// or reads device memory, so every entry point can be captured in a CUDA
// graph. Kernels after the first of a call are launched with programmatic
// dependent launch so that their CTAs are resident before their predecessor
// finishes.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/flashhead.h"
#include "fh_batched.cuh"
#include "fh_stage2_tc.cuh"
#include "fh_spec.cuh"

static_assert(fh::kS2MaskWords == 8, "the selection kernel writes 8 bit-map words per cluster");

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(FH_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define FH_CHECK_LAUNCH(expr, what)           \
  do {                                        \
    cudaError_t _e = (expr);                  \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)


size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
#ifdef FH_TRACE
unsigned long long *g_trace_buf = nullptr;
#endif

template <typename Kern, typename... Args>
cudaError_t launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   bool pdl, Args... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// k_select keeps every key of a row in dynamic shared memory; raise its
// limit once per device.
std::mutex g_attr_mutex;
bool g_select_attr_done[128];

cudaError_t prepare_select() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (!g_select_attr_done[dev]) {
    e = cudaFuncSetAttribute(fh::k_select, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(fh::kSelMaxItems * sizeof(unsigned long long)));
    if (e != cudaSuccess) return e;
    g_select_attr_done[dev] = true;
  }
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// One-kernel step (fh_fused.cuh): cooperative grid of one CTA per SM.
// ---------------------------------------------------------------------------
int g_sm_count[128];

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 0;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

template <typename HT, typename WT, int R, bool SAMPLE>
cudaError_t launch_fused_t(const fh::FusedArgs &a, int grid, cudaStream_t stream) {
  static bool attr_done[128];
  auto kern = fh::k_fused_step<HT, WT, R, SAMPLE>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (!attr_done[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)fh::kFSmemMax);
      if (e != cudaSuccess) return e;
      attr_done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(fh::kFBlock);
  cfg.dynamicSmemBytes = fh::fused_smem_bytes(R, a.D, (int)sizeof(WT));
  cfg.stream = stream;
  // Cooperative (all CTAs resident: the grid barrier needs it) and, where
  // the runtime accepts the pair, programmatic dependent launch: the step may
  // start streaming its stage-1 rows while the previous kernel in the stream
  // drains; it reads the hidden states and the workspace only after
  // griddepcontrol.wait.
  // 0 unknown, 1 accepted, -1 rejected; shared by the host threads of a process
  static std::atomic<int> pdl_ok[128];
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  int known = pdl_ok[dev].load(std::memory_order_relaxed);
  if (known == 0) {
    // A refused trial launch would invalidate a graph being captured: while
    // the stream captures and support is still unknown, launch without PDL
    // and leave the question for an uncaptured call.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
      known = -2;
  }
  if (known >= 0) {
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e == cudaSuccess) {
      pdl_ok[dev].store(1, std::memory_order_relaxed);
      return e;
    }
    if (known == 1) return e;
    (void)cudaGetLastError();  // the pair is not supported here: launch without PDL
    pdl_ok[dev].store(-1, std::memory_order_relaxed);
  }
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename HT, typename WT>
cudaError_t launch_fused_rows(const fh::FusedArgs &a, int grid, cudaStream_t s) {
  if (a.do_sample) {
    if (a.rows == 1) return launch_fused_t<HT, WT, 1, true>(a, grid, s);
    if (a.rows == 2) return launch_fused_t<HT, WT, 2, true>(a, grid, s);
    return launch_fused_t<HT, WT, 4, true>(a, grid, s);
  }
  if (a.rows == 1) return launch_fused_t<HT, WT, 1, false>(a, grid, s);
  if (a.rows == 2) return launch_fused_t<HT, WT, 2, false>(a, grid, s);
  return launch_fused_t<HT, WT, 4, false>(a, grid, s);
}

cudaError_t launch_fused(int hdt, int wdt, const fh::FusedArgs &a, int grid, cudaStream_t s) {
  if (hdt == FH_BF16) {
    if (wdt == FH_FP8_E4M3) return launch_fused_rows<__nv_bfloat16, __nv_fp8_e4m3>(a, grid, s);
    return launch_fused_rows<__nv_bfloat16, __nv_bfloat16>(a, grid, s);
  }
  if (wdt == FH_FP8_E4M3) return launch_fused_rows<__half, __nv_fp8_e4m3>(a, grid, s);
  return launch_fused_rows<__half, __half>(a, grid, s);
}

}  // namespace

struct fh_head {
  fh_head_desc d;
  mutable std::mutex plan_mutex;  // guards the tensor maps, encoded on first use
  mutable CUtensorMap tm_w;  // w_perm rows for the dense tensor-core kernel
  mutable int tm_w_tile = 0;  // its box height, 0: not encoded yet
  mutable CUtensorMap tm_c[2];  // stage-1 matrices (cluster_w, centroid_w) for k_s1_tc
  mutable bool tm_c_ok[2] = {false, false};
  mutable CUtensorMap tm_s2;   // w_perm in 16-row boxes for k_s2_tc (one cluster)
  mutable CUtensorMap tm_s2w;  // w_perm in 128-row boxes (a window of 8 clusters)
  mutable bool tm_s2_ok = false;
};

// ---------------------------------------------------------------------------
// Workspace layout for `rows` hidden states.
// ---------------------------------------------------------------------------
namespace {

// Stage-1 tiling of the tensor-core kernel k_s1_tc: 128-row tiles of the
// stage-1 matrix, each split over the hidden dimension so that tiles x splits
// fills the SMs once; the splits' partial scores are summed by the selection.
int s1_splits(const fh_head_desc &d) {
  const int m_tiles = (d.n_clusters + fh::kS1MTile - 1) / fh::kS1MTile;
  const int nk = (d.hidden + fh::kS1KBlock - 1) / fh::kS1KBlock;
  const int sms = sm_count() > 0 ? sm_count() : 148;
  return std::max(1, std::min(nk, sms / m_tiles));
}

// An fp8 stage-1 matrix is multiplied in f16: bf16 hidden rows need an f16 copy.
bool s1_needs_h16(const fh_head_desc &d) {
  return d.weight_dtype == FH_BF16 &&
         (d.score_dtype == FH_FP8_E4M3 || (d.centroid_w && d.sample_dtype == FH_FP8_E4M3));
}

struct Workspace {
  float *scores;                // [splits][rows, score_stride]: stage-1 (partial) scores
  int score_stride;
  int splits;                   // k_s1_tc partials held (1 below kGemmS1MinRows rows)
  size_t split_stride;          // floats between two splits' partials
  int32_t *probes;              // [rows, p]
  unsigned long long *packed;   // [rows]
  unsigned *counter;            // [1]
  unsigned char *epoch_bufs;    // one-kernel histograms
  void *h16;                    // [rows, D] f16 copy of bf16 hidden rows (fp8 stage 1)
  // batched steps (rows >= kBatchMinRows) only, else null: the cluster-major
  // stage 2's index of one chunk of up to kS2MaxRows rows
  uint32_t *s2_bm;              // [K][kS2MaskWords] row bit map of every cluster,
  fh::S2Meta *s2_meta;          //   followed by the meta words
  fh::S2Tile *s2_tiles;         // tile descriptors
  size_t s2_zero_bytes;         // bytes of s2_bm + s2_meta (zeroed per chunk)
  size_t bytes;                 // bytes needed for `rows`
};

// Persistent state first, at offsets that do not depend on `rows`: state
// words at 0 (three-kernel stage-2 counter, one-kernel barrier / done /
// error / epoch words), the one-kernel step's key histograms at 256, then the
// stage-2 accumulator packed[r].
// Stage 2 leaves both zeroed when it completes, so a workspace zero-filled
// once stays clean across calls with any row count. Per-call scratch
// (probes, scores, the f16 hidden copy, the inverted index) is placed from
// the top of the buffer downwards and never reaches the state of a call
// whose size check passed.
Workspace layout(const fh_head_desc &d, int rows, void *base, size_t ws_bytes) {
  Workspace w;
  char *p = reinterpret_cast<char *>(base);
  w.score_stride = (int)round_up((size_t)d.n_clusters, 64);
  w.splits = rows >= fh::kGemmS1MinRows ? s1_splits(d) : 1;
  w.split_stride = (size_t)rows * w.score_stride;
  const size_t state =
      256 + fh::kHistBytes + round_up((size_t)rows * sizeof(unsigned long long), 256);
  const size_t probes = round_up((size_t)rows * d.n_probes * sizeof(int32_t), 256);
  const size_t scores = round_up((size_t)w.splits * w.split_stride * sizeof(float), 256);
  const size_t h16 = rows >= fh::kGemmS1MinRows && s1_needs_h16(d)
                         ? round_up((size_t)rows * d.hidden * 2, 256)
                         : 0;
  const bool batched = rows >= fh::kBatchMinRows;
  const size_t bmb = round_up((size_t)d.n_clusters * fh::kS2MaskWords * sizeof(uint32_t), 256);
  const size_t max_tiles = (size_t)(d.n_clusters + fh::kS2Clusters - 1) / fh::kS2Clusters +
                           (size_t)(d.n_clusters + fh::kS2TileClusters - 1) / fh::kS2TileClusters +
                           1;
  const size_t s2_tiles = round_up(max_tiles * sizeof(fh::S2Tile), 256);
  const size_t inv = batched ? bmb + sizeof(fh::S2Meta) + s2_tiles : 0;
  w.bytes = state + probes + scores + h16 + inv + 256;
  w.counter = reinterpret_cast<unsigned *>(p);
  w.epoch_bufs = reinterpret_cast<unsigned char *>(p + 256);
  w.packed = reinterpret_cast<unsigned long long *>(p + 256 + fh::kHistBytes);
  const size_t top = (ws_bytes / 256) * 256;
  const size_t probes_off = top >= probes ? top - probes : 0;
  const size_t scores_off = probes_off >= scores ? probes_off - scores : 0;
  const size_t h16_off = scores_off >= h16 ? scores_off - h16 : 0;
  w.probes = reinterpret_cast<int32_t *>(p + probes_off);
  w.scores = reinterpret_cast<float *>(p + scores_off);
  w.h16 = h16 ? p + h16_off : nullptr;
  w.s2_bm = nullptr;
  w.s2_meta = nullptr;
  w.s2_tiles = nullptr;
  w.s2_zero_bytes = bmb + sizeof(fh::S2Meta);
  if (batched) {
    size_t q = h16_off >= inv ? h16_off - inv : 0;
    w.s2_tiles = reinterpret_cast<fh::S2Tile *>(p + q);
    q += s2_tiles;
    w.s2_bm = reinterpret_cast<uint32_t *>(p + q);
    w.s2_meta = reinterpret_cast<fh::S2Meta *>(p + q + bmb);
  }
  return w;
}

int check_call(const fh_head *h, const void *hidden, int rows, const void *out, void *ws,
               size_t ws_bytes) {
  if (!h) return fail(FH_ERR_INVALID_ARGUMENT, "null head");
  if (rows < 0) return fail(FH_ERR_INVALID_ARGUMENT, "rows=%d < 0", rows);
  if (rows == 0) return FH_OK;
  if (!hidden || !out) return fail(FH_ERR_INVALID_ARGUMENT, "null hidden/output pointer");
  if (!aligned16(hidden))
    return fail(FH_ERR_INVALID_ARGUMENT, "hidden states must be 16-byte aligned");
  if (!ws) return fail(FH_ERR_WORKSPACE, "null workspace");
  const size_t need = layout(h->d, rows, nullptr, 0).bytes;
  if (ws_bytes < need)
    return fail(FH_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed for %d rows", ws_bytes,
                need, rows);
  if (!aligned16(ws)) return fail(FH_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  return FH_OK;
}

fh::RngKey rng_key(uint64_t seed, uint64_t offset) {
  fh::RngKey k;
  k.k0 = (uint32_t)seed;
  k.k1 = (uint32_t)(seed >> 32);
  k.off_lo = (uint32_t)offset;
  k.off_hi = (uint32_t)(offset >> 32);
  return k;
}

// ---------------------------------------------------------------------------
// Stage-1 scores launch: picks rows per CTA and clusters per warp.
// ---------------------------------------------------------------------------
template <typename HT, typename WT>
cudaError_t launch_scores_t(const fh::ScoresArgs &a, cudaStream_t s) {
  const int rows = a.rows;
  auto go = [&](auto kern, int rows_per, int cpw) {
    const int warps = (a.K + cpw - 1) / cpw;
    const int ctas = (warps + 7) / 8;
    dim3 grid(ctas, (rows + rows_per - 1) / rows_per);
    return launch(kern, grid, dim3(256), 0, s, false, a);
  };
  if (rows == 1) return go(fh::k_scores<HT, WT, 1, 1, 4>, 1, 1);
  if (rows == 2) return go(fh::k_scores<HT, WT, 2, 2, 2>, 2, 2);
  if (rows <= 4) return go(fh::k_scores<HT, WT, 4, 2, 2>, 4, 2);
  return go(fh::k_scores<HT, WT, 8, 4, 1>, 8, 4);
}

cudaError_t launch_scores(int hdt, int wdt, const fh::ScoresArgs &a, cudaStream_t s) {
  if (hdt == FH_BF16) {
    if (wdt == FH_FP8_E4M3) return launch_scores_t<__nv_bfloat16, __nv_fp8_e4m3>(a, s);
    return launch_scores_t<__nv_bfloat16, __nv_bfloat16>(a, s);
  }
  if (wdt == FH_FP8_E4M3) return launch_scores_t<__half, __nv_fp8_e4m3>(a, s);
  return launch_scores_t<__half, __half>(a, s);
}

template <typename HT, typename IdxT, int MODE>
cudaError_t launch_stage2_t(const fh::Stage2Args &a, int items, cudaStream_t s, bool pdl) {
  // steps of 5+ rows on a workspace (a last-CTA counter to publish with): the
  // streamed kernel, one persistent CTA per SM (8 rows: 33.8 -> 31.2 us on
  // the Llama-3.2-1B head); fewer rows and the stateless entry points keep
  // the one-CTA-per-item kernel, which has less start-up (1 row: 7.0 us
  // against 9.8 us streamed)
  if constexpr (MODE == fh::kGreedy || MODE == fh::kSample) {
    if (a.counter != nullptr && a.rows >= fh::kGemmS1MinRows && (size_t)a.D * sizeof(HT) % 16 == 0 &&
        fh::s2s_smem_bytes(a.D) <= (size_t)fh::kS2SmemMax && sm_count() > 0) {
      static size_t attr_bytes[128];  // dynamic shared memory allowed so far
      auto kern = fh::k_stage2_stream<HT, IdxT, MODE == fh::kSample>;
      const size_t need = fh::s2s_smem_bytes(a.D);
      int dev = 0;
      cudaError_t e = cudaGetDevice(&dev);
      if (e != cudaSuccess) return e;
      if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
      {
        std::lock_guard<std::mutex> lock(g_attr_mutex);
        if (need > attr_bytes[dev]) {
          e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need);
          if (e != cudaSuccess) return e;
          attr_bytes[dev] = need;
        }
      }
      return launch(kern, dim3(sm_count()), dim3(32 * fh::s2s_warps(a.D)), fh::s2s_smem_bytes(a.D),
                    s, pdl, a, (long long)items, reinterpret_cast<uint32_t *>(a.counter) + fh::kSyncError,
                    (uint32_t)(1u << 22));
    }
  }
  constexpr int U = 4;
  const int warps = a.cap < 16 ? a.cap : 16;
  return launch(fh::k_stage2<HT, IdxT, MODE, U>, dim3(items), dim3(32 * warps), 0, s, pdl, a);
}

template <typename IdxT, int MODE>
cudaError_t launch_stage2(int hdt, const fh::Stage2Args &a, int items, cudaStream_t s, bool pdl) {
  if (hdt == FH_BF16) return launch_stage2_t<__nv_bfloat16, IdxT, MODE>(a, items, s, pdl);
  return launch_stage2_t<__half, IdxT, MODE>(a, items, s, pdl);
}

fh::Stage2Args stage2_args(const fh_head_desc &d, const void *hidden, int rows) {
  fh::Stage2Args a;
  memset(&a, 0, sizeof(a));
  a.hidden = hidden;
  a.rows = rows;
  a.D = d.hidden;
  a.w_perm = d.w_perm;
  a.K = d.n_clusters;
  a.cap = d.cluster_size;
  a.vocab_map = d.vocab_map;
  a.special_slots = d.special_slots;
  a.n_special = d.n_special;
  a.cluster_base = d.cluster_base;
  a.temperature = 1.f;
  return a;
}

fh::ScoresArgs scores_args(const fh_head_desc &d, const void *hidden, int rows, bool sample,
                           float temperature, uint64_t seed, uint64_t offset) {
  fh::ScoresArgs a;
  memset(&a, 0, sizeof(a));
  a.hidden = hidden;
  a.rows = rows;
  a.D = d.hidden;
  a.w = sample ? d.centroid_w : d.cluster_w;
  a.scale = sample ? d.centroid_scale : d.cluster_scale;
  a.K = d.n_clusters;
  a.do_sample = sample ? 1 : 0;
  a.temperature = temperature;
  a.rng = rng_key(seed, offset);
  a.cluster_base = d.cluster_base;
  return a;
}

fh::SelectArgs select_dense_args(const fh_head_desc &d, const float *scores, int stride,
                                 int rows) {
  fh::SelectArgs a;
  memset(&a, 0, sizeof(a));
  a.scores = scores;
  a.score_stride = stride;
  a.rows = rows;
  a.n_items = d.n_clusters;
  a.p = d.n_probes;
  a.wait_prior = 1;
  return a;
}

int check_sampling(const fh_head *h, float temperature) {
  if (!h->d.centroid_w)
    return fail(FH_ERR_UNSUPPORTED, "sampling needs the raw centroid matrix (centroid_w)");
  if (!(temperature > 0.f) || !std::isfinite(temperature))
    return fail(FH_ERR_INVALID_ARGUMENT, "temperature must be positive and finite (got %g)",
                (double)temperature);
  return FH_OK;
}

// Stage 1 + selection for the local head. Writes probes (local or global
// ids) and/or signed candidate words; zeroes packed/counter for stage 2.
int run_stage1(const fh_head *h, const void *hidden, int rows, bool sample, float temperature,
               uint64_t seed, uint64_t offset, const Workspace &w, float *scores_out,
               int32_t *probes_out, long long *cand_out, int id_base, cudaStream_t s) {
  const fh_head_desc &d = h->d;
  fh::ScoresArgs sa = scores_args(d, hidden, rows, sample, temperature, seed, offset);
  sa.scores = scores_out ? scores_out : w.scores;
  sa.score_stride = scores_out ? d.n_clusters : w.score_stride;
  sa.packed = w.packed;
  sa.counter = w.counter;
  sa.n_packed = rows;
  const int wdt = sample ? d.sample_dtype : d.score_dtype;
  FH_CHECK_LAUNCH(launch_scores(d.weight_dtype, wdt, sa, s), "stage-1 scores launch");
  FH_CHECK_LAUNCH(prepare_select(), "select kernel attribute");
  fh::SelectArgs se = select_dense_args(d, sa.scores, sa.score_stride, rows);
  se.probes = probes_out;
  se.cand_out = cand_out;
  se.id_base = id_base;
  const size_t smem = (size_t)d.n_clusters * sizeof(unsigned long long);
  FH_CHECK_LAUNCH(launch(fh::k_select, dim3(rows), dim3(fh::kSelThreads), smem, s, true, se),
                  "probe selection launch");
  return FH_OK;
}

// Shapes the one-kernel step supports; everything else takes the
// three-kernel path.
bool fused_ok(const fh_head_desc &d, int rows, bool sample, int grid) {
  if (d.flags & FH_FLAG_NO_FUSED) return false;
  if (rows < 1 || rows > fh::kFMaxRows || grid < rows || grid > 1024 || d.cluster_base != 0)
    return false;
  const int wdt = sample ? d.sample_dtype : d.score_dtype;
  // rows of whole 128-byte group pairs; hidden rows (16-bit) in shared memory
  const int wt_bytes = wdt == FH_FP8_E4M3 ? 1 : 2;
  if ((d.hidden * wt_bytes) % 128 != 0 || (d.hidden * 2) % 128 != 0) return false;
  const int R = rows <= 1 ? 1 : rows <= 2 ? 2 : 4;
  if (fh::fused_smem_bytes(R, d.hidden, wt_bytes) > fh::kFSmemMax) return false;
  if (d.n_clusters > 128 * grid || d.n_clusters > fh::kSelMaxItems) return false;
  if (d.n_probes > fh::kFMaxProbes || d.cluster_size > fh::kS3MaxRows) return false;
  if (d.n_special > fh::kFMaxSpecial || d.n_clusters >= (1 << 24)) return false;
  if ((d.n_clusters + 127) / 128 > fh::kMaxChunks) return false;
  {  // stage-1 chunks of the largest CTA slice, each with its own partial buffer
    const fh::RingGeom g1 = fh::ring_geom(d.hidden * wt_bytes);
    const int nc_max = (d.n_clusters + grid - 1) / grid;
    if ((nc_max + fh::kTileRows - 1) / fh::kTileRows * g1.ndc > fh::kMaxS1Chunks) return false;
  }
  // every CTA holds the score rows in its 128 KB ring; items per CTA fit its work list
  if ((size_t)rows * round_up((size_t)d.n_clusters, 4) * sizeof(float) > (size_t)fh::kRingBytes)
    return false;
  if ((long long)rows * (d.n_probes + d.n_special) > (long long)(fh::kWorkCap - 1) * grid)
    return false;
  return true;
}

int run_fused(const fh_head *h, const void *hidden, int rows, bool sample, float temperature,
              uint64_t seed, uint64_t offset, int64_t *out_ids, const Workspace &w, int grid,
              cudaStream_t s) {
  const fh_head_desc &d = h->d;
  fh::FusedArgs a;
  memset(&a, 0, sizeof(a));
  a.hidden = hidden;
  a.rows = rows;
  a.D = d.hidden;
  a.cw = sample ? d.centroid_w : d.cluster_w;
  a.cscale = sample ? d.centroid_scale : d.cluster_scale;
  a.K = d.n_clusters;
  a.w_perm = d.w_perm;
  a.vocab_map = d.vocab_map;
  a.cap = d.cluster_size;
  a.p = d.n_probes;
  a.special_slots = d.special_slots;
  a.n_special = d.n_special;
  a.do_sample = sample ? 1 : 0;
  a.temperature = temperature;
  a.rng = rng_key(seed, offset);
  a.scores = w.scores;
  a.score_stride = w.score_stride;
  a.sync = reinterpret_cast<uint32_t *>(w.counter);
  a.epoch_bufs = w.epoch_bufs;
  a.packed = w.packed;
  a.out_ids = out_ids;
  const bool test_timeout = (d.flags & FH_FLAG_TEST_TIMEOUT) != 0;
  a.barrier_polls = test_timeout ? (1u << 12) : (1u << 22);
  a.copy_polls = 1u << 22;
  a.extra_arrivals = test_timeout ? 1 : 0;
#ifdef FH_TRACE
  a.trace = g_trace_buf;
#endif
  const int wdt = sample ? d.sample_dtype : d.score_dtype;
  FH_CHECK_LAUNCH(launch_fused(d.weight_dtype, wdt, a, grid, s), "one-kernel step launch");
  return FH_OK;
}

// ---------------------------------------------------------------------------
// Batched steps (rows >= kBatchMinRows): tensor-core stage 1, the selection
// kernel, the inverted index and the inverted stage 2.
bool batched_ok(const fh_head *h, int rows, bool sample, int min_rows = fh::kBatchMinRows) {
  const fh_head_desc &d = h->d;
  if (rows < min_rows || (d.flags & FH_FLAG_NO_FUSED)) return false;
  if (sample && !d.centroid_w) return false;
  if (d.cluster_base != 0) return false;
  if (d.cluster_size > fh::kTileRows || (d.hidden * 2) % 128 != 0) return false;
  return sm_count() > 0;
}

// The inverted stage 2 (any shard): clusters of at most 16 rows of whole
// 128-byte groups, and the index buffers of a workspace laid out for 16+ rows.
bool inv_ok(const fh_head_desc &d, int rows) {
  if (rows < fh::kBatchMinRows || (d.flags & FH_FLAG_NO_FUSED)) return false;
  if (d.cluster_size > fh::kTileRows || (d.hidden * 2) % 128 != 0) return false;
  return sm_count() > 0;
}

// Stage 1 on the tensor cores (k_s1_tc) needs only 16-byte row pitches (the
// tensor maps) and a selection that keeps a row in shared memory.
bool s1_tc_ok(const fh_head_desc &d, bool sample) {
  if (d.flags & FH_FLAG_NO_FUSED) return false;
  if (sample && !d.centroid_w) return false;
  if (d.n_clusters > fh::kSelMaxItems || d.hidden % 16 != 0) return false;
  return sm_count() > 0;
}

cudaError_t prepare_select_hist() {
  static bool done[128];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(fh::k_select_hist<1024>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fh::hsel_smem_bytes(fh::kSelMaxItems, 1024));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fh::k_select_hist<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fh::hsel_smem_bytes(fh::kSelMaxItems, 512));
    if (e != cudaSuccess) return e;
    done[dev] = true;
  }
  return cudaSuccess;
}

int grid_for(long long n, int block) {
  long long g = (n + block - 1) / block;
  const int cap = 4 * (sm_count() > 0 ? sm_count() : 148);
  return (int)(g < 1 ? 1 : g > cap ? cap : g);
}

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime
// (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (!tried) {
    tried = true;
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D map of a row-major [n_rows, D] 16-bit matrix: boxes of box_rows rows x
// one k-block (kDtKBytes bytes) with the swizzle of that width, zero fill
// outside the matrix.
bool encode_rows_map(CUtensorMap *tm, const void *base, int dtype, int D, long long n_rows,
                     int box_rows) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc || !aligned16(base)) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)n_rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {(cuuint32_t)fh::kDtKBlock, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  return enc(tm,
             dtype == FH_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
             2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             fh::kDtKBytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map of a row-major [K, D] stage-1 matrix for k_s1_tc: boxes of 128
// rows x 64 elements; fp8 rows unswizzled (converted in shared memory),
// 16-bit rows with the 128-byte swizzle the MMA reads; zero fill outside.
bool encode_s1_map(CUtensorMap *tm, const void *base, int dtype, int D, int K) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc || !aligned16(base)) return false;
  const bool fp8 = dtype == FH_FP8_E4M3;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)K};
  const cuuint64_t strides[1] = {(cuuint64_t)D * (fp8 ? 1 : 2)};
  const cuuint32_t box[2] = {(cuuint32_t)fh::kS1KBlock, (cuuint32_t)fh::kS1MTile};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType t = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                : dtype == FH_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(tm, t, 2, const_cast<void *>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE,
             fp8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t prepare_s1_tc() {
  static bool done[128];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(fh::k_s1_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fh::kS1SmemMax);
    if (e != cudaSuccess) return e;
    done[dev] = true;
  }
  return cudaSuccess;
}

// Stage 1 of a call of kGemmS1MinRows+ rows on the tensor cores: partial
// scores of every (128-cluster tile, hidden split) by k_s1_tc (one launch per
// 256 hidden rows; bf16 rows against an fp8 matrix first get an f16 copy),
// then one k_select_hist CTA per row sums the partials into the keys (fp8
// row scale; sampling: / T + Gumbel), writes them to scores_out (if given,
// row pitch out_stride) and selects the top-p clusters into probes and/or
// the signed candidate words (global ids) into cand_out.
int run_s1_tc(const fh_head *h, const void *hidden, int rows, bool sample, float temperature,
              uint64_t seed, uint64_t offset, const Workspace &w, float *scores_out,
              int out_stride, int32_t *probes, long long *cand_out, cudaStream_t s,
              uint32_t *s2_bm = nullptr) {
  const fh_head_desc &d = h->d;
  const int which = sample ? 1 : 0;
  const int cdt = sample ? d.sample_dtype : d.score_dtype;
  const void *cmat = sample ? d.centroid_w : d.cluster_w;
  const bool fp8 = cdt == FH_FP8_E4M3;
  if (w.splits != s1_splits(d)) return fail(FH_ERR_WORKSPACE, "workspace laid out for another split count");
  {
    std::lock_guard<std::mutex> lock(h->plan_mutex);
    if (!h->tm_c_ok[which]) {
      if (!encode_s1_map(&h->tm_c[which], cmat, cdt, d.hidden, d.n_clusters))
        return fail(FH_ERR_UNSUPPORTED, "stage-1 matrix tensor map");
      h->tm_c_ok[which] = true;
    }
  }
  const CUtensorMap tm_c = h->tm_c[which];
  // operand type of the MMA: f16 against fp8 rows, else the weight type
  const bool mma_bf16 = !fp8 && d.weight_dtype == FH_BF16;
  const void *hop = hidden;
  bool pdl = false;
  if (fp8 && d.weight_dtype == FH_BF16) {
    if (!w.h16) return fail(FH_ERR_WORKSPACE, "no f16 staging for the hidden rows");
    const int n8 = (int)((size_t)rows * d.hidden / 8);
    FH_CHECK_LAUNCH(launch(fh::k_hidden_to_f16, dim3(grid_for(n8, 256)), dim3(256), 0, s, false,
                           reinterpret_cast<const uint4 *>(hidden), reinterpret_cast<uint4 *>(w.h16),
                           n8),
                    "hidden f16 copy launch");
    hop = w.h16;
    pdl = true;
  }
  FH_CHECK_LAUNCH(prepare_s1_tc(), "stage-1 kernel attribute");
  const int m_tiles = (d.n_clusters + fh::kS1MTile - 1) / fh::kS1MTile;
  fh::S1TcArgs a;
  memset(&a, 0, sizeof(a));
  a.K = d.n_clusters;
  a.nk = (d.hidden + fh::kS1KBlock - 1) / fh::kS1KBlock;
  a.splits = w.splits;
  a.fp8 = fp8 ? 1 : 0;
  a.split_stride = w.split_stride;
  a.row_stride = w.score_stride;
  a.err = reinterpret_cast<uint32_t *>(w.counter) + fh::kSyncError;
  a.polls = 1u << 22;
  for (int r0 = 0; r0 < rows; r0 += fh::kS1MaxN) {
    const int n = std::min(fh::kS1MaxN, rows - r0);
    a.rows = n;
    a.n_pad = (n + 15) / 16 * 16;
    a.tmem_cols = 32;
    while (a.tmem_cols < a.n_pad) a.tmem_cols *= 2;
    const size_t sb = fh::s1tc_stage_bytes(a.n_pad, a.fp8);
    a.stages = (int)std::min<size_t>((size_t)fh::kS1MaxStages,
                                     ((size_t)fh::kS1SmemMax - 1024 - sizeof(fh::S1TcCtrl)) / sb);
    if (a.stages < 2) return fail(FH_ERR_UNSUPPORTED, "stage-1 ring does not fit");
    a.idesc = fh::s1tc_idesc(mma_bf16, a.n_pad);
    a.part = w.scores + (size_t)r0 * w.score_stride;
    CUtensorMap tm_h;
    const char *hrow = reinterpret_cast<const char *>(hop) + (size_t)r0 * d.hidden * 2;
    if (!encode_rows_map(&tm_h, hrow, mma_bf16 ? FH_BF16 : FH_FP16, d.hidden, n, a.n_pad))
      return fail(FH_ERR_UNSUPPORTED, "hidden-state tensor map");
    FH_CHECK_LAUNCH(launch(fh::k_s1_tc, dim3(m_tiles * a.splits), dim3(fh::kS1Threads),
                           fh::s1tc_smem_bytes(a.n_pad, a.fp8, a.stages), s, pdl, tm_c, tm_h, a),
                    "stage-1 tensor-core launch");
    pdl = false;
  }
  if (!probes && !cand_out && !scores_out) return FH_OK;
  FH_CHECK_LAUNCH(prepare_select_hist(), "select kernel attribute");
  fh::HSelArgs se;
  memset(&se, 0, sizeof(se));
  se.part = w.scores;
  se.split_stride = w.split_stride;
  se.row_stride = w.score_stride;
  se.splits = w.splits;
  se.K = d.n_clusters;
  se.p = d.n_probes;
  se.scale = sample ? d.centroid_scale : d.cluster_scale;
  se.do_sample = sample ? 1 : 0;
  se.temperature = temperature;
  se.rng = rng_key(seed, offset);
  se.cluster_base = d.cluster_base;
  se.scores_out = scores_out;
  se.out_stride = out_stride;
  se.probes = probes;
  se.cand_out = cand_out;
  se.bm = rows <= fh::kS2MaxRows ? s2_bm : nullptr;
  // more rows than SMs: two 512-thread CTAs per SM, so one wave selects every row
  if (rows > sm_count())
    FH_CHECK_LAUNCH(launch(fh::k_select_hist<512>, dim3(rows), dim3(512),
                           fh::hsel_smem_bytes(d.n_clusters, 512), s, true, se),
                    "probe selection launch");
  else
    FH_CHECK_LAUNCH(launch(fh::k_select_hist<1024>, dim3(rows), dim3(1024),
                           fh::hsel_smem_bytes(d.n_clusters, 1024), s, true, se),
                    "probe selection launch");
  return FH_OK;
}

cudaError_t prepare_s2_tc() {
  static bool done[128];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(fh::k_s2_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fh::kS2SmemMax);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fh::k_s2_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fh::kS2SmemMax);
    if (e != cudaSuccess) return e;
    done[dev] = true;
  }
  return cudaSuccess;
}

// Stage 2 of a batched step for given probe lists (cluster ids from
// probe_base), per chunk of up to kS2MaxRows rows: the index (the rows of
// every probed cluster), the tiles of 8 probed clusters with the union of
// their rows, and the cluster-major tensor-core stage 2 (k_s2_tc); then the
// special tokens and the publish of ids (out_ids) or of signed packed words
// (out_signed, tensor-parallel shards). packed[] must be zero on entry and is
// zero again on return.
int run_inv_stage2(const fh_head *h, const void *hidden, int rows, bool sample, float temperature,
                   uint64_t seed, uint64_t offset, const Workspace &w, const int32_t *probes,
                   int probe_base, int64_t *out_ids, long long *out_signed, cudaStream_t s,
                   bool index_ready = false) {
  const fh_head_desc &d = h->d;
  const fh::RngKey rng = rng_key(seed, offset);
  const int K = d.n_clusters, p = d.n_probes;
  if (!w.s2_bm) return fail(FH_ERR_WORKSPACE, "workspace laid out without the stage-2 index");
  const long long V = (long long)K * d.cluster_size;
  CUtensorMap tm_w, tm_w8;
  {
    std::lock_guard<std::mutex> lock(h->plan_mutex);
    if (!h->tm_s2_ok) {
      if (!encode_rows_map(&h->tm_s2, d.w_perm, d.weight_dtype, d.hidden, V, 16) ||
          !encode_rows_map(&h->tm_s2w, d.w_perm, d.weight_dtype, d.hidden, V,
                           fh::kS2Clusters * 16))
        return fail(FH_ERR_UNSUPPORTED, "w_perm tensor map");
      h->tm_s2_ok = true;
    }
    tm_w = h->tm_s2;
    tm_w8 = h->tm_s2w;
  }
  // window tiles need 16-row clusters (8 of them fill the MMA's 128 rows)
  const int window_min = d.cluster_size == 16 ? fh::kS2WindowMin : fh::kS2Clusters + 1;
  FH_CHECK_LAUNCH(prepare_s2_tc(), "stage-2 kernel attribute");
  // special tokens first: their words meet the probed ones in packed[], which
  // each stage-2 launch's last CTA publishes
  if (d.n_special > 0) {
    const long long warps = (long long)rows * d.n_special;
    const int n_slots = K * d.cluster_size;
    if (d.weight_dtype == FH_BF16)
      FH_CHECK_LAUNCH(launch(fh::k_special_scores<__nv_bfloat16>, dim3(grid_for(warps * 32, 256)),
                             dim3(256), 0, s, false, hidden, rows, d.hidden, d.w_perm, d.vocab_map,
                             d.special_slots, d.n_special, n_slots, sample ? 1 : 0, temperature,
                             rng, w.packed),
                      "special-token launch");
    else
      FH_CHECK_LAUNCH(launch(fh::k_special_scores<__half>, dim3(grid_for(warps * 32, 256)),
                             dim3(256), 0, s, false, hidden, rows, d.hidden, d.w_perm, d.vocab_map,
                             d.special_slots, d.n_special, n_slots, sample ? 1 : 0, temperature,
                             rng, w.packed),
                      "special-token launch");
  }
  const int tile_ctas = (K + fh::kS2TileClusters - 1) / fh::kS2TileClusters;
  for (int r0 = 0; r0 < rows; r0 += fh::kS2MaxRows) {
    const int n = std::min(fh::kS2MaxRows, rows - r0);
    // the selection may have filled the index of a single chunk already
    if (!(index_ready && rows <= fh::kS2MaxRows)) {
      FH_CHECK_LAUNCH(cudaMemsetAsync(w.s2_bm, 0, w.s2_zero_bytes, s), "index reset");
      const long long pairs = (long long)n * p;
      FH_CHECK_LAUNCH(launch(fh::k_s2_fill, dim3(grid_for(pairs, 256)), dim3(256), 0, s, false,
                             probes + (size_t)r0 * p, n, p, K, probe_base, w.s2_bm),
                      "index fill launch");
    }
    FH_CHECK_LAUNCH(launch(fh::k_s2_tiles, dim3(tile_ctas), dim3(256), 0, s, true,
                           (const uint32_t *)w.s2_bm, K, window_min, w.s2_tiles, w.s2_meta),
                    "tile build launch");
    fh::S2TcArgs a;
    memset(&a, 0, sizeof(a));
    a.hidden = reinterpret_cast<const char *>(hidden) + (size_t)r0 * d.hidden * 2;
    a.rows = n;
    a.D = d.hidden;
    a.nk = d.hidden / 64;
    a.cap = d.cluster_size;
    a.idesc0 = fh::s1tc_idesc(d.weight_dtype == FH_BF16, 0) & ~(0x3Fu << 17);
    a.vocab_map = d.vocab_map;
    a.tiles = w.s2_tiles;
    a.meta = w.s2_meta;
    a.do_sample = sample ? 1 : 0;
    a.temperature = temperature;
    a.rng = rng;
    a.row_base = r0;
    a.packed = w.packed + r0;
    a.err = reinterpret_cast<uint32_t *>(w.counter) + fh::kSyncError;
    a.polls = 1u << 22;
    a.done = reinterpret_cast<uint32_t *>(w.counter) + fh::kSyncS2Done;
    a.out_ids = out_ids ? out_ids + r0 : nullptr;
    a.out_signed = out_signed ? out_signed + r0 : nullptr;
    if (sample)
      FH_CHECK_LAUNCH(launch(fh::k_s2_tc<true>, dim3(sm_count()), dim3(fh::kS2Threads),
                             (size_t)fh::kS2SmemMax, s, true, tm_w, tm_w8, a),
                      "stage-2 tensor-core launch");
    else
      FH_CHECK_LAUNCH(launch(fh::k_s2_tc<false>, dim3(sm_count()), dim3(fh::kS2Threads),
                             (size_t)fh::kS2SmemMax, s, true, tm_w, tm_w8, a),
                      "stage-2 tensor-core launch");
  }
  return FH_OK;
}

// Batched step (rows >= kBatchMinRows): tensor-core stage 1 + selection,
// then the inverted stage 2.
int run_batched(const fh_head *h, const void *hidden, int rows, bool sample, float temperature,
                uint64_t seed, uint64_t offset, int64_t *out_ids, const Workspace &w,
                cudaStream_t s) {
  // up to 256 rows the selection writes the stage-2 index itself (cleared first)
  const bool index_in_select = rows <= fh::kS2MaxRows && w.s2_bm;
  if (index_in_select)
    FH_CHECK_LAUNCH(cudaMemsetAsync(w.s2_bm, 0, w.s2_zero_bytes, s), "index reset");
  const int st = run_s1_tc(h, hidden, rows, sample, temperature, seed, offset, w, nullptr, 0,
                           w.probes, nullptr, s, index_in_select ? w.s2_bm : nullptr);
  if (st != FH_OK) return st;
  return run_inv_stage2(h, hidden, rows, sample, temperature, seed, offset, w, w.probes, 0,
                        out_ids, nullptr, s, index_in_select);
}

// Tiling of the dense tensor-core kernel: vocab tiles of n_tile slots (a
// multiple of 16, at most 256) sized so the tiles split evenly over the SMs.
struct DenseTcPlan {
  int n_tile, n_tiles, mt, stages, grid, n_acc, acc_stride;
  size_t smem;
};
#ifndef FH_DT_MT2_DOUBLE_BUFFER
#define FH_DT_MT2_DOUBLE_BUFFER 0
#endif
bool dense_tc_plan(const fh_head_desc &d, int rows, DenseTcPlan *p) {
  const long long G = sm_count();
  const long long V = (long long)d.n_clusters * d.cluster_size;
  if (G <= 0 || rows < 1 || rows > fh::kDtMaxRows || V < 1 || V > (1ll << 30)) return false;
  p->mt = rows > fh::kDtMTile ? 2 : 1;
  // 512 TMEM columns: one hidden tile -> two 256-column accumulators; two
  // hidden tiles -> one set of two 256-column accumulators, or two sets of
  // 128 columns (narrower vocab tiles)
  const bool db = p->mt == 1 || FH_DT_MT2_DOUBLE_BUFFER;
  p->n_acc = db ? 2 : 1;
  p->acc_stride = fh::kDtTmemCols / (p->n_acc * p->mt);
  const long long cap_n = std::min<long long>(fh::kDtMaxTile, p->acc_stride);
  const long long t = (V + G * cap_n - 1) / (G * cap_n);
  long long n = 16 * ((V + 16 * G * t - 1) / (16 * G * t));
  n = std::min<long long>(std::max<long long>(n, 16), cap_n);
  p->n_tile = (int)n;
  p->n_tiles = (int)((V + n - 1) / n);
  const size_t sb = fh::dense_tc_stage_bytes(p->mt, p->n_tile);
  const size_t avail = (size_t)fh::kDtSmemMax - 1024 - sizeof(fh::DenseTcCtrl);
  p->stages = (int)std::min<size_t>((size_t)fh::kDtMaxStages, avail / sb);
  if (p->stages < 2) return false;
  p->smem = fh::dense_tc_smem_bytes(p->mt, p->n_tile, p->stages);
  p->grid = (int)std::min<long long>(G, p->n_tiles);
  return true;
}

cudaError_t prepare_dense_tc() {
  static bool done[128];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (!done[dev]) {
    e = cudaFuncSetAttribute(fh::k_dense_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fh::kDtSmemMax);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fh::k_dense_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fh::kDtSmemMax);
    if (e != cudaSuccess) return e;
    done[dev] = true;
  }
  return cudaSuccess;
}

// Dense head in one tensor-core kernel per 256 hidden rows (logits stay on
// chip; greedy argmax, or Gumbel-max in sampling mode). Returns
// FH_ERR_UNSUPPORTED without launching anything when the shape or the tensor
// maps do not fit it; the caller then takes the block-sparse route over every
// cluster.
int run_dense_tc(const fh_head *h, const void *hidden, int rows, bool sample, float temperature,
                 uint64_t seed, uint64_t offset, int64_t *out_ids, const Workspace &w,
                 cudaStream_t s) {
  const fh_head_desc &d = h->d;
  if ((d.flags & FH_FLAG_NO_FUSED) || d.cluster_base != 0 || rows < fh::kBatchMinRows)
    return FH_ERR_UNSUPPORTED;
  const long long V = (long long)d.n_clusters * d.cluster_size;
  for (int r0 = 0; r0 < rows; r0 += fh::kDtMaxRows) {
    const int n = std::min(fh::kDtMaxRows, rows - r0);
    DenseTcPlan pl;
    if (!dense_tc_plan(d, n, &pl)) return FH_ERR_UNSUPPORTED;
    CUtensorMap tm_w, tm_h;
    {
      std::lock_guard<std::mutex> lock(h->plan_mutex);
      if (h->tm_w_tile != pl.n_tile) {
        if (!encode_rows_map(&h->tm_w, d.w_perm, d.weight_dtype, d.hidden, V, pl.n_tile))
          return FH_ERR_UNSUPPORTED;
        h->tm_w_tile = pl.n_tile;
      }
      tm_w = h->tm_w;
    }
    const char *hrow = reinterpret_cast<const char *>(hidden) + (size_t)r0 * d.hidden * 2;
    if (!encode_rows_map(&tm_h, hrow, d.weight_dtype, d.hidden, n, fh::kDtMTile))
      return FH_ERR_UNSUPPORTED;
    FH_CHECK_LAUNCH(prepare_dense_tc(), "dense tensor-core kernel attribute");
    fh::DenseTcArgs a;
    memset(&a, 0, sizeof(a));
    a.rows = n;
    a.V = (int)V;
    a.n_tile = pl.n_tile;
    a.n_tiles = pl.n_tiles;
    a.mt = pl.mt;
    a.stages = pl.stages;
    a.n_acc = pl.n_acc;
    a.acc_stride = pl.acc_stride;
    a.nk = (d.hidden + fh::kDtKBlock - 1) / fh::kDtKBlock;
    a.idesc = fh::dense_tc_idesc(d.weight_dtype == FH_BF16, pl.n_tile);
    a.vocab_map = d.vocab_map;
    a.packed = w.packed + r0;
    a.err = reinterpret_cast<uint32_t *>(w.counter) + fh::kSyncError;
    a.polls = 1u << 22;
    a.do_sample = sample ? 1 : 0;
    a.temperature = temperature;
    a.rng = rng_key(seed, offset);
    a.row_base = r0;
    if (sample)
      FH_CHECK_LAUNCH(launch(fh::k_dense_tc<true>, dim3(pl.grid), dim3(fh::kDtThreads), pl.smem,
                             s, false, tm_h, tm_w, a),
                      "dense tensor-core launch");
    else
      FH_CHECK_LAUNCH(launch(fh::k_dense_tc<false>, dim3(pl.grid), dim3(fh::kDtThreads), pl.smem,
                             s, false, tm_h, tm_w, a),
                      "dense tensor-core launch");
  }
  FH_CHECK_LAUNCH(launch(fh::k_inv_finalize, dim3(grid_for(rows, 256)), dim3(256), 0, s, false,
                         w.packed, rows, out_ids, (long long *)nullptr),
                  "finalize launch");
  return FH_OK;
}

int validate_desc(const fh_head_desc *d) {
  if (!d) return fail(FH_ERR_INVALID_ARGUMENT, "null descriptor");
  if (d->hidden <= 0 || d->hidden % 16 != 0)
    return fail(FH_ERR_INVALID_ARGUMENT, "hidden=%d must be a positive multiple of 16", d->hidden);
  if (d->n_clusters <= 0 || d->n_clusters > fh::kSelMaxItems)
    return fail(FH_ERR_INVALID_ARGUMENT, "n_clusters=%d outside 1..%d", d->n_clusters,
                fh::kSelMaxItems);
  if (d->cluster_size < 1 || d->cluster_size > 32)
    return fail(FH_ERR_INVALID_ARGUMENT, "cluster_size=%d outside 1..32", d->cluster_size);
  if (d->n_probes < 1 || d->n_probes > d->n_clusters)
    return fail(FH_ERR_INVALID_ARGUMENT, "n_probes=%d outside 1..n_clusters=%d", d->n_probes,
                d->n_clusters);
  if (d->weight_dtype != FH_BF16 && d->weight_dtype != FH_FP16)
    return fail(FH_ERR_INVALID_ARGUMENT, "weight_dtype must be FH_BF16 or FH_FP16");
  if (d->score_dtype != FH_FP8_E4M3 && d->score_dtype != d->weight_dtype)
    return fail(FH_ERR_INVALID_ARGUMENT, "score_dtype must be FH_FP8_E4M3 or weight_dtype");
  if (d->centroid_w && d->sample_dtype != FH_FP8_E4M3 && d->sample_dtype != d->weight_dtype)
    return fail(FH_ERR_INVALID_ARGUMENT, "sample_dtype must be FH_FP8_E4M3 or weight_dtype");
  if (!d->w_perm || !d->vocab_map || !d->cluster_w)
    return fail(FH_ERR_INVALID_ARGUMENT, "w_perm, vocab_map and cluster_w are required");
  if (!aligned16(d->w_perm) || !aligned16(d->cluster_w) ||
      (d->centroid_w && !aligned16(d->centroid_w)))
    return fail(FH_ERR_INVALID_ARGUMENT, "weight matrices must be 16-byte aligned");
  if ((d->score_dtype == FH_FP8_E4M3) != (d->cluster_scale != nullptr))
    return fail(FH_ERR_INVALID_ARGUMENT, "cluster_scale is required exactly for fp8 cluster_w");
  if (d->centroid_w && (d->sample_dtype == FH_FP8_E4M3) != (d->centroid_scale != nullptr))
    return fail(FH_ERR_INVALID_ARGUMENT, "centroid_scale is required exactly for fp8 centroid_w");
  if (d->n_special < 0 || (d->n_special > 0 && !d->special_slots))
    return fail(FH_ERR_INVALID_ARGUMENT, "n_special=%d with null special_slots", d->n_special);
  if (d->cluster_base < 0) return fail(FH_ERR_INVALID_ARGUMENT, "cluster_base < 0");
  return FH_OK;
}

}  // namespace

// ===========================================================================
// Exported functions
// ===========================================================================
extern "C" {

FH_API int fh_version(void) { return 1; }

#ifdef FH_TRACE
// Profiling builds only (not declared in the public header): device buffer
// for the one-kernel step's phase stamps, passed to every later launch.
FH_API int fh_debug_set_trace(void *buf) {
  g_trace_buf = reinterpret_cast<unsigned long long *>(buf);
  return FH_OK;
}
#endif

FH_API const char *fh_last_error(void) { return g_last_error.c_str(); }

FH_API int fh_head_create(const fh_head_desc *desc, fh_head **out) {
  if (!out) return fail(FH_ERR_INVALID_ARGUMENT, "null output handle pointer");
  *out = nullptr;
  const int st = validate_desc(desc);
  if (st != FH_OK) return st;
  fh_head *h = new (std::nothrow) fh_head;
  if (!h) return fail(FH_ERR_INVALID_ARGUMENT, "out of host memory");
  h->d = *desc;
  *out = h;
  return FH_OK;
}

FH_API int fh_head_destroy(fh_head *head) {
  if (head) {
  }
  delete head;
  return FH_OK;
}

FH_API int fh_step_kernel_count(const fh_head *head, int rows, int do_sample) {
  if (!head || rows <= 0) return 0;
  const fh_head_desc &d = head->d;
  const bool sample = do_sample != 0;
  const int cdt = sample ? d.sample_dtype : d.score_dtype;
  // tensor-core stage 1: [f16 copy of bf16 rows], one k_s1_tc per 256 rows, select
  const int s1 = (cdt == FH_FP8_E4M3 && d.weight_dtype == FH_BF16 ? 1 : 0) +
                 (rows + fh::kS1MaxN - 1) / fh::kS1MaxN + 1;
  if (batched_ok(head, rows, sample)) {
    // stage 1 (whose selection fills the stage-2 index up to 256 rows);
    // [specials]; per 256 rows: [index fill], tiles, stage 2 (publishing)
    const int chunks = (rows + fh::kS2MaxRows - 1) / fh::kS2MaxRows;
    return s1 + (d.n_special > 0 ? 1 : 0) + (chunks > 1 ? 3 : 2) * chunks;
  }
  if (fused_ok(d, rows, sample, sm_count())) return 1;
  // stage 1 + stage 2; or scores, select, stage 2
  if (rows >= fh::kGemmS1MinRows && s1_tc_ok(d, sample)) return s1 + 1;
  return 3;
}

FH_API size_t fh_workspace_error_offset(void) { return fh::kSyncError * sizeof(uint32_t); }

FH_API size_t fh_workspace_bytes(const fh_head *head, int rows) {
  if (!head || rows < 0) return 0;
  return layout(head->d, rows, nullptr, 0).bytes;
}

FH_API int fh_get_next_token(const fh_head *head, const void *hidden, int rows,
                             int64_t *out_ids, void *workspace, size_t workspace_bytes,
                             fh_stream_t stream) {
  int st = check_call(head, hidden, rows, out_ids, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  const int grid = sm_count();
  if (batched_ok(head, rows, false))
    return run_batched(head, hidden, rows, false, 1.f, 0, 0, out_ids, w, s);
  if (fused_ok(head->d, rows, false, grid) && aligned16(hidden))
    return run_fused(head, hidden, rows, false, 1.f, 0, 0, out_ids, w, grid, s);
  if (rows >= fh::kGemmS1MinRows && s1_tc_ok(head->d, false))
    st = run_s1_tc(head, hidden, rows, false, 1.f, 0, 0, w, nullptr, 0, w.probes, nullptr, s);
  else
    st = run_stage1(head, hidden, rows, false, 1.f, 0, 0, w, nullptr, w.probes, nullptr, 0, s);
  if (st != FH_OK) return st;
  fh::Stage2Args a = stage2_args(head->d, hidden, rows);
  a.probes = w.probes;
  a.probe_stride = head->d.n_probes;
  a.P = head->d.n_probes;
  a.cluster_base = 0;
  a.packed = w.packed;
  a.counter = w.counter;
  a.out_ids = out_ids;
  a.wait_prior = 1;
  const int items = rows * (a.P + a.n_special);
  FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kGreedy>(head->d.weight_dtype, a, items, s, true)),
                  "stage-2 launch");
  return FH_OK;
}

namespace {
// Device address of a page-locked host buffer (with unified addressing, the
// same address), or null for pageable memory.
void *mapped_host(const void *p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

size_t host_staging_bytes(const fh_head *head, int rows) {
  return round_up((size_t)rows * head->d.hidden * 2, 256) + round_up((size_t)rows * 8, 256);
}
}  // namespace

FH_API size_t fh_workspace_bytes_host(const fh_head *head, int rows) {
  if (!head || rows < 0) return 0;
  return round_up(layout(head->d, rows, nullptr, 0).bytes, 256) + host_staging_bytes(head, rows);
}

// Longest host spin on the ids of a host-buffer call before falling back to a
// stream synchronisation.
static constexpr int kHostSpinMs = 20;

FH_API int fh_get_next_token_host(const fh_head *head, const void *hidden_host, int rows,
                                  int64_t *out_ids_host, void *workspace, size_t workspace_bytes,
                                  fh_stream_t stream) {
  if (!head) return fail(FH_ERR_INVALID_ARGUMENT, "null head");
  if (rows < 0) return fail(FH_ERR_INVALID_ARGUMENT, "rows=%d < 0", rows);
  if (rows == 0) return FH_OK;
  if (!hidden_host || !out_ids_host) return fail(FH_ERR_INVALID_ARGUMENT, "null host buffer");
  if (!workspace) return fail(FH_ERR_WORKSPACE, "null workspace");
  const size_t need = fh_workspace_bytes_host(head, rows);
  if (workspace_bytes < need)
    return fail(FH_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed for %d host rows",
                workspace_bytes, need, rows);
  // staging at the end of the workspace; the step's own layout below it
  const size_t stage = host_staging_bytes(head, rows);
  const size_t inner = (workspace_bytes / 256) * 256 - stage;
  char *base = reinterpret_cast<char *>(workspace);
  void *dev_h = base + inner;
  int64_t *dev_out = reinterpret_cast<int64_t *>(base + inner +
                                                 round_up((size_t)rows * head->d.hidden * 2, 256));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t hbytes = (size_t)rows * head->d.hidden * 2;
  // Page-locked host buffers are read and written by the kernels themselves
  // over the bus (one small copy kernel in, the step's own id stores out),
  // which costs less latency than two copy-engine transfers; pageable ones
  // go through cudaMemcpyAsync.
  const void *h_mapped = mapped_host(hidden_host);
  if (!(h_mapped && aligned16(h_mapped) && hbytes % 16 == 0)) h_mapped = nullptr;
  int64_t *o_mapped = reinterpret_cast<int64_t *>(mapped_host(out_ids_host));
  // Ids written over the bus land in the host buffer before the kernel has
  // finished: mark every row (-1 is never an id) and return once all rows
  // are overwritten, instead of waiting for the stream to drain.
  volatile int64_t *watch = o_mapped ? reinterpret_cast<volatile int64_t *>(out_ids_host) : nullptr;
  if (watch)
    for (int r = 0; r < rows; ++r) watch[r] = -1;
  if (h_mapped) {
    const int n16 = (int)(hbytes / 16);
    FH_CHECK_LAUNCH(launch(fh::k_stage_in, dim3(grid_for(n16, 256)), dim3(256), 0, s, false,
                           reinterpret_cast<uint4 *>(dev_h),
                           reinterpret_cast<const uint4 *>(h_mapped), n16),
                    "hidden-state copy kernel");
  } else {
    FH_CHECK_LAUNCH(cudaMemcpyAsync(dev_h, hidden_host, hbytes, cudaMemcpyHostToDevice, s),
                    "hidden-state copy to the device");
  }
  const int st =
      fh_get_next_token(head, dev_h, rows, o_mapped ? o_mapped : dev_out, workspace, inner, stream);
  if (st != FH_OK) return st;
  if (!o_mapped)
    FH_CHECK_LAUNCH(cudaMemcpyAsync(out_ids_host, dev_out, (size_t)rows * sizeof(int64_t),
                                    cudaMemcpyDeviceToHost, s),
                    "id copy to the host");
  if (watch) {
    // bounded spin (then the stream synchronisation below reports any error)
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t it = 0;; ++it) {
      int r = 0;
      while (r < rows && watch[r] != -1) ++r;
      if (r == rows) {
        std::atomic_thread_fence(std::memory_order_acquire);
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess || q == cudaErrorNotReady) return FH_OK;
        return fail(FH_ERR_CUDA, "stream: %s", cudaGetErrorString(q));
      }
      if ((it & 1023u) == 1023u &&
          std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(kHostSpinMs))
        break;
    }
  }
  FH_CHECK_LAUNCH(cudaStreamSynchronize(s), "stream synchronisation");
  return FH_OK;
}

FH_API int fh_get_next_token_sample(const fh_head *head, const void *hidden, int rows,
                                    float temperature, uint64_t seed, uint64_t offset,
                                    int64_t *out_ids, void *workspace, size_t workspace_bytes,
                                    fh_stream_t stream) {
  int st = check_call(head, hidden, rows, out_ids, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  st = check_sampling(head, temperature);
  if (st != FH_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  const int grid = sm_count();
  if (batched_ok(head, rows, true))
    return run_batched(head, hidden, rows, true, temperature, seed, offset, out_ids, w, s);
  if (fused_ok(head->d, rows, true, grid) && aligned16(hidden))
    return run_fused(head, hidden, rows, true, temperature, seed, offset, out_ids, w, grid, s);
  if (rows >= fh::kGemmS1MinRows && s1_tc_ok(head->d, true))
    st = run_s1_tc(head, hidden, rows, true, temperature, seed, offset, w, nullptr, 0, w.probes,
                   nullptr, s);
  else
    st = run_stage1(head, hidden, rows, true, temperature, seed, offset, w, nullptr, w.probes,
                    nullptr, 0, s);
  if (st != FH_OK) return st;
  fh::Stage2Args a = stage2_args(head->d, hidden, rows);
  a.probes = w.probes;
  a.probe_stride = head->d.n_probes;
  a.P = head->d.n_probes;
  a.cluster_base = 0;
  a.packed = w.packed;
  a.counter = w.counter;
  a.out_ids = out_ids;
  a.temperature = temperature;
  a.rng = rng_key(seed, offset);
  a.wait_prior = 1;
  const int items = rows * (a.P + a.n_special);
  FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kSample>(head->d.weight_dtype, a, items, s, true)),
                  "stage-2 launch");
  return FH_OK;
}

FH_API int fh_top_clusters(const fh_head *head, const void *hidden, int rows, int do_sample,
                           float temperature, uint64_t seed, uint64_t offset,
                           int32_t *out_probes, float *out_scores, void *workspace,
                           size_t workspace_bytes, fh_stream_t stream) {
  int st = check_call(head, hidden, rows, out_probes, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  if (do_sample) {
    st = check_sampling(head, temperature);
    if (st != FH_OK) return st;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  // the stage 1 of the step the library runs for this many rows
  if (rows >= fh::kGemmS1MinRows && s1_tc_ok(head->d, do_sample != 0))
    return run_s1_tc(head, hidden, rows, do_sample != 0, temperature, seed, offset, w, out_scores,
                     head->d.n_clusters, out_probes, nullptr, s);
  return run_stage1(head, hidden, rows, do_sample != 0, temperature, seed, offset, w, out_scores,
                    out_probes, nullptr, 0, s);
}

FH_API int fh_cluster_scores(const fh_head *head, const void *hidden, int rows, int do_sample,
                             float temperature, uint64_t seed, uint64_t offset, float *out_scores,
                             fh_stream_t stream) {
  if (!head) return fail(FH_ERR_INVALID_ARGUMENT, "null head");
  if (rows < 0) return fail(FH_ERR_INVALID_ARGUMENT, "rows=%d < 0", rows);
  if (rows == 0) return FH_OK;
  if (!hidden || !out_scores) return fail(FH_ERR_INVALID_ARGUMENT, "null hidden/output pointer");
  if (!aligned16(hidden))
    return fail(FH_ERR_INVALID_ARGUMENT, "hidden states must be 16-byte aligned");
  if (do_sample) {
    const int st = check_sampling(head, temperature);
    if (st != FH_OK) return st;
  }
  fh::ScoresArgs sa =
      scores_args(head->d, hidden, rows, do_sample != 0, temperature, seed, offset);
  sa.scores = out_scores;
  sa.score_stride = head->d.n_clusters;
  const int wdt = do_sample ? head->d.sample_dtype : head->d.score_dtype;
  FH_CHECK_LAUNCH(launch_scores(head->d.weight_dtype, wdt, sa, reinterpret_cast<cudaStream_t>(stream)),
                  "stage-1 scores launch");
  return FH_OK;
}

FH_API int fh_stage2_next_token(const fh_head *head, const void *hidden, int rows,
                                const int32_t *probes, int do_sample, float temperature,
                                uint64_t seed, uint64_t offset, int64_t *out_ids, void *workspace,
                                size_t workspace_bytes, fh_stream_t stream) {
  int st = check_call(head, hidden, rows, out_ids, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  if (!probes) return fail(FH_ERR_INVALID_ARGUMENT, "null probe list");
  if (do_sample && (!(temperature > 0.f) || !std::isfinite(temperature)))
    return fail(FH_ERR_INVALID_ARGUMENT, "temperature must be positive and finite");
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the stage 2 fh_get_next_token runs for this many rows
  if (inv_ok(head->d, rows) && head->d.cluster_base == 0)
    return run_inv_stage2(head, hidden, rows, do_sample != 0, do_sample ? temperature : 1.f, seed,
                          offset, w, probes, 0, out_ids, nullptr, s);
  fh::Stage2Args a = stage2_args(head->d, hidden, rows);
  a.probes = probes;
  a.probe_stride = head->d.n_probes;
  a.P = head->d.n_probes;
  a.cluster_base = 0;
  a.packed = w.packed;
  a.counter = w.counter;
  a.out_ids = out_ids;
  a.temperature = do_sample ? temperature : 1.f;
  a.rng = rng_key(seed, offset);
  const int items = rows * (a.P + a.n_special);
  if (do_sample)
    FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kSample>(head->d.weight_dtype, a, items, s, false)),
                    "stage-2 launch");
  else
    FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kGreedy>(head->d.weight_dtype, a, items, s, false)),
                    "stage-2 launch");
  return FH_OK;
}

FH_API int fh_dense_next_token(const fh_head *head, const void *hidden, int rows, int do_sample,
                               float temperature, uint64_t seed, uint64_t offset,
                               int64_t *out_ids, void *workspace, size_t workspace_bytes,
                               fh_stream_t stream) {
  int st = check_call(head, hidden, rows, out_ids, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  if (do_sample && (!(temperature > 0.f) || !std::isfinite(temperature)))
    return fail(FH_ERR_INVALID_ARGUMENT, "temperature must be positive and finite");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  st = run_dense_tc(head, hidden, rows, do_sample != 0, temperature, seed, offset, out_ids, w, s);
  if (st != FH_ERR_UNSUPPORTED) return st;
  FH_CHECK_LAUNCH(launch(fh::k_fill_u64, dim3((rows + 255) / 256), dim3(256), 0, s, false,
                         w.packed, rows, 0ull),
                  "fill launch");
  FH_CHECK_LAUNCH(launch(fh::k_fill_u64, dim3(1), dim3(32), 0, s, false,
                         reinterpret_cast<unsigned long long *>(w.counter), 1, 0ull),
                  "fill launch");
  fh::Stage2Args a = stage2_args(head->d, hidden, rows);
  a.dense = 1;
  a.P = head->d.n_clusters;
  a.n_special = 0;
  a.cluster_base = 0;
  a.packed = w.packed;
  a.counter = w.counter;
  a.out_ids = out_ids;
  a.temperature = temperature;
  a.rng = rng_key(seed, offset);
  const int items = rows * a.P;
  if (do_sample)
    FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kSample>(head->d.weight_dtype, a, items, s, false)),
                    "dense launch");
  else
    FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kGreedy>(head->d.weight_dtype, a, items, s, false)),
                    "dense launch");
  return FH_OK;
}

// ---------------------------------------------------------------------------
// Greedy step with library-owned scratch (no workspace argument, no
// allocation): a file-scope device array, laid out for the three-kernel path
// as counter | packed[4] | probes[4][4096] | scores[4][16384].
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocProbesOff = 512;
constexpr size_t kNoAllocScoresOff =
    kNoAllocProbesOff + (size_t)FH_NOALLOC_MAX_ROWS * FH_NOALLOC_MAX_PROBES * sizeof(int32_t);
constexpr size_t kNoAllocBytes =
    kNoAllocScoresOff + (size_t)FH_NOALLOC_MAX_ROWS * FH_NOALLOC_MAX_CLUSTERS * sizeof(float);
static_assert(kNoAllocBytes == FH_NOALLOC_SCRATCH_BYTES, "scratch size out of sync with the header");
static_assert(FH_NOALLOC_MAX_CLUSTERS % 64 == 0, "score rows are padded to 64 clusters");
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_noalloc_mutex;
void *g_noalloc_addr[128];

// Device address of g_noalloc_scratch on the current device, looked up once.
int noalloc_scratch(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "current device");
  if (dev < 0 || dev >= 128) return fail(FH_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "address of the fixed scratch array");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return FH_OK;
}
}  // namespace

extern "C" FH_API int fh_get_next_token_noalloc(const fh_head *head, const void *hidden,
                                                int rows, int64_t *out_ids, fh_stream_t stream) {
  if (!head) return fail(FH_ERR_INVALID_ARGUMENT, "null head");
  if (rows < 0) return fail(FH_ERR_INVALID_ARGUMENT, "rows=%d < 0", rows);
  if (rows == 0) return FH_OK;
  if (rows > FH_NOALLOC_MAX_ROWS)
    return fail(FH_ERR_UNSUPPORTED, "rows=%d exceeds the fixed scratch limit of %d rows", rows,
                FH_NOALLOC_MAX_ROWS);
  if (head->d.n_clusters > FH_NOALLOC_MAX_CLUSTERS || head->d.n_probes > FH_NOALLOC_MAX_PROBES)
    return fail(FH_ERR_UNSUPPORTED,
                "n_clusters=%d / n_probes=%d exceed the fixed scratch limits (%d / %d)",
                head->d.n_clusters, head->d.n_probes, FH_NOALLOC_MAX_CLUSTERS,
                FH_NOALLOC_MAX_PROBES);
  if (!hidden || !out_ids) return fail(FH_ERR_INVALID_ARGUMENT, "null hidden/output pointer");
  if (!aligned16(hidden))
    return fail(FH_ERR_INVALID_ARGUMENT, "hidden states must be 16-byte aligned");
  void *base = nullptr;
  int st = noalloc_scratch(&base);
  if (st != FH_OK) return st;
  char *p = reinterpret_cast<char *>(base);
  Workspace w;
  w.counter = reinterpret_cast<unsigned *>(p);
  w.packed = reinterpret_cast<unsigned long long *>(p + 256);
  w.probes = reinterpret_cast<int32_t *>(p + kNoAllocProbesOff);
  w.scores = reinterpret_cast<float *>(p + kNoAllocScoresOff);
  w.score_stride = (int)round_up((size_t)head->d.n_clusters, 64);
  w.splits = 1;
  w.split_stride = (size_t)rows * w.score_stride;
  w.epoch_bufs = nullptr;
  w.h16 = nullptr;
  w.s2_bm = nullptr;
  w.s2_meta = nullptr;
  w.s2_tiles = nullptr;
  w.s2_zero_bytes = 0;
  w.bytes = kNoAllocBytes;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // k_scores zeroes the accumulator and the counter before stage 2 uses them.
  st = run_stage1(head, hidden, rows, false, 1.f, 0, 0, w, nullptr, w.probes, nullptr, 0, s);
  if (st != FH_OK) return st;
  fh::Stage2Args a = stage2_args(head->d, hidden, rows);
  a.probes = w.probes;
  a.probe_stride = head->d.n_probes;
  a.P = head->d.n_probes;
  a.cluster_base = 0;
  a.packed = w.packed;
  a.counter = w.counter;
  a.out_ids = out_ids;
  a.wait_prior = 1;
  const int items = rows * (a.P + a.n_special);
  FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kGreedy>(head->d.weight_dtype, a, items, s, true)),
                  "stage-2 launch");
  return FH_OK;
}

// ---------------------------------------------------------------------------
// Stateless kernels with the reference's layout (fused.py)
// ---------------------------------------------------------------------------
static int check_stateless(const void *hs, int T, int D, const void *w_perm, const int64_t *ci,
                           int P, int K, int cap, int dtype, const void *out) {
  if (T < 0 || P < 0) return fail(FH_ERR_INVALID_ARGUMENT, "negative T or P");
  if (T == 0 || P == 0) return FH_OK;
  if (!hs || !w_perm || !ci || !out)
    return fail(FH_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (D <= 0 || D % 8 != 0)
    return fail(FH_ERR_INVALID_ARGUMENT, "D=%d must be a positive multiple of 8", D);
  if (K <= 0 || cap < 1 || cap > 32)
    return fail(FH_ERR_INVALID_ARGUMENT, "n_clusters=%d / cluster_size=%d invalid", K, cap);
  if (dtype != FH_BF16 && dtype != FH_FP16)
    return fail(FH_ERR_INVALID_ARGUMENT, "dtype must be FH_BF16 or FH_FP16");
  if (!aligned16(hs) || !aligned16(w_perm))
    return fail(FH_ERR_INVALID_ARGUMENT, "hs and w_perm must be 16-byte aligned");
  if ((long long)T * P > 0x7FFFFFFFll) return fail(FH_ERR_INVALID_ARGUMENT, "T*P too large");
  return FH_OK;
}

static fh::Stage2Args stateless_args(const void *hs, int T, int D, const void *w_perm,
                                     const int64_t *ci, int P, const int64_t *vocab_maps, int K,
                                     int cap) {
  fh::Stage2Args a;
  memset(&a, 0, sizeof(a));
  a.hidden = hs;
  a.rows = T;
  a.D = D;
  a.w_perm = w_perm;
  a.K = K;
  a.cap = cap;
  a.probes = ci;
  a.probe_stride = P;
  a.P = P;
  a.vocab_map = vocab_maps;
  a.temperature = 1.f;
  return a;
}

FH_API int fh_block_sparse_logits(const void *hs, int T, int D, const void *w_perm,
                                  const int64_t *ci, int P, int n_clusters, int cluster_size,
                                  int dtype, void *out, fh_stream_t stream) {
  int st = check_stateless(hs, T, D, w_perm, ci, P, n_clusters, cluster_size, dtype, out);
  if (st != FH_OK || T == 0 || P == 0) return st;
  fh::Stage2Args a = stateless_args(hs, T, D, w_perm, ci, P, nullptr, n_clusters, cluster_size);
  a.out_logits = out;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  FH_CHECK_LAUNCH((launch_stage2<int64_t, fh::kLogits>(dtype, a, T * P, s, false)),
                  "block_sparse_logits launch");
  return FH_OK;
}

FH_API int fh_block_sparse_logits_argmax(const void *hs, int T, int D, const void *w_perm,
                                         const int64_t *ci, int P, const int64_t *vocab_maps,
                                         int n_clusters, int cluster_size, int dtype,
                                         void *out_max, int64_t *out_vocab, fh_stream_t stream) {
  int st = check_stateless(hs, T, D, w_perm, ci, P, n_clusters, cluster_size, dtype, out_max);
  if (st != FH_OK || T == 0 || P == 0) return st;
  if (!vocab_maps || !out_vocab) return fail(FH_ERR_INVALID_ARGUMENT, "null pointer argument");
  fh::Stage2Args a =
      stateless_args(hs, T, D, w_perm, ci, P, vocab_maps, n_clusters, cluster_size);
  a.out_max = out_max;
  a.out_vocab = out_vocab;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  FH_CHECK_LAUNCH((launch_stage2<int64_t, fh::kProbeMax>(dtype, a, T * P, s, false)),
                  "block_sparse_logits_argmax launch");
  return FH_OK;
}

FH_API int fh_block_sparse_argmax_atomic(const void *hs, int T, int D, const void *w_perm,
                                         const int64_t *ci, int P, const int64_t *vocab_maps,
                                         int n_clusters, int cluster_size, int dtype,
                                         int64_t *out, fh_stream_t stream) {
  int st = check_stateless(hs, T, D, w_perm, ci, P, n_clusters, cluster_size, dtype, out);
  if (st != FH_OK || T == 0) return st;
  if (!vocab_maps && P > 0) return fail(FH_ERR_INVALID_ARGUMENT, "null vocab_maps");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned long long *acc = reinterpret_cast<unsigned long long *>(out);
  FH_CHECK_LAUNCH(launch(fh::k_fill_u64, dim3((T + 255) / 256), dim3(256), 0, s, false, acc, T,
                         0ull),
                  "fill launch");
  if (P > 0) {
    fh::Stage2Args a =
        stateless_args(hs, T, D, w_perm, ci, P, vocab_maps, n_clusters, cluster_size);
    a.packed = acc;
    FH_CHECK_LAUNCH((launch_stage2<int64_t, fh::kGreedy>(dtype, a, T * P, s, false)),
                    "block_sparse_argmax_atomic launch");
  }
  FH_CHECK_LAUNCH(launch(fh::k_unpack_ids, dim3((T + 255) / 256), dim3(256), 0, s, false, acc, T),
                  "unpack launch");
  return FH_OK;
}

FH_API int fh_spec_accept(const int32_t *draft_ids, const int32_t *target_ids,
                          const int32_t *bonus_ids, const int32_t *cu_num_draft, int batch,
                          int max_spec_len, int32_t placeholder, int32_t *out_ids,
                          fh_stream_t stream) {
  if (batch < 0) return fail(FH_ERR_INVALID_ARGUMENT, "batch=%d < 0", batch);
  if (max_spec_len < 0 || max_spec_len > 4096)
    return fail(FH_ERR_INVALID_ARGUMENT, "max_spec_len=%d outside 0..4096", max_spec_len);
  if (batch == 0) return FH_OK;
  if (!bonus_ids || !cu_num_draft || !out_ids ||
      (max_spec_len > 0 && (!draft_ids || !target_ids)))
    return fail(FH_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int warps_per_block = 8;
  FH_CHECK_LAUNCH(launch(fh::k_spec_accept, dim3((batch + warps_per_block - 1) / warps_per_block),
                         dim3(32 * warps_per_block), 0, s, false, draft_ids, target_ids,
                         bonus_ids, cu_num_draft, batch, max_spec_len, placeholder, out_ids),
                  "draft acceptance launch");
  return FH_OK;
}

// ---------------------------------------------------------------------------
// Tensor parallel
// ---------------------------------------------------------------------------
FH_API int fh_tp_local_candidates(const fh_head *head, const void *hidden, int rows,
                                  int do_sample, float temperature, uint64_t seed,
                                  uint64_t offset, int64_t *cand, void *workspace,
                                  size_t workspace_bytes, fh_stream_t stream) {
  int st = check_call(head, hidden, rows, cand, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  if (do_sample) {
    st = check_sampling(head, temperature);
    if (st != FH_OK) return st;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  if (rows >= fh::kGemmS1MinRows && s1_tc_ok(head->d, do_sample != 0))
    return run_s1_tc(head, hidden, rows, do_sample != 0, temperature, seed, offset, w, nullptr, 0,
                     nullptr, reinterpret_cast<long long *>(cand), s);
  return run_stage1(head, hidden, rows, do_sample != 0, temperature, seed, offset, w, nullptr,
                    nullptr, reinterpret_cast<long long *>(cand), head->d.cluster_base, s);
}

FH_API int fh_tp_select_and_score(const fh_head *head, const void *hidden, int rows, int n_ranks,
                                  const int64_t *all_cand, int do_sample, float temperature,
                                  uint64_t seed, uint64_t offset, int64_t *best, void *workspace,
                                  size_t workspace_bytes, fh_stream_t stream) {
  int st = check_call(head, hidden, rows, best, workspace, workspace_bytes);
  if (st != FH_OK || rows == 0) return st;
  if (!all_cand) return fail(FH_ERR_INVALID_ARGUMENT, "null candidate list");
  if (n_ranks < 1 || (long long)n_ranks * head->d.n_probes > fh::kSelMaxItems)
    return fail(FH_ERR_INVALID_ARGUMENT, "n_ranks=%d x n_probes=%d exceeds %d candidates",
                n_ranks, head->d.n_probes, fh::kSelMaxItems);
  if (do_sample && (!(temperature > 0.f) || !std::isfinite(temperature)))
    return fail(FH_ERR_INVALID_ARGUMENT, "temperature must be positive and finite");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = layout(head->d, rows, workspace, workspace_bytes);
  FH_CHECK_LAUNCH(prepare_select(), "select kernel attribute");
  fh::SelectArgs se;
  memset(&se, 0, sizeof(se));
  se.cand = reinterpret_cast<const long long *>(all_cand);
  se.p_in = head->d.n_probes;
  se.n_ranks = n_ranks;
  se.rows = rows;
  se.n_items = n_ranks * head->d.n_probes;
  se.p = head->d.n_probes;
  se.probes = w.probes;
  se.packed = w.packed;
  se.counter = w.counter;
  se.n_packed = rows;
  se.wait_prior = 0;
  const size_t smem = (size_t)se.n_items * sizeof(unsigned long long);
  FH_CHECK_LAUNCH(launch(fh::k_select, dim3(rows), dim3(fh::kSelThreads), smem, s, false, se),
                  "global probe selection launch");
  if (inv_ok(head->d, rows))  // the global probes this shard owns, cluster-major
    return run_inv_stage2(head, hidden, rows, do_sample != 0, do_sample ? temperature : 1.f, seed,
                          offset, w, w.probes, head->d.cluster_base, nullptr,
                          reinterpret_cast<long long *>(best), s);
  fh::Stage2Args a = stage2_args(head->d, hidden, rows);
  a.probes = w.probes;
  a.probe_stride = head->d.n_probes;
  a.P = head->d.n_probes;
  a.packed = w.packed;
  a.counter = w.counter;
  a.out_signed = reinterpret_cast<long long *>(best);
  a.temperature = do_sample ? temperature : 1.f;
  a.rng = rng_key(seed, offset);
  a.wait_prior = 1;
  const int items = rows * (a.P + a.n_special);
  if (do_sample)
    FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kSample>(head->d.weight_dtype, a, items, s, true)),
                    "stage-2 launch");
  else
    FH_CHECK_LAUNCH((launch_stage2<int32_t, fh::kGreedy>(head->d.weight_dtype, a, items, s, true)),
                    "stage-2 launch");
  return FH_OK;
}

FH_API int fh_tp_finalize(const int64_t *best, int rows, int64_t *out_ids, fh_stream_t stream) {
  if (rows < 0) return fail(FH_ERR_INVALID_ARGUMENT, "rows < 0");
  if (rows == 0) return FH_OK;
  if (!best || !out_ids) return fail(FH_ERR_INVALID_ARGUMENT, "null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  FH_CHECK_LAUNCH(launch(fh::k_signed_to_ids, dim3((rows + 255) / 256), dim3(256), 0, s, false,
                         reinterpret_cast<const long long *>(best), rows, out_ids),
                  "finalize launch");
  return FH_OK;
}

}  // extern "C"
