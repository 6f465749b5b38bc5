// One-kernel FlashHead decode step for a few hidden rows (R <= 4).
//
// A persistent cooperative grid of one 512-thread CTA per SM runs the whole
// step with one grid-wide barrier:
//
//  1. stage 1   CTA b streams its contiguous slice of centroid rows
//               [b*K/G, (b+1)*K/G) through a 6-slot ring of shared-memory
//               buffers filled by bulk asynchronous copies (TMA engine,
//               completion on mbarriers) and scores them against the R hidden
//               rows held in registers. Each score's key goes into global
//               two-level histograms (256 coarse x 256 fine bins: bf16
//               resolution).
//  2. barrier   one arrive counter, bounded spin (a timeout sets an error bit
//               and the kernel still runs to completion).
//  3. select    one warp per hidden row finds, from two 1 KB histogram reads,
//               the bf16 bucket that holds the p-th largest score. Each CTA
//               keeps the clusters it scored whose key lies above that bucket;
//               keys inside the bucket (a handful) are published to a small
//               tie list, and only the CTAs owning such keys wait for the
//               bucket's count (known from the histogram) to be reached, then
//               rank their keys exactly (largest score, then smallest id).
//  4. stage 2   every CTA streams the w_perm rows and vocab ids of its own
//               selected clusters (and, for CTA r, row r's special tokens)
//               through four 32 KB slots, scoring them and keeping the best
//               packed (logit or Gumbel key, vocab id) word per row; words
//               meet in a 64-bit atomicMax and the last CTA to finish
//               publishes the ids.
//
// Histograms and tie lists alternate between two buffers by a call epoch;
// each call zeroes the buffers of the next call and the last CTA resets the
// counters, so a workspace zero-filled once stays consistent.
#pragma once

#include "fh_kernels.cuh"

namespace fh {

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kS1Slots = 6;
constexpr int kS1SlotBytes = 24 * 1024;
constexpr int kS3Slots = 4;
constexpr int kS3SlotBytes = 32 * 1024;
constexpr int kFChunkRows = 16;  // max centroid rows per stage-1 chunk
constexpr int kS3MaxRows = 32;   // max w_perm rows per stage-2 chunk
constexpr int kFBins = 512;
constexpr int kFCand = 256;
constexpr int kFMaxRows = 4;
constexpr int kFMaxProbes = 4096;
constexpr int kFMaxSpecial = 256;
constexpr int kTieCap = 1024;
constexpr int kWorkCap = 1024;  // stage-2 items of one CTA (own clusters + specials)

// State words at the start of the workspace (uint32 index).
constexpr int kSyncArrive = 1;
constexpr int kSyncDone = 2;
constexpr int kSyncError = 3;
constexpr int kSyncEpoch = 4;
constexpr int kSyncTieCount = 8;  // [8 + r]

constexpr int kHistCoarse = 256;
constexpr int kHistWords = kHistCoarse + 65536;
// Per-epoch buffers (two of each).
constexpr size_t kHistBufBytes = (size_t)kFMaxRows * kHistWords * sizeof(uint32_t);
constexpr size_t kTieBufBytes = (size_t)kFMaxRows * kTieCap * sizeof(unsigned long long);
constexpr size_t kEpochBufBytes = kHistBufBytes + kTieBufBytes;
constexpr size_t kHistBytes = 2 * kEpochBufBytes;  // workspace bytes of all epoch buffers

constexpr uint32_t kErrBarrierTimeout = 1u;
constexpr uint32_t kErrCopyTimeout = 2u;
constexpr uint32_t kErrTieTimeout = 4u;

// Stage-2 work item: bit 30 special token, bits 28-29 hidden row, bits 0-23
// cluster id (or special-token index).
constexpr uint32_t kItemSpecial = 0x40000000u;

struct FusedArgs {
  const void *hidden;  // [R, D]
  int rows;
  int D;
  const void *cw;      // stage-1 matrix [K, D] (WT)
  const float *cscale; // [K] or null
  int K;
  const void *w_perm;  // [K * cap, D] (HT)
  const int32_t *vocab_map;
  int cap;
  int p;
  const int32_t *special_slots;
  int n_special;
  int do_sample;
  float temperature;
  RngKey rng;
  float *scores;       // [R, K] global scratch (tie fallback)
  uint32_t *sync;      // workspace state words
  unsigned char *epoch_bufs;   // 2 x (histograms, tie lists)
  unsigned long long *packed;  // [R]
  int64_t *out_ids;    // [R]
  uint32_t barrier_polls;      // grid-barrier / tie-list poll limit
  uint32_t copy_polls;         // mbarrier poll limit
  int extra_arrivals;          // >0 only in the timeout test: wait for more CTAs than exist
};

struct S3Desc {
  int src;   // first w_perm row; -1 invalid (empty chunk); -2 end of work
  int n;     // rows
  int row;   // hidden row
  int vid_in_smem;
};

struct RowThreshold {
  uint32_t prefix;  // 16-bit key prefix of the bucket holding the p-th score
  int need;         // keys of that bucket to select
  int cnt;          // keys in that bucket
};

struct FusedSmem {
  uint64_t mbar1[kS1Slots];
  uint64_t mbar3[kS3Slots];
  float part1[2][kFChunkRows][16][kFMaxRows];
  float part3[kS3Slots][kS3MaxRows][16];
  float local[kFMaxRows][128];
  float scale[128];
  uint32_t coarse[kFMaxRows * kHistCoarse];
  __align__(16) int vid[kS3Slots][kS3MaxRows];
  S3Desc desc[kS3Slots];
  RowThreshold thr[kFMaxRows];
  unsigned long long best[kFMaxRows];
  unsigned long long tiek[kTieCap];
  uint32_t work[kWorkCap];
  unsigned long long mytie[64];  // this CTA's keys in a threshold bucket
  int mytie_row[64];
  int n_work, n_mytie;
  // generic refinement select (tie-list overflow fallback)
  uint32_t hist[kFBins];
  unsigned long long cand[kFCand];
  int scan[33];
  int s_bstar, s_above, s_cnt, s_ncand;
  unsigned long long s_T, s_kmin, s_kmax;
  uint32_t s_err;
};

constexpr size_t kFRingBytes = (size_t)kS1Slots * kS1SlotBytes > (size_t)kS3Slots * kS3SlotBytes
                                   ? (size_t)kS1Slots * kS1SlotBytes
                                   : (size_t)kS3Slots * kS3SlotBytes;
constexpr size_t kFSmemBytes = kFRingBytes + sizeof(FusedSmem);

template <typename T>
__device__ __forceinline__ void vec_to_float(const uint4 &v, float *f);
template <>
__device__ __forceinline__ void vec_to_float<__nv_bfloat16>(const uint4 &v, float *f) {
  Vec<__nv_bfloat16>::to_float(v, f);
}
template <>
__device__ __forceinline__ void vec_to_float<__half>(const uint4 &v, float *f) {
  Vec<__half>::to_float(v, f);
}
template <>
__device__ __forceinline__ void vec_to_float<__nv_fp8_e4m3>(const uint4 &v, float *f) {
  Vec<__nv_fp8_e4m3>::to_float(v, f);
}

// ---------------------------------------------------------------------------
// Block-wide top-p selection over K scores in shared memory (512 threads).
// Same rule as k_select: the p largest (score, -id) keys; output ascending ids.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int fsel_bin_value(float s, float vmin, float scale) {
  const float f = (s - vmin) * scale;
  const int b = f >= (float)(kFBins - 1) ? kFBins - 1 : (int)f;
  return b < 0 ? 0 : b;
}

__device__ void fused_select(const float *sc, int K, int p, float vmin, float vmax, int *out,
                             FusedSmem &S) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float vscale = (float)kFBins / (vmax - vmin);
  const bool value_ok = vmax > vmin && isfinite(vscale) && vscale > 0.f;
  auto key_of = [&](int i) { return pack(sanitize(sc[i]), (uint32_t)i); };

  unsigned long long alo = 0ull, ahi = ~0ull, T = 0ull;
  int need = p;
  for (int level = 0; level < kSelMaxLevels; ++level) {
    const bool vm = value_ok && level == 0;
    const unsigned long long range = ahi - alo;
    const int shift = range == 0ull ? 0 : max(0, 64 - __clzll((long long)range) - 9);
    for (int i = tid; i < kFBins; i += kFThreads) S.hist[i] = 0u;
    __syncthreads();
    for (int i = tid; i < K; i += kFThreads) {
      const unsigned long long k = key_of(i);
      if (k < alo || k > ahi) continue;
      const int b = vm ? fsel_bin_value(unmono((uint32_t)(k >> 32)), vmin, vscale)
                       : (int)((k - alo) >> shift);
      atomicAdd(&S.hist[b], 1u);
    }
    __syncthreads();
    const int mybin = kFBins - 1 - tid;  // thread t owns bin 511 - t (highest first)
    const int c = (int)S.hist[mybin];
    int total;
    const int before = block_exclusive_scan(c, S.scan, &total);
    if (before < need && need <= before + c) {
      S.s_bstar = mybin;
      S.s_above = before;
      S.s_cnt = c;
    }
    __syncthreads();
    const int bstar = S.s_bstar, cnt = S.s_cnt;
    need -= S.s_above;
    unsigned long long kmin = ~0ull, kmax = 0ull;
    for (int i = tid; i < K; i += kFThreads) {
      const unsigned long long k = key_of(i);
      if (k < alo || k > ahi) continue;
      const int b = vm ? fsel_bin_value(unmono((uint32_t)(k >> 32)), vmin, vscale)
                       : (int)((k - alo) >> shift);
      if (b == bstar) {
        kmin = k < kmin ? k : kmin;
        kmax = k > kmax ? k : kmax;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long x = __shfl_xor_sync(0xFFFFFFFFu, kmin, o);
      const unsigned long long y = __shfl_xor_sync(0xFFFFFFFFu, kmax, o);
      kmin = x < kmin ? x : kmin;
      kmax = y > kmax ? y : kmax;
    }
    if (tid == 0) {
      S.s_kmin = ~0ull;
      S.s_kmax = 0ull;
      S.s_ncand = 0;
    }
    __syncthreads();
    if (lane == 0) {
      atomicMin(&S.s_kmin, kmin);
      atomicMax(&S.s_kmax, kmax);
    }
    __syncthreads();
    alo = S.s_kmin;
    ahi = S.s_kmax;
    if (cnt == need) {
      T = alo;
      break;
    }
    if (cnt <= kFCand) {
      for (int i = tid; i < K; i += kFThreads) {
        const unsigned long long k = key_of(i);
        if (k >= alo && k <= ahi) {
          const int pos = atomicAdd(&S.s_ncand, 1);
          if (pos < kFCand) S.cand[pos] = k;
        }
      }
      __syncthreads();
      const int nc = min(cnt, kFCand);
      if (tid < nc) {
        const unsigned long long mine = S.cand[tid];
        int rank = 0;
        for (int j = 0; j < nc; ++j) rank += S.cand[j] > mine;
        if (rank == need - 1) S.s_T = mine;
      }
      __syncthreads();
      T = S.s_T;
      break;
    }
    __syncthreads();
    (void)warp;
  }
  // Compaction in id order.
  block_ordered_compact(
      K, [&](int i) { return key_of(i) >= T; },
      [&](int pos, int i) {
        if (pos < p) out[pos] = i;
      },
      S.scan);
}


#ifdef FH_TRACE
// Profiling builds only: per-CTA %globaltimer stamps at phase boundaries.
__device__ unsigned long long *g_fh_trace;
__device__ __forceinline__ void trace_stamp(int phase) {
  if (threadIdx.x == 0 && g_fh_trace) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_fh_trace[blockIdx.x * 16 + phase] = t;
  }
}
#define FH_STAMP(p) trace_stamp(p)
// clock64 accumulators (thread 0): tick() returns cycles since the last tick
#define FH_TICK_DECL long long fh_t0 = clock64(); long long fh_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#define FH_TICK(k) do { const long long _t = clock64(); fh_acc[k] += _t - fh_t0; fh_t0 = _t; } while (0)
#define FH_TICK_FLUSH() do { if (threadIdx.x == 0 && g_fh_trace) for (int _k = 0; _k < 8; ++_k) g_fh_trace[gridDim.x * 16 + blockIdx.x * 8 + _k] = fh_acc[_k]; } while (0)
#else
#define FH_STAMP(p) ((void)0)
#define FH_TICK_DECL
#define FH_TICK(k) ((void)0)
#define FH_TICK_FLUSH() ((void)0)
#endif

__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Warp-level search of a 256-bin histogram (highest bin first) for the bin
// holding the need-th largest key: returns the bin, the count above it and
// the bin's count (all lanes).
__device__ __forceinline__ void warp_find_bin(const uint32_t *bins, int need, int &bin,
                                              int &above, int &cnt) {
  const int lane = threadIdx.x & 31;
  // lane l owns bins 255-8l .. 248-8l (descending)
  const uint4 lo = __ldcg(reinterpret_cast<const uint4 *>(bins + 248 - 8 * lane));
  const uint4 hi = __ldcg(reinterpret_cast<const uint4 *>(bins + 252 - 8 * lane));
  const uint32_t c[8] = {hi.w, hi.z, hi.y, hi.x, lo.w, lo.z, lo.y, lo.x};
  int mine = 0;
#pragma unroll
  for (int u = 0; u < 8; ++u) mine += (int)c[u];
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += t;
  }
  const int before = incl - mine;
  const unsigned m = __ballot_sync(0xFFFFFFFFu, before < need && need <= incl);
  int b = 255, ab = 0, cn = 0;
  if (m) {
    const int src = __ffs(m) - 1;
    if (lane == src) {
      int cum = before;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (cum < need && need <= cum + (int)c[u]) {
          b = 255 - 8 * lane - u;
          ab = cum;
          cn = (int)c[u];
        }
        cum += (int)c[u];
      }
    }
    b = __shfl_sync(0xFFFFFFFFu, b, src);
    ab = __shfl_sync(0xFFFFFFFFu, ab, src);
    cn = __shfl_sync(0xFFFFFFFFu, cn, src);
  }
  bin = b;
  above = ab;
  cnt = cn;
}

template <typename HT, typename WT, int R>
__global__ void __launch_bounds__(kFThreads, 1) k_fused_step(FusedArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char *ring = smem;
  FusedSmem &S = *reinterpret_cast<FusedSmem *>(smem + kFRingBytes);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kS1Slots; ++s) mbar_init(&S.mbar1[s], 1);
    for (int s = 0; s < kS3Slots; ++s) mbar_init(&S.mbar3[s], 1);
    fence_mbar_init();
    S.s_err = 0u;
    S.n_work = 0;
    S.n_mytie = 0;
  }
  if (tid < kFMaxRows) S.best[tid] = 0ull;
  for (int i = tid; i < kFMaxRows * kHistCoarse; i += kFThreads) S.coarse[i] = 0u;
  __syncthreads();
  FH_STAMP(0);

  const uint32_t epoch = __ldcg(&a.sync[kSyncEpoch]);
  unsigned char *buf_cur = a.epoch_bufs + (size_t)(epoch & 1u) * kEpochBufBytes;
  unsigned char *buf_nxt = a.epoch_bufs + (size_t)((epoch + 1u) & 1u) * kEpochBufBytes;
  uint32_t *hist_cur = reinterpret_cast<uint32_t *>(buf_cur);
  unsigned long long *ties = reinterpret_cast<unsigned long long *>(buf_cur + kHistBufBytes);

  // ------------------------------------------------------------------ stage 1
  const int c0 = (int)((long long)b * a.K / G), c1 = (int)((long long)(b + 1) * a.K / G);
  const int nc = c1 - c0;
  const int row1 = a.D * (int)sizeof(WT);
  const int rpc1 = max(1, min(kFChunkRows, kS1SlotBytes / row1));
  const int n1 = (nc + rpc1 - 1) / rpc1;
  const char *wsrc = reinterpret_cast<const char *>(a.cw) + (size_t)c0 * row1;
  auto issue1 = [&](int i) {
    const int s = i % kS1Slots;
    const int rows = min(rpc1, nc - i * rpc1);
    const uint32_t bytes = (uint32_t)(rows * row1);
    fence_proxy_async_smem();
    mbar_expect_tx(&S.mbar1[s], bytes);
    bulk_g2s(ring + (size_t)s * kS1SlotBytes, wsrc + (size_t)i * rpc1 * row1, bytes, &S.mbar1[s]);
  };
  if (tid == 0)
    for (int i = 0; i < min(kS1Slots, n1); ++i) issue1(i);
  if (tid < nc) S.scale[tid] = a.cscale ? a.cscale[c0 + tid] : 1.f;

  constexpr int VE1 = Vec<WT>::kElems;
  const int NV1 = row1 / 16, Q1 = NV1 / 32, RG1 = kFWarps / Q1;
  const int g1 = warp / Q1, q1 = warp % Q1, col1 = q1 * 32 + lane;
  float h1[R][VE1];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const char *hp = reinterpret_cast<const char *>(a.hidden) + (size_t)r * a.D * sizeof(HT) +
                     (size_t)col1 * VE1 * sizeof(HT);
#pragma unroll
    for (int v = 0; v < VE1 / 8; ++v) {
      const uint4 x = (r < a.rows && g1 < RG1) ? ldg_keep(hp + v * 16) : make_uint4(0, 0, 0, 0);
      vec_to_float<HT>(x, &h1[r][v * 8]);
    }
  }

  FH_TICK_DECL
  for (int i = 0; i < n1; ++i) {
    const int s = i % kS1Slots;
    const int rows = min(rpc1, nc - i * rpc1);
    FH_TICK(7);
    if (!mbar_wait(&S.mbar1[s], (i / kS1Slots) & 1, a.copy_polls) && lane == 0)
      atomicOr(&S.s_err, kErrCopyTimeout);
    if (i == 0) FH_STAMP(13);
    if (i == n1 - 1) FH_STAMP(14);
    FH_TICK(0);
    if (g1 < RG1) {
      const unsigned char *base = ring + (size_t)s * kS1SlotBytes + (size_t)col1 * 16;
      for (int r = g1; r < rows; r += RG1) {
        float w[VE1];
        vec_to_float<WT>(lds128(base + (size_t)r * row1), w);
#pragma unroll
        for (int hr = 0; hr < R; ++hr) {
          float acc = 0.f;
#pragma unroll
          for (int e = 0; e < VE1; ++e) acc = fmaf(w[e], h1[hr][e], acc);
          acc = warp_sum(acc);
          if (lane == 0) S.part1[i & 1][r][q1][hr] = acc;
        }
      }
    }
    FH_TICK(1);
    __syncthreads();
    FH_TICK(2);
    if (tid < rows * R) {
      const int r = tid / R, hr = tid - (tid / R) * R;
      if (hr < a.rows) {
        float acc = 0.f;
        for (int q = 0; q < Q1; ++q) acc += S.part1[i & 1][r][q][hr];
        const int k = c0 + i * rpc1 + r;
        float sc = acc * S.scale[k - c0];
        if (a.do_sample)
          sc = sc / a.temperature + gumbel(a.rng, kStageClusters, (uint32_t)hr, (uint32_t)k);
        S.local[hr][k - c0] = sc;
        a.scores[(size_t)hr * a.K + k] = sc;
        const uint32_t key = mono(sanitize(sc));
        atomicAdd(&hist_cur[(size_t)hr * kHistWords + kHistCoarse + (key >> 16)], 1u);
        atomicAdd(&S.coarse[hr * kHistCoarse + (key >> 24)], 1u);
      }
    }
    if (tid == 0 && i + kS1Slots < n1) issue1(i + kS1Slots);
    FH_TICK(3);
  }
  __syncthreads();
  FH_STAMP(7);
  // Speculative L2 prefetch of stage-2 rows. HBM would sit idle through the
  // barrier and the threshold search, so each CTA pulls the w_perm rows of
  // its clusters that are likely to be selected: score above its own
  // mean + z * std, where z is the normal quantile of the selection rate
  // minus a margin. A wrong guess only costs bandwidth that was idle.
  if (!a.do_sample && warp < a.rows && nc > 1) {
    float sum = 0.f, sq = 0.f;
    for (int i = lane; i < nc; i += 32) {
      const float v = S.local[warp][i];
      if (isfinite(v)) {
        sum += v;
        sq += v * v;
      }
    }
    sum = warp_sum(sum);
    sq = warp_sum(sq);
    const float mean = sum / nc;
    const float sd = sqrtf(fmaxf(sq / nc - mean * mean, 0.f));
    const float frac = fminf(0.5f, (float)a.p / (float)a.K);
    const float z = -normcdfinvf(frac) - 0.25f;
    const float t_est = mean + z * sd;
    const size_t cluster_bytes = (size_t)a.cap * a.D * sizeof(HT);
    for (int i = lane; i < nc; i += 32)
      if (S.local[warp][i] > t_est && cluster_bytes % 16 == 0)
        bulk_prefetch_l2(reinterpret_cast<const char *>(a.w_perm) + (size_t)(c0 + i) * cluster_bytes,
                         (uint32_t)cluster_bytes);
  }
  for (int i = tid; i < a.rows * kHistCoarse; i += kFThreads) {
    const uint32_t c = S.coarse[i];
    if (c) atomicAdd(&hist_cur[(size_t)(i / kHistCoarse) * kHistWords + (i % kHistCoarse)], c);
  }
  __syncthreads();
  FH_STAMP(1);

  // ------------------------------------------------------------- grid barrier
  if (tid == 0) {
    __threadfence();
    FH_STAMP(8);
    atomicAdd(&a.sync[kSyncArrive], 1u);
    const uint32_t target = (uint32_t)(G + a.extra_arrivals);
    uint32_t polls = 0;
    while (ld_acquire_gpu(&a.sync[kSyncArrive]) < target) {
      if (++polls >= a.barrier_polls) {
        atomicOr(&S.s_err, kErrBarrierTimeout);
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
  FH_STAMP(2);

  // --------------------------------------------- thresholds: warp r, row r
  if (warp < a.rows) {
    const uint32_t *h = hist_cur + (size_t)warp * kHistWords;
    int cb, above1, cnt1, fb, above2, cnt2;
    warp_find_bin(h, a.p, cb, above1, cnt1);
    warp_find_bin(h + kHistCoarse + cb * 256, a.p - above1, fb, above2, cnt2);
    if (lane == 0) {
      S.thr[warp].prefix = (uint32_t)(cb * 256 + fb);
      S.thr[warp].need = a.p - above1 - above2;
      S.thr[warp].cnt = cnt2;
    }
  }
  __syncthreads();
  FH_STAMP(9);
  // Zero this CTA's share of the buffers the next call will use.
  {
    const size_t n4 = kEpochBufBytes / 16;
    uint4 *z = reinterpret_cast<uint4 *>(buf_nxt);
    for (size_t i = (size_t)b * n4 / G + tid; i < (size_t)(b + 1) * n4 / G; i += kFThreads)
      z[i] = make_uint4(0, 0, 0, 0);
  }

  // ------------- own clusters above the bucket -> work list; bucket -> ties
  for (int i = tid; i < a.rows * nc; i += kFThreads) {
    const int hr = i / nc, k = i - (i / nc) * nc;
    const float v = sanitize(S.local[hr][k]);
    const uint32_t pre = mono(v) >> 16;
    const uint32_t P = S.thr[hr].prefix;
    if (pre > P) {
      const int w = atomicAdd(&S.n_work, 1);
      if (w < kWorkCap) S.work[w] = ((uint32_t)hr << 28) | (uint32_t)(c0 + k);
    } else if (pre == P) {
      const unsigned long long key = pack(v, (uint32_t)(c0 + k));
      const uint32_t t = atomicAdd(&a.sync[kSyncTieCount + hr], 1u);
      if (t < (uint32_t)kTieCap) ties[(size_t)hr * kTieCap + t] = key;
      const int m = atomicAdd(&S.n_mytie, 1);
      if (m < 64) {
        S.mytie[m] = key;
        S.mytie_row[m] = hr;
      }
    }
  }
  // special tokens of row b are scored by CTA b
  if (b < a.rows)
    for (int t = tid; t < a.n_special; t += kFThreads) {
      const int w = atomicAdd(&S.n_work, 1);
      if (w < kWorkCap) S.work[w] = kItemSpecial | ((uint32_t)b << 28) | (uint32_t)t;
    }
  __syncthreads();
  FH_STAMP(10);

  // ------------------------------------------------------------------ stage 2
  const int row3 = a.D * (int)sizeof(HT);
  int rpc3 = min(min(a.cap, kS3MaxRows), kS3SlotBytes / row3);
  if (rpc3 >= 4) rpc3 &= ~3;  // multiples of 4 rows keep the vocab-id copies 16-byte sized
  rpc3 = max(1, rpc3);
  const int NV3 = row3 / 16, Q3 = NV3 / 32, RG3 = kFWarps / Q3;
  const int g3 = warp / Q3, q3 = warp % Q3, col3 = q3 * 32 + lane;
  float h3[R][8];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint4 x = (r < a.rows && g3 < RG3)
                        ? ldg_keep(reinterpret_cast<const char *>(a.hidden) +
                                   (size_t)r * row3 + (size_t)col3 * 16)
                        : make_uint4(0, 0, 0, 0);
    vec_to_float<HT>(x, h3[r]);
  }
  const char *wp = reinterpret_cast<const char *>(a.w_perm);
  // Producer state (thread 0 only): next work item and its next chunk.
  int p_item = 0, p_chunk = 0;
  auto produce = [&](int s) {
    S3Desc d;
    d.src = -2;
    d.n = 0;
    d.row = 0;
    d.vid_in_smem = 0;
    const int nw = min(S.n_work, kWorkCap);
    if (p_item < nw) {
      const uint32_t item = S.work[p_item];
      d.row = (int)((item >> 28) & 3u);
      const int payload = (int)(item & 0x00FFFFFFu);
      if (item & kItemSpecial) {
        const int sp = payload < a.n_special ? a.special_slots[payload] : -1;
        d.src = (sp >= 0 && sp < a.K * a.cap) ? sp : -1;
        d.n = 1;
        ++p_item;
      } else {
        const int start = p_chunk * rpc3;
        d.src = payload < a.K ? payload * a.cap + start : -1;
        d.n = min(rpc3, a.cap - start);
        if (start + rpc3 >= a.cap) {
          ++p_item;
          p_chunk = 0;
        } else {
          ++p_chunk;
        }
      }
    }
    S.desc[s] = d;
    fence_proxy_async_smem();
    if (d.src >= 0) {
      const int *vsrc = a.vocab_map + d.src;
      const bool vid_bulk = ((reinterpret_cast<uintptr_t>(vsrc) & 15u) == 0) && (d.n % 4 == 0);
      S.desc[s].vid_in_smem = vid_bulk ? 1 : 0;
      mbar_expect_tx(&S.mbar3[s], (uint32_t)(d.n * row3) + (vid_bulk ? (uint32_t)(d.n * 4) : 0u));
      bulk_g2s(ring + (size_t)s * kS3SlotBytes, wp + (size_t)d.src * row3, (uint32_t)(d.n * row3),
               &S.mbar3[s]);
      if (vid_bulk) bulk_g2s(&S.vid[s][0], vsrc, (uint32_t)(d.n * 4), &S.mbar3[s]);
    } else {
      mbar_expect_tx(&S.mbar3[s], 0u);  // invalid row or end of work: no data
    }
  };
  // Start streaming the certain clusters, then settle this CTA's bucket keys;
  // slots are only marked end-of-work once the work list is final.
  int n_prod = 0;  // thread 0: chunks produced so far (chunk i uses slot i % kS3Slots)
  if (tid == 0)
    while (n_prod < kS3Slots && p_item < min(S.n_work, kWorkCap)) produce(n_prod++ % kS3Slots);
  {
    const int nmt = min(S.n_mytie, 64);
    if (nmt > 0) {
      // wait until every key of the bucket (count from the histogram) is listed
      if (tid == 0) {
        for (int hr = 0; hr < a.rows; ++hr) {
          bool mine = false;
          for (int m = 0; m < nmt; ++m) mine |= S.mytie_row[m] == hr;
          if (!mine) continue;
          const uint32_t want = (uint32_t)min(S.thr[hr].cnt, kTieCap);
          uint32_t polls = 0;
          while (ld_acquire_gpu(&a.sync[kSyncTieCount + hr]) < want) {
            if (++polls >= a.barrier_polls) {
              atomicOr(&S.s_err, kErrTieTimeout);
              break;
            }
          }
        }
        __threadfence();
      }
      __syncthreads();
      for (int m = 0; m < nmt; ++m) {
        const int hr = S.mytie_row[m];
        const int cnt = min(S.thr[hr].cnt, kTieCap);
        const unsigned long long mine = S.mytie[m];
        int rank = 0;
        for (int t = tid; t < cnt; t += kFThreads)
          rank += __ldcg(&ties[(size_t)hr * kTieCap + t]) > mine;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rank += __shfl_xor_sync(0xFFFFFFFFu, rank, o);
        if (lane == 0) S.scan[warp] = rank;
        __syncthreads();
        if (tid == 0) {
          int tot = 0;
          for (int w = 0; w < kFWarps; ++w) tot += S.scan[w];
          if (tot < S.thr[hr].need) {
            const int w = atomicAdd(&S.n_work, 1);
            if (w < kWorkCap) S.work[w] = ((uint32_t)hr << 28) | packed_id(mine);
          }
        }
        __syncthreads();
      }
    }
  }
  FH_STAMP(4);
  __syncthreads();
  if (tid == 0)
    while (n_prod < kS3Slots) produce(n_prod++ % kS3Slots);
  FH_TICK(7);
  for (int c = 0;; ++c) {
    const int s = c % kS3Slots;
    if (!mbar_wait(&S.mbar3[s], (c / kS3Slots) & 1, a.copy_polls) && lane == 0)
      atomicOr(&S.s_err, kErrCopyTimeout);
    FH_TICK(4);
    const S3Desc d = S.desc[s];
    if (c == 0) FH_STAMP(11);
    if (d.src == -2) break;
    if (d.src >= 0 && g3 < RG3) {
      const unsigned char *base = ring + (size_t)s * kS3SlotBytes + (size_t)col3 * 16;
      for (int r = g3; r < d.n; r += RG3) {
        float w[8];
        vec_to_float<HT>(lds128(base + (size_t)r * row3), w);
        float acc = 0.f;
#pragma unroll
        for (int hh = 0; hh < R; ++hh) {
          if (hh == d.row) {
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(w[e], h3[hh][e], acc);
          }
        }
        acc = warp_sum(acc);
        if (lane == 0) S.part3[s][r][q3] = acc;
      }
    }
    FH_TICK(5);
    __syncthreads();
    if (d.src >= 0 && tid < d.n) {
      float acc = 0.f;
      for (int q = 0; q < Q3; ++q) acc += S.part3[s][tid][q];
      const uint32_t vid = (uint32_t)(d.vid_in_smem ? S.vid[s][tid] : a.vocab_map[d.src + tid]);
      float key = acc;
      if (a.do_sample)
        key = acc / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)d.row, vid);
      atomicMax(&S.best[d.row], pack(key, vid));
    }
    __syncthreads();  // slot s and its descriptor are free
    if (tid == 0) produce(n_prod++ % kS3Slots);
    FH_TICK(6);
  }
  FH_TICK_FLUSH();
  __syncthreads();
  FH_STAMP(5);

  // --------------------------------------------------------------- reduction
  if (tid < a.rows && S.best[tid] != 0ull) atomicMax(&a.packed[tid], S.best[tid]);
  if (tid == 0 && S.s_err) atomicOr(&a.sync[kSyncError], S.s_err);
  __syncthreads();
  __shared__ uint32_t s_last;
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&a.sync[kSyncDone], 1u) == (uint32_t)G - 1;
  }
  __syncthreads();
  FH_STAMP(6);
  if (s_last) {
    __threadfence();
    if (tid < a.rows) {
      const unsigned long long wv = atomicExch(&a.packed[tid], 0ull);
      a.out_ids[tid] = wv ? (int64_t)packed_id(wv) : (int64_t)0xFFFFFFFFll;
    }
    if (tid < kFMaxRows) a.sync[kSyncTieCount + tid] = 0u;
    if (tid == 0) {
      a.sync[kSyncArrive] = 0u;
      a.sync[kSyncDone] = 0u;
      a.sync[kSyncEpoch] = epoch + 1u;
    }
  }
}

}  // namespace fh
