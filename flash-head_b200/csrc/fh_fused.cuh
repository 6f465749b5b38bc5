// One-kernel FlashHead decode step for a few hidden rows (R <= 4).
//
// A persistent cooperative grid of one 512-thread CTA per SM runs all three
// stages with a single grid-wide dependency:
//
//  1. stage 1   CTA b streams its contiguous slice of centroid rows
//               [b*K/G, (b+1)*K/G) through a 4-slot ring of shared-memory
//               buffers filled by bulk asynchronous copies (TMA engine,
//               completion on mbarriers) and scores them against the R hidden
//               rows held in registers; scores go to global memory and
//               their keys into global histograms (see 3).
//  2. barrier   one arrive counter, bounded spin (a timeout sets an error
//               bit and the kernel still runs to completion).
//  3. select    stage 1 also built global two-level histograms of the
//               score keys (256 coarse x 256 fine bins = bf16 resolution),
//               so after the barrier every CTA finds the threshold bin from
//               two 1 KB reads, ranks the few keys that share its 16-bit
//               prefix exactly and compacts the selected ids from the
//               L2-resident scores. Redundant selection costs no second
//               grid-wide dependency.
//  4. stage 2   the R * (p * cap + n_special) w_perm rows to score are split
//               evenly across CTAs in (row, probe, slot) order; each CTA
//               streams its contiguous runs through the same ring, packs
//               (logit or Gumbel key, vocab id) words, and reduces them with a
//               64-bit atomicMax. The last CTA to finish publishes the ids and
//               resets the shared state words.
#pragma once

#include "fh_kernels.cuh"

namespace fh {

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kFSlots = 4;
constexpr int kFSlotBytes = 24 * 1024;
constexpr int kFChunkRows = 16;
constexpr int kFBins = 512;
constexpr int kFCand = 256;
constexpr int kFMaxRows = 4;
constexpr int kFMaxProbes = 4096;

// State words at the start of the workspace (uint32 index).
constexpr int kSyncArrive = 1;
constexpr int kSyncDone = 2;
constexpr int kSyncError = 3;
constexpr int kSyncEpoch = 4;

// Two-level key histograms per hidden row: 256 coarse bins (key >> 24) then
// 65536 fine bins (key >> 16, i.e. bf16 resolution). Two buffers alternate
// by call epoch; each call zeroes the buffer the next call will use.
constexpr int kHistCoarse = 256;
constexpr int kHistWords = kHistCoarse + 65536;
constexpr size_t kHistBytes = 2ull * kFMaxRows * kHistWords * sizeof(uint32_t);

constexpr uint32_t kErrBarrierTimeout = 1u;
constexpr uint32_t kErrCopyTimeout = 2u;

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
  float *scores;       // [R, K] global scratch
  uint32_t *sync;      // workspace state words
  uint32_t *hist;      // [2][kFMaxRows][kHistWords] key histograms
  unsigned long long *packed;  // [R]
  int64_t *out_ids;    // [R]
  uint32_t barrier_polls;      // grid-barrier poll limit
  uint32_t copy_polls;         // mbarrier poll limit
  int extra_arrivals;          // >0 only in the timeout test: wait for more CTAs than exist
};

// One stage-2 chunk: up to rpc3 w_perm rows contiguous in memory.
struct S2Chunk {
  int src;   // first w_perm row, -1 for an invalid special slot
  int w;     // first work index
  short n;   // rows
  short hrow;
};
constexpr int kFMaxChunks = 384;

struct FusedSmem {
  uint64_t mbar[kFSlots];
  float part[kFSlots][kFChunkRows][16][kFMaxRows];
  float local[kFMaxRows][128];
  float scale[128];
  uint32_t coarse[kFMaxRows][kHistCoarse];
  uint32_t hist[kFBins];
  unsigned long long cand[kFCand];
  S2Chunk chunks[kFMaxChunks];
  int s_nchunks;
  unsigned long long best[2];
  int scan[33];
  int s_bstar, s_above, s_cnt, s_ncand, s_cb, s_fb;
  unsigned long long s_T, s_kmin, s_kmax;
  uint32_t s_err;
};

constexpr int kFVidCache = 4096;  // vocab ids of a CTA's stage-2 rows, prefetched
constexpr size_t kFRingBytes = (size_t)kFSlots * kFSlotBytes;
constexpr size_t kFSmemBytes =
    kFRingBytes + sizeof(FusedSmem) + 2ull * kFMaxProbes * 4 + (size_t)kFVidCache * 4;

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

// Stage-2 work walk: work index w of row-major (hidden row, probe, slot) items,
// then the special tokens of each hidden row. Returns the w_perm row of w
// (-1 if invalid) and how many following work items are contiguous in w_perm.
struct S2Item {
  int src;
  int run;
  int hrow;
};

__device__ __forceinline__ S2Item s2_item(const FusedArgs &a, const int *probes_sm, int r_lo,
                                          int w, int w_end) {
  const int per_row = a.p * a.cap + a.n_special;
  S2Item it;
  it.hrow = w / per_row;
  const int j = w - it.hrow * per_row;
  if (j < a.p * a.cap) {
    const int pi = j / a.cap, sl = j - pi * a.cap;
    const int cl = probes_sm[(it.hrow - r_lo) * a.p + pi];
    it.src = (cl >= 0 && cl < a.K) ? cl * a.cap + sl : -1;
    it.run = min(a.cap - sl, w_end - w);
  } else {
    const int sp = a.special_slots[j - a.p * a.cap];
    it.src = (sp >= 0 && sp < a.K * a.cap) ? sp : -1;
    it.run = 1;
  }
  return it;
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
#else
#define FH_STAMP(p) ((void)0)
#endif

template <typename HT, typename WT, int R>
__global__ void __launch_bounds__(kFThreads, 1) k_fused_step(FusedArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char *ring = smem;
  FusedSmem &S = *reinterpret_cast<FusedSmem *>(smem + kFRingBytes);
  int *probes_sm = reinterpret_cast<int *>(smem + kFRingBytes + sizeof(FusedSmem));
  int *vid_sm = probes_sm + 2 * kFMaxProbes;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kFSlots; ++s) mbar_init(&S.mbar[s], 1);
    fence_mbar_init();
    S.s_err = 0u;
    S.best[0] = S.best[1] = 0ull;
  }
  __syncthreads();
  FH_STAMP(0);

  // ------------------------------------------------------------------ stage 1
  const int c0 = (int)((long long)b * a.K / G), c1 = (int)((long long)(b + 1) * a.K / G);
  const int nc = c1 - c0;
  const int row1 = a.D * (int)sizeof(WT);
  const int rpc1 = max(1, min(kFChunkRows, kFSlotBytes / row1));
  const int n1 = (nc + rpc1 - 1) / rpc1;
  const char *wsrc = reinterpret_cast<const char *>(a.cw) + (size_t)c0 * row1;
  uint32_t gi = 0;  // running chunk counter over both stages (slot = gi % kFSlots)

  auto issue1 = [&](int i) {
    const int s = i % kFSlots;
    const int rows = min(rpc1, nc - i * rpc1);
    const uint32_t bytes = (uint32_t)(rows * row1);
    fence_proxy_async_smem();
    mbar_expect_tx(&S.mbar[s], bytes);
    bulk_g2s(ring + (size_t)s * kFSlotBytes, wsrc + (size_t)i * rpc1 * row1, bytes, &S.mbar[s]);
  };
  if (tid == 0)
    for (int i = 0; i < min(kFSlots, n1); ++i) issue1(i);
  if (tid < nc) S.scale[tid] = a.cscale ? a.cscale[c0 + tid] : 1.f;

  constexpr int VE1 = Vec<WT>::kElems;
  const int NV1 = row1 / 16, Q1 = NV1 / 32, RG1 = kFWarps / Q1;
  const int g1 = warp / Q1, q1 = warp % Q1, col1 = q1 * 32 + lane;
  float h1[R][VE1];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    // VE1 elements of hidden row r at column col1 (VE1 * 2 bytes)
    const char *hp = reinterpret_cast<const char *>(a.hidden) + (size_t)r * a.D * sizeof(HT) +
                     (size_t)col1 * VE1 * sizeof(HT);
#pragma unroll
    for (int v = 0; v < VE1 / 8; ++v) {
      const uint4 x = (r < a.rows && g1 < RG1) ? ldg_keep(hp + v * 16) : make_uint4(0, 0, 0, 0);
      vec_to_float<HT>(x, &h1[r][v * 8]);
    }
  }

  for (int i = 0; i < n1; ++i, ++gi) {
    const int s = gi % kFSlots;
    const int rows = min(rpc1, nc - i * rpc1);
    if (!mbar_wait(&S.mbar[s], (gi / kFSlots) & 1, a.copy_polls) && lane == 0)
      atomicOr(&S.s_err, kErrCopyTimeout);
    if (g1 < RG1) {
      const unsigned char *base = ring + (size_t)s * kFSlotBytes + (size_t)col1 * 16;
      for (int r = g1; r < rows; r += RG1) {
        float w[VE1];
        vec_to_float<WT>(lds128(base + (size_t)r * row1), w);
#pragma unroll
        for (int hr = 0; hr < R; ++hr) {
          float acc = 0.f;
#pragma unroll
          for (int e = 0; e < VE1; ++e) acc = fmaf(w[e], h1[hr][e], acc);
          acc = warp_sum(acc);
          if (lane == 0) S.part[s][r][q1][hr] = acc;
        }
      }
    }
    __syncthreads();
    if (tid < rows * R) {
      const int r = tid / R, hr = tid - (tid / R) * R;
      float acc = 0.f;
      for (int q = 0; q < Q1; ++q) acc += S.part[s][r][q][hr];
      const int k = c0 + i * rpc1 + r;
      float sc = acc * S.scale[k - c0];
      if (a.do_sample)
        sc = sc / a.temperature + gumbel(a.rng, kStageClusters, (uint32_t)hr, (uint32_t)k);
      if (hr < a.rows) {
        S.local[hr][k - c0] = sc;
        a.scores[(size_t)hr * a.K + k] = sc;
      }
    }
    if (tid == 0 && i + kFSlots < n1) issue1(i + kFSlots);
  }
  __syncthreads();
  FH_STAMP(1);
  // Publish this CTA's keys to the global two-level histograms of its rows:
  // fine bins directly, coarse bins aggregated in shared memory first (they
  // are few and hot).
  const uint32_t epoch = __ldcg(&a.sync[kSyncEpoch]);
  uint32_t *hist_cur = a.hist + (size_t)(epoch & 1u) * kFMaxRows * kHistWords;
  uint32_t *hist_next = a.hist + (size_t)((epoch + 1u) & 1u) * kFMaxRows * kHistWords;
  for (int i = tid; i < kFMaxRows * kHistCoarse; i += kFThreads) (&S.coarse[0][0])[i] = 0u;
  __syncthreads();
  for (int i = tid; i < a.rows * nc; i += kFThreads) {
    const int hr = i / nc, k = i - (i / nc) * nc;
    const uint32_t key = mono(sanitize(S.local[hr][k]));
    atomicAdd(&hist_cur[(size_t)hr * kHistWords + kHistCoarse + (key >> 16)], 1u);
    atomicAdd(&S.coarse[hr][key >> 24], 1u);
  }
  __syncthreads();
  for (int i = tid; i < a.rows * kHistCoarse; i += kFThreads) {
    const uint32_t c = (&S.coarse[0][0])[i];
    if (c) atomicAdd(&hist_cur[(size_t)(i / kHistCoarse) * kHistWords + (i % kHistCoarse)], c);
  }

  // ------------------------------------------------------------- grid barrier
  __syncthreads();
  FH_STAMP(2);
  if (tid == 0) {
    __threadfence();
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
  FH_STAMP(3);

  // ------------------------------------------------------------------- select
  const int per_row = a.p * a.cap + a.n_special;
  const int W = per_row * a.rows;
  const int w0 = (int)((long long)W * b / G), w1 = (int)((long long)W * (b + 1) / G);
  const int r_lo = w0 / per_row;
  const int r_hi = w1 > w0 ? (w1 - 1) / per_row : r_lo - 1;
  float *sc_sm = reinterpret_cast<float *>(ring);
  for (int hr = r_lo; hr <= r_hi; ++hr) {
    const uint32_t *h1g = hist_cur + (size_t)hr * kHistWords;
    // All loads of this row's scores (and its coarse histogram) in flight at once.
    const uint32_t coarse_v = tid < kHistCoarse ? __ldcg(&h1g[kHistCoarse - 1 - tid]) : 0u;
    {
      const float *src = a.scores + (size_t)hr * a.K;
      for (int base = 0; base < a.K; base += kFThreads * 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = base + u * kFThreads + tid;
          v[u] = i < a.K ? __ldcg(&src[i]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = base + u * kFThreads + tid;
          if (i < a.K) sc_sm[i] = v[u];
        }
      }
    }
    if (hr == r_lo) FH_STAMP(7);
    // Defaults keep every index in range even when the histogram is
    // incomplete (a timed-out barrier); the scan's first barrier publishes them.
    if (tid == 0) {
      S.s_cb = 0;
      S.s_fb = 0;
      S.s_cnt = 0;
      S.s_above = 0;
      S.s_T = ~0ull;
    }
    // coarse level: thread t owns bin 255 - t (highest first)
    int need = a.p;
    {
      const int c = (int)coarse_v;
      int total;
      const int before = block_exclusive_scan(c, S.scan, &total);
      if (before < need && need <= before + c) {
        S.s_cb = kHistCoarse - 1 - tid;
        S.s_above = before;
      }
      __syncthreads();
    }
    need -= S.s_above;
    const int cb = min(max(S.s_cb, 0), kHistCoarse - 1);
    {
      const int f = tid < 256 ? (int)__ldcg(&h1g[kHistCoarse + cb * 256 + 255 - tid]) : 0;
      int total;
      const int before = block_exclusive_scan(f, S.scan, &total);
      if (before < need && need <= before + f) {
        S.s_fb = 255 - tid;
        S.s_above = before;
        S.s_cnt = f;
      }
      if (tid == 0) S.s_ncand = 0;
      __syncthreads();
    }
    need -= S.s_above;
    if (hr == r_lo) FH_STAMP(8);
    const uint32_t prefix = (uint32_t)(cb * 256 + (S.s_fb & 255));
    const int cnt = S.s_cnt;
    int *probes_out = probes_sm + (hr - r_lo) * a.p;
    if (cnt <= kFCand) {
      // exact ranking of the keys that share the threshold's 16-bit prefix
      for (int i = tid; i < a.K; i += kFThreads) {
        const float v = sanitize(sc_sm[i]);
        if ((mono(v) >> 16) == prefix) {
          const int pos = atomicAdd(&S.s_ncand, 1);
          if (pos < kFCand) S.cand[pos] = pack(v, (uint32_t)i);
        }
      }
      __syncthreads();
      const int nc2 = min(cnt, kFCand);
      if (tid < nc2) {
        const unsigned long long mine = S.cand[tid];
        int rank = 0;
        for (int j = 0; j < nc2; ++j) rank += S.cand[j] > mine;
        if (rank == need - 1) S.s_T = mine;
      }
      __syncthreads();
      if (hr == r_lo) FH_STAMP(9);
      const unsigned long long T = S.s_T;
      block_ordered_compact(
          a.K, [&](int i) { return pack(sanitize(sc_sm[i]), (uint32_t)i) >= T; },
          [&](int pos, int i) {
            if (pos < a.p) probes_out[pos] = i;
          },
          S.scan);
    } else {
      // many keys share the threshold's bf16 prefix: full refinement
      fused_select(sc_sm, a.K, a.p, -INFINITY, -INFINITY, probes_out, S);
    }
  }
  FH_STAMP(10);
  // Zero the histogram buffer the next call will use (this call never reads it).
  {
    const size_t n4 = (size_t)kFMaxRows * kHistWords / 4;
    uint4 *z = reinterpret_cast<uint4 *>(hist_next);
    for (size_t i = (size_t)b * n4 / G + tid; i < (size_t)(b + 1) * n4 / G; i += kFThreads)
      z[i] = make_uint4(0, 0, 0, 0);
  }

  FH_STAMP(4);
  // ------------------------------------------------------------------ stage 2
  const int row3 = a.D * (int)sizeof(HT);
  const int rpc3 = max(1, min(kFChunkRows, kFSlotBytes / row3));
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
  FH_STAMP(11);
  // Chunk table of this CTA's stage-2 range (thread 0, 32-bit math).
  if (tid == 0) {
    int w = w0, nch = 0;
    while (w < w1 && nch < kFMaxChunks) {
      const S2Item it = s2_item(a, probes_sm, r_lo, w, w1);
      const int n = min(it.run, rpc3);
      S.chunks[nch].src = it.src;
      S.chunks[nch].w = w;
      S.chunks[nch].n = (short)n;
      S.chunks[nch].hrow = (short)it.hrow;
      ++nch;
      w += n;
    }
    S.s_nchunks = (w < w1) ? -1 : nch;  // -1: range needs more chunks than the table holds
  }
  // Vocab ids of this CTA's stage-2 rows, fetched once (off the per-chunk path).
  const int n_vid = min(kFVidCache, w1 - w0);
  for (int t = tid; t < n_vid; t += kFThreads) {
    const S2Item it = s2_item(a, probes_sm, r_lo, w0 + t, w0 + t + 1);
    vid_sm[t] = it.src >= 0 ? a.vocab_map[it.src] : 0;
  }
  __syncthreads();  // ring free: selection done by every thread; chunk table ready
  const int nch = S.s_nchunks;
  const char *wp = reinterpret_cast<const char *>(a.w_perm);
  auto chunk_at = [&](int c, int &w_walk) -> S2Chunk {
    if (nch >= 0) return S.chunks[c];
    const S2Item it = s2_item(a, probes_sm, r_lo, w_walk, w1);  // overflow fallback
    S2Chunk ch;
    ch.src = it.src;
    ch.w = w_walk;
    ch.n = (short)min(it.run, rpc3);
    ch.hrow = (short)it.hrow;
    w_walk += ch.n;
    return ch;
  };
  int w_issue = w0, w_cons = w0, c_issue = 0;
  auto issue3 = [&](uint32_t gidx) {
    const S2Chunk ch = chunk_at(c_issue++, w_issue);
    const int s = gidx % kFSlots;
    fence_proxy_async_smem();
    if (ch.src >= 0) {
      mbar_expect_tx(&S.mbar[s], (uint32_t)(ch.n * row3));
      bulk_g2s(ring + (size_t)s * kFSlotBytes, wp + (size_t)ch.src * row3,
               (uint32_t)(ch.n * row3), &S.mbar[s]);
    } else {
      mbar_expect_tx(&S.mbar[s], 0u);  // invalid row: empty chunk
    }
  };
  FH_STAMP(12);
  const int n_chunks_total = nch >= 0 ? nch : 0x7FFFFFFF;
  auto more_to_issue = [&]() { return nch >= 0 ? c_issue < nch : w_issue < w1; };
  if (tid == 0) {
    uint32_t gidx = gi;
    for (int k = 0; k < kFSlots && more_to_issue(); ++k) issue3(gidx++);
  }
  for (int c = 0; c < n_chunks_total && w_cons < w1; ++c) {
    int w_dummy = w_cons;
    const S2Chunk ch = nch >= 0 ? S.chunks[c] : chunk_at(c, w_dummy);
    const int n = ch.n;
    const int s = gi % kFSlots;
    if (!mbar_wait(&S.mbar[s], (gi / kFSlots) & 1, a.copy_polls) && lane == 0)
      atomicOr(&S.s_err, kErrCopyTimeout);
    const int hr = ch.hrow;
    if (ch.src >= 0 && g3 < RG3) {
      const unsigned char *base = ring + (size_t)s * kFSlotBytes + (size_t)col3 * 16;
      for (int r = g3; r < n; r += RG3) {
        float w[8];
        vec_to_float<HT>(lds128(base + (size_t)r * row3), w);
        float acc = 0.f;
#pragma unroll
        for (int hh = 0; hh < R; ++hh) {
          if (hh == hr) {
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(w[e], h3[hh][e], acc);
          }
        }
        acc = warp_sum(acc);
        if (lane == 0) S.part[s][r][q3][0] = acc;
      }
    }
    __syncthreads();
    if (ch.src >= 0 && tid < n) {
      float acc = 0.f;
      for (int q = 0; q < Q3; ++q) acc += S.part[s][tid][q][0];
      const int wi = ch.w - w0 + tid;
      const uint32_t vid = (uint32_t)(wi < n_vid ? vid_sm[wi] : a.vocab_map[ch.src + tid]);
      float key = acc;
      if (a.do_sample)
        key = acc / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)hr, vid);
      atomicMax(&S.best[hr - r_lo], pack(key, vid));
    }
    w_cons += n;
    ++gi;
    if (tid == 0 && more_to_issue()) issue3(gi + kFSlots - 1);
  }
  __syncthreads();
  FH_STAMP(5);

  // --------------------------------------------------------------- reduction
  if (tid <= r_hi - r_lo && S.best[tid] != 0ull) atomicMax(&a.packed[r_lo + tid], S.best[tid]);
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
    if (tid == 0) {
      a.sync[kSyncArrive] = 0u;
      a.sync[kSyncDone] = 0u;
      a.sync[kSyncEpoch] = epoch + 1u;
    }
  }
}

}  // namespace fh
