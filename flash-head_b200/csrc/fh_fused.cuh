// One-kernel FlashHead decode step for a few hidden rows (R <= 4).
//
// A persistent cooperative grid of one 512-thread CTA per SM runs the whole
// step with one grid-wide barrier:
//
//  1. stage 1   CTA b streams its contiguous slice of centroid rows
//               [b*K/G, (b+1)*K/G) as 16-row tiles through a 128 KB ring of
//               shared-memory slots filled by bulk asynchronous copies (TMA
//               engine, completion on mbarriers; one copy per tile when 16 rows
//               fit a slot). Each tile is scored on the tensor cores with
//               mma.m16n8k16 fragments (fp8 rows converted exactly to f16),
//               the d-range split over the 16 warps and reduced once per tile.
//               Each score's key goes into global two-level histograms
//               (256 coarse x 256 fine bins: bf16 resolution).
//  2. barrier   one arrive counter, bounded spin (a timeout sets an error bit
//               and the kernel still runs to completion). Before arriving, each
//               CTA prefetches into L2 the w_perm rows of its clusters that are
//               likely to be selected, so HBM works through the barrier.
//  3. select    one warp per hidden row finds, from two 1 KB histogram reads,
//               the bf16 bucket that holds the p-th largest score. Each CTA
//               keeps the clusters it scored whose key lies above that bucket;
//               keys inside the bucket (a handful) are published to a small
//               tie list, and only the CTAs owning such keys wait for the
//               bucket's count (known from the histogram) to be reached, then
//               rank their keys exactly (largest score, then smallest id).
//  4. stage 2   every CTA streams the w_perm rows (and vocab ids) of its own
//               selected clusters, and CTA r row r's special tokens, through
//               the same ring (a whole 16-row cluster per copy when it fits a
//               slot), scores them with mma fragments, and keeps the best
//               packed (logit or Gumbel key, vocab id) word per row; words meet
//               in a 64-bit atomicMax and the last CTA to finish publishes the
//               ids.
//
// Histograms and tie lists alternate between two buffers by a call epoch;
// each call zeroes the buffers of the next call and the last CTA resets the
// counters, so a workspace zero-filled once stays consistent.
#pragma once

#include "fh_kernels.cuh"

namespace fh {

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kRingBytes = 128 * 1024;
constexpr int kMaxSlots = 4;
constexpr int kTileRows = 16;
constexpr int kFMaxRows = 4;
constexpr int kFMaxProbes = 4096;
constexpr int kFMaxSpecial = 256;
constexpr int kTieCap = 1024;
constexpr int kWorkCap = 1024;  // stage-2 items of one CTA (own clusters + specials)
constexpr int kS3MaxRows = 16;  // w_perm rows per stage-2 tile (cluster size limit)

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
  float *scores;       // [R, K] global scratch (exact ranking of large buckets)
  uint32_t *sync;      // workspace state words
  unsigned char *epoch_bufs;   // 2 x (histograms, tie lists)
  unsigned long long *packed;  // [R]
  int64_t *out_ids;    // [R]
  uint32_t barrier_polls;      // grid-barrier / tie-list poll limit
  uint32_t copy_polls;         // mbarrier poll limit
  int extra_arrivals;          // >0 only in the timeout test: wait for more CTAs than exist
};

struct RowThreshold {
  uint32_t prefix;  // 16-bit key prefix of the bucket holding the p-th score
  int need;         // keys of that bucket to select
  int cnt;          // keys in that bucket
};

// One chunk of a stage-2 tile: rows [src, src + n) of w_perm, bytes
// [dc * chunk row bytes, ...) of each row.
struct S2Chunk {
  int src;    // first w_perm row; -1 invalid (empty chunk); -2 end of work
  int n;      // rows (1..16)
  int row;    // hidden row
  int dc;     // d-chunk index within the rows
  int last;   // last d-chunk of this tile
  int vid_in_smem;
};

struct FusedSmem {
  uint64_t mbar[kMaxSlots];
  float part[2][kFWarps][kTileRows][kFMaxRows];  // per-warp partial tile results
  float local[kFMaxRows][128];
  float scale[128];
  uint32_t coarse[kFMaxRows * kHistCoarse];
  __align__(16) int vid[kMaxSlots][kTileRows];
  S2Chunk desc[kMaxSlots];
  RowThreshold thr[kFMaxRows];
  unsigned long long best[kFMaxRows];
  uint32_t work[kWorkCap];
  int n_work;
  int bucket_keys[kFMaxRows];  // this CTA's keys inside row r's threshold bucket
  uint32_t s_err;
  uint32_t s_last;
};

constexpr size_t kFSmemBase = (kRingBytes + sizeof(FusedSmem) + 127) / 128 * 128;
constexpr size_t kFSmemMax = 226 * 1024;

// Dynamic shared memory of k_fused_step: ring, FusedSmem, the hidden rows as
// stage-2 B operands [R][D] (16-bit) and, for fp8 stage-1 rows, as f16
// stage-1 B operands [R][D].
__host__ __device__ __forceinline__ size_t fused_smem_bytes(int R, int D, int wt_bytes) {
  return kFSmemBase + (size_t)R * D * 2 * (wt_bytes == 1 ? 2 : 1);
}

// Ring geometry of one stage for rows of rb bytes: slots of 32 KB when a
// 16-row tile fits, else 64 KB; a tile row is cut into chunks of cb bytes
// when 16 full rows do not fit a slot. Rows sit in a slot at pitch
// (one bulk copy per tile when the tile is one chunk, else one per row).
struct RingGeom {
  int slot_bytes, n_slots, cb, ndc, pitch;
};
__host__ __device__ __forceinline__ RingGeom ring_geom(int rb) {
  RingGeom g;
  g.slot_bytes = kTileRows * rb <= 32 * 1024 ? 32 * 1024 : 64 * 1024;
  g.n_slots = kRingBytes / g.slot_bytes;
  g.cb = rb < g.slot_bytes / kTileRows ? rb : g.slot_bytes / kTileRows;
  g.ndc = (rb + g.cb - 1) / g.cb;
  g.pitch = g.ndc == 1 ? rb : g.cb;
  return g;
}

// ---------------------------------------------------------------------------
// Tensor-core tile GEMV: mma.m16n8k16 with f32 accumulators.
//
// Fragment use (lane = 4g + t): the lane loads 16 contiguous bytes of tile
// rows g and g + 8 and the matching slice of the hidden row that feeds
// column g. Because a dot product may take its k indices in any order as long
// as A and B agree, k-step j of a 64-byte row group uses, for lane t,
// elements (16t + 4j + u) of an fp8 group (4 steps) or (8t + 4j + u) of a
// 16-bit group (2 steps), u = 0..3: slots {2t, 2t+1} take u = 0, 1 and
// slots {2t+8, 2t+9} take u = 2, 3.
//
// Bank conflicts: tile rows lie at a pitch that is a multiple of 128 bytes,
// so rows g and g + 1 (one quarter-warp of 16-byte loads) would hit the same
// banks. Odd g therefore read the neighbouring 64-byte group (q ^ 1) of their
// rows, and B column n carries the hidden slice of parity n & 1: column
// 2r + (g & 1) of row g is the dot product of row g with hidden row r, exact
// over the full row because q -> q ^ 1 permutes the groups of a chunk.
// ---------------------------------------------------------------------------
template <typename MT>
__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, const uint32_t *b);
template <>
__device__ __forceinline__ void mma16816<__half>(float *c, const uint32_t *a, const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float *c, const uint32_t *a,
                                                        const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t fp8x2_to_f16x2(uint32_t v16) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v16, __NV_E4M3);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// MMA operand type for stage-1 rows of type WT: f16 for fp8 and f16 rows,
// bf16 for bf16 rows.
template <typename WT>
struct S1Mma {
  using T = __half;
};
template <>
struct S1Mma<__nv_bfloat16> {
  using T = __nv_bfloat16;
};

// f16 copy of a hidden row for fp8 stage-1 groups: 16-byte granule gr of
// 64-element group q is stored at granule gr ^ (q & 1), so the two granules a
// lane reads (2t, 2t + 1) for groups q and q ^ 1 fall in different banks.
__device__ __forceinline__ int fp8_hidden_slot(int e) {
  const int q = e >> 6, gr = (e >> 3) & 7;
  return (q << 6) | ((gr ^ (q & 1)) << 3) | (e & 7);
}

// One 64-byte group of a tile for this lane: rows g / g + 8 at ra / rb
// (shared memory), hidden slice at h0 (and h1 for fp8: the second granule).
template <typename WT, typename MT>
__device__ __forceinline__ void tile_group(float *c, const unsigned char *ra,
                                           const unsigned char *rb, const MT *h0,
                                           const MT *h1) {
  const uint4 a0 = lds128(ra), b0 = lds128(rb);
  if constexpr (sizeof(WT) == 1) {
    const uint4 x0 = lds128(h0), x1 = lds128(h1);
    const uint32_t wa[4] = {a0.x, a0.y, a0.z, a0.w}, wb[4] = {b0.x, b0.y, b0.z, b0.w};
    const uint32_t hh[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a[4] = {fp8x2_to_f16x2(wa[j] & 0xFFFFu), fp8x2_to_f16x2(wb[j] & 0xFFFFu),
                             fp8x2_to_f16x2(wa[j] >> 16), fp8x2_to_f16x2(wb[j] >> 16)};
      const uint32_t b[2] = {hh[2 * j], hh[2 * j + 1]};
      mma16816<MT>(c, a, b);
    }
  } else {
    const uint4 x0 = lds128(h0);
    {
      const uint32_t a[4] = {a0.x, b0.x, a0.y, b0.y};
      const uint32_t b[2] = {x0.x, x0.y};
      mma16816<MT>(c, a, b);
    }
    {
      const uint32_t a[4] = {a0.z, b0.z, a0.w, b0.w};
      const uint32_t b[2] = {x0.z, x0.w};
      mma16816<MT>(c, a, b);
    }
  }
}

template <typename T>
__device__ __forceinline__ T f2t(float x);
template <>
__device__ __forceinline__ __half f2t<__half>(float x) {
  return __float2half_rn(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 f2t<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
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
  using M1 = typename S1Mma<WT>::T;  // stage-1 mma operand type
  constexpr bool kFp8 = sizeof(WT) == 1;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *ring = smem;
  FusedSmem &S = *reinterpret_cast<FusedSmem *>(smem + kRingBytes);
  HT *hB3 = reinterpret_cast<HT *>(smem + kFSmemBase);  // [R][D] stage-2 B operand
  // stage-1 B operand: a swizzled f16 copy for fp8 rows, else the same array
  M1 *hB1 = kFp8 ? reinterpret_cast<M1 *>(smem + kFSmemBase + (size_t)R * a.D * 2)
                 : reinterpret_cast<M1 *>(hB3);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x;
  const int gq = lane >> 2, tq = lane & 3, odd = gq & 1;  // mma fragment coordinates
  uint32_t phase = 0u;  // parity of the next completion of each slot's mbarrier
  if (tid == 0) {
    for (int s = 0; s < kMaxSlots; ++s) mbar_init(&S.mbar[s], 1);
    fence_mbar_init();
    S.s_err = 0u;
    S.n_work = 0;
  }
  if (tid < kFMaxRows) {
    S.best[tid] = 0ull;
    S.bucket_keys[tid] = 0;
  }
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
  const int rb1 = a.D * (int)sizeof(WT);  // bytes per centroid row
  const RingGeom g1 = ring_geom(rb1);
  const int ntile1 = (nc + kTileRows - 1) / kTileRows;
  const int n1 = ntile1 * g1.ndc;
  const char *wsrc = reinterpret_cast<const char *>(a.cw) + (size_t)c0 * rb1;
  auto issue1 = [&](int c) {
    const int s = c % g1.n_slots, tile = c / g1.ndc, dc = c - tile * g1.ndc;
    const int tr = min(kTileRows, nc - tile * kTileRows);
    const int cb = min(g1.cb, rb1 - dc * g1.cb);
    fence_proxy_async_smem();
    mbar_expect_tx(&S.mbar[s], (uint32_t)(tr * cb));
    unsigned char *dst = ring + (size_t)s * g1.slot_bytes;
    const char *src = wsrc + (size_t)tile * kTileRows * rb1 + (size_t)dc * g1.cb;
    if (g1.ndc == 1) {
      bulk_g2s(dst, src, (uint32_t)(tr * rb1), &S.mbar[s]);
    } else {
      for (int r = 0; r < tr; ++r)
        bulk_g2s(dst + (size_t)r * g1.pitch, src + (size_t)r * rb1, (uint32_t)cb, &S.mbar[s]);
    }
  };
  if (tid == 0)
    for (int c = 0; c < min(g1.n_slots, n1); ++c) issue1(c);
  if (tid < nc) S.scale[tid] = a.cscale ? a.cscale[c0 + tid] : 1.f;
  // hidden rows as mma B operands (16-bit) in shared memory
  for (int i = tid; i < R * a.D; i += kFThreads) {
    const int r = i / a.D, e = i - r * a.D;
    float v = 0.f;
    if (r < a.rows) v = (float)reinterpret_cast<const HT *>(a.hidden)[i];
    hB3[i] = f2t<HT>(v);
    if (kFp8) hB1[(size_t)r * a.D + fp8_hidden_slot(e)] = f2t<M1>(v);
  }
  __syncthreads();

  FH_TICK_DECL
  {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int hrow = (gq >> 1) < R ? (gq >> 1) : 0;  // hidden row feeding column gq
    const M1 *hrow1 = hB1 + (size_t)hrow * a.D;
    for (int c = 0; c < n1; ++c) {
      const int s = c % g1.n_slots, tile = c / g1.ndc, dc = c - tile * g1.ndc;
      const int tr = min(kTileRows, nc - tile * kTileRows);
      const int cb = min(g1.cb, rb1 - dc * g1.cb);
      FH_TICK(7);
      if (!mbar_wait(&S.mbar[s], (phase >> s) & 1u, a.copy_polls) && lane == 0)
        atomicOr(&S.s_err, kErrCopyTimeout);
      phase ^= 1u << s;
      FH_TICK(0);
      const unsigned char *slot = ring + (size_t)s * g1.slot_bytes;
      const int ng = cb / 64;
      const int qbase = dc * (g1.cb / 64);  // first 64-byte group of this chunk in the row
      for (int grp = warp; grp < ng; grp += kFWarps) {
        const int q = grp ^ odd;
        const unsigned char *ra = slot + (size_t)gq * g1.pitch + q * 64 + tq * 16;
        if constexpr (kFp8) {
          const M1 *hg = hrow1 + (size_t)(qbase + q) * 64;
          const int sw = (qbase + q) & 1;
          tile_group<WT, M1>(acc, ra, ra + 8 * g1.pitch, hg + (((2 * tq) ^ sw) << 3),
                             hg + (((2 * tq + 1) ^ sw) << 3));
        } else {
          const M1 *hg = hrow1 + (size_t)(qbase + q) * 32 + tq * 8;
          tile_group<WT, M1>(acc, ra, ra + 8 * g1.pitch, hg, hg);
        }
      }
      const bool last = dc == g1.ndc - 1;
      if (last) {
        // lane (g, t): row g (and g + 8) against hidden row t in c[odd] (c[2 + odd])
        const int par = tile & 1;
        if (tq < R) {
          S.part[par][warp][gq][tq] = acc[odd];
          S.part[par][warp][gq + 8][tq] = acc[2 + odd];
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      }
      FH_TICK(1);
      __syncthreads();
      FH_TICK(2);
      if (tid == 0 && c + g1.n_slots < n1) issue1(c + g1.n_slots);
      if (last && tid < kTileRows * kFWarps) {
        // tile reduction: thread = (row, warp); a 16-lane shuffle tree per row
        const int row = tid >> 4, w = tid & 15, par = tile & 1;
#pragma unroll
        for (int col = 0; col < R; ++col) {
          float v = S.part[par][w][row][col];
          v += __shfl_xor_sync(0xFFFFFFFFu, v, 8);
          v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
          v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
          v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
          if (w == 0 && row < tr && col < a.rows) {
            const int k = c0 + tile * kTileRows + row;
            float sc = v * S.scale[k - c0];
            if (a.do_sample)
              sc = sc / a.temperature + gumbel(a.rng, kStageClusters, (uint32_t)col, (uint32_t)k);
            S.local[col][k - c0] = sc;
            a.scores[(size_t)col * a.K + k] = sc;
            const uint32_t key = mono(sanitize(sc));
            atomicAdd(&hist_cur[(size_t)col * kHistWords + kHistCoarse + (key >> 16)], 1u);
            atomicAdd(&S.coarse[col * kHistCoarse + (key >> 24)], 1u);
          }
        }
      }
      FH_TICK(3);
    }
  }
  __syncthreads();
  FH_STAMP(7);
  for (int i = tid; i < a.rows * kHistCoarse; i += kFThreads) {
    const uint32_t cc = S.coarse[i];
    if (cc) atomicAdd(&hist_cur[(size_t)(i / kHistCoarse) * kHistWords + (i % kHistCoarse)], cc);
  }
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
      atomicAdd(&S.bucket_keys[hr], 1);
      if (S.thr[hr].cnt <= kTieCap) {
        const uint32_t t = atomicAdd(&a.sync[kSyncTieCount + hr], 1u);
        if (t < (uint32_t)kTieCap) ties[(size_t)hr * kTieCap + t] = pack(v, (uint32_t)(c0 + k));
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
  const int rb3 = a.D * (int)sizeof(HT);
  const RingGeom g3 = ring_geom(rb3);
  const char *wp = reinterpret_cast<const char *>(a.w_perm);
  // Producer state (thread 0 only): next work item and its next d-chunk.
  int p_item = 0, p_dc = 0;
  auto produce = [&](int s) {
    S2Chunk d;
    d.src = -2;
    d.n = 0;
    d.row = 0;
    d.dc = 0;
    d.last = 1;
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
      } else {
        d.src = payload < a.K ? payload * a.cap : -1;
        d.n = a.cap;
      }
      d.dc = p_dc;
      d.last = p_dc == g3.ndc - 1;
      if (d.last) {
        ++p_item;
        p_dc = 0;
      } else {
        ++p_dc;
      }
    }
    if (d.src >= 0) {
      const int cb = min(g3.cb, rb3 - d.dc * g3.cb);
      const int *vsrc = a.vocab_map + d.src;
      const bool vid_bulk =
          d.last && ((reinterpret_cast<uintptr_t>(vsrc) & 15u) == 0) && (d.n % 4 == 0);
      d.vid_in_smem = vid_bulk ? 1 : 0;
      S.desc[s] = d;
      fence_proxy_async_smem();
      mbar_expect_tx(&S.mbar[s], (uint32_t)(d.n * cb) + (vid_bulk ? (uint32_t)(d.n * 4) : 0u));
      unsigned char *dst = ring + (size_t)s * g3.slot_bytes;
      const char *src = wp + (size_t)d.src * rb3 + (size_t)d.dc * g3.cb;
      if (g3.ndc == 1) {
        bulk_g2s(dst, src, (uint32_t)(d.n * rb3), &S.mbar[s]);
      } else {
        for (int r = 0; r < d.n; ++r)
          bulk_g2s(dst + (size_t)r * g3.pitch, src + (size_t)r * rb3, (uint32_t)cb, &S.mbar[s]);
      }
      if (vid_bulk) bulk_g2s(&S.vid[s][0], vsrc, (uint32_t)(d.n * 4), &S.mbar[s]);
    } else {
      S.desc[s] = d;
      mbar_expect_tx(&S.mbar[s], 0u);  // invalid row or end of work: no data
    }
  };
  // Start streaming the certain clusters, then settle this CTA's bucket keys;
  // slots are only marked end-of-work once the work list is final. Chunk i of
  // stage 2 uses slot i % n_slots.
  int n_prod = 0;  // thread 0: next chunk to produce
  if (tid == 0)
    while (n_prod < g3.n_slots && p_item < min(S.n_work, kWorkCap)) produce(n_prod++ % g3.n_slots);
  // Rank this CTA's bucket keys exactly, one warp per key, against the full
  // bucket: the published tie list (complete once its count reaches the
  // histogram's), or, for a bucket larger than the list, the scores row itself.
  bool any_bucket = false;
  for (int hr = 0; hr < a.rows; ++hr) any_bucket |= S.bucket_keys[hr] > 0;
  if (any_bucket) {
    if (tid == 0) {
      for (int hr = 0; hr < a.rows; ++hr) {
        if (S.bucket_keys[hr] == 0 || S.thr[hr].cnt > kTieCap) continue;
        const uint32_t want = (uint32_t)S.thr[hr].cnt;
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
    for (int i = warp; i < a.rows * nc; i += kFWarps) {
      const int hr = i / nc, k = i - (i / nc) * nc;
      const float v = sanitize(S.local[hr][k]);
      const uint32_t P = S.thr[hr].prefix;
      if ((mono(v) >> 16) != P) continue;  // warp-uniform
      const unsigned long long mine = pack(v, (uint32_t)(c0 + k));
      const int cnt = S.thr[hr].cnt;
      int rank = 0;
      if (cnt <= kTieCap) {
        for (int t = lane; t < cnt; t += 32) rank += __ldcg(&ties[(size_t)hr * kTieCap + t]) > mine;
      } else {
        for (int t = lane; t < a.K; t += 32) {
          const float u = sanitize(__ldcg(&a.scores[(size_t)hr * a.K + t]));
          rank += (mono(u) >> 16) == P && pack(u, (uint32_t)t) > mine;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) rank += __shfl_xor_sync(0xFFFFFFFFu, rank, o);
      if (lane == 0 && rank < S.thr[hr].need) {
        const int w = atomicAdd(&S.n_work, 1);
        if (w < kWorkCap) S.work[w] = ((uint32_t)hr << 28) | (uint32_t)(c0 + k);
      }
    }
  }
  FH_STAMP(4);
  __syncthreads();
  if (tid == 0)
    while (n_prod < g3.n_slots) produce(n_prod++ % g3.n_slots);
  FH_TICK(7);
  {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int tile = 0;
    for (int c = 0;; ++c) {
      const int s = c % g3.n_slots;
      if (!mbar_wait(&S.mbar[s], (phase >> s) & 1u, a.copy_polls) && lane == 0)
        atomicOr(&S.s_err, kErrCopyTimeout);
      phase ^= 1u << s;
      FH_TICK(4);
      const S2Chunk d = S.desc[s];
      if (c == 0) FH_STAMP(11);
      if (d.src == -2) break;
      if (d.src >= 0) {
        const int cb = min(g3.cb, rb3 - d.dc * g3.cb);
        const unsigned char *slot = ring + (size_t)s * g3.slot_bytes;
        const int ng = cb / 64;
        const HT *hrow3 = hB3 + (size_t)d.row * a.D + (size_t)d.dc * (g3.cb / 2) + tq * 8;
        for (int grp = warp; grp < ng; grp += kFWarps) {
          const int q = grp ^ odd;
          const unsigned char *ra = slot + (size_t)gq * g3.pitch + q * 64 + tq * 16;
          tile_group<HT, HT>(acc, ra, ra + 8 * g3.pitch, hrow3 + q * 32, hrow3 + q * 32);
        }
      }
      // vocab id of tile row tid >> 4, read before the slot is refilled
      uint32_t vid = 0u;
      if (d.last && d.src >= 0 && tid < kTileRows * kFWarps && (tid & 15) == 0 &&
          (tid >> 4) < d.n)
        vid = (uint32_t)(d.vid_in_smem ? S.vid[s][tid >> 4] : __ldg(&a.vocab_map[d.src + (tid >> 4)]));
      if (d.last) {
        // every B column pair holds hidden row d.row: lanes t == 0 carry rows g, g + 8
        const int par = tile & 1;
        if (tq == 0) {
          S.part[par][warp][gq][0] = acc[odd];
          S.part[par][warp][gq + 8][0] = acc[2 + odd];
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      }
      FH_TICK(5);
      __syncthreads();  // slot s is free; partials of a finished tile are visible
      if (tid == 0) produce(n_prod++ % g3.n_slots);
      if (d.last && d.src >= 0 && tid < kTileRows * kFWarps) {
        const int row = tid >> 4, w = tid & 15, par = tile & 1;
        float v = S.part[par][w][row][0];
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 8);
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
        if (w == 0 && row < d.n) {
          float key = v;
          if (a.do_sample)
            key = v / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)d.row, vid);
          atomicMax(&S.best[d.row], pack(key, vid));
        }
      }
      if (d.last) ++tile;
      FH_TICK(6);
    }
  }
  FH_TICK_FLUSH();
  __syncthreads();
  FH_STAMP(5);

  // --------------------------------------------------------------- reduction
  if (tid < a.rows && S.best[tid] != 0ull) atomicMax(&a.packed[tid], S.best[tid]);
  if (tid == 0 && S.s_err) atomicOr(&a.sync[kSyncError], S.s_err);
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    S.s_last = atomicAdd(&a.sync[kSyncDone], 1u) == (uint32_t)G - 1;
  }
  __syncthreads();
  FH_STAMP(6);
  if (S.s_last) {
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
