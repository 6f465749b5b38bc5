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
//  3. select    every CTA copies the full score rows (32 KB per row at
//               K = 8016) from L2 into shared memory while one warp per hidden
//               row finds, from two 1 KB histogram reads, the bf16 bucket that
//               holds the p-th largest score. The exact threshold key inside
//               that bucket (largest score, then smallest id) is ranked from
//               the bucket's few keys, or by a 6-pass radix select over the
//               row when the bucket is large. Every CTA thus knows the whole
//               selection without waiting on any other CTA.
//  4. stage 2   the step's items (per row: the p selected clusters in id order,
//               then the special tokens) are split into G equal contiguous
//               ranges; CTA b streams the w_perm rows (and vocab ids) of its
//               range through the same ring (a whole 16-row cluster per copy
//               when it fits a slot), scores them with mma fragments, and keeps
//               the best packed (logit or Gumbel key, vocab id) word per row;
//               words meet in a 64-bit atomicMax and the last CTA to finish
//               publishes the ids.
//
// Histograms alternate between two buffers by a call epoch; each call zeroes
// the buffers of the next call and the last CTA resets the counters, so a
// workspace zero-filled once stays consistent.
#pragma once

#include "fh_kernels.cuh"

namespace fh {

constexpr int kFThreads = 512;             // 16 compute warps
constexpr int kFWarps = kFThreads / 32;
constexpr int kFBlock = kFThreads + 32;    // + one producer / reducer warp
// Named barriers between the compute warps and the producer warp.
constexpr int kBarSlot0 = 1;  // 1..4: slot s consumed (and a finished tile's partials written)
constexpr int kBarPart0 = 5;  // 5..6: partial buffer (tile & 1) reduced, free again
constexpr int kMaxChunks = 160;  // 128-cluster chunks of a score row
constexpr int kMaxS1Chunks = 8;  // stage-1 chunks of one CTA (each with its own partials)
// Speculative stage-2 prefetch before the grid barrier: clusters scoring above
// mean + (z - margin) * sd of this CTA's scores, z the normal quantile of the
// selection rate p / K. A negative margin keeps it to clusters very likely to
// be selected: more would compete for HBM with CTAs still streaming stage 1
// (measured: margin -1 is ~1.5 us faster per step than +0.25).
constexpr float kPrefetchMargin = -1.0f;
// Bulk copies per stage-2 cluster: four copies of 4 rows complete sooner than
// one of 16 (measured ~0.4 us per step at batch 1).
constexpr int kS2Pieces = 4;
// Bytes per stage-1 bulk copy (whole rows, at least one): pieces of about
// 8 KB keep more requests in flight than one copy per 16-row tile and pay
// less issue cost than one per row (measured at batch 1: 8 KB pieces beat
// 16 KB and 4 KB ones by ~0.7 us per step for 4 KB bf16 rows, and beat 4 KB
// and 16 KB ones for 2 KB fp8 rows).
constexpr int kS1PieceBytes = 8192;
constexpr int kRingBytes = 128 * 1024;
constexpr int kMaxSlots = 4;
constexpr int kTileRows = 16;
constexpr int kFMaxRows = 4;
constexpr int kFMaxProbes = 4096;
constexpr int kFMaxSpecial = 256;
constexpr int kBktCap = 64;     // bucket keys ranked directly; larger buckets: radix select
constexpr int kWorkCap = 1024;  // stage-2 items of one CTA
constexpr int kS3MaxRows = 16;  // w_perm rows per stage-2 tile (cluster size limit)

// State words at the start of the workspace (uint32 index).
constexpr int kSyncArrive = 1;
constexpr int kSyncDone = 2;
constexpr int kSyncError = 3;
constexpr int kSyncEpoch = 4;
constexpr int kSyncS2Done = 5;  // CTAs of a batched stage-2 launch that finished

constexpr int kHistCoarse = 256;
constexpr int kHistWords = kHistCoarse + 65536;
// Per-epoch histogram buffers (two).
constexpr size_t kEpochBufBytes = (size_t)kFMaxRows * kHistWords * sizeof(uint32_t);
constexpr size_t kHistBytes = 2 * kEpochBufBytes;  // workspace bytes of all epoch buffers

constexpr uint32_t kErrBarrierTimeout = 1u;
constexpr uint32_t kErrCopyTimeout = 2u;

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
  float *scores;       // [R, score_stride] global scratch: every CTA reads all scores
  int score_stride;    // multiple of 4
  uint32_t *sync;      // workspace state words
  unsigned char *epoch_bufs;   // 2 x histograms
  unsigned long long *packed;  // [R]
  int64_t *out_ids;    // [R]
  uint32_t barrier_polls;      // grid-barrier poll limit
  uint32_t copy_polls;         // mbarrier poll limit
  int extra_arrivals;          // >0 only in the timeout test: wait for more CTAs than exist
  unsigned long long *trace;   // profiling builds only: phase stamps (else null)
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
  __align__(16) float part[2][kTileRows][kFMaxRows][kFWarps];  // per-warp partial tile results
  float local[kFMaxRows][128];
  float scale[128];
  uint32_t coarse[kFMaxRows * kHistCoarse];
  __align__(16) int vid[kMaxSlots][kTileRows];
  S2Chunk desc[kMaxSlots];
  RowThreshold thr[kFMaxRows];
  float t_est[kFMaxRows];                      // estimated selection threshold per row
  unsigned long long best[kFMaxRows];
  unsigned long long tkey[kFMaxRows];          // selection: key >= tkey[r]
  unsigned long long bkt[kFMaxRows][kBktCap];  // keys of row r's threshold bucket
  int bkt_n[kFMaxRows];
  __align__(16) uint32_t rhist[256];           // radix-select digit histogram
  int rsel_bin, rsel_above;
  int chunk_sel[kFMaxRows][kMaxChunks];        // selected keys per 128-cluster chunk
  int chunk_off[kFMaxRows][kMaxChunks];        // their first position in id order
  uint32_t work[kWorkCap];
  int n_work;
  uint32_t s_err;
  uint32_t s_last;
#ifdef FH_TRACE
  long long trace_clk[24];
#endif
};

constexpr size_t kFSmemBase = (kRingBytes + sizeof(FusedSmem) + 127) / 128 * 128;
constexpr size_t kFSmemMax = 226 * 1024;

// Dynamic shared memory of k_fused_step: ring, FusedSmem, stage-1 partials
// [kMaxS1Chunks][16 rows][R][16 warps], the hidden rows as stage-2 B operands
// [R][D] (16-bit) and, for fp8 stage-1 rows, as f16 stage-1 B operands [R][D].
__host__ __device__ __forceinline__ size_t s1_part_bytes(int R) {
  return (size_t)kMaxS1Chunks * kTileRows * R * kFWarps * sizeof(float);
}
__host__ __device__ __forceinline__ size_t fused_smem_bytes(int R, int D, int wt_bytes) {
  return kFSmemBase + s1_part_bytes(R) + (size_t)R * D * 2 * (wt_bytes == 1 ? 2 : 1);
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
// Even k-steps accumulate into c0, odd ones into c1 (two independent chains).
template <typename WT, typename MT>
__device__ __forceinline__ void tile_group_h(float *c0, float *c1, const unsigned char *ra,
                                             const unsigned char *rb, const uint4 x0,
                                             const uint4 x1) {
  const uint4 a0 = lds128(ra), b0 = lds128(rb);
  if constexpr (sizeof(WT) == 1) {
    const uint32_t wa[4] = {a0.x, a0.y, a0.z, a0.w}, wb[4] = {b0.x, b0.y, b0.z, b0.w};
    const uint32_t hh[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a[4] = {fp8x2_to_f16x2(wa[j] & 0xFFFFu), fp8x2_to_f16x2(wb[j] & 0xFFFFu),
                             fp8x2_to_f16x2(wa[j] >> 16), fp8x2_to_f16x2(wb[j] >> 16)};
      const uint32_t b[2] = {hh[2 * j], hh[2 * j + 1]};
      mma16816<MT>((j & 1) ? c1 : c0, a, b);
    }
  } else {
    {
      const uint32_t a[4] = {a0.x, b0.x, a0.y, b0.y};
      const uint32_t b[2] = {x0.x, x0.y};
      mma16816<MT>(c0, a, b);
    }
    {
      const uint32_t a[4] = {a0.z, b0.z, a0.w, b0.w};
      const uint32_t b[2] = {x0.z, x0.w};
      mma16816<MT>(c1, a, b);
    }
  }
}
template <typename WT, typename MT>
__device__ __forceinline__ void tile_group(float *c0, float *c1, const unsigned char *ra,
                                           const unsigned char *rb, const MT *h0,
                                           const MT *h1) {
  const uint4 x0 = lds128(h0);
  const uint4 x1 = sizeof(WT) == 1 ? lds128(h1) : x0;
  tile_group_h<WT, MT>(c0, c1, ra, rb, x0, x1);
}

// Named barriers (warp-aligned: every lane of a warp calls them together).
__device__ __forceinline__ void nbar_arrive(int id, int n) {
  __syncwarp();
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void nbar_sync(int id, int n) {
  __syncwarp();
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
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
// Profiling builds only. Phase stamps are clock64 values kept in shared
// memory (thread 0, or producer lane 0 for FH_STAMP_P) and written out at the
// end of the kernel as %globaltimer-aligned nanoseconds at 1965 MHz into
// a.trace[b * 24 + p]; thread 0's clock64 accumulators go to
// a.trace[G * 24 + b * 8 + k]. Nothing is stored to global memory before.
#define FH_STAMP_AT(p, who)                                              \
  do {                                                                   \
    if (threadIdx.x == (who) && a.trace) S.trace_clk[p] = clock64();     \
  } while (0)
#define FH_STAMP(p) FH_STAMP_AT(p, 0)
#define FH_STAMP_P(p) FH_STAMP_AT(p, kFThreads)
#define FH_TICK_DECL long long fh_t0 = clock64(); long long fh_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#define FH_TICK(k) do { const long long _t = clock64(); fh_acc[k] += _t - fh_t0; fh_t0 = _t; } while (0)
#define FH_TICK_FLUSH() do { if (threadIdx.x == 0 && a.trace) for (int _k = 0; _k < 8; ++_k) a.trace[gridDim.x * 24 + blockIdx.x * 8 + _k] = fh_acc[_k]; } while (0)
#define FH_TRACE_INIT()                                                  \
  long long fh_clk0 = 0;                                                 \
  unsigned long long fh_gt0 = 0;                                         \
  if (threadIdx.x == 0) {                                                \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(fh_gt0));           \
    fh_clk0 = clock64();                                                 \
  }                                                                      \
  for (int _i = threadIdx.x; _i < 24; _i += blockDim.x) S.trace_clk[_i] = 0;
#define FH_TRACE_WRITE()                                                 \
  do {                                                                   \
    __syncthreads();                                                     \
    if (threadIdx.x == 0 && a.trace)                                     \
      for (int _p = 0; _p < 24; ++_p)                                    \
        a.trace[blockIdx.x * 24 + _p] =                                  \
            S.trace_clk[_p] ? fh_gt0 + (S.trace_clk[_p] - fh_clk0) * 1000 / 1965 : 0; \
  } while (0)
#else
#define FH_STAMP(p) ((void)0)
#define FH_STAMP_P(p) ((void)0)
#define FH_TICK_DECL
#define FH_TICK(k) ((void)0)
#define FH_TICK_FLUSH() ((void)0)
#define FH_TRACE_INIT()
#define FH_TRACE_WRITE() ((void)0)
#endif


// Warp-level search of a 256-bin histogram (highest bin first) for the bin
// holding the need-th largest key: returns the bin, the count above it and
// the bin's count (all lanes).
__device__ __forceinline__ void warp_find_bin_regs(const uint4 lo, const uint4 hi, int need,
                                                   int &bin, int &above, int &cnt);
// lane l owns bins 255-8l .. 248-8l (descending): bins + 248 - 8l (lo), + 252 - 8l (hi)
template <bool kGlobal>
__device__ __forceinline__ void warp_find_bin(const uint32_t *bins, int need, int &bin,
                                              int &above, int &cnt) {
  const int lane = threadIdx.x & 31;
  const uint4 *plo = reinterpret_cast<const uint4 *>(bins + 248 - 8 * lane);
  const uint4 *phi = reinterpret_cast<const uint4 *>(bins + 252 - 8 * lane);
  warp_find_bin_regs(kGlobal ? __ldcg(plo) : *plo, kGlobal ? __ldcg(phi) : *phi, need, bin, above,
                     cnt);
}
__device__ __forceinline__ void warp_find_bin_regs(const uint4 lo, const uint4 hi, int need,
                                                   int &bin, int &above, int &cnt) {
  const int lane = threadIdx.x & 31;
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

// Threshold bucket of one row (the 16-bit key prefix holding the p-th largest
// key) from its two-level histogram: the coarse level and the fine levels of
// the three coarse bins around `guess` are read in one round trip; a guess
// that misses costs a second read.
__device__ __forceinline__ RowThreshold warp_find_bucket(const uint32_t *h, int p, int guess) {
  const int lane = threadIdx.x & 31;
  const int o_lo = 248 - 8 * lane, o_hi = 252 - 8 * lane;
  auto ld = [](const uint32_t *q) { return __ldcg(reinterpret_cast<const uint4 *>(q)); };
  const int g0 = min(max(guess - 1, 0), kHistCoarse - 3);
  const uint32_t *f = h + kHistCoarse + g0 * 256;
  const uint4 clo = ld(h + o_lo), chi = ld(h + o_hi);
  const uint4 f0l = ld(f + o_lo), f0h = ld(f + o_hi);
  const uint4 f1l = ld(f + 256 + o_lo), f1h = ld(f + 256 + o_hi);
  const uint4 f2l = ld(f + 512 + o_lo), f2h = ld(f + 512 + o_hi);
  int cb, above1, cnt1;
  warp_find_bin_regs(clo, chi, p, cb, above1, cnt1);
  uint4 fl, fh;
  const int j = cb - g0;  // warp-uniform
  if (j == 0) {
    fl = f0l;
    fh = f0h;
  } else if (j == 1) {
    fl = f1l;
    fh = f1h;
  } else if (j == 2) {
    fl = f2l;
    fh = f2h;
  } else {
    fl = ld(h + kHistCoarse + cb * 256 + o_lo);
    fh = ld(h + kHistCoarse + cb * 256 + o_hi);
  }
  int fb, above2, cnt2;
  warp_find_bin_regs(fl, fh, p - above1, fb, above2, cnt2);
  RowThreshold t;
  t.prefix = (uint32_t)(cb * 256 + fb);
  t.need = p - above1 - above2;
  t.cnt = cnt2;
  return t;
}

// Large threshold bucket of row r (more keys than the direct rank list holds):
// radix select of the need-th largest key, 8 bits per pass over the 48 key
// bits below the bucket prefix, then a recount of the selected keys per
// 128-cluster chunk. All threads of the block call it; kept out of line so the
// common path does not jump over its code.
template <typename SmemT>
__device__ __noinline__ void fused_radix_row(SmemT &S, const float *row_s, int K, int r, int nch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned long long pre = (unsigned long long)S.thr[r].prefix << 48;
  int need = S.thr[r].need;
  for (int shift = 40; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) S.rhist[i] = 0u;
    __syncthreads();
    const unsigned long long hi_sel = pre >> (shift + 8);
    for (int k = tid; k < K; k += blockDim.x) {
      const unsigned long long key = pack(sanitize(row_s[k]), (uint32_t)k);
      if ((key >> (shift + 8)) == hi_sel) atomicAdd(&S.rhist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      int bin, above, cnt;
      warp_find_bin<false>(S.rhist, need, bin, above, cnt);
      if (lane == 0) {
        S.rsel_bin = bin;
        S.rsel_above = above;
      }
    }
    __syncthreads();
    pre |= (unsigned long long)S.rsel_bin << shift;
    need -= S.rsel_above;
    __syncthreads();  // rsel_* and rhist are reused by the next pass
  }
  if (warp < kFWarps) {
    const float4 *row4 = reinterpret_cast<const float4 *>(row_s);
    for (int ch = warp; ch < nch; ch += kFWarps) {
      const int k0 = (ch << 7) + 4 * lane;
      int cnt = 0;
      if (k0 < K) {
        const float4 v4 = row4[k0 >> 2];
        const float v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) cnt += k0 + u < K && pack(sanitize(v[u]), (uint32_t)(k0 + u)) >= pre;
      }
      cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
      if (lane == 0) S.chunk_sel[r][ch] = cnt;
    }
  }
  if (tid == 0) S.tkey[r] = pre;
  __syncthreads();
}

// Pass A of one row with monotone integer keys (bucket bounds at zero or
// non-finite values, where float order and key order differ): per 128-cluster
// chunk the keys above the bucket, and the bucket's keys. Compute warps only.
template <typename SmemT>
__device__ __noinline__ void fused_pass_a_keys(SmemT &S, const float *row_s, int K, int r, int nch,
                                               uint32_t P, bool want) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t thrA = P >= 0xFFFFu ? 0xFFFFFFFFu : (P + 1u) << 16;
  const uint32_t bktLo = P << 16;
  for (int ch = warp; ch < nch; ch += kFWarps) {
    int cnt = 0;
    for (int u = 0; u < 4; ++u) {
      const int k = (ch << 7) + 4 * lane + u;
      if (k >= K) break;
      const float x = sanitize(row_s[k]);
      const uint32_t m = mono(x);
      cnt += m >= thrA;
      if (want && m - bktLo < 65536u) {
        const int slot = atomicAdd(&S.bkt_n[r], 1);
        if (slot < kBktCap) S.bkt[r][slot] = pack(x, (uint32_t)k);
      }
    }
    cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
    if (lane == 0) S.chunk_sel[r][ch] = cnt;
  }
}

__device__ __forceinline__ const char *wp_bytes(const FusedArgs &a) {
  return reinterpret_cast<const char *>(a.w_perm);
}

// SAMPLE: draws (the sampling calls) instead of greedy ids; a template
// parameter so the greedy instance carries no noise code.
template <typename HT, typename WT, int R, bool SAMPLE>
__global__ void __launch_bounds__(kFBlock, 1) k_fused_step(FusedArgs a) {
  using M1 = typename S1Mma<WT>::T;  // stage-1 mma operand type
  constexpr bool kFp8 = sizeof(WT) == 1;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *ring = smem;
  FusedSmem &S = *reinterpret_cast<FusedSmem *>(smem + kRingBytes);
  float *part1 = reinterpret_cast<float *>(smem + kFSmemBase);  // stage-1 partials
  HT *hB3 = reinterpret_cast<HT *>(smem + kFSmemBase + s1_part_bytes(R));  // [R][D]
  // stage-1 B operand: a swizzled f16 copy for fp8 rows, else the same array
  M1 *hB1 = kFp8 ? reinterpret_cast<M1 *>(reinterpret_cast<unsigned char *>(hB3) + (size_t)R * a.D * 2)
                 : reinterpret_cast<M1 *>(hB3);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool producer = warp == kFWarps;  // TMA issue + tile reductions
  const int G = gridDim.x, b = blockIdx.x;
  const int gq = lane >> 2, tq = lane & 3, odd = gq & 1;  // mma fragment coordinates
  uint32_t phase = 0u;  // compute warps: parity of each slot's next mbarrier completion
  FH_TRACE_INIT()
  FH_STAMP(0);

  // ------------------------------------------------------------------ stage 1
  // slice bounds in 32 bits: the host keeps K <= 128 * G, so b * K < 2^32
  const int c0 = (int)((uint32_t)b * (uint32_t)a.K / (uint32_t)G);
  const int c1 = (int)((uint32_t)(b + 1) * (uint32_t)a.K / (uint32_t)G);
  const int nc = c1 - c0;
  // This CTA's stage-2 items: [lo, hi) of rows * (p + n_special), row-major;
  // row r's selected clusters in id order, then its special tokens.
  const int per_row = a.p + a.n_special;
  const int total = a.rows * per_row;
  // 32-bit bounds: total <= 4 * (4096 + 256) and G <= 1024
  const int lo = (int)((uint32_t)b * (uint32_t)total / (uint32_t)G);
  const int hi = (int)((uint32_t)(b + 1) * (uint32_t)total / (uint32_t)G);
  const int n_items = min(hi - lo, kWorkCap);  // the host keeps hi - lo <= kWorkCap
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
      const int per = max(1, kS1PieceBytes / rb1);  // rows per copy
      for (int r0 = 0; r0 < tr; r0 += per)
        bulk_g2s(dst + (size_t)r0 * rb1, src + (size_t)r0 * rb1,
                 (uint32_t)(min(per, tr - r0) * rb1), &S.mbar[s]);
    } else {
      for (int r = 0; r < tr; ++r)
        bulk_g2s(dst + (size_t)r * g1.pitch, src + (size_t)r * rb1, (uint32_t)cb, &S.mbar[s]);
    }
  };
  // The first copies go out before anything else: producer lane 0 initialises
  // the mbarriers itself; the other threads wait on them only after the block
  // barrier below.
  if (producer && lane == 0) {
    for (int s = 0; s < kMaxSlots; ++s) mbar_init(&S.mbar[s], 1);
    fence_mbar_init();
    for (int c = 0; c < min(g1.n_slots, n1); ++c) issue1(c);
  }
  FH_STAMP_P(15);
  if (tid == 0) {
    S.s_err = 0u;
    S.n_work = 0;
  }
  if (tid < kFMaxRows) {
    S.best[tid] = 0ull;
    S.bkt_n[tid] = 0;
  }
  for (int i = tid; i < kFMaxRows * kHistCoarse; i += kFBlock) S.coarse[i] = 0u;
  // Inputs and workspace may come from the previous kernel in the stream
  // (programmatic dependent launch): wait for it here, after the first
  // weight copies are in flight, and let the next step be scheduled.
  grid_dep_wait();
  grid_dep_launch();
  const uint32_t epoch = __ldcg(&a.sync[kSyncEpoch]);
  unsigned char *buf_cur = a.epoch_bufs + (size_t)(epoch & 1u) * kEpochBufBytes;
  unsigned char *buf_nxt = a.epoch_bufs + (size_t)((epoch + 1u) & 1u) * kEpochBufBytes;
  uint32_t *hist_cur = reinterpret_cast<uint32_t *>(buf_cur);
  if (!producer) {
    if (tid < nc) S.scale[tid] = a.cscale ? a.cscale[c0 + tid] : 1.f;
    // hidden rows as mma B operands (16-bit) in shared memory, 16 bytes per
    // thread and load (one round trip for R * D <= 4096)
    for (int i = tid; i < R * a.D / 8; i += kFThreads) {
      const int e0 = i * 8, r = e0 / a.D, e = e0 - r * a.D;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < a.rows) v = __ldg(reinterpret_cast<const uint4 *>(a.hidden) + i);
      reinterpret_cast<uint4 *>(hB3)[i] = v;
      if constexpr (kFp8) {
        float f[8];
        Vec<HT>::to_float(v, f);
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const __half2 h2 = __floats2half2_rn(f[2 * u], f[2 * u + 1]);
          w[u] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        *reinterpret_cast<uint4 *>(hB1 + (size_t)r * a.D + fp8_hidden_slot(e)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    for (int i = tid; i < n_items; i += kFThreads) S.work[i] = 0xFFFFFFFFu;  // empty until set
    FH_STAMP(16);
  }
  __syncthreads();
  if (tid == 0) S.n_work = n_items;
  FH_STAMP(17);

  FH_TICK_DECL
  if (!producer) {
    // Compute warps: each chunk (a tile, or a d-range of one) into its own
    // partial buffer; a slot is refilled as soon as its chunk is consumed, so
    // the copies never drain between rounds.
    const int hrow = (gq >> 1) < R ? (gq >> 1) : 0;  // hidden row feeding column gq
    const M1 *hrow1 = hB1 + (size_t)hrow * a.D;
    for (int c = 0; c < n1; ++c) {
      const int s = c % g1.n_slots, tile = c / g1.ndc, dc = c - tile * g1.ndc;
      const int cb = min(g1.cb, rb1 - dc * g1.cb);
      FH_TICK(7);
      if (!mbar_wait(&S.mbar[s], (phase >> s) & 1u, a.copy_polls) && lane == 0)
        atomicOr(&S.s_err, kErrCopyTimeout);
      phase ^= 1u << s;
      FH_TICK(0);
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
      const unsigned char *slot = ring + (size_t)s * g1.slot_bytes;
      const int ng = cb / 64;
      const int qbase = dc * (g1.cb / 64);  // first 64-byte group of this chunk in the row
      for (int grp = warp; grp < ng; grp += kFWarps) {
        const int q = grp ^ odd;
        const unsigned char *ra = slot + (size_t)gq * g1.pitch + q * 64 + tq * 16;
        if constexpr (kFp8) {
          const M1 *hg = hrow1 + (size_t)(qbase + q) * 64;
          const int sw = (qbase + q) & 1;
          tile_group<WT, M1>(acc0, acc1, ra, ra + 8 * g1.pitch, hg + (((2 * tq) ^ sw) << 3),
                             hg + (((2 * tq + 1) ^ sw) << 3));
        } else {
          const M1 *hg = hrow1 + (size_t)(qbase + q) * 32 + tq * 8;
          tile_group<WT, M1>(acc0, acc1, ra, ra + 8 * g1.pitch, hg, hg);
        }
      }
      FH_TICK(1);
      // lane (g, t): row g (and g + 8) against hidden row t in c[odd] (c[2 + odd])
      if (tq < R) {
        float *pc = part1 + (size_t)c * (kTileRows * R * kFWarps);
        pc[(gq * R + tq) * kFWarps + warp] = acc0[odd] + acc1[odd];
        pc[((gq + 8) * R + tq) * kFWarps + warp] = acc0[2 + odd] + acc1[2 + odd];
      }
      FH_TICK(2);
      if (c + g1.n_slots < n1) nbar_arrive(kBarSlot0 + s, kFBlock);  // slot s free
    }
  } else {
    // Producer warp: chunk c goes into slot c % n_slots once the chunk before
    // it in that slot has been consumed.
    for (int c = g1.n_slots; c < n1; ++c) {
      nbar_sync(kBarSlot0 + c % g1.n_slots, kFBlock);
      if (lane == 0) issue1(c);
      __syncwarp();
    }
    // Zero this CTA's share of the histograms the next call will use (32-bit
    // bounds: b * n4 < 2^32 for G <= 1024).
    constexpr uint32_t n4 = (uint32_t)(kEpochBufBytes / 16);
    uint4 *z = reinterpret_cast<uint4 *>(buf_nxt);
    const uint32_t z0 = (uint32_t)b * n4 / (uint32_t)G, z1 = (uint32_t)(b + 1) * n4 / (uint32_t)G;
    for (uint32_t i = z0 + lane; i < z1; i += 32) z[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  FH_STAMP(7);
  // Stage-1 scores: one (cluster, hidden row) per thread, summed over the
  // chunks of its tile and the 16 warps.
  for (int qd = tid; qd < nc * R; qd += kFBlock) {
    const int col = qd / nc, kk = qd - col * nc;
    if (col >= a.rows) continue;
    const int tile = kk / kTileRows, row = kk - tile * kTileRows;
    float v = 0.f;
    for (int dc = 0; dc < g1.ndc; ++dc) {
      const float4 *pp = reinterpret_cast<const float4 *>(
          part1 + (size_t)(tile * g1.ndc + dc) * (kTileRows * R * kFWarps) + (row * R + col) * kFWarps);
      const float4 x0 = pp[0], x1 = pp[1], x2 = pp[2], x3 = pp[3];
      v += ((x0.x + x0.y) + (x0.z + x0.w)) + ((x1.x + x1.y) + (x1.z + x1.w)) +
           (((x2.x + x2.y) + (x2.z + x2.w)) + ((x3.x + x3.y) + (x3.z + x3.w)));
    }
    const int k = c0 + kk;
    float sc = v * S.scale[kk];
    if (SAMPLE)
      sc = sc / a.temperature + gumbel(a.rng, kStageClusters, (uint32_t)col, (uint32_t)k);
    S.local[col][kk] = sc;
    a.scores[(size_t)col * a.score_stride + k] = sc;
    const uint32_t key = mono(sanitize(sc));
    atomicAdd(&hist_cur[(size_t)col * kHistWords + kHistCoarse + (key >> 16)], 1u);
    atomicAdd(&S.coarse[col * kHistCoarse + (key >> 24)], 1u);
  }
  __syncthreads();
  for (int i = tid; i < a.rows * kHistCoarse; i += kFBlock) {
    const uint32_t cc = S.coarse[i];
    if (cc) atomicAdd(&hist_cur[(size_t)(i / kHistCoarse) * kHistWords + (i % kHistCoarse)], cc);
  }
  __syncthreads();
  FH_STAMP(1);

  // ------------------------------------------------------------- grid barrier
  if (tid == 0) {
    __threadfence();
    FH_STAMP(8);
    atomicAdd(&a.sync[kSyncArrive], 1u);
  }
  // While the grid meets, the producer warp estimates each row's selection
  // threshold from this CTA's scores (mean + z * std, z the normal quantile
  // of the selection rate minus a margin), used below to guess the histogram
  // bin, and in greedy mode prefetches into L2 the w_perm rows of the
  // clusters above the estimate: HBM would otherwise sit idle through the
  // barrier and the selection, and a wrong guess only costs idle bandwidth.
  if (producer) {
    const size_t cluster_bytes = (size_t)a.cap * a.D * sizeof(HT);
    for (int r = 0; r < a.rows; ++r) {
      float sum = 0.f, sq = 0.f;
      int n = 0;
      for (int i = lane; i < nc; i += 32) {
        const float v = S.local[r][i];
        if (isfinite(v)) {
          sum += v;
          sq += v * v;
          ++n;
        }
      }
      sum = warp_sum(sum);
      sq = warp_sum(sq);
      n = __reduce_add_sync(0xFFFFFFFFu, n);
      const float mean = n > 0 ? sum / n : 0.f;
      const float sd = n > 0 ? sqrtf(fmaxf(sq / n - mean * mean, 0.f)) : 0.f;
      const float frac = fminf(0.5f, (float)a.p / (float)a.K);
      const float z = -normcdfinvf(frac);
      if (lane == 0) S.t_est[r] = mean + z * sd;
      const float t_pf = mean + (z - kPrefetchMargin) * sd;
      if (!SAMPLE && nc > 1 && cluster_bytes % 16 == 0)
        for (int i = lane; i < nc; i += 32)
          if (S.local[r][i] > t_pf)
            bulk_prefetch_l2(wp_bytes(a) + (size_t)(c0 + i) * cluster_bytes, (uint32_t)cluster_bytes);
    }
  }
  if (tid == 0) {
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

  // ---------------------------------------------------------------- select
  // Warps kFMaxRows.. of the compute warps copy the score rows into the ring
  // (stage 1 is done with it) while warp r finds row r's threshold bucket.
  float *sc_s = reinterpret_cast<float *>(ring);  // [rows][Kp]
  const int Kp = (a.K + 3) & ~3;
  if (warp >= kFMaxRows && !producer) {
    const int t0 = tid - kFMaxRows * 32, n4 = Kp / 4;
    constexpr int nt = kFThreads - kFMaxRows * 32;
    for (int r = 0; r < a.rows; ++r) {
      const float4 *src = reinterpret_cast<const float4 *>(a.scores + (size_t)r * a.score_stride);
      float4 *dst = reinterpret_cast<float4 *>(sc_s + (size_t)r * Kp);
      for (int c = t0; c < n4; c += 4 * nt) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c + u * nt < n4) v[u] = __ldcg(src + c + u * nt);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c + u * nt < n4) dst[c + u * nt] = v[u];
      }
    }
  } else if (warp < a.rows) {
    const float te = S.t_est[warp];
    const int guess = isfinite(te) ? (int)(mono(te) >> 24) : kHistCoarse / 2;
    const RowThreshold t = warp_find_bucket(hist_cur + (size_t)warp * kHistWords, a.p, guess);
    if (lane == 0) S.thr[warp] = t;
  }
  __syncthreads();
  FH_STAMP(9);
  // Every cluster of this CTA's slice at or above its row's threshold bucket
  // is (almost surely) selected: the producer warp, idle during the selection,
  // pulls their rows into L2 for whichever CTA processes them.
  if (producer) {
    const size_t cluster_bytes = (size_t)a.cap * a.D * sizeof(HT);
    if (cluster_bytes % 16 == 0)
      for (int r = 0; r < a.rows; ++r) {
        const uint32_t P = S.thr[r].prefix;
        for (int i = lane; i < nc; i += 32)
          if ((mono(sanitize(S.local[r][i])) >> 16) >= P)
            bulk_prefetch_l2(wp_bytes(a) + (size_t)(c0 + i) * cluster_bytes, (uint32_t)cluster_bytes);
      }
  }
  // Pass A: per 128-cluster chunk, the keys above the threshold bucket, and
  // the bucket's keys when any of them is needed. Each warp takes four
  // chunks per pass (loads first). Key order equals float order except at
  // zero and non-finite values, so rows whose bucket bounds are finite and
  // nonzero compare floats; the rest compare the monotone integer keys.
  const int nch = (a.K + 127) >> 7;
  if (!producer) {
    for (int r = 0; r < a.rows; ++r) {
      const uint32_t P = S.thr[r].prefix;
      const uint32_t thrA = P >= 0xFFFFu ? 0xFFFFFFFFu : (P + 1u) << 16;
      const uint32_t bktLo = P << 16;
      const float X = unmono(thrA), Xlo = unmono(bktLo);
      const bool fast = P < 0xFFFFu && isfinite(X) && X != 0.f && isfinite(Xlo) && Xlo != 0.f;
      const bool want = S.thr[r].need > 0;
      const float *row_s = sc_s + r * Kp;
      const float4 *row4 = reinterpret_cast<const float4 *>(row_s);
      if (!fast) {  // zero or non-finite bucket bounds (rare): integer keys, out of line
        fused_pass_a_keys(S, sc_s + r * Kp, a.K, r, nch, P, want);
        continue;
      }
      for (int ch0 = warp; ch0 < nch; ch0 += 4 * kFWarps) {
        float v[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k0 = ((ch0 + j * kFWarps) << 7) + 4 * lane;
          float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
          if (k0 < a.K) v4 = row4[k0 >> 2];
          v[j][0] = v4.x;
          v[j][1] = v4.y;
          v[j][2] = v4.z;
          v[j][3] = v4.w;
        }
        int cnt[4];
        uint32_t inb = 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k0 = ((ch0 + j * kFWarps) << 7) + 4 * lane;
          cnt[j] = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const bool ok = k0 + u < a.K;
            const float x = v[j][u];
            cnt[j] += ok && x >= X;
            inb |= (uint32_t)(ok && x >= Xlo && x < X) << (4 * j + u);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) cnt[j] = __reduce_add_sync(0xFFFFFFFFu, cnt[j]);
        if (lane == 0) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (ch0 + j * kFWarps < nch) S.chunk_sel[r][ch0 + j * kFWarps] = cnt[j];
        }
        if (want && __any_sync(0xFFFFFFFFu, inb != 0u)) {
#pragma unroll 1
          for (uint32_t m = inb; m != 0u; m &= m - 1u) {
            const int bit = __ffs(m) - 1, j = bit >> 2, u = bit & 3;
            const int k = ((ch0 + j * kFWarps) << 7) + 4 * lane + u;
            const int slot = atomicAdd(&S.bkt_n[r], 1);
            if (slot < kBktCap) S.bkt[r][slot] = pack(row_s[k], (uint32_t)k);
          }
        }
      }
    }
  }
  __syncthreads();
  FH_STAMP(12);
  // Large buckets (rare, out of line): exact threshold key and chunk counts.
  for (int r = 0; r < a.rows; ++r) {
    if (S.thr[r].need <= 0 || S.bkt_n[r] <= kBktCap) continue;  // block-uniform
    fused_radix_row(S, sc_s + r * Kp, a.K, r, nch);
  }
  FH_STAMP(13);
  // Warp r, row r: the threshold key (keys above the bucket plus the `need`
  // largest keys of a small bucket: the key of rank need - 1), the bucket
  // winners into their chunks' counts, then the chunks' first positions.
  if (warp < a.rows) {
    const RowThreshold t = S.thr[warp];
    const int n = S.bkt_n[warp];
    if (t.need <= 0 || n <= kBktCap) {
      unsigned long long T =
          t.prefix >= 0xFFFFu ? ~0ull : (unsigned long long)(t.prefix + 1u) << 48;
      if (t.need > 0) {
        T = (unsigned long long)t.prefix << 48;  // fewer keys than needed: the whole bucket
        unsigned long long found = 0ull;
        bool hit = false;
        for (int j = lane; j < n; j += 32) {
          const unsigned long long mine = S.bkt[warp][j];
          int rank = 0;
          for (int m = 0; m < n; ++m) rank += S.bkt[warp][m] > mine;
          if (rank == t.need - 1) {
            found = mine;
            hit = true;
          }
        }
        const unsigned hm = __ballot_sync(0xFFFFFFFFu, hit);
        if (hm) T = __shfl_sync(0xFFFFFFFFu, found, __ffs(hm) - 1);
        for (int j = lane; j < n; j += 32) {
          const unsigned long long key = S.bkt[warp][j];
          if (key >= T) atomicAdd(&S.chunk_sel[warp][(int)(0xFFFFFFFFu - (uint32_t)key) >> 7], 1);
        }
      }
      if (lane == 0) S.tkey[warp] = T;
    }
    __syncwarp();
    const int per = (nch + 31) / 32, j0 = min(nch, lane * per), j1 = min(nch, j0 + per);
    int sum = 0;
    for (int j = j0; j < j1; ++j) sum += S.chunk_sel[warp][j];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int tt = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += tt;
    }
    int off = incl - sum;
    for (int j = j0; j < j1; ++j) {
      S.chunk_off[warp][j] = off;
      off += S.chunk_sel[warp][j];
    }
  }
  __syncthreads();
  FH_STAMP(14);
  // This CTA's items: only the chunks whose positions meet [lo, hi) are walked.
  if (!producer) {
    for (int r = 0; r < a.rows; ++r) {
      const int base = r * per_row;
      const unsigned long long T = S.tkey[r];
      const float4 *row4 = reinterpret_cast<const float4 *>(sc_s + r * Kp);
      for (int ch = warp; ch < nch; ch += kFWarps) {
        const int off = S.chunk_off[r][ch], cnt = S.chunk_sel[r][ch];
        if (cnt == 0 || base + off + cnt <= lo || base + off >= hi || off >= a.p) continue;
        const int k0 = (ch << 7) + 4 * lane;
        bool f[4] = {false, false, false, false};
        if (k0 < a.K) {
          const float4 v4 = row4[k0 >> 2];
          const float v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u)
            f[u] = k0 + u < a.K && pack(sanitize(v[u]), (uint32_t)(k0 + u)) >= T;
        }
        const int c = (int)f[0] + (int)f[1] + (int)f[2] + (int)f[3];
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += t;
        }
        int pos = off + incl - c;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (f[u]) {
            const int idx = base + pos;
            if (pos < a.p && idx >= lo && idx - lo < n_items)
              S.work[idx - lo] = ((uint32_t)r << 28) | (uint32_t)(k0 + u);
            ++pos;
          }
        }
      }
      for (int j = tid; j < a.n_special; j += kFThreads) {
        const int idx = base + a.p + j;
        if (idx >= lo && idx - lo < n_items)
          S.work[idx - lo] = kItemSpecial | ((uint32_t)r << 28) | (uint32_t)j;
      }
    }
  }
  __syncthreads();
  FH_STAMP(10);

  // ------------------------------------------------------------------ stage 2
  const int rb3 = a.D * (int)sizeof(HT);
  const RingGeom g3 = ring_geom(rb3);
  const char *wp = reinterpret_cast<const char *>(a.w_perm);
  // Producer state (producer lane 0 only): next work item and its next d-chunk.
  int p_item = 0, p_dc = 0;
  auto produce = [&](int s) {
    S2Chunk d;
    d.src = -2;
    d.n = 0;
    d.row = 0;
    d.dc = 0;
    d.last = 1;
    d.vid_in_smem = 0;
    if (p_item < S.n_work) {
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
        // the rows as kS2Pieces copies of whole rows (copies proceed in parallel)
        const int per = (d.n + kS2Pieces - 1) / kS2Pieces;
        for (int r0 = 0; r0 < d.n; r0 += per)
          bulk_g2s(dst + (size_t)r0 * rb3, src + (size_t)r0 * rb3,
                   (uint32_t)(min(per, d.n - r0) * rb3), &S.mbar[s]);
      } else {
        for (int r = 0; r < d.n; ++r)
          bulk_g2s(dst + (size_t)r * g3.pitch, src + (size_t)r * rb3, (uint32_t)cb, &S.mbar[s]);
      }
      if (vid_bulk) bulk_g2s(&S.vid[s][0], vsrc, (uint32_t)(d.n * 4), &S.mbar[s]);
    } else {
      S.desc[s] = d;
      mbar_expect_tx(&S.mbar[s], 0u);  // invalid item or end of work: no data
    }
  };
  FH_TICK(7);
  if (!producer) {
    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
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
          tile_group<HT, HT>(acc0, acc1, ra, ra + 8 * g3.pitch, hrow3 + q * 32, hrow3 + q * 32);
        }
      }
      FH_TICK(5);
      if (d.last) {
        // every B column pair holds hidden row d.row: lanes t == 0 carry rows g, g + 8
        const int par = tile & 1;
        if (tile >= 2) nbar_sync(kBarPart0 + par, kFBlock);
        if (tq == 0) {
          S.part[par][gq][0][warp] = acc0[odd] + acc1[odd];
          S.part[par][gq + 8][0][warp] = acc0[2 + odd] + acc1[2 + odd];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) acc0[u] = acc1[u] = 0.f;
        ++tile;
      }
      FH_TICK(6);
      nbar_arrive(kBarSlot0 + s, kFBlock);
    }
    for (int t = max(tile - 2, 0); t < tile; ++t) nbar_sync(kBarPart0 + (t & 1), kFBlock);
  } else {
    int n_prod = 0;  // lane 0: next chunk to produce (chunk i uses slot i % n_slots)
    if (lane == 0)
      while (n_prod < g3.n_slots) produce(n_prod++ % g3.n_slots);
    __syncwarp();
    int tile = 0;
    for (int c = 0;; ++c) {
      const int s = c % g3.n_slots;
      const S2Chunk d = S.desc[s];
      if (d.src == -2) break;
      nbar_sync(kBarSlot0 + s, kFBlock);
      if (d.last) {
        const int par = tile & 1;
        if (d.src >= 0) {
          unsigned long long best = 0ull;
          if (lane < kTileRows) {
            const int row = lane;
            const float4 *pp = reinterpret_cast<const float4 *>(&S.part[par][row][0][0]);
            const float4 x0 = pp[0], x1 = pp[1], x2 = pp[2], x3 = pp[3];
            const float v = ((x0.x + x0.y) + (x0.z + x0.w)) + ((x1.x + x1.y) + (x1.z + x1.w)) +
                            (((x2.x + x2.y) + (x2.z + x2.w)) + ((x3.x + x3.y) + (x3.z + x3.w)));
            if (row < d.n) {
              const uint32_t vid =
                  (uint32_t)(d.vid_in_smem ? S.vid[s][row] : __ldg(&a.vocab_map[d.src + row]));
              float key = v;
              if (SAMPLE)
                key = v / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)d.row, vid);
              best = pack(key, vid);
            }
          }
          best = warp_max_u64(best);
          if (lane == 0 && best > S.best[d.row]) S.best[d.row] = best;
        }
        __syncwarp();
        nbar_arrive(kBarPart0 + par, kFBlock);
        ++tile;
      }
      if (lane == 0) produce(n_prod++ % g3.n_slots);
      __syncwarp();
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
    if (tid == 0) {
      a.sync[kSyncArrive] = 0u;
      a.sync[kSyncDone] = 0u;
      a.sync[kSyncEpoch] = epoch + 1u;
    }
  }
  FH_TRACE_WRITE();
}

}  // namespace fh
