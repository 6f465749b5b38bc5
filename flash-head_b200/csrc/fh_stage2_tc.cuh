// Stage 2 of a batched decode step on the 5th-generation tensor cores,
// cluster-major: every probed cluster's w_perm rows cross HBM once per step,
// however many hidden rows probed it. The reference scores each (row, probe)
// pair separately (src/flash_head/fused.py:119-164, grid (T, P)); the
// packed (logit, vocab id) words and their max reduction follow it
// (fused.py:148-163).
//
//   k_s2_fill      probe lists -> per cluster a bit map of the hidden rows
//                  that probe it (atomicOr).
//   k_s2_tiles     probed clusters -> tiles of 8 clusters (128 w_perm rows,
//                  the MMA's M): an aligned window of 8 consecutive clusters
//                  of which at least kS2WindowMin are probed is one tile,
//                  copied as one 128-row box per k-block; the probed clusters
//                  of the other windows are packed 8 to a tile, one 16-row box
//                  each. Per tile the union of the clusters' rows (the MMA's
//                  N, at most 256) and, per cluster, a bit mask over the union
//                  positions of the rows that probed it.
//   k_s2_tc        persistent, 10 warps; a ring stage holds kps k-blocks (64
//                  elements each; kps = 2 when the ring stays 4 stages deep):
//     warp 0     lane 0 issues the TMA copies of the tile's w_perm rows
//                (128-byte swizzle) and prefetches the next tile's
//                descriptor;
//     warp 1     allocates 512 TMEM columns (two accumulators of 256), lane 0
//                issues tcgen05.mma.kind::f16 (M = 128, N = the tile's padded
//                union, K = 16) per k-block and commits stages and finished
//                accumulators;
//     warps 2-5  gather the union's hidden rows of each k-block with
//                cp.async into the 128-byte-swizzled B operand; each
//                thread's copies arrive on the stage's barrier as they
//                complete (cp.async.mbarrier.arrive), the same barrier the
//                TMA copies complete, and the MMA issuer fences the
//                generic-proxy writes before the tensor core reads them;
//     warps 6-9  epilogue: thread = one w_perm row (TMEM lane); per union
//                column whose row probed this thread's cluster, the logit (or
//                the Gumbel key in sampling mode) packed with the vocab id,
//                the max over the cluster's 16 rows by shuffles, and one
//                atomicMax per (row, cluster) into packed[row]. Accumulators
//                are double-buffered, so the epilogue of tile i overlaps the
//                MMAs of tile i + 1.
// The ring's depth follows the largest union of the step (read from the tile
// builder's meta words), so typical steps keep many stages in flight. The
// last CTA to finish publishes the launch's ids and resets packed[]. Every
// wait is bounded; on a timeout the kernel records kErrCopyTimeout, drains its
// own copies and MMAs (bounded) and frees TMEM before it returns.
#pragma once

#include "fh_s1_tc.cuh"

namespace fh {

constexpr int kS2Threads = 320;
constexpr int kS2Loaders = 128;    // warps 2..5
constexpr int kS2EpiThreads = 128; // warps 6..9
constexpr int kS2Clusters = 8;     // clusters per tile (16 rows each: M = 128)
constexpr int kS2MaxRows = 256;    // hidden rows per launch (union N <= 256)
constexpr int kS2ATile = 128 * 128;  // bytes of the w_perm tile of one k-block
constexpr int kS2MaxStages = 12;
constexpr int kS2SmemMax = 227 * 1024;
constexpr int kS2TileClusters = 64;  // clusters per k_s2_tiles CTA: 8 tiles, one per warp
constexpr int kS2WindowMin = 7;      // probed clusters of 8 that make a window tile
constexpr int kS2MinDeepStages = 4;  // two k-blocks per stage only if the ring keeps this many

struct S2Tile {
  int n_cl;                        // cluster slots in the tile (1..8)
  int n;                           // union rows
  int cl[kS2Clusters];             // local cluster id of slot j, or -1 (unprobed window slot)
  uint32_t mask[kS2Clusters][8];   // bit u: union row u probed cluster j
  unsigned char rows[kS2MaxRows];  // union rows (hidden row within the launch), ascending
  int win;                         // window tile: local id of its first cluster, else -1
  int pad[21];
};
static_assert(sizeof(S2Tile) % 64 == 0, "tile descriptors are whole 64-byte lines");

// meta words: [0] tiles, [1] largest union of any tile
struct S2Meta {
  int n_tiles;
  int n_max;
  int pad[62];
};

// ---------------------------------------------------------------------------
// Index: per cluster a bit map of the hidden rows (of this launch) that probe
// it, 8 words per cluster. Zero on entry (the host clears it per launch).
// ---------------------------------------------------------------------------
constexpr int kS2MaskWords = kS2MaxRows / 32;

__global__ void k_s2_fill(const int32_t *probes, int rows, int p, int K, int base, uint32_t *bm) {
  const int n = rows * p;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int c = probes[i] - base;
    const int r = i / p;
    if (c >= 0 && c < K && r < kS2MaxRows)
      atomicOr(&bm[(size_t)c * kS2MaskWords + (r >> 5)], 1u << (r & 31));
  }
}

// One CTA of 256 threads per kS2TileClusters clusters (8 aligned windows of
// 8): windows with at least window_min probed clusters become window tiles;
// the probed clusters of the other windows (ascending id) are cut into tiles
// of kS2Clusters. At most 8 tiles per CTA, one per warp. Per tile: the union
// of the clusters' row maps, its rows in ascending order (their positions are
// the MMA's N columns), and per cluster a bit mask over those positions,
// built with ballots (lane = position). Tile indices come from one atomic per
// CTA (order across CTAs is irrelevant: the tiles partition the probed
// clusters and their results meet in a max). meta must be zero on entry.
__global__ void __launch_bounds__(256) k_s2_tiles(const uint32_t *bm, int K, int window_min,
                                                  S2Tile *tiles, S2Meta *meta) {
  static_assert(kS2TileClusters == 64 && kS2TileClusters / kS2Clusters == 8, "one tile per warp");
  static_assert(kS2MaskWords == 8, "eight mask words per cluster");
  __shared__ uint32_t s_bm[kS2TileClusters][kS2MaskWords];
  __shared__ int ids[kS2TileClusters];  // local index of the j-th sparse cluster
  __shared__ __align__(16) unsigned char s_rows[8][kS2MaxRows];
  __shared__ int s_base, s_total, s_nmax, s_dense;
  __shared__ unsigned s_wins;  // bit w: window w is a window tile
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * kS2TileClusters;
  grid_dep_wait();    // the bit maps come from the kernel before this one
  grid_dep_launch();  // stage 2 may set up while the tiles are built (it waits for them)
  for (int i = tid; i < kS2TileClusters * kS2MaskWords; i += 256) {
    const int c = c0 + i / kS2MaskWords;
    (&s_bm[0][0])[i] = c < K ? __ldcg(&bm[(size_t)c0 * kS2MaskWords + i]) : 0u;
  }
  if (tid == 0) s_nmax = 0;
  __syncthreads();
  if (warp == 0) {
    // the 64 clusters' probed flags; windows with enough of them; the other
    // windows' probed clusters compacted in id order by two ballots
    bool f[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t any = 0u;
#pragma unroll
      for (int w = 0; w < kS2MaskWords; ++w) any |= s_bm[32 * h + lane][w];
      f[h] = any != 0u;
    }
    const unsigned ma = __ballot_sync(0xFFFFFFFFu, f[0]), mb = __ballot_sync(0xFFFFFFFFu, f[1]);
    const unsigned long long m64 = (unsigned long long)mb << 32 | ma;
    unsigned wins = 0u;
#pragma unroll
    for (int w = 0; w < 8; ++w)
      if (__popcll((m64 >> (8 * w)) & 0xFFull) >= window_min) wins |= 1u << w;
    unsigned long long keep = 0ull;  // clusters of the other windows
#pragma unroll
    for (int w = 0; w < 8; ++w)
      if (!((wins >> w) & 1u)) keep |= 0xFFull << (8 * w);
    const unsigned sa = ma & (unsigned)keep, sb2 = mb & (unsigned)(keep >> 32);
    const bool fa = (sa >> lane) & 1u, fb = (sb2 >> lane) & 1u;
    const unsigned below = (1u << lane) - 1u;
    if (fa) ids[__popc(sa & below)] = lane;
    if (fb) ids[__popc(sa) + __popc(sb2 & below)] = 32 + lane;
    if (lane == 0) {
      s_total = __popc(sa) + __popc(sb2);
      s_wins = wins;
      s_dense = __popc(wins);
    }
  }
  __syncthreads();
  const int total = s_total, n_dense = s_dense;
  const unsigned wins = s_wins;
  const int n_sparse = (total + kS2Clusters - 1) / kS2Clusters;
  const int n_tiles = n_dense + n_sparse;  // <= 8: see the window rule
  if (tid == 0) s_base = n_tiles ? atomicAdd(&meta->n_tiles, n_tiles) : 0;
  __syncthreads();
  const int t = warp;
  if (t < n_tiles) {
    // tiles [0, n_dense): the window tiles in window order; then the sparse tiles
    int win = -1, ncl, lj;
    if (t < n_dense) {
      int w = 0;
      for (int k = 0, seen = 0; k < 8; ++k)
        if ((wins >> k) & 1u) {
          if (seen++ == t) w = k;
        }
      win = 8 * w;
      ncl = kS2Clusters;
      lj = 8 * w + (lane & 7);  // slot j = cluster win + j (probed or not)
    } else {
      const int j0 = (t - n_dense) * kS2Clusters;
      ncl = min(kS2Clusters, total - j0);
      lj = lane < ncl ? ids[j0 + lane] : 0;  // lane j: local index of cluster j
    }
    // union word w on lane w, its set bits' positions before it by a scan
    uint32_t word = 0u;
    for (int j = 0; j < ncl; ++j) {
      const int cj = __shfl_sync(0xFFFFFFFFu, lj, j);
      if (lane < kS2MaskWords) word |= s_bm[cj][lane];
    }
    const int pc = __popc(word);
    int incl = pc;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const int x = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += x;
    }
    const int N = __shfl_sync(0xFFFFFFFFu, incl, 7);
    unsigned char *rows = s_rows[warp];
    // rows in ascending order: lane b places bit b of every union word
#pragma unroll
    for (int w = 0; w < kS2MaskWords; ++w) {
      const uint32_t uw = __shfl_sync(0xFFFFFFFFu, word, w);
      const int before = __shfl_sync(0xFFFFFFFFu, incl - pc, w);
      if ((uw >> lane) & 1u) rows[before + __popc(uw & ((1u << lane) - 1u))] = (unsigned char)(32 * w + lane);
    }
    __syncwarp();
    S2Tile &T = tiles[s_base + t];
    // per cluster and 32 positions: ballot of "the position's row probed it"
#pragma unroll
    for (int w = 0; w < kS2MaskWords; ++w) {
      const int q = 32 * w + lane;
      const int r = q < N ? rows[q] : 0;
#pragma unroll
      for (int j = 0; j < kS2Clusters; ++j) {
        const int cj = __shfl_sync(0xFFFFFFFFu, lj, j);
        const bool hit = q < N && j < ncl && ((s_bm[cj][r >> 5] >> (r & 31)) & 1u);
        const uint32_t bal = __ballot_sync(0xFFFFFFFFu, hit);
        if (lane == j) T.mask[j][w] = bal;
      }
    }
    const uint32_t *rw = reinterpret_cast<const uint32_t *>(rows);
    for (int k = lane; k < kS2MaxRows / 4; k += 32)
      reinterpret_cast<uint32_t *>(T.rows)[k] = 4 * k < N ? rw[k] : 0u;
    if (lane < kS2Clusters) {
      // a window slot whose cluster is unprobed (or past K) keeps cl = -1
      bool live = lane < ncl;
      if (win >= 0) {
        uint32_t any = 0u;
#pragma unroll
        for (int w = 0; w < kS2MaskWords; ++w) any |= s_bm[lj][w];
        live = any != 0u && c0 + lj < K;
      }
      T.cl[lane] = live ? c0 + lj : -1;
    }
    if (lane == 0) {
      T.n_cl = ncl;
      T.n = N;
      T.win = win >= 0 ? c0 + win : -1;
      atomicMax(&s_nmax, N);
    }
  }
  __syncthreads();
  if (tid == 0 && s_nmax > 0) atomicMax(&meta->n_max, s_nmax);
}

// ---------------------------------------------------------------------------
// The tensor-core stage 2.
// ---------------------------------------------------------------------------
struct S2TcArgs {
  const void *hidden;      // [rows, D] (this launch's rows)
  int rows;
  int D;
  int nk;                  // D / 64
  int cap;                 // w_perm rows per cluster (<= 16)
  uint32_t idesc0;         // kind::f16 descriptor without N
  const int32_t *vocab_map;
  const S2Tile *tiles;
  const S2Meta *meta;
  int do_sample;
  float temperature;
  RngKey rng;
  int row_base;            // global row of hidden row 0 (noise stream)
  unsigned long long *packed;  // [rows] (this launch's rows)
  uint32_t *err;
  uint32_t polls;
  uint32_t *done;          // CTAs finished (zero on entry; the last CTA resets it)
  int64_t *out_ids;        // [rows] ids, or null
  long long *out_signed;   // [rows] a shard's signed packed words, or null
};

struct S2TcCtrl {
  __align__(16) S2Tile tile[2];  // the epilogue's copies of its current and previous tile (uint4 stores)
  uint64_t full[kS2MaxStages];   // TMA bytes + one arrival per loader
  uint64_t empty[kS2MaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t s_err;
  int s_last;
};
static_assert(offsetof(S2TcCtrl, tile) % 16 == 0 && sizeof(S2Tile) % 16 == 0,
              "tile copies are 16-byte stores");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// One arrival on bar once every cp.async this thread issued so far has
// completed (the barrier's expected count includes it).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// tm_w: w_perm in 16-row boxes (one cluster); tm_w8: 128-row boxes (a window).
template <bool SAMPLE>
__global__ void __launch_bounds__(kS2Threads, 1)
    k_s2_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w8,
            S2TcArgs a) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  const uint32_t raw = smem_u32(dsm);
  unsigned char *ring = dsm + (((raw + 1023u) & ~1023u) - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  grid_dep_wait();  // the tile list comes from the kernel before this one
  const int n_tiles = __ldcg(&a.meta->n_tiles);
  const int n_max = max(16, (__ldcg(&a.meta->n_max) + 15) & ~15);
  // stage: kps A tiles of 16 KB, then kps B tiles of n_max rows (multiples of 2 KB)
  const size_t kb_bytes = (size_t)kS2ATile + (size_t)n_max * 128;
  const size_t room = (size_t)kS2SmemMax - 1024 - sizeof(S2TcCtrl);
  const int kps = (a.nk % 2 == 0 && room / (2 * kb_bytes) >= kS2MinDeepStages) ? 2 : 1;
  const size_t sb = kps * kb_bytes;
  const uint32_t b_off = (uint32_t)(kps * kS2ATile), b_step = (uint32_t)(n_max * 128);
  const int stages = (int)min((size_t)kS2MaxStages, room / sb);
  const int n_stages = a.nk / kps;  // stages per tile
  S2TcCtrl &S = *reinterpret_cast<S2TcCtrl *>(ring + (size_t)stages * sb);
  const int G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&S.full[s], 1 + kS2Loaders);
      mbar_init(&S.empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&S.acc_full[j], 1);
      mbar_init(&S.acc_empty[j], kS2EpiThreads);
    }
    mbar_init(&S.drain, 1);
    S.s_err = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S.tmem_base)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------ w_perm tiles (TMA)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0u;
      int issued[kS2MaxStages];
      for (int j = 0; j < kS2MaxStages; ++j) issued[j] = -1;
      bool ok = true;
      // descriptor of the tile after the current one, loaded while this one streams
      int nx_ncl = 0, nx_win = -1, nx_cl[kS2Clusters];
      auto fetch = [&](int t) {
        const S2Tile &T = a.tiles[t];
        nx_ncl = min(max(__ldcg(&T.n_cl), 0), kS2Clusters);
        nx_win = __ldcg(&T.win);
#pragma unroll
        for (int j = 0; j < kS2Clusters; ++j) nx_cl[j] = __ldcg(&T.cl[j]);
      };
      if (blockIdx.x < n_tiles) fetch(blockIdx.x);
      for (int t = blockIdx.x; t < n_tiles && ok; t += G) {
        const int ncl = nx_ncl, win = nx_win;
        int cl[kS2Clusters];
#pragma unroll
        for (int j = 0; j < kS2Clusters; ++j) cl[j] = nx_cl[j];
        if (t + G < n_tiles) fetch(t + G);
        // a window tile is one 128-row box per k-block; otherwise one 16-row
        // box per probed cluster
        const uint32_t kb_tx = win >= 0 ? (uint32_t)kS2ATile : (uint32_t)(ncl * 16 * 128);
        for (int sg = 0; sg < n_stages; ++sg) {
          if (!mbar_wait(&S.empty[s], ph ^ 1u, a.polls)) {
            atomicOr(&S.s_err, kErrCopyTimeout);
            ok = false;
            break;
          }
          unsigned char *st = ring + (size_t)s * sb;
          mbar_expect_tx(&S.full[s], kb_tx * (uint32_t)kps);
          for (int k = 0; k < kps; ++k) {
            const int x = (sg * kps + k) * 64;
            unsigned char *at = st + k * kS2ATile;
            if (win >= 0) {
              tma_load_2d(at, &tm_w8, x, win * a.cap, &S.full[s]);
            } else {
#pragma unroll
              for (int j = 0; j < kS2Clusters; ++j)
                if (j < ncl) tma_load_2d(at + j * 16 * 128, &tm_w, x, cl[j] * a.cap, &S.full[s]);
            }
          }
          issued[s] = (int)ph;
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      for (int j = 0; j < stages; ++j)
        if (issued[j] >= 0 && !mbar_wait(&S.full[j], (uint32_t)issued[j], a.polls))
          atomicOr(&S.s_err, kErrCopyTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0u;
      bool ok = true;
      int i = 0;
      int n_next = blockIdx.x < n_tiles ? __ldcg(&a.tiles[blockIdx.x].n) : 0;
      for (int t = blockIdx.x; t < n_tiles && ok; t += G, ++i) {
        const int buf = i & 1, use = i >> 1;
        const int n_pad = max(16, (min(n_next, kS2MaxRows) + 15) & ~15);
        if (t + G < n_tiles) n_next = __ldcg(&a.tiles[t + G].n);  // in flight during this tile
        const uint32_t idesc = a.idesc0 | ((uint32_t)(n_pad >> 3) << 17);
        if (use > 0) {
          if (!mbar_wait(&S.acc_empty[buf], (uint32_t)((use - 1) & 1), a.polls)) {
            atomicOr(&S.s_err, kErrCopyTimeout);
            break;
          }
          tc_fence_after();
        }
        const uint32_t acc = tmem + (uint32_t)(buf * 256);
        for (int sg = 0; sg < n_stages; ++sg) {
          if (!mbar_wait(&S.full[s], ph, a.polls)) {
            atomicOr(&S.s_err, kErrCopyTimeout);
            ok = false;
            break;
          }
          // the gathered hidden rows were written through the generic proxy
          // (cp.async); the tensor core reads them through the async proxy
          fence_proxy_async_smem();
          tc_fence_after();
          const uint32_t st = smem_u32(ring + (size_t)s * sb);
          for (int k = 0; k < kps; ++k) {
            const uint64_t ad = umma_desc_k(st + (uint32_t)(k * kS2ATile));
            const uint64_t bd = umma_desc_k(st + b_off + (uint32_t)k * b_step);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_f16(acc, ad + 2u * kk, bd + 2u * kk, idesc, (sg | k | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&S.empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&S.acc_full[buf]);
      }
      tc_commit(&S.drain);
      if (!mbar_wait(&S.drain, 0u, a.polls)) atomicOr(&S.s_err, kErrCopyTimeout);
    }
  } else if (warp < 6) {
    // ------------------------------------------------ hidden rows (cp.async)
    // stage g of this CTA's sequence uses ring slot g % stages; each loader's
    // copies of it arrive on the slot's barrier when they complete, so the
    // loaders never wait for their own copies.
    const int lt = tid - 64;
    const char *hs = reinterpret_cast<const char *>(a.hidden);
    const size_t rb = (size_t)a.D * 2;
    int s = 0;
    uint32_t ph = 0u;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += G) {
      const S2Tile &T = a.tiles[t];
      const int n = min(max(__ldcg(&T.n), 0), kS2MaxRows);
      const int n_pad = max(16, (n + 15) & ~15);
      const int per = n_pad / 16;  // 16-byte chunks per thread and k-block (<= 16)
      // chunk i of this thread: union row u = (lt + 128 i) / 8, 16-byte chunk c
      const int c = lt & 7;
      const char *src[16];
      uint32_t dst_off[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int u = (lt + kS2Loaders * i) >> 3;
        const int row = u < n ? min((int)__ldcg(&T.rows[u]), a.rows - 1) : 0;
        src[i] = hs + (size_t)row * rb + c * 16;
        dst_off[i] = (uint32_t)(u * 128 + ((c ^ (u & 7)) << 4)) | (u < n ? 0u : 0x80000000u);
      }
      for (int sg = 0; sg < n_stages; ++sg) {
        if (!mbar_wait(&S.empty[s], ph ^ 1u, a.polls)) {
          atomicOr(&S.s_err, kErrCopyTimeout);
          ok = false;
          break;
        }
        for (int k = 0; k < kps; ++k) {
          const uint32_t bst = smem_u32(ring + (size_t)s * sb) + b_off + (uint32_t)k * b_step;
          const size_t x = (size_t)(sg * kps + k) * 128;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (i < per)
              cp_async16(bst + (dst_off[i] & 0x7FFFFFFFu), src[i] + x,
                         (dst_off[i] >> 31) ? 0u : 16u);
        }
        cp_async_arrive_noinc(&S.full[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    cp_async_wait<0>();  // no copy of this thread is in flight when the CTA exits
  } else {
    // ------------------------------------------------ epilogue
    const int q = warp & 3;       // TMEM lane quadrant
    const int m = 32 * q + lane;  // w_perm row of the tile
    const int j = m >> 4, tok = m & 15;
    bool ok = true;
    int i = 0;
    const int et = tid - 192;  // epilogue thread 0..127
    for (int t = blockIdx.x; t < n_tiles; t += G, ++i) {
      const int buf = i & 1, use = i >> 1;
      // the tile's descriptor into shared memory in one round trip (the
      // loop below reads it per column); the barrier also orders this copy
      // after every epilogue warp finished the tile two back
      {
        const uint4 *src = reinterpret_cast<const uint4 *>(&a.tiles[t]);
        uint4 *dst = reinterpret_cast<uint4 *>(&S.tile[buf]);
        for (int k = et; k < (int)(sizeof(S2Tile) / 16); k += kS2EpiThreads) dst[k] = __ldcg(src + k);
        nbar_sync(1, kS2EpiThreads);
      }
      const S2Tile &T = S.tile[buf];
      const int ncl = min(max(T.n_cl, 0), kS2Clusters);
      const int n = min(max(T.n, 0), kS2MaxRows);
      const int cj = j < ncl ? T.cl[j] : -1;
      const bool valid = cj >= 0 && tok < a.cap;
      const uint32_t vid = valid ? (uint32_t)__ldg(&a.vocab_map[cj * a.cap + tok]) : 0u;
      if (ok && !mbar_wait(&S.acc_full[buf], (uint32_t)(use & 1), a.polls)) {
        atomicOr(&S.s_err, kErrCopyTimeout);
        ok = false;
      }
      __syncwarp();
      if (ok) {
        tc_fence_after();
        const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * 256);
        for (int w = 0; w * 32 < n; ++w) {
          // this lane's cluster mask word, and the warp's (both clusters)
          const uint32_t mine = j < ncl ? T.mask[j][w] : 0u;
          const uint32_t both = mine | __shfl_xor_sync(0xFFFFFFFFu, mine, 16);
          if (both == 0u) continue;  // warp-uniform
          uint32_t v[2][16];
          tc_ld16(base + (uint32_t)(32 * w), v[0]);
          tc_ld16(base + (uint32_t)(32 * w + 16), v[1]);
          tc_wait_ld();
#pragma unroll
          for (int b = 0; b < 32; ++b) {
            if (!((both >> b) & 1u)) continue;  // warp-uniform
            const bool take = valid && ((mine >> b) & 1u);
            const int row = take ? (int)T.rows[32 * w + b] : 0;
            unsigned long long key = 0ull;
            if (take) {
              float x = sanitize(__uint_as_float(v[b >> 4][b & 15]));
              if (SAMPLE)
                x = x / a.temperature +
                    gumbel(a.rng, kStageTokens, (uint32_t)(a.row_base + row), vid);
              key = pack(x, vid);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
              const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, key, o);
              key = other > key ? other : key;
            }
            if ((lane & 15) == 0 && key && ((mine >> b) & 1u)) {
              const int r2 = T.rows[32 * w + b];
              atomicMax(&a.packed[r2], key);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cta(&S.acc_empty[buf]);
    }
  }
  grid_dep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
  if (tid == 0 && S.s_err) atomicOr(a.err, S.s_err);
  // Publish: the last CTA to finish turns packed[] into ids (or a shard's
  // signed words) and resets it and the counter for the next launch.
  if (tid == 0) {
    __threadfence();
    S.s_last = atomicAdd(a.done, 1u) == (uint32_t)G - 1u;
  }
  __syncthreads();
  if (S.s_last) {
    __threadfence();
    for (int i = tid; i < a.rows; i += kS2Threads) {
      const unsigned long long w = __ldcg(&a.packed[i]);
      if (a.out_signed) a.out_signed[i] = to_signed(w);
      else if (a.out_ids) a.out_ids[i] = w ? (int64_t)packed_id(w) : (int64_t)0xFFFFFFFFll;
      a.packed[i] = 0ull;
    }
    if (tid == 0) *a.done = 0u;
  }
}

}  // namespace fh
