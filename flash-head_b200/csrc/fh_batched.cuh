// Batched decode steps (rows >= kBatchMinRows): the kernels around the
// tensor-core stage 1 (fh_s1_tc.cuh).
//
//   k_select_hist     per row: the stage-1 keys from the split partials
//                     (sum, fp8 row scale, and in sampling mode / T +
//                     Gumbel(stage 1, r, k): the keys the one-kernel and
//                     three-kernel paths compute), then the top-p clusters.
//   k_inv_*           inverted index: for every probed cluster the rows that
//                     probed it, cut into items of up to kInvRows rows.
//   k_stage2_inv      persistent: every item streams its cluster's w_perm rows
//                     (one bulk copy when the cluster fits a slot) and its
//                     hidden rows into shared memory, scores them on the
//                     tensor cores (mma.m16n8k16: 16 tokens x 4 rows x 2
//                     parities per column set, two column sets per item, so
//                     each row fragment serves 8 rows), and folds each row's
//                     best (logit or Gumbel key, vocab id) into packed[row].
//                     A cluster is read from HBM once per step however many
//                     rows probed it; stage-2 HBM bytes are the distinct
//                     probed clusters, as the roofline counts them.
//   k_special_scores  the special tokens of every row into packed[row].
//   k_inv_finalize    ids from packed[], then packed[] reset.
#pragma once

#include "fh_fused.cuh"

namespace fh {

// From 16 rows; 5..15 rows take the three-kernel path, which streams each
// row's clusters with more memory-level parallelism at that size.
constexpr int kBatchMinRows = 16;
// From this many rows (below kBatchMinRows) the three-kernel path scores
// stage 1 with the tensor-core kernel k_s1_tc + k_select_hist instead of the
// CUDA-core k_scores + k_select.
#ifndef FH_GEMM_S1_MIN_ROWS
#define FH_GEMM_S1_MIN_ROWS 5
#endif
constexpr int kGemmS1MinRows = FH_GEMM_S1_MIN_ROWS;
static_assert(kGemmS1MinRows <= kBatchMinRows, "GEMM stage 1 covers the batched steps");
constexpr int kInvRows = 8;          // hidden rows per item (two mma column sets)
constexpr int kInvThreads = kFThreads;
constexpr int kInvBlock = kFBlock;   // + producer / reducer warp
constexpr int kInvSlots = 2;
constexpr int kInvChunk = 4096;      // max bytes of a row per chunk
// slot: 16 cluster rows + kInvRows hidden rows of one chunk
constexpr int kInvSlotBytes = (kTileRows + kInvRows) * kInvChunk;
constexpr int kInvPrefetch = 32;     // item descriptors fetched per producer round
constexpr int kInvAhead = 4;         // items ahead whose cluster is prefetched into L2

struct InvItem {
  int cluster;  // stage-2 cluster id
  int n;        // rows in this item (1..kInvRows)
  int rows[kInvRows];
  int pad[6];
};
static_assert(sizeof(InvItem) == 64, "item descriptor is one 64-byte line");

// ---------------------------------------------------------------------------
// Top-p clusters of one row per CTA (1024 threads): the same rule as k_select
// (the p largest (score, -id) keys, ids ascending) found with two 8-bit
// histogram levels over the monotone key (bf16 resolution), an exact rank of
// the threshold bucket's few keys (a radix select over the remaining 48 key
// bits when the bucket is large), and one ordered compaction.
// Dynamic shared memory: K floats (the row) + 32 warp histograms of 256 bins.
// ---------------------------------------------------------------------------
constexpr int kHSelThreads = 1024;
constexpr int kHSelWarps = kHSelThreads / 32;
constexpr int kHSelBkt = 256;  // bucket keys ranked directly

struct HSelSmem {
  __align__(16) uint32_t hist[256];
  unsigned long long bkt[kHSelBkt];
  int n_bkt;
  int bin, above, cnt;
  unsigned long long T;
  int warp_counts[kHSelWarps];
};

__host__ __device__ __forceinline__ size_t hsel_row_bytes(int K) {
  return ((size_t)K * sizeof(float) + 15) / 16 * 16;
}
__host__ __device__ __forceinline__ size_t hsel_smem_bytes(int K) {
  return hsel_row_bytes(K) + (size_t)kHSelWarps * 256 * sizeof(uint32_t) + sizeof(HSelSmem);
}

struct HSelArgs {
  const float *part;     // stage-1 partial dot products:
  size_t split_stride;   //   part[s * split_stride + r * row_stride + k], s < splits,
  int row_stride;        //   summed in split order
  int splits;
  int K;
  int p;
  const float *scale;    // [K] fp8 row scale, or null
  int do_sample;         // keys: score / T + Gumbel(stage 1, row, global cluster id)
  float temperature;
  RngKey rng;
  int cluster_base;      // global id of cluster 0 (noise, candidate words)
  float *scores_out;     // [rows, out_stride] the keys as ranked, or null
  int out_stride;
  int32_t *probes;       // [rows, p] local cluster ids ascending, or null
  long long *cand_out;   // [rows, p] signed packed (key, global id) words, or null
};

__global__ void __launch_bounds__(kHSelThreads) k_select_hist(HSelArgs a) {
  extern __shared__ __align__(16) unsigned char hsm[];
  const int K = a.K, p = a.p;
  float *sc = reinterpret_cast<float *>(hsm);
  uint32_t *wh = reinterpret_cast<uint32_t *>(hsm + hsel_row_bytes(K));  // [32][256]
  HSelSmem &S = *reinterpret_cast<HSelSmem *>(hsm + hsel_row_bytes(K) +
                                              (size_t)kHSelWarps * 256 * sizeof(uint32_t));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.x;
  for (int i = tid; i < kHSelWarps * 256; i += kHSelThreads) wh[i] = 0u;
  if (tid < 256) S.hist[tid] = 0u;
  if (tid == 0) S.n_bkt = 0;
  grid_dep_wait();  // the partials come from the stage-1 kernel before this one
  grid_dep_launch();
  const float *row = a.part + (size_t)r * a.row_stride;
  for (int k = tid; k < K; k += kHSelThreads) {
    float v = __ldcg(&row[k]);
    for (int s = 1; s < a.splits; ++s) v += __ldcg(&row[(size_t)s * a.split_stride + k]);
    if (a.scale) v *= __ldg(&a.scale[k]);
    if (a.do_sample)
      v = v / a.temperature +
          gumbel(a.rng, kStageClusters, (uint32_t)r, (uint32_t)(a.cluster_base + k));
    if (a.scores_out) a.scores_out[(size_t)r * a.out_stride + k] = v;
    sc[k] = sanitize(v);
  }
  __syncthreads();
  // level 1: coarse bins (key >> 24), one private histogram per warp
  for (int k = tid; k < K; k += kHSelThreads) atomicAdd(&wh[warp * 256 + (mono(sc[k]) >> 24)], 1u);
  __syncthreads();
  if (tid < 256) {
    uint32_t t = 0;
    for (int w = 0; w < kHSelWarps; ++w) t += wh[w * 256 + tid];
    S.hist[tid] = t;
  }
  __syncthreads();
  if (warp == 0) {
    int b, above, cnt;
    warp_find_bin<false>(S.hist, p, b, above, cnt);
    if (lane == 0) {
      S.bin = b;
      S.above = above;
    }
  }
  __syncthreads();
  const uint32_t cb = (uint32_t)S.bin;
  const int above1 = S.above;
  if (tid < 256) S.hist[tid] = 0u;
  __syncthreads();
  // level 2: fine bins ((key >> 16) & 255) of the coarse bin
  for (int k = tid; k < K; k += kHSelThreads) {
    const uint32_t m = mono(sc[k]);
    if ((m >> 24) == cb) atomicAdd(&S.hist[(m >> 16) & 255u], 1u);
  }
  __syncthreads();
  if (warp == 0) {
    int b, above, cnt;
    warp_find_bin<false>(S.hist, p - above1, b, above, cnt);
    if (lane == 0) {
      S.bin = b;
      S.above = above;
      S.cnt = cnt;
    }
  }
  __syncthreads();
  const uint32_t P = (cb << 8) | (uint32_t)S.bin;  // 16-bit bucket prefix
  const int need = p - above1 - S.above;
  // bucket keys
  if (need > 0)
    for (int k = tid; k < K; k += kHSelThreads) {
      const float v = sc[k];
      if ((mono(v) >> 16) == P) {
        const int m = atomicAdd(&S.n_bkt, 1);
        if (m < kHSelBkt) S.bkt[m] = pack(v, (uint32_t)k);
      }
    }
  __syncthreads();
  const int nb = S.n_bkt;
  if (need <= 0) {
    if (tid == 0) S.T = P >= 0xFFFFu ? ~0ull : (unsigned long long)(P + 1u) << 48;
  } else if (nb <= kHSelBkt) {
    if (tid == 0) S.T = (unsigned long long)P << 48;  // fewer keys than needed: the whole bucket
    __syncthreads();
    for (int j = tid; j < nb; j += kHSelThreads) {
      const unsigned long long mine = S.bkt[j];
      int rank = 0;
      for (int m = 0; m < nb; ++m) rank += S.bkt[m] > mine;
      if (rank == need - 1) S.T = mine;
    }
  } else {
    // large bucket: radix select of the need-th largest key over the low 48 bits
    unsigned long long pre = (unsigned long long)P << 48;
    int nd = need;
    for (int shift = 40; shift >= 0; shift -= 8) {
      if (tid < 256) S.hist[tid] = 0u;
      __syncthreads();
      const unsigned long long hi_sel = pre >> (shift + 8);
      for (int k = tid; k < K; k += kHSelThreads) {
        const unsigned long long key = pack(sc[k], (uint32_t)k);
        if ((key >> (shift + 8)) == hi_sel) atomicAdd(&S.hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        int b, above, cnt;
        warp_find_bin<false>(S.hist, nd, b, above, cnt);
        if (lane == 0) {
          S.bin = b;
          S.above = above;
        }
      }
      __syncthreads();
      pre |= (unsigned long long)S.bin << shift;
      nd -= S.above;
      __syncthreads();
    }
    if (tid == 0) S.T = pre;
  }
  __syncthreads();
  const unsigned long long T = S.T;
  int32_t *out = a.probes ? a.probes + (size_t)r * p : nullptr;
  long long *cand = a.cand_out ? a.cand_out + (size_t)r * p : nullptr;
  block_ordered_compact(
      K, [&](int k) { return pack(sc[k], (uint32_t)k) >= T; },
      [&](int pos, int k) {
        if (pos < p) {
          if (out) out[pos] = k;
          if (cand) cand[pos] = to_signed(pack(sc[k], (uint32_t)(a.cluster_base + k)));
        }
      },
      S.warp_counts);
}

// ---------------------------------------------------------------------------
// Inverted index.
// ---------------------------------------------------------------------------
// Probe lists hold cluster ids starting at `base` (a tensor-parallel shard's
// first global id, else 0); ids outside [base, base + K) are not this head's
// and are skipped.
__global__ void k_inv_count(const int32_t *probes, int rows, int p, int K, int base, int *cnt) {
  const int n = rows * p;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int c = probes[i] - base;
    if (c >= 0 && c < K) atomicAdd(&cnt[c], 1);
  }
}

// One CTA of 1024 threads: off[c] = sum of cnt before c, item_off[c] = sum
// of ceil(cnt / kInvRows) before c, cursor[c] = 0, meta[0] = number of items.
// Dynamic shared memory: K ints. Thread t scans the contiguous counts
// [t * per, (t + 1) * per); thread totals meet in a two-level warp scan.
__global__ void __launch_bounds__(1024) k_inv_build(const int *cnt, int K, int *off, int *item_off,
                                                    int *cursor, int *meta) {
  extern __shared__ int s_cnt[];
  __shared__ int warp_a[32], warp_b[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int c = tid; c < K; c += blockDim.x) s_cnt[c] = __ldcg(&cnt[c]);
  __syncthreads();
  const int per = (K + blockDim.x - 1) / blockDim.x;
  const int c0 = min(K, tid * per), c1 = min(K, c0 + per);
  int sa = 0, sb = 0;
  for (int c = c0; c < c1; ++c) {
    sa += s_cnt[c];
    sb += (s_cnt[c] + kInvRows - 1) / kInvRows;
  }
  int ia = sa, ib = sb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xFFFFFFFFu, ia, o), tb = __shfl_up_sync(0xFFFFFFFFu, ib, o);
    if (lane >= o) {
      ia += ta;
      ib += tb;
    }
  }
  if (lane == 31) {
    warp_a[warp] = ia;
    warp_b[warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int wa = lane < nw ? warp_a[lane] : 0, wb = lane < nw ? warp_b[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xFFFFFFFFu, wa, o), tb = __shfl_up_sync(0xFFFFFFFFu, wb, o);
      if (lane >= o) {
        wa += ta;
        wb += tb;
      }
    }
    if (lane < nw) {  // exclusive warp offsets
      warp_a[lane] = wa - (lane < nw ? warp_a[lane] : 0);
      warp_b[lane] = wb - (lane < nw ? warp_b[lane] : 0);
    }
    if (lane == nw - 1) meta[0] = wb;
  }
  __syncthreads();
  int oa = warp_a[warp] + ia - sa, ob = warp_b[warp] + ib - sb;
  for (int c = c0; c < c1; ++c) {
    const int v = s_cnt[c];
    off[c] = oa;
    item_off[c] = ob;
    cursor[c] = 0;
    oa += v;
    ob += (v + kInvRows - 1) / kInvRows;
  }
}

__global__ void k_inv_scatter(const int32_t *probes, int rows, int p, int K, int base,
                              const int *off, int *cursor, int *list) {
  const int n = rows * p;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int c = probes[i] - base;
    if (c >= 0 && c < K) list[off[c] + atomicAdd(&cursor[c], 1)] = i / p;
  }
}

// Item g of cluster c: rows list[off[c] + g * kInvRows ...].
__global__ void k_inv_items(const int *cnt, const int *off, const int *item_off, const int *list,
                            int K, InvItem *items) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < K; c += gridDim.x * blockDim.x) {
    const int n = cnt[c];
    for (int g = 0; g * kInvRows < n; ++g) {
      InvItem it;
      it.cluster = c;
      it.n = min(kInvRows, n - g * kInvRows);
#pragma unroll
      for (int j = 0; j < kInvRows; ++j)
        it.rows[j] = j < it.n ? list[off[c] + g * kInvRows + j] : 0;
#pragma unroll
      for (int j = 0; j < 6; ++j) it.pad[j] = 0;
      items[item_off[c] + g] = it;
    }
  }
}

// ---------------------------------------------------------------------------
// Stage 2 over the inverted index.
// ---------------------------------------------------------------------------
struct InvArgs {
  const void *hidden;  // [rows, D]
  int rows;
  int D;
  const void *w_perm;  // [K * cap, D]
  const int32_t *vocab_map;
  int K;
  int cap;
  const InvItem *items;
  const int *meta;     // meta[0] = number of items
  int do_sample;
  float temperature;
  RngKey rng;
  unsigned long long *packed;  // [rows]
  uint32_t *err;               // error bits (copy timeout)
  uint32_t copy_polls;
};

struct InvChunk {
  int cluster;  // -1: end of work; -2: invalid item (no data, no result)
  int n;        // hidden rows
  int rows[kInvRows];
  int dc;
  int last;
  int vid_in_smem;
};

struct InvSmem {
  uint64_t mbar[kInvSlots];
  __align__(16) float part[2][kInvRows][kTileRows][kFWarps];
  __align__(16) int vid[kInvSlots][kTileRows];
  InvChunk desc[kInvSlots];
  __align__(16) InvItem pre[kInvPrefetch];
  uint32_t s_err;
};

constexpr size_t kInvSmemBytes = (size_t)kInvSlots * kInvSlotBytes + sizeof(InvSmem);

template <typename HT>
__global__ void __launch_bounds__(kInvBlock, 1) k_stage2_inv(InvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *ring = smem;
  InvSmem &S = *reinterpret_cast<InvSmem *>(smem + (size_t)kInvSlots * kInvSlotBytes);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool producer = warp == kFWarps;
  const int gq = lane >> 2, tq = lane & 3, odd = gq & 1;
  if (tid == 0) {
    for (int s = 0; s < kInvSlots; ++s) mbar_init(&S.mbar[s], 1);
    fence_mbar_init();
    S.s_err = 0u;
  }
  __syncthreads();

  const int n_items = __ldg(&a.meta[0]);
  const int G = gridDim.x, b = blockIdx.x;
  const int i0 = (int)((long long)b * n_items / G), i1 = (int)((long long)(b + 1) * n_items / G);
  const int rb = a.D * (int)sizeof(HT);
  const int cb_max = rb < kInvChunk ? rb : kInvChunk;
  const int ndc = (rb + cb_max - 1) / cb_max;
  const int pitch = ndc == 1 ? rb : cb_max;  // cluster rows in a slot
  const char *wp = reinterpret_cast<const char *>(a.w_perm);
  const char *hs = reinterpret_cast<const char *>(a.hidden);

  if (producer) {
    // Warp-uniform producer state; lane 0 issues the copies. Item descriptors
    // are fetched kInvPrefetch at a time into shared memory by the warp.
    int item = i0, dc = 0, pre_base = i0 - kInvPrefetch;
    auto produce = [&](int s) {
      InvChunk d;
      d.cluster = -1;
      d.n = 0;
      d.dc = 0;
      d.last = 1;
      d.vid_in_smem = 0;
      if (item < i1) {
        if (item >= pre_base + kInvPrefetch) {  // warp-uniform
          pre_base = item;
          __syncwarp();
          for (int j = lane; j < kInvPrefetch && item + j < i1; j += 32) S.pre[j] = a.items[item + j];
          __syncwarp();
        }
        const InvItem &it = S.pre[item - pre_base];
        d.cluster = it.cluster;
        d.n = max(0, min(it.n, kInvRows));
        for (int j = 0; j < kInvRows; ++j) d.rows[j] = it.rows[j];
        d.dc = dc;
        d.last = dc == ndc - 1;
        if (d.last) {
          ++item;
          dc = 0;
        } else {
          ++dc;
        }
      }
      const bool valid = d.cluster >= 0 && d.cluster < a.K;
      if (!valid && d.cluster != -1) {
        d.cluster = -2;
        d.n = 0;
      }
      if (lane != 0) return;
      if (valid) {
        const int cb = min(cb_max, rb - d.dc * cb_max);
        const int src = d.cluster * a.cap;
        const int *vsrc = a.vocab_map + src;
        const bool vid_bulk =
            d.last && ((reinterpret_cast<uintptr_t>(vsrc) & 15u) == 0) && (a.cap % 4 == 0);
        d.vid_in_smem = vid_bulk ? 1 : 0;
        S.desc[s] = d;
        fence_proxy_async_smem();
        uint32_t bytes = (uint32_t)(a.cap * cb + d.n * cb) + (vid_bulk ? (uint32_t)(a.cap * 4) : 0u);
        mbar_expect_tx(&S.mbar[s], bytes);
        unsigned char *dst = ring + (size_t)s * kInvSlotBytes;
        const char *wsrc = wp + (size_t)src * rb + (size_t)d.dc * cb_max;
        if (ndc == 1) {
          const int per = (a.cap + kS2Pieces - 1) / kS2Pieces;  // rows per bulk copy
          for (int r0 = 0; r0 < a.cap; r0 += per)
            bulk_g2s(dst + (size_t)r0 * rb, wsrc + (size_t)r0 * rb,
                     (uint32_t)(min(per, a.cap - r0) * rb), &S.mbar[s]);
        } else {
          for (int r = 0; r < a.cap; ++r)
            bulk_g2s(dst + (size_t)r * pitch, wsrc + (size_t)r * rb, (uint32_t)cb, &S.mbar[s]);
        }
        unsigned char *hdst = dst + (size_t)kTileRows * pitch;
#pragma unroll
        for (int j = 0; j < kInvRows; ++j) {
          if (j < d.n) {
            const int row = min(max(d.rows[j], 0), a.rows - 1);
            bulk_g2s(hdst + (size_t)j * cb_max, hs + (size_t)row * rb + (size_t)d.dc * cb_max,
                     (uint32_t)cb, &S.mbar[s]);
          }
        }
        if (vid_bulk) bulk_g2s(&S.vid[s][0], vsrc, (uint32_t)(a.cap * 4), &S.mbar[s]);
      } else {
        S.desc[s] = d;
        mbar_expect_tx(&S.mbar[s], 0u);  // end of work or invalid item: no data
      }
    };
    int n_prod = 0;
    while (n_prod < kInvSlots) produce(n_prod++ % kInvSlots);
    __syncwarp();
    int tile = 0;
    for (int c = 0;; ++c) {
      const int s = c % kInvSlots;
      const InvChunk d = S.desc[s];
      if (d.cluster == -1) break;
      nbar_sync(kBarSlot0 + s, kInvBlock);
      // lane: hidden row h = lane >> 2, tokens 4 * (lane & 3) .. + 3; their
      // vocab ids are read before the slot is refilled
      const int h = lane >> 2, t0 = 4 * (lane & 3);
      int row_h = 0;  // d.rows[h], selected in registers
#pragma unroll
      for (int j = 0; j < kInvRows; ++j) row_h = j == h ? d.rows[j] : row_h;
      uint32_t vids[4] = {0u, 0u, 0u, 0u};
      if (d.last && d.cluster >= 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (t0 + u < a.cap)
            vids[u] = (uint32_t)(d.vid_in_smem ? S.vid[s][t0 + u]
                                               : __ldg(&a.vocab_map[d.cluster * a.cap + t0 + u]));
      }
      __syncwarp();
      // refill the slot first (the reduction below reads only partials), and
      // pull a later item's cluster into L2 so the refill after it hits L2
      produce(n_prod++ % kInvSlots);
      __syncwarp();
      if (lane == 0 && item + kInvAhead < i1 && item + kInvAhead < pre_base + kInvPrefetch) {
        const int ahead = S.pre[item + kInvAhead - pre_base].cluster;
        if (ahead >= 0 && ahead < a.K && ((size_t)a.cap * rb) % 16 == 0)
          bulk_prefetch_l2(wp + (size_t)ahead * a.cap * rb, (uint32_t)((size_t)a.cap * rb));
      }
      if (d.last) {
        const int par = tile & 1;
        unsigned long long best = 0ull;
        if (h < d.n && d.cluster >= 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int tok = t0 + u;
            const float4 *pp = reinterpret_cast<const float4 *>(&S.part[par][h][tok][0]);
            const float4 x0 = pp[0], x1 = pp[1], x2 = pp[2], x3 = pp[3];
            const float v = ((x0.x + x0.y) + (x0.z + x0.w)) + ((x1.x + x1.y) + (x1.z + x1.w)) +
                            (((x2.x + x2.y) + (x2.z + x2.w)) + ((x3.x + x3.y) + (x3.z + x3.w)));
            if (tok < a.cap) {
              const uint32_t vid = vids[u];
              float key = v;
              if (a.do_sample)
                key = v / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)row_h, vid);
              const unsigned long long w = pack(key, vid);
              best = w > best ? w : best;
            }
          }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
          best = other > best ? other : best;
        }
        if ((lane & 3) == 0 && h < d.n && row_h >= 0 && row_h < a.rows)
          atomicMax(&a.packed[row_h], best);
        __syncwarp();
        nbar_arrive(kBarPart0 + par, kInvBlock);
        ++tile;
      }
    }
  } else {
    float acc[2][2][4];
#pragma unroll
    for (int cs = 0; cs < 2; ++cs)
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[cs][0][u] = acc[cs][1][u] = 0.f;
    uint32_t phase = 0u;
    int tile = 0;
    for (int c = 0;; ++c) {
      const int s = c % kInvSlots;
      if (!mbar_wait(&S.mbar[s], (phase >> s) & 1u, a.copy_polls) && lane == 0)
        atomicOr(&S.s_err, kErrCopyTimeout);
      phase ^= 1u << s;
      const InvChunk d = S.desc[s];
      if (d.cluster == -1) break;
      const int cb = d.cluster >= 0 ? min(cb_max, rb - d.dc * cb_max) : 0;  // invalid: no groups
      const unsigned char *slot = ring + (size_t)s * kInvSlotBytes;
      const unsigned char *hrows = slot + (size_t)kTileRows * pitch;
      // column set cs: hidden row 4 * cs + (gq >> 1) of the item, parity odd
      const int h0 = gq >> 1, h1 = 4 + (gq >> 1);
      const bool v0 = h0 < d.n, v1 = h1 < d.n;
      const int ng = cb / 64;
      for (int grp = warp; grp < ng; grp += kFWarps) {
        const int q = grp ^ odd;
        const unsigned char *ra = slot + (size_t)gq * pitch + q * 64 + tq * 16;
        const uint4 a0 = lds128(ra), b0 = lds128(ra + 8 * pitch);
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        const uint4 x0 = v0 ? lds128(hrows + (size_t)h0 * cb_max + q * 64 + tq * 16) : z;
        const uint4 x1 = v1 ? lds128(hrows + (size_t)h1 * cb_max + q * 64 + tq * 16) : z;
        const uint32_t A0[4] = {a0.x, b0.x, a0.y, b0.y}, A1[4] = {a0.z, b0.z, a0.w, b0.w};
        {
          const uint32_t B0[2] = {x0.x, x0.y}, B1[2] = {x0.z, x0.w};
          mma16816<HT>(acc[0][0], A0, B0);
          mma16816<HT>(acc[0][1], A1, B1);
        }
        {
          const uint32_t B0[2] = {x1.x, x1.y}, B1[2] = {x1.z, x1.w};
          mma16816<HT>(acc[1][0], A0, B0);
          mma16816<HT>(acc[1][1], A1, B1);
        }
      }
      if (d.last) {
        const int par = tile & 1;
        if (tile >= 2) nbar_sync(kBarPart0 + par, kInvBlock);
        // lane (g, t): token g (g + 8) against item row 4 * cs + t in c[odd] (c[2 + odd])
#pragma unroll
        for (int cs = 0; cs < 2; ++cs) {
          const int h = 4 * cs + tq;
          S.part[par][h][gq][warp] = acc[cs][0][odd] + acc[cs][1][odd];
          S.part[par][h][gq + 8][warp] = acc[cs][0][2 + odd] + acc[cs][1][2 + odd];
        }
#pragma unroll
        for (int cs = 0; cs < 2; ++cs)
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[cs][0][u] = acc[cs][1][u] = 0.f;
        ++tile;
      }
      nbar_arrive(kBarSlot0 + s, kInvBlock);
    }
    for (int t = max(tile - 2, 0); t < tile; ++t) nbar_sync(kBarPart0 + (t & 1), kInvBlock);
  }
  __syncthreads();
  if (tid == 0 && S.s_err) atomicOr(a.err, S.s_err);
}

// ---------------------------------------------------------------------------
// Special tokens (one warp per (row, special)) and the publish step.
// ---------------------------------------------------------------------------
template <typename HT>
__global__ void k_special_scores(const void *hidden, int rows, int D, const void *w_perm,
                                 const int32_t *vocab_map, const int32_t *special_slots,
                                 int n_special, int n_slots, int do_sample, float temperature,
                                 RngKey rng, unsigned long long *packed) {
  const int lane = threadIdx.x & 31;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= rows * n_special) return;
  const int r = w / n_special, j = w - r * n_special;
  const int slot = special_slots[j];
  if (slot < 0 || slot >= n_slots) return;
  const HT *h = reinterpret_cast<const HT *>(hidden) + (size_t)r * D;
  const HT *wr = reinterpret_cast<const HT *>(w_perm) + (size_t)slot * D;
  float acc = 0.f;
  for (int e = lane; e < D; e += 32) acc += (float)h[e] * (float)wr[e];
  acc = warp_sum(acc);
  if (lane == 0) {
    const uint32_t vid = (uint32_t)vocab_map[slot];
    float key = acc;
    if (do_sample) key = acc / temperature + gumbel(rng, kStageTokens, (uint32_t)r, vid);
    atomicMax(&packed[r], pack(key, vid));
  }
}

// Dense head on the tensor cores: the vocabulary is cap blocks of K w_perm
// rows; block j's logits [rows, K] (a GEMM into the score scratch) fold into
// packed[row] as (logit or Gumbel key, vocab id). Grid (rows, splits).
__global__ void k_dense_block_argmax(const float *logits, int stride, int rows, int K,
                                    const int32_t *vocab_map, int slot0, int do_sample,
                                    float temperature, RngKey rng, unsigned long long *packed) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float *row = logits + (size_t)r * stride;
  unsigned long long best = 0ull;
  for (int k = blockIdx.y * blockDim.x + threadIdx.x; k < K; k += gridDim.y * blockDim.x) {
    const uint32_t vid = (uint32_t)__ldg(&vocab_map[slot0 + k]);
    float key = sanitize(__ldcg(&row[k]));
    if (do_sample) key = key / temperature + gumbel(rng, kStageTokens, (uint32_t)r, vid);
    const unsigned long long w = pack(key, vid);
    best = w > best ? w : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0 && best) atomicMax(&packed[r], best);
}

// Copies n16 16-byte words from page-locked host memory into device memory;
// lets the dependent step launch at once (the step waits for this grid's
// completion before it reads the copy).
__global__ void k_stage_in(uint4 *dst, const uint4 *src, int n16) {
  grid_dep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// Publish: ids (out_ids), or for a tensor-parallel shard the signed packed
// words the ranks max-reduce (out_signed); then packed[] reset.
__global__ void k_inv_finalize(unsigned long long *packed, int rows, int64_t *out_ids,
                               long long *out_signed) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
    const unsigned long long w = packed[i];
    if (out_signed) out_signed[i] = to_signed(w);
    else out_ids[i] = w ? (int64_t)packed_id(w) : (int64_t)0xFFFFFFFFll;
    packed[i] = 0ull;
  }
}

}  // namespace fh
