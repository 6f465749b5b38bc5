// Batched decode steps (rows >= kBatchMinRows): the kernels around the
// tensor-core stage 1 (fh_s1_tc.cuh) and stage 2 (fh_stage2_tc.cuh).
//
//   k_select_hist     per row: the stage-1 keys from the split partials
//                     (sum, fp8 row scale, and in sampling mode / T +
//                     Gumbel(stage 1, r, k): the keys the one-kernel and
//                     three-kernel paths compute), then the top-p clusters.
//   k_special_scores  the special tokens of every row into packed[row].
//   k_inv_finalize    ids (or signed words of a shard) from packed[], then
//                     packed[] reset (after the dense kernel).
//   k_stage2_stream   stage 2 of the 5..15-row steps: per-warp rings of
//                     whole-row bulk copies over the probed w_perm rows.
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

// ---------------------------------------------------------------------------
// Top-p clusters of one row per CTA: the same rule as k_select (the p largest
// (score, -id) keys, ids ascending) found with two 8-bit histogram levels over
// the monotone key (bf16 resolution), an exact rank of the threshold bucket's
// few keys (a radix select over the remaining 48 key bits when the bucket is
// large), and one ordered compaction.
// NT = 1024 threads for up to one row per SM; NT = 512 (two CTAs per SM) when
// there are more rows than SMs, so that every row is selected in one wave.
// Dynamic shared memory: K floats (the row) + one 256-bin histogram per warp.
// ---------------------------------------------------------------------------
constexpr int kHSelMaxWarps = 32;
constexpr int kHSelBkt = 256;  // bucket keys ranked directly

struct HSelSmem {
  __align__(16) uint32_t hist[256];
  unsigned long long bkt[kHSelBkt];
  int n_bkt;
  int bin, above, cnt;
  unsigned long long T;
  int warp_counts[kHSelMaxWarps];
};

__host__ __device__ __forceinline__ size_t hsel_row_bytes(int K) {
  return ((size_t)K * sizeof(float) + 15) / 16 * 16;
}
__host__ __device__ __forceinline__ size_t hsel_smem_bytes(int K, int threads) {
  return hsel_row_bytes(K) + (size_t)(threads / 32) * 256 * sizeof(uint32_t) + sizeof(HSelSmem);
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
  uint32_t *bm;          // [K][8] row bit maps of the stage-2 index (rows <= 256), or null
};

template <int NT>
__global__ void __launch_bounds__(NT, 1024 / NT) k_select_hist(HSelArgs a) {
  constexpr int kWarps = NT / 32;
  static_assert(kWarps <= kHSelMaxWarps, "one histogram per warp");
  extern __shared__ __align__(16) unsigned char hsm[];
  const int K = a.K, p = a.p;
  float *sc = reinterpret_cast<float *>(hsm);
  uint32_t *wh = reinterpret_cast<uint32_t *>(hsm + hsel_row_bytes(K));  // [kWarps][256]
  HSelSmem &S = *reinterpret_cast<HSelSmem *>(hsm + hsel_row_bytes(K) +
                                              (size_t)kWarps * 256 * sizeof(uint32_t));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.x;
  for (int i = tid; i < kWarps * 256; i += NT) wh[i] = 0u;
  if (tid < 256) S.hist[tid] = 0u;
  if (tid == 0) S.n_bkt = 0;
  __syncthreads();  // the warp histograms are zero before the keys are counted
  grid_dep_wait();  // the partials come from the stage-1 kernel before this one
  grid_dep_launch();
  // The row's partials as float4 groups (rows are padded to 64 floats and
  // 16-byte aligned), 4 groups per thread and pass, the loads of two splits at
  // a time issued before they are summed (in split order).
  const float4 *row4 = reinterpret_cast<const float4 *>(a.part + (size_t)r * a.row_stride);
  const size_t split4 = a.split_stride / 4;
  const int G4 = (K + 3) / 4;
  constexpr int kPer = 4;
  for (int g0 = 0; g0 < G4; g0 += kPer * NT) {
    float4 acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int g = g0 + tid + NT * i;
      acc[i] = g < G4 ? __ldcg(row4 + g) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int s0 = 1; s0 < a.splits; s0 += 2) {
      float4 nx[2][kPer];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int g = g0 + tid + NT * i;
          nx[u][i] = (s0 + u < a.splits && g < G4) ? __ldcg(row4 + (size_t)(s0 + u) * split4 + g)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          if (s0 + u < a.splits) {
            acc[i].x += nx[u][i].x;
            acc[i].y += nx[u][i].y;
            acc[i].z += nx[u][i].z;
            acc[i].w += nx[u][i].w;
          }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int g = g0 + tid + NT * i;
      const float vv[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k = 4 * g + u;
        if (g >= G4 || k >= K) continue;
        float v = vv[u];
        if (a.scale) v *= __ldg(&a.scale[k]);
        if (a.do_sample)
          v = v / a.temperature +
              gumbel(a.rng, kStageClusters, (uint32_t)r, (uint32_t)(a.cluster_base + k));
        if (a.scores_out) a.scores_out[(size_t)r * a.out_stride + k] = v;
        sc[k] = sanitize(v);
        // level 1: coarse bins (key >> 24), one private histogram per warp
        atomicAdd(&wh[warp * 256 + (mono(sc[k]) >> 24)], 1u);
      }
    }
  }
  __syncthreads();
  if (tid < 256) {
    uint32_t t = 0;
    for (int w = 0; w < kWarps; ++w) t += wh[w * 256 + tid];
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
  for (int k = tid; k < K; k += NT) {
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
    for (int k = tid; k < K; k += NT) {
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
    for (int j = tid; j < nb; j += NT) {
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
      for (int k = tid; k < K; k += NT) {
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
          // the stage-2 index directly (8 words of row bits per cluster)
          if (a.bm) atomicOr(&a.bm[(size_t)k * 8 + (r >> 5)], 1u << (r & 31));
        }
      },
      S.warp_counts);
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

// ---------------------------------------------------------------------------
// Stage 2 of the few-row steps (greedy or sampled), streamed: a persistent
// grid whose warps each take a contiguous range of w_perm rows to score (the
// rows of every (row, probe) item in item order, then the special tokens'
// rows) and keep kS2sSlots whole-row bulk copies in flight into their own
// shared-memory slots, so an SM has 2-3 rows per warp on the way instead of
// one register-resident row per warp. A warp keeps the running best packed
// (key, vocab id) of its current hidden row and folds it into packed[row]
// with one atomicMax when the row changes; the last CTA publishes (as
// k_stage2 does). The hidden row is read through L1.
// ---------------------------------------------------------------------------
constexpr int kS2sSlots = 3;
constexpr int kS2sSmemBudget = 192 * 1024;

__host__ __device__ __forceinline__ int s2s_warps(int D) {
  const int rb = D * 2;
  const int w = kS2sSmemBudget / (kS2sSlots * rb);
  return w < 1 ? 1 : (w > 16 ? 16 : w);
}
__host__ __device__ __forceinline__ size_t s2s_smem_bytes(int D) {
  const int nw = s2s_warps(D);
  return (size_t)nw * kS2sSlots * ((size_t)D * 2) + (size_t)nw * kS2sSlots * (8 + 8) + 128;
}

template <typename HT, typename IdxT, bool SAMPLE>
__global__ void __launch_bounds__(512, 1)
    k_stage2_stream(Stage2Args a, long long items, uint32_t *err, uint32_t polls) {
  extern __shared__ __align__(128) unsigned char s2s[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const size_t rb = (size_t)a.D * sizeof(HT);
  unsigned char *ring = s2s + (size_t)warp * kS2sSlots * rb;
  uint64_t *bars = reinterpret_cast<uint64_t *>(s2s + (size_t)nw * kS2sSlots * rb) +
                   warp * kS2sSlots;
  long long *desc = reinterpret_cast<long long *>(
                        s2s + (size_t)nw * kS2sSlots * rb + (size_t)nw * kS2sSlots * 8) +
                    warp * kS2sSlots;
  if (lane == 0) {
    for (int j = 0; j < kS2sSlots; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (a.wait_prior) grid_dep_wait();  // the probe lists come from the kernel before
  const int ipr = a.P + a.n_special;
  const long long n_units = items * a.cap;
  const long long W = (long long)gridDim.x * nw, gw = (long long)blockIdx.x * nw + warp;
  const long long u0 = gw * n_units / W, u1 = (gw + 1) * n_units / W;
  const int n = (int)(u1 - u0);
  // w_perm row of unit u, or -1 (an unused slot of a special item, a probe
  // outside this head's clusters)
  auto resolve = [&](long long u) -> long long {
    const long long item = u / a.cap;
    const int sl = (int)(u - item * a.cap);
    const int r = (int)(item / ipr), j = (int)(item - (long long)r * ipr);
    if (j < a.P) {
      long long cid = a.dense ? (long long)j
                              : (long long)reinterpret_cast<const IdxT *>(a.probes)[(size_t)r * a.probe_stride + j];
      cid -= a.cluster_base;
      return (cid >= 0 && cid < a.K) ? cid * a.cap + sl : -1;
    }
    if (sl != 0) return -1;
    const long long sp = a.special_slots[j - a.P];
    return (sp >= 0 && sp < (long long)a.K * a.cap) ? sp : -1;
  };
  int last_issued[kS2sSlots];  // lane 0: the last unit put in each slot, or -1
  for (int j = 0; j < kS2sSlots; ++j) last_issued[j] = -1;
  auto issue = [&](int k) {  // lane 0: unit u0 + k into slot k % kS2sSlots
    const int s = k % kS2sSlots;
    const long long row = resolve(u0 + k);
    desc[s] = row;
    last_issued[s] = k;
    if (row >= 0) {
      fence_proxy_async_smem();
      mbar_expect_tx(&bars[s], (uint32_t)rb);
      bulk_g2s(ring + (size_t)s * rb, reinterpret_cast<const char *>(a.w_perm) + (size_t)row * rb,
               (uint32_t)rb, &bars[s]);
    } else {
      mbar_expect_tx(&bars[s], 0u);
    }
  };
  if (lane == 0)
    for (int k = 0; k < min(n, kS2sSlots); ++k) issue(k);
  __syncwarp();
  bool ok = true;
  int cur_r = -1;
  unsigned long long best = 0ull;
  const int nvec = a.D / 8;
  for (int k = 0; k < n; ++k) {
    const int s = k % kS2sSlots;
    if (ok) {
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bars[s], (uint32_t)((k / kS2sSlots) & 1), polls));
      if (!ok && lane == 0) atomicOr(err, kErrCopyTimeout);
    }
    const long long u = u0 + k;
    const int r = (int)(u / a.cap / ipr);
    if (r != cur_r) {
      if (lane == 0 && cur_r >= 0 && best) atomicMax(&a.packed[cur_r], best);
      best = 0ull;
      cur_r = r;
    }
    const long long row = desc[s];
    if (ok && row >= 0) {
      const unsigned char *wr = ring + (size_t)s * rb;
      const char *hr = reinterpret_cast<const char *>(a.hidden) + (size_t)r * rb;
      float acc = 0.f;
#pragma unroll 4
      for (int v = lane; v < nvec; v += 32) {
        const uint4 wv = *reinterpret_cast<const uint4 *>(wr + (size_t)v * 16);
        const uint4 hv = ldg_keep(hr + (size_t)v * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 w2 = pair_to_float2<HT>(wv, q);
          const float2 h2 = pair_to_float2<HT>(hv, q);
          acc = fmaf(w2.x, h2.x, acc);
          acc = fmaf(w2.y, h2.y, acc);
        }
      }
      acc = warp_sum(acc);
      const uint32_t vid = (uint32_t)reinterpret_cast<const IdxT *>(a.vocab_map)[row];
      float key = acc;
      if (SAMPLE) key = acc / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)(a.row_base + r), vid);
      const unsigned long long w = pack(key, vid);
      best = w > best ? w : best;
    }
    __syncwarp();  // the slot is read: refill it
    if (lane == 0 && ok && k + kS2sSlots < n) issue(k + kS2sSlots);
    __syncwarp();
  }
  if (lane == 0 && cur_r >= 0 && best) atomicMax(&a.packed[cur_r], best);
  if (lane == 0 && !ok)  // after a timeout: no copy of this warp may still be writing
    for (int j = 0; j < kS2sSlots; ++j)
      if (last_issued[j] >= 0) mbar_wait(&bars[j], (uint32_t)((last_issued[j] / kS2sSlots) & 1), polls);
  if (a.counter == nullptr) return;
  // Last CTA to finish publishes the winners (flag after the descriptors).
  unsigned *s_last = reinterpret_cast<unsigned *>(
      s2s + (size_t)nw * kS2sSlots * rb + (size_t)nw * kS2sSlots * 16);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    *s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (*s_last) {
    __threadfence();
    for (int r = threadIdx.x; r < a.rows; r += blockDim.x) {
      const unsigned long long w = atomicExch(&a.packed[r], 0ull);
      if (a.out_ids) a.out_ids[r] = w ? (int64_t)packed_id(w) : (int64_t)0xFFFFFFFFll;
      if (a.out_signed) a.out_signed[r] = to_signed(w);
    }
    if (threadIdx.x == 0) *a.counter = 0u;
  }
}

}  // namespace fh
