// Batched decode steps (rows >= kBatchMinRows): the kernels around the
// tensor-core stage 1 (fh_s1_tc.cuh) and stage 2 (fh_stage2_tc.cuh).
//
//   k_select_hist     per row: the stage-1 keys from the split partials
//                     (sum, fp8 row scale, and in sampling mode / T +
//                     Gumbel(stage 1, r, k): the keys the one-kernel and
//                     three-kernel paths compute), then the top-p clusters.
//   k_special_scores  the special tokens of every row into packed[row].
//   k_inv_finalize    ids (or signed words of a shard) from packed[], then
//                     packed[] reset.
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

}  // namespace fh
