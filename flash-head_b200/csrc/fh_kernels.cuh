// FlashHead decode-step kernels for sm_100a.
//
//   k_scores   stage 1: centroid scores h . C^T for a few hidden rows
//              (CUDA-core GEMV over fp8/bf16/fp16 centroid rows, streamed
//              with 16-byte non-allocating loads)
//   k_select   stage 1 selection: the top-p clusters of each row, ties to the
//              smaller id, by histogram refinement in shared memory
//   k_stage2   stage 2: gather of each probed cluster's contiguous w_perm
//              rows + block-sparse logits + argmax / Gumbel sample, reduced
//              across probes with a packed 64-bit atomicMax
#pragma once

#include "fh_device.cuh"

namespace fh {

// ===========================================================================
// Stage 1: centroid scores
// ===========================================================================
struct ScoresArgs {
  const void *hidden;  // [rows, D] HT
  int rows;
  int D;
  const void *w;        // [K, D] WT
  const float *scale;   // [K] or null
  int K;
  float *scores;        // [rows, score_stride]
  int score_stride;
  int do_sample;
  float temperature;
  RngKey rng;
  int cluster_base;
  int row_base;                 // global index of hidden row 0 (RNG stream)
  unsigned long long *packed;   // zeroed by block (0,0) when non-null
  unsigned *counter;            // zeroed by block (0,0) when non-null
  int n_packed;
};

template <typename T>
__device__ __forceinline__ float2 pair_to_float2(const uint4 &v, int q);

template <>
__device__ __forceinline__ float2 pair_to_float2<__nv_bfloat16>(const uint4 &v, int q) {
  const uint32_t w = q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ float2 pair_to_float2<__half>(const uint4 &v, int q) {
  const uint32_t w = q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
  return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}
template <>
__device__ __forceinline__ float2 pair_to_float2<__nv_fp8_e4m3>(const uint4 &v, int q) {
  const int wi = q >> 1;
  const uint32_t w = wi == 0 ? v.x : wi == 1 ? v.y : wi == 2 ? v.z : v.w;
  const uint32_t bits = (q & 1) ? (w >> 16) : (w & 0xFFFFu);
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)bits, __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2 *>(&h));
}

// One warp scores CPW clusters for ROWS hidden rows at a time. Lane l reads
// 16-byte vectors l, l+32, ... of each centroid row; the matching slice of
// each hidden row (16 or 32 bytes) comes through L1, where every warp of the
// CTA finds it. U vectors per lane are in flight per cluster.
template <typename HT, typename WT, int ROWS, int CPW, int U>
__global__ void __launch_bounds__(256) k_scores(ScoresArgs a) {
  constexpr int E = Vec<WT>::kElems;            // elements per weight vector
  constexpr int HV = E * (int)sizeof(HT) / 16;  // hidden uint4 per weight vector
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    for (int i = threadIdx.x; i < a.n_packed; i += blockDim.x) a.packed[i] = 0ull;
    if (threadIdx.x == 0 && a.counter) *a.counter = 0u;
  }
  grid_dep_launch();

  const int row0 = blockIdx.y * ROWS;
  const int nvec = a.D / E;
  const size_t wrow_bytes = (size_t)a.D * sizeof(WT);
  const size_t hrow_bytes = (size_t)a.D * sizeof(HT);
  const char *wbase = reinterpret_cast<const char *>(a.w);
  const char *hbase = reinterpret_cast<const char *>(a.hidden) + (size_t)row0 * hrow_bytes;

  for (int kb = (blockIdx.x * 8 + warp) * CPW; kb < a.K; kb += gridDim.x * 8 * CPW) {
    float acc[ROWS][CPW];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int c = 0; c < CPW; ++c) acc[r][c] = 0.f;

    for (int v0 = 0; v0 < nvec; v0 += 32 * U) {
      uint4 wv[CPW][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * 32 + lane;
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const int k = kb + c;
          wv[c][u] = (v < nvec && k < a.K)
                         ? ldg_stream(wbase + (size_t)k * wrow_bytes + (size_t)v * 16)
                         : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v >= nvec) break;
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          if (row0 + r >= a.rows) break;
          uint4 hv[HV];
#pragma unroll
          for (int i = 0; i < HV; ++i)
            hv[i] = ldg_keep(hbase + (size_t)r * hrow_bytes + (size_t)v * E * sizeof(HT) + i * 16);
#pragma unroll
          for (int q = 0; q < E / 2; ++q) {
            const float2 hf = pair_to_float2<HT>(hv[q / 4], q % 4);
#pragma unroll
            for (int c = 0; c < CPW; ++c) {
              const float2 wf = pair_to_float2<WT>(wv[c][u], q);
              acc[r][c] = fmaf(wf.x, hf.x, acc[r][c]);
              acc[r][c] = fmaf(wf.y, hf.y, acc[r][c]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int c = 0; c < CPW; ++c) acc[r][c] = warp_sum(acc[r][c]);
    if (lane == 0) {
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int k = kb + c;
        if (k >= a.K) break;
        const float sc = a.scale ? a.scale[k] : 1.f;
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          const int row = row0 + r;
          if (row >= a.rows) break;
          float s = acc[r][c] * sc;
          if (a.do_sample)
            s = s / a.temperature +
                gumbel(a.rng, kStageClusters, (uint32_t)(a.row_base + row),
                       (uint32_t)(a.cluster_base + k));
          a.scores[(size_t)row * a.score_stride + k] = s;
        }
      }
    }
  }
}

// ===========================================================================
// Stage 1 selection: top-p of each row
// ===========================================================================
// Every item gets a unique 64-bit key (mono(score) << 32 | ~id): the p
// largest keys are the p largest scores with ties to the smaller id. The
// kernel finds T, the p-th largest key, by histogram refinement over the
// "active" key interval: level 0 bins scores linearly between their min and
// max (normal-like scores leave only a handful of items in the threshold
// bin), later levels bin the top bits of (key - lo). When the threshold bin
// holds few enough items they are ranked exactly. Output: ids with key >= T,
// in item order (ascending cluster id in dense mode).
constexpr int kSelThreads = 1024;
constexpr int kSelBins = 2048;
constexpr int kSelCandMax = 1024;
constexpr int kSelMaxItems = 16384;
constexpr int kSelMaxLevels = 8;

struct SelectArgs {
  // dense mode: item i = cluster i with score scores[row * stride + i]
  const float *scores;
  int score_stride;
  // list mode (scores == null): item i = signed packed word cand[row*?]
  const long long *cand;  // [n_ranks][rows][p_in]
  int p_in;
  int n_ranks;
  int rows;
  int n_items;            // K (dense) or n_ranks * p_in (list)
  int p;
  int id_base;            // dense mode: global id of item 0
  int32_t *probes;        // [rows, p] selected ids (may be null)
  long long *cand_out;    // [rows, p] signed packed words (may be null)
  unsigned long long *packed;  // zeroed by block 0 when non-null
  unsigned *counter;
  int n_packed;
  int wait_prior;         // 1: launched with PDL after the scores kernel
};

__device__ __forceinline__ float sanitize(float s) { return s != s ? -INFINITY : s; }

__device__ __forceinline__ unsigned long long sel_key(const SelectArgs &a, int row, int i) {
  if (a.scores) {
    const float s = sanitize(a.scores[(size_t)row * a.score_stride + i]);
    return pack(s, (uint32_t)(a.id_base + i));
  }
  const int r = i / a.p_in, j = i - r * a.p_in;
  return from_signed(a.cand[((size_t)r * a.rows + row) * a.p_in + j]);
}

__device__ __forceinline__ int sel_bin_value(float s, float vmin, float scale) {
  float f = (s - vmin) * scale;
  int b = f >= (float)(kSelBins - 1) ? kSelBins - 1 : (int)f;
  return b < 0 ? 0 : b;
}

__global__ void __launch_bounds__(kSelThreads) k_select(SelectArgs a) {
  extern __shared__ unsigned long long skeys[];  // [n_items]
  __shared__ unsigned hist[kSelBins];
  __shared__ unsigned long long cand[kSelCandMax];
  __shared__ int scan_scratch[33];
  __shared__ unsigned long long red_u64[64];
  __shared__ float red_f[64];
  __shared__ int s_bstar, s_above, s_cnt, s_ncand;
  __shared__ unsigned long long s_T;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int N = a.n_items;
  if (blockIdx.x == 0 && a.packed) {
    for (int i = tid; i < a.n_packed; i += blockDim.x) a.packed[i] = 0ull;
    if (tid == 0 && a.counter) *a.counter = 0u;
  }
  if (a.wait_prior) grid_dep_wait();
  // Stage 2 may now be scheduled; its CTAs wait for this grid to finish.
  grid_dep_launch();

  // Load keys; track the finite score range.
  float vmin = INFINITY, vmax = -INFINITY;
  for (int i = tid; i < N; i += blockDim.x) {
    const unsigned long long k = sel_key(a, row, i);
    skeys[i] = k;
    const float s = unmono((uint32_t)(k >> 32));
    if (isfinite(s)) {
      vmin = fminf(vmin, s);
      vmax = fmaxf(vmax, s);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    vmin = fminf(vmin, __shfl_xor_sync(0xFFFFFFFFu, vmin, o));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xFFFFFFFFu, vmax, o));
  }
  if (lane == 0) {
    red_f[warp] = vmin;
    red_f[32 + warp] = vmax;
  }
  __syncthreads();
  vmin = INFINITY;
  vmax = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    vmin = fminf(vmin, red_f[w]);
    vmax = fmaxf(vmax, red_f[32 + w]);
  }
  const float vscale = (float)kSelBins / (vmax - vmin);
  bool value_mode = vmax > vmin && isfinite(vscale) && vscale > 0.f;

  unsigned long long alo = 0ull, ahi = ~0ull;  // active key interval (inclusive)
  int need = a.p;
  unsigned long long T = 0ull;
  for (int level = 0; level < kSelMaxLevels; ++level) {
    const bool vm = value_mode && level == 0;
    const unsigned long long range = ahi - alo;
    const int shift = range == 0ull ? 0 : max(0, 64 - __clzll((long long)range) - 11);
    for (int i = tid; i < kSelBins; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int i = tid; i < N; i += blockDim.x) {
      const unsigned long long k = skeys[i];
      if (k < alo || k > ahi) continue;
      const int b = vm ? sel_bin_value(unmono((uint32_t)(k >> 32)), vmin, vscale)
                       : (int)((k - alo) >> shift);
      atomicAdd(&hist[b], 1u);
    }
    // Suffix scan over bins, highest bin first: thread t owns bins
    // kSelBins-1-2t and kSelBins-2-2t.
    const int b_hi = kSelBins - 1 - 2 * tid, b_lo = b_hi - 1;
    __syncthreads();
    const int c_hi = tid < kSelBins / 2 ? (int)hist[b_hi] : 0;
    const int c_lo = tid < kSelBins / 2 ? (int)hist[b_lo] : 0;
    int total;
    const int before = block_exclusive_scan(c_hi + c_lo, scan_scratch, &total);
    if (tid < kSelBins / 2) {
      if (before < need && need <= before + c_hi) {
        s_bstar = b_hi;
        s_above = before;
        s_cnt = c_hi;
      } else if (before + c_hi < need && need <= before + c_hi + c_lo) {
        s_bstar = b_lo;
        s_above = before + c_hi;
        s_cnt = c_lo;
      }
    }
    __syncthreads();
    const int bstar = s_bstar, cnt = s_cnt;
    need -= s_above;
    // New active interval: keys of active items in bin bstar.
    unsigned long long kmin = ~0ull, kmax = 0ull;
    for (int i = tid; i < N; i += blockDim.x) {
      const unsigned long long k = skeys[i];
      if (k < alo || k > ahi) continue;
      const int b = vm ? sel_bin_value(unmono((uint32_t)(k >> 32)), vmin, vscale)
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
    if (lane == 0) {
      red_u64[warp] = kmin;
      red_u64[32 + warp] = kmax;
    }
    if (tid == 0) s_ncand = 0;
    __syncthreads();
    kmin = ~0ull;
    kmax = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      kmin = red_u64[w] < kmin ? red_u64[w] : kmin;
      kmax = red_u64[32 + w] > kmax ? red_u64[32 + w] : kmax;
    }
    alo = kmin;
    ahi = kmax;
    if (cnt == need) {
      T = alo;
      break;
    }
    if (cnt <= kSelCandMax) {
      for (int i = tid; i < N; i += blockDim.x) {
        const unsigned long long k = skeys[i];
        if (k >= alo && k <= ahi) {
          const int pos = atomicAdd(&s_ncand, 1);
          if (pos < kSelCandMax) cand[pos] = k;
        }
      }
      __syncthreads();
      const int nc = min(cnt, kSelCandMax);
      if (tid < nc) {
        const unsigned long long mine = cand[tid];
        int rank = 0;
        for (int j = 0; j < nc; ++j) rank += cand[j] > mine;
        if (rank == need - 1) s_T = mine;
      }
      __syncthreads();
      T = s_T;
      break;
    }
    __syncthreads();
  }

  // Compaction in item order (ascending cluster id in dense mode).
  block_ordered_compact(
      N, [&](int i) { return skeys[i] >= T; },
      [&](int pos, int i) {
        if (pos < a.p) {
          const unsigned long long k = skeys[i];
          if (a.probes) a.probes[(size_t)row * a.p + pos] = (int32_t)packed_id(k);
          if (a.cand_out) a.cand_out[(size_t)row * a.p + pos] = to_signed(k);
        }
      },
      scan_scratch);
}

// ===========================================================================
// Stage 2: gather + block-sparse logits + argmax / sample
// ===========================================================================
enum Stage2Mode { kGreedy = 0, kSample = 1, kLogits = 2, kProbeMax = 3 };

struct Stage2Args {
  const void *hidden;  // [rows, D]
  int rows;
  int D;
  const void *w_perm;  // [K * cap, D]
  int K;
  int cap;
  const void *probes;  // [rows, probe_stride] IdxT (ignored when dense)
  int probe_stride;
  int P;               // probes per row (K when dense)
  int dense;
  const void *vocab_map;  // [K * cap] IdxT
  const int32_t *special_slots;
  int n_special;
  int cluster_base;
  int row_base;
  float temperature;
  RngKey rng;
  unsigned long long *packed;  // [rows] (modes 0/1)
  unsigned *counter;           // last-CTA-done counter (null: no finalize)
  int64_t *out_ids;            // finalize: ids
  long long *out_signed;       // finalize: signed packed words (tensor parallel)
  void *out_logits;            // mode 2: [rows, P * cap] HT
  void *out_max;               // mode 3: [rows, P] HT
  int64_t *out_vocab;          // mode 3: [rows, P]
  int wait_prior;
};

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float x) {
  return __float2half_rn(x);
}

// One CTA per (row, probe) item; warp w computes the logits of slots w,
// w + nwarps, ... of the probed cluster (blockDim = 32 * min(cap, 16)). Lane l
// streams 16-byte vectors l, l+32, ... of each w_perm row; the hidden row is
// read through L1.
template <typename HT, typename IdxT, int MODE, int U>
__global__ void __launch_bounds__(512, 2) k_stage2(Stage2Args a) {
  __shared__ unsigned long long red[32];
  __shared__ float red_val[32];
  __shared__ unsigned s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int ipr = a.P + a.n_special;
  const int row = blockIdx.x / ipr;
  const int j = blockIdx.x - row * ipr;
  const int nvec = a.D / 8;
  const size_t row_bytes = (size_t)a.D * sizeof(HT);
  const char *hrow = reinterpret_cast<const char *>(a.hidden) + (size_t)row * row_bytes;

  // The hidden row does not depend on the previous kernel: fetch the first
  // chunk before waiting for the probe list.
  uint4 hv[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int v = u * 32 + lane;
    hv[u] = v < nvec ? ldg_keep(hrow + (size_t)v * 16) : make_uint4(0, 0, 0, 0);
  }
  if (a.wait_prior) grid_dep_wait();

  long long base = -1;  // first w_perm row of this item
  int nslots = 0;
  if (j < a.P) {
    long long cid = a.dense ? (long long)j
                            : (long long)reinterpret_cast<const IdxT *>(a.probes)[(size_t)row * a.probe_stride + j];
    cid -= a.cluster_base;
    if (cid >= 0 && cid < a.K) {
      base = cid * a.cap;
      nslots = a.cap;
    }
  } else {
    base = a.special_slots[j - a.P];
    nslots = (base >= 0 && base < (long long)a.K * a.cap) ? 1 : 0;
  }

  // hv holds the first chunk of the hidden row; with more than one chunk it
  // is overwritten and reloaded per slot.
  const bool one_chunk = nvec <= 32 * U;
  bool hv_first = true;
  for (int sl = warp; sl < nslots; sl += nwarps) {
    const long long slot = base + sl;
    const char *wrow = reinterpret_cast<const char *>(a.w_perm) + (size_t)slot * row_bytes;
    float acc = 0.f;
    for (int v0 = 0; v0 < nvec; v0 += 32 * U) {
      uint4 wv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * 32 + lane;
        wv[u] = v < nvec ? ldg_stream(wrow + (size_t)v * 16) : make_uint4(0, 0, 0, 0);
      }
      if (!(v0 == 0 && hv_first)) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int v = v0 + u * 32 + lane;
          hv[u] = v < nvec ? ldg_keep(hrow + (size_t)v * 16) : make_uint4(0, 0, 0, 0);
        }
      }
      hv_first = one_chunk;
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 w2 = pair_to_float2<HT>(wv[u], q);
          const float2 h2 = pair_to_float2<HT>(hv[u], q);
          acc = fmaf(w2.x, h2.x, acc);
          acc = fmaf(w2.y, h2.y, acc);
        }
      }
    }
    acc = warp_sum(acc);
    if (MODE == kLogits) {
      if (lane == 0)
        reinterpret_cast<HT *>(a.out_logits)[((size_t)row * a.P + j) * a.cap + sl] =
            from_float<HT>(acc);
    } else if (lane == 0) {
      const uint32_t vid = (uint32_t)reinterpret_cast<const IdxT *>(a.vocab_map)[slot];
      float key = acc;
      if (MODE == kSample)
        key = acc / a.temperature + gumbel(a.rng, kStageTokens, (uint32_t)(a.row_base + row), vid);
      red[sl] = pack(key, vid);
      red_val[sl] = acc;
    }
  }
  if (MODE == kLogits) return;
  __syncthreads();
  if (warp == 0) {
    const unsigned long long w = lane < nslots ? red[lane] : 0ull;
    const unsigned long long best = warp_max_u64(w);
    if (MODE == kProbeMax) {
      if (j < a.P) {
        // value of the winning slot, as the reference stores it (fused.py:78)
        const int wl = __ffs(__ballot_sync(0xFFFFFFFFu, lane < nslots && w == best)) - 1;
        if (lane == 0) {
          const float bv = (nslots > 0 && wl >= 0) ? red_val[wl] : 0.f;
          reinterpret_cast<HT *>(a.out_max)[(size_t)row * a.P + j] = from_float<HT>(bv);
          a.out_vocab[(size_t)row * a.P + j] =
              best ? (int64_t)packed_id(best) : (int64_t)0xFFFFFFFFll;
        }
      }
      return;
    }
    if (lane == 0 && best != 0ull) atomicMax(&a.packed[row], best);
  }
  if (MODE == kProbeMax || a.counter == nullptr) return;
  // Last CTA to finish publishes the winners.
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    for (int r = threadIdx.x; r < a.rows; r += blockDim.x) {
      // Every other CTA has finished its atomicMax: read the winner and
      // leave the accumulator zeroed for the next call on this workspace.
      const unsigned long long w = atomicExch(&a.packed[r], 0ull);
      if (a.out_ids) a.out_ids[r] = w ? (int64_t)packed_id(w) : (int64_t)0xFFFFFFFFll;
      if (a.out_signed) a.out_signed[r] = to_signed(w);
    }
    if (threadIdx.x == 0) *a.counter = 0u;
  }
}

// Fill / unpack helpers for the stateless argmax entry point, whose only
// buffer is the caller's int64 output (used as the packed accumulator).
__global__ void k_fill_u64(unsigned long long *p, int n, unsigned long long v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}
__global__ void k_unpack_ids(unsigned long long *p, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const unsigned long long w = p[i];
    reinterpret_cast<int64_t *>(p)[i] = w ? (int64_t)packed_id(w) : (int64_t)0xFFFFFFFFll;
  }
}
__global__ void k_signed_to_ids(const long long *best, int n, int64_t *out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const unsigned long long w = from_signed(best[i]);
    out[i] = w ? (int64_t)packed_id(w) : (int64_t)0xFFFFFFFFll;
  }
}

}  // namespace fh
