// Dense head of a batched call on the 5th-generation tensor cores:
// logits = H (rows x D) . w_perm^T (D x V) by tcgen05.mma, with the argmax
// (largest logit, then smallest vocab id, as packed words) folded into the
// epilogue, so the [rows, V] logits never reach HBM. In sampling mode the
// epilogue ranks logit / T + Gumbel noise instead (Gumbel-max: the argmax of
// the perturbed keys is a draw from softmax(logit / T)). The reference runs
// this branch above 10 rows as F.linear over w_perm + argmax or multinomial
// (src/flash_head/flash_head.py:292-301, :263-275).
//
// One persistent CTA per SM, 10 warps:
//   warp 0  lane 0 issues TMA tensor copies (128-byte swizzle) of the hidden
//           tiles (128 rows x 64 elements) and the w_perm tile (n_tile rows x
//           64 elements) of each k-block into a ring of shared-memory stages;
//   warp 1  allocates 512 TMEM columns; lane 0 issues tcgen05.mma
//           (M = 128 hidden rows, N = n_tile vocab slots, K = 16) per k-block
//           and tcgen05.commit's the stage back to the producer, and the
//           finished accumulator to the epilogue;
//   warps 2..9  read the accumulator with tcgen05.ld (warp w owns TMEM lanes
//           32*(w%4) .., warps 2..5 the first half of the tile's columns,
//           warps 6..9 the second), i.e. each thread one hidden row, and keep
//           that row's best packed (logit, vocab id) word over the CTA's vocab
//           tiles in four independent chains; one atomicMax per row and half
//           at the end.
// When n_acc * mt accumulators fit the 512 TMEM columns they are
// double-buffered, so the epilogue of tile i overlaps the MMAs of tile i + 1.
// Every wait is bounded; on a timeout the kernel records kErrCopyTimeout,
// drains its own copies and MMAs (bounded) and frees TMEM before it returns.
#pragma once

#include <cuda.h>

#include "fh_fused.cuh"

namespace fh {

constexpr int kDtThreads = 320;
constexpr int kDtEpiThreads = 256;  // warps 2..9
// Bytes of a row per k-block: 128 (128-byte swizzle, 64 elements), or 64
// (64-byte swizzle, stages half the size, twice as many in flight; measured
// slower on the Llama-3.2-1B head: 92 vs 86 us at 64 rows, 144 vs 134 us at 256).
#ifndef FH_DT_KBYTES
#define FH_DT_KBYTES 128
#endif
constexpr int kDtKBytes = FH_DT_KBYTES;
static_assert(kDtKBytes == 64 || kDtKBytes == 128, "k-block of 64 or 128 bytes");
constexpr int kDtKBlock = kDtKBytes / 2;       // 16-bit elements per k-block
constexpr int kDtMTile = 128;                  // hidden rows per MMA (TMEM lanes)
constexpr int kDtATileBytes = kDtMTile * kDtKBytes;
constexpr int kDtMaxRows = 2 * kDtMTile;
constexpr int kDtMaxTile = 256;                // vocab slots per tile (MMA N)
constexpr int kDtMaxStages = 12;
constexpr int kDtTmemCols = 512;
constexpr int kDtSmemMax = 227 * 1024;

struct DenseTcArgs {
  int rows;      // hidden rows, 1..kDtMaxRows
  int V;         // w_perm rows
  int n_tile;    // vocab slots per tile: multiple of 16, <= kDtMaxTile
  int n_tiles;   // ceil(V / n_tile)
  int mt;        // 128-row hidden tiles: 1 or 2
  int stages;
  int nk;        // k-blocks: ceil(D / 64)
  int n_acc;     // accumulator sets (2: the epilogue overlaps the next tile's MMAs)
  int acc_stride;  // TMEM columns per accumulator (>= n_tile); n_acc*mt*acc_stride <= 512
  uint32_t idesc;
  const int32_t *vocab_map;
  unsigned long long *packed;  // [rows], max-folded
  uint32_t *err;
  uint32_t polls;
  int do_sample;   // keys logit / T + Gumbel(stage 2, row_base + row, vocab id)
  float temperature;
  RngKey rng;
  int row_base;    // global index of hidden row 0 of this launch (noise stream)
};

struct DenseTcCtrl {
  uint64_t full[kDtMaxStages];
  uint64_t empty[kDtMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t s_err;
  int vid[2][kDtMaxTile];
};

__host__ __device__ inline size_t dense_tc_stage_bytes(int mt, int n_tile) {
  return (size_t)mt * kDtATileBytes + (size_t)n_tile * kDtKBytes;
}
__host__ __device__ inline size_t dense_tc_smem_bytes(int mt, int n_tile, int stages) {
  return 1024 + (size_t)stages * dense_tc_stage_bytes(mt, n_tile) + sizeof(DenseTcCtrl);
}
// Instruction descriptor of kind::f16: f32 accumulator, A and B both bf16 (or
// both f16), both K-major, N = n_tile, M = 128.
__host__ __device__ inline uint32_t dense_tc_idesc(bool bf16, int n_tile) {
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)(n_tile >> 3) << 17) |
         ((uint32_t)(kDtMTile >> 4) << 24);
}

// Shared-memory matrix descriptor of a K-major tile written by a TMA copy
// with the k-block's swizzle (64 or 128 bytes): rows kDtKBytes apart, 8-row
// groups 8 * kDtKBytes apart (stride byte offset), leading byte offset unused
// (1), descriptor version 1, layout type 4 (64-byte swizzle) or 2 (128-byte).
// The tile base is 1024-byte aligned; the k-th 16-element step inside the
// row adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t umma_desc_k(uint32_t saddr) {
  constexpr uint64_t layout = kDtKBytes == 128 ? 2ull : 4ull;
  constexpr uint64_t sbo = (8ull * kDtKBytes) >> 4;
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (sbo << 32) | (1ull << 46) |
         (layout << 61);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives (once) on the mbarrier when every tcgen05 operation this thread
// issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// SAMPLE: rank Gumbel-perturbed keys (a.do_sample set) instead of logits; a
// template parameter so the greedy epilogue carries no noise code.
template <bool SAMPLE>
__global__ void __launch_bounds__(kDtThreads, 1)
    k_dense_tc(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_w,
               DenseTcArgs a) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  const uint32_t raw = smem_u32(dsm);
  unsigned char *ring = dsm + (((raw + 1023u) & ~1023u) - raw);
  const size_t sb = dense_tc_stage_bytes(a.mt, a.n_tile);
  DenseTcCtrl &S = *reinterpret_cast<DenseTcCtrl *>(ring + (size_t)a.stages * sb);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  const int t0 = (int)((long long)b * a.n_tiles / G);
  const int t1 = (int)((long long)(b + 1) * a.n_tiles / G);
  const int n_acc = a.n_acc;

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&S.acc_full[j], 1);
      mbar_init(&S.acc_empty[j], kDtEpiThreads);
    }
    mbar_init(&S.drain, 1);
    S.s_err = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {  // the CTA is alone on its SM (launch bounds, shared memory)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S.tmem_base)),
                 "r"(kDtTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0u;
      int issued[kDtMaxStages];  // parity of the last fill of each stage, -1: none
      for (int j = 0; j < kDtMaxStages; ++j) issued[j] = -1;
      bool ok = true;
      for (int t = t0; t < t1 && ok; ++t) {
        for (int kb = 0; kb < a.nk; ++kb) {
          if (!mbar_wait(&S.empty[s], ph ^ 1u, a.polls)) {
            atomicOr(&S.s_err, kErrCopyTimeout);
            ok = false;
            break;
          }
          unsigned char *st = ring + (size_t)s * sb;
          mbar_expect_tx(&S.full[s], (uint32_t)sb);
          for (int m = 0; m < a.mt; ++m)
            tma_load_2d(st + (size_t)m * kDtATileBytes, &tm_h, kb * kDtKBlock, m * kDtMTile,
                        &S.full[s]);
          tma_load_2d(st + (size_t)a.mt * kDtATileBytes, &tm_w, kb * kDtKBlock, t * a.n_tile,
                      &S.full[s]);
          issued[s] = (int)ph;
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // every copy this thread issued has landed before the CTA may leave
      for (int j = 0; j < a.stages; ++j)
        if (issued[j] >= 0 && !mbar_wait(&S.full[j], (uint32_t)issued[j], a.polls))
          atomicOr(&S.s_err, kErrCopyTimeout);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0u;
      bool ok = true;
      for (int t = t0, i = 0; t < t1 && ok; ++t, ++i) {
        const int buf = i % n_acc, use = i / n_acc;
        if (use > 0) {
          if (!mbar_wait(&S.acc_empty[buf], (uint32_t)((use - 1) & 1), a.polls)) {
            atomicOr(&S.s_err, kErrCopyTimeout);
            break;
          }
          tc_fence_after();
        }
        const uint32_t acc = tmem + (uint32_t)(buf * a.mt * a.acc_stride);
        for (int kb = 0; kb < a.nk; ++kb) {
          if (!mbar_wait(&S.full[s], ph, a.polls)) {
            atomicOr(&S.s_err, kErrCopyTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(ring + (size_t)s * sb);
          const uint64_t bd = umma_desc_k(st + (uint32_t)(a.mt * kDtATileBytes));
          for (int m = 0; m < a.mt; ++m) {
            const uint64_t ad = umma_desc_k(st + (uint32_t)(m * kDtATileBytes));
#pragma unroll
            for (int k = 0; k < kDtKBlock / 16; ++k)
              tc_mma_f16(acc + (uint32_t)(m * a.acc_stride), ad + 2u * k, bd + 2u * k, a.idesc,
                         (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&S.empty[s]);
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&S.acc_full[buf]);
      }
      // all MMAs of this thread complete before TMEM is released
      tc_commit(&S.drain);
      if (!mbar_wait(&S.drain, 0u, a.polls)) atomicOr(&S.s_err, kErrCopyTimeout);
    }
  } else {
    const int q = warp & 3;          // TMEM lane quadrant this warp may access
    const int hf = (warp - 2) >> 2;  // column half of the tile
    const int et = tid - 64;
    const int nc = a.n_tile >> 4;    // 16-column chunks per tile
    const int c_lo = hf ? (nc + 1) >> 1 : 0, c_hi = hf ? nc : (nc + 1) >> 1;
    unsigned long long bst[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int u = 0; u < 4; ++u) bst[m][u] = 0ull;
    bool ok = true;
    for (int t = t0, i = 0; t < t1; ++t, ++i) {
      const int v0 = t * a.n_tile;
      int *vid = S.vid[i & 1];
      for (int j = et; j < a.n_tile; j += kDtEpiThreads)
        vid[j] = v0 + j < a.V ? __ldg(&a.vocab_map[v0 + j]) : 0;
      nbar_sync(1, kDtEpiThreads);
      const int buf = i % n_acc, use = i / n_acc;
      if (ok && !mbar_wait(&S.acc_full[buf], (uint32_t)(use & 1), a.polls)) {
        atomicOr(&S.s_err, kErrCopyTimeout);
        ok = false;
      }
      __syncwarp();
      if (!ok) continue;
      tc_fence_after();
      const int n_valid = min(a.n_tile, a.V - v0);
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (m >= a.mt) break;
        const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) +
                              (uint32_t)((buf * a.mt + m) * a.acc_stride);
        // up to four 16-column loads in flight per wait
        for (int c = c_lo; c < c_hi; c += 4) {
          const int nq = min(4, c_hi - c);
          uint32_t v[4][16];
          tc_ld16(base + (uint32_t)(16 * c), v[0]);
          if (nq > 1) tc_ld16(base + (uint32_t)(16 * (c + 1)), v[1]);
          if (nq > 2) tc_ld16(base + (uint32_t)(16 * (c + 2)), v[2]);
          if (nq > 3) tc_ld16(base + (uint32_t)(16 * (c + 3)), v[3]);
          tc_wait_ld();
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (u < nq) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int col = 16 * (c + u) + j;
                if (col < n_valid) {
                  float key = sanitize(__uint_as_float(v[u][j]));
                  if (SAMPLE)
                    key = key / a.temperature +
                          gumbel(a.rng, kStageTokens,
                                 (uint32_t)(a.row_base + m * kDtMTile + 32 * q + lane),
                                 (uint32_t)vid[col]);
                  const unsigned long long w = pack(key, (uint32_t)vid[col]);
                  bst[m][j & 3] = w > bst[m][j & 3] ? w : bst[m][j & 3];
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cta(&S.acc_empty[buf]);
    }
    const int r0 = 32 * q + lane;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      unsigned long long best = bst[m][0];
#pragma unroll
      for (int u = 1; u < 4; ++u) best = bst[m][u] > best ? bst[m][u] : best;
      const int row = m * kDtMTile + r0;
      if (m < a.mt && row < a.rows && best) atomicMax(&a.packed[row], best);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kDtTmemCols)
                 : "memory");
  }
  if (tid == 0 && S.s_err) atomicOr(a.err, S.s_err);
}

}  // namespace fh
