// Stage 1 of a batched decode step on the 5th-generation tensor cores:
// partial scores P_s[r][k] = sum over the k-blocks of split s of
// C[k, :] . H[r, :], for the K stage-1 rows C (the normalised centroids, or
// the raw ones when sampling) and up to 256 hidden rows H. The reference
// computes cluster_linear(h) (src/flash_head/flash_head.py:213) or
// F.linear(h, centroids.t()) (:203-205) as a library GEMM.
//
// One CTA per (128-row tile of C, split of the hidden dimension), 6 warps:
//   warp 0     lane 0 issues TMA tensor copies of each k-block (64 elements):
//              the C tile (128 rows; fp8 rows land unswizzled, 16-bit rows
//              with the 128-byte swizzle the MMA reads) and the hidden tile
//              (n_pad rows, 128-byte swizzle, zero fill past the last row);
//   warp 1     allocates the TMEM accumulator; lane 0 issues
//              tcgen05.mma.kind::f16 (M = 128 C rows, N = n_pad hidden rows,
//              K = 16) per k-block and commits each stage back to the producer
//              and the finished accumulator to the epilogue;
//   warps 2-5  fp8 C: convert each k-block's 128 x 64 e4m3 tile into the f16
//              tile the MMA reads (exact: every e4m3 value is an f16 value),
//              written in the 128-byte swizzle layout; then, for every C,
//              read the accumulator (thread = one C row, tcgen05.ld 16
//              columns at a time) and store the partial scores, so that a warp
//              writes 32 consecutive clusters of one hidden row.
// With fp8 C the hidden rows must be f16 (the MMA takes one operand type);
// with 16-bit C they are in C's type. The splits' partials are summed, in
// split order, by the selection kernel, which also applies the fp8 row
// scale and the sampling keys. Every wait is bounded; on a timeout the
// kernel records kErrCopyTimeout, drains its own copies and MMAs (bounded)
// and frees TMEM before it returns.
#pragma once

#include "fh_dense_tc.cuh"

namespace fh {

constexpr int kS1Threads = 192;
constexpr int kS1EpiThreads = 128;  // warps 2..5
constexpr int kS1MTile = 128;       // C rows per tile (TMEM lanes)
constexpr int kS1MaxN = 256;        // hidden rows per launch (MMA N)
constexpr int kS1KBlock = 64;       // elements per k-block
constexpr int kS1A16Bytes = kS1MTile * 128;  // f16/bf16 C tile of one k-block
constexpr int kS1A8Bytes = kS1MTile * 64;    // fp8 C tile of one k-block
constexpr int kS1MaxStages = 16;
constexpr int kS1SmemMax = 227 * 1024;

struct S1TcArgs {
  int K;           // C rows
  int rows;        // hidden rows of this launch (1..kS1MaxN)
  int n_pad;       // MMA N: rows rounded up to a multiple of 16
  int nk;          // k-blocks: ceil(D / 64)
  int splits;      // k-block ranges (one per CTA of a tile)
  int stages;
  int fp8;         // C is e4m3 (converted in shared memory)
  int tmem_cols;   // power of two >= n_pad, >= 32
  uint32_t idesc;
  float *part;           // partial scores: part[s * split_stride + r * row_stride + k]
  size_t split_stride;   // floats
  int row_stride;        // floats
  uint32_t *err;
  uint32_t polls;
};

struct S1TcCtrl {
  uint64_t full[kS1MaxStages];   // TMA bytes of the stage landed
  uint64_t conv[kS1MaxStages];   // fp8 tile converted (kS1EpiThreads arrivals)
  uint64_t empty[kS1MaxStages];  // MMAs of the stage done: free for the producer
  uint64_t acc_full;
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t s_err;
};

// Stage layout: [C tile, 16-bit, swizzled | hidden tile | C tile, fp8 (fp8 only)].
__host__ __device__ inline size_t s1tc_stage_bytes(int n_pad, int fp8) {
  return (size_t)kS1A16Bytes + (size_t)n_pad * 128 + (fp8 ? (size_t)kS1A8Bytes : 0);
}
__host__ __device__ inline size_t s1tc_smem_bytes(int n_pad, int fp8, int stages) {
  return 1024 + (size_t)stages * s1tc_stage_bytes(n_pad, fp8) + sizeof(S1TcCtrl);
}
// Instruction descriptor of kind::f16 for M = 128: f32 accumulator, A and B
// both bf16 (or both f16), both K-major, N = n_pad.
__host__ __device__ inline uint32_t s1tc_idesc(bool bf16, int n_pad) {
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)(n_pad >> 3) << 17) |
         ((uint32_t)(kS1MTile >> 4) << 24);
}

// The MMA reads 128-byte-swizzled K-major tiles (see umma_desc_k): the 16-byte
// chunk c of row m of a tile sits at chunk c ^ (m & 7) of that row.
__device__ __forceinline__ void s1_convert_kblock(const unsigned char *a8, unsigned char *a16,
                                                  int t) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = t + kS1EpiThreads * i;  // 16-byte fp8 chunk: row m, chunk c8
    const int m = j >> 2, c8 = j & 3;
    const uint4 v = lds128(a8 + m * 64 + c8 * 16);
    uint4 lo, hi;
    lo.x = fp8x2_to_f16x2(v.x & 0xFFFFu);
    lo.y = fp8x2_to_f16x2(v.x >> 16);
    lo.z = fp8x2_to_f16x2(v.y & 0xFFFFu);
    lo.w = fp8x2_to_f16x2(v.y >> 16);
    hi.x = fp8x2_to_f16x2(v.z & 0xFFFFu);
    hi.y = fp8x2_to_f16x2(v.z >> 16);
    hi.z = fp8x2_to_f16x2(v.w & 0xFFFFu);
    hi.w = fp8x2_to_f16x2(v.w >> 16);
    unsigned char *row = a16 + m * 128;
    const int sw = m & 7;
    *reinterpret_cast<uint4 *>(row + (((2 * c8) ^ sw) << 4)) = lo;
    *reinterpret_cast<uint4 *>(row + (((2 * c8 + 1) ^ sw) << 4)) = hi;
  }
}

__global__ void __launch_bounds__(kS1Threads, 1)
    k_s1_tc(const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_h,
            S1TcArgs a) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  const uint32_t raw = smem_u32(dsm);
  unsigned char *ring = dsm + (((raw + 1023u) & ~1023u) - raw);
  const size_t sb = s1tc_stage_bytes(a.n_pad, a.fp8);
  S1TcCtrl &S = *reinterpret_cast<S1TcCtrl *>(ring + (size_t)a.stages * sb);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = blockIdx.x / a.splits, sp = blockIdx.x - mt * a.splits;
  const int kb0 = (int)((long long)sp * a.nk / a.splits);
  const int kb1 = (int)((long long)(sp + 1) * a.nk / a.splits);
  const uint32_t b_tx = (uint32_t)(a.n_pad * 128);
  const uint32_t c_tx = a.fp8 ? (uint32_t)kS1A8Bytes : (uint32_t)kS1A16Bytes;

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.conv[s], kS1EpiThreads);
      mbar_init(&S.empty[s], 1);
    }
    mbar_init(&S.acc_full, 1);
    mbar_init(&S.drain, 1);
    S.s_err = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S.tmem_base)),
                 "r"(a.tmem_cols)
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
      int issued[kS1MaxStages];  // parity of the last fill of each stage, -1: none
      for (int j = 0; j < kS1MaxStages; ++j) issued[j] = -1;
      // The hidden rows may come from the previous kernel in the stream (the
      // f16 copy): wait for it before the first copy of them.
      grid_dep_wait();
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&S.empty[s], ph ^ 1u, a.polls)) {
          atomicOr(&S.s_err, kErrCopyTimeout);
          break;
        }
        unsigned char *st = ring + (size_t)s * sb;
        mbar_expect_tx(&S.full[s], c_tx + b_tx);
        tma_load_2d(a.fp8 ? st + kS1A16Bytes + b_tx : st, &tm_c, kb * kS1KBlock,
                    mt * kS1MTile, &S.full[s]);
        tma_load_2d(st + kS1A16Bytes, &tm_h, kb * kS1KBlock, 0, &S.full[s]);
        issued[s] = (int)ph;
        if (++s == a.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      for (int j = 0; j < a.stages; ++j)
        if (issued[j] >= 0 && !mbar_wait(&S.full[j], (uint32_t)issued[j], a.polls))
          atomicOr(&S.s_err, kErrCopyTimeout);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0u;
      bool ok = true;
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        if (!mbar_wait(&S.full[s], ph, a.polls) ||
            (a.fp8 && !mbar_wait(&S.conv[s], ph, a.polls))) {
          atomicOr(&S.s_err, kErrCopyTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(ring + (size_t)s * sb);
        const uint64_t ad = umma_desc_k(st);
        const uint64_t bd = umma_desc_k(st + (uint32_t)kS1A16Bytes);
#pragma unroll
        for (int k = 0; k < kS1KBlock / 16; ++k)
          tc_mma_f16(tmem, ad + 2u * k, bd + 2u * k, a.idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        tc_commit(&S.empty[s]);
        if (++s == a.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (ok) tc_commit(&S.acc_full);
      tc_commit(&S.drain);
      if (!mbar_wait(&S.drain, 0u, a.polls)) atomicOr(&S.s_err, kErrCopyTimeout);
    }
  } else {
    const int et = tid - 64;
    bool ok = true;
    if (a.fp8) {
      int s = 0;
      uint32_t ph = 0u;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (ok && !mbar_wait(&S.full[s], ph, a.polls)) {
          atomicOr(&S.s_err, kErrCopyTimeout);
          ok = false;
        }
        unsigned char *st = ring + (size_t)s * sb;
        if (ok) s1_convert_kblock(st + kS1A16Bytes + b_tx, st, et);
        // generic-proxy writes of the f16 tile become visible to the MMA
        fence_proxy_async_smem();
        mbar_arrive_cta(&S.conv[s]);
        if (++s == a.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    if (ok && !mbar_wait(&S.acc_full, 0u, a.polls)) {
      atomicOr(&S.s_err, kErrCopyTimeout);
      ok = false;
    }
    __syncwarp();
    if (ok) {
      tc_fence_after();
      const int q = warp & 3;  // TMEM lane quadrant of this warp
      const int m = 32 * q + lane;
      const int k = mt * kS1MTile + m;
      float *out = a.part + (size_t)sp * a.split_stride + k;
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16);
      for (int c = 0; c < a.n_pad; c += 64) {
        const int nq = min(4, (a.n_pad - c) >> 4);
        uint32_t v[4][16];
        tc_ld16(base + (uint32_t)c, v[0]);
        if (nq > 1) tc_ld16(base + (uint32_t)(c + 16), v[1]);
        if (nq > 2) tc_ld16(base + (uint32_t)(c + 32), v[2]);
        if (nq > 3) tc_ld16(base + (uint32_t)(c + 48), v[3]);
        tc_wait_ld();
        if (k < a.K) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (u < nq) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int r = c + 16 * u + j;
                if (r < a.rows) out[(size_t)r * a.row_stride] = __uint_as_float(v[u][j]);
              }
            }
          }
        }
      }
    }
  }
  // Let the selection kernel's CTAs be scheduled; they wait for this grid's
  // completion before reading the partials.
  grid_dep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(a.tmem_cols)
                 : "memory");
  }
  if (tid == 0 && S.s_err) atomicOr(a.err, S.s_err);
}

// f16 copy of bf16 hidden rows (the operand type of an fp8 stage-1 MMA):
// 8 elements per thread and step. Values outside the f16 range saturate to
// +-inf like any f16 conversion.
__global__ void k_hidden_to_f16(const uint4 *src, uint4 *dst, int n8) {
  grid_dep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
      const __half2 h = __floats2half2_rn(lo, hi);
      o[j] = *reinterpret_cast<const uint32_t *>(&h);
    }
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace fh
