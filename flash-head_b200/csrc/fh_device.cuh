// Device-side helpers shared by the FlashHead kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace fh {

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). A kernel launched with the
// programmatic-serialisation attribute may start while its predecessor is
// still running; grid_dep_wait() blocks until the predecessor grid has
// completed and its memory is visible. grid_dep_launch() lets the next kernel
// in the stream be scheduled early.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Packed (key, id) words. mono() maps fp32 onto uint32 so that unsigned order
// equals numeric order (-inf < ... < -0 < +0 < ... < +inf). The 64-bit word
// (mono(x) << 32) | (0xFFFFFFFF - id) is largest for the largest x and, among
// equal x, the smallest id: the reference's tie rule (fused.py:148-163).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t mono(float x) {
  uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unmono(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}
__device__ __forceinline__ unsigned long long pack(float x, uint32_t id) {
  return ((unsigned long long)mono(x) << 32) | (unsigned long long)(0xFFFFFFFFu - id);
}
__device__ __forceinline__ uint32_t packed_id(unsigned long long w) {
  return 0xFFFFFFFFu - (uint32_t)(w & 0xFFFFFFFFull);
}
// Exchange form for signed 64-bit reductions (NCCL/torch MAX on int64).
__device__ __forceinline__ long long to_signed(unsigned long long w) {
  return (long long)(w ^ 0x8000000000000000ull);
}
__device__ __forceinline__ unsigned long long from_signed(long long s) {
  return (unsigned long long)s ^ 0x8000000000000000ull;
}

// ---------------------------------------------------------------------------
// Philox-4x32-10 (Salmon et al., SC'11). Counter = (id, row, offset_lo,
// offset_hi[29:0] | stage << 30), key = seed. Only the first output word is
// used per (row, id).
// ---------------------------------------------------------------------------
constexpr uint32_t kStageClusters = 1;
constexpr uint32_t kStageTokens = 2;

__device__ __forceinline__ uint32_t philox_x0(uint32_t c0, uint32_t c1, uint32_t c2,
                                              uint32_t c3, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

struct RngKey {
  uint32_t k0, k1, off_lo, off_hi;
};

__device__ __forceinline__ float gumbel(const RngKey &key, uint32_t stage, uint32_t row,
                                        uint32_t id) {
  const uint32_t x = philox_x0(id, row, key.off_lo, (key.off_hi & 0x3FFFFFFFu) | (stage << 30),
                               key.k0, key.k1);
  const float u = ((float)(x >> 8) + 0.5f) * 5.9604644775390625e-8f;  // 2^-24
  return -logf(-logf(u));
}

// ---------------------------------------------------------------------------
// 16-byte vector -> fp32 products. A uint4 holds 8 bf16/fp16 or 16 fp8.
// ---------------------------------------------------------------------------
template <typename T>
struct Vec;

template <>
struct Vec<__nv_bfloat16> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void to_float(const uint4 &v, float *f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};

template <>
struct Vec<__half> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void to_float(const uint4 &v, float *f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h2 = *reinterpret_cast<const __half2 *>(&w[i]);
      float2 t = __half22float2(h2);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

template <>
struct Vec<__nv_fp8_e4m3> {
  static constexpr int kElems = 16;
  __device__ __forceinline__ static void to_float(const uint4 &v, float *f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2_raw lo =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xFFFFu), __NV_E4M3);
      const __half2_raw hi =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
      const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&lo));
      const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&hi));
      f[4 * i] = a.x;
      f[4 * i + 1] = a.y;
      f[4 * i + 2] = b.x;
      f[4 * i + 3] = b.y;
    }
  }
};

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  // Weight rows are read once per step: do not keep them in L1.
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg_keep(const void *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}

// ---------------------------------------------------------------------------
// Bulk asynchronous copies (TMA engine, no tensor map) into shared memory,
// completed on an mbarrier. Addresses 16-byte aligned, sizes multiples of 16.
// Every copy lands in the issuing CTA's own shared memory only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Fire-and-forget bulk prefetch of global memory into L2 (size multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false if the phase did not complete within max_polls polls.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t max_polls) {
  for (uint32_t i = 0; i < max_polls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 lds128(const void *p) {
  return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = t > v ? t : v;
  }
  return v;
}

// Block-wide exclusive prefix sum of one int per thread (blockDim multiple of
// 32, at most 1024). `scratch` holds 33 ints. Returns the exclusive prefix;
// *total receives the block total. Contains three __syncthreads(), the first
// of which protects `scratch` from a previous use.
__device__ __forceinline__ int block_exclusive_scan(int v, int *scratch, int *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  int x = v;
  __syncthreads();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += t;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < nwarps ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += t;
    }
    scratch[lane] = s;  // inclusive warp totals
    if (lane == 31) scratch[32] = s;
  }
  __syncthreads();
  const int before = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[32];
  return before + x - v;
}

// Ordered stream compaction over ids [0, N): calls emit(pos, i) for every i
// with pred(i), pos = rank of i among the selected ids (ascending). Warp w
// owns a contiguous id range and walks it 32 ids at a time (lane = id % 32,
// so shared-memory reads inside pred are conflict-free); ballots give the
// in-warp ranks and one barrier the cross-warp offsets. `warp_counts` holds
// one int per warp. Ends with __syncthreads().
template <typename Pred, typename Emit>
__device__ __forceinline__ void block_ordered_compact(int N, Pred pred, Emit emit,
                                                      int *warp_counts) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int per = (N + nw - 1) / nw;
  const int lo = min(N, warp * per), hi = min(N, lo + per);
  int cnt = 0;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    cnt += __popc(__ballot_sync(0xFFFFFFFFu, i < hi && pred(i)));
  }
  __syncthreads();  // warp_counts may still be read by a previous use
  if (lane == 0) warp_counts[warp] = cnt;
  __syncthreads();
  // this warp's first position: exclusive prefix of the warp counts (one scan)
  const int wc = lane < nw ? warp_counts[lane] : 0;
  int incl = wc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += t;
  }
  int off = __shfl_sync(0xFFFFFFFFu, incl - wc, warp);
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    const bool f = i < hi && pred(i);
    const unsigned m = __ballot_sync(0xFFFFFFFFu, f);
    if (f) emit(off + __popc(m & ((1u << lane) - 1u)), i);
    off += __popc(m);
  }
  __syncthreads();
}

}  // namespace fh
