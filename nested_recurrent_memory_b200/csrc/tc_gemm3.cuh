// fp32 products on the tensor cores for the CUDA-core kernels: each fp32
// operand is split into a bf16 high part and a bf16 low part (x - hi), and
// C = A_hi B_hi + A_hi B_lo + A_lo B_hi is accumulated in fp32 in tensor
// memory (about 16 significant bits per product; the dropped A_lo B_lo term
// is below 2^-16 of it). One CTA of 256 threads: all threads stage the
// operands straight into the no-swizzle core-matrix layouts of tc_ptx.cuh,
// one thread issues the tcgen05.mma instructions, every wait is bounded.
#pragma once

#include <cuda_bf16.h>

#include "tc_ptx.cuh"

namespace ngdn2 {
namespace tc {

// Tiles staged per K-chunk: A 128 x 64 and B 64 x 128, each as hi and lo.
constexpr int kTc3Chunk = 64;
constexpr int kTc3StageBytes = 4 * 128 * kTc3Chunk * 2;  // A_hi | A_lo | B_hi | B_lo
constexpr int kTc3TmemCols = 128;

// Per-CTA state: the TMEM accumulator (kTc3TmemCols columns), one mbarrier
// for MMA completion with its next parity, the staging buffer (1024-byte
// aligned shared memory of kTc3StageBytes), and a timeout flag.
struct Tc3Ctx {
  uint32_t tmem;
  uint64_t* bar;
  uint32_t phase;
  uint8_t* stage;
  int* abort_flag;
};

// Eight consecutive fp32 values as bf16 hi and lo halves, packed for one
// 16-byte core-matrix row each.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat16 h0 = __float2bfloat16_rn(x[2 * i]);
    const __nv_bfloat16 h1 = __float2bfloat16_rn(x[2 * i + 1]);
    const __nv_bfloat16 l0 = __float2bfloat16_rn(x[2 * i] - __bfloat162float(h0));
    const __nv_bfloat16 l1 = __float2bfloat16_rn(x[2 * i + 1] - __bfloat162float(h1));
    h[i] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) |
           (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
    l[i] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) |
           (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Eight consecutive-in-k (AT: strided) values of A row r, or of B row k.
template <bool T>
__device__ __forceinline__ void load8_op(const float* src, int64_t ld, float* x) {
  if (!T && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const float4 v0 = reinterpret_cast<const float4*>(src)[0];
    const float4 v1 = reinterpret_cast<const float4*>(src)[1];
    x[0] = v0.x; x[1] = v0.y; x[2] = v0.z; x[3] = v0.w;
    x[4] = v1.x; x[5] = v1.y; x[6] = v1.z; x[7] = v1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = src[T ? int64_t(j) * ld : j];
  }
}

// C[M x N] = A[M x Kd] . B[Kd x N] for M <= 128, N <= 128 a multiple of 16,
// Kd a multiple of 16. A(m, k) is A[m * lda + k] (AT: A[k * lda + m]); B(k, n)
// is B[k * ldb + n] (BT: B[n * ldb + k]); operands are fp32 in global memory.
// For every output element of rows < M, old = ld(m, n) then epi(m, n, c, old)
// (consecutive threads on consecutive n; each thread issues all its ld
// before its first epi, so an epilogue that reads what it updates keeps its
// loads in flight together). Every thread of the CTA must call it; it
// synchronises on entry and on exit.
template <bool AT = false, bool BT = false, class Ld, class Epi>
__device__ void tc_gemm3(Tc3Ctx& c, int M, int N, int Kd, const float* A, int64_t lda,
                         const float* B, int64_t ldb, Ld ld, Epi epi) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* a_hi = c.stage;
  uint8_t* a_lo = a_hi + 128 * kTc3Chunk * 2;
  uint8_t* b_hi = a_lo + 128 * kTc3Chunk * 2;
  uint8_t* b_lo = b_hi + 128 * kTc3Chunk * 2;
  const uint32_t idesc = idesc_f16(128, N, true, false, true);
  constexpr int kU = 128 * (kTc3Chunk / 8) / 256;  // staging units a thread, per operand
  for (int k0 = 0; k0 < Kd; k0 += kTc3Chunk) {
    const int kc = min(kTc3Chunk, Kd - k0), kg = kc / 8;
    // A: unit (row r, 8-column group g) -> one 16-byte core-matrix row of
    // each half; eight consecutive threads take eight rows of one core
    // matrix (128 contiguous bytes). All of a thread's loads first.
    {
      float x[kU][8];
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int u = tid + 256 * q;
        const int r = (u & 7) + 8 * (u / (8 * kg)), g = (u >> 3) % kg;
        if (u < 128 * kg && r < M) {
          load8_op<AT>(A + (AT ? int64_t(k0 + 8 * g) * lda + r : int64_t(r) * lda + k0 + 8 * g),
                       lda, x[q]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) x[q][j] = 0.f;
        }
      }
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int u = tid + 256 * q;
        if (u < 128 * kg) {
          const int r = (u & 7) + 8 * (u / (8 * kg)), g = (u >> 3) % kg;
          uint4 h, l;
          split8(x[q], h, l);
          const int off = kmajor_off(r, 8 * g, kc) * 2;
          *reinterpret_cast<uint4*>(a_hi + off) = h;
          *reinterpret_cast<uint4*>(a_lo + off) = l;
        }
      }
    }
    // B: unit (k, 8-column group of n) -> one MN-major core-matrix row.
    {
      const int ng = N / 8;
      float x[kU][8];
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int u = tid + 256 * q;
        const int k = (u & 7) + 8 * (u / (8 * ng)), g = (u >> 3) % ng;
        if (u < kc * ng) {
          load8_op<BT>(B + (BT ? int64_t(8 * g) * ldb + k0 + k : int64_t(k0 + k) * ldb + 8 * g),
                       ldb, x[q]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) x[q][j] = 0.f;
        }
      }
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int u = tid + 256 * q;
        if (u < kc * ng) {
          const int k = (u & 7) + 8 * (u / (8 * ng)), g = (u >> 3) % ng;
          uint4 h, l;
          split8(x[q], h, l);
          const int off = mnmajor_off(k, 8 * g, kc) * 2;
          *reinterpret_cast<uint4*>(b_hi + off) = h;
          *reinterpret_cast<uint4*>(b_lo + off) = l;
        }
      }
    }
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      fence_after_sync();
      const uint32_t ah = smem_u32(a_hi), al = smem_u32(a_lo);
      const uint32_t bh = smem_u32(b_hi), bl = smem_u32(b_lo);
      for (int kk = 0; kk < kc / 16; ++kk) {
        const uint64_t dah = desc_tile(ah, kc, kk), dal = desc_tile(al, kc, kk);
        const uint64_t dbh = desc_tile(bh, kc, kk), dbl = desc_tile(bl, kc, kk);
        mma_f16(c.tmem, dah, dbh, idesc, (k0 > 0 || kk > 0) ? 1u : 0u);
        mma_f16(c.tmem, dah, dbl, idesc, 1u);
        mma_f16(c.tmem, dal, dbh, idesc, 1u);
      }
      mma_commit(c.bar);
    }
    // The MMAs must have read the staging buffer before it is refilled (and
    // written the accumulator before it is read).
    if (!mbar_wait(c.bar, c.phase)) *c.abort_flag = 1;
    c.phase ^= 1u;
    fence_after_sync();
  }
  // Read-out in two column halves through the (now free) staging buffer:
  // warp w reads TMEM lanes 32 (w % 4) .. +31 (rows), the warps w < 4 the
  // even and w >= 4 the odd 8-column groups of the half, and writes them
  // row-major; then the epilogue walks the rows with consecutive threads on
  // consecutive columns, so its global accesses are coalesced.
  const int row = 32 * (warp & 3) + lane, W = N / 2, ldo = W + 4;
  float* out = reinterpret_cast<float*>(c.stage);
  for (int half = 0; half < 2; ++half) {
    for (int c0 = 8 * (warp >> 2); c0 < W; c0 += 16) {
      uint32_t r[8];
      tmem_ld8_nowait(taddr(c.tmem, 32 * (warp & 3), half * W + c0), r);
      tmem_wait_ld();
      tmem_regs_after_wait8(r);
      float4* o4 = reinterpret_cast<float4*>(out + row * ldo + c0);
      o4[0] = make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]), __uint_as_float(r[2]),
                          __uint_as_float(r[3]));
      o4[1] = make_float4(__uint_as_float(r[4]), __uint_as_float(r[5]), __uint_as_float(r[6]),
                          __uint_as_float(r[7]));
    }
    __syncthreads();
    // Each thread keeps one column n (W divides 256 for every N a power of
    // two times 16, else a general walk) and loads all its old values (at
    // most 32) before the first update: an update waits for its load, and a
    // later load may not pass an earlier store.
    if (256 % W == 0) {
      const int n = tid % W, m0 = tid / W, step = 256 / W;
      constexpr int kE = 128 * (kTc3TmemCols / 2) / 256;
      float old[kE];
#pragma unroll
      for (int q = 0; q < kE; ++q) {
        const int m = m0 + step * q;
        old[q] = m < M ? ld(m, half * W + n) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < kE; ++q) {
        const int m = m0 + step * q;
        if (m < M) epi(m, half * W + n, out[m * ldo + n], old[q]);
      }
    } else {
      for (int e = tid; e < M * W; e += 256) {
        const int m = e / W, n = e % W;
        epi(m, half * W + n, out[m * ldo + n], ld(m, half * W + n));
      }
    }
    __syncthreads();
  }
  fence_before_sync();
  __syncthreads();
}

}  // namespace tc
}  // namespace ngdn2
