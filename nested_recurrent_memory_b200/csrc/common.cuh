// Shared device helpers for the nested GDN-2 kernels: element loads with
// conversion to fp32, stores from fp32, a block-wide fp32 GEMM used by the
// CUDA-core path, and the math of the promotion gates.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ngdn2.h"

namespace ngdn2 {

// ---------------------------------------------------------------------------
// Element conversion
// ---------------------------------------------------------------------------

__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case NGDN2_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case NGDN2_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

// load_elem with the dtype known at compile time (for loops whose loads
// should all be in flight at once).
template <int DT>
__device__ __forceinline__ float load_typed(const void* p, int64_t i) {
  if constexpr (DT == NGDN2_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  else if constexpr (DT == NGDN2_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  else return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, float x, int dtype) {
  switch (dtype) {
    case NGDN2_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x); break;
    case NGDN2_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(x); break;
    default: reinterpret_cast<float*>(p)[i] = x; break;
  }
}

// ---------------------------------------------------------------------------
// Gate activations of the promotion probe (nested_gdn2/ops/probe.py:34-66)
// ---------------------------------------------------------------------------

constexpr float kBLogitInit = -4.0f;  // probe.py:28
constexpr float kWLogitInit = 0.0f;   // probe.py:29
constexpr float kGLogitInit = -4.0f;  // probe.py:31

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplusf_(float x) {
  return x > 20.0f ? x : log1pf(expf(x));
}

// ---------------------------------------------------------------------------
// Block-wide fp32 GEMM on CUDA cores
//
// For m < M, n < N: epi(m, n, sum_k la(m, k) * lb(k, n)).
// ``la`` and ``lb`` are element loaders (so strides, transposes, dtype
// conversion and elementwise pre-products are free); AT / BT say that the
// loader's source is contiguous along m (A) / along k (B) rather than along
// k / n, so that the tile loads are issued in the coalesced order; PF = false
// loads each tile straight into shared memory when the previous one is
// consumed (fewer live registers, for kernels at their register cap); operands are staged
// through shared memory in 64x16 and 16x64 tiles (the next tile's elements
// load into registers during the current tile's FMAs) and each thread owns
// 4x4 outputs of the 64x64 tile at a stride of 16 (rows tm + 16 i, columns
// tn + 16 j): a warp's operand reads then touch 2 (A) and 16 consecutive (B)
// words, one shared-memory wavefront each, and its epilogue writes runs of
// 16 consecutive columns. The block needs at least kGemmThreads threads (more
// only join the barriers) and every thread must call it (it synchronises). M and N are arbitrary; Kd
// must be a multiple of 16. ``smem`` holds kGemmSmemFloats floats.
// ---------------------------------------------------------------------------

// dst[e] = op(e, src[e]) for e < n over the whole block (dst may be src):
// float4 accesses with U loads in flight per thread when both pointers are
// 16-byte aligned and n is a multiple of 4, else one element at a time.
// For global-memory loops, where one dependent load per iteration would
// cost a full L2 round trip each.
template <int U = 4, class Op>
__device__ __forceinline__ void block_map(float* dst, const float* src, int n, Op op) {
  const int tid = threadIdx.x, nth = blockDim.x;
  if ((((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) &&
      (n & 3) == 0) {
    const int n4 = n >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int base = tid; base < n4; base += U * nth) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * nth;
        v[u] = i < n4 ? s4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * nth;
        if (i < n4) {
          float4 r = v[u];
          r.x = op(4 * i, r.x);
          r.y = op(4 * i + 1, r.y);
          r.z = op(4 * i + 2, r.z);
          r.w = op(4 * i + 3, r.w);
          d4[i] = r;
        }
      }
    }
  } else {
    for (int e = tid; e < n; e += nth) dst[e] = op(e, src[e]);
  }
}

// out(r, sum_c X[r * cols + c]) for r < rows: a warp per row, lanes along
// the row (coalesced), then a shuffle reduction (a fixed order, so the sums
// are reproducible). Lane 0 calls out.
template <class Out>
__device__ __forceinline__ void row_sums(const float* X, int rows, int cols, Out out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  for (int r = warp; r < rows; r += nwarp) {
    float s = 0.f;
#pragma unroll 4
    for (int c = lane; c < cols; c += 32) s += X[int64_t(r) * cols + c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out(r, s);
  }
}

constexpr int kGemmThreads = 256;
constexpr int kGemmLd = 65;
constexpr int kGemmSmemFloats = 2 * 16 * kGemmLd;

template <bool AT = false, bool BT = false, bool PF = true, class LA, class LB, class Epi>
__device__ void block_gemm(int M, int N, int Kd, LA la, LB lb, float* smem, Epi epi) {
  float* As = smem;                 // [16][65], k-major
  float* Bs = smem + 16 * kGemmLd;  // [16][65]
  const int tid = threadIdx.x;
  const bool act = tid < kGemmThreads;  // larger blocks: the rest only join the barriers
  const int tm = tid / 16;
  const int tn = tid % 16;
  constexpr int kPer = 64 * 16 / kGemmThreads;  // tile elements each thread stages
  for (int m0 = 0; m0 < M; m0 += 64) {
    for (int n0 = 0; n0 < N; n0 += 64) {
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      if constexpr (!PF) {
        for (int k0 = 0; k0 < Kd; k0 += 16) {
          if (act) {
            for (int e = tid; e < 64 * 16; e += kGemmThreads) {
              const int mm = AT ? e % 64 : e / 16, ka = AT ? e / 64 : e % 16;
              As[ka * kGemmLd + mm] = m0 + mm < M ? la(m0 + mm, k0 + ka) : 0.f;
            }
            for (int e = tid; e < 64 * 16; e += kGemmThreads) {
              const int kb = BT ? e % 16 : e / 64, nn = BT ? e / 16 : e % 64;
              Bs[kb * kGemmLd + nn] = n0 + nn < N ? lb(k0 + kb, n0 + nn) : 0.f;
            }
          }
          __syncthreads();
          if (act) {
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) {
              float a[4], bb[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) a[i] = As[kk * kGemmLd + tm + 16 * i];
#pragma unroll
              for (int j = 0; j < 4; ++j) bb[j] = Bs[kk * kGemmLd + tn + 16 * j];
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
            }
          }
          __syncthreads();
        }
      } else {
      // The next k-step's elements are loaded into registers while the
      // current one is multiplied, so operand latency overlaps the FMAs.
      float ra[kPer], rb[kPer];
      auto fetch = [&](int k0) {
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
          const int e = tid + q * kGemmThreads;
          const int mm = AT ? e % 64 : e / 16, ka = AT ? e / 64 : e % 16;
          const int kb = BT ? e % 16 : e / 64, nn = BT ? e / 16 : e % 64;
          ra[q] = m0 + mm < M ? la(m0 + mm, k0 + ka) : 0.f;
          rb[q] = n0 + nn < N ? lb(k0 + kb, n0 + nn) : 0.f;
        }
      };
      if (act) fetch(0);
      for (int k0 = 0; k0 < Kd; k0 += 16) {
        if (act) {
#pragma unroll
          for (int q = 0; q < kPer; ++q) {
            const int e = tid + q * kGemmThreads;
            if (AT) As[(e / 64) * kGemmLd + e % 64] = ra[q];
            else As[(e % 16) * kGemmLd + e / 16] = ra[q];
            if (BT) Bs[(e % 16) * kGemmLd + e / 16] = rb[q];
            else Bs[(e / 64) * kGemmLd + e % 64] = rb[q];
          }
        }
        __syncthreads();
        if (act) {
          if (k0 + 16 < Kd) fetch(k0 + 16);
#pragma unroll
          for (int kk = 0; kk < 16; ++kk) {
            float a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk * kGemmLd + tm + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bb[j] = Bs[kk * kGemmLd + tn + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
          }
        }
        __syncthreads();
      }
      }
      if (act) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int gm = m0 + tm + 16 * i, gn = n0 + tn + 16 * j;
            if (gm < M && gn < N) epi(gm, gn, acc[i][j]);
          }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// block_gemm_cp: the same product as block_gemm for operands that are plain
// strided arrays in global memory, staged into shared memory by cp.async
// (4-byte copies, zero-filled past M / N) through 3-4 buffers. The copies
// for the next k-steps are in flight while a step is multiplied, across
// output-tile boundaries, and need no registers. Output tiles are 64 x 128
// (4 x 8 outputs a thread at a stride of 16) when N > 64, else 64 x 64.
// A(m, k) is A[m * lda + k] (AT: A[k * lda + m]); B(k, n) is B[k * ldb + n]
// (BT: B[n * ldb + k]). The epilogue runs as each output tile completes,
// while later copies are in flight, so it must not write what A or B read.
// smem holds kGemmCpSmemFloats floats; Kd must be a multiple of 16; every
// thread of the block must call it.
// ---------------------------------------------------------------------------

constexpr int kCpStages = 4;
// The 64 x 128 variant (4 x 8 outputs a thread) keeps three stages.
constexpr int kCpStagesWide = 3;
constexpr int kGemmLdWide = 129;
constexpr int kGemmCpSmemFloats =
    kCpStages * 2 * 16 * kGemmLd > kCpStagesWide * 16 * (kGemmLd + kGemmLdWide)
        ? kCpStages * 2 * 16 * kGemmLd
        : kCpStagesWide * 16 * (kGemmLd + kGemmLdWide);

__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gsrc, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(gsrc),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Stage g of block_gemm_cp (TN columns a thread: 64 x 16 TN tiles): the
// cp.async copies of its A and B tiles, then a commit (by every thread,
// every call, so the group counts stay uniform).
template <bool AT, bool BT, int TN>
__device__ __forceinline__ void gemm_cp_issue(int g, int total, int nk, int ntn, int M, int N,
                                              const float* A, int64_t lda, const float* B,
                                              int64_t ldb, float* smem) {
  constexpr int NW = 16 * TN, LDB = NW + 1, ST = TN == 4 ? kCpStages : kCpStagesWide;
  const int tid = threadIdx.x;
  if (g < total && tid < kGemmThreads) {
    const int tile = g / nk, k0 = (g % nk) * 16;
    const int m0 = (tile / ntn) * 64, n0 = (tile % ntn) * NW;
    float* As = smem + (g % ST) * (16 * (kGemmLd + LDB));
    float* Bs = As + 16 * kGemmLd;
#pragma unroll
    for (int q = 0; q < 64 * 16 / kGemmThreads; ++q) {
      const int e = tid + q * kGemmThreads;
      const int mm = AT ? e % 64 : e / 16, ka = AT ? e / 64 : e % 16;
      const bool va = m0 + mm < M;
      const float* sa = AT ? A + int64_t(k0 + ka) * lda + (m0 + mm)
                           : A + int64_t(m0 + mm) * lda + (k0 + ka);
      cp_async4(As + ka * kGemmLd + mm, va ? sa : A, va);
    }
#pragma unroll
    for (int q = 0; q < NW * 16 / kGemmThreads; ++q) {
      const int e = tid + q * kGemmThreads;
      const int kb = BT ? e % 16 : e / NW, nn = BT ? e / 16 : e % NW;
      const bool vb = n0 + nn < N;
      const float* sb = BT ? B + int64_t(n0 + nn) * ldb + (k0 + kb)
                           : B + int64_t(k0 + kb) * ldb + (n0 + nn);
      cp_async4(Bs + kb * LDB + nn, vb ? sb : B, vb);
    }
  }
  cp_async_commit();
}

template <bool AT, bool BT, int TN, class Epi>
__device__ __forceinline__ void block_gemm_cp_t(int M, int N, int Kd, const float* A, int64_t lda,
                                                const float* B, int64_t ldb, float* smem, Epi epi) {
  constexpr int NW = 16 * TN, LDB = NW + 1, ST = TN == 4 ? kCpStages : kCpStagesWide;
  constexpr int kStage = 16 * (kGemmLd + LDB);
  const int tid = threadIdx.x;
  const bool act = tid < kGemmThreads;
  const int tm = tid / 16, tn = tid % 16;
  const int ntn = (N + NW - 1) / NW, nk = Kd / 16;
  const int total = ((M + 63) / 64) * ntn * nk;
#pragma unroll
  for (int st = 0; st < ST - 1; ++st)
    gemm_cp_issue<AT, BT, TN>(st, total, nk, ntn, M, N, A, lda, B, ldb, smem);
  const int ntiles = total / nk;
  int g = 0;
  for (int tile = 0; tile < ntiles; ++tile) {
    float acc[4][TN];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
    for (int kt = 0; kt < nk; ++kt, ++g) {
      cp_async_wait<ST - 2>();
      __syncthreads();  // stage g landed for every thread; stage g - 1 is consumed
      gemm_cp_issue<AT, BT, TN>(g + ST - 1, total, nk, ntn, M, N, A, lda, B, ldb, smem);
      if (act) {
        const float* As = smem + (g % ST) * kStage;
        const float* Bs = As + 16 * kGemmLd;
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          float a[4], bb[TN];
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = As[kk * kGemmLd + tm + 16 * i];
#pragma unroll
          for (int j = 0; j < TN; ++j) bb[j] = Bs[kk * LDB + tn + 16 * j];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
        }
      }
    }
    if (act) {
      const int m0 = (tile / ntn) * 64, n0 = (tile % ntn) * NW;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int gm = m0 + tm + 16 * i, gn = n0 + tn + 16 * j;
          if (gm < M && gn < N) epi(gm, gn, acc[i][j]);
        }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
}

// Products with N > 64 take 64 x 128 tiles (4 x 8 outputs a thread, twice
// the multiply-adds per shared-memory read), others 64 x 64.
template <bool AT = false, bool BT = false, class Epi>
__device__ __forceinline__ void block_gemm_cp(int M, int N, int Kd, const float* A, int64_t lda,
                                              const float* B, int64_t ldb, float* smem, Epi epi) {
  if (N > 64) block_gemm_cp_t<AT, BT, 8>(M, N, Kd, A, lda, B, ldb, smem, epi);
  else block_gemm_cp_t<AT, BT, 4>(M, N, Kd, A, lda, B, ldb, smem, epi);
}

}  // namespace ngdn2
