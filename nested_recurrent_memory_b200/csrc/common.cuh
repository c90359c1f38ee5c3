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

}  // namespace ngdn2
