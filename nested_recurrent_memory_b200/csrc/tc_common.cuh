// Pieces shared by the tensor-core (tcgen05) kernel files: tile sizes, the
// chunk record and promotion-operand layouts written by the prep and
// parameter kernels, the workspace layout of the fused family, and small
// device helpers (16-bit packing, element loads, gate activations).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "fwd_params.cuh"
#include "tc_ptx.cuh"

namespace ngdn2 {
namespace tcx {

using bf16 = __nv_bfloat16;
using namespace tc;

constexpr int TK = 128;         // key dim handled by this family
constexpr int TV = 128;         // value dim
constexpr int TILE_QK = kC * TK * 2;   // bytes of a [64 x 128] bf16 tile
constexpr int TILE_A = kC * kC * 2;    // bytes of a [64 x 64] bf16 tile

// Byte offsets inside one chunk record of the tensor-core family. The
// upper levels' read queries are not in it: the scan loads them from q
// itself with the tensor memory accelerator and applies mix * scale.
struct TcRecord {
  int64_t W, Q, Kt, A, U, eg, load_bytes, size;
  __host__ __device__ static TcRecord make(int L) {
    (void)L;
    TcRecord r;
    r.W = 0;                                  // [64 x K] K-major A operand
    r.Q = r.W + TILE_QK;                      // [64 x K] level-0 read queries, K-major
    r.Kt = r.Q + TILE_QK;                     // [64 tok x K] MN-major A operand (K_tail^T)
    r.A = r.Kt + TILE_QK;                     // [64 x 64] K-major A operand
    r.load_bytes = r.A + TILE_A;              // the part the scan copies to smem
    r.U = r.load_bytes;                       // [V/8][64 rows][8] bf16 (16-byte pieces)
    r.eg = r.U + kC * TV * 2;                 // [K] fp32 e^(G_last)
    r.size = (r.eg + TK * 4 + 127) & ~int64_t(127);
    return r;
  }
};

// Promotion operands of one (level, head), bf16, in the scan's shared-memory
// layouts: the query bank as a K-major A operand padded to 64 or 128 rows
// with zeros, and the two B operands of the gate GEMMs
// [W_k^T | W_b] and [W_w | W_g] (N = 256 each, K-major over V).
constexpr int64_t PT_QB = 0;
constexpr int64_t PT_W2A = 32768;
constexpr int64_t PT_W2B = PT_W2A + 65536;
constexpr int64_t PT_SIZE = PT_W2B + 65536;

// Workspace of the fused family: the promotion operands (bf16, per level
// and head), the chunk records, and the learned arm's fp32 masters of the
// upper levels (lane-major, lm_off, per (b, h)).
struct TcLayout {
  TcRecord rec;
  int64_t ptc_off, chunks_off, mast_off, total;
};

__host__ __device__ inline TcLayout tc_layout(const FwdParams& p) {
  TcLayout t;
  t.rec = TcRecord::make(p.L);
  t.ptc_off = 0;
  t.chunks_off = t.ptc_off + int64_t(p.L > 1 ? p.L - 1 : 0) * p.H * PT_SIZE;
  t.mast_off = t.chunks_off + int64_t(p.B) * p.H * p.NT * t.rec.size;
  t.mast_off = (t.mast_off + 255) & ~int64_t(255);
  t.total = t.mast_off + int64_t(p.B) * p.H * (p.L > 1 ? p.L - 1 : 0) * TK * TV * 4;
  return t;
}

// Rows of the promotion MMAs for ``nq`` pairs: 64 or 128.
__host__ __device__ inline int pad_pairs(int nq) { return nq <= 64 ? 64 : 128; }

__device__ __forceinline__ void set_status(const FwdParams& p, int bits) {
  if (p.status) atomicOr(p.status, bits);
}

// Gate activations of the promotion on the tensor-core path, from the fast
// hardware exponential / logarithm / reciprocal (outputs feed bf16 MMA
// operands or fp32 decays averaged over pairs).
__device__ __forceinline__ float fast_sigmoid(float x) {
  return __fdividef(1.f, 1.f + __expf(fminf(-x, 80.f)));
}
// softplus(x) = max(x, 0) + log(1 + e^-|x|) with the hardware exponential
// and logarithm (absolute error about 1e-7; the decay gate's values are
// rounded to fp16 partials right after).
__device__ __forceinline__ float softplus_fast(float x) {
  return fmaxf(x, 0.f) + __logf(1.f + __expf(-fabsf(x)));
}
// sigmoid(x) = (1 + tanh(x / 2)) / 2 with the hardware tanh (absolute error
// about 2.5e-4): used for the write gate, whose values sit near 1/2 and
// only scale a bf16 operand.
__device__ __forceinline__ float sigmoid_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return fmaf(0.5f, t, 0.5f);
}

// 8 consecutive elements starting at element offset ``o`` (element stride
// ``sd``), as fp32. Uses one 16-byte load when the data are contiguous and
// 16-byte aligned, else element loads.
__device__ __forceinline__ void load8_raw(const void* p, int dt, int64_t o, int64_t sd, float* out) {
  const bool aligned16 = (reinterpret_cast<uintptr_t>(p) & 15) == 0;
  if (sd == 1 && aligned16) {
    if (dt != NGDN2_F32 && (o & 7) == 0) {
      const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + o);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f;
        if (dt == NGDN2_BF16) f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        else f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
      }
      return;
    }
    if (dt == NGDN2_F32 && (o & 3) == 0) {
      const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + o);
      const float4 c = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + o + 4);
      out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
      out[4] = c.x; out[5] = c.y; out[6] = c.z; out[7] = c.w;
      return;
    }
  }
  if (sd == 0) {
    // A broadcast (stride-0) channel dimension: one element, eight times.
    const float x = load_elem(p, o, dt);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = x;
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = load_elem(p, o + i * sd, dt);
}

__device__ __forceinline__ void load8(const TokView& tv, int b, int t, int h, int d, float* out) {
  load8_raw(tv.p, tv.dt, tv.off(b, t, h, d), tv.sd, out);
}


// 8 consecutive 16-bit elements of a token row as their raw 16 bytes: one
// vector load when contiguous and aligned, else element loads re-packed in
// the tensor's own 16-bit format (exact).
__device__ __forceinline__ uint4 raw8_at(const void* p, int dt, int64_t o, int64_t sd) {
  if (sd == 1 && (o & 7) == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0)
    return __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + o));
  if (sd == 0) {
    // A broadcast (stride-0) channel dimension: one element, eight times.
    const uint32_t v = __ldg(reinterpret_cast<const uint16_t*>(p) + o);
    const uint32_t w2 = v | (v << 16);
    return make_uint4(w2, w2, w2, w2);
  }
  uint4 r;
  uint16_t* h = reinterpret_cast<uint16_t*>(&r);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = reinterpret_cast<const uint16_t*>(p)[o + i * sd];
  (void)dt;
  return r;
}

__device__ __forceinline__ void unpack8(const uint4& raw, int dt, float* out) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if (dt == NGDN2_BF16) f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    else f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

// Pack 8 floats as 8 bf16 (16 bytes).
__device__ __forceinline__ uint4 pack8(const float* x) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v2 = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&v2);
  }
  return r;
}

// Pack 8 floats as 8 fp16 (16 bytes).
__device__ __forceinline__ uint4 pack8h(const float* x) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 hh = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&hh);
  }
  return r;
}


// Tensor maps of the prep inputs for L2 prefetches: q (level 0), g, k, b, v,
// w, each a 3-D view [H][B * T][K] whose (K, 64, 1) box is one chunk's rows
// of one head. ``valid`` has bit i set when map i could be made (unit
// inner stride, batch and time collapsing into one row stride, 16-byte
// aligned base and strides).
struct PrepMaps {
  CUtensorMap m[6];
  unsigned valid;
};

// fp32 [K][V] states kept in global memory in a lane-major layout: element
// (k, v) at ((v / 4) * K + k) * 4 + v % 4, so the 32 lanes of a warp that own
// rows k .. k + 31 access 512 contiguous bytes per float4.
__host__ __device__ __forceinline__ int lm_off(int k, int v) {
  return ((v >> 2) * TK + k) * 4 + (v & 3);
}

}  // namespace tcx
}  // namespace ngdn2
