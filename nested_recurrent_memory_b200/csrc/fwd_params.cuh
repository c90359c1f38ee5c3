// Host/device description of one forward call: shapes, schedule, tensor
// views and the workspace layout shared by the CUDA-core and tensor-core
// kernel families.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace ngdn2 {

// Element (b, t, h, d) of a per-token tensor, any strides.
struct TokView {
  const void* p;
  int dt;
  int64_t sb, st, sh, sd;
  __device__ __forceinline__ int64_t off(int b, int t, int h, int d) const {
    return b * sb + t * st + h * sh + d * sd;
  }
  __device__ __forceinline__ float at(int b, int t, int h, int d) const {
    return load_elem(p, off(b, t, h, d), dt);
  }
};

// Element (b, t, h, l, d) of q [B, T, H, L, K].
struct QView {
  const void* p;
  int dt;
  int64_t sb, st, sh, sl, sd;
  __device__ __forceinline__ int64_t off(int b, int t, int h, int l, int d) const {
    return b * sb + t * st + h * sh + l * sl + d * sd;
  }
  __device__ __forceinline__ float at(int b, int t, int h, int l, int d) const {
    return load_elem(p, off(b, t, h, l, d), dt);
  }
};

// 8 consecutive elements from element offset o (element stride sd) as fp32:
// one or two vector loads when contiguous and 16-byte aligned, one load
// when the stride is 0 (a broadcast view).
__device__ __forceinline__ void load8_any(const void* base, int dt, int64_t o, int64_t sd,
                                          float* out) {
  if (sd == 0) {
    const float x = load_elem(base, o, dt);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = x;
    return;
  }
  if (sd == 1) {
    if (dt != NGDN2_F32) {
      const uint16_t* p16 = reinterpret_cast<const uint16_t*>(base) + o;
      if ((reinterpret_cast<uintptr_t>(p16) & 15) == 0) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p16);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (dt == NGDN2_BF16) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
          } else {
            out[2 * i] = __half2float(__ushort_as_half(uint16_t(w[i] & 0xffffu)));
            out[2 * i + 1] = __half2float(__ushort_as_half(uint16_t(w[i] >> 16)));
          }
        }
        return;
      }
    } else {
      const float* p32 = reinterpret_cast<const float*>(base) + o;
      if ((reinterpret_cast<uintptr_t>(p32) & 15) == 0) {
        const float4 a = *reinterpret_cast<const float4*>(p32);
        const float4 c = *reinterpret_cast<const float4*>(p32 + 4);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        out[4] = c.x; out[5] = c.y; out[6] = c.z; out[7] = c.w;
        return;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = load_elem(base, o + i * sd, dt);
}

constexpr int kC = NGDN2_CHUNK;  // tokens per chunk

__host__ __device__ inline int64_t align_floats(int64_t n) { return (n + 63) & ~int64_t(63); }

// Per-chunk record written by the prep kernels and read by the scans, fp32.
// All offsets in floats from the start of the record.
struct ChunkRecord {
  int64_t W, U, A, Q, Kt, eg, size;
  __host__ __device__ static ChunkRecord make(int K, int V, int L) {
    ChunkRecord r;
    r.W = 0;                       // [64, K]  (I + A_kk)^-1 (k * b * e^G)
    r.U = r.W + kC * K;            // [64, V]  (I + A_kk)^-1 (w * v)
    r.A = r.U + kC * V;            // [64, 64] mix0 * scale * A_qk, causal
    r.Q = r.A + kC * kC;           // [L, 64, K] read queries, mix and scale folded
    r.Kt = r.Q + int64_t(L) * kC * K;  // [64, K] k * e^(G_last - G)
    r.eg = r.Kt + kC * K;          // [K] e^(G_last)
    r.size = align_floats(r.eg + K);
    return r;
  }
};

// Parameters converted to fp32, [L-1, H, ...] each.
struct ParamLayout {
  int64_t qb, kp, bp, wp, gp, size;
  __host__ __device__ static ParamLayout make(int L, int H, int n_max, int K, int V) {
    ParamLayout p;
    int64_t n = int64_t(L > 1 ? L - 1 : 0) * H;
    p.qb = 0;
    p.kp = align_floats(p.qb + n * n_max * K);
    p.bp = align_floats(p.kp + n * K * V);
    p.wp = align_floats(p.bp + n * V * K);
    p.gp = align_floats(p.wp + n * V * V);
    p.size = align_floats(p.gp + n * V * K);
    return p;
  }
};

// Per-(b, h) scratch of the CUDA-core scan, fp32.
struct ScanScratch {
  int64_t vn, ot, vp, keys, bl, wl, gl, vn2, gvec, bdiag, size;
  __host__ __device__ static ScanScratch make(int K, int V, int NP) {
    ScanScratch s;
    s.vn = 0;
    s.ot = align_floats(s.vn + kC * V);
    s.vp = align_floats(s.ot + kC * V);
    s.keys = align_floats(s.vp + int64_t(NP) * V);
    s.bl = align_floats(s.keys + int64_t(NP) * K);
    s.wl = align_floats(s.bl + int64_t(NP) * K);
    s.gl = align_floats(s.wl + int64_t(NP) * V);
    s.vn2 = align_floats(s.gl + int64_t(NP) * K);
    s.gvec = align_floats(s.vn2 + int64_t(NP) * V);
    s.bdiag = align_floats(s.gvec + K);
    s.size = align_floats(s.bdiag + NP);
    return s;
  }
};

struct FwdParams {
  int B, T, H, K, V, L, NT, n_max, promotion, dtype, param_dtype;
  float scale;
  int nq[NGDN2_MAX_LEVELS];
  int firing[NGDN2_MAX_LEVELS];
  int NP;  // most pairs any level writes per firing
  QView q;
  TokView k, v, g, b, w, mix;  // mix: d indexes the level
  const void* raw_params[5];   // query_banks, key/b/w/g projections as passed
  const float* init;
  void* o;
  float* fin;
  int32_t* status;
  // workspace regions
  float* params32;
  ParamLayout pl;
  float* chunks;
  ChunkRecord rec;
  float* scan;
  ScanScratch ss;
  // Checkpoints for the backward (null in a plain forward): the level-0
  // state entering every chunk plus the final one, [B, H, NT + 1, K, V];
  // each upper level's state entering every group plus the final one,
  // [B, H, NG_l + 1, K, V] at ck_up + ck_up_off[l]; and v_new of every chunk,
  // [B, H, NT, 64, V]. With these set the scan writes no output o.
  float* ck0;
  float* ck_up;
  int64_t ck_up_off[NGDN2_MAX_LEVELS];
  int ck_up_n[NGDN2_MAX_LEVELS];  // NG_l + 1
  float* ck_vnew;
  // And the chunk's A_kk (strict lower) and scale * A_qk (causal, no mix),
  // [B, H, NT, 2, 64, 64].
  float* ck_ta;
};

// True when this forward's start gate timed out: the gate kernel, which
// runs before every other kernel of the forward on the same stream, set
// NGDN2_STATUS_GATE_TIMEOUT. Kernels then return before any other work.
// Nothing sets that bit while the forward's later kernels run, so every
// thread of a CTA reads the same value.
__device__ __forceinline__ bool gate_closed(const FwdParams& p) {
  return p.status &&
         (*reinterpret_cast<const volatile int32_t*>(p.status) & NGDN2_STATUS_GATE_TIMEOUT);
}

// Arguments of the update-scan kernel (update_fwd.py:131-204).
struct UpdParams {
  int B, NF, NG, H, K, V, N, bv, dtype, g_dtype;
  const void* keys;
  int64_t skb, skf, skh, skn;
  const void* values;
  const void* g;
  const void* b;
  const void* w;
  const float* init;
  float* states;
  float* fin;
};

// Arguments of the write-scan backward (update_bwd.py:167-263).
struct UpdBwdParams {
  int B, NF, NG, H, K, V, N, dtype, g_dtype, has_init;
  const float* states;
  const void* keys;
  int64_t skb, skf, skh, skn;
  const void* values;
  const void* g;
  const void* b;
  const void* w;
  const float* d_states;
  const float* d_final;
  float *dkeys, *dvalues, *dg, *db, *dw, *dinit;
  float* scr;  // per (b, h): dS, S_d, dS_d, Z, Y
};

}  // namespace ngdn2
