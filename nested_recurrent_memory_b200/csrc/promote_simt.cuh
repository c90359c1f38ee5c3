// Promotion of one level into the next on CUDA cores, fp32 (shared by the
// CUDA-core scan and the decode step's promotion kernel).
#pragma once

#include "fwd_params.cuh"

namespace ngdn2 {

// Promote level l-1 into level l for one (b, h): probe then update. PF is
// block_gemm's prefetch switch (for a caller at its register cap).
template <bool PF = true>
static __device__ void promote_simt(const FwdParams& p, int b, int h, int l, float* S, float* sc,
                             float* gsm) {
  const int K = p.K, V = p.V;
  const float* Sb = S + int64_t(l - 1) * K * V;
  float* Sl = S + int64_t(l) * K * V;
  const int64_t pidx = int64_t(l - 1) * p.H + h;
  const float* qb = p.params32 + p.pl.qb + pidx * p.n_max * K;
  const float* kp = p.params32 + p.pl.kp + pidx * K * V;
  const float* bp = p.params32 + p.pl.bp + pidx * V * K;
  const float* wp = p.params32 + p.pl.wp + pidx * V * V;
  const float* gp = p.params32 + p.pl.gp + pidx * V * K;
  float* Vp = sc + p.ss.vp;
  float* Kk = sc + p.ss.keys;
  float* Bl = sc + p.ss.bl;
  float* Wl = sc + p.ss.wl;
  float* Gl = sc + p.ss.gl;
  float* Vn2 = sc + p.ss.vn2;
  float* gv = sc + p.ss.gvec;
  float* bd = sc + p.ss.bdiag;
  const int tid = threadIdx.x;
  const bool merge = p.promotion == NGDN2_PROMOTION_MERGE;
  const int m = merge ? K : p.nq[l - 1];
  // values: the bank's reads of the level below (probe.py:97-98), or the
  // level below itself for merge (probe.py:133-136).
  const float* vals = Sb;
  if (!merge) {
    block_gemm<false, false, PF>(m, V, K, [&](int r, int k) { return qb[r * K + k]; },
               [&](int k, int c) { return Sb[k * V + c]; }, gsm,
               [&](int r, int c, float a) { Vp[r * V + c] = a; });
    vals = Vp;
    // u = values . W_k^T (probe.py:99)
    block_gemm<false, true, PF>(m, K, V, [&](int r, int v) { return vals[r * V + v]; },
               [&](int v, int k) { return kp[k * V + v]; }, gsm,
               [&](int r, int k, float a) { Kk[r * K + k] = a; });
  }
  // gate logits (probe.py:59-62)
  block_gemm<false, false, PF>(m, K, V, [&](int r, int v) { return vals[r * V + v]; },
             [&](int v, int k) { return bp[v * K + k]; }, gsm,
             [&](int r, int k, float a) { Bl[r * K + k] = a; });
  block_gemm<false, false, PF>(m, V, V, [&](int r, int v) { return vals[r * V + v]; },
             [&](int v, int u) { return wp[v * V + u]; }, gsm,
             [&](int r, int u, float a) { Wl[r * V + u] = a; });
  block_gemm<false, false, PF>(m, K, V, [&](int r, int v) { return vals[r * V + v]; },
             [&](int v, int k) { return gp[v * K + k]; }, gsm,
             [&](int r, int k, float a) { Gl[r * K + k] = a; });
  if (!merge) {
    // keys = normalize(u) (probe.py:100): one warp per row.
    const int warp = tid / 32, lane = tid % 32;
    for (int r = warp; r < m; r += blockDim.x / 32) {
      float s = 0.f;
      for (int k = lane; k < K; k += 32) s = fmaf(Kk[r * K + k], Kk[r * K + k], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float nrm = fmaxf(sqrtf(s), 1e-12f);
      for (int k = lane; k < K; k += 32) Kk[r * K + k] = Kk[r * K + k] / nrm;
    }
    __syncthreads();
    // k * b and v * w (probe.py:63-64, update_fwd.py:121-122)
    for (int e = tid; e < m * K; e += blockDim.x) Bl[e] = Kk[e] * sigmoidf_(Bl[e] + kBLogitInit);
    for (int e = tid; e < m * V; e += blockDim.x) Wl[e] = vals[e] * sigmoidf_(Wl[e] + kWLogitInit);
  } else {
    for (int r = tid; r < m; r += blockDim.x) bd[r] = sigmoidf_(Bl[r * K + r] + kBLogitInit);
  }
  // g = mean over pairs of -softplus(logit - 4) (probe.py:65)
  for (int k = tid; k < K; k += blockDim.x) {
    float s = 0.f;
#pragma unroll 8
    for (int r = 0; r < m; ++r) s += -softplusf_(Gl[r * K + k] + kGLogitInit);
    gv[k] = s / float(m);
  }
  __syncthreads();
  if (merge) {
    // Identity keys: pair r writes row r only, so the update is elementwise
    // (naive.py:32-39 with keys = I).
    for (int e = tid; e < K * V; e += blockDim.x) {
      const int k = e / V;
      const float s = Sl[e] * expf(gv[k]);
      Sl[e] = s - bd[k] * s + Sb[e] * sigmoidf_(Wl[e] + kWLogitInit);
    }
    __syncthreads();
    return;
  }
  // S <- e^g S; vn = v*w - (k*b) S; S <- S + k^T vn  (update_fwd.py:120-123)
  block_map(Sl, Sl, K * V, [&](int e, float x) { return x * expf(gv[e / V]); });
  __syncthreads();
  block_gemm<false, false, PF>(m, V, K, [&](int r, int k) { return Bl[r * K + k]; },
             [&](int k, int c) { return Sl[k * V + c]; }, gsm,
             [&](int r, int c, float a) { Vn2[r * V + c] = Wl[r * V + c] - a; });
  block_gemm<true, false, PF>(K, V, m, [&](int k, int r) { return Kk[r * K + k]; },
             [&](int r, int c) { return Vn2[r * V + c]; }, gsm,
             [&](int k, int c, float a) { Sl[k * V + c] += a; });
}

}  // namespace ngdn2
