// Backward of the chunkwise nested GDN-2 forward, on CUDA cores in fp32.
//
// The reference's backward (nested_gdn2/ops/chunk.py:368-564,
// ChunkNestedGDN2Function.backward :650-719) is a composition: read-level
// einsums, a probe replay through autograd, update_state's own backward
// (update_bwd.py) and fla's level-0 chunk backward with the promotions'
// gradient injected as dh_ext. Here the same gradient is computed by three
// kernels over the forward's own per-chunk records:
//
//   1. the CUDA-core forward (prep + scan) re-run with checkpoints: the
//      level-0 state entering every chunk, every upper level's state entering
//      every group, and v_new of every chunk;
//   2. bwd_scan -- one CTA per (b, h), chunks in reverse: the state gradient
//      of every level flows back through each chunk's level-0 recurrence,
//      the upper-level reads, and at each firing the promotion (update step
//      then probe, top level first); parameter gradients accumulate across
//      the batch with atomics. Per chunk it leaves dS (leaving the chunk) and
//      dv_new for the local pass;
//   3. bwd_local -- one CTA per (b, h, chunk), fully parallel: the gradients
//      of q, k, v, g, b, w and the mix weights from the chunk's quantities,
//      recomputed from the inputs where cheap.
//
// Notation per chunk (64 tokens; naive.py:329-392): G = cumsum(g),
// T = strictly-lower (b*k) k^T decayed, A_qk = lower q~ k^T decayed
// (q~ = scale q_0), [U | W] = (I + T)^-1 [w*v | k*b*e^G], v_new = U - W S,
// r_0 = A_qk v_new + (q~ e^G) S, o = sum_l mix_l r_l,
// S' = e^(G_last) S + Kt^T v_new with Kt = k e^(G_last - G).

#include <string.h>

#include "fwd_params.cuh"
#include "promote_simt.cuh"
#include "tc_gemm3.cuh"

namespace ngdn2 {

// Per-(b, h) scratch of the promotion backward, fp32, offsets in floats.
struct PromoBwdScratch {
  int64_t vp, keys, nrm, bg, wg, zg, z, y, dkeys, dkb, dvp, sd, dsd, gv, dgv, dos, size;
  __host__ __device__ static PromoBwdScratch make(int K, int V, int NP) {
    PromoBwdScratch s;
    const int64_t mv = int64_t(NP) * V, mk = int64_t(NP) * K, kv = int64_t(K) * V;
    s.vp = 0;                              // [m, V] values V'
    s.keys = align_floats(s.vp + mv);      // [m, K] keys (u / |u|)
    s.nrm = align_floats(s.keys + mk);     // [m] max(|u|, 1e-12)
    s.bg = align_floats(s.nrm + NP);       // [m, K] erase gate b
    s.wg = align_floats(s.bg + mk);        // [m, V] write gate w
    s.zg = align_floats(s.wg + mv);        // [m, K] decay logits V' W_g - 4
    s.z = align_floats(s.zg + mk);         // [m, V] keys . dS'
    s.y = align_floats(s.z + mv);          // [m, V] (keys * b) . S_d
    s.dkeys = align_floats(s.y + mv);      // [m, K]
    s.dkb = align_floats(s.dkeys + mk);    // [m, K] d(keys * b)
    s.dvp = align_floats(s.dkb + mk);      // [m, V] dV'
    s.sd = align_floats(s.dvp + mv);       // [K, V] e^g S
    s.dsd = align_floats(s.sd + kv);       // [K, V] d(e^g S)
    s.gv = align_floats(s.dsd + kv);       // [K] g
    s.dgv = align_floats(s.gv + K);        // [K] dg
    s.dos = align_floats(s.dgv + K);       // [64, V] d_o of the current chunk, fp32
    s.size = align_floats(s.dos + int64_t(kC) * V);
    return s;
  }
};

// Per-chunk scratch of the local pass, fp32, offsets in floats.
struct LocalScratch {
  int64_t dqg, dkt, drw, dru, dkta, dgc, dos, size;
  __host__ __device__ static LocalScratch make(int K, int V) {
    LocalScratch s;
    s.dqg = 0;                                  // [64, K] d(q~ e^G), mix_0 folded
    s.dkt = align_floats(s.dqg + kC * K);       // [64, K] dKt
    s.drw = align_floats(s.dkt + kC * K);       // [64, K] dW, then dR_W
    s.dru = align_floats(s.drw + kC * K);       // [64, V] dU, then dR_U
    s.dkta = align_floats(s.dru + kC * V);      // [64, K] dk from the decayed blocks
    s.dgc = align_floats(s.dkta + kC * K);      // [64, K] dG, column part then whole
    s.dos = align_floats(s.dgc + kC * K);       // [64, V] d_o of the chunk, fp32
    s.size = align_floats(s.dos + kC * V);
    return s;
  }
};

struct BwdParams {
  FwdParams f;  // inputs, converted parameters, records and checkpoints
  const void* d_o;
  int d_o_dtype;
  int64_t dos[4];        // [B, T, H, V] element strides
  const float* d_final;  // [B, H, L, K, V] or null
  float *dq, *dk, *dv, *dg, *db, *dw, *dmix;  // fp32 outputs, contiguous
  float* dparams;        // fp32 [B] x layout f.pl, zeroed before the scan (null when L == 1)
  float* dinit;          // [B, H, L, K, V] or null
  float* dS;             // [B, H, L, K, V] running state gradient
  float* dsn;            // [B, H, NT, K, V] dS0 leaving each chunk
  float* dvn;            // [B, H, NT, 64, V] dv_new of each chunk
  float* pscr;           // [B, H] x PromoBwdScratch
  PromoBwdScratch ps;
  float* lscr;           // [B, H, NT] x LocalScratch
  LocalScratch ls;
};

__device__ __forceinline__ const float* ck_level(const FwdParams& f, int64_t bh, int level, int j) {
  const int64_t kv = int64_t(f.K) * f.V;
  return level == 0 ? f.ck0 + (bh * (f.NT + 1) + j) * kv
                    : f.ck_up + f.ck_up_off[level] + (bh * f.ck_up_n[level] + j) * kv;
}

// Backward of one firing of level l at chunk n: the update step
// (naive.py:7-39) after the probe (probe.py:34-136), both recomputed from the
// checkpoints. In: dS_l after the firing. Out: dS_l before it, dS_{l-1}
// (the source, level l-1 after chunk n) increased by the probe's gradient,
// and the parameter gradients added into p.dparams.
__device__ __forceinline__ void promote_bwd(const BwdParams& p, int b, int h, int l, int n,
                                            tc::Tc3Ctx& tcx) {
  const FwdParams& f = p.f;
  const int K = f.K, V = f.V, tid = threadIdx.x, nth = blockDim.x;
  const int64_t bh = int64_t(b) * f.H + h;
  const bool merge = f.promotion == NGDN2_PROMOTION_MERGE;
  const int m = merge ? K : f.nq[l - 1];
  const float* X = l == 1 ? ck_level(f, bh, 0, n + 1)
                          : ck_level(f, bh, l - 1, (n + 1) / f.firing[l - 1]);
  const float* Sold = ck_level(f, bh, l, n / f.firing[l]);
  float* dSl = p.dS + (bh * f.L + l) * K * V;
  float* dSb = p.dS + (bh * f.L + l - 1) * K * V;
  const int64_t pidx = int64_t(l - 1) * f.H + h;
  const float* qb = f.params32 + f.pl.qb + pidx * f.n_max * K;
  const float* kp = f.params32 + f.pl.kp + pidx * K * V;
  const float* bp = f.params32 + f.pl.bp + pidx * V * K;
  const float* wp = f.params32 + f.pl.wp + pidx * V * V;
  const float* gp = f.params32 + f.pl.gp + pidx * V * K;
  // This batch row's own copy of the parameter gradients (summed over rows
  // in a fixed order afterwards, so the result is reproducible).
  float* dpar = p.dparams + int64_t(b) * f.pl.size;
  float* dqb = dpar + f.pl.qb + pidx * f.n_max * K;
  float* dkp = dpar + f.pl.kp + pidx * K * V;
  float* dbp = dpar + f.pl.bp + pidx * V * K;
  float* dwp = dpar + f.pl.wp + pidx * V * V;
  float* dgp = dpar + f.pl.gp + pidx * V * K;
  float* sc = p.pscr + bh * p.ps.size;
  float* Vp = sc + p.ps.vp;
  float* Kk = sc + p.ps.keys;
  float* Nr = sc + p.ps.nrm;
  float* Bg = sc + p.ps.bg;
  float* Wg = sc + p.ps.wg;
  float* Zg = sc + p.ps.zg;
  float* Z = sc + p.ps.z;
  float* Y = sc + p.ps.y;
  float* dKk = sc + p.ps.dkeys;
  float* dKB = sc + p.ps.dkb;
  float* dVp = sc + p.ps.dvp;
  float* Sd = sc + p.ps.sd;
  float* dSd = sc + p.ps.dsd;
  float* gv = sc + p.ps.gv;
  float* dgv = sc + p.ps.dgv;
  const int warp = tid / 32, lane = tid % 32, nwarp = nth / 32;

  // --- the probe, recomputed (as promote_simt) ---
  const float* vals = X;  // merge: the values are the level below (probe.py:133-136)
  if (!merge) {
    tc::tc_gemm3(tcx, m, V, K, qb, K, X, V, [](int, int) { return 0.f; },
                 [&](int r, int c, float a, float) { Vp[r * V + c] = a; });
    vals = Vp;
    tc::tc_gemm3<false, true>(tcx, m, K, V, vals, V, kp, V, [](int, int) { return 0.f; },
                              [&](int r, int k, float a, float) { Kk[r * K + k] = a; });
    for (int r = warp; r < m; r += nwarp) {
      float s = 0.f;
      for (int k = lane; k < K; k += 32) s = fmaf(Kk[r * K + k], Kk[r * K + k], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float nrm = sqrtf(s);
      for (int k = lane; k < K; k += 32) Kk[r * K + k] /= fmaxf(nrm, 1e-12f);
      if (lane == 0) Nr[r] = nrm;
    }
  }
  // (learned: k * b goes to the d(K*b) buffer, free until its own product)
  tc::tc_gemm3(tcx, m, K, V, vals, V, bp, K, [](int, int) { return 0.f; }, [&](int r, int k, float a, float) {
    const float bg = sigmoidf_(a + kBLogitInit);
    Bg[r * K + k] = bg;
    if (!merge) dKB[r * K + k] = Kk[r * K + k] * bg;
  });
  tc::tc_gemm3(tcx, m, V, V, vals, V, wp, V, [](int, int) { return 0.f; },
               [&](int r, int u, float a, float) { Wg[r * V + u] = sigmoidf_(a + kWLogitInit); });
  tc::tc_gemm3(tcx, m, K, V, vals, V, gp, K, [](int, int) { return 0.f; },
               [&](int r, int k, float a, float) { Zg[r * K + k] = a + kGLogitInit; });
  for (int k = tid; k < K; k += nth) {
    float s = 0.f;
#pragma unroll 8
    for (int r = 0; r < m; ++r) s += -softplusf_(Zg[r * K + k]);
    gv[k] = s / float(m);
  }
  __syncthreads();
  block_map<2>(Sd, Sold, K * V, [&](int e, float x) { return x * expf(gv[e / V]); });
  __syncthreads();

  // --- backward of S' = S_d - K^T (K*b) S_d + K^T (V' * w), S_d = e^g S ---
  // Z = K dS', Y = (K*b) S_d  (merge: K = I)
  if (!merge) {
    const float* KB = dKB;  // K * b, written with the gates above
    tc::tc_gemm3(tcx, m, V, K, Kk, K, dSl, V, [](int, int) { return 0.f; },
                 [&](int r, int c, float a, float) { Z[r * V + c] = a; });
    // Y holds V' * w - (K*b) S_d, the left operand of dK
    tc::tc_gemm3(tcx, m, V, K, KB, K, Sd, V, [](int, int) { return 0.f; }, [&](int r, int c, float a, float) {
      Y[r * V + c] = vals[r * V + c] * Wg[r * V + c] - a;
    });
    // dS_d = dS' - (K*b)^T Z  (before d(K*b) overwrites K * b)
    tc::tc_gemm3<true, false>(
        tcx, K, V, m, KB, K, Z, V, [&](int k, int c) { return dSl[k * V + c]; },
        [&](int k, int c, float a, float old) { dSd[k * V + c] = old - a; });
    // dK = (V' * w - Y) dS'^T;  d(K*b) = -Z S_d^T
    tc::tc_gemm3<false, true>(tcx, m, K, V, Y, V, dSl, V, [](int, int) { return 0.f; },
                              [&](int r, int k, float a, float) { dKk[r * K + k] = a; });
    tc::tc_gemm3<false, true>(tcx, m, K, V, Z, V, Sd, V, [](int, int) { return 0.f; },
                              [&](int r, int k, float a, float) { dKB[r * K + k] = -a; });
  } else {
    for (int e = tid; e < K * V; e += nth) {
      const int k = e / V;
      Z[e] = dSl[e];
      dSd[e] = dSl[e] - Bg[k * K + k] * dSl[e];
    }
    __syncthreads();
    // d(K*b) only matters on the diagonal (b is read there only)
    for (int k = warp; k < K; k += nwarp) {
      float s = 0.f;
      for (int c = lane; c < V; c += 32) s = fmaf(Z[k * V + c], Sd[k * V + c], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) dKB[k * K + k] = -s;
    }
    __syncthreads();
  }
  // dg = sum_v dS_d * S_d;  dS (before the firing) = e^g dS_d
  for (int k = warp; k < K; k += nwarp) {
    float s = 0.f;
    for (int c = lane; c < V; c += 32) s = fmaf(dSd[k * V + c], Sd[k * V + c], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) dgv[k] = s;
  }
  __syncthreads();
  block_map<2>(dSl, dSd, K * V, [&](int e, float x) { return expf(gv[e / V]) * x; });
  // Gates: dV' = Z * w; dw -> d(w logit) = Z * V' * w (1 - w) (into Wg);
  // db = d(K*b) * K -> d(b logit) = db * b (1 - b) (into Bg);
  // dK += d(K*b) * b; d(g logit) = -(dg / m) sigmoid(z) (into Zg).
  for (int e = tid; e < m * V; e += nth) {
    const float w = Wg[e], z = Z[e];
    dVp[e] = z * w;
    Wg[e] = z * vals[e] * w * (1.f - w);
  }
  for (int e = tid; e < m * K; e += nth) {
    const int r = e / K, k = e % K;
    const float bb = Bg[e];
    float db;
    if (merge) {
      db = (r == k) ? dKB[e] : 0.f;
    } else {
      db = dKB[e] * Kk[e];
      dKk[e] += dKB[e] * bb;
    }
    Bg[e] = db * bb * (1.f - bb);
    Zg[e] = -(dgv[k] / float(m)) * sigmoidf_(Zg[e]);
  }
  __syncthreads();
  // dV' += d(g logit) W_g^T + d(b logit) W_b^T + d(w logit) W_w^T
  auto ld_dvp = [&](int r, int v) { return dVp[r * V + v]; };
  auto add_dvp = [&](int r, int v, float a, float old) { dVp[r * V + v] = old + a; };
  tc::tc_gemm3<false, true>(tcx, m, V, K, Zg, K, gp, K, ld_dvp, add_dvp);
  tc::tc_gemm3<false, true>(tcx, m, V, K, Bg, K, bp, K, ld_dvp, add_dvp);
  tc::tc_gemm3<false, true>(tcx, m, V, V, Wg, V, wp, V, ld_dvp, add_dvp);
  // parameter gradients of the gates: V'^T d(logit)
  tc::tc_gemm3<true, false>(
      tcx, V, K, m, vals, V, Zg, K, [&](int v, int j) { return dgp[v * K + j]; },
      [&](int v, int j, float a, float old) { dgp[v * K + j] = old + a; });
  tc::tc_gemm3<true, false>(
      tcx, V, K, m, vals, V, Bg, K, [&](int v, int j) { return dbp[v * K + j]; },
      [&](int v, int j, float a, float old) { dbp[v * K + j] = old + a; });
  tc::tc_gemm3<true, false>(
      tcx, V, V, m, vals, V, Wg, V, [&](int v, int j) { return dwp[v * V + j]; },
      [&](int v, int j, float a, float old) { dwp[v * V + j] = old + a; });
  if (merge) {
    for (int e = tid; e < K * V; e += nth) dSb[e] += dVp[e];
    __syncthreads();
    return;
  }
  // keys = u / max(|u|, 1e-12) (probe.py:100): du = (dK - K (K . dK)) / |u|
  for (int r = warp; r < m; r += nwarp) {
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s = fmaf(Kk[r * K + k], dKk[r * K + k], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float nrm = Nr[r];
    for (int k = lane; k < K; k += 32) {
      const float d = dKk[r * K + k];
      dKk[r * K + k] = nrm > 1e-12f ? (d - Kk[r * K + k] * s) / nrm : d / 1e-12f;
    }
  }
  __syncthreads();
  // dV' += du W_k; dW_k += du^T V'
  tc::tc_gemm3(tcx, m, V, K, dKk, K, kp, V, ld_dvp, add_dvp);
  tc::tc_gemm3<true, false>(
      tcx, K, V, m, dKk, K, vals, V, [&](int k, int v) { return dkp[k * V + v]; },
      [&](int k, int v, float a, float old) { dkp[k * V + v] = old + a; });
  // V' = Q_bank X: dQ_bank += dV' X^T; dX = Q_bank^T dV'
  tc::tc_gemm3<false, true>(
      tcx, m, K, V, dVp, V, X, V, [&](int r, int k) { return dqb[r * K + k]; },
      [&](int r, int k, float a, float old) { dqb[r * K + k] = old + a; });
  tc::tc_gemm3<true, false>(
      tcx, K, V, m, qb, K, dVp, V, [&](int k, int v) { return dSb[k * V + v]; },
      [&](int k, int v, float a, float old) { dSb[k * V + v] = old + a; });
}

// ---------------------------------------------------------------------------
// bwd_scan: grid (H, B), 256 threads; chunks in reverse.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256, 1) bwd_scan_kernel(BwdParams p) {
  __shared__ uint64_t tc_bar;
  __shared__ uint32_t tc_base;
  __shared__ int tc_abort;
  extern __shared__ uint8_t dyn_smem[];
  const FwdParams& f = p.f;
  const int h = blockIdx.x, b = blockIdx.y, K = f.K, V = f.V, L = f.L, tid = threadIdx.x;
  const int64_t bh = int64_t(b) * f.H + h;
  // Tensor-core products (tc::tc_gemm3): TMEM accumulator, MMA barrier, staging.
  if ((tid >> 5) == 0) tc::tmem_alloc(&tc_base, tc::kTc3TmemCols);
  if (tid == 0) {
    tc::mbar_init(&tc_bar, 1);
    tc::fence_mbar_init();
    tc_abort = 0;
  }
  float* dS = p.dS + bh * L * K * V;
  for (int64_t e = tid; e < int64_t(L) * K * V; e += blockDim.x)
    dS[e] = p.d_final ? p.d_final[bh * L * K * V + e] : 0.f;
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  tc::Tc3Ctx tcx{tc_base, &tc_bar, 0u,
            reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023)),
            &tc_abort};
  for (int n = f.NT - 1; n >= 0; --n) {
    const float* rec = f.chunks + (bh * f.NT + n) * f.rec.size;
    const float* Am = rec + f.rec.A;   // mix0 scale A_qk
    const float* Q0 = rec + f.rec.Q;   // mix0 scale q e^G
    const float* Wm = rec + f.rec.W;
    const float* Kt = rec + f.rec.Kt;
    const float* eg = rec + f.rec.eg;
    const int t0 = n * kC;
    // d_o of the chunk as fp32 (rows past T zero), for the GEMMs below.
    float* dOs = p.pscr + bh * p.ps.size + p.ps.dos;
    for (int e = tid; e < kC * V / 8; e += blockDim.x) {
      const int i = e / (V / 8), c0 = 8 * (e % (V / 8)), t = t0 + i;
      float o8[8];
      if (t < f.T) {
        load8_any(p.d_o, p.d_o_dtype, b * p.dos[0] + t * p.dos[1] + h * p.dos[2] + c0 * p.dos[3],
                  p.dos[3], o8);
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) o8[u] = 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) dOs[i * V + c0 + u] = o8[u];
    }
    __syncthreads();
    // The firings after this chunk, top level first (naive.py:394-415 reversed).
    for (int l = L - 1; l >= 1; --l)
      if ((n + 1) % f.firing[l] == 0) promote_bwd(p, b, h, l, n, tcx);
    // Upper-level reads (naive.py:382-385): dS_l += (mix_l scale q_l)^T dO.
    for (int l = 1; l < L; ++l) {
      const float* Ql = rec + f.rec.Q + int64_t(l) * kC * K;
      float* dSl = dS + int64_t(l) * K * V;
      tc::tc_gemm3<true, false>(
          tcx, K, V, kC, Ql, K, dOs, V, [&](int k, int c) { return dSl[k * V + c]; },
          [&](int k, int c, float a, float old) { dSl[k * V + c] = old + a; });
    }
    // Level 0: dv_new = (mix0 scale A_qk)^T dO + Kt dS0 (the S0 entering the
    // next chunk, naive.py:392), kept for the local pass with dS0 itself.
    float* dv = p.dvn + (bh * f.NT + n) * kC * V;
    tc::tc_gemm3<true, false>(
        tcx, kC, V, kC, Am, kC, dOs, V, [](int, int) { return 0.f; },
        [&](int i, int c, float a, float) { dv[i * V + c] = a; });
    tc::tc_gemm3(
        tcx, kC, V, K, Kt, K, dS, V, [&](int i, int c) { return dv[i * V + c]; },
        [&](int i, int c, float a, float old) { dv[i * V + c] = old + a; });
    float* dsn = p.dsn + (bh * f.NT + n) * K * V;
    block_map<2>(dsn, dS, K * V, [](int, float x) { return x; });
    __syncthreads();
    // dS0 <- e^(G_last) dS0 + (mix0 scale q e^G)^T dO - W^T dv_new
    tc::tc_gemm3<true, false>(
        tcx, K, V, kC, Q0, K, dOs, V, [&](int k, int c) { return dS[k * V + c]; },
        [&](int k, int c, float a, float old) { dS[k * V + c] = eg[k] * old + a; });
    tc::tc_gemm3<true, false>(
        tcx, K, V, kC, Wm, K, dv, V, [&](int k, int c) { return dS[k * V + c]; },
        [&](int k, int c, float a, float old) { dS[k * V + c] = old - a; });
  }
  if (p.dinit)
    for (int64_t e = tid; e < int64_t(L) * K * V; e += blockDim.x) p.dinit[bh * L * K * V + e] = dS[e];
  if (tid == 0 && tc_abort && f.status) atomicOr(f.status, NGDN2_STATUS_WAIT_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  if ((tid >> 5) == 0) tc::tmem_dealloc(tc_base, tc::kTc3TmemCols);
}

// ---------------------------------------------------------------------------
// bwd_local: grid (NT, H, B), 256 threads; the level-0 chunk backward and
// the upper-level read gradients of one chunk.
// ---------------------------------------------------------------------------

size_t bwd_local_smem(int K) {
  return sizeof(float) * (5 * size_t(kC) * (K + 1) + 3 * kC * 65 + kC + 2 * K + kGemmSmemFloats);
}

__global__ void __launch_bounds__(256) bwd_local_kernel(BwdParams p) {
  extern __shared__ float sm[];
  const FwdParams& f = p.f;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int K = f.K, V = f.V, KP = K + 1, tid = threadIdx.x, nth = blockDim.x;
  const int64_t bh = int64_t(b) * f.H + h;
  const int t0 = n * kC;
  float* Gs = sm;               // [64][K+1] G = cumsum g
  float* Qs = Gs + kC * KP;     // [64][K+1] scale q_0
  float* Ks = Qs + kC * KP;     // [64][K+1] k
  float* Bs = Ks + kC * KP;     // [64][K+1] b
  float* Eg = Bs + kC * KP;     // [64][K+1] e^g (per token step)
  float* Ts = Eg + kC * KP;     // [64][65] T (strictly lower)
  float* As = Ts + kC * 65;     // [64][65] A_qk, then dA_qk
  float* Dt = As + kC * 65;     // [64][65] dT
  float* mx = Dt + kC * 65;     // [64] mix_l of the rows
  float* dGl = mx + kC;         // [K] dG_last
  int* npos = reinterpret_cast<int*>(dGl + K);  // [K] channel has a g > 0 in the chunk
  float* gsm = dGl + 2 * K;
  const float* rec = f.chunks + (bh * f.NT + n) * f.rec.size;
  const float* Um = rec + f.rec.U;
  const float* Wm = rec + f.rec.W;
  const float* S0 = ck_level(f, bh, 0, n);
  const float* dSn = p.dsn + (bh * f.NT + n) * K * V;
  const float* dvn = p.dvn + (bh * f.NT + n) * kC * V;
  const float* vn = f.ck_vnew + (bh * f.NT + n) * kC * V;
  float* scr = p.lscr + (bh * f.NT + n) * p.ls.size;
  float* dQG = scr + p.ls.dqg;
  float* dKt = scr + p.ls.dkt;
  float* dRW = scr + p.ls.drw;
  float* dRU = scr + p.ls.dru;
  float* dKTA = scr + p.ls.dkta;
  float* dGc = scr + p.ls.dgc;
  float* dOs = scr + p.ls.dos;
  auto dO = [&](int i, int c) { return dOs[i * V + c]; };
  // fp32 output row of token i (rows past T are never written)
  auto orow = [&](int i, int width) { return ((int64_t(b) * f.T + t0 + i) * f.H + h) * width; };

  // Inputs of the chunk, 8 channels per load; tokens past T are zeros
  // (naive.py:302-312). d_o is staged once as fp32 for the GEMMs below.
  for (int e = tid; e < kC * K / 8; e += nth) {
    const int i = e / (K / 8), d0 = 8 * (e % (K / 8)), t = t0 + i;
    float q8[8], k8[8], g8[8], b8[8];
    if (t < f.T) {
      load8_any(f.q.p, f.q.dt, f.q.off(b, t, h, 0, d0), f.q.sd, q8);
      load8_any(f.k.p, f.k.dt, f.k.off(b, t, h, d0), f.k.sd, k8);
      load8_any(f.g.p, f.g.dt, f.g.off(b, t, h, d0), f.g.sd, g8);
      load8_any(f.b.p, f.b.dt, f.b.off(b, t, h, d0), f.b.sd, b8);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) q8[u] = k8[u] = g8[u] = b8[u] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int x = i * KP + d0 + u;
      Qs[x] = q8[u] * f.scale;
      Ks[x] = k8[u];
      Gs[x] = g8[u];
      Eg[x] = expf(g8[u]);
      Bs[x] = b8[u];
    }
  }
  for (int e = tid; e < kC * V / 8; e += nth) {
    const int i = e / (V / 8), c0 = 8 * (e % (V / 8)), t = t0 + i;
    float o8[8];
    if (t < f.T) {
      load8_any(p.d_o, p.d_o_dtype, b * p.dos[0] + t * p.dos[1] + h * p.dos[2] + c0 * p.dos[3],
                p.dos[3], o8);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) o8[u] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) dOs[i * V + c0 + u] = o8[u];
  }
  for (int i = tid; i < kC; i += nth) mx[i] = t0 + i < f.T ? f.mix.at(b, t0 + i, h, 0) : 0.f;
  for (int k = tid; k < K; k += nth) dGl[k] = 0.f;
  __syncthreads();
  if (tid < K) {
    float acc = 0.f;
    int pos = 0;
    for (int i = 0; i < kC; ++i) {
      const float g = Gs[i * KP + tid];
      pos |= g > 0.f;
      acc += g;
      Gs[i * KP + tid] = acc;
    }
    npos[tid] = pos;
  }
  // T and scale * A_qk as the forward's prep computed them (naive.py:335-344,
  // 377-378, clamped decays).
  {
    const float* ta = f.ck_ta + (bh * f.NT + n) * 2 * kC * kC;
    if ((reinterpret_cast<uintptr_t>(ta) & 15) == 0) {
      // 16-byte loads, four of each block in flight per thread
      const float4* t4 = reinterpret_cast<const float4*>(ta);
      constexpr int n4 = kC * kC / 4;
      for (int base = tid; base < n4; base += 4 * nth) {
        float4 a[4], c[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int x = base + u * nth;
          a[u] = x < n4 ? t4[x] : make_float4(0.f, 0.f, 0.f, 0.f);
          c[u] = x < n4 ? t4[n4 + x] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int x = base + u * nth;
          if (x < n4) {
            const int o = (4 * x / kC) * 65 + (4 * x) % kC;
            Ts[o] = a[u].x; Ts[o + 1] = a[u].y; Ts[o + 2] = a[u].z; Ts[o + 3] = a[u].w;
            As[o] = c[u].x; As[o + 1] = c[u].y; As[o + 2] = c[u].z; As[o + 3] = c[u].w;
          }
        }
      }
    } else {
      for (int e = tid; e < kC * kC; e += nth) {
        Ts[(e / kC) * 65 + e % kC] = ta[e];
        As[(e / kC) * 65 + e % kC] = ta[kC * kC + e];
      }
    }
  }
  __syncthreads();
  // dmix_0 = sum_v dO r_0, r_0 = A_qk v_new + (q~ e^G) S0 (naive.py:377-390)
  // (r_0 goes through the dR_U scratch, free until the solve below, and is
  // reduced row by row in a fixed order.)
  block_gemm(kC, V, kC + K,
             [&](int i, int j) {
               return j < kC ? As[i * 65 + j] : Qs[i * KP + j - kC] * expf(Gs[i * KP + j - kC]);
             },
             [&](int j, int c) { return j < kC ? vn[j * V + c] : S0[(j - kC) * V + c]; }, gsm,
             [&](int i, int c, float a) { dRU[i * V + c] = a * dO(i, c); });
  row_sums(dRU, kC, V, [&](int i, float s) {
    if (t0 + i < f.T) p.dmix[(int64_t(b) * f.T + t0 + i) * f.H * f.L + h * f.L] = s;
  });
  __syncthreads();
  // dA_qk = (mix_0 dO) v_new^T on the causal triangle; d(q~ e^G) = (mix_0 dO) S0^T
  block_gemm<false, true>(kC, kC + K, V, [&](int i, int c) { return mx[i] * dO(i, c); },
             [&](int c, int j) { return j < kC ? vn[j * V + c] : S0[(j - kC) * V + c]; }, gsm,
             [&](int i, int j, float a) {
               if (j < kC) As[i * 65 + j] = j <= i ? a : 0.f;
               else dQG[i * K + j - kC] = a;
             });
  // dKt = v_new dS'^T; dW = -dv_new S0^T (the [W] half of dY); dU = dv_new
  block_gemm<false, true>(kC, K, V, [&](int i, int c) { return vn[i * V + c]; },
             [&](int c, int k) { return dSn[k * V + c]; }, gsm,
             [&](int i, int k, float a) { dKt[i * K + k] = a; });
  block_gemm<false, true>(kC, K, V, [&](int i, int c) { return dvn[i * V + c]; },
             [&](int c, int k) { return S0[k * V + c]; }, gsm,
             [&](int i, int k, float a) { dRW[i * K + k] = -a; });
  block_map(dRU, dvn, kC * V, [](int, float x) { return x; });
  // dG_last from S' = e^(G_last) S0: sum_v S0 dS' e^(G_last); a warp per
  // row, its lanes along the row (coalesced), then a shuffle reduction.
  {
    const int lane = tid & 31, warp = tid >> 5, nwarp = nth >> 5;
    for (int k = warp; k < K; k += nwarp) {
      float s = 0.f;
      for (int c = lane; c < V; c += 32) s = fmaf(S0[k * V + c], dSn[k * V + c], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) dGl[k] = s * expf(Gs[(kC - 1) * KP + k]);
    }
  }
  __syncthreads();
  // dR = (I + T)^-T dY: back substitution, one column of [dU | dW] per thread.
  for (int c = tid; c < V + K; c += nth) {
    float* col = c < V ? dRU + c : dRW + (c - V);
    const int ld = c < V ? V : K;
    float x[kC];
#pragma unroll
    for (int i = kC - 1; i >= 0; --i) {
      float r = col[i * ld];
#pragma unroll
      for (int j = i + 1; j < kC; ++j) r = fmaf(-Ts[j * 65 + i], x[j], r);
      x[i] = r;
    }
#pragma unroll
    for (int i = 0; i < kC; ++i) col[i * ld] = x[i];
  }
  __syncthreads();
  // dT = -dR [U | W]^T on the strict lower triangle
  block_gemm<false, true>(kC, kC, V + K,
             [&](int i, int c) { return c < V ? dRU[i * V + c] : dRW[i * K + c - V]; },
             [&](int c, int j) { return c < V ? Um[j * V + c] : Wm[j * K + c - V]; }, gsm,
             [&](int i, int j, float a) { Dt[i * 65 + j] = j < i ? -a : 0.f; });
  // dv = dR_U w, dw = dR_U v (R_V = w * v, naive.py:346)
  for (int e = tid; e < kC * V / 8; e += nth) {
    const int i = e / (V / 8), c0 = 8 * (e % (V / 8)), t = t0 + i;
    if (t < f.T) {
      float w8[8], v8[8], d8[8];
      load8_any(f.w.p, f.w.dt, f.w.off(b, t, h, c0), f.w.sd, w8);
      load8_any(f.v.p, f.v.dt, f.v.off(b, t, h, c0), f.v.sd, v8);
#pragma unroll
      for (int u = 0; u < 8; ++u) d8[u] = dRU[i * V + c0 + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        p.dv[orow(i, V) + c0 + u] = d8[u] * w8[u];
        p.dw[orow(i, V) + c0 + u] = d8[u] * v8[u];
      }
    }
  }
  // Column pass over the decayed blocks: for key j, sums over the rows i.
  // e^(G_i - G_j) is a running product of the steps' e^g (exact to a few ulp);
  // a channel with a positive log-decay in the chunk takes the reference's
  // clamped exponent term by term instead.
  for (int e = tid; e < kC * K; e += nth) {
    const int j = e / K, d = e % K;
    const float gj = Gs[j * KP + d];
    const bool exact = npos[d] != 0;
    float acc = 0.f, accg = 0.f, ex = 1.f;
    if (!exact) {
      // (The same sums as below without the clamp: every exponent is <= 0,
      // so both accumulate every term; one chain, fewer instructions.)
      acc = As[j * 65 + j] * Qs[j * KP + d];
      for (int i = j + 1; i < kC; ++i) {
        ex *= Eg[i * KP + d];
        const float term = Dt[i * 65 + j] * Bs[i * KP + d] * Ks[i * KP + d] +
                           As[i * 65 + j] * Qs[i * KP + d];
        acc = fmaf(term, ex, acc);
      }
      accg = acc;
    } else {
      for (int i = j; i < kC; ++i) {
        const float x = Gs[i * KP + d] - gj;
        ex = expf(fminf(x, 0.f));
        const float term = (i > j ? Dt[i * 65 + j] * Bs[i * KP + d] * Ks[i * KP + d] : 0.f) +
                           As[i * 65 + j] * Qs[i * KP + d];
        acc = fmaf(term, ex, acc);
        if (x <= 0.f) accg = fmaf(term, ex, accg);
      }
    }
    dKTA[j * K + d] = acc;
    dGc[j * K + d] = -Ks[j * KP + d] * accg;
  }
  __syncthreads();
  // Row pass and assembly of every gradient of the token row.
  for (int e = tid; e < kC * K; e += nth) {
    const int i = e / K, d = e % K, t = t0 + i;
    const float gi = Gs[i * KP + d];
    const bool exact = npos[d] != 0;
    float dbk = 0.f, dqs = 0.f, gbk = 0.f, gqs = 0.f, ex = 1.f;
    if (!exact) {
      // (As in the column pass: no clamp, one pair of chains.)
      dqs = As[i * 65 + i] * Ks[i * KP + d];
      for (int j = i - 1; j >= 0; --j) {
        ex *= Eg[(j + 1) * KP + d];
        const float kx = Ks[j * KP + d] * ex;
        dbk = fmaf(Dt[i * 65 + j], kx, dbk);
        dqs = fmaf(As[i * 65 + j], kx, dqs);
      }
      gbk = dbk;
      gqs = dqs;
    } else {
      for (int j = i; j >= 0; --j) {
        const float x = gi - Gs[j * KP + d];
        ex = expf(fminf(x, 0.f));
        const float kx = Ks[j * KP + d] * ex;
        const float tt = j < i ? Dt[i * 65 + j] : 0.f, aa = As[i * 65 + j];
        dbk = fmaf(tt, kx, dbk);
        dqs = fmaf(aa, kx, dqs);
        if (x <= 0.f) {
          gbk = fmaf(tt, kx, gbk);
          gqs = fmaf(aa, kx, gqs);
        }
      }
    }
    const float q = Qs[i * KP + d], k = Ks[i * KP + d], bb = Bs[i * KP + d];
    const float eG = expf(gi), eT = expf(Gs[(kC - 1) * KP + d] - gi);
    const float rw = dRW[i * K + d], qg = dQG[i * K + d], kt = dKt[i * K + d];
    dGc[i * K + d] += bb * k * gbk + q * gqs + rw * k * bb * eG + qg * q * eG - kt * k * eT;
    if (t < f.T) {
      p.dq[(int64_t(b) * f.T + t) * f.H * f.L * K + (int64_t(h) * f.L) * K + d] =
          f.scale * (dqs + qg * eG);
      p.db[orow(i, K) + d] = rw * k * eG + dbk * k;
      p.dk[orow(i, K) + d] = rw * bb * eG + dbk * bb + kt * eT + dKTA[i * K + d];
    }
  }
  __syncthreads();
  // g: dG_last (with the Kt part, sum_i dKt k e^(G_last - G)) joins the last
  // row, then reverse cumsum (G = cumsum g).
  if (tid < K) {
    float acc = dGl[tid];
    const float gl = Gs[(kC - 1) * KP + tid];
#pragma unroll 8
    for (int i = 0; i < kC; ++i)
      acc += dKt[i * K + tid] * Ks[i * KP + tid] * expf(gl - Gs[i * KP + tid]);
#pragma unroll 8
    for (int i = kC - 1; i >= 0; --i) {
      acc += dGc[i * K + tid];
      if (t0 + i < f.T) p.dg[orow(i, K) + tid] = acc;
    }
  }
  // Upper-level reads (naive.py:382-385): dq_l = mix_l scale dO S_l^T,
  // dmix_l = scale sum_v dO (q_l S_l), S_l the state entering the chunk.
  for (int l = 1; l < f.L; ++l) {
    const float* Sl = ck_level(f, bh, l, n / f.firing[l]);
    __syncthreads();
    for (int i = tid; i < kC; i += nth) mx[i] = t0 + i < f.T ? f.mix.at(b, t0 + i, h, l) : 0.f;
    // q_l of the chunk, staged as fp32 in the spent dR_W scratch
    for (int e = tid; e < kC * K / 8; e += nth) {
      const int i = e / (K / 8), d0 = 8 * (e % (K / 8)), t = t0 + i;
      float q8[8];
      if (t < f.T) {
        load8_any(f.q.p, f.q.dt, f.q.off(b, t, h, l, d0), f.q.sd, q8);
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) q8[u] = 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) dRW[i * K + d0 + u] = q8[u];
    }
    __syncthreads();
    block_gemm<false, true>(kC, K, V, [&](int i, int c) { return dO(i, c); },
               [&](int c, int k) { return Sl[k * V + c]; }, gsm,
               [&](int i, int k, float a) {
                 if (t0 + i < f.T)
                   p.dq[(int64_t(b) * f.T + t0 + i) * f.H * f.L * K + (int64_t(h) * f.L + l) * K + k] =
                       f.scale * mx[i] * a;
               });
    block_gemm(kC, V, K,
               [&](int i, int k) { return dRW[i * K + k]; },
               [&](int k, int c) { return Sl[k * V + c]; }, gsm,
               [&](int i, int c, float a) { dRU[i * V + c] = a * dO(i, c); });
    row_sums(dRU, kC, V, [&](int i, float s2) {
      if (t0 + i < f.T) p.dmix[(int64_t(b) * f.T + t0 + i) * f.H * f.L + h * f.L + l] = f.scale * s2;
    });
  }
}

}  // namespace ngdn2

namespace ngdn2 {

cudaError_t launch_fwd_simt(const FwdParams& p, int stage, cudaStream_t stream);

// Workspace of the backward, in floats, region by region.
struct BwdLayout {
  int64_t params32, chunks, scan, fin, ck0, ck_up, ck_vnew, ck_ta, dparams, dS, dsn, dvn, pscr,
      lscr, size;
  int64_t ck_up_off[NGDN2_MAX_LEVELS];
  int ck_up_n[NGDN2_MAX_LEVELS];
};

BwdLayout bwd_layout(const FwdParams& f, const PromoBwdScratch& ps, const LocalScratch& ls) {
  BwdLayout w;
  const int64_t bh = int64_t(f.B) * f.H, kv = int64_t(f.K) * f.V, cv = int64_t(kC) * f.V;
  int64_t o = 0;
  auto take = [&](int64_t n) { const int64_t at = o; o = align_floats(o + n); return at; };
  w.params32 = take(f.pl.size);
  w.chunks = take(bh * f.NT * f.rec.size);
  w.scan = take(bh * f.ss.size);
  w.fin = take(bh * f.L * kv);
  w.ck0 = take(bh * (f.NT + 1) * kv);
  int64_t up = 0;
  for (int l = 0; l < NGDN2_MAX_LEVELS; ++l) {
    w.ck_up_off[l] = up;
    w.ck_up_n[l] = 0;
    if (l >= 1 && l < f.L) {
      w.ck_up_n[l] = (f.NT + f.firing[l] - 1) / f.firing[l] + 1;
      up = align_floats(up + bh * w.ck_up_n[l] * kv);
    }
  }
  w.ck_up = take(up);
  w.ck_vnew = take(bh * f.NT * cv);
  w.ck_ta = take(bh * f.NT * 2 * kC * kC);
  w.dparams = take(int64_t(f.B) * f.pl.size);
  w.dS = take(bh * f.L * kv);
  w.dsn = take(bh * f.NT * kv);
  w.dvn = take(bh * f.NT * cv);
  w.pscr = take(bh * ps.size);
  w.lscr = take(bh * f.NT * ls.size);
  w.size = o;
  return w;
}

int64_t bwd_workspace_floats(const FwdParams& f) {
  return bwd_layout(f, PromoBwdScratch::make(f.K, f.V, f.NP), LocalScratch::make(f.K, f.V)).size;
}

int num_launches_bwd(const FwdParams& f) {
  return (f.L > 1 ? 2 : 0) + (f.NT > 0 ? 1 : 0) + 1 + 1 + (f.NT > 0 ? 1 : 0);
}

// x[i] = sum over rows r < R of x[r * n + i], in row order.
__global__ void reduce_rows_kernel(float* x, int64_t n, int R) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    float s = x[i];
    for (int r = 1; r < R; ++r) s += x[r * n + i];
    x[i] = s;
  }
}

// The forward's SIMT prep and checkpointing scan, then the two backward
// kernels. `bp` carries the caller's pointers; the workspace regions are
// filled in here.
cudaError_t launch_bwd(BwdParams bp, float* ws, float* const dparam_out[5], cudaStream_t stream) {
  FwdParams& f = bp.f;
  bp.ps = PromoBwdScratch::make(f.K, f.V, f.NP);
  bp.ls = LocalScratch::make(f.K, f.V);
  const BwdLayout w = bwd_layout(f, bp.ps, bp.ls);
  f.params32 = ws + w.params32;
  f.chunks = ws + w.chunks;
  f.scan = ws + w.scan;
  f.fin = ws + w.fin;
  f.o = nullptr;
  f.ck0 = ws + w.ck0;
  f.ck_up = ws + w.ck_up;
  for (int l = 0; l < NGDN2_MAX_LEVELS; ++l) {
    f.ck_up_off[l] = w.ck_up_off[l];
    f.ck_up_n[l] = w.ck_up_n[l];
  }
  f.ck_vnew = ws + w.ck_vnew;
  f.ck_ta = ws + w.ck_ta;
  bp.dparams = f.L > 1 ? ws + w.dparams : nullptr;
  bp.dS = ws + w.dS;
  bp.dsn = ws + w.dsn;
  bp.dvn = ws + w.dvn;
  bp.pscr = ws + w.pscr;
  bp.lscr = ws + w.lscr;
  cudaError_t err = launch_fwd_simt(f, 0, stream);
  if (err != cudaSuccess) return err;
  if (bp.dparams) {
    err = cudaMemsetAsync(bp.dparams, 0, sizeof(float) * f.B * f.pl.size, stream);
    if (err != cudaSuccess) return err;
  }
  {
    const int dyn = tc::kTc3StageBytes + 1024;  // staging of the tensor-core products, 1 KB aligned
    err = cudaFuncSetAttribute(bwd_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (err != cudaSuccess) return err;
    bwd_scan_kernel<<<dim3(f.H, f.B), 256, dyn, stream>>>(bp);
  }
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  if (f.NT > 0) {
    const size_t smem = bwd_local_smem(f.K);
    err = cudaFuncSetAttribute(bwd_local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               int(smem));
    if (err != cudaSuccess) return err;
    bwd_local_kernel<<<dim3(f.NT, f.H, f.B), 256, smem, stream>>>(bp);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  if (bp.dparams) {
    reduce_rows_kernel<<<256, 256, 0, stream>>>(bp.dparams, f.pl.size, f.B);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    const int64_t n = int64_t(f.L - 1) * f.H;
    const int64_t counts[5] = {n * f.n_max * f.K, n * f.K * f.V, n * f.V * f.K, n * f.V * f.V,
                               n * f.V * f.K};
    const int64_t offs[5] = {f.pl.qb, f.pl.kp, f.pl.bp, f.pl.wp, f.pl.gp};
    for (int a = 0; a < 5; ++a) {
      if (!dparam_out[a]) continue;
      err = cudaMemcpyAsync(dparam_out[a], bp.dparams + offs[a], sizeof(float) * counts[a],
                            cudaMemcpyDeviceToDevice, stream);
      if (err != cudaSuccess) return err;
    }
  }
  return cudaSuccess;
}

}  // namespace ngdn2

namespace ngdn2 {

cudaError_t launch_bwd_abi(const ngdn2_bwd_args* a, const FwdParams& f, cudaStream_t stream) {
  BwdParams bp;
  memset(&bp, 0, sizeof(bp));
  bp.f = f;
  bp.d_o = a->d_o;
  bp.d_o_dtype = a->d_o_dtype;
  for (int i = 0; i < 4; ++i) bp.dos[i] = a->d_o_stride[i];
  bp.d_final = a->d_final;
  bp.dq = a->dq;
  bp.dk = a->dk;
  bp.dv = a->dv;
  bp.dg = a->dg;
  bp.db = a->db;
  bp.dw = a->dw;
  bp.dmix = a->dmix;
  bp.dinit = a->dinitial_state;
  float* const outs[5] = {a->dquery_banks, a->dkey_projections, a->db_projections,
                          a->dw_projections, a->dg_projections};
  return launch_bwd(bp, reinterpret_cast<float*>(a->workspace), outs, stream);
}

}  // namespace ngdn2
