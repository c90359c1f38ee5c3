// CUDA-core (SIMT) kernel family: fp32 arithmetic throughout.
//
// This is the precision path (fp32 inputs, parity at rel 1e-4) and the path
// for shapes the tensor-core family does not cover. It keeps the two-stage
// structure of the fast path:
//
//   prep  -- one CTA per (b, h, chunk), fully parallel. Per chunk it forms
//            the S-independent operands of the chunkwise gated delta rule
//            (nested_gdn2/ops/naive.py:329-352): cumulative log-decay G,
//            the decay-masked K.K^T and Q.K^T blocks, the unit-lower-
//            triangular solve [U | W] = (I + A_kk)^-1 [w*v | k*b*e^G], the
//            read queries with mix and scale folded in, k*e^(G_last - G)
//            and e^(G_last). Decays follow the reference's clamped exponent
//            e^min(G_i - G_j, 0): element by element where a log-decay is
//            positive, as a row-factor x column-factor GEMM where none is
//            (the clamp cannot bind there).
//   scan  -- one CTA per (b, h), sequential over chunks: the state
//            recurrence and output of level 0 (naive.py:376-392), the reads
//            of levels >= 1 (naive.py:382-390) and, at each firing, the
//            promotion of the level below into the level above
//            (naive.py:394-415, probe.py:34-136, naive.py:7-39).
//
// States live in the caller's final_state buffer (fp32 [B, H, L, K, V]),
// which doubles as the running state; per-(b, h) temporaries live in the
// workspace.

#include <type_traits>

#include "fwd_params.cuh"
#include "promote_simt.cuh"

namespace ngdn2 {

__global__ void convert_params_kernel(FwdParams p) {
  if (gate_closed(p)) return;
  const int64_t n = int64_t(p.L - 1) * p.H;
  const int64_t counts[5] = {n * p.n_max * p.K, n * p.K * p.V, n * p.V * p.K,
                             n * p.V * p.V, n * p.V * p.K};
  const int64_t offs[5] = {p.pl.qb, p.pl.kp, p.pl.bp, p.pl.wp, p.pl.gp};
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int a = 0; a < 5; ++a) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < counts[a]; i += stride)
      p.params32[offs[a] + i] = load_elem(p.raw_params[a], i, p.param_dtype);
  }
}

// ---------------------------------------------------------------------------
// prep: grid (NT, H, B), 256 threads.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) prep_simt_kernel(FwdParams p) {
  if (gate_closed(p)) return;
  extern __shared__ float sm[];
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int K = p.K, V = p.V, KP = K + 1;
  float* Gs = sm;              // [64][K+1] cumulative log-decay
  float* Qs = Gs + kC * KP;    // [64][K+1] level-0 query
  float* Ks = Qs + kC * KP;    // [64][K+1] key
  float* BKs = Ks + kC * KP;   // [64][K+1] b * k
  float* Akk = BKs + kC * KP;  // [64][65]
  float* Aqk = Akk + kC * 65;  // [64][65]
  float* mixs = Aqk + kC * 65 + kGemmSmemFloats;  // [64][L] mix of the rows
  const int tid = threadIdx.x, L = p.L;
  const int t0 = n * kC;

  // Load the chunk, 8 channels per load and all four inputs before any
  // store; tokens past T are zero (naive.py:302-312).
  for (int e = tid; e < kC * K / 8; e += blockDim.x) {
    const int i = e / (K / 8), d0 = 8 * (e % (K / 8)), t = t0 + i;
    float q8[8], k8[8], g8[8], b8[8];
    if (t < p.T) {
      load8_any(p.q.p, p.q.dt, p.q.off(b, t, h, 0, d0), p.q.sd, q8);
      load8_any(p.k.p, p.k.dt, p.k.off(b, t, h, d0), p.k.sd, k8);
      load8_any(p.g.p, p.g.dt, p.g.off(b, t, h, d0), p.g.sd, g8);
      load8_any(p.b.p, p.b.dt, p.b.off(b, t, h, d0), p.b.sd, b8);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) q8[u] = k8[u] = g8[u] = b8[u] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int x = i * KP + d0 + u;
      Qs[x] = q8[u];
      Ks[x] = k8[u];
      Gs[x] = g8[u];
      BKs[x] = b8[u] * k8[u];
    }
  }
  for (int e = tid; e < kC * L; e += blockDim.x) {
    const int i = e / L, l = e % L, t = t0 + i;
    mixs[e] = t < p.T ? p.mix.at(b, t, h, l) : 0.f;
  }
  __syncthreads();
  // G = cumsum of g along the chunk (naive.py:329).
  if (tid < K) {
    float acc = 0.f;
    for (int i = 0; i < kC; ++i) {
      acc += Gs[i * KP + tid];
      Gs[i * KP + tid] = acc;
    }
  }
  __syncthreads();
  // A_kk (strictly lower) and A_qk (lower, diagonal included) with the
  // clamped per-channel decay (naive.py:335-344, 354-358, 377-378).
  //
  // When every log-decay of the chunk is <= 0 (G non-increasing along the
  // chunk on every channel) the clamp never binds for j <= i, and
  // e^(G_i - G_j) = e^(G_i - G_0) e^(G_0 - G_j) splits into a row and a
  // column factor: both blocks become one 128 x 64 x K GEMM over
  // [q e^(G-G_0) ; b k e^(G-G_0)] and (k e^(G_0-G))^T, with 2 * 64 * K
  // exponentials instead of one per (i, j, d). The split needs
  // G_0 - G_63 <= 80 so that e^(G_0 - G_j) stays finite in fp32; other
  // chunks (and K not a multiple of 16) take the exact per-element loop.
  __shared__ int factored;
  float* gsm = Aqk + kC * 65;  // block_gemm staging
  if (tid == 0) factored = (K % 16) == 0;
  __syncthreads();
  if (tid < K) {
    bool ok = Gs[tid] - Gs[(kC - 1) * KP + tid] <= 80.f;
    for (int i = 1; i < kC; ++i) ok = ok && Gs[i * KP + tid] <= Gs[(i - 1) * KP + tid];
    if (!ok) factored = 0;
  }
  __syncthreads();
  float* ta = p.ck_ta ? p.ck_ta + ((int64_t(b) * p.H + h) * p.NT + n) * 2 * kC * kC : nullptr;
  if (factored) {
    block_gemm<false, true>(
        2 * kC, kC, K,
        [&](int r, int d) {
          const int i = r < kC ? r : r - kC;
          const float x = r < kC ? Qs[i * KP + d] : BKs[i * KP + d];
          return x * expf(Gs[i * KP + d] - Gs[d]);
        },
        [&](int d, int j) { return Ks[j * KP + d] * expf(Gs[d] - Gs[j * KP + d]); }, gsm,
        [&](int r, int j, float a) {
          if (r < kC) {
            Aqk[r * 65 + j] = j <= r ? a : 0.f;
          } else {
            const int i = r - kC;
            Akk[i * 65 + j] = j < i ? a : 0.f;
          }
        });
    __syncthreads();
    if (ta) {
      for (int e = tid; e < kC * kC; e += blockDim.x) {
        const int i = e / kC, j = e % kC;
        ta[e] = Akk[i * 65 + j];
        ta[kC * kC + e] = Aqk[i * 65 + j] * p.scale;
      }
    }
  } else {
    for (int e = tid; e < kC * kC; e += blockDim.x) {
      const int i = e / kC, j = e % kC;
      float aq = 0.f, ak = 0.f;
      if (j <= i) {
        const float* gi = Gs + i * KP;
        const float* gj = Gs + j * KP;
        const float* qi = Qs + i * KP;
        const float* bki = BKs + i * KP;
        const float* kj = Ks + j * KP;
        for (int d = 0; d < K; ++d) {
          const float kd = kj[d] * expf(fminf(gi[d] - gj[d], 0.f));
          aq = fmaf(qi[d], kd, aq);
          ak = fmaf(bki[d], kd, ak);
        }
      }
      Aqk[i * 65 + j] = aq;
      Akk[i * 65 + j] = (j < i) ? ak : 0.f;
      if (ta) {
        ta[e] = (j < i) ? ak : 0.f;
        ta[kC * kC + e] = aq * p.scale;
      }
    }
  }
  __syncthreads();

  float* rec = p.chunks + ((int64_t(b) * p.H + h) * p.NT + n) * p.rec.size;

  // [U | W] = (I + A_kk)^-1 [w * v | k * b * e^G] by forward substitution,
  // one column per thread (naive.py:346-351).
  const int c = tid;
  if (c < V + K) {
    // Right-hand sides first (their global loads all in flight), then the
    // dependent substitution chain.
    float x[kC];
    if (c < V) {
      auto rhs = [&](auto dt) {
        constexpr int DT = decltype(dt)::value;
#pragma unroll
        for (int i = 0; i < kC; ++i) {
          const int t = t0 + i;
          x[i] = (t < p.T) ? load_typed<DT>(p.w.p, p.w.off(b, t, h, c)) *
                                 load_typed<DT>(p.v.p, p.v.off(b, t, h, c))
                           : 0.f;
        }
      };
      if (p.w.dt == p.v.dt && p.w.dt == NGDN2_BF16) {
        rhs(std::integral_constant<int, NGDN2_BF16>());
      } else if (p.w.dt == p.v.dt && p.w.dt == NGDN2_F16) {
        rhs(std::integral_constant<int, NGDN2_F16>());
      } else if (p.w.dt == p.v.dt && p.w.dt == NGDN2_F32) {
        rhs(std::integral_constant<int, NGDN2_F32>());
      } else {
#pragma unroll
        for (int i = 0; i < kC; ++i) {
          const int t = t0 + i;
          x[i] = (t < p.T) ? p.w.at(b, t, h, c) * p.v.at(b, t, h, c) : 0.f;
        }
      }
    } else {
      const int d = c - V;
#pragma unroll
      for (int i = 0; i < kC; ++i) x[i] = BKs[i * KP + d] * expf(Gs[i * KP + d]);
    }
#pragma unroll
    for (int i = 0; i < kC; ++i) {
      float r = x[i];
#pragma unroll
      for (int j = 0; j < i; ++j) r = fmaf(-Akk[i * 65 + j], x[j], r);
      x[i] = r;
    }
#pragma unroll
    for (int i = 0; i < kC; ++i) {
      if (c < V) rec[p.rec.U + i * V + c] = x[i];
      else rec[p.rec.W + i * K + (c - V)] = x[i];
    }
  }

  // Output-side operands.
  for (int e = tid; e < kC * kC; e += blockDim.x) {
    const int i = e / kC, j = e % kC;
    const float m0 = mixs[i * L];
    rec[p.rec.A + e] = (j <= i) ? Aqk[i * 65 + j] * p.scale * m0 : 0.f;
  }
  for (int e = tid; e < kC * K; e += blockDim.x) {
    const int i = e / K, d = e % K;
    const float m0 = mixs[i * L];
    const float gi = Gs[i * KP + d];
    rec[p.rec.Q + e] = m0 * p.scale * Qs[i * KP + d] * expf(gi);
    rec[p.rec.Kt + e] = Ks[i * KP + d] * expf(Gs[(kC - 1) * KP + d] - gi);
  }
  for (int l = 1; l < L; ++l) {
    float* dst = rec + p.rec.Q + int64_t(l) * kC * K;
    for (int e = tid; e < kC * K / 8; e += blockDim.x) {
      const int i = e / (K / 8), d0 = 8 * (e % (K / 8)), t = t0 + i;
      float q8[8];
      if (t < p.T) {
        load8_any(p.q.p, p.q.dt, p.q.off(b, t, h, l, d0), p.q.sd, q8);
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) q8[u] = 0.f;
      }
      const float sc = mixs[i * L + l] * p.scale;
#pragma unroll
      for (int u = 0; u < 8; ++u) dst[i * K + d0 + u] = sc * q8[u];
    }
  }
  if (tid < K) rec[p.rec.eg + tid] = expf(Gs[(kC - 1) * KP + tid]);
}

// ---------------------------------------------------------------------------
// scan: grid (H, B), 256 threads.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) scan_simt_kernel(FwdParams p) {
  if (gate_closed(p)) return;
  __shared__ float gsm[kGemmSmemFloats];
  const int h = blockIdx.x, b = blockIdx.y;
  const int K = p.K, V = p.V, L = p.L, tid = threadIdx.x;
  const int64_t bh = int64_t(b) * p.H + h;
  float* S = p.fin + bh * L * K * V;
  float* sc = p.scan + bh * p.ss.size;
  for (int64_t e = tid; e < int64_t(L) * K * V; e += blockDim.x)
    S[e] = p.init ? p.init[bh * L * K * V + e] : 0.f;
  __syncthreads();
  float* Vn = sc + p.ss.vn;
  float* Ot = sc + p.ss.ot;
  const bool ckpt = p.ck0 != nullptr;
  // Backward checkpoints: a copy of the state of `level` into slot `j`.
  auto save = [&](int level, int j) {
    const float* src = S + int64_t(level) * K * V;
    float* dst = level == 0 ? p.ck0 + (bh * (p.NT + 1) + j) * K * V
                            : p.ck_up + p.ck_up_off[level] + (bh * p.ck_up_n[level] + j) * K * V;
    block_map(dst, src, K * V, [](int, float x) { return x; });
  };
  for (int n = 0; n < p.NT; ++n) {
    const float* rec = p.chunks + (bh * p.NT + n) * p.rec.size;
    if (ckpt) {
      save(0, n);
      for (int l = 1; l < L; ++l)
        if (n % p.firing[l] == 0) save(l, n / p.firing[l]);
      __syncthreads();
    }
    const float* Wm = rec + p.rec.W;
    const float* Um = rec + p.rec.U;
    const float* Am = rec + p.rec.A;
    const float* Qm = rec + p.rec.Q;
    const float* Kt = rec + p.rec.Kt;
    const float* eg = rec + p.rec.eg;
    // v_new = U - W S0 (naive.py:376)
    block_gemm(kC, V, K, [&](int i, int k) { return Wm[i * K + k]; },
               [&](int k, int c) { return S[k * V + c]; }, gsm,
               [&](int i, int c, float a) {
                 Vn[i * V + c] = Um[i * V + c] - a;
                 if (ckpt) p.ck_vnew[(bh * p.NT + n) * kC * V + i * V + c] = Um[i * V + c] - a;
               });
    // o = sum_l (mix_l scale q_l [e^G at l=0]) S_l + mix_0 scale A_qk v_new
    // (not formed when only the backward's checkpoints are wanted)
    for (int l = 0; l < L && p.o; ++l) {
      const float* Ql = Qm + int64_t(l) * kC * K;
      const float* Sl = S + int64_t(l) * K * V;
      block_gemm(kC, V, K, [&](int i, int k) { return Ql[i * K + k]; },
                 [&](int k, int c) { return Sl[k * V + c]; }, gsm,
                 [&](int i, int c, float a) {
                   if (l == 0) Ot[i * V + c] = a; else Ot[i * V + c] += a;
                 });
    }
    if (p.o)
      block_gemm(kC, V, kC, [&](int i, int j) { return Am[i * kC + j]; },
                 [&](int j, int c) { return Vn[j * V + c]; }, gsm,
                 [&](int i, int c, float a) { Ot[i * V + c] += a; });
    for (int e = tid; e < kC * V && p.o; e += blockDim.x) {
      const int i = e / V, c = e % V, t = n * kC + i;
      if (t < p.T) store_elem(p.o, ((int64_t(b) * p.T + t) * p.H + h) * V + c, Ot[e], p.dtype);
    }
    // S0 <- e^(G_last) S0 + (k e^(G_last - G))^T v_new (naive.py:392)
    block_gemm<true, false>(K, V, kC, [&](int k, int i) { return Kt[i * K + k]; },
               [&](int i, int c) { return Vn[i * V + c]; }, gsm,
               [&](int k, int c, float a) { S[k * V + c] = eg[k] * S[k * V + c] + a; });
    // Levels whose firing this chunk completes, bottom-up (naive.py:394-415).
    for (int l = 1; l < L; ++l)
      if ((n + 1) % p.firing[l] == 0) promote_simt(p, b, h, l, S, sc, gsm);
  }
  if (ckpt) {
    __syncthreads();
    save(0, p.NT);
    for (int l = 1; l < L; ++l) save(l, p.ck_up_n[l] - 1);
  }
}

// ---------------------------------------------------------------------------
// update_state: grid (V / block_v, H, B), 256 threads.
// ---------------------------------------------------------------------------



__global__ void __launch_bounds__(256) update_simt_kernel(UpdParams u) {
  extern __shared__ float sm[];
  float* gsm = sm;
  float* vn = sm + kGemmSmemFloats;  // [N][bv]
  float* gs = vn + u.N * u.bv;       // [K]
  const int v0 = blockIdx.x * u.bv, h = blockIdx.y, b = blockIdx.z;
  const int K = u.K, V = u.V, N = u.N, bv = u.bv, tid = threadIdx.x;
  const int64_t bh = int64_t(b) * u.H + h;
  float* S = u.fin + bh * K * V;
  for (int e = tid; e < K * bv; e += blockDim.x) {
    const int k = e / bv, c = v0 + e % bv;
    S[k * V + c] = u.init ? u.init[bh * K * V + k * V + c] : 0.f;
  }
  __syncthreads();
  for (int j = 0; j < u.NG; ++j) {
    float* st = u.states + ((int64_t(b) * u.NG + j) * u.H + h) * K * V;
    for (int e = tid; e < K * bv; e += blockDim.x) {
      const int k = e / bv, c = v0 + e % bv;
      st[k * V + c] = S[k * V + c];
    }
    if (j >= u.NF) continue;
    const int64_t base = (int64_t(b) * u.NF + j) * u.H + h;
    for (int k = tid; k < K; k += blockDim.x) gs[k] = load_elem(u.g, base * K + k, u.g_dtype);
    __syncthreads();
    for (int e = tid; e < K * bv; e += blockDim.x) {
      const int k = e / bv, c = v0 + e % bv;
      S[k * V + c] *= expf(gs[k]);
    }
    __syncthreads();
    const int64_t kbase = b * u.skb + j * u.skf + h * u.skh;
    block_gemm(N, bv, K,
               [&](int r, int k) {
                 return load_elem(u.keys, kbase + r * u.skn + k, u.dtype) *
                        load_elem(u.b, (base * N + r) * K + k, u.dtype);
               },
               [&](int k, int c) { return S[k * V + v0 + c]; }, gsm,
               [&](int r, int c, float a) {
                 const int64_t o = (base * N + r) * V + v0 + c;
                 vn[r * bv + c] = load_elem(u.values, o, u.dtype) * load_elem(u.w, o, u.dtype) - a;
               });
    block_gemm(K, bv, N, [&](int k, int r) { return load_elem(u.keys, kbase + r * u.skn + k, u.dtype); },
               [&](int r, int c) { return vn[r * bv + c]; }, gsm,
               [&](int k, int c, float a) { S[k * V + v0 + c] += a; });
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------

size_t prep_simt_smem(int K, int L) {
  return sizeof(float) * (4 * kC * (K + 1) + 2 * kC * 65 + kGemmSmemFloats + kC * L);
}

cudaError_t launch_convert_params(const FwdParams& p, cudaStream_t stream) {
  if (p.L <= 1) return cudaSuccess;
  int64_t total = p.pl.size;
  int blocks = int((total + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  convert_params_kernel<<<blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

int num_launches_simt(const FwdParams& p) {
  return (p.L > 1 ? 1 : 0) + (p.NT > 0 ? 1 : 0) + 1;
}

cudaError_t launch_fwd_simt(const FwdParams& p, int stage, cudaStream_t stream) {
  cudaError_t err;
  if (stage == 0 || stage == 1) {
    if ((err = launch_convert_params(p, stream)) != cudaSuccess) return err;
    if (p.NT > 0) {
      const size_t smem = prep_simt_smem(p.K, p.L);
      err = cudaFuncSetAttribute(prep_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(smem));
      if (err != cudaSuccess) return err;
      prep_simt_kernel<<<dim3(p.NT, p.H, p.B), 256, smem, stream>>>(p);
      if ((err = cudaGetLastError()) != cudaSuccess) return err;
    }
  }
  if (stage == 0 || stage == 2) {
    scan_simt_kernel<<<dim3(p.H, p.B), 256, 0, stream>>>(p);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  return cudaSuccess;
}

cudaError_t launch_update_simt(const UpdParams& u, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (kGemmSmemFloats + size_t(u.N) * u.bv + u.K);
  cudaError_t err = cudaFuncSetAttribute(update_simt_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  update_simt_kernel<<<dim3(u.V / u.bv, u.H, u.B), 256, smem, stream>>>(u);
  return cudaGetLastError();
}

}  // namespace ngdn2
