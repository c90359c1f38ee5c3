// Backward of the promotion write scan (update_bwd.py:167-263,
// update_state_bwd) on CUDA cores in fp32.
//
// The forward scan (update_fwd.py:131-204) keeps states[j] = S_j for every
// group j < NG and applies, at every firing j < NF, the update step of
// naive.py:7-39:
//   S_d = e^g S_j,  S_{j+1} = S_d - K^T (K * b) S_d + K^T (V * w).
// Given d_states and d_final, the firings are reversed one by one with the
// stored S_j: with Z = K dS', Y = (K * b) S_d,
//   dK = (V * w - Y) dS'^T + d(K*b) * b,  d(K*b) = -Z S_d^T,  db = d(K*b) * K,
//   dS_d = dS' - (K * b)^T Z,  dg = sum_v dS_d * S_d,  dS = e^g dS_d,
//   dV = Z * w,  dw = Z * V,
// and the gradient flowing into S_j gains d_states[j]. One CTA per (b, h)
// walks the firings in reverse; the reference splits V into blocks and sums
// partial dkeys / db / dg afterwards, which this full-V CTA does not need.

#include "fwd_params.cuh"

namespace ngdn2 {

__host__ __device__ inline int64_t upd_bwd_scratch_floats(int K, int V, int N) {
  const int64_t kv = int64_t(K) * V, nv = int64_t(N) * V;
  return align_floats(kv) * 3 + align_floats(nv) * 2;
}

__global__ void __launch_bounds__(256) update_bwd_kernel(UpdBwdParams u) {
  __shared__ float gsm[kGemmSmemFloats];
  __shared__ float gsh[128];  // e^g of the firing
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, nth = blockDim.x;
  const int K = u.K, V = u.V, N = u.N;
  const int64_t bh = int64_t(b) * u.H + h, kv = int64_t(K) * V;
  float* dS = u.scr + bh * upd_bwd_scratch_floats(K, V, N);
  float* Sd = dS + align_floats(kv);
  float* dSd = Sd + align_floats(kv);
  float* Z = dSd + align_floats(kv);
  float* Y = Z + align_floats(int64_t(N) * V);
  const int warp = tid / 32, lane = tid % 32, nwarp = nth / 32;
  auto st_at = [&](const float* base, int j) { return base + ((int64_t(b) * u.NG + j) * u.H + h) * kv; };
  // dS' entering the reverse walk: d_final, plus d_states of the last group
  // when that group's state is the final one (NG = NF + 1).
  for (int64_t e = tid; e < kv; e += nth) {
    float d = u.d_final[bh * kv + e];
    if (u.NG > u.NF) d += st_at(u.d_states, u.NF)[e];
    dS[e] = d;
  }
  __syncthreads();
  for (int j = u.NF - 1; j >= 0; --j) {
    const int64_t fb = (int64_t(b) * u.NF + j) * u.H + h;  // firing row
    const int64_t kbase = b * u.skb + j * u.skf + h * u.skh;
    auto key = [&](int r, int k) { return load_elem(u.keys, kbase + r * u.skn + k, u.dtype); };
    auto bb = [&](int r, int k) { return load_elem(u.b, (fb * N + r) * K + k, u.dtype); };
    auto val = [&](int r, int c) { return load_elem(u.values, (fb * N + r) * V + c, u.dtype); };
    auto wg = [&](int r, int c) { return load_elem(u.w, (fb * N + r) * V + c, u.dtype); };
    const float* S = st_at(u.states, j);
    for (int k = tid; k < K; k += nth) gsh[k] = expf(load_elem(u.g, fb * K + k, u.g_dtype));
    __syncthreads();
    for (int64_t e = tid; e < kv; e += nth) Sd[e] = gsh[e / V] * S[e];
    __syncthreads();
    // Z = K dS', Y = (K * b) S_d
    block_gemm(N, V, K, key, [&](int k, int c) { return dS[k * V + c]; }, gsm,
               [&](int r, int c, float a) { Z[r * V + c] = a; });
    block_gemm(N, V, K, [&](int r, int k) { return key(r, k) * bb(r, k); },
               [&](int k, int c) { return Sd[k * V + c]; }, gsm,
               [&](int r, int c, float a) { Y[r * V + c] = a; });
    // dK = (V * w - Y) dS'^T; d(K*b) = -Z S_d^T, added as d(K*b) * b, and
    // db = d(K*b) * K.
    float* dk = u.dkeys + fb * N * K;
    float* db = u.db + fb * N * K;
    block_gemm<false, true>(N, K, V,
                            [&](int r, int c) { return val(r, c) * wg(r, c) - Y[r * V + c]; },
                            [&](int c, int k) { return dS[k * V + c]; }, gsm,
                            [&](int r, int k, float a) { dk[r * K + k] = a; });
    block_gemm<false, true>(N, K, V, [&](int r, int c) { return Z[r * V + c]; },
                            [&](int c, int k) { return Sd[k * V + c]; }, gsm,
                            [&](int r, int k, float a) {
                              dk[r * K + k] -= a * bb(r, k);
                              db[r * K + k] = -a * key(r, k);
                            });
    // dV = Z * w, dw = Z * V
    for (int e = tid; e < N * V; e += nth) {
      const int r = e / V, c = e % V;
      u.dvalues[fb * N * V + e] = Z[e] * wg(r, c);
      u.dw[fb * N * V + e] = Z[e] * val(r, c);
    }
    // dS_d = dS' - (K * b)^T Z
    block_gemm<true, false>(K, V, N, [&](int k, int r) { return key(r, k) * bb(r, k); },
                            [&](int r, int c) { return Z[r * V + c]; }, gsm,
                            [&](int k, int c, float a) { dSd[k * V + c] = dS[k * V + c] - a; });
    // dg = sum_v dS_d S_d; dS (into S_j) = e^g dS_d + d_states[j]
    for (int k = warp; k < K; k += nwarp) {
      float s = 0.f;
      for (int c = lane; c < V; c += 32) s = fmaf(dSd[k * V + c], Sd[k * V + c], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) u.dg[fb * K + k] = s;
    }
    const float* dst = st_at(u.d_states, j);
    for (int64_t e = tid; e < kv; e += nth) dS[e] = gsh[e / V] * dSd[e] + dst[e];
    __syncthreads();
  }
  if (u.has_init && u.dinit)
    for (int64_t e = tid; e < kv; e += nth) u.dinit[bh * kv + e] = dS[e];
}

cudaError_t launch_update_bwd(const UpdBwdParams& u, cudaStream_t stream) {
  update_bwd_kernel<<<dim3(u.H, u.B), 256, 0, stream>>>(u);
  return cudaGetLastError();
}

}  // namespace ngdn2
