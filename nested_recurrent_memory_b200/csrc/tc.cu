// Tensor-core (tcgen05) kernel family for K = V = 128, 16-bit inputs.
//
// Same two-stage structure as the CUDA-core family, with every chunk
// contraction on the 5th-generation tensor cores (bf16 operands staged in
// shared memory in UMMA canonical layouts, fp32 accumulators in TMEM):
//
//   prep_tc  -- one CTA per (b, h, chunk), two CTAs per SM. Builds the
//               decay-scaled operands, computes A_qk / A_kk with four
//               M=64 MMAs (one per 16-token block of queries, each with its
//               own decay reference point so no factor overflows), inverts
//               I + A_kk on CUDA cores in fp32 (16x16 diagonal blocks, then
//               block forward substitution), and forms [U | W] with one
//               M=64, N=256 MMA. Writes a chunk record whose operand tiles
//               are already in the scan's shared-memory layout.
//   scan_tc  -- one CTA per (b, h). The level-0 state S0 lives in TMEM
//               (fp32, lanes = key index) for the whole sequence, a bf16
//               copy of every level's state sits in shared memory as the
//               MMA B operand. Per chunk: bulk copies bring the record in,
//               MMA1 forms W.S0 and the level-0 read, the upper levels' reads
//               q_l.S_l run during E1 (v_new = U - W.S0), MMA2 adds
//               A_qk.v_new to the output and K_tail^T.v_new to S0, and E2
//               mixes the levels per row. Promotions of levels >= 1 run at
//               their firings as tcgen05 MMA round trips (promote_tc for the
//               learned arm, promote_merge_tc for the merge arm) against fp32
//               master states.
//
// Reference: level 0 follows nested_gdn2/ops/naive.py:329-392 (chunk form of
// fla's GDN-2, chunk.py:236-248), reads and mix naive.py:382-390, promotion
// naive.py:394-415 with probe.py:34-136.

#include <cuda.h>
#include <string.h>
#include <cudaTypedefs.h>

#include "tc_api.cuh"
#include "tc_common.cuh"
#include "tc_ptx.cuh"

namespace ngdn2 {


namespace {

using namespace tcx;

}  // namespace
}  // namespace ngdn2

namespace ngdn2 {
namespace {

// ---------------------------------------------------------------------------
// tc_params: grid (L-1, H, kParamSlices). Promotion operands of each
// (level, head) in the scan's shared-memory layouts (bf16), read by bulk
// copies at firings. The 16-byte items of one (level, head) are spread over
// kParamSlices CTAs: its transposed parameter reads are strided, so the
// kernel needs many loads in flight rather than few CTAs.
// ---------------------------------------------------------------------------

constexpr int kParamSlices = 16;

__global__ void __launch_bounds__(256) tc_params_kernel(FwdParams p, TcLayout lay, char* ws) {
  if (gate_closed(p)) return;
  const int l = blockIdx.x + 1, h = blockIdx.y;
  const int i0 = blockIdx.z * blockDim.x + threadIdx.x, di = gridDim.z * blockDim.x;
  const int64_t pidx = int64_t(l - 1) * p.H + h;
  char* base = ws + lay.ptc_off + pidx * PT_SIZE;
  bf16* qb = reinterpret_cast<bf16*>(base + PT_QB);
  bf16* w2a = reinterpret_cast<bf16*>(base + PT_W2A);
  bf16* w2b = reinterpret_cast<bf16*>(base + PT_W2B);
  // (The merge arm ignores n_queries; never read past the bank's rows.)
  const int nq = min(p.nq[l - 1], p.n_max), mp = pad_pairs(nq);
  const int dt = p.param_dtype;
  // Query bank rows past n_queries are ignored (probe.py:97): zero rows.
  for (int it = i0; it < mp * 16; it += di) {
    const int r = it >> 4, k0 = (it & 15) * 8;
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      x[u] = r < nq ? load_elem(p.raw_params[0], (pidx * p.n_max + r) * TK + k0 + u, dt) : 0.f;
    *reinterpret_cast<uint4*>(qb + kmajor_off(r, k0, TK)) = pack8(x);
  }
  // B operands over the reduction index v: row n < 128 of W2A is W_k[n][:]
  // (u = values . W_k^T, probe.py:99), row 128 + k is W_b[:][k]; W2B holds
  // W_w[:][n] and W_g[:][k] (probe.py:60-62).
  for (int it = i0; it < 256 * 16; it += di) {
    const int n = it >> 4, v0 = (it & 15) * 8;
    float xa[8], xb[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int v = v0 + u;
      if (n < 128) {
        xa[u] = load_elem(p.raw_params[1], (pidx * TK + n) * TV + v, dt);
        xb[u] = load_elem(p.raw_params[3], (pidx * TV + v) * TV + n, dt);
      } else {
        xa[u] = load_elem(p.raw_params[2], (pidx * TV + v) * TK + (n - 128), dt);
        xb[u] = load_elem(p.raw_params[4], (pidx * TV + v) * TK + (n - 128), dt);
      }
    }
    *reinterpret_cast<uint4*>(w2a + kmajor_off(n, v0, TV)) = pack8(xa);
    *reinterpret_cast<uint4*>(w2b + kmajor_off(n, v0, TV)) = pack8(xb);
  }
}

// ---------------------------------------------------------------------------
// prep_tc: grid (NT, H, B), 256 threads, two CTAs per SM.
// ---------------------------------------------------------------------------

constexpr int kPrepThreads = 256;
constexpr int kPrepCols = 256;  // TMEM columns

// Shared-memory plan (bytes). Phase 1 holds the operands of the A_qk / A_kk
// MMAs and the B operand of the [U | W] MMA; phase 2 reuses the first region
// for the inverse.
constexpr int P_KG = 0;                  // K^(J), J = 0..3: 20 groups of 8 rows x 128, K-major
constexpr int P_QB = 40960;              // 4 x [32 x 128] K-major: 16 query rows, 16 b*k rows
constexpr int P_AF = 0;                  // fp32 [64][65] strictly lower A_kk
constexpr int XS = 68;                   // row stride (floats) of the inverse: float4 rows
constexpr int P_XF = P_AF + 16640;       // fp32 [64][XS] (I + A_kk)^-1
constexpr int P_XB = P_XF + 64 * XS * 4; // bf16 [64 x 64] K-major: staged A_qk, then the inverse
constexpr int P_TT = P_XB + 8192;        // fp32 block products of the inverse (<= [32][36])
constexpr int P_R = 73728;               // bf16 [64 x 256] MN-major [w*v | k*b*e^G]
constexpr int kPrepSmem = P_R + 32768;   // 106496

// Row-group offset (in elements) of K^(J) inside the P_KG region: K^(J)
// keeps rows 0 .. 16J+15 (later rows are never needed), so the four tiles
// pack into 2 + 4 + 6 + 8 groups. The J-th MMA still reads 64 rows; rows
// past 16J+15 belong to the next tile and land in masked entries.
__device__ __forceinline__ int kgroup_elems(int J) {
  return (J == 0 ? 0 : J == 1 ? 2 : J == 2 ? 6 : 12) * 1024;
}


__global__ void __launch_bounds__(kPrepThreads, 2)
prep_tc_kernel(FwdParams p, TcLayout lay, char* ws, const __grid_constant__ PrepMaps maps) {
  if (gate_closed(p)) return;
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  __shared__ float mixs[1][kC];             // mix_0 * scale per row
  __shared__ __align__(16) float rho[5][TK];  // G[16J + 7] for J = 0..3, then G[63]
  // [0]: e^(G_63 - rho_3); [J]: e^(rho_J - rho_(J-1)), J = 1..3; [4 + I]: e^(rho_I)
  __shared__ __align__(16) float rat[8][TK];
  float* Tt = reinterpret_cast<float*>(sm + P_TT);
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = n * kC;
  char* rec = ws + lay.chunks_off + ((int64_t(b) * p.H + h) * p.NT + n) * lay.rec.size;

  // One L2 prefetch per input tensor of this chunk's rows: the column
  // chunks that the loads below fetch one at a time then come from L2.
  if (tid < 6 && (maps.valid >> tid & 1u)) tc::tma_prefetch_l2_3d(&maps.m[tid], 0, b * p.T + t0, h);
  // g is the first input the kernel waits on. Blocks start in index order as
  // slots free up, so the block two waves ahead (this index + two CTAs per
  // SM) takes this slot about one CTA lifetime from now: its g rows are
  // pulled into L2 as well, so that its first wait sees L2 latency.
  if (tid == 32 && (maps.valid & 2u)) {
    uint32_t nsm;
    asm("mov.u32 %0, %%nsmid;" : "=r"(nsm));
    const int64_t lin2 = n + int64_t(p.NT) * (h + int64_t(p.H) * b) + 2 * int64_t(nsm);
    const int64_t b2 = lin2 / (int64_t(p.NT) * p.H);
    if (b2 < p.B)
      tc::tma_prefetch_l2_3d(&maps.m[1], 0, int(b2 * p.T + (lin2 % p.NT) * kC), int(lin2 / p.NT % p.H));
  }
  // Phase A mapping: warp w owns rows 8w .. 8w+7; lane = 8 * c4 + r8 holds
  // row 8w + r8 and the 8-column chunks c4, c4 + 4, c4 + 8, c4 + 12. A warp
  // load then touches 8 rows x 64 contiguous bytes, and the 16-byte shared
  // stores of 8 consecutive lanes fill one contiguous 128-byte core matrix.
  const int c4 = lane >> 3, r8 = lane & 7;
  const int r = 8 * warp + r8, t = t0 + r;
  const bool valid = t < p.T;
  bf16* Qg = reinterpret_cast<bf16*>(rec + lay.rec.Q);
  bf16* Ktg = reinterpret_cast<bf16*>(rec + lay.rec.Kt);

  // Raw 16-byte chunks of q_0, k, b, v, w for one column chunk; each
  // chunk's loads are issued one chunk ahead of their use.
  auto fetch = [&](int ci, uint4* raw) {
    const int d0 = 8 * (c4 + 4 * ci);
    if (valid) {
      raw[0] = raw8_at(p.q.p, p.q.dt, p.q.off(b, t, h, 0, d0), p.q.sd);
      raw[1] = raw8_at(p.k.p, p.k.dt, p.k.off(b, t, h, d0), p.k.sd);
      raw[2] = raw8_at(p.b.p, p.b.dt, p.b.off(b, t, h, d0), p.b.sd);
      raw[3] = raw8_at(p.v.p, p.v.dt, p.v.off(b, t, h, d0), p.v.sd);
      raw[4] = raw8_at(p.w.p, p.w.dt, p.w.off(b, t, h, d0), p.w.sd);
    } else {
#pragma unroll
      for (int i = 0; i < 5; ++i) raw[i] = make_uint4(0, 0, 0, 0);
    }
  };
  uint4 cur[5], nxt[5];

  // A1. G = cumsum of g along the chunk (naive.py:329): a scan over the 8
  //     rows of each warp, then the carries of the row blocks above.
  //     Every global load of this phase (g, the first column chunk of the
  //     other inputs, mix_0) is issued as raw bits before anything waits on
  //     one, and TMEM and the mbarrier are set up while they are in flight.
  float G[4][8];
  uint4 graw[4];
  const bool g16 = p.g.dt != NGDN2_F32;
#pragma unroll
  for (int ci = 0; ci < 4; ++ci) {
    const int d0 = 8 * (c4 + 4 * ci);
    if (g16) {
      graw[ci] = valid ? raw8_at(p.g.p, p.g.dt, p.g.off(b, t, h, d0), p.g.sd) : make_uint4(0, 0, 0, 0);
    } else if (valid) {
      load8(p.g, b, t, h, d0, G[ci]);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) G[ci][u] = 0.f;
    }
  }
  fetch(0, cur);
  uint32_t mix_bits = 0;
  if (tid < kC && t0 + tid < p.T) {
    const int64_t o = p.mix.off(b, t0 + tid, h, 0);
    mix_bits = p.mix.dt == NGDN2_F32 ? __float_as_uint(reinterpret_cast<const float*>(p.mix.p)[o])
                                     : uint32_t(reinterpret_cast<const uint16_t*>(p.mix.p)[o]);
  }
  if (warp == 0) tmem_alloc(&tbase, kPrepCols);
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (g16) {
#pragma unroll
    for (int ci = 0; ci < 4; ++ci) unpack8(graw[ci], p.g.dt, G[ci]);
  }
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) {
#pragma unroll
    for (int ci = 0; ci < 4; ++ci)
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float y = __shfl_up_sync(0xffffffffu, G[ci][u], off, 8);
        if (r8 >= off) G[ci][u] += y;
      }
  }
  float* carry = reinterpret_cast<float*>(sm + P_R);  // [8][128], before R is built
  if (r8 == 7) {
#pragma unroll
    for (int ci = 0; ci < 4; ++ci)
#pragma unroll
      for (int u = 0; u < 8; ++u) carry[warp * TK + 8 * (c4 + 4 * ci) + u] = G[ci][u];
  }
  if (tid < kC) {
    const float m0 = p.mix.dt == NGDN2_F32   ? __uint_as_float(mix_bits)
                     : p.mix.dt == NGDN2_BF16 ? __uint_as_float(mix_bits << 16)
                                              : __half2float(__ushort_as_half(uint16_t(mix_bits)));
    mixs[0][tid] = m0 * p.scale;
  }
  __syncthreads();
  if (tid < TK) {
    float run = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float c = carry[w * TK + tid];
      carry[w * TK + tid] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int ci = 0; ci < 4; ++ci)
#pragma unroll
    for (int u = 0; u < 8; ++u) G[ci][u] += carry[warp * TK + 8 * (c4 + 4 * ci) + u];
  // Reference points rho_I = G[16I + 7] (row 7 of even warps) and G[63].
  if (r8 == 7 && ((warp & 1) == 0 || warp == 7)) {
    const int slot = warp == 7 ? 4 : warp >> 1;
#pragma unroll
    for (int ci = 0; ci < 4; ++ci)
#pragma unroll
      for (int u = 0; u < 8; ++u) rho[slot][8 * (c4 + 4 * ci) + u] = G[ci][u];
  }
  __syncthreads();
  if (tid < TK) {
    rat[0][tid] = __expf(rho[4][tid] - rho[3][tid]);
#pragma unroll
    for (int J = 1; J < 4; ++J) rat[J][tid] = __expf(rho[J][tid] - rho[J - 1][tid]);
#pragma unroll
    for (int I2 = 0; I2 < 4; ++I2) rat[4 + I2][tid] = __expf(rho[I2][tid]);
  }
  __syncthreads();
  const uint32_t tb = tbase;

  // A2. Operands. Row block I of queries uses rho_I so that
  //       Q_I[i] . K^(I)[j] = q_i . k_j e^(G_i - G_j)
  //     with Q_I[i] = q_i e^(G_i - rho_I), K^(J)[j] = k_j e^(rho_J - G_j):
  //     every factor is bounded by the decay over 8 tokens
  //     (naive.py:335-344, 377-378). The record gets the read queries, K_tail
  //     and e^(G_last); R = [w * v | k * b * e^G] is the B operand of the
  //     [U | W] MMA (naive.py:346-352).
  bf16* KG = reinterpret_cast<bf16*>(sm + P_KG);
  bf16* QB = reinterpret_cast<bf16*>(sm + P_QB);
  bf16* Rs = reinterpret_cast<bf16*>(sm + P_R);
  const int I = r >> 4;
#pragma unroll
  for (int ci = 0; ci < 4; ++ci) {
    if (ci < 3) fetch(ci + 1, nxt);
    const int d0 = 8 * (c4 + 4 * ci);
    float qq[8], kk[8], bb[8], o1[8], o2[8], rr[8];
    unpack8(cur[0], p.q.dt, qq);
    unpack8(cur[1], p.k.dt, kk);
    unpack8(cur[2], p.b.dt, bb);
    const float* g = G[ci];
    {
      const float4* rp = reinterpret_cast<const float4*>(&rho[I][d0]);
      const float4 a0 = rp[0], a1 = rp[1];
      rr[0] = a0.x; rr[1] = a0.y; rr[2] = a0.z; rr[3] = a0.w;
      rr[4] = a1.x; rr[5] = a1.y; rr[6] = a1.z; rr[7] = a1.w;
    }
    // Q_I, BK_I rows (MMA1 B operand)
    float eq[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      eq[u] = __expf(g[u] - rr[u]);
      o1[u] = qq[u] * eq[u];
      o2[u] = bb[u] * kk[u] * eq[u];
    }
    bf16* tile = QB + I * (32 * 128);
    *reinterpret_cast<uint4*>(tile + kmajor_off(r & 15, d0, 128)) = pack8(o1);
    *reinterpret_cast<uint4*>(tile + kmajor_off(16 + (r & 15), d0, 128)) = pack8(o2);
    // K^(J) rows for every J >= I (MMA1 A operands): e^(rho_J - G) by a
    // chain of per-channel factors e^(rho_J - rho_(J-1)) <= 1, ending in
    // e^(rho_3 - G), which also gives K_tail below.
    float ech[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) ech[u] = __expf(rr[u] - g[u]);
    for (int J = I; J < 4; ++J) {
      if (J > I) {
        const float4* rp = reinterpret_cast<const float4*>(&rat[J][d0]);
        const float4 a0 = rp[0], a1 = rp[1];
        const float rj[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int u = 0; u < 8; ++u) ech[u] *= rj[u];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) o1[u] = kk[u] * ech[u];
      *reinterpret_cast<uint4*>(KG + kgroup_elems(J) + kmajor_off(r, d0, 128)) = pack8(o1);
    }
    // e^G = e^(G - rho_I) e^(rho_I): level-0 read query and the k*b*e^G half
    // of R; w*v half of R
    {
      float vv[8], ww[8];
      unpack8(cur[3], p.v.dt, vv);
      unpack8(cur[4], p.w.dt, ww);
      const float m0 = mixs[0][r];
      const float4* ep = reinterpret_cast<const float4*>(&rat[4 + I][d0]);
      const float4 e0 = ep[0], e1 = ep[1];
      const float er[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float e = eq[u] * er[u];
        o1[u] = m0 * qq[u] * e;
        o2[u] = kk[u] * bb[u] * e;
        ww[u] *= vv[u];
      }
      *reinterpret_cast<uint4*>(Qg + kmajor_off(r, d0, 128)) = pack8(o1);
      *reinterpret_cast<uint4*>(Rs + mnmajor_off(r, 128 + d0, 64)) = pack8(o2);
      *reinterpret_cast<uint4*>(Rs + mnmajor_off(r, d0, 64)) = pack8(ww);
    }
    // K_tail = k e^(G_last - G) = k e^(rho_3 - G) e^(G_last - rho_3), the
    // MN-major A operand of K_tail^T . v_new
    {
      const float4* rp = reinterpret_cast<const float4*>(&rat[0][d0]);
      const float4 a0 = rp[0], a1 = rp[1];
      const float rj[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int u = 0; u < 8; ++u) o1[u] = kk[u] * ech[u] * rj[u];
    }
    *reinterpret_cast<uint4*>(Ktg + mnmajor_off(r, d0, 64)) = pack8(o1);
    if (ci < 3) {
#pragma unroll
      for (int i = 0; i < 5; ++i) cur[i] = nxt[i];
    }
  }
  if (tid < TK) reinterpret_cast<float*>(rec + lay.rec.eg)[tid] = __expf(rho[4][tid]);
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();

  // B. MMA1: D[j, 32J + c] = K^(J)[j] . [Q_J ; BK_J][c], N=32, K=128. Issued
  //    as M=128 (same tensor-pipe time as M=64): A rows 64..127 read the
  //    shared memory after the tile and land in TMEM lanes 64..127, which
  //    nothing reads, while rows 0..63 fill lanes 0..63 densely, so the
  //    read-outs below move no idle lanes.
  if (tid == 0) {
    const uint32_t id = idesc_f16(128, 32, true, false, false);
    for (int J = 0; J < 4; ++J)
      mma_tile(tb + 32 * J, smem_u32(KG + kgroup_elems(J)), smem_u32(QB + J * 32 * 128), 128, id,
               false);
    mma_commit(&bar);
  }
  __syncwarp();
  if (!mbar_wait(&bar, 0)) set_status(p, NGDN2_STATUS_WAIT_TIMEOUT);
  fence_after_sync();

  // C. Masks: A_kk to shared fp32, mix0 * scale * A_qk staged as a K-major
  //    bf16 tile and copied to the record with 16-byte stores.
  float* Af = reinterpret_cast<float*>(sm + P_AF);
  bf16* Xb = reinterpret_cast<bf16*>(sm + P_XB);
  if ((warp & 3) < 2) {
    // Warps 0, 1, 4, 5 own TMEM lanes 0..63 (row j = 32q + lane); all 64
    // columns of a warp in one TMEM round trip.
    const int q = warp & 3, ch = warp >> 2, j = 32 * q + lane;
    uint32_t raw[64];
    tmem_ld32_nowait(taddr(tb, 32 * q, 64 * ch), raw);
    tmem_ld32_nowait(taddr(tb, 32 * q, 64 * ch + 32), raw + 32);
    tmem_wait_ld();
    tmem_regs_after_wait32(raw);
    tmem_regs_after_wait32(raw + 32);
#pragma unroll
    for (int c16 = 0; c16 < 4; ++c16) {
      const float* v = reinterpret_cast<const float*>(raw + 16 * c16);
      const int J = 2 * ch + (c16 >> 1);
      if (c16 & 1) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int i = 16 * J + c;
          Af[i * 65 + j] = (j < i) ? v[c] : 0.f;
        }
      } else {
        // Lanes j and j ^ 1 pair up: the even lane writes rows 16J + 2m and
        // the odd lane rows 16J + 2m + 1, each as one 4-byte (j, j + 1)
        // bf16 pair, so a store instruction covers two rows of each core
        // matrix it touches instead of one 2-byte column element.
        const bool odd = lane & 1;
        const int j0 = j & ~1;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int ie = 16 * J + 2 * m, io = ie + 1;
          const float ae = j <= ie ? v[2 * m] * mixs[0][ie] : 0.f;
          const float ao = j <= io ? v[2 * m + 1] * mixs[0][io] : 0.f;
          // Each lane keeps its own row's value and receives the partner's.
          const float other = __shfl_xor_sync(0xffffffffu, odd ? ae : ao, 1);
          const int i = odd ? io : ie;
          const __nv_bfloat162 pr = odd ? __floats2bfloat162_rn(other, ao)
                                        : __floats2bfloat162_rn(ae, other);
          *reinterpret_cast<__nv_bfloat162*>(Xb + kmajor_off(i, j0, 64)) = pr;
        }
      }
    }
  }
  __syncthreads();
  {
    const uint4* src = reinterpret_cast<const uint4*>(Xb);
    uint4* dst = reinterpret_cast<uint4*>(rec + lay.rec.A);
    for (int e = tid; e < TILE_A / 16; e += kPrepThreads) dst[e] = src[e];
  }

  // D. (I + A_kk)^-1 in fp32 by 2x2 block recursion (for unit lower
  //    triangular [[L11, 0], [L21, L22]], X21 = -X22 L21 X11): 16x16
  //    diagonal blocks by forward substitution, then the 16-row off-diagonal
  //    blocks of both 32x32 halves, then the 32-row block of the whole. Both
  //    32x32 diagonal halves of Xf are written in full (zeros above the
  //    diagonal); its upper-right 32x32 block is never read.
  float* Xf = reinterpret_cast<float*>(sm + P_XF);
  if (tid < 64) {
    const int o = 16 * (tid >> 4), c = tid & 15;
    float x[16];
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) {
      float s = (rr == c) ? 1.f : 0.f;
#pragma unroll
      for (int u = 0; u < rr; ++u) s = fmaf(-Af[(o + rr) * 65 + o + u], x[u], s);
      x[rr] = s;
    }
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) Xf[(o + rr) * XS + o + c] = x[rr];
  } else {
    // The upper off-diagonal 16x16 block of each 32x32 half: read, as the
    // zeros of a lower-triangular matrix, by the unrolled 64-level products.
    for (int e = tid - 64; e < 2 * 256; e += kPrepThreads - 64) {
      const int half = e >> 8, rr = (e >> 4) & 15, c = e & 15;
      Xf[(32 * half + rr) * XS + 32 * half + 16 + c] = 0.f;
    }
  }
  __syncthreads();
  auto fma4 = [](float a, const float4& x, float4& acc) {
    acc.x = fmaf(a, x.x, acc.x);
    acc.y = fmaf(a, x.y, acc.y);
    acc.z = fmaf(a, x.z, acc.z);
    acc.w = fmaf(a, x.w, acc.w);
  };
  // 32-level: in half h (rows/cols 32h..), T = L21 X11 then X21 = -X22 T,
  // 16x16 each; a thread owns 4 columns of one row (128 threads).
  {
    const int hh = tid >> 6, rr = (tid >> 2) & 15, cq = (tid & 3) * 4;
    const int r0 = 32 * hh + 16, k0 = 32 * hh;
    if (tid < 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 16; ++m)
        fma4(Af[(r0 + rr) * 65 + k0 + m], *reinterpret_cast<const float4*>(&Xf[(k0 + m) * XS + k0 + cq]), acc);
      *reinterpret_cast<float4*>(&Tt[hh * 256 + rr * 16 + cq]) = acc;
    }
    __syncthreads();
    if (tid < 128) {
      // X22's strict upper triangle holds exact zeros: a fixed trip count
      // adds only zeros and lets every load issue up front.
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 16; ++m)
        fma4(Xf[(r0 + rr) * XS + r0 + m], *reinterpret_cast<const float4*>(&Tt[hh * 256 + m * 16 + cq]), acc);
      *reinterpret_cast<float4*>(&Xf[(r0 + rr) * XS + k0 + cq]) = make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
    }
    __syncthreads();
  }
  // 64-level: T = A[32.., 0..31] X_A, then X[32.., 0..31] = -X_B T; 32x32
  // each. X_A and X_B are fully written lower triangles with exact zeros
  // above the diagonal, so full-length products add only zeros. A thread
  // owns a 4 x 4 block (rows r4 .. r4 + 3, columns cq .. cq + 3) over one
  // quarter kq of the reduction index, and the quarters are summed by two
  // butterfly rounds that leave lane kq with row r4 + kq. Each quarter-warp
  // shares kq, so its 16-byte loads cover one contiguous 128-byte row
  // segment; the 4 x 4 blocking reads each loaded value four times, which
  // matters because the shared-memory pipe is this kernel's busiest unit.
  {
    constexpr int TS = 36;  // row stride (floats) of T
    const int cq = (tid & 7) * 4, kq = (tid >> 3) & 3, r4 = (tid >> 5) * 4;
    const int b0 = kq & 1, b1 = kq >> 1;
    // Sum of the four quarters' partial rows; returns row r4 + kq.
    auto reduce = [&](float4* acc) {
      float4 kept[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float4 mine = b0 ? acc[2 * j + 1] : acc[2 * j];
        const float4 send = b0 ? acc[2 * j] : acc[2 * j + 1];
        kept[j] = make_float4(mine.x + __shfl_xor_sync(0xffffffffu, send.x, 8),
                              mine.y + __shfl_xor_sync(0xffffffffu, send.y, 8),
                              mine.z + __shfl_xor_sync(0xffffffffu, send.z, 8),
                              mine.w + __shfl_xor_sync(0xffffffffu, send.w, 8));
      }
      const float4 mine = b1 ? kept[1] : kept[0];
      const float4 send = b1 ? kept[0] : kept[1];
      return make_float4(mine.x + __shfl_xor_sync(0xffffffffu, send.x, 16),
                         mine.y + __shfl_xor_sync(0xffffffffu, send.y, 16),
                         mine.z + __shfl_xor_sync(0xffffffffu, send.z, 16),
                         mine.w + __shfl_xor_sync(0xffffffffu, send.w, 16));
    };
    float4 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int k = 8 * kq + kk;
      const float4 x = *reinterpret_cast<const float4*>(&Xf[k * XS + cq]);
#pragma unroll
      for (int i = 0; i < 4; ++i) fma4(Af[(32 + r4 + i) * 65 + k], x, acc[i]);
    }
    *reinterpret_cast<float4*>(&Tt[(r4 + kq) * TS + cq]) = reduce(acc);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int mm = 0; mm < 8; ++mm) {
      const int m = 8 * kq + mm;
      const float4 x = *reinterpret_cast<const float4*>(&Tt[m * TS + cq]);
#pragma unroll
      for (int i = 0; i < 4; ++i) fma4(Xf[(32 + r4 + i) * XS + 32 + m], x, acc[i]);
    }
    const float4 x21 = reduce(acc);
    *reinterpret_cast<float4*>(&Xf[(32 + r4 + kq) * XS + cq]) = make_float4(-x21.x, -x21.y, -x21.z, -x21.w);
    __syncthreads();
  }
  // The inverse as a bf16 K-major tile: eight consecutive lanes take the
  // eight rows of one core matrix, so each quarter-warp reads 16 bytes from
  // eight rows in distinct banks (row stride 68 floats) and writes one
  // contiguous 128-byte core matrix.
  for (int it = tid; it < kC * 8; it += kPrepThreads) {
    const int i = 8 * (it >> 6) + (it & 7), j0 = ((it >> 3) & 7) * 8;
    const float4 a0 = *reinterpret_cast<const float4*>(&Xf[i * XS + j0]);
    const float4 a1 = *reinterpret_cast<const float4*>(&Xf[i * XS + j0 + 4]);
    const float raw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = (j0 + u <= i) ? raw[u] : 0.f;
    *reinterpret_cast<uint4*>(Xb + kmajor_off(i, j0, 64)) = pack8(x);
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();

  // E. MMA2: [U | W] = X . R, M=64, N=256, K=64 (naive.py:346-351).
  if (tid == 0) {
    // M=128 for the same reason as MMA1 (A rows 64..127 are the shared
    // memory after the inverse tile; their TMEM lanes are never read).
    mma_tile(tb, smem_u32(Xb), smem_u32(Rs), 64, idesc_f16(128, 256, true, false, true), false);
    mma_commit(&bar);
  }
  __syncwarp();
  if (!mbar_wait(&bar, 1)) set_status(p, NGDN2_STATUS_WAIT_TIMEOUT);
  fence_after_sync();

  // F. U (row-major) and W (K-major A operand) to the record.
  {
    bf16* Ug = reinterpret_cast<bf16*>(rec + lay.rec.U);
    bf16* Wg = reinterpret_cast<bf16*>(rec + lay.rec.W);
    // Warps 0, 1, 4, 5 own TMEM lanes 0..63 (row i = 32q + lane); 64
    // columns per TMEM round trip.
    const int q = warp & 3, ch = warp >> 2, i = 32 * q + lane;
    for (int c64 = 0; c64 < 2 && q < 2; ++c64) {
      uint32_t raw[64];
      tmem_ld32_nowait(taddr(tb, 32 * q, 128 * ch + 64 * c64), raw);
      tmem_ld32_nowait(taddr(tb, 32 * q, 128 * ch + 64 * c64 + 32), raw + 32);
      tmem_wait_ld();
      tmem_regs_after_wait32(raw);
      tmem_regs_after_wait32(raw + 32);
#pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) {
        const float* v = reinterpret_cast<const float*>(raw + 16 * c16);
        const int d0 = 64 * c64 + 16 * c16;
        if (ch == 0) {
          // 8-column pieces, rows consecutive within a piece: the scan's
          // lane-per-row loads of one piece are then contiguous.
          *reinterpret_cast<uint4*>(Ug + (d0 / 8) * (kC * 8) + i * 8) = pack8(v);
          *reinterpret_cast<uint4*>(Ug + (d0 / 8 + 1) * (kC * 8) + i * 8) = pack8(v + 8);
        } else {
          *reinterpret_cast<uint4*>(Wg + kmajor_off(i, d0, 128)) = pack8(v);
          *reinterpret_cast<uint4*>(Wg + kmajor_off(i, d0 + 8, 128)) = pack8(v + 8);
        }
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, kPrepCols);
}

}  // namespace
}  // namespace ngdn2

namespace ngdn2 {
namespace {

// ---------------------------------------------------------------------------
// scan_tc: grid (H, B), 256 threads, one CTA per SM.
// ---------------------------------------------------------------------------

constexpr int kScanThreads = 512;
constexpr int kScanCols = 512;          // TMEM: S0 0..127, chunk accumulators 128..255, promotion 128..511
constexpr int TILE_S = TK * TV * 2;     // bf16 state copy
// Promotion scratch (the record region and what follows it): a 64 KB slot
// for weights / gate partials / keys, and a 32 KB slot for the pairs.
constexpr int kPromoScratch = 98304;

// Shared memory of the scan: L bf16 state copies, then the record, the
// upper levels' query tiles (L - 1), the v_new tile and the CUDA-core
// promotion's GEMM staging; promotions reuse everything after the states.
__host__ __device__ inline int64_t scan_tc_smem(int L, const TcRecord& rec) {
  const int64_t tail = rec.load_bytes + int64_t(L - 1) * TILE_QK + TILE_QK;
  return int64_t(L) * TILE_S + (tail > kPromoScratch ? tail : kPromoScratch) + 1024;
}

// fp32 master [K][V] -> bf16 MN-major B operand copy [Kd = K][N = V].
__device__ __forceinline__ void refresh_copy(bf16* dst, const float* src) {
  for (int it = threadIdx.x; it < TK * (TV / 8); it += kScanThreads) {
    const int k = it / (TV / 8), v0 = (it % (TV / 8)) * 8;
    const float4 a = *reinterpret_cast<const float4*>(src + k * TV + v0);
    const float4 c = *reinterpret_cast<const float4*>(src + k * TV + v0 + 4);
    const float x[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    *reinterpret_cast<uint4*>(dst + mnmajor_off(k, v0, TK)) = pack8(x);
  }
}

// First operands of a learned promotion of level l: the query bank (K-major,
// padded to 64 or 128 rows) and [W_w | W_g], into the promotion scratch X.
// Issued by one thread; completion arrives on ``bar_ld``.
__device__ __forceinline__ void promote_tc_first_loads(const FwdParams& p, const TcLayout& lay,
                                                       const char* ws, int h, int l, uint8_t* X,
                                                       uint64_t* bar_ld) {
  const int mp = pad_pairs(p.nq[l - 1]);
  const char* pt = ws + lay.ptc_off + (int64_t(l - 1) * p.H + h) * PT_SIZE;
  mbar_arrive_expect_tx(bar_ld, uint32_t(mp * 256 + 65536));
  bulk_g2s(X + 65536, pt + PT_QB, uint32_t(mp * 256), bar_ld);
  bulk_g2s(X, pt + PT_W2B, 65536u, bar_ld);
}

// Gate partials of a 64-pair promotion, fp16, at this offset of the scratch
// (after the 64-row bank): [64 pairs][64 column pairs] 32-bit words with the
// column-pair index XOR-swizzled by row.
constexpr int kGpartOff = 65536 + 16384;

// Learned promotion of level l - 1 into level l on the tensor cores
// (probe.py:69-102 with _gates :34-66, then update_fwd.py:120-123):
//   P1  V'  = Q_bank . S_{l-1}
//   P2b [w_logit | g_logit] = V' . [W_w | W_g]   -> v*w, g = mean(-softplus(. - 4))
//   P2a [u | b_logit]       = V' . [W_k^T | W_b] -> keys = u / |u|, b = sigmoid(. - 4)
//   P3  (keys * b * e^g) . S_l                    -> vn = v*w - that
//   P4  S_l <- e^g S_l + keys^T . vn
// fp32 accumulators in TMEM columns 128..511 (the chunk accumulators are
// free between chunks); bf16 operands in ``X`` (the record buffer, reloaded
// after the promotion). The fp32 master of S_l is in global memory,
// lane-major (lm_off) so that lane-per-key TMEM traffic reads and writes it
// as float4 runs of 512 contiguous bytes a warp. With 64 pairs the gate products go to the two
// half-lane groups of the same TMEM columns so every lane has work.
// 512 threads: warp w reads TMEM lane quarter (w & 3), columns 32 * (w >> 2).
__device__ void promote_tc(const FwdParams& p, const TcLayout& lay, const char* ws, int h, int l,
                           uint32_t tb, bf16* Sbf, uint8_t* X, float* Mt, uint64_t* bar_ld,
                           uint64_t* bar_mma, uint32_t& ph_ld, uint32_t& ph_mma, float* egp,
                           float* red, int* abort_flag, bool loaded) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, c0 = 32 * (warp >> 2);
  const int nq = p.nq[l - 1], mp = pad_pairs(nq);
  const char* pt = ws + lay.ptc_off + (int64_t(l - 1) * p.H + h) * PT_SIZE;
  bf16* XW = reinterpret_cast<bf16*>(X);
  bf16* XQ = reinterpret_cast<bf16*>(X + 65536);
  float* Sl = Mt + int64_t(l - 1) * TK * TV;  // fp32 master of level l, lane-major (lm_off)
  const uint32_t tV = tb + 128, tG = tb + 256, tS = tb + 384;
  const int row = (mp == 128) ? 32 * quarter + lane : (lane < 16 ? 16 * quarter + lane : -1);
  const bool split = mp == 64;
  const uint32_t id_read = idesc_f16(mp, 128, true, false, true);
  const uint32_t id_gate = idesc_f16(mp, 256, true, false, false);
  const uint32_t id_half = idesc_f16(64, 128, true, false, false);
  const uint32_t id_upd = idesc_f16(128, 128, true, true, true);

  // Query bank and [W_w | W_g] in (issued by the caller when ``loaded``).
  if (tid == 0 && !loaded) promote_tc_first_loads(p, lay, ws, h, l, X, bar_ld);
  if (!mbar_wait(bar_ld, ph_ld)) *abort_flag = 1;
  ph_ld ^= 1;
  // P1
  if (tid == 0) {
    fence_after_sync();
    mma_tile(tV, smem_u32(XQ), smem_u32(Sbf + (l - 1) * TK * TV), TK, id_read, false);
    mma_commit(bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // V' -> bf16 A operand (over the bank, which P1 has consumed).
  {
    float x[32];
    tmem_ld32(taddr(tV, 32 * quarter, c0), x);
    if (row >= 0) {
#pragma unroll
      for (int c = 0; c < 32; c += 8)
        *reinterpret_cast<uint4*>(XQ + kmajor_off(row, c0 + c, TV)) = pack8(x + c);
    }
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  // P2b
  if (tid == 0) {
    fence_after_sync();
    if (split) {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_half, false);
      mma_tile(tG + (16u << 16), smem_u32(XQ), smem_u32(XW + 128 * 128), TV, id_half, false);
    } else {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_gate, false);
    }
    mma_commit(bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // With 64 pairs [W_w | W_g] is spent now: [W_k^T | W_b] streams in while
  // the gates are formed (their partials live past the bank).
  if (split && tid == 0) {
    mbar_arrive_expect_tx(bar_ld, 65536u);
    bulk_g2s(XW, pt + PT_W2A, 65536u, bar_ld);
  }
  // v * w back into TMEM; -softplus(g_logit - 4) per pair into shared memory
  // (columns XOR-swizzled by row so both the row writes and the column sums
  // are free of bank conflicts).
  float* gpart = reinterpret_cast<float*>(X);
  uint32_t* gpart16 = reinterpret_cast<uint32_t*>(X + kGpartOff);
  {
    float a[32], vp[32];
    if (split) {
      // Lane l < 16 holds the w logits of pair 16q + l, lane l + 16 its g
      // logits. The two lanes swap halves so that each forms 16 of both
      // gates (no divergence): the low lane takes columns 0..15, the high
      // lane 16..31; the high lane hands its w gates back for v * w.
      tmem_ld32(taddr(tG, 32 * quarter, c0), a);
      const bool hi = lane >= 16;
      const int gr = 16 * quarter + (lane & 15), cb = c0 + (hi ? 16 : 0);
      float sw[16];
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        float gg[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float mine_w = hi ? 0.f : a[j + e], mine_g = hi ? a[16 + j + e] : 0.f;
          const float got = __shfl_xor_sync(0xffffffffu, hi ? a[j + e] : a[16 + j + e], 16);
          const float wl = hi ? got : mine_w, gl = hi ? mine_g : got;
          sw[j + e] = sigmoid_tanh(wl + kWLogitInit);
          gg[e] = -softplus_fast(gl + kGLogitInit);
        }
        const __half2 g2 = __floats2half2_rn(gg[0], gg[1]);
        gpart16[gr * 64 + (((cb + j) >> 1) ^ (gr & 31))] = *reinterpret_cast<const uint32_t*>(&g2);
      }
      tmem_ld32(taddr(tV, 32 * quarter, c0), vp);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float back = __shfl_xor_sync(0xffffffffu, sw[j], 16);
        vp[j] *= sw[j];
        vp[16 + j] *= back;
      }
      tmem_st32(taddr(tV, 32 * quarter, c0), vp);  // lanes 16..31 of tV are unused
    } else {
      tmem_ld32(taddr(tV, 32 * quarter, c0), vp);
      tmem_ld32(taddr(tG, 32 * quarter, c0), a);
#pragma unroll
      for (int u = 0; u < 32; ++u) vp[u] *= sigmoid_tanh(a[u] + kWLogitInit);
      tmem_st32(taddr(tV, 32 * quarter, c0), vp);
      tmem_ld32(taddr(tG, 32 * quarter, 128 + c0), a);
#pragma unroll
      for (int u = 0; u < 32; ++u)
        gpart[row * 128 + ((c0 + u) ^ (row & 31))] = -softplus_fast(a[u] + kGLogitInit);
    }
  }
  tmem_wait_st();
  __syncthreads();
  {
    // g = mean over the real pairs, four threads per column.
    const int k = tid & 127, qq = tid >> 7, r0 = qq * (nq >> 2), r1 = r0 + (nq >> 2);
    float s = 0.f;
    if (split) {
      const __half* g16 = reinterpret_cast<const __half*>(gpart16);
      for (int r = r0; r < r1; ++r)
        s += __half2float(g16[2 * (r * 64 + ((k >> 1) ^ (r & 31))) + (k & 1)]);
    } else {
      for (int r = r0; r < r1; ++r) s += gpart[r * 128 + (k ^ (r & 31))];
    }
    red[qq * 128 + k] = s;
  }
  __syncthreads();
  if (tid < 128)
    egp[tid] = expf((red[tid] + red[128 + tid] + red[256 + tid] + red[384 + tid]) / float(nq));
  fence_proxy_async();
  __syncthreads();
  // [W_k^T | W_b] in over the gate scratch (128 pairs).
  if (tid == 0 && !split) {
    mbar_arrive_expect_tx(bar_ld, 65536u);
    bulk_g2s(XW, pt + PT_W2A, 65536u, bar_ld);
  }
  if (!mbar_wait(bar_ld, ph_ld)) *abort_flag = 1;
  ph_ld ^= 1;
  // P2a (u at lanes +0, b logits at lanes +16 when split)
  if (tid == 0) {
    fence_after_sync();
    if (split) {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_half, false);
      mma_tile(tG + (16u << 16), smem_u32(XQ), smem_u32(XW + 128 * 128), TV, id_half, false);
    } else {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_gate, false);
    }
    mma_commit(bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // keys = u / max(|u|, 1e-12) (probe.py:100): row norms across the four parts.
  {
    float u[32];
    tmem_ld32(taddr(tG, 32 * quarter, c0), u);
    float ss = 0.f;
#pragma unroll
    for (int t = 0; t < 32; ++t) ss = fmaf(u[t], u[t], ss);
    if (row >= 0 && (!split || lane < 16)) red[(warp >> 2) * 128 + row] = ss;
  }
  __syncthreads();
  bf16* keysT = XW;                      // MN-major A: keys^T [K x mp]
  bf16* kbg = XW + 16384;                // K-major A: keys * b * e^g [mp x K]
  {
    const float inv =
        row >= 0 ? __fdividef(1.f, fmaxf(sqrtf(red[row] + red[128 + row] + red[256 + row] +
                                               red[384 + row]), 1e-12f))
                 : 0.f;
    if (split) {
      // Lane l < 16 holds u of pair 16q + l, lane l + 16 its b logits. The
      // two swap halves (the low lane keeps columns 0..15, the high lane
      // takes 16..31) and each writes 16 columns of keys and k * b * e^g.
      const bool hi = lane >= 16;
      const int pr = 16 * quarter + (lane & 15), cb = c0 + (hi ? 16 : 0);
      const float iv = __shfl_sync(0xffffffffu, inv, lane & 15);
      float x0[16], x1[16];
      tmem_ld16(taddr(tG, 32 * quarter, c0), x0);
      tmem_ld16(taddr(tG, 32 * quarter, c0 + 16), x1);
#pragma unroll
      for (int c = 0; c < 16; c += 8) {
        float kk[8], kb[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int j = c + t;
          const float got = __shfl_xor_sync(0xffffffffu, hi ? x0[j] : x1[j], 16);
          const float uu = hi ? got : x0[j], bb = hi ? x1[j] : got;
          kk[t] = uu * iv;
          kb[t] = kk[t] * (fast_sigmoid(bb + kBLogitInit) * egp[cb + j]);
        }
        *reinterpret_cast<uint4*>(keysT + mnmajor_off(pr, cb + c, mp)) = pack8(kk);
        *reinterpret_cast<uint4*>(kbg + kmajor_off(pr, cb + c, TK)) = pack8(kb);
      }
    } else {
      float u[32], bl[32];
      tmem_ld32(taddr(tG, 32 * quarter, c0), u);
      tmem_ld32(taddr(tG, 32 * quarter, 128 + c0), bl);
#pragma unroll
      for (int t = 0; t < 32; ++t) bl[t] = fast_sigmoid(bl[t] + kBLogitInit) * egp[c0 + t];
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float kk[8], kb[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          kk[t] = u[c + t] * inv;
          kb[t] = kk[t] * bl[c + t];
        }
        *reinterpret_cast<uint4*>(keysT + mnmajor_off(row, c0 + c, mp)) = pack8(kk);
        *reinterpret_cast<uint4*>(kbg + kmajor_off(row, c0 + c, TK)) = pack8(kb);
      }
    }
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  // P3: (keys * b * e^g) . S_l; meanwhile e^g * S_l (fp32 master) into TMEM.
  if (tid == 0) {
    fence_after_sync();
    mma_tile(tG, smem_u32(kbg), smem_u32(Sbf + l * TK * TV), TK, id_read, false);
    mma_commit(bar_mma);
  }
  __syncwarp();
  {
    const int k = 32 * quarter + lane;
    const float e = egp[k];
    float4 sl4[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) sl4[t] = *reinterpret_cast<const float4*>(Sl + lm_off(k, c0 + 4 * t));
    float x[32];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      x[4 * t] = sl4[t].x * e;
      x[4 * t + 1] = sl4[t].y * e;
      x[4 * t + 2] = sl4[t].z * e;
      x[4 * t + 3] = sl4[t].w * e;
    }
    tmem_st32(taddr(tS, 32 * quarter, c0), x);
    tmem_wait_st();
  }
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // vn = v * w - (keys * b * e^g) . S_l -> MN-major B operand [mp x V].
  {
    float vw[32], d[32];
    tmem_ld32(taddr(tV, 32 * quarter, c0), vw);
    tmem_ld32(taddr(tG, 32 * quarter, c0), d);
    if (row >= 0) {
#pragma unroll
      for (int t = 0; t < 32; ++t) vw[t] -= d[t];
#pragma unroll
      for (int c = 0; c < 32; c += 8)
        *reinterpret_cast<uint4*>(XQ + mnmajor_off(row, c0 + c, mp)) = pack8(vw + c);
    }
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  // P4: S_l += keys^T . vn
  if (tid == 0) {
    fence_after_sync();
    mma_tile(tS, smem_u32(keysT), smem_u32(XQ), mp, id_upd, true);
    mma_commit(bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  {
    const int k = 32 * quarter + lane;
    float x[32];
    tmem_ld32(taddr(tS, 32 * quarter, c0), x);
#pragma unroll
    for (int t = 0; t < 32; t += 4)
      *reinterpret_cast<float4*>(Sl + lm_off(k, c0 + t)) = make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
#pragma unroll
    for (int c = 0; c < 32; c += 8)
      *reinterpret_cast<uint4*>(Sbf + l * TK * TV + mnmajor_off(k, c0 + c, TK)) = pack8(x + c);
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
}

// Merge promotion of level l - 1 into level l on the tensor cores
// (probe.py:105-136 with the gates of :34-66, naive.py:7-39): the values are
// the rows of S_{l-1} and the keys the identity, so the gram matrix is
// diag(b[k][k]) and the update is row by row,
//     S_l[k] <- (1 - b[k][k]) e^(g_k) S_l[k] + S_{l-1}[k] * w[k],
// with w = sigmoid(S_{l-1} . W_w), b = sigmoid(S_{l-1} . W_b - 4) and
// g = mean_k(-softplus(S_{l-1} . W_g - 4)). The three gate GEMMs run as two
// M = 128, N = 256 MMAs ([W_w | W_g] and [W_k^T | W_b]; the W_k^T half is
// unused) on a bf16 copy of S_{l-1}; the update reads and writes the fp32
// masters in final_state. Same TMEM columns and scratch as promote_tc.
__device__ void promote_merge_tc(const FwdParams& p, const TcLayout& lay, const char* ws, int h,
                                 int l, uint32_t tb, bf16* Sbf, uint8_t* X, float* Sg,
                                 uint64_t* bar_ld, uint64_t* bar_mma, uint32_t& ph_ld,
                                 uint32_t& ph_mma, float* egp, float* red, int* abort_flag) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, c0 = 32 * (warp >> 2);
  const int row = 32 * quarter + lane;  // pair index = key index
  const char* pt = ws + lay.ptc_off + (int64_t(l - 1) * p.H + h) * PT_SIZE;
  bf16* XW = reinterpret_cast<bf16*>(X);
  bf16* XQ = reinterpret_cast<bf16*>(X + 65536);
  const uint32_t tV = tb + 128, tG = tb + 256;
  const uint32_t id_gate = idesc_f16(128, 256, true, false, false);
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_ld, 65536u);
    bulk_g2s(XW, pt + PT_W2B, 65536u, bar_ld);
  }
  // V' = S_{l-1} as a K-major A operand: the bf16 copy's 16-byte pieces
  // (8 values of one row) reordered from the MN-major B layout.
  {
    const uint4* src = reinterpret_cast<const uint4*>(Sbf + (l - 1) * TK * TV);
    uint4* dst = reinterpret_cast<uint4*>(XQ);
    for (int e = tid; e < TK * TV / 8; e += kScanThreads) {
      const int e8 = e & 7, kg = (e >> 3) & 15, vg = e >> 7;
      dst[((kg * 16 + vg) << 3) + e8] = src[e];
    }
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  if (!mbar_wait(bar_ld, ph_ld)) *abort_flag = 1;
  ph_ld ^= 1;
  if (tid == 0) {
    fence_after_sync();
    mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_gate, false);
    mma_commit(bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // w = sigmoid(w_logit) into TMEM; -softplus(g_logit - 4) per pair into the
  // (spent) [W_w | W_g] buffer, columns XOR-swizzled by row.
  float* gpart = reinterpret_cast<float*>(X);
  {
    float a[32];
    tmem_ld32(taddr(tG, 32 * quarter, c0), a);
#pragma unroll
    for (int u = 0; u < 32; ++u) a[u] = sigmoidf_(a[u] + kWLogitInit);
    tmem_st32(taddr(tV, 32 * quarter, c0), a);
    tmem_ld32(taddr(tG, 32 * quarter, 128 + c0), a);
#pragma unroll
    for (int u = 0; u < 32; ++u) gpart[row * 128 + ((c0 + u) ^ (row & 31))] = -softplusf_(a[u] + kGLogitInit);
  }
  tmem_wait_st();
  __syncthreads();
  {
    const int k = tid & 127, qq = tid >> 7;
    float sum = 0.f;
    for (int r = qq * 32; r < qq * 32 + 32; ++r) sum += gpart[r * 128 + (k ^ (r & 31))];
    red[qq * 128 + k] = sum;
  }
  __syncthreads();
  if (tid < 128) egp[tid] = expf((red[tid] + red[128 + tid] + red[256 + tid] + red[384 + tid]) / 128.f);
  fence_proxy_async();
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_ld, 65536u);
    bulk_g2s(XW, pt + PT_W2A, 65536u, bar_ld);
  }
  if (!mbar_wait(bar_ld, ph_ld)) *abort_flag = 1;
  ph_ld ^= 1;
  if (tid == 0) {
    fence_after_sync();
    mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_gate, false);
    mma_commit(bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(bar_mma, ph_mma)) *abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // b[k][k] from the warps whose 32 columns hold row k's diagonal.
  if ((warp >> 2) == quarter) {
    float a[32];
    tmem_ld32(taddr(tG, 32 * quarter, 128 + c0), a);
    float d = 0.f;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u == lane) d = a[u];
    red[row] = sigmoidf_(d + kBLogitInit);
  }
  __syncthreads();
  {
    const int k = row;
    const float e = egp[k], keep = 1.f - red[k];
    float w[32];
    tmem_ld32(taddr(tV, 32 * quarter, c0), w);
    float* Sl = Sg + int64_t(l) * TK * TV + k * TV + c0;
    const float* Sb = Sg + int64_t(l - 1) * TK * TV + k * TV + c0;
    float x[32];
#pragma unroll
    for (int t = 0; t < 32; t += 4) {
      const float4 sl = *reinterpret_cast<const float4*>(Sl + t);
      const float4 sb = *reinterpret_cast<const float4*>(Sb + t);
      x[t] = keep * e * sl.x + sb.x * w[t];
      x[t + 1] = keep * e * sl.y + sb.y * w[t + 1];
      x[t + 2] = keep * e * sl.z + sb.z * w[t + 2];
      x[t + 3] = keep * e * sl.w + sb.w * w[t + 3];
    }
#pragma unroll
    for (int t = 0; t < 32; t += 4)
      *reinterpret_cast<float4*>(Sl + t) = make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
#pragma unroll
    for (int c = 0; c < 32; c += 8)
      *reinterpret_cast<uint4*>(Sbf + l * TK * TV + mnmajor_off(k, c0 + c, TK)) = pack8(x + c);
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
}

// qmap views q as 4-D [64 channels, (b, t) tokens, 2 channel halves,
// (head, level) pairs] with 128-byte swizzle: one (64, 64, 2, 1) box is a
// [64 tokens x 128] K-major MMA operand in the swizzled layout (sw128_off).
// hl = h * L + l when hl_mode == 0, l * H + h when 1. With hl_mode == 2 (q
// laid out otherwise) there is no map: the scaling warps read their rows
// from q themselves.
__global__ void __launch_bounds__(kScanThreads, 1)
scan_tc_kernel(FwdParams p, TcLayout lay, char* ws, const __grid_constant__ CUtensorMap qmap,
               int hl_mode) {
  if (gate_closed(p)) return;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  __shared__ uint64_t bar_ld, bar_ld2, bar_mma, bar_q, bar_lvl;
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  __shared__ float egp[128];
  __shared__ float red[512];
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.L;
  const int quarter = warp & 3, c0 = 32 * (warp >> 2);
  const int64_t bh = int64_t(b) * p.H + h;
  const uint32_t load_bytes = static_cast<uint32_t>(lay.rec.load_bytes);
  // The swizzled query tiles need 1024-byte alignment (the launch adds the
  // slack).
  uint8_t* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  bf16* Sbf = reinterpret_cast<bf16*>(sm);
  uint8_t* Rec = sm + int64_t(L) * TILE_S;
  uint8_t* QT = Rec + lay.rec.load_bytes;  // upper-level query tiles (sw128_off)
  bf16* Vn = reinterpret_cast<bf16*>(QT + int64_t(L - 1) * TILE_QK);
  float* Sg = p.fin + bh * L * TK * TV;
  const bool learned = p.promotion != NGDN2_PROMOTION_MERGE;
  // Learned promotions keep the upper levels' fp32 masters lane-major in
  // the workspace; merge promotions (row by row) use final_state as is.
  float* Mt = reinterpret_cast<float*>(ws + lay.mast_off) + bh * (L > 1 ? L - 1 : 0) * TK * TV;
  const char* rec0 = ws + lay.chunks_off + bh * p.NT * lay.rec.size;

  if (warp == 0) tmem_alloc(&tbase, kScanCols);
  if (tid == 0) {
    mbar_init(&bar_ld, 1);
    mbar_init(&bar_ld2, 1);
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_q, 1);
    mbar_init(&bar_lvl, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  for (int64_t e = tid; e < int64_t(L) * TK * TV; e += kScanThreads)
    Sg[e] = p.init ? p.init[bh * L * TK * TV + e] : 0.f;
  if (learned) {
    for (int64_t e = tid; e < int64_t(L - 1) * TK * TV; e += kScanThreads) {
      const int64_t l1 = e / (TK * TV), r2 = e % (TK * TV), k = r2 / TV, v = r2 % TV;
      Mt[l1 * TK * TV + lm_off(int(k), int(v))] = p.init ? p.init[bh * L * TK * TV + (l1 + 1) * TK * TV + r2] : 0.f;
    }
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tb = tbase;
  const uint32_t tS0 = tb;        // S0 [K lanes x V cols], fp32
  // Chunk accumulator, one M = 128 tile: lanes 0..63 W.S0, lanes 64..127
  // the output rows.
  const uint32_t tD = tb + 128;

  // S0 into TMEM, bf16 copies of every level into shared memory.
  {
    const int k = 32 * quarter + lane;
    float x[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) x[t] = Sg[k * TV + c0 + t];
    tmem_st32(taddr(tS0, 32 * quarter, c0), x);
    tmem_wait_st();
  }
  for (int l = 0; l < L; ++l) refresh_copy(Sbf + l * TK * TV, Sg + l * TK * TV);
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();

  const uint32_t id_m128 = idesc_f16(128, 128, true, false, true);  // [128 x K] . [K x V]
  const uint32_t id_state = idesc_f16(128, 128, true, true, true);  // K_tail^T [K x 64] . [64 x V]
  uint32_t ph_ld = 0, ph_mma = 0;
  // Chunks left until each level's next firing (naive.py:394-415 fires level
  // l after chunk n when (n + 1) % f_l == 0).
  // (this family has L <= 3).
  int left1 = L > 1 ? p.firing[1] : 0, left2 = L > 2 ? p.firing[2] : 0;
  // A record arrives in two parts: [W, Q_0] (read by MMA1) on bar_ld and
  // the rest (read by MMA2) on bar_ld2, so each part of the next record can
  // stream in as soon as its MMA has finished with the current one.
  const uint32_t part_a = static_cast<uint32_t>(lay.rec.Q + TILE_QK);
  auto load_part = [&](const char* src, bool a) {
    const uint32_t lo = a ? 0u : part_a, hi = a ? part_a : load_bytes;
    uint64_t* bar = a ? &bar_ld : &bar_ld2;
    mbar_arrive_expect_tx(bar, hi - lo);
    bulk_g2s(Rec + lo, src + lo, hi - lo, bar);
  };
  uint32_t ph_ld2 = 0, ph_q = 0, ph_lvl = 0;
  // The upper levels' raw query tiles of chunk nn (read by MMA2 after the
  // warps idle in E1 scale their rows by mix_l * scale; naive.py:382-385).
  const bool q_tma = hl_mode != 2;
  // Query tiles that need a pass before MMA2 reads them (fp16 to bf16, or
  // plain loads); bf16 tiles from the map are read as they land.
  const bool q_conv = !q_tma || p.q.dt != NGDN2_BF16;
  auto load_q = [&](int nn) {
    if (L < 2 || !q_tma) return;
    mbar_arrive_expect_tx(&bar_q, uint32_t(L - 1) * TILE_QK);
    const int row = b * p.T + nn * kC;
    for (int l = 1; l < L; ++l)
      tma_load_4d(QT + (l - 1) * TILE_QK, &qmap, 0, row, 0, hl_mode ? l * p.H + h : h * L + l,
                  &bar_q);
  };
  if (tid == 0 && p.NT > 0) {
    load_part(rec0, true);
    load_part(rec0, false);
    load_q(0);
  }
  // mix_l * scale of the upper levels for the output row this thread
  // assembles in E2 (threads of lane quarters 2 and 3), one chunk ahead.
  const int jq = (warp >> 2) * 64 + (warp & 1) * 32 + lane;  // 0..255 among them
  // The raw bits are loaded at the top of the chunk before and converted
  // after that chunk's E2, so the load latency hides behind a whole chunk.
  float mixr[2] = {0.f, 0.f};
  uint32_t mixraw[2] = {0u, 0u};
  auto fetch_mix = [&](int nn) {
    if (quarter < 2) return;
    const int t = nn * kC + (jq & 63);
#pragma unroll
    for (int l = 1; l < 3; ++l) {
      if (l >= L) break;
      mixraw[l - 1] = 0u;
      if (t < p.T) {
        const int64_t o = p.mix.off(b, t, h, l);
        mixraw[l - 1] = p.mix.dt == NGDN2_F32
                            ? __ldg(reinterpret_cast<const unsigned int*>(p.mix.p) + o)
                            : uint32_t(__ldg(reinterpret_cast<const unsigned short*>(p.mix.p) + o));
      }
    }
  };
  auto take_mix = [&]() {
#pragma unroll
    for (int l = 0; l < 2; ++l) {
      const uint32_t r = mixraw[l];
      const float m = p.mix.dt == NGDN2_F32    ? __uint_as_float(r)
                      : p.mix.dt == NGDN2_BF16 ? __uint_as_float(r << 16)
                                               : __half2float(__ushort_as_half(uint16_t(r)));
      mixr[l] = m * p.scale;
    }
  };
  // U rows (lanes of quarters 0 and 1) and e^(G_last) of a chunk, read from
  // its record in global memory one chunk ahead of use.
  uint4 urow[4];
  float eg = 0.f;
  auto fetch_rows = [&](int nn) {
    const char* rg = rec0 + int64_t(nn) * lay.rec.size;
    if (quarter < 2) {
      // Piece c0/8 + c of row 32 * quarter + lane: a warp's load is 512
      // contiguous bytes.
      const uint4* Ug = reinterpret_cast<const uint4*>(rg + lay.rec.U) + (c0 / 8) * kC +
                        32 * quarter + lane;
#pragma unroll
      for (int c = 0; c < 4; ++c) urow[c] = __ldg(Ug + c * kC);
    }
  };
  auto fetch_eg = [&](int nn) {
    const char* rg = rec0 + int64_t(nn) * lay.rec.size;
    eg = __ldg(reinterpret_cast<const float*>(rg + lay.rec.eg) + 32 * quarter + lane);
  };
  // S0 decayed by the first chunk's e^(G_last) (naive.py:392, first term);
  // each later chunk's decay is applied where the previous epilogue reads S0.
  if (p.NT > 0) {
    fetch_rows(0);
    fetch_eg(0);
    fetch_mix(0);
    take_mix();
    const uint32_t ta = taddr(tS0, 32 * quarter, c0);
    float x[32];
    tmem_ld32(ta, x);
#pragma unroll
    for (int t = 0; t < 32; ++t) x[t] *= eg;
    tmem_st32(ta, x);
    tmem_wait_st();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
  }
  for (int n = 0; n < p.NT; ++n) {
    const char* recg = rec0 + int64_t(n) * lay.rec.size;
    if (!mbar_wait(&bar_ld, ph_ld)) abort_flag = 1;
    ph_ld ^= 1;
    // e^(G_last) of the next chunk (for the decay in this chunk's E2) and
    // its mix weights.
    if (n + 1 < p.NT) {
      fetch_eg(n + 1);
      fetch_mix(n + 1);
    }
    uint32_t fire_mask = 0;
    if (L > 1 && --left1 == 0) {
      fire_mask |= 2u;
      left1 = p.firing[1];
    }
    if (L > 2 && --left2 == 0) {
      fire_mask |= 4u;
      left2 = p.firing[2];
    }
    const bool fires = fire_mask != 0;
    // The fp32 masters that this chunk's learned promotions read (at P3)
    // are asked into L2 now, a chunk's work ahead of use.
    if (tid == 96 && fires && learned)
      for (int l = 1; l < L; ++l)
        if (fire_mask >> l & 1u) bulk_prefetch_l2(Mt + int64_t(l - 1) * TK * TV, TK * TV * 4);

    // MMA1: [W; Q_0] . S0 as one M = 128 tile (W and Q_0 are adjacent in the
    // record): W.S0 in lanes 0..63 and the level-0 read in lanes 64..127,
    // both from the state entering the chunk (naive.py:376, 379).
    if (tid == 0) {
      fence_after_sync();
      mma_tile(tD, smem_u32(Rec + lay.rec.W), smem_u32(Sbf), TK, id_m128, false);
      mma_commit(&bar_mma);
    }
    // The upper-level reads q_l . S_l (naive.py:382-385) need neither v_new
    // nor S0: with bf16 query tiles from the map they are issued here, by a
    // thread of a warp that E1 leaves idle, so the tensor pipe runs them
    // during E1. Each lands in lanes 64..127 of its own accumulator (the
    // lower half of an M = 128 tile whose upper half, the 64 rows stored
    // before the tile, lands in lanes that are never read) and is weighted
    // by mix_l * scale per row in E2.
    if (tid == 64 && L > 1 && !q_conv) {
      if (!mbar_wait(&bar_q, ph_q)) abort_flag = 1;
      fence_after_sync();
      for (int l = 1; l < L; ++l)
        mma_tile_sw128_lo(tD + 128 * l, smem_u32(QT + (l - 1) * TILE_QK),
                          smem_u32(Sbf + l * TK * TV), id_m128, false);
      mma_commit(&bar_lvl);
    }
    __syncwarp();
    if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
    ph_mma ^= 1;
    fence_after_sync();

    // E1: v_new = U - W.S0 -> bf16 B operand (naive.py:376). Meanwhile, for
    // fp16 q or q without a tensor map, the other warps turn the upper
    // levels' query tiles into bf16 (the state operand's type).
    if (quarter < 2) {
      const int i = 32 * quarter + lane;
      float x[32];
      tmem_ld32(taddr(tD, 32 * quarter, c0), x);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float uu[8];
        unpack8(urow[c], NGDN2_BF16, uu);
#pragma unroll
        for (int t = 0; t < 8; ++t) uu[t] -= x[8 * c + t];
        *reinterpret_cast<uint4*>(Vn + mnmajor_off(i, c0 + 8 * c, kC)) = pack8(uu);
      }
    } else if (L > 1 && q_conv) {
      if (q_tma && !mbar_wait(&bar_q, ph_q)) abort_flag = 1;
      const int r = jq & 63, g4 = jq >> 6;
#pragma unroll
      for (int l = 1; l < 3; ++l) {
        if (l >= L) break;
        bf16* tile = reinterpret_cast<bf16*>(QT + (l - 1) * TILE_QK);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4* q8 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(tile) +
                                               sw128_off(r, 8 * (g4 + 4 * u)));
          float f[8];
          const uint4 raw = q_tma ? *q8
                            : n * kC + r < p.T ? raw8_at(p.q.p, p.q.dt,
                                             p.q.off(b, n * kC + r, h, l, 8 * (g4 + 4 * u)), p.q.sd)
                                   : make_uint4(0, 0, 0, 0);
          unpack8(raw, p.q.dt, f);
          *q8 = pack8(f);
        }
      }
    }
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    if (abort_flag) break;
    // W and Q_0 are spent: the next record's first part streams in (unless
    // a promotion needs the buffer as scratch first). It is issued only after
    // this barrier, which every thread reaches after its wait on bar_ld: a
    // phase completing early could otherwise alias the parity a slow thread
    // still waits for. (Issued by warp 1: thread 0 goes on to MMA2.) The
    // next chunk's U rows load during MMA2 (at a firing they wait for the
    // end of the promotions: they would hold registers across them).
    if (tid == 32 && n + 1 < p.NT && !fires) load_part(recg + lay.rec.size, true);

    // MMA2: S0 += K_tail^T v_new (naive.py:392); (mix0 scale A_qk) v_new
    // into the output lanes 64..127 (naive.py:379), as the lower half of an
    // M = 128 tile like the reads; and the upper-level reads here when their
    // tiles needed the conversion pass.
    if (tid == 0) {
      if (!mbar_wait(&bar_ld2, ph_ld2)) abort_flag = 1;
      fence_after_sync();
      mma_tile(tS0, smem_u32(Rec + lay.rec.Kt), smem_u32(Vn), kC, id_state, true);
      mma_tile(tD, smem_u32(Rec + lay.rec.A - TILE_A), smem_u32(Vn), kC, id_m128, true);
      if (q_conv)
        for (int l = 1; l < L; ++l)
          mma_tile_sw128_lo(tD + 128 * l, smem_u32(QT + (l - 1) * TILE_QK),
                            smem_u32(Sbf + l * TK * TV), id_m128, false);
      mma_commit(&bar_mma);
    }
    if (n + 1 < p.NT && !fires) fetch_rows(n + 1);
    ph_ld2 ^= 1;
    ph_q ^= 1;
    __syncwarp();
    if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
    ph_mma ^= 1;
    if (L > 1 && !q_conv) {
      if (!mbar_wait(&bar_lvl, ph_lvl)) abort_flag = 1;
      ph_lvl ^= 1;
    }
    fence_after_sync();
    // The rest of the next record streams in during the epilogue; at a
    // firing the first learned promotion's operands do instead.
    // (Only when the bank stays clear of the v_new tile that the output
    // rows are staged in.)
    const int first = fires ? __ffs(fire_mask) - 1 : 0;
    const bool early = fires && learned &&
                       65536 + pad_pairs(p.nq[first - 1]) * 256 <= load_bytes + (L - 1) * TILE_QK;
    // (Issued by lanes of three warps of lane quarters 0 and 1, whose share
    // of E2 is the shortest; warp 0's thread 0 issues the MMAs.)
    if (tid == 32 && n + 1 < p.NT && !fires) load_part(recg + lay.rec.size, false);
    if (tid == 128 && n + 1 < p.NT && !fires) load_q(n + 1);
    if (tid == 160 && early) promote_tc_first_loads(p, lay, ws, h, first, Rec, &bar_ld);
    const bool write_master = (fires && !learned) || n + 1 == p.NT;
    const bool stage16 = p.dtype == NGDN2_BF16 || p.dtype == NGDN2_F16;

    // E2: output rows (lanes 64..127) and the new S0 (all lanes). 16-bit
    // outputs go through shared memory (the spent v_new tile, rows of 256
    // bytes with 16-byte chunks XOR-swizzled by row) so that the global
    // stores are whole rows.
    {
      float x[32];
      if (quarter >= 2) {
        // In halves of 16 columns: output = level-0 part + sum_l mix_l scale
        // (q_l . S_l).
        const int i = 32 * (quarter - 2) + lane, t = n * kC + i;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float xo[16];
          uint32_t y[2][16];
          tmem_ld16_nowait(taddr(tD, 32 * quarter, c0 + 16 * hh),
                           reinterpret_cast<uint32_t*>(xo));
          // (Both level accumulators are loaded whatever L is: the columns
          // are allocated; only the levels present are added.)
          tmem_ld16_nowait(taddr(tD + 128, 32 * quarter, c0 + 16 * hh), y[0]);
          tmem_ld16_nowait(taddr(tD + 256, 32 * quarter, c0 + 16 * hh), y[1]);
          tmem_wait_ld();
          tmem_regs_after_wait16(reinterpret_cast<uint32_t*>(xo));
#pragma unroll
          for (int l = 1; l < 3; ++l) {
            tmem_regs_after_wait16(y[l - 1]);
            if (l >= L) break;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              xo[j] = fmaf(mixr[l - 1], __uint_as_float(y[l - 1][j]), xo[j]);
          }
          if (stage16) {
            uint4* row = reinterpret_cast<uint4*>(Vn) + i * 16;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int ch = (c0 >> 3) + 2 * hh + c;
              row[ch ^ (i & 15)] = p.dtype == NGDN2_BF16 ? pack8(xo + 8 * c) : pack8h(xo + 8 * c);
            }
          } else if (t < p.T) {
            const int64_t o = ((int64_t(b) * p.T + t) * p.H + h) * TV + c0 + 16 * hh;
#pragma unroll
            for (int u = 0; u < 16; ++u) store_elem(p.o, o + u, xo[u], p.dtype);
          }
        }
      }
      // The new S0: bf16 copy (and fp32 master), then S0 in TMEM decayed
      // by the next chunk's e^(G_last).
      const int k = 32 * quarter + lane;
      const uint32_t ta = taddr(tS0, 32 * quarter, c0);
      tmem_ld32(ta, x);
#pragma unroll
      for (int c = 0; c < 32; c += 8)
        *reinterpret_cast<uint4*>(Sbf + mnmajor_off(k, c0 + c, TK)) = pack8(x + c);
      if (write_master) {
#pragma unroll
        for (int u = 0; u < 32; u += 4)
          *reinterpret_cast<float4*>(Sg + k * TV + c0 + u) = make_float4(x[u], x[u + 1], x[u + 2], x[u + 3]);
      }
      if (n + 1 < p.NT) {
#pragma unroll
        for (int t = 0; t < 32; ++t) x[t] *= eg;
        tmem_st32(ta, x);
        tmem_wait_st();
      }
    }
    take_mix();
    if (stage16) {
      __syncthreads();
      // 64 rows x 16 chunks of 16 bytes: each warp stores two whole rows per step.
      for (int e = tid; e < kC * 16; e += kScanThreads) {
        const int i = e >> 4, ch = e & 15, t = n * kC + i;
        if (t < p.T) {
          const uint4 v = reinterpret_cast<const uint4*>(Vn)[i * 16 + (ch ^ (i & 15))];
          *(reinterpret_cast<uint4*>(p.o) + (((int64_t(b) * p.T + t) * p.H + h) * TV) / 8 + ch) = v;
        }
      }
    }
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (abort_flag) break;

    // Promotions at this chunk's firings, bottom-up (naive.py:394-415).
    if (fires) {
      for (int l = 1; l < L; ++l) {
        if (!(fire_mask >> l & 1u)) continue;
        if (!learned) {
          promote_merge_tc(p, lay, ws, h, l, tb, Sbf, Rec, Sg, &bar_ld, &bar_mma, ph_ld, ph_mma,
                           egp, red, &abort_flag);
        } else {
          promote_tc(p, lay, ws, h, l, tb, Sbf, Rec, Mt, &bar_ld, &bar_mma, ph_ld, ph_mma, egp,
                     red, &abort_flag, early && l == first);
        }
      }
      fence_before_sync();
      __syncthreads();
      fence_after_sync();
      if (abort_flag) break;
      if (tid == 0 && n + 1 < p.NT) {
        load_part(recg + lay.rec.size, true);
        load_part(recg + lay.rec.size, false);
        load_q(n + 1);
      }
      if (n + 1 < p.NT) fetch_rows(n + 1);
    }
  }
  if (abort_flag && tid == 0) set_status(p, NGDN2_STATUS_WAIT_TIMEOUT);
  // Upper levels' final states from the lane-major masters.
  if (learned) {
    __syncthreads();
    for (int64_t e = tid; e < int64_t(L - 1) * TK * TV; e += kScanThreads) {
      const int64_t l1 = e / (TK * TV), r2 = e % (TK * TV), k = r2 / TV, v = r2 % TV;
      Sg[(l1 + 1) * TK * TV + r2] = Mt[l1 * TK * TV + lm_off(int(k), int(v))];
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, kScanCols);
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static bool is16(int dt) { return dt == NGDN2_BF16 || dt == NGDN2_F16; }

// How the scan's tensor map walks q's (head, level) pairs: 0 when the level
// index is the contiguous one (hl = h * L + l), 1 when the head is (hl =
// l * H + h), -1 when q's layout has no such single stride.
// The map needs 16-byte aligned q and token stride, (b, t) rows in one
// stride and one of the two (head, level) layouts; 2 otherwise.
static int q_hl_mode(const FwdParams& p) {
  const auto& q = p.q;
  if (q.sd != 1 || q.sb != int64_t(p.T) * q.st || q.st % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(q.p) & 15) != 0)
    return 2;
  if (q.sl == TK && q.sh == int64_t(p.L) * TK) return 0;
  if (q.sh == TK && q.sl == int64_t(p.H) * TK) return 1;
  return 2;
}

bool tc_supports(const ngdn2_fwd_args* a) {
  if (a->K != TK || a->V != TV || a->L < 1 || a->L > 3) return false;
  if (!is16(a->q_dtype) || !is16(a->k_dtype) || !is16(a->v_dtype) || !is16(a->b_dtype) ||
      !is16(a->w_dtype) || !is16(a->dtype))
    return false;
  return true;
}

// Tensor map of q for the scan (see scan_tc_kernel): 4-D view whose
// (64, 64, 2, 1) box is one chunk's [64 x 128] operand, 128-byte swizzled.
static PFN_cuTensorMapEncodeTiled g_encode = nullptr;

// Looks up cuTensorMapEncodeTiled once; false when the driver lacks it.
static bool encoder_ready() {
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  return true;
}

static bool make_q_map(const FwdParams& p, CUtensorMap* m) {
  if (!encoder_ready()) return false;
  const auto encode = g_encode;
  // Both (head, level) layouts step from one pair to the next by K elements.
  const cuuint64_t dims[4] = {64, cuuint64_t(p.B) * p.T, TK / 64, cuuint64_t(p.H) * p.L};
  const cuuint64_t strides[3] = {cuuint64_t(p.q.st) * 2, 128, cuuint64_t(TK) * 2};
  const cuuint32_t box[4] = {64, kC, TK / 64, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode(
      m, p.q.dt == NGDN2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      4, const_cast<void*>(p.q.p), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The prep inputs' prefetch maps (see PrepMaps); a tensor whose layout the
// 3-D view cannot describe (a stride-0 broadcast gate, say) is left out.
static void make_prep_maps(const FwdParams& p, PrepMaps* pm) {
  memset(pm, 0, sizeof(*pm));
  if (!encoder_ready()) return;
  struct View { const void* ptr; int dt; int64_t sb, st, sh, sd; };
  const View views[6] = {{p.q.p, p.q.dt, p.q.sb, p.q.st, p.q.sh, p.q.sd},
                         {p.g.p, p.g.dt, p.g.sb, p.g.st, p.g.sh, p.g.sd},
                         {p.k.p, p.k.dt, p.k.sb, p.k.st, p.k.sh, p.k.sd},
                         {p.b.p, p.b.dt, p.b.sb, p.b.st, p.b.sh, p.b.sd},
                         {p.v.p, p.v.dt, p.v.sb, p.v.st, p.v.sh, p.v.sd},
                         {p.w.p, p.w.dt, p.w.sb, p.w.st, p.w.sh, p.w.sd}};
  for (int i = 0; i < 6; ++i) {
    const View& v = views[i];
    const int64_t es = v.dt == NGDN2_F32 ? 4 : 2;
    if (v.sd != 1 || v.st <= 0 || v.sh <= 0 || v.sb != int64_t(p.T) * v.st ||
        (v.st * es) % 16 != 0 || (v.sh * es) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(v.ptr) & 15) != 0)
      continue;
    const cuuint64_t dims[3] = {cuuint64_t(TK), cuuint64_t(p.B) * p.T, cuuint64_t(p.H)};
    const cuuint64_t strides[2] = {cuuint64_t(v.st * es), cuuint64_t(v.sh * es)};
    const cuuint32_t box[3] = {cuuint32_t(TK), cuuint32_t(kC), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = g_encode(
        &pm->m[i], es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 3,
        const_cast<void*>(v.ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS) pm->valid |= 1u << i;
  }
}

size_t tc_workspace_bytes(const FwdParams& p) { return size_t(tc_layout(p).total); }

int num_launches_tc(const FwdParams& p) {
  return (p.L > 1 ? 1 : 0) + (p.NT > 0 ? 1 : 0) + 1;
}

cudaError_t launch_tc_params(const FwdParams& p, const TcLayout& lay, char* ws,
                             cudaStream_t stream) {
  if (p.L <= 1) return cudaSuccess;
  tc_params_kernel<<<dim3(p.L - 1, p.H, kParamSlices), 256, 0, stream>>>(p, lay, ws);
  return cudaGetLastError();
}

cudaError_t launch_tc_prep(const FwdParams& p, const TcLayout& lay, char* ws,
                           cudaStream_t stream) {
  if (p.NT <= 0) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(prep_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem);
  if (err != cudaSuccess) return err;
  PrepMaps pm;
  make_prep_maps(p, &pm);
  prep_tc_kernel<<<dim3(p.NT, p.H, p.B), kPrepThreads, kPrepSmem, stream>>>(p, lay, ws, pm);
  return cudaGetLastError();
}

bool tc_make_q_map(const FwdParams& p, CUtensorMap* m, int* hl_mode) {
  *hl_mode = p.L > 1 ? q_hl_mode(p) : 2;
  memset(m, 0, sizeof(*m));
  return *hl_mode == 2 || make_q_map(p, m);
}

cudaError_t launch_fwd_tc(FwdParams p, void* workspace, int stage, cudaStream_t stream) {
  const TcLayout lay = tc_layout(p);
  char* ws = static_cast<char*>(workspace);
  p.chunks = nullptr;
  cudaError_t err;
  if (stage == 0 || stage == 1) {
    if ((err = launch_tc_params(p, lay, ws, stream)) != cudaSuccess) return err;
    if ((err = launch_tc_prep(p, lay, ws, stream)) != cudaSuccess) return err;
  }
  if (stage == 0 || stage == 2) {
    const int smem = int(scan_tc_smem(p.L, lay.rec));
    err = cudaFuncSetAttribute(scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    CUtensorMap qmap;
    memset(&qmap, 0, sizeof(qmap));
    const int hl_mode = p.L > 1 ? q_hl_mode(p) : 2;
    if (hl_mode != 2 && !make_q_map(p, &qmap)) return cudaErrorInvalidValue;
    scan_tc_kernel<<<dim3(p.H, p.B), kScanThreads, smem, stream>>>(p, lay, ws, qmap, hl_mode);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace ngdn2
