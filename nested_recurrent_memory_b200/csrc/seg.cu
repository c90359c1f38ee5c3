// Level-segmented tensor-core family ("tc_seg") for K = V = 128, 16-bit
// inputs, any number of levels.
//
// Every level of the nested memory is a linear recurrence over its own steps
// -- level 0 over chunks, level l >= 1 over its firings:
//
//     S' = d * S + P^T (Y - R S)          (d scales the rows of S)
//
//   level 0, chunk n  (naive.py:376, 392):  R = W, P = K_tail, Y = U,
//                                           d = e^(G_last)
//   level l, firing i (naive.py:7-39 with probe.py:34-136):
//                                           R = keys * b * e^g, P = keys,
//                                           Y = values * w, d = e^g
//
// and a level's step operands depend only on the level below: the chunk
// prep gives level 0's, and level l's come from probing level l - 1's state
// at each firing (probe.py:69-136), which is known once level l - 1 has been
// scanned. So the forward runs level by level, each level as a segmented
// scan that fills the GPU even when few (batch, head) pairs exist (the
// long-context configuration has four per GPU):
//
//   compose  -- per segment of consecutive steps, in parallel: the
//               segment's transition S_end = M S_start + Z (M from the
//               identity with Y = 0, Z from zero; one CTA each);
//   combine  -- per (batch, head) and quarter of the value columns,
//               sequentially over segments: the state entering each
//               segment, M in two bf16 halves (hi + lo) times the state in
//               two halves, so the chain keeps ~16 bits;
//   replay   -- per segment, in parallel: the recurrence from the true start
//               state, emitting the states that later stages read (bf16, in
//               the MMA operand layout) and the final state (fp32).
//
// Level 0's replay also forms the level-0 part of the output (q0 . S0 +
// A_qk . v_new, naive.py:379). Then for each level l >= 1 a probe kernel
// turns level l - 1's emitted states at level l's firings into step records,
// level l is scanned the same way, and a last kernel adds the upper levels'
// reads sum_l mix_l scale q_l . S_l (naive.py:382-390) to the output.
//
// The chunk prep and the promotion-operand layouts are the fused family's
// (csrc/tc.cu). All contractions are tcgen05 MMAs (bf16 operands in shared
// memory, fp32 accumulators in TMEM); every wait is bounded.

#include <cuda.h>
#include <string.h>

#include "tc_api.cuh"
#include "tc_common.cuh"
#include "tc_ptx.cuh"

namespace ngdn2 {
namespace {

using namespace tcx;
using namespace tc;

constexpr int kSegThreads = 256;
constexpr int kProbeThreads = 512;
constexpr int kReadThreads = 256;
constexpr int kStateBytes = TK * TV * 2;     // one bf16 state in the B-operand layout
constexpr int kMzBytes = 2 * kStateBytes + TK * TV * 4;  // M hi, M lo (bf16), Z (fp32)
constexpr int kSMs = 148;                    // B200; sizes the segment split only

// Byte offsets of one step record's operands (see the file comment).
struct StepRec {
  int rows;                    // rows of R, P, Y: 64 for chunks, the padded pairs for firings
  int R, P, Y, d;              // R: K-major [rows x K]; P: MN-major [Kd = rows][M = K];
                               // Y: [V / 8][rows][8] 16-byte pieces; d: [K] fp32
  int Q, A;                    // level 0 only: read queries and mix0 scale A_qk (output part)
  int a_lo, a_hi, b_lo, b_hi;  // the bulk copy for MMA1 (R) and the one for MMA2 (P, A)
  int smem;                    // bytes of the record's shared-memory copy
  int64_t size;                // bytes per record
};

// Level-0 records are the prep's (TcRecord): W, Q, Kt, A, U, e^(G_last).
inline StepRec level0_rec(bool with_output) {
  const TcRecord r = TcRecord::make(1);
  StepRec s;
  s.rows = kC;
  s.R = int(r.W); s.Q = int(r.Q); s.P = int(r.Kt); s.A = int(r.A); s.Y = int(r.U); s.d = int(r.eg);
  s.a_lo = 0;
  s.a_hi = with_output ? int(r.Q) + TILE_QK : int(r.Q);
  s.b_lo = int(r.Kt);
  s.b_hi = with_output ? int(r.load_bytes) : int(r.A);
  s.smem = int(r.load_bytes);
  s.size = r.size;
  return s;
}

// Records of level l's firings, written by the probe kernel.
inline StepRec probe_rec(int mp) {
  StepRec s;
  s.rows = mp;
  s.R = 0; s.P = mp * 256; s.Y = 2 * mp * 256; s.d = 3 * mp * 256;
  s.Q = -1; s.A = -1;
  s.a_lo = 0; s.a_hi = mp * 256; s.b_lo = mp * 256; s.b_hi = 2 * mp * 256;
  s.smem = 2 * mp * 256;
  s.size = (int64_t(3 * mp * 256 + TK * 4) + 127) & ~int64_t(127);
  return s;
}

// Pairs a firing of level l writes (probe.py:97 learned, :127 merge), and
// the rows of its tiles.
inline int level_pairs(const FwdParams& p, int l) {
  return p.promotion == NGDN2_PROMOTION_MERGE ? TK : p.nq[l - 1];
}
inline int level_rows(const FwdParams& p, int l) {
  return l == 0 ? kC : pad_pairs(level_pairs(p, l));
}

// Steps of level l: chunks for level 0, firings otherwise (chunk.py:34-36).
inline int level_steps(const FwdParams& p, int l) {
  return l == 0 ? p.NT : p.NT / p.firing[l];
}

// Segments of a level, from a cost model of the three stages (per-step
// times measured on B200, microseconds): the compose runs 2 (segments - 1)
// CTAs per (batch, head) and the replay one per segment, each stepping
// through its segment's length (in ceil(CTAs / slots) waves, slots = 2 CTAs
// per SM for 64-row steps, 1 for 128); the combine steps once per segment
// in sequence. The count minimising compose + combine + replay is taken,
// with at least four steps per segment.
inline int level_nseg(const FwdParams& p, int l) {
  const int steps = level_steps(p, l);
  const int bh = p.B * p.H > 0 ? p.B * p.H : 1;
  const bool r64 = level_rows(p, l) == 64;
  const int slots = kSMs * (r64 ? 2 : 1);
  const double t_compose = r64 ? 3.4 : 2.9, t_replay = r64 ? 5.1 : 3.1, t_combine = 1.4;
  int best = 1;
  double best_t = 1e30;
  for (int n = 1; n <= (steps / 4 > 1 ? steps / 4 : 1); ++n) {
    const int len = (steps + n - 1) / n;
    const int64_t wc = (int64_t(2) * bh * (n - 1) + slots - 1) / slots;
    const int64_t wr = (int64_t(bh) * n + slots - 1) / slots;
    const double t = double(wc) * len * t_compose + double(n - 1) * t_combine +
                     double(wr) * len * t_replay;
    if (t < best_t) {
      best_t = t;
      best = n;
    }
  }
  return best;
}

struct SegLayout {
  TcLayout tc;                               // promotion operands and chunk records
  int nseg[NGDN2_MAX_LEVELS], seglen[NGDN2_MAX_LEVELS], nE[NGDN2_MAX_LEVELS];
  int64_t mz_off[NGDN2_MAX_LEVELS], start_off[NGDN2_MAX_LEVELS], E_off[NGDN2_MAX_LEVELS];
  int64_t prec_off[NGDN2_MAX_LEVELS];
  int64_t total;
};

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

inline SegLayout seg_layout(const FwdParams& p) {
  SegLayout s;
  memset(&s, 0, sizeof(s));
  const int64_t bh = int64_t(p.B) * p.H;
  s.tc.rec = TcRecord::make(1);
  s.tc.ptc_off = 0;
  int64_t off = int64_t(p.L > 1 ? p.L - 1 : 0) * p.H * PT_SIZE;
  s.tc.chunks_off = align256(off);
  off = s.tc.chunks_off + bh * p.NT * s.tc.rec.size;
  for (int l = 0; l < p.L; ++l) {
    const int steps = level_steps(p, l);
    const int n = level_nseg(p, l);
    s.nseg[l] = n;
    s.seglen[l] = (steps + n - 1) / n;
    if (s.seglen[l] > 0) s.nseg[l] = (steps + s.seglen[l] - 1) / s.seglen[l];
    if (s.nseg[l] < 1) s.nseg[l] = 1;
    // Emitted states: level 0 at level 1's firings; level l >= 1 after every
    // firing and at the start (the state entering each of its groups).
    s.nE[l] = l == 0 ? (p.L > 1 ? level_steps(p, 1) : 0) : steps + 1;
    s.mz_off[l] = align256(off);
    off = s.mz_off[l] + bh * (s.nseg[l] - 1) * kMzBytes;
    s.start_off[l] = align256(off);
    off = s.start_off[l] + (s.nseg[l] > 1 ? bh * s.nseg[l] * TK * TV * 4 : 0);
    s.E_off[l] = align256(off);
    off = s.E_off[l] + bh * s.nE[l] * kStateBytes;
    s.prec_off[l] = align256(off);
    if (l > 0) off = s.prec_off[l] + bh * steps * probe_rec(level_rows(p, l)).size;
  }
  s.total = align256(off);
  return s;
}

// fp32 [K][V] states kept between kernels (segment transitions Z, segment
// start states) use the lane-major layout of lm_off (tc_common.cuh).

__device__ __forceinline__ bool seg_gate_closed(const int32_t* status) {
  return status && (*reinterpret_cast<const volatile int32_t*>(status) & NGDN2_STATUS_GATE_TIMEOUT);
}

// ---------------------------------------------------------------------------
// seg_scan: compose (grid 2 (nseg - 1), H, B; even blocks M, odd blocks Z) or
// replay (grid nseg, H, B) of one level. 256 threads: warp w owns TMEM lane
// quarter (w & 3) and the 64 columns 64 (w >> 2).
// ---------------------------------------------------------------------------

struct SegScanArgs {
  int level, L, H, T;
  int nsteps, seglen, nseg;
  StepRec rec;
  const char* recs;              // [B][H][nsteps] records
  const float* init;             // [B][H][L][K][V] or null
  const float* starts;           // [B][H][nseg][K][V] (nseg > 1)
  char* mz;                      // [B][H][nseg - 1] compose outputs
  bf16* E;                       // [B][H][nE] emitted states
  int nE, emit_every;            // level 0: level 1's interval; levels: 0 (after every step)
  float* fin;                    // [B][H][L][K][V]
  int out;                       // 1: level 0's replay writes its output part to o
  void* o;                       // [B][T][H][V] (the read kernel adds the upper levels)
  int dtype;
  int32_t* status;
};

template <int ROWS>
__global__ void __launch_bounds__(kSegThreads, ROWS == 64 ? 2 : 1)
seg_scan_kernel(SegScanArgs a, int replay) {
  if (seg_gate_closed(a.status)) return;
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint64_t bar_a, bar_b, bar_mma;
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, c0 = 64 * (warp >> 2);
  const int h = blockIdx.y, b = blockIdx.z;
  const int mode = replay ? 2 : int(blockIdx.x & 1);  // 0: M, 1: Z, 2: replay
  const int s = replay ? int(blockIdx.x) : int(blockIdx.x >> 1);
  const int64_t bh = int64_t(b) * a.H + h;
  const int j0 = s * a.seglen;
  const int j1 = min(a.nsteps, j0 + a.seglen);
  const StepRec& R = a.rec;
  bf16* Xb = reinterpret_cast<bf16*>(sm);
  uint8_t* Rec = sm + kStateBytes;
  bf16* Yv = reinterpret_cast<bf16*>(Rec + R.smem);
  const char* rec0 = a.recs + bh * a.nsteps * R.size;
  const bool out = replay && a.out != 0;
  const bool last_seg = replay && j1 == a.nsteps;
  const int k = 32 * quarter + lane;  // state row of this thread

  if (warp == 0) tmem_alloc(&tbase, 256);
  if (tid == 0) {
    mbar_init(&bar_a, 1);
    mbar_init(&bar_b, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tX = tbase, tD = tbase + 128;

  auto load_a = [&](int j) {
    const char* src = rec0 + int64_t(j) * R.size;
    mbar_arrive_expect_tx(&bar_a, uint32_t(R.a_hi - R.a_lo));
    bulk_g2s(Rec + R.a_lo, src + R.a_lo, uint32_t(R.a_hi - R.a_lo), &bar_a);
  };
  auto load_b = [&](int j) {
    const char* src = rec0 + int64_t(j) * R.size;
    mbar_arrive_expect_tx(&bar_b, uint32_t(R.b_hi - R.b_lo));
    bulk_g2s(Rec + R.b_lo, src + R.b_lo, uint32_t(R.b_hi - R.b_lo), &bar_b);
  };
  if (tid == 0 && j0 < j1) {
    load_a(j0);
    load_b(j0);
  }
  // Y rows (E1 threads) and the row decay d[k] of a step, loaded a step ahead.
  const bool e1 = 32 * quarter < ROWS;
  uint4 yraw[8];
  auto fetch_y = [&](int j) {
    if (!e1 || mode == 0) return;
    const uint4* yg = reinterpret_cast<const uint4*>(rec0 + int64_t(j) * R.size + R.Y) +
                      (c0 / 8) * ROWS + k;
#pragma unroll
    for (int c = 0; c < 8; ++c) yraw[c] = __ldg(yg + c * ROWS);
  };
  auto fetch_d = [&](int j) {
    return __ldg(reinterpret_cast<const float*>(rec0 + int64_t(j) * R.size + R.d) + k);
  };

  // Start state: identity (M), zero (Z), or the state entering the segment.
  const float* src = nullptr;   // start state: segment starts lane-major, init row-major
  bool src_lm = false;
  if (mode == 2) {
    if (a.nseg > 1 && s > 0) {
      src = a.starts + (bh * a.nseg + s) * TK * TV;
      src_lm = true;
    } else if (a.init) {
      src = a.init + (bh * a.L + a.level) * TK * TV;
    }
  }
  float dcur = j0 < j1 ? fetch_d(j0) : 1.f;
  if (j0 < j1) fetch_y(j0);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int cc = c0 + 32 * hh;
    float x[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) x[t] = mode == 0 ? (k == cc + t ? 1.f : 0.f) : 0.f;
    if (src) {
#pragma unroll
      for (int t = 0; t < 32; t += 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + (src_lm ? lm_off(k, cc + t)
                                                                           : k * TV + cc + t));
        x[t] = v.x; x[t + 1] = v.y; x[t + 2] = v.z; x[t + 3] = v.w;
      }
    }
#pragma unroll
    for (int c = 0; c < 32; c += 8)
      *reinterpret_cast<uint4*>(Xb + mnmajor_off(k, cc + c, TK)) = pack8(x + c);
    if (last_seg && j0 >= j1) {
#pragma unroll
      for (int t = 0; t < 32; t += 4)
        *reinterpret_cast<float4*>(a.fin + ((bh * a.L + a.level) * TK + k) * TV + cc + t) =
            make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
    }
#pragma unroll
    for (int t = 0; t < 32; ++t) x[t] *= dcur;
    tmem_st32(taddr(tX, 32 * quarter, cc), x);
  }
  tmem_wait_st();
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  // An emitted state goes out by one bulk copy from Xb (every thread's
  // writes to it are fenced for the async proxy before the barrier that
  // precedes this); thread 0 waits for the copy to have read Xb before the
  // barrier after which Xb is rewritten (E1's). The state entering group 0
  // of an upper level is its start state.
  auto copy_out = [&](int slot) {
    if (tid == 0) {
      bulk_s2g(a.E + (bh * a.nE + slot) * (TK * TV), Xb, kStateBytes);
      bulk_commit();
    }
  };
  if (replay && a.emit_every == 0 && s == 0) copy_out(0);

  const uint32_t id_r = idesc_f16(128, 128, true, false, true);    // R . Xb (K-major A)
  const uint32_t id_p = idesc_f16(128, 128, true, true, true);     // P^T . Yv (MN-major A)
  uint32_t ph_a = 0, ph_b = 0, ph_mma = 0;
  // Level 0's output rows of a step are staged in Yv (free once MMA2 has
  // read it) as bf16 / fp16 rows with 16-byte chunks XOR-swizzled by row,
  // and copied out by all threads, a row per 16 lanes, during the next
  // step's MMA1 (or after the last step).
  uint8_t* Ys = reinterpret_cast<uint8_t*>(Yv);
  auto flush_out = [&](int jj) {
#pragma unroll
    for (int r = 0; r < kC * 16 / kSegThreads; ++r) {
      const int e = tid + kSegThreads * r, row = e >> 4, ch = e & 15, t = jj * kC + row;
      if (t < a.T)
        reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.o) +
                                 ((int64_t(b) * a.T + t) * a.H + h) * TV)[ch] =
            *reinterpret_cast<const uint4*>(Ys + row * 256 + ((ch ^ (row & 15)) << 4));
    }
  };
  int pend = -1;  // step whose output rows wait in Yv
  for (int j = j0; j < j1; ++j) {
    // MMA1: R . X (rows of R in lanes 0 .. ROWS - 1; for level 0 with its
    // output, the read queries Q follow W, so Q . X lands in lanes 64..127).
    if (tid == 0) {
      if (!mbar_wait(&bar_a, ph_a)) abort_flag = 1;
      fence_after_sync();
      mma_tile(tD, smem_u32(Rec + R.R), smem_u32(Xb), TK, id_r, false);
      mma_commit(&bar_mma);
    }
    ph_a ^= 1;
    const float dnext = j + 1 < j1 ? fetch_d(j + 1) : 1.f;
    __syncwarp();
    if (pend >= 0) {
      // (E1 below overwrites Yv.)
      flush_out(pend);
      pend = -1;
      __syncthreads();
    }
    if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
    ph_mma ^= 1;
    fence_after_sync();
    // E1: Yv = Y - R . X -> bf16 MN-major B operand [Kd = ROWS][N = V].
    if (e1) {
      // Both column halves in one TMEM round trip.
      uint32_t raw[64];
      tmem_ld32_nowait(taddr(tD, 32 * quarter, c0), raw);
      tmem_ld32_nowait(taddr(tD, 32 * quarter, c0 + 32), raw + 32);
      tmem_wait_ld();
      tmem_regs_after_wait32(raw);
      tmem_regs_after_wait32(raw + 32);
      const float* x = reinterpret_cast<const float*>(raw);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float y[8];
        if (mode == 0) {
#pragma unroll
          for (int t = 0; t < 8; ++t) y[t] = -x[8 * c + t];
        } else {
          unpack8(yraw[c], NGDN2_BF16, y);
#pragma unroll
          for (int t = 0; t < 8; ++t) y[t] -= x[8 * c + t];
        }
        *reinterpret_cast<uint4*>(Yv + mnmajor_off(k, c0 + 8 * c, ROWS)) = pack8(y);
      }
    }
    if (tid == 0) bulk_wait_read0();  // (E2 below rewrites Xb)
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (abort_flag) break;
    // R (and, for level 0 with its output, Q) are spent: the next record's
    // first part streams in. (Issued after the barrier, which the thread
    // that waits on bar_a passed after its wait.)
    if (tid == 32 && j + 1 < j1) load_a(j + 1);
    // MMA2: X += P^T . Yv (X was scaled by d when it was last written), and
    // for level 0's output the intra-chunk part A . v_new onto Q . X.
    if (tid == 0) {
      if (!mbar_wait(&bar_b, ph_b)) abort_flag = 1;
      fence_after_sync();
      mma_tile(tX, smem_u32(Rec + R.P), smem_u32(Yv), ROWS, id_p, true);
      if (out) mma_tile(tD, smem_u32(Rec + R.A - TILE_A), smem_u32(Yv), kC, id_r, true);
      mma_commit(&bar_mma);
    }
    ph_b ^= 1;
    if (j + 1 < j1) fetch_y(j + 1);
    __syncwarp();
    if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
    ph_mma ^= 1;
    fence_after_sync();
    if (tid == 32 && j + 1 < j1) load_b(j + 1);

    // E2: the new state -> bf16 copy (next MMA1's operand, and the emitted
    // copy), fp32 final / compose outputs at the segment's end, then the
    // TMEM state scaled by the next step's d. Level 0's output rows (lanes
    // 64..127 of tD) go out as well.
    const bool seg_end = j + 1 == j1;
    {
      // Both column halves of the state in one TMEM round trip.
      uint32_t raw[64];
      tmem_ld32_nowait(taddr(tX, 32 * quarter, c0), raw);
      tmem_ld32_nowait(taddr(tX, 32 * quarter, c0 + 32), raw + 32);
      tmem_wait_ld();
      tmem_regs_after_wait32(raw);
      tmem_regs_after_wait32(raw + 32);
      float* x = reinterpret_cast<float*>(raw);
#pragma unroll
      for (int c = 0; c < 64; c += 8)
        *reinterpret_cast<uint4*>(Xb + mnmajor_off(k, c0 + c, TK)) = pack8(x + c);
      if (seg_end && last_seg) {
#pragma unroll
        for (int t = 0; t < 64; t += 4)
          *reinterpret_cast<float4*>(a.fin + ((bh * a.L + a.level) * TK + k) * TV + c0 + t) =
              make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
      }
      if (seg_end && mode == 0) {
        // M as two bf16 halves in the K-major A layout of the combine.
        bf16* mh = reinterpret_cast<bf16*>(a.mz + (bh * (a.nseg - 1) + s) * int64_t(kMzBytes));
        bf16* ml = mh + TK * TV;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          float hi[8], lo[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            hi[t] = __bfloat162float(__float2bfloat16_rn(x[c + t]));
            lo[t] = x[c + t] - hi[t];
          }
          *reinterpret_cast<uint4*>(mh + kmajor_off(k, c0 + c, TK)) = pack8(hi);
          *reinterpret_cast<uint4*>(ml + kmajor_off(k, c0 + c, TK)) = pack8(lo);
        }
      }
      if (seg_end && mode == 1) {
        float* z = reinterpret_cast<float*>(a.mz + (bh * (a.nseg - 1) + s) * int64_t(kMzBytes) +
                                            2 * kStateBytes);
#pragma unroll
        for (int t = 0; t < 64; t += 4)
          *reinterpret_cast<float4*>(z + lm_off(k, c0 + t)) = make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
      }
      if (!seg_end) {
#pragma unroll
        for (int t = 0; t < 64; ++t) x[t] *= dnext;
        tmem_st32(taddr(tX, 32 * quarter, c0), x);
        tmem_st32(taddr(tX, 32 * quarter, c0 + 32), x + 32);
      }
    }
    if (out && quarter >= 2) {
      // Level 0's output rows, both column halves in one round trip.
      const int i = 32 * (quarter - 2) + lane, t = j * kC + i;
      uint32_t raw[64];
      tmem_ld32_nowait(taddr(tD, 32 * quarter, c0), raw);
      tmem_ld32_nowait(taddr(tD, 32 * quarter, c0 + 32), raw + 32);
      tmem_wait_ld();
      tmem_regs_after_wait32(raw);
      tmem_regs_after_wait32(raw + 32);
      const float* y = reinterpret_cast<const float*>(raw);
      (void)t;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<uint4*>(Ys + i * 256 + ((((c0 >> 3) + u) ^ (i & 15)) << 4)) =
            a.dtype == NGDN2_BF16 ? pack8(y + 8 * u) : pack8h(y + 8 * u);
    }
    if (out) pend = j;
    tmem_wait_st();
    dcur = dnext;
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (replay) {
      int slot = -1;
      if (a.emit_every == 0) slot = j + 1;
      else if ((j + 1) % a.emit_every == 0 && (j + 1) / a.emit_every - 1 < a.nE)
        slot = (j + 1) / a.emit_every - 1;
      if (slot >= 0) copy_out(slot);
    }
  }
  if (pend >= 0 && !abort_flag) flush_out(pend);
  if (tid == 0) bulk_wait0();
  if (abort_flag && tid == 0 && a.status) atomicOr(a.status, NGDN2_STATUS_WAIT_TIMEOUT);
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// ---------------------------------------------------------------------------
// seg_combine: grid (kCombineSplit, H, B), 256 threads. The state entering
// each segment of one level: S_{s+1} = M_s S_s + Z_s. The value columns of
// S evolve independently under the same M_s, so each CTA owns
// kCombineCols of them. M_s and the slice of S_s are each split into two
// bf16 halves, and three products keep ~16 bits: M_hi . [S_hi | S_lo] as
// one N = 32 product (M_hi read from shared memory once) and M_lo . S_hi
// (N = 16), fp32 in TMEM; the epilogue sums the three with Z_s. Each MMA
// instruction takes about 50 cycles whatever its N or operand source, so a
// step issues as few as the split allows (16), and the columns are split
// eight ways to shorten the epilogue. M_s streams into shared memory
// kCombineBufs - 1 steps ahead of use (the next copy is issued after the
// step's MMAs). Warp w owns row k = 32 (w & 3) + i (its TMEM lane quarter)
// and 8 of the 16 columns (w >> 2). Off the chain, while a step's MMAs run,
// each thread stores the previous step's state to the segment starts and
// loads its part of Z_{s+1}.
// ---------------------------------------------------------------------------

constexpr int kCombineSplit = 8;
constexpr int kCombineCols = TV / kCombineSplit;   // 16
constexpr int kCombineThreads = 256;
constexpr int kCombineHalf = kCombineCols / 2;    // columns per thread
constexpr int kCombineBufs = 3;
constexpr int kCombineSliceBytes = TK * kCombineCols * 2;
constexpr int kCombineSmem = kCombineBufs * 2 * kStateBytes + 2 * kCombineSliceBytes;

__global__ void __launch_bounds__(kCombineThreads, 1)
seg_combine_kernel(const char* mz, const float* init, float* starts, int L, int level, int H,
                   int nseg, int32_t* status) {
  if (seg_gate_closed(status)) return;
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint64_t bar_ld[kCombineBufs], bar_mma;
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, quarter = warp & 3;
  const int cq = kCombineHalf * (warp >> 2);   // this thread's columns within the slice
  const int v0 = blockIdx.x * kCombineCols, h = blockIdx.y, b = blockIdx.z;
  const int64_t bh = int64_t(b) * H + h;
  const int k = 32 * quarter + (tid & 31);
  // M buffers (hi, lo each), then the slice's hi and lo halves as one N = 32
  // MN-major B operand (hi in its rows 0..15, lo in 16..31).
  bf16* Shi = reinterpret_cast<bf16*>(sm + kCombineBufs * 2 * kStateBytes);
  bf16* Slo = Shi + TK * kCombineCols;
  const char* mz0 = mz + bh * (nseg - 1) * int64_t(kMzBytes);
  const int nsteps = nseg - 1;

  if (warp == 0) tmem_alloc(&tbase, 64);
  int issued = 0;  // (thread 0) M loads issued
  auto load_m = [&](int s) {
    ++issued;
    uint64_t* bar = &bar_ld[s % kCombineBufs];
    mbar_arrive_expect_tx(bar, 2 * kStateBytes);
    bulk_g2s(sm + (s % kCombineBufs) * 2 * kStateBytes, mz0 + s * int64_t(kMzBytes),
             2 * kStateBytes, bar);
  };
  if (tid == 0) {
    for (int i = 0; i < kCombineBufs; ++i) mbar_init(&bar_ld[i], 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
    abort_flag = 0;
    for (int s = 0; s < kCombineBufs - 1 && s < nsteps; ++s) load_m(s);
  }
  auto put_state = [&](const float* x) {
    float hi[kCombineHalf], lo[kCombineHalf];
#pragma unroll
    for (int t = 0; t < kCombineHalf; ++t) {
      hi[t] = __bfloat162float(__float2bfloat16_rn(x[t]));
      lo[t] = x[t] - hi[t];
    }
    *reinterpret_cast<uint4*>(Shi + mnmajor_off(k, cq, TK)) = pack8(hi);
    *reinterpret_cast<uint4*>(Slo + mnmajor_off(k, cq, TK)) = pack8(lo);
  };
  // This thread's part of row k of the slice of Z_s.
  auto fetch_z = [&](int s, float4* z4) {
    const float* z = reinterpret_cast<const float*>(mz0 + s * int64_t(kMzBytes) + 2 * kStateBytes);
#pragma unroll
    for (int t = 0; t < kCombineHalf / 4; ++t)
      z4[t] = *reinterpret_cast<const float4*>(z + lm_off(k, v0 + cq + 4 * t));
  };
  auto store_start = [&](int s, const float* x) {
    float* dst = starts + (bh * nseg + s) * TK * TV;
#pragma unroll
    for (int t = 0; t < kCombineHalf; t += 4)
      *reinterpret_cast<float4*>(dst + lm_off(k, v0 + cq + t)) =
          make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
  };
  float4 zc[kCombineHalf / 4], zn[kCombineHalf / 4];
  float x[kCombineHalf];
  // S_0: the level's initial state (or zero).
#pragma unroll
  for (int t = 0; t < kCombineHalf; ++t)
    x[t] = init ? init[((bh * L + level) * TK + k) * TV + v0 + cq + t] : 0.f;
  put_state(x);
  if (nsteps > 0) fetch_z(0, zc);
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tb = tbase;
  // TMEM: [hi.hi | hi.lo] in columns 0..31, lo.hi in 32..47.
  const uint32_t id_hh = idesc_f16(128, 2 * kCombineCols, true, false, true);
  const uint32_t id_lh = idesc_f16(128, kCombineCols, true, false, true);
  // Descriptors of K step 0; K step kk adds 256 bytes (16 in the address field).
  const uint64_t d_s = desc_tile(smem_u32(Shi), TK, 0);
  const uint64_t d_m0 = desc_tile(smem_u32(sm), TK, 0);
  uint32_t ph_mma = 0;
  int landed = 0;  // (thread 0) M loads waited for
  for (int s = 0; s < nsteps; ++s) {
    if (tid == 0) {
      if (mbar_wait(&bar_ld[s % kCombineBufs], (s / kCombineBufs) & 1)) {
        ++landed;
        fence_after_sync();
        const uint64_t d_hi = d_m0 + uint64_t((s % kCombineBufs) * 2 * kStateBytes) / 16;
        const uint64_t d_lo = d_hi + kStateBytes / 16;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
          mma_f16(tb, d_hi + 16 * kk, d_s + 16 * kk, id_hh, kk > 0 ? 1u : 0u);
          mma_f16(tb + 2 * kCombineCols, d_lo + 16 * kk, d_s + 16 * kk, id_lh, kk > 0 ? 1u : 0u);
        }
      } else {
        abort_flag = 1;
      }
      // (With no MMA issued the commit arrives at once.)
      mma_commit(&bar_mma);
      // (Buffer (s - 1) mod kCombineBufs was last read by step s - 1's
      // MMAs, complete.)
      if (s + kCombineBufs - 1 < nsteps) load_m(s + kCombineBufs - 1);
    }
    __syncwarp();
    // Off the chain: S_s (s >= 1) to the segment starts, Z_{s+1} in.
    if (s > 0) store_start(s, x);
    if (s + 1 < nsteps) fetch_z(s + 1, zn);
    if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
    ph_mma ^= 1;
    fence_after_sync();
    {
      uint32_t r0[kCombineHalf], r1[kCombineHalf], r2[kCombineHalf];
      tmem_ld8_nowait(taddr(tb, 32 * quarter, cq), r0);
      tmem_ld8_nowait(taddr(tb + kCombineCols, 32 * quarter, cq), r1);
      tmem_ld8_nowait(taddr(tb + 2 * kCombineCols, 32 * quarter, cq), r2);
      tmem_wait_ld();
      tmem_regs_after_wait8(r0);
      tmem_regs_after_wait8(r1);
      tmem_regs_after_wait8(r2);
#pragma unroll
      for (int t = 0; t < kCombineHalf / 4; ++t) {
        const float z[4] = {zc[t].x, zc[t].y, zc[t].z, zc[t].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          x[4 * t + e] = (__uint_as_float(r0[4 * t + e]) + z[e]) +
                         (__uint_as_float(r1[4 * t + e]) + __uint_as_float(r2[4 * t + e]));
      }
    }
    put_state(x);
#pragma unroll
    for (int t = 0; t < kCombineHalf / 4; ++t) zc[t] = zn[t];
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (abort_flag) break;
  }
  if (nsteps > 0 && !abort_flag) store_start(nsteps, x);
  if (abort_flag && tid == 0) {
    // Copies still in flight land before the CTA's shared memory is released.
    for (int c = landed; c < issued; ++c)
      if (!mbar_wait(&bar_ld[c % kCombineBufs], (c / kCombineBufs) & 1)) break;
    if (status) atomicOr(status, NGDN2_STATUS_WAIT_TIMEOUT);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 64);
}

// ---------------------------------------------------------------------------
// seg_probe: grid (NF_l, H, B), 512 threads. One firing of level l: probe
// level l - 1's emitted state (probe.py:69-102 learned, :105-136 merge, with
// the gates of :34-66) and write the firing's step record.
// ---------------------------------------------------------------------------

struct ProbeArgs {
  int level, H, nf, f_here, f_below, nE_below;
  const bf16* E_below;      // [B][H][nE_below] states of level l - 1
  int below_is_level0;      // level 0 emits only at level 1's firings
  const char* ptc;          // promotion operands of this level, [H][PT_SIZE]
  char* recs;               // [B][H][nf] records
  StepRec rec;
  int nq, learned;
  int32_t* status;
};

// Probe scratch after the state: [W_w | W_g] (64 KB), the bank then V' (up
// to 32 KB), [W_k^T | W_b] (64 KB). Both weight blocks arrive with the
// first copies, so the second gate product waits on no load; the gate
// partials (fp16) go over the state once P1 has read it.
constexpr int kProbeW2A = 65536 + 32768;
constexpr int kProbeScratch = kProbeW2A + 65536;

__global__ void __launch_bounds__(kProbeThreads, 1) seg_probe_kernel(ProbeArgs a) {
  if (seg_gate_closed(a.status)) return;
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint64_t bar_ld, bar_mma;
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  __shared__ float egp[128];
  __shared__ float red[512];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, c0 = 32 * (warp >> 2);
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t bh = int64_t(b) * a.H + h;
  const int nq = a.nq, mp = a.rec.rows;
  bf16* Sbf = reinterpret_cast<bf16*>(sm);
  uint8_t* X = sm + kStateBytes;
  bf16* XW = reinterpret_cast<bf16*>(X);
  bf16* XQ = reinterpret_cast<bf16*>(X + 65536);
  bf16* XW2 = reinterpret_cast<bf16*>(X + kProbeW2A);
  const char* pt = a.ptc + int64_t(h) * PT_SIZE;
  // The level below's state after its firings up to this one
  // (chunk.py:39-55): group ((i + 1) f_l) // f_{l-1} of the level below.
  const int src = a.below_is_level0 ? i : ((i + 1) * a.f_here) / a.f_below;
  const bf16* S_src = a.E_below + (bh * a.nE_below + src) * (TK * TV);
  char* rec = a.recs + (bh * a.nf + i) * a.rec.size;

  if (warp == 0) tmem_alloc(&tbase, 512);
  if (tid == 0) {
    mbar_init(&bar_ld, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
    abort_flag = 0;
    const uint32_t bytes = kStateBytes + 2 * 65536 + (a.learned ? mp * 256 : 0);
    mbar_arrive_expect_tx(&bar_ld, bytes);
    bulk_g2s(Sbf, S_src, kStateBytes, &bar_ld);
    bulk_g2s(XW, pt + PT_W2B, 65536u, &bar_ld);
    bulk_g2s(XW2, pt + PT_W2A, 65536u, &bar_ld);
    if (a.learned) bulk_g2s(XQ, pt + PT_QB, uint32_t(mp * 256), &bar_ld);
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tb = tbase, tV = tb + 128, tG = tb + 256;
  const bool split = mp == 64;
  const int row = (mp == 128) ? 32 * quarter + lane : (lane < 16 ? 16 * quarter + lane : -1);
  const uint32_t id_read = idesc_f16(mp, 128, true, false, true);
  const uint32_t id_gate = idesc_f16(mp, 256, true, false, false);
  const uint32_t id_half = idesc_f16(64, 128, true, false, false);
  uint32_t ph_ld = 0, ph_mma = 0;
  if (!mbar_wait(&bar_ld, ph_ld)) abort_flag = 1;
  ph_ld ^= 1;
  if (a.learned) {
    // P1: V' = Q_bank . S_{l-1} (probe.py:97-98)
    if (tid == 0) {
      fence_after_sync();
      mma_tile(tV, smem_u32(XQ), smem_u32(Sbf), TK, id_read, false);
      mma_commit(&bar_mma);
    }
    __syncwarp();
    if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
    ph_mma ^= 1;
    fence_after_sync();
    float x[32];
    tmem_ld32(taddr(tV, 32 * quarter, c0), x);
    if (row >= 0) {
#pragma unroll
      for (int c = 0; c < 32; c += 8)
        *reinterpret_cast<uint4*>(XQ + kmajor_off(row, c0 + c, TV)) = pack8(x + c);
    }
  } else {
    // Merge (probe.py:127-136): the values are the rows of S_{l-1}; V' as
    // the K-major A operand and, in fp32, in TMEM.
    const int kk = 32 * quarter + lane;
    float x[32];
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      float f[8];
      const uint4 raw = *reinterpret_cast<const uint4*>(Sbf + mnmajor_off(kk, c0 + c, TK));
      unpack8(raw, NGDN2_BF16, f);
      *reinterpret_cast<uint4*>(XQ + kmajor_off(kk, c0 + c, TV)) = raw;
#pragma unroll
      for (int t = 0; t < 8; ++t) x[c + t] = f[t];
    }
    tmem_st32(taddr(tV, 32 * quarter, c0), x);
    tmem_wait_st();
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  // P2b: [w_logit | g_logit] = V' . [W_w | W_g] (probe.py:60-62)
  if (tid == 0) {
    fence_after_sync();
    if (split) {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_half, false);
      mma_tile(tG + (16u << 16), smem_u32(XQ), smem_u32(XW + 128 * 128), TV, id_half, false);
    } else {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW), TV, id_gate, false);
    }
    mma_commit(&bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  // w = sigmoid(w_logit) into v * w (TMEM); -softplus(g_logit - 4) per pair
  // into shared memory as fp16 pairs (probe.py:63-65), over the state.
  uint32_t* gpart16 = reinterpret_cast<uint32_t*>(Sbf);
  {
    float av[32], vp[32];
    if (split) {
      tmem_ld32(taddr(tG, 32 * quarter, c0), av);
      const bool hi = lane >= 16;
      const int gr = 16 * quarter + (lane & 15), cb = c0 + (hi ? 16 : 0);
      float sw[16];
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        float gg[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float mine_w = hi ? 0.f : av[j + e], mine_g = hi ? av[16 + j + e] : 0.f;
          const float got = __shfl_xor_sync(0xffffffffu, hi ? av[j + e] : av[16 + j + e], 16);
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
      tmem_st32(taddr(tV, 32 * quarter, c0), vp);
    } else {
      tmem_ld32(taddr(tV, 32 * quarter, c0), vp);
      tmem_ld32(taddr(tG, 32 * quarter, c0), av);
#pragma unroll
      for (int u = 0; u < 32; ++u) vp[u] *= sigmoid_tanh(av[u] + kWLogitInit);
      tmem_st32(taddr(tV, 32 * quarter, c0), vp);
      tmem_ld32(taddr(tG, 32 * quarter, 128 + c0), av);
#pragma unroll
      for (int u = 0; u < 32; u += 2) {
        const __half2 g2 = __floats2half2_rn(-softplus_fast(av[u] + kGLogitInit),
                                             -softplus_fast(av[u + 1] + kGLogitInit));
        gpart16[row * 64 + (((c0 + u) >> 1) ^ (row & 31))] = *reinterpret_cast<const uint32_t*>(&g2);
      }
    }
  }
  tmem_wait_st();
  __syncthreads();
  {
    const int kk = tid & 127, qq = tid >> 7, r0 = qq * (nq >> 2), r1 = r0 + (nq >> 2);
    float sum = 0.f;
    const __half* g16 = reinterpret_cast<const __half*>(gpart16);
    for (int r = r0; r < r1; ++r) sum += __half2float(g16[2 * (r * 64 + ((kk >> 1) ^ (r & 31))) + (kk & 1)]);
    red[qq * 128 + kk] = sum;
  }
  __syncthreads();
  if (tid < 128)
    egp[tid] = expf((red[tid] + red[128 + tid] + red[256 + tid] + red[384 + tid]) / float(nq));
  fence_proxy_async();
  __syncthreads();
  // P2a: [u | b_logit] = V' . [W_k^T | W_b] (probe.py:60, :99)
  if (tid == 0) {
    fence_after_sync();
    if (split) {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW2), TV, id_half, false);
      mma_tile(tG + (16u << 16), smem_u32(XQ), smem_u32(XW2 + 128 * 128), TV, id_half, false);
    } else {
      mma_tile(tG, smem_u32(XQ), smem_u32(XW2), TV, id_gate, false);
    }
    mma_commit(&bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(&bar_mma, ph_mma)) abort_flag = 1;
  ph_mma ^= 1;
  fence_after_sync();
  bf16* keysT = XW;              // P: MN-major [Kd = mp][M = K]
  bf16* kbg = XW + 16384;        // R: K-major [mp x K]
  if (a.learned) {
    // keys = u / max(|u|, 1e-12) (probe.py:100)
    {
      float u[32];
      tmem_ld32(taddr(tG, 32 * quarter, c0), u);
      float ss = 0.f;
#pragma unroll
      for (int t = 0; t < 32; ++t) ss = fmaf(u[t], u[t], ss);
      if (row >= 0 && (!split || lane < 16)) red[(warp >> 2) * 128 + row] = ss;
    }
    __syncthreads();
    const float inv =
        row >= 0 ? __fdividef(1.f, fmaxf(sqrtf(red[row] + red[128 + row] + red[256 + row] +
                                               red[384 + row]), 1e-12f))
                 : 0.f;
    if (split) {
      const bool hi = lane >= 16;
      const int pr = 16 * quarter + (lane & 15), cb = c0 + (hi ? 16 : 0);
      const float iv = __shfl_sync(0xffffffffu, inv, lane & 15);
      float x0[16], x1[16];
      tmem_ld16(taddr(tG, 32 * quarter, c0), x0);
      tmem_ld16(taddr(tG, 32 * quarter, c0 + 16), x1);
#pragma unroll
      for (int c = 0; c < 16; c += 8) {
        float kk8[8], kb[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int j = c + t;
          const float got = __shfl_xor_sync(0xffffffffu, hi ? x0[j] : x1[j], 16);
          const float uu = hi ? got : x0[j], bb = hi ? x1[j] : got;
          kk8[t] = uu * iv;
          kb[t] = kk8[t] * (fast_sigmoid(bb + kBLogitInit) * egp[cb + j]);
        }
        *reinterpret_cast<uint4*>(keysT + mnmajor_off(pr, cb + c, mp)) = pack8(kk8);
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
        float kk8[8], kb[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          kk8[t] = u[c + t] * inv;
          kb[t] = kk8[t] * bl[c + t];
        }
        *reinterpret_cast<uint4*>(keysT + mnmajor_off(row, c0 + c, mp)) = pack8(kk8);
        *reinterpret_cast<uint4*>(kbg + kmajor_off(row, c0 + c, TK)) = pack8(kb);
      }
    }
  } else {
    // Merge: identity keys (probe.py:133-136), so P = I and R = diag(b e^g).
    float bl[32];
    tmem_ld32(taddr(tG, 32 * quarter, 128 + c0), bl);
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      float kk8[8], kb[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int col = c0 + c + t;
        kk8[t] = col == row ? 1.f : 0.f;
        kb[t] = col == row ? fast_sigmoid(bl[c + t] + kBLogitInit) * egp[col] : 0.f;
      }
      *reinterpret_cast<uint4*>(keysT + mnmajor_off(row, c0 + c, mp)) = pack8(kk8);
      *reinterpret_cast<uint4*>(kbg + kmajor_off(row, c0 + c, TK)) = pack8(kb);
    }
  }
  // Y = v * w rows from TMEM: [V / 8][mp][8] pieces.
  {
    float vw[32];
    tmem_ld32(taddr(tV, 32 * quarter, c0), vw);  // warp-collective: every lane loads
    if (row >= 0) {
      uint4* yg = reinterpret_cast<uint4*>(rec + a.rec.Y);
#pragma unroll
      for (int c = 0; c < 32; c += 8) yg[((c0 + c) / 8) * mp + row] = pack8(vw + c);
    }
  }
  if (tid < TK) reinterpret_cast<float*>(rec + a.rec.d)[tid] = egp[tid];
  __syncthreads();
  // R and P tiles to the record.
  {
    const uint4* r_s = reinterpret_cast<const uint4*>(kbg);
    const uint4* p_s = reinterpret_cast<const uint4*>(keysT);
    uint4* r_g = reinterpret_cast<uint4*>(rec + a.rec.R);
    uint4* p_g = reinterpret_cast<uint4*>(rec + a.rec.P);
    for (int e = tid; e < mp * 16; e += kProbeThreads) {
      r_g[e] = r_s[e];
      p_g[e] = p_s[e];
    }
  }
  if (abort_flag && tid == 0 && a.status) atomicOr(a.status, NGDN2_STATUS_WAIT_TIMEOUT);
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 512);
}

// ---------------------------------------------------------------------------
// seg_read: persistent, one CTA per SM, 8 consumer warps + 1 producer warp.
// Adds the upper levels' reads sum_{l >= 1} mix_l scale (q_l . S_l) to the
// level-0 output that level 0's replay left in o (chunk.py:129-156,
// naive.py:382-390). A job is a unit of up to four chunks of one (batch,
// head); the unit size divides every upper level's firing interval, so its
// chunks read the same state of each level (the one entering their group).
// A CTA walks its jobs (blockIdx.x, + gridDim.x, ...) level by level: the
// producer streams each (job, level) item's state and query tiles (TMA,
// 128-byte swizzle) into one of two shared-memory stages as soon as the MMAs
// of the stage's previous item have read it, across job boundaries; the
// consumers scale the query rows by mix_l scale in place, one thread issues
// one M = 128 MMA per chunk (the tile in the tile's lower half, as in the
// fused scan's reads) accumulating into that chunk's TMEM accumulator, so
// the levels sum on the tensor cores, and the epilogue adds one accumulator
// per chunk to o while the next job's first items load.
// ---------------------------------------------------------------------------

constexpr int kReadUnit = 4;
constexpr int kReadStage = kStateBytes + kReadUnit * TILE_QK;

struct ReadArgs {
  int B, T, H, L, NT, unit;
  int firing[NGDN2_MAX_LEVELS];
  const bf16* E[NGDN2_MAX_LEVELS];
  int nE[NGDN2_MAX_LEVELS];
  QView q;
  TokView mix;
  float scale;
  void* o;
  int dtype;
  int hl_mode;
  int32_t* status;
};

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kReadThreads) : "memory");
}

__global__ void __launch_bounds__(kReadThreads + 32, 1)
seg_read_kernel(ReadArgs a, const __grid_constant__ CUtensorMap qmap) {
  if (seg_gate_closed(a.status)) return;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  __shared__ uint64_t bar_full[2], bar_free[2], bar_done, bar_fin;
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, c0 = 64 * ((warp >> 2) & 1);
  uint8_t* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  const bool q_tma = a.hl_mode != 2;
  const int nlev = a.L - 1;
  const int units = (a.NT + a.unit - 1) / a.unit;
  const int64_t njobs = int64_t(a.B) * a.H * units;
  // This CTA's jobs: blockIdx.x, + gridDim.x, ...; items = (job, level).
  const int64_t my_jobs =
      njobs > blockIdx.x ? (njobs - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nitems = my_jobs * nlev;

  if (warp == 0) tmem_alloc(&tbase, 512);
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_free[i], 1);
    }
    mbar_init(&bar_done, 1);
    mbar_init(&bar_fin, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tb = tbase;

  if (warp == kReadThreads / 32) {
    // Producer warp: item it's state and query tiles into stage it & 1, once
    // the MMAs of item it - 2 (the stage's previous use) have read it.
    if (lane == 0) {
      int64_t it = 0;
      for (; it < nitems; ++it) {
        const int st = int(it & 1);
        if (it >= 2 && !mbar_wait(&bar_free[st], uint32_t(((it - 2) >> 1) & 1))) {
          abort_flag = 1;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&abort_flag)) break;
        const int64_t job = blockIdx.x + (it / nlev) * gridDim.x;
        const int l = int(it % nlev) + 1;
        const int64_t bh = job / units;
        const int b = int(bh / a.H), h = int(bh % a.H);
        const int n0 = int(job % units) * a.unit;
        const int nc = min(a.unit, a.NT - n0);
        uint8_t* base = sm + st * kReadStage;
        uint64_t* bar = &bar_full[st];
        mbar_arrive_expect_tx(bar, uint32_t(kStateBytes + (q_tma ? nc * TILE_QK : 0)));
        bulk_g2s(base, a.E[l] + (bh * a.nE[l] + n0 / a.firing[l]) * (TK * TV), kStateBytes, bar);
        if (q_tma)
          for (int c = 0; c < nc; ++c)
            tma_load_4d(base + kStateBytes + c * TILE_QK, &qmap, 0, b * a.T + (n0 + c) * kC, 0,
                        a.hl_mode ? l * a.H + h : h * a.L + l, bar);
      }
      // Copies still in flight land before the CTA's shared memory is
      // released (each stage has at most one outstanding).
      for (int64_t j = it - 2 > 0 ? it - 2 : 0; j < it; ++j)
        if (!mbar_wait(&bar_full[j & 1], uint32_t((j >> 1) & 1))) break;
    }
  } else {
    const uint32_t id = idesc_f16(128, 128, true, false, true);
    for (int64_t jj = 0; jj < my_jobs; ++jj) {
      const int64_t job = blockIdx.x + jj * gridDim.x;
      const int64_t bh = job / units;
      const int b = int(bh / a.H), h = int(bh % a.H);
      const int n0 = int(job % units) * a.unit;
      const int nc = min(a.unit, a.NT - n0);
      for (int li = 0; li < nlev; ++li) {
        const int64_t it = jj * nlev + li;
        const int l = li + 1, st = int(it & 1);
        uint8_t* base = sm + st * kReadStage;
        if (!mbar_wait(&bar_full[st], uint32_t((it >> 1) & 1))) abort_flag = 1;
        // Row r of chunk c scaled by mix_l scale (zero past T), as bf16 (fp16
        // q converted; q without a tensor map read here with plain loads).
        {
          const int r = tid & 63, c = tid >> 6;
          if (c < nc) {
            const int t = (n0 + c) * kC + r;
            const float m =
                t < a.T ? load_elem(a.mix.p, a.mix.off(b, t, h, l), a.mix.dt) * a.scale : 0.f;
            uint8_t* tile = base + kStateBytes + c * TILE_QK;
#pragma unroll 4
            for (int u = 0; u < 16; ++u) {
              uint4* q8 = reinterpret_cast<uint4*>(tile + sw128_off(r, 8 * u));
              const uint4 raw =
                  q_tma ? *q8
                        : t < a.T ? raw8_at(a.q.p, a.q.dt, a.q.off(b, t, h, l, 8 * u), a.q.sd)
                                  : make_uint4(0u, 0u, 0u, 0u);
              float f[8];
              unpack8(raw, a.q.dt, f);
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] *= m;
              *q8 = pack8(f);
            }
          }
        }
        fence_proxy_async();
        fence_before_sync();
        consumers_sync();
        fence_after_sync();
        if (tid == 0) {
          for (int c = 0; c < nc; ++c)
            mma_tile_sw128_lo(tb + 128 * c, smem_u32(base + kStateBytes + c * TILE_QK),
                              smem_u32(base), id, li > 0);
          mma_commit(&bar_free[st]);
          if (li == nlev - 1) mma_commit(&bar_done);
        }
        __syncwarp();
      }
      // The job's MMAs complete; its accumulators go to o. Row i's 64
      // columns of o for chunk c + 1 are loaded while chunk c is formed (the
      // first chunk's before the wait), so the loads' latency overlaps.
      const int i = 32 * (quarter - 2) + lane;
      auto o_row = [&](int c) {
        const int t = (n0 + c) * kC + i;
        return t < a.T ? reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.o) +
                                                  ((int64_t(b) * a.T + t) * a.H + h) * TV + c0)
                       : nullptr;
      };
      uint4 ob[2][8];
      if (quarter >= 2) {
        const uint4* src = o_row(0);
#pragma unroll
        for (int u = 0; u < 8; ++u) ob[0][u] = src ? src[u] : make_uint4(0u, 0u, 0u, 0u);
      }
      if (!mbar_wait(&bar_done, uint32_t(jj & 1))) abort_flag = 1;
      fence_after_sync();
      if (quarter >= 2) {
#pragma unroll
        for (int c = 0; c < kReadUnit; ++c) {
          if (c < nc) {
            if (c + 1 < nc) {
              const uint4* src = o_row(c + 1);
#pragma unroll
              for (int u = 0; u < 8; ++u) ob[(c + 1) & 1][u] = src ? src[u] : make_uint4(0u, 0u, 0u, 0u);
            }
            uint4* dst = o_row(c);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              float y[32];
              tmem_ld32(taddr(tb + 128 * c, 32 * quarter, c0 + 32 * hh), y);
              if (dst) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  float f[8];
                  unpack8(ob[c & 1][4 * hh + u], a.dtype, f);
#pragma unroll
                  for (int e = 0; e < 8; ++e) f[e] += y[8 * u + e];
                  dst[4 * hh + u] = a.dtype == NGDN2_BF16 ? pack8(f) : pack8h(f);
                }
              }
            }
          }
        }
      }
      // The next job's MMAs overwrite the accumulators read above.
      fence_before_sync();
      consumers_sync();
      fence_after_sync();
      if (*reinterpret_cast<volatile int*>(&abort_flag)) break;
    }
    if (tid == 0) {
      // Every MMA issued has completed before TMEM is released.
      mma_commit(&bar_fin);
      if (!mbar_wait(&bar_fin, 0)) abort_flag = 1;
    }
  }
  fence_before_sync();
  __syncthreads();
  if (abort_flag && tid == 0 && a.status) atomicOr(a.status, NGDN2_STATUS_WAIT_TIMEOUT);
  if (warp == 0) tmem_dealloc(tbase, 512);
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static bool is16(int dt) { return dt == NGDN2_BF16 || dt == NGDN2_F16; }

bool seg_supports(const ngdn2_fwd_args* a) {
  if (a->K != TK || a->V != TV || a->L < 1) return false;
  return is16(a->q_dtype) && is16(a->k_dtype) && is16(a->v_dtype) && is16(a->b_dtype) &&
         is16(a->w_dtype) && is16(a->dtype);
}

size_t seg_workspace_bytes(const FwdParams& p) { return size_t(seg_layout(p).total); }

int num_launches_seg(const FwdParams& p) {
  const SegLayout s = seg_layout(p);
  int n = (p.L > 1 ? 1 : 0) + (p.NT > 0 ? 1 : 0);
  for (int l = 0; l < p.L; ++l) {
    if (l > 0 && level_steps(p, l) > 0) ++n;       // probe
    if (s.nseg[l] > 1) n += 2;                      // compose, combine
    ++n;                                            // replay
  }
  if (p.L > 1 && p.NT > 0) ++n;                     // upper-level reads
  return n;
}

static int scan_smem(const StepRec& r) { return kStateBytes + r.smem + r.rows * 256; }

template <int ROWS>
static cudaError_t launch_scan(const SegScanArgs& a, bool compose, int nblocks, int B,
                               cudaStream_t stream) {
  const int smem = scan_smem(a.rec);
  cudaError_t err = cudaFuncSetAttribute(seg_scan_kernel<ROWS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  seg_scan_kernel<ROWS><<<dim3(nblocks, a.H, B), kSegThreads, smem, stream>>>(a, compose ? 0 : 1);
  return cudaGetLastError();
}

static cudaError_t scan_level(const FwdParams& p, const SegLayout& lay, char* ws, int l,
                              cudaStream_t stream) {
  const int64_t bh = int64_t(p.B) * p.H;
  (void)bh;
  SegScanArgs a;
  memset(&a, 0, sizeof(a));
  a.level = l;
  a.L = p.L;
  a.H = p.H;
  a.T = p.T;
  a.nsteps = level_steps(p, l);
  a.seglen = lay.seglen[l];
  a.nseg = lay.nseg[l];
  a.init = p.init;
  a.starts = reinterpret_cast<const float*>(ws + lay.start_off[l]);
  a.mz = ws + lay.mz_off[l];
  a.E = reinterpret_cast<bf16*>(ws + lay.E_off[l]);
  a.nE = lay.nE[l];
  a.emit_every = l == 0 ? (p.L > 1 ? p.firing[1] : 1) : 0;
  a.fin = p.fin;
  a.status = p.status;
  const int rows = level_rows(p, l);
  if (l == 0) {
    a.recs = ws + lay.tc.chunks_off;
    a.out = 1;
    a.o = p.o;
    a.dtype = p.dtype;
  } else {
    a.recs = ws + lay.prec_off[l];
    a.out = 0;
  }
  cudaError_t err;
  if (a.nseg > 1) {
    // compose: the segment transitions (no output, smaller record copies)
    SegScanArgs c = a;
    c.rec = l == 0 ? level0_rec(false) : probe_rec(rows);
    err = rows == 64 ? launch_scan<64>(c, true, 2 * (a.nseg - 1), p.B, stream)
                     : launch_scan<128>(c, true, 2 * (a.nseg - 1), p.B, stream);
    if (err != cudaSuccess) return err;
    err = cudaFuncSetAttribute(seg_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kCombineSmem);
    if (err != cudaSuccess) return err;
    seg_combine_kernel<<<dim3(kCombineSplit, p.H, p.B), kCombineThreads, kCombineSmem, stream>>>(
        a.mz, p.init, reinterpret_cast<float*>(ws + lay.start_off[l]), p.L, l, p.H, a.nseg,
        p.status);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  a.rec = l == 0 ? level0_rec(true) : probe_rec(rows);
  return rows == 64 ? launch_scan<64>(a, false, a.nseg, p.B, stream)
                    : launch_scan<128>(a, false, a.nseg, p.B, stream);
}

static cudaError_t probe_level(const FwdParams& p, const SegLayout& lay, char* ws, int l,
                               cudaStream_t stream) {
  const int nf = level_steps(p, l);
  if (nf == 0) return cudaSuccess;
  ProbeArgs a;
  memset(&a, 0, sizeof(a));
  a.level = l;
  a.H = p.H;
  a.nf = nf;
  a.f_here = p.firing[l];
  a.f_below = p.firing[l - 1];
  a.nE_below = lay.nE[l - 1];
  a.E_below = reinterpret_cast<const bf16*>(ws + lay.E_off[l - 1]);
  a.below_is_level0 = l == 1;
  a.ptc = ws + lay.tc.ptc_off + int64_t(l - 1) * p.H * PT_SIZE;
  a.recs = ws + lay.prec_off[l];
  a.rec = probe_rec(level_rows(p, l));
  a.learned = p.promotion != NGDN2_PROMOTION_MERGE;
  a.nq = level_pairs(p, l);
  a.status = p.status;
  const int smem = kStateBytes + kProbeScratch;
  cudaError_t err =
      cudaFuncSetAttribute(seg_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  seg_probe_kernel<<<dim3(nf, p.H, p.B), kProbeThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

// Chunks per read CTA: the largest of 4, 2, 1 dividing every upper level's
// firing interval (so a unit's chunks share each level's group).
static int read_unit(const FwdParams& p) {
  int u = kReadUnit;
  for (int l = 1; l < p.L; ++l)
    while (u > 1 && p.firing[l] % u) u >>= 1;
  return u;
}

static cudaError_t read_levels(const FwdParams& p, const SegLayout& lay, char* ws,
                               cudaStream_t stream) {
  ReadArgs a;
  memset(&a, 0, sizeof(a));
  a.B = p.B; a.T = p.T; a.H = p.H; a.L = p.L; a.NT = p.NT;
  a.unit = read_unit(p);
  for (int l = 1; l < p.L; ++l) {
    a.firing[l] = p.firing[l];
    a.E[l] = reinterpret_cast<const bf16*>(ws + lay.E_off[l]);
    a.nE[l] = lay.nE[l];
  }
  a.q = p.q;
  a.mix = p.mix;
  a.scale = p.scale;
  a.o = p.o;
  a.dtype = p.dtype;
  a.status = p.status;
  CUtensorMap qmap;
  if (!tc_make_q_map(p, &qmap, &a.hl_mode)) return cudaErrorInvalidValue;
  const int smem = 2 * kReadStage + 1024;
  cudaError_t err =
      cudaFuncSetAttribute(seg_read_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  // Persistent: one CTA per SM (or per job, when fewer) walks its jobs.
  const int64_t njobs = int64_t(p.B) * p.H * ((p.NT + a.unit - 1) / a.unit);
  const int grid = int(njobs < kSMs ? njobs : kSMs);
  seg_read_kernel<<<grid, kReadThreads + 32, smem, stream>>>(a, qmap);
  return cudaGetLastError();
}

cudaError_t launch_fwd_seg(FwdParams p, void* workspace, int stage, cudaStream_t stream) {
  const SegLayout lay = seg_layout(p);
  char* ws = static_cast<char*>(workspace);
  cudaError_t err;
  if (stage == 0 || stage == 1) {
    if ((err = launch_tc_params(p, lay.tc, ws, stream)) != cudaSuccess) return err;
    if ((err = launch_tc_prep(p, lay.tc, ws, stream)) != cudaSuccess) return err;
  }
  if (stage == 0 || stage == 2) {
    for (int l = 0; l < p.L; ++l) {
      if (l > 0 && (err = probe_level(p, lay, ws, l, stream)) != cudaSuccess) return err;
      if ((err = scan_level(p, lay, ws, l, stream)) != cudaSuccess) return err;
    }
    if (p.L > 1 && p.NT > 0 && (err = read_levels(p, lay, ws, stream)) != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace ngdn2
