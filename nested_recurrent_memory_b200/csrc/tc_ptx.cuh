// Thin wrappers over the sm_100a PTX used by the tensor-core kernels:
// shared-memory matrix descriptors, tcgen05.mma (kind::f16, one CTA),
// tcgen05.commit, TMEM allocation / loads / stores, mbarriers with bounded
// waits, and 1-D bulk copies. Layout helpers describe the no-swizzle UMMA
// canonical layouts the kernels write their operands in.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace ngdn2 {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Operand layouts (no swizzle). A "core matrix" is 8 rows of 16 bytes
// (8 bf16) stored as 128 contiguous bytes.
//
// K-major tile [R][Kd] (row r holds its Kd reduction elements): core matrix
// (r/8, k/8) at ((r/8) * (Kd/8) + k/8) * 64 elements. Descriptor: LBO = 128 B
// (next core matrix along K), SBO = Kd * 16 B (next 8-row group).
//
// MN-major tile [Kd][R] (row k holds R contiguous M/N elements): core
// matrix (k/8, r/8) at ((r/8) * (Kd/8) + k/8) * 64 elements, with the 8
// elements of a 16-byte row consecutive in r. Descriptor: LBO = 128 B (next
// core matrix along K), SBO = Kd * 16 B (next 8-column group).
//
// Both advance by 256 B per K-step of 16.
// ---------------------------------------------------------------------------

__host__ __device__ __forceinline__ int kmajor_off(int r, int k, int Kd) {
  return ((r >> 3) * (Kd >> 3) + (k >> 3)) * 64 + (r & 7) * 8 + (k & 7);
}

__host__ __device__ __forceinline__ int mnmajor_off(int k, int r, int Kd) {
  return ((r >> 3) * (Kd >> 3) + (k >> 3)) * 64 + (k & 7) * 8 + (r & 7);
}

// Shared-memory matrix descriptor for the layouts above.
__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  return d;                             // base offset 0, no swizzle
}

// Descriptor of K-step ``kk`` (16 elements) of a tile at ``saddr`` with
// reduction extent Kd, in either layout.
__device__ __forceinline__ uint64_t desc_tile(uint32_t saddr, int Kd, int kk) {
  return desc_noswz(saddr + kk * 256, 128, Kd * 16);
}

// 128-byte-swizzled K-major layout (what a TMA copy with SWIZZLE_128B
// writes): rows of 64 bf16 = 128 bytes, 8-row atoms of 1024 bytes (1024-byte
// aligned) whose 16-byte chunks are XOR-permuted by the row within the atom,
// atoms stacked along M; a K extent of 128 is two such [M x 64] blocks.
// sw128_off gives the byte offset of element (r, k) in an M = 64 tile
// (blocks 8 KB apart).
__device__ __forceinline__ int sw128_off(int r, int k) {
  return (k >> 6) * 8192 + (r >> 3) * 1024 + (r & 7) * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4) +
         (k & 7) * 2;
}

// Descriptor of a 128-byte-swizzled K-major operand: 8-row groups SBO bytes
// apart; the leading offset is unused for this layout (encoded as 1).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16 with fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// C[M x N] (+)= A[M x Kd] . B[Kd x N] as Kd/16 MMAs issued by the calling
// thread. a/b are shared addresses of tiles in the layouts above.
__device__ __forceinline__ void mma_tile(uint32_t d_tmem, uint32_t a_saddr, uint32_t b_saddr,
                                         int Kd, uint32_t idesc, bool accumulate) {
  for (int kk = 0; kk < Kd / 16; ++kk)
    mma_f16(d_tmem, desc_tile(a_saddr, Kd, kk), desc_tile(b_saddr, Kd, kk), idesc,
            (accumulate || kk > 0) ? 1u : 0u);
}

// C[128 x N] (+)= A[128 x 128] . B[128 x N] where A's rows 64..127 are the
// M = 64, 128-byte-swizzled tile at a_tile (sw128_off) and rows 0..63 are
// whatever the 8 KB before each of its two K blocks holds; B as mma_tile.
__device__ __forceinline__ void mma_tile_sw128_lo(uint32_t d_tmem, uint32_t a_tile,
                                                  uint32_t b_saddr, uint32_t idesc,
                                                  bool accumulate) {
  for (int kk = 0; kk < 8; ++kk)
    mma_f16(d_tmem, desc_sw128(a_tile + (kk >> 2) * 8192 + (kk & 3) * 32 - 8192, 1024),
            desc_tile(b_saddr, 128, kk), idesc, (accumulate || kk > 0) ? 1u : 0u);
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (MMA, bulk copy).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM
// ---------------------------------------------------------------------------

// Executed by one full warp. Writes the base address to *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 32 lanes x 16 columns of 32 bits: thread t gets lane (taddr.lane + t),
// columns taddr.col .. +15, waited for. Warp-collective.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 columns; no wait (pair with tmem_wait_ld and
// tmem_regs_after_wait16). Warp-collective.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 8 columns; no wait (pair with tmem_wait_ld and
// tmem_regs_after_wait8). Warp-collective.
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_regs_after_wait8(uint32_t* r) {
  asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
               "+r"(r[6]), "+r"(r[7])::"memory");
}

__device__ __forceinline__ void tmem_regs_after_wait16(uint32_t* r) {
  asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
               "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
               "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])::"memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

// 32 lanes x 32 columns; no wait (pair with tmem_wait_ld). Warp-collective.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// Order uses of 32 registers after the preceding tcgen05.wait::ld (asm
// volatile statements keep their order; the "+r" operands tie the registers
// to this point).
__device__ __forceinline__ void tmem_regs_after_wait32(uint32_t* r) {
  asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]) :: "memory");
}

// 32 consecutive columns, waited for, as floats.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  tmem_ld32_nowait(taddr, r);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  tmem_regs_after_wait32(r);
}

// 64 consecutive columns (two x32 loads, one wait) as floats.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  tmem_ld32_nowait(taddr, r);
  tmem_ld32_nowait(taddr + 32, r + 32);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  tmem_regs_after_wait32(r);
  tmem_regs_after_wait32(r + 32);
}

__device__ __forceinline__ void tmem_st64(uint32_t taddr, const float* v) {
  tmem_st32(taddr, v);
  tmem_st32(taddr + 32, v + 32);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column).
__device__ __forceinline__ uint32_t taddr(uint32_t base, int lane, int col) {
  return base + (static_cast<uint32_t>(lane) << 16) + static_cast<uint32_t>(col);
}

// ---------------------------------------------------------------------------
// mbarriers with bounded waits
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Spins at most ``limit`` polls (each poll itself may suspend briefly).
// Returns false on timeout instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, phase)) return true;
  return false;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// 1-D bulk copy shared -> global in the issuing thread's bulk group (commit
// with bulk_commit; bulk_wait_read0 before the source is rewritten,
// bulk_wait0 before the kernel ends). Both addresses 16-byte aligned, bytes
// a multiple of 16.
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(ssrc)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 1-D bulk copy global -> shared, completing ``bytes`` on ``bar``. Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Hint: bring [src, src + bytes) into L2 (16-byte aligned, multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Hint: bring one 3-D box of a tiled tensor map into L2 (no shared memory,
// no completion). The innermost coordinate is always 0 here.
__device__ __forceinline__ void tma_prefetch_l2_3d(const void* tmap, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// Tiled tensor-map load (this CTA only) of one 4-D box into shared memory,
// completing its bytes on ``bar``. The tensor map lives in kernel parameter
// space (__grid_constant__); the innermost coordinate is always 0 here.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int c0, int c1, int c2,
                                            int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

}  // namespace tc
}  // namespace ngdn2
