// Blackwell (sm_100a) primitives as inline PTX: mbarriers with bounded
// waits, TMA tiled loads, tcgen05 MMA / TMEM alloc / TMEM load-store, and
// the shared-memory matrix and instruction descriptors the MMAs consume.
//
// Every wait is bounded by wall time (%globaltimer): a wait that exceeds
// kWaitLimitNs sets the CTA's abort flag, records kStatusWaitTimeout in the
// library status word and returns false; every other wait in the CTA then
// returns false as soon as it sees the flag, so a protocol bug ends the
// kernel with an error status instead of hanging the GPU.
#pragma once

#include <cuda.h>

#include "sbfa_common.cuh"

namespace sbfa {
namespace tc {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         int* status, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort_flag = 1;
        record_status(status, kStatusWaitTimeout);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled, into this CTA's own shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// TMA tiled store shared -> global (no reduction); completion tracked with
// the bulk async-group of the issuing thread.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int x, int y,
                                             int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
// Untiled bulk copies of `bytes` contiguous bytes (16-byte aligned
// addresses, a multiple of 16 bytes): global -> this CTA's shared memory,
// completing on an mbarrier, and shared -> global in the bulk async-group.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also returns the AND of a predicate over its threads,
// so a group leaves a loop together.
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " barrier.cta.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Per-warpgroup register budget changes (all 4 warps of a warpgroup execute
// them).  The sum over the CTA must stay within what it was launched with.
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, fences, MMA, commit, TMEM load / store
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// tcgen05.mma kind::f16 (fp16/bf16 in, fp32 accumulate) and tcgen05.commit,
// issued warp-wide: every lane of the warp executes them with identical
// (warp-uniform) operands and one elected lane issues the instruction, so the
// operands stay in uniform registers and the issue costs a few instructions.
// _ss: D[tmem] (+)= A[smem desc] * B[smem desc]; _ts: A from TMEM (K-major,
// row m in lane m, two consecutive K elements per 32-bit column).  The commit
// arrives once on `bar` when every tcgen05 async op issued so far by the
// elected thread has completed.
__device__ __forceinline__ void mma_f16_ss_w(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f16_ts_w(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit_w(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          bar)
      : "memory");
}
// The value itself, hidden from the optimiser: descriptor offsets derived
// from it are then computed next to each MMA instead of being hoisted out of
// the issue loop as dozens of loop-invariant registers.
__device__ __forceinline__ uint64_t opaque(uint64_t v) {
  asm volatile("mov.b64 %0, %0;" : "+l"(v));
  return v;
}

// Bounded wait executed by a whole warp; false on every lane if any lane's
// wait failed.  The common case, a phase that has already completed, takes a
// uniform fast path (one try_wait and one vote, ~25 cycles) instead of the
// divergence-safe loop (~75).
__device__ __forceinline__ bool wait_bar_w(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                           int* status) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  return __all_sync(0xffffffffu, wait_bar(bar, parity, abort_flag, status));
}

// 32 consecutive TMEM columns of this warp's 32 lanes -> 32 registers.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle, sm100 version bits.
//  K-major operand (rows of 64 16-bit elements = 128 B; 8-row atoms):
//    LBO unused (16 B), SBO = 1024 B between 8-row groups.
//  MN-major operand (128 B = 64 elements along M/N per k; 8 k per atom):
//    LBO = byte distance between 64-element M/N groups,
//    SBO = byte distance between 8-k groups (1024 B when k rows are dense).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}
// The start-address field is the low 14 bits of (address >> 4), so for
// offsets that keep the address inside shared memory
//   desc(addr + off) == desc(addr) + (off >> 4):
// kernels build one base descriptor per buffer and add constant offsets.
__device__ __forceinline__ uint64_t desc_advance(uint64_t desc, uint32_t off_bytes) {
  return desc + (uint64_t)(off_bytes >> 4);
}
// Shared-memory matrix descriptor without swizzle: the operand is made of
// core matrices of 8 rows x 16 bytes, each 128 contiguous bytes.  For an
// MN-major operand a core-matrix row is 8 consecutive M/N elements of one k;
//    LBO = byte distance between core matrices adjacent along K,
//    SBO = byte distance between core matrices adjacent along M/N.
__device__ __forceinline__ uint64_t smem_desc_noswizzle(uint32_t addr, uint32_t lbo_bytes,
                                                        uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm100; layout type 0: no swizzle
  return d;
}
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
  return smem_desc_sw128(addr, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr, uint32_t mn_group_bytes) {
  return smem_desc_sw128(addr, mn_group_bytes, 1024);
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool a_mn_major,
                                                 bool b_mn_major) {
  return (1u << 4)                              // D: f32
         | ((bf16 ? 1u : 0u) << 7)              // A: f16 / bf16
         | ((bf16 ? 1u : 0u) << 10)             // B: f16 / bf16
         | ((a_mn_major ? 1u : 0u) << 15)       // A major
         | ((b_mn_major ? 1u : 0u) << 16)       // B major
         | ((uint32_t)(N >> 3) << 17)           // N / 8
         | ((uint32_t)(M >> 4) << 24);          // M / 16
}

// Byte offset of element (row, col) of a [rows][64] 16-bit tile stored with
// the 128-byte swizzle (16-byte chunk index XOR row % 8), rows 128 B apart.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col) {
  const uint32_t chunk = (col >> 3) ^ (row & 7u);
  return row * 128u + chunk * 16u + (col & 7u) * 2u;
}

// Bits [lo, hi) of a 32-bit word whose bit 0 is column `base` (lo/hi in
// absolute columns, any range).
__device__ __forceinline__ uint32_t range_bits(int lo, int hi, int base) {
  const int a = min(max(lo - base, 0), 32), b = min(max(hi - base, 0), 32);
  const uint32_t upto_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
  const uint32_t upto_a = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
  return upto_b & ~upto_a;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Largest of three floats in one instruction.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// Host: tensor maps
// ---------------------------------------------------------------------------
// 4-D map over a [B][H][rows][cols] 16-bit tensor with element strides
// st (batch, head, row; unit-stride cols), a {64, box_rows, 1, 1} box and the
// 128-byte swizzle (OOB rows read as zero, OOB stores are clipped).  Tiles
// never cross a (batch, head) boundary.  The base must be 16-byte aligned and
// every stride a multiple of 8 elements.
int make_tmap_4d(CUtensorMap* map, const void* base, bool bf16, uint64_t cols, uint64_t rows,
                 uint64_t heads, uint64_t batch, const Strides3& st, uint32_t box_rows);
// True when (base, strides) satisfy the TMA rules above for 16-bit elements.
bool tma_compatible(const void* base, const Strides3& st);

}  // namespace tc
}  // namespace sbfa
