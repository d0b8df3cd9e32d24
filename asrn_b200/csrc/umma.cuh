// Blackwell (sm_100a) tensor-core primitives: mbarriers, TMA tile loads, TMEM allocation, tcgen05.mma (kind::f16,
// bf16 inputs, fp32 accumulator in TMEM) and tcgen05.ld, plus the shared-memory matrix descriptor of a K-major
// operand in the 128-byte-swizzled canonical layout (rows of 64 bf16 = 128 B, 8-row groups of 1024 B, the 16-byte
// chunk index XOR-ed with the row index within its group).
//
// Every wait on an mbarrier is bounded by the global timer: past the limit it records ASRN_ERR_TIMEOUT in the layer's
// device status word (in the prepared-weights buffer, read by asrn_layer_status) and returns false, so a kernel never
// spins forever.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace asrn {

namespace umma {

constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s: far above any legitimate wait of these kernels

ASRN_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

ASRN_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

ASRN_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
ASRN_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
ASRN_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
ASRN_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
ASRN_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete. false: timed out (status word set). Once the status
// word records a timeout, later waits that do not complete at once give up immediately, so a kernel whose copies
// never arrive ends after one wait limit rather than one per wait.
ASRN_DEV bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* status, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  if (status && *reinterpret_cast<volatile int*>(status) == ASRN_ERR_TIMEOUT) return false;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) {
      if (status) atomicCAS(status, ASRN_OK, ASRN_ERR_TIMEOUT);
      return false;
    }
  }
}
ASRN_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  return mbar_wait_limit(bar, parity, status, kWaitLimitNs);
}

// 2-D tiled TMA load of a box into shared memory, completing transaction bytes on `bar`.
// x is the innermost coordinate (elements); it must be a multiple of 16 bytes / element size.
ASRN_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
ASRN_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- TMEM ----------------------------------------------------------------------------------------------------------
// Allocation by one whole warp; the TMEM address (lane 0, first column) is written to *dst (shared memory).
ASRN_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
ASRN_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
ASRN_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
ASRN_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ASRN_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Order this thread's generic-proxy shared-memory writes before later async-proxy reads (tcgen05.mma / TMA).
ASRN_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- MMA -------------------------------------------------------------------------------------------------------------
// Instruction descriptor of kind::f16: bf16 A and B, fp32 D, both operands K-major, shape M x N.
constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Shared-memory descriptor of a K-major, 128-byte-swizzled operand starting at `saddr` (1024-byte aligned tile;
// the K offset of a sub-step is added as bytes / 16 to the start address).
ASRN_DEV uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused by swizzled K-major layouts)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // descriptor version of sm_100
  d |= (uint64_t)2 << 61;                 // 128-byte swizzle
  return d;
}
// The same for a K-major operand in the 64-byte-swizzled layout (rows of 32 bf16 = 64 B, 8-row groups of 512 B, the
// 16-byte chunk index XOR-ed with (row / 2) mod 4); the tile starts on a 512-byte boundary.
ASRN_DEV uint64_t desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;        // stride byte offset: 8 rows x 64 B
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;                 // 64-byte swizzle
  return d;
}
// Shared-memory descriptor of an MN-major, 128-byte-swizzled operand: atoms of 64 MN elements (128 B) x 8 K rows
// (1024 B, the 16-byte chunk index XOR-ed with the row within the atom), consecutive 8-row K groups 1024 B apart
// (stride byte offset), consecutive 64-element MN blocks `mn_stride` bytes apart (leading byte offset).
ASRN_DEV uint64_t desc_mn_sw128(uint32_t saddr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((mn_stride >> 4) & 0x3FFFu) << 16;   // leading byte offset: the next 64 MN elements
  d |= (uint64_t)(1024 >> 4) << 32;                     // stride byte offset: the next 8 K rows
  d |= (uint64_t)1 << 46;                               // descriptor version of sm_100
  d |= (uint64_t)2 << 61;                               // 128-byte swizzle
  return d;
}
// D[tmem] (+)= A[smem] x B[smem]^T, issued by one thread.
ASRN_DEV void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
ASRN_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32 (w % 4) .. + 31).
ASRN_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of the 16-byte chunk `c` (0..7) of row `r` inside a 128-byte-swizzled K-major tile.
ASRN_DEV uint32_t sw128_offset(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

ASRN_DEV uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

}  // namespace umma
}  // namespace asrn
