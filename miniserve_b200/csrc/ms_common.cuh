// Shared device helpers for the MiniServe B200 attention path (sm_100a only).
//
// Everything here is a thin wrapper over one documented PTX instruction: mbarrier phases,
// TMA tensor loads (no multicast anywhere), ldmatrix, mma.sync and ex2.approx.  Every wait is
// bounded: after kSpinLimit polls the caller records an error bit in the device status word and
// leaves its loop instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ms {

// Geometry of the path (Qwen3-0.6B attention: 16 q heads over 8 KV heads, head_dim 128,
// 16-token KV blocks).  The kernels are written for exactly these; the C-ABI rejects others.
constexpr int kHeadDim = 128;
constexpr int kBlockTokens = 16;
constexpr int kGroup = 2;  // query heads per KV head
// One "page" = K or V of one KV head in one block: 16 tokens x 128 dims bf16 = 4 KiB.  In the
// pool layout it is stored as two 2 KiB halves [d/64][token][d%64] so that a 128-byte TMA swizzle
// row is one token's half head.
constexpr int kPageBytes = kBlockTokens * kHeadDim * 2;
constexpr int kPageKVBytes = 2 * kPageBytes;  // K and V of one (block, head): 8 KiB contiguous

// Bits of the device status word (ms_device_status reads and clears it).
constexpr unsigned kErrSlot = 1u;      // a slot_mapping entry outside the pool
constexpr unsigned kErrBlock = 2u;     // a block-table entry outside the pool
constexpr unsigned kErrTimeout = 4u;   // a bounded mbarrier wait gave up
constexpr unsigned kErrPosition = 8u;  // a RoPE position outside the cos/sin table

// ~1e6 polls of try_wait with a 1 us suspend hint: about a second before giving up.
constexpr int kSpinLimit = 1 << 20;

// Programmatic dependent launch (sm_90 and later): every kernel of this library is launched with
// programmatic stream serialization, so its grid may be scheduled while the previous kernel in
// the stream is still running (hiding the launch gap between the per-layer kernels).  Each
// kernel calls pdl_wait() before its first global-memory access -- it returns once the previous
// grid has completed and its writes are visible -- then pdl_trigger(), which lets the next grid
// be scheduled in turn (once every CTA of this grid has triggered or exited).  Both are hardware
// dependencies, not spin-waits; without a programmatic predecessor pdl_wait() returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// Without a suspend-time hint: a hinted try_wait costs about 190 cycles even on a phase that has
// already completed, a plain one about 46.  Threads that feed the tensor core (or sit on its
// critical path) use this form; every cycle they stall is an idle tensor-core cycle.
__device__ __forceinline__ bool mbar_try_wait_nohint(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on the latency-critical path: the abort flag is read only while the phase is still
// open (reading it costs a shared-memory round trip), never on the fast path.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity,
                                               const volatile int* abort_flag) {
  for (int i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_nohint(bar, parity)) return true;
    if (*abort_flag) return false;
  }
  return false;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the thread that issues tcgen05.mma / tcgen05.commit.  A blocking try_wait
// placed after a tcgen05.commit waits for that commit's arrive, i.e. for every MMA in flight
// (about 370 idle tensor-core cycles per wait); the non-blocking test_wait does not.  The abort
// flag is read once every 64 polls.
__device__ __forceinline__ bool mbar_wait_mma(uint64_t* bar, uint32_t parity,
                                              const volatile int* abort_flag) {
  for (int i = 0; i < 16 * kSpinLimit; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 63) == 63 && *abort_flag) return false;
  }
  return false;
}

// ---- TMA (tensor) loads: plain CTA-local destination, no multicast ---------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 5-D tiled load of one box into shared memory; completion is signalled on `bar` as tx bytes.
__device__ __forceinline__ void tma_load_5d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3, int c4,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- warp-level tensor-core fragments (mma.sync m16n8k16, bf16 in, fp32 accumulate) ---------

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of element (row, d) inside a [2 halves][16 rows][64] bf16 tile laid out the way the
// 128-byte TMA swizzle writes it: 16-byte chunk index XOR (row % 8).  The tile must be 1024-byte
// aligned in shared memory.  `rows` is the number of rows per half (16 for a page).
__device__ __forceinline__ uint32_t swz_off(int row, int d, int rows) {
  const int half = d >> 6;
  const int chunk = (d & 63) >> 3;
  return static_cast<uint32_t>(half * rows * 128 + row * 128 + ((chunk ^ (row & 7)) << 4) +
                               ((d & 7) << 1));
}

}  // namespace ms
