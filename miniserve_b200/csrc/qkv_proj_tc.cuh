// Kernel E: the fused qkv projection with kernel A as its epilogue, on the tcgen05 tensor cores.
//
// Replaces, for one layer, `self.qkv_proj(x)` and the split / q_norm / k_norm / apply_rope that
// follow it (src/miniserve/model/qwen3.py:94-98), plus the K/V scatter at the top of
// paged_attention (src/miniserve/attention/backends.py:159-160): the projection output never goes
// to memory.
//
// Work unit: a tile of 128 tokens x (128 * kHeads) features of  qkv = x W^T , i.e. kHeads head row
// blocks of the fused projection for 128 tokens (kHeads = 2 pairs heads of one kind: query heads
// 2p, 2p+1, key heads 2p, 2p+1 or value heads 2p, 2p+1).  Tile i covers token block i / P and head
// group i % P (P = (H + 2 KVH) / kHeads), so the CTAs that run together share their x tile through
// L2.  The kernel is persistent: one CTA per SM walks tiles c, c + G, c + 2G, ...
//
// The main loop is bound by L2 -> SM traffic (every tile streams its x rows and its W rows over
// the whole hidden dimension): kHeads = 2 moves 48 KiB per 64-wide step for two heads instead of
// 32 KiB for one, and the two heads share each token's cos/sin loads in the epilogue.  kHeads = 1
// makes twice as many tiles, for small batches that would not fill the GPU otherwise.
//
//   warp 16     TMA producer: per 64-wide hidden step a 128 x 64 tile of x and kHeads 128 x 64
//               tiles of W (16 KiB each, 128-byte swizzled) into the stage ring; it runs straight on
//               into the next tile.
//   warp 17     TMEM allocator and MMA issuer: D_b += x_tile W_tile^T (M=128, N=128*kHeads, K=16 x 4
//               per step, both operands K-major from shared memory) into one of two TMEM
//               accumulators, so the next tile's MMAs overlap this tile's epilogue.
//   warps 0-15  epilogue, in two stages per tile (the row facts -- pool slot, cos/sin row -- are
//               gathered into shared memory while the MMAs still run):
//               1. TMEM -> registers -> bf16 (the projection's output dtype) -> a row-major
//                  staging tile in shared memory (warp w: lane quarter w % 4, 32-column slice
//                  w / 4 of every head; rows are padded 16 bytes so the 32 rows a warp writes hit
//                  distinct banks), then the accumulator is handed back to the MMA warp;
//               2. kernel A's per-row code on the staged rows, 8 rows per warp, one lane per 4
//                  dims: the same fp32 square sums, the same xor butterfly, the same rsqrt and
//                  rounding points, so the results equal kernel A's on the same bf16 projection
//                  output bit for bit, and every global load (cos/sin rows) and store (q rows,
//                  pool rows) is a whole coalesced row.
//
// Products and sums of two bf16 values use the paired bf16 instructions (mul/add/sub.rn.bf16x2):
// the fp32 product of two bf16 values is exact, so one correctly rounded bf16 product equals
// kernel A's fp32 product rounded to bf16; for the sum of two bf16 values the two can differ only
// if the fp32 sum is inexact, which needs exponents more than 16 apart, and then both give the
// larger operand.
//
// The only difference from cuBLAS + kernel A is the order in which the GEMM accumulates its fp32
// products, which can move a projection output by one bf16 ulp.  Every wait is bounded; on a
// timeout the CTA records kErrTimeout, all roles leave their loops, MMAs in flight are drained,
// TMEM is freed and the CTA exits.
#pragma once

#include "norm_rope_scatter.cuh"
#include "tc_common.cuh"

namespace ms {

template <int kHeads, int kSplit = 1>
struct QkvCfg {
  static_assert(kHeads == 1 || kHeads == 2, "one or two heads per tile");
  static_assert(kSplit == 1 || (kSplit == 2 && kHeads == 1), "split-K pairs run one-head tiles");
  static constexpr int kEpiWarps = 16;
  static constexpr int kProducerWarp = 16;
  static constexpr int kMmaWarp = 17;
  static constexpr int kThreads = 576;
  // A split-K pair runs half of the hidden steps per CTA and needs room for the peer's partial.
  static constexpr int kStages = kSplit == 2 ? 4 : (kHeads == 1 ? 5 : 3);
  static constexpr int kTileRows = 128;     // tokens per tile (M)
  static constexpr int kTileN = 128 * kHeads;
  static constexpr int kKStep = 64;         // hidden elements per stage (one 128-byte row)
  static constexpr int kBoxBytes = 16384;   // 128 rows x 128 bytes
  static constexpr int kStageBytes = kBoxBytes * (1 + kHeads);
  static constexpr int kRowPitch = 256 * kHeads + 16;  // staging row: bf16 features + 16-byte skew
  static constexpr int kStagingOff = kStages * kStageBytes;
  // bf16 staging rows: the whole tile, or a split-K CTA's own 64 rows.
  static constexpr int kStageRows = kSplit == 2 ? 64 : 128;
  static constexpr int kMetaOff = kStagingOff + kStageRows * kRowPitch;  // [128] {slot, cos/sin row}
  static constexpr int kFlagOff = kMetaOff + 128 * 16;  // [16] int: epilogue warp verdicts
  // Split-K pairs: the fp32 partial of 64 rows (two 32-row chunks, one per TMEM lane quarter), as
  // received from the peer (this CTA's rows) and as sent to it (the peer's rows), in one layout:
  // rows padded 16 bytes, so the 32 rows a warp writes or reads start in different banks.  One
  // bulk copy moves a chunk.
  static constexpr int kRecvPitch = 128 * kHeads * 4 + 16;
  static constexpr int kChunkBytes = 32 * kRecvPitch;
  static constexpr int kRecvOff = kFlagOff + 64;
  static constexpr int kRecvBytes = kSplit == 2 ? 2 * kChunkBytes : 0;
  static constexpr int kSendOff = kRecvOff + kRecvBytes;
  static constexpr int kBarOff = kSendOff + kRecvBytes;
  // full, empty, acc_full[2], acc_empty[2], drain; split-K pairs: recv_full[2], send_ready[2],
  // peer_done
  static constexpr int kNumBars = 2 * kStages + 4 + 1 + (kSplit == 2 ? 5 : 0);
  static constexpr int kSmemBytes = 1024 + kBarOff + (kNumBars + 2) * 8;
  static constexpr uint32_t kTmemCols = 256 * kHeads;  // two accumulators
  static_assert(kSmemBytes <= 232448, "kernel E exceeds 227 KiB of shared memory");
  static_assert(kRecvOff % 16 == 0 && kSendOff % 16 == 0 && kChunkBytes % 16 == 0,
                "bulk copies move 16-byte aligned multiples of 16 bytes");
};

struct QkvArgs {
  NormRopeArgs e;   // the epilogue's arguments, exactly kernel A's
  int hidden;       // K of the projection (multiple of 64)
  int num_tiles;    // ceil(T / 128) * (H + 2 KVH) / kHeads
};

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t v) {
  return *reinterpret_cast<__nv_bfloat162*>(&v);
}
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
// The two bf16 of a pair as fp32 (exact).
__device__ __forceinline__ float2 bf2_to_f2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// The 512 epilogue threads meet at named barrier 1 (barrier 0 is __syncthreads).
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, 512;" ::: "memory");
}

__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// ---- a 2-CTA cluster (split-K pairs): the peer's shared memory and barriers ------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_smem(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// One thread: copy `bytes` of this CTA's shared memory to `remote_dst` in the peer CTA; the copy
// completes as transaction bytes on the peer's mbarrier `remote_bar` (no multicast).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t remote_dst, uint32_t local_src,
                                                  uint32_t bytes, uint32_t remote_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(remote_dst),
      "r"(local_src), "r"(bytes), "r"(remote_bar)
      : "memory");
}
// Arrive on an mbarrier of another CTA of the cluster; the writes before it become visible to a
// thread that then completes a cluster-scope acquire wait on that barrier.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
               : "memory");
}
// Bounded wait with cluster-scope acquire (the arrivals come from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  const volatile int* abort_flag) {
  for (int i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (*abort_flag) return false;
  }
  return false;
}
// Cluster barrier halves (every thread, warp-converged).  The relaxed arrive does not wait for
// the thread's earlier memory accesses; the barrier inits are ordered before it by
// fence.mbarrier_init, and nothing else needs ordering through this barrier.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// Per-row facts of the tile's 128 tokens, gathered while the accumulator is still being computed:
// the pool slot (-1: nothing to write -- past the batch, or a slot outside the pool) and the
// cos/sin row to use (validated).
struct RowMeta {
  long long slot;
  long long cs_row;
};

__device__ __forceinline__ RowMeta ld_meta(uint32_t addr) {
  RowMeta m;
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(m.slot), "=l"(m.cs_row) : "r"(addr));
  return m;
}

// A row's cos and sin at this lane's dims, rounded to bf16 pairs (kernel A: .to(bf16)).
struct RopeRow {
  uint32_t c01, c23, s01, s23;
};

// Kernel A's per-row work (lane = dims 4l..4l+3) for N staged rows of the tile's kHeads query or
// key heads, with the rows' cos/sin already in registers.  Tile rows row0 .. row0 + N - 1 are
// staged at staging rows srow0 .. srow0 + N - 1.
template <int kHeads, int N>
__device__ __forceinline__ void norm_rope_rows(const NormRopeArgs& a, uint32_t stage_base,
                                               uint32_t meta_base, int row0, int srow0, int m0,
                                               int head_row0, bool is_q, uint2 w2,
                                               const RopeRow* cs, int lane) {
  using Cfg = QkvCfg<kHeads>;
  const int d0 = lane * 4;
  long long slot[N];
  bool any = false;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    slot[i] = ld_meta(meta_base + (row0 + i) * 16).slot;
    any = any || slot[i] >= 0;
  }
  if (!any) return;  // every row past the batch (the facts are the same in every lane)
  uint2 raw[N][kHeads];
#pragma unroll
  for (int i = 0; i < N; ++i) {
#pragma unroll
    for (int h = 0; h < kHeads; ++h)
      raw[i][h] = ld_shared_v2(stage_base + (srow0 + i) * Cfg::kRowPitch + h * 256 + lane * 8);
  }
  float ss[N][kHeads];
#pragma unroll
  for (int i = 0; i < N; ++i) {
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      const float2 x01 = bf2_to_f2(raw[i][h].x), x23 = bf2_to_f2(raw[i][h].y);
      const float2 ev = make_float2(x01.x, x23.x), od = make_float2(x01.y, x23.y);
      const float2 p = __fadd2_rn(__fmul2_rn(ev, ev), __fmul2_rn(od, od));  // (x0^2+x1^2, x2^2+x3^2)
      ss[i][h] = __fadd_rn(p.x, p.y);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
      for (int h = 0; h < kHeads; ++h)
        ss[i][h] = __fadd_rn(ss[i][h], __shfl_xor_sync(0xffffffffu, ss[i][h], off));
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const __nv_bfloat162 c01 = as_bf2(cs[i].c01), c23 = as_bf2(cs[i].c23);
    const __nv_bfloat162 s01 = as_bf2(cs[i].s01), s23 = as_bf2(cs[i].s23);
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss[i][h], 1.0f / kHeadDim), a.eps));
      const float2 inv2 = make_float2(inv, inv);
      const float2 y01 = __fmul2_rn(bf2_to_f2(raw[i][h].x), inv2);  // (x32 * rsqrt).to(bf16)
      const float2 y23 = __fmul2_rn(bf2_to_f2(raw[i][h].y), inv2);
      const uint32_t z01 = as_u32(__hmul2_rn(as_bf2(w2.x), as_bf2(pack_bf16(y01.x, y01.y))));
      const uint32_t z23 = as_u32(__hmul2_rn(as_bf2(w2.y), as_bf2(pack_bf16(y23.x, y23.y))));
      const uint32_t p01 = __shfl_xor_sync(0xffffffffu, z01, 16);  // rotate_half partner (d +- 64)
      const uint32_t p23 = __shfl_xor_sync(0xffffffffu, z23, 16);
      // rotate_half: dims < 64 take -z[d + 64], dims >= 64 take z[d - 64].
      uint2 o;
      if (lane < 16) {
        o.x = as_u32(__hsub2_rn(__hmul2_rn(as_bf2(z01), c01), __hmul2_rn(as_bf2(p01), s01)));
        o.y = as_u32(__hsub2_rn(__hmul2_rn(as_bf2(z23), c23), __hmul2_rn(as_bf2(p23), s23)));
      } else {
        o.x = as_u32(__hadd2_rn(__hmul2_rn(as_bf2(z01), c01), __hmul2_rn(as_bf2(p01), s01)));
        o.y = as_u32(__hadd2_rn(__hmul2_rn(as_bf2(z23), c23), __hmul2_rn(as_bf2(p23), s23)));
      }
      if (slot[i] < 0) continue;
      if (is_q) {
        const long long t = m0 + row0 + i;
        *reinterpret_cast<uint2*>(a.q_out + t * a.q_out_row_stride + (head_row0 + h) * kHeadDim +
                                  d0) = o;
      } else {
        *reinterpret_cast<uint2*>(a.k_pool + pool_offset(slot[i], head_row0 + h - a.num_heads, d0,
                                                         a.block_stride, a.head_stride)) = o;
      }
    }
  }
}

// kSplit = 2: the kernel runs as clusters of two CTAs that share each tile.  CTA r accumulates
// hidden steps [r * K / 2, (r + 1) * K / 2) and owns the tile rows of TMEM lane quarters r and
// r + 2 (rows 32 r .. +31 and 64 + 32 r .. +31, so a ragged last token block still splits
// evenly).  It writes the fp32 partial of the peer's rows to its send buffer, and per quarter one
// thread moves its 32 rows into the peer's receive buffer with one bulk copy through distributed
// shared memory (quarters wholly past the batch are not sent); each CTA adds the peer's partial
// to its own rows and runs the epilogue on them: per CTA half the operand stream and half the
// epilogue of a whole tile, for steps whose tiles would leave most SMs idle.  No load is
// multicast.
template <int kHeads, int kSplit = 1>
__global__ void __launch_bounds__(QkvCfg<kHeads, kSplit>::kThreads, 1)
    qkv_proj_norm_rope_kernel(const __grid_constant__ CUtensorMap x_map,
                              const __grid_constant__ CUtensorMap w_map, const QkvArgs qa,
                              unsigned* status) {
  using Cfg = QkvCfg<kHeads, kSplit>;
  // The tensor maps are kernel parameters, written by no earlier kernel: fetch them while the
  // previous grid may still run.
  if (threadIdx.x == Cfg::kProducerWarp * 32) {
    tma_prefetch_desc(&x_map);
    tma_prefetch_desc(&w_map);
  }
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int NS = Cfg::kStages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* full = bars;              // [NS] stage landed
  uint64_t* empty = full + NS;        // [NS] stage consumed by the MMAs
  uint64_t* acc_full = empty + NS;    // [2] accumulator b complete
  uint64_t* acc_empty = acc_full + 2; // [2] accumulator b read out by the epilogue
  uint64_t* drain = acc_empty + 2;    // every MMA issued has completed
  uint64_t* recv_full = drain + 1;     // split-K [2]: the peer's partial for a chunk landed
  uint64_t* send_ready = recv_full + 2;  // split-K [2]: a send chunk holds this tile's partial
  uint64_t* peer_done = send_ready + 2;  // split-K: the peer has read what this CTA sent it
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + Cfg::kNumBars + 1);
  const NormRopeArgs& a = qa.e;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups_per_tok = (a.num_heads + 2 * a.num_kv) / kHeads;
  const int ksteps = qa.hidden / Cfg::kKStep;
  // Split-K pairs: CTA `rank` of the pair takes hidden steps [k_begin, k_end) of every tile of
  // its stream; the pairs walk the tiles like single CTAs do (pair blockIdx.x / 2 from tile
  // blockIdx.x / 2 on, every gridDim.x / 2).
  const uint32_t rank = kSplit == 2 ? cluster_ctarank() : 0u;
  const int k_begin = static_cast<int>(rank) * (ksteps / kSplit);
  const int k_end = k_begin + ksteps / kSplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], Cfg::kEpiWarps);
    }
    mbar_init(drain, 1);
    if (kSplit == 2) {
      for (int c = 0; c < 2; ++c) {
        mbar_init(&recv_full[c], 1);   // this CTA's expect_tx; the peer's bulk copy brings the bytes
        mbar_init(&send_ready[c], 4);  // one arrival per sending warp of the chunk
      }
      mbar_init(peer_done, 8);  // one arrival per receiving warp of the peer, every tile
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == Cfg::kMmaWarp) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Both CTAs of a pair must have initialised their barriers before either touches the other's:
  // every thread arrives here and waits before its first access to the peer (the epilogue) or
  // at the end, so the barrier's latency hides under the main loop.
  if (kSplit == 2) cluster_arrive_relaxed();
  const uint32_t tmem = *tmem_holder;
  // Split-K: the threads that arm this CTA's receive barriers (one per chunk), how many phases
  // each has armed and seen complete (a copy still landing is waited for before the CTA exits),
  // and the tiles the epilogue went through.
  uint64_t* recv_bar = nullptr;
  int recv_armed = 0, recv_seen = 0, tiles_seen = 0;

  if (warp == Cfg::kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0;  // stages issued so far (over all of this CTA's tiles)
      for (int tile = kSplit == 2 ? blockIdx.x >> 1 : blockIdx.x; tile < qa.num_tiles && !*abort_flag; tile += kSplit == 2 ? gridDim.x >> 1 : gridDim.x) {
        const int m0 = (tile / groups_per_tok) * Cfg::kTileRows;
        const int n0 = (tile % groups_per_tok) * Cfg::kTileN;
        for (int k = k_begin; k < k_end; ++k, ++g) {
          const int s = g % NS;
          if (g >= NS && !mbar_wait_fast(&empty[s], ((g / NS) - 1) & 1, abort_flag)) {
            atomicOr(status, kErrTimeout);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          uint8_t* st = smem + s * Cfg::kStageBytes;
          // Token rows past the batch read as zeros (TMA out-of-bounds fill).
          tma_load_2d(st, &x_map, &full[s], k * Cfg::kKStep, m0);
#pragma unroll
          for (int h = 0; h < kHeads; ++h)
            tma_load_2d(st + (1 + h) * Cfg::kBoxBytes, &w_map, &full[s], k * Cfg::kKStep,
                        n0 + h * 128);
        }
      }
      // No copy may still be landing when the CTA exits.
      for (int k = g > NS ? g - NS : 0; k < g; ++k) {
        if (!mbar_wait(&full[k % NS], (k / NS) & 1)) {
          atomicOr(status, kErrTimeout);
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp == Cfg::kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_bf16(128, Cfg::kTileN, false);
      const uint64_t d0 = umma_smem_desc_sw128(smem_u32(smem), 16, 1024);
      constexpr uint32_t kStage16 = Cfg::kStageBytes >> 4;
      constexpr uint32_t kBox16 = Cfg::kBoxBytes >> 4;
      bool ok = true;
      int g = 0, j = 0;
      for (int tile = kSplit == 2 ? blockIdx.x >> 1 : blockIdx.x; ok && tile < qa.num_tiles; tile += kSplit == 2 ? gridDim.x >> 1 : gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait_mma(&acc_empty[b], ((j >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * Cfg::kTileN;
        for (int k = k_begin; k < k_end; ++k, ++g) {
          const int s = g % NS;
          if (!mbar_wait_mma(&full[s], (g / NS) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t xd = d0 + s * kStage16;
          const uint64_t wd = xd + kBox16;  // kHeads W boxes, contiguous: one N = 128 kHeads operand
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ss(acc, xd + kk * 2, wd + kk * 2, kIdesc, (k > k_begin || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
      if (!ok) {
        atomicOr(status, kErrTimeout);
        *abort_flag = 1;
      }
      // TMEM is freed after the final barrier: no MMA may still be writing it by then.
      umma_commit(drain);
      if (!mbar_wait(drain, 0)) atomicOr(status, kErrTimeout);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    // Rows per warp in stage 2: 8 of a whole tile, or 4 of a split-K CTA's 64 rows.
    constexpr int kWarpRows = kSplit == 2 ? 4 : 8;
    const int etid = threadIdx.x;  // 0..511
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 = staged rows
    const int colq = warp >> 2;    // columns 32*colq .. +31 of every head
    const uint32_t stage_base = smem_u32(smem + Cfg::kStagingOff);
    const uint32_t meta_base = smem_u32(smem + Cfg::kMetaOff);
    volatile int* verdict = reinterpret_cast<volatile int*>(smem + Cfg::kFlagOff);
    // Split-K: this CTA owns the rows of TMEM lane quarters rank and rank + 2; warps of the other
    // two quarters send their rows' partial to the peer, which owns them.  Quarter q's rows are
    // chunk q / 2 of the send and receive buffers and of the staging rows.
    const bool sender = kSplit == 2 && (quarter & 1) != static_cast<int>(rank);
    const int chunk = quarter >> 1;
    // Per chunk: the sender warp that issues the bulk copy, the receiver lane that arms it.
    const bool issuer = sender && colq == 0;
    const bool recv_leader = kSplit == 2 && !sender && colq == 0 && lane == 0;
    if (recv_leader) recv_bar = &recv_full[chunk];
    const uint32_t recv_base = smem_u32(smem + Cfg::kRecvOff) + chunk * Cfg::kChunkBytes;
    const uint32_t send_base = smem_u32(smem + Cfg::kSendOff) + chunk * Cfg::kChunkBytes;
    const int srow = kSplit == 2 ? chunk * 32 + lane : quarter * 32 + lane;  // stage-1 staging row
    // Stage 2: warp w takes staging rows srow0 .. srow0 + kWarpRows - 1, which hold tile rows
    // row0 .. row0 + kWarpRows - 1.
    const int srow0 = warp * kWarpRows;
    const int row0 = kSplit == 2
                         ? (srow0 >> 5) * 64 + 32 * static_cast<int>(rank) + (srow0 & 31)
                         : srow0;
    int live_tiles = 0;  // split-K: tiles in which this warp's quarter held a token
    if (kSplit == 2) cluster_wait();  // the peer's barriers are initialised
    int j = 0;
    for (int tile = kSplit == 2 ? blockIdx.x >> 1 : blockIdx.x; tile < qa.num_tiles; tile += kSplit == 2 ? gridDim.x >> 1 : gridDim.x, ++j) {
      const int b = j & 1;
      const int m0 = (tile / groups_per_tok) * Cfg::kTileRows;
      const int head_row0 = (tile % groups_per_tok) * kHeads;
      const bool is_q = head_row0 < a.num_heads;
      const bool is_v = head_row0 >= a.num_heads + a.num_kv;
      // Split-K: whether this warp's quarter holds a token of the batch (the same in the peer's
      // warp of the same quarter); chunks of quarters past the batch are not sent.
      const bool live = m0 + 32 * quarter < a.num_tokens;
      if (recv_leader && live) {
        mbar_arrive_expect_tx(recv_bar, Cfg::kChunkBytes);
        ++recv_armed;
      }
      // This warp's stage-2 rows: their facts (into shared memory) and, for query/key heads,
      // their cos/sin at this lane's dims, loaded while the MMAs still run.  The warp's own facts
      // were last read by this warp in the previous tile's stage 2.
      if (lane < kWarpRows) {
        const long long t = m0 + row0 + lane;
        long long slot = -1, cs_row = 0;
        if (t < a.num_tokens) {
          slot = 0;
          if (!is_q) {
            slot = a.slots[t];
            if (slot < 0 || slot >= a.num_slots) {
              atomicOr(status, kErrSlot);
              slot = -1;
            }
          }
          if (!is_v) {
            cs_row = t;
            if (a.positions != nullptr) {
              cs_row = a.positions[t];
              if (cs_row < 0 || cs_row >= a.max_positions) {
                atomicOr(status, kErrPosition);
                cs_row = 0;  // row 0 is used, as kernel A does
              }
            }
          }
        }
        asm volatile("st.shared.v2.b64 [%0], {%1, %2};" ::"r"(meta_base + (row0 + lane) * 16),
                     "l"(slot), "l"(cs_row)
                     : "memory");
      }
      __syncwarp();
      RopeRow rope[kWarpRows];
      if (!is_v) {
        float4 c4[kWarpRows], s4[kWarpRows];
#pragma unroll
        for (int i = 0; i < kWarpRows; ++i) {
          const long long cs_row = ld_meta(meta_base + (row0 + i) * 16).cs_row;
          c4[i] = *reinterpret_cast<const float4*>(a.cos + cs_row * a.cs_row_stride + lane * 4);
          s4[i] = *reinterpret_cast<const float4*>(a.sin + cs_row * a.cs_row_stride + lane * 4);
        }
#pragma unroll
        for (int i = 0; i < kWarpRows; ++i)
          rope[i] = RopeRow{pack_bf16(c4[i].x, c4[i].y), pack_bf16(c4[i].z, c4[i].w),
                            pack_bf16(s4[i].x, s4[i].y), pack_bf16(s4[i].z, s4[i].w)};
      }
      // The q_norm / k_norm weights at this lane's dims (stage 2): loaded ahead where the
      // registers allow (split-K warps hold 4 rows of cos/sin, the others 8).
      uint2 w2 = make_uint2(0u, 0u);
      if (kSplit == 2 && !is_v)
        w2 = *reinterpret_cast<const uint2*>((is_q ? a.q_weight : a.k_weight) + lane * 4);
      // Stage 1: accumulator -> bf16 staging rows (split-K: this CTA's rows only, after adding
      // the peer's partial).  Every epilogue warp reports whether its waits succeeded; all of
      // them leave together if one did not.
      const bool acc_ok =
          __all_sync(0xffffffffu, mbar_wait_fast(&acc_full[b], (j >> 1) & 1, abort_flag));
      tc_fence_after();
      bool mine = acc_ok;  // split-K: also the exchange with the peer succeeded
      if (acc_ok) {
        const uint32_t row_addr = stage_base + srow * Cfg::kRowPitch + colq * 64;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          float v[32];
          tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * Cfg::kTileN +
                        h * 128 + colq * 32,
                    v);
          tmem_wait_ld();
          if constexpr (kSplit == 2) {
            // Row `lane` of the chunk, columns colq * 32 .. +31, in the send buffer (sender) or
            // the receive buffer (owner).
            const uint32_t xrow = lane * Cfg::kRecvPitch + (h * 128 + colq * 32) * 4;
            if (sender) {
              // The previous tile's copy has left the send buffer once the peer has read it.
              mine = __all_sync(0xffffffffu,
                                j == 0 || mbar_wait_cluster(peer_done, (j - 1) & 1, abort_flag));
              if (mine && live) {
#pragma unroll
                for (int u = 0; u < 8; ++u)
                  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(send_base + xrow + u * 16),
                               "f"(v[4 * u]), "f"(v[4 * u + 1]), "f"(v[4 * u + 2]), "f"(v[4 * u + 3])
                               : "memory");
                fence_proxy_async_smem();  // the bulk copy reads these through the async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(&send_ready[chunk]);
                if (issuer) {
                  bool sent = true;
                  if (lane == 0) {
                    sent = mbar_wait_fast(&send_ready[chunk], live_tiles & 1, abort_flag);
                    if (sent)
                      bulk_copy_to_peer(peer_smem(recv_base, rank ^ 1u), send_base, Cfg::kChunkBytes,
                                        peer_smem(smem_u32(&recv_full[chunk]), rank ^ 1u));
                  }
                  mine = __all_sync(0xffffffffu, sent);
                }
              }
              continue;  // the sender stages nothing
            }
            if (live) {
              mine = __all_sync(0xffffffffu,
                                mbar_wait_cluster(&recv_full[chunk], live_tiles & 1, abort_flag));
              if (!mine) continue;
              if (recv_leader) recv_seen = recv_armed;
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                float4 o;
                asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(o.x), "=f"(o.y), "=f"(o.z), "=f"(o.w)
                             : "r"(recv_base + xrow + u * 16));
                v[4 * u] += o.x;
                v[4 * u + 1] += o.y;
                v[4 * u + 2] += o.z;
                v[4 * u + 3] += o.w;
              }
            }
            // Read (or nothing to read): the peer may copy its next partial into this buffer,
            // and may exit once every receiving warp has said so.
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(peer_smem(smem_u32(peer_done), rank ^ 1u));
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float* e = v + u * 8;
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_addr + h * 256 + u * 16),
                         "r"(pack_bf16(e[0], e[1])), "r"(pack_bf16(e[2], e[3])),
                         "r"(pack_bf16(e[4], e[5])), "r"(pack_bf16(e[6], e[7]))
                         : "memory");
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);  // the MMA warp may reuse accumulator b
      }
      if (kSplit == 2 && live) ++live_tiles;
      if (lane == 0) verdict[warp] = (kSplit == 2 ? mine : acc_ok) ? 1 : 0;
      epi_bar_sync();
      bool all_ok = true;
#pragma unroll
      for (int w = 0; w < Cfg::kEpiWarps; ++w) all_ok = all_ok && verdict[w] != 0;
      if (!all_ok) {
        if (lane == 0) atomicOr(status, kErrTimeout);
        if (etid == 0) *abort_flag = 1;  // the producer and the MMA warp stop too
        break;
      }
      // Stage 2: kernel A on the staged rows.
      if (is_v) {
        const int h0 = head_row0 - a.num_heads - a.num_kv;
        __nv_bfloat16* vbase = a.k_pool + 2 * kBlockTokens * 64;
#pragma unroll
        for (int i = 0; i < kWarpRows; ++i) {
          const long long slot = ld_meta(meta_base + (row0 + i) * 16).slot;
          if (slot < 0) continue;
#pragma unroll
          for (int h = 0; h < kHeads; ++h) {
            const uint2 v = ld_shared_v2(stage_base + (srow0 + i) * Cfg::kRowPitch + h * 256 + lane * 8);
            *reinterpret_cast<uint2*>(vbase + pool_offset(slot, h0 + h, lane * 4, a.block_stride,
                                                          a.head_stride)) = v;
          }
        }
      } else {
        if (kSplit == 1)
          w2 = *reinterpret_cast<const uint2*>((is_q ? a.q_weight : a.k_weight) + lane * 4);
        constexpr int kRows = 4 / kHeads;  // rows per batch (register budget)
#pragma unroll
        for (int i = 0; i < kWarpRows; i += kRows)
          norm_rope_rows<kHeads, kRows>(a, stage_base, meta_base, row0 + i, srow0 + i, m0, head_row0, is_q,
                                        w2, rope + i, lane);
      }
      epi_bar_sync();  // the staging tile and the row facts are free for the next tile
    }
    tiles_seen = j;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (kSplit == 2) {
    if (warp >= Cfg::kProducerWarp) cluster_wait();  // their half of the start-up barrier
    // Before the CTA exits: the peer has read every chunk this CTA sent it (so no copy still
    // reads this CTA's send buffer, and no arrival is still on its way here) ...
    if (threadIdx.x == 0 && tiles_seen > 0 && !mbar_wait(peer_done, (tiles_seen - 1) & 1))
      atomicOr(status, kErrTimeout);
    // ... and, after a failed wait, the peer's last copy has landed here (bounded).
    if (recv_seen < recv_armed && !mbar_wait(recv_bar, (recv_armed - 1) & 1))
      atomicOr(status, kErrTimeout);
  }
  if (warp == Cfg::kMmaWarp) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace ms
