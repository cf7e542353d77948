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

template <int kHeads>
struct QkvCfg {
  static_assert(kHeads == 1 || kHeads == 2, "one or two heads per tile");
  static constexpr int kEpiWarps = 16;
  static constexpr int kProducerWarp = 16;
  static constexpr int kMmaWarp = 17;
  static constexpr int kThreads = 576;
  static constexpr int kStages = kHeads == 1 ? 5 : 3;
  static constexpr int kTileRows = 128;     // tokens per tile (M)
  static constexpr int kTileN = 128 * kHeads;
  static constexpr int kKStep = 64;         // hidden elements per stage (one 128-byte row)
  static constexpr int kBoxBytes = 16384;   // 128 rows x 128 bytes
  static constexpr int kStageBytes = kBoxBytes * (1 + kHeads);
  static constexpr int kRowPitch = 256 * kHeads + 16;  // staging row: bf16 features + 16-byte skew
  static constexpr int kStagingOff = kStages * kStageBytes;
  static constexpr int kMetaOff = kStagingOff + 128 * kRowPitch;  // [128] {slot, cos/sin row}
  static constexpr int kFlagOff = kMetaOff + 128 * 16;  // [16] int: epilogue warp verdicts
  static constexpr int kBarOff = kFlagOff + 64;
  static constexpr int kNumBars = 2 * kStages + 4 + 1;  // full, empty, acc_full[2], acc_empty[2], drain
  static constexpr int kSmemBytes = 1024 + kBarOff + (kNumBars + 2) * 8;
  static constexpr uint32_t kTmemCols = 256 * kHeads;  // two accumulators
  static_assert(kSmemBytes <= 232448, "kernel E exceeds 227 KiB of shared memory");
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
// key heads, with the rows' cos/sin already in registers.
template <int kHeads, int N>
__device__ __forceinline__ void norm_rope_rows(const NormRopeArgs& a, uint32_t stage_base,
                                               uint32_t meta_base, int row0, int m0,
                                               int head_row0, bool is_q, uint2 w2,
                                               const RopeRow* cs, int lane) {
  using Cfg = QkvCfg<kHeads>;
  const int d0 = lane * 4;
  uint2 raw[N][kHeads];
  long long slot[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    slot[i] = ld_meta(meta_base + (row0 + i) * 16).slot;
#pragma unroll
    for (int h = 0; h < kHeads; ++h)
      raw[i][h] = ld_shared_v2(stage_base + (row0 + i) * Cfg::kRowPitch + h * 256 + lane * 8);
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

template <int kHeads>
__global__ void __launch_bounds__(QkvCfg<kHeads>::kThreads, 1)
    qkv_proj_norm_rope_kernel(const __grid_constant__ CUtensorMap x_map,
                              const __grid_constant__ CUtensorMap w_map, const QkvArgs qa,
                              unsigned* status) {
  pdl_wait();
  pdl_trigger();
  using Cfg = QkvCfg<kHeads>;
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
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + Cfg::kNumBars + 1);
  const NormRopeArgs& a = qa.e;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups_per_tok = (a.num_heads + 2 * a.num_kv) / kHeads;
  const int ksteps = qa.hidden / Cfg::kKStep;

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
  const uint32_t tmem = *tmem_holder;

  if (warp == Cfg::kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&x_map);
      tma_prefetch_desc(&w_map);
      int g = 0;  // stages issued so far (over all of this CTA's tiles)
      for (int tile = blockIdx.x; tile < qa.num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile / groups_per_tok) * Cfg::kTileRows;
        const int n0 = (tile % groups_per_tok) * Cfg::kTileN;
        for (int k = 0; k < ksteps; ++k, ++g) {
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
      for (int tile = blockIdx.x; ok && tile < qa.num_tiles; tile += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait_mma(&acc_empty[b], ((j >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * Cfg::kTileN;
        for (int k = 0; k < ksteps; ++k, ++g) {
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
            umma_bf16_ss(acc, xd + kk * 2, wd + kk * 2, kIdesc, (k > 0 || kk > 0) ? 1u : 0u);
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
    const int etid = threadIdx.x;  // 0..511
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 = staged rows
    const int colq = warp >> 2;    // columns 32*colq .. +31 of every head
    const uint32_t stage_base = smem_u32(smem + Cfg::kStagingOff);
    const uint32_t meta_base = smem_u32(smem + Cfg::kMetaOff);
    volatile int* verdict = reinterpret_cast<volatile int*>(smem + Cfg::kFlagOff);
    int j = 0;
    for (int tile = blockIdx.x; tile < qa.num_tiles; tile += gridDim.x, ++j) {
      const int b = j & 1;
      const int m0 = (tile / groups_per_tok) * Cfg::kTileRows;
      const int head_row0 = (tile % groups_per_tok) * kHeads;
      const bool is_q = head_row0 < a.num_heads;
      const bool is_v = head_row0 >= a.num_heads + a.num_kv;
      // This warp's 8 stage-2 rows (8w .. 8w + 7): their facts (lanes 0-7, into shared memory)
      // and, for query/key heads, their cos/sin at this lane's dims, loaded while the MMAs still
      // run.  The warp's own facts were last read by this warp in the previous tile's stage 2.
      const int row0 = warp * 8;
      if (lane < 8) {
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
      RopeRow rope[8];
      if (!is_v) {
        float4 c4[8], s4[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const long long cs_row = ld_meta(meta_base + (row0 + i) * 16).cs_row;
          c4[i] = *reinterpret_cast<const float4*>(a.cos + cs_row * a.cs_row_stride + lane * 4);
          s4[i] = *reinterpret_cast<const float4*>(a.sin + cs_row * a.cs_row_stride + lane * 4);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          rope[i] = RopeRow{pack_bf16(c4[i].x, c4[i].y), pack_bf16(c4[i].z, c4[i].w),
                            pack_bf16(s4[i].x, s4[i].y), pack_bf16(s4[i].z, s4[i].w)};
      }
      // Stage 1: accumulator -> bf16 staging rows.  Every epilogue warp reports whether its
      // wait succeeded; all of them leave together if one did not.
      const bool mine =
          __all_sync(0xffffffffu, mbar_wait_fast(&acc_full[b], (j >> 1) & 1, abort_flag));
      tc_fence_after();
      if (mine) {
        const uint32_t row_addr = stage_base + (quarter * 32 + lane) * Cfg::kRowPitch + colq * 64;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          float v[32];
          tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * Cfg::kTileN +
                        h * 128 + colq * 32,
                    v);
          tmem_wait_ld();
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
      if (lane == 0) verdict[warp] = mine ? 1 : 0;
      epi_bar_sync();
      bool all_ok = true;
#pragma unroll
      for (int w = 0; w < Cfg::kEpiWarps; ++w) all_ok = all_ok && verdict[w] != 0;
      if (!all_ok) {
        if (lane == 0) atomicOr(status, kErrTimeout);
        if (etid == 0) *abort_flag = 1;  // the producer and the MMA warp stop too
        break;
      }
      // Stage 2: kernel A on the staged rows; warp w takes rows 8w .. 8w + 7.
      if (is_v) {
        const int h0 = head_row0 - a.num_heads - a.num_kv;
        __nv_bfloat16* vbase = a.k_pool + 2 * kBlockTokens * 64;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const long long slot = ld_meta(meta_base + (row0 + i) * 16).slot;
          if (slot < 0) continue;
#pragma unroll
          for (int h = 0; h < kHeads; ++h) {
            const uint2 v = ld_shared_v2(stage_base + (row0 + i) * Cfg::kRowPitch + h * 256 + lane * 8);
            *reinterpret_cast<uint2*>(vbase + pool_offset(slot, h0 + h, lane * 4, a.block_stride,
                                                          a.head_stride)) = v;
          }
        }
      } else {
        const uint2 w2 = *reinterpret_cast<const uint2*>((is_q ? a.q_weight : a.k_weight) + lane * 4);
        constexpr int kRows = 4 / kHeads;  // rows per batch (register budget: 96)
#pragma unroll
        for (int i = 0; i < 8; i += kRows)
          norm_rope_rows<kHeads, kRows>(a, stage_base, meta_base, row0 + i, m0, head_row0, is_q,
                                        w2, rope + i, lane);
      }
      epi_bar_sync();  // the staging tile and the row facts are free for the next tile
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == Cfg::kMmaWarp) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace ms
