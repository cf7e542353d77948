// Kernel D: chunked-prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the per-chunk SDPA of MiniServe's prefill path (src/miniserve/attention/
// backends.py:182-196) for chunks of more than 64 new tokens.  One CTA owns one work item for one
// KV head: a tile of 64 query tokens x the 2 query heads of the GQA pair = 128 rows (row =
// token * 2 + head), and a range of the sequence's KV pages, walked in blocks of 128 keys.
//
//   warp 4      TMA producer: per 128-key block, 32 boxes of 2 KiB (8 pages x K lo/hi, V lo/hi)
//               into a 2-stage ring; pages past the item's range are loaded from an out-of-range
//               block id so the TMA unit fills them with zeros.
//   warp 5      TMEM allocator (512 columns) and, on one thread, the MMA issuer:
//                 S_j = Q K_j^T   (M=128, N=128, K=128)  -> TMEM columns [128*(j%2), +128)
//                 O  += P_j V_j   (M=128, N=128, K=128)  -> TMEM columns [256, 384)
//               S_{j+1} is issued before O += P_j V_j so the next scores are ready when the
//               softmax warps finish block j.
//   warps 0-3   one thread per row (TMEM lane = row): read S_j with tcgen05.ld, mask (causal with
//               the cached length as offset, and the item's page range), online softmax in the exp2
//               domain, P_j -> shared memory as bf16 in the 128-byte-swizzled K-major layout the
//               MMA reads.  The running max is only moved (and O in TMEM rescaled) when a row's
//               max grows by more than 2^8, so most blocks skip the O round trip.
//
// Operands: Q and P are K-major (A), K is K-major (B), V is MN-major (B); all 128-byte swizzled
// with 8-row atoms 1024 bytes apart.  Every wait is bounded; on a timeout the CTA records
// kErrTimeout, stops, lets issued MMAs and TMA copies finish, frees TMEM and exits.
#pragma once

#include "paged_attention.cuh"
#include "tc_common.cuh"

namespace ms {

struct TcCfg {
  static constexpr int kThreads = 192;
  static constexpr int kRows = 128;
  static constexpr int kBlockKeys = 128;
  static constexpr int kQBytes = 32768;
  static constexpr int kStageBytes = 65536;  // K 32 KiB + V 32 KiB
  static constexpr int kPBytes = 32768;
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQBytes;
  static constexpr int kPOff = kStageOff + 2 * kStageBytes;
  static constexpr int kBarOff = kPOff + kPBytes;
  static constexpr int kSmemBytes = 1024 + kBarOff + 16 * 8 + 16;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kOCol = 256;
};

// Byte offset of (row, 16-byte unit u in 0..15) inside a [2 chunks][128 rows][128 B] swizzled tile.
__device__ __forceinline__ uint32_t tile128_off(int row, int u) {
  return static_cast<uint32_t>((u >> 3) * 16384 + row * 128 + (((u & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void tma_load_5d_plain(void* smem_dst, const CUtensorMap* map,
                                                  uint64_t* bar, int c0, int c1, int c2, int c3,
                                                  int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_u32(bar))
      : "memory");
}

__global__ void __launch_bounds__(TcCfg::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap page_map, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qs = smem + TcCfg::kQOff;
  uint8_t* ps = smem + TcCfg::kPOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcCfg::kBarOff);
  uint64_t* kv_full = bars + 0;   // [2]
  uint64_t* kv_empty = bars + 2;  // [2]
  uint64_t* s_full = bars + 4;    // [2]
  uint64_t* s_free = bars + 6;    // [2]
  uint64_t* p_full = bars + 8;
  uint64_t* o_ready = bars + 9;
  uint64_t* mma_drain = bars + 10;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 12);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int item_idx = blockIdx.x / a.num_kv;
  const int kvh = blockIdx.x - item_idx * a.num_kv;
  const int* it = a.items + static_cast<long long>(item_idx) * kRec;
  const int seq = it[0], tok0 = it[1], n_q = it[2], page_begin = it[3], page_end = it[4],
            part_row = it[5];
  const int* sr = a.seqs + static_cast<long long>(seq) * kRec;
  const int flat_start = sr[0], num_cached = sr[2], table_off = sr[4];
  const int npages = page_end - page_begin;
  const int nblk = (npages + 7) >> 3;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_ready, 1);
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_holder, TcCfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp < 4) {
    // Q tile: row r = token * 2 + head-in-pair, 256 bytes, into the swizzled K-major layout.
    const int r = threadIdx.x;
    const int tok = r >> 1;
    const __nv_bfloat16* src = a.q + static_cast<long long>(flat_start + tok0 + tok) * a.q_row_stride +
                               (kvh * kGroup + (r & 1)) * kHeadDim;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (tok < n_q) v = reinterpret_cast<const uint4*>(src)[u];
      *reinterpret_cast<uint4*>(qs + tile128_off(r, u)) = v;
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    const int* table = a.tables + table_off + page_begin;
    int issued = 0;
    for (int j = 0; j < nblk; ++j) {
      const int s = j & 1;
      int mine = -1;
      if (lane < 8 && j * 8 + lane < npages) mine = table[j * 8 + lane];
      int ok = 1;
      if (lane == 0) {
        if (*abort_flag) ok = 0;
        if (ok && j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1)) {
          atomicOr(&g_status_word, kErrTimeout);
          *abort_flag = 1;
          ok = 0;
        }
        if (ok) mbar_arrive_expect_tx(&kv_full[s], TcCfg::kStageBytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const int p = lane >> 2, q4 = lane & 3;
      const int blk = __shfl_sync(0xffffffffu, mine, p);
      if (j * 8 + p < npages && static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks))
        atomicOr(&g_status_word, kErrBlock);
      uint8_t* dst = smem + TcCfg::kStageOff + s * TcCfg::kStageBytes + (q4 >> 1) * 32768 +
                     (q4 & 1) * 16384 + p * 2048;
      tma_load_5d_plain(dst, &page_map, &kv_full[s], 0, 0, q4, kvh, blk);
      ++issued;
    }
    if (lane == 0) {
      const int first = issued > 2 ? issued - 2 : 0;
      for (int j = first; j < issued; ++j) {
        if (!mbar_wait(&kv_full[j & 1], (j >> 1) & 1)) {
          atomicOr(&g_status_word, kErrTimeout);
          break;
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdescS = umma_idesc_bf16(128, 128, false);
      constexpr uint32_t kIdescPV = umma_idesc_bf16(128, 128, true);
      const uint32_t q_base = smem_u32(qs);
      const uint32_t p_base = smem_u32(ps);
      const uint32_t stage0 = smem_u32(smem + TcCfg::kStageOff);
      bool ok = true;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (*abort_flag) return false;
        if (!mbar_wait(&kv_full[s], (j >> 1) & 1)) return false;
        if (j >= 2 && !mbar_wait(&s_free[s], ((j >> 1) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t kb = stage0 + s * TcCfg::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16_ss(tmem + s * 128, umma_smem_desc_sw128(q_base + off, 16, 1024),
                       umma_smem_desc_sw128(kb + off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        return true;
      };
      if (nblk > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk && !(ok = issue_s(j + 1))) break;
        if (*abort_flag || !mbar_wait(p_full, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vb = stage0 + (j & 1) * TcCfg::kStageBytes + 32768;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_bf16_ss(tmem + TcCfg::kOCol,
                       umma_smem_desc_sw128(p_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                       umma_smem_desc_sw128(vb + kk * 2048, 16384, 1024), kIdescPV,
                       (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[j & 1]);
        umma_commit(o_ready);
      }
      if (!ok) {
        atomicOr(&g_status_word, kErrTimeout);
        *abort_flag = 1;
      }
      // Every MMA issued so far must finish before TMEM is freed or the CTA exits.
      umma_commit(mma_drain);
      if (!mbar_wait(mma_drain, 0)) atomicOr(&g_status_word, kErrTimeout);
    }
    __syncwarp();
  } else {
    // ---------------- softmax warps: thread = row ----------------
    const int r = threadIdx.x;
    const int tok = r >> 1;
    const int qpos = num_cached + tok0 + tok;
    const int key_lo = page_begin * kBlockTokens;
    const int key_end = page_end * kBlockTokens;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const float ninf = -INFINITY;
    float m = ninf, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(&s_full[b], (j >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      float sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + b * 128 + c * 32, sv[c]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[b]);

      const int k0 = key_lo + j * TcCfg::kBlockKeys;
      const bool need_mask = (k0 + TcCfg::kBlockKeys - 1 > qpos) || (k0 + TcCfg::kBlockKeys > key_end);
      float mx = ninf;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = sv[c][i] * a.scale_log2;
          if (need_mask) {
            const int kp = k0 + c * 32 + i;
            if (kp > qpos || kp >= key_end) v = ninf;
          }
          sv[c][i] = v;
          mx = fmaxf(mx, v);
        }
      }
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m + 8.f) {
        alpha = fast_exp2(m - mx);
        rescale = j > 0;
        m = mx;
      }
      const float mu = m == ninf ? 0.f : m;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p = fast_exp2(sv[c][i] - mu);
          sv[c][i] = p;
          sum += p;
        }
      }
      l = l * alpha + sum;

      if (j > 0) {
        ok = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(o_ready, (j - 1) & 1));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
          const float f = rescale ? alpha : 1.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float ov[32];
            tmem_ld32(tmem + lane_base + TcCfg::kOCol + c * 32, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= f;
            tmem_st32(tmem + lane_base + TcCfg::kOCol + c * 32, ov);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int c = u >> 2, i0 = (u & 3) * 8;
        const uint4 v = make_uint4(pack_bf16(sv[c][i0], sv[c][i0 + 1]),
                                   pack_bf16(sv[c][i0 + 2], sv[c][i0 + 3]),
                                   pack_bf16(sv[c][i0 + 4], sv[c][i0 + 5]),
                                   pack_bf16(sv[c][i0 + 6], sv[c][i0 + 7]));
        *reinterpret_cast<uint4*>(ps + tile128_off(r, u)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (!ok) {
      if (lane == 0) {
        atomicOr(&g_status_word, kErrTimeout);
        *abort_flag = 1;
      }
    } else if (nblk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_ready, (nblk - 1) & 1));
      if (!ok && lane == 0) {
        atomicOr(&g_status_word, kErrTimeout);
        *abort_flag = 1;
      }
    }
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = kvh * kGroup + (r & 1);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tmem + lane_base + TcCfg::kOCol + c * 32, ov);
        tmem_wait_ld();
        if (tok < n_q) {
          if (part_row < 0) {
            __nv_bfloat16* dst = a.out + static_cast<long long>(flat_start + tok0 + tok) * a.out_row_stride +
                                 head * kHeadDim + c * 32;
#pragma unroll
            for (int u = 0; u < 4; ++u)
              reinterpret_cast<uint4*>(dst)[u] =
                  make_uint4(pack_bf16(ov[8 * u] * inv, ov[8 * u + 1] * inv),
                             pack_bf16(ov[8 * u + 2] * inv, ov[8 * u + 3] * inv),
                             pack_bf16(ov[8 * u + 4] * inv, ov[8 * u + 5] * inv),
                             pack_bf16(ov[8 * u + 6] * inv, ov[8 * u + 7] * inv));
          } else {
            const long long prow = static_cast<long long>(part_row + r) * a.num_kv + kvh;
            float* dst = a.ws_o + prow * kHeadDim + c * 32;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              reinterpret_cast<float4*>(dst)[u] = make_float4(ov[4 * u] * inv, ov[4 * u + 1] * inv,
                                                              ov[4 * u + 2] * inv, ov[4 * u + 3] * inv);
            if (c == 0) a.ws_lse[prow] = l > 0.f ? m + __log2f(l) : -INFINITY;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, TcCfg::kTmemCols);
}

}  // namespace ms
