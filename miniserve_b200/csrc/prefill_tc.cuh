// Kernel D: chunked-prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the per-chunk SDPA of MiniServe's prefill path (src/miniserve/attention/
// backends.py:182-196) for chunks of more than 64 new tokens.  One CTA owns one work item for one
// KV head: a tile of 64 query tokens x the 2 query heads of the GQA pair = 128 rows (row =
// token * 2 + head), and a range of the sequence's KV pages, walked in blocks of 128 keys.
//
//   warp 4      TMA producer: per 128-key block, 16 boxes of 2 KiB for K and 16 for V (8 pages x
//               two 64-dim halves) into separate 2-stage K and V rings; pages past the item's
//               range are loaded from an out-of-range block id so the TMA unit fills them with
//               zeros.  K_j's slot frees as soon as S_j is computed, V_j's after O += P_j V_j.
//   warp 5      TMEM allocator (512 columns) and, on one thread, the MMA issuer, in the order
//                 S_0, S_1, [O += P_0 V_0, S_2], [O += P_1 V_1, S_3], ...
//               with S_j = Q K_j^T (M=128, N=128, K=128) in TMEM columns [128*(j%2), +128) and
//               O (M=128, N=128) in columns [256, 384); scores for block j+1 are computed while
//               the softmax warps work on block j.
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
  static constexpr int kTileBytes = 32768;  // one 128-key K (or V) block: [2 halves][128][64]
  static constexpr int kPBytes = 32768;  // one P buffer; two alternate between blocks
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQBytes;                 // K ring: 2 x 32 KiB
  static constexpr int kVOff = kKOff + 2 * kTileBytes;  // V ring: 2 x 32 KiB
  static constexpr int kPOff = kVOff + 2 * kTileBytes;
  static constexpr int kBarOff = kPOff + 2 * kPBytes;
  static constexpr int kSmemBytes = 1024 + kBarOff + 18 * 8;
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

// 2^x evaluated on the FMA pipe instead of the MUFU unit (the softmax of a 128x128 score block is
// MUFU-bound otherwise).  Range reduction x = n + f with n = round(x), f in [-1/2, 1/2]: adding
// 1.5 * 2^23 rounds x to an integer held in the low mantissa bits, so no float-to-int conversion
// is needed.  2^f comes from a cubic whose coefficients were fitted here for minimum relative error
// on [-1/2, 1/2] (max 7.5e-5, far below the 2^-9 spacing of the bf16 P it feeds); 2^n is added to
// the exponent field.  x is clamped to [-126, +inf); callers pass x <= 8.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -126.f);
  const float shifted = x + 12582912.f;
  const int n = __float_as_int(shifted) - 0x4B400000;
  const float f = x - (shifted - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.0551716685295105f, f, 0.2426111400127411f), f,
                            0.6932609677314758f),
                       f, 0.9999280571937561f);
  return __int_as_float(__float_as_int(p) + (n << 23));
}

// Pass 2 of the block softmax for one row: p = 2^(s * scale_log2 - m) for 128 scores read back from
// TMEM in 32-column chunks, row sum into 8 accumulators, bf16 P into its swizzled smem row.
// kMasked: apply the causal / range mask and use the MUFU for every exponential (ex2(-inf) = 0);
// otherwise every fourth exponential goes to the FMA pipe.  The two forms are separate
// instantiations: choosing per element at run time doubles the cost of the loop.
template <bool kMasked>
__device__ __forceinline__ float softmax_exp_pass(uint32_t s_addr, float scale_log2, float neg_mu,
                                                  int k0, int qpos, int key_end, uint8_t* prow,
                                                  int r) {
  float suma[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) suma[i] = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float sv[32];
    tmem_ld32(s_addr + c * 32, sv);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float x = fmaf(sv[i], scale_log2, neg_mu);
      float p;
      if constexpr (kMasked) {
        const int kp = k0 + c * 32 + i;
        if (kp > qpos || kp >= key_end) x = -INFINITY;
        p = fast_exp2(x);
      } else {
        p = (i & 3) == 3 ? exp2_fma(x) : fast_exp2(x);
      }
      sv[i] = p;
      suma[i & 7] += p;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i0 = u * 8;
      const uint4 v = make_uint4(pack_bf16(sv[i0], sv[i0 + 1]), pack_bf16(sv[i0 + 2], sv[i0 + 3]),
                                 pack_bf16(sv[i0 + 4], sv[i0 + 5]), pack_bf16(sv[i0 + 6], sv[i0 + 7]));
      *reinterpret_cast<uint4*>(prow + tile128_off(r, c * 4 + u)) = v;
    }
  }
  return ((suma[0] + suma[1]) + (suma[2] + suma[3])) + ((suma[4] + suma[5]) + (suma[6] + suma[7]));
}

__global__ void __launch_bounds__(TcCfg::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap page_map, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qs = smem + TcCfg::kQOff;
  uint8_t* ps = smem + TcCfg::kPOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcCfg::kBarOff);
  uint64_t* k_full = bars + 0;    // [2]
  uint64_t* k_empty = bars + 2;   // [2]
  uint64_t* v_full = bars + 4;    // [2]
  uint64_t* v_empty = bars + 6;   // [2]
  uint64_t* s_full = bars + 8;    // [2]
  uint64_t* p_full = bars + 12;
  uint64_t* o_ready = bars + 13;
  uint64_t* mma_drain = bars + 14;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 16);

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
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
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
    // Loads K_0 V_0 K_1 V_1 ...; K_j waits for S_{j-2} to finish with its slot, V_j for
    // O += P_{j-2} V_{j-2}.  Lane L loads page L/4 of the block, half (L/2)%2, and K or V by L%2.
    const int* table = a.tables + table_off + page_begin;
    int issued_k = 0, issued_v = 0;
    for (int j = 0; j < nblk; ++j) {
      const int s = j & 1;
      int mine = -1;
      if (lane < 8 && j * 8 + lane < npages) mine = table[j * 8 + lane];
      const int p = lane >> 2;
      const int blk = __shfl_sync(0xffffffffu, mine, p);
      if ((lane & 3) == 0 && j * 8 + p < npages &&
          static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks))
        atomicOr(&g_status_word, kErrBlock);
      bool stop = false;
      for (int kv = 0; kv < 2 && !stop; ++kv) {
        uint64_t* full = kv == 0 ? &k_full[s] : &v_full[s];
        uint64_t* empty = kv == 0 ? &k_empty[s] : &v_empty[s];
        int ok = 1;
        if (lane == 0) {
          if (*abort_flag) ok = 0;
          if (ok && j >= 2 && !mbar_wait(empty, ((j >> 1) - 1) & 1)) {
            atomicOr(&g_status_word, kErrTimeout);
            *abort_flag = 1;
            ok = 0;
          }
          if (ok) mbar_arrive_expect_tx(full, TcCfg::kTileBytes);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          stop = true;
          break;
        }
        // 16 boxes per tile: lanes 0..15 take (page = lane/2, half = lane%2), lanes 16..31 idle.
        if (lane < 16) {
          const int pg = lane >> 1, half = lane & 1;
          const int b = __shfl_sync(0x0000ffffu, mine, pg, 16);
          uint8_t* dst = smem + (kv == 0 ? TcCfg::kKOff : TcCfg::kVOff) + s * TcCfg::kTileBytes +
                         half * 16384 + pg * 2048;
          tma_load_5d_plain(dst, &page_map, full, 0, 0, kv * 2 + half, kvh, b);
        }
        __syncwarp();
        if (kv == 0) ++issued_k; else ++issued_v;
      }
      if (stop) break;
    }
    if (lane == 0) {
      for (int kv = 0; kv < 2; ++kv) {
        const int issued = kv == 0 ? issued_k : issued_v;
        const int first = issued > 2 ? issued - 2 : 0;
        for (int j = first; j < issued; ++j) {
          if (!mbar_wait(kv == 0 ? &k_full[j & 1] : &v_full[j & 1], (j >> 1) & 1)) {
            atomicOr(&g_status_word, kErrTimeout);
            break;
          }
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
      const uint32_t k0base = smem_u32(smem + TcCfg::kKOff);
      const uint32_t v0base = smem_u32(smem + TcCfg::kVOff);
      bool ok = true;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (*abort_flag) return false;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t kb = k0base + s * TcCfg::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16_ss(tmem + s * 128, umma_smem_desc_sw128(q_base + off, 16, 1024),
                       umma_smem_desc_sw128(kb + off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[s]);
        umma_commit(&s_full[s]);
        return true;
      };
      if (nblk > 0) ok = issue_s(0);
      if (ok && nblk > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nblk; ++j) {
        // S_{j+2} overwrites S_j's TMEM buffer: the softmax warps have read it once P_j is ready.
        if (*abort_flag || !mbar_wait(p_full, j & 1) || !mbar_wait(&v_full[j & 1], (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vb = v0base + (j & 1) * TcCfg::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_bf16_ss(tmem + TcCfg::kOCol,
                       umma_smem_desc_sw128(p_base + (j & 1) * TcCfg::kPBytes + (kk >> 2) * 16384 +
                                                (kk & 3) * 32, 16, 1024),
                       umma_smem_desc_sw128(vb + kk * 2048, 16384, 1024), kIdescPV,
                       (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[j & 1]);
        umma_commit(o_ready);
        if (j + 2 < nblk && !(ok = issue_s(j + 2))) break;
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
      const uint32_t s_addr = tmem + lane_base + b * 128;
      const int k0 = key_lo + j * TcCfg::kBlockKeys;
      const bool need_mask = (k0 + TcCfg::kBlockKeys - 1 > qpos) || (k0 + TcCfg::kBlockKeys > key_end);
      const bool warp_masks = __any_sync(0xffffffffu, need_mask);

      // Pass 1: row max of the raw scores, 32 columns at a time, 8 independent accumulators.
      float mxa[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxa[i] = ninf;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float sv[32];
        tmem_ld32(s_addr + c * 32, sv);
        tmem_wait_ld();
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kp = k0 + c * 32 + i;
            if (kp > qpos || kp >= key_end) sv[i] = ninf;
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) mxa[i & 7] = fmaxf(mxa[i & 7], sv[i]);
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                             fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7]))) *
                       a.scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m + 8.f) {
        alpha = fast_exp2(m - mx);
        rescale = j > 0;
        m = mx;
      }
      const float neg_mu = m == ninf ? 0.f : -m;

      // Pass 2 writes P buffer b, last read by O += P_{j-2} V_{j-2}: that product is known to be
      // complete because block j-1 waited for o_ready(j-2).  (o_ready is waited on every block, in
      // order, so a parity wait can never be satisfied by an older phase.)
      // Pass 2 (the form is chosen once per warp).
      uint8_t* prow = ps + b * TcCfg::kPBytes;
      const float sum = warp_masks
                            ? softmax_exp_pass<true>(s_addr, a.scale_log2, neg_mu, k0, qpos, key_end, prow, r)
                            : softmax_exp_pass<false>(s_addr, a.scale_log2, neg_mu, k0, qpos, key_end, prow, r);
      l = l * alpha + sum;

      // O holds sum_{i<j} P_i V_i once O += P_{j-1} V_{j-1} has finished; rescale it (rarely).
      if (j > 0) {
        ok = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(o_ready, (j - 1) & 1));
        if (!ok) break;
      }
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        tc_fence_after();
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
