// Kernel D: chunked-prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the per-chunk SDPA of MiniServe's prefill path (src/miniserve/attention/
// backends.py:182-196) for chunks of more than 64 new tokens.  One CTA owns one work item for one
// KV head: up to 128 query tokens x the 2 query heads of the GQA pair, as two 128-row tiles
// (tile A = tokens 0..63 of the item, tile B = tokens 64..127; row = token * 2 + head), and a
// range of the sequence's KV pages, walked in blocks of 128 keys.
//
//   warps 0-3   softmax for tile A, warps 4-7 softmax for tile B: one thread per row (TMEM lane).
//               Per block: read S from TMEM, causal / range mask (cached length as offset), row
//               max, p = 2^(s*scale*log2e - m) (a quarter of them on the FMA pipe), row sum, and P
//               written back as bf16 into the S columns it came from (tcgen05.st).  The running
//               max only moves (and O in TMEM is rescaled) when it grows by more than 2^8.
//   warps 8, 10 TMA producers for K and for V: per 128-key block, 16 boxes of 2 KiB (8 pages x
//               two 64-dim halves, one box per lane) into a 2-stage K ring and a 3-stage V ring;
//               pages past the item's range are read from an out-of-range block id, which the
//               TMA unit fills with zeros.  Separate warps keep K_{j+1} from queueing behind V_j.
//   warp 9      TMEM allocator (512 columns) and, on one thread, the MMA issuer:
//                 S_t(j) = Q_t K_j^T   (M=128, N=128, K=128, A and B from shared memory)
//                 O_t   += P_t(j) V_j  (M=128, N=128, K=128, A = P from TMEM, B from shared memory)
//               in the order S_A(0) S_B(0) | O_A += P_A(0) V_0, S_A(1) | O_B += P_B(0) V_0, S_B(1) |
//               ... so the tensor core works on one tile while the other tile's softmax runs.
//               MMAs execute in issue order, so S_t(j+1) overwrites P_t(j) only after it was read.
//
// TMEM columns: [0,128) S_A / P_A, [128,256) S_B / P_B, [256,384) O_A, [384,512) O_B.
// Operands in shared memory are 128-byte swizzled with 8-row atoms 1024 bytes apart: Q and K
// K-major, V MN-major.  Every wait is bounded; on a timeout the CTA records kErrTimeout, stops,
// lets issued MMAs and TMA copies finish, frees TMEM and exits.
#pragma once

#include "paged_attention.cuh"
#include "tc_common.cuh"

namespace ms {

struct TcCfg {
  static constexpr int kThreads = 352;
  static constexpr int kKStages = 2;
  static constexpr int kVStages = 3;
  static constexpr int kTileTokens = 64;   // query tokens per 128-row tile
  static constexpr int kItemTokens = 128;  // query tokens per work item (two tiles)
  static constexpr int kBlockKeys = 128;
  static constexpr int kQBytes = 32768;     // one tile: [2 halves][128 rows][64]
  static constexpr int kTileBytes = 32768;  // one 128-key K (or V) block
  static constexpr int kQOff = 0;                              // Q_A, Q_B
  static constexpr int kKOff = 2 * kQBytes;                    // K ring
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;  // V ring
  static constexpr int kBarOff = kVOff + kVStages * kTileBytes;
  static constexpr int kSmemBytes = 1024 + kBarOff + 24 * 8;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kOCol = 256;
};

// Byte offset of (row, 16-byte unit u in 0..15) inside a [2 halves][128 rows][128 B] swizzled tile.
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

// 2^x for two arguments on the FMA pipe instead of the MUFU unit (the softmax of a 128x128 score
// block is MUFU-bound otherwise), with the paired fp32 instructions of sm_100 (one FFMA2 / FADD2
// does both lanes), which makes it cheaper per element than the MUFU exponential.  Range
// reduction x = n + f with n = round(x), f in [-1/2, 1/2]: adding 1.5 * 2^23 rounds x to an integer
// held in the low mantissa bits, so no float-to-int conversion is needed.  2^f comes from a cubic
// whose coefficients were fitted here for minimum relative error on [-1/2, 1/2] (max 7.5e-5, far
// below the 2^-9 spacing of the bf16 P it feeds); 2^n is added to the exponent field.  x is
// clamped to [-126, +inf); callers pass x <= 8.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 shifted = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 rounded = __fadd2_rn(shifted, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(rounded, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(make_float2(0.0551716685295105f, 0.0551716685295105f), f,
                        make_float2(0.2426111400127411f, 0.2426111400127411f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  const int nx = __float_as_int(shifted.x) - 0x4B400000;
  const int ny = __float_as_int(shifted.y) - 0x4B400000;
  return make_float2(__int_as_float(__float_as_int(p.x) + (nx << 23)),
                     __int_as_float(__float_as_int(p.y) + (ny << 23)));
}

// The row max of one block's 128 raw scores (masked ones excluded), read from TMEM in 32-column
// chunks with the next chunk's load in flight while the current one is reduced (tcgen05.wait::ld
// waits for every load issued before it, so the buffers alternate).
__device__ __forceinline__ float softmax_max_pass(uint32_t s_addr, bool need_mask, int k0, int qpos,
                                                  int key_end) {
  float buf[2][32];
  float mxa[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mxa[i] = -INFINITY;
  tmem_ld32(s_addr, buf[0]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    if (c + 1 < 4) tmem_ld32(s_addr + (c + 1) * 32, buf[(c + 1) & 1]);
    float* sv = buf[c & 1];
    if (need_mask) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int kp = k0 + c * 32 + i;
        if (kp > qpos || kp >= key_end) sv[i] = -INFINITY;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) mxa[i & 7] = fmaxf(mxa[i & 7], sv[i]);
    if (c + 1 < 4) tmem_wait_ld();
  }
  return fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
               fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
}

// The exponential pass for one row: p = 2^(s * scale_log2 - m) for the 128 scores, read back from
// TMEM with the next chunk's load in flight, the row sum, and P as packed bf16 pairs stored into the
// first 64 columns of the same TMEM region as each chunk finishes (chunk c's 16 columns overwrite
// scores of chunks <= c, already consumed).  Elements are processed in pairs with the paired fp32
// instructions.  kMasked: apply the causal / range mask and use the MUFU for every exponential
// (ex2(-inf) = 0); otherwise 3 of every 8 pairs go to the FMA pipe (exp2_fma2), which balances the
// MUFU pipe against instruction issue when two softmax warps share a sub-partition.  The two forms
// are separate instantiations: choosing per element at run time doubles the cost of the loop.
template <bool kMasked>
__device__ __forceinline__ float softmax_exp_pass(uint32_t s_addr, float scale_log2, float neg_mu,
                                                  int k0, int qpos, int key_end) {
  float buf[2][32];
  float2 suma[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) suma[i] = make_float2(0.f, 0.f);
  const float2 sc2 = make_float2(scale_log2, scale_log2);
  const float2 nm2 = make_float2(neg_mu, neg_mu);
  tmem_ld32(s_addr, buf[0]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    if (c + 1 < 4) tmem_ld32(s_addr + (c + 1) * 32, buf[(c + 1) & 1]);
    const float* sv = buf[c & 1];
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float2 x = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), sc2, nm2);
      float2 p;
      if constexpr (kMasked) {
        const int kp = k0 + c * 32 + 2 * i;
        if (kp > qpos || kp >= key_end) x.x = -INFINITY;
        if (kp + 1 > qpos || kp + 1 >= key_end) x.y = -INFINITY;
        p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
      } else {
        p = (i & 7) < 3 ? exp2_fma2(x) : make_float2(fast_exp2(x.x), fast_exp2(x.y));
      }
      suma[i & 3] = __fadd2_rn(suma[i & 3], p);
      packed[i] = pack_bf16(p.x, p.y);
    }
    tmem_st16(s_addr + c * 16, packed);
    if (c + 1 < 4) tmem_wait_ld();
  }
  tmem_wait_st();
  const float2 s01 = __fadd2_rn(suma[0], suma[1]);
  const float2 s23 = __fadd2_rn(suma[2], suma[3]);
  const float2 st = __fadd2_rn(s01, s23);
  return st.x + st.y;
}

__global__ void __launch_bounds__(TcCfg::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap page_map, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcCfg::kBarOff);
  uint64_t* k_full = bars + 0;    // [kKStages]
  uint64_t* k_empty = bars + 2;   // [kKStages]
  uint64_t* v_full = bars + 4;    // [kVStages]
  uint64_t* v_empty = bars + 7;   // [kVStages]
  uint64_t* s_full = bars + 10;   // [2 tiles]
  uint64_t* p_full = bars + 12;   // [2 tiles]
  uint64_t* o_ready = bars + 14;  // [2 tiles]
  uint64_t* mma_drain = bars + 16;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 18);

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
  const int key_lo = page_begin * kBlockTokens;
  const int key_end = page_end * kBlockTokens;
  // Blocks each tile sees inside this item's page range (a tile's last visible key is
  // num_cached + tok0 + its last token).
  int nblk_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int ntok = min(TcCfg::kTileTokens, n_q - t * TcCfg::kTileTokens);
    const int vis_end = min(key_end, num_cached + tok0 + t * TcCfg::kTileTokens + ntok);
    nblk_t[t] = (ntok <= 0 || vis_end <= key_lo)
                    ? 0
                    : (vis_end - key_lo + TcCfg::kBlockKeys - 1) / TcCfg::kBlockKeys;
  }
  const int nblk = max(nblk_t[0], nblk_t[1]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < TcCfg::kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < TcCfg::kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_ready[s], 1);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_holder, TcCfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp < 8) {
    // Q tiles: thread r loads row r % 128 of tile r / 128 into the swizzled K-major layout.
    const int t = threadIdx.x >> 7, r = threadIdx.x & 127;
    const int tok = t * TcCfg::kTileTokens + (r >> 1);
    const __nv_bfloat16* src = a.q + static_cast<long long>(flat_start + tok0 + tok) * a.q_row_stride +
                               (kvh * kGroup + (r & 1)) * kHeadDim;
    uint8_t* qs = smem + TcCfg::kQOff + t * TcCfg::kQBytes;
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

  if (warp == 8 || warp == 10) {
    // ---------------- TMA producers: warp 8 loads K_0 K_1 ..., warp 10 loads V_0 V_1 ... -----
    // K_j waits until every S that reads K_{j-kKStages} has finished with its slot, V_j until
    // every O += P V_{j-kVStages}.  Lanes 0..15 issue one 2 KiB box each: page lane/2, half lane%2.
    const bool is_v = warp == 10;
    const int stages = is_v ? TcCfg::kVStages : TcCfg::kKStages;
    uint64_t* fulls = is_v ? v_full : k_full;
    uint64_t* empties = is_v ? v_empty : k_empty;
    uint8_t* ring = smem + (is_v ? TcCfg::kVOff : TcCfg::kKOff);
    const int* table = a.tables + table_off + page_begin;
    int issued = 0;
    int next = -1;  // block ids of the next block's pages, loaded one block ahead (lanes 0..7)
    if (lane < 8 && lane < npages) next = table[lane];
    for (int j = 0; j < nblk; ++j) {
      const int s = j % stages;
      const int mine = next;
      next = -1;
      if (lane < 8 && (j + 1) * 8 + lane < npages) next = table[(j + 1) * 8 + lane];
      if (!is_v && lane < 8 && j * 8 + lane < npages &&
          static_cast<unsigned>(mine) >= static_cast<unsigned>(a.num_blocks))
        atomicOr(&g_status_word, kErrBlock);
      int ok = 1;
      if (lane == 0) {
        if (*abort_flag) ok = 0;
        if (ok && j >= stages && !mbar_wait(&empties[s], ((j / stages) - 1) & 1)) {
          atomicOr(&g_status_word, kErrTimeout);
          *abort_flag = 1;
          ok = 0;
        }
        if (ok) mbar_arrive_expect_tx(&fulls[s], TcCfg::kTileBytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const int b = __shfl_sync(0xffffffffu, mine, (lane & 15) >> 1);
      if (lane < 16) {
        const int pg = lane >> 1, half = lane & 1;
        tma_load_5d_plain(ring + s * TcCfg::kTileBytes + half * 16384 + pg * 2048, &page_map,
                          &fulls[s], 0, 0, (is_v ? 2 : 0) + half, kvh, b);
      }
      __syncwarp();
      ++issued;
    }
    if (lane == 0) {
      const int first = issued > stages ? issued - stages : 0;
      for (int j = first; j < issued; ++j) {
        if (!mbar_wait(&fulls[j % stages], (j / stages) & 1)) {
          atomicOr(&g_status_word, kErrTimeout);
          break;
        }
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdescS = umma_idesc_bf16(128, 128, false);
      constexpr uint32_t kIdescPV = umma_idesc_bf16(128, 128, true);
      const uint32_t q_base = smem_u32(smem + TcCfg::kQOff);
      const uint32_t k0base = smem_u32(smem + TcCfg::kKOff);
      const uint32_t v0base = smem_u32(smem + TcCfg::kVOff);
      bool ok = true;
      auto wait_k = [&](int j) -> bool {
        if (*abort_flag || !mbar_wait(&k_full[j % TcCfg::kKStages], (j / TcCfg::kKStages) & 1))
          return false;
        tc_fence_after();
        return true;
      };
      // S_t(j) = Q_t K_j^T into tile t's S columns.
      auto issue_s = [&](int j, int t) {
        const uint32_t kb = k0base + (j % TcCfg::kKStages) * TcCfg::kTileBytes;
        const uint32_t qb = q_base + t * TcCfg::kQBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16_ss(tmem + t * 128, umma_smem_desc_sw128(qb + off, 16, 1024),
                       umma_smem_desc_sw128(kb + off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      if (nblk > 0) {
        ok = wait_k(0);
        if (ok) {
          for (int t = 0; t < 2; ++t)
            if (nblk_t[t] > 0) issue_s(0, t);
          umma_commit(&k_empty[0]);
        }
      }
      for (int j = 0; ok && j < nblk; ++j) {
        if (*abort_flag ||
            !mbar_wait(&v_full[j % TcCfg::kVStages], (j / TcCfg::kVStages) & 1)) {
          ok = false;
          break;
        }
        const uint32_t vb = v0base + (j % TcCfg::kVStages) * TcCfg::kTileBytes;
        bool k_next = false;
        for (int t = 0; t < 2; ++t) {
          if (j < nblk_t[t]) {
            if (*abort_flag || !mbar_wait(&p_full[t], j & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16_ts(tmem + TcCfg::kOCol + t * 128, tmem + t * 128 + kk * 8,
                           umma_smem_desc_sw128(vb + kk * 2048, 16384, 1024), kIdescPV,
                           (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&o_ready[t]);
          }
          if (j + 1 < nblk_t[t]) {
            if (!k_next && !(ok = k_next = wait_k(j + 1))) break;
            issue_s(j + 1, t);
          }
        }
        if (!ok) break;
        umma_commit(&v_empty[j % TcCfg::kVStages]);
        if (k_next) umma_commit(&k_empty[(j + 1) % TcCfg::kKStages]);
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
    // ---------------- softmax warpgroups: thread = row of tile t ----------------
    const int t = warp >> 2;
    const int r = threadIdx.x & 127;
    const int tok = t * TcCfg::kTileTokens + (r >> 1);
    const int qpos = num_cached + tok0 + tok;
    const int nb = nblk_t[t];
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + t * 128;
    const uint32_t o_addr = tmem + lane_base + TcCfg::kOCol + t * 128;
    const float ninf = -INFINITY;
    float m = ninf, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      ok = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(&s_full[t], j & 1));
      if (!ok) break;
      // O += P_{j-1} V_{j-1} was issued before S_t(j), and MMAs complete in order, so o_ready
      // (j-1) is already complete here.  It is still waited on every block, in order, so a parity
      // wait is never satisfied by an older phase.
      if (j > 0) {
        ok = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(&o_ready[t], (j - 1) & 1));
        if (!ok) break;
      }
      tc_fence_after();
      const int k0 = key_lo + j * TcCfg::kBlockKeys;
      const bool need_mask =
          (k0 + TcCfg::kBlockKeys - 1 > qpos) || (k0 + TcCfg::kBlockKeys > key_end);
      const bool warp_masks = __any_sync(0xffffffffu, need_mask);

      // Row max, then p against the running max m, which only moves (and O is rescaled) when the
      // block's max exceeds it by more than 2^8.
      const float mx = softmax_max_pass(s_addr, need_mask, k0, qpos, key_end) * a.scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m + 8.f) {
        alpha = fast_exp2(m - mx);
        rescale = j > 0;
        m = mx;
      }
      const float neg_mu = m == ninf ? 0.f : -m;
      const float sum =
          warp_masks ? softmax_exp_pass<true>(s_addr, a.scale_log2, neg_mu, k0, qpos, key_end)
                     : softmax_exp_pass<false>(s_addr, a.scale_log2, neg_mu, k0, qpos, key_end);
      l = l * alpha + sum;

      // O holds sum_{i<j} P_i V_i; rescale it when the max moved (rare after the first block).
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? alpha : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(o_addr + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= f;
          tmem_st32(o_addr + c * 32, ov);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (!ok) {
      if (lane == 0) {
        atomicOr(&g_status_word, kErrTimeout);
        *abort_flag = 1;
      }
    } else if (nb > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_ready[t], (nb - 1) & 1));
      if (!ok && lane == 0) {
        atomicOr(&g_status_word, kErrTimeout);
        *abort_flag = 1;
      }
    }
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = kvh * kGroup + (r & 1);
      const int prow_r = t * 128 + r;  // row inside the item's 2 * n_q partial rows
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        if (nb > 0) {
          tmem_ld32(o_addr + c * 32, ov);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0.f;
        }
        if (tok < n_q) {
          if (part_row < 0) {
            __nv_bfloat16* dst = a.out +
                                 static_cast<long long>(flat_start + tok0 + tok) * a.out_row_stride +
                                 head * kHeadDim + c * 32;
#pragma unroll
            for (int u = 0; u < 4; ++u)
              reinterpret_cast<uint4*>(dst)[u] =
                  make_uint4(pack_bf16(ov[8 * u] * inv, ov[8 * u + 1] * inv),
                             pack_bf16(ov[8 * u + 2] * inv, ov[8 * u + 3] * inv),
                             pack_bf16(ov[8 * u + 4] * inv, ov[8 * u + 5] * inv),
                             pack_bf16(ov[8 * u + 6] * inv, ov[8 * u + 7] * inv));
          } else {
            const long long prow = static_cast<long long>(part_row + prow_r) * a.num_kv + kvh;
            float* dst = a.ws_o + prow * kHeadDim + c * 32;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              reinterpret_cast<float4*>(dst)[u] = make_float4(
                  ov[4 * u] * inv, ov[4 * u + 1] * inv, ov[4 * u + 2] * inv, ov[4 * u + 3] * inv);
            if (c == 0) a.ws_lse[prow] = l > 0.f ? m + __log2f(l) : -INFINITY;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, TcCfg::kTmemCols);
}

}  // namespace ms
