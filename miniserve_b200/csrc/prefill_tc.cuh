// Kernel D: chunked-prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the per-chunk SDPA of MiniServe's prefill path (src/miniserve/attention/
// backends.py:182-196) for chunks of more than 64 new tokens.  One CTA owns one work item for one
// KV head: up to 128 query tokens x the 2 query heads of the GQA pair, as two 128-row tiles
// (tile A = tokens 0..63 of the item, tile B = tokens 64..127; row = token * 2 + head), and a
// range of the sequence's KV pages, walked in blocks of 128 keys.
//
//   warps 0-3   softmax for tile A, warps 4-7 softmax for tile B: one thread per row (TMEM lane),
//               224 registers each (the producer / MMA warpgroup gives its registers up).
//               Per block: read the row's 128 scores from TMEM and release the S columns at once
//               (the next S then runs on the tensor core during this block's softmax), causal /
//               range mask (cached length as offset), row max, p = 2^(s*scale*log2e - m) (MUFU),
//               row sum, and P packed to bf16 in registers; then, once
//               this tile's previous P*V has finished with its P buffer in shared memory, P is
//               stored there.  The running max only moves (and O in TMEM is rescaled) when it
//               grows by more than 2^8.
//   warp 8      TMA producer: K and V blocks in consumption order K_0, K_1, V_0, K_2, V_1, ... into
//               a 3-slot ring of 32 KiB.  K: 16 boxes of 2 KiB (8 pages x two 64-dim halves), laid
//               out as [half][128 keys][64] for the K-major operand; V: 8 boxes of 4 KiB (one page
//               each), read as an MN-major operand one page per 16-key step.  One box per lane;
//               pages past the item's range are read from an out-of-range block id, which the TMA
//               unit fills with zeros.
//   warp 11     no role (completes the third warpgroup for the register reconfiguration).
//   warps 9, 10 MMA issuers (warp 9 also allocates the 512 TMEM columns); every MMA takes both
//               operands from shared memory, P included:
//                 warp 9:  S_t(j) = Q_t K_j^T  (M=128, N=128, K=128) once tile t holds S_t(j-1)
//                          in registers
//                 warp 10: O_t += P_t(j) V_j   (M=128, N=128, K=128) once P_t(j) is stored
//               One thread's MMA issue queue is shallow, so a wait in a single issuer idles the
//               tensor core; with two independent streams one keeps it busy while the other waits.
//               The scores of the next block are ready before the softmax needs them and the
//               tensor core never waits for a P store of the same block.  P goes through shared
//               memory, not TMEM: tcgen05.st traffic slows the tensor core, plain stores do not.
//
// TMEM columns: S_A at 0, S_B at 128, O_A at 256, O_B at 384.  Shared memory: Q_A, Q_B, P_A, P_B
// (each [2 halves][128 rows][64] bf16, K-major) and the K/V ring, all 128-byte swizzled with
// 8-row atoms 1024 bytes apart.  Every wait is bounded; on a timeout the CTA records
// kErrTimeout, stops, lets issued MMAs and TMA copies finish, frees TMEM and exits.
#pragma once

#include "paged_attention.cuh"
#include "tc_common.cuh"

namespace ms {

struct TcCfg {
  // 12 warps = 3 warpgroups: softmax tile A, softmax tile B, and producer / MMA issuers (warps
  // 8-10; warp 11 only completes the warpgroup, which register reconfiguration works on).
  static constexpr int kThreads = 384;
  // Registers per thread: 168 at launch (65,536 / 384, rounded down to a multiple of 8); then
  // the softmax warpgroups take 224 and the producer / MMA warpgroup keeps 56:
  // 2 x 128 x 224 + 128 x 56 = 64,512 = 384 x 168, exactly the launch's allocation.
  static constexpr int kLaunchRegs = 168;
  static constexpr int kSoftmaxRegs = 224;
  static constexpr int kOtherRegs = 56;
  static_assert(2 * 128 * kSoftmaxRegs + 128 * kOtherRegs <= kThreads * kLaunchRegs,
                "register split exceeds the launch allocation");
  static constexpr int kSlots = 3;          // K/V ring slots (one 128-key K or V block each)
  static constexpr int kTileTokens = 64;    // query tokens per 128-row tile
  static constexpr int kBlockKeys = 128;
  static constexpr int kQBytes = 32768;     // one tile: [2 halves][128 rows][64]
  static constexpr int kSlotBytes = 32768;  // one 128-key K (or V) block
  static constexpr int kQOff = 0;                          // Q_A, Q_B
  static constexpr int kPOff = 2 * kQBytes;                // P_A, P_B
  static constexpr int kRingOff = kPOff + 2 * kQBytes;     // K/V ring
  static constexpr int kBarOff = kRingOff + kSlots * kSlotBytes;
  static constexpr int kNumBars = 2 * kSlots + 2 + 2 + 2 + 2 + 1 + 2;
  static constexpr int kSmemBytes = 1024 + kBarOff + (kNumBars + 2) * 8;
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

// Causal / range mask of 32 consecutive keys: key i is visible iff i < lim, where lim = (the
// row's first invisible key, min(qpos + 1, key_end)) - (the first of the 32 keys).  Within a block
// the invisible keys of a row are a suffix, so one compare with a constant and one select per
// score suffice.
__device__ __forceinline__ void mask_scores32(float (&v)[32], int lim) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = i < lim ? v[i] : -INFINITY;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ float max128(const float (&s0)[32], const float (&s1)[32],
                                        const float (&s2)[32], const float (&s3)[32]) {
  float mxa[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mxa[i] = fmaxf(fmaxf(s0[i], s1[i]), fmaxf(s2[i], s3[i]));
#pragma unroll
  for (int i = 8; i < 32; ++i)
    mxa[i & 7] = fmaxf(mxa[i & 7], fmaxf(fmaxf(s0[i], s1[i]), fmaxf(s2[i], s3[i])));
  return fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
               fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
}

// p = 2^(s * scale_log2 - m) for 32 scores, accumulated into the pair sums and packed as 16 bf16
// pairs, every exponential on the MUFU unit (scores scaled in pairs with the paired fp32
// instructions).  Moving a share of the pairs to the FMA pipe (a cubic 2^f with exponent-field
// scaling) paid off on an earlier form of this kernel (2 of 8 fastest there), but with the P
// halves, the early start and the exact ring waits the MUFU-only form is the fastest: 0, 1, 2 and
// 3 of 8 give 236.7, 237.5, 245.7 and 255.3 us on an 8192-token prompt.  Masked scores (-inf)
// give 0, so blocks with and without masked scores run this same code: with a separate form for
// masked blocks, a warpgroup in its diagonal block and the other warpgroup in an unmasked block
// ran two different unrolled loops side by side, and the diagonal block took ~2.3x as long.
__device__ __forceinline__ void exp_pack32(const float (&sv)[32], float2 sc2, float2 nm2,
                                           float2 (&suma)[4], uint32_t (&packed)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), sc2, nm2);
    const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    suma[i & 3] = __fadd2_rn(suma[i & 3], p);
    packed[i] = pack_bf16(p.x, p.y);
  }
}

__global__ void __launch_bounds__(TcCfg::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap k_map,
                      const __grid_constant__ CUtensorMap v_map, const AttnArgs a) {
  // Programmatic dependent launch.  The plan (items, sequence records, block tables) was uploaded
  // before the kernel preceding this one started, and the K/V rows of keys below a sequence's
  // cached length were written by earlier steps, so the producer reads the plan and streams the
  // blocks made only of such keys before griddepcontrol.wait, while the previous kernel finishes.
  // Everything else (the queries, this step's K/V rows, every store) comes after the wait, which
  // every thread executes.  Each thread triggers the dependents only after its own wait: a grid
  // launched behind this one then knows that the kernel before this one has completed (the
  // persistent decode kernel relies on it for cascade plans).
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int NS = TcCfg::kSlots;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcCfg::kBarOff);
  uint64_t* slot_full = bars;              // [NS]
  uint64_t* slot_empty = slot_full + NS;   // [NS]
  uint64_t* s_full = slot_empty + NS;      // [tile]: S_t(j) computed
  uint64_t* s_free = s_full + 2;           // [tile]: S_t(j) read into registers
  uint64_t* p_full = s_free + 2;           // [tile]: P_t(j) stored (and O_t rescaled)
  uint64_t* pv_done = p_full + 2;          // [tile]: O_t += P_t(j) V_j finished
  uint64_t* mma_drain = pv_done + 2;
  uint64_t* q_ready = mma_drain + 1;      // both Q tiles stored in shared memory
  uint64_t* tmem_ready = q_ready + 1;     // the TMEM allocation's address is in tmem_holder
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + TcCfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + TcCfg::kNumBars + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int item_idx = blockIdx.x / a.num_kv;
  const int kvh = blockIdx.x - item_idx * a.num_kv;
  const int* it = a.items + static_cast<long long>(item_idx) * kRec;
  const int seq = it[0], page_begin = it[3], page_end = it[4], part_row = it[5];
  // First token (inside the chunk) and token count of tile A and tile B (B's count may be 0).
  const int tok_a = it[1], n_a = it[2], tok_b = it[6], n_b = it[7];
  const int* sr = a.seqs + static_cast<long long>(seq) * kRec;
  const int flat_start = sr[0], num_cached = sr[2], table_off = sr[4];
  const int npages = page_end - page_begin;
  const int key_lo = page_begin * kBlockTokens;
  const int key_end = page_end * kBlockTokens;
  // Blocks each tile sees inside this item's page range (a tile's last visible key is
  // num_cached + its last token).  Tile A never sees more blocks than tile B, unless B is empty.
  int nblk_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int ntok = t == 0 ? n_a : n_b;
    const int vis_end = min(key_end, num_cached + (t == 0 ? tok_a : tok_b) + ntok);
    nblk_t[t] = (ntok <= 0 || vis_end <= key_lo)
                    ? 0
                    : (vis_end - key_lo + TcCfg::kBlockKeys - 1) / TcCfg::kBlockKeys;
  }
  const int nblk = max(nblk_t[0], nblk_t[1]);
  // Ring positions: K_0 first, then K_{j+1} (if any) and V_j for j = 0, 1, ...
  auto pos_k = [](int j) { return j == 0 ? 0 : 2 * j - 1; };
  auto pos_v = [nblk](int j) { return j + 1 < nblk ? 2 * j + 2 : 2 * j + 1; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 128);
      mbar_init(&p_full[t], 128);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(mma_drain, 2);
    mbar_init(q_ready, 256);
    mbar_init(tmem_ready, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Start-up overlaps: once the barriers exist the producer streams K and V at once, while the
  // softmax warps load Q and warp 9 allocates TMEM; only the first S waits for Q.
  __syncthreads();
  uint32_t tmem = 0;
  // Waits until warp 9 has published the TMEM allocation; on a timeout records it and stops.
  auto wait_tmem = [&]() -> bool {
    const bool ok = mbar_wait_fast(tmem_ready, 0, abort_flag);
    tc_fence_after();
    if (ok) {
      tmem = *tmem_holder;
    } else if (lane == 0) {
      atomicOr(&g_status_word, kErrTimeout);
      *abort_flag = 1;
    }
    return ok;
  };
  // One branch per warpgroup role, each starting with its register budget (the compiler gives a
  // branch the registers of the setmaxnreg that begins it).  The softmax warpgroups hold a whole
  // 128-score block and its 64 packed P words at once; the producer and the MMA issuers need
  // few registers.
  if (warp >= 8) {
    setmaxnreg_dec<TcCfg::kOtherRegs>();
    if (warp != 8) {
      pdl_wait();
      pdl_trigger();
    }
    if (warp == 8) {
      // ---------------- TMA producer ----------------
      // Position p goes to slot p % NS once every MMA that read position p - NS has finished.
      // K: lanes 0..15 issue one 2 KiB box each (page lane / 2, 64-dim half lane % 2) into
      // [half][128 keys][64]; V: lanes 0..7 issue one 4 KiB box each (page lane) into [page][half]
      // [16 keys][64].
      const int* table = a.tables + table_off + page_begin;
      int ids_j = (lane < 8 && lane < npages) ? table[lane] : -1;           // block j's pages
      int ids_j1 = (lane < 8 && 8 + lane < npages) ? table[8 + lane] : -1;  // block j + 1's
      int issued = 0;
      bool waited = false;
      auto wait_prev = [&]() {
        if (!waited) {
          pdl_wait();
          pdl_trigger();
          waited = true;
        }
      };
      auto load = [&](int p, bool is_v, int ids, int j) -> bool {
        // Block j holds a key of this step (written by the previous kernel) unless all its keys
        // are below the cached length.
        if (key_lo + (j + 1) * TcCfg::kBlockKeys > num_cached) wait_prev();
        const int s = p % NS;
        int ok = 1;
        if (!is_v && lane < 8 && j * 8 + lane < npages &&
            static_cast<unsigned>(ids) >= static_cast<unsigned>(a.num_blocks))
          atomicOr(&g_status_word, kErrBlock);
        if (lane == 0) {
          if (*abort_flag) ok = 0;
          if (ok && p >= NS && !mbar_wait(&slot_empty[s], ((p / NS) - 1) & 1)) {
            atomicOr(&g_status_word, kErrTimeout);
            *abort_flag = 1;
            ok = 0;
          }
          if (ok) mbar_arrive_expect_tx(&slot_full[s], TcCfg::kSlotBytes);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return false;
        uint8_t* slot = smem + TcCfg::kRingOff + s * TcCfg::kSlotBytes;
        if (is_v) {
          const int b = __shfl_sync(0xffffffffu, ids, lane & 7);
          if (lane < 8) tma_load_5d_plain(slot + lane * kPageBytes, &v_map, &slot_full[s], 0, 0, 2, kvh, b);
        } else {
          const int b = __shfl_sync(0xffffffffu, ids, (lane & 15) >> 1);
          if (lane < 16) {
            const int pg = lane >> 1, half = lane & 1;
            tma_load_5d_plain(slot + half * 16384 + pg * (kPageBytes / 2), &k_map, &slot_full[s], 0,
                              0, half, kvh, b);
          }
        }
        __syncwarp();
        ++issued;
        return true;
      };
      if (nblk > 0 && load(pos_k(0), false, ids_j, 0)) {
        for (int j = 0; j < nblk; ++j) {
          if (j + 1 < nblk && !load(pos_k(j + 1), false, ids_j1, j + 1)) break;
          if (!load(pos_v(j), true, ids_j, j)) break;
          ids_j = ids_j1;
          ids_j1 = (lane < 8 && (j + 2) * 8 + lane < npages) ? table[(j + 2) * 8 + lane] : -1;
        }
      }
      wait_prev();
      // No copy may still be landing when the CTA exits: wait for the last use of each slot.
      if (lane == 0) {
        for (int p = issued > NS ? issued - NS : 0; p < issued; ++p) {
          if (!mbar_wait(&slot_full[p % NS], (p / NS) & 1)) {
            atomicOr(&g_status_word, kErrTimeout);
            break;
          }
        }
      }
    } else if (warp == 9 || warp == 10) {
      if (warp == 9) {
        tmem_alloc(tmem_holder, TcCfg::kTmemCols);
        tmem_relinquish();
        tc_fence_before();
        if (lane == 0) mbar_arrive(tmem_ready);
      }
      if (wait_tmem()) {
        // ---------------- MMA issuers: warp 9 issues every S = Q K^T, warp 10 every O += P V ------
        // Two issuing threads, two independent MMA streams (different TMEM columns and operands): the
        // issue queue of one thread is shallow, so any wait in a single issuer would leave the tensor
        // core idle; with two, one stream keeps it busy while the other waits.  tcgen05.commit tracks
        // the MMAs of the committing thread only, so each stream signals its own barriers.
        if (lane == 0) {
          const bool is_pv = warp == 10;
          constexpr uint32_t kIdescS = umma_idesc_bf16(128, 128, false);
          constexpr uint32_t kIdescPV = umma_idesc_bf16(128, 128, true);
          const uint32_t ring = smem_u32(smem + TcCfg::kRingOff);
          bool ok = true;
          auto wait_slot = [&](int p) -> bool {
            return mbar_wait_mma(&slot_full[p % NS], (p / NS) & 1, abort_flag);
          };
          // Descriptors are built once; operand offsets are added to their start-address field
          // (shared-memory addresses >> 4 fit its 14 bits with room to spare).
          const uint64_t dq = umma_smem_desc_sw128(smem_u32(smem + TcCfg::kQOff), 16, 1024);
          const uint64_t dp = umma_smem_desc_sw128(smem_u32(smem + TcCfg::kPOff), 16, 1024);
          const uint64_t dk = umma_smem_desc_sw128(ring, 16, 1024);
          const uint64_t dv = umma_smem_desc_sw128(ring, 2048, 1024);  // [page][half][16 keys][64]
          constexpr uint32_t kSlot16 = TcCfg::kSlotBytes >> 4;
          if (!is_pv) {
            // S_t(j) = Q_t K_j^T into tile t's S columns, as soon as tile t holds S_t(j-1) in
            // registers and K_j has landed (and, for S(0), Q is stored).  The tiles are not coupled:
            // each goes as soon as its own softmax has released its S columns.
            // The ring's full barriers are waited on by parity, which is exact only while the
            // slot's previous fill has completed.  K_j's slot last held V_{j-3} (K_2's held K_0,
            // which this thread waited for): K_j is waited on after the first tile's s_free(j - 1),
            // which that tile's softmax arrives on after its wait for P*V(j - 3), so V_{j-3} had
            // landed.
            ok = nblk == 0 || mbar_wait_mma(q_ready, 0, abort_flag);
            for (int j = 0; ok && j < nblk; ++j) {
              const uint64_t kd = dk + (pos_k(j) % NS) * kSlot16;
              bool k_landed = false;
              for (int t = 0; ok && t < 2; ++t) {
                if (j < nblk_t[t]) {
                  if (j > 0 && !(ok = mbar_wait_mma(&s_free[t], (j - 1) & 1, abort_flag))) break;
                  if (!k_landed) {
                    if (!(ok = wait_slot(pos_k(j)))) break;
                    k_landed = true;
                  }
                  tc_fence_after();
                  const uint64_t qd = dq + t * (TcCfg::kQBytes >> 4);
#pragma unroll
                  for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    umma_bf16_ss(tmem + t * 128, qd + off, kd + off, kIdescS, kk > 0 ? 1u : 0u);
                  }
                  umma_commit(&s_full[t]);
                }
              }
              if (!ok) break;
              umma_commit(&slot_empty[pos_k(j) % NS]);
            }
          } else {
            // O_t += P_t(j) V_j once tile t's P(j) is stored and V_j has landed.  Within an entry
            // the tiles go in the order their P becomes ready, so a tile whose softmax runs late
            // (its diagonal block, or its epilogue beside the other tile) does not hold the other
            // tile's P*V back.  Each tile's p_full phase is j: it takes part in entries 0 .. n - 1.
            // V_j's slot last held K_j (the last block's, V_{j-2}, which this thread waited for),
            // so V_j is waited on (by parity, exact only once that fill has completed) after the
            // first P(j) is ready: P(j) follows S(j), which read K_j.
            for (int j = 0; ok && j < nblk; ++j) {
              const uint64_t vd = dv + (pos_v(j) % NS) * kSlot16;
              bool v_landed = false;
              int pend = (j < nblk_t[0] ? 1 : 0) | (j < nblk_t[1] ? 2 : 0);
              for (int i = 0; pend != 0; ++i) {
                const int t = ((pend & 1) && mbar_test_wait(&p_full[0], j & 1))   ? 0
                              : ((pend & 2) && mbar_test_wait(&p_full[1], j & 1)) ? 1
                                                                                  : -1;
                if (t >= 0) {
                  if (!v_landed) {
                    if (!(ok = wait_slot(pos_v(j)))) break;
                    v_landed = true;
                  }
                  tc_fence_after();
#pragma unroll
                  for (int kk = 0; kk < 8; ++kk)
                    umma_bf16_ss(tmem + TcCfg::kOCol + t * 128,
                                 dp + t * (TcCfg::kQBytes >> 4) +
                                     (((kk >> 2) * 16384 + (kk & 3) * 32) >> 4),
                                 vd + kk * (kPageBytes >> 4), kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
                  umma_commit(&pv_done[t]);
                  pend &= ~(1 << t);
                } else if (i >= 16 * kSpinLimit || ((i & 63) == 63 && *abort_flag)) {
                  ok = false;  // the same bound and abort check as mbar_wait_mma
                  break;
                }
              }
              if (!ok) break;
              umma_commit(&slot_empty[pos_v(j) % NS]);
            }
          }
          if (!ok) {
            atomicOr(&g_status_word, kErrTimeout);
            *abort_flag = 1;
          }
          // Every MMA issued so far (by both issuers) must finish before TMEM is freed or the CTA
          // exits: each issuer commits once to mma_drain (two arrivals complete it).
          umma_commit(mma_drain);
          if (!mbar_wait(mma_drain, 0)) atomicOr(&g_status_word, kErrTimeout);
        }
        __syncwarp();
      }
    }
  } else {
    setmaxnreg_inc<TcCfg::kSoftmaxRegs>();
    pdl_wait();
    pdl_trigger();
      // Q tiles into the swizzled K-major layout: 256 rows (2 tiles x 64 tokens x 2 heads) of 16
      // chunks of 16 bytes; each load instruction of a warp covers two whole rows (512 contiguous
      // bytes: one token's two heads), so the loads coalesce.  All 16 loads are issued before any
      // store (a shared store between them would make each load wait for the previous one).
      uint4 v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int f = i * 256 + threadIdx.x;
        const int t = f >> 11, r = (f >> 4) & 127, u = f & 15;
        const bool valid = (r >> 1) < (t == 0 ? n_a : n_b);
        const int tok = (t == 0 ? tok_a : tok_b) + (r >> 1);
        const __nv_bfloat16* src = a.q + static_cast<long long>(flat_start + tok) * a.q_row_stride +
                                   (kvh * kGroup + (r & 1)) * kHeadDim + u * 8;
        v[i] = valid ? __ldg(reinterpret_cast<const uint4*>(src)) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int f = i * 256 + threadIdx.x;
        const int t = f >> 11, r = (f >> 4) & 127, u = f & 15;
        st_shared_v4(smem_u32(smem + TcCfg::kQOff + t * TcCfg::kQBytes) + tile128_off(r, u), v[i].x,
                     v[i].y, v[i].z, v[i].w);
      }
      fence_proxy_async_smem();
      mbar_arrive(q_ready);
    if (wait_tmem()) {
        // ---------------- softmax warpgroups: thread = row of tile t ----------------
        const int t = warp >> 2;
        const int r = threadIdx.x & 127;
        const bool valid = (r >> 1) < (t == 0 ? n_a : n_b);
        const int tok = (t == 0 ? tok_a : tok_b) + (r >> 1);
        const int qpos = num_cached + tok;
        const int nb = nblk_t[t];
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + t * 128;
        const uint32_t o_addr = tmem + lane_base + TcCfg::kOCol + t * 128;
        const uint32_t p_row = smem_u32(smem + TcCfg::kPOff + t * TcCfg::kQBytes) + r * 128;
        const uint32_t r7 = static_cast<uint32_t>(r & 7);
        const float ninf = -INFINITY;
        const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
        float m = ninf, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
          ok = __all_sync(0xffffffffu, mbar_wait_fast(&s_full[t], j & 1, abort_flag));
          if (!ok) break;
          tc_fence_after();
          const int k0 = key_lo + j * TcCfg::kBlockKeys;
          const bool need_mask =
              (k0 + TcCfg::kBlockKeys - 1 > qpos) || (k0 + TcCfg::kBlockKeys > key_end);
          // All 128 scores of the row come out of TMEM in one read, after which S_t is released at
          // once: the MMA computes S_t(j + 1) while this block's max, exponentials and P run.
          float2 suma[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) suma[i] = make_float2(0.f, 0.f);
          uint32_t pk[4][16];
          float alpha = 1.f;
          bool rescale = false;
          float s0[32], s1[32], s2[32], s3[32];
          tmem_ld32(s_addr, s0);
          tmem_ld32(s_addr + 32, s1);
          tmem_ld32(s_addr + 64, s2);
          tmem_ld32(s_addr + 96, s3);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(&s_free[t]);  // the MMA may now overwrite S_t with S_t(j + 1)
          if (need_mask) {
            const int lim = min(qpos + 1, key_end) - k0;
            mask_scores32(s0, lim);
            mask_scores32(s1, lim - 32);
            mask_scores32(s2, lim - 64);
            mask_scores32(s3, lim - 96);
          }
          {
            const float mx = max128(s0, s1, s2, s3) * a.scale_log2;
            // The running max m only moves (and O is rescaled) when the block's max exceeds it by
            // more than 2^8.
            if (mx > m + 8.f) {
              alpha = fast_exp2(m - mx);
              rescale = j > 0;
              m = mx;
            }
          }
          const float neg_mu = m == ninf ? 0.f : -m;
          const float2 nm2 = make_float2(neg_mu, neg_mu);
          // P goes out in two halves (keys 0-63, 64-127): the first half's stores drain through
          // the shared-memory pipe while the second half's exponentials run.
          exp_pack32(s0, sc2, nm2, suma, pk[0]);
          exp_pack32(s1, sc2, nm2, suma, pk[1]);

          // This tile's previous P*V must be complete before its P buffer is overwritten and before
          // O is rescaled.  It is waited on every block, in order, so a parity wait is never
          // satisfied by an older phase; it was issued a whole block ago, so the wait is normally free.
          if (j > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait_fast(&pv_done[t], (j - 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
          }
          const bool any_rescale = __any_sync(0xffffffffu, rescale);
          if (j > 0 && any_rescale) {
            const float f = rescale ? alpha : 1.f;
            for (int c = 0; c < 16; ++c) {
              float ov[8];
              tmem_ld8(o_addr + c * 8, ov);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 8; ++i) ov[i] *= f;
              tmem_st8(o_addr + c * 8, ov);
            }
            tmem_wait_st();
          }
          // P chunk u (keys 8u .. 8u + 7) of row r: K-half u / 8, chunk (u % 8) ^ (r % 8).
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = u >> 2, i = (u & 3) * 4;
            st_shared_v4(p_row + ((u ^ r7) << 4), pk[c][i], pk[c][i + 1], pk[c][i + 2],
                         pk[c][i + 3]);
          }
          exp_pack32(s2, sc2, nm2, suma, pk[2]);
          exp_pack32(s3, sc2, nm2, suma, pk[3]);
#pragma unroll
          for (int u = 8; u < 16; ++u) {
            const int c = u >> 2, i = (u & 3) * 4;
            st_shared_v4(p_row + 16384 + (((u & 7) ^ r7) << 4), pk[c][i], pk[c][i + 1],
                         pk[c][i + 2], pk[c][i + 3]);
          }
          {
            const float2 s01 = __fadd2_rn(suma[0], suma[1]);
            const float2 s23 = __fadd2_rn(suma[2], suma[3]);
            const float2 st = __fadd2_rn(s01, s23);
            l = l * alpha + (st.x + st.y);
          }
          fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(&p_full[t]);
        }
        if (!ok) {
          if (lane == 0) {
            atomicOr(&g_status_word, kErrTimeout);
            *abort_flag = 1;
          }
        } else if (nb > 0) {
          // This tile's last P*V (the phase before it was waited on in the last block).
          ok = __all_sync(0xffffffffu, mbar_wait_fast(&pv_done[t], (nb - 1) & 1, abort_flag));
          if (!ok && lane == 0) {
            atomicOr(&g_status_word, kErrTimeout);
            *abort_flag = 1;
          }
        }
        if (ok) {
          // Epilogue.  Thread r holds row r of O in TMEM; the rows of a global store are 4 KiB
          // apart (one per token), so stored from the threads directly each 16-byte store of a
          // warp would touch 32 rows (32 L1 wavefronts per instruction, which also starves the
          // other tile's P stores of the shared LSU).  The rows go through this tile's P buffer
          // instead (free: its last P*V has completed) and each warp then writes whole rows: two
          // adjacent 256-byte rows (one token's two heads) per instruction for the output, one
          // 512-byte row per instruction for split-KV partials.  Staging layout: 256 bytes per row
          // as 16 chunks of 16 bytes, chunk u of row r at chunk u ^ (r % 16), so the row-wise
          // writes and the two-row reads are both free of bank conflicts.
          tc_fence_after();
          const float inv = l > 0.f ? 1.f / l : 0.f;
          const uint32_t stg = smem_u32(smem + TcCfg::kPOff + t * TcCfg::kQBytes);
          const int n_t = t == 0 ? n_a : n_b;
          const int tok_t = t == 0 ? tok_a : tok_b;
          const int wrow0 = (warp & 3) * 32;  // this warp's rows
          const uint32_t rsw = static_cast<uint32_t>(r & 15);
          // Columns [c0, c0 + 64) of this thread's row, scaled by 1 / l, into the staging row:
          // bf16 (32 columns = 4 chunks) or fp32 (64 columns fill the whole 256-byte row).
          auto stage_cols = [&](int c0, bool as_bf16) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              float ov[32];
              if (nb > 0) {
                tmem_ld32(o_addr + c0 + c * 32, ov);
                tmem_wait_ld();
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) ov[i] = 0.f;
              }
              if (as_bf16) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const uint32_t chunk = static_cast<uint32_t>((c0 / 32 + c) * 4 + u);
                  st_shared_v4(stg + r * 256 + ((chunk ^ rsw) << 4),
                               pack_bf16(ov[8 * u] * inv, ov[8 * u + 1] * inv),
                               pack_bf16(ov[8 * u + 2] * inv, ov[8 * u + 3] * inv),
                               pack_bf16(ov[8 * u + 4] * inv, ov[8 * u + 5] * inv),
                               pack_bf16(ov[8 * u + 6] * inv, ov[8 * u + 7] * inv));
                }
              } else {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const uint32_t chunk = static_cast<uint32_t>(c * 8 + u);
                  st_shared_v4(stg + r * 256 + ((chunk ^ rsw) << 4),
                               __float_as_uint(ov[4 * u] * inv), __float_as_uint(ov[4 * u + 1] * inv),
                               __float_as_uint(ov[4 * u + 2] * inv),
                               __float_as_uint(ov[4 * u + 3] * inv));
                }
              }
            }
          };
          const int u = lane & 15;
          if (part_row < 0) {
            stage_cols(0, true);
            stage_cols(64, true);
            __syncwarp();
#pragma unroll 4
            for (int i = 0; i < 16; ++i) {
              const int R = wrow0 + 2 * i + (lane >> 4);
              uint4 v;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                           : "r"(stg + R * 256 + ((static_cast<uint32_t>(u) ^ (R & 15)) << 4)));
              if ((R >> 1) < n_t)
                *reinterpret_cast<uint4*>(
                    a.out + static_cast<long long>(flat_start + tok_t + (R >> 1)) * a.out_row_stride +
                    (kvh * kGroup + (R & 1)) * kHeadDim + u * 8) = v;
            }
          } else {
            // Row inside the item's partial rows (split items have adjacent tiles: token order).
            if (valid) {
              const long long prow = static_cast<long long>(part_row + t * 128 + r) * a.num_kv + kvh;
              a.ws_lse[prow] = l > 0.f ? m + __log2f(l) : -INFINITY;
            }
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
              stage_cols(half * 64, false);
              __syncwarp();
#pragma unroll 4
              for (int i = 0; i < 16; ++i) {
                const int R = wrow0 + 2 * i + (lane >> 4);
                uint4 v;
                asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                             : "r"(stg + R * 256 + ((static_cast<uint32_t>(u) ^ (R & 15)) << 4)));
                if ((R >> 1) < n_t) {
                  const long long prow = static_cast<long long>(part_row + t * 128 + R) * a.num_kv + kvh;
                  *reinterpret_cast<uint4*>(a.ws_o + prow * kHeadDim + half * 64 + u * 4) = v;
                }
              }
              __syncwarp();  // the next half reuses the staging rows
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
