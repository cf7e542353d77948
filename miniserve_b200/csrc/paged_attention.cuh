// Kernel B: paged attention over the KV pool, read in place through the block tables.
// Kernel C: merge of split-KV partial results.
//
// Replaces the gather + SDPA loops of MiniServe's paged_attention
// (src/miniserve/attention/backends.py:165-196).  One CTA owns one work item for one KV head: a
// tile of query tokens of one sequence (both query heads of the GQA pair folded into the rows,
// row = token * 2 + head-in-pair) and a contiguous range of that sequence's KV pages.
//
//   * A producer warp walks the block table and issues one 8 KiB TMA tensor load per page
//     (K and V of this head, 128-byte swizzled, no multicast) into a ring of shared-memory
//     stages guarded by full/empty mbarriers.
//   * Consumer warps compute S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in, fp32
//     accumulate) and an fp32 online softmax in the exp2 domain.
//   * Decode mode (<= 8 query tokens, 16 rows): each consumer warp takes every 4th page and the
//     warps merge their (m, l, O) in shared memory at the end.
//   * Tile mode (up to 64 query tokens, 128 rows): each consumer warp owns 16 rows; causal
//     masking uses the sequence's cached length as the offset.  A tile of at most 32 tokens
//     (R <= 4 row groups of 16) leaves warps without rows, so the 8 warps form P = 4 (R <= 2) or
//     P = 2 (R <= 4) page phases of 8 / P warps each: warp w takes row group w % (8 / P) and the
//     pages j with j % P == w / (8 / P), and the phases merge their (m, l, O) through the idle
//     ring at the end.  Longer tiles keep one phase: every warp reads every page.
//   * An item that covers the whole visible context writes bf16 output rows directly; a split
//     item writes normalised fp32 partials + log2-sum-exp, merged by kernel C.
//
// The masking rule is the reference's: the query at position num_cached + i sees keys
// 0..num_cached + i (backends.py:123-125, :140-142).
#pragma once

#include "ms_common.cuh"

namespace ms {

// Packed plan records (int32 x 8 each); the host planner writes them.
//   sequence: {flat_start, num_new, num_cached, context_len, table_offset, table_len, 0, 0}
//   item:     {seq, tok0, n_q, page_begin, page_end, part_row (-1 = write output), 0, 0}
//   combine:  {seq, tok0, n_q, part_row0, n_splits, 0, 0, 0}
constexpr int kRec = 8;

struct AttnArgs {
  const __nv_bfloat16* q;  // [T, H, 128]
  long long q_row_stride;
  __nv_bfloat16* out;  // [T, H, 128]
  long long out_row_stride;
  const int* seqs;    // sequence records
  const int* tables;  // flat block tables
  const int* items;   // this launch's items
  int n_items;
  int num_kv;
  int num_blocks;
  float* ws_o;    // [part_rows, KVH, 128] fp32 partials
  float* ws_lse;  // [part_rows, KVH]
  float scale_log2;
};

template <int kMode, int kConsumerWarps, int kStages>
struct AttnCfg {
  static constexpr int kRows = kMode == 0 ? 16 : 16 * kConsumerWarps;
  static constexpr int kThreads = (kConsumerWarps + 1) * 32;
  static constexpr int kStageBytes = kStages * kPageKVBytes;
  static constexpr int kQBytes = kRows * kHeadDim * 2;
  // Decode mode: every warp's 16 rows of (O, m, l).  Tile mode: the lane-ordered (O, m, l) of the
  // warps outside page phase 0 (at most 6 of 8).
  static constexpr int kMergeBytes = kMode == 0 ? kConsumerWarps * 16 * (kHeadDim + 4) * 4 + 2 * kConsumerWarps * 16 * 4
                                                : (kConsumerWarps - kConsumerWarps / 4) * 17 * 32 * 16;
  static_assert(kMergeBytes <= kStageBytes, "merge scratch reuses the stage ring");
  static constexpr int kBarOffset = kStageBytes + kQBytes;
  static constexpr int kSmemBytes = 1024 + kBarOffset + 2 * kStages * 8 + 16;
};

// One 16-key page for one warp's 16 query rows.
__device__ __forceinline__ void attend_page(uint32_t stage, const uint32_t (&qf)[8][4],
                                            float (&o)[16][4], float (&m)[2], float (&l)[2],
                                            int key0, int qpos0, int qpos1, bool need_mask,
                                            float scale_log2, int lane) {
  float s0[4] = {0.f, 0.f, 0.f, 0.f};
  float s1[4] = {0.f, 0.f, 0.f, 0.f};
  const int mi = lane >> 3;
  {
    const int key = (lane & 7) + (mi >> 1) * 8;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(stage + swz_off(key, ks * 16 + (mi & 1) * 8, 16), b0, b1, b2, b3);
      mma_bf16(s0, qf[ks], b0, b1);
      mma_bf16(s1, qf[ks], b2, b3);
    }
  }
  const float ninf = -INFINITY;
  // Scores stay unscaled (scale_log2 > 0 commutes with max); the scale is folded into the
  // exponent's FMA below.
  if (need_mask) {
    const int ka = key0 + 2 * (lane & 3);
    const int kb = ka + 8;
    if (ka > qpos0) s0[0] = ninf;
    if (ka + 1 > qpos0) s0[1] = ninf;
    if (ka > qpos1) s0[2] = ninf;
    if (ka + 1 > qpos1) s0[3] = ninf;
    if (kb > qpos0) s1[0] = ninf;
    if (kb + 1 > qpos0) s1[1] = ninf;
    if (kb > qpos1) s1[2] = ninf;
    if (kb + 1 > qpos1) s1[3] = ninf;
  }
  float mx0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
  float mx1 = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  mx0 *= scale_log2;
  mx1 *= scale_log2;
  // The running max only moves (and O is rescaled) when a row's page max exceeds it by more
  // than 2^8, so p stays below 2^8 and most pages skip the 64 multiplies of the rescale.
  float al0 = 1.f, al1 = 1.f;
  const bool up0 = mx0 > m[0] + 8.f, up1 = mx1 > m[1] + 8.f;
  if (__any_sync(0xffffffffu, up0 || up1)) {
    if (up0) {
      al0 = fast_exp2(m[0] - mx0);
      m[0] = mx0;
    }
    if (up1) {
      al1 = fast_exp2(m[1] - mx1);
      m[1] = mx1;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
  }
  const float mu0 = m[0] == ninf ? 0.f : m[0];
  const float mu1 = m[1] == ninf ? 0.f : m[1];
  float p0[4], p1[4];
  p0[0] = fast_exp2(__fmaf_rn(s0[0], scale_log2, -mu0));
  p0[1] = fast_exp2(__fmaf_rn(s0[1], scale_log2, -mu0));
  p0[2] = fast_exp2(__fmaf_rn(s0[2], scale_log2, -mu1));
  p0[3] = fast_exp2(__fmaf_rn(s0[3], scale_log2, -mu1));
  p1[0] = fast_exp2(__fmaf_rn(s1[0], scale_log2, -mu0));
  p1[1] = fast_exp2(__fmaf_rn(s1[1], scale_log2, -mu0));
  p1[2] = fast_exp2(__fmaf_rn(s1[2], scale_log2, -mu1));
  p1[3] = fast_exp2(__fmaf_rn(s1[3], scale_log2, -mu1));
  l[0] = l[0] * al0 + ((p0[0] + p0[1]) + (p1[0] + p1[1]));
  l[1] = l[1] * al1 + ((p0[2] + p0[3]) + (p1[2] + p1[3]));
  const uint32_t pa[4] = {pack_bf16(p0[0], p0[1]), pack_bf16(p0[2], p0[3]),
                          pack_bf16(p1[0], p1[1]), pack_bf16(p1[2], p1[3])};
  {
    const int key = (lane & 7) + (mi & 1) * 8;
    const uint32_t vbase = stage + kPageBytes;
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vbase + swz_off(key, np * 16 + (mi >> 1) * 8, 16), b0, b1, b2, b3);
      mma_bf16(o[2 * np], pa, b0, b1);
      mma_bf16(o[2 * np + 1], pa, b2, b3);
    }
  }
}

__device__ unsigned g_status_word;

// Named barrier 1 or 2 (bar_id) for `threads` threads, with the id a constant in the instruction
// (a barrier id held in a register makes the compiler reserve all 16 named barriers).
__device__ __forceinline__ void named_bar_1_or_2(int bar_id, int threads) {
  if (bar_id == 1)
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
  else
    asm volatile("bar.sync 2, %0;" ::"r"(threads) : "memory");
}  // device status bits (kErr*), read by ms_device_status

// Decode mode: merge the consumer warps' (m, l, O) over their page subsets through `merge`
// (kConsumerWarps x 16 x (128 / kPasses + 4) fp32 accumulators, then kConsumerWarps x 16 maxima
// and as many sums) and write the rows: bf16 output (merged with a cascade row's shared-prefix
// partial when merge_row >= 0) or fp32 partial rows and log2-sum-exp for split items.  With
// kPasses = 2 the columns go through the scratch in two halves (half the shared memory, two more
// barriers; the same values).  `pre`, when given, holds the cascade row's prefix partial already
// copied into shared memory ([16 rows][128] O, then 16 log2-sum-exp values; the caller waited for
// the kernel that wrote it); otherwise the partial is read from global memory.  `park`, when
// given, receives a cascade row's own result in that layout (normalised O and log2-sum-exp)
// instead of the output, to be merged with the prefix partial later (finish_parked).  Called by the
// kConsumerWarps warps that attended the item (warp = 0 .. kConsumerWarps - 1 among them, tid =
// 0 .. 32 kConsumerWarps - 1), which synchronise on named barrier bar_id.
template <int kConsumerWarps, int kPasses = 1>
__host__ __device__ constexpr int decode_merge_bytes() {
  return kConsumerWarps * 16 * (kHeadDim / kPasses + 4) * 4 + 2 * kConsumerWarps * 16 * 4;
}
constexpr int kPrefixPartialBytes = 16 * kHeadDim * 4 + 16 * 4;  // one unit's [16][128] O + lse
template <int kConsumerWarps, bool kWaitBeforeMerge = false, int kPasses = 1>
__device__ __forceinline__ void decode_merge_store(float* merge, const float (&o)[16][4],
                                                   const float (&m)[2], const float (&l)[2],
                                                   int warp, int lane, int n_q, int kvh,
                                                   int part_row, int merge_row, int flat_start,
                                                   int tok0, const AttnArgs& a, int bar_id = 1,
                                                   int tid = -1, const float* pre = nullptr,
                                                   float* park = nullptr) {
  if (tid < 0) tid = threadIdx.x;
  static_assert(kPasses == 1 || kPasses == 2, "one or two column passes");
  constexpr int kCols = kHeadDim / kPasses;  // columns per pass
  constexpr int kChunks = kCols / 16;        // 16-column chunks per row and pass
  float* mo = merge;
  float* mm = mo + kConsumerWarps * 16 * (kCols + 4);
  float* ml = mm + kConsumerWarps * 16;
#pragma unroll
  for (int pass = 0; pass < kPasses; ++pass) {
    named_bar_1_or_2(bar_id, kConsumerWarps * 32);  // the scratch is free
    {
      float* wo = mo + warp * 16 * (kCols + 4);
      const int ra = lane >> 2, rb = ra + 8, c = 2 * (lane & 3);
#pragma unroll
      for (int nn = 0; nn < 16 / kPasses; ++nn) {
        const int n = pass * (16 / kPasses) + nn;
        *reinterpret_cast<float2*>(wo + ra * (kCols + 4) + nn * 8 + c) = make_float2(o[n][0], o[n][1]);
        *reinterpret_cast<float2*>(wo + rb * (kCols + 4) + nn * 8 + c) = make_float2(o[n][2], o[n][3]);
      }
      if (pass == 0 && (lane & 3) == 0) {
        mm[warp * 16 + ra] = m[0];
        mm[warp * 16 + rb] = m[1];
        ml[warp * 16 + ra] = l[0];
        ml[warp * 16 + rb] = l[1];
      }
    }
    named_bar_1_or_2(bar_id, kConsumerWarps * 32);
    for (int e = tid; e < 16 * kChunks; e += kConsumerWarps * 32) {
      const int r = e / kChunks;
      const int dcl = (e % kChunks) * 16;  // column inside the pass
      const int dc = pass * kCols + dcl;
      const int tok = r >> 1;
      if (tok >= n_q) continue;
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, mm[w * 16 + r]);
      float wsc[kConsumerWarps];
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = mm[w * 16 + r];
        wsc[w] = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
        L += ml[w * 16 + r] * wsc[w];
      }
      const float invL = L > 0.f ? 1.f / L : 0.f;
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float* src = mo + (w * 16 + r) * (kCols + 4) + dcl;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] += src[i] * wsc[w];
      }
      const int head = kvh * kGroup + (r & 1);
      if (park != nullptr) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(park + r * kHeadDim + dc + i) =
              make_float4(acc[i] * invL, acc[i + 1] * invL, acc[i + 2] * invL, acc[i + 3] * invL);
        if (dc == 0) park[16 * kHeadDim + r] = L > 0.f ? mx + __log2f(L) : -INFINITY;
      } else if (part_row < 0) {
        __nv_bfloat16* dst = a.out + static_cast<long long>(flat_start + tok0 + tok) * a.out_row_stride +
                             head * kHeadDim + dc;
        float scale_u = invL;  // weight of this item's own (unnormalised) accumulator
        float wp = 0.f;        // weight of the merged shared-prefix partial
        const float* op = nullptr;
        if (merge_row >= 0) {
          // Cascade row: merge the shared-prefix partial (normalised O and log2-sum-exp) that the
          // tensor-core kernel wrote before this launch: out = (acc 2^(mx-M) + O_p L_p') / (...).
          const long long prow = static_cast<long long>(merge_row + r) * a.num_kv + kvh;
          if constexpr (kWaitBeforeMerge) {
            if (pre == nullptr) pdl_wait();  // the partial is that kernel's output
          }
          const float lse_p = pre != nullptr ? pre[16 * kHeadDim + r] : a.ws_lse[prow];
          const float lse_u = L > 0.f ? mx + __log2f(L) : -INFINITY;
          const float M = fmaxf(lse_u, lse_p);
          const float wu = lse_u == -INFINITY ? 0.f : fast_exp2(lse_u - M);
          wp = lse_p == -INFINITY ? 0.f : fast_exp2(lse_p - M);
          const float inv = wu + wp > 0.f ? 1.f / (wu + wp) : 0.f;
          scale_u = invL * wu * inv;
          wp *= inv;
          op = pre != nullptr ? pre + r * kHeadDim + dc : a.ws_o + prow * kHeadDim + dc;
        }
        if (op != nullptr) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 pv = *reinterpret_cast<const float4*>(op + i);
            acc[i] = acc[i] * scale_u + pv.x * wp;
            acc[i + 1] = acc[i + 1] * scale_u + pv.y * wp;
            acc[i + 2] = acc[i + 2] * scale_u + pv.z * wp;
            acc[i + 3] = acc[i + 3] * scale_u + pv.w * wp;
          }
          scale_u = 1.f;
        }
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pk[i] = pack_bf16(acc[2 * i] * scale_u, acc[2 * i + 1] * scale_u);
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      } else {
        const long long prow = static_cast<long long>(part_row + r) * a.num_kv + kvh;
        float* dst = a.ws_o + prow * kHeadDim + dc;
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(dst + i) =
              make_float4(acc[i] * invL, acc[i + 1] * invL, acc[i + 2] * invL, acc[i + 3] * invL);
        if (dc == 0) a.ws_lse[prow] = L > 0.f ? mx + __log2f(L) : -INFINITY;
      }
    }
  }
}

// A parked cascade row (decode_merge_store's `park`): out = (O_u 2^(lse_u - M) + O_p 2^(lse_p - M))
// / (2^(lse_u - M) + 2^(lse_p - M)) with the shared-prefix partial (O_p, lse_p) read from global
// memory; the caller has waited for the kernel that wrote it, and the parked rows were written
// before a barrier of the same threads.  kT threads (tid = 0 .. kT - 1) share the 16 x 8 chunks.
template <int kT>
__device__ __forceinline__ void finish_parked(const float* park, int n_q, int kvh, int merge_row,
                                              int flat_start, int tok0, const AttnArgs& a,
                                              int tid) {
  for (int e = tid; e < 16 * 8; e += kT) {
    const int r = e >> 3;
    const int dc = (e & 7) * 16;
    const int tok = r >> 1;
    if (tok >= n_q) continue;
    const long long prow = static_cast<long long>(merge_row + r) * a.num_kv + kvh;
    const float lse_p = a.ws_lse[prow];
    const float lse_u = park[16 * kHeadDim + r];
    const float M = fmaxf(lse_u, lse_p);
    float wu = lse_u == -INFINITY ? 0.f : fast_exp2(lse_u - M);
    float wp = lse_p == -INFINITY ? 0.f : fast_exp2(lse_p - M);
    const float inv = wu + wp > 0.f ? 1.f / (wu + wp) : 0.f;
    wu *= inv;
    wp *= inv;
    const float* ou = park + r * kHeadDim + dc;
    const float* op = a.ws_o + prow * kHeadDim + dc;
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 u4 = *reinterpret_cast<const float4*>(ou + i);
      const float4 p4 = *reinterpret_cast<const float4*>(op + i);
      pk[i / 2] = pack_bf16(u4.x * wu + p4.x * wp, u4.y * wu + p4.y * wp);
      pk[i / 2 + 1] = pack_bf16(u4.z * wu + p4.z * wp, u4.w * wu + p4.w * wp);
    }
    const int head = kvh * kGroup + (r & 1);
    __nv_bfloat16* dst =
        a.out + static_cast<long long>(flat_start + tok0 + tok) * a.out_row_stride + head * kHeadDim + dc;
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
}

// kEarly: the launch fits one resident wave (latency-bound); see the programmatic dependent
// launch note at the top of the kernel.
template <int kMode, int kConsumerWarps, int kStages, bool kEarly = false>
__global__ void __launch_bounds__(AttnCfg<kMode, kConsumerWarps, kStages>::kThreads)
    paged_attn_kernel(const __grid_constant__ CUtensorMap kv_map, const AttnArgs a) {
  // Programmatic dependent launch.  A launch that fits one resident wave (kEarly) is
  // latency-bound: its producer reads the plan (copied in before the previous kernel started)
  // and streams the pool pages holding only tokens cached in earlier steps before pdl_wait(),
  // and the consumers wait before loading the queries; this step's K/V rows (written by the
  // previous kernel) and every write come after the wait.  Only kernels of this library run as
  // a programmatic predecessor, and none of them writes an earlier step's pages.  Any other
  // launch waits at once: for a bandwidth-bound launch the early start only competes with the
  // kernel it overlaps (measured 1-2 % slower on config 2).
  if constexpr (!kEarly) pdl_wait();
  pdl_trigger();
  using Cfg = AttnCfg<kMode, kConsumerWarps, kStages>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* qtile = smem + Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int item_idx = blockIdx.x / a.num_kv;
  const int kvh = blockIdx.x - item_idx * a.num_kv;
  const int* it = a.items + static_cast<long long>(item_idx) * kRec;
  const int seq = it[0], tok0 = it[1], n_q = it[2], page_begin = it[3], page_end = it[4],
            part_row = it[5];
  // Decode items of cascade rows (field 7 = 1) merge the shared-prefix partial rows starting at
  // field 6 into their output.
  const int merge_row = (kMode == 0 && it[7] == 1) ? it[6] : -1;
  // Tile mode: page phases (see the top of this file); decode mode splits pages by warp.
  static_assert(kMode == 0 || (kConsumerWarps == 8 && kStages % 4 == 0),
                "tile-mode page phases need 8 consumer warps and a ring of a multiple of 4 stages");
  const int row_groups = (2 * n_q + 15) >> 4;
  const int phases = kMode == 0 ? 1 : (row_groups <= 2 ? 4 : (row_groups <= 4 ? 2 : 1));
  const int phase_warps = kConsumerWarps / phases;  // warps per phase (tile mode)
  const int* sr = a.seqs + static_cast<long long>(seq) * kRec;
  const int flat_start = sr[0], num_cached = sr[2], table_off = sr[4];
  const int npages = page_end - page_begin;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMode == 0 ? 1 : phase_warps);  // the warps that read the page
    }
    *abort_flag = 0;
    fence_barrier_init();
  }

  // The producer starts streaming pages as soon as the barriers exist; the consumer warps load
  // the query tile meanwhile and synchronise among themselves (named barrier 1).
  __syncthreads();
  if (warp < kConsumerWarps) {
    if constexpr (kEarly) pdl_wait();
    // Query tile -> shared memory, swizzled like a page: [16-row group][d/64][row][d%64].  All of
    // a thread's loads are issued before its shared stores (a store between them would make each
    // load wait for the previous one).
    constexpr int kPer = Cfg::kRows * 16 / (kConsumerWarps * 32);
    static_assert(Cfg::kRows * 16 % (kConsumerWarps * 32) == 0, "query chunks per thread");
    uint4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = threadIdx.x + k * kConsumerWarps * 32;
      const int r = c >> 4;
      const int d = (c & 15) * 8;
      const int tok = r >> 1;
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (tok < n_q)
        v[k] = __ldg(reinterpret_cast<const uint4*>(
            a.q + static_cast<long long>(flat_start + tok0 + tok) * a.q_row_stride +
            (kvh * kGroup + (r & 1)) * kHeadDim + d));
    }
    const uint32_t qbase_s = smem_u32(qtile);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = threadIdx.x + k * kConsumerWarps * 32;
      const int r = c >> 4;
      const int d = (c & 15) * 8;
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                       qbase_s + (r >> 4) * (16 * kHeadDim * 2) + swz_off(r & 15, d, 16)),
                   "r"(v[k].x), "r"(v[k].y), "r"(v[k].z), "r"(v[k].w)
                   : "memory");
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  }

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    const uint64_t policy = l2_policy_evict_first();
    if (lane == 0) tma_prefetch_desc(&kv_map);
    const int* table = a.tables + table_off + page_begin;
    // Pages from here on may hold this step's new tokens (positions >= num_cached).
    const int first_new = kEarly ? num_cached / kBlockTokens - page_begin : 0;
    bool waited = !kEarly;
    int issued = 0;
    bool stop = false;
    for (int j0 = 0; j0 < npages && !stop; j0 += 32) {
      int mine = 0;
      if (j0 + lane < npages) mine = table[j0 + lane];
      const int cnt = min(32, npages - j0);
      for (int jj = 0; jj < cnt; ++jj) {
        const int blk = __shfl_sync(0xffffffffu, mine, jj);
        if constexpr (kEarly) {
          if (!waited && j0 + jj >= first_new) {
            pdl_wait();
            waited = true;
          }
        }
        int ok = 1;
        if (lane == 0) {
          const int j = j0 + jj;
          const int s = j % kStages;
          if (*abort_flag) ok = 0;
          if (ok && j >= kStages && !mbar_wait(&empty[s], ((j / kStages) - 1) & 1)) {
            atomicOr(&g_status_word, kErrTimeout);
            *abort_flag = 1;
            ok = 0;
          }
          if (ok) {
            // Out-of-range block ids are flagged; the TMA unit fills such boxes with zeros.
            if (static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks))
              atomicOr(&g_status_word, kErrBlock);
            mbar_arrive_expect_tx(&full[s], kPageKVBytes);
            tma_load_5d(ring + s * kPageKVBytes, &kv_map, &full[s], 0, 0, 0, kvh, blk, policy);
            ++issued;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          stop = true;
          break;
        }
      }
    }
    // Drain: never leave the CTA with a TMA write in flight.
    if (lane == 0) {
      const int first = issued > kStages ? issued - kStages : 0;
      for (int j = first; j < issued; ++j) {
        if (!mbar_wait(&full[j % kStages], (j / kStages) & 1)) {
          atomicOr(&g_status_word, kErrTimeout);
          break;
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int row_base = kMode == 0 ? 0 : (warp % phase_warps) * 16;
  uint32_t qf[8][4];
  {
    const uint32_t qbase = smem_u32(qtile) + (row_base >> 4) * (16 * kHeadDim * 2);
    const int mi = lane >> 3;
    const int row = (lane & 7) + (mi & 1) * 8;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
      ldsm_x4(qbase + swz_off(row, ks * 16 + (mi >> 1) * 8, 16), qf[ks][0], qf[ks][1], qf[ks][2],
              qf[ks][3]);
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY};
  float l[2] = {0.f, 0.f};
  const int r0 = row_base + (lane >> 2);
  const int r1 = r0 + 8;
  const int qpos_base = num_cached + tok0;
  const int qpos0 = qpos_base + (r0 >> 1);
  const int qpos1 = qpos_base + (r1 >> 1);
  const int min_qpos = qpos_base + (row_base >> 1);         // first row of this warp's rows
  const int max_qpos = qpos_base + ((row_base + 15) >> 1);  // last row (warp-uniform)
  const uint32_t ring_u32 = smem_u32(ring);

  const int jstart = kMode == 0 ? warp : warp / phase_warps;
  const int jstep = kMode == 0 ? kConsumerWarps : phases;
  const bool warp_active = kMode == 0 || (row_base >> 1) < n_q;
  for (int j = jstart; j < npages; j += jstep) {
    const int s = j % kStages;
    // Leave the loop only as a whole warp: the tensor-core ops below are warp-collective.
    const bool ok = __all_sync(0xffffffffu, mbar_wait_fast(&full[s], (j / kStages) & 1, abort_flag));
    if (!ok) {
      if (lane == 0) {
        atomicOr(&g_status_word, kErrTimeout);
        *abort_flag = 1;
      }
      break;
    }
    const int key0 = (page_begin + j) * kBlockTokens;
    if (warp_active && key0 <= max_qpos) {
      attend_page(ring_u32 + s * kPageKVBytes, qf, o, m, l, key0, qpos0, qpos1,
                  key0 + kBlockTokens - 1 > min_qpos, a.scale_log2, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // Row sums were kept per thread; finish them across the quad.
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
    l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
  }

  if constexpr (kMode == 0) {
    // Cross-warp merge of the per-warp page subsets, through the (now idle) stage ring.
    decode_merge_store<kConsumerWarps>(reinterpret_cast<float*>(ring), o, m, l, warp, lane, n_q,
                                       kvh, part_row, merge_row, flat_start, tok0, a);
  } else {
    if (phases > 1) {
      // Merge the page phases of each row group into phase 0's warp, lane by lane (the warps of
      // one row group hold the same rows and columns in the same lanes), through the ring: every
      // page has been consumed once all consumer warps reach the barrier.
      float4* scratch = reinterpret_cast<float4*>(ring);
      const int slot = warp - phase_warps;  // warps of phases 1.. in order
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
      if (slot >= 0 && warp_active) {
#pragma unroll
        for (int n = 0; n < 16; ++n)
          scratch[(slot * 17 + n) * 32 + lane] = make_float4(o[n][0], o[n][1], o[n][2], o[n][3]);
        scratch[(slot * 17 + 16) * 32 + lane] = make_float4(m[0], m[1], l[0], l[1]);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
      if (slot >= 0 || !warp_active) return;
      for (int p = 1; p < phases; ++p) {
        const int sl = (p - 1) * phase_warps + warp;
        const float4 ml = scratch[(sl * 17 + 16) * 32 + lane];
        const float mp[2] = {ml.x, ml.y}, lp[2] = {ml.z, ml.w};
        float wa[2], wb[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float mx = fmaxf(m[h], mp[h]);
          wa[h] = m[h] == -INFINITY ? 0.f : fast_exp2(m[h] - mx);
          wb[h] = mp[h] == -INFINITY ? 0.f : fast_exp2(mp[h] - mx);
          l[h] = l[h] * wa[h] + lp[h] * wb[h];
          m[h] = mx;
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          const float4 v = scratch[(sl * 17 + n) * 32 + lane];
          o[n][0] = o[n][0] * wa[0] + v.x * wb[0];
          o[n][1] = o[n][1] * wa[0] + v.y * wb[0];
          o[n][2] = o[n][2] * wa[1] + v.z * wb[1];
          o[n][3] = o[n][3] * wa[1] + v.w * wb[1];
        }
      }
    } else if (!warp_active) {
      return;
    }
    const int c = 2 * (lane & 3);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half == 0 ? r0 : r1;
      const int tok = r >> 1;
      if (tok >= n_q) continue;
      const float L = l[half];
      const float invL = L > 0.f ? 1.f / L : 0.f;
      const int head = kvh * kGroup + (r & 1);
      if (part_row < 0) {
        __nv_bfloat16* dst = a.out + static_cast<long long>(flat_start + tok0 + tok) * a.out_row_stride +
                             head * kHeadDim + c;
#pragma unroll
        for (int n = 0; n < 16; ++n)
          *reinterpret_cast<uint32_t*>(dst + n * 8) =
              pack_bf16(o[n][2 * half] * invL, o[n][2 * half + 1] * invL);
      } else {
        const long long prow = static_cast<long long>(part_row + r) * a.num_kv + kvh;
        float* dst = a.ws_o + prow * kHeadDim + c;
#pragma unroll
        for (int n = 0; n < 16; ++n)
          *reinterpret_cast<float2*>(dst + n * 8) =
              make_float2(o[n][2 * half] * invL, o[n][2 * half + 1] * invL);
        if ((lane & 3) == 0) a.ws_lse[prow] = L > 0.f ? m[half] + __log2f(L) : -INFINITY;
      }
    }
  }
}

// Decode mode, persistent over work units (unit u = (item u / num_kv, KV head u % num_kv); CTA c
// takes units c, c + G, c + 2G, ..., G = gridDim.x, alternately for its two consumer groups) for
// plans of many short items, where a one-unit CTA spends most of its life starting up and
// finishing: here the producers stream the next units' pages while the consumers finish the
// current ones, and each unit's query rows are copied into shared memory during the group's
// previous unit (from item fields loaded a unit earlier still).  The launcher may give the grid
// fewer than two CTAs per SM (it leaves out the SMs held by the previous kernel's small last
// wave); nothing here depends on the grid size.  Per unit the consumer work is kernel B's decode mode
// (the same attend_page and decode_merge_store) with the unit's pages split over the group's
// warps instead of all consumer warps, so the results equal kernel B's up to the order in which
// the per-warp partial sums are merged; the merge scratch has its own shared memory because the
// ring keeps streaming.
template <int kConsumerWarps, int kStages>
struct UnitsCfg {
  using Base = AttnCfg<0, kConsumerWarps, kStages>;
  // The consumer warps form kGroups groups that take alternate units.  Each group has its own
  // producer warp, kGroupStages slots of the ring, query tile and merge scratch.
  static constexpr int kGroups = 2;
  static constexpr int kGroupWarps = kConsumerWarps / kGroups;
  static constexpr int kGroupStages = kStages / kGroups;
  static_assert(kConsumerWarps % kGroups == 0 && kStages % kGroups == 0, "even split");
  // A slot's previous fill must be a page of the same warp (the parity waits are exact only then):
  // the group's warps take its pages in turn, so its slot count is a multiple of its warps.
  static_assert(kGroupStages % kGroupWarps == 0, "slots per group a multiple of its warps");
  static constexpr int kThreads = (kConsumerWarps + kGroups) * 32;
  static constexpr int kStageBytes = Base::kStageBytes;
  static constexpr int kQBytes = Base::kQBytes;  // per group
  static constexpr int kMergeOff = kStageBytes + kGroups * kQBytes;
  // Per group: the merge scratch (the merge goes through it in two column passes) and a buffer
  // for the unit's shared-prefix partial, copied in while the unit's pages stream.
  static constexpr int kGroupScratchBytes = decode_merge_bytes<kGroupWarps, 2>();
  static constexpr int kGroupMergeBytes = kGroupScratchBytes + kPrefixPartialBytes;
  static_assert(kGroupScratchBytes % 16 == 0, "16-byte aligned partial buffer");
  static constexpr int kMergeBytes = kGroups * kGroupMergeBytes;
  static constexpr int kBarOffset = kMergeOff + kMergeBytes;
  static constexpr int kSmemBytes = 1024 + kBarOffset + 2 * kStages * 8 + 16;
};

// kAfterPrefix: this launch directly follows the tensor-core kernel of a plan with cascade groups
// (launched with programmatic dependent launch).  That kernel triggers its dependents only after
// its own wait has returned, so when this grid starts the kernel before it (which wrote the
// queries and this step's K/V rows) has completed: everything except the shared-prefix partials
// may be read at once, and the page loops run during the tensor-core kernel's last wave.  The
// prefix partials are read after pdl_wait() (a consumer group parks its first cascade unit's own
// result and merges it at its next merge, after the wait, instead of waiting at once), and every
// thread waits before it exits, so this grid never completes before the tensor-core kernel
// (later kernels rely on that ordering).
template <int kConsumerWarps, int kStages, bool kAfterPrefix = false>
__global__ void __launch_bounds__(UnitsCfg<kConsumerWarps, kStages>::kThreads, 2)
    paged_decode_units_kernel(const __grid_constant__ CUtensorMap kv_map, const AttnArgs a) {
  if constexpr (!kAfterPrefix) pdl_wait();
  pdl_trigger();
  using Cfg = UnitsCfg<kConsumerWarps, kStages>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* qtile = smem + Cfg::kStageBytes;
  float* merge = reinterpret_cast<float*>(smem + Cfg::kMergeOff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_units = a.n_items * a.num_kv;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // Group gi takes the CTA's units u = blockIdx.x + (kGroups i + gi) gridDim.x, i = 0, 1, ...
  constexpr int kGS = Cfg::kGroupStages;
  const int ustep = Cfg::kGroups * static_cast<int>(gridDim.x);
  if (warp >= kConsumerWarps) {
    // ---------------- producer warps: one per group, the group's pages in order through the
    // group's own kGS slots of the ring -----------------------------------------------------
    const int pg = warp - kConsumerWarps;
    const uint64_t policy = l2_policy_evict_first();
    if (lane == 0) tma_prefetch_desc(&kv_map);
    uint64_t* gfull = full + pg * kGS;
    uint64_t* gempty = empty + pg * kGS;
    uint8_t* gring = ring + pg * kGS * kPageKVBytes;
    int g = 0;  // pages issued so far (over all of this group's units)
    bool stop = false;
    for (int u = static_cast<int>(blockIdx.x) + pg * static_cast<int>(gridDim.x);
         u < n_units && !stop; u += ustep) {
      const int item_idx = u / a.num_kv;
      const int kvh = u - item_idx * a.num_kv;
      const int* it = a.items + static_cast<long long>(item_idx) * kRec;
      const int page_begin = it[3], npages = it[4] - it[3];
      const int* sr = a.seqs + static_cast<long long>(it[0]) * kRec;
      const int* table = a.tables + sr[4] + page_begin;
      for (int j0 = 0; j0 < npages && !stop; j0 += 32) {
        int mine = 0;
        if (j0 + lane < npages) mine = table[j0 + lane];
        const int cnt = min(32, npages - j0);
        for (int jj = 0; jj < cnt; ++jj) {
          const int blk = __shfl_sync(0xffffffffu, mine, jj);
          int ok = 1;
          if (lane == 0) {
            const int s = g % kGS;
            if (*abort_flag) ok = 0;
            if (ok && g >= kGS && !mbar_wait(&gempty[s], ((g / kGS) - 1) & 1)) {
              atomicOr(&g_status_word, kErrTimeout);
              *abort_flag = 1;
              ok = 0;
            }
            if (ok) {
              // Out-of-range block ids are flagged; the TMA unit fills such boxes with zeros.
              if (static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks))
                atomicOr(&g_status_word, kErrBlock);
              mbar_arrive_expect_tx(&gfull[s], kPageKVBytes);
              tma_load_5d(gring + s * kPageKVBytes, &kv_map, &gfull[s], 0, 0, 0, kvh, blk, policy);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            stop = true;
            break;
          }
          ++g;
        }
      }
    }
    // Drain: never leave the CTA with a TMA write in flight.
    if (lane == 0) {
      for (int j = g > kGS ? g - kGS : 0; j < g; ++j) {
        if (!mbar_wait(&gfull[j % kGS], (j / kGS) & 1)) {
          atomicOr(&g_status_word, kErrTimeout);
          break;
        }
      }
    }
    if constexpr (kAfterPrefix) pdl_wait();
    return;
  }

  // ---------------- consumer warps ----------------
  // Two groups of consumer warps take the CTA's units alternately, so one group's merge and
  // output run while the other group attends its unit's pages: a unit holds ~10 pages, and with
  // all warps on one unit no page was taken during a merge.  Within a group the warps split the
  // unit's pages; each group has its own producer, ring slots, query tile, merge scratch and
  // named barrier (1 + group).  The groups share no slot: a slot's full barrier is waited on by
  // parity, which is exact only while the slot's previous fill has completed, and within a group
  // that previous fill is always a page the same warp (or the group's previous unit) consumed.
  constexpr int kGW = Cfg::kGroupWarps;
  const int grp = warp / kGW;
  const int gw = warp - grp * kGW;                 // warp within the group
  const int gtid = threadIdx.x - grp * kGW * 32;   // thread within the group
  const int bar_id = 1 + grp;
  // A unit's 16 query rows (token r / 2, head kvh * 2 + r % 2), 16 chunks of 16 bytes each,
  // kPer chunks per thread of the group, copied into the group's query tile one unit ahead
  // (cp.async: no registers held across the page loop).
  constexpr int kPer = 16 * 16 / (kGW * 32);
  static_assert(16 * 16 % (kGW * 32) == 0, "query chunks per thread");
  const uint32_t qbase_s = smem_u32(qtile + grp * Cfg::kQBytes);
  // Unit u's query rows from its item fields (token offset, token count, the sequence's first
  // flat row), which the caller loaded a unit ahead, so no dependent global load stalls here.
  auto prefetch_q = [&](int u, int tok0, int n_q, int flat_start) {
    const int kvh = u % a.num_kv;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = gtid + k * kGW * 32;
      const int r = c >> 4;
      const int d = (c & 15) * 8;
      const int tok = r >> 1;
      const uint32_t dst = qbase_s + swz_off(r, d, 16);
      if (tok < n_q) {
        const __nv_bfloat16* src = a.q + static_cast<long long>(flat_start + tok0 + tok) * a.q_row_stride +
                                   (kvh * kGroup + (r & 1)) * kHeadDim + d;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
      } else {
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // The item fields of a unit: token offset, token count and sequence (for its first flat row).
  auto unit_fields = [&](int u, int& tok0, int& n_q, int& seq) {
    const int* it = a.items + static_cast<long long>(u / a.num_kv) * kRec;
    seq = it[0];
    tok0 = it[1];
    n_q = it[2];
  };
  const int u_first = static_cast<int>(blockIdx.x) + grp * static_cast<int>(gridDim.x);
  // Fields of the group's next unit (u + ustep): its query tile is copied at the start of unit
  // u.  Its token offset and count are loaded at the start of the unit before, and its sequence's
  // first flat row after that unit's page loop (it depends on the sequence id).
  int nx_tok0 = 0, nx_nq = 0, nx_seq = 0, nx_flat = 0;
  if (u_first < n_units) {
    int t0, nq, sq;
    unit_fields(u_first, t0, nq, sq);
    prefetch_q(u_first, t0, nq, a.seqs[static_cast<long long>(sq) * kRec]);
    if (u_first + ustep < n_units) {
      unit_fields(u_first + ustep, nx_tok0, nx_nq, nx_seq);
      nx_flat = a.seqs[static_cast<long long>(nx_seq) * kRec];
    }
  }
  const uint32_t ring_u32 = smem_u32(ring + grp * kGS * kPageKVBytes);
  uint64_t* gfull = full + grp * kGS;
  uint64_t* gempty = empty + grp * kGS;
  float* merge_g = merge + grp * (Cfg::kGroupMergeBytes / 4);
  float* partial_g = merge_g + Cfg::kGroupScratchBytes / 4;
  // Whether the kernel that writes the shared-prefix partials is known to have completed (this
  // thread has executed griddepcontrol.wait): from the start unless this launch overlaps it.
  bool partials_ready = !kAfterPrefix;
  // A group's first cascade unit does not wait for that kernel: its own result is parked in the
  // partial buffer and merged with the prefix partial at the group's next merge, by which time
  // that kernel has normally completed, so the group keeps streaming pages meanwhile.
  bool parked = false;
  int pk_n_q = 0, pk_kvh = 0, pk_merge_row = 0, pk_flat = 0, pk_tok0 = 0;
  int g0 = 0;  // this unit's first page in the group's ring sequence
  for (int u = u_first; u < n_units; u += ustep) {
    const int item_idx = u / a.num_kv;
    const int kvh = u - item_idx * a.num_kv;
    const int* it = a.items + static_cast<long long>(item_idx) * kRec;
    const int seq = it[0], tok0 = it[1], n_q = it[2], page_begin = it[3], page_end = it[4],
              part_row = it[5];
    const int merge_row = it[7] == 1 ? it[6] : -1;
    const int* sr = a.seqs + static_cast<long long>(seq) * kRec;
    const int flat_start = sr[0], num_cached = sr[2];
    const int npages = page_end - page_begin;

    // This unit's query tile has landed (every thread's copies), and the group's previous unit
    // has finished with the merge scratch.
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    named_bar_1_or_2(bar_id, kGW * 32);
    uint32_t qf[8][4];
    {
      const int mi = lane >> 3;
      const int row = (lane & 7) + (mi & 1) * 8;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        ldsm_x4(qbase_s + swz_off(row, ks * 16 + (mi >> 1) * 8, 16), qf[ks][0], qf[ks][1],
                qf[ks][2], qf[ks][3]);
    }
    // Every warp of the group holds its query fragments: the tile takes the next unit's rows.
    named_bar_1_or_2(bar_id, kGW * 32);
    // A cascade row's shared-prefix partial (rows r < 2 n_q: 128 fp32 of O and the log2-sum-exp)
    // is copied into the group's buffer while the unit's pages stream, so the merge reads it
    // from shared memory.
    const bool cascade_row = part_row < 0 && merge_row >= 0;
    const bool pre = partials_ready && cascade_row;
    if (pre) {
      const uint32_t pbase = smem_u32(partial_g);
      for (int c = gtid; c < 2 * n_q * 32; c += kGW * 32) {
        const int r = c >> 5, ch = c & 31;
        const float* src =
            a.ws_o + (static_cast<long long>(merge_row + r) * a.num_kv + kvh) * kHeadDim + ch * 4;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pbase + r * 512 + ch * 16),
                     "l"(src)
                     : "memory");
      }
      if (gtid < 2 * n_q) {
        const float* src = a.ws_lse + static_cast<long long>(merge_row + gtid) * a.num_kv + kvh;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(pbase + 16 * kHeadDim * 4 + gtid * 4),
                     "l"(src)
                     : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (u + ustep < n_units) prefetch_q(u + ustep, nx_tok0, nx_nq, nx_flat);
    // The unit after next: its fields are loaded now and land during this unit's page loop.
    const bool has_next2 = u + 2 * ustep < n_units;
    if (has_next2) unit_fields(u + 2 * ustep, nx_tok0, nx_nq, nx_seq);

    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY};
    float l[2] = {0.f, 0.f};
    const int r0 = lane >> 2;
    const int r1 = r0 + 8;
    const int qpos_base = num_cached + tok0;
    const int qpos0 = qpos_base + (r0 >> 1);
    const int qpos1 = qpos_base + (r1 >> 1);
    const int min_qpos = qpos_base;
    const int max_qpos = qpos_base + 7;
    for (int j = gw; j < npages; j += kGW) {
      const int gj = g0 + j;
      const int s = gj % kGS;
      // Leave the loop only as a whole warp: the tensor-core ops below are warp-collective.
      const bool ok =
          __all_sync(0xffffffffu, mbar_wait_fast(&gfull[s], (gj / kGS) & 1, abort_flag));
      if (!ok) {
        if (lane == 0) {
          atomicOr(&g_status_word, kErrTimeout);
          *abort_flag = 1;
        }
        break;
      }
      const int key0 = (page_begin + j) * kBlockTokens;
      if (key0 <= max_qpos) {
        attend_page(ring_u32 + s * kPageKVBytes, qf, o, m, l, key0, qpos0, qpos1,
                    key0 + kBlockTokens - 1 > min_qpos, a.scale_log2, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&gempty[s]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
      l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
    }
    // Its sequence's first flat row lands during the merge.
    if (has_next2) nx_flat = a.seqs[static_cast<long long>(nx_seq) * kRec];
    if (pre) {  // this thread's copies of the partial (not the next query tile's) have landed
      if (u + ustep < n_units)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      else
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    const bool park_now =
        kAfterPrefix && cascade_row && !partials_ready && !parked && u + ustep < n_units;
    if (parked) {
      pdl_wait();  // returns once the kernel that writes the prefix partials has completed
      finish_parked<kGW * 32>(partial_g, pk_n_q, pk_kvh, pk_merge_row, pk_flat, pk_tok0, a, gtid);
      parked = false;
      partials_ready = true;
    }
    decode_merge_store<kGW, kAfterPrefix, 2>(merge_g, o, m, l, gw, lane, n_q, kvh, part_row,
                                             merge_row, flat_start, tok0, a, bar_id, gtid,
                                             pre ? partial_g : nullptr,
                                             park_now ? partial_g : nullptr);
    if (park_now) {
      parked = true;
      pk_n_q = n_q;
      pk_kvh = kvh;
      pk_merge_row = merge_row;
      pk_flat = flat_start;
      pk_tok0 = tok0;
    } else if (cascade_row && !partials_ready) {
      // The merge waited for that kernel only in the threads that read a partial row; every
      // thread copies the next units' partials, so every thread waits (at once, by now).
      if constexpr (kAfterPrefix) pdl_wait();
      partials_ready = true;
    }
    g0 += npages;
  }
  if constexpr (kAfterPrefix) {
    pdl_wait();
    // A unit parked by a group whose loop then ended early (a timeout) is still written out.
    if (parked)
      finish_parked<kGW * 32>(partial_g, pk_n_q, pk_kvh, pk_merge_row, pk_flat, pk_tok0, a, gtid);
  }
}

struct CombineArgs {
  __nv_bfloat16* out;
  long long out_row_stride;
  const int* seqs;
  const int* combines;
  int n_combine;
  int num_kv;
  const float* ws_o;
  const float* ws_lse;
};

// Kernel C: out = sum_s 2^(lse_s - M) * O_s / sum_s 2^(lse_s - M) for every split tile.
// One CTA per (split tile, KV head, run of kCombineRows rows); thread = (row, 16-dim slice).
constexpr int kCombineThreads = 256;
constexpr int kCombineRows = kCombineThreads / 8;  // rows one CTA merges at a time (8 threads each)
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const CombineArgs a) {
  pdl_wait();
  pdl_trigger();
  const int ci = blockIdx.x / a.num_kv;
  const int kvh = blockIdx.x - ci * a.num_kv;
  const int* cr = a.combines + static_cast<long long>(ci) * kRec;
  const int seq = cr[0], tok0 = cr[1], n_q = cr[2], part_row0 = cr[3], n_splits = cr[4];
  const int flat_start = a.seqs[static_cast<long long>(seq) * kRec];
  const int rows = n_q * kGroup;
  // Split s's rows start at part_row0 + s * stride: consecutive (stride = rows) for a split tile;
  // a cascade row's shared-prefix and own-page partials sit apart (stride in field 5).
  const int stride = cr[5] != 0 ? cr[5] : rows;
  const int dc = (threadIdx.x & 7) * 16;
  // Grid y splits the record's rows into runs of kCombineRows; CTAs past its rows do nothing.
  for (int r = blockIdx.y * kCombineRows + (threadIdx.x >> 3); r < rows;
       r += gridDim.y * kCombineRows) {
    float mx = -INFINITY;
    for (int s = 0; s < n_splits; ++s)
      mx = fmaxf(mx, a.ws_lse[(static_cast<long long>(part_row0) + static_cast<long long>(s) * stride + r) *
                                   a.num_kv + kvh]);
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    float L = 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const long long prow =
          (static_cast<long long>(part_row0) + static_cast<long long>(s) * stride + r) * a.num_kv + kvh;
      const float lse = a.ws_lse[prow];
      const float w = lse == -INFINITY ? 0.f : fast_exp2(lse - mx);
      L += w;
      const float4* src = reinterpret_cast<const float4*>(a.ws_o + prow * kHeadDim + dc);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = src[i];
        acc[4 * i] += w * v.x;
        acc[4 * i + 1] += w * v.y;
        acc[4 * i + 2] += w * v.z;
        acc[4 * i + 3] += w * v.w;
      }
    }
    const float invL = L > 0.f ? 1.f / L : 0.f;
    const int head = kvh * kGroup + (r & 1);
    __nv_bfloat16* dst = a.out + static_cast<long long>(flat_start + tok0 + (r >> 1)) * a.out_row_stride +
                         head * kHeadDim + dc;
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) pk[i] = pack_bf16(acc[2 * i] * invL, acc[2 * i + 1] * invL);
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
}

}  // namespace ms
