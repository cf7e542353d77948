// Kernel A: fused per-head q/k RMSNorm + rotate-half RoPE + scatter of the new K/V rows into the
// paged KV pool.  Replaces, for one layer, the op sequence of MiniServe's attention module
// (src/miniserve/model/qwen3.py:94-98 -> layers.py:18-22 and :56-65) and the scatter at the top of
// paged_attention (src/miniserve/attention/backends.py:159-160).
//
// Rows 0..H-1 of a token are query heads, H..H+KVH-1 key heads, H+KVH..H+2*KVH-1 value heads,
// i.e. the 128-column blocks of the fused qkv projection in order.  Each lane owns 4 consecutive
// dims of a row (one 8-byte load, one 8-byte store).
//
// Rounding follows the reference exactly where the order is fixed by it: fp32 squares, fp32 mean,
// rsqrt, fp32 multiply, round to bf16, bf16 weight multiply (rounded), bf16 cos/sin, bf16 products
// and a bf16 sum.  __fmul_rn/__fadd_rn keep nvcc from contracting these into FMAs.  Only the
// summation order of the 128 squares differs from PyTorch's reduction kernel, which can move the
// fp32 mean by an ulp and, rarely, one output by one bf16 ulp.
#pragma once

#include "ms_common.cuh"

namespace ms {

struct NormRopeArgs {
  const __nv_bfloat16* qkv;  // [T, (H + 2*KVH) * 128]
  long long qkv_row_stride;  // elements
  const __nv_bfloat16* q_weight;  // [128]
  const __nv_bfloat16* k_weight;  // [128]
  float eps;
  const float* cos;  // [T, 128] rows already gathered by position, or the [max_pos, 128] table
  const float* sin;
  long long cs_row_stride;
  const long long* positions;  // null: cos/sin are per-token rows; else index into the table
  long long max_positions;
  const long long* slots;  // [T] slot = block * 16 + offset
  __nv_bfloat16* q_out;  // [T, H, 128]
  long long q_out_row_stride;
  __nv_bfloat16* k_pool;  // this layer's K base; V base = K base + 2048 elements
  long long block_stride;  // elements between blocks
  long long head_stride;   // elements between KV heads of one block
  long long num_slots;
  int num_tokens;
  int num_heads;
  int num_kv;
};

// Element offset of (slot, kv head, dim) inside a layer's K region of the pool.
// Within a (block, head) the K page is [d/64][token][d%64]; V follows 4 KiB later.
__device__ __forceinline__ long long pool_offset(long long slot, int head, int d,
                                                 long long block_stride, long long head_stride) {
  const long long block = slot >> 4;
  const int tok = static_cast<int>(slot & 15);
  return block * block_stride + head * head_stride + (d >> 6) * (kBlockTokens * 64) + tok * 64 +
         (d & 63);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// One warp handles 8 head rows of one token: warps 0-1 of a token take the 16 query heads, warp 2
// the 8 key heads, warp 3 the 8 value heads (rows are the 128-column blocks of the fused
// projection, in order), so every warp does one kind of work.  All 8 row loads are issued before
// any arithmetic, and the token's cos/sin values are read once per warp.
constexpr int kRowsPerWarp = 8;

template <int kWarps>
__global__ void __launch_bounds__(kWarps * 32)
    qk_norm_rope_scatter_kernel(const NormRopeArgs a, unsigned* status) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps_per_tok = (a.num_heads + 2 * a.num_kv) / kRowsPerWarp;
  const long long gw = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const long long t = gw / warps_per_tok;
  if (t >= a.num_tokens) return;
  const int row0 = static_cast<int>(gw - t * warps_per_tok) * kRowsPerWarp;
  const int d0 = lane * 4;

  uint2 raw[kRowsPerWarp];
  const __nv_bfloat16* src = a.qkv + t * a.qkv_row_stride + row0 * kHeadDim + d0;
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
    raw[r] = *reinterpret_cast<const uint2*>(src + r * kHeadDim);

  const bool is_v = row0 >= a.num_heads + a.num_kv;
  const bool is_q = row0 < a.num_heads;
  long long slot = 0;
  bool slot_ok = true;
  if (!is_q) {
    slot = a.slots[t];
    slot_ok = slot >= 0 && slot < a.num_slots;
    if (!slot_ok) {
      if (lane == 0) atomicOr(status, kErrSlot);
      return;
    }
  }
  if (is_v) {  // value heads: a pure copy into the pool
    const int h0 = row0 - a.num_heads - a.num_kv;
    __nv_bfloat16* vbase = a.k_pool + 2 * kBlockTokens * 64;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
      *reinterpret_cast<uint2*>(vbase + pool_offset(slot, h0 + r, d0, a.block_stride, a.head_stride)) = raw[r];
    return;
  }

  long long pos_row = t;
  if (a.positions != nullptr) {
    pos_row = a.positions[t];
    if (pos_row < 0 || pos_row >= a.max_positions) {
      if (lane == 0) atomicOr(status, kErrPosition);
      pos_row = 0;
    }
  }
  const float4 c4 = *reinterpret_cast<const float4*>(a.cos + pos_row * a.cs_row_stride + d0);
  const float4 s4 = *reinterpret_cast<const float4*>(a.sin + pos_row * a.cs_row_stride + d0);
  const float cv[4] = {bf16_round(c4.x), bf16_round(c4.y), bf16_round(c4.z), bf16_round(c4.w)};
  const float sv[4] = {bf16_round(s4.x), bf16_round(s4.y), bf16_round(s4.z), bf16_round(s4.w)};
  const __nv_bfloat16* wp = (is_q ? a.q_weight : a.k_weight) + d0;
  float wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = __bfloat162float(wp[i]);

  // fp32 mean of squares per head (8 independent warp reductions, interleaved).
  float x[kRowsPerWarp][4], ss[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&raw[r]);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[r][i] = __bfloat162float(xb[i]);
    ss[r] = __fadd_rn(__fadd_rn(__fmul_rn(x[r][0], x[r][0]), __fmul_rn(x[r][1], x[r][1])),
                      __fadd_rn(__fmul_rn(x[r][2], x[r][2]), __fmul_rn(x[r][3], x[r][3])));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
      ss[r] = __fadd_rn(ss[r], __shfl_xor_sync(0xffffffffu, ss[r], off));
  }

#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss[r], 1.0f / kHeadDim), a.eps));
    float z[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float y = bf16_round(__fmul_rn(x[r][i], inv));  // (x32 * rsqrt).to(bf16)
      z[i] = bf16_round(__fmul_rn(wv[i], y));              // weight * y, in bf16
    }
    __nv_bfloat16 outv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, z[i], 16);
      const float rot = lane < 16 ? -partner : partner;  // rotate_half: [-x2, x1]
      const float p1 = bf16_round(__fmul_rn(z[i], cv[i]));
      const float p2 = bf16_round(__fmul_rn(rot, sv[i]));
      outv[i] = __float2bfloat16_rn(__fadd_rn(p1, p2));
    }
    const uint2 packed = *reinterpret_cast<const uint2*>(outv);
    if (is_q) {
      *reinterpret_cast<uint2*>(a.q_out + t * a.q_out_row_stride + (row0 + r) * kHeadDim + d0) = packed;
    } else {
      *reinterpret_cast<uint2*>(a.k_pool + pool_offset(slot, row0 + r - a.num_heads, d0,
                                                       a.block_stride, a.head_stride)) = packed;
    }
  }
}

// Correctly rounded (round-to-nearest-even) bf16 pair arithmetic.  For bf16 operands the exact
// product or sum of two values fits in fp32 whenever its result is a normal number, so
// bf16(fp32(a) op fp32(b)) -- the reference's order: bf16 tensors multiplied / added in bf16 --
// equals the single rounding these instructions perform.
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Kernel A, 16-byte form (qkv and q_out rows 16-byte aligned; the 8-byte form above serves the
// rest).  One warp handles 8 head rows of one token as 4 pairs: lanes 0-15 take row 2k, lanes
// 16-31 row 2k + 1 (k = 0..3), 8 consecutive dims per lane, so every load and store instruction
// moves two whole 256-byte rows.  The results equal the 8-byte form's bit for bit:
// * the sum of squares keeps its reduction tree: lane l of a half holds the dims of the 8-byte
//   form's lanes 2l and 2l + 1, whose partial sums are reduced separately with xor 8, 4, 2, 1
//   (that form's xor 16, 8, 4, 2) and added last (its xor 1); squares of bf16 values are exact
//   in fp32, so a fused multiply-add forms the same partial sums;
// * weight * y, z * cos, rot * sin and p1 + p2 have bf16 operands: bf16x2_mul / bf16x2_add give
//   the same roundings, two elements per instruction;
// * rotate_half's partner (dim d +- 64) is lane ^ 8.
template <int kWarps>
__global__ void __launch_bounds__(kWarps * 32)
    qk_norm_rope_scatter_v16_kernel(const NormRopeArgs a, unsigned* status) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int wpt = (a.num_heads + 2 * a.num_kv) / kRowsPerWarp;  // warps per token
  long long t;
  int wi;
  if (kWarps % wpt == 0) {
    const int tpc = kWarps / wpt;  // tokens per CTA
    t = static_cast<long long>(blockIdx.x) * tpc + warp / wpt;
    wi = warp % wpt;
  } else {
    const long long gw = static_cast<long long>(blockIdx.x) * kWarps + warp;
    t = gw / wpt;
    wi = static_cast<int>(gw - t * wpt);
  }
  if (t >= a.num_tokens) return;
  const int row0 = wi * kRowsPerWarp;
  const int half = lane >> 4;
  const int l16 = lane & 15;
  const int d0 = l16 * 8;

  uint4 raw[4];
  const __nv_bfloat16* src = a.qkv + t * a.qkv_row_stride + (row0 + half) * kHeadDim + d0;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    raw[k] = *reinterpret_cast<const uint4*>(src + 2 * k * kHeadDim);

  const bool is_v = row0 >= a.num_heads + a.num_kv;
  const bool is_q = row0 < a.num_heads;
  long long slot = 0;
  if (!is_q) {
    slot = a.slots[t];
    if (slot < 0 || slot >= a.num_slots) {
      if (lane == 0) atomicOr(status, kErrSlot);
      return;
    }
  }
  if (is_v) {  // value heads: a pure copy into the pool
    const int h0 = row0 - a.num_heads - a.num_kv + half;
    __nv_bfloat16* vbase = a.k_pool + 2 * kBlockTokens * 64;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<uint4*>(vbase + pool_offset(slot, h0 + 2 * k, d0, a.block_stride,
                                                    a.head_stride)) = raw[k];
    return;
  }

  long long pos_row = t;
  if (a.positions != nullptr) {
    pos_row = a.positions[t];
    if (pos_row < 0 || pos_row >= a.max_positions) {
      if (lane == 0) atomicOr(status, kErrPosition);
      pos_row = 0;
    }
  }
  // cos / sin rounded to bf16 (the reference casts the fp32 tables to the activations' dtype),
  // and the norm weight, as bf16 pairs for dims (d0 + 2i, d0 + 2i + 1).
  uint32_t c2[4], s2[4], w2[4];
  {
    const float* cp = a.cos + pos_row * a.cs_row_stride + d0;
    const float* sp = a.sin + pos_row * a.cs_row_stride + d0;
    const float4 ca = *reinterpret_cast<const float4*>(cp);
    const float4 cb = *reinterpret_cast<const float4*>(cp + 4);
    const float4 sa = *reinterpret_cast<const float4*>(sp);
    const float4 sb = *reinterpret_cast<const float4*>(sp + 4);
    c2[0] = pack_bf16(ca.x, ca.y);
    c2[1] = pack_bf16(ca.z, ca.w);
    c2[2] = pack_bf16(cb.x, cb.y);
    c2[3] = pack_bf16(cb.z, cb.w);
    s2[0] = pack_bf16(sa.x, sa.y);
    s2[1] = pack_bf16(sa.z, sa.w);
    s2[2] = pack_bf16(sb.x, sb.y);
    s2[3] = pack_bf16(sb.z, sb.w);
    const uint4 wv = *reinterpret_cast<const uint4*>((is_q ? a.q_weight : a.k_weight) + d0);
    w2[0] = wv.x;
    w2[1] = wv.y;
    w2[2] = wv.z;
    w2[3] = wv.w;
  }
  const uint32_t neg = l16 < 8 ? 0x80008000u : 0u;  // rotate_half: [-x2, x1]

  // Partial sums of squares: (lanes 2l, 2l + 1 of the 8-byte form) = (dims d0..d0+3, d0+4..d0+7).
  float2 ss[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
    const float2 x0 = make_float2(bf16_lo(w[0]), bf16_lo(w[2]));
    const float2 x1 = make_float2(bf16_hi(w[0]), bf16_hi(w[2]));
    const float2 x2 = make_float2(bf16_lo(w[1]), bf16_lo(w[3]));
    const float2 x3 = make_float2(bf16_hi(w[1]), bf16_hi(w[3]));
    const float2 s01 = __ffma2_rn(x1, x1, __fmul2_rn(x0, x0));
    const float2 s23 = __ffma2_rn(x3, x3, __fmul2_rn(x2, x2));
    ss[k] = __fadd2_rn(s01, s23);
  }
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, ss[k].x, off),
                                   __shfl_xor_sync(0xffffffffu, ss[k].y, off));
      ss[k] = __fadd2_rn(ss[k], o);
    }
  }

#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float inv =
        rsqrtf(__fadd_rn(__fmul_rn(__fadd_rn(ss[k].x, ss[k].y), 1.0f / kHeadDim), a.eps));
    const float2 inv2 = make_float2(inv, inv);
    const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
    uint32_t outw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = __fmul2_rn(make_float2(bf16_lo(w[i]), bf16_hi(w[i])), inv2);
      const uint32_t z = bf16x2_mul(w2[i], pack_bf16(y.x, y.y));  // weight * y, in bf16
      const uint32_t rot = __shfl_xor_sync(0xffffffffu, z, 8) ^ neg;
      outw[i] = bf16x2_add(bf16x2_mul(z, c2[i]), bf16x2_mul(rot, s2[i]));
    }
    const uint4 packed = make_uint4(outw[0], outw[1], outw[2], outw[3]);
    const int row = row0 + 2 * k + half;
    if (is_q) {
      *reinterpret_cast<uint4*>(a.q_out + t * a.q_out_row_stride + row * kHeadDim + d0) = packed;
    } else {
      *reinterpret_cast<uint4*>(a.k_pool + pool_offset(slot, row - a.num_heads, d0,
                                                       a.block_stride, a.head_stride)) = packed;
    }
  }
}

struct ScatterArgs {
  const __nv_bfloat16* k;  // [T, KVH, 128] (row stride k_row_stride, head stride 128)
  long long k_row_stride;
  const __nv_bfloat16* v;
  long long v_row_stride;
  const long long* slots;
  __nv_bfloat16* k_pool;
  long long block_stride;
  long long head_stride;
  long long num_slots;
  int num_tokens;
  int num_kv;
};

// Scatter-only form (backends.py:159-160 alone): k and v are already normalised/rotated.
template <int kWarps>
__global__ void __launch_bounds__(kWarps * 32) kv_scatter_kernel(const ScatterArgs a,
                                                                 unsigned* status) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long long gw = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const long long t = gw / (2 * a.num_kv);
  if (t >= a.num_tokens) return;
  const int r = static_cast<int>(gw - t * 2 * a.num_kv);
  const bool is_v = r >= a.num_kv;
  const int h = is_v ? r - a.num_kv : r;
  const int d0 = lane * 4;
  const long long slot = a.slots[t];
  if (slot < 0 || slot >= a.num_slots) {
    if (lane == 0) atomicOr(status, kErrSlot);
    return;
  }
  const __nv_bfloat16* src =
      is_v ? a.v + t * a.v_row_stride + h * kHeadDim + d0 : a.k + t * a.k_row_stride + h * kHeadDim + d0;
  __nv_bfloat16* dst = a.k_pool + (is_v ? 2 * kBlockTokens * 64 : 0) +
                       pool_offset(slot, h, d0, a.block_stride, a.head_stride);
  *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
}

}  // namespace ms
