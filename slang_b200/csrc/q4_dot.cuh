// Exact dot products of packed int4 codes with 16-bit-quantised activations,
// shared by the GEMV kernels.  A group is 32 consecutive values (16 bytes of
// nibbles, low nibble first).  The activation group is rounded to integers
// x_int = rint(x * 32767 / max|x|) (error <= 2^-16 of the group's max), split
// into a signed high byte and an unsigned low byte, and arranged to line up with
// the even (low) and odd (high) nibbles of each 32-bit word, so that
//   sum (q - 8) * x_int = 256 * dot(q, hi) + dot(q, lo) - 8 * sum(x_int)
// is computed exactly with DP4A in 32-bit integers.
#pragma once

#include "common.cuh"

namespace sbd {

// x of one group as DP4A operands: 4 words x {hi even, hi odd, lo even, lo odd}
// bytes, -8 * sum(x_int), and the group's scale max|x| / 32767.
struct XGroup {
  uint32_t he[4], ho[4], le[4], lo[4];
  int bias;
  float sx;
};

// Pack 32 integer activations (|x_int| < 2^15) and their scale into g.
__device__ __forceinline__ void pack_group(const int (&xi)[32], float sx, XGroup& g) {
  g.sx = sx;
  int sum = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t he = 0, ho = 0, le = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int xe = xi[8 * j + 2 * i];
      const int xo = xi[8 * j + 2 * i + 1];
      sum += xe + xo;
      he |= (static_cast<uint32_t>(xe >> 8) & 0xFFu) << (8 * i);
      ho |= (static_cast<uint32_t>(xo >> 8) & 0xFFu) << (8 * i);
      le |= (static_cast<uint32_t>(xe) & 0xFFu) << (8 * i);
      lo |= (static_cast<uint32_t>(xo) & 0xFFu) << (8 * i);
    }
    g.he[j] = he;
    g.ho[j] = ho;
    g.le[j] = le;
    g.lo[j] = lo;
  }
  g.bias = -8 * sum;
}

// rint(x * inv) for |x * inv| < 2^22 in the low 16 bits of the returned word
// (the rest is 0x4B40 less any borrow): adding 1.5 * 2^23 to the product
// rounds it to the nearest integer, ties to even, as cvt.rni does, and leaves
// that integer in two's complement in the mantissa's low bits.  A NaN product
// gives 0, as cvt does.  Two full-rate FP32 operations (never contracted into
// one FMA) instead of a conversion on the quarter-rate pipe.
constexpr uint32_t kRintBias = 0x4B400000u;  // bits of 1.5 * 2^23
__device__ __forceinline__ uint32_t rint_bits(float x, float inv) {
  const float f = __fmul_rn(x, inv);
  const uint32_t b = __float_as_uint(__fadd_rn(f, 12582912.f));
  return f == f ? b : kRintBias;
}

// Pack the rint_bits of values 8 j .. 8 j + 7 of a group (b[0..7]) into word j
// of he / ho / le / lo: byte i of he (le) is the high (low) byte of value
// 8 j + 2 i, of ho (lo) of value 8 j + 2 i + 1.
__device__ __forceinline__ void pack_word(const uint32_t* b, uint32_t& he, uint32_t& ho, uint32_t& le,
                                          uint32_t& lo) {
  // [lo(a), lo(b), hi(a), hi(b)] of value pairs, then their low and high halves
  const uint32_t e01 = __byte_perm(b[0], b[2], 0x5140), e23 = __byte_perm(b[4], b[6], 0x5140);
  const uint32_t o01 = __byte_perm(b[1], b[3], 0x5140), o23 = __byte_perm(b[5], b[7], 0x5140);
  le = __byte_perm(e01, e23, 0x5410);
  he = __byte_perm(e01, e23, 0x7632);
  lo = __byte_perm(o01, o23, 0x5410);
  ho = __byte_perm(o01, o23, 0x7632);
}

// x_int = rint(x * 32767 / max|x|), scale max|x| / 32767.
__device__ __forceinline__ void quantise_group(const float (&v)[32], XGroup& g) {
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
  const float inv = mx > 0.f ? 32767.f / mx : 0.f;
  uint32_t b[32], sum = 0u;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    b[i] = rint_bits(v[i], inv);
    sum += b[i];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) pack_word(b + 8 * j, g.he[j], g.ho[j], g.le[j], g.lo[j]);
  g.bias = -8 * static_cast<int>(sum - 32u * kRintBias);  // the 32 biases cancel mod 2^32
  g.sx = mx / 32767.f;
}

// The same group quantised by the two lanes of a warp that hold it (lane and
// lane ^ 16): this lane has values 16 h .. 16 h + 15 (h = lane >> 4); the pair
// combines its max, each packs words 2 h and 2 h + 1 of he / ho / le / lo, and
// they swap them, so both lanes end with the group exactly as quantise_group
// makes it, for half the work each.
__device__ __forceinline__ void quantise_group_pair(const float (&v)[16], int h, XGroup& g) {
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
  const float inv = mx > 0.f ? 32767.f / mx : 0.f;
  uint32_t b[16], sum = 0u;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    b[i] = rint_bits(v[i], inv);
    sum += b[i];
  }
  uint32_t w[2][4];  // [word][he, ho, le, lo]
#pragma unroll
  for (int j = 0; j < 2; ++j) pack_word(b + 8 * j, w[j][0], w[j][1], w[j][2], w[j][3]);
  sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) o[t] = __shfl_xor_sync(0xFFFFFFFFu, w[j][t], 16);
    // h = 0 packed words 0, 1 and receives 2, 3; h = 1 the reverse
    g.he[j] = h ? o[0] : w[j][0];
    g.ho[j] = h ? o[1] : w[j][1];
    g.le[j] = h ? o[2] : w[j][2];
    g.lo[j] = h ? o[3] : w[j][3];
    g.he[2 + j] = h ? w[j][0] : o[0];
    g.ho[2 + j] = h ? w[j][1] : o[1];
    g.le[2 + j] = h ? w[j][2] : o[2];
    g.lo[2 + j] = h ? w[j][3] : o[3];
  }
  g.bias = -8 * static_cast<int>(sum - 32u * kRintBias);
  g.sx = mx / 32767.f;
}

// Static range quantisation of an activation (the reference's
// srq(x, s) = clip(round(x / s), -128, 127) * s, gemma4_150/reference.py:30-31):
// the integer code of x.  Division and round-half-to-even as numpy's f32 ops.
__device__ __forceinline__ int srq_code(float x, float s) {
  return max(-128, min(127, __float2int_rn(__fdiv_rn(x, s))));
}

// Exact integer dot of 32 int4 codes (minus 8) with the group's x_int, in four
// independent accumulation chains for instruction-level parallelism.
__device__ __forceinline__ int dot_group(const uint4 q, const XGroup& g) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  int he = 0, ho = 0, le = g.bias, lo = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t e = w[j] & 0x0F0F0F0Fu;
    const uint32_t o = (w[j] >> 4) & 0x0F0F0F0Fu;
    he = dp4a_us(e, g.he[j], he);
    ho = dp4a_us(o, g.ho[j], ho);
    le = dp4a_uu(e, g.le[j], le);
    lo = dp4a_uu(o, g.lo[j], lo);
  }
  return (he + ho) * 256 + le + lo;
}

// ---- 2-bit codes (the checkpoint's 2-bit MLP and lm_head weights): 4 codes
// per byte, low bits first, zero point 2.  A 32-value group is 8 bytes of
// codes, two 32-bit words; field k of word j, (w >> 2k) & 0x03030303, holds the
// codes of values 16 j + 4 b + k (b = byte).  x is arranged to match:
//   sum (q - 2) * x_int = 256 * dot(q, hi) + dot(q, lo) - 2 * sum(x_int).
struct XGroup2 {
  uint32_t hi[8], lo[8];  // [4 j + k]
  int bias;
  float sx;
};

__device__ __forceinline__ void pack_group(const int (&xi)[32], float sx, XGroup2& g) {
  g.sx = sx;
  int sum = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t hi = 0, lo = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int x = xi[16 * j + 4 * b + k];
        sum += x;
        hi |= (static_cast<uint32_t>(x >> 8) & 0xFFu) << (8 * b);
        lo |= (static_cast<uint32_t>(x) & 0xFFu) << (8 * b);
      }
      g.hi[4 * j + k] = hi;
      g.lo[4 * j + k] = lo;
    }
  }
  g.bias = -2 * sum;
}

__device__ __forceinline__ void quantise_group(const float (&v)[32], XGroup2& g) {
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
  const float inv = mx > 0.f ? 32767.f / mx : 0.f;
  int xi[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) xi[i] = __float2int_rn(v[i] * inv);
  pack_group(xi, mx / 32767.f, g);
}

// Exact integer dot of 32 2-bit codes (minus 2) with the group's x_int.
__device__ __forceinline__ int dot_group(const uint2 q, const XGroup2& g) {
  const uint32_t w[2] = {q.x, q.y};
  int h0 = 0, h1 = 0, l0 = g.bias, l1 = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
      const uint32_t f0 = (w[j] >> (2 * k)) & 0x03030303u;
      const uint32_t f1 = (w[j] >> (2 * k + 2)) & 0x03030303u;
      h0 = dp4a_us(f0, g.hi[4 * j + k], h0);
      l0 = dp4a_uu(f0, g.lo[4 * j + k], l0);
      h1 = dp4a_us(f1, g.hi[4 * j + k + 1], h1);
      l1 = dp4a_uu(f1, g.lo[4 * j + k + 1], l1);
    }
  }
  return (h0 + h1) * 256 + l0 + l1;
}

// The SRQ input of a quantised linear: x_int = srq code, scale s -- the dot is
// then exactly sum (q - zp) * code, the reference's sum-a zero-point fold
// (gemma4_150/kernels_dsl.py:396-397) done in integers.
template <typename XG>
__device__ __forceinline__ void srq_group(const float (&v)[32], float s, XG& g) {
  int xi[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) xi[i] = srq_code(v[i], s);
  pack_group(xi, s, g);
}

// The group types and weight chunk of one 32-value group by code width.
template <int BITS>
struct QTraits;
template <>
struct QTraits<4> {
  using XG = XGroup;
  using Chunk = uint4;  // 16 bytes of nibbles
};
template <>
struct QTraits<2> {
  using XG = XGroup2;
  using Chunk = uint2;  // 8 bytes of 2-bit codes
};

}  // namespace sbd
