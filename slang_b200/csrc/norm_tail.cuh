// The last-arriver norm-add tail of a projection GEMV (the reference's
// oproj_73 / down_75 / pleproj_77 tails, gemma4_150/kernels_dsl.py:398-429,
// 928-996, 1057-1127): after every CTA has written its rows of y, the CTA that
// completes a counter computes, per row r,
//   hidden[r] = (hidden[r] + rmsnorm(y[r]) * w_post) * scalar
//   h         = rmsnorm(hidden[r]) * w_next        (when w_next != null)
// and re-arms the counter.  No CTA waits on another.
#pragma once

#include "common.cuh"

namespace sbd {

struct NormTail {
  float* hidden;
  const float* w_post;
  const float* w_next;
  float* h_out;
  __half* h16;
  unsigned int* counter;
  float scalar, eps;
};

__device__ __forceinline__ float tail_block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
  return t;
}

// hidden, h_out, h16 have row stride n.  Run by every thread of the last-arriving CTA, after a fence: the other CTAs'
// rows of y are read through L2 (ld.global.cg), never from a stale L1 line.
// A thread holds up to kTailV4 float4s of a row (n <= 4 * kTailV4 * blockDim,
// n % 4 == 0) and issues each phase's loads together: one L2 round trip per phase.
constexpr int kTailV4 = 8;
static __device__ __noinline__ void norm_tail_rows(const float* y, int ldy, int m, int n, const NormTail& t) {
  __shared__ float red[32];
  const int n4 = n >> 2, nt = blockDim.x;
  for (int r = 0; r < m; ++r) {
    const float4* pr = reinterpret_cast<const float4*>(y + static_cast<int64_t>(r) * ldy);
    float4* hr = reinterpret_cast<float4*>(t.hidden + static_cast<int64_t>(r) * n);
    float4 v[kTailV4], xv[kTailV4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kTailV4; ++j) {
      const int i = threadIdx.x + j * nt;
      v[j] = i < n4 ? __ldcg(pr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      xv[j] = i < n4 ? hr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kTailV4; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    const float d = sqrtf(tail_block_sum(ss, red) / n + t.eps);
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < kTailV4; ++j) {
      const int i = threadIdx.x + j * nt;
      if (i < n4) {
        const float4 wp = reinterpret_cast<const float4*>(t.w_post)[i];
        v[j] = make_float4((xv[j].x + v[j].x / d * wp.x) * t.scalar, (xv[j].y + v[j].y / d * wp.y) * t.scalar,
                           (xv[j].z + v[j].z / d * wp.z) * t.scalar, (xv[j].w + v[j].w / d * wp.w) * t.scalar);
        hr[i] = v[j];
        ss2 += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      }
    }
    if (!t.w_next) continue;
    const float d2 = sqrtf(tail_block_sum(ss2, red) / n + t.eps);
#pragma unroll
    for (int j = 0; j < kTailV4; ++j) {
      const int i = threadIdx.x + j * nt;
      if (i < n4) {
        const float4 wn = reinterpret_cast<const float4*>(t.w_next)[i];
        const float4 h = make_float4(v[j].x / d2 * wn.x, v[j].y / d2 * wn.y, v[j].z / d2 * wn.z, v[j].w / d2 * wn.w);
        if (t.h_out) reinterpret_cast<float4*>(t.h_out + static_cast<int64_t>(r) * n)[i] = h;
        if (t.h16) {
          __half* o16 = t.h16 + static_cast<int64_t>(r) * n + 4 * i;
          o16[0] = __float2half_rn(h.x), o16[1] = __float2half_rn(h.y);
          o16[2] = __float2half_rn(h.z), o16[3] = __float2half_rn(h.w);
        }
      }
    }
  }
}

// The end of a GEMV launch with a tail: count this CTA in once all of its rows
// are written; the CTA that completes the count runs the tail and re-arms the
// counter.  Every thread of every CTA calls this (no early exit in between).
__device__ __forceinline__ void last_arriver_tail(const float* y, int ldy, int m, int n, const NormTail& t) {
  __shared__ unsigned int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(t.counter, 1u) == gridDim.x - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  norm_tail_rows(y, ldy, m, n, t);
  __syncthreads();
  if (threadIdx.x == 0) *t.counter = 0u;
}

}  // namespace sbd
