// Glue of the Gemma-4-E2B-shaped decoder around the quantized matmuls:
// embedding gather, residual add + RMSNorm, q/k/v norm + RoPE + KV-cache
// store, causal softmax (prefill), GEGLU, split-KV decode attention, and the
// per-step position/token bookkeeping that lets a whole decode step replay as
// one CUDA graph.  Arithmetic follows the reference's f32 numpy decoder
// (gemma4/reference.py:19-56, 103-152): RMSNorm is x / sqrt(mean(x^2) + eps) * w,
// RoPE is rotate_half on precomputed cos/sin tables, attention scaling is 1.0.
#include <algorithm>

#include "common.cuh"
#include "q4_dot.cuh"

namespace {

constexpr int kT = 256;  // threads per CTA for the row kernels

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// sum over a CTA of kT threads (red: >= 32 floats of shared memory)
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float load_act(const void* p, int is_f16, size_t i) {
  return is_f16 ? __half2float(static_cast<const __half*>(p)[i]) : static_cast<const float*>(p)[i];
}

using sbd::gelu_tanh;

// ---------------------------------------------------------------- embedding
// Row gather + dequant of a packed table: BITS-bit codes, low bits first in
// each byte (4-bit: ZP 8; 2-bit: ZP 2, the checkpoint's embedding), one scale
// per `group` values.
template <int BITS>
__global__ void embed_kernel(const uint8_t* __restrict__ emb, const void* __restrict__ scales, int sf16, int group,
                             const int32_t* __restrict__ tokens, int k, float mult, float* out32, __half* out16) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  constexpr int kPer = 8 / BITS, kMask = (1 << BITS) - 1, kZp = 1 << (BITS - 1);
  const int row = blockIdx.x;
  const int64_t tok = tokens[row];
  const int gps = k / group;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const uint8_t b = emb[tok * (k / kPer) + i / kPer];
    const int q = ((b >> (BITS * (i % kPer))) & kMask) - kZp;
    const size_t si = static_cast<size_t>(tok) * gps + i / group;
    const float s = sf16 ? __half2float(static_cast<const __half*>(scales)[si]) : static_cast<const float*>(scales)[si];
    // reference: (ints * repeat(scale)) * embed_scale, each product rounded in f32
    const float v = __fmul_rn(__fmul_rn(static_cast<float>(q), s), mult);
    if (out32) out32[static_cast<size_t>(row) * k + i] = v;
    if (out16) out16[static_cast<size_t>(row) * k + i] = __float2half_rn(v);
  }
}

// ---------------------------------------------------------------- add + RMSNorm
// x_out = x + rmsnorm(y) * w_add   (when y != null; else x_out = x)
// h     = rmsnorm(x_out) * w_norm  -> h_out (f32) and/or h16 (f16)
// One CTA per row; n % 4 == 0, n <= 4 * kT * MAXV4; values stay in registers.
constexpr int MAXV4 = 8;

__device__ __forceinline__ float4 load4(const void* p, int is_f16, size_t i) {
  if (is_f16) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + i);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
}

__global__ void add_rmsnorm_kernel(const float* __restrict__ x, const void* __restrict__ y, int y_f16,
                                   const float* __restrict__ w_add, const float* __restrict__ w_norm, float* x_out,
                                   float* h_out, __half* h16, int n, float eps) {
  __shared__ float red[32];
  sbd::griddep_launch_dependents();
  const int row = blockIdx.x;
  const size_t base = static_cast<size_t>(row) * n;
  const int n4 = n >> 2;
  float4 v[MAXV4];
  float ss = 0.f;
  sbd::griddep_wait();
  if (y) {
#pragma unroll
    for (int j = 0; j < MAXV4; ++j) {
      const int i = threadIdx.x + j * kT;
      v[j] = i < n4 ? load4(y, y_f16, base + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
    const float d = sqrtf(block_sum(ss, red) / n + eps);
    ss = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV4; ++j) {
      const int i = threadIdx.x + j * kT;
      if (i < n4) {
        const float4 xv = *reinterpret_cast<const float4*>(x + base + 4 * i);
        const float4 wa = *reinterpret_cast<const float4*>(w_add + 4 * i);
        v[j] = make_float4(xv.x + v[j].x / d * wa.x, xv.y + v[j].y / d * wa.y, xv.z + v[j].z / d * wa.z,
                           xv.w + v[j].w / d * wa.w);
        if (x_out) *reinterpret_cast<float4*>(x_out + base + 4 * i) = v[j];
      }
      ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < MAXV4; ++j) {
      const int i = threadIdx.x + j * kT;
      v[j] = i < n4 ? *reinterpret_cast<const float4*>(x + base + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n4 && x_out && x_out != x) *reinterpret_cast<float4*>(x_out + base + 4 * i) = v[j];
      ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
  }
  const float d = sqrtf(block_sum(ss, red) / n + eps);
#pragma unroll
  for (int j = 0; j < MAXV4; ++j) {
    const int i = threadIdx.x + j * kT;
    if (i < n4) {
      const float4 wn = *reinterpret_cast<const float4*>(w_norm + 4 * i);
      const float4 h = make_float4(v[j].x / d * wn.x, v[j].y / d * wn.y, v[j].z / d * wn.z, v[j].w / d * wn.w);
      if (h_out) *reinterpret_cast<float4*>(h_out + base + 4 * i) = h;
      if (h16) {
        __half2 a = __floats2half2_rn(h.x, h.y), b = __floats2half2_rn(h.z, h.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(h16 + base + 4 * i) = u;
      }
    }
  }
}

// ---------------------------------------------------------------- add + RMSNorm, warp per row
// The same arithmetic for rows of n = 256 * nc (nc <= 8) values: one warp per
// row holds 8 consecutive values per 256-wide chunk in registers, reduces with
// shuffles only, and moves 16-byte vectors.  The RMS divisions become one
// reciprocal per norm and products (within 1.5 ulp of x / d).
constexpr int kRowWarps = 8;  // rows per CTA

__device__ __forceinline__ void ld8(const void* p, int is_f16, size_t i, float (&v)[8]) {
  if (is_f16) {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}
__device__ __forceinline__ void st8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void st8h(__half* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __half2 h = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// The CTA stages w_add and w_norm in shared memory before it waits for the
// previous kernel (they are constants), so a row costs one dependent global
// round trip (x, y) instead of three.
template <int NC>
__global__ void __launch_bounds__(kRowWarps * 32) add_rmsnorm_warp_kernel(
    const float* __restrict__ x, const void* __restrict__ y, int y_f16, const float* __restrict__ w_add,
    const float* __restrict__ w_norm, float* x_out, float* h_out, __half* h16, int m, float eps) {
  constexpr int n = NC * 256;
  extern __shared__ float wsm[];  // [w_add (n, when y)] [w_norm (n)]
  float* wa_s = wsm;
  float* wn_s = wsm + (y ? n : 0);
  sbd::griddep_launch_dependents();
  for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
    if (y) reinterpret_cast<float4*>(wa_s)[i] = __ldg(reinterpret_cast<const float4*>(w_add) + i);
    reinterpret_cast<float4*>(wn_s)[i] = __ldg(reinterpret_cast<const float4*>(w_norm) + i);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  const size_t base = static_cast<size_t>(row) * n;
  sbd::griddep_wait();
  if (row >= m) return;
  float v[NC][8];
  // all of a lane's loads are issued before any is used
  if (y) {
    float yv[NC][8];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      ld8(y, y_f16, base + c * 256 + lane * 8, yv[c]);
      ld8(x, 0, base + c * 256 + lane * 8, v[c]);
    }
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += yv[c][e] * yv[c][e];
    const float rd = 1.0f / sqrtf(warp_sum(ss) / n + eps);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float wa[8];
      ld8(wa_s, 0, c * 256 + lane * 8, wa);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[c][e] = v[c][e] + yv[c][e] * rd * wa[e];
      if (x_out) st8(x_out + base + c * 256 + lane * 8, v[c]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      ld8(x, 0, base + c * 256 + lane * 8, v[c]);
      if (x_out && x_out != x) st8(x_out + base + c * 256 + lane * 8, v[c]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[c][e] * v[c][e];
  const float rd = 1.0f / sqrtf(warp_sum(ss) / n + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float wn[8], h[8];
    ld8(wn_s, 0, c * 256 + lane * 8, wn);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = v[c][e] * rd * wn[e];
    if (h_out) st8(h_out + base + c * 256 + lane * 8, h);
    if (h16) st8h(h16 + base + c * 256 + lane * 8, h);
  }
}

// ---------------------------------------------------------------- q/k/v prep
// One CTA per token (nh + 2 warps): warp h < nh normalises + ropes query head h,
// warp nh the key (written to the f32 cache and its f16 copy), warp nh+1 the
// value (parameter-free RMSNorm).  hd = 32 * VPL; a lane holds VH = VPL / 2
// consecutive values of each half of the head, so the rotate_half pairs
// (i, i + hd/2) meet in one lane and every access is a vector of VH.  The RMS
// division is one reciprocal and products (within 1.5 ulp of x / d).
template <int VH>
__device__ __forceinline__ void ldv(const void* p, int is_f16, size_t i, float (&v)[VH]);
template <int VH>
__device__ __forceinline__ void stv(float* p, const float (&v)[VH]);
template <int VH>
__device__ __forceinline__ void stvh(__half* p, const float (&v)[VH]);

// 8 values (head_dim 512) as two 4-value accesses
template <>
__device__ __forceinline__ void ldv<8>(const void* p, int is_f16, size_t i, float (&v)[8]) {
  float a[4], b[4];
  ldv<4>(p, is_f16, i, a);
  ldv<4>(p, is_f16, i + 4, b);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[e] = a[e];
    v[4 + e] = b[e];
  }
}
template <>
__device__ __forceinline__ void stv<8>(float* p, const float (&v)[8]) {
  const float a[4] = {v[0], v[1], v[2], v[3]}, b[4] = {v[4], v[5], v[6], v[7]};
  stv<4>(p, a);
  stv<4>(p + 4, b);
}
template <>
__device__ __forceinline__ void stvh<8>(__half* p, const float (&v)[8]) {
  const float a[4] = {v[0], v[1], v[2], v[3]}, b[4] = {v[4], v[5], v[6], v[7]};
  stvh<4>(p, a);
  stvh<4>(p + 4, b);
}

template <int VH>
__device__ __forceinline__ void ldv(const void* p, int is_f16, size_t i, float (&v)[VH]) {
  if (is_f16) {
    const __half* h = static_cast<const __half*>(p) + i;
    if constexpr (VH == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(h);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else if constexpr (VH == 2) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(h));
      v[0] = a.x; v[1] = a.y;
    } else {
      v[0] = __half2float(h[0]);
    }
  } else {
    const float* f = static_cast<const float*>(p) + i;
    if constexpr (VH == 4) {
      const float4 a = *reinterpret_cast<const float4*>(f);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    } else if constexpr (VH == 2) {
      const float2 a = *reinterpret_cast<const float2*>(f);
      v[0] = a.x; v[1] = a.y;
    } else {
      v[0] = f[0];
    }
  }
}
template <int VH>
__device__ __forceinline__ void stv(float* p, const float (&v)[VH]) {
  if constexpr (VH == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  else if constexpr (VH == 2) *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  else p[0] = v[0];
}
template <int VH>
__device__ __forceinline__ void stvh(__half* p, const float (&v)[VH]) {
  if constexpr (VH == 4) {
    __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  } else if constexpr (VH == 2) {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v[0], v[1]);
  } else {
    p[0] = __float2half_rn(v[0]);
  }
}

template <int VPL>
__global__ void qkv_prep_kernel(const void* __restrict__ qkv, int qkv_f16, int ld, const float* __restrict__ q_norm,
                                const float* __restrict__ k_norm, const float* __restrict__ cos_t,
                                const float* __restrict__ sin_t, const int32_t* __restrict__ pos_dev, int start_pos,
                                int nh, float eps, __half* q16, float* q32, float* k_cache, float* v_cache,
                                __half* k16, __half* v16, int64_t cache_stride) {
  constexpr int HD = 32 * VPL, HALF = HD / 2, VH = VPL / 2;
  sbd::griddep_launch_dependents();
  const int s = blockIdx.x;  // token (prefill) or sequence (decode)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = lane * VH;  // this lane's offset within each half
  // constants first (norm weights; the RoPE row when the position is known),
  // so they are in registers when the previous kernel's q|k|v arrive
  float wa[VH], wb[VH], c[VH], sn[VH];
  if (warp <= nh) {
    const float* w = warp < nh ? q_norm : k_norm;
    ldv<VH>(w, 0, i0, wa);
    ldv<VH>(w, 0, HALF + i0, wb);
    if (!pos_dev) {
      ldv<VH>(cos_t, 0, static_cast<size_t>(start_pos + s) * HALF + i0, c);
      ldv<VH>(sin_t, 0, static_cast<size_t>(start_pos + s) * HALF + i0, sn);
    }
  }
  sbd::griddep_wait();
  const int pos = pos_dev ? pos_dev[s] : start_pos + s;
  const size_t row = static_cast<size_t>(s) * ld;
  const int col0 = warp * HD;  // q heads, then k, then v
  float a[VH], b[VH];
  ldv<VH>(qkv, qkv_f16, row + col0 + i0, a);
  ldv<VH>(qkv, qkv_f16, row + col0 + HALF + i0, b);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < VH; ++e) ss += a[e] * a[e] + b[e] * b[e];
  const float rd = 1.0f / sqrtf(warp_sum(ss) / HD + eps);
  if (warp <= nh) {
    if (pos_dev) {
      ldv<VH>(cos_t, 0, static_cast<size_t>(pos) * HALF + i0, c);
      ldv<VH>(sin_t, 0, static_cast<size_t>(pos) * HALF + i0, sn);
    }
#pragma unroll
    for (int e = 0; e < VH; ++e) {
      const float x0 = a[e] * rd * wa[e], x1 = b[e] * rd * wb[e];
      // rotate_half: dims i and i + HALF pair up
      a[e] = x0 * c[e] - x1 * sn[e];
      b[e] = x1 * c[e] + x0 * sn[e];
    }
  } else {
#pragma unroll
    for (int e = 0; e < VH; ++e) {
      a[e] *= rd;
      b[e] *= rd;
    }
  }
  if (warp < nh) {
    const size_t qb = (static_cast<size_t>(s) * nh + warp) * HD;
    if (q16) {
      stvh<VH>(q16 + qb + i0, a);
      stvh<VH>(q16 + qb + HALF + i0, b);
    }
    if (q32) {
      stv<VH>(q32 + qb + i0, a);
      stv<VH>(q32 + qb + HALF + i0, b);
    }
  } else {
    const int seq = pos_dev ? s : 0;
    const size_t cb = static_cast<size_t>(seq) * cache_stride + static_cast<size_t>(pos) * HD;
    float* cache = warp == nh ? k_cache : v_cache;
    __half* c16 = warp == nh ? k16 : v16;
    stv<VH>(cache + cb + i0, a);
    stv<VH>(cache + cb + HALF + i0, b);
    if (c16) {
      stvh<VH>(c16 + cb + i0, a);
      stvh<VH>(c16 + cb + HALF + i0, b);
    }
  }
}

// ---------------------------------------------------------------- causal softmax
// Row r is query token s = r / nh (absolute position start + s); keys t <= that
// position get f16(exp(score - max) / sum), later keys (up to n_keys) get 0.
__global__ void softmax_causal_kernel(const float* __restrict__ scores, int ld_s, int nh, int start_pos, int n_keys,
                                      int window, __half* p16, int ld_p) {
  __shared__ float red[32];
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int r = blockIdx.x;
  const int last = start_pos + r / nh;  // inclusive
  // a sliding-window layer sees the `window` keys ending at its own position
  const int first = window > 0 ? max(0, last + 1 - window) : 0;
  const float* srow = scores + static_cast<size_t>(r) * ld_s;
  float m = -INFINITY;
  for (int t = first + threadIdx.x; t <= last; t += blockDim.x) m = fmaxf(m, srow[t]);
  m = warp_max(m);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = (threadIdx.x & 31) < (blockDim.x >> 5) ? red[threadIdx.x & 31] : -INFINITY;
  m = warp_max(m);
  float l = 0.f;
  for (int t = first + threadIdx.x; t <= last; t += blockDim.x) l += expf(srow[t] - m);
  l = block_sum(l, red);
  __half* prow = p16 + static_cast<size_t>(r) * ld_p;
  for (int t = threadIdx.x; t < n_keys; t += blockDim.x)
    prow[t] = t >= first && t <= last ? __float2half_rn(expf(srow[t] - m) / l) : __float2half_rn(0.f);
}

// ---------------------------------------------------------------- SRQ
// out[i] = srq(x[i], s) = clip(round(x / s), -128, 127) * s (gemma4_150/reference.py:30-31),
// read and written as f32 or f16 (f16 output rounds the quantised value).
__global__ void srq_kernel(const void* __restrict__ x, int x_f16, size_t n, float s, void* out, int out_f16) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = static_cast<float>(sbd::srq_code(load_act(x, x_f16, i), s)) * s;
    if (out_f16) static_cast<__half*>(out)[i] = __float2half_rn(v);
    else static_cast<float*>(out)[i] = v;
  }
}

// ---------------------------------------------------------------- GEGLU
// out[r, i] = gelu_tanh(gu[r, 2i]) * gu[r, 2i + 1]  (gate and up rows interleaved)
__global__ void geglu_kernel(const void* __restrict__ gu, int gu_f16, int f, int rows, float* out32, __half* out16) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const size_t total = static_cast<size_t>(rows) * f;
  for (size_t e = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = e / f, i = e - r * f;
    const float g = load_act(gu, gu_f16, r * 2 * f + 2 * i);
    const float u = load_act(gu, gu_f16, r * 2 * f + 2 * i + 1);
    const float v = gelu_tanh(g) * u;
    if (out32) out32[e] = v;
    if (out16) out16[e] = __float2half_rn(v);
  }
}

// ---------------------------------------------------------------- decode attention
// Split-KV decode attention for one KV head shared by NH query heads
// (flash-decoding).  CTA (b, split) owns keys [split * spk, (split + 1) * spk)
// of sequence b and walks them in chunks of CK = 32 keys with an online
// softmax; the merge kernel rescales the splits.  The chunk loop is
// software-pipelined: V of chunk c + 1 is bulk-copied into the other of two
// shared-memory buffers and K of chunk c + 1 is loaded into registers while
// chunk c's softmax and P.V run.  Shared-memory bandwidth, not arithmetic,
// bounds the inner loops, so each loop reuses every shared-memory read:
//   scores:  thread (key pair (p, p + 16), slice s of 16) holds both keys'
//            dims {4 (s + 16 j) .. + 3} in registers and forms 2 x NH partial
//            dots (each q float4 read serves two keys); a reduce-scatter over
//            the 16 slice lanes leaves one (key, head) score per lane.
//   softmax: warp w owns heads w and w + 8 and keeps their running max / sum
//            in registers.
//   P.V:     thread (key half, head group, 4 dims) accumulates HPT heads x 4
//            dims over its 16 keys of every chunk (each V float4 read serves
//            HPT heads); the halves are added once, at the end of the split.
constexpr int CK = 32;

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

// Sum v over the 16 lanes that share lane / 16; afterwards lane s = lane & 15
// holds the totals of entries s * N / 16 .. s * N / 16 + N / 16 - 1 in
// v[0 .. N/16).
template <int N>
__device__ __forceinline__ void reduce_scatter16(float (&v)[N]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int dist = 8 >> step;
    const int cnt = N >> (step + 1);
    const bool up = (lane & dist) != 0;
#pragma unroll
    for (int i = 0; i < cnt; ++i) {
      const float send = up ? v[i] : v[i + cnt];
      const float keep = up ? v[i + cnt] : v[i];
      v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, dist);
    }
  }
}

template <int HD, int NH>
struct DecodeAttnShape {
  static constexpr int kThreads = 256;
  static constexpr int J = HD / 64;                        // float4 of a K row per thread
  static constexpr int NA = NH < 8 ? 8 : NH;               // scores per key (padded: 2 NA >= 16 lanes)
  static constexpr int R = 2 * NA / 16;                    // (key, head) scores per lane after the reduce-scatter
  static constexpr int HPT = NH * HD / 4 >= 128 ? NH * HD / 4 / 128 : 1;  // heads per P.V thread
  static constexpr int PVT = (NH / HPT) * (HD / 4);        // P.V threads per key half
  static constexpr int SP = CK + 4;                        // score row stride (conflict-free, 16-byte rows)
  static constexpr size_t smem_floats = 2 * CK * HD + NH * HD + NH * SP + 16 + 4;
  static_assert(NH <= 16 && PVT <= 128 && NH * HD <= 2 * CK * HD, "shape");
};

template <int HD, int NH>
__global__ void __launch_bounds__(256, 2) attn_decode_split_kernel(const float* __restrict__ q32,
                                                                const float* __restrict__ k_cache,
                                                                const float* __restrict__ v_cache,
                                                                const int32_t* __restrict__ pos_dev,
                                                                int64_t cache_stride, float* part, int spk,
                                                                int max_splits, int window, int* err) {
  using Sh = DecodeAttnShape<HD, NH>;
  constexpr int J = Sh::J, NA = Sh::NA, R = Sh::R, HPT = Sh::HPT, SP = Sh::SP;
  extern __shared__ __align__(16) float sm[];
  float* vs = sm;                  // [2][CK][HD] V of the chunk in flight / in use
  float* qs = vs + 2 * CK * HD;    // [NH][HD]
  float* ss = qs + NH * HD;        // [NH][SP] scores, then probabilities
  float* sc = ss + NH * SP;        // [16] this chunk's rescale factor per head
  uint64_t* bar = reinterpret_cast<uint64_t*>(sc + 16);  // [2] V buffers
  __shared__ int abort_flag;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x, sp = blockIdx.y;
  sbd::griddep_launch_dependents();
  if (tid == 0) {
    abort_flag = 0;
    sbd::mbar_init(&bar[0], 1);
    sbd::mbar_init(&bar[1], 1);
    sbd::fence_mbar_init();
  }
  sbd::griddep_wait();
  const int T = pos_dev[b] + 1;
  // a sliding-window layer attends to the last `window` keys; splits wholly
  // before them do nothing (the merge starts at the split holding the first)
  const int first = window > 0 ? max(0, T - window) : 0;
  const int k0 = max(sp * spk, first);
  if (k0 >= T || (sp + 1) * spk <= first) return;  // uniform over the CTA
  const int k1 = min(T, (sp + 1) * spk);
  const int nchunk = (k1 - k0 + CK - 1) / CK;
  const float* kb = k_cache + static_cast<size_t>(b) * cache_stride;
  const float* vb = v_cache + static_cast<size_t>(b) * cache_stride;
  __syncthreads();  // barrier initialisation before any use
  auto issue_v = [&](int c) {
    const int t0 = k0 + c * CK, nt = min(CK, k1 - t0);
    const uint32_t bytes = static_cast<uint32_t>(nt) * HD * sizeof(float);
    sbd::mbar_arrive_expect_tx(&bar[c & 1], bytes);
    sbd::bulk_load(vs + (c & 1) * CK * HD, vb + static_cast<size_t>(t0) * HD, bytes, &bar[c & 1]);
  };
  if (tid == 0) issue_v(0);
  // score roles: keys kp and kp + 16, slice s16 of 16
  const int kp = warp * 2 + (lane >> 4), s16 = lane & 15;
  float4 kr[2][J];
  auto load_k = [&](int c) {
    const int t0 = k0 + c * CK;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int t = kp + 16 * u;
      const bool in = t0 + t < k1;
      const float4* src = reinterpret_cast<const float4*>(kb + static_cast<size_t>(t0 + (in ? t : 0)) * HD);
#pragma unroll
      for (int j = 0; j < J; ++j) kr[u][j] = in ? src[s16 + 16 * j] : f4_zero();
    }
  };
  load_k(0);
  for (int i = tid; i < NH * HD / 4; i += Sh::kThreads)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(q32 + static_cast<size_t>(b) * NH * HD)[i];
  // P.V role: key half kh (keys 16 kh .. + 15 of each chunk), head group hg, dims 4 c4 .. + 3
  const int kh = tid >> 7, c4 = (tid & 127) % (HD / 4), hg = (tid & 127) / (HD / 4);
  const bool pv = (tid & 127) < Sh::PVT;
  float4 o[HPT];
#pragma unroll
  for (int i = 0; i < HPT; ++i) o[i] = f4_zero();
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  for (int c = 0; c < nchunk; ++c) {
    const int t0 = k0 + c * CK, nt = min(CK, k1 - t0);
    __syncthreads();  // q staged; previous P.V done with ss, sc and V buffer (c + 1) & 1
    if (c + 1 < nchunk && tid == 0) issue_v(c + 1);
    float acc[2 * NA];
#pragma unroll
    for (int e = 0; e < 2 * NA; ++e) acc[e] = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float4 q = reinterpret_cast<const float4*>(qs + h * HD)[s16 + 16 * j];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float a = acc[u * NA + h];
          a = fmaf(q.x, kr[u][j].x, a);
          a = fmaf(q.y, kr[u][j].y, a);
          a = fmaf(q.z, kr[u][j].z, a);
          a = fmaf(q.w, kr[u][j].w, a);
          acc[u * NA + h] = a;
        }
      }
    }
    reduce_scatter16<2 * NA>(acc);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int e = s16 * R + r, u = e / NA, h = e % NA;
      if (h < NH) ss[h * SP + kp + 16 * u] = acc[r];
    }
    if (c + 1 < nchunk) load_k(c + 1);
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int h = warp + 8 * u;
      if (h < NH) {
        const float x = lane < nt ? ss[h * SP + lane] : -INFINITY;
        const float mn = fmaxf(m_run[u], warp_max(x));
        const float pr = lane < nt ? expf(x - mn) : 0.f;
        const float f = expf(m_run[u] - mn);
        l_run[u] = l_run[u] * f + warp_sum(pr);
        m_run[u] = mn;
        ss[h * SP + lane] = pr;
        if (lane == 0) sc[h] = f;
      }
    }
    const bool bad = !sbd::mbar_wait(&bar[c & 1], (c >> 1) & 1, &abort_flag, err);
    if (__syncthreads_or(bad)) {
      // leave no copy in flight into this CTA's shared memory (bounded)
      if (tid == 0 && c + 1 < nchunk) {
        const uint64_t t_start = sbd::global_ns();
        while (!sbd::mbar_try_wait(&bar[(c + 1) & 1], ((c + 1) >> 1) & 1) &&
               sbd::global_ns() - t_start < sbd::kWaitLimitNs) {
        }
      }
      return;
    }
    if (pv) {
      const float* vbuf = vs + (c & 1) * CK * HD;
#pragma unroll
      for (int i = 0; i < HPT; ++i) {
        const float f = sc[hg * HPT + i];
        o[i].x *= f;
        o[i].y *= f;
        o[i].z *= f;
        o[i].w *= f;
      }
      const int te = min(nt, 16 * kh + 16);
      for (int t = 16 * kh; t < te; t += 4) {
        float4 v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          v[e] = t + e < nt ? reinterpret_cast<const float4*>(vbuf + (t + e) * HD)[c4] : f4_zero();
#pragma unroll
        for (int i = 0; i < HPT; ++i) {
          const float4 p4 = *reinterpret_cast<const float4*>(ss + (hg * HPT + i) * SP + t);
          const float pe[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            o[i].x = fmaf(pe[e], v[e].x, o[i].x);
            o[i].y = fmaf(pe[e], v[e].y, o[i].y);
            o[i].z = fmaf(pe[e], v[e].z, o[i].z);
            o[i].w = fmaf(pe[e], v[e].w, o[i].w);
          }
        }
      }
    }
  }
  // add the key halves (through the idle V buffers), then write rows of
  // HD + 2 floats: (HD) unnormalised output, running max, running sum
  __syncthreads();
  float4* ox = reinterpret_cast<float4*>(vs);
  if (pv && kh == 1) {
#pragma unroll
    for (int i = 0; i < HPT; ++i) ox[(hg * HPT + i) * (HD / 4) + c4] = o[i];
  }
  __syncthreads();
  float* pbase = part + (static_cast<size_t>(b) * max_splits + sp) * NH * (HD + 2);
  if (pv && kh == 0) {
#pragma unroll
    for (int i = 0; i < HPT; ++i) {
      const float4 y = ox[(hg * HPT + i) * (HD / 4) + c4];
      float2* d = reinterpret_cast<float2*>(pbase + (hg * HPT + i) * (HD + 2) + 4 * c4);
      d[0] = make_float2(o[i].x + y.x, o[i].y + y.y);
      d[1] = make_float2(o[i].z + y.z, o[i].w + y.w);
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int h = warp + 8 * u;
    if (h < NH && lane == 0) {
      pbase[h * (HD + 2) + HD] = m_run[u];
      pbase[h * (HD + 2) + HD + 1] = l_run[u];
    }
  }
}

// Merge: CTA (b, h), thread d rescales the splits of sequence b.
__global__ void attn_decode_merge_kernel(const float* __restrict__ part, const int32_t* __restrict__ pos_dev, int nh,
                                         int hd, int spk, int max_splits, int window, float* out, __half* out16) {
  sbd::griddep_launch_dependents();
  const int b = blockIdx.x, h = blockIdx.y;
  sbd::griddep_wait();
  const int T = pos_dev[b] + 1;
  const int nc = (T + spk - 1) / spk;
  const int c0 = window > 0 ? max(0, T - window) / spk : 0;  // first split with keys in the window
  const float* base = part + (static_cast<size_t>(b) * max_splits * nh + h) * (hd + 2);
  const size_t cstride = static_cast<size_t>(nh) * (hd + 2);
  float M = -INFINITY;
  for (int c = c0; c < nc; ++c) M = fmaxf(M, base[c * cstride + hd]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int c = c0; c < nc; ++c) {
      const float* pm = base + c * cstride;
      const float f = expf(pm[hd] - M);
      L += pm[hd + 1] * f;
      O += pm[d] * f;
    }
    const size_t o = (static_cast<size_t>(b) * nh + h) * hd + d;
    if (out16) out16[o] = __float2half_rn(O / L);
    else out[o] = O / L;
  }
}

// ---------------------------------------------------------------- step bookkeeping
__global__ void step_advance_kernel(int32_t* pos, const int32_t* tokens, int32_t* cur, int32_t* history, int hist_len,
                                    int m) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= m) return;
  const int p = pos[b] + 1;
  pos[b] = p;
  cur[b] = tokens[b];
  if (history && p < hist_len) history[static_cast<size_t>(b) * hist_len + p] = tokens[b];
}

int grid_for(size_t n, int per) { return static_cast<int>(std::min<size_t>((n + per - 1) / per, 148 * 32)); }

}  // namespace

namespace {
template <int BITS>
int embed_launch(const char* name, const void* emb, const void* scales, int scale_dtype, int group,
                 const int32_t* tokens, int m, int k, float mult, float* out32, void* out16, void* stream) {
  SB_CHECK_ARG(m >= 0 && k > 0 && k % (8 / BITS) == 0 && group > 0 && k % group == 0, "%s: bad shape", name);
  SB_CHECK_ARG(scale_dtype == SB_SCALE_F16 || scale_dtype == SB_SCALE_F32, "%s: bad scale dtype", name);
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(emb && scales && tokens && (out32 || out16), "%s: null pointer", name);
  cudaError_t e = sb::launch_pdl(embed_kernel<BITS>, dim3(m), dim3(kT), 0, static_cast<cudaStream_t>(stream),
                                 static_cast<const uint8_t*>(emb), scales, static_cast<int>(scale_dtype == SB_SCALE_F16),
                                 group, tokens, k, mult, out32, static_cast<__half*>(out16));
  if (e != cudaSuccess) return sb::cuda_fail(e, "embed_kernel");
  return sb::launch_status("embed_kernel");
}
}  // namespace

extern "C" int sb_embed_q4(const void* emb, const void* scales, int scale_dtype, int group, const int32_t* tokens,
                           int m, int k, float mult, float* out32, void* out16, void* stream) {
  return embed_launch<4>("sb_embed_q4", emb, scales, scale_dtype, group, tokens, m, k, mult, out32, out16, stream);
}

extern "C" int sb_embed_q2(const void* emb, const void* scales, int scale_dtype, int group, const int32_t* tokens,
                           int m, int k, float mult, float* out32, void* out16, void* stream) {
  return embed_launch<2>("sb_embed_q2", emb, scales, scale_dtype, group, tokens, m, k, mult, out32, out16, stream);
}

extern "C" int sb_add_rmsnorm(const float* x, const void* y, int y_dtype, const float* w_add, const float* w_norm,
                              float* x_out, float* h_out, void* h16_out, int m, int n, float eps, void* stream) {
  SB_CHECK_ARG(m >= 0 && n > 0 && n % 4 == 0 && n <= 4 * kT * MAXV4, "sb_add_rmsnorm: n=%d must be a multiple of 4 in 4..%d",
               n, 4 * kT * MAXV4);
  SB_CHECK_ARG(!y || y_dtype == SB_F16 || y_dtype == SB_F32, "sb_add_rmsnorm: bad y dtype");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(x && w_norm && (!y || w_add) && (h_out || h16_out), "sb_add_rmsnorm: null pointer");
  // warp per row for rows of 256 * nc values with 16-byte aligned rows; a CTA per row otherwise
  const bool vec = n % 256 == 0 && n <= 2048 && sb::aligned(x, 16) && (!y || sb::aligned(y, 16)) &&
                   sb::aligned(w_norm, 16) && (!w_add || sb::aligned(w_add, 16)) && (!x_out || sb::aligned(x_out, 16)) &&
                   (!h_out || sb::aligned(h_out, 16)) && (!h16_out || sb::aligned(h16_out, 16));
  cudaError_t e;
  if (vec) {
    const dim3 grid((m + kRowWarps - 1) / kRowWarps), block(kRowWarps * 32);
    const size_t smem = static_cast<size_t>(y ? 2 : 1) * n * sizeof(float);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int yf = static_cast<int>(y_dtype == SB_F16);
    __half* h16 = static_cast<__half*>(h16_out);
#define SB_NORM(NC) \
  e = sb::launch_pdl(add_rmsnorm_warp_kernel<NC>, grid, block, smem, st, x, y, yf, w_add, w_norm, x_out, h_out, h16, m, eps)
    switch (n / 256) {
      case 1: SB_NORM(1); break;
      case 2: SB_NORM(2); break;
      case 3: SB_NORM(3); break;
      case 4: SB_NORM(4); break;
      case 5: SB_NORM(5); break;
      case 6: SB_NORM(6); break;
      case 7: SB_NORM(7); break;
      default: SB_NORM(8); break;
    }
#undef SB_NORM
  } else {
    e = sb::launch_pdl(add_rmsnorm_kernel, dim3(m), dim3(kT), 0, static_cast<cudaStream_t>(stream), x, y,
                       static_cast<int>(y_dtype == SB_F16), w_add, w_norm, x_out, h_out, static_cast<__half*>(h16_out), n,
                       eps);
  }
  if (e != cudaSuccess) return sb::cuda_fail(e, "add_rmsnorm_kernel");
  return sb::launch_status("add_rmsnorm_kernel");
}

extern "C" int sb_qkv_prep(const void* qkv, int qkv_dtype, int ld, const float* q_norm, const float* k_norm,
                           const float* cos_t, const float* sin_t, const int32_t* pos_dev, int start_pos, int s,
                           int n_heads, int head_dim, float eps, void* q16, float* q32, float* k_cache,
                           float* v_cache, void* k16, void* v16, int64_t cache_stride, void* stream) {
  SB_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512,
               "sb_qkv_prep: head_dim %d unsupported", head_dim);
  // no caches: a layer that reads another layer's K/V (KV sharing) -- q heads only
  const bool q_only = !k_cache && !v_cache;
  const int warps = n_heads + (q_only ? 0 : 2);
  SB_CHECK_ARG(n_heads >= 1 && warps <= 32 && s >= 0 && ld >= warps * head_dim, "sb_qkv_prep: bad shape");
  SB_CHECK_ARG(qkv_dtype == SB_F16 || qkv_dtype == SB_F32, "sb_qkv_prep: bad dtype");
  if (s == 0) return SB_OK;
  SB_CHECK_ARG(qkv && q_norm && (q_only || k_norm) && cos_t && sin_t && (q_only || (k_cache && v_cache)) &&
                   (q16 || q32),
               "sb_qkv_prep: null pointer (k_cache and v_cache are both given, or both null for q only)");
  const dim3 block(32 * warps);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int f16 = qkv_dtype == SB_F16;
  cudaError_t e;
#define SB_PREP(V)                                                                                                \
  e = sb::launch_pdl(qkv_prep_kernel<V>, dim3(s), block, 0, st, qkv, f16, ld, q_norm, k_norm, cos_t, sin_t, pos_dev, \
                     start_pos, n_heads, eps, static_cast<__half*>(q16), q32, k_cache, v_cache,                   \
                     static_cast<__half*>(k16), static_cast<__half*>(v16), cache_stride)
  if (head_dim == 64) SB_PREP(2);
  else if (head_dim == 128) SB_PREP(4);
  else if (head_dim == 256) SB_PREP(8);
  else SB_PREP(16);
#undef SB_PREP
  if (e != cudaSuccess) return sb::cuda_fail(e, "qkv_prep_kernel");
  return sb::launch_status("qkv_prep_kernel");
}

extern "C" int sb_softmax_causal(const float* scores, int ld_s, int rows, int n_heads, int start_pos, int n_keys,
                                 int window, void* p16, int ld_p, void* stream) {
  SB_CHECK_ARG(rows >= 0 && n_heads > 0 && n_keys >= 0 && ld_s >= n_keys && ld_p >= n_keys && window >= 0,
               "sb_softmax_causal: bad shape");
  SB_CHECK_ARG(start_pos + (rows - 1) / n_heads < n_keys || rows == 0, "sb_softmax_causal: a query sees past n_keys");
  if (rows == 0) return SB_OK;
  SB_CHECK_ARG(scores && p16, "sb_softmax_causal: null pointer");
  cudaError_t e = sb::launch_pdl(softmax_causal_kernel, dim3(rows), dim3(kT), 0, static_cast<cudaStream_t>(stream),
                                 scores, ld_s, n_heads, start_pos, n_keys, window, static_cast<__half*>(p16), ld_p);
  if (e != cudaSuccess) return sb::cuda_fail(e, "softmax_causal_kernel");
  return sb::launch_status("softmax_causal_kernel");
}

extern "C" int sb_srq(const void* x, int x_dtype, size_t n, float scale, void* out, int out_dtype, void* stream) {
  SB_CHECK_ARG((x_dtype == SB_F16 || x_dtype == SB_F32) && (out_dtype == SB_F16 || out_dtype == SB_F32),
               "sb_srq: bad dtype");
  SB_CHECK_ARG(scale > 0.f, "sb_srq: scale must be > 0");
  if (n == 0) return SB_OK;
  SB_CHECK_ARG(x && out, "sb_srq: null pointer");
  cudaError_t e = sb::launch_pdl(srq_kernel, dim3(grid_for(n, kT)), dim3(kT), 0, static_cast<cudaStream_t>(stream), x,
                                 static_cast<int>(x_dtype == SB_F16), n, scale, out, static_cast<int>(out_dtype == SB_F16));
  if (e != cudaSuccess) return sb::cuda_fail(e, "srq_kernel");
  return sb::launch_status("srq_kernel");
}

extern "C" int sb_geglu(const void* gu, int dtype, int m, int f, float* out32, void* out16, void* stream) {
  SB_CHECK_ARG(m >= 0 && f > 0 && (dtype == SB_F16 || dtype == SB_F32), "sb_geglu: bad arguments");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(gu && (out32 || out16), "sb_geglu: null pointer");
  const size_t total = static_cast<size_t>(m) * f;
  cudaError_t e = sb::launch_pdl(geglu_kernel, dim3(grid_for(total, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                                 gu, static_cast<int>(dtype == SB_F16), f, m, out32, static_cast<__half*>(out16));
  if (e != cudaSuccess) return sb::cuda_fail(e, "geglu_kernel");
  return sb::launch_status("geglu_kernel");
}

extern "C" size_t sb_attn_decode_workspace_size(int m, int n_heads, int head_dim, int max_seq) {
  if (m <= 0 || n_heads <= 0 || head_dim <= 0 || max_seq <= 0) return 0;
  const size_t chunks = (static_cast<size_t>(max_seq) + CK - 1) / CK;
  return static_cast<size_t>(m) * chunks * n_heads * (head_dim + 2) * sizeof(float);
}

// Raises the kernel's dynamic shared-memory limit the first time it is
// launched on a device, then launches it over grid (m, splits).
template <int HD, int NH>
static cudaError_t launch_decode_split(int m, int splits, int spk, cudaStream_t st, const float* q32,
                                       const float* k_cache, const float* v_cache, const int32_t* pos_dev,
                                       int64_t cache_stride, float* workspace, int window) {
  using Sh = DecodeAttnShape<HD, NH>;
  constexpr int smem = static_cast<int>(Sh::smem_floats * sizeof(float));
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_split_kernel<HD, NH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) set[dev] = true;
  }
  return sb::launch_pdl(attn_decode_split_kernel<HD, NH>, dim3(m, splits), dim3(Sh::kThreads), smem, st, q32, k_cache,
                        v_cache, pos_dev, cache_stride, workspace, spk, splits, window, sb::device_error_word());
}

template <int HD>
static cudaError_t launch_decode_split_hd(int nh, int m, int splits, int spk, cudaStream_t st, const float* q32,
                                          const float* k_cache, const float* v_cache, const int32_t* pos_dev,
                                          int64_t cache_stride, float* workspace, int window) {
#define SB_DEC(NH) \
  launch_decode_split<HD, NH>(m, splits, spk, st, q32, k_cache, v_cache, pos_dev, cache_stride, workspace, window)
  switch (nh) {
    case 1: return SB_DEC(1);
    case 2: return SB_DEC(2);
    case 4: return SB_DEC(4);
    case 8: return SB_DEC(8);
    default:
      if constexpr (HD <= 256) return SB_DEC(16);
      return cudaErrorInvalidValue;
  }
#undef SB_DEC
}

static int attn_decode_impl(const float* q32, const float* k_cache, const float* v_cache, int64_t cache_stride,
                            const int32_t* pos_dev, int m, int n_heads, int head_dim, int max_seq, int window,
                            float* out, __half* out16, float* workspace, size_t workspace_bytes, void* stream) {
  SB_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512,
               "sb_attn_decode: head_dim %d unsupported", head_dim);
  SB_CHECK_ARG((n_heads == 1 || n_heads == 2 || n_heads == 4 || n_heads == 8 || (n_heads == 16 && head_dim <= 256)) &&
                   m >= 0 && max_seq > 0 && window >= 0,
               "sb_attn_decode: n_heads %d not in {1, 2, 4, 8, 16 (head_dim <= 256)}, or bad shape", n_heads);
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(q32 && k_cache && v_cache && pos_dev && (out || out16) && workspace, "sb_attn_decode: null pointer");
  SB_CHECK_ARG(cache_stride % 4 == 0 && sb::aligned(q32, 16) && sb::aligned(k_cache, 16) && sb::aligned(v_cache, 16),
               "sb_attn_decode: q and the caches must be 16-byte aligned with a cache stride a multiple of 4");
  const size_t need = sb_attn_decode_workspace_size(m, n_heads, head_dim, max_seq);
  if (workspace_bytes < need)
    return sb::fail(SB_ERR_WORKSPACE, "sb_attn_decode: workspace %zu < %zu bytes", workspace_bytes, need);
  // Keys per split.  A CTA streams its chunks at a rate set by its own
  // pipeline and two CTAs per SM run at once; splits of one length finish in
  // waves, and a split costs a fixed set-up and partial write (about 40 keys'
  // worth).  Pick the chunks per split that minimise (waves) x (keys per split
  // + 40): long splits when the batch alone fills the SMs, short ones when it
  // does not.  (Judged on max_seq: the positions are on the device.)
  const int max_chunks = (max_seq + CK - 1) / CK;
  const long long slots = 2LL * sb::num_sms();
  int nch = 1;
  long long best = -1;
  for (int c = 1; c <= max_chunks; ++c) {
    const long long sp = (max_chunks + c - 1) / c;
    if (c > 1 && sp == (max_chunks + c - 2) / (c - 1)) continue;  // same split count as c - 1
    const long long waves = (static_cast<long long>(m) * sp + slots - 1) / slots;
    const long long cost = waves * (static_cast<long long>(c) * CK + 40);
    if (best < 0 || cost < best) {
      best = cost;
      nch = c;
    }
  }
  const int spk = nch * CK;
  const int splits = (max_seq + spk - 1) / spk;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
#define SB_DEC_HD(HDV) \
  launch_decode_split_hd<HDV>(n_heads, m, splits, spk, st, q32, k_cache, v_cache, pos_dev, cache_stride, workspace, window)
  if (head_dim == 64) e = SB_DEC_HD(64);
  else if (head_dim == 128) e = SB_DEC_HD(128);
  else if (head_dim == 256) e = SB_DEC_HD(256);
  else e = SB_DEC_HD(512);
#undef SB_DEC_HD
  if (e != cudaSuccess) return sb::cuda_fail(e, "attn_decode_split_kernel");
  int rc = sb::launch_status("attn_decode_split_kernel");
  if (rc) return rc;
  e = sb::launch_pdl(attn_decode_merge_kernel, dim3(m, n_heads), dim3(head_dim), 0, st,
                     static_cast<const float*>(workspace), pos_dev, n_heads, head_dim, spk, splits, window, out, out16);
  if (e != cudaSuccess) return sb::cuda_fail(e, "attn_decode_merge_kernel");
  return sb::launch_status("attn_decode_merge_kernel");
}

extern "C" int sb_attn_decode(const float* q32, const float* k_cache, const float* v_cache, int64_t cache_stride,
                              const int32_t* pos_dev, int m, int n_heads, int head_dim, int max_seq, int window,
                              float* out, float* workspace, size_t workspace_bytes, void* stream) {
  return attn_decode_impl(q32, k_cache, v_cache, cache_stride, pos_dev, m, n_heads, head_dim, max_seq, window, out,
                          nullptr, workspace, workspace_bytes, stream);
}

extern "C" int sb_attn_decode_f16(const float* q32, const float* k_cache, const float* v_cache, int64_t cache_stride,
                                  const int32_t* pos_dev, int m, int n_heads, int head_dim, int max_seq, int window,
                                  void* out16, float* workspace, size_t workspace_bytes, void* stream) {
  SB_CHECK_ARG(out16 != nullptr, "sb_attn_decode_f16: null output");
  return attn_decode_impl(q32, k_cache, v_cache, cache_stride, pos_dev, m, n_heads, head_dim, max_seq, window, nullptr,
                          static_cast<__half*>(out16), workspace, workspace_bytes, stream);
}

extern "C" int sb_step_advance(int32_t* pos, const int32_t* tokens, int32_t* cur, int32_t* history, int hist_len, int m,
                               void* stream) {
  SB_CHECK_ARG(m >= 0, "sb_step_advance: bad m");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(pos && tokens && cur, "sb_step_advance: null pointer");
  cudaError_t e = sb::launch_pdl(step_advance_kernel, dim3((m + 127) / 128), dim3(128), 0,
                                 static_cast<cudaStream_t>(stream), pos, tokens, cur, history, hist_len, m);
  if (e != cudaSuccess) return sb::cuda_fail(e, "step_advance_kernel");
  return sb::launch_status("step_advance_kernel");
}
