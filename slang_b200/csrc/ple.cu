// Per-layer-embedding (PLE) path of Gemma-4-E2B (gemma4/reference.py:92-101,
// :154-163; gemma4_150/kernels_dsl.py plegather_01 :457-478, plegate_76
// :829-870, pleproj_77 :1000-1125):
//
//   * row GEMVs for decode batches (m <= 8 per launch, any m by repetition):
//     8-bit weights (+128-biased codes, one f32 scale per output row) and
//     bf16 weights, with f32 activations and f32 accumulation; the 8-bit form
//     optionally finishes with gelu_tanh(v) * ple (the PLE input gate);
//   * the PLE tail: hidden = (hidden + rmsnorm(proj) * w_post) * layer_scalar,
//     optionally followed by the next layer's input RMSNorm;
//   * the 4-bit PLE table gather (one f32 scale per `group` values) and the
//     per-layer input combine (rmsnorm(ctx) * w + table row) * 2^-0.5.
//
// Every value stays in f32 as in the reference's weight-only numpy model; the
// GEMV decodes a weight byte with the exact magic-number conversion
// (2^23 + b as an f32 bit pattern, minus 2^23 + 128).
#include "common.cuh"
#include "norm_tail.cuh"

namespace {

constexpr int kWarps = 8;  // warps per CTA of the row GEMV
constexpr int kMaxM = 8;   // activation rows per GEMV launch
constexpr int kT = 256;    // threads per CTA of the row kernels
constexpr int kMaxV4 = 8;  // float4s per thread in the norm tail (n <= 8192)
constexpr int kU = 8;      // 16-byte weight chunks a GEMV lane has in flight

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const float t = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 16 weight bytes -> 16 values (code - 128), exact.
struct FmtQ8 {
  static constexpr int kVals = 16;
  __device__ static void decode(const uint4& w, float* v) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        // 0x4B0000bb is 2^23 + bb exactly; subtracting 2^23 + 128 leaves bb - 128
        const uint32_t bits = __byte_perm(u[j], 0x4B000000u, 0x7650 + b);
        v[4 * j + b] = __uint_as_float(bits) - 8388736.f;
      }
    }
  }
};

// 16 weight bytes -> 8 bf16 values widened to f32, exact.
struct FmtBF16 {
  static constexpr int kVals = 8;
  __device__ static void decode(const uint4& w, float* v) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(u[j] << 16);
      v[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
    }
  }
};

// 16 weight bytes -> 8 f16 values widened to f32, exact (the f16 per-layer
// model projection export.py writes).
struct FmtF16 {
  static constexpr int kVals = 8;
  __device__ static void decode(const uint4& w, float* v) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
};

// y[r, o] = epi(sum_k W[o, k] * x[r, k] * scale(o)),  scale(o) = row_scale[o] * alpha
// (row_scale may be null), epi(v) = v, or gelu_tanh(v) * ple[r * ld_ple + o].
// A group of G lanes owns one output row; each lane issues all of its (up to
// kU) 16-byte chunks of the row at once, the first pass before the dependency
// wait so that the weight reads overlap the previous kernel's tail.  M is the
// activation-row count rounded up to a power of two (m <= M rows are live).
template <class Fmt, int G, int M>
__global__ void __launch_bounds__(kWarps * 32) gemv_rows_kernel(const uint8_t* __restrict__ w, int64_t w_ld,
                                                             const float* __restrict__ row_scale, float alpha,
                                                             const float* __restrict__ x, int ldx, int m, int n,
                                                             int k, const float* __restrict__ ple, int ld_ple,
                                                             float* __restrict__ y, int ldy, sbd::NormTail tail) {
  sbd::griddep_launch_dependents();
  constexpr int kRowsPerWarp = 32 / G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gl = lane % G;
  const int o = (blockIdx.x * static_cast<int>(blockDim.x >> 5) + warp) * kRowsPerWarp + lane / G;
  const bool valid = o < n;
  const int nch = k / Fmt::kVals;
  const uint8_t* row = w + static_cast<int64_t>(valid ? o : 0) * w_ld;

  float acc[M];
#pragma unroll
  for (int r = 0; r < M; ++r) acc[r] = 0.f;
  for (int c0 = 0; c0 < nch; c0 += kU * G) {
    uint4 wv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = c0 + u * G + gl;
      wv[u] = (valid && c < nch) ? ldg_stream(row + 16 * static_cast<int64_t>(c)) : make_uint4(0u, 0u, 0u, 0u);
    }
    if (c0 == 0) sbd::griddep_wait();
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = c0 + u * G + gl;
      if (c < nch) {
        float v[Fmt::kVals];
        Fmt::decode(wv[u], v);
#pragma unroll
        for (int r = 0; r < M; ++r) {
          if (r < m) {
            const float4* xr = reinterpret_cast<const float4*>(x + static_cast<int64_t>(r) * ldx) +
                               c * (Fmt::kVals / 4);
#pragma unroll
            for (int q = 0; q < Fmt::kVals / 4; ++q) {
              const float4 xv = __ldg(xr + q);
              acc[r] = fmaf(v[4 * q], xv.x, acc[r]);
              acc[r] = fmaf(v[4 * q + 1], xv.y, acc[r]);
              acc[r] = fmaf(v[4 * q + 2], xv.z, acc[r]);
              acc[r] = fmaf(v[4 * q + 3], xv.w, acc[r]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < M; ++r) {
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) acc[r] += __shfl_xor_sync(0xFFFFFFFFu, acc[r], off);
  }
  if (valid && gl == 0) {
    const float s = row_scale ? row_scale[o] * alpha : alpha;
#pragma unroll
    for (int r = 0; r < M; ++r) {
      if (r < m) {
        float v = acc[r] * s;
        if (ple) v = sbd::gelu_tanh(v) * ple[static_cast<int64_t>(r) * ld_ple + o];
        y[static_cast<int64_t>(r) * ldy + o] = v;
      }
    }
  }
  if (tail.counter) {
    // last-arriver: publish this CTA's rows, count it in; the CTA that completes the count
    // runs the norm-add tail over all rows and re-arms the counter (no CTA waits on another)
    __shared__ unsigned int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(tail.counter, 1u) == gridDim.x - 1 ? 1u : 0u;
    __syncthreads();
    if (s_last) {
      __threadfence();
      sbd::norm_tail_rows(y, ldy, m, n, tail);
      if (threadIdx.x == 0) *tail.counter = 0u;
    }
  }
}

// hidden[r] = (hidden[r] + rmsnorm(proj[r]) * w_post) * scalar;
// then, when w_next is given, h = rmsnorm(hidden[r]) * w_next -> h_out / h16.
// One CTA per row; n % 4 == 0 and n <= 4 * kT * kMaxV4.
__global__ void __launch_bounds__(kT) ple_norm_add_kernel(const float* __restrict__ proj, float* hidden,
                                                        const float* __restrict__ w_post, float scalar,
                                                        const float* __restrict__ w_next, float* h_out, __half* h16,
                                                        int n, float eps) {
  __shared__ float red[32];
  sbd::griddep_launch_dependents();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * n;
  const int n4 = n >> 2;
  float4 v[kMaxV4];
  float ss = 0.f;
  sbd::griddep_wait();
#pragma unroll
  for (int j = 0; j < kMaxV4; ++j) {
    const int i = threadIdx.x + j * kT;
    v[j] = i < n4 ? *reinterpret_cast<const float4*>(proj + base + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  const float d = sqrtf(block_sum(ss, red) / n + eps);
  ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxV4; ++j) {
    const int i = threadIdx.x + j * kT;
    if (i < n4) {
      const float4 xv = *reinterpret_cast<const float4*>(hidden + base + 4 * i);
      const float4 wp = *reinterpret_cast<const float4*>(w_post + 4 * i);
      v[j] = make_float4((xv.x + v[j].x / d * wp.x) * scalar, (xv.y + v[j].y / d * wp.y) * scalar,
                         (xv.z + v[j].z / d * wp.z) * scalar, (xv.w + v[j].w / d * wp.w) * scalar);
      *reinterpret_cast<float4*>(hidden + base + 4 * i) = v[j];
    }
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  if (!w_next) return;
  const float d2 = sqrtf(block_sum(ss, red) / n + eps);
#pragma unroll
  for (int j = 0; j < kMaxV4; ++j) {
    const int i = threadIdx.x + j * kT;
    if (i < n4) {
      const float4 wn = *reinterpret_cast<const float4*>(w_next + 4 * i);
      const float4 h = make_float4(v[j].x / d2 * wn.x, v[j].y / d2 * wn.y, v[j].z / d2 * wn.z, v[j].w / d2 * wn.w);
      if (h_out) *reinterpret_cast<float4*>(h_out + base + 4 * i) = h;
      if (h16) {
        const __half2 a = __floats2half2_rn(h.x, h.y), b = __floats2half2_rn(h.z, h.w);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&a);
        u.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(h16 + base + 4 * i) = u;
      }
    }
  }
}

// Eight 4-bit table values (one 32-bit word, low nibble first) times their
// group's scale, times mult: (q * s) * mult with each product rounded in f32
// as the reference's (ints * repeat(scale)) * ple_scale.
__device__ __forceinline__ void table_chunk(const uint8_t* __restrict__ table, const float* __restrict__ scales,
                                            int64_t id, int cols, int group, int c, float mult, float* out) {
  const uint32_t word = *reinterpret_cast<const uint32_t*>(table + id * (cols / 2) + 4 * c);
  const float s = scales[id * (cols / group) + (8 * c) / group];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float q = static_cast<float>(static_cast<int>((word >> (4 * j)) & 15u) - 8);
    out[j] = __fmul_rn(__fmul_rn(q, s), mult);
  }
}

// y[r, :] = table row ids[r] dequantised * mult; ids outside [0, vocab) give zeros.
__global__ void __launch_bounds__(kT) ple_gather_kernel(const int32_t* __restrict__ ids,
                                                      const uint8_t* __restrict__ table,
                                                      const float* __restrict__ scales, int vocab, int cols,
                                                      int group, float mult, float* __restrict__ y) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int r = blockIdx.x;
  const int64_t id = ids[r];
  const bool ok = id >= 0 && id < vocab;
  float* yr = y + static_cast<int64_t>(r) * cols;
  for (int c = threadIdx.x; c < cols / 8; c += kT) {
    float v[8];
    if (ok) {
      table_chunk(table, scales, id, cols, group, c, mult, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    reinterpret_cast<float4*>(yr + 8 * c)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(yr + 8 * c)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// out[r, l, :] = (rmsnorm(ctx[r, l, :]) * w_norm + table[ids[r]][l*d : (l+1)*d] * mult) * 2^-0.5
// One warp per (row, layer) slice; d % 256 == 0 (a lane takes 8 values per 256).
__global__ void __launch_bounds__(kT) ple_combine_kernel(const float* __restrict__ ctx,
                                                       const int32_t* __restrict__ ids,
                                                       const uint8_t* __restrict__ table,
                                                       const float* __restrict__ scales, int vocab,
                                                       const float* __restrict__ w_norm, int m, int n_layers, int d,
                                                       int group, float mult, float eps, float* __restrict__ out) {
  sbd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int slice = blockIdx.x * (kT / 32) + (threadIdx.x >> 5);
  if (slice >= m * n_layers) {
    sbd::griddep_wait();
    return;
  }
  const int r = slice / n_layers, l = slice % n_layers;
  const int cols = n_layers * d;
  sbd::griddep_wait();
  const int64_t id = ids[r];
  const bool ok = id >= 0 && id < vocab;
  const float* cr = ctx + static_cast<int64_t>(r) * cols + static_cast<int64_t>(l) * d;
  float* orow = out + static_cast<int64_t>(r) * cols + static_cast<int64_t>(l) * d;
  float ss = 0.f;
  for (int j = lane; j < d / 8; j += 32) {
    const float4 a = reinterpret_cast<const float4*>(cr + 8 * j)[0];
    const float4 b = reinterpret_cast<const float4*>(cr + 8 * j)[1];
    ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
  }
  const float dd = sqrtf(warp_sum(ss) / d + eps);
  const float half_sqrt2 = 0.70710678118654752f;  // f32(2 ** -0.5)
  for (int j = lane; j < d / 8; j += 32) {
    float c[8], t[8];
    const float4 a = reinterpret_cast<const float4*>(cr + 8 * j)[0];
    const float4 b = reinterpret_cast<const float4*>(cr + 8 * j)[1];
    c[0] = a.x, c[1] = a.y, c[2] = a.z, c[3] = a.w, c[4] = b.x, c[5] = b.y, c[6] = b.z, c[7] = b.w;
    if (ok) {
      table_chunk(table, scales, id, cols, group, (l * d) / 8 + j, mult, t);
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) t[q] = 0.f;
    }
    float o[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = (c[q] / dd * w_norm[8 * j + q] + t[q]) * half_sqrt2;
    reinterpret_cast<float4*>(orow + 8 * j)[0] = make_float4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<float4*>(orow + 8 * j)[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}

// out16[r, o] = f16(gelu_tanh(sum_z pre[z][r, o]) * ple[r, o]): the gate tail
// once the gate is a GEMM (prefill) whose K splits wrote `nsplit` f32 planes
// `plane` elements apart, producing the f16 operand of the projection GEMM.
__global__ void __launch_bounds__(kT) ple_gate_act_kernel(const float* __restrict__ pre, int ld_pre, int64_t plane,
                                                        int nsplit, const float* __restrict__ ple, int ld_ple,
                                                        __half* out16, int ld_out, int m, int n) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int64_t total = static_cast<int64_t>(m) * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kT) {
    const int64_t r = i / n;
    const int o = static_cast<int>(i - r * n);
    float acc = pre[r * ld_pre + o];
    for (int z = 1; z < nsplit; ++z) acc += pre[z * plane + r * ld_pre + o];
    const float v = sbd::gelu_tanh(acc) * ple[r * ld_ple + o];
    out16[r * ld_out + o] = __float2half_rn(v);
  }
}

__global__ void __launch_bounds__(kT) cast_f16_kernel(const float* __restrict__ x, __half* out, int64_t n) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * kT)
    out[i] = __float2half_rn(x[i]);
}

int grid_for(int64_t total) {
  const int64_t want = (total + kT - 1) / kT;
  const int64_t cap = 8 * static_cast<int64_t>(sb::num_sms());
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

template <class Fmt, int G>
cudaError_t launch_gemv_m(int mm, dim3 grid, dim3 block, cudaStream_t st, const uint8_t* w, int64_t w_ld,
                          const float* row_scale, float alpha, const float* x, int ldx, int n, int k, const float* ple,
                          int ld_ple, float* y, int ldy, const sbd::NormTail& tail) {
#define SB_GEMV(MM)                                                                                                  \
  return sb::launch_pdl(gemv_rows_kernel<Fmt, G, MM>, grid, block, 0, st, w, w_ld, row_scale, alpha, x, ldx, mm, n, k, \
                        ple, ld_ple, y, ldy, tail)
  if (mm == 1) SB_GEMV(1);
  if (mm == 2) SB_GEMV(2);
  if (mm <= 4) SB_GEMV(4);
  SB_GEMV(8);
#undef SB_GEMV
}

template <class Fmt>
cudaError_t launch_gemv_rows(const uint8_t* w, int64_t w_ld, const float* row_scale, float alpha, const float* x,
                             int ldx, int m, int n, int k, const float* ple, int ld_ple, float* y, int ldy,
                             cudaStream_t st, const sbd::NormTail& tail = sbd::NormTail{}) {
  const int nch = k / Fmt::kVals;
  const int G = nch >= 32 ? 32 : nch >= 16 ? 16 : nch >= 8 ? 8 : 4;
  // warps per CTA: 8, fewer when a short matrix would otherwise leave SMs idle
  const int row_warps = (n + 32 / G - 1) / (32 / G);
  int wpc = kWarps;  // a fused tail keeps 8-warp CTAs: its last CTA does the tail alone
  while (!tail.counter && wpc > 1 && (row_warps + wpc - 1) / wpc < 2 * sb::num_sms()) wpc >>= 1;
  const dim3 grid((row_warps + wpc - 1) / wpc), block(wpc * 32);
  cudaError_t e = cudaSuccess;
  for (int r0 = 0; r0 < m && e == cudaSuccess; r0 += kMaxM) {
    const int mm = m - r0 < kMaxM ? m - r0 : kMaxM;
    const float* xr = x + static_cast<int64_t>(r0) * ldx;
    const float* pr = ple ? ple + static_cast<int64_t>(r0) * ld_ple : nullptr;
    float* yr = y + static_cast<int64_t>(r0) * ldy;
    switch (G) {
      case 32: e = launch_gemv_m<Fmt, 32>(mm, grid, block, st, w, w_ld, row_scale, alpha, xr, ldx, n, k, pr, ld_ple, yr, ldy, tail); break;
      case 16: e = launch_gemv_m<Fmt, 16>(mm, grid, block, st, w, w_ld, row_scale, alpha, xr, ldx, n, k, pr, ld_ple, yr, ldy, tail); break;
      case 8: e = launch_gemv_m<Fmt, 8>(mm, grid, block, st, w, w_ld, row_scale, alpha, xr, ldx, n, k, pr, ld_ple, yr, ldy, tail); break;
      default: e = launch_gemv_m<Fmt, 4>(mm, grid, block, st, w, w_ld, row_scale, alpha, xr, ldx, n, k, pr, ld_ple, yr, ldy, tail); break;
    }
  }
  return e;
}

}  // namespace

extern "C" int sb_gemv_q8(const void* codes, const float* row_scale, const float* x, int ldx, float* y, int ldy,
                          int m, int n, int k, const float* ple, int ld_ple, void* stream) {
  SB_CHECK_ARG(m >= 0 && n > 0 && k >= 64 && k % 16 == 0, "sb_gemv_q8: k=%d must be a multiple of 16 and >= 64", k);
  SB_CHECK_ARG(ldx >= k && ldx % 4 == 0 && ldy >= n && (!ple || ld_ple >= n), "sb_gemv_q8: bad leading dimension");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(codes && row_scale && x && y, "sb_gemv_q8: null pointer");
  if (!sb::aligned(codes, 16) || !sb::aligned(x, 16)) return sb::fail(SB_ERR_ALIGN, "sb_gemv_q8: codes and x need 16-byte alignment");
  cudaError_t e = launch_gemv_rows<FmtQ8>(static_cast<const uint8_t*>(codes), k, row_scale, 1.f, x, ldx, m, n, k, ple,
                                          ld_ple, y, ldy, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return sb::cuda_fail(e, "gemv_rows_kernel<q8>");
  return sb::launch_status("gemv_rows_kernel<q8>");
}

extern "C" int sb_gemv_bf16(const void* w, float alpha, const float* x, int ldx, float* y, int ldy, int m, int n,
                            int k, void* stream) {
  SB_CHECK_ARG(m >= 0 && n > 0 && k >= 32 && k % 8 == 0, "sb_gemv_bf16: k=%d must be a multiple of 8 and >= 32", k);
  SB_CHECK_ARG(ldx >= k && ldx % 4 == 0 && ldy >= n, "sb_gemv_bf16: bad leading dimension");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(w && x && y, "sb_gemv_bf16: null pointer");
  if (!sb::aligned(w, 16) || !sb::aligned(x, 16)) return sb::fail(SB_ERR_ALIGN, "sb_gemv_bf16: w and x need 16-byte alignment");
  cudaError_t e = launch_gemv_rows<FmtBF16>(static_cast<const uint8_t*>(w), 2 * static_cast<int64_t>(k), nullptr, alpha,
                                            x, ldx, m, n, k, nullptr, 0, y, ldy, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return sb::cuda_fail(e, "gemv_rows_kernel<bf16>");
  return sb::launch_status("gemv_rows_kernel<bf16>");
}

extern "C" int sb_gemv_f16(const void* w, float alpha, const float* x, int ldx, float* y, int ldy, int m, int n,
                           int k, void* stream) {
  SB_CHECK_ARG(m >= 0 && n > 0 && k >= 32 && k % 8 == 0, "sb_gemv_f16: k=%d must be a multiple of 8 and >= 32", k);
  SB_CHECK_ARG(ldx >= k && ldx % 4 == 0 && ldy >= n, "sb_gemv_f16: bad leading dimension");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(w && x && y, "sb_gemv_f16: null pointer");
  if (!sb::aligned(w, 16) || !sb::aligned(x, 16)) return sb::fail(SB_ERR_ALIGN, "sb_gemv_f16: w and x need 16-byte alignment");
  cudaError_t e = launch_gemv_rows<FmtF16>(static_cast<const uint8_t*>(w), 2 * static_cast<int64_t>(k), nullptr, alpha,
                                           x, ldx, m, n, k, nullptr, 0, y, ldy, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return sb::cuda_fail(e, "gemv_rows_kernel<f16>");
  return sb::launch_status("gemv_rows_kernel<f16>");
}

extern "C" int sb_ple_norm_add(const float* proj, float* hidden, const float* w_post, float layer_scalar,
                               const float* w_next, float* h_out, void* h16_out, int m, int n, float eps,
                               void* stream) {
  SB_CHECK_ARG(m >= 0 && n > 0 && n % 4 == 0 && n <= 4 * kT * kMaxV4,
               "sb_ple_norm_add: n=%d must be a multiple of 4 in 4..%d", n, 4 * kT * kMaxV4);
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(proj && hidden && w_post && (!w_next || h_out || h16_out), "sb_ple_norm_add: null pointer");
  if (!sb::aligned(proj, 16) || !sb::aligned(hidden, 16) || !sb::aligned(w_post, 16) ||
      (w_next && !sb::aligned(w_next, 16)) || (h_out && !sb::aligned(h_out, 16)) ||
      (h16_out && !sb::aligned(h16_out, 8)))
    return sb::fail(SB_ERR_ALIGN, "sb_ple_norm_add: rows need 16-byte alignment");
  cudaError_t e = sb::launch_pdl(ple_norm_add_kernel, dim3(m), dim3(kT), 0, static_cast<cudaStream_t>(stream), proj,
                                 hidden, w_post, layer_scalar, w_next, h_out, static_cast<__half*>(h16_out), n, eps);
  if (e != cudaSuccess) return sb::cuda_fail(e, "ple_norm_add_kernel");
  return sb::launch_status("ple_norm_add_kernel");
}

extern "C" int sb_ple_gather(const int32_t* ids, const void* table, const float* scales, int vocab, int cols,
                             int group, float ple_scale, float* y, int m, void* stream) {
  SB_CHECK_ARG(m >= 0 && vocab > 0 && cols > 0 && cols % 8 == 0 && group > 0 && group % 8 == 0 && cols % group == 0,
               "sb_ple_gather: bad shape (cols %% 8, group %% 8 and cols %% group must be 0)");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(ids && table && scales && y, "sb_ple_gather: null pointer");
  if (!sb::aligned(table, 4) || !sb::aligned(y, 16)) return sb::fail(SB_ERR_ALIGN, "sb_ple_gather: misaligned table or y");
  cudaError_t e = sb::launch_pdl(ple_gather_kernel, dim3(m), dim3(kT), 0, static_cast<cudaStream_t>(stream), ids,
                                 static_cast<const uint8_t*>(table), scales, vocab, cols, group, ple_scale, y);
  if (e != cudaSuccess) return sb::cuda_fail(e, "ple_gather_kernel");
  return sb::launch_status("ple_gather_kernel");
}

extern "C" int sb_ple_combine(const float* ctx, const int32_t* ids, const void* table, const float* scales, int vocab,
                              const float* w_norm, int n_layers, int d, int group, float ple_scale, float eps,
                              float* out, int m, void* stream) {
  SB_CHECK_ARG(m >= 0 && vocab > 0 && n_layers > 0 && d > 0 && d % 256 == 0 && group > 0 && group % 8 == 0 &&
                   (n_layers * d) % group == 0,
               "sb_ple_combine: bad shape (d %% 256, group %% 8 and cols %% group must be 0)");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(ctx && ids && table && scales && w_norm && out, "sb_ple_combine: null pointer");
  if (!sb::aligned(ctx, 16) || !sb::aligned(out, 16) || !sb::aligned(table, 4))
    return sb::fail(SB_ERR_ALIGN, "sb_ple_combine: misaligned ctx, out or table");
  const int slices = m * n_layers, per = kT / 32;
  cudaError_t e = sb::launch_pdl(ple_combine_kernel, dim3((slices + per - 1) / per), dim3(kT), 0,
                                 static_cast<cudaStream_t>(stream), ctx, ids, static_cast<const uint8_t*>(table), scales,
                                 vocab, w_norm, m, n_layers, d, group, ple_scale, eps, out);
  if (e != cudaSuccess) return sb::cuda_fail(e, "ple_combine_kernel");
  return sb::launch_status("ple_combine_kernel");
}

extern "C" int sb_ple_gate_act(const float* pre, int ld_pre, int64_t plane, int nsplit, const float* ple, int ld_ple,
                               void* out16, int ld_out, int m, int n, void* stream) {
  SB_CHECK_ARG(m >= 0 && n > 0 && ld_pre >= n && ld_ple >= n && ld_out >= n && nsplit >= 1 &&
                   (nsplit == 1 || plane >= static_cast<int64_t>(m) * ld_pre),
               "sb_ple_gate_act: bad shape");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(pre && ple && out16, "sb_ple_gate_act: null pointer");
  cudaError_t e = sb::launch_pdl(ple_gate_act_kernel, dim3(grid_for(static_cast<int64_t>(m) * n)), dim3(kT), 0,
                                 static_cast<cudaStream_t>(stream), pre, ld_pre, plane, nsplit, ple, ld_ple,
                                 static_cast<__half*>(out16), ld_out, m, n);
  if (e != cudaSuccess) return sb::cuda_fail(e, "ple_gate_act_kernel");
  return sb::launch_status("ple_gate_act_kernel");
}

extern "C" int sb_cast_f16(const float* x, void* out16, int64_t n, void* stream) {
  SB_CHECK_ARG(n >= 0, "sb_cast_f16: negative size");
  if (n == 0) return SB_OK;
  SB_CHECK_ARG(x && out16, "sb_cast_f16: null pointer");
  cudaError_t e = sb::launch_pdl(cast_f16_kernel, dim3(grid_for(n)), dim3(kT), 0, static_cast<cudaStream_t>(stream), x,
                                 static_cast<__half*>(out16), n);
  if (e != cudaSuccess) return sb::cuda_fail(e, "cast_f16_kernel");
  return sb::launch_status("cast_f16_kernel");
}

extern "C" int sb_ple_proj_norm_add(const void* codes, const float* row_scale, const float* g, int ldg, float* proj,
                                    int m, int n, int k, float* hidden, const float* w_post, float layer_scalar,
                                    const float* w_next, float* h_out, void* h16_out, float eps, unsigned int* counter,
                                    void* stream) {
  SB_CHECK_ARG(m >= 0 && m <= kMaxM, "sb_ple_proj_norm_add: m=%d must be in 0..%d (one launch)", m, kMaxM);
  SB_CHECK_ARG(n > 0 && n % 4 == 0 && n <= 4 * sbd::kTailV4 * kWarps * 32 && k >= 64 && k % 16 == 0 && ldg >= k &&
                   ldg % 4 == 0,
               "sb_ple_proj_norm_add: n=%d must be a multiple of 4 up to %d, k=%d a multiple of 16 and >= 64", n,
               4 * sbd::kTailV4 * kWarps * 32, k);
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(codes && row_scale && g && proj && hidden && w_post && counter && (!w_next || h_out || h16_out),
               "sb_ple_proj_norm_add: null pointer");
  if (!sb::aligned(codes, 16) || !sb::aligned(g, 16) || !sb::aligned(proj, 16) || !sb::aligned(hidden, 16) ||
      !sb::aligned(w_post, 16) || (w_next && !sb::aligned(w_next, 16)) || (h_out && !sb::aligned(h_out, 16)))
    return sb::fail(SB_ERR_ALIGN, "sb_ple_proj_norm_add: operands need 16-byte alignment");
  sbd::NormTail t{hidden, w_post, w_next, h_out, static_cast<__half*>(h16_out), counter, layer_scalar, eps};
  cudaError_t e = launch_gemv_rows<FmtQ8>(static_cast<const uint8_t*>(codes), k, row_scale, 1.f, g, ldg, m, n, k,
                                          nullptr, 0, proj, n, static_cast<cudaStream_t>(stream), t);
  if (e != cudaSuccess) return sb::cuda_fail(e, "gemv_rows_kernel<q8> + PLE tail");
  return sb::launch_status("gemv_rows_kernel<q8> + PLE tail");
}
