// Decode GEMV over packed int4 weights (sb_gemv_q4) and the tied lm_head GEMV
// fused with greedy argmax (sb_lmhead_argmax).
//
// Work split.  A CTA is 16 half-warps.  The K range is cut into `ks` slices
// (1..16, a power of two) and each half-warp owns one slice for a run of R
// rows; lane l of a half-warp owns the groups slice_begin + l + 16*u,
// u < GPL, of every row it visits.  Because a lane's groups never change, its
// slice of x (32 f32 values per group and decode row) is loaded into
// registers once per CTA and reused for every row: the inner loop touches only
// the weight stream.  Each (row, group) is one 16-byte load of 32 nibbles; a
// half-warp reads 256 contiguous bytes per group index, so loads are fully
// coalesced.  Partial sums are reduced with half-warp shuffles and, across
// K slices, through shared memory, in a fixed order (deterministic results).
//
// Exact dequant without an int->float conversion: for a nibble q at bit p of
// a word (p <= 16), the f32 with exponent 150-p and mantissa (q << p) equals
// 2^(23-p) + q, so subtracting 2^(23-p) + 8 gives q - 8 exactly.  One LOP3 and
// one FADD per value; nibbles 5..7 are first shifted down by 12 bits.
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;

enum { EPI_STORE = 0, EPI_ARGMAX = 1 };

struct GemvParams {
  const uint8_t* w;
  const void* scales;
  const void* x;
  float* y;
  unsigned long long* keys;
  float* logits;
  int m, n, k, group, ldy, ks;
  long long row_offset;
};

__device__ __forceinline__ void nibbles8(uint32_t w, float (&v)[8]) {
  const uint32_t t = w >> 12;
  v[0] = __uint_as_float((w & 0x0000000Fu) | 0x4B000000u) - 8388616.0f;
  v[1] = __uint_as_float((w & 0x000000F0u) | 0x49000000u) - 524296.0f;
  v[2] = __uint_as_float((w & 0x00000F00u) | 0x47000000u) - 32776.0f;
  v[3] = __uint_as_float((w & 0x0000F000u) | 0x45000000u) - 2056.0f;
  v[4] = __uint_as_float((w & 0x000F0000u) | 0x43000000u) - 136.0f;
  v[5] = __uint_as_float((t & 0x00000F00u) | 0x47000000u) - 32776.0f;
  v[6] = __uint_as_float((t & 0x0000F000u) | 0x45000000u) - 2056.0f;
  v[7] = __uint_as_float((t & 0x000F0000u) | 0x43000000u) - 136.0f;
}

__device__ __forceinline__ uint32_t orderable(float f) {
  if (f != f) f = -INFINITY;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long make_key(float v, long long idx) {
  return (static_cast<unsigned long long>(orderable(v)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
}

template <int M, int R, int GPL, bool XF32, bool SF16, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_q4_kernel(const GemvParams p) {
  __shared__ float red[16 * R * M];
  __shared__ unsigned long long best_s[kThreads / 32][M];

  const int tid = threadIdx.x;
  const int hw = tid >> 4, l16 = tid & 15;
  const int ks = p.ks;
  const int kslice = hw % ks, rlane = hw / ks, nrl = 16 / ks;
  const int G = p.k >> 5;
  const int SG = (G + ks - 1) / ks;
  const int g_begin = kslice * SG;
  const int g_end = min(G, g_begin + SG);
  const int row_bytes = p.k >> 1;
  const int gps = p.k / p.group;  // scales per row
  const int gshift = __ffs(p.group) - 1;
  const bool pow2_group = (p.group & (p.group - 1)) == 0;

  int gidx[GPL];
  bool gval[GPL];
#pragma unroll
  for (int u = 0; u < GPL; ++u) {
    gidx[u] = g_begin + l16 + 16 * u;
    gval[u] = gidx[u] < g_end;
  }

  // this lane's slice of x, kept in registers for the whole kernel
  float xr[M][GPL][32];
#pragma unroll
  for (int m = 0; m < M; ++m) {
#pragma unroll
    for (int u = 0; u < GPL; ++u) {
      const bool ok = gval[u] && m < p.m;
      if (XF32) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) +
                                                            static_cast<size_t>(m) * p.k + gidx[u] * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = ok ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          xr[m][u][4 * j + 0] = f.x;
          xr[m][u][4 * j + 1] = f.y;
          xr[m][u][4 * j + 2] = f.z;
          xr[m][u][4 * j + 3] = f.w;
        }
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x) +
                                                          static_cast<size_t>(m) * p.k + gidx[u] * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 h = ok ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
          const uint32_t hv[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hv[e]));
            xr[m][u][8 * j + 2 * e] = f.x;
            xr[m][u][8 * j + 2 * e + 1] = f.y;
          }
        }
      }
    }
  }

  float best_v[M];
  long long best_i[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    best_v[m] = -INFINITY;
    best_i[m] = 0x7FFFFFFF;
  }

  const int rows_per_tile = nrl * R;
  const int ntiles = (p.n + rows_per_tile - 1) / rows_per_tile;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int row0 = tile * rows_per_tile + rlane * R;
    uint4 wv[GPL][R];
    float sv[GPL][R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
      const bool rv = row < p.n;
#pragma unroll
      for (int u = 0; u < GPL; ++u) {
        if (rv && gval[u]) {
          wv[u][r] = sbd::ldg_nc_v4(p.w + static_cast<size_t>(row) * row_bytes + gidx[u] * 16);
          const int gi = pow2_group ? ((gidx[u] * 32) >> gshift) : (gidx[u] * 32) / p.group;
          const size_t si = static_cast<size_t>(row) * gps + gi;
          sv[u][r] = SF16 ? __half2float(static_cast<const __half*>(p.scales)[si])
                          : static_cast<const float*>(p.scales)[si];
        } else {
          wv[u][r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // all q-8 == 0
          sv[u][r] = 0.f;
        }
      }
    }

    float acc[M][R];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < R; ++r) acc[m][r] = 0.f;

#pragma unroll
    for (int u = 0; u < GPL; ++u) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t words[4] = {wv[u][r].x, wv[u][r].y, wv[u][r].z, wv[u][r].w};
        float d[M];
#pragma unroll
        for (int m = 0; m < M; ++m) d[m] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v[8];
          nibbles8(words[j], v);
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int m = 0; m < M; ++m) d[m] = fmaf(v[i], xr[m][u][8 * j + i], d[m]);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m][r] = fmaf(sv[u][r], d[m], acc[m][r]);
      }
    }

#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) acc[m][r] += __shfl_xor_sync(0xFFFFFFFFu, acc[m][r], off, 16);
      }

    bool owner = l16 == 0;
    if (ks > 1) {
      if (l16 == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < M; ++m) red[(hw * R + r) * M + m] = acc[m][r];
      }
      __syncthreads();
      owner = owner && kslice == 0;
      if (owner) {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float s = 0.f;
            for (int q = 0; q < ks; ++q) s += red[((rlane * ks + q) * R + r) * M + m];
            acc[m][r] = s;
          }
      }
      __syncthreads();
    }

    if (owner) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (row >= p.n) continue;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          if (m >= p.m) continue;
          if (EPI == EPI_STORE) {
            p.y[static_cast<size_t>(m) * p.ldy + row] = acc[m][r];
          } else {
            float v = acc[m][r];
            if (p.logits) p.logits[static_cast<size_t>(m) * p.n + row] = v;
            if (v != v) v = -INFINITY;
            const long long gi = p.row_offset + row;
            if (v > best_v[m] || (v == best_v[m] && gi < best_i[m])) {
              best_v[m] = v;
              best_i[m] = gi;
            }
          }
        }
      }
    }
  }

  if (EPI == EPI_ARGMAX) {
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      unsigned long long key = best_i[m] == 0x7FFFFFFF ? 0ull : make_key(best_v[m], best_i[m]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
        key = o > key ? o : key;
      }
      if (lane == 0) best_s[warp][m] = key;
    }
    __syncthreads();
    if (tid < M && tid < p.m) {
      unsigned long long key = 0;
      for (int wi = 0; wi < kThreads / 32; ++wi) key = best_s[wi][tid] > key ? best_s[wi][tid] : key;
      if (key) atomicMax(p.keys + tid, key);
    }
  }
}

__global__ void keys_to_tokens_kernel(const unsigned long long* keys, int32_t* tokens, int m) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < m) tokens[i] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(keys[i] & 0xFFFFFFFFull));
}

struct Plan {
  int gpl, ks, r;
};

// Pick groups-per-lane and K slices so 16*GPL*ks covers the G groups of a row
// with the least waste, then rows-per-half-warp R from the row count.
Plan plan(int mtile, int n, int k, int sms) {
  const int G = k / 32;
  const int max_gpl = mtile == 1 ? 4 : (mtile == 2 ? 2 : 1);
  Plan best{1, 16, 1};
  int best_waste = 1 << 30;
  const int prefs[4] = {3, 4, 2, 1};
  for (int pi = 0; pi < 4; ++pi) {
    const int gpl = prefs[pi];
    if (gpl > max_gpl) continue;
    int ks = 1;
    while (16 * gpl * ks < G && ks < 16) ks *= 2;
    if (16 * gpl * ks < G) continue;
    const int waste = 16 * gpl * ks - G;
    if (waste < best_waste) {
      best_waste = waste;
      best = {gpl, ks, 1};
    }
  }
  const int nrl = 16 / best.ks;
  const long long tiles4 = (n + nrl * 4 - 1) / (nrl * 4);
  const long long tiles2 = (n + nrl * 2 - 1) / (nrl * 2);
  best.r = tiles4 >= 2LL * sms ? 4 : (tiles2 >= sms ? 2 : 1);
  if (mtile >= 2 && best.r == 4) best.r = 2;
  return best;
}

template <int M, int R, int GPL, int EPI>
int launch_t(const GemvParams& p, bool xf32, bool sf16, int sms, cudaStream_t s) {
  const int nrl = 16 / p.ks;
  const long long ntiles = (p.n + nrl * R - 1) / (nrl * R);
  const int grid = static_cast<int>(std::min<long long>(ntiles, static_cast<long long>(sms) * 2));
  if (grid == 0) return SB_OK;
  if (xf32) {
    if (sf16) gemv_q4_kernel<M, R, GPL, true, true, EPI><<<grid, kThreads, 0, s>>>(p);
    else gemv_q4_kernel<M, R, GPL, true, false, EPI><<<grid, kThreads, 0, s>>>(p);
  } else {
    if (sf16) gemv_q4_kernel<M, R, GPL, false, true, EPI><<<grid, kThreads, 0, s>>>(p);
    else gemv_q4_kernel<M, R, GPL, false, false, EPI><<<grid, kThreads, 0, s>>>(p);
  }
  return sb::launch_status("gemv_q4_kernel");
}

template <int M, int EPI>
int launch_m(const GemvParams& p, const Plan& pl, bool xf32, bool sf16, int sms, cudaStream_t s) {
  // instantiated combinations: M=1: GPL 1..4 x R {1,2,4}; M=2: GPL {1,2} x R {1,2}; M=4: GPL 1 x R {1,2}
  if constexpr (M == 1) {
#define SB_GPL_R(G_, R_) \
  if (pl.gpl == G_ && pl.r == R_) return launch_t<M, R_, G_, EPI>(p, xf32, sf16, sms, s);
    SB_GPL_R(1, 1) SB_GPL_R(1, 2) SB_GPL_R(1, 4)
    SB_GPL_R(2, 1) SB_GPL_R(2, 2) SB_GPL_R(2, 4)
    SB_GPL_R(3, 1) SB_GPL_R(3, 2) SB_GPL_R(3, 4)
    SB_GPL_R(4, 1) SB_GPL_R(4, 2) SB_GPL_R(4, 4)
  } else if constexpr (M == 2) {
    SB_GPL_R(1, 1) SB_GPL_R(1, 2) SB_GPL_R(2, 1) SB_GPL_R(2, 2)
  } else {
    SB_GPL_R(1, 1) SB_GPL_R(1, 2)
#undef SB_GPL_R
  }
  return sb::fail(SB_ERR_ARG, "gemv: no kernel for M=%d GPL=%d R=%d", M, pl.gpl, pl.r);
}

int run(GemvParams p, int epi, bool xf32, bool sf16, cudaStream_t s) {
  const int sms = sb::num_sms();
  const int x_elt = xf32 ? 4 : 2;
  const size_t x_row = static_cast<size_t>(p.k) * x_elt;
  int done = 0;
  const int m_total = p.m;
  while (done < m_total) {
    const int left = m_total - done;
    const int mt = left >= 4 ? 4 : (left >= 2 ? 2 : 1);
    GemvParams q = p;
    q.m = mt;
    q.x = static_cast<const char*>(p.x) + done * x_row;
    if (epi == EPI_STORE) q.y = p.y + static_cast<size_t>(done) * p.ldy;
    else {
      q.keys = p.keys + done;
      if (p.logits) q.logits = p.logits + static_cast<size_t>(done) * p.n;
    }
    Plan pl = plan(mt, p.n, p.k, sms);
    q.ks = pl.ks;
    int rc;
    if (epi == EPI_STORE) {
      rc = mt == 1 ? launch_m<1, EPI_STORE>(q, pl, xf32, sf16, sms, s)
                   : mt == 2 ? launch_m<2, EPI_STORE>(q, pl, xf32, sf16, sms, s)
                             : launch_m<4, EPI_STORE>(q, pl, xf32, sf16, sms, s);
    } else {
      rc = mt == 1 ? launch_m<1, EPI_ARGMAX>(q, pl, xf32, sf16, sms, s)
                   : mt == 2 ? launch_m<2, EPI_ARGMAX>(q, pl, xf32, sf16, sms, s)
                             : launch_m<4, EPI_ARGMAX>(q, pl, xf32, sf16, sms, s);
    }
    if (rc != SB_OK) return rc;
    done += mt;
  }
  return SB_OK;
}

int check_common(const char* fn, const void* w, const void* scales, int scale_dtype, int group, const void* x,
                 int x_dtype, int m, int n, int k) {
  SB_CHECK_ARG(m >= 1 && m <= 8, "%s: m=%d must be in 1..8", fn, m);
  SB_CHECK_ARG(n >= 0, "%s: negative n", fn);
  SB_CHECK_ARG(k > 0 && k % 32 == 0, "%s: k=%d must be a positive multiple of 32", fn, k);
  SB_CHECK_ARG(group > 0 && k % group == 0 && group % 32 == 0, "%s: group=%d must be a multiple of 32 dividing k",
               fn, group);
  SB_CHECK_ARG(scale_dtype == SB_SCALE_F16 || scale_dtype == SB_SCALE_F32, "%s: bad scale dtype", fn);
  SB_CHECK_ARG(x_dtype == SB_F16 || x_dtype == SB_F32, "%s: bad x dtype", fn);
  SB_CHECK_ARG(n == 0 || (w && scales && x), "%s: null pointer", fn);
  if (!sb::aligned(w, 16) || !sb::aligned(x, 16))
    return sb::fail(SB_ERR_ALIGN, "%s: weights and activations must be 16-byte aligned", fn);
  return SB_OK;
}

}  // namespace

extern "C" int sb_gemv_q4(const void* w, const void* scales, int scale_dtype, int group, const void* x,
                          int x_dtype, float* y, int ldy, int m, int n, int k, void* stream) {
  int rc = check_common("sb_gemv_q4", w, scales, scale_dtype, group, x, x_dtype, m, n, k);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(ldy >= n, "sb_gemv_q4: ldy=%d < n=%d", ldy, n);
  if (n == 0) return SB_OK;
  SB_CHECK_ARG(y != nullptr, "sb_gemv_q4: null y");
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.scales = scales;
  p.x = x;
  p.y = y;
  p.m = m;
  p.n = n;
  p.k = k;
  p.group = group;
  p.ldy = ldy;
  return run(p, EPI_STORE, x_dtype == SB_F32, scale_dtype == SB_SCALE_F16, static_cast<cudaStream_t>(stream));
}

extern "C" int sb_lmhead_argmax(const void* emb, const void* scales, int scale_dtype, int group, const void* h,
                                int h_dtype, int m, int v, int k, int64_t row_offset, uint64_t* keys,
                                int32_t* tokens, float* logits, void* stream) {
  int rc = check_common("sb_lmhead_argmax", emb, scales, scale_dtype, group, h, h_dtype, m, v, k);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(keys != nullptr, "sb_lmhead_argmax: null keys");
  SB_CHECK_ARG(row_offset >= 0 && row_offset + v <= 0xFFFFFFFFLL, "sb_lmhead_argmax: row indices must fit in 32 bits");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(keys, 0, sizeof(uint64_t) * m, s);
  if (e != cudaSuccess) return sb::cuda_fail(e, "sb_lmhead_argmax: clearing keys");
  if (v > 0) {
    GemvParams p{};
    p.w = static_cast<const uint8_t*>(emb);
    p.scales = scales;
    p.x = h;
    p.keys = reinterpret_cast<unsigned long long*>(keys);
    p.logits = logits;
    p.m = m;
    p.n = v;
    p.k = k;
    p.group = group;
    p.row_offset = row_offset;
    rc = run(p, EPI_ARGMAX, h_dtype == SB_F32, scale_dtype == SB_SCALE_F16, s);
    if (rc != SB_OK) return rc;
  }
  if (tokens) {
    keys_to_tokens_kernel<<<1, 32, 0, s>>>(reinterpret_cast<const unsigned long long*>(keys), tokens, m);
    return sb::launch_status("keys_to_tokens_kernel");
  }
  return SB_OK;
}

extern "C" int sb_keys_to_tokens(const uint64_t* keys, int32_t* tokens, int m, void* stream) {
  SB_CHECK_ARG(m >= 0 && m <= 1 << 20, "sb_keys_to_tokens: bad m");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(keys && tokens, "sb_keys_to_tokens: null pointer");
  keys_to_tokens_kernel<<<(m + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const unsigned long long*>(keys), tokens, m);
  return sb::launch_status("keys_to_tokens_kernel");
}
