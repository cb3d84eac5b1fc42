// tcgen05 GEMMs for prefill: sb_gemm_f16 (f16 x f16, both orientations of B)
// and sb_gemm_q4 (A f16 x dequantised int4 W, fused).
//
// One CTA computes a 128 x 256 tile of C (BM tokens x BN output features) on
// one SM with 128x256x16 UMMAs accumulating f32 in 256 TMEM columns.  The K
// loop runs over 64-wide k-blocks (one 128-byte swizzle row of f16):
//
//   warp 0      TMA producer: A tile [128 x 64] f16 (128B swizzle) and, per
//               mode, the B tile [256 x 64] f16 (K-major, tr=1), four
//               [64 k x 64 n] boxes (MN-major, tr=0), or the packed int4 tile
//               [256 rows x 32 bytes] (no swizzle) into a ring of stages.
//   warp 1      TMEM allocation and the single MMA-issuing thread; MMA
//               completion is signalled back with tcgen05.commit.
//   warps 2..9  (int4 mode only) dequant producers: read the packed stage from
//               shared memory, form f16(scale * (q - 8)) with exact f16 math,
//               and store it in the UMMA K-major 128B-swizzled layout of a
//               second ring; fence.proxy.async then an mbarrier arrive hands it
//               to the tensor core.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)...), scale by alpha, round to f16 and store to C (or
//               store f32 partials to the split-K workspace).
//
// Every mbarrier wait is bounded (2 s of %globaltimer): a stuck pipeline
// raises a shared abort flag, writes SB_ERR_TIMEOUT to the device error word,
// drains the copies it issued and returns.  No TMA multicast is used.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int UMMA_K = 16;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int P_BYTES = BN * BK / 2;   // 8 KB packed int4
constexpr int TMEM_COLS = 256;

enum Mode { MODE_F16_KMAJOR = 0, MODE_F16_MNMAJOR = 1, MODE_Q4 = 2 };

template <int MODE>
struct Cfg {
  static constexpr int kLoadStages = 4;
  static constexpr int kDeqStages = MODE == MODE_Q4 ? 3 : 0;
  static constexpr int kDqWarps = MODE == MODE_Q4 ? 8 : 0;
  static constexpr int kWarps = MODE == MODE_Q4 ? 10 : 6;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kLoadBytes = A_BYTES + (MODE == MODE_Q4 ? P_BYTES : B_BYTES);
  // layout: [A stages][B or packed stages][dequant B stages][barriers]
  static constexpr int kOffB = kLoadStages * A_BYTES;
  static constexpr int kOffD = kOffB + kLoadStages * (MODE == MODE_Q4 ? P_BYTES : B_BYTES);
  static constexpr int kOffBar = kOffD + kDeqStages * B_BYTES;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = kOffBar + kBarBytes + 1024;  // + alignment slack
};

struct GemmParams {
  const void* scales;  // int4 mode
  void* c;
  float* ws;           // split-K partials [splits][m][n] or null
  int* err;
  int m, n, k, ldc, group, scale_f16;
  int kb_per_split, kb_total;
  float alpha;
};

struct Bars {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t dfull[4];
  uint64_t dempty[4];
  uint64_t accum;
  uint32_t tmem_slot;
  int abort;
};

__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = sbd::global_ns();
  while (!sbd::mbar_try_wait(bar, parity)) {
    if (sbd::global_ns() - t0 > sbd::kWaitLimitNs) return false;
  }
  return true;
}

// f16(scale * (q - 8)) for the 8 nibbles of `w`, as 4 half2 in k order.
// byte_perm puts byte j of w in byte 0 and byte j of (w >> 4) in byte 2, so the
// low nibbles of the two 16-bit halves hold the pair (q_2j, q_2j+1); OR-ing 0x6400 makes each half the f16 1024 + q, and
// subtracting 1032 gives q - 8 exactly.  The product with an f16 scale is the
// correctly rounded f16 of the exact product, i.e. f16(float(s) * (q - 8)).
__device__ __forceinline__ void dq8_half(uint32_t w, __half2 s2, uint32_t (&out)[4]) {
  const uint32_t t = w >> 4;
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
  const uint32_t sel[4] = {0x0400u, 0x0501u, 0x0602u, 0x0703u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t r = (__byte_perm(w, t, sel[j]) & 0x000F000Fu) | 0x64006400u;
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&r), bias);
    h = __hmul2(h, s2);
    out[j] = *reinterpret_cast<uint32_t*>(&h);
  }
}

__device__ __forceinline__ void dq8_float(uint32_t w, float s, uint32_t (&out)[4]) {
  const uint32_t t = w >> 4;
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  const uint32_t sel[4] = {0x0400u, 0x0501u, 0x0602u, 0x0703u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t r = (__byte_perm(w, t, sel[j]) & 0x000F000Fu) | 0x64006400u;
    const float2 q = __half22float2(__hsub2(*reinterpret_cast<__half2*>(&r), bias));
    __half2 h = __floats2half2_rn(__fmul_rn(s, q.x), __fmul_rn(s, q.y));
    out[j] = *reinterpret_cast<uint32_t*>(&h);
  }
}

template <int MODE>
__global__ void __launch_bounds__(Cfg<MODE>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  using C = Cfg<MODE>;
  constexpr int S = C::kLoadStages;
  constexpr int S2 = C::kDeqStages > 0 ? C::kDeqStages : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int nkb = min(p.kb_per_split, p.kb_total - kb0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      sbd::mbar_init(&bars->full[i], 1);
      sbd::mbar_init(&bars->empty[i], 1 + C::kDqWarps);
    }
    for (int i = 0; i < C::kDeqStages; ++i) {
      sbd::mbar_init(&bars->dfull[i], C::kDqWarps);
      sbd::mbar_init(&bars->dempty[i], 1);
    }
    sbd::mbar_init(&bars->accum, 1);
    bars->abort = 0;
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    sbd::prefetch_tmap(&tmA);
    sbd::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    sbd::tmem_alloc(&bars->tmem_slot, TMEM_COLS);
    sbd::tmem_relinquish();
  }
  sbd::tc_fence_before();
  __syncthreads();
  sbd::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!sbd::mbar_wait(&bars->empty[s], ph ^ 1, abort, p.err)) break;
        sbd::mbar_arrive_expect_tx(&bars->full[s], C::kLoadBytes);
        const int k0 = (kb0 + kb) * BK;
        sbd::tma_load_2d(&tmA, &bars->full[s], smem + s * A_BYTES, k0, m0);
        uint8_t* bdst = smem + C::kOffB + s * (MODE == MODE_Q4 ? P_BYTES : B_BYTES);
        if (MODE == MODE_F16_KMAJOR) {
          sbd::tma_load_2d(&tmB, &bars->full[s], bdst, k0, n0);
        } else if (MODE == MODE_F16_MNMAJOR) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) sbd::tma_load_2d(&tmB, &bars->full[s], bdst + j * 8192, n0 + 64 * j, k0);
        } else {
          sbd::tma_load_2d(&tmB, &bars->full[s], bdst, k0 / 2, n0);
        }
        issued = kb + 1;
      }
      if (*abort) {
        // let copies already in flight land before this CTA's shared memory is released
        for (int kb = max(0, issued - S); kb < issued; ++kb) drain_wait(&bars->full[kb % S], (kb / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sbd::umma_idesc_f16(BM, BN, 0, MODE == MODE_F16_MNMAJOR ? 1 : 0);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        ok = sbd::mbar_wait(&bars->full[s], ph, abort, p.err);
        int t2 = 0;
        if (ok && MODE == MODE_Q4) {
          t2 = kb % S2;
          ok = sbd::mbar_wait(&bars->dfull[t2], (kb / S2) & 1, abort, p.err);
        }
        if (!ok) break;
        sbd::tc_fence_after();
        const uint32_t a_base = sbd::smem_u32(smem + s * A_BYTES);
        uint32_t b_base;
        if (MODE == MODE_Q4) b_base = sbd::smem_u32(smem + C::kOffD + t2 * B_BYTES);
        else b_base = sbd::smem_u32(smem + C::kOffB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          const uint64_t adesc = sbd::umma_desc(a_base + kk * 32, 16, 1024, sbd::kLayoutSwizzle128B);
          uint64_t bdesc;
          if (MODE == MODE_F16_MNMAJOR) bdesc = sbd::umma_desc(b_base + kk * 2048, 8192, 1024, sbd::kLayoutSwizzle128B);
          else bdesc = sbd::umma_desc(b_base + kk * 32, 16, 1024, sbd::kLayoutSwizzle128B);
          sbd::umma_f16(tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        sbd::umma_commit(&bars->empty[s]);
        if (MODE == MODE_Q4) sbd::umma_commit(&bars->dempty[t2]);
      }
      sbd::umma_commit(&bars->accum);  // fires once every MMA above has completed
    }
  } else {
    // ------------------------------------------------------------ dequant producers
    if (MODE == MODE_Q4) {
      const int dt = threadIdx.x - 64;  // 0..255
      const int gps = p.k / p.group;
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % S;
        const int t2 = kb % S2;
        // scales for this thread's two 32-value chunks (issued before the waits)
        float sc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = dt + 256 * h;
          const int row = n0 + (c >> 1);
          const int kv = (kb0 + kb) * BK + (c & 1) * 32;
          float v = 0.f;
          if (row < p.n && kv < p.k) {
            const size_t si = static_cast<size_t>(row) * gps + kv / p.group;
            v = p.scale_f16 ? __half2float(static_cast<const __half*>(p.scales)[si])
                            : static_cast<const float*>(p.scales)[si];
          }
          sc[h] = v;
        }
        ok = sbd::mbar_wait(&bars->full[s], (kb / S) & 1, abort, p.err);
        if (ok) ok = sbd::mbar_wait(&bars->dempty[t2], ((kb / S2) & 1) ^ 1, abort, p.err);
        if (!ok) break;
        const uint8_t* pk = smem + C::kOffB + s * P_BYTES;
        uint8_t* bt = smem + C::kOffD + t2 * B_BYTES;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = dt + 256 * h;
          const int row = c >> 1, half = c & 1;
          const uint4 q = *reinterpret_cast<const uint4*>(pk + c * 16);
          const uint32_t words[4] = {q.x, q.y, q.z, q.w};
          const __half2 s2 = __float2half2_rn(sc[h]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t o[4];
            if (p.scale_f16) dq8_half(words[j], s2, o);
            else dq8_float(words[j], sc[h], o);
            const int chunk = (half * 4 + j) ^ (row & 7);
            *reinterpret_cast<uint4*>(bt + row * 128 + chunk * 16) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        sbd::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          sbd::mbar_arrive(&bars->dfull[t2]);
          sbd::mbar_arrive(&bars->empty[s]);
        }
      }
    }
    // ------------------------------------------------------------ epilogue
    if (warp >= 2 && warp < 6) {
      // tcgen05.ld is warp-collective: agree on the outcome of the wait first
      const bool ok = __all_sync(0xFFFFFFFFu, sbd::mbar_wait(&bars->accum, 0, abort, p.err));
      if (ok) {
        sbd::tc_fence_after();
        const int quad = warp & 3;
        const int row = m0 + quad * 32 + lane;
        const bool row_ok = row < p.m;
        for (int cc = 0; cc < BN / 32; ++cc) {
          const int col0 = n0 + cc * 32;
          if (col0 >= p.n) break;  // warp-uniform
          uint32_t r[32];
          sbd::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + cc * 32, r);
          sbd::tmem_wait_ld();
          if (!row_ok) continue;
          if (p.ws) {
            float* dst = p.ws + (static_cast<size_t>(blockIdx.z) * p.m + row) * p.n + col0;
            if (col0 + 32 <= p.n && (p.n % 4) == 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                  __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.n) dst[j] = __uint_as_float(r[j]);
            }
          } else {
            __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(row) * p.ldc + col0;
            if (col0 + 32 <= p.n && (p.ldc % 8) == 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  __half2 h = __floats2half2_rn(p.alpha * __uint_as_float(r[j + 2 * e]),
                                                p.alpha * __uint_as_float(r[j + 2 * e + 1]));
                  o[e] = *reinterpret_cast<uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(o[0], o[1], o[2], o[3]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.n) dst[j] = __float2half_rn(p.alpha * __uint_as_float(r[j]));
            }
          }
        }
      }
    }
  }

  sbd::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc(tmem, TMEM_COLS);
  }
}

__global__ void splitk_finalize_kernel(const float* __restrict__ ws, __half* __restrict__ c, int m, int n, int ldc,
                                       int splits, float alpha) {
  const size_t total = static_cast<size_t>(m) * n;
  const size_t plane = total;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int z = 0; z < splits; ++z) s += ws[z * plane + i];
    const size_t row = i / n, col = i - row * n;
    c[row * ldc + col] = __float2half_rn(alpha * s);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dt, int elt, const void* base, uint64_t inner, uint64_t outer,
             uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return sb::fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * elt};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return sb::fail(SB_ERR_ARG, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return SB_OK;
}

template <int MODE>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int splits, cudaStream_t s) {
  using C = Cfg<MODE>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return sb::cuda_fail(e, "gemm_tc_kernel: smem attribute");
    attr_set[dev] = true;
  }
  dim3 grid((p.n + BN - 1) / BN, (p.m + BM - 1) / BM, splits);
  gemm_tc_kernel<MODE><<<grid, C::kThreads, C::kSmem, s>>>(ta, tb, p);
  return sb::launch_status("gemm_tc_kernel");
}

int choose_splits(int m, int n, int k) {
  const int tiles = ((n + BN - 1) / BN) * ((m + BM - 1) / BM);
  const int kb = (k + BK - 1) / BK;
  const int sms = sb::num_sms();
  if (tiles * 4 >= sms * 3) return 1;
  int splits = std::max(1, sms / tiles);
  splits = std::min(splits, std::max(1, kb / 4));
  splits = std::min(splits, 16);
  return splits;
}

int finalize(const GemmParams& p, int splits, cudaStream_t s) {
  const size_t total = static_cast<size_t>(p.m) * p.n;
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, 148 * 16));
  splitk_finalize_kernel<<<grid, 256, 0, s>>>(p.ws, static_cast<__half*>(p.c), p.m, p.n, p.ldc, splits, p.alpha);
  return sb::launch_status("splitk_finalize_kernel");
}

}  // namespace

extern "C" size_t sb_gemm_q4_workspace_size(int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const int splits = choose_splits(m, n, k);
  return splits > 1 ? static_cast<size_t>(splits) * m * n * sizeof(float) : 0;
}

extern "C" int sb_gemm_f16(const void* a, const void* b, void* c, int m, int n, int k, float alpha, int tr, int lda,
                           int ldb, int ldc, void* stream) {
  SB_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "sb_gemm_f16: negative shape");
  if (m == 0 || n == 0) return SB_OK;
  SB_CHECK_ARG(a && b && c, "sb_gemm_f16: null pointer");
  SB_CHECK_ARG(lda >= k && ldc >= n && ldb >= (tr ? k : n), "sb_gemm_f16: leading dimension too small");
  if (!sb::aligned(a, 16) || !sb::aligned(b, 16) || !sb::aligned(c, 2) || lda % 8 || ldb % 8)
    return sb::fail(SB_ERR_ALIGN, "sb_gemm_f16: A and B must be 16-byte aligned with lda, ldb multiples of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k == 0) {
    // C = 0 (an empty sum)
    for (int r = 0; r < m; ++r) {
      cudaError_t e = cudaMemsetAsync(static_cast<__half*>(c) + static_cast<size_t>(r) * ldc, 0, n * 2, s);
      if (e != cudaSuccess) return sb::cuda_fail(e, "sb_gemm_f16: zero fill");
    }
    return SB_OK;
  }
  CUtensorMap ta, tb;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, k, m, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (tr) rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, k, n, ldb, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  else rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, n, k, ldb, 64, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  GemmParams p{};
  p.c = c;
  p.err = sb::device_error_word();
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldc = ldc;
  p.alpha = alpha;
  p.kb_total = (k + BK - 1) / BK;
  p.kb_per_split = p.kb_total;
  return tr ? launch<MODE_F16_KMAJOR>(ta, tb, p, 1, s) : launch<MODE_F16_MNMAJOR>(ta, tb, p, 1, s);
}

extern "C" int sb_gemm_q4(const void* a, const void* w, const void* scales, int scale_dtype, int group, void* c, int m,
                          int n, int k, float alpha, int lda, int ldc, void* workspace, size_t workspace_bytes,
                          void* stream) {
  SB_CHECK_ARG(m >= 0 && n >= 0 && k > 0, "sb_gemm_q4: bad shape");
  SB_CHECK_ARG(k % 64 == 0, "sb_gemm_q4: k=%d must be a multiple of 64", k);
  SB_CHECK_ARG(group > 0 && k % group == 0 && group % 32 == 0, "sb_gemm_q4: group=%d must be a multiple of 32 dividing k",
               group);
  SB_CHECK_ARG(scale_dtype == SB_SCALE_F16 || scale_dtype == SB_SCALE_F32, "sb_gemm_q4: bad scale dtype");
  if (m == 0 || n == 0) return SB_OK;
  SB_CHECK_ARG(a && w && scales && c, "sb_gemm_q4: null pointer");
  SB_CHECK_ARG(lda >= k && ldc >= n, "sb_gemm_q4: leading dimension too small");
  if (!sb::aligned(a, 16) || !sb::aligned(w, 16) || !sb::aligned(c, 2) || lda % 8)
    return sb::fail(SB_ERR_ALIGN, "sb_gemm_q4: A and W must be 16-byte aligned with lda a multiple of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ta, tb;
  int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, k, m, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, k / 2, n, k / 2, BK / 2, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  GemmParams p{};
  p.scales = scales;
  p.c = c;
  p.err = sb::device_error_word();
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldc = ldc;
  p.group = group;
  p.scale_f16 = scale_dtype == SB_SCALE_F16;
  p.alpha = alpha;
  p.kb_total = k / BK;
  int splits = choose_splits(m, n, k);
  const size_t need = splits > 1 ? static_cast<size_t>(splits) * m * n * sizeof(float) : 0;
  if (splits > 1 && (!workspace || workspace_bytes < need)) splits = 1;
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  if (splits > 1) p.ws = static_cast<float*>(workspace);
  rc = launch<MODE_Q4>(ta, tb, p, splits, s);
  if (rc != SB_OK || splits == 1) return rc;
  return finalize(p, splits, s);
}

// ------------------------------------------------------------------------
// Allocation-free variant of sb_gemm_q4.
//
// Some callers cannot allocate device memory on the path that calls us: a host
// that reaches the GPU only through this C ABI (an FFI binding with no CUDA
// allocator of its own), or a process whose device memory is reserved up front
// by its own pool, where a cudaMalloc in the hot path fails or stalls.  For them
// the split-K partial sums live in the array below, which every GPU that loads
// this library holds until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
static __device__ __align__(256) float g_noalloc_splitk[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_noalloc_splitk on the current device.  The host-side
// symbol is only a stand-in: a kernel must be given this address instead.
// Looked up once per device, with that device current, on its first call.
int noalloc_scratch(float** out) {
  static float* addr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sb::cuda_fail(e, "sb_gemm_q4_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return sb::fail(SB_ERR_ARG, "sb_gemm_q4_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_splitk);
    if (e != cudaSuccess) return sb::cuda_fail(e, "sb_gemm_q4_noalloc: cudaGetSymbolAddress");
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return SB_OK;
}

}  // namespace

extern "C" int sb_gemm_q4_noalloc(const void* a, const void* w, const void* scales, int scale_dtype, int group,
                                  void* c, int m, int n, int k, float alpha, int lda, int ldc, void* stream) {
  const size_t need = sb_gemm_q4_workspace_size(m, n, k);
  if (need > kNoAllocScratchBytes)
    return sb::fail(SB_ERR_WORKSPACE,
                    "sb_gemm_q4_noalloc: m=%d n=%d k=%d needs %zu bytes of split-K scratch, more than the "
                    "%zu-byte static scratch; use sb_gemm_q4 with a caller workspace",
                    m, n, k, need, kNoAllocScratchBytes);
  float* ws = nullptr;
  if (need > 0) {
    int rc = noalloc_scratch(&ws);
    if (rc != SB_OK) return rc;
  }
  // Each split writes every element of its partial plane before the finalize
  // kernel reads it, so nothing in the scratch has to start at zero.
  return sb_gemm_q4(a, w, scales, scale_dtype, group, c, m, n, k, alpha, lda, ldc, ws, need > 0 ? kNoAllocScratchBytes : 0,
                    stream);
}
