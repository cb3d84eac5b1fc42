// tcgen05 GEMMs for prefill: sb_gemm_f16 (f16 x f16, both orientations of B)
// and sb_gemm_q4 (A f16 x dequantised int4 W, fused).
//
// f16 kernel (gemm_tc_kernel): one CTA computes a 128 x 256 tile of C with
// 128x256x16 UMMAs (A and B from shared memory) accumulating f32 in 256 TMEM
// columns over 64-wide k-blocks:
//   warp 0      TMA producer: A tile [128 x 64] f16 (128B swizzle) and the B
//               tile [256 x 64] (K-major, tr=1) or four [64 k x 64 n] boxes
//               (MN-major, tr=0) into a ring of stages.
//   warp 1      TMEM allocation and the single MMA-issuing thread; completion
//               is signalled back with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)...), alpha, f16 rounding, stores.
//
// int4 kernel (gemm_q4_kernel): the WEIGHT is the MMA's A operand and lives in
// tensor memory.  A CTA owns 128 weight rows x 256 tokens; per k-block:
//   warp 0      TMA: activation tile [256 tokens x 64] f16 (128B swizzle, the
//               MMA's B operand) and the packed tile [128 rows x 32 bytes].
//   warps 2..17 dequant, in two groups of 8 that take alternate k-blocks (a
//               k-block's dequant chain -- waits, scale and nibble reads,
//               unpack, tcgen05.st, hand-off -- is longer than its MMAs, so
//               two run at once): thread = one weight row (TMEM lane) and
//               one 32-value group; f16(scale * (q - 8)) with exact f16 math,
//               written with tcgen05.st into a 4-stage ring of 32-column A
//               slots in TMEM.  The tile's group scales are loaded into shared
//               memory once, transposed to [group][row] so that a warp's 32
//               rows read 32 consecutive scales.
//   warp 1      tcgen05.mma.cta_group::1.kind::f16 with A from TMEM (M=128
//               weight rows, N=256 tokens, K=16), accumulating D^T in 256
//               TMEM columns.
//   warps 2..17 epilogue: lane = output feature, column = token, so a warp's
//               stores to C[token][feature] are contiguous.
// Putting the dequantised weight in TMEM keeps it out of shared memory (no
// 32 KB store + reload per k-block) and halves the dequant work per FLOP
// compared with dequantising a 256-row B tile.
//
// Every mbarrier wait is bounded (2 s of %globaltimer): a stuck pipeline
// raises a shared abort flag, writes SB_ERR_TIMEOUT to the device error word,
// drains the copies it issued and returns.  No TMA multicast is used.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tmap.cuh"

namespace {

// ---- f16 kernel tile: BM rows of A x BN rows of B (columns of C)
constexpr int BM = 128, BN = 256, BK = 64;
constexpr int UMMA_K = 16;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int TMEM_COLS = 256;

// ---- int4 kernel tile: QW weight rows (MMA M, TMEM lanes) x QT tokens (MMA N)
constexpr int QW = 128, QT = 256;
constexpr int Q_ACT_BYTES = QT * BK * 2;     // 32 KB activation stage
constexpr int Q_PACK_BYTES = QW * BK / 2;    // 4 KB packed stage
constexpr int Q_STAGES = 4;                  // shared-memory load stages
constexpr int Q_ASLOTS = 4;                  // TMEM A slots, 32 columns (64 k) each
constexpr int Q_SCALE_BYTES = 48 * 1024;     // the tile's group scales
constexpr int Q_DQ_GROUPS = 2;               // dequant warp groups, taking alternate k-blocks
constexpr int Q_DQ_WARPS = 8 * Q_DQ_GROUPS;  // a group: 4 TMEM lane quadrants x 2 k halves
constexpr int Q_WARPS = 2 + Q_DQ_WARPS;      // TMA, MMA, dequant/epilogue
constexpr int Q_TMEM_COLS = 512;             // 256 accumulator + 4 x 32 A slots
constexpr int Q_OFF_PACK = Q_STAGES * Q_ACT_BYTES;
constexpr int Q_OFF_SCALE = Q_OFF_PACK + Q_STAGES * Q_PACK_BYTES;
constexpr int Q_OFF_BAR = Q_OFF_SCALE + Q_SCALE_BYTES;
constexpr int Q_SMEM = Q_OFF_BAR + 256 + 1024;

enum Mode { MODE_F16_KMAJOR = 0, MODE_F16_MNMAJOR = 1 };

template <int MODE>
struct Cfg {
  static constexpr int kStages = 4;
  static constexpr int kWarps = 6;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kLoadBytes = A_BYTES + B_BYTES;
  static constexpr int kOffB = kStages * A_BYTES;
  static constexpr int kOffBar = kOffB + kStages * B_BYTES;
  static constexpr int kSmem = kOffBar + 256 + 1024;  // + alignment slack
};

struct GemmParams {
  const void* scales;  // int4 mode
  void* c;
  int c_f32;           // f16 kernel: C is f32 (alpha applied, no rounding to f16)
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
// low nibbles of the two 16-bit halves hold the pair (q_2j, q_2j+1); OR-ing
// 0x6400 makes each half the f16 1024 + q, and subtracting 1032 gives q - 8
// exactly.  The product with an f16 scale is the correctly rounded f16 of the
// exact product, i.e. f16(float(s) * (q - 8)), the reference's dq_f16 value.
__device__ __forceinline__ void dq8_half(uint32_t w, __half2 s2, uint32_t* out) {
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

// Same with an f32 scale: the product is formed in f32 and rounded once.
__device__ __forceinline__ void dq8_float(uint32_t w, float s, uint32_t* out) {
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

// =====================================================================
// f16 x f16 kernel (A and B from shared memory)
// =====================================================================
template <int MODE>
__global__ void __launch_bounds__(Cfg<MODE>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  using C = Cfg<MODE>;
  constexpr int S = C::kStages;
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
      sbd::mbar_init(&bars->empty[i], 1);
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
        uint8_t* bdst = smem + C::kOffB + s * B_BYTES;
        if (MODE == MODE_F16_KMAJOR) {
          sbd::tma_load_2d(&tmB, &bars->full[s], bdst, k0, n0);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) sbd::tma_load_2d(&tmB, &bars->full[s], bdst + j * 8192, n0 + 64 * j, k0);
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
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        if (!sbd::mbar_wait(&bars->full[s], (kb / S) & 1, abort, p.err)) break;
        sbd::tc_fence_after();
        const uint32_t a_base = sbd::smem_u32(smem + s * A_BYTES);
        const uint32_t b_base = sbd::smem_u32(smem + C::kOffB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          const uint64_t adesc = sbd::umma_desc(a_base + kk * 32, 16, 1024, sbd::kLayoutSwizzle128B);
          uint64_t bdesc;
          if (MODE == MODE_F16_MNMAJOR) bdesc = sbd::umma_desc(b_base + kk * 2048, 8192, 1024, sbd::kLayoutSwizzle128B);
          else bdesc = sbd::umma_desc(b_base + kk * 32, 16, 1024, sbd::kLayoutSwizzle128B);
          sbd::umma_f16(tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        sbd::umma_commit(&bars->empty[s]);
      }
      sbd::umma_commit(&bars->accum);  // fires once every MMA above has completed
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
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
        if (p.c_f32) {
          float* dst = static_cast<float*>(p.c) + static_cast<size_t>(row) * p.ldc + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.n) dst[j] = p.alpha * __uint_as_float(r[j]);
          continue;
        }
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

  sbd::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// =====================================================================
// int4 kernel: dequantised weight as the A operand in tensor memory
// =====================================================================
// p.m = tokens (MMA N side), p.n = weight rows (MMA M side).
__global__ void __launch_bounds__(Q_WARPS * 32, 1)
    gemm_q4_kernel(const __grid_constant__ CUtensorMap tmAct, const __grid_constant__ CUtensorMap tmW,
                   const GemmParams p) {
  constexpr int S = Q_STAGES, T = Q_ASLOTS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + Q_OFF_BAR);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w0 = blockIdx.x * QW;  // first weight row
  const int t0 = blockIdx.y * QT;  // first token
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int nkb = min(p.kb_per_split, p.kb_total - kb0);
  // group scales of this split's K range: [g_lo, g_hi)
  const int g_lo = (kb0 * BK) / p.group;
  const int g_hi = ((kb0 + nkb) * BK + p.group - 1) / p.group;
  const int gs = g_hi - g_lo;
  const int gps = p.k / p.group;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      sbd::mbar_init(&bars->full[i], 1);
      sbd::mbar_init(&bars->empty[i], 1 + 8);
    }
    for (int i = 0; i < T; ++i) {
      sbd::mbar_init(&bars->dfull[i], 8);
      sbd::mbar_init(&bars->dempty[i], 1);
    }
    sbd::mbar_init(&bars->accum, 1);
    bars->abort = 0;
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    sbd::prefetch_tmap(&tmAct);
    sbd::prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    sbd::tmem_alloc(&bars->tmem_slot, Q_TMEM_COLS);
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
        if (!sbd::mbar_wait(&bars->empty[s], ((kb / S) & 1) ^ 1, abort, p.err)) break;
        sbd::mbar_arrive_expect_tx(&bars->full[s], Q_ACT_BYTES + Q_PACK_BYTES);
        const int k0 = (kb0 + kb) * BK;
        sbd::tma_load_2d(&tmAct, &bars->full[s], smem + s * Q_ACT_BYTES, k0, t0);
        sbd::tma_load_2d(&tmW, &bars->full[s], smem + Q_OFF_PACK + s * Q_PACK_BYTES, k0 / 2, w0);
        issued = kb + 1;
      }
      if (*abort) {
        for (int kb = max(0, issued - S); kb < issued; ++kb) drain_wait(&bars->full[kb % S], (kb / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sbd::umma_idesc_f16(QW, QT, 0, 0);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S, slot = kb % T;
        if (!sbd::mbar_wait(&bars->full[s], (kb / S) & 1, abort, p.err)) break;
        if (!sbd::mbar_wait(&bars->dfull[slot], (kb / T) & 1, abort, p.err)) break;
        sbd::tc_fence_after();
        const uint32_t b_base = sbd::smem_u32(smem + s * Q_ACT_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          const uint32_t a_tmem = tmem + 256 + slot * 32 + kk * 8;
          const uint64_t bdesc = sbd::umma_desc(b_base + kk * 32, 16, 1024, sbd::kLayoutSwizzle128B);
          sbd::umma_f16_ts(tmem, a_tmem, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        sbd::umma_commit(&bars->empty[s]);
        sbd::umma_commit(&bars->dempty[slot]);
      }
      sbd::umma_commit(&bars->accum);
    }
  } else {
    // ------------------------------------------------------------ dequant producers (warps 2..17)
    const int dw = warp - 2;             // 0..15
    const int grp = dw >> 3;             // k-blocks kb with kb % Q_DQ_GROUPS == grp
    const int quad = warp & 3;           // TMEM lane quadrant this warp may access
    const int khalf = (dw & 7) >> 2;     // which 32-value group of the k-block
    const int r = quad * 32 + lane;      // weight row within the tile
    const int dt = threadIdx.x - 64;     // 0..511
    // the tile's scales -> shared memory [group][row], in their storage type
    const int esz = p.scale_f16 ? 2 : 4;
    uint8_t* sct = smem + Q_OFF_SCALE;
    const int rb = gs * esz;             // bytes of one row's scales in this split
    const uint8_t* sg = static_cast<const uint8_t*>(p.scales);
    const bool vec = (reinterpret_cast<uintptr_t>(sg) % 16 == 0) && (gps * esz) % 16 == 0 && (g_lo * esz) % 16 == 0 &&
                     rb % 16 == 0;
    if (vec) {
      // 16-byte chunks, all loads of a thread in flight together; chunk c is
      // row c % QW, bytes [16 (c / QW), +16) of that row's span
      constexpr int kMaxChunks = Q_SCALE_BYTES / 16 / (Q_DQ_WARPS * 32);
      const int chunks = QW * (rb / 16);
      uint4 v[kMaxChunks];
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = dt + i * Q_DQ_WARPS * 32;
        const int rr = c % QW, cb = c / QW;
        v[i] = make_uint4(0u, 0u, 0u, 0u);
        if (c < chunks && w0 + rr < p.n)
          v[i] = __ldg(reinterpret_cast<const uint4*>(sg + (static_cast<size_t>(w0 + rr) * gps + g_lo) * esz) + cb);
      }
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = dt + i * Q_DQ_WARPS * 32;
        if (c >= chunks) break;
        const int rr = c % QW, g0 = (c / QW) * (16 / esz);
        const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        if (esz == 2) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            reinterpret_cast<uint16_t*>(sct)[(g0 + e) * QW + rr] = static_cast<uint16_t>(wv[e >> 1] >> (16 * (e & 1)));
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) reinterpret_cast<uint32_t*>(sct)[(g0 + e) * QW + rr] = wv[e];
        }
      }
    } else {
      for (int i = dt; i < QW * gs; i += Q_DQ_WARPS * 32) {
        const int g = i / QW, rr = i - g * QW;
        const int row = w0 + rr;
        const size_t si = static_cast<size_t>(row) * gps + g_lo + g;
        if (esz == 2) {
          reinterpret_cast<__half*>(sct)[i] = row < p.n ? static_cast<const __half*>(p.scales)[si] : __float2half(0.f);
        } else {
          reinterpret_cast<float*>(sct)[i] = row < p.n ? static_cast<const float*>(p.scales)[si] : 0.f;
        }
      }
    }
    sbd::named_bar_sync(1, Q_DQ_WARPS * 32);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    // scale group of this thread's 32 values, advanced per k-block step when
    // the group size divides the step (the usual case), else recomputed
    const int kstep = Q_DQ_GROUPS * BK;
    const int gstep = kstep % p.group == 0 ? kstep / p.group : 0;
    int gi = ((kb0 + grp) * BK + khalf * 32) / p.group - g_lo;
    for (int kb = grp; kb < nkb; kb += Q_DQ_GROUPS) {
      const int s = kb % S, slot = kb % T;
      if (gstep == 0) gi = ((kb0 + kb) * BK + khalf * 32) / p.group - g_lo;
      bool ok = sbd::mbar_wait(&bars->full[s], (kb / S) & 1, abort, p.err);
      if (ok) ok = sbd::mbar_wait(&bars->dempty[slot], ((kb / T) & 1) ^ 1, abort, p.err);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      sbd::tc_fence_after();
      const uint4 q = *reinterpret_cast<const uint4*>(smem + Q_OFF_PACK + s * Q_PACK_BYTES + r * 32 + khalf * 16);
      const uint32_t words[4] = {q.x, q.y, q.z, q.w};
      uint32_t o[16];
      if (p.scale_f16) {
        const __half2 s2 = __half2half2(reinterpret_cast<const __half*>(sct)[gi * QW + r]);
#pragma unroll
        for (int j = 0; j < 4; ++j) dq8_half(words[j], s2, o + 4 * j);
      } else {
        const float sf = reinterpret_cast<const float*>(sct)[gi * QW + r];
#pragma unroll
        for (int j = 0; j < 4; ++j) dq8_float(words[j], sf, o + 4 * j);
      }
      sbd::tmem_st_32x32b_x16(lane_addr + 256 + slot * 32 + khalf * 16, o);
      sbd::tmem_wait_st();
      sbd::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        sbd::mbar_arrive(&bars->dfull[slot]);
        sbd::mbar_arrive(&bars->empty[s]);
      }
      gi += gstep;
    }
    // ------------------------------------------------------------ epilogue
    // D^T: TMEM lane = weight row (output feature), column = token; warp dw
    // drains tokens [64 (dw / 4), +64) of its lane quadrant.
    const bool ok = __all_sync(0xFFFFFFFFu, sbd::mbar_wait(&bars->accum, 0, abort, p.err));
    if (ok) {
      sbd::tc_fence_after();
      const int feat = w0 + r;
      const bool feat_ok = feat < p.n;
      for (int cc = 0; cc < 2; ++cc) {
        const int col = (dw >> 2) * 64 + cc * 32;  // token offset within the tile
        if (t0 + col >= p.m) break;                 // warp-uniform
        uint32_t v[32];
        sbd::tmem_ld_32x32b_x32(lane_addr + col, v);
        sbd::tmem_wait_ld();
        if (!feat_ok) continue;
        if (p.ws) {
          float* dst = p.ws + (static_cast<size_t>(blockIdx.z) * p.m + t0 + col) * p.n + feat;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (t0 + col + j < p.m) dst[static_cast<size_t>(j) * p.n] = __uint_as_float(v[j]);
        } else {
          __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(t0 + col) * p.ldc + feat;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (t0 + col + j < p.m) dst[static_cast<size_t>(j) * p.ldc] = __float2half_rn(p.alpha * __uint_as_float(v[j]));
        }
      }
    }
  }

  sbd::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc(tmem, Q_TMEM_COLS);
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
using sb::make_map;

template <typename K>
int set_smem(K kernel, int bytes, bool (&done)[64]) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return sb::cuda_fail(e, "gemm: shared-memory attribute");
    done[dev] = true;
  }
  return SB_OK;
}

template <int MODE>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t s) {
  using C = Cfg<MODE>;
  static bool done[64] = {false};
  int rc = set_smem(gemm_tc_kernel<MODE>, C::kSmem, done);
  if (rc) return rc;
  dim3 grid((p.n + BN - 1) / BN, (p.m + BM - 1) / BM, 1);
  gemm_tc_kernel<MODE><<<grid, C::kThreads, C::kSmem, s>>>(ta, tb, p);
  return sb::launch_status("gemm_tc_kernel");
}

// Scale groups one split of `kbs` k-blocks can touch per row: groups of 32 or 64
// tile a k-block exactly; larger groups may straddle the split's first k-block.
int q4_scale_groups(int kbs, int group) {
  return group <= BK ? kbs * (BK / group) : (kbs * BK + group - 1) / group + 1;
}

// Split-K for the int4 kernel: enough CTAs to fill the SMs when the tile count
// is small, and enough splits that a split's group scales fit in shared memory.
int q4_splits(int m, int n, int k, int group, int scale_bytes) {
  const int tiles = ((n + QW - 1) / QW) * ((m + QT - 1) / QT);
  const int kb = k / BK;
  const int sms = sb::num_sms();
  int splits = 1;
  if (tiles * 4 < sms * 3) {
    splits = std::max(1, sms / tiles);
    splits = std::min(splits, std::max(1, kb / 4));
    splits = std::min(splits, 16);
  }
  while (splits < kb && QW * q4_scale_groups((kb + splits - 1) / splits, group) * scale_bytes > Q_SCALE_BYTES)
    ++splits;
  return splits;
}

int finalize(const GemmParams& p, int splits, cudaStream_t s) {
  const size_t total = static_cast<size_t>(p.m) * p.n;
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, 148 * 16));
  splitk_finalize_kernel<<<grid, 256, 0, s>>>(p.ws, static_cast<__half*>(p.c), p.m, p.n, p.ldc, splits, p.alpha);
  return sb::launch_status("splitk_finalize_kernel");
}

}  // namespace

static size_t q4_workspace(int m, int n, int k, int group, int scale_bytes) {
  if (m <= 0 || n <= 0 || k <= 0 || k % BK || group <= 0) return 0;
  const int splits = q4_splits(m, n, k, group, scale_bytes);
  return splits > 1 ? static_cast<size_t>(splits) * m * n * sizeof(float) : 0;
}

extern "C" size_t sb_gemm_q4_workspace_size(int m, int n, int k) {
  // for the group-32 f16 scales of the benchmark format
  return q4_workspace(m, n, k, 32, 2);
}

static int gemm_f16_impl(const void* a, const void* b, void* c, int c_f32, int m, int n, int k, float alpha, int tr,
                         int lda, int ldb, int ldc, void* stream) {
  SB_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "sb_gemm_f16: negative shape");
  if (m == 0 || n == 0) return SB_OK;
  SB_CHECK_ARG(a && b && c, "sb_gemm_f16: null pointer");
  SB_CHECK_ARG(lda >= k && ldc >= n && ldb >= (tr ? k : n), "sb_gemm_f16: leading dimension too small");
  if (!sb::aligned(a, 16) || !sb::aligned(b, 16) || !sb::aligned(c, 2) || lda % 8 || ldb % 8)
    return sb::fail(SB_ERR_ALIGN, "sb_gemm_f16: A and B must be 16-byte aligned with lda, ldb multiples of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k == 0) {
    // C = 0 (an empty sum)
    const size_t esz = c_f32 ? 4 : 2;
    for (int r = 0; r < m; ++r) {
      cudaError_t e = cudaMemsetAsync(static_cast<char*>(c) + static_cast<size_t>(r) * ldc * esz, 0, n * esz, s);
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
  p.c_f32 = c_f32;
  p.err = sb::device_error_word();
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldc = ldc;
  p.alpha = alpha;
  p.kb_total = (k + BK - 1) / BK;
  p.kb_per_split = p.kb_total;
  return tr ? launch<MODE_F16_KMAJOR>(ta, tb, p, s) : launch<MODE_F16_MNMAJOR>(ta, tb, p, s);
}

extern "C" int sb_gemm_f16(const void* a, const void* b, void* c, int m, int n, int k, float alpha, int tr, int lda,
                           int ldb, int ldc, void* stream) {
  return gemm_f16_impl(a, b, c, 0, m, n, k, alpha, tr, lda, ldb, ldc, stream);
}

extern "C" int sb_gemm_f16_f32out(const void* a, const void* b, float* c, int m, int n, int k, float alpha, int tr,
                                  int lda, int ldb, int ldc, void* stream) {
  if (c && !sb::aligned(c, 4)) return sb::fail(SB_ERR_ALIGN, "sb_gemm_f16_f32out: C must be 4-byte aligned");
  return gemm_f16_impl(a, b, c, 1, m, n, k, alpha, tr, lda, ldb, ldc, stream);
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
  const int esz = scale_dtype == SB_SCALE_F16 ? 2 : 4;
  CUtensorMap tact, tw;
  int rc = make_map(&tact, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, k, m, lda, BK, QT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, k / 2, n, k / 2, BK / 2, QW, CU_TENSOR_MAP_SWIZZLE_NONE);
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
  p.scale_f16 = esz == 2;
  p.alpha = alpha;
  p.kb_total = k / BK;
  int splits = q4_splits(m, n, k, group, esz);
  const size_t need = splits > 1 ? static_cast<size_t>(splits) * m * n * sizeof(float) : 0;
  if (splits > 1 && (!workspace || workspace_bytes < need)) {
    // without room for partial sums run unsplit, if the scales still fit
    if (QW * q4_scale_groups(k / BK, group) * esz > Q_SCALE_BYTES)
      return sb::fail(SB_ERR_WORKSPACE, "sb_gemm_q4: k=%d needs split-K (%zu workspace bytes) for its scales", k, need);
    splits = 1;
  }
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  if (splits > 1) p.ws = static_cast<float*>(workspace);
  static bool done[64] = {false};
  rc = set_smem(gemm_q4_kernel, Q_SMEM, done);
  if (rc) return rc;
  dim3 grid((n + QW - 1) / QW, (m + QT - 1) / QT, splits);
  gemm_q4_kernel<<<grid, Q_WARPS * 32, Q_SMEM, s>>>(tact, tw, p);
  rc = sb::launch_status("gemm_q4_kernel");
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
