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
constexpr int Q_STAGES = 5;                  // shared-memory load stages (cover L2 latency under load + MMA)
constexpr int Q_ASLOTS = 4;                  // TMEM A slots, 32 columns (64 k) each
constexpr int Q_SCALE_BYTES = 24 * 1024;     // the tile's group scales (a split's share of K)
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
  int csplit;          // int4 kernel: > 1 when the K splits of a tile form a cluster and reduce in DSMEM
  int geglu;           // int4 kernel: weight rows are interleaved (gate, up) pairs; C[t][i] = GEGLU of pair i
  unsigned long long* keys;  // int4 kernel: greedy-argmax keys per token (row index offset by row_offset) instead of C
  long long row_offset;
  int bits;            // packed-weight code width: 4 (two per byte) or 2 (four per byte)
  float alpha;
  long long plane;     // f16 kernel, f32 C: elements between the output planes of K splits (blockIdx.z)
  unsigned long long* trace;  // pair kernel, profiling only: kTraceSlots %globaltimer stamps per CTA, or null
  // persistent pair kernel: `pt_pairs` CTA pairs take contiguous runs of the
  // `pt_wtp` weight-row pairs x `pt_ttiles` token tiles (tile = wp * ttiles + tt)
  int pt_pairs, pt_wtp, pt_ttiles;
  int pt_kbc;  // k-blocks per scale tile (scale reload points at multiples of it)
};

// Profiling stamps of the pair kernel (sb_gemm_q4_trace): slot i of CTA b is
// trace[b * kTraceSlots + i], b the CTA's linear index in the grid.
enum {
  TS_SMID = 0,       // the SM the CTA ran on
  TS_ENTRY = 1,      // first instruction
  TS_SETUP = 2,      // barriers initialised, TMEM allocated (after the cluster barrier)
  TS_ACT_GO = 3,     // activation producer: the previous kernel's output may be read
  TS_SCALES = 4,     // dequant warps: the tile's scales are in shared memory
  TS_PACK0 = 5,      // dequant warp 2: first packed stage landed
  TS_MMA0 = 6,       // MMA issuer: first k-block ready
  TS_MMA_END = 7,    // MMA issuer: last MMA issued
  TS_ACCUM = 8,      // epilogue warp 2: accumulator final
  TS_EPI_END = 9,    // epilogue warp 2: its stores (or partial stash) issued
  TS_REDUCED = 10,   // epilogue warp 2: cluster split reduction done
  TS_EXIT = 11,      // TMEM released
  TS_PT_ISSUED0 = 12,  // persistent kernel: MMA issuer, the first tile's MMAs all issued
  TS_PT_FREED0 = 13,   // persistent kernel: epilogue warp 2, first tile's accumulator released
  TS_PT_MMA1 = 14,     // persistent kernel: MMA issuer, the second tile's first MMA
  TS_PT_ACCUM1 = 15,   // persistent kernel: epilogue warp 2, the second tile's accumulator final
  kTraceSlots = 16
};
__device__ __forceinline__ void gemm_stamp(const GemmParams& p, int slot) {
  if (p.trace) {
    const size_t b = blockIdx.x + static_cast<size_t>(gridDim.x) * (blockIdx.y + static_cast<size_t>(gridDim.y) * blockIdx.z);
    p.trace[b * kTraceSlots + slot] = sbd::global_ns();
  }
}

struct Bars {
  uint64_t full[8];
  uint64_t empty[8];
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
          float* dst = static_cast<float*>(p.c) + blockIdx.z * p.plane + static_cast<size_t>(row) * p.ldc + col0;
          if (col0 + 32 <= p.n && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(dst + j) =
                  make_float4(p.alpha * __uint_as_float(r[j]), p.alpha * __uint_as_float(r[j + 1]),
                              p.alpha * __uint_as_float(r[j + 2]), p.alpha * __uint_as_float(r[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.n) dst[j] = p.alpha * __uint_as_float(r[j]);
          }
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
// int4 kernels: dequantised weight as the A operand in tensor memory
// =====================================================================
// p.m = tokens (MMA N side), p.n = weight rows (MMA M side).  Two forms:
//   gemm_q4_kernel       one CTA per 128 weight rows x 256 tokens (cta_group::1)
//   gemm_q4_pair_kernel  a CTA pair per 256 weight rows x 256 tokens
//                        (cta_group::2): each CTA dequantises its own 128
//                        rows into its TMEM and loads half of the 256-token
//                        activation tile; the even CTA issues M=256 MMAs that
//                        read both halves.  Per SM this halves the activation
//                        bytes loaded and read by the tensor core per FLOP,
//                        which shared-memory bandwidth otherwise limits.
// Both share the helpers below.

// The tile's group scales [w0, w0 + 128) x [g_lo, g_lo + gs) -> shared memory
// transposed to [group][row] in their storage type, by `nthreads` threads.
__device__ __forceinline__ void load_scale_tile(const GemmParams& p, uint8_t* sct, int w0, int g_lo, int gs, int dt,
                                                int nthreads) {
  const int esz = p.scale_f16 ? 2 : 4;
  const int gps = p.k / p.group;
  const int rb = gs * esz;  // bytes of one row's scales in this split
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
      const int c = dt + i * nthreads;
      const int rr = c % QW, cb = c / QW;
      v[i] = make_uint4(0u, 0u, 0u, 0u);
      if (c < chunks && w0 + rr < p.n)
        v[i] = __ldg(reinterpret_cast<const uint4*>(sg + (static_cast<size_t>(w0 + rr) * gps + g_lo) * esz) + cb);
    }
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = dt + i * nthreads;
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
    for (int i = dt; i < QW * gs; i += nthreads) {
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
}

// f16(scale * (q - 2)) for the 16 2-bit codes of `w` (byte b holds codes
// 4 b .. 4 b + 3, low bits first), as 8 half2 in k order.  byte_perm copies
// byte b into bytes 0 and 2; masking picks the two codes of a pair into the
// low bits of the two halves; OR-ing 0x6400 makes them 1024 + q and
// subtracting 1026 gives q - 2 exactly.  (q - 2) * s is exact in f16 for an f16
// scale (q - 2 is -2, -1, 0 or 1), so this is the reference's f16 dequant.
__device__ __forceinline__ void dq16_2bit_half(uint32_t w, __half2 s2, uint32_t* out) {
  const __half2 bias = __halves2half2(__ushort_as_half(0x6402), __ushort_as_half(0x6402));  // 1026
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t t = __byte_perm(w, 0u, 0x4040u | (b << 8) | b);  // byte b at bytes 0 and 2
#pragma unroll
    for (int f = 0; f < 2; ++f) {
      uint32_t r = ((t >> (4 * f)) & 0x00000003u) | ((t >> (4 * f + 2)) & 0x00030000u) | 0x64006400u;
      __half2 h = __hsub2(*reinterpret_cast<__half2*>(&r), bias);
      h = __hmul2(h, s2);
      out[2 * b + f] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
}

// Same with an f32 scale: the product is formed in f32 and rounded once.
__device__ __forceinline__ void dq16_2bit_float(uint32_t w, float s, uint32_t* out) {
  const __half2 bias = __halves2half2(__ushort_as_half(0x6402), __ushort_as_half(0x6402));
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t t = __byte_perm(w, 0u, 0x4040u | (b << 8) | b);
#pragma unroll
    for (int f = 0; f < 2; ++f) {
      uint32_t r = ((t >> (4 * f)) & 0x00000003u) | ((t >> (4 * f + 2)) & 0x00030000u) | 0x64006400u;
      const float2 q = __half22float2(__hsub2(*reinterpret_cast<__half2*>(&r), bias));
      __half2 h = __floats2half2_rn(__fmul_rn(s, q.x), __fmul_rn(s, q.y));
      out[2 * b + f] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
}

// One thread's 32 values of a k-block, read from its row of the packed stage
// (16 bytes of 4-bit or 8 bytes of 2-bit codes): f16(scale * (q - zero point))
// packed in pairs.
template <int BITS>
__device__ __forceinline__ void dq_group(const GemmParams& p, const uint8_t* sct, int gi, int r, const uint8_t* codes,
                                         uint32_t (&o)[16]) {
  const bool h16 = p.scale_f16;
  const __half2 s2 = h16 ? __half2half2(reinterpret_cast<const __half*>(sct)[gi * QW + r]) : __half2();
  const float sf = h16 ? 0.f : reinterpret_cast<const float*>(sct)[gi * QW + r];
  if constexpr (BITS == 2) {
    const uint2 q = *reinterpret_cast<const uint2*>(codes);
    const uint32_t words[2] = {q.x, q.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (h16) dq16_2bit_half(words[j], s2, o + 8 * j);
      else dq16_2bit_float(words[j], sf, o + 8 * j);
    }
  } else {
    const uint4 q = *reinterpret_cast<const uint4*>(codes);
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (h16) dq8_half(words[j], s2, o + 4 * j);
      else dq8_float(words[j], sf, o + 4 * j);
    }
  }
}

// Epilogue without split-K: D^T in TMEM (lane = weight row r, column = token);
// warp dw (0..15) drains tokens [64 (dw / 4), +64) of its lane quadrant into
// C (f16, or f32 split partials in p.ws, or GEGLU pairs).
// Greedy argmax over this warp's 32 weight rows for 32 tokens: v[j] is token
// j's value of row `feat` (this lane).  A butterfly leaves lane l holding the
// max key of token l over the warp's rows (31 exchanges instead of 32
// five-step reductions); one atomic MAX per token and warp combines warps
// and CTAs.
__device__ __forceinline__ void argmax_epilogue(const GemmParams& p, const uint32_t (&v)[32], int feat, int lane,
                                                int tok0) {
  unsigned long long k[32];
#pragma unroll
  for (int j = 0; j < 32; ++j)
    k[j] = feat < p.n ? sbd::make_key(p.alpha * __uint_as_float(v[j]), p.row_offset + feat) : 0ull;
#pragma unroll
  for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
    const bool upper = lane & o;  // keep tokens [n/2, n) of the current set, hand the lower half over
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const unsigned long long send = upper ? k[i] : k[i + n / 2];
      const unsigned long long keep = upper ? k[i + n / 2] : k[i];
      const unsigned long long got = __shfl_xor_sync(0xFFFFFFFFu, send, o);
      k[i] = got > keep ? got : keep;
    }
  }
  // lane l now holds token l: the lane bits pick halves most significant first
  if (tok0 + lane < p.m && k[0]) atomicMax(p.keys + tok0 + lane, k[0]);
}

__device__ __forceinline__ void epilogue_direct(const GemmParams& p, uint32_t lane_addr, int dw, int r, int lane,
                                                int w0, int t0, int split, int tile_cols = QT) {
  const int feat = w0 + r;
  const bool feat_ok = feat < p.n;
  for (int cc = 0; cc < 2; ++cc) {
    const int col = (dw >> 2) * 64 + cc * 32;         // token offset within the tile
    if (t0 + col >= p.m || col >= tile_cols) break;  // warp-uniform
    uint32_t v[32];
    sbd::tmem_ld_32x32b_x32(lane_addr + col, v);
    sbd::tmem_wait_ld();
    if (p.keys) {
      argmax_epilogue(p, v, feat, lane, t0 + col);
    } else if (p.ws) {
      if (!feat_ok) continue;
      float* dst = p.ws + (static_cast<size_t>(split) * p.m + t0 + col) * p.n + feat;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (t0 + col + j < p.m) dst[static_cast<size_t>(j) * p.n] = __uint_as_float(v[j]);
    } else if (p.geglu) {
      // lanes 2i, 2i + 1 hold gate and up of output feature feat / 2, rounded
      // to f16 as the GEMM output would be; the even lane forms gelu(gate) * up
      // for tokens col .. col + 15, the odd lane for col + 16 .. col + 31.  A
      // lane rounds its two values (tokens j, 16 + j) with one packed
      // conversion and swaps the pair with its partner in one shuffle.
      const bool odd = lane & 1;
      const bool a1 = p.alpha == 1.f;
      __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(t0 + col + (odd ? 16 : 0)) * p.ldc + (feat >> 1);
      const int jt = t0 + col + (odd ? 16 : 0);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float x0 = __uint_as_float(v[j]), x1 = __uint_as_float(v[16 + j]);
        const __half2 h = a1 ? __floats2half2_rn(x0, x1) : __floats2half2_rn(p.alpha * x0, p.alpha * x1);
        const uint32_t hu = *reinterpret_cast<const uint32_t*>(&h);
        const uint32_t ou = __shfl_xor_sync(0xFFFFFFFFu, hu, 1);
        const __half2 o2 = *reinterpret_cast<const __half2*>(&ou);
        const float g = odd ? __high2float(o2) : __low2float(h);
        const float u = odd ? __high2float(h) : __low2float(o2);
        if (feat_ok && jt + j < p.m) dst[static_cast<size_t>(j) * p.ldc] = __float2half_rn(sbd::gelu_tanh(g) * u);
      }
    } else {
      if (!feat_ok) continue;
      __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(t0 + col) * p.ldc + feat;
      if (p.alpha == 1.f) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (t0 + col + j < p.m) dst[static_cast<size_t>(j) * p.ldc] = __float2half_rn(__uint_as_float(v[j]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (t0 + col + j < p.m)
            dst[static_cast<size_t>(j) * p.ldc] = __float2half_rn(p.alpha * __uint_as_float(v[j]));
      }
    }
  }
}

// Split-K in a cluster: this split's partial tile -> its own shared memory
// (idle activation stages) as [token column][weight row] f32.
__device__ __forceinline__ void stash_partial(uint8_t* smem, uint32_t lane_addr, int dw, int r, int tile_cols = QT) {
  sbd::fence_proxy_async_smem();
  float* red = reinterpret_cast<float*>(smem);
  for (int cc = 0; cc < 2; ++cc) {
    const int col = (dw >> 2) * 64 + cc * 32;
    if (col >= tile_cols) break;  // warp-uniform
    uint32_t v[32];
    sbd::tmem_ld_32x32b_x32(lane_addr + col, v);
    sbd::tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) red[(col + j) * QW + r] = __uint_as_float(v[j]);
  }
}

// Split-K reduction through distributed shared memory, by the 16 epilogue
// warps (ew = 0..15): split `z` of `nz` sums token columns [z QT / nz,
// (z + 1) QT / nz) of the tile over all splits in split order (the order and
// rounding of splitk_finalize_kernel), split z' living in cluster CTA
// rank_base + rank_stride * z'; then writes f16 (or GEGLU pairs).
__device__ __forceinline__ void reduce_splits(const GemmParams& p, uint8_t* smem, int ew, int lane, int w0, int t0,
                                              int z, int nz, int rank_base, int rank_stride, int tile_cols = QT) {
  const int c_lo = z * tile_cols / nz, c_hi = (z + 1) * tile_cols / nz;
  const uint32_t red0 = sbd::smem_u32(smem);
  const int rr = lane * 4;  // weight rows rr .. rr + 3 of the tile
  const int feat = w0 + rr;
  for (int c = c_lo + ew; c < c_hi; c += Q_DQ_WARPS) {
    if (t0 + c >= p.m) break;  // warp-uniform
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int zz = 0; zz < nz; ++zz) {
      const float4 v = sbd::ld_dsmem_v4(sbd::mapa_shared(red0 + (c * QW + rr) * 4, rank_base + rank_stride * zz));
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if (p.geglu) {
      // rows (rr, rr + 1) and (rr + 2, rr + 3) are (gate, up) pairs
      __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(t0 + c) * p.ldc + (feat >> 1);
      const float g0 = __half2float(__float2half_rn(p.alpha * acc.x));
      const float u0 = __half2float(__float2half_rn(p.alpha * acc.y));
      const float g1 = __half2float(__float2half_rn(p.alpha * acc.z));
      const float u1 = __half2float(__float2half_rn(p.alpha * acc.w));
      if (feat + 1 < p.n) dst[0] = __float2half_rn(sbd::gelu_tanh(g0) * u0);
      if (feat + 3 < p.n) dst[1] = __float2half_rn(sbd::gelu_tanh(g1) * u1);
      continue;
    }
    __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(t0 + c) * p.ldc + feat;
    const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
    if (feat + 4 <= p.n && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
      const __half2 h0 = __floats2half2_rn(p.alpha * vals[0], p.alpha * vals[1]);
      const __half2 h1 = __floats2half2_rn(p.alpha * vals[2], p.alpha * vals[3]);
      *reinterpret_cast<uint2*>(dst) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (feat + e < p.n) dst[e] = __float2half_rn(p.alpha * vals[e]);
    }
  }
}

template <int BITS>
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
        sbd::mbar_arrive_expect_tx(&bars->full[s], Q_ACT_BYTES + QW * BK * BITS / 8);
        const int k0 = (kb0 + kb) * BK;
        sbd::tma_load_2d(&tmAct, &bars->full[s], smem + s * Q_ACT_BYTES, k0, t0);
        sbd::tma_load_2d(&tmW, &bars->full[s], smem + Q_OFF_PACK + s * Q_PACK_BYTES, k0 * BITS / 8, w0);
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
    uint8_t* sct = smem + Q_OFF_SCALE;
    load_scale_tile(p, sct, w0, g_lo, gs, dt, Q_DQ_WARPS * 32);
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
      constexpr int rowb = 8 * BITS, halfb = 4 * BITS;  // packed bytes of a row's k-block and of its half
      const uint8_t* q = smem + Q_OFF_PACK + s * Q_PACK_BYTES + r * rowb + khalf * halfb;
      uint32_t o[16];
      dq_group<BITS>(p, sct, gi, r, q, o);
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
      if (p.csplit > 1) stash_partial(smem, lane_addr, dw, r);
      else epilogue_direct(p, lane_addr, dw, r, lane, w0, t0, blockIdx.z);
    }
  }

  if (p.csplit > 1) {
    // every thread of every split reaches both cluster barriers (abort paths
    // included), so a barrier only ever waits on peers' bounded waits
    sbd::cluster_sync_all();
    if (warp >= 2) {
      const int rank = static_cast<int>(sbd::cluster_ctarank());
      reduce_splits(p, smem, warp - 2, lane, w0, t0, rank, p.csplit, 0, 1);
    }
    sbd::cluster_sync_all();
  }

  sbd::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc(tmem, Q_TMEM_COLS);
  }
}


// ---- CTA-pair form (cta_group::2): 256 weight rows x 256 tokens per pair
constexpr int P_STAGES = 8;                       // stages; stage s is also TMEM A slot s (256 + 8 x 32 columns)
constexpr int P_WLOAD = Q_WARPS;                  // warp issuing the packed-weight loads (both CTAs)
constexpr int P_WARPS = P_WLOAD + 1;
constexpr int P_ACT_BYTES = (QT / 2) * BK * 2;    // 16 KB: this CTA's 128 tokens of a k-block
constexpr int P_OFF_PACK = P_STAGES * P_ACT_BYTES;
constexpr int P_OFF_SCALE = P_OFF_PACK + P_STAGES * Q_PACK_BYTES;
constexpr int P_OFF_BAR = P_OFF_SCALE + Q_SCALE_BYTES;
constexpr int P_SMEM = P_OFF_BAR + 512 + 1024;
static_assert(P_STAGES * P_ACT_BYTES >= QT * QW * 4, "split-K partial tile must fit the activation stages");

// Stage s of k-block kb (s = kb % P_STAGES) is both an activation-half buffer
// and TMEM A slot s, so one barrier tells the MMA issuer that k-block kb is
// ready and one commit frees both.
struct PairBars {
  uint64_t ready[P_STAGES];   // even CTA: both activation halves landed (tx) and both CTAs' dequant
                              // groups wrote A slot s (8 local + 8 remote arrives)
  uint64_t empty[P_STAGES];   // each CTA: the pair's MMAs are done with stage / A slot s
  uint64_t pfull[P_STAGES];   // each CTA: its packed tile of stage s landed
  uint64_t pempty[P_STAGES];  // each CTA: its dequant warps are done with that packed tile
  uint64_t accum;             // each CTA: its accumulator rows are final
  uint32_t tmem_slot;
  int abort;
};
static_assert(sizeof(PairBars) <= 512, "pair barrier block");

// Cross-CTA hand-off: the odd CTA's dequant warps arrive on the even CTA's
// `ready` barrier directly, with the default (CTA-scope release) remote arrive
// after tcgen05.wait::st + tcgen05.fence::before_thread_sync -- the hand-off
// CUTLASS's 2-SM async-producer -> UMMA pipeline uses.  A cluster-scope
// release arrive costs about a microsecond per k-block.
template <int BITS, int NT>
__global__ void __launch_bounds__(P_WARPS * 32, 1)
    gemm_q4_pair_kernel(const __grid_constant__ CUtensorMap tmAct, const __grid_constant__ CUtensorMap tmW,
                        const GemmParams p) {
  constexpr int S = P_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + P_OFF_BAR);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0 && p.trace) {
    gemm_stamp(p, TS_ENTRY);
    uint32_t sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    const size_t b = blockIdx.x + static_cast<size_t>(gridDim.x) * (blockIdx.y + static_cast<size_t>(gridDim.y) * blockIdx.z);
    p.trace[b * kTraceSlots + TS_SMID] = sm;
  }
  // cluster (2, 1, csplit): rank = pair position + 2 * split
  const int rank = static_cast<int>(sbd::cluster_ctarank());
  const int lead_rank = rank & ~1;
  const bool lead = rank == lead_rank;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << lead_rank);
  const int w0 = blockIdx.x * QW;                  // this CTA's 128 weight rows
  static_assert(NT % 32 == 0 && NT >= 32 && NT <= QT, "token tile");
  const int t0 = blockIdx.y * NT;                  // the pair's NT tokens (MMA N)
  const int th = t0 + (rank & 1) * (NT / 2);       // this CTA's half of them
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int nkb = min(p.kb_per_split, p.kb_total - kb0);
  const int g_lo = (kb0 * BK) / p.group;
  const int g_hi = ((kb0 + nkb) * BK + p.group - 1) / p.group;
  const int gs = g_hi - g_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      sbd::mbar_init(&bars->ready[i], 1 + 8 + 8);
      sbd::mbar_init(&bars->empty[i], 1);
      sbd::mbar_init(&bars->pfull[i], 1);
      sbd::mbar_init(&bars->pempty[i], 8);
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
    sbd::tmem_alloc_pair(&bars->tmem_slot, Q_TMEM_COLS);
    sbd::tmem_relinquish_pair();
  }
  // barriers initialised and TMEM allocated in both CTAs before any cross-CTA use
  sbd::tc_fence_before();
  sbd::cluster_sync_all();
  sbd::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;
  if (threadIdx.x == 0) gemm_stamp(p, TS_SETUP);

  // the next kernel in the stream may start its prologue; this kernel's own
  // reads of the previous kernel's output (the activations) wait below
  sbd::griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ activation TMA producer (both CTAs)
    if (lane == 0) {
      sbd::griddep_wait();
      gemm_stamp(p, TS_ACT_GO);
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = ((kb / S) & 1) ^ 1;
        const int k0 = (kb0 + kb) * BK;
        if (!sbd::mbar_wait_cluster(&bars->empty[s], ph, abort, p.err)) break;
        if (lead) sbd::mbar_arrive_expect_tx(&bars->ready[s], NT * BK * 2);  // both CTAs' NT/2-token halves
        sbd::tma_load_2d_pair(&tmAct, sbd::mapa_shared(sbd::smem_u32(&bars->ready[s]), lead_rank),
                              smem + s * P_ACT_BYTES, k0, th);
        issued = kb + 1;
      }
      if (*abort && lead) {
        // let copies in flight land before shared memory is released: the even
        // CTA's activation barriers count both CTAs' halves (ready also needs
        // the dequant arrivals, which an aborted step may never make: bound by
        // the drain's own time limit)
        for (int kb = max(0, issued - S); kb < issued; ++kb) drain_wait(&bars->ready[kb % S], (kb / S) & 1);
      }
    }
  } else if (warp == P_WLOAD) {
    // ------------------------------------------------------------ packed-weight TMA producer (both CTAs)
    // Weights do not come from the previous kernel, so they stream before its
    // end; a packed stage is refilled as soon as the dequant warps are done
    // with it, running up to P_STAGES k-blocks ahead of them.
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        if (!sbd::mbar_wait(&bars->pempty[s], ((kb / S) & 1) ^ 1, abort, p.err)) break;
        sbd::mbar_arrive_expect_tx(&bars->pfull[s], QW * BK * BITS / 8);
        sbd::tma_load_2d(&tmW, &bars->pfull[s], smem + P_OFF_PACK + s * Q_PACK_BYTES, (kb0 + kb) * BK * BITS / 8, w0);
        issued = kb + 1;
      }
      if (*abort)
        for (int kb = max(0, issued - S); kb < issued; ++kb) drain_wait(&bars->pfull[kb % S], (kb / S) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    // The tensor pipe takes an MMA only shortly before it can start it, so
    // every instruction this thread runs between MMAs is on the critical path:
    // descriptors are fixed offsets from one base, stage indices are
    // compile-time (the loop is unrolled over one pass of the ring), and the
    // next stage's barrier is tested (without blocking) before this stage's
    // last MMA, so a ready stage costs no wait.
    if (lane == 0 && lead) {
      constexpr uint32_t idesc = sbd::umma_idesc_f16(2 * QW, NT, 0, 0);
      const uint64_t bdesc0 = sbd::umma_desc(sbd::smem_u32(smem), 16, 1024, sbd::kLayoutSwizzle128B);
      const uint32_t a0 = tmem + 256;
      bool ok = nkb > 0 && sbd::mbar_wait_cluster(&bars->ready[0], 0, abort, p.err);
      gemm_stamp(p, TS_MMA0);
      for (int base = 0; ok && base < nkb; base += S) {
        const uint32_t ph = (base / S) & 1;
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int kb = base + j;
          if (kb >= nkb) break;
          constexpr int kStepDesc = (UMMA_K * 2) >> 4;  // 32 bytes along K, in descriptor units
          const uint64_t bd = bdesc0 + static_cast<uint64_t>((j * P_ACT_BYTES) >> 4);
          const uint32_t ad = a0 + j * 32;
          const uint32_t ph_next = j + 1 == S ? ph ^ 1 : ph;
          sbd::tc_fence_after();
          sbd::umma_f16_ts_pair(tmem, ad, bd, idesc, kb != 0 ? 1u : 0u);
          sbd::umma_f16_ts_pair(tmem, ad + 8, bd + kStepDesc, idesc, 1u);
          sbd::umma_f16_ts_pair(tmem, ad + 16, bd + 2 * kStepDesc, idesc, 1u);
          const bool next_ready = kb + 1 >= nkb || sbd::mbar_test_wait_cluster(&bars->ready[(j + 1) % S], ph_next);
          sbd::umma_f16_ts_pair(tmem, ad + 24, bd + 3 * kStepDesc, idesc, 1u);
          sbd::umma_commit_pair(&bars->empty[j], pair_mask);
          if (!next_ready && !sbd::mbar_wait_cluster(&bars->ready[(j + 1) % S], ph_next, abort, p.err)) {
            ok = false;
            break;
          }
        }
      }
      gemm_stamp(p, TS_MMA_END);
      sbd::umma_commit_pair(&bars->accum, pair_mask);
    }
  } else {
    // ------------------------------------------------------------ dequant producers (warps 2..17, both CTAs)
    const int dw = warp - 2;
    const int grp = dw >> 3;
    const int quad = warp & 3;
    const int khalf = (dw & 7) >> 2;
    const int r = quad * 32 + lane;
    const int dt = threadIdx.x - 64;
    uint8_t* sct = smem + P_OFF_SCALE;
    load_scale_tile(p, sct, w0, g_lo, gs, dt, Q_DQ_WARPS * 32);
    sbd::named_bar_sync(1, Q_DQ_WARPS * 32);
    if (dt == 0) gemm_stamp(p, TS_SCALES);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t ready_lead = sbd::mapa_shared(sbd::smem_u32(&bars->ready[0]), lead_rank);
    const int kstep = Q_DQ_GROUPS * BK;
    const int gstep = kstep % p.group == 0 ? kstep / p.group : 0;
    int gi = ((kb0 + grp) * BK + khalf * 32) / p.group - g_lo;
    for (int kb = grp; kb < nkb; kb += Q_DQ_GROUPS) {
      const int s = kb % S, slot = s;
      if (gstep == 0) gi = ((kb0 + kb) * BK + khalf * 32) / p.group - g_lo;
      bool ok = sbd::mbar_wait(&bars->pfull[s], (kb / S) & 1, abort, p.err);
      if (dt == 0 && kb == 0) gemm_stamp(p, TS_PACK0);
      if (ok) ok = sbd::mbar_wait_cluster(&bars->empty[s], ((kb / S) & 1) ^ 1, abort, p.err);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      sbd::tc_fence_after();
      constexpr int rowb = 8 * BITS, halfb = 4 * BITS;  // packed bytes of a row's k-block and of its half
      const uint8_t* q = smem + P_OFF_PACK + s * Q_PACK_BYTES + r * rowb + khalf * halfb;
      uint32_t o[16];
      dq_group<BITS>(p, sct, gi, r, q, o);
      sbd::tmem_st_32x32b_x16(lane_addr + 256 + slot * 32 + khalf * 16, o);
      sbd::tmem_wait_st();
      sbd::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        sbd::mbar_arrive(&bars->pempty[s]);
        if (lead) sbd::mbar_arrive(&bars->ready[s]);
        else sbd::mbar_arrive_remote_cta(ready_lead + s * sizeof(uint64_t));
      }
      gi += gstep;
    }
    // ------------------------------------------------------------ epilogue (this CTA's 128 rows)
    const bool ok = __all_sync(0xFFFFFFFFu, sbd::mbar_wait_cluster(&bars->accum, 0, abort, p.err));
    if (dt == 0) gemm_stamp(p, TS_ACCUM);
    if (ok) {
      sbd::tc_fence_after();
      if (p.csplit > 1) stash_partial(smem, lane_addr, dw, r, NT);
      else epilogue_direct(p, lane_addr, dw, r, lane, w0, t0, blockIdx.z, NT);
    }
    if (dt == 0) gemm_stamp(p, TS_EPI_END);
  }

  if (p.csplit > 1) {
    // every thread of every CTA reaches both cluster barriers (abort paths included)
    sbd::cluster_sync_all();
    if (warp >= 2 && warp < Q_WARPS)
      reduce_splits(p, smem, warp - 2, lane, w0, t0, rank >> 1, p.csplit, rank & 1, 2, NT);
    sbd::cluster_sync_all();
    if (threadIdx.x == 64) gemm_stamp(p, TS_REDUCED);
  }

  // both CTAs are done with TMEM (the pair's MMAs completed before `accum`)
  sbd::tc_fence_before();
  sbd::cluster_sync_all();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc_pair(tmem, Q_TMEM_COLS);
    if (lane == 0) gemm_stamp(p, TS_EXIT);
  }
}

// ---- persistent form of the pair kernel (gemm_q4_persist_kernel)
// For a matrix with more 256 x 256 tiles than the device holds CTA pairs, one
// launch runs one pair per pair slot, and pair p takes the contiguous tiles
// [T p / P, T (p + 1) / P) (tile = weight-row pair wp * token tiles + tt).  The
// rings of the pair kernel run on from tile to tile, and a tile's epilogue
// overlaps the next tile's MMAs: at a tile boundary the dequant warps load the
// next tile's scales and dequantise its first P_STAGES k-blocks (into A slots
// the finishing MMAs free), then read the finished accumulator into registers,
// release it (the MMA issuer starts the next tile on `accfree`, its first
// stages already full) and only then form and store the outputs.  The MMA
// issuer keeps its ring position incrementally: between two MMAs it runs only
// what the next MMA needs.
struct PtBars {
  PairBars pb;
  uint64_t accfree;  // even CTA: both CTAs' epilogue warps have read the accumulator
};
static_assert(sizeof(PtBars) <= 512, "persistent barrier block");

// 32 token columns c0 .. c0 + 31 of output feature `feat` (this lane's weight
// row) -> C, from h[j] = (f16(alpha * sum_j), f16(alpha * sum_{16 + j})): the
// values epilogue_direct forms (the outputs, or for GEGLU the rounded gate / up
// that lanes 2i, 2i + 1 hold for output feature feat / 2; the even lane writes
// gelu(gate) * up for columns c0 .. c0 + 15, the odd lane for c0 + 16 .. + 31).
__device__ __forceinline__ void pt_store_cols(const GemmParams& p, const uint32_t (&h)[16], int feat, int lane,
                                              int c0) {
  const bool feat_ok = feat < p.n;
  if (p.geglu) {
    const bool odd = lane & 1;
    __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(c0 + (odd ? 16 : 0)) * p.ldc + (feat >> 1);
    const int jt = c0 + (odd ? 16 : 0);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t ou = __shfl_xor_sync(0xFFFFFFFFu, h[j], 1);
      const __half2 mine = *reinterpret_cast<const __half2*>(&h[j]);
      const __half2 o2 = *reinterpret_cast<const __half2*>(&ou);
      const float g = odd ? __high2float(o2) : __low2float(mine);
      const float u = odd ? __high2float(mine) : __low2float(o2);
      if (feat_ok && jt + j < p.m) dst[static_cast<size_t>(j) * p.ldc] = __float2half_rn(sbd::gelu_tanh(g) * u);
    }
  } else if (feat_ok) {
    __half* dst = static_cast<__half*>(p.c) + static_cast<size_t>(c0) * p.ldc + feat;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const __half2 hh = *reinterpret_cast<const __half2*>(&h[j]);
      if (c0 + j < p.m) dst[static_cast<size_t>(j) * p.ldc] = __low2half(hh);
      if (c0 + 16 + j < p.m) dst[static_cast<size_t>(16 + j) * p.ldc] = __high2half(hh);
    }
  }
}

// f16(alpha * v[j]), f16(alpha * v[16 + j]) packed for pt_store_cols
__device__ __forceinline__ void pt_round(const GemmParams& p, const uint32_t (&v)[32], uint32_t (&h)[16]) {
  const bool a1 = p.alpha == 1.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float x0 = __uint_as_float(v[j]), x1 = __uint_as_float(v[16 + j]);
    const __half2 hh = a1 ? __floats2half2_rn(x0, x1) : __floats2half2_rn(p.alpha * x0, p.alpha * x1);
    h[j] = *reinterpret_cast<const uint32_t*>(&hh);
  }
}

// One tile's epilogue in the persistent kernel (the ti-th tile of this pair;
// feat / tok: this thread's weight row and first token column): wait for the
// accumulator, read this warp's 64 columns into registers (rounded to f16 as
// stored), release the accumulator to the MMA issuer, then form and store the
// outputs.  Returns the thread's ok flag (false after a failed wait).
__device__ __forceinline__ bool pt_epilogue(const GemmParams& p, PairBars* bars, PtBars* pbars, uint32_t lane_addr,
                                         int feat, int tok, int ti, bool lead, int dt, int lane, bool ok) {
  volatile int* abort = &bars->abort;
  if (ok) ok = sbd::mbar_wait_cluster(&bars->accum, ti & 1, abort, p.err);
  ok = __all_sync(0xFFFFFFFFu, ok);
  if (dt == 0 && ti <= 1) gemm_stamp(p, ti == 0 ? TS_ACCUM : TS_PT_ACCUM1);
  sbd::tc_fence_after();
  uint32_t h[2][16];  // the outputs rounded to f16 (as stored), so the registers held are halved
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    uint32_t a[32];
    sbd::tmem_ld_32x32b_x32(lane_addr + 32 * u, a);
    sbd::tmem_wait_ld();
    pt_round(p, a, h[u]);
  }
  sbd::tc_fence_before();
  sbd::named_bar_sync(1, Q_DQ_WARPS * 32);
  if (dt == 0) {
    if (lead) sbd::mbar_arrive(&pbars->accfree);
    else sbd::mbar_arrive_remote_cta(sbd::mapa_shared(sbd::smem_u32(&pbars->accfree), 0));
    if (ti == 0) gemm_stamp(p, TS_PT_FREED0);
  }
  if (ok) {
    pt_store_cols(p, h[0], feat, lane, tok);
    pt_store_cols(p, h[1], feat, lane, tok + 32);
  }
  if (dt == 0 && ti == 0) gemm_stamp(p, TS_EPI_END);
  return ok;
}

template <int BITS>
__global__ void __launch_bounds__(P_WARPS * 32, 1)
    gemm_q4_persist_kernel(const __grid_constant__ CUtensorMap tmAct, const __grid_constant__ CUtensorMap tmW,
                           const GemmParams p) {
  constexpr int S = P_STAGES, NT = QT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PtBars* pbars = reinterpret_cast<PtBars*>(smem + P_OFF_BAR);
  PairBars* bars = &pbars->pb;
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = static_cast<int>(sbd::cluster_ctarank());  // cluster (2, 1, 1): 0 = even CTA
  const bool lead = rank == 0;
  constexpr uint16_t pair_mask = 3;
  const int KB = p.kb_total;
  const int tiles = p.pt_wtp * p.pt_ttiles;
  const int t_first = static_cast<int>(static_cast<long long>(tiles) * blockIdx.y / p.pt_pairs);
  const int t_end = static_cast<int>(static_cast<long long>(tiles) * (blockIdx.y + 1) / p.pt_pairs);
  auto rows_of = [&](int t) { return (2 * (t / p.pt_ttiles) + rank) * QW; };  // this CTA's 128 weight rows
  auto toks_of = [&](int t) { return (t % p.pt_ttiles) * NT; };              // the pair's 256 tokens
  if (threadIdx.x == 0 && p.trace) {
    gemm_stamp(p, TS_ENTRY);
    uint32_t sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    p.trace[(blockIdx.x + static_cast<size_t>(gridDim.x) * blockIdx.y) * kTraceSlots + TS_SMID] = sm;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      sbd::mbar_init(&bars->ready[i], 1 + 8 + 8);
      sbd::mbar_init(&bars->empty[i], 1);
      sbd::mbar_init(&bars->pfull[i], 1);
      sbd::mbar_init(&bars->pempty[i], 8);
    }
    sbd::mbar_init(&bars->accum, 1);
    sbd::mbar_init(&pbars->accfree, 2);
    bars->abort = 0;
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    sbd::prefetch_tmap(&tmAct);
    sbd::prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    sbd::tmem_alloc_pair(&bars->tmem_slot, Q_TMEM_COLS);
    sbd::tmem_relinquish_pair();
  }
  sbd::tc_fence_before();
  sbd::cluster_sync_all();
  sbd::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;
  if (threadIdx.x == 0) gemm_stamp(p, TS_SETUP);
  sbd::griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ activation TMA producer (both CTAs)
    if (lane == 0) {
      sbd::griddep_wait();
      gemm_stamp(p, TS_ACT_GO);
      int it = 0;
      bool ok = true;
      for (int t = t_first; ok && t < t_end; ++t) {
        const int th = toks_of(t) + rank * (NT / 2);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it & (S - 1);
          if (!sbd::mbar_wait_cluster(&bars->empty[s], ((it / S) & 1) ^ 1, abort, p.err)) {
            ok = false;
            break;
          }
          if (lead) sbd::mbar_arrive_expect_tx(&bars->ready[s], NT * BK * 2);
          sbd::tma_load_2d_pair(&tmAct, sbd::mapa_shared(sbd::smem_u32(&bars->ready[s]), 0),
                                smem + s * P_ACT_BYTES, kb * BK, th);
        }
      }
      if (*abort && lead)
        for (int i = max(0, it - S); i < it; ++i) drain_wait(&bars->ready[i & (S - 1)], (i / S) & 1);
    }
  } else if (warp == P_WLOAD) {
    // ------------------------------------------------------------ packed-weight TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = t_first; ok && t < t_end; ++t) {
        const int w0 = rows_of(t);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it & (S - 1);
          if (!sbd::mbar_wait(&bars->pempty[s], ((it / S) & 1) ^ 1, abort, p.err)) {
            ok = false;
            break;
          }
          sbd::mbar_arrive_expect_tx(&bars->pfull[s], QW * BK * BITS / 8);
          sbd::tma_load_2d(&tmW, &bars->pfull[s], smem + P_OFF_PACK + s * Q_PACK_BYTES, kb * BK * BITS / 8, w0);
        }
      }
      if (*abort)
        for (int i = max(0, it - S); i < it; ++i) drain_wait(&bars->pfull[i & (S - 1)], (i / S) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && lead) {
      constexpr uint32_t idesc = sbd::umma_idesc_f16(2 * QW, NT, 0, 0);
      constexpr int kStepDesc = (UMMA_K * 2) >> 4;  // 32 bytes along K, in descriptor units
      const uint64_t bdesc0 = sbd::umma_desc(sbd::smem_u32(smem), 16, 1024, sbd::kLayoutSwizzle128B);
      const uint32_t a0 = tmem + 256;
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = t_first, ti = 0; t < t_end; ++t, ++ti) {
        // the accumulator is free once both CTAs' epilogue warps have read the previous tile's
        if (ok && ti > 0) ok = sbd::mbar_wait_cluster(&pbars->accfree, (ti - 1) & 1, abort, p.err);
        sbd::tc_fence_after();
        if (ok) ok = sbd::mbar_wait_cluster(&bars->ready[s], ph, abort, p.err);
        if (ti <= 1) gemm_stamp(p, ti == 0 ? TS_MMA0 : TS_PT_MMA1);
        uint32_t acc = 0u;
        for (int n = KB; ok && n > 0; --n) {
          sbd::tc_fence_after();
          const uint64_t bd = bdesc0 + static_cast<uint64_t>((s * P_ACT_BYTES) >> 4);
          const uint32_t ad = a0 + s * 32;
          const int s1 = (s + 1) & (S - 1);
          const uint32_t ph1 = s1 == 0 ? ph ^ 1u : ph;
          sbd::umma_f16_ts_pair(tmem, ad, bd, idesc, acc);
          sbd::umma_f16_ts_pair(tmem, ad + 8, bd + kStepDesc, idesc, 1u);
          sbd::umma_f16_ts_pair(tmem, ad + 16, bd + 2 * kStepDesc, idesc, 1u);
          const bool next_ready = n == 1 || sbd::mbar_test_wait_cluster(&bars->ready[s1], ph1);
          sbd::umma_f16_ts_pair(tmem, ad + 24, bd + 3 * kStepDesc, idesc, 1u);
          sbd::umma_commit_pair(&bars->empty[s], pair_mask);
          acc = 1u;
          s = s1;
          ph = ph1;
          if (n > 1 && !next_ready && !sbd::mbar_wait_cluster(&bars->ready[s], ph, abort, p.err)) ok = false;
        }
        // (also after a failure: the epilogue warps' wait on `accum` then ends
        // at once or on their own abort check)
        sbd::umma_commit_pair(&bars->accum, pair_mask);
        if (ti == 0) gemm_stamp(p, TS_PT_ISSUED0);
      }
      gemm_stamp(p, TS_MMA_END);
    }
  } else {
    // ------------------------------------------------------------ dequant producers + epilogue (warps 2..17, both CTAs)
    // Every one of these 512 threads walks the same tiles, scale tiles and
    // epilogues and meets every named barrier, failures included (a failed
    // wait only skips work), so no barrier waits on a thread that left.
    constexpr int kDq = Q_DQ_WARPS * 32;
    const int dw = warp - 2;
    const int grp = dw >> 3;
    const int quad = warp & 3;
    const int khalf = (dw & 7) >> 2;
    const int r = quad * 32 + lane;
    const int dt = threadIdx.x - 64;
    uint8_t* sct = smem + P_OFF_SCALE;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t ready_lead = sbd::mapa_shared(sbd::smem_u32(&bars->ready[0]), 0);
    const int col0 = (dw >> 2) * 64;  // this warp's 64 token columns of its lane quadrant
    // a group's scale index advances by gstep per k-block it takes (0: recomputed)
    const int gstep = (Q_DQ_GROUPS * BK) % p.group == 0 ? Q_DQ_GROUPS * BK / p.group : 0;
    bool ok = true;
    auto epilogue = [&](int t, int ti) {
      ok = pt_epilogue(p, bars, pbars, lane_addr + col0, rows_of(t) + r, toks_of(t) + col0, ti, lead, dt, lane, ok);
    };
    int it0 = 0;  // ring position of the tile's first k-block
    for (int t = t_first, ti = 0; t < t_end; ++t, ++ti) {
      const int w0 = rows_of(t);
      // k-blocks of this tile dequantised before the previous tile's epilogue
      // (the first scale tile covers them: pt_kbc >= P_STAGES or the whole tile)
      const int E = min(S, KB);
      bool epi = ti == 0;
      for (int c_lo = 0; c_lo < KB;) {
        // one scale tile: k-blocks [c_lo, the next multiple of pt_kbc or the tile end)
        const int c_hi = min(KB, (c_lo / p.pt_kbc + 1) * p.pt_kbc);
        const int g_lo = (c_lo * BK) / p.group;
        const int g_hi = (c_hi * BK + p.group - 1) / p.group;
        sbd::named_bar_sync(1, kDq);  // every dequant warp is done with the previous scale tile
        load_scale_tile(p, sct, w0, g_lo, g_hi - g_lo, dt, kDq);
        sbd::named_bar_sync(1, kDq);
        int kb = c_lo + ((grp - (it0 + c_lo)) & 1);  // this group's first k-block here
        int gi = (kb * BK + khalf * 32) / p.group - g_lo;
        for (; kb < c_hi; kb += Q_DQ_GROUPS) {
          if (!epi && kb >= E) {
            epilogue(t - 1, ti - 1);
            epi = true;
          }
          const int itk = it0 + kb;
          const int s = itk & (S - 1);
          const uint32_t ph = (itk / S) & 1;
          if (gstep == 0) gi = (kb * BK + khalf * 32) / p.group - g_lo;
          if (ok) ok = sbd::mbar_wait(&bars->pfull[s], ph, abort, p.err);
          if (ok) ok = sbd::mbar_wait_cluster(&bars->empty[s], ph ^ 1, abort, p.err);
          ok = __all_sync(0xFFFFFFFFu, ok);
          if (ok) {
            sbd::tc_fence_after();
            constexpr int rowb = 8 * BITS, halfb = 4 * BITS;  // packed bytes of a row's k-block and of its half
            const uint8_t* q = smem + P_OFF_PACK + s * Q_PACK_BYTES + r * rowb + khalf * halfb;
            uint32_t o[16];
            dq_group<BITS>(p, sct, gi, r, q, o);
            sbd::tmem_st_32x32b_x16(lane_addr + 256 + s * 32 + khalf * 16, o);
            sbd::tmem_wait_st();
            sbd::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              sbd::mbar_arrive(&bars->pempty[s]);
              if (lead) sbd::mbar_arrive(&bars->ready[s]);
              else sbd::mbar_arrive_remote_cta(ready_lead + s * sizeof(uint64_t));
            }
          }
          gi += gstep;
        }
        if (!epi && c_hi >= E) {  // a group with no k-block at or past E in this scale tile
          epilogue(t - 1, ti - 1);
          epi = true;
        }
        c_lo = c_hi;
      }
      it0 += KB;
    }
    if (t_end > t_first) epilogue(t_end - 1, t_end - 1 - t_first);
  }

  // both CTAs are done with TMEM (the pair's MMAs completed before `accum`)
  sbd::tc_fence_before();
  sbd::cluster_sync_all();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc_pair(tmem, Q_TMEM_COLS);
    if (lane == 0) gemm_stamp(p, TS_EXIT);
  }
}

__global__ void splitk_finalize_kernel(const float* __restrict__ ws, __half* __restrict__ c, int m, int n, int ldc,
                                       int splits, float alpha, int geglu) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();  // the partial planes are the previous kernel's output
  const size_t plane = static_cast<size_t>(m) * n;
  const int nout = geglu ? n / 2 : n;
  const size_t total = static_cast<size_t>(m) * nout;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / nout, col = i - row * nout;
    if (geglu) {
      // partial planes hold gate (2 col) and up (2 col + 1) rows; round each to
      // f16 as the GEMM output would be, then gelu(gate) * up
      const size_t e = row * n + 2 * col;
      float g = 0.f, u = 0.f;
      for (int z = 0; z < splits; ++z) {
        g += ws[z * plane + e];
        u += ws[z * plane + e + 1];
      }
      const float gh = __half2float(__float2half_rn(alpha * g)), uh = __half2float(__float2half_rn(alpha * u));
      c[row * ldc + col] = __float2half_rn(sbd::gelu_tanh(gh) * uh);
    } else {
      float s = 0.f;
      for (int z = 0; z < splits; ++z) s += ws[z * plane + i];
      c[row * ldc + col] = __float2half_rn(alpha * s);
    }
  }
}

// splitk_finalize_kernel four partial columns at a time (n % 4 == 0): float4
// loads of every split issued before the sums, which run in split order as
// in the scalar kernel (bit-identical results).
__global__ void splitk_finalize_v4_kernel(const float* __restrict__ ws, __half* __restrict__ c, int m, int n, int ldc,
                                          int splits, float alpha, int geglu) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();  // the partial planes are the previous kernel's output
  const size_t plane4 = static_cast<size_t>(m) * n / 4;
  const int n4 = n / 4;
  const float4* w4 = reinterpret_cast<const float4*>(ws);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < plane4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / n4, c4 = i - row * n4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int z = 0;
    for (; z + 4 <= splits; z += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = w4[(z + u) * plane4 + i];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc.x += v[u].x;
        acc.y += v[u].y;
        acc.z += v[u].z;
        acc.w += v[u].w;
      }
    }
    for (; z < splits; ++z) {
      const float4 v = w4[z * plane4 + i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if (geglu) {
      // columns (4 c4 .. + 3) = (gate, up) of outputs 2 c4 and 2 c4 + 1
      const float g0 = __half2float(__float2half_rn(alpha * acc.x)), u0 = __half2float(__float2half_rn(alpha * acc.y));
      const float g1 = __half2float(__float2half_rn(alpha * acc.z)), u1 = __half2float(__float2half_rn(alpha * acc.w));
      *reinterpret_cast<__half2*>(c + row * ldc + 2 * c4) =
          __halves2half2(__float2half_rn(sbd::gelu_tanh(g0) * u0), __float2half_rn(sbd::gelu_tanh(g1) * u1));
    } else {
      const __half2 lo = __floats2half2_rn(alpha * acc.x, alpha * acc.y);
      const __half2 hi = __floats2half2_rn(alpha * acc.z, alpha * acc.w);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&lo);
      o.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(c + row * ldc + 4 * c4) = o;
    }
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
  dim3 grid((p.n + BN - 1) / BN, (p.m + BM - 1) / BM, (p.kb_total + p.kb_per_split - 1) / p.kb_per_split);
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
  const bool v4 = p.n % 4 == 0 && sb::aligned(p.ws, 16) &&
                  (p.geglu ? (p.ldc % 2 == 0 && sb::aligned(p.c, 4)) : (p.ldc % 4 == 0 && sb::aligned(p.c, 8)));
  const size_t items = v4 ? total / 4 : total;
  const int grid = static_cast<int>(std::min<size_t>((items + 255) / 256, static_cast<size_t>(sb::num_sms()) * 16));
  cudaError_t e = v4 ? sb::launch_pdl(splitk_finalize_v4_kernel, dim3(grid), dim3(256), 0, s,
                                      static_cast<const float*>(p.ws), static_cast<__half*>(p.c), p.m, p.n, p.ldc,
                                      splits, p.alpha, p.geglu)
                     : sb::launch_pdl(splitk_finalize_kernel, dim3(grid), dim3(256), 0, s,
                                      static_cast<const float*>(p.ws), static_cast<__half*>(p.c), p.m, p.n, p.ldc,
                                      splits, p.alpha, p.geglu);
  if (e != cudaSuccess) return sb::cuda_fail(e, "splitk_finalize_kernel");
  return sb::launch_status("splitk_finalize_kernel");
}

}  // namespace

// Splits of one tile reduce through distributed shared memory when they fit in
// a cluster (portable size 8); more splits fall back to f32 partial planes in
// a workspace and splitk_finalize_kernel.
constexpr int kMaxClusterSplits = 8;

// The int4 GEMM runs as CTA pairs when a matrix has at least two weight tiles.
static bool q4_pair(int n) { return (n + QW - 1) / QW >= 2; }
// Largest split count reduced inside one cluster (clusters hold <= 8 CTAs).
static int q4_max_cluster_splits(int n) { return q4_pair(n) ? kMaxClusterSplits / 2 : kMaxClusterSplits; }

// How many clusters of the int4 GEMM (a CTA pair, or a single CTA, times
// `csplit` K splits) the device can hold at once (clusters live within one
// GPC, so this is below sm_count / cluster size); cached per device.
static int max_active_clusters(bool pair, int csplit) {
  static int cache[64][2][kMaxClusterSplits + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || csplit < 1 || csplit > kMaxClusterSplits) return 0;
  int& slot = cache[dev][pair ? 1 : 0][csplit];
  if (!slot) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pair ? 2 : 1, 1, csplit);
    cfg.blockDim = dim3((pair ? P_WARPS : Q_WARPS) * 32);
    cfg.dynamicSmemBytes = pair ? P_SMEM : Q_SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = pair ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = static_cast<unsigned>(csplit);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nclus = 0;
    // (every code width and token tile uses the same resources)
    cudaError_t e = pair ? cudaFuncSetAttribute(gemm_q4_pair_kernel<4, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                P_SMEM)
                         : cudaFuncSetAttribute(gemm_q4_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q_SMEM);
    if (e == cudaSuccess)
      e = pair ? cudaOccupancyMaxActiveClusters(&nclus, gemm_q4_pair_kernel<4, QT>, &cfg)
               : cudaOccupancyMaxActiveClusters(&nclus, gemm_q4_kernel<4>, &cfg);
    if (e != cudaSuccess) {
      cudaGetLastError();
      nclus = 0;
    }
    slot = nclus;
  }
  return slot;
}

static size_t q4_workspace(int m, int n, int k, int group, int scale_bytes) {
  if (m <= 0 || n <= 0 || k <= 0 || k % BK || group <= 0) return 0;
  const int splits = q4_splits(m, n, k, group, scale_bytes);
  return splits > q4_max_cluster_splits(n) ? static_cast<size_t>(splits) * m * n * sizeof(float) : 0;
}

extern "C" size_t sb_gemm_q4_workspace_size(int m, int n, int k) {
  // for the group-32 f16 scales of the benchmark format
  return q4_workspace(m, n, k, 32, 2);
}

extern "C" int sb_gemm_q4_kernels(int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0 || k % BK) return 0;
  return q4_splits(m, n, k, 32, 2) > q4_max_cluster_splits(n) ? 2 : 1;
}

static int gemm_f16_impl(const void* a, const void* b, void* c, int c_f32, int m, int n, int k, float alpha, int tr,
                         int lda, int ldb, int ldc, void* stream, int splits = 1) {
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
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.plane = static_cast<long long>(m) * ldc;
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

extern "C" int sb_gemm_f16_f32out_splitk(const void* a, const void* b, float* c, int m, int n, int k, float alpha,
                                         int tr, int lda, int ldb, int ldc, int splits, void* stream) {
  SB_CHECK_ARG(splits >= 1 && k > 0 && splits <= (k + BK - 1) / BK,
               "sb_gemm_f16_f32out_splitk: splits=%d must be in 1..ceil(k/%d)", splits, BK);
  SB_CHECK_ARG(((k + BK - 1) / BK) % splits == 0, "sb_gemm_f16_f32out_splitk: splits must divide ceil(k/%d)", BK);
  if (c && !sb::aligned(c, 4)) return sb::fail(SB_ERR_ALIGN, "sb_gemm_f16_f32out_splitk: C must be 4-byte aligned");
  return gemm_f16_impl(a, b, c, 1, m, n, k, alpha, tr, lda, ldb, ldc, stream, splits);
}

// Raises the pair kernel's shared-memory limit once per (instantiation, device)
// and launches it with `cfg` (cluster and programmatic-serialisation attributes).
template <int BITS, int NT>
static cudaError_t launch_pair(cudaLaunchConfig_t& cfg, const CUtensorMap& tact, const CUtensorMap& tw,
                               const GemmParams& p) {
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !done[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_q4_pair_kernel<BITS, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) done[dev] = true;
  }
  return cudaLaunchKernelEx(&cfg, gemm_q4_pair_kernel<BITS, NT>, tact, tw, p);
}

template <int BITS>
static cudaError_t launch_persist(cudaLaunchConfig_t& cfg, const CUtensorMap& tact, const CUtensorMap& tw,
                                  const GemmParams& p) {
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !done[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_q4_persist_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) done[dev] = true;
  }
  return cudaLaunchKernelEx(&cfg, gemm_q4_persist_kernel<BITS>, tact, tw, p);
}

// Profiling buffer of sb_gemm_q4_trace (null: off) and its size in stamps.
static unsigned long long* g_trace = nullptr;
static size_t g_trace_slots = 0;

static int gemm_q4_impl(const void* a, const void* w, const void* scales, int scale_dtype, int group, void* c, int m,
                        int n, int k, float alpha, int lda, int ldc, void* workspace, size_t workspace_bytes,
                        void* stream, int geglu, uint64_t* keys = nullptr, long long row_offset = 0, int bits = 4) {
  SB_CHECK_ARG(m >= 0 && n >= 0 && k > 0, "sb_gemm_q4: bad shape");
  SB_CHECK_ARG(!geglu || n % 2 == 0, "sb_gemm_q4_geglu: n=%d must be even (interleaved gate/up rows)", n);
  SB_CHECK_ARG(k % 64 == 0, "sb_gemm_q4: k=%d must be a multiple of 64", k);
  SB_CHECK_ARG(group > 0 && k % group == 0 && group % 32 == 0, "sb_gemm_q4: group=%d must be a multiple of 32 dividing k",
               group);
  SB_CHECK_ARG(scale_dtype == SB_SCALE_F16 || scale_dtype == SB_SCALE_F32, "sb_gemm_q4: bad scale dtype");
  if (m == 0 || n == 0) return SB_OK;
  SB_CHECK_ARG(a && w && scales && (c || keys), "sb_gemm_q4: null pointer");
  SB_CHECK_ARG(lda >= k && (keys || ldc >= (geglu ? n / 2 : n)), "sb_gemm_q4: leading dimension too small");
  if (!sb::aligned(a, 16) || !sb::aligned(w, 16) || (c && !sb::aligned(c, 2)) || lda % 8)
    return sb::fail(SB_ERR_ALIGN, "sb_gemm_q4: A and W must be 16-byte aligned with lda a multiple of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int esz = scale_dtype == SB_SCALE_F16 ? 2 : 4;
  CUtensorMap tact, tw;
  const bool pair = q4_pair(n);
  const int max_cs = q4_max_cluster_splits(n);
  // Tokens per pair (the MMA's N): 256, or for a short batch the smallest of
  // 64 / 128 that holds it -- the MMAs then take a quarter / half of the time.
  const int nt = !pair ? QT : (m <= 64 ? 64 : (m <= 128 ? 128 : QT));
  // a CTA of a pair loads half of the pair's activation tile
  int rc = make_map(&tact, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, k, m, lda, BK, pair ? nt / 2 : QT,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // packed weight [n, k * bits / 8] u8; a box is one k-block of QW rows
  rc = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, k * bits / 8, n, k * bits / 8, BK * bits / 8, QW,
                CU_TENSOR_MAP_SWIZZLE_NONE);
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
  p.geglu = geglu;
  p.keys = reinterpret_cast<unsigned long long*>(keys);
  p.row_offset = row_offset;
  p.bits = bits;
  p.kb_total = k / BK;
  // the argmax epilogue needs whole sums: no K split
  int splits = keys ? 1 : q4_splits(m, n, k, group, esz);
  const size_t need = splits > max_cs ? static_cast<size_t>(splits) * m * n * sizeof(float) : 0;
  if (need && (!workspace || workspace_bytes < need)) {
    // without room for partial sums use the largest cluster split instead
    splits = max_cs;
    if (QW * q4_scale_groups((k / BK + splits - 1) / splits, group) * esz > Q_SCALE_BYTES)
      return sb::fail(SB_ERR_WORKSPACE, "sb_gemm_q4: k=%d needs split-K (%zu workspace bytes) for its scales", k, need);
  }
  if (keys) {
    if (QW * q4_scale_groups(k / BK, group) * esz > Q_SCALE_BYTES)
      return sb::fail(SB_ERR_ARG, "sb_gemm_q4_argmax: k=%d has too many scale groups for one split", k);
    rc = sb::zero_keys(reinterpret_cast<unsigned long long*>(keys), m, s);
    if (rc != SB_OK) return rc;
  }
  // More 256 x 256 tiles than the device holds CTA pairs: the persistent
  // kernel (one launch wave; a tile's epilogue overlaps the next tile's MMAs)
  const int pt_pairs = pair && nt == QT && !keys ? max_active_clusters(true, 1) : 0;
  const int pt_tiles = ((n + 2 * QW - 1) / (2 * QW)) * ((m + QT - 1) / QT);
  if (pt_pairs > 0 && pt_tiles > pt_pairs) {
    int kbc = p.kb_total;  // k-blocks per scale tile
    while (kbc > 1 && QW * q4_scale_groups(kbc, group) * esz > Q_SCALE_BYTES) --kbc;
    const int gpk = group > BK ? group / BK : 1;  // scale tiles start on group boundaries
    kbc = std::max(gpk, kbc / gpk * gpk);
    if (kbc >= P_STAGES || kbc >= p.kb_total) {
      p.pt_pairs = pt_pairs;
      p.pt_wtp = (n + 2 * QW - 1) / (2 * QW);
      p.pt_ttiles = (m + QT - 1) / QT;
      p.pt_kbc = kbc;
      if (g_trace && static_cast<size_t>(2) * pt_pairs * kTraceSlots <= g_trace_slots) p.trace = g_trace;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, pt_pairs, 1);
      cfg.blockDim = dim3(P_WARPS * 32);
      cfg.dynamicSmemBytes = P_SMEM;
      cfg.stream = s;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      const cudaError_t e = bits == 2 ? launch_persist<2>(cfg, tact, tw, p) : launch_persist<4>(cfg, tact, tw, p);
      if (e != cudaSuccess) return sb::cuda_fail(e, "gemm_q4_persist_kernel (cluster launch)");
      return sb::launch_status("gemm_q4_persist_kernel");
    }
  }
  if (!pair) {
    static bool done[2][64] = {};
    rc = bits == 2 ? set_smem(gemm_q4_kernel<2>, Q_SMEM, done[1]) : set_smem(gemm_q4_kernel<4>, Q_SMEM, done[0]);
    if (rc) return rc;
  }
  const int wtiles = (n + QW - 1) / QW;
  const int gx = pair ? (wtiles + 1) / 2 * 2 : wtiles;  // a pair's second tile may lie past n
  const int ttiles = (m + nt - 1) / nt;
  const int clusters = (pair ? gx / 2 : gx) * ttiles;  // per split
  // a cluster split pays off only if all its clusters are resident at once;
  // otherwise use fewer splits (while the group scales of a split still fit)
  while (splits > 1 && splits <= max_cs && clusters > max_active_clusters(pair, splits)) {
    const int fewer = splits - 1;
    if (QW * q4_scale_groups((k / BK + fewer - 1) / fewer, group) * esz > Q_SCALE_BYTES) break;
    splits = fewer;
  }
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  const bool in_cluster = splits > 1 && splits <= max_cs;
  if (in_cluster) p.csplit = splits;
  else if (splits > 1) p.ws = static_cast<float*>(workspace);
  const dim3 grid(gx, ttiles, splits);
  if (pair && g_trace && static_cast<size_t>(grid.x) * grid.y * grid.z * kTraceSlots <= g_trace_slots) p.trace = g_trace;
  if (pair || in_cluster) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3((pair ? P_WARPS : Q_WARPS) * 32);
    cfg.dynamicSmemBytes = pair ? P_SMEM : Q_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = pair ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = in_cluster ? static_cast<unsigned>(splits) : 1u;
    // the pair kernel reads the activations only after griddepcontrol.wait, so
    // its set-up and weight stream may overlap the previous kernel's tail
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pair ? 2 : 1;
    cudaError_t e;
    if (pair) {
      const int which = (bits == 2 ? 3 : 0) + (nt == 64 ? 0 : nt == 128 ? 1 : 2);
      switch (which) {
        case 0: e = launch_pair<4, 64>(cfg, tact, tw, p); break;
        case 1: e = launch_pair<4, 128>(cfg, tact, tw, p); break;
        case 2: e = launch_pair<4, QT>(cfg, tact, tw, p); break;
        case 3: e = launch_pair<2, 64>(cfg, tact, tw, p); break;
        case 4: e = launch_pair<2, 128>(cfg, tact, tw, p); break;
        default: e = launch_pair<2, QT>(cfg, tact, tw, p); break;
      }
    } else {
      e = bits == 2 ? cudaLaunchKernelEx(&cfg, gemm_q4_kernel<2>, tact, tw, p)
                    : cudaLaunchKernelEx(&cfg, gemm_q4_kernel<4>, tact, tw, p);
    }
    if (e != cudaSuccess) return sb::cuda_fail(e, "gemm_q4 (cluster launch)");
    rc = sb::launch_status(pair ? "gemm_q4_pair_kernel" : "gemm_q4_kernel");
  } else {
    if (bits == 2) gemm_q4_kernel<2><<<grid, Q_WARPS * 32, Q_SMEM, s>>>(tact, tw, p);
    else gemm_q4_kernel<4><<<grid, Q_WARPS * 32, Q_SMEM, s>>>(tact, tw, p);
    rc = sb::launch_status("gemm_q4_kernel");
  }
  if (rc != SB_OK || in_cluster || splits == 1) return rc;
  return finalize(p, splits, s);
}

extern "C" int sb_gemm_q4_trace(uint64_t* buf, size_t bytes) {
  SB_CHECK_ARG(!buf || sb::aligned(buf, 8), "sb_gemm_q4_trace: buffer must be 8-byte aligned");
  g_trace = buf ? reinterpret_cast<unsigned long long*>(buf) : nullptr;
  g_trace_slots = buf ? bytes / sizeof(uint64_t) : 0;
  return SB_OK;
}

extern "C" int sb_gemm_q4(const void* a, const void* w, const void* scales, int scale_dtype, int group, void* c, int m,
                          int n, int k, float alpha, int lda, int ldc, void* workspace, size_t workspace_bytes,
                          void* stream) {
  return gemm_q4_impl(a, w, scales, scale_dtype, group, c, m, n, k, alpha, lda, ldc, workspace, workspace_bytes,
                      stream, 0);
}

extern "C" int sb_gemm_q4_argmax(const void* a, const void* w, const void* scales, int scale_dtype, int group, int m,
                                 int n, int k, float alpha, int lda, int64_t row_offset, uint64_t* keys, int32_t* tokens,
                                 void* stream) {
  SB_CHECK_ARG(keys != nullptr, "sb_gemm_q4_argmax: null keys");
  SB_CHECK_ARG(n <= 0 || row_offset + n <= (1ll << 32) - 1, "sb_gemm_q4_argmax: row indices exceed 32 bits");
  const int rc = gemm_q4_impl(a, w, scales, scale_dtype, group, nullptr, m, n, k, alpha, lda, 0, nullptr, 0, stream, 0,
                              keys, row_offset);
  if (rc != SB_OK || !tokens || m == 0) return rc;
  return sb_keys_to_tokens(keys, tokens, m, stream);
}

extern "C" int sb_gemm_q4_geglu(const void* a, const void* w, const void* scales, int scale_dtype, int group,
                                void* out, int m, int n, int k, float alpha, int lda, int ldo, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return gemm_q4_impl(a, w, scales, scale_dtype, group, out, m, n, k, alpha, lda, ldo, workspace, workspace_bytes,
                      stream, 1);
}

// The fused GEMM over 2-bit codes (the checkpoint's 2-bit MLP weights of
// layers 15+): W [n, k/4] u8, four codes per byte, value = code - 2.
extern "C" int sb_gemm_q2(const void* a, const void* w, const void* scales, int scale_dtype, int group, void* c, int m,
                          int n, int k, float alpha, int lda, int ldc, void* workspace, size_t workspace_bytes,
                          void* stream) {
  return gemm_q4_impl(a, w, scales, scale_dtype, group, c, m, n, k, alpha, lda, ldc, workspace, workspace_bytes,
                      stream, 0, nullptr, 0, 2);
}

extern "C" int sb_gemm_q2_geglu(const void* a, const void* w, const void* scales, int scale_dtype, int group,
                                void* out, int m, int n, int k, float alpha, int lda, int ldo, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return gemm_q4_impl(a, w, scales, scale_dtype, group, out, m, n, k, alpha, lda, ldo, workspace, workspace_bytes,
                      stream, 1, nullptr, 0, 2);
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
  // the split count depends on the scale tile's bytes: size the scratch for
  // this call's group and scale type, not the benchmark format's
  const size_t need = q4_workspace(m, n, k, group, scale_dtype == SB_F16 ? 2 : 4);
  if (need > kNoAllocScratchBytes)
    return sb::fail(SB_ERR_WORKSPACE,
                    "sb_gemm_q4_noalloc: m=%d n=%d k=%d group=%d needs %zu bytes of split-K scratch, more than "
                    "the %zu-byte static scratch; use sb_gemm_q4 with a caller workspace",
                    m, n, k, group, need, kNoAllocScratchBytes);
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
