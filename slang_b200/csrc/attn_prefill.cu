// Fused causal prefill attention on tcgen05 (sb_attn_prefill): one kernel for
// softmax(q k^T) v over a prompt, replacing the three-kernel chain (f32 score
// GEMM, causal softmax, P.V GEMM) and its S x S x n_heads score round trip
// through HBM.
//
// Shapes: q [S * nh rows][D] f16 with row = token * nh + head (every query
// head shares the single K/V head), k, v [S][D] f16, out [S * nh][D] f16,
// D = head_dim in {64, 128, 256} (a template parameter).
// Scores are unscaled (q and k are RMS-normalised upstream) and causal: row
// (t, h) sees keys 0..t.
//
// A CTA owns 128 query rows (16 tokens x 8 heads for Gemma-4-E2B) and walks
// the key blocks of 64 keys that they can see:
//   warp 0      TMA: the Q tile [128 x D] once, then K_j and V_j (each
//               [64 keys x D], 128B-swizzled boxes of 64 columns) into a
//               two-deep ring.
//   warp 1      one thread issues tcgen05.mma: S_j = Q K_j^T (M 128, N 64,
//               D/16 k-steps, A and B from shared memory) into a two-deep ring
//               of 64-column TMEM score buffers, then O += P_j V_j (M 128, N D,
//               K 64; P_j from TMEM, V_j MN-major from shared memory) into D
//               accumulator columns.  S_{j+1} is issued before O += P_j V_j so
//               the softmax of block j+1 overlaps the P.V MMAs of block j.
//   warps 2..9  softmax, two warps per TMEM lane quadrant (a thread per query
//               row in each): both read the row's 64 scores of S_j and take
//               the same masked maximum; each forms p = 2^(s log2 e - m) in f16
//               for its 32 keys with a running maximum m that is raised --
//               rescaling its half of O and its part of the row sum by
//               2^(m_old - m) -- only when the block maximum exceeds it by more
//               than 2^14, so O is touched rarely and p stays below 2^14 (f16
//               holds it); writes its 16 columns of P_j into TMEM for the MMA.
//               At the end the two halves' row sums are added through shared
//               memory and each warp writes O / (row sum) for its half of the
//               head dimension.
// TMEM: O [0, D), S ring [D, D + 128), P ring [D + 128, D + 192).
//
// Every mbarrier wait is bounded (2 s of %globaltimer); a stuck pipeline
// raises a shared abort flag, records SB_ERR_TIMEOUT and unwinds.  No TMA
// multicast is used.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "tmap.cuh"

namespace {

constexpr int QR = 128;  // query rows per CTA
constexpr int KB = 64;   // keys per block
constexpr int WARPS = 10;  // TMA, MMA, 8 softmax

template <int HD>
struct Cfg {
  static constexpr int Q_BYTES = QR * HD * 2;   // HD/64 boxes [128 rows x 64 cols]
  static constexpr int KV_BYTES = KB * HD * 2;  // HD/64 boxes [64 keys x 64 cols]
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + 2 * KV_BYTES;
  static constexpr int OFF_L = OFF_BAR + 256;           // the two halves' row sums [2][QR] f32
  static constexpr int SMEM = OFF_L + 2 * QR * 4 + 1024;  // + 1 KB alignment slack
  static constexpr uint32_t TM_O = 0, TM_S = HD, TM_P = HD + 2 * KB;
  static constexpr uint32_t TM_COLS = HD + 3 * KB <= 256 ? 256 : 512;
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 14.f;  // log2 units: p < 2^14 fits f16

// 2^x by the SFU (ex2.approx, flush-to-zero): p is rounded to f16 right after.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Bars {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_free[2], p_full[2], p_free[2];
  uint64_t o_final;
  uint64_t drain;
  uint32_t tmem_slot;
  int abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

// A split tile's partial row: O [HD], m (log2 units), l, 2 pad floats, so
// that every row starts on a 16-byte boundary.
template <int HD>
constexpr int part_stride() {
  return HD + 4;
}

struct Params {
  __half* out;
  float* part;  // split tiles: per (tile, chunk, row) a partial row of part_stride<HD>() floats
  int* err;
  int rows;   // S * nh
  int nh;
  int s_len;  // S (keys = queries' tokens)
  int kpc;    // key blocks per chunk (a CTA's share of a tile's key range)
  int maxc;   // chunks of the longest tile (grid.y)
  unsigned long long* trace;  // profiling only: kAttnTraceSlots %globaltimer stamps per CTA, or null
};

// Profiling stamps (sb_attn_prefill_trace): slot i of CTA b (linear grid index)
// is trace[b * kAttnTraceSlots + i].
enum {
  AT_SMID = 0,      // the SM the CTA ran on
  AT_ENTRY = 1,     // first instruction
  AT_SETUP = 2,     // barriers initialised, TMEM allocated
  AT_QFULL = 3,     // MMA issuer: the Q tile landed
  AT_OFINAL = 4,    // softmax warp 2: O final (the last P.V done)
  AT_EPI_END = 5,   // softmax warp 2: output or partial stores issued
  AT_EXIT = 6,      // TMEM released
  AT_NB = 7,        // key blocks of this CTA (a count, not a time)
  AT_S0 = 8,        // softmax warp 2: S_j readable (j = 0..7 at slots 8..15)
  AT_P0 = 16,       // softmax warp 2: P_j written (slots 16..23)
  kAttnTraceSlots = 24
};
__device__ __forceinline__ void attn_stamp(const Params& p, int slot) {
  if (p.trace) p.trace[(blockIdx.x + static_cast<size_t>(gridDim.x) * blockIdx.y) * kAttnTraceSlots + slot] = sbd::global_ns();
}

// Key blocks that query tile `tile` sees.
__host__ __device__ __forceinline__ int tile_key_blocks(int tile, int rows, int nh, int s_len) {
  const int r0 = tile * QR;
  const int last = (r0 + QR < rows ? r0 + QR : rows) - 1;
  const int tok_hi = (last / nh < s_len - 1) ? last / nh : s_len - 1;
  return tok_hi / KB + 1;
}

__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = sbd::global_ns();
  while (!sbd::mbar_try_wait(bar, parity)) {
    if (sbd::global_ns() - t0 > sbd::kWaitLimitNs) return false;
  }
  return true;
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  sbd::tmem_st_32x32b_x16(taddr, *reinterpret_cast<const uint32_t(*)[16]>(&r[0]));
  sbd::tmem_st_32x32b_x16(taddr + 16, *reinterpret_cast<const uint32_t(*)[16]>(&r[16]));
}

template <int HD>
__global__ void __launch_bounds__(WARPS * 32, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<HD>;
  constexpr int Q_BYTES = C::Q_BYTES, KV_BYTES = C::KV_BYTES, OFF_K = C::OFF_K, OFF_V = C::OFF_V;
  constexpr int OFF_BAR = C::OFF_BAR;
  constexpr uint32_t TM_O = C::TM_O, TM_S = C::TM_S, TM_P = C::TM_P, TM_COLS = C::TM_COLS;
  constexpr int NBOX = HD / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the next kernel may start its set-up; this one reads q, k, v (the previous
  // kernel's output) only after griddepcontrol.wait in the TMA warp
  sbd::griddep_launch_dependents();
  // heaviest tiles (latest tokens) first; chunk blockIdx.y of the tile's key blocks
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int r0 = tile * QR;
  const int nb_all = tile_key_blocks(tile, p.rows, p.nh, p.s_len);
  const int nchunks = (nb_all + p.kpc - 1) / p.kpc;
  if (static_cast<int>(blockIdx.y) >= nchunks) return;  // the whole CTA, before any barrier
  const int kb_lo = blockIdx.y * p.kpc;
  const int nb = min(p.kpc, nb_all - kb_lo);  // key blocks of this chunk: kb_lo + [0, nb)
  if (threadIdx.x == 0 && p.trace) {
    attn_stamp(p, AT_ENTRY);
    uint32_t sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    const size_t b = blockIdx.x + static_cast<size_t>(gridDim.x) * blockIdx.y;
    p.trace[b * kAttnTraceSlots + AT_SMID] = sm;
    p.trace[b * kAttnTraceSlots + AT_NB] = static_cast<unsigned long long>(nb);
  }

  if (threadIdx.x == 0) {
    sbd::mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      sbd::mbar_init(&bars->k_full[i], 1);
      sbd::mbar_init(&bars->k_empty[i], 1);
      sbd::mbar_init(&bars->v_full[i], 1);
      sbd::mbar_init(&bars->v_empty[i], 1);
      sbd::mbar_init(&bars->s_full[i], 1);
      sbd::mbar_init(&bars->s_free[i], 8);
      sbd::mbar_init(&bars->p_full[i], 8);
      sbd::mbar_init(&bars->p_free[i], 1);
    }
    sbd::mbar_init(&bars->o_final, 1);
    sbd::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    sbd::prefetch_tmap(&tmQ);
    sbd::prefetch_tmap(&tmK);
    sbd::prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    sbd::tmem_alloc(&bars->tmem_slot, TM_COLS);
    sbd::tmem_relinquish();
  }
  sbd::tc_fence_before();
  __syncthreads();
  sbd::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;
  bool mma_issued = false;
  if (threadIdx.x == 0) attn_stamp(p, AT_SETUP);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued_k = 0, issued_v = 0;
      sbd::griddep_wait();
      sbd::mbar_arrive_expect_tx(&bars->q_full, Q_BYTES);
#pragma unroll
      for (int b = 0; b < NBOX; ++b) sbd::tma_load_2d(&tmQ, &bars->q_full, smem + b * (QR * 128), 64 * b, r0);
      for (int j = 0; j < nb; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!sbd::mbar_wait(&bars->k_empty[st], ph, abort, p.err)) break;
        sbd::mbar_arrive_expect_tx(&bars->k_full[st], KV_BYTES);
#pragma unroll
        for (int b = 0; b < NBOX; ++b)
          sbd::tma_load_2d(&tmK, &bars->k_full[st], smem + OFF_K + st * KV_BYTES + b * (KB * 128), 64 * b,
                           (kb_lo + j) * KB);
        issued_k = j + 1;
        if (!sbd::mbar_wait(&bars->v_empty[st], ph, abort, p.err)) break;
        sbd::mbar_arrive_expect_tx(&bars->v_full[st], KV_BYTES);
#pragma unroll
        for (int b = 0; b < NBOX; ++b)
          sbd::tma_load_2d(&tmV, &bars->v_full[st], smem + OFF_V + st * KV_BYTES + b * (KB * 128), 64 * b,
                           (kb_lo + j) * KB);
        issued_v = j + 1;
      }
      if (*abort) {
        // let copies in flight land before this CTA's shared memory is released
        drain_wait(&bars->q_full, 0);
        for (int j = max(0, issued_k - 2); j < issued_k; ++j) drain_wait(&bars->k_full[j & 1], (j >> 1) & 1);
        for (int j = max(0, issued_v - 2); j < issued_v; ++j) drain_wait(&bars->v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = sbd::umma_idesc_f16(QR, KB, 0, 0);
      constexpr uint32_t idesc_o = sbd::umma_idesc_f16(QR, HD, 0, 1);
      const uint32_t qbase = sbd::smem_u32(smem);
      bool ok = sbd::mbar_wait(&bars->q_full, 0, abort, p.err);
      attn_stamp(p, AT_QFULL);
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          // S_j = Q K_j^T
          const int st = j & 1;
          ok = sbd::mbar_wait(&bars->k_full[st], (j >> 1) & 1, abort, p.err) &&
               sbd::mbar_wait(&bars->s_free[st], ((j >> 1) & 1) ^ 1, abort, p.err);
          if (!ok) break;
          sbd::tc_fence_after();
          const uint32_t kbase = sbd::smem_u32(smem + OFF_K + st * KV_BYTES);
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint64_t adesc =
                sbd::umma_desc(qbase + (ks >> 2) * (QR * 128) + (ks & 3) * 32, 16, 1024, sbd::kLayoutSwizzle128B);
            const uint64_t bdesc =
                sbd::umma_desc(kbase + (ks >> 2) * (KB * 128) + (ks & 3) * 32, 16, 1024, sbd::kLayoutSwizzle128B);
            sbd::umma_f16(tmem + TM_S + st * KB, adesc, bdesc, idesc_s, ks > 0 ? 1u : 0u);
          }
          mma_issued = true;
          sbd::umma_commit(&bars->s_full[st]);
          sbd::umma_commit(&bars->k_empty[st]);
        }
        if (j >= 1) {
          // O += P_i V_i
          const int i = j - 1, st = i & 1;
          ok = sbd::mbar_wait(&bars->p_full[st], (i >> 1) & 1, abort, p.err) &&
               sbd::mbar_wait(&bars->v_full[st], (i >> 1) & 1, abort, p.err);
          if (!ok) break;
          sbd::tc_fence_after();
          const uint32_t vbase = sbd::smem_u32(smem + OFF_V + st * KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < KB / 16; ++kk) {
            const uint64_t bdesc = sbd::umma_desc(vbase + kk * 2048, KB * 128, 1024, sbd::kLayoutSwizzle128B);
            sbd::umma_f16_ts(tmem + TM_O, tmem + TM_P + st * 32 + kk * 8, bdesc, idesc_o,
                             (i > 0 || kk > 0) ? 1u : 0u);
          }
          sbd::umma_commit(&bars->p_free[st]);
          sbd::umma_commit(&bars->v_empty[st]);
        }
      }
      if (ok) sbd::umma_commit(&bars->o_final);
      if (mma_issued) {
        // every MMA issued has finished before TMEM is released
        sbd::umma_commit(&bars->drain);
        drain_wait(&bars->drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue (warps 2..9)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // keys [32 half, +32) of each block; O columns [HD/2 half, +HD/2)
    const int row = quad * 32 + lane;
    const int r = r0 + row;
    const bool row_ok = r < p.rows;
    const int token = row_ok ? r / p.nh : -1;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float m_used = 0.f, l = 0.f;  // l: this half's part of the row sum
    bool ok = true;
    for (int j = 0; j < nb && ok; ++j) {
      const int st = j & 1;
      ok = __all_sync(0xFFFFFFFFu, sbd::mbar_wait(&bars->s_full[st], (j >> 1) & 1, abort, p.err));
      if (!ok) break;
      sbd::tc_fence_after();
      uint32_t sv[2][32];
      if (threadIdx.x == 64 && j < 8) attn_stamp(p, AT_S0 + j);
      sbd::tmem_ld_32x32b_x32(lane_base + TM_S + st * KB, sv[0]);
      sbd::tmem_ld_32x32b_x32(lane_base + TM_S + st * KB + 32, sv[1]);
      sbd::tmem_wait_ld();
      sbd::tc_fence_before();
      __syncwarp();
      if (lane == 0) sbd::mbar_arrive(&bars->s_free[st]);
      // causal mask: key j*KB + c is visible to this row when it is <= token
      const int nvis = max(0, min(KB, token - (kb_lo + j) * KB + 1));
      // masked row maximum over all 64 keys (both halves compute the same one)
      float t[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float a = 2 * e < nvis ? __uint_as_float(sv[(2 * e) >> 5][(2 * e) & 31]) : -INFINITY;
        const float b = 2 * e + 1 < nvis ? __uint_as_float(sv[(2 * e + 1) >> 5][(2 * e + 1) & 31]) : -INFINITY;
        t[e] = fmaxf(a, b);
      }
#pragma unroll
      for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
        for (int e = 0; e < w; ++e) t[e] = fmaxf(t[e], t[e + w]);
      const float mx2 = t[0] * kLog2e;
      if (j == 0) {
        m_used = nvis > 0 ? mx2 : 0.f;
      } else {
        const bool need = nvis > 0 && mx2 > m_used + kRescale;
        if (__any_sync(0xFFFFFFFFu, need)) {
          // O must be quiet: wait for O += P_{j-1} V_{j-1}; each half rescales its columns
          ok = __all_sync(0xFFFFFFFFu,
                          sbd::mbar_wait(&bars->p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, abort, p.err));
          if (!ok) break;
          sbd::tc_fence_after();
          const float alpha = need ? ex2(m_used - mx2) : 1.f;
          for (int cc = 0; cc < HD / 64; ++cc) {
            uint32_t ov[32];
            const uint32_t col = TM_O + half * (HD / 2) + cc * 32;
            sbd::tmem_ld_32x32b_x32(lane_base + col, ov);
            sbd::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st_x32(lane_base + col, ov);
          }
          sbd::tmem_wait_st();
          l *= alpha;
          if (need) m_used = mx2;
        }
      }
      // p = 2^(s log2 e - m_used) in f16 for this half's 32 keys, two per TMEM column
      uint32_t pk[16];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int c = 32 * half + 2 * e;
        const uint32_t s0 = half ? sv[1][2 * e] : sv[0][2 * e];
        const uint32_t s1 = half ? sv[1][2 * e + 1] : sv[0][2 * e + 1];
        const float p0 = c < nvis ? ex2(__uint_as_float(s0) * kLog2e - m_used) : 0.f;
        const float p1 = c + 1 < nvis ? ex2(__uint_as_float(s1) * kLog2e - m_used) : 0.f;
        const __half2 h = __floats2half2_rn(p0, p1);
        const float2 hf = __half22float2(h);
        ls[e & 3] += hf.x + hf.y;
        pk[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // the P buffer is free once O += P_{j-2} V_{j-2} has run
      if (j >= 2) {
        ok = __all_sync(0xFFFFFFFFu, sbd::mbar_wait(&bars->p_free[st], ((j - 2) >> 1) & 1, abort, p.err));
        if (!ok) break;
        sbd::tc_fence_after();
      }
      sbd::tmem_st_32x32b_x16(lane_base + TM_P + st * 32 + half * 16, pk);
      sbd::tmem_wait_st();
      sbd::tc_fence_before();
      __syncwarp();
      if (lane == 0) sbd::mbar_arrive(&bars->p_full[st]);
      if (threadIdx.x == 64 && j < 8) attn_stamp(p, AT_P0 + j);
    }
    // ------------------------------------------------------------ epilogue: O / l -> f16
    if (ok) ok = __all_sync(0xFFFFFFFFu, sbd::mbar_wait(&bars->o_final, 0, abort, p.err));
    if (threadIdx.x == 64) attn_stamp(p, AT_OFINAL);
    // the row sum is the two halves' parts (every softmax warp meets this barrier)
    float* lx = reinterpret_cast<float*>(smem + C::OFF_L);
    lx[half * QR + row] = l;
    sbd::named_bar_sync(1, 8 * 32);
    const float l_row = lx[row] + lx[QR + row];
    if (nchunks > 1) {
      // A share of a split tile: unnormalised O with its running max and sum.
      // The tile's 128 partial rows are one contiguous block of the
      // workspace, so they are laid out in shared memory (the Q / K / V
      // buffers are idle now: every MMA completed before o_final) and written
      // with one bulk copy -- stores of a thread's own row from registers
      // would scatter across 32 rows per instruction.
      constexpr int PS = part_stride<HD>();
      static_assert(QR * PS * 4 <= OFF_V + 2 * KV_BYTES, "the partial tile must fit the Q / K / V buffers");
      float* stile = reinterpret_cast<float*>(smem);
      sbd::tc_fence_after();
      // two 32-column TMEM loads in flight per wait
      for (int cc = 0; cc < HD / 64; cc += 2) {
        uint32_t ov[2][32];
        sbd::tmem_ld_32x32b_x32(lane_base + TM_O + half * (HD / 2) + cc * 32, ov[0]);
        if (cc + 1 < HD / 64) sbd::tmem_ld_32x32b_x32(lane_base + TM_O + half * (HD / 2) + cc * 32 + 32, ov[1]);
        sbd::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (cc + u >= HD / 64) break;
          const int col = half * (HD / 2) + (cc + u) * 32;
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(stile + row * PS + col + e) =
                make_float4(__uint_as_float(ov[u][e]), __uint_as_float(ov[u][e + 1]), __uint_as_float(ov[u][e + 2]),
                            __uint_as_float(ov[u][e + 3]));
        }
      }
      if (half == 0)
        *reinterpret_cast<float4*>(stile + row * PS + HD) = make_float4(m_used, l_row, 0.f, 0.f);
      sbd::fence_proxy_async_smem();  // these generic-proxy writes feed the bulk copy
      // each lane quadrant's 32 rows (its two warps) go out as soon as both wrote them
      sbd::named_bar_sync(2 + quad, 2 * 32);
      if (half == 0 && lane == 0 && ok) {
        const size_t rq = static_cast<size_t>(quad) * 32 * PS;
        float* dst = p.part + (static_cast<size_t>(tile) * p.maxc + blockIdx.y) * QR * PS + rq;
        sbd::bulk_store(dst, stile + rq, 32 * PS * 4);
        sbd::bulk_store_wait_read();  // before the CTA's shared memory is released
      }
    } else if (ok) {
      sbd::tc_fence_after();
      const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
      __half* dst = p.out + static_cast<size_t>(r) * HD;
      for (int cc = 0; cc < HD / 64; ++cc) {
        const int col = half * (HD / 2) + cc * 32;
        uint32_t ov[32];
        sbd::tmem_ld_32x32b_x32(lane_base + TM_O + col, ov);
        sbd::tmem_wait_ld();
        if (!row_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint32_t o4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const __half2 h = __floats2half2_rn(__uint_as_float(ov[e + 2 * q]) * inv,
                                                __uint_as_float(ov[e + 2 * q + 1]) * inv);
            o4[q] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(dst + col + e) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
        }
      }
    }
    if (threadIdx.x == 64) attn_stamp(p, AT_EPI_END);
  }

  sbd::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sbd::tc_fence_after();
    sbd::tmem_dealloc(tmem, TM_COLS);
    if (lane == 0) attn_stamp(p, AT_EXIT);
  }
}

// Combines the chunk partials of every split tile: warp per query row,
// out = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c over chunks that saw
// keys (l_c > 0), M the largest of their m_c.
template <int HD>
__global__ void attn_merge_kernel(const float* __restrict__ part, __half* __restrict__ out, int rows, int nh,
                                  int s_len, int kpc, int maxc) {
  constexpr int VPL = HD / 32;  // values per lane: 2, 4 or 8
  constexpr int PS = part_stride<HD>();
  static_assert(VPL == 2 || VPL % 4 == 0, "lane vector width");
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int tile = blockIdx.x;
  const int row = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int nchunks = (tile_key_blocks(tile, rows, nh, s_len) + kpc - 1) / kpc;
  const int r = tile * QR + row;
  if (nchunks <= 1 || r >= rows) return;
  const size_t cstride = static_cast<size_t>(QR) * PS;
  const float* base = part + (static_cast<size_t>(tile) * maxc * QR + row) * PS;
  float M = -INFINITY;
  for (int c = 0; c < nchunks; ++c)
    if (base[c * cstride + HD + 1] > 0.f) M = fmaxf(M, base[c * cstride + HD]);
  float acc[VPL] = {};
  float L = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    const float* pc = base + c * cstride + lane * VPL;  // 8 * VPL bytes per lane: aligned for its vector width
    const float lc = base[c * cstride + HD + 1];
    if (!(lc > 0.f)) continue;
    const float wgt = exp2f(base[c * cstride + HD] - M);
    L += wgt * lc;
    if constexpr (VPL == 2) {
      const float2 v = *reinterpret_cast<const float2*>(pc);
      acc[0] += wgt * v.x;
      acc[1] += wgt * v.y;
    } else {
#pragma unroll
      for (int e = 0; e < VPL; e += 4) {
        const float4 v = *reinterpret_cast<const float4*>(pc + e);
        acc[e] += wgt * v.x;
        acc[e + 1] += wgt * v.y;
        acc[e + 2] += wgt * v.z;
        acc[e + 3] += wgt * v.w;
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  __half* dst = out + static_cast<size_t>(r) * HD + lane * VPL;
#pragma unroll
  for (int e = 0; e < VPL; e += 2) *reinterpret_cast<__half2*>(dst + e) = __floats2half2_rn(acc[e] * inv, acc[e + 1] * inv);
}

// Key blocks per chunk: the fewest that keep the CTAs (tile x chunk) within
// one wave of the SMs, so the longest chain of key blocks is as short as the
// machine allows.  Returns kpc and sets *maxc.
int choose_kpc(int rows, int nh, int s_len, int* maxc) {
  const int tiles = (rows + QR - 1) / QR;
  const int nb_max = tile_key_blocks(tiles - 1, rows, nh, s_len);
  const int sms = sb::num_sms();
  int kpc = 1;
  for (; kpc < nb_max; ++kpc) {
    long long ctas = 0;
    for (int t = 0; t < tiles; ++t) ctas += (tile_key_blocks(t, rows, nh, s_len) + kpc - 1) / kpc;
    if (ctas <= sms) break;
  }
  *maxc = (nb_max + kpc - 1) / kpc;
  return kpc;
}

// Profiling buffer of sb_attn_prefill_trace (null: off) and its size in stamps.
static unsigned long long* g_attn_trace = nullptr;
static size_t g_attn_trace_slots = 0;

template <int HD>
int launch_attn(const void* q16, const void* k16, const void* v16, void* out16, int s_len, int n_heads, float* part,
                size_t part_bytes, cudaStream_t stream) {
  using C = Cfg<HD>;
  const long long rows = static_cast<long long>(s_len) * n_heads;
  CUtensorMap tq, tk, tv;
  int rc = sb::make_map(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, q16, HD, rows, HD, 64, QR, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = sb::make_map(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, k16, HD, s_len, HD, 64, KB, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = sb::make_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, v16, HD, s_len, HD, 64, KB, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(attn_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return sb::cuda_fail(e, "attn_prefill_kernel smem attribute");
    done[dev] = true;
  }
  Params p{};
  p.out = static_cast<__half*>(out16);
  p.err = sb::device_error_word();
  p.rows = static_cast<int>(rows);
  p.nh = n_heads;
  p.s_len = s_len;
  const int tiles = static_cast<int>((rows + QR - 1) / QR);
  int maxc = 1;
  p.kpc = tile_key_blocks(tiles - 1, p.rows, n_heads, s_len);  // unsplit
  if (part) {
    const int kpc = choose_kpc(p.rows, n_heads, s_len, &maxc);
    if (maxc > 1 && static_cast<size_t>(tiles) * maxc * QR * part_stride<HD>() * sizeof(float) <= part_bytes) {
      p.kpc = kpc;
      p.part = part;
    } else {
      maxc = 1;
    }
  }
  p.maxc = maxc;
  if (g_attn_trace && static_cast<size_t>(tiles) * maxc * kAttnTraceSlots <= g_attn_trace_slots) p.trace = g_attn_trace;
  cudaError_t e = sb::launch_pdl(attn_prefill_kernel<HD>, dim3(tiles, maxc), dim3(WARPS * 32), C::SMEM, stream, tq,
                                 tk, tv, p);
  if (e != cudaSuccess) return sb::cuda_fail(e, "attn_prefill_kernel");
  rc = sb::launch_status("attn_prefill_kernel");
  if (rc != SB_OK || maxc == 1) return rc;
  e = sb::launch_pdl(attn_merge_kernel<HD>, dim3(tiles, QR / 8), dim3(256), 0, stream, static_cast<const float*>(part),
                     p.out, p.rows, n_heads, s_len, p.kpc, maxc);
  if (e != cudaSuccess) return sb::cuda_fail(e, "attn_merge_kernel");
  return sb::launch_status("attn_merge_kernel");
}

}  // namespace

static int attn_prefill_impl(const void* q16, const void* k16, const void* v16, void* out16, int s_len, int n_heads,
                             int head_dim, void* workspace, size_t workspace_bytes, void* stream) {
  SB_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256,
               "sb_attn_prefill: head_dim must be 64, 128 or 256");
  SB_CHECK_ARG(s_len >= 0 && n_heads >= 1, "sb_attn_prefill: bad sizes");
  if (s_len == 0) return SB_OK;
  SB_CHECK_ARG(q16 && k16 && v16 && out16, "sb_attn_prefill: null pointer");
  if (!sb::aligned(q16, 16) || !sb::aligned(k16, 16) || !sb::aligned(v16, 16) || !sb::aligned(out16, 16))
    return sb::fail(SB_ERR_ALIGN, "sb_attn_prefill: q, k, v and out must be 16-byte aligned");
  SB_CHECK_ARG(static_cast<long long>(s_len) * n_heads < (1ll << 31), "sb_attn_prefill: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  if (part && !sb::aligned(part, 16)) return sb::fail(SB_ERR_ALIGN, "sb_attn_prefill: workspace must be 16-byte aligned");
  switch (head_dim) {
    case 64: return launch_attn<64>(q16, k16, v16, out16, s_len, n_heads, part, workspace_bytes, s);
    case 128: return launch_attn<128>(q16, k16, v16, out16, s_len, n_heads, part, workspace_bytes, s);
    default: return launch_attn<256>(q16, k16, v16, out16, s_len, n_heads, part, workspace_bytes, s);
  }
}

extern "C" int sb_attn_prefill_trace(uint64_t* buf, size_t bytes) {
  SB_CHECK_ARG(!buf || sb::aligned(buf, 8), "sb_attn_prefill_trace: buffer must be 8-byte aligned");
  g_attn_trace = buf ? reinterpret_cast<unsigned long long*>(buf) : nullptr;
  g_attn_trace_slots = buf ? bytes / sizeof(uint64_t) : 0;
  return SB_OK;
}

extern "C" int sb_attn_prefill(const void* q16, const void* k16, const void* v16, void* out16, int s_len,
                               int n_heads, int head_dim, void* stream) {
  return attn_prefill_impl(q16, k16, v16, out16, s_len, n_heads, head_dim, nullptr, 0, stream);
}

extern "C" size_t sb_attn_prefill_workspace_size(int s_len, int n_heads, int head_dim) {
  if (s_len <= 0 || n_heads <= 0 || head_dim <= 0) return 0;
  const long long rows = static_cast<long long>(s_len) * n_heads;
  if (rows >= (1ll << 31)) return 0;
  int maxc = 1;
  choose_kpc(static_cast<int>(rows), n_heads, s_len, &maxc);
  if (maxc <= 1) return 0;
  const size_t tiles = static_cast<size_t>((rows + QR - 1) / QR);
  return tiles * maxc * QR * (static_cast<size_t>(head_dim) + 4) * sizeof(float);  // part_stride
}

extern "C" int sb_attn_prefill_ws(const void* q16, const void* k16, const void* v16, void* out16, int s_len,
                                  int n_heads, int head_dim, void* workspace, size_t workspace_bytes, void* stream) {
  return attn_prefill_impl(q16, k16, v16, out16, s_len, n_heads, head_dim, workspace, workspace_bytes, stream);
}
