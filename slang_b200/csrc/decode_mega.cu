// One greedy decode step of the Gemma-4-E2B-shaped int4 decoder for a single
// sequence as ONE persistent cooperative kernel (sb_decode_step_fused).
//
// Why: a step is ~35 x 10 small dependent operations; as separate launches the
// step is dominated by launch and ramp latency, not by the ~1 GB of weights
// it must stream.  Here every SM runs one CTA for the whole step:
//
//   producer warp   walks this CTA's fixed sequence of weight row-slices --
//                   per layer its rows of q|k|v, o, gate|up (rows interleaved
//                   gate/up), down, then its rows of the tied lm_head -- and
//                   streams them (packed rows + their f16 group scales) with
//                   cp.async.bulk into a 6-deep shared-memory ring.  Weights do
//                   not depend on activations, so the stream runs ahead across
//                   the phase barriers below.
//   8 consumer warps  run the phases, separated by grid-wide barriers:
//     qkv:    x = layer input (embedding, or residual + post-FFN RMSNorm of
//             the previous down output), h = RMSNorm(x) * in_norm, GEMV rows
//     attn:   per 32-key chunk (one chunk per CTA): q/k norm + RoPE (the last
//             chunk's CTA also writes k, v of this position to the cache),
//             scores, chunk softmax partials, P.V partials
//     merge:  per (head, 64 dims): rescale the chunk partials -> attention out
//     o:      GEMV rows of o over the attention output
//     gateup: x += RMSNorm(o) * post_attn, h = RMSNorm(x) * pre_ffn, GEMV rows,
//             GEGLU of each interleaved (gate, up) row pair
//     down:   GEMV rows of down over the GEGLU output
//   and finally RMSNorm * final_norm, the lm_head rows with a running
//   (max, lowest index) per CTA, one 64-bit atomicMax per CTA, and block 0
//   decodes the token and advances pos / cur / history.
//
// GEMV arithmetic is the exact int4 x int16 DP4A dot of q4_dot.cuh.  Every wait
// (mbarrier or grid barrier) is bounded by %globaltimer; a timeout raises a
// global abort flag that every CTA polls, writes SB_ERR_TIMEOUT to the device
// error word, and the kernel unwinds.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "q4_dot.cuh"

namespace {

constexpr int kCons = 256;            // consumer threads (8 warps)
constexpr int kThreads = kCons + 32;  // + one producer warp
constexpr int kRing = 6;
constexpr int kStageW = 24 * 1024;
constexpr int kStageS = 3 * 1024;
constexpr int kMaxK = 6144;           // longest GEMV row (values)
constexpr int HD = 256;               // head_dim handled by this kernel
constexpr int CKA = 32;               // keys per attention work item
constexpr int kMaxHeads = 8;
constexpr int kRed = 128;
constexpr int kSegOut = 512;          // rows of one CTA's gate|up slice kept for GEGLU
constexpr unsigned int kTraceLen = 512;  // [0] count, then timestamps

struct Layer {
  const uint8_t* w[4];  // 0 q|k|v [nqkv, H/2], 1 o [H, qd/2], 2 gate|up interleaved [2F, H/2], 3 down [H, F/2]
  const __half* s[4];   // matching [rows, K/32] f16 group scales
  const float* in_norm;
  const float* q_norm;
  const float* k_norm;
  const float* post_attn;
  const float* pre_ffn;
  const float* post_ffn;
  float* kc;  // [max_seq][HD]
  float* vc;
};

struct Params {
  const Layer* layers;
  int n_layers;
  const uint8_t* emb;
  const __half* emb_s;
  const float* final_norm;
  const float* cos_t;
  const float* sin_t;
  int H, nh, F, V, max_seq;
  float eps, embed_scale;
  int32_t* pos;
  int32_t* cur;
  int32_t* tok;
  int32_t* history;
  int hist_len;
  unsigned long long* keys;
  float *xa, *xb, *qkv, *attn, *o, *a, *d, *part;
  unsigned int* bar;  // [0] arrivals, [1] generation, [2] abort
  unsigned long long* trace;  // optional: block 0 stamps %globaltimer at entry and after each barrier
  int* err;
};

struct Smem {
  uint8_t w[kRing][kStageW];
  uint8_t s[kRing][kStageS];
  // [0, kMaxK): the phase input, stored transposed (element i at (i % 32) * G + i / 32);
  // [kMaxK, 2 kMaxK): a second vector.  The attention phase reuses both as scratch.
  float va[2 * kMaxK];
  float red[2][kRed];
  float seg_out[kSegOut];
  unsigned long long best[8];
  uint64_t full[kRing];
  uint64_t empty[kRing];
  int flag;
};

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
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
__device__ __forceinline__ void cons_sync() { sbd::named_bar_sync(1, kCons); }

// sum over the consumer threads
__device__ float cons_sum(float v, Smem& sm) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  cons_sync();
  if (lane == 0) sm.red[0][warp] = v;
  cons_sync();
  float t = lane < kCons / 32 ? sm.red[0][lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ bool aborted(const Params& p) {
  return *reinterpret_cast<volatile const unsigned int*>(p.bar + 2) != 0;
}

__device__ __forceinline__ void raise_abort(const Params& p) {
  atomicExch(p.bar + 2, 1u);
  atomicExch(p.err, SB_ERR_TIMEOUT);
}

// The global abort flag is an L2 round trip: poll it only once a wait has
// lasted this long, so normal waits wake up as soon as their condition holds.
constexpr uint64_t kAbortPollNs = 20000;

// mbarrier wait that also gives up when another CTA raised the global abort
__device__ bool ring_wait(uint64_t* bar, uint32_t parity, const Params& p) {
  if (sbd::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = sbd::global_ns();
  while (!sbd::mbar_try_wait(bar, parity)) {
    const uint64_t dt = sbd::global_ns() - t0;
    if (dt > kAbortPollNs && aborted(p)) return false;
    if (dt > sbd::kWaitLimitNs) {
      raise_abort(p);
      return false;
    }
  }
  return true;
}

// Grid-wide barrier among the consumer warps of every CTA (the producer warp
// never joins: it may be blocked on a ring slot the consumers will free only
// after this barrier).  Bounded spin; false when the step was aborted.
__device__ bool grid_sync(const Params& p, Smem& sm) {
  cons_sync();
  if (threadIdx.x == 0) {
    bool ok = !aborted(p);
    if (ok) {
      __threadfence();
      const unsigned int gen = ld_acquire(p.bar + 1);
      const unsigned int arrived = atomicAdd(p.bar, 1u);
      if (arrived == gridDim.x - 1) {
        atomicExch(p.bar, 0u);
        __threadfence();
        atomicAdd(p.bar + 1, 1u);
      } else {
        const uint64_t t0 = sbd::global_ns();
        while (ld_acquire(p.bar + 1) == gen) {
          const uint64_t dt = sbd::global_ns() - t0;
          if (dt > kAbortPollNs && aborted(p)) {
            ok = false;
            break;
          }
          if (dt > sbd::kWaitLimitNs) {
            raise_abort(p);
            ok = false;
            break;
          }
        }
      }
      __threadfence();
    }
    sm.flag = ok;
    if (p.trace && blockIdx.x == 0) {
      const unsigned int n = static_cast<unsigned int>(p.trace[0]) + 1;
      if (n < kTraceLen) {
        p.trace[n] = sbd::global_ns();
        p.trace[0] = n;
      }
    }
  }
  cons_sync();
  return sm.flag != 0;
}

// ---------------------------------------------------------------- weight segments
// This CTA's rows [r0, r1) of an N x K matrix and the rows per ring stage.
struct Seg {
  int r0, r1, rs;
};
__device__ __forceinline__ Seg segment(int n, int k) {
  int per = (n + gridDim.x - 1) / gridDim.x;
  per = (per + 1) & ~1;  // even: gate/up rows stay paired
  Seg s;
  s.r0 = min(n, static_cast<int>(blockIdx.x) * per);
  s.r1 = min(n, s.r0 + per);
  s.rs = max(1, min(per, kStageW / (k / 2)));
  s.rs = min(s.rs, kStageS / (k / 16));
  return s;
}

struct Plan {
  int gpl, ks;
};
__device__ __forceinline__ Plan plan_for(int k) {
  const int G = k / 32;
  Plan best{1, 16};
  int waste = 1 << 30;
  const int prefs[4] = {3, 2, 4, 1};
  for (int i = 0; i < 4; ++i) {
    int ks = 1;
    while (16 * prefs[i] * ks < G && ks < 16) ks *= 2;
    if (16 * prefs[i] * ks < G) continue;
    const int w = 16 * prefs[i] * ks - G;
    if (w < waste) {
      waste = w;
      best = {prefs[i], ks};
    }
  }
  return best;
}

// producer: stream one matrix's slice through the ring
__device__ bool produce(const Params& p, Smem& sm, const uint8_t* w, const __half* s, int n, int k, int& it) {
  const Seg sg = segment(n, k);
  const int rb = k / 2, sb = k / 16;
  for (int r = sg.r0; r < sg.r1; r += sg.rs) {
    const int nr = min(sg.rs, sg.r1 - r);
    const int slot = it % kRing;
    if (!ring_wait(&sm.empty[slot], ((it / kRing) & 1) ^ 1, p)) return false;
    sbd::mbar_arrive_expect_tx(&sm.full[slot], static_cast<uint32_t>(nr) * (rb + sb));
    sbd::bulk_load(sm.w[slot], w + static_cast<size_t>(r) * rb, static_cast<uint32_t>(nr) * rb, &sm.full[slot]);
    sbd::bulk_load(sm.s[slot], reinterpret_cast<const uint8_t*>(s) + static_cast<size_t>(r) * sb,
                   static_cast<uint32_t>(nr) * sb, &sm.full[slot]);
    ++it;
  }
  return true;
}

enum { EPI_STORE = 0, EPI_SEGOUT = 1, EPI_ARGMAX = 2 };

// consumers: GEMV of this CTA's rows of one matrix over sm.vec (transposed, K values)
template <int GPL, int EPI>
__device__ bool gemv_rows(const Params& p, Smem& sm, int n, int k, int ks, float* out, int& it, float& best_v,
                          long long& best_i) {
  const int tid = threadIdx.x, hw = tid >> 4, l16 = tid & 15;
  const int G = k / 32;
  const int SG = (G + ks - 1) / ks;
  const int kslice = hw % ks, rlane = hw / ks, nrl = 16 / ks;
  const int gb = kslice * SG, ge = min(G, gb + SG);
  sbd::XGroup xg[GPL];
  int gidx[GPL];
  bool gval[GPL];
#pragma unroll
  for (int u = 0; u < GPL; ++u) {
    gidx[u] = gb + l16 + 16 * u;
    gval[u] = gidx[u] < ge;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gval[u] ? sm.va[j * G + gidx[u]] : 0.f;
    sbd::quantise_group(v, xg[u]);
  }
  const Seg sg = segment(n, k);
  const int rb = k / 2;
  for (int r = sg.r0; r < sg.r1; r += sg.rs) {
    const int nr = min(sg.rs, sg.r1 - r);
    const int slot = it % kRing;
    const bool ok = ring_wait(&sm.full[slot], (it / kRing) & 1, p);
    if (!__all_sync(0xFFFFFFFFu, ok)) return false;
    float* red = sm.red[it & 1];
    const uint8_t* wst = sm.w[slot];
    const __half* sst = reinterpret_cast<const __half*>(sm.s[slot]);
    const int iters = (sg.rs + nrl - 1) / nrl;
    for (int t = 0; t < iters; ++t) {
      const int rr = rlane + t * nrl;
      float acc = 0.f;
      if (rr < nr) {
#pragma unroll
        for (int u = 0; u < GPL; ++u) {
          if (!gval[u]) continue;
          const uint4 q = *reinterpret_cast<const uint4*>(wst + rr * rb + gidx[u] * 16);
          const float sw = __half2float(sst[rr * G + gidx[u]]);
          acc = fmaf(static_cast<float>(sbd::dot_group(q, xg[u])), sw * xg[u].sx, acc);
        }
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off, 16);
      if (l16 == 0 && rr < nr) red[rr * ks + kslice] = acc;
    }
    __syncwarp();
    if ((tid & 31) == 0) sbd::mbar_arrive(&sm.empty[slot]);
    cons_sync();
    for (int e = tid; e < nr; e += kCons) {
      float v = 0.f;
      for (int q = 0; q < ks; ++q) v += red[e * ks + q];
      const int row = r + e;
      if (EPI == EPI_STORE) {
        out[row] = v;
      } else if (EPI == EPI_SEGOUT) {
        sm.seg_out[row - sg.r0] = v;
      } else {
        if (v != v) v = -INFINITY;
        if (v > best_v || (v == best_v && row < best_i)) {
          best_v = v;
          best_i = row;
        }
      }
    }
    ++it;
  }
  return true;
}

template <int EPI>
__device__ bool gemv_any(const Params& p, Smem& sm, int n, int k, float* out, int& it, float& bv, long long& bi) {
  const Plan pl = plan_for(k);
  switch (pl.gpl) {
    case 1: return gemv_rows<1, EPI>(p, sm, n, k, pl.ks, out, it, bv, bi);
    case 2: return gemv_rows<2, EPI>(p, sm, n, k, pl.ks, out, it, bv, bi);
    case 3: return gemv_rows<3, EPI>(p, sm, n, k, pl.ks, out, it, bv, bi);
    default: return gemv_rows<4, EPI>(p, sm, n, k, pl.ks, out, it, bv, bi);
  }
}

// sm.vec <- RMSNorm(v) * w in the transposed layout, where v is given by `get(i)`
// (natural index); optionally also stores v (natural layout) to `keep`.
template <typename Get>
__device__ void build_norm(const Params& p, Smem& sm, int n, Get get, const float* w, float* keep) {
  const int G = n / 32;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += kCons) {
    const float v = get(i);
    sm.va[kMaxK + i] = v;
    ss += v * v;
  }
  const float dnm = sqrtf(cons_sum(ss, sm) / n + p.eps);
  for (int i = threadIdx.x; i < n; i += kCons) {
    const float v = sm.va[kMaxK + i];
    if (keep) keep[i] = v;
    sm.va[(i & 31) * G + (i >> 5)] = v / dnm * w[i];
  }
  cons_sync();
}

// residual update x + RMSNorm(y) * w  into sm.aux (natural layout); returns via get
__device__ void residual(const Params& p, Smem& sm, int n, const float* x, const float* y, const float* w) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += kCons) {
    const float v = y[i];
    ss += v * v;
  }
  const float dnm = sqrtf(cons_sum(ss, sm) / n + p.eps);
  for (int i = threadIdx.x; i < n; i += kCons) sm.va[kMaxK + i] = x[i] + y[i] / dnm * w[i];
  cons_sync();
}

__device__ __forceinline__ float gelu_tanh(float x) {
  return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

// ---------------------------------------------------------------- attention phase
// Work item c: keys [32c, min(T, 32c + 32)) of the single sequence.
__device__ void attn_chunk(const Params& p, Smem& sm, const Layer& L, int c, int pos) {
  const int nh = p.nh, qd = nh * HD;
  const int T = pos + 1, t0 = c * CKA, nt = min(CKA, T - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* ks = sm.va;                          // [CKA][HD]
  float* qs = sm.va + CKA * HD;               // [nh][HD]
  float* ps = sm.va + 2 * kMaxK - kMaxHeads * CKA;  // [nh][CKA]
  static_assert(CKA * HD + kMaxHeads * HD <= 2 * kMaxK - kMaxHeads * CKA, "attention scratch overlaps");
  const float* cs = p.cos_t + static_cast<size_t>(pos) * (HD / 2);
  const float* sn = p.sin_t + static_cast<size_t>(pos) * (HD / 2);
  // q heads (warp h), and k / v of this position in the last chunk's CTA
  const bool last = t0 + nt == T;
  for (int h = warp; h < nh + (last ? 2 : 0); h += kCons / 32) {
    const int col = h < nh ? h * HD : (h == nh ? qd : qd + HD);
    float v[8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = p.qkv[col + lane + 32 * j];
      ss += v[j] * v[j];
    }
    const float dnm = sqrtf(warp_sum(ss) / HD + p.eps);
    const float* w = h < nh ? L.q_norm : L.k_norm;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = h <= nh ? v[j] / dnm * w[lane + 32 * j] : v[j] / dnm;
    if (h <= nh) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = lane + 32 * j;
        const float a = v[j], b = v[j + 4];
        v[j] = a * cs[i] - b * sn[i];
        v[j + 4] = b * cs[i] + a * sn[i];
      }
    }
    if (h < nh) {
#pragma unroll
      for (int j = 0; j < 8; ++j) qs[h * HD + lane + 32 * j] = v[j];
    } else {
      float* cache = (h == nh ? L.kc : L.vc) + static_cast<size_t>(pos) * HD;
#pragma unroll
      for (int j = 0; j < 8; ++j) cache[lane + 32 * j] = v[j];
    }
  }
  cons_sync();
  const float* kb = L.kc + static_cast<size_t>(t0) * HD;
  for (int i = threadIdx.x; i < nt * HD / 4; i += kCons)
    reinterpret_cast<float4*>(ks)[i] = reinterpret_cast<const float4*>(kb)[i];
  cons_sync();
  for (int h = warp; h < nh; h += kCons / 32) {
    float q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = qs[h * HD + lane + 32 * j];
    float mine = -INFINITY;
    for (int t = 0; t < nt; ++t) {
      float dd = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) dd += q[j] * ks[t * HD + lane + 32 * j];
      dd = warp_sum(dd);
      if (lane == t) mine = dd;
    }
    const float m = warp_max(mine);
    const float pv = lane < nt ? expf(mine - m) : 0.f;
    const float l = warp_sum(pv);
    ps[h * CKA + lane] = pv;
    if (lane == 0) {
      float* pm = p.part + (static_cast<size_t>(c) * nh + h) * (HD + 2);
      pm[HD] = m;
      pm[HD + 1] = l;
    }
  }
  cons_sync();
  const float* vb = L.vc + static_cast<size_t>(t0) * HD;
  for (int dcol = threadIdx.x; dcol < HD; dcol += kCons) {
    float acc[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) acc[h] = 0.f;
    for (int t = 0; t < nt; ++t) {
      const float vv = vb[static_cast<size_t>(t) * HD + dcol];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h < nh) acc[h] += ps[h * CKA + t] * vv;
    }
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h)
      if (h < nh) p.part[(static_cast<size_t>(c) * nh + h) * (HD + 2) + dcol] = acc[h];
  }
  cons_sync();
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  if (p.bar[3] == 0) p.trace = nullptr;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  const int H = p.H, nh = p.nh, qd = nh * HD, nqkv = qd + 2 * HD, F = p.F;
  if (tid == 0) {
    for (int i = 0; i < kRing; ++i) {
      sbd::mbar_init(&sm.full[i], 1);
      sbd::mbar_init(&sm.empty[i], kCons / 32);
    }
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
  }
  __syncthreads();

  if (tid >= kCons) {
    // ------------------------------------------------------------ producer warp
    if (tid == kCons) {
      int it = 0;
      bool ok = true;
      for (int li = 0; li < p.n_layers && ok; ++li) {
        const Layer& L = p.layers[li];
        ok = produce(p, sm, L.w[0], L.s[0], nqkv, H, it) && produce(p, sm, L.w[1], L.s[1], H, qd, it) &&
             produce(p, sm, L.w[2], L.s[2], 2 * F, H, it) && produce(p, sm, L.w[3], L.s[3], H, F, it);
      }
      if (ok) ok = produce(p, sm, p.emb, p.emb_s, p.V, H, it);
      if (!ok) {
        // let copies in flight land before the CTA releases its shared memory
        const uint64_t t0 = sbd::global_ns();
        for (int i = max(0, it - kRing); i < it; ++i)
          while (!sbd::mbar_try_wait(&sm.full[i % kRing], (i / kRing) & 1) && sbd::global_ns() - t0 < sbd::kWaitLimitNs) {
          }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumer warps
  if (blockIdx.x == 0 && tid == 0) {
    *p.keys = 0ull;  // ordered before the lm_head by the barriers
    if (p.trace) {
      p.trace[0] = 1;
      p.trace[1] = sbd::global_ns();
    }
  }
  const int pos = p.pos[0];
  int it = 0;
  float bv = -INFINITY;
  long long bi = 0x7FFFFFFF;
  const bool lead = blockIdx.x == 0;
  bool ok = true;
  for (int li = 0; li < p.n_layers && ok; ++li) {
    const Layer& L = p.layers[li];
    // ---- qkv: layer input, RMSNorm, GEMV
    if (li == 0) {
      const int64_t tok = p.cur[0];
      const uint8_t* er = p.emb + tok * (H / 2);
      const __half* es = p.emb_s + tok * (H / 32);
      build_norm(p, sm, H,
                 [&](int i) {
                   const uint8_t b = er[i >> 1];
                   const int q = ((i & 1) ? (b >> 4) : (b & 15)) - 8;
                   return __fmul_rn(__fmul_rn(static_cast<float>(q), __half2float(es[i >> 5])), p.embed_scale);
                 },
                 L.in_norm, lead ? p.xa : nullptr);
    } else {
      residual(p, sm, H, p.xb, p.d, p.layers[li - 1].post_ffn);
      build_norm(p, sm, H, [&](int i) { return sm.va[kMaxK + i]; }, L.in_norm, lead ? p.xa : nullptr);
    }
    ok = gemv_any<EPI_STORE>(p, sm, nqkv, H, p.qkv, it, bv, bi) && grid_sync(p, sm);
    if (!ok) break;
    // ---- attention partials
    const int nc = (pos + 1 + CKA - 1) / CKA;
    for (int c = blockIdx.x; c < nc; c += gridDim.x) attn_chunk(p, sm, L, c, pos);
    if (!grid_sync(p, sm)) break;
    // ---- merge: item (head, 64 dims)
    for (int item = blockIdx.x; item < nh * 4; item += gridDim.x) {
      const int h = item >> 2, d0 = (item & 3) * 64;
      if (tid < 64) {
        const float* base = p.part + static_cast<size_t>(h) * (HD + 2);
        const size_t cst = static_cast<size_t>(nh) * (HD + 2);
        float M = -INFINITY;
        for (int c = 0; c < nc; ++c) M = fmaxf(M, base[c * cst + HD]);
        float Lsum = 0.f, O = 0.f;
        for (int c = 0; c < nc; ++c) {
          const float f = expf(base[c * cst + HD] - M);
          Lsum += base[c * cst + HD + 1] * f;
          O += base[c * cst + d0 + tid] * f;
        }
        p.attn[h * HD + d0 + tid] = O / Lsum;
      }
    }
    if (!grid_sync(p, sm)) break;
    // ---- o projection
    for (int i = tid; i < qd; i += kCons) sm.va[(i & 31) * (qd / 32) + (i >> 5)] = p.attn[i];
    cons_sync();
    ok = gemv_any<EPI_STORE>(p, sm, H, qd, p.o, it, bv, bi) && grid_sync(p, sm);
    if (!ok) break;
    // ---- gate|up with GEGLU
    residual(p, sm, H, p.xa, p.o, L.post_attn);
    build_norm(p, sm, H, [&](int i) { return sm.va[kMaxK + i]; }, L.pre_ffn, lead ? p.xb : nullptr);
    ok = gemv_any<EPI_SEGOUT>(p, sm, 2 * F, H, nullptr, it, bv, bi);
    if (!ok) break;
    cons_sync();
    {
      const Seg sg = segment(2 * F, H);
      for (int i = tid; i < (sg.r1 - sg.r0) / 2; i += kCons)
        p.a[sg.r0 / 2 + i] = gelu_tanh(sm.seg_out[2 * i]) * sm.seg_out[2 * i + 1];
    }
    if (!grid_sync(p, sm)) break;
    // ---- down projection
    for (int i = tid; i < F; i += kCons) sm.va[(i & 31) * (F / 32) + (i >> 5)] = p.a[i];
    cons_sync();
    ok = gemv_any<EPI_STORE>(p, sm, H, F, p.d, it, bv, bi) && grid_sync(p, sm);
  }
  if (!ok) return;
  // ---- final norm + tied lm_head with argmax
  residual(p, sm, H, p.xb, p.d, p.layers[p.n_layers - 1].post_ffn);
  build_norm(p, sm, H, [&](int i) { return sm.va[kMaxK + i]; }, p.final_norm, nullptr);
  if (!gemv_any<EPI_ARGMAX>(p, sm, p.V, H, nullptr, it, bv, bi)) return;
  {
    const int lane = tid & 31, warp = tid >> 5;
    unsigned long long key = 0ull;
    if (bi != 0x7FFFFFFF) {
      float f = bv;
      const uint32_t b = __float_as_uint(f);
      const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
      key = (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(bi));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
      key = o > key ? o : key;
    }
    if (lane == 0) sm.best[warp] = key;
    cons_sync();
    if (tid == 0) {
      unsigned long long k2 = 0;
      for (int w = 0; w < kCons / 32; ++w) k2 = sm.best[w] > k2 ? sm.best[w] : k2;
      if (k2) atomicMax(p.keys, k2);
    }
  }
  if (!grid_sync(p, sm)) return;
  if (lead && tid == 0) {
    const unsigned long long k2 = *reinterpret_cast<volatile unsigned long long*>(p.keys);
    const int32_t t = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k2 & 0xFFFFFFFFull));
    const int np = pos + 1;
    p.tok[0] = t;
    p.cur[0] = t;
    p.pos[0] = np;
    if (p.history && np < p.hist_len) p.history[np] = t;
  }
}

int grid_size(int smem) {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  cudaError_t e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return -1;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads, smem);
  if (per_sm < 1) return -1;
  const int g = sb::num_sms();  // one CTA per SM
  if (dev >= 0 && dev < 64) cached[dev] = g;
  return g;
}

}  // namespace

extern "C" size_t sb_decode_step_fused_scratch_size(int hidden, int n_heads, int head_dim, int inter, int max_seq) {
  if (head_dim != HD || n_heads < 1 || n_heads > kMaxHeads) return 0;
  const size_t qd = static_cast<size_t>(n_heads) * HD;
  const size_t chunks = (static_cast<size_t>(max_seq) + CKA - 1) / CKA;
  const size_t floats = 2 * hidden + (qd + 2 * HD) + qd + hidden + inter + hidden + chunks * n_heads * (HD + 2);
  return 64 + kTraceLen * sizeof(unsigned long long) + floats * sizeof(float);
}

extern "C" int sb_decode_step_fused(const void* layers_dev, int n_layers, const void* emb, const void* emb_scales,
                                    const float* final_norm, const float* cos_t, const float* sin_t, int hidden,
                                    int n_heads, int head_dim, int inter, int vocab, int max_seq, float eps,
                                    float embed_scale, int32_t* pos, int32_t* cur, int32_t* tokens, int32_t* history,
                                    int hist_len, uint64_t* keys, void* scratch, size_t scratch_bytes, void* stream) {
  SB_CHECK_ARG(head_dim == HD, "sb_decode_step_fused: head_dim must be %d", HD);
  SB_CHECK_ARG(n_heads >= 1 && n_heads <= kMaxHeads, "sb_decode_step_fused: n_heads must be 1..%d", kMaxHeads);
  SB_CHECK_ARG(hidden % 32 == 0 && hidden <= kMaxK && inter % 32 == 0 && inter <= kMaxK && n_heads * HD <= kMaxK,
               "sb_decode_step_fused: hidden, inter and n_heads*head_dim must be multiples of 32 up to %d", kMaxK);
  SB_CHECK_ARG(n_layers >= 1 && vocab >= 1 && max_seq >= 1, "sb_decode_step_fused: bad sizes");
  SB_CHECK_ARG(layers_dev && emb && emb_scales && final_norm && cos_t && sin_t && pos && cur && tokens && keys &&
                   scratch,
               "sb_decode_step_fused: null pointer");
  const size_t need = sb_decode_step_fused_scratch_size(hidden, n_heads, head_dim, inter, max_seq);
  if (scratch_bytes < need)
    return sb::fail(SB_ERR_WORKSPACE, "sb_decode_step_fused: scratch %zu < %zu bytes", scratch_bytes, need);
  const int smem = static_cast<int>(sizeof(Smem));
  const int grid = grid_size(smem);
  if (grid < 1) return sb::fail(SB_ERR_CUDA, "sb_decode_step_fused: cannot place one CTA per SM");
  // each CTA's gate|up slice must fit the GEGLU staging buffer
  const int per = ((2 * inter + grid - 1) / grid + 1) & ~1;
  SB_CHECK_ARG(per <= kSegOut, "sb_decode_step_fused: inter=%d too large for %d SMs", inter, grid);
  Params p{};
  p.layers = static_cast<const Layer*>(layers_dev);
  p.n_layers = n_layers;
  p.emb = static_cast<const uint8_t*>(emb);
  p.emb_s = static_cast<const __half*>(emb_scales);
  p.final_norm = final_norm;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.H = hidden;
  p.nh = n_heads;
  p.F = inter;
  p.V = vocab;
  p.max_seq = max_seq;
  p.eps = eps;
  p.embed_scale = embed_scale;
  p.pos = pos;
  p.cur = cur;
  p.tok = tokens;
  p.history = history;
  p.hist_len = hist_len;
  p.keys = reinterpret_cast<unsigned long long*>(keys);
  p.err = sb::device_error_word();
  char* base = static_cast<char*>(scratch);
  p.bar = reinterpret_cast<unsigned int*>(base);
  // the trace region is used only when bar[3] (set by the caller) is non-zero
  p.trace = reinterpret_cast<unsigned long long*>(base + 64);
  float* f = reinterpret_cast<float*>(base + 64 + kTraceLen * sizeof(unsigned long long));
  const size_t qd = static_cast<size_t>(n_heads) * HD;
  p.xa = f;
  f += hidden;
  p.xb = f;
  f += hidden;
  p.qkv = f;
  f += qd + 2 * HD;
  p.attn = f;
  f += qd;
  p.o = f;
  f += hidden;
  p.a = f;
  f += inter;
  p.d = f;
  f += hidden;
  p.part = f;
  void* args[] = {&p};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_step_kernel), dim3(grid),
                                              dim3(kThreads), args, smem, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return sb::cuda_fail(e, "decode_step_kernel (cooperative launch)");
  return SB_OK;
}
