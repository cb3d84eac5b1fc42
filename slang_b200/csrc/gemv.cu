// Decode GEMV over packed int4 weights (sb_gemv_q4) and the tied lm_head GEMV
// fused with greedy argmax (sb_lmhead_argmax).
//
// Streaming.  Rows are cut into stages of `rs` consecutive rows; a stage is one
// contiguous span of the packed matrix (and of its scales), moved by a single
// cp.async.bulk (TMA bulk copy) into a 4-deep shared-memory ring whose slots
// complete on mbarriers.  Lane 0 of warp 0 issues the first four stages at
// entry.  When a half-warp covers whole rows (K <= 16 lanes x GPL groups,
// gemv_q4_stream_kernel: every matrix with K <= 2048) each warp releases a
// slot when it is done with it and the last warp to release it refills it,
// with no CTA-wide barrier per stage; otherwise (gemv_q4_kernel) K slices are
// reduced through shared memory and the slot is refilled right after the
// per-stage CTA barrier that already proves every warp is done with it.
// Neither form has a producer warp.  CTAs (8 warps) take stages round robin,
// two per SM, so up to 8 x 24 KB per SM is in flight.  Kernels are launched with programmatic
// dependent launch: weights (which no earlier kernel writes) start streaming
// at once, and the warps wait for the previous kernel (griddepcontrol.wait)
// only before they read x.
//
// Arithmetic.  16 consumer half-warps; K is split into `ks` slices and each
// half-warp owns one slice of some rows of a stage; lane l owns the 32-value
// groups slice_begin + l + 16*u (u < GPL) of every row it visits.  Its slice
// of x is quantised once per CTA to 16-bit integers per group (scale = the
// group's max |x| / 32767, error <= 2^-16 of that max) and split into a
// signed high byte and an unsigned low byte, packed to match the packed
// nibbles.  A 16-byte chunk (32 nibbles) then costs 2 LOP3, 1 SHF and 4 DP4A
// per 8 values, and the int4 x int16 products are summed exactly in int32:
//   sum_k (q_k - 8) x_k = 256*dot(q, x_hi) + dot(q, x_lo) - 8*sum(x_int).
// Per (row, group) the integer dot is scaled by s_w * s_x in f32.  Partial
// sums are reduced with half-warp shuffles and, across K slices, through
// shared memory in a fixed order (deterministic results).
#include <algorithm>
#include <cstddef>
#include <cstring>

#include <atomic>

#include "common.cuh"
#include "norm_tail.cuh"
#include "q4_dot.cuh"

namespace {

constexpr int kConsumers = 256;                 // 8 warps, all computing
constexpr int kThreads = kConsumers;
constexpr int kRing = 4;                        // stages in flight per CTA
constexpr int kStageW = 24 * 1024;              // max weight bytes per stage
constexpr int kStageS = 3 * 1024;               // max scale bytes per stage
constexpr int kCtasPerSm = 2;                   // two CTAs share an SM (registers <= 113)
constexpr int kRedMax = 128;                    // partial-sum slots per stage (rows x ks x M)

// epilogues: store y; running argmax keys; store srq(y) of an SRQ linear (whose
// input is srq-coded too); store y and run the last-arriver norm-add tail.
// The SRQ and tail forms are separate instantiations, so the plain store keeps
// its registers.
enum { EPI_STORE = 0, EPI_ARGMAX = 1, EPI_SRQ = 2, EPI_TAIL = 3 };

struct GemvParams {
  const uint8_t* w;
  const void* scales;
  const void* x;
  float* y;
  unsigned long long* keys;
  float* logits;
  int* err;
  int m, n, k, group, ldy, ks, rs, n_stages, scale_bulk, x_f32;
  int bits;  // code width: 4 (two per byte) or 2 (four per byte)
  int x_stage;  // stream kernel: x quantised once per CTA into shared memory (else per warp)
  long long row_offset;
  // vocabulary shards over peer memory: each CTA's key goes to every rank's
  // mailbox (atomic MAX through NVLink) instead of `keys`
  const unsigned long long* peer_mailboxes;  // device array of `world` mailbox addresses
  uint8_t* peer_own;                         // this rank's mailbox
  int32_t* tokens;                           // peer exchange: the combined tokens
  int world, peer_row0;                      // peer_row0: first batch row of this launch
  int peer_rows, peer_finish;                // rows of the step; 1 in the launch that holds the last rows
  uint64_t peer_wait_ns;                     // bound of the wait for the other ranks
  // static range quantisation (SRQ) of the linear, gemma4_150/reference.py:96-101:
  // y = srq(W @ srq(x, srq_in), out) with out = srq_out_rows[row] when given,
  // else srq_out; a scale of 0 skips that srq
  float srq_in, srq_out;
  const float* srq_out_rows;
  // optional last-arriver residual add + RMSNorm over the launch's rows of y
  // (tail.counter != null; EPI_STORE only)
  sbd::NormTail tail;
  unsigned long long* trace;  // stream kernel, profiling only: kGvTraceSlots stamps per CTA, or null
};

// Profiling stamps of the stream kernel (sb_gemv_trace): slot i of CTA b is
// trace[b * kGvTraceSlots + i]; %globaltimer ns unless noted.  Thread 0's view.
enum {
  GV_SMID = 0,        // the CTA's SM (not a time)
  GV_ENTRY = 1,       // kernel entry
  GV_ISSUED = 2,      // first stages' bulk copies issued
  GV_DEP = 3,         // griddepcontrol.wait returned (the previous kernel is done)
  GV_X = 4,           // x loaded and quantised
  GV_STAGE0 = 5,      // first stage landed (warp 0)
  GV_STAGE0_DONE = 6, // first stage's rows done (warp 0)
  GV_ROWS_DONE = 7,   // warp 0's last stage done
  GV_PUBLISHED = 8,   // keys folded (argmax) / rows stored
  GV_EXIT = 9,        // leaving the kernel
  GV_STAGES = 10,     // stages this CTA ran (not a time)
  GV_LAST = 11,       // 1 when this CTA completed the launch's count (peer exchange; not a time)
  GV_PEER_SENT = 12,  // last CTA: keys sent to every rank
  GV_PEER_DONE = 13,  // last CTA: every rank's keys received
  kGvTraceSlots = 16
};
__device__ __forceinline__ void gv_stamp(const GemvParams& p, int slot, unsigned long long v) {
  if (p.trace) p.trace[static_cast<size_t>(blockIdx.x) * kGvTraceSlots + slot] = v;
}

// The output side of an SRQ linear: srq(y, s) = clip(round(y / s), -128, 127) * s.
__device__ __forceinline__ float srq_out(const GemvParams& p, int row, float v) {
  const float s = p.srq_out_rows ? p.srq_out_rows[row] : p.srq_out;
  return s != 0.f ? static_cast<float>(sbd::srq_code(v, s)) * s : v;
}

struct GemvSmem {
  uint8_t w[kRing][kStageW];
  uint8_t s[kRing][kStageS];
  unsigned long long best[8][4];
  uint64_t full[kRing];
  int released[kRing];  // stream kernel: warps done with the slot's current stage
  int issued;           // stream kernel: stages issued so far
  int abort;
  // gemv_q4_kernel: partial sums across K slices.  The stream kernel has no
  // use for them and keeps its staged x here instead (x_stage), in a region
  // sized at launch: kXqBytes per (batch row, group).
  alignas(16) float red[2][kRedMax];
};
constexpr int kXqBytes = 72;  // one sbd::XGroup: he, ho, le, lo words, bias, sx

using sbd::make_key;

// This lane's groups of x (rows m < M of the batch, groups gidx[u]) quantised
// to 16-bit integers, kept in registers for the whole launch.
template <int M, int GPL, typename XG, bool SRQ>
__device__ __forceinline__ void load_x_groups(const GemvParams& p, const int (&gidx)[GPL], const bool (&gval)[GPL],
                                              XG (&xg)[M][GPL]) {
#pragma unroll
  for (int m = 0; m < M; ++m) {
#pragma unroll
    for (int u = 0; u < GPL; ++u) {
      float v[32];
      const bool ok = gval[u] && m < p.m;
      if (p.x_f32) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) +
                                                            static_cast<size_t>(m) * p.k + gidx[u] * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = ok ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[4 * j] = f.x;
          v[4 * j + 1] = f.y;
          v[4 * j + 2] = f.z;
          v[4 * j + 3] = f.w;
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
            v[8 * j + 2 * e] = f.x;
            v[8 * j + 2 * e + 1] = f.y;
          }
        }
      }
      if constexpr (SRQ) {
        if (p.srq_in != 0.f) {
          sbd::srq_group(v, p.srq_in, xg[m][u]);
          continue;
        }
      }
      sbd::quantise_group(v, xg[m][u]);
    }
  }
}

// load_x_groups for the stream kernel's 4-bit forms, where lanes l and l ^ 16
// of a warp hold the same groups: each lane of the pair loads half of every
// group (all loads issued before any is used) and the pair quantises it
// together (quantise_group_pair).
template <int M, int GPL>
__device__ __forceinline__ void load_x_pairs(const GemvParams& p, const int (&gidx)[GPL], const bool (&gval)[GPL],
                                             sbd::XGroup (&xg)[M][GPL], int h) {
  float v[M][GPL][16];
#pragma unroll
  for (int m = 0; m < M; ++m) {
#pragma unroll
    for (int u = 0; u < GPL; ++u) {
      const bool ok = gval[u] && m < p.m;
      const size_t off = static_cast<size_t>(m) * p.k + gidx[u] * 32 + 16 * h;
      if (p.x_f32) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + off);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 f = ok ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[m][u][4 * j] = f.x;
          v[m][u][4 * j + 1] = f.y;
          v[m][u][4 * j + 2] = f.z;
          v[m][u][4 * j + 3] = f.w;
        }
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x) + off);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint4 hv = ok ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
          const uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
            v[m][u][8 * j + 2 * e] = f.x;
            v[m][u][8 * j + 2 * e + 1] = f.y;
          }
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
#pragma unroll
    for (int u = 0; u < GPL; ++u) sbd::quantise_group_pair(v[m][u], h, xg[m][u]);
  }
}

// x quantised once per CTA for the stream kernel's 4-bit forms: thread pairs
// (t, t ^ 1) take one (batch row, group) each, load half of its values, and
// quantise it together (the pair's max and integer sum by one shuffle each)
// into its kXqBytes record in shared memory; after a barrier every lane reads
// the records of its own groups.  Same XGroups as quantise_group, for 1/8 of
// the per-warp work of load_x_pairs.
template <int M, int GPL>
__device__ __forceinline__ void stage_x(const GemvParams& p, uint8_t* xq, const int (&gidx)[GPL],
                                        const bool (&gval)[GPL], sbd::XGroup (&xg)[M][GPL], int tid) {
  const int G = p.k >> 5;
  const int halves = 2 * M * G;
  if ((tid & ~31) < halves) {  // warp-uniform: whole warps join the shuffles
    const int h = tid & 1, gg = tid >> 1;
    const bool act = tid < halves;
    const int m = act ? gg / G : 0, g = act ? gg - m * G : 0;
    const bool ld = act && m < p.m;
    float v[16];
    const size_t off = static_cast<size_t>(m) * p.k + g * 32 + 16 * h;
    if (p.x_f32) {
      const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + off);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 f = ld ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[4 * j] = f.x;
        v[4 * j + 1] = f.y;
        v[4 * j + 2] = f.z;
        v[4 * j + 3] = f.w;
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x) + off);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 hv = ld ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          v[8 * j + 2 * e] = f.x;
          v[8 * j + 2 * e + 1] = f.y;
        }
      }
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    const float inv = mx > 0.f ? 32767.f / mx : 0.f;
    uint32_t b[16], sum = 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      b[i] = sbd::rint_bits(v[i], inv);
      sum += b[i];
    }
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    if (act) {
      uint32_t* rec = reinterpret_cast<uint32_t*>(xq + static_cast<size_t>(m * G + g) * kXqBytes);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t he, ho, le, lo;
        sbd::pack_word(b + 8 * j, he, ho, le, lo);
        rec[2 * h + j] = he;
        rec[4 + 2 * h + j] = ho;
        rec[8 + 2 * h + j] = le;
        rec[12 + 2 * h + j] = lo;
      }
      if (h == 0) {
        rec[16] = static_cast<uint32_t>(-8 * static_cast<int>(sum - 32u * sbd::kRintBias));
        rec[17] = __float_as_uint(mx / 32767.f);
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int m = 0; m < M; ++m) {
#pragma unroll
    for (int u = 0; u < GPL; ++u) {
      uint32_t r[18];
      if (gval[u]) {
        const uint2* rec = reinterpret_cast<const uint2*>(xq + static_cast<size_t>(m * G + gidx[u]) * kXqBytes);
#pragma unroll
        for (int j = 0; j < 9; ++j) {
          const uint2 w = rec[j];
          r[2 * j] = w.x;
          r[2 * j + 1] = w.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 18; ++j) r[j] = 0u;
      }
      sbd::XGroup& x = xg[m][u];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x.he[j] = r[j];
        x.ho[j] = r[4 + j];
        x.le[j] = r[8 + j];
        x.lo[j] = r[12 + j];
      }
      x.bias = static_cast<int>(r[16]);
      x.sx = __uint_as_float(r[17]);
    }
  }
}

// Combine the per-warp argmax keys (sm.best[warp][m], warps 0..7) and publish
// one key per batch row: atomic MAX into p.keys, or into every rank's mailbox.
// Called by the 256 consumer threads after a barrier over them.
// The vocabulary-sharded lm_head's exchange, at the end of this rank's shard
// GEMV (every thread of every CTA calls it).  Each CTA folds its keys into this
// rank's own mailbox (device-scope atomic MAX) and counts itself in; the CTA
// that completes the count re-arms it and, in the launch holding the step's
// last rows, exchanges every row's key with the other ranks in one warp:
//   1. send: each row's key as two tagged words (tag = step + 1) into slot
//      [step parity][this rank][row] of every rank's mailbox (16-byte
//      system-scope stores over NVLink);
//   2. wait, bounded, until every rank's words of this step are in this
//      mailbox's slots, and take the MAX per row;
//   3. write keys and tokens, clear this rank's own keys, advance the step.
// A rank sends step e + 1's words only after it has read every rank's words of
// step e, which each rank sends only after its own step e - 1 has ended (the
// launch's CTAs wait for the previous kernel first), so the parity-(e + 1)
// slots it overwrites hold step e - 1's words, which every rank has read.
// What the exchange needs besides the keys, read by warp 0 of every CTA right
// after griddepcontrol.wait (the previous launch wrote the step counter), so
// the CTA that turns out last does not wait for them: the step and this rank's
// index (where its own mailbox sits in the peer array; -1 if absent).
struct PeerPre {
  uint32_t epoch;
  int rank;
  bool ready;
};
__device__ __forceinline__ PeerPre peer_preload(const GemvParams& p, int lane) {
  PeerPre r;
  r.epoch = *reinterpret_cast<const volatile uint32_t*>(p.peer_own + sbd::kMailEpoch);
  const unsigned long long own_addr = reinterpret_cast<unsigned long long>(p.peer_own);
  const unsigned int at = __ballot_sync(0xFFFFFFFFu, lane < p.world && p.peer_mailboxes[lane] == own_addr);
  r.rank = at ? __ffs(at) - 1 : -1;
  r.ready = true;
  return r;
}

template <int M>
__device__ __forceinline__ void peer_publish(const GemvParams& p, GemvSmem& sm, int tid, PeerPre pre) {
  if (tid >= 32) return;  // warp 0 folds the CTA's keys, counts in, and (last CTA) exchanges
  uint8_t* own = p.peer_own;
  unsigned long long* local = reinterpret_cast<unsigned long long*>(own + sbd::kMailLocal);
  const int lane = tid;
  if (!pre.ready) pre = peer_preload(p, lane);
  if (lane < M && lane < p.m) {
    unsigned long long key = 0;
    for (int wi = 0; wi < kConsumers / 32; ++wi) key = sm.best[wi][lane] > key ? sm.best[wi][lane] : key;
    if (key) atomicMax(local + p.peer_row0 + lane, key);
  }
  __syncwarp();
  // count in with release (the folds above come first) and acquire (the last
  // CTA then sees every CTA's folds)
  unsigned int old = 0;
  if (lane == 0)
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(own + sbd::kMailCtas)
                 : "memory");
  const bool last = __shfl_sync(0xFFFFFFFFu, old, 0) == gridDim.x - 1;
  if (!last) return;
  if (lane == 0) {
    *reinterpret_cast<volatile unsigned int*>(own + sbd::kMailCtas) = 0u;  // re-arm for the next launch
    gv_stamp(p, GV_LAST, 1ull);
  }
  if (!p.peer_finish) return;
  const int rows = p.peer_rows, world = p.world, rank = pre.rank;
  const uint32_t e = pre.epoch, q = e & 1u;
  const unsigned long long tag = e + 1u;
  const unsigned long long own_addr = reinterpret_cast<unsigned long long>(own);
  auto slot = [&](unsigned long long base, int r, int i) {
    return reinterpret_cast<unsigned long long*>(base + sbd::kMailSlots) +
           2 * ((static_cast<int>(q) * sbd::kMailMaxRanks + r) * sbd::kMailMaxRows + i);
  };
  bool ok = rank >= 0;
  if (ok) {
    for (int idx = lane; idx < world * rows; idx += 32) {
      const int pe = idx / rows, i = idx - pe * rows;
      const unsigned long long key = __ldcg(local + i);
      const unsigned long long w0 = (key & 0xFFFFFFFF00000000ull) | tag, w1 = (key << 32) | tag;
      asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(slot(p.peer_mailboxes[pe], rank, i)),
                   "l"(w0), "l"(w1)
                   : "memory");
    }
  }
  if (lane == 0) gv_stamp(p, GV_PEER_SENT, sbd::global_ns());
  unsigned long long comb0 = 0ull, comb1 = 0ull;  // the combined keys of rows lane and lane + 32
  const uint64_t t0 = sbd::global_ns();
  for (int i = 0; i < rows; ++i) {
    unsigned long long key = 0ull;
    if (ok && lane < world) {
      const unsigned long long* src = slot(own_addr, lane, i);
      for (;;) {
        unsigned long long w0, w1;
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(src) : "memory");
        if ((w0 & 0xFFFFFFFFull) == tag && (w1 & 0xFFFFFFFFull) == tag) {
          key = (w0 & 0xFFFFFFFF00000000ull) | (w1 >> 32);
          break;
        }
        if (sbd::global_ns() - t0 > p.peer_wait_ns) {
          ok = false;
          break;
        }
      }
    }
    ok = __all_sync(0xFFFFFFFFu, ok);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
      key = o > key ? o : key;
    }
    if (lane == (i & 31)) {
      if (i < 32)
        comb0 = key;
      else
        comb1 = key;
    }
  }
  if (!ok && lane == 0 && p.err) atomicExch(p.err, SB_ERR_TIMEOUT);
  if (lane == 0) gv_stamp(p, GV_PEER_DONE, sbd::global_ns());
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = lane + 32 * j;
    if (i >= rows) continue;
    const unsigned long long k = ok ? (j ? comb1 : comb0) : 0ull;
    if (p.keys) p.keys[i] = k;
    if (p.tokens) p.tokens[i] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
    local[i] = 0ull;
  }
  __syncwarp();
  if (lane == 0) *reinterpret_cast<volatile uint32_t*>(own + sbd::kMailEpoch) = e + 1u;
}

template <int M>
__device__ __forceinline__ void publish_keys(const GemvParams& p, GemvSmem& sm, int tid, PeerPre pre = PeerPre{}) {
  if (p.peer_mailboxes) {
    peer_publish<M>(p, sm, tid, pre);
    return;
  }
  if (tid < M && tid < p.m) {
    unsigned long long key = 0;
    for (int wi = 0; wi < kConsumers / 32; ++wi) key = sm.best[wi][tid] > key ? sm.best[wi][tid] : key;
    if (key) atomicMax(p.keys + tid, key);
  }
}

template <int M, int GPL, bool SF16, int EPI, int BITS>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_q4_kernel(const GemvParams p) {
  using XG = typename sbd::QTraits<BITS>::XG;
  using Chunk = typename sbd::QTraits<BITS>::Chunk;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GemvSmem& sm = *reinterpret_cast<GemvSmem*>(smem_raw);
  volatile int* abort = &sm.abort;
  const int tid = threadIdx.x;
  const int row_bytes = p.k * BITS / 8;
  const int gps = p.k / p.group;
  const int esz = SF16 ? 2 : 4;

  sbd::griddep_launch_dependents();
  const int my_stages = p.n_stages > static_cast<int>(blockIdx.x)
                            ? (p.n_stages - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                            : 0;
  // issue the bulk copies of this CTA's i-th stage into ring slot i % kRing
  auto issue = [&](int i) {
    const int slot = i % kRing;
    const int st = blockIdx.x + i * gridDim.x;
    const int r0 = st * p.rs;
    const int nr = min(p.rs, p.n - r0);
    const uint32_t wb = static_cast<uint32_t>(nr) * row_bytes;
    const uint32_t sbytes = p.scale_bulk ? static_cast<uint32_t>(nr) * gps * esz : 0u;
    const uint64_t pol = sbd::l2_policy_evict_first();  // weights are read once per step
    sbd::mbar_arrive_expect_tx(&sm.full[slot], wb + sbytes);
    sbd::bulk_load_hint(sm.w[slot], p.w + static_cast<size_t>(r0) * row_bytes, wb, &sm.full[slot], pol);
    if (sbytes)
      sbd::bulk_load_hint(sm.s[slot], static_cast<const uint8_t*>(p.scales) + static_cast<size_t>(r0) * gps * esz,
                          sbytes, &sm.full[slot], pol);
  };
  if (tid == 0) {
    for (int i = 0; i < kRing; ++i) sbd::mbar_init(&sm.full[i], 1);
    sm.abort = 0;
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
    // weights do not depend on the previous kernel: start streaming now
    for (int i = 0; i < kRing && i < my_stages; ++i) issue(i);
  }
  __syncthreads();

  const int hw = tid >> 4, l16 = tid & 15, warp = tid >> 5;
  const int ks = p.ks;
  const int kslice = hw % ks, rlane = hw / ks, nrl = 16 / ks;
  const int G = p.k >> 5;
  const int SG = (G + ks - 1) / ks;
  const int g_begin = kslice * SG;
  const int g_end = min(G, g_begin + SG);

  int gidx[GPL], gsi[GPL];
  bool gval[GPL];
#pragma unroll
  for (int u = 0; u < GPL; ++u) {
    gidx[u] = g_begin + l16 + 16 * u;
    gval[u] = gidx[u] < g_end;
    gsi[u] = (gidx[u] * 32) / p.group;  // scale index of this group within a row
  }

  // x is the previous kernel's output: wait for it (weights are already streaming)
  sbd::griddep_wait();
  // this lane's groups of x, quantised once (kept in registers)
  XG xg[M][GPL];
  load_x_groups<M, GPL, XG, EPI == EPI_SRQ>(p, gidx, gval, xg);

  float best_v[M];
  long long best_i[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    best_v[m] = -INFINITY;
    best_i[m] = 0x7FFFFFFF;
  }

  for (int i = 0; i < my_stages; ++i) {
    const int slot = i % kRing;
    const bool ok = sbd::mbar_wait(&sm.full[slot], (i / kRing) & 1, abort, p.err);
    if (!__syncthreads_and(ok)) {
      // a copy never landed: let any still in flight finish before the CTA exits
      if (tid == 0) {
        const uint64_t t0 = sbd::global_ns();
        for (int j = i; j < i + kRing && j < my_stages; ++j)
          while (!sbd::mbar_try_wait(&sm.full[j % kRing], (j / kRing) & 1) &&
                 sbd::global_ns() - t0 < sbd::kWaitLimitNs) {
          }
      }
      return;
    }
    const int st = blockIdx.x + i * gridDim.x;
    const int r0 = st * p.rs;
    const int nr = min(p.rs, p.n - r0);
    float* red = sm.red[i & 1];
    const uint8_t* wst = sm.w[slot];
    const uint8_t* sst = sm.s[slot];
    for (int rr = rlane; rr < p.rs; rr += nrl) {  // same trip count for every half-warp
      float acc[M];
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] = 0.f;
      if (rr < nr) {
#pragma unroll
        for (int u = 0; u < GPL; ++u) {
          if (!gval[u]) continue;
          const Chunk q = *reinterpret_cast<const Chunk*>(wst + rr * row_bytes + gidx[u] * (4 * BITS));
          const int gi = gsi[u];
          float sw;
          if (p.scale_bulk) {
            sw = SF16 ? __half2float(reinterpret_cast<const __half*>(sst)[rr * gps + gi])
                      : reinterpret_cast<const float*>(sst)[rr * gps + gi];
          } else {
            const size_t si = static_cast<size_t>(r0 + rr) * gps + gi;
            sw = SF16 ? __half2float(static_cast<const __half*>(p.scales)[si]) : static_cast<const float*>(p.scales)[si];
          }
#pragma unroll
          for (int m = 0; m < M; ++m)
            acc[m] = fmaf(static_cast<float>(sbd::dot_group(q, xg[m][u])), sw * xg[m][u].sx, acc[m]);
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], off, 16);
      }
      if (l16 == 0) {
#pragma unroll
        for (int m = 0; m < M; ++m) red[(rr * ks + kslice) * M + m] = acc[m];
      }
    }
    // every warp is done with this slot: refill it with stage i + kRing
    __syncthreads();
    if (tid == 0 && i + kRing < my_stages) issue(i + kRing);
    // combine K slices in a fixed order and run the epilogue
    for (int e = tid; e < nr * M; e += kConsumers) {
      const int rr = e / M, m = e - rr * M;
      float v = 0.f;
      for (int q = 0; q < ks; ++q) v += red[(rr * ks + q) * M + m];
      const int row = r0 + rr;
      if (m >= p.m) continue;
      if (EPI != EPI_ARGMAX) {
        p.y[static_cast<size_t>(m) * p.ldy + row] = EPI == EPI_SRQ ? srq_out(p, row, v) : v;
      } else {
        if (p.logits) p.logits[static_cast<size_t>(m) * p.n + row] = v;
        if (v != v) v = -INFINITY;
        const long long gi = p.row_offset + row;
#pragma unroll
        for (int mm = 0; mm < M; ++mm) {
          if (mm != m) continue;
          if (v > best_v[mm] || (v == best_v[mm] && gi < best_i[mm])) {
            best_v[mm] = v;
            best_i[mm] = gi;
          }
        }
      }
    }
  }

  if (EPI == EPI_ARGMAX) {
    const int lane = tid & 31;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      unsigned long long key = best_i[m] == 0x7FFFFFFF ? 0ull : make_key(best_v[m], best_i[m]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
        key = o > key ? o : key;
      }
      if (lane == 0) sm.best[warp][m] = key;
    }
    __syncthreads();
    publish_keys<M>(p, sm, tid);
  }
  if constexpr (EPI == EPI_TAIL) sbd::last_arriver_tail(p.y, p.ldy, p.m, p.n, p.tail);
}

// The GEMV for rows a half-warp covers whole (ks = 1: K <= 16 * GPL * 32),
// with no CTA-wide barrier per stage: the lane holding a row's sum writes it
// (or folds it into the running argmax) at once, each warp releases a ring
// slot when it is done with it, and the warp that releases it last refills
// it.  Warps drift freely and the copy engine never waits for the slowest
// warp of a stage.
template <int M, int GPL, bool SF16, int EPI, int BITS>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_q4_stream_kernel(const GemvParams p) {
  using XG = typename sbd::QTraits<BITS>::XG;
  using Chunk = typename sbd::QTraits<BITS>::Chunk;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GemvSmem& sm = *reinterpret_cast<GemvSmem*>(smem_raw);
  volatile int* abort = &sm.abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row_bytes = p.k * BITS / 8;
  const int gps = p.k / p.group;
  const int esz = SF16 ? 2 : 4;
  constexpr bool TR = EPI != EPI_TAIL;  // profiling stamps (the norm-tail form has no registers to spare)

  sbd::griddep_launch_dependents();
  const int my_stages = p.n_stages > static_cast<int>(blockIdx.x)
                            ? (p.n_stages - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                            : 0;
  if (TR && tid == 0 && p.trace) {
    gv_stamp(p, GV_ENTRY, sbd::global_ns());
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    gv_stamp(p, GV_SMID, smid);
    gv_stamp(p, GV_STAGES, static_cast<unsigned long long>(my_stages));
  }
  const uint64_t pol = sbd::l2_policy_evict_first();  // weights are read once per step
  auto issue = [&](int i) {
    const int slot = i % kRing;
    const int st = blockIdx.x + i * gridDim.x;
    const int r0 = st * p.rs;
    const int nr = min(p.rs, p.n - r0);
    const uint32_t wb = static_cast<uint32_t>(nr) * row_bytes;
    const uint32_t sbytes = p.scale_bulk ? static_cast<uint32_t>(nr) * gps * esz : 0u;
    sbd::mbar_arrive_expect_tx(&sm.full[slot], wb + sbytes);
    sbd::bulk_load_hint(sm.w[slot], p.w + static_cast<size_t>(r0) * row_bytes, wb, &sm.full[slot], pol);
    if (sbytes)
      sbd::bulk_load_hint(sm.s[slot], static_cast<const uint8_t*>(p.scales) + static_cast<size_t>(r0) * gps * esz,
                          sbytes, &sm.full[slot], pol);
  };
  if (tid == 0) {
    for (int i = 0; i < kRing; ++i) {
      sbd::mbar_init(&sm.full[i], 1);
      sm.released[i] = 0;
    }
    sm.abort = 0;
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
    // weights do not depend on the previous kernel: start streaming now
    for (int i = 0; i < kRing && i < my_stages; ++i) issue(i);
    sm.issued = min(kRing, my_stages);
    if (TR && p.trace) gv_stamp(p, GV_ISSUED, sbd::global_ns());
  }
  __syncthreads();

  // -------------------------------------------------------------- consumers
  const int hw = tid >> 4, l16 = tid & 15;
  int gidx[GPL], gsi[GPL];
  bool gval[GPL];
  const int G = p.k >> 5;
#pragma unroll
  for (int u = 0; u < GPL; ++u) {
    gidx[u] = l16 + 16 * u;
    gval[u] = gidx[u] < G;
    gsi[u] = (gidx[u] * 32) / p.group;  // scale index of this group within a row
  }
  // x is the previous kernel's output: wait for it (weights are already streaming)
  sbd::griddep_wait();
  if (TR && tid == 0 && p.trace) gv_stamp(p, GV_DEP, sbd::global_ns());
  PeerPre pre{};
  if constexpr (EPI == EPI_ARGMAX) {
    if (p.peer_mailboxes && warp == 0) pre = peer_preload(p, lane);
  }
  XG xg[M][GPL];
  if constexpr (BITS == 4 && EPI != EPI_SRQ) {
    if (p.x_stage)
      stage_x<M, GPL>(p, reinterpret_cast<uint8_t*>(sm.red), gidx, gval, xg, tid);
    else
      load_x_pairs<M, GPL>(p, gidx, gval, xg, lane >> 4);
  } else
    load_x_groups<M, GPL, XG, EPI == EPI_SRQ>(p, gidx, gval, xg);
  if (TR && tid == 0 && p.trace) gv_stamp(p, GV_X, sbd::global_ns());

  float best_v[M];
  long long best_i[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    best_v[m] = -INFINITY;
    best_i[m] = 0x7FFFFFFF;
  }
  for (int i = 0; i < my_stages; ++i) {
    const int slot = i % kRing;
    if (!__all_sync(0xFFFFFFFFu, sbd::mbar_wait(&sm.full[slot], (i / kRing) & 1, abort, p.err))) break;
    if (TR && i == 0 && tid == 0 && p.trace) gv_stamp(p, GV_STAGE0, sbd::global_ns());
    const int st = blockIdx.x + i * gridDim.x;
    const int r0 = st * p.rs;
    const int nr = min(p.rs, p.n - r0);
    const uint8_t* wst = sm.w[slot];
    const uint8_t* sst = sm.s[slot];
    for (int rr = hw; rr < p.rs; rr += 16) {  // the same trip count for both half-warps of a warp
      float acc[M];
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] = 0.f;
      if (rr < nr) {
#pragma unroll
        for (int u = 0; u < GPL; ++u) {
          if (!gval[u]) continue;
          const Chunk q = *reinterpret_cast<const Chunk*>(wst + rr * row_bytes + gidx[u] * (4 * BITS));
          const int gi = gsi[u];
          float sw;
          if (p.scale_bulk) {
            sw = SF16 ? __half2float(reinterpret_cast<const __half*>(sst)[rr * gps + gi])
                      : reinterpret_cast<const float*>(sst)[rr * gps + gi];
          } else {
            const size_t si = static_cast<size_t>(r0 + rr) * gps + gi;
            sw = SF16 ? __half2float(static_cast<const __half*>(p.scales)[si]) : static_cast<const float*>(p.scales)[si];
          }
#pragma unroll
          for (int m = 0; m < M; ++m)
            acc[m] = fmaf(static_cast<float>(sbd::dot_group(q, xg[m][u])), sw * xg[m][u].sx, acc[m]);
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], off, 16);
      }
      if (l16 == 0 && rr < nr) {
        const int row = r0 + rr;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          if (m >= p.m) continue;
          float v = acc[m];
          if (EPI != EPI_ARGMAX) {
            p.y[static_cast<size_t>(m) * p.ldy + row] = EPI == EPI_SRQ ? srq_out(p, row, v) : v;
          } else {
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
    // this warp is done with the slot; the last of the 8 warps refills it
    __syncwarp();
    if (TR && i == 0 && tid == 0 && p.trace) gv_stamp(p, GV_STAGE0_DONE, sbd::global_ns());
    if (lane == 0) {
      __threadfence_block();  // this warp's reads of the slot are done before the release
      if (atomicAdd(&sm.released[slot], 1) == kConsumers / 32 - 1) {
        __threadfence_block();
        sm.released[slot] = 0;
        if (i + kRing < my_stages) {
          sbd::fence_proxy_async_smem();
          issue(i + kRing);
          sm.issued = i + kRing + 1;
        }
      }
    }
  }

  if (TR && tid == 0 && p.trace) gv_stamp(p, GV_ROWS_DONE, sbd::global_ns());
  if (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      unsigned long long key = best_i[m] == 0x7FFFFFFF ? 0ull : make_key(best_v[m], best_i[m]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
        key = o > key ? o : key;
      }
      if (lane == 0) sm.best[warp][m] = key;
    }
    __syncthreads();
    publish_keys<M>(p, sm, tid, pre);
  }
  if (TR && tid == 0 && p.trace) gv_stamp(p, GV_PUBLISHED, sbd::global_ns());
  if (__syncthreads_or(*abort)) {
    // a copy never landed: let the latest one of each slot finish before the CTA exits (bounded)
    if (tid == 0) {
      const uint64_t t0 = sbd::global_ns();
      for (int j = max(0, sm.issued - kRing); j < sm.issued; ++j)
        while (!sbd::mbar_try_wait(&sm.full[j % kRing], (j / kRing) & 1) &&
               sbd::global_ns() - t0 < sbd::kWaitLimitNs) {
        }
    }
  }
  if constexpr (EPI == EPI_TAIL) sbd::last_arriver_tail(p.y, p.ldy, p.m, p.n, p.tail);
  if (TR && tid == 0 && p.trace) gv_stamp(p, GV_EXIT, sbd::global_ns());
}

__global__ void keys_to_tokens_kernel(const unsigned long long* keys, int32_t* tokens, int m) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < m) tokens[i] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(keys[i] & 0xFFFFFFFFull));
}

// Clears the argmax keys.  A kernel rather than a memset so that the GEMV
// launched after it (programmatic dependent launch) starts streaming weights
// at once; the GEMV's atomics come after its griddepcontrol.wait, i.e. after
// this kernel, and this kernel's stores after the previous reader of the keys.
__global__ void zero_keys_kernel(unsigned long long* keys, int m) {
  sbd::griddep_launch_dependents();
  sbd::griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < m) keys[i] = 0ull;
}

struct Plan {
  int gpl, ks, rs;
};

// Groups-per-lane and K slices so 16*GPL*ks covers a row's G groups with the
// least waste; then rows per stage: as many as fit 24 KB, but few enough that
// small matrices still spread over the SMs.
Plan plan(int mtile, int n, int k, int bits, int scale_row_bytes, int sms) {
  const int G = k / 32;
  const int max_gpl = mtile == 1 ? 4 : (mtile == 2 ? 2 : 1);
  Plan best{0, 16, 1};  // gpl 0: no shape of this batch tile covers the row
  int best_waste = 1 << 30;
  const int prefs[4] = {3, 2, 4, 1};
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
  if (best.gpl == 0) return best;
  const int nrl = 16 / best.ks;
  const int row_bytes = k * bits / 8;
  // rows per stage: a stage's codes and (when they ride along) its scales fit their buffers
  int rs = std::max(1, std::min(kStageW / row_bytes, kStageS / std::max(1, scale_row_bytes)));
  const int spread = (n + sms * kCtasPerSm - 1) / (sms * kCtasPerSm);  // rows per CTA if each gets one stage
  rs = std::min(rs, std::max(nrl, spread));
  rs = std::max(nrl, rs / nrl * nrl);
  while (rs * best.ks * mtile > kRedMax && rs > nrl) rs -= nrl;
  best.rs = rs;
  return best;
}

// Profiling buffer of sb_gemv_trace (null: off), its size in stamps and the
// stamps handed out so far: each traced launch (graph captures included) gets
// the next grid x kGvTraceSlots stamps while they last.
static unsigned long long* g_gv_trace = nullptr;
static size_t g_gv_trace_slots = 0, g_gv_trace_used = 0;

// Whether `kCtasPerSm` CTAs of `bytes` dynamic shared memory each fit one SM of
// the current device (its shared memory per SM less the per-CTA reservation).
bool fits_per_sm(int bytes) {
  static int per_sm[64] = {0}, reserved[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return false;
  if (!per_sm[dev]) {
    int a = 0, r = 0;
    if (cudaDeviceGetAttribute(&a, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&r, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess)
      return false;
    reserved[dev] = r;
    per_sm[dev] = a;
  }
  return kCtasPerSm * (bytes + reserved[dev]) <= per_sm[dev];
}

// Dynamic shared memory of the stream kernel with x staged (x_stage): the
// fixed part up to `red`, then one record per (batch row, group); every
// stream-kernel shape has M x G <= 64 (16 lanes x GPL x M <= 64 groups).
constexpr int kStreamFixed = static_cast<int>(offsetof(GemvSmem, red));
constexpr int kStreamStagedMax = (kStreamFixed + 64 * kXqBytes + 15) & ~15;

template <int M, int GPL, int EPI, int BITS>
int launch_t(GemvParams p, bool sf16, int sms, cudaStream_t s) {
  const int grid = std::min(p.n_stages, sms * kCtasPerSm);
  if (grid == 0) return SB_OK;
  p.trace = nullptr;
  if (g_gv_trace && p.ks == 1 && EPI != EPI_TAIL &&
      g_gv_trace_used + static_cast<size_t>(grid) * kGvTraceSlots <= g_gv_trace_slots) {
    p.trace = g_gv_trace + g_gv_trace_used;
    g_gv_trace_used += static_cast<size_t>(grid) * kGvTraceSlots;
  }
  const int smem = static_cast<int>(sizeof(GemvSmem));
  // the stream kernel's 4-bit forms quantise x once per CTA into the tail of
  // their shared memory when two CTAs per SM still fit
  int smem_stream = smem;
  p.x_stage = 0;
  if (p.ks == 1 && BITS == 4 && EPI != EPI_SRQ) {
    const int xq = std::max(static_cast<int>(sizeof(GemvSmem::red)), M * (p.k >> 5) * kXqBytes);
    const int need = (kStreamFixed + xq + 15) & ~15;
    if (M * (p.k >> 5) <= 64 && fits_per_sm(need)) {
      smem_stream = need;
      p.x_stage = 1;
    }
  }
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    // two CTAs per SM need the largest shared-memory carveout
    cudaError_t e = cudaFuncSetAttribute(gemv_q4_kernel<M, GPL, true, EPI, BITS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_kernel<M, GPL, false, EPI, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_kernel<M, GPL, true, EPI, BITS>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_kernel<M, GPL, false, EPI, BITS>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    const int smem_stream_max = std::max(smem, kStreamStagedMax);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_stream_kernel<M, GPL, true, EPI, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem_stream_max);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_stream_kernel<M, GPL, false, EPI, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem_stream_max);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_stream_kernel<M, GPL, true, EPI, BITS>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               100);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_q4_stream_kernel<M, GPL, false, EPI, BITS>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               100);
    if (e != cudaSuccess) return sb::cuda_fail(e, "gemv_q4_kernel: smem attribute");
    done[dev] = true;
  }
  cudaError_t e;
  if (p.ks == 1) {
    e = sf16 ? sb::launch_pdl(gemv_q4_stream_kernel<M, GPL, true, EPI, BITS>, dim3(grid), dim3(kThreads), smem_stream,
                              s, p)
             : sb::launch_pdl(gemv_q4_stream_kernel<M, GPL, false, EPI, BITS>, dim3(grid), dim3(kThreads), smem_stream,
                              s, p);
  } else {
    e = sf16 ? sb::launch_pdl(gemv_q4_kernel<M, GPL, true, EPI, BITS>, dim3(grid), dim3(kThreads), smem, s, p)
             : sb::launch_pdl(gemv_q4_kernel<M, GPL, false, EPI, BITS>, dim3(grid), dim3(kThreads), smem, s, p);
  }
  if (e != cudaSuccess) return sb::cuda_fail(e, "gemv_q4_kernel launch");
  return sb::launch_status("gemv_q4_kernel");
}

template <int M, int EPI, int BITS>
int launch_m(const GemvParams& p, const Plan& pl, bool sf16, int sms, cudaStream_t s) {
  if constexpr (M == 1) {
    switch (pl.gpl) {
      case 1: return launch_t<M, 1, EPI, BITS>(p, sf16, sms, s);
      case 2: return launch_t<M, 2, EPI, BITS>(p, sf16, sms, s);
      case 3: return launch_t<M, 3, EPI, BITS>(p, sf16, sms, s);
      default: return launch_t<M, 4, EPI, BITS>(p, sf16, sms, s);
    }
  } else if constexpr (M == 2) {
    return pl.gpl == 1 ? launch_t<M, 1, EPI, BITS>(p, sf16, sms, s) : launch_t<M, 2, EPI, BITS>(p, sf16, sms, s);
  } else {
    return launch_t<M, 1, EPI, BITS>(p, sf16, sms, s);
  }
}

template <int EPI>
int launch_bits(int bits, int mt, const GemvParams& q, const Plan& pl, bool sf16, int sms, cudaStream_t s) {
  if (bits == 2)
    return mt == 1 ? launch_m<1, EPI, 2>(q, pl, sf16, sms, s)
                   : mt == 2 ? launch_m<2, EPI, 2>(q, pl, sf16, sms, s) : launch_m<4, EPI, 2>(q, pl, sf16, sms, s);
  return mt == 1 ? launch_m<1, EPI, 4>(q, pl, sf16, sms, s)
                 : mt == 2 ? launch_m<2, EPI, 4>(q, pl, sf16, sms, s) : launch_m<4, EPI, 4>(q, pl, sf16, sms, s);
}

int run(GemvParams p, int epi, bool xf32, bool sf16, cudaStream_t s) {
  const int sms = sb::num_sms();
  const int x_elt = xf32 ? 4 : 2;
  const size_t x_row = static_cast<size_t>(p.k) * x_elt;
  const int esz = sf16 ? 2 : 4;
  const int gps = p.k / p.group;
  p.err = sb::device_error_word();
  p.x_f32 = xf32 ? 1 : 0;
  int done = 0;
  const int m_total = p.m;
  while (done < m_total) {
    const int left = m_total - done;
    // the widest batch tile whose lanes can hold a whole row's groups (x
    // registers shrink the groups per lane as the tile grows)
    int mt = left >= 4 ? 4 : (left >= 2 ? 2 : 1);
    const int srow_bytes = gps * esz;
    Plan pl = plan(mt, p.n, p.k, p.bits, srow_bytes, sms);
    while (pl.gpl == 0 && mt > 1) {
      mt /= 2;
      pl = plan(mt, p.n, p.k, p.bits, srow_bytes, sms);
    }
    if (pl.gpl == 0) return sb::fail(SB_ERR_ARG, "gemv: k=%d has more groups than a row's lanes hold", p.k);
    GemvParams q = p;
    q.m = mt;
    q.x = static_cast<const char*>(p.x) + done * x_row;
    if (epi != EPI_ARGMAX) {
      q.y = p.y + static_cast<size_t>(done) * p.ldy;
      if (p.tail.counter) {  // the tail of this launch covers its own rows
        const size_t o = static_cast<size_t>(done) * p.n;
        q.tail.hidden = p.tail.hidden + o;
        if (p.tail.h_out) q.tail.h_out = p.tail.h_out + o;
        if (p.tail.h16) q.tail.h16 = p.tail.h16 + o;
      }
    }
    else {
      if (p.keys && !p.peer_mailboxes) q.keys = p.keys + done;
      q.peer_row0 = p.peer_row0 + done;
      q.peer_finish = done + mt == m_total ? 1 : 0;
      if (p.logits) q.logits = p.logits + static_cast<size_t>(done) * p.n;
    }
    q.ks = pl.ks;
    q.rs = pl.rs;
    q.n_stages = (p.n + pl.rs - 1) / pl.rs;
    // scales ride along in the bulk copy when every stage's scale rows start
    // on a 16-byte boundary, are a multiple of 16 bytes (a short last stage
    // included) and fit the scale buffer
    const size_t srow = static_cast<size_t>(gps) * esz;
    const int last = p.n - (q.n_stages - 1) * pl.rs;
    q.scale_bulk = (srow * pl.rs) % 16 == 0 && (srow * last) % 16 == 0 &&
                   srow * pl.rs <= static_cast<size_t>(kStageS) && sb::aligned(p.scales, 16);
    int rc;
    switch (epi) {
      case EPI_STORE: rc = launch_bits<EPI_STORE>(p.bits, mt, q, pl, sf16, sms, s); break;
      case EPI_ARGMAX: rc = launch_bits<EPI_ARGMAX>(p.bits, mt, q, pl, sf16, sms, s); break;
      case EPI_SRQ: rc = launch_bits<EPI_SRQ>(p.bits, mt, q, pl, sf16, sms, s); break;
      default: rc = launch_bits<EPI_TAIL>(p.bits, mt, q, pl, sf16, sms, s); break;
    }
    if (rc != SB_OK) return rc;
    done += mt;
  }
  return SB_OK;
}

int check_common(const char* fn, const void* w, const void* scales, int scale_dtype, int group, const void* x,
                 int x_dtype, int m, int n, int k, int bits = 4) {
  SB_CHECK_ARG(m >= 1 && m <= 8, "%s: m=%d must be in 1..8", fn, m);
  SB_CHECK_ARG(n >= 0, "%s: negative n", fn);
  SB_CHECK_ARG(k > 0 && k % 32 == 0 && k <= 32768, "%s: k=%d must be a positive multiple of 32, at most 32768", fn,
               k);
  SB_CHECK_ARG(bits == 4 || k % 64 == 0, "%s: 2-bit rows must be a multiple of 16 bytes (k %% 64 == 0), k=%d", fn, k);
  SB_CHECK_ARG(k * bits / 8 <= kStageW, "%s: k=%d is longer than one stage (max %d)", fn, k, kStageW * 8 / bits);
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

namespace sb {
int zero_keys(unsigned long long* keys, int m, cudaStream_t s) {
  if (m <= 0) return SB_OK;
  const cudaError_t e = sb::launch_pdl(zero_keys_kernel, dim3((m + 255) / 256), dim3(256), 0, s, keys, m);
  if (e != cudaSuccess) return sb::cuda_fail(e, "zero_keys_kernel");
  return sb::launch_status("zero_keys_kernel");
}
}  // namespace sb

static int gemv_impl(const char* fn, int bits, const void* w, const void* scales, int scale_dtype, int group,
                     const void* x, int x_dtype, float* y, int ldy, int m, int n, int k, void* stream,
                     float srq_in = 0.f, float srq_out_s = 0.f, const float* srq_out_rows = nullptr) {
  int rc = check_common(fn, w, scales, scale_dtype, group, x, x_dtype, m, n, k, bits);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(ldy >= n, "%s: ldy=%d < n=%d", fn, ldy, n);
  if (n == 0) return SB_OK;
  SB_CHECK_ARG(y != nullptr, "%s: null y", fn);
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
  p.bits = bits;
  p.srq_in = srq_in;
  p.srq_out = srq_out_s;
  p.srq_out_rows = srq_out_rows;
  const bool srq = srq_in != 0.f || srq_out_s != 0.f || srq_out_rows;
  return run(p, srq ? EPI_SRQ : EPI_STORE, x_dtype == SB_F32, scale_dtype == SB_SCALE_F16,
             static_cast<cudaStream_t>(stream));
}

extern "C" int sb_gemv_trace(uint64_t* buf, size_t bytes) {
  SB_CHECK_ARG(!buf || sb::aligned(buf, 8), "sb_gemv_trace: buffer must be 8-byte aligned");
  g_gv_trace = buf ? reinterpret_cast<unsigned long long*>(buf) : nullptr;
  g_gv_trace_slots = buf ? bytes / sizeof(uint64_t) : 0;
  g_gv_trace_used = 0;
  return SB_OK;
}

extern "C" int sb_gemv_q4(const void* w, const void* scales, int scale_dtype, int group, const void* x,
                          int x_dtype, float* y, int ldy, int m, int n, int k, void* stream) {
  return gemv_impl("sb_gemv_q4", 4, w, scales, scale_dtype, group, x, x_dtype, y, ldy, m, n, k, stream);
}

extern "C" int sb_gemv_q2(const void* w, const void* scales, int scale_dtype, int group, const void* x,
                          int x_dtype, float* y, int ldy, int m, int n, int k, void* stream) {
  return gemv_impl("sb_gemv_q2", 2, w, scales, scale_dtype, group, x, x_dtype, y, ldy, m, n, k, stream);
}

extern "C" int sb_gemv_norm_add(const void* w, int bits, const void* scales, int scale_dtype, int group,
                                const void* x, int x_dtype, float* y, int m, int n, int k, float* hidden,
                                const float* w_add, const float* w_next, float* h_out, void* h16_out, float eps,
                                unsigned int* counter, void* stream) {
  SB_CHECK_ARG(bits == 2 || bits == 4, "sb_gemv_norm_add: bits=%d must be 2 or 4", bits);
  SB_CHECK_ARG(n % 4 == 0 && n <= 4 * sbd::kTailV4 * kThreads, "sb_gemv_norm_add: n=%d must be a multiple of 4 up to %d",
               n, 4 * sbd::kTailV4 * kThreads);
  SB_CHECK_ARG(hidden && w_add && counter && (!w_next || h_out || h16_out), "sb_gemv_norm_add: null pointer");
  SB_CHECK_ARG(sb::aligned(y, 16) && sb::aligned(hidden, 16) && sb::aligned(w_add, 16) &&
                   (!w_next || sb::aligned(w_next, 16)) && (!h_out || sb::aligned(h_out, 16)),
               "sb_gemv_norm_add: y, hidden, w_add, w_next and h_out need 16-byte alignment");
  int rc = check_common("sb_gemv_norm_add", w, scales, scale_dtype, group, x, x_dtype, m, n, k, bits);
  if (rc != SB_OK) return rc;
  if (n == 0) return SB_OK;
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.scales = scales;
  p.x = x;
  p.y = y;
  p.m = m;
  p.n = n;
  p.k = k;
  p.group = group;
  p.ldy = n;
  p.bits = bits;
  p.tail = sbd::NormTail{hidden, w_add, w_next, h_out, static_cast<__half*>(h16_out), counter, 1.f, eps};
  return run(p, EPI_TAIL, x_dtype == SB_F32, scale_dtype == SB_SCALE_F16, static_cast<cudaStream_t>(stream));
}

extern "C" int sb_gemv_srq(const void* w, int bits, const void* scales, int scale_dtype, int group, const void* x,
                           int x_dtype, float in_scale, float out_scale, const float* out_scales, float* y, int ldy,
                           int m, int n, int k, void* stream) {
  SB_CHECK_ARG(bits == 2 || bits == 4, "sb_gemv_srq: bits=%d must be 2 or 4", bits);
  SB_CHECK_ARG(in_scale >= 0.f && out_scale >= 0.f && in_scale == in_scale && out_scale == out_scale,
               "sb_gemv_srq: scales must be >= 0 (0 = no quantisation on that side)");
  return gemv_impl("sb_gemv_srq", bits, w, scales, scale_dtype, group, x, x_dtype, y, ldy, m, n, k, stream, in_scale,
                   out_scale, out_scales);
}

static int lmhead_impl(const char* fn, int bits, const void* emb, const void* scales, int scale_dtype, int group,
                       const void* h, int h_dtype, int m, int v, int k, int64_t row_offset, uint64_t* keys,
                       int32_t* tokens, float* logits, void* stream) {
  int rc = check_common(fn, emb, scales, scale_dtype, group, h, h_dtype, m, v, k, bits);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(keys != nullptr, "%s: null keys", fn);
  SB_CHECK_ARG(row_offset >= 0 && row_offset + v <= 0xFFFFFFFFLL, "%s: row indices must fit in 32 bits", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = sb::zero_keys(reinterpret_cast<unsigned long long*>(keys), m, s);
  if (rc != SB_OK) return rc;
  cudaError_t e;
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
    p.bits = bits;
    rc = run(p, EPI_ARGMAX, h_dtype == SB_F32, scale_dtype == SB_SCALE_F16, s);
    if (rc != SB_OK) return rc;
  }
  if (tokens) {
    e = sb::launch_pdl(keys_to_tokens_kernel, dim3((m + 255) / 256), dim3(256), 0, s,
                       reinterpret_cast<const unsigned long long*>(keys), tokens, m);
    if (e != cudaSuccess) return sb::cuda_fail(e, "keys_to_tokens_kernel");
    return sb::launch_status("keys_to_tokens_kernel");
  }
  return SB_OK;
}

extern "C" int sb_lmhead_argmax(const void* emb, const void* scales, int scale_dtype, int group, const void* h,
                                int h_dtype, int m, int v, int k, int64_t row_offset, uint64_t* keys,
                                int32_t* tokens, float* logits, void* stream) {
  return lmhead_impl("sb_lmhead_argmax", 4, emb, scales, scale_dtype, group, h, h_dtype, m, v, k, row_offset, keys,
                     tokens, logits, stream);
}

extern "C" int sb_lmhead_argmax_q2(const void* emb, const void* scales, int scale_dtype, int group, const void* h,
                                   int h_dtype, int m, int v, int k, int64_t row_offset, uint64_t* keys,
                                   int32_t* tokens, float* logits, void* stream) {
  return lmhead_impl("sb_lmhead_argmax_q2", 2, emb, scales, scale_dtype, group, h, h_dtype, m, v, k, row_offset, keys,
                     tokens, logits, stream);
}

namespace {

// How long the sharded lm_head's exchange waits for the other ranks to count in.
std::atomic<uint64_t> g_peer_wait_ns{sbd::kWaitLimitNs};

}  // namespace

extern "C" size_t sb_peer_mailbox_size(void) { return sbd::kMailBytes; }

extern "C" int sb_peer_set_wait_limit_ns(uint64_t ns) {
  SB_CHECK_ARG(ns <= sbd::kWaitLimitNs, "sb_peer_set_wait_limit_ns: %llu ns exceeds the %llu ns limit",
               static_cast<unsigned long long>(ns), static_cast<unsigned long long>(sbd::kWaitLimitNs));
  g_peer_wait_ns.store(ns ? ns : sbd::kWaitLimitNs);
  return SB_OK;
}

extern "C" int sb_peer_buffer_create(size_t bytes, void** dev_ptr, void* ipc_handle) {
  SB_CHECK_ARG(bytes > 0 && dev_ptr && ipc_handle, "sb_peer_buffer_create: bad arguments");
  cudaError_t e = cudaMalloc(dev_ptr, bytes);
  if (e != cudaSuccess) return sb::cuda_fail(e, "sb_peer_buffer_create: cudaMalloc");
  e = cudaMemset(*dev_ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), *dev_ptr);
  if (e != cudaSuccess) {
    cudaFree(*dev_ptr);
    *dev_ptr = nullptr;
    return sb::cuda_fail(e, "sb_peer_buffer_create: IPC handle");
  }
  return SB_OK;
}

extern "C" int sb_peer_buffer_open(const void* ipc_handle, void** dev_ptr) {
  SB_CHECK_ARG(ipc_handle && dev_ptr, "sb_peer_buffer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return sb::cuda_fail(e, "sb_peer_buffer_open");
  return SB_OK;
}

extern "C" int sb_peer_buffer_close(void* dev_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? SB_OK : sb::cuda_fail(e, "sb_peer_buffer_close");
}

extern "C" int sb_peer_buffer_free(void* dev_ptr) {
  cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? SB_OK : sb::cuda_fail(e, "sb_peer_buffer_free");
}

extern "C" int sb_lmhead_argmax_peer(const void* emb, const void* scales, int scale_dtype, int group, const void* h,
                                     int h_dtype, int m, int v, int k, int64_t row_offset,
                                     const uint64_t* peer_mailboxes, int world, void* own_mailbox, uint64_t* keys,
                                     int32_t* tokens, void* stream) {
  int rc = check_common("sb_lmhead_argmax_peer", emb, scales, scale_dtype, group, h, h_dtype, m, v, k);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(m <= sbd::kMailMaxRows, "sb_lmhead_argmax_peer: m=%d > %d", m, sbd::kMailMaxRows);
  SB_CHECK_ARG(v >= 1, "sb_lmhead_argmax_peer: every rank needs a non-empty shard (v=%d)", v);
  SB_CHECK_ARG(world >= 1 && world <= sbd::kMailMaxRanks && peer_mailboxes && own_mailbox, "sb_lmhead_argmax_peer: bad peer arguments");
  SB_CHECK_ARG(row_offset >= 0 && row_offset + v <= 0xFFFFFFFFLL, "sb_lmhead_argmax_peer: row indices must fit in 32 bits");
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(emb);
  p.scales = scales;
  p.x = h;
  p.m = m;
  p.n = v;
  p.k = k;
  p.group = group;
  p.row_offset = row_offset;
  p.bits = 4;
  p.keys = reinterpret_cast<unsigned long long*>(keys);
  p.tokens = tokens;
  p.peer_mailboxes = reinterpret_cast<const unsigned long long*>(peer_mailboxes);
  p.peer_own = static_cast<uint8_t*>(own_mailbox);
  p.world = world;
  p.peer_rows = m;
  p.peer_wait_ns = g_peer_wait_ns.load();
  return run(p, EPI_ARGMAX, h_dtype == SB_F32, scale_dtype == SB_SCALE_F16, static_cast<cudaStream_t>(stream));
}

extern "C" int sb_keys_to_tokens(const uint64_t* keys, int32_t* tokens, int m, void* stream) {
  SB_CHECK_ARG(m >= 0 && m <= 1 << 20, "sb_keys_to_tokens: bad m");
  if (m == 0) return SB_OK;
  SB_CHECK_ARG(keys && tokens, "sb_keys_to_tokens: null pointer");
  keys_to_tokens_kernel<<<(m + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const unsigned long long*>(keys), tokens, m);
  return sb::launch_status("keys_to_tokens_kernel");
}
