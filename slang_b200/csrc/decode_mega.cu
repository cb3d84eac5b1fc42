// One greedy decode step of the Gemma-4-E2B-shaped int4 decoder for a single
// sequence as ONE persistent cooperative kernel (sb_decode_step_fused).
//
// Why: a step is ~35 x 10 small dependent operations; as separate launches the
// step is dominated by launch and ramp latency, not by the ~0.9 GB of weights
// it must stream.  Here every SM runs one CTA for the whole step:
//
//   producer warp   walks this CTA's fixed sequence of weight row-slices --
//                   per layer its rows of q|k|v, o, gate|up (rows interleaved
//                   gate/up), down, then its rows of the tied lm_head -- and
//                   streams them (packed rows + their f16 group scales) with
//                   cp.async.bulk into a shared-memory ring.  Weights do not
//                   depend on activations, so the stream runs ahead across the
//                   phase hand-offs below.
//   8 consumer warps  run the phases, each waiting on its input words:
//     qkv:    x = layer input (embedding, or residual + post-FFN RMSNorm of
//             the previous down output), h = RMSNorm(x) * in_norm, GEMV rows.
//             Also starts the bulk copy of this CTA's attention chunk (16 keys
//             of K and V, q/k norm weights, this position's RoPE row) so it
//             lands while the GEMV and the hand-off run.
//     attn:   per 16-key chunk (one chunk per CTA): q/k norm + RoPE (the CTA
//             owning this position's chunk also writes k, v to the cache),
//             scores, chunk softmax partials, P.V partials
//     merge:  per (head, 16 dims): rescale the chunk partials -> attention out
//     o:      GEMV rows of o over the attention output
//     gateup: x += RMSNorm(o) * post_attn, h = RMSNorm(x) * pre_ffn, GEMV rows,
//             GEGLU of each interleaved (gate, up) row pair
//     down:   GEMV rows of down over the GEGLU output
//   and finally RMSNorm * final_norm, the lm_head rows with a running
//   (max, lowest index) per CTA, one 64-bit atomicMax per CTA, and the CTA
//   that arrives last decodes the token and advances pos / cur / history.
//
// Latency, not bandwidth, bounds this kernel (a phase moves ~20 MB over 148
// SMs), so the phases hand their outputs over with no grid barrier at all.
// Every value produced inside the launch is stored as one 64-bit word: the
// f32 bits in the low half and, in the high half, the epoch of the (launch,
// layer) that wrote it.  A 64-bit store is single-copy atomic, so a reader
// that sees the current epoch in a word also sees its value: a phase waits for
// its input by polling the input itself (ld.relaxed.gpu, every word of a
// thread's slots in flight at once) until every word carries the current
// epoch.  A transition then costs one L2 round trip once the slowest producer
// has stored, instead of a barrier's atomic, its poll and the load after it.
// Each CTA keeps its own copy of the residual stream in shared memory (all
// CTAs compute it identically), so only GEMV outputs, attention partials and
// the attention output cross between CTAs.
//
// Reuse of a buffer in the next layer is safe without a barrier because every
// CTA owns rows of gate|up (inter >= CTAs is checked at launch): a CTA's reads
// of any layer-L buffer precede, in its own program order and through data
// dependence, its gate|up rows of layer L (or L + 1), which every later
// producer of that buffer has consumed first.  The launch ends with one atomic
// count: the CTA that completes it reads the argmax key, advances the
// position and bumps the launch count the epochs derive from.  The next
// layer's norm vectors are prefetched into L2.
//
// GEMV arithmetic is the exact int4 x int16 DP4A dot of q4_dot.cuh.  Every wait
// (mbarrier or input poll) is bounded by %globaltimer; a timeout raises a
// sticky abort flag in the scratch header that every CTA polls, writes
// SB_ERR_TIMEOUT to the device error word, and the kernel unwinds.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "q4_dot.cuh"

namespace {

constexpr int kCons = 256;            // consumer threads (8 warps)
constexpr int kThreads = kCons + 32;  // + one producer warp
constexpr int kRing = 5;
constexpr int kStageW = 24 * 1024;
constexpr int kStageS = 3 * 1024;
constexpr int kMaxK = 6144;           // longest GEMV row (values)
constexpr int kMaxH = 2048;           // hidden size and n_heads * head_dim limit
constexpr int HD = 256;               // head_dim handled by this kernel
constexpr int CKA = 16;               // keys per attention work item
constexpr int kMaxHeads = 8;
constexpr int kMaxChunks = 2048;      // max_seq <= CKA * kMaxChunks
constexpr int kMergeDims = 16;        // attention output dims per merge work item
constexpr int kMaxG = kMaxK / 32;     // activation groups of the longest GEMV row
constexpr int kPasses = kMaxK / (8 * kCons);  // 8-value slots per thread for the longest row
constexpr int kMaxLayers = 48;
constexpr int kRed = 128;
constexpr int kSegOut = 512;          // rows of one CTA's gate|up slice kept for GEGLU
constexpr unsigned int kTraceLen = 2048;  // per CTA: [0] count, then tagged timestamps
constexpr int kTraceCtas = 160;           // trace slots (CTAs beyond this are not traced)
static_assert(kCons == HD, "the P.V step maps one thread to one head dim");
static_assert(CKA == 16, "the score reduction is written for 16-key chunks");
static_assert(2 * kMaxChunks + kCons <= 2 * CKA * HD, "merge scratch must fit the K/V chunk buffer");
static_assert(kMaxH == 8 * kCons, "a hidden vector is one 8-value slot per consumer thread");

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
  // values produced inside the launch, one (epoch << 32 | f32 bits) word each
  uint64_t *qkv, *attn, *o, *a, *d, *part;
  unsigned long long* ctr;    // end-of-step count: arrivals since the scratch was zeroed
  unsigned long long* kmax;   // running argmax key of the step (reset by the last arriver)
  unsigned int* bar;          // [2] sticky abort flag, [3] trace switch, [4] completed launches
  unsigned long long* trace;  // optional: per CTA, tagged %globaltimer stamps
  int* err;
};

// The GEMV input vector, quantised per 32-value group (q4_dot.cuh's XGroup,
// stored structure-of-arrays so that lanes reading consecutive groups hit
// consecutive banks): w[0..3] hi bytes of even values, w[4..7] hi odd, w[8..11]
// lo even, w[12..15] lo odd, then -8 * sum and the group's scale.
struct XQ {
  uint32_t w[16][kMaxG];
  int bias[kMaxG];
  float sx[kMaxG];
};

// This CTA's rows [r0, r1) of an N x K matrix and the rows per ring stage.
struct Seg {
  int r0, r1, rs;
  int kslog, sg;  // GEMV layout: log2 of the K slices per row, groups per slice
};
// the matrices a CTA streams: per layer q|k|v, o, gate|up, down; then the lm_head
enum { M_QKV = 0, M_O = 1, M_GU = 2, M_DOWN = 3, M_HEAD = 4, kMats = 5 };

struct Smem {
  uint8_t w[kRing][kStageW];
  uint8_t s[kRing][kStageS];
  Layer layers[kMaxLayers];
  XQ xq;
  float vb[kMaxH];           // q heads in the attention phase
  float kv[2][CKA][HD];      // K and V rows of one attention chunk; merge scratch
  float qn[HD], kn[HD];      // q / k norm weights
  float cs[HD / 2], sn[HD / 2];  // RoPE row of this position
  float kpos[HD], vpos[HD];  // k and v of this position
  float ps[CKA][kMaxHeads];  // chunk softmax numerators, key-major (a key's heads in two float4)
  float red[2][kRed];
  float seg_out[kSegOut];
  float resid[kMaxH];        // this CTA's copy of the residual stream
  Seg seg[kMats];            // this CTA's rows of each matrix (segment, gemv_layout)
  unsigned long long best[8];
  uint64_t full[kRing];
  uint64_t empty[kRing];
  uint64_t kvbar;
  int flag;
  unsigned int trace_n;
  Params prm;  // the launch parameters, for the out-of-line phase functions
};

static_assert(sizeof(Smem) <= 227 * 1024, "one CTA's shared memory");

// The CTA's shared memory.  Out-of-line functions take it (and the launch
// parameters) from here rather than through a pointer argument, so their
// accesses compile to shared-memory instructions, not generic ones.
__device__ __forceinline__ Smem& smem() {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  return *reinterpret_cast<Smem*>(smem_raw);
}

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Epoch-tagged words (see the file comment): value bits low, epoch high.
__device__ __forceinline__ uint64_t ll_pack(float v, uint32_t ep) {
  return (static_cast<uint64_t>(ep) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }
__device__ __forceinline__ bool ll_is(uint64_t w, uint32_t ep) { return static_cast<uint32_t>(w >> 32) == ep; }
__device__ __forceinline__ void ll_st(uint64_t* p, float v, uint32_t ep) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(ll_pack(v, ep)) : "memory");
}
__device__ __forceinline__ void ll_st2(uint64_t* p, float a, float b, uint32_t ep) {
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(ll_pack(a, ep)), "l"(ll_pack(b, ep))
               : "memory");
}
__device__ __forceinline__ uint64_t ll_ld(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p));
  return w;
}
// p 16-byte aligned; each 64-bit element is a single-copy-atomic access
__device__ __forceinline__ void ll_ld2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p));
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
// consumer barrier that also ORs a flag over the consumer threads
__device__ __forceinline__ bool cons_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kCons)
      : "memory");
  return r != 0;
}

// sum (or max) over the consumer threads
template <bool MAX>
__device__ float cons_reduce(float v, Smem& sm) {
  v = MAX ? warp_max(v) : warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  cons_sync();
  if (lane == 0) sm.red[0][warp] = v;
  cons_sync();
  const float t = lane < kCons / 32 ? sm.red[0][lane] : (MAX ? -INFINITY : 0.f);
  return MAX ? warp_max(t) : warp_sum(t);
}

__device__ __forceinline__ bool aborted(const Params& p) {
  return *reinterpret_cast<volatile const unsigned int*>(p.bar + 2) != 0;
}

__device__ __forceinline__ void raise_abort(const Params& p) {
  atomicExch(p.bar + 2, 1u);
  atomicExch(p.err, SB_ERR_TIMEOUT);
}

// The abort flag is an L2 round trip: poll it only once a wait has lasted this
// long, so normal waits wake up as soon as their condition holds.
constexpr uint64_t kAbortPollNs = 20000;

// mbarrier wait that also gives up when another CTA raised the abort flag.
// `fail` is the calling thread's sticky failure flag: once set, waits return
// false at once, so a failing CTA runs through the rest of its phase (on
// garbage, still joining every consumer barrier) to the next grid barrier,
// where the consumers agree to leave together.
__device__ bool ring_wait(uint64_t* bar, uint32_t parity, const Params& p, bool& fail) {
  if (fail) return false;
  if (sbd::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = sbd::global_ns();
  while (!sbd::mbar_try_wait(bar, parity)) {
    const uint64_t dt = sbd::global_ns() - t0;
    if (dt > kAbortPollNs && aborted(p)) {
      fail = true;
      return false;
    }
    if (dt > sbd::kWaitLimitNs) {
      raise_abort(p);
      fail = true;
      return false;
    }
  }
  return true;
}

// Trace stamp by thread 0 of a CTA: (tag << 56) | %globaltimer.
enum { TR_ENTRY = 1, TR_ARRIVE = 2, TR_EXIT = 3, TR_INPUT = 4, TR_STAGE0 = 5, TR_GEMV = 6, TR_ATT_Q = 7,
       TR_ATT_K = 8, TR_ATT_S = 9, TR_ATT_PV = 10, TR_ROWS0 = 11, TR_FREE0 = 12 };
// The count lives in shared memory (a global read per stamp would distort the
// intervals being measured) and is written out as entry 0 at every stamp.
__device__ void trace_stamp(const Params& p, unsigned int tag) {
  if (p.trace && threadIdx.x == 0) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    unsigned int& n = reinterpret_cast<Smem*>(smem_raw)->trace_n;
    unsigned long long* t = p.trace + static_cast<size_t>(blockIdx.x) * kTraceLen;
    if (n + 1 < kTraceLen) {
      ++n;
      t[n] = (static_cast<unsigned long long>(tag) << 56) | (sbd::global_ns() & ((1ull << 56) - 1));
      t[0] = n;
    }
  }
}

// End of a phase: the consumer threads of the CTA agree whether any of them
// failed (a wait that ran out or saw the abort flag).  If so the CTA raises the
// abort flag -- which ends every other CTA's waits within kAbortPollNs -- and
// leaves; false for every consumer thread.  No other CTA is waited for here:
// the next phase waits on its own input words.
__device__ __forceinline__ bool phase_end(bool& fail) {
  if (cons_sync_or(fail)) {
    if (threadIdx.x == 0) raise_abort(smem().prm);
    fail = true;
    return false;
  }
  return true;
}

// One more round of an input poll?  Starts the clock on the first miss; past
// kAbortPollNs also checks the abort flag, past the wait limit raises it.
// false (and `fail` set) when the wait must end.
__device__ __forceinline__ bool poll_again(const Params& p, uint64_t& t0, bool& fail) {
  if (fail) return false;
  if (t0 == 0) {
    t0 = sbd::global_ns();
    return true;
  }
  const uint64_t dt = sbd::global_ns() - t0;
  if (dt > kAbortPollNs && aborted(p)) {
    fail = true;
    return false;
  }
  if (dt > sbd::kWaitLimitNs) {
    raise_abort(p);
    fail = true;
    return false;
  }
  return true;
}

// Loads of a thread's slots of an epoch-tagged vector: slot s = tid + ps *
// kCons holds values [8 s, 8 s + 8); beyond n a word reads as epoch ep, 0.f.
template <int NP>
__device__ __forceinline__ void ll_issue(uint64_t (&w)[NP][8], const uint64_t* src, int n, uint32_t ep) {
#pragma unroll
  for (int ps = 0; ps < NP; ++ps) {
    const int s = threadIdx.x + ps * kCons;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (8 * s < n) ll_ld2(src + 8 * s + 2 * q, w[ps][2 * q], w[ps][2 * q + 1]);
      else w[ps][2 * q] = w[ps][2 * q + 1] = static_cast<uint64_t>(ep) << 32;
    }
  }
}
template <int NP>
__device__ __forceinline__ bool ll_take(const uint64_t (&w)[NP][8], float (&v)[NP][8], uint32_t ep) {
  bool ok = true;
#pragma unroll
  for (int ps = 0; ps < NP; ++ps)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ok &= ll_is(w[ps][i], ep);
      v[ps][i] = ll_val(w[ps][i]);
    }
  return ok;
}

// v[ps][0..8) <- values [8 s, 8 s + 8) of the epoch-tagged vector src, s = tid
// + ps * kCons, once every one of those words carries epoch ep (zeros beyond
// n).  All of the thread's loads are in flight before any is tested.  (Two
// polls in flight, staggered by half a round trip, measured slower: the extra
// L2 traffic lengthens every other CTA's wait.)
template <int NP>
__device__ __forceinline__ void ll_slots(float (&v)[NP][8], const uint64_t* src, int n, uint32_t ep, bool& fail) {
  const Params& p = smem().prm;
  uint64_t t0 = 0;
  for (;;) {
    uint64_t w[NP][8];
    ll_issue<NP>(w, src, n, ep);
    if (ll_take<NP>(w, v, ep) || !poll_again(p, t0, fail)) return;
  }
}

// ---------------------------------------------------------------- weight segments
// Rows are dealt in pairs (gate/up rows stay together), as evenly as the pair
// count allows: CTA b gets pairs [b P / G, (b + 1) P / G).
// Computed once per launch (sm.seg); the GEMV layout fields are set by gemv_layout.
__device__ __forceinline__ Seg segment(int n, int k) {
  const long long pairs = (n + 1) / 2, g = gridDim.x, b = blockIdx.x;
  Seg s;
  s.r0 = min(n, static_cast<int>(2 * (b * pairs / g)));
  s.r1 = min(n, static_cast<int>(2 * ((b + 1) * pairs / g)));
  const int per = 2 * static_cast<int>((pairs + g - 1) / g);
  s.rs = max(1, min(per, kStageW / (k / 2)));
  s.rs = min(s.rs, kStageS / (k / 16));
  s.kslog = 0;
  s.sg = 0;
  return s;
}

// GEMV work split: 16 half-warps, each lane owning GPL 32-value groups of
// one of `ks` K slices, so 16 * GPL * ks >= K / 32.  Two shapes of code (GPL 3
// for K = 1536 and 6144, GPL 4 for K = 2048, both without idle lanes) serve
// every matrix of the model.
__device__ __forceinline__ int gpl_for(int k) { return (k / 32) % 64 == 0 && k / 32 <= 64 ? 4 : 3; }
__device__ __forceinline__ int ks_for(int k, int gpl) {
  int ks = 1;
  while (16 * gpl * ks < k / 32) ks *= 2;
  return ks;
}
__device__ __forceinline__ Seg gemv_layout(int n, int k) {
  Seg s = segment(n, k);
  const int ks = ks_for(k, gpl_for(k));
  s.kslog = __ffs(ks) - 1;
  s.sg = (k / 32 + ks - 1) / ks;
  return s;
}

// producer: stream one matrix's slice through the ring
__device__ bool produce(const Params& p, Smem& sm, const uint8_t* w, const __half* s, int mat, int k, int& it,
                        bool& fail) {
  const Seg sg = sm.seg[mat];
  const int rb = k / 2, sb = k / 16;
  const uint64_t pol = sbd::l2_policy_evict_first();
  for (int r = sg.r0; r < sg.r1; r += sg.rs) {
    const int nr = min(sg.rs, sg.r1 - r);
    const int slot = it % kRing;
    if (!ring_wait(&sm.empty[slot], ((it / kRing) & 1) ^ 1, p, fail)) return false;
    sbd::mbar_arrive_expect_tx(&sm.full[slot], static_cast<uint32_t>(nr) * (rb + sb));
    sbd::bulk_load_hint(sm.w[slot], w + static_cast<size_t>(r) * rb, static_cast<uint32_t>(nr) * rb,
                        &sm.full[slot], pol);
    sbd::bulk_load_hint(sm.s[slot], reinterpret_cast<const uint8_t*>(s) + static_cast<size_t>(r) * sb,
                        static_cast<uint32_t>(nr) * sb, &sm.full[slot], pol);
    ++it;
  }
  return true;
}

enum { EPI_STORE = 0, EPI_SEGOUT = 1, EPI_ARGMAX = 2 };

// Consumer state carried across phases.
struct Cursor {
  int it;             // ring stages consumed
  float best_v;       // lm_head: running max ...
  long long best_i;   // ... and its row
  bool fail;          // sticky failure (see ring_wait)
  uint32_t ep;        // epoch of the current (launch, layer): tags the words this CTA stores
};

// consumers: GEMV of this CTA's rows of one matrix over the quantised input
// sm.xq (K values).  epi: EPI_STORE (out[row], an epoch-tagged word), EPI_SEGOUT (sm.seg_out) or
// EPI_ARGMAX (running max / lowest row).  Each half-warp works on two rows at
// a time (independent dot chains).  A failed ring wait leaves garbage in this
// CTA's results; the next grid barrier turns it into an abort.
template <int GPL>
__device__ __noinline__ void gemv_phase_t(int mat, int k, int epi, uint64_t* out, Cursor& cur) {
  Smem& sm = smem();
  const Params& p = sm.prm;
  const int tid = threadIdx.x, hw = tid >> 4, l16 = tid & 15;
  const Seg sg = sm.seg[mat];
  const int ks = 1 << sg.kslog;
  const int G = k / 32;
  const int SG = sg.sg;
  const int kslice = hw & (ks - 1), rlane = hw >> sg.kslog, nrl = 16 >> sg.kslog;
  const int gb = kslice * SG, ge = min(G, gb + SG);
  int it = cur.it;
  float best_v = cur.best_v;
  long long best_i = cur.best_i;
  bool fail = cur.fail;
  sbd::XGroup xg[GPL];
  int gidx[GPL];
  bool gval[GPL];
#pragma unroll
  for (int u = 0; u < GPL; ++u) {
    gidx[u] = gb + l16 + 16 * u;
    gval[u] = gidx[u] < ge;
    const int g = gval[u] ? gidx[u] : 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      xg[u].he[j] = sm.xq.w[j][g];
      xg[u].ho[j] = sm.xq.w[4 + j][g];
      xg[u].le[j] = sm.xq.w[8 + j][g];
      xg[u].lo[j] = sm.xq.w[12 + j][g];
    }
    xg[u].bias = sm.xq.bias[g];
    xg[u].sx = sm.xq.sx[g];
  }
  trace_stamp(p, TR_INPUT);
  const int rb = k / 2;
  auto put = [&](int row, float v) {
    if (epi == EPI_STORE) {
      ll_st(out + row, v, cur.ep);
    } else if (epi == EPI_SEGOUT) {
      sm.seg_out[row - sg.r0] = v;
    } else {
      if (v != v) v = -INFINITY;
      if (v > best_v || (v == best_v && row < best_i)) {
        best_v = v;
        best_i = row;
      }
    }
  };
  for (int r = sg.r0; r < sg.r1; r += sg.rs) {
    const int nr = min(sg.rs, sg.r1 - r);
    const int slot = it % kRing;
    ring_wait(&sm.full[slot], (it / kRing) & 1, p, fail);
    if (r == sg.r0) trace_stamp(p, TR_STAGE0);
    float* red = sm.red[it & 1];
    const uint8_t* wst = sm.w[slot];
    const __half* sst = reinterpret_cast<const __half*>(sm.s[slot]);
    for (int r0 = rlane; r0 < nr; r0 += 2 * nrl) {
      const int r1 = r0 + nrl;
      const bool has1 = r1 < nr;
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int u = 0; u < GPL; ++u) {
        if (!gval[u]) continue;
        const uint4 q0 = *reinterpret_cast<const uint4*>(wst + r0 * rb + gidx[u] * 16);
        const uint4 q1 = has1 ? *reinterpret_cast<const uint4*>(wst + r1 * rb + gidx[u] * 16) : q0;
        const float s0 = __half2float(sst[r0 * G + gidx[u]]);
        const float s1 = has1 ? __half2float(sst[r1 * G + gidx[u]]) : 0.f;
        acc0 = fmaf(static_cast<float>(sbd::dot_group(q0, xg[u])), s0 * xg[u].sx, acc0);
        acc1 = fmaf(static_cast<float>(sbd::dot_group(q1, xg[u])), s1 * xg[u].sx, acc1);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) {
        acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, off, 16);
        acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, off, 16);
      }
      if (l16 == 0) {
        if (ks == 1) {  // the half-warp holds whole rows
          put(r + r0, acc0);
          if (has1) put(r + r1, acc1);
        } else {
          red[r0 * ks + kslice] = acc0;
          if (has1) red[r1 * ks + kslice] = acc1;
        }
      }
    }
    if (r == sg.r0) trace_stamp(p, TR_ROWS0);
    __syncwarp();
    if ((tid & 31) == 0) sbd::mbar_arrive(&sm.empty[slot]);
    if (ks > 1) {
      cons_sync();
      for (int e = tid; e < nr; e += kCons) {
        float v = 0.f;
        for (int q = 0; q < ks; ++q) v += red[e * ks + q];
        put(r + e, v);
      }
    }
    if (r == sg.r0) trace_stamp(p, TR_FREE0);
    ++it;
  }
  trace_stamp(p, TR_GEMV);
  cur.it = it;
  cur.best_v = best_v;
  cur.best_i = best_i;
  cur.fail = fail;
}

__device__ __forceinline__ void gemv_phase(int mat, int k, int epi, uint64_t* out, Cursor& cur) {
  if (gpl_for(k) == 4)
    gemv_phase_t<4>(mat, k, epi, out, cur);
  else
    gemv_phase_t<3>(mat, k, epi, out, cur);
}

// ---------------------------------------------------------------- phase inputs
// A phase input of n values (n % 32 == 0) is held as 8-value slots: slot
// s = tid + pass * kCons covers values [8 s, 8 s + 8), so the 4 slots of a
// 32-value group are lanes 4k .. 4k + 3 of one warp.  Each thread loads all of
// its slots before using any (one global round trip per phase input), and the
// group is quantised exactly as sbd::quantise_group does, with the group max
// and integer sum combined over the 4 lanes.

// Quantise slot s (all 32 lanes call this; slots at or beyond n only join the
// shuffles) into sm.xq.
__device__ __forceinline__ void quantise_slot(Smem& sm, int s, int n, const float (&v)[8]) {
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
  // fast reciprocal (<= 2 ulp): x * inv stays below 32767.5, and the scale
  // below is the same factor's inverse up to rounding, both far inside the
  // 2^-16 quantisation step
  const float inv = mx > 0.f ? __fdividef(32767.f, mx) : 0.f;
  int sum = 0;
  uint32_t he = 0, ho = 0, le = 0, lo = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int xe = __float2int_rn(v[2 * i] * inv);
    const int xo = __float2int_rn(v[2 * i + 1] * inv);
    sum += xe + xo;
    he |= (static_cast<uint32_t>(xe >> 8) & 0xFFu) << (8 * i);
    ho |= (static_cast<uint32_t>(xo >> 8) & 0xFFu) << (8 * i);
    le |= (static_cast<uint32_t>(xe) & 0xFFu) << (8 * i);
    lo |= (static_cast<uint32_t>(xo) & 0xFFu) << (8 * i);
  }
  sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
  sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
  if (8 * s < n) {
    const int g = s >> 2, q = s & 3;
    sm.xq.w[q][g] = he;
    sm.xq.w[4 + q][g] = ho;
    sm.xq.w[8 + q][g] = le;
    sm.xq.w[12 + q][g] = lo;
    if (q == 0) {
      sm.xq.bias[g] = -8 * sum;
      sm.xq.sx[g] = mx * (1.f / 32767.f);
    }
  }
}

__device__ __forceinline__ void ld8(float (&v)[8], const float* src, int s, bool in, bool coherent) {
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
  if (in) {
    const float4* q = reinterpret_cast<const float4*>(src) + 2 * s;
    a = coherent ? __ldcg(q) : __ldg(q);
    b = coherent ? __ldcg(q + 1) : __ldg(q + 1);
  }
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ float sumsq8(const float (&v)[8]) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  return ss;
}

// sm.xq <- quantise(RMSNorm(v) * w) for a hidden-sized v held one slot per
// thread (values [8 tid, 8 tid + 8)); with `keep`, v also becomes this CTA's
// residual stream (sm.resid).
__device__ void finish_norm(const Params& p, Smem& sm, int n, float (&v)[8], const float (&w)[8], bool keep) {
  // one reciprocal, then multiplies: eight IEEE divides per thread cost more
  // than the rest of the prologue (differs from v / dnm by at most an ulp)
  const float inv = 1.f / sqrtf(cons_reduce<false>(sumsq8(v), sm) / n + p.eps);
  const int s = threadIdx.x;
  if (keep && 8 * s < n) {
    float4* k4 = reinterpret_cast<float4*>(sm.resid) + 2 * s;
    k4[0] = make_float4(v[0], v[1], v[2], v[3]);
    k4[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * w[i];
  quantise_slot(sm, s, n, v);
  cons_sync();
}

// Wait for the epoch-ep words of the hidden-sized y (another phase's output),
// then resid += RMSNorm(y) * w_res and sm.xq <- quantise(RMSNorm(resid) *
// w_norm) (keep: the sum becomes the residual; the final norm does not need it).
__device__ __noinline__ void residual_norm(int n, const uint64_t* y, uint32_t ep, const float* w_res,
                                          const float* w_norm, bool keep, bool& fail) {
  Smem& sm = smem();
  const Params& p = sm.prm;
  const int s = threadIdx.x;
  const bool in = 8 * s < n;
  float v[8], yv[1][8], wr[8], wn[8];
  ld8(wr, w_res, s, in, false);
  ld8(wn, w_norm, s, in, false);
  trace_stamp(p, TR_ARRIVE);
  ll_slots<1>(yv, y, n, ep, fail);
  trace_stamp(p, TR_EXIT);
  if (in) {
    const float4* r4 = reinterpret_cast<const float4*>(sm.resid) + 2 * s;
    const float4 r0 = r4[0], r1 = r4[1];
    v[0] = r0.x; v[1] = r0.y; v[2] = r0.z; v[3] = r0.w;
    v[4] = r1.x; v[5] = r1.y; v[6] = r1.z; v[7] = r1.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  const float inv = 1.f / sqrtf(cons_reduce<false>(sumsq8(yv[0]), sm) / n + p.eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = v[i] + yv[0][i] * inv * wr[i];
  finish_norm(p, sm, n, v, wn, keep);
}

// sm.xq <- quantise(src[0, n)), once every word carries epoch ep
__device__ __noinline__ void load_input(int n, const uint64_t* src, uint32_t ep, bool& fail) {
  Smem& sm = smem();
  float v[kPasses][8];
  trace_stamp(sm.prm, TR_ARRIVE);
  ll_slots<kPasses>(v, src, n, ep, fail);
  trace_stamp(sm.prm, TR_EXIT);
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps)
    if (ps * 8 * kCons < n) quantise_slot(sm, threadIdx.x + ps * kCons, n, v[ps]);
  cons_sync();
}

// Prefetch into L2 the norm vectors of layer `li` (the final norm when li ==
// n_layers): threads 0..5 of every CTA, one 128-byte line each per CTA index.
__device__ void prefetch_norms(const Params& p, int li) {
  const int tid = threadIdx.x;
  if (tid >= 6 || li > p.n_layers) return;
  const float* v = nullptr;
  int lines = p.H / 32;
  if (li < p.n_layers) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Layer& N = reinterpret_cast<Smem*>(smem_raw)->layers[li];
    v = tid == 0 ? N.in_norm : tid == 1 ? N.post_attn : tid == 2 ? N.pre_ffn : tid == 3 ? N.post_ffn
      : tid == 4 ? N.q_norm : N.k_norm;
    if (tid >= 4) lines = HD / 32;
  } else if (tid == 0) {
    v = p.final_norm;
  }
  if (!v) return;
  for (int l = blockIdx.x; l < lines; l += gridDim.x) prefetch_l2(v + 32 * l);
}

// ---------------------------------------------------------------- attention
// Thread 0: start the bulk copy of chunk c's K and V rows that precede this
// position (row `pos` itself is produced in this step) and, with `consts`, the
// q/k norm weights and this position's RoPE row, completing on sm.kvbar.
__device__ void kv_issue(const Params& p, Smem& sm, const Layer& L, int c, int pos, bool consts,
                         uint32_t& issued) {
  ++issued;
  const int t0 = c * CKA;
  const int nk = max(0, min(CKA, pos - t0));
  uint32_t bytes = 2u * static_cast<uint32_t>(nk) * HD * 4;
  if (consts) bytes += 3u * HD * 4;
  sbd::fence_proxy_async_smem();
  sbd::mbar_arrive_expect_tx(&sm.kvbar, bytes);
  if (nk) {
    sbd::bulk_load(sm.kv[0], L.kc + static_cast<size_t>(t0) * HD, nk * HD * 4, &sm.kvbar);
    sbd::bulk_load(sm.kv[1], L.vc + static_cast<size_t>(t0) * HD, nk * HD * 4, &sm.kvbar);
  }
  if (consts) {
    sbd::bulk_load(sm.qn, L.q_norm, HD * 4, &sm.kvbar);
    sbd::bulk_load(sm.kn, L.k_norm, HD * 4, &sm.kvbar);
    sbd::bulk_load(sm.cs, p.cos_t + static_cast<size_t>(pos) * (HD / 2), HD / 2 * 4, &sm.kvbar);
    sbd::bulk_load(sm.sn, p.sin_t + static_cast<size_t>(pos) * (HD / 2), HD / 2 * 4, &sm.kvbar);
  }
}

// q heads (and k, v of this position when `own`): RMSNorm (weights for q, k;
// none for v), RoPE on q and k; q to sm.vb, k / v to the cache and sm.kpos / vpos.
// A warp takes heads warp and warp + 8 and waits for both heads' epoch-ep
// words of the q|k|v output with all of its loads in flight at once.
__device__ void qkv_heads(const Params& p, Smem& sm, const Layer& L, int pos, bool own, uint32_t ep,
                          bool& fail) {
  const int nh = p.nh, qd = nh * HD, nhead = nh + (own ? 2 : 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  static_assert(kMaxHeads + 2 <= 2 * (kCons / 32), "two heads per warp");
  float vv[2][8];
  {
    uint64_t t0 = 0;
    for (;;) {
      uint64_t w[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int h = warp + u * (kCons / 32);
        const int col = h < nh ? h * HD : (h == nh ? qd : qd + HD);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          w[u][j] = h < nhead ? ll_ld(p.qkv + col + lane + 32 * j) : static_cast<uint64_t>(ep) << 32;
      }
      bool ok = true;
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ok &= ll_is(w[u][j], ep);
          vv[u][j] = ll_val(w[u][j]);
        }
      if (__all_sync(0xFFFFFFFFu, ok)) break;
      // warp-uniform exit: a lane whose wait ended (fail set) ends the warp's
      if (!__all_sync(0xFFFFFFFFu, poll_again(p, t0, fail))) break;
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int h = warp + u * (kCons / 32);
    if (h >= nhead) break;
    float* v = vv[u];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
    const float inv = 1.f / sqrtf(warp_sum(ss) / HD + p.eps);
    const float* w = h < nh ? sm.qn : sm.kn;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = h <= nh ? v[j] * inv * w[lane + 32 * j] : v[j] * inv;
    if (h <= nh) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = lane + 32 * j;
        const float a = v[j], b = v[j + 4];
        v[j] = a * sm.cs[i] - b * sm.sn[i];
        v[j + 4] = b * sm.cs[i] + a * sm.sn[i];
      }
    }
    if (h < nh) {
#pragma unroll
      for (int j = 0; j < 8; ++j) sm.vb[h * HD + lane + 32 * j] = v[j];
    } else {
      float* cache = (h == nh ? L.kc : L.vc) + static_cast<size_t>(pos) * HD;
      float* keep = h == nh ? sm.kpos : sm.vpos;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cache[lane + 32 * j] = v[j];
        keep[lane + 32 * j] = v[j];
      }
    }
  }
}

// Chunk c's scores, softmax partials (max, sum) and P.V partials from sm.kv,
// stored as epoch-ep words.
__device__ void attn_chunk(const Params& p, Smem& sm, int c, int pos, uint32_t ep) {
  const int nh = p.nh;
  const int T = pos + 1, t0 = c * CKA, nt = min(CKA, T - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // scores: warp per head; lane holds dims [4 lane, 4 lane + 4) and [128 + 4 lane, ...)
  for (int h = warp; h < nh; h += kCons / 32) {
    const float4 q0 = reinterpret_cast<const float4*>(sm.vb + h * HD)[lane];
    const float4 q1 = reinterpret_cast<const float4*>(sm.vb + h * HD)[32 + lane];
    // two halves of 8 keys; each half's 8 per-lane partial sums are
    // reduce-scattered over the warp (xor 16, 8, 4) so that lane holds key
    // (lane >> 2) & 7 of the half, then completed over the 4 lanes sharing it
    float sc[2];
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      float s[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float4 k0 = reinterpret_cast<const float4*>(sm.kv[0][hb * 8 + t])[lane];
        const float4 k1 = reinterpret_cast<const float4*>(sm.kv[0][hb * 8 + t])[32 + lane];
        s[t] = q0.x * k0.x + q0.y * k0.y + q0.z * k0.z + q0.w * k0.w + q1.x * k1.x + q1.y * k1.y +
               q1.z * k1.z + q1.w * k1.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool up = lane & 16;
        const float send = up ? s[i] : s[i + 4];
        s[i] = (up ? s[i + 4] : s[i]) + __shfl_xor_sync(0xFFFFFFFFu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const bool up = lane & 8;
        const float send = up ? s[i] : s[i + 2];
        s[i] = (up ? s[i + 2] : s[i]) + __shfl_xor_sync(0xFFFFFFFFu, send, 8);
      }
      {
        const bool up = lane & 4;
        const float send = up ? s[0] : s[1];
        s[0] = (up ? s[1] : s[0]) + __shfl_xor_sync(0xFFFFFFFFu, send, 4);
      }
      s[0] += __shfl_xor_sync(0xFFFFFFFFu, s[0], 2);
      s[0] += __shfl_xor_sync(0xFFFFFFFFu, s[0], 1);
      sc[hb] = s[0];
    }
    const int key = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    const bool v0 = key < nt, v1 = key + 8 < nt;
    const float m = warp_max(fmaxf(v0 ? sc[0] : -INFINITY, v1 ? sc[1] : -INFINITY));
    const float p0 = v0 ? expf(sc[0] - m) : 0.f;
    const float p1 = v1 ? expf(sc[1] - m) : 0.f;
    const float l = warp_sum((lane & 3) ? 0.f : p0 + p1);
    if (!(lane & 3)) {
      sm.ps[key][h] = p0;
      sm.ps[key + 8][h] = p1;
    }
    if (lane == 0) ll_st2(p.part + (static_cast<size_t>(c) * nh + h) * (HD + 2) + HD, m, l, ep);
  }
  cons_sync();
  trace_stamp(p, TR_ATT_S);
  // P.V: thread per head dim
  {
    const int dcol = threadIdx.x;
    float acc[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) acc[h] = 0.f;
    // two keys per iteration, each key's eight numerators in two broadcast
    // float4 loads; kept rolled (this code runs once per layer, and straight-
    // line code costs instruction fetches from L2 every time).  A key past nt
    // has numerator 0 and its V row is not read.
    static_assert(kMaxHeads == 8, "a key's numerators are two float4");
#pragma unroll 1
    for (int t = 0; t < nt; t += 2) {
      const float v0 = sm.kv[1][t][dcol];
      const float v1 = t + 1 < nt ? sm.kv[1][t + 1][dcol] : 0.f;
      const float4* p4 = reinterpret_cast<const float4*>(&sm.ps[t][0]);
      const float4 a0 = p4[0], a1 = p4[1], b0 = p4[2], b1 = p4[3];
      const float pa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float pb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) acc[h] = fmaf(pb[h], v1, fmaf(pa[h], v0, acc[h]));
    }
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h)
      if (h < nh) ll_st(p.part + (static_cast<size_t>(c) * nh + h) * (HD + 2) + dcol, acc[h], ep);
  }
  trace_stamp(p, TR_ATT_PV);
}

// The attention phase: this CTA's chunks c = blockIdx.x, + gridDim.x, ...
// The first chunk's copy was started in the qkv phase (kv_issue with consts).
// kvph counts completed waits on sm.kvbar, issued (thread 0) the copies started.
__device__ void attention(const Params& p, Smem& sm, const Layer& L, int pos, int nc, uint32_t ep,
                          uint32_t& kvph, uint32_t& issued, bool& fail) {
  const int cpos = pos / CKA;
  const bool own = cpos % static_cast<int>(gridDim.x) == static_cast<int>(blockIdx.x);
  for (int c = blockIdx.x; c < nc; c += gridDim.x) {
    if (c != static_cast<int>(blockIdx.x)) {
      cons_sync();  // every thread is done with the previous chunk's rows
      if (threadIdx.x == 0 && !fail) kv_issue(p, sm, L, c, pos, false, issued);
    }
    if (ring_wait(&sm.kvbar, kvph & 1, p, fail)) ++kvph;
    if (c == static_cast<int>(blockIdx.x)) {
      trace_stamp(p, TR_ARRIVE);
      qkv_heads(p, sm, L, pos, own, ep, fail);
      cons_sync();
      trace_stamp(p, TR_EXIT);
      trace_stamp(p, TR_ATT_Q);
    }
    if (c == cpos) {
      sm.kv[0][pos - c * CKA][threadIdx.x] = sm.kpos[threadIdx.x];
      sm.kv[1][pos - c * CKA][threadIdx.x] = sm.vpos[threadIdx.x];
    }
    cons_sync();
    trace_stamp(p, TR_ATT_K);
    attn_chunk(p, sm, c, pos, ep);
  }
}

// Merge of the chunk partials: work item (head, kMergeDims dims).  Waits on
// the partials' epoch-ep words (batches of 8 loads in flight per thread) and
// stores the attention output as epoch-ep words.  A CTA without a work item
// stamps an empty wait so that every CTA's trace has the same phases.
__device__ void merge(const Params& p, Smem& sm, int nc, uint32_t ep, bool& fail) {
  const int nh = p.nh, tid = threadIdx.x;
  constexpr int NG = kCons / kMergeDims;  // chunk groups summed in parallel
  constexpr int B = 8;                    // loads in flight per thread and poll
  const int items = nh * (HD / kMergeDims);
  const size_t cst = static_cast<size_t>(nh) * (HD + 2);
  float* ms = &sm.kv[0][0][0];      // the K/V chunk buffer is free until the next layer
  float* fv = ms;                   // [nc] chunk max, then weight
  float* lv = ms + kMaxChunks;      // [nc] chunk sum
  float* rv = ms + 2 * kMaxChunks;  // [NG][kMergeDims]
  if (static_cast<int>(blockIdx.x) >= items) {
    trace_stamp(p, TR_ARRIVE);
    trace_stamp(p, TR_EXIT);
  }
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int h = item / (HD / kMergeDims), d0 = (item % (HD / kMergeDims)) * kMergeDims;
    const uint64_t* base = p.part + static_cast<size_t>(h) * (HD + 2);
    if (item == static_cast<int>(blockIdx.x)) trace_stamp(p, TR_ARRIVE);
    float mx = -INFINITY;
    for (int c0 = tid; c0 < nc; c0 += B * kCons) {
      uint64_t t0 = 0;
      for (;;) {
        uint64_t wm[B], wl[B];
#pragma unroll
        for (int i = 0; i < B; ++i) {
          const int c = c0 + i * kCons;
          if (c < nc) ll_ld2(base + c * cst + HD, wm[i], wl[i]);
          else wm[i] = wl[i] = static_cast<uint64_t>(ep) << 32;
        }
        bool ok = true;
#pragma unroll
        for (int i = 0; i < B; ++i) ok &= ll_is(wm[i], ep) && ll_is(wl[i], ep);
        if (ok || !poll_again(p, t0, fail)) {
#pragma unroll
          for (int i = 0; i < B; ++i) {
            const int c = c0 + i * kCons;
            if (c < nc) {
              fv[c] = ll_val(wm[i]);
              lv[c] = ll_val(wl[i]);
              mx = fmaxf(mx, ll_val(wm[i]));
            }
          }
          break;
        }
      }
    }
    mx = cons_reduce<true>(mx, sm);
    if (item == static_cast<int>(blockIdx.x)) trace_stamp(p, TR_EXIT);
    float ls = 0.f;
    for (int c = tid; c < nc; c += kCons) {
      const float f = expf(fv[c] - mx);
      ls += lv[c] * f;
      fv[c] = f;
    }
    ls = cons_reduce<false>(ls, sm);  // its barriers also publish fv
    const int dd = tid % kMergeDims, g = tid / kMergeDims;
    float acc = 0.f;
    for (int c0 = g; c0 < nc; c0 += B * NG) {
      uint64_t t0 = 0;
      for (;;) {
        uint64_t w[B];
#pragma unroll
        for (int i = 0; i < B; ++i) {
          const int c = c0 + i * NG;
          w[i] = c < nc ? ll_ld(base + c * cst + d0 + dd) : static_cast<uint64_t>(ep) << 32;
        }
        bool ok = true;
#pragma unroll
        for (int i = 0; i < B; ++i) ok &= ll_is(w[i], ep);
        if (ok || !poll_again(p, t0, fail)) {
#pragma unroll
          for (int i = 0; i < B; ++i) {
            const int c = c0 + i * NG;
            if (c < nc) acc = fmaf(fv[c], ll_val(w[i]), acc);
          }
          break;
        }
      }
    }
    rv[g * kMergeDims + dd] = acc;
    cons_sync();
    if (tid < kMergeDims) {
      float o = 0.f;
      for (int q = 0; q < NG; ++q) o += rv[q * kMergeDims + tid];
      ll_st(p.attn + h * HD + d0 + tid, o / ls, ep);
    }
    cons_sync();
  }
}

using sbd::gelu_tanh;

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  if (p.bar[3] == 0 || blockIdx.x >= kTraceCtas) p.trace = nullptr;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  const int H = p.H, nh = p.nh, qd = nh * HD, nqkv = qd + 2 * HD, F = p.F;
  {
    // the layer table (pointers) into shared memory
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.layers);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(sm.layers);
    constexpr int kWords = sizeof(Layer) / 8;
    for (int i = tid; i < p.n_layers * kWords; i += kThreads) dst[i] = __ldg(src + i);
  }
  if (tid == 0) {
    sm.prm = p;
    sm.trace_n = 0;
    for (int i = 0; i < kRing; ++i) {
      sbd::mbar_init(&sm.full[i], 1);
      sbd::mbar_init(&sm.empty[i], kCons / 32);
    }
    sbd::mbar_init(&sm.kvbar, 1);
    sbd::fence_mbar_init();
    sbd::fence_proxy_async_smem();
  }
  if (tid >= 32 && tid < 32 + kMats) {
    // this CTA's rows and GEMV layout of each matrix, once per launch
    const int m = tid - 32;
    const int n = m == M_QKV ? nqkv : m == M_GU ? 2 * F : m == M_HEAD ? p.V : H;
    const int k = m == M_O ? qd : m == M_DOWN ? F : H;
    sm.seg[m] = gemv_layout(n, k);
  }
  __syncthreads();

  if (tid >= kCons) {
    // ------------------------------------------------------------ producer warp
    if (tid == kCons) {
      int it = 0;
      bool ok = true, pfail = false;
      for (int li = 0; li < p.n_layers && ok; ++li) {
        const Layer& L = sm.layers[li];
        ok = produce(p, sm, L.w[0], L.s[0], M_QKV, H, it, pfail) &&
             produce(p, sm, L.w[1], L.s[1], M_O, qd, it, pfail) &&
             produce(p, sm, L.w[2], L.s[2], M_GU, H, it, pfail) &&
             produce(p, sm, L.w[3], L.s[3], M_DOWN, F, it, pfail);
      }
      if (ok) ok = produce(p, sm, p.emb, p.emb_s, M_HEAD, H, it, pfail);
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
  trace_stamp(p, TR_ENTRY);
  const int pos = p.pos[0];
  const int nc = pos / CKA + 1;  // attention chunks
  // epochs of this launch: e0 + li tags layer li's words; launches completed
  // so far count up from the zeroed scratch (2^26 launches before a repeat)
  const uint32_t e0 = (__ldcg(p.bar + 4) & 0x3FFFFFFu) * 64u + 1u;
  Cursor cur{0, -INFINITY, 0x7FFFFFFF, false, e0};
  // an abort left by an earlier launch stays until the caller zeroes the scratch
  cur.fail = tid == 0 && aborted(p);
  bool& fail = cur.fail;
  uint32_t kvph = 0, kv_issued = 0;
  const bool has_chunk = static_cast<int>(blockIdx.x) < nc;
  bool ok = true;
  for (int li = 0; li < p.n_layers && ok; ++li) {
    const Layer& L = sm.layers[li];
    const uint32_t ep = e0 + li;
    // ---- qkv: start this layer's K/V chunk copy, layer input, RMSNorm, GEMV
    if (has_chunk && tid == 0 && !fail) kv_issue(p, sm, L, blockIdx.x, pos, true, kv_issued);
    prefetch_norms(p, li + 1);
    if (li == 0) {
      // embedding row: 8 values = one 32-bit word of nibbles (low nibble first)
      const int64_t tok = p.cur[0];
      const bool in = 8 * tid < H;
      const uint32_t wd = in ? __ldg(reinterpret_cast<const uint32_t*>(p.emb + tok * (H / 2)) + tid) : 0u;
      const float sc = in ? __half2float(__ldg(p.emb_s + tok * (H / 32) + tid / 4)) : 0.f;
      float v[8], wn[8];
      ld8(wn, L.in_norm, tid, in, false);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = static_cast<int>((wd >> (4 * i)) & 15u) - 8;
        v[i] = in ? __fmul_rn(__fmul_rn(static_cast<float>(q), sc), p.embed_scale) : 0.f;
      }
      finish_norm(p, sm, H, v, wn, true);
    } else {
      // x += RMSNorm(down of the previous layer) * its post-FFN norm
      residual_norm(H, p.d, ep - 1, sm.layers[li - 1].post_ffn, L.in_norm, true, fail);
    }
    cur.ep = ep;
    gemv_phase(M_QKV, H, EPI_STORE, p.qkv, cur);
    if (!(ok = phase_end(fail))) break;
    // ---- attention partials
    if (!has_chunk) {
      trace_stamp(p, TR_ARRIVE);
      trace_stamp(p, TR_EXIT);
    }
    attention(p, sm, L, pos, nc, ep, kvph, kv_issued, fail);
    if (!(ok = phase_end(fail))) break;
    // ---- merge
    merge(p, sm, nc, ep, fail);
    if (!(ok = phase_end(fail))) break;
    // ---- o projection
    load_input(qd, p.attn, ep, fail);
    gemv_phase(M_O, qd, EPI_STORE, p.o, cur);
    if (!(ok = phase_end(fail))) break;
    // ---- gate|up with GEGLU
    residual_norm(H, p.o, ep, L.post_attn, L.pre_ffn, true, fail);
    gemv_phase(M_GU, H, EPI_SEGOUT, nullptr, cur);
    cons_sync();
    {
      const Seg sg = sm.seg[M_GU];
      for (int i = tid; i < (sg.r1 - sg.r0) / 2; i += kCons)
        ll_st(p.a + sg.r0 / 2 + i, gelu_tanh(sm.seg_out[2 * i]) * sm.seg_out[2 * i + 1], ep);
    }
    if (!(ok = phase_end(fail))) break;
    // ---- down projection
    load_input(F, p.a, ep, fail);
    gemv_phase(M_DOWN, F, EPI_STORE, p.d, cur);
    ok = phase_end(fail);
  }
  if (!ok) {
    // a CTA that leaves early must still let its K/V copy land
    if (tid == 0 && kv_issued > kvph) {
      const uint64_t t0 = sbd::global_ns();
      while (!sbd::mbar_try_wait(&sm.kvbar, kvph & 1) && sbd::global_ns() - t0 < sbd::kWaitLimitNs) {
      }
    }
    return;
  }
  // ---- final norm + tied lm_head with argmax
  residual_norm(H, p.d, e0 + p.n_layers - 1, sm.layers[p.n_layers - 1].post_ffn, p.final_norm, false, fail);
  gemv_phase(M_HEAD, H, EPI_ARGMAX, nullptr, cur);
  {
    const int lane = tid & 31, warp = tid >> 5;
    unsigned long long key = 0ull;
    const long long bi = cur.best_i;
    if (bi != 0x7FFFFFFF) {
      float f = cur.best_v;
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
  }
  if (!phase_end(fail)) return;
  if (tid == 0) {
    // the step's argmax key; the CTA whose count completes the step decodes
    // the token (every other CTA's atomicMax is ordered before its count)
    trace_stamp(p, TR_ARRIVE);
    unsigned long long k2 = 0;
    for (int w = 0; w < kCons / 32; ++w) k2 = sm.best[w] > k2 ? sm.best[w] : k2;
    if (k2) atomicMax(p.kmax, k2);
    __threadfence();
    const unsigned long long old = atomicAdd(p.ctr, 1ull);
    trace_stamp(p, TR_EXIT);
    if ((old + 1) % gridDim.x == 0) {
      __threadfence();
      const unsigned long long kf = atomicExch(p.kmax, 0ull);  // read, and clear for the next step
      *p.keys = kf;
      const int32_t t = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(kf & 0xFFFFFFFFull));
      const int np = pos + 1;
      p.tok[0] = t;
      p.cur[0] = t;
      p.pos[0] = np;
      if (p.history && np < p.hist_len) p.history[np] = t;
      atomicAdd(p.bar + 4, 1u);  // the next launch's epochs
    }
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

constexpr size_t kHeaderBytes = 64 + static_cast<size_t>(kTraceCtas) * kTraceLen * sizeof(unsigned long long);

}  // namespace

extern "C" size_t sb_decode_step_fused_scratch_size(int hidden, int n_heads, int head_dim, int inter, int max_seq) {
  if (head_dim != HD || n_heads < 1 || n_heads > kMaxHeads || max_seq < 1 || max_seq > CKA * kMaxChunks) return 0;
  const size_t qd = static_cast<size_t>(n_heads) * HD;
  const size_t chunks = (static_cast<size_t>(max_seq) + CKA - 1) / CKA;
  // epoch-tagged 64-bit words: q|k|v, attention out, o, GEGLU out, down, chunk partials
  const size_t words = (qd + 2 * HD) + qd + hidden + inter + hidden + chunks * n_heads * (HD + 2);
  return kHeaderBytes + words * sizeof(uint64_t);
}

extern "C" int sb_decode_step_fused(const void* layers_dev, int n_layers, const void* emb, const void* emb_scales,
                                    const float* final_norm, const float* cos_t, const float* sin_t, int hidden,
                                    int n_heads, int head_dim, int inter, int vocab, int max_seq, float eps,
                                    float embed_scale, int32_t* pos, int32_t* cur, int32_t* tokens, int32_t* history,
                                    int hist_len, uint64_t* keys, void* scratch, size_t scratch_bytes, void* stream) {
  SB_CHECK_ARG(head_dim == HD, "sb_decode_step_fused: head_dim must be %d", HD);
  SB_CHECK_ARG(n_heads >= 1 && n_heads <= kMaxHeads, "sb_decode_step_fused: n_heads must be 1..%d", kMaxHeads);
  SB_CHECK_ARG(hidden % 32 == 0 && hidden <= kMaxH && inter % 32 == 0 && inter <= kMaxK && n_heads * HD <= kMaxH,
               "sb_decode_step_fused: hidden and n_heads*head_dim must be multiples of 32 up to %d, inter up to %d",
               kMaxH, kMaxK);
  SB_CHECK_ARG(n_layers >= 1 && vocab >= 1 && max_seq >= 1 && max_seq <= CKA * kMaxChunks,
               "sb_decode_step_fused: bad sizes (max_seq <= %d)", CKA * kMaxChunks);
  SB_CHECK_ARG(layers_dev && emb && emb_scales && final_norm && cos_t && sin_t && pos && cur && tokens && keys &&
                   scratch,
               "sb_decode_step_fused: null pointer");
  SB_CHECK_ARG(sb::aligned(scratch, 16), "sb_decode_step_fused: scratch must be 16-byte aligned");
  const size_t need = sb_decode_step_fused_scratch_size(hidden, n_heads, head_dim, inter, max_seq);
  if (scratch_bytes < need)
    return sb::fail(SB_ERR_WORKSPACE, "sb_decode_step_fused: scratch %zu < %zu bytes", scratch_bytes, need);
  const int smem = static_cast<int>(sizeof(Smem));
  const int grid = grid_size(smem);
  if (grid < 1) return sb::fail(SB_ERR_CUDA, "sb_decode_step_fused: cannot place one CTA per SM");
  // each CTA's gate|up slice must fit the GEGLU staging buffer, and every CTA
  // must own gate|up rows (what makes buffer reuse across layers safe)
  const int per = 2 * ((inter + grid - 1) / grid);
  SB_CHECK_ARG(per <= kSegOut, "sb_decode_step_fused: inter=%d too large for %d SMs", inter, grid);
  SB_CHECK_ARG(inter >= grid, "sb_decode_step_fused: inter=%d must be at least the CTA count %d", inter, grid);
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
  // header: u64 step count at byte 0, u32 abort flag at 8, trace switch at 12
  // (set by the caller), completed launches at 16, u64 running argmax key at 24
  p.ctr = reinterpret_cast<unsigned long long*>(base);
  p.bar = reinterpret_cast<unsigned int*>(base);
  p.kmax = reinterpret_cast<unsigned long long*>(base + 24);
  // the trace region is used only when the u32 at byte 12 is non-zero
  p.trace = reinterpret_cast<unsigned long long*>(base + 64);
  uint64_t* f = reinterpret_cast<uint64_t*>(base + kHeaderBytes);
  const size_t qd = static_cast<size_t>(n_heads) * HD;
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
