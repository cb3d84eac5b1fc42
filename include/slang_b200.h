/*
 * slang_b200 -- C ABI of the B200 (sm_100a) int4 quantized-matmul path.
 *
 * Plain pointers and sizes only.  Every pointer argument named "device" is a
 * CUDA device address owned by the caller; the library never allocates device
 * memory.  Every call is stream-ordered on `stream` (a cudaStream_t; NULL =
 * the legacy default stream) and returns SB_OK or an SB_ERR_* code after
 * validating its arguments on the host; nothing is launched when validation
 * fails.  sb_last_error() gives a human-readable message for the calling
 * thread's last failure.
 *
 * Packing (the reference's on-disk format, gemma4_150/export.py:59-61 and
 * gemma4_150/loader.py:75-86): a weight [n_out, n_in] at `bits` bits is
 * row-major bytes [n_out, n_in*bits/8]; value i of a row sits at bit bits*i of
 * the row's little-endian byte stream (low bits first); code q means the
 * integer q - 2^(bits-1).  Scales are [n_out, n_in/group] in f16 (SB_SCALE_F16,
 * the per-group-32 format) or f32 (SB_SCALE_F32; group == n_in is the
 * reference checkpoint's per-row scale, gemma4/qat_loader.py:95-102).
 * Dequantised weight: w = scale[n, k/group] * (q - 2^(bits-1)).
 */
#ifndef SLANG_B200_H
#define SLANG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SB_OK 0
#define SB_ERR_ARG 1          /* bad shape, null pointer, unsupported combination */
#define SB_ERR_ALIGN 2        /* a pointer or leading dimension violates an alignment rule */
#define SB_ERR_CUDA 3         /* a CUDA runtime call failed (message has the CUDA error) */
#define SB_ERR_TIMEOUT 4      /* a bounded device-side wait expired (see sb_device_status) */
#define SB_ERR_WORKSPACE 5    /* the caller's workspace is too small */

/* element types */
#define SB_F16 1
#define SB_F32 2
#define SB_SCALE_F16 SB_F16
#define SB_SCALE_F32 SB_F32

/* Library version and the calling thread's last error message. */
const char* sb_version(void);
const char* sb_last_error(void);

/*
 * Device-side error word: bounded spin-waits inside kernels set it instead of
 * hanging.  Synchronises `stream`, returns SB_OK if no kernel has reported a
 * timeout since the last call, else SB_ERR_TIMEOUT (and clears the word).
 */
int sb_device_status(void* stream);

/*
 * Dequantise a packed weight to f16: out[n, k] = f16(scale * (q - ZP)),
 * the product formed in f32 and rounded once.
 * Replaces PrefillGPU._dq (gemma4_150/prefill_gpu.py:186-200) and the dq_f16
 * kernel (gemma4_150/kernels_dsl.py:2101-2138).  bits in {2,4,8};
 * n_in % (32/bits) == 0; group % 32 == 0 (or group == n_in); n_in % group == 0.
 *   packed  device [n_out, n_in*bits/8] u8 (4-byte aligned)
 *   scales  device [n_out, n_in/group] f16 or f32
 *   out     device [n_out, n_in] f16 (row stride n_in)
 */
int sb_dequant_f16(const void* packed, int bits, const void* scales, int scale_dtype,
                   int group, void* out, int n_out, int n_in, void* stream);

/*
 * Decode GEMV over an int4 weight: y[m, n] = sum_k w[n, k] * x[m, k].
 * The weight is used exactly (no f16 rounding); x is rounded to 16-bit
 * integers per group of 32 (error <= 2^-16 of the group's max |x|), the
 * int4 x int16 products are summed exactly in 32-bit integers and each
 * group's sum is scaled in f32 (max-rel error vs an fp32 oracle ~1e-5).
 * Replaces matvec_dq4 (gemma4/qat_kernels.py:33-77) and the GEMV cores of the
 * decode kernels qkv_70 / oproj_73 / gateup_74 / down_75
 * (gemma4_150/kernels_dsl.py:1384-1480, 872-996, 1232-1300, 322-429), bound by
 * the runner through Batch.dg (gemma4_150/metal_runner.py:53-67).
 *   w       device [n, k/2] u8, 16-byte aligned rows (k % 32 == 0)
 *   scales  device [n, k/group] f16 or f32 (group % 32 == 0, k % group == 0)
 *   x       device [m, k] f16 or f32 (x_dtype), row stride k
 *   y       device [m, n] f32, row stride ldy (>= n)
 *   m       1..8 decode rows
 */
int sb_gemv_q4(const void* w, const void* scales, int scale_dtype, int group,
               const void* x, int x_dtype, float* y, int ldy, int m, int n, int k,
               void* stream);

/*
 * sb_gemv_q4 over 2-bit codes (the checkpoint's 2-bit MLP weights of layers
 * 15+ and its 2-bit lm_head; gemma4/qat_loader.py:33-38, 52-61): four codes per
 * byte, low bits first, value = code - 2.  Replaces the 2-bit decode GEMVs
 * gateup_95 / down_96 (gemma4_150/kernels_dsl.py:1130-1230, 1303-1381); same
 * exact int x int16 arithmetic, same arguments except
 *   w       device [n, k/4] u8 (k % 64 == 0, so every row is 16-byte aligned)
 * Scales are per group (k/group) or per row (group = k: the checkpoint's
 * [n, 1] f32 weight_scale).
 */
int sb_gemv_q2(const void* w, const void* scales, int scale_dtype, int group,
               const void* x, int x_dtype, float* y, int ldy, int m, int n, int k,
               void* stream);

/*
 * Tied lm_head GEMV fused with greedy argmax (ties -> lowest index).
 * Replaces logits_33 + argmax1_34 + argmax2_35 (gemma4_150/kernels_dsl.py:
 * 1483-1534, 481-570; dispatch gemma4_150/metal_runner.py:392-396) and the
 * oracle's `embed @ x` + softcap + argmax (gemma4/reference.py:178-179; the
 * softcap is monotonic and is not applied).
 * The table may be a vocabulary shard: its row r is global token
 * row_offset + r.  For each decode row the result is a 64-bit key
 *   key = (orderable_u32(max logit) << 32) | (0xFFFFFFFF - global index)
 * so the maximum key over shards (an integer MAX all-reduce) is the global
 * greedy token with the lowest-index tie rule; orderable_u32(f) = ~bits(f)
 * for negative f, bits(f) | 0x80000000 otherwise; NaN counts as -inf.
 *   emb     device [v, k/2] u8;  scales device [v, k/group]
 *   h       device [m, k] f16/f32
 *   keys    device [m] u64 (written; no initialisation needed)
 *   tokens  device [m] i32 or NULL: global token ids decoded from `keys`
 *   logits  device [m, v] f32 or NULL: raw logits of this shard
 */
int sb_lmhead_argmax(const void* emb, const void* scales, int scale_dtype, int group,
                     const void* h, int h_dtype, int m, int v, int k, int64_t row_offset,
                     uint64_t* keys, int32_t* tokens, float* logits, void* stream);

/* sb_lmhead_argmax over a 2-bit table (the checkpoint's lm_head, u8 [v, k/4]
 * row-major as stored; gemma4/qat_loader.py:52-53): codes as in sb_gemv_q2. */
int sb_lmhead_argmax_q2(const void* emb, const void* scales, int scale_dtype, int group,
                        const void* h, int h_dtype, int m, int v, int k, int64_t row_offset,
                        uint64_t* keys, int32_t* tokens, float* logits, void* stream);

/* tokens[i] = global index held in keys[i] (after a cross-shard MAX). */
int sb_keys_to_tokens(const uint64_t* keys, int32_t* tokens, int m, void* stream);

/*
 * Vocabulary-sharded lm_head with the cross-GPU exchange in device memory
 * (replaces the NCCL MAX of keys after sb_lmhead_argmax on each shard).  Each
 * rank creates one mailbox of sb_peer_mailbox_size() bytes with
 * sb_peer_buffer_create (zeroed; ipc_handle receives a 64-byte CUDA IPC
 * handle), shares the handle, and maps the other ranks' mailboxes with
 * sb_peer_buffer_open.  sb_lmhead_argmax_peer then runs this rank's shard
 * GEMV (rows row_offset .. row_offset + v, v >= 1) as one launch: its CTAs fold
 * their argmax keys into this rank's mailbox, and the last CTA to finish writes
 * each row's key, tagged with the step, into this rank's slot of every rank's
 * mailbox (16-byte stores over NVLink), waits (bounded by
 * sb_peer_set_wait_limit_ns; timeout -> SB_ERR_TIMEOUT in sb_device_status and
 * keys of 0) until every rank's slots carry this step's tag, and writes the
 * combined keys / tokens (m <= 64 rows, world <= 32).  A timed-out exchange
 * leaves the mailboxes unusable: create them again.
 * peer_mailboxes: device array of the `world` mailbox addresses as this
 * process maps them, own_mailbox among them (its index is this rank; absent:
 * SB_ERR_TIMEOUT at once).  Every rank must make the same sequence of calls.
 */
size_t sb_peer_mailbox_size(void);
int sb_peer_buffer_create(size_t bytes, void** dev_ptr, void* ipc_handle);
int sb_peer_buffer_open(const void* ipc_handle, void** dev_ptr);
int sb_peer_buffer_close(void* dev_ptr);
int sb_peer_buffer_free(void* dev_ptr);
int sb_lmhead_argmax_peer(const void* emb, const void* scales, int scale_dtype, int group, const void* h, int h_dtype,
                          int m, int v, int k, int64_t row_offset, const uint64_t* peer_mailboxes, int world,
                          void* own_mailbox, uint64_t* keys, int32_t* tokens, void* stream);

/* How long sb_lmhead_argmax_peer's exchange waits for the other ranks' keys
 * before it gives up with SB_ERR_TIMEOUT (in sb_device_status) and returns
 * keys of 0: ns nanoseconds, 0 for the default (and maximum) of 2 s.  A rank
 * that never arrives then costs the others this long instead of a hang.
 * Applies to launches made after the call.  No counterpart in the reference
 * (single-device). */
int sb_peer_set_wait_limit_ns(uint64_t ns);

/*
 * f16 GEMM on the tcgen05 tensor cores, f32 accumulate:
 *   C[M, N] = f16(alpha * A[M, K] @ (B[N, K]^T if tr else B[K, N]))
 * Replaces PrefillGPU._gemm (gemma4_150/prefill_gpu.py:151-184) and the
 * gemm_tiled kernel (gemma4_150/kernels_dsl.py:34-141): same (M, N, K, alpha,
 * tr, lda, ldb, ldc) meaning; the reference's byte offsets aoff/boff/coff are
 * folded into the pointers.  Row strides are in elements; A, B, C 16-byte
 * aligned and lda, ldb multiples of 8.
 */
int sb_gemm_f16(const void* a, const void* b, void* c, int m, int n, int k, float alpha,
                int tr, int lda, int ldb, int ldc, void* stream);

/*
 * Same product with C written as f32 (alpha applied, no f16 rounding); used
 * for the prefill attention scores QK^T so the softmax sees f32 logits.
 * Replaces the score GEMM of PrefillGPU._attn_gemm (gemma4_150/prefill_gpu.py:
 * 304-305).  C 4-byte aligned, row stride ldc in elements.
 */
int sb_gemm_f16_f32out(const void* a, const void* b, float* c, int m, int n, int k, float alpha,
                       int tr, int lda, int ldb, int ldc, void* stream);

/* The same product split into `splits` equal runs of 64-deep K blocks (splits
 * divides ceil(k / 64)); split z writes its partial product to the f32 plane
 * c + z * m * ldc, and the consumer sums the planes (sb_ple_gate_act). */
int sb_gemm_f16_f32out_splitk(const void* a, const void* b, float* c, int m, int n, int k, float alpha,
                              int tr, int lda, int ldb, int ldc, int splits, void* stream);

/*
 * Fused prefill projection: dequantise packed int4 tiles into shared memory
 * and feed them to tcgen05 MMAs, f32 accumulate in tensor memory:
 *   C[M, N] = f16(alpha * A[M, K] @ dq_f16(W)[N, K]^T)
 * where dq_f16 is the bit-exact sb_dequant_f16 rounding.  Replaces the
 * reference's per-layer `_dq` + `_gemm` pair (gemma4_150/prefill_gpu.py:
 * 331-373) in one launch.
 *   a       device [M, K] f16, row stride lda (multiple of 8), 16-byte aligned
 *   w       device [N, K/2] u8 (K % 64 == 0), 16-byte aligned
 *   scales  device [N, K/group] f16 or f32
 *   c       device [M, N] f16, row stride ldc
 *   workspace / workspace_bytes: device f32 scratch for split-K partial sums,
 *           or NULL/0.  sb_gemm_q4_workspace_size() gives the bytes this call
 *           wants; with too little (or none) the call runs without split-K.
 */
int sb_gemm_q4(const void* a, const void* w, const void* scales, int scale_dtype, int group,
               void* c, int m, int n, int k, float alpha, int lda, int ldc,
               void* workspace, size_t workspace_bytes, void* stream);

/*
 * sb_gemm_q4 with the gate|up GEGLU fused into the epilogue: W's rows are
 * interleaved (gate row i at 2i, up row i at 2i + 1; n even) and
 * out[t][i] = f16(gelu_tanh(g) * u) with g, u the f16-rounded GEMM outputs
 * of rows 2i and 2i + 1 -- bit-for-bit sb_gemm_q4 followed by sb_geglu, with
 * out [m][n/2] (row stride ldo) and no [m][n] intermediate.  Replaces the
 * reference's gate/up GEMMs + geglu_b (gemma4_150/prefill_gpu.py:365-372;
 * kernels_dsl.py:259).  Workspace as for sb_gemm_q4.
 */
int sb_gemm_q4_geglu(const void* a, const void* w, const void* scales, int scale_dtype, int group,
                     void* out, int m, int n, int k, float alpha, int lda, int ldo, void* workspace,
                     size_t workspace_bytes, void* stream);
size_t sb_gemm_q4_workspace_size(int m, int n, int k);
/* Kernels one sb_gemm_q4 call launches for this shape (group-32 f16 scales,
 * workspace as sized above): 1, or 2 when a split-K finalize follows. */
int sb_gemm_q4_kernels(int m, int n, int k);

/*
 * sb_gemm_q4 / sb_gemm_q4_geglu over 2-bit codes (the checkpoint's 2-bit MLP
 * weights of layers 15+; gemma4/qat_loader.py:33-38, 52-61): w [N, K/4] u8,
 * four codes per byte, low bits first, value = code - 2; dq_f16 is
 * f16(scale * (code - 2)) as sb_dequant_f16 computes it with bits = 2.  The
 * reference dequantises these with `_dq` (bit width from the buffer size,
 * gemma4_150/prefill_gpu.py:186-200) before its f16 GEMM.  Other arguments
 * and the workspace as for sb_gemm_q4.
 */
int sb_gemm_q2(const void* a, const void* w, const void* scales, int scale_dtype, int group,
               void* c, int m, int n, int k, float alpha, int lda, int ldc,
               void* workspace, size_t workspace_bytes, void* stream);
int sb_gemm_q2_geglu(const void* a, const void* w, const void* scales, int scale_dtype, int group,
                     void* out, int m, int n, int k, float alpha, int lda, int ldo, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * Tied lm_head + greedy argmax for many rows at once on the tcgen05 GEMM:
 * keys[t] = max over rows v of key(alpha * (a[t] . dequant(w[v])), row_offset + v),
 * key = (orderable(value) << 32) | (0xFFFFFFFF - index) as in sb_lmhead_argmax
 * (ties -> lowest index); tokens[t] (optional) = the winning index.  a f16
 * [m, k] (row stride lda), w [n, k/2] packed int4.  keys is cleared first.
 * The argmax of each CTA's [rows x tokens] tile happens in its epilogue, so no
 * logits are written.  Replaces logits_33 + argmax1_34/argmax2_35
 * (gemma4_150/kernels_dsl.py:481-570, 1483-1534) for a batch of sequences
 * (batched decode, where a GEMV per row would read the embedding m times).
 */
int sb_gemm_q4_argmax(const void* a, const void* w, const void* scales, int scale_dtype, int group, int m, int n,
                      int k, float alpha, int lda, int64_t row_offset, uint64_t* keys, int32_t* tokens, void* stream);

/*
 * Profiling hook of the fused int4 / 2-bit GEMM's CTA-pair kernel: while `buf`
 * is set (NULL turns it off), every launch whose grid fits in `bytes` writes
 * 16 u64 per CTA at buf[16 * b] (b = the CTA's linear grid index): [0] its SM,
 * then %globaltimer stamps -- [1] entry, [2] set-up done, [3] activations
 * readable, [4] scales loaded, [5] first packed stage, [6] first MMA, [7] last
 * MMA issued, [8] accumulator final, [9] epilogue issued, [10] split-K
 * reduction done, [11] exit.  For measurement only; buf must stay valid.
 */
int sb_gemm_q4_trace(uint64_t* buf, size_t bytes);

/*
 * Profiling hook of the fused prefill attention kernel (no reference
 * counterpart): while `buf` is set (NULL turns it off), every launch whose grid
 * fits in `bytes` writes 24 u64 per CTA at buf[24 * b] (b = the CTA's linear
 * grid index; CTAs past their tile's last chunk write nothing): [0] its SM,
 * %globaltimer stamps [1] entry, [2] set-up done, [3] Q tile landed, [4] O
 * final, [5] epilogue stores issued, [6] exit, [7] its key-block count, then
 * per key block j < 8: [8 + j] scores readable, [16 + j] P written.  For
 * measurement only; buf must stay valid.
 */
int sb_attn_prefill_trace(uint64_t* buf, size_t bytes);

/*
 * Profiling hook of the streaming GEMV (sb_gemv_q4 / sb_lmhead_argmax /
 * sb_lmhead_argmax_peer and the other entry points on the same kernel but the
 * norm-add form; no reference counterpart): while `buf` is set (NULL turns it
 * off; every call restarts at its beginning), each launch of the kernel --
 * graph captures included -- takes the next 16 x grid u64 of `buf` while they
 * last, CTA b's at [16 * b]: [0] its SM, %globaltimer stamps [1] entry, [2]
 * first bulk copies issued, [3] previous kernel complete
 * (griddepcontrol.wait), [4] x quantised, [5] first stage landed, [6] first
 * stage done, [7] last stage done, [8] keys folded or rows stored, [9] exit,
 * then [10] its stage count, [11] 1 in the CTA that completed the launch's
 * count (peer form), with [12] keys sent to every rank and [13] every rank's
 * keys received.  For measurement only; buf must stay valid.
 */
int sb_gemv_trace(uint64_t* buf, size_t bytes);

/*
 * sb_gemm_q4 without a caller workspace; it allocates nothing.  No counterpart
 * in the reference: it is for callers that cannot allocate device memory --
 * a host reaching the GPU only through this C ABI, with no CUDA allocator of
 * its own, or a process whose device memory is reserved up front by its own
 * pool, where a cudaMalloc on this path fails or stalls.
 * Its split-K scratch is a static 32 MiB device array that every GPU loading
 * this library holds until the process exits.  Shapes whose split-K scratch
 * (for this call's group and scale type; sb_gemm_q4_workspace_size for the
 * group-32 f16 format) exceeds 32 MiB are rejected with SB_ERR_WORKSPACE.
 * The first call on each device looks up the array's device address with
 * that device current; make that first call before any stream capture.  The
 * address is kept per device ordinal for the life of the process: after a
 * cudaDeviceReset() it is stale, so do not call this entry point again in a
 * process that has reset a device it used.  Every call shares the array and it keeps the last call's partial
 * sums (nothing in it needs to start at zero), so calls that overlap on the
 * GPU -- other streams, other host threads -- race: order them on one stream.
 * Arguments mean what they mean for sb_gemm_q4.
 */
int sb_gemm_q4_noalloc(const void* a, const void* w, const void* scales, int scale_dtype, int group,
                       void* c, int m, int n, int k, float alpha, int lda, int ldc, void* stream);

/*
 * Decode GEMV with the residual add + RMSNorm as a last-arriver tail (the
 * reference's oproj_73 / down_75, gemma4_150/kernels_dsl.py:928-996, 398-429):
 *   y = W @ x (as sb_gemv_q4 / sb_gemv_q2 by bits; y [m][n], row stride n),
 *   hidden[r] = hidden[r] + rmsnorm(y[r]) * w_add,
 *   h[r] = rmsnorm(hidden[r]) * w_next  -> h_out (f32) and/or h16_out (f16), when w_next != NULL.
 * The CTA that completes `counter` (a caller-owned u32, zero before the first
 * call) runs the tail over all rows and re-arms it; no CTA waits on another.
 * After a call that reported SB_ERR_TIMEOUT, zero the counter again.
 * n % 4 == 0, n <= 8192; y, hidden, w_add, w_next, h_out 16-byte aligned.
 */
int sb_gemv_norm_add(const void* w, int bits, const void* scales, int scale_dtype, int group, const void* x,
                     int x_dtype, float* y, int m, int n, int k, float* hidden, const float* w_add,
                     const float* w_next, float* h_out, void* h16_out, float eps, unsigned int* counter,
                     void* stream);

/*
 * A quantised linear with static range quantisation (SRQ) of its activations,
 * the reference's production decode arithmetic (ReferenceSRQ._qlin,
 * gemma4_150/reference.py:96-101; kernels qkv_70, oproj_73, gateup_74/95,
 * down_75/96 of gemma4_150/kernels_dsl.py):
 *   y = srq(W @ srq(x, in_scale), out)      srq(v, s) = clip(round(v / s), -128, 127) * s
 * with out = out_scales[row] when out_scales is given (rows of several linears
 * concatenated, e.g. q|k|v, or gate|up interleaved), else out_scale; a scale of
 * 0 skips that side's srq.  The input codes are exact integers, so the dot
 * sum (q - zp) * code -- the reference's zero-point fold of sum(a) -- is
 * computed exactly in 32-bit integers; W as in sb_gemv_q4 (bits 4) /
 * sb_gemv_q2 (bits 2), with its group or per-row scales.
 */
int sb_gemv_srq(const void* w, int bits, const void* scales, int scale_dtype, int group, const void* x, int x_dtype,
                float in_scale, float out_scale, const float* out_scales, float* y, int ldy, int m, int n, int k,
                void* stream);

/* out[i] = srq(x[i], scale) elementwise (f16 or f32 in and out; scale > 0):
 * the activation-side quantisations of the reference's SRQ forward, e.g. the
 * attention output before the o projection (gemma4_150/reference.py:176). */
int sb_srq(const void* x, int x_dtype, size_t n, float scale, void* out, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Decoder glue around the matmuls (the Gemma-4-E2B-shaped model: hidden H,
 * nh query heads and one KV head of head_dim, GEGLU FFN).  Activations of the
 * decode path are f32, those of the prefill GEMMs f16; KV caches are f32
 * [m][max_seq][head_dim] per layer (cache_stride = max_seq * head_dim) with
 * optional f16 copies for the prefill attention GEMMs.  RMSNorm is
 * x / sqrt(mean(x^2) + eps) * w (gemma4/reference.py:19-33).
 * ------------------------------------------------------------------------- */

/* out[r, :] = dequant(emb[tokens[r]]) * mult  (f32 and/or f16).
 * Replaces embed_00 (gemma4_150/kernels_dsl.py:433) / gemma4/reference.py:169. */
int sb_embed_q4(const void* emb, const void* scales, int scale_dtype, int group,
                const int32_t* tokens, int m, int k, float mult, float* out32, void* out16,
                void* stream);

/* As sb_embed_q4 for a table of 2-bit codes (four per byte, low bits first,
 * value = code - 2): the checkpoint's embedding (gemma4/qat_loader.py:53-55,
 * per-block f32 scales :106-113), which export.py stores as embed_q /
 * embed_scale (gemma4_150/export.py:84-85). */
int sb_embed_q2(const void* emb, const void* scales, int scale_dtype, int group,
                const int32_t* tokens, int m, int k, float mult, float* out32, void* out16,
                void* stream);

/* x_out = x + rmsnorm(y) * w_add (y may be NULL: x_out = x); h = rmsnorm(x_out) * w_norm.
 * Replaces rmsadd_b + rmssrqh_b / rmssrq_69 (gemma4_150/kernels_dsl.py:622, 660, 158)
 * and the sandwich norms of gemma4/reference.py:112, 142-152.  n <= 8192. */
int sb_add_rmsnorm(const float* x, const void* y, int y_dtype, const float* w_add,
                   const float* w_norm, float* x_out, float* h_out, void* h16_out, int m, int n,
                   float eps, void* stream);

/* Per token (prefill, positions start_pos + s) or per sequence (decode,
 * positions pos_dev[s]): q heads -> rmsnorm * q_norm -> RoPE -> q16/q32
 * [s][nh][hd]; k -> rmsnorm * k_norm -> RoPE -> k_cache (+ k16); v ->
 * parameter-free rmsnorm -> v_cache (+ v16).  cos/sin: [max_seq][hd/2].
 * head_dim in {64, 128, 256, 512} (512: the checkpoint's full-attention
 * layers).  k_cache and v_cache both NULL: a layer that reads another layer's
 * K/V (KV sharing, gemma4/reference.py:117-131) -- only the q heads are
 * prepared and qkv rows hold n_heads * head_dim values.
 * Replaces kvnorm_b + qprep_b (gemma4_150/kernels_dsl.py:1790, 1838) /
 * gemma4/reference.py:114-125. */
int sb_qkv_prep(const void* qkv, int qkv_dtype, int ld, const float* q_norm, const float* k_norm,
                const float* cos_t, const float* sin_t, const int32_t* pos_dev, int start_pos, int s,
                int n_heads, int head_dim, float eps, void* q16, float* q32, float* k_cache,
                float* v_cache, void* k16, void* v16, int64_t cache_stride, void* stream);

/* Causal softmax over f32 score rows (row r = token r / n_heads): p16 =
 * f16(exp(s - max) / sum) for keys <= start_pos + r / n_heads, 0 after; with
 * window > 0 also 0 for keys more than window - 1 before the query (a
 * sliding-window layer, gemma4/reference.py:126-129; 0 = no window).
 * Replaces smax_b + attnout_b (gemma4_150/kernels_dsl.py:1877, 1753) and the
 * banded sliding mask of gemma4_150/prefill_gpu.py:290-310. */
int sb_softmax_causal(const float* scores, int ld_s, int rows, int n_heads, int start_pos,
                      int n_keys, int window, void* p16, int ld_p, void* stream);

/*
 * Fused causal prefill attention on tcgen05: out = softmax(q k^T) v for one
 * prompt at positions 0..s_len-1, unscaled scores (q, k are RMS-normalised),
 * row r = token r / n_heads sees keys 0..token.  q16 [s_len * n_heads][hd],
 * k16, v16 [s_len][hd], out16 [s_len * n_heads][hd], all f16, 16-byte
 * aligned, hd = head_dim in {64, 128, 256}.  Online softmax with f32 scores and accumulators, probabilities
 * rounded to f16 for the P.V MMA.  Replaces the reference's attn_prefill
 * kernel and its _attn_gemm QK^T -> softmax -> PV chain
 * (gemma4_150/prefill_gpu.py:259-314, 348-352).
 */
int sb_attn_prefill(const void* q16, const void* k16, const void* v16, void* out16, int s_len,
                    int n_heads, int head_dim, void* stream);

/* sb_attn_prefill with each query tile's key range split across CTAs (as many
 * as one wave of SMs holds) and the shares merged by a second kernel; needs
 * workspace >= sb_attn_prefill_workspace_size(s_len, n_heads, head_dim) bytes
 * (16-byte aligned; 0 bytes means no split is worth it and none is used). */
int sb_attn_prefill_ws(const void* q16, const void* k16, const void* v16, void* out16, int s_len,
                       int n_heads, int head_dim, void* workspace, size_t workspace_bytes, void* stream);
size_t sb_attn_prefill_workspace_size(int s_len, int n_heads, int head_dim);

/* out[r, i] = gelu_tanh(gu[r, 2i]) * gu[r, 2i + 1]: the fused gate|up weight keeps
 * gate row i and up row i adjacent, so its output interleaves them.
 * Replaces geglu_b (gemma4_150/kernels_dsl.py:259) / gemma4/reference.py:148-150. */
int sb_geglu(const void* gu, int dtype, int m, int f, float* out32, void* out16, void* stream);

/* Split-KV decode attention, one KV head shared by n_heads query heads:
 * out[b, h*hd:(h+1)*hd] = softmax(q[b,h] . K[b, lo..pos]) V[b, lo..pos] with
 * lo = 0, or lo = max(0, pos + 1 - window) for a sliding-window layer
 * (window > 0).  head_dim in {64, 128, 256, 512}; n_heads in {1, 2, 4, 8}, or
 * 16 for head_dim <= 256.
 * Replaces attn_101 (gemma4_150/kernels_dsl.py:1540) / gemma4/reference.py:127-139.
 * workspace >= sb_attn_decode_workspace_size(m, n_heads, head_dim, max_seq) bytes. */
int sb_attn_decode(const float* q32, const float* k_cache, const float* v_cache,
                   int64_t cache_stride, const int32_t* pos_dev, int m, int n_heads, int head_dim,
                   int max_seq, int window, float* out, float* workspace, size_t workspace_bytes,
                   void* stream);
size_t sb_attn_decode_workspace_size(int m, int n_heads, int head_dim, int max_seq);
/* sb_attn_decode writing out16 [m][n_heads * head_dim] as f16 (the A operand of
 * the tcgen05 o-projection in batched decode). */
int sb_attn_decode_f16(const float* q32, const float* k_cache, const float* v_cache, int64_t cache_stride,
                       const int32_t* pos_dev, int m, int n_heads, int head_dim, int max_seq, int window,
                       void* out16, float* workspace, size_t workspace_bytes, void* stream);

/* Device-side step bookkeeping so a decode step replays as one graph:
 * pos[b] += 1; cur[b] = tokens[b]; history[b * hist_len + pos[b]] = tokens[b].
 * Replaces the blit of the argmax token into gen[step] (gemma4_150/metal_runner.py:394-398). */
int sb_step_advance(int32_t* pos, const int32_t* tokens, int32_t* cur, int32_t* history,
                    int hist_len, int m, void* stream);

/* One layer of the model for sb_decode_step_fused (device pointers). */
typedef struct sb_decode_layer {
  const void* w[4];        /* packed int4: q|k|v [nqkv, H/2], o [H, qd/2],
                              gate|up with rows interleaved [2F, H/2], down [H, F/2] */
  const void* s[4];        /* their f16 group-32 scales [rows, K/32] */
  const float* in_norm;
  const float* q_norm;
  const float* k_norm;
  const float* post_attn_norm;
  const float* pre_ffn_norm;
  const float* post_ffn_norm;
  float* k_cache;          /* [max_seq][head_dim] f32 */
  float* v_cache;
} sb_decode_layer;

/*
 * One greedy decode step for a single sequence as one persistent cooperative
 * kernel (one CTA per SM): embed cur[0] at position pos[0], all layers, final
 * norm, tied lm_head argmax; then tokens[0] = next token, cur[0] = it,
 * pos[0] += 1 and history[pos[0]] = it.  Same arithmetic as the per-op path
 * (sb_embed_q4 ... sb_lmhead_argmax).  Replaces the whole per-token dispatch
 * chain of G4._forward (gemma4_150/metal_runner.py:372-402).
 * Requirements: head_dim 256, n_heads <= 8, hidden, inter, n_heads*256 <= 6144
 * and multiples of 32, f16 group-32 scales.  layers_dev: device array of
 * n_layers sb_decode_layer.  scratch: >= sb_decode_step_fused_scratch_size()
 * bytes, zero-filled before the first call (later calls leave it reusable; it
 * holds the step count that tags the phase outputs, so steps sharing one
 * scratch must not overlap on the GPU, and after SB_ERR_TIMEOUT it is zeroed
 * again); inter >= the SM count; keys receives the lm_head key as in
 * sb_lmhead_argmax.
 */
int sb_decode_step_fused(const void* layers_dev, int n_layers, const void* emb, const void* emb_scales,
                         const float* final_norm, const float* cos_t, const float* sin_t, int hidden,
                         int n_heads, int head_dim, int inter, int vocab, int max_seq, float eps,
                         float embed_scale, int32_t* pos, int32_t* cur, int32_t* tokens,
                         int32_t* history, int hist_len, uint64_t* keys, void* scratch,
                         size_t scratch_bytes, void* stream);
size_t sb_decode_step_fused_scratch_size(int hidden, int n_heads, int head_dim, int inter, int max_seq);

/* ---------------------------------------------------------------------------
 * Per-layer embeddings (PLE) of Gemma-4-E2B, weight-only f32 arithmetic as
 * gemma4/reference.py:92-101 (per-layer input) and :154-163 (per-layer block)
 * with the QAT dequant of gemma4/qat_reference.py:39-45.  8-bit linears are
 * the checkpoint's signed int8 codes stored +128-biased (the byte layout of
 * gemma4_150/export.py:150-157) with one f32 scale per output row
 * (gemma4/qat_loader.py:41-48, 98-102).  Activation rows are f32; m is any
 * count (launched in blocks of 8 rows).
 * ------------------------------------------------------------------------- */

/* y[r][o] = row_scale[o] * sum_k (codes[o][k] - 128) * x[r][k], r < m, o < n;
 * with ple != null instead y = gelu_tanh(that) * ple[r * ld_ple + o].
 * k % 16 == 0, k >= 64; codes and x 16-byte aligned, ldx % 4 == 0.
 * Replaces plegate_76 (gemma4_150/kernels_dsl.py:829-870; ple != null) and the
 * matmul of pleproj_77 (:1000-1060; ple == null), without the SRQ steps. */
int sb_gemv_q8(const void* codes, const float* row_scale, const float* x, int ldx, float* y, int ldy,
               int m, int n, int k, const float* ple, int ld_ple, void* stream);

/* The PLE projection GEMV fused with its norm-add tail: proj = sb_gemv_q8(codes,
 * row_scale, g) (m <= 8 rows, written to proj [m][n]), then the CTA that
 * finishes last (an atomic count on *counter, no waiting) runs
 * sb_ple_norm_add(proj, hidden, w_post, layer_scalar, w_next, h_out, h16_out)
 * over all rows and re-arms *counter to 0.  counter: a zero-initialised device
 * u32 that no concurrently running launch shares.  Replaces pleproj_77's
 * last-arriver matmul + norm tail (gemma4_150/kernels_dsl.py:1000-1125). */
int sb_ple_proj_norm_add(const void* codes, const float* row_scale, const float* g, int ldg, float* proj,
                         int m, int n, int k, float* hidden, const float* w_post, float layer_scalar,
                         const float* w_next, float* h_out, void* h16_out, float eps, unsigned int* counter,
                         void* stream);

/* y[r][o] = alpha * sum_k bf16(w[o][k]) * x[r][k]  (w: bf16 bit patterns [n][k]).
 * k % 8 == 0, k >= 32; w and x 16-byte aligned.  Replaces the
 * per_layer_model_projection matmul and its hidden**-0.5 factor
 * (gemma4/reference.py:97-98). */
int sb_gemv_bf16(const void* w, float alpha, const float* x, int ldx, float* y, int ldy,
                 int m, int n, int k, void* stream);

/* As sb_gemv_bf16 with f16 weights: the per_layer_model_projection as
 * export.py stores it (pl_model_proj, cast to f16, gemma4_150/export.py:95). */
int sb_gemv_f16(const void* w, float alpha, const float* x, int ldx, float* y, int ldy,
                int m, int n, int k, void* stream);

/* hidden[r] = (hidden[r] + rmsnorm(proj[r]) * w_post) * layer_scalar, in place;
 * when w_next != null also h = rmsnorm(hidden[r]) * w_next -> h_out (f32)
 * and/or h16_out (f16).  n % 4 == 0, n <= 8192, 16-byte aligned rows.
 * Replaces the norm-add tail of pleproj_77 (gemma4_150/kernels_dsl.py:1062-1125;
 * gemma4/reference.py:160-163). */
int sb_ple_norm_add(const float* proj, float* hidden, const float* w_post, float layer_scalar,
                    const float* w_next, float* h_out, void* h16_out, int m, int n, float eps,
                    void* stream);

/* y[r][c] = (q - 8) * scales[id][c / group] * ple_scale for the 4-bit table row
 * id = ids[r] (cols values, two per byte, low nibble first; ids outside
 * [0, vocab) give a zero row).  cols % 8 == 0, group % 8 == 0.
 * Replaces plegather_01 (gemma4_150/kernels_dsl.py:457-478) and
 * QATReference._ple_table_row * ple_scale (gemma4/qat_reference.py:39-45,
 * gemma4/reference.py:96). */
int sb_ple_gather(const int32_t* ids, const void* table, const float* scales, int vocab, int cols,
                  int group, float ple_scale, float* y, int m, void* stream);

/* out[r][l][:] = (rmsnorm(ctx[r][l][:]) * w_norm + gather(ids[r])[l*d:(l+1)*d]) * 2^-0.5
 * over n_layers slices of d values (ctx from sb_gemv_bf16 with alpha =
 * hidden**-0.5; the gather as sb_ple_gather).  d % 256 == 0.
 * Replaces the rest of ReferenceGemma4._ple_input (gemma4/reference.py:99-101). */
int sb_ple_combine(const float* ctx, const int32_t* ids, const void* table, const float* scales,
                   int vocab, const float* w_norm, int n_layers, int d, int group, float ple_scale,
                   float eps, float* out, int m, void* stream);

/* out16[r][o] = f16(gelu_tanh(sum_z pre[z*plane + r*ld_pre + o]) * ple[r][o]),
 * z < nsplit (the K-split planes of sb_gemm_f16_f32out_splitk), r < m, o < n:
 * the gate tail once the gate is a GEMM at prefill, feeding the projection
 * GEMM.  Replaces plegate's GEMM tail (gemma4_150/kernels_dsl.py:1775) without
 * its SRQ step. */
int sb_ple_gate_act(const float* pre, int ld_pre, int64_t plane, int nsplit, const float* ple, int ld_ple,
                    void* out16, int ld_out, int m, int n, void* stream);

/* out16[i] = f16(x[i]) (round to nearest even), i < n: the f16 A operand of a
 * prefill GEMM taken from an f32 residual stream. */
int sb_cast_f16(const float* x, void* out16, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SLANG_B200_H */
