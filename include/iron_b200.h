/*
 * iron_b200 C ABI -- B200 (sm_100a) kernels for the Qwen3 decode hot path of IRON.
 *
 * Conventions (every entry point):
 *   - Pointers are DEVICE pointers owned by the caller (e.g. torch tensors'
 *     data_ptr()).  bf16 data is passed as uint16_t bit patterns.
 *   - `stream` is a cudaStream_t (or NULL for the legacy default stream) passed
 *     as void*.  Every launch is asynchronous on that stream.
 *   - Return 0 on success, a negative IRON_ERR_* code on failure; the message is
 *     available from iron_last_error() (thread-local).  No entry point
 *     allocates device memory; scratch space ("workspace") is caller-provided,
 *     sized by the matching *_workspace_bytes() query, and zero-filled once before
 *     its first use.  Calls with different workspaces may run on different streams
 *     at the same time; calls sharing a workspace must not overlap.
 *   - Runtime parameters that change between CUDA-graph replays (positions,
 *     KV lengths) are read from device memory when the *_dev pointer is non-NULL.
 *
 * int8 weight wire (IRON's int8 tile wire, gemv_int8/reference.py:59-80 and
 * qwen3_npu_int8.py:381-436): rows are grouped in tiles of `tile_m` rows, each
 * tile stored as [tile_m*K int8 payload | tile_m*(K/group) bf16 scales].  Tiles
 * are grouped into per-core windows of `rows_per_core` rows stored as
 * `tiles_per_core` tiles (a window may carry trailing pad tiles, the fuse_o Wo
 * wire of swiglu_mlp_dp/op_ours.py:357-421).  The plain wire has
 * rows_per_core = M and tiles_per_core = M / tile_m.  The native layout of this
 * library is tile_m = 1 (row-interleaved [K int8 | K/group bf16]).
 * domain: 0 = signed two's complement q, 1 = biased q + 128 (mv_int8.cc).
 * Every row start must be 16-byte aligned.
 */
#ifndef IRON_B200_H
#define IRON_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IRON_OK 0
#define IRON_ERR_ARG (-1)      /* invalid argument / shape */
#define IRON_ERR_ALIGN (-2)    /* pointer or stride misaligned */
#define IRON_ERR_CUDA (-3)     /* CUDA launch / runtime error */
#define IRON_ERR_UNSUPPORTED (-4)
#define IRON_ERR_TIMEOUT (-5)  /* a bounded device-side wait gave up */

/* ---- library ---------------------------------------------------------- */
/* Version string of the library. */
const char* iron_version(void);
/* Copy the calling thread's last error message into buf (NUL-terminated); returns its length. */
int iron_last_error(char* buf, int buflen);
/* Kernels this library has launched in this process (every successful launch, from any
 * thread; replays of a captured CUDA graph are not launches of the library).  A
 * diagnostic with no counterpart in the reference: the difference across one eager or
 * captured decode step is the number of kernels that step runs. */
int64_t iron_launch_count(void);

/* ---- int8 group-dequant GEMV (W8A16) -------------------------------------
 * y[b, m] = bf16( sum_k q[m,k] * s[m, k/group] * x[b, k] )           (epilogue 0)
 * y[b, m] = bf16( r[b, m] + bf16(sum ...) )                          (epilogue 1, residual)
 * Replaces GEMVInt8 (iron/operators/gemv_int8/op.py:20-178), kernel
 * matvec_vectorized_int8_bf16 (aie_kernels/aie2p/mv_int8_signed.cc:103-115,
 * biased: mv_int8.cc:60-114).  batch: activation rows sharing the weight.  Batch 1..8
 * (and 9..15) computes the exact dequantised sum (one bf16 rounding; launches of 8
 * rows); batch 16..4096 on plain wires runs one tcgen05 tensor-core contraction (in row
 * blocks of up to 128 activation rows, a second grid dimension) with
 * each weight q*s written as two bf16 planes (hi + lo, exact products) and float32
 * accumulation: the exact sum up to float32 summation order.  That contraction keeps
 * its scratch (status word, split-K arrival counters and partial tiles, RMS-normalised
 * inputs) in `workspace` (iron_tc_workspace_bytes(M, K, batch) bytes, 256-byte
 * aligned, zero-filled before first use); with no workspace, or a smaller one, batch
 * 16+ runs the exact kernel in launches of 8 rows instead.
 * group in {32, 64, 128}; K a multiple of 16*... see iron_gemv_w8a16 checks.
 */
int iron_gemv_w8a16(const void* wire, int M, int K, int group, int tile_m,
                    int rows_per_core, int tiles_per_core, int domain,
                    const uint16_t* x, int batch, const uint16_t* residual,
                    uint16_t* y, void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace bytes of a batch 16..4096 tensor-core projection of M rows x K columns
 * (any epilogue, a gate/up pair and an RMSNorm prologue included); 256 outside that range.
 * No reference counterpart. */
int64_t iron_tc_workspace_bytes(int M, int K, int batch);
/* Error word of the tensor-core projections that used `workspace` (its first int32):
 * 0, or the code of the first bounded device wait that timed out.  clear != 0 also
 * resets it.  Synchronous.  No reference counterpart. */
int iron_tc_status(void* workspace, int clear);

/* Dequantise a wire to float32 q*s (exact), row-major (M, K).  Test/inspection
 * entry point for the bit-exact dequant check (GEMVInt8.reference, op.py:173-178). */
int iron_dequant_w8(const void* wire, int M, int K, int group, int tile_m,
                    int rows_per_core, int tiles_per_core, int domain,
                    float* out, void* stream);

/* Symmetric per-(row, group) RTN int8 quantiser + packer into the plain wire.
 * w: bf16 (M, K) row-major.  Bit-exact with Qwen3NPU._set_int8_rtn
 * (qwen3_npu_int8.py:457-491): s = bf16(absmax/127) (s = 1 for an all-zero
 * group), q = clamp(rint(w / s), -127, 127). */
int iron_quantize_rtn(const uint16_t* w, int M, int K, int group, int tile_m, int domain,
                      void* wire_out, void* stream);

/* ---- bf16 GEMV ------------------------------------------------------------
 * y[b, m] = bf16( sum_k A[m, k] * x[b, k] )  (f32 accumulation).
 * independent != 0: `batch` independent GEMVs, A[b] (M, K) each (the num_batches
 * mode of iron/operators/gemv/op.py:151-157).  Replaces GEMV (gemv/op.py:20-163,
 * kernel aie_kernels/generic/mv.cc:47-90).  A shared weight with 16..4096 rows runs
 * the tcgen05 contraction of iron_gemv_w8a16 with its scratch in `workspace`
 * (iron_tc_workspace_bytes(M, K, batch); NULL: launches of 8 rows instead). */
int iron_gemv_bf16(const uint16_t* A, int M, int K, const uint16_t* x, int batch,
                   int independent, uint16_t* y, void* workspace, int64_t workspace_bytes,
                   void* stream);

/* lm_head GEMV fused with a greedy argmax over the bf16-rounded logits (ties ->
 * lowest index, as numpy.argmax in qwen3_npu_int8.py:619-620).  logits may be
 * NULL (not stored; the int8 form needs it).  token_out: int32[batch].  workspace:
 * iron_lm_head_workspace_bytes(M, K, batch) bytes, 256-byte aligned, zero-filled
 * before first use.  From batch 16 on it holds the tcgen05 contraction's scratch
 * first (so iron_tc_status reads its status word), then the argmax candidates, then
 * the logits when logits is NULL; iron_argmax_workspace_bytes(batch) bytes (the
 * candidates only) run the launches of 8 rows instead. */
int iron_lm_head_bf16_argmax(const uint16_t* A, int M, int K, const uint16_t* x, int batch,
                             uint16_t* logits, int32_t* token_out, void* workspace,
                             int64_t workspace_bytes, void* stream);
int iron_lm_head_w8_argmax(const void* wire, int M, int K, int group, const uint16_t* x,
                           int batch, uint16_t* logits, int32_t* token_out, void* workspace,
                           int64_t workspace_bytes, void* stream);
int64_t iron_lm_head_workspace_bytes(int M, int K, int batch);
int64_t iron_argmax_workspace_bytes(int batch);
/* Greedy argmax over bf16 rows: token_out[b] = argmax_m logits[b, m]. */
int iron_argmax_bf16(const uint16_t* logits, int M, int batch, int32_t* token_out,
                     void* workspace, void* stream);

/* ---- RMSNorm / elementwise ---------------------------------------------------
 * Weighted RMSNorm per row of `cols` (op iron/operators/rms_norm/op.py:20-130).
 * mode 0: y = bf16(x * rsqrt(mean(x^2) + eps) * w) in f32, the device kernel's
 * arithmetic (aie_kernels/aie2p/rms_norm.cc:9-53).  mode 1: the golden's
 * arithmetic on bf16 tensors (rms_norm/reference.py:8-17), each of x^2, mean,
 * +eps, sqrt, x/rms, *w rounded to bf16.  mode 2: the Llama form (llama_cpu.py:41-46)
 * on bf16 tensors, x^2, mean, +eps, rsqrt, x*r, w* rounded to bf16.  w may be NULL
 * (unweighted). */
int iron_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int cols,
                 float eps, int mode, void* stream);
/* c = bf16(a + b)   (iron/operators/elementwise_add/op.py, aie_kernels/generic/add.cc) */
int iron_add(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n, void* stream);
/* c = bf16(a * b)   (iron/operators/elementwise_mul/op.py, aie_kernels/generic/mul.cc) */
int iron_mul(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n, void* stream);
/* RoPE (two halves, interleaved [cos, sin] rows of ang_table, row = position) of the
 * q and k heads of raw (batch, (Hq + 2 Hkv) HD) and the K/V cache write at each
 * stream's element offset kv_off_dev[b] (per-token [K_t | V_t] layout), without the
 * per-head norms of iron_qkv_head: the Llama path (llama_cpu.py:14-38, 94-115). */
int iron_rope_kv(const uint16_t* raw, const uint16_t* ang_table, uint16_t* q_out, uint16_t* kv_cache, int HD,
                 int Hq, int Hkv, int max_seq, int batch, const int32_t* kv_off_dev, void* stream);
/* The per-head epilogue of iron_qkv_head (q/k RMSNorm with n_qn / n_kn in norm_mode,
 * RoPE from the (max_seq, HD) angle table, q to q_out (rows, Hq*HD), K_t / V_t into the
 * cache) over the consecutive tokens of ONE prompt: raw row r is the token at position
 * pos0 + r, written to that position of the single stream cache kv_cache (Hkv,
 * 2*max_seq*HD).  The prompt-rows form of the decode head (qkv_head_dp/reference.py
 * :29-33), for a prefill that does at once what the reference's token-by-token prompt
 * loop does (check_cosine_int8.py:49-54, one Qwen3NPU.__call__ per token). */
int iron_qkv_rows(const uint16_t* raw, int rows, const uint16_t* n_qn, const uint16_t* n_kn,
                  const uint16_t* ang_table, uint16_t* q_out, uint16_t* kv_cache, int HD, int Hq, int Hkv,
                  int max_seq, int pos0, float eps, int norm_mode, void* stream);
/* y = bf16(silu(x)); mode 0: x*sigmoid(x) in f32 (silu/reference.py:8-10),
 * mode 1: the tanh form with bf16 roundings (aie_kernels/aie2p/silu.cc). */
int iron_silu(const uint16_t* x, uint16_t* y, int64_t n, int mode, void* stream);
/* out[i, :] = table[ids[i], :]  (token embedding gather, bf16 rows of D; an id
 * outside [0, vocab) yields a zero row). */
int iron_embedding(const uint16_t* table, int vocab, const int32_t* ids, int n, int D,
                   uint16_t* out, void* stream);

/* Advance the device-resident decode positions by one token for `batch` streams:
 * pos += 1; seq_len = pos + 1; kv_off = pos * 2 * HD (the host-side per-token
 * parameter writes of qwen3_npu_int8.py:600-610, done on the device so a
 * captured decode step can be replayed back to back). */
int iron_decode_advance(int32_t* pos, int32_t* seq_len, int32_t* kv_off, int batch, int HD,
                        void* stream);

/* ---- data-movement operators of the Llama decode runlist (llama_npu.py:279-557) ---- */
/* RoPE over (rows, cols) bf16 (RoPE, iron/operators/rope/op.py; golden
 * rope/reference.py:88-154): y1 = x1*c - x2*s, y2 = x2*c + x1*s in float32, one bf16
 * rounding, with (x1, x2) columns (j, j + cols/2) for method 0 (two halves) or
 * (2j, 2j + 1) for method 1 (interleaved); angles (angle_rows, cols) interleaved
 * [cos, sin] pairs, angle row r / (rows / angle_rows) for row r.  y may alias x. */
int iron_rope_rows(const uint16_t* x, const uint16_t* angles, uint16_t* y, int rows, int cols,
                   int angle_rows, int method, void* stream);
/* StridedCopy (iron/operators/strided_copy/op.py; golden strided_copy/reference.py):
 * gather by the input access pattern, scatter by the output one.  A pattern is up to 4
 * (size, stride) pairs (host arrays, outermost first, read at call time) and an element
 * offset; the innermost non-empty dimension is cut into `channels` parts paired one to
 * one.  *in_addend_dev / *out_addend_dev (nullable device int32, elements) are the
 * runtime offset parameters.  Out-of-range elements are skipped and set *err_dev = 1
 * (nullable).  Elements of the output the pattern does not visit keep their values. */
int iron_strided_copy(const void* in, int64_t in_elems, void* out, int64_t out_elems, int elem_bytes,
                      int in_ndim, const int64_t* in_sizes, const int64_t* in_strides, int64_t in_offset,
                      int out_ndim, const int64_t* out_sizes, const int64_t* out_strides,
                      int64_t out_offset, int channels, const int32_t* in_addend_dev,
                      const int32_t* out_addend_dev, int32_t* err_dev, void* stream);
/* Repeat (iron/operators/repeat/op.py; golden repeat/reference.py): row r of `in`
 * (row_bytes bytes) becomes rows r*repeat .. r*repeat + repeat - 1 of `out`. */
int iron_repeat_rows(const void* in, void* out, int64_t rows, int64_t row_bytes, int repeat, void* stream);
/* Softmax (iron/operators/softmax/op.py; golden softmax/reference.py) over each of
 * `rows` bf16 rows of `cols`: the first n = clamp(vector_size, 0, cols) entries get
 * float32 exp(x - max) * (1 / sum), the rest are masked to zero; vector_size is read
 * from *vector_size_dev when it is not NULL (the runtime vector-size parameter). */
int iron_softmax_rows(const uint16_t* x, uint16_t* y, int rows, int cols, int vector_size,
                      const int32_t* vector_size_dev, void* stream);
/* Transpose (iron/operators/transpose/op.py; golden transpose/reference.py): `batches`
 * bf16 (M, N) matrices laid back to back -> (N, M) each; not in place. */
int iron_transpose(const uint16_t* in, uint16_t* out, int M, int N, int batches, void* stream);

/* ---- fused QKV head ------------------------------------------------------------
 * QKVHeadDataParallelOurs (iron/operators/qkv_head_dp/op_ours.py:31-262; golden
 * qkv_head_dp/reference.py:13-33): hn = RMSNorm_w(cur, n_in); raw = bf16(Wqkv@hn);
 * q,k = RoPE(RMSNorm_w(head, n_qn|n_kn), ang); v = raw.  q -> q_out (Hq*HD);
 * K_t,V_t -> kv_cache.  `batch` independent streams: cur (batch, D), q_out
 * (batch, Hq*HD), kv_cache (batch, Hkv, 2*max_seq*HD).
 * kv layout: per KV head a region of 2*max_seq*HD bf16 holding per-token
 * [K_t | V_t] (the KV_TOKEN_INTERLEAVED layout, decode_attn.cc:92-99).  K_t is
 * written at element offset kv_off of every head region and V_t at kv_off + HD
 * (kv_off = seq_pos*2*HD, the k_cache_offset parameter of qwen3_npu_int8.py:600,
 * 608); kv_off_dev (int32[batch]) overrides kv_off when non-NULL.
 * An offset that is not a token slot of the cache writes nothing.
 * ang_is_table = 0: ang holds one interleaved [cos, sin, ...] row of HD per stream;
 * 1: ang is a (max_seq, HD) table and the row kv_off/(2*HD) is used.
 * norm_mode selects the RMSNorm arithmetic of the input and q/k norms (see
 * iron_rmsnorm; the QKV golden uses mode 1).
 * raw_ws: bf16 workspace of batch*(Hq+2*Hkv)*HD elements.  workspace: the projection's
 * tensor-core scratch from batch 16 on (iron_tc_workspace_bytes; may be NULL). */
int iron_qkv_head(const uint16_t* cur, const uint16_t* n_in, const void* wqkv_wire, int group,
                  int tile_m, int domain, const uint16_t* n_qn, const uint16_t* n_kn,
                  const uint16_t* ang, int ang_is_table, uint16_t* q_out, uint16_t* kv_cache,
                  int D, int HD, int Hq, int Hkv, int max_seq, int batch, int kv_off,
                  const int32_t* kv_off_dev, float eps, int norm_mode, uint16_t* raw_ws,
                  void* workspace, int64_t workspace_bytes, void* stream);

/* ---- decode attention ---------------------------------------------------------
 * GQA single-query attention per stream over positions [0, seq_len), base-2
 * softmax with scale log2(e)/sqrt(HD) (decode_attn/reference.py:26-38; kernels
 * aie_kernels/aie2p/decode_attn.cc:117-311; op decode_attn/op.py:20-181).
 * q (batch, H, HD); kv per stream per KV head (2*max_seq*HD): kv_layout
 * 0 = per-token [K_t | V_t] (kv_token_interleaved, decode_attn/op.py:49-52),
 * 1 = [K half | V half] (the combined arg of decode_attn/reference.py:74-93),
 * 2 = [K_block | V_block] per block_kv tokens (decode_attn.cc:95-97).  seq_lens_dev (int32[batch]) overrides
 * seq_len when non-NULL (ragged streams).  kv must be 16-byte aligned (rows are
 * read as 16-byte vectors).  Split-KV flash decoding: partial (m, l, o) per split
 * in `workspace`, merged by a second pass.  With q 16-byte aligned and HD 64 or 128,
 * the first pass runs on the tensor pipe (bf16 mma.sync, float32 accumulation);
 * otherwise on 16-byte lane loads.  Both compute in float32 and differ only in
 * summation order. */
int64_t iron_decode_attn_workspace_bytes(int batch, int H, int HD, int max_seq);
int iron_decode_attn(const uint16_t* q, const uint16_t* kv, uint16_t* out, int batch, int H,
                     int KV, int HD, int max_seq, int kv_layout, int block_kv, int seq_len,
                     const int32_t* seq_lens_dev, void* workspace, int64_t workspace_bytes,
                     void* stream);

/* Decode attention that allocates nothing and takes no workspace: for callers
 * that cannot allocate device memory themselves (a host plugin without an
 * allocator, a runtime that forbids allocation while decoding).  No counterpart
 * in the reference.  The split-KV partials live in a fixed 8 MiB array that every
 * GPU loading the library holds until exit; iron_decode_attn_static_capacity_bytes()
 * returns that size, and a shape needing more (iron_decode_attn_workspace_bytes)
 * is rejected with IRON_ERR_UNSUPPORTED.  The first call on a device looks the
 * array's device address up (cudaGetSymbolAddress) and caches it; make that first
 * call before any stream capture on that device.  All calls on a device share the
 * array and keep the last call's contents (each call rewrites all it reads), so
 * calls that overlap on the GPU race.  Arguments as iron_decode_attn. */
int64_t iron_decode_attn_static_capacity_bytes(void);
int iron_decode_attn_static(const uint16_t* q, const uint16_t* kv, uint16_t* out, int batch, int H,
                            int KV, int HD, int max_seq, int kv_layout, int block_kv, int seq_len,
                            const int32_t* seq_lens_dev, void* stream);

/* ---- multi-query attention over one KV stream ------------------------------------
 * The verify mode of DecodeAttention (batch_queries / num_new_tokens / causal,
 * decode_attn/op.py:40-56; golden cpu_reference_batch, decode_attn/test_batch.py:31-46)
 * and the causal attention of a prompt (MHA, mha/op.py:21-153; golden
 * mha/reference.py:26-93).  q, out: (T, H, HD) token-major.  Token t sits at position
 * base + t and attends the positions j < kv_len, and with causal != 0 only j <= base + t.
 * base_dev (int32, may be NULL) overrides base: the S_kv_base runtime parameter.
 * kv: ONE stream's cache (KV, 2*max_seq*HD) in kv_layout 0/1/2 as iron_decode_attn.
 * HD 64 or 128; q and kv 16-byte aligned.  Split-KV partials in `workspace`
 * (iron_attn_mq_workspace_bytes), merged by a second pass. */
int64_t iron_attn_mq_workspace_bytes(int T, int H, int KV, int HD, int max_seq);
int iron_attn_mq(const uint16_t* q, const uint16_t* kv, uint16_t* out, int T, int H, int KV, int HD,
                 int max_seq, int kv_layout, int block_kv, int base, const int32_t* base_dev, int kv_len,
                 int causal, void* workspace, int64_t workspace_bytes, void* stream);

/* ---- fused SwiGLU MLP block ---------------------------------------------------
 * SwiGLUMLPDataParallelOurs (iron/operators/swiglu_mlp_dp/op_ours.py:47-582;
 * golden swiglu_mlp_dp/test.py:79-91, reference.py:8-67):
 *   a  = bf16(Wo @ cx)            (fuse_o; else a is an input of D)
 *   x1 = bf16(cur + a)
 *   hf = bf16(RMSNorm_w(x1, n_pf))
 *   gh = bf16(silu_tanh(bf16(Wg@hf)) * bf16(Wu@hf))
 *   nxt = bf16(x1 + bf16(Wd@gh))
 * Wires are described like iron_gemv_w8a16 (tile_m, rows_per_core, tiles_per_core).
 * x1_ws (batch*D) and gh_ws (batch*FF) are bf16 workspaces (the reference's
 * a_scratch / gh_scratch round-trip buffers); workspace: the projections' tensor-core
 * scratch from batch 16 on (the largest iron_tc_workspace_bytes of the three; may be
 * NULL), used by one projection at a time. */
int iron_mlp_block(const uint16_t* cur, const uint16_t* a_or_cx, int fuse_o, const uint16_t* n_pf,
                   const void* wo, int wo_tile_m, int wo_rows_per_core, int wo_tiles_per_core,
                   const void* wg, const void* wu, int gu_tile_m, const void* wd, int d_tile_m,
                   int group, int domain, uint16_t* x1_ws, uint16_t* gh_ws, uint16_t* nxt,
                   int D, int FF, int QD, int batch, float eps, void* workspace,
                   int64_t workspace_bytes, void* stream);

/* ---- whole decode step ----------------------------------------------------------
 * One greedy Qwen3 decode token (batch 1) in ONE persistent cooperative kernel:
 * the Qwen3NPU.__call__ chain (qwen3_npu_int8.py:594-621; runlist :249-281) of
 * n_layers x [QKV head, decode attention, fused O-proj + SwiGLU MLP], the final
 * RMSNorm and the lm_head with greedy argmax.  The arithmetic of every stage is
 * the one of the per-operator entry points above (iron_qkv_head with the golden
 * RMSNorm form, iron_decode_attn, iron_mlp_block, iron_rmsnorm mode 1,
 * iron_lm_head_*_argmax): exact int8 x block-floating-point dot products summed in
 * float64, one bf16 rounding per projection output; the down projection is summed
 * over its K slices in slice order.  Results do not depend on timing: two steps from
 * the same state give the same bits.
 * The projections read their weights in 16-row tiles made once by
 * iron_qwen3_pack_tiles (the *_t fields); the plain wires stay in the descriptor for
 * the caller's other paths.  wqkv_t holds the QKV rows in KV-head-group order: for
 * each KV head h the q rows of query heads h*Hq/Hkv .. (h+1)*Hq/Hkv - 1, then the k
 * rows of head h, then its v rows.  wo_t holds the row tiles of Wo.  wgu_t tile t holds gate rows
 * 8t..8t+7 then up rows 8t..8t+7.  wd_t holds for every 16-row tile t of Wd its 4
 * column slices of FF/4 (tiles of K = FF/4), at index 4t + j.  lm_w8, when set, is the int8
 * lm_head in tiles (iron_qwen3_pack_tiles of the V x D wire).
 * Every pointer in the descriptor is a device pointer, weight and table pointers
 * 16-byte aligned (they are bulk-copied); `layers` points to a DEVICE array of n_layers
 * iron_qwen3_layer.  The kernel reads the token from tok[0] (embed_input != 0) or
 * the hidden state from x, the position from pos[0], writes the argmax to tok[0],
 * the final hidden state to x and, when advance != 0, moves pos/seq_len/kv_off one
 * token on.  Activations pass between the CTAs as epoch-tagged words in `attn_ws`
 * (iron_qwen3_attn_ws_bytes()); `sync` holds iron_qwen3_sync_words() int32 words (the
 * error word at index 1, the token epoch, the argmax arrival count); both must be
 * zero before the first step.  Every wait is bounded: on timeout sync[1] holds a
 * nonzero code, the step returns early, and iron_qwen3_sync_reset() must clear
 * both before the next step. */
typedef struct iron_qwen3_layer {
  const uint16_t* norm1;  /* (D) bf16 */
  const void* wqkv;       /* ((Hq+2Hkv)*HD, D) wire */
  const uint16_t* qn;     /* (HD) */
  const uint16_t* kn;     /* (HD) */
  const void* wo;         /* (D, Hq*HD) wire */
  const uint16_t* norm2;  /* (D) */
  const void* wg;         /* (FF, D) wire */
  const void* wu;         /* (FF, D) wire */
  const void* wd;         /* (D, FF) wire */
  const void* wqkv_t;     /* tiles of wqkv, rows in KV-head-group order */
  const void* wo_t;       /* tiles of wo (16 rows, all columns) */
  const void* wgu_t;      /* tiles of 8 rows of wg over the same 8 rows of wu */
  const void* wd_t;       /* tiles of wd cut into 4 slices along K, tile-major */
} iron_qwen3_layer;

typedef struct iron_qwen3_model {
  int D, FF, Hq, Hkv, HD, V, n_layers, group, max_seq;
  float eps;
  const iron_qwen3_layer* layers;  /* device array */
  const uint16_t* final_norm;      /* (D) */
  const uint16_t* embed;           /* (V, D) bf16: embedding, and lm_head when lm_w8 == NULL */
  const void* lm_w8;               /* int8 lm_head tiles (iron_qwen3_pack_tiles of the (V, D) wire), or NULL */
  const uint16_t* angles;          /* (max_seq, HD) interleaved [cos, sin] */
  uint16_t* kv;                    /* (n_layers, Hkv, 2*max_seq*HD) per-token [K_t|V_t] */
  uint16_t* x;                     /* (D) hidden state in (embed_input == 0) / final hidden state out */
  uint16_t* raw;                   /* ((Hq+2Hkv)*HD), unused by the step kernel */
  uint16_t* attn;                  /* (Hq*HD), unused by the step kernel */
  uint16_t* x1;                    /* (D), unused by the step kernel */
  uint16_t* gh;                    /* (FF), unused by the step kernel */
  float* attn_ws;                  /* iron_qwen3_attn_ws_bytes(): the hand-off words */
  void* cand;                      /* iron_qwen3_cand_bytes() */
  int32_t* tok;
  int32_t* pos;
  int32_t* seq_len;
  int32_t* kv_off;
  uint16_t* logits;                /* (V) or NULL */
  int32_t* sync;                   /* iron_qwen3_sync_words() int32 */
  uint16_t* trace;                 /* (n_layers + 1, D) or NULL: the hidden state entering each layer,
                                      then the final one (parity checks layer by layer) */
} iron_qwen3_model;

int iron_qwen3_sync_words(const iron_qwen3_model* m);
int64_t iron_qwen3_attn_ws_bytes(const iron_qwen3_model* m);
int64_t iron_qwen3_cand_bytes(void);
/* Grid size the step kernel will use on the current device (one CTA per SM). */
int iron_qwen3_grid(const iron_qwen3_model* m);
int iron_qwen3_decode_step(const iron_qwen3_model* m, int embed_input, int advance, void* stream);
/* One greedy token with HOST buffers, the form of Qwen3NPU.__call__
 * (qwen3_npu_int8.py:594-621: host writes the step's inputs and params, one dispatch,
 * wait, the result read back on the host).  Copies host_in = {token id, position}
 * (int32; pinned memory keeps the copy asynchronous) to m->tok / m->pos, runs
 * iron_qwen3_decode_step(m, embed_input, advance = 0), copies the next token and the
 * step's error word back into host_out = {next token, error word} and waits for the
 * stream.  Returns IRON_ERR_TIMEOUT (host_out[1] = the device code) when the step
 * stopped on a bounded wait; iron_qwen3_sync_reset clears that state. */
int iron_qwen3_step_host(const iron_qwen3_model* m, const int32_t* host_in, int32_t* host_out, int embed_input,
                         void* stream);
/* Weight tiles for the step kernel, made once at load time from plain wires (no
 * reference counterpart: they re-order the wires that qwen3_npu_int8.py:381-436 packs
 * for the NPU).  Rows [0, M) of a wire whose rows are `row_stride` bytes apart
 * ([K_full int8 | K_full/group bf16]), columns [col0, col0 + K), become ceil(M/16)
 * tiles of iron_qwen3_tiles_bytes(M, K, group) bytes in all: per 32-column block,
 * 32 lanes x 16 bytes in the A-fragment order of mma.sync m16n8k32 (lane l: rows
 * l/4 and l/4 + 8, columns 4(l%4).. and 16 + 4(l%4)..), then per quantisation group
 * the scales of rows g and g + 8 side by side (g < 8).  Rows past M are zero. */
int64_t iron_qwen3_tiles_bytes(int M, int K, int group);
int iron_qwen3_pack_tiles(const void* wire, int64_t row_stride, int M, int K_full, int col0, int K, int group,
                          void* out, void* stream);
/* Zero the sync words and the hand-off words (after a timed-out step, or before first use). */
int iron_qwen3_sync_reset(const iron_qwen3_model* m, void* stream);

/* ---- tensor-parallel building blocks ---------------------------------------------
 * No reference counterpart: IRON decodes on one NPU.  Tensor-parallel Qwen3
 * (iron_b200/tp.py) splits QKV by heads, O and down along K (row-parallel), gate/up
 * by rows and the lm_head by vocabulary; these entry points cut the fused blocks at
 * the cross-rank sums and the cross-rank argmax.
 *
 * iron_gemv_w8a16_ex: iron_gemv_w8a16 on plain wires (tile_m = 1) with the
 * epilogues exposed.  wire_b != NULL: gate/up pair, y = bf16(silu_tanh(bf16(Wa@h)) *
 * bf16(Wb@h)) (epi 0 only).  rms_w != NULL: h = bf16(RMSNorm_w(x)) first (rms_mode as
 * iron_rmsnorm).  epi 0: y bf16 = bf16(sum); 1: y bf16 = bf16(residual + bf16(sum));
 * 2: y float32 = float(sum) (a rank's partial sum).  x rows ld_x apart, y rows ld_y.
 * workspace: as iron_gemv_w8a16. */
int iron_gemv_w8a16_ex(const void* wire_a, const void* wire_b, int M, int K, int group, int domain,
                       const uint16_t* x, int ld_x, int batch, const uint16_t* rms_w, float eps,
                       int rms_mode, const uint16_t* residual, int epi, void* y, int ld_y,
                       void* workspace, int64_t workspace_bytes, void* stream);
/* y = bf16(res + bf16(sum)) elementwise (sum: float32, the all-reduced partials). */
int iron_resid_add_f32(const uint16_t* res, const float* sum, uint16_t* y, int64_t n, void* stream);
/* pairs[b] = (float bits of logits[b, tok[b]], tok[b] + offset): a rank's greedy
 * candidate over its vocabulary rows [offset, offset + M). */
int iron_argmax_pair(const uint16_t* logits, int M, int batch, const int32_t* tok, int offset,
                     int32_t* pairs, void* stream);
/* tok_out[b] = index of the largest value over pairs[r][b], r < n (ties -> lowest index). */
int iron_argmax_merge(const int32_t* pairs, int n, int batch, int32_t* tok_out, void* stream);

/* ---- cross-rank steps over peer memory (NVLink) ------------------------------
 * The all-reduce of the row-parallel partial sums and the all-gather of the argmax
 * pairs without NCCL.  Every rank allocates one symmetric buffer of
 * iron_peer_buffer_bytes(world, cap_words) bytes, zero-filled, whose base addresses
 * (as this rank sees them) are in peers_dev[world]; epochs_dev is a zero-filled
 * uint32[iron_peer_epoch_words(cap_words)] of this rank, err_dev an int32.  A call
 * pushes this rank's n_words 32-bit words of `in` into every rank's buffer with plain
 * stores, publishes them with a system-scope release flag, waits (bounded, 200 ms)
 * for every rank's flags in its own buffer and writes `out`: mode 0 the float32 sum
 * over ranks in rank order (n_words floats, in place allowed), mode 1 the rows of all
 * ranks (world * n_words words).  Every rank makes the same calls in the same order,
 * each on its own GPU: the call waits for the other ranks' calls.  A timed-out wait
 * stores 1 in *err_dev and leaves `out` unwritten.  Replaces NCCL's all_reduce /
 * all_gather in the tensor-parallel split (no reference counterpart: IRON decodes on
 * one NPU). */
int64_t iron_peer_buffer_bytes(int world, int cap_words);
int iron_peer_epoch_words(int cap_words);
int iron_peer_exchange(const unsigned long long* peers_dev, int world, int rank, int cap_words, const void* in,
                       void* out, int n_words, int mode, uint32_t* epochs_dev, int* err_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IRON_B200_H */
