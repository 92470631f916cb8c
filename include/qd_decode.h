/* qd_decode.h - C ABI of the B200 (sm_100a) Qwen3 greedy-decode kernels.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream; nothing here allocates,
 * synchronises or reads device memory on the host. The entry points that take their scratch from the
 * caller can be captured in a CUDA graph.
 * All buffers are caller-owned. Scratch buffers (split-K partial sums and tickets) are sized by the
 * matching *_plan call, must be zero-filled once after allocation, and are left zero-ready by every
 * successful launch. Two launches that share a scratch buffer must not overlap on the GPU.
 *
 * Return value: 0 (QD_OK) or a QD_ERR_* code; qd_last_error() describes the last failure of the
 * calling thread. Device-side bounded waits report through the caller's `err` word (QD_DEVERR_*),
 * which the host reads after a step; a wait never spins for more than about one second.
 *
 * The reference (Yokanater/htn-2026) has no C/C++ or CUDA code: its decode path is Python calling
 * Triton kernels through small wrapper classes. Each entry point below names the wrapper and
 * kernel it replaces, by file:line in that repository.
 */
#ifndef QD_DECODE_H
#define QD_DECODE_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  QD_OK = 0,
  QD_ERR_ARG = 1,         /* invalid pointer, size, stride or alignment */
  QD_ERR_SCRATCH = 2,     /* scratch buffer smaller than the plan requires */
  QD_ERR_CUDA = 3,        /* CUDA runtime error at launch */
  QD_ERR_UNSUPPORTED = 4  /* shape outside what the kernels are built for */
};

enum {
  QD_EPI_STORE = 0,
  QD_EPI_RES = 1,
  QD_EPI_SWIGLU = 2,
  QD_EPI_SWIGLU_PACKED = 3,
  QD_EPI_RES_SUMS = 4,
  QD_EPI_STORE_SUMS = 5
};

enum {
  QD_DEVERR_WAIT_FULL = 1,
  QD_DEVERR_WAIT_EMPTY = 2,
  QD_DEVERR_DRAIN = 4,
  QD_DEVERR_TOKEN = 8,
  QD_DEVERR_POS = 16,
  QD_DEVERR_DEP = 32,
  QD_DEVERR_SMEM = 64 /* a kernel found its dynamic shared memory misaligned and did nothing */
};

/* Library identification and the last error message of the calling thread. */
const char* qd_version(void);
const char* qd_last_error(void);
/* Streaming multiprocessors of the current device. */
int qd_sm_count(int* out);

/* ---------------------------------------------------------------- weight packing
 * Replaces the reference loader's layer-stacked packing copies (engine/engine.py:255-282).
 * The packed layout is 16 KiB blocks of 128 rows x 64 columns, row-group-major, each 128-byte row
 * with its 16-byte chunks swizzled (chunk c of row r at position c ^ (r & 7)).
 * qd_pack_rows copies rows j = 0..n_src_rows-1 of a row-major BF16 source [n_src_rows, k] (row
 * stride ld_src elements) into logical rows
 *     (j / span) * group_stride + row_offset + (j % span)
 * of a packed [n_dst_rows, k] destination. Plain stacking: span = n_src_rows, group_stride = 0,
 * row_offset = first row. Gate/up interleave of the SwiGLU matrix: span = 64, group_stride = 128,
 * row_offset = 0 (gate) or 64 (up). n_dst_rows % 128 == 0, k % 64 == 0. */
int64_t qd_packed_bytes(int64_t n_rows, int64_t k);
int qd_pack_rows(const void* src, int64_t ld_src, int64_t n_src_rows, int64_t k, void* dst, int64_t n_dst_rows,
                 int64_t span, int64_t group_stride, int64_t row_offset, cudaStream_t stream);

/* ---------------------------------------------------------------- embedding
 * Replaces embed_ss (engine/kernels/fast.py:53-76) / F.embedding (engine/engine.py:338):
 * x[i, :] = E[tok[i], :] for i < m, gathered from the packed embedding matrix (tied with the LM head).
 * Out-of-range token ids are clamped and flagged with QD_DEVERR_TOKEN in *err. */
int qd_embed(const int64_t* tok, const void* e_packed, int64_t vocab, int64_t k, int m, void* x, int64_t ldx,
             int* err, int pdl, cudaStream_t stream);

/* ---------------------------------------------------------------- streaming GEMV
 * Replaces FastGemm (engine/kernels/fast.py:173-213, kernel :99-158) and Gemv + split-K reduce
 * (engine/kernels/gemv.py:157-248, kernels :60-115):
 *   y[i, :] = xn[i, :] . W^T,  xn = norm_w ? bf16(norm_w * bf16(x * rsqrt(mean(x^2) + eps))) : x
 *   QD_EPI_STORE   out = bf16(y)
 *   QD_EPI_RES     out = bf16(res + bf16(y))                   (out may alias res)
 *   QD_EPI_SWIGLU  W is the gate/up matrix packed interleaved (64 gate rows, then the 64 up rows of
 *                  the same outputs, per 128-row group); out[i, j] = bf16(bf16(silu(bf16 g)) * bf16 u),
 *                  out has n / 2 columns
 * x [m, k] BF16 (row stride ldx), W packed [n, k], 1 <= m <= 8, n % 128 == 0, k % 64 == 0.
 * grid_hint <= 0 picks one CTA per SM. */
int qd_gemv_plan(int64_t n, int64_t k, int m, int grid_hint, int* grid, int64_t* scratch_bytes);
int qd_gemv(const void* x, int64_t ldx, const void* w_packed, int64_t n, int64_t k, int m, void* out, int64_t ldo,
            const void* res, int64_t ldr, const void* norm_w, float eps, int epilogue, int grid, void* scratch,
            int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream);

/* Allocation-free qd_gemv, for callers that cannot allocate device memory: a host whose device
 * memory is owned end to end by its own pool allocator and which passes only input and output
 * buffers, a plugin inside such a host with no allocator handle, or a latency-critical loop that must
 * not call cudaMalloc (it can synchronize the device). Same arguments and results as qd_gemv with
 * grid_hint 0, but no grid or scratch: scratch is a 4 MiB array compiled into the library, which every
 * GPU that loads it holds until exit; shapes whose plan needs more return QD_ERR_UNSUPPORTED. The
 * first call on each device looks up that array's device address (with that device current); make
 * this first call before any stream capture begins. The address is then kept for the life of the
 * process, so a device reset (cudaDeviceReset) or a re-created primary context between calls is not
 * supported. Every call clears the array's tickets (a memset on the stream) and reuses the array, so
 * calls that may overlap on the GPU (other streams, other threads) race and must be serialized by the
 * caller. It has no counterpart in the reference. */
int qd_gemv_noalloc(const void* x, int64_t ldx, const void* w_packed, int64_t n, int64_t k, int m, void* out,
                    int64_t ldo, const void* res, int64_t ldr, const void* norm_w, float eps, int epilogue, int* err,
                    int pdl, cudaStream_t stream);

/* QKV projection with the attention prologue fused into its epilogue. Replaces FastGemm "qkv"
 * (engine/engine.py:472) plus the q/k RMSNorm + RoPE + KV-cache append of FastAttention
 * (engine/kernels/fast.py:240-293) / qk_norm_rope_cache (engine/kernels/fused.py:23-98, pos_mode 1).
 * W packed [(nq + 2 nkv) * 128, k] rows q | k | v (head_dim 128). For every row i < m and position
 * p = *pos: q_out[i, h, :] = rope(rmsnorm(q_h)), k_cache[i, kvh, p, :] = rope(rmsnorm(k_kvh)),
 * v_cache[i, kvh, p, :] = v_kvh; caches are [m, nkv, cap, 128] with strides cs_b, cs_h (elements),
 * cos/sin are [cap, 128] BF16 tables. raw_out (optional) receives the BF16 projection [m, n].
 * A device position outside [0, cap) writes nothing and sets QD_DEVERR_POS in *err. */
int qd_qkv_rope_append(const void* x, int64_t ldx, const void* w_packed, int64_t k, int m, const void* norm_w,
                       float eps, const void* q_norm, const void* k_norm, const void* cos, const void* sin,
                       const int64_t* pos, int64_t cap, int nq_heads, int nkv_heads, void* q_out, void* k_cache,
                       void* v_cache, int64_t cs_b, int64_t cs_h, void* raw_out, int grid, void* scratch,
                       int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream);

/* LM head with final RMSNorm prologue and argmax epilogue. Replaces FastLmHead
 * (engine/kernels/fast.py:380-465) / LmHeadArgmax (engine/kernels/gemv.py:118-287):
 * logits = bf16(xn . E^T), tok[i] = argmax (lowest index on exact ties), *pos += inc_pos.
 * E packed [roundup(vocab, 128), k]; logits_out (optional) [m, vocab] BF16 with row stride ld_logits. */
int qd_lm_head_plan(int64_t vocab, int64_t k, int m, int grid_hint, int* grid, int64_t* scratch_bytes);
int qd_lm_head_argmax(const void* x, int64_t ldx, const void* e_packed, int64_t vocab, int64_t k, int m,
                      const void* norm_w, float eps, int64_t* tok, int64_t* pos, int inc_pos, void* logits_out,
                      int64_t ld_logits, int grid, void* scratch, int64_t scratch_bytes, int* err, int pdl,
                      cudaStream_t stream);

/* ---------------------------------------------------------------- tensor-core batch path (16..64 rows)
 * The same projections for batches of 16 to 64 sequences on the tcgen05 tensor cores (swap-AB: the
 * 128 weight rows of a packed block are the MMA M dimension, the batch padded to n_pad in
 * {16, 32, 48, 64} is N, fp32 accumulators in tensor memory). Replaces FastGemm at M > 8
 * (engine/kernels/fast.py:173-213, whose Triton tl.dot tile covers up to GEMV_MAX_B = 64 rows,
 * engine/engine.py:91) and FastLmHead at the same batch sizes (fast.py:439-465). Results equal
 * qd_gemv / qd_qkv_rope_append / qd_lm_head_argmax up to the fp32 summation order of the dot
 * products (rounded to BF16 at the same points).
 *
 * qd_pack_act writes the activation operand: xpk = [k / 64][n_pad][64] BF16 tiles in the
 * 128-byte-swizzled K-major layout of the weight blocks (16-byte chunk c of row m at c ^ (m & 7)),
 * from x [m_act, k] (row stride ldx), with the RMSNorm prologue applied when norm_w is given. Rows
 * m_act..n_pad-1 are not written: zero them once (their products are computed and discarded).
 * xpk needs k * n_pad * 2 bytes, 16-byte aligned. */
int qd_pack_act(const void* x, int64_t ldx, int m_act, int n_pad, int64_t k, const void* norm_w, float eps, void* xpk,
                int pdl, cudaStream_t stream);
/* grid_hint <= 0 picks one CTA per SM. Scratch (zero-filled once, self-resetting) depends on n_pad. */
int qd_tc_gemv_plan(int64_t n, int64_t k, int n_pad, int grid_hint, int* grid, int64_t* scratch_bytes);
/* qd_gemv's STORE / RES / SWIGLU epilogues for rows 0..m_act-1 of the packed activations.
 * QD_EPI_SWIGLU_PACKED: the SwiGLU output goes straight into the packed activation layout of the next
 * projection (`out` = [n/128][n_pad][64] tiles, as qd_pack_act would write it; ldo unused). */
int qd_tc_gemv(const void* xpk, int n_pad, int m_act, const void* w_packed, int64_t n, int64_t k, void* out,
               int64_t ldo, const void* res, int64_t ldr, int epilogue, int grid, void* scratch,
               int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream);
/* QD_EPI_RES_SUMS (qd_tc_gemv): the residual add is deferred - `out` is an int64 [m_act][n] buffer of
 * fixed-point group sums (value * 2^32, zero on entry), which every CTA adds its split-K partials into
 * with integer atomics (order-independent, so deterministic); res / ldo are unused. qd_pack_act_res
 * then applies it: x row m = bf16(x + bf16(sum)) (written back to x), the sums cleared to zero, and the
 * row packed as qd_pack_act does (RMSNorm-ed when norm_w is given). This takes the split-K last
 * arriver's reduction off the path between a residual projection and the next one. */
int qd_pack_act_res(void* x, int64_t ldx, int m_act, int n_pad, int64_t k, void* fx_sums, const void* norm_w,
                    float eps, void* xpk, int pdl, cudaStream_t stream);
/* QD_EPI_STORE_SUMS (qd_tc_gemv): the projection output stays as fixed-point sums in `out` (int64
 * [m_act][n], zero on entry), as for QD_EPI_RES_SUMS. qd_qkv_rope_sums applies the QKV epilogue to them
 * - the arithmetic of qd_tc_qkv_rope_append's (per-head RMSNorm, RoPE at *pos, q to q_out [m][nq][128],
 * K/V appended at *pos) - and clears them: the decode QKV of the tensor-core chain without a split-K
 * last arriver. A position outside [0, cap) flags QD_DEVERR_POS and writes nothing. */
int qd_qkv_rope_sums(void* sums, int64_t lds, int m_act, int nq_heads, int nkv_heads, const void* q_norm,
                     const void* k_norm, float eps, const void* cos, const void* sin, const int64_t* pos, int64_t cap,
                     void* q_out, void* k_cache, void* v_cache, int64_t cs_b, int64_t cs_h, int* err, int pdl,
                     cudaStream_t stream);
/* qd_qkv_rope_append from packed activations (plan with n = (nq + 2 nkv) * 128). */
int qd_tc_qkv_rope_append(const void* xpk, int n_pad, int m_act, const void* w_packed, int64_t k, const void* q_norm,
                          const void* k_norm, const void* cos, const void* sin, const int64_t* pos, int64_t cap,
                          int nq_heads, int nkv_heads, void* q_out, void* k_cache, void* v_cache, int64_t cs_b,
                          int64_t cs_h, void* raw_out, int grid, void* scratch, int64_t scratch_bytes, int* err,
                          int pdl, cudaStream_t stream);
/* qd_lm_head_argmax from packed activations (plan with n = vocab rounded up to 128). */
int qd_tc_lm_head_argmax(const void* xpk, int n_pad, int m_act, const void* e_packed, int64_t vocab, int64_t k,
                         int64_t* tok, int64_t* pos, int inc_pos, void* logits_out, int64_t ld_logits, int grid,
                         void* scratch, int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream);

/* ---------------------------------------------------------------- decode attention
 * Split-K GQA flash-decode with a log-sum-exp merge. Replaces DecodeAttention
 * (engine/kernels/decode_attn.py:26-119) and the flash-decode + merge part of FastAttention
 * (engine/kernels/fast.py:252-331, :345-376). One query per sequence at position p = *pos over keys
 * [0, p] (the new token's K/V are already in the cache): out[b, h, :] = softmax(q k^T * scale) v with
 * query head h reading KV head h / (nq / nkv). q, out [batch, nq, 128] BF16; caches
 * [batch, nkv, cap, 128] with strides cs_b, cs_h. Scores and softmax in fp32, probabilities rounded
 * to BF16 before P.V, fp32 accumulation; the last split to finish merges (fixed split order).
 * A device position outside [0, cap) reads no key beyond the cache and sets QD_DEVERR_POS in *err. */
int qd_attn_plan(int batch, int nkv_heads, int64_t cap, int grid_hint, int* splits, int64_t* chunk,
                 int64_t* scratch_bytes);
int qd_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out, int batch,
                   int nq_heads, int nkv_heads, int64_t cap, int64_t cs_b, int64_t cs_h, int splits, int64_t chunk,
                   float scale, void* scratch, int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream);

/* Streaming variant of qd_attn_decode for large batch x length (same inputs, outputs and arithmetic
 * up to fp32 summation order). The 32-key chunks of all (sequence, KV head) pairs are dealt out
 * evenly over `grid` CTAs (stream-K), each moving K/V through a shared-memory ring with bulk copies;
 * a pair split across CTAs is merged by its last CTA in CTA order. grid_hint <= 0 picks three CTAs
 * per SM. Scratch (zero-filled once, self-resetting) comes from qd_attn_stream_plan, and grid / smax
 * must be the plan's values. Replaces the same reference kernels as qd_attn_decode. */
int qd_attn_stream_plan(int batch, int nkv_heads, int64_t cap, int grid_hint, int* grid, int* smax,
                        int64_t* scratch_bytes);
int qd_attn_decode_stream(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                          int batch, int nq_heads, int nkv_heads, int64_t cap, int64_t cs_b, int64_t cs_h, int grid,
                          int smax, float scale, void* scratch, int64_t scratch_bytes, int* err, int pdl,
                          cudaStream_t stream);

/* Tensor-core variant of qd_attn_decode_stream: 128-key chunks, q.k and P.V as tcgen05 MMAs (keys /
 * dims x 16 columns holding the 4 query heads), K/V by TMA with 128-byte swizzle, softmax in fp32 on
 * the CUDA cores between the two MMAs, probabilities rounded to BF16. Same inputs, outputs, merge and
 * error behaviour; grid_hint <= 0 picks one CTA per SM; grid / smax must be qd_attn_tc_plan's values.
 * out_npad = 0: out is [batch, nq, 128]; out_npad = 16..64 (>= batch, multiple of 16): out is the packed
 * activation operand of the O projection, [nq * 2][out_npad][64] tiles (qd_pack_act's layout).
 * With pdl = 1 the kernel reads *pos and copies the cached keys / values of every chunk that does not
 * hold position *pos before it waits on the preceding kernel, so those, and *pos, must be written
 * before that kernel starts; the preceding kernel may write q and the new row at *pos. */
int qd_attn_tc_plan(int batch, int nkv_heads, int64_t cap, int grid_hint, int* grid, int* smax,
                    int64_t* scratch_bytes);
int qd_attn_decode_tc(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                      int out_npad, int batch, int nq_heads, int nkv_heads, int64_t cap, int64_t cs_b, int64_t cs_h, int grid,
                      int smax, float scale, void* scratch, int64_t scratch_bytes, int* err, int pdl,
                      cudaStream_t stream);

/* ---------------------------------------------------------------- persistent decode step
 * One launch = one whole decode step: embedding, every layer (the five ops above, same arithmetic,
 * same stream-K partition and attention splits, so bit-identical results) and the LM head with
 * argmax and position advance. Replaces the reference's persistent megakernel tier T6
 * (engine/kernels/mega.py:48-223, MegaStep) and its per-op launch sequence T5
 * (engine/engine.py:463-477). One CTA per SM, launched cooperatively: a producer warp streams every
 * projection's weights in op order through a deep shared-memory ring, consumers wait (bounded, 1 s)
 * on completion counters of the op that produces their input. All fields are 8 bytes wide.
 * Weights are packed (qd_pack_rows) and layer-stacked with the given byte strides; norms are
 * [layers, hidden] (ln1, ln2), [layers, 128] (q_norm, k_norm), [hidden] (final_norm); caches are
 * [layers, batch, nkv, cap, 128] with element strides cache_layer_stride, cs_b, cs_h; x [batch,
 * hidden], q and attn [batch, nq, 128], act [batch, inter]; logits (optional) [batch, ld_logits].
 * `err` is required. 1 <= batch <= 8. qd_decode_step_plan gives the scratch size (zero-fill once;
 * re-zero after any device error) and the attention split count. */
typedef struct qd_step_desc {
  const void* w_qkv;
  int64_t w_qkv_layer_bytes;
  const void* w_o;
  int64_t w_o_layer_bytes;
  const void* w_gu;
  int64_t w_gu_layer_bytes;
  const void* w_down;
  int64_t w_down_layer_bytes;
  const void* e_packed;
  const void* ln1;
  const void* ln2;
  const void* q_norm;
  const void* k_norm;
  const void* final_norm;
  int64_t layers, hidden, inter, nq_heads, nkv_heads, vocab, batch;
  double eps, scale;
  int64_t* tok;
  int64_t* pos;
  void* x;
  void* q;
  void* attn;
  void* act;
  void* k_cache;
  void* v_cache;
  int64_t cache_layer_stride, cs_b, cs_h, cap;
  const void* cos;
  const void* sin;
  void* logits;
  int64_t ld_logits;
  int* err;
  /* optional timeline (%globaltimer ns), [grid][ops][4] with ops = 2 + 5 layers in step order
   * (embed, layers x {qkv, attn, o, gate_up, down}, lm): input ready, inputs staged, op done, and the
   * time the producer issued the op's last block; null disables it */
  uint64_t* trace;
} qd_step_desc;

int qd_decode_step_plan(const qd_step_desc* desc, int64_t* scratch_bytes, int* attn_splits);
int qd_decode_step(const qd_step_desc* desc, void* scratch, int64_t scratch_bytes, cudaStream_t stream);

/* Persistent tcgen05 decode step for batches of 4..64 (one cooperative launch per step): the tensor-core
 * kernel chain (qd_pack_act, qd_tc_qkv_rope_append, qd_attn_decode_tc, qd_tc_gemv, qd_tc_lm_head_argmax)
 * inside one launch with the same partitions and arithmetic, so its tokens and logits are
 * bit-identical to the chain's. Same descriptor as qd_decode_step (its `attn` and `act` buffers are
 * not used) plus the three packed activation operands, each [k/64][n_pad][64] BF16 zero-filled once:
 * xh (k = hidden), xa (k = nq * 128), xi (k = inter); n_pad = batch rounded up to 16 (the plan's).
 * Replaces the reference's per-op FastGemm / FastAttention launches at batch > 8 (engine/engine.py:463-477). */
int qd_tc_decode_step_plan(const qd_step_desc* desc, int64_t* scratch_bytes, int* n_pad);
int qd_tc_decode_step(const qd_step_desc* desc, void* xh, void* xa, void* xi, void* scratch, int64_t scratch_bytes,
                      cudaStream_t stream);

/* ---------------------------------------------------------------- prompt (prefill) path
 * The prefill forward (engine/engine.py:550-592) on the same packed weights as decode.
 *
 * qd_tc_gemm replaces its F.linear calls (engine/engine.py:564, :580-589) and the fused epilogues that
 * follow them: out[t, :] = epilogue(x[t, :] . W^T) for t < m, on the tcgen05 tensor cores (tiles of
 * 128 tokens x 128 or 256 weight rows, fp32 accumulation in tensor memory). x [m, k] BF16 row-major
 * (row stride ldx, 16-byte aligned, ldx % 8 == 0), W packed [n, k] (n % 128 == 0, k % 64 == 0).
 * Epilogues as qd_gemv: QD_EPI_STORE out = bf16(y); QD_EPI_RES out = bf16(res + bf16(y)) (out may
 * alias res); QD_EPI_SWIGLU (W = the interleaved gate/up matrix) out [m, n / 2] =
 * bf16(bf16(silu(bf16 g)) * bf16 u). One launch, persistent over the tiles; the tiles that fill whole
 * waves of SMs run whole, and the tiles of a last, partial wave (all of them for a short prompt) are split
 * along K across CTAs: each split stores its fp32 partial in the caller's scratch and a second launch
 * (programmatic dependent launch, same stream) sums the partials in split order (deterministic) and
 * applies the epilogue. Every launch waits for the previous kernel of the stream (griddepcontrol.wait)
 * before reading x or res. qd_tc_gemm_plan reports the grid, tile width, K split and
 * the scratch bytes needed (0 without a split; otherwise 16-byte aligned, any contents; launches that
 * share one scratch run in stream order, so one buffer of the largest size serves every shape). */
int qd_tc_gemm_plan(int64_t m, int64_t n, int64_t k, int* grid, int* bn, int* ksplit, int64_t* scratch_bytes);
int qd_tc_gemm(const void* x, int64_t ldx, int64_t m, const void* w_packed, int64_t n, int64_t k, void* out,
               int64_t ldo, const void* res, int64_t ldr, int epilogue, void* scratch, int64_t scratch_bytes, int* err,
               cudaStream_t stream);

/* Row RMSNorm, out[i] = bf16(w * bf16(x[i] * rsqrt(mean(x[i]^2) + eps))): replaces the torch / Triton
 * norm of the prefill (engine/engine.py:505-509, engine/kernels/rmsnorm.py:14-32). k % 8 == 0,
 * 16-byte aligned rows. */
int qd_rmsnorm_rows(const void* x, int64_t ldx, int64_t m, int64_t k, const void* norm_w, float eps, void* out,
                    int64_t ldo, cudaStream_t stream);

/* ---------------------------------------------------------------- token-tree verification
 * Replace the reference's tree kernels (engine/kernels/tree.py:25-164: tree q/k RoPE at depth positions,
 * ancestor-masked attention, KV compaction) for exact token-tree speculation. Each of the B sequences
 * verifies one draft tree of T nodes (node 0 = its last emitted token, parents before children); row
 * b * T + t of the B * T activation rows is node t of sequence b. slot0 / prefix (device int32 [B]) is
 * the cache slot of each sequence's root: node t's keys / values go to slot prefix[b] + t. Caches are
 * [B][nkv][cap][128] (sequence stride cs_b, head stride cs_h).
 *
 * qd_tree_qk_rope: per-node q/k RMSNorm + RoPE as qd_prefill_qk_rope_at, rotated at position
 * rope_pos[row] (device int32 [B * T]: the root's slot + the node's depth). A position outside [0, cap)
 * is clamped and flags QD_DEVERR_POS; a sequence whose slots slot0[b] .. slot0[b] + T - 1 leave the
 * cache writes no keys / values and flags QD_DEVERR_POS.
 * qd_tree_attn: out[row] = attention of the node's query heads over its sequence's cache slots
 * [0, prefix[b]) and the tree slots prefix[b] + j with bit j of anc[row] set (device uint32 [B * T]: the
 * node and its ancestors); 1 <= T <= 32, 4 query heads per KV head. Same arithmetic as qd_attn_decode.
 * A sequence with prefix[b] < 0 or prefix[b] + T > cap gets zeros and flags QD_DEVERR_POS in *err.
 * qd_tree_compact: for each move i in order (device int32 [n][3]: sequence, source slot, destination
 * slot), the key and value rows of every layer and KV head are copied from the source to the destination
 * slot of that sequence; caches [layers][B][nkv][cap][128] at layer stride layer_stride; moves naming a
 * sequence or slot outside the cache are skipped; n <= 4096. */
int qd_tree_qk_rope(const void* qkv, int64_t ldqkv, int batch, int T, const int32_t* slot0, const int32_t* rope_pos,
                    int nq_heads, int nkv_heads, const void* q_norm, const void* k_norm, float eps, const void* cos,
                    const void* sin, void* q_out, int64_t ldq, void* k_cache, void* v_cache, int64_t cap,
                    int64_t cs_b, int64_t cs_h, int* err, cudaStream_t stream);
int qd_tree_attn(const void* q, int64_t ldq, int batch, int T, int nq_heads, int nkv_heads, const void* k_cache,
                 const void* v_cache, int64_t cap, int64_t cs_b, int64_t cs_h, const int32_t* prefix,
                 const uint32_t* anc, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream);
/* qd_tree_attn for one sequence on the tensor cores: the T = S - q_begin tree rows (q [T, nq * 128],
 * row stride ldq; node t at slot q_begin + t) attend to the keys [0, q_begin) and to the tree slots of
 * their ancestors (anc: device uint32 [T]); caches [nkv][cap][128] (head stride cs_h). The prompt
 * attention kernel (qd_prefill_attn_rows) with the ancestor mask applied in its softmax; 1 <= T <= 32. */
int qd_tree_attn_rows(const void* q, int64_t ldq, int64_t S, int64_t q_begin, const uint32_t* anc, int nq_heads,
                      int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_h, float scale,
                      void* out, int64_t ldo, int* err, cudaStream_t stream);
int qd_tree_compact(void* k_cache, void* v_cache, int layers, int64_t layer_stride, int batch, int64_t cs_b,
                    int nkv_heads, int64_t cs_h, int64_t cap, const int32_t* moves, int n, cudaStream_t stream);

/* Greedy token of each row of BF16 logits: out[i] = argmax over j < n of logits[i * ld + j], the lowest
 * index among exact ties. Replaces the torch.argmax over the prompt's last-position logits that picks
 * the first generated token (engine/engine.py:583-591). ld % 8 == 0, logits 16-byte aligned. Launched
 * as a programmatic dependent (it waits for the kernel before it). */
int qd_argmax_rows(const void* logits, int64_t ld, int64_t n, int64_t rows, int64_t* out, cudaStream_t stream);

/* Prompt q/k RMSNorm + RoPE + KV-cache write: replaces qk_norm_rope_cache with pos_mode 0
 * (engine/kernels/fused.py:23-98, called from engine/engine.py:566-572). qkv [batch * S, (nq + 2 nkv) * 128]
 * (token i * S + s at position s); q_out [batch * S, nq * 128] receives rope(rmsnorm(q)); k_cache /
 * v_cache [batch, nkv, cap, 128] (strides cs_b, cs_h) receive positions 0..S-1. */
int qd_prefill_qk_rope(const void* qkv, int64_t ldqkv, int batch, int64_t S, int nq_heads, int nkv_heads,
                       const void* q_norm, const void* k_norm, float eps, const void* cos, const void* sin, void* q_out,
                       int64_t ldq, void* k_cache, void* v_cache, int64_t cap, int64_t cs_b, int64_t cs_h,
                       cudaStream_t stream);

/* As qd_prefill_qk_rope with the tokens of every sequence at positions pos0 .. pos0 + S - 1 (token i * S + s
 * at pos0 + s: cos / sin row and cache slot pos0 + s; pos0 + S <= cap): the speculative verify's
 * qk_norm_rope_cache (engine/kernels/fused.py:23-98 with pos_mode 2, called from engine/engine.py:489-490)
 * for sequences that share the position, and a prompt continued after a cached prefix. */
int qd_prefill_qk_rope_at(const void* qkv, int64_t ldqkv, int batch, int64_t S, int64_t pos0, int nq_heads,
                          int nkv_heads, const void* q_norm, const void* k_norm, float eps, const void* cos,
                          const void* sin, void* q_out, int64_t ldq, void* k_cache, void* v_cache, int64_t cap,
                          int64_t cs_b, int64_t cs_h, cudaStream_t stream);

/* Prompt causal attention (flash attention on the tensor cores): replaces the prefill's
 * F.scaled_dot_product_attention(q, K, V, is_causal=True, enable_gqa=True) (engine/engine.py:579,
 * :584, :517-531). For every sequence i < batch, query head h and prompt position s in
 * [q_begin, S): out[i * (S - q_begin) + s - q_begin, h * 128 ..] = softmax(q k^T * scale) v over keys
 * 0..s of KV head h / (nq / nkv). q [batch * S, nq * 128] (row stride ldq, token i * S + s, as
 * qd_prefill_qk_rope writes it); k_cache / v_cache [batch, nkv, cap, 128] hold positions 0..S-1
 * (strides cs_b, cs_h). q_begin = 0 is the whole prompt; q_begin = S - 1 gives the last position
 * only (the reference's last layer, engine/engine.py:577-583). Rows are 16-byte aligned, ldq and
 * ldo multiples of 8. QD_PREFILL_ATTN=2 in the environment selects the two-query-tile variant (query
 * heads 2j and 2j + 1 of a KV head share each K / V tile, P kept in tensor memory); same results up to
 * the fp32 summation order. */
int qd_prefill_attn(const void* q, int64_t ldq, int batch, int64_t S, int64_t q_begin, int nq_heads, int nkv_heads,
                    const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b, int64_t cs_h, float scale,
                    void* out, int64_t ldo, int* err, cudaStream_t stream);

/* As qd_prefill_attn with q holding only the query rows that are computed: q[i * (S - q_begin) + s - q_begin]
 * for positions s in [q_begin, S) (the layout of out). The speculative verify's attention (VerifyAttention,
 * engine/kernels/decode_attn.py:122-206, engine/engine.py:491): the S - q_begin verify tokens attend
 * causally to the cached prefix and to each other. */
int qd_prefill_attn_rows(const void* q, int64_t ldq, int batch, int64_t S, int64_t q_begin, int nq_heads,
                         int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b,
                         int64_t cs_h, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QD_DECODE_H */
