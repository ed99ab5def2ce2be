/* agxc.h — C ABI of libagxcuda.so, the B200 (sm_100a) quantized-decode library.
 *
 * This ABI replaces the process boundary of the reference's decode path: agxforge/inference/execute.py:37-49 runs
 * the Metal executor tools/g17decodegen.m as a subprocess (graph.json in, a JSON report out). Here the host calls
 * these entry points in-process; the Python package agxforge_b200 binds them with ctypes.
 *
 * Conventions
 *   - Every entry point returns 0 (AGXC_OK) or a negative AGXC_E* code; agxc_last_error() gives the message for the
 *     calling thread's last failure.
 *   - Pointers named *_dev are device pointers (e.g. from torch tensors; the caller keeps ownership). Host arrays
 *     are read or written synchronously and never retained.
 *   - A context owns one device and one CUDA stream; calls on one context are not concurrent. A model owns every
 *     device buffer it allocates (weights, KV cache, activations, scratch) and frees them in agxc_model_free.
 *   - `stream` arguments are cudaStream_t values passed as void* (NULL = the context's stream).
 */
#ifndef AGXC_H
#define AGXC_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AGXC_API __attribute__((visibility("default")))
#else
#define AGXC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AGXC_OK 0
#define AGXC_EINVAL (-1)      /* bad argument or shape (the reference raises ValueError, qmv.py:74-80) */
#define AGXC_ECUDA (-2)       /* a CUDA runtime call failed */
#define AGXC_ENCCL (-3)       /* a collective failed */
#define AGXC_ETIMEOUT (-4)    /* a bounded device wait gave up (the kernel set the error word) */
#define AGXC_ECORRUPT (-5)    /* a guard or sentinel check failed */
#define AGXC_ENOMEM (-6)      /* device allocation failed */
#define AGXC_EUNSUPPORTED (-7)

#define AGXC_SCALE_FP16 0
#define AGXC_SCALE_BF16 1

#define AGXC_TOKEN_UNSET 0xFFFFFFFFu  /* a free log entry: the model chooses (agxforge/kernels/argmax.py:133-145) */

typedef struct agxc_ctx agxc_ctx;
typedef struct agxc_pack agxc_pack;
typedef struct agxc_model agxc_model;

/* ---- context -------------------------------------------------------------------------------------------- */
AGXC_API const char* agxc_last_error(void);
AGXC_API int agxc_version(void);
/* Opens `device` and creates the context's stream. */
AGXC_API int agxc_init(int device, agxc_ctx** out);
AGXC_API void agxc_ctx_free(agxc_ctx* ctx);
AGXC_API int agxc_ctx_sync(agxc_ctx* ctx);
/* The context's own stream (the one NULL `stream` arguments and the model / encoder calls enqueue on), as a
 * cudaStream_t in *stream: a caller that produces device inputs on another stream orders the two with events. */
AGXC_API int agxc_ctx_stream(agxc_ctx* ctx, void** stream);
/* The context's device error word (bounded waits that gave up set bits in it); 0 = clean. Reading clears it. */
AGXC_API int agxc_ctx_error_word(agxc_ctx* ctx, uint32_t* word);

/* ---- weight packs (agxforge/kernels/qmv.py:17-18, 1854-1880) ------------------------------------------------
 * Reference format: packed uint32 [n][k*bits/32], element k of row n in bits [bits*(k % (32/bits)), ...) of word
 * k/(32/bits) (low field first); scales and biases 16-bit [n][k/group] (fp16 or bf16 patterns). */
typedef struct {
  int32_t n, k, bits, group, scale_dtype;
} agxc_pack_desc;

/* Quantise fp32 weights [n][k] on the device into the reference format (replaces qmv.quantize, qmv.py:1854). */
AGXC_API int agxc_quantize_dev(agxc_ctx* ctx, const agxc_pack_desc* desc, const float* w_dev, uint32_t* packed_dev,
                      uint16_t* scales_dev, uint16_t* biases_dev, void* stream);

/* Upload a reference-format pack and re-lay it out for the B200 GEMV (16x64 tiles, 128-bit loads per lane).
 * `on_device` = 1 when the three arrays are device pointers, 0 when they are host arrays. */
AGXC_API int agxc_pack_create(agxc_ctx* ctx, const agxc_pack_desc* desc, const void* packed, const void* scales,
                     const void* biases, int on_device, agxc_pack** out);
AGXC_API void agxc_pack_free(agxc_pack* pack);
/* Bytes of the device copy (fields + scale/bias), for roofline accounting. */
AGXC_API int64_t agxc_pack_bytes(const agxc_pack* pack);
/* The pack's fields unpacked to uint8 [n][k] (replaces assemble._unpack, assemble.py:834-840) and its fp32 weights
 * w = fma(q, s, b) rounded once (the dequant contract of qmv_dq_reference, qmv.py:1699-1750). Device outputs. */
AGXC_API int agxc_pack_unpack_dev(const agxc_pack* pack, uint8_t* fields_dev, void* stream);
AGXC_API int agxc_pack_dequant_dev(const agxc_pack* pack, float* w_dev, void* stream);

/* ---- the GEMV family (agxforge/kernels/qmv.py build_qmv2 341-881 and its epilogues) ---------------------------
 * y[b][n] = sum_k x[b][k] * (s[n,g] q[n,k] + b[n,g]) for nb <= 8 activation rows b, with an optional RMSNorm of x
 * fused in front (qmv.with_norm, qmv.py:176-183) and one epilogue: */
#define AGXC_EPI_F32 0        /* y fp32 [nb][n]                                                  (qmv2 plain)    */
#define AGXC_EPI_RES1 1       /* h fp32 = y + x16 residual                              (with_residual add16)    */
#define AGXC_EPI_RES2 2       /* x16 fp16 = fp16(y + h)                            (with_residual add32_to16)    */
#define AGXC_EPI_SWIGLU 3     /* act fp16 [nb][n/2] = fp16(silu(gate) * up); pack made with agxc_pack_create_gateup */

typedef struct {
  const agxc_pack* pack;
  int32_t nb;                 /* activation rows, 1..8 */
  const void* x_dev;          /* [nb][x_ld], fp16 (x_f32 = 0) or fp32 (x_f32 = 1) */
  int32_t x_f32, x_ld;
  const uint16_t* norm_gain_dev; /* fp16 [k]; non-NULL = RMSNorm x first: fp16(x * rsqrt(mean(x^2) + eps) * g) */
  float eps;
  int32_t epi;
  void* out_dev;              /* fp32 [nb][out_ld] (F32, RES1) or fp16 [nb][out_ld] (RES2, SWIGLU) */
  int32_t out_ld;
  const void* res_dev;        /* RES1: fp16 [nb][res_ld]; RES2: fp32 [nb][res_ld] */
  int32_t res_ld;
  int32_t splits;             /* K splits across CTAs; 0 = planner's choice */
  int32_t row_tiles;          /* 16-row tiles per work unit (1, 2, 4, 8); 0 = planner's choice */
  int32_t chunk_groups;       /* 64-k groups per streamed chunk; 0 = planner's choice */
  int32_t stages;             /* shared-memory ring stages (2..8); 0 = planner's choice */
} agxc_qmv_args;

/* Gate and up projections [f][k] each, re-laid out as ONE interleaved pack of 2f rows for the fused SwiGLU
 * (replaces qmv_swiglu_layout, qmv.py:214-219). Arrays as in agxc_pack_create. */
AGXC_API int agxc_pack_create_gateup(agxc_ctx* ctx, const agxc_pack_desc* desc_each, const void* g_packed,
                            const void* g_scales, const void* g_biases, const void* u_packed, const void* u_scales,
                            const void* u_biases, int on_device, agxc_pack** out);

AGXC_API int agxc_qmv(agxc_ctx* ctx, const agxc_qmv_args* args, void* stream);

/* agxc_qmv for callers that may not allocate device memory (no counterpart in the reference, whose GEMV kernels
 * take no scratch). Same arguments, kernels, launch plan and results as agxc_qmv; the split-K scratch comes from a
 * static device block (1,048,576 fp32 partials, 8,192 row-block counters) instead of the stream-ordered allocator.
 * Rejects with AGXC_EINVAL, before launching, a plan whose splits x N x nb partials or N / 16 + 1 counters exceed
 * that block. Clears the counters it uses on `stream` before the launch (cudaMemsetAsync). The block is shared by
 * every call on a device: calls that may overlap there (other streams, threads, a graph replay) race and must be
 * ordered on one stream. The first call on a device looks up the block's address; make it outside stream capture. */
AGXC_API int agxc_qmv_noalloc(agxc_ctx* ctx, const agxc_qmv_args* args, void* stream);

/* The batched GEMM for 32..256 activation rows (a multiple of 16) on the tensor cores (the reference's tensor-unit
 * path, tools/g17qsm.py:1-21, assemble.layer_ops_qsm agxforge/inference/assemble.py:368-426; the weights are
 * dequantised once to fp16 as there): y fp32 [batch][ldy] = x fp16 [batch][k] W^T for a plain pack (n a multiple of
 * 128). `ksplit` splits K over CTAs (0 = until the 128-row tiles fill the SMs; with a split the call zeroes y first
 * and the CTAs add into it). */
AGXC_API int agxc_qmm(agxc_ctx* ctx, const agxc_pack* pack, const void* x_dev, int batch, float* y_dev, int ldy,
                      int ksplit, void* stream);

/* Standalone RMSNorm rows (norm.build_rmsnorm_wide, agxforge/kernels/norm.py:42-155): out fp16 [nb][d]. */
AGXC_API int agxc_rmsnorm_dev(agxc_ctx* ctx, const void* x_dev, int x_f32, int nb, int d, const uint16_t* gain_dev,
                     float eps, uint16_t* out_dev, void* stream);

/* ---- decode attention (agxforge/kernels/attention.py: split 86-165, merge 1326-1371; attn_reference 1458) -----
 * One query row per head at position q0[b] (keys 0..q0, q0 clamped to cap-1); q16 fp16 [nb][heads][head_dim]
 * already scaled by log2(e)/sqrt(head_dim) (the softmax is base 2); caches fp16 [nb][kv_heads][cap][head_dim];
 * out fp16 [nb][heads*head_dim]. Split-KV over `splits` key chunks (a power of two up to 16, one thread-block
 * cluster per KV head; 0 = planner) with a log-sum-exp merge in distributed shared memory. */
AGXC_API int agxc_attention_dev(agxc_ctx* ctx, int nb, int heads, int kv_heads, int head_dim, int cap, const uint32_t* q0_dev,
                       const uint16_t* q16_dev, const uint16_t* k_dev, const uint16_t* v_dev, uint16_t* out_dev,
                       int splits, void* stream);

/* RoPE + q scale + KV append on one token's fp32 qkv row in the reference's logical order [heads | kv_heads |
 * kv_heads] x head_dim (attention.py:1309-1323 attn_rope_reference; numerics.py:340-346 rope_rotate): q16 fp16
 * [heads][head_dim] = fp16(rope(q) * qscale); K and V rows fp16 written at row `pos` (clamped to cap-1) of the caches
 * [kv_heads][cap][head_dim]. cos/sin fp32 [head_dim/2] for that position. Each rotated value is two rounded products
 * and one rounded sum, as rope_rotate. (In the decode step this is the qkv GEMV's epilogue.) */
AGXC_API int agxc_rope_append_dev(agxc_ctx* ctx, const float* qkv_dev, int heads, int kv_heads, int head_dim, int cap,
                                  int pos, const float* cos_dev, const float* sin_dev, float qscale,
                                  uint16_t* q16_dev, uint16_t* kcache_dev, uint16_t* vcache_dev, void* stream);

/* The tensor-parallel all-reduce's local reduction (one-shot): waits (bounded by wait_us of the global timer) until
 * *flag_dev reaches the arrivals of this use (every rank's o_proj or down tiles pushed into recv [ranks][batch][d]),
 * then writes this rank's residual stream: out32 = sum over ranks + res16 (o_proj, add16) or out16 = fp16(sum +
 * res32) (down, add32_to16). A wait that gives up sets the error word's timeout bit and writes nothing; the context
 * stays usable. (In the decode step this runs inside the step's graph; this entry point exposes it to tests.) */
AGXC_API int agxc_tp_reduce_dev(agxc_ctx* ctx, const float* recv_dev, int ranks, int rank, const unsigned* flag_dev,
                                const unsigned* epoch_dev, int uses_per_step, int use_in_step, int tiles_per_rank,
                                const uint16_t* res16_dev, const float* res32_dev, float* out32_dev,
                                uint16_t* out16_dev, int d, int batch, int wait_us, void* stream);

/* The first maximum of an fp32 row of n values (argmax.py:287-288 argmax_reference; NaN-free input): *out_dev =
 * the smallest index holding the largest value. (In the decode step this is the vocabulary GEMV's epilogue.) */
AGXC_API int agxc_argmax_dev(agxc_ctx* ctx, const float* x_dev, int n, int32_t* out_dev, void* stream);

/* ---- the model (agxforge/inference/assemble.py configure 71-92, build 596-828; models.py 26-54) -------------- */
typedef struct {
  int32_t d_model, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab;
  int32_t bits, group, scale_dtype;
  int32_t cap;                /* KV capacity and token-log length per sequence */
  int32_t batch;              /* independent sequences decoded together: 1..8 (GEMV step) or 32..256 in steps of 16
                                 (tensor-core GEMM step; d_model, qkv rows and vocab multiples of 128) */
  int32_t qkv_bias;           /* 1 = the qkv projection has a bias (Qwen2) */
  float eps, rope_theta;
  int32_t keep_logits;        /* 1 = keep the head's fp32 logits [batch][vocab] readable after each step */
  /* Tensor parallelism (no counterpart in the reference, which runs one device): tp_world ranks, one process per
   * GPU, each holding n_heads/tp_world query heads and n_kv_heads/tp_world KV heads (qkv rows of those heads, their
   * KV cache), ffn/tp_world gate/up rows and down columns, the o_proj columns of its heads, and a vocabulary slice of
   * the head in 128-row tiles (agxc_model_vocab_slice). The shapes above stay GLOBAL; set_pack takes the rank's
   * slice of each reference-format pack. The o_proj and down partial sums are all-reduced (fp32 sum) before their
   * residual, and the head's per-rank first maxima are all-gathered before the token choice, so every rank holds the
   * same residual stream, token log and q0. Needs batch >= 32, heads, KV heads divisible by tp_world and ffn by
   * 64 * tp_world. tp_world 0 or 1 = one device. tp_id = the communicator id from agxc_tp_unique_id on rank 0, the
   * same bytes on every rank. Creation is collective: every rank calls agxc_model_create. */
  int32_t tp_world, tp_rank;
  uint8_t tp_id[128];
} agxc_model_desc;

/* A fresh communicator id (128 bytes) for a tensor-parallel model (rank 0 makes it, the caller sends it to the other
 * ranks). The collective library (NCCL, libnccl.so.2) is loaded on first use; AGXC_EUNSUPPORTED without it. */
AGXC_API int agxc_tp_unique_id(void* id128);
/* The rank's vocabulary slice of the head: global token ids [offset, offset + count). */
AGXC_API int agxc_model_vocab_slice(const agxc_model* m, int32_t* offset, int32_t* count);

#define AGXC_ROLE_QKV 0
#define AGXC_ROLE_WO 1
#define AGXC_ROLE_GATE 2
#define AGXC_ROLE_UP 3
#define AGXC_ROLE_DOWN 4
#define AGXC_ROLE_HEAD 5      /* layer ignored */
#define AGXC_VEC_ATTN_GAIN 0  /* fp16 [d] */
#define AGXC_VEC_FFN_GAIN 1   /* fp16 [d] */
#define AGXC_VEC_QKV_BIAS 2   /* fp16 [qkv rows] */
#define AGXC_VEC_FINAL_GAIN 3 /* fp16 [d], layer ignored */
#define AGXC_VEC_EMBED 4      /* fp16 [vocab][d], layer ignored */
#define AGXC_VEC_Q_NORM 5     /* fp16 [head_dim]: the layer's QK-norm gain of q heads (AGXC_OPT_QK_NORM) */
#define AGXC_VEC_K_NORM 6     /* fp16 [head_dim]: the layer's QK-norm gain of k heads */

AGXC_API int agxc_model_create(agxc_ctx* ctx, const agxc_model_desc* desc, agxc_model** out);
AGXC_API void agxc_model_free(agxc_model* m);
/* Set one projection from a reference-format pack (host or device arrays); gate and up are interleaved internally. */
AGXC_API int agxc_model_set_pack(agxc_model* m, int layer, int role, const void* packed, const void* scales,
                        const void* biases, int on_device);
/* Set one fp16 vector (gains, bias, embedding table). */
AGXC_API int agxc_model_set_vector(agxc_model* m, int layer, int which, const void* data, size_t bytes, int on_device);
/* Algorithmic bytes of the model's packs (fields + 16-bit scale and bias), for roofline accounting. */
AGXC_API int64_t agxc_model_weight_bytes(const agxc_model* m);

/* Start sequence b: clears its KV cache and log, writes its prompt (n tokens, n >= 1) into the token log, puts the
 * embedding of prompt[0] in x and sets q0 = 0 (assemble.py:650-669's R_init). Later decode steps take the logged
 * tokens (teacher forcing, tools/g17forcehistory.py) until the log runs out, then choose by argmax. */
AGXC_API int agxc_model_start(agxc_model* m, int b, const int32_t* prompt, int n);
/* Overwrite log entries [pos, pos+n) of sequence b from the host (forcing), without touching q0. */
AGXC_API int agxc_model_force(agxc_model* m, int b, int pos, const int32_t* tokens, int n);
/* Fill positions [0, n) of every layer's KV cache of sequence b with seeded N(0,1) fp16 values and set q0 = n
 * (a stand-in history for throughput runs whose histories are too long to decode through). */
AGXC_API int agxc_model_fill_history(agxc_model* m, int b, int n, uint64_t seed);

/* Run `steps` decode steps (one token per sequence per step, the whole step one CUDA graph replay; the reference's
 * pipelined executor loop, tools/g17decodegen.m:264-290). Each step's token per sequence is: the step's entry of
 * `forced_in` (host, [steps][batch], AGXC_TOKEN_UNSET = none; copied host -> device before the step) if given and
 * set, else the token log's entry at q0 + 1 (the prompt), else the first argmax of the logits. After each step the
 * chosen tokens are device-resident; when `tokens_out` (host, [steps][batch]) is non-NULL each step's tokens are
 * copied back, and when `logits_out` (host, [steps][batch][vocab], needs keep_logits) is non-NULL, the logits too
 * (under tensor parallelism [steps][batch][count]: the rank's vocabulary slice).
 * `sync_each` = 1 waits for every step (the host sees each token before the next launch); 2 keeps one step queued
 * ahead: after queueing step i it waits for step i - 1, whose tokens are then on the host (a streaming server's
 * loop: each token reaches the host one step after it is chosen, and the device never idles between steps). */
typedef struct {
  float gpu_ms;               /* device time of the steps (CUDA events) */
  float host_ms;              /* host wall time of the call */
  int32_t launches_per_step;  /* kernels in one step's graph */
} agxc_timing;
/* Start sequence b with its prompt (as agxc_model_start) and run positions 0 .. n-2 as the PREFILL section
 * (agxforge/inference/prefill.py:1-30: the prompt as M-row passes): chunks of up to 256 rows through every layer on the
 * tensor-core GEMM (agxc_qmm) with a causal attention over the chunk, writing b's KV cache rows 0 .. n-2. Leaves
 * q0 = n-1 and x = embedding(prompt[n-1]), so the next agxc_decode step runs position n-1 and chooses the first
 * generated token: the state n-1 teacher-forced decode steps would leave (within rounding). Needs qkv rows, d_model
 * and 2 x ffn multiples of 128 and one device; `t` (nullable) gets the device time. */
AGXC_API int agxc_model_prefill(agxc_model* m, int b, const int32_t* prompt, int n, agxc_timing* t);

/* The speculative verify step (the reference's verify section, agxforge/inference/assemble.py:244-253,747-803 and its
 * driver tools/g17specgen.m): sequence b's current token and n_draft (0..15) drafted tokens run as rows at positions
 * q0 .. q0 + n_draft through the tensor-core GEMMs (their K/V rows written into the cache), then the final norm, the
 * head and each row's first maximum. Row i chooses the token at position q0 + i + 1 (a logged token where the log
 * fixes it, else the maximum); drafts are accepted while they equal the choices. The accepted drafts and the choice
 * after them (1 .. n_draft + 1 tokens) go to emitted[] / *n_emitted and are committed: logged, q0 advanced past them,
 * the next input row = the last one's embedding. logits_out (nullable): [n_draft + 1][vocab] fp32 of the rows.
 * Single device; needs qkv rows, d_model, 2 x ffn and vocab multiples of 128. */
AGXC_API int agxc_model_verify(agxc_model* m, int b, const int32_t* draft, int n_draft, int32_t* emitted,
                               int32_t* n_emitted, float* logits_out);
AGXC_API int agxc_decode(agxc_model* m, int steps, const int32_t* forced_in, int32_t* tokens_out, float* logits_out,
                int sync_each, agxc_timing* t);

/* Copy the state of sequence b to the host: q0 and the token log (cap entries). */
AGXC_API int agxc_model_state(agxc_model* m, int b, uint32_t* q0, uint32_t* log);

/* Decode-state save and restore of sequence b (the reference keeps a decode's state in its region R and token log and
 * forces a shared history by rewriting that log, tools/g17forcehistory.py:32-80; here the whole state moves): everything
 * the next step reads — q0, the token log, a pending forced token, the next input row x16 [d_model] fp16, and every
 * layer's K and V rows 0 .. q0-1 (fp16) — as one host byte image: a 64-byte header ("AGXS", version 1, the shapes)
 * then those arrays. agxc_model_state_bytes gives the image's size now. A restore checks the header against the model
 * (layers, KV heads, head_dim, d_model, vocab; the cap must hold q0 + 1 positions) and refuses a mismatch with
 * AGXC_EINVAL; it replaces the sequence's state, so the next decode continues exactly where the saved one would
 * have. Single device only (AGXC_EUNSUPPORTED under tensor parallelism). */
AGXC_API int64_t agxc_model_state_bytes(agxc_model* m, int b);
AGXC_API int agxc_model_state_save(agxc_model* m, int b, void* out, size_t capacity, size_t* written);
AGXC_API int agxc_model_state_restore(agxc_model* m, int b, const void* in, size_t bytes);
/* Read back layer `layer`'s K and V cache rows [0, n) of sequence b (fp16 patterns, [kv_heads][n][head_dim] each). */
AGXC_API int agxc_model_read_kv(agxc_model* m, int layer, int b, int n, uint16_t* k_out, uint16_t* v_out);
/* Device pointer of the last step's logits [batch][vocab] fp32 (keep_logits) for in-place checks. */
AGXC_API int agxc_model_logits_dev(agxc_model* m, const float** out);

/* Run `steps` decode steps with every kernel launched on its own between two CUDA events (no graph, no overlap)
 * and return, per kernel kind, the summed device time (ms) and the number of launches. Kinds: */
#define AGXC_KIND_QKV 0
#define AGXC_KIND_ATTN 1
#define AGXC_KIND_WO 2
#define AGXC_KIND_FFN 3
#define AGXC_KIND_DOWN 4
#define AGXC_KIND_HEAD 5
AGXC_API int agxc_model_profile(agxc_model* m, int steps, float* kind_ms /*[6]*/, int32_t* kind_launches /*[6]*/);

/* Model options (each re-captures the step's graph on the next decode). */
#define AGXC_OPT_PDL 0        /* programmatic dependent launch between the step's kernels, so each streams its weights
                                 while its predecessor finishes: 1 (default) a kernel lets its successor start right
                                 after its own dependency wait; 2 only after it staged its inputs (GEMV) or read its
                                 keys (attention); 3 only after its last weight chunk (GEMV) or its keys (attention);
                                 0 plain stream order */
#define AGXC_OPT_TRACE 1      /* 1: every launch of the step records, over its CTAs, the first and last %globaltimer
                                 (ns) at CTA entry, after the dependency wait, and at CTA exit (read with
                                 agxc_model_trace_read); 0 (default): off */
#define AGXC_OPT_FUSED 2      /* 1 (where it fits): a batch-1 model on one device runs each step as ONE persistent
                                 cooperative kernel: one CTA per SM, a producer warp streams every weight chunk and KV
                                 row the CTA reads through a shared-memory ring while the layer's four phases (qkv;
                                 attention; merge + o_proj; gate/up + down) wait only on the counters of the data they
                                 read. 0 (default): one kernel per projection and attention, chained by programmatic
                                 dependent launch (always the case for batch > 1) */
#define AGXC_OPT_BULK 3       /* 1: the per-projection GEMVs move weight chunks by plain bulk copies (one per row tile of
                                 a chunk); 0 (default): by 3-D TMA tensor boxes */
#define AGXC_OPT_TP_FUSED 5    /* tensor parallel: 1 (default when every rank could map the others' buffers) = the
                                 o_proj and down GEMMs carry the all-reduce over NVLink peer memory: with 2 or 4 ranks
                                 each finished tile goes to every rank and a bounded-wait kernel sums the ranks' slots
                                 fused with the residual (one-shot); with 8, each tile goes to the rank owning its
                                 rows and a cooperative kernel reduces them and stores them into every rank's residual
                                 stream (two-shot). 2 / 3 force two-shot / one-shot (before the first fused
                                 step only); 0 = NCCL all-reduce. Every rank must set the same value. */
#define AGXC_OPT_QK_NORM 6     /* 1: QK-norm (Qwen3; attention.py:256-265 with_qknorm): every q and k head of the qkv
                                 projection is RMS-normed over head_dim with the layer's AGXC_VEC_Q_NORM / _K_NORM gain
                                 (fp32, (x r) g, the model's eps) before RoPE, on every path; 0 (default): off */
#define AGXC_OPT_DEVICE_WAIT_US 7 /* the bound (us of the global timer) on every wait of the fused step and of the
                                 tensor-parallel reduce (default 2,000,000): a wait past it sets the error word, the
                                 launch leaves, and the decode call returns AGXC_ETIMEOUT with the step undone */
#define AGXC_OPT_WAIT_MS 4     /* tensor parallel: host bound (ms, default 60000) on a decode call's completion; past it
                                 the communicator is aborted (its kernels end) and the call returns AGXC_ETIMEOUT, so a
                                 rank that died between steps cannot hold the others' GPUs */
AGXC_API int agxc_model_set_option(agxc_model* m, int option, int value);

/* The launch trace accumulated since tracing started or the last read (min and max over all steps in between), then
 * reset: out[launch][12] = {first, last} CTA times in ns of the device's global timer at entry, after the dependency
 * wait, at exit, and (GEMV launches; all-ones and 0 elsewhere) after staging the activation rows, after the last
 * unit's epilogue, and when the first weight chunk had landed. Launches in step order (per layer qkv, attn, wo, ffn,
 * down; then head); *n = launches. */
AGXC_API int agxc_model_trace_read(agxc_model* m, uint64_t* out, int capacity, int32_t* n);
/* The fused step's per-CTA trace of the last traced step: out[mark][CTA] global-timer stamps (ns); per layer eight
 * marks (qkv: dependency met, done; attention: dependency met, done; o_proj: dependency met, done; FFN: dependency
 * met, done), then the head's two (dependency met, done); 0 = not reached (a CTA with no work in that phase).
 * *phases = marks, *ctas = CTAs; at most `capacity` words are written. */
AGXC_API int agxc_model_trace_cta_read(agxc_model* m, uint64_t* out, size_t capacity, int32_t* phases, int32_t* ctas);

/* The model's launch plans as a JSON object (per kernel: row tiles per unit, K splits, groups per unit and chunk,
 * stages, grid, shared memory; attention: key chunks per KV head). Writes at most `len` bytes including the NUL. */
AGXC_API int agxc_model_plan_info(agxc_model* m, char* buf, size_t len);

/* Kernels per decode step and their names (for launch accounting). */
AGXC_API int agxc_model_kernel_count(agxc_model* m, int32_t* n);

/* ---- the BERT sentence encoder (MiniLM; tools/g17inferencereference.py:18-99 graph_reference over the graph of
 * agxforge/g17/inferencegraph.py:208-289 import_graph with sentence pooling; lowered stages
 * tools/g17inferencelower.py:56-139) ---------------------------------------------------------------------------
 * Embedding gather + LayerNorm, per layer q/k/v/o and FFN linears with bias on the tensor cores (fp16 operands,
 * fp32 accumulation), GELU (erf), padding-masked softmax attention, post-attention and post-FFN LayerNorms, then the
 * masked mean over each sequence's valid rows and L2 normalisation. Batches of sequences [batch][seq] with 0/1
 * masks (the reference takes one sequence of exactly 32 tokens). Parameters are fp16, in the checkpoint's layout
 * (linear weights [out][in]). */
typedef struct agxc_encoder agxc_encoder;
typedef struct {
  int32_t hidden, layers, heads, ffn, vocab, max_position, type_vocab;
  float eps;                  /* LayerNorm epsilon (MiniLM: 1e-12) */
  int32_t max_batch, max_seq; /* activation buffers are sized for max_batch x max_seq tokens */
} agxc_encoder_desc;

#define AGXC_ENC_WORD 0       /* [vocab][hidden] */
#define AGXC_ENC_POSITION 1   /* [max_position][hidden] */
#define AGXC_ENC_TOKEN_TYPE 2 /* [type_vocab][hidden] */
#define AGXC_ENC_EMB_LN_W 3   /* [hidden] embeddings.LayerNorm */
#define AGXC_ENC_EMB_LN_B 4
#define AGXC_ENC_Q_W 5        /* per layer: attention.self.query.weight [hidden][hidden] */
#define AGXC_ENC_Q_B 6
#define AGXC_ENC_K_W 7
#define AGXC_ENC_K_B 8
#define AGXC_ENC_V_W 9
#define AGXC_ENC_V_B 10
#define AGXC_ENC_O_W 11       /* attention.output.dense */
#define AGXC_ENC_O_B 12
#define AGXC_ENC_LN1_W 13     /* attention.output.LayerNorm */
#define AGXC_ENC_LN1_B 14
#define AGXC_ENC_FFN1_W 15    /* intermediate.dense [ffn][hidden] */
#define AGXC_ENC_FFN1_B 16
#define AGXC_ENC_FFN2_W 17    /* output.dense [hidden][ffn] */
#define AGXC_ENC_FFN2_B 18
#define AGXC_ENC_LN2_W 19     /* output.LayerNorm */
#define AGXC_ENC_LN2_B 20

/* The encoder's tensor-core GEMM alone (tests): C [M][N] = A [M][K] fp16 x W [N][K]^T fp16 + bias (fp16 [N],
 * nullable), epi 0: out32 fp32; 1: out16 = fp16(gelu_erf(.)); 2: out32 = . + res32; 3: y = LayerNorm(. + res32)
 * with gain ln_g, bias ln_b (fp16 [N]) and eps over whole rows (N 128, 256 or 384), out32 = y (may alias
 * res32), out16 = fp16(y). M % 128, N % 64, K % 64 == 0. */
AGXC_API int agxc_hgemm_dev(agxc_ctx* ctx, const uint16_t* A, const uint16_t* W, int M, int N, int K,
                            const uint16_t* bias, int epi, float* out32, uint16_t* out16, const float* res32,
                            const uint16_t* ln_g, const uint16_t* ln_b, float eps, void* stream);
AGXC_API int agxc_encoder_create(agxc_ctx* ctx, const agxc_encoder_desc* desc, agxc_encoder** out);
AGXC_API void agxc_encoder_free(agxc_encoder* e);
/* One fp16 parameter (layer ignored for the embedding entries); `bytes` must be its exact size. */
AGXC_API int agxc_encoder_set_param(agxc_encoder* e, int layer, int which, const void* data, size_t bytes,
                                    int on_device);
/* Sentence embeddings out [batch][hidden] fp32 of token_ids [batch][seq] (int32), attention_mask [batch][seq] (0/1,
 * at least one 1 per sequence), token_type_ids (NULL = all 0); positions 0..seq-1. on_device = 1: every pointer is
 * device memory and the call only enqueues on the context's stream; 0: host arrays, copied in and out (the call
 * returns when `out` holds the result). Rejects (AGXC_EINVAL) ids, types or masks outside their domain, as the
 * reference refuses them. `t` (nullable) gets the device time of the encoder's kernels. */
AGXC_API int agxc_encoder_forward(agxc_encoder* e, const int32_t* token_ids, const int32_t* attention_mask,
                                  const int32_t* token_type_ids, int batch, int seq, float* out, int on_device,
                                  agxc_timing* t);
/* `reps` forwards on the inputs of the last agxc_encoder_forward call (already on the device), one CUDA graph replay
 * each; t->gpu_ms = their device time (CUDA events on the context's stream). flush_l2 = 1: a 256 MB buffer (twice
 * the L2) is written between forwards and only the forwards are timed, so none starts with the weights in L2. */
AGXC_API int agxc_encoder_replay(agxc_encoder* e, int reps, int flush_l2, agxc_timing* t);
/* Per-stage device time of `reps` forwards (each stage timed on its own): ms[8] = embedding, qkv, attention, o_proj
 * + residual, LayerNorms, FFN up + GELU, FFN down + residual, pooling; launches[8] their launch counts. */
AGXC_API int agxc_encoder_profile(agxc_encoder* e, int batch, int seq, int reps, float* ms, int32_t* launches);

#ifdef __cplusplus
}
#endif
#endif /* AGXC_H */
