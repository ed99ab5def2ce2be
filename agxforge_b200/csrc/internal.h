// internal.h — the library's internal types: context, device pack, GEMV and attention launch descriptions.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/agxc.h"

struct agxc_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  unsigned* err_dev = nullptr;   // the device error word
  int num_sms = 148;
  int max_smem_optin = 0;
  int max_cluster = 8;           // the largest attention cluster the device places
  int cluster_active[5] = {0, 0, 0, 0, 0};  // attention clusters of 1, 2, 4, 8, 16 CTAs resident at once
};

// A pack in the B200 tile layout: tiles[rt][g] of 16 rows x 64 k (512 B at 4 bits, 1,024 B at 8 bits; lane l of a
// warp owns 16 B at 16 l, two 512-B halves at 8 bits) and, per tile, 64 B of scale/bias: entry r (8 B) =
// {s[r], s[r+8], b[r], b[r+8]} as 16-bit patterns.
struct agxc_pack {
  agxc_ctx* ctx = nullptr;
  int n = 0, k = 0, bits = 4, group = 64, sdt = 0;
  int gateup = 0;                 // rows interleaved gate/up per 16-row tile (fused SwiGLU)
  uint8_t* tiles = nullptr;
  uint8_t* sb = nullptr;
  bool owns = true;
  int64_t bytes() const { return int64_t(n) * k * bits / 8 + int64_t(n) * (k / group) * 4; }
};

namespace agxc {

constexpr int kTileRows = 16;
constexpr int kGroup = 64;
constexpr int kSbBytes = 64;
inline int tile_bytes(int bits) { return bits == 4 ? 512 : 1024; }

enum Epi : int { EPI_F32 = 0, EPI_RES1 = 1, EPI_RES2 = 2, EPI_SWIGLU = 3, EPI_QKV = 4, EPI_ARGMAX = 5 };

// Everything one GEMV launch reads and writes (the kernel takes what its epilogue needs).
struct QmvParams {
  const uint8_t* w = nullptr;
  const uint8_t* sb = nullptr;
  int N = 0, K = 0, G = 0;        // rows, columns, groups (K/64)
  int SC = 1, GC = 0, CG = 0;     // K splits, groups per unit (K range of a CTA), groups per streamed chunk
  int bits = 4, sdt = 0, nb = 1;
  int stages = 2;
  // x
  const void* x = nullptr;
  int x_f32 = 0, x_ld = 0;
  const __half* norm_gain = nullptr;
  float eps = 1e-6f;
  // outputs
  float* out_f32 = nullptr;
  int out_ld = 0;
  __half* out_f16 = nullptr;
  const __half* res16 = nullptr;
  const float* res32 = nullptr;
  int res_ld = 0;
  // qkv epilogue: bias, RoPE, q scale, KV append
  const __half* bias = nullptr;
  int H = 0, KVH = 0, hd = 0, cap = 0;
  const float* cos_t = nullptr;
  const float* sin_t = nullptr;
  const uint32_t* q0 = nullptr;
  float qscale = 0.f;
  __half* q16 = nullptr;
  __half* kcache = nullptr;      // this layer: [nb][KVH][cap][hd]
  __half* vcache = nullptr;
  // argmax + generation step
  int V = 0;
  const __half* embed = nullptr; // [V][d]
  __half* x_next = nullptr;      // [nb][d]
  int d = 0;
  uint32_t* q0_rw = nullptr;
  uint32_t* log = nullptr;       // [nb][cap]
  int32_t* tok_out = nullptr;    // [nb]
  uint32_t* force_next = nullptr; // [nb] pending forced tokens (consumed and cleared by the step)
  int pos_ready = 0;              // qkv: q0 was final before the upstream kernel started (RoPE read before the wait)
  int bulk = 0;                   // weights by plain bulk copies (1) or 3-D TMA tensor boxes (0)
  // scratch
  float* part = nullptr;         // [SC][N][nb] partial rows
  float* pairs = nullptr;        // [grid][nb][2] argmax pairs (value, index as float bits)
  unsigned* counters = nullptr;
  unsigned* err = nullptr;
  int pdl = 0;
  unsigned long long* trace = nullptr;  // this launch's six trace words, or NULL
};

struct QmvPlan {
  int SC = 1, GC = 0, CG = 0, RW = 1, EB = 1, stages = 2, grid = 0;
  size_t smem = 0;
};

// force_*: 0 = the planner's choice (tuning and tests override them)
QmvPlan plan_qmv(const agxc_ctx* ctx, int N, int K, int bits, int nb, int epi, int hd, int splits, int force_rw = 0,
                 int force_cg = 0, int force_stages = 0);
// Scratch sizes a plan needs.
size_t qmv_part_floats(const QmvPlan& p, int N, int nb, int epi);
// tw/ts: the plan's tensor maps of the pack (weights, scale/bias); NULL = encode them for this launch.
int launch_qmv_epi(const agxc_ctx* ctx, QmvParams p, const QmvPlan& plan, int epi, cudaStream_t s,
                   const CUtensorMap* tw = nullptr, const CUtensorMap* ts = nullptr);
int qmv_maps(const QmvPlan& plan, const uint8_t* w, const uint8_t* sb, int N, int K, int bits, CUtensorMap* tw,
             CUtensorMap* ts);
int qmv_configure(const agxc_ctx* ctx);

struct AttnParams {
  int nb = 1, H = 0, KVH = 0, hd = 128, cap = 0, S = 1;
  const uint32_t* q0 = nullptr;
  const __half* q16 = nullptr;
  const __half* kc = nullptr;
  const __half* vc = nullptr;
  __half* out = nullptr;
  float* part = nullptr;          // unused (the chunks merge in distributed shared memory)
  unsigned* counters = nullptr;   // unused
  unsigned* err = nullptr;
  int pdl = 0;
  unsigned long long* trace = nullptr;  // this launch's six trace words, or NULL
};
int attn_splits(const agxc_ctx* ctx, int nb, int KVH, int cap);

// ---- the fused step (fstep.cu): a batch-1 decode step as one persistent cooperative kernel, four phases a layer
// with fine-grained counters between them
struct FstepArgs {
  int L = 0, d = 0, H = 0, KVH = 0, hd = 0, F = 0, V = 0, cap = 0, bits = 4, sdt = 0, stages = 0, smax = 1, grid = 0;
  float eps = 1e-6f;
  uint64_t wait_ns = 2000000000ull;   // the bound on every wait of the step (global timer)
  const CUtensorMap* maps = nullptr;  // device: fstep_map_count() maps (per role over all layers, head, K, V)
  const __half* gains = nullptr;
  const __half* bias = nullptr;
  const __half* qkg = nullptr;        // [L][2][hd] QK-norm gains, or NULL (no QK-norm)
  float* qkraw = nullptr;             // [(H + KVH) hd] QK-norm scratch
  const __half* final_gain = nullptr;
  const __half* embed = nullptr;
  __half* kc = nullptr;
  __half* vc = nullptr;
  const float* cos_t = nullptr;
  const float* sin_t = nullptr;
  uint32_t* q0 = nullptr;
  uint32_t* log = nullptr;
  int32_t* tok_out = nullptr;
  uint32_t* force_next = nullptr;
  __half* x16 = nullptr;
  float* logits = nullptr;
  __half* q16 = nullptr;
  float* apart = nullptr;
  float* acc = nullptr;
  unsigned* sync = nullptr;
  int nctr = 0;
  float* pairs = nullptr;
  unsigned* err = nullptr;
  unsigned long long* trace = nullptr;
};
int fstep_configure(const agxc_ctx* ctx);
int fstep_stages(const agxc_ctx* ctx, int d, int G, int hd);
size_t fstep_smem(int d, int G, int hd, int stages);
int fstep_launch(const FstepArgs& a, cudaStream_t s);
int fstep_counters(int L, int KVH);
int fstep_trace_marks(int L);
int fstep_map_count();
int fstep_max_d();                   // the largest d_model the fused step stages
int fstep_tiles_per_stage(int bits);
// A 3-D TMA map over a pack's tiles [RT row tiles][G groups][inner 32-bit words] with a box of (inner, CG, RW).
int encode_pack_map(CUtensorMap* m, const void* base, int inner_words, int G, int RT, int CG, int RW);
// A TMA map over fp16 KV rows [Z][cap][hd] with boxes of 64 dims x box_keys keys x 1, 128-byte swizzle.
int encode_pack_map_layers(CUtensorMap* m, const void* base, int inner_words, int G, int RT, int L,
                           uint64_t layer_stride, int CG, int RW);
int encode_kv_map_box(CUtensorMap* m, const void* base, int hd, int cap, int64_t Z, int box_keys);
// fp16 rows [rows][K] (K % 64 == 0) as boxes of 64 columns x box_rows rows, 128-byte swizzle (the UMMA K-major tile)
int encode_rows_map(CUtensorMap* m, const void* x, int rows, int K, int box_rows);
// A TMA map over fp16 activation rows X [B][K]: boxes of 64 columns x B rows, 128-byte swizzle.
int encode_act_map(CUtensorMap* m, const void* x, int B, int K);

// A GEMM's output rows as its consumers read them: value(b, n) = sum over q < ks of y[q slice + b ld + n] (the K
// ranges' partial sums in a fixed order; ks = 1: the finished rows).
struct YRows {
  const float* y = nullptr;
  int ld = 0;
  int ks = 1;
  size_t slice = 0;
};

// ---- the per-row steps of the batched decode step (batched.cu)
// q0: each row's position; seq < 0: row b is sequence b's (batched decode), else every row is sequence seq's (prefill)
// per row: the first maximum of V columns (and the row to `logits` when given)
int launch_rows_argmax(const YRows& y, int V, int rows, float* logits, int32_t* amax, cudaStream_t s);
// qkg: the layer's QK-norm gains [q hd | k hd] (NULL = no QK-norm), normed with qk_eps before the rotation
int launch_rope_append(const YRows& y, int rows, const __half* bias, const float* cos_t, const float* sin_t,
                       const uint32_t* q0, int H, int KVH, int hd, int cap, float qscale, __half* q16, __half* kc,
                       __half* vc, int B, cudaStream_t s, int seq = -1, const __half* qkg = nullptr,
                       float qk_eps = 1e-6f, int pdl = 0);
// causal attention of M prompt rows at positions p0 .. p0 + M - 1 of cache sequence `seq` (prefill.cu)
int launch_prefill_attention(const __half* q16, const __half* kc, const __half* vc, int M, int p0, int H, int KVH,
                             int hd, int cap, int seq, __half* out, cudaStream_t s);
int prefill_configure(const agxc_ctx* ctx);
int launch_residual16(const YRows& y, const __half* x16, float* h, int d, int B, cudaStream_t s, int pdl = 0);
int launch_residual32(const YRows& y, const float* h, __half* x16, int d, int B, cudaStream_t s, int pdl = 0);
int launch_swiglu(const YRows& y, __half* act, int F, int B, cudaStream_t s, int pdl = 0);
int launch_argmax_gen(const float* logits, int V, const __half* embed, int d, uint32_t* q0, uint32_t* log, int cap,
                      int32_t* tok, uint32_t* force_next, __half* x16, unsigned* err, int B, cudaStream_t s, int pdl = 0);

int launch_argmax_part(const float* logits, int V, int v0, uint32_t* pairs, int B, cudaStream_t s);
int launch_gen_from_pairs(const uint32_t* pairs, int ranks, int V, const __half* embed, int d, uint32_t* q0,
                          uint32_t* log, int cap, int32_t* tok, uint32_t* force_next, __half* x16, unsigned* err, int B,
                          cudaStream_t s, unsigned* epoch = nullptr);

// ---- the encoder's tensor-core GEMM (encoder.cu): C [M][N] = A [M][K] W [N][K]^T (+ bias; epi 0 fp32, 1 fp16
// GELU, 2 fp32 + residual)
// epi 3: out32 (may alias res32), out16 = LayerNorm(. + bias + res32) over whole rows (N 128..512)
int launch_hgemm(const agxc_ctx* ctx, const __half* A, const __half* W, int M, int N, int K, const __half* bias,
                 int epi, float* out32, __half* out16, const float* res32, cudaStream_t s,
                 const __half* ln_g = nullptr, const __half* ln_b = nullptr, float eps = 0.f);
int encoder_configure(const agxc_ctx* ctx);

// ---- tensor parallelism (tp.cu): NCCL loaded at run time
struct TpComm;
int tp_unique_id(void* out128);
int tp_comm_create(int world, int rank, const void* id128, TpComm** out);
void tp_comm_free(TpComm* c);
int tp_allreduce_f32(TpComm* c, float* buf, size_t n, cudaStream_t s);
int tp_allgather_u32(TpComm* c, const uint32_t* send, uint32_t* recv, size_t n, cudaStream_t s);
// Wait for `done` at most timeout_ms; past it abort the communicator and return AGXC_ETIMEOUT.
int tp_wait(TpComm* c, cudaEvent_t done, int timeout_ms);

// ---- the batched GEMM (qmm.cu): Y [B][ldy] fp32 = X [B][K] fp16 W^T, B = 32..256 (multiple of 16), tcgen05 + TMEM
int qmm_configure(const agxc_ctx* ctx);
// The tensor-parallel push of finished output tiles (the GEMM + all-reduce fusion, reduce-scatter half): rank r owns
// output rows [r N / ranks, (r + 1) N / ranks); the last of a tile's K-split CTAs stores the tile's B x 128 block of Y
// into its owner's receive slot for this rank (peer memory over NVLink, plain stores), then adds 1 to the owner's
// arrival counter (system scope, release).
struct QmmPush {
  float* slot[8] = {};      // rank r's receive slot for this rank's partial sums, [B][N]
  unsigned* flag[8] = {};   // rank r's arrival counter of that slot buffer
  int ranks = 0;
  int tiles_per_rank = 0;   // 128-row tiles owned by each rank
  int to_owner = 0;         // 1: each tile to its owner only (two-shot); 0: every tile to every rank (one-shot)
};
// ksplit > 1: `part` [ksplit][B][N] fp32 scratch and `tile_ctr` [N / 128] zeroed counters (also needed by `push`);
// the last K-range CTA of each tile sums the ranges in order into y (deterministic, y need not be cleared). y NULL
// (ksplit > 1, no push): only the partial sums are written, for consumers that add them (YRows).
// pdl: the GEMM may start before its predecessor in the stream finishes (its weight copies start at once; X, the
// outputs and the counters wait for the predecessor)
int launch_qmm(const agxc_ctx* ctx, const agxc_pack* pk, const void* x, int B, float* y, int ldy, int ksplit,
               cudaStream_t s, const QmmPush* push = nullptr, float* part = nullptr, unsigned* tile_ctr = nullptr,
               int pdl = 0);
// After the GEMM's pushes (use = *epoch x uses_per_step + use_in_step; every wait bounded). One-shot: wait until every
// rank's tiles are here (*flag >= (use + 1) x ranks x ranks x tiles_per_rank), reduce every row in rank order plus the
// residual into this rank's own output. Two-shot (one cooperative grid): wait for this rank's rows only (*flag >=
// (use + 1) x ranks x tiles_per_rank), reduce them, store the result into every rank's output rows (peer stores),
// signal every rank's gather counter, then wait until every rank's rows have arrived here. res16 -> out32 (h fp32,
// o_proj) or res32 -> out16 (x16 fp16, down).
struct TpGather {
  float* out32[8] = {};
  __half* out16[8] = {};
  unsigned* gflag[8] = {};  // rank r's gather counter of this buffer
};
// wait_ns: the bound on each of its spins (the global timer; 2 s by default)
int launch_tp_reduce(const float* recv, int ranks, int rank, const unsigned* flag, const unsigned* epoch,
                     int uses_per_step, int use_in_step, int tiles_per_rank, const __half* res16, const float* res32,
                     const TpGather& gather, int d, int B, unsigned* err, cudaStream_t s, bool two_shot,
                     uint64_t wait_ns = 2000000000ull);
size_t attn_part_floats(int nb, int H, int S, int hd);
// (the KV maps are made here over kc/vc with Z = nb x KVH, boxes of the chosen variant's sub-chunk keys)
int launch_attention(const agxc_ctx* ctx, const AttnParams& p, cudaStream_t s);
int attn_configure(agxc_ctx* ctx);

int launch_rmsnorm(const void* x, int x_f32, int nb, int d, const __half* g, float eps, __half* out, cudaStream_t s, int pdl = 0);

// pack kernels
int launch_quantize(const float* w, int N, int K, int bits, int sdt, uint32_t* packed, uint16_t* s16, uint16_t* b16,
                    cudaStream_t s);
// Re-lay out rows [0, n_src) of a reference-format pack into tile rows; source row tile t lands at destination
// row tile t * rt_stride + rt_offset. rope_hd > 0 places the rows of each head of rope_hd rows so that tile t of the
// head holds logical rows 8t..8t+7 (tile rows 0-7) and rope_hd/2 + 8t.. (tile rows 8-15): RoPE pairs share a tile.
int launch_relayout(const uint32_t* packed, const uint16_t* s16, const uint16_t* b16, int n_src, int K, int bits,
                    uint8_t* tiles, uint8_t* sb, int rt_stride, int rt_offset, cudaStream_t s, int rope_hd = 0);
int launch_unpack(const agxc_pack* p, uint8_t* fields, cudaStream_t s);
int launch_dequant(const agxc_pack* p, float* w, cudaStream_t s);

}  // namespace agxc
