// model.cu — the decoder model on one B200: weights, KV cache, activations, the generation state and the decode
// step as one captured CUDA graph (the reference's layer builder and executor: agxforge/inference/assemble.py
// layer_ops 429-461 / all_ops 464-520 / build 596-828, and tools/g17decodegen.m encodeToken 167-199).
//
// One step (one token per sequence), five kernels a layer plus the head:
//   D1 qkv     RMSNorm(x16, g1) -> W_qkv -> (+bias) -> RoPE at q0 -> q16 (scaled), K/V cache row q0
//   D2 attn    split-KV attention over keys 0..q0 with the LSE merge -> attn16
//   D3 wo      W_o attn16 + x16 -> h (fp32)
//   D4 ffn     RMSNorm(h, g2) -> W_gate|W_up -> fp16(silu(g) u) -> act16
//   D5 down    W_down act16 + h -> x16
//   head       RMSNorm(x16, g_final) -> W_head -> first argmax -> generation step (token log, next x16, q0 + 1)
// (the final norm, a dispatch of its own in the reference, is fused as the head's prologue.)
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <random>
#include <vector>

#include "common.cuh"
#include "internal.h"

struct agxc_model {
  agxc_ctx* ctx = nullptr;
  agxc_model_desc d{};
  int qkv_rows = 0, attn_dim = 0;
  // weights
  uint8_t* wmem = nullptr;
  std::vector<agxc_pack> qkv, wo, gu, down;
  agxc_pack head;
  __half* gains = nullptr;      // [L][2][d]
  __half* bias = nullptr;       // [L][qkv_rows]
  __half* final_gain = nullptr; // [d]
  __half* qk_gains = nullptr;   // [L][2][hd] QK-norm gains (q, k), 1.0 until set
  int qk_norm = 0;              // AGXC_OPT_QK_NORM: q and k heads RMS-normed before RoPE (Qwen3)
  float* qkv_raw = nullptr;     // [B][qkv rows] the per-kernel path's qkv GEMV output under QK-norm
  __half* embed = nullptr;      // [V][d]
  // cache and activations
  __half* kcache = nullptr;     // [L][B][KVH][cap][hd]
  __half* vcache = nullptr;
  __half* x16 = nullptr;        // [B][d]
  float* h = nullptr;           // [B][d]
  __half* q16 = nullptr;        // [B][H][hd]
  __half* attn = nullptr;       // [B][H*hd]
  __half* act = nullptr;        // [B][F]
  float* logits = nullptr;      // [B][V] (keep_logits; always for batch >= 32)
  __half* xn16 = nullptr;       // batch >= 32: normed GEMM input [B][d]
  float* ybuf = nullptr;        // batch >= 32: GEMM output rows [B][max(qkv rows, 2F, d)]
  uint32_t* q0 = nullptr;       // [B]
  uint32_t* log = nullptr;      // [B][cap]
  int32_t* tok = nullptr;       // [B]
  uint32_t* force_next = nullptr; // [B] a token the next step must take (a per-step host input), UNSET = none
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  // scratch
  float* part = nullptr;
  float* apart = nullptr;
  float* pairs = nullptr;
  unsigned* counters = nullptr;
  size_t counters_n = 0;
  // plans
  agxc::QmvPlan p_qkv, p_wo, p_gu, p_down, p_head, p_qkv_raw;
  int attn_S = 1;
  int pdl = 1;
  int bulk = 0;                 // GEMV weights by plain bulk copies (AGXC_OPT_BULK)
  // the fused step (batch 1, fstep.cu): one persistent kernel a step, when the device and the shape allow it
  int fused = 0;                // AGXC_OPT_FUSED (opt-in: at the 1.8B shape the per-kernel graph measures faster)
  int fs_ok = 0;                // the shapes and the device fit it
  int fs_stages = 0;            // ring stages
  int fs_smax = 1;              // attention splits per KV group at most
  int fs_nctr = 0;              // counter words of one parity set
  CUtensorMap* fs_maps = nullptr;  // device: the step's TMA maps
  unsigned* fs_sync = nullptr;  // [64 + 2 nctr]: [0] the step counter, then both parities' counters
  float* fs_acc = nullptr;      // [2 parities][2][L][d] the o_proj and down accumulators
  float* fs_apart = nullptr;    // [KVH][smax][G][hd + 2] attention partials
  unsigned long long* trace = nullptr;  // [launches][12] when tracing (AGXC_OPT_TRACE)
  unsigned long long* cta_trace = nullptr;  // fused step, tracing: [mark][CTA]
  int trace_n = 0;
  // graph
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int launches = 0;
  // pinned staging
  int32_t* h_tok = nullptr;
  size_t h_tok_n = 0;
  uint32_t* h_force = nullptr;  // pinned [steps][B]
  size_t h_force_n = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  cudaEvent_t ev_pipe[2] = {nullptr, nullptr};  // sync_each 2: the last two steps' ends
  std::vector<void*> allocs;
  // tensor parallelism: m->d holds this rank's LOCAL shape (heads, KV heads, ffn, vocabulary slice)
  int tp = 1, tp_rank = 0;
  int vt = 0;                   // the global vocabulary (token ids, the embedding table)
  int v0 = 0;                   // the first global token id of this rank's vocabulary slice
  agxc::TpComm* comm = nullptr;
  uint32_t* amax = nullptr;     // [B][2] this rank's (value bits, global index) per sequence
  uint32_t* amax_all = nullptr; // [tp][B][2] every rank's, after the all-gather
  int wait_ms = 60000;
  uint64_t dev_wait_ns = 2000000000ull;  // AGXC_OPT_DEVICE_WAIT_US: the bound on the fused step's and the TP reduce's waits
  // the fused GEMM + all-reduce (peer memory): recv = [2 buffers (o_proj, down)][tp ranks][B][d] fp32 then 2 arrival
  // counters, one allocation exported to the other ranks by CUDA IPC; peer[r] = rank r's allocation, mapped here
  int tp_fused = 0;             // 1: o_proj and down push their tiles to every rank and reduce locally (no NCCL)
  int tp_fused_ok = 0;          // the peer mappings exist on every rank
  int tp_fused_ran = 0;         // a fused step has run (the variant is fixed from then on)
  int tp_two_shot = 0;          // 1 (8 ranks): reduce-scatter by the GEMM + all-gather; 0: every rank's tiles
                                // to every rank (2 ranks: one synchronisation instead of two)
  float* recv = nullptr;
  unsigned* recv_flags = nullptr;
  void* peer[8] = {};
  unsigned* tile_ctr = nullptr; // [widest pack's tiles] GEMM arrival counters (split K, the peer push)
  float* qpart = nullptr;       // batch >= 32: the split-K partial sums of the step's GEMMs
  size_t peer_flags_off = 0;    // byte offsets in every rank's exported allocation: counters (2 arrival, 2 gather),
  size_t peer_h_off = 0;        // the residual stream h [B][d] fp32 and x16 [B][d] fp16 (the model's own h and x16)
  size_t peer_x16_off = 0;
  unsigned* epoch = nullptr;    // steps run in the fused mode
  std::string tp_fused_why;
  // the prefill section (allocated on first use): chunks of up to kPrefillRows prompt rows of one sequence
  __half* pf_x16 = nullptr;     // [rows][d]
  float* pf_h = nullptr;        // [rows][d]
  __half* pf_xn16 = nullptr;    // [rows][d]
  float* pf_y = nullptr;        // [rows][max(qkv rows, 2F, d)]
  __half* pf_q16 = nullptr;     // [rows][H][hd]
  __half* pf_attn = nullptr;    // [rows][H hd]
  __half* pf_act = nullptr;     // [rows][F]
  uint32_t* pf_pos = nullptr;   // [rows]
  uint32_t* pf_tok = nullptr;   // [cap] the prompt
  float* pf_part = nullptr;     // the split-K partial sums of the prefill GEMMs
  float* sp_y = nullptr;        // the verify step's head rows [32][V]
  int32_t* sp_amax = nullptr;   // and their first maxima
};

namespace agxc {

int run_qmm(agxc_model* m, const agxc_pack& pk, const __half* x, int rows, float* y, int ld, cudaStream_t s,
            float* part, const QmmPush* push = nullptr);
int qmm_ksplit(const agxc_ctx* ctx, const agxc_pack& pk);
int qmm_scratch(agxc_model* m, int rows, float** part);
int gemm_rows(agxc_model* m, const agxc_pack& pk, const __half* x, int rows, float* ybuf, int ld, float* part,
              cudaStream_t s, YRows* out);

namespace {

int dalloc(agxc_model* m, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) return fail(AGXC_ENOMEM, std::string("cudaMalloc(") + std::to_string(bytes) +
                                                     "): " + cudaGetErrorString(e));
  m->allocs.push_back(*p);
  return 0;
}

template <typename T>
int dalloc_t(agxc_model* m, T** p, size_t count) {
  void* v = nullptr;
  int rc = dalloc(m, &v, std::max<size_t>(count * sizeof(T), 256));
  *p = static_cast<T*>(v);
  return rc;
}

void pack_init(agxc_pack& p, agxc_model* m, int n, int k) {
  p.ctx = m->ctx;
  p.n = n;
  p.k = k;
  p.bits = m->d.bits;
  p.group = 64;
  p.sdt = m->d.scale_dtype;
  p.owns = false;
}

size_t pack_tile_bytes(int n, int k, int bits) { return static_cast<size_t>(n) * k * bits / 8; }
size_t pack_sb_bytes(int n, int k) { return static_cast<size_t>(n / 16) * (k / 64) * 64; }

// This launch's trace words (the launch index is m->launches), or NULL when not tracing.
unsigned long long* trace_slot(agxc_model* m) {
  return m->trace && m->launches < m->trace_n ? m->trace + 2 * kTraceSlots * m->launches : nullptr;
}

__global__ void trace_reset_kernel(unsigned long long* t, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) t[i] = (i & 1) ? 0ull : ~0ull;
}

// The parameters of layer l's five launches (qkv, attention, o_proj, gate/up, down) and of the head: one place for
// the per-kernel graph.
void layer_params(agxc_model* m, int l, QmvParams& p, AttnParams& a, QmvParams& q, QmvParams& g, QmvParams& w) {
  const agxc_model_desc& D = m->d;
  const int B = D.batch, H = D.n_heads, KVH = D.n_kv_heads, hd = D.head_dim, d = D.d_model, F = D.ffn;
  const size_t layer_kv = static_cast<size_t>(B) * KVH * D.cap * hd;
  // D1: norm + qkv + bias + RoPE + append
  p.w = m->qkv[l].tiles; p.sb = m->qkv[l].sb; p.N = m->qkv_rows; p.K = d; p.bits = D.bits; p.sdt = D.scale_dtype;
  p.nb = B; p.x = m->x16; p.x_f32 = 0; p.x_ld = d; p.norm_gain = m->gains + static_cast<size_t>(l) * 2 * d;
  p.eps = D.eps; p.bias = D.qkv_bias ? m->bias + static_cast<size_t>(l) * m->qkv_rows : nullptr;
  p.H = H; p.KVH = KVH; p.hd = hd; p.cap = D.cap; p.cos_t = m->cos_t; p.sin_t = m->sin_t; p.q0 = m->q0;
  p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(hd)));
  p.q16 = m->q16; p.kcache = m->kcache + l * layer_kv; p.vcache = m->vcache + l * layer_kv;
  p.part = m->part; p.counters = m->counters; p.err = m->ctx->err_dev;
  p.pos_ready = l > 0;  // q0 is advanced by the head, the kernel just before layer 0's qkv
  // D2: attention
  a.nb = B; a.H = H; a.KVH = KVH; a.hd = hd; a.cap = D.cap; a.S = m->attn_S; a.q0 = m->q0; a.q16 = m->q16;
  a.kc = m->kcache + l * layer_kv; a.vc = m->vcache + l * layer_kv; a.out = m->attn; a.part = m->apart;
  a.counters = m->counters + 4096; a.err = m->ctx->err_dev;
  // D3: o_proj + residual -> h
  q.w = m->wo[l].tiles; q.sb = m->wo[l].sb; q.N = d; q.K = m->attn_dim; q.bits = D.bits; q.sdt = D.scale_dtype;
  q.nb = B; q.x = m->attn; q.x_ld = m->attn_dim; q.out_f32 = m->h; q.out_ld = d; q.res16 = m->x16; q.res_ld = d;
  q.part = m->part; q.counters = m->counters + 8192; q.err = m->ctx->err_dev;
  // D4: norm + gate/up + SiLU*mul -> act
  g.w = m->gu[l].tiles; g.sb = m->gu[l].sb; g.N = 2 * F; g.K = d; g.bits = D.bits; g.sdt = D.scale_dtype;
  g.nb = B; g.x = m->h; g.x_f32 = 1; g.x_ld = d; g.norm_gain = m->gains + static_cast<size_t>(l) * 2 * d + d;
  g.eps = D.eps; g.out_f16 = m->act; g.out_ld = F; g.part = m->part; g.counters = m->counters + 12288;
  g.err = m->ctx->err_dev;
  // D5: down + residual -> x16
  w.w = m->down[l].tiles; w.sb = m->down[l].sb; w.N = d; w.K = F; w.bits = D.bits; w.sdt = D.scale_dtype;
  w.nb = B; w.x = m->act; w.x_ld = F; w.out_f16 = m->x16; w.out_ld = d; w.res32 = m->h; w.res_ld = d;
  w.part = m->part; w.counters = m->counters + 16384; w.err = m->ctx->err_dev;
}

void head_params(agxc_model* m, QmvParams& hp) {
  const agxc_model_desc& D = m->d;
  const int d = D.d_model;
  hp.w = m->head.tiles; hp.sb = m->head.sb; hp.N = D.vocab; hp.K = d; hp.bits = D.bits; hp.sdt = D.scale_dtype;
  hp.nb = D.batch; hp.x = m->x16; hp.x_ld = d; hp.norm_gain = m->final_gain; hp.eps = D.eps;
  hp.out_f32 = D.keep_logits ? m->logits : nullptr; hp.V = D.vocab; hp.embed = m->embed; hp.x_next = m->x16;
  hp.d = d; hp.q0_rw = m->q0; hp.log = m->log; hp.tok_out = m->tok; hp.force_next = m->force_next;
  hp.cap = D.cap; hp.pairs = m->pairs;
  hp.counters = m->counters + 20480; hp.err = m->ctx->err_dev;
}

bool fused_active(const agxc_model* m) { return m->d.batch == 1 && m->fused && m->fs_ok; }

const __half* qk_gains_of(const agxc_model* m, int l) {
  return m->qk_norm ? m->qk_gains + static_cast<size_t>(l) * 2 * m->d.head_dim : nullptr;
}

int enqueue_step_fused(agxc_model* m, cudaStream_t s) {
  const agxc_model_desc& D = m->d;
  FstepArgs a;
  a.L = D.n_layers; a.d = D.d_model; a.H = D.n_heads; a.KVH = D.n_kv_heads; a.hd = D.head_dim; a.F = D.ffn;
  a.V = D.vocab; a.cap = D.cap; a.bits = D.bits; a.sdt = D.scale_dtype; a.stages = m->fs_stages; a.smax = m->fs_smax;
  a.grid = m->ctx->num_sms; a.eps = D.eps; a.wait_ns = m->dev_wait_ns;
  a.maps = m->fs_maps; a.gains = m->gains; a.bias = D.qkv_bias ? m->bias : nullptr; a.final_gain = m->final_gain;
  a.qkg = m->qk_norm ? m->qk_gains : nullptr; a.qkraw = m->qkv_raw;
  a.embed = m->embed; a.kc = m->kcache; a.vc = m->vcache; a.cos_t = m->cos_t; a.sin_t = m->sin_t; a.q0 = m->q0;
  a.log = m->log; a.tok_out = m->tok; a.force_next = m->force_next; a.x16 = m->x16;
  a.logits = D.keep_logits ? m->logits : nullptr; a.q16 = m->q16; a.apart = m->fs_apart; a.acc = m->fs_acc;
  a.sync = m->fs_sync; a.nctr = m->fs_nctr; a.pairs = m->pairs; a.err = m->ctx->err_dev; a.trace = m->cta_trace;
  m->launches = 1;
  return fstep_launch(a, s);
}

// The fused step's TMA maps: one per role over all layers (the layers' packs of a role sit at a constant stride in
// the weight arena): the qkv, o_proj, gate/up and down packs (weights and scale/bias), then the head, then the K and
// V caches. Box shapes: row tiles x gchunk groups (qkv, gate/up, head); one row tile x the group's K range (o_proj);
// dn_rows row tiles x one group (down); 64 dims x the stage's keys (caches).
int build_fused_maps(agxc_model* m) {
  const agxc_model_desc& D = m->d;
  const int L = D.n_layers, d = D.d_model, hd = D.head_dim, G = D.n_heads / D.n_kv_heads;
  const int TW = tile_bytes(D.bits) / 4, TPS = fstep_tiles_per_stage(D.bits);
  const int gd = d / 64, gchunk = std::min(gd, TPS), gk = G * hd / 64, dn_rows = std::min(d / 16, TPS);
  std::vector<CUtensorMap> maps(fstep_map_count());
  const uint64_t LS = L > 1 ? static_cast<uint64_t>(m->qkv[1].tiles - m->qkv[0].tiles) : 256;
  auto role = [&](CUtensorMap* mp, const std::vector<agxc_pack>& v, int cg, int rw) -> int {
    for (int l = 0; l < L; ++l)
      if (v[l].tiles != v[0].tiles + l * LS || v[l].sb != v[0].sb + l * LS)
        return fail(AGXC_EINVAL, "fused step: the layers' packs are not at a constant stride");
    const int G_ = v[0].k / 64, RT = v[0].n / 16;
    if (int rc = encode_pack_map_layers(mp, v[0].tiles, TW, G_, RT, L, LS, cg, rw)) return rc;
    return encode_pack_map_layers(mp + 1, v[0].sb, 16, G_, RT, L, LS, cg, rw);
  };
  int rc;
  if ((rc = role(&maps[0], m->qkv, gchunk, 1)) || (rc = role(&maps[2], m->wo, gk, 1)) ||
      (rc = role(&maps[4], m->gu, gchunk, 1)) || (rc = role(&maps[6], m->down, 1, dn_rows)))
    return rc;
  {
    const int G_ = m->head.k / 64, RT = m->head.n / 16;
    if ((rc = encode_pack_map(&maps[8], m->head.tiles, TW, G_, RT, gchunk, 1)) ||
        (rc = encode_pack_map(&maps[9], m->head.sb, 16, G_, RT, gchunk, 1)))
      return rc;
  }
  const int kc_keys = 16384 / (4 * hd);
  const int64_t Z = static_cast<int64_t>(L) * D.n_kv_heads;
  if ((rc = encode_kv_map_box(&maps[10], m->kcache, hd, D.cap, Z, kc_keys))) return rc;
  if ((rc = encode_kv_map_box(&maps[11], m->vcache, hd, D.cap, Z, kc_keys))) return rc;
  AGXC_CUDA(cudaMemcpy(m->fs_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
  return 0;
}

// Both parities' counters and accumulators and the step counter to zero (at creation, and after a step that gave up).
int fused_reset(agxc_model* m) {
  if (!m->fs_ok) return 0;
  const agxc_model_desc& D = m->d;
  AGXC_CUDA(cudaMemset(m->fs_sync, 0, (64 + 2 * static_cast<size_t>(m->fs_nctr)) * 4));
  AGXC_CUDA(cudaMemset(m->fs_acc, 0, static_cast<size_t>(4) * D.n_layers * D.d_model * 4));
  return 0;
}

// The batched step (batch >= 32): RMSNorm -> tensor-core GEMM -> per-row kernel for each projection, attention
// between. With `ev`, events bracket the six kinds (qkv = norm + GEMM + RoPE/append; attn; wo = GEMM + residual; ffn =
// norm + GEMM + SwiGLU; down = GEMM + residual; head = norm + GEMM + argmax/generation).
int enqueue_step_batched(agxc_model* m, cudaStream_t s, cudaEvent_t* ev) {
  const agxc_model_desc& D = m->d;
  const int B = D.batch, d = D.d_model, F = D.ffn, H = D.n_heads, KVH = D.n_kv_heads, hd = D.head_dim;
  int rc;
  int kind = 0;
  auto open = [&]() -> int {
    if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * kind], s));
    return 0;
  };
  auto close = [&]() -> int {
    if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * kind + 1], s));
    ++kind;
    return 0;
  };
  // finished rows in y (the head, the peer push, an NCCL all-reduce) / rows whose consumers add the K ranges
  auto gemm = [&](const agxc_pack& pk, const __half* x, float* y, int ld, const QmmPush* push = nullptr) -> int {
    return run_qmm(m, pk, x, B, y, ld, s, m->qpart, push);
  };
  YRows yr;
  auto gemm_r = [&](const agxc_pack& pk, const __half* x, int ld) -> int {
    return gemm_rows(m, pk, x, B, m->ybuf, ld, m->qpart, s, &yr);
  };
  const YRows ydone{m->ybuf, d, 1, 0};
  const bool fused = m->comm && m->tp_fused && m->tp_fused_ok;
  auto push_of = [&](int buf) {  // this rank's slot of buffer `buf` on every rank, and their arrival counters
    QmmPush ps;
    ps.ranks = m->tp;
    ps.tiles_per_rank = d / 128 / m->tp;
    ps.to_owner = m->tp_two_shot;
    const size_t slot = (static_cast<size_t>(buf) * m->tp + m->tp_rank) * B * d;
    for (int r = 0; r < m->tp; ++r) {
      uint8_t* base = static_cast<uint8_t*>(m->peer[r]);
      ps.slot[r] = reinterpret_cast<float*>(base) + slot;
      ps.flag[r] = reinterpret_cast<unsigned*>(base + m->peer_flags_off) + buf;
    }
    return ps;
  };
  auto gather_of = [&](int buf) {  // every rank's residual stream (h for o_proj, x16 for down) and gather counter
    TpGather g;
    for (int r = 0; r < m->tp; ++r) {
      uint8_t* base = static_cast<uint8_t*>(m->peer[r]);
      g.out32[r] = reinterpret_cast<float*>(base + m->peer_h_off);
      g.out16[r] = reinterpret_cast<__half*>(base + m->peer_x16_off);
      g.gflag[r] = reinterpret_cast<unsigned*>(base + m->peer_flags_off) + 2 + buf;
    }
    return g;
  };
  const float qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(hd)));
  const int pdl = m->pdl ? 1 : 0;  // every kernel of the chain may start before its predecessor ends
  m->launches = 0;
  for (int l = 0; l < D.n_layers; ++l) {
    QmvParams p, q, g, w;
    AttnParams a;
    layer_params(m, l, p, a, q, g, w);
    if ((rc = open()) || (rc = launch_rmsnorm(m->x16, 0, B, d, p.norm_gain, D.eps, m->xn16, s, pdl)) ||
        (rc = gemm_r(m->qkv[l], m->xn16, m->qkv_rows)) ||
        (rc = launch_rope_append(yr, m->qkv_rows, p.bias, m->cos_t, m->sin_t, m->q0, H, KVH, hd, D.cap, qscale, m->q16,
                                 p.kcache, p.vcache, B, s, -1, qk_gains_of(m, l), D.eps, pdl)) ||
        (rc = close()))
      return rc;
    a.pdl = pdl;
    if ((rc = open()) || (rc = launch_attention(m->ctx, a, s)) || (rc = close())) return rc;
    if (fused) {  // o_proj tiles pushed to their owner ranks by the GEMM; each owner's sum + residual to every rank
      QmmPush ps = push_of(0);
      if ((rc = open()) || (rc = gemm(m->wo[l], m->attn, m->ybuf, d, &ps)) ||
          (rc = launch_tp_reduce(m->recv, m->tp, m->tp_rank, m->recv_flags, m->epoch, D.n_layers, l,
                                 ps.tiles_per_rank, m->x16, nullptr, gather_of(0), d, B, m->ctx->err_dev, s,
                                 m->tp_two_shot, m->dev_wait_ns)) ||
          (rc = close()))
        return rc;
    } else if (m->comm) {  // NCCL: the finished rows all-reduced, then the residual
      if ((rc = open()) || (rc = gemm(m->wo[l], m->attn, m->ybuf, d, nullptr)) ||
          (rc = tp_allreduce_f32(m->comm, m->ybuf, static_cast<size_t>(B) * d, s)) ||
          (rc = launch_residual16(ydone, m->x16, m->h, d, B, s, pdl)) || (rc = close()))
        return rc;
    } else if ((rc = open()) || (rc = gemm_r(m->wo[l], m->attn, d)) ||
               (rc = launch_residual16(yr, m->x16, m->h, d, B, s, pdl)) || (rc = close())) {
      return rc;
    }
    if ((rc = open()) || (rc = launch_rmsnorm(m->h, 1, B, d, g.norm_gain, D.eps, m->xn16, s, pdl)) ||
        (rc = gemm_r(m->gu[l], m->xn16, 2 * F)) || (rc = launch_swiglu(yr, m->act, F, B, s, pdl)) ||
        (rc = close()))
      return rc;
    if (fused) {
      QmmPush ps = push_of(1);
      if ((rc = open()) || (rc = gemm(m->down[l], m->act, m->ybuf, d, &ps)) ||
          (rc = launch_tp_reduce(m->recv + static_cast<size_t>(m->tp) * B * d, m->tp, m->tp_rank, m->recv_flags + 1,
                                 m->epoch, D.n_layers, l, ps.tiles_per_rank, nullptr, m->h, gather_of(1), d, B,
                                 m->ctx->err_dev, s, m->tp_two_shot, m->dev_wait_ns)) ||
          (rc = close()))
        return rc;
    } else if (m->comm) {
      if ((rc = open()) || (rc = gemm(m->down[l], m->act, m->ybuf, d, nullptr)) ||
          (rc = tp_allreduce_f32(m->comm, m->ybuf, static_cast<size_t>(B) * d, s)) ||
          (rc = launch_residual32(ydone, m->h, m->x16, d, B, s, pdl)) || (rc = close()))
        return rc;
    } else if ((rc = open()) || (rc = gemm_r(m->down[l], m->act, d)) ||
               (rc = launch_residual32(yr, m->h, m->x16, d, B, s, pdl)) || (rc = close())) {
      return rc;
    }
  }
  if (m->comm) {  // vocabulary sliced over ranks: local first maxima, all-gathered, then the same choice everywhere
    if ((rc = open()) || (rc = launch_rmsnorm(m->x16, 0, B, d, m->final_gain, D.eps, m->xn16, s, pdl)) ||
        (rc = gemm(m->head, m->xn16, m->logits, D.vocab)) ||
        (rc = launch_argmax_part(m->logits, D.vocab, m->v0, m->amax, B, s)) ||
        (rc = tp_allgather_u32(m->comm, m->amax, m->amax_all, static_cast<size_t>(2) * B, s)) ||
        (rc = launch_gen_from_pairs(m->amax_all, m->tp, m->vt, m->embed, d, m->q0, m->log, D.cap, m->tok,
                                    m->force_next, m->x16, m->ctx->err_dev, B, s, fused ? m->epoch : nullptr)) ||
        (rc = close()))
      return rc;
    m->launches = 11 * D.n_layers + 4;  // this library's kernels (the collectives are the communicator's)
    return 0;
  }
  if ((rc = open()) || (rc = launch_rmsnorm(m->x16, 0, B, d, m->final_gain, D.eps, m->xn16, s, pdl)) ||
      (rc = gemm(m->head, m->xn16, m->logits, D.vocab)) ||
      (rc = launch_argmax_gen(m->logits, D.vocab, m->embed, d, m->q0, m->log, D.cap, m->tok, m->force_next, m->x16,
                              m->ctx->err_dev, B, s, pdl)) ||
      (rc = close()))
    return rc;
  m->launches = 11 * D.n_layers + 3;
  return 0;
}

// When `ev` is given, an event is recorded before and after every launch (kind order: qkv, attn, wo, ffn, down per
// layer, then head): ev holds 2 * launches events.
int enqueue_step(agxc_model* m, cudaStream_t s, cudaEvent_t* ev = nullptr) {
  if (m->d.batch >= 32) return enqueue_step_batched(m, s, ev);
  if (!ev && fused_active(m)) return enqueue_step_fused(m, s);
  const agxc_model_desc& D = m->d;
  int rc;
  m->launches = 0;
  auto launch_gemv = [&](QmvParams& x, const QmvPlan& plan, int epi) -> int {
    x.pdl = m->pdl;
    x.bulk = m->bulk;
    x.trace = trace_slot(m);
    if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * m->launches], s));
    if (int r = launch_qmv_epi(m->ctx, x, plan, epi, s)) return r;
    if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * m->launches + 1], s));
    ++m->launches;
    return 0;
  };
  for (int l = 0; l < D.n_layers; ++l) {
    QmvParams p, q, g, w;
    AttnParams a;
    layer_params(m, l, p, a, q, g, w);
    if (m->qk_norm) {
      // QK-norm: the qkv GEMV's fp32 rows (physical order), then the per-head norm + RoPE + append kernel; one
      // "qkv" entry of the launch accounting
      QmvParams r = p;
      r.out_f32 = m->qkv_raw;
      r.out_ld = m->qkv_rows;
      r.pdl = 0;
      r.bulk = m->bulk;
      r.trace = nullptr;
      YRows yr;
      yr.y = m->qkv_raw;
      yr.ld = m->qkv_rows;
      if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * m->launches], s));
      if ((rc = launch_qmv_epi(m->ctx, r, m->p_qkv_raw, EPI_F32, s)) ||
          (rc = launch_rope_append(yr, m->qkv_rows, p.bias, m->cos_t, m->sin_t, m->q0, D.n_heads, D.n_kv_heads,
                                   D.head_dim, D.cap, p.qscale, m->q16, p.kcache, p.vcache, D.batch, s, -1,
                                   qk_gains_of(m, l), D.eps)))
        return rc;
      if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * m->launches + 1], s));
      ++m->launches;
    } else if ((rc = launch_gemv(p, m->p_qkv, EPI_QKV))) {
      return rc;
    }
    a.pdl = m->pdl;
    a.trace = trace_slot(m);
    if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * m->launches], s));
    if ((rc = launch_attention(m->ctx, a, s))) return rc;
    if (ev) AGXC_CUDA(cudaEventRecord(ev[2 * m->launches + 1], s));
    ++m->launches;
    if ((rc = launch_gemv(q, m->p_wo, EPI_RES1)) || (rc = launch_gemv(g, m->p_gu, EPI_SWIGLU)) ||
        (rc = launch_gemv(w, m->p_down, EPI_RES2)))
      return rc;
  }
  QmvParams hp;
  head_params(m, hp);
  return launch_gemv(hp, m->p_head, EPI_ARGMAX);
}

// Wait for an event recorded after a step (or a call's steps): bounded and aborting under tensor parallelism.
int wait_done(agxc_model* m, cudaEvent_t e) {
  if (m->comm) return tp_wait(m->comm, e, m->wait_ms);
  AGXC_CUDA(cudaEventSynchronize(e));
  return 0;
}

int ensure_graph(agxc_model* m) {
  if (m->exec) return 0;
  cudaStream_t s = m->ctx->stream;
  AGXC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(m, s);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  m->graph = g;
  AGXC_CUDA(cudaGraphInstantiate(&m->exec, g, 0));
  return 0;
}

}  // namespace

int model_create_local(agxc_ctx* ctx, const agxc_model_desc& G, int T, agxc_model** out);

// A bounded barrier over the ranks: a one-float all-reduce, waited for on the host.
int tp_barrier(agxc_model* m) {
  cudaStream_t s = m->ctx->stream;
  if (int rc = tp_allreduce_f32(m->comm, m->ybuf, 1, s)) return rc;
  AGXC_CUDA(cudaEventRecord(m->ev1, s));
  return wait_done(m, m->ev1);
}

// The fused GEMM + all-reduce: the receive buffers (one allocation per rank, exported by CUDA IPC), every other
// rank's mapped here; the handles travel by an all-gather on the communicator. Every rank ends with the same
// tp_fused_ok (an all-reduce of the per-rank outcomes), so all ranks take the same path.
int tp_peer_setup(agxc_model* m) {
  const int T = m->tp, B = m->d.batch, d = m->d.d_model;
  cudaStream_t s = m->ctx->stream;
  if ((d / 128) % T) {
    m->tp_fused_why = "d_model / 128 is not a multiple of the ranks";
    return 0;
  }
  // [2][T][B][d] fp32 receive slots | 4 counters | h [B][d] fp32 | x16 [B][d] fp16, each 256-byte aligned
  m->peer_flags_off = static_cast<size_t>(2) * T * B * d * 4;
  m->peer_h_off = m->peer_flags_off + 256;
  m->peer_x16_off = m->peer_h_off + align_up(static_cast<size_t>(B) * d * 4, 256);
  const size_t bytes = m->peer_x16_off + align_up(static_cast<size_t>(B) * d * 2, 256);
  void* base = nullptr;
  AGXC_CUDA(cudaMalloc(&base, bytes));
  m->allocs.push_back(base);
  AGXC_CUDA(cudaMemset(base, 0, bytes));
  m->recv = static_cast<float*>(base);
  m->recv_flags = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(base) + m->peer_flags_off);
  if (int rc = dalloc_t(m, &m->epoch, 1)) return rc;
  AGXC_CUDA(cudaMemset(m->epoch, 0, 4));
  m->peer[m->tp_rank] = base;
  int ok = 1;
  cudaIpcMemHandle_t mine;
  std::memset(&mine, 0, sizeof(mine));
  if (cudaIpcGetMemHandle(&mine, base) != cudaSuccess) {
    cudaGetLastError();
    ok = 0;
    m->tp_fused_why = "cudaIpcGetMemHandle failed";
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle of 64 bytes");
  uint32_t* hd = nullptr;
  if (int rc = dalloc_t(m, &hd, static_cast<size_t>(16) * (T + 1))) return rc;
  AGXC_CUDA(cudaMemcpy(hd, &mine, 64, cudaMemcpyHostToDevice));
  if (int rc = tp_allgather_u32(m->comm, hd, hd + 16, 16, s)) return rc;
  AGXC_CUDA(cudaEventRecord(m->ev1, s));
  if (int rc = wait_done(m, m->ev1)) return rc;
  std::vector<cudaIpcMemHandle_t> all(T);
  AGXC_CUDA(cudaMemcpy(all.data(), hd + 16, static_cast<size_t>(64) * T, cudaMemcpyDeviceToHost));
  for (int r = 0; r < T && ok; ++r) {
    if (r == m->tp_rank) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      m->tp_fused_why = "cudaIpcOpenMemHandle of rank " + std::to_string(r) + " failed";
      break;
    }
    m->peer[r] = p;
  }
  // agree: the sum of the per-rank outcomes must be T
  const float one = ok ? 1.f : 0.f;
  AGXC_CUDA(cudaMemcpy(m->ybuf, &one, 4, cudaMemcpyHostToDevice));
  if (int rc = tp_allreduce_f32(m->comm, m->ybuf, 1, s)) return rc;
  AGXC_CUDA(cudaEventRecord(m->ev1, s));
  if (int rc = wait_done(m, m->ev1)) return rc;
  float sum = 0.f;
  AGXC_CUDA(cudaMemcpy(&sum, m->ybuf, 4, cudaMemcpyDeviceToHost));
  m->tp_fused_ok = sum == static_cast<float>(T);
  // two-shot from 8 ranks: at 4 the one-shot push (4 MB out a rank per all-reduce at 64 sequences) measured faster
  // than the two-shot's extra synchronisation round (o_proj group 44.7 against 63.5 us a layer, 7B TP4)
  m->tp_two_shot = T >= 8;
  if (!m->tp_fused_ok && m->tp_fused_why.empty()) m->tp_fused_why = "a peer rank could not map the buffers";
  m->tp_fused = m->tp_fused_ok;
  if (m->tp_fused_ok) {  // the residual stream lives in the exported allocation: owners write every rank's rows
    AGXC_CUDA(cudaMemcpy(static_cast<uint8_t*>(base) + m->peer_h_off, m->h, static_cast<size_t>(B) * d * 4,
                         cudaMemcpyDeviceToDevice));
    AGXC_CUDA(cudaMemcpy(static_cast<uint8_t*>(base) + m->peer_x16_off, m->x16, static_cast<size_t>(B) * d * 2,
                         cudaMemcpyDeviceToDevice));
    m->h = reinterpret_cast<float*>(static_cast<uint8_t*>(base) + m->peer_h_off);
    m->x16 = reinterpret_cast<__half*>(static_cast<uint8_t*>(base) + m->peer_x16_off);
  }
  return 0;
}

// Before the buffers go: every rank stops using the others' (barrier), unmaps them, and waits until all have.
void tp_peer_teardown(agxc_model* m) {
  if (!m->comm || !m->recv || !m->ev1) return;
  const bool synced = tp_barrier(m) == 0;
  for (int r = 0; r < m->tp; ++r)
    if (r != m->tp_rank && m->peer[r]) cudaIpcCloseMemHandle(m->peer[r]);
  if (synced) tp_barrier(m);
}

int model_create(agxc_ctx* ctx, const agxc_model_desc* desc, agxc_model** out) {
  const agxc_model_desc& D = *desc;
  if (D.bits != 4 && D.bits != 8) return fail(AGXC_EINVAL, "model: bits must be 4 or 8");
  if (D.group != 64) return fail(AGXC_EINVAL, "model: group 64 only");
  if (D.scale_dtype != 0 && D.scale_dtype != 1) return fail(AGXC_EINVAL, "model: scale_dtype fp16 (0) or bf16 (1)");
  if (D.head_dim != 64 && D.head_dim != 128) return fail(AGXC_EINVAL, "model: head_dim 64 or 128");
  if (D.n_kv_heads < 1 || D.n_heads % D.n_kv_heads) return fail(AGXC_EINVAL, "model: heads multiple of kv_heads");
  if (D.n_heads / D.n_kv_heads > 8) return fail(AGXC_EINVAL, "model: at most 8 query heads per KV head");
  if (D.d_model % 64 || D.ffn % 64 || (D.n_heads * D.head_dim) % 64)
    return fail(AGXC_EINVAL, "model: d_model, ffn and heads*head_dim must be multiples of 64");
  if (D.ffn % 16 || D.vocab % 16 || D.vocab < 16) return fail(AGXC_EINVAL, "model: vocab must be a multiple of 16");
  const bool batched = D.batch >= 32;
  if (D.batch < 1 || (D.batch > 8 && !batched) || D.batch > 256 || (batched && D.batch % 16))
    return fail(AGXC_EINVAL, "model: batch 1..8 (GEMV), or 32..256 in steps of 16 (tensor-core GEMM)");
  if (batched && (D.d_model % 128 || D.ffn % 64 || ((D.n_heads + 2 * D.n_kv_heads) * D.head_dim) % 128 ||
                  D.vocab % 128))
    return fail(AGXC_EINVAL, "model: batch >= 32 needs d_model, qkv rows and vocab multiples of 128");
  if (D.cap < 2) return fail(AGXC_EINVAL, "model: cap >= 2");
  if (D.n_layers < 1) return fail(AGXC_EINVAL, "model: at least one layer");
  if (D.d_model % 8) return fail(AGXC_EINVAL, "model: d_model multiple of 8");
  const int T = D.tp_world > 1 ? D.tp_world : 1;
  if (D.tp_world < 0 || T > 8 || D.tp_rank < 0 || D.tp_rank >= T)
    return fail(AGXC_EINVAL, "model: tp_world 0..8 and 0 <= tp_rank < tp_world");
  if (T > 1) {
    if (!batched) return fail(AGXC_EINVAL, "model: tensor parallelism needs batch >= 32 (the tensor-core GEMM step)");
    if (D.n_heads % T || D.n_kv_heads % T || D.ffn % (64 * T))
      return fail(AGXC_EINVAL, "model: tensor parallelism needs heads and KV heads divisible by tp_world, ffn by 64 "
                               "x tp_world");
  }
  return model_create_local(ctx, D, T, out);
}

// The rank's vocabulary slice of the head, in 128-row tiles: [first, first + count).
void vocab_slice(int vocab, int world, int rank, int* first, int* count) {
  const int tiles = vocab / 128;
  const int t0 = static_cast<int>(static_cast<int64_t>(tiles) * rank / world);
  const int t1 = static_cast<int>(static_cast<int64_t>(tiles) * (rank + 1) / world);
  *first = world > 1 ? 128 * t0 : 0;
  *count = world > 1 ? 128 * (t1 - t0) : vocab;
}

int model_create_local(agxc_ctx* ctx, const agxc_model_desc& G, int T, agxc_model** out) {
  agxc_model_desc D = G;  // this rank's local shape
  int v0 = 0, vn = G.vocab;
  vocab_slice(G.vocab, T, T > 1 ? G.tp_rank : 0, &v0, &vn);
  D.n_heads = G.n_heads / T;
  D.n_kv_heads = G.n_kv_heads / T;
  D.ffn = G.ffn / T;
  D.vocab = vn;
  const bool batched = D.batch >= 32;
  if (vn < 128 && T > 1) return fail(AGXC_EINVAL, "model: fewer 128-row vocabulary tiles than ranks");
  if (batched && ((D.n_heads + 2 * D.n_kv_heads) * D.head_dim) % 128)
    return fail(AGXC_EINVAL, "model: batch >= 32 needs each rank's qkv rows a multiple of 128");

  agxc_model* m = new agxc_model();
  m->ctx = ctx;
  m->d = D;
  m->tp = T;
  m->tp_rank = T > 1 ? G.tp_rank : 0;
  m->vt = G.vocab;
  m->v0 = v0;
  const int L = D.n_layers, d = D.d_model, F = D.ffn, V = D.vocab, B = D.batch, hd = D.head_dim;
  m->qkv_rows = (D.n_heads + 2 * D.n_kv_heads) * hd;
  m->attn_dim = D.n_heads * hd;
  int rc = 0;
  auto bail = [&](int code) {
    agxc_model_free(m);
    return code;
  };

  // one allocation for every pack (tiles then scale/bias per matrix, 256-byte aligned)
  struct Mat { agxc_pack* p; int n, k; };
  m->qkv.resize(L); m->wo.resize(L); m->gu.resize(L); m->down.resize(L);
  std::vector<Mat> mats;
  for (int l = 0; l < L; ++l) {
    mats.push_back({&m->qkv[l], m->qkv_rows, d});
    mats.push_back({&m->wo[l], d, m->attn_dim});
    mats.push_back({&m->gu[l], 2 * F, d});
    mats.push_back({&m->down[l], d, F});
  }
  mats.push_back({&m->head, V, d});
  size_t total = 0;
  for (auto& x : mats) {
    total += align_up(pack_tile_bytes(x.n, x.k, D.bits), 256);
    total += align_up(pack_sb_bytes(x.n, x.k), 256);
  }
  void* wm = nullptr;
  if ((rc = dalloc(m, &wm, total))) return bail(rc);
  m->wmem = static_cast<uint8_t*>(wm);
  size_t off = 0;
  for (auto& x : mats) {
    pack_init(*x.p, m, x.n, x.k);
    x.p->tiles = m->wmem + off;
    off += align_up(pack_tile_bytes(x.n, x.k, D.bits), 256);
    x.p->sb = m->wmem + off;
    off += align_up(pack_sb_bytes(x.n, x.k), 256);
  }
  for (int l = 0; l < L; ++l) m->gu[l].gateup = 1;

  if ((rc = dalloc_t(m, &m->gains, static_cast<size_t>(L) * 2 * d))) return bail(rc);
  if ((rc = dalloc_t(m, &m->bias, static_cast<size_t>(L) * m->qkv_rows))) return bail(rc);
  if ((rc = dalloc_t(m, &m->final_gain, d))) return bail(rc);
  if ((rc = dalloc_t(m, &m->qk_gains, static_cast<size_t>(L) * 2 * hd))) return bail(rc);
  if ((rc = dalloc_t(m, &m->qkv_raw, static_cast<size_t>(B) * m->qkv_rows))) return bail(rc);
  if ((rc = dalloc_t(m, &m->embed, static_cast<size_t>(m->vt) * d))) return bail(rc);
  const size_t kv = static_cast<size_t>(L) * B * D.n_kv_heads * D.cap * hd;
  if ((rc = dalloc_t(m, &m->kcache, kv))) return bail(rc);
  if ((rc = dalloc_t(m, &m->vcache, kv))) return bail(rc);
  if ((rc = dalloc_t(m, &m->x16, static_cast<size_t>(B) * d))) return bail(rc);
  if ((rc = dalloc_t(m, &m->h, static_cast<size_t>(B) * d))) return bail(rc);
  if ((rc = dalloc_t(m, &m->q16, static_cast<size_t>(B) * m->attn_dim))) return bail(rc);
  if ((rc = dalloc_t(m, &m->attn, static_cast<size_t>(B) * m->attn_dim))) return bail(rc);
  if ((rc = dalloc_t(m, &m->act, static_cast<size_t>(B) * F))) return bail(rc);
  if ((D.keep_logits || batched) && (rc = dalloc_t(m, &m->logits, static_cast<size_t>(B) * V))) return bail(rc);
  if (batched) {  // the tensor-core GEMMs' normed fp16 inputs and fp32 output rows
    const size_t yn = std::max({static_cast<size_t>(m->qkv_rows), static_cast<size_t>(2) * F,
                                static_cast<size_t>(d)});
    if ((rc = dalloc_t(m, &m->xn16, static_cast<size_t>(B) * d))) return bail(rc);
    if ((rc = dalloc_t(m, &m->ybuf, static_cast<size_t>(B) * yn))) return bail(rc);
    if ((rc = qmm_scratch(m, B, &m->qpart))) return bail(rc);
  }
  if ((rc = dalloc_t(m, &m->q0, B))) return bail(rc);
  if ((rc = dalloc_t(m, &m->log, static_cast<size_t>(B) * D.cap))) return bail(rc);
  if ((rc = dalloc_t(m, &m->tok, B))) return bail(rc);
  if ((rc = dalloc_t(m, &m->force_next, B))) return bail(rc);
  if ((rc = dalloc_t(m, &m->cos_t, static_cast<size_t>(D.cap) * hd / 2))) return bail(rc);
  if ((rc = dalloc_t(m, &m->sin_t, static_cast<size_t>(D.cap) * hd / 2))) return bail(rc);

  // plans and scratch
  const int nbg = std::min(B, 8);  // the GEMV plans (batch >= 32 runs the tensor-core GEMM instead)
  m->p_qkv = plan_qmv(ctx, m->qkv_rows, d, D.bits, nbg, EPI_QKV, hd, 0);
  m->p_qkv_raw = plan_qmv(ctx, m->qkv_rows, d, D.bits, nbg, EPI_F32, hd, 0);
  m->p_wo = plan_qmv(ctx, d, m->attn_dim, D.bits, nbg, EPI_RES1, hd, 0);
  m->p_gu = plan_qmv(ctx, 2 * F, d, D.bits, nbg, EPI_SWIGLU, hd, 0);
  m->p_down = plan_qmv(ctx, d, F, D.bits, nbg, EPI_RES2, hd, 0);
  m->p_head = plan_qmv(ctx, V, d, D.bits, nbg, EPI_ARGMAX, hd, 0);
  m->attn_S = attn_splits(ctx, B, D.n_kv_heads, D.cap);
  size_t part = 0;
  part = std::max(part, qmv_part_floats(m->p_qkv, m->qkv_rows, nbg, EPI_QKV));
  part = std::max(part, qmv_part_floats(m->p_qkv_raw, m->qkv_rows, nbg, EPI_F32));
  part = std::max(part, qmv_part_floats(m->p_wo, d, nbg, EPI_RES1));
  part = std::max(part, qmv_part_floats(m->p_gu, 2 * F, nbg, EPI_SWIGLU));
  part = std::max(part, qmv_part_floats(m->p_down, d, nbg, EPI_RES2));
  if ((rc = dalloc_t(m, &m->part, std::max<size_t>(part, 64)))) return bail(rc);
  if ((rc = dalloc_t(m, &m->pairs, static_cast<size_t>(std::max(m->p_head.grid, ctx->num_sms)) * 16)))
    return bail(rc);
  // the fused step: batch 1 on one device, when a ring of stages fits the shared memory; its maps, counters,
  // accumulators and attention partials
  {
    const int G = D.n_heads / D.n_kv_heads;
    const int nrc = (d / 64 + fstep_tiles_per_stage(D.bits) - 1) / fstep_tiles_per_stage(D.bits);
    m->fs_stages = fstep_stages(ctx, d, G, hd);
    // the qkv tiles of a CTA are consumed as one batch (at most 16 chunks, within the ring); the norm keeps the
    // row's 8-element slices in registers, two per consumer thread at most (fstep_max_d)
    const int qkv_tiles = (D.n_heads + 2 * D.n_kv_heads) * hd / 16;
    const int nq_max = (qkv_tiles + ctx->num_sms - 1) / ctx->num_sms;
    m->fs_ok = B == 1 && T == 1 && d % 64 == 0 && F % 64 == 0 && (G * hd) % 64 == 0 && V % 16 == 0 &&
               m->fs_stages >= 4 * nrc && G <= 8 && d <= fstep_max_d() && nq_max * nrc <= 16 && nq_max * nrc <= m->fs_stages;
    if (m->fs_ok) {
      // attention splits per KV group: the SMs over the groups, and the merge's weights (G per split + G sums) must
      // fit the d floats of the h buffer it borrows
      m->fs_smax = std::max(1, std::min(ctx->num_sms / D.n_kv_heads, d / G - 1));
      m->fs_nctr = fstep_counters(L, D.n_kv_heads);
      void* mp = nullptr;
      if ((rc = dalloc(m, &mp, static_cast<size_t>(fstep_map_count()) * sizeof(CUtensorMap))))
        return bail(rc);
      m->fs_maps = static_cast<CUtensorMap*>(mp);
      if ((rc = dalloc_t(m, &m->fs_sync, 64 + 2 * static_cast<size_t>(m->fs_nctr)))) return bail(rc);
      if ((rc = dalloc_t(m, &m->fs_acc, static_cast<size_t>(4) * L * d))) return bail(rc);
      if ((rc = dalloc_t(m, &m->fs_apart, static_cast<size_t>(D.n_kv_heads) * m->fs_smax * G * (hd + 2))))
        return bail(rc);
      if ((rc = build_fused_maps(m)) || (rc = fused_reset(m))) return bail(rc);
    }
  }
  m->counters_n = 24576;
  if (static_cast<size_t>(m->qkv_rows / hd) > 4096 || static_cast<size_t>(B * D.n_kv_heads) > 4096 ||
      static_cast<size_t>(2 * F / 32) > 4096 || static_cast<size_t>(d / 16) > 4096)
    return bail(fail(AGXC_EINVAL, "model: too many epilogue blocks for the counter regions"));
  if ((rc = dalloc_t(m, &m->counters, m->counters_n))) return bail(rc);
  cudaStream_t s = ctx->stream;
  if (cudaMemsetAsync(m->counters, 0, m->counters_n * sizeof(unsigned), s) != cudaSuccess ||
      cudaMemsetAsync(m->kcache, 0, kv * 2, s) != cudaSuccess || cudaMemsetAsync(m->vcache, 0, kv * 2, s) != cudaSuccess ||
      cudaMemsetAsync(m->q0, 0, B * 4, s) != cudaSuccess ||
      cudaMemsetAsync(m->force_next, 0xFF, B * 4, s) != cudaSuccess ||
      cudaMemsetAsync(m->log, 0xFF, static_cast<size_t>(B) * D.cap * 4, s) != cudaSuccess ||
      cudaMemsetAsync(m->x16, 0, static_cast<size_t>(B) * d * 2, s) != cudaSuccess ||
      cudaMemsetAsync(m->bias, 0, static_cast<size_t>(L) * m->qkv_rows * 2, s) != cudaSuccess)
    return bail(fail(AGXC_ECUDA, "model: initial memset failed"));
  // gains default to 1.0 (fp16 0x3C00)
  {
    std::vector<uint16_t> ones(std::max({static_cast<size_t>(L) * 2 * d, static_cast<size_t>(d),
                                         static_cast<size_t>(L) * 2 * hd}), 0x3C00);
    if (cudaMemcpy(m->gains, ones.data(), static_cast<size_t>(L) * 2 * d * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->final_gain, ones.data(), static_cast<size_t>(d) * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->qk_gains, ones.data(), static_cast<size_t>(L) * 2 * hd * 2, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(AGXC_ECUDA, "model: gain upload failed"));
  }
  // RoPE tables: angle p * theta^(-2i/hd) in double, cos/sin rounded once to fp32 (assemble.py:665-668)
  {
    const int half = hd / 2;
    std::vector<float> c(static_cast<size_t>(D.cap) * half), sn(static_cast<size_t>(D.cap) * half);
    for (int p = 0; p < D.cap; ++p)
      for (int i = 0; i < half; ++i) {
        const double inv = std::pow(static_cast<double>(D.rope_theta), -(2.0 * i) / hd);
        const double ang = static_cast<double>(p) * inv;
        c[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(ang));
        sn[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(ang));
      }
    if (cudaMemcpy(m->cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(AGXC_ECUDA, "model: rope table upload failed"));
  }
  if (cudaEventCreate(&m->ev0) != cudaSuccess || cudaEventCreate(&m->ev1) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->ev_pipe[0], cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->ev_pipe[1], cudaEventDisableTiming) != cudaSuccess)
    return bail(fail(AGXC_ECUDA, "model: event create failed"));
  if (cudaStreamSynchronize(s) != cudaSuccess) return bail(fail(AGXC_ECUDA, "model: setup sync failed"));
  if (T > 1) {  // collective: every rank gets here; one warm-up of each collective before any graph capture
    if ((rc = dalloc_t(m, &m->amax, static_cast<size_t>(2) * B))) return bail(rc);
    if ((rc = dalloc_t(m, &m->amax_all, static_cast<size_t>(2) * B * T))) return bail(rc);
    if ((rc = tp_comm_create(T, m->tp_rank, G.tp_id, &m->comm))) return bail(rc);
    if (cudaMemsetAsync(m->ybuf, 0, static_cast<size_t>(B) * d * 4, s) != cudaSuccess ||
        cudaMemsetAsync(m->amax, 0, static_cast<size_t>(2) * B * 4, s) != cudaSuccess)
      return bail(fail(AGXC_ECUDA, "model: memset"));
    if ((rc = tp_allreduce_f32(m->comm, m->ybuf, static_cast<size_t>(B) * d, s)) ||
        (rc = tp_allgather_u32(m->comm, m->amax, m->amax_all, static_cast<size_t>(2) * B, s)))
      return bail(rc);
    if (cudaEventRecord(m->ev1, s) != cudaSuccess) return bail(fail(AGXC_ECUDA, "model: event record"));
    if ((rc = wait_done(m, m->ev1))) return bail(rc);
    if ((rc = tp_peer_setup(m))) return bail(rc);
  }
  *out = m;
  return 0;
}

int model_set_pack(agxc_model* m, int layer, int role, const void* packed, const void* scales, const void* biases,
                   int on_device) {
  const agxc_model_desc& D = m->d;
  if (role != AGXC_ROLE_HEAD && (layer < 0 || layer >= D.n_layers)) return fail(AGXC_EINVAL, "set_pack: bad layer");
  agxc_pack* dst = nullptr;
  int n = 0, k = 0, stride = 1, offset = 0, rope_hd = 0;
  switch (role) {
    case AGXC_ROLE_QKV: dst = &m->qkv[layer]; n = m->qkv_rows; k = D.d_model; rope_hd = D.head_dim; break;
    case AGXC_ROLE_WO: dst = &m->wo[layer]; n = D.d_model; k = m->attn_dim; break;
    case AGXC_ROLE_GATE: dst = &m->gu[layer]; n = D.ffn; k = D.d_model; stride = 2; offset = 0; break;
    case AGXC_ROLE_UP: dst = &m->gu[layer]; n = D.ffn; k = D.d_model; stride = 2; offset = 1; break;
    case AGXC_ROLE_DOWN: dst = &m->down[layer]; n = D.d_model; k = D.ffn; break;
    case AGXC_ROLE_HEAD: dst = &m->head; n = D.vocab; k = D.d_model; break;
    default: return fail(AGXC_EINVAL, "set_pack: unknown role");
  }
  cudaStream_t s = m->ctx->stream;
  const size_t pb = static_cast<size_t>(n) * k * D.bits / 8, sbb = static_cast<size_t>(n) * (k / 64) * 2;
  const void* dp = packed;
  const void* ds = scales;
  const void* db = biases;
  void* tmp = nullptr;
  if (!on_device) {
    AGXC_CUDA(cudaMalloc(&tmp, pb + 2 * sbb));
    uint8_t* t = static_cast<uint8_t*>(tmp);
    AGXC_CUDA(cudaMemcpy(t, packed, pb, cudaMemcpyHostToDevice));
    AGXC_CUDA(cudaMemcpy(t + pb, scales, sbb, cudaMemcpyHostToDevice));
    AGXC_CUDA(cudaMemcpy(t + pb + sbb, biases, sbb, cudaMemcpyHostToDevice));
    dp = t; ds = t + pb; db = t + pb + sbb;
  }
  int rc = launch_relayout(static_cast<const uint32_t*>(dp), static_cast<const uint16_t*>(ds),
                           static_cast<const uint16_t*>(db), n, k, D.bits, dst->tiles, dst->sb, stride, offset, s,
                           rope_hd);
  cudaError_t e = cudaStreamSynchronize(s);
  if (tmp) cudaFree(tmp);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "set_pack sync");
  return 0;
}

int model_set_vector(agxc_model* m, int layer, int which, const void* data, size_t bytes, int on_device) {
  const agxc_model_desc& D = m->d;
  void* dst = nullptr;
  size_t want = 0;
  switch (which) {
    case AGXC_VEC_ATTN_GAIN: dst = m->gains + static_cast<size_t>(layer) * 2 * D.d_model; want = D.d_model * 2; break;
    case AGXC_VEC_FFN_GAIN:
      dst = m->gains + static_cast<size_t>(layer) * 2 * D.d_model + D.d_model; want = D.d_model * 2; break;
    case AGXC_VEC_QKV_BIAS: dst = m->bias + static_cast<size_t>(layer) * m->qkv_rows; want = m->qkv_rows * 2; break;
    case AGXC_VEC_FINAL_GAIN: dst = m->final_gain; want = D.d_model * 2; break;
    case AGXC_VEC_EMBED: dst = m->embed; want = static_cast<size_t>(m->vt) * D.d_model * 2; break;
    case AGXC_VEC_Q_NORM:
      dst = m->qk_gains + static_cast<size_t>(layer) * 2 * D.head_dim; want = D.head_dim * 2; break;
    case AGXC_VEC_K_NORM:
      dst = m->qk_gains + static_cast<size_t>(layer) * 2 * D.head_dim + D.head_dim; want = D.head_dim * 2; break;
    default: return fail(AGXC_EINVAL, "set_vector: unknown vector");
  }
  if ((which <= AGXC_VEC_QKV_BIAS || which == AGXC_VEC_Q_NORM || which == AGXC_VEC_K_NORM) &&
      (layer < 0 || layer >= D.n_layers))
    return fail(AGXC_EINVAL, "set_vector: layer");
  if (bytes != want) return fail(AGXC_EINVAL, "set_vector: expected " + std::to_string(want) + " bytes");
  AGXC_CUDA(cudaMemcpy(dst, data, bytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  return 0;
}

__global__ void embed_rows_kernel(const __half* emb, int d, const uint32_t* toks, int n, __half* out) {
  const int b = blockIdx.x;
  if (b >= n) return;
  const uint32_t t = toks[b];
  for (int i = threadIdx.x; i < d; i += blockDim.x) out[static_cast<size_t>(b) * d + i] = emb[static_cast<size_t>(t) * d + i];
}

int model_start(agxc_model* m, int b, const int32_t* prompt, int n) {
  const agxc_model_desc& D = m->d;
  if (b < 0 || b >= D.batch) return fail(AGXC_EINVAL, "start: sequence index");
  if (n < 1 || n > D.cap) return fail(AGXC_EINVAL, "start: prompt length must be 1..cap");
  for (int i = 0; i < n; ++i)
    if (prompt[i] < 0 || prompt[i] >= m->vt) return fail(AGXC_EINVAL, "start: token id out of range");
  cudaStream_t s = m->ctx->stream;
  const size_t seq_kv = static_cast<size_t>(D.n_kv_heads) * D.cap * D.head_dim;
  for (int l = 0; l < D.n_layers; ++l) {
    const size_t off = (static_cast<size_t>(l) * D.batch + b) * seq_kv;
    AGXC_CUDA(cudaMemsetAsync(m->kcache + off, 0, seq_kv * 2, s));
    AGXC_CUDA(cudaMemsetAsync(m->vcache + off, 0, seq_kv * 2, s));
  }
  std::vector<uint32_t> log(D.cap, agxc::kTokenUnset);
  for (int i = 0; i < n; ++i) log[i] = static_cast<uint32_t>(prompt[i]);
  AGXC_CUDA(cudaMemcpyAsync(m->log + static_cast<size_t>(b) * D.cap, log.data(), D.cap * 4, cudaMemcpyHostToDevice, s));
  const uint32_t zero = 0;
  AGXC_CUDA(cudaMemcpyAsync(m->q0 + b, &zero, 4, cudaMemcpyHostToDevice, s));
  AGXC_CUDA(cudaMemcpyAsync(m->x16 + static_cast<size_t>(b) * D.d_model,
                            m->embed + static_cast<size_t>(prompt[0]) * D.d_model, D.d_model * 2,
                            cudaMemcpyDeviceToDevice, s));
  AGXC_CUDA(cudaStreamSynchronize(s));
  return 0;
}

constexpr int kPrefillRows = 256;  // rows per prefill chunk (the tensor-core GEMM's largest row count)
constexpr int kVerifyRows = 16;    // rows of the speculative verify step: the current token and up to 15 drafts

__global__ void positions_kernel(uint32_t* pos, int p0, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] = static_cast<uint32_t>(p0 + i);
}

// K ranges of a pack's GEMM: split until the 128-row tiles fill the SMs (a divisor of the groups)
int qmm_ksplit(const agxc_ctx* ctx, const agxc_pack& pk) {
  const int tiles = pk.n / 128, G = pk.k / 64;
  int ks = 1;
  while (tiles * ks * 2 <= ctx->num_sms && G % (ks * 2) == 0) ks *= 2;
  return ks;
}

// Y [rows][ld] = X [rows][K] W^T on the tensor cores; with several K ranges their partial sums go to `part`
// ([ks][rows][N]) and the last range of each tile adds them up in order.
int run_qmm(agxc_model* m, const agxc_pack& pk, const __half* x, int rows, float* y, int ld, cudaStream_t s,
            float* part, const QmmPush* push) {
  return launch_qmm(m->ctx, &pk, x, rows, y, ld, qmm_ksplit(m->ctx, pk), s, push, part, m->tile_ctr, m->pdl ? 1 : 0);
}

// The GEMM for consumers that add the K ranges themselves: split K writes the ranges' partial sums to `part` and
// nothing else (no summing pass); one range writes the finished rows to ybuf.
int gemm_rows(agxc_model* m, const agxc_pack& pk, const __half* x, int rows, float* ybuf, int ld, float* part,
              cudaStream_t s, YRows* out) {
  const int ks = qmm_ksplit(m->ctx, pk);
  if (ks > 1) {
    *out = YRows{part, pk.n, ks, static_cast<size_t>(rows) * pk.n};
    return launch_qmm(m->ctx, &pk, x, rows, nullptr, pk.n, ks, s, nullptr, part, nullptr, m->pdl ? 1 : 0);
  }
  *out = YRows{ybuf, ld, 1, 0};
  return launch_qmm(m->ctx, &pk, x, rows, ybuf, ld, 1, s, nullptr, nullptr, nullptr, m->pdl ? 1 : 0);
}

// The tile counters (the widest pack's tiles) and a partial-sum scratch for `rows` activation rows of any of the
// model's split-K GEMMs.
int qmm_scratch(agxc_model* m, int rows, float** part) {
  const agxc_model_desc& D = m->d;
  size_t need = 0;
  auto take = [&](const agxc_pack& pk) {
    const int ks = qmm_ksplit(m->ctx, pk);
    if (ks > 1) need = std::max(need, static_cast<size_t>(ks) * rows * pk.n);
  };
  for (int l = 0; l < D.n_layers; ++l) {
    take(m->qkv[l]);
    take(m->wo[l]);
    take(m->gu[l]);
    take(m->down[l]);
  }
  take(m->head);
  if (!m->tile_ctr) {
    const size_t tiles = std::max({static_cast<size_t>(m->head.n), static_cast<size_t>(2) * D.ffn,
                                   static_cast<size_t>(m->qkv_rows), static_cast<size_t>(D.d_model)}) / 128 + 1;
    if (int rc = dalloc_t(m, &m->tile_ctr, tiles)) return rc;
    AGXC_CUDA(cudaMemset(m->tile_ctr, 0, tiles * 4));
  }
  return dalloc_t(m, part, std::max<size_t>(need, 64));
}

int prefill_buffers(agxc_model* m) {
  if (m->pf_x16) return 0;
  const agxc_model_desc& D = m->d;
  const size_t R = kPrefillRows, d = D.d_model, F = D.ffn;
  const size_t yn = std::max({static_cast<size_t>(m->qkv_rows), 2 * F, d});
  int rc;
  if ((rc = dalloc_t(m, &m->pf_x16, R * d)) || (rc = dalloc_t(m, &m->pf_h, R * d)) ||
      (rc = dalloc_t(m, &m->pf_xn16, R * d)) || (rc = dalloc_t(m, &m->pf_y, R * yn)) ||
      (rc = dalloc_t(m, &m->pf_q16, R * m->attn_dim)) || (rc = dalloc_t(m, &m->pf_attn, R * m->attn_dim)) ||
      (rc = dalloc_t(m, &m->pf_act, R * F)) || (rc = dalloc_t(m, &m->pf_pos, R)) ||
      (rc = dalloc_t(m, &m->pf_tok, static_cast<size_t>(D.cap))) || (rc = qmm_scratch(m, kPrefillRows, &m->pf_part)))
    return rc;
  // rows past a chunk's end are GEMM padding: they start at zero and only ever hold finite values
  AGXC_CUDA(cudaMemset(m->pf_x16, 0, R * d * 2));
  AGXC_CUDA(cudaMemset(m->pf_attn, 0, R * m->attn_dim * 2));
  AGXC_CUDA(cudaMemset(m->pf_act, 0, R * F * 2));
  return 0;
}

// Mc rows of sequence b at positions p0 .. p0 + Mc - 1 (tokens at m->pf_tok[p0 ..]) through every layer on the
// tensor-core GEMMs: RMSNorm rows -> qkv GEMM -> RoPE + append (the rows' K/V into b's cache) -> causal attention
// over the cache rows 0 .. p0 - 1 and the rows before each row -> o_proj GEMM -> add16 -> RMSNorm rows -> gate/up GEMM
// -> SwiGLU -> down GEMM -> add32_to16. The rows' last-layer x16 stays in m->pf_x16.
int rows_pass(agxc_model* m, int b, int p0, int Mc, cudaStream_t s, int* launches) {
  const agxc_model_desc& D = m->d;
  const int d = D.d_model, F = D.ffn, H = D.n_heads, KVH = D.n_kv_heads, hd = D.head_dim;
  const size_t layer_kv = static_cast<size_t>(D.batch) * KVH * D.cap * hd;
  const float qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(hd)));
  const int Mp = std::max(32, (Mc + 15) / 16 * 16);
  YRows yr;
  int rc = 0;
  embed_rows_kernel<<<Mc, 256, 0, s>>>(m->embed, d, m->pf_tok + p0, Mc, m->pf_x16);
  positions_kernel<<<(Mc + 255) / 256, 256, 0, s>>>(m->pf_pos, p0, Mc);
  AGXC_CUDA(cudaGetLastError());
  *launches += 2;
  for (int l = 0; l < D.n_layers && !rc; ++l) {
    const __half* g1 = m->gains + static_cast<size_t>(l) * 2 * d;
    const __half* bias = D.qkv_bias ? m->bias + static_cast<size_t>(l) * m->qkv_rows : nullptr;
    __half* kc = m->kcache + l * layer_kv;
    __half* vc = m->vcache + l * layer_kv;
    if ((rc = launch_rmsnorm(m->pf_x16, 0, Mp, d, g1, D.eps, m->pf_xn16, s)) ||
        (rc = gemm_rows(m, m->qkv[l], m->pf_xn16, Mp, m->pf_y, m->qkv_rows, m->pf_part, s, &yr)) ||
        (rc = launch_rope_append(yr, m->qkv_rows, bias, m->cos_t, m->sin_t, m->pf_pos, H, KVH, hd, D.cap, qscale,
                                 m->pf_q16, kc, vc, Mc, s, b, qk_gains_of(m, l), D.eps)) ||
        (rc = launch_prefill_attention(m->pf_q16, kc, vc, Mc, p0, H, KVH, hd, D.cap, b, m->pf_attn, s)) ||
        (rc = gemm_rows(m, m->wo[l], m->pf_attn, Mp, m->pf_y, d, m->pf_part, s, &yr)) ||
        (rc = launch_residual16(yr, m->pf_x16, m->pf_h, d, Mp, s)) ||
        (rc = launch_rmsnorm(m->pf_h, 1, Mp, d, g1 + d, D.eps, m->pf_xn16, s)) ||
        (rc = gemm_rows(m, m->gu[l], m->pf_xn16, Mp, m->pf_y, 2 * F, m->pf_part, s, &yr)) ||
        (rc = launch_swiglu(yr, m->pf_act, F, Mp, s)) ||
        (rc = gemm_rows(m, m->down[l], m->pf_act, Mp, m->pf_y, d, m->pf_part, s, &yr)) ||
        (rc = launch_residual32(yr, m->pf_h, m->pf_x16, d, Mp, s)))
      break;
    *launches += 11;
  }
  return rc;
}

// Start sequence b with its prompt and run positions 0 .. n-2 as the prefill section: chunks of up to 256 rows, each
// layer as RMSNorm rows -> qkv GEMM -> RoPE + append (the chunk's K/V rows into b's cache) -> causal attention of the
// chunk -> o_proj GEMM -> add16 -> RMSNorm rows -> gate/up GEMM -> SwiGLU -> down GEMM -> add32_to16 (the reference's
// prefill steps, agxforge/inference/prefill.py:8-14). Then q0 = n-1 and x = embedding(prompt[n-1]): the next decode
// step runs position n-1 and chooses the first generated token, as after n-1 teacher-forced decode steps.
int model_prefill(agxc_model* m, int b, const int32_t* prompt, int n, agxc_timing* t) {
  const agxc_model_desc& D = m->d;
  if (m->comm) return fail(AGXC_EUNSUPPORTED, "prefill: tensor-parallel models feed the prompt through decode steps");
  if (m->qkv_rows % 128 || D.d_model % 128 || (2 * D.ffn) % 128)
    return fail(AGXC_EUNSUPPORTED, "prefill: needs qkv rows, d_model and 2 x ffn multiples of 128");
  if (int rc = model_start(m, b, prompt, n)) return rc;
  if (int rc = prefill_buffers(m)) return rc;
  cudaStream_t s = m->ctx->stream;
  const auto h0 = std::chrono::steady_clock::now();
  AGXC_CUDA(cudaEventRecord(m->ev0, s));
  const int total = n - 1;
  const int d = D.d_model;
  int rc = 0, launches = 0;
  if (total > 0) {
    std::vector<uint32_t> tok(prompt, prompt + n);
    AGXC_CUDA(cudaMemcpyAsync(m->pf_tok, tok.data(), static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, s));
  }
  for (int p0 = 0; p0 < total && !rc; p0 += kPrefillRows) rc = rows_pass(m, b, p0, std::min(kPrefillRows, total - p0), s, &launches);
  if (rc) return rc;
  // the last prompt token is the next decode step's input, at position n-1
  const uint32_t q0 = static_cast<uint32_t>(n - 1);
  AGXC_CUDA(cudaMemcpyAsync(m->q0 + b, &q0, 4, cudaMemcpyHostToDevice, s));
  AGXC_CUDA(cudaMemcpyAsync(m->x16 + static_cast<size_t>(b) * d, m->embed + static_cast<size_t>(prompt[n - 1]) * d,
                            static_cast<size_t>(d) * 2, cudaMemcpyDeviceToDevice, s));
  AGXC_CUDA(cudaEventRecord(m->ev1, s));
  AGXC_CUDA(cudaEventSynchronize(m->ev1));
  if (t) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, m->ev0, m->ev1);
    t->gpu_ms = ms;
    t->host_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - h0).count();
    t->launches_per_step = launches;
  }
  uint32_t err = 0;
  AGXC_CUDA(cudaMemcpy(&err, m->ctx->err_dev, 4, cudaMemcpyDeviceToHost));
  if (err) {
    const uint32_t zero = 0;
    cudaMemcpy(m->ctx->err_dev, &zero, 4, cudaMemcpyHostToDevice);
    if (fused_active(m)) fused_reset(m);  // a step that gave up leaves its counters part-way
    return fail(err & kErrMbarTimeout ? AGXC_ETIMEOUT : AGXC_ECORRUPT, "prefill: device error word " + std::to_string(err));
  }
  return 0;
}

// The speculative verify step (the reference's verify section, agxforge/inference/assemble.py:244-253,747-803, driven
// by tools/g17specgen.m): the current token (log[q0], whose embedding is the next decode input) and n_draft drafted
// tokens as rows at positions q0 .. q0 + n_draft through the row pass (their K/V rows into the cache), the final
// norm, the head and each row's first maximum. Row i's choice is the token at position q0 + i + 1 — the logged one
// where the log fixes it (the generation step's rule), else the maximum. The drafts are accepted while they equal the
// choices; the accepted drafts and the choice after them are emitted and committed: logged, q0 advanced past them,
// x16 = the last one's embedding. Rows past the accepted ones leave K/V rows the next steps overwrite.
int model_verify(agxc_model* m, int b, const int32_t* draft, int n_draft, int32_t* emitted, int32_t* n_emitted,
                 float* logits_out) {
  const agxc_model_desc& D = m->d;
  if (m->comm) return fail(AGXC_EUNSUPPORTED, "verify: a single-device model");
  if (m->qkv_rows % 128 || D.d_model % 128 || (2 * D.ffn) % 128 || D.vocab % 128)
    return fail(AGXC_EUNSUPPORTED, "verify: needs qkv rows, d_model, 2 x ffn and vocab multiples of 128");
  if (b < 0 || b >= D.batch) return fail(AGXC_EINVAL, "verify: sequence index");
  if (n_draft < 0 || n_draft > kVerifyRows - 1) return fail(AGXC_EINVAL, "verify: 0 to 15 drafted tokens");
  for (int i = 0; i < n_draft; ++i)
    if (draft[i] < 0 || draft[i] >= m->vt) return fail(AGXC_EINVAL, "verify: draft token out of range");
  if (int rc = prefill_buffers(m)) return rc;
  cudaStream_t s = m->ctx->stream;
  AGXC_CUDA(cudaStreamSynchronize(s));
  uint32_t q0 = 0;
  AGXC_CUDA(cudaMemcpy(&q0, m->q0 + b, 4, cudaMemcpyDeviceToHost));
  const int R = n_draft + 1;
  if (static_cast<int>(q0) + R >= D.cap) return fail(AGXC_EINVAL, "verify: the rows would pass the cap");
  std::vector<uint32_t> log(R + 1);
  AGXC_CUDA(cudaMemcpy(log.data(), m->log + static_cast<size_t>(b) * D.cap + q0, (R + 1) * 4, cudaMemcpyDeviceToHost));
  if (log[0] == kTokenUnset || log[0] >= static_cast<uint32_t>(m->vt))
    return fail(AGXC_EINVAL, "verify: no current token at q0 (start the sequence first)");
  std::vector<uint32_t> rows(R);
  rows[0] = log[0];
  for (int i = 0; i < n_draft; ++i) rows[i + 1] = static_cast<uint32_t>(draft[i]);
  if (!m->sp_y) {
    int rc;
    if ((rc = dalloc_t(m, &m->sp_y, static_cast<size_t>(32) * D.vocab)) || (rc = dalloc_t(m, &m->sp_amax, 32)))
      return rc;
  }
  AGXC_CUDA(cudaMemcpyAsync(m->pf_tok + q0, rows.data(), R * 4, cudaMemcpyHostToDevice, s));
  int launches = 0;
  int rc = rows_pass(m, b, static_cast<int>(q0), R, s, &launches);
  YRows yr;
  if (!rc) rc = launch_rmsnorm(m->pf_x16, 0, 32, D.d_model, m->final_gain, D.eps, m->pf_xn16, s);
  if (!rc) rc = gemm_rows(m, m->head, m->pf_xn16, 32, m->sp_y, D.vocab, m->pf_part, s, &yr);
  if (!rc) rc = launch_rows_argmax(yr, D.vocab, R, nullptr, m->sp_amax, s);
  if (rc) return rc;
  std::vector<int32_t> amax(R);
  AGXC_CUDA(cudaMemcpyAsync(amax.data(), m->sp_amax, R * 4, cudaMemcpyDeviceToHost, s));
  if (logits_out) {
    if (yr.ks > 1) {   // the head's split-K slices summed into the output rows
      float* dev = m->sp_y;
      if ((rc = launch_rows_argmax(yr, D.vocab, R, dev, m->sp_amax, s))) return rc;
      AGXC_CUDA(cudaMemcpyAsync(logits_out, dev, static_cast<size_t>(R) * D.vocab * 4, cudaMemcpyDeviceToHost, s));
    } else {
      AGXC_CUDA(cudaMemcpyAsync(logits_out, m->sp_y, static_cast<size_t>(R) * D.vocab * 4, cudaMemcpyDeviceToHost, s));
    }
  }
  AGXC_CUDA(cudaStreamSynchronize(s));
  uint32_t err = 0;
  AGXC_CUDA(cudaMemcpy(&err, m->ctx->err_dev, 4, cudaMemcpyDeviceToHost));
  if (err) {
    const uint32_t zero = 0;
    cudaMemcpy(m->ctx->err_dev, &zero, 4, cudaMemcpyHostToDevice);
    return fail(err & kErrMbarTimeout ? AGXC_ETIMEOUT : AGXC_ECORRUPT, "verify: device error word " + std::to_string(err));
  }
  // accept: choice i = the logged token at q0 + i + 1 where set, else row i's maximum
  int k = 0;
  std::vector<uint32_t> out;
  for (int i = 0; i < R; ++i) {
    const uint32_t choice = log[i + 1] != kTokenUnset ? log[i + 1] : static_cast<uint32_t>(amax[i]);
    out.push_back(choice);
    if (i < n_draft && static_cast<uint32_t>(draft[i]) == choice) {
      ++k;
      continue;
    }
    break;
  }
  // commit: log the emitted tokens, q0 past them, x16 = the last one's embedding
  const uint32_t nq0 = q0 + static_cast<uint32_t>(out.size());
  AGXC_CUDA(cudaMemcpy(m->log + static_cast<size_t>(b) * D.cap + q0 + 1, out.data(), out.size() * 4,
                       cudaMemcpyHostToDevice));
  AGXC_CUDA(cudaMemcpy(m->q0 + b, &nq0, 4, cudaMemcpyHostToDevice));
  AGXC_CUDA(cudaMemcpy(m->x16 + static_cast<size_t>(b) * D.d_model, m->embed + static_cast<size_t>(out.back()) * D.d_model,
                       static_cast<size_t>(D.d_model) * 2, cudaMemcpyDeviceToDevice));
  for (size_t i = 0; i < out.size(); ++i) emitted[i] = static_cast<int32_t>(out[i]);
  *n_emitted = static_cast<int32_t>(out.size());
  return 0;
}

int model_force(agxc_model* m, int b, int pos, const int32_t* tokens, int n) {
  const agxc_model_desc& D = m->d;
  if (b < 0 || b >= D.batch || pos < 0 || n < 0 || pos + n > D.cap) return fail(AGXC_EINVAL, "force: range");
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->vt) return fail(AGXC_EINVAL, "force: token id out of range");
  AGXC_CUDA(cudaMemcpy(m->log + static_cast<size_t>(b) * D.cap + pos, tokens, static_cast<size_t>(n) * 4,
                       cudaMemcpyHostToDevice));
  return 0;
}

__global__ void fill_normal_kernel(__half* dst, size_t n, uint64_t seed) {
  // Box-Muller over a counter-based hash (splitmix64); a stand-in history, not a parity input
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (i + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  const float u1 = (static_cast<float>(z >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = static_cast<float>((z >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
  dst[i] = __float2half_rn(sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2));
}

int model_fill_history(agxc_model* m, int b, int n, uint64_t seed) {
  const agxc_model_desc& D = m->d;
  if (b < 0 || b >= D.batch || n < 0 || n >= D.cap) return fail(AGXC_EINVAL, "fill_history: range");
  cudaStream_t s = m->ctx->stream;
  const size_t row = static_cast<size_t>(n) * D.head_dim;
  for (int l = 0; l < D.n_layers; ++l)
    for (int kv = 0; kv < D.n_kv_heads; ++kv) {
      const size_t off = ((static_cast<size_t>(l) * D.batch + b) * D.n_kv_heads + kv) * D.cap * D.head_dim;
      const uint64_t g = static_cast<uint64_t>(m->tp_rank) * D.n_kv_heads + kv;  // the global KV head
      if (row) {
        fill_normal_kernel<<<static_cast<unsigned>((row + 255) / 256), 256, 0, s>>>(m->kcache + off, row,
                                                                                   seed * 131 + l * 17 + g * 2);
        fill_normal_kernel<<<static_cast<unsigned>((row + 255) / 256), 256, 0, s>>>(m->vcache + off, row,
                                                                                   seed * 131 + l * 17 + g * 2 + 1);
      }
    }
  AGXC_CUDA(cudaGetLastError());
  std::mt19937_64 rng(seed);
  std::vector<uint32_t> log(D.cap, agxc::kTokenUnset);
  for (int i = 0; i <= n; ++i) log[i] = static_cast<uint32_t>(rng() % static_cast<uint64_t>(m->vt));
  AGXC_CUDA(cudaMemcpyAsync(m->log + static_cast<size_t>(b) * D.cap, log.data(), D.cap * 4, cudaMemcpyHostToDevice, s));
  const uint32_t q0 = static_cast<uint32_t>(n);
  AGXC_CUDA(cudaMemcpyAsync(m->q0 + b, &q0, 4, cudaMemcpyHostToDevice, s));
  AGXC_CUDA(cudaMemcpyAsync(m->x16 + static_cast<size_t>(b) * D.d_model,
                            m->embed + static_cast<size_t>(log[n]) * D.d_model, D.d_model * 2, cudaMemcpyDeviceToDevice,
                            s));
  AGXC_CUDA(cudaStreamSynchronize(s));
  return 0;
}

int model_decode(agxc_model* m, int steps, const int32_t* forced_in, int32_t* tokens_out, float* logits_out,
                 int sync_each, agxc_timing* t) {
  const agxc_model_desc& D = m->d;
  if (steps < 0) return fail(AGXC_EINVAL, "decode: steps");
  if (sync_each < 0 || sync_each > 2) return fail(AGXC_EINVAL, "decode: sync_each 0, 1 or 2");
  if (forced_in) {
    for (size_t i = 0; i < static_cast<size_t>(steps) * D.batch; ++i) {
      const uint32_t f = static_cast<uint32_t>(forced_in[i]);
      if (f != kTokenUnset && f >= static_cast<uint32_t>(m->vt))
        return fail(AGXC_EINVAL, "decode: forced token out of range");
    }
    const size_t nf = static_cast<size_t>(std::max(steps, 1)) * D.batch;
    if (m->h_force_n < nf) {
      if (m->h_force) cudaFreeHost(m->h_force);
      m->h_force = nullptr;
      AGXC_CUDA(cudaMallocHost(&m->h_force, nf * 4));
      m->h_force_n = nf;
    }
    std::memcpy(m->h_force, forced_in, static_cast<size_t>(steps) * D.batch * 4);
  }
  if (logits_out && !D.keep_logits) return fail(AGXC_EINVAL, "decode: logits_out needs keep_logits");
  int rc = ensure_graph(m);
  if (rc) return rc;
  if (m->comm && m->tp_fused && m->tp_fused_ok) m->tp_fused_ran = 1;
  cudaStream_t s = m->ctx->stream;
  const size_t need = static_cast<size_t>(std::max(steps, 1)) * D.batch;
  if (tokens_out && m->h_tok_n < need) {
    if (m->h_tok) cudaFreeHost(m->h_tok);
    m->h_tok = nullptr;
    AGXC_CUDA(cudaMallocHost(&m->h_tok, need * 4));
    m->h_tok_n = need;
  }
  const auto h0 = std::chrono::steady_clock::now();
  AGXC_CUDA(cudaEventRecord(m->ev0, s));
  for (int i = 0; i < steps; ++i) {
    if (forced_in)  // this step's input: one token per sequence (UNSET = choose), pinned host -> device
      AGXC_CUDA(cudaMemcpyAsync(m->force_next, m->h_force + static_cast<size_t>(i) * D.batch, D.batch * 4,
                                cudaMemcpyHostToDevice, s));
    AGXC_CUDA(cudaGraphLaunch(m->exec, s));
    if (tokens_out)
      AGXC_CUDA(cudaMemcpyAsync(m->h_tok + static_cast<size_t>(i) * D.batch, m->tok, D.batch * 4,
                                cudaMemcpyDeviceToHost, s));
    if (logits_out)
      AGXC_CUDA(cudaMemcpyAsync(logits_out + static_cast<size_t>(i) * D.batch * D.vocab, m->logits,
                                static_cast<size_t>(D.batch) * D.vocab * 4, cudaMemcpyDeviceToHost, s));
    if (sync_each == 2) {  // this step queued behind the previous one; wait for that one (its token is home)
      AGXC_CUDA(cudaEventRecord(m->ev_pipe[i & 1], s));
      if (i > 0 && (rc = wait_done(m, m->ev_pipe[(i - 1) & 1]))) return rc;
    } else if (sync_each) {
      AGXC_CUDA(cudaEventRecord(m->ev1, s));
      if ((rc = wait_done(m, m->ev1))) return rc;
    }
  }
  AGXC_CUDA(cudaEventRecord(m->ev1, s));
  if ((rc = wait_done(m, m->ev1))) return rc;
  const auto h1 = std::chrono::steady_clock::now();
  if (tokens_out) std::memcpy(tokens_out, m->h_tok, static_cast<size_t>(steps) * D.batch * 4);
  uint32_t err = 0;
  AGXC_CUDA(cudaMemcpy(&err, m->ctx->err_dev, 4, cudaMemcpyDeviceToHost));
  if (t) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, m->ev0, m->ev1);
    t->gpu_ms = ms;
    t->host_ms = std::chrono::duration<float, std::milli>(h1 - h0).count();
    t->launches_per_step = m->launches;
  }
  if (err) {
    const uint32_t zero = 0;
    cudaMemcpy(m->ctx->err_dev, &zero, 4, cudaMemcpyHostToDevice);
    if (fused_active(m)) fused_reset(m);  // a step that gave up leaves its counters part-way
    if (err & kErrMbarTimeout) return fail(AGXC_ETIMEOUT, "decode: a bounded device wait gave up");
    return fail(AGXC_ECORRUPT, "decode: device error word " + std::to_string(err));
  }
  return 0;
}

int model_profile(agxc_model* m, int steps, float* kind_ms, int32_t* kind_launches) {
  const int per_step = 5 * m->d.n_layers + 1;
  std::vector<cudaEvent_t> ev(2 * per_step, nullptr);
  for (auto& e : ev)
    if (cudaEventCreate(&e) != cudaSuccess) {
      for (auto& x : ev)
        if (x) cudaEventDestroy(x);
      return fail(AGXC_ECUDA, "profile: event create failed");
    }
  for (int k = 0; k < 6; ++k) { kind_ms[k] = 0.f; kind_launches[k] = 0; }
  cudaStream_t s = m->ctx->stream;
  const int saved_pdl = m->pdl;
  m->pdl = 0;  // events between launches: every kernel timed on its own
  if (m->comm && m->tp_fused && m->tp_fused_ok) m->tp_fused_ran = 1;
  int rc = 0;
  for (int i = 0; i < steps && !rc; ++i) {
    rc = enqueue_step(m, s, ev.data());
    if (rc) break;
    if (cudaEventRecord(m->ev1, s) != cudaSuccess || (rc = wait_done(m, m->ev1))) {
      if (!rc) rc = fail(AGXC_ECUDA, "profile: sync failed");
      break;
    }
    for (int j = 0; j < per_step; ++j) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev[2 * j], ev[2 * j + 1]);
      const int kind = j == per_step - 1 ? 5 : j % 5;
      kind_ms[kind] += ms;
      kind_launches[kind] += 1;
    }
  }
  m->pdl = saved_pdl;
  for (auto& e : ev) cudaEventDestroy(e);
  return rc;
}

void model_free(agxc_model* m) {
  if (!m) return;
  if (m->exec) cudaGraphExecDestroy(m->exec);
  if (m->graph) cudaGraphDestroy(m->graph);
  tp_peer_teardown(m);    // after the graphs, before the buffers the other ranks write (uses ev1)
  tp_comm_free(m->comm);  // after the graphs that hold its collectives
  if (m->ev0) cudaEventDestroy(m->ev0);
  if (m->ev1) cudaEventDestroy(m->ev1);
  for (cudaEvent_t e : m->ev_pipe)
    if (e) cudaEventDestroy(e);
  if (m->h_tok) cudaFreeHost(m->h_tok);
  if (m->h_force) cudaFreeHost(m->h_force);
  if (m->trace) cudaFree(m->trace);
  if (m->cta_trace) cudaFree(m->cta_trace);
  for (void* p : m->allocs) cudaFree(p);
  delete m;
}

}  // namespace agxc

// ---------------------------------------------------------------------------------------------- C ABI (model)
extern "C" {

int agxc_model_create(agxc_ctx* ctx, const agxc_model_desc* desc, agxc_model** out) {
  if (!ctx || !desc || !out) return agxc::fail(AGXC_EINVAL, "model_create: null argument");
  if (cudaSetDevice(ctx->device) != cudaSuccess) return agxc::fail(AGXC_ECUDA, "model_create: cudaSetDevice");
  return agxc::model_create(ctx, desc, out);
}

void agxc_model_free(agxc_model* m) { agxc::model_free(m); }

int agxc_model_set_pack(agxc_model* m, int layer, int role, const void* packed, const void* scales,
                        const void* biases, int on_device) {
  if (!m || !packed || !scales || !biases) return agxc::fail(AGXC_EINVAL, "set_pack: null argument");
  return agxc::model_set_pack(m, layer, role, packed, scales, biases, on_device);
}

int agxc_model_set_vector(agxc_model* m, int layer, int which, const void* data, size_t bytes, int on_device) {
  if (!m || !data) return agxc::fail(AGXC_EINVAL, "set_vector: null argument");
  return agxc::model_set_vector(m, layer, which, data, bytes, on_device);
}

int64_t agxc_model_weight_bytes(const agxc_model* m) {
  if (!m) return 0;
  int64_t t = m->head.bytes();
  for (int l = 0; l < m->d.n_layers; ++l) t += m->qkv[l].bytes() + m->wo[l].bytes() + m->gu[l].bytes() + m->down[l].bytes();
  return t;
}

int agxc_model_start(agxc_model* m, int b, const int32_t* prompt, int n) {
  if (!m || !prompt) return agxc::fail(AGXC_EINVAL, "start: null argument");
  return agxc::model_start(m, b, prompt, n);
}

int agxc_model_prefill(agxc_model* m, int b, const int32_t* prompt, int n, agxc_timing* t) {
  if (!m || !prompt) return agxc::fail(AGXC_EINVAL, "prefill: null argument");
  return agxc::model_prefill(m, b, prompt, n, t);
}

int agxc_model_verify(agxc_model* m, int b, const int32_t* draft, int n_draft, int32_t* emitted, int32_t* n_emitted,
                      float* logits_out) {
  if (!m || (!draft && n_draft) || !emitted || !n_emitted) return agxc::fail(AGXC_EINVAL, "verify: null argument");
  return agxc::model_verify(m, b, draft, n_draft, emitted, n_emitted, logits_out);
}

int agxc_model_force(agxc_model* m, int b, int pos, const int32_t* tokens, int n) {
  if (!m || (!tokens && n)) return agxc::fail(AGXC_EINVAL, "force: null argument");
  return agxc::model_force(m, b, pos, tokens, n);
}

int agxc_model_fill_history(agxc_model* m, int b, int n, uint64_t seed) {
  if (!m) return agxc::fail(AGXC_EINVAL, "fill_history: null model");
  return agxc::model_fill_history(m, b, n, seed);
}

int agxc_decode(agxc_model* m, int steps, const int32_t* forced_in, int32_t* tokens_out, float* logits_out,
                int sync_each, agxc_timing* t) {
  if (!m) return agxc::fail(AGXC_EINVAL, "decode: null model");
  return agxc::model_decode(m, steps, forced_in, tokens_out, logits_out, sync_each, t);
}

int agxc_model_state(agxc_model* m, int b, uint32_t* q0, uint32_t* log) {
  if (!m || b < 0 || b >= m->d.batch) return agxc::fail(AGXC_EINVAL, "state: bad argument");
  if (q0) AGXC_CUDA(cudaMemcpy(q0, m->q0 + b, 4, cudaMemcpyDeviceToHost));
  if (log) AGXC_CUDA(cudaMemcpy(log, m->log + static_cast<size_t>(b) * m->d.cap, m->d.cap * 4, cudaMemcpyDeviceToHost));
  return 0;
}

namespace {

struct StateHeader {            // 64 bytes, little-endian
  char magic[4];                // "AGXS"
  uint32_t version;             // 1
  uint32_t layers, kv_heads, head_dim, d_model, vocab, cap;
  uint32_t q0;                  // the next step's position; K/V rows 0 .. q0-1 follow
  uint32_t force_next;          // a pending forced token (0xFFFFFFFF = none)
  uint32_t reserved[6];
};
static_assert(sizeof(StateHeader) == 64, "the state header is 64 bytes");

size_t state_bytes(const agxc_model* m, uint32_t q0) {
  const agxc_model_desc& D = m->d;
  return sizeof(StateHeader) + static_cast<size_t>(D.cap) * 4 + static_cast<size_t>(D.d_model) * 2 +
         2 * static_cast<size_t>(D.n_layers) * D.n_kv_heads * q0 * D.head_dim * 2;
}

// (layer, KV head) row block of sequence b in the cache [L][B][KVH][cap][hd]
size_t kv_off(const agxc_model* m, int l, int b, int kv) {
  const agxc_model_desc& D = m->d;
  return ((static_cast<size_t>(l) * D.batch + b) * D.n_kv_heads + kv) * D.cap * D.head_dim;
}

}  // namespace

int64_t agxc_model_state_bytes(agxc_model* m, int b) {
  if (!m || b < 0 || b >= m->d.batch) return agxc::fail(AGXC_EINVAL, "state_bytes: bad argument");
  uint32_t q0 = 0;
  AGXC_CUDA(cudaStreamSynchronize(m->ctx->stream));
  AGXC_CUDA(cudaMemcpy(&q0, m->q0 + b, 4, cudaMemcpyDeviceToHost));
  return static_cast<int64_t>(state_bytes(m, q0));
}

int agxc_model_state_save(agxc_model* m, int b, void* out, size_t capacity, size_t* written) {
  if (!m || !out || b < 0 || b >= m->d.batch) return agxc::fail(AGXC_EINVAL, "state_save: bad argument");
  if (m->tp > 1) return agxc::fail(AGXC_EUNSUPPORTED, "state_save: a single-device model");
  const agxc_model_desc& D = m->d;
  AGXC_CUDA(cudaStreamSynchronize(m->ctx->stream));
  StateHeader h{};
  std::memcpy(h.magic, "AGXS", 4);
  h.version = 1;
  h.layers = D.n_layers; h.kv_heads = D.n_kv_heads; h.head_dim = D.head_dim; h.d_model = D.d_model;
  h.vocab = m->vt; h.cap = D.cap;
  AGXC_CUDA(cudaMemcpy(&h.q0, m->q0 + b, 4, cudaMemcpyDeviceToHost));
  AGXC_CUDA(cudaMemcpy(&h.force_next, m->force_next + b, 4, cudaMemcpyDeviceToHost));
  const size_t need = state_bytes(m, h.q0);
  if (capacity < need) return agxc::fail(AGXC_EINVAL, "state_save: the buffer holds " + std::to_string(capacity) +
                                                          " bytes, the state needs " + std::to_string(need));
  uint8_t* o = static_cast<uint8_t*>(out);
  std::memcpy(o, &h, sizeof h);
  o += sizeof h;
  AGXC_CUDA(cudaMemcpy(o, m->log + static_cast<size_t>(b) * D.cap, static_cast<size_t>(D.cap) * 4,
                       cudaMemcpyDeviceToHost));
  o += static_cast<size_t>(D.cap) * 4;
  AGXC_CUDA(cudaMemcpy(o, m->x16 + static_cast<size_t>(b) * D.d_model, static_cast<size_t>(D.d_model) * 2,
                       cudaMemcpyDeviceToHost));
  o += static_cast<size_t>(D.d_model) * 2;
  const size_t rows = static_cast<size_t>(h.q0) * D.head_dim * 2;
  for (int which = 0; which < 2; ++which)
    for (int l = 0; l < D.n_layers; ++l)
      for (int kv = 0; kv < D.n_kv_heads; ++kv) {
        const __half* src = (which ? m->vcache : m->kcache) + kv_off(m, l, b, kv);
        if (rows) AGXC_CUDA(cudaMemcpy(o, src, rows, cudaMemcpyDeviceToHost));
        o += rows;
      }
  if (written) *written = need;
  return 0;
}

int agxc_model_state_restore(agxc_model* m, int b, const void* in, size_t bytes) {
  if (!m || !in || b < 0 || b >= m->d.batch) return agxc::fail(AGXC_EINVAL, "state_restore: bad argument");
  if (m->tp > 1) return agxc::fail(AGXC_EUNSUPPORTED, "state_restore: a single-device model");
  const agxc_model_desc& D = m->d;
  if (bytes < sizeof(StateHeader)) return agxc::fail(AGXC_EINVAL, "state_restore: shorter than its header");
  StateHeader h;
  std::memcpy(&h, in, sizeof h);
  if (std::memcmp(h.magic, "AGXS", 4) || h.version != 1) return agxc::fail(AGXC_EINVAL, "state_restore: not a state image");
  if (h.layers != static_cast<uint32_t>(D.n_layers) || h.kv_heads != static_cast<uint32_t>(D.n_kv_heads) ||
      h.head_dim != static_cast<uint32_t>(D.head_dim) || h.d_model != static_cast<uint32_t>(D.d_model) ||
      h.vocab != static_cast<uint32_t>(m->vt))
    return agxc::fail(AGXC_EINVAL, "state_restore: the image's shapes differ from the model's");
  if (h.q0 + 1 > static_cast<uint32_t>(D.cap)) return agxc::fail(AGXC_EINVAL, "state_restore: q0 beyond the cap");
  if (h.force_next != agxc::kTokenUnset && h.force_next >= h.vocab)
    return agxc::fail(AGXC_EINVAL, "state_restore: forced token out of range");
  const size_t saved_cap = h.cap;
  const size_t need = sizeof h + saved_cap * 4 + static_cast<size_t>(D.d_model) * 2 +
                      2 * static_cast<size_t>(D.n_layers) * D.n_kv_heads * h.q0 * D.head_dim * 2;
  if (bytes != need) return agxc::fail(AGXC_EINVAL, "state_restore: the image's size disagrees with its header");
  const uint8_t* p = static_cast<const uint8_t*>(in) + sizeof h;
  std::vector<uint32_t> log(D.cap, agxc::kTokenUnset);
  const uint32_t* slog = reinterpret_cast<const uint32_t*>(p);
  for (size_t i = 0; i < saved_cap; ++i) {
    const uint32_t t = slog[i];
    if (t != agxc::kTokenUnset && t >= h.vocab) return agxc::fail(AGXC_EINVAL, "state_restore: a logged token is out of range");
    if (i < static_cast<size_t>(D.cap)) log[i] = t;
    else if (t != agxc::kTokenUnset) return agxc::fail(AGXC_EINVAL, "state_restore: the log does not fit the cap");
  }
  p += saved_cap * 4;
  cudaStream_t s = m->ctx->stream;
  AGXC_CUDA(cudaStreamSynchronize(s));
  AGXC_CUDA(cudaMemcpy(m->log + static_cast<size_t>(b) * D.cap, log.data(), log.size() * 4, cudaMemcpyHostToDevice));
  AGXC_CUDA(cudaMemcpy(m->x16 + static_cast<size_t>(b) * D.d_model, p, static_cast<size_t>(D.d_model) * 2,
                       cudaMemcpyHostToDevice));
  p += static_cast<size_t>(D.d_model) * 2;
  const size_t rows = static_cast<size_t>(h.q0) * D.head_dim * 2;
  for (int which = 0; which < 2; ++which)
    for (int l = 0; l < D.n_layers; ++l)
      for (int kv = 0; kv < D.n_kv_heads; ++kv) {
        __half* dst = (which ? m->vcache : m->kcache) + kv_off(m, l, b, kv);
        if (rows) AGXC_CUDA(cudaMemcpy(dst, p, rows, cudaMemcpyHostToDevice));
        p += rows;
      }
  AGXC_CUDA(cudaMemcpy(m->q0 + b, &h.q0, 4, cudaMemcpyHostToDevice));
  AGXC_CUDA(cudaMemcpy(m->force_next + b, &h.force_next, 4, cudaMemcpyHostToDevice));
  return 0;
}

int agxc_model_read_kv(agxc_model* m, int layer, int b, int n, uint16_t* k_out, uint16_t* v_out) {
  if (!m) return agxc::fail(AGXC_EINVAL, "read_kv: null model");
  const agxc_model_desc& D = m->d;
  if (layer < 0 || layer >= D.n_layers || b < 0 || b >= D.batch || n < 0 || n > D.cap)
    return agxc::fail(AGXC_EINVAL, "read_kv: range");
  for (int kv = 0; kv < D.n_kv_heads; ++kv) {
    const size_t off = ((static_cast<size_t>(layer) * D.batch + b) * D.n_kv_heads + kv) * D.cap * D.head_dim;
    const size_t bytes = static_cast<size_t>(n) * D.head_dim * 2;
    if (k_out) AGXC_CUDA(cudaMemcpy(k_out + static_cast<size_t>(kv) * n * D.head_dim, m->kcache + off, bytes, cudaMemcpyDeviceToHost));
    if (v_out) AGXC_CUDA(cudaMemcpy(v_out + static_cast<size_t>(kv) * n * D.head_dim, m->vcache + off, bytes, cudaMemcpyDeviceToHost));
  }
  return 0;
}

int agxc_model_logits_dev(agxc_model* m, const float** out) {
  if (!m || !out) return agxc::fail(AGXC_EINVAL, "logits_dev: null argument");
  if (!m->d.keep_logits) return agxc::fail(AGXC_EINVAL, "logits_dev: model made without keep_logits");
  *out = m->logits;
  return 0;
}

int agxc_model_profile(agxc_model* m, int steps, float* kind_ms, int32_t* kind_launches) {
  if (!m || !kind_ms || !kind_launches || steps < 1) return agxc::fail(AGXC_EINVAL, "profile: bad argument");
  return agxc::model_profile(m, steps, kind_ms, kind_launches);
}

int agxc_model_vocab_slice(const agxc_model* m, int32_t* offset, int32_t* count) {
  if (!m || !offset || !count) return agxc::fail(AGXC_EINVAL, "vocab_slice: null argument");
  *offset = m->v0;
  *count = m->d.vocab;
  return 0;
}

int agxc_model_plan_info(agxc_model* m, char* buf, size_t len) {
  if (!m || !buf || !len) return agxc::fail(AGXC_EINVAL, "plan_info: bad argument");
  auto one = [](const char* name, const agxc::QmvPlan& p) {
    return std::string("\"") + name + "\": {\"row_tiles\": " + std::to_string(p.RW) + ", \"splits\": " +
           std::to_string(p.SC) + ", \"groups\": " + std::to_string(p.GC) + ", \"chunk_groups\": " +
           std::to_string(p.CG) + ", \"stages\": " + std::to_string(p.stages) + ", \"grid\": " +
           std::to_string(p.grid) + ", \"smem\": " + std::to_string(p.smem) + "}";
  };
  std::string j = "{" + one("qkv", m->p_qkv) + ", " + one("wo", m->p_wo) + ", " + one("ffn", m->p_gu) + ", " +
                  one("down", m->p_down) + ", " + one("head", m->p_head) + ", \"attn\": {\"chunks\": " +
                  std::to_string(m->attn_S) + ", \"max_cluster\": " + std::to_string(m->ctx->max_cluster) +
                  "}, \"pdl\": " + std::to_string(m->pdl) + ", \"fused\": {\"on\": " +
                  std::to_string(agxc::fused_active(m)) + ", \"fits\": " + std::to_string(m->fs_ok) +
                  ", \"ring_stages\": " + std::to_string(m->fs_stages) + ", \"max_splits\": " +
                  std::to_string(m->fs_smax) + ", \"grid\": " +
                  std::to_string(m->ctx->num_sms) + "}, \"tp\": {\"world\": " + std::to_string(m->tp) +
                  ", \"rank\": " + std::to_string(m->tp_rank) + ", \"heads\": " + std::to_string(m->d.n_heads) +
                  ", \"kv_heads\": " + std::to_string(m->d.n_kv_heads) + ", \"ffn\": " +
                  std::to_string(m->d.ffn) + ", \"vocab_offset\": " + std::to_string(m->v0) +
                  ", \"vocab_count\": " + std::to_string(m->d.vocab) + ", \"fused\": " +
                  std::to_string(m->comm && m->tp_fused && m->tp_fused_ok) + ", \"two_shot\": " +
                  std::to_string(m->tp_two_shot) + ", \"fused_available\": " +
                  std::to_string(m->tp_fused_ok) + "}}";
  std::snprintf(buf, len, "%s", j.c_str());
  return 0;
}

int agxc_model_trace_read(agxc_model* m, uint64_t* out, int capacity, int32_t* n) {
  if (!m || !out || !n) return agxc::fail(AGXC_EINVAL, "trace_read: null argument");
  if (!m->trace) return agxc::fail(AGXC_EINVAL, "trace_read: tracing is off (AGXC_OPT_TRACE)");
  const int k = std::min(capacity, m->trace_n);
  AGXC_CUDA(cudaStreamSynchronize(m->ctx->stream));
  const int w = 2 * agxc::kTraceSlots;
  AGXC_CUDA(cudaMemcpy(out, m->trace, static_cast<size_t>(k) * w * 8, cudaMemcpyDeviceToHost));
  agxc::trace_reset_kernel<<<(w * m->trace_n + 255) / 256, 256, 0, m->ctx->stream>>>(m->trace, w * m->trace_n);
  AGXC_CUDA(cudaGetLastError());
  *n = k;
  return 0;
}

int agxc_model_trace_cta_read(agxc_model* m, uint64_t* out, size_t capacity, int32_t* phases, int32_t* ctas) {
  if (!m || !out || !phases || !ctas) return agxc::fail(AGXC_EINVAL, "trace_cta_read: null argument");
  if (!m->cta_trace) return agxc::fail(AGXC_EINVAL, "trace_cta_read: no fused-step trace (AGXC_OPT_TRACE)");
  const int marks = agxc::fstep_trace_marks(m->d.n_layers);
  const size_t w = static_cast<size_t>(marks) * m->ctx->num_sms;
  AGXC_CUDA(cudaStreamSynchronize(m->ctx->stream));
  AGXC_CUDA(cudaMemcpy(out, m->cta_trace, std::min(capacity, w) * 8, cudaMemcpyDeviceToHost));
  *phases = marks;
  *ctas = m->ctx->num_sms;
  return 0;
}

int agxc_model_set_option(agxc_model* m, int option, int value) {
  if (!m) return agxc::fail(AGXC_EINVAL, "set_option: null model");
  if (option == AGXC_OPT_PDL) {
    if (value < 0 || value > 3) return agxc::fail(AGXC_EINVAL, "set_option: pdl 0, 1, 2 or 3");
    m->pdl = value;
  } else if (option == AGXC_OPT_BULK) {
    m->bulk = value ? 1 : 0;
  } else if (option == AGXC_OPT_TP_FUSED) {
    if (value < 0 || value > 3) return agxc::fail(AGXC_EINVAL, "set_option: tp_fused 0, 1, 2 or 3");
    if (value && !m->tp_fused_ok)
      return agxc::fail(AGXC_EUNSUPPORTED, "set_option: no fused tensor-parallel path (" +
                                               (m->comm ? m->tp_fused_why : std::string("single device")) + ")");
    const int two = value == 2 ? 1 : value == 3 ? 0 : (m->tp >= 4);
    if (value && two != m->tp_two_shot && m->tp_fused_ran)  // the arrival counters already count the other variant
      return agxc::fail(AGXC_EINVAL, "set_option: the fused variant is fixed once a fused step has run");
    if (value) m->tp_two_shot = two;
    m->tp_fused = value ? 1 : 0;
  } else if (option == AGXC_OPT_WAIT_MS) {
    if (value < 1) return agxc::fail(AGXC_EINVAL, "set_option: wait_ms must be positive");
    m->wait_ms = value;
    return 0;  // no graph change
  } else if (option == AGXC_OPT_FUSED) {
    if (value && !m->fs_ok)
      return agxc::fail(AGXC_EUNSUPPORTED, "set_option: this model has no fused step (batch 1 on one device, and the "
                                           "ring must fit the shared memory)");
    m->fused = value ? 1 : 0;
  } else if (option == AGXC_OPT_DEVICE_WAIT_US) {
    if (value < 0) return agxc::fail(AGXC_EINVAL, "set_option: device_wait_us must be >= 0");
    m->dev_wait_ns = static_cast<uint64_t>(value) * 1000ull;
  } else if (option == AGXC_OPT_QK_NORM) {
    m->qk_norm = value ? 1 : 0;
  } else if (option == AGXC_OPT_TRACE) {
    if (value && !m->trace) {
      const int n = 2 * agxc::kTraceSlots * (5 * m->d.n_layers + 1);
      void* t = nullptr;
      if (cudaMalloc(&t, static_cast<size_t>(n) * 8) != cudaSuccess) {
        cudaGetLastError();
        return agxc::fail(AGXC_ENOMEM, "set_option: trace buffer");
      }
      m->trace = static_cast<unsigned long long*>(t);
      m->trace_n = n / (2 * agxc::kTraceSlots);
      if (m->fs_ok) {
        const size_t cw = static_cast<size_t>(agxc::fstep_trace_marks(m->d.n_layers)) * m->ctx->num_sms;
        if (cudaMalloc(&t, cw * 8) != cudaSuccess) {
          cudaGetLastError();
          return agxc::fail(AGXC_ENOMEM, "set_option: trace buffer");
        }
        m->cta_trace = static_cast<unsigned long long*>(t);
        AGXC_CUDA(cudaMemset(m->cta_trace, 0, cw * 8));
      }
      agxc::trace_reset_kernel<<<(n + 255) / 256, 256, 0, m->ctx->stream>>>(m->trace, n);
      AGXC_CUDA(cudaGetLastError());
    } else if (!value && m->trace) {
      AGXC_CUDA(cudaStreamSynchronize(m->ctx->stream));
      cudaFree(m->trace);
      m->trace = nullptr;
      m->trace_n = 0;
      if (m->cta_trace) cudaFree(m->cta_trace);
      m->cta_trace = nullptr;
    }
  } else {
    return agxc::fail(AGXC_EINVAL, "set_option: unknown option");
  }
  if (m->exec) {
    cudaGraphExecDestroy(m->exec);
    m->exec = nullptr;
  }
  if (m->graph) {
    cudaGraphDestroy(m->graph);
    m->graph = nullptr;
  }
  return 0;
}

int agxc_model_kernel_count(agxc_model* m, int32_t* n) {
  if (!m || !n) return agxc::fail(AGXC_EINVAL, "kernel_count: null argument");
  *n = 5 * m->d.n_layers + 1;
  return 0;
}

}  // extern "C"
