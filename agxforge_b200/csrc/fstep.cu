// fstep.cu — the batch-1 decode step as ONE persistent kernel with fine-grained dependencies (the reference's
// per-token command buffer of the whole model, tools/g17decodegen.m:167-199, and its 7-dispatch layer,
// agxforge/inference/assemble.py:429-520, restructured for a B200: one CTA per SM, every layer in four phases).
//
// Per layer, every CTA runs four phases; work of a phase waits only for the data it reads:
//   Q  qkv        wait until x is complete (all FFN units of the previous layer); x16 = fp16(h + sum of the down
//                 partials); RMSNorm; its qkv row tiles (GEMV, bias, RoPE at q0, q scale, K/V append at q0). Signals
//                 the tile's KV-head group.
//   A  attention  CTA (group j, split s): waits for group j's 32 qkv row tiles only; online base-2 softmax over its
//                 key range on the tensor cores (keys as M, the group's query heads as N); writes its partial
//                 (m, l, o) and signals group j.
//   O  o_proj     the same CTAs: wait for group j's S partials, merge them (log-sum-exp), round to fp16 (the
//                 reference's attention output), and multiply by W_o's columns of group j for a contiguous range of
//                 row tiles: a per-group split-K partial of o_proj, added into the layer's h accumulator in L2.
//   F  FFN        wait until h is complete; h = x16 + the accumulated o_proj rows; RMSNorm; a 64-row group f of
//                 gate and up (GEMV + SiLU * up, fp16 act), then immediately the down projection's 64-column K
//                 slice f for every output row: a per-F-group split-K partial of down, added into the layer's x
//                 accumulator.
// Then the head: wait for the last layer's x; final RMSNorm; a contiguous range of vocabulary row tiles; per-CTA
// first maximum; the last CTA to finish takes the grid's first maximum and runs the generation step (token log,
// next x = embedding row, q0 + 1) — argmax.py:141-215 / assemble.py:918-930.
//
// Within a CTA, one PRODUCER warp streams every chunk the CTA's consumers will read — weight tiles by 3-D TMA boxes
// of the B200 pack (16 rows x 64 k per tile), the KV history by TMA boxes with the 128-byte swizzle — into a ring of
// 18 KB shared-memory stages, in consumption order, as far ahead as the ring allows. Weights and the cache history do
// not depend on this step's activations, so the ring fills while the consumers wait on dependencies, and HBM keeps
// streaming across phase and layer boundaries. 16 CONSUMER warps dequantise into tensor-core fragments (the GEMV's
// group step) and run the epilogues.
//
// Dependencies are monotonic counters in global memory (release adds, acquire polls). Each step uses one of two
// counter/accumulator sets by the step counter's parity and clears the other for the next step, so no host work runs
// between steps. Every wait is bounded (2 s of the global timer); the first that gives up raises an abort bit that
// every other wait honours, and the step leaves with the error word set instead of hanging.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include "gemv_impl.cuh"

namespace agxc {
namespace fstep {

using gemv::group_step;
// 16 consumer warps (with the producer and the signal warp, 18: 96 registers a thread)
constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }
__device__ __forceinline__ bool consumer_sync_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(kConsumers)
      : "memory");
  return r != 0;
}
// 16 consumer warps, the producer warp, and the signal warp: it performs the consumers' release counts (a gpu-scope
// release waits for the CTA's earlier writes to reach L2, ~1 us), so the consumers go on at once
constexpr int kThreads = kConsumers + 64;
constexpr int kSignalWarp = kConsumerWarps + 1;
constexpr int kSigSlots = 16;

constexpr int kStage = 18432;         // one ring stage: 16 KB of weight tiles (or K/V rows) + 2 KB of scale/bias
constexpr int kSbOff = 16384;         // the scale/bias part of a stage
constexpr int kMaxRing = 12;
constexpr int kKeyTile = 16;          // keys per MMA tile (M)
constexpr int kMinKeys = 32;          // the fewest keys an attention split takes
// per layer: 0 Q dependency met, 1 Q done, 2 A dependency met, 3 A done, 4 O dependency met, 5 O done, 6 F dependency
// met, 7 F done; within phases: 8 Q input normed, 9 Q first row tile done, 10 A keys done (before the CTA's merge),
// 11 O partials merged, 12 F input normed, 13 F first gate/up batch done, 14 F gate/up done, 15 F first down chunk
// done; the producer: 16 first Q chunk issued, 17 A chunks begin, 18 first F chunk issued, 19 last F chunk issued;
// 20 / 21 the first qkv tile's chunk landed / thread 0's share done, 22 / 23 the same for the first gate/up batch,
// 24 the second gate/up batch's first chunk landed, 25 the producer's first down chunk issued
constexpr int kTraceMarks = 26;

// The maps of a model: one 4-D map (the pack's 3-D tile grid x the layer) per role of the layer, then the head's two
// and the caches' two. Few descriptors: the TMA unit keeps them cached instead of fetching one from memory for every
// copy (per-layer maps, 8 a layer, cost a descriptor fetch nearly every copy).
enum : int { M_QKV_W = 0, M_QKV_SB, M_WO_W, M_WO_SB, M_GU_W, M_GU_SB, M_DN_W, M_DN_SB, M_HEAD_W, M_HEAD_SB, M_K, M_V,
             kMaps };

__host__ __device__ inline int tps(int bits) { return bits == 4 ? 32 : 16; }          // tiles per stage
__host__ __device__ inline int tile_b(int bits) { return bits == 4 ? 512 : 1024; }
__host__ __device__ inline int ctr_per_layer(int KVH) { return 2 * KVH + 2; }

struct Layout {
  int ring, x16k, hk, xs, xsum, xo, xsumo, act, xsuma, red, ov, om, kn, misc, total;
};

// Shared memory, 1,024-byte aligned base: the ring first (the KV boxes' 128-byte swizzle wants 1,024-byte alignment).
__host__ __device__ inline Layout smem_layout(int d, int kattn, int stages) {
  Layout L;
  L.ring = 0;
  int o = stages * kStage;
  L.x16k = o; o += (d * 2 + 127) / 128 * 128;             // x16 of this layer (fp16)
  L.hk = o; o += (d * 4 + 127) / 128 * 128;               // h of this layer (fp32)
  L.xs = o; o += (d * 2 + 127) / 128 * 128;               // the normed GEMV input (fp16)
  L.xsum = o; o += (d / 64) * 32;                         // its per-group sums, 32 B a group
  L.xo = o; o += (kattn * 2 + 127) / 128 * 128;           // the merged attention output of one group (fp16)
  L.xsumo = o; o += ((kattn / 64) * 32 + 127) / 128 * 128;
  L.act = o; o += 128;                                    // one FFN group's act (64 fp16)
  L.xsuma = o; o += 128;
  L.red = o; o += kConsumerWarps * 16 * 4 * 2;            // per-warp partial rows
  L.ov = o; o += (kattn * 4 + 127) / 128 * 128;           // attention: the CTA's o accumulator [G][hd]
  L.om = o; o += kConsumerWarps * 8 * 2 * 4 + 64;         // attention: per-warp (m, l) per head, then M, L per head
  L.kn = o; o += 256;                                     // QK-norm: the group's new k row (fp16, head_dim <= 128)
  L.misc = o; o += 1024;
  L.total = o;
  return L;
}

struct Params {
  int L, d, H, KVH, hd, G, F, V, cap, bits, sdt, stages;
  float eps, qscale;
  uint64_t wait_ns;        // the bound on every wait (global timer)
  int rt_qkv, rt_d, nf, rt_v, gd, gk, gchunk, dn_rows, smax;
  int o_per, o_sb;         // o_proj: row tiles a stage, and the byte stride of their scale/bias boxes (a TMA
                           // destination starts on a 128-byte boundary)
  const CUtensorMap* maps;
  const __half* gains;     // [L][2][d]
  const __half* bias;      // [L][qkv rows] or null
  const __half* qkg;       // [L][2][hd] QK-norm gains (q, k), or null: no QK-norm
  float* qkraw;            // [(H + KVH) hd] QK-norm: the qkv phase's q and k rows before the norm and RoPE
  const __half* final_gain;
  const __half* embed;     // [V][d]
  __half* kc;              // [L][KVH][cap][hd]
  __half* vc;
  const float* cos_t;      // [cap][hd/2]
  const float* sin_t;
  uint32_t* q0;
  uint32_t* log;
  int32_t* tok_out;
  uint32_t* force_next;
  __half* x16;             // [d]: the step's input row; the next step's on exit
  float* logits;           // [V] or null
  __half* q16;             // [H hd]
  float* apart;            // [KVH][smax][G][hd + 2]
  float* acc;              // [2 parities][2: h, x][L][d]
  unsigned* sync;          // [0] step counter; [64 + parity * nctr ...] counters
  int nctr;
  float* pairs;            // [grid][2]
  unsigned* err;
  unsigned long long* trace;  // [L * kTraceMarks + 2][grid], or null
};

// ------------------------------------------------------------------------------------------------ small helpers
__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_rel(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The consumers' release counts, handed to the signal warp: thread 0 posts (counter, value) after a consumer barrier
// (the mbarrier arrive is a CTA-scope release, the signal warp's wait a CTA-scope acquire, and its gpu-scope release
// count is cumulative over the consumers' writes). A null counter ends the queue.
struct SigQueue {
  unsigned* addr[kSigSlots];
  unsigned val[kSigSlots];
  uint64_t full[kSigSlots], empty[kSigSlots];
};
__device__ __forceinline__ void red_f32(float* p, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
// four consecutive floats (16-byte aligned) added in one reduction operation
__device__ __forceinline__ void red_f32x4(float* p, float4 v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, unsigned cnt) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(cnt) : "memory");
}
__device__ __forceinline__ void tma4(void* dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
// L2 prefetches of a box (no shared memory, no barrier): the weights and history a CTA will load later are brought
// from HBM into L2 ahead of time, so HBM keeps streaming while the CTAs wait on each other.
__device__ __forceinline__ void pf4(const CUtensorMap* map, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void pf3(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}
// 2^x by the SFU (ex2.approx.ftz: relative error about 2^-22; -inf -> 0), as the reference's hardware exp2
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}
// byte offset of (row, 16-byte chunk) in a 128-byte-swizzled box of 128-byte rows
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ bool aborted(const Params& P) {
  return (*reinterpret_cast<volatile unsigned*>(P.err) & kErrAbort) != 0;
}
__device__ __forceinline__ void raise_abort(const Params& P, unsigned bits) { atomicOr(P.err, bits | kErrAbort); }

// A bounded mbarrier wait that also leaves when the launch aborted.
// The slow path of a wait, out of line (one copy, off the hot path's instruction footprint).
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, unsigned parity, const Params& P) {
  const uint64_t t0 = globaltimer_ns();
  for (unsigned it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (aborted(P)) return false;
      if (globaltimer_ns() - t0 > P.wait_ns) {
        raise_abort(P, kErrMbarTimeout);
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, unsigned parity, const Params& P) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, P);
}

// Thread 0 of the consumers polls a counter until it reaches `target` (bounded, abortable); then every consumer
// thread learns the outcome. Reads of the data the counter guards follow (from L2).
__device__ bool wait_counter(const unsigned* c, unsigned target, const Params& P, volatile int* flag) {
  if (threadIdx.x == 0) {
    int ok = 1;
    if (ld_acq(c) < target) {
      const uint64_t t0 = globaltimer_ns();
      for (unsigned it = 0;; ++it) {
        if (ld_acq(c) >= target) break;
        if ((it & 15u) == 15u) {
          if (aborted(P)) { ok = 0; break; }
          if (globaltimer_ns() - t0 > P.wait_ns) {
            raise_abort(P, kErrGridTimeout | kErrMbarTimeout);
            ok = 0;
            break;
          }
        }
      }
    }
    *flag = ok;
  }
  consumer_sync();
  return *flag != 0;
}

__device__ __forceinline__ void mark(const Params& P, int slot) {
  if (P.trace && threadIdx.x == 0) P.trace[static_cast<size_t>(slot) * gridDim.x + blockIdx.x] = globaltimer_ns();
}
// the producer's marks (its one issuing thread)
__device__ __forceinline__ void pmark(const Params& P, int slot) {
  if (P.trace) P.trace[static_cast<size_t>(slot) * gridDim.x + blockIdx.x] = globaltimer_ns();
}

// The cycle profile (when tracing): consumer thread 0's SM cycles, accumulated per region over the step and written
// after the marks as kProfRegions rows [region][CTA]. prof(P, k) closes the current interval into region k. Thread 0
// passes every consumer barrier, so its time line is the CTA's.
enum : int {
  R_TOP = 0, R_PRELOAD, R_WAIT, R_ACTLOAD, R_NORM, R_ROWS, R_REDUCE, R_QKV_EPI, R_SIGNAL, R_ATTN_Q, R_ATTN_KEYS,
  R_ATTN_MERGE, R_ATTN_OUT, R_O_MERGE, R_OWNED, R_SILU, R_HEAD, R_TAIL, R_OWNED_WAIT, R_ROWS_WAIT, R_ATTN_WAIT,
  kProfRegions = 24
};
__device__ __forceinline__ long long* prof_acc() {
  __shared__ long long a[kProfRegions + 1];  // [regions], then the interval's start
  return a;
}
__device__ __forceinline__ void prof(const Params& P, int k) {
  if (P.trace && threadIdx.x == 0) {
    long long* a = prof_acc();
    const long long t = clock64();
    a[k] += t - a[kProfRegions];
    a[kProfRegions] = t;
  }
}
__device__ __forceinline__ void prof_begin(const Params& P) {
  if (P.trace && threadIdx.x == 0) {
    long long* a = prof_acc();
    for (int k = 0; k < kProfRegions; ++k) a[k] = 0;
    a[kProfRegions] = clock64();
  }
}
__device__ __forceinline__ void prof_end(const Params& P) {
  if (P.trace && threadIdx.x == 0) {
    const long long* a = prof_acc();
    for (int k = 0; k < kProfRegions; ++k)
      P.trace[static_cast<size_t>(P.L * kTraceMarks + 2 + k) * gridDim.x + blockIdx.x] = static_cast<unsigned long long>(a[k]);
  }
}

// ------------------------------------------------------------------------------------------------ the schedule
// Which work a CTA owns; the producer and the consumers enumerate it identically.
struct Sched {
  int pos, nk, S;             // q0 (clamped), live keys, attention splits per KV group
  __device__ void init(const Params& P) {
    pos = static_cast<int>(P.q0[0]);
    if (pos > P.cap - 1) pos = P.cap - 1;
    nk = pos + 1;
    S = (nk + kMinKeys - 1) / kMinKeys;
    if (S > P.smax) S = P.smax;
    if (S < 1) S = 1;
  }
  // attention / o_proj: the CTA's group and split (false when it has none)
  __device__ bool attn(const Params& P, int c, int* j, int* s, int* k0, int* k1) const {
    if (c >= P.KVH * S) return false;
    *j = c / S;
    *s = c % S;
    const int Lk = (nk + S - 1) / S;
    *k0 = *s * Lk;
    *k1 = min(nk, *k0 + Lk);
    return true;
  }
  __device__ void orows(const Params& P, int s, int* r0, int* r1) const {
    *r0 = static_cast<int>(static_cast<long long>(s) * P.rt_d / S);
    *r1 = static_cast<int>(static_cast<long long>(s + 1) * P.rt_d / S);
  }
};

// Stage geometry of the chunks (what the producer issues, what the consumers read).
__device__ __forceinline__ int row_chunks(const Params& P) { return (P.gd + P.gchunk - 1) / P.gchunk; }
__device__ __forceinline__ int kv_keys(const Params& P) { return 16384 / (4 * P.hd); }   // keys per KV stage

// ------------------------------------------------------------------------------------------------ producer
struct Prod {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  volatile int* dead;
  int stages, slot = 0, phase = 0;
  long issued = 0;
  __device__ uint8_t* acquire(const Params& P) {
    if (*dead) return nullptr;
    if (issued >= stages && !mbar_wait_abortable(&empty[slot], phase ^ 1, P)) {
      *dead = 1;
      return nullptr;
    }
    return ring + slot * kStage;
  }
  __device__ void advance() {
    ++issued;
    if (++slot == stages) { slot = 0; phase ^= 1; }
  }
  // one box of (gb groups x rb row tiles) of layer l's pack (weights and scale/bias maps; l < 0: the head's 3-D
  // maps), into one stage; gb and rb are the maps' box dimensions (a box reaching past the pack's groups or row tiles
  // still lands whole, zero-filled)
  __device__ bool pack_chunk(const Params& P, int mw, int l, int g0, int rt, int gb, int rb) {
    uint8_t* st = acquire(P);
    if (!st) return false;
    const int TB = tile_b(P.bits);
    mbar_arrive_expect_tx(&full[slot], static_cast<unsigned>(gb * rb * (TB + 64)));
    if (l >= 0) {
      tma4(st, P.maps + mw, 0, g0, rt, l, &full[slot]);
      tma4(st + kSbOff, P.maps + mw + 1, 0, g0, rt, l, &full[slot]);
    } else {
      tma3(st, P.maps + mw, 0, g0, rt, &full[slot]);
      tma3(st + kSbOff, P.maps + mw + 1, 0, g0, rt, &full[slot]);
    }
    advance();
    return true;
  }
};

// The producer's L2 prefetches mirror its loads one layer ahead: layer l + 1's boxes of a phase are prefetched when
// the same phase of layer l is issued, the head's first rows during the last FFN phase and then kHeadAhead row tiles
// ahead, and layer 0's boxes (of the next step) after the head.
constexpr int kHeadAhead = 12;
struct Prefetch {
  const Params& P;
  int c, grid, nrc, KC, HD;
  __device__ void q(int l) const {
    #pragma unroll 1
    for (int t = c; t < P.rt_qkv; t += grid)
      #pragma unroll 1
      for (int k = 0; k < nrc; ++k) {
        pf4(P.maps + M_QKV_W, 0, k * P.gchunk, t, l);
        pf4(P.maps + M_QKV_SB, 0, k * P.gchunk, t, l);
      }
  }
  __device__ void a(int l, int j, int k0, int k1) const {
    const int z = l * P.KVH + j;
    #pragma unroll 1
    for (int a = k0; a < k1; a += KC)
      #pragma unroll 1
      for (int h = 0; h < HD / 64; ++h) {
        pf3(P.maps + M_K, h * 64, a, z);
        pf3(P.maps + M_V, h * 64, a, z);
      }
  }
  __device__ void o(int l, int j, int r0, int r1) const {
    #pragma unroll 1
    for (int r = r0; r < r1; ++r) {
      pf4(P.maps + M_WO_W, 0, j * P.gk, r, l);
      pf4(P.maps + M_WO_SB, 0, j * P.gk, r, l);
    }
  }
  __device__ void f(int l) const {
    #pragma unroll 1
    for (int f = c; f < P.nf; f += grid) {
      #pragma unroll 1
      for (int t = 8 * f; t < 8 * f + 8; ++t)
        #pragma unroll 1
        for (int k = 0; k < nrc; ++k) {
          pf4(P.maps + M_GU_W, 0, k * P.gchunk, t, l);
          pf4(P.maps + M_GU_SB, 0, k * P.gchunk, t, l);
        }
      #pragma unroll 1
      for (int r = 0; r < P.rt_d; r += P.dn_rows) {
        pf4(P.maps + M_DN_W, 0, f, r, l);
        pf4(P.maps + M_DN_SB, 0, f, r, l);
      }
    }
  }
  __device__ void head(int t0, int t1) const {
    #pragma unroll 1
    for (int t = t0; t < t1; ++t)
      #pragma unroll 1
      for (int k = 0; k < nrc; ++k) {
        pf3(P.maps + M_HEAD_W, 0, k * P.gchunk, t);
        pf3(P.maps + M_HEAD_SB, 0, k * P.gchunk, t);
      }
  }
};

template <int BITS, int HD>
__device__ void produce(const Params& P, const Sched& S, Prod& pr) {
  const int c = blockIdx.x, grid = gridDim.x;
  const int nrc = row_chunks(P);
  const int KC = kv_keys(P);
  const CUtensorMap* kmap = P.maps + M_K;
  const CUtensorMap* vmap = P.maps + M_V;
  #pragma unroll 1
  for (int i = 0; i < kMaps; ++i)  // every descriptor of the step into the TMA unit's cache up front
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(P.maps + i)) : "memory");
  const Prefetch pf{P, c, grid, nrc, KC, HD};
  int j, s, k0, k1, r0 = 0, r1 = 0;
  const bool has_attn = S.attn(P, c, &j, &s, &k0, &k1);
  if (has_attn) S.orows(P, s, &r0, &r1);
  const int h0 = static_cast<int>(static_cast<long long>(c) * P.rt_v / grid);
  const int h1 = static_cast<int>(static_cast<long long>(c + 1) * P.rt_v / grid);
  #pragma unroll 1
  for (int l = 0; l < P.L && !*pr.dead; ++l) {
    const bool next = l + 1 < P.L;
    // Q: the CTA's qkv row tiles, each in row_chunks chunks of gchunk groups
    if (next) pf.q(l + 1);
    #pragma unroll 1
    for (int t = c; t < P.rt_qkv; t += grid)
      #pragma unroll 1
      for (int k = 0; k < nrc; ++k) {
        if (!pr.pack_chunk(P, M_QKV_W, l, k * P.gchunk, t, P.gchunk, 1)) return;
        if (t == c && k == 0) pmark(P, l * kTraceMarks + 16);
      }
    if (has_attn) {
      // A: the key range in KC-key chunks (K and V rows of the group's KV head, 64-dim swizzled boxes)
      const int z = l * P.KVH + j;
      if (next) pf.a(l + 1, j, k0, k1);
      pmark(P, l * kTraceMarks + 17);
      #pragma unroll 1
      for (int a = k0; a < k1; a += KC) {
        uint8_t* st = pr.acquire(P);
        if (!st) return;
        mbar_arrive_expect_tx(&pr.full[pr.slot], static_cast<unsigned>(KC * HD * 2 * 2));
#pragma unroll
        for (int h = 0; h < HD / 64; ++h) {
          tma3(st + h * KC * 128, kmap, h * 64, a, z, &pr.full[pr.slot]);
          tma3(st + (HD / 64 + h) * KC * 128, vmap, h * 64, a, z, &pr.full[pr.slot]);
        }
        pr.advance();
      }
      // O: W_o columns of group j for the split's row tiles, one row tile a box, TPS / gk row tiles a stage
      if (next) pf.o(l + 1, j, r0, r1);
      #pragma unroll 1
      for (int r = r0; r < r1; r += P.o_per) {
        uint8_t* st = pr.acquire(P);
        if (!st) return;
        const int nr = min(P.o_per, r1 - r);
        const int TB = tile_b(BITS);
        mbar_arrive_expect_tx(&pr.full[pr.slot], static_cast<unsigned>(nr * P.gk * (TB + 64)));
        #pragma unroll 1
        for (int q = 0; q < nr; ++q) {
          tma4(st + q * P.gk * TB, P.maps + M_WO_W, 0, j * P.gk, r + q, l, &pr.full[pr.slot]);
          tma4(st + kSbOff + q * P.o_sb, P.maps + M_WO_SB, 0, j * P.gk, r + q, l, &pr.full[pr.slot]);
        }
        pr.advance();
      }
    }
    // F: gate/up row tiles 8f .. 8f + 7 (four gate/up tile pairs), then down's K slice f for every row tile
    if (next) pf.f(l + 1);
    else pf.head(h0, min(h1, h0 + kHeadAhead));
    #pragma unroll 1
    for (int f = c; f < P.nf; f += grid) {
      #pragma unroll 1
      for (int t = 8 * f; t < 8 * f + 8; ++t)
        #pragma unroll 1
        for (int k = 0; k < nrc; ++k) {
          if (!pr.pack_chunk(P, M_GU_W, l, k * P.gchunk, t, P.gchunk, 1)) return;
          if (f == c && t == 8 * f && k == 0) pmark(P, l * kTraceMarks + 18);
        }
      #pragma unroll 1
      for (int r = 0; r < P.rt_d; r += P.dn_rows) {
        if (!pr.pack_chunk(P, M_DN_W, l, f, r, 1, P.dn_rows)) return;
        if (f == c && r == 0) pmark(P, l * kTraceMarks + 25);
      }
      if (f == c) pmark(P, l * kTraceMarks + 19);
    }
  }
  // the head: a contiguous range of vocabulary row tiles
  #pragma unroll 1
  for (int t = h0; t < h1; ++t) {
    if (t + kHeadAhead < h1) pf.head(t + kHeadAhead, t + kHeadAhead + 1);
    #pragma unroll 1
    for (int k = 0; k < nrc; ++k)
      if (!pr.pack_chunk(P, M_HEAD_W, -1, k * P.gchunk, t, P.gchunk, 1)) return;
  }
  // the next step's first layer (the same schedule: its keys reach one position further)
  pf.q(0);
  if (has_attn) {
    pf.a(0, j, k0, k1);
    pf.o(0, j, r0, r1);
  }
  pf.f(0);
}

// ------------------------------------------------------------------------------------------------ consumers
struct Cons {
  uint8_t* smem;
  Layout Lo;
  uint64_t* full;
  uint64_t* empty;
  volatile int* flag;     // wait_counter's broadcast
  volatile int* dead;     // a wait gave up (CTA-wide, read after a consumer barrier)
  int stages;
  // the next chunk's stage and its full-barrier parity (the same in every consumer warp), advanced by increments:
  // no division per chunk
  int slot = 0;
  unsigned phase = 0;
  __device__ uint32_t stage_addr(int sl) const { return smem_u32(smem + Lo.ring + sl * kStage); }
  __device__ void step(int& sl, unsigned& ph) const {
    if (++sl == stages) {
      sl = 0;
      ph ^= 1u;
    }
  }
};

// A norm gain's 8-element slices k = tid, tid + kConsumers, ... of this consumer thread (kNormSlices at most),
// loaded ahead of the dependency wait that precedes the norm.
constexpr int kNormSlices = 2;
__device__ __forceinline__ void norm_gains(const Params& P, const __half* g, uint4* out) {
#pragma unroll
  for (int i = 0; i < kNormSlices; ++i) {
    const int k = threadIdx.x + i * kConsumers;
    out[i] = k < P.d / 8 ? __ldg(reinterpret_cast<const uint4*>(g) + k) : make_uint4(0, 0, 0, 0);
  }
}

// The input of a phase, built and normed in one pass: thread t takes the 8-element slices k = t, t + 512, ... of the
// row, forms the value v (mode X_ACC: x16 = fp16(h + a) from the fp32 h in shared memory and the fp32 accumulator a
// in L2, v = x16; X_LOAD: x16 from L2; H_ACC: h = x16 + a, v = h), keeps it in registers, and after one reduction of
// the sum of squares stages y = fp16(v * r * g) (r = rsqrt(mean(v^2) + eps), norm.py:185-203's rounding point) into
// xs with the per-group sums of y (xsum[g * 8]). Two consumer barriers.
enum : int { X_ACC = 0, X_LOAD, H_ACC };
__device__ void stage_input(const Params& P, Cons& C, int mode, const float* a, const uint4* gpre) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __half* x16k = reinterpret_cast<__half*>(C.smem + C.Lo.x16k);
  float* hk = reinterpret_cast<float*>(C.smem + C.Lo.hk);
  __half* xs = reinterpret_cast<__half*>(C.smem + C.Lo.xs);
  float* xsum = reinterpret_cast<float*>(C.smem + C.Lo.xsum);
  float* red = reinterpret_cast<float*>(C.smem + C.Lo.red);
  const int n8 = P.d / 8;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormSlices; ++i) {
    const int k = i * kConsumers + tid;
    if (k >= n8) break;
    float v[8];
    if (mode == X_LOAD) {
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(P.x16) + k);
      reinterpret_cast<uint4*>(x16k)[k] = u;
      __half2 hh[4];
      memcpy(hh, &u, 16);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(hh[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
      }
    } else {
      const float4 a0 = __ldcg(reinterpret_cast<const float4*>(a) + 2 * k);
      const float4 a1 = __ldcg(reinterpret_cast<const float4*>(a) + 2 * k + 1);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      if (mode == X_ACC) {
        const float4 h0 = reinterpret_cast<const float4*>(hk)[2 * k], h1 = reinterpret_cast<const float4*>(hk)[2 * k + 1];
        const float hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        __half2 oh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          oh[e] = __floats2half2_rn(hv[2 * e] + av[2 * e], hv[2 * e + 1] + av[2 * e + 1]);
          const float2 f = __half22float2(oh[e]);
          v[2 * e] = f.x;
          v[2 * e + 1] = f.y;
        }
        uint4 o;
        memcpy(&o, oh, 16);
        reinterpret_cast<uint4*>(x16k)[k] = o;
      } else {
        const uint4 u = reinterpret_cast<const uint4*>(x16k)[k];
        __half2 hh[4];
        memcpy(hh, &u, 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(hh[e]);
          v[2 * e] = f.x + av[2 * e];
          v[2 * e + 1] = f.y + av[2 * e + 1];
        }
        reinterpret_cast<float4*>(hk)[2 * k] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(hk)[2 * k + 1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  consumer_sync();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
  const float r = rsqrtf(tot / static_cast<float>(P.d) + P.eps);
#pragma unroll
  for (int i = 0; i < kNormSlices; ++i) {  // the same trip count in every thread (shuffles below)
    const int k = i * kConsumers + tid;
    if (i * kConsumers >= n8) break;
    const bool live = k < n8;
    float sum = 0.f;
    if (live) {
      float v[8];  // the slice again, from shared memory (x16 or h)
      if (mode == H_ACC) {
        const float4 h0 = reinterpret_cast<const float4*>(hk)[2 * k], h1 = reinterpret_cast<const float4*>(hk)[2 * k + 1];
        v[0] = h0.x; v[1] = h0.y; v[2] = h0.z; v[3] = h0.w; v[4] = h1.x; v[5] = h1.y; v[6] = h1.z; v[7] = h1.w;
      } else {
        const uint4 u = reinterpret_cast<const uint4*>(x16k)[k];
        __half2 hh[4];
        memcpy(hh, &u, 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(hh[e]);
          v[2 * e] = f.x;
          v[2 * e + 1] = f.y;
        }
      }
      __half2 gh[4];
      memcpy(gh, &gpre[i], 16);
      __half2 oh[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 gg = __half22float2(gh[e]);
        oh[e] = __floats2half2_rn((v[2 * e] * r) * gg.x, (v[2 * e + 1] * r) * gg.y);
        const float2 f = __half22float2(oh[e]);
        sum += f.x + f.y;
      }
      uint4 o;
      memcpy(&o, oh, 16);
      reinterpret_cast<uint4*>(xs)[k] = o;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (live && (k & 7) == 0) xsum[(k >> 3) * 8] = sum;
  }
  consumer_sync();
}

// A batch of n chunks (n <= stages): chunk k is row tile rt0 + (k / nrc) * rts over groups g0 = (k % nrc) gchunk ..
// g0 + min(gchunk, gd - g0) of the staged input (xs, xsum) — the layout of the producer's pack_chunk sequence; the
// batch is described arithmetically, not by per-thread arrays (which would live in local memory, behind L1 misses
// to L2). Warp w works on chunk w % n (groups w / n, w / n + warps_k, ...); every warp waits for every chunk of the
// batch in order and releases it (the ring's rule: no release before the chunk landed). The per-row-tile sums over
// the warps land in uv[first chunk of the tile][16] (shared; 0 for a tile's other chunks), all consumer threads
// synchronised. Returns false if a wait gave up.
template <int BITS>
__device__ bool rows_batch(const Params& P, Cons& C, int n, int nrc, int rt0, int rts, uint32_t xs_addr,
                           uint32_t xsum_addr, float* uv, int mk = -1) {
  constexpr int TB = BITS == 4 ? 512 : 1024;
  (void)rt0;
  (void)rts;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r8 = lane >> 2, c4 = lane & 3;
  const int k = warp % n, sub = warp / n;
  const int wk = (kConsumerWarps - k + n - 1) / n;  // warps on chunk k
  float* red = reinterpret_cast<float*>(C.smem + C.Lo.red);
  float ys[4] = {0.f, 0.f, 0.f, 0.f}, yb[4] = {0.f, 0.f, 0.f, 0.f};
  bool ok = true;
  const int g0k = (k % nrc) * P.gchunk;
  const int gbk = min(P.gchunk, P.gd - g0k);
  int sl = C.slot;
  unsigned ph = C.phase;
  for (int q = 0; q < n; ++q, C.step(sl, ph)) {
    prof(P, R_ROWS);
    if (ok && !mbar_wait_abortable(&C.full[sl], ph, P)) ok = false;
    prof(P, R_ROWS_WAIT);
    if (q == 0 && mk >= 0) mark(P, mk);
    if (ok && q == k) {
      const uint32_t st = C.stage_addr(sl);
      uint32_t aw = st + sub * TB + lane * 16;
      uint32_t asb = st + kSbOff + sub * 64 + r8 * 8;
      uint32_t ax = xs_addr + (g0k + sub) * 128 + c4 * 32;
      uint32_t axs = xsum_addr + (g0k + sub) * 32 + c4 * 8;
#pragma unroll 1
      for (int g = sub; g < gbk; g += wk) {
        group_step<BITS, 1>(aw, asb, ax, axs, P.sdt, ys, yb);
        aw += wk * TB;
        asb += wk * 64;
        ax += wk * 128;
        axs += wk * 32;
      }
    }
    __syncwarp();
    if (lane == 0) gemv::mbar_arrive(&C.empty[sl]);
  }
  C.slot = sl;
  C.phase = ph;
  prof(P, R_ROWS);
  if (mk >= 0 && mk != 24) mark(P, mk + 1);
  if (c4 == 0) {
    red[warp * 16 + r8] = fmaf(ys[0], gemv::k2p24, yb[0]);
    red[warp * 16 + r8 + 8] = fmaf(ys[2], gemv::k2p24, yb[2]);
  }
  const bool fail = consumer_sync_or(!ok);
  // the sum over the warps of each row tile (the warps of all nrc chunks of the tile)
  for (int t = tid; t < n * 16; t += kConsumers) {
    const int kk = t / 16, r = t % 16;
    float s = 0.f;
    if (kk % nrc == 0)
      for (int w = 0; w < kConsumerWarps; ++w)
        if ((w % n) / nrc == kk / nrc) s += red[w * 16 + r];
    uv[t] = s;
  }
  consumer_sync();
  prof(P, R_REDUCE);
  return !fail;
}

// A chunk of nr row tiles x gb groups (tile (q, g) at (q gb + g) TB, scale/bias at kSbOff + q sb_stride + 64 g):
// with ks = min(gb, 16 / nr) K parts a row tile (1 when nr >= 16), work item w = (row tile w % nr, K part w / nr)
// goes to warp w mod 16, and each item's rows are added into acc[16 q + row] (fp32 reduction in L2) by the lanes that
// hold them (c4 == 0): the K parts meet in L2, no barrier.
template <int BITS>
__device__ bool owned_chunk(const Params& P, Cons& C, int nr, int gb, int sb_stride, uint32_t xs_addr,
                            uint32_t xsum_addr, float* acc) {
  constexpr int TB = BITS == 4 ? 512 : 1024;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r8 = lane >> 2, c4 = lane & 3;
  const int sl = C.slot;
  prof(P, R_OWNED);
  bool ok = mbar_wait_abortable(&C.full[sl], C.phase, P);
  prof(P, R_OWNED_WAIT);
  if (ok) {
    const uint32_t st = C.stage_addr(sl);
    const int ks = 1;  // (splitting o_proj's K over more warps measured no faster)
    for (int wi = warp; wi < nr * ks; wi += kConsumerWarps) {
      const int q = wi % nr, kp = wi / nr;
      float ys[4] = {0.f, 0.f, 0.f, 0.f}, yb[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t aw = st + (q * gb + kp) * TB + lane * 16;
      uint32_t asb = st + kSbOff + q * sb_stride + kp * 64 + r8 * 8;
      uint32_t ax = xs_addr + kp * 128 + c4 * 32;
      uint32_t axs = xsum_addr + kp * 32 + c4 * 8;
#pragma unroll 1
      for (int g = kp; g < gb; g += ks) {
        group_step<BITS, 1>(aw, asb, ax, axs, P.sdt, ys, yb);
        aw += ks * TB;
        asb += ks * 64;
        ax += ks * 128;
        axs += ks * 32;
      }
      // the tile's 16 rows through the warp's shared-memory slot to four lanes, one 4-float reduction each: every
      // unit of the phase adds into the same rows, and L2 serialises reductions per line, so 4x fewer operations
      float* wsl = reinterpret_cast<float*>(C.smem + C.Lo.red) + warp * 16;
      if (c4 == 0) {
        wsl[r8] = fmaf(ys[0], gemv::k2p24, yb[0]);
        wsl[r8 + 8] = fmaf(ys[2], gemv::k2p24, yb[2]);
      }
      __syncwarp();
      if (lane < 4) red_f32x4(acc + q * 16 + 4 * lane, reinterpret_cast<const float4*>(wsl)[lane]);
      __syncwarp();
    }
  }
  __syncwarp();
  if (lane == 0) gemv::mbar_arrive(&C.empty[sl]);
  C.step(C.slot, C.phase);
  return ok;
}

// ------------------------------------------------------------------------------------------------ attention (A)
// The CTA's keys [k0, k1) of KV group j against the group's G query heads; the CTA's partial (m, l, o) per head to
// P.apart. Warp w takes the 16-key tiles w, w + 16, ...; every warp waits for and releases every chunk.
template <int HD>
__device__ bool attention_split(const Params& P, Cons& C, const Sched& Sc, int l, int j, int s, int k0, int k1) {
  constexpr int KS = HD / 16;
  constexpr int NB = HD / 64;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int G = P.G;
  const int KC = kv_keys(P);
  const int pos = Sc.pos;
  const size_t kvbase = (static_cast<size_t>(l) * P.KVH + j) * P.cap * HD;
  float* ov = reinterpret_cast<float*>(C.smem + C.Lo.ov);     // [G][HD] fp32 (the CTA's rescaled o sum)
  float* om = reinterpret_cast<float*>(C.smem + C.Lo.om);     // [warp][8 heads][m, l]
  __half* qn = reinterpret_cast<__half*>(C.smem + C.Lo.xo);   // QK-norm: the group's q rows [G][HD] (fp16, scaled)
  __half* kn = reinterpret_cast<__half*>(C.smem + C.Lo.kn);   // and its new k row [HD]
  if (P.qkg) {
    // warp g < G: q head j G + g; warp G: k head j. RMS over HD in fp32, (x r) g, rotate-half RoPE at pos, fp16
    // (q scaled for the base-2 softmax) — the qkv epilogue's rounding points, after the per-head norm
    if (warp <= G) {
      const bool isq = warp < G;
      const int head = isq ? j * G + warp : P.H + j;
      const float* src = P.qkraw + static_cast<size_t>(head) * HD;
      const __half* gg = P.qkg + (static_cast<size_t>(l) * 2 + (isq ? 0 : 1)) * HD;
      constexpr int PER = HD / 64;   // RoPE pairs a lane: (i, i + HD/2) for i = lane, lane + 32 (HD 128)
      float a[PER], b[PER];
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        a[e] = __ldcg(src + lane + 32 * e);
        b[e] = __ldcg(src + HD / 2 + lane + 32 * e);
        ss = fmaf(a[e], a[e], fmaf(b[e], b[e], ss));
      }
      ss = warp_sum(ss);
      const float rn = rsqrtf(ss / static_cast<float>(HD) + P.eps);
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const int i = lane + 32 * e;
        const float y1 = (a[e] * rn) * __half2float(gg[i]), y2 = (b[e] * rn) * __half2float(gg[HD / 2 + i]);
        const float cs = P.cos_t[static_cast<size_t>(pos) * (HD / 2) + i];
        const float sn = P.sin_t[static_cast<size_t>(pos) * (HD / 2) + i];
        const float o1 = y1 * cs - y2 * sn, o2 = y2 * cs + y1 * sn;
        if (isq) {
          qn[warp * HD + i] = __float2half_rn(o1 * P.qscale);
          qn[warp * HD + HD / 2 + i] = __float2half_rn(o2 * P.qscale);
        } else {
          kn[i] = __float2half_rn(o1);
          kn[HD / 2 + i] = __float2half_rn(o2);
        }
      }
    }
    consumer_sync();
    // the CTA whose keys hold the new row writes it to the cache (later steps read it from there)
    if (pos >= k0 && pos < k1 && tid < HD / 8)
      reinterpret_cast<uint4*>(P.kc + kvbase + static_cast<size_t>(pos) * HD)[tid] = reinterpret_cast<const uint4*>(kn)[tid];
  }
  if (!P.qkg) {  // the group's q rows into shared memory: one round trip to L2 for the whole CTA
    const uint4* qsrc = reinterpret_cast<const uint4*>(P.q16 + static_cast<size_t>(j * G) * HD);
    for (int t = tid; t < G * HD / 8; t += kConsumers) reinterpret_cast<uint4*>(qn)[t] = __ldcg(qsrc + t);
    consumer_sync();
  }
  // Q^T fragments: lane (g8, t4) holds q[head g8][16 ks + 2 t4 + {0, 1, 8, 9}] (pre-scaled fp16)
  uint32_t qb[KS][2];
  {
    const bool live = g8 < G;
    const uint32_t* qsm = reinterpret_cast<const uint32_t*>(qn + (live ? g8 : 0) * HD);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qb[ks][0] = live ? qsm[ks * 8 + t4] : 0u;
      qb[ks][1] = live ? qsm[ks * 8 + 4 + t4] : 0u;
    }
  }
  for (int t = tid; t < G * HD; t += kConsumers) ov[t] = 0.f;
  prof(P, R_ATTN_Q);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float oacc[KS][4];
#pragma unroll
  for (int dt = 0; dt < KS; ++dt) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.f;
  const int ntile = (k1 - k0 + kKeyTile - 1) / kKeyTile;
  const int nch = (k1 - k0 + KC - 1) / KC;
  const int tpc = KC / kKeyTile;  // tiles per chunk
  bool ok = true;
  int sl = C.slot;
  unsigned ph = C.phase;
  for (int q = 0; q < nch; ++q, C.step(sl, ph)) {
    prof(P, R_ATTN_KEYS);
    if (ok && !mbar_wait_abortable(&C.full[sl], ph, P)) ok = false;
    prof(P, R_ATTN_WAIT);
    uint8_t* Ks = C.smem + C.Lo.ring + sl * kStage;
    uint8_t* Vs = Ks + NB * KC * 128;
    for (int tt = 0; tt < tpc && ok; ++tt) {
      const int t = q * tpc + tt;
      if (t >= ntile || (t % kConsumerWarps) != warp) continue;
      const int a = k0 + t * kKeyTile;      // the tile's first key
      const int n = min(kKeyTile, k1 - a);  // live keys in the tile
      const int row0 = tt * kKeyTile;       // its first row in the chunk
      // the new row (this step's qkv phase wrote it; read from L2) replaces the box's stale copy; V rows past the
      // live keys are zeroed (P = 0 there, and 0 x NaN would not vanish)
      if (pos >= a && pos < a + n) {
        for (int e = lane; e < 2 * HD / 8; e += 32) {
          const int kv = e / (HD / 8), cc = e % (HD / 8);
          const uint4 v = !kv && P.qkg ? reinterpret_cast<const uint4*>(kn)[cc]
                                       : __ldcg(reinterpret_cast<const uint4*>((kv ? P.vc : P.kc) + kvbase +
                                                                               static_cast<size_t>(pos) * HD) + cc);
          *reinterpret_cast<uint4*>((kv ? Vs : Ks) + (cc >> 3) * KC * 128 + swz(row0 + pos - a, cc)) = v;
        }
      }
      for (int e = lane; e < (kKeyTile - n) * (HD / 8); e += 32) {
        const int r = n + e / (HD / 8), cc = e % (HD / 8);
        *reinterpret_cast<uint4*>(Vs + (cc >> 3) * KC * 128 + swz(row0 + r, cc)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
      fence_proxy_async();  // generic writes into a stage that later bulk copies overwrite
      float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
      const int krow = row0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a0, a1, a2, a3;
        const int cc = ks * 2 + (lane >> 4);
        ldsm_x4(smem_u32(Ks + (cc >> 3) * KC * 128 + swz(krow, cc)), a0, a1, a2, a3);
        mma_16816(c0, c1, c2, c3, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
      }
      const bool va = g8 < n, vb = g8 + 8 < n;
      const float s0 = va ? c0 : -INFINITY, s1 = va ? c1 : -INFINITY;
      const float s2 = vb ? c2 : -INFINITY, s3 = vb ? c3 : -INFINITY;
      float x0 = fmaxf(s0, s2), x1 = fmaxf(s1, s3);
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
        x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
      }
      const float mn0 = fmaxf(m0, x0), mn1 = fmaxf(m1, x1);  // finite: key a is live
      const float al0 = ex2(m0 - mn0), al1 = ex2(m1 - mn1);
      const float p0 = ex2(s0 - mn0), p1 = ex2(s1 - mn1), p2 = ex2(s2 - mn0), p3 = ex2(s3 - mn1);
      l0 = fmaf(l0, al0, p0 + p2);
      l1 = fmaf(l1, al1, p1 + p3);
      m0 = mn0;
      m1 = mn1;
      const uint32_t pb0 = movm_t(pack_h2(p0, p1)), pb1 = movm_t(pack_h2(p2, p3));
      const int vrow = row0 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
      for (int dt = 0; dt < KS; ++dt) {
        oacc[dt][0] *= al0;
        oacc[dt][1] *= al1;
        oacc[dt][2] *= al0;
        oacc[dt][3] *= al1;
        uint32_t a0, a1, a2, a3;
        const int cc = dt * 2 + ((lane >> 3) & 1);
        ldsm_x4_t(smem_u32(Vs + (cc >> 3) * KC * 128 + swz(vrow, cc)), a0, a1, a2, a3);
        mma_16816(oacc[dt][0], oacc[dt][1], oacc[dt][2], oacc[dt][3], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncwarp();
    if (lane == 0) gemv::mbar_arrive(&C.empty[sl]);
  }
  C.slot = sl;
  C.phase = ph;
  prof(P, R_ATTN_KEYS);
  mark(P, l * kTraceMarks + 10);
  // l over the warp's key rows (lanes with the same t4), then the CTA's combination: M = max over warps, each warp
  // adds its o scaled by 2^(m_w - M) into ov (shared-memory atomics)
#pragma unroll
  for (int off = 4; off <= 16; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  if (g8 == 0) {
    om[(warp * 8 + 2 * t4) * 2] = m0;
    om[(warp * 8 + 2 * t4) * 2 + 1] = l0;
    om[(warp * 8 + 2 * t4 + 1) * 2] = m1;
    om[(warp * 8 + 2 * t4 + 1) * 2 + 1] = l1;
  }
  const bool fail = consumer_sync_or(!ok);
  if (fail) return false;
  // per head h (thread h): M = the max over the warps, L = sum_w l_w 2^(m_w - M)
  float* mh = om + kConsumerWarps * 16;  // [8] M, then [8] L
  if (tid < G) {
    float M = -INFINITY;
#pragma unroll 4
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, om[(w * 8 + tid) * 2]);
    float Ls = 0.f;
#pragma unroll 4
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float mw = om[(w * 8 + tid) * 2];
      if (mw != -INFINITY) Ls = fmaf(om[(w * 8 + tid) * 2 + 1], ex2(mw - M), Ls);
    }
    mh[tid] = M;
    mh[8 + tid] = Ls;
  }
  consumer_sync();
  const float M0 = mh[2 * t4 < G ? 2 * t4 : 0], M1 = mh[2 * t4 + 1 < G ? 2 * t4 + 1 : 0];
  const float f0 = m0 == -INFINITY ? 0.f : ex2(m0 - M0), f1 = m1 == -INFINITY ? 0.f : ex2(m1 - M1);
  if (m0 != -INFINITY || m1 != -INFINITY) {
#pragma unroll
    for (int dt = 0; dt < KS; ++dt) {
      if (2 * t4 < G) {
        atomicAdd(&ov[(2 * t4) * HD + 16 * dt + g8], oacc[dt][0] * f0);
        atomicAdd(&ov[(2 * t4) * HD + 16 * dt + g8 + 8], oacc[dt][2] * f0);
      }
      if (2 * t4 + 1 < G) {
        atomicAdd(&ov[(2 * t4 + 1) * HD + 16 * dt + g8], oacc[dt][1] * f1);
        atomicAdd(&ov[(2 * t4 + 1) * HD + 16 * dt + g8 + 8], oacc[dt][3] * f1);
      }
    }
  }
  consumer_sync();
  prof(P, R_ATTN_MERGE);
  // the CTA's partial: per head (M, L, o[HD])
  float* dst = P.apart + (static_cast<size_t>(j) * P.smax + s) * G * (HD + 2);
#pragma unroll 1
  for (int t = tid; t < G * (HD + 2); t += kConsumers) {
    const int g = t / (HD + 2), e = t % (HD + 2);
    dst[t] = e == 0 ? mh[g] : e == 1 ? mh[8 + g] : ov[g * HD + e - 2];
  }
  return true;
}

// ------------------------------------------------------------------------------------------------ the kernel
template <int BITS, int HD>
__global__ void __launch_bounds__(kThreads, 1) fstep_kernel(const __grid_constant__ Params P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x, grid = gridDim.x;
  const Layout Lo = smem_layout(P.d, P.G * HD, P.stages);
  __shared__ __align__(8) uint64_t bars[2 * kMaxRing];
  __shared__ int sh_flag, sh_dead;
  __shared__ __align__(8) SigQueue sq;
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxRing;
  const unsigned epoch = P.sync[0];
  const unsigned par = epoch & 1u;
  unsigned* ctr = P.sync + 64 + par * P.nctr;
  const int CL = ctr_per_layer(P.KVH);
  float* acc = P.acc + static_cast<size_t>(par) * 2 * P.L * P.d;     // [h, x][L][d]
  Sched Sc;
  Sc.init(P);

  if (tid == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < kSigSlots; ++s) {
      mbar_init(&sq.full[s], 1);
      mbar_init(&sq.empty[s], 1);
    }
    sh_dead = 0;
    fence_mbar_init();
  }
  // the next step's counter and accumulator set, cleared now (the previous step finished with it)
  {
    unsigned* oc = P.sync + 64 + (par ^ 1u) * P.nctr;
    for (int t = c * kThreads + tid; t < P.nctr; t += grid * kThreads) oc[t] = 0u;
    float4* oa = reinterpret_cast<float4*>(P.acc + static_cast<size_t>(par ^ 1u) * 2 * P.L * P.d);
    const int n4 = 2 * P.L * P.d / 4;
    for (int t = c * kThreads + tid; t < n4; t += grid * kThreads) oa[t] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();

  if (warp == kSignalWarp) {
    if (lane == 0) {
      for (long n = 0;; ++n) {
        const int sl = static_cast<int>(n % kSigSlots);
        if (!mbar_wait_abortable(&sq.full[sl], static_cast<unsigned>((n / kSigSlots) & 1), P)) break;
        unsigned* a = sq.addr[sl];
        const unsigned v = sq.val[sl];
        gemv::mbar_arrive(&sq.empty[sl]);
        if (!a) break;
        red_rel(a, v);
      }
    }
    return;
  }
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      Prod pr;
      pr.ring = smem + Lo.ring;
      pr.full = full;
      pr.empty = empty;
      pr.dead = &sh_dead;
      pr.stages = P.stages;
      produce<BITS, HD>(P, Sc, pr);
      // no copy of this CTA may land after it leaves: wait (bounded) for the last chunk issued into every stage
      for (int st = 0; st < P.stages && st < pr.issued; ++st) {
        const long last = pr.issued - 1 - ((pr.issued - 1 - st) % P.stages);
        mbar_wait_bounded(&full[st], static_cast<unsigned>((last / P.stages) & 1), nullptr, 100000000ull);
      }
    }
    return;
  }

  long nsig = 0;  // thread 0: signals posted
  auto post = [&](unsigned* a, unsigned v) {  // thread 0, after a consumer barrier
    const int sl = static_cast<int>(nsig % kSigSlots);
    if (nsig >= kSigSlots && !mbar_wait_abortable(&sq.empty[sl], static_cast<unsigned>(((nsig / kSigSlots) - 1) & 1), P))
      return;
    sq.addr[sl] = a;
    sq.val[sl] = v;
    gemv::mbar_arrive(&sq.full[sl]);
    ++nsig;
  };
  Cons C;
  C.smem = smem;
  C.Lo = Lo;
  C.full = full;
  C.empty = empty;
  C.flag = &sh_flag;
  C.dead = &sh_dead;
  C.stages = P.stages;
  __half* x16k = reinterpret_cast<__half*>(smem + Lo.x16k);
  float* hk = reinterpret_cast<float*>(smem + Lo.hk);
  const uint32_t xs_a = smem_u32(smem + Lo.xs), xsum_a = smem_u32(smem + Lo.xsum);
  float* uv = reinterpret_cast<float*>(smem + Lo.red) + kConsumerWarps * 16;  // batch results [n][16]
  float* misc = reinterpret_cast<float*>(smem + Lo.misc);
  const int TPS = tps(BITS);
  const int nrc = row_chunks(P);
  bool ok = true;

  // the CTA's qkv row tiles c, c + grid, ... (kMaxQkvTiles at most, checked on the host)
  const int nq = c < P.rt_qkv ? (P.rt_qkv - 1 - c) / grid + 1 : 0;
  prof_begin(P);
  for (int l = 0; l < P.L && ok; ++l) {
    prof(P, R_TOP);
    const __half* g1 = P.gains + static_cast<size_t>(l) * 2 * P.d;
    const __half* g2 = g1 + P.d;
    float* acc_h = acc + static_cast<size_t>(l) * P.d;
    float* acc_x = acc + static_cast<size_t>(P.L + l) * P.d;
    // operands that do not depend on the step's activations, loaded before the dependency waits: the norm gains
    // (a thread's 8-element slices) and, for thread 8 ti + r (r < 8), row pair r of its qkv tile ti: bias and the
    // RoPE (cos, sin) at this position
    uint4 gpre1[kNormSlices];
    norm_gains(P, g1, gpre1);
    float eb1 = 0.f, eb2 = 0.f, ecs = 1.f, esn = 0.f;
    const int eti = tid >> 3, er = tid & 7;
    const int et = c + eti * grid;
    const int ehead = et * 16 / HD, ett = (et * 16 % HD) / 16;
    const int ei1 = 8 * ett + er, ei2 = HD / 2 + 8 * ett + er;
    if (tid < 8 * nq) {
      if (P.bias) {
        const __half* b = P.bias + static_cast<size_t>(l) * P.rt_qkv * 16;
        eb1 = __half2float(b[ehead * HD + ei1]);
        eb2 = __half2float(b[ehead * HD + ei2]);
      }
      if (ehead < P.H + P.KVH && !P.qkg) {
        ecs = P.cos_t[static_cast<size_t>(Sc.pos) * (HD / 2) + ei1];
        esn = P.sin_t[static_cast<size_t>(Sc.pos) * (HD / 2) + ei1];
      }
    }
    prof(P, R_PRELOAD);
    // ---------------- Q
    if (l > 0) {
      if (!wait_counter(ctr + (l - 1) * CL + 2 * P.KVH + 1, static_cast<unsigned>(P.nf), P, C.flag)) { ok = false; break; }
      prof(P, R_WAIT);
    }
    mark(P, l * kTraceMarks + 0);
    stage_input(P, C, l == 0 ? X_LOAD : X_ACC, acc + static_cast<size_t>(P.L + l - 1) * P.d, gpre1);
    prof(P, R_NORM);
    mark(P, l * kTraceMarks + 8);
    if (nq > 0) {
      // every qkv tile of the CTA in one batch
      if (!rows_batch<BITS>(P, C, nq * nrc, nrc, c, grid, xs_a, xsum_a, uv, l * kTraceMarks + 20)) { ok = false; break; }
      mark(P, l * kTraceMarks + 9);
      // epilogue: per tile 8 RoPE pairs (tile rows r, r + 8 = logical rows 8 tt + r, hd/2 + 8 tt + r of the head)
      if (tid < 8 * nq) {
        const float y1 = uv[(eti * nrc) * 16 + er] + eb1, y2 = uv[(eti * nrc) * 16 + er + 8] + eb2;
        if (ehead < P.H + P.KVH && P.qkg) {
          // QK-norm: the head's norm needs all its rows; the attention phase finishes q and k from these
          P.qkraw[ehead * HD + ei1] = y1;
          P.qkraw[ehead * HD + ei2] = y2;
        } else if (ehead < P.H + P.KVH) {
          const float o1 = y1 * ecs - y2 * esn, o2 = y2 * ecs + y1 * esn;
          if (ehead < P.H) {
            P.q16[ehead * HD + ei1] = __float2half_rn(o1 * P.qscale);
            P.q16[ehead * HD + ei2] = __float2half_rn(o2 * P.qscale);
          } else {
            __half* kr = P.kc + ((static_cast<size_t>(l) * P.KVH + ehead - P.H) * P.cap + Sc.pos) * HD;
            kr[ei1] = __float2half_rn(o1);
            kr[ei2] = __float2half_rn(o2);
          }
        } else {
          __half* vr = P.vc + ((static_cast<size_t>(l) * P.KVH + ehead - P.H - P.KVH) * P.cap + Sc.pos) * HD;
          vr[ei1] = __float2half_rn(y1);
          vr[ei2] = __float2half_rn(y2);
        }
      }
      consumer_sync();
      prof(P, R_QKV_EPI);
      if (tid == 0)  // release: the CTA's stores above are ordered before each count (barrier + cumulativity)
        for (int ti = 0; ti < nq; ++ti) {
          const int head = (c + ti * grid) * 16 / HD;
          const int grp = head < P.H ? head / P.G : head < P.H + P.KVH ? head - P.H : head - P.H - P.KVH;
          post(ctr + l * CL + grp, 1u);
        }
      prof(P, R_SIGNAL);
    }
    if (!ok) break;
    mark(P, l * kTraceMarks + 1);
    // ---------------- A
    int j, s, k0, k1;
    const bool has_attn = Sc.attn(P, c, &j, &s, &k0, &k1);
    if (has_attn) {
      const unsigned qkv_tiles = static_cast<unsigned>((P.G + 2) * HD / 16);
      if (!wait_counter(ctr + l * CL + j, qkv_tiles, P, C.flag)) { ok = false; break; }
      prof(P, R_WAIT);
      mark(P, l * kTraceMarks + 2);
      if (!attention_split<HD>(P, C, Sc, l, j, s, k0, k1)) { ok = false; break; }
      consumer_sync();
      prof(P, R_ATTN_OUT);
      if (tid == 0) post(ctr + l * CL + P.KVH + j, 1u);
      prof(P, R_SIGNAL);
      mark(P, l * kTraceMarks + 3);
      // ---------------- O
      int r0, r1;
      Sc.orows(P, s, &r0, &r1);
      if (r1 > r0) {
        if (!wait_counter(ctr + l * CL + P.KVH + j, static_cast<unsigned>(Sc.S), P, C.flag)) { ok = false; break; }
        prof(P, R_WAIT);
        mark(P, l * kTraceMarks + 4);
        // merge the group's S partials: attn = fp16(sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M)). Warp g: head g's
        // S (m, l) pairs at once, its weights 2^(m_s - M) and sum L to shared memory (hk: h is rebuilt in F); then
        // every element's S o values at once
        __half* xo = reinterpret_cast<__half*>(smem + Lo.xo);
        float* xsumo = reinterpret_cast<float*>(smem + Lo.xsumo);
        float* wq = hk;                                   // [G][S] weights, then [G] sums at wq + G S
        const float* src = P.apart + static_cast<size_t>(j) * P.smax * P.G * (HD + 2);
        const int KA = P.G * HD, S_ = Sc.S;
        for (int g = warp; g < P.G; g += kConsumerWarps) {
          float M = -INFINITY;
          for (int q = lane; q < S_; q += 32) M = fmaxf(M, __ldcg(src + (static_cast<size_t>(q) * P.G + g) * (HD + 2)));
          M = warp_max(M);
          float Ls = 0.f;
          for (int q = lane; q < S_; q += 32) {
            const float* pq = src + (static_cast<size_t>(q) * P.G + g) * (HD + 2);
            const float mq = __ldcg(pq);
            const float w = mq == -INFINITY ? 0.f : ex2(mq - M);
            wq[g * S_ + q] = w;
            Ls = fmaf(__ldcg(pq + 1), w, Ls);
          }
          Ls = warp_sum(Ls);
          if (lane == 0) wq[P.G * S_ + g] = Ls;
        }
        consumer_sync();
        for (int t = tid; t < KA; t += kConsumers) {
          const int g = t / HD, e = t % HD;
          const float* pe = src + static_cast<size_t>(g) * (HD + 2) + 2 + e;
          const float* wg = wq + g * S_;
          float Os = 0.f;
#pragma unroll 8
          for (int q = 0; q < S_; ++q) Os = fmaf(__ldcg(pe + static_cast<size_t>(q) * P.G * (HD + 2)), wg[q], Os);
          xo[t] = __float2half_rn(Os / wq[P.G * S_ + g]);
        }
        consumer_sync();
        for (int g = warp; g < KA / 64; g += kConsumerWarps) {
          const float2 f = __half22float2(reinterpret_cast<const __half2*>(xo + g * 64)[lane]);
          const float sm = warp_sum(f.x + f.y);
          if (lane == 0) xsumo[g * 8] = sm;
        }
        consumer_sync();
        prof(P, R_O_MERGE);
        mark(P, l * kTraceMarks + 11);
        for (int r = r0; r < r1 && ok; r += P.o_per) {
          const int nr = min(P.o_per, r1 - r);
          ok = owned_chunk<BITS>(P, C, nr, P.gk, P.o_sb, smem_u32(xo), smem_u32(xsumo), acc_h + r * 16);
        }
        if (consumer_sync_or(!ok)) { ok = false; break; }
        prof(P, R_OWNED);
        if (tid == 0) post(ctr + l * CL + 2 * P.KVH, static_cast<unsigned>(r1 - r0));
        prof(P, R_SIGNAL);
        mark(P, l * kTraceMarks + 5);
      }
    }
    // ---------------- F
    uint4 gpre2[kNormSlices];  // loaded here, not at the layer's start: no registers held through the attention
    norm_gains(P, g2, gpre2);
    if (!wait_counter(ctr + l * CL + 2 * P.KVH, static_cast<unsigned>(P.KVH * P.rt_d), P, C.flag)) { ok = false; break; }
    prof(P, R_WAIT);
    mark(P, l * kTraceMarks + 6);
    stage_input(P, C, H_ACC, acc_h, gpre2);
    prof(P, R_NORM);
    mark(P, l * kTraceMarks + 12);
    for (int f = c; f < P.nf && ok; f += grid) {
      // gate/up: row tiles 8f .. 8f + 7 (pairs: gate tile 2p, up tile 2p + 1), ppb pairs a batch (all four when
      // their chunks fit the ring); warp 0 forms act = fp16(SiLU(gate) up) of each batch and, after the last, the
      // group sum of act for down
      __half* act = reinterpret_cast<__half*>(smem + Lo.act);
      float* xsuma = reinterpret_cast<float*>(smem + Lo.xsuma);
      const int cap_chunks = min(16, P.stages);
      const int ppb = 8 * nrc <= cap_chunks ? 4 : 4 * nrc <= cap_chunks ? 2 : 1;
      for (int pb = 0; pb < 4 && ok; pb += ppb) {
        if (!rows_batch<BITS>(P, C, 2 * ppb * nrc, nrc, 8 * f + 2 * pb, 1, xs_a, xsum_a, uv,
                              f == c && pb == 0 ? l * kTraceMarks + 22 : -1)) { ok = false; break; }
        // uv: [chunk][16]; the first chunk of row tile q of this batch is q * nrc
        if (warp == 0) {
          for (int e = lane; e < ppb * 16; e += 32) {
            const int pp = e / 16, r = e % 16;  // pair pb + pp of the unit
            const float g = uv[(2 * pp) * nrc * 16 + r], u = uv[(2 * pp + 1) * nrc * 16 + r];
            act[(pb + pp) * 16 + r] = __float2half_rn(gemv::silu_f(g) * u);
          }
          if (pb + ppb == 4) {
            __syncwarp();
            const float2 fv = __half22float2(reinterpret_cast<const __half2*>(act)[lane]);
            const float sm = warp_sum(fv.x + fv.y);
            if (lane == 0) xsuma[0] = sm;
          }
        }
      }
      if (!ok) break;
      consumer_sync();  // act and its sum for every warp
      prof(P, R_SILU);
      if (f == c) mark(P, l * kTraceMarks + 14);
      // down: K slice f (one group) of every row tile, dn_rows row tiles a chunk
      for (int r = 0; r < P.rt_d && ok; r += P.dn_rows) {
        const int nr = min(P.dn_rows, P.rt_d - r);
        ok = owned_chunk<BITS>(P, C, nr, 1, 64, smem_u32(act), smem_u32(xsuma), acc_x + r * 16);
        if (r == 0 && f == c) mark(P, l * kTraceMarks + 15);
      }
      if (consumer_sync_or(!ok)) { ok = false; break; }
      prof(P, R_OWNED);
      if (tid == 0) post(ctr + l * CL + 2 * P.KVH + 1, 1u);
      prof(P, R_SIGNAL);
    }
    if (!ok) break;
    mark(P, l * kTraceMarks + 7);
  }

  // ---------------- head
  prof(P, R_TOP);
  uint4 gfin[kNormSlices];
  norm_gains(P, P.final_gain, gfin);
  prof(P, R_PRELOAD);
  if (ok && !wait_counter(ctr + (P.L - 1) * CL + 2 * P.KVH + 1, static_cast<unsigned>(P.nf), P, C.flag)) ok = false;
  prof(P, R_WAIT);
  if (ok) {
    mark(P, P.L * kTraceMarks + 0);
    stage_input(P, C, X_ACC, acc + static_cast<size_t>(2 * P.L - 1) * P.d, gfin);
    prof(P, R_NORM);
    float bv = -INFINITY;  // thread 0's running first maximum of the CTA's rows
    int bi = 0x7fffffff;
    const int h0 = static_cast<int>(static_cast<long long>(c) * P.rt_v / grid);
    const int h1 = static_cast<int>(static_cast<long long>(c + 1) * P.rt_v / grid);
    const int nmax = max(1, min(8, (P.stages / 2) / nrc));  // row tiles a batch: the next batch streams meanwhile
    for (int t0 = h0; t0 < h1 && ok; t0 += nmax) {
      const int nt = min(nmax, h1 - t0);
      if (!rows_batch<BITS>(P, C, nt * nrc, nrc, t0, 1, xs_a, xsum_a, uv)) { ok = false; break; }
      if (warp == 0) {
        float v = -INFINITY;
        int vi = 0x7fffffff;
        for (int e = lane; e < nt * 16; e += 32) {
          const int q = e / 16, r = e % 16;
          const float y = uv[(q * nrc) * 16 + r];
          const int idx = (t0 + q) * 16 + r;
          if (P.logits) P.logits[idx] = y;
          if (y > v) { v = y; vi = idx; }  // ascending per lane: the first of equal values stays
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
          const float o = __shfl_xor_sync(0xffffffffu, v, m);
          const int oi = __shfl_xor_sync(0xffffffffu, vi, m);
          if (o > v || (o == v && oi < vi)) { v = o; vi = oi; }
        }
        if (v > bv || (v == bv && vi < bi)) { bv = v; bi = vi; }
      }
      consumer_sync();
      prof(P, R_HEAD);
    }
    if (tid == 0) {
      P.pairs[2 * c] = bv;
      P.pairs[2 * c + 1] = __int_as_float(bi);
    }
  }
  if (tid == 0) post(nullptr, 0u);  // the signal warp's last entry
  if (consumer_sync_or(!ok)) {
    *C.dead = 1;  // the producer stops at its next stage
    return;
  }
  prof(P, R_TAIL);
  prof_end(P);
  mark(P, P.L * kTraceMarks + 1);
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(ctr + P.L * CL, 1u);
    *C.flag = prev == static_cast<unsigned>(grid) - 1;
  }
  consumer_sync();
  if (!*C.flag) return;
  // the last CTA: the grid's first maximum and the generation step
  __threadfence();
  if (warp == 0) {
    float v = -INFINITY;
    int vi = 0x7fffffff;
    for (int q = lane; q < grid; q += 32) {
      const float y = __ldcg(P.pairs + 2 * q);
      const int yi = __float_as_int(__ldcg(P.pairs + 2 * q + 1));
      if (y > v || (y == v && yi < vi)) { v = y; vi = yi; }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float o = __shfl_xor_sync(0xffffffffu, v, m);
      const int oi = __shfl_xor_sync(0xffffffffu, vi, m);
      if (o > v || (o == v && oi < vi)) { v = o; vi = oi; }
    }
    if (lane == 0) {
      const uint32_t pos = P.q0[0];
      const uint32_t p1 = pos + 1;
      uint32_t f = P.force_next ? P.force_next[0] : kTokenUnset;
      if (P.force_next) P.force_next[0] = kTokenUnset;
      if (f == kTokenUnset && p1 < static_cast<uint32_t>(P.cap)) f = P.log[p1];
      uint32_t tok = f != kTokenUnset ? f : static_cast<uint32_t>(vi);
      if (tok >= static_cast<uint32_t>(P.V)) {
        atomicOr(P.err, kErrBadToken);
        tok = 0;
      }
      if (p1 < static_cast<uint32_t>(P.cap)) P.log[p1] = tok;
      P.q0[0] = p1 < static_cast<uint32_t>(P.cap) ? p1 : static_cast<uint32_t>(P.cap - 1);
      if (P.tok_out) P.tok_out[0] = static_cast<int32_t>(tok);
      misc[0] = __int_as_float(static_cast<int>(tok));
    }
  }
  consumer_sync();
  const int tok = __float_as_int(misc[0]);
  for (int k = tid; k < P.d / 8; k += kConsumers)
    reinterpret_cast<uint4*>(P.x16)[k] = reinterpret_cast<const uint4*>(P.embed + static_cast<size_t>(tok) * P.d)[k];
  if (tid == 0) P.sync[0] = epoch + 1u;
}

}  // namespace fstep

// ------------------------------------------------------------------------------------------------ host side
namespace {

using fstep::Params;

template <int BITS, int HD>
int fstep_allow(int optin) {
  auto kern = fstep::fstep_kernel<BITS, HD>;
  cudaFuncAttributes fa;
  AGXC_CUDA(cudaFuncGetAttributes(&fa, kern));
  AGXC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - static_cast<int>(fa.sharedSizeBytes)));
  return 0;
}

template <int BITS, int HD>
int fstep_launch_t(const Params& p, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(fstep::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, fstep::fstep_kernel<BITS, HD>, p));
  return 0;
}

}  // namespace

// The shared memory one CTA of the fused step needs with `stages` ring stages, plus the 1,024-byte alignment slack.
size_t fstep_smem(int d, int G, int hd, int stages) {
  return static_cast<size_t>(fstep::smem_layout(d, G * hd, stages).total) + 1024;
}

// The deepest ring (up to kMaxRing stages) that fits the device's opt-in shared memory; 0 if fewer than 4 fit.
int fstep_stages(const agxc_ctx* ctx, int d, int G, int hd) {
  // the kernel's static shared memory (barriers, the signal queue, the profile), the largest of the instantiations
  size_t fixed = 0;
  for (auto kern : {fstep::fstep_kernel<4, 64>, fstep::fstep_kernel<4, 128>, fstep::fstep_kernel<8, 64>,
                    fstep::fstep_kernel<8, 128>}) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    fixed = std::max(fixed, static_cast<size_t>(fa.sharedSizeBytes));
  }
  for (int st = fstep::kMaxRing; st >= 4; --st)
    if (fstep_smem(d, G, hd, st) + fixed <= static_cast<size_t>(ctx->max_smem_optin)) return st;
  return 0;
}

int fstep_configure(const agxc_ctx* ctx) {
  const int o = ctx->max_smem_optin;
  int rc;
  if ((rc = fstep_allow<4, 128>(o)) || (rc = fstep_allow<4, 64>(o)) || (rc = fstep_allow<8, 128>(o)) ||
      (rc = fstep_allow<8, 64>(o)))
    return rc;
  return 0;
}

int fstep_launch(const FstepArgs& a, cudaStream_t s) {
  Params p;
  p.L = a.L; p.d = a.d; p.H = a.H; p.KVH = a.KVH; p.hd = a.hd; p.G = a.H / a.KVH; p.F = a.F; p.V = a.V;
  p.cap = a.cap; p.bits = a.bits; p.sdt = a.sdt; p.stages = a.stages; p.eps = a.eps; p.wait_ns = a.wait_ns;
  p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(a.hd)));
  p.rt_qkv = (a.H + 2 * a.KVH) * a.hd / 16;
  p.rt_d = a.d / 16;
  p.nf = a.F / 64;
  p.rt_v = a.V / 16;
  p.gd = a.d / 64;
  p.gk = p.G * a.hd / 64;
  p.gchunk = std::min(p.gd, fstep::tps(a.bits));
  p.dn_rows = std::min(p.rt_d, fstep::tps(a.bits));
  p.o_sb = (p.gk * 64 + 127) / 128 * 128;
  p.o_per = std::max(1, std::min(fstep::tps(a.bits) / p.gk, (fstep::kStage - fstep::kSbOff) / p.o_sb));
  p.smax = a.smax;
  p.maps = a.maps; p.gains = a.gains; p.bias = a.bias; p.final_gain = a.final_gain; p.embed = a.embed;
  p.qkg = a.qkg; p.qkraw = a.qkraw;
  p.kc = a.kc; p.vc = a.vc; p.cos_t = a.cos_t; p.sin_t = a.sin_t; p.q0 = a.q0; p.log = a.log; p.tok_out = a.tok_out;
  p.force_next = a.force_next; p.x16 = a.x16; p.logits = a.logits; p.q16 = a.q16; p.apart = a.apart; p.acc = a.acc;
  p.sync = a.sync; p.nctr = a.nctr; p.pairs = a.pairs; p.err = a.err; p.trace = a.trace;
  const size_t smem = fstep_smem(a.d, p.G, a.hd, a.stages);
  if (a.bits == 4 && a.hd == 128) return fstep_launch_t<4, 128>(p, a.grid, smem, s);
  if (a.bits == 4 && a.hd == 64) return fstep_launch_t<4, 64>(p, a.grid, smem, s);
  if (a.bits == 8 && a.hd == 128) return fstep_launch_t<8, 128>(p, a.grid, smem, s);
  if (a.bits == 8 && a.hd == 64) return fstep_launch_t<8, 64>(p, a.grid, smem, s);
  return fail(AGXC_EINVAL, "fused step: 4- or 8-bit weights, head_dim 64 or 128");
}

// Counter words of one parity set (rounded to 32).
int fstep_counters(int L, int KVH) { return (L * fstep::ctr_per_layer(KVH) + 1 + 31) / 32 * 32; }
int fstep_trace_marks(int L) { return L * fstep::kTraceMarks + 2 + fstep::kProfRegions; }
int fstep_map_count() { return fstep::kMaps; }
int fstep_tiles_per_stage(int bits) { return fstep::tps(bits); }
int fstep_max_d() { return fstep::kNormSlices * fstep::kConsumers * 8; }

}  // namespace agxc
