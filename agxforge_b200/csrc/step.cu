// step.cu — one decode step of a batch-1 model as ONE persistent cooperative kernel (the reference's per-token
// command buffer of the whole model, tools/g17decodegen.m:167-199, as a single B200 launch).
//
// The step is a program of PHASES, per layer: qkv (RMSNorm + GEMV + bias + RoPE + KV append), attention, o_proj
// (+ residual), gate/up (RMSNorm + GEMV + SiLU * up), down (+ residual); then the head (final norm + vocab GEMV +
// first argmax + the generation step). One CTA per SM runs every phase; a grid barrier separates consecutive phases
// (each reads what the previous one wrote). Within a CTA:
//   * the PRODUCER warp streams, in phase order, every weight chunk of the CTA's GEMV units and the cached K/V rows
//     of its attention chunk into a ring of shared-memory stages (plain bulk copies: a pack's tiles are row-tile
//     major, so a chunk is one contiguous range per row tile). Weights and the cache history do not depend on the
//     step's activations, so the producer runs ahead of the consumers across phase boundaries, limited only by the
//     ring: while the consumers wait at a grid barrier, HBM keeps streaming the next phases.
//   * 16 CONSUMER warps run the phases with the GEMV and attention arithmetic of the per-phase kernels (the tile
//     step, epilogues and generation step of gemv_impl.cuh; the tensor-core attention tile), reading activations
//     through L2 (other CTAs wrote them).
// Attention splits each KV head's live keys over S CTAs; the chunks meet in global memory, merged by the last CTA of
// the head to finish (a counter). The head's per-CTA maxima meet the same way. Every wait is bounded and the first
// timeout raises an abort bit that every other wait honours, so a failed step ends in milliseconds, not hangs.
#include <algorithm>
#include <vector>

#include "gemv_impl.cuh"

namespace agxc {
namespace step {

using gemv::kConsumers;
using gemv::kConsumerWarps;
using gemv::kThreads;
using gemv::consumer_sync;

constexpr int kStageBytes = 36864;  // one chunk: 2 row tiles x 32 groups at 4 bits (x 16 at 8 bits), or 64 keys of K
                                    // and V at head_dim 128
constexpr int kMaxRing = 8;         // stages at most (the ring is as deep as shared memory allows)
constexpr int kAttnKeys = 64;       // keys per attention sub-chunk
constexpr int kAttnWarps = 4;       // warps with a 16-key tile of a sub-chunk
constexpr int kUnitBatch = 8;       // GEMV units whose partial rows wait in shared memory for one finalisation

struct Smem {
  int full, empty, misc, phase, xs, xsum, red, pbuf, uvw, ring, total;
};
constexpr int kPhaseBytes = (static_cast<int>(sizeof(StepPhase)) + 127) / 128 * 128;
constexpr int kDescRing = 8;  // phase descriptors the producer may bring in ahead of the consumers
static_assert(sizeof(StepPhase) % 16 == 0, "phase descriptors move by bulk copy");

__host__ __device__ inline Smem smem_layout(int kmax, int stages) {
  Smem L;
  L.full = 0;
  L.empty = 8 * kMaxRing;                                   // then the descriptor ring's full / empty barriers
  L.misc = 16 * kMaxRing + 16 * kDescRing;                  // 1 KB: argmax state (per warp), flags
  L.phase = L.misc + 1024;                                  // the descriptor ring
  L.xs = L.phase + kDescRing * kPhaseBytes;                 // activation row fp16 (+16 B pad) / attention scratch
  const int attn_scratch = kAttnWarps * 8 * 128 * 4 + 2 * kAttnWarps * 8 * 4;
  const int xs_bytes = kmax * 2 + 16 > attn_scratch ? kmax * 2 + 16 : attn_scratch;
  L.xsum = L.xs + (xs_bytes + 127) / 128 * 128;
  L.red = L.xsum + (kmax / 64) * 8 * 4;
  L.pbuf = L.red + kConsumerWarps * 4;                      // [kUnitBatch][warp][16 rows] partial rows
  L.uvw = L.pbuf + kUnitBatch * kConsumerWarps * 16 * 4;    // [warp][32] a finalised unit's rows
  L.ring = (L.uvw + kConsumerWarps * 32 * 4 + 1023) / 1024 * 1024;
  L.total = L.ring + stages * kStageBytes;
  return L;
}

// The deepest ring that fits `optin` bytes of shared memory (with `static_bytes` of static shared memory).
inline int ring_stages(int kmax, int optin, int static_bytes) {
  int st = kMaxRing;
  while (st > 2 && smem_layout(kmax, st).total + static_bytes > optin) --st;
  return st;
}

// Grid barrier among the consumers of every CTA: arrivals count up monotonically during the launch; barrier e waits
// for e * gridDim.x arrivals. Bounded, and abandoned as soon as any CTA raised the abort bit.
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool grid_barrier(unsigned* bar, unsigned target, unsigned* err) {
  consumer_sync();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    // the arrival releases this CTA's writes (the named barrier above ordered every consumer's before it)
    unsigned prev;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(bar) : "memory");
    int ok = 1;
    if (prev + 1 < target) {
      const uint64_t t0 = globaltimer_ns();
      for (unsigned it = 0;; ++it) {
        if (ld_acquire(bar) >= target) break;
        if ((it & 15u) == 15u) {
          if (ld_acquire(err) & kErrAbort) { ok = 0; break; }
          if (globaltimer_ns() - t0 > 2000000000ull) {
            atomicOr(err, kErrGridTimeout | kErrAbort);
            ok = 0;
            break;
          }
        }
      }
    }
    ok_s = ok;
  }
  consumer_sync();
  return ok_s != 0;
}

// The per-CTA trace of a phase (when tracing): [CTA][kTraceSlots] global-timer stamps, plain stores.
__device__ __forceinline__ void mark(const StepPhase& P, int slot) {
  if (P.cta_trace) P.cta_trace[blockIdx.x * kTraceSlots + slot] = globaltimer_ns();
}

// ------------------------------------------------------------------------------------------------ producer
template <int BITS, int HD>
__device__ void produce(const StepParams& sp, uint8_t* smem, const Smem& L, int pos) {
  const int kRing = sp.ring;
  constexpr int TB = BITS == 4 ? 512 : 1024;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
  volatile int* dead = reinterpret_cast<volatile int*>(smem + L.misc + 1000);
  int slot = 0, phase = 0, issued = 0;
  auto acquire = [&]() -> uint8_t* {
    if (issued >= kRing && !*dead) {
      if (!mbar_wait_bounded(&empty[slot], phase ^ 1, sp.err)) {
        *dead = 1;
        atomicOr(sp.err, kErrAbort);
      }
    }
    return *dead ? nullptr : smem + L.ring + slot * kStageBytes;
  };
  auto advance = [&]() {
    ++issued;
    if (++slot == kRing) { slot = 0; phase ^= 1; }
  };
  uint64_t* dfull = empty + kMaxRing;
  uint64_t* dempty = dfull + kDescRing;
  int descs = 0;
  for (int ph = 0; ph < sp.nphases && !*dead; ++ph) {
    const StepPhase& P = sp.phases[ph];
    {  // the phase's descriptor into its ring slot (bulk copy), once the consumers are done with the slot's last
      const int ds = ph % kDescRing;
      if (ph >= kDescRing && !mbar_wait_bounded(&dempty[ds], ((ph / kDescRing) - 1) & 1, sp.err)) {
        *dead = 1;
        atomicOr(sp.err, kErrAbort);
        break;
      }
      mbar_arrive_expect_tx(&dfull[ds], sizeof(StepPhase));  // a multiple of 16 bytes (alignas(16))
      bulk_g2s(smem + L.phase + ds * kPhaseBytes, sp.phases + ph, sizeof(StepPhase), &dfull[ds]);
      ++descs;
    }
    if (P.kind == kPhaseGemv) {
      const QmvParams& q = P.q;
      const size_t G = static_cast<size_t>(q.G);
      for (int u = blockIdx.x; u < P.units && !*dead; u += gridDim.x) {
        for (int c = 0; c < P.nchunks; ++c) {
          uint8_t* dst = acquire();
          if (!dst) break;
          const unsigned wb = P.RW * P.CG * TB;
          mbar_arrive_expect_tx(&full[slot], P.RW * P.CG * (TB + 64));
          for (int rr = 0; rr < P.RW; ++rr) {
            const size_t t = (static_cast<size_t>(u) * P.RW + rr) * G + static_cast<size_t>(c) * P.CG;
            bulk_g2s(dst + rr * P.CG * TB, q.w + t * TB, P.CG * TB, &full[slot]);
            bulk_g2s(dst + wb + rr * P.CG * 64, q.sb + t * 64, P.CG * 64, &full[slot]);
          }
          advance();
        }
      }
    } else {
      const AttnParams& a = P.a;
      if (static_cast<int>(blockIdx.x) < a.KVH * P.S) {
        const int kvh = blockIdx.x / P.S, s = blockIdx.x % P.S;
        const int nk = pos + 1, Lk = (nk + P.S - 1) / P.S;
        const int j0 = s * Lk, j1 = min(nk, j0 + Lk);
        const size_t base = static_cast<size_t>(kvh) * a.cap * HD;
        for (int k0 = j0; k0 < j1 && !*dead; k0 += kAttnKeys) {
          uint8_t* dst = acquire();
          if (!dst) break;
          const int n = max(0, min(min(k0 + kAttnKeys, j1), pos) - k0);  // history rows only (row pos is new)
          mbar_arrive_expect_tx(&full[slot], 2 * n * HD * 2);
          if (n) {
            bulk_g2s(dst, a.kc + base + static_cast<size_t>(k0) * HD, n * HD * 2, &full[slot]);
            bulk_g2s(dst + kAttnKeys * HD * 2, a.vc + base + static_cast<size_t>(k0) * HD, n * HD * 2, &full[slot]);
          }
          advance();
        }
      }
    }
  }
  // no copy of this CTA may land after it leaves: wait (bounded) for the last chunk issued into every stage (already
  // complete unless a wait gave up)
  for (int st = 0; st < kRing && st < issued; ++st) {
    const unsigned parity = static_cast<unsigned>((issued - 1 - st) / kRing) & 1u;
    mbar_wait_bounded(&full[st], parity, nullptr, 100000000ull);
  }
  for (int st = 0; st < kDescRing && st < descs; ++st) {
    const unsigned parity = static_cast<unsigned>((descs - 1 - st) / kDescRing) & 1u;
    mbar_wait_bounded(&dfull[st], parity, nullptr, 100000000ull);
  }
}

// ------------------------------------------------------------------------------------------------ GEMV phase
struct Ring {
  int slot = 0, phase = 0, n = 2;
  __device__ void advance() {
    if (++slot == n) { slot = 0; phase ^= 1; }
  }
};

// The CTA's units (u = blockIdx.x, + gridDim.x, ...) stream through the ring; all 16 warps work on every chunk (RW
// row tiles x 16 / RW K lanes) but never wait for one another inside a unit: each warp parks its partial rows in
// shared memory and moves on. Every kUnitBatch units one barrier, then warp j sums unit j's partials and runs its
// epilogue alone (32 lanes), all warps at once. The argmax keeps one running maximum per warp, combined at the end.
template <int BITS, int RW, int EPI>
__device__ bool gemv_phase(const StepPhase& P, uint8_t* smem, const Smem& L, Ring& ring, unsigned* err) {
  constexpr int TB = BITS == 4 ? 512 : 1024;
  constexpr int KW = kConsumerWarps / RW;
  const QmvParams& p = P.q;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
  __half* xs16 = reinterpret_cast<__half*>(smem + L.xs);
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* pbuf = reinterpret_cast<float*>(smem + L.pbuf);
  float* uvw = reinterpret_cast<float*>(smem + L.uvw) + warp * 32;
  float* misc = reinterpret_cast<float*>(smem + L.misc);
  float* wmisc = EPI == EPI_ARGMAX ? misc + 64 + 2 * warp : misc;  // this warp's running maximum
  volatile int* flag = reinterpret_cast<volatile int*>(misc + 60);

  if (tid == 0) mark(P, 1);
  gemv::stage_row1(p, xs16, xsum, red);
  if (EPI == EPI_ARGMAX && lane == 0) {
    wmisc[0] = -INFINITY;
    wmisc[1] = __int_as_float(0x7fffffff);
  }
  consumer_sync();
  if (tid == 0) mark(P, 3);

  const int CG = P.CG, nchunks = P.nchunks;
  const int rr = warp % RW, kw = warp / RW;
  const int r8 = lane >> 2, c4 = lane & 3;
  const int gpw = kw < CG ? (CG - kw + KW - 1) / KW : 0;
  const uint32_t ax0 = smem_u32(xs16) + c4 * 32;
  const uint32_t axs0 = smem_u32(xsum) + c4 * 8;
  const uint32_t ring0 = smem_u32(smem + L.ring);
  const uint32_t lane_w = static_cast<uint32_t>(rr * CG * TB + lane * 16);
  const uint32_t lane_sb = static_cast<uint32_t>(RW * CG * TB + rr * CG * 64 + r8 * 8);
  const int nu = static_cast<int>(blockIdx.x) < P.units ? (P.units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  bool ok = true;

  for (int k0 = 0; k0 < nu; k0 += kUnitBatch) {
    const int kn = min(kUnitBatch, nu - k0);
    for (int j = 0; j < kn; ++j) {
      float ys[4] = {0.f, 0.f, 0.f, 0.f}, yb[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < nchunks; ++c) {
        if (ok && !mbar_wait_bounded(&full[ring.slot], ring.phase, err)) {
          ok = false;
          atomicOr(err, kErrAbort);
        }
        if (tid == 0 && k0 + j == 0 && c == 0) mark(P, 5);
        const uint32_t st = ring0 + ring.slot * kStageBytes;
        uint32_t aw = st + lane_w + kw * TB;
        uint32_t asb = st + lane_sb + kw * 64;
        uint32_t ax = ax0 + (c * CG + kw) * 128;
        uint32_t axs = axs0 + (c * CG + kw) * 32;
        if (ok) {
#pragma unroll 4
          for (int g = 0; g < gpw; ++g) {
            gemv::group_step<BITS, 1>(aw, asb, ax, axs, p.sdt, ys, yb);
            aw += KW * TB;
            asb += KW * 64;
            ax += KW * 128;
            axs += KW * 32;
          }
        }
        __syncwarp();
        if (lane == 0) gemv::mbar_arrive(&empty[ring.slot]);
        ring.advance();
      }
      if (c4 == 0) {
        float* pw = pbuf + (j * kConsumerWarps + warp) * 16;
        pw[r8] = fmaf(ys[0], gemv::k2p24, yb[0]);
        pw[r8 + 8] = fmaf(ys[2], gemv::k2p24, yb[2]);
      }
    }
    consumer_sync();
    if (warp < kn && ok) {
      const int j = warp;
      const int u = blockIdx.x + (k0 + j) * gridDim.x;
      if (lane < RW * 16) {
        const int rt = lane / 16, rw16 = lane % 16;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < KW; ++q) v += pbuf[(j * kConsumerWarps + rt + q * RW) * 16 + rw16];
        uvw[lane] = v;
      }
      __syncwarp();
      gemv::epilogue<EPI, 1>(p, u * RW * 16, RW * 16, uvw, wmisc, nullptr, lane, 32);
    }
    consumer_sync();  // the partial buffer is reused by the next batch
  }
  ok = !gemv::consumer_sync_or(!ok);  // one verdict for the whole CTA
  if (tid == 0) mark(P, 4);
  if (EPI == EPI_ARGMAX && ok) {
    // the CTA's first maximum over the warps' (ties: the smaller row); the last CTA to finish takes the grid's and
    // runs the generation step
    if (tid == 0) {
      float bv = misc[64];
      int bi = __float_as_int(misc[65]);
      for (int w = 1; w < kConsumerWarps; ++w) {
        const float ov = misc[64 + 2 * w];
        const int oi = __float_as_int(misc[65 + 2 * w]);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      p.pairs[static_cast<size_t>(blockIdx.x) * 16] = bv;
      p.pairs[static_cast<size_t>(blockIdx.x) * 16 + 1] = __int_as_float(bi);
      __threadfence();
      const unsigned prev = atomicAdd(&p.counters[0], 1u);
      *flag = prev == gridDim.x - 1;
      if (*flag) atomicExch(&p.counters[0], 0u);
    }
    consumer_sync();
    if (*flag) {
      __threadfence();
      gemv::argmax_finish(p, misc);
    }
  }
  if (tid == 0) mark(P, 2);
  return ok;
}

// ------------------------------------------------------------------------------------------------ attention phase
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
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

// Keys as the MMA's M, the GQA group's query heads (<= 8) as N: S^T = K Q^T, O^T += V^T P^T (fp16 in, fp32 out).
template <int HD>
__device__ bool attn_phase(const StepPhase& P, uint8_t* smem, const Smem& L, Ring& ring, unsigned* err, int pos) {
  constexpr int KS = HD / 16;
  constexpr int RB = HD * 2;  // shared row bytes (unpadded: the bulk copy lands rows back to back)
  const AttnParams& a = P.a;
  const int S = P.S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int G = a.H / a.KVH;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
  float* scr = reinterpret_cast<float*>(smem + L.xs);
  float (*sm_o)[8][HD] = reinterpret_cast<float (*)[8][HD]>(scr);           // [warp][head][dim]
  float* sm_m = scr + kAttnWarps * 8 * HD;                                   // [warp][head]
  float* sm_l = sm_m + kAttnWarps * 8;
  volatile int* flag = reinterpret_cast<volatile int*>(smem + L.misc + 240);
  bool ok = true;
  if (tid == 0) mark(P, 1);
  if (static_cast<int>(blockIdx.x) >= a.KVH * S) return true;  // no chunk for this CTA
  const int kvh = blockIdx.x / S, s = blockIdx.x % S;
  const int nk = pos + 1, Lk = (nk + S - 1) / S;
  const int j0 = s * Lk, j1 = min(nk, j0 + Lk);
  const size_t base = static_cast<size_t>(kvh) * a.cap * HD;

  uint32_t qb[KS][2];
  {
    const bool live = g8 < G;
    const unsigned* qrow = reinterpret_cast<const unsigned*>(a.q16 + static_cast<size_t>(kvh * G + (live ? g8 : 0)) * HD);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qb[ks][0] = live ? __ldcg(qrow + ks * 8 + t4) : 0u;
      qb[ks][1] = live ? __ldcg(qrow + ks * 8 + 4 + t4) : 0u;
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float oacc[KS][4];
#pragma unroll
  for (int dt = 0; dt < KS; ++dt) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.f;
  const int kt = warp * 16;
  if (tid == 0) mark(P, 3);
  for (int k0 = j0; k0 < j1; k0 += kAttnKeys) {
    const int n = min(kAttnKeys, j1 - k0);
    uint8_t* Ks = smem + L.ring + ring.slot * kStageBytes;
    uint8_t* Vs = Ks + kAttnKeys * RB;
    if (ok && !mbar_wait_bounded(&full[ring.slot], ring.phase, err)) {
      ok = false;
      atomicOr(err, kErrAbort);
    }
    // the new row (appended by this step's qkv phase) and zero V rows up to the next 16-key tile
    const int n16 = (n + 15) & ~15;
    if (pos >= k0 && pos < k0 + n && tid < 2 * HD / 8) {
      const int kv = tid / (HD / 8), c = tid % (HD / 8);
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>((kv ? a.vc : a.kc) + base + static_cast<size_t>(pos) * HD) + c);
      *reinterpret_cast<uint4*>((kv ? Vs : Ks) + (pos - k0) * RB + c * 16) = v;
    }
    for (int t = tid; t < (n16 - n) * (HD / 8); t += kConsumers)
      *reinterpret_cast<uint4*>(Vs + (n + t / (HD / 8)) * RB + (t % (HD / 8)) * 16) = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
    consumer_sync();
    if (ok && warp < kAttnWarps && kt < n) {
      float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
      const uint32_t ka = smem_u32(Ks + (kt + (lane & 7) + ((lane >> 3) & 1) * 8) * RB + (lane >> 4) * 16);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(ka + ks * 32, a0, a1, a2, a3);
        mma_16816(c0, c1, c2, c3, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
      }
      const bool va = kt + g8 < n, vb = kt + g8 + 8 < n;
      const float s0 = va ? c0 : -INFINITY, s1 = va ? c1 : -INFINITY;
      const float s2 = vb ? c2 : -INFINITY, s3 = vb ? c3 : -INFINITY;
      float x0 = fmaxf(s0, s2), x1 = fmaxf(s1, s3);
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
        x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
      }
      const float mn0 = fmaxf(m0, x0), mn1 = fmaxf(m1, x1);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      const float p0 = exp2f(s0 - mn0), p1 = exp2f(s1 - mn1), p2 = exp2f(s2 - mn0), p3 = exp2f(s3 - mn1);
      l0 = fmaf(l0, al0, p0 + p2);
      l1 = fmaf(l1, al1, p1 + p3);
      m0 = mn0;
      m1 = mn1;
      const uint32_t pb0 = movm_t(pack_h2(p0, p1)), pb1 = movm_t(pack_h2(p2, p3));
      const uint32_t va_addr = smem_u32(Vs + (kt + (lane & 7) + (lane >> 4) * 8) * RB + ((lane >> 3) & 1) * 16);
#pragma unroll
      for (int dt = 0; dt < KS; ++dt) {
        oacc[dt][0] *= al0;
        oacc[dt][1] *= al1;
        oacc[dt][2] *= al0;
        oacc[dt][3] *= al1;
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(va_addr + dt * 32, a0, a1, a2, a3);
        mma_16816(oacc[dt][0], oacc[dt][1], oacc[dt][2], oacc[dt][3], a0, a1, a2, a3, pb0, pb1);
      }
    }
    consumer_sync();
    if (lane == 0) gemv::mbar_arrive(&empty[ring.slot]);
    ring.advance();
  }
  ok = !gemv::consumer_sync_or(!ok);  // one verdict for the whole CTA
  if (tid == 0) mark(P, 5);
  if (!ok) return false;
  // the tile warps' partials -> this chunk's partial (m, l, o) -> global; the head's last chunk merges them
  if (warp < kAttnWarps) {
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g8 == 0) {
      sm_m[warp * 8 + 2 * t4] = m0;
      sm_m[warp * 8 + 2 * t4 + 1] = m1;
      sm_l[warp * 8 + 2 * t4] = l0;
      sm_l[warp * 8 + 2 * t4 + 1] = l1;
    }
#pragma unroll
    for (int dt = 0; dt < KS; ++dt) {
      sm_o[warp][2 * t4][16 * dt + g8] = oacc[dt][0];
      sm_o[warp][2 * t4 + 1][16 * dt + g8] = oacc[dt][1];
      sm_o[warp][2 * t4][16 * dt + g8 + 8] = oacc[dt][2];
      sm_o[warp][2 * t4 + 1][16 * dt + g8 + 8] = oacc[dt][3];
    }
  }
  consumer_sync();
  float* part = a.part + static_cast<size_t>(kvh * S + s) * G * (HD + 2);
  for (int t = tid; t < G * HD; t += kConsumers) {
    const int g = t / HD, d = t % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w * 8 + g]);
    float Ls = 0.f, Os = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = sm_m[w * 8 + g] == -INFINITY ? 0.f : exp2f(sm_m[w * 8 + g] - M);
      Ls = fmaf(sm_l[w * 8 + g], f, Ls);
      Os = fmaf(sm_o[w][g][d], f, Os);
    }
    part[g * (HD + 2) + d] = Os;
    if (d == 0) {
      part[g * (HD + 2) + HD] = M;
      part[g * (HD + 2) + HD + 1] = Ls;
    }
  }
  consumer_sync();
  if (tid == 0) {
    __threadfence();  // after the named barrier: orders every consumer's partial before the count
    const unsigned prev = atomicAdd(&a.counters[kvh], 1u);
    *flag = prev == static_cast<unsigned>(S) - 1;
    if (*flag) atomicExch(&a.counters[kvh], 0u);
  }
  consumer_sync();
  if (tid == 0) mark(P, 4);
  if (*flag) {
    __threadfence();
    const float* hp = a.part + static_cast<size_t>(kvh) * S * G * (HD + 2);
    // every chunk's (m, l, o[d]) loaded independently (an empty chunk holds m = -inf, l = 0, o = 0)
    for (int t = tid; t < G * HD; t += kConsumers) {
      const int g = t / HD, d = t % HD;
      float M = -INFINITY;
#pragma unroll 8
      for (int q = 0; q < S; ++q) M = fmaxf(M, __ldcg(hp + (static_cast<size_t>(q) * G + g) * (HD + 2) + HD));
      float Ls = 0.f, Os = 0.f;
#pragma unroll 8
      for (int q = 0; q < S; ++q) {
        const float* pq = hp + (static_cast<size_t>(q) * G + g) * (HD + 2);
        const float mq = __ldcg(pq + HD), lq = __ldcg(pq + HD + 1), oq = __ldcg(pq + d);
        const float w = mq == -INFINITY ? 0.f : exp2f(mq - M);
        Ls = fmaf(lq, w, Ls);
        Os = fmaf(oq, w, Os);
      }
      a.out[static_cast<size_t>(kvh * G + g) * HD + d] = __float2half_rn(Os / Ls);
    }
  }
  if (tid == 0) mark(P, 2);
  return ok;
}

// ------------------------------------------------------------------------------------------------ the kernel
template <int BITS>
__device__ bool run_gemv(const StepPhase& P, uint8_t* smem, const Smem& L, Ring& ring, unsigned* err) {
  const int e = P.q_epi;
  if (P.RW == 2) {
    switch (e) {
      case EPI_QKV: return gemv_phase<BITS, 2, EPI_QKV>(P, smem, L, ring, err);
      case EPI_RES1: return gemv_phase<BITS, 2, EPI_RES1>(P, smem, L, ring, err);
      case EPI_SWIGLU: return gemv_phase<BITS, 2, EPI_SWIGLU>(P, smem, L, ring, err);
      case EPI_RES2: return gemv_phase<BITS, 2, EPI_RES2>(P, smem, L, ring, err);
      default: return gemv_phase<BITS, 2, EPI_ARGMAX>(P, smem, L, ring, err);
    }
  }
  switch (e) {
    case EPI_QKV: return gemv_phase<BITS, 1, EPI_QKV>(P, smem, L, ring, err);
    case EPI_RES1: return gemv_phase<BITS, 1, EPI_RES1>(P, smem, L, ring, err);
    case EPI_RES2: return gemv_phase<BITS, 1, EPI_RES2>(P, smem, L, ring, err);
    default: return gemv_phase<BITS, 1, EPI_ARGMAX>(P, smem, L, ring, err);
  }
}

template <int BITS, int HD>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepParams sp) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const Smem L = smem_layout(sp.kmax, sp.ring);
  const int tid = threadIdx.x, warp = tid >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
  int pos = static_cast<int>(sp.q0[0]);
  if (pos > sp.cap - 1) pos = sp.cap - 1;
  if (tid == 0) {
    for (int s = 0; s < sp.ring; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < kDescRing; ++s) {
      mbar_init(&empty[kMaxRing + s], 1);              // descriptor full: the producer's copy
      mbar_init(&empty[kMaxRing + kDescRing + s], 1);  // descriptor empty: the consumers' release
    }
    *reinterpret_cast<volatile int*>(smem + L.misc + 1000) = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kConsumerWarps) {
    if ((tid & 31) == 0) produce<BITS, HD>(sp, smem, L, pos);
    return;
  }
  Ring ring;
  ring.n = sp.ring;
  bool ok = true;
  // the phase descriptors live in shared memory, brought in by the producer (its fields are read all over a phase;
  // from global memory each first touch would cost a round trip)
  uint64_t* dfull = empty + kMaxRing;
  uint64_t* dempty = dfull + kDescRing;
  for (int ph = 0; ph < sp.nphases; ++ph) {
    const int ds = ph % kDescRing;
    if (!mbar_wait_bounded(&dfull[ds], (ph / kDescRing) & 1, sp.err)) atomicOr(sp.err, kErrAbort);
    const StepPhase& P = *reinterpret_cast<const StepPhase*>(smem + L.phase + ds * kPhaseBytes);
    if (tid == 0) mark(P, 0);  // arrival at the phase's barrier
    if (ph > 0 && !grid_barrier(sp.bar, static_cast<unsigned>(ph) * gridDim.x, sp.err)) {
      ok = false;
      break;
    }
    const bool r = P.kind == kPhaseGemv ? run_gemv<BITS>(P, smem, L, ring, sp.err)
                                        : attn_phase<HD>(P, smem, L, ring, sp.err, pos);
    consumer_sync();  // every consumer is done with the descriptor
    if (tid == 0) gemv::mbar_arrive(&dempty[ds]);
    if (!r) {
      ok = false;
      break;
    }
  }
  // the last CTA out resets the barrier for the next launch (every CTA has passed its last barrier by then)
  consumer_sync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(sp.bar + 1, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(sp.bar, 0u);
      atomicExch(sp.bar + 1, 0u);
    }
  }
  if (!ok && tid == 0) {
    // leave only when this CTA's copies are no longer in flight: the producer stopped at the abort bit
    volatile int* dead = reinterpret_cast<volatile int*>(smem + L.misc + 1000);
    *dead = 1;
  }
}

template <int BITS, int HD>
int launch_t(const StepParams& sp, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_layout(sp.kmax, sp.ring).total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, step_kernel<BITS, HD>, sp));
  return 0;
}

template <int BITS, int HD>
int configure_t(const agxc_ctx* ctx, int kmax, int* ok, int* stages) {
  cudaFuncAttributes fa;
  AGXC_CUDA(cudaFuncGetAttributes(&fa, step_kernel<BITS, HD>));
  const int st = ring_stages(kmax, ctx->max_smem_optin, static_cast<int>(fa.sharedSizeBytes));
  const int smem = smem_layout(kmax, st).total;
  *ok = 0;
  *stages = st;
  if (smem + static_cast<int>(fa.sharedSizeBytes) > ctx->max_smem_optin) return 0;
  AGXC_CUDA(cudaFuncSetAttribute(step_kernel<BITS, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int blocks = 0;
  AGXC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, step_kernel<BITS, HD>, kThreads, smem));
  *ok = blocks >= 1;
  return 0;
}

}  // namespace step

// The launch plan of a GEMV phase: RW row tiles per unit (2 when the row tiles pair up and every CTA still gets a
// unit, always for SwiGLU), the largest chunk of groups dividing K that fits a stage.
int step_plan_gemv(StepPhase* P, int N, int K, int bits, int epi, int grid) {
  const int TB = tile_bytes(bits);
  const int G = K / 64, RT = N / 16;
  int RW = (RT % 2 == 0 && (epi == EPI_SWIGLU || RT / 2 >= grid)) ? 2 : 1;
  if (epi == EPI_SWIGLU && RW != 2) return fail(AGXC_EINVAL, "step: SwiGLU needs paired row tiles");
  int CG = 0;
  for (int c = 1; c <= G; ++c)
    if (G % c == 0 && RW * c * (TB + 64) <= step::kStageBytes) CG = c;
  if (!CG) return fail(AGXC_EINVAL, "step: no chunk fits a stage");
  P->kind = kPhaseGemv;
  P->q_epi = epi;
  P->RW = RW;
  P->CG = CG;
  P->nchunks = G / CG;
  P->units = RT / RW;
  P->q.G = G;
  P->q.GC = G;
  P->q.CG = CG;
  P->q.SC = 1;
  return 0;
}

int step_configure(const agxc_ctx* ctx, int bits, int hd, int kmax, int* ok, int* stages) {
  *ok = 0;
  *stages = 0;
  if (bits == 4 && hd == 128) return step::configure_t<4, 128>(ctx, kmax, ok, stages);
  if (bits == 4 && hd == 64) return step::configure_t<4, 64>(ctx, kmax, ok, stages);
  if (bits == 8 && hd == 128) return step::configure_t<8, 128>(ctx, kmax, ok, stages);
  if (bits == 8 && hd == 64) return step::configure_t<8, 64>(ctx, kmax, ok, stages);
  return 0;
}

int step_launch(const StepParams& sp, int bits, int hd, int grid, cudaStream_t s) {
  if (bits == 4 && hd == 128) return step::launch_t<4, 128>(sp, grid, s);
  if (bits == 4 && hd == 64) return step::launch_t<4, 64>(sp, grid, s);
  if (bits == 8 && hd == 128) return step::launch_t<8, 128>(sp, grid, s);
  if (bits == 8 && hd == 64) return step::launch_t<8, 64>(sp, grid, s);
  return fail(AGXC_EINVAL, "step: 4 or 8 bits, head_dim 64 or 128");
}

size_t step_smem(int kmax, int stages) { return step::smem_layout(kmax, stages).total; }

}  // namespace agxc
