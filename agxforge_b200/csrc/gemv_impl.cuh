// gemv_impl.cuh — the quantized GEMV family of the decode step (the reference's build_qmv2 and its fused epilogues,
// agxforge/kernels/qmv.py:341-881), written for sm_100a.
//
// y[b][n] = sum_g ( s[n,g] * sum_{k in g} q[n,k] x[b][k]  +  b[n,g] * sum_{k in g} x[b][k] )
//
// The reference factorises each trip the same way (qmv.py:1577-1649: t = sum q x, acc += s t + b sx). Here:
//   * WORK: a unit is RW (1, 2 or 4) row tiles of 16 rows over the CTA's K range (all of K unless split, SC > 1). A
//     CTA runs its units in order; a unit streams through shared memory in chunks of CG groups: one 3-D TMA box
//     (RW row tiles x CG tiles x tile bytes) of the tile array [row tile][group][tile], and one of its scale/bias.
//   * PRODUCER: one warp issues the TMA copies (cp.async.bulk.tensor.3d, completing on a "full" mbarrier) of the
//     chunks into a ring of stages, as far ahead as free stages allow — across unit boundaries, and (with
//     programmatic dependent launch) before the upstream kernel has finished, since weights do not depend on it. A
//     stage is refilled when all consumer warps have released it ("empty" mbarrier).
//   * CONSUMERS: 16 warps, RW row tiles x (16 / RW) K lanes. Each dequantises its lane's fields with one AND (4-bit; one PRMT for 8-bit) per two weights
//     into fp16 SUBNORMALS q * 2^-24 (exact), and forms sum q x on the tensor cores with mma.sync m16n8k16 (weight
//     rows = M, activation rows = N <= 8, fp32 accumulate); scale and bias are applied per group on the CUDA cores
//     and the 2^24 once per row at the end. Warps accumulate over their groups across
//     all chunks of a unit and meet once per unit in shared memory.
//   * the activation rows of the CTA's K range are staged once in shared memory as fp16 (every GEMV input of the
//     decode graph holds fp16 values), with their per-group sums; the RMSNorm of the input is fused in front
//     (with_norm, qmv.py:176-183), recomputed per CTA from the row.
//   * EPILOGUES on the unit's rows: fp32 out; + fp16 residual -> fp32 (add16); + fp32 residual -> fp16 (add32_to16);
//     SiLU(gate) * up -> fp16 (gate and up row tiles interleaved, RW = 2); bias + RoPE + q scale + KV append (the qkv
//     pack's rows are placed so tile rows r and r + 8 are a RoPE pair i, i + hd/2); per-CTA first maximum + the
//     generation step (head). When K is split (SC > 1) partial rows meet through scratch and a last-arriver counter.
//   Every wait is bounded; no thread spins on another CTA.
#pragma once

#include <cuda.h>

#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace agxc {
namespace gemv {

constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kMaxStages = 8;
constexpr float k2p24 = 16777216.0f;

struct Smem {
  int full, empty, dead, ring, stage_bytes, wbytes, xs, xstride, xsum, red, uv, ev, resv, misc, total;
};

__host__ __device__ inline Smem smem_layout(int bits, int nbt, int RW, int CG, int GC, int stages) {
  Smem L;
  const int TB = bits == 4 ? 512 : 1024;
  L.full = 0;
  L.empty = 8 * kMaxStages;
  L.dead = 16 * kMaxStages;
  L.ring = 256;
  L.wbytes = RW * CG * TB;
  L.stage_bytes = (L.wbytes + RW * CG * 64 + 127) / 128 * 128;
  L.xs = L.ring + stages * L.stage_bytes;
  L.xstride = GC * 64 + 8;  // halves; the 16-byte pad keeps 8 rows' fragment loads bank-conflict free
  L.xsum = L.xs + ((nbt * L.xstride * 2 + 127) / 128) * 128;
  L.red = L.xsum + GC * 8 * 4;
  L.uv = L.red + kConsumerWarps * 16 * nbt * 4;
  L.ev = L.uv + RW * 16 * nbt * 4;
  L.resv = L.ev + RW * 16 * nbt * 4;  // the first unit's residual rows, prefetched before the dependency wait
  L.misc = L.resv + RW * 16 * nbt * 4;
  L.total = L.misc + 1024;
  return L;
}

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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds32f(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// One group (16 rows x 64 k, one tile) of one warp: dequant + 4 MMAs, from 32-bit shared addresses already offset
// for this lane (w: 16 B per lane; sb: the lane's row entry; x: the lane's 16 activations; xs: the lane's column
// sums). Accumulates per C element  ys += s * T  (T = the group's sum q x scaled by 2^-24)  and  yb += b * sum x,
// so the row's value is ys * 2^24 + yb (applied once, after the last group).
template <int BITS, int NBT>
__device__ __forceinline__ void group_step(uint32_t aw, uint32_t asb, uint32_t ax, uint32_t axs, int sdt, float* ys,
                                          float* yb) {
  const uint2 sv = lds64(asb);
  const uint4 xa = lds128(ax);
  const uint4 xb = lds128(ax + 16);
  float2 xsv;
  if (NBT > 1) xsv = lds64f(axs);
  else xsv.x = xsv.y = lds32f(axs);
  float2 s2, b2;  // (row r8, row r8 + 8)
  if (sdt) {
    s2 = make_float2(__uint_as_float(sv.x << 16), __uint_as_float(sv.x & 0xffff0000u));
    b2 = make_float2(__uint_as_float(sv.y << 16), __uint_as_float(sv.y & 0xffff0000u));
  } else {
    __half2 hs, hb;
    memcpy(&hs, &sv.x, 4);
    memcpy(&hb, &sv.y, 4);
    s2 = __half22float2(hs);
    b2 = __half22float2(hb);
  }
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, b0 = 0.f, b1 = 0.f, b2c = 0.f, b3 = 0.f;
  float T0, T1, T2, T3;
  if (BITS == 4) {
    const uint4 wv = lds128(aw);
    constexpr uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u;
    mma_16816(a0, a1, a2, a3, wv.x & M0, wv.y & M0, wv.z & M0, wv.w & M0, xa.x, xa.y);
    mma_16816(b0, b1, b2c, b3, wv.x & M1, wv.y & M1, wv.z & M1, wv.w & M1, xa.z, xa.w);
    const uint32_t sx = wv.x >> 8, sy = wv.y >> 8, sz = wv.z >> 8, sw = wv.w >> 8;
    mma_16816(a0, a1, a2, a3, sx & M0, sy & M0, sz & M0, sw & M0, xb.x, xb.y);
    mma_16816(b0, b1, b2c, b3, sx & M1, sy & M1, sz & M1, sw & M1, xb.z, xb.w);
    // the upper nibble of each byte carried 2^4: its chain is 16x the lower one's scale
    T0 = fmaf(b0, 0.0625f, a0); T2 = fmaf(b2c, 0.0625f, a2);
    T1 = fmaf(b1, 0.0625f, a1); T3 = fmaf(b3, 0.0625f, a3);
  } else {
    const uint4 w0 = lds128(aw);
    const uint4 w1 = lds128(aw + 512);
    constexpr uint32_t PL = 0x4140u, PH = 0x4342u;
    mma_16816(a0, a1, a2, a3, prmt(w0.x, 0, PL), prmt(w0.x, 0, PH), prmt(w0.y, 0, PL), prmt(w0.y, 0, PH), xa.x, xa.y);
    mma_16816(b0, b1, b2c, b3, prmt(w0.z, 0, PL), prmt(w0.z, 0, PH), prmt(w0.w, 0, PL), prmt(w0.w, 0, PH), xa.z, xa.w);
    mma_16816(a0, a1, a2, a3, prmt(w1.x, 0, PL), prmt(w1.x, 0, PH), prmt(w1.y, 0, PL), prmt(w1.y, 0, PH), xb.x, xb.y);
    mma_16816(b0, b1, b2c, b3, prmt(w1.z, 0, PL), prmt(w1.z, 0, PH), prmt(w1.w, 0, PL), prmt(w1.w, 0, PH), xb.z, xb.w);
    T0 = a0 + b0; T2 = a2 + b2c; T1 = a1 + b1; T3 = a3 + b3;
  }
  ys[0] = fmaf(s2.x, T0, ys[0]);
  ys[2] = fmaf(s2.y, T2, ys[2]);
  yb[0] = fmaf(b2.x, xsv.x, yb[0]);
  yb[2] = fmaf(b2.y, xsv.x, yb[2]);
  if (NBT > 1) {
    ys[1] = fmaf(s2.x, T1, ys[1]);
    ys[3] = fmaf(s2.y, T3, ys[3]);
    yb[1] = fmaf(b2.x, xsv.y, yb[1]);
    yb[3] = fmaf(b2.y, xsv.y, yb[3]);
  }
}

// ------------------------------------------------------------------------------------------------ epilogues
// vals(i): the value of element i = r NBT + b of the block ([rows][NBT] fp32, column = activation row b) of `rows`
// physical rows starting at `row0`: an array read, or the warps' partial sums added on demand.
template <int EPI, int NBT, typename Vals>
// resv: prefetched operands of these rows, or NULL to read them here: the residual ([rows][NBT] fp32) of RES1/RES2,
// the RoPE (cos, sin) per pair ([rows/2][NBT][2]) of QKV
// t0 / tstride: the calling threads' index and count (default: all consumer threads); the argmax keeps its running
// maximum in misc[0], misc[1] of the calling group (one warp, t0 = lane, when a warp finalises a unit alone).
__device__ void epilogue(const QmvParams& p, int row0, int rows, Vals vals, float* misc,
                         const float* resv = nullptr, int t0 = -1, int tstride = kConsumers) {
  const int tid = t0 >= 0 ? t0 : static_cast<int>(threadIdx.x);
  const int nb = p.nb;
  if (EPI == EPI_F32) {
    for (int t = tid; t < rows * NBT; t += tstride) {
      const int r = t / NBT, b = t % NBT;
      if (b >= nb) continue;
      p.out_f32[static_cast<size_t>(b) * p.out_ld + row0 + r] = vals(r * NBT + b);
    }
  } else if (EPI == EPI_RES1) {
    for (int t = tid; t < rows * NBT; t += tstride) {
      const int r = t / NBT, b = t % NBT;
      if (b >= nb) continue;
      const float x = resv ? resv[r * NBT + b]
                           : __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(p.res16) +
                                                                  static_cast<size_t>(b) * p.res_ld + row0 + r)));
      p.out_f32[static_cast<size_t>(b) * p.out_ld + row0 + r] = vals(r * NBT + b) + x;
    }
  } else if (EPI == EPI_RES2) {
    for (int t = tid; t < rows * NBT; t += tstride) {
      const int r = t / NBT, b = t % NBT;
      if (b >= nb) continue;
      const float h = resv ? resv[r * NBT + b] : __ldcg(p.res32 + static_cast<size_t>(b) * p.res_ld + row0 + r);
      p.out_f16[static_cast<size_t>(b) * p.out_ld + row0 + r] = __float2half_rn(vals(r * NBT + b) + h);
    }
  } else if (EPI == EPI_SWIGLU) {
    // pairs of row tiles: a gate tile (rows 0..15 of the pair) and its up tile (rows 16..31); output (row0/32)*16 + r
    for (int t = tid; t < rows / 2 * NBT; t += tstride) {
      const int r = t / NBT, b = t % NBT;
      if (b >= nb) continue;
      const int pr = r / 16, rr = r % 16;
      const float g = vals((pr * 32 + rr) * NBT + b), u = vals((pr * 32 + 16 + rr) * NBT + b);
      p.out_f16[static_cast<size_t>(b) * p.out_ld + (row0 / 32 + pr) * 16 + rr] = __float2half_rn(silu_f(g) * u);
    }
  } else if (EPI == EPI_QKV) {
    // each 16-row tile of a head holds logical rows (8t + r, hd/2 + 8t + r) at tile rows (r, r + 8): a RoPE pair.
    // bias, rotate-half RoPE at the sequence's position (q and k heads), q scaled for the base-2 softmax and stored
    // fp16; k and v stored fp16 into the cache row at the position.
    const int hd = p.hd, half = hd / 2;
    for (int t = tid; t < rows / 2 * NBT; t += tstride) {
      const int pr = t / NBT, b = t % NBT;
      if (b >= nb) continue;
      const int tile = pr / 8, r = pr % 8;
      const int prow0 = row0 + tile * 16;          // physical row of the tile's first row
      const int head = prow0 / hd;
      const int tt = (prow0 % hd) / 16;            // tile index within the head
      const int i1 = 8 * tt + r, i2 = half + 8 * tt + r;
      float y1 = vals((tile * 16 + r) * NBT + b), y2 = vals((tile * 16 + r + 8) * NBT + b);
      if (p.bias) {
        y1 += __half2float(p.bias[head * hd + i1]);
        y2 += __half2float(p.bias[head * hd + i2]);
      }
      int pos = static_cast<int>(p.q0[b]);
      if (pos > p.cap - 1) pos = p.cap - 1;
      if (head < p.H + p.KVH) {
        const float c = resv ? resv[2 * t] : p.cos_t[static_cast<size_t>(pos) * half + i1];
        const float s = resv ? resv[2 * t + 1] : p.sin_t[static_cast<size_t>(pos) * half + i1];
        const float o1 = y1 * c - y2 * s, o2 = y2 * c + y1 * s;
        if (head < p.H) {
          __half* q = p.q16 + (static_cast<size_t>(b) * p.H + head) * hd;
          q[i1] = __float2half_rn(o1 * p.qscale);
          q[i2] = __float2half_rn(o2 * p.qscale);
        } else {
          __half* k = p.kcache + ((static_cast<size_t>(b) * p.KVH + (head - p.H)) * p.cap + pos) * hd;
          k[i1] = __float2half_rn(o1);
          k[i2] = __float2half_rn(o2);
        }
      } else {
        __half* v = p.vcache + ((static_cast<size_t>(b) * p.KVH + (head - p.H - p.KVH)) * p.cap + pos) * hd;
        v[i1] = __float2half_rn(y1);
        v[i2] = __float2half_rn(y2);
      }
    }
  } else if (EPI == EPI_ARGMAX) {
    if (p.out_f32) {
      for (int t = tid; t < rows * NBT; t += tstride) {
        const int r = t / NBT, b = t % NBT;
        if (b >= nb) continue;
        p.out_f32[static_cast<size_t>(b) * p.V + row0 + r] = vals(r * NBT + b);
      }
    }
    // warp b keeps the running first-maximum of column b: misc[2b] value, misc[2b+1] index (int bits)
    const int w = tid >> 5, lane = tid & 31;
    if (w < nb) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int r = lane; r < rows; r += 32) {
        const float v = vals(r * NBT + w);
        if (v > bv) { bv = v; bi = row0 + r; }  // rows ascend per lane: the first of equal values stays
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        const float cv = misc[2 * w];
        const int ci = __float_as_int(misc[2 * w + 1]);
        if (bv > cv || (bv == cv && bi < ci)) { misc[2 * w] = bv; misc[2 * w + 1] = __int_as_float(bi); }
      }
    }
  }
}

// The argmax's cross-CTA step and the generation step, run by the last CTA to finish (argmax.py:141-215,
// assemble.py:918-930): token = the forced token if one is pending, else the logged prompt token, else the first
// maximum; log it, write its embedding row as the next x, advance q0 (clamped to cap - 1).
static __device__ void argmax_finish(const QmvParams& p, float* misc) {
  const int tid = threadIdx.x;
  const int nb = p.nb;
  int* s_tok = reinterpret_cast<int*>(misc + 48);
  for (int b = 0; b < nb; ++b) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = tid; c < static_cast<int>(gridDim.x); c += kConsumers) {
      const float v = ld_cg(p.pairs + (static_cast<size_t>(c) * 8 + b) * 2);
      const int i = __float_as_int(ld_cg(p.pairs + (static_cast<size_t>(c) * 8 + b) * 2 + 1));
      if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((tid & 31) == 0) { misc[16 + 2 * (tid >> 5)] = bv; misc[17 + 2 * (tid >> 5)] = __int_as_float(bi); }
    consumer_sync();
    if (tid == 0) {
      for (int w = 1; w < kConsumerWarps; ++w) {
        const float ov = misc[16 + 2 * w];
        const int oi = __float_as_int(misc[17 + 2 * w]);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      const uint32_t pos = p.q0_rw[b];
      const uint32_t p1 = pos + 1;
      uint32_t f = p.force_next ? p.force_next[b] : kTokenUnset;
      if (p.force_next) p.force_next[b] = kTokenUnset;
      if (f == kTokenUnset && p1 < static_cast<uint32_t>(p.cap)) f = p.log[static_cast<size_t>(b) * p.cap + p1];
      uint32_t tok = f != kTokenUnset ? f : static_cast<uint32_t>(bi);
      if (tok >= static_cast<uint32_t>(p.V)) {
        atomicOr(p.err, kErrBadToken);
        tok = 0;
      }
      if (p1 < static_cast<uint32_t>(p.cap)) p.log[static_cast<size_t>(b) * p.cap + p1] = tok;
      p.q0_rw[b] = p1 < static_cast<uint32_t>(p.cap) ? p1 : static_cast<uint32_t>(p.cap - 1);
      if (p.tok_out) p.tok_out[b] = static_cast<int32_t>(tok);
      s_tok[b] = static_cast<int>(tok);
    }
    consumer_sync();
  }
  // the chosen tokens' embedding rows become the next step's x
  const int dv = p.d / 8;
  for (int t = tid; t < nb * dv; t += kConsumers) {
    const int b = t / dv, i = t % dv;
    const uint4* src = reinterpret_cast<const uint4*>(p.embed + static_cast<size_t>(s_tok[b]) * p.d);
    reinterpret_cast<uint4*>(p.x_next + static_cast<size_t>(b) * p.d)[i] = src[i];
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 8 consecutive elements of activation row b from column `col` (fp16 or fp32 rows of p.x), as fp32. Activations are
// written by other CTAs (or kernels) of the step, so they are read from L2, never from a possibly stale L1 line.
__device__ __forceinline__ void load8(const QmvParams& p, int b, int col, float* v) {
  if (p.x_f32) {
    const float4* src =
        reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + static_cast<size_t>(b) * p.x_ld + col);
    const float4 a = __ldcg(src), c = __ldcg(src + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  } else {
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x) + static_cast<size_t>(b) * p.x_ld + col));
    __half2 h[4];
    memcpy(h, &u, 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// Stage ONE activation row of the whole K range (fp16, RMSNorm fused when a gain is given) and its per-group sums
// (xsum[g * 8]). A thread's vectors (k = tid, tid + 512) and their gains are loaded together and stay in registers
// across the norm's reduction: one L2 round trip and one barrier (rows up to 8,192; wider rows reload the rest).
__device__ __forceinline__ void stage_row1(const QmvParams& p, __half* xs16, float* xsum, float* red) {
  constexpr int kCache = 2;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n8 = p.K / 8;
  const int steps = (n8 + kConsumers - 1) / kConsumers;
  float v[kCache][8];
  uint4 gv[kCache];
#pragma unroll
  for (int st = 0; st < kCache; ++st) {
    const int k = tid + st * kConsumers;
    gv[st] = make_uint4(0u, 0u, 0u, 0u);
    if (st < steps && k < n8) {
      load8(p, 0, k * 8, v[st]);
      if (p.norm_gain) gv[st] = reinterpret_cast<const uint4*>(p.norm_gain)[k];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[st][j] = 0.f;
    }
  }
  float r = 1.0f;
  if (p.norm_gain) {
    float ss = 0.f;
#pragma unroll
    for (int st = 0; st < kCache; ++st)
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[st][j], v[st][j], ss);
    for (int k = tid + kCache * kConsumers; k < n8; k += kConsumers) {  // rows wider than the cache
      float w[8];
      load8(p, 0, k * 8, w);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(w[j], w[j], ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    consumer_sync();
    float tot = 0.f;
    for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
    r = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
  }
  for (int st = 0; st < steps; ++st) {
    const int k = tid + st * kConsumers;
    const bool live = k < n8;
    float x[8];
    uint4 gu = make_uint4(0u, 0u, 0u, 0u);
    if (st < kCache) {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = st == 0 ? v[0][j] : v[1][j];
      gu = st == 0 ? gv[0] : gv[1];
    } else if (live) {
      load8(p, 0, k * 8, x);
      if (p.norm_gain) gu = reinterpret_cast<const uint4*>(p.norm_gain)[k];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = 0.f;
    }
    if (p.norm_gain && live) {
      __half2 gh[4];
      memcpy(gh, &gu, 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 g = __half22float2(gh[j]);
        x[2 * j] = (x[2 * j] * r) * g.x;
        x[2 * j + 1] = (x[2 * j + 1] * r) * g.y;
      }
    }
    __half2 oh[4];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      oh[j] = __floats2half2_rn(x[2 * j], x[2 * j + 1]);
      const float2 f = __half22float2(oh[j]);
      sum += f.x + f.y;
    }
    if (live) {
      uint4 o;
      memcpy(&o, oh, 16);
      reinterpret_cast<uint4*>(xs16)[k] = o;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (live && (k & 7) == 0) xsum[(k >> 3) * 8] = sum;
  }
}

template <int BITS, int NBT, int RW, int EPI>
__global__ void __launch_bounds__(kThreads, 2)
    qmv_kernel(const __grid_constant__ QmvParams p, const __grid_constant__ CUtensorMap tmw,
               const __grid_constant__ CUtensorMap tmsb) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int TB = BITS == 4 ? 512 : 1024;
  const int CG = p.CG, GC = p.GC, SC = p.SC, stages = p.stages;
  const int nchunks = GC / CG;
  const Smem L = smem_layout(BITS, NBT, RW, CG, GC, stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
  volatile int* dead = reinterpret_cast<volatile int*>(smem + L.dead);
  __half* xs16 = reinterpret_cast<__half*>(smem + L.xs);
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* uv = reinterpret_cast<float*>(smem + L.uv);
  float* ev = reinterpret_cast<float*>(smem + L.ev);
  float* misc = reinterpret_cast<float*>(smem + L.misc);
  volatile int* flag = reinterpret_cast<volatile int*>(misc + 60);

  const int rows_units = p.N / 16 / RW;
  const int units = rows_units * SC;
  const int sc = blockIdx.x % SC;         // constant per CTA: gridDim.x is a multiple of SC
  const int k0 = sc * GC * 64;
  const int my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int rb0 = blockIdx.x / SC, rb_step = gridDim.x / SC;  // unit i covers row block rb0 + i rb_step

  if (tid == 0) {
    trace_mark(p.trace, 0);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *dead = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer: stream every chunk of this CTA's units through the ring (weights only, so it
    // runs ahead of the upstream kernel under programmatic dependent launch)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmsb)) : "memory");
      int slot = 0, phase = 0, issued = 0;
      for (int i = 0; i < my_units; ++i) {
        const int rb = rb0 + i * rb_step;
        for (int c = 0; c < nchunks; ++c, ++issued) {
          if (issued >= stages && !*dead) {
            if (!mbar_wait_bounded(&empty[slot], phase ^ 1, p.err)) *dead = 1;
          }
          if (*dead) break;
          uint8_t* dst = smem + L.ring + slot * L.stage_bytes;
          mbar_arrive_expect_tx(&full[slot], RW * CG * (TB + 64));
          if (p.bulk) {
            // plain bulk copies: a row tile's CG groups are contiguous in the row-tile-major pack
            for (int r2 = 0; r2 < RW; ++r2) {
              const size_t t = static_cast<size_t>(rb * RW + r2) * p.G + sc * GC + c * CG;
              bulk_g2s(dst + r2 * CG * TB, p.w + t * TB, CG * TB, &full[slot]);
              bulk_g2s(dst + L.wbytes + r2 * CG * 64, p.sb + t * 64, CG * 64, &full[slot]);
            }
          } else {
            tma_load_3d(dst, &tmw, 0, sc * GC + c * CG, rb * RW, &full[slot]);
            tma_load_3d(dst + L.wbytes, &tmsb, 0, sc * GC + c * CG, rb * RW, &full[slot]);
          }
          if (++slot == stages) { slot = 0; phase ^= 1; }
        }
        if (*dead) break;
      }
    }
    return;
  }

  // ---------------- consumers
  const int nb = p.nb;
  const int n8 = GC * 8;  // 8-element vectors of this CTA's K range, per activation row
  // The staging below gives vector k of every row to thread k % 512, so when 512 is a multiple of n8 each thread
  // owns one vector index: its norm gain (a weight) is loaded before the dependency wait.
  const bool fixed_k = kConsumers % n8 == 0;
  uint4 gpre = make_uint4(0u, 0u, 0u, 0u);
  if (p.norm_gain && fixed_k && tid < n8) gpre = reinterpret_cast<const uint4*>(p.norm_gain + k0)[tid];
  // The residual rows of the first unit: written by a kernel at least two launches back (the upstream kernel only
  // passed its own dependency wait on it), so they are read now, from L2, before this kernel's wait.
  float* resv = reinterpret_cast<float*>(smem + L.resv);
  constexpr bool kRes = EPI == EPI_RES1 || EPI == EPI_RES2;
  if (kRes && my_units > 0) {
    const int row0 = rb0 * RW * 16;
    for (int t = tid; t < RW * 16 * NBT; t += kConsumers) {
      const int r = t / NBT, b = t % NBT;
      float v = 0.f;
      if (b < nb) {
        const size_t at = static_cast<size_t>(b) * p.res_ld + row0 + r;
        v = EPI == EPI_RES1 ? __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(p.res16) + at)))
                            : __ldcg(p.res32 + at);
      }
      resv[t] = v;
    }
  }
  // The RoPE (cos, sin) of the first unit's pairs at the sequence's position, when the position was written by an
  // earlier kernel than the upstream one (pos_ready: every qkv launch after the step's first).
  constexpr bool kRope = EPI == EPI_QKV;
  if (kRope && p.pos_ready && my_units > 0) {
    const int row0 = rb0 * RW * 16, half = p.hd / 2;
    for (int t = tid; t < RW * 8 * NBT; t += kConsumers) {
      const int pr = t / NBT, b = t % NBT;
      float c = 0.f, sn = 0.f;
      if (b < nb) {
        const int tile = pr / 8, r = pr % 8;
        const int tt = ((row0 + tile * 16) % p.hd) / 16;
        int pos = static_cast<int>(__ldcg(p.q0 + b));
        if (pos > p.cap - 1) pos = p.cap - 1;
        c = p.cos_t[static_cast<size_t>(pos) * half + 8 * tt + r];
        sn = p.sin_t[static_cast<size_t>(pos) * half + 8 * tt + r];
      }
      resv[2 * t] = c;
      resv[2 * t + 1] = sn;
    }
  }
  if (p.pdl) {
    pdl_wait();
    if (p.pdl == 1) pdl_launch_dependents();
  }
  if (tid == 0) trace_mark(p.trace, 1);
  if (nb == 1 && SC == 1) {
    stage_row1(p, xs16, xsum, red);  // batch 1: one L2 round trip, x and gains held in registers
  } else {
  // RMSNorm: each row's sum of squares over the whole row (all p.K columns), every row's loads independent
  if (p.norm_gain) {
    float ssb[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      ssb[b] = 0.f;
      if (b < nb) {
        for (int k = tid; k < p.K / 8; k += kConsumers) {
          float v[8];
          load8(p, b, k * 8, v);
#pragma unroll
          for (int j = 0; j < 8; ++j) ssb[b] = fmaf(v[j], v[j], ssb[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const float t = warp_sum(ssb[b]);
      if (lane == 0 && b < nb) red[warp * 8 + b] = t;
    }
    consumer_sync();
  }
  // stage the rows as fp16 (normalised and scaled by the gain when given) and the per-group sums of the staged
  // values; the 8 vectors of a 64-group sit in 8 adjacent lanes. Every thread runs the same number of steps.
  const int steps = (n8 + kConsumers - 1) / kConsumers;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    if (b < nb) {
      float r = 1.0f;
      if (p.norm_gain) {
        float tot = 0.f;
        for (int w = 0; w < kConsumerWarps; ++w) tot += red[w * 8 + b];
        r = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
      }
      __half* dst = xs16 + b * L.xstride;
      for (int st = 0; st < steps; ++st) {
        const int k = tid + st * kConsumers;
        const bool live = k < n8;
        float v[8];
        if (live) {
          load8(p, b, k0 + k * 8, v);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = 0.f;
        }
        if (p.norm_gain && live) {
          const uint4 gu = fixed_k ? gpre : reinterpret_cast<const uint4*>(p.norm_gain + k0)[k];
          __half2 gh[4];
          memcpy(gh, &gu, 16);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 g = __half22float2(gh[j]);
            v[2 * j] = (v[2 * j] * r) * g.x;
            v[2 * j + 1] = (v[2 * j + 1] * r) * g.y;
          }
        }
        __half2 oh[4];
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          oh[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
          const float2 f = __half22float2(oh[j]);
          sum += f.x + f.y;
        }
        if (live) {
          uint4 o;
          memcpy(&o, oh, 16);
          reinterpret_cast<uint4*>(dst)[k] = o;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (live && (k & 7) == 0) xsum[(k >> 3) * 8 + b] = sum;
      }
    }
  }
  }
  if (EPI == EPI_ARGMAX && tid < 8) {
    misc[2 * tid] = -INFINITY;
    misc[2 * tid + 1] = __int_as_float(0x7fffffff);
  }
  consumer_sync();
  if (p.pdl == 2) pdl_launch_dependents();  // the dependent kernel's weight prefetch starts once x is staged
  if (tid == 0) trace_mark(p.trace, 3);

  const int rr = warp % RW, kw = warp / RW;
  constexpr int KW = kConsumerWarps / RW;
  const int r8 = lane >> 2, c4 = lane & 3;
  const int col = r8 < nb ? r8 : nb - 1;
  const int gpw = kw < CG ? (CG - kw + KW - 1) / KW : 0;  // groups of one chunk for this warp
  // this lane's shared addresses: x row, column sums, and (per stage) weights and scale/bias of its row tile
  const uint32_t ax0 = smem_u32(xs16 + col * L.xstride) + c4 * 32;
  const uint32_t axs0 = smem_u32(xsum) + c4 * 8;
  const uint32_t ring0 = smem_u32(smem + L.ring);
  const uint32_t lane_w = static_cast<uint32_t>(rr * CG * TB + lane * 16);
  const uint32_t lane_sb = static_cast<uint32_t>(L.wbytes + rr * CG * 64 + r8 * 8);
  bool waited_ok = true;
  int slot = 0, phase = 0;

  for (int i = 0; i < my_units; ++i) {
    const int rb = rb0 + i * rb_step;
    float ys[4] = {0.f, 0.f, 0.f, 0.f}, yb[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < nchunks; ++c) {
      if (!*dead && !mbar_wait_bounded(&full[slot], phase, p.err)) {
        *dead = 1;
        waited_ok = false;
      }
      if (i == 0 && c == 0 && tid == 0) trace_mark(p.trace, 5);
      const uint32_t st = ring0 + slot * L.stage_bytes;
      uint32_t aw = st + lane_w + kw * TB;
      uint32_t asb = st + lane_sb + kw * 64;
      uint32_t ax = ax0 + (c * CG + kw) * 128;
      uint32_t axs = axs0 + (c * CG + kw) * 32;
#pragma unroll 4
      for (int j = 0; j < gpw; ++j) {
        group_step<BITS, NBT>(aw, asb, ax, axs, p.sdt, ys, yb);
        aw += KW * TB;
        asb += KW * 64;
        ax += KW * 128;
        axs += KW * 32;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == stages) { slot = 0; phase ^= 1; }
    }
    // this warp's partial rows (row r8 and r8 + 8, columns 2 c4 and 2 c4 + 1) to shared memory
    float* rw = red + warp * 16 * NBT;
    if (2 * c4 < NBT) {
      rw[r8 * NBT + 2 * c4] = fmaf(ys[0], k2p24, yb[0]);
      rw[(r8 + 8) * NBT + 2 * c4] = fmaf(ys[2], k2p24, yb[2]);
    }
    if (2 * c4 + 1 < NBT) {
      rw[r8 * NBT + 2 * c4 + 1] = fmaf(ys[1], k2p24, yb[1]);
      rw[(r8 + 8) * NBT + 2 * c4 + 1] = fmaf(ys[3], k2p24, yb[3]);
    }
    consumer_sync();
    // element t = row NBT + b of the unit: the KW K-lane warps' partial sums of its row, added in warp order
    auto reduced = [red](int t) {
      const int row = t / NBT, b = t % NBT;
      const int rt = row / 16, rw16 = row % 16;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < KW; ++q) s += red[(rt + q * RW) * 16 * NBT + rw16 * NBT + b];
      return s;
    };
    const int row0 = rb * RW * 16;
    if (SC == 1 && EPI != EPI_ARGMAX) {
      // each epilogue thread adds up the rows it needs itself (the same sums in the same order): no barrier between
      // the reduction and the epilogue; one before the next unit's partial sums overwrite `red`
      epilogue<EPI, NBT>(p, row0, RW * 16, reduced, misc,
                         (kRes || (kRope && p.pos_ready)) && i == 0 ? resv : nullptr);
      if (i + 1 < my_units) consumer_sync();
      continue;
    }
    for (int t = tid; t < RW * 16 * NBT; t += kConsumers) uv[t] = reduced(t);
    consumer_sync();
    auto uv_at = [uv](int t) { return uv[t]; };
    if (SC == 1) {
      epilogue<EPI, NBT>(p, row0, RW * 16, uv_at, misc, (kRes || (kRope && p.pos_ready)) && i == 0 ? resv : nullptr);
    } else {
      // split K: this unit's partial rows to scratch; the last of the SC units of these rows sums them in order
      for (int t = tid; t < RW * 16 * NBT; t += kConsumers) {
        const int row = t / NBT, b = t % NBT;
        if (b < nb) p.part[(static_cast<size_t>(sc) * p.N + row0 + row) * nb + b] = uv[t];
      }
      __threadfence();
      consumer_sync();
      if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counters[rb], 1u);
        *flag = prev == static_cast<unsigned>(SC) - 1;
        if (*flag) atomicExch(&p.counters[rb], 0u);
      }
      consumer_sync();
      if (*flag) {
        __threadfence();
        for (int t = tid; t < RW * 16 * NBT; t += kConsumers) {
          const int row = t / NBT, b = t % NBT;
          float s = 0.f;
          if (b < nb)
            for (int q = 0; q < SC; ++q) s += ld_cg(p.part + (static_cast<size_t>(q) * p.N + row0 + row) * nb + b);
          ev[t] = s;
        }
        consumer_sync();
        auto ev_at = [ev](int t) { return ev[t]; };
        epilogue<EPI, NBT>(p, row0, RW * 16, ev_at, misc,
                           (kRes || (kRope && p.pos_ready)) && i == 0 ? resv : nullptr);
      }
      consumer_sync();
    }
  }

  if (p.pdl == 3) pdl_launch_dependents();  // mode 3: the successor starts once every chunk is consumed
  if (consumer_sync_or(!waited_ok)) return;  // a stage never landed: the error word is set; leave uniformly
  if (tid == 0) trace_mark(p.trace, 4);

  if (EPI == EPI_ARGMAX) {
    if (tid < 8) {
      p.pairs[(static_cast<size_t>(blockIdx.x) * 8 + tid) * 2] = misc[2 * tid];
      p.pairs[(static_cast<size_t>(blockIdx.x) * 8 + tid) * 2 + 1] = misc[2 * tid + 1];
    }
    __threadfence();
    consumer_sync();
    if (tid == 0) {
      const unsigned prev = atomicAdd(&p.counters[0], 1u);
      *flag = prev == gridDim.x - 1;
      if (*flag) atomicExch(&p.counters[0], 0u);
    }
    consumer_sync();
    if (*flag) {
      __threadfence();
      argmax_finish(p, misc);
    }
  }
  if (tid == 0) trace_mark(p.trace, 2);
}

template <int BITS, int NBT, int RW, int EPI>
int launch_one(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, const CUtensorMap& tw,
               const CUtensorMap& ts, cudaStream_t s) {
  auto kern = qmv_kernel<BITS, NBT, RW, EPI>;
  if (ctx && static_cast<int>(plan.smem) + 1024 > ctx->max_smem_optin)
    return fail(AGXC_EINVAL, "qmv: plan needs more shared memory than the device offers");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (p.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, kern, p, tw, ts));
  return 0;
}

// The opt-in limit covers static + dynamic shared memory: each kernel may take the limit less its static part.
template <typename K>
int allow_smem(K kern, int optin) {
  cudaFuncAttributes fa;
  AGXC_CUDA(cudaFuncGetAttributes(&fa, kern));
  AGXC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - static_cast<int>(fa.sharedSizeBytes)));
  return 0;
}

// The row-tile counts per unit each epilogue is instantiated for (the planner chooses among these).
template <int EPI>
struct RwSet;
template <> struct RwSet<EPI_F32> { static constexpr int v[4] = {1, 2, 4, 8}; };
template <> struct RwSet<EPI_RES1> { static constexpr int v[4] = {1, 2, 4, 8}; };
template <> struct RwSet<EPI_RES2> { static constexpr int v[4] = {1, 2, 4, 8}; };
template <> struct RwSet<EPI_SWIGLU> { static constexpr int v[4] = {2, 4, 8, 8}; };
template <> struct RwSet<EPI_QKV> { static constexpr int v[4] = {1, 2, 4, 8}; };
template <> struct RwSet<EPI_ARGMAX> { static constexpr int v[4] = {1, 2, 4, 8}; };

template <int BITS, int NBT, int EPI>
int dispatch_rw(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, const CUtensorMap& tw,
                const CUtensorMap& ts, cudaStream_t s) {
  switch (plan.RW) {
    case 1: if (EPI != EPI_SWIGLU) return launch_one<BITS, NBT, 1, EPI>(ctx, p, plan, tw, ts, s); break;
    case 2: return launch_one<BITS, NBT, 2, EPI>(ctx, p, plan, tw, ts, s);
    case 4: return launch_one<BITS, NBT, 4, EPI>(ctx, p, plan, tw, ts, s);
    case 8: return launch_one<BITS, NBT, 8, EPI>(ctx, p, plan, tw, ts, s);
  }
  return fail(AGXC_EINVAL, "qmv: no kernel for this RW");
}

template <int BITS, int NBT>
int dispatch_epi(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, int epi, const CUtensorMap& tw,
                 const CUtensorMap& ts, cudaStream_t s) {
  switch (epi) {
    case EPI_F32: return dispatch_rw<BITS, NBT, EPI_F32>(ctx, p, plan, tw, ts, s);
    case EPI_RES1: return dispatch_rw<BITS, NBT, EPI_RES1>(ctx, p, plan, tw, ts, s);
    case EPI_RES2: return dispatch_rw<BITS, NBT, EPI_RES2>(ctx, p, plan, tw, ts, s);
    case EPI_SWIGLU: return dispatch_rw<BITS, NBT, EPI_SWIGLU>(ctx, p, plan, tw, ts, s);
    case EPI_QKV: return dispatch_rw<BITS, NBT, EPI_QKV>(ctx, p, plan, tw, ts, s);
    case EPI_ARGMAX: return dispatch_rw<BITS, NBT, EPI_ARGMAX>(ctx, p, plan, tw, ts, s);
  }
  return fail(AGXC_EINVAL, "qmv: unknown epilogue");
}

template <int BITS, int NBT, int EPI>
int configure_rw(int smem) {
  int rc = 0;
  if (EPI != EPI_SWIGLU && (rc = allow_smem(qmv_kernel<BITS, NBT, 1, EPI>, smem))) return rc;
  if ((rc = allow_smem(qmv_kernel<BITS, NBT, 2, EPI>, smem)) || (rc = allow_smem(qmv_kernel<BITS, NBT, 4, EPI>, smem)) ||
      (rc = allow_smem(qmv_kernel<BITS, NBT, 8, EPI>, smem)))
    return rc;
  return 0;
}

template <int BITS, int NBT>
int configure_nb(int smem) {
  int rc;
  if ((rc = configure_rw<BITS, NBT, EPI_F32>(smem)) || (rc = configure_rw<BITS, NBT, EPI_RES1>(smem)) ||
      (rc = configure_rw<BITS, NBT, EPI_RES2>(smem)) || (rc = configure_rw<BITS, NBT, EPI_QKV>(smem)) ||
      (rc = configure_rw<BITS, NBT, EPI_ARGMAX>(smem)) || (rc = configure_rw<BITS, NBT, EPI_SWIGLU>(smem)))
    return rc;
  return 0;
}

}  // namespace gemv
}  // namespace agxc

// One translation unit per (bits, activation rows) instantiates these.
#define AGXC_GEMV_INSTANTIATE(BITS, NBT)                                                                    \
  namespace agxc {                                                                                          \
  int qmv_dispatch_##BITS##_##NBT(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, int epi,     \
                                  const CUtensorMap& tw, const CUtensorMap& ts, cudaStream_t s) {           \
    return gemv::dispatch_epi<BITS, NBT>(ctx, p, plan, epi, tw, ts, s);                                     \
  }                                                                                                         \
  int qmv_configure_##BITS##_##NBT(int smem) { return gemv::configure_nb<BITS, NBT>(smem); }               \
  }
