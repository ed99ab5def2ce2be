// gemv.cu — the quantized GEMV family of the decode step (the reference's build_qmv2 and its fused epilogues,
// agxforge/kernels/qmv.py:341-881), written for sm_100a.
//
// y[b][n] = sum_g ( s[n,g] * sum_{k in g} q[n,k] x[b][k]  +  b[n,g] * sum_{k in g} x[b][k] )
//
// The reference factorises each trip the same way (qmv.py:1577-1649: t = sum q x, acc += s t + b sx). Here:
//   * the weight stream moves by bulk TMA copies (cp.async.bulk + mbarrier) of whole work units — RW row tiles x GC
//     groups, contiguous in the tile layout — into a ring of shared-memory stages, issued ahead by one thread;
//   * each warp dequantises its lane's fields with one AND (4-bit; one PRMT for 8-bit) per two weights into fp16
//     SUBNORMALS q * 2^-24 (exact), so no subtract or convert is needed, and forms sum q x on the tensor cores with
//     mma.sync m16n8k16 (weight rows = M, activation rows = N <= 8, fp32 accumulate); the 2^24 (2^20 for the
//     upper nibble pair) is folded into the scale on the CUDA cores;
//   * the activation rows are staged in shared memory (fp16 values: every GEMV input of the decode graph is an fp16
//     tensor — the normed rows, the attention output, the SwiGLU product), with their per-group sums;
//   * the RMSNorm of the input is fused in front (with_norm, qmv.py:176-183), recomputed per CTA from the row;
//   * split-K partials (and epilogue blocks wider than a unit: a RoPE head) meet through a scratch buffer and a
//     last-arriver counter (no spin-waits).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr float k2p24 = 16777216.0f;
constexpr float k2p20 = 1048576.0f;

struct Smem {
  // offsets in bytes from the dynamic shared memory base
  int bars, ring, stage_bytes, wbytes, xs, xstride, xsum, red, uv, ev, misc;
};

__host__ __device__ inline Smem smem_layout(int bits, int nbt, int RW, int GC, int stages, int EB) {
  Smem L;
  const int TB = bits == 4 ? 512 : 1024;
  L.bars = 0;
  L.ring = 128;
  L.wbytes = RW * GC * TB;
  L.stage_bytes = (L.wbytes + RW * GC * 64 + 127) / 128 * 128;
  L.xs = L.ring + stages * L.stage_bytes;
  L.xstride = GC * 64 + 8;  // halves; the 16-byte pad keeps 8 rows' fragment loads bank-conflict free
  L.xsum = L.xs + ((nbt * L.xstride * 2 + 127) / 128) * 128;
  L.red = L.xsum + GC * 8 * 4;
  L.uv = L.red + kWarps * 16 * 8 * 4;
  L.ev = L.uv + RW * 16 * 8 * 4;
  L.misc = L.ev + EB * 16 * 8 * 4;
  return L;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// ------------------------------------------------------------------------------------------------ epilogues
// vals: [rows][8] fp32 (row-major, column = activation row b) for the block starting at physical row `row0`.
template <int EPI>
__device__ void epilogue(const QmvParams& p, int row0, int rows, const float* vals, float* misc) {
  const int tid = threadIdx.x;
  const int nb = p.nb;
  if (EPI == EPI_F32) {
    for (int t = tid; t < rows * nb; t += kThreads) {
      const int r = t / nb, b = t % nb;
      p.out_f32[static_cast<size_t>(b) * p.out_ld + row0 + r] = vals[r * 8 + b];
    }
  } else if (EPI == EPI_RES1) {
    for (int t = tid; t < rows * nb; t += kThreads) {
      const int r = t / nb, b = t % nb;
      const float x = __half2float(p.res16[static_cast<size_t>(b) * p.res_ld + row0 + r]);
      p.out_f32[static_cast<size_t>(b) * p.out_ld + row0 + r] = vals[r * 8 + b] + x;
    }
  } else if (EPI == EPI_RES2) {
    for (int t = tid; t < rows * nb; t += kThreads) {
      const int r = t / nb, b = t % nb;
      const float h = p.res32[static_cast<size_t>(b) * p.res_ld + row0 + r];
      p.out_f16[static_cast<size_t>(b) * p.out_ld + row0 + r] = __float2half_rn(vals[r * 8 + b] + h);
    }
  } else if (EPI == EPI_SWIGLU) {
    // the block is a gate tile (rows 0..15) and its up tile (rows 16..31); output index (row0 / 32) * 16 + r
    const int o0 = row0 / 32 * 16;
    for (int t = tid; t < 16 * nb; t += kThreads) {
      const int r = t / nb, b = t % nb;
      const float g = vals[r * 8 + b], u = vals[(16 + r) * 8 + b];
      p.out_f16[static_cast<size_t>(b) * p.out_ld + o0 + r] = __float2half_rn(silu_f(g) * u);
    }
  } else if (EPI == EPI_QKV) {
    // one head: bias, rotate-half RoPE at the sequence's position (q and k), q scaled for the base-2 softmax,
    // fp16 q to the attention's input; fp16 k and v appended to the cache at the position.
    const int hd = p.hd, half = hd / 2;
    const int head = row0 / hd;
    for (int t = tid; t < hd * nb; t += kThreads) {
      const int i = t / nb, b = t % nb;
      float y = vals[i * 8 + b];
      if (p.bias) y += __half2float(p.bias[row0 + i]);
      int pos = static_cast<int>(p.q0[b]);
      if (pos > p.cap - 1) pos = p.cap - 1;
      if (head < p.H + p.KVH) {
        const int j = i < half ? i + half : i - half;
        float yp = vals[j * 8 + b];
        if (p.bias) yp += __half2float(p.bias[row0 + j]);
        const int ci = i < half ? i : i - half;
        const float c = p.cos_t[static_cast<size_t>(pos) * half + ci];
        const float s = p.sin_t[static_cast<size_t>(pos) * half + ci];
        const float o = i < half ? y * c - yp * s : y * c + yp * s;
        if (head < p.H) {
          p.q16[(static_cast<size_t>(b) * p.H + head) * hd + i] = __float2half_rn(o * p.qscale);
        } else {
          const int kv = head - p.H;
          p.kcache[((static_cast<size_t>(b) * p.KVH + kv) * p.cap + pos) * hd + i] = __float2half_rn(o);
        }
      } else {
        const int kv = head - p.H - p.KVH;
        p.vcache[((static_cast<size_t>(b) * p.KVH + kv) * p.cap + pos) * hd + i] = __float2half_rn(y);
      }
    }
  } else if (EPI == EPI_ARGMAX) {
    if (p.out_f32) {
      for (int t = tid; t < rows * nb; t += kThreads) {
        const int r = t / nb, b = t % nb;
        p.out_f32[static_cast<size_t>(b) * p.V + row0 + r] = vals[r * 8 + b];
      }
    }
    if (tid < nb) {
      // running first-maximum of this CTA: misc[2b] value, misc[2b+1] index (as int bits)
      float bv = misc[2 * tid];
      int bi = __float_as_int(misc[2 * tid + 1]);
      for (int r = 0; r < rows; ++r) {
        const float v = vals[r * 8 + tid];
        const int idx = row0 + r;
        if (v > bv || (v == bv && idx < bi)) { bv = v; bi = idx; }
      }
      misc[2 * tid] = bv;
      misc[2 * tid + 1] = __int_as_float(bi);
    }
  }
}

// The argmax's cross-CTA step and the generation step, run by the last CTA to finish (argmax.py:141-215,
// assemble.py:918-930): token = the forced token if one is pending, else the logged prompt token, else the first
// maximum; log it, write its embedding row as the next x, advance q0 (clamped to cap - 1).
__device__ void argmax_finish(const QmvParams& p, float* misc) {
  const int tid = threadIdx.x;
  const int nb = p.nb;
  __shared__ int s_tok[8];
  for (int b = 0; b < nb; ++b) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = tid; c < static_cast<int>(gridDim.x); c += kThreads) {
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
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kWarps; ++w) {
        const float ov = misc[16 + 2 * w];
        const int oi = __float_as_int(misc[17 + 2 * w]);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      uint32_t pos = p.q0_rw[b];
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
    __syncthreads();
  }
  // the chosen tokens' embedding rows become the next step's x
  const int dv = p.d / 8;
  for (int t = tid; t < nb * dv; t += kThreads) {
    const int b = t / dv, i = t % dv;
    const uint4* src = reinterpret_cast<const uint4*>(p.embed + static_cast<size_t>(s_tok[b]) * p.d);
    reinterpret_cast<uint4*>(p.x_next + static_cast<size_t>(b) * p.d)[i] = src[i];
  }
}

template <int BITS, int NBT, int RW, int EPI>
__global__ void __launch_bounds__(kThreads) qmv_kernel(QmvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int TB = BITS == 4 ? 512 : 1024;
  constexpr int EB_MAX = EPI == EPI_QKV ? 8 : (EPI == EPI_SWIGLU ? 2 : 1);
  const int GC = p.GC, SC = p.SC, stages = p.stages;
  const int EB = EPI == EPI_QKV ? p.hd / 16 : (EPI == EPI_SWIGLU ? 2 : 1);
  const Smem L = smem_layout(BITS, NBT, RW, GC, stages, EB_MAX);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  __half* xs16 = reinterpret_cast<__half*>(smem + L.xs);
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* uv = reinterpret_cast<float*>(smem + L.uv);
  float* ev = reinterpret_cast<float*>(smem + L.ev);
  float* misc = reinterpret_cast<float*>(smem + L.misc);
  __shared__ int s_flag;

  const int rows_units = p.N / 16 / RW;
  const int units = rows_units * SC;
  const int sc = blockIdx.x % SC;         // constant per CTA: gridDim.x is a multiple of SC
  const int k0 = sc * GC * 64;
  const int my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  auto issue = [&](int i) {  // unit i of this CTA into stage i % stages
    const int u = blockIdx.x + i * gridDim.x;
    const int rb = u / SC;
    const int st = i % stages;
    uint8_t* dst = smem + L.ring + st * L.stage_bytes;
    mbar_arrive_expect_tx(&bars[st], RW * GC * (TB + 64));
    for (int r = 0; r < RW; ++r) {
      const size_t tile0 = static_cast<size_t>(rb * RW + r) * p.G + static_cast<size_t>(sc) * GC;
      bulk_g2s(dst + r * GC * TB, p.w + tile0 * TB, GC * TB, &bars[st]);
      bulk_g2s(dst + L.wbytes + r * GC * 64, p.sb + tile0 * 64, GC * 64, &bars[st]);
    }
  };

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    for (int i = 0; i < stages && i < my_units; ++i) issue(i);
  }
  // everything above reads only weights: with programmatic dependent launch it overlaps the upstream kernel
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }

  // ---- stage the activation rows of this CTA's K chunk (RMSNorm fused when a gain is given)
  const int nb = p.nb;
  for (int b = 0; b < nb; ++b) {
    float r = 1.0f;
    if (p.norm_gain) {
      float ss = 0.f;
      if (p.x_f32) {
        const float* xr = static_cast<const float*>(p.x) + static_cast<size_t>(b) * p.x_ld;
        for (int k = tid; k < p.K; k += kThreads) { const float v = xr[k]; ss = fmaf(v, v, ss); }
      } else {
        const __half* xr = static_cast<const __half*>(p.x) + static_cast<size_t>(b) * p.x_ld;
        for (int k = tid; k < p.K; k += kThreads) { const float v = __half2float(xr[k]); ss = fmaf(v, v, ss); }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      if (tid == 0) {
        float tot = 0.f;
        for (int w = 0; w < kWarps; ++w) tot += red[w];
        red[64] = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
      }
      __syncthreads();
      r = red[64];
      __syncthreads();
    }
    __half* dst = xs16 + b * L.xstride;
    for (int k = tid; k < GC * 64; k += kThreads) {
      float v;
      if (p.x_f32) v = static_cast<const float*>(p.x)[static_cast<size_t>(b) * p.x_ld + k0 + k];
      else v = __half2float(static_cast<const __half*>(p.x)[static_cast<size_t>(b) * p.x_ld + k0 + k]);
      if (p.norm_gain) v = (v * r) * __half2float(p.norm_gain[k0 + k]);
      dst[k] = __float2half_rn(v);
    }
  }
  __syncthreads();
  for (int t = tid; t < GC * 8; t += kThreads) {
    const int g = t / 8, b = t % 8;
    float s = 0.f;
    if (b < nb) {
      const __half* src = xs16 + b * L.xstride + g * 64;
      for (int k = 0; k < 64; ++k) s += __half2float(src[k]);
    }
    xsum[t] = s;
  }
  if (EPI == EPI_ARGMAX && tid < 8) {
    misc[2 * tid] = -INFINITY;
    misc[2 * tid + 1] = __int_as_float(0x7fffffff);
  }
  __syncthreads();

  const int rr = warp % RW, kw = warp / RW;
  constexpr int KW = kWarps / RW;
  const int r8 = lane >> 2, c4 = lane & 3;
  const int col = r8 < nb ? r8 : nb - 1;
  const __half* xrow = xs16 + col * L.xstride;
  bool ok = true;
  int fail_unit = 0;

  for (int i = 0; i < my_units; ++i) {
    const int u = blockIdx.x + i * gridDim.x;
    const int rb = u / SC;
    const int st = i % stages;
    // every thread waits (bounded); a stage that never lands makes the whole CTA leave at the barrier below
    const bool landed = mbar_wait_bounded(&bars[st], (i / stages) & 1, p.err);
    const uint8_t* wst = smem + L.ring + st * L.stage_bytes + rr * GC * TB;
    const uint8_t* sbst = smem + L.ring + st * L.stage_bytes + L.wbytes + rr * GC * 64;
    float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
    for (int gi = kw; gi < GC; gi += KW) {
      const uint2 sv = *reinterpret_cast<const uint2*>(sbst + gi * 64 + r8 * 8);
      const uint4 xa = *reinterpret_cast<const uint4*>(xrow + gi * 64 + c4 * 16);
      const uint4 xb = *reinterpret_cast<const uint4*>(xrow + gi * 64 + c4 * 16 + 8);
      const float2 xsv = *reinterpret_cast<const float2*>(xsum + gi * 8 + 2 * c4);
      const float s_r = scale_to_f32(static_cast<uint16_t>(sv.x & 0xffffu), p.sdt);
      const float s_r8 = scale_to_f32(static_cast<uint16_t>(sv.x >> 16), p.sdt);
      const float b_r = scale_to_f32(static_cast<uint16_t>(sv.y & 0xffffu), p.sdt);
      const float b_r8 = scale_to_f32(static_cast<uint16_t>(sv.y >> 16), p.sdt);
      if (BITS == 4) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wst + gi * TB + lane * 16);
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
        constexpr uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u;
        mma_16816(a0, a1, a2, a3, wv.x & M0, wv.y & M0, wv.z & M0, wv.w & M0, xa.x, xa.y);
        mma_16816(b0, b1, b2, b3, wv.x & M1, wv.y & M1, wv.z & M1, wv.w & M1, xa.z, xa.w);
        const uint32_t sx = wv.x >> 8, sy = wv.y >> 8, sz = wv.z >> 8, sw = wv.w >> 8;
        mma_16816(a0, a1, a2, a3, sx & M0, sy & M0, sz & M0, sw & M0, xb.x, xb.y);
        mma_16816(b0, b1, b2, b3, sx & M1, sy & M1, sz & M1, sw & M1, xb.z, xb.w);
        const float sr24 = s_r * k2p24, sr20 = s_r * k2p20, s824 = s_r8 * k2p24, s820 = s_r8 * k2p20;
        y0 = fmaf(sr24, a0, y0); y0 = fmaf(sr20, b0, y0); y0 = fmaf(b_r, xsv.x, y0);
        y2 = fmaf(s824, a2, y2); y2 = fmaf(s820, b2, y2); y2 = fmaf(b_r8, xsv.x, y2);
        if (NBT > 1) {
          y1 = fmaf(sr24, a1, y1); y1 = fmaf(sr20, b1, y1); y1 = fmaf(b_r, xsv.y, y1);
          y3 = fmaf(s824, a3, y3); y3 = fmaf(s820, b3, y3); y3 = fmaf(b_r8, xsv.y, y3);
        }
      } else {
        const uint4 w0 = *reinterpret_cast<const uint4*>(wst + gi * TB + lane * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(wst + gi * TB + 512 + lane * 16);
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        constexpr uint32_t PL = 0x4140u, PH = 0x4342u;
        mma_16816(a0, a1, a2, a3, prmt(w0.x, 0, PL), prmt(w0.x, 0, PH), prmt(w0.y, 0, PL), prmt(w0.y, 0, PH), xa.x,
                  xa.y);
        mma_16816(a0, a1, a2, a3, prmt(w0.z, 0, PL), prmt(w0.z, 0, PH), prmt(w0.w, 0, PL), prmt(w0.w, 0, PH), xa.z,
                  xa.w);
        mma_16816(a0, a1, a2, a3, prmt(w1.x, 0, PL), prmt(w1.x, 0, PH), prmt(w1.y, 0, PL), prmt(w1.y, 0, PH), xb.x,
                  xb.y);
        mma_16816(a0, a1, a2, a3, prmt(w1.z, 0, PL), prmt(w1.z, 0, PH), prmt(w1.w, 0, PL), prmt(w1.w, 0, PH), xb.z,
                  xb.w);
        const float sr24 = s_r * k2p24, s824 = s_r8 * k2p24;
        y0 = fmaf(sr24, a0, y0); y0 = fmaf(b_r, xsv.x, y0);
        y2 = fmaf(s824, a2, y2); y2 = fmaf(b_r8, xsv.x, y2);
        if (NBT > 1) {
          y1 = fmaf(sr24, a1, y1); y1 = fmaf(b_r, xsv.y, y1);
          y3 = fmaf(s824, a3, y3); y3 = fmaf(b_r8, xsv.y, y3);
        }
      }
    }
    float* rw = red + warp * 128;
    rw[r8 * 8 + 2 * c4] = y0;
    rw[r8 * 8 + 2 * c4 + 1] = y1;
    rw[(r8 + 8) * 8 + 2 * c4] = y2;
    rw[(r8 + 8) * 8 + 2 * c4 + 1] = y3;
    if (__syncthreads_or(!landed)) {
      ok = false;
      fail_unit = i;
      break;
    }
    if (tid == 0 && i + stages < my_units) issue(i + stages);  // every warp is done with stage st
    for (int t = tid; t < RW * 16 * 8; t += kThreads) {
      const int row = t / 8, b = t % 8;
      const int rt = row / 16, rw16 = row % 16;
      float s = 0.f;
      for (int k = 0; k < KW; ++k) s += red[(rt + k * RW) * 128 + rw16 * 8 + b];
      uv[t] = s;
    }
    __syncthreads();
    const int row0 = rb * RW * 16;
    if (SC == 1 && EB <= RW) {
      epilogue<EPI>(p, row0, RW * 16, uv, misc);
    } else {
      // scratch path: this unit's partial rows, then the block's last arriver sums the chunks and runs the epilogue
      for (int t = tid; t < RW * 16 * nb; t += kThreads) {
        const int row = t / nb, b = t % nb;
        p.part[(static_cast<size_t>(sc) * p.N + row0 + row) * nb + b] = uv[row * 8 + b];
      }
      __threadfence();
      __syncthreads();
      const int blk = row0 / (EB * 16);
      const unsigned expect = static_cast<unsigned>((EB / RW) * SC);
      if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counters[blk], 1u);
        s_flag = prev == expect - 1;
        if (s_flag) atomicExch(&p.counters[blk], 0u);
      }
      __syncthreads();
      if (s_flag) {
        __threadfence();
        const int brow0 = blk * EB * 16;
        for (int t = tid; t < EB * 16 * 8; t += kThreads) {
          const int row = t / 8, b = t % 8;
          float s = 0.f;
          if (b < nb)
            for (int c = 0; c < SC; ++c) s += ld_cg(p.part + (static_cast<size_t>(c) * p.N + brow0 + row) * nb + b);
          ev[t] = s;
        }
        __syncthreads();
        epilogue<EPI>(p, brow0, EB * 16, ev, misc);
      }
    }
    __syncthreads();
  }

  if (!ok) {
    // a stage never arrived: drain what this CTA issued (bounded) and leave; the host reads the error word
    for (int j = fail_unit; j < fail_unit + stages && j < my_units; ++j)
      mbar_wait_bounded(&bars[j % stages], (j / stages) & 1, nullptr, 100000000ull);
    return;
  }

  if (EPI == EPI_ARGMAX) {
    if (tid < 8) {
      p.pairs[(static_cast<size_t>(blockIdx.x) * 8 + tid) * 2] = misc[2 * tid];
      p.pairs[(static_cast<size_t>(blockIdx.x) * 8 + tid) * 2 + 1] = misc[2 * tid + 1];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicAdd(&p.counters[0], 1u);
      s_flag = prev == gridDim.x - 1;
      if (s_flag) atomicExch(&p.counters[0], 0u);
    }
    __syncthreads();
    if (s_flag) {
      __threadfence();
      argmax_finish(p, misc);
    }
  }
}

template <int BITS, int NBT, int RW, int EPI>
int launch_one(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, cudaStream_t s) {
  auto kern = qmv_kernel<BITS, NBT, RW, EPI>;
  if (ctx && static_cast<int>(plan.smem) > ctx->max_smem_optin)
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
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
  return 0;
}

template <int BITS, int NBT>
int dispatch_epi(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, int epi, cudaStream_t s) {
  switch (epi) {
    case EPI_F32: return launch_one<BITS, NBT, 1, EPI_F32>(ctx, p, plan, s);
    case EPI_RES1: return launch_one<BITS, NBT, 1, EPI_RES1>(ctx, p, plan, s);
    case EPI_RES2: return launch_one<BITS, NBT, 1, EPI_RES2>(ctx, p, plan, s);
    case EPI_SWIGLU: return launch_one<BITS, NBT, 2, EPI_SWIGLU>(ctx, p, plan, s);
    case EPI_QKV: return launch_one<BITS, NBT, 1, EPI_QKV>(ctx, p, plan, s);
    case EPI_ARGMAX: return launch_one<BITS, NBT, 1, EPI_ARGMAX>(ctx, p, plan, s);
  }
  return fail(AGXC_EINVAL, "qmv: unknown epilogue");
}

template <int BITS>
int dispatch_nb(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, int epi, cudaStream_t s) {
  if (p.nb == 1) return dispatch_epi<BITS, 1>(ctx, p, plan, epi, s);
  if (p.nb == 2) return dispatch_epi<BITS, 2>(ctx, p, plan, epi, s);
  if (p.nb <= 4) return dispatch_epi<BITS, 4>(ctx, p, plan, epi, s);
  return dispatch_epi<BITS, 8>(ctx, p, plan, epi, s);
}

int nb_tmpl(int nb) { return nb == 1 ? 1 : nb == 2 ? 2 : nb <= 4 ? 4 : 8; }

template <int BITS, int NBT>
int configure_nb(int smem) {
  AGXC_CUDA(cudaFuncSetAttribute(qmv_kernel<BITS, NBT, 1, EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  AGXC_CUDA(cudaFuncSetAttribute(qmv_kernel<BITS, NBT, 1, EPI_RES1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  AGXC_CUDA(cudaFuncSetAttribute(qmv_kernel<BITS, NBT, 1, EPI_RES2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  AGXC_CUDA(cudaFuncSetAttribute(qmv_kernel<BITS, NBT, 2, EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  AGXC_CUDA(cudaFuncSetAttribute(qmv_kernel<BITS, NBT, 1, EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  AGXC_CUDA(cudaFuncSetAttribute(qmv_kernel<BITS, NBT, 1, EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  return 0;
}

}  // namespace

// Every GEMV instantiation may use up to the device's opt-in shared memory (set once per device, outside any
// stream capture).
int qmv_configure(const agxc_ctx* ctx) {
  const int smem = ctx->max_smem_optin;
  int rc;
  if ((rc = configure_nb<4, 1>(smem)) || (rc = configure_nb<4, 2>(smem)) || (rc = configure_nb<4, 4>(smem)) ||
      (rc = configure_nb<4, 8>(smem)) || (rc = configure_nb<8, 1>(smem)) || (rc = configure_nb<8, 2>(smem)) ||
      (rc = configure_nb<8, 4>(smem)) || (rc = configure_nb<8, 8>(smem)))
    return rc;
  return 0;
}

QmvPlan plan_qmv(const agxc_ctx* ctx, int N, int K, int bits, int nb, int epi, int hd, int splits) {
  QmvPlan P;
  P.RW = epi == EPI_SWIGLU ? 2 : 1;
  P.EB = epi == EPI_QKV ? hd / 16 : (epi == EPI_SWIGLU ? 2 : 1);
  const int G = K / 64;
  const int TB = tile_bytes(bits);
  const int rows_units = N / 16 / P.RW;
  const int sms = ctx ? ctx->num_sms : kNumSMs;
  const int target = 2 * sms;
  const int max_stage = 40 * 1024;
  int SC = 0;
  if (splits > 0 && G % splits == 0) {
    SC = splits;
  } else {
    int fallback = 0;
    for (int c = 1; c <= G; ++c) {
      if (G % c) continue;
      const int GC = G / c;
      if (P.RW * GC * (TB + 64) > max_stage) continue;
      if (!fallback) fallback = c;
      SC = c;
      if (rows_units * c >= target) break;
      if (GC <= kWarps / P.RW) break;  // one group per warp: do not split further
    }
    if (!SC) SC = fallback ? fallback : G;
  }
  if (epi == EPI_ARGMAX) SC = 1;  // the argmax needs whole rows per unit
  P.SC = SC;
  P.GC = G / SC;
  const int stage_bytes = (P.RW * P.GC * (TB + 64) + 127) / 128 * 128;
  P.stages = std::max(2, std::min(4, (96 * 1024) / stage_bytes));
  const int units = rows_units * SC;
  int grid = std::min(units, target);
  grid = std::max(SC, grid / SC * SC);
  P.grid = grid;
  const Smem L = smem_layout(bits, nb_tmpl(nb), P.RW, P.GC, P.stages, epi == EPI_QKV ? 8 : (epi == EPI_SWIGLU ? 2 : 1));
  P.smem = L.misc + 256;
  return P;
}

size_t qmv_part_floats(const QmvPlan& p, int N, int nb, int epi) {
  if (p.SC == 1 && p.EB <= p.RW) return 0;
  return static_cast<size_t>(p.SC) * N * nb;
}

int launch_qmv_epi(const agxc_ctx* ctx, QmvParams p, const QmvPlan& plan, int epi, cudaStream_t s) {
  if (p.N % 16 || p.K % 64) return fail(AGXC_EINVAL, "qmv: N must be a multiple of 16 and K of 64");
  if (p.nb < 1 || p.nb > 8) return fail(AGXC_EINVAL, "qmv: 1 to 8 activation rows");
  p.G = p.K / 64;
  p.SC = plan.SC;
  p.GC = plan.GC;
  p.stages = plan.stages;
  if (p.bits == 4) return dispatch_nb<4>(ctx, p, plan, epi, s);
  if (p.bits == 8) return dispatch_nb<8>(ctx, p, plan, epi, s);
  return fail(AGXC_EINVAL, "qmv: 4- or 8-bit weights");
}

}  // namespace agxc
