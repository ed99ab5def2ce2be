// encoder.cu — the BERT sentence encoder (MiniLM) on the B200: the reference's complete-encoder graph
// (agxforge/g17/inferencegraph.py:208-289 import_graph, sentence pooling; its FP64 reference
// tools/g17inferencereference.py:18-99 graph_reference; the lowered stages tools/g17inferencelower.py:56-139),
// for batches of padded sequences.
//
// Rows are tokens, T = batch x seq (padded to a multiple of 128 for the GEMM tiles; the pad rows stay zero):
//   embed_ln     x = word[id] + position[s] + type[t] (fp16 parameters, fp32 sum); LayerNorm -> x32 fp32, x16 fp16
//   per layer    qkv32 = x16 Wqkv^T + b                          (tensor cores: fp16 operands, fp32 accumulate)
//                ctx16 = masked softmax(q k^T / sqrt(hw)) v        (fp32, one CTA per (head, sequence))
//                y32 = ctx16 Wo^T + b + x32;  x32, x16 = LayerNorm(y32)
//                u16 = fp16(gelu_erf(x16 W1^T + b1))
//                y32 = u16 W2^T + b2 + x32;   x32, x16 = LayerNorm(y32)
//   pool         mean of x32 over the valid rows (denominator >= 1e-9), / max(||.||, 1e-12)
// The fp16 roundings are the reference's half-transport points (g17inferencereference.py:50-53): the operands of
// every linear; everything else is fp32.
//
// The GEMM: one CTA per 128 token rows x BN (64 or 128) output features; warp 0 issues the TMA copies of both
// operands (64-column boxes, 128-byte swizzle = the UMMA K-major canonical layout), warp 1 allocates BN TMEM columns
// and issues tcgen05.mma.kind::f16 (M 128, N BN, K 16) four times per 64-column stage, committing each stage back to
// the producer; four epilogue warps read the fp32 accumulator with tcgen05.ld (warp w: TMEM lanes 32 (w % 4)..) and
// apply bias, GELU or the residual on the way out. Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

constexpr int kGM = 128;            // token rows per GEMM CTA (the MMA's M)
constexpr int kGThreads = 192;      // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue
enum { kEpiF32 = 0, kEpiGelu16 = 1, kEpiRes32 = 2, kEpiResLn = 3 };

struct HgemmParams {
  int M = 0, N = 0, K = 0, bn = 128, stages = 3;
  int epi = kEpiF32;
  const __half* bias = nullptr;     // [N]
  float* out32 = nullptr;           // [M][N] (F32, RES32)
  __half* out16 = nullptr;          // [M][N] (GELU16)
  const float* res32 = nullptr;     // [M][N] (RES32, RESLN; may alias out32)
  const __half* ln_g = nullptr;     // [N] LayerNorm gain and bias (RESLN: the tile is the whole row, bn == N)
  const __half* ln_b = nullptr;
  float eps = 0.f;
  unsigned* err = nullptr;
};

struct HgemmSmem {
  int bars, tmem_slot, bias, lng, lnb, stage0, stage_bytes, b_off, total;
};

__host__ __device__ inline HgemmSmem hgemm_layout(int bn, int stages) {
  HgemmSmem L;
  L.bars = 0;              // full[S], empty[S], acc_full, dead flag (S <= 8)
  L.tmem_slot = 256;
  L.bias = 512;            // bn fp32 (bn <= 512)
  L.lng = L.bias + 2048;   // LayerNorm gain, bias: bn fp32 each
  L.lnb = L.lng + 2048;
  L.stage0 = (L.lnb + 2048 + 1023) / 1024 * 1024;  // 1,024-aligned stages (the 128-byte swizzle's atom): A 128 x
                                                  // 128 B, then B bn x 128 B
  L.b_off = kGM * 128;
  L.stage_bytes = L.b_off + bn * 128;
  L.total = L.stage0 + stages * L.stage_bytes;
  return L;
}

// TMEM columns for a bn-wide fp32 accumulator (a power of two >= 32)
__host__ __device__ inline int tmem_cols(int bn) { return bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : bn <= 256 ? 256 : 512; }

__device__ __forceinline__ uint64_t desc_k128(uint32_t saddr) {
  // UMMA shared-memory descriptor, K-major, 128-byte swizzle: start >> 4 (bits 0-13), leading byte offset 16 B
  // (bits 16-29), stride byte offset 1,024 B between 8-row atoms (bits 32-45), version 1 (bit 46), SWIZZLE_128B = 2
  // (bits 61-63)
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

__device__ __forceinline__ void tma_rows(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

__global__ void __launch_bounds__(kGThreads, 1) hgemm_kernel(const HgemmParams p, const __grid_constant__ CUtensorMap ta,
                                                              const __grid_constant__ CUtensorMap tb) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const HgemmSmem L = hgemm_layout(p.bn, p.stages);
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  volatile int* dead = reinterpret_cast<volatile int*>(acc_full + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  float* sbias = reinterpret_cast<float*>(smem + L.bias);
  float* slng = reinterpret_cast<float*>(smem + L.lng);
  float* slnb = reinterpret_cast<float*>(smem + L.lnb);
  const int ncols = tmem_cols(p.bn);
  const int bsub = p.bn > 128 ? 128 : p.bn;  // B rows per TMA box and per MMA (N)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * p.bn, m0 = blockIdx.y * kGM;
  const int KT = p.K / 64;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *dead = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  for (int c = tid; c < p.bn; c += kGThreads) {
    sbias[c] = p.bias ? __half2float(p.bias[n0 + c]) : 0.f;
    if (p.epi == kEpiResLn) {
      slng[c] = __half2float(p.ln_g[c]);
      slnb[c] = __half2float(p.ln_b[c]);
    }
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&ta)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tb)) : "memory");
      const unsigned bytes = static_cast<unsigned>(L.stage_bytes);
      int issued = 0;
      for (int i = 0; i < KT && !*dead; ++i, ++issued) {
        const int s = i % S;
        if (i >= S && !mbar_wait_bounded(&empty[s], ((i / S) - 1) & 1, p.err)) {
          *dead = 1;
          break;
        }
        uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_rows(st, &ta, i * 64, m0, &full[s]);
        for (int j = 0; j < p.bn / bsub; ++j) tma_rows(st + L.b_off + j * bsub * 128, &tb, i * 64, n0 + j * bsub, &full[s]);
      }
      if (*dead) {  // no copy of this CTA may land after it leaves (bounded)
        for (int i = issued > S ? issued - S : 0; i < issued; ++i)
          mbar_wait_bounded(&full[i % S], (i / S) & 1, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(bsub >> 3) << 17) |
                             (static_cast<uint32_t>(kGM >> 4) << 24);  // fp32 accum, fp16 A/B, K-major, N, M
      for (int i = 0; i < KT; ++i) {
        const int s = i % S;
        if (*dead || !mbar_wait_bounded(&full[s], (i / S) & 1, p.err)) {
          *dead = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a0 = smem_u32(smem + L.stage0 + s * L.stage_bytes);
        const uint32_t b0 = a0 + L.b_off;
        for (int j = 0; j < p.bn / bsub; ++j) {  // N sub-blocks of bsub columns (TMEM columns j * bsub ..)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = desc_k128(a0 + 32 * k), bd = desc_k128(b0 + j * bsub * 128 + 32 * k);
            const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem + static_cast<uint32_t>(j * bsub)),
                "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&empty[s]))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(acc_full))
                   : "memory");
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = token rows; columns = output features
    const bool ok = __all_sync(0xffffffffu, !*dead && mbar_wait_bounded(acc_full, 0, p.err));
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (p.epi == kEpiResLn) {
      // the tile's residual rows into shared memory, coalesced (the stages are free: every MMA has completed), rows
      // padded to N + 4 floats so the row-per-thread reads below are conflict-free
      const int rs = p.N + 4;
      float* sres = reinterpret_cast<float*>(smem + L.stage0);
      if (ok) {
        const int n4 = p.N / 4;
        for (int i = tid - 64; i < kGM * n4; i += 128) {
          const int r = i / n4, c = (i % n4) * 4;
          *reinterpret_cast<float4*>(sres + r * rs + c) =
              __ldcg(reinterpret_cast<const float4*>(p.res32 + static_cast<size_t>(m0 + r) * p.N + c));
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
      if (ok) {
      // the whole row is in this thread's TMEM lane: x = acc + bias + residual, LayerNorm in three passes
      const int q4 = warp & 3;
      const int row = m0 + 32 * q4 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(32 * q4) << 16);
      const float* res = sres + (32 * q4 + lane) * rs;
      float mean = 0.f, den = 1.f;
      for (int pass = 0; pass < 3; ++pass) {
        float acc_s = 0.f;
        for (int c0 = 0; c0 < p.bn; c0 += 16) {
          uint32_t v[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15}, [%16];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
              : "r"(base + static_cast<uint32_t>(c0)));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          float x[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 rv = *reinterpret_cast<const float4*>(res + c0 + 4 * j);
            x[4 * j] = __uint_as_float(v[4 * j]) + sbias[c0 + 4 * j] + rv.x;
            x[4 * j + 1] = __uint_as_float(v[4 * j + 1]) + sbias[c0 + 4 * j + 1] + rv.y;
            x[4 * j + 2] = __uint_as_float(v[4 * j + 2]) + sbias[c0 + 4 * j + 2] + rv.z;
            x[4 * j + 3] = __uint_as_float(v[4 * j + 3]) + sbias[c0 + 4 * j + 3] + rv.w;
          }
          if (pass == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc_s += x[j];
          } else if (pass == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float dlt = x[j] - mean;
              acc_s = fmaf(dlt, dlt, acc_s);
            }
          } else {
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = (x[j] - mean) / den * slng[c0 + j] + slnb[c0 + j];
            float4* o32 = reinterpret_cast<float4*>(p.out32 + static_cast<size_t>(row) * p.N + c0);
#pragma unroll
            for (int j = 0; j < 4; ++j) o32[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
            uint32_t hv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const __half2 t2 = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
              hv[j] = *reinterpret_cast<const uint32_t*>(&t2);
            }
            uint4* o16 = reinterpret_cast<uint4*>(p.out16 + static_cast<size_t>(row) * p.N + c0);
            o16[0] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            o16[1] = make_uint4(hv[4], hv[5], hv[6], hv[7]);
          }
        }
        if (pass == 0) mean = acc_s / p.N;
        else if (pass == 1) den = sqrtf(acc_s / p.N + p.eps);
      }
      }
    } else if (ok) {
      const int q4 = warp & 3;
      const int row = m0 + 32 * q4 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(32 * q4) << 16);
      for (int c0 = 0; c0 < p.bn; c0 += 16) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(base + static_cast<uint32_t>(c0)));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float f[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(v[j]) + sbias[c0 + j];
        const size_t at = static_cast<size_t>(row) * p.N + n0 + c0;
        if (p.epi == kEpiGelu16) {
          uint32_t h[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const __half2 t = __floats2half2_rn(gelu_erf(f[2 * j]), gelu_erf(f[2 * j + 1]));
            h[j] = *reinterpret_cast<const uint32_t*>(&t);
          }
          uint4* dst = reinterpret_cast<uint4*>(p.out16 + at);
          dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
          dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
        } else {
          if (p.epi == kEpiRes32) {
            const float4* r = reinterpret_cast<const float4*>(p.res32 + at);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 rv = r[j];
              f[4 * j] += rv.x; f[4 * j + 1] += rv.y; f[4 * j + 2] += rv.z; f[4 * j + 3] += rv.w;
            }
          }
          float4* dst = reinterpret_cast<float4*>(p.out32 + at);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
        }
      }
    }
  }
  if (*dead && tid == 64) mbar_wait_bounded(acc_full, 0, nullptr, 100000000ull);  // the tensor core is done
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// ------------------------------------------------------------------------------------------------ row kernels
// LayerNorm of one row per warp (W = 32 PER): (x - mean) / sqrt(mean((x - mean)^2) + eps) * g + b, two passes over
// the row in registers. EMBED: x = word[id] + position[s] + type[t] first.
template <int PER, bool EMBED>
__global__ void ln_kernel(const float* __restrict__ x, const int32_t* __restrict__ ids, const int32_t* __restrict__ types,
                          const __half* __restrict__ word, const __half* __restrict__ pos,
                          const __half* __restrict__ tok_type, int seq, int vocab, int type_vocab,
                          const __half* __restrict__ g,
                          const __half* __restrict__ b, float eps, int rows, float* __restrict__ out32,
                          __half* __restrict__ out16, unsigned* err) {
  constexpr int W = 32 * PER;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[PER];
  if (EMBED) {
    // device inputs are not validated on the host: an id or type outside its table is reported, and clamped so no
    // read leaves the table
    int id = ids[row], t = types ? types[row] : 0;
    const int s = row % seq;
    if (id < 0 || id >= vocab || t < 0 || t >= type_vocab) {
      atomicOr(err, kErrBadToken);
      id = min(max(id, 0), vocab - 1);
      t = min(max(t, 0), type_vocab - 1);
    }
    const __half* w = word + static_cast<size_t>(id) * W;
    const __half* pp = pos + static_cast<size_t>(s) * W;
    const __half* tt = tok_type + static_cast<size_t>(t) * W;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = lane + 32 * i;
      v[i] = (__half2float(w[c]) + __half2float(pp[c])) + __half2float(tt[c]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) v[i] = x[static_cast<size_t>(row) * W + lane + 32 * i];
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) sum += v[i];
  const float mean = warp_sum(sum) / W;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    v[i] -= mean;
    ss = fmaf(v[i], v[i], ss);
  }
  const float den = sqrtf(warp_sum(ss) / W + eps);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = lane + 32 * i;
    const float y = v[i] / den * __half2float(g[c]) + __half2float(b[c]);
    out32[static_cast<size_t>(row) * W + c] = y;
    out16[static_cast<size_t>(row) * W + c] = __float2half_rn(y);
  }
}

// Masked softmax attention of one (head, sequence): K and V of the head in shared memory (fp32), one query row per
// thread, online softmax over the keys whose mask is 1 (scale 1/sqrt(HW) applied to the dot product).
template <int HW>
__global__ void attn_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ mask, int seq, int width,
                            float scale, __half* __restrict__ ctx) {
  extern __shared__ float sm[];
  float* ks = sm;                       // [seq][HW]
  float* vs = sm + seq * HW;            // [seq][HW]
  int* ms = reinterpret_cast<int*>(vs + seq * HW);
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int ld = 3 * width;
  const size_t r0 = static_cast<size_t>(b) * seq;
  for (int i = tid; i < seq * (HW / 4); i += blockDim.x) {
    const int s = i / (HW / 4), c = (i % (HW / 4)) * 4;
    const float* src = qkv + (r0 + s) * ld + h * HW + c;
    *reinterpret_cast<float4*>(ks + s * HW + c) = *reinterpret_cast<const float4*>(src + width);
    *reinterpret_cast<float4*>(vs + s * HW + c) = *reinterpret_cast<const float4*>(src + 2 * width);
  }
  for (int s = tid; s < seq; s += blockDim.x) ms[s] = mask[r0 + s];
  __syncthreads();
  for (int qi = tid; qi < seq; qi += blockDim.x) {
    float q[HW], acc[HW];
    const float* qs = qkv + (r0 + qi) * ld + h * HW;
#pragma unroll
    for (int c = 0; c < HW; c += 4) {
      const float4 t = *reinterpret_cast<const float4*>(qs + c);
      q[c] = t.x; q[c + 1] = t.y; q[c + 2] = t.z; q[c + 3] = t.w;
    }
#pragma unroll
    for (int c = 0; c < HW; ++c) acc[c] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < seq; ++j) {
      if (!ms[j]) continue;
      const float* kr = ks + j * HW;
      float d = 0.f;
#pragma unroll
      for (int c = 0; c < HW; ++c) d = fmaf(q[c], kr[c], d);
      const float sc = d * scale;
      if (sc > m) {
        const float corr = expf(m - sc);  // 0 on the first valid key (m = -inf)
        l *= corr;
#pragma unroll
        for (int c = 0; c < HW; ++c) acc[c] *= corr;
        m = sc;
      }
      const float pj = expf(sc - m);
      l += pj;
      const float* vr = vs + j * HW;
#pragma unroll
      for (int c = 0; c < HW; ++c) acc[c] = fmaf(pj, vr[c], acc[c]);
    }
    const float inv = l > 0.f ? 1.0f / l : 0.f;  // a sequence without a valid key (refused on the host path)
    __half* o = ctx + (r0 + qi) * width + h * HW;
#pragma unroll
    for (int c = 0; c < HW; c += 2) {
      const __half2 t = __floats2half2_rn(acc[c] * inv, acc[c + 1] * inv);
      *reinterpret_cast<__half2*>(o + c) = t;
    }
  }
}

// fp16 hi/lo split of a pair: hi = fp16(x), lo = fp16(x - hi) (exact residual up to fp16 rounding), so
// hi_a.hi_b + hi_a.lo_b + lo_a.hi_b on the tensor cores carries ~22 significant bits — fp32-class products.
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Masked softmax attention of one (head, sequence) on the tensor cores, seq <= 16 KT, head width 32: each warp takes
// 16-query tiles; S = Q K^T and O = P V by m16n8k16 MMAs with both operands split hi/lo (three MMAs per product), the
// whole score row in registers (no online rescaling), P kept in registers between the two products (the score
// accumulator of keys 16j..16j+15 is the A fragment of step j). Keys past seq or with mask 0 score -inf.
template <int KT>
__global__ void __launch_bounds__(128) attn_tc_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ mask,
                                                      int seq, int width, float scale, __half* __restrict__ ctx) {
  constexpr int HW = 32, SP = 16 * KT, LD = HW + 4;
  extern __shared__ float sm[];
  float* ks = sm;                 // [SP][LD] fp32, zero past seq
  float* vs = sm + SP * LD;
  int* ms = reinterpret_cast<int*>(vs + SP * LD);
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ld = 3 * width;
  const size_t r0 = static_cast<size_t>(b) * seq;
  for (int i = tid; i < SP * (HW / 4); i += 128) {
    const int s = i / (HW / 4), c = (i % (HW / 4)) * 4;
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
    if (s < seq) {
      const float* src = qkv + (r0 + s) * ld + h * HW + c;
      kv = *reinterpret_cast<const float4*>(src + width);
      vv = *reinterpret_cast<const float4*>(src + 2 * width);
    }
    *reinterpret_cast<float4*>(ks + s * LD + c) = kv;
    *reinterpret_cast<float4*>(vs + s * LD + c) = vv;
  }
  for (int s = tid; s < SP; s += 128) ms[s] = s < seq ? mask[r0 + s] != 0 : 0;
  __syncthreads();
  for (int mt = warp; mt < KT; mt += 4) {
    const int qa = mt * 16 + g, qb = qa + 8;  // this thread's two query rows
    // Q fragments (2 k-steps of 16 dims), split
    uint32_t qh[2][4], ql[2][4];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = 16 * k + 2 * t;
      float2 x0 = make_float2(0.f, 0.f), x1 = x0, x2 = x0, x3 = x0;
      if (qa < seq) {
        const float* q = qkv + (r0 + qa) * ld + h * HW;
        x0 = *reinterpret_cast<const float2*>(q + c);
        x2 = *reinterpret_cast<const float2*>(q + c + 8);
      }
      if (qb < seq) {
        const float* q = qkv + (r0 + qb) * ld + h * HW;
        x1 = *reinterpret_cast<const float2*>(q + c);
        x3 = *reinterpret_cast<const float2*>(q + c + 8);
      }
      split2(x0.x, x0.y, qh[k][0], ql[k][0]);
      split2(x1.x, x1.y, qh[k][1], ql[k][1]);
      split2(x2.x, x2.y, qh[k][2], ql[k][2]);
      split2(x3.x, x3.y, qh[k][3], ql[k][3]);
    }
    float sc[2 * KT][4];
#pragma unroll
    for (int nt = 0; nt < 2 * KT; ++nt) {
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
      const float* kr = ks + (nt * 8 + g) * LD;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = 16 * k + 2 * t;
        uint32_t bh0, bl0, bh1, bl1;
        split2(kr[c], kr[c + 1], bh0, bl0);
        split2(kr[c + 8], kr[c + 9], bh1, bl1);
        mma_16816(d0, d1, d2, d3, qh[k][0], qh[k][1], qh[k][2], qh[k][3], bh0, bh1);
        mma_16816(d0, d1, d2, d3, qh[k][0], qh[k][1], qh[k][2], qh[k][3], bl0, bl1);
        mma_16816(d0, d1, d2, d3, ql[k][0], ql[k][1], ql[k][2], ql[k][3], bh0, bh1);
      }
      const int k0 = nt * 8 + 2 * t;
      sc[nt][0] = ms[k0] ? d0 * scale : -INFINITY;
      sc[nt][1] = ms[k0 + 1] ? d1 * scale : -INFINITY;
      sc[nt][2] = ms[k0] ? d2 * scale : -INFINITY;
      sc[nt][3] = ms[k0 + 1] ? d3 * scale : -INFINITY;
    }
    float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2 * KT; ++nt) {
      m0 = fmaxf(m0, fmaxf(sc[nt][0], sc[nt][1]));
      m1 = fmaxf(m1, fmaxf(sc[nt][2], sc[nt][3]));
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if (m0 == -INFINITY) m0 = 0.f;  // no valid key (refused on the host path): all weights 0
    if (m1 == -INFINITY) m1 = 0.f;
    float l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2 * KT; ++nt) {
      sc[nt][0] = expf(sc[nt][0] - m0);
      sc[nt][1] = expf(sc[nt][1] - m0);
      sc[nt][2] = expf(sc[nt][2] - m1);
      sc[nt][3] = expf(sc[nt][3] - m1);
      l0 += sc[nt][0] + sc[nt][1];
      l1 += sc[nt][2] + sc[nt][3];
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    float acc[4][4];
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) acc[dt][0] = acc[dt][1] = acc[dt][2] = acc[dt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
      uint32_t ph[4], pl[4];
      split2(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
      split2(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
      split2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
      split2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
      const float* v0 = vs + (kk * 16 + 2 * t) * LD;
#pragma unroll
      for (int dt = 0; dt < 4; ++dt) {
        const int c = dt * 8 + g;
        uint32_t bh0, bl0, bh1, bl1;
        split2(v0[c], v0[LD + c], bh0, bl0);
        split2(v0[8 * LD + c], v0[9 * LD + c], bh1, bl1);
        mma_16816(acc[dt][0], acc[dt][1], acc[dt][2], acc[dt][3], ph[0], ph[1], ph[2], ph[3], bh0, bh1);
        mma_16816(acc[dt][0], acc[dt][1], acc[dt][2], acc[dt][3], ph[0], ph[1], ph[2], ph[3], bl0, bl1);
        mma_16816(acc[dt][0], acc[dt][1], acc[dt][2], acc[dt][3], pl[0], pl[1], pl[2], pl[3], bh0, bh1);
      }
    }
    const float i0 = l0 > 0.f ? 1.0f / l0 : 0.f, i1 = l1 > 0.f ? 1.0f / l1 : 0.f;
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int c = h * HW + dt * 8 + 2 * t;
      if (qa < seq)
        *reinterpret_cast<__half2*>(ctx + (r0 + qa) * width + c) = __floats2half2_rn(acc[dt][0] * i0, acc[dt][1] * i0);
      if (qb < seq)
        *reinterpret_cast<__half2*>(ctx + (r0 + qb) * width + c) = __floats2half2_rn(acc[dt][2] * i1, acc[dt][3] * i1);
    }
  }
}

// Masked mean over a sequence's valid rows, then L2 normalisation: one CTA per sequence, one thread per feature.
__global__ void pool_kernel(const float* __restrict__ x, const int32_t* __restrict__ mask, int seq, int width,
                            float* __restrict__ out) {
  __shared__ float red[32];
  const int b = blockIdx.x, c = threadIdx.x;
  float sum = 0.f, cnt = 0.f;
  for (int s = 0; s < seq; ++s) {
    const float w = mask[static_cast<size_t>(b) * seq + s] ? 1.f : 0.f;
    cnt += w;
    if (c < width) sum = fmaf(x[(static_cast<size_t>(b) * seq + s) * width + c], w, sum);
  }
  const float mean = sum / fmaxf(cnt, 1e-9f);
  const float sq = warp_sum(c < width ? mean * mean : 0.f);
  if ((c & 31) == 0) red[c >> 5] = sq;
  __syncthreads();
  if (c < 32) {
    float t = c < static_cast<int>(blockDim.x) / 32 ? red[c] : 0.f;
    t = warp_sum(t);
    if (c == 0) red[0] = t;
  }
  __syncthreads();
  if (c < width) out[static_cast<size_t>(b) * width + c] = mean / fmaxf(sqrtf(red[0]), 1e-12f);
}

int hgemm_allow(int optin) {
  cudaFuncAttributes fa;
  AGXC_CUDA(cudaFuncGetAttributes(&fa, hgemm_kernel));
  AGXC_CUDA(cudaFuncSetAttribute(hgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - static_cast<int>(fa.sharedSizeBytes)));
  return 0;
}

}  // namespace

// C [M][N] = A [M][K] fp16 x W [N][K]^T fp16 (+ bias, GELU / residual by `epi`): M % 128, N % 64, K % 64 == 0.
int launch_hgemm(const agxc_ctx* ctx, const __half* A, const __half* W, int M, int N, int K, const __half* bias,
                 int epi, float* out32, __half* out16, const float* res32, cudaStream_t s, const __half* ln_g,
                 const __half* ln_b, float eps) {
  if (M % kGM || N % 64 || K % 64 || M <= 0 || N <= 0 || K <= 0)
    return fail(AGXC_EINVAL, "hgemm: M multiple of 128, N and K multiples of 64");
  if (epi == kEpiResLn && (N % 128 || N > 384 || !ln_g || !ln_b))
    return fail(AGXC_EINVAL, "hgemm: the LayerNorm epilogue needs rows of 128, 256 or 384 features");
  HgemmParams p;
  p.M = M; p.N = N; p.K = K; p.epi = epi; p.bias = bias; p.out32 = out32; p.out16 = out16; p.res32 = res32;
  p.ln_g = ln_g; p.ln_b = ln_b; p.eps = eps;
  p.err = ctx->err_dev;
  if (epi == kEpiResLn) {
    p.bn = N;  // the whole row in one CTA's TMEM
    const int room = ctx->max_smem_optin - 1024 - hgemm_layout(p.bn, 0).total;
    p.stages = std::max(2, std::min({K / 64, 4, room / hgemm_layout(p.bn, 1).stage_bytes}));
  } else {
    // 128 output features per CTA when that alone gives a full wave, else 64 (more CTAs for the narrow outputs)
    p.bn = (N % 128 == 0 && (M / kGM) * (N / 128) >= ctx->num_sms) ? 128 : 64;
    p.stages = std::min(K / 64, p.bn == 128 ? 3 : 4);  // two CTAs per SM
  }
  int smem = hgemm_layout(p.bn, p.stages).total + 1024;
  if (epi == kEpiResLn)  // the residual tile (128 rows of N + 4 floats) reuses the stages
    smem = std::max(smem, hgemm_layout(p.bn, 0).total + kGM * (N + 4) * 4 + 1024);
  if (smem > ctx->max_smem_optin) return fail(AGXC_EINVAL, "hgemm: tile does not fit shared memory");
  CUtensorMap ta, tb;
  if (int rc = encode_rows_map(&ta, A, M, K, kGM)) return rc;
  if (int rc = encode_rows_map(&tb, W, N, K, p.bn > 128 ? 128 : p.bn)) return rc;
  hgemm_kernel<<<dim3(N / p.bn, M / kGM), kGThreads, smem, s>>>(p, ta, tb);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

int encoder_configure(const agxc_ctx* ctx) {
  if (int rc = hgemm_allow(ctx->max_smem_optin)) return rc;
  AGXC_CUDA(cudaFuncSetAttribute(attn_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ctx->max_smem_optin - 1024));
  AGXC_CUDA(cudaFuncSetAttribute(attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ctx->max_smem_optin - 1024));
  return 0;
}

}  // namespace agxc

// ------------------------------------------------------------------------------------------------ the encoder
struct agxc_encoder {
  agxc_ctx* ctx = nullptr;
  agxc_encoder_desc d{};
  int T = 0;                          // token rows (max_batch x max_seq, padded to a multiple of 128)
  __half *word = nullptr, *pos = nullptr, *ttype = nullptr, *eln_w = nullptr, *eln_b = nullptr;
  struct Layer {
    __half *wqkv, *bqkv, *wo, *bo, *ln1w, *ln1b, *w1, *b1, *w2, *b2, *ln2w, *ln2b;
  };
  std::vector<Layer> layers;
  float *x32 = nullptr, *y32 = nullptr, *qkv32 = nullptr, *out = nullptr;
  __half *x16 = nullptr, *ctx16 = nullptr, *u16 = nullptr;
  int32_t *ids = nullptr, *mask = nullptr, *types = nullptr;
  // the captured forward for (batch, seq, types given)
  cudaGraphExec_t exec = nullptr;
  int g_batch = 0, g_seq = 0, g_types = -1;
  int launches = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  void* flush = nullptr;              // 256 MB written between timed forwards (agxc_encoder_replay)
  int32_t* h_in = nullptr;            // pinned staging: ids, mask, types
  float* h_out = nullptr;
  std::vector<void*> allocs;
};

namespace agxc {
namespace {

int ealloc(agxc_encoder* e, void** p, size_t bytes) {
  cudaError_t r = cudaMalloc(p, std::max<size_t>(bytes, 256));
  if (r != cudaSuccess) return fail(AGXC_ENOMEM, std::string("encoder: cudaMalloc: ") + cudaGetErrorString(r));
  e->allocs.push_back(*p);
  return 0;
}
template <typename T>
int ealloc_t(agxc_encoder* e, T** p, size_t n) {
  void* v = nullptr;
  int rc = ealloc(e, &v, n * sizeof(T));
  *p = static_cast<T*>(v);
  return rc;
}

int launch_ln(const agxc_encoder* e, const float* x, bool embed, const int32_t* types, const __half* g,
              const __half* b, int rows, int seq, cudaStream_t s) {
  const int W = e->d.hidden, PER = W / 32;
  const dim3 grid((rows + 7) / 8), block(256);
#define AGXC_LN(P)                                                                                             \
  case P:                                                                                                      \
    if (embed)                                                                                                 \
      ln_kernel<P, true><<<grid, block, 0, s>>>(x, e->ids, types, e->word, e->pos, e->ttype, seq, e->d.vocab,   \
                                                e->d.type_vocab, g, b, e->d.eps, rows, e->x32, e->x16,         \
                                                e->ctx->err_dev);                                              \
    else                                                                                                       \
      ln_kernel<P, false><<<grid, block, 0, s>>>(x, e->ids, types, e->word, e->pos, e->ttype, seq, e->d.vocab,  \
                                                 e->d.type_vocab, g, b, e->d.eps, rows, e->x32, e->x16,        \
                                                 e->ctx->err_dev);                                             \
    break;
  switch (PER) {
    AGXC_LN(4)
    AGXC_LN(8)
    AGXC_LN(12)
    AGXC_LN(16)
    AGXC_LN(24)
    AGXC_LN(32)
    default: return fail(AGXC_EINVAL, "encoder: hidden 128, 256, 384, 512, 768 or 1024");
  }
#undef AGXC_LN
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

// The forward's launches; with `ev` (2 x 8 events) each stage kind's launches are bracketed and `kind_ms` summed.
int enqueue_forward(agxc_encoder* e, int B, int Sq, bool with_types, cudaStream_t s, cudaEvent_t* ev = nullptr,
                    float* kind_ms = nullptr, int32_t* kind_n = nullptr) {
  const agxc_encoder_desc& D = e->d;
  const int W = D.hidden, F = D.ffn, HW = W / D.heads;
  const int rows = B * Sq;
  const int M = (rows + kGM - 1) / kGM * kGM;
  const int32_t* types = with_types ? e->types : nullptr;
  int rc = 0, n = 0;
  auto timed = [&](int kind, auto&& fn) -> int {
    if (ev) AGXC_CUDA(cudaEventRecord(ev[0], s));
    if (int r = fn()) return r;
    ++n;
    if (ev) {
      AGXC_CUDA(cudaEventRecord(ev[1], s));
      AGXC_CUDA(cudaEventSynchronize(ev[1]));
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev[0], ev[1]);
      kind_ms[kind] += ms;
      kind_n[kind] += 1;
    }
    return 0;
  };
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HW)));
  const size_t attn_smem = static_cast<size_t>(Sq) * HW * 4 * 2 + static_cast<size_t>(Sq) * 4;
  if ((rc = timed(0, [&] { return launch_ln(e, nullptr, true, types, e->eln_w, e->eln_b, rows, Sq, s); }))) return rc;
  for (int l = 0; l < D.layers; ++l) {
    const agxc_encoder::Layer& L = e->layers[l];
    if ((rc = timed(1, [&] {
           return launch_hgemm(e->ctx, e->x16, L.wqkv, M, 3 * W, W, L.bqkv, kEpiF32, e->qkv32, nullptr, nullptr, s);
         })))
      return rc;
    if ((rc = timed(2, [&]() -> int {
           if (HW == 32 && Sq <= 128) {
             const int KT = (Sq + 15) / 16;
             const size_t sm = static_cast<size_t>(16 * KT) * 36 * 4 * 2 + static_cast<size_t>(16 * KT) * 4;
             const dim3 grid(D.heads, B);
             switch (KT) {
               case 1: attn_tc_kernel<1><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               case 2: attn_tc_kernel<2><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               case 3: attn_tc_kernel<3><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               case 4: attn_tc_kernel<4><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               case 5: attn_tc_kernel<5><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               case 6: attn_tc_kernel<6><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               case 7: attn_tc_kernel<7><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
               default: attn_tc_kernel<8><<<grid, 128, sm, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16); break;
             }
           } else if (HW == 32)
             attn_kernel<32><<<dim3(D.heads, B), 128, attn_smem, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16);
           else if (HW == 64)
             attn_kernel<64><<<dim3(D.heads, B), 128, attn_smem, s>>>(e->qkv32, e->mask, Sq, W, scale, e->ctx16);
           else
             return fail(AGXC_EINVAL, "encoder: head width 32 or 64");
           AGXC_CUDA(cudaGetLastError());
           return 0;
         })))
      return rc;
    // o_proj + bias + residual + LayerNorm in one kernel when the row fits one CTA's TMEM and the 128-row tiles
    // alone fill the SMs (measured at 32 tiles: 52 us against 19 + 12 us for the GEMM and the LayerNorm kernel apart)
    const bool ln_fused = W <= 384 && M / kGM >= e->ctx->num_sms;
    if (ln_fused) {
      if ((rc = timed(3, [&] {
             return launch_hgemm(e->ctx, e->ctx16, L.wo, M, W, W, L.bo, kEpiResLn, e->x32, e->x16, e->x32, s, L.ln1w,
                                 L.ln1b, D.eps);
           })))
        return rc;
    } else if ((rc = timed(3, [&] {
                  return launch_hgemm(e->ctx, e->ctx16, L.wo, M, W, W, L.bo, kEpiRes32, e->y32, nullptr, e->x32, s);
                })) ||
               (rc = timed(4, [&] { return launch_ln(e, e->y32, false, nullptr, L.ln1w, L.ln1b, M, Sq, s); }))) {
      return rc;
    }
    if ((rc = timed(5, [&] {
           return launch_hgemm(e->ctx, e->x16, L.w1, M, F, W, L.b1, kEpiGelu16, nullptr, e->u16, nullptr, s);
         })))
      return rc;
    if (ln_fused) {  // FFN down + bias + residual + LayerNorm in one kernel
      if ((rc = timed(6, [&] {
             return launch_hgemm(e->ctx, e->u16, L.w2, M, W, F, L.b2, kEpiResLn, e->x32, e->x16, e->x32, s, L.ln2w,
                                 L.ln2b, D.eps);
           })))
        return rc;
    } else if ((rc = timed(6, [&] {
                  return launch_hgemm(e->ctx, e->u16, L.w2, M, W, F, L.b2, kEpiRes32, e->y32, nullptr, e->x32, s);
                })) ||
               (rc = timed(4, [&] { return launch_ln(e, e->y32, false, nullptr, L.ln2w, L.ln2b, M, Sq, s); }))) {
      return rc;
    }
  }
  if ((rc = timed(7, [&]() -> int {
         pool_kernel<<<B, (W + 31) / 32 * 32, 0, s>>>(e->x32, e->mask, Sq, W, e->out);
         AGXC_CUDA(cudaGetLastError());
         return 0;
       })))
    return rc;
  e->launches = n;
  return 0;
}

int ensure_graph(agxc_encoder* e, int B, int Sq, bool with_types) {
  if (e->exec && e->g_batch == B && e->g_seq == Sq && e->g_types == static_cast<int>(with_types)) return 0;
  if (e->exec) cudaGraphExecDestroy(e->exec);
  e->exec = nullptr;
  cudaStream_t s = e->ctx->stream;
  AGXC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_forward(e, B, Sq, with_types, s);
  cudaGraph_t g = nullptr;
  cudaError_t ce = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return cuda_fail(ce, "encoder: cudaStreamEndCapture");
  cudaError_t ie = cudaGraphInstantiate(&e->exec, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return cuda_fail(ie, "encoder: cudaGraphInstantiate");
  e->g_batch = B;
  e->g_seq = Sq;
  e->g_types = with_types;
  return 0;
}

int check_shape(const agxc_encoder* e, int B, int Sq) {
  if (B < 1 || B > e->d.max_batch || Sq < 1 || Sq > e->d.max_seq || Sq > e->d.max_position)
    return fail(AGXC_EINVAL, "refused: batch 1..max_batch and seq 1..min(max_seq, max_position)");
  const int HW = e->d.hidden / e->d.heads;
  if (static_cast<size_t>(Sq) * (HW * 8 + 4) > static_cast<size_t>(e->ctx->max_smem_optin) - 1024)
    return fail(AGXC_EINVAL, "encoder: sequence too long for one attention CTA's shared memory");
  return 0;
}

}  // namespace
}  // namespace agxc

extern "C" {

int agxc_hgemm_dev(agxc_ctx* ctx, const uint16_t* A, const uint16_t* W, int M, int N, int K, const uint16_t* bias,
                   int epi, float* out32, uint16_t* out16, const float* res32, const uint16_t* ln_g,
                   const uint16_t* ln_b, float eps, void* stream) {
  using namespace agxc;
  if (!ctx || !A || !W) return fail(AGXC_EINVAL, "hgemm: null argument");
  if (epi < 0 || epi > 3 || (epi == 1 ? !out16 : !out32) || (epi >= 2 && !res32) || (epi == 3 && !out16))
    return fail(AGXC_EINVAL, "hgemm: epi 0 (out32), 1 (out16), 2 (out32 + res32), 3 (LayerNorm: out32, out16)");
  return launch_hgemm(ctx, reinterpret_cast<const __half*>(A), reinterpret_cast<const __half*>(W), M, N, K,
                      reinterpret_cast<const __half*>(bias), epi, out32, reinterpret_cast<__half*>(out16), res32,
                      stream ? static_cast<cudaStream_t>(stream) : ctx->stream,
                      reinterpret_cast<const __half*>(ln_g), reinterpret_cast<const __half*>(ln_b), eps);
}

int agxc_encoder_create(agxc_ctx* ctx, const agxc_encoder_desc* desc, agxc_encoder** out) {
  using namespace agxc;
  if (!ctx || !desc || !out) return fail(AGXC_EINVAL, "encoder_create: null argument");
  const agxc_encoder_desc& D = *desc;
  if (D.hidden % 128 || D.hidden > 1024 || D.heads < 1 || D.hidden % D.heads ||
      (D.hidden / D.heads != 32 && D.hidden / D.heads != 64))
    return fail(AGXC_EINVAL, "encoder: hidden a multiple of 128 up to 1024, head width 32 or 64");
  if (D.ffn % 64 || D.ffn <= 0 || D.layers < 1 || D.vocab < 1 || D.max_position < 1 || D.type_vocab < 1)
    return fail(AGXC_EINVAL, "encoder: ffn a multiple of 64, positive layers, vocab, positions, token types");
  if (D.max_batch < 1 || D.max_seq < 1 || !(D.eps > 0.f)) return fail(AGXC_EINVAL, "encoder: max_batch, max_seq, eps");
  if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(AGXC_ECUDA, "encoder: cudaSetDevice");
  agxc_encoder* e = new agxc_encoder();
  e->ctx = ctx;
  e->d = D;
  const int W = D.hidden, F = D.ffn;
  e->T = (D.max_batch * D.max_seq + kGM - 1) / kGM * kGM;
  int rc = 0;
  auto bail = [&](int code) {
    agxc_encoder_free(e);
    return code;
  };
  if ((rc = ealloc_t(e, &e->word, static_cast<size_t>(D.vocab) * W)) ||
      (rc = ealloc_t(e, &e->pos, static_cast<size_t>(D.max_position) * W)) ||
      (rc = ealloc_t(e, &e->ttype, static_cast<size_t>(D.type_vocab) * W)) || (rc = ealloc_t(e, &e->eln_w, W)) ||
      (rc = ealloc_t(e, &e->eln_b, W)))
    return bail(rc);
  e->layers.resize(D.layers);
  for (auto& L : e->layers) {
    if ((rc = ealloc_t(e, &L.wqkv, static_cast<size_t>(3) * W * W)) || (rc = ealloc_t(e, &L.bqkv, 3 * W)) ||
        (rc = ealloc_t(e, &L.wo, static_cast<size_t>(W) * W)) || (rc = ealloc_t(e, &L.bo, W)) ||
        (rc = ealloc_t(e, &L.ln1w, W)) || (rc = ealloc_t(e, &L.ln1b, W)) ||
        (rc = ealloc_t(e, &L.w1, static_cast<size_t>(F) * W)) || (rc = ealloc_t(e, &L.b1, F)) ||
        (rc = ealloc_t(e, &L.w2, static_cast<size_t>(W) * F)) || (rc = ealloc_t(e, &L.b2, W)) ||
        (rc = ealloc_t(e, &L.ln2w, W)) || (rc = ealloc_t(e, &L.ln2b, W)))
      return bail(rc);
  }
  const size_t T = e->T;
  if ((rc = ealloc_t(e, &e->x32, T * W)) || (rc = ealloc_t(e, &e->y32, T * W)) ||
      (rc = ealloc_t(e, &e->qkv32, T * 3 * W)) || (rc = ealloc_t(e, &e->x16, T * W)) ||
      (rc = ealloc_t(e, &e->ctx16, T * W)) || (rc = ealloc_t(e, &e->u16, T * F)) ||
      (rc = ealloc_t(e, &e->out, static_cast<size_t>(D.max_batch) * W)) || (rc = ealloc_t(e, &e->ids, T)) ||
      (rc = ealloc_t(e, &e->mask, T)) || (rc = ealloc_t(e, &e->types, T)))
    return bail(rc);
  // the activations start at zero, so the GEMMs' pad rows (past batch x seq) stay finite
  cudaStream_t s = ctx->stream;
  if (cudaMemsetAsync(e->x16, 0, T * W * 2, s) != cudaSuccess || cudaMemsetAsync(e->ctx16, 0, T * W * 2, s) != cudaSuccess ||
      cudaMemsetAsync(e->u16, 0, T * F * 2, s) != cudaSuccess || cudaMemsetAsync(e->x32, 0, T * W * 4, s) != cudaSuccess ||
      cudaMemsetAsync(e->y32, 0, T * W * 4, s) != cudaSuccess)
    return bail(fail(AGXC_ECUDA, "encoder: initial memset"));
  if (cudaMallocHost(&e->h_in, T * 3 * 4) != cudaSuccess ||
      cudaMallocHost(&e->h_out, static_cast<size_t>(D.max_batch) * W * 4) != cudaSuccess)
    return bail(fail(AGXC_ENOMEM, "encoder: pinned staging"));
  if (cudaEventCreate(&e->ev0) != cudaSuccess || cudaEventCreate(&e->ev1) != cudaSuccess)
    return bail(fail(AGXC_ECUDA, "encoder: events"));
  if (cudaStreamSynchronize(s) != cudaSuccess) return bail(fail(AGXC_ECUDA, "encoder: setup sync"));
  *out = e;
  return 0;
}

void agxc_encoder_free(agxc_encoder* e) {
  if (!e) return;
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  if (e->h_in) cudaFreeHost(e->h_in);
  if (e->h_out) cudaFreeHost(e->h_out);
  for (void* p : e->allocs) cudaFree(p);
  delete e;
}

int agxc_encoder_set_param(agxc_encoder* e, int layer, int which, const void* data, size_t bytes, int on_device) {
  using namespace agxc;
  if (!e || !data) return fail(AGXC_EINVAL, "encoder_set_param: null argument");
  const agxc_encoder_desc& D = e->d;
  const size_t W = D.hidden, F = D.ffn;
  __half* dst = nullptr;
  size_t n = 0;
  if (which >= AGXC_ENC_Q_W && (layer < 0 || layer >= D.layers)) return fail(AGXC_EINVAL, "encoder_set_param: layer");
  agxc_encoder::Layer* L = which >= AGXC_ENC_Q_W ? &e->layers[layer] : nullptr;
  switch (which) {
    case AGXC_ENC_WORD: dst = e->word; n = D.vocab * W; break;
    case AGXC_ENC_POSITION: dst = e->pos; n = D.max_position * W; break;
    case AGXC_ENC_TOKEN_TYPE: dst = e->ttype; n = D.type_vocab * W; break;
    case AGXC_ENC_EMB_LN_W: dst = e->eln_w; n = W; break;
    case AGXC_ENC_EMB_LN_B: dst = e->eln_b; n = W; break;
    case AGXC_ENC_Q_W: dst = L->wqkv; n = W * W; break;            // rows [0, W) of the fused qkv weights
    case AGXC_ENC_K_W: dst = L->wqkv + W * W; n = W * W; break;    // rows [W, 2W)
    case AGXC_ENC_V_W: dst = L->wqkv + 2 * W * W; n = W * W; break;
    case AGXC_ENC_Q_B: dst = L->bqkv; n = W; break;
    case AGXC_ENC_K_B: dst = L->bqkv + W; n = W; break;
    case AGXC_ENC_V_B: dst = L->bqkv + 2 * W; n = W; break;
    case AGXC_ENC_O_W: dst = L->wo; n = W * W; break;
    case AGXC_ENC_O_B: dst = L->bo; n = W; break;
    case AGXC_ENC_LN1_W: dst = L->ln1w; n = W; break;
    case AGXC_ENC_LN1_B: dst = L->ln1b; n = W; break;
    case AGXC_ENC_FFN1_W: dst = L->w1; n = F * W; break;
    case AGXC_ENC_FFN1_B: dst = L->b1; n = F; break;
    case AGXC_ENC_FFN2_W: dst = L->w2; n = W * F; break;
    case AGXC_ENC_FFN2_B: dst = L->b2; n = W; break;
    case AGXC_ENC_LN2_W: dst = L->ln2w; n = W; break;
    case AGXC_ENC_LN2_B: dst = L->ln2b; n = W; break;
    default: return fail(AGXC_EINVAL, "encoder_set_param: unknown parameter");
  }
  if (bytes != n * 2) return fail(AGXC_EINVAL, "encoder_set_param: expected " + std::to_string(n * 2) + " bytes");
  AGXC_CUDA(cudaMemcpy(dst, data, bytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  return 0;
}

int agxc_encoder_forward(agxc_encoder* e, const int32_t* token_ids, const int32_t* attention_mask,
                         const int32_t* token_type_ids, int batch, int seq, float* out, int on_device,
                         agxc_timing* t) {
  using namespace agxc;
  if (!e || !token_ids || !attention_mask || !out) return fail(AGXC_EINVAL, "encoder_forward: null argument");
  if (int rc = check_shape(e, batch, seq)) return rc;
  const agxc_encoder_desc& D = e->d;
  const size_t n = static_cast<size_t>(batch) * seq;
  cudaStream_t s = e->ctx->stream;
  const bool with_types = token_type_ids != nullptr;
  const auto h0 = std::chrono::steady_clock::now();
  if (!on_device) {  // validate on the host (the reference's refusals), then one pinned staging copy in
    for (int b = 0; b < batch; ++b) {
      int any = 0;
      for (int q = 0; q < seq; ++q) {
        const size_t i = static_cast<size_t>(b) * seq + q;
        if (token_ids[i] < 0 || token_ids[i] >= D.vocab) return fail(AGXC_EINVAL, "refused: token id outside vocab");
        if (with_types && (token_type_ids[i] < 0 || token_type_ids[i] >= D.type_vocab))
          return fail(AGXC_EINVAL, "refused: token type outside type vocab");
        if (attention_mask[i] != 0 && attention_mask[i] != 1) return fail(AGXC_EINVAL, "refused: mask values 0/1");
        any |= attention_mask[i];
      }
      if (!any) return fail(AGXC_EINVAL, "refused: a sequence without a valid token");
    }
    std::memcpy(e->h_in, token_ids, n * 4);
    std::memcpy(e->h_in + n, attention_mask, n * 4);
    if (with_types) std::memcpy(e->h_in + 2 * n, token_type_ids, n * 4);
  }
  AGXC_CUDA(cudaEventRecord(e->ev0, s));
  if (!on_device) {
    AGXC_CUDA(cudaMemcpyAsync(e->ids, e->h_in, n * 4, cudaMemcpyHostToDevice, s));
    AGXC_CUDA(cudaMemcpyAsync(e->mask, e->h_in + n, n * 4, cudaMemcpyHostToDevice, s));
    if (with_types) AGXC_CUDA(cudaMemcpyAsync(e->types, e->h_in + 2 * n, n * 4, cudaMemcpyHostToDevice, s));
  } else {
    AGXC_CUDA(cudaMemcpyAsync(e->ids, token_ids, n * 4, cudaMemcpyDeviceToDevice, s));
    AGXC_CUDA(cudaMemcpyAsync(e->mask, attention_mask, n * 4, cudaMemcpyDeviceToDevice, s));
    if (with_types) AGXC_CUDA(cudaMemcpyAsync(e->types, token_type_ids, n * 4, cudaMemcpyDeviceToDevice, s));
  }
  if (int rc = ensure_graph(e, batch, seq, with_types)) return rc;
  AGXC_CUDA(cudaGraphLaunch(e->exec, s));
  const size_t ob = static_cast<size_t>(batch) * D.hidden * 4;
  AGXC_CUDA(cudaMemcpyAsync(on_device ? out : e->h_out, e->out, ob,
                            on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s));
  AGXC_CUDA(cudaEventRecord(e->ev1, s));
  if (!on_device) {
    AGXC_CUDA(cudaEventSynchronize(e->ev1));
    std::memcpy(out, e->h_out, ob);
    uint32_t err = 0;
    AGXC_CUDA(cudaMemcpy(&err, e->ctx->err_dev, 4, cudaMemcpyDeviceToHost));
    if (err) {
      const uint32_t zero = 0;
      cudaMemcpy(e->ctx->err_dev, &zero, 4, cudaMemcpyHostToDevice);
      return fail(AGXC_ETIMEOUT, "encoder: a bounded device wait gave up");
    }
  }
  if (t) {
    if (on_device) AGXC_CUDA(cudaEventSynchronize(e->ev1));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e->ev0, e->ev1);
    t->gpu_ms = ms;
    t->host_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - h0).count();
    t->launches_per_step = e->launches;
  }
  return 0;
}

int agxc_encoder_replay(agxc_encoder* e, int reps, int flush_l2, agxc_timing* t) {
  using namespace agxc;
  if (!e || !t || reps < 1) return fail(AGXC_EINVAL, "encoder_replay: bad argument");
  if (!e->exec) return fail(AGXC_EINVAL, "encoder_replay: no forward has run yet");
  cudaStream_t s = e->ctx->stream;
  constexpr size_t kFlush = size_t(256) << 20;
  if (flush_l2 && !e->flush) {
    void* f = nullptr;
    if (int rc = ealloc(e, &f, kFlush)) return rc;
    e->flush = f;
  }
  const auto h0 = std::chrono::steady_clock::now();
  float total = 0.f;
  if (!flush_l2) {
    AGXC_CUDA(cudaEventRecord(e->ev0, s));
    for (int i = 0; i < reps; ++i) AGXC_CUDA(cudaGraphLaunch(e->exec, s));
    AGXC_CUDA(cudaEventRecord(e->ev1, s));
    AGXC_CUDA(cudaEventSynchronize(e->ev1));
    cudaEventElapsedTime(&total, e->ev0, e->ev1);
  } else {
    for (int i = 0; i < reps; ++i) {
      AGXC_CUDA(cudaMemsetAsync(e->flush, i & 0xFF, kFlush, s));
      AGXC_CUDA(cudaEventRecord(e->ev0, s));
      AGXC_CUDA(cudaGraphLaunch(e->exec, s));
      AGXC_CUDA(cudaEventRecord(e->ev1, s));
      AGXC_CUDA(cudaEventSynchronize(e->ev1));
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e->ev0, e->ev1);
      total += ms;
    }
  }
  t->gpu_ms = total;
  t->host_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - h0).count();
  t->launches_per_step = e->launches;
  return 0;
}

int agxc_encoder_profile(agxc_encoder* e, int batch, int seq, int reps, float* ms, int32_t* launches) {
  using namespace agxc;
  if (!e || !ms || !launches || reps < 1) return fail(AGXC_EINVAL, "encoder_profile: bad argument");
  if (int rc = check_shape(e, batch, seq)) return rc;
  for (int k = 0; k < 8; ++k) { ms[k] = 0.f; launches[k] = 0; }
  cudaEvent_t ev[2] = {e->ev0, e->ev1};
  for (int r = 0; r < reps; ++r)
    if (int rc = enqueue_forward(e, batch, seq, false, e->ctx->stream, ev, ms, launches)) return rc;
  return 0;
}

}  // extern "C"
