// batched.cu — the per-row steps of the batched decode step (B >= 32 sequences), between the tensor-core GEMMs of
// qmm.cu: the projections produce fp32 rows y [B][n] in the packs' physical row order, and these kernels finish
// them exactly as the single-sequence GEMV epilogues do (gemv_impl.cuh), so both paths share every rounding point:
//   rope_append   bias, rotate-half RoPE at each row's position, q scale (fp16 q), K and V rows into the cache of the
//                 row's sequence (the row itself, or one sequence for every row of a prefill chunk)
//                 (the qkv pack's tile rows r and r + 8 are a RoPE pair; attention.py:1309-1323)
//   residual_add16     h = y + x16 (fp32)                      (with_residual add16, qmv.py:112-120)
//   residual_add32_16  x16 = fp16(y + h)                       (with_residual add32_to16, qmv.py:825-833)
//   swiglu        act = fp16(silu(gate) * up) over the interleaved gate/up row tiles (qmv.py:214-226)
//   argmax_gen    per sequence: the first maximum of the logits, then the generation step (argmax.py:141-215,
//                 assemble.py:918-930): forced token, else the logged one, else the argmax; log, q0 + 1, x16 = emb[tok]
//   argmax_part / gen_from_pairs   the same split around an all-gather when the vocabulary is sliced over ranks
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// row b, column n of a GEMM's output (its K ranges added in order; with several ranges their loads are issued 8 at a
// time and then added one after the other)
__device__ __forceinline__ float yval(const YRows& y, int b, int n) {
  const float* src = y.y + static_cast<size_t>(b) * y.ld + n;
  float v = src[0];
  if (y.ks == 1) return v;
  for (int q0 = 1; q0 < y.ks; q0 += 8) {
    float t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = q0 + j < y.ks ? src[(q0 + j) * y.slice] : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (q0 + j < y.ks) v += t[j];
  }
  return v;
}

__global__ void rope_append_kernel(const YRows y, int rows, const __half* __restrict__ bias,
                                   const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                   const uint32_t* __restrict__ q0, int H, int KVH, int hd, int cap, float qscale,
                                   __half* __restrict__ q16, __half* __restrict__ kc, __half* __restrict__ vc, int B,
                                   int seq, int pdl) {
  pdl_enter(pdl);
  const int pairs = rows / 2;
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (t >= static_cast<long long>(B) * pairs) return;
  const int b = static_cast<int>(t / pairs), pr = static_cast<int>(t % pairs);
  const int half = hd / 2;
  const int tile = pr / 8, r = pr % 8;
  const int prow0 = tile * 16;
  const int head = prow0 / hd, tt = (prow0 % hd) / 16;
  const int i1 = 8 * tt + r, i2 = half + 8 * tt + r;
  float y1 = yval(y, b, prow0 + r), y2 = yval(y, b, prow0 + r + 8);
  if (bias) {
    y1 += __half2float(bias[head * hd + i1]);
    y2 += __half2float(bias[head * hd + i2]);
  }
  int pos = static_cast<int>(q0[b]);
  if (pos > cap - 1) pos = cap - 1;
  const int sq = seq >= 0 ? seq : b;  // the cache sequence of this row (prefill: every row of one sequence)
  if (head < H + KVH) {
    const float c = cos_t[static_cast<size_t>(pos) * half + i1];
    const float s = sin_t[static_cast<size_t>(pos) * half + i1];
    const float o1 = y1 * c - y2 * s, o2 = y2 * c + y1 * s;
    if (head < H) {
      __half* q = q16 + (static_cast<size_t>(b) * H + head) * hd;
      q[i1] = __float2half_rn(o1 * qscale);
      q[i2] = __float2half_rn(o2 * qscale);
    } else {
      __half* k = kc + ((static_cast<size_t>(sq) * KVH + (head - H)) * cap + pos) * hd;
      k[i1] = __float2half_rn(o1);
      k[i2] = __float2half_rn(o2);
    }
  } else {
    __half* v = vc + ((static_cast<size_t>(sq) * KVH + (head - H - KVH)) * cap + pos) * hd;
    v[i1] = __float2half_rn(y1);
    v[i2] = __float2half_rn(y2);
  }
}

// The same with QK-norm (Qwen3, agxforge/kernels/attention.py:256-265): one CTA per (row, head) and one thread per
// RoPE pair; q and k heads are RMS-normed over head_dim with the layer's shared gains (qkg[0..hd) for q,
// qkg[hd..2hd) for k) in fp32, (x r) g, before the rotation; v heads are stored as they are.
__global__ void rope_append_qknorm_kernel(const YRows y, const __half* __restrict__ bias,
                                          const __half* __restrict__ qkg, float eps, const float* __restrict__ cos_t,
                                          const float* __restrict__ sin_t, const uint32_t* __restrict__ q0, int H,
                                          int KVH, int hd, int cap, float qscale, __half* __restrict__ q16,
                                          __half* __restrict__ kc, __half* __restrict__ vc, int seq) {
  const int head = blockIdx.x, b = blockIdx.y, pr = threadIdx.x;  // pr < hd / 2
  const int half = hd / 2;
  const int tt = pr / 8, r = pr % 8;
  const int prow0 = head * hd + tt * 16;
  const int i1 = 8 * tt + r, i2 = half + 8 * tt + r;
  float y1 = yval(y, b, prow0 + r), y2 = yval(y, b, prow0 + r + 8);
  if (bias) {
    y1 += __half2float(bias[head * hd + i1]);
    y2 += __half2float(bias[head * hd + i2]);
  }
  int pos = static_cast<int>(q0[b]);
  if (pos > cap - 1) pos = cap - 1;
  const int sq = seq >= 0 ? seq : b;
  if (head >= H + KVH) {
    __half* v = vc + ((static_cast<size_t>(sq) * KVH + (head - H - KVH)) * cap + pos) * hd;
    v[i1] = __float2half_rn(y1);
    v[i2] = __float2half_rn(y2);
    return;  // the whole CTA (one head) leaves together
  }
  __shared__ float red[4];
  float ss = warp_sum(fmaf(y1, y1, y2 * y2));
  if ((pr & 31) == 0) red[pr >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < half / 32; ++w) tot += red[w];
  const float rn = rsqrtf(tot / static_cast<float>(hd) + eps);
  const __half* g = qkg + (head < H ? 0 : hd);
  y1 = (y1 * rn) * __half2float(g[i1]);
  y2 = (y2 * rn) * __half2float(g[i2]);
  const float c = cos_t[static_cast<size_t>(pos) * half + i1];
  const float s = sin_t[static_cast<size_t>(pos) * half + i1];
  const float o1 = y1 * c - y2 * s, o2 = y2 * c + y1 * s;
  if (head < H) {
    __half* q = q16 + (static_cast<size_t>(b) * H + head) * hd;
    q[i1] = __float2half_rn(o1 * qscale);
    q[i2] = __float2half_rn(o2 * qscale);
  } else {
    __half* k = kc + ((static_cast<size_t>(sq) * KVH + (head - H)) * cap + pos) * hd;
    k[i1] = __float2half_rn(o1);
    k[i2] = __float2half_rn(o2);
  }
}

// Per row of a GEMM output (its K ranges added in order): the first maximum over V columns, and the row itself to
// `logits` when given (the speculative verify step's rows).
__global__ void __launch_bounds__(1024) rows_argmax_kernel(const YRows y, int V, float* logits, int32_t* amax) {
  const int b = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int n = threadIdx.x; n < V; n += blockDim.x) {
    const float v = yval(y, b, n);
    if (logits) logits[static_cast<size_t>(b) * V + n] = v;
    if (v > bv || (bi == 0x7fffffff)) { bv = v; bi = n; }
  }
  for (int m = 16; m >= 1; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    bv = lane < static_cast<int>(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < static_cast<int>(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) amax[b] = bi;
  }
}

__global__ void residual16_kernel(const YRows y, const __half* __restrict__ x16, float* h, int d, int B, int pdl) {
  pdl_enter(pdl);
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (t >= static_cast<long long>(B) * d) return;
  const int b = static_cast<int>(t / d), i = static_cast<int>(t % d);
  h[t] = yval(y, b, i) + __half2float(x16[t]);
}

__global__ void residual32_kernel(const YRows y, const float* __restrict__ h, __half* x16, int d, int B, int pdl) {
  pdl_enter(pdl);
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (t >= static_cast<long long>(B) * d) return;
  const int b = static_cast<int>(t / d), i = static_cast<int>(t % d);
  x16[t] = __float2half_rn(yval(y, b, i) + h[t]);
}

__global__ void swiglu_kernel(const YRows y, __half* __restrict__ act, int F, int B, int pdl) {
  pdl_enter(pdl);
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (t >= static_cast<long long>(B) * F) return;
  const int b = static_cast<int>(t / F), j = static_cast<int>(t % F);
  const int p = j / 16, r = j % 16;  // gate row tile 2p, up row tile 2p + 1 of the interleaved pack
  const float g = yval(y, b, 32 * p + r), u = yval(y, b, 32 * p + 16 + r);
  act[t] = __float2half_rn(silu(g) * u);
}

constexpr int kArgThreads = 512;

// The first maximum of one sequence's logits over the block: (value, index + v0) in every thread's registers.
__device__ __forceinline__ void block_first_max(const float* __restrict__ lb, int V, int v0, float* sv, int* si,
                                                float& bv, int& bi) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (int i = tid; i < V; i += kArgThreads) {
    const float v = lb[i];
    if (v > bv) { bv = v; bi = i; }  // ascending per thread: the first of equal values stays
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  bv = sv[0];
  bi = si[0];
  for (int w = 1; w < kArgThreads / 32; ++w)
    if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
  if (bi != 0x7fffffff) bi += v0;
}

// The generation step of sequence b given its argmax `best` (thread 0), then x16[b] = embed[token] (all threads).
__device__ void gen_step(int b, int best, int V, const __half* __restrict__ embed, int d, uint32_t* q0, uint32_t* log,
                         int cap, int32_t* tok_out, uint32_t* force_next, __half* x16, unsigned* err, int* s_tok) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    const uint32_t pos = q0[b];
    const uint32_t p1 = pos + 1;
    uint32_t f = force_next[b];
    force_next[b] = kTokenUnset;
    if (f == kTokenUnset && p1 < static_cast<uint32_t>(cap)) f = log[static_cast<size_t>(b) * cap + p1];
    uint32_t tk = f != kTokenUnset ? f : static_cast<uint32_t>(best);
    if (tk >= static_cast<uint32_t>(V)) {
      atomicOr(err, kErrBadToken);
      tk = 0;
    }
    if (p1 < static_cast<uint32_t>(cap)) log[static_cast<size_t>(b) * cap + p1] = tk;
    q0[b] = p1 < static_cast<uint32_t>(cap) ? p1 : static_cast<uint32_t>(cap - 1);
    tok_out[b] = static_cast<int32_t>(tk);
    *s_tok = static_cast<int>(tk);
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(embed + static_cast<size_t>(*s_tok) * d);
  uint4* dst = reinterpret_cast<uint4*>(x16 + static_cast<size_t>(b) * d);
  for (int i = tid; i < d / 8; i += blockDim.x) dst[i] = src[i];
}

__global__ void __launch_bounds__(kArgThreads) argmax_gen_kernel(
    const float* __restrict__ logits, int V, const __half* __restrict__ embed, int d, uint32_t* q0, uint32_t* log,
    int cap, int32_t* tok_out, uint32_t* force_next, __half* x16, unsigned* err, int pdl) {
  pdl_enter(pdl);
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  __shared__ int s_tok;
  const int b = blockIdx.x;
  float bv;
  int bi;
  block_first_max(logits + static_cast<size_t>(b) * V, V, 0, sv, si, bv, bi);
  gen_step(b, bi, V, embed, d, q0, log, cap, tok_out, force_next, x16, err, &s_tok);
}

// Tensor parallel head, step 1: the first maximum of this rank's vocabulary slice [v0, v0 + V) of sequence b as a
// (value bits, global index) pair.
__global__ void __launch_bounds__(kArgThreads) argmax_part_kernel(const float* __restrict__ logits, int V, int v0,
                                                                 uint32_t* pairs) {
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  const int b = blockIdx.x;
  float bv;
  int bi;
  block_first_max(logits + static_cast<size_t>(b) * V, V, v0, sv, si, bv, bi);
  if (threadIdx.x == 0) {
    pairs[2 * b] = __float_as_uint(bv);
    pairs[2 * b + 1] = static_cast<uint32_t>(bi);
  }
}

// Step 2, after the all-gather of every rank's pairs ([ranks][B][2], slices in ascending vocabulary order): the
// largest value, the lowest index among equal values (= the first maximum over the whole vocabulary), then the
// generation step, identically on every rank.
__global__ void gen_from_pairs_kernel(const uint32_t* __restrict__ pairs, int ranks, int B, int V,
                                      const __half* __restrict__ embed, int d, uint32_t* q0, uint32_t* log, int cap,
                                      int32_t* tok_out, uint32_t* force_next, __half* x16, unsigned* err,
                                      unsigned* epoch) {
  if (epoch && blockIdx.x == 0 && threadIdx.x == 0) *epoch += 1;  // the step's last kernel: the next step begins
  __shared__ int s_tok;
  const int b = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int r = 0; r < ranks; ++r) {
    const float v = __uint_as_float(pairs[(static_cast<size_t>(r) * B + b) * 2]);
    const int i = static_cast<int>(pairs[(static_cast<size_t>(r) * B + b) * 2 + 1]);
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
  }
  gen_step(b, bi, V, embed, d, q0, log, cap, tok_out, force_next, x16, err, &s_tok);
}

// A bounded spin until *flag reaches target (the signed difference handles wrap-around); false after limit_ns of
// the global timer (2 s unless the model's device wait limit says otherwise).
__device__ bool wait_flag_sys(const unsigned* flag, unsigned target, unsigned* err, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (unsigned it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (static_cast<int>(v - target) >= 0) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > limit_ns) {
      atomicOr(err, kErrMbarTimeout);
      return false;
    }
  }
}

constexpr int kMaxRanks = 8;

// Tensor parallel, after the GEMM's pushes. Two-shot (one cooperative grid: its blocks wait on one another's gather
// signals, so all are resident): this rank's rows [rank d / ranks, ...) = the sum over ranks in rank order plus the
// residual, stored into every rank's residual stream. One-shot: every row, reduced here and stored here only. Either
// way the sums are bit-identical on every rank: the same slots added in the same order.
__global__ void tp_reduce_kernel(const float* __restrict__ recv, int ranks, int rank, const unsigned* flag,
                                 const unsigned* epoch, int uses_per_step, int use_in_step, int tiles_per_rank,
                                 const __half* __restrict__ res16, const float* __restrict__ res32, TpGather gather,
                                 int d, int B, unsigned* err, int two_shot, uint64_t wait_ns) {
  __shared__ int s_ok;
  const unsigned use = *epoch * static_cast<unsigned>(uses_per_step) + static_cast<unsigned>(use_in_step);
  const unsigned arrivals = static_cast<unsigned>(ranks * tiles_per_rank * (two_shot ? 1 : ranks));
  if (threadIdx.x == 0) s_ok = wait_flag_sys(flag, (use + 1u) * arrivals, err, wait_ns);
  __syncthreads();
  const int w = two_shot ? d / ranks : d, n0 = two_shot ? rank * w : 0;  // the rows reduced here
  const int rlo = two_shot ? 0 : rank, rhi = two_shot ? ranks : rank + 1;  // the ranks whose streams are written
  const size_t slot = static_cast<size_t>(B) * d;
  const int per_row = w / 4;
  // a wait that gave up leaves every residual stream as it was (no partial sum reaches a peer); the gather signal
  // below still goes out so the other ranks' bounded waits end
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; s_ok && i < B * per_row; i += gridDim.x * blockDim.x) {
    const int b = i / per_row;
    const size_t at = static_cast<size_t>(b) * d + n0 + (i % per_row) * 4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s_ok) {
      for (int r = 0; r < ranks; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(recv + r * slot + at));
        a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      }
    }
    if (res16) {  // h = sum + x16 (o_proj, add16)
      const __half2 x01 = *reinterpret_cast<const __half2*>(res16 + at);
      const __half2 x23 = *reinterpret_cast<const __half2*>(res16 + at + 2);
      const float4 o = make_float4(a.x + __low2float(x01), a.y + __high2float(x01), a.z + __low2float(x23),
                                   a.w + __high2float(x23));
      for (int r = rlo; r < rhi; ++r) *reinterpret_cast<float4*>(gather.out32[r] + at) = o;
    } else {      // x16 = fp16(sum + h) (down, add32_to16)
      const float4 h = *reinterpret_cast<const float4*>(res32 + at);
      const __half2 o01 = __floats2half2_rn(a.x + h.x, a.y + h.y), o23 = __floats2half2_rn(a.z + h.z, a.w + h.w);
      for (int r = rlo; r < rhi; ++r) {
        *reinterpret_cast<__half2*>(gather.out16[r] + at) = o01;
        *reinterpret_cast<__half2*>(gather.out16[r] + at + 2) = o23;
      }
    }
  }
  if (!two_shot) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int r = 0; r < ranks; ++r)
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(gather.gflag[r]) : "memory");
    // every rank's rows are here once every block of every rank has signalled this use
    wait_flag_sys(gather.gflag[rank], (use + 1u) * static_cast<unsigned>(ranks) * gridDim.x, err, wait_ns);
  }
  __syncthreads();
}

inline unsigned blocks_for(long long n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

}  // namespace

int launch_rows_argmax(const YRows& y, int V, int rows, float* logits, int32_t* amax, cudaStream_t s) {
  rows_argmax_kernel<<<rows, 1024, 0, s>>>(y, V, logits, amax);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

int launch_rope_append(const YRows& y, int rows, const __half* bias, const float* cos_t, const float* sin_t,
                       const uint32_t* q0, int H, int KVH, int hd, int cap, float qscale, __half* q16, __half* kc,
                       __half* vc, int B, cudaStream_t s, int seq, const __half* qkg, float qk_eps, int pdl) {
  if (qkg) {
    rope_append_qknorm_kernel<<<dim3(H + 2 * KVH, B), hd / 2, 0, s>>>(y, bias, qkg, qk_eps, cos_t, sin_t, q0, H, KVH,
                                                                      hd, cap, qscale, q16, kc, vc, seq);
    AGXC_CUDA(cudaGetLastError());
    return 0;
  }
  return launch_ex(rope_append_kernel, dim3(blocks_for(static_cast<long long>(B) * rows / 2, 256)), dim3(256), 0, s, pdl,
                   y, rows, bias, cos_t, sin_t, q0, H, KVH, hd, cap, qscale, q16, kc, vc, B, seq, pdl);
}

int launch_residual16(const YRows& y, const __half* x16, float* h, int d, int B, cudaStream_t s, int pdl) {
  return launch_ex(residual16_kernel, dim3(blocks_for(static_cast<long long>(B) * d, 256)), dim3(256), 0, s, pdl, y, x16,
                   h, d, B, pdl);
}

int launch_residual32(const YRows& y, const float* h, __half* x16, int d, int B, cudaStream_t s, int pdl) {
  return launch_ex(residual32_kernel, dim3(blocks_for(static_cast<long long>(B) * d, 256)), dim3(256), 0, s, pdl, y, h,
                   x16, d, B, pdl);
}

int launch_swiglu(const YRows& y, __half* act, int F, int B, cudaStream_t s, int pdl) {
  return launch_ex(swiglu_kernel, dim3(blocks_for(static_cast<long long>(B) * F, 256)), dim3(256), 0, s, pdl, y, act,
                   F, B, pdl);
}

int launch_argmax_gen(const float* logits, int V, const __half* embed, int d, uint32_t* q0, uint32_t* log, int cap,
                      int32_t* tok, uint32_t* force_next, __half* x16, unsigned* err, int B, cudaStream_t s, int pdl) {
  return launch_ex(argmax_gen_kernel, dim3(B), dim3(kArgThreads), 0, s, pdl, logits, V, embed, d, q0, log, cap, tok,
                   force_next, x16, err, pdl);
}

int launch_tp_reduce(const float* recv, int ranks, int rank, const unsigned* flag, const unsigned* epoch,
                     int uses_per_step, int use_in_step, int tiles_per_rank, const __half* res16, const float* res32,
                     const TpGather& gather, int d, int B, unsigned* err, cudaStream_t s, bool two_shot,
                     uint64_t wait_ns) {
  if (ranks < 1 || ranks > kMaxRanks) return fail(AGXC_EINVAL, "tp_reduce: 1 to 8 ranks");
  if (d % (4 * ranks)) return fail(AGXC_EINVAL, "tp_reduce: d a multiple of 4 x ranks");
  const long long elems4 = static_cast<long long>(B) * d / (two_shot ? ranks : 1) / 4;
  // two-shot: a fixed grid, the same on every rank (the gather target counts every rank's blocks), all resident
  const int grid = static_cast<int>(two_shot ? std::min<long long>(kNumSMs, (elems4 + 255) / 256) : (elems4 + 255) / 256);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = two_shot ? 1 : 0;
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, tp_reduce_kernel, recv, ranks, rank, flag, epoch, uses_per_step, use_in_step,
                               tiles_per_rank, res16, res32, gather, d, B, err, two_shot ? 1 : 0, wait_ns));
  return 0;
}

int launch_argmax_part(const float* logits, int V, int v0, uint32_t* pairs, int B, cudaStream_t s) {
  argmax_part_kernel<<<B, kArgThreads, 0, s>>>(logits, V, v0, pairs);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

int launch_gen_from_pairs(const uint32_t* pairs, int ranks, int V, const __half* embed, int d, uint32_t* q0,
                          uint32_t* log, int cap, int32_t* tok, uint32_t* force_next, __half* x16, unsigned* err, int B,
                          cudaStream_t s, unsigned* epoch) {
  gen_from_pairs_kernel<<<B, 256, 0, s>>>(pairs, ranks, B, V, embed, d, q0, log, cap, tok, force_next, x16, err,
                                          epoch);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

}  // namespace agxc
