// attention.cu — split-KV decode attention with a log-sum-exp merge (agxforge/kernels/attention.py: the split
// 86-165 and merge 1326-1371, attn_reference 1458-1580), and the standalone RMSNorm (norm.py:42-155).
//
// One CTA per (sequence, KV head, key chunk): the chunk boundaries follow the live length q0 + 1 read on the device,
// so a captured graph serves every position. The CTA's 4 warps stream the chunk's K and V rows (each lane 4 or 2 of
// the head dims, 8-byte loads), score every query head of the GQA group against each key (the group shares the
// K/V stream), and keep an online base-2 softmax per head (q is pre-scaled by log2(e)/sqrt(hd)). Partials
// (m, l, o[hd]) go to scratch; the last CTA of the (sequence, KV head) merges the chunks in order:
// M = max m_s, w_s = 2^(m_s - M), L = sum l_s w_s, O = sum o_s w_s, out = fp16(O / L).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = 4;
constexpr int kKeyBlock = 4;

template <int HD>
struct Lanes;
template <>
struct Lanes<128> {
  static constexpr int D = 4;
  __device__ static void load(const __half* p, float* f) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
};
template <>
struct Lanes<64> {
  static constexpr int D = 2;
  __device__ static void load(const __half* p, float* f) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(p));
    f[0] = a.x; f[1] = a.y;
  }
};

template <int HD, int GM>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnParams p) {
  constexpr int D = Lanes<HD>::D;
  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.H / p.KVH;
  __shared__ float sm_m[kAttnWarps][GM], sm_l[kAttnWarps][GM];
  __shared__ float sm_o[kAttnWarps][GM][HD];
  __shared__ int s_last;

  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  int pos = static_cast<int>(p.q0[b]);
  if (pos > p.cap - 1) pos = p.cap - 1;
  const int nk = pos + 1;
  const int L = (nk + p.S - 1) / p.S;
  const int j0 = s * L;
  const int j1 = min(nk, j0 + L);

  float q[GM][D], o[GM][D], m[GM], l[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) { o[g][d] = 0.f; q[g][d] = 0.f; }
    if (g < G) Lanes<HD>::load(p.q16 + (static_cast<size_t>(b) * p.H + kvh * G + g) * HD + lane * D, q[g]);
  }
  const size_t kvbase = (static_cast<size_t>(b) * p.KVH + kvh) * p.cap * HD;
  const __half* kc = p.kc + kvbase + lane * D;
  const __half* vc = p.vc + kvbase + lane * D;

  // warp w takes key blocks j0 + 4 (w + 4 t) ... ; keys past j1 are skipped, never read
  for (int jb = j0 + warp * kKeyBlock; jb < j1; jb += kAttnWarps * kKeyBlock) {
    float kf[kKeyBlock][D], vf[kKeyBlock][D];
#pragma unroll
    for (int t = 0; t < kKeyBlock; ++t) {
      const int j = jb + t;
      if (j < j1) {
        Lanes<HD>::load(kc + static_cast<size_t>(j) * HD, kf[t]);
        Lanes<HD>::load(vc + static_cast<size_t>(j) * HD, vf[t]);
      } else {
#pragma unroll
        for (int d = 0; d < D; ++d) { kf[t][d] = 0.f; vf[t][d] = 0.f; }
      }
    }
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g >= G) break;
      float sc[kKeyBlock];
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t) {
        float part = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) part = fmaf(q[g][d], kf[t][d], part);
        sc[t] = warp_sum(part);
      }
      float mn = m[g];
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t)
        if (jb + t < j1) mn = fmaxf(mn, sc[t]);
      const float a = exp2f(m[g] - mn);
      float lsum = l[g] * a;
#pragma unroll
      for (int d = 0; d < D; ++d) o[g][d] *= a;
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t) {
        const float pr = jb + t < j1 ? exp2f(sc[t] - mn) : 0.f;
        lsum += pr;
#pragma unroll
        for (int d = 0; d < D; ++d) o[g][d] = fmaf(pr, vf[t][d], o[g][d]);
      }
      l[g] = lsum;
      m[g] = mn;
    }
  }

  // combine the 4 warps
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
#pragma unroll
    for (int d = 0; d < D; ++d) sm_o[warp][g][lane * D + d] = o[g][d];
  }
  __syncthreads();
  const int PW = HD + 2;
  for (int t = tid; t < G * HD; t += kAttnThreads) {
    const int g = t / HD, d = t % HD;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float Ls = 0.f, Os = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = sm_m[w][g] == -INFINITY ? 0.f : exp2f(sm_m[w][g] - M);
      Ls = fmaf(sm_l[w][g], f, Ls);
      Os = fmaf(sm_o[w][g][d], f, Os);
    }
    float* dst = p.part + ((static_cast<size_t>(b) * p.H + kvh * G + g) * p.S + s) * PW;
    if (d == 0) { dst[0] = M; dst[1] = Ls; }
    dst[2 + d] = Os;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned* c = p.counters + static_cast<size_t>(b) * p.KVH + kvh;
    const unsigned prev = atomicAdd(c, 1u);
    s_last = prev == static_cast<unsigned>(p.S) - 1;
    if (s_last) atomicExch(c, 0u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int t = tid; t < G * HD; t += kAttnThreads) {
    const int g = t / HD, d = t % HD;
    const float* src = p.part + ((static_cast<size_t>(b) * p.H + kvh * G + g) * p.S) * PW;
    float M = -INFINITY;
    for (int c = 0; c < p.S; ++c) M = fmaxf(M, ld_cg(src + c * PW));
    float Ls = 0.f, Os = 0.f;
    for (int c = 0; c < p.S; ++c) {
      const float mc = ld_cg(src + c * PW);
      const float w = mc == -INFINITY ? 0.f : exp2f(mc - M);
      Ls = fmaf(ld_cg(src + c * PW + 1), w, Ls);
      Os = fmaf(ld_cg(src + c * PW + 2 + d), w, Os);
    }
    p.out[(static_cast<size_t>(b) * p.H + kvh * G + g) * HD + d] = __float2half_rn(Os / Ls);
  }
}

template <int HD, int GM>
int launch_attn_t(const AttnParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.S, p.KVH, p.nb);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = 0;
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
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<HD, GM>, p));
  return 0;
}

__global__ void rmsnorm_kernel(const void* x, int x_f32, int d, const __half* g, float eps, __half* out) {
  const int b = blockIdx.x, tid = threadIdx.x;
  __shared__ float red[32];
  float ss = 0.f;
  for (int k = tid; k < d; k += blockDim.x) {
    const float v = x_f32 ? static_cast<const float*>(x)[static_cast<size_t>(b) * d + k]
                          : __half2float(static_cast<const __half*>(x)[static_cast<size_t>(b) * d + k]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x) / 32; ++w) t += red[w];
    red[31] = rsqrtf(t / static_cast<float>(d) + eps);
  }
  __syncthreads();
  const float r = red[31];
  for (int k = tid; k < d; k += blockDim.x) {
    const float v = x_f32 ? static_cast<const float*>(x)[static_cast<size_t>(b) * d + k]
                          : __half2float(static_cast<const __half*>(x)[static_cast<size_t>(b) * d + k]);
    out[static_cast<size_t>(b) * d + k] = __float2half_rn((v * r) * __half2float(g[k]));
  }
}

}  // namespace

int attn_splits(const agxc_ctx* ctx, int nb, int KVH, int cap) {
  const int sms = ctx ? ctx->num_sms : kNumSMs;
  int S = std::max(1, 2 * sms / std::max(1, nb * KVH));
  S = std::min(S, std::max(1, cap / 16));
  return std::min(S, 64);
}

size_t attn_part_floats(int nb, int H, int S, int hd) { return static_cast<size_t>(nb) * H * S * (hd + 2); }

int launch_attention(const agxc_ctx* ctx, const AttnParams& p, cudaStream_t s) {
  if (p.H % p.KVH) return fail(AGXC_EINVAL, "attention: heads must be a multiple of kv_heads");
  const int G = p.H / p.KVH;
  if (p.hd != 64 && p.hd != 128) return fail(AGXC_EINVAL, "attention: head_dim 64 or 128");
  if (G > 8) return fail(AGXC_EINVAL, "attention: at most 8 query heads per KV head");
  if (p.S < 1 || p.nb < 1) return fail(AGXC_EINVAL, "attention: splits and batch must be positive");
  if (p.hd == 128) {
    if (G <= 2) return launch_attn_t<128, 2>(p, s);
    if (G <= 4) return launch_attn_t<128, 4>(p, s);
    return launch_attn_t<128, 8>(p, s);
  }
  if (G <= 2) return launch_attn_t<64, 2>(p, s);
  if (G <= 4) return launch_attn_t<64, 4>(p, s);
  return launch_attn_t<64, 8>(p, s);
}

int launch_rmsnorm(const void* x, int x_f32, int nb, int d, const __half* g, float eps, __half* out,
                   cudaStream_t s) {
  rmsnorm_kernel<<<nb, 256, 0, s>>>(x, x_f32, d, g, eps, out);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

}  // namespace agxc
