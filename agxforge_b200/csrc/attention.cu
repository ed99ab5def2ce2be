// attention.cu — split-KV decode attention with a log-sum-exp merge (agxforge/kernels/attention.py: the split
// 86-165 and merge 1326-1371, attn_reference 1458-1580), and the standalone RMSNorm (norm.py:42-155).
//
// One thread-block CLUSTER per (KV head, sequence); its CTAs take consecutive key chunks of the live length q0 + 1
// (read on the device, so a captured graph serves every position). A chunk's K and V rows move into shared memory by
// bulk TMA copies (sub-chunks of 64 keys, two stages; the history rows are requested before the upstream kernel
// finishes, the new row q0 is read after it, into registers). 8 warps take blocks of 4 keys (each lane 4 or 2 of the
// head dims), score every query head of the GQA group against each key (the group shares the K/V stream) and keep an
// online base-2 softmax per head (q is pre-scaled by log2(e)/sqrt(hd)). Each CTA's partial (m, l, o[hd]) stays in its
// shared memory; after a cluster barrier every CTA merges a slice of the outputs by reading the others' partials
// through distributed shared memory: M = max m_s, w_s = 2^(m_s - M), L = sum l_s w_s, O = sum o_s w_s,
// out = fp16(O / L). No global scratch, fences or atomics.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = 8;
constexpr int kKeyBlock = 4;
constexpr int kSub = 64;        // keys per shared-memory sub-chunk (K and V rows of one KV head)
constexpr int kMinChunk = 32;   // the fewest keys a chunk takes before more chunks are used

template <int HD>
struct Lanes;
template <>
struct Lanes<128> {
  static constexpr int D = 4;
  __device__ static void load(const __half* p, float* f) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    __half2 h0, h1;
    memcpy(&h0, &u.x, 4);
    memcpy(&h1, &u.y, 4);
    const float2 a = __half22float2(h0), b = __half22float2(h1);
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

__host__ __device__ inline int attn_smem_bytes(int hd) { return 128 + 2 * 2 * kSub * hd * 2; }

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

// One CLUSTER per (KV head, sequence): its gridDim.x CTAs take consecutive key chunks [s L, min(nk, (s+1) L)),
// L = ceil(nk / gridDim.x), and meet in distributed shared memory for the merge. Every CTA passes both cluster
// barriers on every path (an empty chunk contributes m = -inf), so no CTA waits on one that left.
template <int HD, int GM>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnParams p) {
  constexpr int D = Lanes<HD>::D;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  __half* kv = reinterpret_cast<__half*>(smem + 128);  // stage st: K rows at st*2*kSub*HD, V rows after kSub*HD
  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int CL = gridDim.x;  // the cluster spans gridDim.x: the CTA's rank is blockIdx.x
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.H / p.KVH;
  __shared__ float sm_m[kAttnWarps][GM], sm_l[kAttnWarps][GM];
  __shared__ float sm_o[kAttnWarps][GM][HD];
  __shared__ float part_m[GM], part_l[GM];
  __shared__ float part_o[GM][HD];

  // the history rows (keys before q0) were written by earlier steps: they stream in before the upstream kernel
  // (which appends row q0) has finished
  int pos = static_cast<int>(p.q0[b]);
  if (pos > p.cap - 1) pos = p.cap - 1;
  const int nk = pos + 1;
  const int L = (nk + CL - 1) / CL;
  const int j0 = s * L;
  const int j1 = min(nk, j0 + L);
  const int nsub = j1 > j0 ? (j1 - j0 + kSub - 1) / kSub : 0;
  const size_t kvbase = (static_cast<size_t>(b) * p.KVH + kvh) * p.cap * HD;

  auto issue = [&](int i) {  // sub-chunk i -> stage i % 2: the rows below pos (row pos is read after the wait)
    const int a = j0 + i * kSub;
    const int n = max(0, min(min(a + kSub, j1), pos) - a);
    uint64_t* bar = &bars[i & 1];
    __half* dst = kv + (i & 1) * 2 * kSub * HD;
    mbar_arrive_expect_tx(bar, static_cast<unsigned>(2 * n * HD * 2));
    if (n) {
      bulk_g2s(dst, p.kc + kvbase + static_cast<size_t>(a) * HD, n * HD * 2, bar);
      bulk_g2s(dst + kSub * HD, p.vc + kvbase + static_cast<size_t>(a) * HD, n * HD * 2, bar);
    }
  };
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    for (int i = 0; i < 2 && i < nsub; ++i) issue(i);
  }
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }

  float q[GM][D], o[GM][D], m[GM], l[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) { o[g][d] = 0.f; q[g][d] = 0.f; }
    if (g < G) Lanes<HD>::load(p.q16 + (static_cast<size_t>(b) * p.H + kvh * G + g) * HD + lane * D, q[g]);
  }
  // the new row, appended by the upstream kernel: this lane's dims, in registers
  float knew[D], vnew[D];
  const bool has_new = pos >= j0 && pos < j1;
  if (has_new) {
    Lanes<HD>::load(p.kc + kvbase + static_cast<size_t>(pos) * HD + lane * D, knew);
    Lanes<HD>::load(p.vc + kvbase + static_cast<size_t>(pos) * HD + lane * D, vnew);
  } else {
#pragma unroll
    for (int d = 0; d < D; ++d) knew[d] = vnew[d] = 0.f;
  }

  bool ok = true;
  for (int i = 0; i < nsub; ++i) {
    const int a = j0 + i * kSub;
    const int n = min(kSub, j1 - a);
    const __half* st = kv + (i & 1) * 2 * kSub * HD;
    if (ok && !mbar_wait_bounded(&bars[i & 1], (i >> 1) & 1, p.err)) ok = false;
    for (int kb = warp * kKeyBlock; kb < n; kb += kAttnWarps * kKeyBlock) {
      float kf[kKeyBlock][D], vf[kKeyBlock][D];
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t) {
        const int j = min(kb + t, n - 1);
        if (a + j == pos) {
#pragma unroll
          for (int d = 0; d < D; ++d) { kf[t][d] = knew[d]; vf[t][d] = vnew[d]; }
        } else {
          Lanes<HD>::load(st + j * HD + lane * D, kf[t]);
          Lanes<HD>::load(st + kSub * HD + j * HD + lane * D, vf[t]);
        }
      }
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        if (g < G) {
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
            if (kb + t < n) mn = fmaxf(mn, sc[t]);
          const float al = exp2f(m[g] - mn);
          float lsum = l[g] * al;
#pragma unroll
          for (int d = 0; d < D; ++d) o[g][d] *= al;
#pragma unroll
          for (int t = 0; t < kKeyBlock; ++t) {
            const float pr = kb + t < n ? exp2f(sc[t] - mn) : 0.f;
            lsum += pr;
#pragma unroll
            for (int d = 0; d < D; ++d) o[g][d] = fmaf(pr, vf[t][d], o[g][d]);
          }
          l[g] = lsum;
          m[g] = mn;
        }
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && i + 2 < nsub) issue(i + 2);
  }
  if (!ok) {
    // a sub-chunk never landed (the error word is set): wait out what is still in flight (bounded), then take part
    // in the cluster barriers with an empty partial
    if (tid == 0)
      for (int i = 0; i < nsub && i < 2; ++i) mbar_wait_bounded(&bars[i & 1], 0, nullptr, 100000000ull);
#pragma unroll
    for (int g = 0; g < GM; ++g) m[g] = -INFINITY;
  }

  // combine the warps into this CTA's chunk partial
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      if (lane == 0) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
#pragma unroll
      for (int d = 0; d < D; ++d) sm_o[warp][g][lane * D + d] = o[g][d];
    }
  }
  __syncthreads();
  for (int t = tid; t < G * HD; t += kAttnThreads) {
    const int g = t / HD, d = t % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float Ls = 0.f, Os = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = sm_m[w][g] == -INFINITY ? 0.f : exp2f(sm_m[w][g] - M);
      Ls = fmaf(sm_l[w][g], f, Ls);
      Os = fmaf(sm_o[w][g][d], f, Os);
    }
    if (d == 0) { part_m[g] = M; part_l[g] = Ls; }
    part_o[g][d] = Os;
  }
  // the chunks meet in distributed shared memory: CTA s merges outputs [s per, (s+1) per) of the G x HD
  cluster_sync_all();
  const int total = G * HD, per = (total + CL - 1) / CL;
  for (int t = s * per + tid; t < min(total, (s + 1) * per); t += kAttnThreads) {
    const int g = t / HD, d = t % HD;
    float M = -INFINITY;
    for (int r = 0; r < CL; ++r) M = fmaxf(M, ld_dsmem(dsmem_addr(&part_m[g], r)));
    float Ls = 0.f, Os = 0.f;
    for (int r = 0; r < CL; ++r) {
      const float mr = ld_dsmem(dsmem_addr(&part_m[g], r));
      if (mr == -INFINITY) continue;
      const float w = exp2f(mr - M);
      Ls = fmaf(ld_dsmem(dsmem_addr(&part_l[g], r)), w, Ls);
      Os = fmaf(ld_dsmem(dsmem_addr(&part_o[g][d], r)), w, Os);
    }
    p.out[(static_cast<size_t>(b) * p.H + kvh * G + g) * HD + d] = __float2half_rn(Os / Ls);
  }
  cluster_sync_all();  // no CTA leaves while another still reads its partial
}

template <int HD, int GM>
int launch_attn_t(const AttnParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.S, p.KVH, p.nb);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = attn_smem_bytes(HD);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = p.S;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
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

template <typename K>
int attn_allow(K kern, int optin) {
  cudaFuncAttributes fa;
  AGXC_CUDA(cudaFuncGetAttributes(&fa, kern));
  AGXC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - static_cast<int>(fa.sharedSizeBytes)));
  AGXC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  return 0;
}

// The largest power-of-two cluster (<= 16) the device can place for this kernel.
template <int HD, int GM>
int max_cluster() {
  for (int c = 16; c >= 1; c /= 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c, 1, 1);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(HD);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_kernel<HD, GM>, &cfg) == cudaSuccess && n > 0) return c;
    cudaGetLastError();
  }
  return 1;
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

// The cluster size (key chunks per KV head): a power of two filling the SMs once with the (KV head, sequence)
// clusters, no more chunks than cap / 32 keys, and no larger than the device places.
int attn_splits(const agxc_ctx* ctx, int nb, int KVH, int cap) {
  const int sms = ctx ? ctx->num_sms : kNumSMs;
  const int want = std::max(1, sms / std::max(1, nb * KVH));
  int S = 1;
  while (S * 2 <= want && S * 2 <= std::max(1, cap / kMinChunk) && S * 2 <= (ctx ? ctx->max_cluster : 8)) S *= 2;
  return S;
}

int attn_configure(agxc_ctx* ctx) {
  const int o = ctx->max_smem_optin;
  int rc;
  if ((rc = attn_allow(attn_kernel<128, 1>, o)) || (rc = attn_allow(attn_kernel<128, 2>, o)) ||
      (rc = attn_allow(attn_kernel<128, 4>, o)) || (rc = attn_allow(attn_kernel<128, 8>, o)) ||
      (rc = attn_allow(attn_kernel<64, 1>, o)) || (rc = attn_allow(attn_kernel<64, 2>, o)) ||
      (rc = attn_allow(attn_kernel<64, 4>, o)) || (rc = attn_allow(attn_kernel<64, 8>, o)))
    return rc;
  ctx->max_cluster = max_cluster<128, 8>();  // the largest variant bounds every other
  return 0;
}

size_t attn_part_floats(int nb, int H, int S, int hd) { return static_cast<size_t>(nb) * H * S * (hd + 2); }

int launch_attention(const agxc_ctx* ctx, const AttnParams& p, cudaStream_t s) {
  if (p.H % p.KVH) return fail(AGXC_EINVAL, "attention: heads must be a multiple of kv_heads");
  const int G = p.H / p.KVH;
  if (p.hd != 64 && p.hd != 128) return fail(AGXC_EINVAL, "attention: head_dim 64 or 128");
  if (G > 8) return fail(AGXC_EINVAL, "attention: at most 8 query heads per KV head");
  if (p.S < 1 || p.S > 16 || (p.S & (p.S - 1)) || p.nb < 1)
    return fail(AGXC_EINVAL, "attention: splits a power of two up to 16, and a positive batch");
  if (ctx && p.S > ctx->max_cluster) return fail(AGXC_EINVAL, "attention: splits exceed the device's cluster size");
  if (p.hd == 128) {
    if (G == 1) return launch_attn_t<128, 1>(p, s);
    if (G <= 2) return launch_attn_t<128, 2>(p, s);
    if (G <= 4) return launch_attn_t<128, 4>(p, s);
    return launch_attn_t<128, 8>(p, s);
  }
  if (G == 1) return launch_attn_t<64, 1>(p, s);
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
