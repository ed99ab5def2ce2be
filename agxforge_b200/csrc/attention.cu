// attention.cu — split-KV decode attention with a log-sum-exp merge (agxforge/kernels/attention.py: the split
// 86-165 and merge 1326-1371, attn_reference 1458-1580), and the standalone RMSNorm (norm.py:42-155).
//
// One thread-block CLUSTER per (KV head, sequence); its CTAs take consecutive key chunks of the live length q0 + 1
// (read on the device, so a captured graph serves every position). The scores and the weighted values run on the
// tensor cores (mma.sync m16n8k16, fp16 in, fp32 accumulate) with the KEYS as the M dimension and the GQA group's
// query heads (up to 8) as N, so one MMA covers every head of the group:
//     S^T[16 keys][8 heads]  = K[16 keys][hd] . Q^T[hd][8 heads]        (K fragments by ldmatrix)
//     O^T[hd][8 heads]      += V^T[hd][16 keys] . P^T[16 keys][8 heads]  (V by ldmatrix.trans, P^T by movmatrix.trans)
// q is pre-scaled by log2(e)/sqrt(hd), so the softmax is base 2; P is rounded to fp16 for the second product, the
// running sums stay fp32. K and V move into shared memory by TMA tensor copies (boxes of 64 dims x 128 keys, 128-byte
// swizzle, so ldmatrix reads without bank conflicts) in 64-key sub-chunks, two stages; each warp takes a 16-key tile
// of every sub-chunk. The history rows are requested before the upstream kernel finishes; the new row q0 is read after
// it and replaces its stale copy in shared memory. Each CTA's partial (m, l, o[hd]) stays in its shared memory;
// after a cluster barrier every CTA merges a slice of the outputs by reading the others' partials through
// distributed shared memory: M = max m_s, w_s = 2^(m_s - M), L = sum l_s w_s, O = sum o_s w_s, out = fp16(O / L).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

// Two shapes of CTA: NW = 8 warps and 128-key sub-chunks (132 KB of shared memory at head_dim 128) for one to a few
// sequences, where each KV head's keys split over a cluster; NW = 4 warps and 64-key sub-chunks (66 KB, three CTAs an
// SM) for batched steps, whose sequences x KV heads already fill the SMs and want to be resident at once.
template <int NW> constexpr int kThr = NW * 32;
template <int NW> constexpr int kSubK = NW * 16;  // keys per shared-memory sub-chunk: one 16-key tile per warp
constexpr int kMinChunk = 32;    // the fewest keys a chunk takes before more chunks are used
constexpr int kHeadsN = 8;       // the MMA's N: query heads of one KV head

// A stage holds K then V of one sub-chunk, each as HD / 64 boxes of [kSubK rows][128 B] in the TMA's 128-byte swizzle
// (the 16-byte chunk c of row r sits at chunk c ^ (r % 8)), so ldmatrix reads 8 rows of one chunk without conflicts.
template <int NW> __host__ __device__ constexpr int box_bytes() { return kSubK<NW> * 128; }
template <int NW> __host__ __device__ constexpr int stage_bytes(int hd) { return 2 * (hd / 64) * box_bytes<NW>(); }
template <int NW> __host__ __device__ inline int attn_smem_bytes(int hd) { return 1024 + 2 * stage_bytes<NW>(hd); }

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset of (row, 16-byte chunk) in a box
  return static_cast<uint32_t>(row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
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

// One CLUSTER per (KV head, sequence): its gridDim.x CTAs take consecutive key chunks [s L, min(nk, (s+1) L)),
// L = ceil(nk / gridDim.x), and meet in distributed shared memory for the merge. Every CTA passes both cluster
// barriers on every path (an empty chunk contributes m = -inf), so no CTA waits on one that left.
template <int HD, int NW>
__global__ void __launch_bounds__(kThr<NW>) attn_kernel(AttnParams p, const __grid_constant__ CUtensorMap tk,
                                                            const __grid_constant__ CUtensorMap tv) {
  constexpr int KS = HD / 16;  // k-steps of the score product, dim tiles of the value product
  constexpr int NB = HD / 64;  // boxes per K (or V) sub-chunk
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // the swizzle wants 1,024 B
  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int CL = gridDim.x;  // the cluster spans gridDim.x: the CTA's rank is blockIdx.x
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;  // MMA fragment coordinates
  const int G = p.H / p.KVH;
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ float sm_m[NW][kHeadsN], sm_l[NW][kHeadsN];
  __shared__ float part_m[kHeadsN], part_l[kHeadsN];
  __shared__ float part_o[kHeadsN][HD];

  int pos = static_cast<int>(p.q0[b]);
  if (pos > p.cap - 1) pos = p.cap - 1;
  const int nk = pos + 1;
  const int L = (nk + CL - 1) / CL;
  const int j0 = s * L;
  const int j1 = min(nk, j0 + L);
  const int nsub = j1 > j0 ? (j1 - j0 + kSubK<NW> - 1) / kSubK<NW> : 0;
  const size_t kvbase = (static_cast<size_t>(b) * p.KVH + kvh) * p.cap * HD;
  const int zrow = b * p.KVH + kvh;

  // sub-chunk i -> stage i % 2: whole boxes of kSubK rows from key j0 + i kSubK (rows past the cache end read as zero;
  // rows from pos on are replaced or masked: row pos is written by the upstream kernel, read after the wait)
  auto issue = [&](int i) {
    uint64_t* bar = &bars[i & 1];
    uint8_t* st = smem + (i & 1) * stage_bytes<NW>(HD);
    mbar_arrive_expect_tx(bar, static_cast<unsigned>(stage_bytes<NW>(HD)));
#pragma unroll
    for (int h = 0; h < NB; ++h) {
      tma_load_3d(st + h * box_bytes<NW>(), &tk, h * 64, j0 + i * kSubK<NW>, zrow, bar);
      tma_load_3d(st + (NB + h) * box_bytes<NW>(), &tv, h * 64, j0 + i * kSubK<NW>, zrow, bar);
    }
  };
  if (tid == 0) {
    trace_mark(p.trace, 0);
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
  }
  __syncthreads();
  if (tid == 0) {
    for (int i = 0; i < 2 && i < nsub; ++i) issue(i);
  }
  if (p.pdl) {
    pdl_wait();
    if (p.pdl == 1) pdl_launch_dependents();
  }
  if (tid == 0) trace_mark(p.trace, 1);

  // Q^T fragments (B operand, N = heads): lane (g8, t4) holds Q[head g8][16 ks + 2 t4 + {0, 1, 8, 9}]
  uint32_t qb[KS][2];
  {
    const bool live = g8 < G;
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        p.q16 + (static_cast<size_t>(b) * p.H + kvh * G + (live ? g8 : 0)) * HD);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qb[ks][0] = live ? qrow[ks * 8 + t4] : 0u;
      qb[ks][1] = live ? qrow[ks * 8 + 4 + t4] : 0u;
    }
  }
  // running state for heads 2 t4 and 2 t4 + 1; O^T accumulators: dims 16 dt + g8 (+8) x heads 2 t4 (+1)
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float oacc[KS][4];
#pragma unroll
  for (int dt = 0; dt < KS; ++dt) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.f;

  const int kt = warp * 16;               // this warp's 16-key tile of every sub-chunk
  const int krow = kt + (lane & 7) + ((lane >> 3) & 1) * 8;   // ldmatrix row addresses: K (A = K)
  const int vrow = kt + (lane & 7) + (lane >> 4) * 8;         // and V (A = V^T, transposed load)
  bool ok = true;
  int i = 0;
  for (; i < nsub; ++i) {
    const int a = j0 + i * kSubK<NW>;
    const int n = min(kSubK<NW>, j1 - a);
    uint8_t* Ks = smem + (i & 1) * stage_bytes<NW>(HD);
    uint8_t* Vs = Ks + NB * box_bytes<NW>();
    const bool landed = mbar_wait_bounded(&bars[i & 1], (i >> 1) & 1, p.err);
    if (__syncthreads_or(!landed)) {  // leave together: the error word is set
      ok = false;
      break;
    }
    const int n16 = (n + 15) & ~15;
    if ((pos >= a && pos < a + n) || n16 != n) {  // CTA-uniform
      // the new row from global (after the dependency wait); V rows up to the next tile zeroed (P = 0 there, and
      // 0 x NaN would not vanish in the product)
      if (pos >= a && pos < a + n && tid < 2 * HD / 8) {
        const int kv = tid / (HD / 8), c = tid % (HD / 8);
        const uint4 v = reinterpret_cast<const uint4*>((kv ? p.vc : p.kc) + kvbase + static_cast<size_t>(pos) * HD)[c];
        *reinterpret_cast<uint4*>((kv ? Vs : Ks) + (c >> 3) * box_bytes<NW>() + swz(pos - a, c)) = v;
      }
      for (int t = tid; t < (n16 - n) * (HD / 8); t += kThr<NW>) {
        const int r = n + t / (HD / 8), c = t % (HD / 8);
        *reinterpret_cast<uint4*>(Vs + (c >> 3) * box_bytes<NW>() + swz(r, c)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async();  // generic writes into a buffer that later bulk copies overwrite
      __syncthreads();
    }

    if (kt < n) {
      // S^T tile: keys kt + g8 (c0, c1) and kt + g8 + 8 (c2, c3), heads 2 t4 and 2 t4 + 1
      float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a0, a1, a2, a3;
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(smem_u32(Ks + (c >> 3) * box_bytes<NW>() + swz(krow, c)), a0, a1, a2, a3);
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
      const float mn0 = fmaxf(m0, x0), mn1 = fmaxf(m1, x1);  // finite: key kt is live
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      const float p0 = exp2f(s0 - mn0), p1 = exp2f(s1 - mn1), p2 = exp2f(s2 - mn0), p3 = exp2f(s3 - mn1);
      l0 = fmaf(l0, al0, p0 + p2);
      l1 = fmaf(l1, al1, p1 + p3);
      m0 = mn0;
      m1 = mn1;
      // P^T as the B operand: lane (g8, t4) needs P[head g8][keys 2 t4 (+1)] and [keys 2 t4 + 8 (+9)]
      const uint32_t pb0 = movm_t(pack_h2(p0, p1)), pb1 = movm_t(pack_h2(p2, p3));
#pragma unroll
      for (int dt = 0; dt < KS; ++dt) {
        oacc[dt][0] *= al0;
        oacc[dt][1] *= al1;
        oacc[dt][2] *= al0;
        oacc[dt][3] *= al1;
        uint32_t a0, a1, a2, a3;
        const int c = dt * 2 + ((lane >> 3) & 1);
        ldsm_x4_t(smem_u32(Vs + (c >> 3) * box_bytes<NW>() + swz(vrow, c)), a0, a1, a2, a3);
        mma_16816(oacc[dt][0], oacc[dt][1], oacc[dt][2], oacc[dt][3], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && i + 2 < nsub) issue(i + 2);
  }
  if (!ok) {
    // a sub-chunk never landed: wait out the copies still in flight (bounded), contribute nothing
    if (tid == 0) {
      mbar_wait_bounded(&bars[i & 1], (i >> 1) & 1, nullptr, 100000000ull);
      if (i + 1 < nsub) mbar_wait_bounded(&bars[(i + 1) & 1], ((i + 1) >> 1) & 1, nullptr, 100000000ull);
    }
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int dt = 0; dt < KS; ++dt) oacc[dt][0] = oacc[dt][1] = oacc[dt][2] = oacc[dt][3] = 0.f;
    __syncthreads();
  }

  if (p.pdl >= 2) pdl_launch_dependents();
  // l over the warp's 16 key rows (lanes with the same t4); then the warp's partial to shared memory (the stage
  // buffers are free now)
#pragma unroll
  for (int off = 4; off <= 16; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  float (*sm_o)[kHeadsN][HD] = reinterpret_cast<float (*)[kHeadsN][HD]>(smem);
  if (g8 == 0) {
    sm_m[warp][2 * t4] = m0;
    sm_m[warp][2 * t4 + 1] = m1;
    sm_l[warp][2 * t4] = l0;
    sm_l[warp][2 * t4 + 1] = l1;
  }
#pragma unroll
  for (int dt = 0; dt < KS; ++dt) {
    sm_o[warp][2 * t4][16 * dt + g8] = oacc[dt][0];
    sm_o[warp][2 * t4 + 1][16 * dt + g8] = oacc[dt][1];
    sm_o[warp][2 * t4][16 * dt + g8 + 8] = oacc[dt][2];
    sm_o[warp][2 * t4 + 1][16 * dt + g8 + 8] = oacc[dt][3];
  }
  __syncthreads();
  // combine the warps into this CTA's chunk partial
  for (int t = tid; t < G * HD; t += kThr<NW>) {
    const int g = t / HD, d = t % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][g]);
    float Ls = 0.f, Os = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = sm_m[w][g] == -INFINITY ? 0.f : exp2f(sm_m[w][g] - M);
      Ls = fmaf(sm_l[w][g], f, Ls);
      Os = fmaf(sm_o[w][g][d], f, Os);
    }
    if (d == 0) { part_m[g] = M; part_l[g] = Ls; }
    part_o[g][d] = Os;
  }
  // the chunks meet in distributed shared memory: CTA s merges outputs [s per, (s+1) per) of the G x HD; CL adjacent
  // lanes take one output, lane r reading chunk r's partial, so every remote load of a pass is in flight at once
  cluster_sync_all();
  const int total = G * HD, per = (total + CL - 1) / CL;
  const int ro = kThr<NW> / CL;
  const int r = tid % CL;
  for (int base = 0; base < per; base += ro) {  // the same trip count in every thread
    const int oi = base + tid / CL, t = s * per + oi;
    const bool valid = oi < per && t < total;
    const int tt = valid ? t : 0;
    const int g = tt / HD, d = tt % HD;
    const float mr = ld_dsmem(dsmem_addr(&part_m[g], r));
    const float lr = ld_dsmem(dsmem_addr(&part_l[g], r));
    const float orr = ld_dsmem(dsmem_addr(&part_o[g][d], r));
    float M = mr;
    for (int off = 1; off < CL; off <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float w = mr == -INFINITY ? 0.f : exp2f(mr - M);
    float Ls = lr * w, Os = orr * w;
    for (int off = 1; off < CL; off <<= 1) {
      Ls += __shfl_xor_sync(0xffffffffu, Ls, off);
      Os += __shfl_xor_sync(0xffffffffu, Os, off);
    }
    if (valid && r == 0) p.out[(static_cast<size_t>(b) * p.H + kvh * G + g) * HD + d] = __float2half_rn(Os / Ls);
  }
  cluster_sync_all();  // no CTA leaves while another still reads its partial
  if (tid == 0) trace_mark(p.trace, 2);
}

template <int HD, int NW>
cudaLaunchConfig_t attn_config(const AttnParams& p, cudaStream_t s, cudaLaunchAttribute* attr, int cluster) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster, p.KVH, p.nb);
  cfg.blockDim = dim3(kThr<NW>);
  cfg.dynamicSmemBytes = attn_smem_bytes<NW>(HD);
  cfg.stream = s;
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = cluster;
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
  return cfg;
}

template <int HD, int NW>
int launch_attn_t(const AttnParams& p, cudaStream_t s) {
  // the KV maps: boxes of 64 dims x the variant's sub-chunk keys
  CUtensorMap tk, tv;
  const int64_t Z = static_cast<int64_t>(p.nb) * p.KVH;
  if (int rc = encode_kv_map_box(&tk, p.kc, HD, p.cap, Z, kSubK<NW>)) return rc;
  if (int rc = encode_kv_map_box(&tv, p.vc, HD, p.cap, Z, kSubK<NW>)) return rc;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = attn_config<HD, NW>(p, s, attr, p.S);
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<HD, NW>, p, tk, tv));
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

// How many clusters of each power-of-two size (1 .. 16) the device keeps resident at once.
template <int HD, int NW>
void cluster_residency(int* active) {
  AttnParams p;
  p.KVH = 1;
  for (int i = 0; i < 5; ++i) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = attn_config<HD, NW>(p, nullptr, attr, 1 << i);
    cfg.gridDim = dim3(1 << i, 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_kernel<HD, NW>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    active[i] = n;
  }
}

__global__ void rmsnorm_kernel(const void* x, int x_f32, int d, const __half* g, float eps, __half* out, int pdl) {
  pdl_enter(pdl);
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

// The cluster size (key chunks per KV head): the largest power of two whose nb x KVH clusters are all resident at
// once (one wave), without more CTAs than SMs, and with at least 32 keys of cap per chunk.
int attn_splits(const agxc_ctx* ctx, int nb, int KVH, int cap) {
  const int sms = ctx ? ctx->num_sms : kNumSMs;
  const int clusters = std::max(1, nb * KVH);
  if (nb >= 16) {
    // the 4-warp CTAs (three an SM): split the keys while every CTA still fits one wave; when even unsplit groups
    // overfill it, split in two so the second wave is not a thin tail. Measured (history 1,792 unless noted): 32
    // sequences x 8 KV heads (256 CTAs) unsplit 13.7k tok/s, in two 12.8k; 64 sequences (512) unsplit 18.5k, in two
    // 19.3k; the 7B shape, 64 sequences at 8,192 keys: unsplit 4,350, in two 4,654, in four 4,672.
    const int slots = 3 * sms;
    int S = 1;
    for (int c = 2; c <= 16; c *= 2) {
      if (c * clusters > slots || c > std::max(1, cap / kMinChunk) || (ctx && c > ctx->max_cluster)) break;
      S = c;
    }
    if (S == 1 && clusters > slots && 2 <= cap / kMinChunk && (!ctx || ctx->max_cluster >= 2)) S = 2;
    return S;
  }
  int S = 1;
  for (int i = 1; i < 5; ++i) {
    const int c = 1 << i;
    if (c * clusters > sms || c > std::max(1, cap / kMinChunk)) break;
    if (ctx && (c > ctx->max_cluster || ctx->cluster_active[i] < clusters)) break;
    S = c;
  }
  return S;
}

int attn_configure(agxc_ctx* ctx) {
  const int o = ctx->max_smem_optin;
  int rc;
  if ((rc = attn_allow(attn_kernel<128, 8>, o)) || (rc = attn_allow(attn_kernel<64, 8>, o)) ||
      (rc = attn_allow(attn_kernel<128, 4>, o)) || (rc = attn_allow(attn_kernel<64, 4>, o)))
    return rc;
  cluster_residency<128, 8>(ctx->cluster_active);  // the largest variant bounds the others
  ctx->max_cluster = 1;
  for (int i = 0; i < 5; ++i)
    if (ctx->cluster_active[i] > 0) ctx->max_cluster = 1 << i;
  return 0;
}

size_t attn_part_floats(int nb, int H, int S, int hd) { return static_cast<size_t>(nb) * H * S * (hd + 2); }

int launch_attention(const agxc_ctx* ctx, const AttnParams& p, cudaStream_t s) {
  if (p.H % p.KVH) return fail(AGXC_EINVAL, "attention: heads must be a multiple of kv_heads");
  const int G = p.H / p.KVH;
  if (p.hd != 64 && p.hd != 128) return fail(AGXC_EINVAL, "attention: head_dim 64 or 128");
  if (G > kHeadsN) return fail(AGXC_EINVAL, "attention: at most 8 query heads per KV head");
  if (p.S < 1 || p.S > 16 || (p.S & (p.S - 1)) || p.nb < 1)
    return fail(AGXC_EINVAL, "attention: splits a power of two up to 16, and a positive batch");
  if (ctx && p.S > ctx->max_cluster) return fail(AGXC_EINVAL, "attention: splits exceed the device's cluster size");
  // 16 or more sequences: the 4-warp CTAs (three an SM; their sequences x KV heads fill the SMs); fewer: 8 warps
  // (measured faster there: one sequence's key chunks split over a cluster)
  const bool small_cta = p.nb >= 16;
  if (p.hd == 128) return small_cta ? launch_attn_t<128, 4>(p, s) : launch_attn_t<128, 8>(p, s);
  return small_cta ? launch_attn_t<64, 4>(p, s) : launch_attn_t<64, 8>(p, s);
}

int launch_rmsnorm(const void* x, int x_f32, int nb, int d, const __half* g, float eps, __half* out,
                   cudaStream_t s, int pdl) {
  return launch_ex(rmsnorm_kernel, dim3(nb), dim3(256), 0, s, pdl, x, x_f32, d, g, eps, out, pdl);
}

}  // namespace agxc
