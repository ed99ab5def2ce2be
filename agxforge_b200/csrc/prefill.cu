// prefill.cu — causal attention of a prompt chunk (the reference's prefill section, agxforge/inference/prefill.py:1-30,
// its attention prefill_attention.py / prefill_mma.py): M query rows of one sequence at positions p0 .. p0 + M - 1,
// each attending to the keys 0 .. its own position of the fp16 KV cache (rows p0 .. written by the chunk's append).
//
// One CTA per (64-query block, query head): four warps of 16 query rows; K and V of the head's KV head stream through
// shared memory in 64-key tiles (cp.async, two stages, rows padded to 272 B so ldmatrix reads are conflict-free).
// Per tile: S = Q K^T (mma.sync m16n8k16, fp16 in, fp32 accumulate; K fragments by ldmatrix), causal mask, online
// base-2 softmax (q is pre-scaled by log2(e)/sqrt(hd) like the decode step's), P rounded to fp16 and kept in registers
// as the A operand of O += P V (V fragments by ldmatrix.trans). The same numerics as the decode attention.
#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

constexpr int kPQ = 64;        // query rows per CTA (4 warps x 16)
constexpr int kPK = 64;        // keys per tile

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const unsigned n = pred ? 16u : 0u;  // zero-fill when the row is past the cache
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ uint32_t h2u(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int HD>
__global__ void __launch_bounds__(128) prefill_attn_kernel(const __half* __restrict__ q16, const __half* __restrict__ kc,
                                                           const __half* __restrict__ vc, int M, int p0, int H, int KVH,
                                                           int cap, int seq, __half* __restrict__ out) {
  constexpr int LD = HD + 8;                 // halves per shared row (272 B at HD 128, 144 B at 64)
  constexpr int KS = HD / 16;                // k-steps of Q K^T
  constexpr int NT = HD / 8;                 // n-tiles of P V
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __half* sk = reinterpret_cast<__half*>(smem_raw);      // [2][kPK][LD]
  __half* sv = sk + 2 * kPK * LD;                          // [2][kPK][LD]
  const int qb = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int kvh = h / (H / KVH);
  const __half* kbase = kc + (static_cast<size_t>(seq) * KVH + kvh) * cap * HD;
  const __half* vbase = vc + (static_cast<size_t>(seq) * KVH + kvh) * cap * HD;
  const int r0 = qb * kPQ + warp * 16;       // this warp's first query row (chunk row index)
  const int rows_end = min(M, qb * kPQ + kPQ);
  const int last_pos = p0 + rows_end - 1;    // the CTA's latest query position: keys 0 .. last_pos
  const int ntiles = last_pos / kPK + 1;

  auto load_tile = [&](int j, int st) {
    const int k0 = j * kPK;
    __half* dk = sk + st * kPK * LD;
    __half* dv = sv + st * kPK * LD;
    for (int c = tid; c < kPK * (HD / 8); c += 128) {
      const int r = c / (HD / 8), cc = (c % (HD / 8)) * 8;
      const int key = k0 + r;
      const bool in = key < cap;
      const size_t off = static_cast<size_t>(in ? key : 0) * HD + cc;
      cp_async16(dk + r * LD + cc, kbase + off, in);
      cp_async16(dv + r * LD + cc, vbase + off, in);
    }
    cp_commit();
  };
  load_tile(0, 0);
  if (ntiles > 1) load_tile(1, 1);

  // Q fragments of the warp's 16 rows (rows past M read as zero; their outputs are not written)
  uint32_t qa[KS][4];
  {
    const int ra = r0 + g, rb = r0 + g + 8;
    const __half* qra = q16 + (static_cast<size_t>(ra < M ? ra : 0) * H + h) * HD;
    const __half* qrb = q16 + (static_cast<size_t>(rb < M ? rb : 0) * H + h) * HD;
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      const int c = 16 * k + 2 * t;
      qa[k][0] = ra < M ? *reinterpret_cast<const uint32_t*>(qra + c) : 0u;
      qa[k][1] = rb < M ? *reinterpret_cast<const uint32_t*>(qrb + c) : 0u;
      qa[k][2] = ra < M ? *reinterpret_cast<const uint32_t*>(qra + c + 8) : 0u;
      qa[k][3] = rb < M ? *reinterpret_cast<const uint32_t*>(qrb + c + 8) : 0u;
    }
  }
  const int pa = p0 + r0 + g, pb = pa + 8;   // positions of this thread's two rows
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    const int st = j & 1;
    if (j + 1 < ntiles) cp_wait1();
    else cp_wait0();
    __syncthreads();
    const __half* tk = sk + st * kPK * LD;
    const __half* tv = sv + st * kPK * LD;
    const int k0 = j * kPK;
    const bool warp_live = k0 <= p0 + r0 + 15 && r0 < M;  // some key of the tile is visible to the warp's rows
    if (warp_live) {
      // S = Q K^T: 16 rows x 64 keys = 8 n-tiles
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // key tiles 2np, 2np + 1
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          // matrices: (keys 16np + 0..7, dims 16k + 0..7), (.., dims +8), (keys +8, dims 16k), (keys +8, dims +8)
          const int mi = lane >> 3, rr = lane & 7;
          const int key = 16 * np + (mi >> 1) * 8 + rr, dim = 16 * k + (mi & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm4(smem_u32(tk + key * LD + dim), b0, b1, b2, b3);
          mma_16816(s[2 * np][0], s[2 * np][1], s[2 * np][2], s[2 * np][3], qa[k][0], qa[k][1], qa[k][2], qa[k][3],
                    b0, b1);
          mma_16816(s[2 * np + 1][0], s[2 * np + 1][1], s[2 * np + 1][2], s[2 * np + 1][3], qa[k][0], qa[k][1],
                    qa[k][2], qa[k][3], b2, b3);
        }
      }
      // causal mask and the online softmax (base 2)
      float ta = -INFINITY, tb = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int key = k0 + 8 * n + 2 * t;
        if (key > pa) s[n][0] = -INFINITY;
        if (key + 1 > pa) s[n][1] = -INFINITY;
        if (key > pb) s[n][2] = -INFINITY;
        if (key + 1 > pb) s[n][3] = -INFINITY;
        ta = fmaxf(ta, fmaxf(s[n][0], s[n][1]));
        tb = fmaxf(tb, fmaxf(s[n][2], s[n][3]));
      }
#pragma unroll
      for (int x = 1; x <= 2; x <<= 1) {
        ta = fmaxf(ta, __shfl_xor_sync(0xffffffffu, ta, x));
        tb = fmaxf(tb, __shfl_xor_sync(0xffffffffu, tb, x));
      }
      const float na = fmaxf(ma, ta), nb = fmaxf(mb, tb);
      // a row with no visible key yet keeps m = -inf: its weights are 0 and nothing is rescaled
      const float ca = na == -INFINITY ? 1.f : exp2f(ma - na), cb = nb == -INFINITY ? 1.f : exp2f(mb - nb);
      const float sa = na == -INFINITY ? 0.f : na, sb = nb == -INFINITY ? 0.f : nb;
      ma = na;
      mb = nb;
      float ra = 0.f, rb = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        s[n][0] = exp2f(s[n][0] - sa);
        s[n][1] = exp2f(s[n][1] - sa);
        s[n][2] = exp2f(s[n][2] - sb);
        s[n][3] = exp2f(s[n][3] - sb);
        ra += s[n][0] + s[n][1];
        rb += s[n][2] + s[n][3];
      }
      la = la * ca + ra;
      lb = lb * cb + rb;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= ca;
        o[n][1] *= ca;
        o[n][2] *= cb;
        o[n][3] *= cb;
      }
      // O += P V: P (16 x 64) as four k-steps of 16 keys; V fragments by ldmatrix.trans (rows = keys)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t a0 = h2u(s[2 * kk][0], s[2 * kk][1]), a1 = h2u(s[2 * kk][2], s[2 * kk][3]);
        const uint32_t a2 = h2u(s[2 * kk + 1][0], s[2 * kk + 1][1]), a3 = h2u(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {  // dim tiles 2np, 2np + 1
          // matrices: (keys 16kk + 0..7, dims 16np), (keys +8, dims 16np), (keys 0..7, dims +8), (keys +8, dims +8)
          const int mi = lane >> 3, rr = lane & 7;
          const int key = 16 * kk + (mi & 1) * 8 + rr, dim = 16 * np + (mi >> 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm4t(smem_u32(tv + key * LD + dim), b0, b1, b2, b3);
          mma_16816(o[2 * np][0], o[2 * np][1], o[2 * np][2], o[2 * np][3], a0, a1, a2, a3, b0, b1);
          mma_16816(o[2 * np + 1][0], o[2 * np + 1][1], o[2 * np + 1][2], o[2 * np + 1][3], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
    if (j + 2 < ntiles) load_tile(j + 2, st);
  }
  // row sums over the quad, normalise, store fp16
#pragma unroll
  for (int x = 1; x <= 2; x <<= 1) {
    la += __shfl_xor_sync(0xffffffffu, la, x);
    lb += __shfl_xor_sync(0xffffffffu, lb, x);
  }
  const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
  const int ra = r0 + g, rb = r0 + g + 8;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int c = h * HD + 8 * n + 2 * t;
    if (ra < M) *reinterpret_cast<__half2*>(out + static_cast<size_t>(ra) * H * HD + c) =
        __floats2half2_rn(o[n][0] * ia, o[n][1] * ia);
    if (rb < M) *reinterpret_cast<__half2*>(out + static_cast<size_t>(rb) * H * HD + c) =
        __floats2half2_rn(o[n][2] * ib, o[n][3] * ib);
  }
}

}  // namespace

int launch_prefill_attention(const __half* q16, const __half* kc, const __half* vc, int M, int p0, int H, int KVH,
                             int hd, int cap, int seq, __half* out, cudaStream_t s) {
  if (M < 1 || p0 < 0 || p0 + M > cap || H % KVH) return fail(AGXC_EINVAL, "prefill attention: rows and positions");
  const dim3 grid((M + kPQ - 1) / kPQ, H);
  if (hd == 128) {
    const int smem = 4 * kPK * (128 + 8) * 2;
    prefill_attn_kernel<128><<<grid, 128, smem, s>>>(q16, kc, vc, M, p0, H, KVH, cap, seq, out);
  } else if (hd == 64) {
    const int smem = 4 * kPK * (64 + 8) * 2;
    prefill_attn_kernel<64><<<grid, 128, smem, s>>>(q16, kc, vc, M, p0, H, KVH, cap, seq, out);
  } else {
    return fail(AGXC_EINVAL, "prefill attention: head_dim 64 or 128");
  }
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

int prefill_configure(const agxc_ctx* ctx) {
  (void)ctx;
  AGXC_CUDA(cudaFuncSetAttribute(prefill_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 4 * kPK * (128 + 8) * 2));
  AGXC_CUDA(cudaFuncSetAttribute(prefill_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 4 * kPK * (64 + 8) * 2));
  return 0;
}

}  // namespace agxc
