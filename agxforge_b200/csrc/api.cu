// api.cu — small device entry points: two behind the reference's per-kernel Python functions that the decode step
// itself fuses elsewhere, and the tensor-parallel reduce on its own (for its bounded-wait check):
//   agxc_rope_append_dev   RoPE + q scale + KV append on one token's fp32 qkv row in the reference's logical order
//                          [q heads | k heads | v heads] x head_dim (attention.py:1309-1323 attn_rope_reference); in
//                          the decode step this is the qkv GEMV's epilogue
//   agxc_argmax_dev        the first maximum of an fp32 row (argmax.py:287-288 argmax_reference); in the decode step
//                          this is the vocabulary GEMV's epilogue
//   agxc_tp_reduce_dev     the tensor-parallel all-reduce's local reduction with its bounded flag wait
#include <cfloat>

#include "common.cuh"
#include "internal.h"

namespace agxc {
namespace {

// One thread per RoPE pair (i, i + hd/2) of every q and k head, plus one per v element pair. The rotation is two
// products and one sum per output, each rounded (no contraction), as numerics.rope_rotate computes it.
__global__ void rope_append_one(const float* __restrict__ qkv, int H, int KVH, int hd, int cap, int pos,
                                const float* __restrict__ cos_row, const float* __restrict__ sin_row, float qscale,
                                __half* __restrict__ q16, __half* __restrict__ kc, __half* __restrict__ vc) {
  const int half = hd / 2;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int pairs = (H + 2 * KVH) * half;
  if (t >= pairs) return;
  const int head = t / half, i = t % half;
  const float x1 = qkv[head * hd + i], x2 = qkv[head * hd + half + i];
  if (head >= H + KVH) {
    __half* v = vc + (static_cast<size_t>(head - H - KVH) * cap + pos) * hd;
    v[i] = __float2half_rn(x1);
    v[half + i] = __float2half_rn(x2);
    return;
  }
  const float c = cos_row[i], s = sin_row[i];
  const float o1 = __fadd_rn(__fmul_rn(x1, c), -__fmul_rn(x2, s));
  const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  if (head < H) {
    q16[head * hd + i] = __float2half_rn(__fmul_rn(o1, qscale));
    q16[head * hd + half + i] = __float2half_rn(__fmul_rn(o2, qscale));
  } else {
    __half* k = kc + (static_cast<size_t>(head - H) * cap + pos) * hd;
    k[i] = __float2half_rn(o1);
    k[half + i] = __float2half_rn(o2);
  }
}

// One CTA: each thread scans a strided slice keeping its first maximum, then a (value, index) reduction in which the
// larger value wins and equal values keep the smaller index: the first maximum of the row.
constexpr int kArgThreads = 1024;
__global__ void __launch_bounds__(kArgThreads) argmax_one(const float* __restrict__ x, int n, int32_t* out) {
  float bv = -FLT_MAX;
  int bi = n;
  for (int i = threadIdx.x; i < n; i += kArgThreads) {
    const float v = x[i];
    if (v > bv || (bi == n)) { bv = v; bi = i; }
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
    bv = sv[lane];
    bi = si[lane];
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) *out = bi;
  }
}

}  // namespace
}  // namespace agxc

using namespace agxc;

extern "C" {

AGXC_API int agxc_rope_append_dev(agxc_ctx* ctx, const float* qkv_dev, int heads, int kv_heads, int head_dim, int cap,
                                  int pos, const float* cos_dev, const float* sin_dev, float qscale,
                                  uint16_t* q16_dev, uint16_t* kcache_dev, uint16_t* vcache_dev, void* stream) {
  if (!ctx) return fail(AGXC_EINVAL, "rope_append: null context");
  if (!qkv_dev || !cos_dev || !sin_dev || !q16_dev || !kcache_dev || !vcache_dev)
    return fail(AGXC_EINVAL, "rope_append: null buffer");
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads) return fail(AGXC_EINVAL, "rope_append: heads a multiple of kv_heads");
  if (head_dim <= 0 || head_dim % 2) return fail(AGXC_EINVAL, "rope_append: an even head_dim");
  if (cap <= 0 || pos < 0) return fail(AGXC_EINVAL, "rope_append: cap > 0 and pos >= 0");
  if (pos > cap - 1) pos = cap - 1;  // the reference clamps the append row (attention.py:1313)
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const int pairs = (heads + 2 * kv_heads) * head_dim / 2;
  rope_append_one<<<(pairs + 255) / 256, 256, 0, s>>>(qkv_dev, heads, kv_heads, head_dim, cap, pos, cos_dev, sin_dev,
                                                       qscale, reinterpret_cast<__half*>(q16_dev),
                                                       reinterpret_cast<__half*>(kcache_dev),
                                                       reinterpret_cast<__half*>(vcache_dev));
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

AGXC_API int agxc_tp_reduce_dev(agxc_ctx* ctx, const float* recv_dev, int ranks, int rank, const unsigned* flag_dev,
                                const unsigned* epoch_dev, int uses_per_step, int use_in_step, int tiles_per_rank,
                                const uint16_t* res16_dev, const float* res32_dev, float* out32_dev,
                                uint16_t* out16_dev, int d, int batch, int wait_us, void* stream) {
  if (!ctx || !recv_dev || !flag_dev || !epoch_dev) return fail(AGXC_EINVAL, "tp_reduce: null argument");
  if (ranks < 1 || ranks > 8 || rank < 0 || rank >= ranks || d <= 0 || batch <= 0 || wait_us < 0)
    return fail(AGXC_EINVAL, "tp_reduce: 1..8 ranks, 0 <= rank < ranks, positive d and batch, wait_us >= 0");
  if ((res16_dev == nullptr) == (res32_dev == nullptr))
    return fail(AGXC_EINVAL, "tp_reduce: exactly one residual (fp16 for o_proj, fp32 for down)");
  if ((res16_dev && !out32_dev) || (res32_dev && !out16_dev)) return fail(AGXC_EINVAL, "tp_reduce: null output");
  TpGather g;
  g.out32[rank] = out32_dev;
  g.out16[rank] = reinterpret_cast<__half*>(out16_dev);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return launch_tp_reduce(recv_dev, ranks, rank, flag_dev, epoch_dev, uses_per_step, use_in_step, tiles_per_rank,
                          reinterpret_cast<const __half*>(res16_dev), res32_dev, g, d, batch, ctx->err_dev, s, false,
                          static_cast<uint64_t>(wait_us) * 1000ull);
}

AGXC_API int agxc_argmax_dev(agxc_ctx* ctx, const float* x_dev, int n, int32_t* out_dev, void* stream) {
  if (!ctx) return fail(AGXC_EINVAL, "argmax: null context");
  if (!x_dev || !out_dev) return fail(AGXC_EINVAL, "argmax: null buffer");
  if (n <= 0) return fail(AGXC_EINVAL, "argmax: n > 0");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  argmax_one<<<1, kArgThreads, 0, s>>>(x_dev, n, out_dev);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

}  // extern "C"
