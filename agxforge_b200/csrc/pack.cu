// pack.cu — affine group-64 weight packs on the device.
//
//   quantize   fp32 [N][K] -> the reference format (packed uint32 low field first, 16-bit scale and bias per group):
//              the arithmetic of agxforge/kernels/qmv.py:1854-1871, each step an IEEE fp32 operation rounded to
//              nearest even (subtract, divide, rint), so the result is the reference's bit for bit.
//   relayout   reference format -> the B200 tile layout the GEMV streams (16 rows x 64 k per tile; each lane's
//              fields for its m16n8k16 A fragments contiguous, 16 B per lane; scale/bias beside each tile).
//   unpack     tile layout -> fields uint8 [N][K]       (agxforge/inference/assemble.py:834-840)
//   dequant    tile layout -> fp32 w = fma(q, s, b)     (qmv.py:1699-1750: one rounding)
#include "common.cuh"
#include "internal.h"

namespace agxc {

__device__ __forceinline__ uint16_t to16(float x, int sdt) {
  if (sdt) {  // bf16, round to nearest even on the bit pattern (qmv.py:1874-1876)
    uint32_t u = __float_as_uint(x);
    return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
  }
  return __half_as_ushort(__float2half_rn(x));
}

__global__ void quantize_kernel(const float* __restrict__ w, int N, int K, int bits, int sdt,
                                uint32_t* __restrict__ packed, uint16_t* __restrict__ s16,
                                uint16_t* __restrict__ b16) {
  const int G = K / 64;
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (gid >= static_cast<long long>(N) * G) return;
  const int n = static_cast<int>(gid / G), g = static_cast<int>(gid % G);
  const float4* src = reinterpret_cast<const float4*>(w + static_cast<size_t>(n) * K + g * 64);
  float v[64];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float4 t = src[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float lo = v[0], hi = v[0];
#pragma unroll
  for (int i = 1; i < 64; ++i) { lo = fminf(lo, v[i]); hi = fmaxf(hi, v[i]); }
  const float levels = static_cast<float>((1 << bits) - 1);
  const float scale = hi > lo ? __fdiv_rn(__fsub_rn(hi, lo), levels) : 1.0f;
  const uint16_t sq = to16(scale, sdt), bq = to16(lo, sdt);
  s16[static_cast<size_t>(n) * G + g] = sq;
  b16[static_cast<size_t>(n) * G + g] = bq;
  const float s32 = scale_to_f32(sq, sdt), b32 = scale_to_f32(bq, sdt);
  const int per = 32 / bits;
  uint32_t* dst = packed + static_cast<size_t>(n) * (K / per) + g * (64 / per);
  for (int wd = 0; wd < 64 / per; ++wd) {
    uint32_t word = 0;
    for (int e = 0; e < per; ++e) {
      float qf = rintf(__fdiv_rn(__fsub_rn(v[wd * per + e], b32), s32));
      if (!isfinite(qf)) qf = 0.f;
      qf = fminf(fmaxf(qf, 0.f), levels);
      word |= static_cast<uint32_t>(qf) << (bits * e);
    }
    dst[wd] = word;
  }
}

int launch_quantize(const float* w, int N, int K, int bits, int sdt, uint32_t* packed, uint16_t* s16, uint16_t* b16,
                    cudaStream_t s) {
  const long long groups = static_cast<long long>(N) * (K / 64);
  const int threads = 128;
  quantize_kernel<<<static_cast<unsigned>((groups + threads - 1) / threads), threads, 0, s>>>(w, N, K, bits, sdt,
                                                                                             packed, s16, b16);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

__device__ __forceinline__ uint32_t field_of(const uint32_t* __restrict__ packed, int K, int bits, int row, int k) {
  const int per = 32 / bits;
  const uint32_t word = packed[static_cast<size_t>(row) * (K / per) + k / per];
  return (word >> (bits * (k % per))) & ((1u << bits) - 1u);
}

// The source row of physical row `prow` (identity, or the RoPE-pair placement within heads of rope_hd rows).
__device__ __forceinline__ int src_row(int prow, int rope_hd) {
  if (!rope_hd) return prow;
  const int head = prow / rope_hd, within = prow % rope_hd;
  const int t = within / 16, r16 = within % 16;
  return head * rope_hd + (r16 < 8 ? 8 * t + r16 : rope_hd / 2 + 8 * t + (r16 - 8));
}

// One thread per 32-bit word of the destination tiles.
__global__ void relayout_kernel(const uint32_t* __restrict__ packed, int n_src, int K, int bits,
                                uint8_t* __restrict__ tiles, int rt_stride, int rt_offset, int rope_hd) {
  const int G = K / 64;
  const int words_per_tile = bits == 4 ? 128 : 256;
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(n_src / 16) * G * words_per_tile;
  if (gid >= total) return;
  const int widx = static_cast<int>(gid % words_per_tile);
  const long long tile = gid / words_per_tile;
  const int g = static_cast<int>(tile % G);
  const int rt = static_cast<int>(tile / G);
  const int rt_dst = rt * rt_stride + rt_offset;
  uint32_t word = 0;
  if (bits == 4) {
    const int lane = widx >> 2, i = widx & 3;
    const int r = lane >> 2, c = lane & 3;
    const int row = src_row(rt * 16 + r + ((i & 1) ? 8 : 0), rope_hd);
    const int hi = i >> 1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k0 = 64 * g + 16 * c + 4 * j + 2 * hi;
      word |= field_of(packed, K, 4, row, k0) << (4 * j);
      word |= field_of(packed, K, 4, row, k0 + 1) << (4 * (j + 4));
    }
  } else {
    const int h = widx >> 7, lane = (widx & 127) >> 2, m = widx & 3;
    const int wi = 4 * h + m, j = wi >> 1, hi = wi & 1;
    const int r = lane >> 2, c = lane & 3;
    const int k0 = 64 * g + 16 * c + 4 * j + 2 * hi;
    const int row0 = src_row(rt * 16 + r, rope_hd), row1 = src_row(rt * 16 + r + 8, rope_hd);
    word = field_of(packed, K, 8, row0, k0) | (field_of(packed, K, 8, row0, k0 + 1) << 8) |
           (field_of(packed, K, 8, row1, k0) << 16) | (field_of(packed, K, 8, row1, k0 + 1) << 24);
  }
  const size_t tb = bits == 4 ? 512 : 1024;
  uint32_t* dst = reinterpret_cast<uint32_t*>(tiles + (static_cast<size_t>(rt_dst) * G + g) * tb);
  dst[widx] = word;
}

// One thread per (tile, r): the 8-byte scale/bias entry {s[r], s[r+8], b[r], b[r+8]}.
__global__ void relayout_sb_kernel(const uint16_t* __restrict__ s16, const uint16_t* __restrict__ b16, int n_src,
                                   int K, uint8_t* __restrict__ sb, int rt_stride, int rt_offset, int rope_hd) {
  const int G = K / 64;
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(n_src / 16) * G * 8;
  if (gid >= total) return;
  const int r = static_cast<int>(gid % 8);
  const long long tile = gid / 8;
  const int g = static_cast<int>(tile % G);
  const int rt = static_cast<int>(tile / G);
  const int rt_dst = rt * rt_stride + rt_offset;
  const size_t r0 = src_row(rt * 16 + r, rope_hd), r1 = src_row(rt * 16 + r + 8, rope_hd);
  ushort4 e;
  e.x = s16[r0 * G + g];
  e.y = s16[r1 * G + g];
  e.z = b16[r0 * G + g];
  e.w = b16[r1 * G + g];
  reinterpret_cast<ushort4*>(sb + (static_cast<size_t>(rt_dst) * G + g) * 64)[r] = e;
}

int launch_relayout(const uint32_t* packed, const uint16_t* s16, const uint16_t* b16, int n_src, int K, int bits,
                    uint8_t* tiles, uint8_t* sb, int rt_stride, int rt_offset, cudaStream_t s, int rope_hd) {
  if (rope_hd && (rope_hd % 16 || n_src % rope_hd)) return fail(AGXC_EINVAL, "relayout: rows must be whole heads");
  const int G = K / 64;
  const long long words = static_cast<long long>(n_src / 16) * G * (bits == 4 ? 128 : 256);
  const int threads = 256;
  relayout_kernel<<<static_cast<unsigned>((words + threads - 1) / threads), threads, 0, s>>>(
      packed, n_src, K, bits, tiles, rt_stride, rt_offset, rope_hd);
  AGXC_CUDA(cudaGetLastError());
  const long long ents = static_cast<long long>(n_src / 16) * G * 8;
  relayout_sb_kernel<<<static_cast<unsigned>((ents + threads - 1) / threads), threads, 0, s>>>(
      s16, b16, n_src, K, sb, rt_stride, rt_offset, rope_hd);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

// Where logical element (n, k) of a pack lives in the tile layout.
struct TileLoc {
  size_t word;   // 32-bit word index in the tiles array
  int shift;     // bit offset of the field inside the word
  size_t sbent;  // ushort index of the entry's scale (bias = +2)
};

__device__ __forceinline__ TileLoc locate(int n, int k, int N, int K, int bits, int gateup) {
  const int G = K / 64;
  int rt;
  if (gateup) {
    const int F = N / 2;
    rt = n < F ? 2 * (n / 16) : 2 * ((n - F) / 16) + 1;
  } else {
    rt = n / 16;
  }
  const int r16 = n % 16, r = r16 & 7, upper = r16 >> 3;
  const int g = k / 64, kk = k % 64;
  const int c = kk >> 4, rem = kk & 15, j = rem >> 2, t = rem & 3, hi = t >> 1, e = t & 1;
  const int lane = 4 * r + c;
  const size_t tile = static_cast<size_t>(rt) * G + g;
  TileLoc L;
  if (bits == 4) {
    const int i = upper + 2 * hi;
    L.word = tile * 128 + lane * 4 + i;
    L.shift = 4 * (j + 4 * e);
  } else {
    const int wi = 2 * j + hi, h = wi >> 2, m = wi & 3;
    L.word = tile * 256 + h * 128 + lane * 4 + m;
    L.shift = 8 * (2 * upper + e);
  }
  L.sbent = tile * 32 + r * 4 + upper;
  return L;
}

__global__ void unpack_kernel(const uint32_t* __restrict__ tiles, int N, int K, int bits, int gateup,
                              uint8_t* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (gid >= static_cast<long long>(N) * K) return;
  const int n = static_cast<int>(gid / K), k = static_cast<int>(gid % K);
  const TileLoc L = locate(n, k, N, K, bits, gateup);
  out[gid] = static_cast<uint8_t>((tiles[L.word] >> L.shift) & ((1u << bits) - 1u));
}

__global__ void dequant_kernel(const uint32_t* __restrict__ tiles, const uint16_t* __restrict__ sb, int N, int K,
                               int bits, int sdt, int gateup, float* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (gid >= static_cast<long long>(N) * K) return;
  const int n = static_cast<int>(gid / K), k = static_cast<int>(gid % K);
  const TileLoc L = locate(n, k, N, K, bits, gateup);
  const float q = static_cast<float>((tiles[L.word] >> L.shift) & ((1u << bits) - 1u));
  const float s = scale_to_f32(sb[L.sbent], sdt);
  const float b = scale_to_f32(sb[L.sbent + 2], sdt);
  out[gid] = __fmaf_rn(q, s, b);
}

int launch_unpack(const agxc_pack* p, uint8_t* fields, cudaStream_t s) {
  const long long n = static_cast<long long>(p->n) * p->k;
  unpack_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const uint32_t*>(p->tiles), p->n, p->k, p->bits, p->gateup, fields);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

int launch_dequant(const agxc_pack* p, float* w, cudaStream_t s) {
  const long long n = static_cast<long long>(p->n) * p->k;
  dequant_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const uint32_t*>(p->tiles), reinterpret_cast<const uint16_t*>(p->sb), p->n, p->k, p->bits,
      p->sdt, p->gateup, w);
  AGXC_CUDA(cudaGetLastError());
  return 0;
}

}  // namespace agxc
