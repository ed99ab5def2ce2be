// qmm.cu — the batched quantized GEMM of the decode step for B >= 32 activation rows (the reference's tensor-unit
// path, tools/g17qsm.py:1-21 and assemble.layer_ops_qsm agxforge/inference/assemble.py:368-426:
// Y^T = W^T X^T with W dequantised once to fp16), on Blackwell's 5th-generation tensor cores.
//
// One CTA per 128 weight rows (x a K range when K is split): the MMA's M is the weight rows, its N the activation
// rows (B = 32 .. 256), K advances by cg 64-groups per chunk (cg = 1, 2 or 4, the host's choice). Per chunk:
//   * the PRODUCER warp brings the chunk's 8 packed row tiles x cg groups and their scale/bias (two 3-D TMA boxes of
//     the pack) and the activations' cg x 64 columns (2-D TMA boxes of X [B][K] fp16, 128-byte swizzle) into a ring
//     stage;
//   * sixteen DEQUANT warps turn the tiles into fp16 weights and store them straight into TENSOR MEMORY, the MMA's A
//     operand (two fields at a time: (word >> 4j) & 0x000F000F | 0x64006400 is the fp16 pair 1024 + q, HSUB2 takes
//     1024 away exactly, HFMA2 applies the row's scale and bias with one rounding). One thread is one weight row =
//     one TMEM lane (a warp's 32 lanes are its quarter of the 128 rows); a group is 64 fp16 = 32 columns, written
//     with tcgen05.st. The four warps of a lane quarter split a chunk's cg x 64 k: a group each (cg 4), 32 k
//     (cg 2) or 16 k (cg 1); four of them a scheduler hide one another's latencies (the conversion is latency-bound:
//     the MMA waits for the slowest warp of a chunk, and each warp pays two barrier polls and a TMEM store wait a
//     chunk). The fp16 weights never pass through shared memory;
//   * the MMA warp issues 4 cg tcgen05.mma.kind::f16 (M 128, N B, K 16; A from TMEM, B = X from shared memory)
//     accumulating in TMEM, and commits: the commit releases the stage and the TMEM A buffer when the tensor core has
//     read them.
// After the last chunk the first eight dequant warps read the 128 x B fp32 accumulator back with tcgen05.ld (warp w
// reads TMEM lanes 32 (w % 4) ..; the two warps of a lane quarter split the columns) and store Y (fp32 [B][N]; atomically added when K is split over CTAs). Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

constexpr int kM = 128;          // weight rows per CTA (the MMA's M)
constexpr int kDeqWarps = 16;    // four a TMEM lane quarter
constexpr int kEpiWarps = 8;     // the first eight dequant warps also run the epilogue
constexpr int kThreads = 64 + 32 * kDeqWarps;  // warp 0 producer, warp 1 MMA + TMEM, then the dequant warps
constexpr int kTmemCols = 512;   // the whole tensor memory of the SM (one CTA per SM: the ring takes the shared memory)
constexpr int kAcol = 256;       // A buffers from this column (the accumulator takes columns 0 .. B - 1 <= 255)
constexpr int kABufCols = 256;   // nbuf x cg groups x 32 columns

struct QmmParams {
  const uint8_t* w = nullptr;
  const uint8_t* sb = nullptr;
  int N = 0, K = 0, G = 0, bits = 4, sdt = 0;
  int B = 0;                      // activation rows (MMA N), a multiple of 16 in [32, 256]
  int ksplit = 1;                 // K ranges (CTAs) per 128-row tile
  int stages = 4;
  int cg = 1;                     // 64-groups a chunk
  int nbuf = 4;                   // TMEM A buffers (of cg groups each; nbuf x cg <= 8)
  int pdl = 0;                    // started before the predecessor finished: wait for it before X and any output
  float* y = nullptr;             // fp32 [B][ldy]
  int ldy = 0;
  float* part = nullptr;          // ksplit > 1: [ksplit][B][N] fp32, each K range's partial sums
  unsigned* tile_ctr = nullptr;   // ksplit > 1 or push: [N / 128] arrival counts (zero; reset by the last arrival)
  unsigned* err = nullptr;
  QmmPush push;                   // ranks > 0: push finished tiles to every rank (tensor parallel)
};

struct QmmSmem {
  int bars, tmem_slot, stage0, stage_bytes, x_off, w_off, sb_off, total;
};

__host__ __device__ inline QmmSmem qmm_layout(int bits, int B, int stages, int cg) {
  QmmSmem L;
  const int TB = bits == 4 ? 512 : 1024;
  L.bars = 0;                                   // raw_full[S], raw_empty[S], deq_full[D], deq_empty[D], acc_full
  L.tmem_slot = 512;                            // (S <= 16, D <= 8: the barriers fit below)
  L.stage0 = 1024;
  L.x_off = 0;                                  // X: cg atoms of B rows x 128 B (1,024-aligned for the swizzle)
  L.w_off = (cg * B * 128 + 1023) / 1024 * 1024;
  L.sb_off = L.w_off + 8 * cg * TB;             // the boxes land row tile-major: (row tile, group) at (r cg + c)
  L.stage_bytes = (L.sb_off + 8 * cg * 64 + 1023) / 1024 * 1024;
  L.total = L.stage0 + stages * L.stage_bytes;
  return L;
}

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  // UMMA shared-memory descriptor, K-major, 128-byte swizzle: start >> 4 (bits 0-13), leading byte offset 16 B
  // (bits 16-29), stride byte offset 1,024 B between 8-row atoms (bits 32-45), version 1 (bits 46-47), layout
  // SWIZZLE_128B = 2 (bits 61-63)
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

__device__ __forceinline__ uint32_t idesc_f16(int n) {
  // instruction descriptor: fp32 accumulator (bits 4-5 = 1), fp16 A and B (formats 0), both K-major, N >> 3 at bits
  // 17-22, M >> 4 at bits 24-28
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kM >> 4) << 24);
}

__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Two barrier phases polled together (one round trip): true when both are complete.
__device__ __forceinline__ bool mbar_try_wait2(uint64_t* a, unsigned pa, uint64_t* b, unsigned pb) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p, q;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 q, [%3], %4;\n and.pred p, p, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(a)), "r"(pa), "r"(smem_u32(b)), "r"(pb)
      : "memory");
  return ok != 0;
}

// One lane of the (converged) warp: true there, false elsewhere.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile("{\n .reg .pred P;\n elect.sync _|P, 0xffffffff;\n selp.b32 %0, 1, 0, P;\n}\n" : "=r"(pred));
  return pred != 0;
}
// D (TMEM) += A (TMEM) x B (shared-memory descriptor), or D = A x B when accumulate is false.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// AND of a predicate over the 256 epilogue threads (named barrier 1): their decisions stay uniform.
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ uint32_t hsub_1024(uint32_t v) {  // fp16 pair minus 1024 (exact for 1024 + q, q < 1024)
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64006400u));
  return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint16_t to_f16_bits(uint16_t v, int sdt) {
  if (!sdt) return v;
  return __half_as_ushort(__float2half_rn(__uint_as_float(static_cast<uint32_t>(v) << 16)));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// One weight row of one group, lane slots c0 .. c0 + NC - 1 (16 k each): the row's fp16 weights, k in order, into
// NC x 8 TMEM columns of this thread's lane from column taddr. wt / sbt: the row's tile (16 rows x 64 k in the GEMV
// fragment layout: lane slot (r, c) holds rows r and r + 8 at k = 16c ..) and its scale/bias in the stage; r16: the
// row within the tile.
template <int BITS, int NC>
__device__ __forceinline__ void dequant_row(const uint8_t* wt, const uint8_t* sbt, int r16, int c0, int sdt,
                                            uint32_t taddr) {
  const int r = r16 & 7, h = r16 >> 3;
  const uint2 e = *reinterpret_cast<const uint2*>(sbt + r * 8);  // {s[r], s[r+8]}, {b[r], b[r+8]}
  const uint32_t sv = to_f16_bits(static_cast<uint16_t>(h ? e.x >> 16 : e.x & 0xFFFFu), sdt);
  const uint32_t bv = to_f16_bits(static_cast<uint16_t>(h ? e.y >> 16 : e.y & 0xFFFFu), sdt);
  const uint32_t s2 = sv | (sv << 16), b2 = bv | (bv << 16);
  if (NC == 4) {
    // All four lane slots: loaded in an order rotated by r / 2, so the eight rows of a tile (64 bytes apart, i.e.
    // two 16-byte bank groups) read eight different bank groups per step instead of four-way conflicting; two
    // select levels put the words back in slot order.
    const int rr = r >> 1;
    const bool rot1 = rr & 1, rot2 = rr & 2;
    auto unrotate = [&](uint32_t* x) {  // x[c] holds slot (c + rr) & 3 -> x[j] = slot j
      uint32_t y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = rot1 ? x[(j + 3) & 3] : x[j];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = rot2 ? y[(j + 2) & 3] : y[j];
    };
    if (BITS == 4) {
      uint32_t w0[4], w1[4];  // words h and h + 2 of each slot (hi = 0, 1)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wt + (r * 4 + ((c + rr) & 3)) * 16);
        w0[c] = h ? wv.y : wv.x;
        w1[c] = h ? wv.w : wv.z;
      }
      unrotate(w0);
      unrotate(w1);
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        uint32_t o[16];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[8 * u + 2 * j] = hfma2(hsub_1024(((w0[cc + u] >> (4 * j)) & 0x000F000Fu) | 0x64006400u), s2, b2);
            o[8 * u + 2 * j + 1] = hfma2(hsub_1024(((w1[cc + u] >> (4 * j)) & 0x000F000Fu) | 0x64006400u), s2, b2);
          }
        tmem_st16(taddr + 8 * cc, o);
      }
    } else {
      const uint32_t sel = h ? 0x4342u : 0x4140u;
      uint32_t w[8][4];  // [word of the slot][slot]
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int sl = (c + rr) & 3;
        const uint4 lo = *reinterpret_cast<const uint4*>(wt + (r * 4 + sl) * 16);
        const uint4 hi4 = *reinterpret_cast<const uint4*>(wt + 512 + (r * 4 + sl) * 16);
        w[0][c] = lo.x; w[1][c] = lo.y; w[2][c] = lo.z; w[3][c] = lo.w;
        w[4][c] = hi4.x; w[5][c] = hi4.y; w[6][c] = hi4.z; w[7][c] = hi4.w;
      }
#pragma unroll
      for (int wi = 0; wi < 8; ++wi) unrotate(w[wi]);
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        uint32_t o[16];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int wi = 0; wi < 8; ++wi) o[8 * u + wi] = hfma2(hsub_1024(prmt(w[wi][cc + u], 0x64646464u, sel)), s2, b2);
        tmem_st16(taddr + 8 * cc, o);
      }
    }
    return;
  }
  constexpr int U = NC < 2 ? NC : 2;  // lane slots a store
#pragma unroll
  for (int cc = 0; cc < NC; cc += U) {
    uint32_t o[8 * U];  // columns 8 (c0 + cc) .. : the pair (k0, k0 + 1) at column k0 / 2
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + cc + u;
      if (BITS == 4) {
        // word i of the slot: row r + 8 (i & 1), k0 = 16c + 4j + 2 (i >> 1) for the field pair at bits 4j, 16 + 4j
        const uint4 wv = *reinterpret_cast<const uint4*>(wt + (r * 4 + c) * 16);
        const uint32_t w0 = h ? wv.y : wv.x, w1 = h ? wv.w : wv.z;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[8 * u + 2 * j] = hfma2(hsub_1024(((w0 >> (4 * j)) & 0x000F000Fu) | 0x64006400u), s2, b2);
          o[8 * u + 2 * j + 1] = hfma2(hsub_1024(((w1 >> (4 * j)) & 0x000F000Fu) | 0x64006400u), s2, b2);
        }
      } else {
        // word wi: k0 = 16c + 2 wi; bytes 0, 1 row r, bytes 2, 3 row r + 8
        const uint4 lo = *reinterpret_cast<const uint4*>(wt + (r * 4 + c) * 16);
        const uint4 hi4 = *reinterpret_cast<const uint4*>(wt + 512 + (r * 4 + c) * 16);
        const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi4.x, hi4.y, hi4.z, hi4.w};
        const uint32_t sel = h ? 0x4342u : 0x4140u;
#pragma unroll
        for (int wi = 0; wi < 8; ++wi) o[8 * u + wi] = hfma2(hsub_1024(prmt(w[wi], 0x64646464u, sel)), s2, b2);
      }
    }
    if (U == 2) tmem_st16(taddr + 8 * cc, o);
    else tmem_st8(taddr + 8 * cc, o);
  }
}

template <int BITS>
__global__ void __launch_bounds__(kThreads, 1) qmm_kernel(const QmmParams p, const __grid_constant__ CUtensorMap tw,
                                                          const __grid_constant__ CUtensorMap ts,
                                                          const __grid_constant__ CUtensorMap tx) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int TB = BITS == 4 ? 512 : 1024;
  const int cg = p.cg, D = p.nbuf;
  const QmmSmem L = qmm_layout(BITS, p.B, p.stages, cg);
  const int S = p.stages;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* raw_empty = raw_full + S;
  uint64_t* deq_full = raw_empty + S;
  uint64_t* deq_empty = deq_full + D;
  uint64_t* acc_full = deq_empty + D;
  volatile int* dead = reinterpret_cast<volatile int*>(acc_full + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tile = blockIdx.x / p.ksplit, ks = blockIdx.x % p.ksplit;
  const int gk = p.G / p.ksplit;                // groups of this CTA's K range
  const int g0 = ks * gk;
  const int gper = gk / cg;                     // its chunks

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 1);
    }
    for (int d = 0; d < D; ++d) {
      mbar_init(&deq_full[d], kDeqWarps);
      mbar_init(&deq_empty[d], 1);
    }
    mbar_init(acc_full, 1);
    *dead = 0;
    fence_mbar_init();
  }
  if (warp == 1) {  // TMEM: the accumulator (B fp32 columns x 128 lanes) and the A buffers
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (p.pdl && warp != 0) {  // (the producer starts the weights first, then waits)
    pdl_wait();
    pdl_launch_dependents();
  }

  if (warp == 0) {
    // ---- producer: the whole warp walks the chunks (its coordinates stay warp-uniform), one elected lane issues
    const bool leader = elect_one();
    if (leader) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&ts)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
    }
    const unsigned bytes = static_cast<unsigned>(cg * (p.B * 128 + 8 * TB + 8 * 64));
    auto weights = [&](int i, uint8_t* st, uint64_t* bar) {
      tma_3d(st + L.w_off, &tw, 0, g0 + i * cg, tile * 8, bar);
      tma_3d(st + L.sb_off, &ts, 0, g0 + i * cg, tile * 8, bar);
    };
    auto acts = [&](int i, uint8_t* st, uint64_t* bar) {
      for (int c = 0; c < cg; ++c)  // one 128-byte-swizzled atom of B rows x 64 columns each
        tma_2d(st + L.x_off + c * p.B * 128, &tx, (g0 + i * cg + c) * 64, 0, bar);
    };
    // under programmatic dependent launch: the first stages' weights (independent of the predecessor) at once, then
    // the wait, then their activations
    const int pre = p.pdl ? min(S, gper) : 0;
    if (leader)
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&raw_full[i], bytes);
        weights(i, smem + L.stage0 + i * L.stage_bytes, &raw_full[i]);
      }
    if (p.pdl) {
      pdl_wait();
      pdl_launch_dependents();
    }
    if (leader)
      for (int i = 0; i < pre; ++i) acts(i, smem + L.stage0 + i * L.stage_bytes, &raw_full[i]);
    int issued = pre;
    bool gave_up = false;
    for (int i = pre, s = pre % S, eph = (pre / S + 1) & 1; i < gper; ++i, ++issued) {
      // stage s was last filled for chunk i - S: wait for the commit of its MMAs (phase eph of raw_empty)
      const bool ok = !*dead && (i < S || mbar_wait_quiet(&raw_empty[s], static_cast<unsigned>(eph), p.err));
      if (!__all_sync(0xffffffffu, ok)) {
        gave_up = true;
        break;
      }
      uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
      if (leader) {
        mbar_arrive_expect_tx(&raw_full[s], bytes);
        weights(i, st, &raw_full[s]);
        acts(i, st, &raw_full[s]);
      }
      __syncwarp();
      if (++s == S) { s = 0; eph ^= 1; }
    }
    if (gave_up || *dead) {
      *dead = 1;
      if (leader)  // a wait gave up: no copy of this CTA may land after it leaves (bounded)
        for (int i = issued > S ? issued - S : 0; i < issued; ++i)
          mbar_wait_bounded(&raw_full[i % S], (i / S) & 1, nullptr, 100000000ull);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: the whole warp walks the chunks (its TMEM addresses and descriptors stay warp-uniform), one
    // elected lane issues each chunk's MMAs and commits. The B descriptor of (stage s, group c, k step) is stage 0's
    // plus the byte offset / 16 (the start-address field; smem addresses stay below 2^18, so no carry leaves it).
    const uint32_t idesc = idesc_f16(p.B);
    const uint64_t bd0 = desc_sw128(smem_u32(smem + L.stage0 + L.x_off));
    const uint64_t bd_stage = static_cast<uint64_t>(L.stage_bytes >> 4), bd_atom = static_cast<uint64_t>(p.B * 8);
    const bool leader = elect_one();
    for (int i = 0, d = 0, dph = 0, s = 0; i < gper; ++i) {
      const bool ok = !*dead && mbar_wait_quiet(&deq_full[d], static_cast<unsigned>(dph), p.err);
      if (!__all_sync(0xffffffffu, ok)) {
        *dead = 1;
        break;
      }
      tc_fence_after();
      if (leader) {
        const uint64_t bs = bd0 + static_cast<uint64_t>(s) * bd_stage;
        const uint32_t as = tmem + kAcol + d * cg * 32;  // the chunk's groups: 32 columns of fp16 pairs each
        for (int c = 0; c < cg; ++c) {
#pragma unroll
          for (int k = 0; k < 4; ++k)  // four K = 16 steps: A +8 columns, B +32 bytes in the swizzled 128-byte rows
            tc_mma(tmem, as + c * 32 + 8 * k, bs + c * bd_atom + 2 * k, idesc, (i | c | k) != 0);
        }
        tc_commit(&raw_empty[s]);  // the stage (weights read, X read) is free once these MMAs are done
        tc_commit(&deq_empty[d]);
      }
      __syncwarp();
      if (++s == S) s = 0;
      if (++d == D) { d = 0; dph ^= 1; }
    }
    if (leader) tc_commit(acc_full);  // every MMA of the CTA done: the accumulator is final
    __syncwarp();
  } else {
    // ---- dequant warps, then the epilogue
    const int dw = warp - 2;  // 0 .. kDeqWarps - 1
    const int q4 = warp & 3;  // this warp's TMEM lane quarter: CTA rows 32 q4 .. + 31, one a thread
    const int rt = (32 * q4 + lane) >> 4, r16 = lane & 15;
    // the warp's slice of the chunk (si = 0..3 within its quarter): cg 2: group si / 2, k 32 (si % 2) ..; cg 1: k 16 si
    const int si = dw >> 2;
    const int gc = cg == 4 ? si : cg == 2 ? si >> 1 : 0, cslot = cg == 4 ? 0 : cg == 2 ? 2 * (si & 1) : si;
    const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    for (int i = 0, s = 0, sph = 0, d = 0, dph = 0; i < gper; ++i) {
      // the stage's copies landed and the A buffer's previous MMAs done: both polled in one round trip first
      bool ok2 = !*dead && (i < D ? mbar_try_wait(&raw_full[s], static_cast<unsigned>(sph))
                                  : mbar_try_wait2(&raw_full[s], static_cast<unsigned>(sph), &deq_empty[d],
                                                   static_cast<unsigned>(dph ^ 1)));
      if (!ok2) {
        const bool ok1 = !*dead && mbar_wait_quiet(&raw_full[s], static_cast<unsigned>(sph), p.err);
        ok2 = ok1 && (i < D || mbar_wait_quiet(&deq_empty[d], static_cast<unsigned>(dph ^ 1), p.err));
      }
      if (!__all_sync(0xffffffffu, ok2)) {  // the warp leaves together
        *dead = 1;
        break;
      }
      const uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
      // (row tile rt, group gc) of the chunk sits at (rt cg + gc) in the stage's boxes
      const uint8_t* wt = st + L.w_off + (rt * cg + gc) * TB;
      const uint8_t* sbt = st + L.sb_off + (rt * cg + gc) * 64;
      const uint32_t ta = tlane + kAcol + (d * cg + gc) * 32 + 8 * cslot;
      if (cg == 4) dequant_row<BITS, 4>(wt, sbt, r16, 0, p.sdt, ta);
      else if (cg == 2) dequant_row<BITS, 2>(wt, sbt, r16, cslot, p.sdt, ta);
      else dequant_row<BITS, 1>(wt, sbt, r16, cslot, p.sdt, ta);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();    // the MMA warp reads these columns after its barrier wait
      __syncwarp();
      if (lane == 0) mbar_arrive1(&deq_full[d]);
      if (++s == S) { s = 0; sph ^= 1; }
      if (++d == D) { d = 0; dph ^= 1; }
    }
    // epilogue (the first eight dequant warps): TMEM lanes 32 (warp % 4) .. + 31 = weight rows; columns =
    // activation rows
    if (dw < kEpiWarps) {
      const bool ok = __all_sync(0xffffffffu, !*dead && mbar_wait_quiet(acc_full, 0, p.err));  // warp-uniform:
      tc_fence_after();                                                                        // tcgen05.ld is aligned
      if (ok) {
        const int row = tile * kM + 32 * q4 + lane;
        const uint32_t base = tmem + (static_cast<uint32_t>(32 * q4) << 16);
        const int half = (p.B / 16 + 1) / 2 * 16;  // columns of the first warp of the quarter
        const int cb = dw < 4 ? 0 : half, ce = dw < 4 ? half : p.B;
        for (int c0 = cb; c0 < ce; c0 += 16) {
          uint32_t v[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15}, [%16];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
              : "r"(base + static_cast<uint32_t>(c0)));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (row < p.N) {
            // one K range: straight into Y; several: this range's partial sums into its own slice
            float* dst = p.ksplit > 1 ? p.part + static_cast<size_t>(ks) * p.B * p.N : p.y;
            const int ld = p.ksplit > 1 ? p.N : p.ldy;
  #pragma unroll
            for (int j = 0; j < 16; ++j) dst[static_cast<size_t>(c0 + j) * ld + row] = __uint_as_float(v[j]);
          }
        }
      }
      const bool push = p.push.ranks > 0;
      if ((p.ksplit > 1 && p.y) || push) {  // (y NULL: the consumers add the K ranges themselves)
        // the tile's last K-range CTA sums the ranges in order (the same result every run: no atomics on the data)
        // and, under tensor parallelism, sends the finished B x 128 block of Y to the ranks
        __threadfence();                               // this CTA's partial sums are visible at L2
        const bool all_ok = epi_all(ok);
        volatile int* s_last = dead + 1;
        if (all_ok && dw == 0 && lane == 0) {
          const unsigned prev = atomicAdd(p.tile_ctr + tile, 1u);
          *s_last = prev == static_cast<unsigned>(p.ksplit - 1);
          if (*s_last) p.tile_ctr[tile] = 0;           // every K-range CTA of the tile has arrived
        }
        epi_sync();
        if (all_ok && *s_last) {
          __threadfence();                             // the other CTAs' partials, read below from L2
          // to_owner: the tile's rows go to the one rank owning them (reduce-scatter; d / ranks consecutive rows a
          // rank); else to every rank (each then reduces all rows itself)
          const int r0 = push && p.push.to_owner ? tile / p.push.tiles_per_rank : 0;
          const int r1 = !push ? 0 : p.push.to_owner ? r0 + 1 : p.push.ranks;
          const int et = dw * 32 + lane;               // 0 .. 255
          const size_t slice = static_cast<size_t>(p.B) * p.N;
          for (int i = et; i < p.B * (kM / 4); i += 256) {
            const int b = i / (kM / 4), n = tile * kM + (i % (kM / 4)) * 4;
            float4 v4;
            if (p.ksplit > 1) {
              const float* src = p.part + static_cast<size_t>(b) * p.N + n;
              v4 = __ldcg(reinterpret_cast<const float4*>(src));
              for (int q = 1; q < p.ksplit; ++q) {
                const float4 t4 = __ldcg(reinterpret_cast<const float4*>(src + q * slice));
                v4.x += t4.x; v4.y += t4.y; v4.z += t4.z; v4.w += t4.w;
              }
              *reinterpret_cast<float4*>(p.y + static_cast<size_t>(b) * p.ldy + n) = v4;
            } else {
              v4 = __ldcg(reinterpret_cast<const float4*>(p.y + static_cast<size_t>(b) * p.ldy + n));
            }
            for (int r = r0; r < r1; ++r)
              *reinterpret_cast<float4*>(p.push.slot[r] + static_cast<size_t>(b) * p.N + n) = v4;
          }
          if (push) {
            __threadfence_system();                    // the stores reach their ranks before the counters move
            epi_sync();
            if (et == 0)
              for (int r = r0; r < r1; ++r)
                asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(p.push.flag[r]) : "memory");
          }
        }
      }
    }
  }
  // every role is done (the tensor core too: acc_full waited, or the error path below): free TMEM
  if (*dead && tid == 64) mbar_wait_bounded(acc_full, 0, nullptr, 100000000ull);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <int BITS>
int qmm_allow(int optin) {
  cudaFuncAttributes fa;
  AGXC_CUDA(cudaFuncGetAttributes(&fa, qmm_kernel<BITS>));
  AGXC_CUDA(cudaFuncSetAttribute(qmm_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - static_cast<int>(fa.sharedSizeBytes)));
  return 0;
}

}  // namespace

int qmm_configure(const agxc_ctx* ctx) {
  int rc;
  if ((rc = qmm_allow<4>(ctx->max_smem_optin)) || (rc = qmm_allow<8>(ctx->max_smem_optin))) return rc;
  return 0;
}

// Y [B][ldy] fp32 = X [B][K] fp16 x W^T for a pack W [N][K]: 128-row tiles, the K range split over ksplit CTAs when
// the tiles alone would leave SMs idle (then Y must hold zeros: the CTAs add into it).
int launch_qmm(const agxc_ctx* ctx, const agxc_pack* pk, const void* x, int B, float* y, int ldy, int ksplit,
               cudaStream_t s, const QmmPush* push, float* part, unsigned* tile_ctr, int pdl) {
  if (B < 32 || B > 256 || B % 16) return fail(AGXC_EINVAL, "qmm: 32 to 256 activation rows, a multiple of 16");
  if (pk->n % kM) return fail(AGXC_EINVAL, "qmm: N must be a multiple of 128");
  if (ldy < pk->n) return fail(AGXC_EINVAL, "qmm: ldy < N");
  const int G = pk->k / 64;
  if (ksplit < 1 || G % ksplit) return fail(AGXC_EINVAL, "qmm: ksplit must divide K/64");
  QmmParams p;
  p.w = pk->tiles; p.sb = pk->sb; p.N = pk->n; p.K = pk->k; p.G = G; p.bits = pk->bits; p.sdt = pk->sdt;
  p.B = B; p.ksplit = ksplit; p.y = y; p.ldy = ldy; p.err = ctx->err_dev;
  p.part = part;
  p.tile_ctr = tile_ctr;
  if ((ksplit > 1 && (!part || (y && !tile_ctr))) || (push && (!tile_ctr || !y)) || (!y && ksplit < 2))
    return fail(AGXC_EINVAL, "qmm: split K and the peer push need the partial-sum scratch, the tile counters and Y");
  if (push) {
    if (push->ranks < 1 || push->ranks > 8 || push->tiles_per_rank < 1 ||
        push->tiles_per_rank * push->ranks != pk->n / kM)
      return fail(AGXC_EINVAL, "qmm: push to 1..8 ranks owning equal numbers of 128-row tiles");
    p.push = *push;
  }
  // the chunk: 4 groups where the K range divides and four stages of them fit (one whole group a dequant warp: its two
  // barrier polls, about 200 cycles each, and its TMEM store latency are paid once for four groups), else 2, else 1;
  // the TMEM A buffers hold 8 groups either way; as many stages as fit (at most 16: a stage cycles through the copy,
  // the dequant and the MMA's completion before it is refilled, so small stages want many)
  const int gk = G / ksplit;
  auto stages_for = [&](int cg) {
    int st = 16;
    while (st > 2 && qmm_layout(pk->bits, B, st, cg).total + 1024 > ctx->max_smem_optin - 2048) --st;
    return qmm_layout(pk->bits, B, st, cg).total + 1024 > ctx->max_smem_optin - 2048 ? 0 : st;
  };
  p.cg = gk % 4 == 0 && stages_for(4) >= 4 ? 4 : gk % 2 == 0 ? 2 : 1;
  p.nbuf = kABufCols / 32 / p.cg;
  p.stages = stages_for(p.cg);
  if (!p.stages) return fail(AGXC_EINVAL, "qmm: the batch does not fit the shared memory");
  const int smem = qmm_layout(pk->bits, B, p.stages, p.cg).total + 1024;
  // maps: the pack's tiles and scale/bias as boxes of cg groups x 8 row tiles; X [B][K] fp16 as 64 x B boxes
  QmvPlan plan;
  plan.CG = p.cg;
  plan.RW = 8;
  CUtensorMap tw, ts, tx;
  if (int rc = qmv_maps(plan, pk->tiles, pk->sb, pk->n, pk->k, pk->bits, &tw, &ts)) return rc;
  if (int rc = encode_act_map(&tx, x, B, pk->k)) return rc;
  const int grid = (pk->n / kM) * ksplit;
  p.pdl = pdl;
  if (pk->bits == 4) return launch_ex(qmm_kernel<4>, dim3(grid), dim3(kThreads), smem, s, pdl, p, tw, ts, tx);
  return launch_ex(qmm_kernel<8>, dim3(grid), dim3(kThreads), smem, s, pdl, p, tw, ts, tx);
}

}  // namespace agxc
