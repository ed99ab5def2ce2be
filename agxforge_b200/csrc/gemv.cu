// gemv.cu — host side of the GEMV family: the launch planner, the TMA tensor maps of a pack, and the dispatch to
// the kernels instantiated per (bits, activation rows) in gemv_q{4,8}_b{1,2,4,8}.cu (device code: gemv_impl.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace agxc {

#define AGXC_GEMV_DECLARE(BITS, NBT)                                                                   \
  int qmv_dispatch_##BITS##_##NBT(const agxc_ctx* ctx, const QmvParams& p, const QmvPlan& plan, int epi, \
                                  const CUtensorMap& tw, const CUtensorMap& ts, cudaStream_t s);       \
  int qmv_configure_##BITS##_##NBT(int smem);
AGXC_GEMV_DECLARE(4, 1)
AGXC_GEMV_DECLARE(4, 2)
AGXC_GEMV_DECLARE(4, 4)
AGXC_GEMV_DECLARE(4, 8)
AGXC_GEMV_DECLARE(8, 1)
AGXC_GEMV_DECLARE(8, 2)
AGXC_GEMV_DECLARE(8, 4)
AGXC_GEMV_DECLARE(8, 8)

namespace {

constexpr int kConsumerWarps = 16;  // must match gemv_impl.cuh
constexpr int kMaxStages = 8;

int nb_tmpl(int nb) { return nb == 1 ? 1 : nb == 2 ? 2 : nb <= 4 ? 4 : 8; }

// the same arithmetic as gemv::smem_layout (device side)
size_t smem_total(int bits, int nbt, int RW, int CG, int GC, int stages) {
  const int TB = tile_bytes(bits);
  const size_t stage_bytes = (static_cast<size_t>(RW) * CG * (TB + 64) + 127) / 128 * 128;
  size_t off = 256 + stages * stage_bytes;
  off += (static_cast<size_t>(nbt) * (GC * 64 + 8) * 2 + 127) / 128 * 128;
  off += static_cast<size_t>(GC) * 8 * 4;
  off += static_cast<size_t>(kConsumerWarps) * 16 * nbt * 4;
  off += 3 * static_cast<size_t>(RW) * 16 * nbt * 4;
  return off + 1024;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int encode_fn() {
  if (g_encode) return 0;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  AGXC_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || !fn) return fail(AGXC_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return 0;
}

// A 3-D map over an array [rows][groups][inner 32-bit words] with a box of (inner, CG groups, RW row tiles).
int make_map(CUtensorMap* m, const void* base, int inner_words, int G, int RT, int CG, int RW) {
  if (int rc = encode_fn()) return rc;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner_words), static_cast<cuuint64_t>(G),
                        static_cast<cuuint64_t>(RT)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(inner_words) * 4,
                           static_cast<cuuint64_t>(inner_words) * 4 * G};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(inner_words), static_cast<cuuint32_t>(CG),
                       static_cast<cuuint32_t>(RW)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AGXC_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return 0;
}

}  // namespace

int encode_act_map(CUtensorMap* m, const void* x, int B, int K) { return encode_rows_map(m, x, B, K, B); }

int encode_rows_map(CUtensorMap* m, const void* x, int rows, int K, int box_rows) {
  if (int rc = encode_fn()) return rc;
  if (K % 64 || (reinterpret_cast<uintptr_t>(x) & 15) || box_rows < 1 || box_rows > 256)
    return fail(AGXC_EINVAL, "tensor map: rows of K % 64 == 0 fp16, 16-B aligned, boxes of 1..256 rows");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AGXC_ECUDA, "cuTensorMapEncodeTiled (X) failed (" + std::to_string(r) + ")");
  return 0;
}

int encode_pack_map(CUtensorMap* m, const void* base, int inner_words, int G, int RT, int CG, int RW) {
  return make_map(m, base, inner_words, G, RT, CG, RW);
}

// The same boxes over L layers' packs of one role at a constant byte stride (a 4-D map: words, groups, row tiles,
// layers).
int encode_pack_map_layers(CUtensorMap* m, const void* base, int inner_words, int G, int RT, int L,
                           uint64_t layer_stride, int CG, int RW) {
  if (int rc = encode_fn()) return rc;
  if (layer_stride % 16) return fail(AGXC_EINVAL, "tensor map: a layer stride that is a multiple of 16 bytes");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(inner_words), static_cast<cuuint64_t>(G),
                        static_cast<cuuint64_t>(RT), static_cast<cuuint64_t>(L)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(inner_words) * 4,
                           static_cast<cuuint64_t>(inner_words) * 4 * G, static_cast<cuuint64_t>(layer_stride)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(inner_words), static_cast<cuuint32_t>(CG),
                       static_cast<cuuint32_t>(RW), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AGXC_ECUDA, "cuTensorMapEncodeTiled (layers) failed (" + std::to_string(r) + ")");
  return 0;
}

int encode_kv_map_box(CUtensorMap* m, const void* base, int hd, int cap, int64_t Z, int box_keys) {
  if (int rc = encode_fn()) return rc;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(cap), static_cast<cuuint64_t>(Z)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(hd) * 2, static_cast<cuuint64_t>(hd) * 2 * cap};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_keys), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AGXC_ECUDA, "cuTensorMapEncodeTiled (KV) failed (" + std::to_string(r) + ")");
  return 0;
}

// Every GEMV instantiation may use up to the device's opt-in shared memory (set once per device, outside any
// stream capture).
int qmv_configure(const agxc_ctx* ctx) {
  const int s = ctx->max_smem_optin;
  int rc;
  if ((rc = qmv_configure_4_1(s)) || (rc = qmv_configure_4_2(s)) || (rc = qmv_configure_4_4(s)) ||
      (rc = qmv_configure_4_8(s)) || (rc = qmv_configure_8_1(s)) || (rc = qmv_configure_8_2(s)) ||
      (rc = qmv_configure_8_4(s)) || (rc = qmv_configure_8_8(s)))
    return rc;
  return encode_fn();
}

// The launch plan. One CTA per SM, persistent over units. RW (row tiles per unit: 1, 2, 4 or 8; even for SwiGLU,
// whose units pair a gate tile with its up tile) minimises the row tiles the busiest CTA carries; ties go to the
// larger RW (fewer per-unit reductions). K is split only when the CTA's activation rows would not fit in ~40 KB (or
// when asked). A chunk holds CG groups of every row tile of the unit (at most 36 KB, CG a multiple of the 16 / RW
// K lanes that divides the CTA's groups); as many stages as ~80 KB allows (two CTAs, this kernel and its
// programmatic-dependent successor, share an SM; 160 KB for the head, which has no successor in the step). With one
// activation row, a CTA whose whole weight share fits 160 KB keeps all of it in flight instead (chunks up to 72 KB),
// and a larger share gets a ring of up to 144 KB.
QmvPlan plan_qmv(const agxc_ctx* ctx, int N, int K, int bits, int nb, int epi, int hd, int splits, int force_rw,
                 int force_cg, int force_stages) {
  (void)hd;
  QmvPlan P;
  const int G = K / 64;
  const int TB = tile_bytes(bits);
  const int RT = N / 16;
  const int sms = ctx ? ctx->num_sms : kNumSMs;
  const int nbt = nb_tmpl(nb);
  int SC = 1;
  if (splits > 0 && G % splits == 0) {
    SC = splits;
  } else {
    while (G % (SC * 2) == 0 && static_cast<long>(nbt) * (G / SC) * 64 * 2 > 40 * 1024) SC *= 2;
  }
  if (epi == EPI_ARGMAX) SC = 1;  // the argmax needs whole rows per unit
  const int GC = G / SC;
  auto chunk_groups = [&](int rw) {
    // prefer a multiple of the K lanes (every warp busy); else the largest divisor that fits (some lanes idle)
    const int kw = kConsumerWarps / rw;
    int cg = 0, any = 0;
    for (int c = 1; c <= GC; ++c) {
      if (GC % c || rw * c * (TB + 64) > 36 * 1024) continue;
      any = c;
      if (c % kw == 0) cg = c;
    }
    return cg ? cg : any;
  };
  int best_rw = 0;
  long best_cost = -1;
  for (int rw : {8, 4, 2, 1}) {
    if (RT % rw) continue;
    if (force_rw && rw != force_rw) continue;
    if (epi == EPI_SWIGLU && rw == 1) continue;
    if (!chunk_groups(rw)) continue;
    const long units = static_cast<long>(RT / rw) * SC;
    const long cost = (units + sms - 1) / sms * rw;
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best_rw = rw; }
  }
  if (!best_rw) {
    P.grid = 0;  // no unit shape gives every K lane whole groups: the caller reports the shape as unsupported
    return P;
  }
  P.RW = best_rw;
  P.EB = 1;
  P.SC = SC;
  P.GC = GC;
  P.CG = chunk_groups(P.RW);
  if (force_cg > 0 && GC % force_cg == 0) P.CG = force_cg;
  const int stage_bytes = (P.RW * P.CG * (TB + 64) + 127) / 128 * 128;
  const int units = RT / P.RW * SC;
  const int chunks_per_cta = (units + sms - 1) / sms * (P.GC / P.CG);
  // the vocab head is the graph's last kernel: no programmatic-dependent successor shares its SM, so its ring may take
  // most of the shared memory
  const int ring_cap = epi == EPI_ARGMAX ? 160 * 1024 : 80 * 1024;
  P.stages = std::max(2, std::min({kMaxStages, ring_cap / stage_bytes, std::max(2, chunks_per_cta)}));
  // One activation row, no forced chunk size or depth: more weight bytes in flight per SM than the 80 KB ring. When the
  // CTA's whole weight share fits 160 KB it all goes in flight at entry, in chunks of up to 72 KB (fewer chunk
  // hand-offs); a larger share gets a ring of up to 144 KB in its default chunks. The successor then shares the SM only
  // once this kernel's CTAs leave. Measured per decode step of the 1.8B model (batch 1, history 1,792): 4-bit gate/up
  // (147 KB a CTA) whole in two 72 KB chunks 722 us against 793 us with two 36 KB stages (four 36 KB stages: 731 us);
  // 8-bit down (139 KB a CTA) whole 917 us against 956 us; 8-bit gate/up (278 KB a CTA) four 34 KB stages 835 us
  // against 917 us with two (three: 910 us; two 69 KB chunks: 848 us).
  if (nb == 1 && epi != EPI_ARGMAX && force_cg <= 0 && force_stages < 2 && chunks_per_cta > P.stages) {
    if (static_cast<long>(chunks_per_cta) * stage_bytes <= 160 * 1024) {
      const int kw = kConsumerWarps / P.RW;
      for (int c = P.GC; c > P.CG; --c) {
        if (P.GC % c == 0 && c % kw == 0 && P.RW * c * (TB + 64) <= 72 * 1024) {
          P.CG = c;
          break;
        }
      }
      P.stages = std::max(2, std::min(kMaxStages, (units + sms - 1) / sms * (P.GC / P.CG)));
    } else {
      P.stages = std::max(P.stages, std::min(kMaxStages, 144 * 1024 / stage_bytes));
    }
  }
  if (force_stages >= 2 && force_stages <= kMaxStages) P.stages = force_stages;
  int grid = std::min(units, sms);
  grid = std::max(SC, grid / SC * SC);
  P.grid = grid;
  P.smem = smem_total(bits, nbt, P.RW, P.CG, P.GC, P.stages);
  const size_t optin = ctx ? static_cast<size_t>(ctx->max_smem_optin) : 227 * 1024;
  while (force_stages < 2 && P.stages > 2 && P.smem > optin)  // an unforced ring gives way to the staged activations
    P.smem = smem_total(bits, nbt, P.RW, P.CG, P.GC, --P.stages);
  return P;
}

size_t qmv_part_floats(const QmvPlan& p, int N, int nb, int epi) {
  (void)epi;
  if (p.SC == 1) return 0;
  return static_cast<size_t>(p.SC) * N * nb;
}

int qmv_maps(const QmvPlan& plan, const uint8_t* w, const uint8_t* sb, int N, int K, int bits, CUtensorMap* tw,
             CUtensorMap* ts) {
  const int G = K / 64, RT = N / 16;
  int rc = make_map(tw, w, tile_bytes(bits) / 4, G, RT, plan.CG, plan.RW);
  if (!rc) rc = make_map(ts, sb, 16, G, RT, plan.CG, plan.RW);
  return rc;
}

int launch_qmv_epi(const agxc_ctx* ctx, QmvParams p, const QmvPlan& plan, int epi, cudaStream_t s,
                   const CUtensorMap* tw, const CUtensorMap* ts) {
  if (p.N % 16 || p.K % 64) return fail(AGXC_EINVAL, "qmv: N must be a multiple of 16 and K of 64");
  if (p.nb < 1 || p.nb > 8) return fail(AGXC_EINVAL, "qmv: 1 to 8 activation rows");
  if (plan.grid <= 0) return fail(AGXC_EINVAL, "qmv: no launch plan for this shape (too few groups for the K lanes)");
  if (plan.SC > 1 && (!p.part || !p.counters)) return fail(AGXC_EINVAL, "qmv: split K needs scratch");
  if ((p.N / 16) % plan.RW) return fail(AGXC_EINVAL, "qmv: plan's RW does not divide the row tiles");
  p.G = p.K / 64;
  p.SC = plan.SC;
  p.GC = plan.GC;
  p.CG = plan.CG;
  p.stages = plan.stages;
  CUtensorMap mw, ms;
  if (!tw || !ts) {
    if (int rc = qmv_maps(plan, p.w, p.sb, p.N, p.K, p.bits, &mw, &ms)) return rc;
    tw = &mw;
    ts = &ms;
  }
  const int nbt = nb_tmpl(p.nb);
  if (p.bits == 4) {
    switch (nbt) {
      case 1: return qmv_dispatch_4_1(ctx, p, plan, epi, *tw, *ts, s);
      case 2: return qmv_dispatch_4_2(ctx, p, plan, epi, *tw, *ts, s);
      case 4: return qmv_dispatch_4_4(ctx, p, plan, epi, *tw, *ts, s);
      default: return qmv_dispatch_4_8(ctx, p, plan, epi, *tw, *ts, s);
    }
  }
  if (p.bits == 8) {
    switch (nbt) {
      case 1: return qmv_dispatch_8_1(ctx, p, plan, epi, *tw, *ts, s);
      case 2: return qmv_dispatch_8_2(ctx, p, plan, epi, *tw, *ts, s);
      case 4: return qmv_dispatch_8_4(ctx, p, plan, epi, *tw, *ts, s);
      default: return qmv_dispatch_8_8(ctx, p, plan, epi, *tw, *ts, s);
    }
  }
  return fail(AGXC_EINVAL, "qmv: 4- or 8-bit weights");
}

}  // namespace agxc
