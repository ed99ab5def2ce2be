// qmv_noalloc.cu — agxc_qmv_noalloc: the GEMV entry point for callers that may not allocate device memory.
//
// agxc_qmv takes its split-K scratch (per-split partial rows and the last-arriver counters) from the stream-ordered
// allocator on every call that splits K. Some callers cannot do that: a host runtime that owns every device
// allocation itself and forbids libraries from calling the allocator (for example one that accounts for HBM per
// tenant, or that runs with the caching allocator's pool reserved for its own tensors), and code that must not add
// allocator calls between launches it orders by hand. For them this entry point runs the same kernels with the same
// launch plan, taking the scratch from a fixed block of static device memory instead.
//
// The static block holds kPartFloats fp32 partials (4 MiB) and kCounters counters. A call whose plan needs more
// partials (splits x N x nb) or more counters (N / 16 + 1) than that is rejected with AGXC_EINVAL before anything is
// launched. The counters must read zero when a launch starts: the call clears the ones it uses with
// cudaMemsetAsync on the stream before the launch (the kernel also returns each to zero when its rows are reduced).
// The partials need no initial value.
//
// The block is one per device and not per call: calls that may overlap on one device (two streams, two threads,
// or one stream and a model's graph replaying meanwhile) race on it and give wrong rows. Order them on one stream.
//
// Set-up: the first call on a device looks up the block's address for that device (cudaGetSymbolAddress, with that
// device current) and remembers it; later calls only read it. Make that first call outside any stream capture.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr size_t kPartFloats = size_t(1) << 20;  // 4 MiB of fp32 split-K partials
constexpr size_t kCounters = 8192;               // row blocks of up to N = 131,056 rows
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_part[kPartFloats];
__device__ __align__(256) unsigned g_counters[kCounters];

struct Scratch {
  float* part = nullptr;
  unsigned* counters = nullptr;
};
Scratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// The static block's addresses on `device`, looked up once per device with that device current.
int scratch_for(int device, Scratch* out) {
  if (device < 0 || device >= kMaxDevices) return agxc::fail(AGXC_EINVAL, "qmv_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch& s = g_scratch[device];
  if (!s.part) {
    int prev = -1;
    AGXC_CUDA(cudaGetDevice(&prev));
    if (prev != device) AGXC_CUDA(cudaSetDevice(device));
    void* part = nullptr;
    void* cnt = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&part, g_part);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&cnt, g_counters);
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return agxc::cuda_fail(e, "qmv_noalloc: static scratch lookup");
    s.part = static_cast<float*>(part);
    s.counters = static_cast<unsigned*>(cnt);
  }
  *out = s;
  return 0;
}

}  // namespace

using namespace agxc;

int agxc_qmv_noalloc(agxc_ctx* ctx, const agxc_qmv_args* a, void* stream) {
  if (!ctx || !a || !a->pack || !a->x_dev || !a->out_dev) return fail(AGXC_EINVAL, "qmv_noalloc: null argument");
  const agxc_pack* pk = a->pack;
  if (a->nb < 1 || a->nb > 8) return fail(AGXC_EINVAL, "qmv_noalloc: nb must be 1..8");
  if (a->epi < AGXC_EPI_F32 || a->epi > AGXC_EPI_SWIGLU) return fail(AGXC_EINVAL, "qmv_noalloc: unknown epilogue");
  if (a->epi == AGXC_EPI_SWIGLU && !pk->gateup) return fail(AGXC_EINVAL, "qmv_noalloc: SwiGLU needs a gate/up pack");
  if (a->epi != AGXC_EPI_SWIGLU && pk->gateup)
    return fail(AGXC_EINVAL, "qmv_noalloc: a gate/up pack only takes SwiGLU");
  if ((a->epi == AGXC_EPI_RES1 || a->epi == AGXC_EPI_RES2) && !a->res_dev)
    return fail(AGXC_EINVAL, "qmv_noalloc: residual epilogue without a residual");
  if (a->x_ld < pk->k) return fail(AGXC_EINVAL, "qmv_noalloc: x_ld < K");
  const int nout = a->epi == AGXC_EPI_SWIGLU ? pk->n / 2 : pk->n;
  if (a->out_ld < nout) return fail(AGXC_EINVAL, "qmv_noalloc: out_ld < output width");
  if ((a->epi == AGXC_EPI_RES1 || a->epi == AGXC_EPI_RES2) && a->res_ld < pk->n)
    return fail(AGXC_EINVAL, "qmv_noalloc: res_ld < N");
  const int G = pk->k / 64;
  if (a->splits < 0 || (a->splits > 0 && G % a->splits))
    return fail(AGXC_EINVAL, "qmv_noalloc: splits must divide K/64");
  if (a->row_tiles && a->row_tiles != 1 && a->row_tiles != 2 && a->row_tiles != 4 && a->row_tiles != 8)
    return fail(AGXC_EINVAL, "qmv_noalloc: row_tiles 1, 2, 4 or 8");
  if (a->stages && (a->stages < 2 || a->stages > 8)) return fail(AGXC_EINVAL, "qmv_noalloc: stages 2..8");
  const int epi = a->epi;
  const QmvPlan plan = plan_qmv(ctx, pk->n, pk->k, pk->bits, a->nb, epi, 0, a->splits, a->row_tiles,
                                a->chunk_groups, a->stages);
  const size_t pf = qmv_part_floats(plan, pk->n, a->nb, epi);
  const size_t nblk = static_cast<size_t>(pk->n / 16) + 1;
  if (pf > kPartFloats)
    return fail(AGXC_EINVAL, "qmv_noalloc: the plan's split-K partials (" + std::to_string(pf) +
                                 " floats: splits x N x nb) exceed the static scratch of " +
                                 std::to_string(kPartFloats) + " floats; use fewer splits or agxc_qmv");
  if (pf && nblk > kCounters)
    return fail(AGXC_EINVAL, "qmv_noalloc: N / 16 + 1 = " + std::to_string(nblk) + " row-block counters exceed the " +
                                 "static maximum of " + std::to_string(kCounters));
  QmvParams p;
  p.w = pk->tiles; p.sb = pk->sb; p.N = pk->n; p.K = pk->k; p.bits = pk->bits; p.sdt = pk->sdt; p.nb = a->nb;
  p.x = a->x_dev; p.x_f32 = a->x_f32; p.x_ld = a->x_ld;
  p.norm_gain = reinterpret_cast<const __half*>(a->norm_gain_dev); p.eps = a->eps;
  p.out_ld = a->out_ld; p.res_ld = a->res_ld; p.err = ctx->err_dev;
  if (epi == AGXC_EPI_F32 || epi == AGXC_EPI_RES1) p.out_f32 = static_cast<float*>(a->out_dev);
  else p.out_f16 = static_cast<__half*>(a->out_dev);
  if (epi == AGXC_EPI_RES1) p.res16 = static_cast<const __half*>(a->res_dev);
  if (epi == AGXC_EPI_RES2) p.res32 = static_cast<const float*>(a->res_dev);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  if (pf) {
    Scratch sc;
    if (int rc = scratch_for(ctx->device, &sc)) return rc;
    AGXC_CUDA(cudaMemsetAsync(sc.counters, 0, nblk * sizeof(unsigned), s));
    p.part = sc.part;
    p.counters = sc.counters;
  }
  return launch_qmv_epi(ctx, p, plan, epi, s);
}
