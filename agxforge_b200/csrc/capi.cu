// capi.cu — the extern "C" entry points of libagxcuda.so for contexts, packs and the per-kernel calls
// (the model entry points are in model.cu). Errors: a negative AGXC_E* code and a per-thread message.
#include <cstring>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace agxc {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return AGXC_ECUDA;
}

static int check_desc(const agxc_pack_desc* d) {
  if (!d) return fail(AGXC_EINVAL, "pack: null descriptor");
  if (d->bits != 4 && d->bits != 8) return fail(AGXC_EINVAL, "pack: 4- or 8-bit weights");
  if (d->group != 64) return fail(AGXC_EINVAL, "pack: group 64 only");
  if (d->k % 64 || d->k <= 0) return fail(AGXC_EINVAL, "pack: K must be a positive multiple of the group (64)");
  if (d->n % 16 || d->n <= 0) return fail(AGXC_EINVAL, "pack: N must be a positive multiple of 16");
  if (d->scale_dtype != AGXC_SCALE_FP16 && d->scale_dtype != AGXC_SCALE_BF16)
    return fail(AGXC_EINVAL, "pack: scale_dtype fp16 (0) or bf16 (1)");
  return 0;
}

static cudaStream_t stream_of(agxc_ctx* ctx, void* s) { return s ? static_cast<cudaStream_t>(s) : ctx->stream; }

// device buffers of a reference-format pack, uploaded from the host when needed
struct RefBufs {
  const void* p = nullptr;
  const void* s = nullptr;
  const void* b = nullptr;
  void* tmp = nullptr;
  ~RefBufs() {
    if (tmp) cudaFree(tmp);
  }
  int load(const agxc_pack_desc* d, const void* packed, const void* scales, const void* biases, int on_device) {
    if (on_device) {
      p = packed; s = scales; b = biases;
      return 0;
    }
    const size_t pb = static_cast<size_t>(d->n) * d->k * d->bits / 8, sb = static_cast<size_t>(d->n) * (d->k / 64) * 2;
    AGXC_CUDA(cudaMalloc(&tmp, pb + 2 * sb));
    uint8_t* t = static_cast<uint8_t*>(tmp);
    AGXC_CUDA(cudaMemcpy(t, packed, pb, cudaMemcpyHostToDevice));
    AGXC_CUDA(cudaMemcpy(t + pb, scales, sb, cudaMemcpyHostToDevice));
    AGXC_CUDA(cudaMemcpy(t + pb + sb, biases, sb, cudaMemcpyHostToDevice));
    p = t; s = t + pb; b = t + pb + sb;
    return 0;
  }
};

static int pack_alloc(agxc_ctx* ctx, int n, int k, int bits, int sdt, agxc_pack** out) {
  agxc_pack* p = new agxc_pack();
  p->ctx = ctx;
  p->n = n; p->k = k; p->bits = bits; p->sdt = sdt; p->group = 64;
  const size_t tb = static_cast<size_t>(n) * k * bits / 8, sbb = static_cast<size_t>(n / 16) * (k / 64) * 64;
  void* mem = nullptr;
  cudaError_t e = cudaMalloc(&mem, align_up(tb, 256) + sbb);
  if (e != cudaSuccess) {
    delete p;
    return fail(AGXC_ENOMEM, std::string("pack: cudaMalloc: ") + cudaGetErrorString(e));
  }
  p->tiles = static_cast<uint8_t*>(mem);
  p->sb = p->tiles + align_up(tb, 256);
  p->owns = true;
  *out = p;
  return 0;
}

}  // namespace agxc

using namespace agxc;

extern "C" {

const char* agxc_last_error(void) { return g_last_error.c_str(); }

int agxc_version(void) { return 1; }

int agxc_init(int device, agxc_ctx** out) {
  if (!out) return fail(AGXC_EINVAL, "init: null output");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(AGXC_EINVAL, "init: no such device");
  AGXC_CUDA(cudaSetDevice(device));
  int major = 0, minor = 0;
  AGXC_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  AGXC_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  if (major != 10 || minor != 0)
    return fail(AGXC_EUNSUPPORTED, "init: this library is built for sm_100a (B200); device is sm_" +
                                       std::to_string(major) + std::to_string(minor));
  agxc_ctx* c = new agxc_ctx();
  c->device = device;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&c->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->err_dev, 256);
  if (e == cudaSuccess) e = cudaMemset(c->err_dev, 0, 256);
  if (e == cudaSuccess) {
    // the stream-ordered scratch of agxc_qmv / agxc_qmm (split-K partial sums) comes from the device's default pool:
    // keep freed blocks in the pool (this process only) so each call reuses them instead of mapping new memory
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t keep = ~0ull;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    cudaGetLastError();
  }
  if (e != cudaSuccess) {
    agxc_ctx_free(c);
    return cuda_fail(e, "init");
  }
  if (int rc = qmv_configure(c)) {
    agxc_ctx_free(c);
    return rc;
  }
  if (int rc = attn_configure(c)) {
    agxc_ctx_free(c);
    return rc;
  }
  if (int rc = qmm_configure(c)) {
    agxc_ctx_free(c);
    return rc;
  }
  if (int rc = encoder_configure(c)) {
    agxc_ctx_free(c);
    return rc;
  }
  if (int rc = prefill_configure(c)) {
    agxc_ctx_free(c);
    return rc;
  }
  if (int rc = fstep_configure(c)) {
    agxc_ctx_free(c);
    return rc;
  }
  *out = c;
  return 0;
}

void agxc_ctx_free(agxc_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->err_dev) cudaFree(ctx->err_dev);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

int agxc_ctx_sync(agxc_ctx* ctx) {
  if (!ctx) return fail(AGXC_EINVAL, "sync: null context");
  AGXC_CUDA(cudaStreamSynchronize(ctx->stream));
  return 0;
}

int agxc_ctx_stream(agxc_ctx* ctx, void** stream) {
  if (!ctx || !stream) return fail(AGXC_EINVAL, "ctx_stream: null argument");
  *stream = ctx->stream;
  return 0;
}

int agxc_ctx_error_word(agxc_ctx* ctx, uint32_t* word) {
  if (!ctx || !word) return fail(AGXC_EINVAL, "error_word: null argument");
  AGXC_CUDA(cudaMemcpy(word, ctx->err_dev, 4, cudaMemcpyDeviceToHost));
  AGXC_CUDA(cudaMemset(ctx->err_dev, 0, 4));
  return 0;
}

int agxc_quantize_dev(agxc_ctx* ctx, const agxc_pack_desc* desc, const float* w_dev, uint32_t* packed_dev,
                      uint16_t* scales_dev, uint16_t* biases_dev, void* stream) {
  if (!ctx || !w_dev || !packed_dev || !scales_dev || !biases_dev) return fail(AGXC_EINVAL, "quantize: null argument");
  if (!desc || desc->n <= 0 || desc->k <= 0 || desc->k % 64 || (desc->bits != 4 && desc->bits != 8) ||
      desc->group != 64 || (desc->scale_dtype != AGXC_SCALE_FP16 && desc->scale_dtype != AGXC_SCALE_BF16))
    return fail(AGXC_EINVAL, "quantize: N positive, K a multiple of the group (64), 4 or 8 bits, fp16/bf16 scales");
  if (reinterpret_cast<uintptr_t>(w_dev) % 16) return fail(AGXC_EINVAL, "quantize: weights must be 16-byte aligned");
  return launch_quantize(w_dev, desc->n, desc->k, desc->bits, desc->scale_dtype, packed_dev, scales_dev, biases_dev,
                         stream_of(ctx, stream));
}

int agxc_pack_create(agxc_ctx* ctx, const agxc_pack_desc* desc, const void* packed, const void* scales,
                     const void* biases, int on_device, agxc_pack** out) {
  if (!ctx || !packed || !scales || !biases || !out) return fail(AGXC_EINVAL, "pack_create: null argument");
  if (int rc = check_desc(desc)) return rc;
  RefBufs r;
  if (int rc = r.load(desc, packed, scales, biases, on_device)) return rc;
  agxc_pack* p = nullptr;
  if (int rc = pack_alloc(ctx, desc->n, desc->k, desc->bits, desc->scale_dtype, &p)) return rc;
  int rc = launch_relayout(static_cast<const uint32_t*>(r.p), static_cast<const uint16_t*>(r.s),
                           static_cast<const uint16_t*>(r.b), desc->n, desc->k, desc->bits, p->tiles, p->sb, 1, 0,
                           ctx->stream);
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (!rc && e != cudaSuccess) rc = cuda_fail(e, "pack_create");
  if (rc) {
    agxc_pack_free(p);
    return rc;
  }
  *out = p;
  return 0;
}

int agxc_pack_create_gateup(agxc_ctx* ctx, const agxc_pack_desc* d, const void* g_packed, const void* g_scales,
                            const void* g_biases, const void* u_packed, const void* u_scales, const void* u_biases,
                            int on_device, agxc_pack** out) {
  if (!ctx || !out || !g_packed || !u_packed) return fail(AGXC_EINVAL, "pack_create_gateup: null argument");
  if (int rc = check_desc(d)) return rc;
  RefBufs rg, ru;
  if (int rc = rg.load(d, g_packed, g_scales, g_biases, on_device)) return rc;
  if (int rc = ru.load(d, u_packed, u_scales, u_biases, on_device)) return rc;
  agxc_pack* p = nullptr;
  if (int rc = pack_alloc(ctx, 2 * d->n, d->k, d->bits, d->scale_dtype, &p)) return rc;
  p->gateup = 1;
  int rc = launch_relayout(static_cast<const uint32_t*>(rg.p), static_cast<const uint16_t*>(rg.s),
                           static_cast<const uint16_t*>(rg.b), d->n, d->k, d->bits, p->tiles, p->sb, 2, 0, ctx->stream);
  if (!rc)
    rc = launch_relayout(static_cast<const uint32_t*>(ru.p), static_cast<const uint16_t*>(ru.s),
                         static_cast<const uint16_t*>(ru.b), d->n, d->k, d->bits, p->tiles, p->sb, 2, 1, ctx->stream);
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (!rc && e != cudaSuccess) rc = cuda_fail(e, "pack_create_gateup");
  if (rc) {
    agxc_pack_free(p);
    return rc;
  }
  *out = p;
  return 0;
}

void agxc_pack_free(agxc_pack* p) {
  if (!p) return;
  if (p->owns && p->tiles) cudaFree(p->tiles);
  delete p;
}

int64_t agxc_pack_bytes(const agxc_pack* p) { return p ? p->bytes() : 0; }

int agxc_pack_unpack_dev(const agxc_pack* p, uint8_t* fields_dev, void* stream) {
  if (!p || !fields_dev) return fail(AGXC_EINVAL, "unpack: null argument");
  return launch_unpack(p, fields_dev, stream ? static_cast<cudaStream_t>(stream) : p->ctx->stream);
}

int agxc_pack_dequant_dev(const agxc_pack* p, float* w_dev, void* stream) {
  if (!p || !w_dev) return fail(AGXC_EINVAL, "dequant: null argument");
  return launch_dequant(p, w_dev, stream ? static_cast<cudaStream_t>(stream) : p->ctx->stream);
}

int agxc_qmv(agxc_ctx* ctx, const agxc_qmv_args* a, void* stream) {
  if (!ctx || !a || !a->pack || !a->x_dev || !a->out_dev) return fail(AGXC_EINVAL, "qmv: null argument");
  const agxc_pack* pk = a->pack;
  if (a->nb < 1 || a->nb > 8) return fail(AGXC_EINVAL, "qmv: nb must be 1..8");
  if (a->epi < AGXC_EPI_F32 || a->epi > AGXC_EPI_SWIGLU) return fail(AGXC_EINVAL, "qmv: unknown epilogue");
  if (a->epi == AGXC_EPI_SWIGLU && !pk->gateup) return fail(AGXC_EINVAL, "qmv: SwiGLU needs a gate/up pack");
  if (a->epi != AGXC_EPI_SWIGLU && pk->gateup) return fail(AGXC_EINVAL, "qmv: a gate/up pack only takes SwiGLU");
  if ((a->epi == AGXC_EPI_RES1 || a->epi == AGXC_EPI_RES2) && !a->res_dev)
    return fail(AGXC_EINVAL, "qmv: residual epilogue without a residual");
  if (a->x_ld < pk->k) return fail(AGXC_EINVAL, "qmv: x_ld < K");
  const int nout = a->epi == AGXC_EPI_SWIGLU ? pk->n / 2 : pk->n;
  if (a->out_ld < nout) return fail(AGXC_EINVAL, "qmv: out_ld < output width");
  if ((a->epi == AGXC_EPI_RES1 || a->epi == AGXC_EPI_RES2) && a->res_ld < pk->n)
    return fail(AGXC_EINVAL, "qmv: res_ld < N");
  const int G = pk->k / 64;
  if (a->splits < 0 || (a->splits > 0 && G % a->splits)) return fail(AGXC_EINVAL, "qmv: splits must divide K/64");
  if (a->row_tiles && a->row_tiles != 1 && a->row_tiles != 2 && a->row_tiles != 4 && a->row_tiles != 8)
    return fail(AGXC_EINVAL, "qmv: row_tiles 1, 2, 4 or 8");
  if (a->stages && (a->stages < 2 || a->stages > 8)) return fail(AGXC_EINVAL, "qmv: stages 2..8");
  const int epi = a->epi;
  QmvPlan plan = plan_qmv(ctx, pk->n, pk->k, pk->bits, a->nb, epi, 0, a->splits, a->row_tiles, a->chunk_groups,
                          a->stages);
  QmvParams p;
  p.w = pk->tiles; p.sb = pk->sb; p.N = pk->n; p.K = pk->k; p.bits = pk->bits; p.sdt = pk->sdt; p.nb = a->nb;
  p.x = a->x_dev; p.x_f32 = a->x_f32; p.x_ld = a->x_ld;
  p.norm_gain = reinterpret_cast<const __half*>(a->norm_gain_dev); p.eps = a->eps;
  p.out_ld = a->out_ld; p.res_ld = a->res_ld; p.err = ctx->err_dev;
  if (epi == AGXC_EPI_F32 || epi == AGXC_EPI_RES1) p.out_f32 = static_cast<float*>(a->out_dev);
  else p.out_f16 = static_cast<__half*>(a->out_dev);
  if (epi == AGXC_EPI_RES1) p.res16 = static_cast<const __half*>(a->res_dev);
  if (epi == AGXC_EPI_RES2) p.res32 = static_cast<const float*>(a->res_dev);
  // scratch for split-K (allocated per call: the per-kernel entry points are for tests, the model keeps its own)
  float* part = nullptr;
  unsigned* cnt = nullptr;
  const size_t pf = qmv_part_floats(plan, pk->n, a->nb, epi);
  cudaStream_t s = stream_of(ctx, stream);
  if (pf) {
    AGXC_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&part), pf * 4, s));
    const size_t nblk = static_cast<size_t>(pk->n / 16) + 1;
    AGXC_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&cnt), nblk * 4, s));
    AGXC_CUDA(cudaMemsetAsync(cnt, 0, nblk * 4, s));
  }
  p.part = part;
  p.counters = cnt;
  int rc = launch_qmv_epi(ctx, p, plan, epi, s);
  if (part) cudaFreeAsync(part, s);
  if (cnt) cudaFreeAsync(cnt, s);
  return rc;
}

int agxc_qmm(agxc_ctx* ctx, const agxc_pack* pack, const void* x_dev, int batch, float* y_dev, int ldy, int ksplit,
             void* stream) {
  if (!ctx || !pack || !x_dev || !y_dev) return fail(AGXC_EINVAL, "qmm: null argument");
  if (pack->gateup) return fail(AGXC_EINVAL, "qmm: a plain pack (not gate/up interleaved)");
  cudaStream_t s = stream_of(ctx, stream);
  const int G = pack->k / 64, tiles = pack->n / 128;
  if (ksplit == 0) {  // split K until the tiles fill the SMs (a divisor of the groups)
    ksplit = 1;
    while (tiles * ksplit * 2 <= ctx->num_sms && G % (ksplit * 2) == 0) ksplit *= 2;
  }
  if (ksplit < 2) return launch_qmm(ctx, pack, x_dev, batch, y_dev, ldy, ksplit, s);
  // split K: stream-ordered scratch for the ranges' partial sums and the tile counters
  const size_t part_bytes = static_cast<size_t>(ksplit) * batch * pack->n * 4, ctr_bytes = static_cast<size_t>(tiles) * 4;
  void* scratch = nullptr;
  AGXC_CUDA(cudaMallocAsync(&scratch, part_bytes + ctr_bytes, s));
  unsigned* ctr = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(scratch) + part_bytes);
  int rc = cudaMemsetAsync(ctr, 0, ctr_bytes, s) == cudaSuccess ? 0 : fail(AGXC_ECUDA, "qmm: counter clear");
  if (!rc) rc = launch_qmm(ctx, pack, x_dev, batch, y_dev, ldy, ksplit, s, nullptr, static_cast<float*>(scratch), ctr);
  cudaFreeAsync(scratch, s);
  return rc;
}

int agxc_rmsnorm_dev(agxc_ctx* ctx, const void* x_dev, int x_f32, int nb, int d, const uint16_t* gain_dev, float eps,
                     uint16_t* out_dev, void* stream) {
  if (!ctx || !x_dev || !gain_dev || !out_dev) return fail(AGXC_EINVAL, "rmsnorm: null argument");
  if (nb < 1 || d < 1) return fail(AGXC_EINVAL, "rmsnorm: nb and d must be positive");
  return launch_rmsnorm(x_dev, x_f32, nb, d, reinterpret_cast<const __half*>(gain_dev), eps,
                        reinterpret_cast<__half*>(out_dev), stream_of(ctx, stream));
}

int agxc_attention_dev(agxc_ctx* ctx, int nb, int heads, int kv_heads, int head_dim, int cap, const uint32_t* q0_dev,
                       const uint16_t* q16_dev, const uint16_t* k_dev, const uint16_t* v_dev, uint16_t* out_dev,
                       int splits, void* stream) {
  if (!ctx || !q0_dev || !q16_dev || !k_dev || !v_dev || !out_dev) return fail(AGXC_EINVAL, "attention: null argument");
  if (nb < 1 || heads < 1 || kv_heads < 1 || cap < 1) return fail(AGXC_EINVAL, "attention: sizes must be positive");
  AttnParams p;
  p.nb = nb; p.H = heads; p.KVH = kv_heads; p.hd = head_dim; p.cap = cap;
  p.S = splits > 0 ? splits : attn_splits(ctx, nb, kv_heads, cap);
  p.q0 = q0_dev;
  p.q16 = reinterpret_cast<const __half*>(q16_dev);
  p.kc = reinterpret_cast<const __half*>(k_dev);
  p.vc = reinterpret_cast<const __half*>(v_dev);
  p.out = reinterpret_cast<__half*>(out_dev);
  p.err = ctx->err_dev;
  return launch_attention(ctx, p, stream_of(ctx, stream));
}

}  // extern "C"
