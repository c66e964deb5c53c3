// extern "C" entry points of libfhe_b200.so (declared in include/fhe_b200.h).
#include <chrono>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <map>
#include <memory>
#include <new>
#include <sstream>
#include <string>

#include "../../include/fhe_b200.h"
#include "bootstrap.h"
#include "ckks.h"
#include "context.h"
#include "program.h"
#include "shard.h"
#include "launch_count.h"

namespace fhe {
void rescale_noalloc(Context& c, const uint64_t* in, uint32_t ncomp, uint32_t nq, uint64_t* out);
}

// Member order matters: ck refers to c and is destroyed first.
struct fhe_ctx {
  fhe::Context c;
  std::unique_ptr<fhe::Ckks> ck;
  std::unique_ptr<fhe::Bootstrapper> boot;
  std::map<uint32_t, std::unique_ptr<fhe::Bootstrapper>> sub;  // sub-slot refreshes by slot count
  std::unique_ptr<fhe::ShardKeySwitch> shard;
};
struct fhe_ct {
  std::unique_ptr<fhe::Ct> p;
};
struct fhe_pt {
  std::unique_ptr<fhe::Pt> p;
};

namespace {

thread_local std::string g_last_error;

template <class F>
int guarded(F&& f) {
  try {
    f();
    return FHE_OK;
  } catch (const fhe::Error& e) {
    g_last_error = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return FHE_ERR_ALLOC;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return FHE_ERR_INTERNAL;
  } catch (...) {
    g_last_error = "unknown exception";
    return FHE_ERR_INTERNAL;
  }
}

void init_device(fhe::Context& c, int device) {
  int count = 0;
  FHE_CUDA(cudaGetDeviceCount(&count));
  fhe::require(device >= 0 && device < count, "device ordinal out of range");
  c.device = device;
  FHE_CUDA(cudaSetDevice(device));
  c.sh = std::make_shared<fhe::StreamHolder>();
  c.sh->device = device;
  FHE_CUDA(cudaStreamCreateWithFlags(&c.sh->s, cudaStreamNonBlocking));
  c.stream = c.sh->s;
  // Keep freed ciphertext memory in the device pool instead of returning it
  // to the driver at every synchronisation.
  cudaMemPool_t pool;
  FHE_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
  uint64_t threshold = UINT64_MAX;
  FHE_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold));
}

// Runs a raw transform on host or device memory.
void raw_transform(fhe_ctx* ctx, uint64_t* data, uint32_t n_polys, uint32_t limb0,
                   uint32_t n_limbs, int mem, bool inverse) {
  fhe::require(ctx != nullptr && data != nullptr, "null context or data");
  fhe::Context& c = ctx->c;
  fhe::require(limb0 + n_limbs <= c.n_primes(), "limb range exceeds the context's primes");
  fhe::require(mem == FHE_MEM_HOST || mem == FHE_MEM_DEVICE, "mem must be FHE_MEM_HOST or FHE_MEM_DEVICE");
  c.make_current();
  const size_t words = (size_t)n_polys * n_limbs * c.n;
  if (words == 0) return;
  uint64_t* d = data;
  if (mem == FHE_MEM_HOST) {
    d = c.stage(words);
    FHE_CUDA(cudaMemcpyAsync(d, data, words * 8, cudaMemcpyHostToDevice, c.stream));
  }
  fhe::NttArgs a = c.ntt_args(d, n_polys, limb0, n_limbs, n_limbs);
  FHE_CUDA(inverse ? fhe::ntt_inverse(a) : fhe::ntt_forward(a));
  if (mem == FHE_MEM_HOST) {
    FHE_CUDA(cudaMemcpyAsync(data, d, words * 8, cudaMemcpyDeviceToHost, c.stream));
    FHE_CUDA(cudaStreamSynchronize(c.stream));
  }
}

}  // namespace

extern "C" {

int fhe_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return FHE_ERR_INVALID;
  std::strncpy(buf, g_last_error.c_str(), len - 1);
  buf[len - 1] = 0;
  return FHE_OK;
}

int fhe_ctx_create(const fhe_params* p, fhe_ctx** out) {
  return guarded([&] {
    fhe::require(p != nullptr && out != nullptr, "null params or output handle");
    *out = nullptr;
    fhe::require(p->log_n >= 10 && p->log_n <= 17, "log_n must be in [10, 17]");
    const uint32_t n = 1u << p->log_n;
    fhe::require(p->batch_size >= 1 && p->batch_size <= n / 2 &&
                     (p->batch_size & (p->batch_size - 1)) == 0,
                 "batch_size must be a power of two <= N/2");
    auto h = std::make_unique<fhe_ctx>();
    fhe::Context& c = h->c;
    init_device(c, p->device);
    c.log_n = p->log_n;
    c.n = n;
    c.ckks = true;
    std::vector<uint64_t> q, pp;
    fhe::nt::ckks_moduli(p->log_n, p->mult_depth + 1, p->scaling_mod_size, p->first_mod_size,
                         p->num_large_digits, q, pp);
    c.L = (uint32_t)q.size();
    c.K = (uint32_t)pp.size();
    c.dnum = p->num_large_digits;
    c.alpha = (c.L + c.dnum - 1) / c.dnum;
    c.slots = p->batch_size;
    c.scale_bits = p->scaling_mod_size;
    c.first_bits = p->first_mod_size;
    c.primes = q;
    c.primes.insert(c.primes.end(), pp.begin(), pp.end());
    c.build_tables();
    h->ck = std::make_unique<fhe::Ckks>(c);
    *out = h.release();
  });
}

int fhe_ctx_create_ntt(uint32_t log_n, const uint64_t* primes, uint32_t n_primes, int32_t device,
                       fhe_ctx** out) {
  return guarded([&] {
    fhe::require(out != nullptr && primes != nullptr, "null primes or output handle");
    *out = nullptr;
    fhe::require(log_n >= 10 && log_n <= 17, "log_n must be in [10, 17]");
    fhe::require(n_primes >= 1 && n_primes <= 256, "n_primes must be in [1, 256]");
    const uint64_t m = uint64_t(2) << log_n;
    for (uint32_t i = 0; i < n_primes; ++i) {
      fhe::require(primes[i] < (uint64_t(1) << 62) && primes[i] % m == 1 && fhe::nt::is_prime(primes[i]),
                   "prime " + std::to_string(i) + " is not an NTT-friendly prime below 2^62");
    }
    auto h = std::make_unique<fhe_ctx>();
    fhe::Context& c = h->c;
    init_device(c, device);
    c.log_n = log_n;
    c.n = 1u << log_n;
    c.primes.assign(primes, primes + n_primes);
    c.L = n_primes;
    c.K = 0;
    c.build_tables();
    *out = h.release();
  });
}

int fhe_ctx_destroy(fhe_ctx* ctx) {
  return guarded([&] {
    if (!ctx) return;
    cudaSetDevice(ctx->c.device);
    delete ctx;
  });
}

int fhe_ctx_moduli(const fhe_ctx* ctx, uint64_t* q, uint32_t* n_q, uint64_t* p, uint32_t* n_p) {
  return guarded([&] {
    fhe::require(ctx != nullptr, "null context");
    const fhe::Context& c = ctx->c;
    if (n_q) *n_q = c.L;
    if (n_p) *n_p = c.K;
    if (q) std::memcpy(q, c.primes.data(), c.L * sizeof(uint64_t));
    if (p) std::memcpy(p, c.primes.data() + c.L, c.K * sizeof(uint64_t));
  });
}

int fhe_gen_ckks_moduli(uint32_t log_n, uint32_t mult_depth, uint32_t scaling_mod_size,
                        uint32_t first_mod_size, uint32_t num_large_digits, uint64_t* q,
                        uint32_t* n_q, uint64_t* p, uint32_t* n_p) {
  return guarded([&] {
    fhe::require(log_n >= 10 && log_n <= 17, "log_n must be in [10, 17]");
    std::vector<uint64_t> qq, pp;
    fhe::nt::ckks_moduli(log_n, mult_depth + 1, scaling_mod_size, first_mod_size, num_large_digits,
                         qq, pp);
    if (n_q) *n_q = (uint32_t)qq.size();
    if (n_p) *n_p = (uint32_t)pp.size();
    if (q) std::memcpy(q, qq.data(), qq.size() * sizeof(uint64_t));
    if (p) {
      fhe::require(pp.size() <= 64, "more than 64 P primes");
      std::memcpy(p, pp.data(), pp.size() * sizeof(uint64_t));
    }
  });
}

int fhe_gen_ntt_primes(uint32_t log_n, uint32_t bits, uint32_t count, uint64_t* out) {
  return guarded([&] {
    fhe::require(out != nullptr, "null output");
    fhe::require(log_n >= 1 && log_n <= 17 && bits > log_n + 1 && bits <= 62, "invalid log_n/bits");
    const uint64_t m = uint64_t(2) << log_n;
    uint64_t c = (uint64_t(1) << bits) + 1;
    for (uint32_t i = 0; i < count; ++i) {
      c = fhe::nt::previous_prime(c, m);
      out[i] = c;
    }
  });
}

int fhe_ctx_roots(const fhe_ctx* ctx, uint64_t* roots, uint32_t n) {
  return guarded([&] {
    fhe::require(ctx != nullptr && roots != nullptr, "null context or output");
    fhe::require(n <= ctx->c.roots.size(), "more roots requested than primes");
    std::memcpy(roots, ctx->c.roots.data(), n * sizeof(uint64_t));
  });
}

int fhe_ctx_stream(const fhe_ctx* ctx, void** stream) {
  return guarded([&] {
    fhe::require(ctx != nullptr && stream != nullptr, "null context or output");
    *stream = (void*)ctx->c.stream;
  });
}

int fhe_ctx_synchronize(fhe_ctx* ctx) {
  return guarded([&] {
    fhe::require(ctx != nullptr, "null context");
    ctx->c.make_current();
    FHE_CUDA(cudaStreamSynchronize(ctx->c.stream));
  });
}

int fhe_ntt(fhe_ctx* ctx, uint64_t* data, uint32_t n_polys, uint32_t limb0, uint32_t n_limbs, int mem) {
  return guarded([&] { raw_transform(ctx, data, n_polys, limb0, n_limbs, mem, false); });
}

int fhe_intt(fhe_ctx* ctx, uint64_t* data, uint32_t n_polys, uint32_t limb0, uint32_t n_limbs, int mem) {
  return guarded([&] { raw_transform(ctx, data, n_polys, limb0, n_limbs, mem, true); });
}

int fhe_rescale_noalloc(fhe_ctx* ctx, const uint64_t* in, uint32_t ncomp, uint32_t n_limbs, uint64_t* out) {
  return guarded([&] {
    fhe::require(ctx != nullptr, "null context");
    fhe::rescale_noalloc(ctx->c, in, ncomp, n_limbs, out);
  });
}

// ---------------------------------------------------------------------------
// CKKS

namespace {
fhe::Ckks& ckks(fhe_ctx* ctx) {
  fhe::require(ctx != nullptr, "null context");
  fhe::require(ctx->ck != nullptr, "not a CKKS context (created with fhe_ctx_create_ntt)");
  ctx->c.make_current();
  return *ctx->ck;
}
const fhe::Ct& ct_of(const fhe_ct* c) {
  fhe::require(c != nullptr && c->p != nullptr, "null ciphertext handle");
  return *c->p;
}
const fhe::Pt& pt_of(const fhe_pt* p) {
  fhe::require(p != nullptr && p->p != nullptr, "null plaintext handle");
  return *p->p;
}
void put_ct(fhe_ct** out, std::unique_ptr<fhe::Ct> c) {
  fhe::require(out != nullptr, "null output handle");
  *out = new fhe_ct{std::move(c)};
}
void put_pt(fhe_pt** out, std::unique_ptr<fhe::Pt> p) {
  fhe::require(out != nullptr, "null output handle");
  *out = new fhe_pt{std::move(p)};
}
}  // namespace

int fhe_ctx_info(const fhe_ctx* ctx, fhe_ctx_info_t* info) {
  return guarded([&] {
    fhe::require(ctx != nullptr && info != nullptr, "null context or output");
    const fhe::Context& c = ctx->c;
    info->log_n = c.log_n;
    info->n_q = c.L;
    info->n_p = c.K;
    info->dnum = c.dnum;
    info->alpha = c.alpha;
    info->slots = c.slots;
    info->ckks = ctx->ck ? 1 : 0;
    info->reserved = 0;
  });
}

int fhe_level_scale(fhe_ctx* ctx, uint32_t n_limbs, double* scale) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(scale != nullptr && n_limbs >= 1 && n_limbs <= ctx->c.L, "bad limb count or output");
    *scale = k.level_scale(n_limbs);
  });
}

int fhe_keygen(fhe_ctx* ctx, uint64_t seed) {
  return guarded([&] { ckks(ctx).keygen(seed); });
}

int fhe_galois_element(fhe_ctx* ctx, int32_t step, uint64_t* g) {
  return guarded([&] {
    fhe::require(g != nullptr, "null output");
    *g = ckks(ctx).galois_for_step(step);
  });
}

int fhe_rotation_keygen(fhe_ctx* ctx, const int32_t* steps, uint32_t n) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(steps != nullptr || n == 0, "null steps");
    for (uint32_t i = 0; i < n; ++i) k.rotation_keygen(k.galois_for_step(steps[i]));
  });
}

int fhe_conjugation_keygen(fhe_ctx* ctx) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    k.rotation_keygen(2ull * ctx->c.n - 1);
  });
}

int fhe_key_download(fhe_ctx* ctx, int kind, uint64_t galois, uint64_t* host, size_t words) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(kind >= 0 && kind <= 6, "key kind must be 0..6");
    fhe::require(host != nullptr && words == k.key_words(kind),
                 "host buffer must hold exactly " + std::to_string(k.key_words(kind)) + " words");
    k.download_key(kind, galois, host);
  });
}

int fhe_encode(fhe_ctx* ctx, const double* re, const double* im, uint32_t count, uint32_t n_limbs, double scale,
               fhe_pt** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(re != nullptr || count == 0, "null values");
    const uint32_t nq = n_limbs ? n_limbs : ctx->c.L;
    fhe::require(nq <= ctx->c.L, "n_limbs above the number of Q primes");
    put_pt(out, k.encode(re, im, count, nq, scale > 0 ? scale : k.level_scale(nq)));
  });
}

int fhe_decode(fhe_ctx* ctx, const fhe_pt* pt, double* re, double* im, uint32_t count) {
  return guarded([&] { ckks(ctx).decode(pt_of(pt), re, im, count); });
}

int fhe_encrypt(fhe_ctx* ctx, const fhe_pt* pt, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).encrypt(pt_of(pt))); });
}

int fhe_decrypt(fhe_ctx* ctx, const fhe_ct* ct, fhe_pt** out) {
  return guarded([&] { put_pt(out, ckks(ctx).decrypt(ct_of(ct))); });
}

int fhe_ct_free(fhe_ct* ct) {
  return guarded([&] { delete ct; });
}

int fhe_pt_free(fhe_pt* pt) {
  return guarded([&] { delete pt; });
}

int fhe_ct_info(const fhe_ct* ct, uint32_t* ncomp, uint32_t* n_limbs, uint32_t* noise_deg, double* scale) {
  return guarded([&] {
    const fhe::Ct& c = ct_of(ct);
    if (ncomp) *ncomp = c.ncomp;
    if (n_limbs) *n_limbs = c.nq;
    if (noise_deg) *noise_deg = c.noise_deg;
    if (scale) *scale = c.scale;
  });
}

int fhe_pt_info(const fhe_pt* pt, uint32_t* n_limbs, double* scale) {
  return guarded([&] {
    const fhe::Pt& p = pt_of(pt);
    if (n_limbs) *n_limbs = p.nq;
    if (scale) *scale = p.scale;
  });
}

int fhe_ct_download(fhe_ctx* ctx, const fhe_ct* ct, uint64_t* host) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    const fhe::Ct& c = ct_of(ct);
    fhe::require(host != nullptr, "null host buffer");
    const size_t n = ctx->c.n;
    FHE_CUDA(cudaMemcpy2DAsync(host, (size_t)c.nq * n * 8, c.data(), (size_t)c.cap * n * 8, (size_t)c.nq * n * 8,
                               c.ncomp, cudaMemcpyDeviceToHost, k.ctx.stream));
    FHE_CUDA(cudaStreamSynchronize(k.ctx.stream));
  });
}

int fhe_ct_upload(fhe_ctx* ctx, const uint64_t* host, uint32_t ncomp, uint32_t n_limbs, uint32_t noise_deg,
                  double scale, fhe_ct** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(host != nullptr, "null host buffer");
    fhe::require(ncomp >= 2 && ncomp <= 3 && n_limbs >= 1 && n_limbs <= ctx->c.L, "bad ciphertext shape");
    auto c = k.alloc(n_limbs, ncomp);
    c->noise_deg = noise_deg;
    c->scale = scale;
    FHE_CUDA(cudaMemcpyAsync(c->data(), host, (size_t)ncomp * n_limbs * ctx->c.n * 8, cudaMemcpyHostToDevice,
                             k.ctx.stream));
    FHE_CUDA(cudaStreamSynchronize(k.ctx.stream));
    put_ct(out, std::move(c));
  });
}

int fhe_pt_download(fhe_ctx* ctx, const fhe_pt* pt, uint64_t* host) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    const fhe::Pt& p = pt_of(pt);
    fhe::require(host != nullptr, "null host buffer");
    FHE_CUDA(cudaMemcpyAsync(host, p.data(), (size_t)p.nq * ctx->c.n * 8, cudaMemcpyDeviceToHost, k.ctx.stream));
    FHE_CUDA(cudaStreamSynchronize(k.ctx.stream));
  });
}

int fhe_pt_upload(fhe_ctx* ctx, const uint64_t* host, uint32_t n_limbs, double scale, fhe_pt** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(host != nullptr && n_limbs >= 1 && n_limbs <= ctx->c.L, "bad plaintext shape");
    auto p = std::make_unique<fhe::Pt>();
    p->buf = fhe::DevMem((size_t)n_limbs * ctx->c.n * 8, ctx->c.sh);
    p->nq = n_limbs;
    p->scale = scale;
    FHE_CUDA(cudaMemcpyAsync(p->data(), host, (size_t)n_limbs * ctx->c.n * 8, cudaMemcpyHostToDevice, k.ctx.stream));
    FHE_CUDA(cudaStreamSynchronize(k.ctx.stream));
    put_pt(out, std::move(p));
  });
}

int fhe_ct_clone(fhe_ctx* ctx, const fhe_ct* ct, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).clone(ct_of(ct))); });
}

int fhe_add(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).add(ct_of(a), ct_of(b), false)); });
}

int fhe_sub(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).add(ct_of(a), ct_of(b), true)); });
}

int fhe_negate(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).negate(ct_of(a))); });
}

int fhe_add_plain(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* p, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).add_plain(ct_of(a), pt_of(p), false)); });
}

int fhe_sub_plain(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* p, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).add_plain(ct_of(a), pt_of(p), true)); });
}

int fhe_mul_plain(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* p, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).mul_plain(ct_of(a), pt_of(p))); });
}

int fhe_add_scalar(fhe_ctx* ctx, const fhe_ct* a, double v, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).add_scalar(ct_of(a), v)); });
}

int fhe_mul_scalar(fhe_ctx* ctx, const fhe_ct* a, double v, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).mul_scalar(ct_of(a), v)); });
}

int fhe_mul_int(fhe_ctx* ctx, const fhe_ct* a, int64_t v, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).mul_int(ct_of(a), v)); });
}

int fhe_tensor(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).tensor(ct_of(a), ct_of(b))); });
}

int fhe_relinearize(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).relinearize(ct_of(a))); });
}

int fhe_mul(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).mul(ct_of(a), ct_of(b))); });
}

int fhe_rescale(fhe_ctx* ctx, fhe_ct* ct) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(ct != nullptr && ct->p != nullptr, "null ciphertext handle");
    k.rescale_inplace(*ct->p);
  });
}

int fhe_level_reduce(fhe_ctx* ctx, fhe_ct* ct, uint32_t levels) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(ct != nullptr && ct->p != nullptr, "null ciphertext handle");
    k.level_reduce_inplace(*ct->p, levels);
  });
}

int fhe_rotate(fhe_ctx* ctx, const fhe_ct* a, int32_t step, fhe_ct** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    put_ct(out, k.rotate(ct_of(a), k.galois_for_step(step)));
  });
}

int fhe_conjugate(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).rotate(ct_of(a), 2ull * ctx->c.n - 1)); });
}

int fhe_rotate_hoisted(fhe_ctx* ctx, const fhe_ct* a, const int32_t* steps, uint32_t n, fhe_ct** outs) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(outs != nullptr && (steps != nullptr || n == 0), "null steps or outputs");
    std::vector<uint64_t> gs(n);
    for (uint32_t i = 0; i < n; ++i) gs[i] = k.galois_for_step(steps[i]);
    auto r = k.rotate_hoisted(ct_of(a), gs);
    for (uint32_t i = 0; i < n; ++i) outs[i] = new fhe_ct{std::move(r[i])};
  });
}

int fhe_encode_batch(fhe_ctx* ctx, const double* re, const double* im, uint32_t batch, uint32_t count,
                     uint32_t n_limbs, double scale, fhe_pt** outs) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(outs != nullptr && (re != nullptr || count == 0), "null values or outputs");
    const uint32_t nq = n_limbs ? n_limbs : ctx->c.L;
    fhe::require(nq <= ctx->c.L, "n_limbs above the number of Q primes");
    auto v = k.encode_batch(re, im, batch, count, nq, scale > 0 ? scale : k.level_scale(nq));
    for (uint32_t i = 0; i < batch; ++i) outs[i] = new fhe_pt{std::move(v[i])};
  });
}

int fhe_encode_replicated_diagonals(fhe_ctx* ctx, const double* w_dev, uint32_t m, uint32_t cols, uint32_t R,
                                    uint32_t T, uint32_t win, uint32_t baby, uint32_t n_limbs, double scale,
                                    fhe_pt** outs) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(outs != nullptr, "null outputs");
    const uint32_t nq = n_limbs ? n_limbs : ctx->c.L;
    fhe::require(nq <= ctx->c.L, "n_limbs above the number of Q primes");
    auto v = k.encode_replicated_diagonals(w_dev, m, cols, R, T, win, baby, nq, scale > 0 ? scale : k.level_scale(nq));
    for (uint32_t i = 0; i < T; ++i) outs[i] = new fhe_pt{std::move(v[i])};
  });
}

int fhe_linear_transform(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* const* diags, uint32_t baby,
                         uint32_t giant, int32_t stride, int32_t giant_offset, fhe_ct** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(diags != nullptr, "null diagonal array");
    std::vector<const fhe::Pt*> d((size_t)baby * giant);
    for (size_t i = 0; i < d.size(); ++i) d[i] = diags[i] ? diags[i]->p.get() : nullptr;
    put_ct(out, k.linear_transform(ct_of(a), d, baby, giant, stride, giant_offset));
  });
}

// ---- limb-sharded key switching ----------------------------------------

namespace {
fhe::ShardKeySwitch& shard_of(fhe_ctx* ctx) {
  ckks(ctx);
  fhe::require(ctx->shard != nullptr, "no shard set up (fhe_shard_init)", FHE_ERR_STATE);
  return *ctx->shard;
}
}  // namespace

int fhe_shard_init(fhe_ctx* ctx, uint32_t rank, uint32_t world) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    ctx->shard.reset();
    ctx->shard = std::make_unique<fhe::ShardKeySwitch>(k, rank, world);
  });
}

int fhe_shard_plan_get(fhe_ctx* ctx, uint32_t n_limbs, fhe_shard_plan* out) {
  return guarded([&] {
    fhe::require(out != nullptr, "null plan");
    const fhe::ShardPlan p = shard_of(ctx).plan(n_limbs);
    out->n_limbs = p.nq;
    out->q_own = p.q_own;
    out->q_chunk = p.q_chunk;
    out->p_own = p.p_own;
    out->p_chunk = p.p_chunk;
    out->rows = p.rows;
    out->digits = p.digits;
    out->reserved = 0;
  });
}

int fhe_shard_load_key(fhe_ctx* ctx, int32_t kind, uint64_t galois) {
  return guarded([&] { shard_of(ctx).load_key(kind, galois); });
}

int fhe_shard_modup_prepare(fhe_ctx* ctx, uint32_t n_limbs, const uint64_t* d_own, uint64_t* send) {
  return guarded([&] {
    fhe::require(send != nullptr && (d_own != nullptr || shard_of(ctx).plan(n_limbs).q_own == 0), "null buffer");
    shard_of(ctx).modup_prepare(n_limbs, d_own, send);
  });
}

int fhe_shard_inner(fhe_ctx* ctx, uint32_t n_limbs, int32_t kind, uint64_t galois, const uint64_t* gathered,
                    const uint64_t* d_own, uint64_t* acc, uint64_t* p_send) {
  return guarded([&] {
    const fhe::ShardPlan p = shard_of(ctx).plan(n_limbs);
    fhe::require(gathered != nullptr && (acc != nullptr || p.rows == 0) && (p_send != nullptr || p.p_chunk == 0) &&
                     (d_own != nullptr || p.q_own == 0),
                 "null buffer");
    shard_of(ctx).inner(n_limbs, kind, galois, gathered, d_own, acc, p_send);
  });
}

int fhe_shard_inner_digit(fhe_ctx* ctx, uint32_t n_limbs, uint32_t digit, const uint64_t* gathered_digit,
                          const uint64_t* d_own) {
  return guarded([&] {
    const fhe::ShardPlan p = shard_of(ctx).plan(n_limbs);
    fhe::require(gathered_digit != nullptr && (d_own != nullptr || p.q_own == 0), "null buffer");
    shard_of(ctx).inner_digit(n_limbs, digit, gathered_digit, d_own);
  });
}

int fhe_shard_inner_tail(fhe_ctx* ctx, uint32_t n_limbs, int32_t kind, uint64_t galois, uint64_t* acc,
                         uint64_t* p_send) {
  return guarded([&] {
    const fhe::ShardPlan p = shard_of(ctx).plan(n_limbs);
    fhe::require((acc != nullptr || p.rows == 0) && (p_send != nullptr || p.p_chunk == 0), "null buffer");
    shard_of(ctx).inner_tail(n_limbs, kind, galois, acc, p_send);
  });
}

int fhe_shard_moddown(fhe_ctx* ctx, uint32_t n_limbs, const uint64_t* acc, const uint64_t* p_gathered,
                      const uint64_t* add0, const uint64_t* add1, uint64_t* out) {
  return guarded([&] {
    const fhe::ShardPlan p = shard_of(ctx).plan(n_limbs);
    fhe::require(p.q_own == 0 || (acc != nullptr && p_gathered != nullptr && out != nullptr), "null buffer");
    shard_of(ctx).moddown(n_limbs, acc, p_gathered, add0, add1, out);
  });
}

int fhe_shard_automorphism(fhe_ctx* ctx, uint32_t n_limbs, uint64_t galois, const uint64_t* in, uint64_t* out) {
  return guarded([&] {
    fhe::require(shard_of(ctx).plan(n_limbs).q_own == 0 || (in != nullptr && out != nullptr && in != out),
                 "automorphism needs distinct buffers");
    shard_of(ctx).automorphism(n_limbs, galois, in, out);
  });
}

int fhe_ct_save(fhe_ctx* ctx, const fhe_ct* ct, const char* path) {
  return guarded([&] {
    fhe::require(path != nullptr, "null path");
    fhe::save_ciphertext(ckks(ctx), ct_of(ct), path);
  });
}

int fhe_ct_load(fhe_ctx* ctx, const char* path, fhe_ct** out) {
  return guarded([&] {
    fhe::require(path != nullptr, "null path");
    put_ct(out, fhe::load_ciphertext(ckks(ctx), path));
  });
}

int fhe_keys_save(fhe_ctx* ctx, const char* path, int32_t include_secret) {
  return guarded([&] {
    fhe::require(path != nullptr, "null path");
    ckks(ctx).save_keys(path, include_secret != 0);
  });
}

int fhe_keys_load(fhe_ctx* ctx, const char* path) {
  return guarded([&] {
    fhe::require(path != nullptr, "null path");
    ckks(ctx).load_keys(path);
  });
}

int fhe_ntt_butterfly_ceiling(fhe_ctx* ctx, double* butterflies_per_s) {
  return guarded([&] {
    fhe::require(ctx != nullptr && butterflies_per_s != nullptr, "null argument");
    fhe::Context& c = ctx->c;
    c.make_current();
    int sms = 0;
    FHE_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.device));
    const uint32_t blocks = (uint32_t)sms * 8;
    const int rounds = 64;
    fhe::DevMem out((size_t)blocks * 256 * 8), in(1024 * 8);
    std::vector<uint64_t> h(1024);
    for (size_t i = 0; i < h.size(); ++i) h[i] = 0x9E3779B97F4A7C15ull * (i + 1);
    FHE_CUDA(cudaMemcpy(in.p, h.data(), h.size() * 8, cudaMemcpyHostToDevice));
    const uint64_t q = c.primes[0];
    const uint64_t wv = c.roots[0] % q;
    const fhe::Twiddle w{wv, fhe::nt::shoup(wv, q)};
    cudaEvent_t e0, e1;
    FHE_CUDA(cudaEventCreate(&e0));
    FHE_CUDA(cudaEventCreate(&e1));
    for (int r = 0; r < 2; ++r)
      FHE_CUDA(fhe::ntt_butterfly_ceiling(q, w, out.as<uint64_t>(), in.as<uint64_t>(), blocks, rounds, c.stream));
    FHE_CUDA(cudaEventRecord(e0, c.stream));
    const int reps = 5;
    for (int r = 0; r < reps; ++r)
      FHE_CUDA(fhe::ntt_butterfly_ceiling(q, w, out.as<uint64_t>(), in.as<uint64_t>(), blocks, rounds, c.stream));
    FHE_CUDA(cudaEventRecord(e1, c.stream));
    FHE_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    FHE_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    const double bfly = (double)blocks * 256 * rounds * 8 * 8 * reps;
    *butterflies_per_s = bfly / (ms / 1e3);
  });
}

int fhe_kernel_launches(uint64_t* count) {
  if (!count) return FHE_ERR_INVALID;
  *count = fhe::g_kernel_launches.load();
  return FHE_OK;
}

int fhe_ctx_counters(fhe_ctx* ctx, fhe_counters* out, int32_t reset) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(out != nullptr, "null counters");
    const fhe::Counters& c = k.counters;
    *out = fhe_counters{c.tensor, c.relin, c.rotations, c.modup, c.moddown, c.key_inner, c.rescales, c.ntt_limbs,
                        c.bootstraps};
    if (reset) k.counters = fhe::Counters{};
  });
}

int fhe_ctx_set_conversion(fhe_ctx* ctx, int32_t kernel) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(kernel >= 0 && kernel <= 2,
                 "conversion kernel must be 0 (CUDA cores), 1 (tensor cores where faster) or 2 (tensor cores)");
    k.tc_conversion = kernel;
  });
}

int fhe_device_trim(int32_t device) {
  return guarded([&] {
    int count = 0;
    FHE_CUDA(cudaGetDeviceCount(&count));
    fhe::require(device >= 0 && device < count, "device ordinal out of range");
    FHE_CUDA(cudaSetDevice(device));
    FHE_CUDA(cudaDeviceSynchronize());
    cudaMemPool_t pool;
    FHE_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    FHE_CUDA(cudaMemPoolTrimTo(pool, 0));
  });
}

int fhe_ctx_set_keyswitch_fusion(fhe_ctx* ctx, int32_t fused) {
  return guarded([&] { ckks(ctx).fused_key_inner = fused != 0; });
}

int fhe_ctx_set_giant_hoisting(fhe_ctx* ctx, int32_t on) {
  return guarded([&] { ckks(ctx).hoist_giant_moddown = on != 0; });
}

int fhe_tc_timeouts(uint64_t* count) {
  return guarded([&] {
    fhe::require(count != nullptr, "null count");
    *count = fhe::tc_conversion_timeouts();
  });
}

int fhe_ctx_level_counts(fhe_ctx* ctx, int32_t kind, uint64_t* out, uint32_t n) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(out != nullptr, "null level counts");
    const fhe::Counters& c = k.counters;
    const uint64_t* src = kind == 0 ? c.modup_at : kind == 1 ? c.key_inner_at : kind == 2 ? c.rescale_at
                          : kind == 3 ? c.tensor_at : nullptr;
    fhe::require(src != nullptr, "level count kind must be 0 (ModUp), 1 (key inner product), 2 (rescale) or 3 (tensor)");
    for (uint32_t i = 0; i < n; ++i) out[i] = i < fhe::Counters::kLevels ? src[i] : 0;
  });
}

int fhe_bootstrap_setup(fhe_ctx* ctx, uint32_t budget_cts, uint32_t budget_stc, uint32_t slots,
                        int32_t correction, int32_t s2c_first, uint32_t sparse_h) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(slots == 0 || slots == ctx->c.slots, "bootstrap slots must equal the context's slot count", -1);
    fhe::BootParams p;
    p.budget_cts = budget_cts;
    p.budget_stc = budget_stc;
    p.correction = correction;
    p.s2c_first = s2c_first != 0;
    p.sparse_h = sparse_h;
    ctx->boot = std::make_unique<fhe::Bootstrapper>(k, p);
  });
}

int fhe_bootstrap_subslot_setup(fhe_ctx* ctx, uint32_t slots, uint32_t budget_cts, uint32_t budget_stc,
                                int32_t correction) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(slots >= 2 && slots < ctx->c.slots, "sub-slot refresh slots must be below the context's", -1);
    fhe::BootParams p;
    p.budget_cts = budget_cts;
    p.budget_stc = budget_stc;
    p.correction = correction;
    p.slots = slots;
    ctx->sub[slots] = std::make_unique<fhe::Bootstrapper>(k, p);
  });
}

int fhe_bootstrap_keygen(fhe_ctx* ctx) {
  return guarded([&] {
    ckks(ctx);
    fhe::require(ctx->boot != nullptr || !ctx->sub.empty(), "bootstrap keygen before bootstrap setup", -4);
    if (ctx->boot) ctx->boot->keygen();
    for (auto& [n, b] : ctx->sub) b->keygen();
  });
}

int fhe_bootstrap(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] {
    ckks(ctx);
    fhe::require(ctx->boot != nullptr, "bootstrap before bootstrap setup", -4);
    put_ct(out, ctx->boot->bootstrap(ct_of(a)));
  });
}

namespace {

// PackedEvaluator::refresh / bootstrap_components (packed_fideslib.cpp:235-281):
// bootstrap x / bound; with two passes the residual (x - first) * 4096 is
// bootstrapped again and added back / 4096; the result is scaled by bound.
// A sub-slot bootstrapper gets each input replicated with period n first
// (its inputs are zero outside [0, n)); its outputs are zero there again.
std::unique_ptr<fhe::Ct> refresh_with(fhe::Ckks& k, fhe::Bootstrapper& b, bool sub, const fhe::Ct& a, double bound,
                                      int32_t passes) {
  fhe::require(passes == 1 || passes == 2, "refresh passes must be 1 or 2");
  fhe::require(std::isfinite(bound) && bound > 0, "refresh bound must be positive");
  auto boot = [&](const fhe::Ct& v) { return sub ? b.bootstrap(*b.replicate(v)) : b.bootstrap(v); };
  auto x = k.mul_scalar(a, 1.0 / bound);
  if (x->noise_deg > 1) x = k.rescaled(*x);
  auto first = boot(*x);
  std::unique_ptr<fhe::Ct> r;
  if (passes == 1) {
    r = k.mul_scalar(*first, bound);
  } else {
    auto residual = k.mul_scalar(*k.add(*x, *first, true), 4096.0);
    if (residual->noise_deg > 1) residual = k.rescaled(*residual);
    auto second = boot(*residual);
    r = k.mul_scalar(*k.add(*first, *k.mul_scalar(*second, 1.0 / 4096.0), false), bound);
  }
  if (r->noise_deg > 1) r = k.rescaled(*r);
  return r;
}

}  // namespace

int fhe_refresh(fhe_ctx* ctx, const fhe_ct* a, double bound, int32_t passes, fhe_ct** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(ctx->boot != nullptr, "refresh before bootstrap setup", -4);
    put_ct(out, refresh_with(k, *ctx->boot, false, ct_of(a), bound, passes));
  });
}

int fhe_refresh_support(fhe_ctx* ctx, const fhe_ct* a, double bound, int32_t passes, uint32_t support,
                        fhe_ct** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    // the smallest sub-slot bootstrapper covering [0, support), else the full one
    auto it = support ? ctx->sub.lower_bound(support) : ctx->sub.end();
    if (it != ctx->sub.end()) {
      put_ct(out, refresh_with(k, *it->second, true, ct_of(a), bound, passes));
      return;
    }
    fhe::require(ctx->boot != nullptr, "refresh before bootstrap setup", -4);
    put_ct(out, refresh_with(k, *ctx->boot, false, ct_of(a), bound, passes));
  });
}

int fhe_bootstrap_stage(fhe_ctx* ctx, int32_t stage, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] {
    ckks(ctx);
    fhe::require(ctx->boot != nullptr, "bootstrap before bootstrap setup", -4);
    fhe::Bootstrapper& b = *ctx->boot;
    switch (stage) {
      case 0: put_ct(out, b.raise(ct_of(a))); break;
      case 1: put_ct(out, b.coeff_to_slot(ct_of(a))); break;
      case 2: put_ct(out, b.eval_mod_full(ct_of(a))); break;
      case 3: put_ct(out, b.slot_to_coeff(ct_of(a))); break;
      default: fhe::require(false, "bootstrap stage must be 0..3", -1);
    }
  });
}

int fhe_bootstrap_info(fhe_ctx* ctx, int32_t* correction, uint32_t* cheb_degree, uint32_t* n_rotation_keys) {
  return guarded([&] {
    ckks(ctx);
    fhe::require(ctx->boot != nullptr, "no bootstrap setup", -4);
    if (correction) *correction = ctx->boot->correction();
    if (cheb_degree) *cheb_degree = (uint32_t)ctx->boot->eval_mod_coefficients().size() - 1;
    if (n_rotation_keys) *n_rotation_keys = (uint32_t)ctx->boot->rotation_steps().size() + 1;
  });
}

int fhe_bootstrap_levels(fhe_ctx* ctx, uint32_t* levels) {
  return guarded([&] {
    ckks(ctx);
    fhe::require(ctx->boot != nullptr && levels != nullptr, "no bootstrap setup or null output", -4);
    for (int i = 0; i < 4; ++i) levels[i] = ctx->boot->last_levels()[i];
  });
}

int fhe_program_validate(const char* program_path, int32_t* slots, int32_t* nodes, int32_t* outputs) {
  return guarded([&] {
    fhe::require(program_path != nullptr, "null program path");
    std::ifstream in(program_path);
    fhe::require((bool)in, std::string("cannot open program ") + program_path);
    const fhe::PackedProgram prog = fhe::read_packed_program(in);
    if (slots) *slots = prog.slots;
    if (nodes) *nodes = (int32_t)prog.nodes.size();
    if (outputs) *outputs = (int32_t)prog.outputs.size();
  });
}

namespace {
// Classical-128 parameter audit (the reference's CkksSecurityAudit,
// native/fideslib_stage0/src/fideslib_security.hpp:18-80): exact bit lengths
// of Q, P and Q*P against the 2024 Security Guidelines Table 5.2 bound for
// the ring (uniform ternary secret, error sigma >= 3.19).
uint32_t product_bit_length(const std::vector<uint64_t>& m) {
  std::vector<uint32_t> x{1};  // little-endian 32-bit words
  for (uint64_t q : m) {
    std::vector<uint32_t> y(x.size() + 2, 0);
    for (size_t i = 0; i < x.size(); ++i) {
      unsigned __int128 carry = 0;
      for (size_t j = 0; j < 2; ++j) {
        const uint64_t qj = j == 0 ? (uint32_t)q : (uint32_t)(q >> 32);
        const unsigned __int128 t = (unsigned __int128)x[i] * qj + y[i + j] + carry;
        y[i + j] = (uint32_t)t;
        carry = t >> 32;
      }
      for (size_t k = i + 2; carry; ++k) {
        const unsigned __int128 t = (unsigned __int128)y[k] + carry;
        y[k] = (uint32_t)t;
        carry = t >> 32;
      }
    }
    while (y.size() > 1 && y.back() == 0) y.pop_back();
    x.swap(y);
  }
  uint32_t bits = 32 * (uint32_t)(x.size() - 1), top = x.back();
  while (top) { ++bits; top >>= 1; }
  return bits;
}

uint32_t classical128_bound(uint32_t ring) {
  switch (ring) {
    case 1024: return 26;
    case 2048: return 53;
    case 4096: return 106;
    case 8192: return 214;
    case 16384: return 430;
    case 32768: return 868;
    case 65536: return 1747;
    case 131072: return 3523;
    default: return 0;
  }
}

struct SecurityAudit {
  uint32_t ring = 0, q_bits = 0, p_bits = 0, qp_bits = 0, q_towers = 0, p_towers = 0, digits = 0, bound = 0;
  double sigma = 0;
  bool passed() const { return bound && sigma >= 3.19 && q_towers && p_towers && qp_bits <= bound; }
  std::string json() const {
    std::ostringstream o;
    o << "{\"ring_dimension\":" << ring << ",\"q_bits\":" << q_bits << ",\"p_bits\":" << p_bits
      << ",\"qp_bits\":" << qp_bits << ",\"q_towers\":" << q_towers << ",\"p_towers\":" << p_towers
      << ",\"hybrid_digits\":" << digits << ",\"error_sigma\":" << sigma
      << ",\"guideline_max_qp_bits\":" << bound << ",\"library_classical128\":true"
      << ",\"uniform_ternary\":true,\"hybrid\":true,\"passed\":" << (passed() ? "true" : "false")
      << ",\"basis\":\"2024 Security Guidelines Table 5.2; classical RLWE parameter bound\"}";
    return o.str();
  }
};

SecurityAudit audit_moduli(uint32_t ring, const std::vector<uint64_t>& q, const std::vector<uint64_t>& p,
                           uint32_t dnum) {
  SecurityAudit a;
  a.ring = ring;
  std::vector<uint64_t> qp(q);
  qp.insert(qp.end(), p.begin(), p.end());
  a.q_bits = product_bit_length(q);
  a.p_bits = product_bit_length(p);
  a.qp_bits = product_bit_length(qp);
  a.q_towers = (uint32_t)q.size();
  a.p_towers = (uint32_t)p.size();
  a.digits = dnum;
  a.sigma = std::sqrt(21.0 / 2.0);  // centred binomial error, eta = 21
  a.bound = classical128_bound(ring);
  return a;
}

SecurityAudit audit_parameters(const fhe::Context& c) {
  const std::vector<uint64_t> q(c.primes.begin(), c.primes.begin() + c.L), p(c.primes.begin() + c.L, c.primes.end());
  return audit_moduli(c.n, q, p, c.dnum);
}
}  // namespace

int fhe_security_audit(uint32_t log_n, uint32_t depth, uint32_t scale_bits, uint32_t first_bits, uint32_t dnum,
                       char* json, size_t len, int32_t* passed) {
  return guarded([&] {
    fhe::require(log_n >= 10 && log_n <= 17, "log_n must be in [10, 17]");
    std::vector<uint64_t> q, p;
    fhe::nt::ckks_moduli(log_n, depth + 1, scale_bits, first_bits, dnum, q, p);
    const SecurityAudit a = audit_moduli(1u << log_n, q, p, dnum);
    const std::string j = a.json();
    fhe::require(json == nullptr || len > j.size(), "audit buffer too small");
    if (json) std::memcpy(json, j.c_str(), j.size() + 1);
    if (passed) *passed = a.passed() ? 1 : 0;
  });
}

int fhe_program_run(const char* program_path, const char* client_head_path, const char* result_path,
                    double poly_tol, double exact_tol, const fhe_program_options* options) {
  int verdict = 0;
  const int rc = guarded([&] {
    fhe::require(program_path && result_path, "null program or result path");
    fhe::require(std::isfinite(poly_tol) && std::isfinite(exact_tol) && poly_tol > 0 && exact_tol > 0,
                 "invalid error tolerance");
    fhe_program_options o{};
    if (options) o = *options;
    if (o.security128) {
      // packed_fideslib.cpp:1060-1076: ring 2^17, dnum = security digits,
      // batch size = the program's slots, uniform ternary secret
      fhe::require(o.sparse_h == 0, "128-classic requires the uniform ternary secret");
      if (!o.log_n) o.log_n = 17;
      o.dnum = o.security_digits ? o.security_digits : 4;
      fhe::require(o.dnum >= 1 && o.dnum <= 16, "security digits must be in [1, 16]");
    } else {
      fhe::require(o.security_digits == 0, "security digits apply to --security 128-classic only");
    }
    if (!o.depth) o.depth = 44;
    if (!o.scale_bits) o.scale_bits = 59;
    if (!o.first_bits) o.first_bits = 60;
    if (!o.dnum) o.dnum = 3;
    if (!o.bootstrap_passes) o.bootstrap_passes = 2;
    fhe::require(o.bootstrap_passes == 1 || o.bootstrap_passes == 2, "bootstrap passes must be 1 or 2");
    using Clock = std::chrono::steady_clock;
    auto since = [](Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); };
    std::ifstream in(program_path);
    fhe::require((bool)in, std::string("cannot open program ") + program_path);
    const fhe::PackedProgram prog = fhe::read_packed_program(in);
    uint32_t log_n = o.log_n;
    if (!log_n) {
      log_n = 12;
      while ((1u << (log_n - 1)) < (uint32_t)prog.slots) ++log_n;
    }
    fhe::require((1u << (log_n - 1)) >= (uint32_t)prog.slots, "ring too small for the program's slots");
    fhe::GenerationClient client;
    const bool with_client = client_head_path && *client_head_path;
    if (with_client) {
      client.load(client_head_path);
      fhe::require(prog.nodes[prog.outputs.back().node].size == (int)client.width,
                   "client head and final hidden width mismatch");
    }
    const auto setup0 = Clock::now();
    const uint32_t batch = o.security128 ? (uint32_t)prog.slots : 1u << (log_n - 1);
    fhe_params par{log_n, o.depth, o.scale_bits, o.first_bits, o.dnum, batch, o.device, 0};
    fhe_ctx* raw = nullptr;
    fhe::require(fhe_ctx_create(&par, &raw) == FHE_OK, g_last_error);
    std::unique_ptr<fhe_ctx, int (*)(fhe_ctx*)> ctx(raw, fhe_ctx_destroy);
    std::string audit_json = "null";
    if (o.security128) {
      const SecurityAudit a = audit_parameters(ctx->c);
      audit_json = a.json();
      std::ofstream pj(std::string(result_path) + ".parameters.json");
      fhe::require((bool)pj, "cannot write the parameters audit");
      pj << audit_json << "\n";
      std::cout << "classical128 ring=" << a.ring << " QP_bits=" << a.qp_bits << " bound=" << a.bound
                << " digits=" << a.digits << std::endl;
      fhe::require(a.passed(), "classical-128 CKKS audit failed: HYBRID Q*P (" + std::to_string(a.qp_bits) +
                                   " bits) exceeds the published bound for ring " + std::to_string(a.ring));
    }
    fhe::Ckks& ck = *ctx->ck;
    ck.keygen(o.seed ? o.seed : 1);
    const bool can_boot = ctx->c.L > 4 + 4 + 2 + 21;
    if (can_boot) {
      fhe::BootParams bp;
      bp.s2c_first = o.s2c_first != 0;
      bp.sparse_h = o.sparse_h;
      ctx->boot = std::make_unique<fhe::Bootstrapper>(ck, bp);
      ctx->boot->keygen();
    }
    FHE_CUDA(cudaStreamSynchronize(ctx->c.stream));
    const double setup_seconds = since(setup0);
    fhe::ExecutorOptions eo;
    eo.bootstrap_passes = o.bootstrap_passes;
    eo.trace = o.trace != 0;
    fhe::PackedExecutor ex(ck, ctx->boot.get(), prog, eo);
    std::map<int, size_t> output_pos;
    for (size_t i = 0; i < prog.outputs.size(); ++i) output_pos.emplace(prog.outputs[i].node, i);
    std::vector<int> feedback_outputs;
    for (const auto& nd : prog.nodes)
      if (nd.op == "feedback") {
        auto it = output_pos.find(nd.parents.at(0));
        feedback_outputs.push_back(it == output_pos.end() ? -1 : (int)it->second);
      }
    auto checked_hidden = [&](const fhe::Ct& hidden, int out_index) {
      auto values = ex.decrypt(hidden, (int)client.width);
      if (out_index >= 0) {
        const auto e = fhe::packed_output_errors(values, prog.outputs.at(out_index));
        fhe::require(!e.non_finite && e.polynomial <= poly_tol && e.exact <= exact_tol,
                     "client hidden fails reference tolerance before token " +
                         std::to_string(client.tokens.size() + 1), -4);
      }
      return values;
    };
    if (with_client)
      ex.client_feedback = [&](const fhe::Ct& hidden) {
        return ex.encrypt(client.select(checked_hidden(hidden, feedback_outputs.at(client.tokens.size()))));
      };
    const auto eval0 = Clock::now();
    auto outs = ex.evaluate();
    FHE_CUDA(cudaStreamSynchronize(ctx->c.stream));
    const double eval_seconds = since(eval0);
    if (with_client) client.select(checked_hidden(*outs.back(), (int)prog.outputs.size() - 1));
    double perr = 0, eerr = 0;
    int non_finite = 0;
    std::vector<double> per_poly, per_exact;
    for (size_t i = 0; i < prog.outputs.size(); ++i) {
      const auto values = ex.decrypt(*outs[i], (int)prog.outputs[i].polynomial.size());
      const auto e = fhe::packed_output_errors(values, prog.outputs[i]);
      non_finite += e.non_finite;
      perr = std::max(perr, e.polynomial);
      eerr = std::max(eerr, e.exact);
      per_poly.push_back(e.polynomial);
      per_exact.push_back(e.exact);
    }
    const bool passed = non_finite == 0 && perr <= poly_tol && eerr <= exact_tol;
    std::ofstream r(result_path);
    fhe::require((bool)r, std::string("cannot open result ") + result_path);
    r << std::setprecision(12) << "{\n\"schema\":\"fhemamba-packed-result-v1\",\"backend\":\"fhe_b200\","
      << "\"encrypted\":true,\"security\":\"" << (o.security128 ? "128-classic" : "not-set")
      << "\",\"passed\":" << (passed ? "true" : "false")
      << ",\"slots\":" << ctx->c.slots << ",\"payload_slots\":" << prog.slots
      << ",\"ring_dimension\":" << ctx->c.n << ",\"depth\":" << o.depth << ",\"scale_bits\":" << o.scale_bits
      << ",\"refresh_ring_dimension\":" << ctx->c.n << ",\"security_audit\":" << audit_json
      << ",\"nodes\":" << prog.nodes.size() << ",\"setup_seconds\":" << setup_seconds
      << ",\"s2c_first\":" << (o.s2c_first ? "true" : "false")
      << ",\"refresh_ceiling\":" << ex.refresh_ceiling << ",\"refreshed_level\":" << ex.refreshed_level
      << ",\"evaluated_nodes\":" << prog.nodes.size() << ",\"eval_seconds\":" << eval_seconds
      << ",\"bootstrap_seconds\":" << ex.bootstrap_seconds << ",\"bootstraps\":" << ex.bootstraps
      << ",\"ct_ct_mul\":" << ex.ct_ct << ",\"ct_pt_mul\":" << ex.ct_pt << ",\"rotations\":" << ex.rotations
      << ",\"adds\":" << ex.adds << ",\"rotation_keys_generated\":" << ex.rotation_keys_generated
      << ",\"rotation_keygen_seconds\":" << ex.keygen_seconds
      << ",\"linear_method\":\"bsgs\",\"refresh_policy\":\"baseline\",\"bootstrap_passes\":" << o.bootstrap_passes
      << ",\"logical_refreshes\":" << ex.logical_refreshes
      << ",\"max_abs_error_vs_polynomial\":" << perr << ",\"max_abs_error_vs_exact\":" << eerr
      << ",\"non_finite\":" << non_finite << ",\"polynomial_tolerance\":" << poly_tol
      << ",\"exact_tolerance\":" << exact_tol << ",\"per_output_errors\":[";
    for (size_t i = 0; i < per_poly.size(); ++i)
      r << (i ? "," : "") << "{\"polynomial\":" << per_poly[i] << ",\"exact\":" << per_exact[i] << "}";
    r << "],\"diagnostic_only\":false,\"evaluation_decryptions\":0,\"client_output_decrypt_count\":"
      << client.tokens.size() << ",\"generated_token_ids\":[";
    for (size_t i = 0; i < client.tokens.size(); ++i) r << (i ? "," : "") << client.tokens[i];
    r << "],\"client_logit_margins\":[";
    for (size_t i = 0; i < client.margins.size(); ++i) r << (i ? "," : "") << client.margins[i];
    r << "],\"operation_stats\":{";
    bool first = true;
    for (const auto& [name, st] : ex.operation_stats) {
      r << (first ? "" : ",") << "\"" << name << "\":{\"nodes\":" << st.nodes << ",\"seconds\":" << st.seconds
        << ",\"bootstrap_seconds\":" << st.bootstrap_seconds << ",\"bootstraps\":" << st.bootstraps << "}";
      first = false;
    }
    r << "},\"scope\":\"" << (with_client ? "encrypted backbone with inline client vocabulary head and actual greedy feedback"
                                           : "packed feasibility; inline client fixture")
      << "\"}\n";
    fhe::require((bool)r, "could not write packed result");
    std::cout << "passed=" << passed << " polynomial_error=" << perr << " exact_error=" << eerr
              << " eval_seconds=" << eval_seconds << std::endl;
    verdict = passed ? 0 : 1;
  });
  return rc != FHE_OK ? rc : verdict;
}

int fhe_mod_raise(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).mod_raise(ct_of(a))); });
}

int fhe_mul_i(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out) {
  return guarded([&] { put_ct(out, ckks(ctx).mul_i(ct_of(a))); });
}

int fhe_ct_set_scale(fhe_ctx* ctx, fhe_ct* ct, double scale) {
  return guarded([&] {
    ckks(ctx);
    fhe::require(ct != nullptr && ct->p != nullptr && scale > 0, "null ciphertext or non-positive scale");
    ct->p->scale = scale;
  });
}

int fhe_chebyshev(fhe_ctx* ctx, const fhe_ct* a, const double* coeffs, uint32_t n, double lo, double hi,
                  fhe_ct** out) {
  return guarded([&] {
    fhe::Ckks& k = ckks(ctx);
    fhe::require(coeffs != nullptr && n >= 1, "need at least one coefficient");
    put_ct(out, k.chebyshev(ct_of(a), std::vector<double>(coeffs, coeffs + n), lo, hi));
  });
}

}  // extern "C"
