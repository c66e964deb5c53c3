// extern "C" entry points of libfhe_b200.so (declared in include/fhe_b200.h).
#include <cstring>
#include <memory>
#include <new>
#include <string>

#include "../../include/fhe_b200.h"
#include "context.h"

struct fhe_ctx {
  fhe::Context c;
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
  FHE_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
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

}  // extern "C"
