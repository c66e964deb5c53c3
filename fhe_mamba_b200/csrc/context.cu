// Context set-up: moduli generation, device tables, stream and buffers.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>

#include "context.h"
#include "launch_count.h"

namespace fhe {

std::atomic<uint64_t> g_kernel_launches{0};


typedef unsigned __int128 u128;

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw Error(-2, std::string(what) + ": " + cudaGetErrorString(e));
}

void require(bool ok, const std::string& msg, int code) {
  if (!ok) throw Error(code, msg);
}

StreamHolder::~StreamHolder() {
  if (s) {
    cudaSetDevice(device);
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
  }
}

DevMem::DevMem(size_t b) : bytes(b) {
  if (b == 0) return;
  cudaError_t e = cudaMalloc(&p, b);
  if (e != cudaSuccess) {
    p = nullptr;
    bytes = 0;
    throw Error(-3, std::string("cudaMalloc(") + std::to_string(b) + "): " + cudaGetErrorString(e));
  }
}

DevMem::DevMem(size_t b, const std::shared_ptr<StreamHolder>& stream) : bytes(b), sh(stream) {
  if (b == 0) return;
  cudaError_t e = cudaMallocAsync(&p, b, sh->s);
  if (e != cudaSuccess) {
    p = nullptr;
    bytes = 0;
    throw Error(-3, std::string("cudaMallocAsync(") + std::to_string(b) + "): " + cudaGetErrorString(e));
  }
}

void DevMem::release() {
  if (p) {
    if (sh) cudaFreeAsync(p, sh->s);
    else cudaFree(p);
  }
  p = nullptr;
  bytes = 0;
  sh.reset();
}

DevMem::~DevMem() { release(); }

DevMem& DevMem::operator=(DevMem&& o) noexcept {
  if (this != &o) {
    release();
    p = o.p;
    bytes = o.bytes;
    sh = std::move(o.sh);
    o.p = nullptr;
    o.bytes = 0;
  }
  return *this;
}

namespace nt {

uint64_t mulmod(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }

uint64_t powmod(uint64_t a, uint64_t e, uint64_t q) {
  uint64_t r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = mulmod(r, a, q);
    a = mulmod(a, a, q);
    e >>= 1;
  }
  return r;
}

uint64_t invmod(uint64_t a, uint64_t q) { return powmod(a, q - 2, q); }

// Deterministic Miller-Rabin (first twelve prime bases cover n < 2^64).
bool is_prime(uint64_t n) {
  static const uint64_t bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  if (n < 2) return false;
  for (uint64_t b : bases) {
    if (n == b) return true;
    if (n % b == 0) return false;
  }
  uint64_t d = n - 1;
  int s = 0;
  while (!(d & 1)) { d >>= 1; ++s; }
  for (uint64_t b : bases) {
    uint64_t x = powmod(b, d, n);
    if (x == 1 || x == n - 1) continue;
    bool composite = true;
    for (int r = 1; r < s && composite; ++r) {
      x = mulmod(x, x, n);
      if (x == n - 1) composite = false;
    }
    if (composite) return false;
  }
  return true;
}

uint64_t first_prime(uint32_t bits, uint64_t m) {
  const uint64_t base = uint64_t(1) << bits;
  uint64_t c = base + 1;
  if (base % m) c += m - base % m;
  while (!is_prime(c)) c += m;
  return c;
}

uint64_t previous_prime(uint64_t q, uint64_t m) {
  uint64_t c = q - m;
  while (!is_prime(c)) c -= m;
  return c;
}

uint64_t next_prime(uint64_t q, uint64_t m) {
  uint64_t c = q + m;
  while (!is_prime(c)) c += m;
  return c;
}

uint64_t min_root_of_unity(uint64_t m, uint64_t q) {
  uint64_t g = 0;
  for (uint64_t x = 2;; ++x) {
    g = powmod(x, (q - 1) / m, q);
    if (powmod(g, m / 2, q) == q - 1) break;
  }
  const uint64_t g2 = mulmod(g, g, q);
  uint64_t x = g, best = g;
  for (uint64_t k = 3; k < m; k += 2) {
    x = mulmod(x, g2, q);
    best = std::min(best, x);
  }
  return best;
}

uint64_t shoup(uint64_t w, uint64_t q) { return (uint64_t)(((u128)w << 64) / q); }

uint32_t bitlen(uint64_t x) {
  uint32_t b = 0;
  while (x) { ++b; x >>= 1; }
  return b;
}

static uint32_t product_bits(const uint64_t* m, size_t n) {
  std::vector<uint64_t> acc{1};
  for (size_t i = 0; i < n; ++i) {
    u128 carry = 0;
    for (auto& w : acc) {
      u128 t = (u128)w * m[i] + carry;
      w = (uint64_t)t;
      carry = t >> 64;
    }
    if (carry) acc.push_back((uint64_t)carry);
  }
  return 64 * (uint32_t)(acc.size() - 1) + bitlen(acc.back());
}

// Same selection rule as OpenFHE v1.4.2 for FLEXIBLEAUTO + HYBRID: the top
// prime is FirstPrime(scale_bits); going down, q_i tracks the level scaling
// factor sf_i = sf_{i+1}^2 / q_{i+1}, alternating the nearest prime below and
// above (skipping repeats); q_0 = PreviousPrime(FirstPrime(first_bits)).
// P: ceil(max digit bits / 60) primes PreviousPrime-descending from
// FirstPrime(60), skipping Q primes.
void ckks_moduli(uint32_t log_n, uint32_t num_q, uint32_t scale_bits, uint32_t first_bits,
                 uint32_t dnum, std::vector<uint64_t>& q, std::vector<uint64_t>& p) {
  require(num_q >= 2 && num_q <= 64, "number of Q primes must be in [2, 64]");
  require(dnum >= 1, "num_large_digits must be >= 1");
  // Barrett reductions of raw 64-bit words need primes of at least 33 bits.
  require(scale_bits >= 33 && scale_bits <= 60 && first_bits >= 33 && first_bits <= 60,
          "modulus sizes must be in [33, 60] bits");
  require(first_bits != scale_bits, "first_mod_size must differ from scaling_mod_size");
  const uint64_t m = uint64_t(2) << log_n;
  q.assign(num_q, 0);
  q[num_q - 1] = first_prime(scale_bits, m);
  auto seen = [&](uint64_t v, size_t from) {
    return std::find(q.begin() + from, q.end(), v) != q.end();
  };
  double sf = (double)q[num_q - 1];
  uint32_t cnt = 0;
  for (int i = (int)num_q - 2; i >= 1; --i) {
    sf = std::pow(sf, 2) / (double)q[i + 1];
    const uint64_t sf_int = (uint64_t)std::llround(sf);
    const uint64_t rem = sf_int % m;
    if (cnt % 2 == 0) {
      uint64_t c = sf_int - m - rem + 1;
      do { c = previous_prime(c, m); } while (seen(c, i + 1));
      q[i] = c;
    } else {
      uint64_t c = sf_int + m - rem + 1;
      do { c = next_prime(c, m); } while (seen(c, i + 1));
      q[i] = c;
    }
    ++cnt;
  }
  q[0] = previous_prime(first_prime(first_bits, m), m);

  const uint32_t alpha = (num_q + dnum - 1) / dnum;
  uint32_t max_bits = 0;
  for (uint32_t lo = 0; lo < num_q; lo += alpha)
    max_bits = std::max(max_bits, product_bits(q.data() + lo, std::min(alpha, num_q - lo)));
  const uint32_t size_p = (max_bits + 59) / 60;
  p.clear();
  uint64_t prev = first_prime(60, m);
  for (uint32_t i = 0; i < size_p; ++i) {
    uint64_t c;
    do { c = previous_prime(prev, m); prev = c; } while (std::find(q.begin(), q.end(), c) != q.end());
    p.push_back(c);
  }
}

}  // namespace nt

Context::~Context() {
  if (stream) {
    cudaSetDevice(device);
    cudaStreamSynchronize(stream);
  }
}

void Context::make_current() const { FHE_CUDA(cudaSetDevice(device)); }

static uint32_t bitrev(uint32_t x, uint32_t bits) {
  uint32_t r = 0;
  for (uint32_t i = 0; i < bits; ++i) { r = (r << 1) | (x & 1); x >>= 1; }
  return r;
}

// Roots, twiddle tables (psi^{+-brv(i)} with Shoup companions), Barrett
// constants and the folded 1/N constants, computed on host threads and
// uploaded once.
void Context::build_tables() {
  const uint32_t np = n_primes();
  const uint64_t m = uint64_t(2) * n;
  roots.assign(np, 0);
  std::vector<Twiddle> tw((size_t)np * n), twi((size_t)np * n), ninv(2 * (size_t)np);
  std::vector<Modulus> mods(np);
  auto work = [&](uint32_t i) {
    const uint64_t q = primes[i];
    const uint64_t psi = nt::min_root_of_unity(m, q);
    const uint64_t psi_inv = nt::invmod(psi, q);
    roots[i] = psi;
    uint64_t x = 1, y = 1;
    Twiddle* f = tw.data() + (size_t)i * n;
    Twiddle* g = twi.data() + (size_t)i * n;
    for (uint32_t j = 0; j < n; ++j) {
      const uint32_t r = bitrev(j, log_n);
      f[r] = Twiddle{x, nt::shoup(x, q)};
      g[r] = Twiddle{y, nt::shoup(y, q)};
      x = nt::mulmod(x, psi, q);
      y = nt::mulmod(y, psi_inv, q);
    }
    const uint64_t ni = nt::invmod(n % q, q);
    const uint64_t wn = nt::mulmod(g[1].w, ni, q);
    ninv[2 * i] = Twiddle{ni, nt::shoup(ni, q)};
    ninv[2 * i + 1] = Twiddle{wn, nt::shoup(wn, q)};
    const uint32_t b = nt::bitlen(q);
    const uint64_t r64 = (uint64_t)(((u128)1 << 64) % q);
    mods[i] = Modulus{q, (uint64_t)(((u128)1 << (2 * b)) / q), b, 0, r64, nt::shoup(r64, q), nt::shoup(1, q)};
  };
  // Row-pass round-2 twiddles: for row r, thread t and the j-th twiddle the
  // thread uses (forward: half-distances T/2..1, inverse: 1..T/2, groups g in
  // steps of 2h), entry = table[n/(2h) + r*(S/(2h)) + (R*t + g)/(2h)].
  int rows = 0, R = 0, T = 0, J = 0;
  ntt_row_shape((int)log_n, rows, R, T, J);
  const uint32_t S = n / rows;
  tw2_stride = (uint32_t)rows * J * T;
  std::vector<Twiddle> tw2((size_t)np * tw2_stride), tw2i((size_t)np * tw2_stride);
  auto work2 = [&](uint32_t i) {
    const Twiddle* f = tw.data() + (size_t)i * n;
    const Twiddle* g = twi.data() + (size_t)i * n;
    for (int r = 0; r < rows; ++r) {
      int j = 0;
      for (int h = T / 2; h >= 1; h >>= 1)
        for (int gg = 0; gg < R; gg += 2 * h, ++j)
          for (int t = 0; t < T; ++t)
            tw2[(size_t)i * tw2_stride + ((size_t)r * J + j) * T + t] =
                f[n / (2 * h) + r * (S / (2 * h)) + (R * t + gg) / (2 * h)];
      j = 0;
      for (int h = 1; h <= T / 2; h <<= 1)
        for (int gg = 0; gg < R; gg += 2 * h, ++j)
          for (int t = 0; t < T; ++t)
            tw2i[(size_t)i * tw2_stride + ((size_t)r * J + j) * T + t] =
                g[n / (2 * h) + r * (S / (2 * h)) + (R * t + gg) / (2 * h)];
    }
  };
  const uint32_t nthreads = std::max(1u, std::min<uint32_t>(np, std::thread::hardware_concurrency()));
  std::vector<std::thread> pool;
  for (uint32_t t = 0; t < nthreads; ++t)
    pool.emplace_back([&, t] {
      for (uint32_t i = t; i < np; i += nthreads) work(i);
    });
  for (auto& th : pool) th.join();
  pool.clear();
  if (tw2_stride)
    for (uint32_t t = 0; t < nthreads; ++t)
      pool.emplace_back([&, t] {
        for (uint32_t i = t; i < np; i += nthreads) work2(i);
      });
  for (auto& th : pool) th.join();

  d_primes = DevMem(np * sizeof(uint64_t));
  d_mod = DevMem(np * sizeof(Modulus));
  d_tw = DevMem(tw.size() * sizeof(Twiddle));
  d_tw_inv = DevMem(twi.size() * sizeof(Twiddle));
  d_ninv = DevMem(ninv.size() * sizeof(Twiddle));
  FHE_CUDA(cudaMemcpy(d_primes.p, primes.data(), np * sizeof(uint64_t), cudaMemcpyHostToDevice));
  FHE_CUDA(cudaMemcpy(d_mod.p, mods.data(), np * sizeof(Modulus), cudaMemcpyHostToDevice));
  FHE_CUDA(cudaMemcpy(d_tw.p, tw.data(), tw.size() * sizeof(Twiddle), cudaMemcpyHostToDevice));
  FHE_CUDA(cudaMemcpy(d_tw_inv.p, twi.data(), twi.size() * sizeof(Twiddle), cudaMemcpyHostToDevice));
  FHE_CUDA(cudaMemcpy(d_ninv.p, ninv.data(), ninv.size() * sizeof(Twiddle), cudaMemcpyHostToDevice));
  if (tw2_stride) {
    d_tw2 = DevMem(tw2.size() * sizeof(Twiddle));
    d_tw2_inv = DevMem(tw2i.size() * sizeof(Twiddle));
    FHE_CUDA(cudaMemcpy(d_tw2.p, tw2.data(), tw2.size() * sizeof(Twiddle), cudaMemcpyHostToDevice));
    FHE_CUDA(cudaMemcpy(d_tw2_inv.p, tw2i.data(), tw2i.size() * sizeof(Twiddle), cudaMemcpyHostToDevice));
  }
}

uint64_t* Context::stage(size_t words) {
  if (d_stage.bytes < words * sizeof(uint64_t)) {
    FHE_CUDA(cudaStreamSynchronize(stream));
    d_stage = DevMem(words * sizeof(uint64_t));
  }
  return d_stage.as<uint64_t>();
}

NttArgs Context::ntt_args(uint64_t* data, uint32_t n_polys, uint32_t prime0, uint32_t n_limbs,
                          uint32_t limb_stride) const {
  NttArgs a;
  a.data = data;
  a.tw = d_tw.as<Twiddle>();
  a.tw_inv = d_tw_inv.as<Twiddle>();
  a.primes = d_primes.as<uint64_t>();
  a.ninv = d_ninv.as<Twiddle>();
  a.tw2 = d_tw2.as<Twiddle>();
  a.tw2_inv = d_tw2_inv.as<Twiddle>();
  a.tw2_stride = tw2_stride;
  a.log_n = (int)log_n;
  a.n_polys = n_polys;
  a.n_limbs = n_limbs;
  a.limb_stride = limb_stride;
  a.prime0 = prime0;
  a.stream = stream;
  uint64_t qmax = 0;
  for (uint32_t i = prime0; i < prime0 + n_limbs && i < primes.size(); ++i) qmax = std::max(qmax, primes[i]);
  a.lazy = qmax < (uint64_t(1) << 59) ? 32 : qmax < (uint64_t(1) << 60) ? 16 : 0;
  return a;
}

}  // namespace fhe
