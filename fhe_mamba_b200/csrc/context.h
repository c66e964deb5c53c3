// Host-side context of the fhe_b200 backend: moduli, device tables, stream.
#pragma once
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "modarith.cuh"
#include "ntt.h"

namespace fhe {

// Error carrying one of the FHE_ERR_* codes across the C ABI.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void cuda_check(cudaError_t e, const char* what);
#define FHE_CUDA(call) ::fhe::cuda_check((call), #call)
void require(bool ok, const std::string& msg, int code = -1);

// CUDA stream shared by a context and every buffer allocated on it; the
// stream is destroyed when the last owner goes away.
struct StreamHolder {
  int device = 0;
  cudaStream_t s = nullptr;
  ~StreamHolder();
};

// Owning device allocation.  With a StreamHolder the memory comes from the
// device's stream-ordered pool (cudaMallocAsync / cudaFreeAsync on that
// stream), so allocating and freeing ciphertexts never synchronises.
struct DevMem {
  void* p = nullptr;
  size_t bytes = 0;
  std::shared_ptr<StreamHolder> sh;
  DevMem() = default;
  explicit DevMem(size_t b);
  DevMem(size_t b, const std::shared_ptr<StreamHolder>& stream);
  ~DevMem();
  DevMem(const DevMem&) = delete;
  DevMem& operator=(const DevMem&) = delete;
  DevMem(DevMem&& o) noexcept : p(o.p), bytes(o.bytes), sh(std::move(o.sh)) { o.p = nullptr; o.bytes = 0; }
  DevMem& operator=(DevMem&& o) noexcept;
  void release();
  template <class T>
  T* as() const { return static_cast<T*>(p); }
};

// Host-side number theory used at context set-up (not on the hot path).
namespace nt {
uint64_t mulmod(uint64_t a, uint64_t b, uint64_t q);
uint64_t powmod(uint64_t a, uint64_t e, uint64_t q);
uint64_t invmod(uint64_t a, uint64_t q);
bool is_prime(uint64_t n);
uint64_t first_prime(uint32_t bits, uint64_t m);
uint64_t previous_prime(uint64_t q, uint64_t m);
uint64_t next_prime(uint64_t q, uint64_t m);
uint64_t min_root_of_unity(uint64_t m, uint64_t q);
uint64_t shoup(uint64_t w, uint64_t q);  // floor(w * 2^64 / q)
uint32_t bitlen(uint64_t x);
// FLEXIBLEAUTO Q chain (num_q primes) and HYBRID P primes.
void ckks_moduli(uint32_t log_n, uint32_t num_q, uint32_t scale_bits, uint32_t first_bits,
                 uint32_t dnum, std::vector<uint64_t>& q, std::vector<uint64_t>& p);
}  // namespace nt

struct Context {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::shared_ptr<StreamHolder> sh;  // owns `stream`
  uint32_t log_n = 0;
  uint32_t n = 0;
  bool ckks = false;

  // Moduli: Q primes at indices [0, L), P primes at [L, L + K).
  std::vector<uint64_t> primes;
  std::vector<uint64_t> roots;
  uint32_t L = 0, K = 0;
  uint32_t dnum = 0, alpha = 0;
  uint32_t slots = 0;
  uint32_t scale_bits = 0, first_bits = 0;

  // Device tables.
  DevMem d_primes;  // u64[L+K]
  DevMem d_mod;     // Modulus[L+K]
  DevMem d_tw;      // Twiddle[L+K][N]
  DevMem d_tw_inv;  // Twiddle[L+K][N]
  DevMem d_ninv;    // Twiddle[L+K][2]
  // Round-2 twiddles of the row passes re-laid out thread-fastest so every
  // load of a warp is contiguous: [prime][row][j][t] (forward, inverse).
  DevMem d_tw2, d_tw2_inv;
  uint32_t tw2_stride = 0;  // entries per prime

  // Staging buffer for host-memory entry points.
  DevMem d_stage;

  ~Context();
  void make_current() const;
  uint32_t n_primes() const { return (uint32_t)primes.size(); }
  uint64_t max_prime() const { uint64_t m = 0; for (uint64_t q : primes) m = q > m ? q : m; return m; }
  void build_tables();
  uint64_t* stage(size_t words);
  NttArgs ntt_args(uint64_t* data, uint32_t n_polys, uint32_t prime0, uint32_t n_limbs,
                   uint32_t limb_stride) const;
};

}  // namespace fhe
