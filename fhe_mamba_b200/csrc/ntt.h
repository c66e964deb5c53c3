// Launch interface of the RNS NTT kernels (ntt.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "modarith.cuh"

namespace fhe {

struct NttArgs {
  uint64_t* data;          // u64[n_polys][limb_stride][N], first launched limb at data
  const Twiddle* tw;       // forward tables, Twiddle[n_primes][N]: psi^{brv(i)}
  const Twiddle* tw_inv;   // inverse tables: psi^{-brv(i)}
  const uint64_t* primes;  // u64[n_primes]
  const Twiddle* ninv;     // per prime: (N^{-1}, .), (psi^{-brv(1)} N^{-1}, .)
  int log_n;
  uint32_t n_polys;
  uint32_t n_limbs;
  uint32_t limb_stride;    // limbs between consecutive polys
  uint32_t prime0;         // prime index of the first launched limb
  // Optional explicit limb list (device array, n_limbs entries, n_polys must
  // be 1): entry {x, y} transforms the limb at data + x*N with prime y.
  const uint2* list = nullptr;
  // Lazy-reduction level of the forward transform: 32 when every prime the
  // launch touches is below 2^59, 16 when below 2^60, else 0 (reduce at
  // every butterfly).  See the schedule in ntt.cu.
  int lazy = 0;
  // Row-pass round-2 twiddles, thread-fastest layout (see Context::build_tables).
  const Twiddle* tw2 = nullptr;
  const Twiddle* tw2_inv = nullptr;
  uint32_t tw2_stride = 0;
  // Optional out-of-place input of the inverse transform (dense layout only):
  // its first pass reads limb l of poly c from src + (c*src_limb_stride + l)*N
  // and every pass writes to data.
  const uint64_t* src = nullptr;
  uint32_t src_limb_stride = 0;
  // Optional combine epilogue of the forward transform (dense layout only),
  // the last step of ModDown and of rescaling: for poly c and limb l (prime
  // p = prime0 + l) the transform's output v is not stored; instead
  //   epi_out[c][l] = (epi_x[c][l] - v) * epi_w[p]  (+ epi_add[l] when c == 0)
  // with component strides epi_x_comp / epi_out_comp words and limb stride N.
  const uint64_t* epi_x = nullptr;
  size_t epi_x_comp = 0;
  uint64_t* epi_out = nullptr;
  size_t epi_out_comp = 0;
  const Twiddle* epi_w = nullptr;
  const uint64_t* epi_add = nullptr;
  // Optional key-switching form of that epilogue: epi_x[c][l] is not read but
  // formed as the key inner product sum_j ext[j][l] * key[j][c][l] (128-bit
  // sum, one reduction), so the Q rows of the accumulator are never written
  // and re-read.  ext: [epi_digits][epi_w_rows][N]; key: [digits][2][key_limbs][N]
  // with Q limb l on key row l; mods: per-prime Barrett constants.
  const uint64_t* epi_ext = nullptr;
  const uint64_t* epi_key = nullptr;
  uint32_t epi_digits = 0, epi_w_rows = 0, epi_key_limbs = 0;
  const Modulus* epi_mods = nullptr;
  cudaStream_t stream;
};

// Shape of the row pass for a ring of 2^log_n: rows of 2^LB words, R words per
// thread, T threads per row; J round-2 twiddles per thread.
void ntt_row_shape(int log_n, int& rows, int& R, int& T, int& J);

cudaError_t ntt_forward(const NttArgs& args);
// Register-only throughput probe of the forward butterfly (see ntt.cu):
// blocks x 256 threads, each 128 butterflies per round; scratch_out holds
// blocks*256 words, scratch_in 1024 words.
cudaError_t ntt_butterfly_ceiling(uint64_t q, Twiddle w, uint64_t* scratch_out, const uint64_t* scratch_in,
                                  uint32_t blocks, int rounds, cudaStream_t s);
cudaError_t ntt_inverse(const NttArgs& args);

}  // namespace fhe
