// Negacyclic NTT / inverse NTT over RNS limbs for sm_100a.
//
// Convention (OpenFHE ChineseRemainderTransformFTTNat, used by FIDESlib's
// NTT_ / INTT_ kernels): the forward transform takes natural-order
// coefficients and returns evaluations in bit-reversed order,
//   out[i] = sum_j a[j] * psi^{(2*brv(i)+1)*j}  (mod q),
// psi the minimal primitive 2N-th root of unity mod q.  The inverse undoes it
// exactly, including the 1/N factor.  Outputs are fully reduced to [0, q).
//
// Layout: one transform = one limb = N contiguous u64 words; a batch is
// u64[n_polys][limb_stride][N] where the launch covers limbs
// [limb0, limb0 + n_limbs) of each poly and limb l uses prime prime0 + l.
//
// Structure: N = 2^LA * 2^LB.  The forward transform runs as two passes over
// HBM.  Pass "cols" performs the first LA Cooley-Tukey stages, which only
// couple words whose indices agree mod 2^LB (2^LB independent columns of
// height 2^LA).  Pass "rows" performs the last LB stages, which only couple
// words inside one contiguous row of 2^LB.  Inside a pass each thread holds
// R = 2^LR words in registers and runs LR stages there, the block exchanges
// words once through shared memory, and each thread runs the remaining
// LS - LR stages on a contiguous run of R words.  The inverse mirrors this
// (rows first, then columns, Gentleman-Sande butterflies, 1/N folded into the
// last stage).  Twiddles are read as (w, w') 16-byte pairs.
#include <cstdint>
#include <cuda_runtime.h>

#include "modarith.cuh"
#include "ntt.h"
#include "launch_count.h"

namespace fhe {
namespace {


template <int LS>
struct PassShape {
  static constexpr int LR = (LS + 1) / 2;  // stages in round 1
  static constexpr int R = 1 << LR;        // words per thread
  static constexpr int LT = LS - LR;       // stages in round 2
  static constexpr int T = 1 << LT;        // threads per sub-problem
  static constexpr int S = 1 << LS;        // sub-problem size
  static constexpr int J = R * (T - 1) / T;  // round-2 twiddles per thread
};

// Minimum resident CTAs per SM for a pass of 2^LS words per sub-problem and
// TW sub-problems per CTA: ~100 registers per thread for LS <= 8 (R = 16
// words in registers plus twiddles without spilling), ~170 for LS = 9.
template <int LS, int TW>
constexpr int min_blocks() {
  return LS <= 8 ? 40 / TW : 24 / TW;
}

// Forward Cooley-Tukey (Harvey) butterfly on lazy residues in [0, 4q).
__device__ __forceinline__ void ct_bfly(uint64_t& x, uint64_t& y, const Twiddle tw, uint64_t q,
                                        uint64_t q2) {
  x = csub(x, q2);
  const uint64_t t = shoup_lazy(y, tw.w, tw.wp, q);
  y = x + q2 - t;
  x = x + t;
}

// Greedy lazy schedule.  A forward pass starts with residues below b0 * q and
// every butterfly that does not reduce x raises the bound by 2q.  Stage s
// reduces x below (LZ/2) q (one conditional subtraction of (LZ/2) q) only
// when skipping it would let the bound exceed LZ q, where LZ q < 2^64:
// LZ = 32 needs every prime below 2^59, LZ = 16 below 2^60; LZ = 0 selects
// the reducing Harvey butterfly at every stage.
__host__ __device__ constexpr bool lz_reduce(int LZ, int b0, int s) {
  int b = b0;
  for (int i = 0; i < s; ++i) b = (b + 2 > LZ) ? LZ / 2 + 2 : b + 2;
  return b + 2 > LZ;
}
__host__ __device__ constexpr int lz_bound_after(int LZ, int b0, int stages) {
  int b = b0;
  for (int i = 0; i < stages; ++i) b = (b + 2 > LZ) ? LZ / 2 + 2 : b + 2;
  return b;
}

template <int LZ>
__device__ __forceinline__ void fwd_bfly(bool reduce, uint64_t& x, uint64_t& y, const Twiddle w, uint64_t q,
                                         uint64_t q2, uint64_t qh) {
  if constexpr (LZ == 0) {
    ct_bfly(x, y, w, q, q2);
  } else {
    if (reduce) x = csub(x, qh);
    const uint64_t t = shoup_lazy(y, w.w, w.wp, q);
    y = x + q2 - t;
    x = x + t;
  }
}

// Inverse Gentleman-Sande (Harvey) butterfly on residues in [0, 2q).
__device__ __forceinline__ void gs_bfly(uint64_t& x, uint64_t& y, const Twiddle tw, uint64_t q,
                                        uint64_t q2) {
  const uint64_t s = csub(x + y, q2);
  const uint64_t d = x + q2 - y;
  x = s;
  y = shoup_lazy(d, tw.w, tw.wp, q);
}

// Limb addressed by this block: (poly = blockIdx.y, limb = blockIdx.z) in the
// dense layout, or entry blockIdx.z of the explicit limb list.
__device__ __forceinline__ uint64_t* block_limb(const NttArgs& g, uint32_t n, uint32_t& pidx) {
  if (g.list) {
    const uint2 e = g.list[blockIdx.z];
    pidx = e.y;
    return g.data + (size_t)e.x * n;
  }
  pidx = g.prime0 + blockIdx.z;
  return g.data + ((size_t)blockIdx.y * g.limb_stride + blockIdx.z) * n;
}

__device__ __forceinline__ Twiddle ld_tw(const Twiddle* t, uint32_t i) {
  const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2*>(t) + i);
  return Twiddle{v.x, v.y};
}

// ---------------------------------------------------------------------------
// Forward, pass 1: columns.  Column c of the tile (lane) holds words
// j = col0 + c + 2^LB * k for k in [0, 2^LA).  Warp w is thread t of each
// column.  Round 1: k = t + T*u.  Round 2: k = R*t + u.
template <int LA, int LZ, int COLS>
__global__ void __launch_bounds__(COLS * PassShape<LA>::T, min_blocks<LA, COLS>())
    ntt_fwd_cols(const NttArgs g) {
  using P = PassShape<LA>;
  extern __shared__ uint64_t smem[];
  const int LB = g.log_n - LA;
  const uint32_t n = 1u << g.log_n;
  uint32_t pidx;
  uint64_t* a = block_limb(g, n, pidx);
  const uint64_t q = g.primes[pidx], q2 = 2 * q, qh = (uint64_t)(LZ / 2) * q;
  const Twiddle* tw = g.tw + (size_t)pidx * n;
  const int c = threadIdx.x % COLS;
  const int t = threadIdx.x / COLS;
  const uint32_t col = blockIdx.x * COLS + c;

  uint64_t x[P::R];
#pragma unroll
  for (int u = 0; u < P::R; ++u) x[u] = a[col + ((size_t)(t + P::T * u) << LB)];
  int st = 0;  // stage index within the pass (compile-time after unrolling)

  // Round 1: register half-distance h <-> k half-distance d = h*T.
  // Stage m = S/(2d); group i = k/(2d) = u/(2h) (thread independent).
#pragma unroll
  for (int h = P::R / 2; h >= 1; h >>= 1, ++st) {
    const int m = P::S / (2 * h * P::T);
    const bool red = lz_reduce(LZ, 1, st);
#pragma unroll
    for (int g = 0; g < P::R; g += 2 * h) {
      const Twiddle w = ld_tw(tw, m + g / (2 * h));
#pragma unroll
      for (int v = 0; v < h; ++v) fwd_bfly<LZ>(red, x[g + v], x[g + v + h], w, q, q2, qh);
    }
  }
  if constexpr (P::LT > 0) {
    // Exchange: smem[k][c].
#pragma unroll
    for (int u = 0; u < P::R; ++u) smem[(t + P::T * u) * COLS + c] = x[u];
    __syncthreads();
#pragma unroll
    for (int u = 0; u < P::R; ++u) x[u] = smem[(P::R * t + u) * COLS + c];
    // Round 2: half-distance h (k units), m = S/(2h), group i = (R*t + g)/(2h).
#pragma unroll
    for (int h = P::T / 2; h >= 1; h >>= 1, ++st) {
      const int m = P::S / (2 * h);
      const bool red = lz_reduce(LZ, 1, st);
#pragma unroll
      for (int g = 0; g < P::R; g += 2 * h) {
        const Twiddle w = ld_tw(tw, m + (P::R * t + g) / (2 * h));
#pragma unroll
        for (int v = 0; v < h; ++v) fwd_bfly<LZ>(red, x[g + v], x[g + v + h], w, q, q2, qh);
      }
    }
#pragma unroll
    for (int u = 0; u < P::R; ++u) a[col + ((size_t)(P::R * t + u) << LB)] = x[u];
  } else {
#pragma unroll
    for (int u = 0; u < P::R; ++u) a[col + ((size_t)(t + P::T * u) << LB)] = x[u];
  }
}

// Padded shared index for the row passes: one spare word per 16 keeps the
// stride-R reads of round 2 free of bank conflicts.
__device__ __forceinline__ int rpad(int k) { return k + (k >> 4); }

// ---------------------------------------------------------------------------
// Forward, pass 2: rows.  A CTA owns ROWS rows of 2^LB contiguous words.
// Thread t of a row: round 1 k = t + T*u (loaded straight from HBM, each load
// instruction covering 128-byte runs), round 2 k = R*t + u, then back through
// shared memory to the k = t + T*u layout for the stores.  Final output
// reduced to [0, q).
//
// With LZ > 0 the column pass leaves values below lz_bound_after(LZ, 1, LA) q;
// this pass continues the greedy schedule and reduces the output with one
// Shoup multiplication by 1 and a conditional subtraction.
// EPI: 0 = store the transform, 1 = combine epilogue with epi_x, 2 = combine
// epilogue with the key inner product formed in place of epi_x.
template <int LA, int LB, int ROWS, int LZ, int EPI>
__global__ void __launch_bounds__(ROWS * PassShape<LB>::T, min_blocks<LB, ROWS>())
    ntt_fwd_rows(const NttArgs g) {
  using P = PassShape<LB>;
  extern __shared__ uint64_t smem[];
  constexpr int kRowWords = P::S + P::S / 16;
  const uint32_t n = 1u << g.log_n;
  uint32_t pidx;
  uint64_t* a = block_limb(g, n, pidx) + (size_t)blockIdx.x * ROWS * P::S;
  const uint64_t q = g.primes[pidx], q2 = 2 * q, qh = (uint64_t)(LZ / 2) * q;
  const uint64_t mu = LZ ? ~0ull / q : 0;  // floor(2^64 / q), Shoup companion of 1
  constexpr int b0 = lz_bound_after(LZ, 1, LA);  // bound left by the column pass
  const Twiddle* tw = g.tw + (size_t)pidx * n;
  const int t = threadIdx.x % P::T;
  const int rr = threadIdx.x / P::T;
  const uint32_t row = blockIdx.x * ROWS + rr;
  // Final reduction to [0, q): the lazy schedule leaves values below bf*q,
  // removed by conditional subtractions of 2^k q (ALU pipe) rather than a
  // Shoup product by 1 (the 64-bit multiply pipe is the transform's limit).
  constexpr int bf = LZ ? lz_bound_after(LZ, b0, LB) : 4;
  constexpr int top = bf > 16 ? 4 : bf > 8 ? 3 : bf > 4 ? 2 : 1;  // 2^top < bf <= 2^(top+1)
  auto fwd_final = [](uint64_t v, uint64_t q, uint64_t, uint64_t) {
#pragma unroll
    for (int k = top; k >= 0; --k) v = csub(v, q << k);
    return v;
  };

  // Round-1 layout k = t + T*u: for each u the T threads of a row read T
  // consecutive words, so every load instruction covers whole 128-byte runs.
  uint64_t x[P::R];
  uint64_t* srow = smem + rr * kRowWords;
  uint64_t* grow = a + (size_t)rr * P::S;
#pragma unroll
  for (int u = 0; u < P::R; ++u) x[u] = grow[t + P::T * u];

  // Global stage for k-half-distance d: m = N/(2d); i = row*S/(2d) + k/(2d).
  int st = 0;
#pragma unroll
  for (int h = P::R / 2; h >= 1; h >>= 1, ++st) {
    const int d = h * P::T;
    const uint32_t m = n / (2 * d);
    const uint32_t base = m + row * (P::S / (2 * d));
    const bool red = lz_reduce(LZ, b0, st);
#pragma unroll
    for (int g = 0; g < P::R; g += 2 * h) {
      const Twiddle w = ld_tw(tw, base + g / (2 * h));
#pragma unroll
      for (int v = 0; v < h; ++v) fwd_bfly<LZ>(red, x[g + v], x[g + v + h], w, q, q2, qh);
    }
  }
  if constexpr (P::LT > 0) {
    __syncthreads();
#pragma unroll
    for (int u = 0; u < P::R; ++u) srow[rpad(t + P::T * u)] = x[u];
    __syncthreads();
#pragma unroll
    for (int u = 0; u < P::R; ++u) x[u] = srow[rpad(P::R * t + u)];
    const Twiddle* t2 = g.tw2 + (size_t)pidx * g.tw2_stride + (size_t)row * (P::J * P::T) + t;
    int j = 0;
#pragma unroll
    for (int h = P::T / 2; h >= 1; h >>= 1, ++st) {
      const bool red = lz_reduce(LZ, b0, st);
#pragma unroll
      for (int g = 0; g < P::R; g += 2 * h, ++j) {
        const Twiddle w = ld_tw(t2, j * P::T);
#pragma unroll
        for (int v = 0; v < h; ++v) fwd_bfly<LZ>(red, x[g + v], x[g + v + h], w, q, q2, qh);
      }
    }
#pragma unroll
    for (int u = 0; u < P::R; ++u) srow[rpad(P::R * t + u)] = fwd_final(x[u], q, q2, mu);
  } else {
    __syncthreads();
#pragma unroll
    for (int u = 0; u < P::R; ++u) srow[rpad(t + P::T * u)] = fwd_final(x[u], q, q2, mu);
  }
  __syncthreads();
  if constexpr (EPI == 1) {
    // combine epilogue: (x - v) * w (+ add on component 0), same coalesced layout
    const size_t off = (size_t)blockIdx.z * n + ((size_t)blockIdx.x * ROWS + rr) * P::S;
    const uint64_t* ex = g.epi_x + blockIdx.y * g.epi_x_comp + off;
    uint64_t* eo = g.epi_out + blockIdx.y * g.epi_out_comp + off;
    const uint64_t* ea = (g.epi_add && blockIdx.y == 0) ? g.epi_add + off : nullptr;
    const Twiddle w = g.epi_w[pidx];
#pragma unroll
    for (int u = 0; u < P::R; ++u) {
      const int k = t + P::T * u;
      uint64_t r = shoup_mul(sub_mod(ex[k], srow[rpad(k)], q), w.w, w.wp, q);
      if (ea) r = add_mod(r, ea[k], q);
      eo[k] = r;
    }
  } else if constexpr (EPI == 2) {
    // key-switching combine: x = sum_j ext[j][l] key[j][c][l] (128-bit sum,
    // each product below q^2 and at most 15 digits), then (x - v) w (+ add)
    const size_t row_off = ((size_t)blockIdx.x * ROWS + rr) * P::S;
    const size_t off = (size_t)blockIdx.z * n + row_off;
    uint64_t* eo = g.epi_out + blockIdx.y * g.epi_out_comp + off;
    const uint64_t* ea = (g.epi_add && blockIdx.y == 0) ? g.epi_add + off : nullptr;
    const Twiddle w = g.epi_w[pidx];
    const Modulus m = g.epi_mods[pidx];
    const size_t ext_stride = (size_t)g.epi_w_rows * n, key_stride = (size_t)2 * g.epi_key_limbs * n;
    const uint64_t* e0 = g.epi_ext + off;
    const uint64_t* k0 = g.epi_key + ((size_t)blockIdx.y * g.epi_key_limbs + pidx) * n + row_off;
#pragma unroll
    for (int u = 0; u < P::R; ++u) {
      const int k = t + P::T * u;
      uint64_t hi = 0, lo = 0;
      for (uint32_t j = 0; j < g.epi_digits; ++j) {
        const uint64_t a = e0[j * ext_stride + k], b = k0[j * key_stride + k];
        const uint64_t pl = a * b;
        lo += pl;
        hi += __umul64hi(a, b) + (lo < pl);
      }
      uint64_t r = shoup_mul(sub_mod(reduce_u128(hi, lo, m), srow[rpad(k)], q), w.w, w.wp, q);
      if (ea) r = add_mod(r, ea[k], q);
      eo[k] = r;
    }
  } else {
#pragma unroll
    for (int u = 0; u < P::R; ++u) grow[t + P::T * u] = srow[rpad(t + P::T * u)];
  }
}

// ---------------------------------------------------------------------------
// Inverse, pass 1: rows (stages with half-distance 1 .. 2^(LB-1)).
// Round 1 on contiguous runs k = R*t + u (half-distances 1 .. T/2), exchange,
// round 2 on k = t + T*u (half-distances T .. S/2).  Input in [0, q).
template <int LB, int ROWS>
__global__ void __launch_bounds__(ROWS * PassShape<LB>::T, min_blocks<LB, ROWS>())
    ntt_inv_rows(const NttArgs g) {
  using P = PassShape<LB>;
  extern __shared__ uint64_t smem[];
  constexpr int kRowWords = P::S + P::S / 16;
  const uint32_t n = 1u << g.log_n;
  uint32_t pidx;
  uint64_t* a = block_limb(g, n, pidx) + (size_t)blockIdx.x * ROWS * P::S;
  const uint64_t q = g.primes[pidx], q2 = 2 * q;
  const Twiddle* tw = g.tw_inv + (size_t)pidx * n;
  const int t = threadIdx.x % P::T;
  const int rr = threadIdx.x / P::T;
  const uint32_t row = blockIdx.x * ROWS + rr;

  // Coalesced load in the k = t + T*u layout (from the out-of-place source
  // when one is given), staged through shared memory for round 1's runs.
  uint64_t x[P::R];
  uint64_t* srow = smem + rr * kRowWords;
  {
    const uint64_t* grow =
        (g.src ? g.src + ((size_t)blockIdx.y * g.src_limb_stride + blockIdx.z) * n +
                     (size_t)blockIdx.x * ROWS * P::S
               : a) +
        (size_t)rr * P::S;
#pragma unroll
    for (int u = 0; u < P::R; ++u) srow[rpad(t + P::T * u)] = grow[t + P::T * u];
  }
  __syncthreads();
  if constexpr (P::LT > 0) {
#pragma unroll
    for (int u = 0; u < P::R; ++u) x[u] = srow[rpad(P::R * t + u)];
    const Twiddle* t2 = g.tw2_inv + (size_t)pidx * g.tw2_stride + (size_t)row * (P::J * P::T) + t;
    int j = 0;
#pragma unroll
    for (int h = 1; h <= P::T / 2; h <<= 1) {
#pragma unroll
      for (int g = 0; g < P::R; g += 2 * h, ++j) {
        const Twiddle w = ld_tw(t2, j * P::T);
#pragma unroll
        for (int v = 0; v < h; ++v) gs_bfly(x[g + v], x[g + v + h], w, q, q2);
      }
    }
#pragma unroll
    for (int u = 0; u < P::R; ++u) srow[rpad(P::R * t + u)] = x[u];
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < P::R; ++u) x[u] = srow[rpad(t + P::T * u)];
#pragma unroll
  for (int h = 1; h <= P::R / 2; h <<= 1) {
    const int d = h * P::T;
    const uint32_t m = n / (2 * d);
    const uint32_t base = m + row * (P::S / (2 * d));
#pragma unroll
    for (int g = 0; g < P::R; g += 2 * h) {
      const Twiddle w = ld_tw(tw, base + g / (2 * h));
#pragma unroll
      for (int v = 0; v < h; ++v) gs_bfly(x[g + v], x[g + v + h], w, q, q2);
    }
  }
  // Round-2 layout k = t + T*u stores whole 128-byte runs directly.
  uint64_t* grow = a + (size_t)rr * P::S;
#pragma unroll
  for (int u = 0; u < P::R; ++u) grow[t + P::T * u] = x[u];
}

// ---------------------------------------------------------------------------
// Inverse, pass 2: columns (half-distances 2^LB .. N/2).  Round 1 on
// k = R*t + u (k half-distances 1 .. T/2), exchange, round 2 on k = t + T*u.
// The last stage (m = 1) folds in N^{-1}: x' = (x+y)/N, y' = (x-y)*w/N, with
// tw_last = (N^{-1}, N^{-1}') and tw_last2 = (w_1 N^{-1}, ...).
template <int LA, int COLS>
__global__ void __launch_bounds__(COLS * PassShape<LA>::T, min_blocks<LA, COLS>())
    ntt_inv_cols(const NttArgs g) {
  using P = PassShape<LA>;
  extern __shared__ uint64_t smem[];
  const int LB = g.log_n - LA;
  const uint32_t n = 1u << g.log_n;
  uint32_t pidx;
  uint64_t* a = block_limb(g, n, pidx);
  const uint64_t q = g.primes[pidx], q2 = 2 * q;
  const Twiddle* tw = g.tw_inv + (size_t)pidx * n;
  const int c = threadIdx.x % COLS;
  const int t = threadIdx.x / COLS;
  const uint32_t col = blockIdx.x * COLS + c;
  uint64_t x[P::R];

  if constexpr (P::LT > 0) {
#pragma unroll
    for (int u = 0; u < P::R; ++u) x[u] = a[col + ((size_t)(P::R * t + u) << LB)];
#pragma unroll
    for (int h = 1; h <= P::T / 2; h <<= 1) {
      const int m = P::S / (2 * h);
#pragma unroll
      for (int g = 0; g < P::R; g += 2 * h) {
        const Twiddle w = ld_tw(tw, m + (P::R * t + g) / (2 * h));
#pragma unroll
        for (int v = 0; v < h; ++v) gs_bfly(x[g + v], x[g + v + h], w, q, q2);
      }
    }
#pragma unroll
    for (int u = 0; u < P::R; ++u) smem[(P::R * t + u) * COLS + c] = x[u];
    __syncthreads();
#pragma unroll
    for (int u = 0; u < P::R; ++u) x[u] = smem[(t + P::T * u) * COLS + c];
  } else {
#pragma unroll
    for (int u = 0; u < P::R; ++u) x[u] = a[col + ((size_t)(t + P::T * u) << LB)];
  }
#pragma unroll
  for (int h = 1; h < P::R / 2; h <<= 1) {
    const int m = P::S / (2 * h * P::T);
#pragma unroll
    for (int g = 0; g < P::R; g += 2 * h) {
      const Twiddle w = ld_tw(tw, m + g / (2 * h));
#pragma unroll
      for (int v = 0; v < h; ++v) gs_bfly(x[g + v], x[g + v + h], w, q, q2);
    }
  }
  {  // last stage, m = 1, half-distance R/2 in registers, 1/N folded in.
    const Twiddle ni = g.ninv[2 * pidx];
    const Twiddle wn = g.ninv[2 * pidx + 1];
    constexpr int h = P::R / 2;
#pragma unroll
    for (int v = 0; v < h; ++v) {
      const uint64_t s = x[v] + x[v + h];  // < 4q
      const uint64_t d = x[v] + q2 - x[v + h];
      x[v] = csub(shoup_lazy(s, ni.w, ni.wp, q), q);
      x[v + h] = csub(shoup_lazy(d, wn.w, wn.wp, q), q);
    }
  }
#pragma unroll
  for (int u = 0; u < P::R; ++u) a[col + ((size_t)(t + P::T * u) << LB)] = x[u];
}

template <int LB, int ROWS>
size_t rows_smem() {
  using P = PassShape<LB>;
  return (size_t)ROWS * (P::S + P::S / 16) * sizeof(uint64_t);
}
template <int LA, int COLS>
size_t cols_smem() {
  using P = PassShape<LA>;
  return P::LT > 0 ? (size_t)COLS * P::S * sizeof(uint64_t) : 0;
}

// Tile width: 8 columns / rows per CTA (128 threads at 2^16).  Measured on
// the config-2 batch against 16 and 32 with several register caps: small
// CTAs with ~100 registers keep the integer pipes busiest.

template <int LA, int LB, int LZ, int TW, int EPI>
cudaError_t launch_fwd_impl(const NttArgs& g) {
  using PA = PassShape<LA>;
  using PB = PassShape<LB>;
  const size_t sa = cols_smem<LA, TW>(), sb = rows_smem<LB, TW>();
  cudaError_t e;
  e = cudaFuncSetAttribute(ntt_fwd_cols<LA, LZ, TW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sa);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(ntt_fwd_rows<LA, LB, TW, LZ, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sb);
  if (e != cudaSuccess) return e;
  const uint32_t polys = g.list ? 1 : g.n_polys;
  dim3 ga((1u << LB) / TW, polys, g.n_limbs);
  ntt_fwd_cols<LA, LZ, TW><<<ga, TW * PA::T, sa, g.stream>>>(g); note_launch();
  dim3 gb((1u << LA) / TW, polys, g.n_limbs);
  ntt_fwd_rows<LA, LB, TW, LZ, EPI><<<gb, TW * PB::T, sb, g.stream>>>(g); note_launch();
  return cudaGetLastError();
}

template <int LA, int LB, int TW, int EPI>
cudaError_t launch_fwd_lz(const NttArgs& g) {
  switch (g.lazy) {
    case 32: return launch_fwd_impl<LA, LB, 32, TW, EPI>(g);
    case 16: return launch_fwd_impl<LA, LB, 16, TW, EPI>(g);
    default: return launch_fwd_impl<LA, LB, 0, TW, EPI>(g);
  }
}

template <int LA, int LB, int TW>
cudaError_t launch_fwd_tw(const NttArgs& g) {
  if (g.epi_out && g.epi_ext) {
    if (g.list || !g.epi_key || !g.epi_w || !g.epi_mods || g.epi_digits == 0 || g.epi_digits > 15 ||
        g.n_polys != 2)
      return cudaErrorInvalidValue;
    return launch_fwd_lz<LA, LB, TW, 2>(g);
  }
  if (g.epi_out) {
    if (g.list || !g.epi_x || !g.epi_w) return cudaErrorInvalidValue;
    return launch_fwd_lz<LA, LB, TW, 1>(g);
  }
  return launch_fwd_lz<LA, LB, TW, 0>(g);
}

template <int LA, int LB>
cudaError_t launch_fwd(const NttArgs& g) {
  return launch_fwd_tw<LA, LB, 8>(g);
}

template <int LA, int LB, int TW>
cudaError_t launch_inv_tw(const NttArgs& g) {
  using PA = PassShape<LA>;
  using PB = PassShape<LB>;
  const size_t sa = cols_smem<LA, TW>(), sb = rows_smem<LB, TW>();
  cudaError_t e;
  e = cudaFuncSetAttribute(ntt_inv_cols<LA, TW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sa);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(ntt_inv_rows<LB, TW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sb);
  if (e != cudaSuccess) return e;
  const uint32_t polys = g.list ? 1 : g.n_polys;
  dim3 gb((1u << LA) / TW, polys, g.n_limbs);
  ntt_inv_rows<LB, TW><<<gb, TW * PB::T, sb, g.stream>>>(g); note_launch();
  dim3 ga((1u << LB) / TW, polys, g.n_limbs);
  ntt_inv_cols<LA, TW><<<ga, TW * PA::T, sa, g.stream>>>(g); note_launch();
  return cudaGetLastError();
}

template <int LA, int LB>
cudaError_t launch_inv(const NttArgs& g) {
  if (g.src && g.list) return cudaErrorInvalidValue;
  return launch_inv_tw<LA, LB, 8>(g);
}

// Integer-pipe ceiling of the forward butterfly: the same lazy Shoup
// butterfly and reduction schedule as the column pass (8 stages, LZ = 16),
// on 16 words held in registers with no memory traffic, 2 x 8 butterflies per
// stage.  Each thread stores one word (the XOR of its registers) so the work
// cannot be removed; `in` holds 1024 words.
__global__ void __launch_bounds__(256) k_butterfly_ceiling(uint64_t* out, const uint64_t* in, uint64_t q,
                                                            Twiddle w, int rounds) {
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = in[(tid * 16 + i) & 1023u] % q;
  const uint64_t q2 = 2 * q, qh = 8 * q;
  for (int r = 0; r < rounds; ++r) {
#pragma unroll
    for (int st = 0; st < 8; ++st) {
      const bool red = lz_reduce(16, 1, st);
      const int h = 1 << (st & 3);
#pragma unroll
      for (int g = 0; g < 16; g += 2 * h)
#pragma unroll
        for (int v = 0; v < h; ++v) fwd_bfly<16>(red, x[g + v], x[g + v + h], w, q, q2, qh);
    }
  }
  uint64_t acc = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) acc ^= x[i];
  out[tid] = acc;
}

}  // namespace

cudaError_t ntt_butterfly_ceiling(uint64_t q, Twiddle w, uint64_t* scratch_out, const uint64_t* scratch_in,
                                  uint32_t blocks, int rounds, cudaStream_t s) {
  k_butterfly_ceiling<<<blocks, 256, 0, s>>>(scratch_out, scratch_in, q, w, rounds);
  note_launch();
  return cudaGetLastError();
}

void ntt_row_shape(int log_n, int& rows, int& R, int& T, int& J) {
  const int LA = log_n / 2, LB = log_n - LA;
  const int LR = (LB + 1) / 2, LT = LB - LR;
  rows = 1 << LA;
  R = 1 << LR;
  T = 1 << LT;
  J = R * (T - 1) / T;
}

// log N = LA + LB with LA = floor(logN/2) >= 5 so both passes have at least
// one full tile of 8 columns / rows.
cudaError_t ntt_forward(const NttArgs& g) {
  if (g.n_limbs == 0 || g.n_polys == 0) return cudaSuccess;
  switch (g.log_n) {
    case 10: return launch_fwd<5, 5>(g);
    case 11: return launch_fwd<5, 6>(g);
    case 12: return launch_fwd<6, 6>(g);
    case 13: return launch_fwd<6, 7>(g);
    case 14: return launch_fwd<7, 7>(g);
    case 15: return launch_fwd<7, 8>(g);
    case 16: return launch_fwd<8, 8>(g);
    case 17: return launch_fwd<8, 9>(g);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t ntt_inverse(const NttArgs& g) {
  if (g.n_limbs == 0 || g.n_polys == 0) return cudaSuccess;
  switch (g.log_n) {
    case 10: return launch_inv<5, 5>(g);
    case 11: return launch_inv<5, 6>(g);
    case 12: return launch_inv<6, 6>(g);
    case 13: return launch_inv<6, 7>(g);
    case 14: return launch_inv<7, 7>(g);
    case 15: return launch_inv<7, 8>(g);
    case 16: return launch_inv<8, 8>(g);
    case 17: return launch_inv<8, 9>(g);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fhe
