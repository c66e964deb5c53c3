// RNS-CKKS device kernels for sm_100a (elementwise limb arithmetic, sampling,
// automorphisms, HYBRID key-switching basis conversions, rescale lift,
// special-FFT encode/decode).  The NTT lives in ntt.cu.
#include <cstdint>
#include <cuda_runtime.h>

#include "ckks_kernels.h"
#include "launch_count.h"

namespace fhe {
namespace {

constexpr int kTpb = 256;

// ---------------------------------------------------------------------------
// ChaCha20 block (RFC 8439 rounds), key = (seed, fixed words), 64-bit block
// counter, 64-bit stream nonce.  Word w of the keystream for (seed, stream)
// is 64-bit word (w & 7) of block (w >> 3), little-endian 32-bit halves.
__device__ __forceinline__ uint32_t rotl(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }
#define QR(a, b, c, d)             \
  a += b; d ^= a; d = rotl(d, 16); \
  c += d; b ^= c; b = rotl(b, 12); \
  a += b; d ^= a; d = rotl(d, 8);  \
  c += d; b ^= c; b = rotl(b, 7);

__device__ void chacha_block(uint64_t seed, uint64_t stream, uint64_t counter, uint64_t out[8]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    (uint32_t)seed, (uint32_t)(seed >> 32), 0x243f6a88u, 0x85a308d3u,
                    0x13198a2eu, 0x03707344u, 0xa4093822u, 0x299f31d0u,
                    (uint32_t)counter, (uint32_t)(counter >> 32), (uint32_t)stream,
                    (uint32_t)(stream >> 32)};
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = s[i];
#pragma unroll 1
  for (int r = 0; r < 10; ++r) {
    QR(x[0], x[4], x[8], x[12]);
    QR(x[1], x[5], x[9], x[13]);
    QR(x[2], x[6], x[10], x[14]);
    QR(x[3], x[7], x[11], x[15]);
    QR(x[0], x[5], x[10], x[15]);
    QR(x[1], x[6], x[11], x[12]);
    QR(x[2], x[7], x[8], x[13]);
    QR(x[3], x[4], x[9], x[14]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    out[i] = (uint64_t)(x[2 * i] + s[2 * i]) | ((uint64_t)(x[2 * i + 1] + s[2 * i + 1]) << 32);
}
#undef QR

__global__ void k_sample_small(int kind, uint64_t seed, uint64_t stream, int64_t* out, uint32_t n) {
  const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;  // one block = 8 coefficients
  if (8 * b >= n) return;
  uint64_t w[8];
  chacha_block(seed, stream, b, w);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int64_t v;
    if (kind == 0) {
      const uint64_t r = w[i] % 3;
      v = r == 2 ? -1 : (int64_t)r;
    } else {
      v = (int64_t)__popcll(w[i] & 0x1FFFFFull) - (int64_t)__popcll((w[i] >> 21) & 0x1FFFFFull);
    }
    out[8 * b + i] = v;
  }
}

// Signed 64-bit value -> residue mod q (Barrett; |v| < 2^63).
__device__ __forceinline__ uint64_t lift_signed(int64_t v, const Modulus& m) {
  if (v >= 0) return barrett_reduce(0, (uint64_t)v, m);
  const uint64_t r = barrett_reduce(0, (uint64_t)(-(v + 1)) + 1, m);
  return r ? m.q - r : 0;
}

__global__ void k_lift_small(const int64_t* src, uint64_t* out, uint32_t n, PrimeMap pm, const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y;
  out[(size_t)l * n + k] = lift_signed(src[k], mods[pm(l)]);
}

// Uniform residue from two keystream words: (hi * 2^64 + lo) mod q.
__global__ void k_sample_uniform(uint64_t seed, uint64_t stream, uint64_t* out, uint32_t n, PrimeMap pm,
                                 const Modulus* mods) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;  // 4 coefficients per thread
  if (4 * t >= n) return;
  const uint32_t l = blockIdx.y;
  const uint32_t p = pm(l);
  const Modulus m = mods[p];
  const uint64_t r64 = barrett_reduce(1, 0, m);  // 2^64 mod q
  uint64_t w[8];
  chacha_block(seed, stream, ((uint64_t)p * n + 4 * t) / 4, w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t hi = barrett_reduce(0, w[2 * i], m);
    const uint64_t lo = barrett_reduce(0, w[2 * i + 1], m);
    out[(size_t)l * n + 4 * t + i] = add_mod(mul_mod(hi, r64, m), lo, m.q);
  }
}

// ---------------------------------------------------------------------------
__global__ void k_ew(Ew op, const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* out,
                     size_t so, uint32_t n, PrimeMap pm, const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const Modulus m = mods[pm(l)];
  const size_t off = (size_t)l * n + k;
  const uint64_t x = a[c * sa + off];
  uint64_t r;
  switch (op) {
    case Ew::Add: r = add_mod(x, b[c * sb + off], m.q); break;
    case Ew::Sub: r = sub_mod(x, b[c * sb + off], m.q); break;
    case Ew::Mul: r = mul_mod(x, b[c * sb + off], m); break;
    case Ew::Neg: r = neg_mod(x, m.q); break;
    case Ew::MulAdd: r = add_mod(out[c * so + off], mul_mod(x, b[c * sb + off], m), m.q); break;
    default: r = sub_mod(b[c * sb + off], x, m.q); break;  // SubFrom
  }
  out[c * so + off] = r;
}

__global__ void k_mul_const(const uint64_t* a, size_t sa, const Shoup* cst, const uint64_t* b, size_t sb,
                            uint64_t* out, size_t so, uint32_t n, const uint64_t* primes) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const uint64_t q = primes[l];
  const size_t off = (size_t)l * n + k;
  const Shoup w = cst[l];
  uint64_t r = shoup_mul(a[c * sa + off], w.w, w.wp, q);
  if (b) r = add_mod(r, b[c * sb + off], q);
  out[c * so + off] = r;
}

__global__ void k_add_const(const uint64_t* a, size_t sa, const uint64_t* cst, uint64_t* out, size_t so,
                            uint32_t n, const uint64_t* primes) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const size_t off = (size_t)l * n + k;
  out[c * so + off] = add_mod(a[c * sa + off], cst[l], primes[l]);
}

__global__ void k_mul_const_v(const uint64_t* a, size_t sa, const LimbShoup c, uint64_t* out, size_t so, uint32_t n,
                              const uint64_t* primes) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, comp = blockIdx.z;
  const size_t off = (size_t)l * n + k;
  out[comp * so + off] = shoup_mul(a[comp * sa + off], c.v[l].w, c.v[l].wp, primes[l]);
}

__global__ void k_add_const_v(const uint64_t* a, size_t sa, const LimbWords c, uint64_t* out, size_t so, uint32_t n,
                              const uint64_t* primes) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, comp = blockIdx.z;
  const size_t off = (size_t)l * n + k;
  const uint64_t x = a[comp * sa + off];
  out[comp * so + off] = comp == 0 ? add_mod(x, c.v[l], primes[l]) : x;
}

__global__ void k_linear_wsum(const WsumArgs a, uint32_t m, const uint64_t* w, const LimbWords add, int has_add,
                              uint64_t* out, size_t so, uint32_t nq, uint32_t n, const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, comp = blockIdx.z;
  const size_t off = (size_t)l * n + k;
  uint64_t hi = 0, lo = 0;
  for (uint32_t i = 0; i < m; ++i) {
    const uint64_t x = a.x[i][comp * a.stride[i] + off];
    const uint64_t wi = w[(size_t)i * nq + l];
    const uint64_t plo = x * wi;
    lo += plo;
    hi += __umul64hi(x, wi) + (lo < plo);
  }
  const Modulus md = mods[l];
  uint64_t r = reduce_u128(hi, lo, md);
  if (has_add && comp == 0) r = add_mod(r, add.v[l], md.q);
  out[comp * so + off] = r;
}

__global__ void k_tensor(const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* d, size_t sd,
                         uint32_t n, const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y;
  const Modulus m = mods[l];
  const size_t off = (size_t)l * n + k;
  const uint64_t a0 = a[off], a1 = a[sa + off], b0 = b[off], b1 = b[sb + off];
  d[off] = mul_mod(a0, b0, m);
  d[sd + off] = add_mod(mul_mod(a0, b1, m), mul_mod(a1, b0, m), m.q);
  d[2 * sd + off] = mul_mod(a1, b1, m);
}

__global__ void k_automorphism(const uint64_t* in, size_t si, uint64_t* out, size_t so, uint32_t log_n,
                               uint64_t g) {
  const uint32_t n = 1u << log_n;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const uint64_t mask = 2ull * n - 1;
  const uint64_t e = ((2ull * (__brev(i) >> (32 - log_n)) + 1) * g) & mask;
  const uint32_t j = __brev((uint32_t)((e - 1) >> 1)) >> (32 - log_n);
  out[c * so + (size_t)l * n + i] = __ldg(in + c * si + (size_t)l * n + j);
}

// ---------------------------------------------------------------------------
constexpr int kMaxSrc = 24;  // largest digit / special basis handled by the conversions

#define FHE_NS_CASES(X) \
  X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14) X(15) X(16) X(17) X(18) \
  X(19) X(20) X(21) X(22) X(23) X(24)

#define FHE_NS16_CASES(X) \
  X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11) X(12) X(13) X(14) X(15) X(16)

constexpr int kTgtChunk = 8;  // target limbs per block in the basis conversions

// Conversion constants in shared memory: the word itself, or (SPLIT) its
// 30-bit halves packed as lo | hi << 32.
template <bool SPLIT>
__device__ __forceinline__ uint64_t conv_const(uint64_t w) {
  if constexpr (SPLIT) return (w & ((1ull << 30) - 1)) | ((w >> 30) << 32);
  else return w;
}

// sum_i y_i h_i mod m, exact.  SPLIT (every y_i, h_i < 2^60, NS <= 16): with
// 30-bit halves each partial product is below 2^60, so the four partial sums
// of NS terms fit 64 bits and every term is one 32x32+64 multiply-add; the
// 128-bit total a11 2^60 + (a01 + a10) 2^30 + a00 is reduced once.
// Otherwise: 64x64 -> 128-bit products accumulated with carries.
template <int NS, bool SPLIT>
__device__ __forceinline__ uint64_t conv_dot(const uint64_t (&y)[NS], const uint64_t* h, const Modulus& m) {
  if constexpr (SPLIT) {
    static_assert(NS <= 16, "split accumulation holds at most 16 terms");
    // Karatsuba on 30-bit halves: y h = y1 h1 2^60 + ((y0+y1)(h0+h1) - y0 h0
    // - y1 h1) 2^30 + y0 h0, three 32x32->64 multiply-adds per term.  The
    // middle products are below 2^62, so they are summed in groups of four.
    constexpr int G = (NS + 3) / 4;
    uint64_t s00 = 0, s11 = 0, mid[G] = {};
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      const uint64_t c = h[i];
      const uint32_t h0 = (uint32_t)c, h1 = (uint32_t)(c >> 32);
      const uint32_t y0 = (uint32_t)(y[i] & ((1ull << 30) - 1)), y1 = (uint32_t)(y[i] >> 30);
      s00 += (uint64_t)y0 * h0;
      s11 += (uint64_t)y1 * h1;
      mid[i / 4] += (uint64_t)(y0 + y1) * (h0 + h1);
    }
    // m = sum(mid) - s00 - s11 in 128 bits (exact, below 2^66)
    uint64_t ml = mid[0], mh = 0;
#pragma unroll
    for (int g = 1; g < G; ++g) {
      ml += mid[g];
      mh += ml < mid[g];
    }
    mh -= ml < s00;
    ml -= s00;
    mh -= ml < s11;
    ml -= s11;
    uint64_t lo = s00 + (ml << 30);
    uint64_t hi = ((mh << 30) | (ml >> 34)) + (lo < s00);
    const uint64_t t = s11 << 60;
    lo += t;
    hi += (s11 >> 4) + (lo < t);
    return reduce_u128(hi, lo, m);
  } else {
    uint64_t hi = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      const uint64_t c = h[i];
      const uint64_t pl = y[i] * c;
      lo += pl;
      hi += __umul64hi(y[i], c) + (lo < pl);
    }
    return reduce_u128(hi, lo, m);
  }
}

// Block (x = coefficient tile, y = digit - digit0, z = chunk of kTgtChunk
// target limbs).  NS = source limbs of every digit in the launch.  The sum
// sum_i y_i hat_{i,t} is formed exactly in 128 bits and reduced once.
template <int NS, bool SPLIT>
__global__ void k_modup(const uint64_t* coef, const uint64_t* dntt, uint64_t* ext, uint32_t w, uint32_t n,
                        const ModUpDigit* digits, uint32_t digit0, const Modulus* mods) {
  __shared__ uint64_t sh_hat[kTgtChunk * NS];
  __shared__ Modulus sh_m[kTgtChunk];
  const uint32_t j = digit0 + blockIdx.y;
  const ModUpDigit dg = digits[j];
  const uint32_t t0 = blockIdx.z * kTgtChunk;
  if (t0 >= dg.conv.nt) return;  // uniform across the block
  const uint32_t nt = min((uint32_t)kTgtChunk, dg.conv.nt - t0);
  for (uint32_t i = threadIdx.x; i < nt * NS; i += blockDim.x)
    sh_hat[i] = conv_const<SPLIT>(dg.conv.hat[(size_t)t0 * NS + i].w);
  if (threadIdx.x < nt) sh_m[threadIdx.x] = mods[dg.conv.dst_prime[t0 + threadIdx.x]];
  __syncthreads();
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  uint64_t* e = ext + (size_t)j * w * n;
  uint64_t y[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const uint32_t l = dg.lo + i;
    const Shoup h = dg.conv.hatinv[i];
    y[i] = shoup_mul(coef[(size_t)l * n + k], h.w, h.wp, mods[dg.conv.src_prime[i]].q);
    if (blockIdx.z == 0) e[(size_t)l * n + k] = dntt[(size_t)l * n + k];
  }
  for (uint32_t u = 0; u < nt; ++u) {
    const uint32_t tt = t0 + u;
    const uint32_t l = tt < dg.lo ? tt : tt + NS;
    e[(size_t)l * n + k] = conv_dot<NS, SPLIT>(y, sh_hat + u * NS, sh_m[u]);
  }
}

__global__ void k_key_inner(const uint64_t* ext, uint32_t D, uint32_t w, const uint64_t* evk,
                            uint32_t key_limbs, PrimeMap pm, uint64_t* acc, uint32_t n,
                            const Modulus* mods, uint32_t first_limb) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = first_limb + blockIdx.y;
  const uint32_t p = pm(l);
  const Modulus m = mods[p];
  // 128-bit sums of the D products (each < q^2 < 2^122 / D), one reduction each
  uint64_t h0 = 0, l0 = 0, h1 = 0, l1 = 0;
  for (uint32_t j = 0; j < D; ++j) {
    const uint64_t x = ext[((size_t)j * w + l) * n + k];
    const uint64_t* kb = evk + (size_t)j * 2 * key_limbs * n;
    const uint64_t k0 = kb[(size_t)p * n + k], k1 = kb[((size_t)key_limbs + p) * n + k];
    const uint64_t p0 = x * k0, p1 = x * k1;
    l0 += p0;
    h0 += __umul64hi(x, k0) + (l0 < p0);
    l1 += p1;
    h1 += __umul64hi(x, k1) + (l1 < p1);
  }
  acc[(size_t)l * n + k] = reduce_u128(h0, l0, m);
  acc[((size_t)w + l) * n + k] = reduce_u128(h1, l1, m);
}

// Block (x = coefficient tile, y = component, z = chunk of kTgtChunk targets).
template <int NS, bool SPLIT>
__global__ void k_convert(const uint64_t* src, size_t s_comp, uint64_t* dst, size_t d_comp,
                          const ConvTable* tab, uint32_t n, const Modulus* mods) {
  __shared__ uint64_t sh_hat[kTgtChunk * NS];
  __shared__ Modulus sh_m[kTgtChunk];
  const ConvTable t = *tab;
  const uint32_t t0 = blockIdx.z * kTgtChunk;
  if (t0 >= t.nt) return;
  const uint32_t nt = min((uint32_t)kTgtChunk, t.nt - t0);
  for (uint32_t i = threadIdx.x; i < nt * NS; i += blockDim.x) sh_hat[i] = conv_const<SPLIT>(t.hat[(size_t)t0 * NS + i].w);
  if (threadIdx.x < nt) sh_m[threadIdx.x] = mods[t.dst_prime[t0 + threadIdx.x]];
  __syncthreads();
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t c = blockIdx.y;
  const uint64_t* s = src + c * s_comp;
  uint64_t* d = dst + c * d_comp;
  uint64_t y[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const Shoup h = t.hatinv[i];
    const size_t row = t.src_row ? t.src_row[i] : (uint32_t)i;
    y[i] = shoup_mul(s[row * n + k], h.w, h.wp, mods[t.src_prime[i]].q);
  }
  for (uint32_t u = 0; u < nt; ++u) {
    const size_t row = t.dst_row ? t.dst_row[t0 + u] : t0 + u;
    d[row * n + k] = conv_dot<NS, SPLIT>(y, sh_hat + u * NS, sh_m[u]);
  }
}

__global__ void k_moddown_combine(const uint64_t* x, size_t sx, const uint64_t* conv, size_t sc,
                                  const Shoup* pinv, const uint64_t* add, uint64_t* out, size_t so, uint32_t n,
                                  const uint64_t* primes) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const uint64_t q = primes[l];
  const size_t off = (size_t)l * n + k;
  const Shoup w = pinv[l];
  uint64_t r = shoup_mul(sub_mod(x[c * sx + off], conv[c * sc + off], q), w.w, w.wp, q);
  if (add && c == 0) r = add_mod(r, add[off], q);
  out[c * so + off] = r;
}

__global__ void k_rescale_lift(const uint64_t* last, size_t sl, uint64_t* lifted, size_t sd, uint32_t n,
                               uint64_t q_last, const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const Modulus m = mods[l];
  const uint64_t v = last[c * sl + k];
  uint64_t r;
  if (v > q_last / 2) {
    const uint64_t mag = barrett_reduce(0, q_last - v, m);
    r = mag ? m.q - mag : 0;
  } else {
    r = barrett_reduce(0, v, m);
  }
  lifted[c * sd + (size_t)l * n + k] = r;
}

// ---------------------------------------------------------------------------
// Special FFT (OpenFHE FFTSpecialInv / FFTSpecialForward) stages.  Explicit
// round-to-nearest intrinsics keep every product and sum unfused so that the
// result matches a plain C evaluation of the same expressions.
__global__ void k_fft_inv_stage(double2* v, const double2* tw, uint32_t slots, uint32_t len) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= slots / 2) return;
  double2* x = v + (size_t)blockIdx.y * slots;
  const uint32_t half = len / 2, j = t % half, i = (t / half) * len + j;
  const double2 a = x[i], b = x[i + half], w = tw[half - 1 + j];
  const double vr = __dsub_rn(a.x, b.x), vi = __dsub_rn(a.y, b.y);
  x[i] = make_double2(__dadd_rn(a.x, b.x), __dadd_rn(a.y, b.y));
  x[i + half] = make_double2(__dsub_rn(__dmul_rn(vr, w.x), __dmul_rn(vi, w.y)),
                             __dadd_rn(__dmul_rn(vi, w.x), __dmul_rn(vr, w.y)));
}

__global__ void k_fft_fwd_stage(double2* v, const double2* tw, uint32_t slots, uint32_t len) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= slots / 2) return;
  double2* x = v + (size_t)blockIdx.y * slots;
  const uint32_t lenh = len / 2, j = t % lenh, i = (t / lenh) * len + j;
  const double2 u = x[i], b = x[i + lenh], w = tw[lenh - 1 + j];
  const double tr = __dsub_rn(__dmul_rn(b.x, w.x), __dmul_rn(b.y, w.y));
  const double ti = __dadd_rn(__dmul_rn(b.x, w.y), __dmul_rn(b.y, w.x));
  x[i] = make_double2(__dadd_rn(u.x, tr), __dadd_rn(u.y, ti));
  x[i + lenh] = make_double2(__dsub_rn(u.x, tr), __dsub_rn(u.y, ti));
}

__global__ void k_encode_round(const double2* v, double* coef, uint32_t slots, uint32_t log_slots,
                               uint32_t n, double scale, unsigned* status) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= slots) return;
  const uint32_t gap = n / (2 * slots);
  const uint32_t src = log_slots ? (__brev(i) >> (32 - log_slots)) : 0;
  const double2 x = v[src];
  const double r = __dmul_rn(__ddiv_rn(x.x, (double)slots), scale);
  const double s = __dmul_rn(__ddiv_rn(x.y, (double)slots), scale);
  const double lim = 0x1p126;
  if (!isfinite(r) || !isfinite(s) || fabs(r) >= lim || fabs(s) >= lim) {
    atomicOr(status, 1u);
    return;
  }
  coef[(size_t)i * gap] = round(r);
  coef[(size_t)i * gap + n / 2] = round(s);
}

// Exact residue of an integer-valued double: below 2^63 through int64, above
// as hi 2^64 + lo (both parts exact: power-of-two scaling and a difference
// that fits the mantissa) reduced by the 128-bit reduction.
__device__ __forceinline__ uint64_t lift_double(double d, const Modulus& m) {
  if (fabs(d) < 0x1p63) return lift_signed((int64_t)d, m);
  const double a = fabs(d);
  const double hi = floor(a * 0x1p-64);
  const double lo = a - hi * 0x1p64;
  const uint64_t r = reduce_u128((uint64_t)hi, (uint64_t)lo, m);
  return d < 0 ? (r ? m.q - r : 0) : r;
}

__global__ void k_lift_double(const double* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                              const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, b = blockIdx.z;
  out[((size_t)b * nlimbs + l) * n + k] = lift_double(src[(size_t)b * n + k], mods[pm(l)]);
}

__device__ __forceinline__ double u128_to_double(uint64_t hi, uint64_t lo) {
  return __dadd_rn(__dmul_rn((double)hi, 18446744073709551616.0), (double)lo);
}

__global__ void k_decode_crt(const uint64_t* coef, uint32_t nlimbs, uint32_t slots, uint32_t log_slots,
                             uint32_t n, double scale, uint64_t q0, uint64_t q1, uint64_t q0inv,
                             uint64_t q0inv_sh, Modulus m1, double2* v) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= slots) return;
  const uint32_t gap = n / (2 * slots);
  double part[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const size_t idx = (size_t)i * gap + (h ? n / 2 : 0);
    const uint64_t a0 = coef[idx];
    double val;
    if (nlimbs == 1) {
      val = a0 > q0 / 2 ? -(double)(q0 - a0) : (double)a0;
    } else {
      const uint64_t a1 = coef[(size_t)n + idx];
      const uint64_t a0m = barrett_reduce(0, a0, m1);
      const uint64_t d = sub_mod(a1, a0m, q1);
      const uint64_t t = shoup_mul(d, q0inv, q0inv_sh, q1);
      // x = a0 + q0 * t  < q0 q1 (128-bit)
      uint64_t lo = q0 * t, hi = __umul64hi(q0, t);
      lo += a0;
      hi += lo < a0;
      const uint64_t Qlo = q0 * q1, Qhi = __umul64hi(q0, q1);
      const uint64_t hlo = (Qlo >> 1) | (Qhi << 63), hhi = Qhi >> 1;  // floor(Q/2)
      const bool neg = hi > hhi || (hi == hhi && lo > hlo);
      if (neg) {  // -(Q - x)
        const uint64_t rlo = Qlo - lo;
        const uint64_t rhi = Qhi - hi - (Qlo < lo);
        val = -u128_to_double(rhi, rlo);
      } else {
        val = u128_to_double(hi, lo);
      }
    }
    part[h] = __ddiv_rn(val, scale);
  }
  const uint32_t dst = log_slots ? (__brev(i) >> (32 - log_slots)) : 0;
  v[dst] = make_double2(part[0], part[1]);
}

__global__ void k_encode_round_batch(const double2* v, double* coef, uint32_t slots, uint32_t log_slots,
                                     uint32_t n, double scale, unsigned* status) {
  const uint32_t b = blockIdx.y;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= slots) return;
  const uint32_t gap = n / (2 * slots);
  const uint32_t src = log_slots ? (__brev(i) >> (32 - log_slots)) : 0;
  const double2 x = v[(size_t)b * slots + src];
  const double r = __dmul_rn(__ddiv_rn(x.x, (double)slots), scale);
  const double s = __dmul_rn(__ddiv_rn(x.y, (double)slots), scale);
  const double lim = 0x1p126;
  if (!isfinite(r) || !isfinite(s) || fabs(r) >= lim || fabs(s) >= lim) {
    atomicOr(status, 1u);
    return;
  }
  double* c = coef + (size_t)b * n;
  c[(size_t)i * gap] = round(r);
  c[(size_t)i * gap + n / 2] = round(s);
}

__global__ void k_lift_small_batch(const int64_t* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                                   const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, b = blockIdx.z;
  out[((size_t)b * nlimbs + l) * n + k] = lift_signed(src[(size_t)b * n + k], mods[pm(l)]);
}

// 128-bit accumulator reduced mod q: (hi 2^64 + lo) mod q with hi < 2^62.
__device__ __forceinline__ uint64_t reduce128(uint64_t hi, uint64_t lo, const Modulus& m, uint64_t r64) {
  const uint64_t h = barrett_reduce(0, hi, m);
  const uint64_t l = barrett_reduce(0, lo, m);
  return add_mod(mul_mod(h, r64, m), l, m.q);
}

constexpr int kMaxBaby = 32;
constexpr int kGiantChunk = 8;  // giants per CTA: neighbouring CTAs share the babies' tile in L1/L2

// Block (x = giant chunk, y = coefficient tile, z = limb).  Each thread owns
// one coefficient and accumulates every giant of its chunk in 128 bits; the
// babies are re-read per giant from L1/L2, the diagonals stream from HBM once.
// The chunk's diagonal pointers and the baby pointers sit in shared memory and
// every load of a batch of 8 babies is issued before its products (an absent
// diagonal reads a zero word instead of branching), so each thread keeps 24
// loads in flight: the stream is bound by HBM, not by load latency.
__device__ const uint64_t g_zero_word = 0;

__global__ void __launch_bounds__(128) k_bsgs_dot(const uint64_t* const* babies, const uint64_t* const* diags,
                                                  uint64_t* out, uint32_t b, uint32_t G, uint32_t nq, uint32_t n,
                                                  const Modulus* mods) {
  constexpr uint32_t kBatch = 8;
  __shared__ const uint64_t* s_diag[kGiantChunk * kMaxBaby];
  __shared__ const uint64_t* s_baby[kMaxBaby];
  const uint32_t g0 = blockIdx.x * kGiantChunk, g1 = min(G, g0 + kGiantChunk);
  for (uint32_t i = threadIdx.x; i < (g1 - g0) * b; i += blockDim.x) s_diag[i] = diags[g0 * b + i];
  for (uint32_t i = threadIdx.x; i < b; i += blockDim.x) s_baby[i] = babies[i];
  __syncthreads();
  const uint32_t k = blockIdx.y * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.z;
  const Modulus m = mods[l];
  const uint64_t r64 = barrett_reduce(1, 0, m);
  const size_t off = (size_t)l * n + k, cs = (size_t)nq * n;
  for (uint32_t g = g0; g < g1; ++g) {
    const uint64_t* const* dg = s_diag + (g - g0) * b;
    uint64_t h0 = 0, l0 = 0, h1 = 0, l1 = 0;
    for (uint32_t jb = 0; jb < b; jb += kBatch) {
      uint64_t d[kBatch], x0[kBatch], x1[kBatch];
#pragma unroll
      for (uint32_t u = 0; u < kBatch; ++u) {
        const uint32_t j = jb + u;
        const uint64_t* dp = j < b ? dg[j] : nullptr;
        const uint64_t* bj = j < b ? s_baby[j] : nullptr;
        d[u] = __ldcs(dp ? dp + off : &g_zero_word);  // streamed once: evict first
        x0[u] = bj ? __ldg(bj + off) : 0;
        x1[u] = bj ? __ldg(bj + cs + off) : 0;
      }
#pragma unroll
      for (uint32_t u = 0; u < kBatch; ++u) {
        uint64_t lo = x0[u] * d[u], hi = __umul64hi(x0[u], d[u]);
        l0 += lo;
        h0 += hi + (l0 < lo);
        lo = x1[u] * d[u];
        hi = __umul64hi(x1[u], d[u]);
        l1 += lo;
        h1 += hi + (l1 < lo);
      }
    }
    uint64_t* o = out + (size_t)g * 2 * cs;
    o[off] = reduce128(h0, l0, m, r64);
    o[cs + off] = reduce128(h1, l1, m, r64);
  }
}

__global__ void k_mul_monomial_half(const uint64_t* a, size_t sa, uint64_t* out, size_t so, uint32_t n,
                                    const Twiddle* tw, const uint64_t* primes) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const uint64_t q = primes[l];
  const Twiddle w = tw[(size_t)l * n + 1];  // psi^{N/2}, a primitive 4th root of unity
  const uint64_t v = shoup_mul(a[c * sa + (size_t)l * n + k], w.w, w.wp, q);
  out[c * so + (size_t)l * n + k] = k < n / 2 ? v : neg_mod(v, q);
}

inline dim3 grid1(uint32_t n, uint32_t y = 1, uint32_t z = 1) { return dim3((n + kTpb - 1) / kTpb, y, z); }

uint32_t log2u(uint32_t x) {
  uint32_t l = 0;
  while ((1u << l) < x) ++l;
  return l;
}

}  // namespace

void launch_sample_small(int kind, uint64_t seed, uint64_t stream, int64_t* out, uint32_t n, cudaStream_t s) {
  k_sample_small<<<grid1(n / 8), kTpb, 0, s>>>(kind, seed, stream, out, n); note_launch();
}

void launch_lift_small(const int64_t* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                       const Modulus* mods, cudaStream_t s) {
  if (!nlimbs) return;
  k_lift_small<<<grid1(n, nlimbs), kTpb, 0, s>>>(src, out, n, pm, mods); note_launch();
}

void launch_sample_uniform(uint64_t seed, uint64_t stream, uint64_t* out, uint32_t n, uint32_t nlimbs,
                           PrimeMap pm, const Modulus* mods, cudaStream_t s) {
  if (!nlimbs) return;
  k_sample_uniform<<<grid1(n / 4, nlimbs), kTpb, 0, s>>>(seed, stream, out, n, pm, mods); note_launch();
}

void launch_ew(Ew op, const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* out, size_t so,
               uint32_t ncomp, uint32_t nlimbs, uint32_t n, PrimeMap pm, const Modulus* mods, cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_ew<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(op, a, sa, b, sb, out, so, n, pm, mods); note_launch();
}

void launch_mul_const(const uint64_t* a, size_t sa, const Shoup* c, const uint64_t* b, size_t sb, uint64_t* out,
                      size_t so, uint32_t ncomp, uint32_t nlimbs, uint32_t n, const uint64_t* primes,
                      cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_mul_const<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(a, sa, c, b, sb, out, so, n, primes); note_launch();
}

void launch_add_const(const uint64_t* a, size_t sa, const uint64_t* c, uint64_t* out, size_t so, uint32_t ncomp,
                      uint32_t nlimbs, uint32_t n, const uint64_t* primes, cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_add_const<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(a, sa, c, out, so, n, primes); note_launch();
}

void launch_mul_const_v(const uint64_t* a, size_t sa, const LimbShoup& c, uint64_t* out, size_t so, uint32_t ncomp,
                        uint32_t nlimbs, uint32_t n, const uint64_t* primes, cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_mul_const_v<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(a, sa, c, out, so, n, primes); note_launch();
}

void launch_add_const_v(const uint64_t* a, size_t sa, const LimbWords& c, uint64_t* out, size_t so, uint32_t ncomp,
                        uint32_t nlimbs, uint32_t n, const uint64_t* primes, cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_add_const_v<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(a, sa, c, out, so, n, primes); note_launch();
}

void launch_linear_wsum(const WsumArgs& a, uint32_t m, const uint64_t* w, const LimbWords& add, int has_add,
                        uint64_t* out, size_t so, uint32_t ncomp, uint32_t nq, uint32_t n, const Modulus* mods,
                        cudaStream_t s) {
  if (!nq || !ncomp) return;
  k_linear_wsum<<<grid1(n, nq, ncomp), kTpb, 0, s>>>(a, m, w, add, has_add, out, so, nq, n, mods); note_launch();
}

void launch_tensor(const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* d, size_t sd,
                   uint32_t nq, uint32_t n, const Modulus* mods, cudaStream_t s) {
  k_tensor<<<grid1(n, nq), kTpb, 0, s>>>(a, sa, b, sb, d, sd, n, mods); note_launch();
}

void launch_automorphism(const uint64_t* in, size_t si, uint64_t* out, size_t so, uint32_t ncomp,
                         uint32_t nlimbs, uint32_t log_n, uint64_t g, cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_automorphism<<<grid1(1u << log_n, nlimbs, ncomp), kTpb, 0, s>>>(in, si, out, so, log_n, g); note_launch();
}

void launch_modup(const uint64_t* coef, const uint64_t* dntt, uint64_t* ext, uint32_t nq, uint32_t K, uint32_t n,
                  const ModUpDigit* digits_dev, uint32_t D, uint32_t alpha, const Modulus* mods, cudaStream_t s,
                  bool primes_below_2_60) {
  // Full digits share one launch, a shorter last digit gets its own.
  const uint32_t full = nq / alpha, rest = nq % alpha;
  auto go = [&](uint32_t ns, uint32_t digit0, uint32_t count) {
    if (!count) return;
    const uint32_t chunks = (nq + K - ns + kTgtChunk - 1) / kTgtChunk;
    const dim3 grid = grid1(n, count, chunks);
    if (primes_below_2_60 && ns <= 16) {
      switch (ns) {
#define FHE_CASE(NS) \
  case NS: k_modup<NS, true><<<grid, kTpb, 0, s>>>(coef, dntt, ext, nq + K, n, digits_dev, digit0, mods); note_launch(); break;
        FHE_NS16_CASES(FHE_CASE)
#undef FHE_CASE
        default: break;
      }
      return;
    }
    switch (ns) {
#define FHE_CASE(NS) \
  case NS: k_modup<NS, false><<<grid, kTpb, 0, s>>>(coef, dntt, ext, nq + K, n, digits_dev, digit0, mods); note_launch(); break;
      FHE_NS_CASES(FHE_CASE)
#undef FHE_CASE
      default: break;
    }
  };
  go(alpha, 0, full);
  go(rest, full, rest ? 1 : 0);
  (void)D;
}

void launch_key_inner(const uint64_t* ext, uint32_t D, uint32_t w, const uint64_t* evk, uint32_t key_limbs,
                      PrimeMap pm, uint64_t* acc, uint32_t n, const Modulus* mods, cudaStream_t s, uint32_t l0,
                      uint32_t count) {
  const uint32_t rows = l0 >= w ? 0 : (count < w - l0 ? count : w - l0);
  if (!rows) return;
  k_key_inner<<<grid1(n, rows), kTpb, 0, s>>>(ext, D, w, evk, key_limbs, pm, acc, n, mods, l0); note_launch();
}

void launch_convert(const uint64_t* src, size_t s_comp, uint64_t* dst, size_t d_comp, uint32_t ncomp,
                    const ConvTable* t_dev, uint32_t ns, uint32_t nt, uint32_t n, const Modulus* mods,
                    cudaStream_t s, bool primes_below_2_60) {
  const uint32_t chunks = (nt + kTgtChunk - 1) / kTgtChunk;
  const dim3 grid = grid1(n, ncomp, chunks);
  if (primes_below_2_60 && ns <= 16) {
    switch (ns) {
#define FHE_CASE(NS) \
  case NS: k_convert<NS, true><<<grid, kTpb, 0, s>>>(src, s_comp, dst, d_comp, t_dev, n, mods); note_launch(); break;
      FHE_NS16_CASES(FHE_CASE)
#undef FHE_CASE
      default: break;
    }
    return;
  }
  switch (ns) {
#define FHE_CASE(NS) \
  case NS: k_convert<NS, false><<<grid, kTpb, 0, s>>>(src, s_comp, dst, d_comp, t_dev, n, mods); note_launch(); break;
    FHE_NS_CASES(FHE_CASE)
#undef FHE_CASE
    default: break;
  }
}

void launch_moddown_combine(const uint64_t* x, size_t sx, const uint64_t* conv, size_t sc, const Shoup* pinv,
                            const uint64_t* add, uint64_t* out, size_t so, uint32_t ncomp, uint32_t nq,
                            uint32_t n, const uint64_t* primes, cudaStream_t s) {
  if (!nq || !ncomp) return;
  k_moddown_combine<<<grid1(n, nq, ncomp), kTpb, 0, s>>>(x, sx, conv, sc, pinv, add, out, so, n, primes); note_launch();
}

void launch_rescale_lift(const uint64_t* last, size_t sl, uint64_t* lifted, size_t sd, uint32_t ncomp,
                         uint32_t nlimbs, uint32_t n, uint64_t q_last, const Modulus* mods, cudaStream_t s) {
  if (!nlimbs) return;
  k_rescale_lift<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(last, sl, lifted, sd, n, q_last, mods); note_launch();
}

// dv[u][s] = W[i][(i + r T + t) % cols] with t = t0 + u, p = (s - (t / baby) baby) mod slots,
// r = p / win, i = p % win (r < R, i < m), else 0: the numpy construction of
// the replicated layout's diagonal t followed by np.roll by its giant step.
__global__ void k_replicated_diagonals(double2* dv, const double* w, uint32_t m, uint32_t cols, uint32_t R,
                                       uint32_t T, uint32_t win, uint32_t baby, uint32_t slots, uint32_t t0) {
  const uint32_t sl = blockIdx.x * blockDim.x + threadIdx.x;
  if (sl >= slots) return;
  const uint32_t u = blockIdx.y, t = t0 + u;
  const uint32_t shift = (t / baby) * baby % slots;
  const uint32_t p = (sl + slots - shift) % slots;
  const uint32_t r = p / win, i = p - r * win;
  double v = 0.0;
  if (r < R && i < m) v = w[(size_t)i * cols + ((uint64_t)i + (uint64_t)r * T + t) % cols];
  dv[(size_t)u * slots + sl] = make_double2(v, 0.0);
}

void launch_replicated_diagonals(double2* dv, const double* w, uint32_t m, uint32_t cols, uint32_t R, uint32_t T,
                                 uint32_t win, uint32_t baby, uint32_t slots, uint32_t t0, uint32_t nb,
                                 cudaStream_t s) {
  if (!nb) return;
  k_replicated_diagonals<<<grid1(slots, nb), kTpb, 0, s>>>(dv, w, m, cols, R, T, win, baby, slots, t0);
  note_launch();
}

void launch_fft_special_inv(double2* v, const double2* tw, uint32_t slots, uint32_t batch, cudaStream_t s) {
  for (uint32_t len = slots; len >= 2; len >>= 1)
    { k_fft_inv_stage<<<grid1(slots / 2, batch), kTpb, 0, s>>>(v, tw, slots, len); note_launch(); }
}

void launch_fft_special_fwd(double2* v, const double2* tw, uint32_t slots, uint32_t batch, cudaStream_t s) {
  for (uint32_t len = 2; len <= slots; len <<= 1)
    { k_fft_fwd_stage<<<grid1(slots / 2, batch), kTpb, 0, s>>>(v, tw, slots, len); note_launch(); }
}

void launch_encode_round(const double2* v, double* coef, uint32_t slots, uint32_t n, double scale,
                         unsigned* status, cudaStream_t s) {
  k_encode_round<<<grid1(slots), kTpb, 0, s>>>(v, coef, slots, log2u(slots), n, scale, status); note_launch();
}

void launch_decode_crt(const uint64_t* coef, uint32_t nlimbs, uint32_t slots, uint32_t n, double scale,
                       uint64_t q0, uint64_t q1, uint64_t q0inv_mod_q1, uint64_t q0inv_shoup, Modulus m1,
                       double2* v, cudaStream_t s) {
  k_decode_crt<<<grid1(slots), kTpb, 0, s>>>(coef, nlimbs, slots, log2u(slots), n, scale, q0, q1, q0inv_mod_q1,
                                             q0inv_shoup, m1, v); note_launch();
}

void launch_encode_round_batch(const double2* v, double* coef, uint32_t slots, uint32_t n, double scale,
                               uint32_t batch, unsigned* status, cudaStream_t s) {
  if (!batch) return;
  k_encode_round_batch<<<grid1(slots, batch), kTpb, 0, s>>>(v, coef, slots, log2u(slots), n, scale, status); note_launch();
}

void launch_lift_double(const double* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                        const Modulus* mods, uint32_t batch, cudaStream_t s) {
  if (!nlimbs || !batch) return;
  k_lift_double<<<grid1(n, nlimbs, batch), kTpb, 0, s>>>(src, out, n, nlimbs, pm, mods); note_launch();
}

void launch_lift_small_batch(const int64_t* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                             const Modulus* mods, uint32_t batch, cudaStream_t s) {
  if (!batch || !nlimbs) return;
  k_lift_small_batch<<<grid1(n, nlimbs, batch), kTpb, 0, s>>>(src, out, n, nlimbs, pm, mods); note_launch();
}

void launch_mul_monomial_half(const uint64_t* a, size_t sa, uint64_t* out, size_t so, uint32_t ncomp,
                              uint32_t nlimbs, uint32_t n, const Twiddle* tw, const uint64_t* primes,
                              cudaStream_t s) {
  if (!nlimbs || !ncomp) return;
  k_mul_monomial_half<<<grid1(n, nlimbs, ncomp), kTpb, 0, s>>>(a, sa, out, so, n, tw, primes); note_launch();
}

void launch_bsgs_dot(const uint64_t* const* babies, const uint64_t* const* diags, uint64_t* out, uint32_t b,
                     uint32_t G, uint32_t nq, uint32_t n, const Modulus* mods, cudaStream_t s) {
  k_bsgs_dot<<<dim3((G + kGiantChunk - 1) / kGiantChunk, (n + 127) / 128, nq), 128, 0, s>>>(babies, diags, out, b,
                                                                                           G, nq, n, mods); note_launch();
}

}  // namespace fhe
