/*
 * CPU oracle, part 1: modular arithmetic, prime chains, roots of unity, NTT
 * and the counter-based sampler.  TEST INFRASTRUCTURE ONLY (see ckks_oracle.h).
 */
#include "ckks_oracle.h"
#include "oracle_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

uint64_t oc_mulmod(uint64_t a, uint64_t b, uint64_t q) {
  return (uint64_t)(((u128)a * b) % q);
}

uint64_t oc_powmod(uint64_t a, uint64_t e, uint64_t q) {
  uint64_t r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = oc_mulmod(r, a, q);
    a = oc_mulmod(a, a, q);
    e >>= 1;
  }
  return r;
}

/* q prime: Fermat inverse. */
uint64_t oc_invmod(uint64_t a, uint64_t q) { return oc_powmod(a, q - 2, q); }

/* Deterministic Miller-Rabin for n < 2^64 with the first twelve prime bases.
 * OpenFHE's MillerRabinPrimalityTest is probabilistic with random witnesses;
 * on the 60-bit candidates the chain generator visits, both agree. */
int oc_is_prime(uint64_t n) {
  static const uint64_t bases[12] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  if (n < 2) return 0;
  for (int i = 0; i < 12; ++i) {
    if (n == bases[i]) return 1;
    if (n % bases[i] == 0) return 0;
  }
  uint64_t d = n - 1;
  int s = 0;
  while ((d & 1) == 0) { d >>= 1; ++s; }
  for (int i = 0; i < 12; ++i) {
    uint64_t x = oc_powmod(bases[i], d, n);
    if (x == 1 || x == n - 1) continue;
    int composite = 1;
    for (int r = 1; r < s; ++r) {
      x = oc_mulmod(x, x, n);
      if (x == n - 1) { composite = 0; break; }
    }
    if (composite) return 0;
  }
  return 1;
}

/* OpenFHE nbtheory.h FirstPrime(nBits, m): the smallest prime q > 2^nBits
 * with q = 1 mod m.  (Reference call site: CCParams SetScalingModSize /
 * SetFirstModSize in native/fideslib_stage0/src/packed_fideslib.cpp:1064.) */
uint64_t oc_first_prime(uint32_t bits, uint64_t m) {
  uint64_t q = (uint64_t)1 << bits;
  uint64_t r = q % m;
  uint64_t qn = q + 1;
  if (r > 0) qn += m - r;
  while (!oc_is_prime(qn)) qn += m;
  return qn;
}

/* OpenFHE PreviousPrime(q, m): the largest prime below q that is = q mod m. */
uint64_t oc_previous_prime(uint64_t q, uint64_t m) {
  uint64_t qn = q - m;
  while (!oc_is_prime(qn)) qn -= m;
  return qn;
}

/* OpenFHE NextPrime(q, m). */
uint64_t oc_next_prime(uint64_t q, uint64_t m) {
  uint64_t qn = q + m;
  while (!oc_is_prime(qn)) qn += m;
  return qn;
}

static int in_list(uint64_t v, const uint64_t* a, uint32_t n) {
  for (uint32_t i = 0; i < n; ++i)
    if (a[i] == v) return 1;
  return 0;
}

/* Exact bit length of a product of u64 moduli (BigInteger GetLengthForBase(2)). */
static uint32_t product_bits(const uint64_t* m, uint32_t n) {
  uint64_t acc[64];
  uint32_t len = 1;
  acc[0] = 1;
  for (uint32_t i = 0; i < n; ++i) {
    u128 carry = 0;
    for (uint32_t j = 0; j < len; ++j) {
      u128 t = (u128)acc[j] * m[i] + carry;
      acc[j] = (uint64_t)t;
      carry = t >> 64;
    }
    if (carry) acc[len++] = (uint64_t)carry;
  }
  uint32_t bits = 64 * (len - 1);
  uint64_t top = acc[len - 1];
  while (top) { ++bits; top >>= 1; }
  return bits;
}

/*
 * CKKS modulus chain with FLEXIBLEAUTO prime selection and HYBRID special
 * primes, restating OpenFHE v1.4.2 ParameterGenerationCKKSRNS::ParamsGenCKKSRNS
 * (scaling-factor-tracking selection that alternates PreviousPrime/NextPrime
 * around sf_{i} = sf_{i+1}^2 / q_{i+1}) and the HYBRID P selection in
 * CryptoParametersRNS::PrecomputeCRTTables (sizeP = ceil(maxDigitBits / 60),
 * PreviousPrime from FirstPrime(60, 2N), skipping Q primes).
 * Reference parameters: packed_fideslib.cpp:1060-1068 (depth 44, scale 59,
 * first 60, FLEXIBLEAUTO, HYBRID) and the recorded chain in
 * results/b300/2026-09-28/long-accuracy/oracle-p-r3-base/native.json:1.
 */
int oc_ckks_moduli(uint32_t log_n, uint32_t num_q, uint32_t scale_bits,
                   uint32_t first_bits, uint32_t dnum, uint64_t* q_out,
                   uint64_t* p_out, uint32_t max_p) {
  if (num_q < 1 || num_q > 64 || dnum < 1 || scale_bits > 61 || first_bits > 61) return -1;
  const uint64_t m = (uint64_t)2 << log_n; /* cyclotomic order 2N */
  uint64_t* Q = q_out;
  Q[num_q - 1] = oc_first_prime(scale_bits, m);
  if (num_q > 1) {
    double sf = (double)Q[num_q - 1];
    uint32_t cnt = 0;
    for (int i = (int)num_q - 2; i >= 1; --i) {
      sf = pow(sf, 2) / (double)Q[i + 1];
      uint64_t sf_int = (uint64_t)llround(sf);
      uint64_t sf_rem = sf_int % m;
      if ((cnt % 2) == 0) {
        uint64_t qp = sf_int - m - sf_rem + 1;
        do { qp = oc_previous_prime(qp, m); } while (in_list(qp, Q + i + 1, num_q - i - 1));
        Q[i] = qp;
      } else {
        uint64_t qn = sf_int + m - sf_rem + 1;
        do { qn = oc_next_prime(qn, m); } while (in_list(qn, Q + i + 1, num_q - i - 1));
        Q[i] = qn;
      }
      ++cnt;
    }
    /* Equal first and scaling sizes take a different OpenFHE branch that no
     * recorded chain pins; it is rejected rather than guessed. */
    if (first_bits == scale_bits) return -3;
    Q[0] = oc_previous_prime(oc_first_prime(first_bits, m), m);
  }
  /* HYBRID special primes. */
  uint32_t alpha = (num_q + dnum - 1) / dnum;
  uint32_t parts = (num_q + alpha - 1) / alpha;
  uint32_t max_bits = 0;
  for (uint32_t j = 0; j < parts; ++j) {
    uint32_t lo = j * alpha, hi = lo + alpha < num_q ? lo + alpha : num_q;
    uint32_t b = product_bits(Q + lo, hi - lo);
    if (b > max_bits) max_bits = b;
  }
  const uint32_t aux_bits = 60;
  uint32_t size_p = (max_bits + aux_bits - 1) / aux_bits;
  if (size_p > max_p) return -2;
  uint64_t prev = oc_first_prime(aux_bits, m);
  for (uint32_t i = 0; i < size_p; ++i) {
    uint64_t c;
    do { c = oc_previous_prime(prev, m); prev = c; } while (in_list(c, Q, num_q));
    p_out[i] = c;
  }
  return (int)size_p;
}

void oc_ntt_primes(uint32_t log_n, uint32_t bits, uint32_t k, uint64_t* out) {
  const uint64_t m = (uint64_t)2 << log_n;
  uint64_t q = ((uint64_t)1 << bits) + 1; /* = 1 mod m */
  for (uint32_t i = 0; i < k; ++i) {
    q = oc_previous_prime(q, m);
    out[i] = q;
  }
}

/* OpenFHE RootOfUnity(m, q): the numerically smallest primitive m-th root.
 * (m is a power of two, so the primitive roots are the odd powers of any one.) */
uint64_t oc_root_of_unity(uint64_t m, uint64_t q) {
  uint64_t g = 0;
  for (uint64_t x = 2; x < q; ++x) {
    g = oc_powmod(x, (q - 1) / m, q);
    if (oc_powmod(g, m / 2, q) == q - 1) break;
  }
  uint64_t g2 = oc_mulmod(g, g, q);
  uint64_t x = g, best = g;
  for (uint64_t k = 3; k < m; k += 2) {
    x = oc_mulmod(x, g2, q);
    if (x < best) best = x;
  }
  return best;
}

uint32_t oi_bitrev(uint32_t x, uint32_t bits) {
  uint32_t r = 0;
  for (uint32_t i = 0; i < bits; ++i) { r = (r << 1) | (x & 1); x >>= 1; }
  return r;
}

twiddles_t oi_make_table(uint32_t log_n, uint64_t q, uint64_t root) {
  const uint32_t n = 1u << log_n;
  twiddles_t t;
  t.w = (uint64_t*)malloc(sizeof(uint64_t) * n);
  t.wp = (uint64_t*)malloc(sizeof(uint64_t) * n);
  uint64_t x = 1;
  for (uint32_t i = 0; i < n; ++i) {
    uint32_t r = oi_bitrev(i, log_n);
    t.w[r] = x;
    t.wp[r] = (uint64_t)(((u128)x << 64) / q);
    x = oc_mulmod(x, root, q);
  }
  return t;
}

void oi_free_table(twiddles_t* t) { free(t->w); free(t->wp); }


/* OpenFHE ChineseRemainderTransformFTTNat::ForwardTransformToBitReverseInPlace:
 * Cooley-Tukey, natural-order input, bit-reversed output, table psi^{brv(i)}.
 * Output word i is a(psi^{2*brv(i)+1}) mod q. */
void oi_ntt_fwd_table(uint64_t* a, uint32_t log_n, uint64_t q, const twiddles_t* t) {
  const uint32_t n = 1u << log_n;
  for (uint32_t m = 1, h = n >> 1; m < n; m <<= 1, h >>= 1) {
    for (uint32_t i = 0; i < m; ++i) {
      const uint64_t w = t->w[m + i], wp = t->wp[m + i];
      for (uint32_t j = 2 * i * h; j < 2 * i * h + h; ++j) {
        uint64_t u = a[j];
        uint64_t v = oi_mul_shoup(a[j + h], w, wp, q);
        uint64_t s = u + v;
        a[j] = s >= q ? s - q : s;
        a[j + h] = u >= v ? u - v : u + q - v;
      }
    }
  }
}

/* OpenFHE InverseTransformFromBitReverseInPlace: Gentleman-Sande with
 * psi^{-brv(i)}, then a multiply by N^{-1}. */
void oi_ntt_inv_table(uint64_t* a, uint32_t log_n, uint64_t q, const twiddles_t* t) {
  const uint32_t n = 1u << log_n;
  for (uint32_t m = n >> 1, h = 1; m >= 1; m >>= 1, h <<= 1) {
    for (uint32_t i = 0; i < m; ++i) {
      const uint64_t w = t->w[m + i], wp = t->wp[m + i];
      for (uint32_t j = 2 * i * h; j < 2 * i * h + h; ++j) {
        uint64_t u = a[j], v = a[j + h];
        uint64_t s = u + v;
        a[j] = s >= q ? s - q : s;
        a[j + h] = oi_mul_shoup(u >= v ? u - v : u + q - v, w, wp, q);
      }
    }
  }
  const uint64_t ninv = oc_invmod(n % q, q);
  const uint64_t ninvp = (uint64_t)(((u128)ninv << 64) / q);
  for (uint32_t j = 0; j < n; ++j) a[j] = oi_mul_shoup(a[j], ninv, ninvp, q);
}

void oc_ntt_forward(uint64_t* a, uint32_t log_n, uint64_t q, uint64_t psi) {
  twiddles_t t = oi_make_table(log_n, q, psi);
  oi_ntt_fwd_table(a, log_n, q, &t);
  oi_free_table(&t);
}

void oc_ntt_inverse(uint64_t* a, uint32_t log_n, uint64_t q, uint64_t psi) {
  twiddles_t t = oi_make_table(log_n, q, oc_invmod(psi, q));
  oi_ntt_inv_table(a, log_n, q, &t);
  oi_free_table(&t);
}

void oc_ntt_batch(uint64_t* data, uint32_t n_polys, uint32_t n_limbs,
                  uint32_t log_n, const uint64_t* q, const uint64_t* psi,
                  int inverse, int threads) {
  const uint64_t n = (uint64_t)1 << log_n;
  twiddles_t* tabs = (twiddles_t*)malloc(sizeof(twiddles_t) * n_limbs);
  for (uint32_t l = 0; l < n_limbs; ++l)
    tabs[l] = oi_make_table(log_n, q[l], inverse ? oc_invmod(psi[l], q[l]) : psi[l]);
  const long total = (long)n_polys * n_limbs;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
  for (long k = 0; k < total; ++k) {
    const uint32_t l = (uint32_t)(k % n_limbs);
    uint64_t* a = data + (uint64_t)k * n;
    if (inverse) oi_ntt_inv_table(a, log_n, q[l], &tabs[l]);
    else oi_ntt_fwd_table(a, log_n, q[l], &tabs[l]);
  }
  for (uint32_t l = 0; l < n_limbs; ++l) oi_free_table(&tabs[l]);
  free(tabs);
}

/* ChaCha20 block function (RFC 8439 quarter round and 20 rounds) used as a
 * counter-based generator: key = (seed, derived words), 64-bit block counter,
 * 64-bit stream id as nonce.  Word `index` of the keystream for (seed, stream). */
#define ROTL32(v, c) (((v) << (c)) | ((v) >> (32 - (c))))
#define QR(a, b, c, d)                 \
  a += b; d ^= a; d = ROTL32(d, 16);   \
  c += d; b ^= c; b = ROTL32(b, 12);   \
  a += b; d ^= a; d = ROTL32(d, 8);    \
  c += d; b ^= c; b = ROTL32(b, 7);

static void chacha_block(uint64_t seed, uint64_t stream, uint64_t counter, uint32_t out[16]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    (uint32_t)seed, (uint32_t)(seed >> 32), 0x243f6a88u, 0x85a308d3u,
                    0x13198a2eu, 0x03707344u, 0xa4093822u, 0x299f31d0u,
                    (uint32_t)counter, (uint32_t)(counter >> 32),
                    (uint32_t)stream, (uint32_t)(stream >> 32)};
  uint32_t x[16];
  memcpy(x, s, sizeof(x));
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
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

uint64_t oc_rand_u64(uint64_t seed, uint64_t stream, uint64_t index) {
  uint32_t b[16];
  chacha_block(seed, stream, index >> 3, b);
  const uint32_t w = (uint32_t)(index & 7);
  return (uint64_t)b[2 * w] | ((uint64_t)b[2 * w + 1] << 32);
}
