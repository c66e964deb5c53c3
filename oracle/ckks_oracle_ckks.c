/*
 * CPU oracle, part 2: RNS-CKKS — TEST INFRASTRUCTURE ONLY (see ckks_oracle.h).
 *
 * Restates the algorithms the reference evaluates through OpenFHE v1.4.2 /
 * FIDESlib (HYBRID key switching, FLEXIBLEAUTO rescale, CKKS packed encoding)
 * in plain C with exact integer arithmetic.  Every residue polynomial is kept
 * limb-major, u64[limbs][N]; a polynomial "over Q_l (+P)" has its first nq
 * limbs on primes 0..nq-1 and, when extended, K more limbs on the P primes
 * (context prime indices L..L+K-1).
 */
#include <complex.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "ckks_oracle.h"
#include "oracle_internal.h"

#define OC_MAXP 128

struct oc_ctx {
  uint32_t log_n, n, L, K, dnum, alpha, slots, log_slots;
  uint64_t primes[OC_MAXP];
  uint64_t psi[OC_MAXP];
  twiddles_t fwd[OC_MAXP];
  twiddles_t inv[OC_MAXP];
  uint64_t ninv[OC_MAXP];
  double* fft_re; /* special-FFT twiddles, entry len/2-1+j */
  double* fft_im;
  uint32_t* rot_group; /* 5^j mod 4*slots */
};

static inline uint64_t mulm(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }
static inline uint64_t addm(uint64_t a, uint64_t b, uint64_t q) { uint64_t s = a + b; return s >= q ? s - q : s; }
static inline uint64_t subm(uint64_t a, uint64_t b, uint64_t q) { return a >= b ? a - b : a + q - b; }
static inline uint64_t lift_signed(int64_t v, uint64_t q) {
  if (v >= 0) return (uint64_t)v % q;
  uint64_t m = (uint64_t)(-(v + 1)) + 1; /* |v| without overflow */
  m %= q;
  return m ? q - m : 0;
}

/* prime index of limb l of a poly with nq Q limbs followed by P limbs */
static inline uint32_t pidx(const oc_ctx* c, uint32_t nq, uint32_t l) { return l < nq ? l : c->L + (l - nq); }

oc_ctx* oc_ctx_new(uint32_t log_n, uint32_t L, uint32_t K, const uint64_t* primes, uint32_t dnum,
                   uint32_t slots) {
  if (L + K > OC_MAXP || L == 0 || dnum == 0) return NULL;
  oc_ctx* c = (oc_ctx*)calloc(1, sizeof(oc_ctx));
  c->log_n = log_n;
  c->n = 1u << log_n;
  c->L = L;
  c->K = K;
  c->dnum = dnum;
  c->alpha = (L + dnum - 1) / dnum;
  c->slots = slots;
  c->log_slots = 0;
  while ((1u << c->log_slots) < slots) ++c->log_slots;
  const uint64_t m = 2ull * c->n;
#pragma omp parallel for schedule(dynamic, 1)
  for (int i = 0; i < (int)(L + K); ++i) {
    c->primes[i] = primes[i];
    c->psi[i] = oc_root_of_unity(m, primes[i]);
    c->fwd[i] = oi_make_table(log_n, primes[i], c->psi[i]);
    c->inv[i] = oi_make_table(log_n, primes[i], oc_invmod(c->psi[i], primes[i]));
    c->ninv[i] = oc_invmod(c->n % primes[i], primes[i]);
  }
  /* Special FFT twiddles: OpenFHE order, exponent (4len - 5^j mod 4len) * (M/4len), M = 4*slots
   * (same rule as native/fideslib_stage0/src/gpu_special_fft.cu:89-113). */
  const uint32_t M = 4 * slots;
  c->rot_group = (uint32_t*)malloc(sizeof(uint32_t) * (slots ? slots : 1));
  c->fft_re = (double*)calloc(slots ? slots : 1, sizeof(double));
  c->fft_im = (double*)calloc(slots ? slots : 1, sizeof(double));
  uint32_t p = 1;
  for (uint32_t j = 0; j < slots; ++j) { c->rot_group[j] = p; p = (uint32_t)((uint64_t)p * 5 % M); }
  for (uint32_t len = 2; len <= slots; len *= 2)
    for (uint32_t j = 0; j < len / 2; ++j) {
      const uint32_t index = (4 * len - c->rot_group[j] % (4 * len)) * (M / (4 * len));
      const double angle = 2.0 * M_PI * index / M;
      c->fft_re[len / 2 - 1 + j] = cos(angle);
      c->fft_im[len / 2 - 1 + j] = sin(angle);
    }
  return c;
}

void oc_ctx_free(oc_ctx* c) {
  if (!c) return;
  for (uint32_t i = 0; i < c->L + c->K; ++i) { oi_free_table(&c->fwd[i]); oi_free_table(&c->inv[i]); }
  free(c->fft_re);
  free(c->fft_im);
  free(c->rot_group);
  free(c);
}

uint64_t oc_ctx_psi(const oc_ctx* c, uint32_t i) { return c->psi[i]; }

/* ---- limb transforms ---------------------------------------------------- */

static void ntt_limb(const oc_ctx* c, uint64_t* a, uint32_t p, int inverse) {
  if (inverse) oi_ntt_inv_table(a, c->log_n, c->primes[p], &c->inv[p]);
  else oi_ntt_fwd_table(a, c->log_n, c->primes[p], &c->fwd[p]);
}

void oc_poly_ntt(const oc_ctx* c, uint64_t* a, uint32_t nq, uint32_t np, int inverse) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int l = 0; l < (int)(nq + np); ++l) ntt_limb(c, a + (size_t)l * c->n, pidx(c, nq, l), inverse);
}

/* ---- sampling (identical definition in the CUDA product) ----------------- */

int64_t oc_sample_ternary_coef(uint64_t seed, uint64_t stream, uint64_t k) {
  const uint64_t r = oc_rand_u64(seed, stream, k) % 3;
  return r == 2 ? -1 : (int64_t)r;
}

/* Centred binomial with 21 coin pairs (variance 10.5, sigma 3.24; OpenFHE's
 * discrete Gaussian uses sigma 3.19). */
int64_t oc_sample_error_coef(uint64_t seed, uint64_t stream, uint64_t k) {
  const uint64_t r = oc_rand_u64(seed, stream, k);
  return (int64_t)__builtin_popcountll(r & 0x1FFFFFull) - (int64_t)__builtin_popcountll((r >> 21) & 0x1FFFFFull);
}

uint64_t oc_sample_uniform_coef(uint64_t seed, uint64_t stream, uint32_t prime, uint32_t n,
                                uint64_t k, uint64_t q) {
  const uint64_t idx = 2 * ((uint64_t)prime * n + k);
  const uint64_t hi = oc_rand_u64(seed, stream, idx), lo = oc_rand_u64(seed, stream, idx + 1);
  return (uint64_t)((((u128)hi) << 64 | lo) % q);
}

void oc_sample_small(const oc_ctx* c, uint64_t seed, uint64_t stream, int kind, int64_t* out) {
  for (uint32_t k = 0; k < c->n; ++k)
    out[k] = kind == 0 ? oc_sample_ternary_coef(seed, stream, k) : oc_sample_error_coef(seed, stream, k);
}

/* Small signed polynomial -> RNS over nq Q limbs (+ np P limbs), NTT form if ntt. */
void oc_lift_small(const oc_ctx* c, const int64_t* s, uint64_t* out, uint32_t nq, uint32_t np, int ntt) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int l = 0; l < (int)(nq + np); ++l) {
    const uint32_t p = pidx(c, nq, l);
    uint64_t* a = out + (size_t)l * c->n;
    for (uint32_t k = 0; k < c->n; ++k) a[k] = lift_signed(s[k], c->primes[p]);
    if (ntt) ntt_limb(c, a, p, 0);
  }
}

void oc_sample_uniform_poly(const oc_ctx* c, uint64_t seed, uint64_t stream, uint64_t* out,
                            uint32_t nq, uint32_t np) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int l = 0; l < (int)(nq + np); ++l) {
    const uint32_t p = pidx(c, nq, l);
    uint64_t* a = out + (size_t)l * c->n;
    for (uint32_t k = 0; k < c->n; ++k) a[k] = oc_sample_uniform_coef(seed, stream, p, c->n, k, c->primes[p]);
  }
}

/* ---- keys --------------------------------------------------------------- */

/* Secret key: ternary s, NTT form over all L+K primes (limb-major [L+K][N]). */
void oc_keygen_secret(const oc_ctx* c, uint64_t seed, int64_t* s_coef, uint64_t* s_ntt) {
  oc_sample_small(c, seed, OC_STREAM_SECRET, 0, s_coef);
  oc_lift_small(c, s_coef, s_ntt, c->L, c->K, 1);
}

/* Public key (b, a) over Q: a uniform, b = -a s + e.  pk = [2][L][N]. */
void oc_keygen_public(const oc_ctx* c, uint64_t seed, const uint64_t* s_ntt, uint64_t* pk) {
  const size_t n = c->n;
  uint64_t* b = pk;
  uint64_t* a = pk + (size_t)c->L * n;
  int64_t* e = (int64_t*)malloc(sizeof(int64_t) * n);
  uint64_t* en = (uint64_t*)malloc(sizeof(uint64_t) * n * c->L);
  oc_sample_uniform_poly(c, seed, OC_STREAM_PK_A, a, c->L, 0);
  oc_sample_small(c, seed, OC_STREAM_PK_E, 1, e);
  oc_lift_small(c, e, en, c->L, 0, 1);
  for (uint32_t l = 0; l < c->L; ++l) {
    const uint64_t q = c->primes[l];
    for (size_t k = 0; k < n; ++k)
      b[l * n + k] = subm(en[l * n + k], mulm(a[l * n + k], s_ntt[l * n + k], q), q);
  }
  free(e);
  free(en);
}

/* P mod q_i */
static uint64_t p_mod(const oc_ctx* c, uint64_t q) {
  uint64_t r = 1 % q;
  for (uint32_t k = 0; k < c->K; ++k) r = mulm(r, c->primes[c->L + k] % q, q);
  return r;
}

uint32_t oc_num_digits(const oc_ctx* c, uint32_t nq) { return (nq + c->alpha - 1) / c->alpha; }

/* HYBRID switching key (both keys NTT form over all L+K primes): the key
 * switch of d returns (u0, u1) with u0 + u1 s = d s' + small, i.e.
 * digit j: a_j uniform, b_j = -a_j s + e_j + [l in digit j] (P mod q_l) s'_l.
 * Relinearisation: s' = s^2.  Rotation by g: s' = s_old, s = sigma_g^{-1}(s_old).
 * evk = [D][2][L+K][N], D = ceil(L / alpha). */
void oc_keygen_switch(const oc_ctx* c, uint64_t seed, uint64_t key_id, const uint64_t* s_ntt,
                      const uint64_t* sp_ntt, uint64_t* evk) {
  const size_t n = c->n, lk = c->L + c->K;
  const uint32_t D = oc_num_digits(c, c->L);
  int64_t* e = (int64_t*)malloc(sizeof(int64_t) * n);
  uint64_t* en = (uint64_t*)malloc(sizeof(uint64_t) * n * lk);
  for (uint32_t j = 0; j < D; ++j) {
    uint64_t* b = evk + (size_t)j * 2 * lk * n;
    uint64_t* a = b + lk * n;
    oc_sample_uniform_poly(c, seed, OC_STREAM_KEY_A(key_id, j), a, c->L, c->K);
    oc_sample_small(c, seed, OC_STREAM_KEY_E(key_id, j), 1, e);
    oc_lift_small(c, e, en, c->L, c->K, 1);
    const uint32_t lo = j * c->alpha, hi = lo + c->alpha < c->L ? lo + c->alpha : c->L;
    for (uint32_t l = 0; l < lk; ++l) {
      const uint64_t q = c->primes[l];
      const int in_digit = l >= lo && l < hi;
      const uint64_t pm = in_digit ? p_mod(c, q) : 0;
      for (size_t k = 0; k < n; ++k) {
        uint64_t v = subm(en[l * n + k], mulm(a[l * n + k], s_ntt[l * n + k], q), q);
        if (in_digit) v = addm(v, mulm(pm, sp_ntt[l * n + k], q), q);
        b[l * n + k] = v;
      }
    }
  }
  free(e);
  free(en);
}

/* ---- automorphisms -------------------------------------------------------- */

/* sigma_g on NTT-form limbs: out[i] = in[j], 2 brv(j)+1 = (2 brv(i)+1) g mod 2N. */
void oc_automorphism_ntt(const oc_ctx* c, const uint64_t* in, uint32_t nlimbs, uint64_t g, uint64_t* out) {
  const uint32_t n = c->n, m = 2 * n;
  uint32_t* perm = (uint32_t*)malloc(sizeof(uint32_t) * n);
  for (uint32_t i = 0; i < n; ++i) {
    const uint64_t e = (2ull * oi_bitrev(i, c->log_n) + 1) * g % m;
    perm[i] = oi_bitrev((uint32_t)((e - 1) / 2), c->log_n);
  }
  for (uint32_t l = 0; l < nlimbs; ++l)
    for (uint32_t i = 0; i < n; ++i) out[(size_t)l * n + i] = in[(size_t)l * n + perm[i]];
  free(perm);
}

/* sigma_g on a small signed coefficient vector: X^k -> X^{kg mod 2N} (sign flip past N). */
void oc_automorphism_coef(const oc_ctx* c, const int64_t* in, uint64_t g, int64_t* out) {
  const uint64_t n = c->n, m = 2 * n;
  for (uint64_t k = 0; k < n; ++k) {
    const uint64_t t = k * g % m;
    if (t < n) out[t] = in[k];
    else out[t - n] = -in[k];
  }
}

uint64_t oc_rotation_galois(const oc_ctx* c, int64_t r) {
  const uint64_t m = 2ull * c->n;
  const int64_t order = (int64_t)(c->n / 2);
  int64_t e = r % order;
  if (e < 0) e += order;
  return oc_powmod(5, (uint64_t)e, m);
}

/* ---- encode / decode (CKKS packed encoding, OpenFHE order) --------------- */

static void fft_special_inv(const oc_ctx* c, double* re, double* im) {
  const uint32_t slots = c->slots;
  for (uint32_t len = slots; len >= 2; len >>= 1) {
    const uint32_t half = len / 2;
    for (uint32_t t = 0; t < slots / 2; ++t) {
      const uint32_t j = t % half, i = (t / half) * len + j;
      const double ar = re[i], ai = im[i], br = re[i + half], bi = im[i + half];
      const double wr = c->fft_re[half - 1 + j], wi = c->fft_im[half - 1 + j];
      const double vr = ar - br, vi = ai - bi;
      re[i] = ar + br;
      im[i] = ai + bi;
      re[i + half] = vr * wr - vi * wi;
      im[i + half] = vi * wr + vr * wi;
    }
  }
}

/* Encode `count` complex values at `scale` over nq limbs (NTT form).  Returns
 * 0, or -1 when a scaled coefficient is not finite or exceeds 2^62. */
int oc_encode(const oc_ctx* c, const double* re_in, const double* im_in, uint32_t count, double scale,
              uint32_t nq, uint64_t* out) {
  const uint32_t slots = c->slots, n = c->n, gap = n / (2 * slots);
  double* re = (double*)calloc(slots, sizeof(double));
  double* im = (double*)calloc(slots, sizeof(double));
  for (uint32_t i = 0; i < count && i < slots; ++i) {
    re[i] = re_in[i];
    im[i] = im_in ? im_in[i] : 0.0;
  }
  fft_special_inv(c, re, im);
  int64_t* coef = (int64_t*)calloc(n, sizeof(int64_t));
  int bad = 0;
  for (uint32_t i = 0; i < slots; ++i) {
    const uint32_t src = c->log_slots ? oi_bitrev(i, c->log_slots) : 0;
    const double r = (re[src] / (double)slots) * scale;
    const double s = (im[src] / (double)slots) * scale;
    if (!isfinite(r) || !isfinite(s) || fabs(r) >= 4611686018427387904.0 || fabs(s) >= 4611686018427387904.0) {
      bad = 1;
      break;
    }
    coef[(size_t)i * gap] = llround(r);
    coef[(size_t)i * gap + n / 2] = llround(s);
  }
  if (!bad) oc_lift_small(c, coef, out, nq, 0, 1);
  free(re);
  free(im);
  free(coef);
  return bad ? -1 : 0;
}

/* Centred CRT value of residues r[0..nq) (mixed radix, Garner), as long double. */
static long double crt_centered(const oc_ctx* c, const uint64_t* r, uint32_t nq, uint64_t* digits) {
  /* mixed-radix digits a_i: x = a_0 + a_1 q_0 + a_2 q_0 q_1 + ... */
  for (uint32_t i = 0; i < nq; ++i) {
    const uint64_t qi = c->primes[i];
    uint64_t v = r[i] % qi;
    uint64_t prod = 1 % qi;
    uint64_t acc = 0;
    for (uint32_t j = 0; j < i; ++j) {
      acc = addm(acc, mulm(digits[j] % qi, prod, qi), qi);
      prod = mulm(prod, c->primes[j] % qi, qi);
    }
    v = subm(v, acc, qi);
    digits[i] = mulm(v, oc_invmod(prod, qi), qi);
  }
  /* y = Q - x in mixed radix: Q - 1 has digits (q_i - 1); add 1 with carry. */
  uint64_t* y = (uint64_t*)malloc(sizeof(uint64_t) * (nq ? nq : 1));
  uint64_t carry = 1;
  for (uint32_t i = 0; i < nq; ++i) {
    uint64_t v = c->primes[i] - 1 - digits[i] + carry;
    if (v == c->primes[i]) { v = 0; carry = 1; } else { carry = 0; }
    y[i] = v;
  }
  /* x > Q/2  <=>  x > Q - x (Q odd) */
  int neg = 0;
  for (int i = (int)nq - 1; i >= 0; --i) {
    if (digits[i] != y[i]) { neg = digits[i] > y[i]; break; }
  }
  if (neg) memcpy(digits, y, sizeof(uint64_t) * nq);
  free(y);
  long double v = 0;
  for (int i = (int)nq - 1; i >= 0; --i) v = v * (long double)c->primes[i] + (long double)digits[i];
  return neg ? -v : v;
}

/* Decode an NTT-form plaintext over nq limbs at `scale` into slots complex values. */
void oc_decode(const oc_ctx* c, const uint64_t* pt, uint32_t nq, double scale, double* re, double* im) {
  const uint32_t n = c->n, slots = c->slots, gap = n / (2 * slots);
  uint64_t* a = (uint64_t*)malloc(sizeof(uint64_t) * n * nq);
  memcpy(a, pt, sizeof(uint64_t) * n * nq);
  oc_poly_ntt(c, a, nq, 0, 1);
  uint64_t* res = (uint64_t*)malloc(sizeof(uint64_t) * nq);
  uint64_t* dig = (uint64_t*)malloc(sizeof(uint64_t) * nq);
  double* vr = (double*)malloc(sizeof(double) * slots);
  double* vi = (double*)malloc(sizeof(double) * slots);
  for (uint32_t i = 0; i < slots; ++i) {
    for (uint32_t l = 0; l < nq; ++l) res[l] = a[(size_t)l * n + (size_t)i * gap];
    vr[i] = (double)(crt_centered(c, res, nq, dig) / scale);
    for (uint32_t l = 0; l < nq; ++l) res[l] = a[(size_t)l * n + (size_t)i * gap + n / 2];
    vi[i] = (double)(crt_centered(c, res, nq, dig) / scale);
  }
  /* FFTSpecialForward: bit-reverse, then butterflies len = 2..slots. */
  for (uint32_t i = 0; i < slots; ++i) {
    const uint32_t j = c->log_slots ? oi_bitrev(i, c->log_slots) : 0;
    re[i] = vr[j];
    im[i] = vi[j];
  }
  const uint32_t M = 4 * slots;
  for (uint32_t len = 2; len <= slots; len <<= 1) {
    const uint32_t lenh = len >> 1, lenq = len << 2;
    for (uint32_t i = 0; i < slots; i += len)
      for (uint32_t j = 0; j < lenh; ++j) {
        const uint32_t idx = (c->rot_group[j] % lenq) * (M / lenq);
        const double ang = 2.0 * M_PI * idx / M;
        const double wr = cos(ang), wi = sin(ang);
        const double ur = re[i + j], ui = im[i + j];
        const double xr = re[i + j + lenh], xi = im[i + j + lenh];
        const double tr = xr * wr - xi * wi, ti = xr * wi + xi * wr;
        re[i + j] = ur + tr;
        im[i + j] = ui + ti;
        re[i + j + lenh] = ur - tr;
        im[i + j + lenh] = ui - ti;
      }
  }
  free(a);
  free(res);
  free(dig);
  free(vr);
  free(vi);
}

/* ---- encryption ----------------------------------------------------------- */

/* Public-key encryption at nq limbs: c0 = b v + e0 + m, c1 = a v + e1. ct = [2][nq][N]. */
void oc_encrypt_pk(const oc_ctx* c, uint64_t seed, uint64_t nonce, const uint64_t* pk, const uint64_t* pt,
                   uint32_t nq, uint64_t* ct) {
  const size_t n = c->n;
  int64_t* small = (int64_t*)malloc(sizeof(int64_t) * n);
  uint64_t* v = (uint64_t*)malloc(sizeof(uint64_t) * n * nq);
  uint64_t* e0 = (uint64_t*)malloc(sizeof(uint64_t) * n * nq);
  uint64_t* e1 = (uint64_t*)malloc(sizeof(uint64_t) * n * nq);
  oc_sample_small(c, seed, OC_STREAM_ENC_V(nonce), 0, small);
  oc_lift_small(c, small, v, nq, 0, 1);
  oc_sample_small(c, seed, OC_STREAM_ENC_E0(nonce), 1, small);
  oc_lift_small(c, small, e0, nq, 0, 1);
  oc_sample_small(c, seed, OC_STREAM_ENC_E1(nonce), 1, small);
  oc_lift_small(c, small, e1, nq, 0, 1);
  const uint64_t* b = pk;
  const uint64_t* a = pk + (size_t)c->L * n;
  for (uint32_t l = 0; l < nq; ++l) {
    const uint64_t q = c->primes[l];
    for (size_t k = 0; k < n; ++k) {
      const size_t i = l * n + k;
      ct[i] = addm(addm(mulm(b[i], v[i], q), e0[i], q), pt[i], q);
      ct[nq * n + i] = addm(mulm(a[i], v[i], q), e1[i], q);
    }
  }
  free(small);
  free(v);
  free(e0);
  free(e1);
}

/* m = c0 + c1 s (+ c2 s^2 when ncomp == 3), NTT form over nq limbs. */
void oc_decrypt(const oc_ctx* c, const uint64_t* s_ntt, const uint64_t* ct, uint32_t ncomp, uint32_t nq,
                uint64_t* pt) {
  const size_t n = c->n;
  for (uint32_t l = 0; l < nq; ++l) {
    const uint64_t q = c->primes[l];
    for (size_t k = 0; k < n; ++k) {
      const size_t i = l * n + k;
      const uint64_t s = s_ntt[i];
      uint64_t v = addm(ct[i], mulm(ct[nq * n + i], s, q), q);
      if (ncomp == 3) v = addm(v, mulm(ct[2 * nq * n + i], mulm(s, s, q), q), q);
      pt[i] = v;
    }
  }
}

/* ---- ciphertext arithmetic ------------------------------------------------- */

void oc_add(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nlimbs, uint64_t* out) {
  const size_t n = c->n;
  for (uint32_t l = 0; l < nlimbs; ++l)
    for (size_t k = 0; k < n; ++k) out[l * n + k] = addm(a[l * n + k], b[l * n + k], c->primes[l]);
}

void oc_sub(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nlimbs, uint64_t* out) {
  const size_t n = c->n;
  for (uint32_t l = 0; l < nlimbs; ++l)
    for (size_t k = 0; k < n; ++k) out[l * n + k] = subm(a[l * n + k], b[l * n + k], c->primes[l]);
}

/* Pointwise product of NTT-form polys over nq Q limbs. */
void oc_mul_pointwise(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nlimbs, uint64_t* out) {
  const size_t n = c->n;
  for (uint32_t l = 0; l < nlimbs; ++l)
    for (size_t k = 0; k < n; ++k) out[l * n + k] = mulm(a[l * n + k], b[l * n + k], c->primes[l]);
}

/* (a0,a1) x (b0,b1) -> (a0 b0, a0 b1 + a1 b0, a1 b1); d = [3][nq][N]. */
void oc_tensor(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nq, uint64_t* d) {
  const size_t n = c->n, s = (size_t)nq * n;
  for (uint32_t l = 0; l < nq; ++l) {
    const uint64_t q = c->primes[l];
    for (size_t k = 0; k < n; ++k) {
      const size_t i = l * n + k;
      d[i] = mulm(a[i], b[i], q);
      d[s + i] = addm(mulm(a[i], b[s + i], q), mulm(a[s + i], b[i], q), q);
      d[2 * s + i] = mulm(a[s + i], b[s + i], q);
    }
  }
}

/* ApproxSwitchCRTBasis (OpenFHE): coefficient-form x over source primes src[0..ns)
 * -> target prime t:  sum_i [x_i (S/s_i)^{-1}]_{s_i} [S/s_i]_t  mod t. */
static void basis_convert(const oc_ctx* c, const uint64_t* const* src_limbs, const uint32_t* src_p,
                          uint32_t ns, uint32_t tp, uint64_t* out) {
  const uint32_t n = c->n;
  const uint64_t t = c->primes[tp];
  uint64_t hatinv[OC_MAXP], hat_t[OC_MAXP];
  for (uint32_t i = 0; i < ns; ++i) {
    const uint64_t qi = c->primes[src_p[i]];
    uint64_t h = 1 % qi, ht = 1 % t;
    for (uint32_t j = 0; j < ns; ++j) {
      if (j == i) continue;
      h = mulm(h, c->primes[src_p[j]] % qi, qi);
      ht = mulm(ht, c->primes[src_p[j]] % t, t);
    }
    hatinv[i] = oc_invmod(h, qi);
    hat_t[i] = ht;
  }
  for (uint32_t k = 0; k < n; ++k) {
    u128 acc = 0;
    for (uint32_t i = 0; i < ns; ++i) {
      const uint64_t qi = c->primes[src_p[i]];
      const uint64_t y = mulm(src_limbs[i][k], hatinv[i], qi);
      acc += (u128)y * hat_t[i];
    }
    out[k] = (uint64_t)(acc % t);
  }
}

/* ModUp of every digit: d (NTT form, [nq][N]) -> ext = [D][nq+K][N], NTT form. */
void oc_modup(const oc_ctx* c, const uint64_t* d, uint32_t nq, uint64_t* ext) {
  const size_t n = c->n, w = nq + c->K;
  const uint32_t D = oc_num_digits(c, nq);
  uint64_t* coef = (uint64_t*)malloc(sizeof(uint64_t) * n * nq);
  memcpy(coef, d, sizeof(uint64_t) * n * nq);
  oc_poly_ntt(c, coef, nq, 0, 1);
  for (uint32_t j = 0; j < D; ++j) {
    const uint32_t lo = j * c->alpha, hi = lo + c->alpha < nq ? lo + c->alpha : nq;
    uint64_t* e = ext + (size_t)j * w * n;
    const uint64_t* src[OC_MAXP];
    uint32_t sp[OC_MAXP];
    for (uint32_t i = lo; i < hi; ++i) { src[i - lo] = coef + (size_t)i * n; sp[i - lo] = i; }
#pragma omp parallel for schedule(dynamic, 1)
    for (int l = 0; l < (int)w; ++l) {
      uint64_t* dst = e + (size_t)l * n;
      if ((uint32_t)l >= lo && (uint32_t)l < hi) {
        memcpy(dst, d + (size_t)l * n, sizeof(uint64_t) * n);
      } else {
        const uint32_t tp = pidx(c, nq, (uint32_t)l);
        basis_convert(c, src, sp, hi - lo, tp, dst);
        ntt_limb(c, dst, tp, 0);
      }
    }
  }
  free(coef);
}

/* Key inner product: acc_t = sum_j ext_j * evk_j over nq Q limbs + K P limbs.
 * evk = [D_full][2][L+K][N]; acc = [2][nq+K][N]. */
void oc_key_inner(const oc_ctx* c, const uint64_t* ext, uint32_t nq, const uint64_t* evk, uint64_t* acc) {
  const size_t n = c->n, w = nq + c->K, lk = c->L + c->K;
  const uint32_t D = oc_num_digits(c, nq);
#pragma omp parallel for schedule(dynamic, 1)
  for (int l = 0; l < (int)w; ++l) {
    const uint32_t p = pidx(c, nq, (uint32_t)l);
    const uint64_t q = c->primes[p];
    for (size_t k = 0; k < n; ++k) {
      uint64_t s0 = 0, s1 = 0;
      for (uint32_t j = 0; j < D; ++j) {
        const uint64_t x = ext[((size_t)j * w + l) * n + k];
        const uint64_t* kb = evk + (size_t)j * 2 * lk * n;
        s0 = addm(s0, mulm(x, kb[(size_t)p * n + k], q), q);
        s1 = addm(s1, mulm(x, kb[(lk + p) * n + k], q), q);
      }
      acc[(size_t)l * n + k] = s0;
      acc[(w + l) * n + k] = s1;
    }
  }
}

/* ModDown: x over [nq+K] limbs (NTT form) -> (x_Q - Conv_{P->Q}(x_P)) P^{-1}, [nq][N]. */
void oc_moddown(const oc_ctx* c, const uint64_t* x, uint32_t nq, uint64_t* out) {
  const size_t n = c->n;
  const uint32_t K = c->K;
  uint64_t* pc = (uint64_t*)malloc(sizeof(uint64_t) * n * K);
  memcpy(pc, x + (size_t)nq * n, sizeof(uint64_t) * n * K);
#pragma omp parallel for schedule(dynamic, 1)
  for (int k = 0; k < (int)K; ++k) ntt_limb(c, pc + (size_t)k * n, c->L + k, 1);
  const uint64_t* src[OC_MAXP];
  uint32_t sp[OC_MAXP];
  for (uint32_t k = 0; k < K; ++k) { src[k] = pc + (size_t)k * n; sp[k] = c->L + k; }
#pragma omp parallel for schedule(dynamic, 1)
  for (int l = 0; l < (int)nq; ++l) {
    const uint64_t q = c->primes[l];
    uint64_t* conv = (uint64_t*)malloc(sizeof(uint64_t) * n);
    basis_convert(c, src, sp, K, (uint32_t)l, conv);
    ntt_limb(c, conv, l, 0);
    const uint64_t pinv = oc_invmod(p_mod(c, q), q);
    for (size_t k = 0; k < n; ++k) out[l * n + k] = mulm(subm(x[l * n + k], conv[k], q), pinv, q);
    free(conv);
  }
  free(pc);
}

/* HYBRID key switch of d (NTT form over nq limbs): out = [2][nq][N]. */
void oc_keyswitch(const oc_ctx* c, const uint64_t* d, uint32_t nq, const uint64_t* evk, uint64_t* out) {
  const size_t n = c->n, w = nq + c->K;
  const uint32_t D = oc_num_digits(c, nq);
  uint64_t* ext = (uint64_t*)malloc(sizeof(uint64_t) * n * w * D);
  uint64_t* acc = (uint64_t*)malloc(sizeof(uint64_t) * n * w * 2);
  oc_modup(c, d, nq, ext);
  oc_key_inner(c, ext, nq, evk, acc);
  oc_moddown(c, acc, nq, out);
  oc_moddown(c, acc + w * n, nq, out + (size_t)nq * n);
  free(ext);
  free(acc);
}

/* Relinearisation: (d0, d1, d2) -> (d0 + u0, d1 + u1), (u0, u1) = KS(d2). */
void oc_relinearize(const oc_ctx* c, const uint64_t* d, uint32_t nq, const uint64_t* rlk, uint64_t* out) {
  const size_t s = (size_t)nq * c->n;
  uint64_t* u = (uint64_t*)malloc(sizeof(uint64_t) * 2 * s);
  oc_keyswitch(c, d + 2 * s, nq, rlk, u);
  oc_add(c, d, u, nq, out);
  oc_add(c, d + s, u + s, nq, out + s);
  free(u);
}

/* Rotation by Galois element g, key switch first and automorphism second (the
 * order OpenFHE's EvalAutomorphism / EvalFastRotation use, which makes hoisted
 * rotations word-identical to plain ones): (u0, u1) = KS(c1) with a key that
 * switches s -> sigma_g^{-1}(s); out = (sigma_g(c0 + u0), sigma_g(u1)). */
void oc_rotate(const oc_ctx* c, const uint64_t* ct, uint32_t nq, uint64_t g, const uint64_t* rk, uint64_t* out) {
  const size_t s = (size_t)nq * c->n;
  uint64_t* u = (uint64_t*)malloc(sizeof(uint64_t) * 2 * s);
  oc_keyswitch(c, ct + s, nq, rk, u);
  oc_add(c, ct, u, nq, u);
  oc_automorphism_ntt(c, u, nq, g, out);
  oc_automorphism_ntt(c, u + s, nq, g, out + s);
  free(u);
}

/* Rescale (OpenFHE DropLastElementAndScale): x_i <- (x_i - [lift(x_last)]_{q_i}) q_last^{-1},
 * lift = centred representative; each of ncomp polys [nq][N] -> [nq-1][N]. */
void oc_rescale(const oc_ctx* c, const uint64_t* ct, uint32_t ncomp, uint32_t nq, uint64_t* out) {
  const size_t n = c->n;
  const uint64_t ql = c->primes[nq - 1];
  uint64_t* last = (uint64_t*)malloc(sizeof(uint64_t) * n);
  for (uint32_t comp = 0; comp < ncomp; ++comp) {
    const uint64_t* x = ct + (size_t)comp * nq * n;
    uint64_t* y = out + (size_t)comp * (nq - 1) * n;
    memcpy(last, x + (size_t)(nq - 1) * n, sizeof(uint64_t) * n);
    ntt_limb(c, last, nq - 1, 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int l = 0; l < (int)nq - 1; ++l) {
      const uint64_t q = c->primes[l];
      uint64_t* t = (uint64_t*)malloc(sizeof(uint64_t) * n);
      for (size_t k = 0; k < n; ++k) {
        const uint64_t v = last[k];
        t[k] = v > ql / 2 ? lift_signed(-(int64_t)(ql - v), q) : v % q;
      }
      ntt_limb(c, t, l, 0);
      const uint64_t inv = oc_invmod(ql % q, q);
      for (size_t k = 0; k < n; ++k) y[l * n + k] = mulm(subm(x[l * n + k], t[k], q), inv, q);
      free(t);
    }
  }
  free(last);
}
