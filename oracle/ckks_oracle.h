/*
 * CPU oracle for the RNS-CKKS evaluation path — TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker that the CUDA product (fhe_mamba_b200/csrc) is
 * compared against.  It is imported only by tests/, by __graft_entry__.smoke()
 * and by bench.py's CPU-baseline leg.  Product code never links or calls it.
 *
 * It restates, in plain C with exact 128-bit integer arithmetic, the public
 * algorithms the reference evaluates through OpenFHE v1.4.2
 * (aa391988d354d4360f390f223a90e0d1b98839d7) and FIDESlib
 * (cd171f20f510eeca04c71d7b0034ef073829f761).  Neither library is vendored in
 * the reference; the reference's own call sites are cited per function.
 *
 * Parity status: the CKKS prime chain generator is pinned against the chain
 * the reference recorded from OpenFHE (N=2^17, depth 44, scale 59, first 60,
 * dnum 4: 45 Q + 12 P primes).  NTT outputs are fixed by (q, psi, ordering),
 * so they are pinned through the pinned primes and OpenFHE's minimal-root
 * convention.  Key-dependent words (key switching, relinearisation, rotation)
 * cannot be pinned to OpenFHE here: its PRNG is not available, so those words
 * are pinned GPU == this oracle on identical seeded keys.
 */
#ifndef CKKS_ORACLE_H
#define CKKS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar modular arithmetic (exact, unsigned __int128) ---- */
uint64_t oc_mulmod(uint64_t a, uint64_t b, uint64_t q);
uint64_t oc_powmod(uint64_t a, uint64_t e, uint64_t q);
uint64_t oc_invmod(uint64_t a, uint64_t q);
int oc_is_prime(uint64_t n);

/* ---- prime generation (OpenFHE nbtheory FirstPrime/PreviousPrime/NextPrime) ---- */
uint64_t oc_first_prime(uint32_t bits, uint64_t m);
uint64_t oc_previous_prime(uint64_t q, uint64_t m);
uint64_t oc_next_prime(uint64_t q, uint64_t m);
/* CKKS FLEXIBLEAUTO Q chain + HYBRID P primes.  num_q = depth + 1.
 * Returns the number of P primes, or a negative value on error. */
int oc_ckks_moduli(uint32_t log_n, uint32_t num_q, uint32_t scale_bits,
                   uint32_t first_bits, uint32_t dnum, uint64_t* q_out,
                   uint64_t* p_out, uint32_t max_p);
/* The k largest primes q < 2^bits with q = 1 mod 2N (NTT microbench chain). */
void oc_ntt_primes(uint32_t log_n, uint32_t bits, uint32_t k, uint64_t* out);
/* Minimal primitive m-th root of unity mod q (OpenFHE RootOfUnity). */
uint64_t oc_root_of_unity(uint64_t m, uint64_t q);

/* ---- negacyclic NTT, OpenFHE order (bit-reversed evaluation order) ---- */
void oc_ntt_forward(uint64_t* a, uint32_t log_n, uint64_t q, uint64_t psi);
void oc_ntt_inverse(uint64_t* a, uint32_t log_n, uint64_t q, uint64_t psi);
/* data = u64[n_polys][n_limbs][N]; limb l uses (q[l], psi[l]). */
void oc_ntt_batch(uint64_t* data, uint32_t n_polys, uint32_t n_limbs,
                  uint32_t log_n, const uint64_t* q, const uint64_t* psi,
                  int inverse, int threads);

/* ---- counter-based randomness shared with the product's sampler ---- */
uint64_t oc_rand_u64(uint64_t seed, uint64_t stream, uint64_t index);

/* ---- RNS-CKKS (ckks_oracle_ckks.c) ---- */

/* Randomness streams (64-bit ChaCha20 nonces); the product samples the same. */
#define OC_STREAM_SECRET (1ull << 56)
#define OC_STREAM_PK_A (2ull << 56)
#define OC_STREAM_PK_E (3ull << 56)
#define OC_STREAM_ENC_V(nonce) ((4ull << 56) | ((nonce) & 0xFFFFFFFFFFFFFFull))
#define OC_STREAM_ENC_E0(nonce) ((5ull << 56) | ((nonce) & 0xFFFFFFFFFFFFFFull))
#define OC_STREAM_ENC_E1(nonce) ((6ull << 56) | ((nonce) & 0xFFFFFFFFFFFFFFull))
#define OC_STREAM_KEY_A(id, digit) ((0x10ull << 56) | (((uint64_t)(id) & 0xFFFFFFFFFFull) << 8) | (digit))
#define OC_STREAM_KEY_E(id, digit) ((0x11ull << 56) | (((uint64_t)(id) & 0xFFFFFFFFFFull) << 8) | (digit))

typedef struct oc_ctx oc_ctx;

/* primes = L Q primes followed by K P primes. */
oc_ctx* oc_ctx_new(uint32_t log_n, uint32_t L, uint32_t K, const uint64_t* primes, uint32_t dnum,
                   uint32_t slots);
void oc_ctx_free(oc_ctx* c);
uint64_t oc_ctx_psi(const oc_ctx* c, uint32_t i);
uint32_t oc_num_digits(const oc_ctx* c, uint32_t nq);
void oc_poly_ntt(const oc_ctx* c, uint64_t* a, uint32_t nq, uint32_t np, int inverse);

int64_t oc_sample_ternary_coef(uint64_t seed, uint64_t stream, uint64_t k);
int64_t oc_sample_error_coef(uint64_t seed, uint64_t stream, uint64_t k);
uint64_t oc_sample_uniform_coef(uint64_t seed, uint64_t stream, uint32_t prime, uint32_t n,
                                uint64_t k, uint64_t q);
void oc_sample_small(const oc_ctx* c, uint64_t seed, uint64_t stream, int kind, int64_t* out);
void oc_lift_small(const oc_ctx* c, const int64_t* s, uint64_t* out, uint32_t nq, uint32_t np, int ntt);
void oc_sample_uniform_poly(const oc_ctx* c, uint64_t seed, uint64_t stream, uint64_t* out,
                            uint32_t nq, uint32_t np);

void oc_keygen_secret(const oc_ctx* c, uint64_t seed, int64_t* s_coef, uint64_t* s_ntt);
void oc_keygen_public(const oc_ctx* c, uint64_t seed, const uint64_t* s_ntt, uint64_t* pk);
void oc_keygen_switch(const oc_ctx* c, uint64_t seed, uint64_t key_id, const uint64_t* s_ntt,
                      const uint64_t* sp_ntt, uint64_t* evk);

void oc_automorphism_ntt(const oc_ctx* c, const uint64_t* in, uint32_t nlimbs, uint64_t g, uint64_t* out);
void oc_automorphism_coef(const oc_ctx* c, const int64_t* in, uint64_t g, int64_t* out);
uint64_t oc_rotation_galois(const oc_ctx* c, int64_t r);

int oc_encode(const oc_ctx* c, const double* re, const double* im, uint32_t count, double scale,
              uint32_t nq, uint64_t* out);
void oc_decode(const oc_ctx* c, const uint64_t* pt, uint32_t nq, double scale, double* re, double* im);

void oc_encrypt_pk(const oc_ctx* c, uint64_t seed, uint64_t nonce, const uint64_t* pk, const uint64_t* pt,
                   uint32_t nq, uint64_t* ct);
void oc_decrypt(const oc_ctx* c, const uint64_t* s_ntt, const uint64_t* ct, uint32_t ncomp, uint32_t nq,
                uint64_t* pt);

void oc_add(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nlimbs, uint64_t* out);
void oc_sub(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nlimbs, uint64_t* out);
void oc_mul_pointwise(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nlimbs, uint64_t* out);
void oc_tensor(const oc_ctx* c, const uint64_t* a, const uint64_t* b, uint32_t nq, uint64_t* d);
void oc_modup(const oc_ctx* c, const uint64_t* d, uint32_t nq, uint64_t* ext);
void oc_key_inner(const oc_ctx* c, const uint64_t* ext, uint32_t nq, const uint64_t* evk, uint64_t* acc);
void oc_moddown(const oc_ctx* c, const uint64_t* x, uint32_t nq, uint64_t* out);
void oc_keyswitch(const oc_ctx* c, const uint64_t* d, uint32_t nq, const uint64_t* evk, uint64_t* out);
void oc_relinearize(const oc_ctx* c, const uint64_t* d, uint32_t nq, const uint64_t* rlk, uint64_t* out);
void oc_rotate(const oc_ctx* c, const uint64_t* ct, uint32_t nq, uint64_t g, const uint64_t* rk, uint64_t* out);
void oc_rescale(const oc_ctx* c, const uint64_t* ct, uint32_t ncomp, uint32_t nq, uint64_t* out);

#ifdef __cplusplus
}
#endif
#endif
