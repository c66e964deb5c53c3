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

#ifdef __cplusplus
}
#endif
#endif
