/* Internal helpers shared by the oracle's C files (test infrastructure). */
#ifndef ORACLE_INTERNAL_H
#define ORACLE_INTERNAL_H
#include <stdint.h>

typedef unsigned __int128 u128;

typedef struct {
  uint64_t* w;   /* w[i] = root^{bitrev(i)} */
  uint64_t* wp;  /* Shoup companion floor(w * 2^64 / q) */
} twiddles_t;

static inline uint64_t oi_mul_shoup(uint64_t x, uint64_t w, uint64_t wp, uint64_t q) {
  uint64_t hi = (uint64_t)(((u128)x * wp) >> 64);
  uint64_t r = x * w - hi * q;
  return r >= q ? r - q : r;
}

static inline uint64_t oi_shoup(uint64_t w, uint64_t q) { return (uint64_t)(((u128)w << 64) / q); }

uint32_t oi_bitrev(uint32_t x, uint32_t bits);
twiddles_t oi_make_table(uint32_t log_n, uint64_t q, uint64_t root);
void oi_free_table(twiddles_t* t);
void oi_ntt_fwd_table(uint64_t* a, uint32_t log_n, uint64_t q, const twiddles_t* t);
void oi_ntt_inv_table(uint64_t* a, uint32_t log_n, uint64_t q, const twiddles_t* t);
#endif
