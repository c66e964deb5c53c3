// Launchers of the RNS-CKKS device kernels (ckks_kernels.cu).
//
// Polynomials are limb-major u64[limbs][N].  A polynomial "over Q_l (+P)"
// maps limb l to prime l for l < nq and to prime p_base + (l - nq) beyond
// (p_base = L, the first special prime), described by a PrimeMap.
#pragma once
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>

#include "modarith.cuh"

namespace fhe {

struct PrimeMap {
  uint32_t nq;      // limbs [0, nq) sit on primes [0, nq)
  uint32_t p_base;  // limb nq + k sits on prime p_base + k
  __host__ __device__ uint32_t operator()(uint32_t l) const { return l < nq ? l : p_base + (l - nq); }
};

// Constant multiplier with its Shoup companion (same layout as Twiddle).
using Shoup = Twiddle;

// Fast basis conversion (OpenFHE ApproxSwitchCRTBasis) from `ns` source limbs
// to `nt` target limbs:  out_t = sum_i [x_i * hatinv_i]_{s_i} * hat_{i,t}  mod t.
struct ConvTable {
  uint32_t ns, nt;
  const uint32_t* src_prime;  // [ns]
  const uint32_t* dst_prime;  // [nt]
  const Shoup* hatinv;        // [ns]
  const Shoup* hat;           // [nt][ns]
  // Optional row maps (null: identity): source i is read from row src_row[i]
  // of its component, target t is written to row dst_row[t].
  const uint32_t* src_row = nullptr;
  const uint32_t* dst_row = nullptr;
  // Optional tensor-core operand table (conv_tc.cu): hat split into bytes in
  // the MMA's shared-memory layout, one 32 KiB tile per 16 targets.
  const uint8_t* tc_b = nullptr;
};

// ---- randomness (ChaCha20, same streams as the oracle) ----
void launch_sample_small(int kind, uint64_t seed, uint64_t stream, int64_t* out, uint32_t n,
                         cudaStream_t s);  // kind 0: ternary, 1: CBD(21)
void launch_lift_small(const int64_t* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                       const Modulus* mods, cudaStream_t s);
void launch_sample_uniform(uint64_t seed, uint64_t stream, uint64_t* out, uint32_t n, uint32_t nlimbs,
                           PrimeMap pm, const Modulus* mods, cudaStream_t s);

// ---- elementwise on [ncomp][limbs][N] with per-operand component strides (words) ----
enum class Ew { Add, Sub, Mul, Neg, MulAdd /*out += a*b*/, SubFrom /*out = b - a*/ };
void launch_ew(Ew op, const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* out,
               size_t so, uint32_t ncomp, uint32_t nlimbs, uint32_t n, PrimeMap pm,
               const Modulus* mods, cudaStream_t s);
// out[comp][l] = a[comp][l] * c_l (Shoup constant per limb, prime primes[l]) (+ b[comp][l] if b)
void launch_mul_const(const uint64_t* a, size_t sa, const Shoup* c, const uint64_t* b, size_t sb,
                      uint64_t* out, size_t so, uint32_t ncomp, uint32_t nlimbs, uint32_t n,
                      const uint64_t* primes, cudaStream_t s);
// out[comp][l] = a[comp][l] + c_l
void launch_add_const(const uint64_t* a, size_t sa, const uint64_t* c, uint64_t* out, size_t so,
                      uint32_t ncomp, uint32_t nlimbs, uint32_t n, const uint64_t* primes,
                      cudaStream_t s);
// Per-limb constants passed by value in the kernel parameters (no device
// upload, no host synchronisation); Q limbs only.
constexpr uint32_t kMaxConstLimbs = 64;
struct LimbShoup {
  Shoup v[kMaxConstLimbs];
};
struct LimbWords {
  uint64_t v[kMaxConstLimbs];
};
// out[comp][l] = a[comp][l] * c.v[l]
void launch_mul_const_v(const uint64_t* a, size_t sa, const LimbShoup& c, uint64_t* out, size_t so, uint32_t ncomp,
                        uint32_t nlimbs, uint32_t n, const uint64_t* primes, cudaStream_t s);
// out[0][l] = a[0][l] + c.v[l]; out[comp > 0] = a[comp]
void launch_add_const_v(const uint64_t* a, size_t sa, const LimbWords& c, uint64_t* out, size_t so, uint32_t ncomp,
                        uint32_t nlimbs, uint32_t n, const uint64_t* primes, cudaStream_t s);
// Weighted sum of up to kMaxWsum ciphertexts on one level (OpenFHE EvalLinearWSum):
//   out[c][l] = sum_i w[i * nq + l] * x_i[c][l]  (+ add.v[l] on component 0)  mod q_l,
// products accumulated in 128 bits and reduced once.  w = device array [m][nq].
constexpr uint32_t kMaxWsum = 32;
struct WsumArgs {
  const uint64_t* x[kMaxWsum];
  uint64_t stride[kMaxWsum];  // component stride of x_i (words)
};
void launch_linear_wsum(const WsumArgs& a, uint32_t m, const uint64_t* w, const LimbWords& add, int has_add,
                        uint64_t* out, size_t so, uint32_t ncomp, uint32_t nq, uint32_t n, const Modulus* mods,
                        cudaStream_t s);
// Tensor product of two 2-component ciphertexts into d = [3][nq] (component stride sd).
void launch_tensor(const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* d, size_t sd,
                   uint32_t nq, uint32_t n, const Modulus* mods, cudaStream_t s);

// ---- automorphism in NTT (bit-reversed evaluation) order ----
// out[l][i] = in[l][j], 2 brv(j) + 1 = (2 brv(i) + 1) g mod 2N.
void launch_automorphism(const uint64_t* in, size_t si, uint64_t* out, size_t so, uint32_t ncomp,
                         uint32_t nlimbs, uint32_t log_n, uint64_t g, cudaStream_t s);

// ---- key switching ----
// ModUp for all digits at once.  coef = INTT(d) [nq][N]; dntt = d [nq][N];
// ext = [D][w][N], w = nq + K.  Digit j's own limbs are copied from dntt, the
// others receive the basis conversion (coefficient form, NTT'd afterwards).
struct ModUpDigit {
  uint32_t lo, hi;  // own limbs [lo, hi)
  ConvTable conv;   // sources lo..hi-1, targets = all other limbs of ext (in limb order)
};
// Digits are [j*alpha, min((j+1)*alpha, nq)); at most 24 limbs each.
// primes_below_2_60: every source and target prime is below 2^60 (selects the
// split 30-bit accumulation of the conversions, which needs it).
void launch_modup(const uint64_t* coef, const uint64_t* dntt, uint64_t* ext, uint32_t nq, uint32_t K,
                  uint32_t n, const ModUpDigit* digits_dev, uint32_t D, uint32_t alpha, const Modulus* mods,
                  cudaStream_t s, bool primes_below_2_60);
// acc[2][w][N] = sum_j ext[j] * evk[j][0/1][key limb]; key limb of ext limb l is pm(l).
// Only the limbs [l0, l0 + count) when given (the rest of acc is left alone).
void launch_key_inner(const uint64_t* ext, uint32_t D, uint32_t w, const uint64_t* evk,
                      uint32_t key_limbs, PrimeMap pm, uint64_t* acc, uint32_t n, const Modulus* mods,
                      cudaStream_t s, uint32_t l0 = 0, uint32_t count = ~0u);
// Basis conversion of ncomp polys: src limbs (coefficient form) -> dst (coefficient form).
// ns / nt must equal the table's source / target counts (ns <= 24).
// Slot vectors of replicated-BSGS diagonals t0..t0+nb-1 into dv [nb][slots]
// (real parts; see Ckks::encode_replicated_diagonals).
void launch_replicated_diagonals(double2* dv, const double* w, uint32_t m, uint32_t cols, uint32_t R, uint32_t T,
                                 uint32_t win, uint32_t baby, uint32_t slots, uint32_t t0, uint32_t nb,
                                 cudaStream_t s);

// ---- basis conversion on the tensor cores (conv_tc.cu), same results ----
// Whether the tensor-core conversion handles ns source limbs at ring n.
bool tc_conversion_supported(uint32_t n, uint32_t ns, bool primes_below_2_60);
// Operand table for ConvTable::tc_b from hat[nt][ns].
std::vector<uint8_t> tc_conversion_table(const Shoup* hat, uint32_t ns, uint32_t nt);
void launch_convert_tc(const uint64_t* src, size_t s_comp, uint64_t* dst, size_t d_comp, uint32_t ncomp,
                       const ConvTable* t_dev, uint32_t nt, uint32_t n, const Modulus* mods, cudaStream_t s);
void launch_modup_tc(const uint64_t* coef, const uint64_t* dntt, uint64_t* ext, uint32_t nq, uint32_t K,
                     uint32_t n, const ModUpDigit* digits_dev, uint32_t D, uint32_t alpha, const Modulus* mods,
                     cudaStream_t s);
// Waits for an MMA that ran out of their iteration limit (0 when healthy).
unsigned tc_conversion_timeouts();

void launch_convert(const uint64_t* src, size_t s_comp, uint64_t* dst, size_t d_comp, uint32_t ncomp,
                    const ConvTable* t_dev, uint32_t ns, uint32_t nt, uint32_t n, const Modulus* mods,
                    cudaStream_t s, bool primes_below_2_60);
// out[c][i] = (x[c][i] - conv[c][i]) * pinv_i  (+ add[i] on component 0 when add != null).
void launch_moddown_combine(const uint64_t* x, size_t sx, const uint64_t* conv, size_t sc,
                            const Shoup* pinv, const uint64_t* add, uint64_t* out, size_t so,
                            uint32_t ncomp, uint32_t nq, uint32_t n, const uint64_t* primes,
                            cudaStream_t s);
// Rescale lift: lifted[c][i] = centred(last[c]) mod q_i for i < nlimbs.
void launch_rescale_lift(const uint64_t* last, size_t sl, uint64_t* lifted, size_t sd, uint32_t ncomp,
                         uint32_t nlimbs, uint32_t n, uint64_t q_last, const Modulus* mods,
                         cudaStream_t s);

// ---- encode / decode ----
void launch_fft_special_inv(double2* v, const double2* tw, uint32_t slots, uint32_t batch,
                            cudaStream_t s);
void launch_fft_special_fwd(double2* v, const double2* tw, uint32_t slots, uint32_t batch,
                            cudaStream_t s);
// Bit-reverse, divide by slots, scale, round half away from zero, place at
// coefficient i*gap (real) and i*gap + N/2 (imag) of coef (zeroed elsewhere).
// Coefficients are integer-valued doubles (exact above 2^53 too).
// status bit 0: a coefficient was not finite or reached 2^126.
void launch_encode_round(const double2* v, double* coef, uint32_t slots, uint32_t n, double scale,
                         unsigned* status, cudaStream_t s);
// out[l][k] = src[k] mod q_l for integer-valued doubles |src| < 2^126 (exact).
void launch_lift_double(const double* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                        const Modulus* mods, uint32_t batch, cudaStream_t s);
// Centred CRT of limbs 0 and 1 (or limb 0 alone) of an INTT'd plaintext at the
// slot positions, divided by scale -> complex values in bit-reversed order,
// ready for the forward special FFT.  m1 = Barrett constants of q1.
void launch_decode_crt(const uint64_t* coef, uint32_t nlimbs, uint32_t slots, uint32_t n, double scale,
                       uint64_t q0, uint64_t q1, uint64_t q0inv_mod_q1, uint64_t q0inv_shoup,
                       Modulus m1, double2* v, cudaStream_t s);

// ---- batched encode ----
// Batch versions over B vectors: v = [B][slots] double2, coef = [B][N] int64,
// out = [B][nlimbs][N] u64.
void launch_encode_round_batch(const double2* v, double* coef, uint32_t slots, uint32_t n, double scale,
                               uint32_t batch, unsigned* status, cudaStream_t s);
void launch_lift_small_batch(const int64_t* src, uint64_t* out, uint32_t n, uint32_t nlimbs, PrimeMap pm,
                             const Modulus* mods, uint32_t batch, cudaStream_t s);

// out = a * X^{N/2} in NTT form: the evaluation at psi^{2 brv(i) + 1} is scaled
// by i_q = psi^{N/2} when brv(i) is even (i < N/2) and by -i_q otherwise.
// tw = forward twiddle tables (entry 1 of prime l's table is psi_l^{N/2}).
void launch_mul_monomial_half(const uint64_t* a, size_t sa, uint64_t* out, size_t so, uint32_t ncomp,
                              uint32_t nlimbs, uint32_t n, const Twiddle* tw, const uint64_t* primes,
                              cudaStream_t s);

// ---- BSGS inner products ----
// For every giant g < G and component c < 2:
//   out[g][c][l] = sum_{j < b} baby_j[c][l] * diag_{g*b+j}[l]   (mod q_l),
// babies[j] = [2][nq][N] (component stride nq*N), diags[g*b+j] = [nq_d >= nq][N]
// or null for an all-zero diagonal.  Products accumulate in 128 bits and are
// reduced once per output word.  b <= 32.
void launch_bsgs_dot(const uint64_t* const* babies, const uint64_t* const* diags, uint64_t* out, uint32_t b,
                     uint32_t G, uint32_t nq, uint32_t n, const Modulus* mods, cudaStream_t s);

}  // namespace fhe
