/*
 * fhe_b200 — C ABI of the B200-native RNS-CKKS evaluation backend.
 *
 * This is the drop-in boundary for the reference's native FIDESlib/OpenFHE
 * stage (fhe-mamba: native/fideslib_stage0).  Every entry point:
 *   - returns int status: FHE_OK (0) or a negative FHE_ERR_* code; the message
 *     of the last failure on the calling thread is read with fhe_last_error();
 *   - never throws across the ABI;
 *   - takes plain pointers and sizes (no C++ or torch types);
 *   - is single-threaded per context: one context owns one CUDA stream on one
 *     device, and all device work of the context is ordered on that stream.
 * Handles are opaque, owned by the caller and freed explicitly.
 *
 * Residue layout (device and host buffers alike): limb-major
 * u64[n_polys][n_limbs][N], each limb a full length-N residue polynomial.
 */
#ifndef FHE_B200_H
#define FHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FHE_OK 0
#define FHE_ERR_INVALID (-1)   /* bad argument, shape or handle */
#define FHE_ERR_CUDA (-2)      /* CUDA runtime or kernel launch failure */
#define FHE_ERR_ALLOC (-3)     /* device or host allocation failure */
#define FHE_ERR_STATE (-4)     /* missing key, level underflow, scale mismatch */
#define FHE_ERR_INTERNAL (-5)  /* unexpected exception */

#define FHE_MEM_HOST 0         /* pointer is host memory (pageable or pinned) */
#define FHE_MEM_DEVICE 1       /* pointer is device memory of the context's GPU */

typedef struct fhe_ctx fhe_ctx;

/* CKKS context parameters.  Mirrors the reference's CCParams calls
 * (native/fideslib_stage0/src/packed_fideslib.cpp:1060-1068:
 *  SetRingDim, SetMultiplicativeDepth, SetScalingModSize, SetFirstModSize,
 *  SetScalingTechnique(FLEXIBLEAUTO), SetKeySwitchTechnique(HYBRID),
 *  SetNumLargeDigits, SetBatchSize, SetSecretKeyDist(UNIFORM_TERNARY)). */
typedef struct fhe_params {
  uint32_t log_n;             /* ring dimension N = 2^log_n, 10 <= log_n <= 17 */
  uint32_t mult_depth;        /* number of Q primes = mult_depth + 1 */
  uint32_t scaling_mod_size;  /* bits of the scaling primes */
  uint32_t first_mod_size;    /* bits of q_0 (must differ from scaling_mod_size) */
  uint32_t num_large_digits;  /* dnum of HYBRID key switching */
  uint32_t batch_size;        /* slots (<= N/2, power of two) */
  int32_t device;             /* CUDA device ordinal */
  uint32_t reserved;
} fhe_params;

/* --- context ------------------------------------------------------------ */

/* Replaces GenCryptoContext(CCParams) + LoadContext (packed_fideslib.cpp:1068,1090):
 * generates the FLEXIBLEAUTO Q chain and HYBRID P primes the way OpenFHE
 * v1.4.2 does, their minimal primitive 2N-th roots, and uploads all NTT,
 * basis-conversion and rescale tables to the device. */
int fhe_ctx_create(const fhe_params* params, fhe_ctx** out);

/* NTT-only context on an explicit prime list (q_i = 1 mod 2N, q_i < 2^62);
 * replaces the FIDESlib Context the NTT probe builds
 * (experiments/ntt_warp_tail/probe.cu:93-104) for raw limb transforms. */
int fhe_ctx_create_ntt(uint32_t log_n, const uint64_t* primes, uint32_t n_primes,
                       int32_t device, fhe_ctx** out);

int fhe_ctx_destroy(fhe_ctx* ctx);

/* Copies the Q primes (n_q written) and P primes (n_p written); either array
 * may be NULL to query only the counts.  Replaces the probe's
 * gpu->prime[i].p / gpu->specialPrime[i].p reads (probe.cu:124-140). */
int fhe_ctx_moduli(const fhe_ctx* ctx, uint64_t* q, uint32_t* n_q, uint64_t* p, uint32_t* n_p);

/* Host-only parameter generation (no device work).  Writes the FLEXIBLEAUTO Q
 * chain (mult_depth + 1 primes) and the HYBRID P primes that fhe_ctx_create
 * would use; q/p may be NULL to query counts (q needs >= mult_depth + 1 slots,
 * p >= 64).  Same rule as OpenFHE v1.4.2 ParamsGenCKKSRNS, as the reference's
 * context set-up invokes it (packed_fideslib.cpp:1060-1068). */
int fhe_gen_ckks_moduli(uint32_t log_n, uint32_t mult_depth, uint32_t scaling_mod_size,
                        uint32_t first_mod_size, uint32_t num_large_digits,
                        uint64_t* q, uint32_t* n_q, uint64_t* p, uint32_t* n_p);

/* Host-only: the `count` largest primes q < 2^bits with q = 1 mod 2N, in
 * descending order (the NTT microbench prime set of BASELINE config 2). */
int fhe_gen_ntt_primes(uint32_t log_n, uint32_t bits, uint32_t count, uint64_t* out);

/* Minimal primitive 2N-th roots of unity, one per prime (Q then P). */
int fhe_ctx_roots(const fhe_ctx* ctx, uint64_t* roots, uint32_t n);

/* The context's cudaStream_t (as void*), for callers that time or order work. */
int fhe_ctx_stream(const fhe_ctx* ctx, void** stream);

/* Blocks until all work queued on the context's stream has finished. */
int fhe_ctx_synchronize(fhe_ctx* ctx);

/* Copies the calling thread's last error message (NUL-terminated). */
int fhe_last_error(char* buf, size_t len);

/* --- raw limb transforms (BASELINE config 2 microbench) ------------------ */

/* Forward negacyclic NTT, OpenFHE order (natural coefficients in, bit-reversed
 * evaluations out, minimal psi), in place on u64[n_polys][n_limbs][N]; limb l
 * uses prime limb0 + l.  Inputs must be reduced (< q).  mem = FHE_MEM_HOST
 * copies the buffer to the device and back inside the call.  Replaces FIDESlib
 * NTT_<*, ALGO_SHOUP, NTT_NONE> launched as in probe.cu:57-64 and
 * RNSPoly::NTT (src/fideslib_plaintext_encoder.cpp:264,410). */
int fhe_ntt(fhe_ctx* ctx, uint64_t* data, uint32_t n_polys, uint32_t limb0,
            uint32_t n_limbs, int mem);

/* Inverse of fhe_ntt (bit-reversed evaluations in, coefficients out, 1/N
 * applied).  Replaces FIDESlib INTT_ / RNSPoly::INTT. */
int fhe_intt(fhe_ctx* ctx, uint64_t* data, uint32_t n_polys, uint32_t limb0,
             uint32_t n_limbs, int mem);

/* --- CKKS evaluation (the API packed_fideslib.cpp:117-281 drives) --------- */

typedef struct fhe_ct fhe_ct; /* device ciphertext: 2 or 3 components over n_limbs Q limbs */
typedef struct fhe_pt fhe_pt; /* device plaintext, NTT form over n_limbs Q limbs */

typedef struct fhe_ctx_info_t {
  uint32_t log_n, n_q, n_p, dnum, alpha, slots, ckks, reserved;
} fhe_ctx_info_t;

int fhe_ctx_info(const fhe_ctx* ctx, fhe_ctx_info_t* info);

/* FLEXIBLEAUTO scaling factor of a fresh ciphertext with n_limbs Q limbs
 * (OpenFHE GetScalingFactorReal(level), level = n_q - n_limbs). */
int fhe_level_scale(fhe_ctx* ctx, uint32_t n_limbs, double* scale);

/* KeyGen + EvalMultKeyGen (packed_fideslib.cpp:1078): ternary secret, public
 * key, HYBRID relinearisation key, all sampled on the device from ChaCha20
 * streams keyed by `seed`. */
int fhe_keygen(fhe_ctx* ctx, uint64_t seed);

/* Galois element 5^step mod 2N of a slot rotation (FindAutomorphismIndex2n). */
int fhe_galois_element(fhe_ctx* ctx, int32_t step, uint64_t* g);

/* EvalRotateKeyGen(secretKey, steps) (packed_fideslib.cpp:1079-1083). */
int fhe_rotation_keygen(fhe_ctx* ctx, const int32_t* steps, uint32_t n);

/* Key for EvalConjugate (conjugate API patch, patches/fideslib-v2.1.0-*conjugate*). */
int fhe_conjugation_keygen(fhe_ctx* ctx);

/* Copies a key to host memory: kind 0 secret s (NTT form, [n_q+n_p][N]),
 * 1 public key ([2][n_q][N]), 2 relinearisation key, 3 rotation key of
 * Galois element `galois` ([digits][2][n_q+n_p][N]); after a bootstrap setup
 * with sparse_h > 0: 4 the sparse secret s' (NTT form), 5 the switching key
 * s -> s', 6 the key s' -> s.  `words` must equal the key's size.  For parity
 * tests against an independent implementation. */
int fhe_key_download(fhe_ctx* ctx, int kind, uint64_t galois, uint64_t* host, size_t words);

/* MakeCKKSPackedPlaintext (packed_fideslib.cpp:163-179): special inverse FFT,
 * scale, round half away from zero, RNS lift and NTT, all on the device.
 * n_limbs = 0 means all Q limbs; scale <= 0 means the FLEXIBLEAUTO factor. */
int fhe_encode(fhe_ctx* ctx, const double* re, const double* im, uint32_t count, uint32_t n_limbs,
               double scale, fhe_pt** out);
/* Decode (CKKSPackedEncoding::Decode): count <= slots values. */
int fhe_decode(fhe_ctx* ctx, const fhe_pt* pt, double* re, double* im, uint32_t count);
/* Encrypt(publicKey, pt) (packed_fideslib.cpp:185-189). */
int fhe_encrypt(fhe_ctx* ctx, const fhe_pt* pt, fhe_ct** out);
/* Decrypt(secretKey, ct) (client side, packed_fideslib.cpp:1195-1210). */
int fhe_decrypt(fhe_ctx* ctx, const fhe_ct* ct, fhe_pt** out);

int fhe_ct_free(fhe_ct* ct);
int fhe_pt_free(fhe_pt* pt);
/* GetLevel/GetNoiseScaleDeg/GetScalingFactor of a ciphertext. */
int fhe_ct_info(const fhe_ct* ct, uint32_t* ncomp, uint32_t* n_limbs, uint32_t* noise_deg, double* scale);
int fhe_pt_info(const fhe_pt* pt, uint32_t* n_limbs, double* scale);
/* Raw residues, layout [ncomp][n_limbs][N] (host). */
int fhe_ct_download(fhe_ctx* ctx, const fhe_ct* ct, uint64_t* host);
int fhe_ct_upload(fhe_ctx* ctx, const uint64_t* host, uint32_t ncomp, uint32_t n_limbs, uint32_t noise_deg,
                  double scale, fhe_ct** out);
int fhe_pt_download(fhe_ctx* ctx, const fhe_pt* pt, uint64_t* host);
int fhe_pt_upload(fhe_ctx* ctx, const uint64_t* host, uint32_t n_limbs, double scale, fhe_pt** out);
/* Ciphertext::Clone. */
int fhe_ct_clone(fhe_ctx* ctx, const fhe_ct* ct, fhe_ct** out);

/* EvalAdd / EvalSub (FLEXIBLEAUTO level and scale alignment). */
int fhe_add(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
int fhe_sub(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
int fhe_negate(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out);
/* EvalAdd(ct, pt) / EvalSub(ct, pt) / EvalMult(ct, pt) (packed_fideslib.cpp:155-200). */
int fhe_add_plain(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* p, fhe_ct** out);
int fhe_sub_plain(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* p, fhe_ct** out);
int fhe_mul_plain(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* p, fhe_ct** out);
/* EvalAdd(ct, double) / EvalMult(ct, double). */
int fhe_add_scalar(fhe_ctx* ctx, const fhe_ct* a, double v, fhe_ct** out);
int fhe_mul_scalar(fhe_ctx* ctx, const fhe_ct* a, double v, fhe_ct** out);
/* Exact integer multiple (multIntScalar, src/fideslib_refresh_correction.hpp:16-43). */
int fhe_mul_int(fhe_ctx* ctx, const fhe_ct* a, int64_t v, fhe_ct** out);
/* EvalMult without relinearisation (3-component result). */
int fhe_tensor(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
/* Relinearize (HYBRID key switch of the third component). */
int fhe_relinearize(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out);
/* EvalMult(ct, ct) (packed_fideslib.cpp:128-154): rescale degree-2 inputs,
 * align levels, tensor, relinearise. */
int fhe_mul(fhe_ctx* ctx, const fhe_ct* a, const fhe_ct* b, fhe_ct** out);
/* RescaleInPlace (packed_fideslib.cpp:236) — OpenFHE DropLastElementAndScale. */
int fhe_rescale(fhe_ctx* ctx, fhe_ct* ct);
/* LevelReduceInPlace: drop limbs without scaling. */
int fhe_level_reduce(fhe_ctx* ctx, fhe_ct* ct, uint32_t levels);
/* EvalRotate(ct, step) (packed_fideslib.cpp:207-221): key switch, then automorphism. */
int fhe_rotate(fhe_ctx* ctx, const fhe_ct* a, int32_t step, fhe_ct** out);
/* EvalConjugate. */
int fhe_conjugate(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out);
/* EvalFastRotationPrecompute + EvalFastRotation (src/fideslib_rotation_batch.hpp:8-23):
 * one ModUp shared by n rotations; outs receives n new handles. */
int fhe_rotate_hoisted(fhe_ctx* ctx, const fhe_ct* a, const int32_t* steps, uint32_t n, fhe_ct** outs);

/* Batched MakeCKKSPackedPlaintext: encodes `batch` vectors of `count` values
 * (re[b*count + i], im likewise or NULL) on the device in one pass; outs
 * receives `batch` handles.  The device-side replacement of the reference's
 * per-diagonal host encoding (src/fideslib_plaintext_encoder.cpp:264-410). */
int fhe_encode_batch(fhe_ctx* ctx, const double* re, const double* im, uint32_t batch, uint32_t count,
                     uint32_t n_limbs, double scale, fhe_pt** outs);
/* Diagonal plaintexts of the replicated BSGS layout of y = W x generated on
 * the device from the weights (the device-side diagonal generation of the
 * reference's GPU special FFT + RNS encoder, src/gpu_special_fft.cu:12-113 and
 * src/fideslib_plaintext_rns.cu:119-139, for this layout): w_dev is W, m x
 * cols, row-major fp64 in device memory; diagonal t < T holds
 * W[i][(i + r*T + t) % cols] at slot r*win + i (r < R, i < m), rotated by
 * (t / baby) * baby slots; outs[t] receives its plaintext over n_limbs limbs
 * at `scale` (0: the level's scale).  The words equal fhe_encode_batch of the
 * same vectors built on the host. */
int fhe_encode_replicated_diagonals(fhe_ctx* ctx, const double* w_dev, uint32_t m, uint32_t cols, uint32_t R,
                                    uint32_t T, uint32_t win, uint32_t baby, uint32_t n_limbs, double scale,
                                    fhe_pt** outs);

/* BSGS plaintext-ciphertext matrix-vector product (PackedEvaluator::linear,
 * packed_fideslib.cpp:447-532; LinearTransformInPlace of the reference's
 * FIDESlib patch):
 *   out = sum_g rot( sum_j diags[g*baby+j] (.) rot(a, j*stride), (g*baby - giant_offset)*stride ).
 * Baby rotations share one ModUp; one fused kernel forms every giant's inner
 * sum; diags[i] may be NULL for an all-zero diagonal.  Needs rotation keys
 * for steps j*stride and the non-zero giant amounts (stride 1, offset 0 is
 * the plain matvec). */
int fhe_linear_transform(fhe_ctx* ctx, const fhe_ct* a, const fhe_pt* const* diags, uint32_t baby,
                         uint32_t giant, int32_t stride, int32_t giant_offset, fhe_ct** out);

/* --- limb-sharded key switching (one process per GPU) ----------------------
 * The multi-GPU mode of the north star: RNS limbs dealt out round-robin, rank
 * r of W owning Q limbs l % W == r and P limbs p % W == r, so every
 * limb-local operation (NTT, products, rescale epilogue, automorphism) needs
 * no communication and a HYBRID key switch (FIDESlib's KeySwitch behind
 * EvalMult / EvalRotate, packed_fideslib.cpp:149,215-217) needs exactly two
 * all-gathers, which the caller runs on the context stream (fhe_ctx_stream)
 * with its own collective library:
 *   fhe_shard_modup_prepare  -> all-gather send [q_chunk][N] into [W][q_chunk][N]
 *   fhe_shard_inner          -> all-gather p_send [2][p_chunk][N] into [W][2][p_chunk][N]
 *   fhe_shard_moddown        -> out [2][q_own][N] (+ add0 / add1 per component)
 * Buffers are device pointers on the context's device, rows of N words, own
 * rows in increasing limb order.  Results equal the single-GPU key switch
 * word for word.  Keys are generated whole on every rank and their own rows
 * copied out by fhe_shard_load_key. */
typedef struct fhe_shard_plan {
  uint32_t n_limbs;  /* live Q limbs */
  uint32_t q_own;    /* own Q limbs: l = rank + i*world */
  uint32_t q_chunk;  /* rows per rank in the first all-gather (ceil(n_limbs / world)) */
  uint32_t p_own;    /* own P limbs */
  uint32_t p_chunk;  /* rows per rank and component in the second all-gather */
  uint32_t rows;     /* own extended rows: q_own + p_own (acc is [2][rows][N]) */
  uint32_t digits;   /* HYBRID digits at this level */
  uint32_t reserved;
} fhe_shard_plan;
int fhe_shard_init(fhe_ctx* ctx, uint32_t rank, uint32_t world);
int fhe_shard_plan_get(fhe_ctx* ctx, uint32_t n_limbs, fhe_shard_plan* out);
/* kind 2: relinearisation key; 3: rotation key of Galois element `galois`. */
int fhe_shard_load_key(fhe_ctx* ctx, int32_t kind, uint64_t galois);
int fhe_shard_modup_prepare(fhe_ctx* ctx, uint32_t n_limbs, const uint64_t* d_own, uint64_t* send);
int fhe_shard_inner(fhe_ctx* ctx, uint32_t n_limbs, int32_t kind, uint64_t galois, const uint64_t* gathered,
                    const uint64_t* d_own, uint64_t* acc, uint64_t* p_send);
/* fhe_shard_inner with the first exchange split by HYBRID digit, so that
 * digit j + 1's all-gather overlaps digit j's conversion: for every digit j,
 * rank r sends its own rows of digit j (send rows of limbs in
 * [j*alpha, min((j+1)*alpha, n_limbs)), in limb order) padded with zero rows
 * to dchunk = ceil(alpha / world) rows, the caller all-gathers them into
 * gathered_digit [W][dchunk][N] and calls fhe_shard_inner_digit; then
 * fhe_shard_inner_tail (NTT, key inner product, own P rows into p_send). */
int fhe_shard_inner_digit(fhe_ctx* ctx, uint32_t n_limbs, uint32_t digit, const uint64_t* gathered_digit,
                          const uint64_t* d_own);
int fhe_shard_inner_tail(fhe_ctx* ctx, uint32_t n_limbs, int32_t kind, uint64_t galois, uint64_t* acc,
                         uint64_t* p_send);
int fhe_shard_moddown(fhe_ctx* ctx, uint32_t n_limbs, const uint64_t* acc, const uint64_t* p_gathered,
                      const uint64_t* add0, const uint64_t* add1, uint64_t* out);
/* Slot permutation of both components of the own rows ([2][q_own][N]). */
int fhe_shard_automorphism(fhe_ctx* ctx, uint32_t n_limbs, uint64_t galois, const uint64_t* in, uint64_t* out);

/* --- files for a process-separated client and server ----------------------
 * The reference's handoff (src/fideslib_handoff.cpp:27-85: serialize_ciphertext,
 * deserialize_ciphertext, serialize_context): the client saves its evaluation
 * keys and encrypted inputs, the server loads them into a context created with
 * the same parameters, evaluates, and saves the result for the client.  Files
 * carry a parameter fingerprint and a checksum; loading into a context with
 * other parameters fails.  A key bundle saved without the secret makes an
 * evaluation-only context: it evaluates and encrypts, but decryption and key
 * generation fail with FHE_ERR_STATE.  Sparse-secret bootstrapping keys are not
 * saved. */
int fhe_ct_save(fhe_ctx* ctx, const fhe_ct* ct, const char* path);
int fhe_ct_load(fhe_ctx* ctx, const char* path, fhe_ct** out);
/* Public, relinearisation and every rotation key (and the secret when
 * include_secret != 0). */
int fhe_keys_save(fhe_ctx* ctx, const char* path, int32_t include_secret);
int fhe_keys_load(fhe_ctx* ctx, const char* path);

/* Integer-pipe ceiling of the NTT: butterflies per second of the forward
 * transform's lazy Shoup butterfly (same arithmetic and reduction schedule)
 * run on registers only, all SMs, on the context's device and stream.  The
 * roofline that bounds the NTT on this GPU besides HBM bandwidth. */
int fhe_ntt_butterfly_ceiling(fhe_ctx* ctx, double* butterflies_per_s);

/* Number of kernels this library has launched in this process (all contexts). */
int fhe_kernel_launches(uint64_t* count);

/* Operation counters of a context since creation or the last reset (the
 * reference reports ct_ct / rotations / bootstraps in native.json,
 * packed_fideslib.cpp:1239-1396; the key-switching work behind them too):
 * tensor products, relinearisations, rotations (plain and hoisted), ModUps,
 * ModDowns, key inner products, rescales, limb NTTs (forward + inverse) and
 * bootstraps.  reset != 0 zeroes them after reading. */
typedef struct fhe_counters {
  uint64_t tensor, relin, rotations, modup, moddown, key_inner, rescales, ntt_limbs, bootstraps;
} fhe_counters;
int fhe_ctx_counters(fhe_ctx* ctx, fhe_counters* out, int32_t reset);
/* The same counters by the number of live Q limbs the work ran at: out[nq]
 * for nq < n (the last of 64 entries collects nq >= 63).  kind 0 = ModUps,
 * 1 = key inner products (each followed by one ModDown), 2 = rescales,
 * 3 = tensor products.  Reset together with fhe_ctx_counters(reset).  No
 * counterpart call in the reference: its native.json reports totals only
 * (packed_fideslib.cpp:1239-1396); these weight a CPU cost model by level. */
int fhe_ctx_level_counts(fhe_ctx* ctx, int32_t kind, uint64_t* out, uint32_t n);

/* Kernel of the context's HYBRID basis conversions (ModUp and ModDown, the
 * FIDESlib ModUp / base-extension kernels behind every key switch): 0 = CUDA
 * cores (64-bit integer multiply-accumulates), 1 = tensor cores
 * (tcgen05.mma kind::i8 on the residues split into bytes) for bases of 12 to
 * 16 source limbs with every prime below 2^60, where they are faster, 2 =
 * tensor cores for every base of 1 to 16 limbs (tests); the CUDA-core kernel
 * runs wherever the tensor cores are not used.
 * Both produce identical words.  No counterpart call in the reference. */
int fhe_ctx_set_conversion(fhe_ctx* ctx, int32_t kernel);
/* Returns the device's freed library memory (kept in its stream-ordered
 * pool between contexts for reuse) to the driver, after a device
 * synchronisation: for a caller that switches to parameters with differently
 * sized buffers (ring 2^16 to 2^17).  No counterpart in the reference. */
int fhe_device_trim(int32_t device);
/* fused != 0: the key inner product of the Q limbs is formed inside the
 * ModDown's last NTT pass (its combine epilogue reads the ModUp digits and
 * the key), so the accumulator's Q rows are never written and re-read; the P
 * limbs keep the separate inner product.  The FIDESlib counterpart is its
 * NTT's KSK_DOT / KSK_DOT_ACC modes (experiments/ntt_warp_tail/probe.cu:70-73),
 * which fuse the product into the ModUp side instead.  Identical words. */
int fhe_ctx_set_keyswitch_fusion(fhe_ctx* ctx, int32_t fused);
/* on != 0 (the default): the rotating giant steps of fhe_linear_transform
 * (and of bootstrapping's CoeffToSlot / SlotToCoeff groups) share one
 * ModDown: each giant's key inner product is permuted by its automorphism
 * in the extended Q*P basis and summed there, the way OpenFHE's
 * EvalFastRotationExt / KeySwitchDown pair hoists them in its bootstrapping
 * linear transforms; the sum is brought down once.  on == 0: a full key
 * switch (with its ModDown) per giant, the composition the reference's
 * EvalLinearTransform performs.  Results agree within the key switching
 * noise, not word for word. */
int fhe_ctx_set_giant_hoisting(fhe_ctx* ctx, int32_t on);
/* Number of tensor-core conversion blocks whose bounded wait for their MMA
 * ran out (their outputs were skipped); 0 on a healthy device. */
int fhe_tc_timeouts(uint64_t* count);

/* Bootstrapping of the context's slots (full packing N/2, or sparse packing:
 * a power of two below N/2, where ModRaise is followed by the trace over the
 * rotations by multiples of the slot count, as OpenFHE does for
 * SetBatchSize(slots) < N/2), replacing OpenFHE's
 * EvalBootstrapSetup({budget_cts, budget_stc}, {0, 0}, slots, correction) /
 * EvalBootstrapKeyGen / EvalBootstrap as called at packed_fideslib.cpp:1084-1089,
 * :245 and :259.  ModRaise -> CoeffToSlot (budget_cts levels) -> EvalMod
 * (Chebyshev cosine + double angles) -> SlotToCoeff (budget_stc levels).
 * correction <= 0 picks the default pre-scaling exponent.  The input needs at
 * least 2 limbs and slots of magnitude <= 1.  s2c_first != 0 selects the
 * reference's S2C-first variant (patches/fideslib-v2.1.0-s2c-first-bootstrap.patch:27-60):
 * SlotToCoeff runs on the input's own levels before ModRaise (input needs
 * budget_stc + 2 limbs) and the output keeps budget_stc more limbs.
 * sparse_h > 0 selects sparse-secret encapsulation (FIDESlib's
 * SPARSE_ENCAPSULATED key distribution, the "sparse-encapsulated" choice of
 * native/fideslib_stage0/src/fideslib_ctpt_probe.cpp:130-137; the packed
 * executable fixes UNIFORM_TERNARY at packed_fideslib.cpp:1062): the
 * one-limb ciphertext is switched to a sparse secret of Hamming weight
 * sparse_h for ModRaise and back, so EvalMod covers |I| <= (h+1)/2 with a
 * lower degree and 4-5 fewer levels; 0 keeps the reference's uniform ternary
 * secret throughout. */
int fhe_bootstrap_setup(fhe_ctx* ctx, uint32_t budget_cts, uint32_t budget_stc, uint32_t slots,
                        int32_t correction, int32_t s2c_first, uint32_t sparse_h);
/* Sub-slot refresh (no reference counterpart: the reference bootstraps every
 * refresh over all of the context's slots, packed_fideslib.cpp:1084): a
 * bootstrapper for inputs whose values sit in slots [0, slots) with zeros
 * elsewhere, slots a power of two <= half the context's slot count (fully or
 * sparsely packed).  It bootstraps the input replicated with period `slots`
 * as a sparsely packed ciphertext (trace after ModRaise)
 * with ONE EvalMod (the real and imaginary parts side by side in 2*slots
 * slots; the split folded into the last CoeffToSlot group, the merge into the
 * first SlotToCoeff group) and returns zeros outside [0, slots) (a mask folded
 * into the last SlotToCoeff group): the same levels as the full bootstrap.
 * Several sizes may be set up; fhe_bootstrap_keygen generates the keys of
 * every setup made before it. */
int fhe_bootstrap_subslot_setup(fhe_ctx* ctx, uint32_t slots, uint32_t budget_cts, uint32_t budget_stc,
                                int32_t correction);
int fhe_bootstrap_keygen(fhe_ctx* ctx);
int fhe_bootstrap(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out);
/* The reference's refresh (PackedEvaluator::refresh / bootstrap_components,
 * packed_fideslib.cpp:235-281): bootstrap a / bound (slots within [-bound,
 * bound]); with passes == 2 the residual (x - first) * 4096 is bootstrapped
 * again and added back / 4096; the result is scaled by bound. */
int fhe_refresh(fhe_ctx* ctx, const fhe_ct* a, double bound, int32_t passes, fhe_ct** out);
/* fhe_refresh for an input known to be zero outside slots [0, support): the
 * smallest sub-slot bootstrapper with slots >= support runs it (the output is
 * zero outside [0, slots)), else the full bootstrapper; support 0 = full. */
int fhe_refresh_support(fhe_ctx* ctx, const fhe_ct* a, double bound, int32_t passes, uint32_t support,
                        fhe_ct** out);
/* One step of fhe_bootstrap (EvalCoeffsToSlots / EvalSlotsToCoeffs and their
 * neighbours in OpenFHE's FHECKKSRNS): stage 0 = scale down to one limb and
 * ModRaise, 1 = CoeffToSlot, 2 = EvalMod (real and imaginary parts), 3 =
 * SlotToCoeff.  Chaining 0..3 equals fhe_bootstrap. */
int fhe_bootstrap_stage(fhe_ctx* ctx, int32_t stage, const fhe_ct* a, fhe_ct** out);
/* Any pointer may be NULL. n_rotation_keys counts the conjugation key. */
int fhe_bootstrap_info(fhe_ctx* ctx, int32_t* correction, uint32_t* cheb_degree, uint32_t* n_rotation_keys);
/* Limb counts of the last bootstrap after ModRaise, CoeffToSlot, EvalMod and
 * SlotToCoeff (levels[4]); the reference's trace_levels telemetry. */
int fhe_bootstrap_levels(fhe_ctx* ctx, uint32_t* levels);

/* --- packed programs ------------------------------------------------------ */

/* Options of fhe_program_run; zero fields take the defaults in brackets. */
typedef struct fhe_program_options {
  uint32_t log_n;             /* ring dimension 2^log_n [smallest >= 2^12 with N/2 >= program slots] */
  uint32_t depth;             /* multiplicative depth [44] */
  uint32_t scale_bits;        /* [59] */
  uint32_t first_bits;        /* [60] */
  uint32_t dnum;              /* [3] */
  int32_t bootstrap_passes;   /* 1 or 2 [2] */
  int32_t s2c_first;          /* S2C-first bootstrap variant [0] */
  int32_t trace;              /* print per-node levels [0] */
  int32_t device;             /* CUDA device ordinal [0] */
  uint32_t sparse_h;          /* sparse-secret encapsulation weight for bootstrapping [0: off] */
  uint64_t seed;              /* key seed [1] */
  /* --security 128-classic (packed_fideslib.cpp:1060-1076): ring 2^17 unless
   * log_n is set, dnum = security_digits [4], slots = the program's slots
   * (sparse packing, the reference's SetBatchSize), uniform ternary secret,
   * and Q*P checked against the 2024 guidelines' classical-128 bound for the
   * ring (fideslib_security.hpp:18-30); the audit goes to RESULT.parameters.json
   * and native.json's security_audit. */
  int32_t security128;        /* [0: not-set] */
  uint32_t security_digits;   /* [4] */
} fhe_program_options;

/* The classical-128 audit of a parameter set without a GPU (host prime
 * generation only): the JSON of RESULT.parameters.json and whether Q*P meets
 * the bound.  The reference's CkksSecurityAudit (src/fideslib_security.hpp:33-80). */
int fhe_security_audit(uint32_t log_n, uint32_t depth, uint32_t scale_bits, uint32_t first_bits, uint32_t dnum,
                       char* json, size_t len, int32_t* passed);

/* Parses and validates a program with read_packed_program's admission rules
 * (native/fideslib_stage0/include/packed_program.hpp:60-163) without touching a
 * GPU; any output pointer may be NULL. */
int fhe_program_validate(const char* program_path, int32_t* slots, int32_t* nodes, int32_t* outputs);

/* The reference's packed_fideslib executable as one call
 * (native/fideslib_stage0/src/packed_fideslib.cpp:882-1403): reads a
 * fhemamba-packed-v1/v2 program, owns all crypto state (keys, bootstrapping),
 * evaluates every node on the device (PackedEvaluator::evaluate, :600-836,
 * baseline refresh policy), optionally runs the client vocabulary head for
 * greedy feedback (client_head_path: u32 vocab, u32 width, f32[vocab*width];
 * NULL for none), and writes the fhemamba-packed-result-v1 JSON.
 * Returns 0 when every output is within both tolerances, 1 when a gate fails,
 * a negative error code otherwise (fhe_last_error has the message). */
int fhe_program_run(const char* program_path, const char* client_head_path, const char* result_path,
                    double poly_tol, double exact_tol, const fhe_program_options* options);

/* Bootstrapping ModRaise (EvalBootstrap's first step): the centred
 * coefficients of limb 0 lifted to every Q limb. */
int fhe_mod_raise(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out);

/* Multiplies every slot by the imaginary unit exactly (times X^{N/2}); used to
 * split and merge real/imaginary parts in CoeffToSlot/SlotToCoeff. */
int fhe_mul_i(fhe_ctx* ctx, const fhe_ct* a, fhe_ct** out);

/* SetScalingFactor: reinterprets the ciphertext's scale without touching it. */
int fhe_ct_set_scale(fhe_ctx* ctx, fhe_ct* ct, double scale);

/* EvalChebyshevSeries: sum_{i<n} coeffs[i] T_i((2a - lo - hi)/(hi - lo)) by
 * Paterson-Stockmeyer with the reference's recursion
 * (PackedEvaluator::chebyshev, packed_fideslib.cpp:533-599). */
int fhe_chebyshev(fhe_ctx* ctx, const fhe_ct* a, const double* coeffs, uint32_t n, double lo, double hi,
                  fhe_ct** out);

/* Rescale that allocates nothing.  This entry point has no counterpart in the
 * reference; it exists for callers that cannot let the library allocate
 * device memory when they rescale — code working inside a memory budget
 * reserved in advance, or a host framework that owns every device allocation.
 * `in` holds device residues [ncomp][n_limbs][N] (NTT form), `out` receives
 * [ncomp][n_limbs-1][N] and must not overlap `in` (rejected with
 * FHE_ERR_INVALID); the result equals fhe_rescale word for word.  Scratch
 * comes from one fixed 32 MiB device array that every GPU loading this
 * library keeps until the process exits; sizes needing more (2(n_limbs-1) +
 * ncomp*N*n_limbs words) are rejected with FHE_ERR_INVALID.  The first call
 * on each device looks up that array's device address (set-up once per
 * device), so make that first call before any stream capture.  All calls
 * share the one array, so calls whose GPU work overlaps (other contexts,
 * other streams) race; the array keeps the last call's contents, and every
 * word a call reads was written earlier by the same call. */
int fhe_rescale_noalloc(fhe_ctx* ctx, const uint64_t* in, uint32_t ncomp, uint32_t n_limbs, uint64_t* out);

#ifdef __cplusplus
}
#endif
#endif
