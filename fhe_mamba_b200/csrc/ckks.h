// RNS-CKKS evaluator on the device (host orchestration of ckks_kernels + ntt).
//
// Semantics follow the OpenFHE CryptoContext the reference drives
// (packed_fideslib.cpp:117-281): FLEXIBLEAUTO scaling (level scaling factors
// sf_k = sf_{k-1}^2 / q_{L-k}, automatic rescale of degree-2 inputs before a
// multiplication), HYBRID key switching with dnum digits, rotations by
// key-switch-then-automorphism, hoisted rotations sharing one ModUp.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "ckks_kernels.h"
#include "context.h"

namespace fhe {

// Device ciphertext: ncomp components of cap limbs each; the first nq limbs of
// every component are live.  Component c, limb l at data + (c*cap + l)*N.
struct Ct {
  DevMem buf;
  uint32_t cap = 0, nq = 0, ncomp = 2, noise_deg = 1;
  double scale = 1.0;
  uint64_t* data() const { return buf.as<uint64_t>(); }
};

// Device plaintext in NTT form over nq limbs.
struct Pt {
  DevMem buf;
  uint32_t nq = 0, noise_deg = 1;
  double scale = 1.0;
  uint64_t* data() const { return buf.as<uint64_t>(); }
};

// Per-level key-switching tables (built on first use of a level).
struct LevelTables {
  uint32_t nq = 0, D = 0, w = 0;
  DevMem digits;    // ModUpDigit[D]
  DevMem blob;      // backing store of all ConvTable arrays of this level
  DevMem ntt_list;  // uint2[]: ext limbs that need a forward NTT after ModUp
  uint32_t ntt_list_len = 0;
  DevMem moddown;   // ConvTable (P -> Q_nq)
  DevMem tc_blob;   // tensor-core operand tables of the ModUp digits
  bool tc_modup = false;  // every digit has a tensor-core table
};

// Operation counters (the reference's native.json ct_ct / rotations /
// bootstraps fields plus the key-switching work behind them).
struct Counters {
  uint64_t tensor = 0, relin = 0, rotations = 0, modup = 0, moddown = 0, key_inner = 0, rescales = 0,
           ntt_limbs = 0, bootstraps = 0;
  // The same work by the number of live Q limbs it ran at (index nq, the
  // last slot collects nq >= kLevels - 1): ModUps, key inner products (each
  // followed by its ModDown), rescales and tensor products.  A cost model of
  // another implementation multiplies these by its own per-level times.
  static constexpr uint32_t kLevels = 64;
  uint64_t modup_at[kLevels] = {}, key_inner_at[kLevels] = {}, rescale_at[kLevels] = {}, tensor_at[kLevels] = {};
  static uint32_t slot(uint32_t nq) { return nq < kLevels ? nq : kLevels - 1; }
};

class Ckks {
 public:
  explicit Ckks(Context& c);
  Context& ctx;
  Counters counters;

  // Basis conversions: 0 = CUDA cores, 1 = tensor cores (conv_tc.cu) for
  // bases where they are faster, 2 = tensor cores wherever supported (for
  // tests); every choice gives the same words.
  int tc_conversion = 0;
  // Key inner product of the Q limbs folded into ModDown's combine epilogue
  // (the accumulator's Q rows are never written and re-read); same words.
  bool fused_key_inner = false;
  // Giant steps of a linear transform share ONE ModDown: each rotating giant's
  // key inner product is permuted by its automorphism in the extended basis
  // and summed there (ModDown is linear and commutes with automorphisms up
  // to its rounding), instead of a ModDown per giant.  Different words than
  // a ModDown per giant; the same noise bound.
  bool hoist_giant_moddown = true;

  // FLEXIBLEAUTO scaling factor of a fresh ciphertext with nq live limbs.
  double level_scale(uint32_t nq) const { return sf_[ctx.L - nq]; }

  // keys
  void keygen(uint64_t seed);
  bool has_keys() const { return keyed_; }
  // false for an evaluation-only context loaded from a key bundle without
  // the secret (see serialize.cu)
  bool has_secret() const { return has_secret_; }
  void save_keys(const std::string& path, bool with_secret);
  void load_keys(const std::string& path);
  uint64_t galois_for_step(int64_t step) const;
  uint64_t galois_for_full_step(int64_t step) const;
  void rotation_keygen(uint64_t g);
  bool has_rotation_key(uint64_t g) const { return rot_.count(g) != 0; }
  void download_key(int kind, uint64_t g, uint64_t* host) const;
  // Sparse-secret encapsulation for bootstrapping: a sparse ternary secret s'
  // of Hamming weight h and the switching keys s -> s' and s' -> s.
  void sparse_keygen(uint32_t h);
  uint32_t sparse_weight() const { return sparse_h_; }
  std::unique_ptr<Ct> switch_to_sparse(const Ct& a);
  std::unique_ptr<Ct> switch_to_dense(const Ct& a);
  size_t key_words(int kind) const;

  // encode / encryption
  std::unique_ptr<Pt> encode(const double* re, const double* im, uint32_t count, uint32_t nq, double scale);
  void decode(const Pt& p, double* re, double* im, uint32_t count);
  // Encodes B vectors of `count` values (values[b*count + i]) at nq limbs.
  // Diagonal plaintexts t = 0..T-1 of the replicated BSGS layout of y = W x
  // (W: m x cols, row-major fp64 on this device): window r < R of `win`
  // slots holds W[i][(i + r T + t) % cols] at slot r win + i (i < m), the
  // vector rotated by (t / baby) * baby slots (pre-rotated for its giant step).
  std::vector<std::unique_ptr<Pt>> encode_replicated_diagonals(const double* w_dev, uint32_t m, uint32_t cols,
                                                               uint32_t R, uint32_t T, uint32_t win, uint32_t baby,
                                                               uint32_t nq, double scale);
  std::vector<std::unique_ptr<Pt>> encode_batch(const double* re, const double* im, uint32_t B, uint32_t count,
                                                uint32_t nq, double scale);
  std::unique_ptr<Ct> encrypt(const Pt& p);
  std::unique_ptr<Pt> decrypt(const Ct& c);

  // arithmetic (all outputs are new handles)
  std::unique_ptr<Ct> alloc(uint32_t nq, uint32_t ncomp);
  std::unique_ptr<Ct> clone(const Ct& a);
  std::unique_ptr<Ct> add(const Ct& a, const Ct& b, bool subtract);
  std::unique_ptr<Ct> add_plain(const Ct& a, const Pt& p, bool subtract);
  std::unique_ptr<Ct> mul_plain(const Ct& a, const Pt& p);
  std::unique_ptr<Ct> add_scalar(const Ct& a, double v);
  std::unique_ptr<Ct> mul_scalar(const Ct& a, double v);
  std::unique_ptr<Ct> mul_int(const Ct& a, int64_t v);  // exact integer multiple, scale unchanged
  std::unique_ptr<Ct> negate(const Ct& a);
  std::unique_ptr<Ct> tensor(const Ct& a, const Ct& b);
  std::unique_ptr<Ct> relinearize(const Ct& d);
  std::unique_ptr<Ct> mul(const Ct& a, const Ct& b);
  void rescale_inplace(Ct& a);
  std::unique_ptr<Ct> rescaled(const Ct& a);
  // OpenFHE EvalLinearWSum: sum_i w_i x_i + c0 for ciphertexts on one level with
  // one scale, in one pass (the weights are encoded at the level's scale).
  std::unique_ptr<Ct> linear_wsum(const std::vector<const Ct*>& xs, const std::vector<double>& w, double c0);
  void level_reduce_inplace(Ct& a, uint32_t levels);
  std::unique_ptr<Ct> rotate(const Ct& a, uint64_t g);
  std::vector<std::unique_ptr<Ct>> rotate_hoisted(const Ct& a, const std::vector<uint64_t>& gs);

  // BSGS diagonal linear transform (the reference's PackedEvaluator::linear /
  // LinearTransformInPlace): out = sum_g rot( sum_j diag[g*b+j] (.) rot(a, j), g*b ).
  // diags has b*G entries (null = zero diagonal), each encoded at >= a.nq limbs
  // with the same scale; babies share one ModUp.
  // General form: baby j rotates by j*stride, giant g by (g*b - giant_offset)*stride,
  // so diagonal (g*b + j - giant_offset)*stride is pre-rotated by the giant amount.
  // aux_galois != 0 adds a companion transform of the same shape on
  // sigma_aux(a): diags then has 2b*G entries, [g][0, b) on a and [g][b, 2b) on
  // sigma_aux(a); the companion's babies sigma_aux o rot(j*stride) share the
  // ModUp and every giant step with the main transform.
  std::unique_ptr<Ct> linear_transform(const Ct& a, const std::vector<const Pt*>& diags, uint32_t b, uint32_t G,
                                       int64_t stride = 1, int64_t giant_offset = 0, uint64_t aux_galois = 0);

  // ModRaise for bootstrapping: the centred coefficients of limb 0 lifted to
  // every Q limb (the plaintext becomes m + q_0 I).
  std::unique_ptr<Ct> mod_raise(const Ct& a);
  // Exact multiplication of every slot by the imaginary unit (times X^{N/2}).
  std::unique_ptr<Ct> mul_i(const Ct& a);

  // Paterson-Stockmeyer evaluation of sum_i c_i T_i(u), u = (2x - lo - hi) / (hi - lo),
  // following the reference's PackedEvaluator::chebyshev (packed_fideslib.cpp:533-599):
  // T_{2k} = 2 T_k^2 - 1, T_{2k+1} = 2 T_k T_{k+1} - u, baby size
  // 2^ceil(log2(deg+1)/2), recursive division by T_k for k a power of two.
  std::unique_ptr<Ct> chebyshev(const Ct& x, const std::vector<double>& c, double lo, double hi);

  // Brings `a` to (nq, scale): FLEXIBLEAUTO adjustment by an integer multiple
  // and a rescale, then dropping limbs.
  std::unique_ptr<Ct> adjust(const Ct& a, uint32_t nq, double scale);

  uint64_t enc_nonce = 1;

 private:
  void build_static_tables();
  LevelTables& level(uint32_t nq);
  // Key switch of d (NTT form, nq limbs) with evk: out = (u0 [+ add_c0], u1),
  // component stride so.
  void keyswitch(const uint64_t* d, uint32_t nq, const uint64_t* evk, uint64_t* out, size_t so,
                 const uint64_t* add_c0);
  void modup(const uint64_t* d, uint32_t nq, uint64_t* ext);
  void moddown_pair(uint64_t* acc, uint32_t nq, uint64_t* out, size_t so, const uint64_t* add_c0,
                    const uint64_t* ext = nullptr, const uint64_t* evk = nullptr);
  // Key inner product of the ModUp digits `ext` with `evk` followed by the
  // ModDown pair into out (+ add_c0): with fused_key_inner the Q limbs'
  // inner product is formed inside ModDown's last NTT pass.
  void key_moddown(const uint64_t* ext, const uint64_t* evk, uint32_t nq, uint64_t* out, size_t so,
                   const uint64_t* add_c0);
  void switch_keygen(uint64_t key_id, const uint64_t* s_new, const uint64_t* s_old, DevMem& out);
  void ntt_dense(uint64_t* d, uint32_t polys, uint32_t limbs, uint32_t stride, uint32_t prime0, bool inv);
  void encode_slots_on_device(double2* dv, uint32_t nb, uint32_t nq, double scale, bool check,
                              std::vector<std::unique_ptr<Pt>>& out);
  uint64_t* ws(size_t idx, size_t words);
  std::vector<uint64_t> scalar_residues(long double v, uint32_t nq) const;
  std::unique_ptr<Ct> prepare_mult_input(const Ct& a);
  // `a` itself, or its rescaled copy (kept in `hold`) when a rescale is pending.
  const Ct& ready(const Ct& a, std::unique_ptr<Ct>& hold);
  void rescale_into(const Ct& a, Ct& out);

  std::vector<double> sf_;
  std::map<uint32_t, LevelTables> levels_;
  DevMem pinv_;        // Shoup[L]: P^{-1} mod q_i
  DevMem qinv_;        // Shoup[L][L]: q_last^{-1} mod q_i
  DevMem pmod_;        // Shoup[L+K]: P mod q_i (0 for P primes)
  DevMem mdtab_blob_;  // P -> Q conversion arrays (shared by all levels)
  DevMem mdtab_tc_;    // their tensor-core operand table (empty when not supported)
  std::vector<Modulus> mods_host_;
  DevMem fft_inv_tw_, fft_fwd_tw_;
  bool keyed_ = false;
  bool has_secret_ = false;
  uint64_t seed_ = 0;
  DevMem s_ntt_, pk_, rlk_;
  DevMem s_sparse_, key_to_sparse_, key_to_dense_;
  uint32_t sparse_h_ = 0;
  std::unique_ptr<Ct> switch_with(const Ct& a, const DevMem& key);
  std::map<uint64_t, DevMem> rot_;
  std::vector<DevMem> ws_;
  // Sticky status of the encoders' rounding kernels (non-finite or >= 2^126
  // values); read and cleared by check_encode_status().
  DevMem status_;
  void check_encode_status();
  // Ring of pinned host buffers for host -> device uploads that must not
  // block the host: a slot is rewritten only after the copy that read it
  // (its event) has run, so the host can run up to kStageSlots uploads ahead.
  struct StageSlot {
    void* host = nullptr;
    size_t bytes = 0;
    cudaEvent_t done = nullptr;
    bool pending = false;
  };
  static constexpr size_t kStageSlots = 16;
  std::vector<StageSlot> stage_ring_;
  size_t stage_next_ = 0;
  void stage_upload(void* dev, const void* host, size_t bytes);
  const void* stage_pointers(const void* host, size_t bytes, size_t ws_idx);

 public:
  ~Ckks();
  friend class ShardKeySwitch;
};

// Ciphertext files for a process-separated client and server (serialize.cu).
void save_ciphertext(Ckks& k, const Ct& c, const std::string& path);
std::unique_ptr<Ct> load_ciphertext(Ckks& k, const std::string& path);

}  // namespace fhe
