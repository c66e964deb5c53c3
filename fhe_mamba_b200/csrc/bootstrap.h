// CKKS bootstrapping for fully or sparsely packed ciphertexts (slots a power
// of two <= N/2): ModRaise (+ the sparse-packing trace) -> CoeffToSlot ->
// EvalMod -> SlotToCoeff, the pipeline of OpenFHE's FHECKKSRNS that the
// reference drives through EvalBootstrapSetup({4,4},{0,0},slots,0) /
// EvalBootstrapKeyGen / EvalBootstrap (packed_fideslib.cpp:1084-1089, :245, :259).
//
// CoeffToSlot and SlotToCoeff are the special inverse / forward FFT of the
// slot encoding without its bit reversal (EvalMod is slot-wise, so the two
// reversals cancel), split into `budget` groups of consecutive butterfly
// stages.  A group of k stages with smallest half-distance h is a matrix with
// diagonals at multiples of h (2^{k+1}-1 of them, 2^k for the group holding
// the top stage) and runs as one strided BSGS linear transform, one level.
// EvalMod evaluates sin(2 pi y)/(2 pi) ~ y - round(y) as a Chebyshev
// approximation of cos(2 pi (y - 1/4) / 2^r) followed by r double-angle steps.
#pragma once
#include <complex>
#include <cstdint>
#include <map>
#include <memory>
#include <vector>

#include "ckks.h"

namespace fhe {

struct BootParams {
  uint32_t budget_cts = 4, budget_stc = 4;
  // log2 of the extra down-scaling applied before ModRaise; 0 picks the default.
  int correction = 0;
  double K = 512.0;       // bound on |I| in the raised plaintext m + q0*I (uniform ternary secret)
  int double_angles = 6;  // r
  // SlotToCoeff before ModRaise (the reference's S2C-first patch): the input's
  // own levels pay for SlotToCoeff, so the output keeps budget_stc more limbs.
  bool s2c_first = false;
  // Sparse-secret encapsulation (FIDESlib's SPARSE_ENCAPSULATED key
  // distribution): 0 keeps the uniform ternary secret; h > 0 switches the
  // one-limb ciphertext to a sparse secret of Hamming weight h before
  // ModRaise and back right after it, so |I| <= (h + 1) / 2 and EvalMod needs
  // a far smaller interval, degree and depth.
  uint32_t sparse_h = 0;
  // Sub-slot refresh: 0 bootstraps all of the context's slots; a power of
  // two n <= half the context's slots bootstraps inputs whose values
  // sit in slots [0, n) (zeros elsewhere), replicated with period n by the
  // caller: the sparse-packing pipeline on n slots with ONE EvalMod (the real
  // and imaginary parts of CoeffToSlot's output side by side in 2n slots;
  // the split is folded into the last CoeffToSlot group, the merge into the
  // first SlotToCoeff group) and the output masked to [0, n) inside the last
  // SlotToCoeff group.  No extra level.
  uint32_t slots = 0;
};

class Bootstrapper {
 public:
  Bootstrapper(Ckks& ck, const BootParams& p);

  // Rotation steps (slot amounts) the transforms need; keygen() generates
  // them and the conjugation key.
  std::vector<int64_t> rotation_steps() const;
  void keygen();

  // Refreshes a ciphertext with >= 2 limbs (>= budget_stc + 2 with
  // s2c_first) whose slots are bounded by 1 in magnitude.  The output
  // decrypts to the same slots with fresh levels.
  std::unique_ptr<Ct> bootstrap(const Ct& a);
  // Slots this bootstrapper covers (the context's, or the sub-slot count).
  uint32_t slots() const { return n_; }
  // x replicated with period slots() over the context's slots (x zero
  // outside [0, slots())): log2(context slots / slots()) rotate-and-add
  // doublings.
  std::unique_ptr<Ct> replicate(const Ct& x);

  // The four steps of bootstrap(), each on its own (the pieces that
  // EvalCoeffsToSlots / EvalSlotsToCoeffs expose in OpenFHE):
  //   raise:          adjust to one limb at scale q0 2^-correction, ModRaise,
  //                   scale attribute set to the top level's scale;
  //   coeff_to_slot:  BR(w) / (2K), w = (t_lo + i t_hi) / q0 of the raised plaintext t;
  //   eval_mod:       BR(w mod 1) * 2 pi (real and imaginary parts separately);
  //   slot_to_coeff:  the inverse of coeff_to_slot back to the input's slots.
  std::unique_ptr<Ct> raise(const Ct& a);
  std::unique_ptr<Ct> coeff_to_slot(const Ct& raised);
  std::unique_ptr<Ct> eval_mod_full(const Ct& x);
  std::unique_ptr<Ct> slot_to_coeff(const Ct& w);

  const BootParams& params() const { return p_; }
  int correction() const { return corr_; }
  // Chebyshev coefficients of the EvalMod cosine.
  const std::vector<double>& eval_mod_coefficients() const { return cheb_; }
  // Limb counts seen by the last bootstrap: after ModRaise, CoeffToSlot,
  // EvalMod and SlotToCoeff.
  const uint32_t* last_levels() const { return levels_; }

 private:
  struct Group {
    uint32_t b = 0, G = 0;
    int64_t stride = 0, offset = 0;
    // Diagonal vectors over the context's slots, pre-rotated; empty = zero.
    // With a companion (aux != 0) the group computes LT(x, diags) +
    // LT(aux(x), diags2), aux 1 = conjugate, 2 = rotation by n slots.
    std::vector<std::vector<std::complex<double>>> diags, diags2;
    int aux = 0;
    std::map<uint32_t, std::vector<std::unique_ptr<Pt>>> enc, enc2;  // encodings by limb count
    std::map<uint32_t, double> enc_scale;                            // their encoding scale
  };
  // Edits applied to a group's matrix before its diagonals are laid out:
  // none, the CoeffToSlot split (companion on the conjugate), the
  // SlotToCoeff merge (companion on the rotation by n), the output mask.
  enum class Edit { None, Split, Merge, Mask };
  void build_groups(std::vector<Group>& out, const std::vector<uint32_t>& halves, uint32_t budget, bool inverse,
                    double factor, Edit first, Edit last);
  std::unique_ptr<Ct> transform(std::vector<Group>& groups, std::unique_ptr<Ct> x);
  uint64_t aux_galois(const Group& g) const;  // conjugation (aux 1) or rotation by n (aux 2)
  std::unique_ptr<Ct> eval_mod(const Ct& x);

  Ckks& ck_;
  BootParams p_;
  int corr_ = 0;
  uint32_t n_ = 0;      // slots bootstrapped
  bool single_ = false;  // one EvalMod over 2n slots (sub-slot refresh)
  uint32_t trace_ = 1;  // N / (2 slots): automorphisms summed after ModRaise (sparse packing)
  std::vector<Group> cts_, stc_;
  std::vector<double> cheb_;
  uint32_t levels_[4] = {0, 0, 0, 0};
};

}  // namespace fhe
