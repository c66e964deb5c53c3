// CKKS bootstrapping (host orchestration; every step runs on the device
// through the Ckks evaluator).
#include "bootstrap.h"

#include <algorithm>
#include <cmath>
#include <functional>

namespace fhe {
namespace {

using cd = std::complex<double>;
// Sparse matrix over n slots by diagonals: d -> v, (M x)[r] = sum_d v_d[r] x[(r + d) mod n].
using Sparse = std::map<uint32_t, std::vector<cd>>;

// exp(2 pi i k / m) with the angle reduced exactly first.
cd unit_root(uint64_t k, uint64_t m) {
  const double a = 2.0 * M_PI * (double)(k % m) / (double)m;
  return {std::cos(a), std::sin(a)};
}

void put(Sparse& s, uint32_t n, int64_t d, uint32_t r, cd v) {
  const uint32_t k = (uint32_t)(((d % (int64_t)n) + n) % n);
  auto& row = s[k];
  if (row.empty()) row.assign(n, cd(0, 0));
  row[r] += v;
}

// One butterfly stage of the special FFT with half-distance h (block 2h):
// forward  out[i+j] = u + xi_j v, out[i+j+h] = u - xi_j v;
// inverse  out[i+j] = (u + v)/2,  out[i+j+h] = (u - v) conj(xi_j)/2,
// xi_j = exp(2 pi i (5^j mod 8h) / 8h) (the slot order of the encoder).
Sparse stage(uint32_t n, uint32_t h, bool inverse) {
  Sparse s;
  const uint64_t m = 8ull * h;
  std::vector<cd> xi(h);
  uint64_t p = 1;
  for (uint32_t j = 0; j < h; ++j, p = p * 5 % m) xi[j] = unit_root(p, m);
  for (uint32_t i = 0; i < n; i += 2 * h)
    for (uint32_t j = 0; j < h; ++j) {
      const uint32_t r = i + j, r2 = i + j + h;
      if (!inverse) {
        put(s, n, 0, r, 1.0);
        put(s, n, h, r, xi[j]);
        put(s, n, -(int64_t)h, r2, 1.0);
        put(s, n, 0, r2, -xi[j]);
      } else {
        const cd c = std::conj(xi[j]) * 0.5;
        put(s, n, 0, r, 0.5);
        put(s, n, h, r, 0.5);
        put(s, n, -(int64_t)h, r2, c);
        put(s, n, 0, r2, -c);
      }
    }
  return s;
}

// y = A (B x)
Sparse compose(const Sparse& A, const Sparse& B, uint32_t n) {
  Sparse C;
  for (const auto& [d1, a] : A)
    for (const auto& [d2, b] : B) {
      auto& c = C[(uint32_t)(((uint64_t)d1 + d2) % n)];
      if (c.empty()) c.assign(n, cd(0, 0));
      for (uint32_t r = 0; r < n; ++r) c[r] += a[r] * b[(r + d1) % n];
    }
  return C;
}

uint32_t ceil_log2(uint64_t x) {
  uint32_t k = 0;
  while ((1ull << k) < x) ++k;
  return k;
}

// Chebyshev interpolant of f on [-1, 1] at degree d (nodes cos(pi (k + 1/2) / (d + 1))):
// p = c_0 + sum_j c_j T_j.  The cosine arguments are reduced exactly in integers.
std::vector<double> cheb_fit(const std::function<double(double)>& f, int d) {
  const int64_t m = 4 * (int64_t)(d + 1);  // angle pi j (2k+1) / (2(d+1)) = 2 pi [j (2k+1) mod m] / m
  std::vector<double> fx(d + 1), c(d + 1);
  for (int k = 0; k <= d; ++k) fx[k] = f(unit_root(2 * k + 1, m).real());
  for (int j = 0; j <= d; ++j) {
    long double s = 0;
    for (int k = 0; k <= d; ++k) s += (long double)fx[k] * unit_root((uint64_t)j * (2 * k + 1), m).real();
    c[j] = (double)(2.0L * s / (d + 1));
  }
  c[0] *= 0.5;
  return c;
}

}  // namespace

Bootstrapper::Bootstrapper(Ckks& ck, const BootParams& p) : ck_(ck), p_(p) {
  Context& ctx = ck.ctx;
  n_ = p_.slots ? p_.slots : ctx.slots;
  const uint32_t n = n_;
  require(n >= 2 && n <= ctx.n / 2 && (n & (n - 1)) == 0, "bootstrapping needs a power-of-two slot count <= N/2",
          -1);
  if (p_.slots) {
    // 2n of the context's slots hold the real and imaginary halves
    require(n <= ctx.slots / 2, "sub-slot refresh slots must be a power of two <= half the context's slots", -1);
    require(!p_.s2c_first && !p_.sparse_h, "a sub-slot refresh combines with neither S2C-first nor a sparse secret",
            -1);
    single_ = true;
  }
  // Sparse packing (n < N/2): the plaintext lives in Z[X^g'], g' = N/(2n);
  // after ModRaise the trace over the g = N/(2n) automorphisms fixing that
  // subring (rotations by multiples of n) keeps g times its part of
  // m + q0 I, and CoeffToSlot divides by g.
  trace_ = ctx.n / (2 * n);
  require(!(p_.s2c_first && trace_ > 1), "SlotToCoeff-first bootstrapping needs fully packed slots", -1);
  const uint32_t logn = ceil_log2(n);
  require(p_.budget_cts >= 1 && p_.budget_stc >= 1, "level budgets must be >= 1", -1);
  p_.budget_cts = std::min(p_.budget_cts, logn);
  p_.budget_stc = std::min(p_.budget_stc, logn);
  require(!single_ || p_.budget_stc >= 2, "a sub-slot refresh needs at least two SlotToCoeff groups", -1);
  if (p_.sparse_h) {
    require(p_.sparse_h <= ctx.n / 2, "sparse Hamming weight out of range", -1);
    p_.K = std::ceil((p_.sparse_h + 1) / 2.0) + 2.0;  // |I| <= (h + 1) / 2
    p_.double_angles = 3;
  }
  require(p_.K >= 1 && p_.double_angles >= 0 && p_.double_angles <= 12, "bad EvalMod parameters", -1);
  // Default pre-scaling: the sine approximation error shrinks by 4x per step
  // while the amplified noise grows by 2x; 8 balances them for uniform
  // ternary secrets at N = 2^16 with 59-bit scaling primes, 9 below.
  corr_ = p_.correction > 0 ? p_.correction : (ctx.log_n >= 16 ? 8 : 9);
  require(corr_ <= 40, "correction must be <= 40", -1);
  require(ctx.L > p_.budget_cts + p_.budget_stc + 2, "the modulus chain is too short for bootstrapping", -1);

  // CoeffToSlot: raised slots (q0 / S) U0 w  ->  BR(w) / (2K), S the scale
  // attribute given to the raised ciphertext (the top level's); every group
  // then lands exactly on the FLEXIBLEAUTO scale of its output level.
  const double S = ck.level_scale(ctx.L);
  const double alpha = S / (2.0 * p_.K * (double)ctx.primes[0] * (double)trace_);
  std::vector<uint32_t> halves;
  for (uint32_t h = n / 2; h >= 1; h /= 2) halves.push_back(h);
  build_groups(cts_, halves, p_.budget_cts, true, std::pow(alpha, 1.0 / p_.budget_cts), Edit::None,
               single_ ? Edit::Split : Edit::None);
  // SlotToCoeff: BR(w') -> U0 w' / (2 pi); the 2^correction factor is an exact
  // integer multiplication afterwards.
  std::reverse(halves.begin(), halves.end());
  build_groups(stc_, halves, p_.budget_stc, false, std::pow(1.0 / (2.0 * M_PI), 1.0 / p_.budget_stc),
               single_ ? Edit::Merge : Edit::None, single_ ? Edit::Mask : Edit::None);

  // EvalMod cosine: p(u) ~ cos(2 pi (K u - 1/4) / 2^r) on [-1, 1], truncated
  // where every remaining coefficient is below 2^-48.
  const double K = p_.K, R = std::ldexp(1.0, p_.double_angles);
  auto f = [K, R](double u) { return std::cos(2.0 * M_PI * (K * u - 0.25) / R); };
  std::vector<double> c = cheb_fit(f, 191);
  int deg = (int)c.size() - 1;
  while (deg > 1 && std::fabs(c[deg]) < 0x1p-48) --deg;
  c.resize(deg + 1);
  cheb_ = std::move(c);
}

void Bootstrapper::build_groups(std::vector<Group>& out, const std::vector<uint32_t>& halves, uint32_t budget,
                                bool inverse, double factor, Edit first, Edit last) {
  const uint32_t n = n_, S = ck_.ctx.slots;
  const uint32_t stages = (uint32_t)halves.size();
  size_t pos = 0;
  for (uint32_t gi = 0; gi < budget; ++gi) {
    const uint32_t k = stages / budget + (gi < stages % budget ? 1 : 0);
    Sparse M;
    uint32_t hmin = n, hmax = 0;
    for (uint32_t s = 0; s < k; ++s) {
      const uint32_t h = halves[pos + s];
      Sparse st = stage(n, h, inverse);
      M = M.empty() ? std::move(st) : compose(st, M, n);
      hmin = std::min(hmin, h);
      hmax = std::max(hmax, h);
    }
    pos += k;
    for (auto& [d, v] : M)
      for (auto& x : v) x *= factor;
    Group g;
    g.stride = hmin;
    const bool top = hmax == n / 2;
    // diagonal index t (diagonal t*hmin): t in [0, 2^k) for the top group,
    // [-T, T] with T = 2^k - 1 otherwise.
    const int64_t count = top ? (int64_t)1 << k : ((int64_t)1 << (k + 1)) - 1;
    const int64_t T = ((int64_t)1 << k) - 1;
    g.b = 1u << ((ceil_log2((uint64_t)count) + 1) / 2);
    // giant offset: a multiple of b, so one giant step is the identity
    g.offset = top ? 0 : ((T + g.b - 1) / g.b) * g.b;
    g.G = top ? (uint32_t)((count + g.b - 1) / g.b) : (uint32_t)((g.offset + T + g.b) / g.b);
    // (with one group a CoeffToSlot split, which is always `last`, wins)
    Edit edit = gi == 0 ? first : Edit::None;
    if (gi + 1 == budget && last != Edit::None) edit = last;
    g.aux = edit == Edit::Split ? 1 : edit == Edit::Merge ? 2 : 0;
    g.diags.resize((size_t)g.b * g.G);
    if (g.aux) g.diags2.resize((size_t)g.b * g.G);
    const cd I(0, 1);
    // Over 2n slots (k mod 2n < n: the real parts' half, else the imaginary
    // parts'): z = P x + Q conj(x) splits CoeffToSlot's output x into re / im,
    // w = R1 e + R2 rot(e, n) merges EvalMod's output e back.
    auto lower = [n](int64_t k) { return ((k % (2 * (int64_t)n)) + 2 * (int64_t)n) % (2 * (int64_t)n) < n; };
    for (uint32_t gg = 0; gg < g.G; ++gg)
      for (uint32_t j = 0; j < g.b; ++j) {
        const int64_t t = (int64_t)gg * g.b + j - g.offset;
        if (top ? (t < 0 || t >= count) : (t < -T || t > T)) continue;
        const int64_t amount = t * (int64_t)hmin;  // the diagonal's rotation (signed)
        const uint32_t d = (uint32_t)((amount % (int64_t)n + n) % n);
        auto it = M.find(d);
        if (it == M.end()) continue;
        const auto& v = it->second;
        if (std::all_of(v.begin(), v.end(), [](const cd& x) { return x == cd(0, 0); })) continue;
        // The diagonal over its period P (n, 2n, or S for the masked output).
        const uint32_t P = edit == Edit::None ? n : edit == Edit::Mask ? S : 2 * n;
        std::vector<cd> D(P), D2;
        if (g.aux) D2.resize(P);
        for (uint32_t i = 0; i < P; ++i) {
          const cd x = v[i % n];
          switch (edit) {
            case Edit::None: D[i] = x; break;
            case Edit::Mask: D[i] = i < n ? x : cd(0, 0); break;
            case Edit::Split:
              D[i] = lower(i) ? x : -I * x;
              D2[i] = lower(i) ? std::conj(x) : I * std::conj(x);
              break;
            case Edit::Merge:
              D[i] = x * (lower(i + amount) ? cd(1, 0) : I);
              D2[i] = x * (lower(i + amount) ? I : cd(1, 0));
              break;
          }
        }
        // pre-rotate by the giant amount r over the period, D'[i] = D[(i - r) mod P],
        // then lay the period out over the context's S slots
        const int64_t r = (int64_t)gg * g.b - g.offset;
        const int64_t rr = ((r * (int64_t)hmin) % (int64_t)P + P) % P;
        auto place = [&](const std::vector<cd>& src) {
          std::vector<cd> o(S);
          for (uint32_t i = 0; i < S; ++i) o[i] = src[(i % P + P - (uint32_t)rr) % P];
          return o;
        };
        g.diags[(size_t)gg * g.b + j] = place(D);
        if (g.aux) g.diags2[(size_t)gg * g.b + j] = place(D2);
      }
    out.push_back(std::move(g));
  }
}

std::vector<int64_t> Bootstrapper::rotation_steps() const {
  std::vector<int64_t> s;
  for (const auto* gs : {&cts_, &stc_})
    for (const Group& g : *gs) {
      // baby steps j*stride < n
      for (uint32_t j = 1; j < g.b; ++j) s.push_back((int64_t)j * g.stride);
      // giant steps exactly as linear_transform asks for them (signed): with
      // sparse packing a step and its residue mod n are different keys
      for (uint32_t gg = 0; gg < g.G; ++gg) {
        const int64_t r = ((int64_t)gg * g.b - g.offset) * g.stride;
        if (r) s.push_back(r);
      }
    }
  std::sort(s.begin(), s.end());
  s.erase(std::unique(s.begin(), s.end()), s.end());
  return s;
}

void Bootstrapper::keygen() {
  require(ck_.has_keys(), "bootstrap keygen before keygen", -4);
  for (int64_t st : rotation_steps()) {
    const uint64_t g = ck_.galois_for_step(st);
    if (!ck_.has_rotation_key(g)) ck_.rotation_keygen(g);
  }
  const uint64_t conj = 2ull * ck_.ctx.n - 1;
  if (!ck_.has_rotation_key(conj)) ck_.rotation_keygen(conj);
  // companion babies: sigma_aux o rot(j * stride), j < b
  for (const auto* gs : {&cts_, &stc_})
    for (const Group& g : *gs)
      if (g.aux)
        for (uint32_t j = 0; j < g.b; ++j) {
          const uint64_t a = aux_galois(g);
          const uint64_t e = j ? nt::mulmod(a, ck_.galois_for_step((int64_t)j * g.stride), 2ull * ck_.ctx.n) : a;
          if (!ck_.has_rotation_key(e)) ck_.rotation_keygen(e);
        }
  for (uint32_t j = 1; j < trace_; j *= 2) {  // sparse-packing trace (and the sub-slot replication and merge)
    const uint64_t g = ck_.galois_for_full_step((int64_t)j * n_);
    if (!ck_.has_rotation_key(g)) ck_.rotation_keygen(g);
  }
  if (p_.sparse_h) ck_.sparse_keygen(p_.sparse_h);
}

std::unique_ptr<Ct> Bootstrapper::transform(std::vector<Group>& groups, std::unique_ptr<Ct> x) {
  Context& ctx = ck_.ctx;
  const uint32_t n = ctx.slots;  // diagonal vectors span the context's slots
  for (Group& g : groups) {
    const uint32_t nq = x->nq;
    require(nq >= 2, "bootstrapping ran out of levels", -4);
    // Diagonals encoded at scale level_scale(nq-1) q_{nq-1} / scale(x): after
    // the rescale the ciphertext carries exactly the FLEXIBLEAUTO scale of its
    // new level, so bootstrapped values mix with any other ciphertext there.
    const double target = ck_.level_scale(nq - 1);
    const double dscale = target * (double)ctx.primes[nq - 1] / x->scale;
    auto it = g.enc.find(nq);
    if (it != g.enc.end() && g.enc_scale[nq] != dscale) {
      g.enc.erase(it);
      it = g.enc.end();
    }
    auto encode = [&](const std::vector<std::vector<cd>>& diags) {
      std::vector<double> re, im;
      std::vector<size_t> which;
      for (size_t i = 0; i < diags.size(); ++i)
        if (!diags[i].empty()) {
          which.push_back(i);
          for (const cd& v : diags[i]) {
            re.push_back(v.real());
            im.push_back(v.imag());
          }
        }
      auto pts = ck_.encode_batch(re.data(), im.data(), (uint32_t)which.size(), n, nq, dscale);
      std::vector<std::unique_ptr<Pt>> enc(diags.size());
      for (size_t i = 0; i < which.size(); ++i) enc[which[i]] = std::move(pts[i]);
      return enc;
    };
    if (it == g.enc.end()) {
      it = g.enc.emplace(nq, encode(g.diags)).first;
      if (g.aux) g.enc2[nq] = encode(g.diags2);
      g.enc_scale[nq] = dscale;
    }
    auto ptrs = [](const std::vector<std::unique_ptr<Pt>>& enc) {
      std::vector<const Pt*> d(enc.size());
      for (size_t i = 0; i < d.size(); ++i) d[i] = enc[i].get();
      return d;
    };
    std::unique_ptr<Ct> y;
    if (!g.aux) {
      y = ck_.linear_transform(*x, ptrs(it->second), g.b, g.G, g.stride, g.offset);
    } else {
      // the companion on conj(x) or rot(x, n) shares the ModUp and the giant
      // steps: diagonals [giant][main b | companion b]
      const auto& e2 = g.enc2.at(nq);
      std::vector<const Pt*> d;
      d.reserve(2 * it->second.size());
      for (uint32_t gg = 0; gg < g.G; ++gg) {
        for (uint32_t j = 0; j < g.b; ++j) d.push_back(it->second[(size_t)gg * g.b + j].get());
        for (uint32_t j = 0; j < g.b; ++j) d.push_back(e2[(size_t)gg * g.b + j].get());
      }
      y = ck_.linear_transform(*x, d, g.b, g.G, g.stride, g.offset, aux_galois(g));
    }
    ck_.rescale_inplace(*y);
    y->scale = target;  // equal to the computed scale up to its last bit
    x = std::move(y);
  }
  return x;
}

// sin(2 pi y) for y = K u: the Chebyshev cosine at (y - 1/4) / 2^r, then r double angles.
std::unique_ptr<Ct> Bootstrapper::eval_mod(const Ct& u) {
  auto c = ck_.chebyshev(u, cheb_, -1.0, 1.0);
  for (int i = 0; i < p_.double_angles; ++i) {
    auto sq = ck_.mul(*c, *c);
    auto dbl = ck_.add(*sq, *sq, false);
    c = ck_.add_scalar(*dbl, -1.0);
  }
  return c;
}

std::unique_ptr<Ct> Bootstrapper::raise(const Ct& a) {
  Context& ctx = ck_.ctx;
  require(a.ncomp == 2, "bootstrap expects a 2-component ciphertext", -1);
  auto in = ck_.clone(a);
  if (in->noise_deg > 1 && in->nq > 1) ck_.rescale_inplace(*in);
  require(in->nq >= 2, "bootstrap input needs at least 2 limbs after its pending rescale", -4);
  // Scale the message down to q0 2^-correction on one limb (adjust records
  // exactly that scale), then raise.
  auto low = ck_.adjust(*in, 1, std::ldexp((double)ctx.primes[0], -corr_));
  in.reset();
  if (p_.sparse_h) {
    require(ck_.sparse_weight() == p_.sparse_h, "bootstrap keys for the sparse secret are missing", -4);
    low = ck_.switch_to_sparse(*low);
  }
  auto raised = ck_.mod_raise(*low);
  // The raised plaintext t = m + q0 I is fixed now; switching back to the
  // dense secret keeps it (and I) unchanged.
  if (p_.sparse_h) raised = ck_.switch_to_dense(*raised);
  // Sparse packing: sum of the rotations by j*n, j < g (log2 g doublings).
  for (uint32_t j = 1; j < trace_; j *= 2) {
    auto r = ck_.rotate(*raised, ck_.galois_for_full_step((int64_t)j * n_));
    raised = ck_.add(*raised, *r, false);
  }
  raised->scale = ck_.level_scale(ctx.L);
  levels_[0] = raised->nq;
  return raised;
}

std::unique_ptr<Ct> Bootstrapper::coeff_to_slot(const Ct& raised) {
  require(raised.nq == ck_.ctx.L, "coeff_to_slot expects a raised ciphertext", -1);
  auto x = transform(cts_, ck_.clone(raised));
  levels_[1] = x->nq;
  return x;
}

uint64_t Bootstrapper::aux_galois(const Group& g) const {
  return g.aux == 1 ? 2ull * ck_.ctx.n - 1 : ck_.galois_for_full_step((int64_t)n_);
}

std::unique_ptr<Ct> Bootstrapper::replicate(const Ct& x) {
  // copies over the context's own slots: a sparsely packed context's vector
  // already repeats with period ctx.slots over the N/2 slots of the ring
  auto r = ck_.clone(x);
  for (uint32_t j = 1; j < ck_.ctx.slots / n_; j *= 2) {
    auto t = ck_.rotate(*r, ck_.galois_for_full_step((int64_t)j * n_));
    r = ck_.add(*r, *t, false);
  }
  return r;
}

std::unique_ptr<Ct> Bootstrapper::eval_mod_full(const Ct& x) {
  if (single_) {  // the real and imaginary parts already sit side by side (2n slots)
    auto w = eval_mod(x);
    if (w->noise_deg > 1) ck_.rescale_inplace(*w);
    levels_[2] = w->nq;
    return w;
  }
  // real / imaginary split: re = x + conj(x), im = -i (x - conj(x))
  auto cj = ck_.rotate(x, 2ull * ck_.ctx.n - 1);
  auto re = ck_.add(x, *cj, false);
  auto diff = ck_.add(*cj, x, true);
  auto im = ck_.mul_i(*diff);
  cj.reset();
  diff.reset();
  auto mre = eval_mod(*re);
  auto mim = eval_mod(*im);
  re.reset();
  im.reset();
  auto imi = ck_.mul_i(*mim);
  auto w = ck_.add(*mre, *imi, false);
  if (w->noise_deg > 1) ck_.rescale_inplace(*w);
  levels_[2] = w->nq;
  return w;
}

std::unique_ptr<Ct> Bootstrapper::slot_to_coeff(const Ct& w) {
  auto y = transform(stc_, ck_.clone(w));
  levels_[3] = y->nq;
  return ck_.mul_int(*y, (int64_t)1 << corr_);
}

std::unique_ptr<Ct> Bootstrapper::bootstrap(const Ct& a) {
  ++ck_.counters.bootstraps;
  if (p_.s2c_first) {
    // SlotToCoeff first: the slots z become the plaintext's coefficients
    // (BR(z) / (2 pi) as lo + i hi); after ModRaise and CoeffToSlot the slots
    // hold z 2^-c / (2 pi) + BR(I) in their original order, and EvalMod leaves
    // z 2^-c.
    auto in = ck_.clone(a);
    if (in->noise_deg > 1 && in->nq > 1) ck_.rescale_inplace(*in);
    require(in->nq >= p_.budget_stc + 2, "S2C-first bootstrap input needs budget_stc + 2 limbs", -4);
    auto coeffs = transform(stc_, std::move(in));
    levels_[3] = coeffs->nq;
    auto raised = raise(*coeffs);
    coeffs.reset();
    auto x = coeff_to_slot(*raised);
    raised.reset();
    auto w = eval_mod_full(*x);
    return ck_.mul_int(*w, (int64_t)1 << corr_);
  }
  auto raised = raise(a);
  auto x = coeff_to_slot(*raised);
  raised.reset();
  auto w = eval_mod_full(*x);
  x.reset();
  return slot_to_coeff(*w);
}

}  // namespace fhe
