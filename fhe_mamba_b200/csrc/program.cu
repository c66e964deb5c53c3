// Packed-program executor (see program.h).
#include "program.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <fstream>
#include <iostream>
#include <set>

namespace fhe {
namespace {

using Clock = std::chrono::steady_clock;
double since(Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); }

constexpr int kMaxNodes = 1000000;

bool pow2(long long v) { return v > 0 && (v & (v - 1)) == 0; }
bool integral(double v) { return v == std::floor(v); }

}  // namespace

// ---------------------------------------------------------------------------
// reader: the same admission rules as the reference's read_packed_program

PackedProgram read_packed_program(std::istream& in) {
  PackedProgram p;
  std::string magic;
  int n_nodes = 0, n_outputs = 0;
  if (!(in >> magic >> p.slots >> p.bound >> n_nodes >> n_outputs))
    throw Error(-1, "invalid packed program header");
  if (magic == "fhemamba-packed-v1") p.version = 1;
  else if (magic == "fhemamba-packed-v2") p.version = 2;
  else throw Error(-1, "invalid packed program header");
  require(p.slots >= 2 && p.slots <= 32768 && pow2(p.slots) && std::isfinite(p.bound) && p.bound > 0 &&
              n_nodes >= 1 && n_nodes <= kMaxNodes && n_outputs >= 1 && n_outputs <= n_nodes,
          "invalid packed program header");
  p.nodes.reserve(n_nodes);
  for (int i = 0; i < n_nodes; ++i) {
    PackedNode nd;
    int parents = 0, count = 0;
    if (!(in >> nd.op >> nd.size)) throw Error(-1, "invalid packed node");
    nd.bound = p.bound;
    if (p.version == 2 && (!(in >> nd.bound) || !std::isfinite(nd.bound) || nd.bound <= 0 || nd.bound > p.bound))
      throw Error(-1, "invalid node refresh bound");
    if (!(in >> parents) || nd.size < 1 || nd.size > p.slots || parents < 0 || parents > 2)
      throw Error(-1, "invalid packed node");
    for (int j = 0; j < parents; ++j) {
      int q = -1;
      if (!(in >> q) || q < 0 || q >= i) throw Error(-1, "invalid packed dependency");
      nd.parents.push_back(q);
    }
    if (!(in >> count) || count < 0 || (long long)count > (long long)p.slots * p.slots)
      throw Error(-1, "invalid packed data size");
    nd.data.resize(count);
    for (int j = 0; j < count; ++j)
      if (!(in >> nd.data[j]) || !std::isfinite(nd.data[j])) throw Error(-1, "invalid packed constant");
    const std::string& op = nd.op;
    const bool source = op == "input" || op == "public";
    const bool binary = op == "add" || op == "mul";
    if (parents != (source ? 0 : binary ? 2 : 1)) throw Error(-1, "wrong operand count");
    const int in_size = source ? 0 : p.nodes[nd.parents[0]].size;
    bool ok = false;
    if (source) ok = count == nd.size;
    else if (binary) ok = count == 0 && in_size == nd.size && p.nodes[nd.parents[1]].size == nd.size;
    else if (op == "addp" || op == "mulp") ok = count == nd.size && in_size == nd.size;
    else if (op == "linear") ok = (long long)count == (long long)nd.size * in_size;
    else if (op == "feedback" && p.version == 2) ok = count == 0 && nd.size == in_size;
    else if (op == "linear_ref" && p.version == 2) {
      ok = count == 1 && nd.data[0] >= 0 && nd.data[0] < i && integral(nd.data[0]);
      if (ok) {
        const PackedNode& w = p.nodes[(int)nd.data[0]];
        ok = w.op == "linear" && w.size == nd.size && (long long)w.data.size() == (long long)nd.size * in_size;
      }
    } else if (op == "repeat") {
      ok = count == 3;
      for (double v : nd.data) ok = ok && v >= 1 && v <= p.slots && integral(v);
      if (ok) {
        const int rep = (int)nd.data[2];
        ok = (p.version == 2 || pow2(rep)) && nd.data[0] * nd.data[1] == in_size && (long long)in_size * rep == nd.size;
      }
    } else if (op == "cheb") {
      ok = count >= 4 && count <= 1027 && nd.data[0] < nd.data[1] && in_size == nd.size;
    } else if (op == "sum") {
      ok = count == 1 && nd.data[0] >= 1 && integral(nd.data[0]) && nd.data[0] <= p.slots &&
           pow2((long long)nd.data[0]) && (long long)nd.size * (long long)nd.data[0] == in_size;
    } else if (op == "gather" || op == "scatter") {
      const bool g = op == "gather";
      ok = count == (g ? nd.size : in_size);
      const int limit = g ? in_size : nd.size;
      std::vector<bool> seen(p.slots, false);
      for (double v : nd.data) {
        if (v < 0 || v >= limit || !integral(v)) ok = false;
        else if (!g) {
          if (seen[(int)v]) ok = false;
          seen[(int)v] = true;
        }
      }
    }
    if (!ok) throw Error(-1, "invalid packed operation: " + op);
    p.nodes.push_back(std::move(nd));
  }
  for (int i = 0; i < n_outputs; ++i) {
    PackedOutput o;
    int size = 0;
    if (!(in >> o.node >> size) || o.node < 0 || o.node >= n_nodes || size != p.nodes[o.node].size)
      throw Error(-1, "invalid packed output");
    for (auto* v : {&o.polynomial, &o.exact}) {
      v->resize(size);
      for (int j = 0; j < size; ++j)
        if (!(in >> (*v)[j]) || !std::isfinite((*v)[j])) throw Error(-1, "invalid packed reference");
    }
    p.outputs.push_back(std::move(o));
  }
  std::string tail;
  if (in >> tail) throw Error(-1, "trailing packed program data");
  return p;
}

OutputErrors packed_output_errors(const std::vector<double>& values, const PackedOutput& ref) {
  require(values.size() >= ref.polynomial.size() && ref.exact.size() == ref.polynomial.size(),
          "packed output/reference width mismatch");
  OutputErrors e;
  for (size_t j = 0; j < ref.polynomial.size(); ++j) {
    if (!std::isfinite(values[j]) || !std::isfinite(ref.polynomial[j]) || !std::isfinite(ref.exact[j])) {
      ++e.non_finite;
      continue;
    }
    e.polynomial = std::max(e.polynomial, std::fabs(values[j] - ref.polynomial[j]));
    e.exact = std::max(e.exact, std::fabs(values[j] - ref.exact[j]));
  }
  return e;
}

void GenerationClient::load(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  in.read(reinterpret_cast<char*>(&vocab), sizeof(vocab));
  in.read(reinterpret_cast<char*>(&width), sizeof(width));
  require(in && vocab >= 2 && vocab <= 262144 && width >= 1 && width <= 8192 &&
              (uint64_t)vocab * width <= 268435456ull,
          "invalid client vocabulary head");
  weights.resize((size_t)vocab * width);
  in.read(reinterpret_cast<char*>(weights.data()), weights.size() * sizeof(float));
  require(in && in.peek() == std::char_traits<char>::eof(), "invalid client head length");
  for (float v : weights) require(std::isfinite(v), "nonfinite client head");
}

std::vector<double> GenerationClient::select(const std::vector<double>& hidden) {
  require(hidden.size() >= width, "client hidden width mismatch");
  for (uint32_t j = 0; j < width; ++j) require(std::isfinite(hidden[j]), "nonfinite client output", -4);
  int best = -1;
  double first = -INFINITY, second = -INFINITY;
  for (uint32_t t = 0; t < vocab; ++t) {
    double logit = 0;
    const float* w = weights.data() + (size_t)t * width;
    for (uint32_t j = 0; j < width; ++j) logit += hidden[j] * w[j];
    if (logit > first) {
      second = first;
      first = logit;
      best = (int)t;
    } else if (logit > second) {
      second = logit;
    }
  }
  tokens.push_back(best);
  margins.push_back(first - second);
  const float* row = weights.data() + (size_t)best * width;
  return std::vector<double>(row, row + width);
}

// ---------------------------------------------------------------------------
// executor

PackedExecutor::PackedExecutor(Ckks& ck, Bootstrapper* boot, const PackedProgram& program,
                               const ExecutorOptions& opt)
    : ck_(ck), boot_(boot), p_(program), opt_(opt), slots_(ck.ctx.slots) {
  require((uint32_t)program.slots <= slots_, "program slots exceed the context's slots", -1);
  refresh_ceiling = (int)ck.ctx.L - 1 - opt.refresh_margin;
}

std::unique_ptr<Ct> PackedExecutor::encrypt(const std::vector<double>& values) {
  require(values.size() <= slots_, "value wider than the slots", -1);
  const uint32_t L = ck_.ctx.L;
  auto pt = ck_.encode(values.data(), nullptr, (uint32_t)values.size(), L, ck_.level_scale(L));
  return ck_.encrypt(*pt);
}

std::vector<double> PackedExecutor::decrypt(const Ct& c, int count) {
  auto pt = ck_.decrypt(c);
  std::vector<double> re(count);
  ck_.decode(*pt, re.data(), nullptr, (uint32_t)count);
  return re;
}

std::unique_ptr<Ct> PackedExecutor::scale(const Ct& a, double c) {
  ++ct_pt;
  return ck_.mul_scalar(a, c);
}

std::unique_ptr<Ct> PackedExecutor::add(const Ct& a, const Ct& b, bool subtract) {
  ++adds;
  return ck_.add(a, b, subtract);
}

// The reference's plain(): a public slot vector multiplied into (encoded at the
// level the product happens on, after a pending rescale) or added to (encoded
// at the ciphertext's own level and scale) a ciphertext.
std::unique_ptr<Ct> PackedExecutor::plain(const Ct& a, std::vector<double> values, bool multiply) {
  values.resize(slots_, 0.0);
  if (multiply) {
    ++ct_pt;
    const uint32_t nq = a.noise_deg >= 2 ? a.nq - 1 : a.nq;
    auto pt = ck_.encode(values.data(), nullptr, slots_, nq, ck_.level_scale(nq));
    return ck_.mul_plain(a, *pt);
  }
  ++adds;
  std::unique_ptr<Ct> hold;
  const Ct* x = &a;
  if (a.noise_deg >= 2) {
    hold = ck_.rescaled(a);
    x = hold.get();
  }
  auto pt = ck_.encode(values.data(), nullptr, slots_, x->nq, x->scale);
  return ck_.add_plain(*x, *pt, false);
}

bool PackedExecutor::ensure_key(int step) {
  const uint64_t g = ck_.galois_for_step(step);
  if (g == 1 || ck_.has_rotation_key(g)) return true;
  if (rotation_keys_generated >= opt_.max_rotation_keys) return false;
  const auto t = Clock::now();
  ck_.rotation_keygen(g);
  keygen_seconds += since(t);
  ++rotation_keys_generated;
  return true;
}

std::unique_ptr<Ct> PackedExecutor::rotate(const Ct& a, int offset) {
  const int n = (int)slots_;
  int r = ((offset % n) + n) % n;
  if (r > n / 2) r -= n;
  if (r == 0) return ck_.clone(a);
  if (ensure_key(r)) {
    ++rotations;
    return ck_.rotate(a, ck_.galois_for_step(r));
  }
  // signed binary decomposition over power-of-two keys
  std::unique_ptr<Ct> out;
  const int sign = r < 0 ? -1 : 1;
  for (int bits = std::abs(r), pw = 1; bits; bits >>= 1, pw <<= 1) {
    if (!(bits & 1)) continue;
    require(ensure_key(sign * pw) || ck_.has_rotation_key(ck_.galois_for_step(sign * pw)),
            "rotation key budget exhausted", -4);
    ++rotations;
    out = ck_.rotate(out ? *out : a, ck_.galois_for_step(sign * pw));
  }
  return out;
}

std::vector<std::unique_ptr<Ct>> PackedExecutor::rotate_many(const Ct& a, const std::vector<int>& offsets) {
  std::vector<std::unique_ptr<Ct>> out(offsets.size());
  std::vector<uint64_t> gs;
  std::vector<size_t> where;
  for (size_t i = 0; i < offsets.size(); ++i) {
    const int n = (int)slots_;
    int r = ((offsets[i] % n) + n) % n;
    if (r > n / 2) r -= n;
    if (r == 0) {
      out[i] = ck_.clone(a);
    } else if (ensure_key(r)) {
      gs.push_back(ck_.galois_for_step(r));
      where.push_back(i);
    } else {
      out[i] = rotate(a, r);
    }
  }
  if (!gs.empty()) {
    auto rs = ck_.rotate_hoisted(a, gs);
    rotations += (long long)gs.size();
    for (size_t k = 0; k < rs.size(); ++k) out[where[k]] = std::move(rs[k]);
  }
  return out;
}

// Diagonal transform out = sum_d masks[d] (.) rot(x, d).  Few diagonals: hoisted
// rotations and plaintext products; many: one BSGS transform over their range.
std::unique_ptr<Ct> PackedExecutor::transform(const Ct& x, const std::map<int, std::vector<double>>& masks) {
  if (masks.empty()) return scale(x, 0.0);
  if (masks.size() > 32) return bsgs(x, masks);
  std::vector<int> offsets;
  for (const auto& [d, m] : masks) offsets.push_back(d);
  auto rots = rotate_many(x, offsets);
  std::unique_ptr<Ct> out;
  size_t i = 0;
  for (const auto& [d, m] : masks) {
    auto term = plain(*rots[i++], m, true);
    out = out ? add(*out, *term) : std::move(term);
  }
  return out;
}

std::unique_ptr<Ct> PackedExecutor::bsgs(const Ct& x_in, const std::map<int, std::vector<double>>& masks) {
  std::unique_ptr<Ct> hold;
  const Ct* xp = &x_in;
  if (x_in.noise_deg >= 2) {
    hold = ck_.rescaled(x_in);
    xp = hold.get();
  }
  const Ct& x = *xp;
  const int n = (int)slots_;
  const int dmin = masks.begin()->first, dmax = masks.rbegin()->first;
  const int range = dmax - dmin + 1;
  uint32_t b = 1;
  while ((int)(b * b) < range && b < 32) b *= 2;
  const int off = dmin < 0 ? (int)(((-dmin) + b - 1) / b * b) : 0;
  const int G = (dmax + off) / (int)b + 1;
  // encode at most ~4 GiB of diagonals at a time; each chunk of giants is its
  // own linear transform (the babies are recomputed per chunk)
  const size_t pt_bytes = (size_t)x.nq * ck_.ctx.n * 8;
  const int per_chunk = std::max<int>(1, (int)std::min<size_t>((size_t)G, (4ull << 30) / (pt_bytes * b)));
  const double sc = ck_.level_scale(x.nq);
  std::unique_ptr<Ct> out;
  for (int g0 = 0; g0 < G; g0 += per_chunk) {
    const int Gc = std::min(per_chunk, G - g0);
    std::vector<double> vals;
    std::vector<int> which;
    for (int g = g0; g < g0 + Gc; ++g)
      for (uint32_t j = 0; j < b; ++j) {
        const int t = g * (int)b + (int)j - off;
        auto it = masks.find(t);
        if (it == masks.end()) continue;
        const int r = (((g * (int)b - off) % n) + n) % n;  // pre-rotate by the giant amount
        const auto& m = it->second;
        const size_t base = vals.size();
        vals.resize(base + n, 0.0);
        for (int i = 0; i < n; ++i) vals[base + i] = m[(i - r + n) % n];
        which.push_back((g - g0) * (int)b + (int)j);
      }
    if (which.empty()) continue;
    for (uint32_t j = 1; j < b; ++j) ensure_key((int)j);
    for (int g = g0; g < g0 + Gc; ++g) ensure_key(g * (int)b - off);
    auto pts = ck_.encode_batch(vals.data(), nullptr, (uint32_t)which.size(), (uint32_t)n, x.nq, sc);
    std::vector<const Pt*> diags((size_t)b * Gc, nullptr);
    for (size_t k = 0; k < which.size(); ++k) diags[which[k]] = pts[k].get();
    ct_pt += (long long)which.size();
    rotations += (long long)(b - 1) + Gc;
    auto part = ck_.linear_transform(x, diags, b, (uint32_t)Gc, 1, (int64_t)off - (int64_t)g0 * b);
    out = out ? add(*out, *part) : std::move(part);
  }
  return out ? std::move(out) : scale(x, 0.0);
}

std::unique_ptr<Ct> PackedExecutor::gather(const Ct& x, const std::vector<double>& indices, int size, bool scatter) {
  (void)size;
  const int m = (int)indices.size();
  bool identity = true, monotone = true;
  for (int i = 0; i < m; ++i) {
    identity = identity && indices[i] == i;
    monotone = monotone && (i == 0 || indices[i] > indices[i - 1]);
  }
  if (scatter && identity) return ck_.clone(x);
  std::map<int, std::vector<double>> masks;
  for (int i = 0; i < m; ++i) {
    const int src = scatter ? i : (int)indices[i];
    const int dst = scatter ? (int)indices[i] : i;
    auto& mk = masks[src - dst];
    if (mk.empty()) mk.assign(slots_, 0.0);
    mk[dst] = 1.0;
  }
  if (masks.size() <= 32 || !monotone) return transform(x, masks);
  // Monotone compaction / expansion: route every coordinate by the bits of its
  // displacement (ascending bits for compaction, descending for expansion), one
  // masked rotation per bit; live coordinates never collide.
  std::vector<int> pos(m), dist(m);
  std::vector<double> selected(slots_, 0.0);
  int maximum = 0;
  for (int i = 0; i < m; ++i) {
    pos[i] = scatter ? i : (int)indices[i];
    dist[i] = (int)indices[i] - i;
    selected[pos[i]] = 1.0;
    maximum = std::max(maximum, dist[i]);
  }
  auto out = plain(x, selected, true);
  std::vector<int> shifts;
  for (int s = 1; s <= maximum; s *= 2) shifts.push_back(s);
  if (scatter) std::reverse(shifts.begin(), shifts.end());
  for (int s : shifts) {
    std::vector<double> moving_mask(slots_, 0.0);
    bool any = false;
    for (int i = 0; i < m; ++i)
      if (dist[i] & s) {
        any = true;
        moving_mask[pos[i]] = 1.0;
        pos[i] += scatter ? s : -s;
      }
    if (!any) continue;
    if (level(*out) + 3 > refresh_ceiling) out = refresh(*out, p_.bound);
    auto moving = plain(*out, moving_mask, true);
    auto rest = add(*out, *moving, true);
    auto moved = rotate(*moving, scatter ? -s : s);
    out = add(*rest, *moved);
  }
  return out;
}

std::unique_ptr<Ct> PackedExecutor::linear(const Ct& x, const PackedNode& w, int columns) {
  std::map<int, std::vector<double>> masks;
  for (int i = 0; i < w.size; ++i)
    for (int j = 0; j < columns; ++j) {
      const double v = w.data[(size_t)i * columns + j];
      if (v == 0.0) continue;
      auto& mk = masks[j - i];
      if (mk.empty()) mk.assign(slots_, 0.0);
      mk[i] = v;
    }
  return transform(x, masks);
}

std::unique_ptr<Ct> PackedExecutor::chebyshev(const Ct& x, const PackedNode& nd) {
  const double lo = nd.data[0], hi = nd.data[1];
  std::vector<double> affine(slots_, 0.0), bias(slots_, 0.0), mask(slots_, 0.0);
  for (int i = 0; i < nd.size; ++i) {
    affine[i] = 2.0 / (hi - lo);
    bias[i] = -(lo + hi) / (hi - lo);
    mask[i] = 1.0;
  }
  // zero-padded normalised arguments keep every inactive slot at 0, inside [-1, 1]
  auto u = plain(*plain(x, affine, true), bias, false);
  const std::vector<double> coeffs(nd.data.begin() + 2, nd.data.end());
  auto p = ck_.chebyshev(*u, coeffs, -1.0, 1.0);
  return plain(*p, mask, true);
}

// sum_{r < count} rot(input, r * stride) by the reference's doubling schedule
// (stage1_mamba2_plan.cpp rotation_sum_schedule).
std::unique_ptr<Ct> PackedExecutor::rotation_sum(const Ct& input, int count, int stride) {
  struct Step {
    int offset;
    bool accumulated;
  };
  std::vector<Step> steps;
  int bit = 1;
  while (bit <= count / 2) bit *= 2;
  int filled = 1;
  for (bit /= 2; bit > 0; bit /= 2) {
    steps.push_back({filled, true});
    filled *= 2;
    if (count & bit) {
      steps.push_back({filled, false});
      ++filled;
    }
  }
  auto sum = ck_.clone(input);
  for (const Step& s : steps) {
    auto r = rotate(s.accumulated ? *sum : input, s.offset * stride);
    sum = add(*sum, *r);
  }
  return sum;
}

// PackedEvaluator::refresh / bootstrap_components (packed_fideslib.cpp:235-281),
// baseline form: bootstrap x / bound; with two passes the residual
// (x/bound - first) * 4096 is bootstrapped again and added back / 4096.
std::unique_ptr<Ct> PackedExecutor::refresh(const Ct& value, double bound) {
  require(boot_ != nullptr, "a refresh is needed but bootstrapping is not set up", -4);
  const auto t0 = Clock::now();
  ++logical_refreshes;
  auto x = scale(value, 1.0 / bound);
  if (x->noise_deg > 1) x = ck_.rescaled(*x);
  auto first = boot_->bootstrap(*x);
  ++bootstraps;
  std::unique_ptr<Ct> out;
  if (opt_.bootstrap_passes == 1) {
    out = scale(*first, bound);
  } else {
    auto residual = scale(*add(*x, *first, true), 4096.0);
    if (residual->noise_deg > 1) residual = ck_.rescaled(*residual);
    auto second = boot_->bootstrap(*residual);
    ++bootstraps;
    auto corr = scale(*second, 1.0 / 4096.0);
    out = scale(*add(*first, *corr), bound);
  }
  if (out->noise_deg > 1) out = ck_.rescaled(*out);
  refreshed_level = std::max(refreshed_level, level(*out));
  bootstrap_seconds += since(t0);
  return out;
}

std::vector<std::unique_ptr<Ct>> PackedExecutor::evaluate() {
  const auto& nodes = p_.nodes;
  const int nn = (int)nodes.size();
  std::vector<int> last(nn, -1);
  for (int i = 0; i < nn; ++i)
    for (int q : nodes[i].parents) last[q] = i;
  std::vector<bool> pinned(nn, false);
  for (const auto& o : p_.outputs) pinned[o.node] = true;
  std::vector<std::unique_ptr<Ct>> values(nn);
  for (int i = 0; i < nn; ++i) {
    const PackedNode& nd = nodes[i];
    const std::string& op = nd.op;
    const auto t0 = Clock::now();
    const double boot0 = bootstrap_seconds;
    const long long nb0 = bootstraps;
    int need = 3;
    if (op == "cheb") {
      int lg = 0;
      while ((1 << lg) < (int)nd.data.size() - 2) ++lg;
      need = lg + 5;
    }
    for (int q : nd.parents)
      if (op != "feedback" && level(*values[q]) + need > refresh_ceiling) {
        // never bootstrap unmasked coordinates beyond the value's width
        std::vector<double> mask(nodes[q].size, 1.0);
        auto clean = plain(*values[q], mask, true);
        values[q] = refresh(*clean, nodes[q].bound);
      }
    const Ct* x = nd.parents.empty() ? nullptr : values[nd.parents[0]].get();
    std::unique_ptr<Ct> out;
    if (op == "input" || op == "public") {
      out = encrypt(nd.data);
    } else if (op == "feedback") {
      require((bool)client_feedback, "client feedback requires --client-head", -4);
      out = client_feedback(*x);
    } else if (op == "add") {
      out = add(*x, *values[nd.parents[1]]);
    } else if (op == "mul") {
      ++ct_ct;
      out = ck_.mul(*x, *values[nd.parents[1]]);
    } else if (op == "addp" || op == "mulp") {
      out = plain(*x, nd.data, op == "mulp");
    } else if (op == "gather" || op == "scatter") {
      out = gather(*x, nd.data, nd.size, op == "scatter");
    } else if (op == "linear" || op == "linear_ref") {
      const PackedNode& w = op == "linear" ? nd : nodes[(int)nd.data[0]];
      out = linear(*x, w, nodes[nd.parents[0]].size);
    } else if (op == "cheb") {
      out = chebyshev(*x, nd);
    } else if (op == "repeat") {
      const int outer = (int)nd.data[0], inner = (int)nd.data[1], rep = (int)nd.data[2];
      std::vector<double> dest((size_t)outer * inner);
      for (int g = 0; g < outer; ++g)
        for (int j = 0; j < inner; ++j) dest[(size_t)g * inner + j] = (double)g * inner * rep + j;
      auto spread = gather(*x, dest, nd.size, true);
      out = rotation_sum(*spread, rep, -inner);
    } else if (op == "sum") {
      const int width = (int)nd.data[0];
      auto acc = ck_.clone(*x);
      for (int s = 1; s < width; s *= 2) {
        auto r = rotate(*acc, s);
        acc = add(*acc, *r);
      }
      std::vector<double> idx(nd.size);
      for (int j = 0; j < nd.size; ++j) idx[j] = (double)j * width;
      out = gather(*acc, idx, nd.size, false);
    } else {
      throw Error(-1, "unsupported packed operation: " + op);
    }
    if (opt_.trace)
      std::cout << "level_output node=" << i << " op=" << op << " level=" << level(*out)
                << " degree=" << out->noise_deg << std::endl;
    values[i] = std::move(out);
    for (int q : nd.parents)
      if (last[q] == i && !pinned[q]) values[q].reset();
    auto& st = operation_stats[op];
    ++st.nodes;
    st.seconds += since(t0);
    st.bootstrap_seconds += bootstrap_seconds - boot0;
    st.bootstraps += bootstraps - nb0;
  }
  std::vector<std::unique_ptr<Ct>> outs;
  for (const auto& o : p_.outputs) outs.push_back(ck_.clone(*values[o.node]));
  return outs;
}

}  // namespace fhe
