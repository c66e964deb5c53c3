// RNS-CKKS evaluator: key generation, encoding, encryption, HYBRID key
// switching, rescale, rotations and FLEXIBLEAUTO scale bookkeeping.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>

#include "ckks.h"

namespace fhe {

namespace {
typedef unsigned __int128 u128;

// Randomness streams (same definition as the CPU oracle's OC_STREAM_*).
constexpr uint64_t kStreamSecret = 1ull << 56;
constexpr uint64_t kStreamPkA = 2ull << 56;
constexpr uint64_t kStreamPkE = 3ull << 56;
inline uint64_t stream_enc(uint64_t kind, uint64_t nonce) { return (kind << 56) | (nonce & 0xFFFFFFFFFFFFFFull); }
inline uint64_t stream_key(uint64_t kind, uint64_t id, uint64_t digit) {
  return (kind << 56) | ((id & 0xFFFFFFFFFFull) << 8) | digit;
}

Shoup mk_shoup(uint64_t w, uint64_t q) { return Shoup{w, nt::shoup(w, q)}; }

LimbShoup limb_shoup(const std::vector<uint64_t>& r, const std::vector<uint64_t>& primes) {
  require(r.size() <= kMaxConstLimbs, "too many limbs for a constant product", -1);
  LimbShoup c{};
  for (size_t i = 0; i < r.size(); ++i) c.v[i] = mk_shoup(r[i], primes[i]);
  return c;
}

LimbWords limb_words(const std::vector<uint64_t>& r) {
  require(r.size() <= kMaxConstLimbs, "too many limbs for a constant sum", -1);
  LimbWords c{};
  for (size_t i = 0; i < r.size(); ++i) c.v[i] = r[i];
  return c;
}

template <class T>
DevMem upload(const std::vector<T>& v) {
  DevMem m(std::max<size_t>(v.size() * sizeof(T), 16));
  if (!v.empty()) FHE_CUDA(cudaMemcpy(m.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return m;
}
}  // namespace

Ckks::Ckks(Context& c) : ctx(c) {
  const uint32_t L = c.L;
  sf_.assign(L, 0.0);
  sf_[0] = (double)c.primes[L - 1];
  for (uint32_t k = 1; k < L; ++k) sf_[k] = sf_[k - 1] * sf_[k - 1] / (double)c.primes[L - k];
  mods_host_.resize(c.n_primes());
  FHE_CUDA(cudaMemcpy(mods_host_.data(), c.d_mod.p, mods_host_.size() * sizeof(Modulus), cudaMemcpyDeviceToHost));
  build_static_tables();
  status_ = DevMem(sizeof(unsigned));
  FHE_CUDA(cudaMemset(status_.p, 0, sizeof(unsigned)));
  stage_ring_.resize(kStageSlots);
}

Ckks::~Ckks() {
  for (StageSlot& s : stage_ring_) {
    if (s.pending) cudaEventSynchronize(s.done);
    if (s.done) cudaEventDestroy(s.done);
    if (s.host) cudaFreeHost(s.host);
  }
}

// Copies host data to device memory without blocking the host: through the
// next pinned slot of the ring, which is reused once its previous copy ran.
void Ckks::stage_upload(void* dev, const void* host, size_t bytes) {
  StageSlot& s = stage_ring_[stage_next_];
  stage_next_ = (stage_next_ + 1) % stage_ring_.size();
  if (!s.done) FHE_CUDA(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
  if (s.pending) FHE_CUDA(cudaEventSynchronize(s.done));
  s.pending = false;
  if (s.bytes < bytes) {
    if (s.host) FHE_CUDA(cudaFreeHost(s.host));
    s.host = nullptr;
    s.bytes = 0;
    const size_t want = std::max<size_t>(bytes, 4096);
    FHE_CUDA(cudaMallocHost(&s.host, want));
    s.bytes = want;
  }
  std::memcpy(s.host, host, bytes);
  FHE_CUDA(cudaMemcpyAsync(dev, s.host, bytes, cudaMemcpyHostToDevice, ctx.stream));
  FHE_CUDA(cudaEventRecord(s.done, ctx.stream));
  s.pending = true;
}

// Copies a small host table (pointers) to a device scratch buffer without
// blocking the host.
const void* Ckks::stage_pointers(const void* host, size_t bytes, size_t ws_idx) {
  uint64_t* d = ws(ws_idx, (bytes + 7) / 8);
  stage_upload(d, host, bytes);
  return d;
}

void Ckks::check_encode_status() {
  unsigned st = 0;
  FHE_CUDA(cudaMemcpyAsync(&st, status_.p, sizeof(unsigned), cudaMemcpyDeviceToHost, ctx.stream));
  FHE_CUDA(cudaStreamSynchronize(ctx.stream));
  if (st) {
    FHE_CUDA(cudaMemsetAsync(status_.p, 0, sizeof(unsigned), ctx.stream));
    FHE_CUDA(cudaStreamSynchronize(ctx.stream));
  }
  require(st == 0, "encode: a scaled value is not finite or reaches 2^126", -1);
}

namespace {

// True when the rounding kernel cannot flag these values: all finite and
// (max |re| + max |im|) * scale < 2^120.  Every coefficient of the encoding is
// bounded by the largest slot magnitude (an average of the slots times roots
// of unity), which leaves 2^6 of room below the kernel's 2^126 limit.
bool encode_in_range(const double* re, const double* im, size_t count, double scale) {
  double mr = 0.0, mi = 0.0;
  for (size_t i = 0; i < count; ++i) {
    const double a = re ? std::fabs(re[i]) : 0.0, b = im ? std::fabs(im[i]) : 0.0;
    if (!(a <= 1e300) || !(b <= 1e300)) return false;  // NaN or infinite
    mr = std::max(mr, a);
    mi = std::max(mi, b);
  }
  return std::isfinite(scale) && (mr + mi) * scale < 0x1p120;
}

}  // namespace

// Context-owned scratch buffers, reused across calls (one stream orders all use).
uint64_t* Ckks::ws(size_t idx, size_t words) {
  if (ws_.size() <= idx) ws_.resize(idx + 1);
  if (ws_[idx].bytes < words * 8) {
    FHE_CUDA(cudaStreamSynchronize(ctx.stream));
    ws_[idx] = DevMem(words * 8);
  }
  return ws_[idx].as<uint64_t>();
}

void Ckks::ntt_dense(uint64_t* d, uint32_t polys, uint32_t limbs, uint32_t stride, uint32_t prime0, bool inv) {
  if (!polys || !limbs) return;
  counters.ntt_limbs += (uint64_t)polys * limbs;
  NttArgs a = ctx.ntt_args(d, polys, prime0, limbs, stride);
  FHE_CUDA(inv ? ntt_inverse(a) : ntt_forward(a));
}

void Ckks::build_static_tables() {
  const uint32_t L = ctx.L, K = ctx.K;
  const auto& P = ctx.primes;
  std::vector<Shoup> pinv(L), pmod(L + K), qinv((size_t)L * L);
  for (uint32_t i = 0; i < L + K; ++i) {
    const uint64_t q = P[i];
    uint64_t pm = 1 % q;
    for (uint32_t k = 0; k < K; ++k) pm = nt::mulmod(pm, P[L + k] % q, q);
    pmod[i] = mk_shoup(i < L ? pm : 0, q);
    if (i < L) pinv[i] = mk_shoup(nt::invmod(pm, q), q);
  }
  for (uint32_t last = 1; last < L; ++last)
    for (uint32_t i = 0; i < last; ++i) {
      const uint64_t q = P[i];
      qinv[(size_t)last * L + i] = mk_shoup(nt::invmod(P[last] % q, q), q);
    }
  pinv_ = upload(pinv);
  pmod_ = upload(pmod);
  qinv_ = upload(qinv);
  // P -> Q conversion arrays: sources p_0..p_{K-1}, targets q_0..q_{L-1}.
  if (K) {
    std::vector<uint32_t> srcp(K), dstp(L);
    std::vector<Shoup> hatinv(K), hat((size_t)L * K);
    for (uint32_t k = 0; k < K; ++k) {
      srcp[k] = L + k;
      const uint64_t pk = P[L + k];
      uint64_t h = 1 % pk;
      for (uint32_t j = 0; j < K; ++j)
        if (j != k) h = nt::mulmod(h, P[L + j] % pk, pk);
      hatinv[k] = mk_shoup(nt::invmod(h, pk), pk);
    }
    for (uint32_t t = 0; t < L; ++t) {
      dstp[t] = t;
      const uint64_t q = P[t];
      for (uint32_t k = 0; k < K; ++k) {
        uint64_t h = 1 % q;
        for (uint32_t j = 0; j < K; ++j)
          if (j != k) h = nt::mulmod(h, P[L + j] % q, q);
        hat[(size_t)t * K + k] = mk_shoup(h, q);
      }
    }
    auto a16 = [](size_t x) { return (x + 15) & ~size_t(15); };
    const size_t b1 = a16(K * 4), b2 = a16(b1 + L * 4), b3 = b2 + K * sizeof(Shoup);
    std::vector<char> blob(b3 + hat.size() * sizeof(Shoup));
    std::memcpy(blob.data(), srcp.data(), K * 4);
    std::memcpy(blob.data() + b1, dstp.data(), L * 4);
    std::memcpy(blob.data() + b2, hatinv.data(), K * sizeof(Shoup));
    std::memcpy(blob.data() + b3, hat.data(), hat.size() * sizeof(Shoup));
    mdtab_blob_ = upload(blob);
    if (tc_conversion_supported(ctx.n, K, ctx.max_prime() < (uint64_t(1) << 60)))
      mdtab_tc_ = upload(tc_conversion_table(hat.data(), K, L));
  }
  // Special FFT twiddles: inverse in OpenFHE FFTSpecialInv order, forward in
  // FFTSpecialForward order, computed with the host C library's cos/sin.
  const uint32_t slots = ctx.slots, M = 4 * slots;
  std::vector<uint32_t> rot(slots);
  uint32_t p = 1;
  for (uint32_t j = 0; j < slots; ++j) { rot[j] = p; p = (uint32_t)((uint64_t)p * 5 % M); }
  std::vector<double2> ti(std::max(1u, slots)), tf(std::max(1u, slots));
  for (uint32_t len = 2; len <= slots; len *= 2)
    for (uint32_t j = 0; j < len / 2; ++j) {
      const uint32_t ii = (4 * len - rot[j] % (4 * len)) * (M / (4 * len));
      const double ai = 2.0 * M_PI * ii / M;
      ti[len / 2 - 1 + j] = make_double2(std::cos(ai), std::sin(ai));
      const uint32_t fi = (rot[j] % (4 * len)) * (M / (4 * len));
      const double af = 2.0 * M_PI * fi / M;
      tf[len / 2 - 1 + j] = make_double2(std::cos(af), std::sin(af));
    }
  fft_inv_tw_ = upload(ti);
  fft_fwd_tw_ = upload(tf);
}

LevelTables& Ckks::level(uint32_t nq) {
  auto it = levels_.find(nq);
  if (it != levels_.end()) return it->second;
  LevelTables& T = levels_[nq];
  const uint32_t L = ctx.L, K = ctx.K, a = ctx.alpha;
  const auto& P = ctx.primes;
  T.nq = nq;
  T.D = (nq + a - 1) / a;
  require(T.D <= 15, "more than 15 key-switching digits (the 128-bit key inner product sums at most 15)", -1);
  T.w = nq + K;
  const PrimeMap pm{nq, L};
  // One blob per level; per digit: src_prime[ns] | dst_prime[nt] | hatinv[ns] | hat[nt][ns].
  struct Off { size_t sp, dp, hi, h; uint32_t ns, nt, lo, hil; };
  std::vector<Off> offs(T.D);
  size_t cur = 0;
  auto a16 = [](size_t x) { return (x + 15) & ~size_t(15); };
  for (uint32_t j = 0; j < T.D; ++j) {
    Off& o = offs[j];
    o.lo = j * a;
    o.hil = std::min(o.lo + a, nq);
    o.ns = o.hil - o.lo;
    o.nt = T.w - o.ns;
    require(o.ns <= 24 && K <= 24, "digits or special bases of more than 24 limbs are not supported", -1);
    o.sp = cur; cur += 4 * o.ns;
    o.dp = cur; cur += 4 * o.nt;
    cur = a16(cur);
    o.hi = cur; cur += sizeof(Shoup) * o.ns;
    o.h = cur; cur += sizeof(Shoup) * o.ns * o.nt;
  }
  std::vector<char> blob(std::max<size_t>(cur, 16));
  std::vector<uint2> list;
  for (uint32_t j = 0; j < T.D; ++j) {
    const Off& o = offs[j];
    uint32_t* sp = reinterpret_cast<uint32_t*>(blob.data() + o.sp);
    uint32_t* dp = reinterpret_cast<uint32_t*>(blob.data() + o.dp);
    Shoup* hinv = reinterpret_cast<Shoup*>(blob.data() + o.hi);
    Shoup* hat = reinterpret_cast<Shoup*>(blob.data() + o.h);
    for (uint32_t i = 0; i < o.ns; ++i) {
      sp[i] = o.lo + i;
      const uint64_t qi = P[o.lo + i];
      uint64_t h = 1 % qi;
      for (uint32_t m = 0; m < o.ns; ++m)
        if (m != i) h = nt::mulmod(h, P[o.lo + m] % qi, qi);
      hinv[i] = mk_shoup(nt::invmod(h, qi), qi);
    }
    uint32_t tt = 0;
    for (uint32_t l = 0; l < T.w; ++l) {
      if (l >= o.lo && l < o.hil) continue;
      const uint32_t pr = pm(l);
      dp[tt] = pr;
      const uint64_t t = P[pr];
      for (uint32_t i = 0; i < o.ns; ++i) {
        uint64_t h = 1 % t;
        for (uint32_t m = 0; m < o.ns; ++m)
          if (m != i) h = nt::mulmod(h, P[o.lo + m] % t, t);
        hat[(size_t)tt * o.ns + i] = mk_shoup(h, t);
      }
      list.push_back(make_uint2(j * T.w + l, pr));
      ++tt;
    }
  }
  T.blob = upload(blob);
  // tensor-core operand tables of every digit, when all digits qualify
  const bool small = ctx.max_prime() < (uint64_t(1) << 60);
  T.tc_modup = true;
  for (uint32_t j = 0; j < T.D; ++j) T.tc_modup &= tc_conversion_supported(ctx.n, offs[j].ns, small);
  std::vector<size_t> tc_off(T.D, 0);
  if (T.tc_modup) {
    std::vector<uint8_t> tcb;
    for (uint32_t j = 0; j < T.D; ++j) {
      const Off& o = offs[j];
      tc_off[j] = tcb.size();
      const auto t = tc_conversion_table(reinterpret_cast<const Shoup*>(blob.data() + o.h), o.ns, o.nt);
      tcb.insert(tcb.end(), t.begin(), t.end());
    }
    T.tc_blob = upload(tcb);
  }
  std::vector<ModUpDigit> digs(T.D);
  const char* base = T.blob.as<char>();
  for (uint32_t j = 0; j < T.D; ++j) {
    const Off& o = offs[j];
    digs[j].lo = o.lo;
    digs[j].hi = o.hil;
    digs[j].conv = ConvTable{o.ns, o.nt, reinterpret_cast<const uint32_t*>(base + o.sp),
                             reinterpret_cast<const uint32_t*>(base + o.dp),
                             reinterpret_cast<const Shoup*>(base + o.hi), reinterpret_cast<const Shoup*>(base + o.h)};
    if (T.tc_modup) digs[j].conv.tc_b = T.tc_blob.as<uint8_t>() + tc_off[j];
  }
  T.digits = upload(digs);
  T.ntt_list = upload(list);
  T.ntt_list_len = (uint32_t)list.size();
  if (K) {
    const char* mb = mdtab_blob_.as<char>();
    auto a16b = [](size_t x) { return (x + 15) & ~size_t(15); };
    const size_t b1 = a16b(K * 4), b2 = a16b(b1 + L * 4), b3 = b2 + K * sizeof(Shoup);
    ConvTable md{K, nq, reinterpret_cast<const uint32_t*>(mb), reinterpret_cast<const uint32_t*>(mb + b1),
                 reinterpret_cast<const Shoup*>(mb + b2), reinterpret_cast<const Shoup*>(mb + b3)};
    md.tc_b = mdtab_tc_.as<uint8_t>();
    T.moddown = upload(std::vector<ConvTable>{md});
  }
  return T;
}

// ---------------------------------------------------------------------------
// keys

// Rotation by `step` slots: sigma_{5^e}, e = step mod slots.  With sparse
// packing (slots < N/2) every plaintext lives in the subring the rotations by
// multiples of `slots` fix, so one Galois element per residue serves every
// caller (keys asked for as -768 or 32000 are the same key).
uint64_t Ckks::galois_for_step(int64_t step) const {
  const int64_t order = (int64_t)ctx.slots;
  int64_t e = step % order;
  if (e < 0) e += order;
  return nt::powmod(5, (uint64_t)e, 2ull * ctx.n);
}

// sigma_{5^e} with e = step mod N/2 (distinct for steps that differ by a
// multiple of the slot count): the sparse-packing trace in bootstrapping.
uint64_t Ckks::galois_for_full_step(int64_t step) const {
  const int64_t order = (int64_t)(ctx.n / 2);
  int64_t e = step % order;
  if (e < 0) e += order;
  return nt::powmod(5, (uint64_t)e, 2ull * ctx.n);
}

// HYBRID switching key: digit j has a_j uniform over Q_L P and
// b_j = -a_j s_new + e_j + [l in digit j] (P mod q_l) s_old.
void Ckks::switch_keygen(uint64_t key_id, const uint64_t* s_new, const uint64_t* s_old, DevMem& out) {
  const uint32_t L = ctx.L, K = ctx.K, n = ctx.n, lk = L + K;
  const uint32_t D = (L + ctx.alpha - 1) / ctx.alpha;
  out = DevMem((size_t)D * 2 * lk * n * 8);
  uint64_t* tmp = ws(9, (size_t)lk * n);
  int64_t* e = reinterpret_cast<int64_t*>(ws(10, n));
  const Modulus* mods = ctx.d_mod.as<Modulus>();
  const uint64_t* primes = ctx.d_primes.as<uint64_t>();
  const PrimeMap full{lk, L};
  for (uint32_t j = 0; j < D; ++j) {
    uint64_t* b = out.as<uint64_t>() + (size_t)j * 2 * lk * n;
    uint64_t* a = b + (size_t)lk * n;
    launch_sample_uniform(seed_, stream_key(0x10, key_id, j), a, n, lk, full, mods, ctx.stream);
    launch_sample_small(1, seed_, stream_key(0x11, key_id, j), e, n, ctx.stream);
    launch_lift_small(e, tmp, n, lk, full, mods, ctx.stream);
    ntt_dense(tmp, 1, lk, lk, 0, false);
    launch_ew(Ew::Mul, a, 0, s_new, 0, b, 0, 1, lk, n, full, mods, ctx.stream);
    launch_ew(Ew::SubFrom, b, 0, tmp, 0, b, 0, 1, lk, n, full, mods, ctx.stream);
    const uint32_t lo = j * ctx.alpha, hi = std::min(lo + ctx.alpha, L);
    launch_mul_const(s_old + (size_t)lo * n, 0, pmod_.as<Shoup>() + lo, b + (size_t)lo * n, 0, b + (size_t)lo * n,
                     0, 1, hi - lo, n, primes + lo, ctx.stream);
  }
  FHE_CUDA(cudaGetLastError());
}

void Ckks::keygen(uint64_t seed) {
  const uint32_t L = ctx.L, K = ctx.K, n = ctx.n, lk = L + K;
  seed_ = seed;
  const Modulus* mods = ctx.d_mod.as<Modulus>();
  const uint64_t* primes = ctx.d_primes.as<uint64_t>();
  int64_t* small = reinterpret_cast<int64_t*>(ws(10, n));
  s_ntt_ = DevMem((size_t)lk * n * 8);
  launch_sample_small(0, seed, kStreamSecret, small, n, ctx.stream);
  launch_lift_small(small, s_ntt_.as<uint64_t>(), n, lk, PrimeMap{lk, L}, mods, ctx.stream);
  ntt_dense(s_ntt_.as<uint64_t>(), 1, lk, lk, 0, false);
  pk_ = DevMem((size_t)2 * L * n * 8);
  uint64_t* b = pk_.as<uint64_t>();
  uint64_t* a = b + (size_t)L * n;
  uint64_t* tmp = ws(9, (size_t)lk * n);
  const PrimeMap q{L, L};
  launch_sample_uniform(seed, kStreamPkA, a, n, L, q, mods, ctx.stream);
  launch_sample_small(1, seed, kStreamPkE, small, n, ctx.stream);
  launch_lift_small(small, tmp, n, L, q, mods, ctx.stream);
  ntt_dense(tmp, 1, L, L, 0, false);
  launch_ew(Ew::Mul, a, 0, s_ntt_.as<uint64_t>(), 0, b, 0, 1, L, n, q, mods, ctx.stream);
  launch_ew(Ew::SubFrom, b, 0, tmp, 0, b, 0, 1, L, n, q, mods, ctx.stream);
  uint64_t* s2 = ws(11, (size_t)lk * n);
  launch_ew(Ew::Mul, s_ntt_.as<uint64_t>(), 0, s_ntt_.as<uint64_t>(), 0, s2, 0, 1, lk, n, PrimeMap{lk, L}, mods,
            ctx.stream);
  switch_keygen(0, s_ntt_.as<uint64_t>(), s2, rlk_);
  rot_.clear();
  keyed_ = true;
  has_secret_ = true;
  FHE_CUDA(cudaStreamSynchronize(ctx.stream));
}

// Rotation key for Galois element g: switches s -> sigma_g^{-1}(s), so that a
// rotation is KS(c1) followed by sigma_g on (c0 + u0, u1).
void Ckks::rotation_keygen(uint64_t g) {
  require(keyed_, "rotation key generation before keygen", -4);
  require(has_secret_, "generating keys needs the secret key (this context holds evaluation keys only)", -4);
  if (rot_.count(g)) return;
  const uint32_t lk = ctx.L + ctx.K, n = ctx.n;
  const uint64_t m = 2ull * n;
  require(g % 2 == 1 && g < m, "Galois element must be odd and below 2N", -1);
  const uint64_t ginv = nt::powmod(g, n - 1, m);  // (Z/2N)^* has order N
  require((u128)g * ginv % m == 1, "internal: Galois inverse", -5);
  uint64_t* snew = ws(12, (size_t)lk * n);
  launch_automorphism(s_ntt_.as<uint64_t>(), 0, snew, 0, 1, lk, ctx.log_n, ginv, ctx.stream);
  DevMem key;
  switch_keygen(g, snew, s_ntt_.as<uint64_t>(), key);
  rot_.emplace(g, std::move(key));
  FHE_CUDA(cudaStreamSynchronize(ctx.stream));
}

// Sparse ternary secret of Hamming weight h: h distinct coefficient positions
// (Floyd's sampling) with random signs, from a splitmix64 stream keyed by the
// key seed; then the two switching keys of the encapsulation.
void Ckks::sparse_keygen(uint32_t h) {
  require(keyed_, "sparse key generation before keygen", -4);
  require(has_secret_, "generating keys needs the secret key (this context holds evaluation keys only)", -4);
  const uint32_t n = ctx.n, L = ctx.L, K = ctx.K, lk = L + K;
  require(h >= 1 && h <= n / 2, "sparse Hamming weight out of range", -1);
  if (sparse_h_ == h) return;
  uint64_t st = seed_ ^ 0x9E3779B97F4A7C15ull ^ ((uint64_t)h << 32);
  auto next = [&st]() {
    uint64_t z = (st += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  std::vector<int64_t> coef(n, 0);
  for (uint32_t j = n - h; j < n; ++j) {
    const uint32_t t = (uint32_t)(next() % (j + 1));
    const uint32_t pos = coef[t] == 0 ? t : j;
    coef[pos] = (next() & 1) ? 1 : -1;
  }
  int64_t* small = reinterpret_cast<int64_t*>(ws(10, n));
  FHE_CUDA(cudaMemcpyAsync(small, coef.data(), (size_t)n * 8, cudaMemcpyHostToDevice, ctx.stream));
  s_sparse_ = DevMem((size_t)lk * n * 8);
  launch_lift_small(small, s_sparse_.as<uint64_t>(), n, lk, PrimeMap{lk, L}, ctx.d_mod.as<Modulus>(), ctx.stream);
  ntt_dense(s_sparse_.as<uint64_t>(), 1, lk, lk, 0, false);
  const uint64_t id = 2ull * n + 1;  // beyond every Galois element and the relinearisation key
  switch_keygen(id, s_sparse_.as<uint64_t>(), s_ntt_.as<uint64_t>(), key_to_sparse_);
  switch_keygen(id + 2, s_ntt_.as<uint64_t>(), s_sparse_.as<uint64_t>(), key_to_dense_);
  FHE_CUDA(cudaStreamSynchronize(ctx.stream));
  sparse_h_ = h;
}

std::unique_ptr<Ct> Ckks::switch_with(const Ct& a, const DevMem& key) {
  require(a.ncomp == 2, "key switch expects a 2-component ciphertext", -1);
  std::unique_ptr<Ct> hold;
  const Ct& x = ready(a, hold);
  const uint32_t nq = x.nq, n = ctx.n;
  auto out = alloc(nq, 2);
  keyswitch(x.data() + (size_t)x.cap * n, nq, key.as<uint64_t>(), out->data(), (size_t)nq * n, x.data());
  out->scale = x.scale;
  out->noise_deg = x.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::switch_to_sparse(const Ct& a) {
  require(sparse_h_ != 0, "no sparse secret", -4);
  return switch_with(a, key_to_sparse_);
}

std::unique_ptr<Ct> Ckks::switch_to_dense(const Ct& a) {
  require(sparse_h_ != 0, "no sparse secret", -4);
  return switch_with(a, key_to_dense_);
}

size_t Ckks::key_words(int kind) const {
  const size_t n = ctx.n, L = ctx.L, K = ctx.K;
  const size_t D = (L + ctx.alpha - 1) / ctx.alpha;
  switch (kind) {
    case 0: case 4: return (L + K) * n;
    case 1: return 2 * L * n;
    default: return D * 2 * (L + K) * n;
  }
}

void Ckks::download_key(int kind, uint64_t g, uint64_t* host) const {
  require(keyed_, "no keys generated", -4);
  require(kind != 0 || has_secret_, "this context holds no secret key", -4);
  const DevMem* m = nullptr;
  if (kind == 0) m = &s_ntt_;
  else if (kind == 1) m = &pk_;
  else if (kind == 2) m = &rlk_;
  else if (kind >= 4 && kind <= 6) {
    require(sparse_h_ != 0, "no sparse secret", -4);
    m = kind == 4 ? &s_sparse_ : kind == 5 ? &key_to_sparse_ : &key_to_dense_;
  } else {
    auto it = rot_.find(g);
    require(it != rot_.end(), "no rotation key for Galois element " + std::to_string(g), -4);
    m = &it->second;
  }
  FHE_CUDA(cudaStreamSynchronize(ctx.stream));
  FHE_CUDA(cudaMemcpy(host, m->p, key_words(kind) * 8, cudaMemcpyDeviceToHost));
}

// ---------------------------------------------------------------------------
// encode / encrypt

std::unique_ptr<Pt> Ckks::encode(const double* re, const double* im, uint32_t count, uint32_t nq, double scale) {
  const uint32_t slots = ctx.slots, n = ctx.n;
  require(count <= slots, "more values than slots", -1);
  require(nq >= 1 && nq <= ctx.L, "limb count out of range", -1);
  std::vector<double2> v(slots, make_double2(0.0, 0.0));
  for (uint32_t i = 0; i < count; ++i) v[i] = make_double2(re ? re[i] : 0.0, im ? im[i] : 0.0);
  double2* dv = reinterpret_cast<double2*>(ws(13, 2 * (size_t)slots));
  stage_upload(dv, v.data(), slots * sizeof(double2));
  launch_fft_special_inv(dv, fft_inv_tw_.as<double2>(), slots, 1, ctx.stream);
  double* coef = reinterpret_cast<double*>(ws(14, n));
  FHE_CUDA(cudaMemsetAsync(coef, 0, (size_t)n * 8, ctx.stream));
  launch_encode_round(dv, coef, slots, n, scale, status_.as<unsigned>(), ctx.stream);
  auto p = std::make_unique<Pt>();
  p->buf = DevMem((size_t)nq * n * 8, ctx.sh);
  p->nq = nq;
  p->scale = scale;
  launch_lift_double(coef, p->data(), n, nq, PrimeMap{nq, ctx.L}, ctx.d_mod.as<Modulus>(), 1, ctx.stream);
  ntt_dense(p->data(), 1, nq, nq, 0, false);
  // values the rounding cannot reject return without waiting for the device
  if (!encode_in_range(re, im, count, scale)) check_encode_status();
  return p;
}

std::vector<std::unique_ptr<Pt>> Ckks::encode_batch(const double* re, const double* im, uint32_t B, uint32_t count,
                                                    uint32_t nq, double scale) {
  const uint32_t slots = ctx.slots, n = ctx.n;
  require(count <= slots, "more values than slots", -1);
  require(nq >= 1 && nq <= ctx.L, "limb count out of range", -1);
  std::vector<std::unique_ptr<Pt>> out;
  const uint32_t chunk = std::max(1u, std::min(B, (uint32_t)((64u << 20) / (16ull * slots))));
  std::vector<double2> v((size_t)chunk * slots);
  for (uint32_t b0 = 0; b0 < B; b0 += chunk) {
    const uint32_t nb = std::min(chunk, B - b0);
    for (uint32_t b = 0; b < nb; ++b)
      for (uint32_t i = 0; i < slots; ++i) {
        const size_t src = (size_t)(b0 + b) * count + i;
        v[(size_t)b * slots + i] =
            i < count ? make_double2(re ? re[src] : 0.0, im ? im[src] : 0.0) : make_double2(0.0, 0.0);
      }
    double2* dv = reinterpret_cast<double2*>(ws(18, 2 * (size_t)nb * slots));
    FHE_CUDA(cudaMemcpyAsync(dv, v.data(), (size_t)nb * slots * sizeof(double2), cudaMemcpyHostToDevice, ctx.stream));
    const bool in_range = encode_in_range(re ? re + (size_t)b0 * count : nullptr, im ? im + (size_t)b0 * count : nullptr,
                                          (size_t)nb * count, scale);
    encode_slots_on_device(dv, nb, nq, scale, !in_range, out);
  }
  return out;
}

// Encodes nb slot vectors already on the device (dv, [nb][slots], clobbered):
// special inverse FFT, scale and round, RNS lift, NTT; appends the plaintexts.
void Ckks::encode_slots_on_device(double2* dv, uint32_t nb, uint32_t nq, double scale, bool check,
                                  std::vector<std::unique_ptr<Pt>>& out) {
  const uint32_t slots = ctx.slots, n = ctx.n;
  launch_fft_special_inv(dv, fft_inv_tw_.as<double2>(), slots, nb, ctx.stream);
  double* coef = reinterpret_cast<double*>(ws(19, (size_t)nb * n));
  FHE_CUDA(cudaMemsetAsync(coef, 0, (size_t)nb * n * 8, ctx.stream));
  launch_encode_round_batch(dv, coef, slots, n, scale, nb, status_.as<unsigned>(), ctx.stream);
  uint64_t* res = ws(20, (size_t)nb * nq * n);
  launch_lift_double(coef, res, n, nq, PrimeMap{nq, ctx.L}, ctx.d_mod.as<Modulus>(), nb, ctx.stream);
  ntt_dense(res, nb, nq, nq, 0, false);
  for (uint32_t b = 0; b < nb; ++b) {
    auto p = std::make_unique<Pt>();
    p->buf = DevMem((size_t)nq * n * 8, ctx.sh);
    p->nq = nq;
    p->scale = scale;
    FHE_CUDA(cudaMemcpyAsync(p->data(), res + (size_t)b * nq * n, (size_t)nq * n * 8, cudaMemcpyDeviceToDevice,
                             ctx.stream));
    out.push_back(std::move(p));
  }
  // otherwise the sticky status is read at the next decode
  if (check) check_encode_status();
}

std::vector<std::unique_ptr<Pt>> Ckks::encode_replicated_diagonals(const double* w_dev, uint32_t m, uint32_t cols,
                                                                   uint32_t R, uint32_t T, uint32_t win,
                                                                   uint32_t baby, uint32_t nq, double scale) {
  const uint32_t slots = ctx.slots;
  require(w_dev != nullptr && m >= 1 && cols >= 1 && R >= 1 && T >= 1 && baby >= 1, "bad diagonal layout", -1);
  require(win >= m && (uint64_t)(R - 1) * win + m <= slots, "the windows do not fit the slots", -1);
  require(nq >= 1 && nq <= ctx.L, "limb count out of range", -1);
  std::vector<std::unique_ptr<Pt>> out;
  const uint32_t chunk = std::max(1u, std::min(T, (uint32_t)((64u << 20) / (16ull * slots))));
  for (uint32_t t0 = 0; t0 < T; t0 += chunk) {
    const uint32_t nb = std::min(chunk, T - t0);
    double2* dv = reinterpret_cast<double2*>(ws(18, 2 * (size_t)nb * slots));
    launch_replicated_diagonals(dv, w_dev, m, cols, R, T, win, baby, slots, t0, nb, ctx.stream);
    encode_slots_on_device(dv, nb, nq, scale, false, out);
  }
  return out;
}

void Ckks::decode(const Pt& p, double* re, double* im, uint32_t count) {
  const uint32_t slots = ctx.slots, n = ctx.n;
  require(count <= slots, "more values than slots", -1);
  const uint32_t nl = std::min<uint32_t>(p.nq, 2);
  uint64_t* c = ws(15, (size_t)nl * n);
  FHE_CUDA(cudaMemcpyAsync(c, p.data(), (size_t)nl * n * 8, cudaMemcpyDeviceToDevice, ctx.stream));
  ntt_dense(c, 1, nl, nl, 0, true);
  double2* dv = reinterpret_cast<double2*>(ws(13, 2 * (size_t)slots));
  const uint64_t q0 = ctx.primes[0], q1 = ctx.primes[1];
  const uint64_t q0inv = nt::invmod(q0 % q1, q1);
  launch_decode_crt(c, nl, slots, n, p.scale, q0, q1, q0inv, nt::shoup(q0inv, q1), mods_host_[1], dv, ctx.stream);
  launch_fft_special_fwd(dv, fft_fwd_tw_.as<double2>(), slots, 1, ctx.stream);
  std::vector<double2> v(slots);
  FHE_CUDA(cudaMemcpyAsync(v.data(), dv, slots * sizeof(double2), cudaMemcpyDeviceToHost, ctx.stream));
  check_encode_status();  // also waits for the copy
  for (uint32_t i = 0; i < count; ++i) {
    if (re) re[i] = v[i].x;
    if (im) im[i] = v[i].y;
  }
}

std::unique_ptr<Ct> Ckks::alloc(uint32_t nq, uint32_t ncomp) {
  auto c = std::make_unique<Ct>();
  c->buf = DevMem((size_t)ncomp * nq * ctx.n * 8, ctx.sh);
  c->cap = nq;
  c->nq = nq;
  c->ncomp = ncomp;
  return c;
}

std::unique_ptr<Ct> Ckks::clone(const Ct& a) {
  auto c = alloc(a.nq, a.ncomp);
  c->noise_deg = a.noise_deg;
  c->scale = a.scale;
  const size_t n = ctx.n;
  FHE_CUDA(cudaMemcpy2DAsync(c->data(), (size_t)c->cap * n * 8, a.data(), (size_t)a.cap * n * 8,
                             (size_t)a.nq * n * 8, a.ncomp, cudaMemcpyDeviceToDevice, ctx.stream));
  return c;
}

std::unique_ptr<Ct> Ckks::encrypt(const Pt& p) {
  require(keyed_, "encrypt before keygen", -4);
  const uint32_t nq = p.nq, n = ctx.n, L = ctx.L;
  const Modulus* mods = ctx.d_mod.as<Modulus>();
  const uint64_t* primes = ctx.d_primes.as<uint64_t>();
  const uint64_t nonce = enc_nonce++;
  int64_t* small = reinterpret_cast<int64_t*>(ws(10, n));
  uint64_t* v = ws(16, (size_t)nq * n);
  uint64_t* e = ws(17, (size_t)2 * nq * n);
  const PrimeMap q{nq, L};
  launch_sample_small(0, seed_, stream_enc(4, nonce), small, n, ctx.stream);
  launch_lift_small(small, v, n, nq, q, mods, ctx.stream);
  launch_sample_small(1, seed_, stream_enc(5, nonce), small, n, ctx.stream);
  launch_lift_small(small, e, n, nq, q, mods, ctx.stream);
  launch_sample_small(1, seed_, stream_enc(6, nonce), small, n, ctx.stream);
  launch_lift_small(small, e + (size_t)nq * n, n, nq, q, mods, ctx.stream);
  ntt_dense(v, 1, nq, nq, 0, false);
  ntt_dense(e, 2, nq, nq, 0, false);
  auto c = alloc(nq, 2);
  const size_t s = (size_t)nq * n;
  // c0 = b v + e0 + m ;  c1 = a v + e1
  launch_ew(Ew::Mul, pk_.as<uint64_t>(), (size_t)L * n, v, 0, c->data(), s, 2, nq, n, q, mods, ctx.stream);
  launch_ew(Ew::Add, c->data(), s, e, s, c->data(), s, 2, nq, n, q, mods, ctx.stream);
  launch_ew(Ew::Add, c->data(), 0, p.data(), 0, c->data(), 0, 1, nq, n, q, mods, ctx.stream);
  c->scale = p.scale;
  c->noise_deg = p.noise_deg;
  return c;
}

std::unique_ptr<Pt> Ckks::decrypt(const Ct& c) {
  require(keyed_, "decrypt before keygen", -4);
  require(has_secret_, "decryption needs the secret key (this context holds evaluation keys only)", -4);
  if (c.noise_deg >= 2 && c.nq >= 2 && c.ncomp == 2) {
    // FLEXIBLEAUTO: a degree-2 ciphertext is rescaled before decryption.
    auto t = clone(c);
    rescale_inplace(*t);
    return decrypt(*t);
  }
  const uint32_t nq = c.nq, n = ctx.n;
  const Modulus* mods = ctx.d_mod.as<Modulus>();
  const PrimeMap q{nq, ctx.L};
  auto p = std::make_unique<Pt>();
  p->buf = DevMem((size_t)nq * n * 8, ctx.sh);
  p->nq = nq;
  p->scale = c.scale;
  p->noise_deg = c.noise_deg;
  const size_t cs = (size_t)c.cap * n;
  const uint64_t* s = s_ntt_.as<uint64_t>();
  FHE_CUDA(cudaMemcpyAsync(p->data(), c.data(), (size_t)nq * n * 8, cudaMemcpyDeviceToDevice, ctx.stream));
  launch_ew(Ew::MulAdd, c.data() + cs, 0, s, 0, p->data(), 0, 1, nq, n, q, mods, ctx.stream);
  if (c.ncomp == 3) {
    uint64_t* s2 = ws(11, (size_t)(ctx.L + ctx.K) * n);
    launch_ew(Ew::Mul, s, 0, s, 0, s2, 0, 1, nq, n, q, mods, ctx.stream);
    launch_ew(Ew::MulAdd, c.data() + 2 * cs, 0, s2, 0, p->data(), 0, 1, nq, n, q, mods, ctx.stream);
  }
  return p;
}

// ---------------------------------------------------------------------------
// key switching

// Source limbs from which the tensor-core conversion is used when enabled:
// its epilogue (15 byte-shift sums per output, assembled and reduced once)
// costs the same for any source count, while the CUDA-core conversion's
// multiply-accumulates grow with it.  Measured on a B200 (relinearisation,
// N = 2^16): 7 sources 0.324 vs 0.313 ms (CUDA cores faster), 15 sources at
// 45 limbs 0.613 vs 0.703 ms (tensor cores faster).
constexpr uint32_t kTcMinSources = 12;

void Ckks::modup(const uint64_t* d, uint32_t nq, uint64_t* ext) {
  const uint32_t n = ctx.n;
  LevelTables& T = level(nq);
  uint64_t* coef = ws(1, (size_t)ctx.L * n);
  {  // coef = INTT(d), out of place
    counters.ntt_limbs += nq;
    NttArgs a = ctx.ntt_args(coef, 1, 0, nq, nq);
    a.src = d;
    a.src_limb_stride = nq;
    FHE_CUDA(ntt_inverse(a));
  }
  if (tc_conversion && T.tc_modup && (tc_conversion == 2 || ctx.alpha >= kTcMinSources))
    launch_modup_tc(coef, d, ext, nq, ctx.K, n, T.digits.as<ModUpDigit>(), T.D, ctx.alpha, ctx.d_mod.as<Modulus>(),
                    ctx.stream);
  else
    launch_modup(coef, d, ext, nq, ctx.K, n, T.digits.as<ModUpDigit>(), T.D, ctx.alpha, ctx.d_mod.as<Modulus>(),
                 ctx.stream, ctx.max_prime() < (uint64_t(1) << 60));
  ++counters.modup;
  ++counters.modup_at[Counters::slot(nq)];
  if (T.ntt_list_len) {
    counters.ntt_limbs += T.ntt_list_len;
    NttArgs a = ctx.ntt_args(ext, 1, 0, T.ntt_list_len, 0);
    a.list = T.ntt_list.as<uint2>();
    a.lazy = ctx.max_prime() < (uint64_t(1) << 60) ? 16 : 0;  // the list spans Q and P primes
    FHE_CUDA(ntt_forward(a));
  }
}

// acc = [2][w][N] (NTT form, clobbered) -> out[c] = ModDown(acc[c]) (+ add_c0 on component 0).
void Ckks::moddown_pair(uint64_t* acc, uint32_t nq, uint64_t* out, size_t so, const uint64_t* add_c0,
                        const uint64_t* ext, const uint64_t* evk) {
  const uint32_t n = ctx.n, K = ctx.K, w = nq + K;
  LevelTables& T = level(nq);
  ++counters.moddown;
  ntt_dense(acc + (size_t)nq * n, 2, K, w, ctx.L, true);
  uint64_t* conv = ws(3, (size_t)2 * ctx.L * n);
  if (tc_conversion && mdtab_tc_.as<uint8_t>() && (tc_conversion == 2 || K >= kTcMinSources))
    launch_convert_tc(acc + (size_t)nq * n, (size_t)w * n, conv, (size_t)nq * n, 2, T.moddown.as<ConvTable>(), nq,
                      n, ctx.d_mod.as<Modulus>(), ctx.stream);
  else
    launch_convert(acc + (size_t)nq * n, (size_t)w * n, conv, (size_t)nq * n, 2, T.moddown.as<ConvTable>(), K, nq,
                   n, ctx.d_mod.as<Modulus>(), ctx.stream, ctx.max_prime() < (uint64_t(1) << 60));
  // NTT of the conversion with the combine fused into its last pass:
  // out = (acc - NTT(conv)) * P^{-1} (+ c0 on component 0).
  counters.ntt_limbs += 2ull * nq;
  NttArgs a = ctx.ntt_args(conv, 2, 0, nq, nq);
  a.epi_x = acc;
  a.epi_x_comp = (size_t)w * n;
  a.epi_out = out;
  a.epi_out_comp = so;
  a.epi_w = pinv_.as<Shoup>();
  a.epi_add = add_c0;
  if (ext) {  // acc's Q rows formed in the epilogue from the digits and the key
    a.epi_ext = ext;
    a.epi_key = evk;
    a.epi_digits = T.D;
    a.epi_w_rows = w;
    a.epi_key_limbs = ctx.L + K;
    a.epi_mods = ctx.d_mod.as<Modulus>();
  }
  FHE_CUDA(ntt_forward(a));
}

void Ckks::key_moddown(const uint64_t* ext, const uint64_t* evk, uint32_t nq, uint64_t* out, size_t so,
                       const uint64_t* add_c0) {
  const uint32_t n = ctx.n, K = ctx.K, w = nq + K;
  LevelTables& T = level(nq);
  uint64_t* acc = ws(2, (size_t)2 * (ctx.L + K) * n);
  ++counters.key_inner;
  ++counters.key_inner_at[Counters::slot(nq)];
  if (fused_key_inner) {  // only the P limbs go through the accumulator
    launch_key_inner(ext, T.D, w, evk, ctx.L + K, PrimeMap{nq, ctx.L}, acc, n, ctx.d_mod.as<Modulus>(), ctx.stream,
                     nq, K);
    moddown_pair(acc, nq, out, so, add_c0, ext, evk);
  } else {
    launch_key_inner(ext, T.D, w, evk, ctx.L + K, PrimeMap{nq, ctx.L}, acc, n, ctx.d_mod.as<Modulus>(),
                     ctx.stream);
    moddown_pair(acc, nq, out, so, add_c0);
  }
}

void Ckks::keyswitch(const uint64_t* d, uint32_t nq, const uint64_t* evk, uint64_t* out, size_t so,
                     const uint64_t* add_c0) {
  const uint32_t n = ctx.n, K = ctx.K, w = nq + K;
  LevelTables& T = level(nq);
  uint64_t* ext = ws(0, (size_t)T.D * w * n);
  modup(d, nq, ext);
  key_moddown(ext, evk, nq, out, so, add_c0);
}

std::unique_ptr<Ct> Ckks::relinearize(const Ct& d) {
  require(keyed_, "relinearize before keygen", -4);
  require(d.ncomp == 3, "relinearize expects a 3-component ciphertext", -1);
  const uint32_t nq = d.nq, n = ctx.n;
  const size_t cs = (size_t)d.cap * n;
  auto out = alloc(nq, 2);
  const size_t so = (size_t)nq * n;
  ++counters.relin;
  keyswitch(d.data() + 2 * cs, nq, rlk_.as<uint64_t>(), out->data(), so, nullptr);
  launch_ew(Ew::Add, out->data(), so, d.data(), cs, out->data(), so, 2, nq, n, PrimeMap{nq, ctx.L},
            ctx.d_mod.as<Modulus>(), ctx.stream);
  out->scale = d.scale;
  out->noise_deg = d.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::rotate(const Ct& a, uint64_t g) {
  require(a.ncomp == 2, "rotate expects a 2-component ciphertext", -1);
  auto it = rot_.find(g);
  require(it != rot_.end(), "missing rotation key for Galois element " + std::to_string(g), -4);
  const uint32_t nq = a.nq, n = ctx.n;
  const size_t cs = (size_t)a.cap * n, so = (size_t)nq * n;
  uint64_t* u = ws(4, 2 * so);
  ++counters.rotations;
  keyswitch(a.data() + cs, nq, it->second.as<uint64_t>(), u, so, a.data());
  auto out = alloc(nq, 2);
  launch_automorphism(u, so, out->data(), so, 2, nq, ctx.log_n, g, ctx.stream);
  out->scale = a.scale;
  out->noise_deg = a.noise_deg;
  return out;
}

std::vector<std::unique_ptr<Ct>> Ckks::rotate_hoisted(const Ct& a, const std::vector<uint64_t>& gs) {
  require(a.ncomp == 2, "rotate expects a 2-component ciphertext", -1);
  for (uint64_t g : gs) require(rot_.count(g) != 0, "missing rotation key for Galois element " + std::to_string(g), -4);
  const uint32_t nq = a.nq, n = ctx.n, K = ctx.K, w = nq + K;
  const size_t cs = (size_t)a.cap * n, so = (size_t)nq * n;
  LevelTables& T = level(nq);
  uint64_t* ext = ws(5, (size_t)T.D * w * n);  // one ModUp shared by every rotation
  modup(a.data() + cs, nq, ext);
  std::vector<std::unique_ptr<Ct>> outs;
  uint64_t* u = ws(4, 2 * so);
  for (uint64_t g : gs) {
    ++counters.rotations;
    key_moddown(ext, rot_.at(g).as<uint64_t>(), nq, u, so, a.data());
    auto out = alloc(nq, 2);
    launch_automorphism(u, so, out->data(), so, 2, nq, ctx.log_n, g, ctx.stream);
    out->scale = a.scale;
    out->noise_deg = a.noise_deg;
    outs.push_back(std::move(out));
  }
  return outs;
}

std::unique_ptr<Ct> Ckks::linear_transform(const Ct& a_in, const std::vector<const Pt*>& diags, uint32_t b,
                                           uint32_t G, int64_t stride, int64_t giant_offset, uint64_t aux_galois) {
  require(a_in.ncomp == 2, "linear transform expects a 2-component ciphertext", -1);
  std::unique_ptr<Ct> pre;
  if (a_in.noise_deg >= 2) pre = prepare_mult_input(a_in);
  const Ct& a = pre ? *pre : a_in;
  const uint32_t nb = aux_galois ? 2 * b : b;  // babies of the dot product
  require(b >= 1 && nb <= 32 && G >= 1, "baby step must be in [1, 32] (16 with a companion), giant step >= 1", -1);
  require(diags.size() == (size_t)nb * G, "need baby*giant diagonal entries (twice that with a companion)", -1);
  require(aux_galois == 0 || (aux_galois & 1), "the companion's Galois element must be odd", -1);
  require(stride != 0, "stride must be non-zero", -1);
  const uint32_t nq = a.nq, n = ctx.n;
  double pscale = 0.0;
  for (const Pt* p : diags)
    if (p) {
      require(p->nq >= nq, "a diagonal has fewer limbs than the ciphertext", -1);
      if (pscale == 0.0) pscale = p->scale;
      require(std::fabs(p->scale / pscale - 1.0) < 1e-12, "diagonals must share one scale", -1);
    }
  require(pscale != 0.0, "every diagonal is zero", -1);
  // Babies: j = 0 is the input itself, 1..b-1 (rotations by j*stride) share one ModUp.
  std::vector<uint64_t> gs;
  for (uint32_t j = 1; j < b; ++j) gs.push_back(galois_for_step((int64_t)j * stride));
  // companion babies sigma_aux o sigma_{5^{j stride}} = sigma_{aux 5^{j stride} mod 2N}
  if (aux_galois)
    for (uint32_t j = 0; j < b; ++j)
      gs.push_back(j ? nt::mulmod(aux_galois, galois_for_step((int64_t)j * stride), 2ull * n) : aux_galois);
  auto rot = rotate_hoisted(a, gs);
  auto base = clone(a);  // cap == nq, component stride nq*N like the rotations
  std::vector<const uint64_t*> tab{base->data()};
  for (auto& r : rot) tab.push_back(r->data());
  for (size_t i = 0; i < diags.size(); ++i) tab.push_back(diags[i] ? diags[i]->data() : nullptr);
  const uint64_t* const* d_tab =
      static_cast<const uint64_t* const*>(stage_pointers(tab.data(), tab.size() * sizeof(void*), 23));
  const size_t cs = (size_t)nq * n;
  uint64_t* inner = ws(21, (size_t)G * 2 * cs);
  launch_bsgs_dot(d_tab, d_tab + nb, inner, nb, G, nq, n, ctx.d_mod.as<Modulus>(), ctx.stream);
  auto out = alloc(nq, 2);
  out->scale = a.scale * pscale;
  out->noise_deg = a.noise_deg + 1;
  const PrimeMap pm{nq, ctx.L};
  uint32_t rotating = 0;
  for (uint32_t g = 0; g < G; ++g) rotating += galois_for_step(((int64_t)g * b - giant_offset) * stride) != 1;
  if (hoist_giant_moddown && rotating >= 2) {
    // sum_g sigma_g(KS(c1_g)) = ModDown(sum_g sigma_g(inner_g)) + sum_g sigma_g(c0_g):
    // the key inner products accumulate in the extended basis (Q and P limbs)
    const uint32_t K = ctx.K, w = nq + K;
    LevelTables& T = level(nq);
    uint64_t* ext = ws(0, (size_t)T.D * w * n);
    uint64_t* acc = ws(2, (size_t)2 * (ctx.L + K) * n);   // one giant's inner product [2][w][N]
    uint64_t* sum = ws(25, (size_t)2 * w * n);            // their automorphisms summed [2][w][N]
    uint64_t* c0 = ws(26, cs);                            // sum of sigma_g(c0_g) [nq][N]
    uint64_t* t = ws(27, (size_t)2 * w * n);              // one permuted inner product
    const PrimeMap pe{nq, ctx.L};                         // extended limbs: Q then P primes
    bool first = true, first_id = true;
    for (uint32_t g = 0; g < G; ++g) {
      const uint64_t* ig = inner + (size_t)g * 2 * cs;
      const int64_t amount = ((int64_t)g * b - giant_offset) * stride;
      const uint64_t gal = galois_for_step(amount);
      if (gal == 1) {  // the identity giant joins the output directly
        if (first_id)
          FHE_CUDA(cudaMemcpyAsync(out->data(), ig, 2 * cs * 8, cudaMemcpyDeviceToDevice, ctx.stream));
        else
          launch_ew(Ew::Add, out->data(), cs, ig, cs, out->data(), cs, 2, nq, n, pm, ctx.d_mod.as<Modulus>(),
                    ctx.stream);
        first_id = false;
        continue;
      }
      auto it = rot_.find(gal);
      require(it != rot_.end(), "missing rotation key for giant step " + std::to_string(amount), -4);
      ++counters.rotations;
      modup(ig + cs, nq, ext);
      ++counters.key_inner;
      ++counters.key_inner_at[Counters::slot(nq)];
      launch_key_inner(ext, T.D, w, it->second.as<uint64_t>(), ctx.L + K, pe, acc, n, ctx.d_mod.as<Modulus>(),
                       ctx.stream);
      if (first) {
        launch_automorphism(acc, (size_t)w * n, sum, (size_t)w * n, 2, w, ctx.log_n, gal, ctx.stream);
        launch_automorphism(ig, cs, c0, cs, 1, nq, ctx.log_n, gal, ctx.stream);
      } else {
        launch_automorphism(acc, (size_t)w * n, t, (size_t)w * n, 2, w, ctx.log_n, gal, ctx.stream);
        launch_ew(Ew::Add, sum, (size_t)w * n, t, (size_t)w * n, sum, (size_t)w * n, 2, w, n, pe,
                  ctx.d_mod.as<Modulus>(), ctx.stream);
        launch_automorphism(ig, cs, t, cs, 1, nq, ctx.log_n, gal, ctx.stream);
        launch_ew(Ew::Add, c0, cs, t, cs, c0, cs, 1, nq, n, pm, ctx.d_mod.as<Modulus>(), ctx.stream);
      }
      first = false;
    }
    uint64_t* u = ws(4, 2 * cs);
    moddown_pair(sum, nq, u, cs, c0);
    if (first_id)
      FHE_CUDA(cudaMemcpyAsync(out->data(), u, 2 * cs * 8, cudaMemcpyDeviceToDevice, ctx.stream));
    else
      launch_ew(Ew::Add, out->data(), cs, u, cs, out->data(), cs, 2, nq, n, pm, ctx.d_mod.as<Modulus>(),
                ctx.stream);
    return out;
  }
  for (uint32_t g = 0; g < G; ++g) {
    const uint64_t* ig = inner + (size_t)g * 2 * cs;
    const int64_t amount = ((int64_t)g * b - giant_offset) * stride;
    const uint64_t gal = galois_for_step(amount);
    const uint64_t* term = ig;
    if (gal != 1) {  // rotation by a non-zero amount: key switch, then automorphism
      auto it = rot_.find(gal);
      require(it != rot_.end(), "missing rotation key for giant step " + std::to_string(amount), -4);
      uint64_t* u = ws(4, 2 * cs);
      ++counters.rotations;
      keyswitch(ig + cs, nq, it->second.as<uint64_t>(), u, cs, ig);
      uint64_t* r = ws(22, 2 * cs);
      launch_automorphism(u, cs, r, cs, 2, nq, ctx.log_n, gal, ctx.stream);
      term = r;
    }
    if (g == 0)
      FHE_CUDA(cudaMemcpyAsync(out->data(), term, 2 * cs * 8, cudaMemcpyDeviceToDevice, ctx.stream));
    else
      launch_ew(Ew::Add, out->data(), cs, term, cs, out->data(), cs, 2, nq, n, pm, ctx.d_mod.as<Modulus>(),
                ctx.stream);
  }
  return out;
}

std::unique_ptr<Ct> Ckks::mod_raise(const Ct& a) {
  require(a.ncomp == 2, "mod_raise expects a 2-component ciphertext", -1);
  const uint32_t n = ctx.n, L = ctx.L;
  const size_t cs = (size_t)a.cap * n;
  // coefficients of limb 0 of both components
  uint64_t* c0 = ws(6, 2 * (size_t)n);
  FHE_CUDA(cudaMemcpy2DAsync(c0, (size_t)n * 8, a.data(), cs * 8, (size_t)n * 8, 2, cudaMemcpyDeviceToDevice,
                             ctx.stream));
  ntt_dense(c0, 2, 1, 1, 0, true);
  auto out = alloc(L, 2);
  launch_rescale_lift(c0, n, out->data(), (size_t)L * n, 2, L, n, ctx.primes[0], ctx.d_mod.as<Modulus>(),
                      ctx.stream);
  ntt_dense(out->data(), 2, L, L, 0, false);
  out->scale = a.scale;
  out->noise_deg = 1;
  return out;
}

std::unique_ptr<Ct> Ckks::mul_i(const Ct& a) {
  auto out = alloc(a.nq, a.ncomp);
  launch_mul_monomial_half(a.data(), (size_t)a.cap * ctx.n, out->data(), (size_t)a.nq * ctx.n, a.ncomp, a.nq, ctx.n,
                           ctx.d_tw.as<Twiddle>(), ctx.d_primes.as<uint64_t>(), ctx.stream);
  out->scale = a.scale;
  out->noise_deg = a.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::chebyshev(const Ct& x, const std::vector<double>& coeffs, double lo, double hi) {
  require(!coeffs.empty(), "no Chebyshev coefficients", -1);
  require(hi > lo, "empty Chebyshev interval", -1);
  // u = x * 2/(hi-lo) - (lo+hi)/(hi-lo); no level is spent when [lo, hi] = [-1, 1].
  std::unique_ptr<Ct> u;
  if (lo == -1.0 && hi == 1.0) {
    u = clone(x);
  } else {
    u = mul_scalar(x, 2.0 / (hi - lo));
    u = add_scalar(*u, -(lo + hi) / (hi - lo));
  }
  if (u->noise_deg >= 2 && u->nq >= 2) rescale_inplace(*u);  // once, not at every use of T_1
  std::map<int, std::unique_ptr<Ct>> cache;
  int levels = 0;
  while ((1 << levels) < (int)coeffs.size()) ++levels;
  const int baby = 1 << ((std::max(1, levels) + 1) / 2);
  // T_i brought down to (nq, scale), cached: odd products and the leaf basis
  // ask for the same lowered copies.
  std::map<std::pair<int, uint32_t>, std::unique_ptr<Ct>> lowered;
  std::function<const Ct&(int)> basis;
  auto at_level = [&](int i, uint32_t nq, double sc) -> const Ct& {
    const Ct& b = basis(i);
    if (b.nq == nq) return b;
    auto& slot = lowered[{i, nq}];
    if (!slot) slot = adjust(b, nq, sc);
    return *slot;
  };
  // Each T_i is rescaled once, right after its product, and reused in that
  // form (a lazily rescaled T_i would be rescaled again at every use).
  basis = [&](int i) -> const Ct& {
    if (i == 1) return *u;
    auto it = cache.find(i);
    if (it != cache.end()) return *it->second;
    std::unique_ptr<Ct> out;
    if (i % 2 == 0) {
      const Ct& h = basis(i / 2);
      auto sq = mul(h, h);
      auto dbl = add(*sq, *sq, false);
      out = add_scalar(*dbl, -1.0);
    } else {
      const Ct* a = &basis((i + 1) / 2);
      const Ct* b = &basis(i / 2);
      if (a->nq > b->nq) a = &at_level((i + 1) / 2, b->nq, b->scale);
      else if (b->nq > a->nq) b = &at_level(i / 2, a->nq, a->scale);
      auto pr = mul(*a, *b);
      auto dbl = add(*pr, *pr, false);
      out = add(*dbl, *u, true);
    }
    if (out->noise_deg >= 2 && out->nq >= 2) rescale_inplace(*out);
    const Ct& ref = *out;
    cache[i] = std::move(out);
    return ref;
  };
  // Leaf polynomials (degree < baby) are weighted sums of T_1..T_{baby-1}; the
  // basis is brought once to the level and scale of its deepest member and
  // each leaf is then one fused pass (linear_wsum) instead of a scalar product,
  // an addition and a level alignment per term.
  std::vector<const Ct*> aligned;
  auto aligned_basis = [&](int i) -> const Ct& {
    if (aligned.empty()) {
      const int top = std::min<int>(baby - 1, (int)coeffs.size() - 1);
      uint32_t nq_min = ~0u;
      double sc = 0.0;
      for (int j = 1; j <= top; ++j) {
        const Ct& b = basis(j);
        require(b.noise_deg < 2, "chebyshev: basis left unrescaled", -5);
        if (b.nq < nq_min) {
          nq_min = b.nq;
          sc = b.scale;
        }
      }
      aligned.assign(top + 1, nullptr);
      for (int j = 1; j <= top; ++j) {
        const Ct& b = basis(j);
        if (b.nq == nq_min) require(std::fabs(b.scale / sc - 1.0) < 1e-9, "chebyshev: basis scales differ on one level", -4);
        aligned[j] = &at_level(j, nq_min, sc);
      }
    }
    return *aligned[i];
  };
  std::function<std::unique_ptr<Ct>(std::vector<double>)> evaluate =
      [&](std::vector<double> c) -> std::unique_ptr<Ct> {
    const int degree = (int)c.size() - 1;
    if (degree < baby) {
      std::vector<const Ct*> xs;
      std::vector<double> ws_;
      for (int i = 1; i <= degree; ++i) {
        if (c[i] == 0.0) continue;
        xs.push_back(&aligned_basis(i));
        ws_.push_back(c[i]);
      }
      if (xs.empty()) {
        xs.push_back(&aligned_basis(1));
        ws_.push_back(0.0);
      }
      return linear_wsum(xs, ws_, c[0]);
    }
    int k = baby;
    while (2 * k - 1 < degree) k *= 2;
    std::vector<double> upper(c.begin() + k, c.end()), lower(c.begin(), c.begin() + k);
    for (size_t i = 1; i < upper.size(); ++i) upper[i] *= 2;
    for (int i = k + 1; i <= degree; ++i) lower[2 * k - i] -= c[i];
    auto lo_part = evaluate(lower);
    auto up_part = evaluate(upper);
    auto prod = mul(basis(k), *up_part);
    return add(*lo_part, *prod, false);
  };
  return evaluate(coeffs);
}

// ---------------------------------------------------------------------------
// arithmetic

std::unique_ptr<Ct> Ckks::tensor(const Ct& a, const Ct& b) {
  require(a.ncomp == 2 && b.ncomp == 2, "tensor expects 2-component ciphertexts", -1);
  require(a.nq == b.nq, "tensor operands must have the same number of limbs", -1);
  const uint32_t nq = a.nq, n = ctx.n;
  auto d = alloc(nq, 3);
  ++counters.tensor;
  ++counters.tensor_at[Counters::slot(nq)];
  launch_tensor(a.data(), (size_t)a.cap * n, b.data(), (size_t)b.cap * n, d->data(), (size_t)nq * n, nq, n,
                ctx.d_mod.as<Modulus>(), ctx.stream);
  d->scale = a.scale * b.scale;
  d->noise_deg = a.noise_deg + b.noise_deg;
  return d;
}

// OpenFHE DropLastElementAndScale: x_i <- (x_i - [lift(x_last)]_{q_i}) q_last^{-1}.
void Ckks::rescale_inplace(Ct& a) { rescale_into(a, a); }

std::unique_ptr<Ct> Ckks::rescaled(const Ct& a) {
  require(a.nq >= 2, "rescale: no limb left to drop (level underflow)", -4);
  auto out = alloc(a.nq - 1, a.ncomp);
  rescale_into(a, *out);
  return out;
}

// OpenFHE DropLastElementAndScale from `a` into `o` (o may be a itself, or a
// buffer with >= a.nq - 1 limbs per component).
void Ckks::rescale_into(const Ct& a, Ct& o) {
  require(a.nq >= 2, "rescale: no limb left to drop (level underflow)", -4);
  const uint32_t nq = a.nq, n = ctx.n, nc = a.ncomp;
  const size_t cs = (size_t)a.cap * n, os = (size_t)o.cap * n;
  ++counters.rescales;
  ++counters.rescale_at[Counters::slot(nq)];
  uint64_t* last = ws(6, (size_t)nc * n);
  {  // last[c] = INTT(limb nq-1 of component c), out of place
    counters.ntt_limbs += nc;
    NttArgs la = ctx.ntt_args(last, nc, nq - 1, 1, 1);
    la.src = a.data() + (size_t)(nq - 1) * n;
    la.src_limb_stride = a.cap;
    FHE_CUDA(ntt_inverse(la));
  }
  uint64_t* lifted = ws(7, (size_t)nc * (nq - 1) * n);
  const size_t ls = (size_t)(nq - 1) * n;
  launch_rescale_lift(last, n, lifted, ls, nc, nq - 1, n, ctx.primes[nq - 1], ctx.d_mod.as<Modulus>(), ctx.stream);
  // (measured: fusing this combine into the NTT's last pass, as ModDown does,
  // is 5% slower here; the separate combine streams at full bandwidth)
  ntt_dense(lifted, nc, nq - 1, nq - 1, 0, false);
  launch_moddown_combine(a.data(), cs, lifted, ls, qinv_.as<Shoup>() + (size_t)(nq - 1) * ctx.L, nullptr, o.data(),
                         os, nc, nq - 1, n, ctx.d_primes.as<uint64_t>(), ctx.stream);
  o.scale = a.scale / (double)ctx.primes[nq - 1];
  o.nq = nq - 1;
  o.ncomp = nc;
  o.noise_deg = a.noise_deg > 1 ? a.noise_deg - 1 : 1;
}

void Ckks::level_reduce_inplace(Ct& a, uint32_t levels) {
  require(levels < a.nq, "level reduce would drop every limb", -4);
  a.nq -= levels;
}

std::vector<uint64_t> Ckks::scalar_residues(long double v, uint32_t nq) const {
  const long double r = roundl(v);
  const bool neg = r < 0;
  const long double mag = neg ? -r : r;
  require(mag < 1.7e38L, "scalar constant too large", -1);
  const long double two64 = 18446744073709551616.0L;
  const uint64_t hi = (uint64_t)(mag / two64);
  const uint64_t lo = (uint64_t)(mag - (long double)hi * two64);
  std::vector<uint64_t> out(nq);
  for (uint32_t i = 0; i < nq; ++i) {
    const uint64_t q = ctx.primes[i];
    const uint64_t x = (uint64_t)((((u128)hi << 64) | lo) % q);
    out[i] = neg && x ? q - x : x;
  }
  return out;
}

std::unique_ptr<Ct> Ckks::mul_int(const Ct& a, int64_t v) {
  const LimbShoup c = limb_shoup(scalar_residues((long double)v, a.nq), ctx.primes);
  auto out = alloc(a.nq, a.ncomp);
  launch_mul_const_v(a.data(), (size_t)a.cap * ctx.n, c, out->data(), (size_t)a.nq * ctx.n, a.ncomp, a.nq, ctx.n,
                     ctx.d_primes.as<uint64_t>(), ctx.stream);
  out->scale = a.scale;
  out->noise_deg = a.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::adjust(const Ct& a, uint32_t nq, double scale) {
  require(nq <= a.nq, "adjust: target level is above the ciphertext", -1);
  // Every branch writes a new ciphertext (a rescale or an integer multiple);
  // the input is copied only for a pure limb drop or a scale relabel.
  std::unique_ptr<Ct> c;
  if (a.noise_deg == 2 && a.nq > nq) c = rescaled(a);
  const Ct* cur = c ? c.get() : &a;
  if (cur->scale != scale) {
    // Either times round(scale * q_last / s) and a rescale (consumes the
    // level being dropped anyway), or, when the target carries a squared
    // scale, multiply by round(scale / s) and drop limbs.  FLEXIBLEAUTO
    // scales of neighbouring levels can agree to 1e-12, so "nearly equal" is
    // not "equal": any difference is removed exactly when a level is dropped.
    const long double C = cur->nq > nq
                              ? (long double)scale * (long double)ctx.primes[cur->nq - 1] / (long double)cur->scale
                              : 0.0L;
    if (C >= 1.0L && C < 9.2e18L) {
      auto m = mul_int(*cur, (int64_t)roundl(C));
      m->noise_deg = cur->noise_deg + 1;
      rescale_inplace(*m);
      m->scale = scale;
      c = std::move(m);
    } else if (cur->nq == nq && std::fabs(cur->scale / scale - 1.0) < 1e-9) {
      if (!c) c = clone(*cur);
      c->scale = scale;  // one level, one scale up to rounding of the scale itself
    } else {
      const long double R = (long double)scale / (long double)cur->scale;
      require(R >= 1.0L && R < 4.6e18L, "adjust: scale ratio out of range", -4);
      auto m = mul_int(*cur, (int64_t)roundl(R));  // limb-wise: equal to dropping first
      m->noise_deg = cur->noise_deg + 1;
      m->scale = scale;
      c = std::move(m);
    }
  }
  if (!c) c = clone(*cur);
  if (c->nq > nq) level_reduce_inplace(*c, c->nq - nq);
  return c;
}

std::unique_ptr<Ct> Ckks::add(const Ct& a, const Ct& b, bool subtract) {
  require(a.ncomp == b.ncomp, "add: component counts differ", -1);
  const Ct* x = &a;
  const Ct* y = &b;
  std::unique_ptr<Ct> tx, ty;
  // scales that agree to 1e-9 are one FLEXIBLEAUTO scale up to the rounding
  // of its own computation
  const bool same_scale = std::fabs(a.scale / b.scale - 1.0) <= 1e-9;
  if (a.nq != b.nq) {
    // FLEXIBLEAUTO level alignment: the operand with more limbs is brought to
    // the other's level and scale.
    if (a.nq > b.nq) { tx = adjust(a, b.nq, b.scale); x = tx.get(); }
    else { ty = adjust(b, a.nq, a.scale); y = ty.get(); }
  } else if (!same_scale) {
    // Same level, different scale (degree 1 + degree 2): raise the smaller
    // scale by an exact integer multiple.
    const bool a_small = a.scale < b.scale;
    const Ct& sm = a_small ? a : b;
    const Ct& bg = a_small ? b : a;
    const long double C = (long double)bg.scale / (long double)sm.scale;
    require(C >= 1.0L && C < 4.6e18L, "add: scale ratio out of range", -4);
    // An integer multiple reconciles the scales only when the ratio is large
    // (degree 1 + degree 2) or integral; anything else would silently add
    // values at different scales.
    require(C >= 0x1p30L || fabsl(C - roundl(C)) <= 1e-9L * C,
            "add: operands on one level carry different scales that are not integer multiples", -4);
    auto m = mul_int(sm, (int64_t)roundl(C));
    m->scale = bg.scale;
    m->noise_deg = bg.noise_deg;
    if (a_small) { tx = std::move(m); x = tx.get(); } else { ty = std::move(m); y = ty.get(); }
  }
  const uint32_t nq = std::min(x->nq, y->nq), n = ctx.n;
  auto out = alloc(nq, a.ncomp);
  launch_ew(subtract ? Ew::Sub : Ew::Add, x->data(), (size_t)x->cap * n, y->data(), (size_t)y->cap * n, out->data(),
            (size_t)nq * n, a.ncomp, nq, n, PrimeMap{nq, ctx.L}, ctx.d_mod.as<Modulus>(), ctx.stream);
  out->scale = x->scale;
  out->noise_deg = std::max(x->noise_deg, y->noise_deg);
  return out;
}

std::unique_ptr<Ct> Ckks::negate(const Ct& a) {
  const uint32_t n = ctx.n;
  auto out = alloc(a.nq, a.ncomp);
  launch_ew(Ew::Neg, a.data(), (size_t)a.cap * n, a.data(), (size_t)a.cap * n, out->data(), (size_t)a.nq * n, a.ncomp,
            a.nq, n, PrimeMap{a.nq, ctx.L}, ctx.d_mod.as<Modulus>(), ctx.stream);
  out->scale = a.scale;
  out->noise_deg = a.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::add_plain(const Ct& a, const Pt& p, bool subtract) {
  require(p.nq >= a.nq, "add_plain: plaintext has fewer limbs than the ciphertext", -1);
  require(std::fabs(a.scale / p.scale - 1.0) < 1e-9, "add_plain: scale mismatch", -4);
  auto out = clone(a);
  launch_ew(subtract ? Ew::Sub : Ew::Add, out->data(), 0, p.data(), 0, out->data(), 0, 1, a.nq, ctx.n,
            PrimeMap{a.nq, ctx.L}, ctx.d_mod.as<Modulus>(), ctx.stream);
  return out;
}

std::unique_ptr<Ct> Ckks::mul_plain(const Ct& a_in, const Pt& p) {
  // FLEXIBLEAUTO: a pending rescale happens before the product.
  std::unique_ptr<Ct> pre;
  if (a_in.noise_deg >= 2) pre = prepare_mult_input(a_in);
  const Ct& a = pre ? *pre : a_in;
  require(p.nq >= a.nq, "mul_plain: plaintext has fewer limbs than the ciphertext", -1);
  const uint32_t n = ctx.n;
  auto out = alloc(a.nq, a.ncomp);
  launch_ew(Ew::Mul, a.data(), (size_t)a.cap * n, p.data(), 0, out->data(), (size_t)a.nq * n, a.ncomp, a.nq, n,
            PrimeMap{a.nq, ctx.L}, ctx.d_mod.as<Modulus>(), ctx.stream);
  out->scale = a.scale * p.scale;
  out->noise_deg = a.noise_deg + p.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::add_scalar(const Ct& a, double v) {
  const LimbWords c = limb_words(scalar_residues((long double)v * (long double)a.scale, a.nq));
  auto out = alloc(a.nq, a.ncomp);
  launch_add_const_v(a.data(), (size_t)a.cap * ctx.n, c, out->data(), (size_t)a.nq * ctx.n, a.ncomp, a.nq, ctx.n,
                     ctx.d_primes.as<uint64_t>(), ctx.stream);
  out->scale = a.scale;
  out->noise_deg = a.noise_deg;
  return out;
}

std::unique_ptr<Ct> Ckks::prepare_mult_input(const Ct& a) {
  if (a.noise_deg >= 2) return rescaled(a);
  return clone(a);
}

const Ct& Ckks::ready(const Ct& a, std::unique_ptr<Ct>& hold) {
  if (a.noise_deg < 2) return a;
  hold = rescaled(a);
  return *hold;
}

std::unique_ptr<Ct> Ckks::mul_scalar(const Ct& a, double v) {
  std::unique_ptr<Ct> hold;
  const Ct& c = ready(a, hold);
  const double sf = level_scale(c.nq);
  const LimbShoup k = limb_shoup(scalar_residues((long double)v * (long double)sf, c.nq), ctx.primes);
  auto out = alloc(c.nq, c.ncomp);
  launch_mul_const_v(c.data(), (size_t)c.cap * ctx.n, k, out->data(), (size_t)c.nq * ctx.n, c.ncomp, c.nq, ctx.n,
                     ctx.d_primes.as<uint64_t>(), ctx.stream);
  out->scale = c.scale * sf;
  out->noise_deg = c.noise_deg + 1;
  return out;
}

std::unique_ptr<Ct> Ckks::linear_wsum(const std::vector<const Ct*>& xs, const std::vector<double>& w, double c0) {
  require(!xs.empty() && xs.size() == w.size() && xs.size() <= kMaxWsum, "linear_wsum: 1..32 terms", -1);
  const Ct& x0 = *xs[0];
  const uint32_t nq = x0.nq, nc = x0.ncomp;
  for (const Ct* x : xs)
    require(x->nq == nq && x->ncomp == nc && x->noise_deg == x0.noise_deg &&
                std::fabs(x->scale / x0.scale - 1.0) < 1e-9,
            "linear_wsum: terms must share level, scale and degree (limbs " + std::to_string(x->nq) + "/" +
                std::to_string(nq) + ", degree " + std::to_string(x->noise_deg) + "/" +
                std::to_string(x0.noise_deg) + ", scale ratio " + std::to_string(x->scale / x0.scale) + ")",
            -4);
  const double sf = level_scale(nq);
  WsumArgs args{};
  std::vector<uint64_t> wt((size_t)xs.size() * nq);
  for (size_t i = 0; i < xs.size(); ++i) {
    args.x[i] = xs[i]->data();
    args.stride[i] = (uint64_t)xs[i]->cap * ctx.n;
    const auto r = scalar_residues((long double)w[i] * (long double)sf, nq);
    std::copy(r.begin(), r.end(), wt.begin() + i * nq);
  }
  const uint64_t* dw =
      static_cast<const uint64_t*>(stage_pointers(wt.data(), wt.size() * sizeof(uint64_t), 24));
  const double out_scale = x0.scale * sf;
  const LimbWords add = limb_words(scalar_residues((long double)c0 * (long double)out_scale, nq));
  auto out = alloc(nq, nc);
  launch_linear_wsum(args, (uint32_t)xs.size(), dw, add, c0 != 0.0, out->data(), (size_t)nq * ctx.n, nc, nq, ctx.n,
                     ctx.d_mod.as<Modulus>(), ctx.stream);
  out->scale = out_scale;
  out->noise_deg = x0.noise_deg + 1;
  return out;
}

std::unique_ptr<Ct> Ckks::mul(const Ct& a, const Ct& b) {
  require(keyed_, "mul before keygen", -4);
  std::unique_ptr<Ct> hx, hy;
  const Ct* x = &ready(a, hx);
  const Ct* y = &b == &a ? x : &ready(b, hy);  // a square rescales its operand once
  // FLEXIBLEAUTO level alignment (AdjustLevelsAndDepth): the operand with more
  // limbs is brought to the other's level AND scale, so that ciphertexts on one
  // level keep one scale; dropping limbs alone would leave a nearby but
  // different scale that later additions cannot reconcile exactly.
  if (x->nq > y->nq) {
    hx = adjust(*x, y->nq, y->scale);
    x = hx.get();
  }
  if (y->nq > x->nq) {
    hy = adjust(*y, x->nq, x->scale);
    y = hy.get();
  }
  auto d = tensor(*x, *y);
  auto out = relinearize(*d);
  return out;
}

}  // namespace fhe
