// Limb-sharded HYBRID key switching (see shard.h for the data flow).
#include "shard.h"

#include <algorithm>
#include <cstring>

#include "ckks_kernels.h"
#include "launch_count.h"

namespace fhe {
namespace {

constexpr uint32_t kThreads = 256;

// acc[c][l] = sum_j ext[j][l] * key[j][c][krow(l)] mod q_{row_prime[l]}
// (the single-GPU key inner product restricted to the own extended rows).
__global__ void k_key_inner_rows(const uint64_t* ext, uint32_t D, uint32_t rows, const uint64_t* key,
                                 uint32_t key_rows, PrimeMap krow, const uint32_t* row_prime, uint64_t* acc,
                                 uint32_t n, const Modulus* mods) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y;
  const Modulus m = mods[row_prime[l]];
  const uint32_t kr = krow(l);
  uint64_t h0 = 0, l0 = 0, h1 = 0, l1 = 0;
  for (uint32_t j = 0; j < D; ++j) {
    const uint64_t x = ext[((size_t)j * rows + l) * n + k];
    const uint64_t* kb = key + (size_t)j * 2 * key_rows * n;
    const uint64_t k0 = kb[(size_t)kr * n + k], k1 = kb[((size_t)key_rows + kr) * n + k];
    const uint64_t p0 = x * k0, p1 = x * k1;
    l0 += p0;
    h0 += __umul64hi(x, k0) + (l0 < p0);
    l1 += p1;
    h1 += __umul64hi(x, k1) + (l1 < p1);
  }
  acc[(size_t)l * n + k] = reduce_u128(h0, l0, m);
  acc[((size_t)rows + l) * n + k] = reduce_u128(h1, l1, m);
}

// out[c][l] = (acc[c][l] - conv[c][l]) * P^{-1} mod q_l  (+ add_c[l]).
__global__ void k_combine_rows(const uint64_t* acc, uint32_t rows, const uint64_t* conv, uint32_t q_own,
                               const Shoup* pinv, const uint64_t* qs, const uint64_t* add0, const uint64_t* add1,
                               uint64_t* out, uint32_t n) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const uint32_t l = blockIdx.y, c = blockIdx.z;
  const uint64_t q = qs[l];
  const size_t off = (size_t)l * n + k;
  const Shoup w = pinv[l];
  uint64_t r = shoup_mul(sub_mod(acc[(size_t)c * rows * n + off], conv[(size_t)c * q_own * n + off], q), w.w, w.wp, q);
  const uint64_t* add = c == 0 ? add0 : add1;
  if (add) r = add_mod(r, add[off], q);
  out[(size_t)c * q_own * n + off] = r;
}

Shoup mk(uint64_t w, uint64_t q) { return Shoup{w, nt::shoup(w, q)}; }

}  // namespace

ShardKeySwitch::ShardKeySwitch(Ckks& ck, uint32_t r, uint32_t w) : rank(r), world(w), ck_(ck) {
  require(w >= 1 && r < w, "shard rank must be below the world size", -1);
  require(ck.has_keys(), "sharded key switching needs keys (keygen first)", -4);
  qa_full_ = q_own(ck.ctx.L);
  pa_ = ck.ctx.K > rank ? (ck.ctx.K - 1 - rank) / world + 1 : 0;
}

ShardPlan ShardKeySwitch::plan(uint32_t nq) const {
  const Context& c = ck_.ctx;
  require(nq >= 1 && nq <= c.L, "limb count out of range", -1);
  ShardPlan p;
  p.nq = nq;
  p.q_own = q_own(nq);
  p.q_chunk = (nq + world - 1) / world;
  p.p_own = pa_;
  p.p_chunk = (c.K + world - 1) / world;
  p.rows = p.q_own + p.p_own;
  p.digits = (nq + c.alpha - 1) / c.alpha;
  return p;
}

uint64_t ShardKeySwitch::key_id(int kind, uint64_t g) const { return kind == 2 ? 0 : g; }

void ShardKeySwitch::load_key(int kind, uint64_t g) {
  require(kind == 2 || kind == 3, "shard keys are relinearisation (2) or rotation (3) keys", -1);
  const uint64_t id = key_id(kind, g);
  if (keys_.count(id)) return;
  const Context& c = ck_.ctx;
  const uint32_t L = c.L, K = c.K, n = c.n, lk = L + K;
  const uint32_t D = (L + c.alpha - 1) / c.alpha, kr = qa_full_ + pa_;
  const DevMem* full;
  if (kind == 2) {
    full = &ck_.rlk_;
  } else {
    if (!ck_.has_rotation_key(g)) ck_.rotation_keygen(g);
    full = &ck_.rot_.at(g);
  }
  DevMem own((size_t)D * 2 * kr * n * 8);
  for (uint32_t j = 0; j < D; ++j)
    for (uint32_t comp = 0; comp < 2; ++comp) {
      const uint64_t* src = full->as<uint64_t>() + ((size_t)j * 2 + comp) * lk * n;
      uint64_t* dst = own.as<uint64_t>() + ((size_t)j * 2 + comp) * kr * n;
      // rows l = rank + i*W: one strided 2-D copy per (digit, component) and basis
      if (qa_full_)
        FHE_CUDA(cudaMemcpy2DAsync(dst, (size_t)n * 8, src + (size_t)rank * n, (size_t)world * n * 8,
                                   (size_t)n * 8, qa_full_, cudaMemcpyDeviceToDevice, c.stream));
      if (pa_)
        FHE_CUDA(cudaMemcpy2DAsync(dst + (size_t)qa_full_ * n, (size_t)n * 8, src + (size_t)(L + rank) * n,
                                   (size_t)world * n * 8, (size_t)n * 8, pa_, cudaMemcpyDeviceToDevice, c.stream));
    }
  FHE_CUDA(cudaStreamSynchronize(c.stream));
  keys_.emplace(id, std::move(own));
}

ShardKeySwitch::Level& ShardKeySwitch::level(uint32_t nq) {
  auto it = levels_.find(nq);
  if (it != levels_.end()) return it->second;
  const Context& c = ck_.ctx;
  const auto& P = c.primes;
  const uint32_t L = c.L, K = c.K, a = c.alpha, W = world;
  Level T;
  T.pl = plan(nq);
  const ShardPlan& pl = T.pl;
  require(a <= 24 && K <= 24, "digits or special bases of more than 24 limbs are not supported", -1);
  // Own extended rows: Q limbs rank + i W (i < q_own), then P limbs rank + i W (i < p_own).
  std::vector<uint32_t> row_prime(pl.rows);
  for (uint32_t i = 0; i < pl.q_own; ++i) row_prime[i] = rank + i * W;
  for (uint32_t i = 0; i < pl.p_own; ++i) row_prime[pl.q_own + i] = L + rank + i * W;

  // Host images of every table, packed into one blob with 16-byte alignment.
  std::vector<char> blob;
  auto put = [&blob](const void* src, size_t bytes) {
    const size_t off = (blob.size() + 15) & ~size_t(15);
    blob.resize(off + std::max<size_t>(bytes, 16));
    if (bytes) std::memcpy(blob.data() + off, src, bytes);
    return off;
  };
  struct Tab { size_t sp, dp, sr, dr, hi, h, srs; uint32_t ns, nt; };
  // Per-digit exchange: digit j's own rows of every rank, padded to dchunk
  // rows, gathered into [W][dchunk][N]; limb l of digit j at row
  // (l % W) * dchunk + (index of l among rank l % W's limbs of the digit).
  const uint32_t dchunk = (a + W - 1) / W;
  T.dchunk = dchunk;
  std::vector<Tab> dig(pl.digits);
  std::vector<uint2> ext_list;
  T.digit_ns.resize(pl.digits);
  T.digit_nt.resize(pl.digits);
  T.digit_own_lo.resize(pl.digits);
  T.digit_own_hi.resize(pl.digits);
  for (uint32_t j = 0; j < pl.digits; ++j) {
    const uint32_t lo = j * a, hi = std::min(lo + a, nq), ns = hi - lo;
    std::vector<uint32_t> sp(ns), sr(ns), srs(ns), dp, dr;
    std::vector<Shoup> hinv(ns), hat;
    for (uint32_t i = 0; i < ns; ++i) {
      const uint32_t l = lo + i;
      sp[i] = l;
      sr[i] = (l % W) * pl.q_chunk + l / W;
      const uint32_t first = lo + (l % W + W - lo % W) % W;  // rank l % W's first limb of the digit
      srs[i] = (l % W) * dchunk + (l - first) / W;
      const uint64_t qi = P[l];
      uint64_t h = 1 % qi;
      for (uint32_t m = lo; m < hi; ++m)
        if (m != l) h = nt::mulmod(h, P[m] % qi, qi);
      hinv[i] = mk(nt::invmod(h, qi), qi);
    }
    uint32_t own_lo = pl.q_own, own_hi = 0;
    for (uint32_t r = 0; r < pl.rows; ++r) {
      const uint32_t pr = row_prime[r];
      if (pr >= lo && pr < hi) {  // the digit's own limb: copied from d in NTT form
        own_lo = std::min(own_lo, r);
        own_hi = std::max(own_hi, r + 1);
        continue;
      }
      dp.push_back(pr);
      dr.push_back(r);
      const uint64_t t = P[pr];
      for (uint32_t i = 0; i < ns; ++i) {
        uint64_t h = 1 % t;
        for (uint32_t m = lo; m < hi; ++m)
          if (m != lo + i) h = nt::mulmod(h, P[m] % t, t);
        hat.push_back(mk(h, t));
      }
      ext_list.push_back(make_uint2(j * pl.rows + r, pr));
    }
    if (own_lo >= own_hi) own_lo = own_hi = 0;
    T.digit_ns[j] = ns;
    T.digit_nt[j] = (uint32_t)dp.size();
    T.digit_own_lo[j] = own_lo;
    T.digit_own_hi[j] = own_hi;
    Tab& tb = dig[j];
    tb.ns = ns;
    tb.nt = (uint32_t)dp.size();
    tb.sp = put(sp.data(), sp.size() * 4);
    tb.dp = put(dp.data(), dp.size() * 4);
    tb.sr = put(sr.data(), sr.size() * 4);
    tb.srs = put(srs.data(), srs.size() * 4);
    tb.dr = put(dr.data(), dr.size() * 4);
    tb.hi = put(hinv.data(), hinv.size() * sizeof(Shoup));
    tb.h = put(hat.data(), hat.size() * sizeof(Shoup));
  }
  // ModDown: P limbs 0..K-1 from p_gathered rows (p%W)*2*p_chunk + p/W (component
  // stride p_chunk rows) -> own Q rows 0..q_own-1.
  std::vector<uint32_t> msp(K), msr(K), mdp(pl.q_own);
  std::vector<Shoup> mhinv(K), mhat((size_t)pl.q_own * K), pinv_rows(pl.q_own);
  std::vector<uint64_t> q_rows(pl.q_own);
  for (uint32_t k = 0; k < K; ++k) {
    msp[k] = L + k;
    msr[k] = (k % W) * 2 * pl.p_chunk + k / W;
    const uint64_t pk = P[L + k];
    uint64_t h = 1 % pk;
    for (uint32_t m = 0; m < K; ++m)
      if (m != k) h = nt::mulmod(h, P[L + m] % pk, pk);
    mhinv[k] = mk(nt::invmod(h, pk), pk);
  }
  for (uint32_t i = 0; i < pl.q_own; ++i) {
    const uint32_t pr = row_prime[i];
    const uint64_t t = P[pr];
    mdp[i] = pr;
    q_rows[i] = t;
    uint64_t pm = 1 % t;
    for (uint32_t m = 0; m < K; ++m) pm = nt::mulmod(pm, P[L + m] % t, t);
    pinv_rows[i] = mk(nt::invmod(pm, t), t);
    for (uint32_t k = 0; k < K; ++k) {
      uint64_t h = 1 % t;
      for (uint32_t m = 0; m < K; ++m)
        if (m != k) h = nt::mulmod(h, P[L + m] % t, t);
      mhat[(size_t)i * K + k] = mk(h, t);
    }
  }
  const size_t o_msp = put(msp.data(), msp.size() * 4), o_msr = put(msr.data(), msr.size() * 4),
               o_mdp = put(mdp.data(), mdp.size() * 4), o_mhi = put(mhinv.data(), mhinv.size() * sizeof(Shoup)),
               o_mh = put(mhat.data(), mhat.size() * sizeof(Shoup));
  const size_t o_pinv = put(pinv_rows.data(), pinv_rows.size() * sizeof(Shoup));
  const size_t o_qr = put(q_rows.data(), q_rows.size() * 8);
  const size_t o_rp = put(row_prime.data(), row_prime.size() * 4);
  // NTT lists.
  std::vector<uint2> send_list(pl.q_own), psend_list, conv_list;
  for (uint32_t i = 0; i < pl.q_own; ++i) send_list[i] = make_uint2(i, row_prime[i]);
  for (uint32_t comp = 0; comp < 2; ++comp) {
    for (uint32_t i = 0; i < pl.p_own; ++i)
      psend_list.push_back(make_uint2(comp * pl.p_chunk + i, row_prime[pl.q_own + i]));
    for (uint32_t i = 0; i < pl.q_own; ++i) conv_list.push_back(make_uint2(comp * pl.q_own + i, row_prime[i]));
  }
  const size_t o_sl = put(send_list.data(), send_list.size() * 8), o_el = put(ext_list.data(), ext_list.size() * 8),
               o_pl = put(psend_list.data(), psend_list.size() * 8),
               o_cl = put(conv_list.data(), conv_list.size() * 8);

  T.blob = DevMem(blob.size());
  FHE_CUDA(cudaMemcpy(T.blob.p, blob.data(), blob.size(), cudaMemcpyHostToDevice));
  const char* base = T.blob.as<char>();
  auto u32 = [base](size_t o) { return reinterpret_cast<const uint32_t*>(base + o); };
  auto sh = [base](size_t o) { return reinterpret_cast<const Shoup*>(base + o); };
  std::vector<ConvTable> tabs(2 * pl.digits);  // whole-gather tables, then per-digit-gather tables
  for (uint32_t j = 0; j < pl.digits; ++j) {
    const Tab& tb = dig[j];
    tabs[j] = ConvTable{tb.ns, tb.nt, u32(tb.sp), u32(tb.dp), sh(tb.hi), sh(tb.h), u32(tb.sr), u32(tb.dr)};
    tabs[pl.digits + j] = ConvTable{tb.ns, tb.nt, u32(tb.sp), u32(tb.dp), sh(tb.hi), sh(tb.h), u32(tb.srs),
                                    u32(tb.dr)};
  }
  T.digit_tabs = DevMem(std::max<size_t>(tabs.size() * sizeof(ConvTable), 16));
  if (!tabs.empty())
    FHE_CUDA(cudaMemcpy(T.digit_tabs.p, tabs.data(), tabs.size() * sizeof(ConvTable), cudaMemcpyHostToDevice));
  const ConvTable md{K, pl.q_own, u32(o_msp), u32(o_mdp), sh(o_mhi), sh(o_mh), u32(o_msr), nullptr};
  T.md_tab = DevMem(sizeof(ConvTable));
  FHE_CUDA(cudaMemcpy(T.md_tab.p, &md, sizeof(ConvTable), cudaMemcpyHostToDevice));
  T.send_list = reinterpret_cast<const uint2*>(base + o_sl);
  T.ext_list = reinterpret_cast<const uint2*>(base + o_el);
  T.ext_len = (uint32_t)ext_list.size();
  T.psend_list = reinterpret_cast<const uint2*>(base + o_pl);
  T.conv_list = reinterpret_cast<const uint2*>(base + o_cl);
  T.row_prime = u32(o_rp);
  T.pinv_rows = sh(o_pinv);
  T.q_rows = reinterpret_cast<const uint64_t*>(base + o_qr);
  return levels_.emplace(nq, std::move(T)).first->second;
}

void ShardKeySwitch::ntt_list(uint64_t* base, const uint2* list, uint32_t len, bool inverse) {
  if (!len) return;
  ck_.counters.ntt_limbs += len;
  NttArgs a = ck_.ctx.ntt_args(base, 1, 0, len, 0);
  a.list = list;
  a.lazy = ck_.ctx.max_prime() < (uint64_t(1) << 60) ? 16 : 0;
  FHE_CUDA(inverse ? ntt_inverse(a) : ntt_forward(a));
}

void ShardKeySwitch::modup_prepare(uint32_t nq, const uint64_t* d_own, uint64_t* send) {
  Level& T = level(nq);
  const uint32_t n = ck_.ctx.n;
  if (T.pl.q_own) {
    FHE_CUDA(cudaMemcpyAsync(send, d_own, (size_t)T.pl.q_own * n * 8, cudaMemcpyDeviceToDevice, ck_.ctx.stream));
    ntt_list(send, T.send_list, T.pl.q_own, true);
  }
}

void ShardKeySwitch::inner(uint32_t nq, int kind, uint64_t g, const uint64_t* gathered, const uint64_t* d_own,
                           uint64_t* acc, uint64_t* p_send) {
  Level& T = level(nq);
  require(keys_.count(key_id(kind, g)) != 0, "shard key not loaded (fhe_shard_load_key)", -4);
  ++ck_.counters.modup;
  for (uint32_t j = 0; j < T.pl.digits; ++j) convert_digit(T, j, gathered, false, d_own);
  inner_tail(nq, kind, g, acc, p_send);
}

void ShardKeySwitch::convert_digit(Level& T, uint32_t j, const uint64_t* gathered, bool split,
                                   const uint64_t* d_own) {
  const ShardPlan& pl = T.pl;
  const Context& c = ck_.ctx;
  const uint32_t n = c.n;
  const size_t ext_words = (size_t)pl.digits * pl.rows * n;
  if (ext_.bytes < ext_words * 8) {
    FHE_CUDA(cudaStreamSynchronize(c.stream));
    ext_ = DevMem(ext_words * 8);
  }
  uint64_t* e = ext_.as<uint64_t>() + (size_t)j * pl.rows * n;
  const uint32_t lo = T.digit_own_lo[j], hi = T.digit_own_hi[j];
  if (hi > lo)
    FHE_CUDA(cudaMemcpyAsync(e + (size_t)lo * n, d_own + (size_t)lo * n, (size_t)(hi - lo) * n * 8,
                             cudaMemcpyDeviceToDevice, c.stream));
  if (T.digit_nt[j])
    launch_convert(gathered, 0, e, 0, 1, T.digit_tabs.as<ConvTable>() + (split ? pl.digits : 0) + j,
                   T.digit_ns[j], T.digit_nt[j], n, c.d_mod.as<Modulus>(), c.stream,
                   c.max_prime() < (uint64_t(1) << 60));
}

void ShardKeySwitch::inner_digit(uint32_t nq, uint32_t j, const uint64_t* gathered_j, const uint64_t* d_own) {
  Level& T = level(nq);
  require(j < T.pl.digits, "digit index out of range", -1);
  if (j == 0) ++ck_.counters.modup;
  convert_digit(T, j, gathered_j, true, d_own);
}

void ShardKeySwitch::inner_tail(uint32_t nq, int kind, uint64_t g, uint64_t* acc, uint64_t* p_send) {
  Level& T = level(nq);
  const ShardPlan& pl = T.pl;
  const Context& c = ck_.ctx;
  const uint32_t n = c.n;
  auto key = keys_.find(key_id(kind, g));
  require(key != keys_.end(), "shard key not loaded (fhe_shard_load_key)", -4);
  const size_t ext_words = (size_t)pl.digits * pl.rows * n;
  if (ext_.bytes < ext_words * 8) {
    FHE_CUDA(cudaStreamSynchronize(c.stream));
    ext_ = DevMem(ext_words * 8);
  }
  uint64_t* ext = ext_.as<uint64_t>();
  ntt_list(ext, T.ext_list, T.ext_len, false);
  ++ck_.counters.key_inner;
  if (pl.rows) {
    const dim3 grid((n + kThreads - 1) / kThreads, pl.rows);
    k_key_inner_rows<<<grid, kThreads, 0, c.stream>>>(ext, pl.digits, pl.rows, key->second.as<uint64_t>(),
                                                      qa_full_ + pa_, PrimeMap{pl.q_own, qa_full_}, T.row_prime, acc,
                                                      n, c.d_mod.as<Modulus>());
    note_launch();
    FHE_CUDA(cudaGetLastError());
  }
  if (pl.p_own) {
    for (uint32_t comp = 0; comp < 2; ++comp)
      FHE_CUDA(cudaMemcpyAsync(p_send + (size_t)comp * pl.p_chunk * n,
                               acc + ((size_t)comp * pl.rows + pl.q_own) * n, (size_t)pl.p_own * n * 8,
                               cudaMemcpyDeviceToDevice, c.stream));
    ntt_list(p_send, T.psend_list, 2 * pl.p_own, true);
  }
}

void ShardKeySwitch::moddown(uint32_t nq, const uint64_t* acc, const uint64_t* p_gathered, const uint64_t* add0,
                             const uint64_t* add1, uint64_t* out) {
  Level& T = level(nq);
  const ShardPlan& pl = T.pl;
  const Context& c = ck_.ctx;
  const uint32_t n = c.n;
  ++ck_.counters.moddown;
  if (!pl.q_own) return;
  const size_t conv_words = (size_t)2 * pl.q_own * n;
  if (conv_.bytes < conv_words * 8) {
    FHE_CUDA(cudaStreamSynchronize(c.stream));
    conv_ = DevMem(conv_words * 8);
  }
  uint64_t* conv = conv_.as<uint64_t>();
  launch_convert(p_gathered, (size_t)pl.p_chunk * n, conv, (size_t)pl.q_own * n, 2, T.md_tab.as<ConvTable>(), c.K,
                 pl.q_own, n, c.d_mod.as<Modulus>(), c.stream, c.max_prime() < (uint64_t(1) << 60));
  ntt_list(conv, T.conv_list, 2 * pl.q_own, false);
  const dim3 grid((n + kThreads - 1) / kThreads, pl.q_own, 2);
  k_combine_rows<<<grid, kThreads, 0, c.stream>>>(acc, pl.rows, conv, pl.q_own, T.pinv_rows, T.q_rows, add0, add1,
                                                  out, n);
  note_launch();
  FHE_CUDA(cudaGetLastError());
}

void ShardKeySwitch::automorphism(uint32_t nq, uint64_t g, const uint64_t* in, uint64_t* out) {
  const uint32_t qo = q_own(nq);
  require(g % 2 == 1 && g < 2ull * ck_.ctx.n, "Galois element must be odd and below 2N", -1);
  if (!qo) return;
  const size_t s = (size_t)qo * ck_.ctx.n;
  launch_automorphism(in, s, out, s, 2, qo, ck_.ctx.log_n, g, ck_.ctx.stream);
}

}  // namespace fhe
