// Ciphertext and key files for a process-separated client and server (the
// reference's handoff, native/fideslib_stage0/src/fideslib_handoff.cpp:27-85:
// the client serialises the context's evaluation keys and its encrypted
// inputs, the server deserialises them, evaluates and serialises the result).
//
// Format (little endian): a 48-byte header {magic "FHEB200", version 1, kind,
// log_n, L, K, dnum, fingerprint of every prime}, the payload, and a 64-bit
// checksum of the payload words.  Kind 1: a ciphertext {ncomp, nq,
// noise_deg, scale, ncomp*nq*N words}.  Kind 2: a key bundle {has_secret,
// rotation key count, seed (only with the secret), [secret s in NTT form],
// public key, relinearisation key, (Galois element, key) per rotation key}.
// A bundle without the secret makes an evaluation-only (server) context: it
// evaluates, encrypts with fresh randomness, and refuses to decrypt or to
// generate keys.
#include <cstring>
#include <fstream>
#include <random>
#include <vector>

#include "ckks.h"

namespace fhe {
namespace {

constexpr char kMagic[8] = {'F', 'H', 'E', 'B', '2', '0', '0', '\0'};
constexpr uint32_t kVersion = 1;

struct Header {
  char magic[8];
  uint32_t version, kind, log_n, L, K, dnum;
  uint64_t prime_fp;
  uint32_t pad[2];
};
static_assert(sizeof(Header) == 48, "header layout");

uint64_t prime_fingerprint(const Context& c) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (uint64_t q : c.primes) h = (h ^ q) * 0x100000001b3ull;
  return h;
}

struct Checksum {
  uint64_t h = 0x84222325cbf29ce4ull;
  void add(const uint64_t* w, size_t n) {
    for (size_t i = 0; i < n; ++i) h = ((h ^ w[i]) * 0x100000001b3ull) ^ (h >> 29);
  }
};

void write_header(std::ostream& os, const Context& c, uint32_t kind) {
  Header h{};
  std::memcpy(h.magic, kMagic, 8);
  h.version = kVersion;
  h.kind = kind;
  h.log_n = c.log_n;
  h.L = c.L;
  h.K = c.K;
  h.dnum = c.dnum;
  h.prime_fp = prime_fingerprint(c);
  os.write(reinterpret_cast<const char*>(&h), sizeof h);
}

void read_header(std::istream& is, const Context& c, uint32_t kind) {
  Header h{};
  is.read(reinterpret_cast<char*>(&h), sizeof h);
  require((bool)is && std::memcmp(h.magic, kMagic, 8) == 0, "not a fhe_b200 file", -1);
  require(h.version == kVersion, "unsupported fhe_b200 file version", -1);
  require(h.kind == kind, kind == 1 ? "the file holds no ciphertext" : "the file holds no key bundle", -1);
  require(h.log_n == c.log_n && h.L == c.L && h.K == c.K && h.dnum == c.dnum && h.prime_fp == prime_fingerprint(c),
          "the file was written for different CKKS parameters", -1);
}

template <class T>
void put(std::ostream& os, const T& v) {
  os.write(reinterpret_cast<const char*>(&v), sizeof v);
}
template <class T>
T get(std::istream& is) {
  T v{};
  is.read(reinterpret_cast<char*>(&v), sizeof v);
  require((bool)is, "truncated fhe_b200 file", -1);
  return v;
}

// device words -> stream (through one host buffer), hashed
void put_words(std::ostream& os, const void* dev, size_t words, Checksum& ck, cudaStream_t s) {
  std::vector<uint64_t> h(words);
  FHE_CUDA(cudaMemcpyAsync(h.data(), dev, words * 8, cudaMemcpyDeviceToHost, s));
  FHE_CUDA(cudaStreamSynchronize(s));
  ck.add(h.data(), words);
  os.write(reinterpret_cast<const char*>(h.data()), (std::streamsize)(words * 8));
}

void get_words(std::istream& is, void* dev, size_t words, Checksum& ck, cudaStream_t s) {
  std::vector<uint64_t> h(words);
  is.read(reinterpret_cast<char*>(h.data()), (std::streamsize)(words * 8));
  require((bool)is, "truncated fhe_b200 file", -1);
  ck.add(h.data(), words);
  FHE_CUDA(cudaMemcpyAsync(dev, h.data(), words * 8, cudaMemcpyHostToDevice, s));
  FHE_CUDA(cudaStreamSynchronize(s));
}

void check_sum(std::istream& is, const Checksum& ck) {
  require(get<uint64_t>(is) == ck.h, "fhe_b200 file checksum mismatch (corrupted file)", -1);
}

}  // namespace

void save_ciphertext(Ckks& k, const Ct& c, const std::string& path) {
  std::ofstream os(path, std::ios::binary);
  require((bool)os, "cannot write " + path, -1);
  write_header(os, k.ctx, 1);
  put(os, c.ncomp);
  put(os, c.nq);
  put(os, c.noise_deg);
  put(os, (uint32_t)0);
  put(os, c.scale);
  Checksum ck;
  const size_t n = k.ctx.n;
  for (uint32_t comp = 0; comp < c.ncomp; ++comp)
    put_words(os, c.data() + (size_t)comp * c.cap * n, (size_t)c.nq * n, ck, k.ctx.stream);
  put(os, ck.h);
  require((bool)os, "write failed: " + path, -1);
}

std::unique_ptr<Ct> load_ciphertext(Ckks& k, const std::string& path) {
  std::ifstream is(path, std::ios::binary);
  require((bool)is, "cannot open " + path, -1);
  read_header(is, k.ctx, 1);
  const uint32_t ncomp = get<uint32_t>(is), nq = get<uint32_t>(is), noise_deg = get<uint32_t>(is);
  get<uint32_t>(is);
  const double scale = get<double>(is);
  require(ncomp >= 2 && ncomp <= 3 && nq >= 1 && nq <= k.ctx.L && noise_deg >= 1 && noise_deg <= 3,
          "bad ciphertext shape in " + path, -1);
  auto c = k.alloc(nq, ncomp);
  c->noise_deg = noise_deg;
  c->scale = scale;
  Checksum ck;
  get_words(is, c->data(), (size_t)ncomp * nq * k.ctx.n, ck, k.ctx.stream);
  check_sum(is, ck);
  return c;
}

void Ckks::save_keys(const std::string& path, bool with_secret) {
  require(keyed_, "no keys to save", -4);
  require(!with_secret || has_secret_, "this context holds no secret key", -4);
  require(sparse_h_ == 0, "sparse-secret bootstrapping keys are not serialized", -1);
  std::ofstream os(path, std::ios::binary);
  require((bool)os, "cannot write " + path, -1);
  write_header(os, ctx, 2);
  put(os, (uint32_t)(with_secret ? 1 : 0));
  put(os, (uint32_t)rot_.size());
  put(os, with_secret ? seed_ : (uint64_t)0);
  Checksum ck;
  if (with_secret) put_words(os, s_ntt_.p, key_words(0), ck, ctx.stream);
  put_words(os, pk_.p, key_words(1), ck, ctx.stream);
  put_words(os, rlk_.p, key_words(2), ck, ctx.stream);
  for (const auto& [g, key] : rot_) {
    put(os, g);
    put_words(os, key.p, key_words(3), ck, ctx.stream);
  }
  put(os, ck.h);
  require((bool)os, "write failed: " + path, -1);
}

void Ckks::load_keys(const std::string& path) {
  std::ifstream is(path, std::ios::binary);
  require((bool)is, "cannot open " + path, -1);
  read_header(is, ctx, 2);
  const uint32_t with_secret = get<uint32_t>(is), n_rot = get<uint32_t>(is);
  const uint64_t seed = get<uint64_t>(is);
  require(with_secret <= 1 && n_rot <= 4096, "bad key bundle", -1);
  Checksum ck;
  DevMem s, pk(key_words(1) * 8), rlk(key_words(2) * 8);
  if (with_secret) {
    s = DevMem(key_words(0) * 8);
    get_words(is, s.p, key_words(0), ck, ctx.stream);
  }
  get_words(is, pk.p, key_words(1), ck, ctx.stream);
  get_words(is, rlk.p, key_words(2), ck, ctx.stream);
  std::map<uint64_t, DevMem> rot;
  for (uint32_t i = 0; i < n_rot; ++i) {
    const uint64_t g = get<uint64_t>(is);
    require(g % 2 == 1 && g < 2ull * ctx.n, "bad Galois element in key bundle", -1);
    DevMem key(key_words(3) * 8);
    get_words(is, key.p, key_words(3), ck, ctx.stream);
    rot.emplace(g, std::move(key));
  }
  check_sum(is, ck);
  s_ntt_ = std::move(s);
  pk_ = std::move(pk);
  rlk_ = std::move(rlk);
  rot_ = std::move(rot);
  // keys tied to a previous secret of this context no longer apply
  s_sparse_.release();
  key_to_sparse_.release();
  key_to_dense_.release();
  sparse_h_ = 0;
  has_secret_ = with_secret != 0;
  std::random_device rd;
  // With the secret the seed comes back (new keys equal the saving context's);
  // without it the seed would be the secret, so an evaluation-only context
  // draws its own.  Either way encryption continues from a random nonce, so
  // a restored context never repeats the saving context's randomness.
  seed_ = has_secret_ ? seed : (((uint64_t)rd() << 32) ^ rd());
  enc_nonce = ((((uint64_t)rd() << 32) ^ rd()) & ((1ull << 47) - 1)) + (1ull << 20);
  keyed_ = true;
}

}  // namespace fhe
