// Rescale variant that allocates nothing: fhe_rescale_noalloc.
//
// Some callers cannot allocate device memory at the point where they need a
// rescale: code running inside a fixed memory budget that was reserved up
// front, a host framework that owns every allocation and forbids the library
// from calling cudaMalloc behind its back, or a caller holding a lock under
// which an allocation (which may synchronise the device) is not allowed.
// This entry point lets them rescale ciphertext residues they already hold in
// device memory.  Its scratch memory (the dropped limb, its centred lift into
// every remaining limb, and the q_last^{-1} constants) lives in the fixed
// array below instead of in buffers the library would allocate.
#include <cstring>
#include <mutex>

#include "../../include/fhe_b200.h"
#include "ckks_kernels.h"
#include "context.h"
#include "launch_count.h"

namespace fhe {
namespace {

// 32 MiB of scratch per GPU, held by every GPU that loads this part of the
// library until the process exits.
constexpr size_t kScratchWords = size_t(4) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint64_t g_noalloc_scratch[kScratchWords];

// Device addresses of g_noalloc_scratch, one per device.  In host code the
// array's name is only a host-side stand-in, never a device address.
std::mutex g_mu;
uint64_t* g_ptr[kMaxDevices] = {};

uint64_t* scratch_for(int device) {
  require(device >= 0 && device < kMaxDevices, "device ordinal above the no-alloc table");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_ptr[device]) {
    FHE_CUDA(cudaSetDevice(device));
    void* p = nullptr;
    FHE_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_ptr[device] = static_cast<uint64_t*>(p);
  }
  return g_ptr[device];
}

// out[i] = q_last^{-1} mod q_i with its Shoup companion, for i < count
// (q_last = mods[last].q): Fermat's inverse (every q_i is prime) by square
// and multiply, computed on the device so that no host buffer is involved.
__global__ void k_qinv_table(const Modulus* mods, uint32_t last, uint32_t count, Shoup* out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const Modulus& m = mods[i];
  uint64_t base = mods[last].q % m.q, v = 1;
  for (uint64_t e = m.q - 2; e; e >>= 1) {
    if (e & 1) v = mul_mod(v, base, m);
    base = mul_mod(base, base, m);
  }
  out[i] = Shoup{v, (uint64_t)(((unsigned __int128)v << 64) / m.q)};
}

}  // namespace

// Words of scratch a rescale of ncomp x n_limbs needs.
size_t noalloc_rescale_words(uint32_t ncomp, uint32_t n_limbs, uint32_t n) {
  return 2 * (size_t)(n_limbs - 1) + (size_t)ncomp * n + (size_t)ncomp * (n_limbs - 1) * n;
}

void rescale_noalloc(Context& c, const uint64_t* in, uint32_t ncomp, uint32_t nq, uint64_t* out) {
  require(in != nullptr && out != nullptr, "null input or output");
  require(ncomp >= 1 && ncomp <= 3, "ncomp must be 1, 2 or 3");
  require(nq >= 2 && nq <= c.L && nq <= 64, "n_limbs must be in [2, min(number of Q primes, 64)]");
  const uint32_t n = c.n;
  const size_t need = noalloc_rescale_words(ncomp, nq, n);
  require(need <= kScratchWords,
          "fhe_rescale_noalloc: needs " + std::to_string(need * 8) + " bytes of scratch, above the fixed " +
              std::to_string(kScratchWords * 8) + "-byte maximum (use fhe_rescale)");
  {  // limb i of `out` is written while later limbs of `in` are still to be read
    const uintptr_t i0 = reinterpret_cast<uintptr_t>(in), i1 = i0 + (size_t)ncomp * nq * n * 8;
    const uintptr_t o0 = reinterpret_cast<uintptr_t>(out), o1 = o0 + (size_t)ncomp * (nq - 1) * n * 8;
    require(o1 <= i0 || i1 <= o0, "fhe_rescale_noalloc: out must not overlap in");
  }
  c.make_current();
  uint64_t* base = scratch_for(c.device);
  // Layout: [Shoup q_last^{-1} mod q_i, i < nq-1][last limb per comp][lifted].
  Shoup* qinv = reinterpret_cast<Shoup*>(base);
  uint64_t* last = base + 2 * (size_t)(nq - 1);
  uint64_t* lifted = last + (size_t)ncomp * n;
  const uint64_t ql = c.primes[nq - 1];
  // Every scratch word below is written before it is read, on the caller's
  // context stream; nothing needs to start at zero.
  k_qinv_table<<<1, 64, 0, c.stream>>>(c.d_mod.as<Modulus>(), nq - 1, nq - 1, qinv);
  note_launch();
  const size_t is = (size_t)nq * n, os = (size_t)(nq - 1) * n;
  FHE_CUDA(cudaMemcpy2DAsync(last, (size_t)n * 8, in + (size_t)(nq - 1) * n, is * 8, (size_t)n * 8, ncomp,
                             cudaMemcpyDeviceToDevice, c.stream));
  NttArgs a = c.ntt_args(last, ncomp, nq - 1, 1, 1);
  FHE_CUDA(ntt_inverse(a));
  launch_rescale_lift(last, n, lifted, os, ncomp, nq - 1, n, ql, c.d_mod.as<Modulus>(), c.stream);
  NttArgs b = c.ntt_args(lifted, ncomp, 0, nq - 1, nq - 1);
  FHE_CUDA(ntt_forward(b));
  launch_moddown_combine(in, is, lifted, os, qinv, nullptr, out, os, ncomp, nq - 1, n, c.d_primes.as<uint64_t>(),
                         c.stream);
  FHE_CUDA(cudaGetLastError());
}

}  // namespace fhe
