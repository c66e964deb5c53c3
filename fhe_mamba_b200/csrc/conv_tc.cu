// Fast basis conversion on the tensor cores (tcgen05.mma kind::i8, sm_100a).
//
// The conversion out_t = sum_i y_i * h_{i,t} mod p_t (y_i = [x_i hatinv_i]_{q_i},
// OpenFHE's ApproxSwitchCRTBasis) is a matrix product of the coefficients'
// source residues Y [N x ns] with the constant table H [ns x nt], reduced per
// target column.  With every prime below 2^60, y_i and h_{i,t} are split into
// 8 bytes, y_i = sum_a 2^(8a) y_{i,a} and h = sum_b 2^(8b) h_b, and
//   sum_i y_i h_{i,t} = sum_{s=0..14} 2^(8s) P_{s,t},
//   P_{s,t} = sum_i sum_{a+b=s} y_{i,a} h_{i,t,b}.
// One unsigned 8-bit MMA per CTA forms every P_{s,t}: A = the 128 coefficients'
// bytes (K = 16 sources x 8 bytes = 128), B = for each of 16 targets and each
// shift s the row of bytes h_{i,t,s-a} at K index (i, a) (zero where s - a is
// outside [0, 8)), so D[row][16 t + s] = P_{s,t} with int32 accumulation
// (P < 16 * 8 * 255^2 < 2^23).  The epilogue reads each target's 15 shift
// sums from tensor memory, assembles the exact sum (below 16 * 2^120) in 128
// bits with shifts and adds, and reduces it once.  The multiply-accumulates
// leave the 64-bit integer multiply pipe, which bounds the CUDA-core
// conversion (ckks_kernels.cu k_convert / k_modup); the result is identical
// word for word.
//
// Shared memory operands use the canonical K-major layout without swizzle:
// core matrices of 8 rows x 16 bytes (128 contiguous bytes), the 8 K-chunks
// of one 8-row group adjacent (leading byte offset 128), 8-row groups 1024
// bytes apart (stride byte offset).  The B table is stored in that layout by
// the host (one 32 KiB tile per 16 targets), so a CTA copies it verbatim.
#include <cstdint>
#include <cuda_runtime.h>

#include "ckks_kernels.h"
#include "launch_count.h"

namespace fhe {

namespace {

constexpr uint32_t kRows = 128;      // coefficients per CTA (MMA M)
constexpr uint32_t kTgt = 16;        // target limbs per CTA
constexpr uint32_t kCols = 16 * kTgt;  // MMA N: 16 columns per target (15 shifts + 1 zero)
constexpr uint32_t kK = 128;         // MMA K in bytes (16 sources x 8 bytes)
constexpr uint32_t kBytesA = kRows * kK;   // 16 KiB
constexpr uint32_t kBytesB = kCols * kK;   // 32 KiB
constexpr uint32_t kSmem = kBytesA + kBytesB + 64;
// Dynamic shared memory requested per CTA: above a third of the SM's 228 KiB,
// so at most two CTAs are resident and their two 256-column tensor-memory
// allocations always fit the SM's 512 columns (no CTA waits in tcgen05.alloc).
constexpr uint32_t kSmemLaunch = 96 * 1024;
static_assert(kSmem <= kSmemLaunch, "operands exceed the requested shared memory");
// Bound on the wait for the MMA's completion: far above its microseconds;
// on expiry the kernel records the failure, skips its outputs and frees its
// tensor memory.
constexpr uint32_t kWaitLimit = 1u << 20;

__device__ unsigned g_tc_timeouts = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// K-major, no swizzle: start address, LBO = 128 B (adjacent K chunks), SBO =
// 1024 B (adjacent 8-row groups), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// kind::i8 instruction descriptor: int32 accumulator, unsigned A and B,
// both K-major, N = kCols, M = kRows.
constexpr uint32_t kIdesc = (2u << 4) | ((kCols >> 3) << 17) | ((kRows >> 4) << 24);

__device__ __forceinline__ bool mbar_wait(uint32_t addr, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// sum_{s<15} 2^(8s) p[s] (exact, below 2^124) as (hi, lo), from four groups
// of byte shifts that each fit 64 bits.
__device__ __forceinline__ void assemble(const uint32_t (&p)[16], uint64_t& hi, uint64_t& lo) {
  const uint64_t g0 = (uint64_t)p[0] + ((uint64_t)p[1] << 8) + ((uint64_t)p[2] << 16) + ((uint64_t)p[3] << 24);
  const uint64_t g1 = (uint64_t)p[4] + ((uint64_t)p[5] << 8) + ((uint64_t)p[6] << 16) + ((uint64_t)p[7] << 24);
  const uint64_t g2 = (uint64_t)p[8] + ((uint64_t)p[9] << 8) + ((uint64_t)p[10] << 16) + ((uint64_t)p[11] << 24);
  const uint64_t g3 = (uint64_t)p[12] + ((uint64_t)p[13] << 8) + ((uint64_t)p[14] << 16);
  lo = g0 + (g1 << 32);
  hi = (g1 >> 32) + g2 + (g3 << 32) + (lo < g0);
}

// MODE 0 (convert): blockIdx.y = component; sources at src + y*s_comp +
// src_row(i)*n, targets at dst + y*d_comp + dst_row(t)*n (ConvTable maps).
// MODE 1 (ModUp): blockIdx.y = digit - digit0; sources are the digit's own
// rows lo..hi-1 of coef, targets the other rows of ext (row t < lo: t, else
// t + ns) of digit j at ext + j*w*n; the z == 0 blocks also copy the digit's
// own rows from the NTT-form input.
struct TcArgs {
  const uint64_t* src;
  size_t s_comp;
  uint64_t* dst;
  size_t d_comp;
  const ConvTable* tab;       // MODE 0
  const ModUpDigit* digits;   // MODE 1
  uint32_t digit0, w;         // MODE 1
  const uint64_t* dntt;       // MODE 1
  uint32_t n;
  const Modulus* mods;
};

template <int MODE>
__global__ void __launch_bounds__(kRows, 1) k_conv_tc(const TcArgs g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sa = smem;
  uint8_t* sb = smem + kBytesA;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + kBytesA + kBytesB);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kBytesA + kBytesB + 8);

  ConvTable t;
  uint32_t lo = 0, j = 0;
  if constexpr (MODE == 1) {
    j = g.digit0 + blockIdx.y;
    const ModUpDigit dg = g.digits[j];
    t = dg.conv;
    lo = dg.lo;
  } else {
    t = *g.tab;
  }
  const uint32_t t0 = blockIdx.z * kTgt;
  if (t0 >= t.nt) return;  // uniform across the block, before any tensor memory is held
  const uint32_t nt = min(kTgt, t.nt - t0);
  const uint32_t ns = t.ns;
  const uint32_t n = g.n, r = threadIdx.x, k = blockIdx.x * kRows + r;
  const uint32_t warp = threadIdx.x >> 5;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(mbar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // A: row r = coefficient k, bytes 8i..8i+7 = y_i (zero for i >= ns).
  const uint64_t* src;
  if constexpr (MODE == 1) src = g.src + (size_t)lo * n;
  else src = g.src + (size_t)blockIdx.y * g.s_comp;
#pragma unroll
  for (uint32_t i = 0; i < 16; ++i) {
    uint64_t y = 0;
    if (i < ns) {
      const size_t row = MODE == 1 ? i : (t.src_row ? t.src_row[i] : i);
      const uint64_t x = src[row * n + k];
      const Shoup h = t.hatinv[i];
      y = shoup_mul(x, h.w, h.wp, g.mods[t.src_prime[i]].q);
      if constexpr (MODE == 1) {
        if (blockIdx.z == 0) {
          uint64_t* e = g.dst + (size_t)j * g.w * n;
          e[(size_t)(lo + i) * n + k] = g.dntt[(size_t)(lo + i) * n + k];
        }
      }
    }
    *reinterpret_cast<uint64_t*>(sa + (r >> 3) * 1024 + (i >> 1) * 128 + (r & 7) * 16 + (i & 1) * 8) = y;
  }
  // B: this target tile of the table, stored by the host in the operand layout.
  {
    const uint4* bsrc = reinterpret_cast<const uint4*>(t.tc_b + (size_t)blockIdx.z * kBytesB);
    uint4* bdst = reinterpret_cast<uint4*>(sb);
#pragma unroll 4
    for (uint32_t v = threadIdx.x; v < kBytesB / 16; v += kRows) bdst[v] = __ldg(bsrc + v);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;

  if (threadIdx.x == 0) {
    const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
#pragma unroll
    for (uint32_t s = 0; s < kK / 32; ++s) {
      const uint64_t da = smem_desc(a0 + s * 256), db = smem_desc(b0 + s * 256);
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "setp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
          "l"(da), "l"(db), "r"(kIdesc), "r"(s));
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(mbar))
                 : "memory");
  }
  const bool ok = mbar_wait(smem_u32(mbar), 0);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (!ok) {
    if (threadIdx.x == 0) atomicAdd(&g_tc_timeouts, 1u);
  } else {
    uint64_t* dst;
    if constexpr (MODE == 1) dst = g.dst + (size_t)j * g.w * n;
    else dst = g.dst + (size_t)blockIdx.y * g.d_comp;
    const uint32_t lane_base = (warp * 32) << 16;
    for (uint32_t u = 0; u < nt; ++u) {
      uint32_t p[16];
      tmem_ld16(tmem + lane_base + 16 * u, p);
      uint64_t hi, lo64;
      assemble(p, hi, lo64);
      const uint32_t tt = t0 + u;
      const uint64_t v = reduce_u128(hi, lo64, g.mods[t.dst_prime[tt]]);
      size_t row;
      if constexpr (MODE == 1) row = tt < lo ? tt : tt + ns;
      else row = t.dst_row ? t.dst_row[tt] : tt;
      dst[row * n + k] = v;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
  }
}

template <int MODE>
void launch_tc(const TcArgs& a, uint32_t ny, uint32_t nt_max, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_conv_tc<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLaunch);
    attr = true;
  }
  const dim3 grid(a.n / kRows, ny, (nt_max + kTgt - 1) / kTgt);
  k_conv_tc<MODE><<<grid, kRows, kSmemLaunch, s>>>(a);
  note_launch();
}

}  // namespace

bool tc_conversion_supported(uint32_t n, uint32_t ns, bool primes_below_2_60) {
  return primes_below_2_60 && ns >= 1 && ns <= 16 && n % kRows == 0;
}

std::vector<uint8_t> tc_conversion_table(const Shoup* hat, uint32_t ns, uint32_t nt) {
  const uint32_t tiles = (nt + kTgt - 1) / kTgt;
  std::vector<uint8_t> out((size_t)tiles * kBytesB, 0);
  for (uint32_t tt = 0; tt < nt; ++tt) {
    uint8_t* tile = out.data() + (size_t)(tt / kTgt) * kBytesB;
    const uint32_t u = tt % kTgt;
    for (uint32_t s = 0; s < 15; ++s) {
      const uint32_t row = 16 * u + s;
      for (uint32_t i = 0; i < ns; ++i) {
        const uint64_t h = hat[(size_t)tt * ns + i].w;
        for (uint32_t a = 0; a < 8; ++a) {
          if (s < a || s - a >= 8) continue;
          const uint32_t kk = 8 * i + a;
          tile[(row >> 3) * 1024 + (kk >> 4) * 128 + (row & 7) * 16 + (kk & 15)] = (uint8_t)(h >> (8 * (s - a)));
        }
      }
    }
  }
  return out;
}

void launch_convert_tc(const uint64_t* src, size_t s_comp, uint64_t* dst, size_t d_comp, uint32_t ncomp,
                       const ConvTable* t_dev, uint32_t nt, uint32_t n, const Modulus* mods, cudaStream_t s) {
  TcArgs a{};
  a.src = src;
  a.s_comp = s_comp;
  a.dst = dst;
  a.d_comp = d_comp;
  a.tab = t_dev;
  a.n = n;
  a.mods = mods;
  launch_tc<0>(a, ncomp, nt, s);
}

void launch_modup_tc(const uint64_t* coef, const uint64_t* dntt, uint64_t* ext, uint32_t nq, uint32_t K,
                     uint32_t n, const ModUpDigit* digits_dev, uint32_t D, uint32_t alpha, const Modulus* mods,
                     cudaStream_t s) {
  TcArgs a{};
  a.src = coef;
  a.dst = ext;
  a.digits = digits_dev;
  a.digit0 = 0;
  a.w = nq + K;
  a.dntt = dntt;
  a.n = n;
  a.mods = mods;
  // every digit has at most nq + K - (nq - (D-1) alpha) targets; blocks past a
  // digit's own target count return at once
  const uint32_t shortest = nq - (D - 1) * alpha;
  launch_tc<1>(a, D, nq + K - shortest, s);
}

unsigned tc_conversion_timeouts() {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_timeouts, sizeof(v));
  return v;
}

}  // namespace fhe
