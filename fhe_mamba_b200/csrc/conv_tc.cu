// Fast basis conversion on the tensor cores (tcgen05.mma kind::i8, sm_100a).
//
// The conversion out_t = sum_i y_i * h_{i,t} mod p_t (y_i = [x_i hatinv_i]_{q_i},
// OpenFHE's ApproxSwitchCRTBasis) is a matrix product of the coefficients'
// source residues Y [N x ns] with the constant table H [ns x nt], reduced per
// target column.  With every prime below 2^60, y_i and h_{i,t} are split into
// 8 bytes, y_i = sum_a 2^(8a) y_{i,a} and h = sum_b 2^(8b) h_b, and
//   sum_i y_i h_{i,t} = sum_{s=0..14} 2^(8s) P_{s,t},
//   P_{s,t} = sum_i sum_{a+b=s} y_{i,a} h_{i,t,b}.
// One unsigned 8-bit MMA group per tile of 8 targets forms every P_{s,t}:
// A = the 128 coefficients' bytes (K = 16 sources x 8 bytes = 128), B = for
// each target and each shift s the row of bytes h_{i,t,s-a} at K index (i, a)
// (zero where s - a is outside [0, 8)), so D[row][16 t + s] = P_{s,t} with
// int32 accumulation (P < 16 * 8 * 255^2 < 2^23).  The epilogue reads each target's 15 shift
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
// the host (one 16 KiB tile per 8 targets), so a bulk copy moves it verbatim.
//
// Measured on a B200 (relinearisation at N = 2^16, depth 44, dnum 3, 15
// source limbs): 0.614 ms at 45 limbs against 0.702 ms with the CUDA-core
// conversion, 0.479 vs 0.514 at 31, 0.285 vs 0.294 at 16; with 7 source
// limbs the CUDA cores stay faster (0.312 vs 0.324 ms),
// since the epilogue costs the same for any source count.
#include <cstdint>
#include <cuda_runtime.h>

#include "ckks_kernels.h"
#include "launch_count.h"

namespace fhe {

namespace {

constexpr uint32_t kRows = 128;      // coefficients per CTA (MMA M)
constexpr uint32_t kTgt = 8;         // target limbs per tile
constexpr uint32_t kCols = 16 * kTgt;  // MMA N: 16 columns per target (15 shifts + 1 zero)
constexpr uint32_t kK = 128;         // MMA K in bytes (16 sources x 8 bytes)
constexpr uint32_t kBytesA = kRows * kK;   // 16 KiB
constexpr uint32_t kBytesB = kCols * kK;   // 16 KiB per tile, two buffers
constexpr uint32_t kSmem = kBytesA + 2 * kBytesB + 64;
constexpr uint32_t kTmemCols = 2 * kCols;  // two accumulator buffers
// Dynamic shared memory requested per CTA: above a third of the SM's 228 KiB,
// so at most two CTAs are resident and their tensor-memory allocations
// (2 x 256 columns) always fit the SM's 512 columns (no CTA waits in
// tcgen05.alloc).
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

__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
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
// t + ns) of digit j at ext + j*w*n; every block also copies the digit's own
// rows (its 128 coefficients) from the NTT-form input.
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

// One CTA = 128 coefficients of one component (MODE 0) or digit (MODE 1),
// all tiles of 8 targets.  A (the bytes of y) is formed once.  Thread 0 is
// the producer: it fetches B tiles with bulk asynchronous copies into two
// shared buffers and issues each tile's MMA group into one of two
// tensor-memory accumulators, so the copy of tile t + 2 and the MMA of tile
// t + 1 run while the 8 warps read tile t back (warps w and w + 4 share lane
// quarter w % 4 and take targets 0-3 and 4-7 of the tile).
constexpr uint32_t kThreads = 256;

__device__ __forceinline__ void issue_mma(uint32_t tmem, uint32_t a0, uint32_t b0, uint32_t mbar) {
#pragma unroll
  for (uint32_t s = 0; s < kK / 32; ++s) {
    const uint64_t da = smem_desc(a0 + s * 256), db = smem_desc(b0 + s * 256);
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(kIdesc), "r"(s));
  }
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}

// Bulk asynchronous copy of one B tile (16-byte aligned, a multiple of 16
// bytes) from global to shared memory, completing on mbar.
__device__ __forceinline__ void fetch_b(uint32_t dst, const uint8_t* src, uint32_t mbar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(kBytesB) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(kBytesB), "r"(mbar)
               : "memory");
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) k_conv_tc(const TcArgs g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sa = smem;
  uint8_t* sb = smem + kBytesA;  // two tiles
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kBytesA + 2 * kBytesB);  // B full [2], MMA done [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kBytesA + 2 * kBytesB + 32);

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
  const uint32_t ns = t.ns, n = g.n;
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t r = threadIdx.x & (kRows - 1), half = threadIdx.x / kRows;
  const uint32_t k = blockIdx.x * kRows + r;
  const uint32_t tiles = (t.nt + kTgt - 1) / kTgt;
  const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb), bb = smem_u32(bar), bm = bb + 16;
  const bool producer = threadIdx.x == 0;
  // producer bookkeeping: copies and MMA groups issued / waited per buffer
  uint32_t b_issued[2] = {0, 0}, b_waited[2] = {0, 0}, m_issued[2] = {0, 0};

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (producer) {
    for (uint32_t i = 0; i < 4; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bb + 8 * i));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fetch_b(b0, t.tc_b, bb);
    ++b_issued[0];
    if (tiles > 1) {
      fetch_b(b0 + kBytesB, t.tc_b + kBytesB, bb + 8);
      ++b_issued[1];
    }
  }

  // A: row r = coefficient k, bytes 8i..8i+7 = y_i (zero for i >= ns); the
  // two halves of the block form sources 0-7 and 8-15.  All loads first.
  const uint64_t* src;
  if constexpr (MODE == 1) src = g.src + (size_t)lo * n;
  else src = g.src + (size_t)blockIdx.y * g.s_comp;
  uint64_t* dst;
  if constexpr (MODE == 1) dst = g.dst + (size_t)j * g.w * n;
  else dst = g.dst + (size_t)blockIdx.y * g.d_comp;
  uint64_t x[8];
#pragma unroll
  for (uint32_t ii = 0; ii < 8; ++ii) {
    const uint32_t i = half * 8 + ii;
    x[ii] = 0;
    if (i < ns) {
      const size_t row = MODE == 1 ? i : (t.src_row ? t.src_row[i] : i);
      x[ii] = src[row * n + k];
    }
  }
#pragma unroll
  for (uint32_t ii = 0; ii < 8; ++ii) {
    const uint32_t i = half * 8 + ii;
    uint64_t y = 0;
    if (i < ns) {
      const Shoup h = t.hatinv[i];
      y = shoup_mul(x[ii], h.w, h.wp, g.mods[t.src_prime[i]].q);
      if constexpr (MODE == 1) dst[(size_t)(lo + i) * n + k] = g.dntt[(size_t)(lo + i) * n + k];
    }
    *reinterpret_cast<uint64_t*>(sa + (r >> 3) * 1024 + (i >> 1) * 128 + (r & 7) * 16 + (i & 1) * 8) = y;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  bool ok = true;
  if (producer) {
    ok = mbar_wait(bb, 0);
    b_waited[0] = 1;
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      issue_mma(tmem, a0, b0, bm);
      ++m_issued[0];
    }
  }
  ok = __syncthreads_and(ok);
  const uint32_t lane_base = ((warp & 3) * 32) << 16;
  uint32_t tile = 0;
  for (; tile < tiles && ok; ++tile) {
    const uint32_t buf = tile & 1, nb = buf ^ 1;
    if (producer && tile + 1 < tiles) {  // MMA of the next tile once its B tile has landed
      ok = mbar_wait(bb + 8 * nb, b_waited[nb] & 1);
      ++b_waited[nb];
      if (ok) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        issue_mma(tmem + nb * kCols, a0, b0 + nb * kBytesB, bm + 8 * nb);
        ++m_issued[nb];
      }
    }
    const bool mok = mbar_wait(bm + 8 * buf, (tile >> 1) & 1);  // this tile's MMA is done
    ok = ok && mok;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (producer && ok && tile + 2 < tiles) {  // B buffer `buf` is free again
      fetch_b(b0 + buf * kBytesB, t.tc_b + (size_t)(tile + 2) * kBytesB, bb + 8 * buf);
      ++b_issued[buf];
    }
    if (ok) {
      const uint32_t t0 = tile * kTgt + half * 4;
      uint32_t p[4][16];
      const uint32_t col = tmem + lane_base + buf * kCols + 16 * half * 4;
      tmem_ld16_nowait(col, p[0]);
      tmem_ld16_nowait(col + 16, p[1]);
      tmem_ld16_nowait(col + 32, p[2]);
      tmem_ld16_nowait(col + 48, p[3]);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (uint32_t u = 0; u < 4; ++u) {
        const uint32_t tt = t0 + u;
        if (tt < t.nt) {
          uint64_t hi, lo64;
          assemble(p[u], hi, lo64);
          const uint64_t v = reduce_u128(hi, lo64, g.mods[t.dst_prime[tt]]);
          size_t row;
          if constexpr (MODE == 1) row = tt < lo ? tt : tt + ns;
          else row = t.dst_row ? t.dst_row[tt] : tt;
          dst[row * n + k] = v;
        }
      }
    }
    // every warp's reads of accumulator `buf` are done before the MMA of
    // tile + 2 overwrites it
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    ok = __syncthreads_and(ok);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  if (!ok) {
    // A wait ran out: record it, then let every copy and MMA group the
    // producer issued finish (bounded waits) before the tensor memory goes.
    if (producer) {
      atomicAdd(&g_tc_timeouts, 1u);
      // phases complete in order and at most one per barrier is outstanding,
      // so the last issued phase of each barrier covers the rest
      for (uint32_t q = 0; q < 2; ++q) {
        if (b_issued[q] > b_waited[q]) mbar_wait(bb + 8 * q, (b_issued[q] - 1) & 1);
        if (m_issued[q]) mbar_wait(bm + 8 * q, (m_issued[q] - 1) & 1);
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <int MODE>
void launch_tc(const TcArgs& a, uint32_t ny, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_conv_tc<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLaunch);
    attr = true;
  }
  const dim3 grid(a.n / kRows, ny);
  k_conv_tc<MODE><<<grid, kThreads, kSmemLaunch, s>>>(a);
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
  (void)nt;
  launch_tc<0>(a, ncomp, s);
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
  (void)alpha;
  launch_tc<1>(a, D, s);
}

unsigned tc_conversion_timeouts() {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_timeouts, sizeof(v));
  return v;
}

}  // namespace fhe
