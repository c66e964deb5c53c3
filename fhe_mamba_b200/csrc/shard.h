// Limb-sharded HYBRID key switching: one process per GPU, RNS limbs dealt out
// round-robin.  Rank r of W owns the Q limbs l with l % W == r and the P limbs
// p with p % W == r (cyclic, so every level stays balanced and a rank's key
// rows do not depend on the level).
//
// A key switch of d (NTT form, the rank's own Q rows) runs as three local
// stages around two all-gathers that the caller performs (NCCL through
// torch.distributed, on the context stream):
//   1. modup_prepare: INTT of the own Q rows into a send buffer [q_chunk][N].
//      -> all-gather: gathered [W][q_chunk][N], limb l at row (l%W)*q_chunk + l/W.
//   2. inner: ModUp of every digit into the own extended rows (basis
//      conversion from the gathered coefficients, NTT), key inner product with
//      the own key rows -> acc [2][rows][N] (rows = own Q + own P limbs); the
//      own P rows of acc in coefficient form go to p_send [2][p_chunk][N].
//      -> all-gather: p_gathered [W][2][p_chunk][N].
//   3. moddown: P -> own-Q conversion from p_gathered, NTT, (acc - conv) P^{-1}
//      (+ optional addends per component) -> out [2][q_own][N].
// Every word equals the single-GPU key switch's (same conversion, 128-bit
// accumulation and reduction).
#pragma once
#include <cstdint>
#include <map>

#include "ckks.h"

namespace fhe {

struct ShardPlan {
  uint32_t nq = 0, q_own = 0, q_chunk = 0, p_own = 0, p_chunk = 0, rows = 0, digits = 0;
};

class ShardKeySwitch {
 public:
  ShardKeySwitch(Ckks& ck, uint32_t rank, uint32_t world);
  const uint32_t rank, world;

  ShardPlan plan(uint32_t nq) const;
  // Copies the own rows of a key (kind 2: relinearisation, 3: rotation key of
  // Galois element g, generated on demand) into the shard's key store.
  void load_key(int kind, uint64_t g);
  void modup_prepare(uint32_t nq, const uint64_t* d_own, uint64_t* send);
  void inner(uint32_t nq, int kind, uint64_t g, const uint64_t* gathered, const uint64_t* d_own, uint64_t* acc,
             uint64_t* p_send);
  // The same stage with the first exchange split by digit, so the caller can
  // overlap digit j + 1's all-gather with digit j's conversion:
  // inner_digit for every digit j (gathered_j = digit j's own rows of every
  // rank, [W][dchunk][N], dchunk = ceil(alpha / W); rank r sends its digit-j
  // rows padded to dchunk), then inner_tail.
  void inner_digit(uint32_t nq, uint32_t j, const uint64_t* gathered_j, const uint64_t* d_own);
  void inner_tail(uint32_t nq, int kind, uint64_t g, uint64_t* acc, uint64_t* p_send);
  void moddown(uint32_t nq, const uint64_t* acc, const uint64_t* p_gathered, const uint64_t* add0,
               const uint64_t* add1, uint64_t* out);
  // Slot permutation of 2 components of q_own rows each (limb-local).
  void automorphism(uint32_t nq, uint64_t g, const uint64_t* in, uint64_t* out);

 private:
  struct Level {
    ShardPlan pl;
    DevMem blob;        // conversion tables, row maps and limb lists of this level
    DevMem digit_tabs;  // ConvTable[D] (ModUp, gathered -> own extended rows)
    DevMem md_tab;      // ConvTable (ModDown, p_gathered -> own Q rows)
    const uint2* send_list = nullptr;  // INTT of the send buffer: (row, prime)
    const uint2* ext_list = nullptr;   // NTT of converted ext rows
    const uint2* psend_list = nullptr; // INTT of the own P rows in p_send
    const uint2* conv_list = nullptr;  // NTT of the ModDown conversion
    const uint32_t* row_prime = nullptr;  // prime index of each own extended row
    const Shoup* pinv_rows = nullptr;     // P^{-1} mod q of each own Q row
    const uint64_t* q_rows = nullptr;     // q of each own Q row
    uint32_t ext_len = 0, dchunk = 0;
    std::vector<uint32_t> digit_ns, digit_nt, digit_own_lo, digit_own_hi;
  };
  void convert_digit(Level& T, uint32_t j, const uint64_t* gathered, bool split, const uint64_t* d_own);
  Level& level(uint32_t nq);
  uint64_t key_id(int kind, uint64_t g) const;
  uint32_t q_own(uint32_t nq) const { return nq > rank ? (nq - 1 - rank) / world + 1 : 0; }
  void ntt_list(uint64_t* base, const uint2* list, uint32_t len, bool inverse);

  Ckks& ck_;
  uint32_t qa_full_ = 0, pa_ = 0;
  std::map<uint32_t, Level> levels_;
  std::map<uint64_t, DevMem> keys_;  // [D_full][2][qa_full + pa][N]
  DevMem ext_, conv_;
};

}  // namespace fhe
