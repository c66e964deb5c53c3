// Host-side count of the kernels this library launches (all contexts, all
// devices); every launch site calls note_launch() right after its launch.
#pragma once
#include <atomic>
#include <cstdint>

namespace fhe {
extern std::atomic<uint64_t> g_kernel_launches;
inline void note_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace fhe
