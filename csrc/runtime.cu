// Library-wide runtime state: the launch counter used as bench evidence.
#include <atomic>

#include "common.cuh"

namespace msb {

static std::atomic<long long> g_launches{0};

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

}  // namespace msb
