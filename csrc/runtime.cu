// Library-wide runtime state: the launch counter used as bench evidence, the
// programmatic-dependent-launch switch (MSB_PDL=1 turns it on) and which
// build this is (bounds-checked or release).
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace msb {

static std::atomic<long long> g_launches{0};

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

bool bounds_check_build() {
#ifdef MSB_BOUNDS_CHECK
  return true;
#else
  return false;
#endif
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MSB_PDL");
    return v != nullptr && std::strcmp(v, "1") == 0;
  }();
  return on;
}

}  // namespace msb
