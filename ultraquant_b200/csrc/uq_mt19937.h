// Legacy MT19937 stream with numpy RandomState seeding and bounded draws.
#pragma once
#include <stdint.h>

namespace uq {

struct MT19937 {
    static constexpr int kN = 624, kM = 397;
    uint32_t mt[kN];
    int idx = kN + 1;
    void seed(uint32_t s);
    void twist();
    uint32_t next32();
    uint64_t next64();
    // numpy RandomState.randint(low, high, count) (int64, masked rejection)
    void randint(int64_t low, int64_t high, int64_t count, int64_t *out);
};

}  // namespace uq
