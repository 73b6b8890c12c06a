// Host check of the multiply-shift division the conv producers use (fastdiv.h): every
// quotient is compared with the hardware division over the whole operand range the kernels
// allow (0 <= n < 2^31, 1 <= d < 2^31): all small divisors against dense and boundary
// numerators, then random pairs. Prints "0 failure(s)" on success.
#include "fastdiv.h"

#include <cstdint>
#include <cstdio>
#include <random>

int main() {
    long long failures = 0, checked = 0;
    auto check = [&](uint32_t n, const mfb::FastDiv& f) {
        ++checked;
        if (mfb::fastdiv(n, f) != n / f.d) {
            if (failures < 10) std::printf("n=%u d=%u got=%u want=%u\n", n, f.d, mfb::fastdiv(n, f), n / f.d);
            ++failures;
        }
    };
    const uint32_t top = 0x7fffffffu;
    for (uint32_t d = 1; d <= 4096; ++d) {
        const mfb::FastDiv f = mfb::make_fastdiv(d);
        for (uint32_t n = 0; n < 20000; ++n) check(n, f);
        for (uint32_t q = 1; q < 64; ++q) {  // around multiples of d
            const uint64_t base = static_cast<uint64_t>(q) * d * 997;
            for (int e = -2; e <= 2; ++e)
                if (base + e <= top && static_cast<int64_t>(base) + e >= 0) check(static_cast<uint32_t>(base + e), f);
        }
        for (uint32_t e = 0; e < 64; ++e) check(top - e, f);
    }
    std::mt19937_64 rng(12345);
    for (int i = 0; i < 4000000; ++i) {
        const uint32_t d = 1 + static_cast<uint32_t>(rng() % top);
        const mfb::FastDiv f = mfb::make_fastdiv(d);
        check(static_cast<uint32_t>(rng() % (static_cast<uint64_t>(top) + 1)), f);
        check(d, f);
        check(d - 1, f);
        check(top, f);
    }
    for (int l = 0; l < 31; ++l) {  // powers of two and their neighbours as divisors
        for (int e = -1; e <= 1; ++e) {
            const int64_t d = (int64_t{1} << l) + e;
            if (d < 1 || d > top) continue;
            const mfb::FastDiv f = mfb::make_fastdiv(static_cast<uint32_t>(d));
            for (uint32_t n : {0u, 1u, static_cast<uint32_t>(d - 1), static_cast<uint32_t>(d), top, top - 1})
                check(n, f);
        }
    }
    std::printf("%lld checked, %lld failure(s)\n", checked, failures);
    return failures == 0 ? 0 : 1;
}
