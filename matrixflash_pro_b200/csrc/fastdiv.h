// Division by a run-time invariant divisor as a multiply and a shift.
//
// The TMA producer of the conv kernels turns K-block indices into (image, position) or
// (tap, channel) box coordinates on one thread per CTA; hardware integer division is a
// long dependent instruction sequence and, issued per K block, it set the pace of the
// whole pipeline. The host computes (mul, shift) once per launch; the device evaluates
// floor(n / d) = (umulhi(n, mul) + n) >> shift.
//
// Method: Granlund & Montgomery, "Division by Invariant Integers using Multiplication"
// (PLDI 1994), round-up multiplier: with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1 < 2^32, floor(n / d) = floor((floor(m n / 2^32) + n) / 2^l)
// for 0 <= n < 2^32. The sum is formed in 32 bits, so callers keep n < 2^31 (then the sum
// stays below 2^32); divisors are 1 <= d < 2^31.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define MFB_HD __host__ __device__ __forceinline__
#else
#define MFB_HD inline
#endif

namespace mfb {

struct FastDiv {
    uint32_t mul;
    uint32_t shift;
    uint32_t d;
};

inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while ((static_cast<uint64_t>(1) << l) < d) ++l;
    const uint64_t m = ((static_cast<uint64_t>(1) << 32) * ((static_cast<uint64_t>(1) << l) - d)) / d + 1;
    return FastDiv{static_cast<uint32_t>(m), l, d};
}

MFB_HD uint32_t fastdiv(uint32_t n, const FastDiv& f) {
#if defined(__CUDA_ARCH__)
    const uint32_t hi = __umulhi(n, f.mul);
#else
    const uint32_t hi = static_cast<uint32_t>((static_cast<uint64_t>(n) * f.mul) >> 32);
#endif
    return (hi + n) >> f.shift;
}

}  // namespace mfb
