// CPU SIMT shim (test infrastructure): binary16 for the reference's kernels.
// Conversions go through GCC's _Float16 (correctly rounded, round to nearest
// even), which is independent of the hand-written conversion in the C oracle.
#pragma once
#include <stdint.h>
#include <string.h>

struct __half {
    uint16_t bits;
};
inline float __half2float(__half h) {
    _Float16 v;
    memcpy(&v, &h.bits, 2);
    return (float)v;
}
inline __half __float2half_rn(float f) {
    _Float16 v = (_Float16)f;
    __half h;
    memcpy(&h.bits, &v, 2);
    return h;
}
inline __half __ushort_as_half(uint16_t u) {
    __half h;
    h.bits = u;
    return h;
}
