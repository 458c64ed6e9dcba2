// Host-side argument checks shared by the dense and head C-ABI entry points.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace ornith {

// Null, misaligned or address-wrapping buffers, and any overlap between a
// buffer the call writes (index >= first_written) and any other buffer, are
// invalid arguments (dense_g256_consumer.cpp:178-181,
// head_i8_tile_consumer.cpp:260-269).  The buffer at index `optional` may be
// null; it is then left out of every check.
template <int NB>
inline bool buffers_ok(const void* const (&ptr)[NB], const size_t (&bytes)[NB], const uintptr_t (&align)[NB],
                       int first_written, int optional = -1) {
    uintptr_t lo[NB] = {}, hi[NB] = {};
    bool used[NB];
    for (int i = 0; i < NB; ++i) {
        used[i] = !(i == optional && ptr[i] == nullptr);
        if (!used[i]) continue;
        const uintptr_t p = reinterpret_cast<uintptr_t>(ptr[i]);
        if (!ptr[i] || p % align[i] || bytes[i] > UINTPTR_MAX - p) return false;
        lo[i] = p;
        hi[i] = p + bytes[i];
    }
    for (int i = first_written; i < NB; ++i)
        for (int j = 0; j < NB; ++j)
            if (i != j && used[i] && used[j] && lo[i] < hi[j] && lo[j] < hi[i]) return false;
    return true;
}

}  // namespace ornith
