// ref_compat.hpp -- force-included when compiling the reference's own AVX-512
// CPU backend with GCC.  TEST INFRASTRUCTURE ONLY (oracle build recipe).
//
// The reference is written for Clang and uses three Clang-only builtins in
// src/lib/backend/cpu/avx.hpp (lines 18, 30, 37 and 76).  GCC 13 lacks them,
// so they are mapped to GCC equivalents with the same meaning; nothing else
// in the reference is changed.
#pragma once

#define __builtin_vectorelements(v) (sizeof(v) / sizeof((v)[0]))
#define __builtin_memcpy_inline(dst, src, n) __builtin_memcpy((dst), (src), (n))

#ifdef __cplusplus
template <class V>
inline auto q3_ref_reduce_max(const V& v) {
    auto m = v[0];
    for (unsigned i = 1; i < sizeof(V) / sizeof(v[0]); ++i) m = v[i] > m ? v[i] : m;
    return m;
}
#define __builtin_reduce_max(v) q3_ref_reduce_max(v)
#endif
