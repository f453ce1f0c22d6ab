// Fixed-point primitives of the integer semantics, device side.
//
//   RS(x, n)  = (x + 2^(n-1)) >> n, arithmetic shift, ties toward +inf; n <= 0 is an exact left
//               shift (python/intref.py:42-50, c/intref.c:29-32).
//   SAT(x, b) = clip to [-2^(b-1), 2^(b-1) - 1]; b >= 64 is the identity (c/intref.c:33-37).
//
// All values are two's-complement int64 with wrapping arithmetic, as in the reference (numpy
// int64 and gcc), so the same integers come out for every input.
#pragma once
#include <cstdint>

namespace eii {

__host__ __device__ __forceinline__ int64_t rs64(int64_t x, int n) {
    if (n <= 0) return static_cast<int64_t>(static_cast<uint64_t>(x) << (-n));
    return static_cast<int64_t>(static_cast<uint64_t>(x) + (static_cast<uint64_t>(1) << (n - 1))) >> n;
}

__host__ __device__ __forceinline__ int64_t sat64(int64_t x, int bits) {
    if (bits >= 64) return x;
    const int64_t hi = (static_cast<int64_t>(1) << (bits - 1)) - 1;
    const int64_t lo = -hi - 1;
    return x < lo ? lo : (x > hi ? hi : x);
}

// Byte planes of a signed b-bit value a = sum_p 2^(8p) a_p: planes 0..P-2 are the unsigned low
// bytes, plane P-1 is the signed top byte (arithmetic shift), P = b / 8.
__device__ __forceinline__ uint8_t plane_byte(int64_t a, int p) {
    return static_cast<uint8_t>(static_cast<uint64_t>(a >> (8 * p)) & 0xFFu);
}

}  // namespace eii
