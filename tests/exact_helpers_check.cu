// Host-side check of the engine's exact scalar helpers (compiled by tests/test_exact_helpers_cpu.py):
//   norm_recip_root  U = isqrt(floor(2^80 / (S + eps)))  (python/intref.py:177) against a bisection
//                    on exact 128-bit integers, for random totals and for u^2 Tt near 2^80;
//   prob_q16         floor((e 65536 + floor(Z/2)) / Z)   (python/intref.py:246) against 128-bit division.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <random>

#include "eii_kernels.cuh"

using namespace eii;

static uint64_t isqrt_ref(unsigned __int128 Tt) {
    const unsigned __int128 q = (static_cast<unsigned __int128>(1) << 80) / Tt;
    uint64_t lo = 0, hi = 1ull << 41;
    while (hi - lo > 1) {
        const uint64_t mid = (lo + hi) / 2;
        if (static_cast<unsigned __int128>(mid) * mid <= q) lo = mid; else hi = mid;
    }
    return lo;
}

// Same estimate-and-correct divisions as the attention kernels (host copies of prob_q16 and
// prob_q16_f32: fmaf is correctly rounded on the host as __fmaf_rn is on the device).
static int64_t prob_ref(int64_t e, int64_t Z) { return (e * 65536 + Z / 2) / Z; }
static int64_t prob_fast(int64_t e, int64_t Z) {
    const int64_t n = e * 65536 + Z / 2;
    const double rz = 1.0 / static_cast<double>(Z);
    int64_t p = static_cast<int64_t>(static_cast<double>(n) * rz);
    int64_t r = n - p * Z;
    if (r < 0) { --p; r += Z; }
    if (r < 0) { --p; r += Z; }
    if (r >= Z) { ++p; r -= Z; }
    if (r >= Z) { ++p; }
    return p;
}

static int64_t prob_fast32(int64_t e, int64_t Z) {
    const int64_t n = e * 65536 + Z / 2;
    const float scale = static_cast<float>(65536.0 / static_cast<double>(Z));
    int64_t q = static_cast<int64_t>(floorf(fmaf(static_cast<float>(e), scale, 0.5f)));
    const int64_t r = n - q * Z;
    if (r < 0) --q;
    else if (r >= Z) ++q;
    return q;
}

int main(int argc, char** argv) {
    const long iters = argc > 1 ? atol(argv[1]) : 300000;
    std::mt19937_64 rng(7);
    long n = 0, bad = 0;
    for (long it = 0; it < iters; ++it) {
        const int bits = static_cast<int>(rng() % 73);
        const unsigned __int128 S = ((static_cast<unsigned __int128>(rng()) << 64) | rng()) &
                                    ((static_cast<unsigned __int128>(1) << bits) - 1);
        const int64_t A = static_cast<int64_t>(S >> 32), C = static_cast<int64_t>(S & 0xFFFFFFFFu);
        ++n;
        if (static_cast<uint64_t>(norm_recip_root(A, 0, C)) != isqrt_ref(S + EPS_S)) ++bad;
    }
    for (uint64_t u = 1; u < (1u << 29); u = u * 3 + 1) {
        const unsigned __int128 Tt = (static_cast<unsigned __int128>(1) << 80) / (static_cast<unsigned __int128>(u) * u);
        for (int d = -2; d <= 2; ++d) {
            const unsigned __int128 T2 = Tt + d;
            if (T2 < static_cast<unsigned __int128>(EPS_S) || T2 >= (static_cast<unsigned __int128>(1) << 73)) continue;
            const unsigned __int128 S = T2 - EPS_S;
            ++n;
            if (static_cast<uint64_t>(norm_recip_root(static_cast<int64_t>(S >> 32), 0, static_cast<int64_t>(S & 0xFFFFFFFFu))) !=
                isqrt_ref(T2)) ++bad;
        }
    }
    for (long it = 0; it < iters; ++it) {
        const int64_t Z = (int64_t(1) << 30) + static_cast<int64_t>(rng() % ((int64_t(1) << 39) * 511 / 512));
        const int64_t e = static_cast<int64_t>(rng() % ((int64_t(1) << 30) + 1));
        ++n;
        if (prob_fast(e, Z) != prob_ref(e, Z)) ++bad;
        ++n;
        if (prob_fast32(e, Z) != prob_ref(e, Z)) ++bad;
        const int64_t e2 = static_cast<int64_t>(rng() % 1537);  // small e and e = Z exactly (P = 65536)
        ++n;
        if (prob_fast32(e2, Z) != prob_ref(e2, Z)) ++bad;
        const int64_t zs = int64_t(1) << 30;
        ++n;
        const int64_t z2 = zs + static_cast<int64_t>(rng() % 4);  // a row whose maximum dominates: P near 65536
        if (prob_fast32(zs, z2) != prob_ref(zs, z2)) ++bad;
    }
    printf("checked %ld, mismatches %ld\n", n, bad);
    return bad != 0;
}
