// Independent regeneration of the three model.bin tables (python/intref.py:66-108), host only.
//
//   exp:  E[d]      = floor(2^30 exp(-d/128) + 1/2),                       d in [0, 1536]
//   SiLU: S[i]      = SAT_bits(floor(x / (1 + exp(-x)) 2^f_out + 1/2)),     x = (i - 32768) 2^-f_in
//   RoPE: C[p][j]   = floor(2^30 cos(p theta_j) + 1/2), S[p][j] likewise with sin,
//         theta_j   = 100000^(-2j/64),                                     p < 512, j < 32
//
// The reference evaluates these with mpmath at 50 digits.  Here every value is computed in binary
// fixed point with 320 fractional bits (six 64-bit limbs) from series written out below: exp of a
// dyadic argument as a product of precomputed exp(-2^b) factors (Taylor series with argument
// halving and squaring), 1/(1 + t) by Newton's iteration, pi by Machin's formula, ln 10 from two
// atanh series, cos/sin by Taylor series after reduction by pi/2.  Each result carries a fixed,
// conservative absolute error bound (2^-200 after scaling, against accumulated truncation errors
// near 2^-260); a rounding decision is made only when the whole error interval lies on one side
// of the rounding point, and otherwise the generator reports failure instead of guessing.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace eii {
namespace tables {

constexpr int LIMBS = 6;   // 384 bits
constexpr int FRAC = 320;  // fractional bits: limbs 0..4 are the fraction, limb 5 the integer part

struct Fx {
    uint64_t w[LIMBS];
};
typedef unsigned __int128 u128;

inline Fx fx_zero() {
    Fx r;
    memset(r.w, 0, sizeof(r.w));
    return r;
}
inline Fx fx_int(uint64_t v) {
    Fx r = fx_zero();
    r.w[LIMBS - 1] = v;
    return r;
}
inline bool fx_is_zero(const Fx& a) {
    for (int i = 0; i < LIMBS; ++i)
        if (a.w[i]) return false;
    return true;
}
inline int fx_cmp(const Fx& a, const Fx& b) {
    for (int i = LIMBS - 1; i >= 0; --i)
        if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
    return 0;
}
inline Fx fx_add(const Fx& a, const Fx& b) {
    Fx r;
    u128 c = 0;
    for (int i = 0; i < LIMBS; ++i) {
        c += static_cast<u128>(a.w[i]) + b.w[i];
        r.w[i] = static_cast<uint64_t>(c);
        c >>= 64;
    }
    return r;
}
inline Fx fx_sub(const Fx& a, const Fx& b) {  // a >= b
    Fx r;
    uint64_t borrow = 0;
    for (int i = 0; i < LIMBS; ++i) {
        const uint64_t x = a.w[i], y = b.w[i];
        const uint64_t d = x - y - borrow;
        borrow = (x < y) || (x == y && borrow) ? 1 : 0;
        r.w[i] = d;
    }
    return r;
}
// a * b, truncated to FRAC fractional bits
inline Fx fx_mul(const Fx& a, const Fx& b) {
    uint64_t p[2 * LIMBS];
    memset(p, 0, sizeof(p));
    for (int i = 0; i < LIMBS; ++i) {
        if (!a.w[i]) continue;
        u128 c = 0;
        for (int j = 0; j < LIMBS; ++j) {
            c += static_cast<u128>(a.w[i]) * b.w[j] + p[i + j];
            p[i + j] = static_cast<uint64_t>(c);
            c >>= 64;
        }
        for (int k = i + LIMBS; c && k < 2 * LIMBS; ++k) {
            c += p[k];
            p[k] = static_cast<uint64_t>(c);
            c >>= 64;
        }
    }
    Fx r;
    for (int i = 0; i < LIMBS; ++i) r.w[i] = p[i + FRAC / 64];  // FRAC is a multiple of 64
    return r;
}
inline Fx fx_mul_u(const Fx& a, uint64_t m) {
    Fx r;
    u128 c = 0;
    for (int i = 0; i < LIMBS; ++i) {
        c += static_cast<u128>(a.w[i]) * m;
        r.w[i] = static_cast<uint64_t>(c);
        c >>= 64;
    }
    return r;
}
inline Fx fx_div_u(const Fx& a, uint64_t d) {  // truncated
    Fx r;
    u128 rem = 0;
    for (int i = LIMBS - 1; i >= 0; --i) {
        const u128 cur = (rem << 64) | a.w[i];
        r.w[i] = static_cast<uint64_t>(cur / d);
        rem = cur % d;
    }
    return r;
}
inline Fx fx_shr(const Fx& a, int s) {  // s >= 0, truncated
    Fx r = fx_zero();
    const int q = s / 64, b = s % 64;
    for (int i = 0; i + q < LIMBS; ++i) {
        uint64_t v = a.w[i + q] >> b;
        if (b && i + q + 1 < LIMBS) v |= a.w[i + q + 1] << (64 - b);
        r.w[i] = v;
    }
    return r;
}
inline Fx fx_shl(const Fx& a, int s) {  // s >= 0; the caller keeps the value below 2^64
    Fx r = fx_zero();
    const int q = s / 64, b = s % 64;
    for (int i = LIMBS - 1; i - q >= 0; --i) {
        uint64_t v = a.w[i - q] << b;
        if (b && i - q - 1 >= 0) v |= a.w[i - q - 1] >> (64 - b);
        r.w[i] = v;
    }
    return r;
}
// 2^-k as a fixed-point value (k <= FRAC)
inline Fx fx_pow2neg(int k) {
    Fx r = fx_zero();
    const int bit = FRAC - k;
    r.w[bit / 64] = uint64_t(1) << (bit % 64);
    return r;
}

// exp(-u) for 0 <= u <= 2^-8: Taylor series until the term vanishes (alternating, so the error is
// below the first omitted term).
inline Fx exp_neg_small(const Fx& u) {
    Fx sum = fx_int(1), neg = fx_zero(), term = fx_int(1);
    for (int k = 1; k < 200; ++k) {
        term = fx_div_u(fx_mul(term, u), k);
        if (fx_is_zero(term)) break;
        if (k & 1) neg = fx_add(neg, term);
        else sum = fx_add(sum, term);
    }
    return fx_sub(sum, neg);
}
// exp(-y) for 0 <= y < 2^63: y = u 2^h with u <= 2^-8, exp(-y) = exp(-u)^(2^h).
inline Fx exp_neg(const Fx& y) {
    int h = 0;
    Fx u = y;
    const Fx lim = fx_pow2neg(8);
    while (fx_cmp(u, lim) > 0) {
        u = fx_shr(u, 1);  // loses at most one ulp per halving of the argument
        ++h;
    }
    Fx r = exp_neg_small(u);
    for (int i = 0; i < h && !fx_is_zero(r); ++i) r = fx_mul(r, r);
    return r;
}

// exp(-2^b) for b in [B_LO, B_HI]: the factors of exp(-k 2^-f) over the set bits of k.
struct ExpFactors {
    static constexpr int B_LO = -40, B_HI = 20;
    Fx fac[B_HI - B_LO + 1];
    ExpFactors() {
        for (int b = B_LO; b <= B_HI; ++b) fac[b - B_LO] = exp_neg(b >= 0 ? fx_int(uint64_t(1) << b) : fx_pow2neg(-b));
    }
    // exp(-k 2^-f), k >= 0
    Fx exp_dyadic(uint64_t k, int f) const {
        Fx r = fx_int(1);
        for (int i = 0; i < 64 && (k >> i); ++i)
            if ((k >> i) & 1) {
                const int b = i - f;
                if (b > B_HI) return fx_zero();  // exp(-2^21) underflows far below 2^-320
                r = fx_mul(r, fac[b - B_LO]);
            }
        return r;
    }
};

// 1 / (1 + t) for 0 <= t <= 1, by Newton's iteration r <- r (2 - (1 + t) r) from a double seed.
inline Fx recip_one_plus(const Fx& t) {
    const Fx d = fx_add(fx_int(1), t);
    const double dd = 1.0 + static_cast<double>(t.w[LIMBS - 1]) + std::ldexp(static_cast<double>(t.w[LIMBS - 2] >> 11), -53);
    double seed = 1.0 / dd;
    Fx r = fx_zero();
    {   // seed as fixed point (53 bits)
        const uint64_t m = static_cast<uint64_t>(std::ldexp(seed, 62));
        r.w[LIMBS - 2] = m << 2;
        r.w[LIMBS - 1] = m >> 62;
    }
    const Fx two = fx_int(2);
    for (int it = 0; it < 4; ++it) r = fx_mul(r, fx_sub(two, fx_mul(d, r)));
    return r;
}

// atan(1/n) = sum (-1)^k / ((2k+1) n^(2k+1)) and atanh(1/n) = sum 1 / ((2k+1) n^(2k+1))
inline Fx arc_series(uint64_t n, bool alternating) {
    Fx pos = fx_zero(), neg = fx_zero();
    Fx p = fx_div_u(fx_int(1), n);  // n^-(2k+1)
    for (uint64_t k = 0; !fx_is_zero(p); ++k) {
        const Fx t = fx_div_u(p, 2 * k + 1);
        if (alternating && (k & 1)) neg = fx_add(neg, t);
        else pos = fx_add(pos, t);
        p = fx_div_u(fx_div_u(p, n), n);
    }
    return fx_sub(pos, neg);
}
inline Fx fx_pi() {  // Machin: pi = 16 atan(1/5) - 4 atan(1/239)
    return fx_sub(fx_mul_u(arc_series(5, true), 16), fx_mul_u(arc_series(239, true), 4));
}
inline Fx fx_ln10() {  // ln 10 = 3 ln 2 + ln(5/4), ln 2 = 2 atanh(1/3), ln(5/4) = 2 atanh(1/9)
    return fx_add(fx_mul_u(arc_series(3, false), 6), fx_mul_u(arc_series(9, false), 2));
}

// cos and sin of 0 <= r <= 2 by Taylor series (alternating; error below the first omitted term)
inline void cos_sin_small(const Fx& r, Fx& c, Fx& s) {
    const Fx r2 = fx_mul(r, r);
    Fx cp = fx_int(1), cn = fx_zero(), sp = r, sn = fx_zero();
    Fx tc = fx_int(1), ts = r;
    for (uint64_t k = 1; k < 200; ++k) {
        tc = fx_div_u(fx_div_u(fx_mul(tc, r2), 2 * k - 1), 2 * k);
        ts = fx_div_u(fx_div_u(fx_mul(ts, r2), 2 * k), 2 * k + 1);
        if (fx_is_zero(tc) && fx_is_zero(ts)) break;
        if (k & 1) { cn = fx_add(cn, tc); sn = fx_add(sn, ts); }
        else { cp = fx_add(cp, tc); sp = fx_add(sp, ts); }
    }
    // callers pass 0 <= r < pi/2, where cos and sin are >= 0; a computed value a few ulps below 0
    // (only for r within rounding error of pi/2 or 0) is clamped, and such values round to 0
    c = fx_cmp(cp, cn) >= 0 ? fx_sub(cp, cn) : fx_zero();
    s = fx_cmp(sp, sn) >= 0 ? fx_sub(sp, sn) : fx_zero();
}

// The integer floor(sign * v + 1/2) for |value| = v, if the error interval [v - 2^-200, v + 2^-200]
// does not contain a rounding point; ok = false otherwise.
inline int64_t round_half_up(bool neg, const Fx& v, bool& ok) {
    const Fx eps = fx_pow2neg(200);
    const Fx half = fx_pow2neg(1);
    Fx w;
    int64_t sign = 1;
    if (!neg) {
        w = fx_add(v, half);  // floor(v + 1/2)
    } else if (fx_cmp(v, half) <= 0) {
        w = fx_sub(half, v);  // 1/2 - v in [0, 1/2]: floor is 0, unless v is within eps of 1/2
        const Fx frac = w;
        if (fx_cmp(frac, eps) < 0 && !fx_is_zero(v)) ok = false;
        return 0;
    } else {
        w = fx_sub(v, half);  // floor(1/2 - v) = -ceil(v - 1/2)
        sign = -1;
    }
    Fx frac = w;
    frac.w[LIMBS - 1] = 0;
    const int64_t ip = static_cast<int64_t>(w.w[LIMBS - 1]);
    // a rounding point within the error bound (including a value that lands on it exactly, which
    // the computed value can do when the true value is only close, e.g. after exp(-x) underflows)
    // cannot be decided at this precision
    if (fx_cmp(frac, eps) < 0 || fx_cmp(fx_sub(fx_int(1), frac), eps) < 0) ok = false;
    if (sign > 0) return ip;
    return -(ip + (fx_is_zero(frac) ? 0 : 1));
}

// E[d] = floor(2^30 exp(-d/128) + 1/2), d in [0, 1536]
inline bool exp_table(int64_t* out) {
    const ExpFactors F;
    bool ok = true;
    for (int d = 0; d <= 1536; ++d) out[d] = round_half_up(false, fx_shl(F.exp_dyadic(d, 7), 30), ok);
    return ok;
}

// SiLU table over the 65536 INT16 inputs (python/intref.py:81-93)
inline bool silu_table(int f_in, int f_out, int bits, int64_t* out) {
    if (f_in < 0 || f_in > 40 || f_out < -20 || f_out > 40 || bits < 2 || bits > 63) return false;
    const ExpFactors F;
    bool ok = true;
    const int64_t hi = (int64_t(1) << (bits - 1)) - 1, lo = -hi - 1;
    for (int i = 0; i < 65536; ++i) {
        const int64_t k = i - 32768;
        const uint64_t ak = static_cast<uint64_t>(k < 0 ? -k : k);
        // sigmoid part: x >= 0: 1 / (1 + e^-x); x < 0: e^x / (1 + e^x) = t / (1 + t), t = e^-|x|
        const Fx t = F.exp_dyadic(ak, f_in);
        const Fx r = recip_one_plus(t);
        const Fx sig = k >= 0 ? r : fx_mul(t, r);
        // |x| sigmoid 2^f_out = ak sigmoid 2^(f_out - f_in)
        Fx v = fx_mul_u(sig, ak);
        const int sh = f_out - f_in;
        v = sh >= 0 ? fx_shl(v, sh) : fx_shr(v, -sh);
        int64_t q = round_half_up(k < 0, v, ok);
        out[i] = q < lo ? lo : (q > hi ? hi : q);
    }
    return ok;
}

// RoPE tables C[p][j], S[p][j] = floor(2^30 cos/sin(p theta_j) + 1/2), p < n_pos, j < 32
inline bool rope_tables(int n_pos, int64_t* cos_out, int64_t* sin_out) {
    const Fx pi = fx_pi(), half_pi = fx_shr(pi, 1);
    const Fx ln1e5 = fx_mul_u(fx_ln10(), 5);
    bool ok = true;
    for (int j = 0; j < 32; ++j) {
        const Fx theta = exp_neg(fx_div_u(fx_mul_u(ln1e5, 2 * j), 64));  // 100000^(-2j/64)
        for (int p = 0; p < n_pos; ++p) {
            const Fx z = fx_mul_u(theta, p);
            // z = q pi/2 + r, 0 <= r < pi/2
            uint64_t q = 0;
            {
                const double zd = static_cast<double>(z.w[LIMBS - 1]) + std::ldexp(static_cast<double>(z.w[LIMBS - 2]), -64);
                const double hp = 1.5707963267948966;
                q = static_cast<uint64_t>(zd / hp);
                if (q > 0) --q;  // start below and step up exactly
            }
            Fx base = fx_mul_u(half_pi, q);
            while (fx_cmp(fx_add(base, half_pi), z) <= 0) { base = fx_add(base, half_pi); ++q; }
            const Fx r = fx_sub(z, base);
            Fx c, s;
            cos_sin_small(r, c, s);
            // cos(q pi/2 + r), sin(q pi/2 + r) by quadrant
            Fx cv, sv;
            bool cneg, sneg;
            switch (q & 3) {
                case 0: cv = c; cneg = false; sv = s; sneg = false; break;
                case 1: cv = s; cneg = true; sv = c; sneg = false; break;
                case 2: cv = c; cneg = true; sv = s; sneg = true; break;
                default: cv = s; cneg = false; sv = c; sneg = true; break;
            }
            cos_out[p * 32 + j] = round_half_up(cneg, fx_shl(cv, 30), ok);
            sin_out[p * 32 + j] = round_half_up(sneg, fx_shl(sv, 30), ok);
        }
    }
    return ok;
}

}  // namespace tables
}  // namespace eii
