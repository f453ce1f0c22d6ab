// Byte-plane integer GEMM on tcgen05 kind::i8 with fused fixed-point epilogues.
//
// Computes, for activation a [M,K] of b = 8P bits and int8 weights W [N,K],
//     acc[m,n] = sum_k a[m,k] W[n,k]               (exact)
// as  acc = sum_p 2^(8p) (a_p W^T),  a_p the byte planes of a (u8 low planes, s8 top plane).
// Each plane product accumulates in its own int32 TMEM accumulator; it cannot overflow:
//     |a_p w| <= 255 * 127 = 32385 per product, and K <= 1536 gives <= 49,743,360 < 2^31 - 1
//     (the bound holds for K up to 66,311).  Planes are combined in int64 in the epilogue:
//     |acc| <= 2^31 * 127 * 1536 < 2^48.6, and acc * m <= 2^48.6 * 2^14 < 2^63, the bound the
//     reference asserts (python/intref.py:189,259,279).
//
// Kernel structure (one CTA per SM, persistent over 128x128 output tiles, m-block major):
//   warp 0      TMA producer: per 128-wide K block, P activation-plane tiles [128 x 128 B] and one
//               weight tile [128 x 128 B], 128-byte swizzle, into a STAGES-deep smem ring.
//   warp 1      TMEM allocator + single-thread MMA issuer: 4 (or 2 for a half block) K=32 steps
//               x P planes of tcgen05.mma.cta_group::1.kind::i8, M=128, N=n_valid.
//   warps 2..   epilogue warps (16, 4 per TMEM lane quadrant; 8, 2 per quadrant, for gate/up and
//               QKV, see GemmCfg::EPI_WARPS): tcgen05.ld of the P accumulators, plane combination,
//               requantise RS/SAT, and the fused step of the caller (RoPE, residual add, SiLU-gated
//               product, logits and digest), stored through shared-memory staging and TMA (or
//               straight to the row-blocked gated planes).
// TMEM: P*BN int32 columns per accumulator set; 2 sets (double buffered) for P = 2, one for P = 4.
#pragma once
#include <cstdint>
#include <cuda.h>

#include "eii_int.cuh"
#include "eii_ptx.cuh"

namespace eii {

enum EpiKind : int { EPI_QKV = 0, EPI_RESID = 1, EPI_GATEUP = 2, EPI_LOGITS = 3, EPI_LINEAR = 4, EPI_SWEEP = 5 };

// Error codes written to the engine's device error word.
enum : int {
    ERR_TIMEOUT_PRODUCER = 101,
    ERR_TIMEOUT_MMA_FULL = 102,
    ERR_TIMEOUT_MMA_ACC = 103,
    ERR_TIMEOUT_EPI = 104,
    ERR_TIMEOUT_DRAIN = 105,
    ERR_TIMEOUT_ATTN = 106,
};

struct EpiParams {
    int M, N, K;
    const int2* msh;  // per output column: (m, shift = n + f_in - f_out), in tile-column order
    int* err;
    // EPI_QKV: q [M,576] k [M,192] v [M,192] int16; RoPE tables int32 [512,32]; position = row % T
    int T;
    int pos0;  // position of the first row of each T-row sequence (incremental decoding: the step's position)
    int16_t* q_out;
    int16_t* k_out;
    int16_t* v_out;
    const int32_t* rope_c;
    const int32_t* rope_s;
    int bits_q, bits_k, bits_v, bits_qr, bits_kr, rope_shift_q, rope_shift_k;
    // EPI_RESID: x [M,N] int32, x = SAT32(x + RS(acc m, shift))
    int32_t* x;
    // EPI_GATEUP: gate/up interleaved by tile (cols 0-63 gate j, 64-127 up j), gated -> planes.
    // SiLU: the full 65536-entry table (global), or, when silu_smem is set, its compact form
    //   tab[g] = neg[-|g| - lo] (0 below lo) for g <= 0,  SAT_bits_s(neg[-g - lo] + g * 2^silu_d) for g > 0
    // (silu(x) - silu(-x) = x exactly, so with f_s >= f_g the rounded table obeys it; the engine
    // verifies it for all 65536 inputs before enabling it), staged once per CTA in shared memory.
    const int32_t* silu;
    const void* silu_neg;
    int silu_smem, silu_lo, silu_count, silu_wide, silu_d, bits_s;
    // fast = every column shift is in [1, 31] and every m in [0, 2^15), the RoPE shifts are in
    // [1, 31] and the gated-product shift in [0, 31]: requantisation then runs on 32x32->64
    // multiply-adds and 32-bit funnel shifts; otherwise the generic int64 path is taken.
    int fast;
    // narrow = for every column, |acc m| + 2^(shift-1) < 2^(31 + shift) (checked on the host from the
    // L1 norm of each weight row and the activation range), so RS(acc m, shift) fits int32 and
    // needs no 64-bit saturation test; the RoPE shifts are >= 16 for the same reason.
    int narrow;
    int bits_g, bits_u, gated_shift, bits_m, gated_P;
    // acc32 = for every column, 2^(b-1) * sum_k |W[col][k]| < 2^31 (host-checked): the two-plane
    // accumulator acc = v0 + 2^8 v1 fits int32, so the narrow requantisation needs one 32x32->64
    // multiply-add instead of two
    int acc32;
    // gated planes in the row-blocked layout [gated_P][ceil(M/128)][N/32][128 rows][16 bytes]: each
    // 16-feature group of a 128-row block is one 2 KB run, so an epilogue warp's 32 rows x 16 features
    // of a plane are 512 contiguous bytes (coalesced stores).  The down GEMM reads it with a 4-D map.
    uint8_t* gated_planes;
    // A operand in that row-blocked layout (4-D map, no swizzle) instead of [P][M][K] with 128-byte swizzle
    int a_blocked;
    // Signed-digit gated planes (host-proven |gated| <= 2^30): gated = sum_p 2^(8p) d_p with every digit
    // d_p in [-128, 127]; the digit bytes are the bytes of (gated + 0x808080) ^ 0x808080, and the top
    // digit (byte 3 of gated + 0x808080) is 0 for gated in [-0x808080, 0x7F7F7F].  sd_flags[m_blk]
    // != 0 marks a 128-row block where some top digit is not 0.  EPI_GATEUP writes the digits and
    // the flags; the down GEMM (EPI_RESID, P = 4) skips the top plane (loads and MMAs) in blocks
    // whose flag is 0.  a_sd: the A planes are signed digits (every plane multiplied as s8).
    uint32_t* sd_flags;
    int a_sd;
    // EPI_GATEUP: write the gated planes in offset binary (the bytes of gated + 2^(8 gated_P - 1): all
    // unsigned, the top byte's sign bit flipped), the layout the feature-major down GEMM reads.
    int gated_offset;
    // A planes in offset binary (EPI_LINEAR): every plane is multiplied as unsigned and a_corr[col] =
    // 2^(b-1) sum_k W[col][k] is subtracted from the combined accumulator.
    const int64_t* a_corr;
    // EPI_LOGITS: int32 out[row * ld + col] = RS(acc m, shift) (low 32 bits, no SAT)
    int32_t* logits;
    int64_t ld_logits;
    // EPI_LOGITS, optional per-sequence digest of the logits (sequence = row / T, position t = pos0 + row % T):
    //   dig[seq] += sum over (t, v) of uint32(logit) * dig_b[v] * dig_a[t]  (mod 2^64)
    // accumulated per row in registers over a CTA's contiguous run of tiles, one atomic per row and run.
    unsigned long long* dig;
    const uint64_t* dig_a;
    const uint64_t* dig_b;
    // EPI_LINEAR: int64 out = SAT(RS(acc m, shift), bits_out), optional int64 acc
    int64_t* out64;
    int64_t* acc64;
    int bits_out;
    // EPI_SWEEP (the stand-alone contraction, python/intref.py:186-190, on device buffers):
    //   int32 logits[row * ld_logits + col] = SAT_bits_out(RS(acc m, shift)), bits_out <= 32; optional
    //   per-row digests  dig[row] += sum_col uint32(out) * dig_b[col]  and
    //   dig_acc[row] += sum_col uint64(acc) * dig_b[col]  (mod 2^64, acc the exact int64 contraction).
    unsigned long long* dig_acc;
    // EPI_LINEAR, tests only: when non-zero, each epilogue warp first waits this many ns on a barrier
    // that nothing arrives on, so the bounded wait runs out and the CTA takes its abort-and-drain path
    // (error ERR_TIMEOUT_EPI); the engine sets it from EII_TEST_STALL_NS in eii_linear.
    unsigned long long test_stall_ns;
};

constexpr int SILU_SMEM_BYTES = 48 * 1024;  // compact SiLU table capacity (int16 x 24576 or int32 x 12288)
// RoPE rows staged by the QKV GEMM: up to 128 positions; a 36-word pitch puts the 16-byte loads of
// eight consecutive positions (one per lane) on distinct banks.
constexpr int ROPE_SMEM_ROWS = 128, ROPE_SMEM_PITCH = 36;
constexpr int SMEM_LIMIT = 227 * 1024;
// N-tile width of the 4-plane GEMMs (down, and O at INT32 attn_ctx layers).  128 keeps their
// operand traffic from L2 at the level of the 2-plane GEMMs (the mainloops are L2-bound) at the
// price of a single TMEM accumulator set; 64 would double-buffer the accumulators.
constexpr int BN_P4 = 128;

template <int P, int KIND>
struct GemmCfg {
    // P = 4 uses BN_P4-wide N tiles (128: one accumulator set, so its epilogue does not overlap the
    // next tile's MMAs; 64 would double-buffer them at twice the operand traffic, measured slower).
    static constexpr int BM = 128, BN = (P == 4) ? BN_P4 : 128, BK = 128;
    static constexpr int ACC_COLS = P * BN;
    static constexpr int NB = 512 / ACC_COLS;  // accumulator sets in TMEM
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = P * A_BYTES + B_BYTES;
    // Per-warp staging buffer for TMA tile stores (and the residual tile load): 32 rows x the warp's
    // columns.  LOGITS/RESID: int32, BN/4 columns; QKV: two 32-row x 16 int16 boxes.
    // RESID with 4 planes and 128-wide tiles keeps one 16-column chunk resident (2 KB) to fit.
    // SWEEP: as LOGITS with two planes; with four (and 128-wide tiles) one 16-column chunk (2 KB) to fit.
    static constexpr int STG_BYTES = KIND == EPI_LOGITS ? (BN / 4) * 4 * 32
                                     : (KIND == EPI_RESID || KIND == EPI_SWEEP) ? ((P == 4 && BN == 128) ? 2048 : (BN / 4) * 4 * 32)
                                     : (KIND == EPI_QKV ? 2048 : 0);
    static constexpr int STAGES = (P == 2) ? (KIND == EPI_LINEAR ? 4 : 3) : (BN == 128 ? 2 : 3);
    // Epilogue warps: 4 per TMEM lane quadrant, each owning one 32-column group of the tile.  Gate/up
    // and QKV use 2 per quadrant, each taking two column groups in turn (with a staging buffer for
    // each): 10 warps in all put at most 3 warps on an SM sub-partition, so these heavy epilogues get
    // 168 registers instead of 96 and do not spill (18 warps put 5 on two sub-partitions: 16384 /
    // (5 x 32) registers per thread); measured -10% (gate/up) and -6% (QKV).  The logits epilogue does
    // not spill at 96 and ran 5% slower with 8 warps; the residual epilogue loads one residual tile
    // per warp.  Both keep 16.  (The feature-major GEMM's 4-plane residual epilogue with 8 warps, two
    // row quarters each, stopped spilling but ran 30% slower: its per-row residual loads are latency
    // bound, and half the warps keep half as many in flight.)
    static constexpr int EPI_WARPS = (KIND == EPI_GATEUP || KIND == EPI_QKV) ? 8 : 16;
    static constexpr int CG_PER_WARP = 16 / EPI_WARPS;
    static constexpr int EPI_THREADS = 32 * EPI_WARPS;
    static constexpr int THREADS = 64 + EPI_THREADS;
    static constexpr int BAR_BYTES = 512;
    static constexpr int COLP_BYTES = 2 * BN * 16;  // per-tile column (m, shift, 2^(shift-1), m << 8), x2
    static constexpr int DIGW_BYTES = (KIND == EPI_LOGITS || KIND == EPI_SWEEP) ? 2 * BN * 8 : 0;  // per-tile digest column weights, x2
    static constexpr int SILU_BYTES = KIND == EPI_GATEUP ? SILU_SMEM_BYTES : 0;
    // QKV: the RoPE cos/sin rows of positions pos0 .. pos0 + T - 1 (T <= 128), rows padded to 36 words
    static constexpr int ROPE_BYTES = KIND == EPI_QKV ? 2 * ROPE_SMEM_ROWS * ROPE_SMEM_PITCH * 4 : 0;
    static constexpr int STG_OFFSET = STAGES * STAGE_BYTES;  // 1024-aligned
    static constexpr int BAR_OFFSET = STG_OFFSET + EPI_WARPS * CG_PER_WARP * STG_BYTES;
    static constexpr int SMEM = BAR_OFFSET + 1024 + BAR_BYTES + COLP_BYTES + DIGW_BYTES + SILU_BYTES + ROPE_BYTES;
    static_assert(NB >= 1, "accumulators must fit in TMEM");
    static_assert(STG_BYTES % 1024 == 0, "staging buffers are 1024-byte aligned");
    static_assert(SMEM <= SMEM_LIMIT, "shared memory budget");
};

// Barrier of the nthreads epilogue threads (named barrier 1) that also ANDs a flag across them, so
// that a timed-out wait in one warp makes every epilogue warp leave together.
__device__ __forceinline__ bool epi_barrier_and(bool v, uint32_t nthreads) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, 1, %2, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "r"(nthreads)
        : "memory");
    return r != 0;
}

// ------------------------------------------------------------------------------ epilogue math
// Raw int32 plane accumulators of 16 consecutive columns of this thread's row.
// Plane p of an accumulator set starts at column p * BN (BN = 128 for P = 2, 64 for P = 4).
template <int P, int N>
__device__ __forceinline__ void load_planes(uint32_t taddr, uint32_t (&v)[P][N]) {
    static_assert(N == 8 || N == 16, "8 or 16 columns");
    constexpr int PS = (P == 4) ? BN_P4 : 128;
#pragma unroll
    for (int p = 0; p < P; ++p) {
        if constexpr (N == 16) tmem_ld16(taddr + p * PS, v[p]);
        else tmem_ld8(taddr + p * PS, v[p]);
    }
    tmem_wait_ld();
#pragma unroll
    for (int p = 0; p < P; ++p) tmem_launder(v[p]);
}

// Two sets of columns (e.g. gate and up, or RoPE partners d and d + 32) behind one wait::ld, so the
// second set's TMEM latency overlaps the first's.
template <int P, int N>
__device__ __forceinline__ void load_planes2(uint32_t ta, uint32_t (&va)[P][N], uint32_t tb, uint32_t (&vb)[P][N]) {
    static_assert(N == 8 || N == 16, "8 or 16 columns");
    constexpr int PS = (P == 4) ? BN_P4 : 128;
#pragma unroll
    for (int p = 0; p < P; ++p) {
        if constexpr (N == 16) {
            tmem_ld16(ta + p * PS, va[p]);
            tmem_ld16(tb + p * PS, vb[p]);
        } else {
            tmem_ld8(ta + p * PS, va[p]);
            tmem_ld8(tb + p * PS, vb[p]);
        }
    }
    tmem_wait_ld();
#pragma unroll
    for (int p = 0; p < P; ++p) {
        tmem_launder(va[p]);
        tmem_launder(vb[p]);
    }
}

template <int P, int N>
__device__ __forceinline__ int64_t combine(const uint32_t (&v)[P][N], int i) {
    int64_t a = 0;
#pragma unroll
    for (int p = 0; p < P; ++p) a += static_cast<int64_t>(static_cast<int32_t>(v[p][i])) * (int64_t(1) << (8 * p));
    return a;
}

// Generic path: RS with a per-column shift >= 1 (an array shift of the reference, which
// python/intref.py:49 requires to be >= 1; the engine rejects models and arguments that violate it).
__device__ __forceinline__ int64_t rs_col(int64_t x, int n) {
    return static_cast<int64_t>(static_cast<uint64_t>(x) + (static_cast<uint64_t>(1) << (n - 1))) >> n;
}

// Fast path: acc * m + 2^(sh-1) built directly from the int32 plane accumulators,
// sum_p d_p (m 2^(8p)) + rnd, with 32x32 -> 64 multiply-adds (exact: the total is < 2^63).
template <int P, int N>
__device__ __forceinline__ int64_t mulround(const uint32_t (&v)[P][N], int i, int4 cp) {
    int64_t t = static_cast<int64_t>(static_cast<int32_t>(v[0][i])) * cp.x + static_cast<int64_t>(static_cast<uint32_t>(cp.z));
    t += static_cast<int64_t>(static_cast<int32_t>(v[1][i])) * cp.w;
    if constexpr (P == 4) {
        t += static_cast<int64_t>(static_cast<int32_t>(v[2][i])) * (cp.x << 16);
        t += (static_cast<int64_t>(static_cast<int32_t>(v[3][i])) * cp.x) * (int64_t(1) << 24);
    }
    return t;
}

// t >> sh for 1 <= sh <= 31 as (hi, lo) words, by funnel shift.
__device__ __forceinline__ void shr31(int64_t t, int sh, int32_t& hi, uint32_t& lo) {
    const uint32_t tl = static_cast<uint32_t>(t), th = static_cast<uint32_t>(static_cast<uint64_t>(t) >> 32);
    lo = __funnelshift_r(tl, th, sh);
    hi = static_cast<int32_t>(th) >> sh;
}

// SAT to `bits` (<= 32) of the 64-bit value (hi, lo).
__device__ __forceinline__ int32_t sat_hl(int32_t hi, uint32_t lo, int bits) {
    const bool fits = hi == (static_cast<int32_t>(lo) >> 31);
    int32_t v = fits ? static_cast<int32_t>(lo) : (hi < 0 ? INT32_MIN : INT32_MAX);
    if (bits < 32) {
        const int32_t lim = 1 << (bits - 1);
        v = min(max(v, -lim), lim - 1);
    }
    return v;
}

// Narrow requantisation: RS(acc m, sh) is known to fit int32 (EpiParams::narrow).
template <int P, int N>
__device__ __forceinline__ int32_t rs_narrow(const uint32_t (&v)[P][N], int i, int4 cp) {
    const int64_t t = mulround<P, N>(v, i, cp);
    return static_cast<int32_t>(
        __funnelshift_r(static_cast<uint32_t>(t), static_cast<uint32_t>(static_cast<uint64_t>(t) >> 32), cp.y));
}
__device__ __forceinline__ int32_t clamp16(int32_t v) { return min(max(v, -32768), 32767); }

// Narrow requantisation with the two-plane accumulator combined in 32 bits (EpiParams::acc32).
template <int P, int N>
__device__ __forceinline__ int32_t rs_acc32(const uint32_t (&v)[P][N], int i, int4 cp) {
    const int32_t acc = static_cast<int32_t>(v[0][i]) + static_cast<int32_t>(v[1][i] << 8);
    const int64_t t = static_cast<int64_t>(acc) * cp.x + static_cast<int64_t>(static_cast<uint32_t>(cp.z));
    return static_cast<int32_t>(
        __funnelshift_r(static_cast<uint32_t>(t), static_cast<uint32_t>(static_cast<uint64_t>(t) >> 32), cp.y));
}

// Fast requantisation of one element: SAT_bits(RS(acc m, sh)).
template <int P, int N>
__device__ __forceinline__ int32_t requant_fast(const uint32_t (&v)[P][N], int i, int4 cp, int bits) {
    int32_t hi;
    uint32_t lo;
    shr31(mulround<P, N>(v, i, cp), cp.y, hi, lo);
    return sat_hl(hi, lo, bits);
}

// Generic requantisation (any shift in [1, 62]); bits may be up to 64.
template <int P, int N>
__device__ __forceinline__ int64_t requant_gen(const uint32_t (&v)[P][N], int i, int4 cp, int bits) {
    return sat64(rs_col(combine<P, N>(v, i) * static_cast<int64_t>(cp.x), cp.y), bits);
}

__device__ __forceinline__ int64_t silu_lookup(const EpiParams& ep, const void* tab_smem, int g) {
    if (!ep.silu_smem) return __ldg(ep.silu + (g + 32768));
    const int a = g < 0 ? g : -g;
    int64_t t = 0;
    if (a >= ep.silu_lo) {
        t = ep.silu_wide ? static_cast<const int32_t*>(tab_smem)[a - ep.silu_lo]
                         : static_cast<const int16_t*>(tab_smem)[a - ep.silu_lo];
    }
    if (g > 0) t = sat64(t + (static_cast<int64_t>(g) << ep.silu_d), ep.bits_s);
    return t;
}

// Byte plane p of 16 values -> one 16-byte vector (three byte permutes per 4 values).
template <int PL, int N>
__device__ __forceinline__ void pack_plane(const int32_t (&x)[N], uint32_t (&w)[N / 4]) {
    constexpr uint32_t sel = PL | ((4 + PL) << 4);
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
        const uint32_t t01 = __byte_perm(static_cast<uint32_t>(x[4 * q]), static_cast<uint32_t>(x[4 * q + 1]), sel);
        const uint32_t t23 = __byte_perm(static_cast<uint32_t>(x[4 * q + 2]), static_cast<uint32_t>(x[4 * q + 3]), sel);
        w[q] = __byte_perm(t01, t23, 0x5410);
    }
}

// All byte planes of N values at once by a byte transpose of each group of four: planes 0 and 1
// (two permutes each per four values, against three per plane one plane at a time), and with
// FOUR, planes 2 and 3 as well (eight permutes per four values for the four planes, against twelve).
template <int N, bool FOUR>
__device__ __forceinline__ void pack_planes(const int32_t (&x)[N], uint32_t (&w0)[N / 4], uint32_t (&w1)[N / 4],
                                            uint32_t (&w2)[N / 4], uint32_t (&w3)[N / 4]) {
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
        const uint32_t x0 = static_cast<uint32_t>(x[4 * q]), x1 = static_cast<uint32_t>(x[4 * q + 1]);
        const uint32_t x2 = static_cast<uint32_t>(x[4 * q + 2]), x3 = static_cast<uint32_t>(x[4 * q + 3]);
        const uint32_t t0 = __byte_perm(x0, x1, 0x5140), t2 = __byte_perm(x2, x3, 0x5140);  // bytes 0, 1 of each
        w0[q] = __byte_perm(t0, t2, 0x5410);
        w1[q] = __byte_perm(t0, t2, 0x7632);
        if constexpr (FOUR) {
            const uint32_t t1 = __byte_perm(x0, x1, 0x7362), t3 = __byte_perm(x2, x3, 0x7362);  // bytes 2, 3
            w2[q] = __byte_perm(t1, t3, 0x5410);
            w3[q] = __byte_perm(t1, t3, 0x7632);
        }
    }
}

// Gate/up/SiLU/gated product for 16 features, all-32-bit path: INT16 gate and up, compact INT16
// SiLU table with shift d <= 15 (so g * 2^d < 2^31), gated shift in [0, 31].
// The compact table holds count = 1 - lo_g entries for inputs lo_g .. 0 and a zero past them
// (tab[count] = 0), so inputs below lo_g map there by an unsigned min instead of a test.
template <int P, int N, int BITS_M, bool NARROW, bool ACC32>
__device__ __forceinline__ void gateup_lean(const uint32_t (&vg)[P][N], const uint32_t (&vu)[P][N], const int4* cpg,
                                            const int4* cpu, const int16_t* tab, int lo_g, int count, int d, int gs,
                                            int64_t grnd, int32_t (&gm)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int32_t g = ACC32 ? clamp16(rs_acc32<P, N>(vg, i, cpg[i]))
                                : (NARROW ? clamp16(rs_narrow<P, N>(vg, i, cpg[i])) : requant_fast<P, N>(vg, i, cpg[i], 16));
        const int32_t u = ACC32 ? clamp16(rs_acc32<P, N>(vu, i, cpu[i]))
                                : (NARROW ? clamp16(rs_narrow<P, N>(vu, i, cpu[i])) : requant_fast<P, N>(vu, i, cpu[i], 16));
        const int32_t a = min(g, -g);
        const uint32_t idx = min(static_cast<uint32_t>(a - lo_g), static_cast<uint32_t>(count));
        // silu(g) = silu(-|g|) + g 2^d for g > 0 (SAT16), the table value itself for g <= 0
        const int32_t sg = min(max(static_cast<int32_t>(tab[idx]) + (max(g, 0) << d), -32768), 32767);
        // |sg u| <= 2^30 and 2^(gs-1) <= 2^30, so RS(sg u, gs) lies in [-2^30, 2^30]: it fits int32 and
        // SAT32 never applies; SAT16 is a clamp of that int32
        const int64_t prod = static_cast<int64_t>(sg) * u + grnd;
        const int32_t r = static_cast<int32_t>(
            __funnelshift_r(static_cast<uint32_t>(prod), static_cast<uint32_t>(static_cast<uint64_t>(prod) >> 32), gs));
        gm[i] = BITS_M == 32 ? r : clamp16(r);
    }
}

// ---------------------------------------------------------------------------------------------
// One epilogue warp's share of a 128 x 128 tile: rows quad*32 + lane, column group cg (0..3).
// Byte offset of 16-byte chunk c of row r in a TMA box whose rows are S bytes (S = 32, 64 or 128)
// stored with the matching S-byte swizzle (chunk index XOR address bits 7.., as TMA lays it out).
template <int S>
__device__ __forceinline__ int stg_off(int r, int c) {
    return r * S + (((c ^ ((r * S) >> 7)) & (S / 16 - 1)) << 4);
}

// Output maps of the epilogue (TMA stores; RESID also loads its residual tile through map 0):
// LOGITS 0 = logits; RESID 0 = x; QKV 0/1/2 = q/k/v.
struct EpiMaps {
    const CUtensorMap* c0;
    const CUtensorMap* c1;
    const CUtensorMap* c2;
};


// MODE selects the requantisation at compile time (0 generic int64, 1 fast 32-bit, 2 narrow), so
// the per-element loops carry no run-time branch between the paths.  QKV has two copies only
// (narrow, and fast-or-generic chosen at run time) to stay within its register budget.
template <int P, int KIND, int MODE>
__device__ __forceinline__ void epilogue_tile(const EpiParams& ep, uint32_t tacc, int m_blk, int n_blk, int cg,
                                              int quad, int lane, const int4* colp, const void* silu_tab,
                                              uint8_t* stg, const EpiMaps& maps, uint64_t* xbar, uint32_t& xphase,
                                              volatile int* abort, const uint64_t* digw, uint64_t& dsum,
                                              uint64_t& asum, bool first_cg) {
    constexpr int BN = (P == 4) ? BN_P4 : 128;
    const int row = m_blk * 128 + quad * 32 + lane;
    const bool row_ok = row < ep.M;
    const int n0 = n_blk * BN;
    if constexpr (KIND == EPI_QKV) {
        // cg -> head (cg >> 1) of the tile, dims d in [sub, sub + 16) paired with d + 32 for RoPE
        const int hl = cg >> 1, sub = (cg & 1) * 16;
        const int c0 = n0 + 64 * hl;
        if (c0 >= ep.N) return;
        int region, head;  // 0 = q, 1 = k, 2 = v
        if (c0 < 576) { region = 0; head = c0 / 64; }
        else if (c0 < 768) { region = 1; head = (c0 - 576) / 64; }
        else { region = 2; head = (c0 - 768) / 64; }
        const int bits_in = region == 0 ? ep.bits_q : (region == 1 ? ep.bits_k : ep.bits_v);
        const int bits_r = region == 0 ? ep.bits_qr : ep.bits_kr;
        const int rshift = region == 0 ? ep.rope_shift_q : ep.rope_shift_k;
        const CUtensorMap* omap = region == 0 ? maps.c0 : (region == 1 ? maps.c1 : maps.c2);
        const int pos = row_ok ? ep.pos0 + row % ep.T : 0;
        const bool rope_sm = ep.T <= ROPE_SMEM_ROWS && ep.pos0 + ep.T <= 512;
        const int64_t rrnd = rshift >= 1 ? (int64_t(1) << (rshift - 1)) : 0;
        // staging: dims [sub, sub + 16) and [32 + sub, 32 + sub + 16) of the head, 32 rows each (SW32)
        uint8_t* sa = stg;
        uint8_t* sb = stg + 1024;
        // a warp's first column group of a tile waits until every earlier store has read its staging
        // buffer (one buffer per column group of the warp, so the second group need not wait)
        if (lane == 0 && first_cg) bulk_wait_read0();
        __syncwarp();
#pragma unroll 1
        for (int h8 = 0; h8 < 16; h8 += 8) {  // 8 dims at a time keeps the pass free of spills
            const int d0 = sub + h8;
            // RoPE table rows first, so their load latency overlaps the TMEM loads; from the rows the
            // CTA staged in shared memory (silu_tab holds them for QKV) when T <= 128
            int32_t rc[8], rsn[8];
            if (region < 2 && row_ok) {
                if (rope_sm) {
                    const int32_t* rs = static_cast<const int32_t*>(silu_tab) + (row % ep.T) * ROPE_SMEM_PITCH + d0;
                    reinterpret_cast<int4*>(rc)[0] = reinterpret_cast<const int4*>(rs)[0];
                    reinterpret_cast<int4*>(rc)[1] = reinterpret_cast<const int4*>(rs)[1];
                    rs += ROPE_SMEM_ROWS * ROPE_SMEM_PITCH;
                    reinterpret_cast<int4*>(rsn)[0] = reinterpret_cast<const int4*>(rs)[0];
                    reinterpret_cast<int4*>(rsn)[1] = reinterpret_cast<const int4*>(rs)[1];
                } else {
                    const int4* cpp = reinterpret_cast<const int4*>(ep.rope_c + pos * 32 + d0);
                    const int4* spp = reinterpret_cast<const int4*>(ep.rope_s + pos * 32 + d0);
                    reinterpret_cast<int4*>(rc)[0] = __ldg(cpp);
                    reinterpret_cast<int4*>(rc)[1] = __ldg(cpp + 1);
                    reinterpret_cast<int4*>(rsn)[0] = __ldg(spp);
                    reinterpret_cast<int4*>(rsn)[1] = __ldg(spp + 1);
                }
            }
            uint32_t va[P][8], vb[P][8];
            load_planes2<P, 8>(tacc + 64 * hl + d0, va, tacc + 64 * hl + 32 + d0, vb);
            if (!row_ok) continue;
            int32_t oa[8], ob[8];  // int16 values (the narrow RoPE path leaves SAT16 to the pack below)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int4 ca = colp[64 * hl + d0 + i], cb = colp[64 * hl + 32 + d0 + i];
                int32_t a, b;
                if constexpr (MODE == 2) {
                    a = clamp16(rs_narrow<P, 8>(va, i, ca));
                    b = clamp16(rs_narrow<P, 8>(vb, i, cb));
                } else if (ep.fast) {
                    a = requant_fast<P, 8>(va, i, ca, bits_in);
                    b = requant_fast<P, 8>(vb, i, cb, bits_in);
                } else {
                    a = static_cast<int32_t>(requant_gen<P, 8>(va, i, ca, bits_in));
                    b = static_cast<int32_t>(requant_gen<P, 8>(vb, i, cb, bits_in));
                }
                if (region < 2) {
                    const int64_t t1 = static_cast<int64_t>(a) * rc[i] - static_cast<int64_t>(b) * rsn[i];
                    const int64_t t2 = static_cast<int64_t>(b) * rc[i] + static_cast<int64_t>(a) * rsn[i];
                    if constexpr (MODE == 2) {
                        const int64_t u1 = t1 + rrnd, u2 = t2 + rrnd;
                        oa[i] = static_cast<int32_t>(__funnelshift_r(static_cast<uint32_t>(u1),
                                                                     static_cast<uint32_t>(static_cast<uint64_t>(u1) >> 32), rshift));
                        ob[i] = static_cast<int32_t>(__funnelshift_r(static_cast<uint32_t>(u2),
                                                                     static_cast<uint32_t>(static_cast<uint64_t>(u2) >> 32), rshift));
                    } else if (ep.fast) {
                        int32_t hi;
                        uint32_t lo;
                        shr31(t1 + rrnd, rshift, hi, lo);
                        oa[i] = static_cast<int16_t>(sat_hl(hi, lo, bits_r));
                        shr31(t2 + rrnd, rshift, hi, lo);
                        ob[i] = static_cast<int16_t>(sat_hl(hi, lo, bits_r));
                    } else {
                        oa[i] = static_cast<int16_t>(sat64(rs64(t1, rshift), bits_r));
                        ob[i] = static_cast<int16_t>(sat64(rs64(t2, rshift), bits_r));
                    }
                } else {
                    oa[i] = static_cast<int16_t>(a);
                    ob[i] = static_cast<int16_t>(b);
                }
            }
            // int16 pairs by saturating packs (value 2k in the low half)
            *reinterpret_cast<uint4*>(sa + stg_off<32>(lane, h8 / 8)) =
                make_uint4(pack_sat_s16(oa[1], oa[0]), pack_sat_s16(oa[3], oa[2]), pack_sat_s16(oa[5], oa[4]),
                           pack_sat_s16(oa[7], oa[6]));
            *reinterpret_cast<uint4*>(sb + stg_off<32>(lane, h8 / 8)) =
                make_uint4(pack_sat_s16(ob[1], ob[0]), pack_sat_s16(ob[3], ob[2]), pack_sat_s16(ob[5], ob[4]),
                           pack_sat_s16(ob[7], ob[6]));
        }
        fence_async_smem();
        __syncwarp();
        const int row0 = m_blk * 128 + quad * 32;
        if (lane == 0 && row0 < ep.M) {
            tma_store_2d(omap, sa, head * 64 + sub, row0);
            tma_store_2d(omap, sb, head * 64 + 32 + sub, row0);
            bulk_commit();
        }
    } else if constexpr (KIND == EPI_GATEUP) {
        // cg -> gated features 16 cg .. 16 cg + 15 of the tile: gate cols 16 cg.., up cols 64 + 16 cg..
        if (n0 >= ep.N) return;
        const int64_t plane_stride = static_cast<int64_t>((ep.M + 127) / 128) * 128 * (ep.N / 2);
        uint8_t* gdst = ep.gated_planes + static_cast<int64_t>(m_blk) * 64 * ep.N + (n_blk * 4 + cg) * 2048 +
                        (quad * 32 + lane) * 16;
        uint32_t keep[4][2];  // packed planes of features 0..7, stored with 8..15 as one 16-byte word
        const bool sd = ep.sd_flags != nullptr && ep.gated_P == 4;
        bool big = false;     // some value of this warp needs the top signed digit
        const int gs = ep.gated_shift;
        const int64_t grnd = gs >= 1 ? (int64_t(1) << (gs - 1)) : 0;
        const bool lean = MODE >= 1 && ep.silu_smem && !ep.silu_wide && ep.bits_s == 16 && ep.silu_d <= 15 &&
                          ep.bits_g == 16 && ep.bits_u == 16;
#pragma unroll 1
        for (int h8 = 0; h8 < 16; h8 += 8) {  // 8 features at a time keeps the pass free of spills
            const int f0 = 16 * cg + h8;
            uint32_t vg[P][8], vu[P][8];
            load_planes2<P, 8>(tacc + f0, vg, tacc + 64 + f0, vu);
            if (!row_ok) continue;
            int32_t gm[8];
            const int16_t* tab16 = static_cast<const int16_t*>(silu_tab);
            const int cnt = ep.silu_count;
            if (P == 2 && lean && MODE == 2 && ep.acc32 && ep.bits_m == 32) {
                gateup_lean<P, 8, 32, true, true>(vg, vu, colp + f0, colp + 64 + f0, tab16, ep.silu_lo, cnt, ep.silu_d, gs, grnd, gm);
            } else if (P == 2 && lean && MODE == 2 && ep.acc32 && ep.bits_m == 16) {
                gateup_lean<P, 8, 16, true, true>(vg, vu, colp + f0, colp + 64 + f0, tab16, ep.silu_lo, cnt, ep.silu_d, gs, grnd, gm);
            } else if (lean && MODE == 2 && ep.bits_m == 32) {
                gateup_lean<P, 8, 32, true, false>(vg, vu, colp + f0, colp + 64 + f0, tab16, ep.silu_lo, cnt, ep.silu_d, gs, grnd, gm);
            } else if (lean && MODE == 2 && ep.bits_m == 16) {
                gateup_lean<P, 8, 16, true, false>(vg, vu, colp + f0, colp + 64 + f0, tab16, ep.silu_lo, cnt, ep.silu_d, gs, grnd, gm);
            } else if (lean && ep.bits_m == 32) {
                gateup_lean<P, 8, 32, false, false>(vg, vu, colp + f0, colp + 64 + f0, tab16, ep.silu_lo, cnt, ep.silu_d, gs, grnd, gm);
            } else if (lean && ep.bits_m == 16) {
                gateup_lean<P, 8, 16, false, false>(vg, vu, colp + f0, colp + 64 + f0, tab16, ep.silu_lo, cnt, ep.silu_d, gs, grnd, gm);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int4 cgp = colp[f0 + i], cup = colp[64 + f0 + i];
                    if constexpr (MODE >= 1) {
                        const int32_t g = requant_fast<P, 8>(vg, i, cgp, ep.bits_g);
                        const int32_t u = requant_fast<P, 8>(vu, i, cup, ep.bits_u);
                        const int32_t sg = static_cast<int32_t>(silu_lookup(ep, silu_tab, g));
                        const int64_t prod = static_cast<int64_t>(sg) * u + grnd;
                        int32_t hi;
                        uint32_t lo;
                        shr31(prod, gs, hi, lo);
                        gm[i] = sat_hl(hi, lo, ep.bits_m);
                    } else {
                        const int64_t g = requant_gen<P, 8>(vg, i, cgp, ep.bits_g);
                        const int64_t u = requant_gen<P, 8>(vu, i, cup, ep.bits_u);
                        const int64_t sg = silu_lookup(ep, silu_tab, static_cast<int>(g));
                        gm[i] = static_cast<int32_t>(sat64(rs64(sg * u, gs), ep.bits_m));
                    }
                }
            }
            if (ep.gated_offset) {
                const uint32_t flip = ep.gated_P == 4 ? 0x80000000u : 0x8000u;
#pragma unroll
                for (int i = 0; i < 8; ++i) gm[i] = static_cast<int32_t>(static_cast<uint32_t>(gm[i]) ^ flip);
            } else if (sd) {  // signed digits: the bytes of (gated + 0x808080) ^ 0x808080
                uint32_t any = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t w = static_cast<uint32_t>(gm[i]) + 0x808080u;
                    any |= w;
                    gm[i] = static_cast<int32_t>(w ^ 0x808080u);
                }
                big |= (any >> 24) != 0;
            }
            if (h8 == 0) {
                if (ep.gated_P == 4) pack_planes<8, true>(gm, keep[0], keep[1], keep[2], keep[3]);
                else pack_planes<8, false>(gm, keep[0], keep[1], keep[2], keep[3]);
            } else {
                uint32_t w[4][2];
                if (ep.gated_P == 4) pack_planes<8, true>(gm, w[0], w[1], w[2], w[3]);
                else pack_planes<8, false>(gm, w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4*>(gdst) = make_uint4(keep[0][0], keep[0][1], w[0][0], w[0][1]);
                *reinterpret_cast<uint4*>(gdst + plane_stride) = make_uint4(keep[1][0], keep[1][1], w[1][0], w[1][1]);
                if (ep.gated_P == 4) {
                    *reinterpret_cast<uint4*>(gdst + 2 * plane_stride) = make_uint4(keep[2][0], keep[2][1], w[2][0], w[2][1]);
                    *reinterpret_cast<uint4*>(gdst + 3 * plane_stride) = make_uint4(keep[3][0], keep[3][1], w[3][0], w[3][1]);
                }
            }
        }
        if (sd && __any_sync(0xffffffffu, big) && lane == 0) atomicOr(ep.sd_flags + m_blk, 1u);
    } else if constexpr (KIND == EPI_RESID) {
        // x = SAT32(x + RS(acc m, shift)) on this warp's 32 rows x NCOL columns.  The residual tile is
        // in the staging buffer (TMA load issued before the accumulator wait); with one resident
        // 16-column chunk (XCH == 1) the second chunk is loaded after the first is stored.
        constexpr int NCOL = BN / 4, NCH = NCOL / 16;
        constexpr int XCH = GemmCfg<P, KIND>::STG_BYTES / 2048;
        const bool top4 = P != 4 || !ep.sd_flags || __ldg(ep.sd_flags + m_blk) != 0;
        constexpr int S = XCH * 64;  // staging row bytes
        const int row0 = m_blk * 128 + quad * 32;
        const bool live = row0 < ep.M;
#pragma unroll 1
        for (int ch = 0; ch < NCH; ++ch) {
            const int tc = NCOL * cg + 16 * ch;
            const int gc = n0 + tc;
            if (gc >= ep.N) break;
            const int slot = XCH == 1 ? 0 : ch;
            if (XCH == 1 && ch > 0 && live) {
                if (lane == 0) {
                    bulk_wait_read0();
                    mbar_arrive_expect_tx(xbar, 2048);
                    tma_load_2d(stg, maps.c0, xbar, gc, row0);
                }
                if (!mbar_wait(xbar, xphase, abort, ep.err, ERR_TIMEOUT_EPI)) return;
                xphase ^= 1;
            }
            // two planes: two sub-rounds of 8 columns, whose planes and residuals fit the 96 registers
            // of the 16-warp epilogue without spilling (four planes spill elsewhere; one round of 16)
            constexpr int RW = P == 2 ? 8 : 16;
#pragma unroll
            for (int h = 0; h < 16; h += RW) {
                uint32_t v[P][RW];
                load_planes<P, RW>(tacc + tc + h, v);
                if constexpr (P == 4) {
                    if (!top4) {  // top signed-digit plane not computed for this row block
#pragma unroll
                        for (int q = 0; q < RW; ++q) v[3][q] = 0;
                    }
                }
                if (row_ok) {
                    int32_t xo[RW];
#pragma unroll
                    for (int q = 0; q < RW / 4; ++q)
                        *reinterpret_cast<int4*>(&xo[4 * q]) =
                            *reinterpret_cast<const int4*>(stg + stg_off<S>(lane, 4 * slot + h / 4 + q));
#pragma unroll
                    for (int i = 0; i < RW; ++i) {
                        const int4 cp = colp[tc + h + i];
                        if constexpr (MODE >= 1) {
                            int32_t hi;
                            uint32_t lo;
                            shr31(mulround<P, RW>(v, i, cp), cp.y, hi, lo);
                            const int64_t r = static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(hi)) << 32) | lo);
                            const int64_t y = r + xo[i];
                            xo[i] = sat_hl(static_cast<int32_t>(static_cast<uint64_t>(y) >> 32), static_cast<uint32_t>(y), 32);
                        } else {
                            const int64_t r = rs_col(combine<P, RW>(v, i) * static_cast<int64_t>(cp.x), cp.y);
                            xo[i] = static_cast<int32_t>(sat64(static_cast<int64_t>(xo[i]) + r, 32));
                        }
                    }
#pragma unroll
                    for (int q = 0; q < RW / 4; ++q)
                        *reinterpret_cast<int4*>(stg + stg_off<S>(lane, 4 * slot + h / 4 + q)) = *reinterpret_cast<int4*>(&xo[4 * q]);
                }
            }
            if (XCH == 1) {
                fence_async_smem();
                __syncwarp();
                if (lane == 0 && live) {
                    tma_store_2d(maps.c0, stg, gc, row0);
                    bulk_commit();
                }
            }
        }
        if (XCH > 1) {
            fence_async_smem();
            __syncwarp();
            const int gc0 = n0 + NCOL * cg;
            if (lane == 0 && live && gc0 < ep.N) {
                tma_store_2d(maps.c0, stg, gc0, row0);
                bulk_commit();
            }
        }
    } else if constexpr (KIND == EPI_SWEEP) {
        // out = SAT_bits_out(RS(acc m, shift)) on this warp's 32 rows x NCOL columns, int32 TMA tile
        // stores; digests of out and of the exact acc per row in registers (dsum, asum).  With one
        // resident 16-column chunk (SCH == 1) each chunk is stored before the next is staged.
        constexpr int NCOL = BN / 4, NCH = NCOL / 16;
        constexpr int SCH = GemmCfg<P, KIND>::STG_BYTES / 2048;
        constexpr int S = 64 * SCH;  // staging row bytes
        const int row0 = m_blk * 128 + quad * 32;
        if (lane == 0) bulk_wait_read0();  // the previous tile's store has read the staging buffer
        __syncwarp();
#pragma unroll 1
        for (int ch = 0; ch < NCH; ++ch) {
            const int tc = NCOL * cg + 16 * ch;
            const int gc = n0 + tc;
            if (gc >= ep.N) break;
            const int slot = SCH == 1 ? 0 : ch;
            if (SCH == 1 && ch > 0) {
                if (lane == 0) bulk_wait_read0();
                __syncwarp();
            }
            // 16 columns in sub-rounds of SW (8 with four planes: the accumulators stay in registers)
            constexpr int SW = P == 4 ? 8 : 16;
            int32_t o[16];
#pragma unroll
            for (int h = 0; h < 16; h += SW) {
                uint32_t v[P][SW];
                load_planes<P, SW>(tacc + tc + h, v);
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < SW; ++i) {
                        const int4 cp = colp[tc + h + i];
                        if constexpr (MODE >= 1) {
                            int32_t hi;
                            uint32_t lo;
                            shr31(mulround<P, SW>(v, i, cp), cp.y, hi, lo);
                            o[h + i] = sat_hl(hi, lo, ep.bits_out);
                        } else {
                            o[h + i] = static_cast<int32_t>(requant_gen<P, SW>(v, i, cp, ep.bits_out));
                        }
                    }
                    if (ep.dig_acc) {
#pragma unroll
                        for (int i = 0; i < SW; ++i) asum += static_cast<uint64_t>(combine<P, SW>(v, i)) * digw[tc + h + i];
                    }
                }
            }
            if (row_ok) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<int4*>(stg + stg_off<S>(lane, 4 * slot + q)) = *reinterpret_cast<int4*>(&o[4 * q]);
                if (ep.dig) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) dsum += static_cast<uint64_t>(static_cast<uint32_t>(o[i])) * digw[tc + i];
                }
            }
            if (SCH == 1) {
                fence_async_smem();
                __syncwarp();
                if (lane == 0 && row0 < ep.M) {
                    tma_store_2d(maps.c0, stg, gc, row0);
                    bulk_commit();
                }
            }
        }
        if (SCH > 1) {
            fence_async_smem();
            __syncwarp();
            const int gc0 = n0 + NCOL * cg;
            if (lane == 0 && row0 < ep.M && gc0 < ep.N) {
                tma_store_2d(maps.c0, stg, gc0, row0);
                bulk_commit();
            }
        }
    } else {
        constexpr int NCOL = BN / 4;  // columns of this warp: 32 (P = 2) or 16 (P = 4)
        if constexpr (KIND == EPI_LOGITS) {
            // as QKV: the warp's first column group of the tile waits for every earlier store's read
            if (lane == 0 && first_cg) bulk_wait_read0();
            __syncwarp();
        }
#pragma unroll 1
        for (int ch = 0; ch < NCOL / 16; ++ch) {
            const int tc = NCOL * cg + 16 * ch;
            const int gc = n0 + tc;
            if (gc >= ep.N) break;
            uint32_t v[P][16];
            load_planes<P, 16>(tacc + tc, v);
            if (!row_ok) continue;
            if constexpr (KIND == EPI_LOGITS) {
                int32_t o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int4 cp = colp[tc + i];
                    if constexpr (MODE >= 1) {
                        int32_t hi;
                        uint32_t lo;
                        shr31(mulround<P, 16>(v, i, cp), cp.y, hi, lo);
                        o[i] = static_cast<int32_t>(lo);
                    } else {
                        o[i] = static_cast<int32_t>(rs_col(combine<P, 16>(v, i) * static_cast<int64_t>(cp.x), cp.y));
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<int4*>(stg + stg_off<128>(lane, 4 * ch + q)) = *reinterpret_cast<int4*>(&o[4 * q]);
                if (ep.dig) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) dsum += static_cast<uint64_t>(static_cast<uint32_t>(o[i])) * digw[tc + i];
                }
            } else {  // EPI_LINEAR (generic path only)
                int64_t* op = ep.out64 + static_cast<int64_t>(row) * ep.N + gc;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int64_t acc = combine<P, 16>(v, i) - (ep.a_corr && gc + i < ep.N ? __ldg(ep.a_corr + gc + i) : 0);
                    op[i] = sat64(rs_col(acc * static_cast<int64_t>(colp[tc + i].x), colp[tc + i].y), ep.bits_out);
                }
                if (ep.acc64) {
                    int64_t* ap = ep.acc64 + static_cast<int64_t>(row) * ep.N + gc;
#pragma unroll
                    for (int i = 0; i < 16; ++i) ap[i] = combine<P, 16>(v, i) - (ep.a_corr && gc + i < ep.N ? __ldg(ep.a_corr + gc + i) : 0);
                }
            }
        }
        if constexpr (KIND == EPI_LOGITS) {
            fence_async_smem();
            __syncwarp();
            const int row0 = m_blk * 128 + quad * 32, gc0 = n0 + NCOL * cg;
            if (lane == 0 && row0 < ep.M && gc0 < ep.N) {
                tma_store_2d(maps.c0, stg, gc0, row0);
                bulk_commit();
            }
        }
    }
}

// Column parameters (m, shift, 2^(shift-1), m << 8) of output column c (zero multiplier past N).
__device__ __forceinline__ int4 col_params(const EpiParams& ep, int c) {
    const int2 ms = c < ep.N ? __ldg(ep.msh + c) : make_int2(0, 1);
    const int rnd = (ms.y >= 1 && ms.y <= 31) ? (1 << (ms.y - 1)) : 0;
    return make_int4(ms.x, ms.y, rnd, ms.x << 8);
}

// Digest weight of output column c (0 past N).
__device__ __forceinline__ uint64_t dig_weight(const EpiParams& ep, int c) { return c < ep.N ? __ldg(ep.dig_b + c) : 0; }

// ---------------------------------------------------------------------------------------------
template <int P, int KIND>
__global__ void __launch_bounds__(GemmCfg<P, KIND>::THREADS, 1)
    k_plane_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC0, const __grid_constant__ CUtensorMap tmC1,
                 const __grid_constant__ CUtensorMap tmC2, EpiParams ep) {
    using C = GemmCfg<P, KIND>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + C::STG_OFFSET;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFFSET);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::STAGES;
    uint64_t* acc_full = bars + 2 * C::STAGES;
    uint64_t* acc_empty = acc_full + C::NB;
    uint64_t* drain = acc_empty + C::NB;
    uint64_t* xbar = drain + 1;  // per epilogue warp: residual tile load (RESID)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + C::EPI_WARPS);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int4* colp_all = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);
    uint64_t* digw_all = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(colp_all) + C::COLP_BYTES);
    void* silu_tab = reinterpret_cast<uint8_t*>(colp_all) + C::COLP_BYTES + C::DIGW_BYTES;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_m = (ep.M + 127) / 128, num_n = (ep.N + C::BN - 1) / C::BN;
    const int tiles = num_m * num_n;
    const int KB = (ep.K + 127) / 128;
    // Tile schedule shared by the three roles: LOGITS walks a contiguous run of tiles (rows stay on
    // one CTA for many N tiles, so the digest sums stay in registers); the others stride by the grid.
    int t_first = blockIdx.x, t_end = tiles, t_step = gridDim.x;
    if constexpr (KIND == EPI_LOGITS || KIND == EPI_SWEEP) {
        t_first = static_cast<int>(static_cast<int64_t>(blockIdx.x) * tiles / gridDim.x);
        t_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * tiles / gridDim.x);
        t_step = 1;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < C::NB; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], C::EPI_WARPS); }
        mbar_init(drain, 1);
        for (int w = 0; w < C::EPI_WARPS; ++w) mbar_init(&xbar[w], 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_launch();

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            griddep_wait();  // A is the previous kernel's output
            int stage = 0;
            uint32_t phase = 0;
            uint32_t fills = 0;
            bool ok = true;
            for (int t = t_first; t < t_end && ok; t += t_step) {
                const int m_blk = t / num_n, n_blk = t % num_n;
                // planes of this tile's A operand (3 when the signed-digit top plane is all zero)
                int np = P;
                if constexpr (KIND == EPI_RESID && P == 4)
                    if (ep.sd_flags && __ldg(ep.sd_flags + m_blk) == 0) np = 3;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort, ep.err, ERR_TIMEOUT_PRODUCER)) { ok = false; break; }
                    uint8_t* sA = smem + stage * C::STAGE_BYTES;
                    uint8_t* sB = sA + P * C::A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], np * C::A_BYTES + C::B_BYTES);
                    if (ep.a_blocked) {
#pragma unroll
                        for (int p = 0; p < P; ++p)
                            if (p < np) tma_load_4d(sA + p * C::A_BYTES, &tmA, &full[stage], 0, kb * 8, m_blk, p);
                    } else {
#pragma unroll
                        for (int p = 0; p < P; ++p)
                            tma_load_3d(sA + p * C::A_BYTES, &tmA, &full[stage], kb * 128, m_blk * 128, p);
                    }
                    tma_load_2d(sB, &tmB, &full[stage], kb * 128, n_blk * C::BN);
                    ++fills;
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok) {
                // Let the copies already issued land before the CTA can exit (bounded).
                int s = stage;
                uint32_t ph = phase;
                for (uint32_t i = 0; i < fills && i < (uint32_t)C::STAGES; ++i) {
                    if (--s < 0) { s = C::STAGES - 1; ph ^= 1; }
                    volatile int no_abort = 0;
                    mbar_wait(&full[s], ph, &no_abort, nullptr, 0, 100000000ull);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc_iter = 0;
            bool ok = true;
            bool issued = false;
            griddep_wait();  // the signed-digit flags below are the previous kernel's output
            for (int t = t_first; t < t_end && ok; t += t_step, ++acc_iter) {
                const int n_blk = t % num_n;
                // planes of this tile (the producer loads the same: 3 when the signed-digit top plane is 0)
                int np = P;
                if constexpr (KIND == EPI_RESID && P == 4)
                    if (ep.sd_flags && __ldg(ep.sd_flags + t / num_n) == 0) np = 3;
                const int buf = acc_iter % C::NB;
                const uint32_t acc_phase = (acc_iter / C::NB) & 1;
                if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort, ep.err, ERR_TIMEOUT_MMA_ACC)) { ok = false; break; }
                tc_fence_after();
                const int n_valid = min(C::BN, ep.N - n_blk * C::BN);
                const uint32_t id_lo = idesc_i8(ep.a_sd != 0, true, n_valid);  // low planes u8, or signed digits
                const uint32_t id_hi = idesc_i8(ep.a_corr == nullptr, true, n_valid);  // top plane s8, or u8 (offset binary)
                const uint32_t dbase = tmem_base + buf * C::ACC_COLS;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort, ep.err, ERR_TIMEOUT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sA = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint32_t sB = sA + P * C::A_BYTES;
                    const int ksteps = min(128, ep.K - kb * 128) / 32;
                    for (int ks = 0; ks < ksteps; ++ks) {
                        const uint64_t bdesc = smem_desc_sw128(sB + ks * 32);
#pragma unroll
                        for (int p = 0; p < P; ++p) {
                            if (p >= np) continue;
                            // row-blocked A: 16-byte K chunks 2 KB apart, 8-row groups 128 bytes apart
                            const uint64_t adesc = ep.a_blocked ? smem_desc_noswz(sA + p * C::A_BYTES + ks * 4096, 2048, 128)
                                                                : smem_desc_sw128(sA + p * C::A_BYTES + ks * 32);
                            mma_i8(dbase + p * C::BN, adesc, bdesc, p == P - 1 ? id_hi : id_lo,
                                   (kb > 0 || ks > 0) ? 1u : 0u);
                        }
                    }
                    issued = true;
                    tc_commit(&empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                tc_commit(&acc_full[buf]);
            }
            if (!ok && issued) {
                // Wait (bounded) for every MMA this thread issued before TMEM is released.
                tc_commit(drain);
                volatile int no_abort = 0;
                mbar_wait(drain, 0, &no_abort, ep.err, ERR_TIMEOUT_DRAIN, 100000000ull);
            }
        }
    } else {
        const int e = warp - 2;
        const int et = threadIdx.x - 64;  // 0 .. EPI_THREADS - 1
        const int quad = warp & 3;
        const int cg = e >> 2;  // first column group of this warp
        uint8_t* stg = staging + e * C::CG_PER_WARP * C::STG_BYTES;  // one buffer per column group of the warp
        const EpiMaps maps{&tmC0, &tmC1, &tmC2};
        uint32_t xphase = 0;
        if constexpr (KIND == EPI_QKV) {
            if (ep.T <= ROPE_SMEM_ROWS && ep.pos0 + ep.T <= 512) {  // stage the RoPE rows of this launch's positions
                int32_t* rs = static_cast<int32_t*>(silu_tab);
                for (int q = et; q < 2 * ep.T * 8; q += C::EPI_THREADS) {
                    const int tab = q / (ep.T * 8), r = (q / 8) % ep.T, c4 = q % 8;
                    const int32_t* src = (tab ? ep.rope_s : ep.rope_c) + (ep.pos0 + r) * 32 + c4 * 4;
                    *reinterpret_cast<int4*>(rs + (tab * ROPE_SMEM_ROWS + r) * ROPE_SMEM_PITCH + c4 * 4) =
                        __ldg(reinterpret_cast<const int4*>(src));
                }
            }
        }
        if constexpr (KIND == EPI_GATEUP) {
            if (ep.silu_smem) {  // stage the compact SiLU table (and the zero past it) once per CTA
                const int nbytes = (ep.silu_count + 1) * (ep.silu_wide ? 4 : 2);
                const int n16 = (nbytes + 15) / 16;
                for (int q = et; q < n16; q += C::EPI_THREADS)
                    reinterpret_cast<int4*>(silu_tab)[q] = __ldg(reinterpret_cast<const int4*>(ep.silu_neg) + q);
            }
        }
        griddep_wait();  // outputs (and RESID's residual input) are shared with earlier kernels
        int acc_iter = 0;
        // LOGITS / SWEEP digests: row block whose sums this lane holds, and the sums over the columns
        // seen so far of uint32(out) * dig_b[col] (dsum) and, SWEEP only, of uint64(acc) * dig_b[col] (asum)
        int dig_m = -1;
        uint64_t dsum = 0, asum = 0;
        const bool digs = (KIND == EPI_LOGITS && ep.dig) || (KIND == EPI_SWEEP && (ep.dig || ep.dig_acc));
        auto dig_flush = [&]() {
            const int r = dig_m * 128 + quad * 32 + lane;
            if (dig_m >= 0 && r < ep.M) {
                if constexpr (KIND == EPI_SWEEP) {
                    if (ep.dig) atomicAdd(ep.dig + r, static_cast<unsigned long long>(dsum));
                    if (ep.dig_acc) atomicAdd(ep.dig_acc + r, static_cast<unsigned long long>(asum));
                } else {
                    atomicAdd(ep.dig + r / ep.T, static_cast<unsigned long long>(dsum * __ldg(ep.dig_a + ep.pos0 + r % ep.T)));
                }
            }
            dsum = 0;
            asum = 0;
        };
        for (int t = t_first; t < t_end; t += t_step, ++acc_iter) {
            const int m_blk = t / num_n, n_blk = t % num_n;
            if (digs && m_blk != dig_m) {
                dig_flush();
                dig_m = m_blk;
            }
            const int buf = acc_iter % C::NB;
            const uint32_t acc_phase = (acc_iter / C::NB) & 1;
            // Per-tile column parameters, double buffered: a warp that writes buffer b for this tile
            // has passed the previous tile's barrier, so every warp is done with tile - 2.  The
            // barrier below also publishes the staged SiLU table before the first tile.
            int4* colp = colp_all + (acc_iter & 1) * C::BN;
            if (acc_iter == 0 && et < C::BN) {
                colp[et] = col_params(ep, n_blk * C::BN + et);
                if (digs) digw_all[et] = dig_weight(ep, n_blk * C::BN + et);
            }
            // RESID: the residual tile of this warp (32 rows x BN/4 int32) goes into its staging buffer by
            // TMA while the accumulators are being computed.
            bool xload = false;
            if constexpr (KIND == EPI_RESID) {
                const int row0 = m_blk * 128 + quad * 32, gc0 = n_blk * C::BN + (C::BN / 4) * cg;
                xload = row0 < ep.M && gc0 < ep.N;
                if (xload && lane == 0) {
                    bulk_wait_read0();
                    mbar_arrive_expect_tx(&xbar[e], C::STG_BYTES);
                    tma_load_2d(stg, &tmC0, &xbar[e], gc0, row0);
                }
            }
            bool ok = true;
            if constexpr (KIND == EPI_LINEAR) {
                if (ep.test_stall_ns && acc_iter == 0)  // xbar is unused by this kind: its phase never completes
                    ok = mbar_wait(&xbar[e], 0, abort, ep.err, ERR_TIMEOUT_EPI, ep.test_stall_ns);
            }
            ok = ok && mbar_wait(&acc_full[buf], acc_phase, abort, ep.err, ERR_TIMEOUT_EPI);
            if (xload) {
                ok = ok && mbar_wait(&xbar[e], xphase, abort, ep.err, ERR_TIMEOUT_EPI);
                xphase ^= 1;
            }
            if (!epi_barrier_and(ok, C::EPI_THREADS)) break;
            tc_fence_after();
            // parameters of this CTA's next tile go into the other buffer now (published by the next
            // tile's barrier), so their global-load latency is hidden behind this tile's epilogue
            if (et < C::BN && t + t_step < t_end) {
                const int nc = ((t + t_step) % num_n) * C::BN + et;
                colp_all[((acc_iter + 1) & 1) * C::BN + et] = col_params(ep, nc);
                if (digs) digw_all[((acc_iter + 1) & 1) * C::BN + et] = dig_weight(ep, nc);
            }
            const uint64_t* digw = digw_all + (acc_iter & 1) * C::BN;
            const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * C::ACC_COLS;
#pragma unroll 1
            for (int k = 0; k < C::CG_PER_WARP; ++k) {  // this warp's column groups (one, or two for gate/up)
                const int cgk = cg + k * (C::EPI_WARPS / 4);
                uint8_t* stgk = stg + k * C::STG_BYTES;
                if (KIND != EPI_LINEAR && ep.narrow && (KIND == EPI_QKV || KIND == EPI_GATEUP))
                    epilogue_tile<P, KIND, 2>(ep, tacc, m_blk, n_blk, cgk, quad, lane, colp, silu_tab, stgk, maps, &xbar[e],
                                              xphase, abort, digw, dsum, asum, k == 0);
                else if (KIND != EPI_LINEAR && KIND != EPI_QKV && ep.fast)
                    epilogue_tile<P, KIND, 1>(ep, tacc, m_blk, n_blk, cgk, quad, lane, colp, silu_tab, stgk, maps, &xbar[e],
                                              xphase, abort, digw, dsum, asum, k == 0);
                else
                    epilogue_tile<P, KIND, 0>(ep, tacc, m_blk, n_blk, cgk, quad, lane, colp, silu_tab, stgk, maps, &xbar[e],
                                              xphase, abort, digw, dsum, asum, k == 0);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        if (digs) dig_flush();
        if (lane == 0) bulk_wait0();  // this warp's tile stores are complete before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

}  // namespace eii
