// Feature-major byte-plane integer GEMM on tcgen05 kind::i8: output features in the TMEM lanes,
// activation rows x byte planes in the MMA's N dimension.
//
// Every MMA has N = 256: the activation tile is the P byte planes of BR = 256 / P rows stacked along
// N, so one instruction multiplies a 128-feature weight tile with all planes of BR rows, and the int32
// accumulator of (feature f, plane p, row j) sits in TMEM lane f, column p * BR + j.  A tile's
// accumulators take 256 of the 512 TMEM columns for any plane count, so two tiles are always in
// flight: the epilogue of one runs while the MMAs of the next fill the other half.  (The row-major
// GEMM keeps one accumulator per plane; with four planes its 128-wide tiles fill all of TMEM and its
// epilogue cannot overlap the next tile's MMAs, which is what made the 4-plane down projection slow.)
// The MMA rate itself does not depend on N here: back to back, an M = 128, K = 32 kind::i8 MMA takes
// 64 cycles at N = 128 and 128 at N = 256, the full 8192 MACs per cycle per SM (bench.py --probe-mma).
//
// One instruction needs one operand type for all planes, so the activation planes are offset
// binary: for b-bit activations a, the planes are the bytes of a + 2^(b-1) (all u8; the low planes
// are unchanged and the top byte has its sign bit flipped).  Then
//     acc[r][f] = sum_k a[r][k] W[f][k] = sum_p 2^(8p) v_p[f][r] - 2^(b-1) S_f,   S_f = sum_k W[f][k],
// with v_p the int32 plane accumulators (|v_p| <= 255 * 127 * K < 2^26 for K <= 1536: no int32
// overflow).  The per-feature constant 2^(b-1) S_f folds into the rounding constant of the
// requantisation, so the epilogue computes, with m the feature's multiplier (m < 2^15) and s its
// shift (1 <= s <= 62),
//     RS(acc m, s) = (sum_p 2^(8p) v_p m + (2^(s-1) - 2^(b-1) S_f m)) >> s
// in 64-bit two's-complement arithmetic: intermediate sums may wrap, the result is exact whenever
// |acc m| < 2^62 (the bound the reference asserts, python/intref.py:189,259,279).
//
// Kernel structure (one CTA per SM, persistent over 128-feature x BR-row tiles):
//   warp 0      TMA producer: per 128-byte K block, the weight tile [128 features x 128 B] and the
//               activation planes [P][BR rows][128 B] in one 3-D box, both with the 128-byte swizzle.
//   warp 1      TMEM allocator + MMA issuer: 4 (2 for a half K block) K = 32 steps of
//               tcgen05.mma.cta_group::1.kind::i8, M = 128, N = 256, A = weights (s8), B = planes (u8).
//   warps 2-17  epilogue: warp w reads TMEM lane quadrant w % 4 (32 features, one per lane) for a
//               quarter of the tile's rows; its per-feature constants live in registers.  Stores go
//               straight to global memory: for one row the warp's 32 lanes write 32 consecutive
//               features (128 contiguous bytes of int32).
#pragma once
#include <cstdint>
#include <cuda.h>

#include "eii_gemm.cuh"
#include "eii_ptx.cuh"

namespace eii {

// Per-feature constants of the feature-major GEMM: multiplier m (< 2^15), shift s, and the 64-bit
// rounding constant 2^(s-1) - 2^(b-1) S_f m (low, high words).
struct TFeat {
    int m, sh;
    uint32_t k_lo, k_hi;
};

struct TEpi {
    int M, N, K;
    // A planes in the row-blocked layout [P][ceil(M/128)][K/16][128 rows][16 bytes] (attention context,
    // gated product), read through a 4-D map whose box lands as [8 K chunks][P][BR rows][16 bytes]
    // (no swizzle; K-chunk stride P * BR * 16 bytes, 8-row-group stride 128 bytes); else plane-major
    // [P][M][K] with the 128-byte swizzle.
    int a_blocked;
    int split;               // feature constants are the split-mode ones (tg_rs_split); else TFeat
    const int4* feat;        // TFeat (or split-mode constants) per feature [N] (as int4)
    const uint64_t* corr;    // 2^(b-1) S_f per feature [N] (the digest of the exact acc needs it), or null
    int* err;
    int bits_out;            // SWEEP: SAT to bits_out (<= 32)
    int32_t* out;            // SWEEP / LOGITS: int32 out[row * ld + f]; RESID: the residual x[row * ld + f]
    int64_t ld;
    // per-row digests (SWEEP): dig[row] += sum_f uint32(out) w_f, dig_acc[row] += sum_f uint64(acc) w_f
    unsigned long long* dig;
    unsigned long long* dig_acc;
    const uint64_t* dig_b;   // w_f
    // LOGITS: out = low 32 bits of RS(acc m, s) (every s in [1, 31], checked on the host); optional
    // per-sequence digest dig[row / T] += sum over (t, f) of uint32(out) * dig_b[f] * dig_a[pos0 + row % T]
    int T, pos0;
    const uint64_t* dig_a;
};

// RES: the activation planes of a row block stay resident in shared memory (all K blocks, K <= 640)
// while the CTA walks that row block's feature tiles, so only the weight tiles stream from L2
// (72 KB per tile at K = 576 instead of 221 KB); otherwise planes and weights stream together.
template <int P, bool RES>
struct TCfg {
    static constexpr int BF = 128;             // features per tile (TMEM lanes, MMA M)
    static constexpr int BR = 256 / P;         // rows per tile
    static constexpr int NMMA = 256;           // MMA N = P * BR
    static constexpr int A_BYTES = BF * 128;   // weight tile per 128-byte K block
    static constexpr int B_BYTES = NMMA * 128; // activation planes per K block
    static constexpr int RES_KB = 5;           // resident K blocks (K <= 640)
    static constexpr int STAGE_BYTES = RES ? A_BYTES : A_BYTES + B_BYTES;
    static constexpr int STAGES = RES ? 3 : 4;
    static constexpr int RES_OFFSET = STAGES * STAGE_BYTES;
    static constexpr int EPI_WARPS = 16;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int ROWS_PER_WARP = BR / 4;  // each lane quadrant is split over 4 warps by rows
    static constexpr int BAR_OFFSET = RES_OFFSET + (RES ? RES_KB * B_BYTES : 0);
    static constexpr int SMEM = BAR_OFFSET + 1024 + 512;
    static_assert(SMEM <= SMEM_LIMIT, "shared memory budget");
};

// Sum over the warp's 32 lanes of s[i] for 16 rows i: after the call, lane l holds the full sum of
// row ((l >> 4) & 1) * 8 + ((l >> 3) & 1) * 4 + ((l >> 2) & 1) * 2 + ((l >> 1) & 1) (lanes l and l ^ 1
// hold the same row).  Recursive halving: 16 + 8 + 4 + 2 + 2 shuffles of 64-bit values.
__device__ __forceinline__ uint64_t reduce_rows16(const uint64_t (&s)[16], int lane) {
    uint64_t a[8], b[4], c[2];
    const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4, h1 = lane & 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint64_t send = h4 ? s[k] : s[8 + k], keep = h4 ? s[8 + k] : s[k];
        a[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint64_t send = h3 ? a[k] : a[4 + k], keep = h3 ? a[4 + k] : a[k];
        b[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint64_t send = h2 ? b[k] : b[2 + k], keep = h2 ? b[2 + k] : b[k];
        c[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const uint64_t send = h1 ? c[0] : c[1], keep = h1 ? c[1] : c[0];
    const uint64_t d = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    return d + __shfl_xor_sync(0xffffffffu, d, 1);
}
__device__ __forceinline__ int reduce_rows16_row(int lane) {
    return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// 64-bit requantisation sum of one (feature, row): sum_p 2^(8p) v_p m + K (mod 2^64), m < 2^15.
template <int P, int N = 16>
__device__ __forceinline__ uint64_t tg_sum(const uint32_t (&v)[P][N], int i, int m, uint64_t kc) {
    uint64_t t = static_cast<uint64_t>(static_cast<int64_t>(static_cast<int32_t>(v[0][i])) * m) + kc;
    t += static_cast<uint64_t>(static_cast<int64_t>(static_cast<int32_t>(v[1][i])) * (m << 8));
    if constexpr (P == 4) {
        t += static_cast<uint64_t>(static_cast<int64_t>(static_cast<int32_t>(v[2][i])) * (m << 16));
        t += static_cast<uint64_t>(static_cast<int64_t>(static_cast<int32_t>(v[3][i])) * (m << 16)) << 8;
    }
    return t;
}

// Requantisation without wide multiplies (two-plane activations, |acc| < 2^31 proven on the host for
// every feature, shift s in [1, 31]).  Dense 32x32->64 multiply-accumulate work beside the MMAs slows
// them several-fold, while 32-bit IMAD and ALU work leaves them at full rate (bench.py --probe-mma), so:
//   acc = v0 + 2^8 v1 - 2^15 S_f                (mod 2^32; exact since |acc| < 2^31)
//   acc m = (a1 2^16 + a0) m = p1 2^16 + a0 m,  a1 = acc >> 16 (signed), a0 = acc & 0xFFFF, p1 = a1 m
//   u = a0 m + 2^(s-1) < 2^32;  (hi:lo) = p1 2^16 + u = acc m + 2^(s-1)   (a 48-bit value)
//   RS(acc m, s) = (hi:lo) >> s:  low word by a funnel shift, high word hi >> s (for the saturation test).
// Feature constants in this mode: (m, s, -2^15 S_f mod 2^32, 2^(s-1)).
__device__ __forceinline__ void tg_rs_split(uint32_t v0, uint32_t v1, int m, int sh, uint32_t negc, uint32_t rnd,
                                            uint32_t& ylo, int32_t& yhi) {
    const uint32_t acc = v0 + (v1 << 8) + negc;
    const int32_t p1 = (static_cast<int32_t>(acc) >> 16) * m;
    const uint32_t u = (acc & 0xFFFFu) * static_cast<uint32_t>(m) + rnd;
    const uint32_t lo = (static_cast<uint32_t>(p1) << 16) + u;
    const int32_t hi = (p1 >> 16) + (lo < u ? 1 : 0);
    ylo = __funnelshift_r(lo, static_cast<uint32_t>(hi), sh);
    yhi = hi >> sh;
}

// The exact contraction acc = sum_p 2^(8p) v_p - corr (mod 2^64).
template <int P>
__device__ __forceinline__ uint64_t tg_acc(const uint32_t (&v)[P][16], int i, uint64_t corr) {
    uint64_t a = 0;
#pragma unroll
    for (int p = 0; p < P; ++p) a += static_cast<uint64_t>(static_cast<int64_t>(static_cast<int32_t>(v[p][i]))) << (8 * p);
    return a - corr;
}

// ---------------------------------------------------------------------------------------------
// NODIG: the contraction sweep without its per-row digests (the timed launches), compiled without the
// digest code, which at four planes would otherwise push the epilogue past its 96 registers.
template <int P, int KIND, bool RES, bool NODIG = false>
__global__ void __launch_bounds__(TCfg<P, RES>::THREADS, 1)
    k_tgemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA, TEpi ep) {
    using C = TCfg<P, RES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFFSET);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::STAGES;
    uint64_t* acc_full = bars + 2 * C::STAGES;  // [2]
    uint64_t* acc_empty = acc_full + 2;         // [2]
    uint64_t* drain = acc_empty + 2;
    uint64_t* res_full = drain + 1;   // RES: the resident planes of the current row block have landed
    uint64_t* res_empty = res_full + 1;  // RES: every MMA that read the previous row block's planes is done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_empty + 1);
    uint8_t* res = smem + C::RES_OFFSET;
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x / 32), 0), lane = threadIdx.x % 32;
    const int num_f = (ep.N + C::BF - 1) / C::BF, num_r = (ep.M + C::BR - 1) / C::BR;
    const int tiles = num_f * num_r;
    const int KB = (ep.K + 127) / 128;
    // contiguous run of tiles per CTA, row block major (consecutive tiles share the activation rows,
    // so per-row digest sums stay in registers across the run)
    const int t_first = static_cast<int>(static_cast<int64_t>(blockIdx.x) * tiles / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * tiles / gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], C::EPI_WARPS); }
        mbar_init(drain, 1);
        mbar_init(res_full, 1);
        mbar_init(res_empty, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_launch();

    // activation planes of K block kb and row block r_blk (all P planes, BR rows) into dst
    auto load_act = [&](uint8_t* dst, uint64_t* bar, int kb, int r_blk) {
        if (ep.a_blocked)  // 4-D map: (16-byte rows of the 128-row block as 8-byte pairs, plane, K chunk, row block)
            tma_load_4d(dst, &tmA, bar, ((r_blk * C::BR) & 127) * 2, 0, kb * 8, (r_blk * C::BR) >> 7);
        else
            tma_load_3d(dst, &tmA, bar, kb * 128, r_blk * C::BR, 0);
    };
    if (warp == 0) {
        // TMA producer: the whole warp runs the loop (warp-uniform coordinates), one lane issues
        if (elect_one()) { prefetch_tmap(&tmW); prefetch_tmap(&tmA); }
        __syncwarp();
        griddep_wait();
        int stage = 0;
        uint32_t phase = 0, fills = 0, res_loads = 0;
        int cur_r = -1;
        bool ok = true;
        for (int t = t_first; t < t_end && ok; ++t) {
            const int r_blk = t / num_f, f_blk = t % num_f;
            if (RES && r_blk != cur_r) {
                // the previous row block's MMAs have finished reading the resident planes
                // (the k-th switch waits for the k-th completion of res_empty: parity (k - 1) & 1)
                if (res_loads > 0 &&
                    !__all_sync(0xffffffffu, mbar_wait(res_empty, (res_loads - 1) & 1, abort, ep.err, ERR_TIMEOUT_PRODUCER))) {
                    ok = false;
                    break;
                }
                if (elect_one()) {
                    mbar_arrive_expect_tx(res_full, KB * C::B_BYTES);
                    for (int kb = 0; kb < KB; ++kb) load_act(res + kb * C::B_BYTES, res_full, kb, r_blk);
                }
                __syncwarp();
                ++res_loads;
                cur_r = r_blk;
            }
            for (int kb = 0; kb < KB; ++kb) {
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1, abort, ep.err, ERR_TIMEOUT_PRODUCER))) {
                    ok = false;
                    break;
                }
                uint8_t* sW = smem + stage * C::STAGE_BYTES;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sW, &tmW, &full[stage], kb * 128, f_blk * C::BF);
                    if constexpr (!RES) load_act(sW + C::A_BYTES, &full[stage], kb, r_blk);
                }
                __syncwarp();
                ++fills;
                if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
            }
        }
        if (!ok) {  // let the copies already issued land before the CTA exits (bounded)
            volatile int no_abort = 0;
            if (RES && res_loads > 0)  // the last resident-plane load (completion number res_loads)
                mbar_wait(res_full, (res_loads - 1) & 1, &no_abort, nullptr, 0, 100000000ull);
            int s = stage;
            uint32_t ph = phase;
            for (uint32_t i = 0; i < fills && i < (uint32_t)C::STAGES; ++i) {
                if (--s < 0) { s = C::STAGES - 1; ph ^= 1; }
                mbar_wait(&full[s], ph, &no_abort, nullptr, 0, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // MMA issuer: the whole warp runs the loop, the descriptors are warp-uniform, one lane issues
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true, issued = false;
        const uint32_t idesc = idesc_i8(true, false, C::NMMA);  // weights s8, offset-binary planes u8
        const uint64_t stage_desc = smem_desc_sw128(smem_u32(smem));
        int acc_iter = 0, cur_r = -1;
        uint32_t res_phase = 0;
        for (int t = t_first; t < t_end && ok; ++t, ++acc_iter) {
            if (RES && t / num_f != cur_r) {
                if (cur_r >= 0) {
                    if (elect_one()) tc_commit(res_empty);  // completes when every MMA issued so far is done
                    __syncwarp();
                    res_phase ^= 1;
                }
                cur_r = t / num_f;
                if (!__all_sync(0xffffffffu, mbar_wait(res_full, res_phase, abort, ep.err, ERR_TIMEOUT_MMA_FULL))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            const int buf = acc_iter & 1;
            const uint32_t acc_phase = (acc_iter >> 1) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort, ep.err, ERR_TIMEOUT_MMA_ACC))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + buf * C::NMMA;
            for (int kb = 0; kb < KB; ++kb) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort, ep.err, ERR_TIMEOUT_MMA_FULL))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // descriptor start addresses advance in 16-byte units: a stage is STAGE_BYTES >> 4, a K step 2
                const uint64_t wdesc = stage_desc + static_cast<uint64_t>((stage * C::STAGE_BYTES) >> 4);
                const uint32_t a_addr = RES ? smem_u32(res + kb * C::B_BYTES) : smem_u32(smem + stage * C::STAGE_BYTES) + C::A_BYTES;
                // plane-major: 128-byte swizzled rows, a K step is 32 bytes (+2 in 16-byte units); row-blocked:
                // no swizzle, K chunks CH = P * BR * 16 bytes apart, a K step is two chunks
                constexpr uint32_t CH = C::NMMA * 16;
                const uint64_t adesc = ep.a_blocked ? smem_desc_noswz(a_addr, CH, 128) : smem_desc_sw128(a_addr);
                const uint64_t astep = ep.a_blocked ? static_cast<uint64_t>((2 * CH) >> 4) : 2;
                const int ksteps = min(128, ep.K - kb * 128) / 32;
                if (elect_one()) {
                    for (int ks = 0; ks < ksteps; ++ks)
                        mma_i8(d, wdesc + 2 * ks, adesc + astep * ks, idesc, (kb > 0 || ks > 0) ? 1u : 0u);
                    tc_commit(&empty[stage]);
                }
                __syncwarp();
                issued = true;
                if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            if (elect_one()) tc_commit(&acc_full[buf]);
            __syncwarp();
        }
        if (!ok && issued) {  // wait (bounded) for every MMA issued before TMEM is released
            if (elect_one()) tc_commit(drain);
            __syncwarp();
            volatile int no_abort = 0;
            mbar_wait(drain, 0, &no_abort, ep.err, ERR_TIMEOUT_DRAIN, 100000000ull);
        }
    } else {
        const int quad = warp & 3, rsub = (warp - 2) >> 2;
        griddep_wait();
        const bool digs = !NODIG && KIND == EPI_SWEEP && (ep.dig || ep.dig_acc);
        const bool ldig = KIND == EPI_LOGITS && ep.dig != nullptr;
        // per-row digest sums of this warp's rows (lane: the row reduce_rows16_row names, per 16-row chunk)
        constexpr int NCH = C::ROWS_PER_WARP / 16;
        uint64_t dsum[NCH], asum[NCH];
#pragma unroll
        for (int j = 0; j < NCH; ++j) dsum[j] = asum[j] = 0;
        int dig_r = -1;
        // LOGITS digest, per lane: sum over this CTA's run of feature tiles of dig_b[f] * (sum over the chunk's
        // rows of uint32(out) dig_a[t]) for chunk j (rows of one sequence, lseq[j]); reduced over the warp and
        // added to the sequence's digest when the row block changes (lr) or the run ends
        uint64_t lacc[NCH];
        int lseq[NCH];
        int lr = -1;
#pragma unroll
        for (int j = 0; j < NCH; ++j) { lacc[j] = 0; lseq[j] = -1; }
        auto lflush = [&]() {
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                uint64_t w = lacc[j];
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
                if (lane == 0 && lseq[j] >= 0 && lseq[j] * ep.T < ep.M) atomicAdd(ep.dig + lseq[j], static_cast<unsigned long long>(w));
                lacc[j] = 0;
                lseq[j] = -1;
            }
        };
        auto dig_flush = [&]() {
            if (dig_r < 0 || (lane & 1)) return;
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int row = dig_r * C::BR + rsub * C::ROWS_PER_WARP + 16 * j + reduce_rows16_row(lane);
                if (row < ep.M) {
                    if (ep.dig) atomicAdd(ep.dig + row, static_cast<unsigned long long>(dsum[j]));
                    if (ep.dig_acc) atomicAdd(ep.dig_acc + row, static_cast<unsigned long long>(asum[j]));
                }
            }
        };
        int acc_iter = 0;
        for (int t = t_first; t < t_end; ++t, ++acc_iter) {
            const int r_blk = t / num_f, f_blk = t % num_f;
            const int f = f_blk * C::BF + quad * 32 + lane;
            const bool f_ok = f < ep.N;
            // this lane's feature constants (loaded before the accumulator wait)
            int4 fc = make_int4(0, 1, 0, 0);
            uint64_t wf = 0, corr = 0;
            if (f_ok) {
                fc = __ldg(ep.feat + f);
                if (ldig) wf = __ldg(ep.dig_b + f);
                if (digs) {
                    wf = __ldg(ep.dig_b + f);
                    if (ep.dig_acc) corr = __ldg(ep.corr + f);
                }
            }
            const uint64_t kc = (static_cast<uint64_t>(static_cast<uint32_t>(fc.w)) << 32) | static_cast<uint32_t>(fc.z);
            if (ldig && r_blk != lr) {
                lflush();
                lr = r_blk;
            }
            if (digs && r_blk != dig_r) {
                dig_flush();
#pragma unroll
                for (int j = 0; j < NCH; ++j) dsum[j] = asum[j] = 0;
                dig_r = r_blk;
            }
            const int buf = acc_iter & 1;
            const uint32_t acc_phase = (acc_iter >> 1) & 1;
            const bool ok = mbar_wait(&acc_full[buf], acc_phase, abort, ep.err, ERR_TIMEOUT_EPI);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * C::NMMA +
                                  rsub * C::ROWS_PER_WARP;
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int row0 = r_blk * C::BR + rsub * C::ROWS_PER_WARP + 16 * j;
                if constexpr (KIND == EPI_RESID && P == 4) {
                    // four planes: two halves of 8 rows, so that a half's planes and residuals fit the
                    // 96 registers of the 16-warp epilogue without spilling
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int r0 = row0 + 8 * hh;
                        int32_t* xp = ep.out + static_cast<int64_t>(r0) * ep.ld + f;
                        int32_t x8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) x8[i] = (f_ok && r0 + i < ep.M) ? xp[i * ep.ld] : 0;
                        uint32_t v8[P][8];
#pragma unroll
                        for (int p = 0; p < P; ++p) tmem_ld8(tacc + p * C::BR + 16 * j + 8 * hh, v8[p]);
                        tmem_wait_ld();
#pragma unroll
                        for (int p = 0; p < P; ++p) tmem_launder(v8[p]);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int64_t y = (static_cast<int64_t>(tg_sum<P, 8>(v8, i, fc.x, kc)) >> fc.y) + x8[i];
                            const int32_t r = static_cast<int32_t>(
                                min(max(y, static_cast<int64_t>(INT32_MIN)), static_cast<int64_t>(INT32_MAX)));
                            if (f_ok && r0 + i < ep.M) xp[i * ep.ld] = r;
                        }
                    }
                    continue;
                }
                int32_t xo[16];
                if constexpr (KIND == EPI_RESID) {  // this lane's residual column of the 16 rows (coalesced over lanes)
                    const int32_t* xp = ep.out + static_cast<int64_t>(row0) * ep.ld + f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) xo[i] = (f_ok && row0 + i < ep.M) ? xp[i * ep.ld] : 0;
                }
                uint32_t v[P][16];
#pragma unroll
                for (int p = 0; p < P; ++p) tmem_ld16(tacc + p * C::BR + 16 * j, v[p]);
                tmem_wait_ld();
#pragma unroll
                for (int p = 0; p < P; ++p) tmem_launder(v[p]);
                if constexpr (KIND == EPI_LOGITS) {
                    // logits (python/intref.py:298-300, low 32 bits as exp_logits.i32 stores them)
                    int32_t* op = ep.out + static_cast<int64_t>(row0) * ep.ld + f;
                    uint32_t ys[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const uint64_t tt = tg_sum<P>(v, i, fc.x, kc);
                        ys[i] = __funnelshift_r(static_cast<uint32_t>(tt), static_cast<uint32_t>(tt >> 32), fc.y);
                        if (f_ok && row0 + i < ep.M) __stcs(op + i * ep.ld, static_cast<int32_t>(ys[i]));
                    }
                    // digest: per lane (feature f) s = sum_t uint32(out) dig_a[t] over rows of one sequence, then
                    // dig_b[f] s summed over the warp's lanes is added to that sequence's digest
                    if (ldig) {
                        auto flush = [&](int sq, uint64_t sum) {
                            uint64_t w = sum * wf;
#pragma unroll
                            for (int o = 16; o >= 1; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
                            if (lane == 0 && sq * ep.T < ep.M) atomicAdd(ep.dig + sq, static_cast<unsigned long long>(w));
                        };
                        const int seq0 = row0 / ep.T, t0 = row0 - seq0 * ep.T;
                        if (t0 + 16 <= ep.T) {  // the chunk lies in one sequence (always when 16 divides T)
                            const uint64_t* da = ep.dig_a + ep.pos0 + t0;
                            uint64_t s0 = 0, s1 = 0;
#pragma unroll
                            for (int i = 0; i < 16; i += 2) {
                                const uint64_t a0 = __ldg(da + i), a1 = __ldg(da + i + 1);
                                if (row0 + i < ep.M) s0 += static_cast<uint64_t>(ys[i]) * a0;
                                if (row0 + i + 1 < ep.M) s1 += static_cast<uint64_t>(ys[i + 1]) * a1;
                            }
                            lacc[j] += (s0 + s1) * wf;
                            lseq[j] = seq0;
                        } else {
                            int sq = seq0, t = t0;
                            uint64_t ds = 0;
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                if (row0 + i < ep.M) ds += static_cast<uint64_t>(ys[i]) * __ldg(ep.dig_a + ep.pos0 + t);
                                if (++t == ep.T) {
                                    flush(sq, ds);
                                    ds = 0;
                                    ++sq;
                                    t = 0;
                                }
                            }
                            if (t != 0) flush(sq, ds);
                        }
                    }
                }
                if constexpr (KIND == EPI_RESID) {
                    // x = SAT32(x + RS(acc m, s)) (python/intref.py:261,281; the residual term is not saturated)
                    int32_t* xp = ep.out + static_cast<int64_t>(row0) * ep.ld + f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int64_t y = (static_cast<int64_t>(tg_sum<P>(v, i, fc.x, kc)) >> fc.y) + xo[i];
                        const int32_t r = static_cast<int32_t>(min(max(y, static_cast<int64_t>(INT32_MIN)), static_cast<int64_t>(INT32_MAX)));
                        if (f_ok && row0 + i < ep.M) xp[i * ep.ld] = r;
                    }
                }
                if constexpr (KIND == EPI_SWEEP) {
                    int32_t ys[16];
                    if (P == 2 && ep.split) {
                        const int32_t lim = ep.bits_out < 32 ? (1 << (ep.bits_out - 1)) : 0;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            uint32_t ylo;
                            int32_t yhi;
                            tg_rs_split(v[0][i], v[1][i], fc.x, fc.y, static_cast<uint32_t>(fc.z), static_cast<uint32_t>(fc.w),
                                        ylo, yhi);
                            int32_t y = yhi == (static_cast<int32_t>(ylo) >> 31) ? static_cast<int32_t>(ylo)
                                                                                 : (yhi < 0 ? INT32_MIN : INT32_MAX);
                            if (lim) y = min(max(y, -lim), lim - 1);
                            ys[i] = y;
                        }
                    } else {
                        const int64_t lim = int64_t(1) << (ep.bits_out - 1);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            int64_t y = static_cast<int64_t>(tg_sum<P>(v, i, fc.x, kc)) >> fc.y;
                            y = min(max(y, -lim), lim - 1);
                            ys[i] = static_cast<int32_t>(y);
                        }
                    }
                    if (f_ok) {
                        int32_t* op = ep.out + static_cast<int64_t>(row0) * ep.ld + f;
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (row0 + i < ep.M) __stcs(op + i * ep.ld, ys[i]);
                    }
                    if (digs) {
                        uint64_t q[16];
                        if (ep.dig) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) q[i] = static_cast<uint64_t>(static_cast<uint32_t>(ys[i])) * wf;
                            dsum[j] += reduce_rows16(q, lane);
                        }
                        if (ep.dig_acc) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) q[i] = tg_acc<P>(v, i, corr) * wf;
                            asum[j] += reduce_rows16(q, lane);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        if (digs) dig_flush();
        if (ldig) lflush();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

}  // namespace eii
