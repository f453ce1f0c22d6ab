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
//   warps 2-9   epilogue: tcgen05.ld of the P accumulators, int64 plane combination, requantise
//               RS/SAT, and the fused step of the caller (RoPE, residual add, SiLU-gated product,
//               logits store), written straight to global memory.
// TMEM: P*128 int32 columns per accumulator set; 2 sets (double buffered) for P = 2, one for P = 4.
#pragma once
#include <cstdint>
#include <cuda.h>

#include "eii_int.cuh"
#include "eii_ptx.cuh"

namespace eii {

enum EpiKind : int { EPI_QKV = 0, EPI_RESID = 1, EPI_GATEUP = 2, EPI_LOGITS = 3, EPI_LINEAR = 4 };

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
    int16_t* q_out;
    int16_t* k_out;
    int16_t* v_out;
    const int32_t* rope_c;
    const int32_t* rope_s;
    int bits_q, bits_k, bits_v, bits_qr, bits_kr, rope_shift_q, rope_shift_k;
    // EPI_RESID: x [M,N] int32, x = SAT32(x + RS(acc m, shift))
    int32_t* x;
    // EPI_GATEUP: gate/up interleaved by tile (cols 0-63 gate j, 64-127 up j), gated -> planes
    const int32_t* silu;
    int bits_g, bits_u, gated_shift, bits_m, gated_P;
    uint8_t* gated_planes;  // [gated_P][M][N/2]
    // EPI_LOGITS: int32 out[row * ld + col] = RS(acc m, shift) (low 32 bits, no SAT)
    int32_t* logits;
    int64_t ld_logits;
    // EPI_LINEAR: int64 out = SAT(RS(acc m, shift), bits_out), optional int64 acc
    int64_t* out64;
    int64_t* acc64;
    int bits_out;
};

template <int P>
struct GemmCfg {
    static constexpr int BM = 128, BN = 128, BK = 128;
    static constexpr int ACC_COLS = P * BN;
    static constexpr int NB = 512 / ACC_COLS;  // accumulator sets in TMEM
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = P * A_BYTES + B_BYTES;
    static constexpr int STAGES = (P == 2) ? 4 : 2;
    static constexpr int EPI_WARPS = 8;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
    static_assert(NB >= 1, "accumulators must fit in TMEM");
};

// Load 16 consecutive accumulator columns of all P planes for this thread's row and combine.
template <int P>
__device__ __forceinline__ void load_acc16(uint32_t taddr, int64_t (&acc)[16]) {
    uint32_t v[P][16];
#pragma unroll
    for (int p = 0; p < P; ++p) tmem_ld16(taddr + p * 128, v[p]);
    tmem_wait_ld();
#pragma unroll
    for (int p = 0; p < P; ++p) tmem_launder(v[p]);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        int64_t a = 0;
#pragma unroll
        for (int p = 0; p < P; ++p) a += static_cast<int64_t>(static_cast<int32_t>(v[p][i])) * (int64_t(1) << (8 * p));
        acc[i] = a;
    }
}

__device__ __forceinline__ int64_t requant(int64_t acc, int2 ms, int bits) {
    return sat64(rs64(acc * static_cast<int64_t>(ms.x), ms.y), bits);
}

// ---------------------------------------------------------------------------------------------
template <int P, int KIND>
__device__ __forceinline__ void epilogue_tile(const EpiParams& ep, uint32_t tacc, int m_blk, int n_blk, int half,
                                              int quad, int lane) {
    const int row = m_blk * 128 + quad * 32 + lane;
    const bool row_ok = row < ep.M;
    const int n0 = n_blk * 128;
    if constexpr (KIND == EPI_QKV) {
        const int c0 = n0 + 64 * half;  // one head per warp half
        if (c0 >= ep.N) return;
        int region, head;  // 0 = q, 1 = k, 2 = v
        if (c0 < 576) { region = 0; head = c0 / 64; }
        else if (c0 < 768) { region = 1; head = (c0 - 576) / 64; }
        else { region = 2; head = (c0 - 768) / 64; }
        const int bits_in = region == 0 ? ep.bits_q : (region == 1 ? ep.bits_k : ep.bits_v);
        const int bits_r = region == 0 ? ep.bits_qr : ep.bits_kr;
        const int rshift = region == 0 ? ep.rope_shift_q : ep.rope_shift_k;
        int16_t* out = region == 0 ? ep.q_out : (region == 1 ? ep.k_out : ep.v_out);
        const int width = region == 0 ? 576 : 192;
        const int pos = row_ok ? row % ep.T : 0;
#pragma unroll 1
        for (int sub = 0; sub < 32; sub += 16) {
            int64_t aa[16], bb[16];
            load_acc16<P>(tacc + 64 * half + sub, aa);
            load_acc16<P>(tacc + 64 * half + 32 + sub, bb);
            if (!row_ok) continue;
            int16_t oa[16], ob[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int d = sub + i;
                const int64_t a = requant(aa[i], __ldg(ep.msh + c0 + d), bits_in);
                const int64_t b = requant(bb[i], __ldg(ep.msh + c0 + 32 + d), bits_in);
                if (region < 2) {
                    const int64_t c = __ldg(ep.rope_c + pos * 32 + d), s = __ldg(ep.rope_s + pos * 32 + d);
                    oa[i] = static_cast<int16_t>(sat64(rs64(a * c - b * s, rshift), bits_r));
                    ob[i] = static_cast<int16_t>(sat64(rs64(b * c + a * s, rshift), bits_r));
                } else {
                    oa[i] = static_cast<int16_t>(a);
                    ob[i] = static_cast<int16_t>(b);
                }
            }
            int16_t* dst = out + static_cast<int64_t>(row) * width + head * 64 + sub;
            reinterpret_cast<uint4*>(dst)[0] = *reinterpret_cast<uint4*>(&oa[0]);
            reinterpret_cast<uint4*>(dst)[1] = *reinterpret_cast<uint4*>(&oa[8]);
            reinterpret_cast<uint4*>(dst + 32)[0] = *reinterpret_cast<uint4*>(&ob[0]);
            reinterpret_cast<uint4*>(dst + 32)[1] = *reinterpret_cast<uint4*>(&ob[8]);
        }
    } else if constexpr (KIND == EPI_GATEUP) {
        const int j0 = n_blk * 64 + 32 * half;  // gated feature index of this half
        if (n0 >= ep.N) return;
        const int Nh = ep.N / 2;
#pragma unroll 1
        for (int sub = 0; sub < 32; sub += 16) {
            int64_t ga[16], ua[16];
            load_acc16<P>(tacc + 32 * half + sub, ga);
            load_acc16<P>(tacc + 64 + 32 * half + sub, ua);
            if (!row_ok) continue;
            int32_t gm[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int tc = 32 * half + sub + i;
                const int64_t g = requant(ga[i], __ldg(ep.msh + n0 + tc), ep.bits_g);
                const int64_t u = requant(ua[i], __ldg(ep.msh + n0 + 64 + tc), ep.bits_u);
                const int64_t sg = __ldg(ep.silu + (g + 32768));
                gm[i] = static_cast<int32_t>(sat64(rs64(sg * u, ep.gated_shift), ep.bits_m));
            }
            const int64_t base = static_cast<int64_t>(row) * Nh + j0 + sub;
            for (int p = 0; p < ep.gated_P; ++p) {
                uint8_t b[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) b[i] = plane_byte(gm[i], p);
                *reinterpret_cast<uint4*>(ep.gated_planes + static_cast<int64_t>(p) * ep.M * Nh + base) =
                    *reinterpret_cast<uint4*>(b);
            }
        }
    } else {
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
            const int tc = 64 * half + 16 * ch;
            const int gc = n0 + tc;
            if (gc >= ep.N) break;
            int64_t acc[16];
            load_acc16<P>(tacc + tc, acc);
            if (!row_ok) continue;
            if constexpr (KIND == EPI_RESID) {
                int32_t* xp = ep.x + static_cast<int64_t>(row) * ep.N + gc;
                int4 xv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) xv[q] = reinterpret_cast<const int4*>(xp)[q];
                const int32_t* xs = reinterpret_cast<const int32_t*>(xv);
                int32_t xo[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int2 ms = __ldg(ep.msh + gc + i);
                    const int64_t r = rs64(acc[i] * static_cast<int64_t>(ms.x), ms.y);
                    xo[i] = static_cast<int32_t>(sat64(static_cast<int64_t>(xs[i]) + r, 32));
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) reinterpret_cast<int4*>(xp)[q] = reinterpret_cast<int4*>(xo)[q];
            } else if constexpr (KIND == EPI_LOGITS) {
                int32_t o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int2 ms = __ldg(ep.msh + gc + i);
                    o[i] = static_cast<int32_t>(rs64(acc[i] * static_cast<int64_t>(ms.x), ms.y));
                }
                int32_t* op = ep.logits + static_cast<int64_t>(row) * ep.ld_logits + gc;
#pragma unroll
                for (int q = 0; q < 4; ++q) reinterpret_cast<int4*>(op)[q] = reinterpret_cast<int4*>(o)[q];
            } else {  // EPI_LINEAR
                int64_t* op = ep.out64 + static_cast<int64_t>(row) * ep.N + gc;
#pragma unroll
                for (int i = 0; i < 16; ++i) op[i] = requant(acc[i], __ldg(ep.msh + gc + i), ep.bits_out);
                if (ep.acc64) {
                    int64_t* ap = ep.acc64 + static_cast<int64_t>(row) * ep.N + gc;
#pragma unroll
                    for (int i = 0; i < 16; ++i) ap[i] = acc[i];
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
template <int P, int KIND>
__global__ void __launch_bounds__(GemmCfg<P>::THREADS, 1)
    k_plane_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, EpiParams ep) {
    using C = GemmCfg<P>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::STAGES;
    uint64_t* acc_full = bars + 2 * C::STAGES;
    uint64_t* acc_empty = acc_full + C::NB;
    uint64_t* drain = acc_empty + C::NB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_m = (ep.M + 127) / 128, num_n = (ep.N + 127) / 128;
    const int tiles = num_m * num_n;
    const int KB = (ep.K + 127) / 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < C::NB; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], C::EPI_WARPS); }
        mbar_init(drain, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t fills = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m_blk = t / num_n, n_blk = t % num_n;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort, ep.err, ERR_TIMEOUT_PRODUCER)) { ok = false; break; }
                    uint8_t* sA = smem + stage * C::STAGE_BYTES;
                    uint8_t* sB = sA + P * C::A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
#pragma unroll
                    for (int p = 0; p < P; ++p) tma_load_3d(sA + p * C::A_BYTES, &tmA, &full[stage], kb * 128, m_blk * 128, p);
                    tma_load_2d(sB, &tmB, &full[stage], kb * 128, n_blk * 128);
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
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++acc_iter) {
                const int n_blk = t % num_n;
                const int buf = acc_iter % C::NB;
                const uint32_t acc_phase = (acc_iter / C::NB) & 1;
                if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort, ep.err, ERR_TIMEOUT_MMA_ACC)) { ok = false; break; }
                tc_fence_after();
                const int n_valid = min(128, ep.N - n_blk * 128);
                const uint32_t id_lo = idesc_i8(false, true, n_valid);
                const uint32_t id_hi = idesc_i8(true, true, n_valid);
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
                            const uint64_t adesc = smem_desc_sw128(sA + p * C::A_BYTES + ks * 32);
                            mma_i8(dbase + p * 128, adesc, bdesc, p == P - 1 ? id_hi : id_lo,
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
        const int quad = warp & 3;
        const int half = e >> 2;
        int acc_iter = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++acc_iter) {
            const int m_blk = t / num_n, n_blk = t % num_n;
            const int buf = acc_iter % C::NB;
            const uint32_t acc_phase = (acc_iter / C::NB) & 1;
            if (!mbar_wait(&acc_full[buf], acc_phase, abort, ep.err, ERR_TIMEOUT_EPI)) break;
            tc_fence_after();
            const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * C::ACC_COLS;
            epilogue_tile<P, KIND>(ep, tacc, m_blk, n_blk, half, quad, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

}  // namespace eii
