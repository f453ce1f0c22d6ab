// Bandwidth-bound kernels of the forward pass: embedding gather, RMSNorm to byte planes,
// integer attention, plane split, logits digest.  Warp-per-row layouts with vectorised,
// coalesced HBM access; all arithmetic exact int64 (128-bit for the norm total).
#pragma once
#include <cstdint>

#include "eii_int.cuh"
#include "eii_ptx.cuh"

namespace eii {

constexpr int D_MODEL = 576, D_FF = 1536, VOCAB = 49152, N_LAYERS = 30;
constexpr int N_HEADS = 9, N_KV = 3, HEAD_DIM = 64, ROPE_POS = 512, DMAX = 12 * 128;
constexpr int F_RES = 15, F_SCORE = 7;
constexpr int64_t EPS_S = 6184753;  // round(1e-5 * 576 * 2^30), python/intref.py:37

enum : int { ERR_BAD_TOKEN = 201, ERR_BAD_SHIFT = 202, ERR_BAD_INPUT = 203 };

// --------------------------------------------------------------------------- embedding
// x[t,c] = RS(emb_q[id,c] * emb_m[id], emb_n[id] - 15)   (python/intref.py:163-166)
// One warp per token; lanes cover 576 bytes of the int8 row as 36 x 16-byte chunks.
__global__ void k_embed(const int64_t* __restrict__ ids, int M, const int8_t* __restrict__ emb_q,
                        const int32_t* __restrict__ emb_m, const int32_t* __restrict__ emb_n,
                        int32_t* __restrict__ x, int* err) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    griddep_wait();
    griddep_launch();
    if (row >= M) return;
    int64_t id = ids[row];
    if (id < 0 || id >= VOCAB) {
        if (lane == 0) atomicCAS(err, 0, ERR_BAD_TOKEN);
        id = 0;
    }
    const int64_t m = emb_m[id];
    const int sh = emb_n[id] - F_RES;
    const int4* src = reinterpret_cast<const int4*>(emb_q + id * D_MODEL);
    int32_t* dst = x + static_cast<int64_t>(row) * D_MODEL;
    for (int ch = lane; ch < D_MODEL / 16; ch += 32) {
        const int4 w = __ldg(src + ch);
        const int8_t* b = reinterpret_cast<const int8_t*>(&w);
        int32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = static_cast<int32_t>(rs64(static_cast<int64_t>(b[i]) * m, sh));
        int4* d4 = reinterpret_cast<int4*>(dst + ch * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) d4[q] = reinterpret_cast<int4*>(o)[q];
    }
}

// --------------------------------------------------------------------------- residual grid
// Narrow comparison mode (python/intref.py:303-308): x = SAT16(RS(x, s)) << s, per element, with the
// shift s of the element's channel (s[c], 0 <= s <= 16, so the result fits int32).  The per-tensor
// grid of the reference has one s = k of the residual site for all 576 channels; a per-channel grid
// (a Model subclass with one exponent per channel) has its own s per channel.
__global__ void k_residual_grid(int32_t* __restrict__ x, int64_t n, const uint8_t* __restrict__ s_ch) {
    griddep_wait();
    griddep_launch();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int s = __ldg(s_ch + i % D_MODEL);
        const int64_t rnd = s >= 1 ? (int64_t(1) << (s - 1)) : 0;
        const int64_t r = (static_cast<int64_t>(x[i]) + rnd) >> s;
        x[i] = static_cast<int32_t>(static_cast<uint32_t>(min(max(r, int64_t(-32768)), int64_t(32767))) << s);
    }
}

// --------------------------------------------------------------------------- RMSNorm
// Exact reciprocal root of python/intref.py:170-177 / c/intref.c:96-104:
//   S = A 2^32 + B 2^17 + C = sum x^2 (exact, 128-bit), U = isqrt(floor(2^80 / Tt)), Tt = S + EPS_S.
// For an integer u, u^2 <= floor(2^80 / Tt) iff u^2 Tt <= 2^80, so U is the largest u with
// u^2 Tt <= 2^80.  It is seeded from 2^40 / sqrt(Tt) in double precision (within one of U, since
// U < 2^29) and then corrected with exact 128-bit products, which avoids a 128-bit division.
__host__ __device__ __forceinline__ bool sq_times_le_2p80(uint64_t u, unsigned __int128 Tt) {
    const uint64_t u2 = u * u;  // u < 2^31 here, so u^2 < 2^62
    const uint64_t th = static_cast<uint64_t>(Tt >> 64), tl = static_cast<uint64_t>(Tt);
    const unsigned __int128 hi = static_cast<unsigned __int128>(u2) * th;
    if (hi > (static_cast<unsigned __int128>(1) << 16)) return false;  // (hi << 64) > 2^80
    const unsigned __int128 prod = (hi << 64) + static_cast<unsigned __int128>(u2) * tl;
    return prod <= (static_cast<unsigned __int128>(1) << 80);
}

__host__ __device__ __forceinline__ int64_t norm_recip_root(int64_t A, int64_t B, int64_t C) {
    const __int128 S = static_cast<__int128>(A) * (static_cast<__int128>(1) << 32) +
                       static_cast<__int128>(B) * (static_cast<__int128>(1) << 17) + static_cast<__int128>(C);
    const unsigned __int128 Tt = static_cast<unsigned __int128>(S) + static_cast<unsigned __int128>(EPS_S);
#ifdef __CUDA_ARCH__
    double est = 1099511627776.0 * rsqrt(static_cast<double>(Tt));  // 2^40 / sqrt(Tt); the loops fix U
#else
    double est = 1099511627776.0 / sqrt(static_cast<double>(Tt));
#endif
    if (est > 2147483647.0) est = 2147483647.0;
    uint64_t u = static_cast<uint64_t>(est);
    while (u > 0 && !sq_times_le_2p80(u, Tt)) --u;
    while (u < 2147483647u && sq_times_le_2p80(u + 1, Tt)) ++u;
    return static_cast<int64_t>(u);
}

__device__ __forceinline__ int64_t warp_sum64(int64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// out = SAT(RS(3 RS(x U, 16) g, 21 + fw - f_out), bits_out) (python/intref.py:178-181), written
// as P = bits_out / 8 byte planes [P][M][576] (planes != nullptr) and/or int64 [M,576].
// Two rows per warp: half-warp h owns row 2 w + h, lane l of it columns 64 i + 4 l .. + 3, i < 9
// (16-byte loads; 4-byte plane stores, 64 contiguous bytes per half-warp).
__device__ __forceinline__ int64_t half_sum64(int64_t v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void k_rmsnorm(const int32_t* __restrict__ x, int M, const int32_t* __restrict__ gain, int shift_out,
                          int bits_out, uint8_t* __restrict__ planes, int P, int64_t* __restrict__ out64,
                          int64_t* __restrict__ u_out, int64_t* __restrict__ z_out, uint32_t* __restrict__ zero_ptr,
                          int zero_n, int offset) {
    const int row = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 2 + ((threadIdx.x >> 4) & 1);
    const int l = threadIdx.x & 15;
    const bool live = row < M;
    griddep_wait();
    griddep_launch();
    if (zero_ptr && blockIdx.x == 0)  // flag words the next kernels fill (signed-digit gated planes)
        for (int i = threadIdx.x; i < zero_n; i += blockDim.x) zero_ptr[i] = 0;
    const int4* xr = reinterpret_cast<const int4*>(x + static_cast<int64_t>(live ? row : 0) * D_MODEL);
    int4 v[9];
    int64_t A = 0, B = 0, C = 0;
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        v[i] = live ? xr[16 * i + l] : make_int4(0, 0, 0, 0);
        const int32_t e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t h = e[u] >> 16, lo = e[u] & 0xFFFF;
            A += h * h;
            B += h * lo;
            C += lo * lo;
        }
    }
    A = half_sum64(A);
    B = half_sum64(B);
    C = half_sum64(C);
    if (!live) return;  // both halves of the warp are done with the shuffles
    const int64_t U = norm_recip_root(A, B, C);  // < 2^31
    const int32_t U32 = static_cast<int32_t>(U);
    // Fast path (planes output, bits_out 16, 1 <= shift_out <= 31): z = RS(x U, 16) fits int32
    // (|x U| <= 2^40, python/intref.py:178), 3 g fits int32, and RS(z 3 g, shift_out) is a funnel
    // shift of one 32x32 -> 64 multiply-add.
    // the per-row U and z of python/intref.py:183 for a trace (generic path only)
    if (u_out && l == 0) u_out[row] = U;
    const bool fast = planes && !out64 && !z_out && P == 2 && bits_out == 16 && shift_out >= 1 && shift_out <= 31;
    const int64_t rnd_out = (shift_out >= 1 && shift_out <= 62) ? (int64_t(1) << (shift_out - 1)) : 0;
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        const int c = 64 * i + 4 * l;
        const int4 g4 = __ldg(reinterpret_cast<const int4*>(gain) + 16 * i + l);
        const int32_t e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        const int32_t g[4] = {g4.x, g4.y, g4.z, g4.w};
        if (fast) {
            int32_t o[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t xu = static_cast<int64_t>(e[u]) * U32 + 32768;
                const int32_t z = static_cast<int32_t>(__funnelshift_r(static_cast<uint32_t>(xu),
                                                                       static_cast<uint32_t>(static_cast<uint64_t>(xu) >> 32), 16));
                const int64_t t = static_cast<int64_t>(z) * (3 * g[u]) + rnd_out;
                const uint32_t tl = static_cast<uint32_t>(t), th = static_cast<uint32_t>(static_cast<uint64_t>(t) >> 32);
                const uint32_t lo = __funnelshift_r(tl, th, shift_out);
                const int32_t hi = static_cast<int32_t>(th) >> shift_out;
                const int32_t w = hi == (static_cast<int32_t>(lo) >> 31) ? static_cast<int32_t>(lo) : (hi < 0 ? INT32_MIN : INT32_MAX);
                o[u] = min(max(w, -32768), 32767);
            }
            const uint32_t w01 = (static_cast<uint32_t>(o[0]) & 0xFFFFu) | (static_cast<uint32_t>(o[1]) << 16);
            const uint32_t w23 = (static_cast<uint32_t>(o[2]) & 0xFFFFu) | (static_cast<uint32_t>(o[3]) << 16);
            // plane 0 gets the low bytes (o0, o1, o2, o3), plane 1 the high bytes
            *reinterpret_cast<uint32_t*>(planes + static_cast<int64_t>(row) * D_MODEL + c) = __byte_perm(w01, w23, 0x6420);
            // offset-binary planes: the high byte's sign bit flipped
            *reinterpret_cast<uint32_t*>(planes + (static_cast<int64_t>(M) + row) * D_MODEL + c) =
                __byte_perm(w01, w23, 0x7531) ^ (offset ? 0x80808080u : 0u);
            continue;
        }
        int64_t o[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t z = rs64(static_cast<int64_t>(e[u]) * U, 16);
            if (z_out) z_out[static_cast<int64_t>(row) * D_MODEL + c + u] = z;
            o[u] = sat64(rs64(z * g[u] * 3, shift_out), bits_out);
        }
        if (planes) {
            const int64_t off = offset ? (int64_t(1) << (8 * P - 1)) : 0;  // offset-binary planes of o + 2^(8P-1)
            for (int p = 0; p < P; ++p) {
                const uint32_t quad = static_cast<uint32_t>(plane_byte(o[0] + off, p)) |
                                      (static_cast<uint32_t>(plane_byte(o[1] + off, p)) << 8) |
                                      (static_cast<uint32_t>(plane_byte(o[2] + off, p)) << 16) |
                                      (static_cast<uint32_t>(plane_byte(o[3] + off, p)) << 24);
                *reinterpret_cast<uint32_t*>(planes + (static_cast<int64_t>(p) * M + row) * D_MODEL + c) = quad;
            }
        }
        if (out64) {
#pragma unroll
            for (int u = 0; u < 4; ++u) out64[static_cast<int64_t>(row) * D_MODEL + c + u] = o[u];
        }
    }
}

// RMSNorm of the forward pass proper: two INT16 byte planes [2][M][576] out, output shift in
// [10, 31] (the engine checks both before choosing this kernel), nothing else written.
//  - sum x^2 exactly in 96 bits: |x|^2 by a 32x32 -> 64 multiply-add with carry into three words
//    (|x| <= 2^31, 36 terms per lane < 2^68, a row < 2^72);
//  - U = floor(2^40 / sqrt(Tt)) = isqrt(floor(2^80 / Tt)) seeded in double precision from the two
//    words of Tt and corrected with exact products (norm_recip_root);
//  - z = RS(x U, 16) fits int32 (|x U| <= 2^40), |z 3 g + 2^(s-1)| < 2^40.6 + 2^30, so with s >= 10
//    RS(z 3 g, s) fits int32 and SAT16 is a clamp of the low word of a funnel shift.
__device__ __forceinline__ void sq_acc96(uint32_t& a0, uint32_t& a1, uint32_t& a2, int32_t x) {
    const uint32_t u = x < 0 ? 0u - static_cast<uint32_t>(x) : static_cast<uint32_t>(x);
    asm("mad.lo.cc.u32 %0, %3, %3, %0;\n\t"
        "madc.hi.cc.u32 %1, %3, %3, %1;\n\t"
        "addc.u32 %2, %2, 0;"
        : "+r"(a0), "+r"(a1), "+r"(a2)
        : "r"(u));
}

__device__ __forceinline__ void add96(uint32_t& a0, uint32_t& a1, uint32_t& a2, uint32_t b0, uint32_t b1, uint32_t b2) {
    asm("add.cc.u32 %0, %0, %3;\n\t"
        "addc.cc.u32 %1, %1, %4;\n\t"
        "addc.u32 %2, %2, %5;"
        : "+r"(a0), "+r"(a1), "+r"(a2)
        : "r"(b0), "r"(b1), "r"(b2));
}

// The per-row part of the two-plane RMSNorm, shared by k_rmsnorm_p16 and k_embed_norm.  A warp normalises two rows: lanes 0-15 the
// row `row` of the lower half-warp, lanes 16-31 that of the upper; lane l of a half holds columns
// 64 i + 4 l .. 64 i + 4 l + 3 (i < 9) in v[i].  The whole warp calls it (shuffles); a row >= M
// (live false, v zero) stores nothing.
__device__ __forceinline__ void rmsnorm_pair_finish(const int4 (&v)[9], int row, bool live, int M,
                                                    const int32_t* __restrict__ gain, int shift_out,
                                                    uint8_t* __restrict__ planes, uint32_t top_flip) {
    const int l = threadIdx.x & 15;
    uint32_t a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        sq_acc96(a0, a1, a2, v[i].x);
        sq_acc96(a0, a1, a2, v[i].y);
        sq_acc96(a0, a1, a2, v[i].z);
        sq_acc96(a0, a1, a2, v[i].w);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        const uint32_t b0 = __shfl_xor_sync(0xffffffffu, a0, o), b1 = __shfl_xor_sync(0xffffffffu, a1, o),
                       b2 = __shfl_xor_sync(0xffffffffu, a2, o);
        add96(a0, a1, a2, b0, b1, b2);
    }
    if (!live) return;  // both halves of the warp are done with the shuffles
    add96(a0, a1, a2, static_cast<uint32_t>(EPS_S), 0u, 0u);  // Tt = S + EPS_S (EPS_S < 2^32)
    const uint64_t tlo = (static_cast<uint64_t>(a1) << 32) | a0;
    const unsigned __int128 Tt = (static_cast<unsigned __int128>(a2) << 64) | tlo;
    double est = 1099511627776.0 * rsqrt(fma(static_cast<double>(a2), 18446744073709551616.0, static_cast<double>(tlo)));
    if (est > 2147483647.0) est = 2147483647.0;
    uint64_t u = static_cast<uint64_t>(est);
    while (u > 0 && !sq_times_le_2p80(u, Tt)) --u;
    while (u < 2147483647u && sq_times_le_2p80(u + 1, Tt)) ++u;
    const int32_t U = static_cast<int32_t>(u);
    const int64_t rnd_out = int64_t(1) << (shift_out - 1);
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        const int c = 64 * i + 4 * l;
        const int4 g4 = __ldg(reinterpret_cast<const int4*>(gain) + 16 * i + l);
        const int32_t e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        const int32_t g[4] = {g4.x, g4.y, g4.z, g4.w};
        int32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t xu = static_cast<int64_t>(e[q]) * U + 32768;
            const int32_t z = static_cast<int32_t>(
                __funnelshift_r(static_cast<uint32_t>(xu), static_cast<uint32_t>(static_cast<uint64_t>(xu) >> 32), 16));
            const int64_t t = static_cast<int64_t>(z) * (3 * g[q]) + rnd_out;
            o[q] = static_cast<int32_t>(
                __funnelshift_r(static_cast<uint32_t>(t), static_cast<uint32_t>(static_cast<uint64_t>(t) >> 32), shift_out));
        }
        // SAT16 and the int16 pairs (o0 | o1 << 16, o2 | o3 << 16) by saturating packs
        const uint32_t w01 = pack_sat_s16(o[1], o[0]);
        const uint32_t w23 = pack_sat_s16(o[3], o[2]);
        // plane 0 gets the low bytes (o0, o1, o2, o3), plane 1 the high bytes
        *reinterpret_cast<uint32_t*>(planes + static_cast<int64_t>(row) * D_MODEL + c) = __byte_perm(w01, w23, 0x6420);
        // top_flip = 0x80808080: offset-binary planes (the high byte's sign bit flipped)
        *reinterpret_cast<uint32_t*>(planes + (static_cast<int64_t>(M) + row) * D_MODEL + c) = __byte_perm(w01, w23, 0x7531) ^ top_flip;
    }
}

// Loads the two rows of a warp (layout of rmsnorm_pair_finish) and normalises them.
__device__ __forceinline__ void rmsnorm_pair_p16(const int32_t* __restrict__ x, int row, int M, const int32_t* __restrict__ gain,
                                                 int shift_out, uint8_t* __restrict__ planes, uint32_t top_flip) {
    const int l = threadIdx.x & 15;
    const bool live = row < M;
    const int4* xr = reinterpret_cast<const int4*>(x + static_cast<int64_t>(live ? row : 0) * D_MODEL);
    int4 v[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) v[i] = live ? xr[16 * i + l] : make_int4(0, 0, 0, 0);
    rmsnorm_pair_finish(v, row, live, M, gain, shift_out, planes, top_flip);
}

// Four 256-thread blocks per SM (at most 64 registers): more loads in flight on the HBM-bound path.
__global__ void __launch_bounds__(256, 4) k_rmsnorm_p16(const int32_t* __restrict__ x, int M, const int32_t* __restrict__ gain,
                                                      int shift_out, uint8_t* __restrict__ planes,
                                                      uint32_t* __restrict__ zero_ptr, int zero_n, uint32_t top_flip) {
    const int row = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 2 + ((threadIdx.x >> 4) & 1);
    griddep_wait();
    griddep_launch();
    if (zero_ptr && blockIdx.x == 0)  // flag words the next kernels fill (signed-digit gated planes)
        for (int i = threadIdx.x; i < zero_n; i += blockDim.x) zero_ptr[i] = 0;
    rmsnorm_pair_p16(x, row, M, gain, shift_out, planes, top_flip);
}

// Embedding (as k_embed) with the first layer's RMSNorm fused: two rows per warp in the layout of
// rmsnorm_pair_finish (lane l of a half-warp builds columns 64 i + 4 l .. +3 of its row from one
// 4-byte load per i), x is stored and the norm runs on the values in registers.
__global__ void __launch_bounds__(256) k_embed_norm(const int64_t* __restrict__ ids, int M, const int8_t* __restrict__ emb_q,
                                                   const int32_t* __restrict__ emb_m, const int32_t* __restrict__ emb_n,
                                                   int32_t* __restrict__ x, int* err, const int32_t* __restrict__ gain,
                                                   int shift_out, uint8_t* __restrict__ planes, uint32_t top_flip) {
    const int row = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 2 + ((threadIdx.x >> 4) & 1);
    const int l = threadIdx.x & 15;
    const bool live = row < M;
    griddep_wait();
    griddep_launch();
    int64_t id = live ? ids[row] : 0;
    if (id < 0 || id >= VOCAB) {
        if (l == 0) atomicCAS(err, 0, ERR_BAD_TOKEN);
        id = 0;
    }
    const int64_t m = emb_m[id];
    const int sh = emb_n[id] - F_RES;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(emb_q + id * D_MODEL);
    int4* dst = reinterpret_cast<int4*>(x + static_cast<int64_t>(live ? row : 0) * D_MODEL);
    int4 v[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        const uint32_t w = __ldg(src + 16 * i + l);
        int32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            o[q] = static_cast<int32_t>(rs64(static_cast<int64_t>(static_cast<int8_t>(w >> (8 * q))) * m, sh));
        v[i] = make_int4(o[0], o[1], o[2], o[3]);
        if (live) dst[16 * i + l] = v[i];
    }
    rmsnorm_pair_finish(v, row, live, M, gain, shift_out, planes, top_flip);
}

// --------------------------------------------------------------------------- row-blocked planes
// Activation byte planes read by the GEMMs through the row-blocked layout
// [P][ceil(M/128)][K/16][128 rows][16 bytes]: byte k of row r of a plane sits at blocked_off(r, k, K),
// so 32 consecutive rows x 16 bytes are 512 contiguous bytes (coalesced epilogue stores) and a GEMM
// reads a 128-row x 128-byte K block as eight 2 KB runs (see map_blocked on the host).
__host__ __device__ __forceinline__ int64_t blocked_off(int64_t r, int k, int K) {
    return (r >> 7) * 128 * K + (k >> 4) * 2048 + (r & 127) * 16 + (k & 15);
}
__host__ __device__ __forceinline__ int64_t blocked_plane_stride(int64_t M, int K) { return ((M + 127) / 128) * 128 * K; }

// --------------------------------------------------------------------------- attention
// Integer causal attention of one sequence and one KV group (3 query heads), CUDA cores.
//   s_ij = SAT16(RS(q_i . k_j, shift_s)), j <= i; rowmax; e = E[rowmax - s] (0 beyond DMAX);
//   Z = sum e; P = floor((e 65536 + floor(Z/2)) / Z); ctx = SAT(RS(sum_j P v_j, shift_c), bits_c)
// (python/intref.py:227-254, c/intref.c:160-187).  K and V of the group sit in shared memory as
// int16 pairs with a 33-word row pitch (conflict-free column access); each warp owns one query
// row at a time; lanes split the keys for the scores and the 64 dims for P.V.
// The division by the per-row invariant Z is exact: a double-precision estimate of n / Z
// (n < 2^47, Z < 2^40) is off by at most one and is corrected with integer remainders.
struct AttnParams {
    const int16_t* q;  // [M, 576]
    const int16_t* k;  // [M, 192]
    const int16_t* v;  // [M, 192]
    const int32_t* exp_tab;  // [DMAX + 1]
    uint8_t* ctx_planes;     // row-blocked [P][ceil(M/128)][576/16][128 rows][16 bytes] (see blocked_off)
    int P;
    int offset;              // context planes in offset binary (the bytes of ctx + 2^(8P-1)), as the feature-major O GEMM reads them
    int M, T;
    int shift_s, shift_c, bits_c;
    int generic;  // k_attention_tc: take the 64-bit score and context requantisation for every shift (test switch)
    // optional trace outputs of k_attention (python/intref.py:249-250): [M/T][9][T][T] scores (s for
    // j <= i) and probabilities P; entries above the diagonal are left to the caller (zeroed)
    int32_t* score_out;
    int32_t* prob_out;
};

constexpr int ATTN_WARPS = 8;

__host__ __device__ constexpr int attn_smem_bytes(int T) {
    return 2 * T * 33 * 4 + (DMAX + 1 + 3) * 4 + ATTN_WARPS * (T + 32) * 4;
}

__device__ __forceinline__ int64_t dot_pair(uint32_t a, uint32_t b) {
    const int32_t a0 = static_cast<int16_t>(a & 0xFFFF), a1 = static_cast<int16_t>(a >> 16);
    const int32_t b0 = static_cast<int16_t>(b & 0xFFFF), b1 = static_cast<int16_t>(b >> 16);
    return static_cast<int64_t>(a0) * b0 + static_cast<int64_t>(a1) * b1;
}

__global__ void __launch_bounds__(ATTN_WARPS * 32) k_attention(AttnParams ap) {
    extern __shared__ __align__(16) uint32_t sm[];
    const int T = ap.T;
    const int seq = blockIdx.x / N_KV, g = blockIdx.x % N_KV;
    const int64_t row0 = static_cast<int64_t>(seq) * T;
    uint32_t* Ks = sm;                 // [T][33]
    uint32_t* Vs = Ks + T * 33;        // [T][33]
    int32_t* E = reinterpret_cast<int32_t*>(Vs + T * 33);  // [DMAX + 1]
    int32_t* wbuf = E + DMAX + 1 + 3;  // per warp: [T] scores/probabilities + [32] q row
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    griddep_wait();
    griddep_launch();

    for (int i = threadIdx.x; i < T * 32; i += blockDim.x) {
        const int j = i / 32, w = i % 32;
        Ks[j * 33 + w] = reinterpret_cast<const uint32_t*>(ap.k + (row0 + j) * 192 + g * 64)[w];
        Vs[j * 33 + w] = reinterpret_cast<const uint32_t*>(ap.v + (row0 + j) * 192 + g * 64)[w];
    }
    for (int i = threadIdx.x; i <= DMAX; i += blockDim.x) E[i] = ap.exp_tab[i];
    __syncthreads();

    int32_t* sc = wbuf + warp * (T + 32);
    uint32_t* qrow = reinterpret_cast<uint32_t*>(sc + T);
    for (int item = warp; item < 3 * T; item += ATTN_WARPS) {
        const int hh = g * 3 + item / T;
        const int i = item % T;
        qrow[lane] = reinterpret_cast<const uint32_t*>(ap.q + (row0 + i) * D_MODEL + hh * 64)[lane];
        __syncwarp();
        int32_t lmax = INT32_MIN;
        for (int j = lane; j <= i; j += 32) {
            int64_t acc = 0;
            const uint32_t* kr = Ks + j * 33;
#pragma unroll 8
            for (int w = 0; w < 32; ++w) acc += dot_pair(qrow[w], kr[w]);
            const int32_t s = static_cast<int32_t>(sat64(rs64(acc, ap.shift_s), 16));
            sc[j] = s;
            lmax = max(lmax, s);
            if (ap.score_out) ap.score_out[((static_cast<int64_t>(seq) * N_HEADS + hh) * T + i) * T + j] = s;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
        int64_t lz = 0;
        for (int j = lane; j <= i; j += 32) {
            const int32_t d = lmax - sc[j];
            const int32_t e = d <= DMAX ? E[d] : 0;
            sc[j] = e;
            lz += e;
        }
        const int64_t Z = warp_sum64(lz);
        const int64_t half = Z / 2;
        const double rz = 1.0 / static_cast<double>(Z);
        for (int j = lane; j <= i; j += 32) {
            const int64_t n = static_cast<int64_t>(sc[j]) * 65536 + half;
            int64_t p = static_cast<int64_t>(static_cast<double>(n) * rz);
            int64_t r = n - p * Z;
            if (r < 0) { --p; r += Z; }
            if (r < 0) { --p; r += Z; }
            if (r >= Z) { ++p; r -= Z; }
            if (r >= Z) { ++p; }
            sc[j] = static_cast<int32_t>(p);
            if (ap.prob_out) ap.prob_out[((static_cast<int64_t>(seq) * N_HEADS + hh) * T + i) * T + j] = static_cast<int32_t>(p);
        }
        __syncwarp();
        int64_t a0 = 0, a1 = 0;
        for (int j = 0; j <= i; ++j) {
            const int64_t p = sc[j];
            const uint32_t vv = Vs[j * 33 + lane];
            a0 += p * static_cast<int16_t>(vv & 0xFFFF);
            a1 += p * static_cast<int16_t>(vv >> 16);
        }
        const int64_t c0 = sat64(rs64(a0, ap.shift_c), ap.bits_c), c1 = sat64(rs64(a1, ap.shift_c), ap.bits_c);
        const int64_t r = row0 + i;
        const int col = hh * 64 + 2 * lane;
        const int64_t pstride = blocked_plane_stride(ap.M, D_MODEL);
        const int64_t off = ap.offset ? (int64_t(1) << (8 * ap.P - 1)) : 0;
        for (int p = 0; p < ap.P; ++p) {
            const uint16_t pair =
                static_cast<uint16_t>(plane_byte(c0 + off, p)) | (static_cast<uint16_t>(plane_byte(c1 + off, p)) << 8);
            *reinterpret_cast<uint16_t*>(ap.ctx_planes + p * pstride + blocked_off(r, col, D_MODEL)) = pair;
        }
        __syncwarp();
    }
}

// --------------------------------------------------------------------------- decode attention
// One query row per sequence against a K/V cache (incremental decoding): row i = L - 1 of the causal
// attention above, with keys 0 .. L-1 read from the cache [n_seq][max_T][192] (post-RoPE k, and v,
// exactly as the prompt pass stored them).  Same integer operations
// as k_attention, so the row equals the one a full recomputation produces.
struct AttnDecodeParams {
    const int16_t* q;        // [n, 576] queries of this step
    const int16_t* k_step;   // [n, 192] this step's k (post-RoPE) and v rows: key L - 1, appended to the
    const int16_t* v_step;   //   cache at row L - 1 by the kernel
    int16_t* kc;             // cache of this layer, first sequence of the launch
    int16_t* vc;
    int max_T;               // cache rows per sequence
    int L;                   // keys per sequence (position + 1), <= DECODE_MAX_L
    const int32_t* exp_tab;  // [DMAX + 1]
    uint8_t* ctx_planes;     // row-blocked planes (blocked_off), rows = sequences
    int P, M;
    int offset;              // offset-binary context planes (AttnParams::offset)
    int shift_s, shift_c, bits_c;
};

constexpr int DECODE_MAX_L = ROPE_POS;

// 4-way byte dot products with mixed signedness (PTX dp4a.atype.btype): u8 x u8, s8 x u8, u8 x s8.
__device__ __forceinline__ int32_t dp4a_uu(uint32_t a, uint32_t b, int32_t c) {
    uint32_t d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(static_cast<uint32_t>(c)));
    return static_cast<int32_t>(d);
}
__device__ __forceinline__ int32_t dp4a_su(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
constexpr int DECODE_THREADS = 128;

// Appends this step's k and v rows of (sequence seq, KV group g) to the cache at row L - 1: 128 bytes
// each, as eight 16-byte pieces (threads 0 .. 15).  Only this block reads that part of the cache in
// this launch, and it reads key L - 1 from the step's rows, so the append needs no ordering.
__device__ __forceinline__ void decode_append(const AttnDecodeParams& ap, int seq, int g, int tid) {
    if (tid < 16) {
        const int c = tid & 7;
        const int16_t* src = (tid < 8 ? ap.k_step : ap.v_step) + static_cast<int64_t>(seq) * 192 + g * 64;
        int16_t* dst = (tid < 8 ? ap.kc : ap.vc) + (static_cast<int64_t>(seq) * ap.max_T + ap.L - 1) * 192 + g * 64;
        reinterpret_cast<int4*>(dst)[c] = reinterpret_cast<const int4*>(src)[c];
    }
}

// Block = one (sequence, KV group): each key row k_j is read once and scored against the group's
// three query heads; scores, then e, then P live in shared memory; P.V runs one thread per (head,
// dim pair).  For any L <= DECODE_MAX_L; k_attention_decode_s below covers L <= DECODE_STAGE_L.
__global__ void __launch_bounds__(DECODE_THREADS) k_attention_decode(AttnDecodeParams ap) {
    __shared__ int32_t E[DMAX + 1 + 3];
    __shared__ uint2 qb[3][16];  // per head, 4 dims per entry: (low bytes u8 x4, high bytes s8 x4)
    __shared__ __align__(16) int32_t S[3][DECODE_MAX_L];  // also the P.V partial sums (6 KB) at the end
    __shared__ int32_t red_max[3][DECODE_THREADS / 32];
    __shared__ int64_t red_z[3][DECODE_THREADS / 32];
    const int seq = blockIdx.x / N_KV, g = blockIdx.x % N_KV;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32, L = ap.L;
    griddep_wait();
    griddep_launch();
    for (int i = tid; i <= DMAX; i += DECODE_THREADS) E[i] = ap.exp_tab[i];
    if (tid < 48) {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(ap.q + static_cast<int64_t>(seq) * D_MODEL + (g * 3 + tid / 16) * 64) +
                              tid % 16);
        qb[tid / 16][tid % 16] = make_uint2(__byte_perm(w.x, w.y, 0x6420), __byte_perm(w.x, w.y, 0x7531));
    }
    decode_append(ap, seq, g, tid);
    __syncthreads();
    const int16_t* kb = ap.kc + static_cast<int64_t>(seq) * ap.max_T * 192 + g * 64;
    const int16_t* vb = ap.vc + static_cast<int64_t>(seq) * ap.max_T * 192 + g * 64;
    const int16_t* k_last = ap.k_step + static_cast<int64_t>(seq) * 192 + g * 64;
    const int16_t* v_last = ap.v_step + static_cast<int64_t>(seq) * 192 + g * 64;
    // scores s_hj = SAT16(RS(q_h . k_j, shift_s))
    int32_t lmax[3] = {INT32_MIN, INT32_MIN, INT32_MIN};
    for (int j = tid; j < L; j += DECODE_THREADS) {
        const uint4* k4 = reinterpret_cast<const uint4*>(j == L - 1 ? k_last : kb + static_cast<int64_t>(j) * 192);
        // q.k = 65536 D2 + 256 D1 + D0 over byte planes with 4-way byte dot products (each partial
        // sum is below 64 * 255 * 255 < 2^31, as in the tensor-core attention)
        int32_t d0[3] = {0, 0, 0}, d1[3] = {0, 0, 0}, d2[3] = {0, 0, 0};
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const uint4 t = __ldg(k4 + w);
            const uint32_t k0a = __byte_perm(t.x, t.y, 0x6420), k1a = __byte_perm(t.x, t.y, 0x7531);
            const uint32_t k0b = __byte_perm(t.z, t.w, 0x6420), k1b = __byte_perm(t.z, t.w, 0x7531);
#pragma unroll
            for (int h = 0; h < 3; ++h) {
                const uint2 qa = qb[h][2 * w], qc = qb[h][2 * w + 1];
                d0[h] = dp4a_uu(qa.x, k0a, d0[h]);
                d0[h] = dp4a_uu(qc.x, k0b, d0[h]);
                d1[h] = dp4a_su(qa.y, k0a, d1[h]);
                d1[h] = dp4a_su(qc.y, k0b, d1[h]);
                d1[h] = dp4a_us(qa.x, k1a, d1[h]);
                d1[h] = dp4a_us(qc.x, k1b, d1[h]);
                d2[h] = __dp4a(static_cast<int>(qa.y), static_cast<int>(k1a), d2[h]);
                d2[h] = __dp4a(static_cast<int>(qc.y), static_cast<int>(k1b), d2[h]);
            }
        }
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            const int64_t acc = static_cast<int64_t>(d2[h]) * 65536 + static_cast<int64_t>(d1[h]) * 256 + d0[h];
            const int32_t sj = static_cast<int32_t>(sat64(rs64(acc, ap.shift_s), 16));
            S[h][j] = sj;
            lmax[h] = max(lmax[h], sj);
        }
    }
#pragma unroll
    for (int h = 0; h < 3; ++h) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lmax[h] = max(lmax[h], __shfl_xor_sync(0xffffffffu, lmax[h], o));
        if (lane == 0) red_max[h][warp] = lmax[h];
    }
    __syncthreads();
    int32_t rmax[3];
#pragma unroll
    for (int h = 0; h < 3; ++h) {
        rmax[h] = red_max[h][0];
#pragma unroll
        for (int w = 1; w < DECODE_THREADS / 32; ++w) rmax[h] = max(rmax[h], red_max[h][w]);
    }
    // e_hj = E[rowmax_h - s_hj] (0 beyond DMAX), Z_h = sum_j e_hj
    int64_t lz[3] = {0, 0, 0};
    for (int j = tid; j < L; j += DECODE_THREADS) {
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            const int32_t dd = rmax[h] - S[h][j];
            const int32_t ej = dd <= DMAX ? E[dd] : 0;
            S[h][j] = ej;
            lz[h] += ej;
        }
    }
#pragma unroll
    for (int h = 0; h < 3; ++h) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lz[h] += __shfl_xor_sync(0xffffffffu, lz[h], o);
        if (lane == 0) red_z[h][warp] = lz[h];
    }
    __syncthreads();
    // P_hj = floor((e_hj 65536 + floor(Z_h/2)) / Z_h), exact (double estimate, integer remainder fix-up)
#pragma unroll
    for (int h = 0; h < 3; ++h) {
        int64_t Z = 0;
#pragma unroll
        for (int w = 0; w < DECODE_THREADS / 32; ++w) Z += red_z[h][w];
        const int64_t half = Z / 2;
        const double rz = 1.0 / static_cast<double>(Z);
        for (int j = tid; j < L; j += DECODE_THREADS) {
            const int64_t n = static_cast<int64_t>(S[h][j]) * 65536 + half;
            int64_t p = static_cast<int64_t>(static_cast<double>(n) * rz);
            int64_t r = n - p * Z;
            if (r < 0) { --p; r += Z; }
            if (r < 0) { --p; r += Z; }
            if (r >= Z) { ++p; r -= Z; }
            if (r >= Z) { ++p; }
            S[h][j] = static_cast<int32_t>(p);
        }
    }
    __syncthreads();
    // ctx_hd = SAT(RS(sum_j P_hj v_jd, shift_c), bits_c): thread (key quarter tid / 32, dims 2 lane,
    // 2 lane + 1) sums keys j = quarter (mod 4) for the three heads; the quarters add up in shared memory.
    const int kq = tid / 32;
    int64_t a0[3] = {0, 0, 0}, a1[3] = {0, 0, 0};
    const uint32_t* vl = reinterpret_cast<const uint32_t*>(vb) + lane;
#pragma unroll 4
    for (int j = kq; j < L; j += 4) {
        const uint32_t vv = j == L - 1 ? __ldg(reinterpret_cast<const uint32_t*>(v_last) + lane)
                                       : __ldg(vl + static_cast<int64_t>(j) * 96);
        const int32_t v0 = static_cast<int16_t>(vv & 0xFFFF), v1 = static_cast<int16_t>(vv >> 16);
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            const int64_t p = S[h][j];
            a0[h] += p * v0;
            a1[h] += p * v1;
        }
    }
    __syncthreads();  // S is no longer read: reuse it for the partial sums
    int64_t* part = reinterpret_cast<int64_t*>(&S[0][0]);  // [4 quarters][3 heads][32 lanes][2]
#pragma unroll
    for (int h = 0; h < 3; ++h) {
        part[((kq * 3 + h) * 32 + lane) * 2] = a0[h];
        part[((kq * 3 + h) * 32 + lane) * 2 + 1] = a1[h];
    }
    __syncthreads();
    if (tid >= 96) return;
    const int h = tid / 32;
    int64_t c0 = 0, c1 = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        c0 += part[((q * 3 + h) * 32 + lane) * 2];
        c1 += part[((q * 3 + h) * 32 + lane) * 2 + 1];
    }
    c0 = sat64(rs64(c0, ap.shift_c), ap.bits_c);
    c1 = sat64(rs64(c1, ap.shift_c), ap.bits_c);
    const int col = (g * 3 + h) * 64 + 2 * lane;
    const int64_t pstride = blocked_plane_stride(ap.M, D_MODEL);
    const int64_t off = ap.offset ? (int64_t(1) << (8 * ap.P - 1)) : 0;
    for (int p = 0; p < ap.P; ++p) {
        const uint16_t pair =
            static_cast<uint16_t>(plane_byte(c0 + off, p)) | (static_cast<uint16_t>(plane_byte(c1 + off, p)) << 8);
        *reinterpret_cast<uint16_t*>(ap.ctx_planes + p * pstride + blocked_off(seq, col, D_MODEL)) = pair;
    }
}

// Decode attention for L <= DECODE_STAGE_L keys, with the block's K and V rows staged in shared memory.
// The same integer operations as k_attention_decode, so both give the row a full recomputation gives.
// Latency is what bounds a decoding step (a few hundred sequences, tens of microseconds per kernel),
// so the block issues every cache read up front as 16-byte asynchronous copies (one DRAM latency
// instead of one per dependent load batch), looks the exp table up through L1 instead of staging
// all of it, accumulates P.V with 32x32->64 multiply-adds, and keeps to 46 registers per thread and
// about 19 KB of shared memory at L = 66, so that 11 blocks fit on an SM and the 1536 blocks of a
// 512-sequence step run as one wave.
constexpr int DECODE_STAGE_L = 128;
constexpr int DECODE_K_PITCH = 144;  // bytes per staged key row: 8 threads' 16-byte reads of 8 rows hit distinct banks

__host__ __device__ constexpr int decode_stage_smem(int L) {
    // [K rows, pitch 144 B; reused for the P.V partial sums, 6 KB] [V rows, 128 B] [scores / e / P: 3 x L int32]
    return ((L * DECODE_K_PITCH > 6144 ? L * DECODE_K_PITCH : 6144) + L * 128 + 3 * L * 4 + 15) & ~15;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

__global__ void __launch_bounds__(DECODE_THREADS, 11) k_attention_decode_s(AttnDecodeParams ap) {
    extern __shared__ __align__(16) uint8_t dsm[];
    const int L = ap.L;
    const int kbytes = L * DECODE_K_PITCH > 6144 ? L * DECODE_K_PITCH : 6144;
    uint8_t* Ks = dsm;
    uint8_t* Vs = dsm + kbytes;
    int32_t* S = reinterpret_cast<int32_t*>(Vs + L * 128);  // [3][L]
    __shared__ uint2 qb[3][16];  // per head, 4 dims per entry: (low bytes u8 x4, high bytes s8 x4)
    __shared__ int32_t red_max[3][DECODE_THREADS / 32];
    __shared__ int64_t red_z[3][DECODE_THREADS / 32];
    const int seq = blockIdx.x / N_KV, g = blockIdx.x % N_KV;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    griddep_wait();  // q, k, v of this step are the previous kernel's output
    griddep_launch();
    {   // stage keys 0 .. L-2 from the cache and key L - 1 from this step's rows; append the latter
        const int16_t* kb = ap.kc + static_cast<int64_t>(seq) * ap.max_T * 192 + g * 64;
        const int16_t* vb = ap.vc + static_cast<int64_t>(seq) * ap.max_T * 192 + g * 64;
        const int16_t* k_last = ap.k_step + static_cast<int64_t>(seq) * 192 + g * 64;
        const int16_t* v_last = ap.v_step + static_cast<int64_t>(seq) * 192 + g * 64;
        for (int u = tid; u < L * 8; u += DECODE_THREADS) {
            const int j = u >> 3, c = u & 7;
            const int16_t* ks = j == L - 1 ? k_last : kb + static_cast<int64_t>(j) * 192;
            const int16_t* vs = j == L - 1 ? v_last : vb + static_cast<int64_t>(j) * 192;
            cp_async16(Ks + j * DECODE_K_PITCH + c * 16, ks + c * 8);
            cp_async16(Vs + j * 128 + c * 16, vs + c * 8);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    decode_append(ap, seq, g, tid);
    if (tid < 48) {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(ap.q + static_cast<int64_t>(seq) * D_MODEL + (g * 3 + tid / 16) * 64) +
                              tid % 16);
        qb[tid / 16][tid % 16] = make_uint2(__byte_perm(w.x, w.y, 0x6420), __byte_perm(w.x, w.y, 0x7531));
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // scores s_hj = SAT16(RS(q_h . k_j, shift_s)), thread j for key j
    int32_t lmax[3] = {INT32_MIN, INT32_MIN, INT32_MIN};
    if (tid < L) {
        const uint4* k4 = reinterpret_cast<const uint4*>(Ks + tid * DECODE_K_PITCH);
        int32_t d0[3] = {0, 0, 0}, d1[3] = {0, 0, 0}, d2[3] = {0, 0, 0};
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const uint4 t = k4[w];
            const uint32_t k0a = __byte_perm(t.x, t.y, 0x6420), k1a = __byte_perm(t.x, t.y, 0x7531);
            const uint32_t k0b = __byte_perm(t.z, t.w, 0x6420), k1b = __byte_perm(t.z, t.w, 0x7531);
#pragma unroll
            for (int h = 0; h < 3; ++h) {
                const uint2 qa = qb[h][2 * w], qc = qb[h][2 * w + 1];
                d0[h] = dp4a_uu(qa.x, k0a, d0[h]);
                d0[h] = dp4a_uu(qc.x, k0b, d0[h]);
                d1[h] = dp4a_su(qa.y, k0a, d1[h]);
                d1[h] = dp4a_su(qc.y, k0b, d1[h]);
                d1[h] = dp4a_us(qa.x, k1a, d1[h]);
                d1[h] = dp4a_us(qc.x, k1b, d1[h]);
                d2[h] = __dp4a(static_cast<int>(qa.y), static_cast<int>(k1a), d2[h]);
                d2[h] = __dp4a(static_cast<int>(qc.y), static_cast<int>(k1b), d2[h]);
            }
        }
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            const int64_t acc = static_cast<int64_t>(d2[h]) * 65536 + static_cast<int64_t>(d1[h]) * 256 + d0[h];
            const int32_t sj = static_cast<int32_t>(sat64(rs64(acc, ap.shift_s), 16));
            S[h * L + tid] = sj;
            lmax[h] = sj;
        }
    }
#pragma unroll
    for (int h = 0; h < 3; ++h) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lmax[h] = max(lmax[h], __shfl_xor_sync(0xffffffffu, lmax[h], o));
        if (lane == 0) red_max[h][warp] = lmax[h];
    }
    __syncthreads();
    // e_hj = E[rowmax_h - s_hj] (0 beyond DMAX), Z_h = sum_j e_hj; the table is read through L1
    int64_t lz[3] = {0, 0, 0};
    if (tid < L) {
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            int32_t rmax = red_max[h][0];
#pragma unroll
            for (int w = 1; w < DECODE_THREADS / 32; ++w) rmax = max(rmax, red_max[h][w]);
            const int32_t dd = rmax - S[h * L + tid];
            const int32_t ej = dd <= DMAX ? __ldg(ap.exp_tab + dd) : 0;
            S[h * L + tid] = ej;
            lz[h] = ej;
        }
    }
#pragma unroll
    for (int h = 0; h < 3; ++h) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lz[h] += __shfl_xor_sync(0xffffffffu, lz[h], o);
        if (lane == 0) red_z[h][warp] = lz[h];
    }
    __syncthreads();
    // P_hj = floor((e_hj 65536 + floor(Z_h/2)) / Z_h), exact (double estimate, integer remainder fix-up)
    if (tid < L) {
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            int64_t Z = 0;
#pragma unroll
            for (int w = 0; w < DECODE_THREADS / 32; ++w) Z += red_z[h][w];
            const int64_t n = static_cast<int64_t>(S[h * L + tid]) * 65536 + Z / 2;
            int64_t p = static_cast<int64_t>(static_cast<double>(n) * (1.0 / static_cast<double>(Z)));
            int64_t r = n - p * Z;
            if (r < 0) { --p; r += Z; }
            if (r < 0) { --p; r += Z; }
            if (r >= Z) { ++p; r -= Z; }
            if (r >= Z) { ++p; }
            S[h * L + tid] = static_cast<int32_t>(p);
        }
    }
    __syncthreads();
    // ctx_hd = SAT(RS(sum_j P_hj v_jd, shift_c), bits_c): thread (key quarter tid / 32, dims 2 lane,
    // 2 lane + 1) sums keys j = quarter (mod 4) for the three heads (P <= 65536 and |v| < 2^15, so each
    // product is one 32x32->64 multiply-add); the quarters add up in shared memory.
    const int kq = tid / 32;
    int64_t a0[3] = {0, 0, 0}, a1[3] = {0, 0, 0};
#pragma unroll 4
    for (int j = kq; j < L; j += 4) {
        const uint32_t vv = reinterpret_cast<const uint32_t*>(Vs + j * 128)[lane];
        const int32_t v0 = static_cast<int16_t>(vv & 0xFFFF), v1 = static_cast<int16_t>(vv >> 16);
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            const int32_t p = S[h * L + j];
            a0[h] += static_cast<int64_t>(p) * v0;
            a1[h] += static_cast<int64_t>(p) * v1;
        }
    }
    int64_t* part = reinterpret_cast<int64_t*>(Ks);  // [4 quarters][3 heads][32 lanes][2]: K is no longer read
#pragma unroll
    for (int h = 0; h < 3; ++h) {
        part[((kq * 3 + h) * 32 + lane) * 2] = a0[h];
        part[((kq * 3 + h) * 32 + lane) * 2 + 1] = a1[h];
    }
    __syncthreads();
    if (tid >= 96) return;
    const int h = tid / 32;
    int64_t c0 = 0, c1 = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        c0 += part[((q * 3 + h) * 32 + lane) * 2];
        c1 += part[((q * 3 + h) * 32 + lane) * 2 + 1];
    }
    c0 = sat64(rs64(c0, ap.shift_c), ap.bits_c);
    c1 = sat64(rs64(c1, ap.shift_c), ap.bits_c);
    const int col = (g * 3 + h) * 64 + 2 * lane;
    const int64_t pstride = blocked_plane_stride(ap.M, D_MODEL);
    const int64_t off = ap.offset ? (int64_t(1) << (8 * ap.P - 1)) : 0;
    for (int p = 0; p < ap.P; ++p) {
        const uint16_t pair =
            static_cast<uint16_t>(plane_byte(c0 + off, p)) | (static_cast<uint16_t>(plane_byte(c1 + off, p)) << 8);
        *reinterpret_cast<uint16_t*>(ap.ctx_planes + p * pstride + blocked_off(seq, col, D_MODEL)) = pair;
    }
}

// --------------------------------------------------------------------------- plane split
// int64 activations [M,K] (values within b = 8P bits) -> P byte planes [P][M][K].
__global__ void k_split_planes(const int64_t* __restrict__ a, int64_t count, int P, int64_t plane_stride,
                               uint8_t* __restrict__ planes, int* err) {
    const int64_t lo = -(int64_t(1) << (8 * P - 1)), hi = (int64_t(1) << (8 * P - 1)) - 1;
    bool bad = false;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t v = a[i];
        bad |= v < lo || v > hi;
        for (int p = 0; p < P; ++p) planes[p * plane_stride + i] = plane_byte(v, p);
    }
    if (bad && err) atomicCAS(err, 0, ERR_BAD_INPUT);
}

// int32 activations [M,K] (values within b = 8P bits; count a multiple of 16, 16-byte aligned) ->
// P byte planes [P][M][K]: 16 values per thread and step (four 16-byte loads, one 16-byte store per
// plane).  A value outside the signed b-bit range records ERR_BAD_INPUT.
// offset_binary: the planes are those of a + 2^(b-1) (all unsigned bytes; the top byte's sign bit
// flipped), as the feature-major GEMM (k_tgemm) reads them.
__global__ void k_split_i32(const int32_t* __restrict__ a, int64_t count, int P, int64_t plane_stride,
                            uint8_t* __restrict__ planes, int* err, int offset_binary) {
    const int32_t lo = P == 2 ? -32768 : INT32_MIN, hi = P == 2 ? 32767 : INT32_MAX;
    const uint32_t flip = offset_binary ? (P == 2 ? 0x8000u : 0x80000000u) : 0u;
    bool bad = false;
    const int64_t n16 = count / 16;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int32_t v[16];
        const int4* src = reinterpret_cast<const int4*>(a) + 4 * i;
#pragma unroll
        for (int q = 0; q < 4; ++q) *reinterpret_cast<int4*>(&v[4 * q]) = __ldg(src + q);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            bad |= v[j] < lo || v[j] > hi;
            v[j] = static_cast<int32_t>(static_cast<uint32_t>(v[j]) ^ flip);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            if (p >= P) break;
            const uint32_t sel = p | ((4 + p) << 4);
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t t01 = __byte_perm(static_cast<uint32_t>(v[4 * q]), static_cast<uint32_t>(v[4 * q + 1]), sel);
                const uint32_t t23 = __byte_perm(static_cast<uint32_t>(v[4 * q + 2]), static_cast<uint32_t>(v[4 * q + 3]), sel);
                w[q] = __byte_perm(t01, t23, 0x5410);
            }
            *reinterpret_cast<uint4*>(planes + p * plane_stride + 16 * i) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    if (bad && err) atomicCAS(err, 0, ERR_BAD_INPUT);
}

__global__ void k_i64_to_i32(const int64_t* __restrict__ a, int64_t n, int32_t* __restrict__ o) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        o[i] = static_cast<int32_t>(a[i]);
}

// --------------------------------------------------------------------------- digest
// splitmix64 finaliser forced odd: the logits digest weights (position t -> mix64(t), vocabulary
// id v -> mix64(2^32 + v)); the digest itself is accumulated in the logits GEMM epilogue.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return (z ^ (z >> 31)) | 1ull;
}

}  // namespace eii
