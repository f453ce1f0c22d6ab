// Integer causal attention on tcgen05 kind::i8 for sequences of T <= 128 tokens.
//
// One CTA per (sequence, KV group): the group's K and V and its three query heads are split into
// byte planes in shared memory (128-byte swizzled K-major tiles, the layout TMA would write), and
// for each head:
//   S  = Q K^T  as three int32 TMEM accumulators over the 64-dim head:
//        D0 = q0.k0, D1 = q1.k0 + q0.k1, D2 = q1.k1      (q0,k0 u8 low bytes, q1,k1 s8 top bytes)
//        S = 65536 D2 + 256 D1 + D0 exactly (|partial sums| <= 64 * 255 * 255 < 2^31).
//   scores: each warp reads its TMEM lane quadrant (32 query rows) and 32-key block and writes
//        s = SAT16(RS(S, shift_s)) as int16 into a shared score tile (rows padded to 288 bytes);
//   softmax per query row, four threads per row (exactly as python/intref.py:239-246):
//        rowmax over j <= i, e = E[rowmax - s] (0 beyond DMAX), Z = sum e, both reduced with two
//        shuffles inside the row's thread quad, P = floor((e 65536 + floor(Z/2)) / Z) in [0, 65536]
//        (an fp32 estimate of the quotient corrected with the integer remainder).  A row's keys
//        are split into groups of four taken round-robin by its four threads, and warp w holds
//        rows 8w .. 8w + 7, so every SM sub-partition (warps w = s mod 4) gets one warp of each
//        32-row query block and the causal work is balanced without block-wide reductions.
//        P = 65536 * [P == 65536] + 256 p1 + p0; the two low bytes are written as u8 planes and
//        the (at most one) P == 65536 key of a row is added back in the epilogue.
//   ctx = P V   as three TMEM accumulators over the T keys (V transposed, K-major):
//        C0 = p0.v0, C1 = p1.v0 + p0.v1, C2 = p1.v1 (|partial sums| <= 128 * 255 * 255 < 2^31)
//        ctx = SAT(RS(65536 C2 + 256 C1 + C0 + 65536 v[j*], shift_c), bits_c) -> byte planes.
// (python/intref.py:227-254, c/intref.c:160-187.)
#pragma once
#include <cstdint>

#include "eii_gemm.cuh"
#include "eii_int.cuh"
#include "eii_kernels.cuh"
#include "eii_ptx.cuh"

namespace eii {

constexpr int ATTN_TC_THREADS = 512;   // 16 warps: warp w owns TMEM lane quadrant w % 4 and key/dim block w / 4
constexpr int ATTN_TC_TILE = 128 * 128;  // one 128 x 128-byte swizzled tile
// Score tile row pitch: 144 int16 (288 bytes = 72 words, 8 mod 32), so the four rows a half-warp
// reads with 8-byte loads start 8 banks apart.
constexpr int ATTN_SS_PITCH = 144;
// e values of the softmax, private to each thread: [8 key groups][512 threads] int4 (a warp's 16-byte
// accesses are 512 contiguous bytes, so conflict-free)
constexpr int ATTN_ET_BYTES = 8 * 512 * 16;
// smem: Q (3 tiles) | K (1) | V^T planes (2 x 64 rows x 128 B = 1 tile) | P planes (2 tiles) |
//       e values | scores [128][144] int16 | E | j* [128] int32 | barrier, TMEM slot, abort
constexpr int ATTN_TC_SMEM = 7 * ATTN_TC_TILE + 1024 + ATTN_ET_BYTES + 128 * ATTN_SS_PITCH * 2 + (DMAX + 1 + 3) * 4 + 128 * 4 + 64;

// Byte offset of byte b of row r inside a 128-byte-row tile with the 128-byte swizzle.
__device__ __forceinline__ int sw128(int r, int b) { return r * 128 + ((((b >> 4) ^ r) & 7) << 4) + (b & 15); }

// floor((e * 65536 + floor(Z/2)) / Z) for 0 <= e <= 2^30, 2^30 <= Z < 2^40.
// n / Z = e (65536 / Z) + floor(Z/2) / Z, the second term in (0.5 - 1/(2Z), 0.5]; in fp32 the
// estimate e * (65536 / Z) + 0.5 has absolute error < 0.05 (quotient < 2^17), so its floor is within
// one of the true quotient, which the integer remainder r = n - q Z then fixes exactly.
__device__ __forceinline__ int32_t prob_q16_f32(int32_t e, int64_t Z, int64_t halfZ, float scale) {
    const int64_t n = static_cast<int64_t>(e) * 65536 + halfZ;
    int32_t q = __float2int_rd(__fmaf_rn(static_cast<float>(e), scale, 0.5f));
    const int64_t r = n - static_cast<int64_t>(q) * Z;
    if (r < 0) --q;
    else if (r >= Z) ++q;
    return q;
}

__global__ void __launch_bounds__(ATTN_TC_THREADS, 1) k_attention_tc(AttnParams ap, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm;                       // 3 tiles: row i = [q0 bytes 0..63 | q1 bytes 64..127]
    uint8_t* Ks = sm + 3 * ATTN_TC_TILE;    // row j = [k0 | k1]
    uint8_t* VT = sm + 4 * ATTN_TC_TILE;    // plane p at VT + p * 8192: row d, byte j
    uint8_t* Ps = sm + 5 * ATTN_TC_TILE;    // plane p at Ps + p * ATTN_TC_TILE: row i, byte j
    int4* Et = reinterpret_cast<int4*>(sm + 7 * ATTN_TC_TILE);        // [8][512]: e of key group m of thread tid
    int16_t* Ss = reinterpret_cast<int16_t*>(sm + 7 * ATTN_TC_TILE + ATTN_ET_BYTES);  // [128][ATTN_SS_PITCH]
    int32_t* E = reinterpret_cast<int32_t*>(Ss + 128 * ATTN_SS_PITCH);
    int32_t* jstar_s = E + DMAX + 1 + 3;                                  // [128]
    uint64_t* bar = reinterpret_cast<uint64_t*>(jstar_s + 128);  // [0]: S = Q K^T, [1]: P V
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int T = ap.T;
    const int items = (ap.M / T) * N_KV;  // (sequence, KV group) pairs; CTA b takes b, b + grid, ...
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int quad = warp & 3, kb = warp >> 2;  // rows 32 quad .. +31, key block / dim block kb
    const int i = quad * 32 + lane;             // tile row of this thread (TMEM lane)

    if (warp == 0) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (tid == 0) { mbar_init(bar, 1); mbar_init(bar + 1, 1); *abort = 0; fence_mbar_init(); }
    for (int u = tid; u <= DMAX; u += ATTN_TC_THREADS) E[u] = ap.exp_tab[u];  // model table
    if (tid == 0) E[DMAX + 1] = 0;  // the softmax clamps distances past DMAX to this entry
    griddep_wait();  // q, k, v are the previous kernel's output
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    uint32_t phase_s = 0, phase_p = 0;
    const uint32_t sK = smem_u32(Ks), sV0 = smem_u32(VT), sV1 = smem_u32(VT + 8192);
    const uint32_t sP0 = smem_u32(Ps), sP1 = smem_u32(Ps + ATTN_TC_TILE);
    // key block kb holds keys 32 kb .. 32 kb + 31; it has unmasked keys for this quadrant iff kb <= quad
    // Packed query tiles: the three heads' 32-row query blocks (head h, block b: positions 32 b ..
    // 32 b + 31) fill the twelve (tile, lane quadrant) slots s = 4 t + q in order of decreasing b:
    // s -> head s % 3, block 3 - s / 3.  A quadrant holding block b has b + 1 live key blocks under
    // the causal mask, and each tile waits for its slowest quadrant, so the three tiles cost 4, 3
    // and 2 key blocks instead of 4 each with one head per tile.
    bool active = false;
    const bool fast = !ap.generic && ap.shift_s >= 8 && ap.shift_s <= 31;  // 32-bit score path (see the score pass)
    const int64_t srnd = fast ? (int64_t(1) << (ap.shift_s - 1)) : 0;
    // S of packed tile t covers its live key blocks only: nt = 128, 96, 64 keys for t = 0, 1, 2, with
    // the three accumulators at TMEM columns 0, nt and 2 nt (at most 288 columns after tile 0).  P V
    // goes to columns 320 .. 511, so the next tile's S can be computed while this tile's softmax,
    // P V and epilogue run: it is issued as soon as this tile's scores have left TMEM.
    constexpr uint32_t PV_COL = 320;
    auto issue_s = [&](int t) {
        const int nt = 128 - 32 * t;
        const uint32_t sQ = smem_u32(Qs + t * ATTN_TC_TILE);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            const uint32_t qlo = sQ + ks * 32, qhi = sQ + 64 + ks * 32, klo = sK + ks * 32, khi = sK + 64 + ks * 32;
            const uint32_t acc = ks > 0 ? 1u : 0u;
            mma_i8(tmem + 0, smem_desc_sw128(qlo), smem_desc_sw128(klo), idesc_i8(false, false, nt), acc);
            mma_i8(tmem + nt, smem_desc_sw128(qhi), smem_desc_sw128(klo), idesc_i8(true, false, nt), acc);
            mma_i8(tmem + nt, smem_desc_sw128(qlo), smem_desc_sw128(khi), idesc_i8(false, true, nt), 1u);
            mma_i8(tmem + 2 * nt, smem_desc_sw128(qhi), smem_desc_sw128(khi), idesc_i8(true, true, nt), acc);
        }
        tc_commit(bar);
    };

    // Persistent over (sequence, KV group) items: the TMEM allocation, barriers and exp table above are
    // set up once per CTA.  Between items every MMA has completed (the last P V was waited for) and the
    // end-of-tile barrier has passed, so the staging below may overwrite Q, K, V^T and the P planes.
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const int seq = item / N_KV, g = item % N_KV;
        const int64_t row0 = static_cast<int64_t>(seq) * T;

        // ---- stage K, Q (3 heads) and V^T as byte planes; rows/keys >= T are zero.  Every global load of
        // the staging is issued before the first shared-memory store, so their latencies overlap.
        constexpr int QK_ITERS = 128 * 4 * 4 / ATTN_TC_THREADS;  // 32-byte pieces per thread
        int4 qka[QK_ITERS], qkb[QK_ITERS], va = make_int4(0, 0, 0, 0), vb = make_int4(0, 0, 0, 0);
#pragma unroll
        for (int it = 0; it < QK_ITERS; ++it) {
            const int idx = tid + it * ATTN_TC_THREADS;
            const int r = idx / 16, c = (idx / 4) % 4, which = idx % 4;  // which: 0..2 = q head, 3 = k
            qka[it] = qkb[it] = make_int4(0, 0, 0, 0);
            if (r < T) {
                const int16_t* src = which < 3 ? ap.q + (row0 + r) * D_MODEL + (g * 3 + which) * 64 + c * 16
                                               : ap.k + (row0 + r) * 192 + g * 64 + c * 16;
                qka[it] = reinterpret_cast<const int4*>(src)[0];
                qkb[it] = reinterpret_cast<const int4*>(src)[1];
            }
        }
        const int vj = tid & 127, vdq = tid >> 7;  // V^T: thread (key, dim quarter)
        if (vj < T) {
            const int4* src = reinterpret_cast<const int4*>(ap.v + (row0 + vj) * 192 + g * 64 + vdq * 16);
            va = src[0];
            vb = src[1];
        }
#pragma unroll
        for (int it = 0; it < QK_ITERS; ++it) {
            const int idx = tid + it * ATTN_TC_THREADS;
            const int r = idx / 16, c = (idx / 4) % 4, which = idx % 4;
            // low bytes of the 16 values (bytes 0 and 2 of each word) and high bytes (1 and 3)
            const uint32_t w[8] = {static_cast<uint32_t>(qka[it].x), static_cast<uint32_t>(qka[it].y),
                                   static_cast<uint32_t>(qka[it].z), static_cast<uint32_t>(qka[it].w),
                                   static_cast<uint32_t>(qkb[it].x), static_cast<uint32_t>(qkb[it].y),
                                   static_cast<uint32_t>(qkb[it].z), static_cast<uint32_t>(qkb[it].w)};
            const uint4 lo = make_uint4(__byte_perm(w[0], w[1], 0x6420), __byte_perm(w[2], w[3], 0x6420),
                                        __byte_perm(w[4], w[5], 0x6420), __byte_perm(w[6], w[7], 0x6420));
            const uint4 hi = make_uint4(__byte_perm(w[0], w[1], 0x7531), __byte_perm(w[2], w[3], 0x7531),
                                        __byte_perm(w[4], w[5], 0x7531), __byte_perm(w[6], w[7], 0x7531));
            // q rows go to their packed tile slot (see the tile loop); k rows to the K tile
            uint8_t* tile = Ks;
            int tr = r;
            if (which < 3) {
                const int sl = 3 * (3 - r / 32) + which;
                tile = Qs + (sl / 4) * ATTN_TC_TILE;
                tr = (sl % 4) * 32 + r % 32;
            }
            *reinterpret_cast<uint4*>(tile + sw128(tr, c * 16)) = lo;
            *reinterpret_cast<uint4*>(tile + sw128(tr, 64 + c * 16)) = hi;
        }
        {   // V^T: key vj's 16 values go into column vj of both planes
            const int16_t* v = reinterpret_cast<const int16_t*>(&va);
            const int16_t* v2 = reinterpret_cast<const int16_t*>(&vb);
#pragma unroll
            for (int d = 0; d < 16; ++d) {
                const int16_t x = d < 8 ? v[d] : v2[d - 8];
                VT[sw128(vdq * 16 + d, vj)] = static_cast<uint8_t>(x & 0xFF);
                VT[8192 + sw128(vdq * 16 + d, vj)] = static_cast<uint8_t>((x >> 8) & 0xFF);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) issue_s(0);
        {   // the CTA's next item: its q (3 heads), k and v rows into L2 while this item runs, so that its
            // staging reads hit L2 instead of every CTA reading DRAM at once at each item start
            const int nitem = item + gridDim.x;
            if (nitem < items) {
                const int64_t nrow0 = static_cast<int64_t>(nitem / N_KV) * T;
                const int ng = nitem % N_KV;
                for (int u = tid; u < T * 5; u += ATTN_TC_THREADS) {  // five 128-byte lines per row
                    const int r = u / 5, w = u % 5;
                    const int16_t* a = w < 3 ? ap.q + (nrow0 + r) * D_MODEL + ng * 192 + w * 64
                                             : (w == 3 ? ap.k : ap.v) + (nrow0 + r) * 192 + ng * 64;
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
                }
            }
        }

        for (int h = 0; h < 3; ++h) {  // h = packed tile
            const int slot = 4 * h + quad, hq = slot % 3, bq = 3 - slot / 3;
            const int pos = 32 * bq + lane;  // sequence position of this thread's query row
            const int nt = 128 - 32 * h;
            active = kb <= bq;
            if (tid < 128) jstar_s[tid] = -1;
            // ---- S = Q_h K^T (M = 128 queries, N = nt keys, K = 64 dims per plane pair), issued earlier
            if (!__syncthreads_and(mbar_wait(bar, phase_s, abort, err, ERR_TIMEOUT_ATTN))) { ok = false; break; }
            phase_s ^= 1;
            tc_fence_after();

            // ---- scores of my 32-key block for my quadrant's rows -> the shared score tile
            if (active) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int col = kb * 32 + c * 16;
                    uint32_t d0[16], d1[16], d2[16];
                    tmem_ld16(tq + col, d0);
                    tmem_ld16(tq + nt + col, d1);
                    tmem_ld16(tq + 2 * nt + col, d2);
                    tmem_wait_ld();
                    tmem_launder(d0); tmem_launder(d1); tmem_launder(d2);
                    uint32_t sp[8];  // s as int16 pairs
#pragma unroll
                    for (int q = 0; q < 16; q += 2) {
                        int32_t s2[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int32_t a0 = static_cast<int32_t>(d0[q + u]), a1 = static_cast<int32_t>(d1[q + u]),
                                          a2 = static_cast<int32_t>(d2[q + u]);
                            if (fast) {
                                // S + 2^(sh-1) = 2^8 (2^8 a2 + a1 + ((a0 + 2^(sh-1)) >> 8)) + ((a0 + 2^(sh-1)) & 255),
                                // so RS(S, sh) = (2^8 a2 + a1 + ((a0 + 2^(sh-1)) >> 8)) >> (sh - 8): every term
                                // fits int32 (|a0| < 2^22, |a1| < 2^22, |a2| <= 2^20, 2^(sh-1) <= 2^30); SAT16 is
                                // applied by the saturating pack below
                                const int32_t t = a2 * 256 + a1 + ((a0 + static_cast<int32_t>(srnd)) >> 8);
                                s2[u] = t >> (ap.shift_s - 8);
                            } else {
                                const int64_t S = static_cast<int64_t>(a2) * 65536 + static_cast<int64_t>(a1) * 256 +
                                                  static_cast<int64_t>(a0);
                                s2[u] = static_cast<int32_t>(sat64(rs64(S, ap.shift_s), 16));
                            }
                        }
                        sp[q / 2] = pack_sat_s16(s2[1], s2[0]);  // key q in the low half, q + 1 in the high
                    }
                    uint4* dst = reinterpret_cast<uint4*>(Ss + i * ATTN_SS_PITCH + col);
                    dst[0] = make_uint4(sp[0], sp[1], sp[2], sp[3]);
                    dst[1] = make_uint4(sp[4], sp[5], sp[6], sp[7]);
                }
            }
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0 && h < 2) issue_s(h + 1);  // S columns are free again

            // ---- softmax of tile row r by threads 4 r .. 4 r + 3: thread jq takes key groups g = jq + 4 m
            // (keys 4 g .. 4 g + 3), m = 0 .. 7; rows past T or keys past the row's position get P = 0
            {
                const int r = tid >> 2, jq = tid & 3;
                const int rslot = 4 * h + (r >> 5);
                const int rpos = 32 * (3 - rslot / 3) + (r & 31);
                const int nk = rpos < T ? rpos + 1 : 0;  // live keys of this row
                const int16_t* srow = Ss + r * ATTN_SS_PITCH;
                // a thread's key groups ascend with m, so the live ones are m < nm (branches, not predicates:
                // the unrolled division would otherwise run for every key of the row's 128)
                const int nm = nk > 4 * jq ? (nk - 4 * jq + 15) / 16 : 0;
                // scores stay packed as int16 pairs: the row max by 16-bit SIMD max, the keys of the row's
                // last group past its position (live < 4) replaced by -32768, which cannot raise it
                uint2 sv[8];
                uint32_t mx2 = 0x80008000u;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    if (m >= nm) break;
                    const int k0 = 4 * (jq + 4 * m);
                    sv[m] = *reinterpret_cast<const uint2*>(srow + k0);
                    uint2 w = sv[m];
                    const int live = nk - k0;  // >= 1
                    if (live < 4) {
                        if (live < 2) w.x = (w.x & 0xFFFFu) | 0x80000000u;
                        w.y = live < 3 ? 0x80008000u : ((w.y & 0xFFFFu) | 0x80000000u);
                    }
                    mx2 = __vmaxs2(mx2, __vmaxs2(w.x, w.y));
                }
                int32_t mx = max(static_cast<int32_t>(static_cast<int16_t>(mx2 & 0xFFFFu)),
                                 static_cast<int32_t>(static_cast<int16_t>(mx2 >> 16)));
                mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                // e of each live key (0 past the row's position or beyond DMAX, which makes P = 0 below),
                // kept in this thread's shared-memory slots for the division pass
                // distances mx - s in [0, 65535] by 16-bit SIMD subtraction (exact modulo 2^16), clamped to
                // DMAX + 1 (E there is 0); pairs of e <= 2^30 add up exactly in 32 bits
                int64_t z = 0;
                const uint32_t mxx = (static_cast<uint32_t>(mx) & 0xFFFFu) * 0x10001u;
                constexpr uint32_t cap = static_cast<uint32_t>(DMAX + 1) * 0x10001u;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    if (m >= nm) break;
                    const int k0 = 4 * (jq + 4 * m);
                    const uint32_t d01 = __vminu2(__vsub2(mxx, sv[m].x), cap);
                    const uint32_t d23 = __vminu2(__vsub2(mxx, sv[m].y), cap);
                    int32_t ev[4] = {E[d01 & 0xFFFFu], E[d01 >> 16], E[d23 & 0xFFFFu], E[d23 >> 16]};
                    const int live = nk - k0;  // keys past the row's position get e = 0
                    if (live < 4) {
                        if (live < 2) ev[1] = 0;
                        if (live < 3) ev[2] = 0;
                        ev[3] = 0;
                    }
                    z += static_cast<int64_t>(static_cast<uint32_t>(ev[0]) + static_cast<uint32_t>(ev[1])) +
                         static_cast<int64_t>(static_cast<uint32_t>(ev[2]) + static_cast<uint32_t>(ev[3]));
                    Et[m * ATTN_TC_THREADS + tid] = make_int4(ev[0], ev[1], ev[2], ev[3]);
                }
                z += __shfl_xor_sync(0xffffffffu, z, 1);
                z += __shfl_xor_sync(0xffffffffu, z, 2);
                const int64_t halfZ = z / 2;
                const float scale = z > 0 ? static_cast<float>(65536.0 / static_cast<double>(z)) : 0.f;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const int k0 = 4 * (jq + 4 * m);
                    uint32_t b0 = 0, b1 = 0;
                    if (m < nm) {
                        const int4 e4 = Et[m * ATTN_TC_THREADS + tid];
                        const int32_t ev[4] = {e4.x, e4.y, e4.z, e4.w};
                        uint32_t p[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            p[u] = static_cast<uint32_t>(prob_q16_f32(ev[u], z, halfZ, scale));  // 0 for e = 0
                            if (p[u] == 65536u) jstar_s[r] = k0 + u;
                        }
                        // plane 0: byte 0 of each P, plane 1: byte 1 (the P = 65536 key is added back via j*)
                        b0 = __byte_perm(__byte_perm(p[0], p[1], 0x0040), __byte_perm(p[2], p[3], 0x0040), 0x5410);
                        b1 = __byte_perm(__byte_perm(p[0], p[1], 0x0051), __byte_perm(p[2], p[3], 0x0051), 0x5410);
                    }
                    *reinterpret_cast<uint32_t*>(Ps + sw128(r, k0)) = b0;
                    *reinterpret_cast<uint32_t*>(Ps + ATTN_TC_TILE + sw128(r, k0)) = b1;
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();

            // ---- ctx = P V (M = 128 queries, N = 64 dims, K = 128 keys) into columns PV_COL ..
            if (tid == 0) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint32_t acc = ks > 0 ? 1u : 0u;
                    const uint64_t p0 = smem_desc_sw128(sP0 + ks * 32), p1 = smem_desc_sw128(sP1 + ks * 32);
                    const uint64_t v0 = smem_desc_sw128(sV0 + ks * 32), v1 = smem_desc_sw128(sV1 + ks * 32);
                    mma_i8(tmem + PV_COL, p0, v0, idesc_i8(false, false, 64), acc);
                    mma_i8(tmem + PV_COL + 64, p1, v0, idesc_i8(false, false, 64), acc);
                    mma_i8(tmem + PV_COL + 64, p0, v1, idesc_i8(false, true, 64), 1u);
                    mma_i8(tmem + PV_COL + 128, p1, v1, idesc_i8(false, true, 64), acc);
                }
                tc_commit(bar + 1);
            }
            if (!__syncthreads_and(mbar_wait(bar + 1, phase_p, abort, err, ERR_TIMEOUT_ATTN))) { ok = false; break; }
            phase_p ^= 1;
            tc_fence_after();
            {   // epilogue: rows of my quadrant, dims 16 kb .. 16 kb + 15
                const int hh = g * 3 + hq;
                const int col = kb * 16;
                uint32_t c0[16], c1[16], c2[16];
                tmem_ld16(tq + PV_COL + col, c0);
                tmem_ld16(tq + PV_COL + 64 + col, c1);
                tmem_ld16(tq + PV_COL + 128 + col, c2);
                tmem_wait_ld();
                tmem_launder(c0); tmem_launder(c1); tmem_launder(c2);
                if (pos < T) {
                    const int js = jstar_s[i];
                    int32_t out[16];
                    if (!ap.generic && ap.shift_c >= 8 && ap.shift_c <= 31) {
                        // ctx + 2^(sh-1) = 2^8 (2^8 C2 + C1 + 2^8 v_j* + ((C0 + 2^(sh-1)) >> 8)) + ((C0 + 2^(sh-1)) & 255),
                        // so RS(ctx, sh) = (...) >> (sh - 8), every term in int32: |2^8 C2| <= 2^8 * 128 * 255 * 128
                        // < 2^30, |C1| < 2^24, |2^8 v_j*| <= 2^23, |C0| < 2^23, 2^(sh-1) <= 2^30
                        const int32_t crnd = 1 << (ap.shift_c - 1);
                        const int32_t lim = ap.bits_c < 32 ? (1 << (ap.bits_c - 1)) : 0;
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const int d = col + q;
                            int32_t t = static_cast<int32_t>(c2[q]) * 256 + static_cast<int32_t>(c1[q]) +
                                        ((static_cast<int32_t>(c0[q]) + crnd) >> 8);
                            if (js >= 0) {
                                const int32_t vj = static_cast<int32_t>(VT[sw128(d, js)]) |
                                                   (static_cast<int32_t>(static_cast<int8_t>(VT[8192 + sw128(d, js)])) * 256);
                                t += vj * 256;
                            }
                            int32_t r = t >> (ap.shift_c - 8);
                            if (lim && ap.P != 2) r = min(max(r, -lim), lim - 1);  // two planes: SAT16 by the pack below
                            out[q] = r;
                        }
                    } else {
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const int d = col + q;
                            int64_t a = static_cast<int64_t>(static_cast<int32_t>(c2[q])) * 65536 +
                                        (static_cast<int64_t>(static_cast<int32_t>(c1[q])) * 256 +
                                         static_cast<int64_t>(static_cast<int32_t>(c0[q])));
                            if (js >= 0) {
                                const int32_t vj = static_cast<int32_t>(VT[sw128(d, js)]) |
                                                   (static_cast<int32_t>(static_cast<int8_t>(VT[8192 + sw128(d, js)])) << 8);
                                a += static_cast<int64_t>(vj) * 65536;
                            }
                            out[q] = static_cast<int32_t>(sat64(rs64(a, ap.shift_c), ap.bits_c));
                        }
                    }
                    // row-blocked planes: this warp's 32 rows x 16 dims are 512 contiguous bytes per plane
                    const int64_t pstride = blocked_plane_stride(ap.M, D_MODEL);
                    uint4* dst = reinterpret_cast<uint4*>(ap.ctx_planes + blocked_off(row0 + pos, hh * 64 + col, D_MODEL));
                    if (ap.P == 2) {
                        // int16 pairs by saturating packs (SAT16), the offset-binary flip per pair, then the
                        // low and high bytes of four values per word
                        uint32_t wp[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) wp[k] = pack_sat_s16(out[2 * k + 1], out[2 * k]) ^ (ap.offset ? 0x80008000u : 0u);
                        uint32_t w0[4], w1[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            w0[k] = __byte_perm(wp[2 * k], wp[2 * k + 1], 0x6420);
                            w1[k] = __byte_perm(wp[2 * k], wp[2 * k + 1], 0x7531);
                        }
                        dst[0] = make_uint4(w0[0], w0[1], w0[2], w0[3]);
                        dst[pstride / 16] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
                    } else {
                        if (ap.offset) {  // offset binary: the bytes of ctx + 2^31
#pragma unroll
                            for (int q = 0; q < 16; ++q) out[q] = static_cast<int32_t>(static_cast<uint32_t>(out[q]) ^ 0x80000000u);
                        }
                        uint32_t w[4][4];
                        pack_planes<16, true>(out, w[0], w[1], w[2], w[3]);
                        dst[0] = make_uint4(w[0][0], w[0][1], w[0][2], w[0][3]);
                        dst[pstride / 16] = make_uint4(w[1][0], w[1][1], w[1][2], w[1][3]);
                        dst[2 * pstride / 16] = make_uint4(w[2][0], w[2][1], w[2][2], w[2][3]);
                        dst[3 * pstride / 16] = make_uint4(w[3][0], w[3][1], w[3][2], w[3][3]);
                    }
                }
            }
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
        }
    }  // item
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(*tmem_slot, 512);
}

// ---------------------------------------------------------------------------------------------
// Integer causal attention on tcgen05 kind::i8 for 128 < T <= 512 (python/intref.py:227-254; T is
// bounded by the 512-row RoPE table, :151).  One work item = (sequence, query head, 128-row query
// tile qt); persistent CTAs take the items in order of decreasing qt (the tiles with the most keys
// first).  Per item:
//   1. S phase, for each 128-key tile kt <= qt: the K tile of the head's KV group is staged as byte
//      planes, S = Q K^T runs as the three int32 TMEM accumulators of the short kernel (D0, D1, D2
//      at columns 0, 128, 256), and the scores s = SAT16(RS(S, shift_s)) go to a [128][T] int16
//      score buffer in shared memory (only the 32-key blocks that hold a key j <= i of some row of
//      the warp's lane quadrant).  The next K tile's global loads are issued before the MMA wait.
//   2. Row statistics over every live key j <= i, four threads per row: rowmax, then
//      Z = sum E[rowmax - s] (0 beyond DMAX); Z >= E[0] = 2^30 and Z <= 512 * 2^30 < 2^40.
//   3. PV phase, for each kt <= qt: P = floor((e 65536 + floor(Z/2)) / Z) of the tile's keys as two
//      u8 planes (the P = 65536 key of a row is kept aside), V^T of the tile's keys as two planes,
//      and ctx += P V as three TMEM accumulators at columns 0, 64, 128 (the scores have left TMEM).
//      The next tile's P values and V loads are computed while the current tile's MMAs run.
//   4. Epilogue as in the short kernel; the v row of a P = 65536 key is read from global memory.
// Accumulator bounds over up to 512 keys: D0..D2 as in the short kernel (64 dims);
// C0 <= 512 * 255 * 255 < 2^26, |C1| <= 2 * 512 * 255 * 255 < 2^27, and since
// sum_j p1_j <= sum_j P_j / 256 <= (65536 + 512) / 256, |C2| <= 258 * 128 < 2^16: the 32-bit
// context path below stays exact (every term below 2^31).
constexpr int ATTNL_SS_PITCH = 528;  // int16 per score row: 1056 bytes = 264 words (8 mod 32, as the short kernel)
constexpr int ATTNL_OFF_Q = 0, ATTNL_OFF_K = ATTN_TC_TILE, ATTNL_OFF_VT = 2 * ATTN_TC_TILE,
              ATTNL_OFF_P = 3 * ATTN_TC_TILE, ATTNL_OFF_S = 5 * ATTN_TC_TILE,
              ATTNL_OFF_E = ATTNL_OFF_S + 128 * ATTNL_SS_PITCH * 2;
constexpr int ATTNL_SMEM = ATTNL_OFF_E + (DMAX + 1 + 3) * 4 + 128 * 4 + 64 + 1024;
static_assert(ATTNL_SMEM <= 227 * 1024, "long attention shared memory");

// Byte planes of 16 int16 values (two 16-byte loads) into row r, bytes 16c.. (low) and 64 + 16c.. (high)
// of a 128-byte-row swizzled tile.
__device__ __forceinline__ void stage_planes16(uint8_t* tile, int r, int c, const int4& a, const int4& b) {
    const uint32_t w[8] = {static_cast<uint32_t>(a.x), static_cast<uint32_t>(a.y), static_cast<uint32_t>(a.z),
                           static_cast<uint32_t>(a.w), static_cast<uint32_t>(b.x), static_cast<uint32_t>(b.y),
                           static_cast<uint32_t>(b.z), static_cast<uint32_t>(b.w)};
    const uint4 lo = make_uint4(__byte_perm(w[0], w[1], 0x6420), __byte_perm(w[2], w[3], 0x6420),
                                __byte_perm(w[4], w[5], 0x6420), __byte_perm(w[6], w[7], 0x6420));
    const uint4 hi = make_uint4(__byte_perm(w[0], w[1], 0x7531), __byte_perm(w[2], w[3], 0x7531),
                                __byte_perm(w[4], w[5], 0x7531), __byte_perm(w[6], w[7], 0x7531));
    *reinterpret_cast<uint4*>(tile + sw128(r, c * 16)) = lo;
    *reinterpret_cast<uint4*>(tile + sw128(r, 64 + c * 16)) = hi;
}

__global__ void __launch_bounds__(ATTN_TC_THREADS, 1) k_attention_tc_long(AttnParams ap, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm + ATTNL_OFF_Q;    // row i = [q0 bytes | q1 bytes] of query 128 qt + i
    uint8_t* Ks = sm + ATTNL_OFF_K;    // row j = [k0 | k1] of key 128 kt + j
    uint8_t* VT = sm + ATTNL_OFF_VT;   // plane p at VT + p * 8192: row d, byte j (key 128 kt + j)
    uint8_t* Ps = sm + ATTNL_OFF_P;    // plane p at Ps + p * ATTN_TC_TILE: row i, byte j
    int16_t* Ss = reinterpret_cast<int16_t*>(sm + ATTNL_OFF_S);  // [128][ATTNL_SS_PITCH]: s of row i, key j
    int32_t* E = reinterpret_cast<int32_t*>(sm + ATTNL_OFF_E);
    int32_t* jstar_s = E + DMAX + 1 + 3;  // [128]
    uint64_t* bar = reinterpret_cast<uint64_t*>(jstar_s + 128);  // [0]: S = Q K^T, [1]: P V
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int T = ap.T;
    const int nqt = (T + 127) / 128;
    const int per_qt = (ap.M / T) * N_HEADS;  // (sequence, head) pairs per query-tile index
    const int items = per_qt * nqt;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int quad = warp & 3, kb = warp >> 2;  // TMEM lane quadrant; key block (S) / dim block (ctx)
    const int i = quad * 32 + lane;             // tile row of this thread (TMEM lane)

    if (warp == 0) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (tid == 0) { mbar_init(bar, 1); mbar_init(bar + 1, 1); *abort = 0; fence_mbar_init(); }
    for (int u = tid; u <= DMAX; u += ATTN_TC_THREADS) E[u] = ap.exp_tab[u];
    griddep_wait();  // q, k, v are the previous kernel's output
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    uint32_t phase_s = 0, phase_p = 0;
    const uint32_t sQ = smem_u32(Qs), sK = smem_u32(Ks), sV0 = smem_u32(VT), sV1 = smem_u32(VT + 8192);
    const uint32_t sP0 = smem_u32(Ps), sP1 = smem_u32(Ps + ATTN_TC_TILE);
    const bool fast = !ap.generic && ap.shift_s >= 8 && ap.shift_s <= 31;
    const int32_t srnd = fast ? (1 << (ap.shift_s - 1)) : 0;
    // staging assignment: thread -> (row or key r = tid / 4, 16-value piece c = tid % 4)
    const int sr = tid >> 2, sc = tid & 3;
    // softmax assignment: row r = tid / 4, key groups G = jq + 4 m (keys 4 G .. 4 G + 3)
    const int r = tid >> 2, jq = tid & 3;
    // V^T assignment: key vj of the tile, dims 16 vdq .. 16 vdq + 15
    const int vj = tid & 127, vdq = tid >> 7;

    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const int qt = nqt - 1 - item / per_qt;
        const int rem = item % per_qt;
        const int seq = rem / N_HEADS, hh = rem % N_HEADS, g = hh / 3;
        const int64_t row0 = static_cast<int64_t>(seq) * T;
        const int q0 = 128 * qt;
        if (tid < 128) jstar_s[tid] = -1;

        // ---- stage Q (this head, rows q0..) and K tile 0; rows past T are zero
        {
            int4 qa = make_int4(0, 0, 0, 0), qb = qa, ka = qa, kb2 = qa;
            if (q0 + sr < T) {
                const int4* src = reinterpret_cast<const int4*>(ap.q + (row0 + q0 + sr) * D_MODEL + hh * 64 + sc * 16);
                qa = src[0];
                qb = src[1];
            }
            if (sr < T) {
                const int4* src = reinterpret_cast<const int4*>(ap.k + (row0 + sr) * 192 + g * 64 + sc * 16);
                ka = src[0];
                kb2 = src[1];
            }
            stage_planes16(Qs, sr, sc, qa, qb);
            stage_planes16(Ks, sr, sc, ka, kb2);
        }

        // ---- S phase: scores of every key tile kt <= qt into Ss
        for (int kt = 0; kt <= qt; ++kt) {
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    const uint32_t qlo = sQ + ks * 32, qhi = sQ + 64 + ks * 32, klo = sK + ks * 32, khi = sK + 64 + ks * 32;
                    const uint32_t acc = ks > 0 ? 1u : 0u;
                    mma_i8(tmem + 0, smem_desc_sw128(qlo), smem_desc_sw128(klo), idesc_i8(false, false, 128), acc);
                    mma_i8(tmem + 128, smem_desc_sw128(qhi), smem_desc_sw128(klo), idesc_i8(true, false, 128), acc);
                    mma_i8(tmem + 128, smem_desc_sw128(qlo), smem_desc_sw128(khi), idesc_i8(false, true, 128), 1u);
                    mma_i8(tmem + 256, smem_desc_sw128(qhi), smem_desc_sw128(khi), idesc_i8(true, true, 128), acc);
                }
                tc_commit(bar);
            }
            // the next K tile's loads overlap the MMAs
            int4 ka = make_int4(0, 0, 0, 0), kb2 = ka;
            if (kt < qt && 128 * (kt + 1) + sr < T) {
                const int4* src =
                    reinterpret_cast<const int4*>(ap.k + (row0 + 128 * (kt + 1) + sr) * 192 + g * 64 + sc * 16);
                ka = src[0];
                kb2 = src[1];
            }
            if (!__syncthreads_and(mbar_wait(bar, phase_s, abort, err, ERR_TIMEOUT_ATTN))) { ok = false; break; }
            phase_s ^= 1;
            tc_fence_after();
            // key block kb of tile kt holds a live key for some row of this quadrant iff kt < qt or kb <= quad
            if (kt < qt || kb <= quad) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int col = kb * 32 + c * 16;
                    uint32_t d0[16], d1[16], d2[16];
                    tmem_ld16(tq + col, d0);
                    tmem_ld16(tq + 128 + col, d1);
                    tmem_ld16(tq + 256 + col, d2);
                    tmem_wait_ld();
                    tmem_launder(d0); tmem_launder(d1); tmem_launder(d2);
                    uint32_t sp[8];
#pragma unroll
                    for (int q = 0; q < 16; q += 2) {
                        int32_t s2[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int32_t a0 = static_cast<int32_t>(d0[q + u]), a1 = static_cast<int32_t>(d1[q + u]),
                                          a2 = static_cast<int32_t>(d2[q + u]);
                            if (fast) {  // exact 32-bit form of RS(65536 a2 + 256 a1 + a0, sh), as the short kernel
                                const int32_t t = a2 * 256 + a1 + ((a0 + srnd) >> 8);
                                s2[u] = t >> (ap.shift_s - 8);  // SAT16 by the saturating pack
                            } else {
                                const int64_t S = static_cast<int64_t>(a2) * 65536 + static_cast<int64_t>(a1) * 256 +
                                                  static_cast<int64_t>(a0);
                                s2[u] = static_cast<int32_t>(sat64(rs64(S, ap.shift_s), 16));
                            }
                        }
                        sp[q / 2] = pack_sat_s16(s2[1], s2[0]);
                    }
                    uint4* dst = reinterpret_cast<uint4*>(Ss + i * ATTNL_SS_PITCH + 128 * kt + col);
                    dst[0] = make_uint4(sp[0], sp[1], sp[2], sp[3]);
                    dst[1] = make_uint4(sp[4], sp[5], sp[6], sp[7]);
                }
            }
            tc_fence_before();
            __syncthreads();  // Ks and the S columns are free; on the last tile, every score is written
            tc_fence_after();
            if (kt < qt) stage_planes16(Ks, sr, sc, ka, kb2);
        }
        if (!ok) break;

        // ---- row statistics: rowmax and Z over the live keys j <= position of row r
        const int rpos = q0 + r;
        const int nk = rpos < T ? rpos + 1 : 0;
        const int16_t* srow = Ss + r * ATTNL_SS_PITCH;
        const int nm = nk > 4 * jq ? (nk - 4 * jq + 15) / 16 : 0;  // live key groups of this thread
        int32_t mx = -32768;
#pragma unroll 4
        for (int m = 0; m < nm; ++m) {
            const int k0 = 4 * (jq + 4 * m);
            const uint2 sv = *reinterpret_cast<const uint2*>(srow + k0);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int32_t sk = static_cast<int16_t>((u < 2 ? sv.x : sv.y) >> (16 * (u & 1)));
                if (k0 + u < nk) mx = max(mx, sk);
            }
        }
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        int64_t z = 0;
#pragma unroll 4
        for (int m = 0; m < nm; ++m) {
            const int k0 = 4 * (jq + 4 * m);
            const uint2 sv = *reinterpret_cast<const uint2*>(srow + k0);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int32_t sk = static_cast<int16_t>((u < 2 ? sv.x : sv.y) >> (16 * (u & 1)));
                const int32_t dd = mx - sk;
                z += (k0 + u < nk && dd <= DMAX) ? E[dd] : 0;
            }
        }
        z += __shfl_xor_sync(0xffffffffu, z, 1);
        z += __shfl_xor_sync(0xffffffffu, z, 2);
        const int64_t halfZ = z / 2;
        const float scale = z > 0 ? static_cast<float>(65536.0 / static_cast<double>(z)) : 0.f;

        // P bytes of key tile kt for this thread's groups G = 32 kt + jq + 4 m (m = 0..7)
        auto p_tile = [&](int kt, uint32_t (&b0)[8], uint32_t (&b1)[8]) {
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int k0 = 4 * (32 * kt + jq + 4 * m);
                b0[m] = 0;
                b1[m] = 0;
                if (k0 < nk) {
                    const uint2 sv = *reinterpret_cast<const uint2*>(srow + k0);
                    uint32_t p[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int32_t sk = static_cast<int16_t>((u < 2 ? sv.x : sv.y) >> (16 * (u & 1)));
                        const int32_t dd = mx - sk;
                        const int32_t ev = (k0 + u < nk && dd <= DMAX) ? E[dd] : 0;
                        p[u] = static_cast<uint32_t>(prob_q16_f32(ev, z, halfZ, scale));  // 0 for e = 0
                        if (p[u] == 65536u) jstar_s[r] = k0 + u;
                    }
                    b0[m] = __byte_perm(__byte_perm(p[0], p[1], 0x0040), __byte_perm(p[2], p[3], 0x0040), 0x5410);
                    b1[m] = __byte_perm(__byte_perm(p[0], p[1], 0x0051), __byte_perm(p[2], p[3], 0x0051), 0x5410);
                }
            }
        };
        auto v_load = [&](int kt, int4& va, int4& vb) {
            va = make_int4(0, 0, 0, 0);
            vb = va;
            const int key = 128 * kt + vj;
            if (key < T) {
                const int4* src = reinterpret_cast<const int4*>(ap.v + (row0 + key) * 192 + g * 64 + vdq * 16);
                va = src[0];
                vb = src[1];
            }
        };

        // ---- PV phase
        uint32_t b0[8], b1[8];
        int4 va, vb;
        p_tile(0, b0, b1);
        v_load(0, va, vb);
        for (int kt = 0; kt <= qt; ++kt) {
            if (kt > 0) {  // the MMAs of tile kt - 1 have read P and V^T
                if (!__syncthreads_and(mbar_wait(bar + 1, phase_p, abort, err, ERR_TIMEOUT_ATTN))) { ok = false; break; }
                phase_p ^= 1;
                tc_fence_after();
            }
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int kl = 4 * (jq + 4 * m);  // key of the tile
                *reinterpret_cast<uint32_t*>(Ps + sw128(r, kl)) = b0[m];
                *reinterpret_cast<uint32_t*>(Ps + ATTN_TC_TILE + sw128(r, kl)) = b1[m];
            }
            {
                const int16_t* v = reinterpret_cast<const int16_t*>(&va);
                const int16_t* v2 = reinterpret_cast<const int16_t*>(&vb);
#pragma unroll
                for (int d = 0; d < 16; ++d) {
                    const int16_t x = d < 8 ? v[d] : v2[d - 8];
                    VT[sw128(vdq * 16 + d, vj)] = static_cast<uint8_t>(x & 0xFF);
                    VT[8192 + sw128(vdq * 16 + d, vj)] = static_cast<uint8_t>((x >> 8) & 0xFF);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint32_t acc = (kt > 0 || ks > 0) ? 1u : 0u;
                    const uint64_t p0 = smem_desc_sw128(sP0 + ks * 32), p1 = smem_desc_sw128(sP1 + ks * 32);
                    const uint64_t v0 = smem_desc_sw128(sV0 + ks * 32), v1 = smem_desc_sw128(sV1 + ks * 32);
                    mma_i8(tmem + 0, p0, v0, idesc_i8(false, false, 64), acc);
                    mma_i8(tmem + 64, p1, v0, idesc_i8(false, false, 64), acc);
                    mma_i8(tmem + 64, p0, v1, idesc_i8(false, true, 64), 1u);
                    mma_i8(tmem + 128, p1, v1, idesc_i8(false, true, 64), acc);
                }
                tc_commit(bar + 1);
            }
            if (kt < qt) {
                p_tile(kt + 1, b0, b1);
                v_load(kt + 1, va, vb);
            }
        }
        if (!ok) break;
        if (!__syncthreads_and(mbar_wait(bar + 1, phase_p, abort, err, ERR_TIMEOUT_ATTN))) { ok = false; break; }
        phase_p ^= 1;
        tc_fence_after();

        // ---- epilogue: rows of my quadrant, dims 16 kb .. 16 kb + 15
        {
            const int col = kb * 16;
            const int pos = q0 + i;
            uint32_t c0[16], c1[16], c2[16];
            tmem_ld16(tq + col, c0);
            tmem_ld16(tq + 64 + col, c1);
            tmem_ld16(tq + 128 + col, c2);
            tmem_wait_ld();
            tmem_launder(c0); tmem_launder(c1); tmem_launder(c2);
            if (pos < T) {
                const int js = jstar_s[i];
                int16_t vs[16];
                if (js >= 0) {  // v row of the P = 65536 key (int16, the head's KV group, these 16 dims)
                    const int4* src = reinterpret_cast<const int4*>(ap.v + (row0 + js) * 192 + g * 64 + col);
                    *reinterpret_cast<int4*>(&vs[0]) = src[0];
                    *reinterpret_cast<int4*>(&vs[8]) = src[1];
                }
                int32_t out[16];
                if (!ap.generic && ap.shift_c >= 8 && ap.shift_c <= 31) {
                    const int32_t crnd = 1 << (ap.shift_c - 1);
                    const int32_t lim = ap.bits_c < 32 ? (1 << (ap.bits_c - 1)) : 0;
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        int32_t t = static_cast<int32_t>(c2[q]) * 256 + static_cast<int32_t>(c1[q]) +
                                    ((static_cast<int32_t>(c0[q]) + crnd) >> 8);
                        if (js >= 0) t += static_cast<int32_t>(vs[q]) * 256;
                        int32_t rr = t >> (ap.shift_c - 8);
                        if (lim) rr = min(max(rr, -lim), lim - 1);
                        out[q] = rr;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        int64_t a = static_cast<int64_t>(static_cast<int32_t>(c2[q])) * 65536 +
                                    (static_cast<int64_t>(static_cast<int32_t>(c1[q])) * 256 +
                                     static_cast<int64_t>(static_cast<int32_t>(c0[q])));
                        if (js >= 0) a += static_cast<int64_t>(vs[q]) * 65536;
                        out[q] = static_cast<int32_t>(sat64(rs64(a, ap.shift_c), ap.bits_c));
                    }
                }
                if (ap.offset) {  // offset binary: the bytes of ctx + 2^(8P - 1)
                    const uint32_t flip = ap.P == 4 ? 0x80000000u : 0x8000u;
#pragma unroll
                    for (int q = 0; q < 16; ++q) out[q] = static_cast<int32_t>(static_cast<uint32_t>(out[q]) ^ flip);
                }
                const int64_t pstride = blocked_plane_stride(ap.M, D_MODEL);
                uint4* dst = reinterpret_cast<uint4*>(ap.ctx_planes + blocked_off(row0 + pos, hh * 64 + col, D_MODEL));
                uint32_t w[4];
                pack_plane<0, 16>(out, w);
                dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                pack_plane<1, 16>(out, w);
                dst[pstride / 16] = make_uint4(w[0], w[1], w[2], w[3]);
                if (ap.P == 4) {
                    pack_plane<2, 16>(out, w);
                    dst[2 * pstride / 16] = make_uint4(w[0], w[1], w[2], w[3]);
                    pack_plane<3, 16>(out, w);
                    dst[3 * pstride / 16] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }  // item
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(*tmem_slot, 512);
}

}  // namespace eii
