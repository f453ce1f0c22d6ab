// Rate of tcgen05.mma kind::i8 (M = 128, K = 32) from shared-memory operands on one CTA per SM, alone
// and beside warps that keep one class of CUDA-core work busy: the ceiling the GEMM mainloops are
// measured against (on B200: 64 cycles at N = 128, 128 at N = 256, i.e. 8192 int8 MACs per cycle per
// SM; unchanged beside shared-memory, TMEM, ALU, FFMA, 32-bit IMAD or store work, several times slower
// beside dense 32x32->64 multiply-accumulate chains).
//
// Thread 0 issues `iters` x 4 MMAs of N = n into one TMEM accumulator and waits (bounded) for them;
// warps 4.. run the chosen background work until thread 0 sets a flag:
//   0 none, 1 shared-memory loads, 2 TMEM loads (columns 256-511, which the MMAs never write),
//   3 64-bit multiply-add chains, 4 coalesced int32 global stores (evict-first), 5 32-bit IMAD chains,
//   6 FFMA chains, 7 integer ALU chains (xor/shift/add), 8 32x32->64 multiply-accumulate chains,
//   9 shared-memory stores, 10 global -> shared asynchronous copies (cp.async, 16 bytes per thread),
//   11 bulk global -> shared copies (cp.async.bulk, 8 KB each, one per background warp in flight).
// Every access stays inside this kernel's own shared memory, TMEM allocation and the caller's scratch
// buffer (noise 4 writes 64 Ki int32 per CTA).
#pragma once
#include <cstdint>

#include "eii_ptx.cuh"

namespace eii {

constexpr int MMA_PROBE_SMEM = 100 * 1024;

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__global__ void __launch_bounds__(640, 1) k_mma_probe(int nn, int iters, int noise, unsigned long long* clk_out,
                                                      int* scratch, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* A = sm;             // 16 KB: 128 rows x 128 B
    uint8_t* B = sm + 16384;     // 32 KB: up to 256 rows x 128 B
    uint8_t* X = sm + 49152;     // 32 KB: background shared-memory loads
    __shared__ uint64_t bar;
    __shared__ uint32_t tslot;
    __shared__ int stop;
    for (int i = threadIdx.x; i < (16384 + 32768 + 32768) / 16; i += blockDim.x)
        reinterpret_cast<int4*>(sm)[i] = make_int4(0x01010101, 0x02020202, 0x03030303, 0x04040404);
    if (threadIdx.x == 0) { mbar_init(&bar, 1); fence_mbar_init(); stop = 0; }
    if (threadIdx.x < 32) { tmem_alloc(&tslot, 512); tmem_relinquish(); }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const int warp = threadIdx.x / 32;
    if (threadIdx.x == 0) {
        const unsigned long long t0 = clock64();
        const uint32_t sA = smem_u32(A), sB = smem_u32(B);
        const uint32_t id = idesc_i8(false, true, nn);
        for (int it = 0; it < iters; ++it)
            for (int ks = 0; ks < 4; ++ks)
                mma_i8(tmem, smem_desc_sw128(sA + ks * 32), smem_desc_sw128(sB + ks * 32), id, (it > 0 || ks > 0) ? 1u : 0u);
        tc_commit(&bar);
        volatile int no_abort = 0;
        mbar_wait(&bar, 0, &no_abort, err, 1);
        const unsigned long long t1 = clock64();
        if (blockIdx.x == 0) clk_out[0] = t1 - t0;
        stop = 1;
    } else if (warp >= 4 && noise) {
        // the stop flag is read once per warp (lane 0's read, shuffled to all lanes), so the whole warp
        // leaves its loop together: loops with warp-collective instructions (tcgen05.ld, __syncwarp)
        // must not see lanes leave at different iterations
        volatile int* vstop = &stop;
        uint32_t acc = 0;
        if (noise == 1) {
            int i = threadIdx.x * 16;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 8
                for (int u = 0; u < 8; ++u) acc += reinterpret_cast<const int4*>(X + ((i + u * 4096) & 32767))->x;
                i += 512;
            }
        } else if (noise == 2) {
            const uint32_t ta = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 256;
            int c = 0;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
                uint32_t v[16];
                tmem_ld16(ta + (c & 15) * 16, v);
                tmem_wait_ld();
                tmem_launder(v);
#pragma unroll
                for (int q = 0; q < 16; ++q) acc += v[q];
                ++c;
            }
        } else if (noise == 3) {
            uint64_t a = threadIdx.x, b = 0x9E3779B97F4A7C15ull;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 32
                for (int q = 0; q < 32; ++q) { a = a * 0x5851F42D4C957F2Dull + b; b ^= a >> 29; }
            }
            acc = static_cast<uint32_t>(a ^ b);
        } else if (noise == 4) {
            int* g = scratch + static_cast<int64_t>(blockIdx.x) * 65536;
            int c = 0;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 8
                for (int q = 0; q < 8; ++q) __stcs(g + ((c * 8 + q) * 512 + (threadIdx.x - 128)) % 65536, c + q);
                ++c;
            }
        } else if (noise == 5) {
            uint32_t a = threadIdx.x, b = 0x9E3779B9u, c = 7;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 32
                for (int q = 0; q < 32; ++q) { a = a * 0x2C9277B5u + b; b = b * 0x5851F42Du + c; c = c * 0x14057B7Fu + a; }
            }
            acc = a ^ b ^ c;
        } else if (noise == 6) {
            float a = threadIdx.x, b = 1.0001f, c = 0.999f;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 32
                for (int q = 0; q < 32; ++q) { a = fmaf(a, 1.0000001f, b); b = fmaf(b, 0.9999999f, c); c = fmaf(c, 1.0000002f, a); }
            }
            acc = __float_as_uint(a + b + c);
        } else if (noise == 7) {
            uint32_t a = threadIdx.x, b = 0x9E3779B9u, c = 7;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 32
                for (int q = 0; q < 32; ++q) { a = (a ^ (b >> 3)) + c; b = (b ^ (c << 5)) + a; c = (c ^ (a >> 7)) + b; }
            }
            acc = a ^ b ^ c;
        } else if (noise == 8) {
            uint64_t a = threadIdx.x, b = 11, c = 13;
            uint32_t x = threadIdx.x, y = 77, z = 99;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 32
                for (int q = 0; q < 32; ++q) {
                    a += static_cast<uint64_t>(x) * 0x2C9277B5u;
                    b += static_cast<uint64_t>(y) * 0x5851F42Du;
                    c += static_cast<uint64_t>(z) * 0x14057B7Fu;
                    x ^= static_cast<uint32_t>(a >> 32); y ^= static_cast<uint32_t>(b >> 32); z ^= static_cast<uint32_t>(c >> 32);
                }
            }
            acc = static_cast<uint32_t>(a ^ b ^ c);
        }
        else if (noise == 9) {
            int i = threadIdx.x * 16;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 8
                for (int u = 0; u < 8; ++u) *reinterpret_cast<int4*>(X + ((i + u * 4096) & 32767)) = make_int4(i, u, i, u);
                i += 512;
            }
        } else if (noise == 10) {
            const int* src = scratch + static_cast<int64_t>(blockIdx.x) * 65536;
            int c = 0;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
#pragma unroll 4
                for (int u = 0; u < 4; ++u) {
                    const int off = ((c * 4 + u) * 512 + (threadIdx.x - 128)) % 8192;  // 16-byte units in 128 KB
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(X + (off & 2047) * 16)),
                                 "l"(src + off * 4)
                                 : "memory");
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                asm volatile("cp.async.wait_group 2;" ::: "memory");
                ++c;
            }
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        } else if (noise == 11) {
            // one 8 KB bulk copy at a time per background warp, into that warp's slice of X (16 warps x 2 KB
            // would not fit, so warps share X in 2 KB slices; the data is never read)
            __shared__ uint64_t nbar[16];
            const int w = warp - 4;
            if (lane_id() == 0) { mbar_init(&nbar[w], 1); fence_mbar_init(); }
            __syncwarp();
            const int* src = scratch + static_cast<int64_t>(blockIdx.x) * 65536;
            uint32_t ph = 0;
            int c = 0;
            while (!__shfl_sync(0xffffffffu, *vstop, 0)) {
                if (lane_id() == 0) {
                    mbar_arrive_expect_tx(&nbar[w], 2048);
                    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], 2048, [%2];"
                                 ::"r"(smem_u32(X + (w & 15) * 2048)), "l"(src + ((c * 16 + w) % 128) * 512),
                                 "r"(smem_u32(&nbar[w]))
                                 : "memory");
                    volatile int no_abort = 0;
                    mbar_wait(&nbar[w], ph, &no_abort, nullptr, 0, 100000000ull);
                }
                __syncwarp();
                ph ^= 1;
                ++c;
            }
        }
        if (acc == 0x12345678u) clk_out[1] = acc;  // keeps the background work observable
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

}  // namespace eii
