// Host side of the B200 engine: model.bin -> device layout, the per-layer launch schedule, and
// the C ABI declared in include/eii.h.
//
// Device layout (all weights resident, about 135 MB):
//   emb_q   int8 [49152][576]   shared by the embedding gather and the tied-logits GEMM (B operand)
//   per layer: W_qkv int8 [960][576] (q | k | v rows), W_o [576][576],
//              W_gu  int8 [3072][576] gate/up interleaved per 128-row tile (64 gate rows j..j+63,
//                    then the 64 up rows j..j+63) so one GEMM tile yields gate and up of the same
//                    features for the SiLU-gated epilogue,
//              W_d   int8 [576][1536];
//              per output column (m, n + f_in - f_out) as int2; norm gains, SiLU table int32.
// Activations live in a chunk workspace of R rows (R = sequences in flight x T):
//   x       int32 [R][576]          residual stream (f = 15)
//   h       uint8 [2][R][576]       norm output byte planes (INT16)
//   q,k,v   int16 [R][576|192|192]  RoPE'd q/k and v for attention
//   ctx     uint8 [Pc][R][576]      attention output planes (Pc = 2 or 4 per layer format)
//   gated   uint8 [Pm][R][1536]     SiLU-gated product planes (Pm = 2 or 4)
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "eii.h"
#include "eii_attn.cuh"
#include "eii_tables.h"
#include "eii_gemm.cuh"
#include "eii_tgemm.cuh"
#include "eii_mma_probe.cuh"
#include "eii_kernels.cuh"

using namespace eii;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                                      \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess)                                                                        \
            return fail(EII_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)
#define TRY(...)                         \
    do {                                 \
        int rc_ = (__VA_ARGS__);         \
        if (rc_ != EII_OK) return rc_;   \
    } while (0)

constexpr int MODEL_LIN_N[7] = {576, 192, 192, 576, 1536, 1536, 576};
constexpr int MODEL_LIN_K[7] = {576, 576, 576, 576, 576, 576, 1536};

size_t model_bin_bytes() {
    size_t n = (size_t)VOCAB * D_MODEL + 2 * (size_t)VOCAB * 8 + D_MODEL * 8 + 16 + (DMAX + 1) * 8 + 2 * ROPE_POS * 32 * 8;
    size_t per = 24 * 8 + 2 * (D_MODEL * 8 + 8) + 65536 * 8;
    for (int i = 0; i < 7; ++i) per += (size_t)MODEL_LIN_N[i] * MODEL_LIN_K[i] + 2 * (size_t)MODEL_LIN_N[i] * 8;
    return n + N_LAYERS * per;
}

struct Fmt {
    int bits, f;
};

struct LayerDev {
    Fmt h, q, k, v, qr, kr, c, h2, g, u, s, m;
    int f_m, Pc, Pm;
    int norm1_shift, norm2_shift, rope_shift_q, rope_shift_k, shift_s, shift_c, gated_shift;
    int32_t *ln1, *ln2, *silu;
    void* silu_neg;  // compact SiLU table (negative half, dense range) or null
    int silu_lo, silu_count, silu_wide, silu_d;
    int fast_qkv, fast_o, fast_gu, fast_d;  // fast requantisation path applies (see EpiParams::fast)
    int narrow_qkv, narrow_gu;              // requantised values provably fit int32 (EpiParams::narrow)
    int acc32_qkv, acc32_gu;                // two-plane accumulators provably fit int32 (EpiParams::acc32)
    int gated_sd;                           // |gated| <= 2^30: signed-digit planes (EpiParams::sd_flags)
    // down projection on the feature-major GEMM (k_tgemm): the gate/up epilogue writes offset-binary
    // gated planes; per-feature constants of W_d for the layer's gated format, and 2^(b-1) S_f (the
    // trace's row-major GEMM on the same planes subtracts it)
    int t_down = 0;
    int4* tfeat_d = nullptr;
    int64_t* corr_d = nullptr;
    // O projection on the feature-major GEMM: the attention kernels write offset-binary context planes
    int t_o = 0;
    int4* tfeat_o = nullptr;
    int64_t* corr_o = nullptr;
    int8_t *w_qkv, *w_o, *w_gu, *w_d;
    int2 *msh_qkv, *msh_o, *msh_gu, *msh_d;
    CUtensorMap tm_qkv, tm_o, tm_gu, tm_d, tm_o64, tm_d64;  // *64: boxes of BN_P4 rows for 4-plane GEMMs
};

struct ActMaps {
    CUtensorMap h, ctx2, ctx4, gated2, gated4;
    CUtensorMap gated2t, gated4t, ctx2t, ctx4t, ht;  // the same planes for the feature-major GEMM (all planes of BR rows per box)
    CUtensorMap x32, x16;  // residual tiles for the O/down epilogues (32 or 16 columns x 32 rows)
    CUtensorMap q, k, v;   // RoPE'd q/k and v stores of the QKV epilogue (16 int16 x 32 rows)
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode(EncodeTiledFn* fn) {
    static EncodeTiledFn cached = nullptr;
    if (!cached) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t st = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (st != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(st));
        cached = reinterpret_cast<EncodeTiledFn>(p);
    }
    *fn = cached;
    return EII_OK;
}

// K-major uint8 tile maps with 128-byte swizzle: boxes of 128 bytes x box_rows rows (the GEMM's
// N tile: 128 for two activation planes, 64 for four).
int map_2d(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows = 128) {
    EncodeTiledFn enc;
    TRY(get_encode(&enc));
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {K};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled(2d K=%llu rows=%llu) failed: %d",
                                       (unsigned long long)K, (unsigned long long)rows, (int)r);
    return EII_OK;
}
// Row-major 2-D maps for the epilogue's TMA tile stores/loads: elements of elem_bytes, `cols` per row,
// row pitch `pitch_bytes`, box of box_cols x box_rows with the swizzle matching box_cols * elem_bytes.
int map_out(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes, uint64_t cols,
            uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
    EncodeTiledFn enc;
    TRY(get_encode(&enc));
    const uint32_t span = box_cols * elem_bytes;
    const CUtensorMapSwizzle sw = span == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : span == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : span == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled(out cols=%llu rows=%llu) failed: %d",
                                       (unsigned long long)cols, (unsigned long long)rows, (int)r);
    return EII_OK;
}

int map_planes(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t planes) {
    EncodeTiledFn enc;
    TRY(get_encode(&enc));
    cuuint64_t dims[3] = {K, rows, planes};
    cuuint64_t strides[2] = {K, K * rows};
    cuuint32_t box[3] = {128, 128, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled(3d K=%llu rows=%llu P=%llu) failed: %d",
                                       (unsigned long long)K, (unsigned long long)rows, (unsigned long long)planes, (int)r);
    return EII_OK;
}

// Planes [planes][rows][K] read by the feature-major GEMM: one box holds all `planes` planes of
// box_rows rows of a 128-byte K block (128-byte swizzle), stacked plane-major.
int map_planes_stacked(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t planes, uint32_t box_rows) {
    EncodeTiledFn enc;
    TRY(get_encode(&enc));
    cuuint64_t dims[3] = {K, rows, planes};
    cuuint64_t strides[2] = {K, K * rows};
    cuuint32_t box[3] = {128, box_rows, static_cast<cuuint32_t>(planes)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled(stacked K=%llu rows=%llu P=%llu) failed: %d",
                                       (unsigned long long)K, (unsigned long long)rows, (unsigned long long)planes, (int)r);
    return EII_OK;
}

// Row-blocked planes for the feature-major GEMM: a 4-D map over (16-byte rows of a 128-row block as
// 8-byte pairs, plane, K chunk, row block) whose box of (box_rows rows, all planes, 8 chunks) lands in
// shared memory as [8 K chunks][planes][box_rows][16 bytes], the planes stacked along the MMA's N.
int map_blocked_stacked(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t planes, uint32_t box_rows) {
    EncodeTiledFn enc;
    TRY(get_encode(&enc));
    const uint64_t mblk = (rows + 127) / 128;
    cuuint64_t dims[4] = {256, planes, K / 16, mblk};
    cuuint64_t strides[3] = {128 * K * mblk, 2048, 128 * K};
    cuuint32_t box[4] = {2 * box_rows, static_cast<cuuint32_t>(planes), 8, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled(blocked stacked K=%llu rows=%llu P=%llu) failed: %d",
                                       (unsigned long long)K, (unsigned long long)rows, (unsigned long long)planes, (int)r);
    return EII_OK;
}

// Row-blocked planes [planes][ceil(rows/128)][K/16][128 rows][16 bytes] (the gated activations): a
// 4-D map whose box (8 K-chunks of 2 KB) lands in shared memory as 8 K-chunks of 128 rows x 16 bytes
// (no swizzle), the K-major core-matrix layout the MMA reads with 2 KB / 128-byte strides.
int map_blocked(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t planes) {
    EncodeTiledFn enc;
    TRY(get_encode(&enc));
    // each 2 KB run (128 rows x 16 bytes) is one TMA row of 256 eight-byte elements
    const uint64_t mblk = (rows + 127) / 128;
    cuuint64_t dims[4] = {256, K / 16, mblk, planes};
    cuuint64_t strides[3] = {2048, 128 * K, 128 * K * mblk};
    cuuint32_t box[4] = {256, 8, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(EII_ERR_CUDA, "cuTensorMapEncodeTiled(blocked K=%llu rows=%llu P=%llu) failed: %d",
                                       (unsigned long long)K, (unsigned long long)rows, (unsigned long long)planes, (int)r);
    return EII_OK;
}

}  // namespace

struct eii_engine {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    int8_t* emb_q = nullptr;
    int32_t *emb_m = nullptr, *emb_n = nullptr;
    int2* msh_logits = nullptr;
    CUtensorMap tm_emb;
    int32_t* final_q = nullptr;
    int final_f = 0, f_y = 0, final_shift = 0;
    int fast_logits = 0;
    // tied logits on the feature-major GEMM (every shift in [1, 31], m < 2^15): the final norm writes
    // offset-binary planes; per-vocabulary-row constants
    int t_logits = 0;
    int4* tfeat_logits = nullptr;
    uint64_t *dig_a = nullptr, *dig_b = nullptr;  // logits digest weights (positions, vocabulary)
    // narrow_residual mode: per-channel shifts of the residual grid before (grid_dev[0][l]) and after
    // (grid_dev[1][l]) each layer, uint8 [2][N_LAYERS][D_MODEL] on the device
    uint8_t* grid_dev = nullptr;
    bool grid_on = false;
    int32_t *exp_tab = nullptr, *rope_c = nullptr, *rope_s = nullptr;
    LayerDev L[N_LAYERS];
    // chunk workspace
    int cap_rows = 0;
    int32_t* x = nullptr;
    uint8_t* h_planes = nullptr;
    int16_t *q = nullptr, *k = nullptr, *v = nullptr;
    uint8_t* ctx_planes = nullptr;
    uint8_t* gated_planes = nullptr;
    uint32_t* sd_flags = nullptr;  // [N_LAYERS][ceil(cap_rows / 128)]: top signed digit needed per row block
    int32_t* logits_ws = nullptr;
    int64_t logits_ws_rows = 0;
    int64_t* ids_dev = nullptr;
    int64_t ids_cap = 0;
    int* err_dev = nullptr;
    std::map<int, ActMaps> maps;
    std::vector<void*> weights;
    std::vector<void*> workspace;
    // optional per-kernel timing (eii_profile_enable): event pairs around each launch
    bool generic_norm = false;  // EII_NORM=generic: always the generic RMSNorm kernel
    bool fuse_norm = true;      // EII_NO_NORM_FUSION: the first layer's RMSNorm as its own kernel
    int generic_attention = 0;  // EII_ATTENTION=generic: 64-bit requantisation in the tensor-core attention
    bool force_cuda_core_attention = false;  // EII_ATTENTION=cuda_core selects the CUDA-core kernel (any T)
    bool decode_unstaged = false;  // EII_DECODE_UNSTAGED: decoding steps use k_attention_decode at every L
    bool prof_on = false;
    std::vector<cudaEvent_t> prof_pool;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> prof_pending;
    double prof_ms[EII_NUM_KERNEL_KINDS] = {};
    int64_t prof_n[EII_NUM_KERNEL_KINDS] = {};
};

// K/V cache of a decoder: per layer [n_seq][max_T][192] int16 post-RoPE k and v.
struct eii_decoder {
    eii_engine* e = nullptr;
    int n_seq = 0, max_T = 0, pos = 0;
    int16_t* kc = nullptr;
    int16_t* vc = nullptr;
    std::vector<void*> mem;
};

namespace {

template <class T>
int dalloc(std::vector<void*>& owner, T** p, size_t count) {
    void* q = nullptr;
    CK(cudaMalloc(&q, count * sizeof(T) + 16));
    owner.push_back(q);
    *p = static_cast<T*>(q);
    return EII_OK;
}

void free_list(std::vector<void*>& v) {
    for (void* p : v) cudaFree(p);
    v.clear();
}

cudaEvent_t prof_event(eii_engine* e) {
    if (!e->prof_pool.empty()) {
        cudaEvent_t ev = e->prof_pool.back();
        e->prof_pool.pop_back();
        return ev;
    }
    cudaEvent_t ev = nullptr;
    cudaEventCreate(&ev);
    return ev;
}

// Records an event pair around one launch when profiling is on.
struct ProfScope {
    eii_engine* e;
    int kind;
    cudaStream_t st;
    cudaEvent_t a = nullptr;
    ProfScope(eii_engine* e_, int kind_, cudaStream_t st_) : e(e_), kind(kind_), st(st_) {
        if (e->prof_on) {
            a = prof_event(e);
            cudaEventRecord(a, st);
        }
    }
    ~ProfScope() {
        if (a) {
            cudaEvent_t b = prof_event(e);
            cudaEventRecord(b, st);
            e->prof_pending.push_back({kind, {a, b}});
        }
    }
};

void prof_resolve(eii_engine* e) {
    for (auto& p : e->prof_pending) {
        float ms = 0.f;
        if (cudaEventSynchronize(p.second.second) == cudaSuccess &&
            cudaEventElapsedTime(&ms, p.second.first, p.second.second) == cudaSuccess) {
            e->prof_ms[p.first] += ms;
            e->prof_n[p.first] += 1;
        }
        e->prof_pool.push_back(p.second.first);
        e->prof_pool.push_back(p.second.second);
    }
    e->prof_pending.clear();
}

int free_workspace(eii_engine* e) {
    free_list(e->workspace);
    e->cap_rows = 0;
    e->x = nullptr;
    e->h_planes = e->ctx_planes = e->gated_planes = nullptr;
    e->sd_flags = nullptr;
    e->q = e->k = e->v = nullptr;
    e->logits_ws = nullptr;
    e->logits_ws_rows = 0;
    e->ids_dev = nullptr;
    e->ids_cap = 0;
    e->maps.clear();
    return EII_OK;
}

int ensure_rows(eii_engine* e, int rows) {
    if (rows <= e->cap_rows) return EII_OK;
    free_workspace(e);
    auto& W = e->workspace;
    TRY(dalloc(W, &e->x, (size_t)rows * D_MODEL));
    TRY(dalloc(W, &e->h_planes, (size_t)2 * rows * D_MODEL));
    TRY(dalloc(W, &e->q, (size_t)rows * D_MODEL));
    TRY(dalloc(W, &e->k, (size_t)rows * 192));
    TRY(dalloc(W, &e->v, (size_t)rows * 192));
    TRY(dalloc(W, &e->ctx_planes, (size_t)4 * ((rows + 127) / 128) * 128 * D_MODEL));  // row-blocked
    TRY(dalloc(W, &e->gated_planes, (size_t)4 * ((rows + 127) / 128) * 128 * D_FF));  // row-blocked
    TRY(dalloc(W, &e->sd_flags, (size_t)N_LAYERS * ((rows + 127) / 128)));
    e->cap_rows = rows;
    return EII_OK;
}

int ensure_logits_ws(eii_engine* e, int rows) {
    if (rows <= e->logits_ws_rows) return EII_OK;
    if (e->logits_ws) {
        for (auto it = e->workspace.begin(); it != e->workspace.end(); ++it)
            if (*it == e->logits_ws) { cudaFree(*it); e->workspace.erase(it); break; }
        e->logits_ws = nullptr;
    }
    TRY(dalloc(e->workspace, &e->logits_ws, (size_t)rows * VOCAB));
    e->logits_ws_rows = rows;
    return EII_OK;
}

int ensure_ids(eii_engine* e, int64_t n) {
    if (n <= e->ids_cap) return EII_OK;
    if (e->ids_dev) {
        for (auto it = e->workspace.begin(); it != e->workspace.end(); ++it)
            if (*it == e->ids_dev) { cudaFree(*it); e->workspace.erase(it); break; }
    }
    e->ids_dev = nullptr;
    TRY(dalloc(e->workspace, &e->ids_dev, (size_t)n));
    e->ids_cap = n;
    return EII_OK;
}

int act_maps(eii_engine* e, int rows, const ActMaps** out) {
    auto it = e->maps.find(rows);
    if (it == e->maps.end()) {
        ActMaps am;
        TRY(map_planes(&am.h, e->h_planes, D_MODEL, rows, 2));
        TRY(map_blocked(&am.ctx2, e->ctx_planes, D_MODEL, rows, 2));
        TRY(map_blocked(&am.ctx4, e->ctx_planes, D_MODEL, rows, 4));
        TRY(map_blocked(&am.gated2, e->gated_planes, D_FF, rows, 2));
        TRY(map_blocked(&am.gated4, e->gated_planes, D_FF, rows, 4));
        TRY(map_blocked_stacked(&am.gated2t, e->gated_planes, D_FF, rows, 2, 128));
        TRY(map_blocked_stacked(&am.ctx2t, e->ctx_planes, D_MODEL, rows, 2, 128));
        TRY(map_planes_stacked(&am.ht, e->h_planes, D_MODEL, rows, 2, 128));
        TRY(map_blocked_stacked(&am.ctx4t, e->ctx_planes, D_MODEL, rows, 4, 64));
        TRY(map_blocked_stacked(&am.gated4t, e->gated_planes, D_FF, rows, 4, 64));
        TRY(map_out(&am.x32, e->x, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, D_MODEL, rows, D_MODEL * 4, 32, 32));
        TRY(map_out(&am.x16, e->x, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, D_MODEL, rows, D_MODEL * 4, 16, 32));
        TRY(map_out(&am.q, e->q, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, D_MODEL, rows, D_MODEL * 2, 16, 32));
        TRY(map_out(&am.k, e->k, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, 192, rows, 192 * 2, 16, 32));
        TRY(map_out(&am.v, e->v, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, 192, rows, 192 * 2, 16, 32));
        it = e->maps.emplace(rows, am).first;
    }
    *out = &it->second;
    return EII_OK;
}

// Every hot-path kernel is launched with programmatic stream serialization: it may be scheduled
// while the previous kernel in the stream drains (each kernel does its weight-only setup, then
// griddep_wait() before touching earlier kernels' outputs).  EII_PDL=0 launches them plainly.
bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("EII_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <int P, int KIND>
int launch_gemm_raw(int device, int num_sms, const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& C0,
                    const CUtensorMap& C1, const CUtensorMap& C2, const EpiParams& ep, cudaStream_t st) {
    using C = GemmCfg<P, KIND>;
    static std::atomic<unsigned long long> attr_done{0};  // one bit per device
    const unsigned long long bit = (device >= 0 && device < 64) ? (1ull << device) : 0ull;
    if (!bit || !(attr_done.load() & bit)) {
        CK(cudaFuncSetAttribute(k_plane_gemm<P, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_done.fetch_or(bit);
    }
    const int tiles = ((ep.M + 127) / 128) * ((ep.N + C::BN - 1) / C::BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    CK(launch_k(k_plane_gemm<P, KIND>, dim3(grid), dim3(C::THREADS), C::SMEM, st, A, B, C0, C1, C2, ep));
    return EII_OK;
}

template <int P, int KIND>
int launch_gemm(eii_engine* e, const CUtensorMap& A, const CUtensorMap& B, const EpiParams& ep, cudaStream_t st,
                int prof_kind, const CUtensorMap* C0 = nullptr, const CUtensorMap* C1 = nullptr,
                const CUtensorMap* C2 = nullptr) {
    ProfScope ps(e, prof_kind, st);
    return launch_gemm_raw<P, KIND>(e->device, e->num_sms, A, B, C0 ? *C0 : A, C1 ? *C1 : A, C2 ? *C2 : A, ep, st);
}

template <int KIND>
int launch_gemm_p(eii_engine* e, int P, const CUtensorMap& A, const CUtensorMap& B, const EpiParams& ep,
                  cudaStream_t st, int prof_kind, const CUtensorMap* C0_p2 = nullptr, const CUtensorMap* C0_p4 = nullptr) {
    if (P == 2) return launch_gemm<2, KIND>(e, A, B, ep, st, prof_kind, C0_p2);
    if (P == 4) return launch_gemm<4, KIND>(e, A, B, ep, st, prof_kind, C0_p4);
    return fail(EII_ERR_FORMAT, "unsupported plane count %d", P);
}

template <int P, int KIND, bool RES, bool NODIG = false>
int launch_tgemm_r(eii_engine* e, const CUtensorMap& W, const CUtensorMap& A, const TEpi& ep, cudaStream_t st) {
    using C = TCfg<P, RES>;
    static std::atomic<unsigned long long> attr_done{0};  // one bit per device
    const unsigned long long bit = (e->device >= 0 && e->device < 64) ? (1ull << e->device) : 0ull;
    if (!bit || !(attr_done.load() & bit)) {
        CK(cudaFuncSetAttribute(k_tgemm<P, KIND, RES, NODIG>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_done.fetch_or(bit);
    }
    const int tiles = ((ep.N + C::BF - 1) / C::BF) * ((ep.M + C::BR - 1) / C::BR);
    const int grid = tiles < e->num_sms ? tiles : e->num_sms;
    CK(launch_k(k_tgemm<P, KIND, RES, NODIG>, dim3(grid), dim3(C::THREADS), C::SMEM, st, W, A, ep));
    return EII_OK;
}

// Resident activation planes when the K blocks fit (K <= 640), unless EII_TGEMM_STREAM is set.
template <int P, int KIND>
int launch_tgemm(eii_engine* e, const CUtensorMap& W, const CUtensorMap& A, const TEpi& ep, cudaStream_t st,
                 int prof_kind) {
    ProfScope ps(e, prof_kind, st);
    const bool stream_only = getenv("EII_TGEMM_STREAM") != nullptr;
    const bool res = ep.K <= 128 * TCfg<P, true>::RES_KB && !stream_only;
    if constexpr (KIND == EPI_SWEEP && P == 4) {  // the sweep without digests: the spill-free no-digest kernel
        if (!ep.dig && !ep.dig_acc)
            return res ? launch_tgemm_r<P, KIND, true, true>(e, W, A, ep, st) : launch_tgemm_r<P, KIND, false, true>(e, W, A, ep, st);
    }
    if (res) return launch_tgemm_r<P, KIND, true>(e, W, A, ep, st);
    return launch_tgemm_r<P, KIND, false>(e, W, A, ep, st);
}

// Per-feature constants of the feature-major GEMM for weights W [N][K], columns (m, shift) and
// b-bit activations: (m, shift, 2^(shift-1) - 2^(b-1) S_f m) and 2^(b-1) S_f (mod 2^64), S_f the row
// sum of W.  False (the row-major GEMM is used) when some m is 2^15 or more.
// Split-mode constants (tg_rs_split) when the activations have two planes, every shift is in [1, 31]
// and every feature's |acc| <= 2^(b-1) * sum_k |W[f][k]| is below 2^31: (m, shift, -2^15 S_f mod 2^32,
// 2^(shift-1)).  False otherwise.
bool t_features_split(const int8_t* W, int N, int K, const std::vector<int2>& msh, int bits, std::vector<int4>* feat) {
    if (bits != 16) return false;
    feat->resize(N);
    for (int f = 0; f < N; ++f) {
        const int m = msh[f].x, sh = msh[f].y;
        if (m < 0 || m >= (1 << 15) || sh < 1 || sh > 31) return false;
        int64_t S = 0, L1 = 0;
        for (int k = 0; k < K; ++k) {
            S += W[(size_t)f * K + k];
            L1 += std::abs(static_cast<int>(W[(size_t)f * K + k]));
        }
        if ((L1 << (bits - 1)) >= (int64_t(1) << 31)) return false;
        const uint32_t negc = static_cast<uint32_t>(-(static_cast<uint64_t>(S) << (bits - 1)));
        (*feat)[f] = make_int4(m, sh, static_cast<int>(negc), static_cast<int>(1u << (sh - 1)));
    }
    return true;
}

bool t_features(const int8_t* W, int N, int K, const std::vector<int2>& msh, int bits, std::vector<int4>* feat,
                std::vector<uint64_t>* corr) {
    feat->resize(N);
    corr->resize(N);
    for (int f = 0; f < N; ++f) {
        const int m = msh[f].x, sh = msh[f].y;
        if (m < 0 || m >= (1 << 15) || sh < 1 || sh > 62) return false;
        int64_t S = 0;
        for (int k = 0; k < K; ++k) S += W[(size_t)f * K + k];
        const uint64_t c = static_cast<uint64_t>(S) << (bits - 1);
        const uint64_t kc = (uint64_t(1) << (sh - 1)) - c * static_cast<uint64_t>(m);
        (*feat)[f] = make_int4(m, sh, static_cast<int>(static_cast<uint32_t>(kc)), static_cast<int>(static_cast<uint32_t>(kc >> 32)));
        (*corr)[f] = c;
    }
    return true;
}

int launch_norm(eii_engine* e, const int32_t* x, int rows, const int32_t* gain, int shift, int bits,
                uint8_t* planes, int P, int64_t* out64, cudaStream_t st, int64_t* u_out = nullptr,
                int64_t* z_out = nullptr, uint32_t* zero_ptr = nullptr, int zero_n = 0, bool offset = false) {
    const int rows_per_block = 16;  // 8 warps, two rows each
    ProfScope ps(e, EII_K_NORM, st);
    // the forward pass's own case (two INT16 planes, output shift in [10, 31]) has a lean kernel
    if (planes && P == 2 && bits == 16 && !out64 && !u_out && !z_out && shift >= 10 && shift <= 31 && !e->generic_norm) {
        CK(launch_k(k_rmsnorm_p16, dim3((rows + rows_per_block - 1) / rows_per_block), dim3(256), 0, st, x, rows, gain,
                    shift, planes, zero_ptr, zero_n, offset ? 0x80808080u : 0u));
        return EII_OK;
    }
    CK(launch_k(k_rmsnorm, dim3((rows + rows_per_block - 1) / rows_per_block), dim3(256), 0, st, x, rows, gain, shift,
                bits, planes, P, out64, u_out, z_out, zero_ptr, zero_n, offset ? 1 : 0));
    return EII_OK;
}

// The embedding of `rows` tokens into x.  With normed != nullptr, the first layer's RMSNorm planes are
// produced in the same kernel (k_embed_norm) when launch_norm would take its lean two-plane kernel and
// no residual grid runs before the layer; *normed tells whether they were.  (The same fusion into the
// feature-major down projection, for the next layer's norm, measured slower than the norm kernel: the
// GEMM's 16 epilogue warps hide the norm's L2 latency and isqrt far worse than 32 warps per SM do.)
int launch_embed(eii_engine* e, const int64_t* ids, int rows, cudaStream_t st, bool* normed = nullptr) {
    if (normed) *normed = false;
    const LayerDev& L0 = e->L[0];
    if (normed && e->fuse_norm && !e->generic_norm && !e->grid_on && L0.h.bits == 16 && L0.norm1_shift >= 10 &&
        L0.norm1_shift <= 31) {
        ProfScope ps(e, EII_K_EMBED, st);
        CK(launch_k(k_embed_norm, dim3((rows + 15) / 16), dim3(256), 0, st, ids, rows, (const int8_t*)e->emb_q,
                    (const int32_t*)e->emb_m, (const int32_t*)e->emb_n, e->x, e->err_dev, (const int32_t*)L0.ln1,
                    L0.norm1_shift, e->h_planes, 0u));
        *normed = true;
        return EII_OK;
    }
    const int rows_per_block = 8;
    ProfScope ps(e, EII_K_EMBED, st);
    CK(launch_k(k_embed, dim3((rows + rows_per_block - 1) / rows_per_block), dim3(32 * rows_per_block), 0, st, ids, rows,
                (const int8_t*)e->emb_q, (const int32_t*)e->emb_m, (const int32_t*)e->emb_n, e->x, e->err_dev));
    return EII_OK;
}

// K/V cache hook of run_layer for incremental decoding: the layer's cache [n_seq][max_T][192]
// (post-RoPE k, and v) starting at sequence seq0 of the launch.  pos < 0: a prompt pass of T
// tokens per sequence (rows stored at positions 0..T-1, attention as usual); pos >= 0: one token
// per sequence at position pos (stored there, attention against positions 0..pos of the cache).
struct KvHook {
    int16_t* kc;
    int16_t* vc;
    int max_T;
    int pos;
};

// Per-site trace hook of run_layer (python/intref.py:192-286 with trace): device buffers for the
// sites the fused kernels never materialise.  The norms run a second time in their generic form
// (U, z, int64 output), the projections and residual terms run as EPI_LINEAR GEMMs on the same
// operands (int64 output), and the attention runs on CUDA cores with score/probability outputs.
struct TraceHook {
    int64_t *u1, *z1, *n1, *q, *k, *v, *ores, *u2, *z2, *n2, *gu, *dres;
    int32_t *score, *prob, *xmid;
};

int trace_linear(eii_engine* e, int P, const CUtensorMap& A, bool a_blocked, const int8_t* W, int K, int N,
                 const int2* msh, int bits_out, int64_t* out, int rows, cudaStream_t st, bool a_sd = false,
                 const int64_t* a_corr = nullptr) {
    CUtensorMap tmB;
    TRY(map_2d(&tmB, W, K, N, P == 4 ? BN_P4 : 128));
    EpiParams ep{};
    ep.M = rows; ep.N = N; ep.K = K; ep.msh = msh; ep.err = e->err_dev; ep.out64 = out; ep.bits_out = bits_out;
    ep.a_blocked = a_blocked ? 1 : 0;
    ep.a_sd = a_sd ? 1 : 0;
    ep.a_corr = a_corr;  // offset-binary A planes: acc = (planes as unsigned) - a_corr[col]
    return launch_gemm_p<EPI_LINEAR>(e, P, A, tmB, ep, st, EII_K_GEMM_LINEAR);
}

// which = 0: the grid before layer l, 1: after it
int launch_grid(eii_engine* e, int rows, int which, int l, cudaStream_t st) {
    const int64_t n = (int64_t)rows * D_MODEL;
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)e->num_sms * 16);
    const uint8_t* s_ch = e->grid_dev + ((size_t)which * N_LAYERS + l) * D_MODEL;
    CK(launch_k(k_residual_grid, dim3(blocks), dim3(256), 0, st, e->x, n, s_ch));
    return EII_OK;
}

// norm_done: the layer's first norm is already in h_planes (the embedding produced it).
int run_layer(eii_engine* e, int l, int rows, int T, cudaStream_t st, const KvHook* kv = nullptr,
              const TraceHook* trh = nullptr, bool norm_done = false) {
    if (e->grid_on && !trh) TRY(launch_grid(e, rows, 0, l, st));
    LayerDev& L = e->L[l];
    const ActMaps* am;
    TRY(act_maps(e, rows, &am));
    const int nseq = rows / T;
    const bool decode = kv && kv->pos >= 0;
    if (!norm_done) TRY(launch_norm(e, e->x, rows, L.ln1, L.norm1_shift, L.h.bits, e->h_planes, 2, nullptr, st));
    if (trh) {
        TRY(launch_norm(e, e->x, rows, L.ln1, L.norm1_shift, L.h.bits, nullptr, 0, trh->n1, st, trh->u1, trh->z1));
        TRY(trace_linear(e, 2, am->h, false, L.w_qkv, D_MODEL, 576, L.msh_qkv, L.q.bits, trh->q, rows, st));
        TRY(trace_linear(e, 2, am->h, false, L.w_qkv + 576 * D_MODEL, D_MODEL, 192, L.msh_qkv + 576, L.k.bits, trh->k,
                         rows, st));
        TRY(trace_linear(e, 2, am->h, false, L.w_qkv + 768 * D_MODEL, D_MODEL, 192, L.msh_qkv + 768, L.v.bits, trh->v,
                         rows, st));
    }

    EpiParams ep{};
    ep.M = rows; ep.N = 960; ep.K = D_MODEL; ep.msh = L.msh_qkv; ep.err = e->err_dev;
    ep.T = T; ep.q_out = e->q; ep.k_out = e->k; ep.v_out = e->v; ep.rope_c = e->rope_c; ep.rope_s = e->rope_s;
    ep.bits_q = L.q.bits; ep.bits_k = L.k.bits; ep.bits_v = L.v.bits; ep.bits_qr = L.qr.bits; ep.bits_kr = L.kr.bits;
    ep.rope_shift_q = L.rope_shift_q; ep.rope_shift_k = L.rope_shift_k; ep.fast = L.fast_qkv; ep.narrow = L.narrow_qkv;
    ep.pos0 = decode ? kv->pos : 0;
    TRY(launch_gemm<2, EPI_QKV>(e, am->h, L.tm_qkv, ep, st, EII_K_GEMM_QKV, &am->q, &am->k, &am->v));

    if (kv && !decode) {  // keep the prompt's k, v rows (T per sequence); a step's row is appended by the attention
        const size_t row = 192 * sizeof(int16_t), pitch = row * kv->max_T;
        CK(cudaMemcpy2DAsync(kv->kc, pitch, e->k, row * T, row * T, nseq, cudaMemcpyDeviceToDevice, st));
        CK(cudaMemcpy2DAsync(kv->vc, pitch, e->v, row * T, row * T, nseq, cudaMemcpyDeviceToDevice, st));
    }
    if (decode) {
        AttnDecodeParams dp{};
        dp.q = e->q; dp.k_step = e->k; dp.v_step = e->v; dp.kc = kv->kc; dp.vc = kv->vc; dp.max_T = kv->max_T;
        dp.L = kv->pos + 1; dp.exp_tab = e->exp_tab;
        dp.ctx_planes = e->ctx_planes; dp.P = L.Pc; dp.M = rows;
        dp.shift_s = L.shift_s; dp.shift_c = L.shift_c; dp.bits_c = L.c.bits; dp.offset = L.t_o;
        ProfScope ps(e, EII_K_ATTENTION, st);
        if (dp.L <= DECODE_STAGE_L && !e->decode_unstaged)
            CK(launch_k(k_attention_decode_s, dim3(nseq * N_KV), dim3(DECODE_THREADS), decode_stage_smem(dp.L), st, dp));
        else
            CK(launch_k(k_attention_decode, dim3(nseq * N_KV), dim3(DECODE_THREADS), 0, st, dp));
    }
    AttnParams ap{};
    ap.q = e->q; ap.k = e->k; ap.v = e->v; ap.exp_tab = e->exp_tab; ap.ctx_planes = e->ctx_planes; ap.P = L.Pc;
    ap.M = rows; ap.T = T; ap.shift_s = L.shift_s; ap.shift_c = L.shift_c; ap.bits_c = L.c.bits; ap.offset = L.t_o;
    ap.generic = e->generic_attention;
    if (trh) {
        ap.score_out = trh->score;
        ap.prob_out = trh->prob;
    }
    if (!decode) {
        ProfScope ps(e, EII_K_ATTENTION, st);
        if (T <= 128 && !e->force_cuda_core_attention && !trh) {
            // persistent: one CTA per SM (its resources allow one), each looping over (sequence, KV group) items
            const int items = nseq * N_KV;
            CK(launch_k(k_attention_tc, dim3(items < e->num_sms ? items : e->num_sms), dim3(ATTN_TC_THREADS), ATTN_TC_SMEM,
                        st, ap, e->err_dev));
        } else if (!e->force_cuda_core_attention && !trh) {
            // 128 < T <= 512: persistent over (sequence, head, 128-row query tile) items
            const int items = nseq * N_HEADS * ((T + 127) / 128);
            CK(launch_k(k_attention_tc_long, dim3(items < e->num_sms ? items : e->num_sms), dim3(ATTN_TC_THREADS),
                        ATTNL_SMEM, st, ap, e->err_dev));
        } else
            CK(launch_k(k_attention, dim3(nseq * N_KV), dim3(ATTN_WARPS * 32), attn_smem_bytes(T), st, ap));
    }

    if (trh)
        TRY(trace_linear(e, L.Pc, L.Pc == 2 ? am->ctx2 : am->ctx4, true, L.w_o, D_MODEL, D_MODEL, L.msh_o, 64, trh->ores,
                         rows, st, false, L.t_o ? L.corr_o : nullptr));
    if (L.t_o) {
        TEpi tp{};
        tp.M = rows; tp.N = D_MODEL; tp.K = D_MODEL; tp.a_blocked = 1; tp.feat = L.tfeat_o; tp.err = e->err_dev;
        tp.out = e->x; tp.ld = D_MODEL;
        if (L.Pc == 2) TRY(launch_tgemm<2, EPI_RESID>(e, L.tm_o, am->ctx2t, tp, st, EII_K_GEMM_O));
        else TRY(launch_tgemm<4, EPI_RESID>(e, L.tm_o, am->ctx4t, tp, st, EII_K_GEMM_O));
    } else {
        ep = EpiParams{};
        ep.M = rows; ep.N = D_MODEL; ep.K = D_MODEL; ep.msh = L.msh_o; ep.err = e->err_dev; ep.x = e->x; ep.fast = L.fast_o;
        ep.a_blocked = 1;
        TRY(launch_gemm_p<EPI_RESID>(e, L.Pc, L.Pc == 2 ? am->ctx2 : am->ctx4, L.Pc == 2 ? L.tm_o : L.tm_o64, ep, st,
                                     EII_K_GEMM_O, &am->x32, &am->x16));
    }
    if (trh) CK(cudaMemcpyAsync(trh->xmid, e->x, sizeof(int32_t) * rows * D_MODEL, cudaMemcpyDeviceToDevice, st));

    uint32_t* sd_flags = L.gated_sd ? e->sd_flags + (size_t)l * ((e->cap_rows + 127) / 128) : nullptr;
    TRY(launch_norm(e, e->x, rows, L.ln2, L.norm2_shift, L.h2.bits, e->h_planes, 2, nullptr, st, nullptr, nullptr,
                    sd_flags, (rows + 127) / 128));
    if (trh) {
        TRY(launch_norm(e, e->x, rows, L.ln2, L.norm2_shift, L.h2.bits, nullptr, 0, trh->n2, st, trh->u2, trh->z2));
        // gate and up columns interleaved per 128-column tile, as W_gu is stored
        TRY(trace_linear(e, 2, am->h, false, L.w_gu, D_MODEL, 2 * D_FF, L.msh_gu, L.g.bits, trh->gu, rows, st));
    }

    ep = EpiParams{};
    ep.M = rows; ep.N = 2 * D_FF; ep.K = D_MODEL; ep.msh = L.msh_gu; ep.err = e->err_dev;
    ep.silu = L.silu; ep.bits_g = L.g.bits; ep.bits_u = L.u.bits; ep.gated_shift = L.gated_shift;
    ep.silu_neg = L.silu_neg; ep.silu_smem = L.silu_neg != nullptr; ep.silu_lo = L.silu_lo;
    ep.silu_count = L.silu_count; ep.silu_wide = L.silu_wide; ep.silu_d = L.silu_d; ep.bits_s = L.s.bits;
    ep.fast = L.fast_gu; ep.narrow = L.narrow_gu; ep.acc32 = L.acc32_gu;
    ep.bits_m = L.m.bits; ep.gated_P = L.Pm; ep.gated_planes = e->gated_planes; ep.sd_flags = sd_flags;
    ep.gated_offset = L.t_down;
    TRY(launch_gemm<2, EPI_GATEUP>(e, am->h, L.tm_gu, ep, st, EII_K_GEMM_GATEUP));
    if (trh)
        TRY(trace_linear(e, L.Pm, L.Pm == 2 ? am->gated2 : am->gated4, true, L.w_d, D_FF, D_MODEL, L.msh_d, 64, trh->dres,
                         rows, st, L.gated_sd != 0, L.t_down ? L.corr_d : nullptr));
    if (L.t_down) {
        TEpi tp{};
        tp.M = rows; tp.N = D_MODEL; tp.K = D_FF; tp.a_blocked = 1; tp.feat = L.tfeat_d; tp.err = e->err_dev;
        tp.out = e->x; tp.ld = D_MODEL;
        if (L.Pm == 2) TRY(launch_tgemm<2, EPI_RESID>(e, L.tm_d, am->gated2t, tp, st, EII_K_GEMM_DOWN));
        else TRY(launch_tgemm<4, EPI_RESID>(e, L.tm_d, am->gated4t, tp, st, EII_K_GEMM_DOWN));
        if (e->grid_on && !trh) TRY(launch_grid(e, rows, 1, l, st));
        return EII_OK;
    }

    ep = EpiParams{};
    ep.M = rows; ep.N = D_MODEL; ep.K = D_FF; ep.msh = L.msh_d; ep.err = e->err_dev; ep.x = e->x; ep.fast = L.fast_d;
    ep.a_blocked = 1; ep.sd_flags = sd_flags; ep.a_sd = sd_flags != nullptr;
    TRY(launch_gemm_p<EPI_RESID>(e, L.Pm, L.Pm == 2 ? am->gated2 : am->gated4, L.Pm == 2 ? L.tm_d : L.tm_d64, ep, st,
                                 EII_K_GEMM_DOWN, &am->x32, &am->x16));
    if (e->grid_on && !trh) TRY(launch_grid(e, rows, 1, l, st));
    return EII_OK;
}

// Final norm and logits of `rows` rows (whole sequences of T tokens); with digests != nullptr the
// per-sequence digests of these rows are accumulated into digests[0 .. rows / T) (zeroed by the caller).
int run_logits(eii_engine* e, int rows, int T, int32_t* logits, int64_t ld, uint64_t* digests, cudaStream_t st,
               int pos0 = 0) {
    const ActMaps* am;
    TRY(act_maps(e, rows, &am));
    TRY(launch_norm(e, e->x, rows, e->final_q, e->final_shift, 16, e->h_planes, 2, nullptr, st, nullptr, nullptr, nullptr,
                    0, e->t_logits != 0));
    if (e->t_logits) {
        TEpi tp{};
        tp.M = rows; tp.N = VOCAB; tp.K = D_MODEL; tp.feat = e->tfeat_logits; tp.err = e->err_dev;
        tp.out = logits; tp.ld = ld; tp.T = T; tp.pos0 = pos0;
        tp.dig = reinterpret_cast<unsigned long long*>(digests); tp.dig_a = e->dig_a; tp.dig_b = e->dig_b;
        return launch_tgemm<2, EPI_LOGITS>(e, e->tm_emb, am->ht, tp, st, EII_K_GEMM_LOGITS);
    }
    EpiParams ep{};
    ep.M = rows; ep.N = VOCAB; ep.K = D_MODEL; ep.msh = e->msh_logits; ep.err = e->err_dev;
    ep.logits = logits; ep.ld_logits = ld; ep.fast = e->fast_logits;
    ep.T = T; ep.pos0 = pos0;
    ep.dig = reinterpret_cast<unsigned long long*>(digests); ep.dig_a = e->dig_a; ep.dig_b = e->dig_b;
    CUtensorMap lm;
    TRY(map_out(&lm, logits, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, VOCAB, rows, (uint64_t)ld * 4, 32, 32));
    return launch_gemm<2, EPI_LOGITS>(e, am->h, e->tm_emb, ep, st, EII_K_GEMM_LOGITS, &lm);
}

int check_device_error(eii_engine* e, cudaStream_t st) {
    CK(cudaStreamSynchronize(st));
    prof_resolve(e);
    int code = 0;
    CK(cudaMemcpy(&code, e->err_dev, sizeof(int), cudaMemcpyDeviceToHost));
    if (code) {
        CK(cudaMemset(e->err_dev, 0, sizeof(int)));
        if (code == ERR_BAD_TOKEN) return fail(EII_ERR_ARG, "token id outside [0, %d)", VOCAB);
        if (code == ERR_BAD_INPUT) return fail(EII_ERR_ARG, "an activation lies outside the signed range of its format");
        return fail(EII_ERR_DEVICE, "kernel reported error %d (bounded wait timed out)", code);
    }
    return EII_OK;
}

// Sequences per chunk.  The chunk workspace holds about 65536 rows (larger chunks amortise each
// kernel's ramp: 592 x 128 rows ran a forward 3.7% faster than 148 x 128); the n_seq sequences are
// split into the fewest chunks of at most that many rows, all of (nearly) equal size, so no chunk
// is a small remainder: 4096 sequences of 128 tokens run as 8 x 512, and the 512-sequence shard of
// one of 8 GPUs as one chunk of 512 (a remainder chunk of 68 sequences filled under half of the
// SMs in every kernel).  EII_CHUNK_ROWS=R sets chunks of exactly R / T sequences instead.
int chunk_seqs_for(const eii_engine* e, int n_seq, int T) {
    (void)e;
    const char* s = getenv("EII_CHUNK_ROWS");
    const int v = s ? atoi(s) : 0;
    int cap = (v > 0 ? v : 65536) / T;
    if (cap < 1) cap = 1;
    if (cap >= n_seq) return n_seq;
    if (v > 0) return cap;
    const int chunks = (n_seq + cap - 1) / cap;
    return (n_seq + chunks - 1) / chunks;
}

// ------------------------------------------------------------------------- model loading
struct Reader {
    const uint8_t* p;
    size_t left;
    template <class T>
    const T* take(size_t count) {
        const size_t b = count * sizeof(T);
        if (b > left) return nullptr;
        const T* r = reinterpret_cast<const T*>(p);
        p += b;
        left -= b;
        return r;
    }
};

int narrow32(const int64_t* src, size_t n, std::vector<int32_t>& dst, const char* what) {
    dst.resize(n);
    for (size_t i = 0; i < n; ++i) {
        if (src[i] < INT32_MIN || src[i] > INT32_MAX)
            return fail(EII_ERR_FORMAT, "%s[%zu] = %lld does not fit int32", what, i, (long long)src[i]);
        dst[i] = static_cast<int32_t>(src[i]);
    }
    return EII_OK;
}

template <class T>
int upload(eii_engine* e, T** dst, const T* src, size_t count) {
    TRY(dalloc(e->weights, dst, count));
    CK(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
    return EII_OK;
}

// Compact SiLU table for shared memory.  Since silu(x) - silu(-x) = x, the half-up rounded table
// satisfies tab[g] = SAT_bits_s(tab[-g] + g * 2^(f_s - f_g)) for g > 0 whenever f_s >= f_g; below
// some lo <= 0 the table is 0.  The identity is checked for all 65536 inputs; if it fails, or the
// dense range does not fit SILU_SMEM_BYTES, the kernel gathers from the full table instead.
int compact_silu(eii_engine* e, LayerDev& L, const int64_t* tab) {
    L.silu_neg = nullptr;
    if (const char* mode = getenv("EII_SILU"))  // EII_SILU=global: always gather from the full table
        if (strcmp(mode, "global") == 0) return EII_OK;
    const int d = L.s.f - L.g.f;
    if (d < 0 || d > 30) return EII_OK;
    int lo = 0;
    for (int g = -32768; g <= 0; ++g)
        if (tab[g + 32768] != 0) { lo = g; break; }
    bool wide = false;
    for (int g = lo; g <= 0; ++g)
        if (tab[g + 32768] < INT16_MIN || tab[g + 32768] > INT16_MAX) wide = true;
    const int count = 1 - lo;
    if ((size_t)(count + 1) * (wide ? 4 : 2) > (size_t)SILU_SMEM_BYTES) return EII_OK;  // + the zero past the table
    const int64_t smax = (int64_t(1) << (L.s.bits - 1)) - 1, smin = -smax - 1;
    for (int g = -32768; g <= 32767; ++g) {
        const int a = g < 0 ? g : -g;
        int64_t t = a >= lo ? tab[a + 32768] : 0;
        if (g > 0) {
            t += static_cast<int64_t>(g) << d;
            t = t < smin ? smin : (t > smax ? smax : t);
        }
        if (t != tab[g + 32768]) return EII_OK;
    }
    std::vector<uint8_t> buf((size_t)count * (wide ? 4 : 2) + 16, 0);
    for (int k = 0; k < count; ++k) {
        const int64_t v = tab[lo + k + 32768];
        if (wide) reinterpret_cast<int32_t*>(buf.data())[k] = static_cast<int32_t>(v);
        else reinterpret_cast<int16_t*>(buf.data())[k] = static_cast<int16_t>(v);
    }
    uint8_t* dev;
    TRY(upload(e, &dev, buf.data(), buf.size()));
    L.silu_neg = dev;
    L.silu_lo = lo;
    L.silu_count = count;
    L.silu_wide = wide ? 1 : 0;
    L.silu_d = d;
    return EII_OK;
}

// True when, for every output column j of int8 weight rows w (K per row), an activation of magnitude
// at most amax gives |acc m_j| + 2^(sh_j - 1) < 2^(31 + sh_j): RS(acc m_j, sh_j) then fits int32.
bool cols_narrow(const int8_t* w, int N, int K, const std::vector<int2>& msh, int64_t amax) {
    for (int j = 0; j < N; ++j) {
        int64_t l1 = 0;
        for (int k = 0; k < K; ++k) l1 += std::abs(static_cast<int>(w[(size_t)j * K + k]));
        const int sh = msh[j].y;
        if (sh < 1 || sh > 31 || msh[j].x < 0) return false;
        const __int128 bound = static_cast<__int128>(amax) * l1 * msh[j].x + (static_cast<__int128>(1) << (sh - 1));
        if (bound >= (static_cast<__int128>(1) << (31 + sh))) return false;
    }
    return true;
}

// True when every column's |acc| <= amax * sum_k |w[j][k]| is below 2^31 (EpiParams::acc32).
bool cols_acc32(const int8_t* w, int N, int K, int64_t amax) {
    for (int j = 0; j < N; ++j) {
        int64_t l1 = 0;
        for (int k = 0; k < K; ++k) l1 += std::abs(static_cast<int>(w[(size_t)j * K + k]));
        if (amax * l1 >= (int64_t(1) << 31)) return false;
    }
    return true;
}

// The fast epilogue path needs every column shift in [1, 31] and every multiplier in [0, 2^15).
bool cols_fast(const std::vector<int2>& msh) {
    for (const int2& c : msh)
        if (c.y < 1 || c.y > 31 || c.x < 0 || c.x >= (1 << 15)) return false;
    return true;
}

// Per-column requantisation shifts are array shifts of the reference, which it requires to be >= 1
// (python/intref.py:49); the GEMM epilogues rely on that.
int check_col_shifts(const std::vector<int2>& msh, const char* what, int layer) {
    for (size_t j = 0; j < msh.size(); ++j)
        if (msh[j].y < 1 || msh[j].y > 62)
            return fail(EII_ERR_FORMAT, "%s shift %d at layer %d column %zu: per-element shift must be >= 1 "
                        "(python/intref.py:49)", what, msh[j].y, layer, j);
    return EII_OK;
}

int load_model(eii_engine* e, const uint8_t* data, size_t nbytes) {
    if (nbytes != model_bin_bytes())
        return fail(EII_ERR_IO, "model.bin has %zu bytes, expected %zu (layout of c/intref.c:8-13)", nbytes, model_bin_bytes());
    Reader r{data, nbytes};
    const int8_t* emb_q = r.take<int8_t>((size_t)VOCAB * D_MODEL);
    const int64_t* emb_m = r.take<int64_t>(VOCAB);
    const int64_t* emb_n = r.take<int64_t>(VOCAB);
    const int64_t* fgq = r.take<int64_t>(D_MODEL);
    const int64_t* fgf = r.take<int64_t>(1);
    const int64_t* fy = r.take<int64_t>(1);
    const int64_t* expt = r.take<int64_t>(DMAX + 1);
    const int64_t* rc = r.take<int64_t>(ROPE_POS * 32);
    const int64_t* rsn = r.take<int64_t>(ROPE_POS * 32);
    std::vector<int32_t> tmp;
    TRY(upload(e, &e->emb_q, emb_q, (size_t)VOCAB * D_MODEL));
    TRY(narrow32(emb_m, VOCAB, tmp, "emb_m"));
    TRY(upload(e, &e->emb_m, tmp.data(), VOCAB));
    TRY(narrow32(emb_n, VOCAB, tmp, "emb_n"));
    TRY(upload(e, &e->emb_n, tmp.data(), VOCAB));
    TRY(narrow32(fgq, D_MODEL, tmp, "final_gain"));
    TRY(upload(e, &e->final_q, tmp.data(), D_MODEL));
    e->final_f = (int)*fgf;
    e->f_y = (int)*fy;
    e->final_shift = 21 + e->final_f - e->f_y;
    TRY(narrow32(expt, DMAX + 1, tmp, "exp_table"));
    TRY(upload(e, &e->exp_tab, tmp.data(), DMAX + 1));
    int64_t rope_max = 0;
    for (int i = 0; i < ROPE_POS * 32; ++i) rope_max = std::max(rope_max, std::max(std::abs(rc[i]), std::abs(rsn[i])));
    TRY(narrow32(rc, ROPE_POS * 32, tmp, "rope_cos"));
    TRY(upload(e, &e->rope_c, tmp.data(), ROPE_POS * 32));
    TRY(narrow32(rsn, ROPE_POS * 32, tmp, "rope_sin"));
    TRY(upload(e, &e->rope_s, tmp.data(), ROPE_POS * 32));
    {   // logits digest weights: position t -> mix64(t), vocabulary id v -> mix64(2^32 + v)
        std::vector<uint64_t> wa(ROPE_POS), wb(VOCAB);
        for (int t = 0; t < ROPE_POS; ++t) wa[t] = mix64(static_cast<uint64_t>(t));
        for (int v = 0; v < VOCAB; ++v) wb[v] = mix64((uint64_t(1) << 32) + static_cast<uint64_t>(v));
        TRY(upload(e, &e->dig_a, wa.data(), ROPE_POS));
        TRY(upload(e, &e->dig_b, wb.data(), VOCAB));
    }
    {
        std::vector<int2> msh(VOCAB);
        for (int i = 0; i < VOCAB; ++i) msh[i] = make_int2((int)emb_m[i], (int)(emb_n[i] + e->f_y - 16));
        TRY(check_col_shifts(msh, "logits", -1));
        e->fast_logits = cols_fast(msh);
        TRY(upload(e, &e->msh_logits, msh.data(), VOCAB));
        std::vector<int4> tf;
        std::vector<uint64_t> tc;
        bool sh31 = true;
        for (const int2& c : msh) sh31 = sh31 && c.y >= 1 && c.y <= 31;
        // (measured: with the fused per-sequence digest the feature-major logits GEMM is ~5% slower per clock
        // than the row-major one at the bench's size, ~20% faster without it; EII_LOGITS_FEATURE_MAJOR=1
        // selects it)
        e->t_logits = getenv("EII_LOGITS_FEATURE_MAJOR") != nullptr && sh31 &&
                      t_features(reinterpret_cast<const int8_t*>(emb_q), VOCAB, D_MODEL, msh, 16, &tf, &tc);
        if (e->t_logits) TRY(upload(e, &e->tfeat_logits, tf.data(), VOCAB));
    }
    TRY(map_2d(&e->tm_emb, e->emb_q, D_MODEL, VOCAB));

    for (int l = 0; l < N_LAYERS; ++l) {
        LayerDev& L = e->L[l];
        const int64_t* fm = r.take<int64_t>(24);
        const int64_t* ln1 = r.take<int64_t>(D_MODEL);
        const int64_t* ln1f = r.take<int64_t>(1);
        const int64_t* ln2 = r.take<int64_t>(D_MODEL);
        const int64_t* ln2f = r.take<int64_t>(1);
        const int8_t* wq[7];
        const int64_t *wm[7], *wn[7];
        for (int i = 0; i < 7; ++i) {
            wq[i] = r.take<int8_t>((size_t)MODEL_LIN_N[i] * MODEL_LIN_K[i]);
            wm[i] = r.take<int64_t>(MODEL_LIN_N[i]);
            wn[i] = r.take<int64_t>(MODEL_LIN_N[i]);
        }
        const int64_t* silu = r.take<int64_t>(65536);
        if (!silu) return fail(EII_ERR_IO, "model.bin truncated in layer %d", l);
        Fmt* F[12] = {&L.h, &L.q, &L.k, &L.v, &L.qr, &L.kr, &L.c, &L.h2, &L.g, &L.u, &L.s, &L.m};
        for (int i = 0; i < 12; ++i) {
            F[i]->bits = (int)fm[2 * i];
            F[i]->f = (int)fm[2 * i + 1];
            if (F[i]->bits != 16 && F[i]->bits != 32)
                return fail(EII_ERR_FORMAT, "layer %d site %d has %d bits (16 or 32 expected)", l, i, F[i]->bits);
        }
        // Engine layout assumptions: norm outputs are two planes; q/k/v/rope outputs are int16;
        // the gate value indexes the 65536-entry SiLU table (python/intref.py:272).
        if (L.h.bits != 16 || L.h2.bits != 16) return fail(EII_ERR_FORMAT, "layer %d: norm output must be INT16", l);
        if (L.q.bits != 16 || L.k.bits != 16 || L.v.bits != 16 || L.qr.bits != 16 || L.kr.bits != 16)
            return fail(EII_ERR_FORMAT, "layer %d: q/k/v/rope formats must be INT16", l);
        if (L.g.bits != 16) return fail(EII_ERR_FORMAT, "layer %d: gate_proj must be INT16", l);
        L.f_m = (L.m.bits == 32) ? (L.m.f < L.s.f + L.u.f ? L.m.f : L.s.f + L.u.f) : L.m.f;
        L.Pc = L.c.bits / 8;
        L.Pm = L.m.bits / 8;
        L.norm1_shift = 21 + (int)*ln1f - L.h.f;
        L.norm2_shift = 21 + (int)*ln2f - L.h2.f;
        L.rope_shift_q = 30 + L.q.f - L.qr.f;
        L.rope_shift_k = 30 + L.k.f - L.kr.f;
        L.shift_s = L.qr.f + L.kr.f + 3 - F_SCORE;
        L.shift_c = 16 + L.v.f - L.c.f;
        L.gated_shift = L.s.f + L.u.f - L.f_m;
        TRY(narrow32(ln1, D_MODEL, tmp, "ln1"));
        TRY(upload(e, &L.ln1, tmp.data(), D_MODEL));
        TRY(narrow32(ln2, D_MODEL, tmp, "ln2"));
        TRY(upload(e, &L.ln2, tmp.data(), D_MODEL));
        TRY(narrow32(silu, 65536, tmp, "silu"));
        TRY(upload(e, &L.silu, tmp.data(), 65536));
        TRY(compact_silu(e, L, silu));

        // q | k | v
        {
            std::vector<int8_t> w((size_t)960 * D_MODEL);
            std::vector<int2> msh(960);
            size_t off = 0;
            const Fmt outf[3] = {L.q, L.k, L.v};
            int col = 0;
            for (int i = 0; i < 3; ++i) {
                const size_t nb = (size_t)MODEL_LIN_N[i] * D_MODEL;
                memcpy(w.data() + off, wq[i], nb);
                off += nb;
                for (int j = 0; j < MODEL_LIN_N[i]; ++j, ++col)
                    msh[col] = make_int2((int)wm[i][j], (int)(wn[i][j] + L.h.f - outf[i].f));
            }
            TRY(check_col_shifts(msh, "q/k/v", l));
            L.fast_qkv = cols_fast(msh) && L.rope_shift_q >= 1 && L.rope_shift_q <= 31 && L.rope_shift_k >= 1 &&
                         L.rope_shift_k <= 31;
            // RoPE: |a c - b s| <= 2 * 2^15 * 2^30 (tables are Q30), so shifts >= 16 keep it in int32
            L.narrow_qkv = L.fast_qkv && cols_narrow(w.data(), 960, D_MODEL, msh, 32768) && L.rope_shift_q >= 16 &&
                           L.rope_shift_k >= 16 && rope_max <= (int64_t(1) << 30);
            TRY(upload(e, &L.w_qkv, w.data(), w.size()));
            TRY(upload(e, &L.msh_qkv, msh.data(), 960));
            TRY(map_2d(&L.tm_qkv, L.w_qkv, D_MODEL, 960));
        }
        // o
        {
            std::vector<int2> msh(D_MODEL);
            for (int j = 0; j < D_MODEL; ++j) msh[j] = make_int2((int)wm[3][j], (int)(wn[3][j] + L.c.f - F_RES));
            TRY(check_col_shifts(msh, "o_proj", l));
            L.fast_o = cols_fast(msh);
            TRY(upload(e, &L.w_o, wq[3], (size_t)D_MODEL * D_MODEL));
            TRY(upload(e, &L.msh_o, msh.data(), D_MODEL));
            TRY(map_2d(&L.tm_o, L.w_o, D_MODEL, D_MODEL));
            TRY(map_2d(&L.tm_o64, L.w_o, D_MODEL, D_MODEL, BN_P4));
            std::vector<int4> tf;
            std::vector<uint64_t> tc;
            // (measured: with K = 576 the O projection is bound by its epilogue, where the row-major GEMM's
            // 32-bit residual path is faster; EII_O_FEATURE_MAJOR=1 selects the feature-major GEMM)
            L.t_o = getenv("EII_O_FEATURE_MAJOR") != nullptr &&
                    t_features(reinterpret_cast<const int8_t*>(wq[3]), D_MODEL, D_MODEL, msh, L.c.bits, &tf, &tc);
            if (L.t_o) {
                TRY(upload(e, &L.tfeat_o, tf.data(), D_MODEL));
                TRY(upload(e, &L.corr_o, reinterpret_cast<const int64_t*>(tc.data()), D_MODEL));
            }
        }
        // gate / up interleaved per 128-row tile
        {
            std::vector<int8_t> w((size_t)2 * D_FF * D_MODEL);
            std::vector<int2> msh(2 * D_FF);
            for (int t = 0; t < D_FF / 64; ++t) {
                for (int r2 = 0; r2 < 64; ++r2) {
                    const int j = 64 * t + r2;
                    memcpy(w.data() + ((size_t)128 * t + r2) * D_MODEL, wq[4] + (size_t)j * D_MODEL, D_MODEL);
                    memcpy(w.data() + ((size_t)128 * t + 64 + r2) * D_MODEL, wq[5] + (size_t)j * D_MODEL, D_MODEL);
                    msh[128 * t + r2] = make_int2((int)wm[4][j], (int)(wn[4][j] + L.h2.f - L.g.f));
                    msh[128 * t + 64 + r2] = make_int2((int)wm[5][j], (int)(wn[5][j] + L.h2.f - L.u.f));
                }
            }
            TRY(check_col_shifts(msh, "gate/up", l));
            L.fast_gu = cols_fast(msh) && L.gated_shift >= 0 && L.gated_shift <= 31;
            L.narrow_gu = L.fast_gu && cols_narrow(w.data(), 2 * D_FF, D_MODEL, msh, 32768);
            L.acc32_gu = L.narrow_gu && cols_acc32(w.data(), 2 * D_FF, D_MODEL, 32768) && !getenv("EII_NO_ACC32");
            // |SAT32(RS(silu * up, gs))| <= |silu * up| <= 2^15 * 2^15 when both are INT16 and gs >= 0
            L.gated_sd = L.m.bits == 32 && L.s.bits == 16 && L.u.bits == 16 && L.gated_shift >= 0 && !getenv("EII_NO_SD");
            TRY(upload(e, &L.w_gu, w.data(), w.size()));
            TRY(upload(e, &L.msh_gu, msh.data(), 2 * D_FF));
            TRY(map_2d(&L.tm_gu, L.w_gu, D_MODEL, 2 * D_FF));
        }
        // down
        {
            std::vector<int2> msh(D_MODEL);
            for (int j = 0; j < D_MODEL; ++j) msh[j] = make_int2((int)wm[6][j], (int)(wn[6][j] + L.f_m - F_RES));
            TRY(check_col_shifts(msh, "down", l));
            L.fast_d = cols_fast(msh);
            TRY(upload(e, &L.w_d, wq[6], (size_t)D_MODEL * D_FF));
            TRY(upload(e, &L.msh_d, msh.data(), D_MODEL));
            TRY(map_2d(&L.tm_d, L.w_d, D_FF, D_MODEL));
            TRY(map_2d(&L.tm_d64, L.w_d, D_FF, D_MODEL, BN_P4));
            std::vector<int4> tf;
            std::vector<uint64_t> tc;
            L.t_down = !getenv("EII_DOWN_ROW_MAJOR") &&
                       t_features(reinterpret_cast<const int8_t*>(wq[6]), D_MODEL, D_FF, msh, L.m.bits, &tf, &tc);
            if (L.t_down) {
                TRY(upload(e, &L.tfeat_d, tf.data(), D_MODEL));
                TRY(upload(e, &L.corr_d, reinterpret_cast<const int64_t*>(tc.data()), D_MODEL));
                L.gated_sd = 0;  // offset-binary planes replace the signed digits
            }
        }
    }
    if (r.left != 0) return fail(EII_ERR_IO, "model.bin has %zu trailing bytes", r.left);
    return EII_OK;
}

int open_common(const void* data, size_t nbytes, int device, eii_engine** out) {
    if (!out) return fail(EII_ERR_ARG, "out is null");
    *out = nullptr;
    int ndev = 0;
    cudaError_t st = cudaGetDeviceCount(&ndev);
    if (st != cudaSuccess || ndev == 0) return fail(EII_ERR_CUDA, "no CUDA device (%s)", cudaGetErrorString(st));
    if (device < 0 || device >= ndev) return fail(EII_ERR_ARG, "device %d out of range [0, %d)", device, ndev);
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(EII_ERR_CUDA, "device %d is sm_%d%d; this build needs sm_100", device, prop.major, prop.minor);
    eii_engine* e = new eii_engine();
    e->device = device;
    e->num_sms = prop.multiProcessorCount;
    int rc = EII_OK;
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) rc = fail(EII_ERR_CUDA, "stream create failed");
    if (rc == EII_OK) rc = dalloc(e->weights, &e->err_dev, 1);
    if (rc == EII_OK && cudaMemset(e->err_dev, 0, sizeof(int)) != cudaSuccess) rc = fail(EII_ERR_CUDA, "memset failed");
    if (rc == EII_OK) rc = load_model(e, static_cast<const uint8_t*>(data), nbytes);
    if (rc == EII_OK && getenv("EII_GENERIC_REQUANT")) {  // test switch: always take the int64 epilogue path
        e->fast_logits = 0;
        for (LayerDev& L : e->L) L.fast_qkv = L.fast_o = L.fast_gu = L.fast_d = L.narrow_qkv = L.narrow_gu = 0;
    }
    if (rc == EII_OK && getenv("EII_NO_NARROW"))  // test switch: keep the 64-bit saturation tests
        for (LayerDev& L : e->L) L.narrow_qkv = L.narrow_gu = 0;
    if (rc == EII_OK && (cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              attn_smem_bytes(ROPE_POS)) != cudaSuccess ||
                         cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              ATTN_TC_SMEM) != cudaSuccess ||
                         cudaFuncSetAttribute(k_attention_tc_long, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              ATTNL_SMEM) != cudaSuccess))
        rc = fail(EII_ERR_CUDA, "attention smem attribute failed");
    if (rc == EII_OK && getenv("EII_DECODE_UNSTAGED")) e->decode_unstaged = true;
    if (const char* a = getenv("EII_ATTENTION")) {
        e->force_cuda_core_attention = strcmp(a, "cuda_core") == 0;
        e->generic_attention = strcmp(a, "generic") == 0;
    }
    if (const char* a = getenv("EII_NORM")) e->generic_norm = strcmp(a, "generic") == 0;
    if (getenv("EII_NO_NORM_FUSION")) e->fuse_norm = false;
    if (rc != EII_OK) {
        eii_close(e);
        return rc;
    }
    *out = e;
    return EII_OK;
}


// ------------------------------------------------------------------------- incremental decoding
KvHook dec_hook(eii_decoder* d, int l, int seq0, int pos) {
    const size_t off = ((size_t)l * d->n_seq + seq0) * d->max_T * 192;
    return KvHook{d->kc + off, d->vc + off, d->max_T, pos};
}

int check_forward_args(eii_engine* e, int n_seq, int T) {
    if (!e) return fail(EII_ERR_ARG, "engine is null");
    if (n_seq < 1) return fail(EII_ERR_ARG, "n_seq must be >= 1 (got %d)", n_seq);
    if (T < 1 || T > ROPE_POS) return fail(EII_ERR_ARG, "T must be in [1, %d] (got %d)", ROPE_POS, T);
    return EII_OK;
}

int check_ids_host(const int64_t* ids, int64_t n) {
    for (int64_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= VOCAB) return fail(EII_ERR_ARG, "ids[%lld] = %lld outside [0, %d)", (long long)i, (long long)ids[i], VOCAB);
    return EII_OK;
}

// The forward pass of n_seq sequences of T tokens from host ids (eii_forward), or with a decoder:
// pos < 0 a prompt pass that also fills the K/V cache, pos >= 0 one decoding step (T = 1) at that
// position.  Sequences are processed in chunks of the engine's workspace.
int forward_host(eii_engine* e, const int64_t* ids, int n_seq, int T, int32_t* embed_out, int32_t* resid_out,
                 int32_t* logits_out, uint64_t* digests, eii_decoder* dec, int pos) {
    if (!ids) return fail(EII_ERR_ARG, "ids is null");
    TRY(check_ids_host(ids, (int64_t)n_seq * T));
    CK(cudaSetDevice(e->device));
    cudaStream_t st = e->stream;
    const int cs = chunk_seqs_for(e, n_seq, T);
    TRY(ensure_rows(e, cs * T));
    TRY(ensure_ids(e, (int64_t)cs * T));
    if (logits_out || digests) TRY(ensure_logits_ws(e, cs * T));
    uint64_t* dig_dev = nullptr;
    std::vector<void*> tmp;
    if (digests) TRY(dalloc(tmp, &dig_dev, (size_t)cs));
    int rc = EII_OK;
    const size_t row_bytes = (size_t)D_MODEL * sizeof(int32_t);
    for (int s0 = 0; s0 < n_seq && rc == EII_OK; s0 += cs) {
        const int ns = (n_seq - s0) < cs ? (n_seq - s0) : cs;
        const int rows = ns * T;
        if (cudaMemcpyAsync(e->ids_dev, ids + (int64_t)s0 * T, sizeof(int64_t) * rows, cudaMemcpyHostToDevice, st) != cudaSuccess) {
            rc = fail(EII_ERR_CUDA, "ids upload failed");
            break;
        }
        bool normed = false;
        rc = launch_embed(e, e->ids_dev, rows, st, &normed);
        if (rc == EII_OK && embed_out &&
            cudaMemcpyAsync(embed_out + (int64_t)s0 * T * D_MODEL, e->x, row_bytes * rows, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            rc = fail(EII_ERR_CUDA, "embed download failed");
        for (int l = 0; l < N_LAYERS && rc == EII_OK; ++l) {
            KvHook kv;
            if (dec) kv = dec_hook(dec, l, s0, pos);
            rc = run_layer(e, l, rows, T, st, dec ? &kv : nullptr, nullptr, l == 0 && normed);
            if (rc == EII_OK && resid_out) {
                // resid_out is [n_seq][30][T][576]: one T x 576 block per sequence and layer.
                const size_t blk = row_bytes * T;
                if (cudaMemcpy2DAsync(resid_out + ((int64_t)s0 * N_LAYERS + l) * T * D_MODEL, blk * N_LAYERS, e->x, blk,
                                      blk, ns, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                    rc = fail(EII_ERR_CUDA, "residual download failed");
            }
        }
        if (rc == EII_OK && (logits_out || digests)) {
            if (digests && cudaMemsetAsync(dig_dev, 0, sizeof(uint64_t) * ns, st) != cudaSuccess)
                rc = fail(EII_ERR_CUDA, "digest reset failed");
            if (rc == EII_OK) rc = run_logits(e, rows, T, e->logits_ws, VOCAB, digests ? dig_dev : nullptr, st, pos < 0 ? 0 : pos);
            if (rc == EII_OK && logits_out &&
                cudaMemcpyAsync(logits_out + (int64_t)s0 * T * VOCAB, e->logits_ws, sizeof(int32_t) * (size_t)rows * VOCAB,
                                cudaMemcpyDeviceToHost, st) != cudaSuccess)
                rc = fail(EII_ERR_CUDA, "logits download failed");
            if (rc == EII_OK && digests &&
                cudaMemcpyAsync(digests + s0, dig_dev, sizeof(uint64_t) * ns, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                rc = fail(EII_ERR_CUDA, "digest download failed");
        }
        if (rc == EII_OK) rc = check_device_error(e, st);
    }
    free_list(tmp);
    return rc;
}

// Device-resident forward (eii_forward_device), or a decoder prompt pass / step as in forward_host.
// sync = false: return once the work is enqueued (eii_decoder_step_device_async); device-side errors
// stay in the error word for the next check.
int forward_device(eii_engine* e, const int64_t* ids_dev, int n_seq, int T, int32_t* logits_dev, int64_t ld,
                   uint64_t* digests_dev, void* stream, eii_decoder* dec, int pos, bool sync = true) {
    if (!ids_dev) return fail(EII_ERR_ARG, "ids_dev is null");
    if (logits_dev && (ld < VOCAB || (ld % 4) != 0 || (reinterpret_cast<uintptr_t>(logits_dev) & 15)))
        return fail(EII_ERR_ARG, "logits_dev must be 16-byte aligned with ld >= %d, ld %% 4 == 0", VOCAB);
    CK(cudaSetDevice(e->device));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
    const int cs = chunk_seqs_for(e, n_seq, T);
    TRY(ensure_rows(e, cs * T));
    if (!logits_dev && digests_dev) TRY(ensure_logits_ws(e, cs * T));
    if (digests_dev) CK(cudaMemsetAsync(digests_dev, 0, sizeof(uint64_t) * n_seq, st));
    for (int s0 = 0; s0 < n_seq; s0 += cs) {
        const int ns = (n_seq - s0) < cs ? (n_seq - s0) : cs;
        const int rows = ns * T;
        bool normed = false;
        TRY(launch_embed(e, ids_dev + (int64_t)s0 * T, rows, st, &normed));
        for (int l = 0; l < N_LAYERS; ++l) {
            KvHook kv;
            if (dec) kv = dec_hook(dec, l, s0, pos);
            TRY(run_layer(e, l, rows, T, st, dec ? &kv : nullptr, nullptr, l == 0 && normed));
        }
        if (logits_dev || digests_dev) {
            int32_t* lg = logits_dev ? logits_dev + (int64_t)s0 * T * ld : e->logits_ws;
            const int64_t lld = logits_dev ? ld : VOCAB;
            TRY(run_logits(e, rows, T, lg, lld, digests_dev ? digests_dev + s0 : nullptr, st, pos < 0 ? 0 : pos));
        }
    }
    return sync ? check_device_error(e, st) : EII_OK;
}

}  // namespace

// =========================================================================================== C ABI
extern "C" {

const char* eii_last_error(void) { return g_err.c_str(); }

int eii_version(void) { return 100; }

const char* eii_kernel_name(int kind) {
    static const char* names[EII_NUM_KERNEL_KINDS] = {"embed", "rmsnorm", "gemm_qkv_rope", "attention", "gemm_o_resid",
                                                     "gemm_gateup_silu", "gemm_down_resid", "gemm_logits", "digest",
                                                     "gemm_linear", "split_planes", "gemm_sweep"};
    return (kind >= 0 && kind < EII_NUM_KERNEL_KINDS) ? names[kind] : "";
}

int eii_chunk_sequences(const eii_engine* e, int n_seq, int T) {
    if (!e) return -fail(EII_ERR_ARG, "engine is null");
    if (n_seq < 1 || T < 1) return -fail(EII_ERR_ARG, "n_seq and T must be positive");
    return chunk_seqs_for(e, n_seq, T);
}

int eii_profile_enable(eii_engine* e, int on) {
    if (!e) return fail(EII_ERR_ARG, "engine is null");
    CK(cudaSetDevice(e->device));
    if (!e->prof_pending.empty()) {
        CK(cudaDeviceSynchronize());
        prof_resolve(e);
    }
    e->prof_on = on != 0;
    for (int i = 0; i < EII_NUM_KERNEL_KINDS; ++i) { e->prof_ms[i] = 0; e->prof_n[i] = 0; }
    return EII_OK;
}

int eii_profile_read(eii_engine* e, int kind, double* total_ms, int64_t* launches) {
    if (!e || kind < 0 || kind >= EII_NUM_KERNEL_KINDS || !total_ms || !launches) return fail(EII_ERR_ARG, "bad arguments");
    CK(cudaSetDevice(e->device));
    if (!e->prof_pending.empty()) {
        CK(cudaDeviceSynchronize());
        prof_resolve(e);
    }
    *total_ms = e->prof_ms[kind];
    *launches = e->prof_n[kind];
    return EII_OK;
}

int eii_open_memory(const void* data, size_t nbytes, int device, eii_engine** out) {
    if (!data) return fail(EII_ERR_ARG, "data is null");
    return open_common(data, nbytes, device, out);
}

int eii_open(const char* path, int device, eii_engine** out) {
    if (!path) return fail(EII_ERR_ARG, "path is null");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(EII_ERR_IO, "%s: %s", path, strerror(errno));
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz < 0) { fclose(f); return fail(EII_ERR_IO, "%s: cannot size file", path); }
    std::vector<uint8_t> buf((size_t)sz);
    const size_t got = fread(buf.data(), 1, buf.size(), f);
    fclose(f);
    if (got != buf.size()) return fail(EII_ERR_IO, "%s: short read", path);
    return open_common(buf.data(), buf.size(), device, out);
}

void eii_close(eii_engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    prof_resolve(e);
    for (cudaEvent_t ev : e->prof_pool) cudaEventDestroy(ev);
    free_list(e->workspace);
    free_list(e->weights);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

int eii_forward_device(eii_engine* e, const int64_t* ids_dev, int n_seq, int T, int32_t* logits_dev, int64_t ld,
                       uint64_t* digests_dev, void* stream) {
    TRY(check_forward_args(e, n_seq, T));
    return forward_device(e, ids_dev, n_seq, T, logits_dev, ld, digests_dev, stream, nullptr, -1);
}

int eii_forward(eii_engine* e, const int64_t* ids, int n_seq, int T, int32_t* embed_out, int32_t* resid_out,
                int32_t* logits_out, uint64_t* digests) {
    TRY(check_forward_args(e, n_seq, T));
    return forward_host(e, ids, n_seq, T, embed_out, resid_out, logits_out, digests, nullptr, -1);
}

int eii_table_exp(int64_t* out) {
    if (!out) return fail(EII_ERR_ARG, "out is null");
    if (!tables::exp_table(out)) return fail(EII_ERR_FORMAT, "exp table: a value is within 2^-200 of a rounding point");
    return EII_OK;
}

int eii_table_silu(int f_in, int f_out, int bits, int64_t* out) {
    if (!out) return fail(EII_ERR_ARG, "out is null");
    if (f_in < 0 || f_in > 40 || f_out < -20 || f_out > 40 || bits < 2 || bits > 63)
        return fail(EII_ERR_ARG, "SiLU table format (f_in %d, f_out %d, bits %d) out of range", f_in, f_out, bits);
    if (!tables::silu_table(f_in, f_out, bits, out))
        return fail(EII_ERR_FORMAT, "SiLU table (%d, %d, %d): a value is within 2^-200 of a rounding point", f_in, f_out, bits);
    return EII_OK;
}

int eii_table_rope(int n_pos, int64_t* cos_out, int64_t* sin_out) {
    if (!cos_out || !sin_out) return fail(EII_ERR_ARG, "null output");
    if (n_pos < 1 || n_pos > 4096) return fail(EII_ERR_ARG, "n_pos must be in [1, 4096] (got %d)", n_pos);
    if (!tables::rope_tables(n_pos, cos_out, sin_out))
        return fail(EII_ERR_FORMAT, "RoPE tables: a value is within 2^-200 of a rounding point");
    return EII_OK;
}

int eii_verify_tables(const void* data, size_t nbytes) {
    if (!data) return fail(EII_ERR_ARG, "model.bin buffer is null");
    const uint8_t* p = static_cast<const uint8_t*>(data);
    // offsets of the model.bin layout (c/intref.c:8-13): emb_q, emb_m, emb_n, final gain + f, f_y, exp,
    // rope cos, rope sin, then per layer fm[24], ln1[576] + f, ln2[576] + f, 7 weights + m + n, silu[65536]
    size_t off = (size_t)VOCAB * D_MODEL + 2 * 8 * (size_t)VOCAB + 8 * (size_t)(D_MODEL + 1) + 8;
    const size_t exp_off = off;
    off += 8 * (size_t)(DMAX + 1);
    const size_t rope_off = off;
    off += 2 * 8 * (size_t)ROPE_POS * 32;
    static const int N_[7] = {576, 192, 192, 576, 1536, 1536, 576}, K_[7] = {576, 576, 576, 576, 576, 576, 1536};
    size_t layer_bytes = 24 * 8 + 2 * 8 * (D_MODEL + 1) + 65536 * 8;
    for (int i = 0; i < 7; ++i) layer_bytes += (size_t)N_[i] * K_[i] + 2 * 8 * (size_t)N_[i];
    if (nbytes != off + N_LAYERS * layer_bytes)
        return fail(EII_ERR_FORMAT, "model.bin is %zu bytes, the layout of c/intref.c:8-13 needs %zu", nbytes,
                    off + N_LAYERS * layer_bytes);
    auto i64 = [&](size_t o) { int64_t v; memcpy(&v, p + o, 8); return v; };
    std::vector<int64_t> gen(65536), gen2((size_t)ROPE_POS * 32);
    TRY(eii_table_exp(gen.data()));
    for (int d = 0; d <= DMAX; ++d)
        if (gen[d] != i64(exp_off + 8 * (size_t)d))
            return fail(EII_ERR_FORMAT, "exp table differs at d = %d: model.bin %lld, regenerated %lld", d,
                        (long long)i64(exp_off + 8 * (size_t)d), (long long)gen[d]);
    TRY(eii_table_rope(ROPE_POS, gen.data(), gen2.data()));
    for (int i = 0; i < ROPE_POS * 32; ++i) {
        if (gen[i] != i64(rope_off + 8 * (size_t)i))
            return fail(EII_ERR_FORMAT, "RoPE cos differs at [%d][%d]", i / 32, i % 32);
        if (gen2[i] != i64(rope_off + 8 * (size_t)(ROPE_POS * 32 + i)))
            return fail(EII_ERR_FORMAT, "RoPE sin differs at [%d][%d]", i / 32, i % 32);
    }
    std::map<long long, std::vector<int64_t>> cache;
    for (int l = 0; l < N_LAYERS; ++l) {
        const size_t lo = off + (size_t)l * layer_bytes;
        const int f_g = (int)i64(lo + 8 * 17), bits_s = (int)i64(lo + 8 * 20), f_s = (int)i64(lo + 8 * 21);
        const long long key = ((long long)f_g << 32) | ((long long)(f_s + 64) << 8) | bits_s;
        auto it = cache.find(key);
        if (it == cache.end()) {
            std::vector<int64_t> t(65536);
            TRY(eii_table_silu(f_g, f_s, bits_s, t.data()));
            it = cache.emplace(key, std::move(t)).first;
        }
        const size_t so = lo + layer_bytes - 65536 * 8;
        for (int i = 0; i < 65536; ++i)
            if (it->second[i] != i64(so + 8 * (size_t)i))
                return fail(EII_ERR_FORMAT, "SiLU table of layer %d (f_g %d, f_s %d, bits %d) differs at input %d", l,
                            f_g, f_s, bits_s, i - 32768);
    }
    return EII_OK;
}

static int set_grid(eii_engine* e, const int32_t* shift_in, const int32_t* shift_out, bool per_channel) {
    if (!e) return fail(EII_ERR_ARG, "engine is null");
    if (!shift_in && !shift_out) {
        e->grid_on = false;
        return EII_OK;
    }
    if (!shift_in || !shift_out) return fail(EII_ERR_ARG, "give both shift arrays, or neither to turn the grid off");
    const int per = per_channel ? D_MODEL : 1;
    std::vector<uint8_t> h((size_t)2 * N_LAYERS * D_MODEL);
    for (int w = 0; w < 2; ++w)
        for (int l = 0; l < N_LAYERS; ++l)
            for (int c = 0; c < D_MODEL; ++c) {
                const int32_t v = (w ? shift_out : shift_in)[(size_t)l * per + (per_channel ? c : 0)];
                if (v < 0 || v > 16)
                    return fail(EII_ERR_ARG, "residual grid shifts must be in [0, 16] (layer %d, channel %d: %d)", l, c, v);
                h[((size_t)w * N_LAYERS + l) * D_MODEL + c] = (uint8_t)v;
            }
    CK(cudaSetDevice(e->device));
    if (!e->grid_dev) TRY(dalloc(e->weights, &e->grid_dev, h.size()));
    CK(cudaStreamSynchronize(e->stream));
    CK(cudaMemcpy(e->grid_dev, h.data(), h.size(), cudaMemcpyHostToDevice));
    e->grid_on = true;
    return EII_OK;
}

int eii_set_residual_grid(eii_engine* e, const int32_t* shift_in, const int32_t* shift_out) {
    return set_grid(e, shift_in, shift_out, false);
}

int eii_set_residual_grid_channels(eii_engine* e, const int32_t* shift_in, const int32_t* shift_out) {
    return set_grid(e, shift_in, shift_out, true);
}

int eii_decoder_open(eii_engine* e, int n_seq, int max_T, eii_decoder** out) {
    if (!out) return fail(EII_ERR_ARG, "out is null");
    *out = nullptr;
    if (!e) return fail(EII_ERR_ARG, "engine is null");
    if (n_seq < 1) return fail(EII_ERR_ARG, "n_seq must be >= 1 (got %d)", n_seq);
    if (max_T < 1 || max_T > DECODE_MAX_L) return fail(EII_ERR_ARG, "max_T must be in [1, %d] (got %d)", DECODE_MAX_L, max_T);
    CK(cudaSetDevice(e->device));
    eii_decoder* d = new eii_decoder();
    d->e = e;
    d->n_seq = n_seq;
    d->max_T = max_T;
    const size_t n = (size_t)N_LAYERS * n_seq * max_T * 192;
    int rc = dalloc(d->mem, &d->kc, n);
    if (rc == EII_OK) rc = dalloc(d->mem, &d->vc, n);
    if (rc != EII_OK) {
        free_list(d->mem);
        delete d;
        return rc;
    }
    *out = d;
    return EII_OK;
}

int eii_decoder_prefill(eii_decoder* d, const int64_t* ids, int T0, int32_t* logits_out, uint64_t* digests) {
    if (!d) return fail(EII_ERR_ARG, "decoder is null");
    if (d->pos != 0) return fail(EII_ERR_ARG, "prefill comes first (the decoder is at position %d; reset it)", d->pos);
    if (T0 < 1 || T0 > d->max_T) return fail(EII_ERR_ARG, "T0 must be in [1, %d] (got %d)", d->max_T, T0);
    CK(cudaSetDevice(d->e->device));
    TRY(forward_host(d->e, ids, d->n_seq, T0, nullptr, nullptr, logits_out, digests, d, -1));
    d->pos = T0;
    return EII_OK;
}

int eii_decoder_step(eii_decoder* d, const int64_t* ids, int32_t* logits_out, uint64_t* digests) {
    if (!d) return fail(EII_ERR_ARG, "decoder is null");
    if (d->pos >= d->max_T) return fail(EII_ERR_ARG, "the K/V cache is full (max_T = %d)", d->max_T);
    CK(cudaSetDevice(d->e->device));
    TRY(forward_host(d->e, ids, d->n_seq, 1, nullptr, nullptr, logits_out, digests, d, d->pos));
    ++d->pos;
    return EII_OK;
}

int eii_decoder_step_device(eii_decoder* d, const int64_t* ids_dev, int32_t* logits_dev, int64_t ld,
                            uint64_t* digests_dev, void* stream) {
    if (!d) return fail(EII_ERR_ARG, "decoder is null");
    if (d->pos >= d->max_T) return fail(EII_ERR_ARG, "the K/V cache is full (max_T = %d)", d->max_T);
    TRY(forward_device(d->e, ids_dev, d->n_seq, 1, logits_dev, ld, digests_dev, stream, d, d->pos));
    ++d->pos;
    return EII_OK;
}

int eii_decoder_step_device_async(eii_decoder* d, const int64_t* ids_dev, int32_t* logits_dev, int64_t ld,
                                  uint64_t* digests_dev, void* stream) {
    if (!d) return fail(EII_ERR_ARG, "decoder is null");
    if (d->pos >= d->max_T) return fail(EII_ERR_ARG, "the K/V cache is full (max_T = %d)", d->max_T);
    TRY(forward_device(d->e, ids_dev, d->n_seq, 1, logits_dev, ld, digests_dev, stream, d, d->pos, false));
    ++d->pos;
    return EII_OK;
}

int eii_decoder_sync(eii_decoder* d, void* stream) {
    if (!d) return fail(EII_ERR_ARG, "decoder is null");
    CK(cudaSetDevice(d->e->device));
    return check_device_error(d->e, stream ? static_cast<cudaStream_t>(stream) : d->e->stream);
}

int eii_decoder_position(const eii_decoder* d) { return d ? d->pos : -1; }

int eii_decoder_reset(eii_decoder* d) {
    if (!d) return fail(EII_ERR_ARG, "decoder is null");
    d->pos = 0;
    return EII_OK;
}

void eii_decoder_close(eii_decoder* d) {
    if (!d) return;
    cudaSetDevice(d->e->device);
    if (d->e->stream) cudaStreamSynchronize(d->e->stream);
    free_list(d->mem);
    delete d;
}

int eii_embed(eii_engine* e, const int64_t* ids, int n, int64_t* x_out) {
    if (!e || !ids || !x_out || n < 1) return fail(EII_ERR_ARG, "bad arguments to eii_embed");
    TRY(check_ids_host(ids, n));
    CK(cudaSetDevice(e->device));
    TRY(ensure_rows(e, n));
    TRY(ensure_ids(e, n));
    CK(cudaMemcpyAsync(e->ids_dev, ids, sizeof(int64_t) * n, cudaMemcpyHostToDevice, e->stream));
    TRY(launch_embed(e, e->ids_dev, n, e->stream));
    std::vector<int32_t> h((size_t)n * D_MODEL);
    CK(cudaMemcpyAsync(h.data(), e->x, h.size() * 4, cudaMemcpyDeviceToHost, e->stream));
    TRY(check_device_error(e, e->stream));
    for (size_t i = 0; i < h.size(); ++i) x_out[i] = h[i];
    return EII_OK;
}

static int upload_x(eii_engine* e, const int64_t* x, int rows) {
    std::vector<int32_t> h((size_t)rows * D_MODEL);
    for (size_t i = 0; i < h.size(); ++i) {
        if (x[i] < INT32_MIN || x[i] > INT32_MAX) return fail(EII_ERR_ARG, "x[%zu] does not fit the INT32 residual", i);
        h[i] = (int32_t)x[i];
    }
    CK(cudaMemcpy(e->x, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
    return EII_OK;
}

int eii_block(eii_engine* e, int layer, const int64_t* x_in, int n_seq, int T, int64_t* x_out) {
    TRY(check_forward_args(e, n_seq, T));
    if (layer < 0 || layer >= N_LAYERS) return fail(EII_ERR_ARG, "layer %d out of range", layer);
    if (!x_in || !x_out) return fail(EII_ERR_ARG, "null buffer");
    CK(cudaSetDevice(e->device));
    const int rows = n_seq * T;
    TRY(ensure_rows(e, rows));
    TRY(upload_x(e, x_in, rows));
    TRY(run_layer(e, layer, rows, T, e->stream));
    std::vector<int32_t> h((size_t)rows * D_MODEL);
    CK(cudaMemcpyAsync(h.data(), e->x, h.size() * 4, cudaMemcpyDeviceToHost, e->stream));
    TRY(check_device_error(e, e->stream));
    for (size_t i = 0; i < h.size(); ++i) x_out[i] = h[i];
    return EII_OK;
}

int eii_block_trace(eii_engine* e, int layer, const int64_t* x_in, int T, eii_trace* tr) {
    TRY(check_forward_args(e, 1, T));
    if (layer < 0 || layer >= N_LAYERS) return fail(EII_ERR_ARG, "layer %d out of range", layer);
    if (!x_in || !tr) return fail(EII_ERR_ARG, "null buffer");
    LayerDev& L = e->L[layer];
    if (L.g.bits != L.u.bits) return fail(EII_ERR_FORMAT, "trace: gate and up formats differ at layer %d", layer);
    CK(cudaSetDevice(e->device));
    cudaStream_t st = e->stream;
    const int rows = T;
    const size_t RD = (size_t)rows * D_MODEL, RK = (size_t)rows * 192, RF = (size_t)rows * D_FF;
    TRY(ensure_rows(e, rows));
    TRY(upload_x(e, x_in, rows));
    std::vector<void*> tmp;
    TraceHook h{};
    int rc = EII_OK;
    auto A64 = [&](int64_t** p, size_t n) { if (rc == EII_OK) rc = dalloc(tmp, p, n); };
    auto A32 = [&](int32_t** p, size_t n) { if (rc == EII_OK) rc = dalloc(tmp, p, n); };
    A64(&h.u1, rows); A64(&h.z1, RD); A64(&h.n1, RD); A64(&h.q, RD); A64(&h.k, RK); A64(&h.v, RK); A64(&h.ores, RD);
    A64(&h.u2, rows); A64(&h.z2, RD); A64(&h.n2, RD); A64(&h.gu, 2 * RF); A64(&h.dres, RD);
    A32(&h.score, (size_t)N_HEADS * T * T); A32(&h.prob, (size_t)N_HEADS * T * T); A32(&h.xmid, RD);
    if (rc == EII_OK && (cudaMemsetAsync(h.score, 0, sizeof(int32_t) * N_HEADS * T * T, st) != cudaSuccess ||
                         cudaMemsetAsync(h.prob, 0, sizeof(int32_t) * N_HEADS * T * T, st) != cudaSuccess))
        rc = fail(EII_ERR_CUDA, "trace buffers");
    if (rc == EII_OK) rc = run_layer(e, layer, rows, T, st, nullptr, &h);
    // downloads
    std::vector<int64_t> u1(rows), z1(RD), n1(RD), q(RD), k(RK), v(RK), ores(RD), u2(rows), z2(RD), n2(RD), gu(2 * RF),
        dres(RD);
    std::vector<int32_t> score((size_t)N_HEADS * T * T), prob((size_t)N_HEADS * T * T), xmid(RD), xout(RD);
    std::vector<int16_t> qr(RD), kr(RK);
    std::vector<int32_t> silu(65536);
    const int64_t cstride = blocked_plane_stride(rows, D_MODEL), gstride = blocked_plane_stride(rows, D_FF);
    std::vector<uint8_t> ctxp((size_t)L.Pc * cstride), gatedp((size_t)L.Pm * gstride);
    struct Dl { void* dst; const void* src; size_t bytes; };
    const Dl dls[] = {{u1.data(), h.u1, rows * 8ull}, {z1.data(), h.z1, RD * 8}, {n1.data(), h.n1, RD * 8},
                      {q.data(), h.q, RD * 8}, {k.data(), h.k, RK * 8}, {v.data(), h.v, RK * 8},
                      {ores.data(), h.ores, RD * 8}, {u2.data(), h.u2, rows * 8ull}, {z2.data(), h.z2, RD * 8},
                      {n2.data(), h.n2, RD * 8}, {gu.data(), h.gu, 2 * RF * 8}, {dres.data(), h.dres, RD * 8},
                      {score.data(), h.score, score.size() * 4}, {prob.data(), h.prob, prob.size() * 4},
                      {xmid.data(), h.xmid, RD * 4}, {xout.data(), e->x, RD * 4}, {qr.data(), e->q, RD * 2},
                      {kr.data(), e->k, RK * 2}, {silu.data(), L.silu, 65536 * 4},
                      {ctxp.data(), e->ctx_planes, ctxp.size()}, {gatedp.data(), e->gated_planes, gatedp.size()}};
    for (const Dl& d : dls)
        if (rc == EII_OK && cudaMemcpyAsync(d.dst, d.src, d.bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            rc = fail(EII_ERR_CUDA, "trace download failed");
    if (rc == EII_OK) rc = check_device_error(e, st);
    free_list(tmp);
    if (rc != EII_OK) return rc;
    // planes -> values (row-blocked layout; low planes unsigned, top plane signed)
    // plane bytes -> values: two's complement (top plane signed), signed digits (all planes signed), or
    // offset binary (all planes unsigned, minus 2^(8P - 1))
    auto unblock = [&](const std::vector<uint8_t>& buf, int P, int K, int64_t stride, int64_t* out, bool all_signed,
                       bool offset = false) {
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < K; ++c) {
                const int64_t off = blocked_off(r, c, K);
                int64_t val = offset ? -((int64_t)1 << (8 * P - 1)) : 0;
                for (int p = 0; p < P; ++p) {
                    const uint8_t b = buf[p * stride + off];
                    const bool sgn = !offset && (p == P - 1 || all_signed);
                    val += (sgn ? (int64_t)(int8_t)b : (int64_t)b) * ((int64_t)1 << (8 * p));
                }
                out[(size_t)r * K + c] = val;
            }
    };
    auto put = [](int64_t* dst, const auto& src) {
        if (dst) for (size_t i = 0; i < src.size(); ++i) dst[i] = (int64_t)src[i];
    };
    if (tr->resid_in) memcpy(tr->resid_in, x_in, RD * 8);
    put(tr->norm1_U, u1); put(tr->norm1_z, z1); put(tr->norm1_out, n1);
    put(tr->q_proj, q); put(tr->k_proj, k); put(tr->v_proj, v); put(tr->q_rope, qr); put(tr->k_rope, kr);
    put(tr->attn_score, score); put(tr->attn_prob, prob);
    if (tr->attn_ctx) unblock(ctxp, L.Pc, D_MODEL, cstride, tr->attn_ctx, false, L.t_o != 0);
    put(tr->o_res, ores); put(tr->resid_mid, xmid);
    put(tr->norm2_U, u2); put(tr->norm2_z, z2); put(tr->norm2_out, n2);
    for (int r = 0; r < rows; ++r)
        for (int j = 0; j < D_FF; ++j) {  // W_gu tile t = j / 64 holds gate j at column 128 t + j % 64, up j at + 64
            const size_t cg = (size_t)r * 2 * D_FF + 128 * (j / 64) + j % 64;
            const int64_t g = gu[cg], u = gu[cg + 64];
            if (tr->gate_proj) tr->gate_proj[(size_t)r * D_FF + j] = g;
            if (tr->up_proj) tr->up_proj[(size_t)r * D_FF + j] = u;
            if (tr->silu_gate) tr->silu_gate[(size_t)r * D_FF + j] = silu[(size_t)(g + 32768)];
        }
    if (tr->mlp_gated) unblock(gatedp, L.Pm, D_FF, gstride, tr->mlp_gated, L.gated_sd != 0, L.t_down != 0);
    put(tr->down_res, dres); put(tr->resid_out, xout);
    return EII_OK;
}

int eii_rmsnorm_trace(eii_engine* e, const int64_t* x, int rows, const int64_t* gain_q, int gain_f, int f_out,
                      int bits_out, int64_t* out, int64_t* U_out, int64_t* z_out) {
    if (!e || !x || !gain_q || !out || rows < 1) return fail(EII_ERR_ARG, "bad arguments to eii_rmsnorm");
    if (bits_out < 2 || bits_out > 64) return fail(EII_ERR_ARG, "bits_out %d out of range", bits_out);
    CK(cudaSetDevice(e->device));
    TRY(ensure_rows(e, rows));
    TRY(upload_x(e, x, rows));
    std::vector<int32_t> g(D_MODEL);
    for (int i = 0; i < D_MODEL; ++i) {
        if (gain_q[i] < INT32_MIN || gain_q[i] > INT32_MAX) return fail(EII_ERR_ARG, "gain does not fit int32");
        g[i] = (int32_t)gain_q[i];
    }
    std::vector<void*> tmp;
    int32_t* gd;
    int64_t *od, *ud = nullptr, *zd = nullptr;
    TRY(dalloc(tmp, &gd, D_MODEL));
    int rc = dalloc(tmp, &od, (size_t)rows * D_MODEL);
    if (rc == EII_OK && U_out) rc = dalloc(tmp, &ud, (size_t)rows);
    if (rc == EII_OK && z_out) rc = dalloc(tmp, &zd, (size_t)rows * D_MODEL);
    if (rc == EII_OK && cudaMemcpy(gd, g.data(), D_MODEL * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = fail(EII_ERR_CUDA, "gain upload");
    if (rc == EII_OK) rc = launch_norm(e, e->x, rows, gd, 21 + gain_f - f_out, bits_out, nullptr, 0, od, e->stream, ud, zd);
    struct Dl { void* dst; const void* src; size_t bytes; };
    const Dl dls[] = {{out, od, (size_t)rows * D_MODEL * 8}, {U_out, ud, (size_t)rows * 8}, {z_out, zd, (size_t)rows * D_MODEL * 8}};
    for (const Dl& d : dls)
        if (rc == EII_OK && d.dst && cudaMemcpyAsync(d.dst, d.src, d.bytes, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
            rc = fail(EII_ERR_CUDA, "download failed");
    if (rc == EII_OK) rc = check_device_error(e, e->stream);
    free_list(tmp);
    return rc;
}

int eii_rmsnorm(eii_engine* e, const int64_t* x, int rows, const int64_t* gain_q, int gain_f, int f_out, int bits_out,
                int64_t* out) {
    return eii_rmsnorm_trace(e, x, rows, gain_q, gain_f, f_out, bits_out, out, nullptr, nullptr);
}

static int linear_device(eii_engine* e, const int64_t* a_dev, int M, int K, int bits_in, const CUtensorMap& tmB,
                         const int2* msh_dev, int N, int bits_out, int64_t* out_dev, int64_t* acc_dev,
                         std::vector<void*>& tmp) {
    const int P = bits_in / 8;
    uint8_t* planes;
    TRY(dalloc(tmp, &planes, (size_t)P * M * K));
    k_split_planes<<<1184, 256, 0, e->stream>>>(a_dev, (int64_t)M * K, P, (int64_t)M * K, planes, e->err_dev);
    CK(cudaGetLastError());
    CUtensorMap tmA;
    TRY(map_planes(&tmA, planes, K, M, P));
    EpiParams ep{};
    ep.M = M; ep.N = N; ep.K = K; ep.msh = msh_dev; ep.err = e->err_dev; ep.out64 = out_dev; ep.acc64 = acc_dev;
    ep.bits_out = bits_out;
    // tests only: EII_TEST_STALL_NS=t makes the epilogue's first wait run out after t ns (bounded-wait
    // abort path; the call then reports EII_ERR_DEVICE and the handle stays usable)
    if (const char* st = getenv("EII_TEST_STALL_NS")) ep.test_stall_ns = strtoull(st, nullptr, 10);
    return launch_gemm_p<EPI_LINEAR>(e, P, tmA, tmB, ep, e->stream, EII_K_GEMM_LINEAR);
}

int eii_linear(eii_engine* e, const int64_t* a, int M, int K, int bits_in, const int8_t* W, const int64_t* m,
               const int64_t* n, int N, int f_in, int f_out, int bits_out, int64_t* out, int64_t* acc) {
    if (!e || !a || !W || !m || !n || !out) return fail(EII_ERR_ARG, "null argument to eii_linear");
    if (M < 1 || K < 32 || K > 1536 || K % 32 != 0) return fail(EII_ERR_ARG, "K must be a multiple of 32 in [32, 1536] (got %d)", K);
    if (N < 16 || N % 16 != 0) return fail(EII_ERR_ARG, "N must be a positive multiple of 16 (got %d)", N);
    if (bits_in != 16 && bits_in != 32) return fail(EII_ERR_ARG, "bits_in must be 16 or 32 (got %d)", bits_in);
    if (bits_out < 2 || bits_out > 64) return fail(EII_ERR_ARG, "bits_out %d out of range", bits_out);
    const int64_t lo = -(int64_t(1) << (bits_in - 1)), hi = (int64_t(1) << (bits_in - 1)) - 1;
    for (int64_t i = 0; i < (int64_t)M * K; ++i)
        if (a[i] < lo || a[i] > hi) return fail(EII_ERR_ARG, "a[%lld] outside the signed %d-bit range", (long long)i, bits_in);
    CK(cudaSetDevice(e->device));
    std::vector<int2> msh(N);
    for (int j = 0; j < N; ++j) msh[j] = make_int2((int)m[j], (int)(n[j] + f_in - f_out));
    TRY(check_col_shifts(msh, "linear", -1));
    std::vector<void*> tmp;
    int64_t *a_dev, *out_dev, *acc_dev = nullptr;
    int8_t* w_dev;
    int2* msh_dev;
    int rc = EII_OK;
    rc = dalloc(tmp, &a_dev, (size_t)M * K);
    if (rc == EII_OK) rc = dalloc(tmp, &out_dev, (size_t)M * N);
    if (rc == EII_OK && acc) rc = dalloc(tmp, &acc_dev, (size_t)M * N);
    if (rc == EII_OK) rc = dalloc(tmp, &w_dev, (size_t)N * K);
    if (rc == EII_OK) rc = dalloc(tmp, &msh_dev, (size_t)N);
    if (rc == EII_OK && (cudaMemcpy(a_dev, a, (size_t)M * K * 8, cudaMemcpyHostToDevice) != cudaSuccess ||
                         cudaMemcpy(w_dev, W, (size_t)N * K, cudaMemcpyHostToDevice) != cudaSuccess ||
                         cudaMemcpy(msh_dev, msh.data(), (size_t)N * sizeof(int2), cudaMemcpyHostToDevice) != cudaSuccess))
        rc = fail(EII_ERR_CUDA, "upload failed");
    CUtensorMap tmB;
    if (rc == EII_OK) rc = map_2d(&tmB, w_dev, K, N, bits_in == 32 ? BN_P4 : 128);
    if (rc == EII_OK) rc = linear_device(e, a_dev, M, K, bits_in, tmB, msh_dev, N, bits_out, out_dev, acc_dev, tmp);
    if (rc == EII_OK && cudaMemcpyAsync(out, out_dev, (size_t)M * N * 8, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
        rc = fail(EII_ERR_CUDA, "download failed");
    if (rc == EII_OK && acc && cudaMemcpyAsync(acc, acc_dev, (size_t)M * N * 8, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
        rc = fail(EII_ERR_CUDA, "download failed");
    if (rc == EII_OK) rc = check_device_error(e, e->stream);
    free_list(tmp);
    return rc;
}

int eii_logits(eii_engine* e, const int64_t* x, int rows, int64_t* logits) {
    if (!e || !x || !logits || rows < 1) return fail(EII_ERR_ARG, "bad arguments to eii_logits");
    CK(cudaSetDevice(e->device));
    TRY(ensure_rows(e, rows));
    TRY(upload_x(e, x, rows));
    std::vector<void*> tmp;
    int64_t *y, *out;
    TRY(dalloc(tmp, &y, (size_t)rows * D_MODEL));
    int rc = dalloc(tmp, &out, (size_t)rows * VOCAB);
    if (rc == EII_OK) rc = launch_norm(e, e->x, rows, e->final_q, e->final_shift, 16, nullptr, 0, y, e->stream);
    if (rc == EII_OK) rc = linear_device(e, y, rows, D_MODEL, 16, e->tm_emb, e->msh_logits, VOCAB, 64, out, nullptr, tmp);
    if (rc == EII_OK && cudaMemcpyAsync(logits, out, (size_t)rows * VOCAB * 8, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
        rc = fail(EII_ERR_CUDA, "download failed");
    if (rc == EII_OK) rc = check_device_error(e, e->stream);
    free_list(tmp);
    return rc;
}

}  // extern "C"

// =========================================================================== device-resident linear
// A contraction with fixed int8 weights (Model.linear, python/intref.py:186-190, with W, f_in,
// f_out and bits_out bound once) run on device-resident activations: the weights and the per-column
// (m, shift) table are uploaded once at plan creation, like the model's own weights; each run splits
// the int32 activation values into byte planes (a plan-owned workspace) and runs the tcgen05 GEMM
// with the EPI_SWEEP epilogue (int32 outputs, optional per-row digests of out and of the exact acc).
struct eii_linear_plan {
    eii_engine* e = nullptr;
    int N = 0, K = 0, P = 0, bits_in = 0, bits_out = 0, fast = 0;
    int8_t* w = nullptr;
    int2* msh = nullptr;
    // feature-major GEMM (k_tgemm): per-feature (m, shift, rounding constant) and 2^(b-1) S_f; used
    // when every m < 2^15 (always for the reference's quantiser, whose m lies in [2^13, 2^14])
    int4* tfeat = nullptr;
    uint64_t* tcorr = nullptr;
    bool use_t = false;
    int4* tfeat_split = nullptr;  // split-mode constants, or null
    CUtensorMap tmB;
    std::vector<void*> mem;
    uint8_t* planes = nullptr;
    size_t planes_cap = 0;
};

extern "C" {

int eii_linear_plan_open(eii_engine* e, const int8_t* W, const int64_t* m, const int64_t* n, int N, int K,
                         int bits_in, int f_in, int f_out, int bits_out, eii_linear_plan** out) {
    if (!e || !W || !m || !n || !out) return fail(EII_ERR_ARG, "null argument to eii_linear_plan_open");
    if (K < 32 || K > 1536 || K % 32 != 0) return fail(EII_ERR_ARG, "K must be a multiple of 32 in [32, 1536] (got %d)", K);
    if (N < 16 || N % 16 != 0 || N > VOCAB) return fail(EII_ERR_ARG, "N must be a multiple of 16 in [16, %d] (got %d)", VOCAB, N);
    if (bits_in != 16 && bits_in != 32) return fail(EII_ERR_ARG, "bits_in must be 16 or 32 (got %d)", bits_in);
    if (bits_out < 2 || bits_out > 32) return fail(EII_ERR_ARG, "bits_out must be in [2, 32] for int32 outputs (got %d)", bits_out);
    std::vector<int2> msh(N);
    for (int j = 0; j < N; ++j) {
        if (m[j] < 0 || m[j] > INT32_MAX) return fail(EII_ERR_ARG, "m[%d] = %lld outside [0, 2^31)", j, (long long)m[j]);
        msh[j] = make_int2((int)m[j], (int)(n[j] + f_in - f_out));
    }
    TRY(check_col_shifts(msh, "linear plan", -1));
    CK(cudaSetDevice(e->device));
    eii_linear_plan* p = new eii_linear_plan;
    p->e = e; p->N = N; p->K = K; p->P = bits_in / 8; p->bits_in = bits_in; p->bits_out = bits_out;
    p->fast = cols_fast(msh) ? 1 : 0;
    std::vector<int4> tfeat;
    std::vector<uint64_t> tcorr;
    p->use_t = !getenv("EII_SWEEP_ROW_MAJOR") && t_features(W, N, K, msh, bits_in, &tfeat, &tcorr);
    int rc = dalloc(p->mem, &p->w, (size_t)N * K);
    if (rc == EII_OK) rc = dalloc(p->mem, &p->msh, (size_t)N);
    if (rc == EII_OK && p->use_t) rc = dalloc(p->mem, &p->tfeat, (size_t)N);
    if (rc == EII_OK && p->use_t) rc = dalloc(p->mem, &p->tcorr, (size_t)N);
    if (rc == EII_OK && (cudaMemcpy(p->w, W, (size_t)N * K, cudaMemcpyHostToDevice) != cudaSuccess ||
                         cudaMemcpy(p->msh, msh.data(), (size_t)N * sizeof(int2), cudaMemcpyHostToDevice) != cudaSuccess))
        rc = fail(EII_ERR_CUDA, "weight upload failed");
    std::vector<int4> tsplit;
    if (rc == EII_OK && p->use_t && !getenv("EII_TGEMM_WIDE") && t_features_split(W, N, K, msh, bits_in, &tsplit)) {
        rc = dalloc(p->mem, &p->tfeat_split, (size_t)N);
        if (rc == EII_OK && cudaMemcpy(p->tfeat_split, tsplit.data(), (size_t)N * sizeof(int4), cudaMemcpyHostToDevice) != cudaSuccess)
            rc = fail(EII_ERR_CUDA, "feature constant upload failed");
    }
    if (rc == EII_OK && p->use_t &&
        (cudaMemcpy(p->tfeat, tfeat.data(), (size_t)N * sizeof(int4), cudaMemcpyHostToDevice) != cudaSuccess ||
         cudaMemcpy(p->tcorr, tcorr.data(), (size_t)N * sizeof(uint64_t), cudaMemcpyHostToDevice) != cudaSuccess))
        rc = fail(EII_ERR_CUDA, "feature constant upload failed");
    if (rc == EII_OK) rc = map_2d(&p->tmB, p->w, K, N, p->P == 4 ? BN_P4 : 128);
    if (rc != EII_OK) {
        free_list(p->mem);
        delete p;
        return rc;
    }
    *out = p;
    return EII_OK;
}

int eii_linear_plan_run(eii_linear_plan* p, const int32_t* a_dev, int M, int32_t* out_dev, int64_t ld_out,
                        uint64_t* dig_out_dev, uint64_t* dig_acc_dev, void* stream) {
    if (!p || !a_dev || !out_dev) return fail(EII_ERR_ARG, "null argument to eii_linear_plan_run");
    if (M < 1) return fail(EII_ERR_ARG, "M must be >= 1 (got %d)", M);
    if ((reinterpret_cast<uintptr_t>(a_dev) & 15) || (reinterpret_cast<uintptr_t>(out_dev) & 15))
        return fail(EII_ERR_ARG, "a_dev and out_dev must be 16-byte aligned");
    if (ld_out < p->N || ld_out % 4 != 0) return fail(EII_ERR_ARG, "ld_out must be >= N (%d) and a multiple of 4", p->N);
    eii_engine* e = p->e;
    CK(cudaSetDevice(e->device));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
    const size_t need = (size_t)p->P * M * p->K;
    if (need > p->planes_cap) {
        for (auto it = p->mem.begin(); it != p->mem.end(); ++it)
            if (*it == p->planes) { CK(cudaFree(*it)); p->mem.erase(it); break; }
        p->planes = nullptr;
        p->planes_cap = 0;
        TRY(dalloc(p->mem, &p->planes, need));
        p->planes_cap = need;
    }
    if (dig_out_dev) CK(cudaMemsetAsync(dig_out_dev, 0, sizeof(uint64_t) * M, st));
    if (dig_acc_dev) CK(cudaMemsetAsync(dig_acc_dev, 0, sizeof(uint64_t) * M, st));
    const int64_t count = (int64_t)M * p->K;
    {
        ProfScope ps(e, EII_K_SPLIT_PLANES, st);
        const int64_t n16 = count / 16;
        const int64_t want = (n16 + 255) / 256, cap = (int64_t)e->num_sms * 8;
        CK(launch_k(k_split_i32, dim3((unsigned)(want < cap ? want : cap)), dim3(256), 0, st, a_dev, count, p->P,
                    count, p->planes, e->err_dev, p->use_t ? 1 : 0));
    }
    if (p->use_t) {
        CUtensorMap tmA;
        TRY(map_planes_stacked(&tmA, p->planes, p->K, M, p->P, 256 / p->P));
        TEpi tp{};
        tp.M = M; tp.N = p->N; tp.K = p->K; tp.feat = p->tfeat; tp.corr = p->tcorr; tp.err = e->err_dev;
        if (p->tfeat_split) { tp.feat = p->tfeat_split; tp.split = 1; }  // (the acc digest uses tcorr)
        tp.bits_out = p->bits_out; tp.out = out_dev; tp.ld = ld_out;
        tp.dig = reinterpret_cast<unsigned long long*>(dig_out_dev);
        tp.dig_acc = reinterpret_cast<unsigned long long*>(dig_acc_dev);
        tp.dig_b = e->dig_b;
        if (p->P == 2) TRY(launch_tgemm<2, EPI_SWEEP>(e, p->tmB, tmA, tp, st, EII_K_GEMM_SWEEP));
        else TRY(launch_tgemm<4, EPI_SWEEP>(e, p->tmB, tmA, tp, st, EII_K_GEMM_SWEEP));
        return check_device_error(e, st);
    }
    CUtensorMap tmA, om;
    TRY(map_planes(&tmA, p->planes, p->K, M, p->P));
    // output boxes: 32 rows x 32 int32 (128-byte rows) with two planes, 32 x 16 (64-byte rows) with four
    TRY(map_out(&om, out_dev, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, p->N, M, (uint64_t)ld_out * 4, p->P == 2 ? 32 : 16, 32));
    EpiParams ep{};
    ep.M = M; ep.N = p->N; ep.K = p->K; ep.msh = p->msh; ep.err = e->err_dev; ep.fast = p->fast;
    ep.logits = out_dev; ep.ld_logits = ld_out; ep.bits_out = p->bits_out;
    ep.dig = reinterpret_cast<unsigned long long*>(dig_out_dev);
    ep.dig_acc = reinterpret_cast<unsigned long long*>(dig_acc_dev);
    ep.dig_b = e->dig_b;
    TRY(launch_gemm_p<EPI_SWEEP>(e, p->P, tmA, p->tmB, ep, st, EII_K_GEMM_SWEEP, &om, &om));
    return check_device_error(e, st);
}

void eii_linear_plan_close(eii_linear_plan* p) {
    if (!p) return;
    cudaSetDevice(p->e->device);
    if (p->e->stream) cudaStreamSynchronize(p->e->stream);
    free_list(p->mem);
    delete p;
}

}  // extern "C"

// =========================================================================== allocation-free linear
// eii_linear_noalloc: the byte-plane linear of eii_linear for callers that must not allocate device
// memory.  Its scratch (the activation byte planes, the per-column (m, shift) table and the error
// word) lives in the file-scope __device__ arrays below, which every GPU that loads this library
// holds until the process exits.  Host code cannot use these names as device addresses; the
// addresses come from cudaGetSymbolAddress, once per device, on the first call made on that device.
namespace {

constexpr size_t kNoAllocPlaneBytes = EII_NOALLOC_PLANE_BYTES;
constexpr int kNoAllocMaxN = EII_NOALLOC_MAX_N;

__device__ __align__(256) uint8_t g_noalloc_planes[kNoAllocPlaneBytes];
__device__ __align__(256) int2 g_noalloc_msh[kNoAllocMaxN];
__device__ __align__(256) int g_noalloc_err[64];

struct NoAllocDevice {
    bool ready = false;
    uint8_t* planes = nullptr;
    int2* msh = nullptr;
    int* err = nullptr;
    int num_sms = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc[64];

// Per-device set-up: resolve the device addresses of the scratch arrays with that device current.
int noalloc_setup(int dev, NoAllocDevice** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocDevice& d = g_noalloc[dev];
    if (!d.ready) {
        int major = 0;
        CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10) return fail(EII_ERR_CUDA, "device %d is not sm_100", dev);
        CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.planes), g_noalloc_planes));
        CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.msh), g_noalloc_msh));
        CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.err), g_noalloc_err));
        CK(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
        d.ready = true;
    }
    *out = &d;
    return EII_OK;
}

// Per-column (m, n + f_in - f_out).  A shift outside [1, 62] violates the reference's array-shift
// rule (python/intref.py:49); it is reported through the error word and clamped so the GEMM stays
// well defined.
__global__ void k_msh_from_mn(const int64_t* __restrict__ m, const int64_t* __restrict__ n, int N, int dshift,
                              int2* __restrict__ msh, int* err) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < N; j += gridDim.x * blockDim.x) {
        int64_t sh = n[j] + dshift;
        if (sh < 1 || sh > 62) {
            atomicCAS(err, 0, ERR_BAD_SHIFT);
            sh = 1;
        }
        msh[j] = make_int2(static_cast<int>(m[j]), static_cast<int>(sh));
    }
}

}  // namespace

extern "C" int eii_linear_noalloc(const int64_t* a_dev, int M, int K, int bits_in, const int8_t* w_dev,
                                  const int64_t* m_dev, const int64_t* n_dev, int N, int f_in, int f_out,
                                  int bits_out, int64_t* out_dev, int64_t* acc_dev, void* stream) {
    if (!a_dev || !w_dev || !m_dev || !n_dev || !out_dev) return fail(EII_ERR_ARG, "null argument to eii_linear_noalloc");
    if (M < 1 || K < 32 || K > 1536 || K % 32 != 0) return fail(EII_ERR_ARG, "K must be a multiple of 32 in [32, 1536] (got %d)", K);
    if (N < 16 || N % 16 != 0) return fail(EII_ERR_ARG, "N must be a positive multiple of 16 (got %d)", N);
    if (bits_in != 16 && bits_in != 32) return fail(EII_ERR_ARG, "bits_in must be 16 or 32 (got %d)", bits_in);
    if (bits_out < 2 || bits_out > 64) return fail(EII_ERR_ARG, "bits_out %d out of range", bits_out);
    const int P = bits_in / 8;
    if ((size_t)P * M * K > kNoAllocPlaneBytes)
        return fail(EII_ERR_ARG, "eii_linear_noalloc: %d planes x M=%d x K=%d = %zu bytes exceeds the static scratch of %zu bytes",
                    P, M, K, (size_t)P * M * K, kNoAllocPlaneBytes);
    if (N > kNoAllocMaxN) return fail(EII_ERR_ARG, "eii_linear_noalloc: N=%d exceeds the maximum of %d", N, kNoAllocMaxN);
    if (reinterpret_cast<uintptr_t>(w_dev) & 15) return fail(EII_ERR_ARG, "w_dev must be 16-byte aligned");
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(EII_ERR_ARG, "device %d out of range", dev);
    NoAllocDevice* d;
    TRY(noalloc_setup(dev, &d));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CK(cudaMemsetAsync(d->err, 0, sizeof(int), st));
    k_msh_from_mn<<<(N + 255) / 256, 256, 0, st>>>(m_dev, n_dev, N, f_in - f_out, d->msh, d->err);
    CK(cudaGetLastError());
    const int64_t count = (int64_t)M * K;
    k_split_planes<<<(unsigned)((count + 255) / 256 < 4096 ? (count + 255) / 256 : 4096), 256, 0, st>>>(a_dev, count, P,
                                                                                                        count, d->planes, d->err);
    CK(cudaGetLastError());
    CUtensorMap tmA, tmB;
    TRY(map_planes(&tmA, d->planes, K, M, P));
    TRY(map_2d(&tmB, w_dev, K, N, bits_in == 32 ? BN_P4 : 128));
    EpiParams ep{};
    ep.M = M; ep.N = N; ep.K = K; ep.msh = d->msh; ep.err = d->err; ep.out64 = out_dev; ep.acc64 = acc_dev;
    ep.bits_out = bits_out;
    if (P == 2) TRY(launch_gemm_raw<2, EPI_LINEAR>(dev, d->num_sms, tmA, tmB, tmA, tmA, tmA, ep, st));
    else TRY(launch_gemm_raw<4, EPI_LINEAR>(dev, d->num_sms, tmA, tmB, tmA, tmA, tmA, ep, st));
    int code = 0;
    CK(cudaMemcpyAsync(&code, d->err, sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (code == ERR_BAD_SHIFT) return fail(EII_ERR_ARG, "n + f_in - f_out outside [1, 62] (python/intref.py:49)");
    if (code == ERR_BAD_INPUT) return fail(EII_ERR_ARG, "a_dev holds a value outside the signed %d-bit range", bits_in);
    if (code) return fail(EII_ERR_DEVICE, "kernel reported error %d (bounded wait timed out)", code);
    return EII_OK;
}

// =========================================================================== MMA-rate probe
extern "C" int eii_mma_rate(int device, int n, int noise, int threads, int iters, double* cycles_per_mma) {
    if (!cycles_per_mma) return fail(EII_ERR_ARG, "null output of eii_mma_rate");
    if (n < 16 || n > 256 || n % 16) return fail(EII_ERR_ARG, "n must be a multiple of 16 in [16, 256] (got %d)", n);
    if (noise < 0 || noise > 11) return fail(EII_ERR_ARG, "noise must be in [0, 11] (got %d)", noise);
    if (threads != 128 && threads != 256 && threads != 640) return fail(EII_ERR_ARG, "threads must be 128, 256 or 640");
    if (iters < 1 || iters > 100000) return fail(EII_ERR_ARG, "iters must be in [1, 100000]");
    CK(cudaSetDevice(device));
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    CK(cudaFuncSetAttribute(k_mma_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, MMA_PROBE_SMEM));
    std::vector<void*> mem;
    unsigned long long* clk = nullptr;
    int* err = nullptr;
    int* scratch = nullptr;
    int rc = dalloc(mem, &clk, 2);
    if (rc == EII_OK) rc = dalloc(mem, &err, 1);
    if (rc == EII_OK) rc = dalloc(mem, &scratch, (size_t)sms * 65536);
    if (rc == EII_OK && cudaMemset(err, 0, sizeof(int)) != cudaSuccess) rc = fail(EII_ERR_CUDA, "memset failed");
    if (rc == EII_OK) {
        k_mma_probe<<<sms, threads, MMA_PROBE_SMEM>>>(n, iters, noise, clk, scratch, err);
        if (cudaDeviceSynchronize() != cudaSuccess) rc = fail(EII_ERR_CUDA, "MMA probe failed: %s", cudaGetErrorString(cudaGetLastError()));
    }
    unsigned long long c = 0;
    int e = 0;
    if (rc == EII_OK && (cudaMemcpy(&c, clk, sizeof(c), cudaMemcpyDeviceToHost) != cudaSuccess ||
                         cudaMemcpy(&e, err, sizeof(e), cudaMemcpyDeviceToHost) != cudaSuccess))
        rc = fail(EII_ERR_CUDA, "probe readback failed");
    if (rc == EII_OK && e) rc = fail(EII_ERR_DEVICE, "MMA probe wait timed out");
    free_list(mem);
    if (rc == EII_OK) *cycles_per_mma = static_cast<double>(c) / (4.0 * iters);
    return rc;
}
