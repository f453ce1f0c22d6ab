/*
 * eii.h -- C ABI of the B200 engine for the integer-only SmolLM2-135M forward pass
 * (standardgalactic/exact-integer-inference, python/intref.py is the definition).
 *
 * Plain C types only.  Every call returns an EII_* status; on failure eii_last_error() gives a
 * message (thread local).  Nothing in the library calls exit().  A handle is bound to one CUDA
 * device and owns the device copy of the weights and its workspaces; calls on one handle must be
 * serialised by the caller, different handles may be used from different host threads.
 *
 * Integer results are bit-identical to python/intref.py: int64-valued states are returned as the
 * int32/int64 the reference exports (exp_embed.i32, exp_resid_out.i32, exp_logits.i32).
 */
#ifndef EII_H
#define EII_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1..3 mirror the reference programs' exit codes where they overlap:
 * c/intref.c and cuda/intref.cu exit 2 on I/O errors and 3 on CUDA errors. */
#define EII_OK 0
#define EII_ERR_ARG 1      /* bad argument: null pointer, shape, T > 512, token id out of range */
#define EII_ERR_IO 2       /* model file missing, unreadable or of the wrong size */
#define EII_ERR_CUDA 3     /* CUDA runtime/driver error, or no usable sm_100 device */
#define EII_ERR_DEVICE 4   /* a kernel reported an error (bounded wait timed out, bad token) */
#define EII_ERR_FORMAT 5   /* model.bin holds a format this engine does not implement */

typedef struct eii_engine eii_engine;

/* Message of the last failed call on this thread ("" if none). */
const char* eii_last_error(void);

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int eii_version(void);

/* Load model.bin (layout of c/intref.c:8-13, writer python/export_vectors.py:24-45) onto
 * `device`.  Replaces load_model() of c/intref.c:70-91 and cuda/intref.cu:184-206. */
int eii_open(const char* model_bin_path, int device, eii_engine** out);

/* Same, from a caller-owned buffer holding the model.bin bytes (copied; may be freed after). */
int eii_open_memory(const void* data, size_t nbytes, int device, eii_engine** out);

void eii_close(eii_engine* e);

/* Forward pass of n_seq independent sequences of T tokens each (1 <= T <= 512), host buffers.
 * Replaces Model.forward (python/intref.py:288-301) applied to each sequence, plus the state
 * export of python/export_vectors.py:47-57.
 *   ids        [n_seq][T] int64 token ids in [0, 49152)
 *   embed_out  nullable, [n_seq][T][576] int32 embedding output (exp_embed.i32 per sequence)
 *   resid_out  nullable, [n_seq][30][T][576] int32 residual after each block (exp_resid_out.i32)
 *   logits_out nullable, [n_seq][T][49152] int32 logits, f = 16 (exp_logits.i32)
 *   digests    nullable, [n_seq] uint64 order-independent digest of each sequence's logits:
 *              sum over (t, v) of uint32(logit[t][v]) * mix64(t) * mix64(2^32 + v) mod 2^64, mix64
 *              the splitmix64 finaliser with the low bit forced to 1 (so every weight is odd and
 *              any single changed logit changes the digest).  It is accumulated inside the logits
 *              GEMM epilogue; the logits are not read back to compute it. */
int eii_forward(eii_engine* e, const int64_t* ids, int n_seq, int T, int32_t* embed_out,
                int32_t* resid_out, int32_t* logits_out, uint64_t* digests);

/* Device-resident variant: ids_dev, logits_dev (row stride ld_logits elements, 16-byte aligned
 * rows) and digests_dev are device pointers on the handle's device; either output may be null.
 * `stream` is a cudaStream_t (null = the handle's own stream).  Returns after the work is
 * enqueued and completed. */
int eii_forward_device(eii_engine* e, const int64_t* ids_dev, int n_seq, int T, int32_t* logits_dev,
                       int64_t ld_logits, uint64_t* digests_dev, void* stream);

/* Independent regeneration of the model.bin tables (python/intref.py:66-108: exp_table, silu_table,
 * rope_tables), host only (no device needed).  The reference computes them with mpmath at 50
 * digits and lists an independent cross-check as open work; these compute every value in 320-bit
 * binary fixed point from their own series and round half up only where an error bound proves
 * the decision (EII_ERR_FORMAT otherwise).
 *   eii_table_exp:  out[1537],  E[d] = floor(2^30 exp(-d/128) + 1/2)
 *   eii_table_silu: out[65536], SAT_bits(floor(x / (1 + exp(-x)) 2^f_out + 1/2)), x = (i - 32768) 2^-f_in
 *   eii_table_rope: cos_out, sin_out [n_pos][32], floor(2^30 cos/sin(p 100000^(-2j/64)) + 1/2)
 * eii_verify_tables regenerates every table of a model.bin image and reports the first difference. */
int eii_table_exp(int64_t* out);
int eii_table_silu(int f_in, int f_out, int bits, int64_t* out);
int eii_table_rope(int n_pos, int64_t* cos_out, int64_t* sin_out);
int eii_verify_tables(const void* model_bin, size_t nbytes);

/* Narrow comparison mode of Model.forward(ids, narrow_residual=True) (python/intref.py:288-308):
 * the residual is put on its INT16 per-tensor grid, x = SAT16(RS(x, s)) << s, before layer l with
 * s = shift_in[l] and after it with s = shift_out[l] (s = k of the resid_in|l / resid_out|l sites
 * of the format proposal, in [0, 16]).  It applies to eii_forward*, eii_block and the decoder
 * until turned off with two null pointers.  The narrow site formats (wide=False) need no engine
 * setting: they are a model.bin with INT16 formats and tables (see the drop-in Model). */
int eii_set_residual_grid(eii_engine* e, const int32_t* shift_in, const int32_t* shift_out);
/* Same with one shift per channel: shift_in, shift_out [30][576] (x[:, c] = SAT16(RS(x[:, c], s_c)) << s_c,
 * s_c in [0, 16]), the grid of a Model subclass whose _grid uses per-channel exponents (the
 * reference's ablate_perchannel.py:31-36 and ablate_layers.py:31-44 restate _grid that way). */
int eii_set_residual_grid_channels(eii_engine* e, const int32_t* shift_in, const int32_t* shift_out);

/* Incremental (cached) decoding, bit-exact with recomputation.  No reference counterpart: the
 * reference recomputes the whole prefix (python/intref.py:288-301) and lists cached decoding as
 * open work.  A decoder holds, per layer, the post-RoPE k and v rows [n_seq][max_T][192] of its
 * sequences (max_T <= 512, the RoPE table length).  eii_decoder_prefill runs the forward pass on
 * T0 prompt tokens per sequence (outputs as eii_forward: logits [n_seq][T0][49152], digests) and
 * fills the cache; each eii_decoder_step then takes one token per sequence (ids [n_seq]) at the
 * current position t and returns its logits row [n_seq][49152] and/or per-sequence digests with
 * position weight t.  The logits of step t equal row t of eii_forward on the first t + 1 tokens,
 * and the prefill and step digests add up (mod 2^64) to the eii_forward digest of the whole
 * sequence.  Decoding may also start at position 0 without a prefill.  The decoder uses the
 * engine's stream and workspace: calls on one engine (and its decoders) are serialised, and the
 * engine must outlive its decoders. */
typedef struct eii_decoder eii_decoder;
int eii_decoder_open(eii_engine* e, int n_seq, int max_T, eii_decoder** out);
int eii_decoder_prefill(eii_decoder* d, const int64_t* ids, int T0, int32_t* logits_out, uint64_t* digests);
int eii_decoder_step(eii_decoder* d, const int64_t* ids, int32_t* logits_out, uint64_t* digests);
/* Device pointers as in eii_forward_device (logits_dev rows of ld_logits elements). */
int eii_decoder_step_device(eii_decoder* d, const int64_t* ids_dev, int32_t* logits_dev, int64_t ld_logits,
                            uint64_t* digests_dev, void* stream);
/* The same step, returning once it is enqueued on `stream` (no synchronisation): a serving loop
 * issues its steps back to back and calls eii_decoder_sync when it needs the results.  Argument
 * errors are returned at once; device-side errors of the enqueued steps (a token id outside the
 * vocabulary, a bounded wait that ran out) are returned by the next eii_decoder_sync, after which
 * the cache contents are undefined (eii_decoder_reset and prefill again).  Consecutive steps of one
 * decoder must go to the same stream, or the caller orders them. */
int eii_decoder_step_device_async(eii_decoder* d, const int64_t* ids_dev, int32_t* logits_dev, int64_t ld_logits,
                                  uint64_t* digests_dev, void* stream);
/* Waits for the work on `stream` (null = the engine's stream) and reports a device-side error. */
int eii_decoder_sync(eii_decoder* d, void* stream);
int eii_decoder_position(const eii_decoder* d); /* tokens in the cache, -1 for a null decoder */
int eii_decoder_reset(eii_decoder* d);          /* back to position 0 (the cache is reused) */
void eii_decoder_close(eii_decoder* d);

/* Single steps for the drop-in Python Model (host int64 buffers, python/intref.py names). */

/* Model.embed (python/intref.py:163-166): ids [n] -> x [n][576]. */
int eii_embed(eii_engine* e, const int64_t* ids, int n, int64_t* x_out);

/* Model.block (python/intref.py:192-286) for layer `layer` on n_seq sequences of T rows:
 * x_in, x_out [n_seq*T][576] (may alias). */
int eii_block(eii_engine* e, int layer, const int64_t* x_in, int n_seq, int T, int64_t* x_out);

/* Model.block(l, x, trace) (python/intref.py:192-286): layer `layer` on one sequence of T rows
 * (x_in [T][576]) with every per-site value of the reference's trace, as int64 (any pointer may be
 * null).  Shapes: norm*_U [T]; attn_score, attn_prob [9][T][T] (zero above the diagonal, as the
 * reference stores them); k_proj, v_proj, k_rope [T][192]; gate_proj, up_proj, silu_gate,
 * mlp_gated [T][1536]; the rest [T][576].  The exponents of the sites are the layer's formats
 * (python/intref.py:285-286). */
typedef struct eii_trace {
    int64_t *resid_in, *norm1_U, *norm1_z, *norm1_out, *q_proj, *k_proj, *v_proj, *q_rope, *k_rope;
    int64_t *attn_score, *attn_prob, *attn_ctx, *o_res, *resid_mid, *norm2_U, *norm2_z, *norm2_out;
    int64_t *gate_proj, *up_proj, *silu_gate, *mlp_gated, *down_res, *resid_out;
} eii_trace;
int eii_block_trace(eii_engine* e, int layer, const int64_t* x_in, int T, eii_trace* trace);

/* Model.rmsnorm (python/intref.py:168-184) with an explicit gain (q int16-valued [576], f):
 * x [rows][576] int32-valued -> out [rows][576]; bits_out 16 or 32. */
int eii_rmsnorm(eii_engine* e, const int64_t* x, int rows, const int64_t* gain_q, int gain_f, int f_out,
                int bits_out, int64_t* out);
/* Model.rmsnorm(x, gain, f_out, bits_out, trace) (python/intref.py:168-184): as eii_rmsnorm, plus the
 * trace values U [rows] (the exact reciprocal root) and z [rows][576] = RS(x U, 16); either may be null. */
int eii_rmsnorm_trace(eii_engine* e, const int64_t* x, int rows, const int64_t* gain_q, int gain_f, int f_out,
                      int bits_out, int64_t* out, int64_t* U_out, int64_t* z_out);

/* Final norm + tied logits (python/intref.py:296-300): x [rows][576] -> logits [rows][49152]
 * int64 (f = 16, no saturation). */
int eii_logits(eii_engine* e, const int64_t* x, int rows, int64_t* logits);

/* Model.linear (python/intref.py:186-190): out = SAT(RS(acc * m, n + f_in - f_out), bits_out),
 * acc = a W^T exact.  a [M][K] with values in signed bits_in (16 or 32), W int8 [N][K], m/n [N].
 * bits_out 64 means no saturation.  out and acc are int64 [M][N]; acc may be null.
 * K must be a multiple of 32 and <= 1536 (the proven int32 plane-accumulator range);
 * N a multiple of 16.  Works on any handle (the weights are uploaded per call). */
int eii_linear(eii_engine* e, const int64_t* a, int M, int K, int bits_in, const int8_t* W, const int64_t* m,
               const int64_t* n, int N, int f_in, int f_out, int bits_out, int64_t* out, int64_t* acc);

/* Device-resident Model.linear (python/intref.py:186-190) with the weights bound once: the path of
 * the stand-alone contraction sweep (int8 weights x wide activations at M up to 262144 rows).
 * eii_linear_plan_open uploads W int8 [N][K] and the per-column (m, n + f_in - f_out) table (m, n
 * host int64 [N]) to the handle's device; N a multiple of 16 up to 49152, K a multiple of 32 up to
 * 1536, bits_in 16 or 32, bits_out <= 32.  eii_linear_plan_run then computes, on device buffers,
 *   out_dev[r * ld_out + c] = SAT_bits_out(RS(acc[r][c] * m[c], n[c] + f_in - f_out)),  int32,
 *   acc = a_dev W^T exact,  a_dev int32 [M][K] (values within signed bits_in, else EII_ERR_ARG),
 * and, when the pointers are not null, per-row digests (uint64 [M], zeroed by the call)
 *   dig_out_dev[r] = sum_c uint32(out[r][c]) * mix64(2^32 + c),
 *   dig_acc_dev[r] = sum_c uint64(acc[r][c]) * mix64(2^32 + c)      (mod 2^64)
 * with mix64 the digest weight of eii_forward, so a caller can check an M x N result (51.5 GB at
 * M = 262144, N = 49152) and its exact int64 accumulators without copying them.  a_dev and out_dev
 * must be 16-byte aligned and ld_out a multiple of 4.  `stream` is a cudaStream_t (null = the
 * handle's stream); the call returns once the work is complete.  The plan owns a byte-plane
 * workspace of (bits_in / 8) * M * K bytes, grown on demand; calls on a plan and its engine are
 * serialised by the caller.  No reference counterpart as an API (the reference's linear is the
 * numpy Model.linear on host arrays; eii_linear is its host-buffer drop-in). */
typedef struct eii_linear_plan eii_linear_plan;
int eii_linear_plan_open(eii_engine* e, const int8_t* W, const int64_t* m, const int64_t* n, int N, int K,
                         int bits_in, int f_in, int f_out, int bits_out, eii_linear_plan** out);
int eii_linear_plan_run(eii_linear_plan* p, const int32_t* a_dev, int M, int32_t* out_dev, int64_t ld_out,
                        uint64_t* dig_out_dev, uint64_t* dig_acc_dev, void* stream);
void eii_linear_plan_close(eii_linear_plan* p);

/* Allocation-free linear: the same contraction and requantisation as eii_linear, for callers that
 * must not allocate device memory -- code whose device memory is owned by another allocator (a
 * framework or serving runtime that reserved the GPU up front) or that cannot afford the implicit
 * synchronisation of cudaMalloc/cudaFree in a latency-critical loop.  It calls no cudaMalloc,
 * cudaFree or other allocating routine and needs no engine handle.  No counterpart in the
 * reference.
 *   All pointers are device pointers on the CURRENT device: a_dev int64 [M][K] (values within
 *   signed bits_in, 16 or 32; a value outside it, or a column shift n + f_in - f_out outside
 *   [1, 62], is reported as EII_ERR_ARG after the call has run), w_dev int8 [N][K] (16-byte
 *   aligned), m_dev and n_dev int64 [N],
 *   out_dev int64 [M][N], acc_dev int64 [M][N] or null.  `stream` is a cudaStream_t (null = the
 *   legacy default stream); the call returns after the work on it has finished.
 *   Scratch: the activation byte planes, the per-column multiplier/shift table and an error word
 *   live in fixed __device__ arrays of this library (about 16.4 MB that every GPU loading the
 *   library holds until the process exits).  Limits: (bits_in / 8) * M * K <= EII_NOALLOC_PLANE_BYTES,
 *   N <= EII_NOALLOC_MAX_N, K a multiple of 32 up to 1536, N a multiple of 16; larger sizes are
 *   rejected with EII_ERR_ARG.
 *   Every call reads its error word back and synchronises `stream` before it returns, so no call
 *   can be captured into a CUDA graph.  The first call on a device also resolves the scratch
 *   addresses for that device (cudaGetSymbolAddress).  Every call shares the same scratch: calls
 *   that overlap on the GPU (different streams or threads at the same time) race and must be
 *   serialised by the caller. */
#define EII_NOALLOC_PLANE_BYTES (16u * 1024u * 1024u)
#define EII_NOALLOC_MAX_N 49152
int eii_linear_noalloc(const int64_t* a_dev, int M, int K, int bits_in, const int8_t* w_dev, const int64_t* m_dev,
                       const int64_t* n_dev, int N, int f_in, int f_out, int bits_out, int64_t* out_dev,
                       int64_t* acc_dev, void* stream);

/* Per-kernel timing.  While enabled, every launch of the engine is bracketed by CUDA events on
 * its stream (this adds a few microseconds per launch, so time whole runs with it off).
 * eii_profile_enable resets the counters; eii_profile_read returns the summed device time (ms)
 * and the launch count of one kernel kind.  No reference counterpart: the reference times only
 * whole runs (c/intref.c:225,256, cuda/intref.cu:283,302-304). */
#define EII_K_EMBED 0
#define EII_K_NORM 1
#define EII_K_GEMM_QKV 2
#define EII_K_ATTENTION 3
#define EII_K_GEMM_O 4
#define EII_K_GEMM_GATEUP 5
#define EII_K_GEMM_DOWN 6
#define EII_K_GEMM_LOGITS 7
#define EII_K_DIGEST 8 /* no launches: the digest is fused into the logits GEMM */
#define EII_K_GEMM_LINEAR 9
#define EII_K_SPLIT_PLANES 10 /* int32 activations -> byte planes (eii_linear_plan_run) */
#define EII_K_GEMM_SWEEP 11   /* the contraction of eii_linear_plan_run */
#define EII_NUM_KERNEL_KINDS 12
const char* eii_kernel_name(int kind);
int eii_profile_enable(eii_engine* e, int on);
int eii_profile_read(eii_engine* e, int kind, double* total_ms, int64_t* launches);

/* Sequences per chunk that eii_forward / eii_forward_device use for n_seq sequences of T tokens
 * (the engine works through the sequences in chunks of its device workspace).  The sequences are
 * split into the fewest chunks of at most 65536 rows, all of (nearly) equal size; the environment
 * variable EII_CHUNK_ROWS=R sets chunks of exactly R / T sequences instead.  Returns the count, or
 * minus an error code for a null engine or a non-positive size.  No reference counterpart (the
 * reference runs one sequence at a time). */
int eii_chunk_sequences(const eii_engine* e, int n_seq, int T);

/* Measurement probe (no reference counterpart): cycles per tcgen05.mma.kind::i8 of M = 128, N = n,
 * K = 32 from shared-memory operands, issued back to back by one thread per SM on every SM of
 * `device`, while warps 4 .. threads/32 - 1 of each CTA run background work `noise` (0 none,
 * 1 shared-memory loads, 2 TMEM loads, 3 64-bit multiply-adds, 4 global stores, 5 32-bit IMAD,
 * 6 FFMA, 7 integer ALU, 8 32x32->64 multiply-accumulate, 9 shared-memory stores, 10 cp.async global ->
 * shared copies, 11 cp.async.bulk global -> shared copies).  n a multiple of 16 in [16, 256];
 * threads 128, 256 or 640; iters in [1, 100000] (4 MMAs each).  The numbers behind the GEMMs' tile
 * shapes (bench.py --probe-mma). */
int eii_mma_rate(int device, int n, int noise, int threads, int iters, double* cycles_per_mma);

#ifdef __cplusplus
}
#endif
#endif /* EII_H */
