/*
 * g4b.h -- C ABI of the B200 (sm_100a) int4/int8 quantized-weight matmul library.
 *
 * Drop-in for the quantized-weight dispatches of gemma4-adreno's Vulkan engine
 * (src/vk_engine.py).  The reference binds these kernels through Vulkan
 * descriptor sets plus a std140 uniform; each entry point below replaces one
 * such dispatch (or dispatch pair) and takes the same buffers and sizes as plain
 * device pointers.  Every reference citation is file:line within the reference
 * project.
 *
 * Conventions (all entry points):
 *   - All array pointers are DEVICE pointers owned by the caller.  Calls are
 *     stream-ordered and asynchronous on `stream` (NULL = the legacy default
 *     stream); none synchronises the device or allocates device memory.
 *   - Return 0 (G4B_OK) on success, a negative G4B_E_* code otherwise.  On
 *     error nothing was launched and g4b_last_error() (per host thread) says why.
 *   - Layouts are the reference's packing layout (src/vk_engine.py:125-159):
 *       wp      [K, N/8] uint32, nibble j of word (k, g) = column 8g+j, value q in
 *               [0,15] standing for the weight (q - 8) * scale
 *       scales  [K/32, N] f16 (G4B_SCALE_F16) or e4m3 bytes (G4B_SCALE_E4M3)
 *       int8 W  [K, N] int8, row-major (the W8A8 prefill weights)
 *     Activations are row-major [M, K]; outputs row-major [M, N].
 *   - Pointers must be 16-byte aligned; N % 16 == 0; K % 32 == 0 (one scale
 *     block), as the reference requires (src/vk_engine.py:126, 219).
 *   - Thread safety: calls on distinct streams from distinct host threads are
 *     safe; a workspace must not be shared by calls that can overlap on the GPU.
 */
#ifndef G4B_H
#define G4B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* exported symbols (the library is built with hidden visibility otherwise) */
#if defined(G4B_BUILDING) && defined(__GNUC__)
#define G4B_API __attribute__((visibility("default")))
#else
#define G4B_API
#endif

/* cudaStream_t without pulling in the CUDA headers */
typedef struct CUstream_st* g4b_stream_t;

/* ----------------------------------------------------------------- status */
#define G4B_OK                 0
#define G4B_E_SHAPE           -1  /* unsupported or inconsistent sizes          */
#define G4B_E_ALIGN           -2  /* a pointer is not 16-byte aligned            */
#define G4B_E_ARCH            -3  /* current device is not an sm_100 GPU         */
#define G4B_E_CUDA            -4  /* a CUDA runtime call failed                  */
#define G4B_E_FAULT_INJECTED  -5  /* G4B_FAULT asked this call to fail           */
#define G4B_E_ARG             -6  /* bad enum value or NULL pointer              */
#define G4B_E_WORKSPACE       -7  /* workspace missing or too small              */
#define G4B_E_TIMEOUT         -8  /* g4b_stream_wait gave up                     */

/* ------------------------------------------------------------- enumerations */
#define G4B_DT_F32  0
#define G4B_DT_F16  1

#define G4B_SCALE_F16   0   /* scales [K/32, N] f16: the reference's default          */
#define G4B_SCALE_E4M3  1   /* scales [K/32, N] float8 e4m3fn bytes (GEMV_FP8=1)       */

/* g4b_query() selectors */
#define G4B_Q_VERSION        0  /* library version, major*10000 + minor*100 + patch */
#define G4B_Q_DEVICE_OK      1  /* 1 if the current device can run the kernels     */
#define G4B_Q_SM_COUNT       2  /* streaming multiprocessors on the current device */
#define G4B_Q_LAUNCHES       3  /* kernels this process has launched through g4b   */
#define G4B_Q_FAULT_COUNTER  4  /* calls seen by the fault injector                */
#define G4B_Q_KERNEL_STATUS  5  /* read-and-clear the kernels' device status word:
                                   0 = clean, 1 = a bounded wait timed out (the
                                   kernel gave up and its outputs are invalid);
                                   synchronises the device */

/* --------------------------------------------------------------- utilities */
/* Message for the last failing call on this host thread ("" if none). */
G4B_API const char* g4b_last_error(void);

/* Library version as major*10000 + minor*100 + patch. */
G4B_API int g4b_version(void);

/* Integer facts about the library and the current device (G4B_Q_*); -1 on error. */
G4B_API long long g4b_query(int what);

/* Wait for all work queued on `stream` with a host-side time limit, the
 * counterpart of the engine's fence wait with GEMMA4_FENCE_TIMEOUT_MS
 * (src/vk_engine.py:294-302).  timeout_ms <= 0 waits without limit.
 * Returns G4B_E_TIMEOUT (work still running) or G4B_E_CUDA (the stream failed). */
G4B_API int g4b_stream_wait(g4b_stream_t stream, int timeout_ms);

/* ------------------------------------------------------------ decode GEMV */
/* Bytes of workspace g4b_gemv_i4 needs for these sizes.  `split` as passed to
 * g4b_gemv_i4 (0 = the library chooses).  0 means no workspace is needed. */
G4B_API size_t g4b_gemv_workspace_bytes(int M, int N, int K, int split);

/* int4 block-scaled GEMV (M = 1) or small-batch GEMM (M <= 8 tokens):
 *     y[m, n] = sum_k x[m, k] * (q[k, n] - 8) * scale[k/32, n]   (* inv for e4m3)
 * Replaces one gemv (+ reduce) dispatch pair recorded by gemv() with the
 * descriptor set from gemv_ds() (src/vk_engine.py:214-226, 270-272): the
 * shaders vk/gemv.comp:11-33, vk/gemv_fp8.comp:20-40 and vk/reduce.comp:8-12.
 *   x        [M, K] f32 or f16 (x_dtype)
 *   scales   f16 or e4m3 per scale_fmt; inv is the e4m3 scales' 2^-shift
 *            (ignored for f16 scales), the uniform's e.x in the reference
 *   y        [M, N] f32 or f16 (y_dtype); f32 accumulation throughout
 *   split    number of K-slices (must divide K/32), the reference's `split`
 *            from quant(); 0 lets the library pick one for the B200's SMs
 *   workspace  device scratch of g4b_gemv_workspace_bytes() bytes (NULL if that
 *            is 0), zero-filled once when allocated: it holds the K-slice
 *            partial sums and per-tile arrival counters, and every call leaves
 *            the counters at zero again.
 * The K-slice partials are summed in slice order, so results are deterministic. */
G4B_API int g4b_gemv_i4(const void* x, int x_dtype, int M,
                const uint32_t* wp, const void* scales, int scale_fmt, float inv,
                void* y, int y_dtype, int N, int K, int split,
                void* workspace, size_t ws_bytes, g4b_stream_t stream);

/* g4b_gemv_i4 with launch flags:
 *   G4B_GEMV_PDL  programmatic dependent launch: the kernel may start while the
 *                 previous kernel in `stream` is still running and begins
 *                 streaming wp/scales at once; it reads x and writes y and the
 *                 workspace only after that kernel has completed.  Use it when
 *                 the preceding kernel does not write wp or scales (a decode
 *                 step's chain of GEMVs): it hides launch latency and the
 *                 previous kernel's tail.  Captured into CUDA graphs as a
 *                 programmatic edge.
 * flags == 0 behaves exactly as g4b_gemv_i4. */
#define G4B_GEMV_PDL 1u
G4B_API int g4b_gemv_i4_ex(const void* x, int x_dtype, int M,
                   const uint32_t* wp, const void* scales, int scale_fmt, float inv,
                   void* y, int y_dtype, int N, int K, int split,
                   void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream);

/* g4b_gemv_i4 for callers that cannot allocate device memory: no workspace
 * argument.  This entry point has no counterpart in the reference (whose
 * engine owns all its buffers); it exists for hosts that may not call
 * cudaMalloc on the decode path -- e.g. code running inside a CUDA-graph
 * capture or under a custom allocator that forbids allocation after
 * start-up, or a plugin handed only input and output buffers.
 *   - The split-K scratch lives in a fixed 4 MiB array inside the library,
 *     held on every GPU that loads it until the process exits.  Sizes that
 *     need more (g4b_gemv_workspace_bytes() > 4 MiB, e.g. M = 8 tokens of a
 *     15360-wide GEMV) are rejected with G4B_E_WORKSPACE before anything runs.
 *   - The first call on each device looks the array's address up
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - Every accepted call enqueues a small memset of the array's counters,
 *     then the same kernel as g4b_gemv_i4; nothing is allocated or freed.
 *     Arguments are checked first: a rejected call enqueues nothing.
 *   - All calls share the one array, which keeps the last call's contents:
 *     calls that can overlap on the GPU (different streams, or concurrent
 *     host threads without ordering) race on it.  Serialise them on one stream. */
G4B_API int g4b_gemv_i4_noalloc(const void* x, int x_dtype, int M,
                        const uint32_t* wp, const void* scales, int scale_fmt, float inv,
                        void* y, int y_dtype, int N, int K, int split, g4b_stream_t stream);

/* One GEMV of a fused launch (g4b_gemv_i4_fused): packed words [K, N/8],
 * scales [K/32, N] (f16 or e4m3 per the call's scale_fmt), the e4m3 inverse
 * scale 2^-shift (ignored for f16 scales) and the output y [N]. */
typedef struct g4b_gemv_segment {
    const uint32_t* wp;
    const void* scales;
    float inv;
    void* y;
    int N;
} g4b_gemv_segment;

/* Workspace bytes for g4b_gemv_i4_fused over segments of these widths. */
G4B_API size_t g4b_gemv_fused_workspace_bytes(int nseg, const int* Ns, int K);

/* Up to three M = 1 GEMVs that read the same x in one launch: the engine's
 * consecutive gemv() dispatches on one input buffer -- q, k, v on the normed
 * hidden state, then gate and up (src/vk_engine.py:280-284; each a
 * vk/gemv.comp or vk/gemv_fp8.comp dispatch with its reduce).  Every
 * segment's result is what g4b_gemv_i4 would give it alone, up to f32
 * summation order; the work of all segments is spread over the SMs as one
 * grid, so the small k/v GEMVs do not each pay a launch and a ramp.
 *   x [K] f32 or f16; each segment N % 32 == 0; K % 64 == 0; 1 <= nseg <= 3.
 *   flags: 0 or G4B_GEMV_PDL (as g4b_gemv_i4_ex). */
G4B_API int g4b_gemv_i4_fused(const void* x, int x_dtype, int nseg, const g4b_gemv_segment* segs, int scale_fmt,
                              int y_dtype, int K, void* workspace, size_t ws_bytes, unsigned flags,
                              g4b_stream_t stream);

/* A recorded chain of M = 1 GEMV steps run by ONE persistent launch: the
 * engine's per-token command buffer of gemv() dispatches with a barrier after
 * each (src/vk_engine.py:254-290, bar() at :261).  Step j may read what any
 * earlier step wrote; a step starts reading x only after every column tile of
 * the step before it has been written.  The weight stream does not wait: a
 * step's packed words and scales are in flight while the previous step
 * finishes.  Each step's y equals g4b_gemv_i4_fused (or g4b_gemv_i4) on the
 * same x up to f32 summation order; one chain gives the same bits every run.
 *
 *   create   validates the steps, encodes their TMA descriptors, picks each
 *            step's partition of work over the SMs and copies the plan to
 *            device memory (setup time: allocates and synchronises); all steps
 *            share x_dtype, scale_fmt and y_dtype; per step 1 <= nseg <= 3,
 *            K % 256 == 0, every N % 32 == 0, x and the weights 16-byte
 *            aligned.  The buffers named in the steps must stay allocated
 *            while the chain is used.
 *   run      one launch on `stream` (cooperative: every CTA resident); the
 *            workspace (g4b_gemv_chain_workspace_bytes, 16-byte aligned) is
 *            zero-filled once before first use.  Never allocates or
 *            synchronises; capturable in a CUDA graph.  A step whose x is the
 *            step before's first output (same dtype, no element-wise work)
 *            receives it slice by slice as forwarded words in the workspace
 *            instead of waiting for the whole step; the results are the same
 *            bits (G4B_CHAIN_FORWARD=0 in the environment at create turns it
 *            off).
 *   destroy  frees the plan.
 *
 * Tensor parallel (create_tp): a step flagged G4B_CHAIN_ALLREDUCE (one
 * segment: a row-parallel o / down shard) has its y summed over the `world`
 * ranks inside the launch -- the cross-GPU counterpart of vk/reduce.comp:8-12.
 * Every y value it writes is also stored, paired with the run's epoch in one
 * 64-bit word, into slot [rank] of that all-reduce's region of every rank's
 * exchange buffer (NVLink peer stores); the next step (K = that N; its x is
 * ignored) reads each 256-row slice of x as the rank-order sum of the world
 * slots once every word carries the epoch.  peers_dev is a device array of the
 * world exchange buffers (this rank's own at [rank]: g4b_comm_alloc, mapped
 * with g4b_ipc_open), each g4b_gemv_chain_exchange_bytes long and zero-filled
 * once; every rank runs the same chain the same number of times.  Waits are
 * bounded (2 s, then the kernel status word is raised). */
#define G4B_CHAIN_ALLREDUCE 1u
typedef struct g4b_gemv_chain g4b_gemv_chain;
typedef struct g4b_gemv_chain_step {
    const void* x;                 /* [K] activations of this step (ignored after an all-reduced step) */
    int K;
    int nseg;
    g4b_gemv_segment seg[3];
    unsigned flags;                /* 0 or G4B_CHAIN_ALLREDUCE */
} g4b_gemv_chain_step;

G4B_API int g4b_gemv_chain_create(const g4b_gemv_chain_step* steps, int nsteps, int x_dtype, int scale_fmt,
                                  int y_dtype, g4b_gemv_chain** chain);
G4B_API size_t g4b_gemv_chain_exchange_bytes(const g4b_gemv_chain_step* steps, int nsteps, int world);
G4B_API int g4b_gemv_chain_create_tp(const g4b_gemv_chain_step* steps, int nsteps, int x_dtype, int scale_fmt,
                                     int y_dtype, void* const* peers_dev, int rank, int world,
                                     size_t exchange_bytes, g4b_gemv_chain** chain);
/* Element-wise work fused into a chain step's activation load: the engine's
 * rmsnorm / normadd / gelumul dispatches between a decode layer's GEMVs
 * (descriptor sets src/vk_engine.py:232, 243-251; dispatches :278-287).  Step j's x
 * is then computed from the vectors below instead of read from step.x (which
 * may be NULL); f32 arithmetic, K elements:
 *   G4B_XF_RMSNORM   x = a * rsqrt(sum(a^2) / K + eps) * w          vk/rmsnorm.comp:8-12
 *   G4B_XF_NORMADD   h' = (b + a * rsqrt(sum(a^2) / K + eps) * w_post) * scale
 *                    x  = h' * rsqrt(sum(h'^2) / K + eps) * w       vk/normadd.comp:8-12,
 *                    and h' is stored to h_out                      then vk/rmsnorm.comp
 *   G4B_XF_GELU_MUL  x = 0.5 a (1 + tanh(0.7978845608 (a + 0.044715 a^3))) * b
 *                                                                   vk/gelumul.comp:7-8
 * Vectors and dtypes: a is step j-1's first output y (chain y dtype) -- for
 * RMSNORM it may instead be a vector no step writes (f32: the token's input
 * hidden state); b is the residual h (f32) for NORMADD, step
 * j-1's `up` output (y dtype) for GELU_MUL; w, w_post (norm weights) and
 * h_out are f32.  All 16-byte aligned; h_out must not overlap b.
 * The sums come from step j-1's tile writers (per-tile partial sums, added in
 * a fixed order, so a chain gives the same bits every run); the squares of h'
 * are expanded as scale^2 (sum b^2 + 2 r sum b (a w_post) + r^2 sum (a w_post)^2)
 * with r = rsqrt(sum(a^2) / K + eps).  One rank only (no G4B_CHAIN_ALLREDUCE
 * next to a fused step). */
#define G4B_XF_NONE      0
#define G4B_XF_RMSNORM   1
#define G4B_XF_NORMADD   2
#define G4B_XF_GELU_MUL  3
typedef struct g4b_chain_xform {
    int kind;              /* G4B_XF_* */
    const void* a;
    const void* b;
    const float* w;
    const float* w_post;
    float* h_out;
    float scale;           /* NORMADD: the layer scalar (vk/normadd.comp's d.y; 1 = none) */
    float eps;             /* 1e-6 in the reference */
} g4b_chain_xform;

/* g4b_gemv_chain_create with one g4b_chain_xform per step (kind G4B_XF_NONE:
 * the step reads step.x as usual): a decode token's GEMVs and the element-wise
 * work between them as one launch. */
G4B_API int g4b_gemv_chain_create_fused(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xforms, int nsteps,
                                        int x_dtype, int scale_fmt, int y_dtype, g4b_gemv_chain** chain);

/* The chain's plan for where each step's x comes from, as g4b_gemv_chain_create*
 * decides it, on the host only (no device, nothing allocated; no counterpart in
 * the reference -- it exposes the barrier decisions for tests and tooling):
 *   x_forwarded  x is the step before's first output read as forwarded words
 *                (same dtype, no element-wise work, no all-reduce between them,
 *                and the step's outputs overlap nothing the step before reads
 *                from memory or writes);
 *   wait_from    the first step whose completion its x load waits for (it
 *                waits for wait_from .. j-1 unless x is forwarded or
 *                all-reduced);
 *   x_early      x is written by no step, and its first slice is loaded
 *                before that wait.
 * xforms may be NULL.  out has nsteps entries. */
typedef struct g4b_chain_step_plan {
    int x_forwarded;
    int wait_from;
    int x_early;
    int reserved;
} g4b_chain_step_plan;
G4B_API int g4b_gemv_chain_plan(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xforms, int nsteps,
                                int x_dtype, int y_dtype, g4b_chain_step_plan* out);
G4B_API size_t g4b_gemv_chain_workspace_bytes(const g4b_gemv_chain* chain);
G4B_API int g4b_gemv_chain_run(const g4b_gemv_chain* chain, void* workspace, size_t ws_bytes, g4b_stream_t stream);
/* g4b_gemv_chain_run with launch flags:
 *   G4B_CHAIN_RUN_PDL  programmatic dependent launch: the chain may start while
 *                      the previous kernel in `stream` is still running and
 *                      begins streaming its weights at once; it reads its first
 *                      x, and writes anything, only after that kernel has
 *                      completed.  For a decode token split at attention: the
 *                      next layer's weights stream while attention runs.  The
 *                      chain itself lets a programmatic dependent after it
 *                      start early (g4b_attn_decode* is launched that way). */
#define G4B_CHAIN_RUN_PDL 1u
G4B_API int g4b_gemv_chain_run_ex(const g4b_gemv_chain* chain, void* workspace, size_t ws_bytes, unsigned flags,
                                  g4b_stream_t stream);
G4B_API void g4b_gemv_chain_destroy(g4b_gemv_chain* chain);

/* Split-K partial reduction, vk/reduce.comp:8-12:
 *     y[n] = sum_{c=0}^{split-1} partial[c*N + n]   (c ascending, f32)
 * Exposed on its own for parity with the reference's reduce dispatch
 * (src/vk_engine.py:223-226, 272); g4b_gemv_i4 performs it internally. */
G4B_API int g4b_reduce_partials(const float* partial, float* y, int N, int split, g4b_stream_t stream);

/* Dequantise packed int4 weights to a dense [K, N] matrix:
 *   out_dtype F16, scale_fmt F16 : f16((q - 8) * f32(scale))  -- bit-exact the
 *       tile vk/coopgemm_i4h.comp:19-25 writes to shared memory
 *   out_dtype F32                : (q - 8) * f32(scale), exact in f32
 * With scale_fmt E4M3 the scale is decoded as vk/gemv_fp8.comp:14-18 and the
 * product is multiplied by inv (a power of two, so still exact). */
G4B_API int g4b_dequant_i4(const uint32_t* wp, const void* scales, int scale_fmt, float inv,
                   void* out, int out_dtype, int N, int K, g4b_stream_t stream);

/* ------------------------------------------------------------ weight packing */
/* The engine's int4 packing, quant() (src/vk_engine.py:126-131), on the GPU,
 * bit-exact to the host packer:  W [N, K] f32 (row-major, HF layout) ->
 *   scale[n, b] = max(max_{k in block b} |W[n,k]| / 7, 1e-8)           (f32)
 *   q = clip(round_half_even(W / scale) + 8, 0, 15) packed into wp [K, N/8]
 *   scales_f16 [K/32, N] = f16(scale)
 * scales_f32 (nullable) receives the f32 scales as [N, K/32] (the input of
 * g4b_quant_e4m3 / g4b_quant_w8a8); amax_bits (nullable, initialised by the
 * caller to 0) receives atomicMax of the scales' f32 bit patterns: the
 * tensor-wide max scale the e4m3 shift is computed from.  N % 8, K % 32. */
G4B_API int g4b_quant_i4(const float* W, int N, int K, uint32_t* wp, uint16_t* scales_f16,
                         float* scales_f32, uint32_t* amax_bits, g4b_stream_t stream);

/* e4m3 scales for GEMV_FP8 (src/vk_engine.py:133-137): with the caller's
 * shift = floor(log2(256 / max scale)) (inv = 2^-shift),
 *   scales_e4m3[b, n] = e4m3_rne(clip(scale[n, b] * 2^shift, 0, 448))
 * scales_f32 is the [N, K/32] output of g4b_quant_i4. */
G4B_API int g4b_quant_e4m3(const float* scales_f32, int N, int K, int shift, uint8_t* scales_e4m3,
                           g4b_stream_t stream);

/* W8A8 prefill weights (src/vk_engine.py:152-157) from the packed int4 ones:
 *   deq = (q - 8) * scale (f32);  s_w[n] = max(max_k |deq[n,k]| / 127, 1e-12)
 *   w8 [K, N] int8 = clip(round_half_even(deq / s_w), -127, 127);  sw_f16 = f16(s_w)
 * sw_f32 (nullable) receives s_w; ratio_f16 (nullable, [K/32, N]) receives the
 * W4A8 requant ratio f16(scale / s_w) (benchmarks/coopgemm_w4a8.py:84). */
G4B_API int g4b_quant_w8a8(const uint32_t* wp, const float* scales_f32, int N, int K, int8_t* w8,
                           uint16_t* sw_f16, float* sw_f32, uint16_t* ratio_f16, g4b_stream_t stream);

/* ------------------------------------------------------------ prefill path */
/* Element-wise f32 <-> f16 conversion (round-to-nearest-even), the engine's
 * vk/cast_dn.comp:7 (f32 -> f16) and vk/cast_up.comp:7 (f16 -> f32) dispatches
 * around each prefill GEMM (src/vk_engine.py:398-400). */
G4B_API int g4b_cast(const void* src, int src_dtype, void* dst, int dst_dtype, size_t n, g4b_stream_t stream);

/* Per-token int8 activation quantiser, vk/cast_i8.comp:11-19 (dispatched by
 * gmm() under PREFILL_I8, src/vk_engine.py:392-394):
 *     s = max(max_k |X[m,k]| / 127, 1e-12);  inv = 1/s  (both correctly rounded)
 *     A8[m,k] = clamp(round_half_even(X[m,k] * inv), -127, 127);  sa[m] = s   */
G4B_API int g4b_cast_i8(const void* X, int x_dtype, int8_t* A8, float* sa, int M, int K, g4b_stream_t stream);

/* ---------------------------------------------------------------- prefill GEMMs */

/* Bytes of workspace g4b_gemm_i4 can use for these sizes: the f16 copy of an
 * f32 X (the cast_dn step; required for f32 X), plus, for small M whose
 * column tiles cannot fill the SMs (batched decode), the f32 partials of a
 * K split across the SMs.  With a smaller workspace -- or none, for f16 X --
 * the GEMM runs without the split; the result is the same up to f32
 * summation order. */
G4B_API size_t g4b_gemm_i4_workspace_bytes(int M, int N, int K, int x_dtype);

/* W4A16 prefill GEMM with in-kernel dequantisation: vk/coopgemm_i4h.comp:13-35
 * (the engine's path), vk/coopgemm_i4.comp:14-36 and vk/coopgemm_i4f.comp:12-35,
 * dispatched by gmm() (src/vk_engine.py:391-400) between cast_dn and cast_up:
 *     Y[m, n] = sum_k f16(X[m, k]) * f16((q[k, n] - 8) * f32(scale[k/32, n]))
 * wp / scales_f16 are quant()'s packed words and f16 block scales (the
 * prefill path always uses f16 scales, src/vk_engine.py:150).  The
 * dequantised weights are bit-identical to the shader's; the accumulator is
 * f32 (the i4h shader accumulates in f16).  X [M, K] f16 or f32 (f32 is
 * converted to f16 in `workspace`, RNE, as cast_dn does); Y [M, N] f16 or f32.
 * M >= 1 (any), N % 128 == 0, K % 64 == 0; pointers 16-byte aligned.  M <= 64
 * runs 64-token tiles; a K split (see g4b_gemm_i4_workspace_bytes) adds a
 * second launch that sums the splits' partials in split order. */
G4B_API int g4b_gemm_i4(const void* X, int x_dtype, const uint32_t* wp, const uint16_t* scales_f16,
                        void* Y, int y_dtype, int M, int N, int K,
                        void* workspace, size_t ws_bytes, g4b_stream_t stream);
/* g4b_gemm_i4 with launch flags:
 *   G4B_GEMM_PDL  programmatic dependent launch: the GEMM may start while the
 *                 previous kernel in `stream` is still running; it prefetches
 *                 its first weight tiles into L2 and reads X, and writes Y or
 *                 the workspace, only after that kernel has completed.  For a
 *                 batched decode's chain of dependent GEMMs.  (The split-K sum
 *                 is always launched that way after its GEMM.)
 * flags == 0 behaves exactly as g4b_gemm_i4. */
#define G4B_GEMM_PDL 1u
G4B_API int g4b_gemm_i4_ex(const void* X, int x_dtype, const uint32_t* wp, const uint16_t* scales_f16,
                           void* Y, int y_dtype, int M, int N, int K,
                           void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream);

/* 2 or 3 W4A16 GEMMs on one X as one launch, for batched decode (M <= 64): a
 * layer's q, k and v, or gate and up -- the gemm_ds() calls the engine records
 * back to back on the same input (src/vk_engine.py:369-379).  Weight g writes
 * Y_g = X @ dequant(W_g) to segs[g].y [M, segs[g].N]; the column tiles of all
 * weights share the SMs and one split-K plan, whose workspace is
 * g4b_gemm_i4_workspace_bytes(M, sum of N, K, x_dtype).  Otherwise as
 * g4b_gemm_i4_ex (flags, dtypes, alignment). */
typedef struct {
    const uint32_t* wp;            /* packed words [K, N/8] */
    const uint16_t* scales_f16;    /* f16 block scales [K/32, N] */
    void* y;                       /* [M, N], y_dtype */
    int N;                         /* a multiple of 128 */
} g4b_gemm_seg;
G4B_API int g4b_gemm_i4_fused(const void* X, int x_dtype, int M, int K, const g4b_gemm_seg* segs, int nseg,
                              int y_dtype, void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream);

/* W8A8 prefill GEMM (PREFILL_I8), vk/coopgemm_w8a8.comp:18-37, dispatched by
 * gmm() after cast_i8 (src/vk_engine.py:391-397):
 *     C[m, n] = sum_k A8[m, k] * W8[k, n]                 (exact int32)
 *     Y[m, n] = f16((float(C) * sa[m]) * f32(sw_f16[n]))
 *   A8       [M, K] int8 and sa [M] f32: g4b_cast_i8's outputs
 *   W8       [K, N] int8 row-major and sw_f16 [N]: quant()'s prefill weights
 *            (src/vk_engine.py:152-157) -- used as they are, no repacking
 *   Y        [M, N] f16 or f32 (y_dtype; f32 skips the final f16 rounding)
 *   C_debug  nullable [M, N] int32: the raw accumulators, for exact checks
 * M >= 1, N % 16 == 0, K % 32 == 0.  A last wave of tiles that fills at most a
 * quarter of the SMs runs as quarter-height tiles (the same bits;
 * G4B_S8_QUARTER_TAIL=0 in the environment keeps whole tiles). */
G4B_API int g4b_gemm_w8a8(const int8_t* A8, const int8_t* W8, const float* sa, const uint16_t* sw_f16,
                          void* Y, int y_dtype, int32_t* C_debug, int M, int N, int K, g4b_stream_t stream);

/* W4A8 prefill GEMM, vk/coopgemm_w4a8.comp:21-50: the int4 weights are
 * requantised in the kernel against a per-column scale,
 *     W8[k, n] = clamp(round_half_even((q[k, n] - 8) * f32(ratio_f16[k/32, n])), -127, 127)
 * and then multiplied as g4b_gemm_w8a8 does.  ratio_f16 [K/32, N] is
 * f16(scale / s_w) (benchmarks/coopgemm_w4a8.py:84; g4b_quant_w8a8 makes it).
 * M >= 1, N % 32 == 0, K % 32 == 0. */
G4B_API int g4b_gemm_w4a8(const int8_t* A8, const uint32_t* wp, const uint16_t* ratio_f16, const float* sa,
                          const uint16_t* sw_f16, void* Y, int y_dtype, int32_t* C_debug,
                          int M, int N, int K, g4b_stream_t stream);

/* ------------------------------------------------------------ attention */
/* KV-cache write for one decode token, vk/prepkv.comp:14-31 (the prepkv dispatch
 * forward() records per layer, src/vk_engine.py:281): for every KV head h,
 *   k = RoPE(rmsnorm(qkv[koff + h*hd ..], knw))   with the token's rotation (cos_t, sin_t: [hd] f32),
 *   v = qkv[voff + h*hd ..] * rsqrt(mean(v^2) + 1e-6)          (keqv: v is read at koff instead)
 *   kc / vc [(h*stride + slot)*hd + i] = f16(k[i] / v[i]),  slot = window ? pos % window : pos
 * (sliding layers keep a ring of `window` slots).  qkv is the q|k|v output (f32 or f16); knw is f32;
 * pos is read from device memory (*pos_dev), so one captured graph serves every token.
 * hd 128, 256 or 512; window <= stride. */
G4B_API int g4b_attn_prepkv(const void* qkv, int dtype, const float* knw, const float* cos_t, const float* sin_t,
                            uint16_t* kc, uint16_t* vc, int nkv, int hd, int koff, int voff, int keqv, int stride,
                            int window, const int* pos_dev, g4b_stream_t stream);

/* Workspace bytes g4b_attn_decode needs for a cache of max_T keys (window, or stride for
 * full-attention layers); 0 when the keys are not split.  The workspace starts with one arrival
 * counter per KV head: zero-initialise it once; every call leaves the counters at zero, and calls
 * that share a workspace must be ordered (one stream). */
G4B_API size_t g4b_attn_workspace_bytes(int nH, int nkv, int hd, int max_T);

/* Decode attention for one token, vk/attn.comp:15-55 (the attn dispatch, src/vk_engine.py:282):
 * for every query head h (KV head h / (nH / nkv)),
 *   q = RoPE(rmsnorm(qkv[qoff + h*hd ..], qnw)),  T = window ? min(pos + 1, window) : pos + 1,
 *   out[h*hd + i] = sum_{j < T} softmax_j(q . k_j) v_j[i]            (no 1/sqrt(hd) scale, as the shader)
 * over the cached keys (slots 0 .. T-1).  The keys are split over the SMs (flash decoding): a
 * split's softmax partial goes to `workspace` and the last split of each KV head to finish
 * combines them (one launch).
 * Shapes: hd 128 (up to 8 query heads per KV head), 256 (up to 4) or 512 (up to 2).
 * out [nH, hd] f32 or f16. */
G4B_API int g4b_attn_decode(const void* qkv, int dtype, const float* qnw, const float* cos_t, const float* sin_t,
                            const uint16_t* kc, const uint16_t* vc, void* out, int out_dtype, int nH, int nkv,
                            int hd, int qoff, int stride, int window, const int* pos_dev, void* workspace,
                            size_t ws_bytes, g4b_stream_t stream);

/* The engine's prepkv and attn dispatches for one decode token in one launch: what
 * g4b_attn_prepkv then g4b_attn_decode compute, with the token's k / v written by the
 * CTA whose key split holds its slot before that CTA reads it.  Arguments as those two calls'. */
G4B_API int g4b_attn_decode_prepkv(const void* qkv, int dtype, const float* qnw, const float* knw,
                                   const float* cos_t, const float* sin_t, uint16_t* kc, uint16_t* vc, void* out,
                                   int out_dtype, int nH, int nkv, int hd, int qoff, int koff, int voff, int keqv,
                                   int stride, int window, const int* pos_dev, void* workspace, size_t ws_bytes,
                                   g4b_stream_t stream);

/* KV-cache write for a prefill chunk, vk/pre_prepkv.comp:15-30 (src/vk_engine.py:416): token m of
 * M (position *p0_dev + m) writes what g4b_attn_prepkv writes for one token, from its own rows
 * k + m*row_stride, v + m*row_stride (element offsets; head h at h*hd; k == v for attention_k_eq_v)
 * and its own rotation rows cosM / sinM [M, hd] f32.  On a sliding ring a chunk longer than the
 * window writes a slot more than once: the latest token's k / v stay.  Slots past the cache
 * (pos >= stride on a full-attention layer) are not written.  hd 128, 256 or 512. */
G4B_API int g4b_attn_prefill_prepkv(const void* k, const void* v, int dtype, int row_stride, int M,
                                    const float* knw, const float* cosM, const float* sinM, uint16_t* kc,
                                    uint16_t* vc, int nkv, int hd, int stride, int window, const int* p0_dev,
                                    g4b_stream_t stream);

/* Causal attention for a prefill chunk, vk/pre_attn.comp:16-53 (src/vk_engine.py:417): for token m
 * (position pos = *p0_dev + m) and query head h,
 *   q = RoPE(rmsnorm(q[m*q_stride + h*hd ..], qnw), cosM[m], sinM[m]),
 *   T = window ? min(pos + 1, window) : pos + 1,
 *   out[m*out_stride + h*hd + i] = sum_j softmax_j(q . k_j) v_j[i]  over the slots j < T, leaving out,
 *   on a sliding ring, the slots whose position (base - ((base + window - j) % window), base =
 *   *p0_dev + M - 1: the chunk's keys are all written first) is after pos.
 * Tensor cores (mma.sync, f32 accumulate) with q and the softmax weights as f16 hi + lo pairs.
 * q f32 or f16; out f32 or f16; q_stride, out_stride multiples of 8 (>= nH*hd); hd 128, 256 or 512;
 * nH a multiple of nkv; q, kc, vc, out 16-byte aligned. */
G4B_API int g4b_attn_prefill(const void* q, int dtype, int q_stride, int M, const float* qnw, const float* cosM,
                             const float* sinM, const uint16_t* kc, const uint16_t* vc, void* out, int out_dtype,
                             int out_stride, int nH, int nkv, int hd, int stride, int window, const int* p0_dev,
                             g4b_stream_t stream);

/* ------------------------------------------------------------ prefill element-wise rows */
/* The prefill layer's norm and activation dispatches over [M, D] token rows
 * (src/vk_engine.py:413-424), one CTA per row for the norms:
 *   g4b_rows_rmsnorm  vk/pre_norm.comp:8-13   y[m] = x[m] * rsqrt(mean(x[m]^2) + 1e-6) * w
 *   g4b_rows_normadd  vk/pre_na.comp:9-15     h[m] = (h[m] + x[m] * rsqrt(mean(x[m]^2) + 1e-6) * w) * scl
 *   g4b_gelumul       vk/gelumul.comp:7-8     out[i] = gelu_tanh(gate[i]) * up[i]   (n elements)
 * x, y, gate, up, out are f32 or f16 (G4B_DT_*); w and the residual h are f32.  D and n are
 * multiples of 4; every pointer 16-byte aligned.  (The decode token fuses the same work into the
 * GEMV chain: g4b_gemv_chain_create_fused.) */
G4B_API int g4b_rows_rmsnorm(const void* x, int x_dtype, const float* w, void* y, int y_dtype, int M, int D,
                             g4b_stream_t stream);
G4B_API int g4b_rows_normadd(const void* x, int x_dtype, const float* w, float* h, int M, int D, float scl,
                             g4b_stream_t stream);
G4B_API int g4b_gelumul(const void* gate, const void* up, int dtype, void* out, int out_dtype, size_t n,
                        g4b_stream_t stream);

/* ------------------------------------------------------------ tensor parallel */
/* The all-reduce after the row-parallel o and down GEMVs of a tensor-parallel
 * decode -- the cross-GPU counterpart of vk/reduce.comp:8-12 (the reference
 * runs on one GPU and has no collective).  One kernel, over NVLink peer
 * memory: each rank stores every element of x, paired with the call's epoch in
 * one 64-bit word, into slot [rank] of every rank's exchange buffer; each
 * thread then polls its elements of all slots in its own buffer until they
 * carry the epoch (bounded, 2 s, then the kernel status word is raised) and
 * writes y = the slots summed in rank order, identical bits on every rank.
 * No fence or flag round trip is needed.  In-place (x == y) is allowed.  For
 * the 15 KB per-layer reductions of a batch-1 decode this is latency-bound,
 * where NCCL's general algorithms are not tuned for it.
 *   bufs_dev  device array of `world` pointers: bufs_dev[r] = rank r's exchange
 *             buffer of g4b_allreduce_buffer_bytes(world, n) bytes, from
 *             g4b_comm_alloc (zero-filled), mapped into this process with
 *             g4b_ipc_open (own buffer: its own pointer)
 *   counter   this rank's device u32 call counter (zero-filled once); every rank
 *             makes the same calls in the same order (stream order, graphs too)
 *   flags     0 or G4B_GEMV_PDL (the kernel waits for its predecessor before it
 *             reads x or stores anything, and lets its successor launch early)
 * 1 <= world <= 8. */
G4B_API size_t g4b_allreduce_buffer_bytes(int world, int n);
G4B_API int g4b_allreduce_f32(const float* x, float* y, int n, int rank, int world, void* const* bufs_dev,
                              unsigned* counter, unsigned flags, g4b_stream_t stream);

/* Setup-time helpers for the exchange buffers (never on the hot path):
 * cudaMalloc + zero fill, cudaFree, and CUDA IPC export / import / close
 * (a handle is 64 bytes). */
G4B_API int g4b_comm_alloc(size_t bytes, void** dptr);
G4B_API int g4b_comm_free(void* dptr);
G4B_API int g4b_ipc_handle(const void* dptr, void* handle64);
G4B_API int g4b_ipc_open(const void* handle64, void** dptr);
G4B_API int g4b_ipc_close(void* dptr);

#ifdef __cplusplus
}
#endif
#endif /* G4B_H */
