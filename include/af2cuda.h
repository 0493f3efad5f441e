/*
 * af2cuda.h -- C ABI of libaf2cuda.so, the B200 (sm_100a) implementation of
 * the Evoformer pair-stack contractions of alphafold2-webgpu.
 *
 * Every entry point is plain C: opaque handles, plain pointers, sizes and
 * enums, no exceptions.  Each returns an af2_status; af2_last_error() gives
 * the message of the last failure on a context.
 *
 * Two call forms mirror the reference's two layers (all paths relative to the
 * reference repository):
 *
 *   host form   -- mirrors the standalone operator classes, whose run() takes
 *                  host Float32Arrays, uploads them, runs, reads back and
 *                  returns a fresh Float32Array plus timing
 *                  (src/triangle/webgpu.ts:56-201,
 *                   src/evoformer/outer-product-mean.ts:549-646,
 *                   src/evoformer/transition.ts:264-361);
 *   device form -- mirrors the in-model encoders on device-resident tensors,
 *                  with an optional residual add into the output
 *                  (src/evoformer/block.ts:1497-1671, :1115-1246, :625-740).
 *
 * Tensor layouts are the reference's: row-major, pair tensors [N, N, C],
 * triangle weights [out, in] (src/triangle/types.ts:9-26), OPM and transition
 * weights [in, out] (outer-product-mean.ts:10-19, transition.ts:9-16), packed
 * in the reference's orders (src/triangle/weights.ts:4-10,
 * outer-product-mean.ts:68-72, transition.ts:140-177).
 *
 * Arithmetic: operands are rounded to f16 (bf16-range activations are
 * normalised first) and multiplied on the tcgen05 tensor cores with f32
 * accumulation; LayerNorm statistics, gating and bias terms are f32.
 *
 * Threading: one context per device; calls on one context are serialised by
 * the caller.  Device-form calls are asynchronous on the given stream
 * (NULL = the context's stream); af2_sync() waits and reports any
 * device-side failure flagged by the kernels.
 */
#ifndef AF2CUDA_H
#define AF2CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AF2CUDA_VERSION 1

#if defined(__GNUC__)
#define AF2_API __attribute__((visibility("default")))
#else
#define AF2_API
#endif

typedef struct af2_ctx af2_ctx;

typedef enum af2_status {
    AF2_OK = 0,
    /* A shape, length or epsilon the reference rejects with RangeError
     * (src/triangle/types.ts:42-89, outer-product-mean.ts:45-65). */
    AF2_ERR_INVALID_ARGUMENT = 1,
    /* A valid shape outside what the kernels cover (for example c_z > 128). */
    AF2_ERR_UNSUPPORTED = 2,
    /* Device allocation failed (GpuMemoryBudgetError, runtime/allocator.ts:76-90). */
    AF2_ERR_OUT_OF_MEMORY = 3,
    /* A CUDA runtime error ("WebGPU validation failed", triangle/webgpu.ts:191-192). */
    AF2_ERR_CUDA = 4,
    /* A kernel's bounded wait ran out; the kernel returned without finishing. */
    AF2_ERR_DEVICE_TIMEOUT = 5,
    /* An NCCL call failed or a rank did not answer. */
    AF2_ERR_NCCL = 6,
    /* No CUDA device, or the device is not sm_100. */
    AF2_ERR_NO_DEVICE = 7
} af2_status;

typedef enum af2_dtype { AF2_F32 = 0, AF2_F16 = 1, AF2_BF16 = 2 } af2_dtype;

typedef enum af2_direction { AF2_OUTGOING = 0, AF2_INCOMING = 1 } af2_direction;

/* TriangleShape, src/triangle/types.ts:3-7. */
typedef struct af2_triangle_shape {
    int64_t length;
    int64_t c_z;
    int64_t c_hidden;
} af2_triangle_shape;

/* TriangleGpuOptions, src/triangle/webgpu.ts:9-15, plus the encoder's residual. */
typedef struct af2_triangle_options {
    /* Output rows per block; 0 = the whole length.  Bounds the contracted
     * scratch only: results are bit-identical for every value. */
    int32_t block_rows;
    /* 1: out += update (encodeTriangleMultiplication with residualTarget). */
    int32_t residual;
} af2_triangle_options;

/* What a call cost: the counterpart of {elapsedMilliseconds, memory}. */
typedef struct af2_op_stats {
    double device_milliseconds; /* CUDA-event time of the kernels */
    double host_milliseconds;   /* host form: copies in, kernels, copy out */
    double flops;               /* algorithmic FLOPs (src/runtime/kernel-cost.ts:71-162) */
    uint64_t workspace_bytes;   /* scratch the call used */
    uint64_t peak_bytes;        /* context's device allocation high-water mark */
} af2_op_stats;

/* ---- context --------------------------------------------------------- */

/* Opens device `device_ordinal` (replaces requestAlphaFoldDevice, runtime/device.ts:375). */
AF2_API af2_status af2_create(int device_ordinal, af2_ctx **out);
AF2_API void af2_destroy(af2_ctx *ctx);
AF2_API const char *af2_last_error(const af2_ctx *ctx);
AF2_API const char *af2_status_string(af2_status status);
AF2_API int af2_version(void);
/* Waits for `stream` (NULL = context stream) and reports kernel-side failures. */
AF2_API af2_status af2_sync(af2_ctx *ctx, void *stream);
/* Number of kernels this context has launched (monotonic). */
AF2_API uint64_t af2_launch_count(const af2_ctx *ctx);
/* Device memory the context holds now and its high-water mark, in bytes: the
 * currentBytes / peakBytes of the reference allocator's snapshot()
 * (src/runtime/allocator.ts:8-10,376-382).  Either pointer may be NULL. */
AF2_API af2_status af2_memory_snapshot(const af2_ctx *ctx, uint64_t *current_bytes, uint64_t *peak_bytes);

/*
 * What the GEMMs multiply in: the counterpart of the reference's installed
 * GEMM variant (src/runtime/gemm.ts:175,208-228, whose precision is "f32" or
 * "matrix" among others, chosen once per device).  AF2_GEMM_MATRIX (the
 * default): f16 operands on the tcgen05 tensor cores, f32 accumulation.
 * AF2_GEMM_F32: every operand of the outer-product mean's three GEMMs is
 * carried as an f16 pair hi + lo (about 22 significant bits) and each
 * product summed as hi.hi + hi.lo + lo.hi, still on the tensor cores with f32
 * accumulation, for results within f32 rounding of the reference's f32 path
 * (three times the tensor-core work, and the two-kernel OPM path).  The
 * triangle multiplication, attention and transition kernels multiply f16
 * operands in either mode.  Per context; takes effect at the next call.
 */
typedef enum af2_gemm_precision { AF2_GEMM_MATRIX = 0, AF2_GEMM_F32 = 1 } af2_gemm_precision;
AF2_API af2_status af2_set_gemm_precision(af2_ctx *ctx, int precision);
AF2_API int af2_get_gemm_precision(const af2_ctx *ctx);

/*
 * Prepared-weights cache (the role of the reference's packing cache per
 * weights object, src/evoformer/block.ts:1310-1333).  While enabled, each
 * device-form call looks its weights up by their device pointers and the
 * dimensions their preparation depends on; the first call prepares them
 * (f16 operand layouts, folded LayerNorm, scales) into a context-owned
 * buffer, later calls skip the preparation kernels.  The caller promises
 * that cached weights are not changed in place: after changing them call
 * af2_clear_weight_cache (which synchronises the device and frees the
 * buffers).  Off by default; disabling clears it.  The allocation-free
 * triangle entry point never uses it.
 */
AF2_API af2_status af2_set_weight_cache(af2_ctx *ctx, int enable);
AF2_API af2_status af2_clear_weight_cache(af2_ctx *ctx);

/*
 * Per-kernel device timing (the counterpart of the reference's timestamp-query
 * profile, src/runtime/execution.ts:482-533).  While enabled every kernel
 * launch is bracketed by CUDA events on its own stream.  af2_profile_read
 * synchronises, folds the recorded launches into per-kernel totals and
 * returns the totals of `kernel` (names as af2_profile_kernel_name gives them).
 */
AF2_API af2_status af2_profile_enable(af2_ctx *ctx, int enable);
AF2_API af2_status af2_profile_reset(af2_ctx *ctx);
AF2_API const char *af2_profile_kernel_name(int index);
AF2_API af2_status af2_profile_read(af2_ctx *ctx, const char *kernel, uint64_t *launches, double *milliseconds);

/*
 * Kernel selection.  Each op picks its kernels from the shape: the fused
 * outer-product mean (c = 32, S <= 1024, c_z <= 128) with three residues j
 * per tile where their operands fit in shared memory (two otherwise), else
 * the two-kernel path through an HBM scratch; the fused transition (C <= 128,
 * H <= 1024), else LayerNorm plus two linear GEMMs; the 16-bit MSA's
 * LayerNorm fused into the OPM projection.  Two environment variables select
 * the alternative where both are valid, to measure the choice:
 * AF2_OPM_TILE_RESIDUES=2 (two residues per fused OPM tile; results are
 * bit-identical) and AF2_TRANSITION_WIDE=1 (the two-GEMM transition for
 * shapes the fused kernel holds; results agree to f16 rounding).  They are
 * read at each call.
 */

/* ---- triangle multiplication ------------------------------------------ */

/* expectedWeightElementCount, src/triangle/weights.ts:36-40. */
AF2_API int64_t af2_triangle_weight_count(int64_t c_z, int64_t c_hidden);

/*
 * validateTriangleInput (src/triangle/types.ts:54-89) for what a C caller
 * passes: positive safe-integer dimensions, the packed weight count, a finite
 * positive epsilon; then the kernels' own limits.  Needs no device.  The
 * message (NUL-terminated, truncated to `capacity`) may be NULL.
 */
AF2_API af2_status af2_triangle_check(int direction, const af2_triangle_shape *shape, int64_t weight_count, double epsilon,
                              char *message, size_t capacity);

/* Scratch bytes the device form needs for this shape and options. */
AF2_API af2_status af2_triangle_workspace_bytes(const af2_triangle_shape *shape,
                                        const af2_triangle_options *options, uint64_t *bytes);

/*
 * Host form of TriangleMultiplication{Outgoing,Incoming}Gpu.run
 * (src/triangle/webgpu.ts:56-201, classes :204-214).
 * z [N,N,c_z] and out [N,N,c_z] are host arrays of `io_dtype` (AF2_F32 is the
 * reference's Float32Array); mask [N,N] f32; packed_weights f32 in ORDER with
 * weight_count = af2_triangle_weight_count(c_z, c_hidden).  Host buffers may
 * be pageable or pinned.  options may be NULL; stats may be NULL.
 */
AF2_API af2_status af2_triangle_multiplication_host(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                            const void *z, const float *mask, const float *packed_weights,
                                            int64_t weight_count, double epsilon,
                                            const af2_triangle_options *options, int io_dtype, void *out,
                                            af2_op_stats *stats);

/*
 * Device form: encodeTriangleMultiplication (src/evoformer/block.ts:1497-1671).
 * All pointers are device pointers.  z has z_dtype, out has out_dtype; with
 * options->residual = 1 the update is added into out (pass out == z to update
 * the pair in place).  workspace: NULL = context-owned scratch, else at least
 * af2_triangle_workspace_bytes() bytes, 256-byte aligned.
 */
AF2_API af2_status af2_triangle_multiplication(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                       const void *z, int z_dtype, const float *mask,
                                       const float *packed_weights, int64_t weight_count, double epsilon,
                                       const af2_triangle_options *options, void *out, int out_dtype,
                                       void *workspace, void *stream);

/*
 * The device form above, taking its scratch from a fixed array in device
 * memory instead of allocating.  No counterpart in the reference.  For hosts
 * that cannot let a library call cudaMalloc: a memory manager that owns the
 * device under a fixed budget, or a latency-sensitive path where cudaMalloc
 * and cudaFree would synchronise the device.  The call allocates nothing; the
 * array (16.5 MiB, enough for length <= 128 at c_z = c_hidden = 128) is held
 * on each device where the library is loaded until the process exits, and
 * larger shapes return AF2_ERR_UNSUPPORTED.  The first call on each device
 * looks up the array's device address (once); make that first call before any
 * stream capture, and do not reset the device while the library is loaded.
 * All calls share the array: calls that overlap on the GPU race.  Arguments
 * as af2_triangle_multiplication, without `workspace`.
 */
AF2_API af2_status af2_triangle_multiplication_static(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                                      const void *z, int z_dtype, const float *mask,
                                                      const float *packed_weights, int64_t weight_count,
                                                      double epsilon, const af2_triangle_options *options,
                                                      void *out, int out_dtype, void *stream);

/* ---- the pair sharded by rows across the GPUs of one box ---------------- */

/*
 * One process and one context per GPU.  Rank 0 creates a unique id (128
 * bytes), the host hands it to every rank (for instance with
 * torch.distributed.broadcast_object_list), and every rank calls
 * af2_comm_init with it; NCCL carries the exchanges over NVLink.  No
 * counterpart in the reference, which runs on one device.
 */
#define AF2_COMM_UNIQUE_ID_BYTES 128
AF2_API af2_status af2_comm_unique_id(void *unique_id);
AF2_API af2_status af2_comm_init(af2_ctx *ctx, const void *unique_id, int nranks, int rank);
AF2_API af2_status af2_comm_destroy(af2_ctx *ctx);

/*
 * Failure detection.  All ranks must make the same sequence of sharded calls
 * with the same shapes (as NCCL's collectives require); a rank that fails or
 * leaves otherwise leaves its peers' collectives waiting.  Every host wait of
 * a context with a communicator (af2_sync, af2_comm_destroy, the library's
 * own waits) polls the stream and ncclCommGetAsyncError; at the
 * communicator's first asynchronous error, or when the work has not finished
 * `seconds` after the wait began (default 600; 0 = no deadline), it aborts
 * the communicator (ncclCommAbort ends its kernels, so the stream drains and
 * the context stays usable) and returns AF2_ERR_NCCL.  Later sharded calls
 * return AF2_ERR_NCCL until af2_comm_destroy and a new af2_comm_init.  The
 * detection is on the host only; ranks should leave between steps (nothing
 * of theirs in flight) and tell the others through the host (a store or a
 * heartbeat) before the others' next launch.
 */
AF2_API af2_status af2_comm_set_timeout(af2_ctx *ctx, double seconds);
/* Ends this rank's communicator without any collective -- for a rank whose
 * peer is lost, or that leaves -- and frees the exchange resources; the
 * context stays usable for single-GPU calls and a new af2_comm_init. */
AF2_API af2_status af2_comm_abort(af2_ctx *ctx);

/*
 * The device form of triangle multiplication on a pair sharded by rows: this
 * rank holds rows [rank * L, (rank + 1) * L) of z, mask and out (L = length /
 * nranks, a multiple of 64; nranks divides 128), shape->length is the full
 * length.  Each rank projects its rows; an all-to-all gives every rank 128 /
 * nranks hidden channels of all rows, which it contracts over the whole
 * length; a second all-to-all returns all channels of the rank's own rows for
 * the output projection.  Every rank calls it with the same arguments,
 * collectively.  Results are bit-identical to the single-GPU
 * af2_triangle_multiplication.
 */
AF2_API af2_status af2_triangle_multiplication_sharded(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                                       const void *z, int z_dtype, const float *mask,
                                                       const float *packed_weights, int64_t weight_count,
                                                       double epsilon, const af2_triangle_options *options,
                                                       void *out, int out_dtype, void *stream);

/*
 * The device form of the outer-product mean on a row-sharded pair: m [S, L,
 * c_m] holds this rank's residue columns [rank * L, (rank + 1) * L) of the
 * MSA, mask [S, N] the whole MSA mask (every rank passes the same), out this
 * rank's rows of the [N, N, c_z] update (L = N / nranks, a multiple of 8).
 * Each rank normalises and projects its own residues; the right operand is
 * all-gathered.  Collective.
 */
struct af2_opm_shape;
struct af2_opm_options;
AF2_API af2_status af2_outer_product_mean_sharded(af2_ctx *ctx, const struct af2_opm_shape *shape, const void *m,
                                                  int m_dtype, const float *mask, const float *packed_weights,
                                                  int64_t weight_count, const struct af2_opm_options *options,
                                                  void *out, int out_dtype, void *stream);

/* ---- weights: f32 or mixed-q8 ------------------------------------------ */

typedef enum af2_weight_format {
    /* f32 values. */
    AF2_WEIGHTS_F32 = 0,
    /* int8 codes with one f16 scale (stored as its 16 bits) per `block`
     * consecutive elements of the flattened matrix: w[i] = code[i] *
     * f16(scale[i / block]).  The reference's mixed-q8 files use block = 64
     * (src/reference/dtype.ts:86-97, tools/quantize-web-model.ts:98-119). */
    AF2_WEIGHTS_Q8_BLOCK = 1,
    /* int8 codes with one f32 scale per output column of an [in, out]
     * matrix: w[k][o] = code[k][o] * scale[o]. */
    AF2_WEIGHTS_Q8_CHANNEL = 2
} af2_weight_format;

/* One weight matrix, [in, out] row-major (transition.ts:115). */
typedef struct af2_matrix {
    int32_t format;     /* af2_weight_format */
    int32_t block;      /* AF2_WEIGHTS_Q8_BLOCK: elements per scale (64 in the reference's files) */
    const void *values; /* float[in * out] or int8_t[in * out] */
    const void *scales; /* uint16_t[ceil(in * out / block)] (Q8_BLOCK), float[out] (Q8_CHANNEL), NULL (F32) */
} af2_matrix;

/*
 * Bit-exact decode of a q8 matrix to f32 (readTensorRange's int8 branch,
 * src/reference/dtype.ts:86-97, for the whole tensor; for Q8_CHANNEL the f32
 * product code * scale[o]).  Device pointers; out holds inner * cols floats.
 */
AF2_API af2_status af2_dequant_q8(af2_ctx *ctx, const af2_matrix *matrix, int64_t inner, int64_t cols, float *out,
                                  void *stream);

/*
 * Per-tensor weights.  The reference's model files hold each weight tensor on
 * its own (a TensorStore record: f32, or int8 codes with one f16 scale per 64
 * elements, src/reference/tensor-store.ts:4-13, dtype.ts:66-99), and its host
 * decodes them to f32 before packing.  These forms take the tensors as they
 * are stored, one af2_matrix each (AF2_WEIGHTS_F32 or AF2_WEIGHTS_Q8_BLOCK;
 * AF2_WEIGHTS_Q8_CHANNEL returns AF2_ERR_UNSUPPORTED), and turn the codes into
 * the kernels' f16 operands on the device.  The decode is the reference's own,
 * bit for bit (a 7-bit code times an 11-bit scale is exact in f32), so the
 * results equal the packed forms given the decoded f32 weights.
 */

/* TriangleMultiplicationWeights (src/triangle/types.ts:9-26) in ORDER
 * (src/triangle/weights.ts:4-10); projection weights are [out, in]. */
#define AF2_TRIANGLE_TENSORS 16
/* Device form of the triangle multiplication from 16 tensors; other arguments
 * and the workspace as af2_triangle_multiplication. */
AF2_API af2_status af2_triangle_multiplication_weights(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                                       const void *z, int z_dtype, const float *mask,
                                                       const af2_matrix *tensors, double epsilon,
                                                       const af2_triangle_options *options, void *out, int out_dtype,
                                                       void *workspace, void *stream);

/* ---- transition ---------------------------------------------------------- */

/* TransitionInput's dimensions, src/evoformer/transition.ts:18-25. */
typedef struct af2_transition_shape {
    int64_t rows;
    int64_t channels;
    int64_t hidden_channels;
} af2_transition_shape;

/* TransitionWeights (transition.ts:9-16), each matrix f32 or q8. */
typedef struct af2_transition_weights {
    const float *layer_norm_scale;  /* [channels] */
    const float *layer_norm_offset; /* [channels] */
    af2_matrix first_weight;        /* [channels, hidden_channels] */
    const float *first_bias;        /* [hidden_channels] */
    af2_matrix second_weight;       /* [hidden_channels, channels] */
    const float *second_bias;       /* [channels] */
} af2_transition_weights;

typedef struct af2_transition_options {
    /* TransitionGpuOptions.maxChunkRows (transition.ts:33-36): 0 = none.  It
     * bounds the reference's scratch only; results are identical for every
     * value, and the fused kernel keeps the hidden activations on chip. */
    int32_t max_chunk_rows;
    /* 1: out += transition(x) (encodeTransition with residualTarget). */
    int32_t residual;
} af2_transition_options;

/* Length of packTransitionWeights(input).data (transition.ts:140-177). */
AF2_API int64_t af2_transition_weight_count(int64_t channels, int64_t hidden_channels);

/* validate (transition.ts:140-156) plus the kernels' limits; no device needed. */
AF2_API af2_status af2_transition_check(const af2_transition_shape *shape, int64_t weight_count, double epsilon,
                                        char *message, size_t capacity);

AF2_API af2_status af2_transition_workspace_bytes(const af2_transition_shape *shape, uint64_t *bytes);

/*
 * Host form of TransitionGpu.run (transition.ts:264-361): x and out are host
 * arrays [rows, channels] of io_dtype; packed_weights is f32 in the order of
 * packTransitionWeights.  out = Linear2(ReLU(Linear1(LayerNorm(x)))), plus x
 * when options->residual is 1.
 */
AF2_API af2_status af2_transition_host(af2_ctx *ctx, const af2_transition_shape *shape, const void *x,
                                       const float *packed_weights, int64_t weight_count, double epsilon,
                                       const af2_transition_options *options, int io_dtype, void *out,
                                       af2_op_stats *stats);

/*
 * Device form: encodeTransition (src/evoformer/block.ts:625-740).  x [rows,
 * channels] of x_dtype, out of out_dtype; weights hold device pointers, f32
 * or q8.  With options->residual = 1 the result is added into out (out == x
 * updates the activations in place).  workspace: NULL = context-owned, else
 * af2_transition_workspace_bytes() bytes, 256-byte aligned.
 */
AF2_API af2_status af2_transition(af2_ctx *ctx, const af2_transition_shape *shape, const void *x, int x_dtype,
                                  const af2_transition_weights *weights, double epsilon,
                                  const af2_transition_options *options, void *out, int out_dtype, void *workspace,
                                  void *stream);

/* ---- outer-product mean -------------------------------------------------- */

/* OuterProductMeanInput's dimensions, src/evoformer/outer-product-mean.ts:21-34. */
typedef struct af2_opm_shape {
    int64_t sequences; /* S */
    int64_t length;    /* N residues */
    int64_t c_m;
    int64_t c_outer;   /* c */
    int64_t c_z;
} af2_opm_shape;

typedef struct af2_opm_options {
    double layer_norm_epsilon;    /* layerNormEpsilon: 0 = 1e-5 */
    double normalization_epsilon; /* normalizationEpsilon: 0 = 1e-3 */
    /* rowBlockResidues: output residues per block (0 = automatic).  It bounds
     * the outer-product scratch only; results are bit-identical for every value. */
    int32_t row_block_residues;
    /* 1: out += OPM(m) (encodeOuterProductMean with residualTarget). */
    int32_t residual;
} af2_opm_options;

/* Length of packOuterProductMeanWeights(input).data (outer-product-mean.ts:68-80). */
AF2_API int64_t af2_opm_weight_count(const af2_opm_shape *shape);

/* validate (outer-product-mean.ts:45-65) plus the kernels' limits (c_outer = 32,
 * c_m <= 256, c_z <= 4096); no device needed. */
AF2_API af2_status af2_opm_check(const af2_opm_shape *shape, int64_t weight_count, char *message, size_t capacity);

AF2_API af2_status af2_opm_workspace_bytes(const af2_opm_shape *shape, const af2_opm_options *options,
                                           uint64_t *bytes);

/*
 * Host form of OuterProductMeanGpu.run (outer-product-mean.ts:538-647): m
 * [S, N, c_m] of io_dtype, mask [S, N] f32, packed_weights f32 in the order of
 * packOuterProductMeanWeights; out [N, N, c_z] of io_dtype.
 */
AF2_API af2_status af2_outer_product_mean_host(af2_ctx *ctx, const af2_opm_shape *shape, const void *m,
                                               const float *mask, const float *packed_weights, int64_t weight_count,
                                               const af2_opm_options *options, int io_dtype, void *out,
                                               af2_op_stats *stats);

/* Device form: encodeOuterProductMean (src/evoformer/block.ts:1115-1246).  All
 * pointers on the device; workspace NULL = context-owned (required in the
 * AF2_GEMM_F32 precision; af2_opm_workspace_bytes sizes the default one). */
AF2_API af2_status af2_outer_product_mean(af2_ctx *ctx, const af2_opm_shape *shape, const void *m, int m_dtype,
                                          const float *mask, const float *packed_weights, int64_t weight_count,
                                          const af2_opm_options *options, void *out, int out_dtype, void *workspace,
                                          void *stream);

/* OuterProductMeanWeights in the order of packOuterProductMeanWeights
 * (outer-product-mean.ts:68-72): LayerNorm scale and offset, leftWeight
 * [c_m, c], leftBias, rightWeight [c_m, c], rightBias, outputWeight
 * [c*c, c_z], outputBias. */
#define AF2_OPM_TENSORS 8
/* Device form of the outer product mean from 8 tensors (per-tensor weights
 * above); other arguments and the workspace as af2_outer_product_mean. */
AF2_API af2_status af2_outer_product_mean_weights(af2_ctx *ctx, const af2_opm_shape *shape, const void *m, int m_dtype,
                                                  const float *mask, const af2_matrix *tensors,
                                                  const af2_opm_options *options, void *out, int out_dtype,
                                                  void *workspace, void *stream);

/* ---- gated multi-head attention: triangle attention ---------------------- */

/* AttentionInput's dimensions (src/evoformer/attention.ts:47-58): `batch`
 * independent rows of `queries` positions, `channels` = heads x 32. */
typedef struct af2_attention_shape {
    int64_t batch;
    int64_t queries;  /* queryLength; the keys are the same positions */
    int64_t channels;
    int64_t heads;
} af2_attention_shape;

/* AttentionPairBias (attention.ts:31-45): none, or "normalized-input" -- the
 * bias of head h at (query q, key k) is LN(x)[q, k] . projectionWeight[:, h],
 * projected from the attention's own normalised source (triangle attention,
 * src/evoformer/block.ts:1727-1745; needs batch == queries).  The "separate"
 * source of MSA row attention is not covered. */
typedef enum af2_pair_bias { AF2_PAIR_BIAS_NONE = 0, AF2_PAIR_BIAS_NORMALIZED_INPUT = 1 } af2_pair_bias;

typedef struct af2_attention_options {
    /* AttentionInput.transpose: the column view (row b, position q is source
     * row q * batch + b) -- the ending-node triangle attention. */
    int32_t transpose;
    int32_t pair_bias; /* af2_pair_bias */
    /* 1: out += attention(x) (encodeAttention with residualTarget). */
    int32_t residual;
} af2_attention_options;

/* Length of packAttentionWeights(input).data (attention.ts:179-201): queryNorm
 * scale and offset [C], query / key / value / gating weights [C, C] ([in,
 * out]), gating bias [C], output weight [C, C] ([in, out]), output bias [C],
 * then for a normalized-input bias the projection weight [C, heads]. */
AF2_API int64_t af2_attention_weight_count(const af2_attention_shape *shape, int pair_bias);

/* validate (attention.ts:102-141) plus the kernels' limits (head dimension 32,
 * channels <= 256, batch == queries for a normalized-input bias); no device needed. */
AF2_API af2_status af2_attention_check(const af2_attention_shape *shape, int pair_bias, int64_t weight_count,
                                       double epsilon, char *message, size_t capacity);

AF2_API af2_status af2_attention_workspace_bytes(const af2_attention_shape *shape, int pair_bias, uint64_t *bytes);

/*
 * Host form of AttentionGpu.run (attention.ts:1334-1453): x [batch *
 * queries, channels] and mask [batch * queries] are host f32 arrays in the
 * source's row order (the transposed view reads them as the reference does);
 * out [batch * queries, channels] f32 receives the output rows (plus x when
 * options->residual is 1).
 */
AF2_API af2_status af2_attention_host(af2_ctx *ctx, const af2_attention_shape *shape, const float *x,
                                      const float *mask, const float *packed_weights, int64_t weight_count,
                                      double epsilon, const af2_attention_options *options, float *out,
                                      af2_op_stats *stats);

/*
 * Device form: encodeAttention on device-resident tensors (the triangle
 * attention calls of src/evoformer/block.ts:1727-1745).  x of x_dtype, mask
 * f32, packed_weights f32, out of out_dtype; with options->residual = 1 the
 * result is added into out (out == x updates the pair in place).  workspace:
 * NULL = context-owned, else af2_attention_workspace_bytes() bytes, 256-byte aligned.
 */
AF2_API af2_status af2_attention(af2_ctx *ctx, const af2_attention_shape *shape, const void *x, int x_dtype,
                                 const float *mask, const float *packed_weights, int64_t weight_count, double epsilon,
                                 const af2_attention_options *options, void *out, int out_dtype, void *workspace,
                                 void *stream);

/* ---- the Evoformer pair block ------------------------------------------------ */

/* The dimensions encodeEvoformerPairBlock reads from EvoformerShape and its
 * weights (src/evoformer/block.ts:174-181,1753-1805). */
typedef struct af2_pair_block_shape {
    int64_t length;            /* N residues: pair [N, N, c_z] */
    int64_t sequences;         /* S: MSA [S, N, c_m] */
    int64_t c_m;
    int64_t c_z;
    int64_t c_outer;           /* outer-product-mean channels */
    int64_t c_hidden;          /* triangle multiplication hidden channels */
    int64_t pair_heads;        /* triangle attention heads (head dimension 32) */
    int64_t transition_hidden; /* pair transition hidden channels */
} af2_pair_block_shape;

/* EvoformerPairBlockWeights (block.ts:174-181), each op's weights as its own
 * packed f32 array (device pointers), in the orders the op entry points take:
 * packOuterProductMeanWeights, triangle ORDER, packAttentionWeights with the
 * normalized-input pair projection last; the pair transition as
 * af2_transition_weights (f32 or q8 matrices). */
typedef struct af2_pair_block_weights {
    const float *outer_product_mean;
    const float *triangle_outgoing;
    const float *triangle_incoming;
    const float *attention_starting;
    const float *attention_ending;
    af2_transition_weights pair_transition;
} af2_pair_block_weights;

typedef struct af2_pair_block_options {
    /* encodeEvoformerPairBlock's includeOuterProductMean (0 skips the OPM and
     * then msa / msa_mask may be NULL). */
    int32_t include_outer_product_mean;
    /* LayerNorm epsilon of every op (0 = 1e-5); the OPM's normalisation epsilon stays 1e-3. */
    double epsilon;
} af2_pair_block_options;

/*
 * encodeEvoformerPairBlock (src/evoformer/block.ts:1753-1805) on device
 * tensors: the outer-product mean of the MSA, triangle multiplication
 * outgoing and incoming, triangle attention around the starting and the
 * ending node, and the pair transition, each added into the pair in place, in
 * that order, on one stream.  msa [S, N, c_m] of msa_dtype, msa_mask [S, N]
 * f32, pair [N, N, c_z] of pair_dtype, pair_mask [N, N] f32.  Scratch is the
 * context's, sized once for the largest op.  options may be NULL.
 */
AF2_API af2_status af2_evoformer_pair_block(af2_ctx *ctx, const af2_pair_block_shape *shape,
                                            const af2_pair_block_weights *weights, const void *msa, int msa_dtype,
                                            const float *msa_mask, void *pair, int pair_dtype, const float *pair_mask,
                                            const af2_pair_block_options *options, void *stream);

/* ---- the shared dense projection ----------------------------------------- */

/* createLinearShader (transition.ts:91-138): out (=, +=) act(A W + b). */
typedef struct af2_linear_shape {
    int64_t rows;
    int64_t inner;
    int64_t columns;
} af2_linear_shape;

typedef enum af2_activation { AF2_ACTIVATION_NONE = 0, AF2_ACTIVATION_RELU = 1 } af2_activation;

AF2_API af2_status af2_linear_workspace_bytes(const af2_linear_shape *shape, int a_dtype, uint64_t *bytes);

/*
 * Device form: A [rows, inner] of a_dtype, weight [inner, columns] ([in, out],
 * f32 or q8), bias [columns] f32 or NULL, out [rows, columns] of out_dtype;
 * residual = 1 adds into out.  Operands are multiplied as f16 with f32
 * accumulation.  workspace NULL = context-owned.
 */
AF2_API af2_status af2_linear(af2_ctx *ctx, const af2_linear_shape *shape, const void *a, int a_dtype,
                              const af2_matrix *weight, const float *bias, int activation, int residual, void *out,
                              int out_dtype, void *workspace, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* AF2CUDA_H */
