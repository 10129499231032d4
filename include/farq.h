/*
 * farq.h — C ABI of the B200 (sm_100a) fused residual-add + RMSNorm +
 * per-token group quantisation library (libfarq.so).
 *
 * The library replaces the device work behind the reference operator
 *   fused_add_rmsnorm_group_quant(x, residual, gamma, residual_out, norm_out,
 *                                 x_q, x_scale, eps, group_size)
 * in src/task01_fused_add_rmsnorm_group_quant.py:1731-1851 of
 * sinpeyw/flagos-kernelgen-72h-shanghai-2026, i.e. the Triton kernels it routes
 * to on NVIDIA parts:
 *   _preweighted_full_row_kernel                  (task01…py:65-121)
 *   _preweighted_segmented_streaming_kernel       (task01…py:1127-1348)
 *   _nvidia_parallel_row_group_streaming_kernel   (task01…py:1401-1546)
 * All three compute the same per-row math; one kernel here covers all of them.
 *
 * Per row m (all arithmetic in fp32, d = 0..D-1, g = d / G):
 *   r[d]     = f32(x[m,d]) + f32(residual[m,d])        -> residual_out (RNE)
 *   inv_rms  = 1 / sqrt(sum_d r[d]^2 / D + eps)
 *   w[d]     = r[d] * f32(gamma[d])
 *   norm[d]  = w[d] * inv_rms                           -> norm_out (RNE, optional)
 *   scale[g] = max(max_{d in g} |w[d]| * (inv_rms / QMAX), 1e-12)
 *              (UE8M0 flag: rounded up to a power of two)
 *   q[d]     = INT8 : trunc(clamp(norm[d] * (1/scale[g]), -127, 127)), QMAX = 127
 *              E4M3 : rne_satfinite_e4m3(norm[d] * (1/scale[g])),       QMAX = 448
 *
 * Memory contract: destination passing. Every pointer is a device pointer the
 * caller owns; nothing is allocated by farq_launch. The launch is asynchronous
 * on the given stream and performs no host synchronisation. residual_out may
 * alias x or residual (each row is fully read before any of its outputs are
 * written, and rows are disjoint).
 */
#ifndef FARQ_H
#define FARQ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FARQ_ABI_VERSION 1

/* Element types. */
enum farq_dtype {
    FARQ_DTYPE_BF16 = 0,
    FARQ_DTYPE_FP16 = 1,
    FARQ_DTYPE_FP32 = 2,
    FARQ_DTYPE_INT8 = 3,
    FARQ_DTYPE_E4M3 = 4
};

/* flags bits. */
enum farq_flags {
    FARQ_FLAG_UE8M0 = 1,  /* round every scale up to a power of two            */
    /* x_scale is column-major [D/G, ld] ("MN-major", the layout blockwise-FP8
     * GEMMs read scales in): scale of (row m, group g) at x_scale[g*ld + m],
     * ld = x_scale_row_stride (0 = M). No reference counterpart: the reference
     * writes [M, D/G] row-major only (task01…py:1112). */
    FARQ_FLAG_SCALE_COLUMN_MAJOR = 2,
    /* farq_ar_launch only: at world 1 the all-reduce is the identity and the
     * call runs the single-GPU kernel (x = partial[0]); this flag runs the
     * fused all-reduce kernel at world 1 too (tests of that kernel on one GPU). */
    FARQ_FLAG_AR_KERNEL_AT_WORLD1 = 4,
    /* Test only: the first row team of every CTA waits for a slot sequence
     * value that is never written, with every device wait limited to 1 ms,
     * so the bounded-wait path (status word, drained copies, clean exit) can
     * be exercised without a GPU fault. Rows of that team are not written. */
    FARQ_FLAG_TEST_FORCE_TIMEOUT = 1 << 30
};

/* Status codes returned by every entry point. Never a device trap. */
enum farq_status {
    FARQ_OK = 0,
    FARQ_ERR_NULL_POINTER = 1,     /* a required pointer is NULL            */
    FARQ_ERR_BAD_SHAPE = 2,        /* M < 0, D <= 0, D % G != 0, D % 8 != 0  */
    FARQ_ERR_BAD_GROUP = 3,        /* G not a power of two in [8, 256]       */
    FARQ_ERR_BAD_DTYPE = 4,        /* unsupported dtype combination          */
    FARQ_ERR_ALIGNMENT = 5,        /* row base or row stride not 16-B aligned */
    FARQ_ERR_UNSUPPORTED = 6,      /* D or a tuning choice out of range      */
    FARQ_ERR_CUDA = 7,             /* a CUDA runtime call failed             */
    FARQ_ERR_BAD_ARGS_SIZE = 8,    /* struct_size does not match this build,
                                      or a reserved field is not 0          */
    FARQ_ERR_DEVICE_TIMEOUT = 9,   /* a bounded device wait ran out          */
    FARQ_ERR_NOALLOC_TOO_LARGE = 10 /* call needs more than the 64 MiB staging
                                       array of farq_launch_host_noalloc     */
};

/*
 * Arguments of one call. Row strides are in ELEMENTS of the tensor they
 * describe; 0 means "contiguous" (D for the [M,D] tensors, D/G for x_scale).
 * The inner dimension is always contiguous.
 *
 * Replaces the positional arguments of the reference operator
 * (task01…py:1731-1741). Differences, all extensions:
 *   - norm_out may be NULL: the normalised tensor is then not written
 *     (7N + 4N/G + 2D bytes moved instead of 9N + 4N/G + 2D).
 *   - q_dtype selects INT8 (reference semantics) or E4M3.
 *   - status, when non-NULL, is a device int the kernel sets to a non-zero
 *     farq_status if a bounded wait on the device ran out. The kernel never
 *     clears it; the caller zeroes it.
 */
typedef struct farq_args {
    uint32_t struct_size;          /* = sizeof(farq_args_t)                 */
    int32_t  x_dtype;              /* BF16 | FP16; residual has the same    */
    int32_t  gamma_dtype;          /* BF16 | FP16 | FP32                    */
    int32_t  residual_out_dtype;   /* BF16 | FP16 | FP32                    */
    int32_t  norm_out_dtype;       /* BF16 | FP16 | FP32 (ignored if NULL)  */
    int32_t  q_dtype;              /* INT8 | E4M3                           */
    int32_t  flags;                /* farq_flags                            */
    int32_t  group_size;           /* G                                     */
    int64_t  M;                    /* rows (tokens); 0 is a no-op           */
    int64_t  D;                    /* hidden size                           */
    float    eps;
    int32_t  tune_ctas_per_sm;     /* 0 = auto (1)                          */
    int32_t  tune_teams_per_cta;   /* 0 = auto; upper bound on row teams    */
    int32_t  tune_stages;          /* 0 = auto; ring slots per CTA (>= teams) */
    int32_t  tune_vec_per_thread;  /* 0 = auto; 1..8 16-byte vectors        */
    int32_t  reserved0;            /* must be 0                             */
    const void* x;                 /* [M, D]                                */
    const void* residual;          /* [M, D]                                */
    const void* gamma;             /* [D]                                   */
    void*    residual_out;         /* [M, D]                                */
    void*    norm_out;             /* [M, D] or NULL                        */
    void*    x_q;                  /* [M, D] int8 / e4m3 bytes              */
    float*   x_scale;              /* [M, D/G] fp32                         */
    int32_t* status;               /* device int or NULL                    */
    int64_t  x_row_stride;
    int64_t  residual_row_stride;
    int64_t  residual_out_row_stride;
    int64_t  norm_out_row_stride;
    int64_t  x_q_row_stride;
    int64_t  x_scale_row_stride;
} farq_args_t;

/*
 * Launch the fused kernel on `stream` (a cudaStream_t; NULL = legacy default
 * stream) on the current CUDA device. Validates every argument first and
 * returns a farq_status; on FARQ_OK the work is queued, not finished.
 * Replaces: fused_add_rmsnorm_group_quant, task01…py:1731-1851 (the routing
 * at :1772-1817 and :1548-1728 collapses to one kernel with host-chosen
 * template parameters).
 */
int farq_launch(const farq_args_t* args, void* stream);

/* Static string for a farq_status (never NULL). No reference counterpart:
 * the reference raises whatever Triton raises. */
const char* farq_strerror(int status);

/* FARQ_ABI_VERSION of the loaded library. No reference counterpart. */
int farq_abi_version(void);

/* Largest hidden size D farq_launch accepts. The reference's segmented
 * kernel stops at 4 x 2048 columns (task01…py:1128-1348). */
int64_t farq_max_hidden(void);

/*
 * Launch plan the library would use for (M, D, G, x_dtype) on the current
 * device, written into out[0..5] = {threads per row team, row teams per CTA,
 * 16-byte vectors per thread, CTAs in the grid, pipeline slots per team,
 * dynamic shared-memory bytes}. Host-only query for tests and profiling;
 * launches nothing. No reference counterpart (Triton picks num_warps and the
 * kernel at task01…py:1772-1817).
 */
int farq_plan(int64_t M, int64_t D, int32_t group_size, int32_t x_dtype,
              int32_t tune_ctas_per_sm, int32_t tune_teams_per_cta,
              int32_t tune_stages, int32_t tune_vec_per_thread, int64_t out[6]);

/*
 * farq_launch with HOST buffers and no device allocation: x, residual, gamma,
 * residual_out, norm_out (or NULL), x_q and x_scale in `args` are host
 * pointers (pinned memory keeps the copies asynchronous); the call copies the
 * inputs into a device array compiled into the library, runs the kernel and
 * copies the outputs back, all queued on `stream`. The outputs are valid once
 * the stream has been synchronised.
 *
 * For callers that cannot allocate GPU memory: plugins inside a process whose
 * device allocator belongs to another framework, or C/FFI callers that only
 * hold host buffers. The array holds 64 MiB on every GPU that loads the
 * library, until the process exits; a call needing more staging (inputs,
 * gamma and outputs of all M rows, each rounded up to 256 bytes — about
 * 1,330 rows at D = 7168, bf16 -> e4m3) returns FARQ_ERR_NOALLOC_TOO_LARGE;
 * split the rows. Tensors must be contiguous with row-major x_scale. Every
 * argument check is made before the first copy is queued, so a rejected call
 * leaves no copy in flight. `status`, when non-NULL, is a HOST int here: it
 * is copied to the device with the inputs and back with the outputs (set to
 * a farq_status if a device wait ran out, never cleared). The first call on
 * a device looks up the array's device address (make it before any stream
 * capture). All calls share the array: calls that overlap on the GPU
 * (several streams or host threads) race; calls on one stream are ordered.
 *
 * No counterpart in the reference, which has no host-buffer path.
 */
int farq_launch_host_noalloc(const farq_args_t* args, void* stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel variant: all-reduce fused with the operator.
 *
 * Every rank of a W-rank group (W <= 8, one GPU each, peers reachable over
 * NVLink) holds a partial activation P_k [M, D]; x = sum of the partials,
 * rounded once to x_dtype, and the operator above is applied to x with the
 * rank's residual. Rank `rank` computes the rows [rank*M/W slab] and writes
 * every output row to all W ranks' output buffers, so on return every rank
 * holds the full residual_out, x_q, x_scale (and norm_out) — the replicated
 * result an all-reduce followed by the operator would give.
 *
 * All arrays are indexed by rank and hold pointers valid on THIS device
 * (peer mappings, e.g. from symmetric memory). Tensors are contiguous:
 * [M, D] activations, [M, D/G] row-major scales. `signal[k]` is rank k's
 * zero-initialised signal buffer of FARQ_AR_SIGNAL_WORDS uint32 words, used
 * only by this entry point; `epoch` must increase by one per call (starting
 * at 1) and be the same on every rank. Every rank must make the same call
 * (same M, D, dtypes, tuning); each blocks on the others inside the kernel
 * with waits bounded at 2 s, after which the status word (if any) is set to
 * FARQ_ERR_DEVICE_TIMEOUT.
 *
 * No counterpart in the reference, which runs on one device; this is the
 * producer-side fusion of the all-reduce that precedes
 * fused_add_rmsnorm_group_quant (task01…py:1731) in tensor-parallel models.
 * ---------------------------------------------------------------------- */
#define FARQ_AR_MAX_WORLD 8
#define FARQ_AR_SIGNAL_WORDS (2 * 1024 * 8)

typedef struct farq_ar_args {
    uint32_t struct_size;          /* = sizeof(farq_ar_args_t)                */
    int32_t  x_dtype;              /* BF16 | FP16: partials, residual, residual_out */
    int32_t  gamma_dtype;          /* BF16 | FP16 | FP32                       */
    int32_t  norm_out_dtype;       /* BF16 | FP16 | FP32 (ignored if no norm_out) */
    int32_t  q_dtype;              /* INT8 | E4M3                              */
    int32_t  flags;                /* FARQ_FLAG_UE8M0; FARQ_FLAG_AR_KERNEL_AT_WORLD1;
                                      FARQ_FLAG_TEST_FORCE_TIMEOUT
                                      makes the start barrier wait (1 ms) for
                                      an epoch no rank signals (tests only)    */
    int32_t  group_size;
    int32_t  world;                /* W, 1..8                                  */
    int32_t  rank;                 /* this rank, 0..W-1                        */
    uint32_t epoch;                /* 1, 2, 3, ... identical on every rank     */
    int64_t  M;
    int64_t  D;
    float    eps;
    int32_t  reserved0;            /* must be 0                                */
    const void* partial[FARQ_AR_MAX_WORLD];      /* [M, D] per rank           */
    const void* residual;                        /* [M, D] on this rank       */
    const void* gamma;                           /* [D] on this rank          */
    void*    residual_out[FARQ_AR_MAX_WORLD];    /* [M, D] per rank           */
    void*    norm_out[FARQ_AR_MAX_WORLD];        /* [M, D] per rank, or all NULL */
    void*    x_q[FARQ_AR_MAX_WORLD];             /* [M, D] per rank           */
    float*   x_scale[FARQ_AR_MAX_WORLD];         /* [M, D/G] per rank         */
    uint32_t* signal[FARQ_AR_MAX_WORLD];         /* per rank                  */
    int32_t* status;                             /* device int or NULL        */
} farq_ar_args_t;

/* Launch the fused all-reduce + operator on `stream` of the current device.
 * Returns a farq_status; validation errors are reported before any launch. */
int farq_ar_launch(const farq_ar_args_t* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FARQ_H */
