/* cusr_co.h — C ABI of the cusr-b200 batched Levenberg–Marquardt constant-fitting engine.
 *
 * One shared library, libcusr_b200.so (also installed under the names the CuSR loader
 * expects, see below), exports:
 *
 *   - the four entry points of the reference in-process drop-in, with identical
 *     signatures, argument meaning and return codes, so the reference's ctypes loader
 *     binds this library unchanged:
 *         co_init        replaces cusr/kernel/co_lib.h:45   (co_lib.cu:165-183)
 *         co_optimize    replaces cusr/kernel/co_lib.h:56-63 (co_lib.cu:188-521)
 *         co_last_split  replaces cusr/kernel/co_lib.h:70    (co_lib.cu:531-541)
 *         co_teardown    replaces cusr/kernel/co_lib.h:73    (co_lib.cu:549-568)
 *   - co_optimize_ex / co_get_stats: the extended entry (precision, shared targets,
 *     damping / tolerance knobs, fp64 outputs, per-tree iteration counts, timings).
 *
 * libcusr_co_ad.so is this library under the AD variant's name; libcusr_co_fd.so is a small
 * library of its own whose co_optimize has the FD variant's acceptance order
 * (CoOptions.fd_ordering) and which takes every other symbol from this one.
 *
 * pop.bin structures (PopHeader 64 B, TreeMeta 16 B) keep the byte layout of
 * cusr/kernel/pop_format.h:32-51 because the file format and the ABI carry them.
 *
 * All pointers are HOST pointers, borrowed for the duration of the call; outputs are
 * caller-allocated. Calls are synchronous. A handle is bound to one device and is not
 * re-entrant (one call at a time per handle). No entry point ever exits the process.
 */
#ifndef CUSR_CO_H
#define CUSR_CO_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define POP_MAGIC   0x4D4C344D   /* 'M' '4' 'L' 'M' little-endian */
#define POP_VERSION 1

/* 64-byte population header (pop_format.h:32-43). */
typedef struct PopHeader {
    int32_t magic;
    int32_t version;
    int32_t M_prob;        /* number of trees                              */
    int32_t total_nodes;   /* sum of n_nodes                               */
    int32_t total_c;       /* sum of K                                     */
    int32_t N;             /* samples                                      */
    int32_t n_vars;        /* input variables                              */
    int32_t K_max;         /* max K over trees                             */
    int32_t max_stack;     /* max evaluation-stack depth                   */
    int32_t reserved[7];
} PopHeader;

/* 16-byte per-tree record (pop_format.h:45-51). */
typedef struct TreeMeta {
    int32_t node_offset;
    int32_t n_nodes;
    int32_t c_offset;
    int32_t K;
} TreeMeta;

/* Return codes (co_lib.h:35-41, plus -6 for malformed bytecode). */
#define CO_OK              0
#define CO_ERR_BOUNDS      2   /* K_max > 32, max_stack > 64, or beyond an engine limit */
#define CO_ERR_CUDA       -1   /* a CUDA runtime call failed                            */
#define CO_ERR_SUM_C      -2   /* sum(K) != header.total_c                              */
#define CO_ERR_SUM_NODES  -3   /* sum(n_nodes) != header.total_nodes                    */
#define CO_ERR_NULLARG    -4   /* null pointer / bad argument                           */
#define CO_ERR_OOM        -5   /* device or host allocation failed                      */
#define CO_ERR_BADTREE    -6   /* malformed tree: unknown node type, stack underflow,
                                  var index >= n_vars, const rank outside [0,K)          */

/* Per-tree status written to status_out (lm_core.cuh:46-56). */
#define STATUS_CONVERGED      0
#define STATUS_MAXITER        1
#define STATUS_FAIL_NAN       2
#define STATUS_K0_SKIP        3
#define STATUS_FAIL_CHOLESKY  4

/* Engine limits (the reference's are K<=32, stack<=64, nodes<=128). */
#define CO_MAX_K        32
#define CO_MAX_STACK    64    /* header.max_stack bound, as in the reference          */
#define CO_MAX_NODES    1023  /* per tree                                              */
#define CO_MAX_VARS     255
#define CO_MAX_DEVICES  8     /* devices of one multi-device call (CoOptions.device_ids)     */

/* ---- reference-compatible entry points ------------------------------------------ */

/* Bind device `device_id`, create its primary context once, return an opaque handle.
 * 0 OK; CO_ERR_NULLARG if handle_out is NULL; CO_ERR_CUDA if the device is unusable. */
int  co_init(int device_id, void **handle_out);

/* One batched LM fit (fp32 arithmetic, like the reference AD variant) of the population
 * described by `header` and the arrays that follow (pop.bin layout). `ym` is [M_prob][N];
 * rows that are all identical are detected and kept once on the device.
 * Outputs: c_final_out[total_c], status_out[M_prob], loss_init_out[M_prob] and
 * loss_final_out[M_prob] (both 0.5*sum(r^2); either may be NULL).
 * Every call starts from c_init (no state carries over between calls). */
int  co_optimize(void *handle, const PopHeader *header,
                 const int32_t *nt, const float *nv, const int32_t *ci,
                 const TreeMeta *metas,
                 const float *c_init, const float *xs, const float *ym,
                 int max_iter,
                 float *c_final_out, int32_t *status_out,
                 float *loss_init_out, float *loss_final_out);

/* Setup / loop wall-clock split (ms) of the last co_optimize* call in this process.
 * Always returns 0 and fills both (the engine always times its phases). */
int  co_last_split(double *setup_ms_out, double *loop_ms_out);

/* Free every device and host buffer of the handle. Safe on NULL. */
void co_teardown(void *handle);

/* ---- extended entry ---------------------------------------------------------------- */

#define CO_PREC_FP32 0
#define CO_PREC_FP64 1
/* fp32 with the reference kernel's numerics: the interpreter is compiled with its
 * --use_fast_math flags (hardware sin/cos/exp/log/pow approximations, approximate division and
 * square root, denormals flushed), as cusr/kernel/Makefile:9 builds batch_lm_ad. The LM step
 * and the fp64 audit are unchanged. */
#define CO_PREC_FP32_FAST 2

typedef struct CoOptions {
    int32_t struct_size;    /* sizeof(CoOptions); lets the struct grow compatibly      */
    int32_t precision;      /* CO_PREC_FP32 (default), CO_PREC_FP64, CO_PREC_FP32_FAST */
    int32_t max_iter;       /* LM iterations (reference default 50)                    */
    int32_t y_shared;       /* 1: ym points at ONE row of N targets shared by all trees;
                               0: ym is [M_prob][N] (identical rows are still detected) */
    double  lambda0;        /* initial Marquardt damping (reference 1e-3)              */
    double  xtol;           /* step test |d| < xtol(|c_try| + xtol) (reference 1e-6)    */
    int32_t fp64_audit;     /* -1 auto (on for fp32, off for fp64), 0 off, 1 on        */
    int32_t early_exit;     /* 1 (default): stop launching once every tree is finished */
    int32_t sample_sharded; /* 1: all-reduce over the co_shard_init group (set by      */
                            /* co_optimize_sharded; honoured by co_fit_loaded; ignored  */
                            /* by co_optimize_ex)                                       */
    int32_t keep_inputs;    /* 1: reuse the inputs X and the SHARED target row resident  */
                            /* from the previous call on this handle (same N, n_vars);   */
                            /* xs / ym are not read and may be NULL. In-loop callers     */
                            /* (new trees and c_init every generation, fixed data) skip  */
                            /* the re-upload. CO_ERR_NULLARG if nothing compatible is    */
                            /* resident. (co_optimize_ex, co_optimize_sharded, co_load)  */
    int32_t ad_mode;        /* Jacobian: CO_AD_AUTO (reverse mode everywhere: measured   */
                            /* fastest on B200), CO_AD_FORWARD (forward-mode tangents    */
                            /* for K <= 2, reverse above), CO_AD_REVERSE                 */
    int32_t damping_always; /* with damping_floor > 0: 1 = always the floored damping    */
    double  damping_floor;  /* 0 (default): the reference Marquardt damping only,        */
                            /* diag *= 1+lam (a zero Jacobian column -> FAIL_CHOLESKY).   */
                            /* f > 0: a system that damping cannot factor is retried with */
                            /* diag + lam * max(diag, f * max(diag)) (robust fits)        */
    /* ---- algorithm and start axis (fields past this point take their defaults when ---- */
    /* ---- struct_size ends before them) ---------------------------------------------- */
    int32_t algorithm;      /* CO_ALG_REFERENCE (default): the reference LM schedule      */
                            /* (lambda x0.1 / x10, co_lib.cu:438-455); CO_ALG_TRUST_REGION:*/
                            /* the trust-region LM of MINPACK lmder (More 1977), the       */
                            /* algorithm of the reference's scipy backend; max_iter then   */
                            /* bounds function evaluations per fit, the first included     */
                            /* (scipy's max_nfev); xtol / ftol / gtol are MINPACK's         */
    int32_t n_starts;       /* fits per tree (0 or 1: one, from c_init). S > 1: start 0 is  */
                            /* c_init, starts 1.. are points around it and fresh draws,     */
                            /* generated on the device from start_seed; the programs are    */
                            /* compiled and stored once per tree; every output is the start */
                            /* with the lowest final loss (fp64 audit loss for fp32 fits)  */
    int32_t tr_starts;      /* > 0: starts 0 .. tr_starts-1 use the trust-region LM, the    */
                            /* others the reference schedule (with damping_floor as a       */
                            /* fallback, every second one with the floored damping always); */
                            /* 0: `algorithm` applies to every start                        */
    int32_t wave1;          /* 0: all starts at once. W in (0, n_starts): starts 0..W-1 run */
                            /* first; a tree whose first-wave fits agree (two or more within */
                            /* agree_tol of the best) retires its other starts unrun, the  */
                            /* others start them                                           */
    double  ftol;           /* trust region: relative reduction tolerance (default 1e-10)   */
    double  gtol;           /* trust region: gradient tolerance (default 1e-8, scipy's)     */
    double  agree_tol;      /* wave agreement, relative (default 1e-7)                      */
    uint64_t start_seed;    /* start points (default 0)                                     */
    int32_t fd_ordering;    /* reference schedule, 1: the FD variant's acceptance order     */
                            /* (co_lib.cu:456-471): a step below xtol is CONVERGED and kept */
                            /* before the improvement test, improvement is strict (<);      */
                            /* 0 (default): the AD variant's (improvement first, <=)        */
    int32_t n_devices;      /* co_optimize_ex: 0 / 1 = the handle's device. 2..8: the trees */
                            /* are split into cost-balanced shards (longest first on        */
                            /* nodes x (1 + K)) fitted concurrently on device_ids[0..n-1],  */
                            /* one host thread and context each (the handle's own where a   */
                            /* listed device is its device), outputs in the caller's order  */
    int32_t device_ids[CO_MAX_DEVICES];
    int32_t tr_dd;          /* 1: trust-region fits (fp64 only) form and factor their normal  */
                            /* equations in double-double: J^T J keeps the small singular     */
                            /* directions of Jacobians rank-deficient to machine precision,   */
                            /* as MINPACK's QR of J does. Per-sample values and Jacobians of  */
                            /* the fits are kept on the device (fits x K_max x N doubles).    */
    int32_t reserved[1];
} CoOptions;

#define CO_AD_AUTO    0
#define CO_AD_FORWARD 1
#define CO_AD_REVERSE 2

#define CO_ALG_REFERENCE    0
#define CO_ALG_TRUST_REGION 1
#define CO_MAX_STARTS       1024

/* Fill `opt` with the reference defaults (fp32, 50 iterations, lambda0 1e-3, xtol 1e-6,
 * audit auto, early exit on, the reference schedule, one start; trust-region tolerances
 * ftol 1e-10, gtol 1e-8; wave agreement 1e-7). */
void co_default_options(CoOptions *opt);

/* Extended fit. Same inputs as co_optimize (ym may be a single shared row, see
 * CoOptions.y_shared); outputs are fp64 so fp64 fits lose nothing. iters_out[M_prob]
 * (may be NULL) receives the LM iterations each tree consumed. */
int  co_optimize_ex(void *handle, const PopHeader *header,
                    const int32_t *nt, const float *nv, const int32_t *ci,
                    const TreeMeta *metas,
                    const float *c_init, const float *xs, const float *ym,
                    const CoOptions *opt,
                    double *c_final_out, int32_t *status_out,
                    double *loss_init_out, double *loss_final_out,
                    int32_t *iters_out);

typedef struct CoStats {
    double  setup_ms;       /* entry .. first LM iteration (pack, H2D, initial pass)   */
    double  loop_ms;        /* LM iterations                                            */
    double  finish_ms;      /* audit + D2H                                              */
    double  eval_ms;        /* device time of the fused evaluation kernels (events)     */
    double  step_ms;        /* device time of the per-tree LM step kernels (events)     */
    double  device_ms;      /* device time of the whole fit: init .. last D2H (events)  */
    double  flops;          /* algorithmic FP work: per evaluated (tree, sample) 2 flops per
                               operator node (value + adjoint) + 2 per normal-equation
                               entry ((K+1)(K+2)/2)                                      */
    int64_t node_evals;     /* sum_m n_nodes(m) * N * (1 + evaluated trials of m)       */
    int64_t sample_evals;   /* sum_m N * (1 + evaluated trials of m)                    */
    int64_t eval_launches;  /* fused evaluation kernel launches                         */
    int64_t kernel_launches;/* all kernel launches of the call                          */
    int32_t iters_run;      /* LM iterations launched                                   */
    int32_t n_bins;         /* scheduler bins used                                      */
    int32_t y_shared;       /* 1 if targets were kept as one shared row                 */
    int32_t precision;      /* CO_PREC_* of the call                                    */
    int32_t n_reverted;     /* fits reverted to their start by the fp64 audit           */
    int32_t n_starts;       /* fits per tree of the call                                */
    int64_t fits_run;       /* fits (tree x start) evaluated at least once              */
    int32_t trees_retired;  /* trees whose later starts were retired unrun (wave1)      */
    int32_t reserved0;
    double  comm_ms;        /* sample-sharded mode: device time of the per-pass chunk sum
                               and NCCL all-reduce (events; waiting for the slowest rank
                               included); 0 otherwise. eval_ms excludes it               */
} CoStats;

/* Resident problem: co_load compiles, schedules and uploads a population (programs,
 * inputs, targets, c_init) into the handle's device buffers in the given precision;
 * co_fit_loaded then runs a complete LM fit from the loaded c_init with every input
 * already in HBM, as often as needed (the next co_load / co_optimize* / co_evaluate call
 * replaces the resident problem). opt->precision must match the loaded precision;
 * opt->y_shared applies to co_load. Outputs as co_optimize_ex. */
int  co_load(void *handle, const PopHeader *header,
             const int32_t *nt, const float *nv, const int32_t *ci,
             const TreeMeta *metas,
             const float *c_init, const float *xs, const float *ym,
             const CoOptions *opt);
int  co_fit_loaded(void *handle, const CoOptions *opt,
                   double *c_final_out, int32_t *status_out,
                   double *loss_init_out, double *loss_final_out,
                   int32_t *iters_out);

/* ---- sample-sharded mode (one process per GPU, samples split across ranks) ----------- */

/* A 128-byte id for a new group of ranks: created on one rank, shared with the others by any
 * means (e.g. torch.distributed broadcast). Needs NCCL (loaded at run time). */
int  co_shard_unique_id(unsigned char id_out[128]);

/* Join the group as `rank` of `nranks` on the handle's device. Every later wait of a
 * sharded fit is bounded by timeout_s: a peer that fails or never arrives makes the call
 * return CO_ERR_CUDA (the communicator is aborted) instead of hanging. */
int  co_shard_init(void *handle, const unsigned char id[128], int nranks, int rank,
                   double timeout_s);

/* Sample-sharded fit: every rank passes the WHOLE population (same trees, same c_init) but
 * only its own slice of the samples (header->N = local sample count; xs / ym hold those
 * samples). Per-tree JtJ / Jtr / 0.5*sum r^2 are all-reduced each iteration (and the fp64
 * audit losses once), so all ranks take identical steps and return identical outputs, equal
 * to one fit over all samples up to the order of the floating-point sums.
 * (No counterpart in the reference, which has no multi-GPU path.) */
int  co_optimize_sharded(void *handle, const PopHeader *header,
                         const int32_t *nt, const float *nv, const int32_t *ci,
                         const TreeMeta *metas,
                         const float *c_init, const float *xs, const float *ym,
                         const CoOptions *opt,
                         double *c_final_out, int32_t *status_out,
                         double *loss_init_out, double *loss_final_out,
                         int32_t *iters_out);

/* Finite-difference Jacobian (the reference FD variant's forward difference,
 * batch_lm_ad.cu:95-132): for each constant column k, h = eps*|c_k| (eps when c_k == 0),
 * taken as the representable step (c_k + h) - c_k, and J[m][k][i] = (f(c + h e_k; x_i) -
 * f(c; x_i)) / h, evaluated on the device by value passes of the same interpreter. jac_out is
 * [M_prob][K_max][N] fp64 (rows k >= K are 0). eps <= 0 selects 1e-3 (fp32, the reference's
 * eps_rel) or 1e-7 (fp64). An independent check of the reverse-mode Jacobian. */
int  co_jacobian_fd(void *handle, const PopHeader *header,
                    const int32_t *nt, const float *nv, const int32_t *ci,
                    const TreeMeta *metas, const double *c,
                    const float *xs, const float *ym, int precision, int y_shared,
                    double eps, double *jac_out);

/* The start each tree's outputs of the last fit on `handle` came from (0 = its c_init), for
 * fits with CoOptions.n_starts > 1; start_out[M_prob] of that fit. (No counterpart in the
 * reference, which fits every tree once.) */
int  co_last_starts(void *handle, int32_t *start_out);

/* Statistics of the last co_optimize* / co_fit_loaded call on `handle`. */
int  co_get_stats(void *handle, CoStats *out);

/* Evaluate every tree at the constants c[total_c] (fp64 in; computed in `precision`) and
 * return any of (NULL skips an output):
 *   vals_out   [M_prob][N]        tree value at each sample
 *   jac_out    [M_prob][K_max][N] df/dc_k at each sample (the reference d_J layout,
 *                                 cusr/kernel/ad_interp.cuh:240-244; rows k >= K stay 0)
 *   blocks_out per tree in tree order, (K+1)(K+2)/2 values: JtJ lower triangle packed
 *              row-major, Jtr, 0.5*sum r^2 (r = f - y)
 * This is the same fused device pass the fit runs every iteration (no counterpart entry in
 * the reference, whose eval_kernel_batched / *_jacobian_kernel are internal). */
int  co_evaluate(void *handle, const PopHeader *header,
                 const int32_t *nt, const float *nv, const int32_t *ci,
                 const TreeMeta *metas, const double *c, const float *xs, const float *ym,
                 int precision, int y_shared,
                 double *vals_out, double *jac_out, double *blocks_out);

/* Measured FMA throughput of the bound device (independent FMA chains, no memory traffic):
 * the FP32 / FP64 non-tensor peak the engine's roofline is reported against. */
int  co_probe_peak(void *handle, double *fp32_tflops, double *fp64_tflops);

/* Allocation-free evaluation (no counterpart in the reference). For callers that cannot
 * allocate device memory — their GPU memory is owned by their own pool allocator, or they
 * cannot afford the device-wide synchronisation of cudaMalloc/cudaFree inside their loop.
 * Same fused pass as co_evaluate (fp32 normal-equation blocks only), but every scratch buffer
 * (compiled programs, descriptors, work lists, counters, transposed inputs, the padded target
 * row, per-chunk partial sums) lives in one fixed 32 MiB device array inside the library; the
 * call makes no cudaMalloc / cudaFree or other allocating CUDA call.
 *   header, nt, nv, ci, metas  HOST pointers (pop.bin layout; compiled on the host)
 *   c_dev                      DEVICE float[total_c] constants
 *   xs_dev                     DEVICE float[N][n_vars] inputs (pop.bin layout)
 *   y_dev                      DEVICE float[N], one target row shared by every tree
 *   blocks_dev                 DEVICE float output, per tree in tree order (K+1)(K+2)/2
 *                              values: JtJ lower triangle, Jtr, 0.5*sum r^2
 *   stream                     cudaStream_t (NULL = legacy default stream)
 * Returns CO_ERR_BOUNDS when the population needs more than the fixed array or a tree's
 * reverse tape does not fit in shared memory. The first call on a device resolves the array's
 * device address (cudaGetSymbolAddress) and configures the kernels: make it before any stream
 * capture. Every call shares the one array and overwrites it; calls are serialised inside the
 * library and return after their work completes, because work of two calls overlapping on the
 * GPU would race on it. The caller's current device is restored on return. */
int  co_evaluate_noalloc(int device_id, const PopHeader *header,
                         const int32_t *nt, const float *nv, const int32_t *ci,
                         const TreeMeta *metas,
                         const float *c_dev, const float *xs_dev, const float *y_dev,
                         float *blocks_dev, void *stream);

/* Human-readable message for a return code (static storage). */
const char *co_strerror(int code);

#ifdef __cplusplus
}
#endif

#endif /* CUSR_CO_H */
