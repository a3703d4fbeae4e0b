// engine.cu — persistent per-device context, the per-call LM driver, and the C ABI
// (include/cusr_co.h).
//
// Per call (co_optimize / co_optimize_ex):
//   1. argument, sum and structure checks (before any device work; co_lib.cu:195-220);
//   2. compile every tree to a register-stack program and build the cost-binned schedule;
//   3. H2D of programs, inputs (transposed on device to [n_vars][N]) and targets (one row
//      when every tree shares it);
//   4. initial fused pass at c_init, then max_iter LM iterations, each
//        build work items of the pending trees -> one fused evaluation launch per bin
//        -> one LM-step launch (accept/reject, lambda, Cholesky solve of the next step),
//      with no host round trip inside the loop (a lagged counter read lets the host stop
//      launching once every tree has finished);
//   5. fp64 audit for fp32 fits; D2H of the outputs.
// The bins of a pass run concurrently on the context's bin streams (fork / join events on
// the context stream); each bin takes the narrow or the wide block instantiation, whichever
// keeps more warps resident. In the sample-sharded mode (co_optimize_sharded) the per-tree
// sums of every pass are all-reduced over the NCCL group before the step kernel reads them,
// and every wait is bounded by the group's deadline (shard_comm.h).
// Device buffers grow by byte capacity and never shrink (co_lib.cu:129-153); every call
// re-seeds all per-tree state from c_init (co_lib.cu:284-305).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "../../include/cusr_co.h"
#include "launch.h"
#include "lm_kernels.cuh"
#include "pack.h"
#include "shard_comm.h"
#include "starts.cuh"

namespace cusr {

namespace {

double g_last_setup_ms = -1.0, g_last_loop_ms = -1.0;

struct DBuf {
    void *ptr = nullptr;
    size_t cap = 0;
};

// Host + device state of one prepared problem (compiled programs, schedule, inputs on the
// device). Shared by the fit and the evaluation entry points.
struct Prep {
    PackResult pk;
    Schedule sc;
    int64_t ldx = 0, y_rows = 0;
    bool y_shared = false;
    // start axis: S fits per tree (fit i = tree i / S, start i % S); S = 1 is the plain fit
    int S = 1;
    int64_t M_fit = 0, total_c_fit = 0;
    std::vector<int32_t> tree_coff;   // per tree: offset of its constants in c_init
};

struct Ctx {
    int device = -1;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    // bins of one pass run on these streams concurrently, so one bin's tail overlaps the next
    static constexpr int kBinStreams = 8;
    cudaStream_t bin_streams[kBinStreams] = {};
    cudaEvent_t ev_fork = nullptr, ev_join[kBinStreams] = {};
    DBuf tape_gs[kBinStreams];
    DBuf code, desc, bin_trees, bin_tree_off, bin_item_off, items, n_items, counter;
    DBuf xs_raw, xs, ym;
    DBuf c, ctry, delta, cinit_f, lam, loss, loss_init, status, iters, pending, n_run, n_eval;
    DBuf partials, blk;
    DBuf c64, l64, n_rev;
    DBuf vals, jac;            // per-sample values / Jacobians (co_evaluate; tr_dd fits)
    DBuf dd_g, dd_blk;         // double-double sums of a pass / accepted blocks (tr_dd fits)
    // start axis and trust-region state (per fit), tree-level inputs and outputs
    DBuf c_tree, tree_coff, imode, tr, diag, outer, resolved, n_retired;
    DBuf out_c, out_status, out_li, out_lf, out_iters, out_start;
    int *h_nrun = nullptr;                  // pinned, one slot per iteration parity
    std::vector<int32_t> h_start;           // winning start per tree of the last fit
    std::vector<cudaEvent_t> events;        // timing events, reused across calls
    cudaEvent_t ev_nrun[2] = {nullptr, nullptr};
    bool step_attr_set[2] = {false, false};
    int smem_optin = 0;
    cudaEvent_t ev_fit[2] = {nullptr, nullptr};
    // resident problem (co_load / co_fit_loaded and every fit)
    Prep prep;
    PopHeader hdr{};
    std::vector<int32_t> n_nodes, n_ops;
    int prep_prec = -1;     // arithmetic type of the loaded problem (CO_PREC_FP32 / _FP64)
    bool fast = false;      // fp32 launches use the fast-math instantiations (CO_PREC_FP32_FAST)
    int wide_mode = -1;     // block width per bin: -1 by occupancy, 0 narrow, 1 wide
    int n_bin_streams = kBinStreams;   // streams the bins of a pass are spread over
    int fwd_max = 0;        // trees with K <= fwd_max use the forward-mode classes
    int fwd_default = 0;    // fwd_max of CO_AD_AUTO
    // the inputs resident in xs / ym (for CoOptions.keep_inputs)
    bool in_valid = false, in_shared = false;
    int in_N = -1, in_nvars = -1;
    bool loaded = false;
    // sample-sharded mode
    ShardComm shard;
    DBuf red;
    // multi-device fits (CoOptions.n_devices): the contexts of the other shards, by shard slot
    Ctx *peers[CO_MAX_DEVICES] = {};
    cudaEvent_t ev_sync = nullptr;
    CoStats stats{};
};

int grow(DBuf &b, size_t bytes) {
    if (bytes == 0) bytes = 16;
    if (bytes <= b.cap) return CO_OK;
    if (b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.cap = 0;
    cudaError_t e = cudaMalloc(&b.ptr, bytes);
    if (e != cudaSuccess) {
        fprintf(stderr, "[cusr_b200] cudaMalloc %zu B failed: %s\n", bytes, cudaGetErrorString(e));
        cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? CO_ERR_OOM : CO_ERR_CUDA;
    }
    b.cap = bytes;
    return CO_OK;
}

void release(DBuf &b) {
    if (b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.cap = 0;
}

#define CK(x)                                                                                \
    do {                                                                                     \
        cudaError_t _e = (x);                                                                \
        if (_e != cudaSuccess) {                                                             \
            fprintf(stderr, "[cusr_b200] CUDA error %s at %s:%d\n", cudaGetErrorString(_e),  \
                    __FILE__, __LINE__);                                                     \
            return CO_ERR_CUDA;                                                              \
        }                                                                                    \
    } while (0)
#define GROW(buf, bytes)                    \
    do {                                            \
        int _r = grow(buf, (size_t)(bytes));        \
        if (_r) return _r;                          \
    } while (0)

template <typename T> T *P(DBuf &b) { return reinterpret_cast<T *>(b.ptr); }

cudaEvent_t event_at(Ctx *ctx, size_t i) {
    while (ctx->events.size() <= i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
        ctx->events.push_back(e);
    }
    return ctx->events[i];
}

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// Output sinks of one call (float for the reference ABI, double for the extended one).
struct Outputs {
    float *c_f = nullptr, *li_f = nullptr, *lf_f = nullptr;
    double *c_d = nullptr, *li_d = nullptr, *lf_d = nullptr;
    int32_t *status = nullptr, *iters = nullptr;
};

struct Problem {
    const PopHeader *h;
    const int32_t *nt;
    const float *nv;
    const int32_t *ci;
    const TreeMeta *metas;
    const float *c_init, *xs, *ym;
    bool keep_inputs = false;   // X / shared y resident from the previous upload
};

int check_args(const Problem &pr) {
    const PopHeader *h = pr.h;
    if (h->M_prob < 0 || h->N < 0 || h->n_vars < 0 || h->total_c < 0 || h->total_nodes < 0)
        return CO_ERR_NULLARG;
    // reference bounds on the header fields (co_lib.cu:211-212)
    if (h->K_max > CO_MAX_K) return CO_ERR_BOUNDS;
    if (h->max_stack > CO_MAX_STACK) return CO_ERR_BOUNDS;
    if (h->n_vars > CO_MAX_VARS) return CO_ERR_BOUNDS;
    // sum checks before any device work (co_lib.cu:214-220)
    int64_t ks = 0, ns = 0;
    for (int m = 0; m < h->M_prob; ++m) {
        ks += pr.metas[m].K;
        ns += pr.metas[m].n_nodes;
    }
    if (ks != (int64_t)h->total_c) return CO_ERR_SUM_C;
    if (ns != (int64_t)h->total_nodes) return CO_ERR_SUM_NODES;
    return CO_OK;
}

// Evaluate the pending trees of every bin at constants `cdev` (one fused launch per bin).
template <typename T>
int launch_pass(Ctx *ctx, const Schedule &sc, const PackResult &pk, const T *cdev, T *partials,
                const PopHeader &hd, int64_t ldx, bool grad, T *vals = nullptr, T *jac = nullptr,
                int jac_kmax = 0, const uint8_t *imode = nullptr) {
    const int n_bins = (int)sc.bins.size();
    {
        ItemsParams ip;
        ip.desc = P<TreeDesc>(ctx->desc);
        ip.bin_trees = P<int32_t>(ctx->bin_trees);
        ip.bin_tree_off = P<int64_t>(ctx->bin_tree_off);
        ip.bin_item_off = P<int64_t>(ctx->bin_item_off);
        ip.pending = P<int32_t>(ctx->pending);
        ip.items = P<int2>(ctx->items);
        ip.n_items = P<int>(ctx->n_items);
        ip.counter = P<int>(ctx->counter);
        build_items_kernel<<<n_bins, ITEMS_THREADS, 0, ctx->stream>>>(ip);
        CK(cudaGetLastError());
        ctx->stats.kernel_launches++;
    }
    const int n_streams = std::min(n_bins, ctx->n_bin_streams);
    CK(cudaEventRecord(ctx->ev_fork, ctx->stream));
    for (int si = 0; si < n_streams; ++si) CK(cudaStreamWaitEvent(ctx->bin_streams[si], ctx->ev_fork, 0));
    for (int b = 0; b < n_bins; ++b) {
        const int si = b % n_streams;
        const Bin &bin = sc.bins[(size_t)b];
        EvalParams<T> p;
        p.code = P<uint32_t>(ctx->code);
        p.desc = P<TreeDesc>(ctx->desc);
        p.items = P<int2>(ctx->items) + bin.item_off;
        p.n_items = P<int>(ctx->n_items) + b;
        p.counter = P<int>(ctx->counter) + b;
        p.c = cdev;
        p.xs = P<float>(ctx->xs);
        p.ym = P<float>(ctx->ym);
        p.partials = partials;
        p.ldx = ldx;
        p.N = hd.N;
        p.chunk = sc.chunk;
        p.n_vars = hd.n_vars;
        p.code_cap = bin.max_instr;
        p.spill_cap = std::max(bin.max_spill, 1);
        p.tape_cap = grad ? std::max(bin.max_tape, 1) : 1;
        p.vals = vals;
        p.jac = jac;
        p.jac_kmax = jac_kmax;
        p.imode = imode;
        const int kc = grad ? bin.kc : 4;
        // Block width: the narrow (EVAL_NT) or the wide (EVAL_NT_WIDE) instantiation, whichever
        // keeps more warps resident (registers and shared memory both counted); a bin whose
        // items do not fill the narrow slots takes the wide blocks, which finish an item in
        // about half the time.
        struct Shape { bool tg; size_t smem; int occ; };
        auto shape = [&](bool w) -> Shape {
            Shape sh{false, Launch<T>::smem(kc, p.code_cap, p.n_vars, p.spill_cap, p.tape_cap, true, w), 0};
#ifdef CUSR_FORCE_GLOBAL_TAPE
            if (grad) {
#else
            // tape in shared memory unless that leaves room for fewer than two resident blocks
            if (grad && 2 * (sh.smem + 1024) > (size_t)ctx->smem_optin) {
#endif
                sh.tg = true;
                sh.smem = Launch<T>::smem(kc, p.code_cap, p.n_vars, p.spill_cap, p.tape_cap, false, w);
            }
            sh.occ = sh.smem + 64 > (size_t)ctx->smem_optin
                         ? 0 : Launch<T>::occ(kc, grad, sh.tg, ctx->fast, w, sh.smem);
            return sh;
        };
        const Shape nrw = shape(false);
        bool wide = false;
        Shape sh = nrw;
        if (grad && ctx->wide_mode != 0) {
            const Shape wd = shape(true);
            const int64_t warps_n = (int64_t)nrw.occ * EVAL_NT / 32, warps_w = (int64_t)wd.occ * EVAL_NT_WIDE / 32;
            if (wd.occ > 0 &&
                (ctx->wide_mode == 1 || warps_w >= warps_n ||
                 bin.max_items < (int64_t)nrw.occ * ctx->sm_count)) {
                wide = true;
                sh = wd;
            }
        }
        if (sh.occ < 1 && sh.smem + 64 > (size_t)ctx->smem_optin) return CO_ERR_BOUNDS;
        const int nt = wide ? EVAL_NT_WIDE : EVAL_NT;
        const bool tg = sh.tg;
        const size_t smem = sh.smem;
        int occ = sh.occ;
        if (occ < 1) occ = 1;
        int64_t grid = (int64_t)occ * ctx->sm_count;
        if (grid > bin.max_items) grid = std::max<int64_t>(1, bin.max_items);
        p.tape_g = nullptr;
        if (tg) {
            // one global tape per stream: bins on different streams run concurrently
            GROW(ctx->tape_gs[si], (size_t)grid * p.tape_cap * nt * EVAL_V * sizeof(T));
            p.tape_g = ctx->tape_gs[si].ptr;
        }
        CK(Launch<T>::eval(kc, grad, tg, ctx->fast, wide, p, (int)grid, smem, ctx->bin_streams[si]));
        ctx->stats.eval_launches++;
        ctx->stats.kernel_launches++;
    }
    for (int si = 0; si < n_streams; ++si) {
        CK(cudaEventRecord(ctx->ev_join[si], ctx->bin_streams[si]));
        CK(cudaStreamWaitEvent(ctx->stream, ctx->ev_join[si], 0));
    }
    (void)pk;
    return CO_OK;
}

template <typename T>
int prepare(Ctx *ctx, const Problem &pr, bool y_shared_in, Prep &pp, int S = 1) {
    const PopHeader *h = pr.h;
    const int M = h->M_prob, N = h->N, n_vars = h->n_vars;
    const int64_t total_c = h->total_c;
    const bool fp64 = sizeof(T) == 8;
    CoStats &st = ctx->stats;

    // ---- compile + schedule (host) ----
    int rc = compile_population(h, pr.nt, pr.nv, pr.ci, pr.metas, &pp.pk);
    if (rc != CO_OK) return rc;
    // start axis: S fits per tree sharing its program, constants of their own
    S = std::max(1, S);
    if ((int64_t)M * S > INT32_MAX / 2) return CO_ERR_BOUNDS;
    pp.S = S;
    pp.M_fit = (int64_t)M * S;
    pp.tree_coff.resize((size_t)M);
    for (int m = 0; m < M; ++m) pp.tree_coff[(size_t)m] = pr.metas[m].c_offset;
    PackResult pk_fit;
    std::vector<TreeMeta> metas_fit;
    const PackResult *pks = &pp.pk;
    const TreeMeta *ms = pr.metas;
    pp.total_c_fit = total_c;
    if (S > 1) {
        pk_fit.trees.reserve((size_t)pp.M_fit);
        metas_fit.reserve((size_t)pp.M_fit);
        int64_t coff = 0;
        for (int m = 0; m < M; ++m)
            for (int s_ = 0; s_ < S; ++s_) {
                pk_fit.trees.push_back(pp.pk.trees[(size_t)m]);
                TreeMeta tm = pr.metas[m];
                tm.c_offset = (int32_t)coff;
                coff += tm.K;
                metas_fit.push_back(tm);
            }
        if (coff > INT32_MAX) return CO_ERR_BOUNDS;
        pp.total_c_fit = coff;
        pks = &pk_fit;
        ms = metas_fit.data();
    }
    const int M_fit = (int)pp.M_fit;
    const int64_t total_c_fit = pp.total_c_fit;
    if (pr.keep_inputs &&
        !(ctx->in_valid && ctx->in_shared && ctx->in_N == N && ctx->in_nvars == n_vars))
        return CO_ERR_NULLARG;
    // shared targets: an explicit single row, or every row equal to row 0
    bool y_shared = y_shared_in || pr.keep_inputs;
    if (!y_shared && N > 0 && M > 0) {
        y_shared = true;
        const size_t rb = (size_t)N * sizeof(float);
        for (int m = 1; m < M && y_shared; ++m)
            if (std::memcmp(pr.ym, pr.ym + (size_t)m * N, rb) != 0) y_shared = false;
    }
    pp.y_shared = y_shared;
    st.y_shared = y_shared ? 1 : 0;
    const int round = EVAL_ROUND;
    Schedule &sc = pp.sc;
    build_schedule(*pks, ms, M_fit, N, y_shared, fp64, round, ctx->sm_count * 3, &sc,
                   ctx->fwd_max, S);
    st.n_bins = (int)sc.bins.size();
    pp.ldx = ((int64_t)N + round - 1) / round * round;
    pp.y_rows = y_shared ? 1 : M;
    const int64_t ldx = pp.ldx, y_rows = pp.y_rows;

    // ---- device buffers (grow-only) ----
    CK(cudaSetDevice(ctx->device));
    GROW(ctx->code, pp.pk.code.size() * sizeof(uint32_t));
    GROW(ctx->desc, (size_t)M_fit * sizeof(TreeDesc));
    GROW(ctx->bin_trees, (size_t)M_fit * sizeof(int32_t));
    GROW(ctx->bin_tree_off, (sc.bins.size() + 1) * sizeof(int64_t));
    GROW(ctx->bin_item_off, sc.bins.size() * sizeof(int64_t));
    GROW(ctx->items, (size_t)sc.total_items * sizeof(int2));
    GROW(ctx->n_items, sc.bins.size() * sizeof(int));
    GROW(ctx->counter, sc.bins.size() * sizeof(int));
    GROW(ctx->xs_raw, (size_t)N * n_vars * sizeof(float));
    GROW(ctx->xs, (size_t)n_vars * ldx * sizeof(float));
    GROW(ctx->ym, (size_t)y_rows * ldx * sizeof(float));
    GROW(ctx->c, total_c_fit * sizeof(T));
    GROW(ctx->ctry, total_c_fit * sizeof(T));
    GROW(ctx->delta, total_c_fit * sizeof(T));
    GROW(ctx->cinit_f, total_c_fit * sizeof(float));
    GROW(ctx->diag, total_c_fit * sizeof(double));
    GROW(ctx->lam, (size_t)M_fit * sizeof(T));
    GROW(ctx->loss, (size_t)M_fit * sizeof(T));
    GROW(ctx->loss_init, (size_t)M_fit * sizeof(T));
    GROW(ctx->status, (size_t)M_fit * sizeof(int32_t));
    GROW(ctx->iters, (size_t)M_fit * sizeof(int32_t));
    GROW(ctx->pending, (size_t)M_fit * sizeof(int32_t));
    GROW(ctx->n_eval, (size_t)M_fit * sizeof(int32_t));
    GROW(ctx->outer, (size_t)M_fit * sizeof(int32_t));
    GROW(ctx->imode, (size_t)M_fit);
    GROW(ctx->tr, (size_t)M_fit * TR_FIELDS * sizeof(double));
    GROW(ctx->n_run, 2 * sizeof(int));
    GROW(ctx->c_tree, total_c * sizeof(float));
    GROW(ctx->tree_coff, (size_t)M * sizeof(int32_t));
    GROW(ctx->resolved, (size_t)M);
    GROW(ctx->n_retired, sizeof(int));
    GROW(ctx->out_c, total_c * sizeof(T));
    GROW(ctx->out_status, (size_t)M * sizeof(int32_t));
    GROW(ctx->out_li, (size_t)M * sizeof(T));
    GROW(ctx->out_lf, (size_t)M * sizeof(T));
    GROW(ctx->out_iters, (size_t)M * sizeof(int32_t));
    GROW(ctx->out_start, (size_t)M * sizeof(int32_t));
    GROW(ctx->partials, (size_t)sc.partial_elems * sizeof(T));
    GROW(ctx->blk, (size_t)sc.block_elems * sizeof(T));

    // ---- H2D ----
    cudaStream_t s = ctx->stream;
    std::vector<int32_t> bin_trees;
    std::vector<int64_t> bin_tree_off, bin_item_off;
    bin_trees.reserve((size_t)M_fit);
    for (const Bin &b : sc.bins) {
        bin_tree_off.push_back((int64_t)bin_trees.size());
        bin_item_off.push_back(b.item_off);
        bin_trees.insert(bin_trees.end(), b.trees.begin(), b.trees.end());
    }
    bin_tree_off.push_back((int64_t)bin_trees.size());
    if (!pp.pk.code.empty())
        CK(cudaMemcpyAsync(ctx->code.ptr, pp.pk.code.data(), pp.pk.code.size() * sizeof(uint32_t),
                           cudaMemcpyHostToDevice, s));
    if (M > 0) {
        CK(cudaMemcpyAsync(ctx->desc.ptr, sc.desc.data(), (size_t)M_fit * sizeof(TreeDesc),
                           cudaMemcpyHostToDevice, s));
        CK(cudaMemcpyAsync(ctx->tree_coff.ptr, pp.tree_coff.data(), (size_t)M * sizeof(int32_t),
                           cudaMemcpyHostToDevice, s));
        CK(cudaMemcpyAsync(ctx->bin_trees.ptr, bin_trees.data(),
                           bin_trees.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    }
    CK(cudaMemcpyAsync(ctx->bin_tree_off.ptr, bin_tree_off.data(),
                       bin_tree_off.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    if (!bin_item_off.empty())
        CK(cudaMemcpyAsync(ctx->bin_item_off.ptr, bin_item_off.data(),
                           bin_item_off.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    if (pr.keep_inputs) {
        // X and the shared row are already in xs / ym, in this layout (same N, n_vars)
    } else {
    ctx->in_valid = false;
    if ((size_t)N * n_vars > 0) {
        CK(cudaMemcpyAsync(ctx->xs_raw.ptr, pr.xs, (size_t)N * n_vars * sizeof(float),
                           cudaMemcpyHostToDevice, s));
        transpose_x_kernel<<<std::max(1, std::min(4 * ctx->sm_count,
                                                  (int)((n_vars * ldx + 255) / 256))),
                             256, 0, s>>>(P<float>(ctx->xs_raw), N, n_vars, ldx, P<float>(ctx->xs));
        CK(cudaGetLastError());
        st.kernel_launches++;
    }
    CK(cudaMemsetAsync(ctx->ym.ptr, 0, (size_t)y_rows * ldx * sizeof(float), s));
    if (N > 0 && y_rows > 0) {
        CK(cudaMemcpy2DAsync(ctx->ym.ptr, (size_t)ldx * sizeof(float), pr.ym,
                             (size_t)N * sizeof(float), (size_t)N * sizeof(float), (size_t)y_rows,
                             cudaMemcpyHostToDevice, s));
    }
    ctx->in_valid = true;
    ctx->in_shared = y_shared;
    ctx->in_N = N;
    ctx->in_nvars = n_vars;
    }
    // the caller's c_init, per tree; the fits' start points are made from it on the device
    if (total_c > 0)
        CK(cudaMemcpyAsync(ctx->c_tree.ptr, pr.c_init, total_c * sizeof(float),
                           cudaMemcpyHostToDevice, s));
    return CO_OK;
}

inline int grid_for(Ctx *ctx, int64_t n) {
    return (int)std::max<int64_t>(1, std::min<int64_t>(4 * ctx->sm_count, (n + 255) / 256));
}

// Wait for all work queued on the context stream; in the sample-sharded mode the wait is
// bounded by the group's deadline (a failed peer would otherwise stall the all-reduce).
int sync_stream(Ctx *ctx, bool sharded) {
    if (!sharded) {
        CK(cudaStreamSynchronize(ctx->stream));
        return CO_OK;
    }
    CK(cudaEventRecord(ctx->ev_sync, ctx->stream));
    return shard_wait_event(ctx->shard, ctx->ev_sync);
}

// chunks per tree from which the step's chunk sums run as their own block-parallel kernel
constexpr int64_t PRESUM_CHUNKS = 64;
// largest per-sample Jacobian kept for double-double trust-region fits (fits x K_max x N x 8 B)
constexpr double DD_JAC_MAX_BYTES = 64.0 * (1 << 30);

// Per-tree sums of the chunk partials into ctx->red (chunk_sum_kernel).
template <typename T>
int chunk_sums(Ctx *ctx, int M, int64_t block_elems, cudaStream_t s) {
    GROW(ctx->red, (size_t)block_elems * sizeof(T));
    const int grid = std::max(1, std::min(M, 8 * ctx->sm_count));
    chunk_sum_kernel<T><<<grid, CSUM_THREADS, 0, s>>>(P<TreeDesc>(ctx->desc), M,
                                                      P<T>(ctx->partials), P<T>(ctx->red));
    CK(cudaGetLastError());
    ctx->stats.kernel_launches++;
    return CO_OK;
}

// Sample-sharded mode: sum this rank's chunk partials per tree and all-reduce them.
template <typename T>
int shard_reduce_blocks(Ctx *ctx, int M, int64_t block_elems) {
    const int rc = chunk_sums<T>(ctx, M, block_elems, ctx->stream);
    if (rc) return rc;
    return shard_allreduce(ctx->shard, ctx->red.ptr, (size_t)block_elems, sizeof(T) == 8,
                           ctx->stream);
}


// Compile, schedule and upload a problem; it stays resident in the context until the next
// load (inputs in HBM across fits).
template <typename T>
int load(Ctx *ctx, const Problem &pr, bool y_shared, int S = 1) {
    ctx->loaded = false;
    ctx->stats = CoStats{};
    ctx->stats.precision = sizeof(T) == 8 ? CO_PREC_FP64 : CO_PREC_FP32;
    int rc = prepare<T>(ctx, pr, y_shared, ctx->prep, S);
    if (rc != CO_OK) return rc;
    ctx->hdr = *pr.h;
    ctx->n_nodes.resize((size_t)pr.h->M_prob);
    ctx->n_ops.resize((size_t)pr.h->M_prob);
    for (int m = 0; m < pr.h->M_prob; ++m) {
        const TreeMeta &tm = pr.metas[m];
        ctx->n_nodes[(size_t)m] = tm.n_nodes;
        int ops = 0;
        for (int i = 0; i < tm.n_nodes; ++i) {
            const int t = pr.nt[tm.node_offset + i];
            ops += (t == NT_UFUNC || t == NT_BFUNC) ? 1 : 0;
        }
        ctx->n_ops[(size_t)m] = ops;
    }
    ctx->prep_prec = ctx->stats.precision;
    ctx->loaded = true;
    return CO_OK;
}

// One LM fit of the loaded problem, from its c_init.
template <typename T>
int fit_loaded(Ctx *ctx, const CoOptions &opt, const Outputs &out,
               std::chrono::steady_clock::time_point t_entry) {
    const PopHeader *h = &ctx->hdr;
    const int M = h->M_prob, N = h->N;
    const int64_t total_c = h->total_c;
    const bool fp64 = sizeof(T) == 8;
    CoStats &st = ctx->stats;
    const int keep_bins = st.n_bins, keep_ys = st.y_shared;
    st = CoStats{};
    st.n_bins = keep_bins;
    st.y_shared = keep_ys;
    st.precision = fp64 ? CO_PREC_FP64 : (ctx->fast ? CO_PREC_FP32_FAST : CO_PREC_FP32);
    if (M == 0) {
        st.setup_ms = ms_since(t_entry);
        g_last_setup_ms = st.setup_ms;
        g_last_loop_ms = 0.0;
        return CO_OK;
    }
    int rc = CO_OK;
    const Prep &pp = ctx->prep;
    const PackResult &pk = pp.pk;
    const Schedule &sc = pp.sc;
    const int64_t ldx = pp.ldx;
    const int S = pp.S;
    const int M_fit = (int)pp.M_fit;
    const int64_t total_c_fit = pp.total_c_fit;
    st.n_starts = S;
    cudaStream_t s = ctx->stream;
    const bool sharded = opt.sample_sharded != 0;
    if (sharded && !ctx->shard.comm) return CO_ERR_NULLARG;
    // which fits use the trust-region algorithm: tr_starts > 0 names the first starts,
    // otherwise `algorithm` applies to every start
    const int tr_fits = opt.tr_starts > 0 ? std::min(opt.tr_starts, S)
                                          : (opt.algorithm == CO_ALG_TRUST_REGION ? S : 0);
    const bool has_tr = tr_fits > 0, has_ref = tr_fits < S;
    // trust-region fits in double-double: per-sample values and Jacobians stay on the device
    const bool tr_dd = fp64 && has_tr && opt.tr_dd != 0;
    const int dd_kmax = std::max(h->K_max, 1);
    if (tr_dd) {
        const double jac_bytes = (double)M_fit * dd_kmax * h->N * sizeof(double);
        if (jac_bytes > DD_JAC_MAX_BYTES) return CO_ERR_BOUNDS;
        GROW(ctx->vals, (size_t)M_fit * h->N * sizeof(double));
        GROW(ctx->jac, (size_t)M_fit * dd_kmax * h->N * sizeof(double));
        GROW(ctx->dd_g, 2 * (size_t)sc.block_elems * sizeof(double));
        GROW(ctx->dd_blk, 2 * (size_t)sc.block_elems * sizeof(double));
    }
    const int wave1 = (S > 1 && opt.wave1 > 0 && opt.wave1 < S) ? opt.wave1 : 0;
    if (sharded && has_tr) return CO_ERR_NULLARG;   // sample-sharded fits: reference schedule
    CK(cudaEventRecord(ctx->ev_fit[0], s));
    {
        StartsParams<T> ip;
        ip.desc = P<TreeDesc>(ctx->desc);
        ip.tree_coff = P<int32_t>(ctx->tree_coff);
        ip.c_tree = P<float>(ctx->c_tree);
        ip.M_fit = M_fit;
        ip.S = S;
        ip.wave1 = wave1;
        ip.tr_starts = tr_fits;
        ip.damp_alternate = (S > 1 && opt.damping_floor > 0.0) ? 1 : 0;
        ip.tr_dd = tr_dd ? 1 : 0;
        ip.seed = opt.start_seed;
        ip.lam0 = (T)opt.lambda0;
        ip.c_start = P<float>(ctx->cinit_f);
        ip.c = P<T>(ctx->c);
        ip.ctry = P<T>(ctx->ctry);
        ip.lam = P<T>(ctx->lam);
        ip.status = P<int32_t>(ctx->status);
        ip.iters = P<int32_t>(ctx->iters);
        ip.pending = P<int32_t>(ctx->pending);
        ip.n_eval = P<int32_t>(ctx->n_eval);
        ip.outer = P<int32_t>(ctx->outer);
        ip.imode = P<uint8_t>(ctx->imode);
        ip.tr = P<double>(ctx->tr);
        ip.diag = P<double>(ctx->diag);
        init_starts_kernel<T><<<grid_for(ctx, M_fit), 256, 0, s>>>(ip);
        CK(cudaGetLastError());
        st.kernel_launches++;
    }
    if (wave1) {
        CK(cudaMemsetAsync(ctx->resolved.ptr, 0, (size_t)M, s));
        CK(cudaMemsetAsync(ctx->n_retired.ptr, 0, sizeof(int), s));
    }

    // ---- step-kernel launch geometry ----
    const size_t step_smem = (size_t)STEP_WARPS * STEP_WARP_D * sizeof(double);
    const size_t tr_smem = (size_t)(TR_THREADS / 32) * TR_WARP_D * sizeof(double);
    const size_t tr_smem_dd = (size_t)(TR_THREADS_DD / 32) * TR_WARP_D * sizeof(DD);
    if (!ctx->step_attr_set[fp64 ? 1 : 0]) {
        CK(cudaFuncSetAttribute(lm_step_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)step_smem));
        CK(cudaFuncSetAttribute(lm_tr_step_kernel_s<T, double>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tr_smem));
        if constexpr (sizeof(T) == 8)
            CK(cudaFuncSetAttribute(lm_tr_step_kernel_s<double, DD>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tr_smem_dd));
        ctx->step_attr_set[fp64 ? 1 : 0] = true;
    }
    int step_occ = 0, tr_occ = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&step_occ, lm_step_kernel<T>, STEP_THREADS,
                                                     step_smem));
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&tr_occ, lm_tr_step_kernel_s<T, double>,
                                                     TR_THREADS, tr_smem));
    const int step_grid = std::max(1, std::min((M_fit + STEP_WARPS - 1) / STEP_WARPS,
                                               std::max(1, step_occ) * ctx->sm_count));
    const int tr_grid = std::max(1, std::min((M_fit + TR_WARPS - 1) / TR_WARPS,
                                             std::max(1, tr_occ) * ctx->sm_count));
    int tr_occ_dd = 0;
    if constexpr (sizeof(T) == 8)
        CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&tr_occ_dd, lm_tr_step_kernel_s<double, DD>,
                                                         TR_THREADS_DD, tr_smem_dd));
    const int tr_grid_dd = std::max(1, std::min((M_fit + TR_THREADS_DD / 32 - 1) / (TR_THREADS_DD / 32),
                                                std::max(1, tr_occ_dd) * ctx->sm_count));
    const int ddg_grid = std::max(1, std::min(M_fit, 8 * ctx->sm_count));

    StepParams<T> sp;
    sp.desc = P<TreeDesc>(ctx->desc);
    sp.M = M_fit;
    sp.partials = P<T>(ctx->partials);
    sp.blk = P<T>(ctx->blk);
    sp.c = P<T>(ctx->c);
    sp.ctry = P<T>(ctx->ctry);
    sp.delta = P<T>(ctx->delta);
    sp.lam = P<T>(ctx->lam);
    sp.loss = P<T>(ctx->loss);
    sp.loss_init = P<T>(ctx->loss_init);
    sp.status = P<int32_t>(ctx->status);
    sp.iters = P<int32_t>(ctx->iters);
    sp.pending = P<int32_t>(ctx->pending);
    sp.n_eval = P<int32_t>(ctx->n_eval);
    sp.reduced = nullptr;
    sp.damping_floor = opt.damping_floor > 0.0 ? opt.damping_floor : 0.0;
    sp.damping_always = opt.damping_always ? 1 : 0;
    sp.imode = P<uint8_t>(ctx->imode);
    sp.max_iter = std::max(0, opt.max_iter);
    sp.fd_order = opt.fd_ordering ? 1 : 0;
    sp.xtol = (T)opt.xtol;

    TrParams<T> tp;
    tp.desc = sp.desc;
    tp.M = M_fit;
    tp.partials = sp.partials;
    tp.blk = sp.blk;
    tp.c = sp.c;
    tp.ctry = sp.ctry;
    tp.delta = sp.delta;
    tp.loss = sp.loss;
    tp.loss_init = sp.loss_init;
    tp.status = sp.status;
    tp.iters = sp.iters;
    tp.pending = sp.pending;
    tp.n_eval = sp.n_eval;
    tp.imode = sp.imode;
    tp.tr = P<double>(ctx->tr);
    tp.diag = P<double>(ctx->diag);
    tp.outer = P<int32_t>(ctx->outer);
    tp.max_nfev = std::max(1, opt.max_iter);
    tp.ftol = opt.ftol;
    tp.xtol = opt.xtol;
    tp.gtol = opt.gtol;
    tp.factor = 100.0;
    tp.ddg = tr_dd ? P<double>(ctx->dd_g) : nullptr;
    tp.blk_dd = tr_dd ? P<double>(ctx->dd_blk) : nullptr;
    // double-double fits: the pass also writes per-sample values and Jacobians, from which
    // dd_gram_kernel forms their normal equations
    T *dd_vals = tr_dd ? P<T>(ctx->vals) : nullptr;
    T *dd_jac = tr_dd ? P<T>(ctx->jac) : nullptr;
    auto dd_gram = [&]() -> int {
        if (!tr_dd) return CO_OK;
        dd_gram_kernel<<<ddg_grid, DDG_THREADS, 0, s>>>(
            P<TreeDesc>(ctx->desc), M_fit, P<uint8_t>(ctx->imode), P<int32_t>(ctx->status),
            P<int32_t>(ctx->pending), P<double>(ctx->vals), P<double>(ctx->jac), dd_kmax,
            P<float>(ctx->ym), h->N, P<double>(ctx->dd_g));
        CK(cudaGetLastError());
        st.kernel_launches++;
        return CO_OK;
    };

    // passes: one per LM iteration (reference) / per function evaluation after the first
    // (trust region); a second wave can start as late as the first wave's last pass
    const int max_iter = std::max(0, opt.max_iter);
    const int max_passes = wave1 ? 2 * max_iter + 2 : max_iter;
    size_t ev_i = 0;
    auto rec = [&](void) -> cudaEvent_t {
        cudaEvent_t e = event_at(ctx, ev_i++);
        if (e) cudaEventRecord(e, s);
        return e;
    };
    std::vector<std::pair<size_t, size_t>> eval_spans, step_spans, comm_spans;
    // the step kernels of one pass (and the wave update), counting running fits into n_running
    auto steps = [&](int *n_running) -> int {
        CK(cudaMemsetAsync(n_running, 0, sizeof(int), s));
        if (has_ref) {
            sp.n_running = n_running;
            lm_step_kernel<T><<<step_grid, STEP_THREADS, step_smem, s>>>(sp);
            CK(cudaGetLastError());
            st.kernel_launches++;
        }
        if (has_tr) {
            tp.n_running = n_running;
            lm_tr_step_kernel_s<T, double><<<tr_grid, TR_THREADS, tr_smem, s>>>(tp);
            CK(cudaGetLastError());
            st.kernel_launches++;
            if constexpr (sizeof(T) == 8) {
                if (tr_dd) {
                    lm_tr_step_kernel_s<double, DD><<<tr_grid_dd, TR_THREADS_DD, tr_smem_dd, s>>>(tp);
                    CK(cudaGetLastError());
                    st.kernel_launches++;
                }
            }
        }
        if (wave1) {
            waves_kernel<T><<<grid_for(ctx, M), 256, 0, s>>>(
                M, S, wave1, opt.agree_tol, P<T>(ctx->loss), P<int32_t>(ctx->status),
                P<int32_t>(ctx->pending), P<uint8_t>(ctx->resolved), n_running,
                P<int>(ctx->n_retired));
            CK(cudaGetLastError());
            st.kernel_launches++;
        }
        return CO_OK;
    };

    // with hundreds of chunks per tree (N of millions) the chunk partials are summed by a
    // block per tree before the step, instead of by the step kernel's one warp per tree
    const int64_t n_chunks = ((int64_t)h->N + sc.chunk - 1) / std::max(sc.chunk, 1);
    const bool presum = !sharded && n_chunks >= PRESUM_CHUNKS;

    // ---- initial pass at the start points + solve of iteration 0 ----
    size_t e0 = ev_i; rec();
    rc = launch_pass<T>(ctx, sc, pk, P<T>(ctx->c), P<T>(ctx->partials), *h, ldx, true, dd_vals,
                        dd_jac, tr_dd ? dd_kmax : 0, P<uint8_t>(ctx->imode));
    if (rc) return rc;
    rc = dd_gram();
    if (rc) return rc;
    size_t e1 = ev_i; rec();
    eval_spans.push_back({e0, e1});
    if (sharded) {
        rc = shard_reduce_blocks<T>(ctx, M_fit, sc.block_elems);
        if (rc) return rc;
        sp.reduced = P<T>(ctx->red);
        size_t ec = ev_i; rec();
        comm_spans.push_back({e1, ec});
        e1 = ec;
    } else if (presum) {
        rc = chunk_sums<T>(ctx, M_fit, sc.block_elems, s);
        if (rc) return rc;
        sp.reduced = P<T>(ctx->red);
    }
    rc = steps(P<int>(ctx->n_run));
    if (rc) return rc;
    size_t e2 = ev_i; rec();
    step_spans.push_back({e1, e2});
    rc = sync_stream(ctx, sharded);
    if (rc) return rc;
    st.setup_ms = ms_since(t_entry);
    auto t_loop = std::chrono::steady_clock::now();

    // ---- LM iterations ----
    // At most two iterations are in flight: before launching iteration `it` the host waits
    // for the running-fit count of step it-2 and stops once no fit is running.
    int iters_run = 0;
    for (int it = 0; it < max_passes; ++it) {
        const int slot = it & 1;
        if (opt.early_exit && it >= 2) {
            if (sharded) {
                rc = shard_wait_event(ctx->shard, ctx->ev_nrun[slot]);
                if (rc) return rc;
            } else {
                CK(cudaEventSynchronize(ctx->ev_nrun[slot]));
            }
            if (ctx->h_nrun[slot] == 0) break;
        }
        iters_run++;
        size_t a = ev_i; rec();
        rc = launch_pass<T>(ctx, sc, pk, P<T>(ctx->ctry), P<T>(ctx->partials), *h, ldx, true,
                            dd_vals, dd_jac, tr_dd ? dd_kmax : 0, P<uint8_t>(ctx->imode));
        if (rc) return rc;
        rc = dd_gram();
        if (rc) return rc;
        size_t b = ev_i; rec();
        eval_spans.push_back({a, b});
        if (sharded) {
            rc = shard_reduce_blocks<T>(ctx, M_fit, sc.block_elems);
            if (rc) return rc;
            size_t bc = ev_i; rec();
            comm_spans.push_back({b, bc});
            b = bc;
        } else if (presum) {
            rc = chunk_sums<T>(ctx, M_fit, sc.block_elems, s);
            if (rc) return rc;
        }
        rc = steps(P<int>(ctx->n_run) + slot);
        if (rc) return rc;
        size_t c = ev_i; rec();
        step_spans.push_back({b, c});
        if (opt.early_exit) {
            CK(cudaMemcpyAsync(ctx->h_nrun + slot, P<int>(ctx->n_run) + slot, sizeof(int),
                               cudaMemcpyDeviceToHost, s));
            CK(cudaEventRecord(ctx->ev_nrun[slot], s));
        }
    }
    rc = sync_stream(ctx, sharded);
    if (rc) return rc;
    st.loop_ms = ms_since(t_loop);
    st.iters_run = iters_run;
    auto t_fin = std::chrono::steady_clock::now();

    // ---- fp64 audit of fp32 fits (lm_core.cuh:299-351; fp64 fits accept in fp64 already) ----
    const bool audit = !fp64 && opt.fp64_audit != 0 && total_c > 0;
    if (audit) {
        GROW(ctx->c64, total_c_fit * sizeof(double));
        GROW(ctx->l64, 2 * (size_t)M_fit * sizeof(double));
        GROW(ctx->n_rev, sizeof(int));
        // per-item partials are not needed any more: reuse the buffer for fp64 sums
        GROW(ctx->partials, (size_t)sc.partial_elems * sizeof(double));
        double *c64 = P<double>(ctx->c64), *l64 = P<double>(ctx->l64);
        const int g1 = grid_for(ctx, std::max<int64_t>(total_c_fit, M_fit));
        const float *srcs[2] = {reinterpret_cast<const float *>(ctx->c.ptr), P<float>(ctx->cinit_f)};
        for (int pass = 0; pass < 2; ++pass) {
            audit_prepare_kernel<<<g1, 256, 0, s>>>(P<TreeDesc>(ctx->desc), M_fit, srcs[pass],
                                                    total_c_fit, c64, P<int32_t>(ctx->pending),
                                                    P<int32_t>(ctx->n_eval));
            CK(cudaGetLastError());
            rc = launch_pass<double>(ctx, sc, pk, c64, P<double>(ctx->partials), *h, ldx, false);
            if (rc) return rc;
            audit_loss_kernel<<<g1, 256, 0, s>>>(P<TreeDesc>(ctx->desc), M_fit,
                                                  P<double>(ctx->partials), l64 + (size_t)pass * M_fit);
            CK(cudaGetLastError());
            st.kernel_launches += 2;
        }
        if (sharded) {   // the fp64 losses over all samples: sum the ranks' halves
            rc = shard_allreduce(ctx->shard, l64, 2 * (size_t)M_fit, true, s);
            if (rc) return rc;
        }
        CK(cudaMemsetAsync(ctx->n_rev.ptr, 0, sizeof(int), s));
        audit_apply_kernel<T><<<g1, 256, 0, s>>>(P<TreeDesc>(ctx->desc), M_fit, l64,
                                                 l64 + M_fit, P<float>(ctx->cinit_f),
                                                 P<T>(ctx->c), P<T>(ctx->loss),
                                                 P<int32_t>(ctx->status),
                                                 P<int32_t>(ctx->n_eval), P<int>(ctx->n_rev));
        CK(cudaGetLastError());
        st.kernel_launches++;
    }
    // ---- per tree, the start with the lowest final loss (the identity for one start) ----
    select_best_kernel<T><<<grid_for(ctx, M), 256, 0, s>>>(
        P<TreeDesc>(ctx->desc), P<int32_t>(ctx->tree_coff), M, S, P<T>(ctx->loss),
        P<T>(ctx->loss_init), audit ? P<double>(ctx->l64) : nullptr, P<int32_t>(ctx->status),
        P<int32_t>(ctx->iters), P<int32_t>(ctx->n_eval), P<T>(ctx->c), P<T>(ctx->out_c),
        P<int32_t>(ctx->out_status), P<T>(ctx->out_li), P<T>(ctx->out_lf),
        P<int32_t>(ctx->out_iters), P<int32_t>(ctx->out_start));
    CK(cudaGetLastError());
    st.kernel_launches++;

    // ---- D2H ----
    std::vector<T> hc((size_t)total_c), hli((size_t)M), hlf((size_t)M);
    std::vector<int32_t> hst((size_t)M), hit((size_t)M), hne((size_t)M_fit);
    if (total_c > 0)
        CK(cudaMemcpyAsync(hc.data(), ctx->out_c.ptr, total_c * sizeof(T), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(hli.data(), ctx->out_li.ptr, (size_t)M * sizeof(T), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(hlf.data(), ctx->out_lf.ptr, (size_t)M * sizeof(T), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(hst.data(), ctx->out_status.ptr, (size_t)M * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(hit.data(), ctx->out_iters.ptr, (size_t)M * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(hne.data(), ctx->n_eval.ptr, (size_t)M_fit * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    ctx->h_start.assign((size_t)M, 0);
    if (S > 1)
        CK(cudaMemcpyAsync(ctx->h_start.data(), ctx->out_start.ptr, (size_t)M * sizeof(int32_t),
                           cudaMemcpyDeviceToHost, s));
    int n_rev = 0, n_ret = 0;
    if (audit)
        CK(cudaMemcpyAsync(&n_rev, ctx->n_rev.ptr, sizeof(int), cudaMemcpyDeviceToHost, s));
    if (wave1)
        CK(cudaMemcpyAsync(&n_ret, ctx->n_retired.ptr, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(ctx->ev_fit[1], s));
    rc = sync_stream(ctx, sharded);
    if (rc) return rc;
    {
        float dms = 0.f;
        if (cudaEventElapsedTime(&dms, ctx->ev_fit[0], ctx->ev_fit[1]) == cudaSuccess)
            st.device_ms = dms;
    }
    st.n_reverted = n_rev;
    st.trees_retired = n_ret;

    for (int64_t i = 0; i < total_c; ++i) {
        if (out.c_f) out.c_f[i] = (float)hc[(size_t)i];
        if (out.c_d) out.c_d[i] = (double)hc[(size_t)i];
    }
    for (int m = 0; m < M; ++m) {
        out.status[m] = hst[(size_t)m];
        if (out.li_f) out.li_f[m] = (float)hli[(size_t)m];
        if (out.lf_f) out.lf_f[m] = (float)hlf[(size_t)m];
        if (out.li_d) out.li_d[m] = (double)hli[(size_t)m];
        if (out.lf_d) out.lf_d[m] = (double)hlf[(size_t)m];
        if (out.iters) out.iters[m] = hit[(size_t)m];
    }
    // evaluation counts: initial pass + every evaluated trial, per fit
    int64_t node_evals = 0, sample_evals = 0, fits_run = 0;
    double flops = 0.0;
    for (int64_t i = 0; i < M_fit; ++i) {
        const int64_t evals = hne[(size_t)i];
        const int m = (int)(i / S);
        const int K = (int)pk.trees[(size_t)m].K;
        fits_run += evals > 0 ? 1 : 0;
        node_evals += evals * ctx->n_nodes[(size_t)m] * (int64_t)N;
        sample_evals += evals * (int64_t)N;
        // value + adjoint per operator node, plus the normal-equation update
        flops += (double)evals * N * (2.0 * ctx->n_ops[(size_t)m] + 2.0 * nblock_size(K));
    }
    st.flops = flops;
    st.node_evals = node_evals;
    st.sample_evals = sample_evals;
    st.fits_run = fits_run;

    // device-time split from the recorded events
    auto span_ms = [&](const std::vector<std::pair<size_t, size_t>> &spans) {
        double t = 0.0;
        for (auto &sp_ : spans) {
            float x = 0.f;
            if (cudaEventElapsedTime(&x, ctx->events[sp_.first], ctx->events[sp_.second]) ==
                cudaSuccess)
                t += x;
        }
        return t;
    };
    st.eval_ms = span_ms(eval_spans);
    st.step_ms = span_ms(step_spans);
    st.comm_ms = span_ms(comm_spans);
    st.finish_ms = ms_since(t_fin);
    g_last_setup_ms = st.setup_ms;
    g_last_loop_ms = st.loop_ms;
    return CO_OK;
}

template <typename T>
int run_fit(Ctx *ctx, const Problem &pr, const CoOptions &opt, const Outputs &out) {
    auto t_entry = std::chrono::steady_clock::now();
    int rc = load<T>(ctx, pr, opt.y_shared != 0, opt.n_starts);
    if (rc != CO_OK) return rc;
    return fit_loaded<T>(ctx, opt, out, t_entry);
}

// Evaluate every tree at given constants: values, Jacobian, normal-equation blocks.
template <typename T>
int run_eval(Ctx *ctx, const Problem &pr, bool y_shared, const double *c, double *vals_out,
             double *jac_out, double *blocks_out) {
    const PopHeader *h = pr.h;
    const int M = h->M_prob, N = h->N;
    const int64_t total_c = h->total_c;
    ctx->stats = CoStats{};
    ctx->stats.precision = sizeof(T) == 8 ? CO_PREC_FP64 : CO_PREC_FP32;
    Prep pp;
    ctx->loaded = false;   // the evaluation reuses the resident buffers
    int rc = prepare<T>(ctx, pr, y_shared, pp);
    if (rc != CO_OK) return rc;
    if (M == 0) return CO_OK;
    if (jac_out && pp.pk.max_K > h->K_max) return CO_ERR_NULLARG;
    cudaStream_t s = ctx->stream;
    GROW(ctx->c64, total_c * sizeof(double));
    if (total_c > 0)
        CK(cudaMemcpyAsync(ctx->c64.ptr, c, total_c * sizeof(double), cudaMemcpyHostToDevice, s));
    load_point_kernel<T><<<grid_for(ctx, std::max<int64_t>(total_c, M)), 256, 0, s>>>(
        P<double>(ctx->c64), total_c, P<T>(ctx->ctry), M, P<int32_t>(ctx->pending));
    CK(cudaGetLastError());
    T *dv = nullptr, *dj = nullptr;
    const int kmax = std::max(h->K_max, 1);
    if (vals_out) {
        GROW(ctx->vals, (size_t)M * N * sizeof(T));
        dv = P<T>(ctx->vals);
    }
    if (jac_out) {
        GROW(ctx->jac, (size_t)M * kmax * N * sizeof(T));
        dj = P<T>(ctx->jac);
        CK(cudaMemsetAsync(dj, 0, (size_t)M * kmax * N * sizeof(T), s));
    }
    rc = launch_pass<T>(ctx, pp.sc, pp.pk, P<T>(ctx->ctry), P<T>(ctx->partials), *pr.h, pp.ldx,
                        true, dv, dj, kmax);
    if (rc) return rc;
    sum_blocks_kernel<T><<<grid_for(ctx, M), 256, 0, s>>>(P<TreeDesc>(ctx->desc), M,
                                                           P<T>(ctx->partials), P<T>(ctx->blk));
    CK(cudaGetLastError());
    std::vector<T> hv, hj, hb;
    if (vals_out) {
        hv.resize((size_t)M * N);
        CK(cudaMemcpyAsync(hv.data(), dv, hv.size() * sizeof(T), cudaMemcpyDeviceToHost, s));
    }
    if (jac_out) {
        hj.resize((size_t)M * kmax * N);
        CK(cudaMemcpyAsync(hj.data(), dj, hj.size() * sizeof(T), cudaMemcpyDeviceToHost, s));
    }
    if (blocks_out) {
        hb.resize((size_t)pp.sc.block_elems);
        CK(cudaMemcpyAsync(hb.data(), ctx->blk.ptr, hb.size() * sizeof(T), cudaMemcpyDeviceToHost, s));
    }
    CK(cudaStreamSynchronize(s));
    for (size_t i = 0; i < hv.size(); ++i) vals_out[i] = (double)hv[i];
    if (jac_out) {
        // reference d_J layout [M][K_max][N] (cusr/kernel/ad_interp.cuh:240-244)
        for (size_t i = 0; i < hj.size(); ++i) jac_out[i] = (double)hj[i];
    }
    for (size_t i = 0; i < hb.size(); ++i) blocks_out[i] = (double)hb[i];
    return CO_OK;
}

// Finite-difference Jacobian of every tree at constants c: one value pass at c and one per
// constant column with that column stepped (fd_perturb_kernel), J in the reference d_J
// layout [M][K_max][N]. An independent on-device check of the reverse-mode Jacobian.
template <typename T>
int run_jac_fd(Ctx *ctx, const Problem &pr, bool y_shared, const double *c, double eps,
               double *jac_out) {
    const PopHeader *h = pr.h;
    const int M = h->M_prob, N = h->N;
    const int64_t total_c = h->total_c;
    ctx->stats = CoStats{};
    ctx->stats.precision = sizeof(T) == 8 ? CO_PREC_FP64 : CO_PREC_FP32;
    Prep pp;
    ctx->loaded = false;
    int rc = prepare<T>(ctx, pr, y_shared, pp);
    if (rc != CO_OK) return rc;
    if (M == 0) return CO_OK;
    if (pp.pk.max_K > h->K_max) return CO_ERR_NULLARG;
    cudaStream_t s = ctx->stream;
    const int kmax = std::max(h->K_max, 1);
    GROW(ctx->c64, total_c * sizeof(double));
    GROW(ctx->vals, 2 * (size_t)M * N * sizeof(T));
    GROW(ctx->jac, (size_t)M * kmax * N * sizeof(T));
    if (total_c > 0)
        CK(cudaMemcpyAsync(ctx->c64.ptr, c, total_c * sizeof(double), cudaMemcpyHostToDevice, s));
    load_point_kernel<T><<<grid_for(ctx, std::max<int64_t>(total_c, M)), 256, 0, s>>>(
        P<double>(ctx->c64), total_c, P<T>(ctx->ctry), M, P<int32_t>(ctx->pending));
    CK(cudaGetLastError());
    T *v0 = P<T>(ctx->vals), *vk = v0 + (size_t)M * N, *dj = P<T>(ctx->jac);
    CK(cudaMemsetAsync(dj, 0, (size_t)M * kmax * N * sizeof(T), s));
    rc = launch_pass<T>(ctx, pp.sc, pp.pk, P<T>(ctx->ctry), P<T>(ctx->partials), *pr.h, pp.ldx,
                        false, v0);
    if (rc) return rc;
    const int g = grid_for(ctx, (int64_t)M * N);
    for (int k = 0; k < pp.pk.max_K; ++k) {
        fd_perturb_kernel<T><<<grid_for(ctx, M), 256, 0, s>>>(
            P<TreeDesc>(ctx->desc), M, P<T>(ctx->ctry), k, (T)eps, P<T>(ctx->c), P<T>(ctx->lam),
            P<int32_t>(ctx->pending));
        CK(cudaGetLastError());
        rc = launch_pass<T>(ctx, pp.sc, pp.pk, P<T>(ctx->c), P<T>(ctx->partials), *pr.h, pp.ldx,
                            false, vk);
        if (rc) return rc;
        fd_column_kernel<T><<<g, 256, 0, s>>>(P<TreeDesc>(ctx->desc), M, N, k, kmax, vk, v0,
                                               P<T>(ctx->lam), dj);
        CK(cudaGetLastError());
    }
    std::vector<T> hj((size_t)M * kmax * N);
    CK(cudaMemcpyAsync(hj.data(), dj, hj.size() * sizeof(T), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    for (size_t i = 0; i < hj.size(); ++i) jac_out[i] = (double)hj[i];
    return CO_OK;
}

}  // namespace
}  // namespace cusr

using namespace cusr;

extern "C" {

void co_default_options(CoOptions *opt) {
    if (!opt) return;
    std::memset(opt, 0, sizeof(*opt));
    opt->struct_size = (int32_t)sizeof(CoOptions);
    opt->precision = CO_PREC_FP32;
    opt->max_iter = 50;
    opt->y_shared = 0;
    opt->lambda0 = 1e-3;
    opt->xtol = 1e-6;
    opt->fp64_audit = -1;
    opt->early_exit = 1;
    opt->algorithm = CO_ALG_REFERENCE;
    opt->n_starts = 1;
    opt->tr_starts = 0;
    opt->wave1 = 0;
    opt->ftol = 1e-10;
    opt->gtol = 1e-8;
    opt->agree_tol = 1e-7;
    opt->start_seed = 0;
}

// Options that every fit entry checks.
static bool valid_fit_options(const CoOptions &o) {
    if (o.n_devices < 0 || o.n_devices > CO_MAX_DEVICES) return false;
    for (int i = 0; i < (o.n_devices > 1 ? o.n_devices : 0); ++i)
        if (o.device_ids[i] < 0) return false;
    return o.lambda0 > 0.0 && o.xtol >= 0.0 && o.ftol >= 0.0 && o.gtol >= 0.0 &&
           o.agree_tol >= 0.0 && o.n_starts >= 0 && o.n_starts <= CO_MAX_STARTS &&
           o.tr_starts >= 0 && o.wave1 >= 0 &&
           (o.tr_dd == 0 || (o.tr_dd == 1 && o.precision == CO_PREC_FP64)) &&
           (o.algorithm == CO_ALG_REFERENCE || o.algorithm == CO_ALG_TRUST_REGION);
}

// Caller options over the defaults: the first struct_size bytes of the caller's struct are
// taken (at least the fields up to early_exit, the original layout), later fields keep their
// defaults, so callers built against an older, shorter CoOptions keep working.
static bool read_options(const CoOptions *in, CoOptions *out) {
    co_default_options(out);
    if (!in) return true;
    const int32_t min_size = (int32_t)offsetof(CoOptions, sample_sharded);
    if (in->struct_size < min_size) return false;
    const size_t n = std::min<size_t>((size_t)in->struct_size, sizeof(CoOptions));
    std::memcpy(out, in, n);
    out->struct_size = (int32_t)sizeof(CoOptions);
    return true;
}

static bool has_inputs(const float *xs, const float *ym, const CoOptions *opt_in) {
    return (xs && ym) || (opt_in && opt_in->struct_size >= (int32_t)offsetof(CoOptions, reserved) &&
                          opt_in->keep_inputs);
}

int co_init(int device_id, void **handle_out) {
    if (!handle_out) return CO_ERR_NULLARG;
    *handle_out = nullptr;
    cudaError_t e = cudaSetDevice(device_id);
    if (e != cudaSuccess) {
        fprintf(stderr, "[cusr_b200] cudaSetDevice(%d): %s\n", device_id, cudaGetErrorString(e));
        return CO_ERR_CUDA;
    }
    e = cudaFree(0);
    if (e != cudaSuccess) {
        fprintf(stderr, "[cusr_b200] context init: %s\n", cudaGetErrorString(e));
        return CO_ERR_CUDA;
    }
    Ctx *ctx = new (std::nothrow) Ctx();
    if (!ctx) return CO_ERR_OOM;
    ctx->device = device_id;
    struct Step { const char *what; cudaError_t e; };
    int optin = 0;
    Step steps[] = {
        {"sm count", cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device_id)},
        {"smem opt-in", cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device_id)},
        {"stream", cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking)},
        {"pinned counter", cudaMallocHost(&ctx->h_nrun, 2 * sizeof(int))},
        {"event 0", cudaEventCreateWithFlags(&ctx->ev_nrun[0], cudaEventDisableTiming)},
        {"event 1", cudaEventCreateWithFlags(&ctx->ev_nrun[1], cudaEventDisableTiming)},
        {"fork event", cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming)},
        {"sync event", cudaEventCreateWithFlags(&ctx->ev_sync, cudaEventDisableTiming)},
        {"fit event 0", cudaEventCreate(&ctx->ev_fit[0])},
        {"fit event 1", cudaEventCreate(&ctx->ev_fit[1])},
        {"fp32 kernels", eval_prepare_f32()},
        {"fp32 fast-math kernels", eval_prepare_f32_fast()},
        {"fp64 kernels", eval_prepare_f64()},
    };
    for (int i = 0; i < Ctx::kBinStreams; ++i) {
        cudaError_t e = cudaStreamCreateWithFlags(&ctx->bin_streams[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_join[i], cudaEventDisableTiming);
        if (e != cudaSuccess) {
            fprintf(stderr, "[cusr_b200] device %d setup (bin stream %d): %s\n", device_id, i,
                    cudaGetErrorString(e));
            cudaGetLastError();
            co_teardown(ctx);
            return CO_ERR_CUDA;
        }
    }
    for (const Step &st : steps) {
        if (st.e != cudaSuccess) {
            fprintf(stderr, "[cusr_b200] device %d setup (%s): %s\n", device_id, st.what,
                    cudaGetErrorString(st.e));
            cudaGetLastError();
            co_teardown(ctx);
            return CO_ERR_CUDA;
        }
    }
    // CUSR_EVAL_WIDE=0 / 1 pins the evaluation block width (measurements); unset: per bin
    if (const char *e = std::getenv("CUSR_EVAL_WIDE")) ctx->wide_mode = std::atoi(e) ? 1 : 0;
    // CUSR_BIN_STREAMS=1..8: streams the bins of a pass run on (measurements)
    if (const char *e = std::getenv("CUSR_BIN_STREAMS"))
        ctx->n_bin_streams = std::min((int)Ctx::kBinStreams, std::max(1, std::atoi(e)));
    // CUSR_EVAL_FWD=k (0..2): trees with K <= k use forward-mode tangents (measurements)
    if (const char *e = std::getenv("CUSR_EVAL_FWD"))
        ctx->fwd_default = ctx->fwd_max = std::min(2, std::max(0, std::atoi(e)));
    ctx->smem_optin = optin;
    *handle_out = ctx;
    return CO_OK;
}

// Jacobian mode of the next schedule built on this context (CoOptions.ad_mode).
static void set_ad_mode(Ctx *ctx, int ad_mode) {
    ctx->fwd_max = ad_mode == CO_AD_FORWARD ? 2 : (ad_mode == CO_AD_REVERSE ? 0 : ctx->fwd_default);
}

static bool valid_prec(int p) {
    return p == CO_PREC_FP32 || p == CO_PREC_FP64 || p == CO_PREC_FP32_FAST;
}

static int optimize_common(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                           const int32_t *ci, const TreeMeta *metas, const float *c_init,
                           const float *xs, const float *ym, const CoOptions &opt,
                           const Outputs &out) {
    Ctx *ctx = (Ctx *)handle;
    Problem pr{h, nt, nv, ci, metas, c_init, xs, ym};
    pr.keep_inputs = opt.keep_inputs != 0;
    int rc = check_args(pr);
    if (rc != CO_OK) return rc;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    ctx->fast = opt.precision == CO_PREC_FP32_FAST;
    set_ad_mode(ctx, opt.ad_mode);
    if (opt.precision == CO_PREC_FP64) return run_fit<double>(ctx, pr, opt, out);
    return run_fit<float>(ctx, pr, opt, out);
}

// One fit spread over several devices (CoOptions.n_devices): the trees are split into
// cost-balanced shards (longest processing time first on nodes x (1 + K); the samples are
// common to all trees), each shard is fitted by the context of its device on a host thread of
// its own (the handle's context for its own device, a child context per other slot, created
// on first use and kept), and the outputs are written back in the caller's tree order. A
// target matrix whose rows are all equal is passed to the shards as one shared row.
static int optimize_multi(Ctx *ctx, const PopHeader *h, const int32_t *nt, const float *nv,
                          const int32_t *ci, const TreeMeta *metas, const float *c_init,
                          const float *xs, const float *ym, const CoOptions &opt,
                          const Outputs &out) {
    const int nd = opt.n_devices, M = h->M_prob, N = h->N;
    if (opt.keep_inputs || opt.sample_sharded) return CO_ERR_NULLARG;
    Problem pr{h, nt, nv, ci, metas, c_init, xs, ym};
    int rc = check_args(pr);
    if (rc != CO_OK) return rc;
    // contexts per shard slot
    std::vector<Ctx *> cx((size_t)nd, nullptr);
    bool own_used = false;
    for (int i = 0; i < nd; ++i) {
        const int dev = opt.device_ids[i];
        if (dev == ctx->device && !own_used) {
            cx[(size_t)i] = ctx;
            own_used = true;
            continue;
        }
        if (ctx->peers[i] && ctx->peers[i]->device != dev) {
            co_teardown(ctx->peers[i]);
            ctx->peers[i] = nullptr;
        }
        if (!ctx->peers[i]) {
            void *hnd = nullptr;
            rc = co_init(dev, &hnd);
            if (rc != CO_OK) return rc;
            ctx->peers[i] = (Ctx *)hnd;
        }
        cx[(size_t)i] = ctx->peers[i];
    }
    // LPT shards
    std::vector<int> order((size_t)M), owner((size_t)M);
    for (int m = 0; m < M; ++m) order[(size_t)m] = m;
    auto cost = [&](int m) { return (double)metas[m].n_nodes * (1.0 + metas[m].K); };
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost(a) > cost(b); });
    std::vector<double> load((size_t)nd, 0.0);
    for (int m : order) {
        const int sl = (int)(std::min_element(load.begin(), load.end()) - load.begin());
        owner[(size_t)m] = sl;
        load[(size_t)sl] += cost(m);
    }
    // one shared target row when every row is equal
    bool shared = opt.y_shared != 0;
    if (!shared && M > 0 && N > 0) {
        shared = true;
        for (int m = 1; m < M && shared; ++m)
            if (std::memcmp(ym, ym + (size_t)m * N, (size_t)N * sizeof(float)) != 0) shared = false;
    }
    struct Shard {
        std::vector<int32_t> trees, nt, ci, status, iters;
        std::vector<float> nv, c0, ym;
        std::vector<TreeMeta> metas;
        std::vector<double> c, li, lf;
        PopHeader h{};
        int rc = CO_OK;
    };
    std::vector<Shard> sh((size_t)nd);
    for (int m = 0; m < M; ++m) sh[(size_t)owner[(size_t)m]].trees.push_back(m);
    for (Shard &d : sh) {
        int32_t node = 0, coff = 0;
        for (int m : d.trees) {
            const TreeMeta &tm = metas[m];
            d.metas.push_back(TreeMeta{node, tm.n_nodes, coff, tm.K});
            d.nt.insert(d.nt.end(), nt + tm.node_offset, nt + tm.node_offset + tm.n_nodes);
            d.nv.insert(d.nv.end(), nv + tm.node_offset, nv + tm.node_offset + tm.n_nodes);
            d.ci.insert(d.ci.end(), ci + tm.node_offset, ci + tm.node_offset + tm.n_nodes);
            d.c0.insert(d.c0.end(), c_init + tm.c_offset, c_init + tm.c_offset + tm.K);
            if (!shared) d.ym.insert(d.ym.end(), ym + (size_t)m * N, ym + (size_t)(m + 1) * N);
            node += tm.n_nodes;
            coff += tm.K;
        }
        d.h = *h;
        d.h.M_prob = (int32_t)d.trees.size();
        d.h.total_nodes = node;
        d.h.total_c = coff;
        d.c.resize((size_t)coff);
        d.li.resize(d.trees.size());
        d.lf.resize(d.trees.size());
        d.status.resize(d.trees.size());
        d.iters.resize(d.trees.size());
    }
    CoOptions o = opt;
    o.n_devices = 0;
    o.y_shared = shared ? 1 : 0;
    std::vector<std::thread> th;
    for (int i = 0; i < nd; ++i) {
        th.emplace_back([&, i]() {
            Shard &d = sh[(size_t)i];
            Outputs so;
            so.c_d = d.c.data();
            so.status = d.status.data();
            so.li_d = d.li.data();
            so.lf_d = d.lf.data();
            so.iters = d.iters.data();
            d.rc = optimize_common(cx[(size_t)i], &d.h, d.nt.data(), d.nv.data(), d.ci.data(),
                                   d.metas.data(), d.c0.data(), xs, shared ? ym : d.ym.data(),
                                   o, so);
        });
    }
    for (std::thread &t : th) t.join();
    for (const Shard &d : sh)
        if (d.rc != CO_OK) return d.rc;
    // outputs in the caller's order; statistics: device time of the slowest shard, work summed
    CoStats agg{};
    ctx->h_start.assign((size_t)M, 0);
    for (int i = 0; i < nd; ++i) {
        const Shard &d = sh[(size_t)i];
        const Ctx *c = cx[(size_t)i];
        for (size_t j = 0; j < d.trees.size(); ++j) {
            const int m = d.trees[j];
            const TreeMeta &tm = metas[m];
            const TreeMeta &sm = d.metas[j];
            for (int k = 0; k < tm.K; ++k) {
                const double v = d.c[(size_t)sm.c_offset + k];
                if (out.c_d) out.c_d[tm.c_offset + k] = v;
                if (out.c_f) out.c_f[tm.c_offset + k] = (float)v;
            }
            out.status[m] = d.status[j];
            if (out.li_d) out.li_d[m] = d.li[j];
            if (out.lf_d) out.lf_d[m] = d.lf[j];
            if (out.li_f) out.li_f[m] = (float)d.li[j];
            if (out.lf_f) out.lf_f[m] = (float)d.lf[j];
            if (out.iters) out.iters[m] = d.iters[j];
            if (j < c->h_start.size()) ctx->h_start[(size_t)m] = c->h_start[j];
        }
        const CoStats &s_ = c->stats;
        agg.setup_ms = std::max(agg.setup_ms, s_.setup_ms);
        agg.loop_ms = std::max(agg.loop_ms, s_.loop_ms);
        agg.finish_ms = std::max(agg.finish_ms, s_.finish_ms);
        agg.eval_ms = std::max(agg.eval_ms, s_.eval_ms);
        agg.step_ms = std::max(agg.step_ms, s_.step_ms);
        agg.comm_ms = std::max(agg.comm_ms, s_.comm_ms);
        agg.device_ms = std::max(agg.device_ms, s_.device_ms);
        agg.flops += s_.flops;
        agg.node_evals += s_.node_evals;
        agg.sample_evals += s_.sample_evals;
        agg.eval_launches += s_.eval_launches;
        agg.kernel_launches += s_.kernel_launches;
        agg.iters_run = std::max(agg.iters_run, s_.iters_run);
        agg.n_bins += s_.n_bins;
        agg.n_reverted += s_.n_reverted;
        agg.fits_run += s_.fits_run;
        agg.trees_retired += s_.trees_retired;
        agg.n_starts = s_.n_starts;
        agg.precision = s_.precision;
        agg.y_shared = s_.y_shared;
    }
    ctx->stats = agg;
    return CO_OK;
}

int co_optimize(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                const int32_t *ci, const TreeMeta *metas, const float *c_init, const float *xs,
                const float *ym, int max_iter, float *c_final_out, int32_t *status_out,
                float *loss_init_out, float *loss_final_out) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c_init || !xs || !ym || !c_final_out ||
        !status_out)
        return CO_ERR_NULLARG;
    CoOptions opt;
    co_default_options(&opt);
    opt.max_iter = max_iter;
    Outputs out;
    out.c_f = c_final_out;
    out.status = status_out;
    out.li_f = loss_init_out;
    out.lf_f = loss_final_out;
    return optimize_common(handle, h, nt, nv, ci, metas, c_init, xs, ym, opt, out);
}

int co_optimize_ex(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                   const int32_t *ci, const TreeMeta *metas, const float *c_init, const float *xs,
                   const float *ym, const CoOptions *opt_in, double *c_final_out,
                   int32_t *status_out, double *loss_init_out, double *loss_final_out,
                   int32_t *iters_out) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c_init ||
        !has_inputs(xs, ym, opt_in) || !c_final_out || !status_out)
        return CO_ERR_NULLARG;
    CoOptions opt;
    if (!read_options(opt_in, &opt)) return CO_ERR_NULLARG;
    if (!valid_prec(opt.precision)) return CO_ERR_NULLARG;
    if (!valid_fit_options(opt)) return CO_ERR_NULLARG;
    opt.sample_sharded = 0;
    Outputs out;
    out.c_d = c_final_out;
    out.status = status_out;
    out.li_d = loss_init_out;
    out.lf_d = loss_final_out;
    out.iters = iters_out;
    if (opt.n_devices > 1)
        return optimize_multi((Ctx *)handle, h, nt, nv, ci, metas, c_init, xs, ym, opt, out);
    return optimize_common(handle, h, nt, nv, ci, metas, c_init, xs, ym, opt, out);
}

int co_evaluate(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                const int32_t *ci, const TreeMeta *metas, const double *c, const float *xs,
                const float *ym, int precision, int y_shared, double *vals_out,
                double *jac_out, double *blocks_out) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c || !xs || !ym) return CO_ERR_NULLARG;
    if (!valid_prec(precision)) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    Problem pr{h, nt, nv, ci, metas, nullptr, xs, ym};
    int rc = check_args(pr);
    if (rc != CO_OK) return rc;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    std::vector<float> c_f((size_t)std::max(h->total_c, 0));
    for (size_t i = 0; i < c_f.size(); ++i) c_f[i] = (float)c[i];
    pr.c_init = c_f.data();
    ctx->fast = precision == CO_PREC_FP32_FAST;
    set_ad_mode(ctx, CO_AD_AUTO);
    if (precision == CO_PREC_FP64)
        return run_eval<double>(ctx, pr, y_shared != 0, c, vals_out, jac_out, blocks_out);
    return run_eval<float>(ctx, pr, y_shared != 0, c, vals_out, jac_out, blocks_out);
}

int co_jacobian_fd(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                   const int32_t *ci, const TreeMeta *metas, const double *c, const float *xs,
                   const float *ym, int precision, int y_shared, double eps, double *jac_out) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c || !xs || !ym || !jac_out)
        return CO_ERR_NULLARG;
    if (!valid_prec(precision)) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    Problem pr{h, nt, nv, ci, metas, nullptr, xs, ym};
    int rc = check_args(pr);
    if (rc != CO_OK) return rc;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    std::vector<float> c_f((size_t)std::max(h->total_c, 0));
    for (size_t i = 0; i < c_f.size(); ++i) c_f[i] = (float)c[i];
    pr.c_init = c_f.data();
    ctx->fast = precision == CO_PREC_FP32_FAST;
    if (precision == CO_PREC_FP64)
        return run_jac_fd<double>(ctx, pr, y_shared != 0, c, eps > 0 ? eps : 1e-7, jac_out);
    return run_jac_fd<float>(ctx, pr, y_shared != 0, c, eps > 0 ? eps : 1e-3, jac_out);
}

int co_load(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
            const int32_t *ci, const TreeMeta *metas, const float *c_init, const float *xs,
            const float *ym, const CoOptions *opt_in) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c_init || !has_inputs(xs, ym, opt_in))
        return CO_ERR_NULLARG;
    CoOptions opt;
    if (!read_options(opt_in, &opt)) return CO_ERR_NULLARG;
    if (!valid_prec(opt.precision)) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    Problem pr{h, nt, nv, ci, metas, c_init, xs, ym};
    pr.keep_inputs = opt.keep_inputs != 0;
    int rc = check_args(pr);
    if (rc != CO_OK) return rc;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    if (!valid_fit_options(opt)) return CO_ERR_NULLARG;
    set_ad_mode(ctx, opt.ad_mode);
    rc = opt.precision == CO_PREC_FP64 ? load<double>(ctx, pr, opt.y_shared != 0, opt.n_starts)
                                       : load<float>(ctx, pr, opt.y_shared != 0, opt.n_starts);
    if (rc == CO_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess) return CO_ERR_CUDA;
    return rc;
}

int co_fit_loaded(void *handle, const CoOptions *opt_in, double *c_final_out,
                  int32_t *status_out, double *loss_init_out, double *loss_final_out,
                  int32_t *iters_out) {
    if (!handle || !c_final_out || !status_out) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    CoOptions opt;
    if (!read_options(opt_in, &opt)) return CO_ERR_NULLARG;
    if (!ctx->loaded || !valid_prec(opt.precision) ||
        (opt.precision == CO_PREC_FP64) != (ctx->prep_prec == CO_PREC_FP64))
        return CO_ERR_NULLARG;
    ctx->fast = opt.precision == CO_PREC_FP32_FAST;
    if (opt.sample_sharded && !ctx->shard.comm) return CO_ERR_NULLARG;
    if (!valid_fit_options(opt)) return CO_ERR_NULLARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    Outputs out;
    out.c_d = c_final_out;
    out.status = status_out;
    out.li_d = loss_init_out;
    out.lf_d = loss_final_out;
    out.iters = iters_out;
    auto t0 = std::chrono::steady_clock::now();
    return opt.precision == CO_PREC_FP64 ? fit_loaded<double>(ctx, opt, out, t0)
                                         : fit_loaded<float>(ctx, opt, out, t0);
}

int co_probe_peak(void *handle, double *fp32_tflops, double *fp64_tflops) {
    if (!handle) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    GROW(ctx->c64, 64);
    cudaStream_t s = ctx->stream;
    const int blocks = ctx->sm_count * 8, threads = 256, iters = 8192;
    const double fmas = (double)blocks * threads * iters * 16;
    cudaEvent_t e0 = event_at(ctx, 0), e1 = event_at(ctx, 1);
    for (int prec = 0; prec < 2; ++prec) {
        double best = 0.0;
        for (int rep = 0; rep < 3; ++rep) {
            CK(cudaEventRecord(e0, s));
            if (prec == 0)
                fma_probe_kernel<float><<<blocks, threads, 0, s>>>(P<float>(ctx->c64), iters,
                                                                  0.999f, 0.001f);
            else
                fma_probe_kernel<double><<<blocks, threads, 0, s>>>(P<double>(ctx->c64), iters / 4,
                                                                   0.999, 0.001);
            CK(cudaGetLastError());
            CK(cudaEventRecord(e1, s));
            CK(cudaEventSynchronize(e1));
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, e0, e1));
            const double tf = 2.0 * fmas / (prec == 0 ? 1.0 : 4.0) / (ms * 1e-3) / 1e12;
            best = std::max(best, tf);
        }
        if (prec == 0 && fp32_tflops) *fp32_tflops = best;
        if (prec == 1 && fp64_tflops) *fp64_tflops = best;
    }
    return CO_OK;
}

int co_shard_unique_id(unsigned char id_out[128]) {
    if (!id_out) return CO_ERR_NULLARG;
    return shard_unique_id(id_out);
}

int co_shard_init(void *handle, const unsigned char id[128], int nranks, int rank,
                  double timeout_s) {
    if (!handle || !id) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return CO_ERR_CUDA;
    return shard_init(ctx->shard, id, nranks, rank, timeout_s);
}

int co_optimize_sharded(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                        const int32_t *ci, const TreeMeta *metas, const float *c_init,
                        const float *xs, const float *ym, const CoOptions *opt_in,
                        double *c_final_out, int32_t *status_out, double *loss_init_out,
                        double *loss_final_out, int32_t *iters_out) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c_init ||
        !has_inputs(xs, ym, opt_in) || !c_final_out || !status_out)
        return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    if (!ctx->shard.comm) return CO_ERR_NULLARG;   // co_shard_init first
    CoOptions opt;
    if (!read_options(opt_in, &opt)) return CO_ERR_NULLARG;
    opt.sample_sharded = 1;
    if (!valid_prec(opt.precision)) return CO_ERR_NULLARG;
    if (!valid_fit_options(opt)) return CO_ERR_NULLARG;
    // one fit per tree from c_init with the reference schedule: the per-iteration all-reduce
    // carries the trees' normal equations
    if (opt.n_starts > 1 || opt.algorithm != CO_ALG_REFERENCE || opt.tr_starts > 0)
        return CO_ERR_NULLARG;
    Outputs out;
    out.c_d = c_final_out;
    out.status = status_out;
    out.li_d = loss_init_out;
    out.lf_d = loss_final_out;
    out.iters = iters_out;
    return optimize_common(handle, h, nt, nv, ci, metas, c_init, xs, ym, opt, out);
}

int co_last_split(double *setup_ms_out, double *loop_ms_out) {
    if (setup_ms_out) *setup_ms_out = g_last_setup_ms;
    if (loop_ms_out) *loop_ms_out = g_last_loop_ms;
    return 0;
}

int co_last_starts(void *handle, int32_t *start_out) {
    if (!handle || !start_out) return CO_ERR_NULLARG;
    Ctx *ctx = (Ctx *)handle;
    for (size_t m = 0; m < ctx->h_start.size(); ++m) start_out[m] = ctx->h_start[m];
    return CO_OK;
}

int co_get_stats(void *handle, CoStats *out) {
    if (!handle || !out) return CO_ERR_NULLARG;
    *out = ((Ctx *)handle)->stats;
    return CO_OK;
}

void co_teardown(void *handle) {
    if (!handle) return;
    Ctx *ctx = (Ctx *)handle;
    for (Ctx *&peer : ctx->peers) {
        if (peer) co_teardown(peer);
        peer = nullptr;
    }
    cudaSetDevice(ctx->device);
    DBuf *bufs[] = {&ctx->code, &ctx->desc, &ctx->bin_trees, &ctx->bin_tree_off,
                    &ctx->bin_item_off, &ctx->items, &ctx->n_items, &ctx->counter,
                    &ctx->xs_raw, &ctx->xs, &ctx->ym, &ctx->c, &ctx->ctry, &ctx->delta,
                    &ctx->cinit_f, &ctx->lam, &ctx->loss, &ctx->loss_init, &ctx->status,
                    &ctx->iters, &ctx->pending, &ctx->n_run, &ctx->n_eval, &ctx->partials, &ctx->blk,
                    &ctx->c64, &ctx->l64, &ctx->n_rev, &ctx->vals, &ctx->jac, &ctx->red,
                    &ctx->dd_g, &ctx->dd_blk,
                    &ctx->c_tree, &ctx->tree_coff, &ctx->imode, &ctx->tr, &ctx->diag,
                    &ctx->outer, &ctx->resolved, &ctx->n_retired, &ctx->out_c,
                    &ctx->out_status, &ctx->out_li, &ctx->out_lf, &ctx->out_iters,
                    &ctx->out_start,
                    &ctx->tape_gs[0], &ctx->tape_gs[1], &ctx->tape_gs[2], &ctx->tape_gs[3],
                    &ctx->tape_gs[4], &ctx->tape_gs[5], &ctx->tape_gs[6], &ctx->tape_gs[7]};
    for (DBuf *b : bufs) release(*b);
    for (cudaEvent_t e : ctx->events) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->ev_nrun)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->ev_fit)
        if (e) cudaEventDestroy(e);
    if (ctx->h_nrun) cudaFreeHost(ctx->h_nrun);
    shard_destroy(ctx->shard);
    if (ctx->ev_sync) cudaEventDestroy(ctx->ev_sync);
    for (cudaStream_t bs : ctx->bin_streams)
        if (bs) cudaStreamDestroy(bs);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    for (cudaEvent_t e : ctx->ev_join)
        if (e) cudaEventDestroy(e);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

const char *co_strerror(int code) {
    switch (code) {
        case CO_OK: return "ok";
        case CO_ERR_BOUNDS: return "K_max > 32 or max_stack > 64, or a tree beyond an engine limit";
        case CO_ERR_CUDA: return "CUDA error";
        case CO_ERR_SUM_C: return "sum(metas.K) != header.total_c";
        case CO_ERR_SUM_NODES: return "sum(metas.n_nodes) != header.total_nodes";
        case CO_ERR_NULLARG: return "null pointer / bad argument";
        case CO_ERR_OOM: return "out of memory";
        case CO_ERR_BADTREE: return "malformed tree bytecode";
        default: return "unknown code";
    }
}

}  // extern "C"
