// noalloc.cu — co_evaluate_noalloc: the fused evaluation pass with every scratch buffer in a
// fixed, file-scope device array, for callers that cannot allocate device memory.
//
// Who needs it: a caller whose device memory is owned by its own pool allocator (a framework
// that reserved the GPU up front), or one that must not take the device-wide synchronisation a
// cudaMalloc / cudaFree implies in the middle of its pipeline. It passes its own device
// buffers for the constants, inputs, targets and output; everything else the pass needs —
// compiled programs, tree descriptors, work lists and counters, the transposed inputs, the
// padded target row and the per-chunk partial sums — lives in g_noalloc_scratch below, so
// the call allocates no device memory at all (host-side compilation uses ordinary host memory).
//
// Limits: kNoAllocScratchBytes (32 MiB) in total, fp32 arithmetic, one target row shared by
// every tree, and trees whose reverse tape fits in shared memory (no global-tape bins);
// anything beyond returns CO_ERR_BOUNDS without launching work.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/cusr_co.h"
#include "launch.h"
#include "pack.h"

namespace cusr {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

// Every GPU that loads this library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct DeviceSetup {
    unsigned char *scratch = nullptr;   // device address of g_noalloc_scratch on this device
    int sm_count = 0;
    int smem_optin = 0;
    bool ready = false;
};

std::mutex g_mu;                        // calls share the array: one at a time per process
DeviceSetup g_dev[kMaxDevices];

// Once per device, with that device current: resolve the array's device address (the
// host-side symbol is only a stand-in, never a device pointer) and raise the kernels' dynamic
// shared-memory limit.
int device_setup(int dev, DeviceSetup **out) {
    if (dev < 0 || dev >= kMaxDevices) return CO_ERR_NULLARG;
    DeviceSetup &s = g_dev[dev];
    if (!s.ready) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            fprintf(stderr, "[cusr_b200] cudaGetSymbolAddress(scratch) on device %d: %s\n", dev,
                    cudaGetErrorString(e));
            return CO_ERR_CUDA;
        }
        if (cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&s.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
                cudaSuccess ||
            eval_prepare_f32() != cudaSuccess)
            return CO_ERR_CUDA;
        s.scratch = static_cast<unsigned char *>(p);
        s.ready = true;
    }
    *out = &s;
    return CO_OK;
}

size_t up256(size_t b) { return (b + 255) & ~size_t(255); }

// inputs [N][n_vars] (pop.bin) -> [n_vars][ldx], zero padded
__global__ void na_transpose_x(const float *__restrict__ xs, int64_t N, int n_vars, int64_t ldx,
                               float *__restrict__ out) {
    const int64_t total = (int64_t)n_vars * ldx;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t v = e / ldx, i = e - v * ldx;
        out[e] = (i < N) ? xs[i * n_vars + v] : 0.0f;
    }
}

// per-tree block = sum of its chunk partials in chunk order; the loss entry is halved
__global__ void na_sum_blocks(const TreeDesc *desc, int M, const float *partials, float *blk) {
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const TreeDesc d = desc[m];
        const int P = nblock_size(d.K);
        for (int e = 0; e < P; ++e) {
            float s = 0.0f;
            for (int ch = 0; ch < d.n_chunks; ++ch) s += partials[d.p_off + (int64_t)ch * P + e];
            blk[d.q_off + e] = (e == P - 1) ? 0.5f * s : s;
        }
    }
}

int evaluate_noalloc(int dev, const PopHeader *h, const int32_t *nt, const float *nv,
                     const int32_t *ci, const TreeMeta *metas, const float *c_dev,
                     const float *xs_dev, const float *y_dev, float *blocks_dev,
                     cudaStream_t stream) {
    DeviceSetup *ds = nullptr;
    int rc = device_setup(dev, &ds);
    if (rc != CO_OK) return rc;
    const int M = h->M_prob, N = h->N, n_vars = h->n_vars;
    if (M == 0) return CO_OK;

    PackResult pk;
    rc = compile_population(h, nt, nv, ci, metas, &pk);
    if (rc != CO_OK) return rc;
    const int round = EVAL_ROUND;
    Schedule sc;
    build_schedule(pk, metas, M, N, /*y_shared=*/true, /*fp64=*/false, round, ds->sm_count * 3,
                   &sc);
    const int64_t ldx = ((int64_t)N + round - 1) / round * round;
    const int n_bins = (int)sc.bins.size();

    // work lists on the host: every chunk of every tree, bin order
    std::vector<int2> items((size_t)sc.total_items);
    for (const Bin &b : sc.bins) {
        int64_t o = b.item_off;
        for (int32_t t : b.trees)
            for (int c = 0; c < sc.desc[(size_t)t].n_chunks; ++c) items[(size_t)o++] = make_int2(t, c);
    }
    std::vector<int> counts(2 * (size_t)n_bins, 0);   // n_items, then counters (start at 0)
    for (int b = 0; b < n_bins; ++b) counts[(size_t)b] = (int)sc.bins[(size_t)b].max_items;

    // carve the scratch array
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off += up256(std::max<size_t>(bytes, 1)); return o; };
    const size_t o_code = take(pk.code.size() * sizeof(uint32_t));
    const size_t o_desc = take((size_t)M * sizeof(TreeDesc));
    const size_t o_items = take(items.size() * sizeof(int2));
    const size_t o_counts = take(counts.size() * sizeof(int));
    const size_t o_x = take((size_t)n_vars * ldx * sizeof(float));
    const size_t o_y = take((size_t)ldx * sizeof(float));
    const size_t o_part = take((size_t)sc.partial_elems * sizeof(float));
    if (off > kNoAllocScratchBytes) {
        fprintf(stderr, "[cusr_b200] co_evaluate_noalloc: needs %zu bytes of scratch, the fixed "
                        "array holds %zu\n", off, kNoAllocScratchBytes);
        return CO_ERR_BOUNDS;
    }
    // launch geometry per bin; bins that need the global tape are beyond this entry
    std::vector<size_t> smem((size_t)n_bins);
    std::vector<int> grid((size_t)n_bins);
    for (int b = 0; b < n_bins; ++b) {
        const Bin &bin = sc.bins[(size_t)b];
        smem[(size_t)b] = eval_smem_f32(bin.kc, bin.max_instr, n_vars, std::max(bin.max_spill, 1),
                                       std::max(bin.max_tape, 1), true, false);
        if (2 * (smem[(size_t)b] + 1024) > (size_t)ds->smem_optin) return CO_ERR_BOUNDS;
        int occ = std::max(1, eval_blocks_per_sm_f32(bin.kc, true, false, false, smem[(size_t)b]));
        grid[(size_t)b] = (int)std::min<int64_t>((int64_t)occ * ds->sm_count,
                                                 std::max<int64_t>(1, bin.max_items));
    }

    unsigned char *S = ds->scratch;
    // From here on work is queued on `stream` and reads or writes the shared array: an error
    // path first waits for whatever was queued (its own result ignored), so no copy or kernel
    // of this call still uses the array when the next call takes the lock.
#define NA_CK(x)                                                                             \
    do {                                                                                     \
        cudaError_t _e = (x);                                                                \
        if (_e != cudaSuccess) {                                                             \
            fprintf(stderr, "[cusr_b200] co_evaluate_noalloc: %s\n", cudaGetErrorString(_e)); \
            cudaStreamSynchronize(stream);                                                   \
            cudaGetLastError();                                                              \
            return CO_ERR_CUDA;                                                              \
        }                                                                                    \
    } while (0)
    NA_CK(cudaMemcpyAsync(S + o_code, pk.code.data(), pk.code.size() * sizeof(uint32_t),
                          cudaMemcpyHostToDevice, stream));
    NA_CK(cudaMemcpyAsync(S + o_desc, sc.desc.data(), (size_t)M * sizeof(TreeDesc),
                          cudaMemcpyHostToDevice, stream));
    NA_CK(cudaMemcpyAsync(S + o_items, items.data(), items.size() * sizeof(int2),
                          cudaMemcpyHostToDevice, stream));
    // item counts and zeroed work counters: the array keeps the previous call's contents
    NA_CK(cudaMemcpyAsync(S + o_counts, counts.data(), counts.size() * sizeof(int),
                          cudaMemcpyHostToDevice, stream));
    float *xS = reinterpret_cast<float *>(S + o_x);
    float *yS = reinterpret_cast<float *>(S + o_y);
    if (n_vars > 0 && N > 0) {
        na_transpose_x<<<std::max(1, std::min(4 * ds->sm_count, (int)((n_vars * ldx + 255) / 256))),
                             256, 0, stream>>>(xs_dev, N, n_vars, ldx, xS);
        NA_CK(cudaGetLastError());
    }
    NA_CK(cudaMemsetAsync(yS, 0, (size_t)ldx * sizeof(float), stream));
    if (N > 0)
        NA_CK(cudaMemcpyAsync(yS, y_dev, (size_t)N * sizeof(float), cudaMemcpyDeviceToDevice, stream));

    const TreeDesc *dDesc = reinterpret_cast<const TreeDesc *>(S + o_desc);
    int *dCounts = reinterpret_cast<int *>(S + o_counts);
    float *dPart = reinterpret_cast<float *>(S + o_part);
    for (int b = 0; b < n_bins; ++b) {
        const Bin &bin = sc.bins[(size_t)b];
        EvalParams<float> p;
        p.code = reinterpret_cast<const uint32_t *>(S + o_code);
        p.desc = dDesc;
        p.items = reinterpret_cast<const int2 *>(S + o_items) + bin.item_off;
        p.n_items = dCounts + b;
        p.counter = dCounts + n_bins + b;
        p.c = c_dev;
        p.xs = xS;
        p.ym = yS;
        p.partials = dPart;
        p.ldx = ldx;
        p.N = N;
        p.chunk = sc.chunk;
        p.n_vars = n_vars;
        p.code_cap = bin.max_instr;
        p.spill_cap = std::max(bin.max_spill, 1);
        p.tape_cap = std::max(bin.max_tape, 1);
        p.tape_g = nullptr;
        p.vals = nullptr;
        p.jac = nullptr;
        p.jac_kmax = 0;
        NA_CK(eval_launch_f32(bin.kc, true, false, false, p, grid[(size_t)b], smem[(size_t)b], stream));
    }
    na_sum_blocks<<<std::max(1, std::min(4 * ds->sm_count, (M + 255) / 256)), 256, 0, stream>>>(
        dDesc, M, dPart, blocks_dev);
    NA_CK(cudaGetLastError());
    // host-side staging is released on return, and the next call reuses the array
    NA_CK(cudaStreamSynchronize(stream));
#undef NA_CK
    return CO_OK;
}

}  // namespace
}  // namespace cusr

extern "C" int co_evaluate_noalloc(int device_id, const PopHeader *h, const int32_t *nt,
                                   const float *nv, const int32_t *ci, const TreeMeta *metas,
                                   const float *c_dev, const float *xs_dev, const float *y_dev,
                                   float *blocks_dev, void *stream) {
    if (!h || !nt || !nv || !ci || !metas || !c_dev || !xs_dev || !y_dev || !blocks_dev)
        return CO_ERR_NULLARG;
    if (h->M_prob < 0 || h->N < 0 || h->n_vars < 0 || h->total_c < 0 || h->total_nodes < 0)
        return CO_ERR_NULLARG;
    if (h->K_max > CO_MAX_K || h->max_stack > CO_MAX_STACK || h->n_vars > CO_MAX_VARS)
        return CO_ERR_BOUNDS;
    int64_t ks = 0, ns = 0;
    for (int m = 0; m < h->M_prob; ++m) {
        ks += metas[m].K;
        ns += metas[m].n_nodes;
    }
    if (ks != (int64_t)h->total_c) return CO_ERR_SUM_C;
    if (ns != (int64_t)h->total_nodes) return CO_ERR_SUM_NODES;

    std::lock_guard<std::mutex> lock(cusr::g_mu);
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return CO_ERR_CUDA;
    if (cudaSetDevice(device_id) != cudaSuccess) return CO_ERR_CUDA;
    int rc = cusr::evaluate_noalloc(device_id, h, nt, nv, ci, metas, c_dev, xs_dev, y_dev,
                                    blocks_dev, static_cast<cudaStream_t>(stream));
    cudaSetDevice(prev);
    return rc;
}
