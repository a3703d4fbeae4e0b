// batch_lm_cli.cpp — command-line front end with the reference binary's interface
// (cusr/kernel/batch_lm_ad.cu:196-251, 526-551), so subprocess callers (the benchmark runner's
// CudaKernelPop, kernel_bridge._run_kernel) run unchanged against this engine:
//
//   batch_lm_b200 <pop.bin> [out_dir] [--max-iter N] [--quiet]
//                 [--precision fp32|fp64|fp32_fast] [--device D]
//
// Writes into out_dir (default: the directory of pop.bin)
//   status.bin      int32[M]      STATUS_* per tree
//   c_final.bin     float32[total_c]
//   loss_final.bin  float32[M]    0.5 * sum r^2 at c_final
//   loss_init.bin   float32[M]    0.5 * sum r^2 at c_init
// and, unless --quiet, a summary whose last line carries the wall time of the whole run in
// the reference's wording ("总耗时 X 秒"), which CudaKernelPop parses.
// Exit codes: 0 ok, 1 usage / I/O / engine error, 2 beyond the engine's limits (K_max > 32,
// max_stack > 64), as the reference.
#include <errno.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <string>
#include <vector>

#include "../../include/cusr_co.h"

namespace {

double now_s() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + (double)t.tv_nsec * 1e-9;
}

struct Pop {
    PopHeader h;
    std::vector<int32_t> nt, ci;
    std::vector<float> nv, c_init, xs, ym;
    std::vector<TreeMeta> metas;
};

template <typename V>
bool read_array(FILE *f, V &v, size_t count) {
    v.resize(count);
    return count == 0 || fread(v.data(), sizeof(v[0]), count, f) == count;
}

// pop.bin reader (layout of cusr/kernel/pop_format.h:1-51, loader.c:17-69): 64-byte header,
// then nt, nv, ci, metas, c_init, xs, ym, all little-endian 4-byte elements.
bool load_pop(const char *path, Pop &p) {
    FILE *f = fopen(path, "rb");
    if (!f) {
        fprintf(stderr, "[batch-lm] cannot open %s: %s\n", path, strerror(errno));
        return false;
    }
    bool ok = fread(&p.h, sizeof(PopHeader), 1, f) == 1;
    if (ok && (p.h.magic != POP_MAGIC || p.h.version != POP_VERSION)) {
        fprintf(stderr, "[batch-lm] %s: bad magic/version (0x%08x, %d)\n", path,
                (unsigned)p.h.magic, p.h.version);
        ok = false;
    }
    if (ok && (p.h.M_prob < 0 || p.h.total_nodes < 0 || p.h.total_c < 0 || p.h.N < 0 ||
               p.h.n_vars < 0)) {
        fprintf(stderr, "[batch-lm] %s: negative size in header\n", path);
        ok = false;
    }
    if (ok) {
        const size_t M = (size_t)p.h.M_prob, T = (size_t)p.h.total_nodes;
        const size_t N = (size_t)p.h.N;
        ok = read_array(f, p.nt, T) && read_array(f, p.nv, T) && read_array(f, p.ci, T) &&
             read_array(f, p.metas, M) && read_array(f, p.c_init, (size_t)p.h.total_c) &&
             read_array(f, p.xs, N * (size_t)p.h.n_vars) && read_array(f, p.ym, M * N);
        if (!ok) fprintf(stderr, "[batch-lm] %s: short read\n", path);
    }
    fclose(f);
    return ok;
}

bool write_blob(const std::string &path, const void *buf, size_t bytes) {
    FILE *f = fopen(path.c_str(), "wb");
    if (!f) {
        fprintf(stderr, "[batch-lm] fopen %s failed: %s\n", path.c_str(), strerror(errno));
        return false;
    }
    const bool ok = bytes == 0 || fwrite(buf, 1, bytes, f) == bytes;
    fclose(f);
    if (!ok) fprintf(stderr, "[batch-lm] short write %s\n", path.c_str());
    return ok;
}

}  // namespace

int main(int argc, char **argv) {
    const double t_start = now_s();
    if (argc < 2) {
        fprintf(stderr,
                "usage: %s <pop.bin> [out_dir] [--max-iter N] [--quiet] "
                "[--precision fp32|fp64|fp32_fast] [--device D]\n",
                argv[0]);
        return 1;
    }
    const char *pop_path = argv[1];
    std::string out_dir;
    int max_iter = 50, quiet = 0, device = 0, precision = CO_PREC_FP32;
    for (int i = 2; i < argc; ++i) {
        if (!strcmp(argv[i], "--max-iter") && i + 1 < argc) {
            max_iter = atoi(argv[++i]);
        } else if (!strcmp(argv[i], "--quiet")) {
            quiet = 1;
        } else if (!strcmp(argv[i], "--device") && i + 1 < argc) {
            device = atoi(argv[++i]);
        } else if (!strcmp(argv[i], "--precision") && i + 1 < argc) {
            const char *p = argv[++i];
            if (!strcmp(p, "fp32")) precision = CO_PREC_FP32;
            else if (!strcmp(p, "fp64")) precision = CO_PREC_FP64;
            else if (!strcmp(p, "fp32_fast")) precision = CO_PREC_FP32_FAST;
            else {
                fprintf(stderr, "[batch-lm] unknown precision %s\n", p);
                return 1;
            }
        } else if (argv[i][0] != '-') {
            out_dir = argv[i];
        }
    }
    if (out_dir.empty()) {
        const char *slash = strrchr(pop_path, '/');
        out_dir = slash ? std::string(pop_path, (size_t)(slash - pop_path)) : std::string(".");
        if (out_dir.empty()) out_dir = "/";
    }

    Pop pop;
    if (!load_pop(pop_path, pop)) {
        fprintf(stderr, "load failed.\n");
        return 1;
    }
    const PopHeader &h = pop.h;
    if (!quiet)
        printf("[batch-lm] loaded %s: M_prob=%d total_nodes=%d total_c=%d N=%d n_vars=%d "
               "K_max=%d max_stack=%d\n",
               pop_path, h.M_prob, h.total_nodes, h.total_c, h.N, h.n_vars, h.K_max,
               h.max_stack);
    if (h.K_max > CO_MAX_K || h.max_stack > CO_MAX_STACK) {
        fprintf(stderr, "[batch-lm] K_max=%d / max_stack=%d beyond the engine limits (%d / %d)\n",
                h.K_max, h.max_stack, CO_MAX_K, CO_MAX_STACK);
        return 2;
    }

    const size_t M = (size_t)h.M_prob, C = (size_t)h.total_c;
    std::vector<int32_t> status(M, 0);
    std::vector<float> c_final(C), loss_init(M), loss_final(M);
    void *co = nullptr;
    int rc = co_init(device, &co);
    if (rc != CO_OK) {
        fprintf(stderr, "[batch-lm] co_init: %s\n", co_strerror(rc));
        return 1;
    }
    if (precision == CO_PREC_FP32) {
        // the reference entry point (fp32 outputs)
        rc = co_optimize(co, &h, pop.nt.data(), pop.nv.data(), pop.ci.data(), pop.metas.data(),
                         pop.c_init.data(), pop.xs.data(), pop.ym.data(), max_iter,
                         c_final.data(), status.data(), loss_init.data(), loss_final.data());
    } else {
        CoOptions opt;
        co_default_options(&opt);
        opt.precision = precision;
        opt.max_iter = max_iter;
        std::vector<double> c64(C), li(M), lf(M);
        rc = co_optimize_ex(co, &h, pop.nt.data(), pop.nv.data(), pop.ci.data(),
                            pop.metas.data(), pop.c_init.data(), pop.xs.data(), pop.ym.data(),
                            &opt, c64.data(), status.data(), li.data(), lf.data(), nullptr);
        for (size_t i = 0; i < C; ++i) c_final[i] = (float)c64[i];
        for (size_t m = 0; m < M; ++m) {
            loss_init[m] = (float)li[m];
            loss_final[m] = (float)lf[m];
        }
    }
    co_teardown(co);
    if (rc != CO_OK) {
        fprintf(stderr, "[batch-lm] fit failed: %s (code %d)\n", co_strerror(rc), rc);
        return rc == CO_ERR_BOUNDS ? 2 : 1;
    }

    bool ok = write_blob(out_dir + "/status.bin", status.data(), M * sizeof(int32_t)) &&
              write_blob(out_dir + "/c_final.bin", c_final.data(), C * sizeof(float)) &&
              write_blob(out_dir + "/loss_final.bin", loss_final.data(), M * sizeof(float)) &&
              write_blob(out_dir + "/loss_init.bin", loss_init.data(), M * sizeof(float));
    if (!ok) return 1;

    const double elapsed = now_s() - t_start;
    if (!quiet) {
        int n[5] = {0, 0, 0, 0, 0};
        for (int32_t s : status)
            if (s >= 0 && s < 5) n[s]++;
        const double pct = M ? 100.0 * n[STATUS_CONVERGED] / (double)M : 0.0;
        printf("[batch-lm] done: converged=%d (%.1f%%)  maxiter=%d  fail_nan=%d  "
               "fail_cholesky=%d  k0_skip=%d  (M_prob=%d)\n",
               n[STATUS_CONVERGED], pct, n[STATUS_MAXITER], n[STATUS_FAIL_NAN],
               n[STATUS_FAIL_CHOLESKY], n[STATUS_K0_SKIP], h.M_prob);
        printf("[batch-lm] wrote %s/status.bin (%zu B) + %s/c_final.bin (%zu B)\n",
               out_dir.c_str(), M * sizeof(int32_t), out_dir.c_str(), C * sizeof(float));
        // the reference's wording of the timing line ("total time X s"), parsed by callers
        printf("[batch-lm] 总耗时 %.3f 秒 (%.0f trees/s, M_prob=%d)\n", elapsed,
               elapsed > 0 ? (double)M / elapsed : 0.0, h.M_prob);
    }
    return 0;
}
