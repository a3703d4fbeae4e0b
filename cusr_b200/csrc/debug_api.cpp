// debug_api.cpp — host-only exports for testing the compiler on machines without a GPU.
#include <cmath>
#include <vector>

#include "../../include/cusr_co.h"
#include "../../include/cusr_debug.h"
#include "pack.h"

extern "C" int cusr_compile_tree(const int32_t *nt, const float *nv, const int32_t *ci,
                                 int n_nodes, int K, int n_vars, uint32_t *code_out, int cap,
                                 int32_t *info_out) {
    if (!nt || !nv || !ci || !code_out || !info_out) return CO_ERR_NULLARG;
    std::vector<uint32_t> code;
    cusr::CompiledTree ct;
    int rc = cusr::compile_tree(nt, nv, ci, n_nodes, K, n_vars, code, ct);
    if (rc != CO_OK) return rc;
    if ((int)code.size() > cap) return CO_ERR_NULLARG;
    for (size_t i = 0; i < code.size(); ++i) code_out[i] = code[i];
    info_out[0] = ct.n_instr;
    info_out[1] = ct.n_spill;
    info_out[2] = ct.n_tape;
    info_out[3] = ct.unique_const ? 1 : 0;
    info_out[4] = ct.n_bwd;
    return CO_OK;
}

extern "C" double cusr_eval_program(const uint32_t *fwd, int n_fwd, const uint32_t *bwd,
                                    int n_bwd, const double *x, const double *c, int K,
                                    double *grad) {
    return cusr::host_eval_program(fwd, n_fwd, bwd, n_bwd, x, c, K, grad);
}

// The device start generator (starts.cuh: mix64, start_normal, the four start kinds) compiled
// for the host: the start points of tree m (constants c0[0..K)) for starts 0..S-1, written to
// out[s * K + k].
namespace {
uint64_t host_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
double host_start_normal(uint64_t seed, int64_t m, int s, int k, int j) {
    uint64_t h = host_mix64(seed ^ host_mix64((uint64_t)m));
    h = host_mix64(h ^ (((uint64_t)(uint32_t)s << 32) | (uint64_t)(uint32_t)(2 * k + j)));
    const uint64_t h2 = host_mix64(h);
    const double u1 = ((double)(h >> 11) + 0.5) * 0x1.0p-53;
    const double u2 = (double)(h2 >> 11) * 0x1.0p-53;
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}
}  // namespace

extern "C" void cusr_start_points(uint64_t seed, int64_t m, int S, int K, const float *c0,
                                  float *out) {
    for (int s = 0; s < S; ++s)
        for (int k = 0; k < K; ++k) {
            double v = c0[k];
            if (s > 0) {
                const double z1 = host_start_normal(seed, m, s, k, 0);
                switch ((s - 1) % 4) {
                    case 0: v = v * std::exp(0.5 * z1) + 0.05 * host_start_normal(seed, m, s, k, 1); break;
                    case 1: v = v + 0.5 * (std::fabs(v) + 1.0) * z1; break;
                    case 2: v = z1; break;
                    default: v = 3.0 * z1; break;
                }
            }
            out[s * K + k] = (float)v;
        }
}
