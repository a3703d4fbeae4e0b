// debug_api.cpp — host-only exports for testing the compiler on machines without a GPU.
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
