// fd_variant.cpp — libcusr_co_fd.so: the reference FD variant's library name and co_optimize
// semantics (cusr/kernel/co_lib.h:56-63 built without USE_AD, co_lib.cu:456-471) over the
// engine in libcusr_b200.so. The reference loader picks the variant from the library name
// (co_inproc.py:257-259, get_inproc_co's default is "fd"); this library defines only
// co_optimize — with CoOptions.fd_ordering set: a step below xtol is CONVERGED and kept before
// the improvement test, an improvement must be strict — and takes co_init, co_last_split,
// co_teardown and every extended symbol from libcusr_b200.so, which it links against.
// The Jacobian is the engine's exact one, not the FD variant's forward differences.
#include <vector>

#include "../../include/cusr_co.h"

extern "C" int co_optimize(void *handle, const PopHeader *h, const int32_t *nt, const float *nv,
                           const int32_t *ci, const TreeMeta *metas, const float *c_init,
                           const float *xs, const float *ym, int max_iter, float *c_final_out,
                           int32_t *status_out, float *loss_init_out, float *loss_final_out) {
    if (!handle || !h || !nt || !nv || !ci || !metas || !c_init || !xs || !ym || !c_final_out ||
        !status_out)
        return CO_ERR_NULLARG;
    if (h->M_prob < 0 || h->total_c < 0) return CO_ERR_NULLARG;
    CoOptions opt;
    co_default_options(&opt);
    opt.max_iter = max_iter;
    opt.fd_ordering = 1;
    std::vector<double> c((size_t)h->total_c), li((size_t)h->M_prob), lf((size_t)h->M_prob);
    const int rc = co_optimize_ex(handle, h, nt, nv, ci, metas, c_init, xs, ym, &opt, c.data(),
                                  status_out, li.data(), lf.data(), nullptr);
    if (rc != CO_OK) return rc;
    for (size_t i = 0; i < c.size(); ++i) c_final_out[i] = (float)c[i];
    for (size_t m = 0; m < li.size(); ++m) {
        if (loss_init_out) loss_init_out[m] = (float)li[m];
        if (loss_final_out) loss_final_out[m] = (float)lf[m];
    }
    return CO_OK;
}
