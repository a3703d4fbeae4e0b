"""oracle — TEST INFRASTRUCTURE ONLY.

CPU restatement of the reference (TensorConv/CuSR) batched-LM constant-fitting path, used as
the checker for the CUDA engine in `cusr_b200`:

  interp.py     numpy fp64 tree interpreter (cusr/benchmark/interp.py) and the reverse-mode
                Jacobian rules of cusr/kernel/revad_interp.cuh, vectorised over samples
  lm.py         the reference LM iteration (cusr/kernel/co_lib.cu:284-518, AD ordering)
                in numpy, fp32 or fp64, with the fp64 audit (cusr/kernel/lm_core.cuh:299-351)
  scipy_lm.py   the reference CPU backend ScipyPop (cusr/benchmark/backends.py:97-162):
                scipy.optimize.least_squares(method='lm') per tree, spawn pool
  ref_host.py   ctypes binding of the reference's own host-compiled interpreters
                (ad_interp.cuh / revad_interp.cuh) built by oracle/Makefile into oracle/_ref/
  Makefile      builds oracle/_ref/ from the sources under the reference checkout

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm may import this
package. The product (`cusr_b200`) never does: its fits run on the GPU or fail.
"""
