// pack.h — host-side compiler (pop.bin bytecode -> device program) and the cost-binned
// scheduler that groups trees into evaluation bins and sample chunks.
#pragma once
#include <stdint.h>
#include <vector>
#include "../../include/cusr_co.h"
#include "program.h"

namespace cusr {

// One compiled tree.
struct CompiledTree {
    int32_t code_off = 0;
    int32_t n_instr = 0;      // forward instructions
    int32_t bcode_off = 0;
    int32_t n_bwd = 0;        // reverse instructions
    int32_t n_nodes = 0;
    int32_t K = 0;
    int32_t n_spill = 0;
    int32_t n_tape = 0;
    bool unique_const = true;
};

struct PackResult {
    std::vector<uint32_t> code;
    std::vector<CompiledTree> trees;
    int32_t max_instr = 0;
    int32_t max_spill = 0;
    int32_t max_tape = 0;
    int32_t max_K = 0;
    int32_t bad_tree = -1;     // index of the first malformed tree (CO_ERR_BADTREE)
};

// Validate and compile every tree. Returns CO_OK, CO_ERR_BOUNDS or CO_ERR_BADTREE.
int compile_population(const PopHeader *h, const int32_t *nt, const float *nv,
                       const int32_t *ci, const TreeMeta *metas, PackResult *out);

// Compile one tree (prefix bytecode of n nodes, K constants, n_vars inputs) and append
// its program to `code`. Returns CO_OK / CO_ERR_BOUNDS / CO_ERR_BADTREE.
int compile_tree(const int32_t *nt, const float *nv, const int32_t *ci, int n, int K,
                 int n_vars, std::vector<uint32_t> &code, CompiledTree &ct);

// Scheduler bins: trees are grouped by constant-count class (the register footprint of
// the fused accumulation), each bin evaluated by one kernel instantiation.
struct Bin {
    int kc = 0;                       // constant-count class (template parameter)
    int tclass = 0;                   // tape-size class (shared-memory reservation)
    std::vector<int32_t> trees;       // tree ids, most expensive first
    int32_t max_instr = 0, max_spill = 0, max_tape = 0;
    int64_t max_items = 0;            // sum of chunks of the bin's trees
    int64_t item_off = 0;             // offset of the bin in the device item array
    int64_t tree_off = 0;             // offset of the bin in the device tree-list array
    double cost = 0.0;
};

struct Schedule {
    std::vector<Bin> bins;
    std::vector<TreeDesc> desc;       // per tree, device layout
    int32_t chunk = 0;                // samples per work item
    int32_t round = 0;                // samples per thread-block round (threads * V)
    int64_t partial_elems = 0;        // per-chunk partial sums, all trees
    int64_t block_elems = 0;          // current normal-equation blocks, all trees
    int64_t total_items = 0;
};

// K classes for fp32 and fp64 arithmetic (largest class = cooperative accumulation; 1 and 2
// = forward-mode tangents, for K <= fwd_max).
int kc_class(int K, bool fp64, int fwd_max = 0);
// Tape-size classes (slot bounds 8, 16, 24, 32, 48, 64, 96, 128, 192, 256).
int tape_class(int n_tape);

// Build the schedule: bins, per-tree descriptors, chunking (round = samples per round of a
// block, resident = concurrently resident blocks on the device).
// With S > 1 the entries are fits (tree m = entry / S, start entry % S): `pk.trees` and
// `metas` hold one record per fit (the fits of a tree share its program), the target row is
// the tree's.
void build_schedule(const PackResult &pk, const TreeMeta *metas, int M, int N,
                    bool y_shared, bool fp64, int round, int resident, Schedule *out,
                    int fwd_max = 0, int S = 1);

// Reference evaluation of a compiled program on the host (fp64), forward value plus the
// reverse sweep into grad[0..K) (read through the row table that follows the n_bwd reverse
// words). Used by the CPU tests of the compiler.
double host_eval_program(const uint32_t *fwd, int n_fwd, const uint32_t *bwd, int n_bwd,
                         const double *x, const double *c, int K, double *grad);
void decode_xop(uint32_t xop, uint32_t &op, uint32_t &mode, uint32_t &swap);

}  // namespace cusr
