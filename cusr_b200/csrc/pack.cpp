// pack.cpp — validate pop.bin trees, compile them to register-stack programs, and build the
// cost-binned evaluation schedule.
#include "pack.h"

#include <thread>
#include "ops.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace cusr {

// Decode a forward opcode back to (op, mode, swap).
void decode_xop(uint32_t xop, uint32_t &op, uint32_t &mode, uint32_t &swap) {
    if (xop < 8) { op = OP_LOAD; mode = (xop & 1) ? M_CONST : M_VAR; swap = 0; return; }
    if (xop < 32) { op = OP_SIN + (xop - 8); mode = M_NONE; swap = 0; return; }
    const uint32_t r = xop - 32;
    op = OP_ADD + r / 6;
    const uint32_t m = (r % 6) / 2;
    mode = m == 0 ? M_VAR : (m == 1 ? M_CONST : M_POP);
    swap = r & 1;
}

namespace {

struct Node {
    int32_t type;     // NodeType
    int32_t op;       // OP_* for functions
    int32_t idx;      // var index / const rank for leaves
    int32_t left = -1, right = -1;
    int32_t need = 1; // Sethi–Ullman register need
};

uint32_t map_unary(int fid) {
    switch (fid) {
        case F_SIN: return OP_SIN;   case F_COS: return OP_COS;   case F_TAN: return OP_TAN;
        case F_SINH: return OP_SINH; case F_COSH: return OP_COSH; case F_TANH: return OP_TANH;
        case F_LOG: return OP_LOG;   case F_LOOSE_LOG: return OP_LOGABS;
        case F_EXP: return OP_EXP;   case F_INV: return OP_INV;   case F_LOOSE_INV: return OP_INV;
        case F_NEG: return OP_NEG;   case F_ABS: return OP_ABS;
        case F_SQRT: return OP_SQRT; case F_LOOSE_SQRT: return OP_SQRTABS;
        default: return OP_UZERO;    // unknown id: value 0 (lm_core.cuh:82)
    }
}

uint32_t map_binary(int fid) {
    switch (fid) {
        case F_ADD: return OP_ADD; case F_SUB: return OP_SUB; case F_MUL: return OP_MUL;
        case F_DIV: return OP_DIV; case F_LOOSE_DIV: return OP_DIV;
        case F_POW: return OP_POW; case F_LOOSE_POW: return OP_POWABS;
        case F_MAX: return OP_MAX; case F_MIN: return OP_MIN;
        case F_LT: return OP_LT;   case F_GT: return OP_GT;
        case F_LE: return OP_LE;   case F_GE: return OP_GE;
        default: return OP_BZERO;  // unknown id: value 0 (lm_core.cuh:100)
    }
}

// Code generation. Forward: each node's value is left in TOS (register), leaves feeding a
// binary operator are folded into it, two subtree children run in Sethi–Ullman order with
// the first one spilled. Reverse: generated from the same tree walk, so it addresses the
// forward program's spill and tape slots.
//
// Activity: a node is active when its subtree holds a constant. Only active nodes have
// adjoint work (the derivative of f with respect to the constants never flows through a
// constant-free subtree), so the reverse program skips inactive subtrees entirely, and the
// tape partials of inactive nodes are not kept: their forward stores go to two dump slots
// (0, 1) instead of slots of their own. Values are unchanged; the gradient is the same
// sum of the same products, minus the terms that are structurally zero.
struct Gen {
    const std::vector<Node> &nodes;
    const std::vector<char> &act;
    std::vector<uint32_t> &code;
    std::vector<uint32_t> word;   // per node: its forward instruction (leaf: PUSH / LOAD)
    std::vector<int32_t> first;   // per two-subtree node: the child evaluated (and spilled) first
    int dep = 0, max_dep = 0, tape = 0;
    bool overflow = false;

    bool is_leaf(int i) const { return nodes[i].type == NT_VAR || nodes[i].type == NT_CONST; }
    uint32_t leaf_mode(int i) const { return nodes[i].type == NT_VAR ? M_VAR : M_CONST; }

    uint32_t alloc_tape(uint32_t op, uint32_t mode, bool keep) {
        int n = tape_slots(op, mode);
        if (!n) return 0;
        if (!keep) return 0;           // dump slots 0..1
        int ts = tape;
        tape += n;
        if (tape > PROG_MAX_TAPE) overflow = true;
        return (uint32_t)ts;
    }

    void emit_leaf(int i, bool live) {
        uint32_t sd = 0;
        if (live) {
            sd = (uint32_t)dep++;
            max_dep = std::max(max_dep, dep);
            if (dep > PROG_MAX_SPILL) overflow = true;
        }
        const bool var = nodes[i].type == NT_VAR;
        const uint32_t xop = live ? (var ? XOP_PUSH_VAR : XOP_PUSH_CONST)
                                  : (var ? XOP_LOAD_VAR : XOP_LOAD_CONST);
        word[(size_t)i] = enc(xop, (uint32_t)nodes[i].idx, sd, 0);
        code.push_back(word[(size_t)i]);
    }

    // binary instruction with canonical operand order: commutative operators never swap, a
    // swapped comparison becomes the mirrored comparison
    void emit_bin(int i, uint32_t op, uint32_t mode, uint32_t swap, uint32_t idx, uint32_t sd) {
        if (swap && (op == OP_ADD || op == OP_MUL || op == OP_BZERO)) swap = 0;
        if (swap && (op == OP_LT || op == OP_GT || op == OP_LE || op == OP_GE)) {
            op = op == OP_LT ? OP_GT : op == OP_GT ? OP_LT : op == OP_LE ? OP_GE : OP_LE;
            swap = 0;
        }
        const uint32_t ts = alloc_tape(op, mode, act[(size_t)i] != 0);
        word[(size_t)i] = enc(xop_bin(op, mode, swap), idx, sd, ts);
        code.push_back(word[(size_t)i]);
    }

    // Emit code leaving node i's value in TOS. `live`: TOS holds a value that must survive.
    void gen(int i, bool live) {
        const Node &n = nodes[i];
        if (is_leaf(i)) { emit_leaf(i, live); return; }
        if (n.type == NT_UFUNC) {
            gen(n.left, live);
            const uint32_t op = (uint32_t)n.op;
            const uint32_t ts = alloc_tape(op, M_NONE, act[(size_t)i] != 0);
            word[(size_t)i] = enc(xop_un(op), 0, 0, ts);
            code.push_back(word[(size_t)i]);
            return;
        }
        const int L = n.left, R = n.right;
        const uint32_t op = (uint32_t)n.op;
        if (is_leaf(R)) {                       // TOS = value(L) OP leaf
            gen(L, live);
            emit_bin(i, op, leaf_mode(R), 0, (uint32_t)nodes[R].idx, 0);
            return;
        }
        if (is_leaf(L)) {                       // TOS = leaf OP value(R)
            gen(R, live);
            emit_bin(i, op, leaf_mode(L), 1, (uint32_t)nodes[L].idx, 0);
            return;
        }
        // both children are subtrees: the one with the larger need goes first and is spilled
        const bool left_first = nodes[L].need >= nodes[R].need;
        const int f = left_first ? L : R, second = left_first ? R : L;
        first[(size_t)i] = f;
        gen(f, live);
        gen(second, true);
        --dep;
        emit_bin(i, op, M_POP, left_first ? 1u : 0u, 0, (uint32_t)dep);
    }

    // ---- reverse program ----
    std::vector<uint32_t> *rev = nullptr;
    void put(uint32_t b, uint32_t idx, uint32_t sd, uint32_t ts) { rev->push_back(enc(b, idx, sd, ts)); }

    // Reverse of node i's subtree with its adjoint in `adj`. `restore`: the forward code of
    // this subtree began with a PUSH whose spill slot `rsd` holds the adjoint of an active
    // sibling evaluated earlier; that adjoint is reloaded once this subtree is done.
    void rgen(int i, bool restore, uint32_t rsd) {
        const Node &n = nodes[(size_t)i];
        if (n.type == NT_CONST) {
            if (restore) put(B_GRAD_RESTORE, (uint32_t)n.idx, rsd, 0);
            else put(B_GRAD, (uint32_t)n.idx, 0, 0);
            return;
        }
        if (!act[(size_t)i]) {                  // VAR leaf or constant-free subtree
            if (restore) put(B_RESTORE, 0, rsd, 0);
            return;
        }
        const uint32_t w = word[(size_t)i];
        uint32_t op, mode, swap;
        decode_xop(w_code(w), op, mode, swap);
        const uint32_t idx = w_idx(w), sd = w_sd(w), ts = w_ts(w);
        if (n.type == NT_UFUNC) {
            const uint32_t b = op == OP_NEG ? B_NEG : (op == OP_UZERO ? B_ZERO : B_SCALE_T0);
            // two chained scaling unary nodes: one instruction
            const Node &c = nodes[(size_t)n.left];
            if (b == B_SCALE_T0 && c.type == NT_UFUNC && c.op != OP_NEG && c.op != OP_UZERO) {
                put(B_SCALE2_T, w_ts(word[(size_t)n.left]), 0, ts);
                rgen(c.left, restore, rsd);
                return;
            }
            put(b, 0, 0, ts);
            rgen(n.left, restore, rsd);
            return;
        }
        const bool V = mode == M_VAR, C = mode == M_CONST;
        if (V || C) {
            // TOS = the subtree child t, source = the folded leaf (active iff a constant)
            const int t = is_leaf(n.right) ? n.left : n.right;
            const bool at = act[(size_t)t] != 0;
            int b = -1;
            switch (op) {
                case OP_ADD: b = V ? -1 : B_GRAD; break;
                case OP_SUB:
                    if (!swap) b = V ? -1 : B_GRAD_NEG;
                    else b = V ? B_NEG : (at ? B_GRAD_THEN_NEG : B_GRAD);
                    break;
                case OP_MUL: b = V ? B_SCALE_X : B_MULC; break;
                case OP_DIV: case OP_POW: case OP_POWABS: b = V ? B_SCALE_T0 : B_GRAD_T1_T0; break;
                case OP_MAX: case OP_MIN: b = V ? B_SCALE_T0 : B_GRAD_1MT0_T0; break;
                default: b = V ? B_ZERO : B_GRAD_ZERO; break;
            }
            if (C && !at) {
                // only the constant needs its partial; the TOS subtree is inactive
                if (b == B_GRAD && restore) { put(B_GRAD_RESTORE, idx, rsd, 0); return; }
                put((uint32_t)b, idx, 0, ts);
                if (restore) put(B_RESTORE, 0, rsd, 0);
                return;
            }
            if (b >= 0) put((uint32_t)b, idx, 0, ts);
            rgen(t, restore, rsd);
            return;
        }
        // M_POP: TOS = the second-evaluated child, the spill slot sd = the first
        const int fc = first[(size_t)i], second = fc == n.left ? n.right : n.left;
        const bool af = act[(size_t)fc] != 0, as = act[(size_t)second] != 0;
        // partials: dt (TOS) at ts, ds (spilled operand) at ts + 1 (MAX / MIN: ds = 1 - dt)
        if (af && as) {
            int b;
            switch (op) {
                case OP_ADD: b = B_SPILL; break;
                case OP_SUB: b = swap ? B_SPILL_THEN_NEG : B_SPILL_NEG; break;
                case OP_MUL: case OP_DIV: case OP_POW: case OP_POWABS: b = B_SPILL_T1_T0; break;
                case OP_MAX: case OP_MIN: b = B_SPILL_1MT0_T0; break;
                default: b = B_SPILL_ZERO; break;
            }
            put((uint32_t)b, 0, sd, ts);
            rgen(second, true, sd);
            rgen(fc, restore, rsd);
        } else if (as) {                        // adjoint to the TOS operand only
            int b;
            switch (op) {
                case OP_ADD: b = -1; break;
                case OP_SUB: b = swap ? B_NEG : -1; break;
                case OP_MUL: case OP_DIV: case OP_POW: case OP_POWABS:
                case OP_MAX: case OP_MIN: b = B_SCALE_T0; break;
                default: b = B_ZERO; break;
            }
            if (b >= 0) put((uint32_t)b, 0, 0, ts);
            rgen(second, false, 0);
            if (restore) put(B_RESTORE, 0, rsd, 0);
        } else {                                // adjoint to the spilled operand only
            int b;
            uint32_t t = ts;
            switch (op) {
                case OP_ADD: b = -1; break;
                case OP_SUB: b = swap ? -1 : B_NEG; break;
                case OP_MUL: case OP_DIV: case OP_POW: case OP_POWABS: b = B_SCALE_T0; t = ts + 1; break;
                case OP_MAX: case OP_MIN: b = B_SCALE_1MT0; break;
                default: b = B_ZERO; break;
            }
            if (b >= 0) put((uint32_t)b, 0, 0, t);
            rgen(fc, restore, rsd);
        }
    }
};

// Tape slots a reverse word reads.
int reverse_reads(uint32_t w, uint32_t (&s)[2]) {
    switch (w_bop(w)) {
        case B_SCALE_T0: case B_MULC: case B_GRAD_1MT0_T0: case B_SPILL_1MT0_T0:
        case B_SCALE_1MT0:
            s[0] = w_ts(w);
            return 1;
        case B_GRAD_T1_T0: case B_SPILL_T1_T0:
            s[0] = w_ts(w); s[1] = w_ts(w) + 1;
            return 2;
        case B_SCALE2_T:
            s[0] = w_ts(w); s[1] = w_idx(w);
            return 2;
        default:
            return 0;
    }
}

// Gradient rows in dead tape slots. A tape slot is dead once the reverse program has read it
// for the last time; slots it never reads (the dump slots of inactive nodes, the unused
// partial of a node with one active operand) are dead from the start. Row k goes to a slot
// that is dead at the reverse program's first write of constant k — a word reads its tape
// entries before it writes its row, and every thread touches only its own column — and the
// residual row and one shared zero row (constants that do not occur in the tree) take slots
// that are dead at the end. A row finds a new slot past the tape only when no dead one is
// left. Among dead slots the lowest whose residue mod 8 no other row of the same 8-row group
// holds is taken: the rows are padded so that residues map to distinct shared-memory banks of
// the tensor-core fragment loads. Rewrites the row writes of `rev` (slot field, B_ACC for
// the second and later writes of a constant), appends B_ROW_ZERO when a zero row is needed,
// and returns the slot of each row (K + 1 entries, the residual last) and the slot count.
bool place_rows(std::vector<uint32_t> &rev, int n_tape, int K, std::vector<int> &row_slot,
                int &n_slots) {
    const int P = (int)rev.size();
    int last[256];                             // last reverse word reading the slot
    for (int i = 0; i < 256; ++i) last[i] = -1;
    for (int p = 0; p < P; ++p) {
        uint32_t s[2];
        const int n = reverse_reads(rev[(size_t)p], s);
        for (int i = 0; i < n; ++i) last[s[i]] = p;
    }
    char taken[256] = {};
    std::vector<uint8_t> group_res((size_t)K / 8 + 1, 0);   // residues mod 8 used per 8-row group
    n_slots = n_tape;
    auto pick = [&](int row, int p) -> int {   // p = -1: dead at the end
        int best = -1;
        for (int s = 0; s < n_tape; ++s) {
            if (taken[(size_t)s] || (p >= 0 && last[(size_t)s] > p)) continue;
            if (!(group_res[(size_t)row / 8] & (1u << (s & 7)))) { best = s; break; }
            if (best < 0) best = s;
        }
        if (best < 0) best = n_slots++;
        if (best > PROG_MAX_TAPE) return -1;
        taken[(size_t)best] = 1;
        group_res[(size_t)row / 8] |= (uint8_t)(1u << (best & 7));
        return best;
    };
    row_slot.assign((size_t)K + 1, -1);
    for (int p = 0; p < P; ++p) {
        uint32_t w = rev[(size_t)p];
        const uint32_t b = w_bop(w);
        if (!is_row_write(b)) continue;
        const int k = (int)w_idx(w);
        bool acc = true;
        if (row_slot[(size_t)k] < 0) {
            row_slot[(size_t)k] = pick(k, p);
            if (row_slot[(size_t)k] < 0) return false;
            acc = false;
        }
        const uint32_t code = b | (acc ? B_ACC : 0u);
        const uint32_t slot = (uint32_t)row_slot[(size_t)k];
        w = b == B_GRAD_RESTORE ? enc(code, w_idx(w), w_sd(w), slot) : enc(code, w_idx(w), slot, w_ts(w));
        rev[(size_t)p] = w;
    }
    int zero = -1;
    for (int k = 0; k < K; ++k) {
        if (row_slot[(size_t)k] >= 0) continue;
        if (zero < 0) {
            zero = pick(k, -1);
            if (zero < 0) return false;
            rev.push_back(enc(B_ROW_ZERO, 0, 0, (uint32_t)zero));
        }
        row_slot[(size_t)k] = zero;
    }
    row_slot[(size_t)K] = pick(K, -1);
    return row_slot[(size_t)K] >= 0;
}

}  // namespace

int compile_tree(const int32_t *nt, const float *nv, const int32_t *ci, int n, int K,
                 int n_vars, std::vector<uint32_t> &code, CompiledTree &ct) {
    if (n <= 0) return CO_ERR_BADTREE;
    if (n > CO_MAX_NODES) return CO_ERR_BOUNDS;
    std::vector<Node> nodes((size_t)n);
    std::vector<int32_t> st;
    st.reserve((size_t)n);
    std::vector<int32_t> seen((size_t)std::max(K, 1), 0);
    std::vector<char> act((size_t)n, 0);   // subtree holds a constant (children first)
    bool unique = true;
    // Right-to-left scan: the same visiting order as the reference interpreter
    // (lm_core.cuh:63), building the child links of each function node.
    for (int i = n - 1; i >= 0; --i) {
        Node &nd = nodes[(size_t)i];
        nd.type = nt[i];
        switch (nt[i]) {
            case NT_VAR: {
                int v = (int)nv[i];
                if (!(nv[i] >= 0.0f) || v < 0 || v >= n_vars || v > CO_MAX_VARS) return CO_ERR_BADTREE;
                nd.idx = v; nd.need = 1;
                st.push_back(i);
                break;
            }
            case NT_CONST: {
                int k = ci[i];
                if (k < 0 || k >= K) return CO_ERR_BADTREE;
                nd.idx = k; nd.need = 1;
                if (seen[(size_t)k]++) unique = false;
                act[(size_t)i] = 1;
                st.push_back(i);
                break;
            }
            case NT_UFUNC: {
                if (st.empty()) return CO_ERR_BADTREE;
                nd.left = st.back(); st.pop_back();
                nd.op = (int32_t)map_unary((int)nv[i]);
                nd.need = nodes[(size_t)nd.left].need;
                act[(size_t)i] = act[(size_t)nd.left];
                st.push_back(i);
                break;
            }
            case NT_BFUNC: {
                if (st.size() < 2) return CO_ERR_BADTREE;
                nd.left = st.back(); st.pop_back();    // first child in prefix order = left
                nd.right = st.back(); st.pop_back();
                nd.op = (int32_t)map_binary((int)nv[i]);
                act[(size_t)i] = (char)(act[(size_t)nd.left] | act[(size_t)nd.right]);
                const Node &l = nodes[(size_t)nd.left], &r = nodes[(size_t)nd.right];
                const bool lleaf = l.type == NT_VAR || l.type == NT_CONST;
                const bool rleaf = r.type == NT_VAR || r.type == NT_CONST;
                if (rleaf) nd.need = l.need;
                else if (lleaf) nd.need = r.need;
                else nd.need = (l.need == r.need) ? l.need + 1 : std::max(l.need, r.need);
                st.push_back(i);
                break;
            }
            default:
                return CO_ERR_BADTREE;
        }
    }
    if (st.size() != 1 || st[0] != 0) return CO_ERR_BADTREE;
    for (int k = 0; k < K; ++k)
        if (seen[(size_t)k] != 1) unique = false;

    ct.code_off = (int32_t)code.size();
    // dump slots for the partials of inactive nodes (only when some inactive node has any)
    bool dump = false;
    for (int i = 0; i < n && !dump; ++i) {
        const Node &nd = nodes[(size_t)i];
        if (act[(size_t)i] || (nd.type != NT_UFUNC && nd.type != NT_BFUNC)) continue;
        uint32_t mode = M_NONE;
        if (nd.type == NT_BFUNC) {
            const Node &r = nodes[(size_t)nd.right], &l = nodes[(size_t)nd.left];
            if (r.type == NT_VAR || r.type == NT_CONST) mode = r.type == NT_VAR ? M_VAR : M_CONST;
            else if (l.type == NT_VAR || l.type == NT_CONST) mode = l.type == NT_VAR ? M_VAR : M_CONST;
            else mode = M_POP;
        }
        dump = tape_slots((uint32_t)nd.op, mode) > 0;
    }
    Gen g{nodes, act, code};
    g.word.assign((size_t)n, 0u);
    g.first.assign((size_t)n, -1);
    g.tape = dump ? 2 : 0;
    g.gen(0, false);
    if (g.overflow) { code.resize((size_t)ct.code_off); return CO_ERR_BOUNDS; }
    ct.n_instr = (int32_t)code.size() - ct.code_off;
    ct.bcode_off = (int32_t)code.size();
    int n_slots = g.tape;
    std::vector<int> row_slot;
    {
        std::vector<uint32_t> rev;
        g.rev = &rev;
        g.rgen(0, false, 0);
        if (!place_rows(rev, g.tape, K, row_slot, n_slots)) {
            code.resize((size_t)ct.code_off);
            return CO_ERR_BOUNDS;
        }
        code.insert(code.end(), rev.begin(), rev.end());
    }
    ct.n_bwd = (int32_t)code.size() - ct.bcode_off;
    // the row table follows the reverse program
    for (int i = 0; i < row_table_words(K); ++i) {
        uint32_t t = 0;
        for (int b = 0; b < 4; ++b) {
            const int r = 4 * i + b;
            if (r <= K) t |= (uint32_t)row_slot[(size_t)r] << (8 * b);
        }
        code.push_back(t);
    }
    // the interpreter dispatches without a bounds check: every word must be a known opcode
    for (int i = 0; i < ct.n_instr; ++i)
        if (!valid_forward_code(w_code(code[(size_t)(ct.code_off + i)]))) return CO_ERR_BADTREE;
    for (int i = 0; i < ct.n_bwd; ++i)
        if (!valid_reverse_code(w_code(code[(size_t)(ct.bcode_off + i)]))) return CO_ERR_BADTREE;
    ct.n_nodes = n;
    ct.K = K;
    ct.n_spill = g.max_dep;
    ct.n_tape = n_slots;
    ct.unique_const = unique;
    return CO_OK;
}

namespace {

// Compile trees [m0, m1) into `code` (offsets relative to its start). On failure returns the
// code and sets `bad` to the first failing tree.
int compile_range(const PopHeader *h, const int32_t *nt, const float *nv, const int32_t *ci,
                  const TreeMeta *metas, int m0, int m1, std::vector<uint32_t> &code,
                  std::vector<CompiledTree> &trees, int &bad) {
    for (int m = m0; m < m1; ++m) {
        const TreeMeta &tm = metas[m];
        bad = m;
        if (tm.K < 0 || tm.K > CO_MAX_K) return CO_ERR_BOUNDS;
        if (tm.n_nodes <= 0 || tm.node_offset < 0 ||
            (int64_t)tm.node_offset + tm.n_nodes > (int64_t)h->total_nodes ||
            tm.c_offset < 0 || (int64_t)tm.c_offset + tm.K > (int64_t)h->total_c)
            return CO_ERR_BADTREE;
        int rc = compile_tree(nt + tm.node_offset, nv + tm.node_offset, ci + tm.node_offset,
                              tm.n_nodes, tm.K, h->n_vars, code, trees[(size_t)m]);
        if (rc != CO_OK) return rc;
    }
    bad = -1;
    return CO_OK;
}

}  // namespace

// Trees compile independently: large populations are split into contiguous ranges of about
// equal node count, compiled on host threads and concatenated in tree order, so the
// program layout (and every result) is the same as a serial compile.
int compile_population(const PopHeader *h, const int32_t *nt, const float *nv,
                       const int32_t *ci, const TreeMeta *metas, PackResult *out) {
    const int M = h->M_prob;
    out->code.clear();
    out->trees.assign((size_t)M, CompiledTree{});
    out->bad_tree = -1;
    unsigned hw = std::thread::hardware_concurrency();
    int n_parts = (int)std::min<unsigned>(hw ? hw : 1, 16);
    if (M < 4096 || h->total_nodes < (1 << 16)) n_parts = 1;
    // range boundaries by node count (metas are validated inside the ranges; a corrupt
    // n_nodes only skews the split)
    std::vector<int> bounds{0};
    if (n_parts > 1) {
        const double per = (double)std::max<int64_t>(h->total_nodes, 1) / n_parts;
        double acc = 0.0;
        for (int m = 0; m < M && (int)bounds.size() < n_parts; ++m) {
            acc += (double)std::max(metas[m].n_nodes, 0);
            if (acc >= per * (double)bounds.size()) bounds.push_back(m + 1);
        }
    }
    if (bounds.back() != M) bounds.push_back(M);
    const int P = (int)bounds.size() - 1;
    std::vector<std::vector<uint32_t>> codes((size_t)P);
    std::vector<int> rcs((size_t)P, CO_OK), bads((size_t)P, -1);
    auto work = [&](int p) {
        codes[(size_t)p].reserve((size_t)h->total_nodes / (size_t)P + 64);
        rcs[(size_t)p] = compile_range(h, nt, nv, ci, metas, bounds[(size_t)p],
                                       bounds[(size_t)p + 1], codes[(size_t)p], out->trees,
                                       bads[(size_t)p]);
    };
    if (P == 1) {
        work(0);
    } else {
        std::vector<std::thread> th;
        th.reserve((size_t)P);
        for (int p = 0; p < P; ++p) th.emplace_back(work, p);
        for (std::thread &t : th) t.join();
    }
    for (int p = 0; p < P; ++p) {
        if (rcs[(size_t)p] != CO_OK) {   // the lowest failing tree, as a serial compile
            out->bad_tree = bads[(size_t)p];
            return rcs[(size_t)p];
        }
    }
    size_t total = 0;
    for (const auto &c : codes) total += c.size();
    out->code.reserve(total);
    for (int p = 0; p < P; ++p) {
        const int32_t base = (int32_t)out->code.size();
        for (int m = bounds[(size_t)p]; m < bounds[(size_t)p + 1]; ++m) {
            CompiledTree &ct = out->trees[(size_t)m];
            ct.code_off += base;
            ct.bcode_off += base;
        }
        out->code.insert(out->code.end(), codes[(size_t)p].begin(), codes[(size_t)p].end());
    }
    for (const CompiledTree &ct : out->trees) {
        out->max_instr = std::max(out->max_instr, ct.n_instr + ct.n_bwd + row_table_words(ct.K));
        out->max_spill = std::max(out->max_spill, ct.n_spill);
        out->max_tape = std::max(out->max_tape, ct.n_tape);
        out->max_K = std::max(out->max_K, ct.K);
    }
    return CO_OK;
}

int tape_class(int n_tape) {
#ifdef CUSR_NO_TAPE_CLASSES
    (void)n_tape;
    return 0;
#else
    static const int bounds[] = {8, 16, 24, 32, 48, 64, 96, 128, 192, 256};
    int c = 0;
    while (c < 9 && n_tape > bounds[c]) ++c;
    return c;
#endif
}

// K <= fwd_max (0, 1 or 2) goes to the forward-mode classes 1 and 2 (tangents in registers).
int kc_class(int K, bool fp64, int fwd_max) {
    if (K <= fwd_max) return K <= 1 ? 1 : 2;
    if (fp64) {
        if (K <= 4) return 4;
        if (K <= 8) return 8;
        return 32;
    }
    if (K <= 4) return 4;
    if (K <= 8) return 8;
    if (K <= 12) return 12;
    if (K <= 16) return 16;
    return 32;
}

void build_schedule(const PackResult &pk, const TreeMeta *metas, int M, int N,
                    bool y_shared, bool fp64, int round, int resident, Schedule *out,
                    int fwd_max, int S) {
    out->bins.clear();
    out->desc.assign((size_t)M, TreeDesc{});
    out->round = round;
    const int64_t rounds_per_tree = (N + round - 1) / round;
    const int64_t total_rounds = rounds_per_tree * (int64_t)M;
    int64_t per_item = total_rounds / std::max<int64_t>(1, 8 * (int64_t)resident);
    // at most 4,096 samples per item
    per_item = std::min<int64_t>(std::max(1, 4096 / round), std::max<int64_t>(1, per_item));
    out->chunk = (int32_t)(per_item * round);
    const int n_chunks = (int)((N + out->chunk - 1) / out->chunk);
    const int64_t ldy = ((int64_t)N + round - 1) / round * round;

    // bins: (constant-count class, tape class); a launch reserves shared memory for the
    // largest tape of its bin, so trees of very different tape sizes are kept apart
    std::vector<int> bin_of_class(33 * 16, -1);
    std::vector<double> cost((size_t)M);
    int64_t p_off = 0, q_off = 0;
    for (int m = 0; m < M; ++m) {
        const CompiledTree &ct = pk.trees[(size_t)m];
        TreeDesc &d = out->desc[(size_t)m];
        d.code_off = ct.code_off;
        d.n_instr = ct.n_instr;
        d.bcode_off = ct.bcode_off;
        d.n_bwd = ct.n_bwd;
        d.K = ct.K;
        d.c_off = metas[m].c_offset;
        d.y_off = y_shared ? 0 : (int64_t)(m / S) * ldy;
        d.p_off = p_off;
        d.q_off = q_off;
        d.n_chunks = n_chunks;
        d.n_spill = (uint16_t)ct.n_spill;
        d.n_tape = (uint8_t)ct.n_tape;
        d.flags = ct.unique_const ? TD_UNIQUE_CONST : 0;
        const int P = nblock_size(ct.K);
        p_off += (int64_t)n_chunks * P;
        q_off += P;
        // forward + reverse sweep per instruction, plus the normal-equation update
        cost[(size_t)m] = (double)N * (2.0 * ct.n_instr + 0.5 * ct.K * (ct.K + 1) * 0.25);
        const int kc = kc_class(ct.K, fp64, fwd_max);
        const int tc = kc <= 2 ? 0 : tape_class(ct.n_tape);   // forward mode keeps no tape
        const size_t key = (size_t)kc * 16 + (size_t)tc;
        if (bin_of_class[key] < 0) {
            bin_of_class[key] = (int)out->bins.size();
            out->bins.push_back(Bin{});
            out->bins.back().kc = kc;
            out->bins.back().tclass = tc;
        }
        Bin &b = out->bins[(size_t)bin_of_class[key]];
        b.trees.push_back(m);
        b.max_instr = std::max(b.max_instr, ct.n_instr + ct.n_bwd + row_table_words(ct.K));
        b.max_spill = std::max(b.max_spill, ct.n_spill);
        b.max_tape = std::max(b.max_tape, ct.n_tape);
        b.max_items += n_chunks;
        b.cost += cost[(size_t)m];
    }
    // bins in ascending class order; trees inside a bin most expensive first (LPT order)
    std::sort(out->bins.begin(), out->bins.end(), [](const Bin &a, const Bin &b) {
        return a.kc != b.kc ? a.kc < b.kc : a.tclass < b.tclass;
    });
    int64_t item_off = 0, tree_off = 0;
    for (Bin &b : out->bins) {
        std::stable_sort(b.trees.begin(), b.trees.end(), [&](int32_t x, int32_t y) {
            return cost[(size_t)x] > cost[(size_t)y];
        });
        b.item_off = item_off;
        b.tree_off = tree_off;
        item_off += b.max_items;
        tree_off += (int64_t)b.trees.size();
    }
    out->partial_elems = p_off;
    out->block_elems = q_off;
    out->total_items = item_off;
}

double host_eval_program(const uint32_t *fwd, int n_fwd, const uint32_t *bwd, int n_bwd,
                         const double *x, const double *c, int K, double *grad) {
    double spill[PROG_MAX_SPILL + 1] = {};
    double tape[PROG_MAX_TAPE + 2] = {};
    double tos = 0.0;
    for (int pc = 0; pc < n_fwd; ++pc) {
        const uint32_t w = fwd[pc];
        const uint32_t idx = w_idx(w), sd = w_sd(w), ts = w_ts(w);
        uint32_t op, mode, swap;
        decode_xop(w_code(w), op, mode, swap);
        if (op == OP_LOAD) {
            if (w_code(w) >= XOP_PUSH_VAR) spill[sd] = tos;
            tos = (mode == M_VAR) ? x[idx] : c[idx];
        } else if (op < OP_ADD) {
            double r, d;
            unary_op<double>(op, tos, r, d);
            if (tape_slots(op, M_NONE)) tape[ts] = d;
            tos = r;
        } else {
            const double s = (mode == M_VAR) ? x[idx] : (mode == M_CONST ? c[idx] : spill[sd]);
            double o, da, db;
            binary_op<double>(op, swap ? s : tos, swap ? tos : s, o, da, db);
            const double dt = swap ? db : da, ds = swap ? da : db;
            switch (op) {
                case OP_MUL:
                    if (mode == M_CONST) tape[ts] = ds;
                    else if (mode == M_POP) { tape[ts] = dt; tape[ts + 1] = ds; }
                    break;
                case OP_DIV: case OP_POW: case OP_POWABS:
                    tape[ts] = dt;
                    if (mode != M_VAR) tape[ts + 1] = ds;
                    break;
                case OP_MAX: case OP_MIN: tape[ts] = dt; break;
                default: break;
            }
            tos = o;
        }
    }
    const double value = tos;
    if (!grad) return value;
    // gradient rows live in tape slots (row table after the reverse program)
    double adj = 1.0;
    for (int pc = 0; pc < n_bwd; ++pc) {
        const uint32_t w = bwd[pc];
        const uint32_t idx = w_idx(w), sd = w_sd(w), ts = w_ts(w);
        const double t0 = tape[ts], t1 = tape[ts + 1];
        const bool acc = (w_code(w) & B_ACC) != 0;
        const uint32_t rs = w_row(w);
        auto row = [&](double v) { tape[rs] = acc ? tape[rs] + v : v; };
        switch (w_bop(w)) {
            case B_GRAD: row(adj); break;
            case B_GRAD_RESTORE: row(adj); adj = spill[sd]; break;
            case B_RESTORE: adj = spill[sd]; break;
            case B_GRAD_NEG: row(-adj); break;
            case B_SPILL: spill[sd] = adj; break;
            case B_SPILL_NEG: spill[sd] = -adj; break;
            case B_NEG: adj = -adj; break;
            case B_GRAD_THEN_NEG: row(adj); adj = -adj; break;
            case B_SPILL_THEN_NEG: spill[sd] = adj; adj = -adj; break;
            case B_SCALE_X: adj = safe_mul(adj, x[idx]); break;
            case B_SCALE_T0: adj = safe_mul(adj, t0); break;
            case B_MULC: row(safe_mul(adj, t0)); adj = safe_mul(adj, c[idx]); break;
            case B_GRAD_T1_T0: row(safe_mul(adj, t1)); adj = safe_mul(adj, t0); break;
            case B_SPILL_T1_T0: spill[sd] = safe_mul(adj, t1); adj = safe_mul(adj, t0); break;
            case B_GRAD_1MT0_T0: row(safe_mul(adj, 1.0 - t0)); adj = safe_mul(adj, t0); break;
            case B_SPILL_1MT0_T0: spill[sd] = safe_mul(adj, 1.0 - t0); adj = safe_mul(adj, t0); break;
            case B_ZERO: adj = 0.0; break;
            case B_GRAD_ZERO: row(0.0); adj = 0.0; break;
            case B_SPILL_ZERO: spill[sd] = 0.0; adj = 0.0; break;
            case B_SCALE_1MT0: adj = safe_mul(adj, 1.0 - t0); break;
            case B_SCALE2_T: adj = safe_mul(safe_mul(adj, t0), tape[w_idx(w)]); break;
            case B_ROW_ZERO: tape[ts] = 0.0; break;
            default: break;
        }
    }
    const uint32_t *tab = bwd + n_bwd;
    for (int k = 0; k < K; ++k) grad[k] = tape[(tab[k / 4] >> (8 * (k % 4))) & 255u];
    return value;
}

}  // namespace cusr
