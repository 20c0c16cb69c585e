// fusion.cu -- plan-time layout fusion over the OpNode array.
//
// The reference pipeline emits pure data-movement nodes around attention:
// a merged QKV projection is split by SLICE (last dim), each head split by a
// TRANSPOSE [B,S,H,D] -> [B,H,S,D] (runtime/ops.py:149-171, 310-329), and the
// attention output is merged back by another TRANSPOSE.  The tensor-core
// attention kernel can read Q/K/V and write O through strided views, so
// those copies can be skipped -- but only when the node array proves it safe,
// since the library sees pointers, not tensor names:
//   * the skipped node's output is read by nobody but its one consumer and
//     is not a graph output: callers register graph outputs with rt_protect
//     (the Python executor does), and the last node's output is always kept;
//   * the source the fused consumer reads instead is not written by any node
//     between the skipped producer and the consumer;
//   * for the output side, nothing between attention and the merge TRANSPOSE
//     touches the merge's output region;
//   * the fused output does not overlap Q; it may overlap K and V, which the
//     tensor-core path's pre-passes have consumed before O is written.
// Every node's read and write extents are computed from its op, shape and
// extras; a node whose read extent is not known blocks any fusion across it.
// RT_FUSE=0 disables the pass (RT_FUSE_GEMM=0 only the GEMM epilogue chains;
// RT_FUSE_HANDOFF=1 turns on the split-operand hand-off between GEMMs;
// RT_FUSE_NORM_SPLIT=0 turns off the norm -> GEMM split-operand hand-off).
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <vector>

#include "gemm.h"
#include "rt_internal.h"

namespace rt {


namespace {

struct Range {
    uintptr_t lo = 0, hi = 0;
};
inline bool overlaps(Range a, Range b) { return a.lo < b.hi && b.lo < a.hi; }
inline Range rng(const void* p, size_t bytes) {
    Range r;
    r.lo = reinterpret_cast<uintptr_t>(p);
    r.hi = r.lo + bytes;
    return r;
}
constexpr Range ALL{0, ~(uintptr_t)0};

int64_t bcast_extent(const int* strides, const int* shape, int nd) {
    int64_t e = 0;
    for (int d = 0; d < nd; d++) e += (int64_t)(shape[d] - 1) * strides[d];
    return e + 1;
}

Range write_range(const OpNode& n) { return rng(n.output, (size_t)total_elements(n) * n.elem_size); }

// What a node reads; ALL when the extent is not derivable.
void read_ranges(const OpNode& n, std::vector<Range>& out) {
    out.clear();
    const size_t numel = (size_t)total_elements(n), es = n.elem_size;
    const size_t C = (size_t)last_dim(n);
    auto in = [&](int i, size_t bytes) { out.push_back(rng(n.inputs[i], bytes)); };
    switch (n.op) {
        case RT_OP_RELU: case RT_OP_EXP: case RT_OP_TANH: case RT_OP_POW: case RT_OP_GELU:
        case RT_OP_RSQRT: case RT_OP_SILU: case RT_OP_NEG: case RT_OP_COS: case RT_OP_SIN:
        case RT_OP_SOFTMAX: case RT_OP_RESHAPE: case RT_OP_TRANSPOSE:
            in(0, numel * es);
            return;
        case RT_OP_ADD: case RT_OP_SUB: case RT_OP_MUL: case RT_OP_DIV: {
            const int mode = n.extra[0];
            const bool add = n.op == RT_OP_ADD;
            const int scalar = add ? 2 : 1, same = add ? 1 : 0, bc = add ? 3 : 2;
            if (mode == scalar) { in(0, numel * 4); return; }
            if (mode == same) { in(0, numel * 4); in(1, numel * 4); return; }
            if (add && mode == 0) { in(0, numel * 4); in(1, C * 4); return; }
            if (mode == bc) {
                const int nd = n.extra[1];
                if (nd < 1 || nd > 7) { out.push_back(ALL); return; }
                const int* as = &n.extra[2];
                const int* bs = &n.extra[2 + nd];
                const int* sh = &n.extra[2 + 2 * nd];
                in(0, (size_t)bcast_extent(as, sh, nd) * 4);
                in(1, (size_t)bcast_extent(bs, sh, nd) * 4);
                return;
            }
            out.push_back(ALL);
            return;
        }
        case RT_OP_FUSED_BIAS_RELU:
            in(0, numel * 4); in(1, C * 4);
            return;
        case RT_OP_GATED_ACT:
            in(0, numel * 4);
            if (n.extra[0]) { in(1, C * 4); in(2, numel * 4); } else in(1, numel * 4);
            return;
        case RT_OP_LAYERNORM:
            in(0, numel * 4); in(1, C * 4); in(2, C * 4);
            return;
        case RT_OP_RMSNORM:
            in(0, numel * 4); in(1, C * 4);
            return;
        case RT_OP_MATMUL: case RT_OP_MATMUL_ADD: {
            GemmProblem g;
            if (!decode_gemm(n, &g).good()) { out.push_back(ALL); return; }
            in(0, (size_t)(g.batches * g.M * g.K) * 4);
            in(1, (size_t)(n.extra[2] ? g.N * g.K : g.batches * g.N * g.K) * 4);
            if (g.bias) in(2, (size_t)g.N * 4);
            return;
        }
        case RT_OP_ATTENTION: {
            const int group = n.extra[4] > 0 ? n.extra[4] : 1;
            const size_t S = (size_t)n.extra[0];
            in(0, numel * 4);
            in(1, numel / group * 4);
            in(2, numel / group * 4);
            if (n.extra[3]) in(3, numel / (size_t)n.extra[1] * S * 4);   // mask [BH, S, S]
            return;   // the planned scratch input is not used by this library's kernels
        }
        case RT_OP_SLICE:
            in(0, (size_t)n.extra[0] * n.extra[1] * n.extra[4] * es);
            return;
        case RT_OP_CAT: {
            const int dim = n.extra[0];
            size_t outer = 1, inner = 1;
            for (int i = 0; i < dim; i++) outer *= n.out_shape[i];
            for (int i = dim + 1; i < n.n_dims; i++) inner *= n.out_shape[i];
            for (int k = 0; k < n.n_inputs; k++) in(k, outer * (size_t)n.extra[1 + k] * inner * es);
            return;
        }
        case RT_OP_MAX: case RT_OP_SUM: {
            const int axis = n.extra[0];
            size_t outer = 1, inner = 1;
            for (int i = 0; i < axis && i < n.n_dims; i++) outer *= n.out_shape[i];
            for (int i = axis; i < n.n_dims; i++) inner *= n.out_shape[i];
            in(0, outer * (size_t)n.extra[1] * inner * 4);
            return;
        }
        default:
            out.push_back(ALL);   // e.g. EMBEDDING: table extent unknown
            return;
    }
}

struct Analysis {
    const std::vector<OpNode>& nodes;
    std::vector<std::vector<Range>> reads;
    std::vector<Range> writes;

    // `gone`: nodes already folded away (they neither read nor write);
    // `reads_of`: nodes that now run a fused kernel reading other ranges
    explicit Analysis(const std::vector<OpNode>& ns, const std::vector<bool>* gone = nullptr,
                      const std::vector<std::pair<int, std::vector<Range>>>* reads_of = nullptr)
        : nodes(ns), reads(ns.size()), writes(ns.size()) {
        for (size_t i = 0; i < ns.size(); i++) {
            if (gone && (*gone)[i]) continue;
            read_ranges(ns[i], reads[i]);
            writes[i] = write_range(ns[i]);
        }
        if (reads_of)
            for (auto& ro : *reads_of) reads[ro.first] = ro.second;
    }
    int last_writer(Range r, int before) const {
        for (int j = before - 1; j >= 0; j--)
            if (overlaps(writes[j], r)) return j;
        return -1;
    }
};

bool aligned_view(const void* base, int64_t a, int64_t b, int64_t c) {
    return aligned16(base) && a % 4 == 0 && b % 4 == 0 && c % 4 == 0;
}

// One candidate fusion around attention node `a`.
struct Proposal {
    int a = -1;
    AttnViews views{};
    std::vector<std::pair<int, int>> skips;       // (folded node, its consumer in the original schedule)
    std::vector<std::pair<Range, int>> sources;   // range read through a view, chain start index
    std::vector<int> source_op;                   // which operand each source feeds: 0 Q, 1 K, 2 V
    Range out{};                                  // what the fused attention writes
    int out_skip = -1;                            // merge TRANSPOSE folded into the attention
    std::vector<std::pair<int, int>> redirect;    // (node, input slot) now reading `out` instead of the merge's output
};

// Pattern: operand written by a head-split TRANSPOSE [B,S,Hx,D] -> [B,Hx,S,D],
// whose input is (optionally) a last-dim SLICE of a [B,S,W] projection.
bool match_operand(const Analysis& an, int a, int which, int64_t B, int64_t Hx, int64_t S, int64_t D,
                   Proposal& pr) {
    const OpNode& att = an.nodes[a];
    const void* x = att.inputs[which];
    const Range R = rng(x, (size_t)(B * Hx * S * D) * 4);
    const int t = an.last_writer(R, a);
    if (t < 0) return false;
    const OpNode& tr = an.nodes[t];
    if (tr.op != RT_OP_TRANSPOSE || tr.n_dims != 4 || tr.elem_size != 4 || tr.output != x ||
        an.writes[t].hi != R.hi || tr.extra[0] != B || tr.extra[1] != S || tr.extra[2] != 1 ||
        tr.extra[3] != Hx || tr.extra[4] != D)
        return false;
    const Range Tin = rng(tr.inputs[0], (size_t)(R.hi - R.lo));
    const float* base = static_cast<const float*>(tr.inputs[0]);
    int64_t sb = S * Hx * D, sh = D, ss = Hx * D;
    Range src = Tin;
    int start = t;
    int slice_skip = -1;
    const int sidx = an.last_writer(Tin, t);
    if (sidx >= 0) {
        const OpNode& sl = an.nodes[sidx];
        const int64_t W = sl.extra[1];
        const float* sbase = static_cast<const float*>(sl.inputs[0]) + sl.extra[2];
        if (sl.op == RT_OP_SLICE && sl.elem_size == 4 && sl.output == tr.inputs[0] && an.writes[sidx].hi == Tin.hi &&
            sl.extra[0] == B * S && sl.extra[3] == Hx * D && sl.extra[4] == 1 && aligned_view(sbase, S * W, W, D)) {
            base = sbase;
            sb = S * W;
            ss = W;
            src = rng(sl.inputs[0], (size_t)(B * S * W) * 4);
            start = sidx;
            slice_skip = sidx;
        }
    }
    if (!aligned_view(base, sb, ss, sh)) return false;
    pr.skips.push_back({t, a});
    if (slice_skip >= 0) pr.skips.push_back({slice_skip, t});
    AttnViews& v = pr.views;
    if (which == 0) { v.q = base; v.q_sb = sb; v.q_sh = sh; v.q_ss = ss; }
    if (which == 1) { v.k = base; v.k_sb = sb; v.k_sh = sh; v.k_ss = ss; }
    if (which == 2) { v.v = base; v.v_sb = sb; v.v_sh = sh; v.v_ss = ss; }
    pr.sources.push_back({src, start});
    pr.source_op.push_back(which);
    return true;
}

// Pattern: attention output consumed by a head-merge TRANSPOSE [B,H,S,D] -> [B,S,H,D].
void match_output(const Analysis& an, int a, int64_t B, int64_t H, int64_t S, int64_t D, Proposal& pr) {
    const OpNode& att = an.nodes[a];
    for (size_t j = a + 1; j < an.nodes.size(); j++) {
        const OpNode& tr = an.nodes[j];
        if (tr.op == RT_OP_TRANSPOSE && tr.inputs[0] == att.output) {
            if (tr.n_dims == 4 && tr.elem_size == 4 && tr.extra[0] == B && tr.extra[1] == H && tr.extra[2] == 1 &&
                tr.extra[3] == S && tr.extra[4] == D && aligned_view(tr.output, S * H * D, H * D, D)) {
                pr.out_skip = (int)j;
                pr.out = an.writes[j];
                pr.views.o = static_cast<float*>(tr.output);
                pr.views.o_sb = S * H * D;
                pr.views.o_sh = D;
                pr.views.o_ss = H * D;
            }
            return;
        }
        if (overlaps(an.writes[j], an.writes[a])) return;
    }
}

// Variant: the attention writes the merged [B,S,H,D] layout into its own
// output buffer and the merge's readers are redirected there.
bool match_output_inplace(const Analysis& an, int a, int64_t B, int64_t H, int64_t S, int64_t D, Proposal& pr) {
    Proposal tmp = pr;
    match_output(an, a, B, H, S, D, tmp);
    if (tmp.out_skip < 0) return false;
    const int u = tmp.out_skip;
    const OpNode& tr = an.nodes[u];
    const Range U = an.writes[u];
    // readers of U until it is rewritten: each must read exactly U through one input slot
    std::vector<std::pair<int, int>> red;
    for (size_t j = u + 1; j < an.nodes.size(); j++) {
        bool rd = false;
        for (const Range& x : an.reads[j]) rd |= overlaps(x, U);
        if (rd) {
            int slot = -1, hits = 0;
            for (int i = 0; i < an.nodes[j].n_inputs; i++)
                if (an.nodes[j].inputs[i] == tr.output) { slot = i; hits++; }
            if (hits != 1 || an.reads[j].size() <= (size_t)slot || an.reads[j][slot].hi - an.reads[j][slot].lo !=
                                                                         U.hi - U.lo)
                return false;
            for (size_t i = 0; i < an.reads[j].size(); i++)
                if ((int)i != slot && overlaps(an.reads[j][i], U)) return false;
            red.push_back({(int)j, slot});
        }
        if (overlaps(an.writes[j], U)) break;
    }
    if (red.empty()) return false;
    pr.out_skip = u;
    pr.out = an.writes[a];
    pr.views.o = static_cast<float*>(an.nodes[a].output);
    pr.views.o_sb = S * H * D;
    pr.views.o_sh = D;
    pr.views.o_ss = H * D;
    pr.redirect = red;
    return true;
}

// The node array as it would execute with the proposals applied: skipped
// nodes neither read nor write; a fused attention reads its view sources.
struct Effective {
    std::vector<std::vector<Range>> reads;
    std::vector<Range> writes;
    std::vector<bool> skipped;
};

Effective effective(const Analysis& an, const std::vector<Proposal>& props) {
    Effective e;
    const size_t n = an.nodes.size();
    e.reads = an.reads;
    e.writes = an.writes;
    e.skipped.assign(n, false);
    for (const Proposal& p : props) {
        for (auto& k : p.skips) e.skipped[k.first] = true;
        if (p.out_skip >= 0) e.skipped[p.out_skip] = true;
    }
    for (const Proposal& p : props) {
        std::vector<Range> r;
        const std::vector<Range>& orig = an.reads[p.a];
        // operands not fused keep their contiguous ranges (orig[0..2] = q, k, v)
        const void* ptrs[3] = {p.views.q, p.views.k, p.views.v};
        const void* origp[3] = {an.nodes[p.a].inputs[0], an.nodes[p.a].inputs[1], an.nodes[p.a].inputs[2]};
        for (int i = 0; i < 3 && i < (int)orig.size(); i++)
            if (ptrs[i] == origp[i]) r.push_back(orig[i]);
        for (size_t i = 3; i < orig.size(); i++) r.push_back(orig[i]);
        for (auto& sr : p.sources) r.push_back(sr.first);
        e.reads[p.a] = r;
        e.writes[p.a] = p.out;
        for (auto& rd : p.redirect) {   // redirected readers see the attention's buffer
            const int j = rd.first, slot = rd.second;
            e.reads[j][slot] = rng(an.nodes[p.a].output, (size_t)(an.reads[j][slot].hi - an.reads[j][slot].lo));
        }
    }
    for (size_t j = 0; j < n; j++)
        if (e.skipped[j]) {
            e.reads[j].clear();
            e.writes[j] = Range{};
        }
    return e;
}

bool eff_reads(const Effective& e, int j, Range r) {
    for (const Range& x : e.reads[j])
        if (overlaps(x, r)) return true;
    return false;
}

// A folded node's output is dead: in the original schedule nobody but its
// fused consumer reads it before the memory is rewritten, and if it is never
// rewritten it is not a graph output (rt_protect ranges, the last node's output).
bool dead_output(const Analysis& an, int k, int consumer, const std::vector<Range>& protect) {
    const Range r = an.writes[k];
    for (size_t j = k + 1; j < an.nodes.size(); j++) {
        bool rd = false;
        for (const Range& x : an.reads[j]) rd |= overlaps(x, r);
        if (rd && (int)j != consumer) {
            if (getenv("RT_FUSE_DEBUG")) fprintf(stderr, "[fusion]   node %d output read by node %zu\n", k, j);
            return false;
        }
        if (overlaps(an.writes[j], r)) return true;   // recycled: the planner only reuses dead memory
    }
    // never rewritten: k would leave the final contents here, which matter
    // if they are a graph output (registered, or the last node's output)
    for (const Range& pr : protect)
        if (overlaps(pr, r)) {
            if (getenv("RT_FUSE_DEBUG")) fprintf(stderr, "[fusion]   node %d output is a graph output\n", k);
            return false;
        }
    return true;
}

static bool dbg() {
    static const bool on = getenv("RT_FUSE_DEBUG") != nullptr;
    return on;
}
#define FAIL(msg)                                                               \
    do {                                                                        \
        if (dbg()) fprintf(stderr, "[fusion] attention %d: %s\n", p.a, msg);   \
        return false;                                                           \
    } while (0)

bool valid(const Analysis& an, const Effective& e, const Proposal& p, const std::vector<Range>& protect) {
    // view sources intact from the start of their chain to the attention.
    // The output may overlap K / V (views or not): a fused attention always
    // runs the tensor-core path, whose pre-passes (V maximum, K/V pack into
    // the plan's workspace) read all of K and V before the attention kernel
    // writes any of O.  Q is read by the attention kernel itself.
    for (size_t i = 0; i < p.sources.size(); i++) {
        const auto& sr = p.sources[i];
        for (int j = sr.second + 1; j < p.a; j++)
            if (overlaps(e.writes[j], sr.first)) FAIL("source overwritten before the attention");
        if (p.source_op[i] == 0 && overlaps(p.out, sr.first)) FAIL("output overlaps the Q source");
    }
    for (auto& k : p.skips)
        if (!dead_output(an, k.first, k.second, protect)) FAIL("a folded node's output is still needed");
    if (p.out_skip >= 0 && !p.redirect.empty()) {
        // the merged result stays in the attention's buffer until its last reader
        const int last = p.redirect.back().first;
        for (int j = p.a + 1; j < last; j++)
            if (overlaps(e.writes[j], p.out)) FAIL("merged output overwritten before its readers");
        // the attention buffer's original reader was the merge only
        if (!dead_output(an, p.a, p.out_skip, protect)) FAIL("attention output still needed");
        // the merge's output: read only by the redirected nodes, never a graph output
        const Range U = an.writes[p.out_skip];
        for (size_t j = p.out_skip + 1; j < an.nodes.size(); j++) {
            bool redirected = false;
            for (auto& rd : p.redirect) redirected |= rd.first == (int)j;
            if (!redirected && eff_reads(e, (int)j, U)) FAIL("merge output read elsewhere");
            if (overlaps(an.writes[j], U)) break;
        }
        bool rewritten = false;
        for (size_t j = p.out_skip + 1; j < an.nodes.size(); j++) rewritten |= overlaps(an.writes[j], U);
        if (!rewritten)
            for (const Range& pr : protect)
                if (overlaps(pr, U)) FAIL("merge output is a graph output");
        for (size_t i = 0; i < p.sources.size(); i++)
            if (p.source_op[i] == 0 && overlaps(p.sources[i].first, p.out)) FAIL("output overlaps the Q source");
    } else if (p.out_skip >= 0) {
        // nothing between the attention and the folded merge touches either buffer
        for (int j = p.a + 1; j < p.out_skip; j++)
            if (overlaps(e.writes[j], p.out) || eff_reads(e, j, p.out) || eff_reads(e, j, an.writes[p.a]))
                FAIL("merge buffer touched between attention and merge");
        // nor does the output overlap Q (K and V are consumed by the pre-passes)
        if (overlaps(an.reads[p.a][0], p.out)) FAIL("merge output overlaps Q");
        if (!dead_output(an, p.a, p.out_skip, protect)) FAIL("attention output still needed");
    }
    return true;
}

// Bias fold: a bias-less GEMM whose output [.., N] is consumed only by
// last-dim SLICEs, each followed (first reader, nothing in between) by an
// in-place ADD of a constant bias [len] -- the custom blocks' merged QKV
// projection.  The GEMM adds one merged bias [N] (the slices' biases at their
// column ranges, zero elsewhere; built at plan time in a plan-owned buffer)
// and the ADDs are not launched, which leaves SLICE -> TRANSPOSE chains for
// the layout fusion.  Returns the folded ADDs in `gone`.
void plan_bias_folds(const std::vector<OpNode>& nodes, const std::vector<Range>& protect,
                     std::vector<PlanItem>& items, std::vector<bool>& gone, BiasPlan* bp) {
    Analysis an(nodes);
    const int n = (int)nodes.size();
    for (int g = 0; g < n; g++) {
        const OpNode& gn = nodes[g];
        if (gn.op != RT_OP_MATMUL || !gemm_fusable(gn)) continue;
        GemmProblem gp;
        if (!decode_gemm(gn, &gp).good() || gp.bias || gp.alpha != 1.0f) continue;
        const Range W = an.writes[g];
        const int64_t M = gp.batches * gp.M, N = gp.N;
        std::vector<int> slices;
        bool ok = true;
        for (int j = g + 1; j < n && ok; j++) {
            bool rd = false;
            for (const Range& x : an.reads[j]) rd |= overlaps(x, W);
            if (rd) {
                const OpNode& sl = nodes[j];
                if (sl.op == RT_OP_SLICE && sl.inputs[0] == gn.output && sl.elem_size == 4 && sl.extra[0] == M &&
                    sl.extra[1] == N && sl.extra[4] == 1)
                    slices.push_back(j);
                else
                    ok = false;
            }
            if (overlaps(an.writes[j], W)) break;
        }
        if (!ok || slices.empty()) continue;
        bool recycled = false;
        for (int j = g + 1; j < n; j++) recycled |= overlaps(an.writes[j], W);
        if (!recycled)
            for (const Range& pr : protect) ok &= !overlaps(pr, W);
        std::vector<std::pair<int, int>> adds;          // (ADD node, slice)
        std::vector<std::pair<int64_t, int64_t>> cols;  // column ranges, for disjointness
        for (int sidx : slices) {
            if (!ok) break;
            const OpNode& sl = nodes[sidx];
            const Range O = an.writes[sidx];
            int a = -1;
            for (int j = sidx + 1; j < n; j++) {
                bool rd = false;
                for (const Range& x : an.reads[j]) rd |= overlaps(x, O);
                if (rd) { a = j; break; }
                if (overlaps(an.writes[j], O)) break;
            }
            if (a < 0) { ok = false; break; }
            const OpNode& ad = nodes[a];
            const int64_t len = sl.extra[3];
            if (ad.op != RT_OP_ADD || ad.extra[0] != 0 || ad.inputs[0] != sl.output || ad.output != sl.output ||
                ad.elem_size != 4 || last_dim(ad) != len || !is_constant_range(ad.inputs[1], (size_t)len * 4)) {
                ok = false;
                break;
            }
            for (auto& c : cols)
                if (sl.extra[2] < c.second && c.first < sl.extra[2] + len) ok = false;
            cols.push_back({sl.extra[2], sl.extra[2] + len});
            adds.push_back({a, sidx});
        }
        if (!ok) continue;
        const int64_t off = (int64_t)bp->bytes;
        bp->bytes += ((size_t)N * 4 + 255) & ~(size_t)255;
        bp->zero.push_back({off, N * 4});
        for (auto& ap : adds) {
            const OpNode& sl = nodes[ap.second];
            bp->copies.push_back({off + sl.extra[2] * 4, nodes[ap.first].inputs[1], sl.extra[3] * 4});
            items[ap.first].skip = true;
            gone[ap.first] = true;
        }
        items[g].epi_bias_off = off;
        if (dbg()) fprintf(stderr, "[fusion] gemm %d: %zu slice biases folded into the epilogue\n", g, adds.size());
    }
}


// Rotary fold: the exporter's per-head RMSNorm + rotary embedding (Qwen3),
//   Y -(SLICE)-> [B,S,H*D] -> RMSNORM(w, rows of D) -> TRANSPOSE -> X [B,H,S,D]
//   m1 = MUL(X, cos[1,1,S,D]);  x1 = SLICE(X, 0, D/2);  x2 = SLICE(X, D/2, D/2)
//   n2 = NEG(x2);  c = CAT(n2, x1);  m2 = MUL(c, sin);  out = ADD(m1, m2)
// runs as one kernel at the ADD (norm_rope_kernel).  Conditions: the chain
// is exactly this; every intermediate output is read by chain members only
// (and is not a graph output); Y, w, cos and sin are not written between the
// chain's first node and the ADD; the ADD's output does not overlap them.
struct RopeMatch {
    int add = -1;
    std::vector<int> chain;        // every node of the chain but the ADD
    RopeFold rp{};
    std::vector<Range> reads;      // what the fused kernel reads
    int first = -1;
};

int writer_of(const Analysis& an, const void* p, size_t bytes, int before) {
    return an.last_writer(rng(p, bytes), before);
}

bool rope_chain(const Analysis& an, int a, RopeMatch& m) {
    const std::vector<OpNode>& N = an.nodes;
    const OpNode& ad = N[a];
    if (ad.op != RT_OP_ADD || ad.extra[0] != 1 || ad.n_dims != 4 || ad.elem_size != 4) return false;
    const int64_t B = ad.out_shape[0], H = ad.out_shape[1], S = ad.out_shape[2], D = ad.out_shape[3];
    if (D != 64 && D != 128) return false;
    const size_t bytes = (size_t)(B * H * S * D) * 4, half = bytes / 2;
    // the two MULs, in either input order
    int w0 = writer_of(an, ad.inputs[0], bytes, a), w1 = writer_of(an, ad.inputs[1], bytes, a);
    if (w0 < 0 || w1 < 0) return false;
    auto is_bmul = [&](int k) {
        const OpNode& x = N[k];
        return x.op == RT_OP_MUL && x.extra[0] == 2 && x.extra[1] == 4 && x.n_dims == 4 &&
               x.out_shape[0] == B && x.out_shape[1] == H && x.out_shape[2] == S && x.out_shape[3] == D &&
               x.extra[2] == H * S * D && x.extra[3] == S * D && x.extra[4] == D && x.extra[5] == 1 &&
               x.extra[6] == 0 && x.extra[7] == 0 && x.extra[9] == 1 && x.extra[8] > 0;
    };
    if (!is_bmul(w0) || !is_bmul(w1)) return false;
    // m2 is the MUL whose first input comes from the CAT
    int m1 = w0, m2 = w1;
    int cat = writer_of(an, N[m2].inputs[0], bytes, m2);
    if (cat < 0 || N[cat].op != RT_OP_CAT) {
        std::swap(m1, m2);
        cat = writer_of(an, N[m2].inputs[0], bytes, m2);
        if (cat < 0 || N[cat].op != RT_OP_CAT) return false;
    }
    if (N[m1].output != ad.inputs[0] && N[m1].output != ad.inputs[1]) return false;
    const OpNode& ct = N[cat];
    if (ct.n_inputs != 2 || ct.extra[0] != 3 || ct.extra[1] != D / 2 || ct.extra[2] != D / 2 || ct.n_dims != 4 ||
        ct.output != N[m2].inputs[0])
        return false;
    const int neg = writer_of(an, ct.inputs[0], half, cat);
    if (neg < 0 || N[neg].op != RT_OP_NEG || N[neg].output != ct.inputs[0]) return false;
    const int x2 = writer_of(an, N[neg].inputs[0], half, neg);
    const int x1 = writer_of(an, ct.inputs[1], half, cat);
    auto is_half_slice = [&](int k, int start, const void* out) {
        if (k < 0) return false;
        const OpNode& x = N[k];
        return x.op == RT_OP_SLICE && x.elem_size == 4 && x.output == out && x.extra[0] == B * H * S &&
               x.extra[1] == D && x.extra[2] == start && x.extra[3] == D / 2 && x.extra[4] == 1;
    };
    if (!is_half_slice(x2, (int)(D / 2), N[neg].inputs[0]) || !is_half_slice(x1, 0, ct.inputs[1])) return false;
    const void* X = N[m1].inputs[0];
    if (N[x1].inputs[0] != X || N[x2].inputs[0] != X) return false;
    const int tr = writer_of(an, X, bytes, std::min(m1, std::min(x1, x2)));
    if (tr < 0) return false;
    const OpNode& t = N[tr];
    if (t.op != RT_OP_TRANSPOSE || t.output != X || t.n_dims != 4 || t.extra[0] != B || t.extra[1] != S ||
        t.extra[2] != 1 || t.extra[3] != H || t.extra[4] != D)
        return false;
    const int rn = writer_of(an, t.inputs[0], bytes, tr);
    if (rn < 0) return false;
    const OpNode& r = N[rn];
    if (r.op != RT_OP_RMSNORM || r.output != t.inputs[0] || last_dim(r) != D || r.elem_size != 4) return false;
    // Y: the RMSNORM input, or the projection a last-dim SLICE took it from
    const float* y = static_cast<const float*>(r.inputs[0]);
    int64_t y_ss = H * D, y_sb = S * H * D;
    Range ysrc = rng(r.inputs[0], bytes);
    int first = rn;
    std::vector<int> chain = {rn, tr, m1, x1, x2, neg, cat, m2};
    const int sl = writer_of(an, r.inputs[0], bytes, rn);
    if (sl >= 0 && N[sl].op == RT_OP_SLICE && N[sl].output == r.inputs[0] && N[sl].elem_size == 4 &&
        N[sl].extra[0] == B * S && N[sl].extra[3] == H * D && N[sl].extra[4] == 1) {
        const int64_t W = N[sl].extra[1];
        y = static_cast<const float*>(N[sl].inputs[0]) + N[sl].extra[2];
        y_ss = W;
        y_sb = S * W;
        ysrc = rng(N[sl].inputs[0], (size_t)(B * S * W) * 4);
        first = sl;
        chain.push_back(sl);
    }
    if (!aligned_view(y, y_sb, y_ss, D)) return false;
    const int64_t cs_ss = N[m1].extra[8];
    if (N[m2].extra[8] != cs_ss) return false;
    m.add = a;
    m.chain = chain;
    m.first = first;
    m.rp = RopeFold{y, y_sb, y_ss, static_cast<const float*>(r.inputs[1]), extra_float(r, 0),
                    static_cast<const float*>(N[m1].inputs[1]), static_cast<const float*>(N[m2].inputs[1]), cs_ss,
                    static_cast<float*>(ad.output), (int)B, (int)H, (int)S, (int)D};
    const size_t cs_bytes = (size_t)((S - 1) * cs_ss + D) * 4;
    m.reads = {ysrc, rng(r.inputs[1], (size_t)D * 4), rng(N[m1].inputs[1], cs_bytes), rng(N[m2].inputs[1], cs_bytes)};
    return true;
}

bool rope_valid(const Analysis& an, const RopeMatch& m, const std::vector<Range>& protect) {
    std::vector<bool> in_chain(an.nodes.size(), false);
    for (int k : m.chain) in_chain[k] = true;
    in_chain[m.add] = true;
    // No reader outside the chain, and no graph output, may see a value a
    // folded chain node would have written: walking back from each such read
    // over earlier writers of the range, a folded node must not come before
    // a kept writer that covers the range.
    auto covers = [](Range w, Range x) { return w.lo <= x.lo && x.hi <= w.hi; };
    auto sees_folded = [&](Range x, int before) {
        for (int i = before - 1; i >= m.first; i--) {
            if (!overlaps(an.writes[i], x)) continue;
            if (in_chain[i] && i != m.add) return true;
            if (covers(an.writes[i], x)) return false;
        }
        return false;
    };
    for (int j = m.first + 1; j < (int)an.nodes.size(); j++) {
        if (in_chain[j]) continue;
        for (const Range& x : an.reads[j])
            if (sees_folded(x, j)) {
                if (dbg()) fprintf(stderr, "[fusion]   rotary: node %d reads a folded value\n", j);
                return false;
            }
    }
    for (const Range& pr : protect)
        if (sees_folded(pr, (int)an.nodes.size())) {
            if (dbg()) fprintf(stderr, "[fusion]   rotary: a graph output holds a folded value\n");
            return false;
        }
    // sources intact from the chain's start to the ADD; output clear of them
    for (int j = m.first + 1; j < m.add; j++)
        if (!in_chain[j])
            for (const Range& src : m.reads)
                if (overlaps(an.writes[j], src)) {
                    if (dbg()) fprintf(stderr, "[fusion]   rotary: source written by node %d\n", j);
                    return false;
                }
    for (const Range& src : m.reads)
        if (overlaps(an.writes[m.add], src)) {
            if (dbg()) fprintf(stderr, "[fusion]   rotary: output overlaps a source\n");
            return false;
        }
    return true;
}

void plan_rope_folds(const std::vector<OpNode>& nodes, const std::vector<Range>& protect,
                     std::vector<PlanItem>& items, std::vector<bool>& gone,
                     std::vector<std::pair<int, std::vector<Range>>>& reads_of) {
    Analysis an(nodes, &gone, &reads_of);
    for (int a = 0; a < (int)nodes.size(); a++) {
        if (gone[a]) continue;
        RopeMatch m;
        if (!rope_chain(an, a, m)) continue;
        bool clash = false;
        for (int k : m.chain) clash |= gone[k];
        if (clash || !rope_valid(an, m, protect)) {
            if (dbg()) fprintf(stderr, "[fusion] rotary chain ending at %d: not folded\n", a);
            continue;
        }
        for (int k : m.chain) {
            items[k].skip = true;
            gone[k] = true;
        }
        items[a].rope = true;
        items[a].rp = m.rp;
        reads_of.push_back({a, m.reads});
        if (dbg()) fprintf(stderr, "[fusion] rotary chain of %zu nodes folded into node %d\n", m.chain.size() + 1, a);
    }
}


// Gated GEMM fold: MATMUL G = A . W^T (W a constant [2N, K] weight, alpha 1)
// -> SLICE x = G[..., :N] -> SLICE up = G[..., N:] -> GATED_ACT(x, up) (no
// bias).  The GEMM takes W's rows in the gated order (per 256-row tile: 64
// gate rows, their 64 up rows, the next 64 gate rows, their up rows) so that
// each epilogue thread holds matching gate and up columns, applies the
// activation and writes the GATED_ACT's output directly (N columns); the
// slices and the GATED_ACT are not launched.  Conditions: G and the slices'
// outputs are read by nobody else (and are not graph outputs), the GATED_ACT
// output overlaps none of the GEMM's operands but A (which the tensor-core GEMM
// reads only through its split planes, written before it starts), and no node
// between the GEMM
// and the GATED_ACT touches that output (the GEMM now writes it earlier).
// The GATED_ACT arithmetic is the same fp32 function of the same fp32 values.
void plan_gated_gemm_folds(const std::vector<OpNode>& nodes, const std::vector<Range>& protect,
                           std::vector<PlanItem>& items, std::vector<bool>& gone,
                           std::vector<std::pair<int, std::vector<Range>>>& reads_of) {
    static const bool on = [] {
        const char* v = getenv("RT_FUSE_GATED_GEMM");
        const char* bn = getenv("RT_GEMM_BN");
        return !(v && v[0] == '0') && !(bn && atoi(bn) == 128);   // the gated order assumes 256-wide N tiles
    }();
    if (!on) return;
    Analysis an(nodes, &gone);
    const int n = (int)nodes.size();
    for (int g = 0; g < n; g++) {
        const OpNode& ga = nodes[g];
        if (gone[g] || ga.op != RT_OP_GATED_ACT || ga.elem_size != 4 || ga.extra[0] != 0 ||
            (ga.extra[1] != 0 && ga.extra[1] != 1))
            continue;
        const int64_t N = last_dim(ga), rows = N ? total_elements(ga) / N : 0;
        if (N % 128 != 0 || rows == 0) continue;
        const size_t half_bytes = (size_t)(rows * N) * 4;
        const int sx = an.last_writer(rng(ga.inputs[0], half_bytes), g);
        const int su = an.last_writer(rng(ga.inputs[1], half_bytes), g);
        auto why = [&](const char* m) {
            if (dbg()) fprintf(stderr, "[fusion] gated GEMM fold at %d: %s\n", g, m);
        };
        if (sx < 0 || su < 0 || sx == su || gone[sx] || gone[su]) { why("inputs not written by two slices"); continue; }
        const OpNode& X = nodes[sx];
        const OpNode& U = nodes[su];
        auto is_half = [&](const OpNode& s, int64_t start, const void* out) {
            return s.op == RT_OP_SLICE && s.elem_size == 4 && s.output == out && s.extra[0] == rows &&
                   s.extra[1] == 2 * N && s.extra[2] == start && s.extra[3] == N && s.extra[4] == 1;
        };
        if (!is_half(X, 0, ga.inputs[0]) || !is_half(U, N, ga.inputs[1]) || X.inputs[0] != U.inputs[0]) {
            why("not the two halves of one tensor");
            continue;
        }
        const void* G = X.inputs[0];
        const Range GR = rng(G, (size_t)(rows * 2 * N) * 4);
        const int m = an.last_writer(GR, std::min(sx, su));
        if (m < 0 || gone[m]) { why("no producer of the sliced tensor"); continue; }
        const OpNode& gm = nodes[m];
        GemmProblem p;
        if (gm.op != RT_OP_MATMUL || gm.output != G || gm.extra[3] != 0 || !decode_gemm(gm, &p).good() ||
            !p.trans_b || p.batches * p.M != rows || p.N != 2 * N || !gemm_fusable(gm) || items[m].views ||
            items[m].epi_out) {
            why("producer is not a plain MATMUL of the right shape");
            continue;
        }
        // G read only by the two slices (a read of x before node j sees G's
        // contents if, walking back, m writes the overlap before any node
        // covering x does); their outputs only by the GATED_ACT
        auto covers = [](Range w, Range x) { return w.lo <= x.lo && x.hi <= w.hi; };
        auto sees_g = [&](Range x, int before) {
            if (!overlaps(x, GR)) return false;
            for (int i = before - 1; i >= m; i--) {
                if (!overlaps(an.writes[i], x)) continue;
                if (i == m) return true;
                if (covers(an.writes[i], x)) return false;
            }
            return false;
        };
        bool ok = true;
        for (int j = m + 1; j < n && ok; j++) {
            if (j == sx || j == su) continue;
            for (const Range& r : an.reads[j]) ok &= !sees_g(r, j);
            if (!ok) why(("G read by node " + std::to_string(j)).c_str());
        }
        for (const Range& pr : protect) ok &= !sees_g(pr, n);
        if (!ok) { why("G read elsewhere or a graph output"); continue; }
        if (!dead_output(an, sx, g, protect) || !dead_output(an, su, g, protect)) { why("a slice output is read elsewhere"); continue; }
        const Range O = an.writes[g];
        // A may overlap O: the tensor-core GEMM reads A only through its split
        // planes, written by a pre-pass (or a norm's hand-off) before it starts
        for (size_t i = 1; i < an.reads[m].size(); i++) ok &= !overlaps(an.reads[m][i], O);
        for (int j = m + 1; j < g && ok; j++) {
            if (j == sx || j == su || gone[j]) continue;
            ok &= !overlaps(an.writes[j], O);
            for (const Range& r : an.reads[j]) ok &= !overlaps(r, O);
        }
        if (!ok) { why("a buffer is read elsewhere or overlaps"); continue; }
        if (!is_constant_range(p.b, (size_t)(p.N * p.K) * 4)) { why("weight is not a marked constant"); continue; }
        items[m].epi_gate = 1 + ga.extra[1];
        items[m].epi_out = ga.output;
        // The slices vanish from later analyses; the GATED_ACT is not launched
        // but stays in them as the writer of its output (the GEMM now writes
        // it, earlier) that reads nothing, so their dead / recycled reasoning
        // about both regions holds.
        for (int k : {sx, su}) {
            items[k].skip = true;
            gone[k] = true;
        }
        items[g].skip = true;
        reads_of.push_back({g, {}});
        if (dbg()) fprintf(stderr, "[fusion] gemm %d applies GATED_ACT %d in its epilogue (slices %d, %d)\n", m, g, sx, su);
    }
}

// Gated-MLP fold: GATED_ACT whose x and/or up input is a last-dim SLICE of a
// wider tensor (Qwen3: the merged gate/up projection) reads that tensor through
// a row-strided view; the SLICE is not launched.  Conditions as for the
// rotary fold: nobody outside (slice -> GATED_ACT) sees the slice's output, and
// the sliced tensor is not written before the GATED_ACT, whose output does not
// overlap it.
void plan_gated_folds(const std::vector<OpNode>& nodes, const std::vector<Range>& protect,
                      std::vector<PlanItem>& items, std::vector<bool>& gone,
                      std::vector<std::pair<int, std::vector<Range>>>& reads_of) {
    Analysis an(nodes, &gone, &reads_of);
    const int n = (int)nodes.size();
    for (int g = 0; g < n; g++) {
        const OpNode& ga = nodes[g];
        if (gone[g] || items[g].skip || ga.op != RT_OP_GATED_ACT || ga.elem_size != 4) continue;
        const int64_t N = last_dim(ga), rows = N ? total_elements(ga) / N : 0;
        const int slot_x = 0, slot_up = ga.extra[0] ? 2 : 1;
        GatedViews v{static_cast<const float*>(ga.inputs[slot_x]), static_cast<const float*>(ga.inputs[slot_up]), N, N};
        std::vector<int> folded;
        std::vector<Range> reads = an.reads[g];
        for (int slot : {slot_x, slot_up}) {
            const size_t bytes = (size_t)(rows * N) * 4;
            const int sl = an.last_writer(rng(ga.inputs[slot], bytes), g);
            if (sl < 0 || gone[sl]) continue;
            const OpNode& s = nodes[sl];
            if (s.op != RT_OP_SLICE || s.output != ga.inputs[slot] || s.elem_size != 4 || s.extra[0] != rows ||
                s.extra[3] != N || s.extra[4] != 1)
                continue;
            const int64_t W = s.extra[1];
            const float* base = static_cast<const float*>(s.inputs[0]) + s.extra[2];
            const Range src = rng(s.inputs[0], (size_t)(rows * W) * 4);
            // the slice's output: read by this GATED_ACT only (walking back from every other reader)
            bool ok = true;
            const Range out = an.writes[sl];
            auto covers = [](Range w, Range x) { return w.lo <= x.lo && x.hi <= w.hi; };
            auto sees_slice = [&](Range x, int before) {
                for (int i = before - 1; i >= sl; i--) {
                    if (!overlaps(an.writes[i], x)) continue;
                    if (i == sl) return true;
                    if (covers(an.writes[i], x)) return false;
                }
                return false;
            };
            for (int j = sl + 1; j < n && ok; j++) {
                if (j == g) continue;
                for (const Range& x : an.reads[j]) ok &= !(overlaps(x, out) && sees_slice(x, j));
            }
            for (const Range& pr : protect) ok &= !(overlaps(pr, out) && sees_slice(pr, n));
            for (int j = sl + 1; j < g && ok; j++) ok &= !overlaps(an.writes[j], src);
            ok &= !overlaps(an.writes[g], src);
            if (!ok) continue;
            (slot == slot_x ? v.x : v.up) = base;
            (slot == slot_x ? v.x_ld : v.up_ld) = W;
            folded.push_back(sl);
            reads.push_back(src);
        }
        if (folded.empty()) continue;
        for (int sl : folded) {
            items[sl].skip = true;
            gone[sl] = true;
        }
        items[g].gated = true;
        items[g].gv = v;
        reads_of.push_back({g, reads});
        if (dbg()) fprintf(stderr, "[fusion] gated activation %d reads %zu slice(s) through views\n", g, folded.size());
    }
}

// Regions of the plan's carry buffer (split operands handed from a producer
// to the GEMM that reads them): a region is reused once the span of the
// hand-off that last used it (producer .. consumer node) is over.
struct CarryAlloc {
    struct Region { int64_t off, size; int busy_until; };
    std::vector<Region> regions;
    int64_t total = 0;
    int64_t take(int start, int end, int64_t size) {
        for (Region& r : regions)
            if (r.busy_until < start && r.size >= size) {
                r.busy_until = end;
                return r.off;
            }
        regions.push_back({total, size, end});
        total += size;
        return regions.back().off;
    }
};

// GEMM epilogue fusion on the schedule left by layout fusion:
//   GEMM g -> GELU u: g applies the GELU and writes u's output; u is skipped.
//   ... -> GEMM k reading u's output as its A operand: g writes k's split A
//   planes (carry buffer) instead, k skips its split pass (opt-in,
//   RT_FUSE_HANDOFF=1: the plane stores cost the first GEMM more than the
//   second one saves, under every scheme).
// Conditions mirror the layout folds: g's output is read by u alone and is
// not a graph output; nothing between g and u touches u's output, which g
// now writes earlier (and g's own operands do not overlap it); for the
// hand-off, u's output is read by k alone, through A only.  Chains share one
// carry buffer, so their [g, k] spans must not overlap.
void plan_gemm_chains(const Analysis& an, const Effective& e, std::vector<PlanItem>& items,
                      const std::vector<Range>& protect, CarryAlloc& carry_alloc) {
    const int n = (int)an.nodes.size();
    auto is_gemm = [](const OpNode& x) { return x.op == RT_OP_MATMUL || x.op == RT_OP_MATMUL_ADD; };
    auto next_reader = [&](int from, Range r) {
        for (int j = from + 1; j < n; j++) {
            if (e.skipped[j]) continue;
            if (eff_reads(e, j, r)) return j;
            if (overlaps(e.writes[j], r)) return -1;
        }
        return -1;
    };
    for (int g = 0; g < n; g++) {
        const OpNode& gn = an.nodes[g];
        if (e.skipped[g] || items[g].views || !is_gemm(gn) || !gemm_fusable(gn)) continue;
        const Range W = an.writes[g];
        const int u = next_reader(g, W);
        if (u < 0) continue;
        const OpNode& un = an.nodes[u];
        if (un.op != RT_OP_GELU || un.inputs[0] != gn.output || un.elem_size != 4 || items[u].redirect_slot >= 0 ||
            an.writes[u].hi - an.writes[u].lo != W.hi - W.lo)
            continue;
        if (!dead_output(an, g, u, protect)) continue;
        const Range U = an.writes[u];
        bool ok = true;
        for (int j = g + 1; j < u && ok; j++)
            if (!e.skipped[j] && (overlaps(e.writes[j], U) || eff_reads(e, j, U))) ok = false;
        for (const Range& r : e.reads[g])
            if (overlaps(r, U)) ok = false;
        if (!ok) continue;
        items[u].skip = true;
        items[g].epi_act = 1;
        items[g].epi_out = un.output;
        if (dbg()) fprintf(stderr, "[fusion] gemm %d: GELU %d folded into the epilogue\n", g, u);

        // The hand-off (opt-in, RT_FUSE_HANDOFF=1).  Under the fp16 scheme
        // the plane and its per-(row, 128 columns) scales replace the fp32
        // output and the consumer's split pass goes, but the plane epilogue
        // holds up the producer's MMAs (the next tile's accumulator waits on
        // the stores): 1B-8K FFN pair 1282 -> 1307 us, GPT-2 258 -> 305 us.
        const char* hv = getenv("RT_FUSE_HANDOFF");   // read per plan
        const bool f16 = gemm_scheme() == 2;
        if (!(hv && hv[0] == '1')) continue;
        const int k = next_reader(u, U);
        if (k < 0) continue;
        const OpNode& kn = an.nodes[k];
        if (!is_gemm(kn) || kn.inputs[0] != un.output || items[k].redirect_slot >= 0 || !gemm_fusable(kn)) continue;
        GemmProblem gp, kp;
        if (!decode_gemm(gn, &gp).good() || !decode_gemm(kn, &kp).good()) continue;
        if ((uintptr_t)(kp.batches * kp.M * kp.K * 4) != U.hi - U.lo || kp.K != gp.N || kp.K % 4 != 0 ||
            kp.batches * kp.M != gp.batches * gp.M || (f16 && kp.K % 128 != 0))
            continue;
        bool only_a = true;
        for (size_t i = 1; i < e.reads[k].size(); i++) only_a &= !overlaps(e.reads[k][i], U);
        if (!only_a || !dead_output(an, u, k, protect)) continue;
        // fp16: one plane of 4 bytes per element, then a float per 128 columns
        const int64_t plane = (int64_t)(((U.hi - U.lo) + 255) & ~(uintptr_t)255);
        const int64_t second = f16 ? (int64_t)(((uintptr_t)(kp.batches * kp.M * (kp.K / 128) * 4) + 255) & ~(uintptr_t)255)
                                   : plane;
        const int64_t off = carry_alloc.take(g, k, plane + second);
        items[g].carry_off = off;
        items[g].carry_plane_bytes = plane;
        items[k].presplit_off = off;
        items[k].presplit_seg = f16;
        items[k].presplit_plane_bytes = plane;
        if (dbg()) fprintf(stderr, "[fusion] gemm %d: writes the split A operand of gemm %d\n", g, k);
    }
}

// Residual fold: GEMM g -> same-shape ADD u (u = y + x or x + y, y = g's
// output): g adds x in its epilogue and writes u's output; u is skipped.
// Conditions as for the GELU fold -- y read by u alone and not a graph
// output; nothing between g and u reads or writes u's output or writes x;
// g's B and bias do not overlap u's output (A is split before the kernel
// writes) -- and u's output is x itself or clear of it (the epilogue reads
// each x element just before writing it).  Opt-in (RT_FUSE_RESIDUAL=1): the
// epilogue's residual loads (one row per thread, like its stores) double its
// L1 -> L2 requests; measured GPT-2 1.040 -> 1.160 ms, Qwen3 1.884 -> 1.901,
// 7b 8.52 -> 8.66; only the 1B-8K block gains (22.45 -> 22.04 ms at the same
// clock: its K = 2048 / 8192 GEMMs leave the epilogue room).
void plan_residual_folds(const Analysis& an, const Effective& e, std::vector<PlanItem>& items,
                         const std::vector<Range>& protect) {
    const int n = (int)an.nodes.size();
    for (int g = 0; g < n; g++) {
        const OpNode& gn = an.nodes[g];
        PlanItem& gi = items[g];
        if (e.skipped[g] || gi.skip || gi.views || (gn.op != RT_OP_MATMUL && gn.op != RT_OP_MATMUL_ADD) ||
            !gemm_fusable(gn) || gi.epi_act || gi.epi_out || gi.carry_off >= 0 ||
            (gn.op == RT_OP_MATMUL && gn.extra[3] != 0))   // alpha 1 only: the residual joins the raw sum
            continue;
        const Range W = an.writes[g];
        int u = -1;
        for (int j = g + 1; j < n; j++) {
            if (e.skipped[j] || items[j].skip) continue;
            if (eff_reads(e, j, W)) { u = j; break; }
            if (overlaps(e.writes[j], W)) break;
        }
        if (u < 0) continue;
        const OpNode& un = an.nodes[u];
        PlanItem& ui = items[u];
        if (dbg() && un.op == RT_OP_ADD) fprintf(stderr, "[fusion] gemm %d: next reader ADD %d\n", g, u);
        if (un.op != RT_OP_ADD || un.n_inputs != 2 || un.elem_size != 4 || un.extra[0] != 1 || ui.rope ||
            ui.gated || ui.redirect_slot >= 0 || ui.norm_planes_off >= 0)
            continue;
        const int ys = un.inputs[0] == gn.output ? 0 : un.inputs[1] == gn.output ? 1 : -1;
        if (ys < 0 || un.inputs[1 - ys] == gn.output) continue;
        const Range U = an.writes[u];
        if (U.hi - U.lo != W.hi - W.lo || e.reads[u].size() < 2) { if (dbg()) fprintf(stderr, "[fusion]   sizes\n"); continue; }
        const Range X = e.reads[u][1 - ys];
        if (X.hi - X.lo != W.hi - W.lo || (overlaps(X, U) && X.lo != U.lo)) { if (dbg()) fprintf(stderr, "[fusion]   x vs output\n"); continue; }
        if (overlaps(X, W) && X.lo != U.lo) continue;   // x lives where g writes y
        if (!dead_output(an, g, u, protect)) { if (dbg()) fprintf(stderr, "[fusion]   y not dead\n"); continue; }
        bool ok = true;
        for (int j = g + 1; j < u && ok; j++)
            if (!e.skipped[j] && (overlaps(e.writes[j], U) || eff_reads(e, j, U) || overlaps(e.writes[j], X)))
                ok = false;
        // A (slot 0) is consumed by the split pre-pass (or arrives split) before
        // the GEMM kernel writes anything, so only B and the bias must stay clear
        for (size_t i = 1; i < e.reads[g].size(); i++)
            if (overlaps(e.reads[g][i], U)) ok = false;
        if (!ok) { if (dbg()) fprintf(stderr, "[fusion]   touched in between / operand overlap\n"); continue; }
        ui.skip = true;
        gi.epi_out = un.output;
        gi.epi_res = un.inputs[1 - ys];
        if (dbg()) fprintf(stderr, "[fusion] gemm %d: residual ADD %d folded into the epilogue\n", g, u);
    }
}

// Norm -> GEMM hand-off: a LAYERNORM / RMSNORM whose output is read only as
// the A operand of the next GEMM writes that GEMM's split planes (the same
// bits its split pass would produce) into the carry buffer, and the GEMM
// skips its split pass: 8 bytes written per element instead of 4, and the
// pass's 12 bytes and a launch saved.
void plan_norm_handoffs(const Analysis& an, const Effective& e, std::vector<PlanItem>& items,
                        const std::vector<Range>& protect, CarryAlloc& carry_alloc) {
    const int n = (int)an.nodes.size();
    for (int m = 0; m < n; m++) {
        const OpNode& nm = an.nodes[m];
        PlanItem& it = items[m];
        if (e.skipped[m] || it.skip || it.rope || it.gated || it.redirect_slot >= 0 || !norm_planes_supported(nm))
            continue;
        const Range L = an.writes[m];
        int k = -1;
        for (int j = m + 1; j < n; j++) {
            if (e.skipped[j] || items[j].skip) continue;
            if (eff_reads(e, j, L)) { k = j; break; }
            if (overlaps(e.writes[j], L)) break;
        }
        if (k < 0) continue;
        const OpNode& kn = an.nodes[k];
        PlanItem& ki = items[k];
        if ((kn.op != RT_OP_MATMUL && kn.op != RT_OP_MATMUL_ADD) || kn.inputs[0] != nm.output ||
            ki.presplit_off >= 0 || ki.redirect_slot >= 0 || !gemm_fusable(kn))
            continue;
        GemmProblem kp;
        if (!decode_gemm(kn, &kp).good() || (uintptr_t)(kp.batches * kp.M * kp.K * 4) != L.hi - L.lo ||
            kp.K != last_dim(nm))
            continue;
        bool only_a = true;
        for (size_t i = 1; i < e.reads[k].size(); i++) only_a &= !overlaps(e.reads[k][i], L);
        if (!only_a || !dead_output(an, m, k, protect)) continue;
        const int64_t plane = (int64_t)(((L.hi - L.lo) + 255) & ~(uintptr_t)255);
        const int64_t off = carry_alloc.take(m, k, 2 * plane);
        it.norm_planes_off = off;
        it.carry_plane_bytes = plane;
        ki.presplit_off = off;
        ki.presplit_plane_bytes = plane;
        if (dbg()) fprintf(stderr, "[fusion] norm %d: writes the split A operand of gemm %d\n", m, k);
    }
}

// Attention -> GEMM split hand-off: an attention writing the merged
// [B, S, H*D] layout whose output is read only by the next GEMM, as its A
// operand, writes that GEMM's split A planes (carry buffer) from its O store;
// the GEMM skips its split pass.  Conditions as for the norm hand-off, on the
// schedule left by the layout folds (the output is the fused attention's).
// Opt-in (RT_FUSE_ATTN_SPLIT=1): on GPT-2 the plane stores cost the attention
// (+14 us per forward) about what the projection GEMMs save (-22 us), so the
// forward time does not move.
void plan_attn_handoffs(const Analysis& an, const Effective& e, std::vector<PlanItem>& items,
                        const std::vector<Range>& protect, CarryAlloc& carry_alloc) {
    const int n = (int)an.nodes.size();
    for (int a = 0; a < n; a++) {
        PlanItem& it = items[a];
        if (!it.views || e.skipped[a] || it.skip || an.nodes[a].n_dims != 4) continue;
        const AttnViews& v = it.attn;
        const OpNode& na = an.nodes[a];
        const int64_t B = na.out_shape[0], H = na.out_shape[1], S = na.out_shape[2], D = na.out_shape[3];
        const Range L = e.writes[a];
        if (L.hi - L.lo != (uintptr_t)(B * H * S * D * 4) || reinterpret_cast<uintptr_t>(v.o) != L.lo ||
            v.o_sh != D || v.o_ss != H * D || v.o_sb != S * H * D || (H * D) % 16 != 0) {
            if (dbg()) fprintf(stderr, "[fusion] attention %d: output not merged [rows][H*D] (%zu bytes, o %p lo %p, strides %lld %lld %lld)\n", a,
                               (size_t)(L.hi - L.lo), (void*)v.o, (void*)L.lo, (long long)v.o_sb, (long long)v.o_sh, (long long)v.o_ss);
            continue;
        }
        int k = -1;
        for (int j = a + 1; j < n; j++) {
            if (e.skipped[j] || items[j].skip) continue;
            if (eff_reads(e, j, L)) { k = j; break; }
            if (overlaps(e.writes[j], L)) break;
        }
        if (k < 0) continue;
        const OpNode& kn = an.nodes[k];
        PlanItem& ki = items[k];
        if (dbg()) fprintf(stderr, "[fusion] attention %d: first reader %d (op %d)\n", a, k, kn.op);
        if (kn.op != RT_OP_MATMUL && kn.op != RT_OP_MATMUL_ADD) continue;
        const void* a_ptr = ki.redirect_slot == 0 ? ki.redirect_ptr : kn.inputs[0];
        if (reinterpret_cast<uintptr_t>(a_ptr) != L.lo || ki.presplit_off >= 0 || !gemm_fusable(kn)) {
            if (dbg()) fprintf(stderr, "[fusion]   A %p L %p presplit %lld fusable %d\n", a_ptr, (void*)L.lo,
                               (long long)ki.presplit_off, (int)gemm_fusable(kn));
            continue;
        }
        GemmProblem kp;
        if (!decode_gemm(kn, &kp).good() || (uintptr_t)(kp.batches * kp.M * kp.K * 4) != L.hi - L.lo ||
            kp.K != H * D) {
            if (dbg()) fprintf(stderr, "[fusion]   gemm shape does not match\n");
            continue;
        }
        bool only_a = true;
        for (size_t i = 1; i < e.reads[k].size(); i++) only_a &= !overlaps(e.reads[k][i], L);
        if (!only_a) {
            if (dbg()) fprintf(stderr, "[fusion]   read through B / bias too\n");
            continue;
        }
        // dead after k: no other reader before the memory is rewritten, not a graph output
        bool dead = true, rewritten = false;
        for (int j = a + 1; j < n && dead && !rewritten; j++) {
            if (j != k && eff_reads(e, j, L)) {
                dead = false;
                if (dbg()) fprintf(stderr, "[fusion]   read by %d\n", j);
            }
            if (j >= k && overlaps(e.writes[j], L)) rewritten = true;   // k may write its output over L
        }
        if (!rewritten)
            for (const Range& pr : protect) dead &= !overlaps(pr, L);
        if (!dead) {
            if (dbg()) fprintf(stderr, "[fusion]   output read again or a graph output\n");
            continue;
        }
        const int64_t plane = (int64_t)(((L.hi - L.lo) + 255) & ~(uintptr_t)255);
        const int64_t off = carry_alloc.take(a, k, 2 * plane);
        it.attn_planes_off = off;
        it.carry_plane_bytes = plane;
        ki.presplit_off = off;
        ki.presplit_plane_bytes = plane;
        if (dbg()) fprintf(stderr, "[fusion] attention %d: writes the split A operand of gemm %d\n", a, k);
    }
}

bool fusion_enabled() {
    static const bool on = [] {
        const char* e = getenv("RT_FUSE");
        return !(e && e[0] == '0');
    }();
    return on;
}

}  // namespace

std::vector<PlanItem> plan_fusions(const std::vector<OpNode>& nodes,
                                   const std::vector<std::pair<uintptr_t, size_t>>& protected_ranges,
                                   size_t* carry_bytes, BiasPlan* bias_plan) {
    std::vector<PlanItem> items(nodes.size());
    if (carry_bytes) *carry_bytes = 0;
    std::vector<Range> protect;
    for (auto& pr : protected_ranges) protect.push_back(Range{pr.first, pr.first + pr.second});
    // last entry: the final node's output (a graph output unless recycled)
    protect.push_back(nodes.empty() ? Range{} : write_range(nodes.back()));
    std::vector<bool> gone(nodes.size(), false);
    BiasPlan local_bp;
    std::vector<std::pair<int, std::vector<Range>>> reads_of;
    if (fusion_enabled()) {
        plan_bias_folds(nodes, protect, items, gone, bias_plan ? bias_plan : &local_bp);
        plan_gated_gemm_folds(nodes, protect, items, gone, reads_of);   // before the rotary folds: it sees every node
        plan_rope_folds(nodes, protect, items, gone, reads_of);
        plan_gated_folds(nodes, protect, items, gone, reads_of);
    }
    Analysis an(nodes, &gone, &reads_of);
    // candidates per attention node, most ambitious first
    std::vector<std::vector<Proposal>> cands;
    for (size_t a = 0; a < nodes.size(); a++) {
        const OpNode& n = nodes[a];
        if (n.op != RT_OP_ATTENTION || !attention_takes_views(n)) continue;
        AttnViews dv;
        if (!attention_default_views(n, &dv)) continue;
        items[a].views = true;
        items[a].attn = dv;
        if (!fusion_enabled() || n.n_dims != 4) continue;
        const int64_t B = n.out_shape[0], H = n.out_shape[1], S = n.out_shape[2], D = n.out_shape[3];
        const int group = n.extra[4] > 0 ? n.extra[4] : 1;
        Proposal pr;
        pr.a = (int)a;
        pr.views = dv;
        pr.out = an.writes[a];
        match_operand(an, (int)a, 0, B, H, S, D, pr);
        match_operand(an, (int)a, 1, B, H / group, S, D, pr);
        match_operand(an, (int)a, 2, B, H / group, S, D, pr);
        std::vector<Proposal> c;
        Proposal with_out = pr;
        match_output(an, (int)a, B, H, S, D, with_out);
        if (with_out.out_skip >= 0) c.push_back(with_out);
        Proposal inplace = pr;
        if (match_output_inplace(an, (int)a, B, H, S, D, inplace)) c.push_back(inplace);
        if (!pr.skips.empty()) c.push_back(pr);
        if (!c.empty()) cands.push_back(c);
    }
    // choose the first candidate of every node; when one is invalid under the
    // combined effect of all current choices, fall back to its next candidate
    std::vector<size_t> pick(cands.size(), 0);
    for (int iter = 0; iter < 256; iter++) {
        std::vector<Proposal> cur;
        std::vector<size_t> owner;
        for (size_t i = 0; i < cands.size(); i++)
            if (pick[i] < cands[i].size()) {
                cur.push_back(cands[i][pick[i]]);
                owner.push_back(i);
            }
        Effective e = effective(an, cur);
        int bad = -1;
        for (size_t i = 0; i < cur.size() && bad < 0; i++)
            if (!valid(an, e, cur[i], protect)) bad = (int)i;
        if (bad < 0) {
            for (const Proposal& p : cur) {
                items[p.a].attn = p.views;
                for (auto& k : p.skips) items[k.first].skip = true;
                if (p.out_skip >= 0) items[p.out_skip].skip = true;
                for (auto& rd : p.redirect) {
                    items[rd.first].redirect_slot = rd.second;
                    items[rd.first].redirect_ptr = an.nodes[p.a].output;
                }
            }
            static const bool gemm_chains = [] {
                const char* v = getenv("RT_FUSE_GEMM");
                return !(v && v[0] == '0');
            }();
            CarryAlloc carry_alloc;
            if (fusion_enabled() && gemm_chains) plan_gemm_chains(an, e, items, protect, carry_alloc);
            const char* rv = getenv("RT_FUSE_RESIDUAL");   // read per plan; opt-in (see plan_residual_folds)
            if (fusion_enabled() && gemm_chains && rv && rv[0] == '1') plan_residual_folds(an, e, items, protect);
            static const bool norm_handoff = [] {
                const char* v = getenv("RT_FUSE_NORM_SPLIT");
                return !(v && v[0] == '0');
            }();
            if (fusion_enabled() && norm_handoff) plan_norm_handoffs(an, e, items, protect, carry_alloc);
            const char* av = getenv("RT_FUSE_ATTN_SPLIT");   // read per plan; opt-in (see plan_attn_handoffs)
            const bool attn_handoff = av && av[0] == '1';
            if (fusion_enabled() && attn_handoff && gemm_planes_from_epilogues()) plan_attn_handoffs(an, e, items, protect, carry_alloc);
            if (carry_bytes) *carry_bytes = (size_t)carry_alloc.total;
            break;
        }
        pick[owner[bad]]++;
    }
    return items;
}

}  // namespace rt
