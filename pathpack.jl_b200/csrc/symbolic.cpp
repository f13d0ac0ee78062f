// symbolic.cpp — host-side symbolic analysis: the stand-in for PATHPACK.jl's `ssymbolic`.
//
// In production the symbolic phase stays in Julia (src/CPU/chordal_ssymbolic.jl:26-57 with CliqueTrees.jl's
// ordering and clique tree) and only its output crosses the C ABI (pp_set_structure).  This file produces the
// same kind of output for callers without Julia (the Python host package, the tests and bench.py):
//
//   1. strongly connected components (Kosaraju's two passes), listed sources first so that every arc
//      between components goes from an earlier one to a later one, as the reference's sccs!
//      (src/CPU/utils.jl:18-70) lists them;
//   2. per component (scliquetree, src/CPU/chordal_ssymbolic.jl:59-184): one front for components of one or
//      two vertices, otherwise a fill-reducing ordering of the symmetrised component (nested dissection by
//      breadth-first level structures, minimum degree inside the small pieces; CliqueTrees' default AMF is
//      not available here) and its clique tree of maximal supernodes, fronts in postorder;
//   3. the coupling graph N between components (soffd, src/CPU/chordal_ssymbolic.jl:212-269).
//
// Output layout (0-based, permuted labels), as pp_set_structure takes it after the shift from 1-based:
// Rptr/Sptr/Stgt (residuals and separators), Bptr/Fptr (vertex and front ranges of components),
// Nptr/Ntgt (coupling rows), perm (perm[p] = original vertex at position p).

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "pathpack_b200_internal.h"

namespace {

using i32 = int32_t;
using i64 = int64_t;

struct Graph {  // compressed adjacency
    i32 n = 0;
    std::vector<i64> ptr;
    std::vector<i32> tgt;
};

// ---------------------------------------------------------------- strongly connected components
// Kosaraju's two depth-first passes, iterative (an explicit stack of (vertex, next arc)).  neighbors(v) are
// the rows of column v of A: the in-neighbours of v.  Pass 1 searches along in-arcs and records vertices as
// they finish; pass 2 searches along out-arcs, starting from the unvisited vertex that finished last, and
// each of its search trees is one component.  Pass 2 meets the components sinks first (a sink component's
// search cannot leave it), so reversing its list puts them sources first: every arc between two components
// then goes from an earlier one to a later one, the order the blocked solves need (the property the
// reference's sccs!, src/CPU/utils.jl:18-70, guarantees; any such order gives the same star).
// Returns the component pointers and the vertices listed component by component.
void sccs(const Graph &g, std::vector<i64> &cptr, std::vector<i32> &ctgt) {
    const i32 n = g.n;
    const i64 m = g.ptr[n];
    // out-arcs: the transpose of the in-neighbour lists
    std::vector<i64> optr(n + 1, 0);
    for (i64 p = 0; p < m; p++) optr[(i64)g.tgt[p] + 1]++;
    for (i32 v = 0; v < n; v++) optr[v + 1] += optr[v];
    std::vector<i32> otgt(std::max<i64>(m, 1));
    {
        std::vector<i64> next(optr.begin(), optr.end() - 1);
        for (i32 v = 0; v < n; v++)
            for (i64 p = g.ptr[v]; p < g.ptr[v + 1]; p++) otgt[next[g.tgt[p]]++] = v;
    }
    std::vector<std::pair<i32, i64>> stack;
    stack.reserve(64);
    // pass 1: finishing order of a search along in-arcs
    std::vector<i32> finished;
    finished.reserve(n);
    std::vector<char> seen(n, 0);
    for (i32 s = 0; s < n; s++) {
        if (seen[s]) continue;
        seen[s] = 1;
        stack.push_back({s, g.ptr[s]});
        while (!stack.empty()) {
            const i32 v = stack.back().first;
            const i64 p = stack.back().second;
            if (p < g.ptr[v + 1]) {
                stack.back().second = p + 1;
                const i32 w = g.tgt[p];
                if (!seen[w]) {
                    seen[w] = 1;
                    stack.push_back({w, g.ptr[w]});
                }
            } else {
                finished.push_back(v);
                stack.pop_back();
            }
        }
    }
    // pass 2: search trees along out-arcs, latest finisher first; comp[v] = index of v's tree
    std::vector<i32> comp(n, -1), order;
    order.reserve(n);
    std::vector<i64> tree_start;
    for (i32 t = n - 1; t >= 0; t--) {
        const i32 s = finished[t];
        if (comp[s] >= 0) continue;
        const i32 c = (i32)tree_start.size();
        tree_start.push_back((i64)order.size());
        comp[s] = c;
        order.push_back(s);
        stack.push_back({s, optr[s]});
        while (!stack.empty()) {
            const i32 v = stack.back().first;
            const i64 p = stack.back().second;
            if (p < optr[v + 1]) {
                stack.back().second = p + 1;
                const i32 w = otgt[p];
                if (comp[w] < 0) {
                    comp[w] = c;
                    order.push_back(w);
                    stack.push_back({w, optr[w]});
                }
            } else {
                stack.pop_back();
            }
        }
    }
    tree_start.push_back((i64)order.size());
    // the trees in reverse: sources first
    const i64 nc = (i64)tree_start.size() - 1;
    cptr.assign(nc + 1, 0);
    ctgt.assign(n, 0);
    i64 at = 0;
    for (i64 c = nc - 1; c >= 0; c--) {
        cptr[nc - 1 - c] = at;
        for (i64 q = tree_start[c]; q < tree_start[c + 1]; q++) ctgt[at++] = order[q];
    }
    cptr[nc] = at;
}

// ---------------------------------------------------------------- ordering of one component
// Symmetric adjacency of the component in local labels 0..m-1 (no self loops, no duplicates).
struct Ordering {
    const Graph &g;
    std::vector<i32> stamp, level, queue, inpart;
    i32 tick = 0;
    std::vector<i32> out;  // elimination order (local labels)
    i32 leaf;

    Ordering(const Graph &g_, i32 leaf_) : g(g_), stamp(g_.n, 0), level(g_.n, -1), queue(g_.n), inpart(g_.n, 0), leaf(leaf_) {
        out.reserve(g.n);
    }

    // breadth-first levels of the part marked inpart == tag from root; returns the number reached
    i32 bfs(i32 root, i32 tag, std::vector<i32> &order, i32 &height) {
        ++tick;
        i32 head = 0, tail = 0;
        order.clear();
        queue[tail++] = root;
        stamp[root] = tick;
        level[root] = 0;
        height = 0;
        while (head < tail) {
            const i32 v = queue[head++];
            order.push_back(v);
            height = std::max(height, level[v]);
            for (i64 p = g.ptr[v]; p < g.ptr[v + 1]; p++) {
                const i32 w = g.tgt[p];
                if (inpart[w] == tag && stamp[w] != tick) {
                    stamp[w] = tick;
                    level[w] = level[v] + 1;
                    queue[tail++] = w;
                }
            }
        }
        return tail;
    }

    i32 degree_in(i32 v, i32 tag) const {
        i32 d = 0;
        for (i64 p = g.ptr[v]; p < g.ptr[v + 1]; p++) d += (inpart[g.tgt[p]] == tag);
        return d;
    }

    // greedy minimum degree on a small part by explicit elimination
    void mindeg(const std::vector<i32> &V) {
        const i32 m = (i32)V.size();
        if (m == 0) return;
        std::vector<i32> loc(m);
        std::vector<std::vector<i32>> adj(m);
        // local index through stamp/level scratch
        ++tick;
        for (i32 k = 0; k < m; k++) {
            stamp[V[k]] = tick;
            level[V[k]] = k;
        }
        for (i32 k = 0; k < m; k++) {
            const i32 v = V[k];
            for (i64 p = g.ptr[v]; p < g.ptr[v + 1]; p++) {
                const i32 w = g.tgt[p];
                if (stamp[w] == tick && w != v) adj[k].push_back(level[w]);
            }
            std::sort(adj[k].begin(), adj[k].end());
            adj[k].erase(std::unique(adj[k].begin(), adj[k].end()), adj[k].end());
        }
        std::vector<char> done(m, 0);
        for (i32 step = 0; step < m; step++) {
            i32 best = -1;
            size_t bd = SIZE_MAX;
            for (i32 k = 0; k < m; k++)
                if (!done[k] && adj[k].size() < bd) {
                    bd = adj[k].size();
                    best = k;
                }
            done[best] = 1;
            out.push_back(V[best]);
            const std::vector<i32> nb = adj[best];
            for (i32 a : nb) {
                auto &A = adj[a];
                A.erase(std::remove(A.begin(), A.end(), best), A.end());
                for (i32 b : nb)
                    if (b != a) A.push_back(b);
                std::sort(A.begin(), A.end());
                A.erase(std::unique(A.begin(), A.end()), A.end());
            }
            adj[best].clear();
        }
    }

    // nested dissection of the part V (all marked inpart == tag)
    void nd(std::vector<i32> V, i32 tag, i32 &nexttag) {
        struct Frame {
            std::vector<i32> V;
            i32 tag;
            std::vector<i32> sep;  // appended after both halves are done
            int state;
            std::vector<i32> V2;
            i32 tag2;
        };
        std::vector<Frame> st;
        st.push_back(Frame{std::move(V), tag, {}, 0, {}, 0});
        std::vector<i32> order, order2;
        while (!st.empty()) {
            Frame &F = st.back();
            if (F.state == 0) {
                if ((i32)F.V.size() <= leaf) {
                    mindeg(F.V);
                    st.pop_back();
                    continue;
                }
                // connected pieces of the part
                i32 h = 0;
                i32 reached = bfs(F.V[0], F.tag, order, h);
                if (reached < (i32)F.V.size()) {
                    // split into the reached piece and the rest; order piece by piece
                    const i32 t1 = ++nexttag;
                    const i32 t2 = ++nexttag;
                    std::vector<i32> A(order), B;
                    ++tick;
                    for (i32 v : A) stamp[v] = tick;
                    for (i32 v : F.V)
                        if (stamp[v] != tick) B.push_back(v);
                    for (i32 v : A) inpart[v] = t1;
                    for (i32 v : B) inpart[v] = t2;
                    F.state = 2;  // nothing to append
                    Frame fa{std::move(A), t1, {}, 0, {}, 0};
                    Frame fb{std::move(B), t2, {}, 0, {}, 0};
                    st.push_back(std::move(fb));
                    st.push_back(std::move(fa));
                    continue;
                }
                // pseudo-peripheral root: repeat BFS from a farthest vertex of smallest degree
                i32 root = F.V[0];
                i32 ecc = h;
                for (int it = 0; it < 6; it++) {
                    i32 best = -1, bd = INT32_MAX;
                    for (i32 v : order)
                        if (level[v] == ecc) {
                            const i32 d = degree_in(v, F.tag);
                            if (d < bd) {
                                bd = d;
                                best = v;
                            }
                        }
                    i32 h2 = 0;
                    bfs(best, F.tag, order2, h2);
                    if (h2 <= ecc) break;
                    root = best;
                    ecc = h2;
                    std::swap(order, order2);
                }
                bfs(root, F.tag, order, h);
                if (h < 2) {
                    mindeg(F.V);
                    st.pop_back();
                    continue;
                }
                std::vector<i32> cnt(h + 1, 0);
                for (i32 v : order) cnt[level[v]]++;
                const i32 half = (i32)order.size() / 2;
                i32 k = 1, acc = cnt[0];
                while (k < h - 1 && acc + cnt[k] <= half) acc += cnt[k++];
                // separator: the vertices of level k with a neighbour in level k + 1
                std::vector<i32> A, B, S;
                for (i32 v : order) {
                    const i32 lv = level[v];
                    if (lv < k)
                        A.push_back(v);
                    else if (lv > k)
                        B.push_back(v);
                    else {
                        bool touches = false;
                        for (i64 p = g.ptr[v]; p < g.ptr[v + 1] && !touches; p++) {
                            const i32 w = g.tgt[p];
                            touches = (inpart[w] == F.tag && stamp[w] == tick && level[w] == k + 1);
                        }
                        (touches ? S : A).push_back(v);
                    }
                }
                const i32 t1 = ++nexttag;
                const i32 t2 = ++nexttag;
                for (i32 v : A) inpart[v] = t1;
                for (i32 v : B) inpart[v] = t2;
                for (i32 v : S) inpart[v] = 0;
                F.sep = std::move(S);
                F.state = 1;
                Frame fa{std::move(A), t1, {}, 0, {}, 0};
                Frame fb{std::move(B), t2, {}, 0, {}, 0};
                st.push_back(std::move(fb));
                st.push_back(std::move(fa));
                continue;
            }
            // state 1: both halves are ordered; the separator comes last
            if (F.state == 1)
                for (i32 v : F.sep) out.push_back(v);
            st.pop_back();
        }
    }
};

// ---------------------------------------------------------------- clique tree of one component
// Input: symmetric adjacency (local labels), an elimination order.  Output: postordered fronts of
// maximal supernodes, the final local order (position -> local vertex), res pointers and separators
// in positions.
struct Fronts {
    std::vector<i32> order;       // position -> local vertex
    std::vector<i64> Rptr;        // fronts' residual ranges (positions)
    std::vector<i64> Sptr;        // separator pointers
    std::vector<i32> Stgt;        // separator positions
};

Fronts cliquetree(const Graph &g, const std::vector<i32> &elim) {
    const i32 m = g.n;
    Fronts F;
    std::vector<i32> pos(m);
    for (i32 k = 0; k < m; k++) pos[elim[k]] = k;
    // adjacency in elimination positions
    auto adj_of = [&](i32 p, std::vector<i32> &out) {
        out.clear();
        const i32 v = elim[p];
        for (i64 q = g.ptr[v]; q < g.ptr[v + 1]; q++) out.push_back(pos[g.tgt[q]]);
    };
    // elimination tree (Liu, with path compression)
    std::vector<i32> parent(m, -1), anc(m, -1);
    std::vector<i32> nb;
    for (i32 j = 0; j < m; j++) {
        adj_of(j, nb);
        for (i32 i : nb) {
            if (i >= j) continue;
            i32 r = i;
            while (anc[r] != -1 && anc[r] != j) {
                const i32 t = anc[r];
                anc[r] = j;
                r = t;
            }
            if (anc[r] == -1) {
                anc[r] = j;
                parent[r] = j;
            }
        }
    }
    // postorder (children in increasing order)
    std::vector<i32> head(m, -1), next(m, -1);
    for (i32 j = m - 1; j >= 0; j--)
        if (parent[j] >= 0) {
            next[j] = head[parent[j]];
            head[parent[j]] = j;
        }
    std::vector<i32> post;
    post.reserve(m);
    {
        std::vector<i32> stack;
        std::vector<i32> it(m);
        for (i32 r = 0; r < m; r++) {
            if (parent[r] != -1) continue;
            stack.push_back(r);
            it[r] = head[r];
            while (!stack.empty()) {
                const i32 v = stack.back();
                if (it[v] != -1) {
                    const i32 c = it[v];
                    it[v] = next[c];
                    it[c] = head[c];
                    stack.push_back(c);
                } else {
                    post.push_back(v);
                    stack.pop_back();
                }
            }
        }
    }
    std::vector<i32> ipost(m);
    for (i32 k = 0; k < m; k++) ipost[post[k]] = k;
    // relabel to postorder: final position q holds elimination position post[q]
    F.order.resize(m);
    for (i32 q = 0; q < m; q++) F.order[q] = elim[post[q]];
    std::vector<i32> par(m, -1);
    for (i32 q = 0; q < m; q++) par[q] = parent[post[q]] >= 0 ? ipost[parent[post[q]]] : -1;
    std::vector<i32> fpos(m);
    for (i32 q = 0; q < m; q++) fpos[F.order[q]] = q;
    // column counts from row subtrees
    std::vector<i64> cc(m, 1);
    std::vector<i32> mark(m, -1);
    std::vector<i32> nchild(m, 0);
    for (i32 q = 0; q < m; q++)
        if (par[q] >= 0) nchild[par[q]]++;
    for (i32 i = 0; i < m; i++) {
        mark[i] = i;
        const i32 v = F.order[i];
        for (i64 p = g.ptr[v]; p < g.ptr[v + 1]; p++) {
            i32 j = fpos[g.tgt[p]];
            if (j >= i) continue;
            while (mark[j] != i) {
                mark[j] = i;
                cc[j]++;
                j = par[j];
            }
        }
    }
    // maximal supernodes: q joins q - 1's supernode when q - 1 is a child of q and the column counts nest
    // (q's structure is q - 1's minus q - 1), whatever q's other children
    std::vector<i32> snode_start;
    for (i32 q = 0; q < m; q++) {
        const bool join = q > 0 && par[q - 1] == q && cc[q - 1] == cc[q] + 1;
        if (!join) snode_start.push_back(q);
    }
    const i32 nf = (i32)snode_start.size();
    snode_start.push_back(m);
    std::vector<i32> idx(m);
    for (i32 f = 0; f < nf; f++)
        for (i32 q = snode_start[f]; q < snode_start[f + 1]; q++) idx[q] = f;
    // separators by merging the residual's adjacency and the children's separators
    F.Rptr.assign(nf + 1, 0);
    F.Sptr.assign(nf + 1, 0);
    for (i32 f = 0; f <= nf; f++) F.Rptr[f] = snode_start[f];
    std::vector<std::vector<i32>> sep(nf);
    std::vector<i32> seen(m, -1);
    std::vector<std::vector<i32>> kids(nf);
    for (i32 f = 0; f < nf; f++) {
        const i32 lo = snode_start[f], hi = snode_start[f + 1];
        std::vector<i32> &S = sep[f];
        for (i32 q = lo; q < hi; q++) {
            const i32 v = F.order[q];
            for (i64 p = g.ptr[v]; p < g.ptr[v + 1]; p++) {
                const i32 w = fpos[g.tgt[p]];
                if (w >= hi && seen[w] != f) {
                    seen[w] = f;
                    S.push_back(w);
                }
            }
        }
        for (i32 c : kids[f]) {
            for (i32 w : sep[c])
                if (w >= hi && seen[w] != f) {
                    seen[w] = f;
                    S.push_back(w);
                }
            std::vector<i32>().swap(sep[c]);
        }
        std::sort(S.begin(), S.end());
        F.Sptr[f + 1] = F.Sptr[f] + (i64)S.size();
        F.Stgt.insert(F.Stgt.end(), S.begin(), S.end());
        if (!S.empty()) kids[idx[S[0]]].push_back(f);
    }
    return F;
}

}  // namespace

// ---------------------------------------------------------------- C ABI of the symbolic stand-in

struct pp_symbolic_result {
    i64 n = 0, nf = 0, nB = 0;
    std::vector<i64> Rptr, Sptr, Stgt, Bptr, Fptr, Nptr, Ntgt, perm;
};

extern "C" int32_t pp_symbolic(int64_t n, const int64_t *colptr, const int64_t *rowval, int32_t method,
                               int32_t leaf, pp_symbolic_result **out) {
    if (!out) return PP_EINVAL;
    *out = nullptr;
    if (n < 0 || (n > 0 && (!colptr || (colptr[n] > 0 && !rowval)))) return PP_EINVAL;
    if (n >= (int64_t)INT32_MAX) return PP_EUNSUPPORTED;
    try {
        auto *R = new pp_symbolic_result();
        R->n = n;
        Graph A;
        A.n = (i32)n;
        A.ptr.assign(colptr, colptr + n + 1);
        A.tgt.resize(colptr[n]);
        for (i64 p = 0; p < colptr[n]; p++) {
            if (rowval[p] < 0 || rowval[p] >= n) {
                delete R;
                return PP_EINVAL;
            }
            A.tgt[p] = (i32)rowval[p];
        }
        // 1. components
        std::vector<i64> cptr;
        std::vector<i32> ctgt;
        sccs(A, cptr, ctgt);
        const i64 nB = (i64)cptr.size() - 1;
        std::vector<i32> index(n);
        for (i64 a = 0; a < n; a++) index[ctgt[a]] = (i32)a;
        std::vector<i32> comp(n);
        for (i64 c = 0; c < nB; c++)
            for (i64 a = cptr[c]; a < cptr[c + 1]; a++) comp[a] = (i32)c;
        // grouped graph: neighbours of grouped vertex a are the grouped labels of the rows of column ctgt[a]
        R->nB = nB;
        R->Bptr.assign(cptr.begin(), cptr.end());
        R->Fptr.assign(nB + 1, 0);
        R->Rptr.push_back(0);
        R->Sptr.push_back(0);
        std::vector<i32> Rtgt(n);  // position -> grouped label
        for (i64 c = 0; c < nB; c++) {
            const i64 vstrt = cptr[c], vstop = cptr[c + 1], m = vstop - vstrt;
            if (m <= 2) {
                for (i64 a = vstrt; a < vstop; a++) Rtgt[a] = (i32)a;
                R->Rptr.push_back(vstop);
                R->Sptr.push_back(R->Sptr.back());
                R->Fptr[c + 1] = (i64)R->Rptr.size() - 1;
                continue;
            }
            // symmetrised subgraph of the component, local labels
            std::vector<std::vector<i32>> adj(m);
            for (i64 a = vstrt; a < vstop; a++) {
                const i32 v = ctgt[a];
                for (i64 p = A.ptr[v]; p < A.ptr[v + 1]; p++) {
                    const i64 b = index[A.tgt[p]];
                    if (b >= vstrt && b < vstop && b != a) {
                        adj[a - vstrt].push_back((i32)(b - vstrt));
                        adj[b - vstrt].push_back((i32)(a - vstrt));
                    }
                }
            }
            Graph G;
            G.n = (i32)m;
            G.ptr.assign(m + 1, 0);
            for (i64 k = 0; k < m; k++) {
                auto &v = adj[k];
                std::sort(v.begin(), v.end());
                v.erase(std::unique(v.begin(), v.end()), v.end());
                G.ptr[k + 1] = G.ptr[k] + (i64)v.size();
            }
            G.tgt.reserve(G.ptr[m]);
            for (i64 k = 0; k < m; k++) G.tgt.insert(G.tgt.end(), adj[k].begin(), adj[k].end());
            std::vector<std::vector<i32>>().swap(adj);
            std::vector<i32> elim;
            if (method == 1) {  // natural order
                elim.resize(m);
                for (i64 k = 0; k < m; k++) elim[k] = (i32)k;
            } else {
                Ordering O(G, leaf > 0 ? leaf : 64);
                std::vector<i32> V(m);
                for (i64 k = 0; k < m; k++) V[k] = (i32)k;
                for (i64 k = 0; k < m; k++) O.inpart[k] = 1;
                i32 nexttag = 1;
                O.nd(std::move(V), 1, nexttag);
                elim.swap(O.out);
            }
            Fronts F = cliquetree(G, elim);
            const i64 nf0 = (i64)R->Rptr.size() - 1;
            const i64 sbase = R->Sptr.back();
            for (size_t f = 1; f < F.Rptr.size(); f++) {
                R->Rptr.push_back(vstrt + F.Rptr[f]);
                R->Sptr.push_back(sbase + F.Sptr[f]);
            }
            for (i32 s : F.Stgt) R->Stgt.push_back(vstrt + s);
            for (i64 q = 0; q < m; q++) Rtgt[vstrt + q] = (i32)(vstrt + F.order[q]);
            (void)nf0;
            R->Fptr[c + 1] = (i64)R->Rptr.size() - 1;
        }
        R->nf = (i64)R->Rptr.size() - 1;
        // final permutation: position -> original vertex
        R->perm.resize(n);
        std::vector<i32> ipos(n);  // grouped label -> position
        for (i64 a = 0; a < n; a++) {
            R->perm[a] = ctgt[Rtgt[a]];
            ipos[Rtgt[a]] = (i32)a;
        }
        // 3. coupling N (soffd): for position j, the positions of in-neighbours in earlier components
        R->Nptr.assign(n + 1, 0);
        std::vector<i64> rows;
        for (i64 j = 0; j < n; j++) {
            const i64 jstrt = cptr[comp[Rtgt[j]]];
            const i32 v = ctgt[Rtgt[j]];
            rows.clear();
            for (i64 p = A.ptr[v]; p < A.ptr[v + 1]; p++) {
                const i64 b = index[A.tgt[p]];
                if (b < jstrt) rows.push_back(ipos[b]);
            }
            std::sort(rows.begin(), rows.end());
            rows.erase(std::unique(rows.begin(), rows.end()), rows.end());
            R->Nptr[j + 1] = R->Nptr[j] + (i64)rows.size();
            R->Ntgt.insert(R->Ntgt.end(), rows.begin(), rows.end());
        }
        *out = R;
        return PP_OK;
    } catch (const std::bad_alloc &) {
        return PP_ENOMEM;
    } catch (...) {
        return PP_EINVAL;
    }
}

extern "C" void pp_symbolic_sizes(const pp_symbolic_result *R, int64_t *sizes) {
    // n, nf, nB, |Stgt|, |Ntgt|
    sizes[0] = R->n;
    sizes[1] = R->nf;
    sizes[2] = R->nB;
    sizes[3] = (int64_t)R->Stgt.size();
    sizes[4] = (int64_t)R->Ntgt.size();
}

extern "C" void pp_symbolic_get(const pp_symbolic_result *R, int64_t *Rptr, int64_t *Sptr, int64_t *Stgt,
                                int64_t *Bptr, int64_t *Fptr, int64_t *Nptr, int64_t *Ntgt, int64_t *perm) {
    auto cp = [](const std::vector<i64> &v, int64_t *o) {
        if (o && !v.empty()) std::memcpy(o, v.data(), sizeof(int64_t) * v.size());
    };
    cp(R->Rptr, Rptr);
    cp(R->Sptr, Sptr);
    cp(R->Stgt, Stgt);
    cp(R->Bptr, Bptr);
    cp(R->Fptr, Fptr);
    cp(R->Nptr, Nptr);
    cp(R->Ntgt, Ntgt);
    cp(R->perm, perm);
}

extern "C" void pp_symbolic_free(pp_symbolic_result *R) { delete R; }
