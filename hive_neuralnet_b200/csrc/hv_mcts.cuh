// hv_mcts.cuh -- MCTS tree kernels (select / replay / expand / backup /
// policy / root noise) on the reference's SoA tree layout
// (hive_gpu/csrc/mcts_tree.cuh:31-45, tensors [B, max_nodes]).
//
// One warp owns one game and walks that game's simulations in simulation
// index order (sim = j * B + game).  Child scoring at each tree level is
// warp-parallel (lanes stride the children, then a (score, index) argmax
// reduction that keeps the reference's first-maximum rule); every tree
// update is done by one lane, so no atomics are needed and the result is
// deterministic: it equals the reference kernels executed one simulation at
// a time in index order.  (The reference launches one thread per simulation
// with atomic virtual loss, so several simulations of one game race.)
// Scores use explicit round-to-nearest intrinsics so that no fused
// multiply-add changes a comparison.
#pragma once

#include "hv_core.cuh"

namespace hv {

constexpr int kTreeDepth = 128;
constexpr int kTreeThreads = 256;  // block of the per-game tree kernels (8 warps)

struct TreeDev {
    int32_t* vc;
    float* tv;
    float* pr;
    int32_t* pa;
    float* vq;
    uint8_t* mb;
    int32_t* ai;
    int32_t* fc;
    int32_t* nc;
    int8_t* it;
    float* tval;
    int32_t* cnt;
    int32_t max_nodes;
};

__device__ __forceinline__ int64_t tix(const TreeDev& t, int g, int n) {
    return (int64_t)g * t.max_nodes + n;
}

// PUCT score (mcts_tree.cuh:55-67), evaluated in the reference's order
__device__ __forceinline__ float puct(const TreeDev& t, int g, int parent_visits, int child, float c) {
    int64_t ci = tix(t, g, child);
    int n = t.vc[ci];
    float q = n > 0 ? __fdiv_rn(-t.tv[ci], (float)n) : 0.0f;
    q = __fsub_rn(q, t.vq[ci]);
    float u = __fmul_rn(c, t.pr[ci]);
    u = __fmul_rn(u, __fsqrt_rn((float)parent_visits));
    u = __fdiv_rn(u, __fadd_rn(1.0f, (float)n));
    return __fadd_rn(q, u);
}

// (score, index) argmax over lanes: higher score wins, lower index on ties;
// idx < 0 marks "no candidate"
__device__ __forceinline__ void warp_argmax(float& s, int& idx) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float s2 = __shfl_xor_sync(kFull, s, o);
        int i2 = __shfl_xor_sync(kFull, idx, o);
        bool take = i2 >= 0 && (idx < 0 || s2 > s || (s2 == s && i2 < idx));
        if (take) {
            s = s2;
            idx = i2;
        }
    }
}

// Gumbel completed-Q child below the root (mcts_tree.cuh:77-143); one lane,
// children in order (its sums are order dependent)
__device__ __noinline__ int completed_q_child(const TreeDev& t, int g, int first, int n, float sigma,
                                              const float* init_q) {
    float sumv = 0.0f, mx = -1e30f, se = 0.0f;
    for (int c = 0; c < n; c++) {
        if (first + c < 0 || first + c >= t.max_nodes) break;
        sumv = __fadd_rn(sumv, (float)t.vc[tix(t, g, first + c)]);
    }
    for (int pass = 0; pass < 2; pass++) {
        for (int c = 0; c < n; c++) {
            if (first + c < 0 || first + c >= t.max_nodes) break;
            int64_t ci = tix(t, g, first + c);
            float v = (float)t.vc[ci];
            float q = v > 0.0f ? __fdiv_rn(-t.tv[ci], v) : init_q[ci];
            q = __fsub_rn(q, t.vq[ci]);
            float lq = __fadd_rn(logf(fmaxf(t.pr[ci], 1e-20f)), __fmul_rn(sigma, q));
            if (pass == 0) {
                if (lq > mx) mx = lq;
            } else {
                se = __fadd_rn(se, expf(__fsub_rn(lq, mx)));
            }
        }
    }
    se = fmaxf(se, 1e-20f);
    int best = -1;
    float bs = -1e30f, den = __fadd_rn(1.0f, sumv);
    for (int c = 0; c < n; c++) {
        if (first + c < 0 || first + c >= t.max_nodes) break;
        int64_t ci = tix(t, g, first + c);
        float v = (float)t.vc[ci];
        float q = v > 0.0f ? __fdiv_rn(-t.tv[ci], v) : init_q[ci];
        q = __fsub_rn(q, t.vq[ci]);
        float lq = __fadd_rn(logf(fmaxf(t.pr[ci], 1e-20f)), __fmul_rn(sigma, q));
        float pi0 = __fdiv_rn(expf(__fsub_rn(lq, mx)), se);
        float s = __fsub_rn(pi0, __fdiv_rn(v, den));
        if (s > bs) {
            bs = s;
            best = first + c;
        }
    }
    return best;
}

struct SelectArgs {
    int mode;  // 0 plain PUCT, 1 root alive-mask, 2 root slots
    const float* init_q;
    const int8_t* active;
    const int32_t* roots;
    const int8_t* alive;
    const int32_t* slots;
    int C;
    int max_root_children;
    float c_puct;
    int B;
    int total;
    int det;
    float sigma;
    float qpen;
    int32_t* leaf;
    uint8_t* paths;
    int32_t* plen;
    int32_t* vlp;
    int32_t* vll;
};

// one recorded step: virtual loss (or penalty) and path entries, lane 0 only
__device__ __forceinline__ void sel_step(const TreeDev& t, const SelectArgs& a, int g, int s, int node,
                                         bool vl, bool det_step, int& plen, int& vlen) {
    int64_t ni = tix(t, g, node);
    if (vl) {
        t.vc[ni] += 1;
        if (det_step) t.vq[ni] = __fadd_rn(t.vq[ni], a.qpen);
        else t.tv[ni] = __fadd_rn(t.tv[ni], -1.0f);
        if (vlen < kTreeDepth) a.vlp[(int64_t)s * kTreeDepth + vlen++] = node;
    }
    if (plen < kTreeDepth) {
        uint8_t* dst = a.paths + ((int64_t)s * kTreeDepth + plen) * 6;
        const uint8_t* src = t.mb + ni * 6;
#pragma unroll
        for (int b = 0; b < 6; b++) dst[b] = src[b];
        plen++;
    }
}

// One selection step at `node`: the chosen child, or -1 where the walk
// stops (an unexpanded or terminal node, no candidate).  pv_at < 0: the
// node's visit count from the tree, else that count (the parent visits the
// scores use).  det_step: the step used the completed-Q rule.
__device__ __forceinline__ int select_child(const TreeDev& t, const SelectArgs& a, int g, int node, int root,
                                            int pv_at, bool& det_step) {
    const int l = lane_id();
    const int64_t ni = tix(t, g, node);
    const int fc = t.fc[ni], nc = t.nc[ni];
    det_step = false;
    if (fc < 0 || t.it[ni] || nc == 0 || nc <= 0 || nc > 1024) return -1;
    const bool at_root = a.mode != 2 && node == root;
    const bool use_det = a.det && a.mode != 0 && !at_root;
    det_step = use_det;
    int best;
    if (use_det) {
        best = 0;
        if (l == 0) best = completed_q_child(t, g, fc, nc, a.sigma, a.init_q);
        best = __shfl_sync(kFull, best, 0);
    } else {
        const int pv = pv_at >= 0 ? pv_at : t.vc[ni];
        int lim = nc;
        if (fc + lim > t.max_nodes) lim = t.max_nodes - fc;  // reference breaks there
        float bs = 0.0f;
        int bi = -1;
        for (int c = l; c < lim; c += 32) {
            if (a.mode == 1 && at_root &&
                (c >= a.max_root_children || !a.alive[(int64_t)g * a.max_root_children + c]))
                continue;
            float sc = puct(t, g, pv, fc + c, a.c_puct);
            if (!(sc > -1e30f)) continue;  // strict > from -1e30: NaN never wins
            if (bi < 0 || sc > bs) {
                bs = sc;
                bi = c;
            }
        }
        warp_argmax(bs, bi);
        best = bi >= 0 ? fc + bi : (a.mode == 0 ? fc : -1);
    }
    return best;
}

// the walk of simulation s below `node` (steps it0 .., path entries so far)
__device__ __forceinline__ void select_descend(const TreeDev& t, const SelectArgs& a, int g, int s, int node,
                                               int root, int it0, int plen, int vlen, int pv_first) {
    const int l = lane_id();
    for (int it = it0; it < kTreeDepth; it++) {
        bool det_step;
        const int best = select_child(t, a, g, node, root, it == it0 ? pv_first : -1, det_step);
        if (best < 0) break;
        node = best;
        if (l == 0) sel_step(t, a, g, s, node, true, det_step, plen, vlen);
        __syncwarp();
    }
    if (l == 0) {
        a.leaf[s] = node;
        a.plen[s] = plen;
        a.vll[s] = vlen;
    }
    __syncwarp();
}

// one simulation s of game g (the warp's lanes score children in parallel)
__device__ __forceinline__ void select_sim(const TreeDev& t, const SelectArgs& a, int g, int s) {
    const int l = lane_id();
    int node = -1, plen = 0, vlen = 0;
    bool ok = a.active[g] != 0;
    const int root = a.roots[g];
    int iter0 = 0;
    if (ok) node = root;
    if (ok && a.mode == 2) {
        int slot = a.slots[(int64_t)g * a.C + (s / a.B) % a.C];
        int64_t ri = tix(t, g, root);
        int fc = t.fc[ri], nc = t.nc[ri];
        ok = slot >= 0 && slot < a.max_root_children && fc >= 0 && !t.it[ri] && nc > 0 && slot < nc &&
             fc + slot >= 0 && fc + slot < t.max_nodes;
        if (ok) {
            node = fc + slot;
            if (l == 0) sel_step(t, a, g, s, node, !a.det, false, plen, vlen);
            iter0 = 1;
        }
    }
    __syncwarp();
    if (!ok) {
        if (l == 0) {
            a.leaf[s] = -1;
            a.plen[s] = plen;
            a.vll[s] = vlen;
        }
        __syncwarp();
        return;
    }
    plen = __shfl_sync(kFull, plen, 0);
    vlen = __shfl_sync(kFull, vlen, 0);
    select_descend(t, a, g, s, node, root, iter0, plen, vlen, -1);
}

// Plain and root-mask selects (modes 0, 1), one block per game: warp 0 takes
// every simulation's root step in simulation order (each scoring the root's
// children with the earlier simulations' virtual losses on them) and records
// the chosen child and that child's visit count after the simulation's own
// virtual loss -- the parent visits its first step below the child sees in
// the sequential order; then each simulation descends below its root child,
// the simulations of one child in order in one warp (warp = child mod the
// block's warps).  Below the root, simulations of different children read
// and write disjoint subtrees, so every one sees the tree of the sequential
// order.  rc / pvc: shared, two words per simulation of the game.
__device__ void select_game_tree(const TreeDev& t, const SelectArgs& a, int g, int32_t* rc, int32_t* pvc) {
    const int l = lane_id(), w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int per = a.total / a.B;
    const int root = a.roots[g];
    const bool active = a.active[g] != 0;
    if (w == 0) {
        for (int k = 0; k < per; k++) {
            const int s = g + k * a.B;
            int c = -1;
            if (active) {
                bool det_step;
                c = select_child(t, a, g, root, root, -1, det_step);
                if (c >= 0 && l == 0) {
                    int plen = 0, vlen = 0;
                    sel_step(t, a, g, s, c, true, det_step, plen, vlen);
                    pvc[k] = t.vc[tix(t, g, c)];
                }
            }
            if (l == 0) {
                rc[k] = c;
                if (c < 0) {
                    a.leaf[s] = active ? root : -1;
                    a.plen[s] = 0;
                    a.vll[s] = 0;
                }
            }
            __syncwarp();
        }
    }
    __syncthreads();
    for (int k = 0; k < per; k++) {
        const int c = rc[k];
        if (c < 0 || c % nw != w) continue;
        select_descend(t, a, g, g + k * a.B, c, root, 1, 1, 1, pvc[k]);
    }
}

// the simulations of game g in order (s = g, g + B, ...)
__device__ __noinline__ void select_game(const TreeDev& t, const SelectArgs& a, int g) {
    for (int s = g; s < a.total; s += a.B) select_sim(t, a, g, s);
}

// Root-slot mode: the simulations of candidate j of game g (s = g + k B with
// k = j, j + C, j + 2C, ...), in order.  Each descends below a distinct root
// child, so the virtual losses and statistics it reads and writes belong to
// that child's subtree alone: candidates of one game can run in separate
// warps and every simulation sees the tree it sees in the sequential order
// (the reference's).  A game whose candidate table repeats a slot runs all of
// its simulations in order in the warp of candidate 0.  C <= 32.
__device__ __noinline__ void select_game_slot(const TreeDev& t, const SelectArgs& a, int g, int j) {
    const int l = lane_id();
    const int sl = l < a.C ? a.slots[(int64_t)g * a.C + l] : -1;
    const bool v = l < a.C && sl >= 0;
    const uint32_t same = __match_any_sync(kFull, v ? sl : -1 - l);  // unset / unused lanes: keys of their own
    if (__any_sync(kFull, v && __popc(same) > 1)) {
        if (j == 0) select_game(t, a, g);
        return;
    }
    const int per_game = a.total / a.B;
    for (int k = j; k < per_game; k += a.C) select_sim(t, a, g, g + k * a.B);
}

// terminal value from the leaf player's perspective (mcts_tree.cuh:182-188)
__device__ __forceinline__ float result_value(int result, int turn) {
    if (result == 3) return 0.0f;
    bool white = (turn & 1) == 0;
    if (result == 1) return white ? 1.0f : -1.0f;
    if (result == 2) return white ? -1.0f : 1.0f;
    return 0.0f;
}

struct ExpandArgs {
    int dense;
    int backprop;
    float* init_q;
    const float* child_q;
    const int32_t* leaf;
    const uint8_t* leaf_states;
    const uint8_t* legal;
    const int32_t* num_legal;
    const float* priors;  // dense [T,256] or action-space [T,85834]
    const int32_t* results;
    const float* values;
    const int32_t* vlp;
    const int32_t* vll;
    int8_t* was;
    float qpen;
    int B;
    int total;
};

// round-half-to-even of sum / n (state_encoder.cuh:55-79)
__device__ __forceinline__ int rhe_div(int sum, int n) {
    int q = sum / n, r = sum - q * n;
    int twice = 2 * (r < 0 ? -r : r);
    if (twice < n) return q;
    int away = sum > 0 ? q + 1 : q - 1;
    if (twice > n) return away;
    return (q & 1) == 0 ? q : away;
}

// move -> action index around the centroid (mcts_tree.cuh:146-179)
__device__ __forceinline__ int move_action(const uint8_t* x, int cq, int cr) {
    int type = x[0], pt = x[1], from = x[2] | (x[3] << 8), to = x[4] | (x[5] << 8);
    if (type == 2) return 85833;
    if (type == 0) {
        int ec = (to % kBoard - 11) - cq + 8, er = (to / kBoard - 11) - cr + 8;
        if (ec < 0 || ec >= 17 || er < 0 || er >= 17) return -1;
        return (pt - 1) * 289 + er * 17 + ec;
    }
    int sc = (from % kBoard - 11) - cq + 8, sr = (from / kBoard - 11) - cr + 8;
    int dc = (to % kBoard - 11) - cq + 8, dr = (to / kBoard - 11) - cr + 8;
    if (sc < 0 || sc >= 17 || sr < 0 || sr >= 17 || dc < 0 || dc >= 17 || dr < 0 || dr >= 17) return -1;
    return 2312 + (sr * 17 + sc) * 289 + dr * 17 + dc;
}

// centroid of a state in global memory, warp-cooperative
__device__ __forceinline__ void warp_centroid(const uint8_t* st, int& cq, int& cr) {
    const uint8_t* h = st + kOffHeight;
    int sq = 0, sr = 0, n = 0;
    for (int c = lane_id(); c < kCells; c += 32) {
        if (h[c]) {
            int r = c / kBoard;
            sq += c - r * kBoard - 11;
            sr += r - 11;
            n++;
        }
    }
    sq = __reduce_add_sync(kFull, sq);
    sr = __reduce_add_sync(kFull, sr);
    n = __reduce_add_sync(kFull, n);
    cq = n ? rhe_div(sq, n) : 0;
    cr = n ? rhe_div(sr, n) : 0;
}

// Expansion (dense: mcts_tree.cuh:971-1062; action space: :330-423) and the
// optional backup (:1068-1187, :435-549) of every simulation of game g.
__device__ __noinline__ void expand_game(const TreeDev& t, const ExpandArgs& a, int g) {
    const int l = lane_id();
    const uint32_t lt = lanemask_lt();
    for (int s = g; s < a.total; s += a.B) {
        const int leafn = a.leaf[s];
        if (leafn < 0) {
            if (!a.backprop && a.was && l == 0) a.was[s] = 0;
            continue;
        }
        const int64_t li = tix(t, g, leafn);
        const uint8_t* lst = a.leaf_states + (int64_t)s * kStateBytes;
        int expanded = 0;
        if (a.results[s] != 0) {
            if (l == 0) {
                t.it[li] = 1;
                t.tval[li] = result_value(a.results[s], lst[kOffTurn] | (lst[kOffTurn + 1] << 8));
            }
        } else if (t.fc[li] == -1) {
            const int n = a.num_legal[s];
            const int base = t.cnt[g];
            if (n > 0 && base + n <= t.max_nodes) {
                int cq, cr;
                warp_centroid(lst, cq, cr);
                const uint8_t* mv = a.legal + (int64_t)s * kMaxMoves * kMoveBytes;
                int made = 0;
                for (int m0 = 0; m0 < n; m0 += 32) {
                    int m = m0 + l;
                    int act = m < n ? move_action(mv + m * 6, cq, cr) : -1;
                    bool keep = m < n && (a.dense || act >= 0);
                    uint32_t b = __ballot_sync(kFull, keep);
                    if (keep) {
                        int child = base + made + __popc(b & lt);
                        int64_t ci = tix(t, g, child);
                        t.vc[ci] = 0;
                        t.tv[ci] = 0.0f;
                        t.pr[ci] = a.dense ? a.priors[(int64_t)s * kMaxMoves + m]
                                           : a.priors[(int64_t)s * 85834 + act];
                        t.pa[ci] = leafn;
                        t.ai[ci] = act;
                        t.fc[ci] = -1;
                        t.nc[ci] = 0;
                        t.it[ci] = 0;
                        t.tval[ci] = 0.0f;
                        if (a.dense) a.init_q[ci] = a.child_q[(int64_t)s * kMaxMoves + m];
#pragma unroll
                        for (int k = 0; k < 6; k++) t.mb[ci * 6 + k] = mv[m * 6 + k];
                    }
                    made += __popc(b);
                }
                __syncwarp();
                if (l == 0) {
                    t.cnt[g] = base + made;
                    t.nc[li] = made;
                    t.fc[li] = base;
                }
                expanded = 1;
            }
        }
        __syncwarp();
        if (!a.backprop) {
            if (a.was && l == 0) a.was[s] = (int8_t)expanded;
            continue;
        }
        if (l == 0) {
            float v = t.it[li] ? t.tval[li] : (expanded ? a.values[s] : 0.0f);
            const int vl = a.vll[s];
            for (int k = 0; k < vl; k++) {
                int64_t ni = tix(t, g, a.vlp[(int64_t)s * kTreeDepth + k]);
                if (a.qpen > 0.0f) {
                    t.vq[ni] = __fadd_rn(t.vq[ni], -a.qpen);
                } else {
                    t.vc[ni] -= 1;
                    t.tv[ni] = __fadd_rn(t.tv[ni], 1.0f);
                }
            }
            int node = leafn;
            for (int k = 0; k < kTreeDepth + 1 && node >= 0; k++) {
                int64_t ni = tix(t, g, node);
                t.vc[ni] += 1;
                t.tv[ni] = __fadd_rn(t.tv[ni], v);
                v = -v;
                node = t.pa[ni];
            }
        }
        __syncwarp();
    }
}

// The dense expansion + backup of one game, one block per game, with the
// results of expand_game, for simulations whose walks below the root fall
// into disjoint groups: slots != NULL -- the root-slot select, group of
// simulation s = its candidate (s / B) % C, one warp each (C warps); slots
// == NULL -- the plain / root-mask selects, group = the root child at the
// head of the simulation's virtual-loss path, warp = child mod the block's
// warps (simulations that stop at the root itself go to warp 0).
//  1. node allocation in simulation order (warp 0): a simulation expands iff
//     its leaf is unexpanded, not terminal, has moves and fits, and no earlier
//     simulation of the game expanded the same leaf (a leaf lies in one group,
//     so with candidates only the same candidate's earlier simulations are
//     checked);
//  2. each warp runs its groups' simulations in order: expansion at the
//     allocated base, virtual-loss removal and the backup up to the root
//     (every node below the root belongs to one group's subtree);
//  3. thread 0 adds the root-level updates (root and any ancestors) of every
//     simulation in simulation order, as the sequential backup does.
// A candidate table that repeats a slot takes expand_game instead.  Shared
// memory: 7 words per simulation of the game.
__device__ void expand_game_groups(const TreeDev& t, const ExpandArgs& a, const int32_t* roots,
                                   const int32_t* slots, int C, int g, int32_t* sm) {
    const int l = lane_id(), j = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int per = a.total / a.B;
    int32_t *leafv = sm, *nl = sm + per, *base = sm + 2 * per, *steps = sm + 3 * per, *stopn = sm + 4 * per;
    float* vroot = reinterpret_cast<float*>(sm + 5 * per);
    int32_t* grp = sm + 6 * per;  // warp of each simulation (-1: no walk)
    const int root = roots[g];
    __shared__ int dup;
    if (j == 0 && slots) {
        const int sl = l < C ? slots[(int64_t)g * C + l] : -1;
        const bool v = l < C && sl >= 0;
        const uint32_t same = __match_any_sync(kFull, v ? sl : -1 - l);
        const bool d = __any_sync(kFull, v && __popc(same) > 1);
        if (l == 0) dup = d;
    } else if (threadIdx.x == 0) {
        dup = 0;
    }
    __syncthreads();
    if (dup) {
        if (j == 0) expand_game(t, a, g);
        return;
    }
    // ---- 1. allocation
    if (j == 0) {
        for (int k = l; k < per; k += 32) {
            const int s = g + k * a.B, leafn = a.leaf[s];
            int n = 0;
            if (leafn >= 0 && a.results[s] == 0 && t.fc[tix(t, g, leafn)] == -1) n = a.num_legal[s];
            leafv[k] = leafn;
            nl[k] = n;  // > 0: a candidate for expansion
            int w = -1;
            if (leafn >= 0) {
                if (slots) w = k % C;
                else w = a.vll[s] > 0 ? a.vlp[(int64_t)s * kTreeDepth] % nw : 0;
            }
            grp[k] = w;
        }
        __syncwarp();
        if (l == 0) {
            int cur = t.cnt[g];
            for (int k = 0; k < per; k++) {
                int b = -1;
                const int n = nl[k];
                if (n > 0) {
                    bool seen = false;
                    const int stride = slots ? C : 1;
                    for (int q = k - stride; q >= 0 && !seen; q -= stride)
                        seen = base[q] >= 0 && leafv[q] == leafv[k];
                    if (!seen && cur + n <= t.max_nodes) {
                        b = cur;
                        cur += n;
                    }
                }
                base[k] = b;
            }
            t.cnt[g] = cur;
        }
    }
    __syncthreads();
    // ---- 2. each warp's groups, in simulation order
    for (int k = 0; k < per; k++) {
        if (grp[k] != j) {
            if (grp[k] < 0 && j == 0 && l == 0) steps[k] = -1;
            continue;
        }
        const int s = g + k * a.B, leafn = leafv[k];
        const int64_t li = tix(t, g, leafn);
        const uint8_t* lst = a.leaf_states + (int64_t)s * kStateBytes;
        int expanded = 0;
        if (a.results[s] != 0) {
            if (l == 0) {
                t.it[li] = 1;
                t.tval[li] = result_value(a.results[s], lst[kOffTurn] | (lst[kOffTurn + 1] << 8));
            }
        } else if (base[k] >= 0) {
            const int n = nl[k], b0 = base[k];
            int cq, cr;
            warp_centroid(lst, cq, cr);
            const uint8_t* mv = a.legal + (int64_t)s * kMaxMoves * kMoveBytes;
            for (int m = l; m < n; m += 32) {
                const int64_t ci = tix(t, g, b0 + m);
                t.vc[ci] = 0;
                t.tv[ci] = 0.0f;
                t.pr[ci] = a.priors[(int64_t)s * kMaxMoves + m];
                t.pa[ci] = leafn;
                t.ai[ci] = move_action(mv + m * 6, cq, cr);
                t.fc[ci] = -1;
                t.nc[ci] = 0;
                t.it[ci] = 0;
                t.tval[ci] = 0.0f;
                a.init_q[ci] = a.child_q[(int64_t)s * kMaxMoves + m];
#pragma unroll
                for (int q = 0; q < 6; q++) t.mb[ci * 6 + q] = mv[m * 6 + q];
            }
            __syncwarp();
            if (l == 0) {
                t.nc[li] = n;
                t.fc[li] = b0;
            }
            expanded = 1;
        }
        __syncwarp();
        if (l == 0) {
            float v = t.it[li] ? t.tval[li] : (expanded ? a.values[s] : 0.0f);
            const int vl = a.vll[s];
            for (int q = 0; q < vl; q++) {
                const int64_t ni = tix(t, g, a.vlp[(int64_t)s * kTreeDepth + q]);
                if (a.qpen > 0.0f) {
                    t.vq[ni] = __fadd_rn(t.vq[ni], -a.qpen);
                } else {
                    t.vc[ni] -= 1;
                    t.tv[ni] = __fadd_rn(t.tv[ni], 1.0f);
                }
            }
            int node = leafn, q = 0;
            for (; q < kTreeDepth + 1 && node >= 0 && node != root; q++) {
                const int64_t ni = tix(t, g, node);
                t.vc[ni] += 1;
                t.tv[ni] = __fadd_rn(t.tv[ni], v);
                v = -v;
                node = t.pa[ni];
            }
            steps[k] = q;
            stopn[k] = node;
            vroot[k] = v;
        }
        __syncwarp();
    }
    __syncthreads();
    // ---- 3. root-level updates in simulation order (one node cached in registers)
    if (threadIdx.x == 0) {
        int cn = -1, cvc = 0;
        float ctv = 0.0f;
        for (int k = 0; k < per; k++) {
            int q = steps[k], node = stopn[k];
            if (q < 0) continue;
            float v = vroot[k];
            for (; q < kTreeDepth + 1 && node >= 0; q++) {
                const int64_t ni = tix(t, g, node);
                if (node != cn) {
                    if (cn >= 0) {
                        t.vc[tix(t, g, cn)] = cvc;
                        t.tv[tix(t, g, cn)] = ctv;
                    }
                    cn = node;
                    cvc = t.vc[ni];
                    ctv = t.tv[ni];
                }
                cvc += 1;
                ctv = __fadd_rn(ctv, v);
                v = -v;
                node = t.pa[ni];
            }
        }
        if (cn >= 0) {
            t.vc[tix(t, g, cn)] = cvc;
            t.tv[tix(t, g, cn)] = ctv;
        }
    }
}

// legacy backup given was_expanded (mcts_tree.cuh:555-605)
__device__ __noinline__ void backprop_game(const TreeDev& t, const int32_t* leaf, const float* values,
                                           const int32_t* vlp, const int32_t* vll, const int8_t* was,
                                           int B, int total, int g) {
    if (lane_id() != 0) return;
    for (int s = g; s < total; s += B) {
        int leafn = leaf[s];
        if (leafn < 0) continue;
        int64_t li = tix(t, g, leafn);
        float v = t.it[li] ? t.tval[li] : (was[s] ? values[s] : 0.0f);
        for (int k = 0; k < vll[s]; k++) {
            int64_t ni = tix(t, g, vlp[(int64_t)s * kTreeDepth + k]);
            t.vc[ni] -= 1;
            t.tv[ni] = __fadd_rn(t.tv[ni], 1.0f);
        }
        int node = leafn;
        for (int k = 0; k < kTreeDepth + 1 && node >= 0; k++) {
            int64_t ni = tix(t, g, node);
            t.vc[ni] += 1;
            t.tv[ni] = __fadd_rn(t.tv[ni], v);
            v = -v;
            node = t.pa[ni];
        }
    }
}

}  // namespace hv
