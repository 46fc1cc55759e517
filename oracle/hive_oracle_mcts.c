/*
 * hive_oracle_mcts.c -- CPU oracle (TEST INFRASTRUCTURE ONLY) for the GPU
 * MCTS tree operations of the reference (hive_gpu/csrc/mcts_tree.cuh), in
 * the defined sequential order: simulations are processed in increasing
 * simulation index, each seeing the virtual loss / expansions / backups of
 * the ones before it.  The reference's own GPU launch runs them concurrently
 * (its wave results then depend on thread timing); the B200 kernels
 * reproduce this sequential order exactly.  Pinned against the reference's
 * kernels executed sequentially on the host (oracle/ref_driver.cpp) in
 * tests/test_oracle_mcts.py.
 */
#include <math.h>
#include <string.h>

#include "hive_oracle.h"

typedef struct {
    int32_t* vc;   /* visit_count */
    float* tv;     /* total_value */
    float* pr;     /* prior */
    int32_t* pa;   /* parent_idx */
    float* vq;     /* virtual_q_penalty */
    uint8_t* mb;   /* move_bytes [.., 6] */
    int32_t* ai;   /* action_idx */
    int32_t* fc;   /* first_child */
    int32_t* nc;   /* num_children */
    int8_t* it;    /* is_terminal */
    float* tval;   /* terminal_value */
    int32_t* cnt;  /* node_count [B] */
    int32_t max_nodes;
} orc_tree;

#define DEPTH 128
#define ACTIONS 85834

static inline long ix(const orc_tree* t, int g, int n) { return (long)g * t->max_nodes + n; }

/* PUCT (mcts_tree.cuh:55-67): Q = -W/N - penalty, U = c P sqrt(N_parent)/(1+N) */
static float puct(const orc_tree* t, int g, int parent, int child, float c) {
    long ci = ix(t, g, child), pi = ix(t, g, parent);
    int n = t->vc[ci];
    float q = n > 0 ? -t->tv[ci] / (float)n : 0.0f;
    q -= t->vq[ci];
    float u = c * t->pr[ci];
    u = u * sqrtf((float)t->vc[pi]);
    u = u / (1.0f + (float)n);
    return q + u;
}

/* Gumbel completed-Q child choice below the root (mcts_tree.cuh:77-143) */
static int completed_q_child(const orc_tree* t, int g, int first, int n, float sigma,
                             const float* init_q) {
    float sumv = 0.0f, mx = -1e30f, se = 0.0f;
    for (int c = 0; c < n; c++) {
        if (first + c < 0 || first + c >= t->max_nodes) break;
        sumv += (float)t->vc[ix(t, g, first + c)];
    }
    for (int pass = 0; pass < 2; pass++) {
        for (int c = 0; c < n; c++) {
            if (first + c < 0 || first + c >= t->max_nodes) break;
            long ci = ix(t, g, first + c);
            float v = (float)t->vc[ci];
            float q = v > 0.0f ? -t->tv[ci] / v : init_q[ci];
            q -= t->vq[ci];
            float lq = logf(fmaxf(t->pr[ci], 1e-20f)) + sigma * q;
            if (pass == 0) { if (lq > mx) mx = lq; }
            else se += expf(lq - mx);
        }
    }
    se = fmaxf(se, 1e-20f);
    int best = -1;
    float bs = -1e30f, den = 1.0f + sumv;
    for (int c = 0; c < n; c++) {
        if (first + c < 0 || first + c >= t->max_nodes) break;
        long ci = ix(t, g, first + c);
        float v = (float)t->vc[ci];
        float q = v > 0.0f ? -t->tv[ci] / v : init_q[ci];
        q -= t->vq[ci];
        float pi0 = expf(logf(fmaxf(t->pr[ci], 1e-20f)) + sigma * q - mx) / se;
        float s = pi0 - v / den;
        if (s > bs) { bs = s; best = first + c; }
    }
    return best;
}

static void record(const orc_tree* t, int g, int node, uint8_t* paths, int* plen, int32_t* vls,
                   int* vlen) {
    if (*vlen < DEPTH) vls[(*vlen)++] = node;
    if (*plen < DEPTH) {
        memcpy(paths + (long)(*plen) * 6, t->mb + ix(t, g, node) * 6, 6);
        (*plen)++;
    }
}

/*
 * mode 0: plain PUCT from the root (mcts_tree.cuh:205-291)
 * mode 1: root children filtered by alive_mask (:689-800)
 * mode 2: simulation pinned to root slot root_slots[g, (s / B) % C] (:811-955)
 */
void orc_mcts_select(const orc_tree* t, int mode, const float* init_q, const int8_t* active,
                     const int32_t* roots, const int8_t* alive, const int32_t* slots, int C,
                     int max_root_children, float c_puct, int B, int W, int det, float sigma,
                     float qpen, int32_t* leaf, uint8_t* mpaths, int32_t* plens, int32_t* vlpaths,
                     int32_t* vlens) {
    int total = mode == 2 ? W * C * B : W * B;
    for (int s = 0; s < total; s++) {
        int g = s % B, plen = 0, vlen = 0;
        uint8_t* paths = mpaths + (long)s * DEPTH * 6;
        int32_t* vls = vlpaths + (long)s * DEPTH;
        leaf[s] = -1;
        plens[s] = vlens[s] = 0;
        if (!active[g]) continue;
        int root = roots[g], node = root, start_iter = 0;
        if (mode == 2) {
            int slot = slots[(long)g * C + (s / B) % C];
            if (slot < 0 || slot >= max_root_children) continue;
            long ri = ix(t, g, root);
            int fc = t->fc[ri], nc = t->nc[ri];
            if (fc < 0 || t->it[ri] || nc <= 0 || slot >= nc) continue;
            node = fc + slot;
            if (node < 0 || node >= t->max_nodes) continue;
            long ni = ix(t, g, node);
            if (!det) {
                t->vc[ni] += 1;
                t->tv[ni] += -1.0f;
                if (vlen < DEPTH) vls[vlen++] = node;
            }
            if (plen < DEPTH) {
                memcpy(paths + (long)plen * 6, t->mb + ni * 6, 6);
                plen++;
            }
            start_iter = 1;
        }
        for (int it = start_iter; it < DEPTH; it++) {
            long ni = ix(t, g, node);
            int fc = t->fc[ni], nc = t->nc[ni];
            if (fc < 0 || t->it[ni] || nc == 0) break;
            if (nc <= 0 || nc > 1024) break;
            int at_root = mode != 2 && node == root;
            int best = mode == 0 ? fc : -1;
            float bs = -1e30f;
            int use_det = det && mode != 0 && !at_root;
            if (use_det) {
                best = completed_q_child(t, g, fc, nc, sigma, init_q);
            } else {
                for (int c = 0; c < nc; c++) {
                    if (fc + c < 0 || fc + c >= t->max_nodes) break;
                    if (mode == 1 && at_root && (c >= max_root_children || !alive[(long)g * max_root_children + c]))
                        continue;
                    float sc = puct(t, g, node, fc + c, c_puct);
                    if (sc > bs) { bs = sc; best = fc + c; }
                }
            }
            if (best < 0) break;
            node = best;
            long bi = ix(t, g, node);
            t->vc[bi] += 1;
            if (use_det) t->vq[bi] += qpen;
            else t->tv[bi] += -1.0f;
            if (vlen < DEPTH) vls[vlen++] = node;
            if (plen < DEPTH) {
                memcpy(paths + (long)plen * 6, t->mb + bi * 6, 6);
                plen++;
            }
        }
        (void)record;
        leaf[s] = node;
        plens[s] = plen;
        vlens[s] = vlen;
    }
}

/* mcts_replay_kernel, mcts_tree.cuh:298-320 */
void orc_mcts_replay(const uint8_t* roots, uint8_t* leaves, const uint8_t* mpaths,
                     const int32_t* plens, const int32_t* leaf, int B, int total) {
    for (int s = 0; s < total; s++) {
        if (leaf[s] < 0) continue;
        orc_state* st = (orc_state*)(leaves + (long)s * ORC_STATE_BYTES);
        memcpy(st, roots + (long)(s % B) * ORC_STATE_BYTES, ORC_STATE_BYTES);
        for (int d = 0; d < plens[s]; d++)
            orc_apply_move(st, (const orc_move*)(mpaths + ((long)s * DEPTH + d) * 6));
    }
}

/* terminal value from the leaf player's perspective (mcts_tree.cuh:182-188) */
static float result_value(int result, int turn) {
    if (result == 3) return 0.0f;
    int white = (turn & 1) == 0;
    if (result == 1) return white ? 1.0f : -1.0f;
    if (result == 2) return white ? -1.0f : 1.0f;
    return 0.0f;
}

static int leaf_turn(const uint8_t* st) { return st[3412] | (st[3413] << 8); }

/* Shared expansion: returns 1 if this simulation created the children.
 * dense: priors per legal slot + child_init_q; else action-space priors. */
static int expand_one(const orc_tree* t, int s, int B, int leafn, const uint8_t* lstate,
                      const uint8_t* legal, const int32_t* num_legal, const float* priors,
                      const float* child_q, float* init_q, const int32_t* results, int dense) {
    int g = s % B;
    long li = ix(t, g, leafn);
    if (results[s] != 0) {
        t->it[li] = 1;
        t->tval[li] = result_value(results[s], leaf_turn(lstate));
        return 0;
    }
    if (t->fc[li] != -1) return 0;
    t->fc[li] = -2;
    int n = num_legal[s];
    if (n <= 0) { t->fc[li] = -1; return 0; }
    int cq, cr;
    orc_centroid((const orc_state*)lstate, &cq, &cr);
    int base = t->cnt[g];
    t->cnt[g] += n;
    if (base + n > t->max_nodes) {
        t->cnt[g] -= n;
        t->fc[li] = -1;
        return 0;
    }
    int made = 0;
    for (int m = 0; m < n; m++) {
        const orc_move* mv = (const orc_move*)(legal + ((long)s * ORC_MAX_MOVES + m) * 6);
        int a = orc_move_to_action(mv, cq, cr);
        if (!dense && a < 0) continue;
        long ci = ix(t, g, base + made);
        t->vc[ci] = 0;
        t->tv[ci] = 0.0f;
        t->pr[ci] = dense ? priors[(long)s * ORC_MAX_MOVES + m] : priors[(long)s * ACTIONS + a];
        t->pa[ci] = leafn;
        t->ai[ci] = a;
        t->fc[ci] = -1;
        t->nc[ci] = 0;
        t->it[ci] = 0;
        t->tval[ci] = 0.0f;
        if (dense) init_q[ci] = child_q[(long)s * ORC_MAX_MOVES + m];
        memcpy(t->mb + ci * 6, mv, 6);
        made++;
    }
    t->nc[li] = made;
    if (made < n) t->cnt[g] -= n - made;
    t->fc[li] = base;
    return 1;
}

static void backup(const orc_tree* t, int s, int B, int leafn, int expanded, const float* values,
                   const int32_t* vlpaths, const int32_t* vlens, float qpen) {
    int g = s % B;
    long li = ix(t, g, leafn);
    float v = t->it[li] ? t->tval[li] : (expanded ? values[s] : 0.0f);
    for (int k = 0; k < vlens[s]; k++) {
        long ni = ix(t, g, vlpaths[(long)s * DEPTH + k]);
        if (qpen > 0.0f) t->vq[ni] += -qpen;
        else {
            t->vc[ni] += -1;
            t->tv[ni] += 1.0f;
        }
    }
    int node = leafn;
    for (int k = 0; k < DEPTH + 1 && node >= 0; k++) {
        long ni = ix(t, g, node);
        t->vc[ni] += 1;
        t->tv[ni] += v;
        v = -v;
        node = t->pa[ni];
    }
}

/* dense-prior expansion (:971-1062), optionally fused with the backup (:1068-1187) */
void orc_mcts_expand_dense(const orc_tree* t, float* init_q, const float* child_q,
                           const int32_t* leaf, const uint8_t* lstates, const uint8_t* legal,
                           const int32_t* num_legal, const float* priors, const int32_t* results,
                           const float* values, const int32_t* vlpaths, const int32_t* vlens, int B,
                           int total, float qpen, int with_backprop, int8_t* was_expanded) {
    for (int s = 0; s < total; s++) {
        if (leaf[s] < 0) {
            if (!with_backprop && was_expanded) was_expanded[s] = 0;
            continue;
        }
        int e = expand_one(t, s, B, leaf[s], lstates + (long)s * ORC_STATE_BYTES, legal, num_legal,
                           priors, child_q, init_q, results, 1);
        if (with_backprop) backup(t, s, B, leaf[s], e, values, vlpaths, vlens, qpen);
        else if (was_expanded) was_expanded[s] = (int8_t)e;
    }
}

/* action-space expansion (:330-423), fused expand+backup (:435-549), backup (:555-605) */
void orc_mcts_expand_action(const orc_tree* t, const int32_t* leaf, const uint8_t* lstates,
                            const uint8_t* legal, const int32_t* num_legal, const float* probs,
                            const int32_t* results, const float* values, const int32_t* vlpaths,
                            const int32_t* vlens, int B, int total, int mode, int8_t* was_expanded) {
    for (int s = 0; s < total; s++) {
        if (leaf[s] < 0) {
            if (mode == 0) was_expanded[s] = 0;
            continue;
        }
        if (mode == 2) {
            backup(t, s, B, leaf[s], was_expanded[s], values, vlpaths, vlens, 0.0f);
            continue;
        }
        int e = expand_one(t, s, B, leaf[s], lstates + (long)s * ORC_STATE_BYTES, legal, num_legal,
                           probs, 0, 0, results, 0);
        if (mode == 0) was_expanded[s] = (int8_t)e;
        else backup(t, s, B, leaf[s], e, values, vlpaths, vlens, 0.0f);
    }
}

/* visit-count policy over the action space (:607-684) */
void orc_mcts_extract_policy(const orc_tree* t, float* pol, const int32_t* move_numbers,
                             const int32_t* roots, float temperature, int drop, float prune, int B) {
    for (int g = 0; g < B; g++) {
        float* p = pol + (long)g * ACTIONS;
        long ri = ix(t, g, roots[g]);
        int fc = t->fc[ri], nc = t->nc[ri];
        if (fc < 0 || nc == 0) continue;
        float temp = move_numbers[g] >= drop ? 0.0f : temperature;
        if (temp <= 0.0f) {
            int ba = -1, bv = -1;
            for (int c = 0; c < nc; c++) {
                long ci = ix(t, g, fc + c);
                if (t->vc[ci] > bv) { bv = t->vc[ci]; ba = t->ai[ci]; }
            }
            if (ba >= 0 && ba < ACTIONS) p[ba] = 1.0f;
            continue;
        }
        float mx = 0.0f, sum = 0.0f;
        for (int c = 0; c < nc; c++) {
            float v = (float)t->vc[ix(t, g, fc + c)];
            if (v > mx) mx = v;
        }
        for (int c = 0; c < nc; c++) {
            long ci = ix(t, g, fc + c);
            float v = (float)t->vc[ci];
            if (prune > 0.0f && mx > 0.0f && v < mx * prune) v = 0.0f;
            if (temp != 1.0f) v = powf(v, 1.0f / temp);
            int a = t->ai[ci];
            if (a >= 0 && a < ACTIONS) { p[a] = v; sum += v; }
        }
        for (int c = 0; c < nc; c++) {
            int a = t->ai[ix(t, g, fc + c)];
            if (a >= 0 && a < ACTIONS) p[a] = sum > 0.0f ? p[a] / sum : 1.0f / (float)nc;
        }
    }
}

/* root prior temperature and Dirichlet mix (:1192-1234) */
void orc_mcts_root_noise(const orc_tree* t, const float* noise, const int32_t* roots, int pad,
                         float eps, float temp, int B) {
    for (int g = 0; g < B; g++) {
        long ri = ix(t, g, roots[g]);
        int fc = t->fc[ri], nc = t->nc[ri];
        if (fc < 0 || nc == 0) continue;
        if (temp > 1.0f) {
            float inv = 1.0f / temp, sum = 0.0f;
            for (int c = 0; c < nc; c++) {
                long ci = ix(t, g, fc + c);
                t->pr[ci] = powf(t->pr[ci], inv);
                sum += t->pr[ci];
            }
            if (sum > 0.0f)
                for (int c = 0; c < nc; c++) t->pr[ix(t, g, fc + c)] /= sum;
        }
        if (eps > 0.0f)
            for (int c = 0; c < nc; c++) {
                long ci = ix(t, g, fc + c);
                float a = (1.0f - eps) * t->pr[ci];
                float b = eps * noise[(long)g * pad + c];
                t->pr[ci] = a + b;
            }
    }
}
