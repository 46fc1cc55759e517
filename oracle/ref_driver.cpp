// ref_driver.cpp -- builds the REFERENCE's own game-logic headers on the host.
//
// TEST INFRASTRUCTURE ONLY.  This file contains no reference code: it
// #includes the reference's headers from the reference tree at build time
// (oracle/Makefile passes -I <reference>/hive_gpu/csrc) and wraps their
// __device__ functions in batched extern "C" loops, the way the reference's
// own host build hive_gpu/csrc/cpu_native.cpp:14-46 does.  The resulting
// oracle/_ref/libhive_ref.so is used (a) to validate the C restatement in
// oracle/hive_oracle.c and (b) as the timed CPU baseline ("kind":
// "reference") in bench.py.  It is never part of the product.
//
// Kernel loops mirror the reference kernels in hive_gpu/csrc/game_logic.cu:
//   generate_legal_moves_and_fnn_features_kernel  game_logic.cu:76-91
//   fnn_successor_features_kernel                 game_logic.cu:182-229
//   apply_moves_kernel                            game_logic.cu:233-244
//   legal_moves_to_actions_kernel                 game_logic.cu:811-835

#include <cstdint>
#include <cstring>
#include <cmath>
#include <omp.h>

#define HIVE_CPU_NATIVE 1
#define __CUDACC__ 1
#define __device__
#define __host__
#define __forceinline__ inline
#define __global__
#define __managed__
#define __constant__
#define max(a, b) (((a) > (b)) ? (a) : (b))
#define min(a, b) (((a) < (b)) ? (a) : (b))

static inline int __ffsll(unsigned long long x) { return x ? __builtin_ctzll(x) + 1 : 0; }
template <typename T>
static inline T atomicAdd(T* p, T v) { T o = *p; *p += v; return o; }
static inline int atomicCAS(int* p, int cmp, int v) { int o = *p; if (o == cmp) *p = v; return o; }
static inline void __threadfence() {}
struct hv_dim3 { unsigned x, y, z; };
static thread_local hv_dim3 threadIdx = {0, 0, 0}, blockIdx = {0, 0, 0};
static const hv_dim3 blockDim = {1, 1, 1};

#include "hex_grid.cuh"
#include "hive_state.cuh"
#include "articulation.cuh"
#include "move_gen.cuh"
#include "fnn_features.cuh"
#include "state_encoder.cuh"
#include "mcts_tree.cuh"

#undef max
#undef min

using namespace hive_gpu;

static_assert(sizeof(HiveState) == 3424, "HiveState layout");
static_assert(sizeof(GPUMove) == 6, "GPUMove layout");

static void tables_once() {
    static bool done = false;
    if (done) return;
#pragma omp critical(ref_tables)
    {
        if (!done) {
            init_hex_tables();
            std::memcpy(NEIGHBORS, HOST_NEIGHBOR_TABLE, sizeof(HOST_NEIGHBOR_TABLE));
            std::memcpy(SLIDE_FLANKS, HOST_SLIDE_TABLE, sizeof(HOST_SLIDE_TABLE));
            done = true;
        }
    }
}

static inline int nthreads(int t) { return t > 0 ? t : omp_get_max_threads(); }

extern "C" {

int ref_sizeof_state() { return (int)sizeof(HiveState); }

void ref_init_states(uint8_t* out, int64_t count, int mask) {
    tables_once();
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memset(&s, 0, sizeof(s));
        init_state(s, (uint8_t)mask);
        std::memcpy(out + i * sizeof(HiveState), &s, sizeof(s));
    }
}

void ref_legal_moves_features_batch(const uint8_t* states, int64_t count, uint8_t* moves,
                                    int32_t* num_legal, float* feats, int threads) {
    tables_once();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads(threads))
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        GPUMove mv[MAX_LEGAL_MOVES];
        std::memset(mv, 0, sizeof(mv));
        int n = generate_legal_moves(s, mv);
        num_legal[i] = n;
        if (moves) std::memcpy(moves + i * sizeof(mv), mv, sizeof(mv));
        if (feats) extract_fnn_features_device(s, mv, n, feats + i * FNN_FEAT_DIM);
    }
}

void ref_features_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                        int64_t count, float* feats, int threads) {
    tables_once();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads(threads))
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        extract_fnn_features_device(
            s, reinterpret_cast<const GPUMove*>(moves + i * MAX_LEGAL_MOVES * sizeof(GPUMove)),
            num_legal[i], feats + i * FNN_FEAT_DIM);
    }
}

void ref_compact_moves_batch(const uint8_t* states, int64_t count, uint8_t* moves,
                             int32_t* num_legal, int threads) {
    tables_once();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads(threads))
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        GPUMove mv[MAX_LEGAL_MOVES];
        std::memset(mv, 0, sizeof(mv));
        num_legal[i] = generate_fnn_feature_moves(s, mv);
        std::memcpy(moves + i * sizeof(mv), mv, sizeof(mv));
    }
}

void ref_successor_features_batch(const uint8_t* states, const uint8_t* moves,
                                  const int64_t* action_to_root, const int64_t* move_indices,
                                  int64_t count, float* feats, int threads) {
    tables_once();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads(threads))
    for (int64_t i = 0; i < count; i++) {
        int64_t root = action_to_root[i];
        HiveState child;
        std::memcpy(&child, states + root * sizeof(HiveState), sizeof(child));
        GPUMove mv;
        std::memcpy(&mv, moves + (root * MAX_LEGAL_MOVES + move_indices[i]) * sizeof(GPUMove),
                    sizeof(mv));
        apply_move(child, mv);
        GPUMove cm[MAX_LEGAL_MOVES];
        int n = generate_fnn_feature_moves(child, cm);
        extract_fnn_features_device(child, cm, n, feats + i * FNN_FEAT_DIM);
    }
}

void ref_apply_moves_batch(uint8_t* states, const uint8_t* moves, int64_t count) {
    tables_once();
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        GPUMove mv;
        std::memcpy(&mv, moves + i * sizeof(GPUMove), sizeof(mv));
        apply_move(s, mv);
        std::memcpy(states + i * sizeof(HiveState), &s, sizeof(s));
    }
}

void ref_articulation_batch(const uint8_t* states, int64_t count, uint64_t* ap, int threads) {
    tables_once();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads(threads))
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        Bitboard b = find_articulation_points(s);
        std::memcpy(ap + i * BB_WORDS, b.w, sizeof(b.w));
    }
}

void ref_actions_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                       int64_t count, int32_t* actions, int32_t* centroids) {
    tables_once();
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        int cq, cr;
        compute_centroid(s, cq, cr);
        if (centroids) { centroids[2 * i] = cq; centroids[2 * i + 1] = cr; }
        const GPUMove* mv =
            reinterpret_cast<const GPUMove*>(moves + i * MAX_LEGAL_MOVES * sizeof(GPUMove));
        for (int m = 0; m < MAX_LEGAL_MOVES; m++) actions[i * MAX_LEGAL_MOVES + m] = -1;
        for (int m = 0; m < num_legal[i]; m++)
            actions[i * MAX_LEGAL_MOVES + m] = gpu_move_to_action(mv[m], cq, cr);
    }
}

// Seeded playout generator with the same counter RNG as oracle/hive_oracle.c
// (orc_rng / orc_playout), driven by the reference's own move generator.
static inline uint64_t rmix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
static inline uint64_t rrng(uint64_t seed, uint64_t game, uint64_t ply) {
    return rmix(rmix(seed ^ rmix(game)) + ply);
}

void ref_generate_positions(uint64_t seed, int64_t first_game, int64_t count, int max_ply,
                            int mask, uint8_t* out, int threads) {
    tables_once();
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads(threads))
    for (int64_t i = 0; i < count; i++) {
        uint64_t g = (uint64_t)(first_game + i);
        HiveState s;
        std::memset(&s, 0, sizeof(s));
        init_state(s, (uint8_t)mask);
        int stop = (int)(rrng(seed, g, 0) % (uint64_t)(max_ply + 1));
        GPUMove mv[MAX_LEGAL_MOVES];
        for (int p = 1; p <= stop; p++) {
            if (s.result != IN_PROGRESS) break;
            int n = generate_legal_moves(s, mv);
            apply_move(s, mv[rrng(seed, g, (uint64_t)p) % (uint64_t)n]);
        }
        std::memcpy(out + i * sizeof(HiveState), &s, sizeof(s));
    }
}

void ref_queen_escape_batch(const uint8_t* states, int64_t count, uint8_t* flags) {
    tables_once();
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        flags[i] = has_queen_escape_move(s) ? 1 : 0;
    }
}

}  // extern "C"

// ---------------------------------------------------------------------------
// MCTS: the reference's tree kernels (mcts_tree.cuh) executed sequentially in
// simulation-index order on the host.  This is the defined order the B200
// kernels reproduce (the reference's own GPU launch races when several
// simulations of one game share a wave).
// ---------------------------------------------------------------------------
struct ref_tree_ptrs {
    int32_t* visit_count;
    float* total_value;
    float* prior;
    int32_t* parent_idx;
    float* virtual_q_penalty;
    uint8_t* move_bytes;
    int32_t* action_idx;
    int32_t* first_child;
    int32_t* num_children;
    int8_t* is_terminal;
    float* terminal_value;
    int32_t* node_count;
    int32_t max_nodes;
};

static MCTSTree to_tree(const ref_tree_ptrs* p) {
    MCTSTree t;
    t.visit_count = p->visit_count;
    t.total_value = p->total_value;
    t.prior = p->prior;
    t.virtual_q_penalty = p->virtual_q_penalty;
    t.parent_idx = p->parent_idx;
    t.move_bytes = p->move_bytes;
    t.action_idx = p->action_idx;
    t.first_child = p->first_child;
    t.num_children = p->num_children;
    t.is_terminal = p->is_terminal;
    t.terminal_value = p->terminal_value;
    t.node_count = p->node_count;
    t.max_nodes = p->max_nodes;
    return t;
}

static inline void as_thread(int sim) {
    blockIdx.x = (unsigned)sim;
    threadIdx.x = 0;
}

extern "C" {

void ref_mcts_select(const ref_tree_ptrs* tp, int mode, const float* child_init_q,
                     const int8_t* game_active, const int32_t* root_nodes, const int8_t* alive_mask,
                     const int32_t* root_slots, int num_candidates, int max_root_children,
                     float c_puct, int B, int W, int deterministic_non_root, float non_root_sigma,
                     float q_penalty, int32_t* leaf, uint8_t* move_paths, int32_t* path_len,
                     int32_t* vl_paths, int32_t* vl_len) {
    tables_once();
    MCTSTree t = to_tree(tp);
    int total = mode == 2 ? W * num_candidates * B : W * B;
    for (int s = 0; s < total; s++) {
        as_thread(s);
        if (mode == 0)
            mcts_select_kernel(t, leaf, move_paths, path_len, vl_paths, vl_len, game_active,
                               root_nodes, c_puct, B, total);
        else if (mode == 1)
            mcts_select_with_root_mask_kernel(t, leaf, move_paths, path_len, vl_paths, vl_len,
                                              game_active, root_nodes, alive_mask,
                                              max_root_children, c_puct,
                                              deterministic_non_root != 0, non_root_sigma,
                                              q_penalty, child_init_q, B, total);
        else
            mcts_select_with_root_slots_kernel(t, leaf, move_paths, path_len, vl_paths, vl_len,
                                               game_active, root_nodes, root_slots, num_candidates,
                                               max_root_children, c_puct,
                                               deterministic_non_root != 0, non_root_sigma,
                                               q_penalty, child_init_q, B, total);
    }
}

void ref_mcts_replay(const uint8_t* root_states, uint8_t* leaf_states, const uint8_t* move_paths,
                     const int32_t* path_len, const int32_t* leaf, int B, int total) {
    tables_once();
    for (int s = 0; s < total; s++) {
        as_thread(s);
        mcts_replay_kernel(reinterpret_cast<const HiveState*>(root_states),
                           reinterpret_cast<HiveState*>(leaf_states), move_paths, path_len, leaf, B,
                           total);
    }
}

// dense-prior expansion, optionally fused with the backup
void ref_mcts_expand_dense(const ref_tree_ptrs* tp, float* child_init_q, const float* child_q,
                           const int32_t* leaf, const uint8_t* leaf_states, const uint8_t* legal,
                           const int32_t* num_legal, const float* priors, const int32_t* results,
                           const float* values, const int32_t* vl_paths, const int32_t* vl_len,
                           int B, int total, float q_penalty, int with_backprop,
                           int8_t* was_expanded) {
    tables_once();
    MCTSTree t = to_tree(tp);
    for (int s = 0; s < total; s++) {
        as_thread(s);
        if (with_backprop)
            mcts_expand_and_backprop_dense_priors_kernel(
                t, leaf, reinterpret_cast<const HiveState*>(leaf_states),
                reinterpret_cast<const GPUMove*>(legal), num_legal, priors, child_q, child_init_q,
                results, values, vl_paths, vl_len, q_penalty, B, total);
        else
            mcts_expand_dense_priors_kernel(t, leaf, reinterpret_cast<const HiveState*>(leaf_states),
                                            reinterpret_cast<const GPUMove*>(legal), num_legal,
                                            priors, child_q, child_init_q, results, was_expanded, B,
                                            total);
    }
}

// action-space expansion / backup (legacy path)
void ref_mcts_expand_action(const ref_tree_ptrs* tp, const int32_t* leaf, const uint8_t* leaf_states,
                            const uint8_t* legal, const int32_t* num_legal, const float* probs,
                            const int32_t* results, const float* values, const int32_t* vl_paths,
                            const int32_t* vl_len, int B, int total, int mode, int8_t* was_expanded) {
    tables_once();
    MCTSTree t = to_tree(tp);
    for (int s = 0; s < total; s++) {
        as_thread(s);
        if (mode == 0)
            mcts_expand_kernel(t, leaf, reinterpret_cast<const HiveState*>(leaf_states),
                               reinterpret_cast<const GPUMove*>(legal), num_legal, probs, results,
                               was_expanded, B, total);
        else if (mode == 1)
            mcts_expand_and_backprop_kernel(t, leaf, reinterpret_cast<const HiveState*>(leaf_states),
                                            reinterpret_cast<const GPUMove*>(legal), num_legal, probs,
                                            results, values, vl_paths, vl_len, B, total);
        else
            mcts_backprop_kernel(t, leaf, values, vl_paths, vl_len, was_expanded, B, total);
    }
}

void ref_mcts_extract_policy(const ref_tree_ptrs* tp, float* policies, const int32_t* move_numbers,
                             const int32_t* root_nodes, float temperature, int temp_drop_move,
                             float pruning_threshold, int B) {
    tables_once();
    MCTSTree t = to_tree(tp);
    for (int g = 0; g < B; g++) {
        as_thread(g);
        mcts_extract_policy_kernel(t, policies, move_numbers, root_nodes, temperature,
                                   temp_drop_move, pruning_threshold, B);
    }
}

void ref_mcts_root_noise(const ref_tree_ptrs* tp, const float* noise, const int32_t* root_nodes,
                         int max_children_pad, float dir_eps, float root_policy_temp, int B) {
    tables_once();
    MCTSTree t = to_tree(tp);
    for (int g = 0; g < B; g++) {
        as_thread(g);
        mcts_root_noise_kernel(t, noise, root_nodes, max_children_pad, dir_eps, root_policy_temp, B);
    }
}

}  // extern "C"

// root_tactical_probe_kernel (game_logic.cu:290-397) lives in a .cu file
// with torch host code, so its body is followed here step by step over the
// reference's own helpers from move_gen.cuh / hive_state.cuh
// (num_occupied_neighbors, has_immediate_surround_win_for_current_player,
// generate_non_decreasing_surround_replies, apply_move).
extern "C" void ref_tactical_probe_batch(const uint8_t* states, const uint8_t* moves,
                                         const int32_t* num_legal, const float* priors, int64_t count,
                                         int w1, int chk, int w2, int64_t* winning_out,
                                         uint8_t* allowed_out, uint8_t* forced_out, int threads) {
    tables_once();
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int64_t idx = 0; idx < count; idx++) {
        HiveState root;
        std::memcpy(&root, states + idx * sizeof(HiveState), sizeof(root));
        const GPUMove* root_moves = reinterpret_cast<const GPUMove*>(moves) + idx * MAX_LEGAL_MOVES;
        const float* root_priors = priors + idx * MAX_LEGAL_MOVES;
        uint8_t* allowed = allowed_out + idx * MAX_LEGAL_MOVES;
        int nlegal = num_legal[idx];
        winning_out[idx] = -1;
        forced_out[idx] = 0;
        for (int i = 0; i < MAX_LEGAL_MOVES; ++i) allowed[i] = (i < nlegal) ? 1 : 0;
        if (nlegal <= 0 || root.result != IN_PROGRESS) continue;
        Color me = current_player(root);
        Color opp = (me == WHITE) ? BLACK : WHITE;
        int opp_s = queen_surround_count_for_color_device(root, opp);
        int own_s = queen_surround_count_for_color_device(root, me);
        auto won = [&](const HiveState& s) {
            return (me == WHITE && s.result == WHITE_WINS) || (me == BLACK && s.result == BLACK_WINS);
        };
        bool done = false;
        if (w1 && opp_s == 5) {
            int best = -1;
            float bp = -1e30f;
            for (int i = 0; i < nlegal; ++i) {
                HiveState c = root;
                apply_move(c, root_moves[i]);
                if (won(c) && (best < 0 || root_priors[i] > bp)) {
                    best = i;
                    bp = root_priors[i];
                }
            }
            if (best >= 0) {
                winning_out[idx] = best;
                done = true;
            }
        }
        if (!done && chk && own_s == 5) {
            bool any_safe = false;
            for (int i = 0; i < nlegal; ++i) {
                HiveState c = root;
                apply_move(c, root_moves[i]);
                bool bad = has_immediate_surround_win_for_current_player(c);
                allowed[i] = bad ? 0 : 1;
                any_safe |= !bad;
            }
            if (!any_safe) {
                forced_out[idx] = 1;
                done = true;
            }
        }
        if (done || !w2 || !(opp_s == 4 || opp_s == 5)) continue;
        for (int i = 0; i < nlegal; ++i) {
            if (!allowed[i]) continue;
            HiveState c = root;
            apply_move(c, root_moves[i]);
            int cs = queen_surround_count_for_color_device(c, opp);
            if (opp_s == 4 && cs <= opp_s) continue;
            if (opp_s == 5 && cs < opp_s) continue;
            GPUMove replies[MAX_LEGAL_MOVES];
            bool all_nd = true;
            int nr = generate_non_decreasing_surround_replies(c, opp, cs, replies, all_nd);
            if (!all_nd) continue;
            bool ok = true;
            for (int r = 0; r < nr; ++r) {
                HiveState g = c;
                apply_move(g, replies[r]);
                if (!won(g) && !has_immediate_surround_win_for_current_player(g)) {
                    ok = false;
                    break;
                }
            }
            if (ok) {
                winning_out[idx] = i;
                break;
            }
        }
    }
}

// hybrid_transformer_encode_states_kernel / hybrid_transformer_move_features_kernel
// (state_encoder.cuh:552-597): the reference's device functions run per state.
extern "C" void ref_hybrid_encode_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                                        int64_t count, float* tf, int32_t* tq, int32_t* tr, int32_t* tz,
                                        uint8_t* tm, float* gf, int32_t* ntok, float* mf, int threads) {
    tables_once();
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int64_t i = 0; i < count; i++) {
        HiveState s;
        std::memcpy(&s, states + i * sizeof(HiveState), sizeof(s));
        bool mask[HYBRID_MAX_PIECE_TOKENS];
        int n = 0;
        extract_hybrid_transformer_tokens_device(s, tf + i * HYBRID_MAX_PIECE_TOKENS * HYBRID_NODE_FEAT_DIM,
                                                 tq + i * HYBRID_MAX_PIECE_TOKENS, tr + i * HYBRID_MAX_PIECE_TOKENS,
                                                 tz + i * HYBRID_MAX_PIECE_TOKENS, mask,
                                                 gf + i * HYBRID_GLOBAL_FEAT_DIM, n);
        for (int k = 0; k < HYBRID_MAX_PIECE_TOKENS; k++) tm[i * HYBRID_MAX_PIECE_TOKENS + k] = mask[k] ? 1 : 0;
        if (ntok) ntok[i] = n;
        if (mf)
            extract_hybrid_transformer_move_features_device(
                s, reinterpret_cast<const GPUMove*>(moves) + i * MAX_LEGAL_MOVES, num_legal[i],
                mf + i * MAX_LEGAL_MOVES * HYBRID_MOVE_FEAT_DIM);
    }
}

// legal_mask_kernel (state_encoder.cuh:908-976) run per state (blockDim 1)
extern "C" void ref_legal_mask_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                                     int64_t count, float* masks) {
    tables_once();
    std::memset(masks, 0, sizeof(float) * (size_t)count * ACTION_SPACE_SIZE);
    for (int64_t i = 0; i < count; i++) {
        as_thread((int)i);
        legal_mask_kernel(reinterpret_cast<const HiveState*>(states), reinterpret_cast<const GPUMove*>(moves),
                          num_legal, masks, (int)count);
    }
}
