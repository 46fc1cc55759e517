/*
 * hive_b200.h -- C ABI of the B200-native Hive self-play hot path.
 *
 * Plain pointers and sizes only.  Every pointer argument named states /
 * moves / features / ... is DEVICE memory on the current CUDA device; the
 * library never allocates behind the caller's back.  `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Every entry
 * point returns an hv_status; kernels are launched asynchronously on
 * `stream`, and device-side conditions are accumulated in a sticky error
 * word read by hv_get_error().
 *
 * Byte formats at the boundary are the reference's (chrismejias/hive_neuralnet):
 *   state  3424-byte HiveState   hive_gpu/csrc/hive_state.cuh:239-269
 *   move   6-byte GPUMove        hive_gpu/csrc/hive_state.cuh:228-233
 *   moves  [B, 256, 6] uint8, zero padded after num_legal[b]
 *   features [B, 122] float32    hive_gpu/csrc/fnn_features.cuh:21-38
 *
 * Each entry point below names the reference operator it replaces
 * (hive_gpu/csrc/bindings.cpp and the host wrapper in
 * hive_gpu/csrc/game_logic.cu).  Buffers for states and move lists must be
 * 16-byte aligned (torch allocations are).
 */
#ifndef HIVE_B200_H
#define HIVE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HV_ABI_VERSION 1

enum hv_status {
    HV_OK = 0,
    HV_EINVAL = 1,      /* null / misaligned pointer, negative size */
    HV_ECUDA = 2,       /* CUDA runtime or launch error */
    HV_ENOMEM_TREE = 3, /* MCTS node pool exhausted */
    HV_ETIMEOUT = 4,    /* a bounded device wait gave up */
    HV_EDEVICE = 5,     /* device error word set */
    HV_ESCRATCH = 6     /* request larger than a no-alloc entry point's fixed scratch */
};

int hv_version(void);
const char* hv_status_string(int status);

/* Read (and optionally clear) the sticky device error word of the current
 * device.  Synchronous: call it between steps, not inside a hot loop. */
int hv_get_error(uint32_t* out, int clear);

/* Test hook, no counterpart in the reference: set the current device's limit
 * on the tensor-core kernels' bounded waits (mbarrier waits for bulk copies
 * and MMAs; default 1e9 ns).  0 makes every such wait give up at once, with
 * its copy or MMA still in flight: the kernel sets its error bit (4: the
 * hybrid trunk, 8: the row and leaf networks), waits up to 1 s for the work
 * it started, frees its tensor memory and returns, and the call's outputs are
 * undefined.  Synchronous; not for use inside a step. */
int hv_set_wait_limit_ns(uint64_t ns);

/* create_initial_states(batch_size, expansion_mask)
 * replaces bindings.cpp:264-266 / game_logic.cu:413-428.
 * states: [batch, 3424] uint8 (written). */
int hv_create_initial_states(uint8_t* states, int64_t batch, int expansion_mask, void* stream);

/* generate_legal_moves_batch(states, batch_size)
 * replaces bindings.cpp:268-270 / game_logic.cu:436-459. */
int hv_generate_legal_moves(const uint8_t* states, int64_t batch, uint8_t* moves,
                            int32_t* num_legal, void* stream);

/* generate_legal_moves_and_fnn_features_batch(states, batch_size)
 * replaces bindings.cpp:335-338 / game_logic.cu:1440-1464.  `features`
 * must be 8-byte aligned: until the call's feature kernels write them, the
 * feature rows carry working data between its kernels (each row's
 * articulation mask, and position counters in row 0).  The call is
 * hv_generate_legal_moves_linked followed by hv_fnn_features_linked. */
int hv_generate_legal_moves_and_fnn_features(const uint8_t* states, int64_t batch, uint8_t* moves,
                                             int32_t* num_legal, float* features, void* stream);

/* The two halves of hv_generate_legal_moves_and_fnn_features, callable
 * apart so that a caller (a profiler, the benchmark) can time each; no
 * counterpart in the reference, whose fused kernel computes both in one.
 * hv_generate_legal_moves_linked writes the move lists and num_legal and
 * leaves working data in `features` (see above); hv_fnn_features_linked must
 * follow it on the same buffers and stream and writes the features.  Each
 * hv_fnn_features_linked call needs its own hv_generate_legal_moves_linked
 * call just before it: the feature half reads the position counters (bytes
 * 16..23 of row 0) and each row's articulation mask (its first word) that
 * only the generator half leaves behind, and overwrites them.  A second
 * feature half on the same buffers, or one without the generator half
 * first, reads feature values as counters and masks and writes wrong
 * features without any error: the feature half cannot be repeated alone
 * (for example to time it). */
int hv_generate_legal_moves_linked(const uint8_t* states, int64_t batch, uint8_t* moves, int32_t* num_legal,
                                   float* features, void* stream);
int hv_fnn_features_linked(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal, int64_t batch,
                           float* features, void* stream);

/* Host -> device staging of `count` 3424-byte states for the host-buffer
 * pipeline (the reference's callers pass host tensors through .cuda() before
 * generate_legal_moves_and_fnn_features_batch, game_logic.cu:1440-1464).
 * Move generation and feature extraction read stack level L of a cell only
 * when the cell's height exceeds L, so from pinned (device-mapped) host
 * memory this copies each state's heights, bitboards and fields (bytes
 * 2645..3423) with one strided copy, then a kernel reads level L from host
 * memory over the board rows holding a cell higher than L, in 16-byte words.
 * The remaining level bytes of dev_states are left as they were: the staged
 * states are inputs for the read-only kernels, not a byte copy to hand back.
 * Pageable memory, or either pointer off a 16-byte boundary: one full copy.
 * Asynchronous on `stream`; the host buffer must stay valid until the stream
 * reaches it. */
int hv_stage_host_states(const uint8_t* host_states, int64_t count, uint8_t* dev_states, void* stream);

/* The download half of the host-buffer movegen pipeline: a chunk's move
 * rows [count, 256, 6] from the device into pinned host memory, sending
 * over the host link only the first `prefix` moves of every row (one
 * pitched copy) and, for positions with more legal moves, the moves past
 * the prefix (a kernel that stores into the mapped host rows).  Bytes
 * 6*prefix .. 1535 of every host row must already be zero (the caller
 * clears them on the host, before this call; the device rows are zero past
 * num_legal).  prefix: 0 .. 256, a multiple of 8.  Pageable host memory,
 * prefix 256, or either pointer off a 16-byte boundary: one full copy, no
 * precondition.  Asynchronous on `stream`.  No reference counterpart (the
 * reference returns device tensors). */
int hv_download_moves(const uint8_t* dev_moves, const int32_t* dev_num_legal, int64_t count, uint8_t* host_moves,
                      int prefix, void* stream);

/* extract_fnn_features_batch(states, legal_moves, num_legal, batch_size)
 * replaces bindings.cpp:330-333 / game_logic.cu:1409-1431. */
int hv_extract_fnn_features(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                            int64_t batch, float* features, void* stream);

/* fnn_successor_features_batch(states, legal_moves, action_to_root,
 * move_indices, num_actions) replaces bindings.cpp:371-376 /
 * game_logic.cu:1648-1671.  features: [num_actions, 122] float32.
 * num_states bounds action_to_root; an out-of-range (root, move) pair gets a
 * zero row and sets the device error word instead of reading out of bounds. */
int hv_fnn_successor_features(const uint8_t* states, int64_t num_states, const uint8_t* legal_moves,
                              const int64_t* action_to_root, const int64_t* move_indices,
                              int64_t num_actions, float* features, void* stream);

/* FNN leaf evaluation fused with successor generation: the body of
 * FNNMCTSOrchestrator._eval_states (hive_fnn/fnn_mcts_orchestrator.py:243-316)
 * with HiveFNN.encode / value_head / score_actions
 * (hive_fnn/fnn_network.py:98-143), which the reference runs as
 * fnn_successor_features_batch + torch GEMMs + softmax/scatter.
 * Per leaf p (count leaves): priors[p, 0..255] = softmax of the successor
 * logits over the num_legal[p] slots (zero elsewhere); values[p] = root value;
 * child_q[p, i] = -value(successor i) (zero past num_legal).  root_features
 * [count, 122] may be NULL (computed from states + legal_moves); logits
 * [count, 256] may be NULL.  weights: packed fp32 (layout in
 * hive_neuralnet_b200/fnn.py pack_weights); dims 1..64. */
int hv_fnn_eval_leaves(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                       const float* root_features, int64_t count, const float* weights, int hidden,
                       int embed, int action_hidden, float* priors, float* values, float* child_q,
                       float* logits, void* stream);

/* number of floats hv_fnn_eval_leaves expects in `weights` */
int hv_fnn_weights_size(int hidden, int embed, int action_hidden);

/* ---------------------------------------------------------------------------
 * MCTS tree: the reference's SoA tree (hive_gpu/csrc/mcts_tree.cuh:31-45),
 * per-game arrays [B, max_nodes] in the binding order of bindings.cpp:130-135.
 * Every tree entry point processes the simulations of one game in
 * simulation-index order (sim = j * B + game), which is the reference's
 * kernel semantics with its concurrent simulations serialised: results are
 * deterministic and equal to the reference kernels run one simulation at a
 * time in index order.
 * ------------------------------------------------------------------------- */
typedef struct hv_tree {
    int32_t* visit_count;      /* [B, max_nodes] */
    float* total_value;        /* [B, max_nodes] */
    float* prior;              /* [B, max_nodes] */
    int32_t* parent_idx;       /* [B, max_nodes], -1 = none */
    float* virtual_q_penalty;  /* [B, max_nodes] */
    uint8_t* move_bytes;       /* [B, max_nodes, 6] */
    int32_t* action_idx;       /* [B, max_nodes], -1 = none */
    int32_t* first_child;      /* [B, max_nodes], -1 = unexpanded */
    int32_t* num_children;     /* [B, max_nodes] */
    int8_t* is_terminal;       /* [B, max_nodes] */
    float* terminal_value;     /* [B, max_nodes] */
    int32_t* node_count;       /* [B] */
    int32_t max_nodes;
} hv_tree;

/* Selection with virtual loss.  mode 0: mcts_select_batch (bindings.cpp:
 * 112-116, mcts_tree.cuh:205-291), W * B simulations; mode 1:
 * mcts_select_with_root_mask_batch (:166-175, :689-800) with alive_mask
 * [B, max_root_children]; mode 2: mcts_select_with_root_slots_batch
 * (:177-186, :811-955) with root_slots [B, num_candidates], W * C * B
 * simulations.  Outputs leaf [T], move_paths [T,128,6], path_len [T],
 * vl_paths [T,128], vl_len [T]. */
int hv_mcts_select(const hv_tree* tree, int mode, const float* child_init_q, const int8_t* game_active,
                   const int32_t* root_nodes, const int8_t* alive_mask, const int32_t* root_slots,
                   int num_candidates, int max_root_children, float c_puct, int B, int W,
                   int deterministic_non_root, float non_root_sigma, float q_penalty, int32_t* leaf,
                   uint8_t* move_paths, int32_t* path_len, int32_t* vl_paths, int32_t* vl_len,
                   void* stream);

/* mcts_replay_batch (bindings.cpp:118-121, mcts_tree.cuh:298-320):
 * leaf_states[s] = root_states[s % B] + move path s; a slot with leaf[s] < 0
 * (no simulation) is written as an all-zero state, where the reference
 * leaves its buffer as it was (its callers zero-fill it, the rows are
 * unused), so a caller needs no zero-fill before the call. */
int hv_mcts_replay(const uint8_t* root_states, uint8_t* leaf_states, const uint8_t* move_paths,
                   const int32_t* path_len, const int32_t* leaf, int B, int total, void* stream);

/* Expansion, optionally fused with the backup.
 * dense=1: per-legal priors [T,256] + child_q -> child_init_q
 *   (mcts_expand_dense_priors_batch / ..._and_backprop_dense_priors_batch,
 *    bindings.cpp:200-219, mcts_tree.cuh:971-1187);
 * dense=0: action-space priors [T,85834] (mcts_expand_batch /
 *   mcts_expand_and_backprop_batch, bindings.cpp:123-147, :330-549).
 * was_expanded [T] is written when backprop=0 (may be NULL). */
int hv_mcts_expand(const hv_tree* tree, int dense, int backprop, float* child_init_q,
                   const float* child_q, const int32_t* leaf, const uint8_t* leaf_states,
                   const uint8_t* legal_moves, const int32_t* num_legal, const float* priors,
                   const int32_t* results, const float* values, const int32_t* vl_paths,
                   const int32_t* vl_len, int8_t* was_expanded, float q_penalty, int B, int total,
                   void* stream);

/* hv_mcts_expand with dense = 1 and backprop = 1, for the simulations of
 * one hv_mcts_select call with the same root_nodes:
 *   root_slots != NULL: a root-slot select (mode 2, the same root_slots;
 *     total = W * num_candidates * B, simulation s below candidate
 *     (s / B) % num_candidates of game s % B);
 *   root_slots == NULL: a plain or root-mask select (modes 0, 1: each
 *     simulation's virtual-loss path starts at its root child).
 * The tree it leaves is the one hv_mcts_expand leaves: node allocation in
 * simulation order, root-level backups in simulation order; the subtrees
 * below different candidates / root children, which no two groups share,
 * are updated in parallel.  A game whose candidate table repeats a slot, or
 * a shape outside num_candidates <= 32 and total / B <= 1024, runs
 * hv_mcts_expand's kernel.  No reference counterpart as a separate call:
 * the reference's waves call mcts_expand_and_backprop_dense_priors_batch
 * (bindings.cpp:200-219). */
int hv_mcts_expand_slots(const hv_tree* tree, float* child_init_q, const float* child_q, const int32_t* leaf,
                         const uint8_t* leaf_states, const uint8_t* legal_moves, const int32_t* num_legal,
                         const float* priors, const int32_t* results, const float* values,
                         const int32_t* vl_paths, const int32_t* vl_len, const int32_t* root_nodes,
                         const int32_t* root_slots, int num_candidates, float q_penalty, int B, int total,
                         void* stream);

/* mcts_backprop_batch (bindings.cpp:131-136, mcts_tree.cuh:555-605). */
int hv_mcts_backprop(const hv_tree* tree, const int32_t* leaf, const float* values,
                     const int32_t* vl_paths, const int32_t* vl_len, const int8_t* was_expanded, int B,
                     int total, void* stream);

/* mcts_apply_root_noise (bindings.cpp:221-226, mcts_tree.cuh:1192-1234). */
int hv_mcts_root_noise(const hv_tree* tree, const float* noise, const int32_t* root_nodes,
                       int max_children_pad, float dir_eps, float root_policy_temp, int B,
                       void* stream);

/* mcts_extract_policy_batch (bindings.cpp:149-155, mcts_tree.cuh:607-684):
 * policies [B, 85834] must be zeroed by the caller. */
int hv_mcts_extract_policy(const hv_tree* tree, float* policies, const int32_t* move_numbers,
                           const int32_t* root_nodes, float temperature, int temp_drop_move,
                           float pruning_threshold, int B, void* stream);

/* queen_escape_flags_batch(states, batch_size) replaces bindings.cpp:339-342 /
 * game_logic.cu:1538-1554: flags[b] = 1 when the side to move's queen has a
 * slide or a pillbug / pillbug-adjacent mosquito throw (move_gen.cuh:771-821). */
int hv_queen_escape_flags(const uint8_t* states, int64_t batch, uint8_t* flags, void* stream);

/* Per (state b, legal slot m < num_legal[b]): the child after move m, its
 * result (check_results), the occupied-neighbour count of the child's
 * side-to-move queen and (want_escape) its queen-escape flag; outputs
 * [batch, 256], zero past num_legal.  Replaces the per-successor
 * apply_moves_batch + check_results_batch + queen_escape_flags_batch
 * passes of FNNMCTSOrchestrator._find_immediate_wins and
 * _queen_surround_qualifying_mask (hive_fnn/fnn_mcts_orchestrator.py:339-493). */
int hv_child_probe(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                   int64_t batch, int want_escape, int32_t* results, int32_t* surround,
                   uint8_t* escape, void* stream);

/* hybrid_transformer_encode_with_moves_batch(states, legal_moves, num_legal, batch_size)
 * replaces bindings.cpp:48-52,361-363 / game_logic.cu:652-702 (the move list
 * is not read by the token encoder, so it is not an argument here).
 * token_features [batch, 28, 27] f32, token_q/r/z [batch, 28] i32 (column,
 * row, stack level), token_mask [batch, 28] u8 (0/1, torch bool),
 * global_features [batch, 6] f32, num_tokens [batch] i32.  Every element of
 * every output is written. */
int hv_hybrid_encode(const uint8_t* states, int64_t batch, float* token_features, int32_t* token_q,
                     int32_t* token_r, int32_t* token_z, uint8_t* token_mask, float* global_features,
                     int32_t* num_tokens, void* stream);

/* hybrid_transformer_move_features_batch(states, legal_moves, num_legal, batch_size)
 * replaces bindings.cpp:110-114,356-358 / game_logic.cu:704-727.
 * move_features [batch, 256, 31] f32, zero past num_legal. */
int hv_hybrid_move_features(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            int64_t batch, float* move_features, void* stream);

/* generate_legal_moves_and_hybrid_root_features_batch(states, batch_size)
 * replaces bindings.cpp:78-81,322-324 / game_logic.cu:93-131,1469-1535:
 * legal moves, FNN features, piece tokens and move features in one pass. */
int hv_generate_legal_moves_and_hybrid_root_features(const uint8_t* states, int64_t batch, uint8_t* moves,
                                                     int32_t* num_legal, float* fnn_features, float* token_features,
                                                     int32_t* token_q, int32_t* token_r, int32_t* token_z,
                                                     uint8_t* token_mask, float* global_features,
                                                     int32_t* num_tokens, float* move_features, void* stream);

/* Relative transformer trunk of the hybrid evaluator (hive_fnn_transformer/
 * fnn_transformer_net.py:159-209 HybridRelativeTransformerTrunk.forward), the
 * default / `small` presets: hidden 64, 8 heads, MLP 96, 4 blocks.  Inputs are
 * hv_hybrid_encode's outputs (token_features [batch, 28, 27], first
 * node_feat_dim columns used); weight_image (fp16 bits) and params (f32) are
 * packed by hive_neuralnet_b200.hybrid.pack_trunk, sizes from
 * hv_hybrid_trunk_sizes.  graph_summary [batch, 64] f32.  No reference
 * counterpart as a single call: it replaces the torch module's forward. */
int hv_hybrid_trunk_sizes(int* image_elems, int* param_floats);
int hv_hybrid_trunk(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                    const int32_t* token_z, const uint8_t* token_mask, int64_t batch, int node_feat_dim,
                    const uint16_t* weight_image, const float* params, float* graph_summary, void* stream);

/* hv_hybrid_trunk with the positions packed: two positions whose valid
 * tokens all lie in their first 15 token slots share one 32-row slot of the
 * kernel's tiles (16 rows each), so a batch of early-game positions takes
 * fewer rows; when fewer than a quarter of the batch qualify, one position
 * per slot as in hv_hybrid_trunk.  The same graph_summary bit for bit (rows
 * are independent in every GEMM and LayerNorm, and a position attends
 * within its own rows).
 * workspace: 16-byte aligned, at least
 * hv_hybrid_trunk_packed_workspace_bytes(batch) bytes (the slot table,
 * built on the device); batch <= 2^31 - 1.  No reference counterpart. */
int hv_hybrid_trunk_packed_workspace_bytes(int64_t batch, size_t* bytes);
int hv_hybrid_trunk_packed(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                           const int32_t* token_z, const uint8_t* token_mask, int64_t batch, int node_feat_dim,
                           const uint16_t* weight_image, const float* params, float* graph_summary, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Hybrid leaf evaluation: HybridMCTSOrchestrator._eval_states
 * (hive_fnn_transformer/fnn_transformer_mcts_orchestrator.py:42-169) given
 * the trunk's graph_summary [count, 64] and the encoder's global_features
 * [count, 6]: FNN encode of the root (root_features [count, 122] or NULL to
 * compute them) and of every legal successor, tanh value head, hybrid action
 * scores, masked softmax.  priors / child_q / logits [count, 256] (child_q is
 * zero, as in the reference), values [count].  fnn_weights as for
 * hv_fnn_eval_leaves; head_weights packed by
 * hive_neuralnet_b200.hybrid.pack_heads (hv_hybrid_head_weights_size floats). */
int hv_hybrid_head_weights_size(int embed, int action_hidden, int value_hidden);
int hv_hybrid_eval_leaves(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                          const float* root_features, const float* graph_summary, const float* global_features,
                          int64_t count, const float* fnn_weights, int hidden, int embed, int action_hidden,
                          const float* head_weights, int value_hidden, float* priors, float* values,
                          float* child_q, float* logits, void* stream);

/* The whole hybrid leaf evaluation in one call (HybridMCTSOrchestrator._eval_states,
 * hive_fnn_transformer/fnn_transformer_mcts_orchestrator.py:42-169): piece
 * tokens (hv_hybrid_encode) -> trunk (hv_hybrid_trunk) -> heads
 * (hv_hybrid_eval_leaves).  The intermediate tokens and summaries live in the
 * caller's device workspace: 256-byte aligned, at least
 * hv_hybrid_workspace_bytes(count) bytes.  Nothing is allocated. */
int hv_hybrid_workspace_bytes(int64_t count, size_t* bytes);
int hv_hybrid_evaluate(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                       const float* root_features, int64_t count, int node_feat_dim, const uint16_t* trunk_image,
                       const float* trunk_params, const float* fnn_weights, int hidden, int embed,
                       int action_hidden, const float* head_weights, int value_hidden, float* priors,
                       float* values, float* child_q, float* logits, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Dense legal-action mask: legal_mask_kernel (state_encoder.cuh:908-976), the
 * second half of generate_legal_mask_batch / generate_legal_moves_and_mask_batch
 * (bindings.cpp:54-57, game_logic.cu:737-809).  masks [batch, 85834] f32
 * (8-byte aligned): 1.0 at every legal move's action index inside the 17x17
 * window around the centroid, 0 elsewhere; every element is written. */
int hv_legal_mask(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal, int64_t batch,
                  float* masks, void* stream);

/* No-alloc variant of hv_hybrid_evaluate (no reference counterpart): the
 * same evaluation, with the intermediate tokens and summaries in a fixed
 * 32 MiB file-scope device array instead of a caller workspace, so a caller
 * that owns no device allocator can still run it.  At most 9137 positions per
 * call; larger requests return HV_ESCRATCH and launch nothing.  The scratch
 * address is looked up on the first call in each device context (once per
 * device, and again after the context was reset and re-created, e.g. by
 * cudaDeviceReset), so make the first call before any stream capture.  The
 * scratch is shared by every call on a device: calls that overlap (other
 * streams, other host threads) race. */
int hv_hybrid_evaluate_noalloc(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                               const float* root_features, int64_t count, int node_feat_dim,
                               const uint16_t* trunk_image, const float* trunk_params, const float* fnn_weights,
                               int hidden, int embed, int action_hidden, const float* head_weights,
                               int value_hidden, float* priors, float* values, float* child_q, float* logits,
                               void* stream);

/* Leaf evaluation as a row pipeline, the evaluators' default path: the
 * successors of all `count` leaves are compacted into `rows` rows
 * (rows = sum over leaves of min(max(num_legal, 0), 256)), their features
 * written to the workspace, the network run as a tiled fp32 GEMM pipeline
 * over rows, the per-leaf parts and the softmax by warp-per-leaf kernels
 * (the hybrid trunk runs packed, as hv_hybrid_trunk_packed).
 * Same outputs as hv_fnn_eval_leaves / hv_hybrid_evaluate (fp32, a
 * different summation order).  workspace: 256-byte aligned, at least
 * hv_leaf_rows_workspace_bytes(count, rows, hybrid) bytes; with logits ==
 * NULL the raw logits live in the workspace.  Rows beyond `rows` are dropped
 * (device error word bit 0). */
int hv_leaf_rows_workspace_bytes(int64_t count, int64_t rows, int hybrid, size_t* bytes);
int hv_fnn_eval_leaves_rows(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            const float* root_features, int64_t count, int64_t rows, const float* weights,
                            int hidden, int embed, int action_hidden, float* priors, float* values, float* child_q,
                            float* logits, void* workspace, size_t workspace_bytes, void* stream);
int hv_hybrid_evaluate_rows(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            const float* root_features, int64_t count, int64_t rows, int node_feat_dim,
                            const uint16_t* trunk_image, const float* trunk_params, const float* fnn_weights,
                            int hidden, int embed, int action_hidden, const float* head_weights, int value_hidden,
                            float* priors, float* values, float* child_q, float* logits, void* workspace,
                            size_t workspace_bytes, void* stream);

/* root_tactical_probe_batch(states, legal_moves, num_legal, priors, batch_size,
 *     enable_win_in_one, enable_check_opponent_wins, enable_win_in_two)
 * replaces bindings.cpp:91-100,336-339 / game_logic.cu:290-397,1579-1615.
 * priors: [batch, 256] f32.  Outputs: winning_move [batch] i64 (-1 none),
 * allowed_slots [batch, 256] u8, forced_random [batch] u8.  The outputs
 * need no initialisation: every byte is written. */
int hv_root_tactical_probe(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                           const float* priors, int64_t batch, int enable_win_in_one,
                           int enable_check_opponent_wins, int enable_win_in_two, int64_t* winning_move,
                           uint8_t* allowed_slots, uint8_t* forced_random, void* stream);

/* apply_moves_batch(states, moves, batch_size)
 * replaces bindings.cpp:272-274 / game_logic.cu:465-477.  moves: [batch, 6]. */
int hv_apply_moves(uint8_t* states, const uint8_t* moves, int64_t batch, void* stream);

/* check_results_batch(states, batch_size)
 * replaces bindings.cpp:276-278 / game_logic.cu:483-497. */
int hv_check_results(const uint8_t* states, int64_t batch, int32_t* results, void* stream);

/* compute_centroids_batch(states, batch_size)
 * replaces bindings.cpp:302-304 / game_logic.cu:910-926.  centroids: [batch, 2]. */
int hv_compute_centroids(const uint8_t* states, int64_t batch, int32_t* centroids, void* stream);

/* legal_moves_to_actions_batch(states, legal_moves, num_legal, batch_size)
 * replaces bindings.cpp:306-309 / game_logic.cu:837-857.  actions: [batch, 256]. */
int hv_legal_moves_to_actions(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                              int64_t batch, int32_t* actions, void* stream);

/* Seeded uniform random legal playouts: game g of the batch is game
 * first_game + g; stop ply U[0, max_ply]; at each ply the move index is a
 * counter-based splitmix64 draw modulo num_legal.  Benchmark/test inputs in
 * the spirit of hive_gpu/endgame_generator.py:284-289 (random playouts). */
int hv_generate_positions(uint64_t seed, int64_t first_game, int64_t count, int max_ply,
                          int expansion_mask, uint8_t* states, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HIVE_B200_H */
