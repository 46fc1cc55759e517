/*
 * hive_oracle.h -- CPU oracle for the Hive self-play hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the
 * reference's game logic (the hive_gpu/csrc headers of chrismejias/hive_neuralnet),
 * used as the parity checker for the CUDA kernels of hive_neuralnet_b200.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may load it.  The product path never does.
 *
 * Parity pinning: tests/test_oracle_vs_ref.py checks every function here
 * against the reference's own headers compiled on the host
 * (oracle/ref_driver.cpp -> oracle/_ref/libhive_ref.so) and against the
 * committed golden fixtures in tests/golden/.
 *
 * The byte layout of hv_state is the reference's HiveState
 * (hive_gpu/csrc/hive_state.cuh:239-269), 3424 bytes, and hv_move is the
 * reference's GPUMove (hive_state.cuh:228-233), 6 bytes; both are the
 * drop-in boundary format and therefore identical by necessity.
 */
#ifndef HIVE_ORACLE_H
#define HIVE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_BOARD 23
#define ORC_HALF 11
#define ORC_CELLS 529
#define ORC_WORDS 9
#define ORC_MAX_STACK 5
#define ORC_MAX_MOVES 256
#define ORC_FEAT 122
#define ORC_STATE_BYTES 3424

#pragma pack(push, 1)
typedef struct {
    uint8_t type;       /* 0 place, 1 move, 2 pass */
    uint8_t pt;         /* 1..8 = Q A G S B M L P, 0 = none */
    uint16_t from;
    uint16_t to;
} orc_move;
#pragma pack(pop)

typedef struct {
    uint8_t pieces[ORC_MAX_STACK][ORC_CELLS];
    uint8_t height[ORC_CELLS];
    uint64_t occupied[ORC_WORDS];
    uint64_t white_top[ORC_WORDS];
    uint64_t black_top[ORC_WORDS];
    uint16_t queen_cell[2];
    uint8_t hands[2][8];
    uint16_t turn;
    uint8_t queen_placed;
    uint8_t result;
    uint16_t stunned_cell;
    int8_t center_q;
    int8_t center_r;
} orc_state;

/* Scalar API (one state). */
void orc_init_tables(void);
void orc_init_state(orc_state* s, int expansion_mask);
void orc_apply_move(orc_state* s, const orc_move* m);
int orc_legal_moves(const orc_state* s, orc_move* out);
int orc_compact_moves(const orc_state* s, orc_move* out);
void orc_features(const orc_state* s, const orc_move* mv, int n, float* f);
void orc_articulation(const orc_state* s, uint64_t* ap_words);
void orc_centroid(const orc_state* s, int* cq, int* cr);
int orc_move_to_action(const orc_move* m, int cq, int cr);
int orc_queen_escape(const orc_state* s);
uint64_t orc_rng(uint64_t seed, uint64_t game, uint64_t ply);
void orc_playout(uint64_t seed, int64_t game, int max_ply, int expansion_mask,
                 orc_state* out);

/* Batched API over contiguous byte buffers.  threads <= 0 uses all cores. */
void orc_generate_positions(uint64_t seed, int64_t first_game, int64_t count,
                            int max_ply, int expansion_mask, uint8_t* states,
                            int threads);
void orc_legal_moves_features_batch(const uint8_t* states, int64_t count,
                                    uint8_t* moves, int32_t* num_legal,
                                    float* feats, int threads);
void orc_legal_moves_batch(const uint8_t* states, int64_t count,
                           uint8_t* moves, int32_t* num_legal, int threads);
void orc_features_batch(const uint8_t* states, const uint8_t* moves,
                        const int32_t* num_legal, int64_t count, float* feats,
                        int threads);
void orc_compact_moves_batch(const uint8_t* states, int64_t count,
                             uint8_t* moves, int32_t* num_legal, int threads);
void orc_successor_features_batch(const uint8_t* states, const uint8_t* moves,
                                  const int64_t* action_to_root,
                                  const int64_t* move_indices, int64_t count,
                                  float* feats, int threads);
void orc_apply_moves_batch(uint8_t* states, const uint8_t* moves, int64_t count);
void orc_articulation_batch(const uint8_t* states, int64_t count,
                            uint64_t* ap_words, int threads);
void orc_actions_batch(const uint8_t* states, const uint8_t* moves,
                       const int32_t* num_legal, int64_t count,
                       int32_t* actions, int32_t* centroids);
void orc_queen_escape_batch(const uint8_t* states, int64_t count, uint8_t* flags);
void orc_tactical_probe(const orc_state* root, const orc_move* moves, int nlegal, const float* priors,
                        int w1, int chk, int w2, int64_t* winning, uint8_t* allowed, uint8_t* forced);
void orc_tactical_probe_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                              const float* priors, int64_t count, int w1, int chk, int w2,
                              int64_t* winning, uint8_t* allowed, uint8_t* forced, int threads);
int orc_hybrid_tokens(const orc_state* s, float* tf, int32_t* tq, int32_t* tr, int32_t* tz, uint8_t* tm,
                      float* gf);
void orc_hybrid_move_features(const orc_state* s, const orc_move* mv, int n, float* out);
void orc_hybrid_encode_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal, int64_t count,
                             float* tf, int32_t* tq, int32_t* tr, int32_t* tz, uint8_t* tm, float* gf,
                             int32_t* ntok, float* mf, int threads);
int orc_num_threads(void);

#ifdef __cplusplus
}
#endif

#endif
