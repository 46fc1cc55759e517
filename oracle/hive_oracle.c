/*
 * hive_oracle.c -- CPU oracle (TEST INFRASTRUCTURE ONLY) for the Hive
 * self-play hot path.  A plain-C restatement of the reference game logic of
 * chrismejias/hive_neuralnet; each function cites the reference file:line it
 * restates.  It is the checker for the CUDA kernels, never a product path.
 *
 * Reference files (paths inside the reference project):
 *   hive_gpu/csrc/hex_grid.cuh      grid, directions, neighbour tables
 *   hive_gpu/csrc/hive_state.cuh    state layout, place/move/apply, game over
 *   hive_gpu/csrc/articulation.cuh  One-Hive articulation points
 *   hive_gpu/csrc/move_gen.cuh      full and compact legal move generation
 *   hive_gpu/csrc/fnn_features.cuh  122-float FNN feature vector
 *   hive_gpu/csrc/state_encoder.cuh centroid and banker's rounding
 *   hive_gpu/csrc/mcts_tree.cuh     move -> action index
 *
 * The articulation points are computed here by a different algorithm than
 * the reference's Tarjan DFS (vertex removal + reachability); the results
 * are identical by the standard theorem and are cross-checked against the
 * compiled reference in tests/test_oracle_vs_ref.py.
 */
#include "hive_oracle.h"

#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* Grid (hex_grid.cuh:24-49, 69-108)                                   */
/* ------------------------------------------------------------------ */

/* Direction order E, NE, NW, W, SW, SE as (dcol, drow). */
static const int DCOL[6] = {+1, +1, 0, -1, -1, 0};
static const int DROW[6] = {0, -1, -1, 0, +1, +1};

static int16_t NB[ORC_CELLS][6];
static int tables_ready = 0;

void orc_init_tables(void) {
    if (tables_ready) return;
    for (int c = 0; c < ORC_CELLS; c++) {
        int row = c / ORC_BOARD, col = c % ORC_BOARD;
        for (int d = 0; d < 6; d++) {
            int r2 = row + DROW[d], c2 = col + DCOL[d];
            NB[c][d] = (r2 >= 0 && r2 < ORC_BOARD && c2 >= 0 && c2 < ORC_BOARD)
                           ? (int16_t)(r2 * ORC_BOARD + c2)
                           : (int16_t)-1;
        }
    }
    tables_ready = 1;
}

/* clockwise / counter-clockwise flank directions (hex_grid.cuh:43-46) */
static inline int cw_of(int d) { return (d + 5) % 6; }
static inline int ccw_of(int d) { return (d + 1) % 6; }

static inline int bb_get(const uint64_t* w, int cell) {
    return (int)((w[cell >> 6] >> (cell & 63)) & 1u);
}
static inline void bb_set(uint64_t* w, int cell) { w[cell >> 6] |= 1ull << (cell & 63); }
static inline void bb_clr(uint64_t* w, int cell) { w[cell >> 6] &= ~(1ull << (cell & 63)); }
static inline int bb_pop(const uint64_t* w) {
    int n = 0;
    for (int i = 0; i < ORC_WORDS; i++) n += __builtin_popcountll(w[i]);
    return n;
}

#define OCC(s, c) bb_get((s)->occupied, (c))
#define TOP_BYTE(s, c) ((s)->height[c] ? (s)->pieces[(s)->height[c] - 1][c] : 0)
#define TOP_TYPE(s, c) (TOP_BYTE(s, c) & 0x0F)
#define BYTE_COLOR(b) (((b) >> 4) & 1)
#define HGT(s, c) ((c) >= 0 ? (int)(s)->height[c] : 0)

static inline int imax(int a, int b) { return a > b ? a : b; }

/* ------------------------------------------------------------------ */
/* State mutation (hive_state.cuh:321-517)                             */
/* ------------------------------------------------------------------ */

static const uint8_t PER_TYPE[8] = {1, 3, 3, 2, 2, 1, 1, 1};

void orc_init_state(orc_state* s, int expansion_mask) {
    /* hive_state.cuh:454-492 */
    memset(s, 0, sizeof(*s));
    s->queen_cell[0] = s->queen_cell[1] = 0xFFFF;
    for (int c = 0; c < 2; c++) {
        for (int p = 0; p < 5; p++) s->hands[c][p] = PER_TYPE[p];
        s->hands[c][5] = (expansion_mask & 1) ? 1 : 0;
        s->hands[c][6] = (expansion_mask & 2) ? 1 : 0;
        s->hands[c][7] = (expansion_mask & 4) ? 1 : 0;
    }
    s->stunned_cell = 0xFFFF;
}

static void set_top_color(orc_state* s, int cell, int color) {
    if (color == 0) {
        bb_set(s->white_top, cell);
        bb_clr(s->black_top, cell);
    } else {
        bb_set(s->black_top, cell);
        bb_clr(s->white_top, cell);
    }
}

/* place_piece, hive_state.cuh:321-353: refused silently on a full stack */
static void place_piece(orc_state* s, int cell, int pt, int color) {
    int h = s->height[cell];
    if (h >= ORC_MAX_STACK) return;
    s->pieces[h][cell] = (uint8_t)(pt | (color << 4));
    s->height[cell] = (uint8_t)(h + 1);
    if (h == 0) bb_set(s->occupied, cell);
    set_top_color(s, cell, color);
    if (pt == 1) {
        s->queen_cell[color] = (uint16_t)cell;
        s->queen_placed |= (uint8_t)(1 << color);
    }
    s->hands[color][pt - 1]--;
}

/* remove_top, hive_state.cuh:359-384 */
static uint8_t remove_top(orc_state* s, int cell) {
    int h = s->height[cell];
    if (h <= 0) return 0;
    uint8_t b = s->pieces[h - 1][cell];
    s->pieces[h - 1][cell] = 0;
    s->height[cell] = (uint8_t)(h - 1);
    if (h == 1) {
        bb_clr(s->occupied, cell);
        bb_clr(s->white_top, cell);
        bb_clr(s->black_top, cell);
    } else {
        set_top_color(s, cell, BYTE_COLOR(s->pieces[h - 2][cell]));
    }
    return b;
}

/* move_piece, hive_state.cuh:390-428: a full destination stack is a no-op */
static void move_piece(orc_state* s, int from, int to) {
    if (s->height[from] == 0) return;
    if (s->height[to] >= ORC_MAX_STACK) return;
    uint8_t b = remove_top(s, from);
    int h = s->height[to];
    s->pieces[h][to] = b;
    s->height[to] = (uint8_t)(h + 1);
    if (h == 0) bb_set(s->occupied, to);
    set_top_color(s, to, BYTE_COLOR(b));
    if ((b & 0x0F) == 1) s->queen_cell[BYTE_COLOR(b)] = (uint16_t)to;
}

static int occupied_neighbours(const orc_state* s, int cell) {
    int n = 0;
    for (int d = 0; d < 6; d++) {
        int nb = NB[cell][d];
        if (nb >= 0 && OCC(s, nb)) n++;
    }
    return n;
}

/* check_game_over, hive_state.cuh:433-448 */
static void check_game_over(orc_state* s) {
    int surr[2];
    for (int c = 0; c < 2; c++)
        surr[c] = ((s->queen_placed >> c) & 1) && occupied_neighbours(s, s->queen_cell[c]) == 6;
    if (surr[0] && surr[1]) s->result = 3;
    else if (surr[0]) s->result = 2;
    else if (surr[1]) s->result = 1;
}

/* apply_move, hive_state.cuh:497-517 */
void orc_apply_move(orc_state* s, const orc_move* m) {
    int color = s->turn & 1;
    if (m->type == 0) {
        if (m->to < ORC_CELLS && m->pt >= 1 && m->pt <= 8) place_piece(s, m->to, m->pt, color);
        s->stunned_cell = 0xFFFF;
    } else if (m->type == 1) {
        if (m->from < ORC_CELLS && m->to < ORC_CELLS) {
            move_piece(s, m->from, m->to);
            s->stunned_cell = m->to;
        }
    } else {
        s->stunned_cell = 0xFFFF;
    }
    s->turn++;
    check_game_over(s);
}

/* ------------------------------------------------------------------ */
/* One-Hive articulation points (articulation.cuh:34-179)              */
/* ------------------------------------------------------------------ */

/*
 * The reference runs Tarjan's DFS from the lowest occupied cell only, so the
 * result is the articulation-point set of that cell's connected component
 * (empty when fewer than three cells are occupied).  Restated here as: a cell
 * v of that component is an articulation point iff removing v leaves the rest
 * of the component unreachable from one of its remaining cells.
 */
void orc_articulation(const orc_state* s, uint64_t* ap) {
    memset(ap, 0, sizeof(uint64_t) * ORC_WORDS);
    int cells[32], n = 0;
    for (int c = 0; c < ORC_CELLS && n < 28; c++)
        if (OCC(s, c)) cells[n++] = c;
    if (n <= 2) return;
    uint32_t adj[32];
    for (int i = 0; i < n; i++) {
        adj[i] = 0;
        for (int d = 0; d < 6; d++) {
            int nb = NB[cells[i]][d];
            if (nb < 0 || !OCC(s, nb)) continue;
            for (int j = 0; j < n; j++)
                if (cells[j] == nb) adj[i] |= 1u << j;
        }
    }
    /* reach(start, removed): vertices reachable from start avoiding removed */
    uint32_t comp = 0;
    {
        uint32_t frontier = 1u;
        comp = 1u;
        while (frontier) {
            int v = __builtin_ctz(frontier);
            frontier &= frontier - 1;
            uint32_t nw = adj[v] & ~comp;
            comp |= nw;
            frontier |= nw;
        }
    }
    for (int x = 0; x < n; x++) {
        if (!((comp >> x) & 1)) continue;
        uint32_t rest = comp & ~(1u << x);
        if (!rest) continue;
        int start = __builtin_ctz(rest);
        uint32_t seen = 1u << start, frontier = seen;
        while (frontier) {
            int v = __builtin_ctz(frontier);
            frontier &= frontier - 1;
            uint32_t nw = adj[v] & rest & ~seen;
            seen |= nw;
            frontier |= nw;
        }
        if (seen != rest) bb_set(ap, cells[x]);
    }
}

typedef struct {
    uint64_t pinned[ORC_WORDS];
    uint64_t perimeter[ORC_WORDS];
} gen_ctx;

/* init_movegen_state_cache, move_gen.cuh:161-178; perimeter :133-152 */
static void ctx_init(const orc_state* s, gen_ctx* g) {
    uint64_t ap[ORC_WORDS];
    orc_articulation(s, ap);
    memset(g, 0, sizeof(*g));
    for (int c = 0; c < ORC_CELLS; c++) {
        if (bb_get(ap, c) && s->height[c] == 1) bb_set(g->pinned, c);
        if (OCC(s, c)) {
            for (int d = 0; d < 6; d++) {
                int nb = NB[c][d];
                if (nb >= 0 && !OCC(s, nb)) bb_set(g->perimeter, nb);
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* Piece movement (move_gen.cuh:82-1049)                               */
/* ------------------------------------------------------------------ */

/* can_slide, move_gen.cuh:82-104 (skip = the moving piece's cell) */
static int slide_ok(const orc_state* s, int from, int d, int skip) {
    int dest = NB[from][d];
    if (dest < 0) return 0;
    if (OCC(s, dest) && dest != skip) return 0;
    int a = NB[from][cw_of(d)], b = NB[from][ccw_of(d)];
    int ao = a >= 0 && OCC(s, a) && a != skip;
    int bo = b >= 0 && OCC(s, b) && b != skip;
    return ao != bo;
}

/* can_slide_ant_occ, move_gen.cuh:120-131 (occ excludes the ant) */
static int ant_step_ok(const uint64_t* occ, const uint64_t* perim, int from, int d) {
    int dest = NB[from][d];
    if (dest < 0 || !bb_get(perim, dest)) return 0;
    int a = NB[from][cw_of(d)], b = NB[from][ccw_of(d)];
    int ao = a >= 0 && bb_get(occ, a);
    int bo = b >= 0 && bb_get(occ, b);
    return ao != bo;
}

/* elevated gate, move_gen.cuh:659-667 */
static int gate_blocked(const orc_state* s, int from, int d, int h) {
    int a = NB[from][cw_of(d)], b = NB[from][ccw_of(d)];
    return HGT(s, a) > h && HGT(s, b) > h;
}

static int queen_dests(const orc_state* s, int cell, uint16_t* out) {
    int n = 0; /* move_gen.cuh:202-212 */
    for (int d = 0; d < 6; d++)
        if (slide_ok(s, cell, d, cell)) out[n++] = (uint16_t)NB[cell][d];
    return n;
}

static int hopper_dests(const orc_state* s, int cell, uint16_t* out) {
    int n = 0; /* move_gen.cuh:228-245 */
    for (int d = 0; d < 6; d++) {
        int p = NB[cell][d];
        if (p < 0 || !OCC(s, p)) continue;
        while (p >= 0 && OCC(s, p)) p = NB[p][d];
        if (p >= 0) out[n++] = (uint16_t)p;
    }
    return n;
}

/*
 * Ant breadth-first search, move_gen.cuh:267-313 (capped list) and
 * :348-388 (emitting straight into the move list).  The queue is the output
 * itself; cap bounds the number of destinations.
 */
static int ant_bfs(const orc_state* s, int cell, const uint64_t* perim, uint16_t* q, int cap) {
    uint64_t occ[ORC_WORDS], seen[ORC_WORDS];
    memcpy(occ, s->occupied, sizeof(occ));
    bb_clr(occ, cell);
    memset(seen, 0, sizeof(seen));
    bb_set(seen, cell);
    int rd = 0, wr = 0;
    if (cap <= 0) return 0;
    for (int d = 0; d < 6 && wr < cap; d++) {
        if (!ant_step_ok(occ, perim, cell, d)) continue;
        int dest = NB[cell][d];
        if (bb_get(seen, dest)) continue;
        bb_set(seen, dest);
        q[wr++] = (uint16_t)dest;
    }
    while (rd < wr && wr < cap) {
        int cur = q[rd++];
        for (int d = 0; d < 6; d++) {
            if (!ant_step_ok(occ, perim, cur, d)) continue;
            int dest = NB[cur][d];
            if (bb_get(seen, dest)) continue;
            bb_set(seen, dest);
            q[wr++] = (uint16_t)dest;
            if (wr >= cap) break;
        }
    }
    return wr;
}

static int ant_any(const orc_state* s, int cell, const uint64_t* perim) {
    uint64_t occ[ORC_WORDS]; /* move_gen.cuh:330-338 */
    memcpy(occ, s->occupied, sizeof(occ));
    bb_clr(occ, cell);
    for (int d = 0; d < 6; d++)
        if (ant_step_ok(occ, perim, cell, d)) return 1;
    return 0;
}

/* spider: exactly three slides, first-seen order, at most 32 (move_gen.cuh:397-431) */
static int spider_dests(const orc_state* s, int cell, uint16_t* out, int first_only) {
    uint64_t got[ORC_WORDS];
    memset(got, 0, sizeof(got));
    int n = 0;
    for (int d1 = 0; d1 < 6; d1++) {
        if (!slide_ok(s, cell, d1, cell)) continue;
        int p1 = NB[cell][d1];
        for (int d2 = 0; d2 < 6; d2++) {
            if (!slide_ok(s, p1, d2, cell)) continue;
            int p2 = NB[p1][d2];
            if (p2 == cell || p2 == p1) continue;
            for (int d3 = 0; d3 < 6; d3++) {
                if (!slide_ok(s, p2, d3, cell)) continue;
                int p3 = NB[p2][d3];
                if (p3 == cell || p3 == p1 || p3 == p2) continue;
                if (first_only) return 1;
                if (!bb_get(got, p3) && n < 32) {
                    bb_set(got, p3);
                    out[n++] = (uint16_t)p3;
                }
            }
        }
    }
    return n;
}

/* beetle, move_gen.cuh:468-524 */
static int beetle_dests(const orc_state* s, int cell, uint16_t* out, int first_only) {
    int n = 0, below = s->height[cell] - 1;
    for (int d = 0; d < 6; d++) {
        int dest = NB[cell][d];
        if (dest < 0) continue;
        int mh = imax(s->height[dest], below);
        int ok = mh > 0 ? !gate_blocked(s, cell, d, mh) : slide_ok(s, cell, d, cell);
        if (!ok) continue;
        if (first_only) return 1;
        out[n++] = (uint16_t)dest;
    }
    return n;
}

/* ladybug: up, across, down; first-seen order, at most 32 (move_gen.cuh:538-637) */
static int ladybug_dests(const orc_state* s, int cell, uint16_t* out, int first_only) {
    uint64_t got[ORC_WORDS];
    memset(got, 0, sizeof(got));
    int n = 0;
    for (int d1 = 0; d1 < 6; d1++) {
        int p1 = NB[cell][d1];
        if (p1 < 0 || !OCC(s, p1)) continue;
        int h1 = imax(s->height[cell] - 1, s->height[p1]);
        if (gate_blocked(s, cell, d1, h1)) continue;
        for (int d2 = 0; d2 < 6; d2++) {
            int p2 = NB[p1][d2];
            if (p2 < 0 || p2 == cell || !OCC(s, p2)) continue;
            int h2 = imax(s->height[p1], s->height[p2]);
            if (gate_blocked(s, p1, d2, h2)) continue;
            for (int d3 = 0; d3 < 6; d3++) {
                int p3 = NB[p2][d3];
                if (p3 < 0 || p3 == cell || p3 == p1 || OCC(s, p3)) continue;
                if (gate_blocked(s, p2, d3, s->height[p2])) continue;
                if (first_only) return 1;
                if (!bb_get(got, p3) && n < 32) {
                    bb_set(got, p3);
                    out[n++] = (uint16_t)p3;
                }
            }
        }
    }
    return n;
}

/* neighbour top-piece types seen by a ground mosquito (move_gen.cuh:917-925) */
static unsigned mosquito_types(const orc_state* s, int cell) {
    unsigned t = 0;
    for (int d = 0; d < 6; d++) {
        int nb = NB[cell][d];
        if (nb < 0 || !OCC(s, nb)) continue;
        int pt = TOP_TYPE(s, nb);
        if (pt != 6) t |= 1u << pt;
    }
    return t;
}

/* mosquito union Q/P, A, G, S, B, L with dedup, cap 128 (move_gen.cuh:907-1008) */
static int mosquito_dests(const orc_state* s, int cell, const uint64_t* perim, uint16_t* out) {
    if (s->height[cell] > 1) return beetle_dests(s, cell, out, 0);
    unsigned t = mosquito_types(s, cell);
    uint64_t got[ORC_WORDS];
    memset(got, 0, sizeof(got));
    uint16_t tmp[128];
    int n = 0;
    for (int part = 0; part < 6; part++) {
        int k = 0;
        switch (part) {
            case 0: if (t & ((1u << 1) | (1u << 8))) k = queen_dests(s, cell, tmp); break;
            case 1: if (t & (1u << 2)) k = ant_bfs(s, cell, perim, tmp, 128); break;
            case 2: if (t & (1u << 3)) k = hopper_dests(s, cell, tmp); break;
            case 3: if (t & (1u << 4)) k = spider_dests(s, cell, tmp, 0); break;
            case 4: if (t & (1u << 5)) k = beetle_dests(s, cell, tmp, 0); break;
            case 5: if (t & (1u << 7)) k = ladybug_dests(s, cell, tmp, 0); break;
        }
        for (int i = 0; i < k; i++) {
            if (bb_get(got, tmp[i])) continue;
            bb_set(got, tmp[i]);
            if (n < 128) out[n++] = tmp[i];
        }
    }
    return n;
}

static int mosquito_any(const orc_state* s, int cell, const uint64_t* perim) {
    if (s->height[cell] > 1) return beetle_dests(s, cell, 0, 1); /* :1010-1049 */
    unsigned t = mosquito_types(s, cell);
    uint16_t tmp[6];
    if ((t & ((1u << 1) | (1u << 8))) && queen_dests(s, cell, tmp)) return 1;
    if ((t & (1u << 2)) && ant_any(s, cell, perim)) return 1;
    if ((t & (1u << 3)) && hopper_dests(s, cell, tmp)) return 1;
    if ((t & (1u << 4)) && spider_dests(s, cell, 0, 1)) return 1;
    if ((t & (1u << 5)) && beetle_dests(s, cell, 0, 1)) return 1;
    if ((t & (1u << 7)) && ladybug_dests(s, cell, 0, 1)) return 1;
    return 0;
}

/* ------------------------------------------------------------------ */
/* Placement cells (move_gen.cuh:1064-1140)                            */
/* ------------------------------------------------------------------ */

static void placement_cells(const orc_state* s, int color, uint64_t* res) {
    memset(res, 0, sizeof(uint64_t) * ORC_WORDS);
    if (s->turn == 0) { /* first stone goes to the centre cell */
        bb_set(res, ORC_HALF * ORC_BOARD + ORC_HALF);
        return;
    }
    if (s->turn == 1) { /* any empty neighbour of the pieces on the board */
        for (int c = 0; c < ORC_CELLS; c++) {
            if (!OCC(s, c)) continue;
            for (int d = 0; d < 6; d++) {
                int nb = NB[c][d];
                if (nb >= 0 && !OCC(s, nb)) bb_set(res, nb);
            }
        }
        return;
    }
    const uint64_t* mine = color ? s->black_top : s->white_top;
    const uint64_t* theirs = color ? s->white_top : s->black_top;
    for (int c = 0; c < ORC_CELLS; c++) {
        if (!bb_get(mine, c)) continue;
        for (int d = 0; d < 6; d++) {
            int nb = NB[c][d];
            if (nb < 0 || OCC(s, nb)) continue;
            int bad = 0;
            for (int e = 0; e < 6 && !bad; e++) {
                int n2 = NB[nb][e];
                if (n2 >= 0 && bb_get(theirs, n2)) bad = 1;
            }
            if (!bad) bb_set(res, nb);
        }
    }
}

/* ------------------------------------------------------------------ */
/* Pillbug throws (move_gen.cuh:691-769, 1379-1410)                    */
/* ------------------------------------------------------------------ */

/* Is the piece at target throwable by the piece at pb, and into which cells? */
static int throw_targets(const orc_state* s, const gen_ctx* g, int pb, int target,
                         uint16_t* dests) {
    if (target < 0 || !OCC(s, target)) return 0;
    if (s->height[target] != 1) return 0;
    if (s->stunned_cell != 0xFFFF && s->stunned_cell == target) return 0;
    if (bb_get(g->pinned, target)) return 0;
    int pbh = s->height[pb];
    int lift = imax(s->height[target] - 1, pbh);
    int back = -1;
    for (int d = 0; d < 6; d++)
        if (NB[target][d] == pb) { back = d; break; }
    if (back < 0) return 0;
    if (gate_blocked(s, target, back, lift)) return 0;
    int n = 0;
    for (int dd = 0; dd < 6; dd++) {
        int dest = NB[pb][dd];
        if (dest < 0 || dest == target || OCC(s, dest)) continue;
        if (gate_blocked(s, pb, dd, pbh)) continue;
        dests[n++] = (uint16_t)dest;
    }
    return n;
}

static int next_to_pillbug(const orc_state* s, int cell) {
    for (int d = 0; d < 6; d++) {
        int nb = NB[cell][d];
        if (nb >= 0 && OCC(s, nb) && TOP_TYPE(s, nb) == 8) return 1;
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Full legal move list (move_gen.cuh:1151-1360)                        */
/* ------------------------------------------------------------------ */

static inline void put(orc_move* out, int i, int type, int pt, int from, int to) {
    out[i].type = (uint8_t)type;
    out[i].pt = (uint8_t)pt;
    out[i].from = (uint16_t)from;
    out[i].to = (uint16_t)to;
}

int orc_legal_moves(const orc_state* s, orc_move* out) {
    if (s->result != 0) return 0;
    int color = s->turn & 1, ptn = s->turn / 2, n = 0;
    int queen_down = (s->queen_placed >> color) & 1;
    int forced_queen = (ptn == 3 && !queen_down);
    int placeable[8], any = 0;
    for (int p = 0; p < 8; p++) {
        placeable[p] = forced_queen ? (p == 0 && s->hands[color][0] > 0) : (s->hands[color][p] > 0);
        any |= placeable[p];
    }
    if (any) {
        uint64_t pc[ORC_WORDS];
        placement_cells(s, color, pc);
        for (int c = 0; c < ORC_CELLS; c++) {
            if (!bb_get(pc, c)) continue;
            for (int p = 0; p < 8; p++) {
                if (!placeable[p] || (ptn == 0 && p == 0)) continue;
                if (n < ORC_MAX_MOVES) put(out, n++, 0, p + 1, 0, c);
            }
        }
    }
    if (queen_down) {
        gen_ctx g;
        ctx_init(s, &g);
        const uint64_t* mine = color ? s->black_top : s->white_top;
        for (int c = 0; c < ORC_CELLS; c++) {
            if (!bb_get(mine, c)) continue;
            if (s->stunned_cell != 0xFFFF && s->stunned_cell == c) continue;
            if (bb_get(g.pinned, c)) continue;
            int pt = TOP_TYPE(s, c);
            uint16_t d[128];
            int k = 0;
            switch (pt) {
                case 1: case 8: k = queen_dests(s, c, d); break;
                case 2:
                    if (n < ORC_MAX_MOVES) {
                        k = ant_bfs(s, c, g.perimeter, d, ORC_MAX_MOVES - n);
                        for (int i = 0; i < k; i++) put(out, n++, 1, 2, c, d[i]);
                    }
                    k = 0;
                    break;
                case 3: k = hopper_dests(s, c, d); break;
                case 4: k = spider_dests(s, c, d, 0); break;
                case 5: k = beetle_dests(s, c, d, 0); break;
                case 6: k = mosquito_dests(s, c, g.perimeter, d); break;
                case 7: k = ladybug_dests(s, c, d, 0); break;
                default: break;
            }
            for (int i = 0; i < k && n < ORC_MAX_MOVES; i++) put(out, n++, 1, pt, c, d[i]);
        }
        /* second pass: throws by own pillbugs and pillbug-adjacent ground mosquitoes */
        for (int c = 0; c < ORC_CELLS; c++) {
            if (!bb_get(mine, c)) continue;
            int pt = TOP_TYPE(s, c);
            int thrower = (pt == 8) || (pt == 6 && s->height[c] == 1 && next_to_pillbug(s, c));
            if (!thrower) continue;
            for (int dt = 0; dt < 6; dt++) {
                int target = NB[c][dt];
                uint16_t dd[6];
                int k = throw_targets(s, &g, c, target, dd);
                for (int i = 0; i < k; i++)
                    if (n < ORC_MAX_MOVES) put(out, n++, 1, TOP_TYPE(s, target), target, dd[i]);
            }
        }
    }
    if (n == 0) {
        put(out, 0, 2, 0, 0, 0);
        n = 1;
    }
    return n;
}

/* ------------------------------------------------------------------ */
/* Compact list for successor features (move_gen.cuh:1362-1563)         */
/* ------------------------------------------------------------------ */

static void flag_move(const orc_state* s, orc_move* out, int* n, uint32_t* seen, int pt, int from) {
    int h = s->height[from]; /* emit_fnn_move_flag, move_gen.cuh:1362-1377 */
    if (h <= 0) return;
    int owner = BYTE_COLOR(s->pieces[h - 1][from]);
    uint32_t bit = 1u << ((pt - 1) * 2 + owner);
    if (*seen & bit) return;
    *seen |= bit;
    put(out, (*n)++, 1, pt, from, 0);
}

int orc_compact_moves(const orc_state* s, orc_move* out) {
    if (s->result != 0) return 0;
    int color = s->turn & 1, ptn = s->turn / 2, n = 0;
    int queen_down = (s->queen_placed >> color) & 1;
    int forced_queen = (ptn == 3 && !queen_down);
    int any = 0;
    for (int p = 0; p < 8; p++) {
        int ok = forced_queen ? (p == 0 && s->hands[color][0] > 0) : (s->hands[color][p] > 0);
        if (ptn == 0 && p == 0) ok = 0;
        any |= ok;
    }
    if (any) {
        uint64_t pc[ORC_WORDS];
        placement_cells(s, color, pc);
        for (int c = 0; c < ORC_CELLS && n < ORC_MAX_MOVES; c++)
            if (bb_get(pc, c)) put(out, n++, 0, 0, 0, c);
    }
    if (!queen_down || n >= ORC_MAX_MOVES) {
        if (n == 0) { put(out, 0, 2, 0, 0, 0); return 1; }
        return n;
    }
    gen_ctx g;
    ctx_init(s, &g);
    uint32_t seen = 0;
    const uint64_t* mine = color ? s->black_top : s->white_top;
    for (int c = 0; c < ORC_CELLS && n < ORC_MAX_MOVES; c++) {
        if (!bb_get(mine, c)) continue;
        if (s->stunned_cell != 0xFFFF && s->stunned_cell == c) continue;
        if (bb_get(g.pinned, c)) continue;
        int pt = TOP_TYPE(s, c);
        if (seen & (1u << ((pt - 1) * 2 + color))) continue;
        uint16_t tmp[6];
        int can = 0;
        switch (pt) {
            case 1: case 8: can = queen_dests(s, c, tmp) > 0; break;
            case 2: can = ant_any(s, c, g.perimeter); break;
            case 3: can = hopper_dests(s, c, tmp) > 0; break;
            case 4: can = spider_dests(s, c, 0, 1); break;
            case 5: can = beetle_dests(s, c, 0, 1); break;
            case 6: can = mosquito_any(s, c, g.perimeter); break;
            case 7: can = ladybug_dests(s, c, 0, 1); break;
            default: break;
        }
        if (can) flag_move(s, out, &n, &seen, pt, c);
    }
    for (int c = 0; c < ORC_CELLS && n < ORC_MAX_MOVES; c++) {
        if (!bb_get(mine, c)) continue;
        int pt = TOP_TYPE(s, c);
        int thrower = (pt == 8) || (pt == 6 && s->height[c] == 1 && next_to_pillbug(s, c));
        if (!thrower) continue;
        for (int dt = 0; dt < 6; dt++) {
            int target = NB[c][dt];
            uint16_t dd[6];
            if (throw_targets(s, &g, c, target, dd) > 0) flag_move(s, out, &n, &seen, TOP_TYPE(s, target), target);
        }
    }
    if (n == 0) { put(out, 0, 2, 0, 0, 0); return 1; }
    return n;
}

/* ------------------------------------------------------------------ */
/* FNN features (fnn_features.cuh:45-331)                               */
/* ------------------------------------------------------------------ */

static int hex_dist(int a, int b) {
    int dq = (b % ORC_BOARD) - (a % ORC_BOARD);
    int dr = (b / ORC_BOARD) - (a / ORC_BOARD);
    int ds = -(dq + dr);
    if (dq < 0) dq = -dq;
    if (dr < 0) dr = -dr;
    if (ds < 0) ds = -ds;
    return imax(dq, imax(dr, ds));
}

void orc_features(const orc_state* s, const orc_move* mv, int nmv, float* f) {
    memset(f, 0, sizeof(float) * ORC_FEAT);
    float dsum[2][8];
    int dcnt[2][8];
    memset(dsum, 0, sizeof(dsum));
    memset(dcnt, 0, sizeof(dcnt));
    int surround[2] = {0, 0};
    uint64_t ap[ORC_WORDS];
    orc_articulation(s, ap);
    int pbc[2][8], npb[2] = {0, 0};
    int stun = s->stunned_cell;

    for (int c = 0; c < ORC_CELLS; c++) {
        int h = s->height[c];
        if (!h) continue;
        uint8_t top = s->pieces[h - 1][c];
        int pt = top & 0x0F, col = BYTE_COLOR(top);
        int tc = (pt - 1) * 2 + col;
        f[tc] += 1.0f; /* [0:16] */
        int occn = 0;
        for (int d = 0; d < 6; d++) {
            int nb = NB[c][d];
            if (nb >= 0 && s->height[nb] > 0) occn++;
        }
        if (occn == 0) f[96 + col] += 1.0f; /* [96:98] */
        int oq = s->queen_cell[1 - col];
        if (oq != 0xFFFF) {
            for (int d = 0; d < 6; d++)
                if (NB[c][d] >= 0 && NB[c][d] == oq) { f[32 + tc] += 1.0f; break; }
        }
        for (int q = 0; q < 2; q++) {
            int qc = s->queen_cell[q];
            if (qc == 0xFFFF) continue;
            for (int d = 0; d < 6; d++)
                if (NB[qc][d] >= 0 && NB[qc][d] == c) { surround[q]++; break; }
        }
        if (oq != 0xFFFF) {
            dsum[col][pt - 1] += (float)hex_dist(c, oq);
            dcnt[col][pt - 1]++;
        }
        if (h == 1 && bb_get(ap, c)) f[80 + tc] += 1.0f; /* [80:96] */
        if (pt != 1) {
            for (int lv = 0; lv < h - 1; lv++) {
                uint8_t b = s->pieces[lv][c];
                if ((b & 0x0F) == 1) f[98 + BYTE_COLOR(b)] = 1.0f; /* [98:100] */
            }
        }
        int capable = (stun != c) && pt == 8;
        if (!capable && stun != c && pt == 6 && h == 1) {
            for (int d = 0; d < 6; d++) {
                int nb = NB[c][d];
                if (nb < 0 || s->height[nb] == 0 || stun == nb) continue;
                if (TOP_TYPE(s, nb) == 8) { capable = 1; break; }
            }
        }
        if (capable) {
            f[104 + col] = 1.0f;
            if (npb[col] < 8) pbc[col][npb[col]++] = c;
        }
    }
    for (int col = 0; col < 2; col++)
        for (int t = 0; t < 8; t++)
            if (dcnt[col][t] > 0)
                f[48 + t * 2 + col] = dsum[col][t] / (float)dcnt[col][t] / 10.0f;
    for (int col = 0; col < 2; col++)
        for (int t = 0; t < 8; t++)
            f[16 + t * 2 + col] = (float)s->hands[col][t] / (float)PER_TYPE[t];

    /* [64:80] distinct source cells per (type, owner); [100:102] placement cells */
    uint64_t srcs[16][ORC_WORDS];
    memset(srcs, 0, sizeof(srcs));
    uint64_t place[ORC_WORDS];
    memset(place, 0, sizeof(place));
    int nplace = 0, cur = s->turn & 1;
    for (int m = 0; m < nmv; m++) {
        if (mv[m].type == 1) {
            int from = mv[m].from, h = s->height[from];
            int owner = h > 0 ? BYTE_COLOR(s->pieces[h - 1][from]) : cur;
            bb_set(srcs[(mv[m].pt - 1) * 2 + owner], from);
        } else if (mv[m].type == 0) {
            if (!bb_get(place, mv[m].to)) {
                bb_set(place, mv[m].to);
                nplace++;
            }
        }
    }
    for (int i = 0; i < 16; i++) f[64 + i] = (float)bb_pop(srcs[i]);
    f[100 + cur] = (float)nplace / 10.0f;
    int left = 200 - (int)s->turn;
    if (left < 0) left = 0;
    f[102] = (float)left / 200.0f;
    float t = (float)s->turn / 100.0f;
    f[103] = t < 1.0f ? t : 1.0f;
    for (int col = 0; col < 2; col++) {
        for (int i = 0; i < npb[col]; i++) {
            int p = pbc[col][i];
            for (int d = 0; d < 6; d++) {
                int nb = NB[p][d];
                if (nb < 0 || s->height[nb] == 0 || stun == nb) continue;
                int nc = BYTE_COLOR(s->pieces[s->height[nb] - 1][nb]);
                if (nc == col) f[106 + col] += 1.0f;
                else f[108 + nc] += 1.0f;
            }
        }
    }
    for (int q = 0; q < 2; q++)
        if (surround[q] >= 1 && surround[q] <= 6) f[110 + q * 6 + surround[q] - 1] = 1.0f;
}

/* ------------------------------------------------------------------ */
/* Centroid and action index (state_encoder.cuh:55-79, 889-906;        */
/* mcts_tree.cuh:146-179)                                               */
/* ------------------------------------------------------------------ */

/* round-half-to-even of sum/n for n > 0 (Python round()) */
static int round_half_even(int sum, int n) {
    int q = sum / n, r = sum - q * n;
    int twice = 2 * (r < 0 ? -r : r);
    if (twice < n) return q;
    int away = sum > 0 ? q + 1 : q - 1;
    if (twice > n) return away;
    return (q % 2 == 0) ? q : away;
}

void orc_centroid(const orc_state* s, int* cq, int* cr) {
    int sq = 0, sr = 0, n = 0;
    for (int c = 0; c < ORC_CELLS; c++) {
        if (!s->height[c]) continue;
        sq += c % ORC_BOARD - ORC_HALF;
        sr += c / ORC_BOARD - ORC_HALF;
        n++;
    }
    *cq = n ? round_half_even(sq, n) : 0;
    *cr = n ? round_half_even(sr, n) : 0;
}

int orc_move_to_action(const orc_move* m, int cq, int cr) {
    const int G = 17, H = 8, G2 = 289;
    if (m->type == 2) return 85833;
    if (m->type == 0) {
        int ec = (m->to % ORC_BOARD - ORC_HALF) - cq + H;
        int er = (m->to / ORC_BOARD - ORC_HALF) - cr + H;
        if (ec < 0 || ec >= G || er < 0 || er >= G) return -1;
        return (m->pt - 1) * G2 + er * G + ec;
    }
    int sc = (m->from % ORC_BOARD - ORC_HALF) - cq + H;
    int sr = (m->from / ORC_BOARD - ORC_HALF) - cr + H;
    int dc = (m->to % ORC_BOARD - ORC_HALF) - cq + H;
    int dr = (m->to / ORC_BOARD - ORC_HALF) - cr + H;
    if (sc < 0 || sc >= G || sr < 0 || sr >= G || dc < 0 || dc >= G || dr < 0 || dr >= G) return -1;
    return 2312 + (sr * G + sc) * G2 + dr * G + dc;
}

/* has_queen_escape_move, move_gen.cuh:771-821 */
int orc_queen_escape(const orc_state* s) {
    int color = s->turn & 1;
    if (!((s->queen_placed >> color) & 1)) return 0;
    int q = s->queen_cell[color];
    if (q >= ORC_CELLS || !OCC(s, q)) return 0;
    gen_ctx g;
    ctx_init(s, &g);
    uint16_t tmp[6];
    uint8_t top = TOP_BYTE(s, q);
    if ((top & 0x0F) == 1 && BYTE_COLOR(top) == color && !bb_get(g.pinned, q) && queen_dests(s, q, tmp))
        return 1;
    const uint64_t* mine = color ? s->black_top : s->white_top;
    for (int c = 0; c < ORC_CELLS; c++) {
        if (!bb_get(mine, c)) continue;
        int pt = TOP_TYPE(s, c);
        int thrower = (pt == 8) || (pt == 6 && s->height[c] == 1 && next_to_pillbug(s, c));
        if (!thrower) continue;
        int adj = 0;
        for (int d = 0; d < 6; d++) if (NB[c][d] == q) adj = 1;
        if (adj && throw_targets(s, &g, c, q, tmp) > 0) return 1;
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Seeded playout position generator (benchmark/test inputs)           */
/* ------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* counter-based splitmix64 stream: (seed, game, ply) -> 64 random bits */
uint64_t orc_rng(uint64_t seed, uint64_t game, uint64_t ply) {
    return mix64(mix64(seed ^ mix64(game)) + ply);
}

/*
 * Uniform random legal playout: stop ply ~ U[0, max_ply] from draw 0, then
 * at ply p (1-based) the move index is draw p mod num_legal over the full
 * list (duplicates included), stopping early when the game ends.
 */
void orc_playout(uint64_t seed, int64_t game, int max_ply, int expansion_mask, orc_state* s) {
    orc_init_tables();
    orc_init_state(s, expansion_mask);
    int stop = (int)(orc_rng(seed, (uint64_t)game, 0) % (uint64_t)(max_ply + 1));
    orc_move mv[ORC_MAX_MOVES];
    for (int p = 1; p <= stop; p++) {
        if (s->result != 0) break;
        int n = orc_legal_moves(s, mv);
        int k = (int)(orc_rng(seed, (uint64_t)game, (uint64_t)p) % (uint64_t)n);
        orc_apply_move(s, &mv[k]);
    }
}

/* ------------------------------------------------------------------ */
/* Batched drivers                                                      */
/* ------------------------------------------------------------------ */

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

#ifdef _OPENMP
#define PAR_FOR(threads) _Pragma("omp parallel for schedule(dynamic, 64) num_threads(nt)")
#define SET_NT(threads) int nt = (threads) > 0 ? (threads) : omp_get_max_threads();
#else
#define PAR_FOR(threads)
#define SET_NT(threads) (void)(threads);
#endif

void orc_generate_positions(uint64_t seed, int64_t first_game, int64_t count, int max_ply,
                            int expansion_mask, uint8_t* states, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++)
        orc_playout(seed, first_game + i, max_ply, expansion_mask,
                    (orc_state*)(states + i * ORC_STATE_BYTES));
}

void orc_legal_moves_features_batch(const uint8_t* states, int64_t count, uint8_t* moves,
                                    int32_t* num_legal, float* feats, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++) {
        const orc_state* s = (const orc_state*)(states + i * ORC_STATE_BYTES);
        orc_move* mv = (orc_move*)(moves + i * ORC_MAX_MOVES * 6);
        memset(mv, 0, ORC_MAX_MOVES * 6);
        int n = orc_legal_moves(s, mv);
        num_legal[i] = n;
        orc_features(s, mv, n, feats + i * ORC_FEAT);
    }
}

void orc_legal_moves_batch(const uint8_t* states, int64_t count, uint8_t* moves,
                           int32_t* num_legal, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++) {
        orc_move* mv = (orc_move*)(moves + i * ORC_MAX_MOVES * 6);
        memset(mv, 0, ORC_MAX_MOVES * 6);
        num_legal[i] = orc_legal_moves((const orc_state*)(states + i * ORC_STATE_BYTES), mv);
    }
}

void orc_features_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                        int64_t count, float* feats, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++)
        orc_features((const orc_state*)(states + i * ORC_STATE_BYTES),
                     (const orc_move*)(moves + i * ORC_MAX_MOVES * 6), num_legal[i],
                     feats + i * ORC_FEAT);
}

void orc_compact_moves_batch(const uint8_t* states, int64_t count, uint8_t* moves,
                             int32_t* num_legal, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++) {
        orc_move* mv = (orc_move*)(moves + i * ORC_MAX_MOVES * 6);
        memset(mv, 0, ORC_MAX_MOVES * 6);
        num_legal[i] = orc_compact_moves((const orc_state*)(states + i * ORC_STATE_BYTES), mv);
    }
}

/* successor features with the GPU semantics: apply, compact list, features
 * (game_logic.cu:182-229 fnn_successor_features_kernel) */
void orc_successor_features_batch(const uint8_t* states, const uint8_t* moves,
                                  const int64_t* action_to_root, const int64_t* move_indices,
                                  int64_t count, float* feats, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++) {
        int64_t r = action_to_root[i];
        orc_state child;
        memcpy(&child, states + r * ORC_STATE_BYTES, sizeof(child));
        const orc_move* mv = (const orc_move*)(moves + (r * ORC_MAX_MOVES + move_indices[i]) * 6);
        orc_apply_move(&child, mv);
        orc_move cm[ORC_MAX_MOVES];
        int n = orc_compact_moves(&child, cm);
        orc_features(&child, cm, n, feats + i * ORC_FEAT);
    }
}

void orc_apply_moves_batch(uint8_t* states, const uint8_t* moves, int64_t count) {
    orc_init_tables();
    for (int64_t i = 0; i < count; i++)
        orc_apply_move((orc_state*)(states + i * ORC_STATE_BYTES), (const orc_move*)(moves + i * 6));
}

void orc_articulation_batch(const uint8_t* states, int64_t count, uint64_t* ap_words, int threads) {
    orc_init_tables();
    SET_NT(threads)
    PAR_FOR(threads)
    for (int64_t i = 0; i < count; i++)
        orc_articulation((const orc_state*)(states + i * ORC_STATE_BYTES), ap_words + i * ORC_WORDS);
}

void orc_actions_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                       int64_t count, int32_t* actions, int32_t* centroids) {
    orc_init_tables();
    for (int64_t i = 0; i < count; i++) {
        const orc_state* s = (const orc_state*)(states + i * ORC_STATE_BYTES);
        int cq, cr;
        orc_centroid(s, &cq, &cr);
        if (centroids) { centroids[i * 2] = cq; centroids[i * 2 + 1] = cr; }
        for (int m = 0; m < ORC_MAX_MOVES; m++) actions[i * ORC_MAX_MOVES + m] = -1;
        for (int m = 0; m < num_legal[i]; m++)
            actions[i * ORC_MAX_MOVES + m] =
                orc_move_to_action((const orc_move*)(moves + (i * ORC_MAX_MOVES + m) * 6), cq, cr);
    }
}

void orc_queen_escape_batch(const uint8_t* states, int64_t count, uint8_t* flags) {
    orc_init_tables();
    for (int64_t i = 0; i < count; i++)
        flags[i] = (uint8_t)orc_queen_escape((const orc_state*)(states + i * ORC_STATE_BYTES));
}

/* ------------------------------------------------------------------ */
/* Root tactical probe (game_logic.cu:290-397 root_tactical_probe_kernel */
/* with move_gen.cuh:825-899 helpers)                                   */
/* ------------------------------------------------------------------ */

/* queen_surround_count_for_color_device, move_gen.cuh:825-831 */
static int surround_count(const orc_state* s, int color) {
    if (!((s->queen_placed >> color) & 1)) return 0;
    return occupied_neighbours(s, s->queen_cell[color]);
}

/* lone_empty_neighbor_of_queen, move_gen.cuh:833-852 */
static int lone_empty_neighbour(const orc_state* s, int target) {
    if (!((s->queen_placed >> target) & 1)) return -1;
    int q = s->queen_cell[target];
    if (q >= ORC_CELLS) return -1;
    if (occupied_neighbours(s, q) != 5) return -1;
    int e = -1;
    for (int d = 0; d < 6; d++) {
        int nb = NB[q][d];
        if (nb < 0) continue;
        if (!OCC(s, nb)) {
            if (e >= 0) return -1;
            e = nb;
        }
    }
    return e;
}

static inline int wins_for(int result, int color) { return result == (color == 0 ? 1 : 2); }

/* has_immediate_surround_win_for_current_player, move_gen.cuh:854-874 */
static int immediate_win(const orc_state* s) {
    int player = s->turn & 1;
    int cell = lone_empty_neighbour(s, player ^ 1);
    if (cell < 0) return 0;
    orc_move mv[ORC_MAX_MOVES];
    int n = orc_legal_moves(s, mv);
    for (int i = 0; i < n; i++) {
        if (mv[i].to != cell) continue;
        orc_state c = *s;
        orc_apply_move(&c, &mv[i]);
        if (wins_for(c.result, player)) return 1;
    }
    return 0;
}

void orc_tactical_probe(const orc_state* root, const orc_move* moves, int nlegal, const float* priors,
                        int w1, int chk, int w2, int64_t* winning, uint8_t* allowed, uint8_t* forced) {
    *winning = -1;
    *forced = 0;
    for (int i = 0; i < ORC_MAX_MOVES; i++) allowed[i] = i < nlegal;
    if (nlegal <= 0 || root->result != 0) return;
    int me = root->turn & 1, opp = me ^ 1;
    int opp_s = surround_count(root, opp), own_s = surround_count(root, me);
    if (w1 && opp_s == 5) {
        int best = -1;
        float bp = -1e30f;
        for (int i = 0; i < nlegal; i++) {
            orc_state c = *root;
            orc_apply_move(&c, &moves[i]);
            if (wins_for(c.result, me) && (best < 0 || priors[i] > bp)) {
                best = i;
                bp = priors[i];
            }
        }
        if (best >= 0) {
            *winning = best;
            return;
        }
    }
    if (chk && own_s == 5) {
        int any_safe = 0;
        for (int i = 0; i < nlegal; i++) {
            orc_state c = *root;
            orc_apply_move(&c, &moves[i]);
            int bad = immediate_win(&c);
            allowed[i] = !bad;
            any_safe |= !bad;
        }
        if (!any_safe) {
            *forced = 1;
            return;
        }
    }
    if (!w2 || !(opp_s == 4 || opp_s == 5)) return;
    orc_move rep[ORC_MAX_MOVES];
    for (int i = 0; i < nlegal; i++) {
        if (!allowed[i]) continue;
        orc_state c = *root;
        orc_apply_move(&c, &moves[i]);
        int cs = surround_count(&c, opp);
        if (opp_s == 4 && cs <= opp_s) continue;
        if (opp_s == 5 && cs < opp_s) continue;
        /* generate_non_decreasing_surround_replies, move_gen.cuh:876-899 */
        int nr = orc_legal_moves(&c, rep), ok = 1;
        for (int r = 0; r < nr && ok; r++) {
            orc_state g = c;
            orc_apply_move(&g, &rep[r]);
            if (surround_count(&g, opp) < cs) ok = 0;
        }
        if (!ok) continue;
        for (int r = 0; r < nr && ok; r++) {
            orc_state g = c;
            orc_apply_move(&g, &rep[r]);
            if (!wins_for(g.result, me) && !immediate_win(&g)) ok = 0;
        }
        if (ok) {
            *winning = i;
            return;
        }
    }
}

void orc_tactical_probe_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                              const float* priors, int64_t count, int w1, int chk, int w2,
                              int64_t* winning, uint8_t* allowed, uint8_t* forced, int threads) {
    orc_init_tables();
    if (threads <= 0) threads = orc_num_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int64_t i = 0; i < count; i++)
        orc_tactical_probe((const orc_state*)(states + i * ORC_STATE_BYTES),
                           (const orc_move*)(moves + i * ORC_MAX_MOVES * 6), num_legal[i],
                           priors + i * ORC_MAX_MOVES, w1, chk, w2, winning + i,
                           allowed + i * ORC_MAX_MOVES, forced + i);
}

/* ------------------------------------------------------------------ */
/* Hybrid transformer inputs (state_encoder.cuh:372-550)               */
/* ------------------------------------------------------------------ */

#define ORC_TOKENS 28
#define ORC_TOK_FEAT 27
#define ORC_MOVE_FEAT 31

static int height_neighbours(const orc_state* s, int cell, int* flags) {
    int n = 0;
    for (int d = 0; d < 6; d++) {
        int nb = NB[cell][d];
        int f = nb >= 0 && s->height[nb] > 0;
        if (flags) flags[d] = f;
        n += f;
    }
    return n;
}

/* extract_hybrid_transformer_tokens_device, state_encoder.cuh:372-468 */
int orc_hybrid_tokens(const orc_state* s, float* tf, int32_t* tq, int32_t* tr, int32_t* tz, uint8_t* tm,
                      float* gf) {
    memset(tf, 0, sizeof(float) * ORC_TOKENS * ORC_TOK_FEAT);
    memset(tq, 0, sizeof(int32_t) * ORC_TOKENS);
    memset(tr, 0, sizeof(int32_t) * ORC_TOKENS);
    memset(tz, 0, sizeof(int32_t) * ORC_TOKENS);
    memset(tm, 0, ORC_TOKENS);
    memset(gf, 0, sizeof(float) * 6);
    float qs[2] = {0.0f, 0.0f};
    uint64_t ap[ORC_WORDS];
    orc_articulation(s, ap);
    for (int c = 0; c < 2; c++) {
        int q = s->queen_cell[c];
        if (q != 0xFFFF && q < ORC_CELLS) qs[c] = (float)height_neighbours(s, q, NULL) / 6.0f;
    }
    int n = 0;
    for (int cell = 0; cell < ORC_CELLS; cell++) {
        int h = s->height[cell];
        if (h == 0) continue;
        int fl[6];
        int oc = height_neighbours(s, cell, fl);
        for (int lv = 0; lv < h && lv < ORC_MAX_STACK; lv++) {
            if (n >= ORC_TOKENS) break;
            uint8_t b = s->pieces[lv][cell];
            int pt = b & 0x0F, pc = BYTE_COLOR(b), top = lv == h - 1;
            float* f = tf + n * ORC_TOK_FEAT;
            if (pt >= 1 && pt <= 8) f[pt - 1] = 1.0f;
            f[8 + pc] = 1.0f;
            f[10] = lv == 0 ? 1.0f : 0.0f;
            f[11] = top ? 1.0f : 0.0f;
            f[12] = (float)h / 4.0f;
            f[13] = pt == 1 ? 1.0f : 0.0f;
            f[14] = qs[pc];
            f[15] = (float)oc / 6.0f;
            if (top)
                for (int d = 0; d < 6; d++)
                    if (!fl[d]) f[16 + d] = 1.0f;
            f[24] = (float)lv * 0.25f;
            f[25] = (s->stunned_cell != 0xFFFF && s->stunned_cell == cell) ? 1.0f : 0.0f;
            if (top) f[26] = bb_get(ap, cell) ? 1.0f : 0.0f;
            tq[n] = cell % ORC_BOARD;
            tr[n] = cell / ORC_BOARD;
            tz[n] = lv;
            tm[n] = 1;
            n++;
        }
    }
    int cur = s->turn & 1, wh = 0, bh = 0;
    gf[0] = cur == 0 ? 1.0f : 0.0f;
    gf[1] = ((float)s->turn / 100.0f < 1.0f) ? (float)s->turn / 100.0f : 1.0f;
    gf[2] = (s->queen_placed & 1) ? 1.0f : 0.0f;
    gf[3] = (s->queen_placed & 2) ? 1.0f : 0.0f;
    for (int p = 0; p < 8; p++) {
        wh += s->hands[0][p];
        bh += s->hands[1][p];
    }
    gf[4] = (float)wh / 14.0f;
    gf[5] = (float)bh / 14.0f;
    return n;
}

/* queen_surround_count_current, state_encoder.cuh:109-121 */
static int qs_current(const orc_state* s, int color) {
    if (!((s->queen_placed >> color) & 1)) return 0;
    int q = s->queen_cell[color];
    return q < ORC_CELLS ? height_neighbours(s, q, NULL) : 0;
}

/* queen_surround_count_after_move, state_encoder.cuh:123-165 */
static int qs_after(const orc_state* s, const orc_move* m, int qc, int mover, int moved) {
    int placed = (s->queen_placed >> qc) & 1;
    int being_placed = m->type == 0 && m->pt == 1 && mover == qc && m->to < ORC_CELLS;
    int being_moved = m->type == 1 && m->pt == 1 && moved == qc && m->to < ORC_CELLS;
    if (!placed && !being_placed) return 0;
    int q = placed ? (int)s->queen_cell[qc] : -1;
    if (being_placed || being_moved) q = m->to;
    if (q < 0 || q >= ORC_CELLS) return 0;
    int has_src = m->type == 1 && m->from < ORC_CELLS;
    int src = has_src ? m->from : -1;
    int dst = m->to < ORC_CELLS ? m->to : -1;
    int src_stays = has_src && s->height[src] > 1;
    int n = 0;
    for (int d = 0; d < 6; d++) {
        int nb = NB[q][d];
        if (nb < 0) continue;
        int occ = s->height[nb] > 0;
        if (has_src && nb == src) occ = src_stays;
        if (dst >= 0 && nb == dst) occ = 1;
        n += occ;
    }
    return n;
}

/* extract_hybrid_transformer_move_features_device, state_encoder.cuh:470-550 */
void orc_hybrid_move_features(const orc_state* s, const orc_move* mv, int n, float* out) {
    memset(out, 0, sizeof(float) * ORC_MAX_MOVES * ORC_MOVE_FEAT);
    if (n > ORC_MAX_MOVES) n = ORC_MAX_MOVES;
    int me = s->turn & 1, op = me ^ 1;
    int oq = s->queen_cell[me], pq = s->queen_cell[op];
    int oqc = oq != 0xFFFF ? oq % ORC_BOARD - ORC_HALF : 0, oqr = oq != 0xFFFF ? oq / ORC_BOARD - ORC_HALF : 0;
    int pqc = pq != 0xFFFF ? pq % ORC_BOARD - ORC_HALF : 0, pqr = pq != 0xFFFF ? pq / ORC_BOARD - ORC_HALF : 0;
    int os0 = qs_current(s, me), ps0 = qs_current(s, op);
    const float H = (float)ORC_HALF;
    for (int i = 0; i < n; i++) {
        const orc_move* m = &mv[i];
        float* f = out + i * ORC_MOVE_FEAT;
        int moved = me;
        if (m->type == 1 && m->from < ORC_CELLS && s->height[m->from] > 0)
            moved = BYTE_COLOR(s->pieces[s->height[m->from] - 1][m->from]);
        if (m->type < ORC_MOVE_FEAT) f[m->type] = 1.0f;
        if (m->pt >= 1 && m->pt <= 8) f[3 + m->pt - 1] = 1.0f;
        int src = m->type == 1;
        f[11] = src ? 1.0f : 0.0f;
        int sq = 0, sr = 0, dq = 0, dr = 0, ss = 0, ds = 0, docc = 0;
        if (m->to < ORC_CELLS) {
            dq = m->to % ORC_BOARD - ORC_HALF;
            dr = m->to / ORC_BOARD - ORC_HALF;
            ds = s->height[m->to];
            docc = ds > 0;
        }
        if (src && m->from < ORC_CELLS) {
            sq = m->from % ORC_BOARD - ORC_HALF;
            sr = m->from / ORC_BOARD - ORC_HALF;
            ss = s->height[m->from];
        }
        f[12] = src ? (float)(dq - sq) / H : 0.0f;
        f[13] = src ? (float)(dr - sr) / H : 0.0f;
        f[14] = (float)(dq - oqc) / H;
        f[15] = (float)(dr - oqr) / H;
        f[16] = (float)(dq - pqc) / H;
        f[17] = (float)(dr - pqr) / H;
        f[18] = src ? (float)(sq - oqc) / H : 0.0f;
        f[19] = src ? (float)(sr - oqr) / H : 0.0f;
        f[20] = src ? (float)(sq - pqc) / H : 0.0f;
        f[21] = src ? (float)(sr - pqr) / H : 0.0f;
        f[22] = (float)ss / 5.0f;
        f[23] = (float)ds / 5.0f;
        f[24] = (float)docc;
        int od = qs_after(s, m, me, me, moved) - os0, pd = qs_after(s, m, op, me, moved) - ps0;
        od = od < -1 ? -1 : (od > 1 ? 1 : od);
        pd = pd < -1 ? -1 : (pd > 1 ? 1 : pd);
        f[25 + od + 1] = 1.0f;
        f[28 + pd + 1] = 1.0f;
    }
}

void orc_hybrid_encode_batch(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal, int64_t count,
                             float* tf, int32_t* tq, int32_t* tr, int32_t* tz, uint8_t* tm, float* gf,
                             int32_t* ntok, float* mf, int threads) {
    orc_init_tables();
    if (threads <= 0) threads = orc_num_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int64_t i = 0; i < count; i++) {
        const orc_state* s = (const orc_state*)(states + i * ORC_STATE_BYTES);
        int n = orc_hybrid_tokens(s, tf + i * ORC_TOKENS * ORC_TOK_FEAT, tq + i * ORC_TOKENS, tr + i * ORC_TOKENS,
                                  tz + i * ORC_TOKENS, tm + i * ORC_TOKENS, gf + i * 6);
        if (ntok) ntok[i] = n;
        if (mf)
            orc_hybrid_move_features(s, (const orc_move*)(moves + i * ORC_MAX_MOVES * 6), num_legal[i],
                                     mf + i * ORC_MAX_MOVES * ORC_MOVE_FEAT);
    }
}
