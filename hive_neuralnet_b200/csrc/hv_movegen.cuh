// hv_movegen.cuh -- warp-cooperative legal move generation, the compact
// successor list and the 122-float FNN features (sm_100a).
//
// Semantics follow the reference exactly (it is the parity target):
//   full list      hive_gpu/csrc/move_gen.cuh:1151-1360
//   compact list   hive_gpu/csrc/move_gen.cuh:1362-1563
//   features       hive_gpu/csrc/fnn_features.cuh:68-331
// including its emission order, duplicates (throws vs. ordinary moves),
// truncation at 256 moves, 32-destination caps for spider/ladybug and the
// 128-destination cap of a mosquito's union.  Cells are p-space (see
// hv_core.cuh) internally; move lists hold the reference's cell index.
//
// All piece movements run through one warp-cooperative walk engine (walk()),
// so the kernel carries a single copy of the generator loop: its instruction
// footprint is what bounds this code on the SM, not arithmetic.
#pragma once

#include "hv_core.cuh"

namespace hv {

// move list entry in reference cell indices
__device__ __forceinline__ void put_move(WarpSmem* w, int m, int type, int pt, int from_c, int to_c) {
    w->mv[3 * m] = (uint16_t)(type | (pt << 8));
    w->mv[3 * m + 1] = (uint16_t)from_c;
    w->mv[3 * m + 2] = (uint16_t)to_c;
}

__device__ __forceinline__ bool set_has(const uint32_t* s, int p) { return (s[p >> 5] >> (p & 31)) & 1u; }
__device__ __forceinline__ void set_add(uint32_t* s, int p) { atomicOr(&s[p >> 5], 1u << (p & 31)); }
__device__ __forceinline__ void set_clear(uint32_t* s) {
    if (lane_id() < 24) s[lane_id()] = 0u;
    __syncwarp();
}

// occupancy minus one cell -> slx (the mover is lifted off the board)
__device__ __forceinline__ void lift_mover(WarpSmem* w, uint32_t occ_row, int cell) {
    uint32_t x = occ_row;
    if (lane_id() == (cell >> 5)) x &= ~(1u << (cell & 31));
    build_slide_masks(x, w->slx);
    __syncwarp();
}

// ---------------------------------------------------------------------------
// walk engine
// ---------------------------------------------------------------------------
enum WalkMode : int {
    WM_STEP = 0,    // queen / pillbug one-step slide      move_gen.cuh:202-219, 644-651
    WM_BEETLE = 1,  // beetle: elevated gate or slide       move_gen.cuh:468-524
    WM_HOP = 2,     // grasshopper jump                     move_gen.cuh:228-257
    WM_ANT = 3,     // ant breadth-first search             move_gen.cuh:267-388
    WM_SPIDER = 4,  // exactly three slides, no revisits    move_gen.cuh:397-454
    WM_LADY = 5,    // up, across, down                     move_gen.cuh:538-637
};

// Destinations of the piece at `cell` moving as `mode`, in the reference's
// emission order, into out (at most cap).  Lanes take (queue item, direction)
// pairs, five items per round: the queue holds the ant's reached cells (the
// output list itself, as in the reference) or the spider/ladybug partial
// paths (level-1 then level-2 cells, i.e. lexicographic (d1, d2) order).  A
// destination reached by several lanes in one round is kept by the lowest
// lane, which reproduces the reference's sequential first-seen order.
// first_only: return 1 as soon as one destination exists (has_*_move).
// Ant and spider need slx built for this cell.
__device__ __forceinline__ int walk_body(WarpSmem* w, int cell, int mode, uint16_t* out, int cap,
                                        bool first_only) {
    Pos P{w};
    const int l = lane_id();
    const uint32_t lt = lanemask_lt();
    const int k = l / 6, d = l - 6 * (l / 6);  // lanes 30, 31 idle (k == 5)
    uint16_t* Q = mode == WM_ANT ? out : w->qcell;
    const int hcell = P.height(cell);
    set_clear(w->seen);
    if (mode == WM_ANT && l == 0) set_add(w->seen, cell);
    __syncwarp();
    int rd = 0, wr = 0, cnt = 0, l2start = 0;
    bool seed = true;
#pragma unroll 1
    while (true) {
        int items = 1;
        if (!seed) {
            if (rd >= wr || (mode == WM_ANT && wr >= cap)) break;
            items = min(5, wr - rd);
        }
        int dest = -1, cur = cell;
        bool fin = false, app = false;
        if (k < items) {
            int lev = 0, anc = cell;
            if (!seed) {
                cur = Q[rd + k];
                lev = (mode == WM_ANT || rd + k < l2start) ? 1 : 2;
                if (lev == 2) anc = w->qanc[rd + k];
            }
            const int nb = nbr(cur, d);
            switch (mode) {
                case WM_STEP:
                    fin = rowbit(w->sl[d], cur);
                    dest = nb;
                    break;
                case WM_BEETLE:
                    if (nb >= 0) {
                        int hd = P.height(nb), mh = hd > hcell - 1 ? hd : hcell - 1;
                        fin = mh > 0 ? !P.gate_blocked(cur, d, mh) : (bool)rowbit(w->sl[d], cur);
                        dest = nb;
                    }
                    break;
                case WM_HOP:
                    if (nb >= 0 && P.occupied(nb)) {
                        int p = nb;
#pragma unroll 1
                        while (p >= 0 && P.occupied(p)) p = nbr(p, d);
                        fin = p >= 0;
                        dest = p;
                    }
                    break;
                case WM_ANT:
                    if (rowbit(w->slx[d], cur)) {
                        dest = nb;
                        fin = !set_has(w->seen, nb);
                    }
                    break;
                case WM_SPIDER:
                    if (rowbit(w->slx[d], cur)) {
                        dest = nb;
                        if (lev == 0) app = true;
                        else if (nb != cell && (lev == 1 || nb != anc)) {
                            app = lev == 1;
                            fin = lev == 2;
                        }
                    }
                    break;
                default:  // WM_LADY
                    if (nb >= 0) {
                        dest = nb;
                        int hn = P.height(nb);
                        bool on = P.occupied(nb);
                        if (lev == 0) {
                            app = on && !P.gate_blocked(cur, d, hn > hcell - 1 ? hn : hcell - 1);
                        } else if (lev == 1) {
                            int hc = P.height(cur);
                            app = nb != cell && on && !P.gate_blocked(cur, d, hn > hc ? hn : hc);
                        } else {
                            fin = nb != cell && nb != anc && !on &&
                                  !P.gate_blocked(cur, d, P.height(cur));
                        }
                    }
                    break;
            }
            if (fin && mode >= WM_SPIDER) fin = !set_has(w->seen, dest);
        }
        if (first_only) {
            if (__ballot_sync(kFull, fin)) return 1;
        } else {
            uint32_t mm = __match_any_sync(kFull, fin ? dest : -1);  // one shared key for idle lanes
            bool keep = fin && ((mm & lt) == 0u);
            uint32_t b = __ballot_sync(kFull, keep);
            int pos = cnt + __popc(b & lt);
            if (keep && pos < cap) {
                out[pos] = (uint16_t)dest;
                set_add(w->seen, dest);
            }
            cnt = min(cap, cnt + __popc(b));
        }
        uint32_t ba = __ballot_sync(kFull, app);
        if (app) {
            int pos = wr + __popc(ba & lt);
            Q[pos] = (uint16_t)dest;
            w->qanc[pos] = (uint16_t)cur;
        }
        wr = mode == WM_ANT ? cnt : wr + __popc(ba);
        if (seed) l2start = wr;
        else rd += items;
        seed = false;
        __syncwarp();
        if (!first_only && cnt >= cap) break;
    }
    return first_only ? 0 : cnt;
}

// The walk engine out of line: one copy of its code serves every piece of
// the move generator.  (The compact list's existence tests inline
// walk_body instead: specialised to first_only, it is short.)
__device__ __noinline__ int walk(WarpSmem* w, int cell, int mode, uint16_t* out, int cap, bool first_only) {
    return walk_body(w, cell, mode, out, cap, first_only);
}

// The ant's breadth-first search (move_gen.cuh:267-388), the hottest walk:
// the walk engine's ant path without its mode dispatch and path bookkeeping.
// Lanes take (queue item, direction) pairs, five items per round; the queue
// is the output list, as in the reference, and first occurrences are kept in
// (item, direction) order -- the reference's sequential order.  Needs slx
// built for this cell.  The duplicate test is one match over the lanes that
// found a new cell: the idle lanes share one key, since a match costs the SM
// about two cycles per distinct key (unique idle keys made it the ant's
// dominant cost).
__device__ __noinline__ int ant_walk(WarpSmem* w, int cell, uint16_t* out, int cap) {
    const int l = lane_id();
    const uint32_t lt = lanemask_lt();
    const int k = l / 6, d = l - 6 * (l / 6);
    const uint32_t* slx = w->slx[d < 6 ? d : 0];
    const int step = dstep(d < 6 ? d : 0);
    set_clear(w->seen);
    if (l == 0) set_add(w->seen, cell);
    __syncwarp();
    int rd = -1, cnt = 0;  // rd < 0: the seed round (the ant's own cell)
#pragma unroll 1
    while (true) {
        const int items = cnt >= cap ? 0 : (rd < 0 ? 1 : min(5, cnt - rd));
        if (items <= 0) break;
        int dest = -1;
        bool fin = false;
        if (k < items) {
            const int cur = rd < 0 ? cell : out[rd + k];
            if (rowbit(slx, cur)) {
                dest = cur + step;
                fin = !set_has(w->seen, dest);
            }
        }
        const uint32_t mm = __match_any_sync(kFull, fin ? dest : -1);
        const bool keep = fin && ((mm & lt) == 0u);
        const uint32_t b = __ballot_sync(kFull, keep);
        const int pos = cnt + __popc(b & lt);
        if (keep && pos < cap) {
            out[pos] = (uint16_t)dest;
            set_add(w->seen, dest);
        }
        cnt = min(cap, cnt + __popc(b));
        rd = rd < 0 ? 0 : rd + items;
        __syncwarp();
    }
    return cnt;
}

// top types of the six neighbours, mosquito excluded (move_gen.cuh:917-925)
__device__ __forceinline__ uint32_t neighbour_types(WarpSmem* w, int cell) {
    Pos P{w};
    int l = lane_id();
    uint32_t t = 0;
    if (l < 6) {
        int nb = nbr(cell, l);
        if (nb >= 0 && P.occupied(nb)) {
            int pt = P.top(nb) & 15;
            if (pt != 6) t = 1u << pt;
        }
    }
    return __reduce_or_sync(kFull, t);
}

// ---------------------------------------------------------------------------
// existence of a move (the compact list's has_*_move predicates,
// move_gen.cuh:1416-1563): lane d tests direction d, one ballot.  Same tests
// as the walk engine's first round for these modes.
// ---------------------------------------------------------------------------
// queen / ant / pillbug: a slide out of the cell (lifting the piece does not
// change the slides out of its own cell, so the position's masks serve)
__device__ __forceinline__ bool slide_out(WarpSmem* w, int cell) {
    const int l = lane_id();
    return __ballot_sync(kFull, l < 6 && rowbit(w->sl[l < 6 ? l : 0], cell)) != 0u;
}

// beetle (or a stacked mosquito): elevated gate or slide (WM_BEETLE)
__device__ __forceinline__ bool beetle_out(WarpSmem* w, int cell) {
    Pos P{w};
    const int l = lane_id();
    bool ok = false;
    if (l < 6) {
        const int nb = nbr(cell, l);
        if (nb >= 0) {
            const int hc = P.height(cell), hd = P.height(nb), mh = hd > hc - 1 ? hd : hc - 1;
            ok = mh > 0 ? !P.gate_blocked(cell, l, mh) : (bool)rowbit(w->sl[l], cell);
        }
    }
    return __ballot_sync(kFull, ok) != 0u;
}

// grasshopper: over a line of pieces onto the first empty cell on the grid (WM_HOP)
__device__ __forceinline__ bool hop_out(WarpSmem* w, int cell) {
    Pos P{w};
    const int l = lane_id();
    bool ok = false;
    if (l < 6) {
        const int nb = nbr(cell, l);
        if (nb >= 0 && P.occupied(nb)) {
            int p = nb;
#pragma unroll 1
            while (p >= 0 && P.occupied(p)) p = nbr(p, l);
            ok = p >= 0;
        }
    }
    return __ballot_sync(kFull, ok) != 0u;
}

// walk mode of a piece type (1..8), pillbug moves like the queen
__device__ __forceinline__ int mode_of(int pt) {
    // Q A G S B M L P -> STEP ANT HOP SPIDER BEETLE (mosquito) LADY STEP
    return (int)((0x05014230u >> (4 * (pt - 1))) & 15u);
}

// Mosquito: beetle when stacked, otherwise the union of the neighbours'
// movements in Q/P, A, G, S, B, L order, first occurrence kept, capped at
// 128 (move_gen.cuh:907-1049).  Needs slx built for this cell.  The list goes
// to w->tmp.
__device__ __forceinline__ int gen_mosquito(WarpSmem* w, int cell, bool first_only, uint32_t* err) {
    Pos P{w};
    if (P.height(cell) > 1) return walk(w, cell, WM_BEETLE, w->tmp, 6, first_only);
    const uint32_t t = neighbour_types(w, cell);
    const int l = lane_id();
    const uint32_t lt = lanemask_lt();
    uint32_t* uni = w->pl;  // union set
    if (!first_only) set_clear(uni);
    int cnt = 0;
    // part order Q/P, A, G, S, B, L: walk modes 0 3 2 4 1 5, and the
    // neighbour type bits each part needs
#pragma unroll 1
    for (int part = 0; part < 6; part++) {
        const uint32_t need = part == 0 ? 0x102u : (part == 5 ? 0x80u : (1u << (part + 1)));
        if (!(t & need)) continue;
        const int mode = (int)((0x514230u >> (4 * part)) & 15u);
        int k = (mode == WM_ANT && !first_only) ? ant_walk(w, cell, w->dst, 128)
                                                : walk(w, cell, mode, w->dst, mode == WM_ANT ? 128 : 32, first_only);
        if (first_only) {
            if (k) return 1;
            continue;
        }
        if (mode == WM_ANT && k >= 128 && l == 0) atomicOr(err, kErrBuffer);
#pragma unroll 1
        for (int base = 0; base < k; base += 32) {
            int i = base + l;
            int v = i < k ? (int)w->dst[i] : -1;
            bool fresh = i < k && !set_has(uni, v);
            uint32_t b = __ballot_sync(kFull, fresh);
            int pos = cnt + __popc(b & lt);
            if (fresh) {
                if (pos < 128) w->tmp[pos] = (uint16_t)v;
                set_add(uni, v);
            }
            cnt = min(128, cnt + __popc(b));
            __syncwarp();
        }
    }
    return cnt;
}

// Does a mosquito have a move (gen_mosquito's first_only answer)?  Stacked:
// as a beetle.  On the ground: any copied movement has one; the cheap
// lane-per-direction tests go first, and the slide masks are rebuilt with
// the mosquito lifted only if a spider part is still to test.
__device__ __forceinline__ bool mosquito_out(WarpSmem* w, uint32_t occ_row, int cell) {
    Pos P{w};
    if (P.height(cell) > 1) return beetle_out(w, cell);
    const uint32_t t = neighbour_types(w, cell);
    if ((t & 0x106u) && slide_out(w, cell)) return true;  // queen, pillbug, ant
    if ((t & 0x8u) && hop_out(w, cell)) return true;      // grasshopper
    if ((t & 0x20u) && beetle_out(w, cell)) return true;  // beetle
    if ((t & 0x80u) && walk_body(w, cell, WM_LADY, w->dst, 32, true)) return true;
    if (t & 0x10u) {                                      // spider
        lift_mover(w, occ_row, cell);
        return walk_body(w, cell, WM_SPIDER, w->dst, 32, true) != 0;
    }
    return false;
}

// Destinations of one own piece; returns the list (w->dst or w->tmp) and count.
__device__ __forceinline__ int piece_moves(WarpSmem* w, uint32_t occ_row, int cell, int pt, int cap,
                                           bool first_only, uint32_t* err, const uint16_t** list) {
    *list = w->dst;
    if (pt == 2 || pt == 4 || pt == 6) lift_mover(w, occ_row, cell);
    if (pt == 6) {
        *list = w->tmp;
        return gen_mosquito(w, cell, first_only, err);
    }
    if (pt < 1 || pt > 8) return 0;
    int mode = mode_of(pt);
    int c = mode == WM_ANT ? cap : (mode >= WM_SPIDER ? 32 : 6);
    if (mode == WM_ANT && !first_only) return ant_walk(w, cell, w->dst, c);
    return walk(w, cell, mode, w->dst, c, first_only);
}

// Is the cell of a piece in `lanes` (piece-list indices) a neighbour of
// cell?  Neighbours differ by +-1, +-31 or +-32 on the padded grid, and no
// other pair of cells does (a row's padding columns hold no piece).
__device__ __forceinline__ bool next_to_any(const WarpSmem* w, uint32_t lanes, int cell) {
#pragma unroll 1
    while (lanes) {
        const int j = __ffs(lanes) - 1;
        lanes &= lanes - 1;
        const int dp = (int)w->pcell[j] - cell, a = dp < 0 ? -dp : dp;
        if (a == 1 || a == 31 || a == 32) return true;
    }
    return false;
}

// Is any neighbour topped by a pillbug (move_gen.cuh:1326-1336)?
__device__ __forceinline__ bool next_to_pillbug(WarpSmem* w, int cell) {
    Pos P{w};
#pragma unroll 1
    for (int d = 0; d < 6; d++) {
        int nb = nbr(cell, d);
        if (nb >= 0 && P.occupied(nb) && (P.top(nb) & 15) == 8) return true;
    }
    return false;
}

// Pillbug throws from thrower pb: valid targets x valid drop cells, in
// (target direction, drop direction) order (move_gen.cuh:691-769).
__device__ __noinline__ void throw_sets(WarpSmem* w, int pb, uint32_t& tmask, uint32_t& dmask) {
    Pos P{w};
    int l = lane_id();
    int pbh = P.height(pb);
    int stun = P.stunned();
    bool okt = false, okd = false;
    if (l < 6) {
        int t = nbr(pb, l);
        if (t >= 0 && P.occupied(t) && P.height(t) == 1 && stun != t) {
            int j = P.pidx(t);
            bool pinned = j < 32 && (w->pflag[j] & 1);
            if (!pinned) {
                int ht = P.height(t) - 1;
                okt = !P.gate_blocked(t, opp_dir(l), ht > pbh ? ht : pbh);
            }
        }
        okd = t >= 0 && !P.occupied(t) && !P.gate_blocked(pb, l, pbh);
    }
    tmask = __ballot_sync(kFull, okt);
    dmask = __ballot_sync(kFull, okd);
}

// ---------------------------------------------------------------------------
// placement cells (move_gen.cuh:1064-1140) into w->prow / w->ppref
// ---------------------------------------------------------------------------
__device__ __forceinline__ int placement_cells(WarpSmem* w, uint32_t occ, uint32_t own, uint32_t opp,
                                            int turn) {
    int l = lane_id();
    uint32_t p;
    if (turn == 0) p = (l == 11) ? (1u << 11) : 0u;
    else if (turn == 1) p = dilate(occ) & ~occ;
    else p = dilate(own) & ~occ & ~dilate(opp);
    p &= row_valid_mask();
    int c = __popc(p);
    int pre = warp_excl_scan(c);
    if (l < 24) {
        w->prow[l] = p;
        w->ppref[l] = (uint16_t)pre;
    }
    __syncwarp();
    return __shfl_sync(kFull, pre + c, 31);
}

// The placement cells of w->prow in ascending order, as reference cell
// indices, into w->dst (free until the first mover's walk): lane r lists the
// cells of row r from the row's prefix count, so that a placement move
// finds its cell by one load instead of a search over the rows.  At most
// 6 x 14 cells border the side's pieces, inside dst's 128 entries.
__device__ __forceinline__ void placement_list(WarpSmem* w) {
    const int l = lane_id();
    if (l < kBoard) {
        uint32_t bits = w->prow[l];
        int k = w->ppref[l];
#pragma unroll 1
        while (bits) {
            const int q = __ffs(bits) - 1;
            bits &= bits - 1;
            if (k < 128) w->dst[k] = (uint16_t)p_to_c((l << 5) + q);
            k++;
        }
    }
    __syncwarp();
}

// placeable piece-type mask of the side to move (move_gen.cuh:1161-1174)
static_assert(kOffHands % 4 == 0, "the hand counts are read as 32-bit words");
__device__ __forceinline__ uint32_t placeable_types(const Pos& P, int color, bool forced) {
    // the eight hand counts as two words: bit 7 of a byte is set iff the byte
    // is nonzero, then bits 7, 15, 23, 31 move to 0..3 by one multiply (the
    // partial products land on distinct bits)
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(P.w->st + kOffHands + color * 8);
    auto nz4 = [](uint32_t x) {
        x = (((x & 0x7f7f7f7fu) + 0x7f7f7f7fu) | x) & 0x80808080u;
        return (((x >> 7) * 0x00204081u) >> 21) & 15u;
    };
    const uint32_t m = nz4(hw[0]) | (nz4(hw[1]) << 4);
    return forced ? (m & 1u) : m;
}

// ---------------------------------------------------------------------------
// full legal move list -> w->mv, returns the count
// ---------------------------------------------------------------------------
// Inlined into its kernels, with placement_cells and gen_mosquito: the calls'
// saved registers went through local memory once per position (generator
// 1.81 -> 1.52 ms per 262,144 positions); the walks stay out of line (their
// code is shared by every piece, and inlining them spilled).  S: the Setup
// that setup_position returned for the staged position.
__device__ __forceinline__ int gen_legal(WarpSmem* w, const Setup& S, uint32_t* err) {
    Pos P{w};
    int l = lane_id();
    if (P.result() != 0) return 0;
    const int color = S.color, turn = P.turn(), ptn = turn >> 1;
    const bool queen_down = (P.queen_placed() >> color) & 1;
    const uint32_t placeable = placeable_types(P, color, ptn == 3 && !queen_down);
    int count = 0;
    if (placeable) {
        int np = placement_cells(w, S.occ, S.own, S.opp, turn);
        uint32_t types = placeable & ~(ptn == 0 ? 1u : 0u);
        int nt = __popc(types);
        int total = np * nt;
        if (total > kMaxMoves) total = kMaxMoves;
        placement_list(w);
        // cell-major, type-minor (move k * nt + j): a lane per cell writes its
        // cell's types in ascending order
#pragma unroll 1
        for (int k = l; k < np && k * nt < total; k += 32) {
            const int c = w->dst[k < 128 ? k : 127];
            uint32_t t = types;
#pragma unroll 1
            for (int m = k * nt; t && m < total; m++) {
                put_move(w, m, 0, __ffs(t), 0, c);
                t &= t - 1;
            }
        }
        count = total;
    }
    if (queen_down) {
        const int stun = P.stunned();
        // own top pieces according to the side's top bitboard
        bool mine = S.my_cell >= 0 && rowbit(w->own, S.my_cell);
        // movers: own, not stunned, not pinned (move_gen.cuh:1221-1234)
        bool mov = mine && stun != S.my_cell && !(w->pflag[l] & 1);
        uint32_t movers = __ballot_sync(kFull, mov);
#pragma unroll 1
        while (movers) {
            int i = __ffs(movers) - 1;
            movers &= movers - 1;
            int cell = w->pcell[i];
            int pt = P.top(cell) & 15;
            int room = kMaxMoves - count;
            const uint16_t* list;
            int k = piece_moves(w, S.occ, cell, pt, room < 128 ? room : 128, false, err, &list);
            if (pt == 2 && k >= 128 && room > 128 && l == 0) atomicOr(err, kErrBuffer);
            const int from_c = p_to_c(cell);
#pragma unroll 1
            for (int m = l; m < k; m += 32)
                if (count + m < kMaxMoves) put_move(w, count + m, 1, pt, from_c, p_to_c(list[m]));
            count = min(kMaxMoves, count + k);
            __syncwarp();
        }
        // throws by own pillbugs and pillbug-adjacent ground mosquitoes
        // (the piece lane's fields read again: nothing held across the calls)
        const Setup T = reload_setup(w);
        const int mt = T.my_top & 15;
        // cells topped by a pillbug, of either side (move_gen.cuh:1326-1336)
        const uint32_t pbt = __ballot_sync(kFull, T.my_cell >= 0 && mt == 8);
        const bool thr = T.my_cell >= 0 && rowbit(w->own, T.my_cell) &&
                         (mt == 8 || (mt == 6 && T.my_h == 1 && next_to_any(w, pbt, T.my_cell)));
        uint32_t throwers = __ballot_sync(kFull, thr);
#pragma unroll 1
        while (throwers) {
            int i = __ffs(throwers) - 1;
            throwers &= throwers - 1;
            int pb = w->pcell[i];
            uint32_t tm, dm;
            throw_sets(w, pb, tm, dm);
            int nt = __popc(tm), nd = __popc(dm), total = nt * nd;
            // m / nd for m < 64 and nd <= 6 as a multiply by 2^16 / nd + 1
            // (exact over that range), no integer division per move
            const uint32_t inv = nd ? 0x10000u / (uint32_t)nd + 1u : 0u;
#pragma unroll 1
            for (int m = l; m < total; m += 32) {
                int kt = (int)(((uint32_t)m * inv) >> 16), kd = m - kt * nd;
                int target = nbr(pb, __fns(tm, 0, kt + 1));
                int dest = nbr(pb, __fns(dm, 0, kd + 1));
                if (count + m < kMaxMoves)
                    put_move(w, count + m, 1, P.top(target) & 15, p_to_c(target), p_to_c(dest));
            }
            count = min(kMaxMoves, count + total);
            __syncwarp();
        }
    }
    if (count == 0) {
        if (l == 0) put_move(w, 0, 2, 0, 0, 0);
        count = 1;
    }
    __syncwarp();
    return count;
}

// the same from the Setup of the staged position, re-read from the warp slot
__device__ __forceinline__ int gen_legal(WarpSmem* w, uint32_t* err) { return gen_legal(w, reload_setup(w), err); }

// ---------------------------------------------------------------------------
// compact list for successor features (move_gen.cuh:1362-1563)
// ---------------------------------------------------------------------------
// (gen_compact_body is the inlined form, for the successor kernel: a call's
// saved registers cost local-memory traffic per row there, and the kernel
// measured 7 to 9 % faster with both of its callees inlined)
__device__ __forceinline__ int gen_compact_body(WarpSmem* w, uint32_t* err) {
    const Setup S = reload_setup(w);
    Pos P{w};
    int l = lane_id();
    if (P.result() != 0) return 0;
    const int color = S.color, turn = P.turn(), ptn = turn >> 1;
    const bool queen_down = (P.queen_placed() >> color) & 1;
    const uint32_t any = placeable_types(P, color, ptn == 3 && !queen_down) & ~(ptn == 0 ? 1u : 0u);
    int count = 0;
    if (any) {
        int np = placement_cells(w, S.occ, S.own, S.opp, turn);
        int total = np < kMaxMoves ? np : kMaxMoves;
        placement_list(w);
#pragma unroll 1
        for (int m = l; m < total; m += 32) put_move(w, m, 0, 0, 0, w->dst[m < 128 ? m : 127]);
        count = total;
    }
    if (!queen_down || count >= kMaxMoves) {
        if (count == 0) {
            if (l == 0) put_move(w, 0, 2, 0, 0, 0);
            count = 1;
        }
        __syncwarp();
        return count;
    }
    const int stun = P.stunned();
    bool mine = S.my_cell >= 0 && rowbit(w->own, S.my_cell);
    bool mov = mine && stun != S.my_cell && !(w->pflag[l] & 1);
    uint32_t movers = __ballot_sync(kFull, mov);
    uint32_t seen = 0;  // (type, owner) flags, emit_fnn_move_flag move_gen.cuh:1362-1377
#pragma unroll 1
    while (movers && count < kMaxMoves) {
        int i = __ffs(movers) - 1;
        movers &= movers - 1;
        int cell = w->pcell[i];
        int pt = P.top(cell) & 15;
        uint32_t bit = 1u << ((pt - 1) * 2 + color);
        if (seen & bit) continue;
        // queen, ant, pillbug: a move exists iff one slide out of the cell is
        // legal (the first step of each; lifting the piece does not change
        // slides out of its own cell), read from the position's slide masks
        bool has;
        if (pt == 1 || pt == 2 || pt == 8) has = slide_out(w, cell);
        else if (pt == 3) has = hop_out(w, cell);
        else if (pt == 5) has = beetle_out(w, cell);
        else if (pt == 6) has = mosquito_out(w, S.occ, cell);
        else if (pt == 4) {  // spider: three slides with the spider lifted
            lift_mover(w, S.occ, cell);
            has = walk_body(w, cell, WM_SPIDER, w->dst, 32, true) != 0;
        } else if (pt == 7) {  // ladybug
            has = walk_body(w, cell, WM_LADY, w->dst, 32, true) != 0;
        } else {
            has = false;
        }
        if (has) {
            seen |= bit;
            if (l == 0) put_move(w, count, 1, pt, p_to_c(cell), 0);
            count++;
        }
        __syncwarp();
    }
    const Setup T = reload_setup(w);
    const int mt = T.my_top & 15;
    // cells topped by a pillbug, of either side (move_gen.cuh:1326-1336)
    const uint32_t pbt = __ballot_sync(kFull, T.my_cell >= 0 && mt == 8);
    const bool thr = T.my_cell >= 0 && rowbit(w->own, T.my_cell) &&
                     (mt == 8 || (mt == 6 && T.my_h == 1 && next_to_any(w, pbt, T.my_cell)));
    uint32_t throwers = __ballot_sync(kFull, thr);
#pragma unroll 1
    while (throwers && count < kMaxMoves) {
        int i = __ffs(throwers) - 1;
        throwers &= throwers - 1;
        int pb = w->pcell[i];
        uint32_t tm, dm;
        throw_sets(w, pb, tm, dm);
        if (dm == 0u) continue;
        // summarize_pillbug_throws_for_fnn, move_gen.cuh:1379-1410: targets in
        // direction order, one entry per (type, owner) not seen yet.  Lane d
        // takes target d; of the targets sharing a new (type, owner) the
        // lowest direction is kept, as the sequential scan keeps the first.
        const int target = (l < 6 && ((tm >> l) & 1u)) ? nbr(pb, l) : -1;
        const int tt = target >= 0 ? P.top(target) : 0;
        const bool live = target >= 0 && P.height(target) > 0;
        const uint32_t bit = live ? 1u << (((tt & 15) - 1) * 2 + ((tt >> 4) & 1)) : 0u;
        const bool fresh = live && !(seen & bit);
        const uint32_t grp = __match_any_sync(kFull, fresh ? (int)bit : -1);
        const bool keep = fresh && (grp & lanemask_lt()) == 0u;
        const uint32_t kb = __ballot_sync(kFull, keep);
        const int pos = count + __popc(kb & lanemask_lt());
        if (keep && pos < kMaxMoves) put_move(w, pos, 1, tt & 15, p_to_c(target), 0);
        // entries past the list's end are dropped, and so are their flags
        seen |= __reduce_or_sync(kFull, (keep && pos < kMaxMoves) ? bit : 0u);
        count = min(kMaxMoves, count + __popc(kb));
        __syncwarp();
    }
    if (count == 0) {
        if (l == 0) put_move(w, 0, 2, 0, 0, 0);
        count = 1;
    }
    __syncwarp();
    return count;
}

// ---------------------------------------------------------------------------
// 122-float FNN features (fnn_features.cuh:68-331) from state + move list
// ---------------------------------------------------------------------------
enum : int {
    A_CNT = 0, A_QADJ = 16, A_DSUM = 32, A_DCNT = 48, A_SRC = 64, A_AP = 80,
    A_SINGLE = 96, A_COVER = 98, A_CAP = 100, A_TOWN = 102, A_TOPP = 104,
    A_PLACE = 106, A_SURR = 107, A_N = 110
};

// top byte of a reference-index cell c (< 529)
__device__ __forceinline__ int top_c(const WarpSmem* w, int c) {
    int h = w->st[kOffHeight + c];
    h = h > 5 ? 5 : h;
    return h ? w->st[(h - 1) * kCells + c] : 0;
}

// RUNS: the list is a full legal list, whose moves come in runs (the moves
// of one piece, the types placed on one cell): the source-cell and
// placement sets are then set once per run instead of by every lane of it
// (atomics of one instruction to one word serialise).  A compact list has
// one entry per (type, owner) and per placement cell: no runs to skip.
template <bool RUNS = false>
__device__ __forceinline__ void features_body(WarpSmem* w, int nmoves, float* out) {
    const Setup S = reload_setup(w);
    Pos P{w};
    int l = lane_id();
    {
        // accumulators and source-cell sets are contiguous: 16-byte stores
        static_assert(sizeof(w->acc) % 16 == 0 && (sizeof(w->acc) + sizeof(w->bm)) % 16 == 0, "acc/bm layout");
        uint4* z = reinterpret_cast<uint4*>(w->acc);
#pragma unroll
        for (int i = l; i < (int)(sizeof(w->acc) + sizeof(w->bm)) / 16; i += 32) z[i] = make_uint4(0u, 0u, 0u, 0u);
        if (l < 17) w->pl[l] = 0u;
    }
    __syncwarp();
    const int turn = P.turn(), cur = turn & 1, stun = P.stunned();
    const int q0 = P.queen_cell(0), q1 = P.queen_cell(1);
    const int cell = S.my_cell, h = S.my_h, top = S.my_top;
    const int pt = top & 15, col = (top >> 4) & 1, tc = (pt - 1) * 2 + col;
    bool capable = false;
    bool adjq0 = false, adjq1 = false;
    // the pieces whose cell is topped by a pillbug that is not stunned
    const uint32_t pbm = __ballot_sync(kFull, cell >= 0 && pt == 8 && stun != cell);
    if (cell >= 0 && pt >= 1 && pt <= 8) {
        atomicAdd(&w->acc[A_CNT + tc], 1);
        // occupied neighbours from the occupancy row words (a cell is
        // occupied iff its height is nonzero; padding bits are zero): row r-1
        // columns q, q+1; row r columns q-1, q+1; row r+1 columns q-1, q
        const int rr = cell >> 5, qq = cell & 31;
        const uint32_t up = rr ? w->occ[rr - 1] : 0u, mid = w->occ[rr], dn = w->occ[rr + 1];
        const int occn =
            __popc(((up >> qq) & 3u) | ((((mid << 1) >> qq) & 5u) << 2) | ((((dn << 1) >> qq) & 3u) << 5));
        if (occn == 0) atomicAdd(&w->acc[A_SINGLE + col], 1);
        int oq = col ? q0 : q1;
        if (oq >= 0) {
            int dist = hex_distance(cell, oq);
            if (oq < kPCells && dist == 1) atomicAdd(&w->acc[A_QADJ + tc], 1);
            atomicAdd(&w->acc[A_DSUM + tc], dist);
            atomicAdd(&w->acc[A_DCNT + tc], 1);
        }
        adjq0 = q0 >= 0 && q0 < kPCells && hex_distance(cell, q0) == 1;
        adjq1 = q1 >= 0 && q1 < kPCells && hex_distance(cell, q1) == 1;
        if (h == 1 && S.my_ap) atomicAdd(&w->acc[A_AP + tc], 1);
        if (pt != 1) {
            const int c = p_to_c(cell);
#pragma unroll 1
            for (int lv = 0; lv < h - 1 && lv < 4; lv++) {
                int b = w->st[lv * kCells + c];
                if ((b & 15) == 1) w->acc[A_COVER + ((b >> 4) & 1)] = 1;
            }
        }
        capable = stun != cell && pt == 8;
        if (!capable && stun != cell && pt == 6 && h == 1) capable = next_to_any(w, pbm, cell);
        if (capable) w->acc[A_CAP + col] = 1;
    }
    uint32_t s0 = __ballot_sync(kFull, adjq0), s1 = __ballot_sync(kFull, adjq1);
    // throwable counts from the first eight capable cells of each colour
    uint32_t cap0 = __ballot_sync(kFull, capable && col == 0);
    uint32_t cap1 = __ballot_sync(kFull, capable && col == 1);
    if (capable && __popc((col ? cap1 : cap0) & lanemask_lt()) < 8) {
        // occupied neighbours and those topped by the side to move, from the
        // row words (bits: row r-1 q, q+1 -> 0, 1; row r q-1, q+1 -> 2, 4;
        // row r+1 q-1, q -> 5, 6), the stunned cell taken out; a cell's top
        // piece belongs to the side to move or to the other side
        const int rr = cell >> 5, qq = cell & 31;
        auto nb7 = [&](const uint32_t* rows) {
            const uint32_t up = rr ? rows[rr - 1] : 0u, mid = rows[rr], dn = rows[rr + 1];
            return ((up >> qq) & 3u) | ((((mid << 1) >> qq) & 5u) << 2) | ((((dn << 1) >> qq) & 3u) << 5);
        };
        uint32_t occm = nb7(w->occ), ownm = nb7(w->own);
        if (stun >= 0) {
            const int dr = (stun >> 5) - rr + 1, dc = (stun & 31) - qq + 1;
            if ((unsigned)dr < 3u && (unsigned)dc < 3u) {
                // bit of (dr, dc) in row-major 3 x 3 order; 7 (outside the code) for none
                const uint32_t bit = (uint32_t)((0x765472107ull >> (4 * (dr * 3 + dc))) & 15ull);
                occm &= ~(1u << bit);
                ownm &= ~(1u << bit);
            }
        }
        const int n_occ = __popc(occm), n_own = __popc(ownm);
        const int same = col == cur ? n_own : n_occ - n_own;
        if (same) atomicAdd(&w->acc[A_TOWN + col], same);
        if (n_occ - same) atomicAdd(&w->acc[A_TOPP + (col ^ 1)], n_occ - same);
    }
    // source cells per (type, owner) and placement cells from the list
    if (RUNS) {
#pragma unroll 1
        for (int base = 0; base < nmoves; base += 32) {
            const int m = base + l;
            // the bit a move sets: (piece type, source cell) for a movement,
            // the cell for a placement; in a run of equal keys only the
            // first lane sets it (the owner is that of the cell's top piece)
            int key = -1;
            if (m < nmoves) {
                const int tp = w->mv[3 * m], from = w->mv[3 * m + 1], to = w->mv[3 * m + 2];
                const int type = tp & 255, mpt = tp >> 8;
                if (type == 1) {
                    if (mpt >= 1 && mpt <= 8 && from < kCells) key = (mpt << 10) | from;
                } else if (type == 0 && to < kCells) {
                    key = (1 << 14) | to;
                }
            }
            const int prev = __shfl_up_sync(kFull, key, 1);
            if (key >= 0 && (l == 0 || prev != key)) {
                const int c = key & 1023;
                if (key >> 14) {
                    atomicOr(&w->pl[c >> 5], 1u << (c & 31));
                } else {
                    const int owner = w->st[kOffHeight + c] > 0 ? ((top_c(w, c) >> 4) & 1) : cur;
                    atomicOr(&w->bm[(((key >> 10) - 1) * 2 + owner) * 17 + (c >> 5)], 1u << (c & 31));
                }
            }
        }
    } else {
#pragma unroll 1
        for (int m = l; m < nmoves; m += 32) {
            int tp = w->mv[3 * m], from = w->mv[3 * m + 1], to = w->mv[3 * m + 2];
            int type = tp & 255, mpt = tp >> 8;
            if (type == 1) {
                if (mpt >= 1 && mpt <= 8 && from < kCells) {
                    int owner = w->st[kOffHeight + from] > 0 ? ((top_c(w, from) >> 4) & 1) : cur;
                    atomicOr(&w->bm[((mpt - 1) * 2 + owner) * 17 + (from >> 5)], 1u << (from & 31));
                }
            } else if (type == 0 && to < kCells) {
                atomicOr(&w->pl[to >> 5], 1u << (to & 31));
            }
        }
    }
    __syncwarp();
    // lane t < 16 counts the source cells of (type, owner) t, lane 16 the
    // placement cells: 17 words each (stride 17: no bank conflicts)
    if (l <= 16) {
        const uint32_t* set = l < 16 ? &w->bm[l * 17] : w->pl;
        int c = 0;
#pragma unroll
        for (int k = 0; k < 17; k++) c += __popc(set[k]);
        w->acc[l < 16 ? A_SRC + l : A_PLACE] = c;
    }
    if (l == 0) {
        w->acc[A_SURR] = __popc(s0);
        w->acc[A_SURR + 1] = __popc(s1);
    }
    __syncwarp();
    // write-out in three uniform lane groups (no per-lane formula switch)
    if (l < 16) {
        out[l] = (float)w->acc[A_CNT + l];
        out[32 + l] = (float)w->acc[A_QADJ + l];
        out[64 + l] = (float)w->acc[A_SRC + l];
        out[80 + l] = (float)w->acc[A_AP + l];
        const int t = l >> 1;
        const float per = (t == 1 || t == 2) ? 3.0f : ((t == 3 || t == 4) ? 2.0f : 1.0f);
        out[16 + l] = (float)P.hand(l & 1, t) / per;
        const int n = w->acc[A_DCNT + l];
        out[48 + l] = n > 0 ? (float)w->acc[A_DSUM + l] / (float)n / 10.0f : 0.0f;
    } else if (l < 28) {
        const int j = l - 16, qc = j >= 6, b = j - 6 * qc;
        out[110 + j] = w->acc[A_SURR + qc] == b + 1 ? 1.0f : 0.0f;
    } else {
        // lanes 28..31: features 96..109, up to four each
        const int j = l - 28;
        const int left = 200 - turn;
        const float tt = (float)turn / 100.0f;
        float v[4];
        if (j == 0) {  // 96..99
            v[0] = (float)w->acc[A_SINGLE];
            v[1] = (float)w->acc[A_SINGLE + 1];
            v[2] = (float)w->acc[A_COVER];
            v[3] = (float)w->acc[A_COVER + 1];
        } else if (j == 1) {  // 100..103
            const float pl = (float)w->acc[A_PLACE] / 10.0f;
            v[0] = cur == 0 ? pl : 0.0f;
            v[1] = cur == 1 ? pl : 0.0f;
            v[2] = (float)(left < 0 ? 0 : left) / 200.0f;
            v[3] = tt < 1.0f ? tt : 1.0f;
        } else if (j == 2) {  // 104..107
            v[0] = (float)w->acc[A_CAP];
            v[1] = (float)w->acc[A_CAP + 1];
            v[2] = (float)w->acc[A_TOWN];
            v[3] = (float)w->acc[A_TOWN + 1];
        } else {  // 108..109
            v[0] = (float)w->acc[A_TOPP];
            v[1] = (float)w->acc[A_TOPP + 1];
        }
        const int base = 96 + 4 * j, cntv = j == 3 ? 2 : 4;
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (i < cntv) out[base + i] = v[i];
    }
    __syncwarp();
}

// out-of-line forms for the kernels that are not bound by their calls
__device__ __noinline__ int gen_compact(WarpSmem* w, uint32_t* err) { return gen_compact_body(w, err); }
__device__ __noinline__ void features(WarpSmem* w, int nmoves, float* out) { features_body(w, nmoves, out); }
// the features of a position from its full legal list
__device__ __noinline__ void features_full(WarpSmem* w, int nmoves, float* out) {
    features_body<true>(w, nmoves, out);
}

}  // namespace hv
