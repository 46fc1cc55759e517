// hv_movegen.cuh -- warp-cooperative legal move generation, the compact
// successor list and the 122-float FNN features (sm_100a).
//
// Semantics follow the reference exactly (it is the parity target):
//   full list      hive_gpu/csrc/move_gen.cuh:1151-1360
//   compact list   hive_gpu/csrc/move_gen.cuh:1362-1563
//   features       hive_gpu/csrc/fnn_features.cuh:68-331
// including its emission order, duplicates (throws vs. ordinary moves),
// truncation at 256 moves, 32-destination caps for spider/ladybug and the
// 128-destination cap of a mosquito's union.
#pragma once

#include "hv_core.cuh"

namespace hv {

__device__ __forceinline__ void put_move(WarpSmem* w, int m, int type, int pt, int from, int to) {
    w->mv[3 * m] = (uint16_t)(type | (pt << 8));
    w->mv[3 * m + 1] = (uint16_t)from;
    w->mv[3 * m + 2] = (uint16_t)to;
}

__device__ __forceinline__ bool set_has(const uint32_t* s, int c) { return (s[c >> 5] >> (c & 31)) & 1u; }
__device__ __forceinline__ void set_add(uint32_t* s, int c) { atomicOr(&s[c >> 5], 1u << (c & 31)); }
__device__ __forceinline__ void set_clear(uint32_t* s) {
    if (lane_id() < 18) s[lane_id()] = 0u;
    __syncwarp();
}

// occupancy minus one cell -> slx (the mover is lifted off the board)
__device__ __forceinline__ void lift_mover(WarpSmem* w, uint32_t occ_row, int cell) {
    int l = lane_id();
    int r = cell / kBoard;
    uint32_t x = occ_row;
    if (l == r) x &= ~(1u << (cell - r * kBoard));
    build_slide_masks(x, w->slx);
    __syncwarp();
}

// one-step slide in the six directions (queen / pillbug), move_gen.cuh:202-212
__device__ __forceinline__ int gen_step1(WarpSmem* w, int cell, uint16_t* out, bool first_only) {
    int l = lane_id();
    bool ok = l < 6 && rowbit(w->sl[l], cell);
    uint32_t b = __ballot_sync(kFull, ok);
    if (first_only) return b ? 1 : 0;
    if (ok) out[__popc(b & lanemask_lt())] = (uint16_t)nbr(cell, l);
    __syncwarp();
    return __popc(b);
}

// grasshopper jumps, move_gen.cuh:228-257
__device__ __forceinline__ int gen_hopper(WarpSmem* w, int cell, uint16_t* out, bool first_only) {
    Pos P{w};
    int l = lane_id();
    bool ok = false;
    int p = -1;
    if (l < 6) {
        p = nbr(cell, l);
        if (p >= 0 && P.occupied(p)) {
            while (p >= 0 && P.occupied(p)) p = nbr(p, l);
            ok = p >= 0;
        }
    }
    uint32_t b = __ballot_sync(kFull, ok);
    if (first_only) return b ? 1 : 0;
    if (ok) out[__popc(b & lanemask_lt())] = (uint16_t)p;
    __syncwarp();
    return __popc(b);
}

// beetle: elevated gate or ground slide, move_gen.cuh:468-524
__device__ __forceinline__ int gen_beetle(WarpSmem* w, int cell, uint16_t* out, bool first_only) {
    Pos P{w};
    int l = lane_id();
    bool ok = false;
    int dest = -1;
    if (l < 6) {
        dest = nbr(cell, l);
        if (dest >= 0) {
            int below = P.height(cell) - 1;
            int hd = P.height(dest);
            int mh = hd > below ? hd : below;
            ok = mh > 0 ? !P.gate_blocked(cell, l, mh) : (bool)rowbit(w->sl[l], cell);
        }
    }
    uint32_t b = __ballot_sync(kFull, ok);
    if (first_only) return b ? 1 : 0;
    if (ok) out[__popc(b & lanemask_lt())] = (uint16_t)dest;
    __syncwarp();
    return __popc(b);
}

// Ant breadth-first search over slide steps with the ant lifted (slx).
// Lanes take (queue item, direction) pairs, five items per round; the
// lowest lane wins a shared destination, which is exactly the reference's
// sequential first-seen order (move_gen.cuh:267-313, 348-388).
// out doubles as the queue; at most cap (<= 128) entries.
__device__ __forceinline__ int gen_ant(WarpSmem* w, int cell, uint16_t* out, int cap,
                                       bool first_only) {
    int l = lane_id();
    if (first_only) {
        bool ok = l < 6 && rowbit(w->slx[l], cell);
        return __ballot_sync(kFull, ok) ? 1 : 0;
    }
    if (cap <= 0) return 0;
    set_clear(w->seen);
    if (l == 0) set_add(w->seen, cell);
    __syncwarp();
    int rd = 0, wr = 0;
    bool seed = true;
    const uint32_t lt = lanemask_lt();
    const int k = l / 6, d = l - (l / 6) * 6;
    while (seed || (rd < wr && wr < cap)) {
        int items = seed ? 1 : min(5, wr - rd);
        bool ok = false;
        int dest = -1;
        if (k < items) {
            int cur = seed ? cell : (int)out[rd + k];
            if (rowbit(w->slx[d], cur)) {
                dest = nbr(cur, d);
                ok = !set_has(w->seen, dest);
            }
        }
        uint32_t mm = __match_any_sync(kFull, ok ? dest : -1 - l);
        bool keep = ok && ((mm & lt) == 0u);
        uint32_t b = __ballot_sync(kFull, keep);
        int pos = wr + __popc(b & lt);
        if (keep && pos < cap) {
            out[pos] = (uint16_t)dest;
            set_add(w->seen, dest);
        }
        wr = min(cap, wr + __popc(b));
        if (!seed) rd += items;
        seed = false;
        __syncwarp();
    }
    return wr;
}

// Three-step walks: spider (three slides, no revisits, move_gen.cuh:397-454)
// and ladybug (up, across, down, move_gen.cuh:538-637).  Candidates are
// enumerated level by level in (d1, d2, d3) lexicographic order, 32 per
// round; duplicates keep their first occurrence; at most 32 destinations.
template <bool LADY>
__device__ __noinline__ int gen_walk3(WarpSmem* w, int cell, uint16_t* out, bool first_only) {
    Pos P{w};
    int l = lane_id();
    const uint32_t lt = lanemask_lt();
    bool v1 = false;
    int p1 = -1;
    if (l < 6) {
        if (!LADY) {
            v1 = rowbit(w->slx[l], cell);
            p1 = v1 ? nbr(cell, l) : -1;
        } else {
            p1 = nbr(cell, l);
            if (p1 >= 0 && P.occupied(p1)) {
                int a = P.height(cell) - 1, b = P.height(p1);
                v1 = !P.gate_blocked(cell, l, a > b ? a : b);
            }
        }
    }
    uint32_t b1 = __ballot_sync(kFull, v1);
    int c1 = 6 * __popc(b1);
    int n2 = 0;
    for (int base = 0; base < c1; base += 32) {
        int c = base + l;
        bool in = c < c1;
        int k1 = c / 6, d2 = c - (c / 6) * 6;
        int src = in ? __fns(b1, 0, k1 + 1) : 0;
        int a = __shfl_sync(kFull, p1, src & 31);
        bool v2 = false;
        int bcell = -1;
        if (in) {
            if (!LADY) {
                if (rowbit(w->slx[d2], a)) {
                    bcell = nbr(a, d2);
                    v2 = bcell != cell && bcell != a;
                }
            } else {
                bcell = nbr(a, d2);
                if (bcell >= 0 && bcell != cell && P.occupied(bcell)) {
                    int ha = P.height(a), hb = P.height(bcell);
                    v2 = !P.gate_blocked(a, d2, ha > hb ? ha : hb);
                }
            }
        }
        uint32_t b2 = __ballot_sync(kFull, v2);
        if (v2) {
            int pos = n2 + __popc(b2 & lt);
            w->l2a[pos] = (uint16_t)a;
            w->l2b[pos] = (uint16_t)bcell;
        }
        n2 += __popc(b2);
    }
    __syncwarp();
    if (!first_only) set_clear(w->seen);
    int c3 = 6 * n2, cnt = 0;
    for (int base = 0; base < c3; base += 32) {
        int c = base + l;
        bool v3 = false;
        int p3 = -1;
        if (c < c3) {
            int k2 = c / 6, d3 = c - (c / 6) * 6;
            int a = w->l2a[k2], bcell = w->l2b[k2];
            if (!LADY) {
                if (rowbit(w->slx[d3], bcell)) {
                    p3 = nbr(bcell, d3);
                    v3 = p3 != cell && p3 != a && p3 != bcell;
                }
            } else {
                p3 = nbr(bcell, d3);
                v3 = p3 >= 0 && p3 != cell && p3 != a && !P.occupied(p3) &&
                     !P.gate_blocked(bcell, d3, P.height(bcell));
            }
        }
        if (first_only) {
            if (__ballot_sync(kFull, v3)) return 1;
            continue;
        }
        bool fresh = v3 && !set_has(w->seen, p3);
        uint32_t mm = __match_any_sync(kFull, fresh ? p3 : -1 - l);
        bool keep = fresh && ((mm & lt) == 0u);
        uint32_t b = __ballot_sync(kFull, keep);
        int pos = cnt + __popc(b & lt);
        if (keep && pos < 32) {
            out[pos] = (uint16_t)p3;
            set_add(w->seen, p3);
        }
        cnt = min(32, cnt + __popc(b));
        __syncwarp();
    }
    return first_only ? 0 : cnt;
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

// Mosquito: beetle when stacked, otherwise the union of the neighbours'
// movements in Q/P, A, G, S, B, L order, first occurrence kept, capped at
// 128 (move_gen.cuh:907-1049).  Needs slx built for this cell.
__device__ __noinline__ int gen_mosquito(WarpSmem* w, int cell, bool first_only, uint32_t* err) {
    Pos P{w};
    if (P.height(cell) > 1) return gen_beetle(w, cell, w->tmp, first_only);
    uint32_t t = neighbour_types(w, cell);
    if (first_only) {
        if ((t & 0x102u) && gen_step1(w, cell, w->dst, true)) return 1;
        if ((t & 0x4u) && gen_ant(w, cell, w->dst, 128, true)) return 1;
        if ((t & 0x8u) && gen_hopper(w, cell, w->dst, true)) return 1;
        if ((t & 0x10u) && gen_walk3<false>(w, cell, w->dst, true)) return 1;
        if ((t & 0x20u) && gen_beetle(w, cell, w->dst, true)) return 1;
        if ((t & 0x80u) && gen_walk3<true>(w, cell, w->dst, true)) return 1;
        return 0;
    }
    int l = lane_id();
    const uint32_t lt = lanemask_lt();
    uint32_t* uni = w->bm + 16 * 17;  // 529-bit union set (free during generation)
    set_clear(uni);
    int cnt = 0;
    for (int part = 0; part < 6; part++) {
        int k = 0;
        switch (part) {
            case 0: if (t & 0x102u) k = gen_step1(w, cell, w->dst, false); break;
            case 1:
                if (t & 0x4u) {
                    k = gen_ant(w, cell, w->dst, 128, false);
                    if (k >= 128 && l == 0) atomicOr(err, kErrBuffer);
                }
                break;
            case 2: if (t & 0x8u) k = gen_hopper(w, cell, w->dst, false); break;
            case 3: if (t & 0x10u) k = gen_walk3<false>(w, cell, w->dst, false); break;
            case 4: if (t & 0x20u) k = gen_beetle(w, cell, w->dst, false); break;
            case 5: if (t & 0x80u) k = gen_walk3<true>(w, cell, w->dst, false); break;
        }
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

// Is the top piece at cell a mosquito-or-pillbug thrower (move_gen.cuh:1316-1345)?
__device__ __forceinline__ bool next_to_pillbug(WarpSmem* w, int cell) {
    Pos P{w};
    for (int d = 0; d < 6; d++) {
        int nb = nbr(cell, d);
        if (nb >= 0 && P.occupied(nb) && (P.top(nb) & 15) == 8) return true;
    }
    return false;
}

// Pillbug throws from thrower pb: valid targets x valid drop cells, in
// (target direction, drop direction) order (move_gen.cuh:691-769).
__device__ __forceinline__ void throw_sets(WarpSmem* w, int pb, uint32_t& tmask, uint32_t& dmask) {
    Pos P{w};
    int l = lane_id();
    int pbh = P.height(pb);
    bool okt = false, okd = false;
    if (l < 6) {
        int t = nbr(pb, l);
        if (t >= 0 && P.occupied(t) && P.height(t) == 1 && !P.is_stunned(t)) {
            int j = P.pidx(t);
            bool pinned = j < 32 && (w->pflag[j] & 1);
            if (!pinned) {
                int ht = P.height(t) - 1;
                okt = !P.gate_blocked(t, opp_dir(l), ht > pbh ? ht : pbh);
            }
        }
        int dcell = nbr(pb, l);
        okd = dcell >= 0 && !P.occupied(dcell) && !P.gate_blocked(pb, l, pbh);
    }
    tmask = __ballot_sync(kFull, okt);
    dmask = __ballot_sync(kFull, okd);
}

// ---------------------------------------------------------------------------
// placement cells (move_gen.cuh:1064-1140) into w->prow / w->ppref
// ---------------------------------------------------------------------------
__device__ __forceinline__ int placement_cells(WarpSmem* w, const Setup& S, int turn) {
    int l = lane_id();
    uint32_t p;
    if (turn == 0) p = (l == 11) ? (1u << 11) : 0u;
    else if (turn == 1) p = dilate(S.occ) & ~S.occ;
    else p = dilate(S.own) & ~S.occ & ~dilate(S.opp);
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

// ---------------------------------------------------------------------------
// full legal move list -> w->mv, returns the count
// ---------------------------------------------------------------------------
__device__ __noinline__ int gen_legal(WarpSmem* w, const Setup& S, uint32_t* err) {
    Pos P{w};
    int l = lane_id();
    if (P.result() != 0) return 0;
    const int color = S.color, turn = P.turn(), ptn = turn >> 1;
    const bool queen_down = (P.queen_placed() >> color) & 1;
    const bool forced = ptn == 3 && !queen_down;
    uint32_t placeable = 0;
    for (int t = 0; t < 8; t++) {
        bool ok = forced ? (t == 0 && P.hand(color, 0) > 0) : (P.hand(color, t) > 0);
        if (ok) placeable |= 1u << t;
    }
    int count = 0;
    if (placeable) {
        int np = placement_cells(w, S, turn);
        uint32_t types = placeable & ~(ptn == 0 ? 1u : 0u);
        int nt = __popc(types);
        int total = np * nt;
        if (total > kMaxMoves) total = kMaxMoves;
        for (int m = l; m < total; m += 32) {
            int k = m / nt, j = m - (m / nt) * nt;
            int cell = kth_cell(w->prow, w->ppref, k);
            put_move(w, m, 0, __fns(types, 0, j + 1) + 1, 0, cell);
        }
        count = total;
    }
    if (queen_down) {
        const int stun = P.stunned();
        // own top pieces according to the side's top bitboard
        bool mine = S.my_cell >= 0 && rowbit(w->own, S.my_cell);
        // movers: own, not stunned, not pinned (move_gen.cuh:1221-1234)
        bool mov = mine && !(stun != 0xFFFF && stun == S.my_cell) && !(w->pflag[l] & 1);
        uint32_t movers = __ballot_sync(kFull, mov);
        while (movers) {
            int i = __ffs(movers) - 1;
            movers &= movers - 1;
            int cell = w->pcell[i];
            int pt = P.top(cell) & 15;
            int k = 0;
            const uint16_t* list = w->dst;
            switch (pt) {
                case 1:
                case 8: k = gen_step1(w, cell, w->dst, false); break;
                case 2: {
                    lift_mover(w, S.occ, cell);
                    int room = kMaxMoves - count;
                    int cap = room < 128 ? room : 128;
                    k = gen_ant(w, cell, w->dst, cap, false);
                    if (k >= 128 && room > 128 && l == 0) atomicOr(err, kErrBuffer);
                    break;
                }
                case 3: k = gen_hopper(w, cell, w->dst, false); break;
                case 4:
                    lift_mover(w, S.occ, cell);
                    k = gen_walk3<false>(w, cell, w->dst, false);
                    break;
                case 5: k = gen_beetle(w, cell, w->dst, false); break;
                case 6:
                    lift_mover(w, S.occ, cell);
                    k = gen_mosquito(w, cell, false, err);
                    list = w->tmp;
                    break;
                case 7: k = gen_walk3<true>(w, cell, w->dst, false); break;
                default: break;
            }
            for (int m = l; m < k; m += 32)
                if (count + m < kMaxMoves) put_move(w, count + m, 1, pt, cell, list[m]);
            count = min(kMaxMoves, count + k);
            __syncwarp();
        }
        // throws by own pillbugs and pillbug-adjacent ground mosquitoes
        int mt = S.my_top & 15;
        bool thr = mine && (mt == 8 || (mt == 6 && S.my_h == 1 && next_to_pillbug(w, S.my_cell)));
        uint32_t throwers = __ballot_sync(kFull, thr);
        while (throwers) {
            int i = __ffs(throwers) - 1;
            throwers &= throwers - 1;
            int pb = w->pcell[i];
            uint32_t tm, dm;
            throw_sets(w, pb, tm, dm);
            int nt = __popc(tm), nd = __popc(dm), total = nt * nd;
            for (int m = l; m < total; m += 32) {
                int kt = m / nd, kd = m - (m / nd) * nd;
                int target = nbr(pb, __fns(tm, 0, kt + 1));
                int dest = nbr(pb, __fns(dm, 0, kd + 1));
                if (count + m < kMaxMoves) put_move(w, count + m, 1, P.top(target) & 15, target, dest);
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

// ---------------------------------------------------------------------------
// compact list for successor features (move_gen.cuh:1362-1563)
// ---------------------------------------------------------------------------
__device__ __noinline__ int gen_compact(WarpSmem* w, const Setup& S, uint32_t* err) {
    Pos P{w};
    int l = lane_id();
    if (P.result() != 0) return 0;
    const int color = S.color, turn = P.turn(), ptn = turn >> 1;
    const bool queen_down = (P.queen_placed() >> color) & 1;
    const bool forced = ptn == 3 && !queen_down;
    bool any = false;
    for (int t = 0; t < 8; t++) {
        bool ok = forced ? (t == 0 && P.hand(color, 0) > 0) : (P.hand(color, t) > 0);
        if (ptn == 0 && t == 0) ok = false;
        any |= ok;
    }
    int count = 0;
    if (any) {
        int np = placement_cells(w, S, turn);
        int total = np < kMaxMoves ? np : kMaxMoves;
        for (int m = l; m < total; m += 32) put_move(w, m, 0, 0, 0, kth_cell(w->prow, w->ppref, m));
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
    bool mov = mine && !(stun != 0xFFFF && stun == S.my_cell) && !(w->pflag[l] & 1);
    uint32_t movers = __ballot_sync(kFull, mov);
    uint32_t seen = 0;  // (type, owner) flags, emit_fnn_move_flag move_gen.cuh:1362-1377
    while (movers && count < kMaxMoves) {
        int i = __ffs(movers) - 1;
        movers &= movers - 1;
        int cell = w->pcell[i];
        int pt = P.top(cell) & 15;
        uint32_t bit = 1u << ((pt - 1) * 2 + color);
        if (seen & bit) continue;
        int has = 0;
        switch (pt) {
            case 1:
            case 8: has = gen_step1(w, cell, w->dst, true); break;
            case 2:
                lift_mover(w, S.occ, cell);
                has = gen_ant(w, cell, w->dst, 128, true);
                break;
            case 3: has = gen_hopper(w, cell, w->dst, true); break;
            case 4:
                lift_mover(w, S.occ, cell);
                has = gen_walk3<false>(w, cell, w->dst, true);
                break;
            case 5: has = gen_beetle(w, cell, w->dst, true); break;
            case 6:
                lift_mover(w, S.occ, cell);
                has = gen_mosquito(w, cell, true, err);
                break;
            case 7: has = gen_walk3<true>(w, cell, w->dst, true); break;
            default: break;
        }
        if (has) {
            seen |= bit;
            if (l == 0) put_move(w, count, 1, pt, cell, 0);
            count++;
        }
        __syncwarp();
    }
    int mt = S.my_top & 15;
    bool thr = mine && (mt == 8 || (mt == 6 && S.my_h == 1 && next_to_pillbug(w, S.my_cell)));
    uint32_t throwers = __ballot_sync(kFull, thr);
    while (throwers && count < kMaxMoves) {
        int i = __ffs(throwers) - 1;
        throwers &= throwers - 1;
        int pb = w->pcell[i];
        uint32_t tm, dm;
        throw_sets(w, pb, tm, dm);
        if (dm == 0u) continue;
        while (tm) {  // summarize_pillbug_throws_for_fnn, move_gen.cuh:1379-1410
            int dt = __ffs(tm) - 1;
            tm &= tm - 1;
            int target = nbr(pb, dt);
            int h = P.height(target);
            int tt = P.top(target);
            int owner = (tt >> 4) & 1;
            uint32_t bit = 1u << (((tt & 15) - 1) * 2 + owner);
            if (h > 0 && !(seen & bit) && count < kMaxMoves) {
                seen |= bit;
                if (l == 0) put_move(w, count, 1, tt & 15, target, 0);
                count++;
            }
        }
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

__device__ __noinline__ void features(WarpSmem* w, const Setup& S, int nmoves, float* out) {
    Pos P{w};
    int l = lane_id();
    for (int i = l; i < A_N; i += 32) w->acc[i] = 0;
    for (int i = l; i < 16 * 17 + 18; i += 32) w->bm[i] = 0u;
    __syncwarp();
    const int turn = P.turn(), cur = turn & 1, stun = P.stunned();
    const int q0 = P.queen_cell(0), q1 = P.queen_cell(1);
    const int cell = S.my_cell, h = S.my_h, top = S.my_top;
    const int pt = top & 15, col = (top >> 4) & 1, tc = (pt - 1) * 2 + col;
    bool capable = false;
    bool adjq0 = false, adjq1 = false;
    if (cell >= 0 && pt >= 1 && pt <= 8) {
        atomicAdd(&w->acc[A_CNT + tc], 1);
        int occn = 0;
        for (int d = 0; d < 6; d++) occn += P.height(nbr(cell, d)) > 0;
        if (occn == 0) atomicAdd(&w->acc[A_SINGLE + col], 1);
        int oq = col ? q0 : q1;
        if (oq != 0xFFFF) {
            if (oq < kCells && hex_distance(cell, oq) == 1) atomicAdd(&w->acc[A_QADJ + tc], 1);
            atomicAdd(&w->acc[A_DSUM + tc], hex_distance(cell, oq));
            atomicAdd(&w->acc[A_DCNT + tc], 1);
        }
        adjq0 = q0 != 0xFFFF && q0 < kCells && hex_distance(cell, q0) == 1;
        adjq1 = q1 != 0xFFFF && q1 < kCells && hex_distance(cell, q1) == 1;
        if (h == 1 && S.my_ap) atomicAdd(&w->acc[A_AP + tc], 1);
        if (pt != 1) {
            for (int lv = 0; lv < h - 1 && lv < 4; lv++) {
                int b = w->st[lv * kCells + cell];
                if ((b & 15) == 1) w->acc[A_COVER + ((b >> 4) & 1)] = 1;
            }
        }
        capable = stun != cell && pt == 8;
        if (!capable && stun != cell && pt == 6 && h == 1) {
            for (int d = 0; d < 6; d++) {
                int nb = nbr(cell, d);
                if (nb < 0 || P.height(nb) == 0 || stun == nb) continue;
                if ((P.top(nb) & 15) == 8) {
                    capable = true;
                    break;
                }
            }
        }
        if (capable) w->acc[A_CAP + col] = 1;
    }
    uint32_t s0 = __ballot_sync(kFull, adjq0), s1 = __ballot_sync(kFull, adjq1);
    // throwable counts from the first eight capable cells of each colour
    uint32_t cap0 = __ballot_sync(kFull, capable && col == 0);
    uint32_t cap1 = __ballot_sync(kFull, capable && col == 1);
    if (capable && __popc((col ? cap1 : cap0) & lanemask_lt()) < 8) {
        for (int d = 0; d < 6; d++) {
            int nb = nbr(cell, d);
            if (nb < 0 || P.height(nb) == 0 || stun == nb) continue;
            int nc = (P.top(nb) >> 4) & 1;
            if (nc == col) atomicAdd(&w->acc[A_TOWN + col], 1);
            else atomicAdd(&w->acc[A_TOPP + nc], 1);
        }
    }
    // source cells per (type, owner) and placement cells from the list
    for (int m = l; m < nmoves; m += 32) {
        int tp = w->mv[3 * m], from = w->mv[3 * m + 1], to = w->mv[3 * m + 2];
        int type = tp & 255, mpt = tp >> 8;
        if (type == 1) {
            if (mpt >= 1 && mpt <= 8 && from < kCells) {
                int owner = P.height(from) > 0 ? ((P.top(from) >> 4) & 1) : cur;
                atomicOr(&w->bm[((mpt - 1) * 2 + owner) * 17 + (from >> 5)], 1u << (from & 31));
            }
        } else if (type == 0 && to < kCells) {
            atomicOr(&w->bm[16 * 17 + (to >> 5)], 1u << (to & 31));
        }
    }
    __syncwarp();
    for (int i = l; i < 16 * 17 + 17; i += 32) {
        int c = __popc(w->bm[i]);
        if (c) atomicAdd(&w->acc[i < 16 * 17 ? A_SRC + i / 17 : A_PLACE], c);
    }
    if (l == 0) {
        w->acc[A_SURR] = __popc(s0);
        w->acc[A_SURR + 1] = __popc(s1);
    }
    __syncwarp();
    for (int k = l; k < kFeat; k += 32) {
        float v = 0.0f;
        if (k < 16) v = (float)w->acc[A_CNT + k];
        else if (k < 32) {
            int t = (k - 16) >> 1, c = (k - 16) & 1;
            const float per = (t == 1 || t == 2) ? 3.0f : ((t == 3 || t == 4) ? 2.0f : 1.0f);
            v = (float)P.hand(c, t) / per;
        } else if (k < 48) v = (float)w->acc[A_QADJ + k - 32];
        else if (k < 64) {
            int n = w->acc[A_DCNT + k - 48];
            if (n > 0) v = (float)w->acc[A_DSUM + k - 48] / (float)n / 10.0f;
        } else if (k < 80) v = (float)w->acc[A_SRC + k - 64];
        else if (k < 96) v = (float)w->acc[A_AP + k - 80];
        else if (k < 98) v = (float)w->acc[A_SINGLE + k - 96];
        else if (k < 100) v = (float)w->acc[A_COVER + k - 98];
        else if (k < 102) v = (k - 100 == cur) ? (float)w->acc[A_PLACE] / 10.0f : 0.0f;
        else if (k == 102) {
            int left = 200 - turn;
            v = (float)(left < 0 ? 0 : left) / 200.0f;
        } else if (k == 103) {
            float t = (float)turn / 100.0f;
            v = t < 1.0f ? t : 1.0f;
        } else if (k < 106) v = (float)w->acc[A_CAP + k - 104];
        else if (k < 108) v = (float)w->acc[A_TOWN + k - 106];
        else if (k < 110) v = (float)w->acc[A_TOPP + k - 108];
        else {
            int qc = (k - 110) / 6, b = (k - 110) - qc * 6;
            int s = w->acc[A_SURR + qc];
            v = (s == b + 1) ? 1.0f : 0.0f;
        }
        out[k] = v;
    }
    __syncwarp();
}

}  // namespace hv
