// hv_state.cuh -- single-thread state mutation on the boundary byte layout
// (apply a move, detect game end, initial state), shared by the playout,
// successor and tree kernels.  Semantics: hive_gpu/csrc/hive_state.cuh:321-517.
#pragma once

#include "hv_core.cuh"

namespace hv {

__device__ __forceinline__ void st_bb_set(uint8_t* st, int off, int c) {
    reinterpret_cast<uint64_t*>(st + off)[c >> 6] |= 1ull << (c & 63);
}
__device__ __forceinline__ void st_bb_clr(uint8_t* st, int off, int c) {
    reinterpret_cast<uint64_t*>(st + off)[c >> 6] &= ~(1ull << (c & 63));
}
__device__ __forceinline__ bool st_bb_get(const uint8_t* st, int off, int c) {
    return (reinterpret_cast<const uint64_t*>(st + off)[c >> 6] >> (c & 63)) & 1ull;
}
__device__ __forceinline__ int st_u16(const uint8_t* st, int off) { return st[off] | (st[off + 1] << 8); }
__device__ __forceinline__ void st_put_u16(uint8_t* st, int off, int v) {
    st[off] = (uint8_t)(v & 255);
    st[off + 1] = (uint8_t)(v >> 8);
}

__device__ __forceinline__ void st_top_color(uint8_t* st, int c, int color) {
    if (color == 0) {
        st_bb_set(st, kOffWTop, c);
        st_bb_clr(st, kOffBTop, c);
    } else {
        st_bb_set(st, kOffBTop, c);
        st_bb_clr(st, kOffWTop, c);
    }
}

__device__ __forceinline__ bool st_queen_surrounded(const uint8_t* st, int color) {
    if (!((st[kOffQPlaced] >> color) & 1)) return false;
    int q = st_u16(st, kOffQCell + 2 * color);
    if (q >= kCells) return false;
    int p = c_to_p(q), n = 0;
    for (int d = 0; d < 6; d++) {
        int nb = nbr(p, d);
        if (nb >= 0 && st_bb_get(st, kOffOcc, p_to_c(nb))) n++;
    }
    return n == 6;
}

// apply_move (hive_state.cuh:497-517) including its silent refusals: a full
// destination stack leaves the board unchanged but still advances the turn.
// This part moves the piece and advances turn and stun; the result follows.
__device__ inline void st_apply_board(uint8_t* st, int type, int pt, int from, int to) {
    int turn = st_u16(st, kOffTurn);
    int color = turn & 1;
    int stun = st_u16(st, kOffStun);
    if (type == 0) {
        if (to < kCells && pt >= 1 && pt <= 8) {
            int h = st[kOffHeight + to];
            if (h < 5) {
                st[h * kCells + to] = (uint8_t)(pt | (color << 4));
                st[kOffHeight + to] = (uint8_t)(h + 1);
                if (h == 0) st_bb_set(st, kOffOcc, to);
                st_top_color(st, to, color);
                if (pt == 1) {
                    st_put_u16(st, kOffQCell + 2 * color, to);
                    st[kOffQPlaced] |= (uint8_t)(1 << color);
                }
                st[kOffHands + color * 8 + pt - 1]--;
            }
        }
        stun = 0xFFFF;
    } else if (type == 1) {
        if (from < kCells && to < kCells) {
            int hf = st[kOffHeight + from], ht = st[kOffHeight + to];
            if (hf > 0 && hf <= 5 && ht < 5) {
                uint8_t b = st[(hf - 1) * kCells + from];
                st[(hf - 1) * kCells + from] = 0;
                st[kOffHeight + from] = (uint8_t)(hf - 1);
                if (hf == 1) {
                    st_bb_clr(st, kOffOcc, from);
                    st_bb_clr(st, kOffWTop, from);
                    st_bb_clr(st, kOffBTop, from);
                } else {
                    st_top_color(st, from, (st[(hf - 2) * kCells + from] >> 4) & 1);
                }
                ht = st[kOffHeight + to];  // from == to re-reads the lowered stack
                st[ht * kCells + to] = b;
                st[kOffHeight + to] = (uint8_t)(ht + 1);
                if (ht == 0) st_bb_set(st, kOffOcc, to);
                int bc = (b >> 4) & 1;
                st_top_color(st, to, bc);
                if ((b & 15) == 1) st_put_u16(st, kOffQCell + 2 * bc, to);
            }
            stun = to;
        }
    } else {
        stun = 0xFFFF;
    }
    st_put_u16(st, kOffStun, stun);
    st_put_u16(st, kOffTurn, turn + 1);
}

__device__ __forceinline__ void st_set_result(uint8_t* st, bool w, bool b) {
    if (w && b) st[kOffResult] = 3;
    else if (w) st[kOffResult] = 2;
    else if (b) st[kOffResult] = 1;
}

// one thread
__device__ inline void st_apply(uint8_t* st, int type, int pt, int from, int to) {
    st_apply_board(st, type, pt, from, to);
    st_set_result(st, st_queen_surrounded(st, 0), st_queen_surrounded(st, 1));
}

// one warp (all lanes, same arguments): lane 0 moves the piece, then lanes
// 0..11 test the six neighbours of both queens at once
__device__ inline void st_apply_warp(uint8_t* st, int type, int pt, int from, int to) {
    const int l = threadIdx.x & 31;
    if (l == 0) st_apply_board(st, type, pt, from, to);
    __syncwarp();
    bool occ = false;
    if (l < 12) {
        const int color = l >= 6, d = l - 6 * color;
        const int q = st_u16(st, kOffQCell + 2 * color);
        if (((st[kOffQPlaced] >> color) & 1) && q < kCells) {
            const int nb = nbr(c_to_p(q), d);
            occ = nb >= 0 && st_bb_get(st, kOffOcc, p_to_c(nb));
        }
    }
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, occ);
    if (l == 0) st_set_result(st, (m & 63u) == 63u, ((m >> 6) & 63u) == 63u);
    __syncwarp();
}

// initial state (hive_state.cuh:454-492) into a zeroed buffer; one thread
__device__ __forceinline__ void st_init_fields(uint8_t* st, int mask) {
    st_put_u16(st, kOffQCell, 0xFFFF);
    st_put_u16(st, kOffQCell + 2, 0xFFFF);
    const uint8_t per[5] = {1, 3, 3, 2, 2};
    for (int c = 0; c < 2; c++) {
        for (int t = 0; t < 5; t++) st[kOffHands + c * 8 + t] = per[t];
        st[kOffHands + c * 8 + 5] = (mask & 1) ? 1 : 0;
        st[kOffHands + c * 8 + 6] = (mask & 2) ? 1 : 0;
        st[kOffHands + c * 8 + 7] = (mask & 4) ? 1 : 0;
    }
    st_put_u16(st, kOffStun, 0xFFFF);
}

// counter-based splitmix64 stream (seed, game, ply) -> 64 random bits; the
// seeded playout generator of the benchmark inputs (identical to the CPU
// oracle's generator so both sides see the same positions)
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
__device__ __forceinline__ uint64_t game_rng(uint64_t seed, uint64_t game, uint64_t ply) {
    return mix64(mix64(seed ^ mix64(game)) + ply);
}

}  // namespace hv
