// hv_tactics.cuh -- root tactical probe (game_logic.cu:290-397
// root_tactical_probe_kernel with the move_gen.cuh:825-899 helpers).
//
// The reference runs the whole probe of a root in one thread: win-in-one
// over every child, the opponent's immediate-win screen over every child
// (a move generation per child) and the win-in-two search (a move
// generation per child and per reply).  Here the children of all roots are
// independent work items, one warp each, so a root with 200 candidate
// children spreads over 200 warps; per-root decisions that depend on all
// children (best prior, "any safe move", first winning candidate) are taken
// by small per-root passes between them.  The outputs double as the state
// between passes: allowed[] bit 0 = allowed, bit 1 = child wins at once,
// bit 2 = forced win in two; forced[] holds the per-root flags below until
// the last pass writes 0/1.
#pragma once

#include "hv_core.cuh"
#include "hv_movegen.cuh"
#include "hv_state.cuh"

namespace hv {

constexpr int kTacS1 = 1;       // win-in-one probe active (opponent queen surround 5)
constexpr int kTacS2 = 2;       // opponent-win screen active (own queen surround 5)
constexpr int kTacS3 = 4;       // win-in-two probe active (opponent queen surround 4 or 5)
constexpr int kTacDone = 8;     // decided before the win-in-two probe
constexpr int kTacForced = 16;  // no safe move: forced random
constexpr int kTacOppShift = 5; // opponent surround count (0..6) in bits 5..7

// per-warp scratch of the win-in-two pass: the child and its reply list
struct __align__(16) TacSmem {
    uint8_t child[kStateBytes];
    uint16_t rep[3 * kMaxMoves];
};

__device__ __forceinline__ int nbr_c(int c, int d) {
    int p = nbr(c_to_p(c), d);
    return p < 0 ? -1 : p_to_c(p);
}

__device__ __forceinline__ bool wins_for(int result, int color) { return result == (color == 0 ? 1 : 2); }

// queen_surround_count_for_color_device (move_gen.cuh:825-831): occupied
// on-grid neighbours of `color`'s queen, 0 when it is not placed.  Lanes 0-5
// test one direction each; the result is warp-uniform.  `st` may be global or
// shared memory.
__device__ __forceinline__ int surround_count(const uint8_t* st, int color) {
    if (!((st[kOffQPlaced] >> color) & 1)) return 0;
    const int q = st_u16(st, kOffQCell + 2 * color);
    if (q >= kCells) return 0;
    const int l = lane_id();
    const int nb = l < 6 ? nbr_c(q, l) : -1;
    return __popc(__ballot_sync(kFull, nb >= 0 && st_bb_get(st, kOffOcc, nb)));
}

// lone_empty_neighbor_of_queen (move_gen.cuh:833-852): the single empty
// on-grid neighbour of `target`'s queen when five are occupied, else -1.
__device__ __forceinline__ int lone_empty(const uint8_t* st, int target) {
    if (!((st[kOffQPlaced] >> target) & 1)) return -1;
    const int q = st_u16(st, kOffQCell + 2 * target);
    if (q >= kCells) return -1;
    const int l = lane_id();
    const int nb = l < 6 ? nbr_c(q, l) : -1;
    const bool on = nb >= 0;
    const bool occ = on && st_bb_get(st, kOffOcc, nb);
    const uint32_t o = __ballot_sync(kFull, occ);
    const uint32_t e = __ballot_sync(kFull, on && !occ);
    if (__popc(o) != 5 || __popc(e) != 1) return -1;
    return __shfl_sync(kFull, nb, __ffs(e) - 1);
}

__device__ __forceinline__ void apply_bytes(uint8_t* st, const uint8_t* m) {
    st_apply(st, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8));
}
__device__ __forceinline__ void apply_list(uint8_t* st, const uint16_t* mv, int k) {
    st_apply(st, mv[3 * k] & 0xFF, mv[3 * k] >> 8, mv[3 * k + 1], mv[3 * k + 2]);
}

__device__ __forceinline__ void copy_state(uint8_t* dst, const uint8_t* src) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int i = lane_id(); i < kStateBytes / 16; i += 32) d4[i] = s4[i];
    __syncwarp();
}

// has_immediate_surround_win_for_current_player (move_gen.cuh:854-874) of the
// state staged in w->st: a legal move onto the lone empty neighbour of the
// opponent queen that wins.  `rebuild()` re-stages that state; each candidate
// is applied to a fresh copy while the move list stays in w->mv.
template <typename Rebuild>
__device__ bool immediate_win_staged(WarpSmem* w, Rebuild rebuild, uint32_t* err) {
    const int player = st_u16(w->st, kOffTurn) & 1;
    const int cell = lone_empty(w->st, player ^ 1);
    if (cell < 0) return false;
    Setup S = setup_position(w);
    const int n = gen_legal(w, err);
    for (int base = 0; base < n; base += 32) {
        const int m = base + lane_id();
        uint32_t hits = __ballot_sync(kFull, m < n && w->mv[3 * m + 2] == cell);
        while (hits) {
            const int k = base + __ffs(hits) - 1;
            hits &= hits - 1;
            rebuild();
            if (lane_id() == 0) apply_list(w->st, w->mv, k);
            __syncwarp();
            if (wins_for(w->st[kOffResult], player)) return true;
        }
    }
    return false;
}

}  // namespace hv
