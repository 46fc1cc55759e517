// hv_core.cuh -- warp-per-position Hive game logic for sm_100a.
//
// One warp owns one position.  The 3424-byte HiveState (the boundary format
// of the reference, hive_gpu/csrc/hive_state.cuh:239-269) is staged in the
// warp's shared-memory slot; everything else is derived from it.
//
// Internal cell index.  Inside the kernels a cell is p = row * 32 + col
// (rows and columns 0..22 of the reference's 23x23 grid): one grid row is one
// 32-bit word, so a neighbour is p + step, a bit test is a shift, and a
// 529-cell set is 23 words.  The reference's index c = row * 23 + col is used
// only where bytes cross the boundary (state arrays, move lists):
// c = p - 9 * (p >> 5).
//
//   * row bitboards: lane r (r < 23) holds the occupancy word of grid row r,
//     so a hex-direction shift of the whole board is one shuffle plus one
//     shift;
//   * piece lanes: lane i (i < N <= 28) owns the i-th occupied cell in
//     ascending cell order (the reference's iteration order);
//   * slide masks sl[d]: the cells that can slide one step in direction d
//     (destination empty, exactly one flank occupied), built for the whole
//     board with row-bitboard algebra, so each freedom-to-move test of the
//     reference (move_gen.cuh:82-131) becomes one shared-memory bit test.
#pragma once

#include <cstddef>
#include <cstdint>

namespace hv {

constexpr int kBoard = 23;
constexpr int kCells = 529;
constexpr int kPCells = kBoard * 32;  // padded index space
constexpr int kMaxMoves = 256;
constexpr int kFeat = 122;
constexpr int kStateBytes = 3424;
constexpr int kMoveBytes = 6;
constexpr int kOffHeight = 2645;
constexpr int kOffOcc = 3176;
constexpr int kOffWTop = 3248;
constexpr int kOffBTop = 3320;
constexpr int kOffQCell = 3392;
constexpr int kOffHands = 3396;
constexpr int kOffTurn = 3412;
constexpr int kOffQPlaced = 3414;
constexpr int kOffResult = 3415;
constexpr int kOffStun = 3416;
constexpr uint32_t kFull = 0xffffffffu;
constexpr uint32_t kRowBits = 0x7fffffu;

// The move generators are called from several places (full list, compact
// list, mosquito union); keeping one out-of-line copy of each keeps the
// kernel's instruction footprint small.
#ifndef HV_GEN_INLINE
#define HV_GEN_INLINE __noinline__
#endif

// Error bits reported through the device error word.
constexpr uint32_t kErrBuffer = 1u;  // a generator list exceeded its buffer
constexpr uint32_t kErrIndex = 2u;   // a root / move index was out of range

// The fields up to and including the union are all that the feature launch
// of the fused movegen + features entry touches (articulation masks given,
// no slide masks): that launch gives each warp only that prefix
// (kFeatSlotBytes) and fits one more block per SM.
struct __align__(16) WarpSmem {
    uint8_t st[kStateBytes];     // staged HiveState
    uint16_t mv[kMaxMoves * 3];  // move list: (type | pt << 8, from, to) per move
    uint32_t occ[24];            // occupied row words
    uint32_t own[24];            // side-to-move top-piece row words
    uint16_t pcell[32];          // cell of piece i
    uint16_t pref[24];           // piece index of the first occupied cell of row r
    uint8_t pflag[32];           // bit0: pinned (articulation point at height 1), bit1: articulation point
    uint32_t pl[24];             // mosquito union set (generators) / placement-cell set (features)
    // Generator scratch and feature accumulators are never live together
    // (features run on a finished move list), so they share storage: 1.3 KB
    // less per warp, one more resident block per SM.
    union {
        struct {
            uint32_t slx[6][24];  // slide masks with the current mover lifted
            uint16_t dst[128];    // destination list of the running generator
            uint16_t tmp[128];    // sub-generator list (mosquito)
            uint16_t qcell[48];   // walk queue (spider / ladybug paths): cell
            uint16_t qanc[48];    //                                      previous cell
        };
        struct {
            int acc[112];          // feature accumulators
            uint32_t bm[16 * 17];  // per (type, owner) source-cell sets
        };
    };
    // generator-only fields (past the feature launch's prefix)
    uint32_t sl[6][24];          // slide masks of the position
    uint32_t seen[24];           // scratch cell set
    uint32_t prow[24];           // placement row words
    uint32_t adj[32];            // piece adjacency (piece-index space)
    uint16_t ppref[24];          // placement index of the first placement cell of row r
};
static_assert(offsetof(WarpSmem, acc) % 16 == 0, "feature accumulators are cleared with 16-byte stores");
constexpr int kFeatSlotBytes = (int)offsetof(WarpSmem, sl);
static_assert(kFeatSlotBytes % 16 == 0, "feature-launch warp slots stay 16-byte aligned");

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ int p_to_c(int p) { return p - 9 * (p >> 5); }
__device__ __forceinline__ int c_to_p(int c) { return c + 9 * (c / kBoard); }

// direction order E, NE, NW, W, SW, SE (hex_grid.cuh:41-49) as p-steps
// +1, -31, -32, -1, +31, +32, packed (step + 32) in 7 bits each
constexpr unsigned long long kDirPack =
    33ull | (1ull << 7) | (0ull << 14) | (31ull << 21) | (63ull << 28) | (64ull << 35);
__device__ __forceinline__ int dstep(int d) { return (int)((kDirPack >> (7 * d)) & 127ull) - 32; }
__device__ __forceinline__ int cw_dir(int d) { return d == 0 ? 5 : d - 1; }
__device__ __forceinline__ int ccw_dir(int d) { return d == 5 ? 0 : d + 1; }
__device__ __forceinline__ int opp_dir(int d) { return d < 3 ? d + 3 : d - 3; }

// neighbour of p in direction d, -1 off the grid
__device__ __forceinline__ int nbr(int p, int d) {
    int q = p + dstep(d);
    return ((unsigned)q < (unsigned)kPCells && (q & 31) < kBoard) ? q : -1;
}

__device__ __forceinline__ int rowbit(const uint32_t* rows, int p) {
    return (int)((rows[p >> 5] >> (p & 31)) & 1u);
}

// hex distance (fnn_features.cuh:45-60) on (row, col) of p-space indices
__device__ __forceinline__ int hex_distance(int a, int b) {
    int dq = (b & 31) - (a & 31), dr = (b >> 5) - (a >> 5), ds = -(dq + dr);
    dq = dq < 0 ? -dq : dq;
    dr = dr < 0 ? -dr : dr;
    ds = ds < 0 ? -ds : ds;
    int m = dq > dr ? dq : dr;
    return m > ds ? m : ds;
}

// ---------------------------------------------------------------------------
// state field access (boundary byte layout)
// ---------------------------------------------------------------------------

struct Pos {
    WarpSmem* w;
    __device__ __forceinline__ int height(int p) const { return p >= 0 ? w->st[kOffHeight + p_to_c(p)] : 0; }
    // top piece byte; a corrupt height above the stack limit reads level 5
    __device__ __forceinline__ int top(int p) const {
        int h = height(p);
        h = h > 5 ? 5 : h;
        return h ? w->st[(h - 1) * kCells + p_to_c(p)] : 0;
    }
    __device__ __forceinline__ bool occupied(int p) const { return p >= 0 && rowbit(w->occ, p); }
    __device__ __forceinline__ int turn() const {
        return w->st[kOffTurn] | (w->st[kOffTurn + 1] << 8);
    }
    // reference-index field -> p-space (-1 for the 0xFFFF "none" marker)
    __device__ __forceinline__ int cell_field(int off) const {
        int c = w->st[off] | (w->st[off + 1] << 8);
        return c == 0xFFFF ? -1 : c_to_p(c);
    }
    __device__ __forceinline__ int stunned() const { return cell_field(kOffStun); }
    __device__ __forceinline__ int queen_cell(int color) const { return cell_field(kOffQCell + 2 * color); }
    __device__ __forceinline__ int hand(int color, int t) const {
        return w->st[kOffHands + color * 8 + t];
    }
    __device__ __forceinline__ int result() const { return w->st[kOffResult]; }
    __device__ __forceinline__ int queen_placed() const { return w->st[kOffQPlaced]; }
    // piece index of an occupied cell
    __device__ __forceinline__ int pidx(int p) const {
        int r = p >> 5;
        return w->pref[r] + __popc(w->occ[r] & ((1u << (p & 31)) - 1u));
    }
    // elevated gate (move_gen.cuh:659-667): both flanks strictly higher than h
    __device__ __forceinline__ bool gate_blocked(int p, int d, int h) const {
        return height(nbr(p, cw_dir(d))) > h && height(nbr(p, ccw_dir(d))) > h;
    }
};

// ---------------------------------------------------------------------------
// row bitboards (lane r = grid row r; lanes >= 23 hold zero)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t row_valid_mask() { return lane_id() < kBoard ? kRowBits : 0u; }

// X[r-1] and X[r+1] for the calling lane
__device__ __forceinline__ uint32_t from_row_above(uint32_t x) {
    uint32_t v = __shfl_up_sync(kFull, x, 1);
    return lane_id() == 0 ? 0u : v;
}
__device__ __forceinline__ uint32_t from_row_below(uint32_t x) { return __shfl_down_sync(kFull, x, 1); }

// N_d(X): cells whose neighbour in direction d lies in X, all six directions.
__device__ __forceinline__ void neighbour_sets(uint32_t x, uint32_t* out) {
    uint32_t up = from_row_above(x), dn = from_row_below(x), m = row_valid_mask();
    out[0] = (x >> 1) & m;   // E : (r, q+1)
    out[1] = (up >> 1) & m;  // NE: (r-1, q+1)
    out[2] = up & m;         // NW: (r-1, q)
    out[3] = (x << 1) & m;   // W : (r, q-1)
    out[4] = (dn << 1) & m;  // SW: (r+1, q-1)
    out[5] = dn & m;         // SE: (r+1, q)
}

__device__ __forceinline__ uint32_t dilate(uint32_t x) {
    uint32_t n[6];
    neighbour_sets(x, n);
    return n[0] | n[1] | n[2] | n[3] | n[4] | n[5];
}

// Slide masks for occupancy x (freedom to move, move_gen.cuh:82-118):
// sl[d] = {p : nb(p,d) on grid and empty, occ(nb(p,cw d)) xor occ(nb(p,ccw d))}
__device__ __forceinline__ void build_slide_masks(uint32_t x, uint32_t (*sl)[24]) {
    uint32_t nx[6], ne[6];
    uint32_t m = row_valid_mask();
    neighbour_sets(x, nx);
    neighbour_sets(~x & m, ne);
    int l = lane_id();
    if (l < 24) {
#pragma unroll
        for (int d = 0; d < 6; d++) sl[d][l] = ne[d] & (nx[(d + 5) % 6] ^ nx[(d + 1) % 6]);
    }
}

// exclusive prefix sum over lanes
__device__ __forceinline__ int warp_excl_scan(int v) {
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(kFull, x, o);
        if (lane_id() >= o) x += y;
    }
    return x - v;
}

// ---------------------------------------------------------------------------
// per-position setup
// ---------------------------------------------------------------------------

struct Setup {
    int n;          // occupied cells (<= 28 used, as the reference's MAX_PIECES)
    int color;      // side to move
    int my_cell;    // piece lane: cell p (or -1)
    int my_h;       // piece lane: stack height
    int my_top;     // piece lane: top byte
    bool my_ap;     // piece lane: articulation point
    uint32_t own;   // row lane: own top pieces
    uint32_t opp;   // row lane: opponent top pieces
    uint32_t occ;   // row lane: occupancy
};

// row r of a reference bitboard (bits c = 23r .. 23r+22) as a 23-bit word
__device__ __forceinline__ uint32_t load_row(const uint8_t* st, int off, int lane) {
    if (lane >= kBoard) return 0u;
    const uint32_t* w32 = reinterpret_cast<const uint32_t*>(st + off);
    int b = lane * kBoard;
    uint32_t lo = w32[b >> 5], hi = w32[(b >> 5) + 1];
    return __funnelshift_r(lo, hi, b & 31) & kRowBits;
}

// Articulation flag of the piece lane: every lane removes its vertex and
// floods the rest (the lane loops run for the longest flood).
__device__ __forceinline__ bool articulation_flood(WarpSmem* w, const Setup& S) {
    const int l = lane_id();
    // adjacency in piece-index space, from the occupancy words and piece
    // prefixes of the three rows around the cell (neighbours E (r, q+1),
    // NE (r-1, q+1), NW (r-1, q), W (r, q-1), SW (r+1, q-1), SE (r+1, q);
    // padding bits are zero, row 23 is empty)
    uint32_t adj = 0;
    if (S.my_cell >= 0) {
        const int r = S.my_cell >> 5, q = S.my_cell & 31;
        const uint32_t ou = r ? w->occ[r - 1] : 0u, om = w->occ[r], od = w->occ[r + 1];
        const int pu = r ? w->pref[r - 1] : 0, pm = w->pref[r], pd = w->pref[r + 1];
        auto take = [&](uint32_t row, int pre, int col) {
            if (col >= 0 && ((row >> col) & 1u)) {
                const int j = pre + __popc(row & ((1u << col) - 1u));
                if (j < S.n) adj |= 1u << j;
            }
        };
        take(ou, pu, q);
        take(ou, pu, q + 1);
        take(om, pm, q - 1);
        take(om, pm, q + 1);
        take(od, pd, q - 1);
        take(od, pd, q);
    }
    w->adj[l] = adj;
    __syncwarp();
    // One-Hive rule (articulation.cuh:34-168): the reference runs Tarjan from
    // the lowest occupied cell, i.e. it reports the articulation points of
    // that cell's component.  Lane x < n removes vertex x and floods from a
    // vertex of that component; lane 31 floods the component itself.
    uint32_t all = S.n >= 32 ? kFull : ((1u << S.n) - 1u);
    uint32_t adj0 = w->adj[0];
    uint32_t allowed = all;
    int start = 0;
    bool active = S.n > 2 && (l < S.n || l == 31);
    if (l < S.n) {
        allowed = all & ~(1u << l);
        if (l == 0) start = adj0 ? __ffs(adj0) - 1 : -1;
    }
    uint32_t seen = 0;
    if (active && start >= 0) {
        seen = 1u << start;
        uint32_t fr = seen;
#pragma unroll 1
        while (fr) {
            int v = __ffs(fr) - 1;
            fr &= fr - 1;
            uint32_t nw = w->adj[v] & allowed & ~seen;
            seen |= nw;
            fr |= nw;
        }
    }
    uint32_t comp = __shfl_sync(kFull, seen, 31);
    bool ap = false;
    if (S.n > 2 && l < S.n && ((comp >> l) & 1u)) {
        uint32_t rest = comp & ~(1u << l);
        ap = (l == 0) ? (adj0 != 0 && seen != rest) : (seen != rest);
    }
    return ap;
}

// Articulation flag of the piece lane, flooding only from vertices whose
// neighbours form two or more arcs of their ring.
__device__ __forceinline__ bool articulation_arc(WarpSmem* w, const Setup& S) {
    Pos P{w};
    const int l = lane_id();
    // adjacency in piece-index space, and the occupied neighbours of the
    // piece's cell as a 6-bit ring in direction order
    uint32_t adj = 0, ring = 0;
    if (S.my_cell >= 0) {
#pragma unroll 1
        for (int d = 0; d < 6; d++) {
            int nb = nbr(S.my_cell, d);
            if (nb >= 0 && rowbit(w->occ, nb)) {
                int j = P.pidx(nb);
                if (j < S.n) {
                    adj |= 1u << j;
                    ring |= 1u << d;
                }
            }
        }
    }
    w->adj[l] = adj;
    __syncwarp();
    // The component of the lowest occupied cell (the reference's Tarjan
    // root) grows level by level, one warp OR-reduction per level.  A vertex
    // x of it is an articulation point iff its neighbours are not all
    // connected once x is removed (every other vertex of the component
    // reaches x through one of them).  Neighbours forming one contiguous arc
    // of x's six-cell ring are connected (consecutive ring cells touch), so
    // only a vertex with two or more arcs floods, and it stops as soon as it
    // has reached all its neighbours.
    const uint32_t all = S.n >= 32 ? kFull : ((1u << S.n) - 1u);
    uint32_t comp = S.n > 0 ? 1u : 0u;
#pragma unroll 1
    while (true) {
        const uint32_t grow = (comp | __reduce_or_sync(kFull, ((comp >> l) & 1u) ? adj : 0u)) & all;
        if (grow == comp) break;
        comp = grow;
    }
    bool ap = false;
    if (S.n > 2 && l < S.n && ((comp >> l) & 1u) && adj != 0u) {
        const uint32_t starts = ring & ~(((ring << 1) | (ring >> 5)) & 63u);  // first cell of each arc
        if (__popc(starts) >= 2) {
            const uint32_t allowed = all & ~(1u << l);
            uint32_t seen = 1u << (__ffs(adj) - 1), fr = seen;
#pragma unroll 1
            while (fr && (seen & adj) != adj) {
                const int v = __ffs(fr) - 1;
                fr &= fr - 1;
                const uint32_t nw = w->adj[v] & allowed & ~seen;
                seen |= nw;
                fr |= nw;
            }
            ap = (seen & adj) != adj;
        }
    }
    return ap;
}

// Bitboards, piece list, slide masks, articulation points.  SLIDES = false
// skips the slide masks (a caller that generates no moves); ARC selects the
// articulation test that floods only from vertices whose neighbours form
// two or more arcs of their ring (shorter, faster where the kernel is not
// bound by branch issue; the result is the same).
// GIVEN_AP: the articulation flags come in as ap_mask (bit i: piece i, in
// the piece-list order built here), from a generator launch on the same
// position.
template <bool SLIDES = true, bool ARC = false, bool GIVEN_AP = false>
__device__ __forceinline__ Setup setup_position(WarpSmem* w, uint32_t ap_mask = 0u) {
    Setup S;
    Pos P{w};
    int l = lane_id();
    S.occ = load_row(w->st, kOffOcc, l);
    uint32_t wt = load_row(w->st, kOffWTop, l), bt = load_row(w->st, kOffBTop, l);
    S.color = P.turn() & 1;
    S.own = S.color ? bt : wt;
    S.opp = S.color ? wt : bt;
    if (l < 24) {
        w->occ[l] = S.occ;
        w->own[l] = S.own;
    }
    int cnt = __popc(S.occ);
    int pre = warp_excl_scan(cnt);
    if (l < 24) w->pref[l] = (uint16_t)pre;
    S.n = __shfl_sync(kFull, pre + cnt, 31);
    if (S.n > 28) S.n = 28;
    // cells of this row into the piece list (ascending order)
    {
        uint32_t bits = S.occ;
        int k = pre;
#pragma unroll 1
        while (bits) {
            int q = __ffs(bits) - 1;
            bits &= bits - 1;
            if (k < 32) w->pcell[k] = (uint16_t)((l << 5) + q);
            k++;
        }
    }
    if (SLIDES) build_slide_masks(S.occ, w->sl);
    __syncwarp();
    S.my_cell = l < S.n ? (int)w->pcell[l] : -1;
    S.my_h = P.height(S.my_cell);
    S.my_top = P.top(S.my_cell);

    if (GIVEN_AP)
        S.my_ap = l < S.n && ((ap_mask >> l) & 1u);
    else
        S.my_ap = ARC ? articulation_arc(w, S) : articulation_flood(w, S);
    w->pflag[l] = ((S.my_ap && S.my_h == 1) ? 1 : 0) | (S.my_ap ? 2 : 0);
    __syncwarp();
    return S;
}

// The Setup of the staged position, re-read from the warp's shared slot
// after setup_position.  Functions that are not inlined start from this
// instead of a Setup passed by reference: such a Setup lives in local
// memory, and local memory misses the small L1 left beside the shared
// memory these kernels take (a round trip to L2 per field).
__device__ __forceinline__ Setup reload_setup(WarpSmem* w) {
    Setup S;
    Pos P{w};
    const int l = lane_id();
    S.occ = l < 24 ? w->occ[l] : 0u;
    S.own = l < 24 ? w->own[l] : 0u;
    S.color = P.turn() & 1;
    S.opp = load_row(w->st, S.color ? kOffWTop : kOffBTop, l);
    S.n = min(28, (int)w->pref[23]);
    S.my_cell = l < S.n ? (int)w->pcell[l] : -1;
    S.my_h = P.height(S.my_cell);
    S.my_top = P.top(S.my_cell);
    S.my_ap = (w->pflag[l] >> 1) & 1;
    return S;
}

}  // namespace hv
