// hv_hybrid.cuh -- inputs of the hybrid FNN-transformer evaluator:
// piece tokens (state_encoder.cuh:372-468
// extract_hybrid_transformer_tokens_device) and per-move features
// (state_encoder.cuh:470-550 extract_hybrid_transformer_move_features_device),
// one warp per state.  Lane l owns the l-th occupied cell (ascending), which
// is the reference's token order; its stack levels follow each other.
#pragma once

#include "hv_core.cuh"
#include "hv_state.cuh"

namespace hv {

constexpr int kTokens = 28;
constexpr int kTokFeat = 27;
constexpr int kMoveFeat = 31;
constexpr int kGlobFeat = 6;

// occupied (height > 0) on-grid neighbours of reference cell c; flags per direction
__device__ __forceinline__ int height_neighbours(const Pos& P, int p, int* flags) {
    int n = 0;
#pragma unroll
    for (int d = 0; d < 6; d++) {
        int f = P.height(nbr(p, d)) > 0;
        if (flags) flags[d] = f;
        n += f;
    }
    return n;
}

// global features (state_encoder.cuh:452-467), written by the calling lane
__device__ __forceinline__ void hybrid_global(const uint8_t* st, float* gf) {
    const int turn = st_u16(st, kOffTurn);
    int wh = 0, bh = 0;
#pragma unroll
    for (int p = 0; p < 8; p++) {
        wh += st[kOffHands + p];
        bh += st[kOffHands + 8 + p];
    }
    const float t = __fdiv_rn((float)turn, 100.0f);
    gf[0] = (turn & 1) == 0 ? 1.0f : 0.0f;
    gf[1] = t < 1.0f ? t : 1.0f;
    gf[2] = (st[kOffQPlaced] & 1) ? 1.0f : 0.0f;
    gf[3] = (st[kOffQPlaced] & 2) ? 1.0f : 0.0f;
    gf[4] = __fdiv_rn((float)wh, 14.0f);
    gf[5] = __fdiv_rn((float)bh, 14.0f);
}

// Token rows of the staged position (after setup_position).  Writes every
// row of tf [28][27], tq/tr/tz/tm [28] (zero past the token count) and gf;
// returns the token count (warp-uniform).
__device__ __noinline__ int hybrid_tokens(WarpSmem* w, float* tf, int32_t* tq, int32_t* tr, int32_t* tz, uint8_t* tm,
                                          float* gf) {
    const Setup S = reload_setup(w);
    Pos P{w};
    const int l = lane_id();
    // queen surround by colour as the token encoder reads it: queen_cell
    // field set, occupied = height > 0 (state_encoder.cuh:390-400)
    float qs[2];
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const int qc = st_u16(w->st, kOffQCell + 2 * c);
        const int q = (qc != 0xFFFF && qc < kCells) ? c_to_p(qc) : -1;
        const int nb = (q >= 0 && l < 6) ? nbr(q, l) : -1;
        const int cnt = __popc(__ballot_sync(kFull, P.height(nb) > 0));
        qs[c] = q >= 0 ? __fdiv_rn((float)cnt, 6.0f) : 0.0f;
    }
    const int p = S.my_cell;
    const int h = (p >= 0) ? min(P.height(p), 5) : 0;
    const int first = warp_excl_scan(h);
    const int total = min(__shfl_sync(kFull, first + h, 31), kTokens);
    if (p >= 0) {
        int fl[6];
        const int oc = height_neighbours(P, p, fl);
        const int c = p_to_c(p);
        const bool stun = P.stunned() == p;
        for (int lv = 0; lv < h && first + lv < kTokens; lv++) {
            const int t = first + lv;
            const uint8_t b = w->st[lv * kCells + c];
            const int pt = b & 15, pc = (b >> 4) & 1;
            const bool top = lv == h - 1;
            float f[kTokFeat];
#pragma unroll
            for (int k = 0; k < kTokFeat; k++) f[k] = 0.0f;
#pragma unroll
            for (int k = 1; k <= 8; k++)
                if (pt == k) f[k - 1] = 1.0f;
            f[8 + pc] = 1.0f;
            f[10] = lv == 0 ? 1.0f : 0.0f;
            f[11] = top ? 1.0f : 0.0f;
            f[12] = __fdiv_rn((float)h, 4.0f);
            f[13] = pt == 1 ? 1.0f : 0.0f;
            f[14] = qs[pc];
            f[15] = __fdiv_rn((float)oc, 6.0f);
            if (top) {
#pragma unroll
                for (int d = 0; d < 6; d++)
                    if (!fl[d]) f[16 + d] = 1.0f;
                f[26] = S.my_ap ? 1.0f : 0.0f;
            }
            f[24] = (float)lv * 0.25f;
            f[25] = stun ? 1.0f : 0.0f;
            float* row = tf + t * kTokFeat;
#pragma unroll
            for (int k = 0; k < kTokFeat; k++) row[k] = f[k];
            tq[t] = c % kBoard;
            tr[t] = c / kBoard;
            tz[t] = lv;
            tm[t] = 1;
        }
    }
    // zero rows past the token count
    for (int i = total * kTokFeat + l; i < kTokens * kTokFeat; i += 32) tf[i] = 0.0f;
    if (l >= total && l < kTokens) {
        tq[l] = 0;
        tr[l] = 0;
        tz[l] = 0;
        tm[l] = 0;
    }
    if (l == 0) hybrid_global(w->st, gf);
    __syncwarp();
    return total;
}

// per-position context of the move features
struct MoveCtx {
    int me, oqc, oqr, pqc, pqr, os0, ps0;
};

// queen_surround_count_current (state_encoder.cuh:109-121)
__device__ __forceinline__ int qs_current(const Pos& P, const uint8_t* st, int color) {
    if (!((st[kOffQPlaced] >> color) & 1)) return 0;
    const int q = st_u16(st, kOffQCell + 2 * color);
    return q < kCells ? height_neighbours(P, c_to_p(q), nullptr) : 0;
}

__device__ __forceinline__ MoveCtx move_ctx(WarpSmem* w) {
    Pos P{w};
    MoveCtx m;
    m.me = st_u16(w->st, kOffTurn) & 1;
    const int oq = st_u16(w->st, kOffQCell + 2 * m.me), pq = st_u16(w->st, kOffQCell + 2 * (m.me ^ 1));
    m.oqc = oq != 0xFFFF ? oq % kBoard - 11 : 0;
    m.oqr = oq != 0xFFFF ? oq / kBoard - 11 : 0;
    m.pqc = pq != 0xFFFF ? pq % kBoard - 11 : 0;
    m.pqr = pq != 0xFFFF ? pq / kBoard - 11 : 0;
    m.os0 = qs_current(P, w->st, m.me);
    m.ps0 = qs_current(P, w->st, m.me ^ 1);
    return m;
}

// queen_surround_count_after_move (state_encoder.cuh:123-165), reference cells
__device__ __forceinline__ int qs_after(const Pos& P, const uint8_t* st, int type, int pt, int from, int to,
                                        int qc, int mover, int moved) {
    const bool placed = (st[kOffQPlaced] >> qc) & 1;
    const bool being_placed = type == 0 && pt == 1 && mover == qc && to < kCells;
    const bool being_moved = type == 1 && pt == 1 && moved == qc && to < kCells;
    if (!placed && !being_placed) return 0;
    int q = placed ? st_u16(st, kOffQCell + 2 * qc) : -1;
    if (being_placed || being_moved) q = to;
    if (q < 0 || q >= kCells) return 0;
    const bool has_src = type == 1 && from < kCells;
    const int src = has_src ? from : -1;
    const int dst = to < kCells ? to : -1;
    const bool src_stays = has_src && st[kOffHeight + src] > 1;
    const int qp = c_to_p(q);
    int n = 0;
#pragma unroll
    for (int d = 0; d < 6; d++) {
        const int nb = nbr(qp, d);
        if (nb < 0) continue;
        const int c = p_to_c(nb);
        bool occ = P.height(nb) > 0;
        if (has_src && c == src) occ = src_stays;
        if (dst >= 0 && c == dst) occ = true;
        n += occ;
    }
    return n;
}

// the 31 features of one move (state_encoder.cuh:494-548)
__device__ __forceinline__ void move_features(const Pos& P, const uint8_t* st, const MoveCtx& X, int type, int pt,
                                              int from, int to, float* f) {
#pragma unroll
    for (int k = 0; k < kMoveFeat; k++) f[k] = 0.0f;
    int moved = X.me;
    if (type == 1 && from < kCells && st[kOffHeight + from] > 0)
        moved = (st[(st[kOffHeight + from] - 1) * kCells + from] >> 4) & 1;
#pragma unroll
    for (int k = 0; k < 3; k++)
        if (type == k) f[k] = 1.0f;
#pragma unroll
    for (int k = 1; k <= 8; k++)
        if (pt == k) f[2 + k] = 1.0f;
    const bool src = type == 1;
    f[11] = src ? 1.0f : 0.0f;
    int sq = 0, sr = 0, dq = 0, dr = 0, ss = 0, ds = 0;
    if (to < kCells) {
        dq = to % kBoard - 11;
        dr = to / kBoard - 11;
        ds = st[kOffHeight + to];
    }
    if (src && from < kCells) {
        sq = from % kBoard - 11;
        sr = from / kBoard - 11;
        ss = st[kOffHeight + from];
    }
    const float H = 11.0f;
    f[12] = src ? __fdiv_rn((float)(dq - sq), H) : 0.0f;
    f[13] = src ? __fdiv_rn((float)(dr - sr), H) : 0.0f;
    f[14] = __fdiv_rn((float)(dq - X.oqc), H);
    f[15] = __fdiv_rn((float)(dr - X.oqr), H);
    f[16] = __fdiv_rn((float)(dq - X.pqc), H);
    f[17] = __fdiv_rn((float)(dr - X.pqr), H);
    f[18] = src ? __fdiv_rn((float)(sq - X.oqc), H) : 0.0f;
    f[19] = src ? __fdiv_rn((float)(sr - X.oqr), H) : 0.0f;
    f[20] = src ? __fdiv_rn((float)(sq - X.pqc), H) : 0.0f;
    f[21] = src ? __fdiv_rn((float)(sr - X.pqr), H) : 0.0f;
    f[22] = __fdiv_rn((float)ss, 5.0f);
    f[23] = __fdiv_rn((float)ds, 5.0f);
    f[24] = ds > 0 ? 1.0f : 0.0f;
    int od = qs_after(P, st, type, pt, from, to, X.me, X.me, moved) - X.os0;
    int pd = qs_after(P, st, type, pt, from, to, X.me ^ 1, X.me, moved) - X.ps0;
    od = od < -1 ? -1 : (od > 1 ? 1 : od);
    pd = pd < -1 ? -1 : (pd > 1 ? 1 : pd);
#pragma unroll
    for (int k = 0; k < 3; k++) {
        if (od + 1 == k) f[25 + k] = 1.0f;
        if (pd + 1 == k) f[28 + k] = 1.0f;
    }
}

}  // namespace hv

namespace hv {

// ---------------------------------------------------------------------------
// hybrid policy / value heads (fnn_transformer_net.py:233-327), fp32:
//   value  = tanh(vh2 . relu(vh1 [e_root ; g ; global6] + b) + b)
//   g_ctx  = pg g + b                                   (policy_graph_proj)
//   logit  = pf2 . sigmoid(pf1 [e_root ; g_ctx ; e_succ ; pm m + b] + b) + b
// The move-projection block of pf1 is folded on the host:
//   pf1[:, 3E:4E] (pm m + bm) = C m + c,  C = pf1[:, 3E:4E] pm,  c = pf1[:, 3E:4E] bm
// Packed layout (transposed so lane o reads row k at column o):
//   pgT [64][E]  pgb [E]  pf1T [3E][A]  cT [31][A]  pf1b' [A] (b + c)
//   pf2 [A]  pf2b [1]  vh1T [E+70][V]  vh1b [V]  vh2 [V]  vh2b [1]
// ---------------------------------------------------------------------------
constexpr int kHybGraph = 64;
constexpr int kHybMaxValue = 128;

struct HybDims {
    int E, A, V;
};

struct HybOffsets {
    int pgT, pgb, pf1T, cT, pf1b, pf2, pf2b, vh1T, vh1b, vh2, vh2b, tcimg, rootimg, total;
};

// fp16 operand image of the per-successor network for the tensor-core row
// kernel (hv_mlp_tc.cuh), at the end of the head weights: W1 [64 x 128],
// W2 [64 x 64], [A1s | C] [64 x 96] in the K-major slab layout, zero padded
constexpr int kTcImgHalves = 64 * 128 + 64 * 64 + 64 * 96;  // 18432
// fp16 operand image of the per-leaf root network (k_leaf_root_tc), after
// it: W1 [64 x 128], W2 [64 x 64], the value layer's three K blocks
// VH1e / VH1g / VH1x [128 x 64, 128 x 64, 128 x 16] (embedding, graph,
// global features), PG [64 x 64], PF1e / PF1g [64 x 64 each] (the root and
// graph-context blocks of the action layer)
constexpr int kRootImgHalves = 64 * 128 + 64 * 64 + 128 * 64 + 128 * 64 + 128 * 16 + 64 * 64 + 2 * 64 * 64;  // 43008

__host__ __device__ inline HybOffsets hyb_offsets(HybDims d) {
    HybOffsets o;
    int p = 0;
    o.pgT = p; p += kHybGraph * d.E;
    o.pgb = p; p += d.E;
    o.pf1T = p; p += 3 * d.E * d.A;
    o.cT = p; p += kMoveFeat * d.A;
    o.pf1b = p; p += d.A;
    o.pf2 = p; p += d.A;
    o.pf2b = p; p += 1;
    o.vh1T = p; p += (d.E + kHybGraph + kGlobFeat) * d.V;
    o.vh1b = p; p += d.V;
    o.vh2 = p; p += d.V;
    o.vh2b = p; p += 1;
    p = (p + 3) & ~3;  // 16-byte aligned image
    o.tcimg = p; p += kTcImgHalves / 2;
    o.rootimg = p; p += kRootImgHalves / 2;
    o.total = p;
    return o;
}

}  // namespace hv
