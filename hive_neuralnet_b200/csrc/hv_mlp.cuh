// hv_mlp.cuh -- the leaf evaluator's per-successor network as a tiled fp32
// GEMM pipeline over successor rows (hive_fnn/fnn_network.py:98-143 encode /
// value_head / score_actions; fnn_transformer_net.py:316-327 for the hybrid
// action head).
//
// Rows are the successors of all leaves of a wave, compacted (row r belongs
// to leaf atr[r], legal slot mi[r]); their 122 features were written by the
// successor-feature kernel.  A CTA of 256 threads owns 64 rows at a time and
// keeps the network's weights resident in shared memory; every thread holds
// a 4 x 4 block of (row, neuron) accumulators, so each shared-memory operand
// load feeds 4 FMAs, against 1-2 in the warp-per-leaf evaluator.  fp32
// throughout (the FNN is checked at 1e-5 relative).
//   encode:   h = LayerNorm(sigmoid(X W1 + b1)),  e = h W2 + b2
//   FNN:      child_q = -tanh(wv . e + bv)
//             logit   = a2 . sigmoid(root_pre[leaf] + A1s e) + a2b
//   hybrid:   logit   = pf2 . sigmoid(root_pre[leaf] + PF1s e + C m) + pf2b
// root_pre holds the per-leaf half of the action layer (bias + root terms).
#pragma once

#include "hv_core.cuh"
#include "hv_fnn.cuh"
#include "hv_hybrid.cuh"

namespace hv {

constexpr int kMlpRows = 64;
constexpr int kMlpThreads = 256;
constexpr int kMlpHs = 65;  // row stride of the hidden / embedding tile

// Tile buffer (floats): the feature tile [64][122] at 0; once it is consumed,
// the hidden rows h [64][65] at 0, then the embeddings e [64][65] over them;
// the hybrid's move features [64][32] after the feature tile at kMlpM.
constexpr int kMlpM = kMlpRows * kFeat;  // 7808
template <bool HYB>
struct MlpSmem {
    float w1[kFeat][64];     // W1^T, columns >= H zero
    float w2[64][64];        // W2^T, rows >= H and columns >= E zero
    float a1[64][64];        // successor block of the action layer, rows >= E / columns >= A zero
    float c[HYB ? 32 : 1][64];  // hybrid: folded move projection C^T, rows >= 31 zero
    float b1[64], g1[64], be1[64], b2[64], wv[64], a2[64];
    float bv, a2b, pad_[2];
    float buf[kMlpM + (HYB ? kMlpRows * 32 : 0)];  // two 8-warp CTAs per SM for both variants
};

// sum over the 16 lanes (tx) that share a row
__device__ __forceinline__ float row_sum16(float v) {
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <bool HYB, bool ROOT = false>
__device__ void mlp_load_weights(MlpSmem<HYB>* s, const float* __restrict__ fw, FnnDims fd, const float* __restrict__ hw,
                                 HybDims hd) {
    const FnnOffsets fo = fnn_offsets(fd);
    const int t = threadIdx.x;
    const int H = fd.H, E = fd.E;
    const int A = HYB ? hd.A : fd.A;
    for (int i = t; i < kFeat * 64; i += kMlpThreads) {
        const int k = i >> 6, o = i & 63;
        s->w1[k][o] = o < H ? __ldg(fw + fo.w1t + k * H + o) : 0.0f;
    }
    for (int i = t; i < 64 * 64; i += kMlpThreads) {
        const int k = i >> 6, o = i & 63;
        s->w2[k][o] = (k < H && o < E) ? __ldg(fw + fo.w2t + k * E + o) : 0.0f;
        float a = 0.0f;
        if (k < E && o < A) {
            if (HYB) a = __ldg(hw + hyb_offsets(hd).pf1T + (2 * E + k) * A + o);
            else a = __ldg(fw + fo.a1t + ((ROOT ? 0 : E) + k) * A + o);  // root or successor half
        }
        s->a1[k][o] = a;
    }
    if (HYB) {
        const HybOffsets ho = hyb_offsets(hd);
        for (int i = t; i < 32 * 64; i += kMlpThreads) {
            const int k = i >> 6, o = i & 63;
            s->c[k][o] = (k < kMoveFeat && o < A) ? __ldg(hw + ho.cT + k * A + o) : 0.0f;
        }
    }
    for (int o = t; o < 64; o += kMlpThreads) {
        s->b1[o] = o < H ? __ldg(fw + fo.b1 + o) : 0.0f;
        s->g1[o] = o < H ? __ldg(fw + fo.g1 + o) : 0.0f;
        s->be1[o] = o < H ? __ldg(fw + fo.be1 + o) : 0.0f;
        s->b2[o] = o < E ? __ldg(fw + fo.b2 + o) : 0.0f;
        s->wv[o] = o < E ? __ldg(fw + fo.wv + o) : 0.0f;
        if (HYB) s->a2[o] = o < A ? __ldg(hw + hyb_offsets(hd).pf2 + o) : 0.0f;
        else if (ROOT) s->a2[o] = o < A ? __ldg(fw + fo.a1b + o) : 0.0f;  // ROOT: the action layer's bias
        else s->a2[o] = o < A ? __ldg(fw + fo.a2 + o) : 0.0f;
    }
    if (t == 0) {
        s->bv = __ldg(fw + fo.bv);
        s->a2b = HYB ? __ldg(hw + hyb_offsets(hd).pf2b) : __ldg(fw + fo.a2b);
    }
}

// rows [0, N): features X [N][122] (+ move features MF [N][31] for the hybrid),
// leaf / slot of each row, per-leaf action pre-activations root_pre [T][64];
// writes logits[leaf * 256 + slot] and (FNN) child_q[leaf * 256 + slot].
// ROOT (FNN): the rows are the leaves' own root features; writes the value
// (child_q: values [N]) and the root half of the action layer
// (root_pre [N][64]: a1b + A1[:, 0:E] e, zero past A) -- the per-leaf part of
// the evaluator (fnn_network.py:98-143), tiled.
template <bool HYB, bool ROOT = false>
__global__ void __launch_bounds__(kMlpThreads, 2) k_mlp_rows(const float* __restrict__ X,
                                                            const float* __restrict__ MF,
                                                            const int64_t* __restrict__ atr,
                                                            const int64_t* __restrict__ mi, int64_t N,
                                                            const float* __restrict__ root_pre,
                                                            const float* __restrict__ fw, FnnDims fd,
                                                            const float* __restrict__ hw, HybDims hd,
                                                            float* __restrict__ logits, float* __restrict__ child_q,
                                                            const int64_t* __restrict__ n_actual) {
    extern __shared__ __align__(16) uint8_t mlp_raw[];
    MlpSmem<HYB>* s = reinterpret_cast<MlpSmem<HYB>*>(mlp_raw);
    float* xs = s->buf;            // feature tile, row stride 122
    float* hs = s->buf;            // hidden rows, stride 65 (after the tile is consumed)
    float* es = s->buf;            // embeddings, stride 65 (after the hidden rows are consumed)
    float* ms = s->buf + kMlpM;    // hybrid move features, stride 32
    const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
    const int H = fd.H, E = fd.E;
    const int A = HYB ? hd.A : fd.A;
    const float invH = 1.0f / (float)H;
    mlp_load_weights<HYB, ROOT>(s, fw, fd, hw, hd);
    __syncthreads();
    if (n_actual) N = min(N, *n_actual);  // rows actually filled
    const int64_t tiles = (N + kMlpRows - 1) / kMlpRows;
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int64_t r0 = tile * kMlpRows;
        const int nrows = (int)min((int64_t)kMlpRows, N - r0);
        // feature tile (rows past N are zero)
        const float* xg = X + r0 * kFeat;
#pragma unroll 8
        for (int i = t; i < kMlpRows * kFeat; i += kMlpThreads) xs[i] = i < nrows * kFeat ? __ldg(xg + i) : 0.0f;
        if (HYB) {
#pragma unroll 8
            for (int i = t; i < kMlpRows * 32; i += kMlpThreads) {
                const int r = i >> 5, k = i & 31;
                ms[i] = (r < nrows && k < kMoveFeat) ? MF[(r0 + r) * kMoveFeat + k] : 0.0f;
            }
        }
        __syncthreads();
        // ---- h = LayerNorm(sigmoid(X W1 + b1))
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = s->b1[4 * tx + j];
#pragma unroll 2
        for (int k = 0; k < kFeat; k++) {
            const float4 w = *reinterpret_cast<const float4*>(&s->w1[k][4 * tx]);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float x = xs[(4 * ty + i) * kFeat + k];
                acc[i][0] = fmaf(x, w.x, acc[i][0]);
                acc[i][1] = fmaf(x, w.y, acc[i][1]);
                acc[i][2] = fmaf(x, w.z, acc[i][2]);
                acc[i][3] = fmaf(x, w.w, acc[i][3]);
            }
        }
        __syncthreads();  // the feature tile is consumed: h overwrites it
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float a[4], sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                a[j] = (4 * tx + j) < H ? sigmoidf_(acc[i][j]) : 0.0f;
                sum += a[j];
            }
            const float mean = row_sum16(sum) * invH;
            float sq = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float d = (4 * tx + j) < H ? a[j] - mean : 0.0f;
                a[j] = d;
                sq += d * d;
            }
            const float rstd = 1.0f / sqrtf(row_sum16(sq) * invH + 1e-5f);
#pragma unroll
            for (int j = 0; j < 4; j++)
                hs[(4 * ty + i) * kMlpHs + 4 * tx + j] = a[j] * rstd * s->g1[4 * tx + j] + s->be1[4 * tx + j];
        }
        __syncthreads();
        // ---- e = h W2 + b2
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = s->b2[4 * tx + j];
#pragma unroll 2
        for (int k = 0; k < H; k++) {
            const float4 w = *reinterpret_cast<const float4*>(&s->w2[k][4 * tx]);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float h = hs[(4 * ty + i) * kMlpHs + k];
                acc[i][0] = fmaf(h, w.x, acc[i][0]);
                acc[i][1] = fmaf(h, w.y, acc[i][1]);
                acc[i][2] = fmaf(h, w.z, acc[i][2]);
                acc[i][3] = fmaf(h, w.w, acc[i][3]);
            }
        }
        __syncthreads();  // the hidden rows are consumed: e overwrites them
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = 4 * ty + i;
#pragma unroll
            for (int j = 0; j < 4; j++) es[r * kMlpHs + 4 * tx + j] = acc[i][j];
            if (!HYB) {
                float pv = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; j++) pv += s->wv[4 * tx + j] * acc[i][j];
                pv = row_sum16(pv);
                if (ROOT) {
                    if (tx == 0 && r < nrows) child_q[r0 + r] = tanhf(pv + s->bv);
                } else if (tx == 0 && r < nrows) {
                    child_q[atr[r0 + r] * kMaxMoves + mi[r0 + r]] = -tanhf(pv + s->bv);
                }
            }
        }
        __syncthreads();
        // ---- logits: a2 . sigmoid(root_pre + A1s e (+ C m)) + a2b
        int64_t leaf[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = 4 * ty + i;
            leaf[i] = ROOT ? 0 : (r < nrows ? atr[r0 + r] : 0);
#pragma unroll
            for (int j = 0; j < 4; j++)
                acc[i][j] = (4 * tx + j) < A ? (ROOT ? s->a2[4 * tx + j] : root_pre[leaf[i] * 64 + 4 * tx + j]) : 0.0f;
        }
#pragma unroll 2
        for (int k = 0; k < E; k++) {
            const float4 w = *reinterpret_cast<const float4*>(&s->a1[k][4 * tx]);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float e = es[(4 * ty + i) * kMlpHs + k];
                acc[i][0] = fmaf(e, w.x, acc[i][0]);
                acc[i][1] = fmaf(e, w.y, acc[i][1]);
                acc[i][2] = fmaf(e, w.z, acc[i][2]);
                acc[i][3] = fmaf(e, w.w, acc[i][3]);
            }
        }
        if (HYB) {
#pragma unroll 2
            for (int k = 0; k < kMoveFeat; k++) {
                const float4 w = *reinterpret_cast<const float4*>(&s->c[k][4 * tx]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float m = ms[(4 * ty + i) * 32 + k];
                    acc[i][0] = fmaf(m, w.x, acc[i][0]);
                    acc[i][1] = fmaf(m, w.y, acc[i][1]);
                    acc[i][2] = fmaf(m, w.z, acc[i][2]);
                    acc[i][3] = fmaf(m, w.w, acc[i][3]);
                }
            }
        }
        if (ROOT) {
            float* rp = logits;  // ROOT: root_pre [N][64]
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = 4 * ty + i;
                if (r < nrows)
                    *reinterpret_cast<float4*>(rp + (r0 + r) * 64 + 4 * tx) = make_float4(acc[i][0], acc[i][1],
                                                                                       acc[i][2], acc[i][3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = 4 * ty + i;
                float p = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if ((4 * tx + j) < A) p += s->a2[4 * tx + j] * sigmoidf_(acc[i][j]);
                p = row_sum16(p);
                if (tx == 0 && r < nrows) logits[leaf[i] * kMaxMoves + mi[r0 + r]] = p + s->a2b;
            }
        }
        __syncthreads();
    }
}

}  // namespace hv
