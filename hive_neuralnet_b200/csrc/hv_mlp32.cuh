// hv_mlp32.cuh -- the FNN leaf evaluator's per-successor network over the
// successor rows of a wave, fp32 on the CUDA cores (hive_fnn/fnn_network.py:
// 98-143 encode / value_head / score_actions):
//   h = LayerNorm(sigmoid(X W1 + b1)),  e = h W2 + b2,
//   child_q = -tanh(wv . e + bv),
//   logit   = a2 . sigmoid(root_pre[leaf] + A1s e) + a2b
// The rows arrive as fp32 tiles of 64 rows in 4-feature chunks (written so
// by k_successor_features<kSlabF32>): tile t is [32 chunks][64 rows][4]
// floats, 32 KB, copied whole into shared memory by one bulk copy while the
// previous tile computes.  A CTA (one per SM, the weights resident in shared
// memory) holds two independent groups of 8 warps with their own tiles,
// copy barriers and named barrier, so one group's epilogues (sigmoid,
// LayerNorm, tanh) overlap the other's FMAs.  A group computes 64 rows x 64
// neurons per layer; a thread holds 4 rows (ty + 16 i) x 4 neurons (4 tx):
// per 4-feature chunk it loads 4 row vectors and 4 weight vectors for 64
// FMAs (the row-major kernel, k_mlp_rows, loads 5 values per 16 FMAs and is
// bound by shared-memory bandwidth).  Every output is the same fmaf chain as
// in k_mlp_rows: from the bias, k ascending; the features past 122 and the
// neurons past H are zero and add exact zeros.  fp32 throughout (checked at
// 1e-5 relative).
// The copy waits are bounded; a CTA that gives up sets 8 (bit 3) in the error
// word, waits (bounded) for its copies in flight and returns.
#pragma once

#include "hv_fnn.cuh"
#include "hv_tc.cuh"

namespace hv {

constexpr int kF32Rows = 64, kF32Groups = 2, kF32GroupThreads = 256, kF32Chunks = 32;
constexpr int kF32Threads = kF32Groups * kF32GroupThreads;
constexpr int kF32Ty = kF32GroupThreads / 16, kF32Rpt = kF32Rows / kF32Ty;  // row groups; rows per thread
constexpr uint32_t kF32TileBytes = kF32Chunks * kF32Rows * 4 * sizeof(float);  // 32 KB
constexpr uint32_t kErrF32Wait = 8u;

struct __align__(128) F32Smem {
    float x[kF32Groups][2][kF32Chunks][kF32Rows][4];  // per group: feature tiles (double-buffered); h, then e,
                                                      // overwrite the current one
    float w1[4 * 31][64];                 // W1^T over features 0..123 (122, 123 and neurons >= H zero)
    float w2[64][64];                     // W2^T, rows >= H and columns >= E zero
    float a1[64][64];                     // successor block of the action layer, rows >= E and columns >= A zero
    float b1[64], g1[64], be1[64], b2[64], wv[64], a2[64];
    float bv, a2b;
    uint64_t bar[kF32Groups][2];
    int fail[kF32Groups];
};

// barrier of one group's 256 threads (named barrier 1 + g)
__device__ __forceinline__ void f32_group_sync(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kF32GroupThreads) : "memory");
}

// 16 lanes (tx) share a row
__device__ __forceinline__ float f32_row_sum16(float v) {
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// acc[i][j] (+)= sum over the features of chunks [0, NC) of
// src[c][row ty + 32 i] * w[4 c + q][4 tx + j].  SWZ: the layer's own h / e
// rows, stored at row r ^ (c & 7) within chunk c (the 16 lanes that write one
// row's 16 chunks then hit 8 different bank groups instead of one).
template <int NC, bool SWZ>
__device__ __forceinline__ void f32_chunks(const float (*src)[kF32Rows][4], const float (*w)[64], int tx, int ty,
                                           float (&acc)[kF32Rpt][4]) {
#pragma unroll 1
    for (int c = 0; c < NC; c++) {
        float4 wq[4];
#pragma unroll
        for (int q = 0; q < 4; q++) wq[q] = *reinterpret_cast<const float4*>(&w[4 * c + q][4 * tx]);
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++) {
            const int r = SWZ ? ((ty + kF32Ty * i) ^ (c & 7)) : ty + kF32Ty * i;
            const float4 xv = *reinterpret_cast<const float4*>(&src[c][r][0]);
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                acc[i][0] = fmaf(xs[q], wq[q].x, acc[i][0]);
                acc[i][1] = fmaf(xs[q], wq[q].y, acc[i][1]);
                acc[i][2] = fmaf(xs[q], wq[q].z, acc[i][2]);
                acc[i][3] = fmaf(xs[q], wq[q].w, acc[i][3]);
            }
        }
    }
}

// rows [0, N) of X (slab tiles), leaf / slot of each row in atr / mi,
// per-leaf action pre-activations root_pre [T][64]; writes
// logits[leaf * 256 + slot] and child_q[leaf * 256 + slot]
__global__ void __launch_bounds__(kF32Threads, 1) k_fnn_rows(const float* __restrict__ X,
                                                             const int64_t* __restrict__ atr,
                                                             const int64_t* __restrict__ mi, int64_t N,
                                                             const float* __restrict__ root_pre,
                                                             const float* __restrict__ fw, FnnDims fd,
                                                             float* __restrict__ logits, float* __restrict__ child_q,
                                                             const int64_t* __restrict__ n_actual,
                                                             uint32_t* __restrict__ err_word) {
    extern __shared__ __align__(128) uint8_t f32_raw[];
    F32Smem* s = reinterpret_cast<F32Smem*>(f32_raw);
    const int t = threadIdx.x, g = t / kF32GroupThreads, gt = t - g * kF32GroupThreads;
    const int tx = gt & 15, ty = gt >> 4;
    const int H = fd.H, E = fd.E, A = fd.A;
    const float invH = 1.0f / (float)H;
    const FnnOffsets fo = fnn_offsets(fd);
    if (n_actual) N = min(N, *n_actual);  // rows actually filled
    const int64_t tiles = (N + kF32Rows - 1) / kF32Rows;

    // group g takes tiles first, first + stride, ...
    const int64_t first = (int64_t)blockIdx.x * kF32Groups + g, stride = (int64_t)gridDim.x * kF32Groups;
    if (t == 0) {
        for (int i = 0; i < kF32Groups; i++) {
            mbar_init(&s->bar[i][0], 1);
            mbar_init(&s->bar[i][1], 1);
            s->fail[i] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (gt == 0 && first < tiles) {
        mbar_expect_tx(&s->bar[g][0], kF32TileBytes);
        bulk_g2s(&s->x[g][0][0][0][0], X + first * (kF32TileBytes / 4), kF32TileBytes, &s->bar[g][0]);
    }
    for (int i = t; i < 4 * 31 * 64; i += kF32Threads) {
        const int k = i >> 6, o = i & 63;
        s->w1[k][o] = (k < kFeat && o < H) ? __ldg(fw + fo.w1t + k * H + o) : 0.0f;
    }
    for (int i = t; i < 64 * 64; i += kF32Threads) {
        const int k = i >> 6, o = i & 63;
        s->w2[k][o] = (k < H && o < E) ? __ldg(fw + fo.w2t + k * E + o) : 0.0f;
        s->a1[k][o] = (k < E && o < A) ? __ldg(fw + fo.a1t + (E + k) * A + o) : 0.0f;
    }
    for (int o = t; o < 64; o += kF32Threads) {
        s->b1[o] = o < H ? __ldg(fw + fo.b1 + o) : 0.0f;
        s->g1[o] = o < H ? __ldg(fw + fo.g1 + o) : 0.0f;
        s->be1[o] = o < H ? __ldg(fw + fo.be1 + o) : 0.0f;
        s->b2[o] = o < E ? __ldg(fw + fo.b2 + o) : 0.0f;
        s->wv[o] = o < E ? __ldg(fw + fo.wv + o) : 0.0f;
        s->a2[o] = o < A ? __ldg(fw + fo.a2 + o) : 0.0f;
    }
    if (t == 0) {
        s->bv = __ldg(fw + fo.bv);
        s->a2b = __ldg(fw + fo.a2b);
    }
    __syncthreads();

    // bit b: wait parity of the group's buffer b; copies in flight per buffer
    // (the group's thread 0's view)
    uint32_t phases = 0u, pend = first < tiles ? 1u : 0u;
    bool failed = false;
    int buf = 0;
    for (int64_t tile = first; tile < tiles; tile += stride, buf ^= 1) {
        // the next tile into the other buffer (its last reader finished at
        // the group barrier that ended the previous tile)
        const int64_t nt = tile + stride;
        if (gt == 0 && nt < tiles) {
            fence_proxy_async();
            mbar_expect_tx(&s->bar[g][buf ^ 1], kF32TileBytes);
            bulk_g2s(&s->x[g][buf ^ 1][0][0][0], X + nt * (kF32TileBytes / 4), kF32TileBytes, &s->bar[g][buf ^ 1]);
            pend |= 2u >> buf;
        }
        const bool ok = mbar_wait(&s->bar[g][buf], (phases >> buf) & 1u);  // every thread, bounded
        if (!ok) s->fail[g] = 1;
        f32_group_sync(g);
        if (s->fail[g]) {
            failed = true;
            break;
        }
        phases ^= 1u << buf;
        pend &= ~(1u << buf);
        float (*xb)[kF32Rows][4] = s->x[g][buf];
        const int64_t r0 = tile * kF32Rows;
        const int nrows = (int)min((int64_t)kF32Rows, N - r0);
        float acc[kF32Rpt][4];
        // the rows' leaf, slot and root pre-activations, loaded now: their
        // latency passes under the first layer
        int lf[kF32Rpt], sl[kF32Rpt];
        float4 rp[kF32Rpt];
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++) {
            const int r = ty + kF32Ty * i;
            lf[i] = r < nrows ? (int)atr[r0 + r] : 0;
            sl[i] = r < nrows ? (int)mi[r0 + r] : 0;
            rp[i] = *reinterpret_cast<const float4*>(root_pre + (int64_t)lf[i] * 64 + 4 * tx);
        }

        // ---- h = LayerNorm(sigmoid(X W1 + b1))
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = s->b1[4 * tx + j];
        f32_chunks<31, false>(xb, s->w1, tx, ty, acc);
        f32_group_sync(g);  // the feature tile is consumed: h overwrites it
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++) {
            float a[4], sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                a[j] = (4 * tx + j) < H ? sigmoidf_(acc[i][j]) : 0.0f;
                sum += a[j];
            }
            const float mean = f32_row_sum16(sum) * invH;
            float sq = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float d = (4 * tx + j) < H ? a[j] - mean : 0.0f;
                a[j] = d;
                sq += d * d;
            }
            const float rstd = 1.0f / sqrtf(f32_row_sum16(sq) * invH + 1e-5f);
            float hv4[4];
#pragma unroll
            for (int j = 0; j < 4; j++) hv4[j] = a[j] * rstd * s->g1[4 * tx + j] + s->be1[4 * tx + j];
            *reinterpret_cast<float4*>(&xb[tx][(ty + kF32Ty * i) ^ (tx & 7)][0]) =
                make_float4(hv4[0], hv4[1], hv4[2], hv4[3]);
        }
        f32_group_sync(g);

        // ---- e = h W2 + b2, child_q = -tanh(wv . e + bv)
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = s->b2[4 * tx + j];
        f32_chunks<16, true>(xb, s->w2, tx, ty, acc);
        f32_group_sync(g);  // the hidden rows are consumed: e overwrites them
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++) {
            const int r = ty + kF32Ty * i;
            *reinterpret_cast<float4*>(&xb[tx][r ^ (tx & 7)][0]) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            float pv = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) pv += s->wv[4 * tx + j] * acc[i][j];
            pv = f32_row_sum16(pv);
            if (tx == 0 && r < nrows) child_q[(int64_t)lf[i] * kMaxMoves + sl[i]] = -tanhf(pv + s->bv);
        }
        f32_group_sync(g);

        // ---- logit = a2 . sigmoid(root_pre[leaf] + A1s e) + a2b
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++) {
            acc[i][0] = (4 * tx + 0) < A ? rp[i].x : 0.0f;
            acc[i][1] = (4 * tx + 1) < A ? rp[i].y : 0.0f;
            acc[i][2] = (4 * tx + 2) < A ? rp[i].z : 0.0f;
            acc[i][3] = (4 * tx + 3) < A ? rp[i].w : 0.0f;
        }
        f32_chunks<16, true>(xb, s->a1, tx, ty, acc);
#pragma unroll
        for (int i = 0; i < kF32Rpt; i++) {
            const int r = ty + kF32Ty * i;
            float p = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++)
                if ((4 * tx + j) < A) p += s->a2[4 * tx + j] * sigmoidf_(acc[i][j]);
            p = f32_row_sum16(p);
            if (tx == 0 && r < nrows) logits[(int64_t)lf[i] * kMaxMoves + sl[i]] = p + s->a2b;
        }
        f32_group_sync(g);  // this buffer takes the tile after next
    }
    if (failed) {
        // a bounded wait gave up: record it, let the copies in flight land
        // (bounded again) and return
        if (gt == 0) {
            atomicOr(err_word, kErrF32Wait);
            for (int b = 0; b < 2; b++)
                if ((pend >> b) & 1u) mbar_drain(&s->bar[g][b], (phases >> b) & 1u);
        }
    }
}

}  // namespace hv
