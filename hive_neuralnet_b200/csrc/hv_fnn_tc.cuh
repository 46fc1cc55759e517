// hv_fnn_tc.cuh -- the FNN leaf evaluator's per-successor network on the
// sm_100a tensor cores at fp32-level accuracy (hive_fnn/fnn_network.py:98-143
// encode / value_head / score_actions, over the successor rows of a wave):
//   h = LayerNorm(sigmoid(X W1 + b1)),  e = h W2 + b2,
//   child_q = -tanh(wv . e + bv),
//   logit   = a2 . sigmoid(root_pre[leaf] + A1s e) + a2b
//
// The reference computes this network in fp32.  Each fp32 operand x is held
// as two fp16 values, hi = fp16(x) and lo = fp16(x - hi) (x = hi + lo to
// about 2^-22 relative), and every product is formed as
// hi_x hi_w + hi_x lo_w + lo_x hi_w: three fp16 tcgen05.mma GEMMs into one
// fp32 TMEM accumulator (the lo x lo term, ~2^-22, is left out).  fp16
// products are exact in the fp32 accumulator, so the result is fp32-accurate
// (checked at 1e-5 relative against the fp32 statement).
//
// The rows arrive as 128-row tiles written by k_successor_features<
// kSlabF16x2>: the 122 features' hi parts in the K-major slab layout of
// hv_tc.cuh ([16 chunks][128 rows][8], features 122..127 zero), then the lo
// parts, 64 KB, copied whole into the group's A operands by one bulk copy.
// A CTA (one per SM) holds the weights' hi / lo images, built in its
// prologue from the fp32 weights, and two independent groups of 4 warps:
// a group owns one tile (one thread and one TMEM lane per row, 64 TMEM
// columns), its own copy and MMA barriers and named barrier, so one group's
// epilogues overlap the other's copies and GEMMs.  The epilogues run in
// fp32 on the row's thread straight from TMEM and write the next layer's A
// operand (hi / lo) over the consumed one; the LayerNorm statistics and the
// two output dot products accumulate in fp64 (cheap per row, and it keeps the
// split's rounding from reaching the outputs through the normalisation).
// Every wait is bounded; a CTA that gives up sets 8 (bit 3) in the error
// word, lets its own copies and MMAs finish, frees its TMEM and returns.
#pragma once

#include <cuda_fp16.h>

#include "hv_fnn.cuh"
#include "hv_mlp_tc.cuh"
#include "hv_tc.cuh"

namespace hv {

constexpr int kFxRows = 128, kFxGroups = 2, kFxThreads = kFxGroups * kTcGroupThreads;
constexpr uint32_t kFxTileBytes = 2u * 16u * kFxRows * 8u * 2u;  // hi and lo slabs: 64 KB

struct __align__(128) FxGroup {
    __half hi[16][kFxRows][8];  // A operand, high parts: X, then h, then e
    __half lo[16][kFxRows][8];  // low parts
};

struct __align__(128) FxSmem {
    __half w1h[16][64][8], w1l[16][64][8];  // W1 [64 x 128] (features padded 122 -> 128, neurons >= H zero)
    __half w2h[8][64][8], w2l[8][64][8];    // W2 [64 x 64] (rows >= E, columns >= H zero)
    __half a1h[8][64][8], a1l[8][64][8];    // A1s [64 x 64]: successor block of the action layer
    FxGroup g[kFxGroups];
    float b1[64], g1[64], be1[64], b2[64], wv[64], a2[64];
    float bv, a2b;
    uint64_t bar[kFxGroups], bar_x[kFxGroups];
    uint32_t tmem;
    int fail[kFxGroups];
};

// x -> (hi, lo) fp16 pair
__device__ __forceinline__ void split_f16(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

// 8 values -> row r of chunk c of a hi / lo slab pair (two 16-byte stores)
__device__ __forceinline__ void fx_put8(__half (*hi)[kFxRows][8], __half (*lo)[kFxRows][8], int c, int r,
                                        const float* x) {
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; i++) split_f16(x[i], h[i], l[i]);
    *reinterpret_cast<uint4*>(&hi[c][r][0]) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(&lo[c][r][0]) = *reinterpret_cast<const uint4*>(l);
}

// B operand element (n, k) of a [64 x K] slab image
__device__ __forceinline__ int fx_bidx(int n, int k) { return ((k >> 3) * 64 + n) * 8 + (k & 7); }

// the three products of one layer into accumulator d: hi hi + hi lo + lo hi
__device__ __forceinline__ void fx_gemm3(uint32_t d, const FxGroup* G, const void* wh, const void* wl, int k) {
    tc_gemm(d, &G->hi[0][0][0], wh, k, false);
    tc_gemm(d, &G->hi[0][0][0], wl, k, true);
    tc_gemm(d, &G->lo[0][0][0], wh, k, true);
}

// one group round: operands visible to the tensor core, the group's thread 0
// issues and commits, the group waits (bounded); uniform over the group
template <typename F>
__device__ __forceinline__ bool fx_round(FxSmem* s, int g, int gt, uint32_t& phase, F issue) {
    fence_proxy_async();
    tc_fence_before();
    group_sync(g);
    if (gt == 0) {
        tc_fence_after();
        issue();
        mma_commit(&s->bar[g]);
    }
    const bool ok = mbar_wait(&s->bar[g], phase);
    phase ^= 1u;
    tc_fence_after();
    if (!ok) s->fail[g] = 1;
    group_sync(g);
    return s->fail[g] == 0;
}

// rows [0, N) of X (tiles as above), leaf / slot of each row in atr / mi,
// per-leaf action pre-activations root_pre [T][64]; writes
// logits[leaf * 256 + slot] and child_q[leaf * 256 + slot]
__global__ void __launch_bounds__(kFxThreads, 1) k_fnn_rows_tc(const __half* __restrict__ X,
                                                              const int64_t* __restrict__ atr,
                                                              const int64_t* __restrict__ mi, int64_t N,
                                                              const float* __restrict__ root_pre,
                                                              const float* __restrict__ fw, FnnDims fd,
                                                              float* __restrict__ logits, float* __restrict__ child_q,
                                                              const int64_t* __restrict__ n_actual,
                                                              uint32_t* __restrict__ err_word) {
    extern __shared__ __align__(128) uint8_t fx_raw[];
    FxSmem* s = reinterpret_cast<FxSmem*>(fx_raw);
    const int t = threadIdx.x, w = t >> 5;
    const int g = t / kTcGroupThreads, gt = t - g * kTcGroupThreads;  // group, row within the tile
    FxGroup* G = &s->g[g];
    const int H = fd.H, E = fd.E, A = fd.A;
    const FnnOffsets fo = fnn_offsets(fd);
    if (n_actual) N = min(N, *n_actual);  // rows actually filled
    const int64_t tiles = (N + kFxRows - 1) / kFxRows;

    // weights: fp32 -> hi / lo fp16 slab images
    for (int i = t; i < 64 * 128; i += kFxThreads) {
        const int n = i >> 7, k = i & 127;
        const float v = (n < H && k < kFeat) ? __ldg(fw + fo.w1t + k * H + n) : 0.0f;
        split_f16(v, (&s->w1h[0][0][0])[fx_bidx(n, k)], (&s->w1l[0][0][0])[fx_bidx(n, k)]);
    }
    for (int i = t; i < 64 * 64; i += kFxThreads) {
        const int n = i >> 6, k = i & 63;
        const float v2 = (n < E && k < H) ? __ldg(fw + fo.w2t + k * E + n) : 0.0f;
        split_f16(v2, (&s->w2h[0][0][0])[fx_bidx(n, k)], (&s->w2l[0][0][0])[fx_bidx(n, k)]);
        const float v3 = (n < A && k < E) ? __ldg(fw + fo.a1t + (E + k) * A + n) : 0.0f;
        split_f16(v3, (&s->a1h[0][0][0])[fx_bidx(n, k)], (&s->a1l[0][0][0])[fx_bidx(n, k)]);
    }
    for (int o = t; o < 64; o += kFxThreads) {
        s->b1[o] = o < H ? __ldg(fw + fo.b1 + o) : 0.0f;
        s->g1[o] = o < H ? __ldg(fw + fo.g1 + o) : 0.0f;
        s->be1[o] = o < H ? __ldg(fw + fo.be1 + o) : 0.0f;
        s->b2[o] = o < E ? __ldg(fw + fo.b2 + o) : 0.0f;
        s->wv[o] = o < E ? __ldg(fw + fo.wv + o) : 0.0f;
        s->a2[o] = o < A ? __ldg(fw + fo.a2 + o) : 0.0f;
    }
    if (t < kFxGroups) s->fail[t] = 0;
    if (t == 0) {
        s->bv = __ldg(fw + fo.bv);
        s->a2b = __ldg(fw + fo.a2b);
        for (int i = 0; i < kFxGroups; i++) {
            mbar_init(&s->bar[i], 1);
            mbar_init(&s->bar_x[i], 1);
        }
        fence_mbar_init();
    }
    if (w == 0) {
        tmem_alloc(&s->tmem, 128);
        tmem_relinquish();
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tcol = s->tmem + 64u * (uint32_t)g;
    const uint32_t lane = tcol + ((uint32_t)((w & 3) * 32) << 16);  // this thread's TMEM lane (row gt)
    uint32_t phase = 0, xphase = 0;
    bool failed = false, pending = false, xpend = false;
    for (int64_t tile = (int64_t)blockIdx.x * kFxGroups + g; tile < tiles; tile += (int64_t)gridDim.x * kFxGroups) {
        const int64_t r0 = tile * kFxRows;
        const int nrows = (int)min((int64_t)kFxRows, N - r0);
        // ---- this tile's hi / lo slabs (the previous tile's MMAs have completed)
        if (gt == 0) {
            mbar_expect_tx(&s->bar_x[g], kFxTileBytes);
            bulk_g2s(&G->hi[0][0][0], X + tile * (kFxTileBytes / 2), kFxTileBytes, &s->bar_x[g]);
        }
        xpend = true;
        {
            const bool ok = mbar_wait(&s->bar_x[g], xphase);
            if (!ok) s->fail[g] = 1;
            group_sync(g);
            if (s->fail[g]) {
                failed = true;
                break;
            }
        }
        xphase ^= 1u;
        xpend = false;
        const bool mine = gt < nrows;
        const int64_t leaf = mine ? atr[r0 + gt] : 0;
        const int64_t slot = mine ? mi[r0 + gt] : 0;

        // ---- h = LayerNorm(sigmoid(X W1 + b1))
        pending = true;
        if (!fx_round(s, g, gt, phase, [&] { fx_gemm3(tcol, G, s->w1h, s->w1l, 128); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
            // LayerNorm statistics in fp64: the split products carry ~2^-22
            // of their own, and the normalisation amplifies what comes in
            double sum = 0.0;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                d[j] = j < H ? sigmoidf_(d[j] + s->b1[j]) : 0.0f;
                sum += (double)d[j];
            }
            const double mean = sum / (double)H;
            double sq = 0.0;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                const double dj = j < H ? (double)d[j] - mean : 0.0;
                sq += dj * dj;
            }
            const double rstd = 1.0 / sqrt(sq / (double)H + 1e-5);
#pragma unroll
            for (int j = 0; j < 64; j++)
                d[j] = j < H ? (float)(((double)d[j] - mean) * rstd) * s->g1[j] + s->be1[j] : 0.0f;
#pragma unroll
            for (int c = 0; c < 8; c++) fx_put8(G->hi, G->lo, c, gt, d + 8 * c);
        }

        // ---- e = h W2 + b2, child_q = -tanh(wv . e + bv)
        pending = true;
        if (!fx_round(s, g, gt, phase, [&] { fx_gemm3(tcol, G, s->w2h, s->w2l, 64); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
            double pv = 0.0;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                d[j] = j < E ? d[j] + s->b2[j] : 0.0f;
                pv += (double)s->wv[j] * (double)d[j];
            }
            if (mine) child_q[leaf * kMaxMoves + slot] = -tanhf((float)pv + s->bv);
#pragma unroll
            for (int c = 0; c < 8; c++) fx_put8(G->hi, G->lo, c, gt, d + 8 * c);
        }

        // ---- logit = a2 . sigmoid(root_pre[leaf] + A1s e) + a2b
        pending = true;
        if (!fx_round(s, g, gt, phase, [&] { fx_gemm3(tcol, G, s->a1h, s->a1l, 64); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
            if (mine) {
                const float4* rp = reinterpret_cast<const float4*>(root_pre + leaf * 64);
                double p = 0.0;
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const float4 v = __ldg(rp + q);
                    const float pre[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int j = 4 * q + u;
                        if (j < A) p += (double)s->a2[j] * (double)sigmoidf_(pre[u] + d[j]);
                    }
                }
                logits[leaf * kMaxMoves + slot] = (float)p + s->a2b;
            }
        }
        // the slabs are rewritten by the next tile only after every thread of
        // the group has read its TMEM lane (the next round's group barrier)
        group_sync(g);
    }
    if (failed) {
        // a bounded wait gave up: record it, let the group's MMAs and its copy
        // finish (bounded again), free TMEM and return
        if (gt == 0) atomicOr(err_word, kErrMlpWait);
        if (pending) mbar_drain(&s->bar[g], phase ^ 1u);
        if (gt == 0 && xpend) mbar_drain(&s->bar_x[g], xphase);
    }
    tc_fence_before();
    __syncthreads();
    if (w == 0) {
        tc_fence_after();
        tmem_dealloc(s->tmem, 128);
    }
}

}  // namespace hv
