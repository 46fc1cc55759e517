// hv_mlp_tc.cuh -- the hybrid evaluator's per-successor network on the
// sm_100a tensor cores (fnn_network.py:98-117 HiveFNN.encode;
// fnn_transformer_net.py:316-327 score_hybrid_actions), over the successor
// rows of a wave:
//   h = LayerNorm(sigmoid(X W1 + b1)),  e = h W2 + b2,
//   logit = pf2 . sigmoid(root_pre[leaf] + [e | m] [A1s | C]^T) + pf2b
// with X the row's 122 successor features, m its 31 move features and
// root_pre the per-leaf half of the action layer (bias, root and graph
// terms, from the leaf-root kernel).
//
// A CTA holds four independent groups of 4 warps; a group owns 128 rows at a
// time (one thread and one TMEM lane per row) with its own operands, MMA
// barrier, named barrier and 128 TMEM columns, so an SM overlaps four tiles'
// copies, GEMMs and epilogues.  The three linear layers are fp16 tcgen05.mma GEMMs (M = 128,
// N = 64, K = 128 / 64 / 64 + 32) with fp32 accumulators in TMEM, issued by
// one thread; sigmoid, LayerNorm and the output head run in fp32 on the
// row's thread straight from TMEM.  fp16 operands with fp32 accumulation
// are the reference's own arithmetic for this network (it evaluates under
// CUDA autocast).  The weights arrive once per CTA as the host-packed fp16
// image (K-major slab layout of hv_tc.cuh) by one bulk copy; a group's rows
// are read straight from global memory into its slabs.
// Every wait is bounded; a CTA that gives up sets 8 (bit 3) in the error word,
// lets its own MMAs finish, frees its TMEM and returns.
#pragma once

#include <cuda_fp16.h>

#include <cstddef>

#include "hv_fnn.cuh"
#include "hv_hybrid.cuh"
#include "hv_tc.cuh"

namespace hv {

constexpr int kTcRows = 128, kTcGroups = 4, kTcGroupThreads = 128, kTcThreads = kTcGroups * kTcGroupThreads;
constexpr uint32_t kErrMlpWait = 8u;

struct __align__(128) MlpTcGroup {
    __half a[16][kTcRows][8];  // A operand: X, then h, then e
    __half m[4][kTcRows][8];   // move features (31, padded to 32)
};

struct __align__(128) MlpTcSmem {
    __half w1[16][64][8];   // W1 [64 x 128] (features padded 122 -> 128), slab layout
    __half w2[8][64][8];    // W2 [64 x 64]
    __half w3[12][64][8];   // [A1s | C] [64 x 96]: successor block, then the folded move projection
    MlpTcGroup g[kTcGroups];
    float b1[64], g1[64], be1[64], b2[64], a2[64];
    float a2b;
    uint64_t bar_w, bar[kTcGroups], bar_x[kTcGroups];
    uint32_t tmem;
    int fail[kTcGroups];
};
static_assert(sizeof(__half) * kTcImgHalves == sizeof(MlpTcSmem::w1) + sizeof(MlpTcSmem::w2) + sizeof(MlpTcSmem::w3),
              "weight image size");

// 8 values -> one 16-byte slab row (row r of chunk c)
__device__ __forceinline__ void tc_put8(__half (*slab)[kTcRows][8], int c, int r, const float* x) {
    __half2 p0 = __floats2half2_rn(x[0], x[1]);
    __half2 p1 = __floats2half2_rn(x[2], x[3]);
    __half2 p2 = __floats2half2_rn(x[4], x[5]);
    __half2 p3 = __floats2half2_rn(x[6], x[7]);
    uint4 u;
    u.x = *reinterpret_cast<uint32_t*>(&p0);
    u.y = *reinterpret_cast<uint32_t*>(&p1);
    u.z = *reinterpret_cast<uint32_t*>(&p2);
    u.w = *reinterpret_cast<uint32_t*>(&p3);
    *reinterpret_cast<uint4*>(&slab[c][r][0]) = u;
}

// issue K/16 MMA steps D (+)= A[128 x k] B[64 x k]^T, both in slab layout
// (A: 128 rows per 8-wide K chunk, B: 64 rows)
__device__ __forceinline__ void tc_gemm(uint32_t d, const void* a, const void* b, int k, bool acc) {
    const uint32_t id = idesc_f16_m128(64);
    const char* pa = static_cast<const char*>(a);
    const char* pb = static_cast<const char*>(b);
    for (int s = 0; s < k / 16; s++)
        mma_f16(d, sdesc(pa + s * 2 * kTcRows * 16, kTcRows * 16, 128), sdesc(pb + s * 2 * 64 * 16, 64 * 16, 128), id,
                (acc || s > 0) ? 1u : 0u);
}

// barrier of one group's 128 threads (named barrier 1 + g)
__device__ __forceinline__ void group_sync(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kTcGroupThreads) : "memory");
}

// one group: make the slab writes visible to the tensor core, the group's
// thread 0 issues `issue` and commits; the group waits (bounded).  Uniform
// over the group: false if any of its threads' waits gave up.
template <typename F>
__device__ __forceinline__ bool tc_round(MlpTcSmem* s, int g, int gt, uint32_t& phase, F issue) {
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

// X / MF: the rows' successor and move features as fp16 slab tiles (written
// so by k_successor_features<true> / k_row_move_features): one tile is
// 16 x 128 x 8 and 4 x 128 x 8 halves, copied as they are into the group's
// A operands
__global__ void __launch_bounds__(kTcThreads, 1) k_mlp_rows_tc(const __half* __restrict__ X,
                                                               const __half* __restrict__ MF,
                                                               const int64_t* __restrict__ atr,
                                                               const int64_t* __restrict__ mi, int64_t N,
                                                               const float* __restrict__ root_pre,
                                                               const float* __restrict__ fw, FnnDims fd,
                                                               const float* __restrict__ hw, HybDims hd,
                                                               float* __restrict__ logits,
                                                               const int64_t* __restrict__ n_actual,
                                                               uint32_t* __restrict__ err_word) {
    extern __shared__ __align__(128) uint8_t tc_raw[];
    MlpTcSmem* s = reinterpret_cast<MlpTcSmem*>(tc_raw);
    const int t = threadIdx.x, w = t >> 5;
    const int g = t / kTcGroupThreads, gt = t - g * kTcGroupThreads;  // group, row within the tile
    MlpTcGroup* G = &s->g[g];
    const int H = fd.H, E = fd.E, A = hd.A;
    const FnnOffsets fo = fnn_offsets(fd);
    const HybOffsets ho = hyb_offsets(hd);
    if (n_actual) N = min(N, *n_actual);  // rows actually filled
    const int64_t tiles = (N + kTcRows - 1) / kTcRows;

    for (int o = t; o < 64; o += kTcThreads) {
        s->b1[o] = o < H ? __ldg(fw + fo.b1 + o) : 0.0f;
        s->g1[o] = o < H ? __ldg(fw + fo.g1 + o) : 0.0f;
        s->be1[o] = o < H ? __ldg(fw + fo.be1 + o) : 0.0f;
        s->b2[o] = o < E ? __ldg(fw + fo.b2 + o) : 0.0f;
        s->a2[o] = o < A ? __ldg(hw + ho.pf2 + o) : 0.0f;
    }
    if (t < kTcGroups) s->fail[t] = 0;
    const bool live = (int64_t)blockIdx.x * kTcGroups < tiles;
    if (t == 0) {
        s->a2b = __ldg(hw + ho.pf2b);
        mbar_init(&s->bar_w, 1);
        for (int i = 0; i < kTcGroups; i++) {
            mbar_init(&s->bar[i], 1);
            mbar_init(&s->bar_x[i], 1);
        }
        fence_mbar_init();
        if (live) {
            // the weight image (host-packed fp16 slabs)
            mbar_expect_tx(&s->bar_w, (uint32_t)(kTcImgHalves * 2));
            bulk_g2s(&s->w1[0][0][0], hw + ho.tcimg, (uint32_t)(kTcImgHalves * 2), &s->bar_w);
        }
    }
    if (w == 0) {
        tmem_alloc(&s->tmem, 512);
        tmem_relinquish();
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    bool failed = false, pending = false;
    if (live) {
        const bool ok = mbar_wait(&s->bar_w, 0);  // every thread, bounded
        failed = __syncthreads_or(!ok) != 0;
    }
    const uint32_t tcol = s->tmem + 128u * (uint32_t)g;
    const uint32_t lane = tcol + ((uint32_t)((w & 3) * 32) << 16);  // this thread's TMEM lane (row gt)
    uint32_t phase = 0, xphase = 0;
    bool xpend = false;
    for (int64_t tile = (int64_t)blockIdx.x * kTcGroups + g; tile < tiles && !failed;
         tile += (int64_t)gridDim.x * kTcGroups) {
        const int64_t r0 = tile * kTcRows;
        const int nrows = (int)min((int64_t)kTcRows, N - r0);
        // ---- this tile's slabs, as written by the feature kernels (the
        // previous tile's MMAs reading the operands have completed)
        {
            constexpr uint32_t bx = sizeof(G->a), bm = sizeof(G->m);
            if (gt == 0) {
                mbar_expect_tx(&s->bar_x[g], bx + bm);
                bulk_g2s(&G->a[0][0][0], X + tile * (bx / 2), bx, &s->bar_x[g]);
                bulk_g2s(&G->m[0][0][0], MF + tile * (bm / 2), bm, &s->bar_x[g]);
            }
            xpend = true;
            const bool ok = mbar_wait(&s->bar_x[g], xphase);
            if (!ok) s->fail[g] = 1;
            group_sync(g);
            if (s->fail[g]) {
                failed = true;
                break;
            }
            xphase ^= 1u;
            xpend = false;
        }
        // ---- D[0:64] = X W1^T
        pending = true;
        if (!tc_round(s, g, gt, phase, [&] { tc_gemm(tcol, &G->a[0][0][0], &s->w1[0][0][0], 128, false); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
            float mean = 0.0f;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                d[j] = j < H ? sigmoidf_(d[j] + s->b1[j]) : 0.0f;
                mean += d[j];
            }
            mean /= (float)H;
            float var = 0.0f;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                d[j] = j < H ? d[j] - mean : 0.0f;
                var += d[j] * d[j];
            }
            const float rstd = 1.0f / sqrtf(var / (float)H + 1e-5f);
#pragma unroll
            for (int j = 0; j < 64; j++) d[j] = d[j] * rstd * s->g1[j] + s->be1[j];
#pragma unroll
            for (int c = 0; c < 8; c++) tc_put8(G->a, c, gt, d + 8 * c);
        }
        // ---- D[64:128] = h W2^T
        pending = true;
        if (!tc_round(s, g, gt, phase, [&] { tc_gemm(tcol + 64, &G->a[0][0][0], &s->w2[0][0][0], 64, false); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane + 64, d);
            tmem_ld32(lane + 96, d + 32);
#pragma unroll
            for (int j = 0; j < 64; j++) d[j] += s->b2[j];
#pragma unroll
            for (int c = 0; c < 8; c++) tc_put8(G->a, c, gt, d + 8 * c);
        }
        // ---- D[0:64] = e A1s^T + m C^T
        pending = true;
        if (!tc_round(s, g, gt, phase, [&] {
                tc_gemm(tcol, &G->a[0][0][0], &s->w3[0][0][0], 64, false);
                tc_gemm(tcol, &G->m[0][0][0], &s->w3[8][0][0], 32, true);
            })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
            if (gt < nrows) {
                const int64_t leaf = atr[r0 + gt];
                const float4* rp = reinterpret_cast<const float4*>(root_pre + leaf * 64);
                float p = 0.0f;
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const float4 v = __ldg(rp + q);
                    const float pre[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int j = 4 * q + u;
                        if (j < A) p += s->a2[j] * sigmoidf_(pre[u] + d[j]);
                    }
                }
                logits[leaf * kMaxMoves + mi[r0 + gt]] = p + s->a2b;
            }
        }
        // the slabs are rewritten by the next tile only after every thread of
        // the group has read its TMEM lane (the next round's group barrier)
    }
    if (failed) {
        // a bounded wait gave up: record it, let the group's MMAs and the
        // weight copy finish (bounded again), free TMEM and return
        if (gt == 0) atomicOr(err_word, kErrMlpWait);
        if (pending) mbar_drain(&s->bar[g], phase ^ 1u);
        if (gt == 0 && xpend) mbar_drain(&s->bar_x[g], xphase);
        if (t == 0 && live) mbar_drain(&s->bar_w, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (w == 0) {
        tc_fence_after();
        tmem_dealloc(s->tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// per-leaf root network (the hybrid's part of HybridMCTSOrchestrator.
// _eval_states that depends on the leaf alone, fnn_transformer_net.py:
// 316-357): e = encode(root features), value = tanh(vh2 . relu(VH1 [e | g |
// global] + vh1b) + vh2b), g_ctx = PG g + pgb, root_pre = pf1b' + PF1e e +
// PF1g g_ctx.  Three independent 4-warp groups per CTA, 128 leaves per
// group tile, five fp16 tcgen05 GEMMs with fp32 accumulators in TMEM.
// ---------------------------------------------------------------------------
constexpr int kRtGroups = 3, kRtThreads = kRtGroups * kTcGroupThreads;

struct __align__(128) RootTcGroup {
    __half a[16][kTcRows][8];  // X; then h | g; then e | g; then e | g_ctx
    __half x[2][kTcRows][8];   // global features (6, padded to 16)
};

struct __align__(128) RootTcSmem {
    __half w1[16][64][8], w2[8][64][8];
    __half vhe[8][128][8], vhg[8][128][8], vhx[2][128][8];
    __half pg[8][64][8], pfe[8][64][8], pfg[8][64][8];
    RootTcGroup g[kRtGroups];
    float b1[64], g1[64], be1[64], b2[64], vh1b[128], vh2[128], pgb[64], pf1b[64];
    float vh2b;
    uint64_t bar_w, bar[kRtGroups];
    uint32_t tmem;
    int fail[kRtGroups];
};
static_assert(sizeof(__half) * kRootImgHalves ==
                  offsetof(RootTcSmem, g) - offsetof(RootTcSmem, w1), "root weight image size");

// D (+)= A[128 x k] B[n x k]^T, both in slab layout (A 128 rows, B n rows)
__device__ __forceinline__ void tc_gemm_n(uint32_t d, const void* a, const void* b, int k, int n, bool acc) {
    const uint32_t id = idesc_f16_m128(n);
    const char* pa = static_cast<const char*>(a);
    const char* pb = static_cast<const char*>(b);
    for (int s = 0; s < k / 16; s++)
        mma_f16(d, sdesc(pa + s * 2 * kTcRows * 16, kTcRows * 16, 128), sdesc(pb + s * 2 * n * 16, n * 16, 128), id,
                (acc || s > 0) ? 1u : 0u);
}

template <typename F>
__device__ __forceinline__ bool rt_round(RootTcSmem* s, int g, int gt, uint32_t& phase, F issue) {
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

__global__ void __launch_bounds__(kRtThreads, 1) k_leaf_root_tc(const float* __restrict__ root_feats,
                                                                const float* __restrict__ graph,
                                                                const float* __restrict__ glob, int64_t count,
                                                                const float* __restrict__ fw, FnnDims fd,
                                                                const float* __restrict__ hw, HybDims hd,
                                                                float* __restrict__ values,
                                                                float* __restrict__ root_pre,
                                                                uint32_t* __restrict__ err_word) {
    extern __shared__ __align__(128) uint8_t rt_raw[];
    RootTcSmem* s = reinterpret_cast<RootTcSmem*>(rt_raw);
    const int t = threadIdx.x, w = t >> 5;
    const int g = t / kTcGroupThreads, gt = t - g * kTcGroupThreads;
    RootTcGroup* G = &s->g[g];
    const int H = fd.H, E = fd.E, A = hd.A, V = hd.V;
    const FnnOffsets fo = fnn_offsets(fd);
    const HybOffsets ho = hyb_offsets(hd);
    const int64_t tiles = (count + kTcRows - 1) / kTcRows;

    for (int o = t; o < 128; o += kRtThreads) {
        if (o < 64) {
            s->b1[o] = o < H ? __ldg(fw + fo.b1 + o) : 0.0f;
            s->g1[o] = o < H ? __ldg(fw + fo.g1 + o) : 0.0f;
            s->be1[o] = o < H ? __ldg(fw + fo.be1 + o) : 0.0f;
            s->b2[o] = o < E ? __ldg(fw + fo.b2 + o) : 0.0f;
            s->pgb[o] = o < E ? __ldg(hw + ho.pgb + o) : 0.0f;
            s->pf1b[o] = o < A ? __ldg(hw + ho.pf1b + o) : 0.0f;
        }
        s->vh1b[o] = o < V ? __ldg(hw + ho.vh1b + o) : 0.0f;
        s->vh2[o] = o < V ? __ldg(hw + ho.vh2 + o) : 0.0f;
    }
    {
        uint4* z = reinterpret_cast<uint4*>(&s->g[0]);
        for (int i = t; i < (int)(sizeof(s->g) / 16); i += kRtThreads) z[i] = make_uint4(0, 0, 0, 0);
    }
    if (t < kRtGroups) s->fail[t] = 0;
    const bool live = (int64_t)blockIdx.x * kRtGroups < tiles;
    if (t == 0) {
        s->vh2b = __ldg(hw + ho.vh2b);
        mbar_init(&s->bar_w, 1);
        for (int i = 0; i < kRtGroups; i++) mbar_init(&s->bar[i], 1);
        fence_mbar_init();
        if (live) {
            mbar_expect_tx(&s->bar_w, (uint32_t)(kRootImgHalves * 2));
            bulk_g2s(&s->w1[0][0][0], hw + ho.rootimg, (uint32_t)(kRootImgHalves * 2), &s->bar_w);
        }
    }
    if (w == 0) {
        tmem_alloc(&s->tmem, 512);
        tmem_relinquish();
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    bool failed = false, pending = false;
    if (live) {
        const bool ok = mbar_wait(&s->bar_w, 0);
        failed = __syncthreads_or(!ok) != 0;
    }
    const uint32_t tcol = s->tmem + 128u * (uint32_t)g;
    const uint32_t lane = tcol + ((uint32_t)((w & 3) * 32) << 16);
    uint32_t phase = 0;
    for (int64_t tile = (int64_t)blockIdx.x * kRtGroups + g; tile < tiles && !failed;
         tile += (int64_t)gridDim.x * kRtGroups) {
        const int64_t p0 = tile * kTcRows;
        const int nl = (int)min((int64_t)kTcRows, count - p0);
        const int64_t p = p0 + gt;
        const bool mine = gt < nl;
        {
            const float2* xg = reinterpret_cast<const float2*>(root_feats + p0 * kFeat);
            const int nx = nl * (kFeat / 2);
#pragma unroll 4
            for (int i = gt; i < nx; i += kTcGroupThreads) {
                const int r = i / (kFeat / 2), k = 2 * (i - r * (kFeat / 2));
                const float2 v = __ldg(xg + i);
                *reinterpret_cast<__half2*>(&G->a[k >> 3][r][k & 7]) = __floats2half2_rn(v.x, v.y);
            }
            if (mine) {
#pragma unroll
                for (int k = 0; k < kGlobFeat; k++) G->x[0][gt][k] = __float2half_rn(__ldg(glob + p * kGlobFeat + k));
            }
        }
        // ---- encode: D[0:64] = X W1^T, h = LayerNorm(sigmoid(. + b1))
        pending = true;
        if (!rt_round(s, g, gt, phase, [&] { tc_gemm_n(tcol, &G->a[0][0][0], &s->w1[0][0][0], 128, 64, false); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
            float mean = 0.0f;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                d[j] = j < H ? sigmoidf_(d[j] + s->b1[j]) : 0.0f;
                mean += d[j];
            }
            mean /= (float)H;
            float var = 0.0f;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                d[j] = j < H ? d[j] - mean : 0.0f;
                var += d[j] * d[j];
            }
            const float rstd = 1.0f / sqrtf(var / (float)H + 1e-5f);
#pragma unroll
            for (int j = 0; j < 64; j++) d[j] = d[j] * rstd * s->g1[j] + s->be1[j];
#pragma unroll
            for (int c = 0; c < 8; c++) tc_put8(G->a, c, gt, d + 8 * c);
            // the trunk's graph summary into K 64..127
            if (mine) {
                const float4* gp = reinterpret_cast<const float4*>(graph + p * kHybGraph);
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const float4 v = __ldg(gp + q);
                    d[4 * q] = v.x;
                    d[4 * q + 1] = v.y;
                    d[4 * q + 2] = v.z;
                    d[4 * q + 3] = v.w;
                }
#pragma unroll
                for (int c = 0; c < 8; c++) tc_put8(G->a, 8 + c, gt, d + 8 * c);
            }
        }
        // ---- D[64:128] = h W2^T, e = . + b2
        pending = true;
        if (!rt_round(s, g, gt, phase, [&] { tc_gemm_n(tcol + 64, &G->a[0][0][0], &s->w2[0][0][0], 64, 64, false); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane + 64, d);
            tmem_ld32(lane + 96, d + 32);
#pragma unroll
            for (int j = 0; j < 64; j++) d[j] += s->b2[j];
#pragma unroll
            for (int c = 0; c < 8; c++) tc_put8(G->a, c, gt, d + 8 * c);
        }
        // ---- value hidden: D[0:128] = e VH1e^T + g VH1g^T + x VH1x^T
        pending = true;
        if (!rt_round(s, g, gt, phase, [&] {
                tc_gemm_n(tcol, &G->a[0][0][0], &s->vhe[0][0][0], 64, 128, false);
                tc_gemm_n(tcol, &G->a[8][0][0], &s->vhg[0][0][0], 64, 128, true);
                tc_gemm_n(tcol, &G->x[0][0][0], &s->vhx[0][0][0], 16, 128, true);
            })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float part = 0.0f, d[32];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                tmem_ld32(lane + 32 * c, d);
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int j = 32 * c + i;
                    if (j < V) part += s->vh2[j] * fmaxf(d[i] + s->vh1b[j], 0.0f);
                }
            }
            if (mine) values[p] = tanhf(part + s->vh2b);
        }
        // ---- graph context: D[0:64] = g PG^T, g_ctx = . + pgb (over g in K 64..127)
        pending = true;
        if (!rt_round(s, g, gt, phase, [&] { tc_gemm_n(tcol, &G->a[8][0][0], &s->pg[0][0][0], 64, 64, false); })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane, d);
            tmem_ld32(lane + 32, d + 32);
#pragma unroll
            for (int j = 0; j < 64; j++) d[j] += s->pgb[j];
#pragma unroll
            for (int c = 0; c < 8; c++) tc_put8(G->a, 8 + c, gt, d + 8 * c);
        }
        // ---- root half of the action layer: D[64:128] = e PF1e^T + g_ctx PF1g^T
        pending = true;
        if (!rt_round(s, g, gt, phase, [&] {
                tc_gemm_n(tcol + 64, &G->a[0][0][0], &s->pfe[0][0][0], 64, 64, false);
                tc_gemm_n(tcol + 64, &G->a[8][0][0], &s->pfg[0][0][0], 64, 64, true);
            })) {
            failed = true;
            break;
        }
        pending = false;
        {
            float d[64];
            tmem_ld32(lane + 64, d);
            tmem_ld32(lane + 96, d + 32);
            if (mine) {
                float4* rp = reinterpret_cast<float4*>(root_pre + p * 64);
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    float v[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int j = 4 * q + u;
                        v[u] = j < A ? d[j] + s->pf1b[j] : 0.0f;
                    }
                    rp[q] = make_float4(v[0], v[1], v[2], v[3]);
                }
            }
        }
    }
    if (failed) {
        // as in k_mlp_rows_tc: record, drain this group's MMAs and the weight copy (bounded)
        if (gt == 0) atomicOr(err_word, kErrMlpWait);
        if (pending) mbar_drain(&s->bar[g], phase ^ 1u);
        if (t == 0 && live) mbar_drain(&s->bar_w, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (w == 0) {
        tc_fence_after();
        tmem_dealloc(s->tmem, 512);
    }
}

}  // namespace hv
