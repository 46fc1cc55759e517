// hv_trunk.cuh -- the hybrid evaluator's relative transformer trunk
// (fnn_transformer_net.py:75-209 RelativeSelfAttention /
// RelativeTransformerBlock / HybridRelativeTransformerTrunk), hidden 64,
// 8 heads of 8, GELU MLP 96, 4 pre-LayerNorm blocks, on sm_100a.
//
// One CTA of 16 warps owns two tiles of 4 positions = 2 x 128 rows (a
// position is 32 rows: CLS, its 28 piece tokens, 3 padding rows).  Two
// threads share a row, each holding half of its 64-wide residual stream in
// registers (warps u*8 + h*4 + q: tile u, half h, position q of the tile);
// the halves exchange their LayerNorm statistics through shared memory.
// Each tile has its own 256 TMEM columns, and one issuing thread drives both
// tiles' MMAs per GEMM.  The five linear layers of a block (token projection
// once, then QKV, attention output, MLP in and out) are fp16 tcgen05.mma
// GEMMs with M = 128 and fp32 accumulators in TMEM (fp16 operands as the
// reference's autocast, fp32 accumulation); each half reads its own columns
// back.  The per-head 32 x 32 attention of a position (head width 8, below
// the tcgen05 K step and M tile) runs on warp-level fp16 MMAs: the warp of
// half h takes heads 4h..4h+3, whose queries, keys and values its own lanes
// wrote; the queries live in the A-operand slabs of the output projection,
// which the heads overwrite one by one.  Block weights stream from global
// memory (L2-resident) into shared memory with a bulk copy issued as soon as
// the previous block's last GEMM has completed.
#pragma once

#include <cuda_fp16.h>

#include "hv_core.cuh"
#include "hv_tc.cuh"

namespace hv {

constexpr int kTrH = 64, kTrHeads = 8, kTrFfn = 96, kTrLayers = 4;
constexpr int kTrWarps = 16, kTrThreads = kTrWarps * 32, kTrTiles = 2;
constexpr int kTrPos = 8, kTrRows = kTrPos * 32;  // 8 positions (256 rows) per CTA pass
constexpr int kTrKin = 32;   // token features, zero-padded to two MMA K steps
constexpr int kTrQkStride = 72;  // fp16 row stride of Q / K (conflict-free fragment loads)
constexpr int kTrVtStride = 40;  // fp16 row stride of the transposed V of one position

// fp16 image (elements): token projection, then per block Wqkv, Wo, W1, W2
constexpr int kImgTp = kTrH * kTrKin;                      // 2048
constexpr int kImgQkv = 3 * kTrH * kTrH, kImgO = kTrH * kTrH, kImgW1 = kTrFfn * kTrH, kImgW2 = kTrH * kTrFfn;
constexpr int kImgLayer = kImgQkv + kImgO + kImgW1 + kImgW2;  // 28672
constexpr uint32_t kImgLayerBytes = kImgLayer * 2;           // 57344

// fp32 parameters: global block, then per transformer block
constexpr int kParTpB = 0, kParCls = 64, kParFnG = 128, kParFnB = 192, kParLayer0 = 256;
constexpr int kLLn1G = 0, kLLn1B = 64, kLBqkv = 128, kLBo = 320, kLLn2G = 384, kLLn2B = 448, kLB1 = 512,
              kLB2 = 608, kLDq = 672, kLDr = 808, kLDz = 944, kLEnd = 984;
// relative-bias classes: (dq, dr, dz) clipped offsets, 17 x 17 x 5, then one
// entry for a masked key (fp16 lowest: its softmax weight is exactly 0)
constexpr int kRbClasses = 17 * 17 * 5, kRbStride = kRbClasses + 1;

struct __align__(16) TrunkSmem {
    __half w[kImgLayer];                           // this block's weights
    __half tp[kImgTp];                             // token projection weights
    __half a[kTrTiles][kTrFfn / 8][128][8];        // A operand per tile (K <= 96); queries during attention
    __half k[kTrRows * kTrQkStride];               // keys, row-major (bias added)
    __half vt[kTrPos][kTrH * kTrVtStride];         // values, transposed per position [dim][key]
    int32_t cq[kTrRows], cr[kTrRows], cz[kTrRows];  // token coordinates (CLS and padding 0)
    float par[kLEnd];                              // this block's fp32 parameters
    __half rb[kTrHeads * kRbStride];               // this block's relative bias per head and class
    float2 lnx[2][kTrRows];                        // LayerNorm statistics (mean, M2) of each row's halves
    uint64_t bar_w, bar_mma;
    uint32_t tmem;
    int err;
};
static_assert(sizeof(TrunkSmem) <= 232448, "trunk shared memory above the 227 KB opt-in limit");

// 8 values of this thread's row -> slab c of its tile's A operand (one 16-byte store)
__device__ __forceinline__ void put_chunk8(TrunkSmem* s, int c, int t, const float* x) {
    __half2 p0 = __floats2half2_rn(x[0], x[1]);
    __half2 p1 = __floats2half2_rn(x[2], x[3]);
    __half2 p2 = __floats2half2_rn(x[4], x[5]);
    __half2 p3 = __floats2half2_rn(x[6], x[7]);
    uint4 u;
    u.x = *reinterpret_cast<uint32_t*>(&p0);
    u.y = *reinterpret_cast<uint32_t*>(&p1);
    u.z = *reinterpret_cast<uint32_t*>(&p2);
    u.w = *reinterpret_cast<uint32_t*>(&p3);
    *reinterpret_cast<uint4*>(&s->a[t >> 7][c][t & 127][0]) = u;
}

// n values of this thread's row into its tile's A operand, slabs c0 .. c0 + n / 8 - 1
__device__ __forceinline__ void put_chunks(TrunkSmem* s, int c0, int t, const float* x, int n) {
#pragma unroll
    for (int c = 0; c < n / 8; c++) put_chunk8(s, c0 + c, t, x + 8 * c);
}

// packed fp32 pair arithmetic (sm_100 f32x2: one instruction for two lanes of work)
__device__ __forceinline__ uint64_t f2_bits(float2 a) { return *reinterpret_cast<uint64_t*>(&a); }
__device__ __forceinline__ float2 f2_val(uint64_t a) { return *reinterpret_cast<float2*>(&a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(r);
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(r);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_val(r);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_val(r);
}
__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 pair(const float* x, int i) { return make_float2(x[i], x[i + 1]); }
__device__ __forceinline__ void put2(float* x, int i, float2 v) {
    x[i] = v.x;
    x[i + 1] = v.y;
}

__device__ __forceinline__ void bar_pair(int id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }

// LayerNorm (eps 1e-5, biased variance) of a 64-wide row held as two 32-wide
// halves by two threads (same lane of warps w and w ^ 4).  Each half's mean
// and sum of squared deviations go through lnx; the pair meets at named
// barrier `bar` and combines them as m = (m0 + m1) / 2,
// M2 = M2_0 + M2_1 + 16 (m0 - m1)^2 (the pairwise update of Chan, Golub and
// LeVeque), so both halves compute identical statistics.  g, b: this half's
// gamma / beta (8-byte aligned); sums as four independent pair accumulators.
__device__ __forceinline__ void layer_norm_half(TrunkSmem* s, int row, int hf, int bar, const float* x,
                                                const float* g, const float* b, float* y) {
    float2 s2[4];
#pragma unroll
    for (int k = 0; k < 4; k++) s2[k] = pair(x, 2 * k);
#pragma unroll
    for (int i = 8; i < 32; i += 8)
#pragma unroll
        for (int k = 0; k < 4; k++) s2[k] = add2(s2[k], pair(x, i + 2 * k));
    const float2 sa = add2(add2(s2[0], s2[1]), add2(s2[2], s2[3]));
    const float mh = (sa.x + sa.y) * (1.0f / 32.0f);
    const float2 mh2 = make_float2(mh, mh);
    float2 v2[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 d = sub2(pair(x, 2 * k), mh2);
        v2[k] = mul2(d, d);
    }
#pragma unroll
    for (int i = 8; i < 32; i += 8)
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float2 d = sub2(pair(x, i + 2 * k), mh2);
            v2[k] = fma2(d, d, v2[k]);
        }
    const float2 va = add2(add2(v2[0], v2[1]), add2(v2[2], v2[3]));
    const float m2h = va.x + va.y;
    s->lnx[hf][row] = make_float2(mh, m2h);
    bar_pair(bar);
    const float2 o = s->lnx[hf ^ 1][row];
    const float m = 0.5f * (mh + o.x), dm = mh - o.x;
    const float r = rsqrtf((m2h + o.y + 16.0f * dm * dm) * (1.0f / 64.0f) + 1e-5f);
    const float2 m2 = make_float2(m, m), r2 = make_float2(r, r);
#pragma unroll
    for (int i = 0; i < 32; i += 2) put2(y, i, fma2(mul2(sub2(pair(x, i), m2), r2), ld2(g + i), ld2(b + i)));
}

// D[128 x n] = A[128 x k] * B[row0 .. row0 + n) of a B matrix with ntot rows,
// both in the slab layout of gemm_m128
__device__ __forceinline__ void gemm_m128_rows(uint32_t d_tmem, const void* a, const void* b, int ntot, int row0,
                                               int n, int k) {
    const uint32_t id = idesc_f16_m128(n);
    const char* pa = static_cast<const char*>(a);
    const char* pb = static_cast<const char*>(b) + row0 * 16;
    for (int st = 0; st < k / 16; st++)
        mma_f16(d_tmem, sdesc(pa + st * 2 * 128 * 16, 128 * 16, 128), sdesc(pb + st * 2 * ntot * 16, ntot * 16, 128),
                id, st > 0 ? 1u : 0u);
}

// one GEMM round: operands visible to the tensor core, issue, commit, wait
// (uniform result: false if any thread's wait gave up).  split: the n output
// columns go out as two halves of n / 2, at d_col and d_col + 64, so that
// each thread half reads 32-column-aligned TMEM blocks.
__device__ __forceinline__ bool trunk_gemm(TrunkSmem* s, uint32_t d_col, const void* b, int n, int k,
                                           uint32_t& mphase, bool split = false) {
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        tc_fence_after();
#pragma unroll
        for (int u = 0; u < kTrTiles; u++) {
            const uint32_t d = s->tmem + 256 * u + d_col;
            if (split) {
                gemm_m128_rows(d, &s->a[u][0][0][0], b, n, 0, n / 2, k);
                gemm_m128_rows(d + 64, &s->a[u][0][0][0], b, n, n / 2, n / 2, k);
            } else {
                gemm_m128(d, &s->a[u][0][0][0], b, n, k);
            }
        }
        mma_commit(&s->bar_mma);
    }
    const bool ok = mbar_wait(&s->bar_mma, mphase);
    mphase ^= 1u;
    tc_fence_after();
    return __syncthreads_and(ok) != 0;
}

// TMEM address of this thread's row: warp w reads lanes 32 (w % 4) of tile w / 8's columns
__device__ __forceinline__ uint32_t lane_taddr(const TrunkSmem* s, int col) {
    const int w = threadIdx.x >> 5;
    return s->tmem + ((uint32_t)((w & 3) * 32) << 16) + (uint32_t)(256 * (w >> 3) + col);
}

__device__ __forceinline__ void prefetch_block(TrunkSmem* s, const __half* img, int layer) {
    const __half* src = img + kImgTp + (size_t)layer * kImgLayer;
    mbar_expect_tx(&s->bar_w, kImgLayerBytes);
    // four copies, one per matrix (each a multiple of 16 bytes)
    bulk_g2s(&s->w[0], src, kImgQkv * 2, &s->bar_w);
    bulk_g2s(&s->w[kImgQkv], src + kImgQkv, kImgO * 2, &s->bar_w);
    bulk_g2s(&s->w[kImgQkv + kImgO], src + kImgQkv + kImgO, kImgW1 * 2, &s->bar_w);
    bulk_g2s(&s->w[kImgQkv + kImgO + kImgW1], src + kImgQkv + kImgO + kImgW1, kImgW2 * 2, &s->bar_w);
}

__device__ __forceinline__ uint32_t ld_b32(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

// D += A(16x8, row) * B(8x8, col), fp16 in, fp32 accumulate
__device__ __forceinline__ void mma_k8(float* d, uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}

// D += A(16x16, row) * B(16x8, col)
__device__ __forceinline__ void mma_k16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// This block's relative bias of every (dq, dr, dz) class and head: the
// three embedding rows summed in fp32 and rounded to fp16, as the reference
// adds bias.to(scores.dtype) to its fp16 autocast scores
// (fnn_transformer_net.py RelativeSelfAttention.forward); head h's table is
// rb[h * kRbStride ...], class index ((dq * 17) + dr) * 5 + dz.
__device__ __forceinline__ void build_rel_bias(TrunkSmem* s) {
    for (int c = threadIdx.x; c < kRbStride; c += kTrThreads) {
        float v[kTrHeads];
        if (c < kRbClasses) {
            const int dq = c / 85, rem = c - 85 * dq, dr = rem / 5, dz = rem - 5 * dr;
            const float4* q4 = reinterpret_cast<const float4*>(s->par + kLDq + 8 * dq);
            const float4* r4 = reinterpret_cast<const float4*>(s->par + kLDr + 8 * dr);
            const float4* z4 = reinterpret_cast<const float4*>(s->par + kLDz + 8 * dz);
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const float4 a = q4[k], b = r4[k], z = z4[k];
                v[4 * k + 0] = (a.x + b.x) + z.x;
                v[4 * k + 1] = (a.y + b.y) + z.y;
                v[4 * k + 2] = (a.z + b.z) + z.z;
                v[4 * k + 3] = (a.w + b.w) + z.w;
            }
        } else {
#pragma unroll
            for (int h = 0; h < kTrHeads; h++) v[h] = -65504.0f;
        }
#pragma unroll
        for (int h = 0; h < kTrHeads; h++) s->rb[h * kRbStride + c] = __float2half_rn(v[h]);
    }
}

__device__ __forceinline__ float lds_f16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Attention of one position (this warp's 32 rows, from per-row index base)
// for heads h0 .. h0 + 3: per head, S = Q K^T on
// fp16 warp MMAs with fp32 accumulation (head width 8 = one k8 step; fp16
// keeps the softmax weights to 11 significant bits), scale + relative bias + key mask,
// row softmax on the accumulator fragments (quad shuffles), O = P V with the
// score fragments reused as the A operand; O goes straight into the A
// operand slab of the output projection.  Fragment coordinates: g = lane/4
// selects rows g and g+8 of a 16-row tile, c = lane%4 selects columns 2c, 2c+1.
// MT 16-row query tiles and NT 8-key blocks are computed: the rows and keys
// past the last valid token are dead (masked as keys, and their residual is
// zeroed after each block), so their scores are not formed; their slab rows
// keep the (finite) queries.
template <int MT, int NT>
__device__ __forceinline__ void attention_heads(TrunkSmem* s, int base, int h0, int l, uint32_t kmask) {
    constexpr int KB = (NT + 1) / 2;
    const int g = l >> 2, c = l & 3, u = base >> 7, tb = base & 127;
    const float scale = 0.35355339059327373f;  // 8 ** -0.5
    const float kLog2e = 1.4426950408889634f;
    // shared-memory address of each of this thread's 32 (row, key) pairs'
    // bias class in head 0's table (a masked key: the masked entry)
    const uint32_t rb0 = static_cast<uint32_t>(__cvta_generic_to_shared(s->rb));
    uint32_t rel[MT][2][NT][2];
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int i = base + 16 * mt + g + 8 * hh;
            const int qi = s->cq[i], ri = s->cr[i], zi = s->cz[i];
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int j = base + 8 * nt + 2 * c + e;
                    const int dq = min(max(s->cq[j] - qi, -8), 8) + 8;
                    const int dr = min(max(s->cr[j] - ri, -8), 8) + 8;
                    const int dz = min(max(s->cz[j] - zi, -2), 2) + 2;
                    const int cls = ((kmask >> (8 * nt + 2 * c + e)) & 1u) ? (dq * 17 + dr) * 5 + dz : kRbClasses;
                    rel[mt][hh][nt][e] = rb0 + 2u * (uint32_t)cls;
                }
        }
#pragma unroll 1
    for (int h = h0; h < h0 + kTrHeads / 2; h++) {
        const uint32_t hoff = 2u * (uint32_t)(h * kRbStride);
        // this head's bias of the thread's pairs (issued before the MMAs)
        float bias[MT][2][NT][2];
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int e = 0; e < 2; e++) bias[mt][hh][nt][e] = lds_f16(rel[mt][hh][nt][e] + hoff);
        // S = Q_h K_h^T
        float sc[MT][NT][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            const __half* qa = &s->a[u][h][tb + 16 * mt + g][2 * c];
            const uint32_t a0 = ld_b32(qa), a1 = ld_b32(qa + 8 * 8);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const uint32_t b0 = ld_b32(s->k + (base + 8 * nt + g) * kTrQkStride + 8 * h + 2 * c);
                sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.0f;
                mma_k8(sc[mt][nt], a0, a1, b0);
            }
        }
        // scale + bias (a masked key's bias is fp16 lowest); row max / sum over the quad
        float rinv[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                float mx = -3.0e38f;
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const float2 v = fma2(pair(sc[mt][nt], 2 * hh), make_float2(scale, scale),
                                          make_float2(bias[mt][hh][nt][0], bias[mt][hh][nt][1]));
                    put2(sc[mt][nt], 2 * hh, v);
                    mx = fmaxf(mx, fmaxf(v.x, v.y));
                }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mxl = -mx * kLog2e;
                float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const float2 z = fma2(pair(sc[mt][nt], 2 * hh), make_float2(kLog2e, kLog2e), make_float2(mxl, mxl));
                    const float2 p = make_float2(ex2_approx(z.x), ex2_approx(z.y));
                    put2(sc[mt][nt], 2 * hh, p);
                    sum2 = add2(sum2, p);
                }
                float sum = sum2.x + sum2.y;
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                rinv[mt][hh] = sum > 0.0f ? 1.0f / sum : 0.0f;
            }
        // O = P V_h (the keys in k16 steps), normalised, into the A slab of head h
        const __half* vt = s->vt[base >> 5] + (8 * h + g) * kTrVtStride + 2 * c + (base & 31);
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kb = 0; kb < KB; kb++) {
                const uint32_t a0 = pack_f16(sc[mt][2 * kb][0], sc[mt][2 * kb][1]);
                const uint32_t a1 = pack_f16(sc[mt][2 * kb][2], sc[mt][2 * kb][3]);
                // (a key block past NT: zero weights)
                const uint32_t a2 = 2 * kb + 1 < NT ? pack_f16(sc[mt][(2 * kb + 1) % NT][0], sc[mt][(2 * kb + 1) % NT][1]) : 0u;
                const uint32_t a3 = 2 * kb + 1 < NT ? pack_f16(sc[mt][(2 * kb + 1) % NT][2], sc[mt][(2 * kb + 1) % NT][3]) : 0u;
                mma_k16(o, a0, a1, a2, a3, ld_b32(vt + 16 * kb), ld_b32(vt + 16 * kb + 8));
            }
            const int r0 = tb + 16 * mt + g;
            *reinterpret_cast<uint32_t*>(&s->a[u][h][r0][2 * c]) = pack_f16(o[0] * rinv[mt][0], o[1] * rinv[mt][0]);
            *reinterpret_cast<uint32_t*>(&s->a[u][h][r0 + 8][2 * c]) =
                pack_f16(o[2] * rinv[mt][1], o[3] * rinv[mt][1]);
        }
    }
}

// the position's attention: rows and keys up to the last valid one
__device__ __noinline__ void attention_warp(TrunkSmem* s, int base, int h0, int l, uint32_t kmask) {
    if (kmask < (1u << 16))
        attention_heads<1, 2>(s, base, h0, l, kmask);
    else if (kmask < (1u << 24))
        attention_heads<2, 3>(s, base, h0, l, kmask);
    else
        attention_heads<2, 4>(s, base, h0, l, kmask);
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// The exact (erf) GELU of two values, x * Phi(x) with Phi the standard normal
// CDF, from Abramowitz & Stegun's erfc approximation 7.1.26 (Hastings; absolute
// error of erf at most 1.5e-7): with z = |x| / sqrt(2) and t = 1 / (1 + p z),
// erfc(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), and
// Phi(x) = 1 - erfc(z) / 2 for x >= 0, erfc(z) / 2 otherwise.  Branch free;
// the result is rounded to fp16 for the next GEMM, far above these errors.
__device__ __forceinline__ float2 gelu2(float2 x) {
    const float2 t = make_float2(rcp_approx(fmaf(0.3275911f * 0.70710678118654752f, fabsf(x.x), 1.0f)),
                                 rcp_approx(fmaf(0.3275911f * 0.70710678118654752f, fabsf(x.y), 1.0f)));
    float2 p = fma2(make_float2(1.061405429f, 1.061405429f), t, make_float2(-1.453152027f, -1.453152027f));
    p = fma2(p, t, make_float2(1.421413741f, 1.421413741f));
    p = fma2(p, t, make_float2(-0.284496736f, -0.284496736f));
    p = fma2(p, t, make_float2(0.254829592f, 0.254829592f));
    p = mul2(p, mul2(t, make_float2(0.5f, 0.5f)));  // erfc(z) / 2 without the Gaussian factor
    // exp(-z^2) = 2^(-x^2 log2(e) / 2)
    const float2 a = mul2(mul2(x, x), make_float2(-0.72134752044448170f, -0.72134752044448170f));
    const float2 h = mul2(p, make_float2(ex2_approx(a.x), ex2_approx(a.y)));
    return make_float2(x.x * (x.x >= 0.0f ? 1.0f - h.x : h.x), x.y * (x.y >= 0.0f ? 1.0f - h.y : h.y));
}

// A slot is 32 rows of a tile: one position (CLS, 28 tokens, 3 padding
// rows), or, packed, two positions whose valid tokens all lie in their first
// 15 token slots (16 rows each: CLS and 15 tokens).  Packed, slot si is table
// entry si for si < nbig (one position: (p, -1)) and entry
// batch - npair + (si - nbig) after them (a pair (p, q), or (p, -1) for a
// lone one); unpacked, slot si is position si.
constexpr int kSlotTok = 30;  // staged token rows per slot (28, or 15 + 15)
struct SlotMap {
    const int2* table;  // NULL: unpacked
    int64_t nbig, npair, batch;
    __device__ __forceinline__ int64_t count() const { return table ? nbig + npair : batch; }
    __device__ __forceinline__ int2 at(int64_t si) const {
        if (!table) return make_int2((int)si, -1);
        return table[si < nbig ? si : batch - npair + (si - nbig)];
    }
};

// The token features of a pass's 8 slots (slot s0 ..) into shared memory,
// [8][30][27] floats, by asynchronous 4-byte copies (no alignment asked of
// the caller's array); slots past the table are left alone (not read).
__device__ __forceinline__ void stage_tokens(float* dst, const float* __restrict__ tf, const SlotMap& sm,
                                             int64_t s0) {
    constexpr int kPer = 28 * 27, kSlot = kSlotTok * 27;
    const int64_t nslots = sm.count();
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    for (int i = threadIdx.x; i < kTrPos * kSlot; i += kTrThreads) {
        const int k = i / kSlot, r = i - k * kSlot;
        if (s0 + k >= nslots) break;  // (k grows with i)
        const int2 sp = sm.at(s0 + k);
        int64_t src = -1;
        if (sp.y < 0) {
            if (r < kPer) src = (int64_t)sp.x * kPer + r;
        } else {
            const int h = r >= 15 * 27, rr = r - h * 15 * 27;
            src = (int64_t)(h ? sp.y : sp.x) * kPer + rr;
        }
        if (src >= 0)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d + 4u * (uint32_t)i), "l"(tf + src)
                         : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// The slot table, a thread per position: a position with no valid token
// past its first 15 is "small" and takes half of a pair entry (filled from
// the table's end), the others take single entries from its start; cnt =
// (singles, smalls) and the entries' second halves start at -1 (the host
// clears both).  The order of the entries depends on the atomics' order; a
// position's result does not depend on its slot (rows are independent in
// every GEMM and LayerNorm, and a position attends within its own rows).
__global__ void k_trunk_classify(const uint8_t* __restrict__ tm, int64_t batch, int2* __restrict__ table,
                                 int* __restrict__ cnt) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= batch) return;
    bool any = false;
#pragma unroll
    for (int k = 15; k < 28; k++) any |= tm[p * 28 + k] != 0;
    if (any) {
        table[atomicAdd(&cnt[0], 1)] = make_int2((int)p, -1);
    } else {
        const int k = atomicAdd(&cnt[1], 1);
        reinterpret_cast<int*>(table + (batch - 1 - k / 2))[k & 1] = (int)p;
    }
}

// token_features [B,28,27] (first `nfeat` used), token_q/r/z [B,28], token_mask [B,28] (0/1),
// img: fp16 weight image, par: fp32 parameters; out [B,64]: the normalised CLS row
__global__ void __launch_bounds__(kTrThreads, 1) k_hybrid_trunk(const float* __restrict__ tf, const int32_t* __restrict__ tq,
                                                         const int32_t* __restrict__ tr, const int32_t* __restrict__ tz,
                                                         const uint8_t* __restrict__ tm, int64_t batch, int nfeat,
                                                         const int2* __restrict__ slots,
                                                         const int* __restrict__ slot_cnt,
                                                         const __half* __restrict__ img,
                                                         const float* __restrict__ par, float* __restrict__ out,
                                                         uint32_t* err_word) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    TrunkSmem* s = reinterpret_cast<TrunkSmem*>(smem_raw);
    const int t = threadIdx.x, w = t >> 5, l = t & 31;
    // warp w = u * 8 + hf * 4 + q: tile u, half hf of every row, position q of the tile
    const int u = w >> 3, hf = (w >> 2) & 1, q = w & 3;
    const int base = 128 * u + 32 * q;  // per-row index of the position's row 0
    const int row = base + l;           // this thread's row (0 .. 255)
    const int lnbar = 1 + 4 * u + q;    // named barrier of the row pair's two warps
    const int hc = 32 * hf;             // first hidden column of this half
    // the slots (slots NULL: one position each); packed only when at least a
    // quarter of the batch is small (pairs then save an eighth of the slots)
    SlotMap sm{nullptr, 0, 0, batch};
    if (slots) {
        const int nsmall = slot_cnt[1];
        if (4 * (int64_t)nsmall >= batch) sm = SlotMap{slots, slot_cnt[0], (nsmall + 1) / 2, batch};
    }
    const int64_t nslots = sm.count();
    const int64_t npass = (nslots + kTrPos - 1) / kTrPos;  // 8 slots per pass

    if (t == 0) {
        mbar_init(&s->bar_w, 1);
        mbar_init(&s->bar_mma, 1);
        s->err = 0;
        fence_mbar_init();
    }
    if (w == 0) {
        tmem_alloc(&s->tmem, 512);
        tmem_relinquish();
    }
    {
        const uint4* src = reinterpret_cast<const uint4*>(img);
        uint4* dst = reinterpret_cast<uint4*>(s->tp);
        for (int i = t; i < kImgTp / 8; i += kTrThreads) dst[i] = __ldg(src + i);
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    uint32_t mphase = 0, wphase = 0;
    bool wpend = false;
    bool mpend = false;
    bool failed = false;
    if (t == 0 && blockIdx.x < npass) {
        prefetch_block(s, img, 0);
        wpend = true;
    }
    // token features of each pass staged in the key buffer (free outside the attention)
    float* stf = reinterpret_cast<float*>(s->k);
    static_assert(sizeof(TrunkSmem::k) >= kTrPos * kSlotTok * 27 * sizeof(float), "token staging");
    if (blockIdx.x < npass) stage_tokens(stf, tf, sm, (int64_t)blockIdx.x * kTrPos);

    for (int64_t pass = blockIdx.x; pass < npass && !failed; pass += gridDim.x) {
        const int64_t si = pass * kTrPos + (base >> 5);
        const int2 sp = si < nslots ? sm.at(si) : make_int2(-1, -1);
        const bool paired = sp.y >= 0;         // two 16-row positions in this slot
        const int half = paired ? l >> 4 : 0;  // which of them this row belongs to
        const int64_t b = half ? sp.y : sp.x;
        const bool live = b >= 0;
        // ---- inputs of this row: token features (rows 1..), CLS (row 0 of the position), padding
        const int tok = (paired ? (l & 15) : l) - 1;
        const bool cls = live && tok < 0;
        const bool is_tok = live && tok >= 0 && tok < (paired ? 15 : 28);
        const bool valid = cls || (is_tok && tm[b * 28 + tok] != 0);
        if (hf == 0) {
            s->cq[row] = is_tok ? tq[b * 28 + tok] : 0;
            s->cr[row] = is_tok ? tr[b * 28 + tok] : 0;
            s->cz[row] = is_tok ? tz[b * 28 + tok] : 0;
        }
        const uint32_t kmask = __ballot_sync(0xffffffffu, valid);
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // every thread's staged token features
        {
            // this half's 16 of the 32 (zero-padded) input columns
            float f[kTrKin / 2];
            const float* src = stf + ((base >> 5) * kSlotTok + half * 15 + tok) * 27;
#pragma unroll
            for (int i = 0; i < kTrKin / 2; i++) {
                const int j = kTrKin / 2 * hf + i;
                f[i] = (is_tok && j < nfeat) ? src[j] : 0.0f;
            }
            put_chunks(s, 2 * hf, row, f, kTrKin / 2);
        }
        float x[kTrH / 2];  // this half of the row's residual stream
        mpend = true;
        if (!trunk_gemm(s, 192, s->tp, kTrH, kTrKin, mphase)) {
            failed = true;
            break;
        }
        mpend = false;
        {
            float d[32];
            tmem_ld32(lane_taddr(s, 192 + hc), d);
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const int j = hc + i;
                // CLS row: the learned token; pieces: projection times mask; padding: 0
                x[i] = cls ? __ldg(par + kParCls + j) : ((is_tok && valid) ? d[i] + __ldg(par + kParTpB + j) : 0.0f);
            }
        }

        for (int layer = 0; layer < kTrLayers; layer++) {
            // this block's fp32 parameters and relative-bias table
            __syncthreads();
            for (int i = t; i < kLEnd; i += kTrThreads) s->par[i] = __ldg(par + kParLayer0 + layer * kLEnd + i);
            __syncthreads();
            build_rel_bias(s);  // read by attention_warp, after the QKV GEMM's barriers
            // ---- attention
            float y[kTrH / 2];
            layer_norm_half(s, row, hf, lnbar, x, s->par + kLLn1G + hc, s->par + kLLn1B + hc, y);
            put_chunks(s, 4 * hf, row, y, kTrH / 2);
            bool okw = true;
            if (t == 0) {
                okw = mbar_wait(&s->bar_w, wphase);
                if (okw) {
                    wphase ^= 1u;  // on failure the parity stays: the exit path waits for this copy
                    wpend = false;
                }
            }
            if (!__syncthreads_and(okw)) {
                failed = true;
                break;
            }
            const __half* W = s->w;
            mpend = true;
            if (!trunk_gemm(s, 0, W, 3 * kTrH, kTrH, mphase)) {
                failed = true;
                break;
            }
            mpend = false;
            {
                // this half's heads 4 hf .. 4 hf + 3: queries into their A slabs,
                // keys row-major, values transposed per position; fp16, biases added
                float d[32];
                tmem_ld32(lane_taddr(s, hc), d);
#pragma unroll
                for (int i = 0; i < 32; i += 2) put2(d, i, add2(pair(d, i), ld2(s->par + kLBqkv + hc + i)));
                put_chunks(s, 4 * hf, row, d, 32);
                tmem_ld32(lane_taddr(s, 64 + hc), d);
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float2 v = add2(pair(d, i), ld2(s->par + kLBqkv + 64 + hc + i));
                    *reinterpret_cast<__half2*>(s->k + row * kTrQkStride + hc + i) = __floats2half2_rn(v.x, v.y);
                }
                tmem_ld32(lane_taddr(s, 128 + hc), d);
                __half* vt = s->vt[base >> 5] + hc * kTrVtStride + l;
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float2 v = add2(pair(d, i), ld2(s->par + kLBqkv + 128 + hc + i));
                    vt[i * kTrVtStride] = __float2half_rn(v.x);
                    vt[(i + 1) * kTrVtStride] = __float2half_rn(v.y);
                }
            }
            // the residual waits in TMEM (columns hc .. hc + 31 of the row's lane,
            // free until the next block's QKV GEMM) while the attention runs
            tmem_st32(lane_taddr(s, hc), x);
            __syncwarp();
            if (paired) {  // each position of the slot attends within its own 16 rows
                attention_warp(s, base, 4 * hf, l, kmask & 0xffffu);
                attention_warp(s, base + 16, 4 * hf, l, kmask >> 16);
            } else {
                attention_warp(s, base, 4 * hf, l, kmask);
            }
            mpend = true;
            if (!trunk_gemm(s, 192, W + kImgQkv, kTrH, kTrH, mphase)) {
                failed = true;
                break;
            }
            mpend = false;
            // every warp's attention is done with the key buffer: stage the
            // token features of this CTA's next pass there
            if (layer == kTrLayers - 1 && pass + gridDim.x < npass)
                stage_tokens(stf, tf, sm, (pass + gridDim.x) * kTrPos);
            {
                float d[32];
                tmem_ld32(lane_taddr(s, hc), x);
                tmem_ld32(lane_taddr(s, 192 + hc), d);
#pragma unroll
                for (int i = 0; i < 32; i += 2)
                    put2(x, i, add2(pair(x, i), add2(pair(d, i), ld2(s->par + kLBo + hc + i))));
            }
            // ---- MLP
            layer_norm_half(s, row, hf, lnbar, x, s->par + kLLn2G + hc, s->par + kLLn2B + hc, y);
            put_chunks(s, 4 * hf, row, y, kTrH / 2);
            mpend = true;
            // output columns 0..47 and 64..111: this half's 48 at 64 hf
            if (!trunk_gemm(s, 0, W + kImgQkv + kImgO, kTrFfn, kTrH, mphase, true)) {
                failed = true;
                break;
            }
            mpend = false;
            {
                float d[32];
                tmem_ld32(lane_taddr(s, 64 * hf), d);
#pragma unroll
                for (int i = 0; i < 32; i += 2) put2(d, i, gelu2(add2(pair(d, i), ld2(s->par + kLB1 + 48 * hf + i))));
                put_chunks(s, 6 * hf, row, d, 32);
                tmem_ld16(lane_taddr(s, 64 * hf + 32), d);
#pragma unroll
                for (int i = 0; i < 16; i += 2)
                    put2(d, i, gelu2(add2(pair(d, i), ld2(s->par + kLB1 + 48 * hf + 32 + i))));
                put_chunks(s, 6 * hf + 4, row, d, 16);
            }
            mpend = true;
            if (!trunk_gemm(s, 192, W + kImgQkv + kImgO + kImgW1, kTrH, kTrFfn, mphase)) {
                failed = true;
                break;
            }
            mpend = false;
            // every MMA reading this block's weights has completed: fetch the
            // next block (next layer, or layer 0 of this CTA's next pass)
            if (t == 0 && (layer + 1 < kTrLayers || pass + gridDim.x < npass)) {
                prefetch_block(s, img, (layer + 1) % kTrLayers);
                wpend = true;
            }
            {
                float d[32];
                const float keep = valid ? 1.0f : 0.0f;
                tmem_ld32(lane_taddr(s, 192 + hc), d);
#pragma unroll
                for (int i = 0; i < 32; i += 2)
                    put2(x, i, mul2(add2(add2(pair(x, i), pair(d, i)), ld2(s->par + kLB2 + hc + i)),
                                    make_float2(keep, keep)));
            }
        }
        if (failed) break;
        // the final LayerNorm of every row pair (the pair's barrier needs
        // both warps); the CLS row of a live position is the output
        {
            float y[kTrH / 2];
            layer_norm_half(s, row, hf, lnbar, x, par + kParFnG + hc, par + kParFnB + hc, y);
            if (cls) {
                float4* o4 = reinterpret_cast<float4*>(out + b * kTrH + hc);
#pragma unroll
                for (int i = 0; i < 8; i++) o4[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
            }
        }
    }

    if (failed) {
        // a bounded wait gave up: record it, let this CTA's own copies and
        // MMAs in flight finish (bounded again), free TMEM and return
        if (t == 0) {
            atomicOr(err_word, 4u);
            if (wpend) mbar_drain(&s->bar_w, wphase);
        }
        if (mpend) mbar_drain(&s->bar_mma, mphase ^ 1u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // no staged copy outlives the CTA
    tc_fence_before();
    __syncthreads();
    if (w == 0) {
        tc_fence_after();
        tmem_dealloc(s->tmem, 512);
    }
}

}  // namespace hv
