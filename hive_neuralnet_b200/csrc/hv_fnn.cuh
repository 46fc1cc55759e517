// hv_fnn.cuh -- the FNN leaf evaluator fused with successor generation.
//
// Network (reference hive_fnn/fnn_network.py:47-143, HiveFNN):
//   encode(x)        = fc2(LayerNorm(sigmoid(fc1 x)))          x: 122 floats
//   value(e)         = tanh(value_fc e)
//   score(e_r, e_s)  = action_fc2(sigmoid(action_fc1 [e_r ; e_s]))
// and the leaf evaluation of hive_fnn/fnn_mcts_orchestrator.py:243-316:
//   priors  = softmax over the legal slots of score(e_root, e_succ_i)
//   value   = value(e_root)
//   child_q = -value(e_succ_i)
// computed in fp32 on CUDA cores.  One warp owns one leaf: it builds each
// successor (apply + compact list + features, exactly as
// fnn_successor_features_batch does) into shared memory, CH successors at a
// time, and runs the MLP on the chunk with each lane owning output neurons
// lane and lane+32, so every weight read (transposed, coalesced, L1-resident)
// is reused CH times.
#pragma once

#include "hv_core.cuh"
#include "hv_movegen.cuh"
#include "hv_state.cuh"

namespace hv {

constexpr int kFnnChunk = 4;   // successors per MLP pass
constexpr int kFnnMaxDim = 64; // hidden / embed / action-hidden upper bound

// Packed fp32 weights, transposed so that lane o reads W[k][o] (coalesced):
//   W1T [F][H]  b1 [H]  g1 [H]  be1 [H]
//   W2T [H][E]  b2 [E]
//   wv  [E]     bv [1]
//   A1T [2E][A] a1b [A]
//   a2  [A]     a2b [1]
struct FnnDims {
    int H, E, A;
};

struct FnnOffsets {
    int w1t, b1, g1, be1, w2t, b2, wv, bv, a1t, a1b, a2, a2b, total;
};

__host__ __device__ inline FnnOffsets fnn_offsets(FnnDims d) {
    FnnOffsets o;
    int p = 0;
    o.w1t = p; p += kFeat * d.H;
    o.b1 = p; p += d.H;
    o.g1 = p; p += d.H;
    o.be1 = p; p += d.H;
    o.w2t = p; p += d.H * d.E;
    o.b2 = p; p += d.E;
    o.wv = p; p += d.E;
    o.bv = p; p += 1;
    o.a1t = p; p += 2 * d.E * d.A;
    o.a1b = p; p += d.A;
    o.a2 = p; p += d.A;
    o.a2b = p; p += 1;
    o.total = p;
    return o;
}

struct FnnSmem {
    float xs[kFnnChunk][kFeat];        // successor (or root) features
    float ys[kFnnChunk][kFnnMaxDim];   // post-LayerNorm hidden / embedding
    float logit[kMaxMoves];
    float root_pre[kFnnMaxDim];        // action_fc1 bias + root half
    float root_emb[kFnnMaxDim];
};

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// Encode ns (<= kFnnChunk) feature rows xs[0..ns) -> embeddings in ys, and
// return per-row value in val[] (all lanes), emb kept in ys[s][0..E).
__device__ __noinline__ void fnn_encode_chunk(const float* __restrict__ w, FnnDims d, FnnOffsets o,
                                              FnnSmem* f, int ns, float* val) {
    const int l = lane_id();
    const int o0 = l, o1 = l + 32;
    float h[kFnnChunk][2];
#pragma unroll
    for (int s = 0; s < kFnnChunk; s++) {
        h[s][0] = o0 < d.H ? __ldg(w + o.b1 + o0) : 0.0f;
        h[s][1] = o1 < d.H ? __ldg(w + o.b1 + o1) : 0.0f;
    }
#pragma unroll 2
    for (int k = 0; k < kFeat; k++) {
        float w0 = o0 < d.H ? __ldg(w + o.w1t + k * d.H + o0) : 0.0f;
        float w1 = o1 < d.H ? __ldg(w + o.w1t + k * d.H + o1) : 0.0f;
#pragma unroll
        for (int s = 0; s < kFnnChunk; s++) {
            float x = f->xs[s][k];
            h[s][0] = fmaf(w0, x, h[s][0]);
            h[s][1] = fmaf(w1, x, h[s][1]);
        }
    }
    const float invH = 1.0f / (float)d.H;
    const float g0 = o0 < d.H ? __ldg(w + o.g1 + o0) : 0.0f, g1v = o1 < d.H ? __ldg(w + o.g1 + o1) : 0.0f;
    const float c0 = o0 < d.H ? __ldg(w + o.be1 + o0) : 0.0f, c1 = o1 < d.H ? __ldg(w + o.be1 + o1) : 0.0f;
#pragma unroll
    for (int s = 0; s < kFnnChunk; s++) {
        float a = o0 < d.H ? sigmoidf_(h[s][0]) : 0.0f;
        float b = o1 < d.H ? sigmoidf_(h[s][1]) : 0.0f;
        float mean = warp_sum(a + b) * invH;
        float da = o0 < d.H ? a - mean : 0.0f, db = o1 < d.H ? b - mean : 0.0f;
        float var = warp_sum(da * da + db * db) * invH;
        float rstd = 1.0f / sqrtf(var + 1e-5f);
        if (o0 < d.H) f->ys[s][o0] = da * rstd * g0 + c0;
        if (o1 < d.H) f->ys[s][o1] = db * rstd * g1v + c1;
    }
    __syncwarp();
    float e[kFnnChunk][2];
#pragma unroll
    for (int s = 0; s < kFnnChunk; s++) {
        e[s][0] = o0 < d.E ? __ldg(w + o.b2 + o0) : 0.0f;
        e[s][1] = o1 < d.E ? __ldg(w + o.b2 + o1) : 0.0f;
    }
#pragma unroll 2
    for (int k = 0; k < d.H; k++) {
        float w0 = o0 < d.E ? __ldg(w + o.w2t + k * d.E + o0) : 0.0f;
        float w1 = o1 < d.E ? __ldg(w + o.w2t + k * d.E + o1) : 0.0f;
#pragma unroll
        for (int s = 0; s < kFnnChunk; s++) {
            float y = f->ys[s][k];
            e[s][0] = fmaf(w0, y, e[s][0]);
            e[s][1] = fmaf(w1, y, e[s][1]);
        }
    }
    __syncwarp();
    const float v0 = o0 < d.E ? __ldg(w + o.wv + o0) : 0.0f, v1 = o1 < d.E ? __ldg(w + o.wv + o1) : 0.0f;
    const float bv = __ldg(w + o.bv);
#pragma unroll
    for (int s = 0; s < kFnnChunk; s++) {
        if (o0 < d.E) f->ys[s][o0] = e[s][0];
        if (o1 < d.E) f->ys[s][o1] = e[s][1];
        float z = warp_sum(v0 * e[s][0] + v1 * e[s][1]) + bv;
        val[s] = s < ns ? tanhf(z) : 0.0f;
    }
    __syncwarp();
}

// Root half of action_fc1 (+ its bias) from the root embedding in ys[0].
__device__ __forceinline__ void fnn_root_pre(const float* __restrict__ w, FnnDims d, FnnOffsets o,
                                             FnnSmem* f) {
    const int l = lane_id();
    const int o0 = l, o1 = l + 32;
    float a = o0 < d.A ? __ldg(w + o.a1b + o0) : 0.0f, b = o1 < d.A ? __ldg(w + o.a1b + o1) : 0.0f;
    for (int k = 0; k < d.E; k++) {
        float e = f->ys[0][k];
        if (o0 < d.A) a = fmaf(__ldg(w + o.a1t + k * d.A + o0), e, a);
        if (o1 < d.A) b = fmaf(__ldg(w + o.a1t + k * d.A + o1), e, b);
    }
    if (o0 < d.A) f->root_pre[o0] = a;
    if (o1 < d.A) f->root_pre[o1] = b;
    __syncwarp();
}

// logits of ns successor embeddings ys[0..ns) against the root
__device__ __noinline__ void fnn_score_chunk(const float* __restrict__ w, FnnDims d, FnnOffsets o,
                                             FnnSmem* f, int ns, float* logit) {
    const int l = lane_id();
    const int o0 = l, o1 = l + 32;
    float z[kFnnChunk][2];
    const float r0 = o0 < d.A ? f->root_pre[o0] : 0.0f, r1 = o1 < d.A ? f->root_pre[o1] : 0.0f;
#pragma unroll
    for (int s = 0; s < kFnnChunk; s++) {
        z[s][0] = r0;
        z[s][1] = r1;
    }
#pragma unroll 2
    for (int k = 0; k < d.E; k++) {
        float w0 = o0 < d.A ? __ldg(w + o.a1t + (d.E + k) * d.A + o0) : 0.0f;
        float w1 = o1 < d.A ? __ldg(w + o.a1t + (d.E + k) * d.A + o1) : 0.0f;
#pragma unroll
        for (int s = 0; s < kFnnChunk; s++) {
            float e = f->ys[s][k];
            z[s][0] = fmaf(w0, e, z[s][0]);
            z[s][1] = fmaf(w1, e, z[s][1]);
        }
    }
    const float u0 = o0 < d.A ? __ldg(w + o.a2 + o0) : 0.0f, u1 = o1 < d.A ? __ldg(w + o.a2 + o1) : 0.0f;
    const float b2 = __ldg(w + o.a2b);
#pragma unroll
    for (int s = 0; s < kFnnChunk; s++) {
        float t = (o0 < d.A ? u0 * sigmoidf_(z[s][0]) : 0.0f) + (o1 < d.A ? u1 * sigmoidf_(z[s][1]) : 0.0f);
        float lg = warp_sum(t) + b2;
        logit[s] = s < ns ? lg : 0.0f;
    }
}

}  // namespace hv
