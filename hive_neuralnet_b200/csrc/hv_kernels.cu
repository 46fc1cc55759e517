// hv_kernels.cu -- sm_100a kernels of the Hive self-play hot path and the
// C-ABI entry points declared in include/hive_b200.h.
//
// Every kernel is a persistent grid of warps (one warp per position, a
// grid of SMs x resident blocks) that strides over the batch.  Inputs are
// staged into the warp's shared-memory slot with 16-byte vector loads; the
// move list is assembled in shared memory and written back as 16-byte
// vector stores including its zero padding, so the [B, 256, 6] output needs
// no separate memset pass.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "hv_core.cuh"
#include "hv_movegen.cuh"
#include "hv_state.cuh"
#include "hv_fnn.cuh"
#include "hv_mcts.cuh"
#include "hv_tactics.cuh"
#include "hv_hybrid.cuh"
#include "hv_trunk.cuh"
#include "hv_mlp.cuh"
#include "hv_mlp_tc.cuh"
#include "hv_mlp32.cuh"
#include "hv_fnn_tc.cuh"
#include "../../include/hive_b200.h"

namespace hv {

#ifndef HV_WARPS_PER_BLOCK
#define HV_WARPS_PER_BLOCK 4  // warps (positions in flight) per block of the warp-per-unit kernels
#endif
#ifndef HV_MIN_BLOCKS
#define HV_MIN_BLOCKS 7  // resident blocks per SM the register budget is sized for
#endif
constexpr int kWarpsPerBlock = HV_WARPS_PER_BLOCK;
constexpr int kThreads = kWarpsPerBlock * 32;

// device error word (sticky until read and cleared by hv_get_error)
__device__ uint32_t g_error;

__device__ __forceinline__ WarpSmem* warp_slot() {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    return reinterpret_cast<WarpSmem*>(smem_raw) + (threadIdx.x >> 5);
}

// a slot of kFeatSlotBytes: only the fields before WarpSmem::sl exist
__device__ __forceinline__ WarpSmem* feat_warp_slot() {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    return reinterpret_cast<WarpSmem*>(smem_raw + (threadIdx.x >> 5) * kFeatSlotBytes);
}

// N16 16-byte words from global into shared memory by asynchronous copies:
// all of a lane's copies are in flight together (a load/store loop waits one
// memory latency per iteration).  Both addresses 16-byte aligned; the data
// is there after stage_wait().
template <int N16>
__device__ __forceinline__ void stage_async(void* smem_dst, const void* src) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const char* g = static_cast<const char*>(src);
#pragma unroll
    for (int k = 0; k < (N16 + 31) / 32; k++) {
        const int i = lane_id() + 32 * k;
        if (i < N16)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d + 16 * i), "l"(g + 16 * i) : "memory");
    }
}

__device__ __forceinline__ void stage_wait() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
}

constexpr int kState16 = kStateBytes / 16, kMoves16 = kMaxMoves * kMoveBytes / 16;

__device__ __forceinline__ void stage_state(WarpSmem* w, const uint8_t* src) {
    stage_async<kState16>(w->st, src);
    stage_wait();
}

// state and stored move list of one position
__device__ __forceinline__ void stage_state_moves(WarpSmem* w, const uint8_t* st, const uint8_t* mv) {
    stage_async<kState16>(w->st, st);
    stage_async<kMoves16>(w->mv, mv);
    stage_wait();
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

// The first n moves of the shared list out to a zero-padded global row; the
// shared list past n is never read (no zeroing pass over it).
__device__ __forceinline__ void store_moves(const WarpSmem* w, uint8_t* dst, int n) {
    const uint4* m4 = reinterpret_cast<const uint4*>(w->mv);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    const int bytes = n * kMoveBytes;
    for (int i = lane_id(); i < kMoves16; i += 32) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        const int valid = bytes - 16 * i;
        if (valid > 0) {
            v = m4[i];
            if (valid < 16) {
                uint32_t* u = &v.x;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int keep = valid - 4 * j;  // bytes of word j inside the list
                    u[j] = keep >= 4 ? u[j] : (keep <= 0 ? 0u : (u[j] & ((1u << (8 * keep)) - 1u)));
                }
            }
        }
        d4[i] = v;
    }
}

// ---------------------------------------------------------------------------
// root positions: legal moves (+ features), or features of a given list
// (game_logic.cu:63-91 generate_legal_moves[_and_fnn_features]_kernel,
//  fnn_features.cuh:334-350 extract_fnn_features_kernel)
// ---------------------------------------------------------------------------
// AP_LINK (the launches of hv_generate_legal_moves_and_fnn_features): the
// generator leaves each position's articulation mask in the first word of
// its feature row, and the feature launch takes it from there before it
// writes the row, instead of computing the articulation points again.
// DYNF: a feature launch of that entry that claims positions 1.. from a
// counter in bytes 16..23 of feature row 0; position 0 (whose row holds the
// counters) is left to a one-warp launch that follows.
template <bool GEN, bool WRITE_MOVES, bool FEATS, bool AP_LINK = false, bool DYNF = false>
__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_root(const uint8_t* __restrict__ states,
                                                   const uint8_t* __restrict__ moves_in,
                                                   const int32_t* __restrict__ nl_in, int64_t batch,
                                                   uint8_t* __restrict__ moves_out,
                                                   int32_t* __restrict__ nl_out,
                                                   float* __restrict__ feats_out) {
    // the feature launch of the fused entry touches only the slot's prefix
    WarpSmem* w = (!GEN && AP_LINK) ? feat_warp_slot() : warp_slot();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    // DYN (the generator launch of the fused entry): warps take positions
    // from a counter in the second 8 bytes of feature row 0 (zeroed by the
    // host before the launch; the generator writes only word 0 of a row), so
    // a warp that drew cheap positions takes more: position costs vary
    // widely (opening to late game) and a static stride left the slowest
    // warps running alone at the end.
    constexpr bool DYN = (GEN && AP_LINK) || DYNF;
    unsigned long long* ctr = DYN ? reinterpret_cast<unsigned long long*>(feats_out + (GEN ? 2 : 4)) : nullptr;
    auto claim = [&]() -> int64_t {
        unsigned long long v = 0;
        if (lane_id() == 0) v = atomicAdd(ctr, 1ull);
        return (int64_t)__shfl_sync(kFull, v, 0) + (DYNF ? 1 : 0);
    };
    int64_t p = DYN ? claim() : (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    while (p < batch) {
        if (GEN)
            stage_state(w, states + p * kStateBytes);
        else
            stage_state_moves(w, states + p * kStateBytes, moves_in + p * (kMaxMoves * kMoveBytes));
        // the warp's next position, claimed now, into L2 while this one is
        // computed (the feature launch waits on these loads otherwise)
        const int64_t q = DYN ? claim() : p + nwarps;
        {
            const int l = lane_id();
            if (q < batch) {
                if (l < kStateBytes / 128 + 1)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(states + q * kStateBytes + 128 * l));
                if (!GEN && l < kMaxMoves * kMoveBytes / 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(moves_in + q * (kMaxMoves * kMoveBytes) + 128 * l));
            }
        }
        int n;
        if (GEN) {
            Setup S = setup_position(w);
            if (AP_LINK) {
                const uint32_t apm = __ballot_sync(kFull, S.my_ap);
                if (lane_id() == 0) reinterpret_cast<uint32_t*>(feats_out)[p * kFeat] = apm;
            }
            n = gen_legal(w, S, &g_error);
            if (WRITE_MOVES) {
                store_moves(w, moves_out + p * (kMaxMoves * kMoveBytes), n);
                if (lane_id() == 0) nl_out[p] = n;
            }
            if (FEATS) features_full(w, n, feats_out + p * kFeat);
        } else {
            n = nl_in[p];
            n = n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n);
            // no moves generated here
            if (AP_LINK)
                setup_position<false, true, true>(w, reinterpret_cast<const uint32_t*>(feats_out)[p * kFeat]);
            else
                setup_position<false, true>(w);
            features_full(w, n, feats_out + p * kFeat);
        }
        __syncwarp();
        p = q;
    }
}

// ---------------------------------------------------------------------------
// successor features: apply one root move, compact list, features
// (game_logic.cu:182-229 fnn_successor_features_kernel)
// ---------------------------------------------------------------------------
// OUT selects the row format: kRowsF32 = fp32 [rows][122]; kSlabF16 = fp16
// in the K-major slab layout of 128-row tiles that the hybrid's tensor-core
// row network copies straight into its A operand (row r: tile r / 128, chunk
// c of 8 features at ((tile * 16 + c) * 128 + r % 128) * 8 halves, features
// 122..127 zero); kSlabF32 = fp32 tiles of kF32Rows (64) rows in 4-feature
// chunks (chunk c of row r at ((tile * 32 + c) * 64 + r % 64) * 4 floats,
// features 122..127 zero) for the FNN row network.
// kSlabF16x2 = 128-row tiles of the features split into fp16 high and low
// parts (x = hi + lo to ~2^-22) for the FNN's tensor-core row network: tile t
// holds the hi slab [16 chunks][128 rows][8] then the lo slab, 64 KB.
enum : int { kRowsF32 = 0, kSlabF16 = 1, kSlabF32 = 2, kSlabF16x2 = 3 };

// row a's chunk c (8 halves) of a kSlabF16x2 tile buffer: hi part; the lo part follows 16 x 128 x 8 halves later
__device__ __forceinline__ int64_t f16x2_at(int64_t a, int c) {
    return (a >> 7) * (2 * 16 * 128 * 8) + ((int64_t)c * 128 + (a & 127)) * 8;
}
template <int OUT>
__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_successor_features(
    const uint8_t* __restrict__ states, int64_t num_states, const uint8_t* __restrict__ legal_moves,
    const int64_t* __restrict__ action_to_root, const int64_t* __restrict__ move_indices,
    int64_t num_actions, void* __restrict__ out, const int64_t* __restrict__ n_actual,
    unsigned long long* __restrict__ ctr) {
    float* feats_out = static_cast<float*>(out);
    __half* slab = static_cast<__half*>(out);
    constexpr bool SLAB = OUT != kRowsF32;
    WarpSmem* w = warp_slot();
    if (n_actual) num_actions = min(num_actions, *n_actual);  // row pipeline: rows actually filled
    // The block's warps take consecutive rows and cross one block barrier
    // between the compact list and the features: the warps of an SM then run
    // fewer distinct code regions at a time, and this kernel is bound by
    // instruction fetch (measured: 25 % faster than free-running warps).
    // With a counter (ctr, zeroed before the launch), blocks claim their next
    // rows from it instead of a static stride, so a block that drew cheap rows
    // takes more; the claim for the next round is made before the barrier and
    // read after it (two slots: a slot is rewritten only two barriers later).
    __shared__ int64_t next_base[2];
    if (ctr) {
        if (threadIdx.x == 0) next_base[1] = (int64_t)atomicAdd(ctr, (unsigned long long)kWarpsPerBlock);
        __syncthreads();
    }
    int round = 0;
    for (int64_t base = ctr ? next_base[1] : (int64_t)blockIdx.x * kWarpsPerBlock; base < num_actions; round ^= 1) {
        const int64_t a = base + (threadIdx.x >> 5);
        bool ok = a < num_actions;
        int64_t root = 0, mi = 0;
        if (ok) {
            root = action_to_root[a];
            mi = move_indices[a];
            if (root < 0 || root >= num_states || mi < 0 || mi >= kMaxMoves) {
                // out-of-range request: zero row, flag it, touch nothing else
                if (OUT == kSlabF16) {
                    if (lane_id() < 16)
                        *reinterpret_cast<uint4*>(slab + (((a >> 7) * 16 + lane_id()) * 128 + (a & 127)) * 8) =
                            make_uint4(0, 0, 0, 0);
                } else if (OUT == kSlabF16x2) {
                    if (lane_id() < 16) {
                        __half* q = slab + f16x2_at(a, lane_id());
                        *reinterpret_cast<uint4*>(q) = make_uint4(0, 0, 0, 0);
                        *reinterpret_cast<uint4*>(q + 16 * 128 * 8) = make_uint4(0, 0, 0, 0);
                    }
                } else if (OUT == kSlabF32) {
                    *reinterpret_cast<float4*>(feats_out + (((a / kF32Rows) * 32 + lane_id()) * kF32Rows +
                                                            a % kF32Rows) * 4) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                } else {
                    for (int k = lane_id(); k < kFeat; k += 32) feats_out[a * kFeat + k] = 0.0f;
                }
                if (lane_id() == 0) atomicOr(&g_error, kErrIndex);
                ok = false;
            }
        }
        Setup S;
        int n = 0;
        if (ok) {
            stage_async<kState16>(w->st, states + root * kStateBytes);
            // the move's three 16-bit words load while the state copies are in flight
            const uint16_t* m = reinterpret_cast<const uint16_t*>(legal_moves + (root * kMaxMoves + mi) * kMoveBytes);
            const uint32_t m0 = __ldg(m), m1 = __ldg(m + 1), m2 = __ldg(m + 2);
            stage_wait();
            st_apply_warp(w->st, m0 & 255, m0 >> 8, m1, m2);
            S = setup_position(w);
            n = gen_compact_body(w, &g_error);
        }
        if (ctr && threadIdx.x == 0) next_base[round] = (int64_t)atomicAdd(ctr, (unsigned long long)kWarpsPerBlock);
        __syncthreads();
        const int64_t nb = ctr ? next_base[round] : base + (int64_t)gridDim.x * kWarpsPerBlock;
        if (ok) {
            if (SLAB) {
                // the move list is consumed once the features are written: stage them there
                float* f = reinterpret_cast<float*>(w->mv);
                features_body(w, n, f);
                __syncwarp();
                const int c = lane_id();
                if (OUT == kSlabF16x2) {
                    if (c < 16) {
                        __align__(16) __half hi[8], lo[8];
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const float x = 8 * c + i < kFeat ? f[8 * c + i] : 0.0f;
                            hi[i] = __float2half_rn(x);
                            lo[i] = __float2half_rn(x - __half2float(hi[i]));
                        }
                        __half* q = slab + f16x2_at(a, c);
                        *reinterpret_cast<uint4*>(q) = *reinterpret_cast<const uint4*>(hi);
                        *reinterpret_cast<uint4*>(q + 16 * 128 * 8) = *reinterpret_cast<const uint4*>(lo);
                    }
                } else if (OUT == kSlabF32) {
                    float v[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) v[i] = 4 * c + i < kFeat ? f[4 * c + i] : 0.0f;
                    *reinterpret_cast<float4*>(feats_out + (((a / kF32Rows) * 32 + c) * kF32Rows + a % kF32Rows) * 4) =
                        make_float4(v[0], v[1], v[2], v[3]);
                } else if (c < 16) {
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = 8 * c + i < kFeat ? f[8 * c + i] : 0.0f;
                    uint4 u;
                    u.x = pack_half2(v[0], v[1]);
                    u.y = pack_half2(v[2], v[3]);
                    u.z = pack_half2(v[4], v[5]);
                    u.w = pack_half2(v[6], v[7]);
                    *reinterpret_cast<uint4*>(slab + (((a >> 7) * 16 + c) * 128 + (a & 127)) * 8) = u;
                }
            } else {
                features_body(w, n, feats_out + a * kFeat);
            }
        }
        __syncwarp();
        base = nb;
    }
}

// ---------------------------------------------------------------------------
// fused leaf evaluation: successors + FNN + softmax
// (fnn_mcts_orchestrator.py:243-316 _eval_states with fnn_network.py encode /
//  value_head / score_actions)
// ---------------------------------------------------------------------------
__device__ __forceinline__ FnnSmem* fnn_slot() {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    return reinterpret_cast<FnnSmem*>(smem_raw + sizeof(WarpSmem) * kWarpsPerBlock) +
           (threadIdx.x >> 5);
}

__global__ void __launch_bounds__(kThreads, 2) k_fnn_eval(
    const uint8_t* __restrict__ states, const uint8_t* __restrict__ legal_moves,
    const int32_t* __restrict__ num_legal, const float* __restrict__ root_feats, int64_t count,
    const float* __restrict__ wts, FnnDims dims, float* __restrict__ priors,
    float* __restrict__ values, float* __restrict__ child_q, float* __restrict__ logits_out) {
    WarpSmem* w = warp_slot();
    FnnSmem* f = fnn_slot();
    const FnnOffsets off = fnn_offsets(dims);
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < count;
         p += nwarps) {
        int n = num_legal[p];
        n = n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n);
        const uint8_t* st_g = states + p * kStateBytes;
        const uint8_t* mv_g = legal_moves + p * (kMaxMoves * kMoveBytes);
        if (root_feats) {
            for (int k = l; k < kFeat; k += 32) f->xs[0][k] = root_feats[p * kFeat + k];
            __syncwarp();
        } else {
            stage_state_moves(w, st_g, mv_g);
            Setup S = setup_position(w);
            features_full(w, n, f->xs[0]);
        }
        float val[kFnnChunk], lg[kFnnChunk];
        fnn_encode_chunk(wts, dims, off, f, 1, val);
        const float root_value = val[0];
        fnn_root_pre(wts, dims, off, f);
        float* cq = child_q + p * kMaxMoves;
#pragma unroll 1
        for (int base = 0; base < n; base += kFnnChunk) {
            const int ns = min(kFnnChunk, n - base);
#pragma unroll 1
            for (int s = 0; s < ns; s++) {
                stage_state(w, st_g);
                {
                    const uint8_t* m = mv_g + (base + s) * kMoveBytes;
                    st_apply_warp(w->st, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8));
                }
                Setup S = setup_position(w);
                int cn = gen_compact(w, &g_error);
                features(w, cn, f->xs[s]);
            }
            fnn_encode_chunk(wts, dims, off, f, ns, val);
            fnn_score_chunk(wts, dims, off, f, ns, lg);
            if (l < ns) {
                // lane s stores successor s (values are warp-uniform)
                float lv = lg[0], vv = val[0];
#pragma unroll
                for (int s = 1; s < kFnnChunk; s++)
                    if (l == s) {
                        lv = lg[s];
                        vv = val[s];
                    }
                f->logit[base + l] = lv;
                cq[base + l] = -vv;
            }
            __syncwarp();
        }
        // softmax over the legal slots (-1e30 padding, then zeroed)
        float mx = -INFINITY;
        for (int i = l; i < n; i += 32) mx = fmaxf(mx, f->logit[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        float sum = 0.0f;
        for (int i = l; i < n; i += 32) sum += expf(f->logit[i] - mx);
        sum = warp_sum(sum);
        float* pr = priors + p * kMaxMoves;
        for (int i = l; i < kMaxMoves; i += 32) {
            pr[i] = i < n ? expf(f->logit[i] - mx) / sum : 0.0f;
            if (i >= n) cq[i] = 0.0f;
            if (logits_out) logits_out[p * kMaxMoves + i] = i < n ? f->logit[i] : 0.0f;
        }
        if (l == 0) values[p] = root_value;
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// hybrid leaf evaluation (fnn_transformer_mcts_orchestrator.py:42-169
// _eval_states): FNN encode of the root and of every successor (generated
// in shared memory, as in k_fnn_eval), the transformer summary g from the
// trunk kernel, value and hybrid action scores, masked softmax; child Q = 0
// ---------------------------------------------------------------------------
struct HybSmem {
    float xm[kFnnChunk][32];  // move features of the chunk's moves
};

__device__ __forceinline__ HybSmem* hyb_slot() {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    return reinterpret_cast<HybSmem*>(smem_raw + (sizeof(WarpSmem) + sizeof(FnnSmem)) * kWarpsPerBlock) +
           (threadIdx.x >> 5);
}

// Root part of the hybrid evaluation for leaf p, root features in f->xs[0]:
// FNN root embedding (f->root_emb), tanh value head over [e_root ; g ;
// global6] (returned), graph context and the root half of policy_fc1
// (f->root_pre).  Uses f->logit[0..136) as scratch.
__device__ __noinline__ float hybrid_root(FnnSmem* f, int64_t p, const float* __restrict__ graph,
                                      const float* __restrict__ glob, const float* __restrict__ fw, FnnDims fd,
                                      const float* __restrict__ hw, HybDims hd) {
    const FnnOffsets fo = fnn_offsets(fd);
    const HybOffsets ho = hyb_offsets(hd);
    const int E = hd.E, A = hd.A, V = hd.V;
    const int l = lane_id();
    const int o0 = l, o1 = l + 32;
    float val[kFnnChunk];
    fnn_encode_chunk(fw, fd, fo, f, 1, val);
    for (int k = l; k < E; k += 32) f->root_emb[k] = f->ys[0][k];
    // per-leaf scratch in the (not yet used) logit row: g, global features, g_ctx
    float* sg = f->logit;
    float* sgl = f->logit + kHybGraph;
    float* sgc = f->logit + kHybGraph + 8;
    for (int k = l; k < kHybGraph; k += 32) sg[k] = graph[p * kHybGraph + k];
    if (l < kGlobFeat) sgl[l] = glob[p * kGlobFeat + l];
    __syncwarp();
    // value head: lane owns hidden units l, l+32, l+64, l+96
    float root_value;
    {
        float acc[4];
#pragma unroll
        for (int i = 0; i < 4; i++) acc[i] = (l + 32 * i) < V ? __ldg(hw + ho.vh1b + l + 32 * i) : 0.0f;
        const int nin = E + kHybGraph + kGlobFeat;
#pragma unroll 2
        for (int k = 0; k < nin; k++) {
            const float in = k < E ? f->root_emb[k] : (k < E + kHybGraph ? sg[k - E] : sgl[k - E - kHybGraph]);
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (l + 32 * i < V) acc[i] = fmaf(__ldg(hw + ho.vh1T + k * V + l + 32 * i), in, acc[i]);
        }
        float part = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (l + 32 * i < V) part += __ldg(hw + ho.vh2 + l + 32 * i) * fmaxf(acc[i], 0.0f);
        root_value = tanhf(warp_sum(part) + __ldg(hw + ho.vh2b));
    }
    // graph context g_ctx = pg g + b
    {
        float a = o0 < E ? __ldg(hw + ho.pgb + o0) : 0.0f, b = o1 < E ? __ldg(hw + ho.pgb + o1) : 0.0f;
        for (int k = 0; k < kHybGraph; k++) {
            const float gk = sg[k];
            if (o0 < E) a = fmaf(__ldg(hw + ho.pgT + k * E + o0), gk, a);
            if (o1 < E) b = fmaf(__ldg(hw + ho.pgT + k * E + o1), gk, b);
        }
        __syncwarp();
        if (o0 < E) sgc[o0] = a;
        if (o1 < E) sgc[o1] = b;
        __syncwarp();
    }
    // root half of policy_fc1: b' + W[:, 0:E] e_root + W[:, E:2E] g_ctx
    {
        float a = o0 < A ? __ldg(hw + ho.pf1b + o0) : 0.0f, b = o1 < A ? __ldg(hw + ho.pf1b + o1) : 0.0f;
        for (int k = 0; k < E; k++) {
            const float er = f->root_emb[k], gc = sgc[k];
            if (o0 < A) a = fmaf(__ldg(hw + ho.pf1T + k * A + o0), er, fmaf(__ldg(hw + ho.pf1T + (E + k) * A + o0), gc, a));
            if (o1 < A) b = fmaf(__ldg(hw + ho.pf1T + k * A + o1), er, fmaf(__ldg(hw + ho.pf1T + (E + k) * A + o1), gc, b));
        }
        if (o0 < A) f->root_pre[o0] = a;
        if (o1 < A) f->root_pre[o1] = b;
        __syncwarp();
    }
    return root_value;
}

__global__ void __launch_bounds__(kThreads, 2) k_hybrid_eval(
    const uint8_t* __restrict__ states, const uint8_t* __restrict__ legal_moves,
    const int32_t* __restrict__ num_legal, const float* __restrict__ root_feats, const float* __restrict__ graph,
    const float* __restrict__ glob, int64_t count, const float* __restrict__ fw, FnnDims fd,
    const float* __restrict__ hw, HybDims hd, float* __restrict__ priors, float* __restrict__ values,
    float* __restrict__ child_q, float* __restrict__ logits_out) {
    WarpSmem* w = warp_slot();
    FnnSmem* f = fnn_slot();
    HybSmem* x = hyb_slot();
    const FnnOffsets fo = fnn_offsets(fd);
    const HybOffsets ho = hyb_offsets(hd);
    const int E = hd.E, A = hd.A;
    const int l = lane_id();
    const int o0 = l, o1 = l + 32;
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < count;
         p += nwarps) {
        int n = num_legal[p];
        n = n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n);
        const uint8_t* st_g = states + p * kStateBytes;
        const uint8_t* mv_g = legal_moves + p * (kMaxMoves * kMoveBytes);
        if (root_feats) {
            for (int k = l; k < kFeat; k += 32) f->xs[0][k] = root_feats[p * kFeat + k];
            __syncwarp();
        } else {
            stage_state_moves(w, st_g, mv_g);
            Setup S = setup_position(w);
            features_full(w, n, f->xs[0]);
        }
        float val[kFnnChunk], lg[kFnnChunk];
        const float root_value = hybrid_root(f, p, graph, glob, fw, fd, hw, hd);
        float* cq = child_q + p * kMaxMoves;
#pragma unroll 1
        for (int base = 0; base < n; base += kFnnChunk) {
            const int ns = min(kFnnChunk, n - base);
            // move features of this chunk, read off the leaf position
            stage_state(w, st_g);
            {
                Pos P{w};
                const MoveCtx X = move_ctx(w);
                if (l < ns) {
                    const uint8_t* m = mv_g + (base + l) * kMoveBytes;
                    float mf[kMoveFeat];
                    move_features(P, w->st, X, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8), mf);
#pragma unroll
                    for (int k = 0; k < kMoveFeat; k++) x->xm[l][k] = mf[k];
                }
                __syncwarp();
            }
#pragma unroll 1
            for (int s = 0; s < ns; s++) {
                stage_state(w, st_g);
                {
                    const uint8_t* m = mv_g + (base + s) * kMoveBytes;
                    st_apply_warp(w->st, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8));
                }
                Setup S = setup_position(w);
                int cn = gen_compact(w, &g_error);
                features(w, cn, f->xs[s]);
            }
            fnn_encode_chunk(fw, fd, fo, f, ns, val);
            // z = root_pre + W[:, 2E:3E] e_succ + C m
            float z[kFnnChunk][2];
            const float r0 = o0 < A ? f->root_pre[o0] : 0.0f, r1 = o1 < A ? f->root_pre[o1] : 0.0f;
#pragma unroll
            for (int s = 0; s < kFnnChunk; s++) {
                z[s][0] = r0;
                z[s][1] = r1;
            }
#pragma unroll 2
            for (int k = 0; k < E; k++) {
                const float w0 = o0 < A ? __ldg(hw + ho.pf1T + (2 * E + k) * A + o0) : 0.0f;
                const float w1 = o1 < A ? __ldg(hw + ho.pf1T + (2 * E + k) * A + o1) : 0.0f;
#pragma unroll
                for (int s = 0; s < kFnnChunk; s++) {
                    const float e = f->ys[s][k];
                    z[s][0] = fmaf(w0, e, z[s][0]);
                    z[s][1] = fmaf(w1, e, z[s][1]);
                }
            }
#pragma unroll 1
            for (int k = 0; k < kMoveFeat; k++) {
                const float w0 = o0 < A ? __ldg(hw + ho.cT + k * A + o0) : 0.0f;
                const float w1 = o1 < A ? __ldg(hw + ho.cT + k * A + o1) : 0.0f;
#pragma unroll
                for (int s = 0; s < kFnnChunk; s++) {
                    const float mk = x->xm[s][k];
                    z[s][0] = fmaf(w0, mk, z[s][0]);
                    z[s][1] = fmaf(w1, mk, z[s][1]);
                }
            }
            const float u0 = o0 < A ? __ldg(hw + ho.pf2 + o0) : 0.0f, u1 = o1 < A ? __ldg(hw + ho.pf2 + o1) : 0.0f;
            const float b2 = __ldg(hw + ho.pf2b);
#pragma unroll
            for (int s = 0; s < kFnnChunk; s++) {
                float t = (o0 < A ? u0 * sigmoidf_(z[s][0]) : 0.0f) + (o1 < A ? u1 * sigmoidf_(z[s][1]) : 0.0f);
                lg[s] = warp_sum(t) + b2;
            }
            if (l < ns) {
                float lv = lg[0];
#pragma unroll
                for (int s = 1; s < kFnnChunk; s++)
                    if (l == s) lv = lg[s];
                f->logit[base + l] = lv;
            }
            __syncwarp();
        }
        float mx = -INFINITY;
        for (int i = l; i < n; i += 32) mx = fmaxf(mx, f->logit[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        float sum = 0.0f;
        for (int i = l; i < n; i += 32) sum += expf(f->logit[i] - mx);
        sum = warp_sum(sum);
        float* pr = priors + p * kMaxMoves;
        for (int i = l; i < kMaxMoves; i += 32) {
            pr[i] = i < n ? expf(f->logit[i] - mx) / sum : 0.0f;
            cq[i] = 0.0f;
            if (logits_out) logits_out[p * kMaxMoves + i] = i < n ? f->logit[i] : 0.0f;
        }
        if (l == 0) values[p] = root_value;
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// leaf evaluation as a row pipeline (the default evaluator path): successor
// rows are compacted over all leaves, their features written by
// k_successor_features, the network run by the tiled k_mlp_rows, the
// per-leaf parts by warp-per-leaf kernels.  Launch order:
//   k_row_offsets -> k_row_index -> k_successor_features (+ k_row_move_features)
//   -> k_leaf_root_{fnn,hybrid} -> k_mlp_rows -> k_leaf_softmax
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t clamp_rows(int n) { return n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n); }

// exclusive prefix sum of the clamped legal counts: row_start[T + 1] (one block)
__global__ void __launch_bounds__(1024) k_row_offsets(const int32_t* __restrict__ num_legal, int64_t T,
                                                      int64_t* __restrict__ row_start) {
    __shared__ int64_t part[1024];
    const int t = threadIdx.x;
    const int64_t per = (T + 1023) / 1024;
    const int64_t lo = min(T, (int64_t)t * per), hi = min(T, lo + per);
    int64_t sum = 0;
    for (int64_t i = lo; i < hi; i++) sum += clamp_rows(num_legal[i]);
    part[t] = sum;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
        const int64_t v = t >= off ? part[t - off] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    int64_t run = part[t] - sum;
    for (int64_t i = lo; i < hi; i++) {
        row_start[i] = run;
        run += clamp_rows(num_legal[i]);
    }
    if (t == 1023) row_start[T] = part[1023];
}

// leaf / slot of every row (rows past the capacity are dropped and flagged)
__global__ void __launch_bounds__(kThreads) k_row_index(const int32_t* __restrict__ num_legal, int64_t T,
                                                        const int64_t* __restrict__ row_start, int64_t cap,
                                                        int64_t* __restrict__ atr, int64_t* __restrict__ mi) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < T; p += nwarps) {
        const int64_t start = row_start[p], n = clamp_rows(num_legal[p]);
        for (int64_t i = l; i < n; i += 32) {
            if (start + i < cap) {
                atr[start + i] = p;
                mi[start + i] = i;
            }
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && row_start[T] > cap) atomicOr(&g_error, kErrBuffer);
}

// hybrid: the 31 move features of every row, read off the leaf position
__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_row_move_features(
    const uint8_t* __restrict__ states, const uint8_t* __restrict__ legal_moves,
    const int32_t* __restrict__ num_legal, int64_t T, const int64_t* __restrict__ row_start, int64_t cap,
    __half* __restrict__ mf) {
    WarpSmem* w = warp_slot();
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < T; p += nwarps) {
        const int64_t start = row_start[p], n = clamp_rows(num_legal[p]);
        if (n == 0) continue;
        stage_state(w, states + p * kStateBytes);
        Pos P{w};
        const MoveCtx X = move_ctx(w);
        const uint8_t* mv = legal_moves + p * (kMaxMoves * kMoveBytes);
        for (int64_t i = l; i < n; i += 32) {
            if (start + i >= cap) continue;
            const uint8_t* m = mv + i * kMoveBytes;
            float f[32];
            move_features(P, w->st, X, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8), f);
            f[31] = 0.0f;
            // fp16, slab layout of 128-row tiles (4 chunks of 8; feature 31 zero)
            const int64_t r = start + i;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint4 u;
                u.x = pack_half2(f[8 * c], f[8 * c + 1]);
                u.y = pack_half2(f[8 * c + 2], f[8 * c + 3]);
                u.z = pack_half2(f[8 * c + 4], f[8 * c + 5]);
                u.w = pack_half2(f[8 * c + 6], f[8 * c + 7]);
                *reinterpret_cast<uint4*>(mf + (((r >> 7) * 4 + c) * 128 + (r & 127)) * 8) = u;
            }
        }
        __syncwarp();
    }
}

// per-leaf part: root features (given, or from the leaf's own list), FNN
// root embedding, value, and the root half of the action layer -> root_pre[T][64]
template <bool HYB>
__global__ void __launch_bounds__(kThreads, 2) k_leaf_root(
    const uint8_t* __restrict__ states, const uint8_t* __restrict__ legal_moves,
    const int32_t* __restrict__ num_legal, const float* __restrict__ root_feats, const float* __restrict__ graph,
    const float* __restrict__ glob, int64_t count, const float* __restrict__ fw, FnnDims fd,
    const float* __restrict__ hw, HybDims hd, float* __restrict__ values, float* __restrict__ root_pre) {
    WarpSmem* w = warp_slot();
    FnnSmem* f = fnn_slot();
    const int l = lane_id();
    const int A = HYB ? hd.A : fd.A;
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < count;
         p += nwarps) {
        if (root_feats) {
            for (int k = l; k < kFeat; k += 32) f->xs[0][k] = root_feats[p * kFeat + k];
            __syncwarp();
        } else {
            int n = (int)clamp_rows(num_legal[p]);
            stage_state_moves(w, states + p * kStateBytes, legal_moves + p * (kMaxMoves * kMoveBytes));
            Setup S = setup_position(w);
            features_full(w, n, f->xs[0]);
        }
        float v;
        if (HYB) {
            v = hybrid_root(f, p, graph, glob, fw, fd, hw, hd);
        } else {
            float val[kFnnChunk];
            const FnnOffsets fo = fnn_offsets(fd);
            fnn_encode_chunk(fw, fd, fo, f, 1, val);
            v = val[0];
            fnn_root_pre(fw, fd, fo, f);
        }
        for (int k = l; k < 64; k += 32) root_pre[p * 64 + k] = k < A ? f->root_pre[k] : 0.0f;
        if (l == 0) values[p] = v;
        __syncwarp();
    }
}

// per-leaf softmax over the legal slots (-inf padding, then zeroed); the
// padding of child_q / logits is zeroed (the hybrid's child_q entirely)
template <bool HYB>
__global__ void __launch_bounds__(kThreads) k_leaf_softmax(const int32_t* __restrict__ num_legal, int64_t count,
                                                           const int64_t* __restrict__ row_start, int64_t cap,
                                                           float* __restrict__ logits, float* __restrict__ priors,
                                                           float* __restrict__ child_q) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < count;
         p += nwarps) {
        int64_t n = clamp_rows(num_legal[p]);
        n = min(n, max((int64_t)0, cap - row_start[p]));  // rows dropped at the capacity count as absent
        float* lg = logits + p * kMaxMoves;
        float mx = -INFINITY;
        for (int i = l; i < n; i += 32) mx = fmaxf(mx, lg[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        float sum = 0.0f;
        for (int i = l; i < n; i += 32) sum += expf(lg[i] - mx);
        sum = warp_sum(sum);
        for (int i = l; i < kMaxMoves; i += 32) {
            priors[p * kMaxMoves + i] = i < n ? expf(lg[i] - mx) / sum : 0.0f;
            if (HYB || i >= n) child_q[p * kMaxMoves + i] = 0.0f;
            if (i >= n) lg[i] = 0.0f;
        }
    }
}

// ---------------------------------------------------------------------------
// queen escape flags (game_logic.cu:133-142, move_gen.cuh:771-821): can the
// side to move's queen slide away, or be thrown by an own pillbug / a ground
// mosquito next to a pillbug?
// ---------------------------------------------------------------------------
// queen escape of the staged state (move_gen.cuh:771-821); warp-uniform result
__device__ __noinline__ bool queen_escape_staged(WarpSmem* w) {
    Pos P{w};
    const int color = P.turn() & 1;
    const int q = P.queen_cell(color);
    if (!((P.queen_placed() >> color) & 1) || q < 0 || q >= kPCells || (q & 31) >= kBoard) return false;
    Setup S = setup_position(w);
    if (!P.occupied(q)) return false;
    const int top = P.top(q);
    const int qi = P.pidx(q);
    const bool pinned = qi < 32 && (w->pflag[qi] & 1);
    if ((top & 15) == 1 && ((top >> 4) & 1) == color && !pinned && walk(w, q, WM_STEP, w->dst, 6, true))
        return true;
    int mt = S.my_top & 15;
    bool mine = S.my_cell >= 0 && rowbit(w->own, S.my_cell);
    bool adj = S.my_cell >= 0 && hex_distance(S.my_cell, q) == 1;
    bool thr = mine && adj && (mt == 8 || (mt == 6 && S.my_h == 1 && next_to_pillbug(w, S.my_cell)));
    uint32_t throwers = __ballot_sync(kFull, thr);
    while (throwers) {
        int i = __ffs(throwers) - 1;
        throwers &= throwers - 1;
        int pb = w->pcell[i];
        uint32_t tm, dm;
        throw_sets(w, pb, tm, dm);
        int dq = -1;
        for (int d = 0; d < 6; d++)
            if (nbr(pb, d) == q) dq = d;
        if (dq >= 0 && ((tm >> dq) & 1) && dm) return true;
    }
    return false;
}

// Per (state, legal slot): apply the move to a copy and report the child's
// result, the number of occupied neighbours of the child's side-to-move
// queen (0 if unplaced) and, optionally, whether that queen can escape.
// Backs FNNMCTSOrchestrator._find_immediate_wins (fnn_mcts_orchestrator.py:
// 446-493) and _queen_surround_qualifying_mask (:339-382).
__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_child_probe(
    const uint8_t* __restrict__ states, const uint8_t* __restrict__ legal,
    const int32_t* __restrict__ num_legal, int64_t batch, int want_escape,
    int32_t* __restrict__ results, int32_t* __restrict__ surround, uint8_t* __restrict__ escape) {
    WarpSmem* w = warp_slot();
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        int n = num_legal[p];
        n = n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n);
        for (int m = l; m < kMaxMoves; m += 32) {
            if (m < n) continue;
            results[p * kMaxMoves + m] = 0;
            surround[p * kMaxMoves + m] = 0;
            if (escape) escape[p * kMaxMoves + m] = 0;
        }
        for (int m = 0; m < n; m++) {
            stage_state(w, states + p * kStateBytes);
            {
                const uint8_t* x = legal + (p * kMaxMoves + m) * kMoveBytes;
                st_apply_warp(w->st, x[0], x[1], x[2] | (x[3] << 8), x[4] | (x[5] << 8));
            }
            Pos P{w};
            const int color = P.turn() & 1;
            // occupied (height > 0) neighbours of the queen cell field, as
            // _queen_surround_count (fnn_mcts_orchestrator.py:318-337) reads it
            int cnt = 0;
            int qc = w->st[kOffQCell + 2 * color] | (w->st[kOffQCell + 2 * color + 1] << 8);
            if (qc != 0xFFFF) {
                const int q = c_to_p(qc < kCells ? qc : kCells - 1);
                int nb = l < 6 ? nbr(q, l) : -1;
                cnt = __popc(__ballot_sync(kFull, nb >= 0 && P.height(nb) > 0));
            }
            bool esc = want_escape ? queen_escape_staged(w) : false;
            if (l == 0) {
                results[p * kMaxMoves + m] = w->st[kOffResult];
                surround[p * kMaxMoves + m] = cnt;
                if (escape) escape[p * kMaxMoves + m] = esc ? 1 : 0;
            }
            __syncwarp();
        }
    }
}

__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_queen_escape(
    const uint8_t* __restrict__ states, int64_t batch, uint8_t* __restrict__ flags) {
    WarpSmem* w = warp_slot();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        stage_state(w, states + p * kStateBytes);
        bool esc = queen_escape_staged(w);
        if (lane_id() == 0) flags[p] = esc ? 1 : 0;
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// hybrid transformer inputs (game_logic.cu:93-131 generate_legal_moves_and_
// hybrid_root_features_kernel, state_encoder.cuh:552-597): piece tokens,
// move features, optionally fused with move generation and FNN features
// ---------------------------------------------------------------------------
struct HybridOut {
    float* tf;
    int32_t* tq;
    int32_t* tr;
    int32_t* tz;
    uint8_t* tm;
    float* gf;
    int32_t* ntok;
    float* mf;
};

template <bool GEN, bool TOKENS, bool MOVEF>
__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_hybrid(const uint8_t* __restrict__ states,
                                                                    const uint8_t* __restrict__ moves_in,
                                                                    const int32_t* __restrict__ nl_in,
                                                                    int64_t batch, uint8_t* __restrict__ moves_out,
                                                                    int32_t* __restrict__ nl_out,
                                                                    float* __restrict__ feats_out, HybridOut o) {
    WarpSmem* w = warp_slot();
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        stage_state(w, states + p * kStateBytes);
        int n = 0;
        if (GEN) {
            Setup S = setup_position(w);
            n = gen_legal(w, &g_error);
            store_moves(w, moves_out + p * (kMaxMoves * kMoveBytes), n);
            if (l == 0) nl_out[p] = n;
            features_full(w, n, feats_out + p * kFeat);
            if (TOKENS) {
                // reads only the staged state and S, which features() leaves intact
                int t = hybrid_tokens(w, o.tf + p * kTokens * kTokFeat, o.tq + p * kTokens,
                                      o.tr + p * kTokens, o.tz + p * kTokens, o.tm + p * kTokens,
                                      o.gf + p * kGlobFeat);
                if (l == 0) o.ntok[p] = t;
            }
        } else {
            if (TOKENS) {
                Setup S = setup_position(w);
                int t = hybrid_tokens(w, o.tf + p * kTokens * kTokFeat, o.tq + p * kTokens,
                                      o.tr + p * kTokens, o.tz + p * kTokens, o.tm + p * kTokens,
                                      o.gf + p * kGlobFeat);
                if (l == 0) o.ntok[p] = t;
            }
            if (MOVEF) {
                stage_async<kMoves16>(w->mv, moves_in + p * (kMaxMoves * kMoveBytes));
                n = nl_in[p];
                n = n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n);
                stage_wait();
            }
        }
        if (MOVEF) {
            Pos P{w};
            const MoveCtx X = move_ctx(w);
            for (int m = l; m < kMaxMoves; m += 32) {
                float f[kMoveFeat];
                if (m < n) {
                    const uint16_t a = w->mv[3 * m];
                    move_features(P, w->st, X, a & 0xFF, a >> 8, w->mv[3 * m + 1], w->mv[3 * m + 2], f);
                } else {
#pragma unroll
                    for (int k = 0; k < kMoveFeat; k++) f[k] = 0.0f;
                }
                float* row = o.mf + (p * kMaxMoves + m) * kMoveFeat;
#pragma unroll
                for (int k = 0; k < kMoveFeat; k++) row[k] = f[k];
            }
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// root tactical probe (game_logic.cu:290-397), five passes (hv_tactics.cuh)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int clamp_legal(int n) { return n < 0 ? 0 : (n > kMaxMoves ? kMaxMoves : n); }

// pass 1, warp per root: stage flags, winning = -1, allowed = slot < n
__global__ void __launch_bounds__(kThreads) k_tac_flags(const uint8_t* __restrict__ states,
                                                        const int32_t* __restrict__ num_legal,
                                                        int64_t batch, int w1, int chk, int w2,
                                                        int64_t* __restrict__ winning,
                                                        uint8_t* __restrict__ allowed,
                                                        uint8_t* __restrict__ flags) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        const int n = clamp_legal(num_legal[p]);
        for (int i = l; i < kMaxMoves; i += 32) allowed[p * kMaxMoves + i] = i < n ? 1 : 0;
        const uint8_t* st = states + p * kStateBytes;
        const int me = st_u16(st, kOffTurn) & 1;
        const int opp_s = surround_count(st, me ^ 1);
        const int own_s = surround_count(st, me);
        int f = opp_s << kTacOppShift;
        if (n > 0 && st[kOffResult] == 0) {
            if (w1 && opp_s == 5) f |= kTacS1;
            if (chk && own_s == 5) f |= kTacS2;
            if (w2 && (opp_s == 4 || opp_s == 5)) f |= kTacS3;
        }
        if (l == 0) {
            winning[p] = -1;
            flags[p] = (uint8_t)f;
        }
    }
}

// pass 2, warp per (root, child): does the child win at once (win-in-one
// probe), can the opponent win at once from it (screen)?
__global__ void __launch_bounds__(kThreads, HV_MIN_BLOCKS) k_tac_children(
    const uint8_t* __restrict__ states, const uint8_t* __restrict__ legal,
    const int32_t* __restrict__ num_legal, int64_t batch, const uint8_t* __restrict__ flags,
    uint8_t* __restrict__ allowed) {
    WarpSmem* w = warp_slot();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t t = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); t < batch * kMaxMoves;
         t += nwarps) {
        const int64_t p = t >> 8;
        const int i = (int)(t & 255);
        const int f = flags[p];
        if (!(f & (kTacS1 | kTacS2)) || i >= clamp_legal(num_legal[p])) continue;
        const uint8_t* root = states + p * kStateBytes;
        const uint8_t* mi = legal + (p * kMaxMoves + i) * kMoveBytes;
        auto rebuild = [&]() {
            stage_state(w, root);
            if (lane_id() == 0) apply_bytes(w->st, mi);
            __syncwarp();
        };
        rebuild();
        const int me = (st_u16(w->st, kOffTurn) & 1) ^ 1;
        int a = 1;
        if ((f & kTacS1) && wins_for(w->st[kOffResult], me)) a |= 2;
        if ((f & kTacS2) && immediate_win_staged(w, rebuild, &g_error)) a &= ~1;
        if (lane_id() == 0) allowed[p * kMaxMoves + i] = (uint8_t)a;
        __syncwarp();
    }
}

// pass 3, warp per root: win-in-one by best prior (first of equal priors),
// else the screen's "no safe move" verdict
__global__ void __launch_bounds__(kThreads) k_tac_decide(const int32_t* __restrict__ num_legal,
                                                         const float* __restrict__ priors, int64_t batch,
                                                         int64_t* __restrict__ winning,
                                                         uint8_t* __restrict__ allowed,
                                                         uint8_t* __restrict__ flags) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        int f = flags[p];
        if (!(f & (kTacS1 | kTacS2))) continue;
        const int n = clamp_legal(num_legal[p]);
        uint8_t* a = allowed + p * kMaxMoves;
        int best = -1;
        if (f & kTacS1) {
            // sequential scan keeps the reference's comparison order exactly (NaN included)
            if (l == 0) {
                float bp = -1e30f;
                for (int i = 0; i < n; i++)
                    if ((a[i] & 2) && (best < 0 || priors[p * kMaxMoves + i] > bp)) {
                        best = i;
                        bp = priors[p * kMaxMoves + i];
                    }
            }
            best = __shfl_sync(kFull, best, 0);
        }
        bool safe = false;
        for (int i = l; i < n; i += 32) safe |= (a[i] & 1) != 0;
        safe = __any_sync(kFull, safe);
        if (best >= 0) {
            f |= kTacDone;  // the probe returns before the screen: allowed stays "slot < n"
            for (int i = l; i < kMaxMoves; i += 32) a[i] = i < n ? 1 : 0;
            if (l == 0) winning[p] = best;
        } else {
            if ((f & kTacS2) && !safe) f |= kTacDone | kTacForced;
            for (int i = l; i < kMaxMoves; i += 32) a[i] &= 1;
        }
        if (l == 0) flags[p] = (uint8_t)f;
    }
}

// pass 4, warp per (root, allowed child): forced win in two -- every reply
// keeps the opponent queen's surround from dropping and leaves a win at once
__global__ void __launch_bounds__(kThreads, 2) k_tac_win2(const uint8_t* __restrict__ states,
                                                          const uint8_t* __restrict__ legal,
                                                          const int32_t* __restrict__ num_legal,
                                                          int64_t batch, const uint8_t* __restrict__ flags,
                                                          uint8_t* __restrict__ allowed) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    WarpSmem* w = warp_slot();
    TacSmem* x = reinterpret_cast<TacSmem*>(smem_raw + sizeof(WarpSmem) * kWarpsPerBlock) + (threadIdx.x >> 5);
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t t = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); t < batch * kMaxMoves;
         t += nwarps) {
        const int64_t p = t >> 8;
        const int i = (int)(t & 255);
        const int f = flags[p];
        if (!(f & kTacS3) || (f & kTacDone) || i >= clamp_legal(num_legal[p])) continue;
        if (!(allowed[p * kMaxMoves + i] & 1)) continue;
        stage_state(w, states + p * kStateBytes);
        if (lane_id() == 0) apply_bytes(w->st, legal + (p * kMaxMoves + i) * kMoveBytes);
        __syncwarp();
        copy_state(x->child, w->st);
        const int me = (st_u16(x->child, kOffTurn) & 1) ^ 1;
        const int opp = me ^ 1;
        const int opp_s = f >> kTacOppShift;
        const int cs = surround_count(x->child, opp);
        if (opp_s == 4 && cs <= opp_s) continue;
        if (opp_s == 5 && cs < opp_s) continue;
        Setup S = setup_position(w);
        const int nr = gen_legal(w, &g_error);
        for (int k = lane_id(); k < 3 * nr; k += 32) x->rep[k] = w->mv[k];
        __syncwarp();
        int r = 0;
        auto rebuild = [&]() {
            copy_state(w->st, x->child);
            if (lane_id() == 0) apply_list(w->st, x->rep, r);
            __syncwarp();
        };
        // generate_non_decreasing_surround_replies (move_gen.cuh:876-899)
        bool ok = true;
        for (r = 0; r < nr; r++) {
            rebuild();
            if (surround_count(w->st, opp) < cs) {
                ok = false;
                break;
            }
        }
        for (r = 0; ok && r < nr; r++) {
            rebuild();
            if (wins_for(w->st[kOffResult], me)) continue;
            if (!immediate_win_staged(w, rebuild, &g_error)) ok = false;
        }
        if (ok && lane_id() == 0) allowed[p * kMaxMoves + i] |= 4;
        __syncwarp();
    }
}

// pass 5, warp per root: first forced win in two; final 0/1 outputs
__global__ void __launch_bounds__(kThreads) k_tac_final(const int32_t* __restrict__ num_legal,
                                                        int64_t batch, int64_t* __restrict__ winning,
                                                        uint8_t* __restrict__ allowed,
                                                        uint8_t* __restrict__ flags) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        const int f = flags[p];
        const int n = clamp_legal(num_legal[p]);
        uint8_t* a = allowed + p * kMaxMoves;
        if ((f & kTacS3) && !(f & kTacDone)) {
            int first = -1;
            for (int base = 0; base < n && first < 0; base += 32) {
                const int i = base + l;
                const uint32_t b = __ballot_sync(kFull, i < n && (a[i] & 4));
                if (b) first = base + __ffs(b) - 1;
            }
            if (first >= 0 && l == 0) winning[p] = first;
        }
        __syncwarp();
        for (int i = l; i < kMaxMoves; i += 32) a[i] &= 1;
        if (l == 0) flags[p] = (f & kTacForced) ? 1 : 0;
    }
}

// ---------------------------------------------------------------------------
// MCTS tree kernels: one warp per game (hv_mcts.cuh)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_mcts_select(TreeDev t, SelectArgs a) {
    const int nwarps = gridDim.x * kWarpsPerBlock;
    for (int g = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); g < a.B; g += nwarps)
        select_game(t, a, g);
}

// plain / root-mask modes: one block per game (root steps, then the descents)
__global__ void __launch_bounds__(kTreeThreads) k_mcts_select_tree(TreeDev t, SelectArgs a) {
    extern __shared__ __align__(16) int32_t sel_sm[];
    const int per = a.total / a.B;
    select_game_tree(t, a, blockIdx.x, sel_sm, sel_sm + per);
}

// root-slot mode: one warp per (game, candidate)
__global__ void __launch_bounds__(kThreads) k_mcts_select_slots(TreeDev t, SelectArgs a) {
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock, n = (int64_t)a.B * a.C;
    for (int64_t i = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); i < n; i += nwarps)
        select_game_slot(t, a, (int)(i / a.C), (int)(i % a.C));
}

// dense expansion + backup in simulation groups: one block per game (C warps
// for root slots, kTreeThreads otherwise)
__global__ void __launch_bounds__(1024) k_mcts_expand_slots(TreeDev t, ExpandArgs a, const int32_t* roots,
                                                            const int32_t* slots, int C) {
    extern __shared__ __align__(16) int32_t xs_sm[];
    expand_game_groups(t, a, roots, slots, C, blockIdx.x, xs_sm);
}

__global__ void __launch_bounds__(kThreads) k_mcts_expand(TreeDev t, ExpandArgs a) {
    const int nwarps = gridDim.x * kWarpsPerBlock;
    for (int g = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); g < a.B; g += nwarps)
        expand_game(t, a, g);
}

__global__ void __launch_bounds__(kThreads) k_mcts_backprop(TreeDev t, const int32_t* leaf,
                                                            const float* values, const int32_t* vlp,
                                                            const int32_t* vll, const int8_t* was,
                                                            int B, int total) {
    const int nwarps = gridDim.x * kWarpsPerBlock;
    for (int g = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); g < B; g += nwarps)
        backprop_game(t, leaf, values, vlp, vll, was, B, total, g);
}

// leaf state = root state + path moves (mcts_tree.cuh:298-320); one warp per simulation
__global__ void __launch_bounds__(kThreads) k_mcts_replay(const uint8_t* __restrict__ roots,
                                                          uint8_t* __restrict__ leaves,
                                                          const uint8_t* __restrict__ paths,
                                                          const int32_t* __restrict__ plen,
                                                          const int32_t* __restrict__ leaf, int B,
                                                          int total) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* st = smem_raw + (threadIdx.x >> 5) * kStateBytes;
    const int nwarps = gridDim.x * kWarpsPerBlock;
    for (int s = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); s < total; s += nwarps) {
        if (leaf[s] < 0) {
            // no simulation in this slot: an all-zero state, as the
            // reference's zero-filled leaf buffer holds there (so the caller
            // needs no zero-fill of the whole buffer first)
            uint4* o4 = reinterpret_cast<uint4*>(leaves + (int64_t)s * kStateBytes);
            for (int i = lane_id(); i < kStateBytes / 16; i += 32) o4[i] = make_uint4(0u, 0u, 0u, 0u);
            continue;
        }
        stage_async<kState16>(st, roots + (int64_t)(s % B) * kStateBytes);
        stage_wait();
        if (lane_id() == 0) {
            int n = plen[s];
            n = n < 0 ? 0 : (n > kTreeDepth ? kTreeDepth : n);
            for (int k = 0; k < n; k++) {
                const uint8_t* m = paths + ((int64_t)s * kTreeDepth + k) * 6;
                st_apply(st, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8));
            }
        }
        __syncwarp();
        uint4* o4 = reinterpret_cast<uint4*>(leaves + (int64_t)s * kStateBytes);
        const uint4* d4 = reinterpret_cast<const uint4*>(st);
        for (int i = lane_id(); i < kStateBytes / 16; i += 32) o4[i] = d4[i];
        __syncwarp();
    }
}

// root prior temperature + Dirichlet mix (mcts_tree.cuh:1192-1234); one thread per game
__global__ void k_mcts_root_noise(TreeDev t, const float* noise, const int32_t* roots, int pad,
                                  float eps, float temp, int B) {
    int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= B) return;
    int64_t ri = tix(t, g, roots[g]);
    int fc = t.fc[ri], nc = t.nc[ri];
    if (fc < 0 || nc == 0) return;
    if (temp > 1.0f) {
        float inv = __fdiv_rn(1.0f, temp), sum = 0.0f;
        for (int c = 0; c < nc; c++) {
            int64_t ci = tix(t, g, fc + c);
            float p = powf(t.pr[ci], inv);
            t.pr[ci] = p;
            sum = __fadd_rn(sum, p);
        }
        if (sum > 0.0f)
            for (int c = 0; c < nc; c++) {
                int64_t ci = tix(t, g, fc + c);
                t.pr[ci] = __fdiv_rn(t.pr[ci], sum);
            }
    }
    if (eps > 0.0f)
        for (int c = 0; c < nc; c++) {
            int64_t ci = tix(t, g, fc + c);
            float x = __fmul_rn(__fsub_rn(1.0f, eps), t.pr[ci]);
            float y = __fmul_rn(eps, noise[(int64_t)g * pad + c]);
            t.pr[ci] = __fadd_rn(x, y);
        }
}

// visit-count policy over the action space (mcts_tree.cuh:607-684); one thread per game
__global__ void k_mcts_extract_policy(TreeDev t, float* pol, const int32_t* move_numbers,
                                      const int32_t* roots, float temperature, int drop, float prune,
                                      int B) {
    int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= B) return;
    float* p = pol + (int64_t)g * 85834;
    int64_t ri = tix(t, g, roots[g]);
    int fc = t.fc[ri], nc = t.nc[ri];
    if (fc < 0 || nc == 0) return;
    float temp = move_numbers[g] >= drop ? 0.0f : temperature;
    if (temp <= 0.0f) {
        int ba = -1, bv = -1;
        for (int c = 0; c < nc; c++) {
            int64_t ci = tix(t, g, fc + c);
            if (t.vc[ci] > bv) {
                bv = t.vc[ci];
                ba = t.ai[ci];
            }
        }
        if (ba >= 0 && ba < 85834) p[ba] = 1.0f;
        return;
    }
    float mx = 0.0f, sum = 0.0f;
    for (int c = 0; c < nc; c++) {
        float v = (float)t.vc[tix(t, g, fc + c)];
        if (v > mx) mx = v;
    }
    for (int c = 0; c < nc; c++) {
        int64_t ci = tix(t, g, fc + c);
        float v = (float)t.vc[ci];
        if (prune > 0.0f && mx > 0.0f && v < __fmul_rn(mx, prune)) v = 0.0f;
        if (temp != 1.0f) v = powf(v, __fdiv_rn(1.0f, temp));
        int act = t.ai[ci];
        if (act >= 0 && act < 85834) {
            p[act] = v;
            sum = __fadd_rn(sum, v);
        }
    }
    for (int c = 0; c < nc; c++) {
        int act = t.ai[tix(t, g, fc + c)];
        if (act >= 0 && act < 85834) p[act] = sum > 0.0f ? __fdiv_rn(p[act], sum) : __fdiv_rn(1.0f, (float)nc);
    }
}

// ---------------------------------------------------------------------------
// state operations
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_init_states(uint8_t* __restrict__ states,
                                                          int64_t batch, int mask) {
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        uint8_t* st = states + p * kStateBytes;
        uint4* d4 = reinterpret_cast<uint4*>(st);
        for (int i = lane_id(); i < kStateBytes / 16; i += 32) d4[i] = make_uint4(0, 0, 0, 0);
        __syncwarp();
        if (lane_id() == 0) st_init_fields(st, mask);
        __syncwarp();
    }
}

__global__ void k_apply_moves(uint8_t* __restrict__ states, const uint8_t* __restrict__ moves,
                              int64_t batch) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch) return;
    const uint8_t* m = moves + i * kMoveBytes;
    st_apply(states + i * kStateBytes, m[0], m[1], m[2] | (m[3] << 8), m[4] | (m[5] << 8));
}

__global__ void k_check_results(const uint8_t* __restrict__ states, int64_t batch,
                                int32_t* __restrict__ results) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < batch) results[i] = states[i * kStateBytes + kOffResult];
}

// seeded uniform random legal playouts (benchmark / test inputs)
__global__ void __launch_bounds__(kThreads) k_playouts(uint64_t seed, int64_t first_game,
                                                       int64_t count, int max_ply, int mask,
                                                       uint8_t* __restrict__ out) {
    WarpSmem* w = warp_slot();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t i = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); i < count;
         i += nwarps) {
        uint64_t g = (uint64_t)(first_game + i);
        uint4* d4 = reinterpret_cast<uint4*>(w->st);
        for (int k = lane_id(); k < kStateBytes / 16; k += 32) d4[k] = make_uint4(0, 0, 0, 0);
        __syncwarp();
        if (lane_id() == 0) st_init_fields(w->st, mask);
        __syncwarp();
        int stop = (int)(game_rng(seed, g, 0) % (uint64_t)(max_ply + 1));
        for (int p = 1; p <= stop; p++) {
            if (w->st[kOffResult] != 0) break;
            Setup S = setup_position(w);
            int n = gen_legal(w, &g_error);
            int k = (int)(game_rng(seed, g, (uint64_t)p) % (uint64_t)n);
            {
                const uint16_t* m = w->mv + 3 * k;
                st_apply_warp(w->st, m[0] & 255, m[0] >> 8, m[1], m[2]);
            }
        }
        uint4* o4 = reinterpret_cast<uint4*>(out + i * kStateBytes);
        for (int k = lane_id(); k < kStateBytes / 16; k += 32) o4[k] = d4[k];
        __syncwarp();
    }
}

constexpr int kActionSpace = 85834;  // ENC_GRID 17: 8 x 289 placements + 289 x 289 moves + pass

// round-half-to-even of sum / n (state_encoder.cuh:55-79)
__device__ __forceinline__ int round_half_even(int sum, int n) {
    int q = sum / n, r = sum - q * n;
    int twice = 2 * (r < 0 ? -r : r);
    if (twice < n) return q;
    int away = sum > 0 ? q + 1 : q - 1;
    if (twice > n) return away;
    return (q & 1) == 0 ? q : away;
}

// centroid (state_encoder.cuh:889-906) and move -> action index
// (mcts_tree.cuh:146-179, game_logic.cu:811-835); one warp per state
__global__ void __launch_bounds__(kThreads) k_actions(const uint8_t* __restrict__ states,
                                                      const uint8_t* __restrict__ moves,
                                                      const int32_t* __restrict__ num_legal,
                                                      int64_t batch, int32_t* __restrict__ actions,
                                                      int32_t* __restrict__ centroids,
                                                      float* __restrict__ masks) {
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    const int l = lane_id();
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < batch;
         p += nwarps) {
        const uint8_t* h = states + p * kStateBytes + kOffHeight;
        int sq = 0, sr = 0, n = 0;
        for (int c = l; c < kCells; c += 32) {
            if (h[c]) {
                int r = c / kBoard;
                sq += c - r * kBoard - 11;
                sr += r - 11;
                n++;
            }
        }
        sq = __reduce_add_sync(kFull, sq);
        sr = __reduce_add_sync(kFull, sr);
        n = __reduce_add_sync(kFull, n);
        int cq = n ? round_half_even(sq, n) : 0, cr = n ? round_half_even(sr, n) : 0;
        if (centroids && l == 0) {
            centroids[2 * p] = cq;
            centroids[2 * p + 1] = cr;
        }
        float* mrow = masks ? masks + p * (int64_t)kActionSpace : nullptr;
        if (mrow) {
            // zero the row (8-byte aligned: 85834 floats per row), then set the legal actions
            float2* m2 = reinterpret_cast<float2*>(mrow);
            for (int i = l; i < kActionSpace / 2; i += 32) m2[i] = make_float2(0.0f, 0.0f);
            __syncwarp();
        }
        if (actions || mrow) {
            int nl = num_legal[p];
            nl = nl < 0 ? 0 : (nl > kMaxMoves ? kMaxMoves : nl);
            const uint8_t* mv = moves + p * (kMaxMoves * kMoveBytes);
            for (int m = l; m < kMaxMoves; m += 32) {
                int a = -1;
                if (m < nl) {
                    const uint8_t* x = mv + m * kMoveBytes;
                    int type = x[0], pt = x[1], from = x[2] | (x[3] << 8), to = x[4] | (x[5] << 8);
                    if (type == 2) a = 85833;
                    else if (type == 0) {
                        int ec = (to % kBoard - 11) - cq + 8, er = (to / kBoard - 11) - cr + 8;
                        if (ec >= 0 && ec < 17 && er >= 0 && er < 17) a = (pt - 1) * 289 + er * 17 + ec;
                    } else {
                        int sc = (from % kBoard - 11) - cq + 8, srr = (from / kBoard - 11) - cr + 8;
                        int dc = (to % kBoard - 11) - cq + 8, dr = (to / kBoard - 11) - cr + 8;
                        if (sc >= 0 && sc < 17 && srr >= 0 && srr < 17 && dc >= 0 && dc < 17 &&
                            dr >= 0 && dr < 17)
                            a = 2312 + (srr * 17 + sc) * 289 + dr * 17 + dc;
                    }
                }
                if (actions) actions[p * kMaxMoves + m] = a;
                if (mrow && a >= 0 && a < kActionSpace) mrow[a] = 1.0f;
            }
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------
struct DeviceInfo {
    int sms = 0;
    int blocks_per_sm = 0;
};
static DeviceInfo g_dev[64];

template <typename K>
static int grid_for(K kernel, int64_t units, size_t smem, int* out_grid) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HV_ECUDA;
    DeviceInfo& d = g_dev[dev];
    if (d.sms == 0) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return HV_ECUDA;
    }
    int per_sm = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return HV_ECUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) !=
        cudaSuccess)
        return HV_ECUDA;
    if (per_sm < 1) per_sm = 1;
    int64_t want = (units + kWarpsPerBlock - 1) / kWarpsPerBlock;
    int64_t cap = (int64_t)d.sms * per_sm;
    *out_grid = (int)(want < cap ? want : cap);
    if (*out_grid < 1) *out_grid = 1;
    return HV_OK;
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? HV_OK : HV_ECUDA;
}

template <bool GEN, bool WM, bool FE, bool AP_LINK = false, bool DYNF = false>
static int launch_root(const uint8_t* states, const uint8_t* mi, const int32_t* nli, int64_t batch,
                       uint8_t* mo, int32_t* nlo, float* fo, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (!states || !aligned16(states)) return HV_EINVAL;
    if (WM && (!mo || !nlo || !aligned16(mo))) return HV_EINVAL;
    if ((FE || AP_LINK) && !fo) return HV_EINVAL;
    if (!GEN && (!mi || !nli || !aligned16(mi))) return HV_EINVAL;
    size_t smem = (size_t)((!GEN && AP_LINK) ? kFeatSlotBytes : (int)sizeof(WarpSmem)) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_root<GEN, WM, FE, AP_LINK, DYNF>, batch, smem, &grid);
    if (rc) return rc;
    k_root<GEN, WM, FE, AP_LINK, DYNF><<<grid, kThreads, smem, (cudaStream_t)stream>>>(states, mi, nli, batch, mo,
                                                                                       nlo, fo);
    return launch_status();
}

template <bool GEN, bool TOKENS, bool MOVEF>
static int launch_hybrid(const uint8_t* states, const uint8_t* mi, const int32_t* nli, int64_t batch,
                         uint8_t* mo, int32_t* nlo, float* fo, HybridOut o, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (!states || !aligned16(states)) return HV_EINVAL;
    if (GEN && (!mo || !nlo || !fo || !aligned16(mo))) return HV_EINVAL;
    if (!GEN && MOVEF && (!mi || !nli || !aligned16(mi))) return HV_EINVAL;
    if (TOKENS && (!o.tf || !o.tq || !o.tr || !o.tz || !o.tm || !o.gf || !o.ntok)) return HV_EINVAL;
    if (MOVEF && !o.mf) return HV_EINVAL;
    size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_hybrid<GEN, TOKENS, MOVEF>, batch, smem, &grid);
    if (rc) return rc;
    k_hybrid<GEN, TOKENS, MOVEF><<<grid, kThreads, smem, (cudaStream_t)stream>>>(states, mi, nli, batch, mo, nlo,
                                                                                fo, o);
    return launch_status();
}

struct RowWorkspace {
    int64_t* row_start;  // [count + 1]
    int64_t* atr;        // [rows]
    int64_t* mi;         // [rows]
    float* x;            // FNN: fp32 slab tiles of the successor features, 512 bytes per row
    __half* xh;          // hybrid: fp16 slab tiles of the successor features, 256 bytes per row
    __half* mfh;         // hybrid: fp16 slab tiles of the move features, 64 bytes per row
    float* root_pre;     // [count][64]
    float* logits;       // [count][256] (when the caller passes none)
};

// The FNN row network of widths 32 and up (the medium and large presets)
// runs on the tensor cores with split fp16 products; the 8-wide small
// preset keeps the fp32 CUDA-core kernel: LayerNorm over 8 neurons amplifies
// rounding differences to the edge of the 1e-5 check even with exact
// products, and the split adds its own ~2^-22 on top.
static inline bool fnn_rows_on_tensor_cores(FnnDims fd) { return fd.H >= 32; }

template <bool HYB>
static int run_row_pipeline(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            const float* root_features, const float* graph, const float* glob, int64_t count,
                            int64_t rows, const float* fw, FnnDims fd, const float* hw, HybDims hd, float* priors,
                            float* values, float* child_q, float* logits, RowWorkspace& w, cudaStream_t s) {
    float* lg = logits ? logits : w.logits;
    k_row_offsets<<<1, 1024, 0, s>>>(num_legal, count, w.row_start);
    int grid = 0;
    int rc = grid_for(k_row_index, count, 0, &grid);
    if (rc) return rc;
    k_row_index<<<grid, kThreads, 0, s>>>(num_legal, count, w.row_start, rows, w.atr, w.mi);
    if (rows > 0) {
        size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
        // the row counter lives in root_pre, which the per-leaf kernel writes only later
        unsigned long long* ctr = reinterpret_cast<unsigned long long*>(w.root_pre);
        if (cudaMemsetAsync(ctr, 0, sizeof(unsigned long long), s) != cudaSuccess) return HV_ECUDA;
        if (HYB) {
            rc = grid_for(k_successor_features<kSlabF16>, rows, smem, &grid);
            if (rc) return rc;
            k_successor_features<kSlabF16><<<grid, kThreads, smem, s>>>(states, count, legal_moves, w.atr, w.mi,
                                                                        rows, w.xh, w.row_start + count, ctr);
        } else if (fnn_rows_on_tensor_cores(fd)) {
            rc = grid_for(k_successor_features<kSlabF16x2>, rows, smem, &grid);
            if (rc) return rc;
            k_successor_features<kSlabF16x2><<<grid, kThreads, smem, s>>>(states, count, legal_moves, w.atr, w.mi,
                                                                          rows, w.x, w.row_start + count, ctr);
        } else {
            rc = grid_for(k_successor_features<kSlabF32>, rows, smem, &grid);
            if (rc) return rc;
            k_successor_features<kSlabF32><<<grid, kThreads, smem, s>>>(states, count, legal_moves, w.atr, w.mi,
                                                                        rows, w.x, w.row_start + count, ctr);
        }
        if (HYB) {
            rc = grid_for(k_row_move_features, count, smem, &grid);
            if (rc) return rc;
            k_row_move_features<<<grid, kThreads, smem, s>>>(states, legal_moves, num_legal, count, w.row_start,
                                                            rows, w.mfh);
        }
    }
    if (HYB && root_features) {
        // the hybrid's per-leaf network on the tensor cores
        uint32_t* err = nullptr;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_error) != cudaSuccess) return HV_ECUDA;
        const size_t smem = sizeof(RootTcSmem);
        const int64_t tiles = (count + kTcRows - 1) / kTcRows, ctas = (tiles + kRtGroups - 1) / kRtGroups;
        rc = grid_for(k_leaf_root_tc, ctas * kWarpsPerBlock, smem, &grid);  // one CTA per SM (shared memory)
        if (rc) return rc;
        k_leaf_root_tc<<<grid, kRtThreads, smem, s>>>(root_features, graph, glob, count, fw, fd, hw, hd, values,
                                                      w.root_pre, err);
    } else if (!HYB && root_features) {
        // the FNN's per-leaf network tiled like the successor rows (fp32)
        const size_t smem = sizeof(MlpSmem<false>);
        const int64_t tiles = (count + kMlpRows - 1) / kMlpRows;
        rc = grid_for(k_mlp_rows<false, true>, tiles * kWarpsPerBlock, smem, &grid);
        if (rc) return rc;
        k_mlp_rows<false, true><<<grid, kMlpThreads, smem, s>>>(root_features, nullptr, nullptr, nullptr, count,
                                                                nullptr, fw, fd, hw, hd, w.root_pre, values,
                                                                nullptr);
    } else {
        size_t smem = (sizeof(WarpSmem) + sizeof(FnnSmem)) * kWarpsPerBlock;
        rc = grid_for(k_leaf_root<HYB>, count, smem, &grid);
        if (rc) return rc;
        k_leaf_root<HYB><<<grid, kThreads, smem, s>>>(states, legal_moves, num_legal, root_features, graph, glob,
                                                      count, fw, fd, hw, hd, values, w.root_pre);
    }
    if constexpr (HYB) {
      if (rows > 0) {
        // the hybrid network on the tensor cores (fp16 operands, as the reference's autocast)
        uint32_t* err = nullptr;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_error) != cudaSuccess) return HV_ECUDA;
        const size_t smem = sizeof(MlpTcSmem);
        const int64_t tiles = (rows + kTcRows - 1) / kTcRows, ctas = (tiles + kTcGroups - 1) / kTcGroups;
        rc = grid_for(k_mlp_rows_tc, ctas * kWarpsPerBlock, smem, &grid);  // one CTA per SM (shared memory)
        if (rc) return rc;
        k_mlp_rows_tc<<<grid, kTcThreads, smem, s>>>(w.xh, w.mfh, w.atr, w.mi, rows, w.root_pre, fw, fd, hw, hd, lg,
                                                     w.row_start + count, err);
      }
    } else if (rows > 0) {
        uint32_t* err = nullptr;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_error) != cudaSuccess) return HV_ECUDA;
        if (fnn_rows_on_tensor_cores(fd)) {
            // the network on the tensor cores over the hi / lo fp16 slab
            // tiles (fp32-accurate), one CTA per SM (shared memory)
            const size_t smem = sizeof(FxSmem);
            const int64_t tiles = (rows + kFxRows - 1) / kFxRows, ctas = (tiles + kFxGroups - 1) / kFxGroups;
            rc = grid_for(k_fnn_rows_tc, ctas * kWarpsPerBlock, smem, &grid);
            if (rc) return rc;
            k_fnn_rows_tc<<<grid, kFxThreads, smem, s>>>(reinterpret_cast<const __half*>(w.x), w.atr, w.mi, rows,
                                                         w.root_pre, fw, fd, lg, child_q, w.row_start + count, err);
        } else {
            // the network over the fp32 slab tiles on the CUDA cores, one CTA per SM (shared memory)
            const size_t smem = sizeof(F32Smem);
            const int64_t tiles = (rows + kF32Rows - 1) / kF32Rows, ctas = (tiles + kF32Groups - 1) / kF32Groups;
            rc = grid_for(k_fnn_rows, ctas * kWarpsPerBlock, smem, &grid);
            if (rc) return rc;
            k_fnn_rows<<<grid, kF32Threads, smem, s>>>(w.x, w.atr, w.mi, rows, w.root_pre, fw, fd, lg, child_q,
                                                       w.row_start + count, err);
        }
    }
    rc = grid_for(k_leaf_softmax<HYB>, count, 0, &grid);
    if (rc) return rc;
    k_leaf_softmax<HYB><<<grid, kThreads, 0, s>>>(num_legal, count, w.row_start, rows, lg, priors, child_q);
    return launch_status();
}

// Stack levels of a chunk of states, read from mapped host memory after the
// heights are on the device.  Level L of a cell is read by the kernels only
// when the cell's height exceeds L, so level L is fetched over the board rows
// r0..r1 that hold such a cell: bytes L*529 + 23*r0 up to L*529 + 23*(r1+1),
// widened to 16-byte words (the widening rewrites neighbouring bytes with the
// host's own values).  Other level bytes of dev are left as they were.
__global__ void __launch_bounds__(kThreads) k_stage_levels(const uint8_t* __restrict__ host, int64_t count,
                                                           uint8_t* __restrict__ dev) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < count; p += nwarps) {
        const uint8_t* h = dev + p * kStateBytes + kOffHeight;
        unsigned lo[5], hi[5];
#pragma unroll
        for (int t = 0; t < 5; t++) lo[t] = kBoard, hi[t] = 0;
        for (int c = l; c < kCells; c += 32) {
            const unsigned ht = h[c], r = c / kBoard;
#pragma unroll
            for (int t = 0; t < 5; t++)
                if (ht > (unsigned)t) lo[t] = min(lo[t], r), hi[t] = max(hi[t], r + 1);
        }
        const uint4* src = reinterpret_cast<const uint4*>(host + p * kStateBytes);
        uint4* dst = reinterpret_cast<uint4*>(dev + p * kStateBytes);
#pragma unroll
        for (int t = 0; t < 5; t++) {
            const unsigned r0 = __reduce_min_sync(kFull, lo[t]), r1 = __reduce_max_sync(kFull, hi[t]);
            if (r0 >= r1) break;  // no cell above level t, none above t + 1 either
            const int w0 = (t * kCells + (int)r0 * kBoard) >> 4, w1 = (t * kCells + (int)r1 * kBoard + 15) >> 4;
            for (int i = w0 + l; i < w1; i += 32) dst[i] = src[i];
        }
    }
}

// The moves of a chunk past its first `prefix` (a multiple of 8) of each
// position, written into mapped host memory: warp per position, 16-byte
// stores over bytes 6*prefix up to 6*n rounded up to 16 (the device rows are
// zero past n, so the rounding writes zeros over the host's zeroed tail).
__global__ void __launch_bounds__(kThreads) k_download_tail(const uint8_t* __restrict__ dev,
                                                            const int32_t* __restrict__ num_legal, int64_t count,
                                                            uint8_t* __restrict__ host, int prefix) {
    const int l = lane_id();
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); p < count; p += nwarps) {
        const int n = min(max(num_legal[p], 0), kMaxMoves);
        if (n <= prefix) continue;
        const int w0 = (prefix * kMoveBytes) >> 4, w1 = (n * kMoveBytes + 15) >> 4;
        const uint4* src = reinterpret_cast<const uint4*>(dev + p * (kMaxMoves * kMoveBytes));
        uint4* dst = reinterpret_cast<uint4*>(host + p * (kMaxMoves * kMoveBytes));
        for (int i = w0 + l; i < w1; i += 32) dst[i] = src[i];
    }
}

}  // namespace hv

using namespace hv;

extern "C" {

int hv_version(void) { return HV_ABI_VERSION; }

const char* hv_status_string(int status) {
    switch (status) {
        case HV_OK: return "ok";
        case HV_EINVAL: return "invalid argument (null, misaligned or negative size)";
        case HV_ECUDA: return "CUDA launch or runtime error";
        case HV_ENOMEM_TREE: return "tree node pool exhausted";
        case HV_ETIMEOUT: return "bounded device wait gave up";
        case HV_EDEVICE: return "device error word set (a generator buffer overflowed)";
        case HV_ESCRATCH:
            return "request exceeds the fixed 32 MiB scratch of hv_hybrid_evaluate_noalloc (at most 9137 positions)";
        default: return "unknown status";
    }
}

int hv_get_error(uint32_t* out, int clear) {
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, g_error, sizeof(v)) != cudaSuccess) return HV_ECUDA;
    if (out) *out = v;
    if (clear && v) {
        uint32_t z = 0;
        if (cudaMemcpyToSymbol(g_error, &z, sizeof(z)) != cudaSuccess) return HV_ECUDA;
    }
    return HV_OK;
}

int hv_set_wait_limit_ns(uint64_t ns) {
    if (cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)) != cudaSuccess) return HV_ECUDA;
    return HV_OK;
}

int hv_create_initial_states(uint8_t* states, int64_t batch, int expansion_mask, void* stream) {
    if (batch < 0 || (batch && (!states || !aligned16(states)))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    int grid = 0;
    int rc = grid_for(k_init_states, batch, 0, &grid);
    if (rc) return rc;
    k_init_states<<<grid, kThreads, 0, (cudaStream_t)stream>>>(states, batch, expansion_mask & 7);
    return launch_status();
}

int hv_generate_legal_moves(const uint8_t* states, int64_t batch, uint8_t* moves,
                            int32_t* num_legal, void* stream) {
    return launch_root<true, true, false>(states, nullptr, nullptr, batch, moves, num_legal,
                                          nullptr, stream);
}

// Two launches, not one fused kernel: the generator and the feature code
// together overflow the SM's instruction cache (instruction-fetch stalls
// lead the fused kernel's profile), while each alone fits.  Measured on
// 262,144 positions: fused 6.2 ms, generator 3.2 ms + features from the
// stored list 1.7 ms; re-reading the states and lists costs ~0.2 ms of HBM.
int hv_generate_legal_moves_linked(const uint8_t* states, int64_t batch, uint8_t* moves, int32_t* num_legal,
                                   float* features, void* stream) {
    if (batch > 0 && !features) return HV_EINVAL;
    // the feature rows carry the generator's articulation masks to the
    // feature launch, and row 0 the position counters of the generator
    // (bytes 8..15) and of the feature launch (16..23)
    if (batch > 0 && (reinterpret_cast<uintptr_t>(features) & 7) != 0) return HV_EINVAL;
    if (batch > 0 &&
        cudaMemsetAsync(features + 2, 0, 2 * sizeof(unsigned long long), (cudaStream_t)stream) != cudaSuccess)
        return HV_ECUDA;
    return launch_root<true, true, false, true>(states, nullptr, nullptr, batch, moves, num_legal, features, stream);
}

int hv_fnn_features_linked(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal, int64_t batch,
                           float* features, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch > 0 && (!features || (reinterpret_cast<uintptr_t>(features) & 7) != 0)) return HV_EINVAL;
    // positions 1.. claim from the counter in row 0; position 0 goes last
    if (batch > 1) {
        const int rc = launch_root<false, false, true, true, true>(states, moves, num_legal, batch, nullptr, nullptr,
                                                                   features, stream);
        if (rc) return rc;
    }
    return launch_root<false, false, true, true>(states, moves, num_legal, batch > 0 ? 1 : 0, nullptr, nullptr,
                                                 features, stream);
}

int hv_generate_legal_moves_and_fnn_features(const uint8_t* states, int64_t batch, uint8_t* moves,
                                             int32_t* num_legal, float* features, void* stream) {
    const int rc = hv_generate_legal_moves_linked(states, batch, moves, num_legal, features, stream);
    if (rc) return rc;
    return hv_fnn_features_linked(states, moves, num_legal, batch, features, stream);
}

int hv_stage_host_states(const uint8_t* host_states, int64_t count, uint8_t* dev_states, void* stream) {
    if (count < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!host_states || !dev_states) return HV_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    cudaPointerAttributes attr;
    const void* mapped = nullptr;
    // the level kernel moves 16-byte words: other alignments take the full copy
    if (aligned16(host_states) && aligned16(dev_states)) {
        if (cudaPointerGetAttributes(&attr, host_states) == cudaSuccess && attr.type == cudaMemoryTypeHost)
            mapped = attr.devicePointer;
        else
            cudaGetLastError();  // a pageable pointer is not an error here
    }
    if (!mapped) {
        if (cudaMemcpyAsync(dev_states, host_states, (size_t)count * kStateBytes, cudaMemcpyHostToDevice, s) !=
            cudaSuccess)
            return HV_ECUDA;
        return HV_OK;
    }
    // heights, bitboards and fields (bytes 2645..3423) of every state
    if (cudaMemcpy2DAsync(dev_states + kOffHeight, kStateBytes, host_states + kOffHeight, kStateBytes,
                          kStateBytes - kOffHeight, (size_t)count, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return HV_ECUDA;
    int grid = 0;
    int rc = grid_for(k_stage_levels, count, 0, &grid);
    if (rc) return rc;
    k_stage_levels<<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(mapped), count, dev_states);
    return launch_status();
}

int hv_download_moves(const uint8_t* dev_moves, const int32_t* dev_num_legal, int64_t count, uint8_t* host_moves,
                      int prefix, void* stream) {
    if (count < 0 || prefix < 0 || prefix > kMaxMoves || (prefix & 7)) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!dev_moves || !dev_num_legal || !host_moves) return HV_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    constexpr size_t kRow = (size_t)kMaxMoves * kMoveBytes;
    cudaPointerAttributes attr;
    uint8_t* mapped = nullptr;
    if (prefix < kMaxMoves && aligned16(dev_moves) && aligned16(host_moves)) {
        if (cudaPointerGetAttributes(&attr, host_moves) == cudaSuccess && attr.type == cudaMemoryTypeHost)
            mapped = static_cast<uint8_t*>(attr.devicePointer);
        else
            cudaGetLastError();  // a pageable pointer is not an error here
    }
    if (!mapped) {
        if (cudaMemcpyAsync(host_moves, dev_moves, (size_t)count * kRow, cudaMemcpyDeviceToHost, s) != cudaSuccess)
            return HV_ECUDA;
        return HV_OK;
    }
    if (prefix > 0 && cudaMemcpy2DAsync(host_moves, kRow, dev_moves, kRow, (size_t)prefix * kMoveBytes, (size_t)count,
                                         cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return HV_ECUDA;
    int grid = 0;
    int rc = grid_for(k_download_tail, count, 0, &grid);
    if (rc) return rc;
    k_download_tail<<<grid, kThreads, 0, s>>>(dev_moves, dev_num_legal, count, mapped, prefix);
    return launch_status();
}

int hv_extract_fnn_features(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                            int64_t batch, float* features, void* stream) {
    return launch_root<false, false, true>(states, moves, num_legal, batch, nullptr, nullptr,
                                           features, stream);
}

int hv_fnn_successor_features(const uint8_t* states, int64_t num_states, const uint8_t* legal_moves,
                              const int64_t* action_to_root, const int64_t* move_indices,
                              int64_t num_actions, float* features, void* stream) {
    if (num_actions < 0 || num_states < 0) return HV_EINVAL;
    if (num_actions == 0) return HV_OK;
    if (!states || !legal_moves || !action_to_root || !move_indices || !features ||
        !aligned16(states))
        return HV_EINVAL;
    size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_successor_features<kRowsF32>, num_actions, smem, &grid);
    if (rc) return rc;
    k_successor_features<kRowsF32><<<grid, kThreads, smem, (cudaStream_t)stream>>>(
        states, num_states, legal_moves, action_to_root, move_indices, num_actions, features, nullptr, nullptr);
    return launch_status();
}

int hv_fnn_eval_leaves(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                       const float* root_features, int64_t count, const float* weights, int hidden,
                       int embed, int action_hidden, float* priors, float* values, float* child_q,
                       float* logits, void* stream) {
    if (count < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!states || !legal_moves || !num_legal || !weights || !priors || !values || !child_q ||
        !aligned16(states) || !aligned16(legal_moves))
        return HV_EINVAL;
    if (hidden < 1 || hidden > kFnnMaxDim || embed < 1 || embed > kFnnMaxDim || action_hidden < 1 ||
        action_hidden > kFnnMaxDim)
        return HV_EINVAL;
    size_t smem = (sizeof(WarpSmem) + sizeof(FnnSmem)) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_fnn_eval, count, smem, &grid);
    if (rc) return rc;
    FnnDims d{hidden, embed, action_hidden};
    k_fnn_eval<<<grid, kThreads, smem, (cudaStream_t)stream>>>(states, legal_moves, num_legal,
                                                                root_features, count, weights, d,
                                                                priors, values, child_q, logits);
    return launch_status();
}

int hv_hybrid_encode(const uint8_t* states, int64_t batch, float* token_features, int32_t* token_q,
                     int32_t* token_r, int32_t* token_z, uint8_t* token_mask, float* global_features,
                     int32_t* num_tokens, void* stream) {
    HybridOut o{token_features, token_q, token_r, token_z, token_mask, global_features, num_tokens, nullptr};
    return launch_hybrid<false, true, false>(states, nullptr, nullptr, batch, nullptr, nullptr, nullptr, o, stream);
}

int hv_hybrid_move_features(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            int64_t batch, float* move_features, void* stream) {
    HybridOut o{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, move_features};
    return launch_hybrid<false, false, true>(states, legal_moves, num_legal, batch, nullptr, nullptr, nullptr, o,
                                             stream);
}

int hv_generate_legal_moves_and_hybrid_root_features(const uint8_t* states, int64_t batch, uint8_t* moves,
                                                     int32_t* num_legal, float* fnn_features, float* token_features,
                                                     int32_t* token_q, int32_t* token_r, int32_t* token_z,
                                                     uint8_t* token_mask, float* global_features,
                                                     int32_t* num_tokens, float* move_features, void* stream) {
    HybridOut o{token_features, token_q, token_r, token_z, token_mask, global_features, num_tokens, move_features};
    return launch_hybrid<true, true, true>(states, nullptr, nullptr, batch, moves, num_legal, fnn_features, o,
                                           stream);
}

int hv_hybrid_trunk_sizes(int* image_elems, int* param_floats) {
    if (!image_elems || !param_floats) return HV_EINVAL;
    *image_elems = kImgTp + kTrLayers * kImgLayer;
    *param_floats = kParLayer0 + kTrLayers * kLEnd;
    return HV_OK;
}

// the trunk over slots (slots NULL: one position per slot)
static int launch_trunk(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                        const int32_t* token_z, const uint8_t* token_mask, int64_t batch, int node_feat_dim,
                        const uint16_t* weight_image, const float* params, float* graph_summary,
                        const int2* slots, const int* slot_cnt, void* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HV_ECUDA;
    DeviceInfo& d = g_dev[dev];
    if (d.sms == 0 && cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return HV_ECUDA;
    const size_t smem = sizeof(TrunkSmem);
    if (cudaFuncSetAttribute(k_hybrid_trunk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return HV_ECUDA;
    const int64_t passes = (batch + kTrPos - 1) / kTrPos;
    const int grid = (int)(passes < d.sms ? passes : d.sms);
    uint32_t* err = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_error) != cudaSuccess) return HV_ECUDA;
    k_hybrid_trunk<<<grid, kTrThreads, smem, (cudaStream_t)stream>>>(
        token_features, token_q, token_r, token_z, token_mask, batch, node_feat_dim, slots, slot_cnt,
        reinterpret_cast<const __half*>(weight_image), params, graph_summary, err);
    return launch_status();
}

static bool trunk_args_ok(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                          const int32_t* token_z, const uint8_t* token_mask, int node_feat_dim,
                          const uint16_t* weight_image, const float* params, const float* graph_summary) {
    return token_features && token_q && token_r && token_z && token_mask && weight_image && params &&
           graph_summary && aligned16(weight_image) && aligned16(graph_summary) && node_feat_dim >= 1 &&
           node_feat_dim <= 27;
}

int hv_hybrid_trunk(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                    const int32_t* token_z, const uint8_t* token_mask, int64_t batch, int node_feat_dim,
                    const uint16_t* weight_image, const float* params, float* graph_summary, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (!trunk_args_ok(token_features, token_q, token_r, token_z, token_mask, node_feat_dim, weight_image, params,
                       graph_summary))
        return HV_EINVAL;
    return launch_trunk(token_features, token_q, token_r, token_z, token_mask, batch, node_feat_dim, weight_image,
                        params, graph_summary, nullptr, nullptr, stream);
}

int hv_hybrid_trunk_packed_workspace_bytes(int64_t batch, size_t* bytes) {
    if (batch < 0 || !bytes) return HV_EINVAL;
    *bytes = 16 + 8 * (size_t)batch;
    return HV_OK;
}

// the slot table, then the trunk over it (workspace: two counters, then the table)
static int trunk_packed(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                        const int32_t* token_z, const uint8_t* token_mask, int64_t batch, int node_feat_dim,
                        const uint16_t* weight_image, const float* params, float* graph_summary, void* ws,
                        void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    int* cnt = static_cast<int*>(ws);
    int2* slots = reinterpret_cast<int2*>(static_cast<uint8_t*>(ws) + 16);
    if (cudaMemsetAsync(cnt, 0, 16, s) != cudaSuccess ||
        cudaMemsetAsync(slots, 0xFF, 8 * (size_t)batch, s) != cudaSuccess)
        return HV_ECUDA;
    k_trunk_classify<<<(unsigned)((batch + 255) / 256), 256, 0, s>>>(token_mask, batch, slots, cnt);
    const int rc = launch_status();
    if (rc) return rc;
    return launch_trunk(token_features, token_q, token_r, token_z, token_mask, batch, node_feat_dim, weight_image,
                        params, graph_summary, slots, cnt, stream);
}

int hv_hybrid_trunk_packed(const float* token_features, const int32_t* token_q, const int32_t* token_r,
                           const int32_t* token_z, const uint8_t* token_mask, int64_t batch, int node_feat_dim,
                           const uint16_t* weight_image, const float* params, float* graph_summary, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (!trunk_args_ok(token_features, token_q, token_r, token_z, token_mask, node_feat_dim, weight_image, params,
                       graph_summary) ||
        !workspace || (reinterpret_cast<uintptr_t>(workspace) & 15) || workspace_bytes < 16 + 8 * (size_t)batch ||
        batch > INT32_MAX)
        return HV_EINVAL;
    return trunk_packed(token_features, token_q, token_r, token_z, token_mask, batch, node_feat_dim, weight_image,
                        params, graph_summary, workspace, stream);
}

// workspace of hv_hybrid_evaluate: per position tokens, coordinates, mask,
// global features, token count and the trunk's summary, each array 256-byte aligned
struct HybridWorkspace {
    float* tf;
    int32_t *tq, *tr, *tz;
    uint8_t* tm;
    float* gf;
    int32_t* ntok;
    float* graph;
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static size_t hybrid_workspace_layout(int64_t count, uint8_t* base, HybridWorkspace* w) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off += align256(bytes);
        return p;
    };
    const size_t n = (size_t)count;
    uint8_t* tf = take(n * kTokens * kTokFeat * sizeof(float));
    uint8_t* tq = take(n * kTokens * sizeof(int32_t));
    uint8_t* tr = take(n * kTokens * sizeof(int32_t));
    uint8_t* tz = take(n * kTokens * sizeof(int32_t));
    uint8_t* tm = take(n * kTokens);
    uint8_t* gf = take(n * kGlobFeat * sizeof(float));
    uint8_t* nt = take(n * sizeof(int32_t));
    uint8_t* gr = take(n * kHybGraph * sizeof(float));
    if (w) {
        w->tf = reinterpret_cast<float*>(tf);
        w->tq = reinterpret_cast<int32_t*>(tq);
        w->tr = reinterpret_cast<int32_t*>(tr);
        w->tz = reinterpret_cast<int32_t*>(tz);
        w->tm = tm;
        w->gf = reinterpret_cast<float*>(gf);
        w->ntok = reinterpret_cast<int32_t*>(nt);
        w->graph = reinterpret_cast<float*>(gr);
    }
    return off;
}

int hv_hybrid_workspace_bytes(int64_t count, size_t* bytes) {
    if (count < 0 || !bytes) return HV_EINVAL;
    *bytes = hybrid_workspace_layout(count, nullptr, nullptr);
    return HV_OK;
}

int hv_hybrid_evaluate(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                       const float* root_features, int64_t count, int node_feat_dim, const uint16_t* trunk_image,
                       const float* trunk_params, const float* fnn_weights, int hidden, int embed,
                       int action_hidden, const float* head_weights, int value_hidden, float* priors,
                       float* values, float* child_q, float* logits, void* workspace, size_t workspace_bytes,
                       void* stream) {
    if (count < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
        workspace_bytes < hybrid_workspace_layout(count, nullptr, nullptr))
        return HV_EINVAL;
    HybridWorkspace w;
    hybrid_workspace_layout(count, static_cast<uint8_t*>(workspace), &w);
    int rc = hv_hybrid_encode(states, count, w.tf, w.tq, w.tr, w.tz, w.tm, w.gf, w.ntok, stream);
    if (rc) return rc;
    rc = hv_hybrid_trunk(w.tf, w.tq, w.tr, w.tz, w.tm, count, node_feat_dim, trunk_image, trunk_params, w.graph,
                         stream);
    if (rc) return rc;
    return hv_hybrid_eval_leaves(states, legal_moves, num_legal, root_features, w.graph, w.gf, count, fnn_weights,
                                 hidden, embed, action_hidden, head_weights, value_hidden, priors, values, child_q,
                                 logits, stream);
}

// Fixed scratch of hv_hybrid_evaluate_noalloc: enough for 9137 positions in
// the hybrid_workspace_layout arrays.  Its address is resolved once per device
// context: a context that was destroyed and re-created (cudaDeviceReset) loads
// the module again, at a new address, so the cache is keyed on the context
// handle as well as the device index.
static __device__ __align__(256) uint8_t g_hybrid_scratch[32u << 20];
static void* g_hybrid_scratch_ptr[64];
static void* g_hybrid_scratch_ctx[64];
static std::mutex g_hybrid_scratch_mu;

// The current driver context (cuCtxGetCurrent through the runtime's entry-point
// query, so the library needs no link against libcuda).  nullptr if unknown.
static void* current_context() {
    typedef int (*CtxGetCurrent)(void**);
    static CtxGetCurrent fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<CtxGetCurrent>(f);
    }();
    void* ctx = nullptr;
    if (!fn || fn(&ctx) != 0) return nullptr;
    return ctx;
}

int hv_hybrid_evaluate_noalloc(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                               const float* root_features, int64_t count, int node_feat_dim,
                               const uint16_t* trunk_image, const float* trunk_params, const float* fnn_weights,
                               int hidden, int embed, int action_hidden, const float* head_weights,
                               int value_hidden, float* priors, float* values, float* child_q, float* logits,
                               void* stream) {
    if (count < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (hybrid_workspace_layout(count, nullptr, nullptr) > sizeof(g_hybrid_scratch)) return HV_ESCRATCH;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HV_ECUDA;
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_hybrid_scratch_mu);
        void* ctx = current_context();
        if (!g_hybrid_scratch_ptr[dev] || !ctx || ctx != g_hybrid_scratch_ctx[dev]) {
            // resolving the symbol makes the device's primary context current
            // when no context was, so the context is read again afterwards
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_hybrid_scratch) != cudaSuccess || !p) return HV_ECUDA;
            g_hybrid_scratch_ptr[dev] = p;
            g_hybrid_scratch_ctx[dev] = current_context();
        }
        scratch = g_hybrid_scratch_ptr[dev];
    }
    return hv_hybrid_evaluate(states, legal_moves, num_legal, root_features, count, node_feat_dim, trunk_image,
                              trunk_params, fnn_weights, hidden, embed, action_hidden, head_weights, value_hidden,
                              priors, values, child_q, logits, scratch, sizeof(g_hybrid_scratch), stream);
}

// ---- leaf evaluation as a row pipeline ------------------------------------

static size_t row_workspace_layout(int64_t count, int64_t rows, bool hybrid, bool own_logits, uint8_t* base,
                                   RowWorkspace* w) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off += align256(bytes);
        return p;
    };
    const size_t n = (size_t)count, r = (size_t)rows;
    uint8_t* rs = take((n + 1) * sizeof(int64_t));
    uint8_t* at = take(r * sizeof(int64_t));
    uint8_t* mi = take(r * sizeof(int64_t));
    const size_t rt = (r + 127) / 128 * 128;  // whole 128-row tiles
    uint8_t* x = hybrid ? nullptr : take(rt * 128 * sizeof(float));  // fp32 slab tiles
    uint8_t* xh = hybrid ? take(rt * 128 * 2) : nullptr;
    uint8_t* mf = hybrid ? take(rt * 32 * 2) : nullptr;
    uint8_t* rp = take(n * 64 * sizeof(float));
    uint8_t* lg = own_logits ? take(n * kMaxMoves * sizeof(float)) : nullptr;
    if (w) {
        w->row_start = reinterpret_cast<int64_t*>(rs);
        w->atr = reinterpret_cast<int64_t*>(at);
        w->mi = reinterpret_cast<int64_t*>(mi);
        w->x = reinterpret_cast<float*>(x);
        w->xh = reinterpret_cast<__half*>(xh);
        w->mfh = reinterpret_cast<__half*>(mf);
        w->root_pre = reinterpret_cast<float*>(rp);
        w->logits = reinterpret_cast<float*>(lg);
    }
    return off;
}

int hv_leaf_rows_workspace_bytes(int64_t count, int64_t rows, int hybrid, size_t* bytes) {
    if (count < 0 || rows < 0 || !bytes) return HV_EINVAL;
    *bytes = row_workspace_layout(count, rows, hybrid != 0, true, nullptr, nullptr);
    if (hybrid) *bytes += hybrid_workspace_layout(count, nullptr, nullptr) + align256(16 + 8 * (size_t)count);
    return HV_OK;
}

int hv_fnn_eval_leaves_rows(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            const float* root_features, int64_t count, int64_t rows, const float* weights,
                            int hidden, int embed, int action_hidden, float* priors, float* values, float* child_q,
                            float* logits, void* workspace, size_t workspace_bytes, void* stream) {
    if (count < 0 || rows < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!states || !legal_moves || !num_legal || !weights || !priors || !values || !child_q ||
        !aligned16(states) || !aligned16(legal_moves) || !workspace ||
        (reinterpret_cast<uintptr_t>(workspace) & 255))
        return HV_EINVAL;
    if (hidden < 1 || hidden > kFnnMaxDim || embed < 1 || embed > kFnnMaxDim || action_hidden < 1 ||
        action_hidden > kFnnMaxDim)
        return HV_EINVAL;
    if (workspace_bytes < row_workspace_layout(count, rows, false, logits == nullptr, nullptr, nullptr))
        return HV_EINVAL;
    RowWorkspace w;
    row_workspace_layout(count, rows, false, logits == nullptr, static_cast<uint8_t*>(workspace), &w);
    return run_row_pipeline<false>(states, legal_moves, num_legal, root_features, nullptr, nullptr, count, rows,
                                   weights, FnnDims{hidden, embed, action_hidden}, nullptr, HybDims{0, 0, 0}, priors,
                                   values, child_q, logits, w, (cudaStream_t)stream);
}

int hv_hybrid_evaluate_rows(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                            const float* root_features, int64_t count, int64_t rows, int node_feat_dim,
                            const uint16_t* trunk_image, const float* trunk_params, const float* fnn_weights,
                            int hidden, int embed, int action_hidden, const float* head_weights, int value_hidden,
                            float* priors, float* values, float* child_q, float* logits, void* workspace,
                            size_t workspace_bytes, void* stream) {
    if (count < 0 || rows < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!states || !legal_moves || !num_legal || !fnn_weights || !head_weights || !priors || !values ||
        !child_q || !aligned16(states) || !aligned16(legal_moves) || !workspace ||
        (reinterpret_cast<uintptr_t>(workspace) & 255))
        return HV_EINVAL;
    if (hidden < 1 || hidden > kFnnMaxDim || embed < 1 || embed > kFnnMaxDim || action_hidden < 1 ||
        action_hidden > kFnnMaxDim || value_hidden < 1 || value_hidden > kHybMaxValue || count > INT32_MAX ||
        !trunk_image || !trunk_params || !aligned16(trunk_image) || node_feat_dim < 1 || node_feat_dim > 27)
        return HV_EINVAL;
    // tokens and summary, then the row arrays, then the trunk's slot table
    const size_t tok_bytes = hybrid_workspace_layout(count, nullptr, nullptr);
    const size_t slot_at =
        tok_bytes + row_workspace_layout(count, rows, true, logits == nullptr, nullptr, nullptr);
    if (workspace_bytes < slot_at + 16 + 8 * (size_t)count) return HV_EINVAL;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    HybridWorkspace hw;
    hybrid_workspace_layout(count, ws, &hw);
    RowWorkspace w;
    row_workspace_layout(count, rows, true, logits == nullptr, ws + tok_bytes, &w);
    int rc = hv_hybrid_encode(states, count, hw.tf, hw.tq, hw.tr, hw.tz, hw.tm, hw.gf, hw.ntok, stream);
    if (rc) return rc;
    // early-game leaves have few tokens: the packed trunk pairs them two to a slot
    rc = trunk_packed(hw.tf, hw.tq, hw.tr, hw.tz, hw.tm, count, node_feat_dim, trunk_image, trunk_params, hw.graph,
                      ws + slot_at, stream);
    if (rc) return rc;
    return run_row_pipeline<true>(states, legal_moves, num_legal, root_features, hw.graph, hw.gf, count, rows,
                                  fnn_weights, FnnDims{hidden, embed, action_hidden}, head_weights,
                                  HybDims{embed, action_hidden, value_hidden}, priors, values, child_q, logits, w,
                                  (cudaStream_t)stream);
}

int hv_root_tactical_probe(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                           const float* priors, int64_t batch, int enable_win_in_one,
                           int enable_check_opponent_wins, int enable_win_in_two, int64_t* winning_move,
                           uint8_t* allowed_slots, uint8_t* forced_random, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (!states || !legal_moves || !num_legal || !priors || !winning_move || !allowed_slots ||
        !forced_random || !aligned16(states))
        return HV_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t want = (batch + kWarpsPerBlock - 1) / kWarpsPerBlock;
    const int root_grid = (int)(want < 4096 ? want : 4096);  // warp-per-root passes stride the rest
    k_tac_flags<<<root_grid, kThreads, 0, s>>>(states, num_legal, batch, enable_win_in_one != 0,
                                              enable_check_opponent_wins != 0, enable_win_in_two != 0,
                                              winning_move, allowed_slots, forced_random);
    if (enable_win_in_one || enable_check_opponent_wins) {
        size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
        int grid = 0;
        int rc = grid_for(k_tac_children, batch * kMaxMoves, smem, &grid);
        if (rc) return rc;
        k_tac_children<<<grid, kThreads, smem, s>>>(states, legal_moves, num_legal, batch, forced_random,
                                                   allowed_slots);
        k_tac_decide<<<root_grid, kThreads, 0, s>>>(num_legal, priors, batch, winning_move, allowed_slots,
                                                   forced_random);
    }
    if (enable_win_in_two) {
        size_t smem = (sizeof(WarpSmem) + sizeof(TacSmem)) * kWarpsPerBlock;
        int grid = 0;
        int rc = grid_for(k_tac_win2, batch * kMaxMoves, smem, &grid);
        if (rc) return rc;
        k_tac_win2<<<grid, kThreads, smem, s>>>(states, legal_moves, num_legal, batch, forced_random,
                                               allowed_slots);
    }
    k_tac_final<<<root_grid, kThreads, 0, s>>>(num_legal, batch, winning_move, allowed_slots, forced_random);
    return launch_status();
}

int hv_hybrid_head_weights_size(int embed, int action_hidden, int value_hidden) {
    return hyb_offsets(HybDims{embed, action_hidden, value_hidden}).total;
}

int hv_hybrid_eval_leaves(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                          const float* root_features, const float* graph_summary, const float* global_features,
                          int64_t count, const float* fnn_weights, int hidden, int embed, int action_hidden,
                          const float* head_weights, int value_hidden, float* priors, float* values,
                          float* child_q, float* logits, void* stream) {
    if (count < 0) return HV_EINVAL;
    if (count == 0) return HV_OK;
    if (!states || !legal_moves || !num_legal || !graph_summary || !global_features || !fnn_weights ||
        !head_weights || !priors || !values || !child_q || !aligned16(states) || !aligned16(legal_moves))
        return HV_EINVAL;
    if (hidden < 1 || hidden > kFnnMaxDim || embed < 1 || embed > kFnnMaxDim || action_hidden < 1 ||
        action_hidden > kFnnMaxDim || value_hidden < 1 || value_hidden > kHybMaxValue)
        return HV_EINVAL;
    size_t smem = (sizeof(WarpSmem) + sizeof(FnnSmem) + sizeof(HybSmem)) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_hybrid_eval, count, smem, &grid);
    if (rc) return rc;
    k_hybrid_eval<<<grid, kThreads, smem, (cudaStream_t)stream>>>(
        states, legal_moves, num_legal, root_features, graph_summary, global_features, count, fnn_weights,
        FnnDims{hidden, embed, action_hidden}, head_weights, HybDims{embed, action_hidden, value_hidden}, priors,
        values, child_q, logits);
    return launch_status();
}

int hv_fnn_weights_size(int hidden, int embed, int action_hidden) {
    return fnn_offsets(FnnDims{hidden, embed, action_hidden}).total;
}

static bool tree_ok(const hv_tree* t) {
    return t && t->visit_count && t->total_value && t->prior && t->parent_idx && t->virtual_q_penalty &&
           t->move_bytes && t->action_idx && t->first_child && t->num_children && t->is_terminal &&
           t->terminal_value && t->node_count && t->max_nodes > 0;
}

static TreeDev tree_dev(const hv_tree* t) {
    return TreeDev{t->visit_count, t->total_value, t->prior, t->parent_idx, t->virtual_q_penalty,
                   t->move_bytes, t->action_idx, t->first_child, t->num_children, t->is_terminal,
                   t->terminal_value, t->node_count, t->max_nodes};
}

static int game_grid(int B) { return (B + kWarpsPerBlock - 1) / kWarpsPerBlock; }

int hv_mcts_select(const hv_tree* tree, int mode, const float* child_init_q, const int8_t* game_active,
                   const int32_t* root_nodes, const int8_t* alive_mask, const int32_t* root_slots,
                   int num_candidates, int max_root_children, float c_puct, int B, int W,
                   int deterministic_non_root, float non_root_sigma, float q_penalty, int32_t* leaf,
                   uint8_t* move_paths, int32_t* path_len, int32_t* vl_paths, int32_t* vl_len,
                   void* stream) {
    if (!tree_ok(tree) || mode < 0 || mode > 2 || B < 0 || W < 0) return HV_EINVAL;
    if (mode == 2 && num_candidates < 1) return HV_EINVAL;
    const int total = mode == 2 ? W * num_candidates * B : W * B;
    if (total == 0) return HV_OK;
    if (!game_active || !root_nodes || !leaf || !move_paths || !path_len || !vl_paths || !vl_len)
        return HV_EINVAL;
    if ((mode == 1 && !alive_mask) || (mode == 2 && !root_slots)) return HV_EINVAL;
    if (deterministic_non_root && mode != 0 && !child_init_q) return HV_EINVAL;
    SelectArgs a{mode, child_init_q, game_active, root_nodes, alive_mask, root_slots, num_candidates,
                 max_root_children, c_puct, B, total, deterministic_non_root, non_root_sigma,
                 q_penalty, leaf, move_paths, path_len, vl_paths, vl_len};
    if (mode == 2 && num_candidates <= 32)  // candidates' subtrees are disjoint: a warp each
        k_mcts_select_slots<<<game_grid(B * num_candidates), kThreads, 0, (cudaStream_t)stream>>>(tree_dev(tree), a);
    else if (mode != 2 && total / B <= 4096)  // root steps in order, then the root children's subtrees in parallel
        k_mcts_select_tree<<<B, kTreeThreads, 2 * sizeof(int32_t) * (total / B), (cudaStream_t)stream>>>(
            tree_dev(tree), a);
    else
        k_mcts_select<<<game_grid(B), kThreads, 0, (cudaStream_t)stream>>>(tree_dev(tree), a);
    return launch_status();
}

int hv_mcts_replay(const uint8_t* root_states, uint8_t* leaf_states, const uint8_t* move_paths,
                   const int32_t* path_len, const int32_t* leaf, int B, int total, void* stream) {
    if (B <= 0 || total < 0) return total == 0 ? HV_OK : HV_EINVAL;
    if (total == 0) return HV_OK;
    if (!root_states || !leaf_states || !move_paths || !path_len || !leaf || !aligned16(root_states) ||
        !aligned16(leaf_states))
        return HV_EINVAL;
    size_t smem = (size_t)kStateBytes * kWarpsPerBlock;
    int grid = (total + kWarpsPerBlock - 1) / kWarpsPerBlock;
    k_mcts_replay<<<grid, kThreads, smem, (cudaStream_t)stream>>>(root_states, leaf_states, move_paths,
                                                                  path_len, leaf, B, total);
    return launch_status();
}

int hv_mcts_expand(const hv_tree* tree, int dense, int backprop, float* child_init_q,
                   const float* child_q, const int32_t* leaf, const uint8_t* leaf_states,
                   const uint8_t* legal_moves, const int32_t* num_legal, const float* priors,
                   const int32_t* results, const float* values, const int32_t* vl_paths,
                   const int32_t* vl_len, int8_t* was_expanded, float q_penalty, int B, int total,
                   void* stream) {
    if (!tree_ok(tree) || B < 0 || total < 0) return HV_EINVAL;
    if (total == 0 || B == 0) return HV_OK;
    if (!leaf || !leaf_states || !legal_moves || !num_legal || !priors || !results) return HV_EINVAL;
    if (dense && (!child_init_q || !child_q)) return HV_EINVAL;
    if (backprop && (!values || !vl_paths || !vl_len)) return HV_EINVAL;
    ExpandArgs a{dense, backprop, child_init_q, child_q, leaf, leaf_states, legal_moves, num_legal,
                 priors, results, values, vl_paths, vl_len, was_expanded, q_penalty, B, total};
    k_mcts_expand<<<game_grid(B), kThreads, 0, (cudaStream_t)stream>>>(tree_dev(tree), a);
    return launch_status();
}

int hv_mcts_expand_slots(const hv_tree* tree, float* child_init_q, const float* child_q, const int32_t* leaf,
                         const uint8_t* leaf_states, const uint8_t* legal_moves, const int32_t* num_legal,
                         const float* priors, const int32_t* results, const float* values,
                         const int32_t* vl_paths, const int32_t* vl_len, const int32_t* root_nodes,
                         const int32_t* root_slots, int num_candidates, float q_penalty, int B, int total,
                         void* stream) {
    if (!tree_ok(tree) || B < 0 || total < 0 || (root_slots && num_candidates < 1)) return HV_EINVAL;
    if (total == 0 || B == 0) return HV_OK;
    if (!leaf || !leaf_states || !legal_moves || !num_legal || !priors || !results || !child_init_q ||
        !child_q || !values || !vl_paths || !vl_len || !root_nodes)
        return HV_EINVAL;
    ExpandArgs a{1, 1, child_init_q, child_q, leaf, leaf_states, legal_moves, num_legal, priors, results,
                 values, vl_paths, vl_len, nullptr, q_penalty, B, total};
    const int64_t per = total / B;
    const bool shape_ok = root_slots ? (num_candidates <= 32 && total % ((int64_t)B * num_candidates) == 0)
                                     : total % B == 0;
    if (!shape_ok || per > 1024) {
        // outside the parallel form's shape: the per-game kernel, same results
        k_mcts_expand<<<game_grid(B), kThreads, 0, (cudaStream_t)stream>>>(tree_dev(tree), a);
        return launch_status();
    }
    k_mcts_expand_slots<<<B, root_slots ? 32 * num_candidates : kTreeThreads, 7 * sizeof(int32_t) * per,
                          (cudaStream_t)stream>>>(tree_dev(tree), a, root_nodes, root_slots, num_candidates);
    return launch_status();
}

int hv_mcts_backprop(const hv_tree* tree, const int32_t* leaf, const float* values,
                     const int32_t* vl_paths, const int32_t* vl_len, const int8_t* was_expanded, int B,
                     int total, void* stream) {
    if (!tree_ok(tree) || B < 0 || total < 0) return HV_EINVAL;
    if (total == 0 || B == 0) return HV_OK;
    if (!leaf || !values || !vl_paths || !vl_len || !was_expanded) return HV_EINVAL;
    k_mcts_backprop<<<game_grid(B), kThreads, 0, (cudaStream_t)stream>>>(tree_dev(tree), leaf, values,
                                                                         vl_paths, vl_len,
                                                                         was_expanded, B, total);
    return launch_status();
}

int hv_mcts_root_noise(const hv_tree* tree, const float* noise, const int32_t* root_nodes,
                       int max_children_pad, float dir_eps, float root_policy_temp, int B,
                       void* stream) {
    if (!tree_ok(tree) || B < 0) return HV_EINVAL;
    if (B == 0) return HV_OK;
    if (!root_nodes || (dir_eps > 0.0f && !noise)) return HV_EINVAL;
    k_mcts_root_noise<<<(B + 127) / 128, 128, 0, (cudaStream_t)stream>>>(
        tree_dev(tree), noise, root_nodes, max_children_pad, dir_eps, root_policy_temp, B);
    return launch_status();
}

int hv_mcts_extract_policy(const hv_tree* tree, float* policies, const int32_t* move_numbers,
                           const int32_t* root_nodes, float temperature, int temp_drop_move,
                           float pruning_threshold, int B, void* stream) {
    if (!tree_ok(tree) || B < 0) return HV_EINVAL;
    if (B == 0) return HV_OK;
    if (!policies || !move_numbers || !root_nodes) return HV_EINVAL;
    k_mcts_extract_policy<<<(B + 127) / 128, 128, 0, (cudaStream_t)stream>>>(
        tree_dev(tree), policies, move_numbers, root_nodes, temperature, temp_drop_move,
        pruning_threshold, B);
    return launch_status();
}

int hv_queen_escape_flags(const uint8_t* states, int64_t batch, uint8_t* flags, void* stream) {
    if (batch < 0 || (batch && (!states || !flags || !aligned16(states)))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_queen_escape, batch, smem, &grid);
    if (rc) return rc;
    k_queen_escape<<<grid, kThreads, smem, (cudaStream_t)stream>>>(states, batch, flags);
    return launch_status();
}

int hv_child_probe(const uint8_t* states, const uint8_t* legal_moves, const int32_t* num_legal,
                   int64_t batch, int want_escape, int32_t* results, int32_t* surround,
                   uint8_t* escape, void* stream) {
    if (batch < 0) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (!states || !legal_moves || !num_legal || !results || !surround || !aligned16(states) ||
        (want_escape && !escape))
        return HV_EINVAL;
    size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_child_probe, batch, smem, &grid);
    if (rc) return rc;
    k_child_probe<<<grid, kThreads, smem, (cudaStream_t)stream>>>(
        states, legal_moves, num_legal, batch, want_escape, results, surround, escape);
    return launch_status();
}

int hv_apply_moves(uint8_t* states, const uint8_t* moves, int64_t batch, void* stream) {
    if (batch < 0 || (batch && (!states || !moves || !aligned16(states)))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    int blocks = (int)((batch + 255) / 256);
    k_apply_moves<<<blocks, 256, 0, (cudaStream_t)stream>>>(states, moves, batch);
    return launch_status();
}

int hv_check_results(const uint8_t* states, int64_t batch, int32_t* results, void* stream) {
    if (batch < 0 || (batch && (!states || !results))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    int blocks = (int)((batch + 255) / 256);
    k_check_results<<<blocks, 256, 0, (cudaStream_t)stream>>>(states, batch, results);
    return launch_status();
}

int hv_compute_centroids(const uint8_t* states, int64_t batch, int32_t* centroids, void* stream) {
    if (batch < 0 || (batch && (!states || !centroids))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    int grid = 0;
    int rc = grid_for(k_actions, batch, 0, &grid);
    if (rc) return rc;
    k_actions<<<grid, kThreads, 0, (cudaStream_t)stream>>>(states, nullptr, nullptr, batch, nullptr,
                                                            centroids, nullptr);
    return launch_status();
}

int hv_legal_moves_to_actions(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal,
                              int64_t batch, int32_t* actions, void* stream) {
    if (batch < 0 || (batch && (!states || !moves || !num_legal || !actions))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    int grid = 0;
    int rc = grid_for(k_actions, batch, 0, &grid);
    if (rc) return rc;
    k_actions<<<grid, kThreads, 0, (cudaStream_t)stream>>>(states, moves, num_legal, batch, actions,
                                                            nullptr, nullptr);
    return launch_status();
}

int hv_legal_mask(const uint8_t* states, const uint8_t* moves, const int32_t* num_legal, int64_t batch,
                  float* masks, void* stream) {
    if (batch < 0 || (batch && (!states || !moves || !num_legal || !masks))) return HV_EINVAL;
    if (batch == 0) return HV_OK;
    if (reinterpret_cast<uintptr_t>(masks) & 7) return HV_EINVAL;
    int grid = 0;
    int rc = grid_for(k_actions, batch, 0, &grid);
    if (rc) return rc;
    k_actions<<<grid, kThreads, 0, (cudaStream_t)stream>>>(states, moves, num_legal, batch, nullptr, nullptr,
                                                            masks);
    return launch_status();
}

int hv_generate_positions(uint64_t seed, int64_t first_game, int64_t count, int max_ply,
                          int expansion_mask, uint8_t* states, void* stream) {
    if (count < 0 || max_ply < 0 || (count && (!states || !aligned16(states)))) return HV_EINVAL;
    if (count == 0) return HV_OK;
    size_t smem = sizeof(WarpSmem) * kWarpsPerBlock;
    int grid = 0;
    int rc = grid_for(k_playouts, count, smem, &grid);
    if (rc) return rc;
    k_playouts<<<grid, kThreads, smem, (cudaStream_t)stream>>>(seed, first_game, count, max_ply,
                                                                expansion_mask & 7, states);
    return launch_status();
}

}  // extern "C"
