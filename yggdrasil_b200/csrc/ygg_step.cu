// The int8 decode step and the fused scoring loop of Yggdrasil on sm_100a.
//
// One warp serves one stream; lane l owns the C = n/32 state coordinates [C l, C l + C) of every layer (layout in
// ygg_model.h). Per layer the warp
//   1. computes rho from the new state of the layer below (exact int32 sum of squares, then the reference's f32 ops),
//   2. descends the router LOOK = 3 levels per round of loads: the 7 rows of the 3-level subtree under the current
//      node are fetched together (16-byte lanes, n/16 lanes per row), their dots reduced within the row's lanes and
//      compared in f32 with the thresholds of (token, node), so D dependent levels cost ceil(D / 3) L2 round trips,
//   3. takes a leaf slot from the block's pool (a slot is held only from the copy to the readout, a small part of a
//      layer's time, so a block runs more warps than it has slots) and has lane 0 issue one bulk copy
//      (cp.async.bulk, the 1-D TMA, no multicast) of the chosen expert's record and one of its table row into it,
//      completing on the slot's mbarrier,
//   4. meanwhile computes the layer input zl (lane k: the dot of down-projection row k with the state below),
//   5. waits on the mbarrier (bounded: it gives up after ~1 s with an error status instead of hanging),
//   6. runs the block-diagonal int16 x int8 transition (__dp2a), the table / factored input and the layer input in
//      int32, saturates to the new int8 state and stores it,
//   7. reads out z = P_r q (per-row partials + redux.sync), releases the slot, quantises zq, and adds f32(Q zq) * s
//      to the logits each lane holds in registers for its classes 32 m + lane.
// Every f32 operation is the reference's, single-rounded and in the reference's order (__fmul_rn / __fadd_rn /
// __fsqrt_rn / __fdiv_rn; no contraction), and f32 -> int32 rounds half to even with the x86 out-of-range value, so
// routes, int32 accumulators, states and logits equal cpu/ygg.cpp bit for bit.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ygg_device.cuh"

namespace ygg {

// blocks of 8 warps per SM the register budget is sized for: 4 (64 registers a thread) for n <= 128; n = 256 needs
// more registers per lane (8 coordinates) and runs 2 blocks
template <int N> constexpr int blocks_per_sm() { return N >= 256 ? 2 : 4; }

// ------------------------------------------------------------------------------------------------ shared memory

// Block layout: [S slots][S mbarriers][S owners][S phases] pad 128, then [W warp scratch][W states (score only)].
// A slot holds one expert record and one table row; the warp scratch holds the old state of the current layer, the
// new state of the layer below, the layer-input codes and the readout codes.
struct Pool {
    uint8_t *slots;
    uint32_t slot_bytes;
    uint32_t bars;     // shared address of mbarrier 0
    int *owner;        // -1 free, else the owning warp
    int *phase;        // parity of the slot's mbarrier to wait for next
    int S;
};
struct Scratch {
    int8_t *qold, *qb, *zl, *zq;
};

__host__ __device__ constexpr uint32_t pool_slot_bytes(uint32_t rec_max, int n) { return (rec_max + 2 * n + 127) / 128 * 128; }
__host__ __device__ constexpr uint32_t pool_meta_bytes(int S) { return (16u * S + 127) / 128 * 128; }
__host__ __device__ constexpr uint32_t scratch_bytes(int n) { return (2 * n + 64 + 32 + 127) / 128 * 128; }
__host__ __device__ constexpr uint32_t block_smem(uint32_t rec_max, int n, int S, int W, int state_bytes) {
    return S * pool_slot_bytes(rec_max, n) + pool_meta_bytes(S) + W * (scratch_bytes(n) + state_bytes);
}

// Lane 0 claims a free slot (CAS on its owner word, starting from the warp's home slot); -1 after ~1 s without one.
__device__ __forceinline__ int slot_claim(const Pool &p, int home, int warp) {
    const long long t0 = clock64();
    int i = home;
    while (true) {
        if (atomicCAS(p.owner + i, -1, warp) == -1) break;
        if (++i == p.S) {
            i = 0;
            if (clock64() - t0 > kWaitCycles) return -1;
            __nanosleep(32);
        }
    }
    __threadfence_block();
    return i;
}

struct StepOut {
    float *logits;      // [V] of this stream, or null
    int32_t *routes;    // [L] or null
    int32_t *acc;       // [L][n] or null
};

// What a token's layers share: the block's pool and the warp's scratch, the token, the state pointers (qstride
// coordinates per layer; qlane: this lane's coordinates exist there), the debug outputs and the new state of the
// layer below (carried from one layer to the next).
template <int C>
struct TokenCtx {
    const DevModel &m;
    const Pool &pool;
    const Scratch &sc;
    int home, warp, lane, x;
    const int8_t *q_in;
    int8_t *q_out;
    int qstride;
    bool qlane;
    const StepOut &dbg;
    LaneQ<C> qbelow;
};

// Layer l of a token (cpu/ygg.cpp:443-458). Returns false if a bounded wait gave up. Always inlined: the warp
// collectives in it (shuffles, ballots, redux) rely on the caller's converged warp.
template <int N, int BLK, int R, int R2T, int NVT>
__device__ __forceinline__ bool layer_step(TokenCtx<N / 32> &t, const int l, float (&lg)[kMaxClassesPerLane]) {
    constexpr int C = N / 32;
    const DevModel &m = t.m;
    const Pool &pool = t.pool;
    const Scratch &sc = t.sc;
    const int lane = t.lane, x = t.x, home = t.home, warp = t.warp;
    const int E = m.E, D = m.D;
    const int nv = NVT ? NVT : m.VP / 32;
    const int8_t *q_in = t.q_in;
    int8_t *q_out = t.q_out;
    const int qstride = t.qstride;
    const bool qlane = t.qlane;
    const StepOut &dbg = t.dbg;
    LaneQ<C> &qbelow = t.qbelow;
    const DevLayer &y = m.layer[l];
    LaneQ<C> qold = {};
    if (qlane) qold = load_q<C>(q_in + (size_t)l * qstride + C * lane);
    int r = x;
    float rho = 0.0f;
    const bool low = l > 0 && (R2T > 0 || m.R2 > 0);
    if (l > 0) {
        rho = rms_rho<N>(qbelow, y.r2b, y.rms_eps, m.inv_n);
        store_q<C>(sc.qb + C * lane, qbelow);
        __syncwarp();
        const uint4 qrow = *(const uint4 *)(sc.qb + 16 * (lane % (N / 16)));
        r = route_look<N>(y.w, y.thr + (size_t)x * E, D, qrow, rho, lane) - E;
    }
    // -- lane 0 claims a slot and issues the bulk copies of the expert record and its table row into it; the
    // slot index and the parity to wait for reach the other lanes in one shuffle
    const uint32_t rec_bytes = y.rec_bytes;
    const bool has_table = y.table != nullptr;
    int tag = -1;
    if (lane == 0) {
        const int slot = slot_claim(pool, home, warp);
        if (slot >= 0) {
            uint8_t *rec = pool.slots + (size_t)slot * pool.slot_bytes;
            const uint32_t bar = pool.bars + 8u * slot;
            fence_proxy_async();
            mbar_expect_tx(bar, rec_bytes + (has_table ? 2u * N : 0u));
            bulk_g2s(smem_addr(rec), y.rec + (size_t)r * rec_bytes, rec_bytes, bar);
            if (has_table) {
                const int16_t *src = y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N;
                bulk_g2s(smem_addr(rec + pool.slot_bytes - 2 * N), src, 2u * N, bar);
            }
            tag = 2 * slot + pool.phase[slot];
        }
    }
    tag = __shfl_sync(kFull, tag, 0);
    if (tag < 0) return false;
    const int slot = tag >> 1;
    const uint32_t parity = (uint32_t)(tag & 1);
    const uint8_t *rec = pool.slots + (size_t)slot * pool.slot_bytes;
    const int16_t *trow = (const int16_t *)(rec + (pool.slot_bytes - 2 * N));
    const uint32_t bar = pool.bars + 8u * slot;
    // -- layer input codes while the copy is in flight (cpu/ygg.cpp:285-296)
    if (low) layer_input_codes<N, R2T>(m, y, sc.qb, rho, sc.zl, lane);
    store_q<C>(sc.qold + C * lane, qold);
    __syncwarp();
    if (!__all_sync(kFull, mbar_wait_bounded(bar, parity))) return false;

    int acc[C];
    LaneQ<C> qn;
    leaf_update<N, BLK, R2T>(m, y, rec, has_table ? trow : nullptr, x, sc.qold, sc.zl, low, lane, acc, qn);
    if (m.ns < N && C * lane >= m.ns) {   // padding of a narrower model: held at exactly 0
#pragma unroll
        for (int i = 0; i < (C >= 4 ? C / 4 : 1); i++) qn.w[i] = 0;
#pragma unroll
        for (int ii = 0; ii < C; ii++) acc[ii] = 0;
    }
    if (qlane) store_q<C>(q_out + (size_t)l * qstride + C * lane, qn);
    if (dbg.routes != nullptr && lane == 0) dbg.routes[l] = r;
    if (dbg.acc != nullptr && qlane) {
#pragma unroll
        for (int ii = 0; ii < C; ii++) dbg.acc[(size_t)l * qstride + C * lane + ii] = acc[ii];
    }
    const ReadoutWords<N, R> ro = load_readout<N, R>(y, rec, lane);
    // the slot is free once its bytes are in registers: flip its parity and hand it back
    __syncwarp();
    if (lane == 0) {
        pool.phase[slot] = (int)(parity ^ 1u);
        __threadfence_block();
        atomicExch(pool.owner + slot, -1);
    }
    const int zq = readout_code<N, R>(ro, qn, lane);
    if (lane < R) sc.zq[lane] = (int8_t)zq;
    __syncwarp();
    head_accumulate<R, NVT>(m, y, sc.zq, lg, lane);
    qbelow = qn;
    __syncwarp();
    return true;
}

// One token of one stream through every layer. q_in / q_out: the stream's state [L][qstride] (global memory in the
// caller's layout, qstride = the model's ns, or shared memory in the device layout, qstride = n; they may alias).
// lg: the logits of the lane's classes (out). Returns false if a bounded wait gave up.
// Compile-time shape where a fast instance fixes it (0: read from the model at run time): R2T the padded layer-input
// rank, LT the number of layers, NVT the classes per lane (VP / 32).
template <int N, int BLK, int R, int R2T, int LT, int NVT>
__device__ __forceinline__ bool token_step(const DevModel &m, const Pool &pool, const Scratch &sc, int home, int warp,
                                           int x, const int8_t *q_in, int8_t *q_out, int qstride,
                                           float (&lg)[kMaxClassesPerLane], const StepOut &dbg, int lane) {
    const int V = m.V;
    const int nv = NVT ? NVT : m.VP / 32;
#pragma unroll
    for (int c = 0; c < kMaxClassesPerLane; c++) lg[c] = c < nv ? __ldg(m.head_b + 32 * c + lane) : 0.0f;
    TokenCtx<N / 32> t{m, pool, sc, home, warp, lane, x, q_in, q_out, qstride, (N / 32) * lane < qstride, dbg, {}};
    if constexpr (LT > 0) {
        // not unrolled: an unrolled layer loop with its early exits defeats the compiler's proof that the warp is
        // converged at the collectives, and each shuffle / ballot / redux then pays a re-convergence loop
#pragma unroll 1
        for (int l = 0; l < LT; l++)
            if (!layer_step<N, BLK, R, R2T, NVT>(t, l, lg)) return false;
    } else {
#pragma unroll 1
        for (int l = 0; l < m.L; l++)
            if (!layer_step<N, BLK, R, R2T, NVT>(t, l, lg)) return false;
    }
    if (dbg.logits != nullptr) {
#pragma unroll
        for (int c = 0; c < kMaxClassesPerLane; c++) {
            const int cls = 32 * c + lane;
            if (c < nv && cls < V) dbg.logits[cls] = lg[c];
        }
    }
    return true;
}

// ------------------------------------------------------------------------------------------------ kernels

// Pool and scratch of this block; the first warp initialises the slots' mbarriers and owners.
__device__ __forceinline__ void block_init(uint8_t *smem, uint32_t rec_max, int n, int S, int state_bytes, int warp,
                                           int lane, Pool &pool, Scratch &sc, int8_t *&state) {
    pool.slot_bytes = pool_slot_bytes(rec_max, n);
    pool.slots = smem;
    uint8_t *meta = smem + (size_t)S * pool.slot_bytes;
    pool.bars = smem_addr(meta);
    pool.owner = (int *)(meta + 8 * S);
    pool.phase = (int *)(meta + 12 * S);
    pool.S = S;
    uint8_t *ws = meta + pool_meta_bytes(S) + (size_t)warp * (scratch_bytes(n) + state_bytes);
    sc.qold = (int8_t *)ws;
    sc.qb = sc.qold + n;
    sc.zl = sc.qb + n;
    sc.zq = sc.zl + 64;
    state = (int8_t *)(ws + scratch_bytes(n));
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(pool.bars + 8u * i, 1);
            pool.owner[i] = -1;
            pool.phase[i] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();
}

template <int N, int BLK, int R, int R2T, int LT, int NVT>
__global__ void __launch_bounds__(256, blocks_per_sm<N>()) step_kernel(const __grid_constant__ DevModel m, int B,
                                                   const int32_t *__restrict__ tokens, const int8_t *state_in,
                                                   int8_t *state_out, float *__restrict__ logits,
                                                   int32_t *__restrict__ routes, int32_t *__restrict__ acc_out,
                                                   uint32_t rec_max, int S) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    Pool pool;
    Scratch sc;
    int8_t *unused;
    block_init(smem, rec_max, N, S, 0, warp, lane, pool, sc, unused);
    const int home = warp % S;
    const int L = m.L, V = m.V, ns = m.ns;
    for (int s = blockIdx.x * W + warp; s < B; s += gridDim.x * W) {
        const int x = tokens[s];
        if (x < 0 || x >= V) {   // cpu/ygg.cpp:493-495 rejects the whole input; here the stream is skipped
            if (lane == 0) atomicOr(m.status, kStatusBadToken);
            if (logits != nullptr)
                for (int c = lane; c < V; c += 32) logits[(size_t)s * V + c] = __int_as_float(0x7fc00000);
            if (state_out != state_in)
                for (int i = lane; i < L * ns; i += 32) state_out[(size_t)s * L * ns + i] = state_in[(size_t)s * L * ns + i];
            if (routes != nullptr && lane < L) routes[(size_t)s * L + lane] = -1;
            continue;
        }
        float lg[kMaxClassesPerLane];
        StepOut o{logits ? logits + (size_t)s * V : nullptr, routes ? routes + (size_t)s * L : nullptr,
                  acc_out ? acc_out + (size_t)s * L * ns : nullptr};
        if (!token_step<N, BLK, R, R2T, LT, NVT>(m, pool, sc, home, warp, x, state_in + (size_t)s * L * ns,
                                                 state_out + (size_t)s * L * ns, ns, lg, o, lane)) {
            if (lane == 0) atomicOr(m.status, kStatusTimeout);
            return;
        }
    }
}

// Rows of `steps` tokens; the state of a row lives in the warp's shared memory between tokens, the logits in
// registers, and the f64 NLL of the next token is summed on chip (cpu/ygg.cpp:513-517).
template <int N, int BLK, int R, int R2T, int LT, int NVT>
__global__ void __launch_bounds__(256, blocks_per_sm<N>()) score_kernel(const __grid_constant__ DevModel m, int B, int T,
                                                    const int32_t *__restrict__ tokens, int8_t *state,
                                                    double *__restrict__ bits, uint32_t rec_max, int S) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int L = m.L, V = m.V, nv = m.VP / 32, ns = m.ns;
    Pool pool;
    Scratch sc;
    int8_t *qs;
    block_init(smem, rec_max, N, S, (L * N + 127) / 128 * 128, warp, lane, pool, sc, qs);
    const int home = warp % S;
    const StepOut none{nullptr, nullptr, nullptr};
    for (int s = blockIdx.x * W + warp; s < B; s += gridDim.x * W) {
        const int32_t *tok = tokens + (size_t)s * T;
        bool bad = false;
        for (int t = lane; t < T; t += 32) bad |= tok[t] < 0 || tok[t] >= V;
        if (__any_sync(kFull, bad)) {
            if (lane == 0) { atomicOr(m.status, kStatusBadToken); bits[s] = __longlong_as_double(0x7ff8000000000000LL); }
            continue;
        }
        // the row's state into the device layout (n per layer; coordinates past the model's ns are 0)
        for (int i = lane; i < L * N; i += 32) {
            const int li = i / N, c = i % N;
            qs[i] = (state != nullptr && c < ns) ? state[((size_t)s * L + li) * ns + c] : (int8_t)0;
        }
        __syncwarp();
        double nll = 0.0;
        for (int t = 0; t + 1 < T; t++) {
            float lg[kMaxClassesPerLane];
            if (!token_step<N, BLK, R, R2T, LT, NVT>(m, pool, sc, home, warp, tok[t], qs, qs, N, lg, none, lane)) {
                if (lane == 0) atomicOr(m.status, kStatusTimeout);
                return;
            }
            nll += nll_of(lg, nv, V, tok[t + 1], lane);
        }
        if (lane == 0) bits[s] = nll / 0.69314718055994530942;
        __syncwarp();
        if (state)
            for (int i = lane; i < L * N; i += 32) {
                const int li = i / N, c = i % N;
                if (c < ns) state[((size_t)s * L + li) * ns + c] = qs[i];
            }
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------------------ launchers

// The dynamic shared-memory limit of a kernel, raised once per device to the largest size asked for so far (the
// attribute is per device; raising it on every launch would cost a driver call per step).
constexpr int kMaxDevices = 64;
struct SmemLimits { size_t set[kMaxDevices]; };
template <int N, int BLK, int R, int R2T, int LT, int NVT> static SmemLimits &step_limit() { static SmemLimits l{}; return l; }
template <int N, int BLK, int R, int R2T, int LT, int NVT> static SmemLimits &score_limit() { static SmemLimits l{}; return l; }
static cudaError_t raise_smem_limit(const void *fn, size_t smem, SmemLimits &lim) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && lim.set[dev] >= smem) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) lim.set[dev] = smem;
    return e;
}

template <int N, int BLK, int R, int R2T, int LT, int NVT>
static cudaError_t launch_step_t(const DevModel &dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                                 float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps, int slots,
                                 int grid_cap, cudaStream_t st) {
    const size_t smem = block_smem(rec_max, N, slots, warps, 0);
    cudaError_t e = raise_smem_limit((const void *)step_kernel<N, BLK, R, R2T, LT, NVT>, smem, step_limit<N, BLK, R, R2T, LT, NVT>());
    if (e != cudaSuccess) return e;
    int grid = (B + warps - 1) / warps;
    if (grid > grid_cap) grid = grid_cap;
    step_kernel<N, BLK, R, R2T, LT, NVT><<<grid, 32 * warps, smem, st>>>(dm, B, tok, sin, sout, lg, routes, acc, rec_max, slots);
    return cudaGetLastError();
}

template <int N, int BLK, int R, int R2T, int LT, int NVT>
static cudaError_t launch_score_t(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                                  uint32_t rec_max, int warps, int slots, int grid_cap, cudaStream_t st) {
    const size_t smem = block_smem(rec_max, N, slots, warps, (dm.L * N + 127) / 128 * 128);
    cudaError_t e = raise_smem_limit((const void *)score_kernel<N, BLK, R, R2T, LT, NVT>, smem, score_limit<N, BLK, R, R2T, LT, NVT>());
    if (e != cudaSuccess) return e;
    int grid = (B + warps - 1) / warps;
    if (grid > grid_cap) grid = grid_cap;
    score_kernel<N, BLK, R, R2T, LT, NVT><<<grid, 32 * warps, smem, st>>>(dm, B, T, tok, state, bits, rec_max, slots);
    return cudaGetLastError();
}

#define YGG_DISPATCH(FN, ...)                                                                          \
    /* fast instances with the benchmark shapes fixed at compile time: c3 (n128 R16 R2=32, 4 layers, V <= 32), */ \
    /* c4 (same, V = 256), c1 / c2 (n64 R8 R2=16, 2 / 4 layers, V = 256) */                                    \
    if (n == 128 && blk == 16 && r == 16 && r2p == 32 && L == 4 && nv == 1) return FN<128, 16, 16, 32, 4, 1>(__VA_ARGS__); \
    if (n == 128 && blk == 16 && r == 16 && r2p == 32 && L == 4 && nv == 8) return FN<128, 16, 16, 32, 4, 8>(__VA_ARGS__); \
    if (n == 64 && blk == 16 && r == 8 && r2p == 16 && L == 2 && nv == 8) return FN<64, 16, 8, 16, 2, 8>(__VA_ARGS__);     \
    if (n == 64 && blk == 16 && r == 8 && r2p == 16 && L == 4 && nv == 8) return FN<64, 16, 8, 16, 4, 8>(__VA_ARGS__);     \
    switch (n * 1000 + blk * 100 + r) {                                                                \
        case 64 * 1000 + 8 * 100 + 8: return FN<64, 8, 8, 0, 0, 0>(__VA_ARGS__);                     \
        case 64 * 1000 + 8 * 100 + 16: return FN<64, 8, 16, 0, 0, 0>(__VA_ARGS__);                   \
        case 64 * 1000 + 8 * 100 + 32: return FN<64, 8, 32, 0, 0, 0>(__VA_ARGS__);                   \
        case 64 * 1000 + 16 * 100 + 8: return FN<64, 16, 8, 0, 0, 0>(__VA_ARGS__);                   \
        case 64 * 1000 + 16 * 100 + 16: return FN<64, 16, 16, 0, 0, 0>(__VA_ARGS__);                 \
        case 64 * 1000 + 16 * 100 + 32: return FN<64, 16, 32, 0, 0, 0>(__VA_ARGS__);                 \
        case 128 * 1000 + 8 * 100 + 8: return FN<128, 8, 8, 0, 0, 0>(__VA_ARGS__);                   \
        case 128 * 1000 + 8 * 100 + 16: return FN<128, 8, 16, 0, 0, 0>(__VA_ARGS__);                 \
        case 128 * 1000 + 8 * 100 + 32: return FN<128, 8, 32, 0, 0, 0>(__VA_ARGS__);                 \
        case 128 * 1000 + 16 * 100 + 8: return FN<128, 16, 8, 0, 0, 0>(__VA_ARGS__);                 \
        case 128 * 1000 + 16 * 100 + 16: return FN<128, 16, 16, 0, 0, 0>(__VA_ARGS__);               \
        case 128 * 1000 + 16 * 100 + 32: return FN<128, 16, 32, 0, 0, 0>(__VA_ARGS__);               \
        case 256 * 1000 + 8 * 100 + 8: return FN<256, 8, 8, 0, 0, 0>(__VA_ARGS__);                   \
        case 256 * 1000 + 8 * 100 + 16: return FN<256, 8, 16, 0, 0, 0>(__VA_ARGS__);                 \
        case 256 * 1000 + 8 * 100 + 32: return FN<256, 8, 32, 0, 0, 0>(__VA_ARGS__);                 \
        case 256 * 1000 + 16 * 100 + 8: return FN<256, 16, 8, 0, 0, 0>(__VA_ARGS__);                 \
        case 256 * 1000 + 16 * 100 + 16: return FN<256, 16, 16, 0, 0, 0>(__VA_ARGS__);               \
        case 256 * 1000 + 16 * 100 + 32: return FN<256, 16, 32, 0, 0, 0>(__VA_ARGS__);               \
        default: return cudaErrorInvalidValue;                                                         \
    }

cudaError_t launch_step(int n, int blk, int r, int r2p, const DevModel &dm, int B, const int32_t *tok, const int8_t *sin,
                        int8_t *sout, float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps,
                        int slots, int grid_cap, cudaStream_t st) {
    const int L = dm.L, nv = dm.VP / 32;
    YGG_DISPATCH(launch_step_t, dm, B, tok, sin, sout, lg, routes, acc, rec_max, warps, slots, grid_cap, st)
}

cudaError_t launch_score(int n, int blk, int r, int r2p, const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state,
                         double *bits, uint32_t rec_max, int warps, int slots, int grid_cap, cudaStream_t st) {
    const int L = dm.L, nv = dm.VP / 32;
    YGG_DISPATCH(launch_score_t, dm, B, T, tok, state, bits, rec_max, warps, slots, grid_cap, st)
}

size_t block_smem_bytes(uint32_t rec_max, int n, int slots, int warps, int state_bytes) {
    return block_smem(rec_max, n, slots, warps, state_bytes);
}

}  // namespace ygg
