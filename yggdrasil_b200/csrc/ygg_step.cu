// The int8 decode step and the fused scoring loop of Yggdrasil on sm_100a, for batches past the latency kernels'
// (ygg_coop.cu).
//
// G lanes serve one stream: a warp per stream (G = 32), or two streams per warp (G = 16, records interleaved over 16
// lanes; n <= 128 with readout rank <= 16), which shares every per-stream step a lane does not own (the router's
// decisions, rho, the copy handshakes, the descriptor loads, the loop control) between two streams. Lane gl of a group
// owns the C = n/G state coordinates [C gl, C gl + C) of every layer (layout in ygg_model.h). Per layer the group
//   1. computes rho from the new state of the layer below (exact int32 sum of squares, then the reference's f32 ops),
//   2. descends the router kLook = 3 levels per round of loads: the 7 rows of the 3-level subtree under the current
//      node are fetched together (16-byte lanes, n/16 lanes per row), their dots reduced within the row's lanes and
//      compared in f32 with the thresholds of (token, node), so D dependent levels cost ceil(D / 3) L2 round trips
//      (depth 13, the benchmark shapes', runs an unrolled copy),
//   3. gets the chosen expert's record and table row: staged (DIRECT = 0), a warp claims one slot per stream it serves
//      from the block's pool (a slot is held only from the copy to the readout, so a block runs more streams than it
//      has slots) and each group's first lane issues the bulk copies (cp.async.bulk, the 1-D TMA, no multicast) into
//      its slot, completing on the slot's mbarrier; direct (DIRECT = 1), the first lane asks L2 for the record
//      (cp.async.bulk.prefetch.L2) and the lanes later read their chunks from global memory,
//   4. meanwhile computes the layer input zl (lane gl: the dots of down-projection rows gl, gl + G, ... with the state
//      below),
//   5. (staged) waits on the mbarrier (bounded: it gives up after ~1 s with an error status instead of hanging),
//   6. runs the block-diagonal int16 x int8 transition (__dp2a), the table / factored input and the layer input in
//      int32, saturates to the new int8 state and stores it,
//   7. reads out z = P_r q (per-row partials, then redux.sync or a butterfly over the group; staged slots are handed
//      back first), quantises zq, and adds f32(Q zq) * s to the logits each lane holds in registers for its classes
//      G m + gl.
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
// The score kernel of a warp per stream runs where streams are few (below 32 768 rows per launch) and each row's
// latency sets the pace: 3 blocks, so that its row loop, f64 NLL and token pointers stay in registers
template <int N, int G> constexpr int score_blocks_per_sm() { return N >= 256 ? 2 : G == 32 ? 3 : 4; }

// ------------------------------------------------------------------------------------------------ shared memory

// Block layout: [S slots][S mbarriers][S owners][S phases] pad 128, then per stream of the block (W warps x P) its
// scratch and, for the score kernel, its state. A slot holds one expert record and one table row; the scratch holds
// the old state of the current layer, the new state of the layer below, the layer-input codes and the readout codes.
struct Pool {
    uint8_t *slots;
    uint32_t slot_bytes;
    uint32_t bars;     // shared address of mbarrier 0 (one per slot)
    int *owner;        // per unit of P slots: -1 free, else the owning warp
    int *phase;        // per slot: parity of the slot's mbarrier to wait for next
    int S, units;      // slots, and units of P = 32 / G slots (S is a multiple of P)
};
struct Scratch {
    int8_t *qold, *qb, *zl, *zq;
};

__host__ __device__ constexpr uint32_t pool_slot_bytes(uint32_t rec_max, int n) { return (rec_max + 2 * n + 127) / 128 * 128; }
__host__ __device__ constexpr uint32_t pool_meta_bytes(int S) { return (16u * S + 127) / 128 * 128; }
// readout codes zq: one 32-byte slot, or one per layer when the head runs after the last layer (defer_head); the
// scratch is kept to what a kernel uses, since its shared memory comes out of the SM's L1
constexpr int kZqSlot = 32;
__host__ __device__ constexpr uint32_t scratch_bytes(int n, int zq_bytes) {
    return (2 * n + 64 + zq_bytes + 127) / 128 * 128;
}
// Whether the head runs after the last layer (true) or layer by layer inside the layer loop: after, when a lane holds
// many classes (a wide vocabulary, or a shape not fixed at compile time), so that its logits take no registers across
// the layer loop (c4, V 256: +11 % tokens/s); inside, for the few classes of a small vocabulary (c3, V 5), where the
// loop's register allocation came out better with it.
template <int NVT, int G> __host__ __device__ constexpr bool defer_head() { return NVT == 0 || NVT * G > 64; }
template <int NVT, int G> __host__ __device__ constexpr int zq_bytes() {
    return defer_head<NVT, G>() ? kMaxLayers * kZqSlot : kZqSlot;
}
__host__ __device__ constexpr uint32_t block_smem(uint32_t rec_max, int n, int S, int streams, int state_bytes,
                                                  int zqb) {
    return S * pool_slot_bytes(rec_max, n) + pool_meta_bytes(S) + streams * (scratch_bytes(n, zqb) + state_bytes);
}

// Lane 0 claims a free unit of P slots for its warp, one slot per stream of the warp (CAS of the warp's id into the
// unit's owner word, starting from the warp's home unit); -1 after ~1 s without one. A warp claims all its slots in
// one step and releases them together, so a warp that holds slots never waits for more: no two warps can each hold
// part of what the other needs.
__device__ __forceinline__ int unit_claim(const Pool &p, int home, int owner) {
    const long long t0 = clock64();
    int i = home;
    while (true) {
        if (atomicCAS(p.owner + i, -1, owner) == -1) break;
        if (++i == p.units) {
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
    int32_t *acc;       // [L][ns] or null
};

// What a token's layers share: the block's pool and the stream's scratch, the token, the state pointers (qstride
// coordinates per layer; qlane: this lane's coordinates exist there and are read and written), the debug outputs and
// the new state of the layer below (carried from one layer to the next).
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

// The new state of layer l (padding of a narrower model held at exactly 0) into the stream's state, and the debug
// outputs.
template <int N, int G, bool QS>
__device__ __forceinline__ void finish_state(const DevModel &m, TokenCtx<N / G> &t, int l, int r, int (&acc)[N / G],
                                             LaneQ<N / G> &qn) {
    constexpr int C = N / G;
    const int gl = t.lane & (G - 1);
    const int qstride = QS ? N : t.qstride;
    const bool qlane = QS || t.qlane;
    if (m.ns < N && C * gl >= m.ns) {
#pragma unroll
        for (int i = 0; i < (C >= 4 ? C / 4 : 1); i++) qn.w[i] = 0;
#pragma unroll
        for (int ii = 0; ii < C; ii++) acc[ii] = 0;
    }
    if (QS) {   // the score kernel's state lives in shared memory, and it has no debug outputs
        store_q<C>(t.q_out + (size_t)l * qstride + C * gl, qn);
        return;
    }
    if (qlane) store_q_stream<C>(t.q_out + (size_t)l * qstride + C * gl, qn);
    if (t.dbg.routes != nullptr && gl == 0) t.dbg.routes[l] = r;
    if (t.dbg.acc != nullptr && qlane) {
#pragma unroll
        for (int ii = 0; ii < C; ii++) t.dbg.acc[(size_t)l * qstride + C * gl + ii] = acc[ii];
    }
}

// Layer l of a token (cpu/ygg.cpp:443-458) for the stream of the caller's lane group (G lanes). DIRECT: the expert
// record is read from global memory after an L2 prefetch; else it is staged in a shared-memory slot by a bulk copy.
// QS: the state is the stream's shared-memory copy in the device layout (stride n, every lane's coordinates; the score
// kernel). Returns false if a bounded wait gave up (for every stream of the warp). Always inlined: the warp collectives
// in it (shuffles, ballots, redux) rely on the caller's converged warp, and both stream groups of a warp run it
// together.
template <int N, int BLK, int R, int R2T, int NVT, int G, bool DIRECT, bool QS, bool PH = false>
__device__ __forceinline__ bool layer_step(TokenCtx<N / G> &t, const int l, float (&lg)[kMaxClasses<G>]) {
    constexpr int C = N / G;
    const DevModel &m = t.m;
    const Pool &pool = t.pool;
    const Scratch &sc = t.sc;
    const int lane = t.lane, x = t.x;
    const int gl = lane & (G - 1);
    const int E = m.E, D = m.D;
    LaneQ<C> &qbelow = t.qbelow;
    const DevLayer &y = m.layer[l];
    LaneQ<C> qold = {};
    if (QS) qold = load_q<C>(t.q_in + (size_t)l * N + C * gl);
    else if (t.qlane) qold = load_q_stream<C>(t.q_in + (size_t)l * t.qstride + C * gl);
    int r = x;
    float rho = 0.0f;
    const bool low = l > 0 && (R2T > 0 || m.R2 > 0);
    if (l > 0) {
        rho = rms_rho<N, G>(qbelow, y.r2b, y.rms_eps, m.inv_n, lane);
        store_q<C>(sc.qb + C * gl, qbelow);
        __syncwarp();
        const uint4 qrow = *(const uint4 *)(sc.qb + 16 * (gl % (N / 16)));
        // the benchmark depth (13: c3, c4) runs an unrolled copy of the router
        r = (D == 13 ? route_look<N, G, 13>(y.w, y.thr + (size_t)x * E, D, qrow, rho, lane)
                     : route_look<N, G>(y.w, y.thr + (size_t)x * E, D, qrow, rho, lane)) - E;
    }
    const uint32_t rec_bytes = y.rec_bytes;
    const bool has_table = y.table != nullptr;
    int acc[C];
    LaneQ<C> qn;
    ReadoutPart<N, R, G> ro;
    if constexpr (DIRECT) {
        // -- the record and its table row are read straight from global memory: the group's first lane asks L2 for
        // them now, and the layer-input codes run while they arrive
        const uint8_t *rec = y.rec + (size_t)r * rec_bytes;
        const int16_t *trow =
            has_table ? y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N : nullptr;
        if (gl == 0) {
            prefetch_l2(rec, rec_bytes);
            if (has_table) prefetch_l2(trow, 2u * N);
        }
        if (low) layer_input_codes<N, R2T, G>(m, y, sc.qb, rho, sc.zl, lane);
        store_q<C>(sc.qold + C * gl, qold);
        __syncwarp();
        leaf_update<N, BLK, R2T, G, true>(m, y, rec, trow, x, sc.qold, sc.zl, low, lane, acc, qn);
        finish_state<N, G, QS>(m, t, l, r, acc, qn);
        ro = readout_partials<N, R, G, true>(y, rec, qn, lane);
    } else {
        // -- lane 0 claims a unit of slots for the warp (slot unit * P + group for each stream group); each group's
        // first lane issues the bulk copies of its expert record and table row into its slot; the slot index and the
        // parity to wait for reach the group's lanes in one shuffle
        constexpr int P = 32 / G;
        const int leader = lane & (32 - G);
        // the group leader's copies into slot unit * P + group (one group, lane 0, when G = 32)
        auto issue = [&](int unit) {
            const int slot = unit * P + lane / G;
            uint8_t *rec = pool.slots + (size_t)slot * pool.slot_bytes;
            const uint32_t bar = pool.bars + 8u * slot;
            fence_proxy_async();
            mbar_expect_tx(bar, rec_bytes + (has_table ? 2u * N : 0u));
            bulk_g2s(smem_addr(rec), y.rec + (size_t)r * rec_bytes, rec_bytes, bar);
            if (has_table) {
                const int16_t *src = y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N;
                bulk_g2s(smem_addr(rec + pool.slot_bytes - 2 * N), src, 2u * N, bar);
            }
            return 2 * slot + pool.phase[slot];
        };
        int unit = 0, tag = -1;
        if constexpr (G == 32) {   // one stream: lane 0 claims and copies in one region, one shuffle
            if (lane == 0) {
                unit = unit_claim(pool, t.home, t.warp);
                if (unit >= 0) tag = issue(unit);
            }
            tag = __shfl_sync(kFull, tag, 0);
            if (tag < 0) return false;
            unit = tag >> 1;
        } else {
            if (lane == 0) unit = unit_claim(pool, t.home, t.warp);
            unit = __shfl_sync(kFull, unit, 0);
            if (unit < 0) return false;
            __syncwarp();   // the phases the unit's last holder flipped are visible to every group leader
            if (gl == 0) tag = issue(unit);
            tag = __shfl_sync(kFull, tag, leader);
        }
        const int slot = tag >> 1;
        const uint32_t parity = (uint32_t)(tag & 1);
        const uint8_t *rec = pool.slots + (size_t)slot * pool.slot_bytes;
        const int16_t *trow = (const int16_t *)(rec + (pool.slot_bytes - 2 * N));
        const uint32_t bar = pool.bars + 8u * slot;
        // -- layer input codes while the copy is in flight (cpu/ygg.cpp:285-296)
        if (low) layer_input_codes<N, R2T, G>(m, y, sc.qb, rho, sc.zl, lane);
        store_q<C>(sc.qold + C * gl, qold);
        __syncwarp();
        if (!__all_sync(kFull, mbar_wait_bounded(bar, parity))) return false;
        leaf_update<N, BLK, R2T, G>(m, y, rec, has_table ? trow : nullptr, x, sc.qold, sc.zl, low, lane, acc, qn);
        finish_state<N, G, QS>(m, t, l, r, acc, qn);
        ro = readout_partials<N, R, G>(y, rec, qn, lane);
        // the slots are free once their bytes are used: flip their parities and hand the unit back
        __syncwarp();
        if (gl == 0) pool.phase[slot] = (int)(parity ^ 1u);
        if (G < 32) __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            atomicExch(pool.owner + unit, -1);
        }
    }
    const int zq = readout_code<N, R, G>(ro, lane);
    const int row = readout_row<R, G>(gl);
    constexpr bool kDefer = defer_head<NVT, G>();
    int8_t *zqs = sc.zq + (kDefer ? l * kZqSlot : 0);
    if (row >= 0 && (G == 32 || R == 16 || (gl & 1) == 0)) zqs[row] = (int8_t)zq;
    if constexpr (!kDefer && !PH) {
        __syncwarp();
        head_accumulate<R, NVT, G>(m, y, zqs, lg, lane);
    }
    qbelow = qn;
    __syncwarp();
    return true;
}

// One token of the stream of the caller's lane group through every layer. q_in / q_out: the stream's state
// [L][qstride] (global memory in the caller's layout, qstride = the model's ns, or shared memory in the device layout,
// qstride = n; they may alias); qlane false: the state is neither read (zeros) nor written (a stream that only keeps
// its warp's collectives company). lg: the logits of the lane's classes (out). Returns false if a bounded wait gave
// up. Compile-time shape where a fast instance fixes it (0: read from the model at run time): R2T the padded
// layer-input rank, LT the number of layers, NVT the classes per lane (VP / G).
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool DIRECT, bool QS>
__device__ __forceinline__ bool token_step(const DevModel &m, const Pool &pool, const Scratch &sc, int home, int warp,
                                           int x, const int8_t *q_in, int8_t *q_out, int qstride, bool qlane,
                                           float (&lg)[kMaxClasses<G>], const StepOut &dbg, int lane) {
    const int V = m.V;
    const int nv = NVT ? NVT : m.VP / G;
    const int gl = lane & (G - 1);
    TokenCtx<N / G> t{m, pool, sc, home, warp, lane, x, q_in, q_out, qstride, qlane && (N / G) * gl < qstride,
                      dbg, {}};
    constexpr bool kDefer = defer_head<NVT, G>();
    if constexpr (!kDefer) {
#pragma unroll
        for (int c = 0; c < kMaxClasses<G>; c++) lg[c] = c < nv ? __ldg(m.head_b + G * c + gl) : 0.0f;
    }
    if constexpr (LT > 0 && DIRECT && N <= 64) {
        // the direct path has no early exit (no slot claims, no waits): its fixed layer loop unrolls (n = 64: +8 % on
        // c1; at n = 128 the unrolled body spills)
#pragma unroll
        for (int l = 0; l < LT; l++) layer_step<N, BLK, R, R2T, NVT, G, DIRECT, QS>(t, l, lg);
    } else if constexpr (LT > 0) {
        // not unrolled: an unrolled layer loop with its early exits defeats the compiler's proof that the warp is
        // converged at the collectives, and each shuffle / ballot / redux then pays a re-convergence loop
#pragma unroll 1
        for (int l = 0; l < LT; l++)
            if (!layer_step<N, BLK, R, R2T, NVT, G, DIRECT, QS>(t, l, lg)) return false;
    } else {
#pragma unroll 1
        for (int l = 0; l < m.L; l++)
            if (!layer_step<N, BLK, R, R2T, NVT, G, DIRECT, QS>(t, l, lg)) return false;
    }
    // a deferred head after the last layer, from every layer's readout codes in shared memory: the lane's classes
    // start at the output bias and add f32(Q_l zq_l) s_l layer by layer (cpu/ygg.cpp:421-434, the reference's order),
    // so the logits take registers only here; skipped when nothing reads them
    if constexpr (kDefer) {
        if (!QS && dbg.logits == nullptr) return true;
#pragma unroll
        for (int c = 0; c < kMaxClasses<G>; c++) lg[c] = c < nv ? __ldg(m.head_b + G * c + gl) : 0.0f;
        if constexpr (LT > 0) {
#pragma unroll 1
            for (int l = 0; l < LT; l++) head_accumulate<R, NVT, G>(m, m.layer[l], sc.zq + l * kZqSlot, lg, lane);
        } else {
#pragma unroll 1
            for (int l = 0; l < m.L; l++) head_accumulate<R, NVT, G>(m, m.layer[l], sc.zq + l * kZqSlot, lg, lane);
        }
    }
    if (!QS) {
#pragma unroll
        for (int c = 0; c < kMaxClasses<G>; c++) {
            const int cls = G * c + gl;
            if (c < nv && cls < V) dbg.logits[cls] = lg[c];
        }
    }
    return true;
}

// ------------------------------------------------------------------------------------------------ kernels

// Pool and the scratch of this block's stream `sidx` (warp * P + group); the first thread initialises the slots'
// mbarriers and phases and the units' owners.
__device__ __forceinline__ void block_init(uint8_t *smem, uint32_t rec_max, int n, int S, int P, int state_bytes,
                                           int zqb, int sidx, Pool &pool, Scratch &sc, int8_t *&state) {
    pool.slot_bytes = pool_slot_bytes(rec_max, n);
    pool.slots = smem;
    uint8_t *meta = smem + (size_t)S * pool.slot_bytes;
    pool.bars = smem_addr(meta);
    pool.owner = (int *)(meta + 8 * S);
    pool.phase = (int *)(meta + 12 * S);
    pool.S = S;
    pool.units = S / P;   // 0: no slots (records read from global memory)
    uint8_t *ws = meta + pool_meta_bytes(S) + (size_t)sidx * (scratch_bytes(n, zqb) + state_bytes);
    sc.qold = (int8_t *)ws;
    sc.qb = sc.qold + n;
    sc.zl = sc.qb + n;
    sc.zq = sc.zl + 64;        // zq_bytes: one or kMaxLayers slots of kZqSlot codes
    state = (int8_t *)(ws + scratch_bytes(n, zqb));
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(pool.bars + 8u * i, 1);
            pool.owner[i] = -1;   // units < S: owner words of the units, the rest unused
            pool.phase[i] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();
}

// Each warp serves P = 32 / G streams at a time, stream base + (lane / G); a warp whose second stream is past B runs
// it on a copy of its first (nothing of it is read or written) so that its collectives stay full-warp.
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool DIRECT>
__global__ void __launch_bounds__(256, blocks_per_sm<N>()) step_kernel(const __grid_constant__ DevModel m, int B,
                                                   const int32_t *__restrict__ tokens, const int8_t *state_in,
                                                   int8_t *state_out, float *__restrict__ logits,
                                                   int32_t *__restrict__ routes, int32_t *__restrict__ acc_out,
                                                   uint32_t rec_max, int S) {
    constexpr int P = 32 / G;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int gh = lane / G, gl = lane & (G - 1);
    const int sidx = warp * P + gh;
    Pool pool;
    Scratch sc;
    int8_t *unused;
    block_init(smem, rec_max, N, S, P, 0, zq_bytes<NVT, G>(), sidx, pool, sc, unused);
    const int home = pool.units ? warp % pool.units : 0;
    const int L = m.L, V = m.V, ns = m.ns;
    for (int base = (blockIdx.x * W + warp) * P; base < B; base += gridDim.x * W * P) {
        const int s = base + gh;
        const bool real = s < B;
        const int se = real ? s : base;
        const int x = tokens[se];
        // a token out of range (cpu/ygg.cpp:493-495 rejects the whole input): the stream is skipped, NaN logits and
        // its state unchanged; it runs token 0 unseen so that its warp's collectives stay full
        const bool bad = x < 0 || x >= V;
        const bool live = real && !bad;
        if (real && bad && gl == 0) atomicOr(m.status, kStatusBadToken);
        float lg[kMaxClasses<G>];
        StepOut o{(live && logits) ? logits + (size_t)s * V : nullptr, (live && routes) ? routes + (size_t)s * L : nullptr,
                  (live && acc_out) ? acc_out + (size_t)se * L * ns : nullptr};
        if (!token_step<N, BLK, R, R2T, LT, NVT, G, DIRECT, false>(m, pool, sc, home, warp, bad ? 0 : x, state_in + (size_t)se * L * ns,
                                                    state_out + (size_t)se * L * ns, ns, live, lg, o, lane)) {
            if (lane == 0) atomicOr(m.status, kStatusTimeout);
            return;
        }
        if (real && bad) {
            if (logits != nullptr)
                for (int c = gl; c < V; c += G) logits[(size_t)s * V + c] = __int_as_float(0x7fc00000);
            if (state_out != state_in)
                for (int i = gl; i < L * ns; i += G) state_out[(size_t)s * L * ns + i] = state_in[(size_t)s * L * ns + i];
            if (routes != nullptr && gl < L) routes[(size_t)s * L + gl] = -1;
        }
    }
}

// Layer l of a layer-phased step: one launch per layer over every stream, so that the records the streams gather
// at a time are one layer's (c3 / c4: 84 MB, which L2 holds) instead of every layer's (252 MB, which it does not).
// Between the launches a stream's new state of layer l - 1 waits in state_out (read back here as the state below) and
// its readout codes in zq_all [B][L][kZqSlot]; the launch of the last layer runs the head of every layer, in layer
// order (cpu/ygg.cpp:421-434). The arithmetic of each layer is the fused step's (layer_step), so the results are the
// same bit for bit. Records are read from global memory (no staging slots).
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G>
__global__ void __launch_bounds__(256, blocks_per_sm<N>()) phase_kernel(const __grid_constant__ DevModel m, int B, int l,
                                                    const int32_t *__restrict__ tokens, const int8_t *state_in,
                                                    int8_t *state_out, float *__restrict__ logits,
                                                    int32_t *__restrict__ routes, int32_t *__restrict__ acc_out,
                                                    int8_t *__restrict__ zq_all) {
    constexpr int P = 32 / G, C = N / G;
    constexpr bool kDefer = defer_head<NVT, G>();
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int gh = lane / G, gl = lane & (G - 1);
    const int sidx = warp * P + gh;
    Pool pool;
    Scratch sc;
    int8_t *unused;
    block_init(smem, 0, N, 0, P, 0, kMaxLayers * kZqSlot, sidx, pool, sc, unused);
    const int L = LT > 0 ? LT : m.L, V = m.V, ns = m.ns;
    const int nv = NVT ? NVT : m.VP / G;
    for (int base = (blockIdx.x * W + warp) * P; base < B; base += gridDim.x * W * P) {
        const int s = base + gh;
        const bool real = s < B;
        const int se = real ? s : base;
        const int x = tokens[se];
        const bool bad = x < 0 || x >= V;   // skipped as in step_kernel: NaN logits, state unchanged
        const bool live = real && !bad;
        if (l == 0 && real && bad && gl == 0) atomicOr(m.status, kStatusBadToken);
        const StepOut o{nullptr, (live && routes) ? routes + (size_t)s * L : nullptr,
                        (live && acc_out) ? acc_out + (size_t)se * L * ns : nullptr};
        TokenCtx<C> t{m, pool, sc, 0, warp, lane, bad ? 0 : x, state_in + (size_t)se * L * ns,
                      state_out + (size_t)se * L * ns, ns, live && C * gl < ns, o, {}};
        if (l > 0 && t.qlane) t.qbelow = load_q<C>(state_out + ((size_t)se * L + l - 1) * ns + C * gl);
        float lg[kMaxClasses<G>];
        layer_step<N, BLK, R, R2T, NVT, G, true, false, true>(t, l, lg);
        const int8_t *zqs = sc.zq + (kDefer ? l * kZqSlot : 0);
        __syncwarp();
        if (live && gl < R) zq_all[((size_t)s * L + l) * kZqSlot + gl] = zqs[gl];
        if (l == L - 1) {
            // every layer's codes into the stream's slots, then the head in layer order
            __syncwarp();
            if (gl < R)
                for (int j = 0; j < L; j++) sc.zq[j * kZqSlot + gl] = live ? zq_all[((size_t)s * L + j) * kZqSlot + gl] : 0;
            __syncwarp();
            if (live && logits != nullptr) {
#pragma unroll
                for (int c = 0; c < kMaxClasses<G>; c++) lg[c] = c < nv ? __ldg(m.head_b + G * c + gl) : 0.0f;
#pragma unroll 1
                for (int j = 0; j < L; j++) head_accumulate<R, NVT, G>(m, m.layer[j], sc.zq + j * kZqSlot, lg, lane);
#pragma unroll
                for (int c = 0; c < kMaxClasses<G>; c++) {
                    const int cls = G * c + gl;
                    if (c < nv && cls < V) logits[(size_t)s * V + cls] = lg[c];
                }
            }
            if (real && bad) {
                if (logits != nullptr)
                    for (int c = gl; c < V; c += G) logits[(size_t)s * V + c] = __int_as_float(0x7fc00000);
                if (routes != nullptr && gl < L) routes[(size_t)s * L + gl] = -1;
            }
            __syncwarp();
        }
        if (real && bad && state_out != state_in)
            for (int i = gl; i < ns; i += G) state_out[((size_t)s * L + l) * ns + i] = state_in[((size_t)s * L + l) * ns + i];
    }
}

// Rows of `steps` tokens; the state of a row lives in its group's shared memory between tokens, the logits in
// registers, and the f64 NLL of the next token is summed on chip (cpu/ygg.cpp:513-517). Each warp scores P = 32 / G
// rows at a time; a row past B, or with a token out of range, runs unseen (token 0, nothing written; the bad row
// scores NaN).
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool DIRECT>
__global__ void __launch_bounds__(256, score_blocks_per_sm<N, G>()) score_kernel(const __grid_constant__ DevModel m, int B, int T,
                                                    const int32_t *__restrict__ tokens, int8_t *state,
                                                    double *__restrict__ bits, uint32_t rec_max, int S) {
    constexpr int P = 32 / G;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int gh = lane / G, gl = lane & (G - 1);
    const int sidx = warp * P + gh;
    const int L = m.L, V = m.V, nv = m.VP / G, ns = m.ns;
    Pool pool;
    Scratch sc;
    int8_t *qs;
    block_init(smem, rec_max, N, S, P, (L * N + 127) / 128 * 128, zq_bytes<NVT, G>(), sidx, pool, sc, qs);
    const int home = pool.units ? warp % pool.units : 0;
    const StepOut none{nullptr, nullptr, nullptr};
    for (int base = (blockIdx.x * W + warp) * P; base < B; base += gridDim.x * W * P) {
        const int s = base + gh;
        const bool real = G == 32 || s < B;        // a warp per stream: its one row is always real
        const int32_t *tok = tokens + (size_t)(real ? s : base) * T;
        bool bad = false;
        for (int t = gl; t < T; t += G) bad |= tok[t] < 0 || tok[t] >= V;
        const uint32_t bb = __ballot_sync(kFull, bad);
        bad = ((bb >> (lane & (32 - G))) & (G == 32 ? kFull : 0xFFFFu)) != 0;
        if (real && bad && gl == 0) {
            atomicOr(m.status, kStatusBadToken);
            bits[s] = __longlong_as_double(0x7ff8000000000000LL);
        }
        if (G == 32 && bad) continue;              // the whole warp skips its row
        const bool live = real && !bad;
        // the row's state into the device layout (n per layer; coordinates past the model's ns are 0)
        for (int i = gl; i < L * N; i += G) {
            const int li = i / N, c = i % N;
            qs[i] = (live && state != nullptr && c < ns) ? state[((size_t)s * L + li) * ns + c] : (int8_t)0;
        }
        __syncwarp();
        double nll = 0.0;
        for (int t = 0; t + 1 < T; t++) {
            float lg[kMaxClasses<G>];
            const int xt = live ? tok[t] : 0;
            if (!token_step<N, BLK, R, R2T, LT, NVT, G, DIRECT, true>(m, pool, sc, home, warp, xt, qs, qs, N, true, lg, none, lane)) {
                if (lane == 0) atomicOr(m.status, kStatusTimeout);
                return;
            }
            nll += nll_of<G>(lg, nv, V, live ? tok[t + 1] : 0, lane);
        }
        if (live && gl == 0) bits[s] = nll / 0.69314718055994530942;
        __syncwarp();
        if (live && state)
            for (int i = gl; i < L * N; i += G) {
                const int li = i / N, c = i % N;
                if (c < ns) state[((size_t)s * L + li) * ns + c] = qs[i];
            }
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------------------ self test

// The bounded wait of the kernels, made to run out: one warp waits on an mbarrier that nothing arrives at (its
// expected arrival never comes), gives up after `limit` cycles as every wait of the step does, and writes the timeout
// status. Nothing faults or spins forever, and the context stays usable.
__global__ void wait_selftest_kernel(long long limit, int *status) {
    __shared__ __align__(8) uint64_t bar_word;
    const uint32_t bar = smem_addr(&bar_word);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    const bool ok = __all_sync(kFull, mbar_wait_bounded(bar, 0, limit));
    if (threadIdx.x == 0) *status = ok ? (int)kStatusOk : (int)kStatusTimeout;
}

cudaError_t launch_wait_selftest(long long limit, int *d_status, cudaStream_t st) {
    wait_selftest_kernel<<<1, 32, 0, st>>>(limit, d_status);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ launchers

template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool D> static SmemLimits &step_limit() { static SmemLimits l{}; return l; }
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool D> static SmemLimits &score_limit() { static SmemLimits l{}; return l; }

// blocks for B streams: W warps of P = 32 / G streams each, at most grid_cap blocks
template <int G> static int grid_for(int B, int warps, int grid_cap) {
    const int per = warps * (32 / G);
    const int grid = (B + per - 1) / per;
    return grid > grid_cap ? grid_cap : grid;
}

// D (direct): records read from global memory, no slots; else `slots` staging slots per block.
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool D>
static cudaError_t launch_step_t(const DevModel &dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                                 float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps, int slots,
                                 int grid_cap, cudaStream_t st) {
    const int S = D ? 0 : slots;
    const size_t smem = block_smem(rec_max, N, S, warps * (32 / G), 0, zq_bytes<NVT, G>());
    cudaError_t e = raise_smem_limit((const void *)step_kernel<N, BLK, R, R2T, LT, NVT, G, D>, smem,
                                     step_limit<N, BLK, R, R2T, LT, NVT, G, D>());
    if (e != cudaSuccess) return e;
    step_kernel<N, BLK, R, R2T, LT, NVT, G, D><<<grid_for<G>(B, warps, grid_cap), 32 * warps, smem, st>>>(
        dm, B, tok, sin, sout, lg, routes, acc, rec_max, S);
    return cudaGetLastError();
}

template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool D> static SmemLimits &phase_limit() { static SmemLimits l{}; return l; }

// The layer-phased step: one phase_kernel launch per layer (D, the record path, is always direct here).
template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool D>
static cudaError_t launch_phased_t(const DevModel &dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                                   float *lg, int32_t *routes, int32_t *acc, int8_t *zq, int warps, int grid_cap,
                                   cudaStream_t st) {
    const size_t smem = block_smem(0, N, 0, warps * (32 / G), 0, kMaxLayers * kZqSlot);
    cudaError_t e = raise_smem_limit((const void *)phase_kernel<N, BLK, R, R2T, LT, NVT, G>, smem,
                                     phase_limit<N, BLK, R, R2T, LT, NVT, G, false>());
    if (e != cudaSuccess) return e;
    const int L = LT > 0 ? LT : dm.L;
    for (int l = 0; l < L && e == cudaSuccess; l++) {
        phase_kernel<N, BLK, R, R2T, LT, NVT, G><<<grid_for<G>(B, warps, grid_cap), 32 * warps, smem, st>>>(
            dm, B, l, tok, sin, sout, lg, routes, acc, zq);
        e = cudaGetLastError();
    }
    return e;
}

template <int N, int BLK, int R, int R2T, int LT, int NVT, int G, bool D>
static cudaError_t launch_score_t(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                                  uint32_t rec_max, int warps, int slots, int grid_cap, cudaStream_t st) {
    const int S = D ? 0 : slots;
    const size_t smem = block_smem(rec_max, N, S, warps * (32 / G), (dm.L * N + 127) / 128 * 128, zq_bytes<NVT, G>());
    cudaError_t e = raise_smem_limit((const void *)score_kernel<N, BLK, R, R2T, LT, NVT, G, D>, smem,
                                     score_limit<N, BLK, R, R2T, LT, NVT, G, D>());
    if (e != cudaSuccess) return e;
    score_kernel<N, BLK, R, R2T, LT, NVT, G, D><<<grid_for<G>(B, warps, grid_cap), 32 * warps, smem, st>>>(
        dm, B, T, tok, state, bits, rec_max, S);
    return cudaGetLastError();
}

// Instances: lw = 16 (two streams per warp; the layout the loader picks for n 64 / 128 with readout rank <= 16) or
// lw = 32 (a warp per stream: every shape). Fast instances fix the benchmark shapes at compile time: c3 (n128 R16
// R2=32, 4 layers, V <= 32), c4 (the same, V = 256), c1 / c2 (n64 R8 R2=16, 2 / 4 layers, V = 256).
#define YGG_DISPATCH(FN, ...)                                                                                          \
    if (lw == 16) {                                                                                                    \
        if (n == 128 && blk == 16 && r == 16 && r2p == 32 && L == 4 && VP == 32) return dm.direct ? FN<128, 16, 16, 32, 4, 2, 16, true>(__VA_ARGS__) : FN<128, 16, 16, 32, 4, 2, 16, false>(__VA_ARGS__); \
        if (n == 128 && blk == 16 && r == 16 && r2p == 32 && L == 4 && VP == 256) return dm.direct ? FN<128, 16, 16, 32, 4, 16, 16, true>(__VA_ARGS__) : FN<128, 16, 16, 32, 4, 16, 16, false>(__VA_ARGS__); \
        if (n == 64 && blk == 16 && r == 8 && r2p == 16 && L == 2 && VP == 256) return dm.direct ? FN<64, 16, 8, 16, 2, 16, 16, true>(__VA_ARGS__) : FN<64, 16, 8, 16, 2, 16, 16, false>(__VA_ARGS__);     \
        if (n == 64 && blk == 16 && r == 8 && r2p == 16 && L == 4 && VP == 256) return dm.direct ? FN<64, 16, 8, 16, 4, 16, 16, true>(__VA_ARGS__) : FN<64, 16, 8, 16, 4, 16, 16, false>(__VA_ARGS__);     \
        switch (n * 1000 + blk * 100 + r) {                                                                            \
            case 64 * 1000 + 8 * 100 + 8: return FN<64, 8, 8, 0, 0, 0, 16, false>(__VA_ARGS__);                              \
            case 64 * 1000 + 8 * 100 + 16: return FN<64, 8, 16, 0, 0, 0, 16, false>(__VA_ARGS__);                            \
            case 64 * 1000 + 16 * 100 + 8: return FN<64, 16, 8, 0, 0, 0, 16, false>(__VA_ARGS__);                            \
            case 64 * 1000 + 16 * 100 + 16: return FN<64, 16, 16, 0, 0, 0, 16, false>(__VA_ARGS__);                          \
            case 128 * 1000 + 8 * 100 + 8: return FN<128, 8, 8, 0, 0, 0, 16, false>(__VA_ARGS__);                            \
            case 128 * 1000 + 8 * 100 + 16: return FN<128, 8, 16, 0, 0, 0, 16, false>(__VA_ARGS__);                          \
            case 128 * 1000 + 16 * 100 + 8: return FN<128, 16, 8, 0, 0, 0, 16, false>(__VA_ARGS__);                          \
            case 128 * 1000 + 16 * 100 + 16: return FN<128, 16, 16, 0, 0, 0, 16, false>(__VA_ARGS__);                        \
            default: return cudaErrorInvalidValue;                                                                     \
        }                                                                                                              \
    }                                                                                                                  \
    if (n == 128 && blk == 16 && r == 16 && r2p == 32 && L == 4 && VP == 32) return dm.direct ? FN<128, 16, 16, 32, 4, 1, 32, true>(__VA_ARGS__) : FN<128, 16, 16, 32, 4, 1, 32, false>(__VA_ARGS__); \
    if (n == 128 && blk == 16 && r == 16 && r2p == 32 && L == 4 && VP == 256) return dm.direct ? FN<128, 16, 16, 32, 4, 8, 32, true>(__VA_ARGS__) : FN<128, 16, 16, 32, 4, 8, 32, false>(__VA_ARGS__); \
    if (n == 64 && blk == 16 && r == 8 && r2p == 16 && L == 2 && VP == 256) return dm.direct ? FN<64, 16, 8, 16, 2, 8, 32, true>(__VA_ARGS__) : FN<64, 16, 8, 16, 2, 8, 32, false>(__VA_ARGS__);     \
    if (n == 64 && blk == 16 && r == 8 && r2p == 16 && L == 4 && VP == 256) return dm.direct ? FN<64, 16, 8, 16, 4, 8, 32, true>(__VA_ARGS__) : FN<64, 16, 8, 16, 4, 8, 32, false>(__VA_ARGS__);     \
    switch (n * 1000 + blk * 100 + r) {                                                                                \
        case 64 * 1000 + 8 * 100 + 8: return FN<64, 8, 8, 0, 0, 0, 32, false>(__VA_ARGS__);                                  \
        case 64 * 1000 + 8 * 100 + 16: return FN<64, 8, 16, 0, 0, 0, 32, false>(__VA_ARGS__);                                \
        case 64 * 1000 + 8 * 100 + 32: return FN<64, 8, 32, 0, 0, 0, 32, false>(__VA_ARGS__);                                \
        case 64 * 1000 + 16 * 100 + 8: return FN<64, 16, 8, 0, 0, 0, 32, false>(__VA_ARGS__);                                \
        case 64 * 1000 + 16 * 100 + 16: return FN<64, 16, 16, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 64 * 1000 + 16 * 100 + 32: return FN<64, 16, 32, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 128 * 1000 + 8 * 100 + 8: return FN<128, 8, 8, 0, 0, 0, 32, false>(__VA_ARGS__);                                \
        case 128 * 1000 + 8 * 100 + 16: return FN<128, 8, 16, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 128 * 1000 + 8 * 100 + 32: return FN<128, 8, 32, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 128 * 1000 + 16 * 100 + 8: return FN<128, 16, 8, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 128 * 1000 + 16 * 100 + 16: return FN<128, 16, 16, 0, 0, 0, 32, false>(__VA_ARGS__);                            \
        case 128 * 1000 + 16 * 100 + 32: return FN<128, 16, 32, 0, 0, 0, 32, false>(__VA_ARGS__);                            \
        case 256 * 1000 + 8 * 100 + 8: return FN<256, 8, 8, 0, 0, 0, 32, false>(__VA_ARGS__);                                \
        case 256 * 1000 + 8 * 100 + 16: return FN<256, 8, 16, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 256 * 1000 + 8 * 100 + 32: return FN<256, 8, 32, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 256 * 1000 + 16 * 100 + 8: return FN<256, 16, 8, 0, 0, 0, 32, false>(__VA_ARGS__);                              \
        case 256 * 1000 + 16 * 100 + 16: return FN<256, 16, 16, 0, 0, 0, 32, false>(__VA_ARGS__);                            \
        case 256 * 1000 + 16 * 100 + 32: return FN<256, 16, 32, 0, 0, 0, 32, false>(__VA_ARGS__);                            \
        default: return cudaErrorInvalidValue;                                                                         \
    }

cudaError_t launch_step(int n, int blk, int r, int r2p, const DevModel &dm, int B, const int32_t *tok, const int8_t *sin,
                        int8_t *sout, float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps,
                        int slots, int grid_cap, cudaStream_t st) {
    const int L = dm.L, VP = dm.VP, lw = dm.lw;
    YGG_DISPATCH(launch_step_t, dm, B, tok, sin, sout, lg, routes, acc, rec_max, warps, slots, grid_cap, st)
}

cudaError_t launch_phased(int n, int blk, int r, int r2p, const DevModel &dm, int B, const int32_t *tok,
                          const int8_t *sin, int8_t *sout, float *lg, int32_t *routes, int32_t *acc, int8_t *zq, int warps,
                          int grid_cap, cudaStream_t st) {
    const int L = dm.L, VP = dm.VP, lw = dm.lw;
    YGG_DISPATCH(launch_phased_t, dm, B, tok, sin, sout, lg, routes, acc, zq, warps, grid_cap, st)
}

cudaError_t launch_score(int n, int blk, int r, int r2p, const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state,
                         double *bits, uint32_t rec_max, int warps, int slots, int grid_cap, cudaStream_t st) {
    const int L = dm.L, VP = dm.VP, lw = dm.lw;
    YGG_DISPATCH(launch_score_t, dm, B, T, tok, state, bits, rec_max, warps, slots, grid_cap, st)
}

// the largest shared memory of a block of the step or score kernels (the deferred head's zq slots), for the slot sizing
size_t block_smem_bytes(uint32_t rec_max, int n, int slots, int warps, int state_bytes) {
    return block_smem(rec_max, n, slots, warps, state_bytes, kMaxLayers * kZqSlot);
}

}  // namespace ygg
