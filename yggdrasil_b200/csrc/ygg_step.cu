// The int8 decode step and the fused scoring loop of Yggdrasil on sm_100a.
//
// One warp serves one stream; lane l owns the C = n/32 state coordinates [C l, C l + C) of every layer (layout in
// ygg_model.h). Per layer the warp
//   1. computes rho from the new state of the layer below (exact int32 sum of squares, then the reference's f32 ops),
//   2. descends the router: D dependent levels, each one coalesced n-byte row (lane C bytes), __dp4a and a
//      single-instruction warp reduction (redux.sync), compared in f32 with the threshold of (token, node),
//   3. has lane 0 issue one bulk copy (cp.async.bulk, the 1-D TMA) of the chosen expert's record, and one of its
//      table row, into the warp's shared-memory slot, completing on the warp's mbarrier,
//   4. meanwhile computes the layer input zl (lane k: the dot of down-projection row k with the state below),
//   5. waits on the mbarrier (bounded: it gives up after ~1 s with an error status instead of hanging),
//   6. runs the block-diagonal int16 x int8 transition (__dp2a), the table / factored input and the layer input in
//      int32, saturates to the new int8 state and stores it,
//   7. reads out z = P_r q (per-row partials + redux.sync), quantises zq, and adds f32(Q zq) * s to the logits each
//      lane holds in registers for its classes 32 m + lane.
// Every f32 operation is the reference's, single-rounded and in the reference's order (__fmul_rn / __fadd_rn /
// __fsqrt_rn / __fdiv_rn; no contraction), and f32 -> int32 rounds half to even with the x86 out-of-range value, so
// routes, int32 accumulators, states and logits equal cpu/ygg.cpp bit for bit.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ygg_model.h"

namespace ygg {

constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr int kMaxClassesPerLane = 8;   // VP <= 256
constexpr long long kWaitCycles = 2000000000LL;

// ------------------------------------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast), completion counted on the mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Bounded wait for the phase `parity` of the warp's mbarrier: false after ~1 s (the caller reports a timeout).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}

// f32 -> int32 rounded half to even; NaN and values outside int32 give INT_MIN, as x86 cvtps2dq (the reference's
// _mm512_cvtps_epi32), which the callers then clamp.
__device__ __forceinline__ int cvt_rne(float v) {
    return (v >= -2147483648.0f && v < 2147483648.0f) ? __float2int_rn(v) : (int)0x80000000;
}
__device__ __forceinline__ float i2f(int v) { return __int2float_rn(v); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }

// --------------------------------------------------------------------------------------------- lane state words

// The C state bytes of one lane as int32 words: C = 2 uses the low half of one word (high half zero).
template <int C> struct LaneQ { uint32_t w[C >= 4 ? C / 4 : 1]; };

template <int C> __device__ __forceinline__ LaneQ<C> load_q(const int8_t *p) {
    LaneQ<C> q;
    if constexpr (C == 2) q.w[0] = *(const uint16_t *)p;
    else if constexpr (C == 4) q.w[0] = *(const uint32_t *)p;
    else { const uint2 v = *(const uint2 *)p; q.w[0] = v.x; q.w[1] = v.y; }
    return q;
}
template <int C> __device__ __forceinline__ void store_q(int8_t *p, const LaneQ<C> &q) {
    if constexpr (C == 2) *(uint16_t *)p = (uint16_t)q.w[0];
    else if constexpr (C == 4) *(uint32_t *)p = q.w[0];
    else *(uint2 *)p = make_uint2(q.w[0], q.w[1]);
}
template <int C> __device__ __forceinline__ int dot_q(const LaneQ<C> &a, const LaneQ<C> &b) {
    int s = 0;
#pragma unroll
    for (int i = 0; i < (C >= 4 ? C / 4 : 1); i++) s = __dp4a((int)a.w[i], (int)b.w[i], s);
    return s;
}
// byte j (< C) of the lane's state, sign-extended
template <int C> __device__ __forceinline__ int q_byte(const LaneQ<C> &q, int j) {
    return (int)(int8_t)(q.w[j >> 2] >> (8 * (j & 3)));
}

// ------------------------------------------------------------------------------------------------ per-warp slot

struct Slot {
    uint8_t *rec;      // the expert record (bulk copy destination)
    int16_t *trow;     // the table row (bulk copy destination)
    int8_t *qold;      // this layer's old state, for the transition's block reads
    int8_t *qb;        // the new state of the layer below, for the layer-input dots
    int8_t *zl;        // layer input codes [R2P]
    int8_t *zq;        // readout codes [R]
    uint32_t bar;      // mbarrier (shared address)
};

__device__ __forceinline__ Slot make_slot(uint8_t *base, uint32_t rec_max, int n) {
    Slot s;
    s.rec = base;
    s.trow = (int16_t *)(base + rec_max);
    s.qold = (int8_t *)(base + rec_max + 2 * n);
    s.qb = s.qold + n;
    s.zl = s.qb + n;
    s.zq = s.zl + 64;
    s.bar = smem_addr(s.zq + 32);
    return s;
}
// bytes of a slot: record, table row, qold, qb, zl, zq, mbarrier
__host__ __device__ constexpr uint32_t slot_bytes(uint32_t rec_max, int n) {
    return (rec_max + 2 * n + n + n + 64 + 32 + 8 + 127) / 128 * 128;
}

// Lane-interleaved part: the lane's 16-byte chunk j.
__device__ __forceinline__ uint4 lane_chunk(const uint8_t *part, int j, int lane) {
    return *(const uint4 *)(part + ((size_t)j * 32 + lane) * 16);
}

// ------------------------------------------------------------------------------------------------ one layer

// rho = 1 / sqrt(f32(sum q^2) * (1/n) + eps), or with group scales the sequential f32 sum over groups of 16 of
// r2[g] * f32(S_g) (cpu/ygg.cpp:248-266).
template <int N>
__device__ __forceinline__ float rms_rho(const LaneQ<N / 32> &qb, const float *r2b, float eps, int lane) {
    constexpr int C = N / 32;
    const float inv_n = 1.0f / (float)N;
    int part = dot_q<C>(qb, qb);
    if (r2b == nullptr) {
        const int S = __reduce_add_sync(kFull, part);
        return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(i2f(S), inv_n), eps)));
    }
    constexpr int kLanesPerGroup = 16 / C;
#pragma unroll
    for (int off = 1; off < kLanesPerGroup; off <<= 1) part += __shfl_xor_sync(kFull, part, off);
    float s = 0.0f;
#pragma unroll
    for (int g = 0; g < N / 16; g++) {
        const int sg = __shfl_sync(kFull, part, g * kLanesPerGroup);
        s = __fadd_rn(s, __fmul_rn(__ldg(r2b + g), i2f(sg)));
    }
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, inv_n), eps)));
}

// Heap-order descent from node 1: right iff f32(w_ix . qb) * rho > thr[x][ix] (cpu/ygg.cpp:271-280).
template <int N>
__device__ __forceinline__ int route(const int8_t *__restrict__ w, const float *__restrict__ thr_x, int depth,
                                     const LaneQ<N / 32> &qb, float rho, int lane) {
    constexpr int C = N / 32;
    int ix = 1;
    for (int d = 0; d < depth; d++) {
        LaneQ<C> wr;
        const int8_t *row = w + (size_t)ix * N + C * lane;
        if constexpr (C == 2) wr.w[0] = __ldg((const unsigned short *)row);
        else if constexpr (C == 4) wr.w[0] = __ldg((const unsigned int *)row);
        else { const uint2 v = __ldg((const uint2 *)row); wr.w[0] = v.x; wr.w[1] = v.y; }
        const float t = __ldg(thr_x + ix);
        const int dot = __reduce_add_sync(kFull, dot_q<C>(wr, qb));
        ix = 2 * ix + (__fmul_rn(i2f(dot), rho) > t ? 1 : 0);
    }
    return ix;
}

struct StepOut {
    float *logits;      // [V] of this stream, or null
    int32_t *routes;    // [L] or null
    int32_t *acc;       // [L][n] or null
};

// One token of one stream through every layer. q_in / q_out: the stream's state [L][n] (global or shared memory;
// they may alias). lg: the logits of the lane's classes (out). Returns false if a bounded wait gave up.
template <int N, int BLK, int R>
__device__ __forceinline__ bool token_step(const DevModel *__restrict__ mp, const Slot &sl, uint32_t &phase, int x,
                                           const int8_t *q_in, int8_t *q_out, float (&lg)[kMaxClassesPerLane],
                                           const StepOut &dbg, int lane) {
    constexpr int C = N / 32;
    const int L = mp->L, VP = mp->VP, E = mp->E, D = mp->D, V = mp->V;
    const int nv = VP / 32;
#pragma unroll
    for (int m = 0; m < kMaxClassesPerLane; m++) lg[m] = m < nv ? __ldg(mp->head_b + 32 * m + lane) : 0.0f;

    LaneQ<C> qbelow{};
    for (int l = 0; l < L; l++) {
        const DevLayer &y = mp->layer[l];
        const LaneQ<C> qold = load_q<C>(q_in + (size_t)l * N + C * lane);
        int r = x;
        float rho = 0.0f;
        if (l > 0) {
            rho = rms_rho<N>(qbelow, y.r2b, y.rms_eps, lane);
            r = route<N>(y.w, y.thr + (size_t)x * E, D, qbelow, rho, lane) - E;
        }
        // -- the expert record and its table row into the slot (previous readers of the slot are done)
        const uint32_t rec_bytes = y.rec_bytes;
        const bool has_table = y.table != nullptr;
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async();
            mbar_expect_tx(sl.bar, rec_bytes + (has_table ? 2u * N : 0u));
            bulk_g2s(smem_addr(sl.rec), y.rec + (size_t)r * rec_bytes, rec_bytes, sl.bar);
            if (has_table) {
                const int16_t *trow = y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N;
                bulk_g2s(smem_addr(sl.trow), trow, 2u * N, sl.bar);
            }
        }
        // -- layer input codes while the copy is in flight (cpu/ygg.cpp:285-296)
        const bool low = l > 0 && mp->R2 > 0;
        if (low) {
            store_q<C>(sl.qb + C * lane, qbelow);
            __syncwarp();
            const int R2P = mp->R2P;
            for (int k = lane; k < R2P; k += 32) {
                int a = 0;
#pragma unroll 4
                for (int j = 0; j < N / 16; j++) {
                    const uint4 v = __ldg((const uint4 *)(y.vl + ((size_t)j * R2P + k) * 16));
                    const uint4 q = *(const uint4 *)(sl.qb + 16 * j);
                    a = __dp4a((int)v.x, (int)q.x, a);
                    a = __dp4a((int)v.y, (int)q.y, a);
                    a = __dp4a((int)v.z, (int)q.z, a);
                    a = __dp4a((int)v.w, (int)q.w, a);
                }
                const float zf = __fmul_rn(__fmul_rn(i2f(a), __ldg(y.mv + k)), rho);
                sl.zl[k] = (int8_t)(k < mp->R2 ? clampi(cvt_rne(zf), -127, 127) : 0);
            }
        }
        store_q<C>(sl.qold + C * lane, qold);
        __syncwarp();
        const bool ok = __all_sync(kFull, mbar_wait_bounded(sl.bar, phase));
        phase ^= 1u;
        if (!ok) return false;

        // -- transition: acc_i = (sum_j A16[i][j] q[j] + 2^(shift-1)) >> shift over the row's block (cpu/ygg.cpp:312-332)
        int acc[C];
        {
            const int blk0 = ((C * lane) / BLK) * BLK;
            uint32_t qblk[BLK / 4];
            if constexpr (BLK == 8) {
                const uint2 v = *(const uint2 *)(sl.qold + blk0);
                qblk[0] = v.x; qblk[1] = v.y;
            } else {
                const uint4 v = *(const uint4 *)(sl.qold + blk0);
                qblk[0] = v.x; qblk[1] = v.y; qblk[2] = v.z; qblk[3] = v.w;
            }
            constexpr int kWords = C * BLK / 2;            // int16 pairs of the lane
            uint32_t aw[kWords];
            const uint8_t *pa = sl.rec + y.off_a;
#pragma unroll
            for (int j = 0; j < kWords / 4; j++) {
                const uint4 v = lane_chunk(pa, j, lane);
                aw[4 * j] = v.x; aw[4 * j + 1] = v.y; aw[4 * j + 2] = v.z; aw[4 * j + 3] = v.w;
            }
            const int rnd = 1 << (mp->shift - 1), sh = mp->shift;
#pragma unroll
            for (int ii = 0; ii < C; ii++) {
                int s = 0;
#pragma unroll
                for (int p = 0; p < BLK / 2; p++) {
                    const uint32_t a = aw[ii * (BLK / 2) + p];
                    s = (p & 1) ? __dp2a_hi((int)a, (int)qblk[p >> 1], s) : __dp2a_lo((int)a, (int)qblk[p >> 1], s);
                }
                acc[ii] = (s + rnd) >> sh;
            }
        }
        // -- input: table row (cpu/ygg.cpp:334-337) or factored (cpu/ygg.cpp:339-358)
        if (has_table) {
#pragma unroll
            for (int ii = 0; ii < C; ii++) acc[ii] += sl.trow[C * lane + ii];
        } else {
            const int KP = mp->KP;
            const uint8_t *pf = sl.rec + y.off_f;
            const int8_t *v = y.vt + (size_t)x * KP;
            const float su = *(const float *)(sl.rec + y.off_su);
            const int16_t *cb = (const int16_t *)(sl.rec + y.off_cb);
#pragma unroll
            for (int ii = 0; ii < C; ii++) {
                int lt = 0;
                for (int j = 0; j < KP / 16; j++) {
                    const uint4 u = lane_chunk(pf, ii * (KP / 16) + j, lane);
                    const uint4 t = __ldg((const uint4 *)(v + 16 * j));
                    lt = __dp4a((int)u.x, (int)t.x, lt);
                    lt = __dp4a((int)u.y, (int)t.y, lt);
                    lt = __dp4a((int)u.z, (int)t.z, lt);
                    lt = __dp4a((int)u.w, (int)t.w, lt);
                }
                const float mul = __fmul_rn(su, __ldg(y.mt + C * lane + ii));
                acc[ii] += cvt_rne(__fmul_rn(i2f(lt), mul)) + cb[C * lane + ii];
            }
        }
        // -- layer input: acc_i += rint(f32(U'_r zl) m_ul) (cpu/ygg.cpp:360-377)
        if (low) {
            const int R2P = mp->R2P;
            const uint8_t *pu = sl.rec + y.off_u;
#pragma unroll
            for (int ii = 0; ii < C; ii++) {
                int la = 0;
                for (int j = 0; j < R2P / 16; j++) {
                    const uint4 u = lane_chunk(pu, ii * (R2P / 16) + j, lane);
                    const uint4 z = *(const uint4 *)(sl.zl + 16 * j);
                    la = __dp4a((int)u.x, (int)z.x, la);
                    la = __dp4a((int)u.y, (int)z.y, la);
                    la = __dp4a((int)u.z, (int)z.z, la);
                    la = __dp4a((int)u.w, (int)z.w, la);
                }
                const float mu = y.mulv ? __ldg(y.mulv + C * lane + ii) : y.layer_input_scale;
                acc[ii] += cvt_rne(__fmul_rn(i2f(la), mu));
            }
        }
        // -- saturate to the new int8 state (cpu/ygg.cpp:388)
        LaneQ<C> qn{};
#pragma unroll
        for (int ii = 0; ii < C; ii++) {
            const uint32_t b = (uint32_t)(uint8_t)(int8_t)clampi(acc[ii], -128, 127);
            qn.w[ii >> 2] |= b << (8 * (ii & 3));
        }
        store_q<C>(q_out + (size_t)l * N + C * lane, qn);
        if (dbg.routes != nullptr && lane == 0) dbg.routes[l] = r;
        if (dbg.acc != nullptr) {
#pragma unroll
            for (int ii = 0; ii < C; ii++) dbg.acc[(size_t)l * N + C * lane + ii] = acc[ii];
        }

        // -- readout z = P_r q, zq = sat(rint(f32(z) m_z)) (cpu/ygg.cpp:395-420)
        int myz = 0;
        {
            const uint8_t *pp = sl.rec + y.off_p;
            constexpr int kPWords = R * C / 4;
            uint32_t pw[kPWords];
#pragma unroll
            for (int j = 0; j < kPWords / 4; j++) {
                const uint4 v = lane_chunk(pp, j, lane);
                pw[4 * j] = v.x; pw[4 * j + 1] = v.y; pw[4 * j + 2] = v.z; pw[4 * j + 3] = v.w;
            }
#pragma unroll
            for (int rr = 0; rr < R; rr++) {
                int part;
                if constexpr (C == 2) {
                    const uint32_t word = pw[rr >> 1];
                    part = __dp4a((int)((rr & 1) ? (word >> 16) : (word & 0xFFFFu)), (int)qn.w[0], 0);
                } else {
                    part = 0;
#pragma unroll
                    for (int w = 0; w < C / 4; w++) part = __dp4a((int)pw[rr * (C / 4) + w], (int)qn.w[w], part);
                }
                const int z = __reduce_add_sync(kFull, part);
                if (lane == rr) myz = z;
            }
        }
        if (lane < R) {
            const float mz = mp->has_mz && y.off_mz != kNone ? *(const float *)(sl.rec + y.off_mz + 4 * lane)
                                                             : y.readout_scale;
            sl.zq[lane] = (int8_t)clampi(cvt_rne(__fmul_rn(i2f(myz), mz)), -127, 127);
        }
        __syncwarp();
        // -- head: lg[c] += f32(Q_c . zq) * s (cpu/ygg.cpp:421-434)
        {
            uint32_t zw[R / 4];
#pragma unroll
            for (int j = 0; j < R / 4; j++) zw[j] = *(const uint32_t *)(sl.zq + 4 * j);
#pragma unroll
            for (int m = 0; m < kMaxClassesPerLane; m++) {
                if (m < nv) {
                    const int c = 32 * m + lane;
                    const int8_t *qrow = y.unembed + (size_t)c * R;
                    int a = 0;
#pragma unroll
                    for (int j = 0; j < R / 16 + (R % 16 ? 1 : 0); j++) {
                        if constexpr (R == 8) {
                            const uint2 v = __ldg((const uint2 *)qrow);
                            a = __dp4a((int)v.x, (int)zw[0], a);
                            a = __dp4a((int)v.y, (int)zw[1], a);
                        } else {
                            const uint4 v = __ldg((const uint4 *)(qrow + 16 * j));
                            a = __dp4a((int)v.x, (int)zw[4 * j], a);
                            a = __dp4a((int)v.y, (int)zw[4 * j + 1], a);
                            a = __dp4a((int)v.z, (int)zw[4 * j + 2], a);
                            a = __dp4a((int)v.w, (int)zw[4 * j + 3], a);
                        }
                    }
                    const float s = y.sqv ? __ldg(y.sqv + c) : y.unembed_scale;
                    lg[m] = __fadd_rn(lg[m], __fmul_rn(i2f(a), s));
                }
            }
        }
        qbelow = qn;
    }
    if (dbg.logits != nullptr) {
#pragma unroll
        for (int m = 0; m < kMaxClassesPerLane; m++) {
            const int c = 32 * m + lane;
            if (m < nv && c < V) dbg.logits[c] = lg[m];
        }
    }
    return true;
}

// ------------------------------------------------------------------------------------------------ kernels

__device__ __forceinline__ void slot_init(const Slot &sl, int lane) {
    if (lane == 0) {
        mbar_init(sl.bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
}

template <int N, int BLK, int R>
__global__ void __launch_bounds__(256) step_kernel(const DevModel *__restrict__ mp, int B,
                                                   const int32_t *__restrict__ tokens, const int8_t *state_in,
                                                   int8_t *state_out, float *__restrict__ logits,
                                                   int32_t *__restrict__ routes, int32_t *__restrict__ acc_out,
                                                   uint32_t rec_max) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const Slot sl = make_slot(smem + (size_t)warp * slot_bytes(rec_max, N), rec_max, N);
    slot_init(sl, lane);
    uint32_t phase = 0;
    const int L = mp->L, V = mp->V;
    for (int s = blockIdx.x * W + warp; s < B; s += gridDim.x * W) {
        const int x = tokens[s];
        if (x < 0 || x >= V) {   // cpu/ygg.cpp:493-495 rejects the whole input; here the stream is skipped
            if (lane == 0) atomicOr(mp->status, kStatusBadToken);
            if (logits != nullptr)
                for (int c = lane; c < V; c += 32) logits[(size_t)s * V + c] = __int_as_float(0x7fc00000);
            if (state_out != state_in)
                for (int i = lane; i < L * N; i += 32) state_out[(size_t)s * L * N + i] = state_in[(size_t)s * L * N + i];
            if (routes != nullptr && lane < L) routes[(size_t)s * L + lane] = -1;
            continue;
        }
        float lg[kMaxClassesPerLane];
        StepOut o{logits ? logits + (size_t)s * V : nullptr, routes ? routes + (size_t)s * L : nullptr,
                  acc_out ? acc_out + (size_t)s * L * N : nullptr};
        if (!token_step<N, BLK, R>(mp, sl, phase, x, state_in + (size_t)s * L * N, state_out + (size_t)s * L * N,
                                   lg, o, lane)) {
            if (lane == 0) atomicOr(mp->status, kStatusTimeout);
            return;
        }
    }
}

// Rows of `steps` tokens; the state of a row lives in the warp's shared memory between tokens, the logits in
// registers, and the f64 NLL of the next token is summed on chip (cpu/ygg.cpp:513-517).
template <int N, int BLK, int R>
__global__ void __launch_bounds__(256) score_kernel(const DevModel *__restrict__ mp, int B, int T,
                                                    const int32_t *__restrict__ tokens, int8_t *state,
                                                    double *__restrict__ bits, uint32_t rec_max) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int L = mp->L, V = mp->V, nv = mp->VP / 32;
    const uint32_t sb = slot_bytes(rec_max, N) + (uint32_t)((L * N + 127) / 128 * 128);
    uint8_t *base = smem + (size_t)warp * sb;
    const Slot sl = make_slot(base, rec_max, N);
    int8_t *qs = (int8_t *)(base + slot_bytes(rec_max, N));
    slot_init(sl, lane);
    uint32_t phase = 0;
    const StepOut none{nullptr, nullptr, nullptr};
    for (int s = blockIdx.x * W + warp; s < B; s += gridDim.x * W) {
        const int32_t *tok = tokens + (size_t)s * T;
        bool bad = false;
        for (int t = lane; t < T; t += 32) bad |= tok[t] < 0 || tok[t] >= V;
        if (__any_sync(kFull, bad)) {
            if (lane == 0) { atomicOr(mp->status, kStatusBadToken); bits[s] = __longlong_as_double(0x7ff8000000000000LL); }
            continue;
        }
        for (int i = lane; i < L * N; i += 32) qs[i] = state ? state[(size_t)s * L * N + i] : 0;
        __syncwarp();
        double nll = 0.0;
        for (int t = 0; t + 1 < T; t++) {
            float lg[kMaxClassesPerLane];
            if (!token_step<N, BLK, R>(mp, sl, phase, tok[t], qs, qs, lg, none, lane)) {
                if (lane == 0) atomicOr(mp->status, kStatusTimeout);
                return;
            }
            // -log p(next) in f64: max, sum of exp over the V classes, the target's logit
            float mx = -__int_as_float(0x7f800000);
#pragma unroll
            for (int m = 0; m < kMaxClassesPerLane; m++)
                if (m < nv && 32 * m + lane < V) mx = fmaxf(mx, lg[m]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
            double se = 0.0;
#pragma unroll
            for (int m = 0; m < kMaxClassesPerLane; m++)
                if (m < nv && 32 * m + lane < V) se += exp((double)lg[m] - (double)mx);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) se += __shfl_xor_sync(kFull, se, off);
            const int y = tok[t + 1];
            float ly = 0.0f;
#pragma unroll
            for (int m = 0; m < kMaxClassesPerLane; m++)
                if (m == (y >> 5)) ly = lg[m];
            ly = __shfl_sync(kFull, ly, y & 31);
            nll += log(se) + (double)mx - (double)ly;
        }
        if (lane == 0) bits[s] = nll / 0.69314718055994530942;
        __syncwarp();
        if (state)
            for (int i = lane; i < L * N; i += 32) state[(size_t)s * L * N + i] = qs[i];
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------------------ launchers

struct LaunchShape {
    int grid, block;
    size_t smem;
};

template <int N, int BLK, int R>
static cudaError_t launch_step_t(const DevModel *dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                                 float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps, int grid_cap,
                                 cudaStream_t st) {
    const size_t smem = (size_t)warps * slot_bytes(rec_max, N);
    cudaError_t e = cudaFuncSetAttribute(step_kernel<N, BLK, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int grid = (B + warps - 1) / warps;
    if (grid > grid_cap) grid = grid_cap;
    step_kernel<N, BLK, R><<<grid, 32 * warps, smem, st>>>(dm, B, tok, sin, sout, lg, routes, acc, rec_max);
    return cudaGetLastError();
}

template <int N, int BLK, int R>
static cudaError_t launch_score_t(const DevModel *dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                                  uint32_t rec_max, int L, int warps, int grid_cap, cudaStream_t st) {
    const size_t per = slot_bytes(rec_max, N) + (size_t)((L * N + 127) / 128 * 128);
    const size_t smem = (size_t)warps * per;
    cudaError_t e = cudaFuncSetAttribute(score_kernel<N, BLK, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int grid = (B + warps - 1) / warps;
    if (grid > grid_cap) grid = grid_cap;
    score_kernel<N, BLK, R><<<grid, 32 * warps, smem, st>>>(dm, B, T, tok, state, bits, rec_max);
    return cudaGetLastError();
}

#define YGG_DISPATCH(FN, ...)                                                                    \
    switch (n * 1000 + blk * 100 + r) {                                                          \
        case 64 * 1000 + 8 * 100 + 8: return FN<64, 8, 8>(__VA_ARGS__);                         \
        case 64 * 1000 + 8 * 100 + 16: return FN<64, 8, 16>(__VA_ARGS__);                        \
        case 64 * 1000 + 8 * 100 + 32: return FN<64, 8, 32>(__VA_ARGS__);                        \
        case 64 * 1000 + 16 * 100 + 8: return FN<64, 16, 8>(__VA_ARGS__);                        \
        case 64 * 1000 + 16 * 100 + 16: return FN<64, 16, 16>(__VA_ARGS__);                      \
        case 64 * 1000 + 16 * 100 + 32: return FN<64, 16, 32>(__VA_ARGS__);                      \
        case 128 * 1000 + 8 * 100 + 8: return FN<128, 8, 8>(__VA_ARGS__);                        \
        case 128 * 1000 + 8 * 100 + 16: return FN<128, 8, 16>(__VA_ARGS__);                      \
        case 128 * 1000 + 8 * 100 + 32: return FN<128, 8, 32>(__VA_ARGS__);                      \
        case 128 * 1000 + 16 * 100 + 8: return FN<128, 16, 8>(__VA_ARGS__);                      \
        case 128 * 1000 + 16 * 100 + 16: return FN<128, 16, 16>(__VA_ARGS__);                    \
        case 128 * 1000 + 16 * 100 + 32: return FN<128, 16, 32>(__VA_ARGS__);                    \
        case 256 * 1000 + 8 * 100 + 8: return FN<256, 8, 8>(__VA_ARGS__);                        \
        case 256 * 1000 + 8 * 100 + 16: return FN<256, 8, 16>(__VA_ARGS__);                      \
        case 256 * 1000 + 8 * 100 + 32: return FN<256, 8, 32>(__VA_ARGS__);                      \
        case 256 * 1000 + 16 * 100 + 8: return FN<256, 16, 8>(__VA_ARGS__);                      \
        case 256 * 1000 + 16 * 100 + 16: return FN<256, 16, 16>(__VA_ARGS__);                    \
        case 256 * 1000 + 16 * 100 + 32: return FN<256, 16, 32>(__VA_ARGS__);                    \
        default: return cudaErrorInvalidValue;                                                   \
    }

cudaError_t launch_step(int n, int blk, int r, const DevModel *dm, int B, const int32_t *tok, const int8_t *sin,
                        int8_t *sout, float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps,
                        int grid_cap, cudaStream_t st) {
    YGG_DISPATCH(launch_step_t, dm, B, tok, sin, sout, lg, routes, acc, rec_max, warps, grid_cap, st)
}

cudaError_t launch_score(int n, int blk, int r, const DevModel *dm, int B, int T, const int32_t *tok, int8_t *state,
                         double *bits, uint32_t rec_max, int L, int warps, int grid_cap, cudaStream_t st) {
    YGG_DISPATCH(launch_score_t, dm, B, T, tok, state, bits, rec_max, L, warps, grid_cap, st)
}

size_t step_slot_bytes(uint32_t rec_max, int n) { return slot_bytes(rec_max, n); }

}  // namespace ygg
