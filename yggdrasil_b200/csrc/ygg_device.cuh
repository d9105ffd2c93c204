// Device code shared by the fused step/score kernels (ygg_step.cu) and the grouped scoring path (ygg_grouped.cu):
// PTX helpers (mbarrier, bulk copy), the reference's f32 -> int32 conversion, the lane-owned state words, rho, the
// router descent, and the per-stream expert update, readout and head of one layer.
//
// G is the number of lanes that serve one stream: 32 (a warp per stream) or 16 (two streams per warp, one per half;
// the model's layout interleaves its records over 16 lanes then). Lane l of a warp belongs to stream group l / G and
// is lane gl = l % G of it; it owns the C = n / G state coordinates [C gl, C gl + C). Warp collectives always name
// the full warp: a reduction within a group is a butterfly of xor shuffles that never crosses the group, and a
// ballot's bits are sliced per group.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ygg_model.h"

namespace ygg {

constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr long long kWaitCycles = 2000000000LL;
constexpr int kLook = 3;                // router levels per round of loads
constexpr int kLookRows = (1 << kLook) - 1;


// ------------------------------------------------------------------------------------------------ host side

// The dynamic shared-memory limit of a kernel, raised once per device to the largest size asked for so far (the
// attribute is per device; raising it on every launch would cost a driver call per step). One SmemLimits per kernel.
constexpr int kMaxDevices = 64;
struct SmemLimits { size_t set[kMaxDevices]; };
static inline cudaError_t raise_smem_limit(const void *fn, size_t smem, SmemLimits &lim) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && lim.set[dev] >= smem) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) lim.set[dev] = smem;
    return e;
}

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
// try_wait suspends the thread until the phase completes or the hint (ns) runs out, so a waiting warp costs few
// issue slots
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast), completion counted on the mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-aligned) of global memory into L2; no completion to wait for.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16 bytes of an expert record: from shared memory (a staged slot), or straight from global memory (GL) through the
// non-coherent path without allocating in L1 (each record is read once per stream).
template <bool GL> __device__ __forceinline__ uint4 ld16(const void *p) {
    if constexpr (GL) {
        uint4 v;
        asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
            : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
            : "l"(p));
        return v;
    } else {
        return *(const uint4 *)p;
    }
}

// Bounded wait for the phase `parity` of an mbarrier: false after `limit` cycles (~1 s by default; the caller reports
// a timeout).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, long long limit = kWaitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > limit) return false;
    return true;
}

// f32 -> int32 rounded half to even; NaN and values outside int32 give INT_MIN, as x86 cvtps2dq (the reference's
// _mm512_cvtps_epi32), which the callers then clamp.
__device__ __forceinline__ int cvt_rne(float v) {
    return (v >= -2147483648.0f && v < 2147483648.0f) ? __float2int_rn(v) : (int)0x80000000;
}
__device__ __forceinline__ float i2f(int v) { return __int2float_rn(v); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }
__device__ __forceinline__ int dot16(const uint4 &a, const uint4 &b, int s) {
    s = __dp4a((int)a.x, (int)b.x, s);
    s = __dp4a((int)a.y, (int)b.y, s);
    s = __dp4a((int)a.z, (int)b.z, s);
    return __dp4a((int)a.w, (int)b.w, s);
}

// --------------------------------------------------------------------------------------------- lane state words

// Logits a lane holds: classes G m + gl for m < VP / G (VP <= 256).
template <int G> constexpr int kMaxClasses = 256 / G;

// The C state bytes of one lane as int32 words: C = 2 uses the low half of one word (high half zero).
template <int C> struct LaneQ { uint32_t w[C >= 4 ? C / 4 : 1]; };

template <int C> __device__ __forceinline__ LaneQ<C> load_q(const int8_t *p) {
    LaneQ<C> q;
    if constexpr (C == 2) q.w[0] = *(const uint16_t *)p;
    else if constexpr (C == 4) q.w[0] = *(const uint32_t *)p;
    else if constexpr (C == 8) { const uint2 v = *(const uint2 *)p; q.w[0] = v.x; q.w[1] = v.y; }
    else { const uint4 v = *(const uint4 *)p; q.w[0] = v.x; q.w[1] = v.y; q.w[2] = v.z; q.w[3] = v.w; }
    return q;
}
template <int C> __device__ __forceinline__ void store_q(int8_t *p, const LaneQ<C> &q) {
    if constexpr (C == 2) *(uint16_t *)p = (uint16_t)q.w[0];
    else if constexpr (C == 4) *(uint32_t *)p = q.w[0];
    else if constexpr (C == 8) *(uint2 *)p = make_uint2(q.w[0], q.w[1]);
    else *(uint4 *)p = make_uint4(q.w[0], q.w[1], q.w[2], q.w[3]);
}
// The same for a stream's state in global memory, read and written once per step: cache-streaming loads and stores
// (ld/st.global.cs, evict first), so that the states a step streams through L2 do not displace the leaf records that
// many streams share (c3: +4 % tokens/s; the logits stay plain stores, which measured 1 % faster on c4).
#ifndef YGG_STREAM_HINTS
#define YGG_STREAM_HINTS 1
#endif
template <int C> __device__ __forceinline__ LaneQ<C> load_q_stream(const int8_t *p) {
#if YGG_STREAM_HINTS
    LaneQ<C> q;
    if constexpr (C == 2) {
        unsigned short v;
        asm volatile("ld.global.cs.u16 %0, [%1];" : "=h"(v) : "l"(p));
        q.w[0] = v;
    } else if constexpr (C == 4) {
        asm volatile("ld.global.cs.u32 %0, [%1];" : "=r"(q.w[0]) : "l"(p));
    } else if constexpr (C == 8) {
        asm volatile("ld.global.cs.v2.u32 {%0, %1}, [%2];" : "=r"(q.w[0]), "=r"(q.w[1]) : "l"(p));
    } else {
        asm volatile("ld.global.cs.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(q.w[0]), "=r"(q.w[1]), "=r"(q.w[2]), "=r"(q.w[3]) : "l"(p));
    }
    return q;
#else
    return load_q<C>(p);
#endif
}
template <int C> __device__ __forceinline__ void store_q_stream(int8_t *p, const LaneQ<C> &q) {
#if YGG_STREAM_HINTS
    if constexpr (C == 2) {
        asm volatile("st.global.cs.u16 [%0], %1;" ::"l"(p), "h"((unsigned short)q.w[0]) : "memory");
    } else if constexpr (C == 4) {
        asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(q.w[0]) : "memory");
    } else if constexpr (C == 8) {
        asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(q.w[0]), "r"(q.w[1]) : "memory");
    } else {
        asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(q.w[0]), "r"(q.w[1]), "r"(q.w[2]),
                     "r"(q.w[3])
                     : "memory");
    }
#else
    store_q<C>(p, q);
#endif
}
template <int C> __device__ __forceinline__ int dot_q(const LaneQ<C> &a, const LaneQ<C> &b) {
    int s = 0;
#pragma unroll
    for (int i = 0; i < (C >= 4 ? C / 4 : 1); i++) s = __dp4a((int)a.w[i], (int)b.w[i], s);
    return s;
}

// Sum of v over the G lanes of the caller's stream group (every lane gets it).
template <int G> __device__ __forceinline__ int group_sum(int v) {
    if constexpr (G == 32) {
        return __reduce_add_sync(kFull, v);
    } else {
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
        return v;
    }
}

// ------------------------------------------------------------------------------------------------ one layer

// rho = 1 / sqrt(f32(sum q^2) * (1/n) + eps), or with group scales the sequential f32 sum over groups of 16 of
// r2[g] * f32(S_g) (cpu/ygg.cpp:248-266). inv_n = f32(1 / n) of the model's own n (the device layout may be padded:
// padded coordinates are 0 and padded groups have r2 = 0, so they add exactly nothing).
template <int N, int G>
__device__ __forceinline__ float rms_rho(const LaneQ<N / G> &qb, const float *r2b, float eps, float inv_n, int lane) {
    constexpr int C = N / G;
    int part = dot_q<C>(qb, qb);
    if (r2b == nullptr) {
        const int S = group_sum<G>(part);
        return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(i2f(S), inv_n), eps)));
    }
    constexpr int kLanesPerGroup = 16 / C;   // lanes per group of 16 coordinates
#pragma unroll
    for (int off = 1; off < kLanesPerGroup; off <<= 1) part += __shfl_xor_sync(kFull, part, off);
    const int base = lane & (32 - G);
    float s = 0.0f;
#pragma unroll
    for (int g = 0; g < N / 16; g++) {
        const int sg = __shfl_sync(kFull, part, base + g * kLanesPerGroup);
        s = __fadd_rn(s, __fmul_rn(__ldg(r2b + g), i2f(sg)));
    }
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, inv_n), eps)));
}

// Heap-order descent from node 1, right iff f32(w_ix . qb) * rho > thr[x][ix] (cpu/ygg.cpp:271-280), kLook levels
// per round of loads. Row k of a round's subtree (k = 0: ix; 1-2: 2ix + k-1; 3-6: 4ix + k-3, i.e. ix * 2^lvl(k) +
// k + 1 - 2^lvl(k)) is read by the LPR = n/16 lanes of row group k % RPI (RPI = G / LPR) in load k / RPI, 16 bytes
// each (qrow: the lane's 16 bytes of qb at 16 (gl % LPR)). The NI partial dots of a lane are then reduce-scattered
// over its row group: halving exchanges leave each lane the whole dot of one load i, then plain butterflies finish
// the sum; so each lane converts and compares one row, loads only that row's threshold, and one ballot per round
// carries every decision of both stream groups. DT > 0: the depth fixed at compile time (= depth), which unrolls the
// rounds with their row counts known. Returns the leaf node index in [E, 2E).
template <int N, int G, int DT = 0>
__device__ __forceinline__ int route_look(const int8_t *__restrict__ w, const float *__restrict__ thr_x, int depth,
                                          const uint4 &qrow, float rho, int lane) {
    constexpr int LPR = N / 16;                 // lanes per row
    constexpr int RPI = G / LPR;                // rows of one stream per warp-wide 16-byte load
    constexpr int NI = (kLookRows + RPI - 1) / RPI;
    constexpr int LS = LPR == 4 ? 2 : LPR == 8 ? 3 : 4;     // log2 LPR
    constexpr int LN = NI == 1 ? 0 : NI == 2 ? 1 : 2;       // log2 NI
    static_assert(G == 32 || N <= 128, "two streams per warp need rows of at most 8 lanes");
    static_assert((1 << LN) == NI && NI <= LPR, "NI a power of two within a row group");
    const int gl = lane & (G - 1);
    const int g = gl / LPR;
    const int8_t *wl = w + 16 * (gl % LPR);
    // the load whose whole dot this lane holds after the reduce-scatter, and that row's subtree index
    const int mine = (gl % LPR) >> (LS - LN);
    const int kmine = mine * RPI + g;
    const int lvm = kmine == 0 ? 0 : kmine < 3 ? 1 : 2;
    const int mulm = 1 << lvm, addm = kmine + 1 - mulm;
    // per-lane constants of the subtree rows this lane reads: row = ix * mul + add
    int mul[NI], add[NI], kk[NI];
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int k = i * RPI + g;
        const int lvl = k == 0 ? 0 : k < 3 ? 1 : 2;
        kk[i] = k;
        mul[i] = 1 << lvl;
        add[i] = k + 1 - (1 << lvl);
    }
    int ix = 1;
    // one round: the lv <= kLook levels under ix
    auto round = [&](const int lv) {
        const int nrows = (1 << lv) - 1;
        int dot[NI];
#pragma unroll
        for (int i = 0; i < NI; i++) {
            dot[i] = 0;
            if (kk[i] < nrows) {
                const uint4 v = __ldg((const uint4 *)(wl + (size_t)(ix * mul[i] + add[i]) * N));
                dot[i] = dot16(v, qrow, 0);
            }
        }
        const bool live = kmine < nrows;
        const float t = live ? __ldg(thr_x + ix * mulm + addm) : 0.0f;
        // reduce-scatter over the row group: offsets LPR/2, LPR/4, ... halve the values a lane keeps (the upper half
        // where the lane's offset bit is set), then the remaining offsets sum the last value
        int cnt = NI;
#pragma unroll
        for (int st = 0; st < LS; st++) {
            const int off = LPR >> (st + 1);
            if (st < LN) {
                const int half = cnt >> 1;
                const bool hi = (gl & off) != 0;
#pragma unroll
                for (int i = 0; i < NI / 2; i++) {
                    if (i < half) {
                        const int keep = hi ? dot[i + half] : dot[i], send = hi ? dot[i] : dot[i + half];
                        dot[i] = keep + __shfl_xor_sync(kFull, send, off);
                    }
                }
                cnt = half;
            } else {
                dot[0] += __shfl_xor_sync(kFull, dot[0], off);
            }
        }
        const bool right = live && __fmul_rn(i2f(dot[0]), rho) > t;
        uint32_t bits = __ballot_sync(kFull, right);
        if constexpr (G == 16) bits = (bits >> (lane & 16)) & 0xFFFFu;
        // row k's decision sits at lane (k % RPI) LPR + (k / RPI) 2^(LS - LN) of the group
        int k = 0;
#pragma unroll
        for (int j = 0; j < kLook; j++) {
            if (j < lv) {
                const int pos = (k % RPI) * LPR + ((k / RPI) << (LS - LN));
                const int b = (int)((bits >> pos) & 1u);
                ix = 2 * ix + b;
                k = 2 * k + 1 + b;
            }
        }
    };
    if constexpr (DT > 0) {
#pragma unroll
        for (int d = 0; d < DT; d += kLook) round(DT - d < kLook ? DT - d : kLook);
    } else {
        for (int d = 0; d < depth; d += kLook) round(min(kLook, depth - d));
    }
    return ix;
}

// Layer-input codes zl[k] = clamp(rint((f32(V'_k . qb) * mv[k]) * rho), +-127) for k < R2, 0 for the padding up to
// R2P (cpu/ygg.cpp:285-296). qb: the n new state bytes of the layer below (shared or global memory, 16-aligned);
// lane gl computes rows gl, gl + G, ...
template <int N, int R2T, int G>
__device__ __forceinline__ void layer_input_codes(const DevModel &m, const DevLayer &y, const int8_t *qb, float rho,
                                                  int8_t *zl, int lane) {
    const int R2P = R2T ? R2T : m.R2P;
#pragma unroll
    for (int k = lane & (G - 1); k < (R2T ? R2T : 64); k += G) {
        if (!R2T && k >= R2P) break;
        const int8_t *vk = y.vl + (size_t)k * 16;
        int a = 0;
#pragma unroll
        for (int j = 0; j < N / 16; j++)
            a = dot16(__ldg((const uint4 *)(vk + (size_t)j * R2P * 16)), *(const uint4 *)(qb + 16 * j), a);
        const float zf = __fmul_rn(__fmul_rn(i2f(a), __ldg(y.mv + k)), rho);
        zl[k] = (int8_t)(k < m.R2 ? clampi(cvt_rne(zf), -127, 127) : 0);
    }
}

// The expert update of one stream (cpu/ygg.cpp:312-389): acc = transition + input (table row or factored) + layer
// input, saturated into the new state words qn. rec: the expert record in the layout interleaved over G lanes (shared
// or global memory), trow: its table row (table storage), qold: the n old state bytes of this layer (16-aligned), zl:
// the layer-input codes (R2P bytes) when `low`.
template <int N, int BLK, int R2T, int G, bool GL = false>
__device__ __forceinline__ void leaf_update(const DevModel &m, const DevLayer &y, const uint8_t *rec,
                                            const int16_t *trow, int x, const int8_t *qold, const int8_t *zl,
                                            bool low, int lane, int (&acc)[N / G], LaneQ<N / G> &qn) {
    constexpr int C = N / G;
    constexpr int kChunk = 16 * G;                 // bytes between a lane's consecutive 16-byte chunks
    const int gl = lane & (G - 1);
    // -- transition: acc_i = (sum_j A16[i][j] q[j] + 2^(shift-1)) >> shift over the row's block (cpu/ygg.cpp:312-332);
    // the lane's C rows lie in one block
    {
        static_assert(C <= BLK, "a lane's rows must lie in one diagonal block");
        const int blk0 = ((C * gl) / BLK) * BLK;
        uint32_t qblk[BLK / 4];
        if constexpr (BLK == 8) {
            const uint2 v = *(const uint2 *)(qold + blk0);
            qblk[0] = v.x; qblk[1] = v.y;
        } else {
            const uint4 v = *(const uint4 *)(qold + blk0);
            qblk[0] = v.x; qblk[1] = v.y; qblk[2] = v.z; qblk[3] = v.w;
        }
        constexpr int kRowWords = BLK / 2;             // int16 pairs of one row
        const uint8_t *pa = rec + y.off_a + 16 * gl;
        const int rnd = 1 << (m.shift - 1), sh = m.shift;
        // G = 32 (C <= 4 rows): every word of the lane first, so that the loads overlap; G = 16 (8 rows): four rows'
        // words at a time (c4: +7 % tokens/s over row by row; c3 the same)
        constexpr int kPre = G == 32 ? C : (C >= 4 ? 4 : C);
        uint32_t aw[kPre * kRowWords];
#pragma unroll
        for (int ii0 = 0; ii0 < C; ii0 += kPre) {
#pragma unroll
            for (int j = 0; j < kPre * kRowWords / 4; j++) {
                const uint4 v = ld16<GL>(pa + kChunk * (ii0 * (kRowWords / 4) + j));
                aw[4 * j] = v.x; aw[4 * j + 1] = v.y; aw[4 * j + 2] = v.z; aw[4 * j + 3] = v.w;
            }
#pragma unroll
            for (int i1 = 0; i1 < kPre; i1++) {
                int s = 0;
#pragma unroll
                for (int p = 0; p < kRowWords; p++) {
                    const uint32_t a = aw[i1 * kRowWords + p];
                    s = (p & 1) ? __dp2a_hi((int)a, (int)qblk[p >> 1], s) : __dp2a_lo((int)a, (int)qblk[p >> 1], s);
                }
                acc[ii0 + i1] = (s + rnd) >> sh;
            }
        }
    }
    // -- input: table row (cpu/ygg.cpp:334-337) or factored (cpu/ygg.cpp:339-358)
    if (trow != nullptr) {
        const int16_t *tr = trow + C * gl;
        if constexpr (C == 8) {
            const uint4 v = ld16<GL>(tr);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int ii = 0; ii < 8; ii++) acc[ii] += (int)(int16_t)(u[ii >> 1] >> (16 * (ii & 1)));
        } else {
#pragma unroll
            for (int ii = 0; ii < C; ii++) acc[ii] += tr[ii];
        }
    } else {
        const int KP = m.KP;
        const uint8_t *pf = rec + y.off_f + 16 * gl;
        const int8_t *v = y.vt + (size_t)x * KP;
        const float su = *(const float *)(rec + y.off_su);
        const int16_t *cb = (const int16_t *)(rec + y.off_cb);
#pragma unroll
        for (int ii = 0; ii < C; ii++) {
            int lt = 0;
            for (int j = 0; j < KP / 16; j++)
                lt = dot16(ld16<GL>(pf + kChunk * (ii * (KP / 16) + j)), __ldg((const uint4 *)(v + 16 * j)), lt);
            const float mul = __fmul_rn(su, __ldg(y.mt + C * gl + ii));
            acc[ii] += cvt_rne(__fmul_rn(i2f(lt), mul)) + cb[C * gl + ii];
        }
    }
    // -- layer input: acc_i += rint(f32(U'_r zl) m_ul) (cpu/ygg.cpp:360-377)
    if (low) {
        const int R2P = R2T ? R2T : m.R2P;
        const uint8_t *pu = rec + y.off_u + 16 * gl;
        constexpr int kZw = R2T ? R2T / 16 : 4;
        uint4 z[kZw];
#pragma unroll
        for (int j = 0; j < kZw; j++)
            if (R2T || j < R2P / 16) z[j] = *(const uint4 *)(zl + 16 * j);
#pragma unroll
        for (int ii = 0; ii < C; ii++) {
            int la = 0;
#pragma unroll
            for (int j = 0; j < kZw; j++)
                if (R2T || j < R2P / 16) la = dot16(ld16<GL>(pu + kChunk * (ii * (R2P / 16) + j)), z[j], la);
            const float mu = y.mulv ? __ldg(y.mulv + C * gl + ii) : y.layer_input_scale;
            acc[ii] += cvt_rne(__fmul_rn(i2f(la), mu));
        }
    }
    // -- saturate to the new int8 state (cpu/ygg.cpp:388)
#pragma unroll
    for (int w = 0; w < (C >= 4 ? C / 4 : 1); w++) qn.w[w] = 0;
#pragma unroll
    for (int ii = 0; ii < C; ii++) {
        const uint32_t b = (uint32_t)(uint8_t)(int8_t)clampi(acc[ii], -128, 127);
        qn.w[ii >> 2] |= b << (8 * (ii & 3));
    }
}

// The readout partials of this lane, part[r] = P_r[r][C gl .. C gl + C) . q[C gl ..] over the lane's coordinates,
// and, for the lane that keeps row r (readout_code), the row's scale (group scales) or the tensor scale. rec: the
// record, read before the slot is handed back.
template <int N, int R, int G>
struct ReadoutPart {
    int part[R];
    float mz;
};
// The row a lane keeps after readout_code: gl for G = 32 and for G = 16 with R = 16; gl / 2 for G = 16 and R = 8
// (two lanes per row); none (-1) past the rows.
template <int R, int G> __device__ __forceinline__ int readout_row(int gl) {
    if constexpr (G == 16 && R == 8) return gl >> 1;
    else return gl < R ? gl : -1;
}
template <int N, int R, int G, bool GL = false>
__device__ __forceinline__ ReadoutPart<N, R, G> readout_partials(const DevLayer &y, const uint8_t *rec,
                                                                  const LaneQ<N / G> &qn, int lane) {
    constexpr int C = N / G;
    constexpr int kChunk = 16 * G;
    const int gl = lane & (G - 1);
    ReadoutPart<N, R, G> o;
    const uint8_t *pp = rec + y.off_p + 16 * gl;
    // lane words: word r * C/4 + w = P[r][C gl + 4w .. +3] (C >= 4); C = 2: word w = (P[2w][2gl..], P[2w+1][2gl..])
    constexpr int kWords = R * C / 4;
    uint32_t pw[kWords];
#pragma unroll
    for (int j = 0; j < kWords / 4; j++) {
        const uint4 v = ld16<GL>(pp + kChunk * j);
        pw[4 * j] = v.x; pw[4 * j + 1] = v.y; pw[4 * j + 2] = v.z; pw[4 * j + 3] = v.w;
    }
#pragma unroll
    for (int rr = 0; rr < R; rr++) {
        if constexpr (C == 2) {
            const uint32_t word = pw[rr >> 1];
            o.part[rr] = __dp4a((int)((rr & 1) ? (word >> 16) : (word & 0xFFFFu)), (int)qn.w[0], 0);
        } else {
            int part = 0;
#pragma unroll
            for (int w = 0; w < C / 4; w++) part = __dp4a((int)pw[rr * (C / 4) + w], (int)qn.w[w], part);
            o.part[rr] = part;
        }
    }
    o.mz = y.readout_scale;
    const int row = readout_row<R, G>(gl);
    if (y.off_mz != kNone && row >= 0) o.mz = *(const float *)(rec + y.off_mz + 4 * row);
    return o;
}

// zq of the readout z = P_r q (cpu/ygg.cpp:395-420): the partials of every row summed over the stream's G lanes; the
// lane that keeps row r (readout_row) returns zq[r] = clamp(rint(f32(z_r) mz), +-127), the other lanes 0. G = 32:
// one redux.sync per row. G = 16: a butterfly reduce-scatter over the half (xor 8, 4, 2, 1), which leaves each lane
// the whole sum of its own row with no select of the results.
template <int N, int R, int G>
__device__ __forceinline__ int readout_code(const ReadoutPart<N, R, G> &o, int lane) {
    const int gl = lane & (G - 1);
    int myz = 0;
    if constexpr (G == 32) {
#pragma unroll
        for (int rr = 0; rr < R; rr++) {
            const int z = __reduce_add_sync(kFull, o.part[rr]);
            if (gl == rr) myz = z;
        }
    } else {
        static_assert(R == 8 || R == 16, "two streams per warp: readout rank 8 or 16");
        int v[R];
#pragma unroll
        for (int i = 0; i < R; i++) v[i] = o.part[i];
        int cnt = R;
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            if (cnt > 1) {
                const int half = cnt / 2;
                const bool hi = (gl & off) != 0;        // this lane keeps the upper half of the rows
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    if (i < half) {
                        const int keep = hi ? v[i + half] : v[i], send = hi ? v[i] : v[i + half];
                        v[i] = keep + __shfl_xor_sync(kFull, send, off);
                    }
                }
                cnt = half;
            } else {
                v[0] += __shfl_xor_sync(kFull, v[0], off);
            }
        }
        myz = v[0];
    }
    return readout_row<R, G>(gl) >= 0 ? clampi(cvt_rne(__fmul_rn(i2f(myz), o.mz)), -127, 127) : 0;
}

// The head of one layer (cpu/ygg.cpp:421-434): lg[c] += f32(Q_c . zq) * s for the lane's classes G c + gl.
// zq: the R codes (shared or global memory, 4-aligned).
template <int R, int NVT, int G>
__device__ __forceinline__ void head_accumulate(const DevModel &m, const DevLayer &y, const int8_t *zq,
                                                float (&lg)[kMaxClasses<G>], int lane) {
    const int nv = NVT ? NVT : m.VP / G;
    const int gl = lane & (G - 1);
    uint32_t zw[R / 4];
#pragma unroll
    for (int j = 0; j < R / 4; j++) zw[j] = *(const uint32_t *)(zq + 4 * j);
#pragma unroll
    for (int c = 0; c < (NVT ? NVT : kMaxClasses<G>); c++) {
        if (NVT || c < nv) {
            const int cls = G * c + gl;
            const int8_t *qrow = y.unembed + (size_t)cls * R;
            int a = 0;
            if constexpr (R == 8) {
                const uint2 v = __ldg((const uint2 *)qrow);
                a = __dp4a((int)v.x, (int)zw[0], a);
                a = __dp4a((int)v.y, (int)zw[1], a);
            } else {
#pragma unroll
                for (int j = 0; j < R / 16; j++)
                    a = dot16(__ldg((const uint4 *)(qrow + 16 * j)),
                              make_uint4(zw[4 * j], zw[4 * j + 1], zw[4 * j + 2], zw[4 * j + 3]), a);
            }
            const float s = y.sqv ? __ldg(y.sqv + cls) : y.unembed_scale;
            lg[c] = __fadd_rn(lg[c], __fmul_rn(i2f(a), s));
        }
    }
}

// -log p(y) in f64 of the logits the stream's lanes hold (max, sum of exp over the V classes, the target's logit),
// summed the way cpu/ygg.cpp:513-517 defines it (the order of the exp sum differs: lanes, then a butterfly).
template <int G>
__device__ __forceinline__ double nll_of(const float (&lg)[kMaxClasses<G>], int nv, int V, int y, int lane) {
    constexpr int MC = kMaxClasses<G>;
    const int gl = lane & (G - 1);
    float mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int c = 0; c < MC; c++)
        if (c < nv && G * c + gl < V) mx = fmaxf(mx, lg[c]);
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
    double se = 0.0;
#pragma unroll
    for (int c = 0; c < MC; c++)
        if (c < nv && G * c + gl < V) se += exp((double)lg[c] - (double)mx);
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) se += __shfl_xor_sync(kFull, se, off);
    float ly = 0.0f;
#pragma unroll
    for (int c = 0; c < MC; c++)
        if (c == y / G) ly = lg[c];
    ly = __shfl_sync(kFull, ly, (lane & (32 - G)) + y % G);
    return log(se) + (double)mx - (double)ly;
}

}  // namespace ygg
